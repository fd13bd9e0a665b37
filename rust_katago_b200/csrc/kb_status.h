/* Status-word flags shared by device kernels and host code.
 *
 * The sticky status word is two uint32 values [flags, first_layer], the same
 * protocol the reference keeps for its MXFP8 path
 * (crates/kata_nn/src/backends/mxfp8.rs:22-30, cuda-kernels/mxfp8.cu:8-19):
 * flags are OR-ed together, first_layer keeps the first layer that reported
 * (0xffffffff = none).  This library uses the same word for INT8 and MXFP8.
 */
#ifndef KB_STATUS_H
#define KB_STATUS_H

#define KB_STATUS_NAN 1u               /* NaN input to a quantiser */
#define KB_STATUS_INF 2u               /* infinite input to a quantiser */
#define KB_STATUS_OUTPUT_NONFINITE 4u  /* a non-finite value reached an output */
#define KB_STATUS_WEIGHT_OVERFLOW 8u   /* an MXFP8 weight decodes to a non-finite value */
#define KB_STATUS_UNSUPPORTED_ARCH 16u /* kernel ran on a device other than sm_100 */
#define KB_STATUS_TIMEOUT 32u          /* a bounded device wait gave up (no hang, no trap) */

#define KB_NO_LAYER 0xffffffffu

#endif
