/* CPU oracle for the quantized trunk forward — TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, the smoke check of
 * __graft_entry__.py and bench.py's cpu_baseline / --impl reference legs load
 * it.  It restates, in plain C, the reference's CPU arithmetic for the W8A8
 * path (Rust_KataGo, crates/kata_nn), each function citing the lines it
 * follows.  Parity is pinned by the reference's own known answers and
 * closed-form test inputs (tests/test_oracle_golden.py).
 *
 * Build: gcc -O3 -fno-fast-math -ffp-contract=off -fopenmp -shared -fPIC
 * (see oracle/build.py).  -ffp-contract=off matters: every multiply-add below
 * is either two rounded operations or an explicit fmaf(), exactly as in the
 * GPU kernels, so both sides round identically.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ 16-bit codecs */

/* IEEE binary16 round-to-nearest-even, restated from the reference's
 * independent codec (crates/kata_nn/tests/test_mxfp8.rs:25-61). */
uint16_t or_f16_encode(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  int32_t exponent = (int32_t)((bits >> 23) & 255u);
  uint32_t mantissa = bits & 0x7fffffu;
  if (exponent == 255) return (uint16_t)(sign | 0x7c00u | (mantissa ? 0x200u : 0u));
  int32_t e = exponent - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return sign;
    mantissa |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t rounded = mantissa >> shift;
    uint32_t remainder = mantissa & ((1u << shift) - 1u);
    uint32_t midpoint = 1u << (shift - 1);
    if (remainder > midpoint || (remainder == midpoint && (rounded & 1u))) rounded += 1;
    return (uint16_t)(sign | rounded);
  }
  uint32_t rounded = mantissa >> 13;
  uint32_t remainder = mantissa & 0x1fffu;
  if (remainder > 0x1000u || (remainder == 0x1000u && (rounded & 1u))) {
    rounded += 1;
    if (rounded == 0x400u) {
      rounded = 0;
      e += 1;
      if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    }
  }
  return (uint16_t)(sign | ((uint32_t)e << 10) | rounded);
}

/* test_mxfp8.rs:8-23 */
float or_f16_decode(uint16_t bits) {
  uint32_t exponent = (bits >> 10) & 31u;
  uint32_t mantissa = bits & 1023u;
  double magnitude;
  if (exponent == 0) magnitude = (double)mantissa * ldexp(1.0, -24);
  else if (exponent == 31) magnitude = mantissa == 0 ? INFINITY : NAN;
  else magnitude = (double)(1024 + mantissa) * ldexp(1.0, (int)exponent - 25);
  float m = (float)magnitude;
  return (bits & 0x8000u) ? -m : m;
}

/* bfloat16 round-to-nearest-even (the upper 16 bits of binary32). */
uint16_t or_bf16_encode(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(((bits >> 16) & 0x8000u) | 0x7fc0u);
  uint32_t lsb = (bits >> 16) & 1u;
  bits += 0x7fffu + lsb;
  return (uint16_t)(bits >> 16);
}

float or_bf16_decode(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static float round16(float v, int f16) {
  return f16 ? or_f16_decode(or_f16_encode(v)) : or_bf16_decode(or_bf16_encode(v));
}

void or_encode16(const float* x, size_t n, int f16, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = f16 ? or_f16_encode(x[i]) : or_bf16_encode(x[i]);
}

void or_decode16(const uint16_t* x, size_t n, int f16, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = f16 ? or_f16_decode(x[i]) : or_bf16_decode(x[i]);
}

/* ------------------------------------------------------------------ elementwise math */

/* e^x for the SiLU denominator 1 + e^x (x = -g), the same operation sequence
 * as silu_exp in the kernels (rust_katago_b200/csrc/kb_numeric.cuh): x clamped
 * to [-20, 89] (which leaves 1 + e^x unchanged: below -17.4 it rounds to 1,
 * above ln(FLT_MAX) the arithmetic overflows as the true value does);
 * n = x*log2(e) rounded to the nearest integer by one fused multiply-add with
 * the shifter 1.5 * 2^23; Cody-Waite reduction with the Cephes ln2 split; the
 * degree-7 Taylor polynomial; the scaling (p * 2^(n-1)) * 2. */
float or_silu_exp(float x) {
  const float xc = fminf(fmaxf(x, -20.0f), 89.0f);
  const float k = fmaf(xc, 0x1.715476p+0f, 0x1.8p+23f);
  const float n = k - 0x1.8p+23f;
  float r = fmaf(-n, 0x1.63p-1f, xc);
  r = fmaf(n, 0x1.bd0106p-13f, r);
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const uint32_t bits = ((uint32_t)((int)n + 126)) << 23; /* 2^(n-1) */
  float s;
  memcpy(&s, &bits, 4);
  return (p * s) * 2.0f;
}

/* g / (1 + e^-g): the SiLU inside the reference's SwiGLU (int8_ops.cu:111-113). */
float or_silu(float g) { return g / (1.0f + or_silu_exp(-g)); }

/* GELU(x) = x * Phi(x): t = min(RN(x*x), 16), P = the degree-7 polynomial of
 * rust_katago_b200/gelu_fit.py in t (Horner, fused),
 * Phi = saturate(fma(x, P, 0.5)) to [0, 1] with NaN -> 0 (the PTX .sat rule);
 * the same operation sequence as kb_gelu in the kernels. */
float or_gelu(float x) {
  static const float c[8] = {0x1.985bf8p-2f, -0x1.0eb09cp-4f, 0x1.3b2a38p-7f, -0x1.0fadb6p-10f,
                             0x1.4b96f4p-14f, -0x1.0b18b6p-18f, 0x1.f68866p-24f, -0x1.9e1896p-30f};
  const float t = fminf(x * x, 16.0f);
  float p = c[7];
  for (int i = 6; i >= 0; --i) p = fmaf(p, t, c[i]);
  float phi = fmaf(x, p, 0.5f);
  if (!(phi > 0.0f)) phi = 0.0f; /* negative, zero or NaN */
  if (phi > 1.0f) phi = 1.0f;
  return x * phi;
}

void or_act(const float* x, size_t n, int act, float* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = act == 1 ? or_gelu(x[i]) : (act == 2 ? or_silu(x[i]) : x[i]);
}

/* ------------------------------------------------------------------ INT8 quantisation */

/* Per-output-channel weight quantisation: QuantizedWeights::new
 * (crates/kata_nn/src/backends/int8.rs:171-211). q is [n, kp], kp = ceil(k/16)*16. */
int or_int8_quantize_weights(const float* w, int n, int k, int8_t* q, float* scales) {
  if (n <= 0 || k <= 0 || k > 8192 || n % 4 != 0) return 1;
  for (size_t i = 0; i < (size_t)n * k; ++i)
    if (!isfinite(w[i])) return 2;
  const int kp = (k + 15) / 16 * 16;
  for (int r = 0; r < n; ++r) {
    const float* row = w + (size_t)r * k;
    float amax = 0.0f;
    for (int c = 0; c < k; ++c) amax = fmaxf(amax, fabsf(row[c]));
    float s = amax == 0.0f ? 1.0f : fmaxf(amax / 127.0f, FLT_MIN);
    scales[r] = s;
    for (int c = 0; c < kp; ++c) {
      float v = c < k ? rintf(row[c] / s) : 0.0f;
      v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
      q[(size_t)r * kp + c] = (int8_t)v;
    }
  }
  return 0;
}

/* Shared tail of every activation quantiser: scale = NaN for a row holding a
 * non-finite value, 1 for an all-zero row, amax/127 otherwise; q = clamp(rne(v/s))
 * (int8_ops.cu:36-46, :72-88; CPU form tests/int8_kernels.rs:277-283). */
static void quantize_values(const float* v, int width, int kp, int8_t* q, float* scale_out) {
  float amax = 0.0f;
  int bad = 0;
  for (int c = 0; c < width; ++c) {
    amax = fmaxf(amax, fabsf(v[c]));
    bad |= !isfinite(v[c]);
  }
  const float scale = bad ? NAN : (amax == 0.0f ? 1.0f : amax / 127.0f);
  *scale_out = scale;
  for (int c = 0; c < kp; ++c) {
    int qi = 0;
    if (c < width && !bad) {
      float r = rintf(v[c] / scale);
      r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
      qi = (int)r;
    }
    q[c] = (int8_t)qi;
  }
}

/* Row quantiser on already-decoded values (x[rows, stride] floats that were
 * 16-bit values): int8_quantize_rows_kernel (int8_ops.cu:62-89, :140-176). */
void or_int8_quantize_rows(const float* x, int rows, int width, int stride, int kp, int8_t* q,
                           float* scales) {
  for (int r = 0; r < rows; ++r)
    quantize_values(x + (size_t)r * stride, width, kp, q + (size_t)r * kp, scales + r);
}

/* Fused RMSNorm quantiser: int8_rms_quantize (int8_ops.cu:8-47) — one warp per
 * row, per-lane partial sums then the xor butterfly 16, 8, 4, 2, 1 — in the
 * product's lane assignment: lane l owns the 8-column groups l, l+32, ... and
 * accumulates fma(x, x, s) over them in order (the reference strides single
 * columns over lanes instead; the butterfly is identical).  rstd =
 * 1/sqrt(sum/W + eps) correctly rounded (the reference calls CUDA's rsqrtf).
 * The normalised value is (x*rstd)*gamma rounded to the 16-bit boundary. */
void or_int8_rms_quantize(const float* x, int rows, int width, int stride, const float* gamma,
                          float eps, int bound_f16, int kp, int8_t* q, float* scales,
                          float* normed /* nullable [rows, width] */) {
  float* v = (float*)malloc(sizeof(float) * (size_t)width);
  const int groups = (width + 7) / 8;
  for (int r = 0; r < rows; ++r) {
    const float* row = x + (size_t)r * stride;
    float lanes[32];
    for (int l = 0; l < 32; ++l) {
      float s = 0.0f;
      for (int g = l; g < groups; g += 32)
        for (int t = 0; t < 8; ++t) {
          const int c = 8 * g + t;
          const float xv = c < width ? row[c] : 0.0f;
          s = fmaf(xv, xv, s);
        }
      lanes[l] = s;
    }
    for (int step = 16; step; step >>= 1) {
      float next[32];
      for (int l = 0; l < 32; ++l) next[l] = lanes[l] + lanes[l ^ step];
      memcpy(lanes, next, sizeof(lanes));
    }
    const float rstd = 1.0f / sqrtf(lanes[0] / (float)width + eps);
    for (int c = 0; c < width; ++c) v[c] = round16((row[c] * rstd) * gamma[c], bound_f16);
    if (normed) memcpy(normed + (size_t)r * width, v, sizeof(float) * (size_t)width);
    quantize_values(v, width, kp, q + (size_t)r * kp, scales + r);
  }
  free(v);
}

/* ------------------------------------------------------------------ integer GEMM */

/* dots[m, n] = sum_k a[m, k] * w[n, k] in int32 (tests/int8_kernels.rs:287-291). */
void or_igemm(const int8_t* a, const int8_t* w, int m, int n, int kp, int32_t* dots, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static) if (threads != 1)
#endif
  for (int i = 0; i < m; ++i) {
    const int8_t* ar = a + (size_t)i * kp;
    for (int j = 0; j < n; ++j) {
      const int8_t* wr = w + (size_t)j * kp;
      int32_t s = 0;
      for (int k = 0; k < kp; ++k) s += (int32_t)ar[k] * (int32_t)wr[k];
      dots[(size_t)i * n + j] = s;
    }
  }
}

/* value = (f32(dot) * sa[row]) * sw[col] with two rounded multiplies
 * (int8_ops.cu:182; tests/int8_kernels.rs:296). */
void or_dequant(const int32_t* dots, const float* sa, const float* sw, int m, int n, float* out) {
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) out[(size_t)i * n + j] = ((float)dots[(size_t)i * n + j] * sa[i]) * sw[j];
}

/* value = fma(f32(dot) * sa[row], sw[col], bias[col]): the dequant with the
 * bias of the BASELINE topology's projections added by one fused multiply-add
 * (the product f32(dot)*sa is rounded, then t*sw + bias is rounded once),
 * the arithmetic of the GPU epilogue when a bias is given.  C99 fmaf is
 * correctly rounded. */
void or_dequant_bias(const int32_t* dots, const float* sa, const float* sw, const float* bias, int m, int n,
                     float* out) {
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j)
      out[(size_t)i * n + j] = fmaf((float)dots[(size_t)i * n + j] * sa[i], sw[j], bias[j]);
}

/* The reference's complete CPU W8A8 projection (tests/int8_kernels.rs:273-301):
 * quantise fp16 rows, integer dot, dequant, round to fp16.  Used as the timed
 * CPU baseline.  x16: [m, k] fp16 bits; wq: [n, kp]; out16: [m, n]. */
void or_w8a8_project_half(const uint16_t* x16, int m, int k, const int8_t* wq, const float* sw,
                          int n, int threads, uint16_t* out16) {
  const int kp = (k + 15) / 16 * 16;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel if (threads != 1)
#endif
  {
    float* v = (float*)malloc(sizeof(float) * (size_t)k);
    int8_t* q = (int8_t*)malloc((size_t)kp);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int i = 0; i < m; ++i) {
      for (int c = 0; c < k; ++c) v[c] = or_f16_decode(x16[(size_t)i * k + c]);
      float sa;
      quantize_values(v, k, kp, q, &sa);
      for (int j = 0; j < n; ++j) {
        const int8_t* wr = wq + (size_t)j * kp;
        int32_t s = 0;
        for (int c = 0; c < kp; ++c) s += (int32_t)q[c] * (int32_t)wr[c];
        out16[(size_t)i * n + j] = or_f16_encode(((float)s * sa) * sw[j]);
      }
    }
    free(v);
    free(q);
  }
}

/* Sets the OpenMP thread count for the oracle's parallel loops (the launcher
 * of a multi-process run may have set OMP_NUM_THREADS=1); returns the count
 * now in effect. */
int or_set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
  return omp_get_max_threads();
#else
  (void)threads;
  return 1;
#endif
}

int or_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ rotary tables */

/* Learned 2-D RoPE tables of one attention layer (native_model.rs:200-228):
 * angle = x * f[2p] + y * f[2p+1] in f32 (two rounded products, one rounded
 * sum), cos / sin by the C library's cosf / sinf, as the reference's f32::cos /
 * f32::sin call them.  freqs [heads, pairs, 2]; cos_t, sin_t [361, heads, pairs]. */
void or_rope_tables(const float* freqs, int heads, int pairs, float* cos_t, float* sin_t) {
  for (int y = 0; y < 19; ++y)
    for (int x = 0; x < 19; ++x)
      for (int h = 0; h < heads; ++h)
        for (int p = 0; p < pairs; ++p) {
          const int f = (h * pairs + p) * 2;
          const float a = (float)x * freqs[f];
          const float b = (float)y * freqs[f + 1];
          const float angle = a + b;
          const size_t i = ((size_t)(y * 19 + x) * heads + h) * pairs + p;
          cos_t[i] = cosf(angle);
          sin_t[i] = sinf(angle);
        }
}

/* ------------------------------------------------------------------ tensor-core accumulation */

/* The fp32 accumulation of tcgen05.mma kind::f16 (bf16 or f16 operands) on
 * sm_100, restated from measurements of this library's GEMM on a B200 (every
 * output of random and crafted shapes reproduced, K from 16 to 768): each
 * instruction adds a block of 16 products to the fp32 accumulator as
 *   e   = max over the block's nonzero products of (exp(a) + exp(b)) and of
 *         exp(acc) (unbiased exponents of the operands, not of the product;
 *         a subnormal operand counts with the minimum exponent),
 *   t_i = each product and the accumulator truncated toward zero to a multiple
 *         of 2^(e - 25),
 *   acc = the exact sum of the t_i rounded toward zero to fp32.
 * A K that is not a multiple of 16 is zero padded (zero products do not count
 * towards e).  The first block starts from an empty accumulator. */

/* v = sig * 2^(e - (mbits - 1)) with sig an integer (mbits = 11 for binary16,
 * 8 for bfloat16) and e the exponent the tensor core aligns by: the unbiased
 * exponent of a normal value, the minimum exponent (-14 binary16, -126
 * bfloat16) for a subnormal one (its exponent field's value, as measured);
 * returns 0 if v == 0. */
static int split16(float v, int f16, int64_t* sig, int* e) {
  if (v == 0.0f) {
    *sig = 0;
    *e = -100000;
    return 0;
  }
  const int mbits = f16 ? 11 : 8, emin = f16 ? -14 : -126;
  int ex;
  const double fr = frexp((double)v, &ex); /* v = fr * 2^ex, 0.5 <= |fr| < 1 */
  if (ex - 1 < emin) {
    *e = emin;
    *sig = (int64_t)ldexp((double)v, (mbits - 1) - emin); /* exact: v lies on the subnormal grid */
  } else {
    *e = ex - 1;
    *sig = (int64_t)ldexp(fr, mbits);
  }
  return 1;
}

/* One K=16 block: acc (fp32) plus sum_i a[i]*b[i] with the truncation above. */
static float tc_block16(float acc, const float* a, const float* b, int f16) {
  int64_t sa[16], sb[16];
  int ea[16], eb[16], nz[16];
  int emax = -100000;
  for (int i = 0; i < 16; ++i) {
    nz[i] = split16(a[i], f16, &sa[i], &ea[i]) & split16(b[i], f16, &sb[i], &eb[i]);
    if (nz[i] && ea[i] + eb[i] > emax) emax = ea[i] + eb[i];
  }
  int eacc = -100000;
  int64_t sacc = 0;
  if (acc != 0.0f) {
    int ex;
    const double fr = frexp((double)acc, &ex);
    sacc = (int64_t)ldexp(fr, 24); /* 24-bit significand: acc = sacc * 2^(ex - 24) */
    eacc = ex - 1;
    if (eacc > emax) emax = eacc;
  }
  if (emax == -100000) return 0.0f;
  const int unit = emax - 25; /* every term truncated to a multiple of 2^unit */
  const int mbits = f16 ? 11 : 8;
  int64_t total = 0;
  for (int i = 0; i < 16; ++i) {
    if (!nz[i]) continue;
    /* product = sa*sb * 2^(ea - (mbits-1) + eb - (mbits-1)) */
    const int64_t pm = sa[i] * sb[i];
    const int pe = ea[i] + eb[i] - 2 * (mbits - 1);
    const int sh = pe - unit;
    int64_t mag = pm < 0 ? -pm : pm;
    if (sh >= 0) mag <<= sh;
    else mag = sh <= -62 ? 0 : mag >> (-sh);
    total += pm < 0 ? -mag : mag;
  }
  if (sacc != 0) {
    const int sh = (eacc - 23) - unit;
    int64_t mag = sacc < 0 ? -sacc : sacc;
    if (sh >= 0) mag <<= sh;
    else mag = sh <= -62 ? 0 : mag >> (-sh);
    total += sacc < 0 ? -mag : mag;
  }
  if (total == 0) return 0.0f;
  /* round toward zero to 24 significant bits */
  uint64_t mag = (uint64_t)(total < 0 ? -total : total);
  int len = 0;
  while ((mag >> len) != 0) ++len;
  int ex = unit;
  if (len > 24) {
    mag >>= (len - 24);
    ex += len - 24;
  }
  float r = (float)ldexp((double)mag, ex);
  return total < 0 ? -r : r;
}

/* dot(a, b) over k (padded to a multiple of 16) as one tensor-core accumulator. */
static float tc_dot(const float* a, const float* b, int k, int f16) {
  float acc = 0.0f;
  float ab[16], bb[16];
  for (int k0 = 0; k0 < k; k0 += 16) {
    const int w = k - k0 < 16 ? k - k0 : 16;
    for (int i = 0; i < 16; ++i) {
      ab[i] = i < w ? a[k0 + i] : 0.0f;
      bb[i] = i < w ? b[k0 + i] : 0.0f;
    }
    acc = tc_block16(acc, ab, bb, f16);
  }
  return acc;
}

/* out[m, n] (fp32) = a[m, k] . w[n, k]^T with the tensor-core accumulation,
 * from 16-bit operand bits (f16 = 1: binary16, else bfloat16). */
void or_tc_gemm16(const uint16_t* a16, const uint16_t* w16, int m, int n, int k, int f16, float* out) {
  float* wf = (float*)malloc(sizeof(float) * (size_t)n * k);
  for (size_t i = 0; i < (size_t)n * k; ++i) wf[i] = f16 ? or_f16_decode(w16[i]) : or_bf16_decode(w16[i]);
#ifdef _OPENMP
#pragma omp parallel
#endif
  {
    float* af = (float*)malloc(sizeof(float) * (size_t)k);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int i = 0; i < m; ++i) {
      for (int c = 0; c < k; ++c) af[c] = f16 ? or_f16_decode(a16[(size_t)i * k + c]) : or_bf16_decode(a16[(size_t)i * k + c]);
      for (int j = 0; j < n; ++j) out[(size_t)i * n + j] = tc_dot(af, wf + (size_t)j * k, k, f16);
    }
    free(af);
  }
  free(wf);
}

/* The fp32 accumulation of tcgen05.mma kind::mxf8f6f4.block_scale (E4M3 x
 * E4M3, one UE8M0 scale per 32 K for each operand), measured the same way:
 * each instruction adds one 32-element K block to the accumulator with the
 * rule of tc_block16, the alignment exponent of a product being
 * exp(a) + exp(b) + (scale_a - 127) + (scale_b - 127) (an E4M3 subnormal
 * counting as exponent -6).  codes [rows, kp] E4M3 bytes, scales [rows, kp/32]
 * (unpacked UE8M0); out [m, n] fp32. */
static void e4m3_split(uint8_t c, int64_t* sig, int* e) {
  const int ef = (c >> 3) & 15, mant = c & 7;
  const int64_t s = ef == 0 ? mant : (mant | 8);
  *sig = (c & 0x80) ? -s : s;
  *e = ef == 0 ? -6 : ef - 7; /* value = sig * 2^(e - 3) */
}

void or_tc_gemm_mxf8(const uint8_t* a, const uint8_t* sa, const uint8_t* w, const uint8_t* sw, int m, int n,
                     int kp, float* out) {
  const int blocks = kp / 32;
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int i = 0; i < m; ++i) {
    for (int j = 0; j < n; ++j) {
      float acc = 0.0f;
      for (int b = 0; b < blocks; ++b) {
        int64_t ps[32];
        int pe[32];
        int emax = -100000;
        const int sc = ((int)sa[(size_t)i * blocks + b] - 127) + ((int)sw[(size_t)j * blocks + b] - 127);
        for (int t = 0; t < 32; ++t) {
          int64_t s1, s2;
          int e1, e2;
          e4m3_split(a[(size_t)i * kp + 32 * b + t], &s1, &e1);
          e4m3_split(w[(size_t)j * kp + 32 * b + t], &s2, &e2);
          ps[t] = s1 * s2;
          pe[t] = e1 + e2 + sc;
          if (ps[t] != 0 && pe[t] > emax) emax = pe[t];
        }
        int eacc = -100000;
        int64_t sacc = 0;
        if (acc != 0.0f) {
          int ex;
          const double fr = frexp((double)acc, &ex);
          sacc = (int64_t)ldexp(fr, 24);
          eacc = ex - 1;
          if (eacc > emax) emax = eacc;
        }
        if (emax == -100000) continue; /* nothing to add */
        const int unit = emax - 25;
        int64_t total = 0;
        for (int t = 0; t < 32; ++t) {
          if (ps[t] == 0) continue;
          const int sh = (pe[t] - 6) - unit; /* product = ps * 2^(pe - 6) */
          int64_t mag = ps[t] < 0 ? -ps[t] : ps[t];
          if (sh >= 0) mag <<= sh;
          else mag = sh <= -62 ? 0 : mag >> (-sh);
          total += ps[t] < 0 ? -mag : mag;
        }
        if (sacc != 0) {
          const int sh = (eacc - 23) - unit;
          int64_t mag = sacc < 0 ? -sacc : sacc;
          if (sh >= 0) mag <<= sh;
          else mag = sh <= -62 ? 0 : mag >> (-sh);
          total += sacc < 0 ? -mag : mag;
        }
        if (total == 0) {
          acc = 0.0f;
          continue;
        }
        uint64_t mg = (uint64_t)(total < 0 ? -total : total);
        int len = 0;
        while ((mg >> len) != 0) ++len;
        int ex = unit;
        if (len > 24) {
          mg >>= (len - 24);
          ex += len - 24;
        }
        const float r = (float)ldexp((double)mg, ex);
        acc = total < 0 ? -r : r;
      }
      out[(size_t)i * n + j] = acc;
    }
  }
}

/* ------------------------------------------------------------------ attention softmax */

/* 2^x on the FMA pipe, the attention kernel's own definition (attention_tc.cu
 * exp2_poly2): x clamped to -126, n = rint(x) by the 1.5*2^23 magic add,
 * f = x - n, a degree-3 polynomial in f, n added to the exponent field. */
static float exp2_poly(float x) {
  const float magic = 12582912.0f;
  x = fmaxf(x, -126.0f);
  const float j = x + magic;
  const float n = j - magic;
  const float f = fmaf(n, -1.0f, x);
  float p = fmaf(0x1.c2ccd4p-5f, f, 0x1.f02456p-3f);
  p = fmaf(p, f, 0x1.62f21p-1f);
  p = fmaf(p, f, 0x1.fff9ap-1f);
  uint32_t pb, jb;
  memcpy(&pb, &p, 4);
  memcpy(&jb, &j, 4);
  pb += jb << 23;
  memcpy(&p, &pb, 4);
  return p;
}

/* Softmax attention over one board per (position, head) with the arithmetic
 * of the tcgen05 attention kernel, which computes the reference's
 * softmax(q.k * scale) . v (cuda-kernels/attention_fa2_q64.cu:82-390;
 * tests/debug_exec_units.rs:161-242) with these definitional choices:
 *   - scores s = q.k on the tensor cores (tc_dot: blocks of 16 dims);
 *   - the keys form two halves, [0, 192) and [192, 368), each with its own
 *     maximum m (max of the fp32 scores over the half's keys below seq);
 *   - P = exp2_poly(fma(s, c, -(m*c))) with c = fp32(scale * log2 e), in
 *     slices of 48 keys (the last slice of the second half has 32); keys past
 *     seq have P = 0;
 *   - head dim 64: the row sum l of each slice sums the unrounded P pairwise
 *     into four partial sums (pair i into i % 4), combined as
 *     (l0 + l1) + (l2 + l3); a half's l combines its four slices the same way;
 *     head dim 32: a half's l is P.1 on the tensor cores, the rounded P in
 *     blocks of 16 keys (tc_block16), the accumulation O_h gets;
 *   - O_h = P.V of each half on the tensor cores, P rounded to the 16-bit type
 *     (f16 or bf16), blocks of 16 keys in key order (tc_block16);
 *   - out = 16-bit(O_A wa + O_B wb) with fa = 2^((m_A - m) c) (1 if m_A is the
 *     maximum), inv = 1 / (l_A fa + l_B fb), wa = fa inv, wb = fb inv, each
 *     operation rounded on its own.
 * qkv: 16-bit bits [n*seq, 3*heads*hd] with Q and K already rotated; out:
 * 16-bit bits [n*seq, heads*hd]. */
void or_attention_tc(const uint16_t* qkv, int n, int seq, int heads, int hd, float scale, int f16,
                     uint16_t* out) {
  const int c = heads * hd;
  const size_t ld = 3 * (size_t)c;
  const float sl = scale * 1.4426950408889634f;
  const int kpad = 368, half_a = 192;
  float ones[368]; /* the B operand of P.1 (head dim 32), read-only below */
  for (int j = 0; j < kpad; ++j) ones[j] = 1.0f;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic)
#endif
  for (int bh = 0; bh < n * heads; ++bh) {
    const int b = bh / heads, h = bh % heads;
    float* kf = (float*)malloc(sizeof(float) * (size_t)seq * hd);
    float* vt = (float*)calloc((size_t)hd * kpad, sizeof(float)); /* V transposed [d][key], keys >= seq zero */
    float* s = (float*)malloc(sizeof(float) * kpad);
    float* p16 = (float*)calloc(kpad, sizeof(float));
    const uint16_t* base = qkv + (size_t)b * seq * ld;
    for (int j = 0; j < seq; ++j)
      for (int d = 0; d < hd; ++d) {
        const uint16_t kb = base[j * ld + c + h * hd + d], vb = base[j * ld + 2 * c + h * hd + d];
        kf[(size_t)j * hd + d] = f16 ? or_f16_decode(kb) : or_bf16_decode(kb);
        vt[(size_t)d * kpad + j] = f16 ? or_f16_decode(vb) : or_bf16_decode(vb);
      }
    for (int qi = 0; qi < seq; ++qi) {
      float q[64];
      for (int d = 0; d < hd; ++d)
        q[d] = f16 ? or_f16_decode(base[qi * ld + h * hd + d]) : or_bf16_decode(base[qi * ld + h * hd + d]);
      for (int j = 0; j < kpad; ++j) s[j] = j < seq ? tc_dot(q, kf + (size_t)j * hd, hd, f16) : 0.0f;
      float m_h[2], l_h[2];
      for (int hf = 0; hf < 2; ++hf) {
        const int k0 = hf ? half_a : 0, k1 = hf ? kpad : half_a;
        float m = -INFINITY;
        for (int j = k0; j < k1 && j < seq; ++j) m = fmaxf(m, s[j]);
        const float mc = m * sl;
        float ls[4];
        for (int sub = 0; sub < 4; ++sub) {
          const int s0 = k0 + 48 * sub;
          const int nk = (hf && sub == 3) ? 32 : 48;
          const int valid = seq - s0 < nk ? seq - s0 : nk;
          float lp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int i = 0; i < nk / 2; ++i) {
            const int j0 = s0 + 2 * i, j1 = j0 + 1;
            const float e0 = exp2_poly(fmaf(s[j0], sl, -mc)), e1 = exp2_poly(fmaf(s[j1], sl, -mc));
            const float p0 = 2 * i < valid ? e0 : 0.0f;
            const float p1 = 2 * i + 1 < valid ? e1 : 0.0f;
            lp[i & 3] = lp[i & 3] + (p0 + p1);
            p16[j0] = round16(p0, f16);
            p16[j1] = round16(p1, f16);
          }
          ls[sub] = (lp[0] + lp[1]) + (lp[2] + lp[3]);
        }
        m_h[hf] = m;
        if (hd == 32) {
          l_h[hf] = tc_dot(p16 + k0, ones, k1 - k0, f16);
        } else {
          l_h[hf] = (ls[0] + ls[1]) + (ls[2] + ls[3]);
        }
      }
      const float mx = fmaxf(m_h[0], m_h[1]);
      const float fa = m_h[0] == mx ? 1.0f : exp2_poly((m_h[0] - mx) * sl);
      const float fb = m_h[1] == mx ? 1.0f : exp2_poly((m_h[1] - mx) * sl);
      const float inv = 1.0f / (l_h[0] * fa + l_h[1] * fb);
      const float wa = fa * inv, wb = fb * inv;
      uint16_t* o = out + ((size_t)b * seq + qi) * c + h * hd;
      for (int d = 0; d < hd; ++d) {
        const float oa = tc_dot(p16, vt + (size_t)d * kpad, half_a, f16);
        const float ob = tc_dot(p16 + half_a, vt + (size_t)d * kpad + half_a, kpad - half_a, f16);
        const float x = oa * wa + ob * wb;
        o[d] = f16 ? or_f16_encode(x) : or_bf16_encode(x);
      }
    }
    free(kf);
    free(vt);
    free(s);
    free(p16);
  }
}
