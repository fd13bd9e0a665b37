"""CPU restatement of the reference's board-symmetry helpers — TEST INFRASTRUCTURE ONLY.

Follows crates/kata_game/src/symmetry.rs of the reference:
  * bit meanings (:12-24): bit 2 transpose, bit 1 flip x, bit 0 flip y;
  * get_sym_loc_xy (:27-38): flip first, then swap x and y;
  * invert (:79-87): 5 and 6 trade places, every other symmetry is its own inverse;
  * compose (:90-96);
  * copy_with_symmetry (:138-224), behind copy_inputs_with_symmetry (:108-123,
    reverse = false) and copy_outputs_with_symmetry (:126-136, reverse = true):
    the transpose only applies to square planes, and on the forward (input)
    direction the two flips trade places when transposing, so that the copy
    agrees with get_sym_loc_xy and the reverse copy undoes it.

The copies are restated with the reference's own stride bookkeeping (a base
offset and a signed stride per axis, strides swapped for a transpose), in numpy.
"""

from __future__ import annotations

import numpy as np


def is_transpose(sym: int) -> bool:
    return (sym & 4) != 0


def is_flip_x(sym: int) -> bool:
    return (sym & 2) != 0


def is_flip_y(sym: int) -> bool:
    return (sym & 1) != 0


def sym_loc_xy(x: int, y: int, x_size: int, y_size: int, sym: int) -> tuple[int, int]:
    """symmetry.rs:27-38."""
    if is_flip_x(sym):
        x = x_size - x - 1
    if is_flip_y(sym):
        y = y_size - y - 1
    if is_transpose(sym):
        x, y = y, x
    return x, y


def invert(sym: int) -> int:
    """symmetry.rs:79-87."""
    return {5: 6, 6: 5}.get(sym, sym)


def compose(first: int, nxt: int) -> int:
    """symmetry.rs:90-96: apply `first`, then `nxt`."""
    if is_transpose(first):
        nxt = (nxt & 4) | ((nxt & 2) >> 1) | ((nxt & 1) << 1)
    return first ^ nxt


def copy_with_symmetry(src, n: int, h: int, w: int, c: int, nhwc: bool, sym: int, reverse: bool) -> np.ndarray:
    """symmetry.rs:138-224 on a flat buffer of n*h*w*c values."""
    src = np.asarray(src).reshape(-1)
    dst = np.zeros_like(src)
    transpose = is_transpose(sym) and h == w
    flip_x, flip_y = is_flip_x(sym), is_flip_y(sym)
    if transpose and not reverse:
        flip_x, flip_y = flip_y, flip_x
    if nhwc:
        outer, outer_stride = n, h * w * c
        h_stride, w_stride, inner = w * c, c, c
    else:
        outer, outer_stride = n * c, h * w
        h_stride, w_stride, inner = w, 1, 1
    h_base, h_new = 0, h_stride
    w_base, w_new = 0, w_stride
    if flip_y:
        h_base, h_new = (h - 1) * h_new, -h_new
    if flip_x:
        w_base, w_new = (w - 1) * w_new, -w_new
    if transpose:
        h_new, w_new = w_new, h_new
    hh, ww = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
    old = (hh * h_stride + ww * w_stride).reshape(-1)
    new = (h_base + hh * h_new + w_base + ww * w_new).reshape(-1)
    for o in range(outer):
        base = o * outer_stride
        for k in range(inner):
            dst[base + new + k] = src[base + old + k]
    return dst


def copy_inputs(src, n: int, h: int, w: int, c: int, nhwc: bool, sym: int) -> np.ndarray:
    """copy_inputs_with_symmetry (symmetry.rs:108-123)."""
    return copy_with_symmetry(src, n, h, w, c, nhwc, sym, reverse=False)


def copy_outputs(src, n: int, h: int, w: int, sym: int) -> np.ndarray:
    """copy_outputs_with_symmetry (symmetry.rs:126-136)."""
    return copy_with_symmetry(src, n, h, w, 1, False, sym, reverse=True)


def apply_to_positions(spatial: np.ndarray, symmetry, nhwc: bool = False) -> np.ndarray:
    """Per-row copy_inputs_with_symmetry of [n, 22, 19, 19] (or NHWC
    [n, 19, 19, 22]) spatial inputs, as the reference's submit_output does for
    each row (crates/kata_nn/src/backends/cuda.rs:2233-2245)."""
    out = np.empty_like(spatial)
    for i, s in enumerate(symmetry):
        out[i] = copy_inputs(spatial[i], 1, 19, 19, 22, nhwc, int(s)).reshape(spatial[i].shape)
    return out
