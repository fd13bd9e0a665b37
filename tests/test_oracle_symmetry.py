"""The symmetry oracle against the reference's own known answers
(crates/kata_game/src/symmetry.rs:445-578) and the properties that tie the
input copy, the output copy and get_sym_loc_xy together."""

import numpy as np
import pytest

from oracle import symmetry as sy


def test_known_answer_flip_x_nchw():
    # symmetry.rs test_copy_inputs_with_symmetry_flip_x_nchw
    src = np.arange(6, dtype=np.float32)
    assert sy.copy_inputs(src, 1, 2, 3, 1, False, 2).tolist() == [2.0, 1.0, 0.0, 5.0, 4.0, 3.0]


def test_known_answer_transpose_nhwc():
    # symmetry.rs test_copy_inputs_with_symmetry_transpose_nhwc
    src = np.arange(4, dtype=np.float32)
    assert sy.copy_inputs(src, 1, 2, 2, 1, True, 4).tolist() == [0.0, 2.0, 1.0, 3.0]


def test_known_answer_locations():
    # test_identity, test_flip_x_roundtrip, test_transpose_swaps_size
    assert sy.sym_loc_xy(4, 4, 9, 9, 0) == (4, 4)
    assert sy.sym_loc_xy(*sy.sym_loc_xy(2, 3, 9, 9, 2), 9, 9, 2) == (2, 3)
    assert sy.sym_loc_xy(1, 2, 9, 9, 4) == (2, 1)


def test_compose_and_invert():
    # test_compose_identity, test_invert_involution
    assert sy.compose(0, 3) == 3
    for s in range(8):
        assert sy.invert(sy.invert(s)) == s
        assert sy.compose(s, sy.invert(s)) == 0


@pytest.mark.parametrize("sym", range(8))
@pytest.mark.parametrize("nhwc", [False, True])
def test_input_copy_agrees_with_sym_loc(sym, nhwc):
    """The feature at board (x, y) appears at get_sym_loc_xy(x, y) in the
    network's frame, for every channel and both layouts."""
    rng = np.random.default_rng(sym)
    c = 3
    src = rng.standard_normal((2, 19, 19, c) if nhwc else (2, c, 19, 19)).astype(np.float32)
    dst = sy.copy_inputs(src, 2, 19, 19, c, nhwc, sym).reshape(src.shape)
    for y in range(19):
        for x in range(19):
            nx, ny = sy.sym_loc_xy(x, y, 19, 19, sym)
            if nhwc:
                assert np.array_equal(dst[:, ny, nx, :], src[:, y, x, :])
            else:
                assert np.array_equal(dst[:, :, ny, nx], src[:, :, y, x])


@pytest.mark.parametrize("sym", range(8))
def test_output_copy_undoes_input_copy(sym):
    """decode_raw_outputs relies on copy_outputs_with_symmetry(sym) undoing
    copy_inputs_with_symmetry(sym) (output_postprocess.rs:39-41)."""
    src = np.random.default_rng(10 + sym).standard_normal(3 * 361).astype(np.float32)
    there = sy.copy_inputs(src, 3, 19, 19, 1, False, sym)
    assert np.array_equal(sy.copy_outputs(there, 3, 19, 19, sym), src)


def test_rectangular_plane_skips_transpose():
    src = np.arange(6, dtype=np.float32)
    assert np.array_equal(sy.copy_inputs(src, 1, 2, 3, 1, False, 4), src)
    assert sy.copy_inputs(src, 1, 2, 3, 1, False, 5).tolist() == sy.copy_inputs(src, 1, 2, 3, 1, False, 1).tolist()


def test_device_gather_formula():
    """The stem gather reads network cell (r, c) from the input cell given by
    sym_source in trunk.cu; restated here and checked against the oracle copy
    for every symmetry (the GPU test then checks the kernel end to end)."""
    def sym_source(s, r, c):
        a, b = (c, r) if s & 4 else (r, c)
        if s & 1:
            a = 18 - a
        if s & 2:
            b = 18 - b
        return a * 19 + b

    src = np.arange(361, dtype=np.float32)
    for s in range(8):
        dst = sy.copy_inputs(src, 1, 19, 19, 1, False, s)
        for cell in range(361):
            assert dst[cell] == src[sym_source(s, cell // 19, cell % 19)]
