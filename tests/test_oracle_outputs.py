"""The output-decoding oracle against the reference's own known answers
(crates/kata_nn/src/output_postprocess_tests.rs), the device kernel's index
formula against the oracle's symmetry, and the C structs' layout against the
host mirror."""

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import outputs as oo
from oracle import symmetry as sy
from rust_katago_b200 import _capi
from rust_katago_b200.backend import ROW_PARAMS_DTYPE

ROOT = Path(__file__).resolve().parents[1]
AREA, POLICY = 361, 362


class Heads:
    """Raw heads of `batch` rows, as the reference tests build them."""

    def __init__(self, batch):
        self.batch = batch
        self.policy = np.zeros((batch, 6, POLICY), np.float32)
        self.value = np.zeros((batch, 3), np.float32)
        self.misc = np.zeros((batch, 10), np.float32)
        self.moremisc = np.zeros((batch, 8), np.float32)
        self.ownership = np.zeros((batch, AREA), np.float32)

    def decode(self, row, symmetry=0, optimism=0.0, include_owner=True):
        return oo.decode_row(self.policy[row], self.value[row], self.misc[row], self.moremisc[row],
                             self.ownership[row], symmetry, optimism, include_owner)

    def packed(self):
        return np.concatenate([a.reshape(-1) for a in (self.policy, self.value, self.misc, self.moremisc,
                                                       self.ownership)])


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


# Legal masks of the reference tests: an empty 19x19 board, and one with a
# black stone on (9, 9) (every other point and the pass stay legal).
EMPTY = np.ones(POLICY, bool)
OCCUPIED = 9 * 19 + 9
ONE_STONE = EMPTY.copy()
ONE_STONE[OCCUPIED] = False
# chinese(): simple ko, area scoring -> no result kept; area_without_no_result:
# situational ko, area scoring -> suppressed; territory keeps it.
CHINESE = dict(no_result_off=False)
AREA_NO_RESULT_OFF = dict(no_result_off=True)


def known_answer_cases():
    """(name, heads, decode kwargs, post kwargs or None, check) for every known
    answer of output_postprocess_tests.rs; shared with the GPU test, which runs
    the same cases through kb_decode_device."""
    cases = []

    # decode_uses_each_rows_six_pass_aware_policy_channels_and_exact_head_offsets
    h = Heads(2)
    for row in range(2):
        for ch in range(6):
            h.policy[row, ch] = -100.0 - ch
    h.policy[0, 0], h.policy[0, 5], h.policy[1, 0], h.policy[1, 5] = 11.0, 19.0, 2.0, 10.0
    h.policy[1, 0, AREA], h.policy[1, 5, AREA] = 3.0, 19.0
    h.value[1] = [2.0, 3.0, 5.0]
    h.misc[1, :4] = [7.0, 11.0, 13.0, 17.0]
    h.moremisc[1, :2] = [19.0, 23.0]
    h.ownership[1] = 29.0

    def check_offsets(out):
        assert np.all(out["policy"][:AREA] == 4.0) and out["policy"][AREA] == 7.0
        assert bits(np.concatenate([out["value"], out["misc"], out["moremisc"]])).tolist() == \
            bits([2.0, 3.0, 5.0, 7.0, 11.0, 13.0, 17.0, 19.0, 23.0]).tolist()
        assert np.all(out["ownership"] == 29.0)
    cases.append(("offsets", h, 1, dict(optimism=0.25), None, check_offsets))

    # quarter_turn_outputs_undo_the_production_input_transform_once
    original = np.arange(AREA, dtype=np.float32) - 128.0
    owner = (np.arange(AREA, dtype=np.float32) - 90.0) * np.float32(0.125)
    for sym in (5, 6):
        h = Heads(1)
        t = sy.copy_inputs(original, 1, 19, 19, 1, False, sym)
        assert not np.array_equal(t, original)
        h.policy[0, 0, :AREA] = t
        h.policy[0, 5, :AREA] = t
        h.policy[0, 0, AREA], h.policy[0, 5, AREA] = 17.0, 33.0
        h.ownership[0] = sy.copy_inputs(owner, 1, 19, 19, 1, False, sym)

        def check_turn(out):
            assert bits(out["policy"][:AREA]).tolist() == bits(original).tolist()
            assert out["policy"][AREA] == 21.0
            assert bits(out["ownership"]).tolist() == bits(owner).tolist()
        cases.append((f"quarter_turn_{sym}", h, 0, dict(symmetry=sym, optimism=0.25), None, check_turn))

    # player_to_move_outputs_flip_only_the_white_perspective_fields (both sides
    # are compared inside one check).
    h = Heads(1)
    h.value[0] = [2.0, -1.0, -2.0]
    h.misc[0, :4] = [0.25, 0.5, 0.75, 1.0]
    h.moremisc[0, :2] = [0.3, 0.6]
    h.ownership[0, 0], h.ownership[0, 1] = 0.75, -0.5
    cases.append(("white_to_move", h, 0, {}, dict(legal=EMPTY, next_white=True, **CHINESE), None))
    cases.append(("black_to_move", h, 0, {}, dict(legal=EMPTY, next_white=False, **CHINESE), None))

    # chinese_simple_ko_retains_no_result_and_only_non_simple_area_suppresses_it
    h = Heads(1)

    def third(out):
        assert abs(out["value"][2] - 1.0 / 3.0) <= 1e-7

    def suppressed(out):
        assert out["value"][2] == 0.0 and out["value"][0] == 0.5 and out["value"][1] == 0.5
    cases.append(("chinese", h, 0, {}, dict(legal=EMPTY, **CHINESE), third))
    cases.append(("area_situational", h, 0, {}, dict(legal=EMPTY, **AREA_NO_RESULT_OFF), suppressed))
    cases.append(("territory", h, 0, {}, dict(legal=EMPTY, no_result_off=False), third))

    # score_channel_one_is_stdev_and_model_multipliers_have_distinct_roles
    h = Heads(1)
    h.misc[0, :4] = [2.0, 0.0, 5.0, 50.0]
    pp = dict(score_mean_multiplier=3.0, score_stdev_multiplier=4.0, lead_multiplier=7.0,
              variance_time_multiplier=2.0)

    def score_base(out):
        assert out["misc"][0] == 6.0 and out["misc"][2] == 35.0 and out["misc"][3] == 100.0
        assert abs(out["misc"][1] - 43.68725) <= 1e-4

    def score_wider(out):
        assert out["misc"][0] == 6.0 and out["misc"][2] == 35.0
        base_sq = 36.0 + (math.log(2.0) * 4.0) ** 2
        assert abs((out["misc"][1] - 36.0) - 4.0 * (base_sq - 36.0)) <= 2e-5

    def score_scaled(out):
        assert out["misc"][0] == 12.0 and out["misc"][2] == 70.0 and out["misc"][3] == 200.0
    cases.append(("score_base", h, 0, {}, dict(legal=EMPTY, pp=pp, **AREA_NO_RESULT_OFF), score_base))
    cases.append(("score_wider", h, 0, {}, dict(legal=EMPTY, pp=dict(pp, score_stdev_multiplier=8.0),
                                                **AREA_NO_RESULT_OFF), score_wider))
    cases.append(("score_scaled", h, 0, {}, dict(legal=EMPTY, pp=dict(pp, output_scale_multiplier=2.0),
                                                 **AREA_NO_RESULT_OFF), score_scaled))

    # uncertainty_uses_model_version_branches_and_preserves_old_sentinels
    h = Heads(1)
    for version, ew, es in ((8, -1.0, -1.0), (9, 0.6931472, 6.931472), (10, 1.6651093, 2.4976637),
                            (13, 1.6651093, 2.4976637), (14, 1.3862944, 2.0794415), (17, 1.3862944, 2.0794415)):
        def check_version(out, version=version, ew=ew, es=es):
            assert abs(out["moremisc"][0] - ew) <= 1e-6 and abs(out["moremisc"][1] - es) <= 1e-6
            assert (out["misc"][3] == -1.0) if version < 9 else (out["misc"][3] > 0.0)
        cases.append((f"version_{version}", h, 0, {},
                      dict(legal=EMPTY, pp=dict(model_version=version, shortterm_value_error_multiplier=4.0,
                                                shortterm_score_error_multiplier=9.0), **CHINESE), check_version))

    # legal_mask_temperature_scaling_and_pass_hack_share_production_semantics
    h = Heads(1)
    h.policy[0, 0, OCCUPIED] = 1000.0
    h.policy[0, 0, 0] = 4.0

    def legal_sum(out):
        assert out["policy"][OCCUPIED] == -1.0
        assert abs(out["policy"][out["policy"] >= 0].sum() - 1.0) <= 2e-5
    cases.append(("cold", h, 0, {}, dict(legal=ONE_STONE, **CHINESE), legal_sum))
    cases.append(("warm", h, 0, {}, dict(legal=ONE_STONE, temperature=2.0, **CHINESE), legal_sum))
    cases.append(("equivalent", h, 0, {}, dict(legal=ONE_STONE, temperature=2.0, pp=dict(output_scale_multiplier=2.0),
                                               **CHINESE), legal_sum))
    h = Heads(1)
    h.policy[0, 0, AREA] = 10.0

    def plain_pass(out):
        assert out["policy"][AREA] > 0.95

    def capped_pass(out):
        assert abs(out["policy"][AREA] - 0.95) <= 1e-6 and out["policy"][OCCUPIED] == -1.0
        assert abs(out["policy"][out["policy"] >= 0].sum() - 1.0) <= 2e-5
    cases.append(("plain_pass", h, 0, {}, dict(legal=ONE_STONE, **CHINESE), plain_pass))
    cases.append(("capped_pass", h, 0, {}, dict(legal=ONE_STONE, passing_hacks=True, **CHINESE), capped_pass))
    h = Heads(1)
    h.policy[0, 0] = -1000.0
    h.policy[0, 0, AREA] = 1000.0

    def underflow(out):
        assert out["policy"][AREA] == 1.0
        expect = np.zeros(AREA, np.float32)
        expect[OCCUPIED] = -1.0
        assert np.array_equal(out["policy"][:AREA], expect)
    cases.append(("underflow", h, 0, {}, dict(legal=ONE_STONE, passing_hacks=True, **CHINESE), underflow))
    return cases


def run_oracle_case(h, row, dec_kw, post_kw):
    out = h.decode(row, **dec_kw)
    if post_kw is not None:
        out = oo.postprocess_row(out, **post_kw)
    return out


CASES = known_answer_cases()


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_known_answers(case):
    name, h, row, dec_kw, post_kw, check = case
    out = run_oracle_case(h, row, dec_kw, post_kw)
    if check is not None:
        check(out)


def test_player_flip_relations():
    """player_to_move_outputs_flip_only_the_white_perspective_fields."""
    by = {c[0]: c for c in CASES}
    w = run_oracle_case(*by["white_to_move"][1:5])
    b = run_oracle_case(*by["black_to_move"][1:5])
    check_flip(w, b)


def check_flip(w, b):
    assert w["value"][0] > w["value"][1]
    assert bits(w["value"][0]) == bits(b["value"][1]) and bits(w["value"][1]) == bits(b["value"][0])
    assert bits(w["value"][2]) == bits(b["value"][2])
    assert w["misc"][0] > 0.0 and w["misc"][2] > 0.0
    assert bits(w["misc"][0]) == bits(-b["misc"][0]) and bits(w["misc"][2]) == bits(-b["misc"][2])
    assert bits([w["misc"][1], w["misc"][3], *w["moremisc"]]).tolist() == \
        bits([b["misc"][1], b["misc"][3], *b["moremisc"]]).tolist()
    assert bits(w["policy"]).tolist() == bits(b["policy"]).tolist()
    assert bits(w["ownership"]).tolist() == bits(-b["ownership"]).tolist()
    assert np.all(np.abs(w["ownership"]) <= 1.0)
    assert w["ownership"][0] > 0.0 and w["ownership"][1] < 0.0


def test_temperature_relations():
    """cold[0] > warm[0], cold[1] < warm[1], and scale 2 at temperature 2
    equals temperature 1 bit for bit."""
    by = {c[0]: c for c in CASES}
    cold, warm, eq = (run_oracle_case(*by[k][1:5]) for k in ("cold", "warm", "equivalent"))
    check_temperature(cold, warm, eq)


def check_temperature(cold, warm, eq):
    assert cold["policy"][0] > warm["policy"][0] and cold["policy"][1] < warm["policy"][1]
    assert bits(eq["policy"]).tolist() == bits(cold["policy"]).tolist()


def test_score_wider_exact_relation():
    by = {c[0]: c for c in CASES}
    base = run_oracle_case(*by["score_base"][1:5])
    wider = run_oracle_case(*by["score_wider"][1:5])
    assert abs((wider["misc"][1] - 36.0) - 4.0 * (base["misc"][1] - 36.0)) <= 2e-5


def test_without_owner_map_keeps_policy():
    by = {c[0]: c for c in CASES}
    _, h, row, dec_kw, _, _ = by["offsets"]
    with_owner = h.decode(row, **dec_kw)
    without = h.decode(row, include_owner=False, **{k: v for k, v in dec_kw.items() if k != "include_owner"})
    assert np.all(without["ownership"] == 0.0)
    assert bits(without["policy"]).tolist() == bits(with_owner["policy"]).tolist()


@pytest.mark.parametrize("sym", range(8))
def test_device_scatter_formula(sym):
    """decode.cu's sym_target (network cell (r, c) -> board cell), restated,
    against the oracle's copy_outputs_with_symmetry."""
    def sym_target(s, r, c):
        a, b = (c, r) if s & 4 else (r, c)
        return (18 - a if s & 1 else a) * 19 + (18 - b if s & 2 else b)

    src = np.arange(AREA, dtype=np.float32)
    dst = sy.copy_outputs(src, 1, 19, 19, sym)
    for cell in range(AREA):
        assert dst[sym_target(sym, cell // 19, cell % 19)] == src[cell]


def test_packed_decode_matches_rows():
    rng = np.random.default_rng(5)
    n = 3
    h = Heads(n)
    for a in (h.policy, h.value, h.misc, h.moremisc, h.ownership):
        a[...] = rng.standard_normal(a.shape).astype(np.float32)
    rows = [dict(symmetry=s, policy_optimism=o, include_owner_map=1, policy_temperature=1.0, next_player_white=1,
                 passing_hacks=0, no_result_off=0, board_x=19, board_y=19) for s, o in ((0, 0.0), (5, 0.5), (3, 1.0))]
    out = oo.decode_packed(h.packed(), n, rows)
    for i, r in enumerate(rows):
        d = h.decode(i, r["symmetry"], r["policy_optimism"])
        for k in d:
            assert bits(out[k][i]).tolist() == bits(d[k]).tolist()


def test_c_struct_layout_matches_host_mirror(tmp_path):
    """offsetof / sizeof of kb_row_params and kb_postprocess_params, compiled
    from include/katab200.h with gcc, against ROW_PARAMS_DTYPE and
    _capi.PostProcessParams."""
    src = tmp_path / "layout.c"
    row_fields = list(ROW_PARAMS_DTYPE.names)
    pp_fields = [f for f, _ in _capi.PostProcessParams._fields_]
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "katab200.h"', "int main(void) {",
             'printf("%zu %zu\\n", sizeof(kb_row_params), sizeof(kb_postprocess_params));']
    lines += [f'printf("%zu\\n", offsetof(kb_row_params, {f}));' for f in row_fields]
    lines += [f'printf("%zu\\n", offsetof(kb_postprocess_params, {f}));' for f in pp_fields]
    lines += ["return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals[0] == ROW_PARAMS_DTYPE.itemsize == 24
    assert vals[1] == ctypes.sizeof(_capi.PostProcessParams) == 64
    assert vals[2:2 + len(row_fields)] == [ROW_PARAMS_DTYPE.fields[f][1] for f in row_fields]
    assert vals[2 + len(row_fields):] == [getattr(_capi.PostProcessParams, f).offset for f in pp_fields]
