"""CPU restatement of the reference's output decoding — TEST INFRASTRUCTURE ONLY.

Follows crates/kata_nn/src/output_postprocess.rs of the reference:
  * decode_raw_outputs (:29-112): per row, policy channels 0 and 5 of the raw
    [6, 362] head (each with its own pass logit, :23-26), the row's symmetry
    reversed by copy_outputs_with_symmetry, blended as
    base + (opt - base) * optimism in f32 (:66-75); value, the first four misc
    and the first two moremisc fields copied (:76-87); ownership with the
    symmetry reversed when the row asks for it (:88-105);
  * postprocess_output (:140-330): policy scaled by
    output_scale_multiplier / clamp(temperature), illegal moves at -1e30, max,
    exp, the passing-hack cap on the pass entry, an index-order f32 sum, -1 for
    illegal moves; value and score in f64 with the model-version branches
    and the flip to white's perspective; ownership tanh'd and flipped, zero
    outside the board;
  * softplus (:333-339).
Pinned by the reference's own known answers (output_postprocess_tests.rs),
restated in tests/test_oracle_outputs.py.

f32 steps are numpy float32 scalars (one rounding per operation).  The f32
exp and tanh of the reference (Rust's f32::exp / tanh, i.e. libm expf /
tanhf) are taken as the correctly rounded float32 of the f64 function;
f64 steps use Python's math module (the same libm as the reference's f64).
"""

from __future__ import annotations

import math

import numpy as np

from . import symmetry as sy

AREA, POLICY = 361, 362
f32 = np.float32

# ModelPostProcessParams::default (crates/kata_nn/src/desc.rs:682-695).
DEFAULT_PP = dict(model_version=17, output_scale_multiplier=1.0, td_score_multiplier=20.0,
                  score_mean_multiplier=20.0, score_stdev_multiplier=20.0, lead_multiplier=20.0,
                  variance_time_multiplier=40.0, shortterm_value_error_multiplier=0.25,
                  shortterm_score_error_multiplier=30.0)


def _exp32(x) -> np.float32:
    x = float(x)
    try:
        return f32(math.exp(x))
    except OverflowError:
        return f32(np.inf)


def softplus(x: float) -> float:
    """output_postprocess.rs:333-339."""
    return x if x > 40.0 else math.log(1.0 + math.exp(x))


def decode_row(policy6, value, misc, moremisc, ownership, symmetry: int, optimism: float,
               include_owner: bool = True) -> dict:
    """decode_raw_outputs for one row of raw heads: policy6 [6, 362], value [3],
    misc [10], moremisc [8], ownership [361]."""
    policy6 = np.asarray(policy6, np.float32).reshape(6, POLICY)
    base, opt = policy6[0], policy6[5]
    if symmetry != 0:
        base_b = sy.copy_outputs(base[:AREA], 1, 19, 19, symmetry)
        opt_b = sy.copy_outputs(opt[:AREA], 1, 19, 19, symmetry)
    else:
        base_b, opt_b = base[:AREA].copy(), opt[:AREA].copy()
    o = f32(optimism)
    pol = np.empty(POLICY, np.float32)
    for pos in range(AREA):
        pol[pos] = base_b[pos] + (opt_b[pos] - base_b[pos]) * o
    pol[AREA] = base[AREA] + (opt[AREA] - base[AREA]) * o
    own = np.zeros(AREA, np.float32)
    if include_owner:
        src = np.asarray(ownership, np.float32).reshape(AREA)
        own = sy.copy_outputs(src, 1, 19, 19, symmetry) if symmetry != 0 else src.copy()
    return dict(policy=pol, value=np.asarray(value, np.float32)[:3].copy(),
                misc=np.asarray(misc, np.float32)[:4].copy(), moremisc=np.asarray(moremisc, np.float32)[:2].copy(),
                ownership=own)


def postprocess_row(dec: dict, legal, temperature: float = 1.0, next_white: bool = True,
                    passing_hacks: bool = False, no_result_off: bool = False, board_x: int = 19,
                    board_y: int = 19, include_owner: bool = True, pp: dict | None = None) -> dict:
    """postprocess_output on one decoded row (a copy is returned)."""
    pp = dict(DEFAULT_PP, **(pp or {}))
    version = pp["model_version"]
    legal = np.asarray(legal).astype(bool).reshape(POLICY)
    pol = dec["policy"].astype(np.float32).copy()
    scaling = f32(pp["output_scale_multiplier"]) / f32(min(max(f32(temperature), f32(1e-6)), f32(1e6)))
    max_policy = f32(-1e25)
    count = 0
    for i in range(POLICY):
        if legal[i]:
            count += 1
            v = pol[i] * scaling
        else:
            v = f32(-1e30)
        pol[i] = v
        if v > max_policy:
            max_policy = v
    total = f32(0.0)
    if passing_hacks:
        for i in range(POLICY - 1):
            v = _exp32(pol[i] - max_policy)
            pol[i] = v
            total = f32(total + v)
        v = _exp32(pol[AREA] - max_policy)
        v = max(min(v, f32(total * f32(19.0))), f32(1e-20))
        pol[AREA] = v
        total = f32(total + v)
    else:
        for i in range(POLICY):
            v = _exp32(pol[i] - max_policy)
            pol[i] = v
            total = f32(total + v)
    if total <= 0.0:
        uniform = f32(1.0) / f32(max(count, 1))
        pol = np.where(legal, uniform, f32(-1.0)).astype(np.float32)
    else:
        pol = np.array([pol[i] / total if legal[i] else f32(-1.0) for i in range(POLICY)], np.float32)

    value = dec["value"].copy()
    misc = dec["misc"].copy()
    more = dec["moremisc"].copy()
    if version >= 4:
        osm = float(f32(pp["output_scale_multiplier"]))
        win_l, loss_l, nr_l = (float(value[i]) * osm for i in range(3))
        sm_pre, sd_pre, lead_pre, vt_pre = (float(misc[i]) * osm for i in range(4))
        sw_pre, ss_pre = (float(more[i]) * osm for i in range(2))
        if no_result_off:
            nr_l -= 100000.0
        mx = max(max(win_l, loss_l), nr_l)
        win, loss, nr = math.exp(win_l - mx), math.exp(loss_l - mx), math.exp(nr_l - mx)
        if no_result_off:
            nr = 0.0
        s = win + loss + nr
        win, loss, nr = win / s, loss / s, nr / s
        score_mean = sm_pre * pp["score_mean_multiplier"]
        score_stdev = softplus(sd_pre) * pp["score_stdev_multiplier"]
        score_mean_sq = score_mean * score_mean + score_stdev * score_stdev
        lead = lead_pre * pp["lead_multiplier"]
        var_time = softplus(vt_pre) * pp["variance_time_multiplier"]
        score_mean *= 1.0 - nr
        score_mean_sq *= 1.0 - nr
        lead *= 1.0 - nr
        if version >= 14:
            s1, s2 = softplus(sw_pre * 0.5), softplus(ss_pre * 0.5)
            st_w = math.sqrt(s1 * s1 * pp["shortterm_value_error_multiplier"])
            st_s = math.sqrt(s2 * s2 * pp["shortterm_score_error_multiplier"])
        elif version >= 10:
            st_w = math.sqrt(softplus(sw_pre) * pp["shortterm_value_error_multiplier"])
            st_s = math.sqrt(softplus(ss_pre) * pp["shortterm_score_error_multiplier"])
        else:
            st_w, st_s = softplus(sw_pre), softplus(ss_pre) * 10.0
        if next_white:
            value = np.array([win, loss, nr], np.float32)
            misc[0], misc[1], misc[2] = f32(score_mean), f32(score_mean_sq), f32(lead)
        else:
            value = np.array([loss, win, nr], np.float32)
            misc[0], misc[1], misc[2] = -f32(score_mean), f32(score_mean_sq), -f32(lead)
        if version >= 9:
            misc[3], more[0], more[1] = f32(var_time), f32(st_w), f32(st_s)
        else:
            misc[3], more[0], more[1] = f32(-1.0), f32(-1.0), f32(-1.0)

    own = dec["ownership"].copy()
    if include_owner:
        s = f32(pp["output_scale_multiplier"])
        for pos in range(AREA):
            y, x = divmod(pos, 19)
            if y >= board_y or x >= board_x:
                own[pos] = 0.0
            else:
                t = f32(math.tanh(float(own[pos] * s)))
                own[pos] = t if next_white else -t
    return dict(policy=pol, value=value, misc=misc, moremisc=more, ownership=own)


def decode_packed(raw_flat, n: int, rows, legal=None, pp: dict | None = None) -> dict:
    """Decode n rows of the packed head-major raw output (policy [n, 6, 362] |
    value [n, 3] | misc [n, 10] | moremisc [n, 8] | ownership [n, 361]).
    `rows` is a sequence of dicts with the kb_row_params field names; with
    `legal` ([n, 362]) every row is post-processed too.  Returns stacked arrays."""
    raw_flat = np.asarray(raw_flat, np.float32).reshape(-1)
    o = 0
    pol = raw_flat[o:o + n * 6 * POLICY].reshape(n, 6, POLICY)
    o += n * 6 * POLICY
    val = raw_flat[o:o + n * 3].reshape(n, 3)
    o += n * 3
    misc = raw_flat[o:o + n * 10].reshape(n, 10)
    o += n * 10
    more = raw_flat[o:o + n * 8].reshape(n, 8)
    o += n * 8
    own = raw_flat[o:o + n * AREA].reshape(n, AREA)
    out = {k: [] for k in ("policy", "value", "misc", "moremisc", "ownership")}
    for i in range(n):
        r = rows[i]
        d = decode_row(pol[i], val[i], misc[i], more[i], own[i], int(r["symmetry"]), float(r["policy_optimism"]),
                       bool(r["include_owner_map"]))
        if legal is not None:
            d = postprocess_row(d, legal[i], float(r["policy_temperature"]), bool(r["next_player_white"]),
                                bool(r["passing_hacks"]), bool(r["no_result_off"]), int(r["board_x"]),
                                int(r["board_y"]), bool(r["include_owner_map"]), pp)
        for k in out:
            out[k].append(d[k])
    return {k: np.stack(v) for k, v in out.items()}
