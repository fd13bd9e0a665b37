"""GPU tests of the output decoder (kb_decode_device, kb_submit_rows /
kb_finish_rows) against the CPU oracle (oracle/outputs.py) and the
reference's known answers (output_postprocess_tests.rs).

Tolerances: decoding (symmetry reversal, optimism blend) is bit-exact.
Post-processing calls CUDA's expf / tanhf (max 2 ulp) and f64 exp / log
where the reference calls libm: policy probabilities within 1e-5 relative
(1e-12 absolute for underflowed moves), illegal moves exactly -1, value /
score / ownership within 1e-6 relative (1e-7 absolute).
"""

import numpy as np
import pytest

from oracle import outputs as oo
from rust_katago_b200 import _capi, backend, synthetic

from test_oracle_outputs import CASES, check_flip, check_temperature

pytestmark = pytest.mark.gpu

FIELDS = ("policy", "value", "misc", "moremisc", "ownership")


def device_decode(torch, raw_flat, rows, legal=None, **pp):
    n = rows.shape[0]
    d_raw = torch.from_numpy(np.ascontiguousarray(raw_flat, np.float32)).cuda()
    d_rows = torch.from_numpy(np.ascontiguousarray(rows).view(np.uint8).reshape(n, 24)).cuda()
    d_legal = None if legal is None else torch.from_numpy(np.ascontiguousarray(legal, np.uint8)).cuda()
    d_out = torch.full((n * backend.DEC_PER_POS,), float("nan"), dtype=torch.float32, device="cuda")
    backend.decode_device(n, d_raw, d_rows, d_legal, d_out, int(torch.cuda.current_stream().cuda_stream), **pp)
    torch.cuda.synchronize()
    out = backend.unpack_decoded(d_out.cpu().numpy(), n)
    return {f: getattr(out, f) for f in FIELDS}


def case_rows(h, row, dec_kw, post_kw):
    """kb_row_params for every row of a known-answer case (the checked row
    carries the case's parameters, the others the defaults)."""
    rows = backend.row_params(h.batch)
    r = rows[row]
    r["symmetry"] = dec_kw.get("symmetry", 0)
    r["policy_optimism"] = dec_kw.get("optimism", 0.0)
    r["include_owner_map"] = 1 if dec_kw.get("include_owner", True) else 0
    legal = None
    if post_kw is not None:
        r["policy_temperature"] = post_kw.get("temperature", 1.0)
        r["next_player_white"] = 1 if post_kw.get("next_white", True) else 0
        r["passing_hacks"] = 1 if post_kw.get("passing_hacks", False) else 0
        r["no_result_off"] = 1 if post_kw.get("no_result_off", False) else 0
        r["board_x"], r["board_y"] = post_kw.get("board_x", 19), post_kw.get("board_y", 19)
        legal = np.ones((h.batch, 362), np.uint8)
        legal[row] = np.asarray(post_kw["legal"], np.uint8)
    return rows, legal


def run_device_case(torch, case):
    _, h, row, dec_kw, post_kw, _ = case
    rows, legal = case_rows(h, row, dec_kw, post_kw)
    pp = (post_kw or {}).get("pp") or {}
    out = device_decode(torch, h.packed(), rows, legal, **pp)
    return {f: out[f][row] for f in FIELDS}


def assert_post_close(got, ref):
    pol_g, pol_r = got["policy"], ref["policy"]
    illegal = pol_r == -1.0
    assert np.array_equal(pol_g[illegal], pol_r[illegal])
    np.testing.assert_allclose(pol_g[~illegal], pol_r[~illegal], rtol=1e-5, atol=1e-12)
    for f in ("value", "misc", "moremisc", "ownership"):
        np.testing.assert_allclose(got[f], ref[f], rtol=1e-6, atol=1e-7, err_msg=f)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_known_answers_on_device(cuda, case):
    name, h, row, dec_kw, post_kw, check = case
    got = run_device_case(cuda, case)
    if check is not None:
        check(got)
    ref = oo.decode_row(h.policy[row], h.value[row], h.misc[row], h.moremisc[row], h.ownership[row],
                        dec_kw.get("symmetry", 0), dec_kw.get("optimism", 0.0), dec_kw.get("include_owner", True))
    if post_kw is None:
        for f in FIELDS:
            assert np.array_equal(got[f].view(np.uint32), ref[f].view(np.uint32)), f
    else:
        assert_post_close(got, oo.postprocess_row(ref, **post_kw))


def test_known_relations_on_device(cuda):
    by = {c[0]: c for c in CASES}
    check_flip(run_device_case(cuda, by["white_to_move"]), run_device_case(cuda, by["black_to_move"]))
    check_temperature(*(run_device_case(cuda, by[k]) for k in ("cold", "warm", "equivalent")))


def random_heads(rng, n):
    h = np.concatenate([
        (rng.standard_normal(n * 6 * 362) * 3.0), rng.standard_normal(n * 3) * 2.0,
        rng.standard_normal(n * 10) * 2.0, rng.standard_normal(n * 8), rng.standard_normal(n * 361) * 1.5])
    return h.astype(np.float32)


def random_rows(rng, n):
    return backend.row_params(
        n, symmetry=rng.integers(0, 8, n), policy_optimism=rng.choice([0.0, 0.25, 1.0, 0.7], n),
        policy_temperature=rng.choice([1.0, 0.5, 2.0, 1e-9], n), board_x=rng.choice([19, 19, 13, 9], n),
        board_y=rng.choice([19, 19, 13, 9], n), include_owner_map=rng.integers(0, 2, n),
        next_player_white=rng.integers(0, 2, n), passing_hacks=rng.integers(0, 2, n),
        no_result_off=rng.integers(0, 2, n))


def rows_as_dicts(rows):
    return [{k: rows[i][k] for k in rows.dtype.names} for i in range(rows.shape[0])]


@pytest.mark.parametrize("n", [1, 37])
def test_decode_bit_exact_random(cuda, n):
    rng = np.random.default_rng(n)
    raw = random_heads(rng, n)
    rows = random_rows(rng, n)
    got = device_decode(cuda, raw, rows)
    ref = oo.decode_packed(raw, n, rows_as_dicts(rows))
    for f in FIELDS:
        assert np.array_equal(got[f].view(np.uint32), ref[f].view(np.uint32)), f


@pytest.mark.parametrize("version", [3, 8, 10, 14, 17])
def test_postprocess_random(cuda, version):
    rng = np.random.default_rng(100 + version)
    n = 29
    raw = random_heads(rng, n)
    rows = random_rows(rng, n)
    legal = (rng.random((n, 362)) < 0.8).astype(np.uint8)
    legal[3] = 0  # no legal move: uniform fallback never divides by zero
    pp = dict(model_version=version, output_scale_multiplier=1.5, score_mean_multiplier=18.0)
    got = device_decode(cuda, raw, rows, legal, **pp)
    ref = oo.decode_packed(raw, n, rows_as_dicts(rows), legal, pp)
    for i in range(n):
        assert_post_close({f: got[f][i] for f in FIELDS}, {f: ref[f][i] for f in FIELDS})


def test_submit_rows_matches_raw_submit_and_oracle(cuda):
    """kb_submit_rows / kb_finish_rows: the forward under each row's symmetry,
    decoded on the device, equals kb_submit / kb_finish's raw heads decoded by
    the oracle (bit for bit), and post-processed within the tolerances."""
    topo = synthetic.Topology(256, 2, 4, 64, 1024)
    blob = synthetic.make_blob(topo, 5)
    n = 6
    spatial, glob = synthetic.make_positions(n, 41)
    rng = np.random.default_rng(3)
    rows = random_rows(rng, n)
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, n)
    raw = h.get_output(spatial, glob, rows["symmetry"].astype(np.int32))
    flat = np.concatenate([getattr(raw, f).reshape(-1) for f in FIELDS])
    dec = h.finish_rows(h.submit_rows(spatial, glob, rows))
    ref = oo.decode_packed(flat, n, rows_as_dicts(rows))
    for f in FIELDS:
        assert np.array_equal(getattr(dec, f).view(np.uint32), ref[f].view(np.uint32)), f
    legal = (rng.random((n, 362)) < 0.9).astype(np.uint8)
    pp = dict(model_version=14, lead_multiplier=10.0)
    h.set_postprocess(**pp)
    post = h.finish_rows(h.submit_rows(spatial, glob, rows, legal))
    ref = oo.decode_packed(flat, n, rows_as_dicts(rows), legal, pp)
    for i in range(n):
        assert_post_close({f: getattr(post, f)[i] for f in FIELDS}, {f: ref[f][i] for f in FIELDS})
    # Tokens are tied to the call that made them; bad rows are rejected.
    tok = h.submit_rows(spatial, glob, rows)
    with pytest.raises(_capi.KbError, match="kb_finish_rows"):
        h.finish_output(tok)
    bad = rows.copy()
    bad["policy_optimism"][0] = 1.5
    with pytest.raises(_capi.KbError, match="policy_optimism"):
        h.submit_rows(spatial, glob, bad)


def test_two_submissions_in_flight(cuda):
    """Both pipeline slots in use: the second submission's input copies run on
    the copy stream while the first forward runs; each result equals the one
    computed alone, bit for bit, for the raw and the decoding entry points."""
    topo = synthetic.Topology(256, 2, 4, 64, 1024)
    blob = synthetic.make_blob(topo, 5)
    n = 5
    sa, ga = synthetic.make_positions(n, 51)
    sb, gb = synthetic.make_positions(n, 52)
    rows = random_rows(np.random.default_rng(9), n)
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, n)
    alone_a, alone_b = h.finish_rows(h.submit_rows(sa, ga, rows)), h.finish_rows(h.submit_rows(sb, gb, rows))
    raw_a, raw_b = h.get_output(sa, ga), h.get_output(sb, gb)
    for _ in range(3):
        ta, tb = h.submit_rows(sa, ga, rows), h.submit_rows(sb, gb, rows)
        got_a, got_b = h.finish_rows(ta), h.finish_rows(tb)
        for got, ref in ((got_a, alone_a), (got_b, alone_b)):
            for f in FIELDS:
                assert np.array_equal(getattr(got, f), getattr(ref, f)), f
        ta, tb = h.submit_output(sa, ga), h.submit_output(sb, gb)
        # finished in the other order
        got_b, got_a = h.finish_output(tb), h.finish_output(ta)
        for got, ref in ((got_a, raw_a), (got_b, raw_b)):
            assert np.array_equal(got.policy, ref.policy) and np.array_equal(got.ownership, ref.ownership)
    with pytest.raises(_capi.KbError, match="slots"):
        h.submit_output(sa, ga)
        h.submit_output(sb, gb)
        h.submit_output(sa, ga)
