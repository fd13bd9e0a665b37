"""GPU tests of the bounded device waits (the abort path).

Every wait inside this library's kernels gives up after a time limit, records
KB_STATUS_TIMEOUT in the status word, lets what it has issued (TMA copies,
tensor-core MMAs, TMA stores) finish, frees its tensor memory and returns, so
a fault never hangs the GPU.  These tests make waits run out on purpose
without any fault: a barrier that nothing arrives at, and a GEMM whose work
waits are limited to far less than the GEMM takes.  Afterwards the stream and
the device must still be usable and a normal GEMM on the same stream must be
bit-exact (which it cannot be if an aborted CTA left tensor memory allocated
or MMAs in flight).
"""

import numpy as np
import pytest

from rust_katago_b200 import _capi, int8

pytestmark = pytest.mark.gpu

TIMEOUT = 32  # KB_STATUS_TIMEOUT


def fresh_status(torch):
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    _capi.call("kb_status_reset", st.data_ptr(), int(torch.cuda.current_stream().cuda_stream))
    return st


def test_wait_on_unset_barrier_times_out(cuda):
    torch = cuda
    st = fresh_status(torch)
    stream = int(torch.cuda.current_stream().cuda_stream)
    _capi.call("kb_test_wait_timeout", 200_000, st.data_ptr(), stream)  # 200 us
    torch.cuda.synchronize()
    flags, layer = (int(v) & 0xFFFFFFFF for v in st.cpu().numpy())
    assert flags == TIMEOUT and layer == 0xFFFFFFFF
    # the context is intact
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == 1023 * 1024 / 2


@pytest.mark.parametrize("limit_ns", [1, 3_000])
def test_gemm_abort_then_exact_gemm(cuda, oracle, limit_ns):
    torch = cuda
    rng = np.random.default_rng(limit_ns)
    m, n, kp = 512, 512, 8192  # 64 K stages per tile: tens of microseconds per accumulator
    a = rng.integers(-127, 128, (m, kp), dtype=np.int8)
    w = rng.integers(-127, 128, (n, kp), dtype=np.int8)
    da, dw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    dots = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    st = fresh_status(torch)
    stream = int(torch.cuda.current_stream().cuda_stream)
    _capi.call("kb_test_int8_gemm_i32_wait_limit", da.data_ptr(), dw.data_ptr(), dots.data_ptr(), m, n, kp,
               limit_ns, st.data_ptr(), stream)
    torch.cuda.synchronize()
    flags = int(st.cpu().numpy()[0]) & 0xFFFFFFFF
    assert flags & TIMEOUT, "a wait limit far below the GEMM's duration must abort it"
    # the same stream runs the full GEMM next, twice (every SM's tensor memory
    # must have been released by the aborted CTAs)
    ref = oracle.igemm(a, w)
    for _ in range(2):
        dots.zero_()
        int8.gemm_i32(da, dw, dots, m, n, kp)
        torch.cuda.synchronize()
        assert np.array_equal(dots.cpu().numpy(), ref)


def test_gemm_full_limit_does_not_abort(cuda, oracle):
    """With a limit well above the GEMM's duration nothing is recorded."""
    torch = cuda
    rng = np.random.default_rng(5)
    m, n, kp = 300, 256, 1024
    a = rng.integers(-127, 128, (m, kp), dtype=np.int8)
    w = rng.integers(-127, 128, (n, kp), dtype=np.int8)
    da, dw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    dots = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    st = fresh_status(torch)
    _capi.call("kb_test_int8_gemm_i32_wait_limit", da.data_ptr(), dw.data_ptr(), dots.data_ptr(), m, n, kp,
               1_000_000_000, st.data_ptr(), int(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(st.cpu().numpy()[0]) == 0
    assert np.array_equal(dots.cpu().numpy(), oracle.igemm(a, w))
