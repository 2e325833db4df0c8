"""tb_gemm_fused_noalloc (split-K partial sums in the library's fixed device
array, nothing allocated) against tb_gemm_fused with a caller workspace and
against the oracle.

The file name makes pytest collect it last, so that a run stopping at the
first failure has run every other test before it.  It passes either way it
is run: alone in a fresh process (its first call then does the one-time
set-up on the device) or after the other GPU tests.  The shapes split K, so
the fixed array is really used; two calls in a row check that the contents
left by one call do not leak into the next, and the device memory the CUDA
driver and PyTorch report stays the same across calls (nothing allocated)."""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev, empty_dev, from_dev

pytestmark = pytest.mark.gpu

TOL = 1e-3


def operands(fmt, M, N, K, seed):
    a = O.normal(seed, (M, K), 0.02)
    b = O.normal(seed + 1, (N, K), 1.0)
    s = O.per_tensor_scale(a, fmt)
    return O.quantize(fmt, a, s), O.f32_to_f16_bits(b).reshape(N, K), float(np.float32(1.0) / np.float32(s))


def with_workspace(tb, cuda, fmt, dA, dB, M, N, K, alpha):
    ws_bytes = tb.fused_workspace_bytes(fmt, M, N, K)
    ws = empty_dev(cuda, ws_bytes)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_fused(fmt, dA, dB, dD, M, N, K, alpha=alpha, workspace=ws, workspace_bytes=ws_bytes)
    cuda.cuda.synchronize()
    return from_dev(dD, np.float32).reshape(M, N)


def no_alloc(tb, cuda, fmt, dA, dB, M, N, K, alpha):
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_fused_noalloc(fmt, dA, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    return from_dev(dD, np.float32).reshape(M, N)


@pytest.mark.parametrize("fmt,M,N,K", [
    (O.E4M3, 256, 16, 8192),    # 2 tiles -> many splits
    (O.E2M1, 1024, 128, 4096),  # 8 tiles
    (O.BF16, 384, 200, 2048),   # ragged N
])
def test_no_alloc_matches_workspace_path(tb, cuda, fmt, M, N, K):
    assert tb.fused_workspace_bytes(fmt, M, N, K) > 0, "shape must take the split-K path"
    A, B16, alpha = operands(fmt, M, N, K, seed=fmt * 31 + M)
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    want = with_workspace(tb, cuda, fmt, dA, dB, M, N, K, alpha)
    first = no_alloc(tb, cuda, fmt, dA, dB, M, N, K, alpha)
    second = no_alloc(tb, cuda, fmt, dA, dB, M, N, K, alpha)
    oracle = O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha)
    for got in (first, second):
        assert np.all(np.isfinite(got))
        assert O.rel_frob(got, want) <= TOL
        assert O.rel_frob(got, oracle) <= TOL
    # Same kernels, same split count, same summation order: identical bits.
    np.testing.assert_array_equal(first.view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(second.view(np.uint32), want.view(np.uint32))


def test_no_alloc_alternating_shapes(tb, cuda):
    """A smaller call after a larger one reads none of the larger call's
    leftovers."""
    big = (O.E4M3, 1024, 256, 4096)
    small = (O.E4M3, 256, 16, 4096)
    outs = []
    for fmt, M, N, K in (big, small, big, small):
        A, B16, alpha = operands(fmt, M, N, K, seed=M + N)
        dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
        got = no_alloc(tb, cuda, fmt, dA, dB, M, N, K, alpha)
        want = with_workspace(tb, cuda, fmt, dA, dB, M, N, K, alpha)
        assert O.rel_frob(got, want) <= TOL
        outs.append(got)
    np.testing.assert_array_equal(outs[0], outs[2])
    np.testing.assert_array_equal(outs[1], outs[3])


def test_no_alloc_allocates_nothing(tb, cuda):
    """After a first call (the one-time set-up), further calls change neither
    the device's free memory nor PyTorch's reserved pool."""
    fmt, M, N, K = O.E4M3, 512, 16, 8192
    assert tb.fused_workspace_bytes(fmt, M, N, K) > 0
    A, B16, alpha = operands(fmt, M, N, K, seed=77)
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_fused_noalloc(fmt, dA, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    free0, _ = cuda.cuda.mem_get_info()
    reserved0 = cuda.cuda.memory_reserved()
    for _ in range(5):
        tb.gemm_fused_noalloc(fmt, dA, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    free1, _ = cuda.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    assert cuda.cuda.memory_reserved() == reserved0
    got = from_dev(dD, np.float32).reshape(M, N)
    assert O.rel_frob(got, O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha)) <= TOL
