"""The GEMMs at the full sizes of the benchmark configurations, against the
oracle and against decode-kernel-then-GEMM:

  * weight-only MLP shapes: W 14336 x 4096 and 4096 x 14336 (output features x
    K), N(0, 0.02) quantized per tensor to FP8 E4M3 and packed FP4 E2M1,
    activations FP16 N(0, 1) with 1, 16, 128 and 2048 tokens;
  * 8192^3 packed FP4 (N(0, 1), scale 6/maxabs) with FP16 output;
  * the 16384 x 53248 E4M3 weight used as its transpose (53248 output rows,
    K = 16384) with 8192 FP16 tokens and FP16 output, on one GPU.

Operands are drawn and quantized on the device (tb_quantize is bit-exact to
the reference quantizer, tests/test_quantize_gpu.py); the oracle reads the
same stored bytes.  Checks, as the reference checks its own path
(bench/bench_fused.cu:85-87 fused == unfused, bench/bench_formats.cu:97-103
relative Frobenius error):
  * the fused GEMM with the workspace the benchmark gives it (split K where
    the launcher splits) within 1e-3 relative Frobenius error of the oracle on
    row bands that straddle 128-row tile boundaries and on the last rows;
  * the fused GEMM without workspace (one accumulation over all of K) equal,
    bit for bit over the whole of D, to the decode kernel followed by the
    FP16 GEMM, and within 1e-3 of the oracle on the same bands.  Few-token
    shapes (N <= 128) run the weight-streaming kernel, whose MMAs read the
    decoded weights from tensor memory: tcgen05.mma rounds its FP32
    accumulation differently with A in tensor memory than with A in shared
    memory (measured relative error against an FP64 product 3.9e-6 against
    8.1e-7 at K = 4096), so there the whole-D comparison is a relative
    Frobenius difference of at most 1e-4 instead of bit equality.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-3
FMAX = {O.E4M3: 448.0, O.E2M1: 6.0}


def device_operands(cuda, tb, fmt, M, N, K, a_std, seed):
    """A [M x K] N(0, a_std) quantized per tensor on the device, B [N x K]
    FP16 N(0, 1); alpha = 1/scale."""
    g = cuda.Generator(device="cuda")
    g.manual_seed(seed)
    a = cuda.randn(M, K, generator=g, device="cuda") * a_std
    amax = cuda.zeros(1, dtype=cuda.float32, device="cuda")
    tb.absmax(a, a.numel(), amax)
    scale = float(np.float32(FMAX[fmt]) / np.float32(float(amax.item())))
    A = cuda.empty(tb.stored_bytes(fmt, M * K), dtype=cuda.uint8, device="cuda")
    tb.quantize(fmt, a, A, M * K, scale=scale)
    del a
    g.manual_seed(seed + 1)
    B = cuda.randn(N, K, generator=g, device="cuda").half()
    return A, B, float(np.float32(1.0) / np.float32(scale))


def bands(M):
    mid = (M // 2) // 128 * 128
    return [(100, 164), (mid - 28, mid + 36), (M - 48, M)]


def host_rows(A, fmt, K, r0, r1):
    w = tb_row_bytes(fmt, K)
    return A[r0 * w:r1 * w].cpu().numpy().reshape(r1 - r0, w)


def tb_row_bytes(fmt, K):
    return K // 2 if fmt == O.E2M1 else K


def check_bands(cuda, got, A, B16h, fmt, M, N, K, alpha, out_f16=False):
    """`got`: device D; the bands are copied to the host and compared."""
    worst = 0.0
    iv = cuda.int16 if out_f16 else cuda.int32
    for r0, r1 in bands(M):
        want = O.gemm(fmt, host_rows(A, fmt, K, r0, r1), O.F16, B16h, r1 - r0, N, K, alpha=alpha, out_f16=out_f16)
        g = got[r0:r1].view(iv).cpu().numpy().view(np.uint16 if out_f16 else np.float32)
        if out_f16:
            g, want = O.f16_bits_to_f32(g), O.f16_bits_to_f32(want)
        assert np.all(np.isfinite(g)), f"non-finite outputs in rows {r0}-{r1}"
        err = O.rel_frob(g, want)
        assert err <= TOL, f"rows {r0}-{r1}: rel-Frobenius {err:.3e} > {TOL}"
        worst = max(worst, err)
    return worst


def run_three(cuda, tb, fmt, A, B, M, N, K, alpha, out):
    """Fused with workspace, fused without: (D_ws, D_one, D_one == decode +
    FP16 GEMM bit for bit, D_ws == D_one bit for bit, workspace bytes,
    relative Frobenius difference of D_one and decode + FP16 GEMM)."""
    odt = cuda.float16 if out == tb.Out.F16 else cuda.float32
    wsb = tb.fused_workspace_bytes(fmt, M, N, K)
    ws = cuda.empty(max(wsb, 1), dtype=cuda.uint8, device="cuda")
    D_ws = cuda.empty(M, N, dtype=odt, device="cuda")
    D_one = cuda.empty(M, N, dtype=odt, device="cuda")
    D_unf = cuda.empty(M, N, dtype=odt, device="cuda")
    tb.gemm_fused(fmt, A, B, D_ws, M, N, K, out=out, alpha=alpha, workspace=ws, workspace_bytes=wsb)
    tb.gemm_fused(fmt, A, B, D_one, M, N, K, out=out, alpha=alpha)
    A16 = cuda.empty(M * K, dtype=cuda.float16, device="cuda")
    tb.decode(fmt, A, A16, M * K)
    tb.gemm_f16(A16, B, D_unf, M, N, K, out=out, alpha=alpha)
    cuda.cuda.synchronize()
    assert tb.device_error() == 0
    iv = cuda.int16 if out == tb.Out.F16 else cuda.int32
    same = bool(cuda.equal(D_one.view(iv), D_unf.view(iv)))
    ws_same = bool(cuda.equal(D_one.view(iv), D_ws.view(iv)))
    diff = float(cuda.linalg.norm(D_one.double() - D_unf.double()) / cuda.linalg.norm(D_unf.double()))
    del D_unf, A16
    return D_ws, D_one, same, ws_same, wsb, diff


_W = {}


def mlp_weight(cuda, tb, fmt, M, K):
    key = (fmt, M, K)
    if key not in _W:
        _W.clear()
        _W[key] = device_operands(cuda, tb, fmt, M, 1, K, 0.02, seed=M + K + fmt)[::2]
    return _W[key]


@pytest.mark.parametrize("tokens", [1, 16, 128, 2048])
@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("M,K", [(14336, 4096), (4096, 14336)])
def test_mlp_shapes_full_size(tb, cuda, M, K, fmt, tokens):
    A, alpha = mlp_weight(cuda, tb, fmt, M, K)
    N = tokens
    g = cuda.Generator(device="cuda")
    g.manual_seed(1000 + N)
    B = cuda.randn(N, K, generator=g, device="cuda").half()
    d_ws, d_one, same, ws_same, wsb, diff = run_three(cuda, tb, fmt, A, B, M, N, K, alpha, tb.Out.F32)
    B16h = B.view(cuda.int16).cpu().numpy().view(np.uint16)
    check_bands(cuda, d_one, A, B16h, fmt, M, N, K, alpha)
    if N <= 128:
        assert diff <= 1e-4, f"fused and decode + FP16 GEMM differ by {diff:.3e}"
    else:
        assert same, "fused (unsplit) and decode + FP16 GEMM differ"
    if wsb:
        check_bands(cuda, d_ws, A, B16h, fmt, M, N, K, alpha)
    else:
        assert ws_same


def test_fp4_8192_cube_f16_out(tb, cuda):
    n = 8192
    A, B, alpha = device_operands(cuda, tb, O.E2M1, n, n, n, 1.0, seed=8192)
    d_ws, d_one, same, ws_same, wsb, _ = run_three(cuda, tb, O.E2M1, A, B, n, n, n, alpha, tb.Out.F16)
    assert wsb == 0 and ws_same
    assert same, "fused and decode + FP16 GEMM differ"
    B16h = B.view(cuda.int16).cpu().numpy().view(np.uint16)
    check_bands(cuda, d_one, A, B16h, O.E2M1, n, n, n, alpha, out_f16=True)


def test_sharded_config_on_one_gpu(tb, cuda):
    """The 16384 x 53248 E4M3 weight as 53248 output rows, K = 16384, 8192
    FP16 tokens, FP16 out: the single-GPU product the sharded runs must
    reproduce bit for bit (tests/test_sharded_gpu.py)."""
    M, N, K = 53248, 8192, 16384
    A, B, alpha = device_operands(cuda, tb, O.E4M3, M, N, K, 0.02, seed=5)
    d_ws, d_one, same, ws_same, wsb, _ = run_three(cuda, tb, O.E4M3, A, B, M, N, K, alpha, tb.Out.F16)
    assert wsb == 0 and ws_same
    assert same, "fused and decode + FP16 GEMM differ"
    B16h = B.view(cuda.int16).cpu().numpy().view(np.uint16)
    check_bands(cuda, d_one, A, B16h, O.E4M3, M, N, K, alpha, out_f16=True)
