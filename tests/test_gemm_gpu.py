"""tcgen05 GEMMs on the GPU against the oracle (decode -> FP16 -> FP32 sums).

Tolerance: relative Frobenius error <= 1e-3 against the oracle on the same
inputs (the bound the decode+GEMM path is held to); both sides compute exact
FP32 products of FP16 values and differ only in summation order, so the
observed errors are ~1e-6.
"""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev, empty_dev, from_dev

pytestmark = pytest.mark.gpu

TOL = 1e-3


def make_operands(fmt, M, N, K, seed=0, dist="normal"):
    """Weight A [M x K] quantized to fmt with a per-tensor scale, activations
    B [N x K] FP16.  Returns (A stored, B16 bits, alpha = 1/scale)."""
    if dist == "normal":
        a = O.normal(seed, (M, K), 0.02)
        b = O.normal(seed + 1, (N, K), 1.0)
    else:
        a = O.uniform(seed, (M, K))
        b = O.uniform(seed + 1, (N, K))
    s = O.per_tensor_scale(a, fmt)
    A = O.quantize(fmt, a, s) if fmt != O.F16 else O.f32_to_f16_bits(a).reshape(M, K)
    B16 = O.f32_to_f16_bits(b).reshape(N, K)
    return A, B16, float(np.float32(1.0) / np.float32(s))


def run_fused(tb, torch, fmt, A, B16, M, N, K, alpha, out=None, force_ws=True):
    out = out if out is not None else tb.Out.F32
    dA, dB = to_dev(torch, A), to_dev(torch, B16)
    esz = 2 if out == tb.Out.F16 else 4
    dD = empty_dev(torch, M * N * esz + 256)
    ws_bytes = tb.fused_workspace_bytes(fmt, M, N, K) if force_ws else 0
    ws = empty_dev(torch, ws_bytes) if ws_bytes else None
    tb.gemm_fused(fmt, dA, dB, dD, M, N, K, out=out, alpha=alpha, workspace=ws, workspace_bytes=ws_bytes)
    torch.cuda.synchronize()
    raw = from_dev(dD, np.uint8)
    assert np.all(raw[M * N * esz:] == 0xA5), "wrote past the end of D"
    body = raw[: M * N * esz]
    if out == tb.Out.F16:
        return O.f16_bits_to_f32(body.view(np.uint16)).reshape(M, N)
    return body.view(np.float32).reshape(M, N)


def check(got, want, tol=TOL):
    err = O.rel_frob(got, want)
    assert np.all(np.isfinite(got)), "non-finite outputs"
    assert err <= tol, f"rel-Frobenius {err:.3e} > {tol}"
    return err


SHAPES = [
    (2500, 2000, 128),   # pair tiles with ragged M and N
    (256, 256, 256),     # the 256^3 configuration
    (128, 256, 64),      # one tile, one k-block
    (200, 72, 48),       # ragged M/N, K not a multiple of 64
    (384, 520, 320),     # several tiles, ragged N
    (1000, 1, 512),      # one token
    (640, 16, 1024),     # 16 tokens
    (512, 128, 4096),    # 128 tokens, long K (split-K candidates)
    (130, 300, 96),
    (256, 16, 16384),    # one tile column, 256 k-blocks: many ring phases per slot
    (512, 40, 2048),     # 17..64 tokens
    (1000, 64, 1536),
    (300, 24, 4160),     # ragged M, K with a partial raw stage
    (256, 8, 80),
    (300, 100, 1056),    # 65..128 tokens (128-column narrow tiles), partial last round
    (1000, 128, 4160),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_f16(tb, cuda, M, N, K):
    A, B16, _ = make_operands(O.F16, M, N, K, seed=M + N + K, dist="uniform")
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_f16(dA, dB, dD, M, N, K)
    cuda.cuda.synchronize()
    got = from_dev(dD, np.float32).reshape(M, N)
    check(got, O.gemm(O.F16, A, O.F16, B16, M, N, K))


@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2, O.E2M1, O.E2M1_UNPACKED, O.BF16, O.TF32])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_fused(tb, cuda, fmt, M, N, K):
    if fmt == O.E2M1 and K % 32:
        pytest.skip("packed FP4 needs K % 32 == 0")
    A, B16, alpha = make_operands(fmt, M, N, K, seed=fmt * 7 + M)
    got = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha)
    check(got, O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha))


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_gemm_fused_f16_out(tb, cuda, fmt):
    M, N, K = 384, 264, 512
    A, B16, alpha = make_operands(fmt, M, N, K, seed=3)
    got = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, out=tb.Out.F16)
    want = O.f16_bits_to_f32(O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha, out_f16=True))
    check(got, want)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_gemm_fused_without_workspace(tb, cuda, fmt):
    """Short-and-wide shapes split K when given a workspace and still run
    (unsplit) without one; both agree with the oracle."""
    M, N, K = 256, 16, 8192
    A, B16, alpha = make_operands(fmt, M, N, K, seed=4)
    assert tb.fused_workspace_bytes(fmt, M, N, K) > 0
    want = O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha)
    check(run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, force_ws=True), want)
    check(run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, force_ws=False), want)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1, O.BF16, O.TF32])
def test_fused_equals_unfused_bitwise(tb, cuda, fmt):
    """Decode-in-shared-memory and decode-kernel-then-GEMM run the same MMAs in
    the same order: identical bits (the reference checks the same property,
    bench/bench_fused.cu:85-87)."""
    M, N, K = 512, 384, 1024
    A, B16, alpha = make_operands(fmt, M, N, K, seed=6)
    fused = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, force_ws=False)
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    A16 = empty_dev(cuda, M * K * 2)
    tb.decode(fmt, dA, A16, M * K)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_f16(A16, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    unfused = from_dev(dD, np.float32).reshape(M, N)
    np.testing.assert_array_equal(fused.view(np.uint32), unfused.view(np.uint32))


# Shapes the launcher gives to the SM-pair kernel (256 x 512 pair tiles, each
# CTA decoding its own 128 rows; chosen when at least 512 columns need no
# split and no more waves than the one-CTA kernel): ragged M and N inside a
# pair tile (1900 rows leave the second CTA of the last tile row no rows;
# 3700 columns leave the last tile's second half none), K with a partial k-block
# or a partial raw stage, several tiles per cluster.  Bit-identical to
# decode-then-GEMM everywhere, and against the oracle on bands of rows that
# straddle tile boundaries and on the last rows.
PAIR_SHAPES = [(1900, 3700, 320), (2048, 4096, 96), (1024, 8192, 4160)]


@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2, O.E2M1, O.E2M1_UNPACKED, O.BF16, O.TF32])
@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
def test_fused_pair_tiles(tb, cuda, fmt, M, N, K):
    A, B16, alpha = make_operands(fmt, M, N, K, seed=fmt * 5 + N)
    got = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, force_ws=False)
    unfused = run_unfused(tb, cuda, fmt, A, B16, M, N, K, alpha)
    np.testing.assert_array_equal(got.view(np.uint32), unfused.view(np.uint32))
    for rows in ((100, 164), (230, 290), (M - 40, M)):
        check(got[rows[0]:rows[1]], O.gemm(fmt, A, O.F16, B16, M, N, K, rows=rows, alpha=alpha))


def test_narrow_chain_dependencies(tb, cuda):
    """Back-to-back narrow GEMMs on one stream start before their predecessor
    has finished (programmatic dependent launch) and stream their weights
    early, but must wait for it before reading activations and before storing:
    GEMM 2 reads GEMM 1's FP16 output as its activations, and GEMM 3 then
    overwrites that buffer while GEMM 2 may still be streaming.  Each result
    must equal, bit for bit, the same GEMM run alone."""
    M1, N1, K1 = 1024, 64, 512        # D1: 1024 x 64 FP16 = B2 viewed as 16 x 4096
    M2, N2, K2 = 2048, 16, 4096
    A1, B1, al1 = make_operands(O.E4M3, M1, N1, K1, seed=31)
    A2, _, al2 = make_operands(O.E2M1, M2, N2, K2, seed=32)
    _, B3, _ = make_operands(O.E4M3, M1, N1, K1, seed=33)
    dA1, dB1, dA2, dB3 = to_dev(cuda, A1), to_dev(cuda, B1), to_dev(cuda, A2), to_dev(cuda, B3)
    X = empty_dev(cuda, M1 * N1 * 2)
    D2 = empty_dev(cuda, M2 * N2 * 4)
    F16 = tb.Out.F16

    def g1(out):
        tb.gemm_fused(O.E4M3, dA1, dB1, out, M1, N1, K1, out=F16, alpha=al1)

    def g2(b, out):
        tb.gemm_fused(O.E2M1, dA2, b, out, M2, N2, K2, alpha=al2)

    def g3(out):
        tb.gemm_fused(O.E4M3, dA1, dB3, out, M1, N1, K1, out=F16, alpha=al1)

    # each GEMM alone
    R1, R2, R3 = empty_dev(cuda, M1 * N1 * 2), empty_dev(cuda, M2 * N2 * 4), empty_dev(cuda, M1 * N1 * 2)
    g1(R1); cuda.cuda.synchronize()
    g2(R1, R2); cuda.cuda.synchronize()
    g3(R3); cuda.cuda.synchronize()
    want2, want3 = from_dev(R2, np.uint32), from_dev(R3, np.uint16)
    check(want2.view(np.float32).reshape(M2, N2),
          O.gemm(O.E2M1, A2, O.F16, from_dev(R1, np.uint16).reshape(N2, K2), M2, N2, K2, alpha=al2))
    for _ in range(5):
        X.fill_(0xA5)
        D2.fill_(0xA5)
        g1(X)
        g2(X, D2)
        g3(X)
        cuda.cuda.synchronize()
        np.testing.assert_array_equal(from_dev(D2, np.uint32), want2)
        np.testing.assert_array_equal(from_dev(X, np.uint16), want3)


def test_narrow_chain_tf32_weights_from_previous_output(tb, cuda):
    """A narrow GEMM with TF32 weights that are the previous narrow GEMM's FP32
    output: its raw-weight stream must wait for that GEMM (BF16 and TF32
    weights are read only after the dependency wait)."""
    M1, N1, K1 = 1024, 64, 512      # D1: 1024 x 64 FP32 = A2 viewed as 128 x 512 TF32 words
    M2, N2, K2 = 128, 16, 512
    A1, B1, al1 = make_operands(O.E4M3, M1, N1, K1, seed=51)
    _, B2, _ = make_operands(O.E4M3, M2, N2, K2, seed=52)
    dA1, dB1, dB2 = to_dev(cuda, A1), to_dev(cuda, B1), to_dev(cuda, B2)
    X = empty_dev(cuda, M1 * N1 * 4)
    R = empty_dev(cuda, M1 * N1 * 4)
    D2, W2 = empty_dev(cuda, M2 * N2 * 4), empty_dev(cuda, M2 * N2 * 4)
    tb.gemm_fused(O.E4M3, dA1, dB1, R, M1, N1, K1, alpha=al1)
    cuda.cuda.synchronize()
    tb.gemm_fused(O.TF32, R, dB2, W2, M2, N2, K2)
    cuda.cuda.synchronize()
    want = from_dev(W2, np.uint32)
    check(want.view(np.float32).reshape(M2, N2),
          O.gemm(O.TF32, from_dev(R, np.uint32).reshape(M2, K2), O.F16, B2, M2, N2, K2))
    for _ in range(5):
        X.fill_(0xA5)
        D2.fill_(0xA5)
        tb.gemm_fused(O.E4M3, dA1, dB1, X, M1, N1, K1, alpha=al1)
        tb.gemm_fused(O.TF32, X, dB2, D2, M2, N2, K2)
        cuda.cuda.synchronize()
        np.testing.assert_array_equal(from_dev(D2, np.uint32), want)


def test_narrow_split_chain_shares_workspace(tb, cuda):
    """Split-K narrow GEMMs back to back with one workspace: the second
    GEMM's partials overwrite the workspace the first one's reduction reads,
    and both the GEMM and the reduction start early (programmatic dependent
    launch).  Each result must equal the same GEMM run alone, bit for bit."""
    M, N, K = 1024, 16, 8192
    A1, B1, al1 = make_operands(O.E4M3, M, N, K, seed=41)
    A2, B2, al2 = make_operands(O.E4M3, M, N, K, seed=42)
    ws_bytes = tb.fused_workspace_bytes(O.E4M3, M, N, K)
    assert ws_bytes > 0
    ws = empty_dev(cuda, ws_bytes)
    dA1, dB1, dA2, dB2 = to_dev(cuda, A1), to_dev(cuda, B1), to_dev(cuda, A2), to_dev(cuda, B2)
    D1, D2 = empty_dev(cuda, M * N * 4), empty_dev(cuda, M * N * 4)

    def run(a, b, d, al):
        tb.gemm_fused(O.E4M3, a, b, d, M, N, K, alpha=al, workspace=ws, workspace_bytes=ws_bytes)

    run(dA1, dB1, D1, al1); cuda.cuda.synchronize()
    want1 = from_dev(D1, np.uint32)
    run(dA2, dB2, D2, al2); cuda.cuda.synchronize()
    want2 = from_dev(D2, np.uint32)
    check(want1.view(np.float32).reshape(M, N), O.gemm(O.E4M3, A1, O.F16, B1, M, N, K, alpha=al1))
    for _ in range(5):
        D1.fill_(0xA5)
        D2.fill_(0xA5)
        run(dA1, dB1, D1, al1)
        run(dA2, dB2, D2, al2)
        run(dA1, dB1, D1, al1)
        cuda.cuda.synchronize()
        np.testing.assert_array_equal(from_dev(D1, np.uint32), want1)
        np.testing.assert_array_equal(from_dev(D2, np.uint32), want2)


def kernels_launched(cuda, fn):
    """Names of the kernels `fn` launches (CUPTI trace through torch.profiler)."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
        fn()
        cuda.cuda.synchronize()
    return {e.name for e in prof.events()}


@pytest.mark.parametrize("M,N,K,pair", [(1900, 3700, 320, True), (2048, 4096, 96, True), (1024, 8192, 4160, True),
                                        (4096, 2304, 1024, False), (300, 600, 640, False)])
def test_fused_pair_choice(tb, cuda, M, N, K, pair):
    """The pair-tile shapes above do run on the SM-pair kernel, and shapes
    whose pair tiles would take more waves stay on the one-CTA kernel."""
    fmt = O.E2M1
    A, B16, alpha = make_operands(fmt, M, N, K, seed=1)
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    dD = empty_dev(cuda, M * N * 4)
    names = kernels_launched(cuda, lambda: tb.gemm_fused(fmt, dA, dB, dD, M, N, K, alpha=alpha))
    assert any("k_fused_pair" in n for n in names) == pair, names


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1, O.TF32])
def test_fused_pair_tiles_f16_out(tb, cuda, fmt):
    M, N, K = 1900, 3700, 320
    A, B16, alpha = make_operands(fmt, M, N, K, seed=fmt * 3)
    got = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, out=tb.Out.F16, force_ws=False)
    for rows in ((100, 164), (M - 40, M)):
        want = O.f16_bits_to_f32(O.gemm(fmt, A, O.F16, B16, M, N, K, rows=rows, alpha=alpha, out_f16=True))
        check(got[rows[0]:rows[1]], want)


def run_unfused(tb, cuda, fmt, A, B16, M, N, K, alpha):
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    A16 = empty_dev(cuda, M * K * 2)
    tb.decode(fmt, dA, A16, M * K)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_f16(A16, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    return from_dev(dD, np.float32).reshape(M, N)


# Persistent CTAs walk several output tiles each once the tile count exceeds the
# SM count (148 on B200): these shapes give every CTA 2 to 4 tiles, so the raw
# and operand rings wrap across tile boundaries with TMA refills that hit L2.
MULTI_TILE = [(4096, 4096, 4096), (2048, 4096, 512), (4096, 2304, 1024), (1024, 8192, 256), (4096, 8192, 192)]


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1, O.BF16, O.TF32])
@pytest.mark.parametrize("M,N,K", MULTI_TILE)
def test_fused_multi_tile_per_cta(tb, cuda, fmt, M, N, K):
    """Fused equals decode-then-GEMM bit for bit on every tile, and a band of
    rows from each tile row agrees with the oracle."""
    A, B16, alpha = make_operands(fmt, M, N, K, seed=fmt * 13 + K)
    fused = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, force_ws=False)
    unfused = run_unfused(tb, cuda, fmt, A, B16, M, N, K, alpha)
    bad = np.argwhere(fused.view(np.uint32) != unfused.view(np.uint32))
    assert bad.size == 0, f"{len(bad)} mismatches, first tiles {sorted({(r // 128, c // 256) for r, c in bad[:64]})}"
    for r0 in range(0, M, 1024):
        rows = (r0 + 100, r0 + 164)  # straddles the boundary of two 128-row tiles
        want = O.gemm(fmt, A, O.F16, B16, M, N, K, rows=rows, alpha=alpha)
        check(fused[rows[0]:rows[1]], want)


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (384, 200, 640), (128, 16, 2048)])
def test_gemm_native_e4m3(tb, cuda, M, N, K):
    a = O.normal(10, (M, K), 0.02)
    b = O.normal(11, (N, K), 1.0)
    sa, sb = O.per_tensor_scale(a, O.E4M3), O.per_tensor_scale(b, O.E4M3)
    A, B = O.quantize(O.E4M3, a, sa), O.quantize(O.E4M3, b, sb)
    alpha = float(np.float32(1.0) / (np.float32(sa) * np.float32(sb)))
    dA, dB = to_dev(cuda, A), to_dev(cuda, B)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_native(tb.Format.E4M3, dA, tb.Format.E4M3, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    got = from_dev(dD, np.float32).reshape(M, N)
    check(got, O.gemm(O.E4M3, A, O.E4M3, B, M, N, K, alpha=alpha))


NATIVE_PAIRS = [(O.E2M1_HW, O.E2M1_HW), (O.E4M3, O.E2M1_HW), (O.E2M1_HW, O.E4M3), (O.E5M2, O.E5M2),
                (O.E4M3, O.E5M2)]


@pytest.mark.parametrize("fa,fb", NATIVE_PAIRS)
@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (384, 200, 640), (128, 16, 2048), (1000, 72, 96),
                                   (2500, 2000, 128)])  # pair tiles, ragged M and N
def test_gemm_native_formats(tb, cuda, fa, fb, M, N, K):
    """qA @ qB on kind::f8f6f4 for FP4 (16U4_ALIGN16B TMA expansion), E5M2
    and mixed pairs, each operand with its own per-tensor scale."""
    if O.E2M1_HW in (fa, fb) and K % 128:
        pytest.skip("native FP4 needs K % 128 == 0")
    a = O.normal(12, (M, K), 0.02)
    b = O.normal(13, (N, K), 1.0)
    sa, sb = O.per_tensor_scale(a, fa), O.per_tensor_scale(b, fb)
    A, B = O.quantize(fa, a, sa), O.quantize(fb, b, sb)
    alpha = float(np.float32(1.0) / (np.float32(sa) * np.float32(sb)))
    dA, dB = to_dev(cuda, A), to_dev(cuda, B)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_native(fa, dA, fb, dB, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    got = from_dev(dD, np.float32).reshape(M, N)
    check(got, O.gemm(fa, A, fb, B, M, N, K, alpha=alpha))


def test_native_fp4_matches_fused_after_repack(tb, cuda):
    """Reference-packed FP4 weights repacked to the tensor-core nibble order
    give the same product natively as the fused decode path does with FP16
    activations that hold exactly the FP4 values."""
    M, N, K = 512, 256, 1024
    a, b = O.normal(14, (M, K), 1.0), O.normal(15, (N, K), 1.0)
    sa, sb = O.per_tensor_scale(a, O.E2M1), O.per_tensor_scale(b, O.E2M1)
    A_ref, B_ref = O.quantize(O.E2M1, a, sa), O.quantize(O.E2M1, b, sb)
    dA, dB = to_dev(cuda, A_ref), to_dev(cuda, B_ref)
    dA_hw, dB_hw = empty_dev(cuda, A_ref.nbytes), empty_dev(cuda, B_ref.nbytes)
    tb.fp4_repack_hw(dA, dA_hw, A_ref.nbytes)
    tb.fp4_repack_hw(dB, dB_hw, B_ref.nbytes)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_native(tb.Format.E2M1_HW, dA_hw, tb.Format.E2M1_HW, dB_hw, dD, M, N, K)
    B16 = empty_dev(cuda, N * K * 2)
    tb.decode(tb.Format.E2M1, dB, B16, N * K)
    dF = empty_dev(cuda, M * N * 4)
    tb.gemm_fused(tb.Format.E2M1, dA, B16, dF, M, N, K)
    cuda.cuda.synchronize()
    native = from_dev(dD, np.float32).reshape(M, N)
    fused = from_dev(dF, np.float32).reshape(M, N)
    check(native, fused, tol=1e-6)


@pytest.mark.parametrize("M,N,K,codes", [(512, 512, 512, "quantized"), (200, 72, 80, "all"),
                                         (384, 136, 1040, "all")])
def test_fp8_fused_fp16_mirror(tb, cuda, M, N, K, codes):
    """tb_gemm_fp8_fused_fp16 mirrors gemm_fp8_fused_fp16: both operands E4M3,
    B given [K x N] row-major as the reference reads it.  It runs on the FP8
    tensor cores after flushing the subnormal codes the way the reference
    decoder does; "all" draws both operands from every non-NaN code
    (subnormals and the largest magnitudes included), on ragged shapes whose
    B transpose has partial 64 x 64 tiles."""
    if codes == "quantized":
        a, b = O.uniform(20, (M, K)), O.uniform(21, (K, N))
        A, Bkn = O.quantize(O.E4M3, a), O.quantize(O.E4M3, b)
    else:
        rng = np.random.default_rng(M + N + K)
        pool = np.array([c for c in range(256) if c & 0x7F != 0x7F], dtype=np.uint8)
        A = rng.choice(pool, size=(M, K)).astype(np.uint8)
        Bkn = rng.choice(pool, size=(K, N)).astype(np.uint8)
    dA, dB = to_dev(cuda, A), to_dev(cuda, Bkn)
    ws_bytes = tb.lib().tb_gemm_fp8_fused_workspace(M, N, K)
    ws = empty_dev(cuda, ws_bytes)
    dD = empty_dev(cuda, M * N * 4)
    tb.call("tb_gemm_fp8_fused_fp16", dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), M, N, K, ws.data_ptr(), ws_bytes,
            cuda.cuda.current_stream().cuda_stream)
    cuda.cuda.synchronize()
    got = from_dev(dD, np.float32).reshape(M, N)
    Bnk = np.ascontiguousarray(Bkn.reshape(K, N).T)
    check(got, O.gemm(O.E4M3, A, O.E4M3, Bnk, M, N, K))


def test_no_device_error_word(tb, cuda):
    assert tb.device_error(clear=True) == 0


def test_quantize_then_narrow_gemm_same_stream(tb, cuda):
    """tb_quantize writes the weights and a narrow GEMM reads them on the same
    stream with no host synchronisation, separated as the header asks by one
    kernel launched without programmatic dependent launch (a fill of another
    buffer): every result equals, bit for bit, the same GEMM run after a full
    synchronisation."""
    M, N, K = 2048, 16, 4096
    g = cuda.Generator(device="cuda")
    g.manual_seed(61)
    ws = [cuda.randn(M, K, generator=g, device="cuda") * 0.02 for _ in range(2)]
    B = cuda.randn(N, K, generator=g, device="cuda").half()
    for fmt in (O.E4M3, O.E2M1):
        A = cuda.empty(tb.stored_bytes(fmt, M * K), dtype=cuda.uint8, device="cuda")
        want = []
        for w in ws:
            tb.quantize(fmt, w, A, M * K, scale=64.0)
            cuda.cuda.synchronize()
            D = cuda.empty(M, N, dtype=cuda.float32, device="cuda")
            tb.gemm_fused(fmt, A, B, D, M, N, K, alpha=1.0 / 64)
            cuda.cuda.synchronize()
            want.append(D)
        outs = [cuda.empty(M, N, dtype=cuda.float32, device="cuda") for _ in range(8)]
        sep = cuda.empty(1024, dtype=cuda.float32, device="cuda")
        for i, D in enumerate(outs):
            tb.quantize(fmt, ws[i & 1], A, M * K, scale=64.0)
            sep.fill_(float(i))
            tb.gemm_fused(fmt, A, B, D, M, N, K, alpha=1.0 / 64)
        cuda.cuda.synchronize()
        for i, D in enumerate(outs):
            assert cuda.equal(D.view(cuda.int32), want[i & 1].view(cuda.int32)), (fmt, i)
