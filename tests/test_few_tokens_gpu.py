"""The few-token fused GEMM (N <= 16: the weight-streaming kernel with the
decoded weights in tensor memory) against the oracle and against
decode-kernel-then-GEMM, for every stored weight format.

Shapes cover ragged M (rows past M in the last 128-row tile), 1 to 16
tokens, and K whose last k-block or raw stage is partial, down to K = 32;
a long K gives each TMEM slot many ring phases.  Tolerances: relative
Frobenius error <= 1e-3 against the oracle (decode -> FP16 -> FP32 sums),
<= 1e-4 against the decode kernel followed by the FP16 GEMM (the MMA rounds
its FP32 accumulation differently with A in tensor memory).  run_fused also
checks that nothing is written past the end of D.
"""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev
from test_gemm_gpu import make_operands, run_fused, run_unfused, check

pytestmark = pytest.mark.gpu

FORMATS = [O.E4M3, O.E5M2, O.E2M1, O.E2M1_UNPACKED, O.BF16, O.TF32]

# (M, N, K); every K is valid for packed FP4 (K % 32 == 0).
SHAPES = [
    (37, 1, 96),        # one partial tile, K of one and a half k-blocks
    (1000, 5, 512),     # 5 tokens, rows past M in the last tile
    (300, 9, 1056),     # 9 tokens, a partial last round
    (4100, 16, 4096),   # 16 tokens, more tiles than SMs, ragged M
    (65, 16, 32),       # K of half a k-block
    (512, 12, 14336),   # long K: many ring phases per TMEM slot
]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_few_tokens_vs_oracle_and_unfused(tb, cuda, fmt, M, N, K):
    A, B16, alpha = make_operands(fmt, M, N, K, seed=fmt * 31 + N)
    got = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha)
    check(got, O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha))
    unfused = run_unfused(tb, cuda, fmt, A, B16, M, N, K, alpha)
    diff = O.rel_frob(got, unfused)
    assert diff <= 1e-4, f"fused and decode + FP16 GEMM differ by {diff:.3e}"


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1, O.BF16])
def test_few_tokens_f16_out(tb, cuda, fmt):
    M, N, K = 2000, 16, 2048
    A, B16, alpha = make_operands(fmt, M, N, K, seed=fmt + 5)
    got = run_fused(tb, cuda, fmt, A, B16, M, N, K, alpha, out=tb.Out.F16)
    want = O.f16_bits_to_f32(O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha, out_f16=True))
    check(got, want)


def test_few_tokens_every_e4m3_code(tb, cuda):
    """Weights drawn from all 254 non-NaN E4M3 codes (subnormals, which the
    reference flushes to zero, and the largest magnitudes included); one row
    then gets a NaN code, which must make that row of D NaN and no other."""
    M, N, K = 96, 16, 1024
    rng = np.random.default_rng(3)
    codes = np.array([c for c in range(256) if c & 0x7F != 0x7F], dtype=np.uint8)
    A = rng.choice(codes, size=(M, K)).astype(np.uint8)
    B16 = O.f32_to_f16_bits(O.uniform(4, (N, K))).reshape(N, K)
    got = run_fused(tb, cuda, O.E4M3, A, B16, M, N, K, 1.0)
    check(got, O.gemm(O.E4M3, A, O.F16, B16, M, N, K, alpha=1.0))
    A[40, 517] = 0xFF
    got = run_fused(tb, cuda, O.E4M3, A, B16, M, N, K, 1.0)
    assert np.all(np.isnan(got[40]))
    rest = np.delete(got, 40, axis=0)
    assert np.all(np.isfinite(rest))
    check(rest, np.delete(O.gemm(O.E4M3, A, O.F16, B16, M, N, K, alpha=1.0), 40, axis=0))


def test_few_tokens_back_to_back_chain(tb, cuda):
    """Two dependent launches on one stream: the second GEMM's activations are
    the first one's FP16 output (transposed to [N x K] by a torch kernel in
    between), so the second must wait for the first before reading them.  The
    result must match the oracle applied twice."""
    K, N = 1024, 16
    A, B16, alpha = make_operands(O.E4M3, K, N, K, seed=9)
    dA, dB = to_dev(cuda, A), to_dev(cuda, B16)
    d1 = cuda.empty(K, N, dtype=cuda.float16, device="cuda")
    tb.gemm_fused(O.E4M3, dA, dB, d1, K, N, K, out=tb.Out.F16, alpha=alpha)
    x2 = d1.t().contiguous()
    d2 = cuda.empty(K, N, dtype=cuda.float16, device="cuda")
    tb.gemm_fused(O.E4M3, dA, x2, d2, K, N, K, out=tb.Out.F16, alpha=alpha)
    cuda.cuda.synchronize()
    want1 = O.gemm(O.E4M3, A, O.F16, B16, K, N, K, alpha=alpha, out_f16=True)  # FP16 bits [K x N]
    x2h = np.ascontiguousarray(want1.reshape(K, N).T)
    want2 = O.f16_bits_to_f32(O.gemm(O.E4M3, A, O.F16, x2h, K, N, K, alpha=alpha, out_f16=True))
    got2 = d2.float().cpu().numpy()
    check(got2, want2, tol=2e-3)
