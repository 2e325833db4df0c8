"""Block-scaled FP4 GEMM (tb_gemm_nvfp4, tcgen05 kind::mxf4nvf4) against the
oracle: both operands quantized two-level (per-tensor FP32 scale g, one E4M3
scale byte per 16 values, E2M1 codes), decoded exactly by the oracle's
block-scaled decode (oracle_decode_nvfp4, every product an FP16 value), then
an FP32-accumulate GEMM.  Tolerance: relative Frobenius error <= 1e-3."""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev, empty_dev, from_dev

pytestmark = pytest.mark.gpu

TOL = 1e-3


def hw_order(q):
    """Reference packing (first value high) -> tensor-core packing (first value low)."""
    q = np.asarray(q, dtype=np.uint8)
    return ((q & 0x0F) << 4) | (q >> 4)


def operand(seed, rows, K, std=1.0):
    x = O.normal(seed, (rows, K), std)
    q, sc, g = O.quantize_nvfp4(x)
    return q, sc, g


def run(tb, cuda, qa, sa, qb, sb, M, N, K, alpha, out=None):
    out = out if out is not None else tb.Out.F32
    esz = 2 if out == tb.Out.F16 else 4
    dA, dSA, dB, dSB = to_dev(cuda, hw_order(qa)), to_dev(cuda, sa), to_dev(cuda, hw_order(qb)), to_dev(cuda, sb)
    dD = empty_dev(cuda, M * N * esz + 256)
    tb.gemm_nvfp4(dA, dSA, dB, dSB, dD, M, N, K, out=out, alpha=alpha)
    cuda.cuda.synchronize()
    raw = from_dev(dD, np.uint8)
    assert np.all(raw[M * N * esz:] == 0xA5), "wrote past the end of D"
    body = raw[: M * N * esz]
    if out == tb.Out.F16:
        return O.f16_bits_to_f32(body.view(np.uint16)).reshape(M, N)
    return body.view(np.float32).reshape(M, N)


def want(qa, sa, qb, sb, M, N, K, alpha, out_f16=False):
    A16 = O.decode_nvfp4(qa, sa, M * K).reshape(M, K)
    B16 = O.decode_nvfp4(qb, sb, N * K).reshape(N, K)
    w = O.gemm(O.F16, A16, O.F16, B16, M, N, K, alpha=alpha, out_f16=out_f16)
    return O.f16_bits_to_f32(w) if out_f16 else w


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 384, 1024), (300, 200, 512), (128, 16, 256),
                                   (1000, 72, 2048), (2048, 1024, 4096), (520, 1000, 768)])
def test_gemm_nvfp4(tb, cuda, M, N, K):
    qa, sa, ga = operand(M + K, M, K)
    qb, sb, gb = operand(N + K + 1, N, K)
    alpha = float(np.float32(ga) * np.float32(gb))
    got = run(tb, cuda, qa, sa, qb, sb, M, N, K, alpha)
    w = want(qa, sa, qb, sb, M, N, K, alpha)
    assert np.all(np.isfinite(got))
    err = O.rel_frob(got, w)
    assert err <= TOL, f"rel-Frobenius {err:.3e}"


def test_gemm_nvfp4_f16_out(tb, cuda):
    M, N, K = 512, 512, 512
    qa, sa, ga = operand(3, M, K)
    qb, sb, gb = operand(4, N, K)
    alpha = float(np.float32(ga) * np.float32(gb))
    got = run(tb, cuda, qa, sa, qb, sb, M, N, K, alpha, out=tb.Out.F16)
    assert O.rel_frob(got, want(qa, sa, qb, sb, M, N, K, alpha, out_f16=True)) <= TOL


def test_gemm_nvfp4_every_scale_byte(tb, cuda):
    """Every finite UE4M3 scale byte (0x00-0x7E, subnormals included) and every
    E2M1 code: random codes with scale bytes cycling through all 127 values,
    per-row magnitudes as different as the scales make them."""
    M, N, K = 256, 256, 1024
    rng = np.random.default_rng(9)
    qa = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
    qb = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    sa = (np.arange(M * K // 16) % 127).astype(np.uint8).reshape(M, K // 16)
    sb = rng.integers(0x30, 0x48, size=(N, K // 16), dtype=np.uint8)
    got = run(tb, cuda, qa, sa, qb, sb, M, N, K, 1.0)
    w = want(qa, sa, qb, sb, M, N, K, 1.0)
    err = O.rel_frob(got, w)
    assert err <= TOL, f"rel-Frobenius {err:.3e}"


def test_gemm_nvfp4_matches_decode_then_gemm(tb, cuda):
    """Native block-scaled MMA against the exact decode streamer followed by
    the FP16 GEMM on the device, at a size with many tiles per cluster."""
    M, N, K = 2048, 4096, 1024
    qa, sa, ga = operand(21, M, K)
    qb, sb, gb = operand(22, N, K)
    alpha = float(np.float32(ga) * np.float32(gb))
    got = run(tb, cuda, qa, sa, qb, sb, M, N, K, alpha)
    A16, B16 = empty_dev(cuda, M * K * 2), empty_dev(cuda, N * K * 2)
    tb.decode_nvfp4(to_dev(cuda, qa), to_dev(cuda, sa), A16, M * K)
    tb.decode_nvfp4(to_dev(cuda, qb), to_dev(cuda, sb), B16, N * K)
    dD = empty_dev(cuda, M * N * 4)
    tb.gemm_f16(A16, B16, dD, M, N, K, alpha=alpha)
    cuda.cuda.synchronize()
    ref = from_dev(dD, np.float32).reshape(M, N)
    assert O.rel_frob(got, ref) <= 1e-5
    assert tb.device_error() == 0


def test_gemm_nvfp4_rejects(tb, cuda):
    dA = empty_dev(cuda, 1024)
    with pytest.raises(tb.TBError):
        tb.gemm_nvfp4(dA, dA, dA, dA, dA, 16, 16, 128)  # K % 256
