"""Block-scaled FP4 decode on the GPU (tb_decode_nvfp4): bit-exact against the
oracle on every (code byte, scale byte) pair, on misaligned buffers and on
sizes around the streamer's chunking; then block-scaled weights through the
FP16 GEMM with the per-tensor scale in alpha, against the oracle's GEMM."""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev, empty_dev, from_dev
from test_nvfp4_oracle import all_pairs

pytestmark = pytest.mark.gpu


def run(tb, torch, q, scales, n, src_off=0, dst_off=0):
    dq = empty_dev(torch, q.size + 64)
    dq[src_off: src_off + q.size].copy_(torch.from_numpy(q.copy()))
    ds = to_dev(torch, scales, pad=16)
    d = empty_dev(torch, 2 * n + 64)
    tb.decode_nvfp4(dq.data_ptr() + src_off, ds, d.data_ptr() + 2 * dst_off, n)
    torch.cuda.synchronize()
    return from_dev(d, np.uint8)[2 * dst_off: 2 * dst_off + 2 * n].view(np.uint16)


def test_every_code_scale_pair(tb, cuda):
    q, scales, n = all_pairs()
    np.testing.assert_array_equal(run(tb, cuda, q, scales, n), O.decode_nvfp4(q, scales, n))


@pytest.mark.parametrize("src_off,dst_off", [(1, 0), (0, 1), (3, 5)])
def test_misaligned_buffers(tb, cuda, src_off, dst_off):
    q, scales, n = all_pairs()
    q, scales, n = q[:4096], scales[:512], 8192
    np.testing.assert_array_equal(run(tb, cuda, q, scales, n, src_off, dst_off), O.decode_nvfp4(q, scales, n))


# one block; one warp chunk (32 lanes x 16 items x 8 values) and one block
# past it; a grid stride and a ragged remainder
@pytest.mark.parametrize("n", [16, 4096, 4112, 16 * 77777])
def test_sizes(tb, cuda, n):
    rng = np.random.default_rng(n)
    q = rng.integers(0, 256, size=n // 2, dtype=np.uint8)
    scales = rng.integers(0, 256, size=n // 16, dtype=np.uint8)
    d = run(tb, cuda, q, scales, n)
    np.testing.assert_array_equal(d, O.decode_nvfp4(q, scales, n))


def test_output_past_n_untouched(tb, cuda):
    q, scales, n = all_pairs()
    q, scales, n = q[:64], scales[:8], 128
    dq, ds = to_dev(cuda, q), to_dev(cuda, scales)
    d = empty_dev(cuda, 2 * n + 256, fill=0x5A)
    tb.decode_nvfp4(dq, ds, d, n)
    cuda.cuda.synchronize()
    tail = from_dev(d, np.uint8)[2 * n:]
    assert np.all(tail == 0x5A)


@pytest.mark.parametrize("M,N,K", [(256, 128, 512), (1000, 48, 2048)])
def test_block_scaled_weights_through_gemm(tb, cuda, M, N, K):
    """W [M x K] quantized with per-16 E4M3 scales and a per-tensor FP32 scale
    g; decode on the device, then D = g * W16 @ X^T on the FP16 GEMM.  Within
    1e-3 relative Frobenius error of the oracle's FP32 GEMM over the same
    decoded values, and a quantization error well under per-tensor FP4's on
    rows of very different magnitude."""
    W = O.normal(21, (M, K)) * np.exp(2 * O.normal(22, (M, 1)))
    X = O.normal(23, (N, K))
    q, s, g = O.quantize_nvfp4(W)
    X16 = O.f32_to_f16_bits(X)
    dq, ds, dX = to_dev(cuda, q), to_dev(cuda, s), to_dev(cuda, X16)
    W16 = empty_dev(cuda, 2 * M * K)
    tb.decode_nvfp4(dq, ds, W16, M * K)
    dD = empty_dev(cuda, 4 * M * N)
    tb.gemm_f16(W16, dX, dD, M, N, K, alpha=g)
    cuda.cuda.synchronize()
    got = from_dev(dD, np.float32).reshape(M, N)
    Wd = O.decode_nvfp4(q, s, M * K).reshape(M, K)
    ref = O.gemm(O.F16, Wd, O.F16, X16, M, N, K, alpha=g)
    assert O.rel_frob(got, ref) < 1e-3
    exact = W.astype(np.float64) @ O.f16_bits_to_f32(X16).astype(np.float64).T
    sc = O.per_tensor_scale(W, O.E2M1)
    Wt = O.f16_bits_to_f32(O.decode(O.E2M1, O.quantize(O.E2M1, W, sc), M * K)).reshape(M, K) / sc
    per_tensor = Wt.astype(np.float64) @ O.f16_bits_to_f32(X16).astype(np.float64).T
    assert O.rel_frob(got, exact) < 0.5 * O.rel_frob(per_tensor, exact)
