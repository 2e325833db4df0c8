"""The INT8 path on the GPU against the oracle: FP8 E4M3 -> INT8 conversion
(src/gemm.cu:35-41) bit for bit, straight and transposed, and the tcgen05
kind::i8 GEMM (src/gemm.cu:58-70) and the FP8 -> INT8 fused entry
(src/gemm_fused.cu:52-81), whose INT32 results are exact integers and must
equal the oracle's exactly."""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev, empty_dev, from_dev

pytestmark = pytest.mark.gpu

ALL_CODES = np.arange(256, dtype=np.uint8)
SCALES = [float(np.float32(127.0) / np.float32(448.0)), 1.0, 8.0, 1e30, -3.5, 0.0, 0.37]


@pytest.mark.parametrize("scale", SCALES)
def test_decode_all_codes(tb, cuda, scale):
    src = np.tile(ALL_CODES, 9)  # 2304 codes: whole 16-byte items
    d = empty_dev(cuda, src.size)
    tb.decode_e4m3_to_i8(to_dev(cuda, src), d, src.size, scale)
    cuda.cuda.synchronize()
    np.testing.assert_array_equal(from_dev(d, np.int8), O.decode_e4m3_i8(src, scale))


@pytest.mark.parametrize("n,off", [(1, 0), (1003, 0), (4096 + 7, 3), (65536, 1)])
def test_decode_tails_and_misalignment(tb, cuda, n, off):
    rng = np.random.default_rng(n)
    src = rng.integers(0, 256, size=n, dtype=np.uint8)
    scale = float(np.float32(127.0) / np.float32(448.0))
    dsrc = to_dev(cuda, np.concatenate([np.zeros(off, np.uint8), src]))
    d = empty_dev(cuda, n + off)
    tb.decode_e4m3_to_i8(dsrc[off:], d[off:], n, scale)
    cuda.cuda.synchronize()
    got = from_dev(d, np.int8)
    np.testing.assert_array_equal(got[off:], O.decode_e4m3_i8(src, scale))
    assert np.all(got[:off].view(np.uint8) == 0xA5), "wrote before the destination"


@pytest.mark.parametrize("rows,cols", [(64, 32), (100, 33), (4096, 16), (7, 300), (256, 192), (192, 130), (1024, 1024)])
def test_decode_transposed(tb, cuda, rows, cols):
    rng = np.random.default_rng(rows * cols)
    src = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    scale = 0.37
    d = empty_dev(cuda, rows * cols)
    tb.decode_e4m3_to_i8_transposed(to_dev(cuda, src), d, rows, cols, scale)
    cuda.cuda.synchronize()
    want = O.decode_e4m3_i8(src, scale).reshape(rows, cols).T
    np.testing.assert_array_equal(from_dev(d, np.int8).reshape(cols, rows), want)


SHAPES = [(256, 256, 256), (128, 256, 128), (200, 72, 48), (384, 520, 320), (1000, 16, 4096), (128, 1, 2048),
          (300, 100, 1056), (4096, 512, 512), (2500, 2000, 128)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_i8_exact(tb, cuda, M, N, K):
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    B = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    d = empty_dev(cuda, M * N * 4 + 256)
    tb.gemm_i8(to_dev(cuda, A), to_dev(cuda, B), d, M, N, K)
    cuda.cuda.synchronize()
    raw = from_dev(d, np.uint8)
    assert np.all(raw[M * N * 4:] == 0xA5), "wrote past the end of D"
    got = raw[: M * N * 4].view(np.int32).reshape(M, N)
    np.testing.assert_array_equal(got, O.gemm_i8(A, B, M, N, K))


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (300, 100, 1056), (1000, 16, 4096)])
def test_fp8_fused_int8_matches_reference_rule(tb, cuda, M, N, K):
    """A [M x K] and B [K x N] E4M3 from N(0, 1) data quantized with 448/maxabs,
    both converted with the per-tensor scale 127/maxabs of the decoded values
    (the scale the reference's comment prescribes), then the INT8 GEMM."""
    a = O.normal(11, (M, K), 1.0)
    b = O.normal(12, (K, N), 1.0)
    A = O.quantize(O.E4M3, a, O.per_tensor_scale(a, O.E4M3))
    B = O.quantize(O.E4M3, b, O.per_tensor_scale(b, O.E4M3))
    scale = float(np.float32(127.0) / np.float32(448.0))
    ws_bytes = tb.lib().tb_gemm_fp8_fused_int8_workspace(M, N, K)
    ws = empty_dev(cuda, ws_bytes)
    d = empty_dev(cuda, M * N * 4)
    tb.gemm_fp8_fused_int8(to_dev(cuda, A), to_dev(cuda, B), d, M, N, K, scale, ws, ws_bytes)
    cuda.cuda.synchronize()
    A8 = O.decode_e4m3_i8(A, scale).reshape(M, K)
    B8 = O.decode_e4m3_i8(B, scale).reshape(K, N).T.copy()
    want = O.gemm_i8(A8, B8, M, N, K)
    np.testing.assert_array_equal(from_dev(d, np.int32).reshape(M, N), want)
    assert np.abs(want).max() > 0
