"""Decode kernels on the GPU, bit-exact against the oracle on every code."""
import numpy as np
import pytest

import oracle as O
from golden_inputs import tf32_all_patterns
from gpu_util import to_dev, empty_dev, from_dev

pytestmark = pytest.mark.gpu

FORMATS = [O.E4M3, O.E5M2, O.E2M1, O.E2M1_UNPACKED, O.BF16, O.TF32, O.F16]


def all_codes(fmt, reps=3):
    """Every stored code of the format (repeated to fill several vector units),
    in a fixed shuffled order."""
    rng = np.random.default_rng(fmt)
    if fmt in (O.E4M3, O.E5M2, O.E2M1, O.E2M1_UNPACKED):
        base = np.arange(256, dtype=np.uint8)
    elif fmt in (O.BF16, O.F16):
        base = np.arange(65536, dtype=np.uint16)
    else:
        base = np.concatenate([tf32_all_patterns(),
                               rng.integers(0, 1 << 32, size=1 << 16, dtype=np.uint64).astype(np.uint32)])
    codes = np.concatenate([rng.permutation(base) for _ in range(reps)])
    n = codes.size * (2 if fmt == O.E2M1 else 1)
    return codes, n


def run_decode(tb, torch, fmt, src, n, src_offset=0, dst_offset=0):
    s = to_dev(torch, src, pad=64)
    d = empty_dev(torch, n * 2 + 64)
    sp = s.data_ptr()
    if src_offset:
        # shift the source by whole elements (misaligned start)
        s2 = empty_dev(torch, s.numel() + 64)
        esz = np.dtype(O.stored_dtype(fmt)).itemsize
        s2[src_offset * esz: src_offset * esz + s.numel()].copy_(s)
        s, sp = s2, s2.data_ptr() + src_offset * esz
    tb.decode(fmt, sp, d.data_ptr() + dst_offset * 2, n)
    torch.cuda.synchronize()
    out = from_dev(d, np.uint8)
    return out[dst_offset * 2: dst_offset * 2 + n * 2].view(np.uint16), out


@pytest.mark.parametrize("fmt", FORMATS)
def test_decode_every_code(tb, cuda, fmt):
    codes, n = all_codes(fmt)
    got, _ = run_decode(tb, cuda, fmt, codes, n)
    np.testing.assert_array_equal(got, O.decode(fmt, codes, n))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("n", [1, 7, 15, 31, 33, 1000, 4099])
def test_decode_tails(tb, cuda, fmt, n):
    codes, _ = all_codes(fmt, reps=1)
    src = np.resize(codes, O.stored_count(fmt, n))  # repeats the table as needed
    got, raw = run_decode(tb, cuda, fmt, src, n)
    np.testing.assert_array_equal(got, O.decode(fmt, src, n))
    assert np.all(raw[n * 2: n * 2 + 64] == 0xA5), "wrote past the end"


@pytest.mark.parametrize("fmt", [O.E4M3, O.BF16, O.TF32])
def test_decode_misaligned(tb, cuda, fmt):
    codes, _ = all_codes(fmt, reps=1)
    n = 5000
    codes = np.resize(codes, n)
    got, _ = run_decode(tb, cuda, fmt, codes, n, src_offset=1, dst_offset=3)
    np.testing.assert_array_equal(got, O.decode(fmt, codes, n))


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_decode_large(tb, cuda, fmt):
    # 64 M values: several grid-stride rounds.
    n = 64 << 20
    rng = np.random.default_rng(5)
    src = rng.integers(0, 256, size=O.stored_count(fmt, n), dtype=np.uint8)
    got, _ = run_decode(tb, cuda, fmt, src, n)
    np.testing.assert_array_equal(got, O.decode(fmt, src, n))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("rows,cols", [(1, 2), (64, 32), (96, 80), (37, 130), (300, 258), (256, 192), (1024, 1024)])
def test_decode_transposed(tb, cuda, fmt, rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    n = rows * cols
    if fmt in (O.BF16, O.F16):
        src = rng.integers(0, 65536, size=n, dtype=np.uint16)
    elif fmt == O.TF32:
        src = rng.integers(0, 1 << 32, size=n, dtype=np.uint64).astype(np.uint32)
    else:
        src = rng.integers(0, 256, size=O.stored_count(fmt, n), dtype=np.uint8)
    s = to_dev(cuda, src)
    d = empty_dev(cuda, n * 2 + 64)
    tb.decode_transposed(fmt, s, d, rows, cols)
    cuda.cuda.synchronize()
    got = from_dev(d, np.uint8)
    want = O.decode(fmt, src, n).reshape(rows, cols).T.copy()
    np.testing.assert_array_equal(got[: n * 2].view(np.uint16).reshape(cols, rows), want)
    assert np.all(got[n * 2:] == 0xA5)


@pytest.mark.parametrize("name,fmt", [("tb_decode_fp8_to_half", O.E4M3), ("tb_decode_bf16_to_half", O.BF16),
                                      ("tb_decode_tf32_to_half", O.TF32), ("tb_decode_fp4_to_half", O.E2M1_UNPACKED)])
def test_reference_shaped_decode(tb, cuda, name, fmt):
    """decode A [M x K] straight and B [K x N] transposed in one call, as the
    reference's decode kernels do (src/gemm.cu:25-30)."""
    M, N, K = 48, 80, 64
    rng = np.random.default_rng(2)
    dt = O.stored_dtype(fmt)
    hi = {np.uint8: 256, np.uint16: 65536, np.uint32: 1 << 32}[dt]
    if fmt == O.E2M1_UNPACKED:
        hi = 16
    A = rng.integers(0, hi, size=M * K, dtype=np.uint64).astype(dt)
    B = rng.integers(0, hi, size=K * N, dtype=np.uint64).astype(dt)
    dA, dB = to_dev(cuda, A), to_dev(cuda, B)
    A16, B16 = empty_dev(cuda, M * K * 2), empty_dev(cuda, N * K * 2)
    tb.call(name, dA.data_ptr(), dB.data_ptr(), A16.data_ptr(), B16.data_ptr(), M, N, K, cuda.cuda.current_stream().cuda_stream)
    cuda.cuda.synchronize()
    np.testing.assert_array_equal(from_dev(A16, np.uint16), O.decode(fmt, A, M * K))
    np.testing.assert_array_equal(from_dev(B16, np.uint16).reshape(N, K), O.decode(fmt, B, K * N).reshape(K, N).T)


def test_fp4_repack(tb, cuda):
    src = np.random.default_rng(9).integers(0, 256, size=100003, dtype=np.uint8)
    s = to_dev(cuda, src)
    d = empty_dev(cuda, src.size)
    tb.fp4_repack_hw(s, d, src.size)
    cuda.cuda.synchronize()
    got = from_dev(d, np.uint8)
    np.testing.assert_array_equal(got, ((src >> 4) | (src << 4)).astype(np.uint8))
    n = 2 * src.size
    np.testing.assert_array_equal(O.decode(O.E2M1_HW, got, n), O.decode(O.E2M1, src, n))
