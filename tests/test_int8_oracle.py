"""The INT8 path's oracle (oracle/tb_oracle.c: oracle_e4m3_to_i8,
oracle_gemm_i8) against values worked out by hand from the reference's rule
in src/gemm.cu:35-41 -- (int8_t)__float2int_rn(__half2float(fp8_e4m3_to_half(c))
* scale) -- and its int32-accumulating GEMM (src/gemm.cu:58-70)."""
import numpy as np

import oracle as O


def test_known_answers():
    codes = np.array([0x38, 0xB8, 0x7E, 0xFE, 0x00, 0x80, 0x01, 0x7F, 0xFF, 0x30, 0x3C], dtype=np.uint8)
    # 1.0, -1.0, 448, -448, 0, -0, subnormal (flushed to 0), NaN, NaN, 0.5, 1.5
    s = np.float32(127.0) / np.float32(448.0)
    got = O.decode_e4m3_i8(codes, float(s))
    want = [0, 0, 127, -127, 0, 0, 0, 0, 0, 0, 0]
    # 1.0 * 127/448 = 0.2834 -> 0; 448 * s = 127.0 exactly in FP32 -> 127
    assert list(got) == want
    got = O.decode_e4m3_i8(codes, 1.0)
    assert list(got) == [1, -1, 448 - 512, -(448 - 512), 0, 0, 0, 0, 0, 0, 2]  # 448 wraps to -64; 1.5 -> 2 (even)
    # ties go to even: 0.5 -> 0, 1.5 -> 2, 2.5 -> 2 (code 0x42 = 2.5)
    assert list(O.decode_e4m3_i8(np.array([0x30, 0x3C, 0x42], np.uint8), 1.0)) == [0, 2, 2]
    # the reference's own warning: a fixed *8 overflows E4M3's range -- 448 * 8 = 3584 (0xE00) -> low
    # byte 0; code 0x6E is 112, 112 * 8 = 896 (0x380) -> 0x80 = -128
    assert list(O.decode_e4m3_i8(np.array([0x7E, 0x6E], np.uint8), 8.0)) == [0, -128]
    # beyond int32: the conversion clamps (INT32_MAX -> 0xFF = -1, INT32_MIN -> 0)
    assert list(O.decode_e4m3_i8(np.array([0x7E, 0xFE], np.uint8), 1e30)) == [-1, 0]


def test_gemm_i8_small():
    rng = np.random.default_rng(3)
    A = rng.integers(-128, 128, size=(5, 7), dtype=np.int8)
    B = rng.integers(-128, 128, size=(3, 7), dtype=np.int8)
    want = A.astype(np.int64) @ B.astype(np.int64).T
    assert np.array_equal(O.gemm_i8(A, B, 5, 3, 7), want.astype(np.int32))
