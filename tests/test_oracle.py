"""Pin the CPU oracle: the reference's own known-answer vectors, the golden
tables generated from the reference headers, and (where the reference was
built here) a direct exhaustive comparison with it."""
import hashlib

import numpy as np
import pytest

import oracle
from golden_inputs import quant_inputs, tf32_all_patterns, gemm_case, GEMM_CASES

O = oracle


def f(h):
    return float(np.uint16(h).view(np.float16))


def dec1(fmt, code):
    arr = np.array([code], dtype=O.stored_dtype(fmt))
    return int(O.decode(fmt, arr, 1)[0])


def q1(fmt, v):
    return int(O.quantize(fmt, np.array([v], dtype=np.float32))[0])


# ---- known-answer vectors of tests/test_conversions.cu:25-85 (reference) ----------

def test_kat_e4m3_decode():
    assert f(dec1(O.E4M3, 0x00)) == 0.0
    assert f(dec1(O.E4M3, 0x38)) == 1.0
    assert f(dec1(O.E4M3, 0x30)) == 0.5
    assert f(dec1(O.E4M3, 0x40)) == 2.0
    assert f(dec1(O.E4M3, 0xB8)) == -1.0
    assert f(dec1(O.E4M3, 0x3C)) == 1.5
    assert f(dec1(O.E4M3, 0x7E)) == 448.0
    assert np.isnan(f(dec1(O.E4M3, 0x7F)))


def test_kat_e5m2_decode():
    assert f(dec1(O.E5M2, 0x3C)) == 1.0
    assert f(dec1(O.E5M2, 0x38)) == 0.5
    assert f(dec1(O.E5M2, 0x40)) == 2.0
    assert f(dec1(O.E5M2, 0x7B)) == 57344.0
    assert np.isinf(f(dec1(O.E5M2, 0x7C)))
    assert np.isnan(f(dec1(O.E5M2, 0x7F)))


def test_kat_bf16_decode():
    assert f(dec1(O.BF16, 0x3F80)) == 1.0
    assert f(dec1(O.BF16, 0x3F00)) == 0.5
    assert f(dec1(O.BF16, 0x4000)) == 2.0
    assert f(dec1(O.BF16, 0xBF80)) == -1.0
    assert np.isinf(f(dec1(O.BF16, 0x7F80)))
    assert np.isnan(f(dec1(O.BF16, 0x7FC0)))


def test_kat_fp4_all_nibbles_and_packing():
    want = [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]
    got = [f(dec1(O.E2M1_UNPACKED, i)) for i in range(16)]
    assert got == want
    assert dec1(O.E2M1_UNPACKED, 8) == 0x8000  # -0
    # fp4_e2m1_byte_to_half2(0x72) -> (6.0, 1.0): first value in the high nibble
    pair = O.decode(O.E2M1, np.array([0x72], dtype=np.uint8), 2)
    assert (f(pair[0]), f(pair[1])) == (6.0, 1.0)


def test_kat_fp4_round_trips():
    rt = lambda v: f(dec1(O.E2M1_UNPACKED, q1(O.E2M1_UNPACKED, v)))  # noqa: E731
    assert rt(1.0) == 1.0
    assert rt(5.5) == 6.0
    assert rt(-1.0) == -1.0
    assert rt(-2.0) == -2.0
    assert rt(0.5) == 0.5
    assert rt(-5.0) == -4.0   # tie resolved to the lower magnitude


def test_kat_tf32_decode():
    assert f(dec1(O.TF32, 0x3F800000)) == 1.0
    assert f(dec1(O.TF32, 0x40000000)) == 2.0
    assert np.isinf(f(dec1(O.TF32, 0x7F800000)))
    assert np.isnan(f(dec1(O.TF32, 0x7FC00000)))


def test_kat_e4m3_round_trips():
    for v in (1.0, 0.5, 448.0):
        assert f(dec1(O.E4M3, q1(O.E4M3, v))) == v


# ---- golden tables (outputs of the reference headers) -----------------------------

def test_golden_decode_tables(golden):
    codes = np.arange(256, dtype=np.uint8)
    np.testing.assert_array_equal(O.decode(O.E4M3, codes, 256), golden["e4m3_to_half"])
    np.testing.assert_array_equal(O.decode(O.E5M2, codes, 256), golden["e5m2_to_half"])
    np.testing.assert_array_equal(O.decode(O.BF16, np.arange(65536, dtype=np.uint16), 65536), golden["bf16_to_half"])
    tf = tf32_all_patterns()
    digest = hashlib.sha256(O.decode(O.TF32, tf, tf.size).tobytes()).hexdigest()
    assert digest == str(golden["tf32_all_sha256"])
    rin = golden["tf32_random_in"]
    np.testing.assert_array_equal(O.decode(O.TF32, rin, rin.size), golden["tf32_random_out"])


@pytest.mark.parametrize("fmt,key", [(O.E4M3, "q_e4m3"), (O.E5M2, "q_e5m2"), (O.E2M1_UNPACKED, "q_e2m1"),
                                     (O.BF16, "q_bf16"), (O.TF32, "q_tf32"), (O.F16, "q_f16")])
def test_golden_quantizers(golden, fmt, key):
    q = golden["quant_in"]
    np.testing.assert_array_equal(q, quant_inputs(), err_msg="input recipe drifted")
    got = O.quantize(fmt, q)
    want = golden[key]
    if fmt == O.F16:  # NaN payloads are not part of the contract; compare the non-NaN lanes
        keep = ~np.isnan(q)
        got, want = got[keep], want[keep]
    np.testing.assert_array_equal(got, want)


def test_golden_half_helpers(golden):
    halves = O.f16_bits_to_f32(np.arange(65536, dtype=np.uint16))
    np.testing.assert_array_equal(O.quantize(O.E2M1_UNPACKED, halves), golden["half_to_e2m1"])
    np.testing.assert_array_equal(O.quantize(O.BF16, halves), golden["half_to_bf16"])


@pytest.mark.parametrize("name", list(GEMM_CASES))
def test_golden_gemm(golden, name):
    fmt = GEMM_CASES[name]
    A, B16 = golden[f"gemm_{name}_A"], golden[f"gemm_{name}_B16"]
    alpha = float(golden[f"gemm_{name}_alpha"])
    M, K = 40, 96
    N = B16.shape[0]
    got = O.gemm(fmt, A, O.F16, B16, M, N, K, alpha=alpha)
    # Same decode, same FP32 k-order accumulation: bit-identical.
    np.testing.assert_array_equal(got, golden[f"gemm_{name}"])
    # The recipe that made the inputs still produces them.
    f2, A2, B2, *_ = gemm_case(name)
    np.testing.assert_array_equal(A2, A)
    np.testing.assert_array_equal(B2, B16)


def test_f32_to_f16_matches_numpy():
    x = np.random.default_rng(3).integers(0, 1 << 32, size=200000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = x[~np.isnan(x)]
    np.testing.assert_array_equal(O.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))


def test_fp4_packing_orders():
    vals = np.array([6.0, 1.0, -0.5, 3.0], dtype=np.float32)
    ref = O.quantize(O.E2M1, vals)
    hw = O.quantize(O.E2M1_HW, vals)
    assert ref.tolist() == [0x72, 0x95]
    assert hw.tolist() == [0x27, 0x59]
    np.testing.assert_array_equal(O.decode(O.E2M1, ref, 4), O.decode(O.E2M1_HW, hw, 4))


def test_fp4_quantizer_quirks():
    # ties to the lower magnitude, -0 and NaN give code 0, huge values give 0 (fp4.h:46-53)
    assert [q1(O.E2M1_UNPACKED, v) for v in (0.25, 0.75, 1.25, 2.5, 3.5, 5.0)] == [0, 1, 2, 4, 5, 6]
    assert q1(O.E2M1_UNPACKED, -0.0) == 0
    assert q1(O.E2M1_UNPACKED, float("nan")) == 0
    assert q1(O.E2M1_UNPACKED, 7.0) == 7
    assert q1(O.E2M1_UNPACKED, 2.0 ** 27) == 7   # 2^27 - 6 still rounds below 2^27
    assert q1(O.E2M1_UNPACKED, 2.0 ** 28) == 0   # every distance rounds to |v|: code 0
    assert q1(O.E2M1_UNPACKED, 1e30) == 0
    assert q1(O.E2M1_UNPACKED, float("-inf")) == 8


def test_e4m3_quantizer_quirks():
    assert q1(O.E4M3, float("nan")) == 0x7E   # NaN clamps to +448
    assert q1(O.E4M3, 1e9) == 0x7E
    assert q1(O.E4M3, -1e9) == 0xFE
    assert q1(O.E4M3, 2.0 ** -7) == 0x00     # below the smallest normal: flushed
    assert q1(O.E4M3, -(2.0 ** -7)) == 0x80


# ---- direct comparison with the reference build (when present) -------------------

ref = O.ref_lib()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built (no reference checkout)")


@needs_ref
def test_oracle_matches_reference_on_random_floats():
    import ctypes
    x = np.random.default_rng(11).integers(0, 1 << 32, size=1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([x, O.normal(12, 1 << 18, 30.0)])
    c = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    for fn, fmt, dt in ((ref.ref_fp32_to_e4m3, O.E4M3, np.uint8), (ref.ref_fp32_to_e5m2, O.E5M2, np.uint8),
                        (ref.ref_fp32_to_e2m1, O.E2M1_UNPACKED, np.uint8), (ref.ref_fp32_to_bf16, O.BF16, np.uint16),
                        (ref.ref_fp32_to_tf32, O.TF32, np.uint32)):
        want = np.empty(x.size, dtype=dt)
        fn(c(x), c(want), x.size)
        np.testing.assert_array_equal(O.quantize(fmt, x), want)
