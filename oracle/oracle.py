"""CPU oracle for the decode + GEMM path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only to check or time the CUDA path; the product never calls it.

Two libraries, both built by oracle/Makefile:
  liboracle.so      plain-C restatement of tensor-bridge's conversion
                    primitives and decode -> FP16 -> FP32-accumulate GEMM
                    (tb_oracle.c, each function citing the reference lines);
  _ref/libtbref.so  tensor-bridge's own headers compiled as host code
                    (ref_shim.cu); present only where the reference checkout
                    was available at build time.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtbref.so")

F16, E4M3, E5M2, E2M1, E2M1_UNPACKED, BF16, TF32, E2M1_HW = range(8)
FORMAT_MAX = {E4M3: 448.0, E5M2: 57344.0, E2M1: 6.0, E2M1_UNPACKED: 6.0, E2M1_HW: 6.0}

_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing; run `make -C oracle`")
        l = ctypes.CDLL(ORACLE_SO)
        p, sz, i, f = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
        l.oracle_decode.argtypes = [i, p, p, sz]
        l.oracle_quantize.argtypes = [i, p, p, sz, f]
        l.oracle_gemm.argtypes = [i, p, i, p, p, i, i, i, i, i, f, i, i]
        l.oracle_f32_to_f16.restype = ctypes.c_uint16
        l.oracle_f32_to_f16.argtypes = [f]
        l.oracle_decode_e4m3_i8.argtypes = [p, p, sz, f]
        l.oracle_gemm_i8.argtypes = [p, p, p, i, i, i, i]
        l.oracle_e4m3_scale_to_f32.restype = f
        l.oracle_e4m3_scale_to_f32.argtypes = [ctypes.c_uint8]
        l.oracle_decode_nvfp4.argtypes = [p, p, p, sz]
        _lib = l
    return _lib


def ref_lib():
    """The reference's own primitives, or None when _ref was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        l = ctypes.CDLL(REF_SO)
        p, sz, i, f = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
        for name in ("ref_e4m3_to_half", "ref_e5m2_to_half", "ref_bf16_to_half", "ref_tf32_to_half",
                     "ref_fp32_to_e4m3", "ref_fp32_to_e5m2", "ref_fp32_to_e2m1", "ref_half_to_e2m1",
                     "ref_fp32_to_bf16", "ref_half_to_bf16", "ref_fp32_to_tf32", "ref_fp32_to_half"):
            getattr(l, name).argtypes = [p, p, sz]
        l.ref_cpu_decode_gemm.argtypes = [i, p, p, p, i, i, i, i, i, f, i]
        l.ref_naive_decode_gemm.argtypes = [i, p, p, p, i, i, i, f]
        _ref = l
    return _ref


def _c(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def stored_dtype(fmt: int):
    return {F16: np.uint16, BF16: np.uint16, TF32: np.uint32}.get(fmt, np.uint8)


def stored_count(fmt: int, n: int) -> int:
    return (n + 1) // 2 if fmt in (E2M1, E2M1_HW) else n


def decode(fmt: int, src: np.ndarray, n: int) -> np.ndarray:
    src = np.ascontiguousarray(src)
    need = stored_count(fmt, n) * np.dtype(stored_dtype(fmt)).itemsize
    if src.nbytes < need:
        raise ValueError(f"decode of {n} values needs {need} bytes, got {src.nbytes}")
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_decode(fmt, _c(src), _c(out), n)
    return out


def quantize(fmt: int, x: np.ndarray, scale: float = 1.0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    out = np.empty(stored_count(fmt, n), dtype=stored_dtype(fmt))
    lib().oracle_quantize(fmt, _c(x.ravel()), _c(out), n, float(scale))
    return out.reshape(x.shape[:-1] + (-1,)) if x.ndim > 1 else out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    return quantize(F16, x).view(np.uint16)


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    """FP16 bits -> FP32; every NaN becomes 0x7FFFFFFF, as CUDA's __half2float."""
    out = np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)
    out[np.isnan(out)] = np.uint32(0x7FFFFFFF).view(np.float32)
    return out


def gemm(a_fmt: int, A: np.ndarray, b_fmt: int, B: np.ndarray, M: int, N: int, K: int, rows=None,
         alpha: float = 1.0, out_f16: bool = False, threads: int = 0) -> np.ndarray:
    """alpha * decode(A)[rows] @ decode(B).T with FP32 accumulation in k order.
    B is [N x K] in b_fmt.  Returns float32 (or float16 bits as uint16)."""
    r0, r1 = (0, M) if rows is None else rows
    A = np.ascontiguousarray(A)
    B = np.ascontiguousarray(B)
    out = np.empty((r1 - r0, N), dtype=np.uint16 if out_f16 else np.float32)
    lib().oracle_gemm(a_fmt, _c(A), b_fmt, _c(B), _c(out), M, N, K, r0, r1, float(alpha), int(out_f16), threads)
    return out


def ref_cpu_gemm(a_fmt: int, A: np.ndarray, B16: np.ndarray, M: int, N: int, K: int, rows=None,
                 alpha: float = 1.0, threads: int = 0) -> np.ndarray:
    """The reference's CPU path (its decode primitives + its FP32 loop)."""
    r = ref_lib()
    if r is None:
        raise RuntimeError("oracle/_ref was not built (needs the reference checkout at build time)")
    r0, r1 = (0, M) if rows is None else rows
    out = np.empty((r1 - r0, N), dtype=np.float32)
    r.ref_cpu_decode_gemm(a_fmt, _c(np.ascontiguousarray(A)), _c(np.ascontiguousarray(B16)), _c(out), M, N, K, r0, r1,
                          float(alpha), threads)
    return out


def ref_naive_gemm(a_fmt: int, A: np.ndarray, B16_kn: np.ndarray, M: int, N: int, K: int,
                   alpha: float = 1.0) -> np.ndarray:
    """The reference's naive single-thread check loop (bench/bench_formats.cu:183-186)
    on decoded A [M x K] and FP16 B [K x N]: D [M x N] FP32."""
    r = ref_lib()
    if r is None:
        raise RuntimeError("oracle/_ref was not built (needs the reference checkout at build time)")
    out = np.empty((M, N), dtype=np.float32)
    r.ref_naive_decode_gemm(a_fmt, _c(np.ascontiguousarray(A)), _c(np.ascontiguousarray(B16_kn)), _c(out), M, N, K,
                            float(alpha))
    return out


def decode_nvfp4(q: np.ndarray, scales: np.ndarray, n: int) -> np.ndarray:
    """Block-scaled FP4 -> FP16 bits: packed E2M1 codes (element 2j in the high
    nibble of byte j) times one E4M3 scale byte per 16 values."""
    q = np.ascontiguousarray(q, dtype=np.uint8).ravel()
    scales = np.ascontiguousarray(scales, dtype=np.uint8).ravel()
    if n % 16 or q.size < n // 2 or scales.size < n // 16:
        raise ValueError(f"block-scaled FP4 of {n} values needs {n // 2} code bytes and {n // 16} scale bytes")
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_decode_nvfp4(_c(q), _c(scales), _c(out), n)
    return out


def e4m3_scale_values() -> np.ndarray:
    """All 256 scale bytes as float32 (OCP E4M3 with subnormals; 0x7F/0xFF NaN)."""
    return np.array([lib().oracle_e4m3_scale_to_f32(c) for c in range(256)], dtype=np.float32)


def quantize_nvfp4(x: np.ndarray):
    """Two-level block-scaled FP4 of a [rows x cols] matrix (cols a multiple of
    16): g = amax / (6 * 448); each 16-value block's scale is the E4M3 value
    nearest to amax_block / (6 * g); codes = E2M1 of x / (scale * g) by the
    reference's rounding (fp4.h:46-53).  Returns (packed codes, scale bytes, g)
    with x ~= decode_nvfp4(codes, scales) * g."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    assert cols % 16 == 0
    amax = float(np.max(np.abs(x))) if x.size else 0.0
    g = np.float32(amax / (6.0 * 448.0)) if amax > 0 else np.float32(1.0)
    blocks = x.reshape(rows, cols // 16, 16)
    want = np.max(np.abs(blocks), axis=2) / (np.float32(6.0) * g)
    table = e4m3_scale_values()[:127]  # positive finite codes, ascending
    hi = np.clip(np.searchsorted(table, want), 1, 126)
    code = np.where(np.abs(table[hi] - want) < np.abs(want - table[hi - 1]), hi, hi - 1).astype(np.uint8)
    sv = table[code].astype(np.float32)[..., None] * g
    y = np.where(sv > 0, blocks / np.where(sv > 0, sv, 1), 0).astype(np.float32)
    q = quantize(E2M1, y.reshape(rows, cols), 1.0)
    return q.reshape(rows, cols // 2), code.reshape(rows, cols // 16), float(g)


def rel_frob(x: np.ndarray, ref: np.ndarray) -> float:
    """sqrt(sum (x-ref)^2 / sum ref^2) in float64 (bench/bench_formats.cu:97-103)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = float(np.sum(ref * ref))
    return float(np.sqrt(np.sum((x - ref) ** 2) / den)) if den > 0 else float(np.sqrt(np.sum((x - ref) ** 2)))


# ---- seeded synthetic inputs (shared by tests, smoke and bench) -----------------------

def uniform(seed: int, shape, lo=-1.0, hi=1.0) -> np.ndarray:
    return np.random.default_rng(seed).uniform(lo, hi, size=shape).astype(np.float32)


def normal(seed: int, shape, std=1.0) -> np.ndarray:
    return np.random.default_rng(seed).normal(0.0, std, size=shape).astype(np.float32)


def per_tensor_scale(x: np.ndarray, fmt: int) -> float:
    """FORMAT_MAX / maxabs as in bench/bench_formats.cu:128-130 (1.0 for BF16/TF32/F16)."""
    if fmt not in FORMAT_MAX:
        return 1.0
    m = float(np.max(np.abs(x))) if x.size else 0.0
    return float(np.float32(FORMAT_MAX[fmt]) / np.float32(m if m > 0 else 1.0))


def decode_e4m3_i8(codes: np.ndarray, scale: float) -> np.ndarray:
    """E4M3 codes -> INT8 by the reference's integer-path rule (src/gemm.cu:35-41)."""
    src = np.ascontiguousarray(np.asarray(codes, dtype=np.uint8).ravel())
    out = np.empty(src.size, dtype=np.int8)
    lib().oracle_decode_e4m3_i8(src.ctypes.data, out.ctypes.data, src.size, float(scale))
    return out


def gemm_i8(A8: np.ndarray, B8: np.ndarray, M: int, N: int, K: int, threads: int = 0) -> np.ndarray:
    """D [M x N] INT32 = A8 [M x K] * B8 [N x K]^T (src/gemm.cu:58-70)."""
    a = np.ascontiguousarray(np.asarray(A8, dtype=np.int8).ravel())
    b = np.ascontiguousarray(np.asarray(B8, dtype=np.int8).ravel())
    out = np.empty(M * N, dtype=np.int32)
    lib().oracle_gemm_i8(a.ctypes.data, b.ctypes.data, out.ctypes.data, M, N, K, threads)
    return out.reshape(M, N)
