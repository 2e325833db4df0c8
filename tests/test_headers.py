"""The source-compatible primitives in include/tensor_bridge/*.h are bit-exact
to the reference (golden tables made from the reference headers) when built
as host code, both by nvcc and by a plain host C++ compiler."""
import ctypes
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

import oracle as O
from golden_inputs import quant_inputs, tf32_all_patterns

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROBE = os.path.join(ROOT, "tests", "header_probe.cpp")
CUDA_INC = "/usr/local/cuda/include"


def _build(compiler: str, tmp: str) -> ctypes.CDLL:
    out = os.path.join(tmp, f"probe_{compiler}.so")
    inc = ["-I", os.path.join(ROOT, "include")]
    if compiler == "nvcc":
        cmd = ["nvcc", "-O2", "-std=c++17", "-x", "cu", "-Xcompiler", "-fPIC", "-shared",
               "-gencode", "arch=compute_100a,code=sm_100a", *inc, PROBE, "-o", out]
    else:
        gxx = shutil.which("g++")
        cmd = [gxx, "-O2", "-std=c++17", "-fPIC", "-shared", *inc, "-I", CUDA_INC, PROBE, "-o", out]
    subprocess.run(cmd, check=True, capture_output=True, timeout=300)
    return ctypes.CDLL(out)


@pytest.fixture(scope="module", params=["nvcc", "g++"])
def probe(request):
    if request.param == "nvcc" and shutil.which("nvcc") is None:
        pytest.skip("nvcc not available")
    if request.param == "g++" and (shutil.which("g++") is None or not os.path.isdir(CUDA_INC)):
        pytest.skip("g++ or CUDA headers not available")
    tmp = tempfile.mkdtemp(prefix="tb_probe_")
    try:
        yield _build(request.param, tmp)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def c(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def run(fn, inp, dt, n_out=None):
    inp = np.ascontiguousarray(inp)
    out = np.empty(n_out or inp.size, dtype=dt)
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    fn(c(inp), c(out), inp.size)
    return out


def test_decode_tables(probe, golden):
    codes = np.arange(256, dtype=np.uint8)
    np.testing.assert_array_equal(run(probe.p_e4m3_to_half, codes, np.uint16), golden["e4m3_to_half"])
    np.testing.assert_array_equal(run(probe.p_e5m2_to_half, codes, np.uint16), golden["e5m2_to_half"])
    np.testing.assert_array_equal(run(probe.p_bf16_to_half, np.arange(65536, dtype=np.uint16), np.uint16),
                                  golden["bf16_to_half"])
    tf = tf32_all_patterns()
    np.testing.assert_array_equal(run(probe.p_tf32_to_half, tf, np.uint16), O.decode(O.TF32, tf, tf.size))
    rin = golden["tf32_random_in"]
    np.testing.assert_array_equal(run(probe.p_tf32_to_half, rin, np.uint16), golden["tf32_random_out"])
    # FP4: every nibble (the reference table, fp4.h:27-30) and every packed byte.
    np.testing.assert_array_equal(run(probe.p_fp4_to_half, np.arange(16, dtype=np.uint8), np.uint16),
                                  O.decode(O.E2M1_UNPACKED, np.arange(16, dtype=np.uint8), 16))
    packed = np.arange(256, dtype=np.uint8)
    np.testing.assert_array_equal(run(probe.p_fp4_byte_to_half2, packed, np.uint16, 512),
                                  O.decode(O.E2M1, packed, 512))


@pytest.mark.parametrize("fn,key,dt", [("p_fp32_to_e4m3", "q_e4m3", np.uint8), ("p_fp32_to_e5m2", "q_e5m2", np.uint8),
                                       ("p_fp32_to_e2m1", "q_e2m1", np.uint8), ("p_fp32_to_bf16", "q_bf16", np.uint16),
                                       ("p_fp32_to_tf32", "q_tf32", np.uint32)])
def test_quantizers(probe, golden, fn, key, dt):
    q = quant_inputs()
    got = run(getattr(probe, fn), q, dt)
    want = golden[key]
    # Signaling-NaN inputs to the FP8 quantizers depend on how the host
    # compiler treats fminf (glibc returns NaN for them, a folded builtin
    # returns the other operand); they are outside the contract.
    bits = q.view(np.uint32)
    snan = ((bits & 0x7F800000) == 0x7F800000) & ((bits & 0x7FFFFF) != 0) & ((bits & 0x400000) == 0)
    np.testing.assert_array_equal(got[~snan], want[~snan])


def test_half_helpers(probe, golden):
    h = np.arange(65536, dtype=np.uint16)
    np.testing.assert_array_equal(run(probe.p_half_to_e2m1, h, np.uint8), golden["half_to_e2m1"])
    np.testing.assert_array_equal(run(probe.p_half_to_bf16, h, np.uint16), golden["half_to_bf16"])


def test_scale_helpers(probe):
    x = O.normal(5, 4096, 0.02)
    for fmt, qfn, dfn in ((O.E4M3, probe.p_e4m3_scaled, probe.p_e4m3_dequant),
                          (O.E2M1_UNPACKED, probe.p_e2m1_scaled, probe.p_e2m1_dequant)):
        s = O.per_tensor_scale(x, fmt)
        qfn.argtypes = dfn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float]
        q = np.empty(x.size, dtype=np.uint8)
        qfn(c(x), c(q), x.size, s)
        np.testing.assert_array_equal(q, O.quantize(fmt, x, s))
        d = np.empty(x.size, dtype=np.float32)
        dfn(c(q), c(d), x.size, s)
        want = (O.f16_bits_to_f32(O.decode(fmt, q, x.size)) / np.float32(s)).astype(np.float32)
        np.testing.assert_array_equal(d, want)
