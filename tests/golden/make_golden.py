"""Generate tests/golden/golden.npz from tensor-bridge's OWN conversion primitives.

Run in a container that has the reference checkout and a built
oracle/_ref/libtbref.so (``make -C oracle``):

    python tests/golden/make_golden.py

Every array in the archive is an output of the reference's headers
(include/tensor_bridge/{fp8,fp4,bf16,tf32}.h) or of its CPU decode + FP32 GEMM
loop, on inputs that are either exhaustive code tables or seeded draws that
this script also records.  Large sweeps are stored as SHA-256 digests of the
output bytes (the inputs are regenerated from the same recipe).
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

from golden_inputs import (  # noqa: E402
    quant_inputs, tf32_all_patterns, tf32_random_words, gemm_case, GEMM_CASES,
)


def _c(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def run(fn, inp, out_dtype):
    inp = np.ascontiguousarray(inp)
    out = np.empty(inp.size, dtype=out_dtype)
    fn(_c(inp), _c(out), inp.size)
    return out


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    r = oracle.ref_lib()
    if r is None:
        sys.exit("oracle/_ref/libtbref.so not built: needs the reference checkout; run `make -C oracle`")
    g = {}
    codes8 = np.arange(256, dtype=np.uint8)
    g["e4m3_to_half"] = run(r.ref_e4m3_to_half, codes8, np.uint16)
    g["e5m2_to_half"] = run(r.ref_e5m2_to_half, codes8, np.uint16)
    g["bf16_to_half"] = run(r.ref_bf16_to_half, np.arange(65536, dtype=np.uint16), np.uint16)
    tf_all = tf32_all_patterns()
    g["tf32_all_sha256"] = np.array(sha(run(r.ref_tf32_to_half, tf_all, np.uint16)))
    tf_rand = tf32_random_words()
    g["tf32_random_in"] = tf_rand
    g["tf32_random_out"] = run(r.ref_tf32_to_half, tf_rand, np.uint16)

    q = quant_inputs()
    g["quant_in"] = q
    g["q_e4m3"] = run(r.ref_fp32_to_e4m3, q, np.uint8)
    g["q_e5m2"] = run(r.ref_fp32_to_e5m2, q, np.uint8)
    g["q_e2m1"] = run(r.ref_fp32_to_e2m1, q, np.uint8)
    g["q_bf16"] = run(r.ref_fp32_to_bf16, q, np.uint16)
    g["q_tf32"] = run(r.ref_fp32_to_tf32, q, np.uint32)
    g["q_f16"] = run(r.ref_fp32_to_half, q, np.uint16)
    all_half = np.arange(65536, dtype=np.uint16)
    g["half_to_e2m1"] = run(r.ref_half_to_e2m1, all_half, np.uint8)
    g["half_to_bf16"] = run(r.ref_half_to_bf16, all_half, np.uint16)

    for name in GEMM_CASES:
        fmt, A, B16, M, N, K, alpha = gemm_case(name)
        g[f"gemm_{name}_A"] = A
        g[f"gemm_{name}_B16"] = B16
        g[f"gemm_{name}_alpha"] = np.array(alpha, dtype=np.float32)
        g[f"gemm_{name}"] = oracle.ref_cpu_gemm(fmt, A, B16, M, N, K, alpha=alpha)

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **g)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
