"""The C-ABI library loads, exports exactly what include/tensor_bridge_b200.h
declares, and rejects bad arguments with the documented status codes before
touching a device (so these run on CPU)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tensor_bridge_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tb_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(tb):
    lib = tb.lib()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    # ... and the Python binding declares the same set.
    assert sorted(tb.SIGNATURES) == names


def test_dynamic_symbol_table_matches_header(tb):
    out = subprocess.run(["nm", "-D", "--defined-only", tb.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = sorted(set(re.findall(r"\bT (tb_\w+)", out)))
    assert exported == declared_functions()


def test_status_strings(tb):
    lib = tb.lib()
    for s in tb.Status:
        assert lib.tb_status_string(int(s)).decode() == "TB_" + ("OK" if s == 0 else "ERR_" + s.name)


def test_argument_validation_without_device(tb):
    lib = tb.lib()
    null = None
    # null pointers
    assert lib.tb_decode(int(tb.Format.E4M3), null, null, 16, null) == tb.Status.INVALID_ARGUMENT
    # n == 0 is a no-op success
    assert lib.tb_decode(int(tb.Format.E4M3), null, null, 0, null) == tb.Status.OK
    # bad enum
    assert lib.tb_decode(99, null, null, 16, null) == tb.Status.INVALID_ARGUMENT
    # shapes: K not a multiple of 16, packed FP4 needs K % 32
    p = ctypes.c_void_p(256)
    assert lib.tb_gemm_f16(p, p, p, 64, 64, 40, 0, 1.0, null) == tb.Status.SHAPE
    assert lib.tb_gemm_f16(p, p, p, 0, 64, 64, 0, 1.0, null) == tb.Status.SHAPE
    assert lib.tb_gemm_fused(int(tb.Format.E2M1), p, p, p, 64, 64, 48, 0, 1.0, null, 0, null) == tb.Status.SHAPE
    assert lib.tb_gemm_fused(int(tb.Format.E2M1_HW), p, p, p, 64, 64, 64, 0, 1.0, null, 0, null) == \
        tb.Status.INVALID_ARGUMENT
    assert "multiple of" in lib.tb_last_error().decode() or lib.tb_last_error().decode()
    assert lib.tb_decode_transposed(int(tb.Format.E2M1), p, p, 4, 5, null) == tb.Status.SHAPE
    # unsupported native pairing
    assert lib.tb_gemm_native(int(tb.Format.BF16), p, int(tb.Format.BF16), p, p, 64, 64, 64, 0, 1.0, null) == \
        tb.Status.UNSUPPORTED
    # native FP4: K % 128 and 32-byte alignment
    assert lib.tb_gemm_native(int(tb.Format.E2M1_HW), p, int(tb.Format.E2M1_HW), p, p, 64, 64, 96, 0, 1.0, null) == \
        tb.Status.SHAPE
    p16 = ctypes.c_void_p(256 + 16)
    assert lib.tb_gemm_native(int(tb.Format.E4M3), p, int(tb.Format.E2M1_HW), p16, p, 64, 64, 128, 0, 1.0, null) == \
        tb.Status.ALIGNMENT
    assert lib.tb_gemm_native(int(tb.Format.E4M3), p, int(tb.Format.E2M1), p, p, 64, 64, 128, 0, 1.0, null) == \
        tb.Status.UNSUPPORTED
    # fp8 mirror needs its workspace
    assert lib.tb_gemm_fp8_fused_fp16(p, p, p, 64, 64, 64, null, 0, null) == tb.Status.WORKSPACE
    # flushed copies of A [M x K] and of B transposed [N x K], each rounded to 256 bytes
    assert lib.tb_gemm_fp8_fused_workspace(64, 48, 64) == 64 * 64 + 48 * 64
    assert lib.tb_gemm_fp8_fused_workspace(10, 3, 16) == 256 + 256
    # peer buffers: nothing to release, and no GEMM or registration without a handle / communicator
    # (TB_ERR_NCCL where NCCL cannot be loaded)
    assert lib.tb_peer_buffer_release(null, null) == tb.Status.OK
    st = lib.tb_gemm_sharded_fused_p2p(int(tb.Format.E4M3), p, p, null, 1024, 64, 64, 0, 1.0, 1, null)
    assert st in (tb.Status.INVALID_ARGUMENT, tb.Status.NCCL)
    h = ctypes.c_void_p()
    st = lib.tb_peer_buffer_register(null, p, 1024, null, ctypes.byref(h))
    assert st in (tb.Status.INVALID_ARGUMENT, tb.Status.NCCL) and not h.value


def test_python_binding_raises(tb):
    with pytest.raises(tb.TBError) as e:
        tb.gemm_f16(256, 256, 256, 64, 64, 40, stream=0)
    assert e.value.status == tb.Status.SHAPE


def test_stored_bytes(tb):
    assert tb.stored_bytes(tb.Format.E2M1, 7) == 4
    assert tb.stored_bytes(tb.Format.TF32, 3) == 12
    assert tb.stored_bytes(tb.Format.E4M3, 5) == 5
