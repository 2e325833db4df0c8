"""tensor_bridge_b200 -- Python binding of the C ABI in include/tensor_bridge_b200.h.

The product is the shared library libtensor_bridge_b200.so (CUDA kernels for
sm_100a behind extern "C" entry points).  This module loads it with ctypes,
declares every entry point's signature, raises TBError on a non-OK status,
and offers small helpers that take anything with a ``data_ptr()`` (torch
tensors) or plain integer device addresses.

There is no fallback: if the library is missing, importing works but the
first call raises LibraryNotBuilt.
"""
from __future__ import annotations

import ctypes
import enum
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtensor_bridge_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "tensor_bridge_b200.h")


class Format(enum.IntEnum):
    F16 = 0
    E4M3 = 1
    E5M2 = 2
    E2M1 = 3            # packed, first value in the high nibble (reference order)
    E2M1_UNPACKED = 4   # one value per byte
    BF16 = 5
    TF32 = 6
    E2M1_HW = 7         # packed, first value in the low nibble (tensor-core order)


class Out(enum.IntEnum):
    F32 = 0
    F16 = 1


class Status(enum.IntEnum):
    OK = 0
    INVALID_ARGUMENT = 1
    SHAPE = 2
    ALIGNMENT = 3
    CUDA = 4
    LAUNCH = 5
    TIMEOUT = 6
    UNSUPPORTED = 7
    WORKSPACE = 8
    NCCL = 9


class LibraryNotBuilt(RuntimeError):
    pass


class TBError(RuntimeError):
    def __init__(self, status: int, func: str, detail: str):
        self.status = Status(status) if status in Status._value2member_map_ else status
        super().__init__(f"{func}: {getattr(self.status, 'name', status)}: {detail}")


# Bytes per stored element, as (numerator, denominator).
STORED_BYTES = {
    Format.F16: (2, 1), Format.E4M3: (1, 1), Format.E5M2: (1, 1), Format.E2M1: (1, 2),
    Format.E2M1_UNPACKED: (1, 1), Format.BF16: (2, 1), Format.TF32: (4, 1), Format.E2M1_HW: (1, 2),
}


def stored_bytes(fmt: Format, n: int) -> int:
    num, den = STORED_BYTES[Format(fmt)]
    return (n * num + den - 1) // den


_p = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_f = ctypes.c_float
_st = ctypes.c_int  # tb_status

# name -> (restype, argtypes); the set of names is exactly the header's.
SIGNATURES = {
    "tb_status_string": (ctypes.c_char_p, [_st]),
    "tb_last_error": (ctypes.c_char_p, []),
    "tb_device_supported": (_st, [_i]),
    "tb_device_error": (_st, [ctypes.POINTER(_i), _i]),
    "tb_decode": (_st, [_i, _p, _p, _sz, _p]),
    "tb_decode_transposed": (_st, [_i, _p, _p, _i, _i, _p]),
    "tb_decode_nvfp4": (_st, [_p, _p, _p, _sz, _p]),
    "tb_decode_fp8_to_half": (_st, [_p, _p, _p, _p, _i, _i, _i, _p]),
    "tb_decode_bf16_to_half": (_st, [_p, _p, _p, _p, _i, _i, _i, _p]),
    "tb_decode_tf32_to_half": (_st, [_p, _p, _p, _p, _i, _i, _i, _p]),
    "tb_decode_fp4_to_half": (_st, [_p, _p, _p, _p, _i, _i, _i, _p]),
    "tb_quantize": (_st, [_i, _p, _p, _sz, _f, _p]),
    "tb_absmax": (_st, [_p, _sz, _p, _p]),
    "tb_gemm_f16": (_st, [_p, _p, _p, _i, _i, _i, _i, _f, _p]),
    "tb_gemm_fused": (_st, [_i, _p, _p, _p, _i, _i, _i, _i, _f, _p, _sz, _p]),
    "tb_gemm_fused_workspace": (_sz, [_i, _i, _i, _i]),
    "tb_gemm_fused_noalloc": (_st, [_i, _p, _p, _p, _i, _i, _i, _i, _f, _p]),
    "tb_gemm_native": (_st, [_i, _p, _i, _p, _p, _i, _i, _i, _i, _f, _p]),
    "tb_gemm_nvfp4": (_st, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _f, _p]),
    "tb_fp4_repack_hw": (_st, [_p, _p, _sz, _p]),
    "tb_gemm_fp8_fused_fp16": (_st, [_p, _p, _p, _i, _i, _i, _p, _sz, _p]),
    "tb_gemm_fp8_fused_workspace": (_sz, [_i, _i, _i]),
    "tb_decode_e4m3_to_i8": (_st, [_p, _p, _sz, _f, _p]),
    "tb_decode_e4m3_to_i8_transposed": (_st, [_p, _p, _i, _i, _f, _p]),
    "tb_decode_fp8_to_int8": (_st, [_p, _p, _p, _p, _i, _i, _i, _f, _p]),
    "tb_gemm_i8": (_st, [_p, _p, _p, _i, _i, _i, _p]),
    "tb_gemm_fp8_fused_int8": (_st, [_p, _p, _p, _i, _i, _i, _f, _p, _sz, _p]),
    "tb_gemm_fp8_fused_int8_workspace": (_sz, [_i, _i, _i]),
    "tb_gemm_sharded_fused": (_st, [_i, _p, _p, _p, _i, _i, _i, _i, _f, _p, _i, _p, _p]),
    "tb_gemm_sharded_fused_p2p": (_st, [_i, _p, _p, _p, _i, _i, _i, _i, _f, _i, _p]),
    "tb_peer_buffer_register": (_st, [_p, _p, _sz, _p, ctypes.POINTER(_p)]),
    "tb_peer_buffer_release": (_st, [_p, _p]),
    "tb_nccl_unique_id": (_st, [ctypes.c_char_p]),
    "tb_nccl_comm_init": (_st, [ctypes.POINTER(_p), _i, _i, ctypes.c_char_p]),
    "tb_nccl_comm_destroy": (_st, [_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libtensor_bridge_b200.so once and declare its signatures."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryNotBuilt(f"{LIB_PATH} is missing; run `make -C tensor-bridge_b200` (or __graft_entry__.build())")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _check(status: int, func: str):
    if status != 0:
        detail = lib().tb_last_error().decode(errors="replace")
        raise TBError(status, func, detail)


def call(name: str, *args):
    """Call an entry point by name and raise TBError on a non-OK status."""
    fn = getattr(lib(), name)
    st = fn(*args)
    if SIGNATURES[name][0] is _st:
        _check(st, name)
    return st


# ---- helpers over device buffers ------------------------------------------------------

def decode(fmt, src, dst, n: int, stream=None):
    call("tb_decode", int(fmt), _ptr(src), _ptr(dst), n, _stream(stream))


def decode_transposed(fmt, src, dst, rows: int, cols: int, stream=None):
    call("tb_decode_transposed", int(fmt), _ptr(src), _ptr(dst), rows, cols, _stream(stream))


def decode_nvfp4(src, scales, dst, n: int, stream=None):
    call("tb_decode_nvfp4", _ptr(src), _ptr(scales), _ptr(dst), n, _stream(stream))


def quantize(fmt, src, dst, n: int, scale: float = 1.0, stream=None):
    call("tb_quantize", int(fmt), _ptr(src), _ptr(dst), n, scale, _stream(stream))


def absmax(src, n: int, out, stream=None):
    call("tb_absmax", _ptr(src), n, _ptr(out), _stream(stream))


def gemm_f16(A, B, D, M: int, N: int, K: int, out=Out.F32, alpha: float = 1.0, stream=None):
    call("tb_gemm_f16", _ptr(A), _ptr(B), _ptr(D), M, N, K, int(out), alpha, _stream(stream))


def fused_workspace_bytes(fmt, M: int, N: int, K: int) -> int:
    return lib().tb_gemm_fused_workspace(int(fmt), M, N, K)


def gemm_fused(fmt, A, B, D, M: int, N: int, K: int, out=Out.F32, alpha: float = 1.0, workspace=None,
               workspace_bytes: int = 0, stream=None):
    call("tb_gemm_fused", int(fmt), _ptr(A), _ptr(B), _ptr(D), M, N, K, int(out), alpha, _ptr(workspace),
         workspace_bytes, _stream(stream))


def gemm_fused_noalloc(fmt, A, B, D, M: int, N: int, K: int, out=Out.F32, alpha: float = 1.0, stream=None):
    """tb_gemm_fused with split-K partial sums in the library's fixed scratch."""
    call("tb_gemm_fused_noalloc", int(fmt), _ptr(A), _ptr(B), _ptr(D), M, N, K, int(out), alpha, _stream(stream))


def gemm_native(a_fmt, A, b_fmt, B, D, M: int, N: int, K: int, out=Out.F32, alpha: float = 1.0, stream=None):
    call("tb_gemm_native", int(a_fmt), _ptr(A), int(b_fmt), _ptr(B), _ptr(D), M, N, K, int(out), alpha,
         _stream(stream))


def gemm_nvfp4(A, A_scales, B, B_scales, D, M: int, N: int, K: int, out=Out.F32, alpha: float = 1.0, stream=None):
    """Block-scaled FP4 GEMM: codes in the tensor-core nibble order (E2M1_HW),
    one UE4M3 scale byte per 16 values of a row (tcgen05 kind::mxf4nvf4)."""
    call("tb_gemm_nvfp4", _ptr(A), _ptr(A_scales), _ptr(B), _ptr(B_scales), _ptr(D), M, N, K, int(out), alpha,
         _stream(stream))


def decode_e4m3_to_i8(src, dst, n: int, scale: float, stream=None):
    """E4M3 codes -> INT8 with the reference's integer-path conversion."""
    call("tb_decode_e4m3_to_i8", _ptr(src), _ptr(dst), n, scale, _stream(stream))


def decode_e4m3_to_i8_transposed(src, dst, rows: int, cols: int, scale: float, stream=None):
    call("tb_decode_e4m3_to_i8_transposed", _ptr(src), _ptr(dst), rows, cols, scale, _stream(stream))


def gemm_i8(A, B, D, M: int, N: int, K: int, stream=None):
    """D [M x N] INT32 = A [M x K] INT8 * B [N x K] INT8 ^T (tcgen05 kind::i8)."""
    call("tb_gemm_i8", _ptr(A), _ptr(B), _ptr(D), M, N, K, _stream(stream))


def gemm_fp8_fused_int8(A, B, D, M: int, N: int, K: int, scale: float, workspace, workspace_bytes: int,
                        stream=None):
    call("tb_gemm_fp8_fused_int8", _ptr(A), _ptr(B), _ptr(D), M, N, K, scale, _ptr(workspace), workspace_bytes,
         _stream(stream))


def fp4_repack_hw(src, dst, n_bytes: int, stream=None):
    call("tb_fp4_repack_hw", _ptr(src), _ptr(dst), n_bytes, _stream(stream))


def device_error(clear: bool = True) -> int:
    code = ctypes.c_int(0)
    call("tb_device_error", ctypes.byref(code), 1 if clear else 0)
    return code.value


# ---- column-sharded weight GEMM (tb_gemm_sharded_fused) -------------------------------

def shard_blocks(M: int, world: int, chunks: int, rank: int):
    """Row blocks of a weight with M output rows that rank `rank` owns under the
    block-cyclic layout of tb_gemm_sharded_fused: world*chunks blocks of
    Mc = M / (world*chunks) rows; rank r owns blocks c*world + r, c < chunks.
    Returns [(first_global_row, Mc), ...] in shard order."""
    if M % (world * chunks * 128):
        raise ValueError(f"M = {M} must be a multiple of world*chunks*128 = {world * chunks * 128}")
    mc = M // (world * chunks)
    return [((c * world + rank) * mc, mc) for c in range(chunks)]


def shard_rows(A, M: int, world: int, chunks: int, rank: int):
    """This rank's A_shard from the full weight A (numpy array or torch tensor
    holding M rows of the stored format, any row width): its blocks stacked in
    block order, as tb_gemm_sharded_fused expects."""
    rows = A.reshape(M, -1)
    parts = [rows[r0:r0 + mc] for r0, mc in shard_blocks(M, world, chunks, rank)]
    if hasattr(rows, "new_empty"):  # torch
        import torch
        return torch.cat(parts).contiguous()
    import numpy as np
    return np.ascontiguousarray(np.concatenate(parts))


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    call("tb_nccl_unique_id", buf)
    return buf.raw


def nccl_comm_init(world: int, rank: int, uid: bytes) -> int:
    """An ncclComm_t (as an int handle) for this rank, from rank 0's unique id."""
    comm = ctypes.c_void_p()
    call("tb_nccl_comm_init", ctypes.byref(comm), world, rank, ctypes.create_string_buffer(bytes(uid), 128))
    return comm.value


def nccl_comm_destroy(comm: int):
    call("tb_nccl_comm_destroy", comm)


def gemm_sharded_fused(fmt, A_shard, B, D, M: int, N: int, K: int, comm: int, chunks: int, out=Out.F32,
                       alpha: float = 1.0, stream=None, comm_stream=None):
    """Fused GEMM of this rank's block-cyclic weight rows straight into D, with
    in-place NCCL all-gathers on comm_stream; every rank ends with all of D."""
    call("tb_gemm_sharded_fused", int(fmt), _ptr(A_shard), _ptr(B), _ptr(D), M, N, K, int(out), alpha, comm,
         chunks, _stream(stream), _ptr(comm_stream) if comm_stream is not None else _stream(None))


def peer_buffer_register(comm: int, D, nbytes: int = None, stream=None) -> int:
    """Collective: map every rank's device buffer D (a torch tensor or pointer;
    same byte size on all ranks) into the other ranks' processes for
    gemm_sharded_fused_p2p.  Returns the handle."""
    h = ctypes.c_void_p()
    if nbytes is None:
        nbytes = D.numel() * D.element_size()
    call("tb_peer_buffer_register", comm, _ptr(D), nbytes, _stream(stream), ctypes.byref(h))
    return h.value


def peer_buffer_release(handle: int, stream=None):
    """Collective: unmap the peers' buffers once every rank has reached it."""
    call("tb_peer_buffer_release", handle, _stream(stream))


def gemm_sharded_fused_p2p(fmt, A_shard, B, peer_buffer: int, M: int, N: int, K: int, chunks: int = 1,
                           out=Out.F32, alpha: float = 1.0, stream=None):
    """The sharded GEMM of gemm_sharded_fused whose fused-kernel epilogue stores
    every output tile into all ranks' registered D (peer_buffer) over NVLink;
    no NCCL data kernel."""
    call("tb_gemm_sharded_fused_p2p", int(fmt), _ptr(A_shard), _ptr(B), peer_buffer, M, N, K, int(out), alpha,
         chunks, _stream(stream))
