"""One rank of the multi-GPU sharded-GEMM test (launched by tests/test_sharded_gpu.py
through torch.distributed.run, two or four ranks).  gloo carries only the NCCL unique id; the
GEMM's all-gather (or, for the p2p path, its barriers and the peer-buffer exchange) runs on the
library's own NCCL communicator.

Both sharded paths are checked on every rank against the whole D: bit for bit
against the single-GPU fused GEMM (no workspace, so unsplit: the same
accumulation order over K) and against the oracle on a band of rows.  The p2p cases cover a ragged last tile column (N = 520), two
chunks, F16 and F32 output, and a row stride without 16-byte vectors
(N = 300, element copies); D is filled with NaN first, so every element must
have been written by the path under test."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402
import __graft_entry__ as ge  # noqa: E402
from gpu_util import to_dev, empty_dev, from_dev  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    tb = ge._import_package()
    uid = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(tb.nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = tb.nccl_comm_init(world, rank, bytes(uid.numpy()))
    try:
        cases = [("nccl", O.E4M3, tb.Out.F32, 2, (world * 2 * 128 * 3, 264, 512)),
                 ("nccl", O.E2M1, tb.Out.F16, 3, (world * 3 * 128 * 2, 72, 1024)),
                 ("p2p", O.E4M3, tb.Out.F32, 1, (world * 512, 520, 512)),
                 ("p2p", O.E2M1, tb.Out.F16, 2, (world * 2 * 384, 264, 1024)),
                 ("p2p", O.BF16, tb.Out.F16, 1, (world * 256, 300, 256))]
        for path, fmt, out, chunks, (M, N, K) in cases:
            a = O.normal(50 + fmt, (M, K), 0.02)
            s = O.per_tensor_scale(a, fmt)
            A = O.quantize(fmt, a, s)
            alpha = float(np.float32(1.0) / np.float32(s))
            B16 = O.f32_to_f16_bits(O.normal(51, (N, K), 1.0)).reshape(N, K)
            esz = 2 if out == tb.Out.F16 else 4
            dA_shard = to_dev(torch, tb.shard_rows(A, M, world, chunks, rank))
            dA, dB = to_dev(torch, A), to_dev(torch, B16)
            dD = empty_dev(torch, M * N * esz)
            dD.view(torch.uint8).fill_(0xFF)  # NaN in F16 and F32
            st, cst = torch.cuda.Stream(), torch.cuda.Stream()
            torch.cuda.synchronize()
            if path == "nccl":
                tb.gemm_sharded_fused(fmt, dA_shard, dB, dD, M, N, K, comm, chunks, out=out, alpha=alpha,
                                      stream=st.cuda_stream, comm_stream=cst.cuda_stream)
            else:
                h = tb.peer_buffer_register(comm, dD, stream=st.cuda_stream)
                try:
                    for _ in range(2):  # a second call into the same buffers
                        tb.gemm_sharded_fused_p2p(fmt, dA_shard, dB, h, M, N, K, chunks=chunks, out=out,
                                                  alpha=alpha, stream=st.cuda_stream)
                    st.synchronize()
                finally:
                    tb.peer_buffer_release(h, stream=st.cuda_stream)
            st.synchronize()
            cst.synchronize()
            dR = empty_dev(torch, M * N * esz)
            tb.gemm_fused(fmt, dA, dB, dR, M, N, K, out=out, alpha=alpha)
            torch.cuda.synchronize()
            got = from_dev(dD, np.uint8)
            ref = from_dev(dR, np.uint8)
            assert np.array_equal(got, ref), f"rank {rank} {path}: sharded D differs from the unsharded fused GEMM"
            rows = (M // 2 - 32, M // 2 + 32)
            want = O.gemm(fmt, A, O.F16, B16, M, N, K, rows=rows, alpha=alpha, out_f16=out == tb.Out.F16)
            g = got.view(np.uint16 if esz == 2 else np.float32).reshape(M, N)[rows[0]:rows[1]]
            if esz == 2:
                g, want = O.f16_bits_to_f32(g), O.f16_bits_to_f32(want)
            err = O.rel_frob(g, want)
            assert err <= 1e-3, f"rank {rank}: rel-Frobenius {err:.3e}"
            assert tb.device_error() == 0
        print(f"rank {rank} OK", flush=True)
    finally:
        tb.nccl_comm_destroy(comm)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
