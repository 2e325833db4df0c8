"""Host logic of the column-sharded GEMM, run as two gloo ranks on the CPU.

tb_gemm_sharded_fused splits the weight's output rows block-cyclically
(rank r owns blocks c*world + r), computes each block straight into its place
in D, and all-gathers block group c in place.  Here each rank takes its shard
with the package's shard_rows, computes its blocks with the oracle, writes
them at the same places and runs the same per-group all-gather over gloo; the
assembled D must equal the oracle's unsharded product bit for bit on every
rank.  The CUDA + NCCL version of the same contract is tests/test_sharded_gpu.py.
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, fmt_id: int, M: int, N: int, K: int, chunks: int):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "oracle"))
    sys.path.insert(0, root)
    import oracle as O
    import torch.distributed as dist
    import __graft_entry__ as ge
    tb = ge._import_package()

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        a = O.normal(40, (M, K), 0.02)
        s = O.per_tensor_scale(a, fmt_id)
        A = O.quantize(fmt_id, a, s)
        alpha = float(np.float32(1.0) / np.float32(s))
        B16 = O.f32_to_f16_bits(O.normal(41, (N, K), 1.0)).reshape(N, K)
        A_shard = tb.shard_rows(A, M, world, chunks, rank)
        blocks = tb.shard_blocks(M, world, chunks, rank)
        mc = blocks[0][1]
        D = torch.full((M, N), float("nan"), dtype=torch.float32)
        shard_rows = A_shard.reshape(chunks * mc, -1)
        for c, (g0, _) in enumerate(blocks):
            blk = shard_rows[c * mc:(c + 1) * mc]
            D[g0:g0 + mc] = torch.from_numpy(O.gemm(fmt_id, blk, O.F16, B16, mc, N, K, alpha=alpha))
            group = D[c * world * mc:(c + 1) * world * mc]
            parts = [torch.empty(mc, N) for _ in range(world)]
            dist.all_gather(parts, D[g0:g0 + mc].clone())
            for r in range(world):
                group[r * mc:(r + 1) * mc] = parts[r]
        want = O.gemm(fmt_id, A, O.F16, B16, M, N, K, alpha=alpha)
        np.testing.assert_array_equal(D.numpy().view(np.uint32), want.view(np.uint32))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt_name,chunks", [("E4M3", 2), ("E2M1", 1), ("BF16", 3)])
def test_block_cyclic_all_gather_two_ranks(fmt_name, chunks):
    import oracle as O
    fmt_id = getattr(O, fmt_name)
    world = 2
    M, N, K = world * chunks * 128 * 2, 40, 256
    torch.multiprocessing.spawn(_rank_main, args=(world, _free_port(), fmt_id, M, N, K, chunks), nprocs=world,
                                join=True)


def test_shard_blocks_layout(tb):
    assert tb.shard_blocks(1024, 2, 2, 0) == [(0, 256), (512, 256)]
    assert tb.shard_blocks(1024, 2, 2, 1) == [(256, 256), (768, 256)]
    # the 16384 x 53248 weight on 8 ranks: 4 chunks of 1664 rows (13 tiles)
    assert tb.shard_blocks(53248, 8, 4, 3)[1] == ((1 * 8 + 3) * 1664, 1664)
    # one chunk (the peer-store path's layout): each rank's M / world contiguous rows
    assert tb.shard_blocks(53248, 8, 1, 3) == [(3 * 6656, 6656)]
    with pytest.raises(ValueError):
        tb.shard_blocks(1000, 2, 2, 0)
    A = np.arange(1024 * 5, dtype=np.uint32).reshape(1024, 5)
    s = tb.shard_rows(A, 1024, 2, 2, 1)
    np.testing.assert_array_equal(s[:256], A[256:512])
    np.testing.assert_array_equal(s[256:], A[768:1024])
