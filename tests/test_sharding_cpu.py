"""Head-sharded attention on CPU ranks (gloo, world size 2): the partition and gather logic.

Each rank takes its column shard of the Q/K/V projections, runs the oracle's self-attention on
its heads, all-gathers the head outputs rank-major (what kd_attn_allgather_heads does with NCCL)
and unshards them; the result must equal the unsharded oracle bit for bit, since heads are
independent.  No GPU is involved.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(N, L, H, d):
    sys.path.insert(0, ROOT)
    import oracle
    C = H * d
    q = oracle.philox_randn(5, N * L * C, 0).reshape(N, L, C)
    k = oracle.philox_randn(5, N * L * C, 1).reshape(N, L, C)
    v = oracle.philox_randn(5, N * L * C, 2).reshape(N, L, C)
    return q, k, v, oracle.visual_rope_table((2, 4, 8))


def _rank_main(rank, world, port, out_path):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "kandinsky.cpp_b200"))
    os.environ["KD_ORACLE_THREADS"] = "2"
    import oracle
    from kd_attn.sharding import column_shard, head_range, unshard_rank_major
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    N, L, H, d = 2, 64, 4, 128
    q, k, v, tab = _inputs(N, L, H, d)
    h0, h1 = head_range(rank, world, H)
    qs, ks, vs = (np.ascontiguousarray(column_shard(x, rank, world, H)) for x in (q, k, v))
    shard = oracle.self_attention(qs, ks, vs, h1 - h0, rope_table=tab, kv_type=oracle.BF16, mode=oracle.EXACT)
    local = torch.from_numpy(shard.reshape(N * L, -1))
    gathered = torch.empty(world * N * L, local.shape[1])         # rank-major concatenation
    dist.all_gather_into_tensor(gathered, local)
    full = unshard_rank_major(gathered.view(world, N * L, -1), world).reshape(N, L, H * d).numpy()
    if rank == 0:
        np.save(out_path, full)
    dist.barrier()
    dist.destroy_process_group()


def test_head_sharding_gather_matches_unsharded(tmp_path):
    import oracle
    out = str(tmp_path / "full.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    N, L, H, d = 2, 64, 4, 128
    q, k, v, tab = _inputs(N, L, H, d)
    ref = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=oracle.BF16, mode=oracle.EXACT)
    np.testing.assert_array_equal(np.load(out), ref)


def test_head_range_rejects_uneven_split():
    sys.path.insert(0, os.path.join(ROOT, "kandinsky.cpp_b200"))
    from kd_attn.sharding import head_range
    assert head_range(3, 8, 32) == (12, 16)
    with pytest.raises(ValueError):
        head_range(0, 3, 32)
