"""Head-sharded self-attention on 2 GPUs through the C ABI (skipped with fewer than 2 GPUs).

Rank r runs kd_attn_self_attention on its column shard of the config-1-like projections and
kd_attn_allgather_heads (one ncclAllGather + permute) rebuilds [C, L, N]; the result must equal
the single-GPU call on the full projections bit for bit (heads are independent and the kernels
are deterministic).  The fused exchange's result is also checked against the fp64 CPU oracle.  Child processes, one per GPU, 127.0.0.1 rendezvous, NVLS off.
"""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "kandinsky.cpp_b200"))
    import kd_attn
    from kd_attn.sharding import column_shard
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    obj = [kd_attn.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    N, H, d, grid = 2, 8, 128, (4, 16, 16)
    L, C = grid[0] * grid[1] * grid[2], H * d
    rope = kd_attn.Rope3D.make(grid, scale=(1, 2, 2))
    with kd_attn.Context(device=rank, n_ranks=world, rank=rank, nccl_id=obj[0]) as ctx:
        full_in = []
        for off in range(3):
            t = torch.empty(N * L * C, device="cuda")
            ctx.fill_randn(t, seed=77, offset=off)            # same full projections on every rank
            full_in.append(t.view(N, L, C))
        shard_in = [column_shard(x, rank, world, H).contiguous() for x in full_in]
        Hs = H // world
        shard_out = torch.empty(N, L, Hs * d, device="cuda", dtype=torch.bfloat16)
        ctx.self_attention(*shard_in, Hs, shard_out, rope=rope, op_type=kd_attn.BF16)
        gathered = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
        ctx.allgather_heads(shard_out.view(N, L, Hs, d), gathered.view(N, L, H, d))
        ctx.device_status()
        if rank == 0:
            with kd_attn.Context(device=0) as single:
                ref = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
                single.self_attention(*full_in, H, ref, rope=rope, op_type=kd_attn.BF16)
                single.device_status()
            torch.save({"got": gathered.cpu(), "ref": ref.cpu()}, os.path.join(out_dir, "r0.pt"))
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_two_gpu_head_sharding_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r = torch.load(os.path.join(str(tmp_path), "r0.pt"))
    assert torch.equal(r["got"], r["ref"])


def _rank_main_fused(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "kandinsky.cpp_b200"))
    import kd_attn
    from kd_attn.sharding import column_shard
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    obj = [kd_attn.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    N, H, d, grid = 2, 8, 128, (4, 16, 16)
    L, C = grid[0] * grid[1] * grid[2], H * d
    rope = kd_attn.Rope3D.make(grid, scale=(1, 2, 2))
    res = {}
    with kd_attn.Context(device=rank, n_ranks=world, rank=rank, nccl_id=obj[0]) as ctx:
        full_in = []
        for off in range(3):
            t = torch.empty(N * L * C, device="cuda")
            ctx.fill_randn(t, seed=78, offset=off)
            full_in.append(t.view(N, L, C))
        shard_in = [column_shard(x, rank, world, H).contiguous() for x in full_in]
        Hs = H // world
        for dt in (torch.float32, torch.bfloat16):
            out_full = ctx.symmetric_tensor((N, L, C), dt)
            out_full.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier(device_ids=[rank])
            for _ in range(2):    # the second call overwrites the first in place
                ctx.self_attention_sharded(*shard_in, Hs, out_full, rope=rope, op_type=kd_attn.BF16)
            ctx.device_status()
            with kd_attn.Context(device=rank) as single:
                ref = torch.empty(N, L, C, device="cuda", dtype=dt)
                single.self_attention(*full_in, H, ref, rope=rope, op_type=kd_attn.BF16)
                single.device_status()
            res[str(dt)] = (out_full.cpu(), ref.cpu())
            # cross-attention against text states of 77 tokens, valid lengths per sequence
            Lt = 77
            kt = torch.empty(N * Lt * C, device="cuda"); ctx.fill_randn(kt, seed=79, offset=0)
            vt = torch.empty(N * Lt * C, device="cuda"); ctx.fill_randn(vt, seed=79, offset=1)
            kt, vt = kt.view(N, Lt, C), vt.view(N, Lt, C)
            kv_len = torch.tensor([77, 40], dtype=torch.int32, device="cuda")
            out_full.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier(device_ids=[rank])
            ctx.cross_attention_sharded(shard_in[0], column_shard(kt, rank, world, H).contiguous(),
                                        column_shard(vt, rank, world, H).contiguous(), Hs, out_full, kv_len=kv_len,
                                        op_type=kd_attn.BF16)
            ctx.device_status()
            with kd_attn.Context(device=rank) as single:
                ref = torch.empty(N, L, C, device="cuda", dtype=dt)
                single.cross_attention(full_in[0], kt, vt, H, ref, kv_len=kv_len, op_type=kd_attn.BF16)
                single.device_status()
            res[str(dt) + " cross"] = (out_full.cpu(), ref.cpu())
            ctx.symmetric_free(out_full)
        if rank == 0:
            res["inputs"] = [x.cpu() for x in full_in]
    torch.save(res, os.path.join(out_dir, f"fused_r{rank}.pt"))
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_two_gpu_fused_exchange_matches_single_gpu(tmp_path):
    """kd_attn_self_attention_sharded: each rank's flash epilogue stores its heads into both ranks'
    symmetric out_full; every rank must end with the full single-GPU result, bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_rank_main_fused, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        res = torch.load(os.path.join(str(tmp_path), f"fused_r{r}.pt"))
        inputs = res.pop("inputs", None)
        for got, ref in res.values():
            assert torch.equal(got, ref)
        if inputs is not None:
            # every rank's exchanged copy also against the fp64 CPU oracle (both ranks' heads)
            import oracle
            from helpers import assert_gates
            q, k, v = (x.numpy() for x in inputs)
            tab = oracle.visual_rope_table((4, 16, 16), scale=(1, 2, 2))
            exact = oracle.self_attention(q, k, v, 8, rope_table=tab, kv_type=oracle.BF16, mode=oracle.EXACT)
            got = res[str(torch.float32)][0].numpy()
            assert_gates(got, exact, label="2-GPU fused exchange (f32 out) vs oracle")


def _rank_main_block(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "kandinsky.cpp_b200"))
    import kd_attn
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    obj = [kd_attn.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    N, H, d, grid = 2, 8, 128, (4, 16, 16)
    L, C = grid[0] * grid[1] * grid[2], H * d
    Cl = C // world
    rope = kd_attn.Rope3D.make(grid, scale=(1, 2, 2))
    g = torch.Generator(device="cuda").manual_seed(91)      # the same weights on every rank
    ws = [(torch.randn(C, C, device="cuda", generator=g) / 32).to(torch.float16) for _ in range(4)]
    bs = [torch.randn(C, device="cuda", generator=g) * 0.1 for _ in range(4)]
    gains = [1 + 0.1 * torch.randn(128, device="cuda", generator=g) for _ in range(2)]
    res = {}
    with kd_attn.Context(device=rank, n_ranks=world, rank=rank, nccl_id=obj[0]) as ctx:
        x = torch.empty(N * L * C, device="cuda")
        ctx.fill_randn(x, seed=92, offset=0)
        x = x.view(N, L, C)
        rows = slice(rank * Cl, (rank + 1) * Cl)              # this rank's heads' output features
        shard = [kd_attn.KdLinear.of(ws[i][rows], kd_attn.F16, C, Cl, bs[i][rows]) for i in range(3)]
        wo = kd_attn.KdLinear.of(ws[3], kd_attn.F16, C, C, bs[3])
        attn_full = ctx.symmetric_tensor((N, L, C), torch.bfloat16)
        y = torch.full((N, L, C), float("nan"), device="cuda")
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        for _ in range(2):    # the second call overwrites the first in place
            ctx.self_attention_block_sharded(x, *shard, wo, Cl // 128, attn_full, y, q_gain=gains[0], k_gain=gains[1],
                                             rope=rope)
        ctx.device_status()
        # y in a symmetric buffer: each rank computes its half of the token rows of the out-projection and
        # stores them into both copies of y
        ys = ctx.symmetric_tensor((N, L, C), torch.float32)
        ys.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        for _ in range(2):
            ctx.self_attention_block_sharded(x, *shard, wo, Cl // 128, attn_full, ys, q_gain=gains[0],
                                             k_gain=gains[1], rope=rope)
        ctx.device_status()
        with kd_attn.Context(device=rank) as single:
            full = [kd_attn.KdLinear.of(ws[i], kd_attn.F16, C, C, bs[i]) for i in range(4)]
            ref = torch.empty(N, L, C, device="cuda")
            single.self_attention_block(x, *full, C // 128, ref, q_gain=gains[0], k_gain=gains[1], rope=rope)
            single.device_status()
        res["y"] = (y.cpu(), ref.cpu())
        res["y_row_sharded"] = ys.cpu()
        ctx.symmetric_free(ys)
        ctx.symmetric_free(attn_full)
    torch.save(res, os.path.join(out_dir, f"block_r{rank}.pt"))
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_two_gpu_sharded_block_matches_single_gpu(tmp_path):
    """kd_attn_self_attention_block_sharded: each rank projects and attends its heads from its weight
    shards, the exchange fills every rank's attn_full, and out_layer runs either on every rank (y a plain
    buffer) or on each rank's half of the token rows with the rows stored into both copies (y symmetric);
    each rank's y must equal the single-GPU kd_attn_self_attention_block bit for bit both ways."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_rank_main_block, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        saved = torch.load(os.path.join(str(tmp_path), f"block_r{r}.pt"))
        got, ref = saved["y"]
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref)
        assert torch.equal(saved["y_row_sharded"], ref)
