"""GPU parity at the BASELINE full sizes (configs 1-4), checked on sampled rows.

The whole call runs on the GPU at full size; the fp64 oracle then recomputes a
sample of (sequence, head, query-row) outputs from the same inputs, and every
output is checked for size-independent properties (finite values, finite LSE,
rows of a head agreeing with their oracle rows).
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_gates, seeded

pytestmark = pytest.mark.gpu


def _sample_rows(L, n, seed):
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, 1, 127, 128, L - 1], rng.choice(L, n, replace=False)]))
    return rows


def _oracle_head_rows(q_in, k_in, v_in, n, h, rows, table, kv_type, mask_row=None, kv_len=None, table_q=None,
                      table_k=None, d=128):
    """fp64 oracle for query rows `rows` of head h, sequence n (prologue + flash, like the GPU call).
    table_q / table_k: RoPE rows for the given q rows and all keys, when q_in holds only those rows."""
    qs = q_in[n:n + 1, rows, h * d:(h + 1) * d]
    ks = k_in[n:n + 1, :, h * d:(h + 1) * d]
    vs = v_in[n:n + 1, :, h * d:(h + 1) * d]
    qn = oracle.rms_norm_heads(qs, d)
    kn = oracle.rms_norm_heads(ks, d)
    if table is not None:
        qn = oracle.rope_apply(qn, 1, d, table[rows])
        kn = oracle.rope_apply(kn, 1, d, table)
    if table_q is not None:
        qn = oracle.rope_apply(qn, 1, d, table_q)
        kn = oracle.rope_apply(kn, 1, d, table_k)
    q4 = qn[:, None]                                            # (1, 1, R, d)
    k4 = oracle.to_type(kn[:, None], kv_type)
    v4 = oracle.to_type(vs[:, None], kv_type)
    m = None if mask_row is None else mask_row[None, None]
    kl = None if kv_len is None else np.array([kv_len], np.int32)
    o, l = oracle.flash_attn_ext(q4, k4, v4, mask=m, kv_len=kl, mode=oracle.EXACT, lse=True)
    return o[0, :, 0], l[0, 0]


def test_config1_full_size_self_attention(ctx, kd):
    """B2 x 31,744 tokens (31x32x32) x 32 heads x d128, bf16 operands.  Eight
    (batch, head) planes are checked, the last one (1, 31) included, on rows that include the first
    and last rows of the first, a middle and the last 128-row tile."""
    N, L, H, d = 2, 31744, 32, 128
    C = H * d
    grid = (31, 32, 32)
    q = seeded((N, L, C), 1, 0)
    k = seeded((N, L, C), 1, 1)
    v = seeded((N, L, C), 1, 2)
    out = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(N, H, L, device="cuda")
    ctx.self_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), H, out,
                       rope=kd.Rope3D.make(grid), op_type=kd.BF16, lse=lse)
    ctx.device_status()
    o = out.float().cpu().numpy()
    ls = lse.cpu().numpy()
    assert np.all(np.isfinite(o)) and np.all(np.isfinite(ls))
    table = oracle.visual_rope_table(grid)
    edge = np.array([L // 2 - 1, L // 2, L - 129, L - 128, L - 2])
    for n, h in [(0, 0), (1, 31), (0, 17), (1, 0), (0, 31), (1, 7), (0, 9), (1, 23)]:
        rows = np.unique(np.concatenate([_sample_rows(L, 48, seed=n * 100 + h), edge]))
        ref, lref = _oracle_head_rows(q, k, v, n, h, rows, table, oracle.BF16)
        got = o[n, rows, h * d:(h + 1) * d]
        assert_gates(got, ref, lse=ls[n, h, rows], lse_ref=lref, label=f"cfg1 n{n} h{h}", out_type="bf16")


def _device_projections(ctx, N, L, C, seed):
    """Seeded f32 projections [C, L, N] made on the device (3 x N*L*C floats)."""
    out = []
    for off in range(3):
        t = torch.empty(N * L * C, device="cuda")
        ctx.fill_randn(t, seed=seed, offset=off)
        out.append(t.view(N, L, C))
    return out


def _head_slice(x, n, h, rows=None, d=128):
    """Host float32 copy of head h of sequence n (all rows, or `rows`), shape (1, R, d)."""
    t = x[n, :, h * d:(h + 1) * d] if rows is None else x[n, torch.as_tensor(rows, device=x.device), h * d:(h + 1) * d]
    return t.float().cpu().numpy()[None]


def test_config3_full_size_self_attention(ctx, kd):
    """B2 x 71,424 tokens (31x48x48 grid, 558 K/V tiles per plane) x 32 heads, bf16
    operands, the whole call on one GPU; sampled rows of four planes against the fp64 oracle."""
    N, L, H, d = 2, 71424, 32, 128
    C = H * d
    grid = (31, 48, 48)
    q, k, v = _device_projections(ctx, N, L, C, seed=33)
    out = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(N, H, L, device="cuda")
    ctx.self_attention(q, k, v, H, out, rope=kd.Rope3D.make(grid), op_type=kd.BF16, lse=lse)
    ctx.device_status()
    assert bool(torch.isfinite(out).all()) and bool(torch.isfinite(lse).all())
    table = oracle.visual_rope_table(grid)
    for n, h in [(0, 0), (1, 31), (0, 21), (1, 10)]:
        rows = _sample_rows(L, 64, seed=300 + n * 100 + h)
        qh, kh, vh = _head_slice(q, n, h, rows), _head_slice(k, n, h), _head_slice(v, n, h)
        ref, lref = _oracle_head_rows(qh, kh, vh, 0, 0, np.arange(len(rows)), None, oracle.BF16,
                                      table_q=table[rows], table_k=table)
        got = out[n, torch.as_tensor(rows, device="cuda"), h * d:(h + 1) * d].float().cpu().numpy()
        assert_gates(got, ref, lse=lse[n, h].cpu().numpy()[rows], lse_ref=lref, label=f"cfg3 n{n} h{h}",
                     out_type="bf16")


def test_config4_full_size_block_sparse(ctx, kd):
    """62,464 tokens (61x32x32), 32 heads, the 64x64 block mask of the benchmark
    (diagonal, +-1 latent frame over adjacent strips, 14 % seeded random tiles), one mask plane for all
    heads -- the head-pair instantiation.  The tile bitmap alone and the dense f16 mask (7.8 GB) give
    bit-identical outputs, the device counters equal the counts the bitmap implies, and sampled rows of
    four heads match the fp64 oracle with the row's mask."""
    from bench import block_sparse_tiles
    N, L, H, d = 1, 62464, 32, 128
    C = H * d
    grid = (61, 32, 32)
    keep = block_sparse_tiles(grid, 0.14)
    q, k, v = _device_projections(ctx, N, L, C, seed=44)
    qs = torch.empty(N, H, L, d, device="cuda", dtype=torch.bfloat16)
    ks, vs = torch.empty_like(qs), torch.empty_like(qs)
    ctx.qk_prologue(q, k, v, qs, ks, vs, rope=kd.Rope3D.make(grid))
    del q, k, v
    bits = torch.from_numpy(kd.tile_bitmap(keep)).cuda()
    out_b = torch.empty(N, L, H, d, device="cuda", dtype=torch.bfloat16)
    lse_b = torch.empty(N, H, L, device="cuda")
    ctx.tile_stats(reset=True)
    ctx.flash_attn_ext(qs, ks, vs, out_b, tile_mask=bits, lse=lse_b)
    loaded, pairs = ctx.tile_stats(reset=True)
    qt = keep.reshape(keep.shape[0] // 2, 2, keep.shape[1] // 2, 2).any(axis=(1, 3))
    assert loaded == int(qt.sum()) * N * H and pairs == int(qt.sum()) * N * H
    keep_t = torch.from_numpy(keep).cuda()
    mask = torch.zeros(1, 1, L, L, device="cuda", dtype=torch.float16)
    mask.view(L, L).masked_fill_(~keep_t.repeat_interleave(64, 0).repeat_interleave(64, 1), float("-inf"))
    out_m = torch.empty_like(out_b)
    ctx.flash_attn_ext(qs, ks, vs, out_m, mask=mask)
    ctx.device_status()
    assert torch.equal(out_b, out_m)
    del mask, out_m
    for h in (0, 13, 22, 31):
        rows = _sample_rows(L, 64, seed=400 + h)
        rsel = torch.as_tensor(rows, device="cuda")
        qh = qs[0, h, rsel].float().cpu().numpy()[None, None]
        kh = ks[0, h].float().cpu().numpy()[None, None]
        vh = vs[0, h].float().cpu().numpy()[None, None]
        mrow = np.where(np.repeat(np.repeat(keep[rows // 64], 64, axis=1), 1, axis=0)[:, :L], 0.0, -np.inf)
        mrow = mrow.astype(np.float16)[None, None]
        ref, lref = oracle.flash_attn_ext(qh, oracle.to_type(kh, oracle.BF16), oracle.to_type(vh, oracle.BF16),
                                          mask=mrow, mode=oracle.EXACT, lse=True)
        got = out_b[0, rsel, h].float().cpu().numpy()
        assert_gates(got, ref[0, :, 0], lse=lse_b[0, h, rsel].cpu().numpy(), lse_ref=lref[0, 0],
                     label=f"cfg4 h{h}", out_type="bf16")


@pytest.mark.parametrize("use_mask", [False, True])
def test_config2_full_size_cross_attention(ctx, kd, use_mask):
    """31,744 visual queries x 256 padded text keys, valid lengths U[40,256]."""
    N, Lq, Lk, H, d = 2, 31744, 256, 32, 128
    C = H * d
    rng = np.random.default_rng(2)
    kv_len = rng.integers(40, 257, size=N).astype(np.int32)
    q = seeded((N, Lq, C), 3, 0)
    text = seeded((N, Lk, C), 3, 1) * 0.5
    wk = seeded((C, C), 3, 2) / np.sqrt(C)
    wv = seeded((C, C), 3, 3) / np.sqrt(C)
    k = (text @ wk).astype(np.float32)
    v = (text @ wv).astype(np.float32)
    out = torch.empty(N, Lq, C, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(N, H, Lq, device="cuda")
    mask_np = None
    if use_mask:
        mask_np = np.zeros((N, 1, Lq, Lk), np.float16)
        for n in range(N):
            mask_np[n, 0, :, kv_len[n]:] = -np.inf
        ctx.cross_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), H,
                            out, mask=torch.from_numpy(mask_np).cuda(), op_type=kd.BF16, lse=lse)
    else:
        ctx.cross_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), H,
                            out, kv_len=torch.from_numpy(kv_len).cuda(), op_type=kd.BF16, lse=lse)
    ctx.device_status()
    o = out.float().cpu().numpy()
    assert np.all(np.isfinite(o))
    ls = lse.cpu().numpy()
    for n, h in [(0, 3), (1, 30)]:
        rows = _sample_rows(Lq, 128, seed=7 + n)
        ref, lref = _oracle_head_rows(q, k, v, n, h, rows, None, oracle.BF16, kv_len=int(kv_len[n]))
        got = o[n, rows, h * d:(h + 1) * d]
        assert_gates(got, ref, lse=ls[n, h, rows], lse_ref=lref, label=f"cfg2 n{n} h{h} mask={use_mask}", out_type="bf16")


def test_lite_video_full_size_self_attention(ctx, kd):
    """The lite video model at config 1's tokens: B2 x 31,744 tokens (31x32x32) x 28 heads x d64 (RoPE axes
    {16, 24, 24}, scale {1, 2, 2}), bf16 operands -- the head_dim-64 long-key kernel over 248 K/V tiles per
    plane; sampled rows of four planes, the last one (1, 27) included, against the fp64 oracle."""
    N, L, H, d = 2, 31744, 28, 64
    C = H * d
    grid, axes, scale = (31, 32, 32), (16, 24, 24), (1, 2, 2)
    q, k, v = _device_projections(ctx, N, L, C, seed=37)
    out = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(N, H, L, device="cuda")
    ctx.self_attention(q, k, v, H, out, rope=kd.Rope3D.make(grid, axes=axes, scale=scale), op_type=kd.BF16, lse=lse)
    ctx.device_status()
    assert bool(torch.isfinite(out).all()) and bool(torch.isfinite(lse).all())
    table = oracle.visual_rope_table(grid, axes=axes, scale=scale)
    for n, h in [(0, 0), (1, 27), (0, 13), (1, 6)]:
        rows = _sample_rows(L, 64, seed=700 + n * 100 + h)
        qh, kh, vh = _head_slice(q, n, h, rows, d), _head_slice(k, n, h, d=d), _head_slice(v, n, h, d=d)
        ref, lref = _oracle_head_rows(qh, kh, vh, 0, 0, np.arange(len(rows)), None, oracle.BF16,
                                      table_q=table[rows], table_k=table, d=d)
        got = out[n, torch.as_tensor(rows, device="cuda"), h * d:(h + 1) * d].float().cpu().numpy()
        assert_gates(got, ref, lse=lse[n, h].cpu().numpy()[rows], lse_ref=lref, label=f"lite n{n} h{h}",
                     out_type="bf16")
