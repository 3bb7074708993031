"""GPU parity at the BASELINE full sizes (configs 1 and 2), checked on sampled rows.

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


def _oracle_head_rows(q_in, k_in, v_in, n, h, rows, table, kv_type, mask_row=None, kv_len=None):
    """fp64 oracle for query rows `rows` of head h, sequence n (prologue + flash, like the GPU call)."""
    d = 128
    qs = q_in[n:n + 1, rows, h * d:(h + 1) * d]
    ks = k_in[n:n + 1, :, h * d:(h + 1) * d]
    vs = v_in[n:n + 1, :, h * d:(h + 1) * d]
    qn = oracle.rms_norm_heads(qs, d)
    kn = oracle.rms_norm_heads(ks, d)
    if table is not None:
        qn = oracle.rope_apply(qn, 1, d, table[rows])
        kn = oracle.rope_apply(kn, 1, d, table)
    q4 = qn[:, None]                                            # (1, 1, R, d)
    k4 = oracle.to_type(kn[:, None], kv_type)
    v4 = oracle.to_type(vs[:, None], kv_type)
    m = None if mask_row is None else mask_row[None, None]
    kl = None if kv_len is None else np.array([kv_len], np.int32)
    o, l = oracle.flash_attn_ext(q4, k4, v4, mask=m, kv_len=kl, mode=oracle.EXACT, lse=True)
    return o[0, :, 0], l[0, 0]


def test_config1_full_size_self_attention(ctx, kd):
    """B2 x 31,744 tokens (31x32x32) x 32 heads x d128, bf16 operands."""
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
    for n, h in [(0, 0), (1, 31), (0, 17)]:
        rows = _sample_rows(L, 96, seed=n * 100 + h)
        ref, lref = _oracle_head_rows(q, k, v, n, h, rows, table, oracle.BF16)
        got = o[n, rows, h * d:(h + 1) * d]
        assert_gates(got, ref, lse=ls[n, h, rows], lse_ref=lref, label=f"cfg1 n{n} h{h}", out_type="bf16")


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
