"""kd_attn_qkv_projection: to_query/to_key/to_value (crossdit.hpp:123-125) as one tcgen05 GEMM whose
epilogue is the prologue (bias, per-head RMSNorm, 3D RoPE, cast, operand layout).

Every case is checked twice against the fp64 oracle (oracle.qkv_projection: numpy dequantization of the
ggml blocks, float64 matmul + bias, rounded to f32, then the prologue restatement):
  - on the exact operands (f32 x, dequantized weights) with the north-star gates -- the GEMM rounds x and
    the weights to bf16, which these gates absorb;
  - on the operands rounded to bf16 as the GEMM reads them, where only the fp32 accumulation order and the
    output rounding remain: max-abs beyond the output format's half ulp <= 2e-3 x RMS.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_gates, seeded

pytestmark = pytest.mark.gpu

TIGHT = 2e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_weight(kd, seed, off, C, K, wtype, bias=True):
    """Seeded N(0, 1/K) weight stored as `wtype` on the device; returns (KdLinear, keep-alive, dequantized
    f32 rows (C, K), bias f32 or None)."""
    w = seeded((C, K), seed, off) / np.float32(np.sqrt(K))
    b = (0.5 * seeded((C,), seed, off + 1)).astype(np.float32) if bias else None
    if wtype == kd.Q8_0:
        raw = oracle.quantize_q8_0(w)
    elif wtype == kd.Q4_0:
        raw = oracle.quantize_q4_0(w)
    elif wtype == kd.F16:
        raw = w.astype(np.float16)
    elif wtype == kd.BF16:
        raw = oracle.to_type(w, oracle.BF16).view(np.int16)
    else:
        raw = w
    deq = oracle.dequantize(raw.view(np.uint16) if wtype == kd.BF16 else raw, wtype, K)
    t = dev(raw)
    if wtype == kd.BF16:
        t = t.view(torch.bfloat16)
    bt = None if b is None else dev(b)
    return kd.KdLinear.of(t, wtype, K, C, bt), (t, bt), deq, b


def bf16_round(a):
    return oracle.to_f32(oracle.to_type(np.ascontiguousarray(a, np.float32), oracle.BF16), oracle.BF16)


def check(got, x, w, b, H, q_gain, k_gain, tab, out_type, label):
    """got: 3 device tensors (or None) (N, H, L, 128)."""
    exact = oracle.qkv_projection(x, w, b, H, q_gain, k_gain, tab)
    wr = [None if a is None else bf16_round(a) for a in w]
    rounded = oracle.qkv_projection(bf16_round(x), wr, b, H, q_gain, k_gain, tab)
    half = 2.0 ** -8 if out_type == "bf16" else 2.0 ** -11
    for name, g, e, r in zip("qkv", got, exact, rounded):
        if g is None:
            continue
        gn = g.float().cpu().numpy()
        assert_gates(gn, e, label=f"{label} {name} vs exact operands", out_type=out_type)
        rms = float(np.sqrt(np.mean(np.asarray(r, np.float64) ** 2)))
        excess = float(np.max(np.abs(gn - r) - np.abs(r) * half)) / rms
        assert excess <= TIGHT, f"{label} {name}: {excess:.3e} x RMS beyond {out_type} rounding vs bf16-rounded operands"


WTYPES = {"q8_0": 8, "q4_0": 2, "f16": 1, "bf16": 30, "f32": 0}


@pytest.mark.parametrize("wname", list(WTYPES))
def test_self_attention_projection_matches_oracle(ctx, kd, wname):
    """Q, K, V of self-attention from one x, every weight type, bias, gains, RoPE with scale (1, 2, 2);
    600 tokens = 4 full 128-row tiles and a ragged fifth."""
    N, grid, K, H = 2, (3, 10, 10), 1024, 8
    L, C = int(np.prod(grid)), H * 128
    x = seeded((N, L, K), 71, 0)
    lin = [make_weight(kd, 72, 10 * i, C, K, WTYPES[wname], bias=(i != 1)) for i in range(3)]
    q_gain = (1.0 + 0.1 * seeded((128,), 73, 0)).astype(np.float32)
    k_gain = (1.0 + 0.1 * seeded((128,), 73, 1)).astype(np.float32)
    tab = oracle.visual_rope_table(grid, scale=(1.0, 2.0, 2.0))
    outs = [torch.full((N, H, L, 128), float("nan"), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    ctx.qkv_projection(dev(x), lin[0][0], lin[1][0], lin[2][0], *outs, q_gain=dev(q_gain), k_gain=dev(k_gain),
                       rope=kd.Rope3D.make(grid, scale=(1.0, 2.0, 2.0)))
    ctx.device_status()
    check(outs, x, [l[2] for l in lin], [l[3] for l in lin], H, q_gain, k_gain, tab, "bf16", wname)


def test_model_width_q8_0_f16_operands(ctx, kd):
    """The Kandinsky 5 Pro width (4096 = 32 heads of 128) with q8_0 weights and f16 operands; unit gains."""
    N, grid, K, H = 1, (2, 10, 11), 4096, 32
    L, C = int(np.prod(grid)), H * 128
    x = seeded((N, L, K), 81, 0) * 2.0
    lin = [make_weight(kd, 82, 10 * i, C, K, kd.Q8_0) for i in range(3)]
    tab = oracle.visual_rope_table(grid)
    outs = [torch.empty((N, H, L, 128), device="cuda", dtype=torch.float16) for _ in range(3)]
    ctx.qkv_projection(dev(x), lin[0][0], lin[1][0], lin[2][0], *outs, rope=kd.Rope3D.make(grid))
    ctx.device_status()
    check(outs, x, [l[2] for l in lin], [l[3] for l in lin], H, None, None, tab, "f16", "width 4096")


def test_ragged_k_and_strided_x(ctx, kd):
    """in_features 544 (not a multiple of the 64-wide K step: the last step is zero-filled) and x given as a
    strided view (rows of a wider buffer)."""
    N, L, K, H = 2, 77, 544, 2
    C = H * 128
    wide = seeded((N, L, K + 32), 91, 0)
    x = wide[:, :, :K]
    lin = [make_weight(kd, 92, 10 * i, C, K, kd.F16) for i in range(3)]
    outs = [torch.empty((N, H, L, 128), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    ctx.qkv_projection(dev(wide)[:, :, :K], lin[0][0], lin[1][0], lin[2][0], *outs)
    ctx.device_status()
    check(outs, x, [l[2] for l in lin], [l[3] for l in lin], H, None, None, None, "bf16", "K=544")


def test_cross_attention_projections(ctx, kd):
    """Cross-attention (crossdit.hpp:174-200): Q alone from the visual tokens (RMSNorm, no RoPE), then K and
    V from 77 text tokens in a second call -- slots left out of the GEMM."""
    N, Lq, Lt, K, H = 2, 256, 77, 512, 4
    C = H * 128
    xv, xt = seeded((N, Lq, K), 95, 0), seeded((N, Lt, K), 95, 1)
    lq, lk, lv = (make_weight(kd, 96, 10 * i, C, K, kd.Q4_0) for i in range(3))
    q = torch.empty((N, H, Lq, 128), device="cuda", dtype=torch.bfloat16)
    k = torch.empty((N, H, Lt, 128), device="cuda", dtype=torch.bfloat16)
    v = torch.empty_like(k)
    ctx.qkv_projection(dev(xv), lq[0], None, None, q, None, None)
    ctx.qkv_projection(dev(xt), None, lk[0], lv[0], None, k, v)
    ctx.device_status()
    check([q, None, None], xv, [lq[2], None, None], [lq[3], None, None], H, None, None, None, "bf16", "cross q")
    check([None, k, v], xt, [None, lk[2], lv[2]], [None, lk[3], lv[3]], H, None, None, None, "bf16", "cross kv")


def test_projection_feeds_flash_attention(ctx, kd):
    """x -> kd_attn_qkv_projection -> kd_attn_flash_ext (bf16 operands, no copies between them) against
    the oracle's linear + self_attention on the exact operands."""
    N, grid, K, H = 1, (2, 8, 16), 512, 4
    L, C = int(np.prod(grid)), H * 128
    x = seeded((N, L, K), 101, 0)
    lin = [make_weight(kd, 102, 10 * i, C, K, kd.Q8_0) for i in range(3)]
    outs = [torch.empty((N, H, L, 128), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    ctx.qkv_projection(dev(x), lin[0][0], lin[1][0], lin[2][0], *outs, rope=kd.Rope3D.make(grid))
    o = torch.empty(N, L, H, 128, device="cuda")
    ctx.flash_attn_ext(*outs, o)
    ctx.device_status()
    proj = [oracle.linear(x, l[2], l[3]).astype(np.float32) for l in lin]
    ref = oracle.self_attention(*proj, H, rope_table=oracle.visual_rope_table(grid), kv_type=oracle.BF16,
                                q_type=oracle.BF16, mode=oracle.EXACT)
    m = oracle.parity_metrics(o.cpu().numpy().reshape(N, L, C), ref)
    assert m["cos"] >= 0.9999 and m["maxabs_over_rms"] <= 5e-2, m


def test_rejected_shapes(ctx, kd):
    K, C = 256, 256
    x = torch.zeros(1, 8, K, device="cuda")
    w = torch.zeros(C, K, device="cuda", dtype=torch.float16)
    lin = kd.KdLinear.of(w, kd.F16, K, C)
    out = torch.empty(1, 2, 8, 128, device="cuda", dtype=torch.bfloat16)
    for bad_out, status in ((torch.empty(1, 2, 8, 128, device="cuda"), kd.ERR_UNSUPPORTED),      # f32 operands
                            (torch.empty(1, 2, 9, 128, device="cuda", dtype=torch.bfloat16), kd.ERR_INVALID_ARGUMENT)):
        with pytest.raises(kd.KdAttnError) as e:
            ctx.qkv_projection(x, None, None, lin, None, None, bad_out)
        assert e.value.status == status
    w128 = torch.zeros(128, K, device="cuda", dtype=torch.float16)        # 128 output features: one head
    with pytest.raises(kd.KdAttnError) as e:
        ctx.qkv_projection(x, None, None, kd.KdLinear.of(w128, kd.F16, K, 128), None, None, out[:, :1])
    assert e.value.status == kd.ERR_UNSUPPORTED
    with pytest.raises(kd.KdAttnError) as e:                               # q4_1 is not a supported block type
        ctx.qkv_projection(x, None, None, kd.KdLinear.of(w, 3, K, C), None, None, out)
    assert e.value.status == kd.ERR_UNSUPPORTED
    with pytest.raises(kd.KdAttnError) as e:                               # a weight without its output
        ctx.qkv_projection(x, lin, None, None, None, None, None)
    assert e.value.status == kd.ERR_INVALID_ARGUMENT
    ctx.qkv_projection(x, None, None, lin, None, None, out)
    ctx.device_status()
    assert torch.count_nonzero(out.float()) == 0


# ------------------------------------------------------------------ kd_attn_linear and the whole block
def test_linear_matches_oracle(ctx, kd):
    """ops::linear through kd_attn_linear: f32 x, q8_0 weight with bias, f32 y against the fp64 product of
    the dequantized weight; 600 tokens (ragged last tile)."""
    N, L, K, C = 2, 300, 1024, 512
    x = seeded((N, L, K), 111, 0)
    lin, keep, deq, b = make_weight(kd, 112, 0, C, K, kd.Q8_0)
    y = torch.full((N, L, C), float("nan"), device="cuda")
    ctx.linear(dev(x), lin, y)
    ctx.device_status()
    exact = oracle.linear(x, deq, b)
    got = y.cpu().numpy()
    assert_gates(got, exact, label="linear vs exact operands")
    rounded = oracle.linear(bf16_round(x), bf16_round(deq), b)
    rms = float(np.sqrt(np.mean(rounded ** 2)))
    assert float(np.max(np.abs(got - rounded))) / rms <= TIGHT


def test_linear_bf16_input_read_in_place(ctx, kd):
    """bf16 x whose K is a whole number of K steps is read without a copy; f16 weight, bf16 y."""
    N, L, K, C = 1, 200, 512, 256
    xb = oracle.to_type(seeded((N, L, K), 121, 0), oracle.BF16)
    x = oracle.to_f32(xb, oracle.BF16)
    lin, keep, deq, b = make_weight(kd, 122, 0, C, K, kd.F16)
    y = torch.empty((N, L, C), device="cuda", dtype=torch.bfloat16)
    ctx.linear(torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16), lin, y)
    ctx.device_status()
    exact = oracle.linear(x, deq, b)
    assert_gates(y.float().cpu().numpy(), exact, label="bf16 linear", out_type="bf16")


def test_self_attention_block_matches_oracle(ctx, kd):
    """DiTSelfAttention::forward (crossdit.hpp:117-154) from the hidden states: q8_0 Q/K/V weights with
    biases, RMSNorm gains, 3D RoPE, f16 out-projection; against the oracle's linear -> RMSNorm -> RoPE ->
    flash_attn_ext -> linear chain on the exact operands (the block rounds x, the weights, the operands and
    the attention output to bf16)."""
    N, grid, C = 1, (2, 8, 16), 512
    H, L = C // 128, int(np.prod(grid))
    x = seeded((N, L, C), 131, 0)
    lin = [make_weight(kd, 132, 10 * i, C, C, kd.Q8_0) for i in range(3)]
    lo, keep_o, deq_o, b_o = make_weight(kd, 133, 0, C, C, kd.F16)
    q_gain = (1.0 + 0.1 * seeded((128,), 134, 0)).astype(np.float32)
    k_gain = (1.0 + 0.1 * seeded((128,), 134, 1)).astype(np.float32)
    y = torch.full((N, L, C), float("nan"), device="cuda")
    ctx.self_attention_block(dev(x), lin[0][0], lin[1][0], lin[2][0], lo, H, y, q_gain=dev(q_gain),
                             k_gain=dev(k_gain), rope=kd.Rope3D.make(grid))
    ctx.device_status()
    proj = [oracle.linear(x, l[2], l[3]).astype(np.float32) for l in lin]
    attn = oracle.self_attention(*proj, H, q_gain=q_gain, k_gain=k_gain, rope_table=oracle.visual_rope_table(grid),
                                 kv_type=oracle.BF16, q_type=oracle.BF16, mode=oracle.EXACT)
    ref = oracle.linear(attn, deq_o, b_o)
    m = oracle.parity_metrics(y.cpu().numpy(), ref)
    assert m["cos"] >= 0.9999 and m["maxabs_over_rms"] <= 5e-2, m


@pytest.mark.parametrize("N,L,K,C", [(1, 5, 32, 256), (3, 129, 96, 512), (2, 0, 64, 256)])
def test_small_and_degenerate_shapes(ctx, kd, N, L, K, C):
    """One K step that is mostly padding (K = 32), a single 256-feature tile, fewer tokens than one CTA
    pair's 256 rows, three sequences of 129 tokens, and zero tokens (nothing launched)."""
    H = C // 128
    x = seeded((N, L, K), 141, 0)
    lin = [make_weight(kd, 142, 10 * i, C, K, kd.Q4_0) for i in range(3)]
    outs = [torch.zeros((N, H, L, 128), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    ctx.qkv_projection(dev(x), lin[0][0], lin[1][0], lin[2][0], *outs)
    y = torch.zeros((N, L, C), device="cuda")
    ctx.linear(dev(x), lin[2][0], y)
    ctx.device_status()
    if L == 0:
        return
    check(outs, x, [l[2] for l in lin], [l[3] for l in lin], H, None, None, None, "bf16", f"small {N}x{L}x{K}")
    assert_gates(y.cpu().numpy(), oracle.linear(x, lin[2][2], lin[2][3]), label="small linear")


def test_cross_attention_block_matches_oracle(ctx, kd):
    """DiTCrossAttention::forward (crossdit.hpp:174-200): 256 visual queries against 77 text tokens with valid
    lengths {77, 40}, q4_0 Q/K/V weights with biases, RMSNorm gains, f16 out-projection; against the oracle's
    linear -> RMSNorm -> flash_attn_ext(kv_len) -> linear chain.  The same call with the valid lengths given
    as an f16 -inf mask instead gives the same output."""
    N, Lq, Lt, C = 2, 256, 77, 512
    H = C // 128
    xq, xt = seeded((N, Lq, C), 151, 0), seeded((N, Lt, C), 151, 1)
    lin = [make_weight(kd, 152, 10 * i, C, C, kd.Q4_0) for i in range(3)]
    lo, keep_o, deq_o, b_o = make_weight(kd, 153, 0, C, C, kd.F16)
    q_gain = (1.0 + 0.1 * seeded((128,), 154, 0)).astype(np.float32)
    k_gain = (1.0 + 0.1 * seeded((128,), 154, 1)).astype(np.float32)
    kv_len = np.array([77, 40], np.int32)
    y = torch.full((N, Lq, C), float("nan"), device="cuda")
    ctx.cross_attention_block(dev(xq), dev(xt), lin[0][0], lin[1][0], lin[2][0], lo, H, y, q_gain=dev(q_gain),
                              k_gain=dev(k_gain), kv_len=dev(kv_len))
    mask = np.zeros((N, 1, Lq, Lt), np.float16)
    mask[1, :, :, 40:] = -np.inf
    y2 = torch.full((N, Lq, C), float("nan"), device="cuda")
    ctx.cross_attention_block(dev(xq), dev(xt), lin[0][0], lin[1][0], lin[2][0], lo, H, y2, q_gain=dev(q_gain),
                              k_gain=dev(k_gain), mask=dev(mask))
    ctx.device_status()
    q = oracle.linear(xq, lin[0][2], lin[0][3]).astype(np.float32)
    k = oracle.linear(xt, lin[1][2], lin[1][3]).astype(np.float32)
    v = oracle.linear(xt, lin[2][2], lin[2][3]).astype(np.float32)
    attn = oracle.self_attention(q, k, v, H, q_gain=q_gain, k_gain=k_gain, kv_type=oracle.BF16, q_type=oracle.BF16,
                                 kv_len=kv_len, mode=oracle.EXACT)
    ref = oracle.linear(attn, deq_o, b_o)
    got = y.cpu().numpy()
    m = oracle.parity_metrics(got, ref)
    assert m["cos"] >= 0.9999 and m["maxabs_over_rms"] <= 5e-2, m
    m2 = oracle.parity_metrics(y2.cpu().numpy(), got)
    assert m2["cos"] >= 0.999999 and m2["maxabs_over_rms"] <= 1e-3, m2


def test_sharded_block_single_rank_equals_block(ctx, kd):
    """kd_attn_self_attention_block_sharded on a one-rank context (no peers to exchange with) writes the
    attention output into the caller's attn_full and equals kd_attn_self_attention_block bit for bit."""
    N, grid, C = 1, (2, 8, 8), 512
    L = int(np.prod(grid))
    x = seeded((N, L, C), 161, 0)
    lin = [make_weight(kd, 162, 10 * i, C, C, kd.Q8_0) for i in range(4)]
    rope = kd.Rope3D.make(grid)
    y = torch.empty((N, L, C), device="cuda")
    ctx.self_attention_block(dev(x), *(l[0] for l in lin), C // 128, y, rope=rope)
    attn_full = torch.empty((N, L, C), device="cuda", dtype=torch.bfloat16)
    y1 = torch.full((N, L, C), float("nan"), device="cuda")
    ctx.self_attention_block_sharded(dev(x), *(l[0] for l in lin), C // 128, attn_full, y1, rope=rope)
    ctx.device_status()
    assert torch.equal(y, y1)
    with pytest.raises(kd.KdAttnError):  # attn_full must be bf16
        ctx.self_attention_block_sharded(dev(x), *(l[0] for l in lin), C // 128, attn_full.float(), y1, rope=rope)
