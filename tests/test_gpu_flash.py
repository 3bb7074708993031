"""GPU parity: libkd_attn (through its C ABI) against the CPU oracle on identical seeded inputs."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_gates, lse_err, seeded

pytestmark = pytest.mark.gpu

TT = {oracle.F16: torch.float16, oracle.BF16: torch.bfloat16}


def dev(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def op_tensor(a_np, t):
    """numpy f32 -> device tensor of operand type t, rounded exactly like the oracle (RNE)."""
    bits = oracle.to_type(a_np, t)
    if t == oracle.F16:
        return torch.from_numpy(bits).cuda()
    return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)


# ------------------------------------------------------------------ config 0: the tiny self-attention block
@pytest.mark.parametrize("kv_type", [oracle.F16, oracle.BF16])
@pytest.mark.parametrize("scale", [(1, 1, 1), (1, 2, 2)])
def test_config0_self_attention(ctx, kd, kv_type, scale):
    """1,280 tokens (5x16x16), 32 heads, d128, RMSNorm + 3D RoPE, K/V cast."""
    N, L, H, d = 1, 1280, 32, 128
    C = H * d
    q = seeded((N, L, C), 2024, 0)
    k = seeded((N, L, C), 2024, 1)
    v = seeded((N, L, C), 2024, 2)
    tab = oracle.visual_rope_table((5, 16, 16), scale=scale)
    exact, lse_ref = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=kv_type, mode=oracle.EXACT, lse=True)
    ggml = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=kv_type, mode=oracle.GGML)
    out = torch.empty(N, L, C, device="cuda")
    lse = torch.empty(N, H, L, device="cuda")
    rope = kd.Rope3D.make((5, 16, 16), scale=scale)
    ctx.self_attention(dev(q), dev(k), dev(v), H, out, rope=rope, op_type=kv_type, lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, ggml, lse.cpu().numpy(), lse_ref, label=f"cfg0 {kv_type} {scale}")


# ------------------------------------------------------------------ flash_attn_ext on edge shapes
SHAPES = [  # N, H, Hkv, Lq, Lk
    (1, 1, 1, 1, 1), (1, 2, 2, 63, 40), (1, 2, 1, 64, 127), (2, 2, 2, 65, 128), (1, 1, 1, 127, 129),
    (1, 2, 2, 129, 255), (2, 4, 2, 255, 256), (1, 1, 1, 257, 300), (1, 2, 2, 256, 1), (1, 1, 1, 513, 640),
]


@pytest.mark.parametrize("N,H,Hkv,Lq,Lk", SHAPES)
@pytest.mark.parametrize("kv_type", [oracle.F16, oracle.BF16])
def test_flash_ext_shapes(ctx, N, H, Hkv, Lq, Lk, kv_type):
    D = 128
    qf = seeded((N, H, Lq, D), 7 + Lq, 0)
    kf = seeded((N, Hkv, Lk, D), 7 + Lq, 1)
    vf = seeded((N, Hkv, Lk, D), 7 + Lq, 2)
    kb, vb = oracle.to_type(kf, kv_type), oracle.to_type(vf, kv_type)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mode=oracle.EXACT, lse=True)
    out = torch.empty(N, Lq, H, D, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, kv_type), op_tensor(vf, kv_type), out, lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=f"{N,H,Hkv,Lq,Lk}")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_flash_ext_output_types_and_strided_q(ctx, out_dtype):
    """Q given as the strided f32 view ops::attention builds (permute of [C, L, N]); out in 3 types."""
    N, L, H, D = 2, 300, 4, 128
    q_in = seeded((N, L, H * D), 99, 0)
    kf = seeded((N, H, L, D), 99, 1)
    vf = seeded((N, H, L, D), 99, 2)
    kb, vb = oracle.to_type(kf, oracle.BF16), oracle.to_type(vf, oracle.BF16)
    qf = np.ascontiguousarray(q_in.reshape(N, L, H, D).transpose(0, 2, 1, 3))
    exact = oracle.flash_attn_ext(qf, kb, vb, mode=oracle.EXACT)
    qd = dev(q_in).view(N, L, H, D).permute(0, 2, 1, 3)          # strided: ggml [D, L, H, N] view
    out = torch.empty(N, L, H, D, device="cuda", dtype=out_dtype)
    ctx.flash_attn_ext(qd, op_tensor(kf, oracle.BF16), op_tensor(vf, oracle.BF16), out)
    ctx.device_status()
    ot = {torch.float32: None, torch.bfloat16: "bf16", torch.float16: "f16"}[out_dtype]
    assert_gates(out.float().cpu().numpy(), exact, label=str(out_dtype), out_type=ot)


# ------------------------------------------------------------------ masks, kv_len, fully masked rows
def _mask_case(kind, N, Lq, Lk, seed):
    rng = np.random.default_rng(seed)
    if kind == "random":          # per-element -inf plus finite additive values: mixed tiles
        m = (rng.normal(size=(N, 1, Lq, Lk)) * 0.5).astype(np.float16)
        m[rng.random(m.shape) < 0.25] = -np.inf
    elif kind == "block":         # 64x64 block-sparse with a kept diagonal
        nb_q, nb_k = (Lq + 63) // 64, (Lk + 63) // 64
        keep = rng.random((nb_q, nb_k)) < 0.3
        for i in range(min(nb_q, nb_k)):
            keep[i, i] = True
        m = np.where(np.kron(keep, np.ones((64, 64)))[:Lq, :Lk], 0, -np.inf).astype(np.float16)[None, None]
        m = np.repeat(m, N, axis=0)
    elif kind == "rows":          # some fully masked rows and a masked head block
        m = np.zeros((N, 1, Lq, Lk), np.float16)
        m[:, :, ::7, :] = -np.inf
        m[:, :, :64, 128:] = -np.inf
    else:
        raise ValueError(kind)
    return m


@pytest.mark.parametrize("kind", ["random", "block", "rows"])
def test_flash_ext_masks(ctx, kind):
    N, H, Lq, Lk, D = 2, 2, 320, 384, 128
    qf = seeded((N, H, Lq, D), 31, 0)
    kf = seeded((N, H, Lk, D), 31, 1)
    vf = seeded((N, H, Lk, D), 31, 2)
    kb, vb = oracle.to_type(kf, oracle.F16), oracle.to_type(vf, oracle.F16)
    mask = _mask_case(kind, N, Lq, Lk, 5)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mask=mask, mode=oracle.EXACT, lse=True)
    out = torch.empty(N, Lq, H, D, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, oracle.F16), op_tensor(vf, oracle.F16), out,
                       mask=torch.from_numpy(mask).cuda(), lse=lse)
    ctx.device_status()
    got = out.cpu().numpy()
    assert_gates(got, exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=kind)
    dead = np.isneginf(lse_ref).transpose(0, 2, 1)                   # (N, Lq, H)
    assert np.all(got[dead] == 0)


def test_flash_ext_kv_len(ctx):
    N, H, Lq, Lk, D = 3, 2, 200, 256, 128
    qf = seeded((N, H, Lq, D), 41, 0)
    kf = seeded((N, H, Lk, D), 41, 1)
    vf = seeded((N, H, Lk, D), 41, 2)
    kv_len = np.array([40, 256, 0], np.int32)
    kb, vb = oracle.to_type(kf, oracle.BF16), oracle.to_type(vf, oracle.BF16)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, kv_len=kv_len, mode=oracle.EXACT, lse=True)
    out = torch.full((N, Lq, H, D), 7.0, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, oracle.BF16), op_tensor(vf, oracle.BF16), out,
                       kv_len=torch.from_numpy(kv_len).cuda(), lse=lse)
    ctx.device_status()
    got = out.cpu().numpy()
    assert np.all(got[2] == 0) and np.all(np.isneginf(lse.cpu().numpy()[2]))
    assert_gates(got[:2], exact[:2], lse=lse.cpu().numpy()[:2], lse_ref=lse_ref[:2], label="kv_len")


@pytest.mark.parametrize("kv_type", [oracle.F16, oracle.BF16])
def test_flash_ext_kv_len_remainders(ctx, kv_type):
    """Valid lengths at every kind of remainder of the 128-key tile and of its 16-key MMA steps, through
    the short-key instantiation (keys past the valid length masked in the softmax, padded chunks zero)."""
    kv_len = np.array([1, 15, 16, 17, 100, 128, 129, 200, 255, 256], np.int32)
    N, H, Lq, Lk, D = len(kv_len), 2, 130, 256, 128
    qf = seeded((N, H, Lq, D), 43, 0)
    kf = seeded((N, H, Lk, D), 43, 1)
    vf = seeded((N, H, Lk, D), 43, 2)
    kb, vb = oracle.to_type(kf, kv_type), oracle.to_type(vf, kv_type)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, kv_len=kv_len, mode=oracle.EXACT, lse=True)
    out = torch.full((N, Lq, H, D), 7.0, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, kv_type), op_tensor(vf, kv_type), out,
                       kv_len=torch.from_numpy(kv_len).cuda(), lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=f"kv_len remainders {kv_type}")


def test_mask_broadcast_over_heads_and_sequences(ctx):
    """mask planes (mh, mn) broadcast as h % mh, n % mn (ggml's rule)."""
    N, H, Lq, Lk, D = 2, 4, 130, 200, 128
    qf = seeded((N, H, Lq, D), 51, 0)
    kf = seeded((N, H, Lk, D), 51, 1)
    vf = seeded((N, H, Lk, D), 51, 2)
    rng = np.random.default_rng(1)
    mask = (rng.normal(size=(1, 2, Lq, Lk))).astype(np.float16)
    mask[rng.random(mask.shape) < 0.5] = -np.inf
    kb, vb = oracle.to_type(kf, oracle.F16), oracle.to_type(vf, oracle.F16)
    exact = oracle.flash_attn_ext(qf, kb, vb, mask=mask, mode=oracle.EXACT)
    out = torch.empty(N, Lq, H, D, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, oracle.F16), op_tensor(vf, oracle.F16), out,
                       mask=torch.from_numpy(mask).cuda())
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, label="broadcast")


# ------------------------------------------------------------------ prologue and generator
@pytest.mark.parametrize("scale", [(1, 1, 1), (1, 2, 2)])
def test_prologue_matches_oracle(ctx, kd, scale):
    N, L, H, d = 2, 60, 3, 128
    x = seeded((N, L, H * d), 61, 0) * 3.0
    gain = (1.0 + 0.1 * seeded((d,), 61, 1)).astype(np.float32)
    tab = oracle.visual_rope_table((3, 4, 5), scale=scale)
    ref = oracle.prologue(x, H, gain=gain, rope_table=tab)                 # (N, H, L, d) f32
    y = torch.empty(N, H, L, d, device="cuda")
    ctx.prologue(dev(x), H, y, norm=True, gain=dev(gain), rope=kd.Rope3D.make((3, 4, 5), scale=scale))
    ctx.device_status()
    got = y.cpu().numpy()
    # float ops replicate the reference's; sin/cos may differ by an ulp from the host libm
    np.testing.assert_allclose(got, ref, rtol=0, atol=4e-6)
    yb = torch.empty(N, H, L, d, device="cuda", dtype=torch.bfloat16)
    ctx.prologue(dev(x), H, yb, norm=True, gain=dev(gain), rope=kd.Rope3D.make((3, 4, 5), scale=scale))
    rb = oracle.to_f32(oracle.to_type(ref, oracle.BF16), oracle.BF16)
    diff = np.abs(yb.float().cpu().numpy() - rb)
    assert np.mean(diff == 0) > 0.999 and np.all(diff <= np.abs(rb) * 2 ** -7 + 1e-30)
    # V path: no norm, no RoPE: an exact cast + permute
    yv = torch.empty(N, H, L, d, device="cuda", dtype=torch.float16)
    ctx.prologue(dev(x), H, yv, norm=False)
    np.testing.assert_array_equal(yv.cpu().numpy(), x.reshape(N, L, H, d).transpose(0, 2, 1, 3).astype(np.float16))


def test_fill_randn_matches_oracle(ctx):
    n = 1 << 20
    t = torch.empty(n, device="cuda")
    ctx.fill_randn(t, seed=42, offset=3)
    ref = oracle.philox_randn(42, n, 3)
    got = t.cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=2e-6)     # libm sin/log/sqrt ulp differences only


# ------------------------------------------------------------------ ops::attention mirror
def test_ops_attention_mirror(ctx, kd):
    """kd_attn.attention = ops::attention flash branch: [C, L, N] f32 in, f16 K/V, [C, Lq, N] f32 out."""
    N, Lq, Lk, H, d = 1, 200, 77, 4, 128
    q = seeded((N, Lq, H * d), 71, 0)
    k = seeded((N, Lk, H * d), 71, 1)
    v = seeded((N, Lk, H * d), 71, 2)
    q4 = np.ascontiguousarray(q.reshape(N, Lq, H, d).transpose(0, 2, 1, 3))
    k4 = oracle.to_type(np.ascontiguousarray(k.reshape(N, Lk, H, d).transpose(0, 2, 1, 3)), oracle.F16)
    v4 = oracle.to_type(np.ascontiguousarray(v.reshape(N, Lk, H, d).transpose(0, 2, 1, 3)), oracle.F16)
    exact = oracle.flash_attn_ext(q4, k4, v4, mode=oracle.EXACT).reshape(N, Lq, H * d)
    got = kd.attention(ctx, dev(q), dev(k), dev(v), H)
    ctx.device_status()
    assert_gates(got.cpu().numpy(), exact, label="ops::attention")


# ------------------------------------------------------------------ argument errors come back as statuses
def test_rejects_unsupported_and_invalid(ctx, kd):
    q = torch.zeros(1, 2, 16, 96, device="cuda", dtype=torch.float16)   # head_dim 96: not a CrossDiT head
    out = torch.empty(1, 16, 2, 96, device="cuda")
    with pytest.raises(kd.KdAttnError) as e:
        ctx.flash_attn_ext(q, q, q, out)
    assert e.value.status == kd.ERR_UNSUPPORTED
    q = torch.zeros(1, 2, 16, 128, device="cuda", dtype=torch.float16)
    bad_out = torch.empty(1, 16, 3, 128, device="cuda")
    with pytest.raises(kd.KdAttnError) as e:
        ctx.flash_attn_ext(q, q, q, bad_out)
    assert e.value.status == kd.ERR_INVALID_ARGUMENT
    with pytest.raises(kd.KdAttnError) as e:
        ctx.flash_attn_ext(q, q, q, torch.empty(1, 16, 2, 128, device="cuda"), max_bias=1.0)
    assert e.value.status == kd.ERR_UNSUPPORTED
    ctx.device_status()


# ------------------------------------------------------------------ host-buffer pipelined entry point
@pytest.mark.parametrize("H,grid,N,out_dtype,pinned,gap", [
    (32, (5, 16, 16), 1, torch.float32, True, 0),     # config 0 shape: 4 groups of 8 heads
    (6, (2, 8, 12), 2, torch.bfloat16, True, 0),      # 6 groups of 1 head, two sequences
    (3, (1, 9, 13), 2, torch.float32, False, 5),      # fewer heads than 4 groups, pageable, sequence gaps
])
def test_self_attention_host_matches_device_path(ctx, kd, H, grid, N, out_dtype, pinned, gap):
    """kd_attn_self_attention_host (upload / compute / download by head group) must equal the
    device-buffer call on the same projections bit for bit, whatever the host layout."""
    L, C = grid[0] * grid[1] * grid[2], H * 128
    rope = kd.Rope3D.make(grid, scale=(1, 2, 2))
    ins = []
    for off in range(3):
        x = torch.from_numpy(seeded((N, L + gap, C), 99, off))
        ins.append((x.pin_memory() if pinned else x)[:, :L])   # gap rows between sequences
    ref = torch.empty(N, L, C, device="cuda", dtype=out_dtype)
    ctx.self_attention(*[x.cuda() for x in ins], H, ref, rope=rope, op_type=kd.BF16)
    out = torch.full((N, L + gap, C), float("nan"), dtype=out_dtype)
    out = (out.pin_memory() if pinned else out)[:, :L]
    s = torch.cuda.Stream()
    ctx.self_attention_host(*ins, H, out, rope=rope, op_type=kd.BF16, stream=s)
    s.synchronize()
    ctx.device_status()
    assert torch.equal(out, ref.cpu())
    # a second call reuses the context's copy streams and staging
    out2 = torch.zeros_like(out)
    ctx.self_attention_host(*ins, H, out2, rope=rope, op_type=kd.BF16, stream=s)
    s.synchronize()
    assert torch.equal(out2, ref.cpu())


# ------------------------------------------------------------------ tile bitmap, tile counters, fused prologue
def expected_tile_counts(keep, Lq, Lk, units_per_plane_mult, head_pairs=False):
    """K/V tiles (128 keys of one head) loaded and Q-tile (128 rows) x K/V-tile products computed for
    one (head, sequence) plane, times the number of planes.  Units of 256 rows of one head: a tile is
    loaded when any of the unit's 64x64 sub-tiles is kept and computed for each Q tile with a kept
    sub-tile.  Head-pair units (one mask plane for all heads): 128 rows of two heads, every tile
    the rows need is loaded and computed once per head."""
    n_qb, n_kb = keep.shape
    n_kv = (Lk + 127) // 128
    if head_pairs:
        n = 0
        for b in range((Lq + 127) // 128):
            for t in range(n_kv):
                n += bool(keep[2 * b: 2 * b + 2, 2 * t: 2 * t + 2].any())
        return n * units_per_plane_mult, n * units_per_plane_mult
    n_units = (Lq + 255) // 256
    loaded = pairs = 0
    for u in range(n_units):
        for t in range(n_kv):
            need = []
            for i in range(2):
                sub = keep[4 * u + 2 * i: 4 * u + 2 * i + 2, 2 * t: 2 * t + 2]
                need.append(bool(sub.any()))
            loaded += any(need)
            pairs += sum(need)
    return loaded * units_per_plane_mult, pairs * units_per_plane_mult


def test_tile_bitmap_skips_tiles_and_matches_dense_mask(ctx, kd):
    """Block-sparse attention from the 64x64 tile bitmap alone equals the dense f16 block mask bit for
    bit, and the device counters show exactly the kept tiles were loaded and multiplied (one mask
    plane for the even head count: head-pair units)."""
    N, H, Lq, Lk, D = 2, 2, 1000, 1000, 128
    qf = seeded((N, H, Lq, D), 61, 0)
    kf = seeded((N, H, Lk, D), 61, 1)
    vf = seeded((N, H, Lk, D), 61, 2)
    rng = np.random.default_rng(8)
    n_qb, n_kb = (Lq + 63) // 64, (Lk + 63) // 64
    keep = rng.random((n_qb, n_kb)) < 0.2
    np.fill_diagonal(keep, True)
    dense = np.where(np.kron(keep, np.ones((64, 64)))[:Lq, :Lk], 0, -np.inf).astype(np.float16)[None, None]
    kb, vb = oracle.to_type(kf, oracle.BF16), oracle.to_type(vf, oracle.BF16)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mask=dense, mode=oracle.EXACT, lse=True)
    bits = torch.from_numpy(kd.tile_bitmap(keep)).cuda()
    assert bits.shape == (n_qb, (n_kb + 7) // 8)
    q, k, v = dev(qf), op_tensor(kf, oracle.BF16), op_tensor(vf, oracle.BF16)
    outs = {}
    want = expected_tile_counts(keep, Lq, Lk, H * N, head_pairs=True)
    dense_counts = expected_tile_counts(np.ones_like(keep), Lq, Lk, H * N)
    for name, kw in (("dense", dict(mask=torch.from_numpy(dense).cuda())), ("bitmap", dict(tile_mask=bits)),
                     ("both", dict(mask=torch.from_numpy(dense).cuda(), tile_mask=bits)), ("none", {})):
        ctx.tile_stats(reset=True)
        out = torch.empty(N, Lq, H, D, device="cuda")
        lse = torch.empty(N, H, Lq, device="cuda")
        ctx.flash_attn_ext(q, k, v, out, lse=lse, **kw)
        counts = ctx.tile_stats(reset=True)
        ctx.device_status()
        outs[name] = (out.cpu(), lse.cpu())
        assert counts == (dense_counts if name == "none" else want), (name, counts)
    assert want[1] < dense_counts[1]   # fewer products than dense (head pairs may load more tiles: per head)
    assert_gates(outs["bitmap"][0].numpy(), exact, lse=outs["bitmap"][1].numpy(), lse_ref=lse_ref, label="bitmap")
    for name in ("dense", "both"):
        assert torch.equal(outs[name][0], outs["bitmap"][0]) and torch.equal(outs[name][1], outs["bitmap"][1])


@pytest.mark.parametrize("Lq,Lk", [(1280, 1280), (700, 77)])
def test_qk_prologue_one_launch_equals_separate_calls(ctx, kd, Lq, Lk):
    """kd_attn_qk_prologue (Q, K, V in one launch; two jobs when Lq != Lk) equals three
    kd_attn_prologue calls bit for bit, with gains, with and without RoPE, and with pairs left out."""
    N, H = 2, 3
    C = H * 128
    q = dev(seeded((N, Lq, C), 71, 0))
    k = dev(seeded((N, Lk, C), 71, 1))
    v = dev(seeded((N, Lk, C), 71, 2))
    gq = torch.linspace(0.5, 1.5, 128, device="cuda")
    gk = torch.linspace(1.5, 0.5, 128, device="cuda")
    rope = kd.Rope3D.make((5, 16, 16), scale=(1, 2, 2)) if Lq == Lk == 1280 else None
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        ref = [torch.empty(N, H, L, 128, device="cuda", dtype=dt) for L in (Lq, Lk, Lk)]
        ctx.prologue(q, H, ref[0], norm=True, gain=gq, rope=rope)
        ctx.prologue(k, H, ref[1], norm=True, gain=gk, rope=rope)
        ctx.prologue(v, H, ref[2], norm=False)
        got = [torch.full_like(r, 3.0) for r in ref]
        ctx.qk_prologue(q, k, v, *got, q_gain=gq, k_gain=gk, rope=rope)
        ctx.device_status()
        for g, r in zip(got, ref):
            assert torch.equal(g, r)
        only_kv = [torch.full_like(r, 3.0) for r in ref[1:]]
        ctx.qk_prologue(None, k, v, None, *only_kv, k_gain=gk, rope=rope)
        ctx.device_status()
        assert torch.equal(only_kv[0], ref[1]) and torch.equal(only_kv[1], ref[2])


def test_sharded_entry_points_on_one_rank(ctx, kd):
    """With one rank the sharded calls are the plain ones into out_full (no peers, barriers no-ops):
    self- and cross-attention bit-identical to kd_attn_self_attention / kd_attn_cross_attention, into
    a symmetric buffer and into an ordinary tensor."""
    N, H, grid = 2, 4, (2, 8, 8)
    L, Lt, C = 128, 77, 4 * 128
    rope = kd.Rope3D.make(grid)
    q = dev(seeded((N, L, C), 81, 0))
    k = dev(seeded((N, L, C), 81, 1))
    v = dev(seeded((N, L, C), 81, 2))
    kt = dev(seeded((N, Lt, C), 81, 3))
    vt = dev(seeded((N, Lt, C), 81, 4))
    kv_len = torch.tensor([77, 30], dtype=torch.int32, device="cuda")
    ref_self = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
    ctx.self_attention(q, k, v, H, ref_self, rope=rope, op_type=kd.BF16)
    ref_cross = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
    ctx.cross_attention(q, kt, vt, H, ref_cross, kv_len=kv_len, op_type=kd.BF16)
    sym = ctx.symmetric_tensor((N, L, C), torch.bfloat16)
    plain = torch.empty(N, L, C, device="cuda", dtype=torch.bfloat16)
    for out in (sym, plain):
        out.fill_(7.0)
        ctx.self_attention_sharded(q, k, v, H, out, rope=rope, op_type=kd.BF16)
        ctx.device_status()
        assert torch.equal(out, ref_self)
        out.fill_(7.0)
        ctx.cross_attention_sharded(q, kt, vt, H, out, kv_len=kv_len, op_type=kd.BF16)
        ctx.device_status()
        assert torch.equal(out, ref_cross)
    ctx.symmetric_free(sym)


def test_bounded_wait_reports_timeout_and_context_recovers(ctx, kd):
    """Failure detection without a fault: a device wait that nothing releases gives up after its
    limit, the host reads ERR_DEVICE_TIMEOUT from the error word, and the next call works."""
    import time
    t0 = time.time()
    ctx.selftest_wait(wait_ms=50)
    with pytest.raises(kd.KdAttnError) as e:
        ctx.device_status()
    assert e.value.status == kd.ERR_DEVICE_TIMEOUT
    assert time.time() - t0 < 30
    ctx.device_status()   # the error word was cleared
    q = op_tensor(seeded((1, 1, 130, 128), 91, 0), oracle.BF16)
    out = torch.empty(1, 130, 1, 128, device="cuda")
    ctx.flash_attn_ext(q, q, q, out)
    ctx.device_status()
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("Lt", [77, 512])
def test_text_block_self_attention_with_1d_rope(ctx, kd, Lt):
    """The CrossDiT text blocks (crossdit.hpp:606) run DiTSelfAttention with 1D text RoPE
    (rope.hpp:36-49): the same fused path with axes (128, 0, 0) over a (L, 1, 1) grid, checked
    against the oracle with the text table pinned to the reference's compute_text_rope."""
    N, H = 1, 32
    C = H * 128
    q = seeded((N, Lt, C), 97, 0)
    k = seeded((N, Lt, C), 97, 1)
    v = seeded((N, Lt, C), 97, 2)
    tab = oracle.text_rope_table(Lt, 128)
    exact, lse_ref = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=oracle.BF16, mode=oracle.EXACT, lse=True)
    out = torch.empty(N, Lt, C, device="cuda")
    lse = torch.empty(N, H, Lt, device="cuda")
    rope = kd.Rope3D.make((Lt, 1, 1), axes=(128, 0, 0))
    ctx.self_attention(dev(q), dev(k), dev(v), H, out, rope=rope, op_type=kd.BF16, lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=f"text L{Lt}")


# ------------------------------------------------------------------ batched CFG over two separate buffers
def test_cfg_halves_in_separate_buffers_as_one_batch2_call(ctx, kd):
    """The reference runs classifier-free guidance as two batch-1 DiT forwards (pipeline.cpp:1571-1592);
    integration/kd_ggml_bridge.hpp pairs the two forwards' tensors into ONE batch-2 call by giving the
    sequence dimension the address difference of the two buffers.  That call must equal the two
    batch-1 calls bit for bit.  Here each role's two halves sit 4 KB apart (not packed), cond first."""
    L, H, d = 1280, 8, 128
    C = H * d
    gap = 1024                                   # floats between the halves (4 KB)
    rope = kd.Rope3D.make((5, 16, 16), scale=(1, 2, 2))

    def pair_buffers(dtype):
        buf = torch.empty(2, L * C + gap, device="cuda", dtype=dtype)
        return buf, [buf[i, :L * C].view(1, L, C) for i in range(2)]

    ins = []
    for off in range(3):
        buf, halves = pair_buffers(torch.float32)
        for i, h in enumerate(halves):      # cond, uncond
            t = torch.empty(L * C, device="cuda")
            ctx.fill_randn(t, seed=11 + i, offset=off)
            h.copy_(t.view(1, L, C))
        ins.append((buf, halves))
    obuf, outs = pair_buffers(torch.bfloat16)
    refs = []
    for i in range(2):
        r = torch.empty(1, L, C, device="cuda", dtype=torch.bfloat16)
        ctx.self_attention(*(x[1][i] for x in ins), H, r, rope=rope, op_type=kd.BF16)
        refs.append(r)

    def paired(halves):
        t = kd.KdTensor.of(halves[0])
        diff = halves[1].data_ptr() - halves[0].data_ptr()
        assert diff > 0 and diff % 16 == 0 and diff > halves[0].numel() * halves[0].element_size()
        t.ne[2] = 2
        t.nb[2] = diff
        t.nb[3] = 2 * diff
        return t

    tq, tk, tv = (paired(x[1]) for x in ins)
    to = paired(outs)
    rc = kd.lib.kd_attn_self_attention(ctx.handle, kd.ctypes.byref(tq), kd.ctypes.byref(tk), kd.ctypes.byref(tv), H,
                                       None, None, kd.ctypes.c_float(1e-6), kd.ctypes.byref(rope), kd.BF16,
                                       kd.ctypes.byref(to), None, None)
    assert rc == kd.OK, kd.lib.kd_attn_last_error(ctx.handle)
    ctx.device_status()
    for i in range(2):
        assert torch.equal(outs[i], refs[i])


# ------------------------------------------------------------------ head_dim 512: the VAE mid-block attention
@pytest.mark.parametrize("N,H,L,kv_type,out_dtype", [
    (1, 1, 64 * 64, oracle.F16, torch.float32),      # 512 x 512 image: 64 x 64 latent, ggml types
    (2, 2, 37 * 41, oracle.BF16, torch.bfloat16),    # ragged: partial Q tile and partial 64-key tile
])
def test_flash_ext_head_dim_512(ctx, N, H, L, kv_type, out_dtype):
    """VAEAttnBlock::forward (vae.hpp:89) attends with one head of the full channel count (512) through
    ops::attention's flash branch; kd_attn_flash_ext takes it with f32 Q (rounded to K's type on the
    device), 16-bit K/V, f32 or 16-bit output and the LSE."""
    D = 512
    qf = seeded((N, H, L, D), 512 + L, 0)
    kf = seeded((N, H, L, D), 512 + L, 1)
    vf = seeded((N, H, L, D), 512 + L, 2)
    kb, vb = oracle.to_type(kf, kv_type), oracle.to_type(vf, kv_type)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mode=oracle.EXACT, lse=True)
    out = torch.empty(N, L, H, D, device="cuda", dtype=out_dtype)
    lse = torch.empty(N, H, L, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, kv_type), op_tensor(vf, kv_type), out, lse=lse)
    ctx.device_status()
    ot = None if out_dtype == torch.float32 else "bf16"
    ggml = oracle.flash_attn_ext(qf, kb, vb, mode=oracle.GGML) if ot is None else None
    assert_gates(out.float().cpu().numpy(), exact, ggml, lse.cpu().numpy(), lse_ref, label=f"d512 {N,H,L}", out_type=ot)


def test_ops_attention_vae_mid_block(ctx, kd):
    """ops::attention as VAEAttnBlock::forward calls it (vae.hpp:89): one head over the 64 x 64 latent
    positions of a 512 x 512 image with the full 512 channels, f32 q/k/v [512, H*W, 1], f16 operands
    (ggml's flash branch), f32 output -- through the C ABI entry point that mirrors ops::attention."""
    N, L, C = 1, 64 * 64, 512
    q = seeded((N, L, C), 77, 0)
    k = seeded((N, L, C), 77, 1)
    v = seeded((N, L, C), 77, 2)
    out = torch.empty(N, L, C, device="cuda")
    lse = torch.empty(N, 1, L, device="cuda")
    ctx.ops_attention(dev(q), dev(k), dev(v), 1, out, op_type=kd.F16, lse=lse)
    ctx.device_status()
    q4, k4, v4 = (x.reshape(N, 1, L, C) for x in (q, k, v))
    kb, vb = oracle.to_type(k4, oracle.F16), oracle.to_type(v4, oracle.F16)
    exact, lse_ref = oracle.flash_attn_ext(q4, kb, vb, mode=oracle.EXACT, lse=True)
    ggml = oracle.flash_attn_ext(q4, kb, vb, mode=oracle.GGML)
    assert_gates(out.cpu().numpy().reshape(N, L, 1, C), exact, ggml, lse.cpu().numpy(), lse_ref, label="VAE mid block")
