"""GPU parity at head_dim 64: the lite video model (CrossDiTConfig::lite_video, crossdit.hpp:48-56 --
model_dim 1792 = 28 heads of 64, RoPE axes {16, 24, 24}, scale_factor {1, 2, 2}) through the same
C ABI entry points as head_dim 128, against the CPU oracle on identical seeded inputs."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_gates, seeded
from test_gpu_flash import _mask_case, dev, op_tensor

pytestmark = pytest.mark.gpu

D = 64
LITE_AXES = (16, 24, 24)
LITE_SCALE = (1, 2, 2)

SHAPES = [  # N, H, Hkv, Lq, Lk: short keys (<= 1024, the short-key instantiation) and long keys
    (1, 1, 1, 1, 1), (1, 2, 2, 63, 40), (2, 2, 2, 65, 128), (1, 1, 1, 127, 129), (2, 4, 2, 255, 256),
    (1, 1, 1, 513, 640), (1, 2, 2, 300, 1500), (1, 3, 1, 257, 2100),
]


@pytest.mark.parametrize("N,H,Hkv,Lq,Lk", SHAPES)
@pytest.mark.parametrize("kv_type", [oracle.F16, oracle.BF16])
def test_flash_ext_d64_shapes(ctx, N, H, Hkv, Lq, Lk, kv_type):
    qf = seeded((N, H, Lq, D), 17 + Lq, 0)
    kf = seeded((N, Hkv, Lk, D), 17 + Lq, 1)
    vf = seeded((N, Hkv, Lk, D), 17 + Lq, 2)
    kb, vb = oracle.to_type(kf, kv_type), oracle.to_type(vf, kv_type)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mode=oracle.EXACT, lse=True)
    out = torch.full((N, Lq, H, D), 7.0, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, kv_type), op_tensor(vf, kv_type), out, lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=f"d64 {N,H,Hkv,Lq,Lk}")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Lk", [300, 1300])
def test_flash_ext_d64_output_types_and_strided_q(ctx, out_dtype, Lk):
    """Strided f32 Q (the permuted [C, L, N] view ops::attention builds, rounded by the Q conversion),
    outputs in three types -- the short-key call with a 16-bit output stores its O tiles by TMA."""
    N, Lq, H = 2, 300, 4
    q_in = seeded((N, Lq, H * D), 19, 0)
    kf = seeded((N, H, Lk, D), 19, 1)
    vf = seeded((N, H, Lk, D), 19, 2)
    kb, vb = oracle.to_type(kf, oracle.BF16), oracle.to_type(vf, oracle.BF16)
    qf = np.ascontiguousarray(q_in.reshape(N, Lq, H, D).transpose(0, 2, 1, 3))
    exact = oracle.flash_attn_ext(qf, kb, vb, mode=oracle.EXACT)
    qd = dev(q_in).view(N, Lq, H, D).permute(0, 2, 1, 3)
    out = torch.empty(N, Lq, H, D, device="cuda", dtype=out_dtype)
    ctx.flash_attn_ext(qd, op_tensor(kf, oracle.BF16), op_tensor(vf, oracle.BF16), out)
    ctx.device_status()
    ot = {torch.float32: None, torch.bfloat16: "bf16", torch.float16: "f16"}[out_dtype]
    assert_gates(out.float().cpu().numpy(), exact, label=f"d64 {out_dtype} Lk {Lk}", out_type=ot)


@pytest.mark.parametrize("kind", ["random", "block", "rows"])
@pytest.mark.parametrize("H", [2, 3])
def test_flash_ext_d64_masks(ctx, kind, H):
    """Masked instantiations at head_dim 64: one mask plane and an even head count runs the head-pair
    units, an odd head count the 256-row units."""
    N, Lq, Lk = 2, 320, 384
    qf = seeded((N, H, Lq, D), 23, 0)
    kf = seeded((N, H, Lk, D), 23, 1)
    vf = seeded((N, H, Lk, D), 23, 2)
    kb, vb = oracle.to_type(kf, oracle.F16), oracle.to_type(vf, oracle.F16)
    mask = _mask_case(kind, N, Lq, Lk, 7)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mask=mask, mode=oracle.EXACT, lse=True)
    out = torch.empty(N, Lq, H, D, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, oracle.F16), op_tensor(vf, oracle.F16), out,
                       mask=torch.from_numpy(mask).cuda(), lse=lse)
    ctx.device_status()
    got = out.cpu().numpy()
    assert_gates(got, exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=f"d64 {kind} H{H}")
    dead = np.isneginf(lse_ref).transpose(0, 2, 1)
    assert np.all(got[dead] == 0)


def test_flash_ext_d64_kv_len(ctx):
    kv_len = np.array([1, 17, 100, 128, 129, 255, 0], np.int32)
    N, H, Lq, Lk = len(kv_len), 2, 130, 256
    qf = seeded((N, H, Lq, D), 29, 0)
    kf = seeded((N, H, Lk, D), 29, 1)
    vf = seeded((N, H, Lk, D), 29, 2)
    kb, vb = oracle.to_type(kf, oracle.BF16), oracle.to_type(vf, oracle.BF16)
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, kv_len=kv_len, mode=oracle.EXACT, lse=True)
    out = torch.full((N, Lq, H, D), 7.0, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.flash_attn_ext(dev(qf), op_tensor(kf, oracle.BF16), op_tensor(vf, oracle.BF16), out,
                       kv_len=torch.from_numpy(kv_len).cuda(), lse=lse)
    ctx.device_status()
    got, l = out.cpu().numpy(), lse.cpu().numpy()
    assert np.all(got[-1] == 0) and np.all(np.isneginf(l[-1]))
    assert_gates(got[:-1], exact[:-1], lse=l[:-1], lse_ref=lse_ref[:-1], label="d64 kv_len")


@pytest.mark.parametrize("H", [3, 4])
def test_prologue_d64_matches_oracle(ctx, kd, H):
    """RMSNorm over 64-wide heads and the {16, 24, 24} RoPE; two heads per warp row, an odd head count
    leaves the last row half empty."""
    N, grid = 2, (3, 4, 5)
    L = grid[0] * grid[1] * grid[2]
    x = seeded((N, L, H * D), 31, 0) * 3.0
    gain = (1.0 + 0.1 * seeded((D,), 31, 1)).astype(np.float32)
    tab = oracle.visual_rope_table(grid, axes=LITE_AXES, scale=LITE_SCALE)
    ref = oracle.prologue(x, H, gain=gain, rope_table=tab)                  # (N, H, L, 64) f32
    rope = kd.Rope3D.make(grid, axes=LITE_AXES, scale=LITE_SCALE)
    y = torch.full((N, H, L, D), float("nan"), device="cuda")
    ctx.prologue(dev(x), H, y, norm=True, gain=dev(gain), rope=rope)
    ctx.device_status()
    np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=0, atol=4e-6)
    yv = torch.empty(N, H, L, D, device="cuda", dtype=torch.bfloat16)
    ctx.prologue(dev(x), H, yv, norm=False)
    rv = oracle.to_f32(oracle.to_type(x.reshape(N, L, H, D).transpose(0, 2, 1, 3), oracle.BF16), oracle.BF16)
    np.testing.assert_array_equal(yv.float().cpu().numpy(), rv)


@pytest.mark.parametrize("kv_type", [oracle.F16, oracle.BF16])
def test_lite_video_self_attention(ctx, kd, kv_type):
    """DiTSelfAttention of the lite video model: 28 heads of 64, RMSNorm, 3D RoPE {16, 24, 24} with
    scale {1, 2, 2}, against the fp64 and ggml-faithful oracles."""
    N, H, grid = 1, 28, (3, 16, 16)
    L, C = grid[0] * grid[1] * grid[2], H * D
    q = seeded((N, L, C), 37, 0)
    k = seeded((N, L, C), 37, 1)
    v = seeded((N, L, C), 37, 2)
    tab = oracle.visual_rope_table(grid, axes=LITE_AXES, scale=LITE_SCALE)
    exact, lse_ref = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=kv_type, mode=oracle.EXACT, lse=True)
    ggml = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=kv_type, mode=oracle.GGML)
    out = torch.empty(N, L, C, device="cuda")
    lse = torch.empty(N, H, L, device="cuda")
    ctx.self_attention(dev(q), dev(k), dev(v), H, out, rope=kd.Rope3D.make(grid, axes=LITE_AXES, scale=LITE_SCALE),
                       op_type=kv_type, lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, ggml, lse.cpu().numpy(), lse_ref, label=f"lite self {kv_type}")


def test_lite_video_cross_attention(ctx, kd):
    """DiTCrossAttention of the lite video model: visual queries against padded text keys with valid
    lengths, RMSNorm on Q and K, no RoPE."""
    N, H, Lq, Lt = 2, 28, 700, 256
    C = H * D
    q = seeded((N, Lq, C), 41, 0)
    k = seeded((N, Lt, C), 41, 1) * 0.5
    v = seeded((N, Lt, C), 41, 2)
    kv_len = np.array([77, 200], np.int32)
    exact, lse_ref = oracle.self_attention(q, k, v, H, kv_type=oracle.BF16, kv_len=kv_len, mode=oracle.EXACT,
                                           lse=True)
    out = torch.empty(N, Lq, C, device="cuda")
    lse = torch.empty(N, H, Lq, device="cuda")
    ctx.cross_attention(dev(q), dev(k), dev(v), H, out, kv_len=torch.from_numpy(kv_len).cuda(), op_type=kd.BF16,
                        lse=lse)
    ctx.device_status()
    assert_gates(out.cpu().numpy(), exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label="lite cross")


@pytest.mark.parametrize("n_kv_head", [28, 14])
def test_lite_ops_attention_mirror(ctx, kd, n_kv_head):
    """ops::attention (flash branch) with n_head = 28 over 1792 channels: head_dim 64 derived as
    q.ne[0] / n_head (ops.hpp:116); K/V with fewer heads broadcast (GQA)."""
    N, Lq, Lk, H = 1, 200, 77, 28
    q = seeded((N, Lq, H * D), 43, 0)
    k = seeded((N, Lk, n_kv_head * D), 43, 1)
    v = seeded((N, Lk, n_kv_head * D), 43, 2)
    q4 = np.ascontiguousarray(q.reshape(N, Lq, H, D).transpose(0, 2, 1, 3))
    k4 = oracle.to_type(np.ascontiguousarray(k.reshape(N, Lk, n_kv_head, D).transpose(0, 2, 1, 3)), oracle.F16)
    v4 = oracle.to_type(np.ascontiguousarray(v.reshape(N, Lk, n_kv_head, D).transpose(0, 2, 1, 3)), oracle.F16)
    exact = oracle.flash_attn_ext(q4, k4, v4, mode=oracle.EXACT).reshape(N, Lq, H * D)
    got = kd.attention(ctx, dev(q), dev(k), dev(v), H)
    ctx.device_status()
    assert_gates(got.cpu().numpy(), exact, label=f"lite ops::attention kv heads {n_kv_head}")


def test_lite_host_pipeline_matches_device_path(ctx, kd):
    """kd_attn_self_attention_host at head_dim 64 equals the device-buffer call bit for bit."""
    N, H, grid = 2, 28, (2, 8, 12)
    L, C = grid[0] * grid[1] * grid[2], H * D
    rope = kd.Rope3D.make(grid, axes=LITE_AXES, scale=LITE_SCALE)
    ins = [torch.from_numpy(seeded((N, L, C), 47, off)).pin_memory() for off in range(3)]
    ref = torch.empty(N, L, C, device="cuda")
    ctx.self_attention(*[x.cuda() for x in ins], H, ref, rope=rope, op_type=kd.BF16)
    out = torch.full((N, L, C), float("nan")).pin_memory()
    s = torch.cuda.Stream()
    ctx.self_attention_host(*ins, H, out, rope=rope, op_type=kd.BF16, stream=s)
    s.synchronize()
    ctx.device_status()
    assert torch.equal(out, ref.cpu())


def test_lite_rejects_rope_of_the_wrong_width(ctx, kd):
    """A RoPE whose axes sum to 128 cannot rotate 64-wide heads: INVALID_ARGUMENT, nothing launched."""
    N, H, grid = 1, 4, (1, 2, 3)
    L = 6
    x = dev(seeded((N, L, H * D), 53, 0))
    y = torch.empty(N, H, L, D, device="cuda")
    with pytest.raises(kd.KdAttnError) as e:
        ctx.prologue(x, H, y, norm=True, rope=kd.Rope3D.make(grid))
    assert e.value.status == kd.ERR_INVALID_ARGUMENT
    ctx.device_status()


# ------------------------------------------------------------------ the fused QKV projection at head_dim 64
@pytest.mark.parametrize("wname", ["q8_0", "q4_0"])
def test_lite_qkv_projection_matches_oracle(ctx, kd, wname):
    """to_query/to_key/to_value of the lite video model (model_dim 1792 = 28 heads of 64) as one GEMM whose
    epilogue normalises each 64-wide head alone and rotates it with the {16, 24, 24} RoPE."""
    from test_gpu_projection import WTYPES, check, make_weight
    from test_gpu_projection import dev as pdev
    N, grid, K, H = 2, (3, 10, 10), 1792, 28
    L, C = int(np.prod(grid)), H * D
    x = seeded((N, L, K), 61, 0)
    lin = [make_weight(kd, 62, 10 * i, C, K, WTYPES[wname], bias=(i != 1)) for i in range(3)]
    q_gain = (1.0 + 0.1 * seeded((D,), 63, 0)).astype(np.float32)
    k_gain = (1.0 + 0.1 * seeded((D,), 63, 1)).astype(np.float32)
    tab = oracle.visual_rope_table(grid, axes=LITE_AXES, scale=LITE_SCALE)
    outs = [torch.full((N, H, L, D), float("nan"), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    ctx.qkv_projection(pdev(x), lin[0][0], lin[1][0], lin[2][0], *outs, q_gain=pdev(q_gain), k_gain=pdev(k_gain),
                       rope=kd.Rope3D.make(grid, axes=LITE_AXES, scale=LITE_SCALE))
    ctx.device_status()
    check(outs, x, [l[2] for l in lin], [l[3] for l in lin], H, q_gain, k_gain, tab, "bf16", f"lite {wname}")


def test_lite_projection_feeds_flash(ctx, kd):
    """Lite projection -> flash attention (head_dim 64) against the oracle's composition."""
    from test_gpu_projection import make_weight
    from test_gpu_projection import dev as pdev
    N, grid, K, H = 1, (2, 8, 10), 1792, 28
    L, C = int(np.prod(grid)), H * D
    x = seeded((N, L, K), 67, 0)
    lin = [make_weight(kd, 68, 10 * i, C, K, kd.Q8_0) for i in range(3)]
    tab = oracle.visual_rope_table(grid, axes=LITE_AXES, scale=LITE_SCALE)
    ops = [torch.empty((N, H, L, D), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    ctx.qkv_projection(pdev(x), lin[0][0], lin[1][0], lin[2][0], *ops,
                       rope=kd.Rope3D.make(grid, axes=LITE_AXES, scale=LITE_SCALE))
    out = torch.empty(N, L, H, D, device="cuda")
    ctx.flash_attn_ext(*ops, out)
    ctx.device_status()
    q, k, v = oracle.qkv_projection(x, [l[2] for l in lin], [l[3] for l in lin], H, rope_table=tab)
    exact = oracle.flash_attn_ext(q, oracle.to_type(k, oracle.BF16), oracle.to_type(v, oracle.BF16),
                                  mode=oracle.EXACT)
    assert_gates(out.cpu().numpy(), exact, label="lite projection -> flash")


# ------------------------------------------------------------------ whole lite attention modules
def test_lite_self_attention_block_matches_oracle(ctx, kd):
    """DiTSelfAttention::forward of the lite video model (crossdit.hpp:117-154 with num_heads 28 of 64):
    q8_0 Q/K/V weights with biases, RMSNorm gains over 64-wide heads, the {16, 24, 24} RoPE, q4_0
    out-projection; against the oracle's linear -> RMSNorm -> RoPE -> flash_attn_ext -> linear chain.  The
    same hidden states with n_head 14 (head dim 128) are rejected by the RoPE's width."""
    from test_gpu_projection import make_weight
    from test_gpu_projection import dev as pdev
    N, grid, H = 1, (2, 8, 16), 28
    C, L = H * D, int(np.prod(grid))
    x = seeded((N, L, C), 171, 0)
    lin = [make_weight(kd, 172, 10 * i, C, C, kd.Q8_0) for i in range(3)]
    lo, keep_o, deq_o, b_o = make_weight(kd, 173, 0, C, C, kd.Q4_0)
    q_gain = (1.0 + 0.1 * seeded((D,), 174, 0)).astype(np.float32)
    k_gain = (1.0 + 0.1 * seeded((D,), 174, 1)).astype(np.float32)
    rope = kd.Rope3D.make(grid, axes=LITE_AXES, scale=LITE_SCALE)
    y = torch.full((N, L, C), float("nan"), device="cuda")
    ctx.self_attention_block(pdev(x), lin[0][0], lin[1][0], lin[2][0], lo, H, y, q_gain=pdev(q_gain),
                             k_gain=pdev(k_gain), rope=rope)
    ctx.device_status()
    proj = [oracle.linear(x, l[2], l[3]).astype(np.float32) for l in lin]
    attn = oracle.self_attention(*proj, H, q_gain=q_gain, k_gain=k_gain,
                                 rope_table=oracle.visual_rope_table(grid, axes=LITE_AXES, scale=LITE_SCALE),
                                 kv_type=oracle.BF16, q_type=oracle.BF16, mode=oracle.EXACT)
    ref = oracle.linear(attn, deq_o, b_o)
    m = oracle.parity_metrics(y.cpu().numpy(), ref)
    assert m["cos"] >= 0.9999 and m["maxabs_over_rms"] <= 5e-2, m
    with pytest.raises(kd.KdAttnError) as e:
        ctx.self_attention_block(pdev(x), lin[0][0], lin[1][0], lin[2][0], lo, H // 2, y, rope=rope)
    assert e.value.status == kd.ERR_INVALID_ARGUMENT
    ctx.device_status()


def test_lite_cross_attention_block_matches_oracle(ctx, kd):
    """DiTCrossAttention::forward of the lite video model: visual queries against text states with valid
    lengths, q4_0 weights, 28 heads of 64, RMSNorm on Q and K, no RoPE."""
    from test_gpu_projection import make_weight
    from test_gpu_projection import dev as pdev
    N, Lq, Lt, H = 2, 256, 77, 28
    C = H * D
    xq, xt = seeded((N, Lq, C), 181, 0), seeded((N, Lt, C), 181, 1)
    lin = [make_weight(kd, 182, 10 * i, C, C, kd.Q4_0) for i in range(3)]
    lo, keep_o, deq_o, b_o = make_weight(kd, 183, 0, C, C, kd.F16)
    kv_len = np.array([77, 40], np.int32)
    y = torch.full((N, Lq, C), float("nan"), device="cuda")
    ctx.cross_attention_block(pdev(xq), pdev(xt), lin[0][0], lin[1][0], lin[2][0], lo, H, y, kv_len=pdev(kv_len))
    ctx.device_status()
    q = oracle.linear(xq, lin[0][2], lin[0][3]).astype(np.float32)
    k = oracle.linear(xt, lin[1][2], lin[1][3]).astype(np.float32)
    v = oracle.linear(xt, lin[2][2], lin[2][3]).astype(np.float32)
    attn = oracle.self_attention(q, k, v, H, kv_type=oracle.BF16, q_type=oracle.BF16, kv_len=kv_len,
                                 mode=oracle.EXACT)
    m = oracle.parity_metrics(y.cpu().numpy(), oracle.linear(attn, deq_o, b_o))
    assert m["cos"] >= 0.9999 and m["maxabs_over_rms"] <= 5e-2, m
