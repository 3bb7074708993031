"""CPU oracle checks (no GPU).

1. Pinning against the reference's own code: tests/golden/ref_pin.npz holds the
   outputs of the reference's src/rng.hpp and src/rope.hpp compiled from the
   reference sources (tests/golden/make_golden.py); the oracle must reproduce
   them bit for bit.
2. The fp64 flash_attn_ext restatement against an independent implementation
   (torch, float64) on small shapes with masks, GQA and kv_len.
3. Known-answer tests for the operator and the prologue.
"""
import os

import numpy as np
import pytest
import torch

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden", "ref_pin.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


# ------------------------------------------------------------------ 1. pinning
def test_philox_matches_reference(gold):
    assert np.array_equal(oracle.philox_randn(42, 4096, 0), gold["philox_s42_off0"])
    assert np.array_equal(oracle.philox_randn(42, 4096, 1), gold["philox_s42_off1"])
    assert np.array_equal(oracle.philox_randn(0x1234567890ABCDEF, 1000, 0), gold["philox_s1234567890abcdef_off0"])


def test_rope_freqs_match_reference(gold):
    assert np.array_equal(oracle.rope_freqs(16), gold["freqs_16"])
    assert np.array_equal(oracle.rope_freqs(24), gold["freqs_24"])


def test_text_rope_matches_reference(gold):
    assert np.array_equal(oracle.text_rope_table(7, 128).ravel(), gold["text_rope_7x128"])


@pytest.mark.parametrize("scale,key", [((1, 1, 1), "visual_rope_3x4x5_s111"), ((1, 2, 2), "visual_rope_3x4x5_s122")])
def test_visual_rope_matches_reference(gold, scale, key):
    assert np.array_equal(oracle.visual_rope_table((3, 4, 5), scale=scale).ravel(), gold[key])


def test_visual_rope_lite_axes_match_reference(gold):
    """The lite video model's axes {16, 24, 24} (head_dim 64, crossdit.hpp:36,52) with its scale {1, 2, 2}."""
    t = oracle.visual_rope_table((3, 4, 5), axes=(16, 24, 24), scale=(1, 2, 2))
    assert t.shape == (60, 64)
    assert np.array_equal(t.ravel(), gold["visual_rope_3x4x5_a162424_s122"])


def test_visual_rope_benchmark_grids_match_reference(gold):
    t = oracle.visual_rope_table((5, 16, 16), scale=(1, 2, 2))
    assert np.array_equal(t[gold["rows_5x16x16"]].ravel(), gold["visual_rope_5x16x16_s122_rows"])
    t = oracle.visual_rope_table((31, 32, 32))
    assert np.array_equal(t[gold["rows_31x32x32"]].ravel(), gold["visual_rope_31x32x32_s111_rows"])


# ------------------------------------------------------------------ 2. fp64 restatement vs torch
def _torch_ref(q, k, v, mask=None, kv_len=None, scale=None):
    """float64 attention with ggml's broadcast rules; q (N,H,Lq,D), k/v (Nk,Hk,Lk,D), mask (mn,mh,>=Lq,>=Lk)."""
    q = torch.from_numpy(np.asarray(q, np.float64))
    k = torch.from_numpy(np.asarray(k, np.float64))
    v = torch.from_numpy(np.asarray(v, np.float64))
    N, H, Lq, D = q.shape
    Nk, Hk, Lk, _ = k.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    k = k.repeat_interleave(H // Hk, dim=1).repeat_interleave(N // Nk, dim=0)
    v = v.repeat_interleave(H // Hk, dim=1).repeat_interleave(N // Nk, dim=0)
    s = torch.einsum("nhqd,nhkd->nhqk", q, k) * scale
    if mask is not None:
        m = torch.from_numpy(np.asarray(mask, np.float64))[:, :, :Lq, :Lk]
        m = m.repeat(N // m.shape[0], H // m.shape[1], 1, 1)
        s = s + m
    if kv_len is not None:
        for n in range(N):
            s[n, :, :, int(kv_len[n]):] = -np.inf
    mx = s.amax(-1, keepdim=True)
    mx = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
    p = torch.exp(s - mx)
    den = p.sum(-1, keepdim=True)
    o = torch.where(den > 0, (p @ v) / den, torch.zeros_like(p @ v))
    lse = torch.where(den[..., 0] > 0, torch.log(den[..., 0]) + mx[..., 0], torch.full_like(den[..., 0], -np.inf))
    return o.permute(0, 2, 1, 3).numpy(), lse.numpy()   # (N, Lq, H, D), (N, H, Lq)


def _rand(shape, seed, off=0):
    return oracle.philox_randn(seed, int(np.prod(shape)), off).reshape(shape)


@pytest.mark.parametrize("N,H,Hk,Lq,Lk", [(1, 2, 2, 7, 9), (2, 4, 2, 33, 65), (2, 2, 1, 1, 1), (1, 3, 3, 70, 130)])
def test_exact_mode_matches_torch(N, H, Hk, Lq, Lk):
    D = 128
    q = _rand((N, H, Lq, D), 1, 0)
    k = oracle.to_type(_rand((N, Hk, Lk, D), 1, 1), oracle.F16)
    v = oracle.to_type(_rand((N, Hk, Lk, D), 1, 2), oracle.F16)
    o, l = oracle.flash_attn_ext(q, k, v, mode=oracle.EXACT, lse=True)
    qr = oracle.to_f32(oracle.to_type(q, oracle.F16), oracle.F16)   # ggml rounds Q to K's type
    ro, rl = _torch_ref(qr, oracle.to_f32(k, oracle.F16), oracle.to_f32(v, oracle.F16))
    np.testing.assert_allclose(o, ro, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l, rl, rtol=1e-6, atol=1e-6)


def test_exact_mode_mask_and_kv_len_match_torch():
    N, H, Lq, Lk, D = 2, 2, 20, 50, 128
    rng = np.random.default_rng(3)
    q = _rand((N, H, Lq, D), 5, 0)
    k = oracle.to_type(_rand((N, H, Lk, D), 5, 1), oracle.BF16)
    v = oracle.to_type(_rand((N, H, Lk, D), 5, 2), oracle.BF16)
    mask = rng.normal(size=(N, 1, Lq + 3, Lk + 5)).astype(np.float16)
    mask[rng.random(mask.shape) < 0.3] = -np.inf
    mask[0, 0, 4, :] = -np.inf                      # a fully masked row
    kv_len = np.array([50, 17], np.int32)
    o, l = oracle.flash_attn_ext(q, k, v, mask=mask, kv_len=kv_len, mode=oracle.EXACT, lse=True)
    qr = oracle.to_f32(oracle.to_type(q, oracle.BF16), oracle.BF16)
    ro, rl = _torch_ref(qr, oracle.to_f32(k, oracle.BF16), oracle.to_f32(v, oracle.BF16), mask.astype(np.float64),
                        kv_len)
    np.testing.assert_allclose(o, ro, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l, rl, rtol=1e-6, atol=1e-6)
    assert np.all(o[0, 4, 0] == 0) and np.isneginf(l[0, 0, 4])


# ------------------------------------------------------------------ 3. known answers
def test_kat_single_key_returns_v():
    q = _rand((1, 1, 5, 128), 9)
    k = oracle.to_type(_rand((1, 1, 1, 128), 9, 1), oracle.F16)
    v = oracle.to_type(_rand((1, 1, 1, 128), 9, 2), oracle.F16)
    for mode in (oracle.EXACT, oracle.GGML):
        o = oracle.flash_attn_ext(q, k, v, mode=mode)
        np.testing.assert_allclose(o[0, :, 0], np.broadcast_to(oracle.to_f32(v, oracle.F16)[0, 0], (5, 128)), rtol=0, atol=0)


def test_kat_uniform_keys_give_mean_v():
    k = oracle.to_type(np.broadcast_to(_rand((1, 1, 1, 128), 2), (1, 1, 64, 128)).copy(), oracle.F16)
    v = _rand((1, 1, 64, 128), 2, 1)
    q = _rand((1, 1, 3, 128), 2, 2)
    o = oracle.flash_attn_ext(q, k, oracle.to_type(v, oracle.BF16), mode=oracle.EXACT)
    vm = oracle.to_f32(oracle.to_type(v, oracle.BF16), oracle.BF16)[0, 0].astype(np.float64).mean(0)
    np.testing.assert_allclose(o[0, :, 0], np.broadcast_to(vm, (3, 128)), rtol=1e-6, atol=1e-6)


def test_kat_all_masked_but_one():
    q = _rand((1, 1, 4, 128), 4)
    k = oracle.to_type(_rand((1, 1, 10, 128), 4, 1), oracle.F16)
    v = oracle.to_type(_rand((1, 1, 10, 128), 4, 2), oracle.F16)
    mask = np.full((1, 1, 4, 10), -np.inf, np.float16)
    for i in range(4):
        mask[0, 0, i, 2 * i] = 0
    for mode in (oracle.EXACT, oracle.GGML):
        o = oracle.flash_attn_ext(q, k, v, mask=mask, mode=mode)
        for i in range(4):
            np.testing.assert_array_equal(o[0, i, 0], oracle.to_f32(v, oracle.F16)[0, 0, 2 * i])


def test_kat_rope_position_zero_is_identity():
    tab = oracle.visual_rope_table((2, 3, 4))
    x = _rand((1, 24, 2 * 128), 6)
    y = oracle.rope_apply(x, 2, 128, tab)
    np.testing.assert_array_equal(y[0, 0], x[0, 0])           # token (0,0,0)
    assert not np.array_equal(y[0, 1], x[0, 1])


def test_kat_rope_composition():
    """Rotating by the table of position p equals rotating by angle(p) with a 2x2 matrix."""
    tab = oracle.visual_rope_table((3, 4, 5), scale=(1, 2, 2))
    x = _rand((1, 60, 128), 7)
    y = oracle.rope_apply(x, 1, 128, tab)
    c, s = tab[:, 0::2].astype(np.float64), tab[:, 1::2].astype(np.float64)
    x0, x1 = x[0, :, 0::2].astype(np.float64), x[0, :, 1::2].astype(np.float64)
    np.testing.assert_allclose(y[0, :, 0::2], x0 * c - x1 * s, atol=2e-6)
    np.testing.assert_allclose(y[0, :, 1::2], x0 * s + x1 * c, atol=2e-6)
    # norm preserved per pair
    np.testing.assert_allclose(np.hypot(y[0, :, 0::2], y[0, :, 1::2]), np.hypot(x0, x1), rtol=1e-5)


def test_kat_rms_norm_of_constant_vector():
    x = np.full((3, 128), 2.5, np.float32)
    y = oracle.rms_norm_heads(x, 128, eps=1e-6)
    np.testing.assert_allclose(y, np.ones_like(y), rtol=1e-6)
    g = np.linspace(0.5, 1.5, 128).astype(np.float32)
    y = oracle.rms_norm_heads(-x, 128, gain=g, eps=1e-6)
    np.testing.assert_allclose(y, -np.broadcast_to(g, y.shape), rtol=1e-6)


def test_ggml_mode_f16_accumulator_is_the_only_difference():
    """bf16 V: ggml accumulates in f32, so the faithful mode equals the fp64 mode closely;
    f16 V: ggml's f16 accumulator leaves a visible but bounded error."""
    N, L, H, d = 1, 256, 2, 128
    q = _rand((N, L, H * d), 11, 0)
    k = _rand((N, L, H * d), 11, 1)
    v = _rand((N, L, H * d), 11, 2)
    tab = oracle.visual_rope_table((1, 16, 16))
    ob_e = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=oracle.BF16, mode=oracle.EXACT)
    ob_g = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=oracle.BF16, mode=oracle.GGML)
    assert oracle.parity_metrics(ob_g, ob_e)["maxabs_over_rms"] < 1e-4
    of_e = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=oracle.F16, mode=oracle.EXACT)
    of_g = oracle.self_attention(q, k, v, H, rope_table=tab, kv_type=oracle.F16, mode=oracle.GGML)
    m = oracle.parity_metrics(of_g, of_e)
    assert m["cos"] > 0.9999 and m["maxabs_over_rms"] < 0.2


def test_f16_conversion_round_trip_matches_numpy():
    x = np.concatenate([_rand((10000,), 13) * 1000, np.array([65504, 65519.99, 65520, 1e-8, 6e-5, -0.0, 3e-8], np.float32)])
    np.testing.assert_array_equal(oracle.to_type(x, oracle.F16), x.astype(np.float16))


# ------------------------------------------------------------------ Linear weight formats
QUANT_GOLD = os.path.join(os.path.dirname(__file__), "golden", "quant_pin.npz")


@pytest.mark.parametrize("case", ["rand", "heavy", "edge"])
def test_quantizers_match_reference_converter(case):
    """q8_0 / q4_0 bytes equal those of the reference converter (scripts/convert_to_gguf.py:90-146),
    stored by tests/golden/make_quant_golden.py, including round-half-even ties and all-zero blocks."""
    g = np.load(QUANT_GOLD)
    w = g[f"{case}_w"]
    np.testing.assert_array_equal(oracle.quantize_q8_0(w), g[f"{case}_q8_0"])
    np.testing.assert_array_equal(oracle.quantize_q4_0(w), g[f"{case}_q4_0"])


def test_dequantize_known_blocks():
    """Hand-built blocks: q8_0 d = 0.5 with q = -128..127 pattern; q4_0 d = -0.25 with element j in the low
    nibble and j + 16 in the high nibble."""
    q8 = np.zeros((1, 34), np.uint8)
    q8[0, :2] = np.array([0.5], np.float16).view(np.uint8)
    q = (np.arange(32) * 8 - 128).astype(np.int8)
    q8[0, 2:] = q.view(np.uint8)
    np.testing.assert_array_equal(oracle.dequantize(q8, oracle.Q8_0, 32)[0], q.astype(np.float32) * 0.5)
    q4 = np.zeros((1, 18), np.uint8)
    q4[0, :2] = np.array([-0.25], np.float16).view(np.uint8)
    lo, hi = np.arange(16, dtype=np.uint8), (15 - np.arange(16)).astype(np.uint8)
    q4[0, 2:] = lo | (hi << 4)
    want = np.concatenate([lo, hi]).astype(np.float32) - 8.0
    np.testing.assert_array_equal(oracle.dequantize(q4, oracle.Q4_0, 32)[0], want * -0.25)


def test_quantize_dequantize_error_bounds():
    """Round trip within half a step, plus the f16 rounding of the stored scale (the quantizers divide by
    the f32 scale): q8_0 |w - deq| <= d/2 + 127 d 2^-11; q4_0 within one step (the +8 end clips to 7)."""
    w = (np.random.default_rng(5).standard_normal((16, 256)) * 0.05).astype(np.float32)
    b = np.abs(w.reshape(16, 8, 32)).max(axis=2)
    e8 = np.abs(oracle.dequantize(oracle.quantize_q8_0(w), oracle.Q8_0, 256) - w).reshape(16, 8, 32).max(axis=2)
    assert np.all(e8 <= b / 127 * (0.5 + 127 * 2.0 ** -11) * (1 + 1e-3))
    e4 = np.abs(oracle.dequantize(oracle.quantize_q4_0(w), oracle.Q4_0, 256) - w).reshape(16, 8, 32).max(axis=2)
    assert np.all(e4 <= b / 8 * (1 + 8 * 2.0 ** -11) * (1 + 1e-3))


def test_qkv_projection_oracle_is_linear_then_prologue():
    """The projection oracle = f64 matmul + bias, rounded to f32, then the prologue (Q, K) or a permute (V)."""
    rng = np.random.default_rng(3)
    N, L, K, H = 1, 12, 64, 2
    x = rng.standard_normal((N, L, K)).astype(np.float32)
    w = [rng.standard_normal((H * 128, K)).astype(np.float32) * 0.1 for _ in range(3)]
    b = [rng.standard_normal(H * 128).astype(np.float32), None, rng.standard_normal(H * 128).astype(np.float32)]
    tab = oracle.visual_rope_table((1, 3, 4))
    q, k, v = oracle.qkv_projection(x, w, b, H, rope_table=tab)
    yq = (x.astype(np.float64) @ w[0].T.astype(np.float64) + b[0]).astype(np.float32)
    np.testing.assert_array_equal(q, oracle.prologue(yq, H, rope_table=tab))
    yv = (x.astype(np.float64) @ w[2].T.astype(np.float64) + b[2]).astype(np.float32)
    np.testing.assert_array_equal(v, yv.reshape(N, L, H, 128).transpose(0, 2, 1, 3))
    assert k.shape == (N, H, L, 128)


def test_dequantize_matches_ggml_python_reference():
    """The block formats pinned a second way: gguf (ggml's own Python package, gguf-py 0.19.0 in this
    image) dequantizes the reference converter's q8_0 / q4_0 bytes to exactly the oracle's values.  (gguf's
    own q8_0 quantizer differs from the converter only on an all-zero block, stored with scale 0 instead of
    1 -- both decode to zeros; the oracle follows the converter that writes the model's GGUF files.)"""
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    g = np.load(QUANT_GOLD)
    for case in ("rand", "heavy", "edge"):
        K = g[f"{case}_w"].shape[1]
        for t, gt in ((oracle.Q8_0, gguf.GGMLQuantizationType.Q8_0), (oracle.Q4_0, gguf.GGMLQuantizationType.Q4_0)):
            raw = g[f"{case}_{'q8_0' if t == oracle.Q8_0 else 'q4_0'}"]
            ref = quants.dequantize(raw, gt).reshape(raw.shape[0], K)
            np.testing.assert_array_equal(oracle.dequantize(raw, t, K), ref)
