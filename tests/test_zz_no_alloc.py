"""The allocation-free flash-attention entry point (kd_attn_flash_ext_noalloc).

Some callers cannot allocate device memory: code that runs while a CUDA graph
is being captured, or an embedder whose device memory belongs to another
allocator (a ggml backend buffer, a serving arena).  For them the library
offers one entry point that needs no context and allocates nothing; its
scratch is a fixed-size device array inside the library.  This test calls it
through the C ABI twice in a row -- with different inputs, so stale scratch
from the first call would show in the second -- and checks each result
against the ordinary context-based kd_attn_flash_ext on the same inputs, with
the same gates the other parity tests use.  It lives in its own file, named to
be collected last, and works alone in a fresh process or after the others.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_gates, lse_err, seeded

pytestmark = pytest.mark.gpu


def _case(seed, N=2, H=4, Lq=333, Lk=270, D=128):
    """f32 strided Q (so the Q-rounding scratch is used) and an f16 mask with mixed tiles (class scratch)."""
    q_in = seeded((N, Lq, H * D), seed, 0)
    kf = seeded((N, H, Lk, D), seed, 1)
    vf = seeded((N, H, Lk, D), seed, 2)
    rng = np.random.default_rng(seed)
    mask = (rng.normal(size=(N, 1, Lq, Lk)) * 0.3).astype(np.float16)
    mask[rng.random(mask.shape) < 0.2] = -np.inf
    mask[:, :, :64, 192:] = -np.inf
    q = torch.from_numpy(q_in).cuda().view(N, Lq, H, D).permute(0, 2, 1, 3)
    k = torch.from_numpy(kf).cuda().to(torch.bfloat16)
    v = torch.from_numpy(vf).cuda().to(torch.bfloat16)
    return q, k, v, torch.from_numpy(mask).cuda()


def test_noalloc_matches_context_entry_twice(kd):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = kd.Context(device=torch.cuda.current_device())
    try:
        for i, seed in enumerate((101, 202)):
            q, k, v, mask = _case(seed)
            N, H, Lq, D = q.shape
            ref = torch.empty(N, Lq, H, D, device="cuda")
            ref_lse = torch.empty(N, H, Lq, device="cuda")
            ctx.flash_attn_ext(q, k, v, ref, mask=mask, lse=ref_lse)
            ctx.device_status()
            out = torch.full((N, Lq, H, D), float("nan"), device="cuda")
            lse = torch.full((N, H, Lq), float("nan"), device="cuda")
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            kd.flash_attn_ext_noalloc(q, k, v, out, mask=mask, lse=lse)
            torch.cuda.synchronize()
            if i == 1:   # after the first call's one-time set-up nothing may be allocated
                assert torch.cuda.mem_get_info()[0] == free_before
            assert_gates(out.cpu().numpy(), ref.cpu().numpy(), label=f"noalloc call {i + 1}")
            assert lse_err(lse.cpu().numpy(), ref_lse.cpu().numpy()) <= 1e-3
    finally:
        ctx.close()


def test_noalloc_rejects_problems_beyond_its_scratch(kd):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    # f32 Q of 2 x 32 x 2048 rows needs 32 MiB of rounding scratch > 16 MiB
    q = torch.zeros(2, 32, 2048, 128, device="cuda")
    k = torch.zeros(2, 32, 2048, 128, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(2, 2048, 32, 128, device="cuda")
    with pytest.raises(kd.KdAttnError) as e:
        kd.flash_attn_ext_noalloc(q, k, k, out)
    assert e.value.status == kd.ERR_UNSUPPORTED
    # the same problem with Q already in K's type needs no scratch and runs
    kd.flash_attn_ext_noalloc(q.to(torch.bfloat16), k, k, out)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
