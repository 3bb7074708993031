"""The allocation-free flash-attention entry point (kd_attn_flash_ext_noalloc).

Some callers cannot allocate device memory: an embedder whose device memory
belongs to another allocator (a ggml backend buffer, a serving arena) may not
call cudaMalloc behind that allocator's back.  For them the library offers one
entry point that needs no context and allocates nothing; its scratch is a
fixed-size device array inside the library.  This test calls it through the C
ABI twice in a row -- with different inputs, so stale scratch from the first
call would show in the second -- and checks each result against the fp64 CPU
oracle on the same rounded operands (the gates every parity test uses) and
against the ordinary context-based kd_attn_flash_ext.  It also checks that a
bounded device wait that runs out is reported by kd_attn_noalloc_status.  It
lives in its own file, named to be collected last, and works alone in a fresh
process or after the others.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_gates, lse_err, seeded

pytestmark = pytest.mark.gpu

# Whole-device free memory moves with other processes on a shared GPU and with the CUDA
# runtime's own lazy pools; a change below this bound cannot be a scratch-sized allocation.
FREE_MEM_SLACK = 2 << 20


def _case(seed, N=2, H=4, Lq=333, Lk=270, D=128):
    """f32 strided Q (so the Q-rounding scratch is used) and an f16 mask with mixed tiles (class scratch)."""
    q_in = seeded((N, Lq, H * D), seed, 0)
    kf = seeded((N, H, Lk, D), seed, 1)
    vf = seeded((N, H, Lk, D), seed, 2)
    rng = np.random.default_rng(seed)
    mask = (rng.normal(size=(N, 1, Lq, Lk)) * 0.3).astype(np.float16)
    mask[rng.random(mask.shape) < 0.2] = -np.inf
    mask[:, :, :64, 192:] = -np.inf
    kb, vb = oracle.to_type(kf, oracle.BF16), oracle.to_type(vf, oracle.BF16)
    qf = np.ascontiguousarray(q_in.reshape(N, Lq, H, D).transpose(0, 2, 1, 3))
    exact, lse_ref = oracle.flash_attn_ext(qf, kb, vb, mask=mask, mode=oracle.EXACT, lse=True)
    q = torch.from_numpy(q_in).cuda().view(N, Lq, H, D).permute(0, 2, 1, 3)
    k = torch.from_numpy(kb.view(np.int16)).cuda().view(torch.bfloat16)
    v = torch.from_numpy(vb.view(np.int16)).cuda().view(torch.bfloat16)
    return q, k, v, torch.from_numpy(mask).cuda(), exact, lse_ref


def test_noalloc_matches_oracle_and_context_entry_twice(kd):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = kd.Context(device=torch.cuda.current_device())
    try:
        for i, seed in enumerate((101, 202)):
            q, k, v, mask, exact, lse_ref = _case(seed)
            N, H, Lq, D = q.shape
            ref = torch.empty(N, Lq, H, D, device="cuda")
            ref_lse = torch.empty(N, H, Lq, device="cuda")
            ctx.flash_attn_ext(q, k, v, ref, mask=mask, lse=ref_lse)
            ctx.device_status()
            out = torch.full((N, Lq, H, D), float("nan"), device="cuda")
            lse = torch.full((N, H, Lq), float("nan"), device="cuda")
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            alloc_before, reserved_before = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
            kd.flash_attn_ext_noalloc(q, k, v, out, mask=mask, lse=lse)
            kd.noalloc_status()          # synchronises; no device-side wait ran out
            if i == 1:   # after the first call's one-time set-up nothing may be allocated
                assert torch.cuda.memory_allocated() == alloc_before
                assert torch.cuda.memory_reserved() == reserved_before
                assert abs(torch.cuda.mem_get_info()[0] - free_before) <= FREE_MEM_SLACK
            got = out.cpu().numpy()
            assert_gates(got, exact, lse=lse.cpu().numpy(), lse_ref=lse_ref, label=f"noalloc call {i + 1} vs oracle")
            assert_gates(got, ref.cpu().numpy(), label=f"noalloc call {i + 1} vs context path")
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
    # host memory is refused before anything is launched
    with pytest.raises(kd.KdAttnError) as e:
        kd.flash_attn_ext_noalloc(q.to(torch.bfloat16), k, k, torch.empty(2, 2048, 32, 128))
    assert e.value.status == kd.ERR_INVALID_ARGUMENT
    # the same problem with Q already in K's type needs no scratch and runs
    kd.flash_attn_ext_noalloc(q.to(torch.bfloat16), k, k, out)
    kd.noalloc_status()
    assert torch.isfinite(out).all()


def test_noalloc_status_reports_an_expired_wait(kd):
    """A bounded wait that nothing releases sets the sticky word; the status call reports it once."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    kd.noalloc_status()
    kd.noalloc_selftest_wait(50)
    with pytest.raises(kd.KdAttnError) as e:
        kd.noalloc_status()
    assert e.value.status == kd.ERR_DEVICE_TIMEOUT
    kd.noalloc_status()              # cleared by the read
