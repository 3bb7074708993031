"""The C-ABI library loads and exports every entry point include/kd_attn.h declares (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kd_attn.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:kd_attn_status|void|const char\s*\*|int32_t)\s+(kd_attn_\w+)\s*\(", src,
                                 flags=re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("kd_attn_create", "kd_attn_destroy", "kd_attn_flash_ext", "kd_attn_prologue",
                 "kd_attn_self_attention", "kd_attn_cross_attention", "kd_attn_allgather_heads"):
        assert must in names


def test_library_exports_every_declared_symbol(kd):
    lib = ctypes.CDLL(kd.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(kd.EXPORTED) == declared_functions()


def test_version(kd):
    assert kd.version() == (0, 2)


def test_create_without_gpu_fails_cleanly(kd):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    init = kd._Init()
    init.device, init.n_ranks, init.rank = 0, 1, 0
    h = ctypes.c_void_p(1234)
    rc = kd.lib.kd_attn_create(ctypes.byref(init), ctypes.byref(h))
    assert rc == kd.ERR_CUDA and not h.value


def test_create_rejects_bad_arguments(kd):
    init = kd._Init()
    init.device, init.n_ranks, init.rank = 0, 2, 5
    h = ctypes.c_void_p()
    assert kd.lib.kd_attn_create(ctypes.byref(init), ctypes.byref(h)) == kd.ERR_INVALID_ARGUMENT
    assert kd.lib.kd_attn_create(None, ctypes.byref(h)) == kd.ERR_INVALID_ARGUMENT
    assert kd.lib.kd_attn_flash_ext(None, None, None, None, None, 1.0, 0.0, 0.0, None, None, None, None, None) == \
        kd.ERR_INVALID_ARGUMENT


def test_kd_tensor_maps_torch_layout_to_ggml(kd):
    import torch
    t = torch.empty(2, 32, 100, 128, dtype=torch.bfloat16)      # ggml [128, 100, 32, 2]
    k = kd.KdTensor.of(t)
    assert list(k.ne) == [128, 100, 32, 2]
    assert list(k.nb) == [2, 256, 256 * 100, 256 * 100 * 32]
    v = t.permute(0, 2, 1, 3)                                   # ggml [128, 32, 100, 2] strided
    k = kd.KdTensor.of(v)
    assert list(k.ne) == [128, 32, 100, 2] and list(k.nb) == [2, 256 * 100, 256, 256 * 100 * 32]
    k = kd.KdTensor.of(torch.empty(5, 7, dtype=torch.float32))
    assert list(k.ne) == [7, 5, 1, 1] and list(k.nb) == [4, 28, 140, 140]


def test_tile_bitmap_layout(kd):
    """tile_mask layout of kd_attn_flash_ext: row qb holds ceil(n_kb / 8) bytes, tile kb is bit kb % 8
    of byte kb // 8 (least significant bit first)."""
    import numpy as np
    keep = np.zeros((3, 11), bool)
    keep[0, 0] = keep[1, 8] = keep[2, 10] = keep[2, 7] = True
    b = kd.tile_bitmap(keep)
    assert b.shape == (3, 2) and b.dtype == np.uint8
    assert b[0].tolist() == [1, 0] and b[1].tolist() == [0, 1] and b[2].tolist() == [0x80, 0x04]


def test_set_log_callback_roundtrip(kd):
    """The process-wide logger is callable without a GPU: set, then restore the default."""
    kd.set_log_callback(lambda lvl, txt: None)
    kd.set_log_callback(None)


def test_noalloc_argument_checks_without_a_device(kd):
    """kd_attn_flash_ext_noalloc rejects malformed calls with ggml_flash_attn_ext's error classes
    before it touches a device: unsupported features and layouts -> ERR_UNSUPPORTED, inconsistent
    shapes -> ERR_INVALID_ARGUMENT.  Host tensors stand in for the operands (only their shapes and
    strides are read).  Skipped where a GPU is present, so that no launch could ever see them."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    bf = torch.bfloat16
    N, H, Lq, Lk = 1, 4, 64, 96
    q = torch.zeros(N, H, Lq, 128, dtype=bf)
    k = torch.zeros(N, H, Lk, 128, dtype=bf)
    v = torch.zeros(N, H, Lk, 128, dtype=bf)
    out = torch.zeros(N, Lq, H, 128, dtype=bf)

    def status(q=q, k=k, v=v, out=out, mask=None, scale=0.088, max_bias=0.0, logit_softcap=0.0):
        return kd.lib.kd_attn_flash_ext_noalloc(kd._ref(q), kd._ref(k), kd._ref(v), kd._ref(mask), float(scale),
                                                float(max_bias), float(logit_softcap), None, None, kd._ref(out),
                                                None, None)

    assert status(max_bias=1.0) == kd.ERR_UNSUPPORTED                       # ALiBi
    assert status(logit_softcap=30.0) == kd.ERR_UNSUPPORTED                 # soft-capping
    assert status(scale=-1.0) == kd.ERR_UNSUPPORTED
    assert status(q=torch.zeros(N, H, Lq, 64, dtype=bf)) == kd.ERR_UNSUPPORTED      # head_dim 64
    assert status(k=k.float(), v=v.float()) == kd.ERR_UNSUPPORTED           # K/V must be f16 or bf16
    assert status(k=k.half()) == kd.ERR_UNSUPPORTED                         # K and V types differ
    assert status(v=torch.zeros(N, H, Lk + 1, 128, dtype=bf)) == kd.ERR_INVALID_ARGUMENT
    assert status(k=torch.zeros(N, 3, Lk, 128, dtype=bf), v=torch.zeros(N, 3, Lk, 128, dtype=bf)) == \
        kd.ERR_INVALID_ARGUMENT                                             # 4 heads over 3 K/V heads
    assert status(out=torch.zeros(N, Lq, H + 1, 128, dtype=bf)) == kd.ERR_INVALID_ARGUMENT
    assert status(mask=torch.zeros(1, 1, Lq, Lk, dtype=torch.float32)) == kd.ERR_UNSUPPORTED   # f32 mask
    assert status(mask=torch.zeros(1, 1, Lq, Lk - 1, dtype=torch.float16)) == kd.ERR_INVALID_ARGUMENT
    assert status(mask=torch.zeros(1, 3, Lq, Lk, dtype=torch.float16)) == kd.ERR_INVALID_ARGUMENT  # 3 planes, 4 heads
    # a well-formed call passes every check and stops at the first device query
    assert status() == kd.ERR_CUDA
