"""kd_attn -- Python host side of libkd_attn (include/kd_attn.h) over ctypes.

Mirrors the operator interface of kandinsky.cpp's attention path:
  - ``attention(...)``       ops::attention flash branch (src/core/ops.hpp:107-207)
  - ``self_attention(...)``  DiTSelfAttention::forward core (src/models/crossdit.hpp:117-154)
  - ``cross_attention(...)`` DiTCrossAttention::forward core (src/models/crossdit.hpp:174-200)
  - ``flash_attn_ext(...)``  ggml_flash_attn_ext operator semantics (called at ops.hpp:176)
  - ``prologue(...)``        RMSNorm + RoPE + cast + permute (crossdit.hpp:132-141, rope.hpp:109-155)
with torch tensors as device buffers (PyTorch is only the allocator and the
stream provider here).  The compute always runs in libkd_attn.so; if that
library is missing this module raises at import -- there is no fallback.

Layout convention: a ggml tensor with sizes ne = (ne0, ne1, ne2, ne3) is the
torch tensor of shape (ne3, ne2, ne1, ne0); ``KdTensor.of`` converts shape and
strides accordingly (dim 0 = the last torch dim).
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# $KD_ATTN_LIBRARY selects another build of the library (e.g. one compiled with other tuning knobs)
LIB_PATH = os.environ.get("KD_ATTN_LIBRARY") or os.path.join(_HERE, "libkd_attn.so")

# status codes (kd_attn_status)
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_OUT_OF_MEMORY = -4
ERR_DEVICE_TIMEOUT = -5
ERR_NCCL = -6

# ggml type ids (kd_attn_type; Q4_0 / Q8_0 for Linear weights)
F32, F16, BF16 = 0, 1, 30
Q4_0, Q8_0 = 2, 8

EXPORTED = [
    "kd_attn_create", "kd_attn_destroy", "kd_attn_last_error", "kd_attn_device_status",
    "kd_attn_prologue", "kd_attn_flash_ext", "kd_attn_self_attention", "kd_attn_cross_attention",
    "kd_attn_allgather_heads", "kd_attn_fill_randn", "kd_attn_nccl_unique_id", "kd_attn_version",
    "kd_attn_flash_ext_noalloc", "kd_attn_self_attention_host", "kd_attn_qk_prologue",
    "kd_attn_tile_stats", "kd_attn_set_log_callback", "kd_attn_symmetric_alloc", "kd_attn_symmetric_free",
    "kd_attn_self_attention_sharded", "kd_attn_cross_attention_sharded", "kd_attn_attention",
    "kd_attn_selftest_wait", "kd_attn_noalloc_status", "kd_attn_noalloc_selftest_wait",
    "kd_attn_qkv_projection", "kd_attn_linear", "kd_attn_self_attention_block", "kd_attn_cross_attention_block",
    "kd_attn_self_attention_block_sharded",
]

# scratch held by the allocation-free entry point on each device (KD_ATTN_NOALLOC_SCRATCH_BYTES)
NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024


class KdAttnError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"kd_attn status {status}: {msg}")
        self.status = status


class KdTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("type", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4)]

    @staticmethod
    def of(t):
        """kd_tensor view of a torch tensor (ggml ne/nb from torch shape/strides, reversed)."""
        import torch
        types = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
        if t.dtype not in types:
            raise TypeError(f"unsupported dtype {t.dtype}")
        if t.dim() > 4:
            raise ValueError("at most 4 dims")
        es = t.element_size()
        shape = list(reversed(t.shape))      # ggml order: dim 0 fastest
        strides = list(reversed(t.stride()))
        k = KdTensor()
        k.data = t.data_ptr() if t.numel() else None
        k.type = types[t.dtype]
        for i in range(4):
            if i < t.dim():
                k.ne[i] = shape[i]
                k.nb[i] = strides[i] * es
            else:  # missing outer dims: size 1 with the packed stride
                k.ne[i] = 1
                k.nb[i] = k.nb[i - 1] * k.ne[i - 1] if i > 0 else es
        return k


class KdLinear(ctypes.Structure):
    """kd_linear: a Linear layer's weight in ggml layout [K, C] (C rows of K elements of `type`) + f32 bias."""
    _fields_ = [("data", ctypes.c_void_p), ("type", ctypes.c_int32), ("ne", ctypes.c_int64 * 2),
                ("nb1", ctypes.c_size_t), ("bias", ctypes.c_void_p)]

    @staticmethod
    def of(weight, type, in_features, out_features, bias=None):
        """weight: device tensor holding the rows (uint8 bytes of ggml blocks for q4_0/q8_0, or
        f32/f16/bf16 elements) shaped (out_features, row) -- one row per output feature."""
        w = KdLinear()
        w.data = weight.data_ptr()
        w.type = int(type)
        w.ne[0] = int(in_features)
        w.ne[1] = int(out_features)
        w.nb1 = weight.stride(0) * weight.element_size()
        w.bias = None if bias is None else bias.data_ptr()
        return w


class Rope3D(ctypes.Structure):
    """kd_rope3d: 3D (t,h,w) RoPE of rope.hpp:56-102, computed on the fly."""
    _fields_ = [("axes_dim", ctypes.c_int32 * 3), ("grid", ctypes.c_int32 * 3),
                ("scale_factor", ctypes.c_float * 3), ("theta", ctypes.c_float)]

    @staticmethod
    def make(grid, axes=(32, 48, 48), scale=(1.0, 1.0, 1.0), theta=10000.0):
        r = Rope3D()
        for i in range(3):
            r.axes_dim[i] = int(axes[i])
            r.grid[i] = int(grid[i])
            r.scale_factor[i] = float(scale[i])
        r.theta = float(theta)
        return r


LOG_CB = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p)


class _Init(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("n_ranks", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("nccl_unique_id", ctypes.c_void_p), ("log_cb", LOG_CB), ("log_user_data", ctypes.c_void_p)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with kandinsky.cpp_b200/build.py "
                          "(libkd_attn has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, T = ctypes.c_void_p, ctypes.POINTER(KdTensor)
    st = ctypes.c_int
    L.kd_attn_create.argtypes = [ctypes.POINTER(_Init), ctypes.POINTER(ctypes.c_void_p)]
    L.kd_attn_create.restype = st
    L.kd_attn_destroy.argtypes = [P]
    L.kd_attn_destroy.restype = None
    L.kd_attn_last_error.argtypes = [P]
    L.kd_attn_last_error.restype = ctypes.c_char_p
    L.kd_attn_device_status.argtypes = [P, P]
    L.kd_attn_device_status.restype = st
    L.kd_attn_prologue.argtypes = [P, T, ctypes.c_int32, ctypes.c_int32, P, ctypes.c_float,
                                   ctypes.POINTER(Rope3D), T, P]
    L.kd_attn_prologue.restype = st
    L.kd_attn_attention.argtypes = [P, T, T, T, ctypes.c_int32, T, ctypes.c_int32, T, P, P]
    L.kd_attn_attention.restype = st
    L.kd_attn_qk_prologue.argtypes = [P, T, T, T, P, P, ctypes.c_float, ctypes.POINTER(Rope3D), ctypes.c_int32,
                                      T, T, T, P]
    L.kd_attn_qk_prologue.restype = st
    W = ctypes.POINTER(KdLinear)
    L.kd_attn_qkv_projection.argtypes = [P, T, W, W, W, P, P, ctypes.c_float, ctypes.POINTER(Rope3D),
                                         ctypes.c_int32, T, T, T, P]
    L.kd_attn_qkv_projection.restype = st
    L.kd_attn_linear.argtypes = [P, T, W, T, P]
    L.kd_attn_linear.restype = st
    L.kd_attn_self_attention_block.argtypes = [P, T, W, W, W, W, ctypes.c_int32, P, P, ctypes.c_float,
                                               ctypes.POINTER(Rope3D), T, P]
    L.kd_attn_self_attention_block.restype = st
    L.kd_attn_cross_attention_block.argtypes = [P, T, T, W, W, W, W, ctypes.c_int32, P, P, ctypes.c_float, T, P, T, P]
    L.kd_attn_cross_attention_block.restype = st
    L.kd_attn_self_attention_block_sharded.argtypes = [P, T, W, W, W, W, ctypes.c_int32, P, P, ctypes.c_float,
                                                       ctypes.POINTER(Rope3D), T, T, P]
    L.kd_attn_self_attention_block_sharded.restype = st
    L.kd_attn_flash_ext.argtypes = [P, T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float, P, P, T, P, P]
    L.kd_attn_flash_ext.restype = st
    L.kd_attn_self_attention.argtypes = [P, T, T, T, ctypes.c_int32, P, P, ctypes.c_float,
                                         ctypes.POINTER(Rope3D), ctypes.c_int32, T, P, P]
    L.kd_attn_self_attention.restype = st
    L.kd_attn_self_attention_host.argtypes = [P, T, T, T, ctypes.c_int32, P, P, ctypes.c_float,
                                              ctypes.POINTER(Rope3D), ctypes.c_int32, T, P]
    L.kd_attn_self_attention_host.restype = st
    L.kd_attn_cross_attention.argtypes = [P, T, T, T, ctypes.c_int32, P, P, ctypes.c_float, T, P,
                                          ctypes.c_int32, T, P, P]
    L.kd_attn_cross_attention.restype = st
    L.kd_attn_allgather_heads.argtypes = [P, T, T, P]
    L.kd_attn_allgather_heads.restype = st
    L.kd_attn_fill_randn.argtypes = [P, P, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32, P]
    L.kd_attn_fill_randn.restype = st
    L.kd_attn_nccl_unique_id.argtypes = [P]
    L.kd_attn_nccl_unique_id.restype = st
    L.kd_attn_flash_ext_noalloc.argtypes = [T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float, P, P, T, P,
                                            P]
    L.kd_attn_flash_ext_noalloc.restype = st
    L.kd_attn_noalloc_status.argtypes = [P]
    L.kd_attn_noalloc_status.restype = st
    L.kd_attn_noalloc_selftest_wait.argtypes = [ctypes.c_uint32, P]
    L.kd_attn_noalloc_selftest_wait.restype = st
    L.kd_attn_symmetric_alloc.argtypes = [P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
    L.kd_attn_symmetric_alloc.restype = st
    L.kd_attn_symmetric_free.argtypes = [P, P, P]
    L.kd_attn_symmetric_free.restype = st
    L.kd_attn_self_attention_sharded.argtypes = [P, T, T, T, ctypes.c_int32, P, P, ctypes.c_float,
                                                 ctypes.POINTER(Rope3D), ctypes.c_int32, T, P]
    L.kd_attn_self_attention_sharded.restype = st
    L.kd_attn_cross_attention_sharded.argtypes = [P, T, T, T, ctypes.c_int32, P, P, ctypes.c_float, T, P,
                                                  ctypes.c_int32, T, P]
    L.kd_attn_cross_attention_sharded.restype = st
    L.kd_attn_selftest_wait.argtypes = [P, ctypes.c_uint32, P]
    L.kd_attn_selftest_wait.restype = st
    L.kd_attn_tile_stats.argtypes = [P, P, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int32]
    L.kd_attn_tile_stats.restype = st
    L.kd_attn_set_log_callback.argtypes = [LOG_CB, P]
    L.kd_attn_set_log_callback.restype = None
    L.kd_attn_version.argtypes = []
    L.kd_attn_version.restype = ctypes.c_int32
    return L


lib = _load()


def version():
    v = lib.kd_attn_version()
    return (v >> 16, v & 0xFFFF)


_global_log_cb = None


def set_log_callback(log=None):
    """kd_attn_set_log_callback: process-wide logger log(level, text) for contexts created without
    one and for the allocation-free entry point; None restores the stderr default."""
    global _global_log_cb
    cb = LOG_CB(lambda lvl, txt, _u: log(lvl, txt.decode())) if log else LOG_CB()
    lib.kd_attn_set_log_callback(cb, None)
    _global_log_cb = cb  # keep the trampoline alive while the library may call it


def tile_bitmap(keep):
    """Pack a (n_qb, n_kb) bool array of kept 64x64 tiles into kd_attn_flash_ext's tile_mask layout
    (row qb = ceil(n_kb / 8) bytes, tile kb = bit kb % 8 of byte kb // 8)."""
    import numpy as np
    keep = np.asarray(keep, dtype=bool)
    return np.packbits(keep, axis=1, bitorder="little")


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    rc = lib.kd_attn_nccl_unique_id(buf)
    if rc != OK:
        raise KdAttnError(rc, "ncclGetUniqueId failed")
    return buf.raw


def _stream_ptr(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _ref(t):
    return None if t is None else ctypes.byref(KdTensor.of(t))


class _DeviceBuffer:
    """__cuda_array_interface__ over library-owned device memory, so torch can view it without a copy."""

    def __init__(self, ptr, shape, dtype, device):
        self.ptr, self.shape, self.dtype, self.device = ptr, shape, dtype, device

    def tensor(self):
        import torch
        if self.dtype == torch.bfloat16:   # no bf16 typestr: view 16-bit storage, reinterpret
            t = _DeviceBuffer(self.ptr, self.shape, torch.int16, self.device).tensor()
            return t.view(torch.bfloat16)
        self.__cuda_array_interface__ = {"shape": self.shape, "typestr": {torch.float32: "<f4", torch.float16: "<f2",
                                                                         torch.int16: "<i2"}[self.dtype],
                                         "data": (self.ptr, False), "version": 3, "strides": None}
        with torch.cuda.device(self.device):
            return torch.as_tensor(self, device=f"cuda:{self.device}")


class Context:
    """kd_attn_ctx: per-device state (operand scratch, error words, NCCL communicator)."""

    def __init__(self, device=0, n_ranks=1, rank=0, nccl_id: bytes | None = None, log=None):
        init = _Init()
        init.device, init.n_ranks, init.rank = int(device), int(n_ranks), int(rank)
        self._id_buf = None
        if nccl_id is not None:
            self._id_buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
            init.nccl_unique_id = ctypes.cast(self._id_buf, ctypes.c_void_p)
        self._cb = LOG_CB(lambda lvl, txt, _u: log(lvl, txt.decode())) if log else LOG_CB()
        init.log_cb = self._cb
        h = ctypes.c_void_p()
        rc = lib.kd_attn_create(ctypes.byref(init), ctypes.byref(h))
        if rc != OK:
            raise KdAttnError(rc, f"kd_attn_create(device={device}) failed")
        self.handle = h
        self.device = int(device)
        self.n_ranks = int(n_ranks)
        self.rank = int(rank)

    def close(self):
        if getattr(self, "handle", None):
            lib.kd_attn_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def check(self, rc):
        if rc != OK:
            raise KdAttnError(rc, lib.kd_attn_last_error(self.handle).decode())

    def device_status(self, stream=None):
        """Synchronise and read/clear the device error word (bounded-wait timeouts)."""
        self.check(lib.kd_attn_device_status(self.handle, _stream_ptr(stream)))

    # -------------------------------------------------------------- entry points
    def prologue(self, x, n_head, y, norm=True, gain=None, eps=1e-6, rope=None, stream=None):
        """x: (N, L, C) f32 -> y: (N, n_head, L, d) f32/f16/bf16 (ggml [d, L, H, N]), d = C / n_head = 128 or 64."""
        self.check(lib.kd_attn_prologue(self.handle, _ref(x), int(n_head), 1 if norm else 0, _ptr(gain),
                                        float(eps), None if rope is None else ctypes.byref(rope), _ref(y),
                                        _stream_ptr(stream)))
        return y

    def qk_prologue(self, q_in, k_in, v_in, q_out, k_out, v_out, q_gain=None, k_gain=None, eps=1e-6, rope=None,
                    stream=None):
        """One launch: q_in/k_in (N, L, C) f32 -> RMSNorm (+RoPE) -> q_out/k_out (N, H, L, d); v_in -> v_out
        cast only.  Any (in, out) pair may be None."""
        if len({t.dtype for t in (q_out, k_out, v_out) if t is not None}) != 1:
            raise ValueError("outputs must share one dtype")
        out_dtype = KdTensor.of(next(t for t in (q_out, k_out, v_out) if t is not None)).type
        self.check(lib.kd_attn_qk_prologue(self.handle, _ref(q_in), _ref(k_in), _ref(v_in), _ptr(q_gain),
                                           _ptr(k_gain), float(eps), None if rope is None else ctypes.byref(rope),
                                           int(out_dtype), _ref(q_out), _ref(k_out), _ref(v_out),
                                           _stream_ptr(stream)))
        return q_out, k_out, v_out

    def qkv_projection(self, x, wq, wk, wv, q_out, k_out, v_out, q_gain=None, k_gain=None, eps=1e-6, rope=None,
                       stream=None):
        """to_query/to_key/to_value + prologue as one GEMM: x (N, L, K) f32; wq/wk/wv KdLinear or None;
        q_out/k_out/v_out (N, H, L, 128) f16/bf16 (ggml [128, L, H, N]) or None with their weight."""
        outs = [t for t in (q_out, k_out, v_out) if t is not None]
        if len({t.dtype for t in outs}) > 1:
            raise ValueError("outputs must share one dtype")
        out_dtype = KdTensor.of(outs[0]).type if outs else BF16
        ref_w = lambda w: None if w is None else ctypes.byref(w)
        self.check(lib.kd_attn_qkv_projection(self.handle, _ref(x), ref_w(wq), ref_w(wk), ref_w(wv), _ptr(q_gain),
                                              _ptr(k_gain), float(eps), None if rope is None else ctypes.byref(rope),
                                              int(out_dtype), _ref(q_out), _ref(k_out), _ref(v_out),
                                              _stream_ptr(stream)))
        return q_out, k_out, v_out

    def linear(self, x, w, y, stream=None):
        """ops::linear: y (N, L, C) = x (N, L, K) W^T + b; x f32 or bf16, w a KdLinear, y f32/bf16/f16."""
        self.check(lib.kd_attn_linear(self.handle, _ref(x), ctypes.byref(w), _ref(y), _stream_ptr(stream)))
        return y

    def self_attention_block(self, x, wq, wk, wv, wo, n_head, y, q_gain=None, k_gain=None, eps=1e-6, rope=None,
                             stream=None):
        """DiTSelfAttention::forward from the hidden states x (N, L, C) f32 to y (N, L, C_out); n_head heads of
        C / n_head = 128 or 64."""
        self.check(lib.kd_attn_self_attention_block(self.handle, _ref(x), ctypes.byref(wq), ctypes.byref(wk),
                                                    ctypes.byref(wv), ctypes.byref(wo), int(n_head), _ptr(q_gain),
                                                    _ptr(k_gain),
                                                    float(eps), None if rope is None else ctypes.byref(rope), _ref(y),
                                                    _stream_ptr(stream)))
        return y

    def cross_attention_block(self, x_query, x_kv, wq, wk, wv, wo, n_head, y, q_gain=None, k_gain=None, eps=1e-6,
                              mask=None, kv_len=None, stream=None):
        """DiTCrossAttention::forward: x_query (N, Lq, C) f32 visual, x_kv (N, Lk, C) f32 text -> y (N, Lq, C_out);
        kv_len: device int32 (N,) valid text lengths, mask: f16 (mn, mh, >=Lq, >=Lk), either may be None."""
        self.check(lib.kd_attn_cross_attention_block(self.handle, _ref(x_query), _ref(x_kv), ctypes.byref(wq),
                                                     ctypes.byref(wk), ctypes.byref(wv), ctypes.byref(wo),
                                                     int(n_head), _ptr(q_gain), _ptr(k_gain), float(eps), _ref(mask),
                                                     _ptr(kv_len), _ref(y), _stream_ptr(stream)))
        return y

    def flash_attn_ext(self, q, k, v, out, mask=None, scale=None, kv_len=None, lse=None, max_bias=0.0,
                       logit_softcap=0.0, tile_mask=None, stream=None):
        """ggml_flash_attn_ext.  q: (N, H, Lq, D); k, v: (Nkv, Hkv, Lk, D), D = 128, 64 or 512;
        mask: (mn, mh, >=Lq, >=Lk) f16 or None; out: (N, Lq, H, D); lse: (N, H, Lq) f32 or None;
        tile_mask: device uint8 bitmap of kept 64x64 tiles (tile_bitmap layout) or None."""
        if scale is None:
            scale = 1.0 / (q.shape[-1] ** 0.5)
        self.check(lib.kd_attn_flash_ext(self.handle, _ref(q), _ref(k), _ref(v), _ref(mask), float(scale),
                                         float(max_bias), float(logit_softcap), _ptr(kv_len), _ptr(tile_mask),
                                         _ref(out), _ptr(lse), _stream_ptr(stream)))
        return out

    def selftest_wait(self, wait_ms=50, stream=None):
        """kd_attn_selftest_wait: one bounded device wait that nothing releases; the next
        device_status() raises ERR_DEVICE_TIMEOUT."""
        self.check(lib.kd_attn_selftest_wait(self.handle, int(wait_ms), _stream_ptr(stream)))

    def tile_stats(self, reset=False, stream=None):
        """(K/V tiles loaded, Q-tile x K/V-tile products computed) since the last reset."""
        out = (ctypes.c_uint64 * 2)()
        self.check(lib.kd_attn_tile_stats(self.handle, _stream_ptr(stream), out, 1 if reset else 0))
        return int(out[0]), int(out[1])

    def ops_attention(self, q_in, k_in, v_in, n_head, out, mask=None, op_type=F16, lse=None, stream=None):
        """kd_attn_attention = ops::attention's flash branch: q_in (N, Lq, C), k_in/v_in (N, Lk, C_kv) f32
        (GQA when C_kv < C), no RMSNorm/RoPE; mask f16 (mn, mh, >=Lq, >=Lk) or None; out (N, Lq, C)."""
        self.check(lib.kd_attn_attention(self.handle, _ref(q_in), _ref(k_in), _ref(v_in), int(n_head), _ref(mask),
                                         int(op_type), _ref(out), _ptr(lse), _stream_ptr(stream)))
        return out

    def self_attention(self, q_in, k_in, v_in, n_head, out, rope=None, q_gain=None, k_gain=None, eps=1e-6,
                       op_type=BF16, lse=None, stream=None):
        """q_in/k_in/v_in: (N, L, C) f32 -> out (N, L, C) f32/bf16."""
        self.check(lib.kd_attn_self_attention(self.handle, _ref(q_in), _ref(k_in), _ref(v_in), int(n_head),
                                              _ptr(q_gain), _ptr(k_gain), float(eps),
                                              None if rope is None else ctypes.byref(rope), int(op_type), _ref(out),
                                              _ptr(lse), _stream_ptr(stream)))
        return out

    def self_attention_host(self, q_in, k_in, v_in, n_head, out, rope=None, q_gain=None, k_gain=None, eps=1e-6,
                            op_type=BF16, stream=None):
        """Host tensors q_in/k_in/v_in: (N, L, C) f32 (pinned for overlap) -> host out (N, L, C) f32/bf16;
        uploads, computes and downloads head group by head group.  Done when `stream` has drained."""
        for name, t in (("q_in", q_in), ("k_in", k_in), ("v_in", v_in), ("out", out)):
            if t.is_cuda:
                raise ValueError(f"{name} must be a host tensor")
        self.check(lib.kd_attn_self_attention_host(self.handle, _ref(q_in), _ref(k_in), _ref(v_in), int(n_head),
                                                   _ptr(q_gain), _ptr(k_gain), float(eps),
                                                   None if rope is None else ctypes.byref(rope), int(op_type),
                                                   _ref(out), _stream_ptr(stream)))
        return out

    def cross_attention(self, q_in, k_in, v_in, n_head, out, mask=None, kv_len=None, q_gain=None, k_gain=None,
                        eps=1e-6, op_type=BF16, lse=None, stream=None):
        self.check(lib.kd_attn_cross_attention(self.handle, _ref(q_in), _ref(k_in), _ref(v_in), int(n_head),
                                               _ptr(q_gain), _ptr(k_gain), float(eps), _ref(mask), _ptr(kv_len),
                                               int(op_type), _ref(out), _ptr(lse), _stream_ptr(stream)))
        return out

    def symmetric_tensor(self, shape, dtype):
        """kd_attn_symmetric_alloc (collective): a device tensor whose copies on every rank are mapped
        into each other, for self_attention_sharded's out_full.  Freed by symmetric_free or close()."""
        import torch
        n = 1
        for s_ in shape:
            n *= int(s_)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        self.check(lib.kd_attn_symmetric_alloc(self.handle, nbytes, ctypes.byref(ptr)))
        return _DeviceBuffer(ptr.value, tuple(int(x) for x in shape), dtype, self.device).tensor()

    def symmetric_free(self, t, stream=None):
        """kd_attn_symmetric_free (collective)."""
        self.check(lib.kd_attn_symmetric_free(self.handle, ctypes.c_void_p(t.data_ptr()), _stream_ptr(stream)))

    def self_attention_sharded(self, q_in, k_in, v_in, n_head_local, out_full, rope=None, q_gain=None, k_gain=None,
                               eps=1e-6, op_type=BF16, stream=None):
        """This rank's column shard (N, L, n_head_local*d) f32 of the projections -> every rank's
        out_full (N, L, n_ranks*n_head_local*d), the exchange fused into the flash epilogue."""
        self.check(lib.kd_attn_self_attention_sharded(self.handle, _ref(q_in), _ref(k_in), _ref(v_in),
                                                      int(n_head_local), _ptr(q_gain), _ptr(k_gain), float(eps),
                                                      None if rope is None else ctypes.byref(rope), int(op_type),
                                                      _ref(out_full), _stream_ptr(stream)))
        return out_full

    def self_attention_block_sharded(self, x, wq, wk, wv, wo, n_head_local, attn_full, y, q_gain=None, k_gain=None,
                                     eps=1e-6, rope=None, stream=None):
        """Heads sharded over the group: x (N, L, C) f32 replicated, this rank's Q/K/V weight shards (KdLinear,
        C_local = n_head_local * d outputs), the full wo; attn_full a symmetric bf16 (N, L, n_ranks*C_local);
        y (N, L, C_out)."""
        self.check(lib.kd_attn_self_attention_block_sharded(self.handle, _ref(x), ctypes.byref(wq), ctypes.byref(wk),
                                                            ctypes.byref(wv), ctypes.byref(wo), int(n_head_local),
                                                            _ptr(q_gain),
                                                            _ptr(k_gain), float(eps),
                                                            None if rope is None else ctypes.byref(rope),
                                                            _ref(attn_full), _ref(y), _stream_ptr(stream)))
        return y

    def cross_attention_sharded(self, q_in, k_in, v_in, n_head_local, out_full, mask=None, kv_len=None,
                                q_gain=None, k_gain=None, eps=1e-6, op_type=BF16, stream=None):
        """Cross-attention on this rank's heads -> every rank's out_full (exchange fused as above)."""
        self.check(lib.kd_attn_cross_attention_sharded(self.handle, _ref(q_in), _ref(k_in), _ref(v_in),
                                                       int(n_head_local), _ptr(q_gain), _ptr(k_gain), float(eps),
                                                       _ref(mask), _ptr(kv_len), int(op_type), _ref(out_full),
                                                       _stream_ptr(stream)))
        return out_full

    def allgather_heads(self, shard, full, stream=None):
        """shard: (N, Lq, H/n, D) -> full: (N, Lq, H, D), one NCCL all-gather + permute."""
        self.check(lib.kd_attn_allgather_heads(self.handle, _ref(shard), _ref(full), _stream_ptr(stream)))
        return full

    def fill_randn(self, dst, seed, offset=0, stream=None):
        """Philox4x32-10 + Box-Muller N(0,1) into a contiguous f32 tensor (rng.hpp:51-69 layout)."""
        self.check(lib.kd_attn_fill_randn(self.handle, _ptr(dst), dst.numel(), int(seed), int(offset),
                                          _stream_ptr(stream)))
        return dst


def flash_attn_ext_noalloc(q, k, v, out, mask=None, scale=None, kv_len=None, lse=None, max_bias=0.0,
                           logit_softcap=0.0, tile_mask=None, stream=None):
    """kd_attn_flash_ext_noalloc: flash_attn_ext without a Context and without any device allocation.

    For callers that may not allocate device memory (an embedder whose memory belongs to another
    allocator).  Runs on the current CUDA device, whose memory every tensor must be in; its scratch
    is a fixed NOALLOC_SCRATCH_BYTES device array shared by every call on that device, so calls must
    not overlap on the GPU.  Make the first call on a device before any stream capture.  Problems
    needing more scratch are rejected with ERR_UNSUPPORTED.  ``noalloc_status`` reports whether a
    device-side wait ran out since the last check.
    """
    if scale is None:
        scale = 1.0 / (q.shape[-1] ** 0.5)
    rc = lib.kd_attn_flash_ext_noalloc(_ref(q), _ref(k), _ref(v), _ref(mask), float(scale), float(max_bias),
                                       float(logit_softcap), _ptr(kv_len), _ptr(tile_mask), _ref(out), _ptr(lse),
                                       _stream_ptr(stream))
    if rc != OK:
        raise KdAttnError(rc, "kd_attn_flash_ext_noalloc failed (details on stderr)")
    return out


def noalloc_status(stream=None):
    """kd_attn_noalloc_status: synchronise, read and clear the allocation-free path's error word."""
    rc = lib.kd_attn_noalloc_status(_stream_ptr(stream))
    if rc != OK:
        raise KdAttnError(rc, "kd_attn_noalloc_status (details on stderr)")


def noalloc_selftest_wait(wait_ms=50, stream=None):
    """kd_attn_noalloc_selftest_wait: one bounded device wait that runs out on purpose."""
    rc = lib.kd_attn_noalloc_selftest_wait(int(wait_ms), _stream_ptr(stream))
    if rc != OK:
        raise KdAttnError(rc, "kd_attn_noalloc_selftest_wait (details on stderr)")


def attention(ctx: Context, q, k, v, n_head, mask=None, flash=True, op_type=F16, out_dtype=None, stream=None):
    """ops::attention (src/core/ops.hpp:107-207), flash branch, on device tensors.

    q: (N, Lq, C) f32, k, v: (N, Lk, C_kv) f32 -- the [C, L, N] ggml tensors of the reference.
    Permutes to [d, L, H, N] (ops.hpp:122-131), casts K/V to op_type (ops.hpp:167-169, f16 in the
    reference), runs flash_attn_ext with scale 1/sqrt(d) (ops.hpp:161,176) and returns (N, Lq, C)
    (ops.hpp:204-206).  GQA (C_kv < C) is broadcast by the kernel instead of repeated
    (ops.hpp:135-157).  The causal / non-flash branch is not covered (UNSUPPORTED).
    """
    import torch
    if not flash:
        raise KdAttnError(ERR_UNSUPPORTED, "only the flash branch of ops::attention is implemented")
    N, Lq, C = q.shape
    out = torch.empty(N, Lq, C, device=q.device, dtype=out_dtype or torch.float32)
    m = None
    if mask is not None:
        m = mask.to(torch.float16)
        while m.dim() < 4:
            m = m.unsqueeze(0)
    # one kd_attn_attention call: permutes + casts in the prologue kernel, then flash attention
    ctx.ops_attention(q, k, v, n_head, out, mask=m, op_type=op_type, stream=stream)
    return out
