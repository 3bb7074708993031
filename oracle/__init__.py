"""numpy front end of the CPU oracle (oracle/kd_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline / reference arm.  The shipped
library never imports it.

Array convention: a ggml tensor with sizes ne = {ne0, ne1, ne2, ne3} is the
numpy array of shape (ne3, ne2, ne1, ne0) -- the last axis is ggml's
fastest-varying dim 0.  bf16 data is carried as uint16 bit patterns with an
explicit type tag.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .build_oracle import LIB, build_oracle

F32, F16, BF16 = 0, 1, 30
EXACT, GGML = 0, 1

_lib = None


class _Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("type", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_int64 * 4)]


def lib():
    global _lib
    if _lib is None:
        build_oracle()
        L = ctypes.CDLL(LIB)
        L.kdo_philox_randn.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64,
                                       ctypes.c_void_p, ctypes.c_int]
        L.kdo_rope_freqs.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
        L.kdo_text_rope_table.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
        L.kdo_visual_rope_table.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p]
        L.kdo_rms_norm_heads.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_float, ctypes.c_void_p, ctypes.c_int]
        L.kdo_rope_apply.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        L.kdo_flash_attn_ext.argtypes = [ctypes.POINTER(_Tensor)] * 4 + [
            ctypes.c_float, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.kdo_flash_attn_ext.restype = ctypes.c_int
        L.kdo_f32_to_f16.argtypes = [ctypes.c_float]
        L.kdo_f32_to_f16.restype = ctypes.c_uint16
        L.kdo_convert.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p]
        L.kdo_to_f32.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p]
        _lib = L
    return _lib


def nthreads():
    return int(os.environ.get("KD_ORACLE_THREADS", os.cpu_count() or 1))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- dtypes
def to_type(x, t):
    """f32 array -> array holding type t (float32, float16, or uint16 bf16 bits), RNE."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if t == F32:
        return x.copy()
    out = np.empty(x.shape, dtype=np.float16 if t == F16 else np.uint16)
    lib().kdo_convert(_ptr(x), x.size, t, _ptr(out))
    return out


def to_f32(x, t):
    x = np.ascontiguousarray(x)
    out = np.empty(x.shape, dtype=np.float32)
    lib().kdo_to_f32(_ptr(x), t, x.size, _ptr(out))
    return out


def type_of(a):
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(f"unsupported dtype {a.dtype}")


# ---------------------------------------------------------------- inputs / rope / norm
def philox_randn(seed, n, offset=0):
    out = np.empty(int(n), dtype=np.float32)
    lib().kdo_philox_randn(seed, offset, int(n), _ptr(out), nthreads())
    return out


def rope_freqs(dim, theta=10000.0):
    out = np.empty(dim, dtype=np.float32)
    lib().kdo_rope_freqs(dim, theta, _ptr(out))
    return out


def text_rope_table(seq_len, head_dim, theta=10000.0):
    out = np.empty((seq_len, head_dim), dtype=np.float32)
    lib().kdo_text_rope_table(seq_len, head_dim, theta, _ptr(out))
    return out


def visual_rope_table(grid, axes=(32, 48, 48), scale=(1.0, 1.0, 1.0), theta=10000.0):
    nt, nh, nw = grid
    ax = np.asarray(axes, dtype=np.int32)
    sc = np.asarray(scale, dtype=np.float32)
    out = np.empty((nt * nh * nw, int(ax.sum())), dtype=np.float32)
    lib().kdo_visual_rope_table(nt, nh, nw, _ptr(ax), _ptr(sc), theta, _ptr(out))
    return out


def rms_norm_heads(x, head_dim, gain=None, eps=1e-6):
    """x: float32 array whose size is a multiple of head_dim; normalises each head_dim row."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    g = None if gain is None else np.ascontiguousarray(gain, dtype=np.float32)
    lib().kdo_rms_norm_heads(_ptr(x), x.size // head_dim, head_dim, None if g is None else _ptr(g),
                             eps, _ptr(y), nthreads())
    return y


def rope_apply(x, n_head, head_dim, table):
    """x: (N, L, n_head*head_dim) float32 (ggml [C, L, N]); returns a rotated copy."""
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    N, L = x.shape[0], x.shape[1]
    t = np.ascontiguousarray(table, dtype=np.float32)
    lib().kdo_rope_apply(_ptr(x), L, N, n_head, head_dim, _ptr(t), nthreads())
    return x


# ---------------------------------------------------------------- flash_attn_ext
def _tensor(a, t=None):
    if a.ndim != 4:
        raise ValueError("oracle tensors are 4-D (ne3, ne2, ne1, ne0)")
    T = _Tensor()
    T.data = a.ctypes.data
    T.type = type_of(a) if t is None else t
    for i in range(4):
        T.ne[i] = a.shape[3 - i]
        T.nb[i] = a.strides[3 - i]
    return T


def flash_attn_ext(q, k, v, mask=None, scale=None, kv_len=None, mode=GGML, lse=False):
    """ggml_flash_attn_ext on numpy arrays.

    q: (N, H, Lq, D) f32/f16/bf16-bits; k, v: (Nkv, Hkv, Lk, D) f16 or bf16-bits (or f32);
    mask: (mn, mh, >=Lq, >=Lk) float16 or None; kv_len: (N,) int32 or None.
    Returns out (N, Lq, H, D) float32 [= ggml dst [D, H, Lq, N]] and, if lse, (N, H, Lq) float32.
    """
    N, H, Lq, D = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    out = np.empty((N, Lq, H, v.shape[3]), dtype=np.float32)
    l = np.empty((N, H, Lq), dtype=np.float32) if lse else None
    kl = None if kv_len is None else np.ascontiguousarray(kv_len, dtype=np.int32)
    tq, tk, tv = _tensor(q), _tensor(k), _tensor(v)
    tm = None if mask is None else _tensor(mask, F16)
    rc = lib().kdo_flash_attn_ext(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                  None if tm is None else ctypes.byref(tm), float(scale),
                                  None if kl is None else _ptr(kl), mode, _ptr(out),
                                  None if l is None else _ptr(l), nthreads())
    if rc != 0:
        raise ValueError(f"kdo_flash_attn_ext rejected the shapes (code {rc})")
    return (out, l) if lse else out


def self_attention(q_in, k_in, v_in, n_head, q_gain=None, k_gain=None, rope_table=None,
                   kv_type=F16, q_type=None, eps=1e-6, mask=None, kv_len=None, mode=GGML, lse=False):
    """The CrossDiT attention core, as the reference runs it on the flash path.

    q_in/k_in/v_in: (N, L, C) float32, the to_query/to_key/to_value outputs (ggml [C, L, N]).
    RMSNorm per head on q and k (crossdit.hpp:135-136 / :192-193), RoPE when a table is
    given (crossdit.hpp:140-141), permute to [d, L, H, N] (ops.hpp:122-131), K and V cast to
    kv_type (ops.hpp:167-169), Q kept f32 (ggml converts it to K's type for the dot, or to
    q_type when given), flash_attn_ext with scale 1/sqrt(d) (ops.hpp:161,176).
    Returns (N, Lq, C) float32 [= ggml [C, Lq, N], ops.hpp:204-206] (and the LSE).
    """
    N, Lq, C = q_in.shape
    Lk = k_in.shape[1]
    d = C // n_head
    q = rms_norm_heads(q_in, d, q_gain, eps)
    k = rms_norm_heads(k_in, d, k_gain, eps)
    if rope_table is not None:
        q = rope_apply(q, n_head, d, rope_table)
        k = rope_apply(k, n_head, d, rope_table)
    q4 = np.ascontiguousarray(q.reshape(N, Lq, n_head, d).transpose(0, 2, 1, 3))
    k4 = np.ascontiguousarray(k.reshape(N, Lk, n_head, d).transpose(0, 2, 1, 3))
    v4 = np.ascontiguousarray(np.asarray(v_in, np.float32).reshape(N, Lk, n_head, d).transpose(0, 2, 1, 3))
    if q_type is not None and q_type != F32:
        q4 = to_type(q4, q_type)
    k4 = to_type(k4, kv_type)
    v4 = to_type(v4, kv_type)
    r = flash_attn_ext(q4, k4, v4, mask=mask, kv_len=kv_len, mode=mode, lse=lse)
    if lse:
        o, l = r
        return o.reshape(N, Lq, C), l
    return r.reshape(N, Lq, C)


def prologue(x_in, n_head, gain=None, rope_table=None, eps=1e-6):
    """RMSNorm (+RoPE) of one projection, returned as [d, L, H, N] f32 = numpy (N, H, L, d)."""
    N, L, C = x_in.shape
    d = C // n_head
    x = rms_norm_heads(x_in, d, gain, eps)
    if rope_table is not None:
        x = rope_apply(x, n_head, d, rope_table)
    return np.ascontiguousarray(x.reshape(N, L, n_head, d).transpose(0, 2, 1, 3))


# ---------------------------------------------------------------- metrics used by the gates
def parity_metrics(got, ref):
    """cosine, max-abs error / RMS(ref), max-abs error (float64)."""
    g = np.asarray(got, dtype=np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    cos = float(np.dot(g, r) / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-300))
    rms = float(np.sqrt(np.mean(r * r)))
    mae = float(np.max(np.abs(g - r))) if g.size else 0.0
    return {"cos": cos, "maxabs_over_rms": mae / (rms + 1e-300), "maxabs": mae, "rms": rms}
