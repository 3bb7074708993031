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


# ---------------------------------------------------------------- Linear weights (ggml block formats)
# A Linear weight of ggml shape [K, C] is C rows of K elements; the quantized types store each row as
# K/32 blocks.  The quantizers restate the reference converter (scripts/convert_to_gguf.py:90-146), the
# dequantizers ggml's published block formats:
#   q8_0: 34 bytes = f16 d, 32 x int8 q;                        value = d * q
#   q4_0: 18 bytes = f16 d, 16 bytes, element j low nibble,
#         element j+16 high nibble;                              value = d * (nibble - 8)
Q4_0, Q8_0 = 2, 8
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}


def quantize_q8_0(w):
    """(rows, K) float -> (rows, K/32*34) uint8.  d = amax/127 (1 for an all-zero block), q = round-half-even
    (x / d) clipped to int8 -- numpy's round, as the converter uses; d is computed in f32 and stored as f16."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, K = w.shape
    b = w.reshape(rows, K // 32, 32)
    d = (np.abs(b).max(axis=2) / np.float32(127.0)).astype(np.float32)
    d[d == 0] = 1.0
    q = np.clip(np.round(b / d[..., None]), -128, 127).astype(np.int8)
    out = np.empty((rows, K // 32, 34), dtype=np.uint8)
    out[..., :2] = d.astype(np.float16)[..., None].view(np.uint8)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def quantize_q4_0(w):
    """(rows, K) float -> (rows, K/32*18) uint8.  d = (the element of largest magnitude, with its sign) / -8,
    nibble = trunc(x / d + 8.5) clipped to [0, 15] (x / d taken as x * (1/d) in f32; 1/d = 0 for an
    all-zero block); d stored as f16."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, K = w.shape
    b = w.reshape(rows, K // 32, 32)
    idx = np.abs(b).argmax(axis=2)
    signed_max = np.take_along_axis(b, idx[..., None], axis=2)[..., 0]
    d = (signed_max / np.float32(-8.0)).astype(np.float32)
    inv = np.zeros_like(d)
    nz = np.abs(b).max(axis=2) > 0
    inv[nz] = np.float32(1.0) / d[nz]
    lo = np.clip((b[..., :16] * inv[..., None] + np.float32(8.5)).astype(np.int32), 0, 15).astype(np.uint8)
    hi = np.clip((b[..., 16:] * inv[..., None] + np.float32(8.5)).astype(np.int32), 0, 15).astype(np.uint8)
    out = np.empty((rows, K // 32, 18), dtype=np.uint8)
    out[..., :2] = d.astype(np.float16)[..., None].view(np.uint8)
    out[..., 2:] = lo | (hi << 4)
    return out.reshape(rows, -1)


def dequantize(wq, type_, K):
    """ggml weight rows -> (rows, K) float32: q8_0 / q4_0 bytes, or f32 / f16 / bf16 (uint16 bits) elements."""
    if type_ == F32:
        return np.asarray(wq, np.float32).reshape(-1, K)
    if type_ in (F16, BF16):
        return to_f32(np.asarray(wq).reshape(-1, K), type_)
    wq = np.ascontiguousarray(wq, dtype=np.uint8)
    blocks = wq.reshape(wq.shape[0], K // 32, BLOCK_BYTES[type_])
    d = blocks[..., :2].copy().view(np.float16)[..., 0].astype(np.float32)
    if type_ == Q8_0:
        q = blocks[..., 2:].view(np.int8).astype(np.float32)
    elif type_ == Q4_0:
        p = blocks[..., 2:]
        q = np.concatenate([(p & 0x0F), (p >> 4)], axis=2).astype(np.float32) - 8.0
    else:
        raise ValueError(f"unknown weight type {type_}")
    return (d[..., None] * q).reshape(-1, K)


def linear(x, w, bias=None):
    """ops::linear (ops.hpp:27-42): ggml_mul_mat(w, x) + bias, in float64 on the given float32 operands.
    x: (..., K); w: (C, K) float32 (dequantized rows); bias: (C,) or None.  Returns (..., C) float64."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y


def qkv_projection(x, w, bias, n_head, q_gain=None, k_gain=None, rope_table=None, eps=1e-6):
    """to_query/to_key/to_value (crossdit.hpp:123-125) followed by the prologue of each projection.

    x: (N, L, K) float32; w / bias: 3-lists (q, k, v) of (C, K) float32 rows and (C,) or None -- an entry
    may be None to skip that projection.  Returns 3 arrays [d, L, H, N] = numpy (N, H, L, d) float32 (the
    f32 projections rounded to float32 before the prologue, as ggml stores them)."""
    outs = []
    for i in range(3):
        if w[i] is None:
            outs.append(None)
            continue
        y = linear(x, w[i], bias[i]).astype(np.float32)
        if i < 2:
            outs.append(prologue(y, n_head, q_gain if i == 0 else k_gain, rope_table, eps))
        else:
            N, L, C = y.shape
            outs.append(np.ascontiguousarray(y.reshape(N, L, n_head, C // n_head).transpose(0, 2, 1, 3)))
    return outs
