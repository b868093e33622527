"""ctypes wrapper over liboracle.so, the CPU restatement of eyebrowse's
attention-path references.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker. The product package
(eyebrowse_b200) never imports it.

Each wrapper names the reference function it restates (crate-relative
path:line in the eyebrowse workspace); the C source keeps the reference's loop
order and f32 arithmetic.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32, F16, BF16 = 0, 1, 2

_fp = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t


def build() -> str:
    """Compile liboracle.so from eb_oracle.c (make, in this directory)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "eb_oracle.c")
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_rel_l2.restype = ctypes.c_float
        L.orc_rel_l2.argtypes = [_fp, _fp, _sz]
        L.orc_max_abs.restype = ctypes.c_float
        L.orc_max_abs.argtypes = [_fp, _fp, _sz]
        L.orc_round_f16.argtypes = [_fp, _sz]
        L.orc_round_bf16.argtypes = [_fp, _sz]
        L.orc_rmsnorm.argtypes = [_fp, _fp, _fp, _sz, _sz, ctypes.c_float]
        L.orc_rope.argtypes = [_fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz]
        L.orc_rope_tables.argtypes = [_fp, _fp, _sz, _sz, _sz, ctypes.c_float]
        L.orc_kv_write.argtypes = [_fp, _fp, _sz, _sz, _sz, _sz, _sz]
        L.orc_linear.argtypes = [_fp, _fp, _fp, _sz, _sz, _sz]
        L.orc_linear_threaded.argtypes = [_fp, _fp, _fp, _sz, _sz, _sz, ctypes.c_int]
        L.orc_attn_prefill.argtypes = [_fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz, ctypes.c_float]
        L.orc_attn_prefill_window.argtypes = [_fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz,
                                              ctypes.c_float, _sz]
        L.orc_attn_prefill_part.argtypes = [_fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz,
                                            ctypes.c_float, _sz, _sz, _sz, _sz, ctypes.c_int,
                                            _sz]
        L.orc_attn_decode.argtypes = [_fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz, _sz,
                                      ctypes.c_float]
        L.orc_attn_decode_window.argtypes = [_fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz, _sz,
                                             ctypes.c_float, _sz]
        L.orc_attn_decode_batched.argtypes = [_fp, _fp, _fp, _fp, _sz,
                                              ctypes.POINTER(ctypes.c_int32), _sz, _sz, _sz,
                                              _sz, _sz, ctypes.c_float, ctypes.c_int, _sz]
        L.orc_attention_prefill.argtypes = [_fp, _fp, _fp, _fp, _fp, _fp, ctypes.c_float, _fp,
                                            _fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz, _sz,
                                            ctypes.c_float, ctypes.c_int, ctypes.c_int, _sz]
        L.orc_attention_decode.argtypes = [_fp, _fp, _fp, _fp, _fp, _fp, ctypes.c_float, _fp,
                                           _fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz, _sz,
                                           ctypes.c_float, ctypes.c_int, _sz]
        _lib = L
    return _lib


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _p(a):
    if a is None:
        return None
    return a.ctypes.data_as(_fp)


def rel_l2(a, b) -> float:
    """testutil.rs:16-26"""
    a, b = _f32(a).ravel(), _f32(b).ravel()
    assert a.size == b.size, "rel_l2 length mismatch"
    return float(lib().orc_rel_l2(_p(a), _p(b), a.size))


def max_abs(a, b) -> float:
    a, b = _f32(a).ravel(), _f32(b).ravel()
    assert a.size == b.size
    return float(lib().orc_max_abs(_p(a), _p(b), a.size))


def round_f16(x) -> np.ndarray:
    """testutil.rs:62-64 (IEEE binary16, round to nearest even)."""
    y = _f32(x).copy()
    lib().orc_round_f16(_p(y), y.size)
    return y


def round_bf16(x) -> np.ndarray:
    y = _f32(x).copy()
    lib().orc_round_bf16(_p(y), y.size)
    return y


def round_as(x, kind: int) -> np.ndarray:
    if kind == F16:
        return round_f16(x)
    if kind == BF16:
        return round_bf16(x)
    return _f32(x).copy()


def rmsnorm(x, w, rows: int, dim: int, eps: float) -> np.ndarray:
    """testutil.rs:83-97"""
    x, w = _f32(x), _f32(w)
    out = np.empty(rows * dim, np.float32)
    lib().orc_rmsnorm(_p(x), _p(w), _p(out), rows, dim, eps)
    return out


def rope(x, cos, sin, seq: int, n_heads: int, hd: int, base_pos: int = 0) -> np.ndarray:
    """testutil.rs:101-125 with the kernel's base_pos (rope.rs:25-26)."""
    x, cos, sin = _f32(x), _f32(cos), _f32(sin)
    out = np.empty(seq * n_heads * hd, np.float32)
    lib().orc_rope(_p(x), _p(cos), _p(sin), _p(out), seq, n_heads, hd, base_pos)
    return out


def rope_tables(max_seq: int, hd: int, theta: float, rope_angles: int | None = None):
    """eyebrowse-nn/src/rope.rs:24-50 (Rope::build / build_partial)."""
    if rope_angles is None:
        rope_angles = hd // 2
    cos = np.empty(max_seq * (hd // 2), np.float32)
    sin = np.empty(max_seq * (hd // 2), np.float32)
    lib().orc_rope_tables(_p(cos), _p(sin), max_seq, hd, rope_angles, theta)
    return cos, sin


def kv_write(cache, src, hkv: int, count: int, hd: int, max_seq: int, dst_start: int):
    """ops.rs:70-87; returns an updated copy of `cache`."""
    cache = _f32(cache).copy()
    src = _f32(src)
    lib().orc_kv_write(_p(cache), _p(src), hkv, count, hd, max_seq, dst_start)
    return cache


def linear(x, w, m: int, in_f: int, out_f: int) -> np.ndarray:
    """testutil.rs:66-79 (cpu_linear): y [m, out_f] = x [m, in_f] @ w [out_f, in_f]^T,
    f32, k summed in order. Pass w already rounded to f16 (round_f16)."""
    x, w = _f32(x), _f32(w)
    y = np.empty(m * out_f, np.float32)
    lib().orc_linear(_p(x), _p(w), _p(y), m, in_f, out_f)
    return y


def linear_threaded(x, w, m: int, in_f: int, out_f: int, nthreads: int) -> np.ndarray:
    """linear() over `nthreads` threads by output feature (bit-identical)."""
    x, w = _f32(x), _f32(w)
    y = np.empty(m * out_f, np.float32)
    lib().orc_linear_threaded(_p(x), _p(w), _p(y), m, in_f, out_f, nthreads)
    return y


def attn_prefill(q, k, v, h: int, hkv: int, s: int, hd: int, scale: float | None = None,
                 window: int = 0):
    """testutil.rs:130-172 (scale defaults to the reference's hard-coded 1/sqrt(hd)).
    window > 0: row i attends key rows i - window < j <= i (HF's sliding-window
    causal mask; the reference has no sliding window)."""
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    q, k, v = _f32(q), _f32(k), _f32(v)
    o = np.empty(s * h * hd, np.float32)
    if window:
        lib().orc_attn_prefill_window(_p(q), _p(k), _p(v), _p(o), h, hkv, s, hd, float(scale),
                                      window)
    else:
        lib().orc_attn_prefill(_p(q), _p(k), _p(v), _p(o), h, hkv, s, hd, float(scale))
    return o


def attn_prefill_part(q, k, v, h, hkv, s, hd, scale, rows, heads, nthreads: int = 1,
                      window: int = 0):
    """Rows [rows[0], rows[1]) x heads [heads[0], heads[1]) of attn_prefill, threaded.
    Returns the full-size output buffer (untouched entries are zero)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    o = np.zeros(s * h * hd, np.float32)
    lib().orc_attn_prefill_part(_p(q), _p(k), _p(v), _p(o), h, hkv, s, hd, float(scale),
                                rows[0], rows[1], heads[0], heads[1], nthreads, window)
    return o


def attn_decode(q, kc, vc, h, hkv, pos, hd, max_seq, scale: float | None = None,
                window: int = 0):
    """testutil.rs:177-218 (window > 0: cache rows pos - window < j <= pos only)"""
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    q, kc, vc = _f32(q), _f32(kc), _f32(vc)
    o = np.empty(h * hd, np.float32)
    if window:
        lib().orc_attn_decode_window(_p(q), _p(kc), _p(vc), _p(o), h, hkv, pos, hd, max_seq,
                                     float(scale), window)
    else:
        lib().orc_attn_decode(_p(q), _p(kc), _p(vc), _p(o), h, hkv, pos, hd, max_seq,
                              float(scale))
    return o


def attn_decode_batched(q, kc, vc, pos, h, hkv, hd, max_seq, cache_stride, scale,
                        nthreads: int = 1, window: int = 0):
    """testutil.rs:177-218 applied per sequence of a batch (threaded)."""
    q, kc, vc = _f32(q), _f32(kc), _f32(vc)
    pos = np.ascontiguousarray(np.asarray(pos, dtype=np.int32))
    batch = pos.size
    o = np.empty(batch * h * hd, np.float32)
    lib().orc_attn_decode_batched(_p(q), _p(kc), _p(vc), _p(o), batch,
                                  pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                  h, hkv, hd, max_seq, cache_stride, float(scale), nthreads,
                                  window)
    return o


def attention_prefill(q, k, v, *, seq, h, hkv, hd, max_seq, scale, eps=1e-6,
                      q_norm_w=None, k_norm_w=None, v_norm_w=None, cos=None, sin=None,
                      kcache=None, vcache=None, cache_round=F32, q_round=F32, window=0):
    """eyebrowse-nn/src/attention.rs:49-117 after the projections.
    Returns (o, kcache, vcache)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    kc = np.zeros(max_seq * hkv * hd, np.float32) if kcache is None else _f32(kcache).copy()
    vc = np.zeros(max_seq * hkv * hd, np.float32) if vcache is None else _f32(vcache).copy()
    o = np.empty(seq * h * hd, np.float32)
    qn, kn, vn = (None if w is None else _f32(w) for w in (q_norm_w, k_norm_w, v_norm_w))
    c = None if cos is None else _f32(cos)
    s = None if sin is None else _f32(sin)
    lib().orc_attention_prefill(_p(q), _p(k), _p(v), _p(qn), _p(kn), _p(vn), eps, _p(c), _p(s),
                                _p(kc), _p(vc), _p(o), seq, h, hkv, hd, max_seq, float(scale),
                                cache_round, q_round, window)
    return o, kc, vc


def attention_decode(q, k, v, *, pos, h, hkv, hd, max_seq, scale, kcache, vcache, eps=1e-6,
                     q_norm_w=None, k_norm_w=None, v_norm_w=None, cos=None, sin=None,
                     cache_round=F32, window=0):
    """eyebrowse-nn/src/attention.rs:120-185 after the projections.
    Returns (o, kcache, vcache) with the caches updated at row pos."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    kc = _f32(kcache).copy()
    vc = _f32(vcache).copy()
    o = np.empty(h * hd, np.float32)
    qn, kn, vn = (None if w is None else _f32(w) for w in (q_norm_w, k_norm_w, v_norm_w))
    c = None if cos is None else _f32(cos)
    s = None if sin is None else _f32(sin)
    lib().orc_attention_decode(_p(q), _p(k), _p(v), _p(qn), _p(kn), _p(vn), eps, _p(c), _p(s),
                               _p(kc), _p(vc), _p(o), pos, h, hkv, hd, max_seq, float(scale),
                               cache_round, window)
    return o, kc, vc


def ramp(n: int, off: float, step: float) -> np.ndarray:
    """The reference's test input generator, eyebrowse-kernels/src/attention.rs:170-172
    (`off + i as f32 * step`, evaluated in f32)."""
    i = np.arange(n, dtype=np.float32)
    return (np.float32(off) + i * np.float32(step)).astype(np.float32)


def prng(n: int, seed: int) -> np.ndarray:
    """eyebrowse-nn/src/testutil.rs:30-41 (xorshift64, values in [-1, 1))."""
    mask = (1 << 64) - 1
    s = (seed + 0x9E3779B97F4A7C15) & mask
    out = np.empty(n, np.float32)
    for i in range(n):
        s ^= (s << 13) & mask
        s ^= s >> 7
        s ^= (s << 17) & mask
        u = (s >> 11) / float(1 << 53)
        out[i] = np.float32(u * 2.0 - 1.0)
    return out
