"""eyebrowse_b200 -- B200 (sm_100a) attention path for eyebrowse, behind a C ABI.

The product is libeyebrowse_attn.so (include/eyebrowse_attn.h). This module
binds it with ctypes for Python callers (tests, bench.py, the head-sharded
multi-GPU driver in eyebrowse_b200.sharded). Tensors are torch CUDA tensors;
only their device pointers cross the boundary. There is no CPU fallback:
importing works without a GPU, but every call needs the CUDA library and an
sm_100 device, and a non-OK status raises EbError.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeyebrowse_attn.so")

EB_F32, EB_F16, EB_BF16 = 0, 1, 2
STATUS = {0: "EB_OK", 1: "EB_ERR_INVALID_ARGUMENT", 2: "EB_ERR_UNSUPPORTED", 3: "EB_ERR_CUDA",
          4: "EB_ERR_WORKSPACE", 5: "EB_ERR_NO_DEVICE", 6: "EB_ERR_DEVICE_TIMEOUT"}

# Every symbol include/eyebrowse_attn.h declares.
EXPORTS = (
    "eb_status_string", "eb_version", "eb_attn_prefill", "eb_attn_prefill_workspace_bytes",
    "eb_attn_decode", "eb_attn_decode_workspace_bytes", "eb_rope", "eb_kv_write", "eb_rmsnorm",
    "eb_rope_tables", "eb_attention_prefill", "eb_attention_prefill_workspace_bytes",
    "eb_attention_prefill_kv", "eb_attention_prefill_attend",
    "eb_attention_prefill_gather", "eb_attention_prefill_attend_gather",
    "eb_attention_decode", "eb_attention_decode_batched", "eb_attention_decode_workspace_bytes",
    "eb_workspace_init", "eb_head_concat", "eb_get_device_error",
    "eb_attention_decode_noalloc", "eb_head_broadcast", "eb_linear_f16w",
    "eb_linear_f16w_workspace_bytes", "eb_selftest_wait_timeout",
    "eb_attention_decode_batched_gather",
)


class HeadGather(ctypes.Structure):
    """eb_head_gather: where a head-sharded prefill stores its heads (dst is a
    host array of device addresses, one per rank)."""
    _fields_ = [("n_dst", ctypes.c_int32), ("head_offset", ctypes.c_int32),
                ("n_heads_total", ctypes.c_int64), ("dst", ctypes.POINTER(ctypes.c_uint64))]


class EbError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {STATUS.get(status, status)} ({_lib.eb_status_string(status).decode()})")


class AttnDesc(ctypes.Structure):
    """eb_attn_desc (include/eyebrowse_attn.h)."""
    _fields_ = [("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("max_seq", ctypes.c_int32),
                ("dtype_qkv", ctypes.c_int32), ("dtype_cache", ctypes.c_int32),
                ("dtype_out", ctypes.c_int32), ("q_stride", ctypes.c_int32),
                ("kv_stride", ctypes.c_int32), ("o_stride", ctypes.c_int32),
                ("eps", ctypes.c_float), ("scale", ctypes.c_float),
                ("window", ctypes.c_int32)]


class AttnLayer(ctypes.Structure):
    """eb_attn_layer (include/eyebrowse_attn.h)."""
    _fields_ = [("q_norm_w", ctypes.c_void_p), ("k_norm_w", ctypes.c_void_p),
                ("v_norm_w", ctypes.c_void_p), ("rope_cos", ctypes.c_void_p),
                ("rope_sin", ctypes.c_void_p)]


_lib = None
_vp, _i64, _f, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


def lib() -> ctypes.CDLL:
    """Load libeyebrowse_attn.so (built by eyebrowse_b200.build). Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run `python -m eyebrowse_b200.build` "
                           "(there is no fallback path)")
    L = ctypes.CDLL(LIB_PATH)
    L.eb_status_string.restype = ctypes.c_char_p
    L.eb_status_string.argtypes = [ctypes.c_int]
    L.eb_version.restype = ctypes.c_char_p
    L.eb_attn_prefill.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _vp, _sz, _vp]
    L.eb_attn_prefill_workspace_bytes.restype = _sz
    L.eb_attn_prefill_workspace_bytes.argtypes = [_i64, _i64, _i64, _i64]
    L.eb_attn_decode.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f, _vp, _sz, _vp]
    L.eb_attn_decode_workspace_bytes.restype = _sz
    L.eb_attn_decode_workspace_bytes.argtypes = [_i64, _i64, _i64, _i64]
    L.eb_rope.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]
    L.eb_kv_write.argtypes = [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]
    L.eb_rmsnorm.argtypes = [_vp, _vp, _vp, _i64, _i64, _f, _vp]
    L.eb_linear_f16w.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]
    L.eb_linear_f16w_workspace_bytes.restype = _sz
    L.eb_linear_f16w_workspace_bytes.argtypes = [_i64, _i64, _i64]
    L.eb_rope_tables.argtypes = [_vp, _vp, _i64, _i64, _i64, _f]
    dp, lp = ctypes.POINTER(AttnDesc), ctypes.POINTER(AttnLayer)
    L.eb_attention_prefill.argtypes = [dp, lp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.eb_attention_prefill_kv.argtypes = [dp, lp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.eb_attention_prefill_attend.argtypes = [dp, lp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.eb_head_broadcast.argtypes = [_vp, _vp, _i64, _i64, ctypes.c_int32, ctypes.c_int32, _i64,
                                    ctypes.c_int32, _vp]
    gp = ctypes.POINTER(HeadGather)
    L.eb_attention_prefill_gather.argtypes = [dp, lp, _i64, _vp, _vp, _vp, _vp, _vp, gp, _vp, _sz,
                                              _vp]
    L.eb_attention_prefill_attend_gather.argtypes = [dp, lp, _i64, _vp, _vp, _vp, gp, _vp, _sz,
                                                     _vp]
    L.eb_attention_prefill_workspace_bytes.restype = _sz
    L.eb_attention_prefill_workspace_bytes.argtypes = [dp, _i64]
    L.eb_attention_decode.argtypes = [dp, lp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.eb_attention_decode_batched.argtypes = [dp, lp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp,
                                              _i64, _vp, _vp, _sz, _vp]
    L.eb_attention_decode_batched_gather.argtypes = [dp, lp, _i64, _vp, _i64, _vp, _vp, _vp, _vp,
                                                     _vp, _i64, gp, _vp, _vp, _sz, _vp]
    L.eb_attention_decode_workspace_bytes.restype = _sz
    L.eb_attention_decode_workspace_bytes.argtypes = [dp, _i64, _i64]
    L.eb_attention_decode_noalloc.argtypes = [dp, lp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
    L.eb_workspace_init.argtypes = [_vp, _sz, _vp]
    L.eb_head_concat.argtypes = [_vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int32, _vp]
    L.eb_get_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    L.eb_selftest_wait_timeout.argtypes = [ctypes.c_uint32, _vp]
    _lib = L
    return L


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _check(status: int, what: str) -> None:
    if status != 0:
        raise EbError(status, what)


def torch_dtype_code(dt) -> int:
    import torch
    return {torch.float32: EB_F32, torch.float16: EB_F16, torch.bfloat16: EB_BF16}[dt]


# ---------------------------------------------------------------- kernel level
def attn_prefill(q, k, v, o, h, hkv, s, hd, scale, workspace=None, stream=None):
    """eb_attn_prefill: drop-in for eyebrowse-kernels attn_prefill (f32)."""
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attn_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(o), h, hkv, s, hd, scale,
                                 _ptr(workspace), ws_bytes, _stream(stream)), "eb_attn_prefill")


def attn_prefill_workspace_bytes(h, hkv, s, hd) -> int:
    return lib().eb_attn_prefill_workspace_bytes(h, hkv, s, hd)


def attn_decode(q, kcache, vcache, o, h, hkv, pos, hd, max_seq, scale, workspace=None,
                stream=None):
    """eb_attn_decode: drop-in for eyebrowse-kernels attn_decode (f32)."""
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attn_decode(_ptr(q), _ptr(kcache), _ptr(vcache), _ptr(o), h, hkv, pos, hd,
                                max_seq, scale, _ptr(workspace), ws_bytes, _stream(stream)),
           "eb_attn_decode")


def attn_decode_workspace_bytes(h, hkv, pos, hd) -> int:
    return lib().eb_attn_decode_workspace_bytes(h, hkv, pos, hd)


def rope(x, cos, sin, out, seq, n_heads, head_dim, base_pos, stream=None):
    _check(lib().eb_rope(_ptr(x), _ptr(cos), _ptr(sin), _ptr(out), seq, n_heads, head_dim,
                         base_pos, _stream(stream)), "eb_rope")


def kv_write(cache, src, hkv, count, hd, max_seq, dst_start, stream=None):
    _check(lib().eb_kv_write(_ptr(cache), _ptr(src), hkv, count, hd, max_seq, dst_start,
                             _stream(stream)), "eb_kv_write")


def rmsnorm(x, weight, out, rows, dim, eps, stream=None):
    _check(lib().eb_rmsnorm(_ptr(x), _ptr(weight), _ptr(out), rows, dim, eps, _stream(stream)),
           "eb_rmsnorm")


def linear_f16w_workspace_bytes(m, in_f, out_f) -> int:
    return lib().eb_linear_f16w_workspace_bytes(m, in_f, out_f)


def linear_f16w(x, w, y, m, in_f, out_f, workspace=None, stream=None):
    """eb_linear_f16w: y [m, out_f] = x [m, in_f] (f32) @ w[out_f, in_f]^T (f16),
    f32 accumulation (linear_f16w, crates/eyebrowse-kernels/src/matmul.rs:128-149).
    m > 8 needs linear_f16w_workspace_bytes of workspace."""
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_linear_f16w(_ptr(x), _ptr(w), _ptr(y), m, in_f, out_f, _ptr(workspace),
                                ws_bytes, _stream(stream)), "eb_linear_f16w")


def rope_tables(max_seq: int, head_dim: int, theta: float, rope_angles: int | None = None):
    """Rope::build / build_partial tables (host, f64 math) as numpy f32 arrays."""
    import numpy as np
    if rope_angles is None:
        rope_angles = head_dim // 2
    cos = np.empty(max_seq * (head_dim // 2), np.float32)
    sin = np.empty_like(cos)
    _check(lib().eb_rope_tables(cos.ctypes.data, sin.ctypes.data, max_seq, head_dim, rope_angles,
                                theta), "eb_rope_tables")
    return cos, sin


# ---------------------------------------------------------------- fused primitive
def make_desc(n_heads, n_kv_heads, head_dim, max_seq, *, dtype_qkv=EB_F32, dtype_cache=EB_F32,
              dtype_out=EB_F32, eps=1e-6, scale=None, q_stride=0, kv_stride=0, o_stride=0,
              window=0):
    """eb_attn_desc. window > 0 restricts each query row i to key rows
    i - window < j <= i (sliding-window layers); 0 attends the whole causal
    context."""
    if scale is None:
        scale = head_dim ** -0.5
    return AttnDesc(n_heads, n_kv_heads, head_dim, max_seq, dtype_qkv, dtype_cache, dtype_out,
                    q_stride, kv_stride, o_stride, eps, scale, window)


def make_layer(q_norm_w=None, k_norm_w=None, v_norm_w=None, rope_cos=None, rope_sin=None):
    """eb_attn_layer over device tensors. The struct keeps references to the
    tensors, so they stay allocated for as long as the layer object lives."""
    layer = AttnLayer(_ptr(q_norm_w), _ptr(k_norm_w), _ptr(v_norm_w), _ptr(rope_cos),
                      _ptr(rope_sin))
    layer._keepalive = (q_norm_w, k_norm_w, v_norm_w, rope_cos, rope_sin)
    return layer


def attention_prefill_workspace_bytes(desc, seq) -> int:
    return lib().eb_attention_prefill_workspace_bytes(ctypes.byref(desc), seq)


def attention_prefill(desc, layer, seq, q, k, v, kcache, vcache, o, workspace=None, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_prefill(ctypes.byref(desc), ctypes.byref(layer), seq, _ptr(q),
                                      _ptr(k), _ptr(v), _ptr(kcache), _ptr(vcache), _ptr(o),
                                      _ptr(workspace), ws_bytes, _stream(stream)),
           "eb_attention_prefill")


def attention_prefill_kv(desc, layer, seq, k, v, kcache, vcache, workspace=None, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_prefill_kv(ctypes.byref(desc), ctypes.byref(layer), seq, _ptr(k),
                                         _ptr(v), _ptr(kcache), _ptr(vcache), _ptr(workspace),
                                         ws_bytes, _stream(stream)), "eb_attention_prefill_kv")


def attention_prefill_attend(desc, layer, seq, q, kcache, vcache, o, workspace=None,
                             stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_prefill_attend(ctypes.byref(desc), ctypes.byref(layer), seq,
                                             _ptr(q), _ptr(kcache), _ptr(vcache), _ptr(o),
                                             _ptr(workspace), ws_bytes, _stream(stream)),
           "eb_attention_prefill_attend")


def attention_prefill_gather(desc, layer, seq, q, k, v, kcache, vcache, gather: HeadGather,
                             workspace=None, stream=None):
    """eb_attention_prefill with the head gather fused into the attention kernel."""
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_prefill_gather(ctypes.byref(desc), ctypes.byref(layer), seq,
                                             _ptr(q), _ptr(k), _ptr(v), _ptr(kcache),
                                             _ptr(vcache), ctypes.byref(gather), _ptr(workspace),
                                             ws_bytes, _stream(stream)),
           "eb_attention_prefill_gather")


def attention_prefill_attend_gather(desc, layer, seq, q, kcache, vcache, gather: HeadGather,
                                    workspace=None, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_prefill_attend_gather(ctypes.byref(desc), ctypes.byref(layer), seq,
                                                    _ptr(q), _ptr(kcache), _ptr(vcache),
                                                    ctypes.byref(gather), _ptr(workspace),
                                                    ws_bytes, _stream(stream)),
           "eb_attention_prefill_attend_gather")


def head_broadcast(local, multicast_ptr: int, rows, n_heads_total, head_offset, n_heads,
                   head_dim, dtype, stream=None):
    """eb_head_broadcast: this rank's heads of `local` into every rank's buffer
    through the multicast address."""
    _check(lib().eb_head_broadcast(_ptr(local), multicast_ptr, rows, n_heads_total, head_offset,
                                   n_heads, head_dim, dtype, _stream(stream)),
           "eb_head_broadcast")


def attention_decode_workspace_bytes(desc, batch, max_pos) -> int:
    return lib().eb_attention_decode_workspace_bytes(ctypes.byref(desc), batch, max_pos)


def attention_decode(desc, layer, pos, q, k, v, kcache, vcache, o, workspace=None, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_decode(ctypes.byref(desc), ctypes.byref(layer), pos, _ptr(q),
                                     _ptr(k), _ptr(v), _ptr(kcache), _ptr(vcache), _ptr(o),
                                     _ptr(workspace), ws_bytes, _stream(stream)),
           "eb_attention_decode")


def attention_decode_batched(desc, layer, batch, positions, max_pos, q, k, v, kcache, vcache,
                             cache_batch_stride, o, workspace=None, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_decode_batched(ctypes.byref(desc), ctypes.byref(layer), batch,
                                             _ptr(positions), max_pos, _ptr(q), _ptr(k), _ptr(v),
                                             _ptr(kcache), _ptr(vcache), cache_batch_stride,
                                             _ptr(o), _ptr(workspace), ws_bytes, _stream(stream)),
           "eb_attention_decode_batched")


def attention_decode_batched_gather(desc, layer, batch, positions, max_pos, q, k, v, kcache,
                                    vcache, cache_batch_stride, gather: HeadGather,
                                    seq_index=None, workspace=None, stream=None):
    """eb_attention_decode_batched_gather: batched decode whose kernel stores
    each output row into every rank's gathered buffer (row seq_index[b] or b,
    heads gather.head_offset + h) instead of o."""
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().eb_attention_decode_batched_gather(
        ctypes.byref(desc), ctypes.byref(layer), batch, _ptr(positions), max_pos, _ptr(q),
        _ptr(k), _ptr(v), _ptr(kcache), _ptr(vcache), cache_batch_stride, ctypes.byref(gather),
        _ptr(seq_index), _ptr(workspace), ws_bytes, _stream(stream)),
        "eb_attention_decode_batched_gather")


def attention_decode_noalloc(desc, layer, pos, q, k, v, kcache, vcache, o, stream=None):
    """eb_attention_decode_noalloc: the decode step using the library's own
    fixed device scratch instead of a caller workspace (for callers that
    cannot allocate; calls on one device must not overlap)."""
    _check(lib().eb_attention_decode_noalloc(ctypes.byref(desc), ctypes.byref(layer), pos,
                                             _ptr(q), _ptr(k), _ptr(v), _ptr(kcache),
                                             _ptr(vcache), _ptr(o), _stream(stream)),
           "eb_attention_decode_noalloc")


def workspace_init(workspace, stream=None):
    _check(lib().eb_workspace_init(_ptr(workspace), workspace.numel() * workspace.element_size(),
                                   _stream(stream)), "eb_workspace_init")


def head_concat(src, dst, shards, rows, heads_per, head_dim, dtype_code, stream=None):
    _check(lib().eb_head_concat(_ptr(src), _ptr(dst), shards, rows, heads_per, head_dim,
                                dtype_code, _stream(stream)), "eb_head_concat")


def device_error() -> int:
    """Device error word (bounded-wait timeouts) of the current device; clears it."""
    bits = ctypes.c_uint32(0)
    st = lib().eb_get_device_error(ctypes.byref(bits))
    if st not in (0, 6):
        raise EbError(st, "eb_get_device_error")
    return bits.value


DEVICE_ERROR_TMA = 1 << 0       # bits of the device error word (EB_DEVICE_ERROR_*)
DEVICE_ERROR_MMA = 1 << 1
DEVICE_ERROR_SOFTMAX = 1 << 2
DEVICE_ERROR_EPILOGUE = 1 << 3
DEVICE_ERROR_SELFTEST = 1 << 5


def selftest_wait_timeout(timeout_us: int, stream=None):
    """eb_selftest_wait_timeout: a kernel whose bounded wait never completes
    gives up after timeout_us and sets DEVICE_ERROR_SELFTEST in the device
    error word (read and cleared by device_error())."""
    _check(lib().eb_selftest_wait_timeout(timeout_us, _stream(stream)),
           "eb_selftest_wait_timeout")


def alloc_workspace(nbytes: int, device=None):
    """A zeroed, 256-byte-aligned workspace tensor of at least nbytes (torch owns it)."""
    import torch
    n = max(1, (nbytes + 255) // 256 * 256)
    return torch.zeros(n, dtype=torch.uint8, device=device or "cuda")
