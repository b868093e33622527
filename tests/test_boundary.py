"""CPU-side checks of the C-ABI boundary: the library loads, exports every
symbol the header declares, validates arguments on the host before touching
a device, and its host-side RoPE table builder matches the oracle bit for bit."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"^EB_API[^;(]*?\b(eb_\w+)\(", txt, flags=re.M))
    return names


def test_header_declares_the_abi():
    names = _declared()
    assert {"eb_attn_prefill", "eb_attn_decode", "eb_rope", "eb_kv_write", "eb_rmsnorm",
            "eb_attention_prefill", "eb_attention_decode", "eb_attention_decode_batched"} <= names


def test_library_exports_every_declared_symbol(eb):
    L = eb.lib()
    for n in sorted(_declared()):
        assert hasattr(L, n), n
    assert set(eb.EXPORTS) == _declared()


def test_device_error_bits_match_the_header(eb):
    txt = open(os.path.join(ROOT, "include", "eyebrowse_attn.h")).read()
    bits = {m[0]: int(m[1]) for m in re.findall(r"#define EB_DEVICE_ERROR_(\w+) \(1u << (\d+)\)", txt)}
    assert set(bits) == {"TMA", "MMA", "SOFTMAX", "EPILOGUE", "SELFTEST"}
    for name, shift in bits.items():
        assert getattr(eb, f"DEVICE_ERROR_{name}") == 1 << shift, name
    assert len(set(bits.values())) == len(bits)


def test_rope_tables_match_oracle_bitwise(eb, orc):
    for (ms, hd, th, ra) in [(64, 128, 1e6, None), (40, 256, 1e6, 32), (8, 4, 1e4, None),
                             (33, 64, 5e5, 3)]:
        c1, s1 = eb.rope_tables(ms, hd, th, ra)
        c2, s2 = orc.rope_tables(ms, hd, th, rope_angles=ra)
        assert np.array_equal(c1, c2) and np.array_equal(s1, s2)


def test_host_validation_precedes_device_work(eb):
    L = eb.lib()
    # h % hkv != 0, odd head_dim, pos >= max_seq, kv_write past the cache: rejected on the host
    assert L.eb_attn_prefill(None, None, None, None, 3, 2, 4, 8, 0.3, None, 0, None) == 1
    assert L.eb_attn_prefill(None, None, None, None, 2, 2, 4, 7, 0.3, None, 0, None) == 1
    assert L.eb_attn_decode(None, None, None, None, 4, 2, 16, 8, 16, 0.3, None, 0, None) == 1
    assert L.eb_kv_write(None, None, 2, 4, 8, 8, 6, None) == 1
    assert L.eb_rope(None, None, None, None, 1, 1, 7, 0, None) == 1
    # empty work is a no-op and succeeds without a device
    assert L.eb_attn_prefill(None, None, None, None, 2, 1, 0, 8, 0.3, None, 0, None) == 0
    d = eb.make_desc(16, 8, 128, 4096)
    lay = eb.make_layer()
    assert L.eb_attention_prefill(ctypes.byref(d), ctypes.byref(lay), 0, None, None, None, None,
                                  None, None, None, 0, None) == 0
    bad = eb.make_desc(16, 6, 128, 4096)  # 16 % 6 != 0
    assert L.eb_attention_prefill(ctypes.byref(bad), ctypes.byref(lay), 4, 1, 1, 1, 1, 1, 1, None,
                                  0, None) == 1
    assert L.eb_attention_decode(ctypes.byref(d), ctypes.byref(lay), 4096, 1, 1, 1, 1, 1, 1, None,
                                 0, None) == 1
    neg = eb.make_desc(16, 8, 128, 4096, window=-1)  # a window is a row count
    assert L.eb_attention_prefill(ctypes.byref(neg), ctypes.byref(lay), 4, 1, 1, 1, 1, 1, 1, None,
                                  0, None) == 1
    # the no-workspace decode checks the descriptor as eb_attention_decode
    # does: an unknown dtype code (here 7) is refused before any device work
    for field in ("dtype_qkv", "dtype_cache", "dtype_out"):
        bad_dt = eb.make_desc(16, 8, 128, 4096)
        setattr(bad_dt, field, 7)
        assert L.eb_attention_decode_noalloc(ctypes.byref(bad_dt), ctypes.byref(lay), 5, 16, 16,
                                             16, 16, 16, 16, None) == 1, field
        assert L.eb_attention_decode(ctypes.byref(bad_dt), ctypes.byref(lay), 5, 16, 16, 16, 16,
                                     16, 16, None, 0, None) == 1, field
    neg_stride = eb.make_desc(16, 8, 128, 4096, q_stride=-4)
    assert L.eb_attention_decode_noalloc(ctypes.byref(neg_stride), ctypes.byref(lay), 5, 16, 16,
                                         16, 16, 16, 16, None) == 1
    assert L.eb_attention_decode_noalloc(ctypes.byref(d), ctypes.byref(lay), 4096, 16, 16, 16, 16,
                                         16, 16, None) == 1  # pos >= max_seq
    # linear_f16w: shapes are checked before anything else; m = 0 is a no-op
    assert L.eb_linear_f16w(16, 16, 16, -1, 64, 64, None, 0, None) == 1
    assert L.eb_linear_f16w(16, 16, 16, 4, 0, 64, None, 0, None) == 1
    assert L.eb_linear_f16w(16, 16, 16, 0, 64, 64, None, 0, None) == 0


def test_no_device_is_reported_not_faked(eb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    L = eb.lib()
    # valid arguments, no GPU: the call must refuse, never compute elsewhere
    assert L.eb_rope(1, 1, 1, 1, 1, 1, 8, 0, None) == 5
    assert L.eb_linear_f16w(16, 16, 16, 4, 64, 64, None, 0, None) == 5


def test_linear_workspace_sizes(eb):
    # m <= 8 streams the weights (no workspace); m > 8 splits x into two f16
    # planes, each rounded up to 256 bytes; other shapes take the scalar kernel
    assert eb.linear_f16w_workspace_bytes(8, 1024, 4096) == 0
    assert eb.linear_f16w_workspace_bytes(9, 1024, 4096) == 2 * 9 * 1024 * 2
    assert eb.linear_f16w_workspace_bytes(300, 200, 260) == 2 * ((300 * 200 * 2 + 255) // 256 * 256)
    assert eb.linear_f16w_workspace_bytes(100, 33, 64) == 0   # k not a multiple of 8
    assert eb.linear_f16w_workspace_bytes(100, 64, 62) == 0   # out not a multiple of 4
    assert eb.linear_f16w_workspace_bytes(0, 64, 64) == 0


def test_window_caps_decode_workspace(eb):
    """A sliding-window layer's decode never attends more than `window` rows:
    its workspace is the full-context workspace of a window-row context."""
    full = eb.make_desc(16, 8, 128, 1 << 17)
    win = eb.make_desc(16, 8, 128, 1 << 17, window=1024)
    assert (eb.attention_decode_workspace_bytes(win, 1, (1 << 17) - 1)
            == eb.attention_decode_workspace_bytes(full, 1, 1023))
    assert (eb.attention_decode_workspace_bytes(win, 1, 500)
            == eb.attention_decode_workspace_bytes(full, 1, 500))


def test_workspace_sizes(eb):
    d = eb.make_desc(16, 8, 128, 4096)
    a = eb.attention_decode_workspace_bytes(d, 1, 2047)
    b = eb.attention_decode_workspace_bytes(d, 64, 32767)
    assert a > 0 and b > a and a % 256 == 0
    assert eb.attention_decode_workspace_bytes(d, 1, 10) == 0  # short context: one CTA per head
    # one workspace sized at max_pos serves every shorter context: the size
    # never shrinks as max_pos grows (the split-K chunk count itself can)
    for desc, batch in ((d, 1), (eb.make_desc(32, 8, 64, 1 << 17, dtype_cache=eb.EB_F16), 2),
                        (eb.make_desc(8, 1, 256, 1 << 17), 1)):
        sizes = [eb.attention_decode_workspace_bytes(desc, batch, p) for p in range(0, 20000, 7)]
        assert all(x <= y for x, y in zip(sizes, sizes[1:]))
    # f16 hi/lo planes of k and v, then of the prepared q rows
    assert eb.attn_prefill_workspace_bytes(16, 8, 128, 128) == (4 * 128 * 8 + 2 * 128 * 16) * 128 * 2
    assert eb.attn_prefill_workspace_bytes(2, 1, 5, 8) == 0  # SIMT path
    f16 = eb.make_desc(32, 8, 128, 8192, dtype_qkv=eb.EB_F16, dtype_cache=eb.EB_F16)
    # f16 q and cache: q is normalised and rotated inside the attention
    # kernel, the cache is read directly: nothing is staged
    assert eb.attention_prefill_workspace_bytes(f16, 8192) == 0
    mixed = eb.make_desc(32, 8, 128, 8192, dtype_qkv=eb.EB_F32, dtype_cache=eb.EB_F16)
    # f32 q for an f16 cache: the row pass stages the f16 q rows
    assert eb.attention_prefill_workspace_bytes(mixed, 8192) == 8192 * 32 * 128 * 2
    odd = eb.make_desc(4, 2, 96, 64, dtype_qkv=eb.EB_F16, dtype_cache=eb.EB_F16)
    assert eb.attention_prefill_workspace_bytes(odd, 64) == 0  # SIMT path
