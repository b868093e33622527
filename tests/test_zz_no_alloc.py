"""eb_attention_decode_noalloc: the decode step for callers that cannot
allocate device memory (a plugin whose host framework owns the device pool
and passes it only inputs and outputs, or a serving loop that must not touch
an allocator between steps). It uses the library's own fixed device scratch
instead of a caller workspace.

Checked through the C ABI against eb_attention_decode (the workspace-taking
entry point) on the same inputs, for two calls in a row, at the tolerance
the other parity tests use. This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest

from _util import MAX_ABS, REL_L2

pytestmark = pytest.mark.gpu


def _case(eb, seed, H=16, Hkv=8, hd=128, max_seq=4096):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(max_seq, Hkv, hd, device="cuda", generator=g)
    vc = torch.randn(max_seq, Hkv, hd, device="cuda", generator=g)
    ones = torch.ones(hd, device="cuda")
    cos, sin = eb.rope_tables(max_seq, hd, 1e6)
    desc = eb.make_desc(H, Hkv, hd, max_seq, eps=1e-6)
    layer = eb.make_layer(ones, ones, None, torch.from_numpy(cos).cuda(),
                          torch.from_numpy(sin).cuda())
    return desc, layer, kc, vc, g


def test_noalloc_decode_matches_workspace_decode(eb):
    import torch
    H, Hkv, hd = 16, 8, 128
    desc, layer, kc, vc, g = _case(eb, 7)
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, 1, 4095))
    kc_ref, vc_ref = kc.clone(), vc.clone()
    for pos in (2047, 2048):  # two calls in a row, the second one step later
        q = torch.randn(H, hd, device="cuda", generator=g)
        k = torch.randn(Hkv, hd, device="cuda", generator=g)
        v = torch.randn(Hkv, hd, device="cuda", generator=g)
        o_ref = torch.empty(H, hd, device="cuda")
        o = torch.full((H, hd), float("nan"), device="cuda")
        eb.attention_decode(desc, layer, pos, q, k, v, kc_ref, vc_ref, o_ref, ws)
        eb.attention_decode_noalloc(desc, layer, pos, q, k, v, kc, vc, o)
        torch.cuda.synchronize()
        got, want = o.cpu().numpy().ravel(), o_ref.cpu().numpy().ravel()
        assert np.isfinite(got).all()
        diff = np.abs(got - want).max()
        rel = np.linalg.norm(got - want) / (np.linalg.norm(want) + 1e-12)
        assert diff <= MAX_ABS and rel <= REL_L2, (pos, diff, rel)
        assert torch.equal(kc[pos], kc_ref[pos]) and torch.equal(vc[pos], vc_ref[pos])
    assert eb.device_error() == 0


def test_noalloc_refuses_shapes_beyond_its_scratch(eb):
    import torch
    # 256 query heads x hd 256 over 128K positions needs more split-K
    # partials than the fixed scratch holds: refused on the host, nothing
    # launched.
    desc = eb.make_desc(256, 8, 256, 131072)
    layer = eb.make_layer()
    assert eb.attention_decode_workspace_bytes(desc, 1, 131071) > 8 << 20
    x = torch.zeros(16, device="cuda")
    with pytest.raises(eb.EbError) as e:
        eb.attention_decode_noalloc(desc, layer, 131071, x, x, x, x, x, x)
    assert e.value.status == 4  # EB_ERR_WORKSPACE
