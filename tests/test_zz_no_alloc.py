"""eb_attention_decode_noalloc: the decode step for callers that cannot
allocate device memory -- a plugin whose host framework owns the whole device
pool and hands it only its inputs and outputs, or a serving loop that must not
call an allocator between steps. It uses a fixed scratch array inside the
library instead of a caller workspace.

Every case runs two calls in a row through the C ABI (position pos, then
pos + 1, the second on the cache the first wrote) and checks each against
the existing entry point, eb_attention_decode with a caller workspace, and
against the oracle (the reference's CPU decode, restated), at the tolerance
the other parity tests use. The shapes cover the f32 vector kernel, the f16
tensor-core kernel and a sliding-window hd256 layer; one test alternates
shapes with different head counts on the shared array, whose split-K
tickets every call must leave at zero for the next.

This file is named to be collected last (pytest orders test files by name):
a run that stops at the first failure has then already run every other test.
Each test builds its own inputs, so the file passes alone as well.
"""
import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu

# name: (H, Hkv, hd, max_seq, pos, cache dtype, window, scale, qk-norm weights, v-norm,
#        rope theta, rope_angles)
CASES = {
    "f32_hd128": (16, 8, 128, 4096, 2047, "f32", 0, None, "ones", False, 1e6, None),
    "f16_tc_hd128": (32, 8, 128, 8192, 6000, "f16", 0, None, None, False, 5e5, None),
    "f32_hd256_window": (8, 4, 256, 4352, 3000, "f32", 1024, 1.0, "n1", True, 1e6, 32),
}


class _Case:
    def __init__(self, eb, orc, name, seed):
        import torch
        (H, Hkv, hd, max_seq, pos, cdt, window, scale, qkw, vnorm, theta,
         angles) = CASES[name]
        self.name, self.H, self.Hkv, self.hd, self.max_seq, self.pos = name, H, Hkv, hd, max_seq, pos
        self.f16 = cdt == "f16"
        self.tdt = torch.float16 if self.f16 else torch.float32
        code = eb.EB_F16 if self.f16 else eb.EB_F32
        self.cround = orc.F16 if self.f16 else orc.F32
        self.scale = hd ** -0.5 if scale is None else scale
        rnd = (lambda x: orc.round_f16(x)) if self.f16 else (lambda x: x)
        self.rnd = rnd
        # rows past pos are never read (pos and pos + 1 are written by the calls)
        self.kc = rnd(randn((max_seq, Hkv, hd), seed)).reshape(max_seq, Hkv, hd)
        self.vc = rnd(randn((max_seq, Hkv, hd), seed + 1)).reshape(max_seq, Hkv, hd)
        self.kc[pos:] = np.nan
        self.vc[pos:] = np.nan
        if qkw == "ones":
            self.qw = self.kw = np.ones(hd, np.float32)
        elif qkw == "n1":
            self.qw = (1 + 0.1 * randn((hd,), seed + 2)).astype(np.float32)
            self.kw = (1 + 0.1 * randn((hd,), seed + 3)).astype(np.float32)
        else:
            self.qw = self.kw = None
        self.vw = np.ones(hd, np.float32) if vnorm else None
        self.cos, self.sin = eb.rope_tables(max_seq, hd, theta, angles)
        self.desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=code, dtype_cache=code,
                                 dtype_out=eb.EB_F32, eps=1e-6, scale=self.scale, window=window)
        dev = lambda w: None if w is None else to_dev(w)
        self.layer = eb.make_layer(dev(self.qw), dev(self.kw), dev(self.vw), to_dev(self.cos),
                                   to_dev(self.sin))
        self.window = window
        # device caches: one for the no-allocation path, one for the workspace path
        self.kcd, self.vcd = to_dev(self.kc, self.tdt), to_dev(self.vc, self.tdt)
        self.kcw, self.vcw = self.kcd.clone(), self.vcd.clone()
        nb = eb.attention_decode_workspace_bytes(self.desc, 1, max_seq - 1)
        self.ws = eb.alloc_workspace(nb) if nb else None
        self.seed = seed

    def step(self, eb, orc, pos, i):
        """One call of each entry point at pos; both checked against the oracle."""
        import torch
        q = self.rnd(randn((self.H, self.hd), self.seed + 10 + i))
        k = self.rnd(randn((self.Hkv, self.hd), self.seed + 20 + i))
        v = self.rnd(randn((self.Hkv, self.hd), self.seed + 30 + i))
        qd, kd, vd = to_dev(q, self.tdt), to_dev(k, self.tdt), to_dev(v, self.tdt)
        o = torch.full((self.H * self.hd,), float("nan"), device="cuda")
        o_ws = torch.full_like(o, float("nan"))
        eb.attention_decode_noalloc(self.desc, self.layer, pos, qd, kd, vd, self.kcd, self.vcd, o)
        eb.attention_decode(self.desc, self.layer, pos, qd, kd, vd, self.kcw, self.vcw, o_ws,
                            self.ws)
        want, kc, vc = orc.attention_decode(
            q, k, v, pos=pos, h=self.H, hkv=self.Hkv, hd=self.hd, max_seq=self.max_seq,
            scale=self.scale, kcache=self.kc.ravel(), vcache=self.vc.ravel(), eps=1e-6,
            q_norm_w=self.qw, k_norm_w=self.kw, v_norm_w=self.vw, cos=self.cos, sin=self.sin,
            cache_round=self.cround, window=self.window)
        self.kc = kc.reshape(self.kc.shape)
        self.vc = vc.reshape(self.vc.shape)
        got, got_ws = to_np(o), to_np(o_ws)
        what = f"{self.name} pos={pos}"
        assert_close(orc, got, want, what=what + " no-alloc vs oracle")
        assert_close(orc, got, got_ws, what=what + " no-alloc vs workspace entry point")
        # the written cache row equals the workspace path's and the oracle's
        assert torch.equal(self.kcd[pos], self.kcw[pos]) and torch.equal(self.vcd[pos], self.vcw[pos])
        assert_close(orc, to_np(self.kcd[pos]), self.kc[pos], max_abs=2e-3, rel_l2=1e-3,
                     what=what + " k row")


@pytest.mark.parametrize("name", list(CASES))
def test_noalloc_decode_two_calls(eb, orc, name):
    c = _Case(eb, orc, name, 7000 + 100 * list(CASES).index(name))
    for i, pos in enumerate((c.pos, c.pos + 1)):
        c.step(eb, orc, pos, i)
    assert eb.device_error() == 0


def test_noalloc_shared_scratch_across_shapes(eb, orc):
    """Calls with 16, then 32, then 16 query heads share the one array: each
    must find its tickets at zero where the call before left them."""
    a = _Case(eb, orc, "f32_hd128", 7500)
    b = _Case(eb, orc, "f16_tc_hd128", 7600)
    a.step(eb, orc, a.pos, 0)
    b.step(eb, orc, b.pos, 0)
    a.step(eb, orc, a.pos + 1, 1)
    b.step(eb, orc, b.pos + 1, 1)
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
