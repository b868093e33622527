"""The failure path of the bounded waits, exercised without a GPU fault.

Every tcgen05 kernel here (prefill, tensor-core decode, projection GEMM)
waits on mbarriers with a limit, after which the wait sets a bit in the
device error word, the kernel returns early and eb_get_device_error reports
EB_ERR_DEVICE_TIMEOUT. eb_selftest_wait_timeout runs that same wait on a
barrier nothing ever completes, with a short limit. The tests check that the
kernel returns after about the limit, that the error word reports the bit
once and is cleared by reading it, that the context stays usable (a decode
call afterwards matches the oracle), and that a failure also resets the
no-workspace decode's split-K tickets.
"""
import time

import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def _decode_case(eb, orc, seed):
    import torch
    H, Hkv, hd, max_seq, pos = 16, 8, 128, 4096, 3000
    kc = randn((max_seq, Hkv, hd), seed)
    vc = randn((max_seq, Hkv, hd), seed + 1)
    q, k, v = randn((H, hd), seed + 2), randn((Hkv, hd), seed + 3), randn((Hkv, hd), seed + 4)
    desc = eb.make_desc(H, Hkv, hd, max_seq)
    layer = eb.make_layer()
    want, _, _ = orc.attention_decode(q, k, v, pos=pos, h=H, hkv=Hkv, hd=hd, max_seq=max_seq,
                                      scale=hd ** -0.5, kcache=kc, vcache=vc)
    return desc, layer, pos, [to_dev(x) for x in (q, k, v, kc, vc)], want, H * hd


def test_bounded_wait_gives_up_and_reports(eb):
    import torch
    assert eb.device_error() == 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eb.selftest_wait_timeout(2000)  # 2 ms
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert 0.0015 <= dt < 0.5, f"kernel returned after {dt * 1e3:.2f} ms"
    bits = eb.device_error()
    assert bits & eb.DEVICE_ERROR_SELFTEST, hex(bits)
    assert eb.device_error() == 0  # reading cleared it


def test_context_usable_after_a_timeout(eb, orc):
    import torch
    eb.selftest_wait_timeout(1000)
    assert eb.device_error() & eb.DEVICE_ERROR_SELFTEST
    desc, layer, pos, (q, k, v, kc, vc), want, n = _decode_case(eb, orc, 90)
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, 1, pos))
    o = torch.empty(n, device="cuda")
    eb.attention_decode(desc, layer, pos, q, k, v, kc, vc, o, ws)
    assert_close(orc, to_np(o), want, what="decode after a reported timeout")
    assert eb.device_error() == 0


def test_noalloc_tickets_reset_after_a_reported_failure(eb, orc):
    """eb_get_device_error, on reporting a failure, zeroes the no-workspace
    decode's tickets (a real failed kernel could have left them set); the
    next call must still be right."""
    import torch
    desc, layer, pos, (q, k, v, kc, vc), want, n = _decode_case(eb, orc, 95)
    o = torch.empty(n, device="cuda")
    eb.attention_decode_noalloc(desc, layer, pos, q, k, v, kc, vc, o)
    assert_close(orc, to_np(o), want, what="no-alloc decode before")
    eb.selftest_wait_timeout(500)
    assert eb.device_error() & eb.DEVICE_ERROR_SELFTEST
    o2 = torch.full((n,), float("nan"), device="cuda")
    eb.attention_decode_noalloc(desc, layer, pos, q, k, v, kc, vc, o2)
    assert_close(orc, to_np(o2), want, what="no-alloc decode after")
    assert np.array_equal(to_np(o), to_np(o2))
    assert eb.device_error() == 0


def test_selftest_rejects_bad_limits(eb):
    for bad in (0, 2_000_000):
        with pytest.raises(eb.EbError) as e:
            eb.selftest_wait_timeout(bad)
        assert e.value.status == 1
