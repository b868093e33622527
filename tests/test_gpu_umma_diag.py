"""Tensor-core operand layouts, checked one at a time on a 128x128xK f16
product (tests/diag/umma_diag.cu): K-major A and B loaded by TMA, K-major A
written by threads with the attention kernel's swizzle formula, an MN-major
B, and A read from tensor memory. Each result must equal an f32 matmul of
the same f16 inputs to f32 accumulation accuracy."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("K", [64, 128])
def test_umma_operand_layouts(K):
    import torch
    lib = ctypes.CDLL(os.path.join(HERE, "diag", "libumma_diag.so"))
    vp = ctypes.c_void_p
    lib.diag_umma.argtypes = [vp] * 7 + [ctypes.c_int, vp]
    g = torch.Generator().manual_seed(K)
    A = torch.randn(128, K, generator=g).half()
    B = torch.randn(128, K, generator=g).half()
    Bt = B.t().contiguous()  # [K, N]
    Ad, Bd, Btd_ = A.cuda(), B.cuda(), Bt.cuda()
    D = [torch.full((128, 128), float("nan"), device="cuda") for _ in range(4)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.diag_umma(Ad.data_ptr(), Bd.data_ptr(), Btd_.data_ptr(), *[d.data_ptr() for d in D],
                       K, status.data_ptr())
    assert rc == 0, rc
    assert int(status.item()) == 0, f"bounded wait gave up: {int(status.item())}"
    want = (A.float() @ B.float().t()).numpy()
    errs = [float(np.abs(d.cpu().numpy() - want).max()) for d in D]
    names = ["TMA K-major A,B", "hand-swizzled A", "MN-major B", "A from TMEM"]
    msg = ", ".join(f"{n}: {e:.2e}" for n, e in zip(names, errs))
    assert all(e < 1e-2 for e in errs), msg
