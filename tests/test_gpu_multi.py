"""Multi-GPU parity (tests/mgpu_parity.py) as a pytest case: two ranks under
torchrun on the first two GPUs, NCCL and the fused head gathers (prefill and
decode) checked against each other and the oracle. Skipped on a machine with
fewer than two GPUs."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_gpu_parity():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES="0,1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(port), os.path.join(ROOT, "tests", "mgpu_parity.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    out = p.stdout + p.stderr
    assert p.returncode == 0 and "[mgpu] PASS" in out, out[-4000:]
