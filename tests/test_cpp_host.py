"""The C++ host mirror of the reference interface (eyebrowse_b200/host/
eyebrowse.hpp) and its parity tests (tests/cpp/test_attention_path.cpp,
ported from the reference's own Rust unit tests, CPU side from the C
oracle). The CPU test builds the test program and lists its tests (no
device work); the GPU test runs them all."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(HERE, "cpp", "_build", "test_attention_path")
NAMES = ["attn_prefill_matches_cpu", "attn_decode_matches_cpu", "rope_matches_cpu",
         "rmsnorm_matches_cpu", "kv_write_places_rows", "rope_build_tables",
         "prefill_decode_consistency", "attn_prefill_tensor_core_hd128",
         "attention_decode_long_context_hd128", "sliding_window_prefill_and_decode",
         "linear_f16w_matches_cpu", "linear_forward_decode_and_prefill",
         "attention_forward_with_projections", "invalid_shapes_throw"]


def _build():
    if shutil.which("nvcc") is None and not os.path.exists(BIN):
        pytest.skip("nvcc not available to build the C++ tests")
    if shutil.which("nvcc") is not None:
        subprocess.run(["make", "-s", "-C", os.path.join(HERE, "cpp")], check=True,
                       capture_output=True, text=True)


def test_cpp_host_mirror_builds_and_lists_tests(eb, orc):
    _build()
    r = subprocess.run([BIN, "--list"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == NAMES


@pytest.mark.gpu
def test_cpp_host_mirror_parity(eb, orc):
    _build()
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"0 of {len(NAMES)} tests failed" in r.stdout
