"""Host-side arithmetic of bench.py: the algorithmic FLOP counts the reported
TFLOP/s and roofline fractions divide by (no device needed)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def _brute(hd, H, S, window):
    keys = sum(min(i + 1, window) if window else i + 1 for i in range(S))
    return 4.0 * hd * H * keys  # QK^T and PV, 2 FLOP per MAC


def test_prefill_flops_causal_and_windowed():
    w = bench.make_workload("cfg3")
    assert w.flops() == 2.0 * 128 * 32 * 8192 * 8193 == 5.498229227520e11
    assert w.flops() == _brute(128, 32, 8192, 0)
    w = bench.make_workload("cfg3w")
    assert w.window == 1024 and w.flops() == _brute(128, 32, 8192, 1024)
    for S, W in ((200, 50), (200, 199), (200, 200), (200, 1000), (1, 1)):
        w.S, w.window = S, W
        assert w.flops() == _brute(128, 32, S, W if W < S else 0), (S, W)


def test_prefill_kernel_units_are_the_ranks_share():
    w = bench.make_workload("cfg3w")
    w.Hl = 8  # one rank of four
    assert w.kernel_units() == w.flops() / 4


def test_linear_units():
    w = bench.make_workload("proj3")
    assert w.bound == "tensor" and w.flops() == 2.0 * 8192 * 6144 * 4096
    w = bench.make_workload("projd")
    assert w.bound == "hbm"
    assert w.bytes_total() == 2.0 * 151936 * 1024 + 4.0 * (1024 + 151936)


def test_profile_traffic_is_keyed_to_the_kernel_code(tmp_path, monkeypatch):
    """A traffic[...] line counts only while the kernel code it was captured
    from is unchanged: comment edits keep it, a code edit drops it (None)."""
    csrc = tmp_path / "eyebrowse_b200" / "csrc"
    csrc.mkdir(parents=True)
    prof = tmp_path / "profiles"
    prof.mkdir()
    src = csrc / "k.cu"
    src.write_text("// kernel\n__global__ void k(int* p) { p[0] = 1; }  /* note */\n")
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    monkeypatch.setitem(bench.KERNEL_SOURCES, "toy", ("k.cu",))
    h = bench.source_hash("toy")
    (prof / "toy.md").write_text(f"traffic[toy]: 1234 bytes per launch, source {h}\n")
    assert bench.profile_traffic("toy") == 1234.0
    src.write_text("// the same kernel, re-commented\n__global__ void k(int* p) {\n  p[0] = 1;\n}\n")
    assert bench.source_hash("toy") == h and bench.profile_traffic("toy") == 1234.0
    src.write_text("__global__ void k(int* p) { p[0] = 2; }\n")
    assert bench.source_hash("toy") != h and bench.profile_traffic("toy") is None
    assert bench.rank_traffic("toy", 0.5) is None
