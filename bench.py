"""Benchmark of the eyebrowse B200 attention path (BASELINE.json metric:
"prefill attn TFLOP/s & decode KV GB/s at 1/2/4/8 B200 vs roofline").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W]
                    [--impl ours|reference] [--no-decode] [--no-cpu] [--gather fused|nccl]

Workloads: cfg3 (default), cfg1, cfg2, cfg4, cfg4d (config 4's decode step),
cfg5, cfg3w (config 3 with a sliding window), cfg3r4 / cfg3r8 (one rank's
head share of config 3 at 4 / 8 GPUs, on one GPU without the gather), proj3,
projd (projections).

The headline line is config 3 (causal GQA prefill, S8192 H32 Hkv8 hd128, f16
q/k/v/cache/out, f32 accumulate, RoPE theta 5e5), heads sharded over N ranks
(strong scaling): each rank runs the fused prefill on its H/N query heads and
Hkv/N KV heads, and the attention kernel stores its output tiles into every
rank's gathered [S, H, hd] buffer over NVLink (--gather nccl: an NCCL
all-gather and a concat kernel instead). A "step" is that whole sequence.
`value` is total algorithmic FLOP / max-over-ranks step time.
The "decode" object is config 5 (64 sequences, contexts U[512, 32768], f16
caches), sharded by KV head, in KV GB/s.

--impl reference times the reference's CPU attention (the oracle port under
oracle/, the reference being Rust + wgpu, which this image cannot build or
run) on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from eyebrowse_b200.sharded import (GatheredOutput, decode_shard, gather_heads,  # noqa: E402
                                    head_shard)

METRIC = "prefill attn TFLOP/s & decode KV GB/s at 1/2/4/8 B200 vs roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# Untimed seconds before each timed loop: long enough for the SM clock to
# settle under the 1000 W power cap, so the timed region sees steady clocks.
WARM_S = 1.5
# Head-concat exchange for N > 1: "fused" (the attention kernel stores into
# every rank's output over NVLink) or "nccl" (all-gather + eb_head_concat).
GATHER = "fused"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# The CUDA sources each profiled kernel is built from. A profile's traffic
# line records their hash; once a source changes, the recorded figure no
# longer describes the shipping kernel and the bench reports null instead.
KERNEL_SOURCES = {
    "prefill_cfg3": ("eb_prefill.cu", "eb_common.cuh", "eb_tc.cuh"),
    "prefill_cfg4": ("eb_prefill.cu", "eb_common.cuh", "eb_tc.cuh"),
    "prep_cfg3": ("eb_small.cu", "eb_rowops.cuh", "eb_common.cuh"),
    "decode_cfg5": ("eb_decode_tc.cu", "eb_common.cuh", "eb_tc.cuh"),
    "decode_cfg2": ("eb_decode_cl.cu", "eb_decode_out.cuh", "eb_common.cuh", "eb_rowops.cuh"),
    "linear_proj3": ("eb_linear.cu", "eb_common.cuh", "eb_tc.cuh"),
}


def source_hash(key: str):
    """sha256 (first 16 hex digits) of the kernel sources behind `key`, with
    comments and white space removed: a capture stays valid across comment
    edits and goes stale with any change to the code."""
    import hashlib
    import re
    names = KERNEL_SOURCES.get(key)
    if not names:
        return None
    h = hashlib.sha256()
    for n in names:
        with open(os.path.join(ROOT, "eyebrowse_b200", "csrc", n)) as f:
            src = f.read()
        src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)  # block comments
        src = re.sub(r"//[^\n]*", " ", src)                # line comments
        h.update("".join(src.split()).encode())
    return h.hexdigest()[:16]


def rank_traffic(key: str, share: float):
    """profile_traffic scaled to one rank's launch: the captures are of the
    one-GPU workload, and a rank of a sharded run processes `share` of its
    units (heads, or sequences x heads) in a launch of the same kernel."""
    t = profile_traffic(key)
    return None if t is None else t * share


def profile_traffic(key: str):
    """Per-launch DRAM traffic recorded from an ncu capture in profiles/*.md
    (a line `traffic[<key>]: <bytes per launch> ... source <hash>`), or None
    when there is none or it was captured from other kernel sources."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    want = source_hash(key)
    for fn in sorted(os.listdir(d)):
        if not fn.endswith(".md"):
            continue
        for line in open(os.path.join(d, fn)):
            if line.startswith(f"traffic[{key}]:"):
                words = line.split(":", 1)[1].split()
                if want is None or "source" not in words or \
                        words[words.index("source") + 1].strip("().,") != want:
                    return None
                try:
                    return float(words[0])
                except ValueError:
                    return None
    return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """This GPU's SM clock and clock-event reasons, sampled every few ms while a
    timed region runs: NVML polled from a thread (nvidia_ml_py), else
    `nvidia-smi -lms` as a fallback. Only samples inside the marked region are
    summarised."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, uuid: str | None, period_ms: int = 5):
        self.uuid = uuid
        self.samples = []  # (t, sm, max, reasons:set, watts)
        self.proc = None
        self.period_ms = period_ms
        self.t_lo = self.t_hi = None
        self._stop = threading.Event()
        self.source = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        want = (self.uuid or "").lower().replace("gpu-", "")
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUUID(h)
            u = (u.decode() if isinstance(u, bytes) else u).lower().replace("gpu-", "")
            if want and want in u:
                return pynvml, h
        if not want and pynvml.nvmlDeviceGetCount() == 1:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(0)
        raise RuntimeError("device not found in NVML")

    def start(self):
        try:
            nv, h = self._nvml_handle()
        except Exception:
            nv = None
        if nv is not None:
            self.source = "nvml"
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def poll():
                while not self._stop.is_set():
                    try:
                        sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        w = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    except Exception:
                        break
                    self.samples.append((time.time(), sm, mx, {n for n, b in bits.items() if rs & b}, w))
                    time.sleep(self.period_ms / 1000.0)
            threading.Thread(target=poll, daemon=True).start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "25"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.source = "nvidia-smi"
        threading.Thread(target=self._read, daemon=True).start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            if self.uuid and self.uuid not in parts[0]:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
                w = float(parts[3])
            except ValueError:
                continue
            reasons = {n for n, v in zip(self.REASONS, parts[5:9]) if v.lower().startswith("active")}
            self.samples.append((time.time(), sm, mx, reasons, w))

    def mark(self, lo, hi):
        self.t_lo, self.t_hi = lo, hi

    def stop(self):
        self._stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        s = self.samples
        if self.t_lo is not None:
            s = [x for x in s if self.t_lo <= x[0] <= self.t_hi]
        if not s:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": self.source}
        reasons = sorted(set().union(*[x[3] for x in s]))
        return {"sm_mhz": statistics.median(x[1] for x in s), "sm_min_mhz": min(x[1] for x in s),
                "sm_max_mhz": max(x[2] for x in s), "reasons": reasons, "samples": len(s),
                "power_w_median": round(statistics.median(x[4] for x in s), 1),
                "source": self.source}


# ---------------------------------------------------------------- distributed
def init_dist(n_gpus: int):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if world != n_gpus and rank == 0:
        print(f"[bench] note: --gpus {n_gpus} but WORLD_SIZE {world}", file=sys.stderr)
    return rank, world, local


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------- workloads
class PrefillWork:
    """Head-sharded fused prefill (eb_attention_prefill) + all-gather + concat."""

    def __init__(self, name, S, H, Hkv, hd, theta, dt, in_scale=1.0, scale=None, qk_norm=False,
                 v_norm=False, rope_angles=None, seed=0, window=0):
        self.name, self.S, self.H, self.Hkv, self.hd = name, S, H, Hkv, hd
        self.window = window
        self.theta, self.dt, self.in_scale, self.seed = theta, dt, in_scale, seed
        self.scale = scale if scale is not None else hd ** -0.5
        self.qk_norm, self.v_norm, self.rope_angles = qk_norm, v_norm, rope_angles
        self.graph_reps = 20 if S <= 1024 else 0  # launch-bound sizes replay a CUDA graph

    def flops(self) -> float:
        # 4 FLOP per (query row, visible key, dim): QK^T and PV, 2 per MAC
        if self.window and self.window < self.S:
            W, S = self.window, self.S
            keys = W * (W + 1) / 2 + (S - W) * W  # rows i < W see i + 1 keys, later rows W
            return 4.0 * self.hd * self.H * keys
        return 2.0 * self.hd * self.H * self.S * (self.S + 1)

    def describe(self, world):
        return {"workload": self.name, "seq_len": self.S, "n_heads": self.H,
                "n_kv_heads": self.Hkv, "head_dim": self.hd, "rope_theta": self.theta,
                "scale": round(self.scale, 6), "qk_norm": self.qk_norm, "v_norm": self.v_norm,
                "rope_angles": self.rope_angles or self.hd // 2, "batch": 1,
                "window": self.window or None,
                "parallelism": f"heads/{world}" if world > 1 else "1 GPU",
                "head_concat": self._concat_desc(world)}

    def _concat_desc(self, world):
        if world == 1:
            return None
        if GATHER != "fused":
            return "NCCL all-gather + eb_head_concat"
        g = getattr(self, "gout", None)
        if g is not None and g.mode == "multicast":
            return ("own-buffer write + eb_head_broadcast through the NVLink multicast "
                    "address (multimem)")
        return "fused: the attention kernel TMA-stores each output tile into every rank's buffer"

    def setup(self, rank, world):
        import torch

        import eyebrowse_b200 as eb
        self.eb = eb
        sh = head_shard(self.H, self.Hkv, world, rank)
        self.world = world
        self.Hl, self.Hkvl = sh.n_heads, sh.n_kv_heads
        tdt = {eb.EB_F32: torch.float32, eb.EB_F16: torch.float16, eb.EB_BF16: torch.bfloat16}[self.dt]
        self.tdt = tdt
        g = torch.Generator(device="cuda").manual_seed(self.seed * 1000 + rank)
        S, hd = self.S, self.hd
        mk = lambda *shape: (torch.randn(*shape, device="cuda", generator=g) * self.in_scale).to(tdt)
        self.q = mk(S, self.Hl, hd)
        self.k = mk(S, self.Hkvl, hd)
        self.v = mk(S, self.Hkvl, hd)
        self.kc = torch.empty(S, self.Hkvl, hd, device="cuda", dtype=tdt)
        self.vc = torch.empty_like(self.kc)
        self.o = torch.empty(S, self.Hl, hd, device="cuda", dtype=tdt)
        cos, sin = eb.rope_tables(S, hd, self.theta, self.rope_angles)
        self.cos = torch.from_numpy(cos).cuda()
        self.sin = torch.from_numpy(sin).cuda()
        qw = kw = vw = None
        if self.qk_norm:
            qw = (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).float()
            kw = (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).float()
        if self.v_norm:
            vw = torch.ones(hd, device="cuda")
        self._keep = (qw, kw, vw)
        self.desc = eb.make_desc(self.Hl, self.Hkvl, hd, S, dtype_qkv=self.dt,
                                 dtype_cache=self.dt, dtype_out=self.dt, scale=self.scale,
                                 window=self.window)
        self.layer = eb.make_layer(qw, kw, vw, self.cos, self.sin)
        nb = eb.attention_prefill_workspace_bytes(self.desc, S)
        self.ws = eb.alloc_workspace(nb) if nb else None
        self.gout = None
        if world > 1 and GATHER == "fused":
            # the attention kernel stores every rank's heads into every rank's
            # gathered output over NVLink (double-buffered: one device barrier
            # per step)
            self.gout = GatheredOutput(S, self.H, hd, tdt, sh)
            self.full = self.gout.bufs[0]
            # K/V prep, q prep, attention, barrier (+ the multicast broadcast)
            self.launches_per_step = 4 + (1 if self.gout.mode == "multicast" else 0)
        elif world > 1:
            self.gath = torch.empty(world, S, self.Hl, hd, device="cuda", dtype=tdt)
            self.full = torch.empty(S, self.H, hd, device="cuda", dtype=tdt)
            self.launches_per_step = 4  # K/V prep, q prep, attention, head concat
        else:
            self.full = self.o
            self.launches_per_step = 3  # K/V prep, q prep, attention
        if self.q_in_kernel():
            self.launches_per_step -= 1  # q normalised and rotated inside the attention kernel
        self.bytes_in = sum(t.numel() * t.element_size() for t in (self.q, self.k, self.v))

    def q_in_kernel(self):
        """q already in the cache's 16-bit type: the attention kernel transforms
        its query tiles itself (no q row-prep launch)."""
        return self.dt != 0

    def step(self):
        eb = self.eb
        if self.gout is not None:
            eb.attention_prefill_gather(self.desc, self.layer, self.S, self.q, self.k, self.v,
                                        self.kc, self.vc, self.gout.next(), self.ws)
            self.gout.finish()
            self.full = self.gout.full
            return
        eb.attention_prefill(self.desc, self.layer, self.S, self.q, self.k, self.v, self.kc,
                             self.vc, self.o, self.ws)
        self._gather()

    def _gather(self):
        if self.world > 1:
            gather_heads(self.o, self.gath, self.full, self.world, self.S, self.Hl, self.hd,
                         self.dt)

    def kernel_only(self):
        """The dominant kernel alone: the tensor-core attention (K/V already in the cache),
        with its q row-prep launch; with the fused gather, its NVLink stores included.
        Back-to-back calls store the same values into disjoint head columns, so
        no barrier is needed between them."""
        if self.gout is not None:
            self.eb.attention_prefill_attend_gather(self.desc, self.layer, self.S, self.q,
                                                    self.kc, self.vc, self.gout.gathers[0],
                                                    self.ws)
            return
        self.eb.attention_prefill_attend(self.desc, self.layer, self.S, self.q, self.kc, self.vc,
                                         self.o, self.ws)

    def kernel_units(self):
        return self.flops() * self.Hl / self.H  # this rank's FLOP per launch

    # e2e through the public API with host buffers
    def setup_e2e(self):
        """q, k and v packed in one pinned buffer (one upload per step); the
        workload's q/k/v become views of its device copy, which the public
        API reads: a small prompt's step is otherwise mostly three copies'
        set-up."""
        import torch
        srcs = (self.q, self.k, self.v)
        self.h_in = torch.cat([t.reshape(-1) for t in srcs]).cpu().pin_memory()
        self.d_in = self.h_in.cuda()
        self.q, self.k, self.v = self.qkv_views(self.d_in)
        self.hout = torch.empty(self.full.shape, dtype=self.full.dtype).pin_memory()

    def qkv_views(self, buf):
        out, off = [], 0
        for shape in (self.q.shape, self.k.shape, self.v.shape):
            n = math.prod(shape)
            out.append(buf[off:off + n].view(shape))
            off += n
        return out

    def e2e_pipelined(self, steps, unit, total_units):
        """One GPU: the e2e loop pipelined over two slots (time_e2e_pipelined),
        each with its own packed q/k/v buffer and output."""
        import torch
        self.setup_e2e()
        d_in = [self.d_in, torch.empty_like(self.d_in)]
        qkv = [self.qkv_views(d) for d in d_in]
        outs = [self.o, torch.empty_like(self.o)]
        slots = [([d_in[0]], outs[0], self.hout),
                 ([d_in[1]], outs[1], torch.empty_like(self.hout).pin_memory())]
        api = self.eb

        def run(a):
            q, k, v = qkv[a]
            api.attention_prefill(self.desc, self.layer, self.S, q, k, v, self.kc, self.vc,
                                  outs[a], self.ws)
        ems = time_e2e_pipelined(slots, [self.h_in], run, steps, 2)
        return {"value": total_units / (ems / steps * 1e-3) / 1e12, "unit": unit,
                "h2d_bytes_per_step": int(self.h_in.numel() * self.h_in.element_size()),
                "d2h_bytes_per_step": int(self.hout.numel() * self.hout.element_size()),
                "note": "pinned host q/k/v (one packed upload) in, o out every step through "
                        "eb_attention_prefill; steps pipelined over two slots (upload, compute, "
                        "download on separate streams)"}

    def step_e2e(self, rank):
        self.d_in.copy_(self.h_in, non_blocking=True)
        self.step()
        if rank == 0:
            self.hout.copy_(self.full, non_blocking=True)
        return self.bytes_in, (self.hout.numel() * self.hout.element_size() if rank == 0 else 0)


class BatchedDecodeWork:
    """Config 5: batched decode. On N GPUs each rank owns a KV-head group of a
    context-balanced bucket of the sequences (eyebrowse_b200.sharded.
    decode_shard: the head split first, the sequences over the rest) and its
    kernel stores the output rows into every rank's gathered [B, H, hd]
    buffer over NVLink (--gather nccl: head split only, NCCL all-gather +
    eb_head_concat)."""

    def __init__(self, name="cfg5", B=64, H=32, Hkv=8, hd=128, max_seq=32768, ctx_lo=512,
                 ctx_hi=32768, theta=5e5, dt=1, seed=5):
        self.name, self.B, self.H, self.Hkv, self.hd, self.max_seq = name, B, H, Hkv, hd, max_seq
        self.theta, self.dt, self.seed = theta, dt, seed
        rng = np.random.default_rng(seed)
        self.ctx = rng.integers(ctx_lo, ctx_hi + 1, size=B).astype(np.int64)
        self.pos = (self.ctx - 1).astype(np.int32)

    def describe(self, world):
        sh = getattr(self, "sh", None)
        par = "1 GPU"
        if world > 1 and sh is not None:
            par = f"kv-heads/{sh.head_groups} x sequences/{world // sh.head_groups}"
        return {"workload": self.name, "batch": self.B, "n_heads": self.H, "n_kv_heads": self.Hkv,
                "head_dim": self.hd, "max_seq": self.max_seq, "ctx_sum": int(self.ctx.sum()),
                "ctx_range": [int(self.ctx.min()), int(self.ctx.max())], "parallelism": par,
                "head_concat": None if world == 1 else (
                    "NCCL all-gather + eb_head_concat" if GATHER != "fused" else
                    "fused: the decode kernel stores its rows into every rank's buffer")}

    def _bytes(self, seqs, hkv, h):
        es = 2 if self.dt != 0 else 4
        n = len(seqs)
        kv_rows = 2.0 * self.ctx[list(seqs)].sum() * hkv * self.hd * es  # cache rows read (incl. new)
        new_kv = 2.0 * n * hkv * self.hd * es * 2                          # new k/v read + written
        qo = n * h * self.hd * es * 2                                      # q read, o written
        return kv_rows + new_kv + qo

    def bytes_total(self) -> float:
        return self._bytes(range(self.B), self.Hkv, self.H)

    def setup(self, rank, world):
        import torch

        import eyebrowse_b200 as eb
        self.eb = eb
        self.world = world
        if world > 1 and GATHER != "fused":
            self.sh = decode_shard(self.H, self.Hkv, world, rank, self.ctx, head_groups=world)
        else:
            self.sh = decode_shard(self.H, self.Hkv, world, rank, self.ctx)
        sh = self.sh
        self.seqs = list(sh.seqs)
        self.Bl, self.Hl, self.Hkvl = len(self.seqs), sh.n_heads, sh.n_kv_heads
        tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[self.dt]
        self.tdt = tdt
        g = torch.Generator(device="cuda").manual_seed(self.seed * 1000 + rank)
        Bl, hd = self.Bl, self.hd
        self.kc = torch.randn(Bl, self.max_seq, self.Hkvl, hd, device="cuda", generator=g).to(tdt)
        self.vc = torch.randn(Bl, self.max_seq, self.Hkvl, hd, device="cuda", generator=g).to(tdt)
        self.q = torch.randn(Bl, self.Hl, hd, device="cuda", generator=g).to(tdt)
        self.k = torch.randn(Bl, self.Hkvl, hd, device="cuda", generator=g).to(tdt)
        self.v = torch.randn(Bl, self.Hkvl, hd, device="cuda", generator=g).to(tdt)
        self.o = torch.empty(Bl, self.Hl, hd, device="cuda", dtype=tdt)
        lpos = self.pos[self.seqs]
        self.posd = torch.from_numpy(np.ascontiguousarray(lpos)).cuda()
        self.seq_idx = torch.tensor(self.seqs, dtype=torch.int32, device="cuda")
        cos, sin = eb.rope_tables(self.max_seq, hd, self.theta)
        self.cos = torch.from_numpy(cos).cuda()
        self.sin = torch.from_numpy(sin).cuda()
        self.desc = eb.make_desc(self.Hl, self.Hkvl, hd, self.max_seq, dtype_qkv=self.dt,
                                 dtype_cache=self.dt, dtype_out=self.dt)
        self.layer = eb.make_layer(rope_cos=self.cos, rope_sin=self.sin)
        self.max_pos = int(lpos.max())
        nb = eb.attention_decode_workspace_bytes(self.desc, Bl, self.max_pos)
        self.ws = eb.alloc_workspace(nb) if nb else None
        self.gout = None
        if world > 1 and GATHER == "fused":
            self.gout = GatheredOutput(self.B, self.H, hd, tdt, sh)
            self.full = self.gout.bufs[0]
            self.launches_per_step = 2  # decode (with the peer stores), barrier
        elif world > 1:
            self.gath = torch.empty(world, self.B, self.Hl, hd, device="cuda", dtype=tdt)
            self.full = torch.empty(self.B, self.H, hd, device="cuda", dtype=tdt)
            self.launches_per_step = 2  # decode, head concat (plus NCCL's all-gather)
        else:
            self.full = self.o
            self.launches_per_step = 1

    def _call(self, gather=None):
        if gather is None:
            self.eb.attention_decode_batched(self.desc, self.layer, self.Bl, self.posd,
                                             self.max_pos, self.q, self.k, self.v, self.kc,
                                             self.vc, self.max_seq * self.Hkvl * self.hd, self.o,
                                             self.ws)
        else:
            self.eb.attention_decode_batched_gather(
                self.desc, self.layer, self.Bl, self.posd, self.max_pos, self.q, self.k, self.v,
                self.kc, self.vc, self.max_seq * self.Hkvl * self.hd, gather, self.seq_idx,
                self.ws)

    def step(self):
        if self.gout is not None:
            self._call(self.gout.next())
            self.gout.finish()
            self.full = self.gout.full
            return
        self._call()
        if self.world > 1:
            gather_heads(self.o, self.gath, self.full, self.world, self.B, self.Hl, self.hd,
                         self.dt)

    def kernel_only(self):
        """The decode kernel alone (with its NVLink stores when fused; calls
        back to back store the same values into this rank's rows, so no
        barrier is needed between them)."""
        self._call(self.gout.gathers[0] if self.gout is not None else None)

    def kernel_units(self):
        return self._bytes(self.seqs, self.Hkvl, self.Hl)


class DecodeWork:
    """Config 2 (and config 4's decode): one sequence, fused decode step; the
    timed loop rotates over `n_rot` independent caches so the working set
    exceeds L2."""

    def __init__(self, name, H, Hkv, hd, max_seq, pos, theta, qk_norm, v_norm=False, scale=None,
                 rope_angles=None, n_rot=32, seed=2):
        self.name, self.H, self.Hkv, self.hd, self.max_seq, self.pos = name, H, Hkv, hd, max_seq, pos
        self.theta, self.qk_norm, self.v_norm, self.rope_angles = theta, qk_norm, v_norm, rope_angles
        self.scale = scale if scale is not None else hd ** -0.5
        self.n_rot, self.seed = n_rot, seed
        self.graph_reps = n_rot  # one pass over the rotating caches per graph replay

    def describe(self, world):
        return {"workload": self.name, "n_heads": self.H, "n_kv_heads": self.Hkv, "head_dim": self.hd,
                "max_seq": self.max_seq, "pos": self.pos, "caches_rotated": self.n_rot,
                "parallelism": "1 GPU (replicas)" if world > 1 else "1 GPU"}

    def bytes_total(self):
        rows = self.pos  # cached rows read (0..pos-1) plus the new row below
        return (2.0 * rows * self.Hkv * self.hd * 4 + self.H * self.hd * 4 * 2
                + 2 * self.Hkv * self.hd * 4 * 3)

    def setup(self, rank, world):
        import torch

        import eyebrowse_b200 as eb
        self.eb = eb
        self.world = world
        g = torch.Generator(device="cuda").manual_seed(self.seed)
        n, hd = self.n_rot, self.hd
        self.kcs = [torch.randn(self.max_seq, self.Hkv, hd, device="cuda", generator=g)
                    for _ in range(n)]
        self.vcs = [torch.randn(self.max_seq, self.Hkv, hd, device="cuda", generator=g)
                    for _ in range(n)]
        self.q = torch.randn(self.H, hd, device="cuda", generator=g)
        self.k = torch.randn(self.Hkv, hd, device="cuda", generator=g)
        self.v = torch.randn(self.Hkv, hd, device="cuda", generator=g)
        self.o = torch.empty(self.H, hd, device="cuda")
        cos, sin = eb.rope_tables(self.max_seq, hd, self.theta, self.rope_angles)
        self.cos, self.sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
        w = torch.ones(hd, device="cuda") if self.qk_norm else None
        vw = torch.ones(hd, device="cuda") if self.v_norm else None
        self._keep = (w, vw)
        self.desc = eb.make_desc(self.H, self.Hkv, hd, self.max_seq, scale=self.scale)
        self.layer = eb.make_layer(w, w, vw, self.cos, self.sin)
        nb = eb.attention_decode_workspace_bytes(self.desc, 1, self.pos)
        self.ws = eb.alloc_workspace(nb) if nb else None
        self.i = 0
        self.full = self.o
        self.launches_per_step = 1

    def step(self):
        j = self.i % self.n_rot
        self.i += 1
        self.eb.attention_decode(self.desc, self.layer, self.pos, self.q, self.k, self.v,
                                 self.kcs[j], self.vcs[j], self.o, self.ws)

    kernel_only = step

    def kernel_units(self):
        return self.bytes_total()


class LinearWork:
    """The projections around the path (linear_f16w through eb_linear_f16w):
    y [m, n] = x [m, k] (f32) @ w [n, k]^T (f16). m > 8 runs on the tensor
    cores (x as f16 hi + lo planes: 2 * 2mnk MMA FLOP per 2mnk of algorithmic
    work) and is reported in TFLOP/s; m <= 8 streams w and is reported in
    GB/s. The weights stay resident (they are the model); the e2e step copies
    x in from pinned host memory and y back."""

    def __init__(self, name, m, k, n, seed=6):
        self.name, self.m, self.k, self.n, self.seed = name, m, k, n, seed
        self.bound = "tensor" if m > 8 else "hbm"

    def describe(self, world):
        return {"workload": self.name, "m": self.m, "in_features": self.k,
                "out_features": self.n, "weights": "f16", "activations": "f32",
                "parallelism": "1 GPU (replicas)" if world > 1 else "1 GPU"}

    def flops(self):
        return 2.0 * self.m * self.n * self.k

    def bytes_total(self):
        return 2.0 * self.n * self.k + 4.0 * self.m * (self.k + self.n)

    def setup(self, rank, world):
        import torch

        import eyebrowse_b200 as eb
        self.eb, self.world = eb, world
        g = torch.Generator(device="cuda").manual_seed(self.seed)
        self.x = torch.randn(self.m, self.k, device="cuda", generator=g)
        self.w = (torch.randn(self.n, self.k, device="cuda", generator=g) * 0.02).half()
        self.y = torch.empty(self.m, self.n, device="cuda")
        nb = eb.linear_f16w_workspace_bytes(self.m, self.k, self.n)
        self.ws = eb.alloc_workspace(nb) if nb else None
        self.launches_per_step = 2 if nb else 1  # split of x + GEMM, or the GEMV
        self.full = self.y

    def step(self):
        self.eb.linear_f16w(self.x, self.w, self.y, self.m, self.k, self.n, self.ws)

    kernel_only = step

    def kernel_units(self):
        return self.flops() if self.bound == "tensor" else self.bytes_total()

    def e2e(self, rank, world, steps, unit):
        import torch
        hx = self.x.cpu().pin_memory()
        x2, y2 = torch.empty_like(self.x), torch.empty_like(self.y)
        slots = [([self.x], self.y, torch.empty(self.y.shape).pin_memory()),
                 ([x2], y2, torch.empty(self.y.shape).pin_memory())]
        eb = self.eb

        def run(a):
            xs, ys = (self.x, self.y) if a == 0 else (x2, y2)
            eb.linear_f16w(xs, self.w, ys, self.m, self.k, self.n, self.ws)
        ems = max_over_ranks(time_e2e_pipelined(slots, [hx], run, steps, 2), world)
        units = self.flops() / 1e12 if self.bound == "tensor" else self.bytes_total() / 1e9
        return {"value": units / (ems / steps * 1e-3), "unit": unit,
                "h2d_bytes_per_step": int(hx.numel() * 4),
                "d2h_bytes_per_step": int(self.y.numel() * 4),
                "note": "pinned host x in, y out every step; steps pipelined over two slots "
                        "(upload, compute, download on separate streams)"}


def _median_time(fn, reps: int) -> float:
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def _host_threads() -> int:
    return len(os.sched_getaffinity(0))


def cpu_baseline_linear(w: LinearWork, threads: int | None = None, reps: int = 3):
    """Oracle cpu_linear (the reference's loop order) on a fixed sample -- 8
    rows (m, if smaller) x 2048 output features (all, if fewer) at the
    workload's k -- on all host threads (parallel over output features) and
    on one thread (256 features), median of `reps` timings each, scaled to
    the workload's unit."""
    from oracle import oracle as orc
    threads = threads or _host_threads()
    rng = np.random.default_rng(0)
    m = min(w.m, 8)
    x = rng.standard_normal((m, w.k)).astype(np.float32)

    def measure(n, nt):
        wt = (rng.standard_normal((n, w.k)) * 0.02).astype(np.float16).astype(np.float32)
        dt = _median_time(lambda: orc.linear_threaded(x, wt, m, w.k, n, nt), reps)
        flop, nbytes = 2.0 * m * n * w.k, 2.0 * n * w.k
        return (flop / dt / 1e12 if w.bound == "tensor" else nbytes / dt / 1e9), dt

    n_all, n_one = min(w.n, 2048), min(w.n, 256)
    v_all, dt_all = measure(n_all, threads)
    v_one, dt_one = measure(n_one, 1)
    unit = "TFLOP/s" if w.bound == "tensor" else "GB/s"
    return {"value": v_all, "unit": unit, "cores": threads, "kind": "port",
            "sample": f"oracle cpu_linear, {m} rows x {n_all} of {w.n} outputs, k={w.k}; median of "
                      f"{reps} ({dt_all:.2f} s each; f32, gcc -O3 -ffp-contract=off, {threads} "
                      f"threads)",
            "single_thread": {"value": v_one, "unit": unit, "cores": 1,
                              "sample": f"{m} rows x {n_one} outputs; median of {reps} "
                                        f"({dt_one:.2f} s each)"}}


def make_workload(name, batch=None):
    if name == "cfg1":
        return PrefillWork("cfg1 causal GQA prefill S128 H16 Hkv8 hd128 f32 (Qwen3-0.6B layer)",
                           128, 16, 8, 128, 1e6, 0, seed=1)
    if name == "cfg3":
        return PrefillWork("cfg3 causal GQA prefill S8192 H32 Hkv8 hd128 f16 (Llama-3-8B layer)",
                           8192, 32, 8, 128, 5e5, 1, in_scale=0.5, seed=3)
    if name == "cfg3w":
        return PrefillWork("cfg3w config 3 with a 1024-row sliding window (S8192 H32 Hkv8 hd128 "
                           "f16)", 8192, 32, 8, 128, 5e5, 1, in_scale=0.5, seed=3, window=1024)
    if name in ("cfg3r4", "cfg3r8"):
        g = 4 if name == "cfg3r4" else 8
        return PrefillWork(f"{name} one rank's head share of config 3 at {g} GPUs, run on one GPU "
                           f"without the gather: S8192 H{32 // g} Hkv{8 // g} hd128 f16",
                           8192, 32 // g, 8 // g, 128, 5e5, 1, in_scale=0.5, seed=3)
    if name == "cfg4":
        return PrefillWork("cfg4 Gemma-style prefill S4096 H8 Hkv4 hd256 f32 scale 1.0 "
                           "QK-norm V-norm partial rotary 32/128", 4096, 8, 4, 256, 1e6, 0,
                           scale=1.0, qk_norm=True, v_norm=True, rope_angles=32, seed=4)
    if name == "cfg2":
        return DecodeWork("cfg2 decode cache[4096,8,128] f32 pos 2047 QK-norm RoPE fused write",
                          16, 8, 128, 4096, 2047, 1e6, True)
    if name == "cfg4d":
        return DecodeWork("cfg4 decode step hd256 f32 pos 4224", 8, 4, 256, 4352, 4224, 1e6, True,
                          v_norm=True, scale=1.0, rope_angles=32, n_rot=8)
    if name == "cfg5":
        return BatchedDecodeWork(B=batch or 64)
    if name == "proj3":
        return LinearWork("proj3 fused q/k/v projection S8192 hidden 4096 -> (32+2x8)x128 "
                          "(Llama-3-8B layer, config 3's geometry)", 8192, 4096, 6144)
    if name == "projd":
        return LinearWork("projd tied LM head, one decode row: 1024 -> 151936 "
                          "(Qwen3-0.6B geometry)", 1, 1024, 151936)
    raise SystemExit(f"unknown workload {name}")


# ---------------------------------------------------------------- timing
def time_steps(fn, steps, warmup, world, stream=None, min_warm_s=0.0):
    """Device time of `steps` calls of fn (CUDA events), max over ranks. First
    `warmup` untimed calls, then (min_warm_s > 0) enough further untimed calls
    to fill about min_warm_s seconds: a long dense loop settles under the
    power cap, and timing starts once it has. Every rank runs the same number
    of calls (the count is the max over ranks)."""
    import torch
    t_w = time.time()
    for _ in range(warmup):
        fn()
    if min_warm_s > 0:
        torch.cuda.synchronize()
        el = time.time() - t_w
        per = el / max(1, warmup)
        extra = int(min(100000, max(0.0, (min_warm_s - el) / max(per, 1e-6))))
        extra = int(max_over_ranks(float(extra), world))
        for _ in range(extra):
            fn()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record()
    for _ in range(steps):
        fn()
    ev1.record()
    torch.cuda.synchronize()
    t_wall1 = time.time()
    barrier(world)
    ms = ev0.elapsed_time(ev1)
    return max_over_ranks(ms, world), (t_wall0, t_wall1)


def time_e2e_pipelined(slots, h_inputs, run, steps, warmup):
    """Device time (CUDA events) of `steps` end-to-end steps: every step copies
    its inputs in from pinned host memory, runs the public API call and copies
    its result back to pinned host memory. Steps alternate between two device
    slots on three streams (upload, compute, download), so step i+1's upload
    and step i-1's download overlap step i's compute, as a serving loop
    would. slots[a] = (device inputs, device output, pinned host output);
    run(a) issues slot a's computation on the current stream."""
    import torch
    s_in, s_cmp, s_out = (torch.cuda.Stream() for _ in range(3))
    ev_in, ev_cmp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    n = [0]

    def one():
        i = n[0]
        a = i & 1
        d_in, d_out, h_out = slots[a]
        if i >= 2:
            s_in.wait_event(ev_cmp[a])   # step i-2's compute has read this slot's inputs
        with torch.cuda.stream(s_in):
            for d, h in zip(d_in, h_inputs):
                d.copy_(h, non_blocking=True)
        ev_in[a].record(s_in)
        s_cmp.wait_event(ev_in[a])
        if i >= 2:
            s_cmp.wait_event(ev_out[a])  # step i-2's download has read this slot's output
        with torch.cuda.stream(s_cmp):
            run(a)
        ev_cmp[a].record(s_cmp)
        s_out.wait_event(ev_cmp[a])
        with torch.cuda.stream(s_out):
            h_out.copy_(d_out, non_blocking=True)
        ev_out[a].record(s_out)
        n[0] = i + 1
        return a

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for st in (s_in, s_cmp, s_out):
        st.wait_event(e0)
    a = 0
    for _ in range(steps):
        a = one()
    cur.wait_event(ev_out[a])  # the download stream is in order: its last copy ends the run
    e1.record(cur)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


_CPU_INPUTS = {}


def _cpu_inputs(w: PrefillWork):
    key = (w.S, w.H, w.Hkv, w.hd, w.in_scale)
    if key not in _CPU_INPUTS:
        rng = np.random.default_rng(0)
        _CPU_INPUTS[key] = tuple(
            (rng.standard_normal(shape).astype(np.float32) * np.float32(w.in_scale))
            for shape in ((w.S, w.H, w.hd), (w.S, w.Hkv, w.hd), (w.S, w.Hkv, w.hd)))
    return _CPU_INPUTS[key]


# Fixed CPU samples, the same in the bench arm and the reference arm: the last
# `rows` query rows (the longest causal rows) of the first `heads` heads.
PREFILL_SAMPLE_ALL = (1024, 8)   # all host threads, parallel over query rows
PREFILL_SAMPLE_ONE = (128, 1)    # one thread: the single-threaded Rust loop's order


def _prefill_sample(w: PrefillWork, sample, threads: int, reps: int):
    from oracle import oracle as orc
    S, H, Hkv, hd = w.S, w.H, w.Hkv, w.hd
    q, k, v = _cpu_inputs(w)
    rows_n, nh = min(S, sample[0]), min(H, sample[1])
    r0 = S - rows_n
    W = w.window if w.window and w.window < S else S
    dt = _median_time(lambda: orc.attn_prefill_part(q, k, v, H, Hkv, S, hd, w.scale, (r0, S),
                                                    (0, nh), threads,
                                                    window=W if W < S else 0), reps)
    flop = sum(4.0 * hd * min(i + 1, W) for i in range(r0, S)) * nh
    return flop / dt / 1e12, dt, flop, rows_n, nh


def cpu_baseline_prefill(w: PrefillWork, threads: int | None = None, reps: int = 3):
    """Oracle attention (the reference's CPU attention, restated) on fixed
    samples of the workload: PREFILL_SAMPLE_ALL on all host threads and
    PREFILL_SAMPLE_ONE on one thread, median of `reps` timings each."""
    threads = threads or _host_threads()
    v_all, dt_all, f_all, r_all, h_all = _prefill_sample(w, PREFILL_SAMPLE_ALL, threads, reps)
    v_one, dt_one, f_one, r_one, h_one = _prefill_sample(w, PREFILL_SAMPLE_ONE, 1, reps)
    name = w.name.split()[0]
    return {"value": v_all, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"oracle attn_prefill rows [{w.S - r_all},{w.S}) x heads [0,{h_all}) of "
                      f"{name} ({f_all:.3e} FLOP, median of {reps}: {dt_all:.2f} s; f32, gcc -O3 "
                      f"-ffp-contract=off, {threads} threads)",
            "single_thread": {"value": v_one, "unit": "TFLOP/s", "cores": 1,
                              "sample": f"rows [{w.S - r_one},{w.S}) x heads [0,{h_one}) "
                                        f"({f_one:.3e} FLOP, median of {reps}: {dt_one:.2f} s)"}}


DECODE_SAMPLE_ALL = 8   # sequences (the first of the workload's), all host threads
DECODE_SAMPLE_ONE = 1   # one sequence, one thread


def _decode_sample(w: BatchedDecodeWork, n_seq: int, threads: int, reps: int):
    from oracle import oracle as orc
    B = min(n_seq, w.B)
    ms = int(w.ctx[:B].max())
    rng = np.random.default_rng(1)
    kc = rng.standard_normal((B, ms, w.Hkv, w.hd)).astype(np.float32)
    vc = rng.standard_normal((B, ms, w.Hkv, w.hd)).astype(np.float32)
    q = rng.standard_normal((B, w.H, w.hd)).astype(np.float32)
    pos = w.pos[:B]
    dt = _median_time(lambda: orc.attn_decode_batched(q, kc, vc, pos, w.H, w.Hkv, w.hd, ms,
                                                      ms * w.Hkv * w.hd, w.hd ** -0.5,
                                                      nthreads=threads), reps)
    nbytes = 2.0 * (pos.astype(np.int64) + 1).sum() * w.Hkv * w.hd * 2  # at the f16 cache width
    return nbytes / dt / 1e9, dt, B


def cpu_baseline_decode(w: BatchedDecodeWork, threads: int | None = None, reps: int = 3):
    """Oracle decode on the workload's first DECODE_SAMPLE_ALL sequences (all
    host threads, parallel over (sequence, head)) and on its first sequence
    (one thread), median of `reps` timings; bytes counted at the f16 cache
    width the GPU streams."""
    threads = threads or _host_threads()
    v_all, dt_all, b_all = _decode_sample(w, DECODE_SAMPLE_ALL, threads, reps)
    v_one, dt_one, b_one = _decode_sample(w, DECODE_SAMPLE_ONE, 1, reps)
    return {"value": v_all, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle attn_decode on the first {b_all} of {w.B} sequences (f32 math, "
                      f"bytes counted at f16 cache width), median of {reps}: {dt_all:.2f} s, "
                      f"{threads} threads",
            "single_thread": {"value": v_one, "unit": "GB/s", "cores": 1,
                              "sample": f"the first sequence, median of {reps}: {dt_one:.2f} s"}}


# ---------------------------------------------------------------- main
def run_reference(args):
    """The reference arm: the reference's CPU implementation of the path (the
    oracle port; the Rust/wgpu reference cannot run here) on the host cores,
    each step one timing of the same fixed all-threads sample the bench arm
    reports, `value` the median over the timed steps."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = make_workload(args.workload, args.batch)
    threads = _host_threads()
    if isinstance(w, PrefillWork):
        one = lambda: cpu_baseline_prefill(w, threads=threads, reps=1)
    elif isinstance(w, BatchedDecodeWork):
        one = lambda: cpu_baseline_decode(w, threads=threads, reps=1)
    elif isinstance(w, LinearWork):
        one = lambda: cpu_baseline_linear(w, threads=threads, reps=1)
    else:
        raise SystemExit("--impl reference supports cfg1, cfg3, cfg3w, cfg4, cfg5, proj3, projd")
    vals, singles, base = [], [], None
    for i in range(args.warmup + args.steps):
        b = one()
        if i >= args.warmup:
            vals.append(b["value"])
            singles.append(b["single_thread"]["value"])
            base = b
    v = statistics.median(vals)
    single = dict(base["single_thread"], value=statistics.median(singles))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": base["unit"],
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "data": "synthetic", "dtype": "f32",
            "config": w.describe(1),
            "cpu_baseline": {"value": v, "unit": base["unit"], "cores": base["cores"],
                             "kind": "port", "sample": base["sample"].split("; median")[0]
                             + f"; median of {args.steps} timed steps",
                             "single_thread": single},
            "e2e": {"value": v, "unit": base["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference = oracle/ C restatement of crates/eyebrowse-kernels/src/testutil.rs "
                    "CPU attention (cpu_linear for proj3/projd); the Rust/wgpu reference cannot "
                    "be built or run on this box"}
    print(json.dumps(line), flush=True)
    return 0


def graphed(fn, reps: int):
    """A CUDA graph of `reps` back-to-back calls of fn (captured after a warm
    call), returned as a function that replays it. Used for workloads whose
    step is a few microseconds, so host launch overhead does not set the
    measured time."""
    import torch
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    return g.replay, g


def measure(w, rank, world, steps, warmup, peaks, peak_kind, sampler=None):
    """Step time and dominant-kernel time for one workload (CUDA events).
    Workloads flagged `graph_reps` replay a CUDA graph of that many steps."""
    import torch
    w.setup(rank, world)
    reps = getattr(w, "graph_reps", 0) if world == 1 else 0
    step, kern = w.step, w.kernel_only
    if reps:
        step, w._g1 = graphed(w.step, reps)
        kern, w._g2 = graphed(w.kernel_only, reps)
        steps = max(1, steps // reps)
    if sampler:
        sampler.start()
    ms, (t0, t1) = time_steps(step, steps, warmup, world, min_warm_s=WARM_S)
    if sampler:
        sampler.mark(t0, t1)
    # dominant kernel alone (CUDA events on the launching stream)
    kms, _ = time_steps(kern, steps, max(1, warmup), world, min_warm_s=WARM_S)
    n = steps * max(1, reps)
    return {"ms_per_step": ms / n, "kernel_ms": kms / n, "graph_reps": reps}


def main():
    global WARM_S, GATHER
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="cfg3")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="N>1 head-concat exchange: fused into the attention kernel "
                         "(default) or NCCL all-gather + concat")
    ap.add_argument("--warm-s", type=float, default=None,
                    help="untimed seconds before each timed loop (default %.1f; 0 for "
                         "profiling runs)" % WARM_S)
    ap.add_argument("--batch", type=int, default=None,
                    help="cfg5 only: sequences per step (default 64; smaller for profiling)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.warm_s is not None:
        WARM_S = max(0.0, args.warm_s)
    GATHER = args.gather
    if args.impl == "reference":
        return run_reference(args)

    import torch
    rank, world, local = init_dist(args.gpus)
    peaks, peak_kind = load_peaks()
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid) if rank == 0 else None

    w = make_workload(args.workload, args.batch)
    res = measure(w, rank, world, args.steps, args.warmup, peaks, peak_kind, sampler)
    is_prefill = isinstance(w, PrefillWork)
    is_tensor = is_prefill or getattr(w, "bound", "") == "tensor"
    if is_tensor:
        total_units = w.flops()
        unit, bound = "TFLOP/s", "tensor"
        value = total_units / (res["ms_per_step"] * 1e-3) / 1e12
        kern_units = w.kernel_units()
        achieved = kern_units / (res["kernel_ms"] * 1e-3) / 1e12
        # the kernel is timed inside a seconds-long loop under the power cap
        peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
        peak_unit, peak_name = "TFLOP/s", "bf16_tflops_sustained"
    else:
        total_units = w.bytes_total()
        kern_units = w.kernel_units()
        unit, bound = "GB/s", "hbm"
        value = total_units / (res["ms_per_step"] * 1e-3) / 1e9
        achieved = w.kernel_units() / (res["kernel_ms"] * 1e-3) / 1e9
        peak = peaks.get("hbm_gbs")
        peak_unit, peak_name = "GB/s", "hbm_gbs"
    # `achieved` is per GPU: this rank's units over the slowest rank's kernel time

    # e2e: the same step through the public API with host buffers
    e2e = None
    if hasattr(w, "e2e"):
        e2e = w.e2e(rank, world, args.e2e_steps, unit)
    elif is_prefill and world == 1:
        e2e = w.e2e_pipelined(args.e2e_steps, unit, total_units)
    elif is_prefill:
        w.setup_e2e()
        bi = bo = 0

        def e2e_step():
            nonlocal bi, bo
            bi, bo = w.step_e2e(rank)
        ems, _ = time_steps(e2e_step, args.e2e_steps, 2, world)
        tot_in = sum_over_ranks(float(bi), world)
        e2e = {"value": total_units / (ems / args.e2e_steps * 1e-3) / 1e12, "unit": unit,
               "h2d_bytes_per_step": int(tot_in), "d2h_bytes_per_step": int(bo),
               "note": "h2d summed over ranks from pinned host buffers; rank 0 reads the "
                       "gathered [S,H,hd] output back"}
    else:
        e2e = decode_e2e(w, rank, world, args.e2e_steps, unit)
    if sampler:
        sampler.stop()
    clocks = sampler.summary() if sampler else None

    decode = None
    if is_prefill and not args.no_decode and args.workload == "cfg3":
        dw = BatchedDecodeWork()
        dres = measure(dw, rank, world, max(20, args.steps // 10), args.warmup, peaks, peak_kind)
        dval = dw.bytes_total() / (dres["ms_per_step"] * 1e-3) / 1e9
        dach = dw.kernel_units() / (dres["kernel_ms"] * 1e-3) / 1e9
        decode = {"workload": dw.describe(world)["workload"] + " batched decode B64 H32 Hkv8 "
                  "hd128 f16 cache ctx U[512,32768]", "value": dval, "unit": "GB/s",
                  "ms_per_step": dres["ms_per_step"], "config": dw.describe(world),
                  "roofline": {"bound": "hbm", "achieved": dach, "peak": peaks.get("hbm_gbs"),
                               "unit": "GB/s", "frac": dach / peaks.get("hbm_gbs"),
                               "traffic": rank_traffic("decode_cfg5", dw.kernel_units() /
                                                       dw.bytes_total() if world > 1 else 1.0),
                               "peak_source": f"{peak_kind} hbm_gbs"}}
        if not args.no_cpu and rank == 0 and world == 1:
            decode["cpu_baseline"] = cpu_baseline_decode(dw)
        del dw

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        if is_prefill:
            cpu = cpu_baseline_prefill(w)
        elif isinstance(w, BatchedDecodeWork):
            cpu = cpu_baseline_decode(w)
        elif isinstance(w, LinearWork):
            cpu = cpu_baseline_linear(w)

    launches = w.launches_per_step * args.steps
    if rank == 0:
        tkey = {"cfg3": "prefill_cfg3", "cfg1": "prefill_cfg1", "cfg4": "prefill_cfg4",
                "cfg2": "decode_cfg2", "cfg5": "decode_cfg5", "proj3": "linear_proj3",
                "projd": "linear_projd"}.get(args.workload)
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": {0: "f32", 1: "f16", 2: "bf16"}.get(getattr(w, "dt", 0), "f32"),
            "data": "synthetic (seeded N(0,1) inputs of the config's shapes; no dataset)",
            "config": dict(w.describe(world), l2="inputs larger than L2 (no flush)"
                           if is_prefill or isinstance(w, (BatchedDecodeWork, LinearWork))
                           else "rotating caches larger than L2",
                           untimed_warm_s=WARM_S),
            "cuda_graph_steps": res.get("graph_reps", 0),
            "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": peak_unit,
                         "frac": achieved / peak,
                         "traffic": (rank_traffic(tkey, kern_units / total_units if world > 1 else 1.0)
                                     if tkey else None),
                         "peak_source": f"{peak_kind} {peak_name}",
                         "kernel_ms": res["kernel_ms"]},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if decode:
            line["decode"] = decode
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def decode_e2e(w, rank, world, steps, unit):
    """Decode e2e: every step uploads the new token's q/k/v rows from pinned
    host memory, runs the step through the public API and reads o back.
    With one dtype, q, k and v sit packed in one pinned buffer and the
    workload's device tensors become views of its device copy, so a step
    pays one upload's DMA set-up instead of three (a few microseconds each,
    most of a single-sequence step)."""
    import torch
    srcs = (w.q, w.k, w.v)
    if len({t.dtype for t in srcs}) == 1:
        flat = torch.cat([t.reshape(-1) for t in srcs])
        hbuf, dbuf = flat.cpu().pin_memory(), flat.clone()
        views, off = [], 0
        for t in srcs:
            views.append(dbuf[off:off + t.numel()].view(t.shape))
            off += t.numel()
        w.q, w.k, w.v = views
        uploads = [(dbuf, hbuf)]
    else:
        uploads = [(t, t.cpu().pin_memory()) for t in srcs]
    hout = torch.empty(w.full.shape, dtype=w.full.dtype).pin_memory()
    nb_in = sum(h.numel() * h.element_size() for _, h in uploads)

    def st():
        for d, h in uploads:
            d.copy_(h, non_blocking=True)
        w.step()
        if rank == 0:
            hout.copy_(w.full, non_blocking=True)
    ems, _ = time_steps(st, steps, 2, world)
    total = w.bytes_total()
    return {"value": total / (ems / steps * 1e-3) / 1e9, "unit": unit,
            "h2d_bytes_per_step": int(sum_over_ranks(float(nb_in), world)),
            "d2h_bytes_per_step": int(hout.numel() * hout.element_size()),
            "note": f"pinned host q/k/v in ({len(uploads)} upload(s)), o out every step"}


if __name__ == "__main__":
    sys.exit(main())
