#!/usr/bin/env python3
"""Benchmark of the B200-native attention / Gated DeltaNet hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload attn_c5|attn_c1|attn_c2|attn_gated_d256|gdn_decode|gdn_decode_state16|gdn_prefill
                                |gdn_prefill_fused|<any secondary attention shape, e.g. attn_splitkv_q1>]

One JSON line on stdout (rank 0).  The headline workload is the long-context
causal GQA attention config (B4 Hq32 Hkv8 S16384 D128 bf16), the config the
reference's metric is sharded across 1/2/4/8 GPUs on; GDN decode (GB/s), GDN
prefill (tok/s), gated attention and the other attention shapes (C1, C2, the
C5 shape at S 4096 / 8192 with D 128 / 64, split-KV short queries) are
reported in the same line under "secondary", each with its own roofline, and
the line ends with a compact "summary" of every figure.

Multi-GPU: one process per GPU (torchrun), units sharded across ranks with no
data-path collective -- attention by (batch, kv-head) with its q-heads, GDN
decode by sequence, GDN prefill by v-head.  Timing: CUDA events on the stream
the kernels are launched on, barrier + synchronize around the timed region,
MAX over ranks.  The optional NCCL all-gather of attention outputs is timed
separately ("allgather").

--impl reference: the CPU implementation of the path timed on this host's
cores (the reference has no CPU attention, so the fp64 restatement of its
naive kernel in oracle/ stands in), on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "turing-sm75_b200"))
sys.path.insert(0, ROOT)

BASELINE_METRIC = "attn fwd TFLOP/s, GDN prefill tok/s, GDN decode GB/s; % roofline @1/2/4/8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------------------
# small utilities
# ----------------------------------------------------------------------------
def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def _scaled(x, f):
    return None if x is None else x * f


def profile_traffic(name, key=None):
    """Per-launch DRAM bytes of the dominant kernel, read from the committed ncu
    summary profiles/<name>.md (line `traffic_bytes_per_launch: <float>`, or
    `traffic_bytes_per_launch[<key>]: <float>` in a summary that covers several workloads)."""
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    tag = "traffic_bytes_per_launch:" if key is None else f"traffic_bytes_per_launch[{key}]:"
    try:
        for line in open(path):
            if line.strip().startswith(tag):
                return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


class L2Flush:
    """Evicts the timed kernel's inputs from L2 between launches: writes a buffer larger
    than L2, then reads another, so L2 is left holding clean unrelated lines (the write
    alone would leave ~126 MB of dirty lines for the timed kernel to write back)."""

    def __init__(self, dev, nbytes=256 << 20):
        import torch
        self.w = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.r = torch.ones(nbytes // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.sum()


def host_ahead(n_steps, us_per_step=250.0, min_us=50000.0):
    """Queues a GPU spin of max(n_steps x us_per_step, min_us) microseconds before a loop that
    times every call with its own pair of events.  The host enqueues the whole loop (flush,
    events, launches) while the GPU spins, so no call's events include host time, and the SM
    clock, which drops while the GPU idles between legs (input set-up, the clock sampler's
    start), is back at its boost before the first timed call: a leg timed over a few
    milliseconds otherwise runs on the ramp (one GPU prefill leg sampled 1762 of 1965 MHz).
    The spin itself lies outside every event pair."""
    import torch

    us = max(n_steps * us_per_step, min_us)
    torch.cuda._sleep(int(us * 2000))  # ~2000 SM cycles a microsecond


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    NAMES = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, torch_device, period_s=0.05):
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            uuid = "GPU-" + str(torch.cuda.get_device_properties(torch_device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report, do not fail the bench
            self.h = None
            self.err = repr(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception as e:
                self.err = repr(e)
            self._stop.wait(self.period)

    def __enter__(self):
        if self.h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.err or "no samples"}
        busy = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = set()
        for _, r in busy:
            for bit, name in self.NAMES.items():
                if r & bit and bit != 0x1:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in busy), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(busy)}


# ----------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------
class Dist:
    def __init__(self, want_gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != want_gpus:
            raise SystemExit(f"--gpus {want_gpus} but WORLD_SIZE={self.world}")
        self.pg = None

    def init(self):
        import torch
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([float(x)], device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def split_units(total, world, rank):
    import sharding
    try:
        return sharding.split_units(total, world, rank)
    except ValueError as e:
        raise SystemExit(str(e))


# ----------------------------------------------------------------------------
# workloads (ours)
# ----------------------------------------------------------------------------
def attn_shard(cfg, world, rank):
    """(batch, kv-head) units with their q-heads; returns the local (B, Hq, Hkv)."""
    import sharding
    b0, nb, h0, nh = sharding.attn_shard(cfg["B"], cfg["Hq"], cfg["Hkv"], world, rank)
    return nb, nh * (cfg["Hq"] // cfg["Hkv"]), nh


def attn_flops(B, Hq, S, D, causal):
    return (2.0 * B * Hq * S * (S + 1) * D) if causal else (4.0 * B * Hq * S * S * D)


def bench_attention(name, cfg, args, dist, peaks):
    import torch
    import b200lab
    import workloads

    B, Hq, Hkv = attn_shard(cfg, dist.world, dist.rank)
    S, D, causal, dtype = cfg["S"], cfg["D"], cfg["causal"], cfg["dtype"]
    dev = torch.device("cuda", dist.local)
    Q, K, V = workloads.attn_inputs(B, Hq, Hkv, S, D, dtype, seed=42 + dist.rank, device=dev)
    O = torch.empty_like(Q)
    stream = torch.cuda.current_stream()
    flops_local = attn_flops(B, Hq, S, D, causal)
    flops_total = attn_flops(cfg["B"], cfg["Hq"], S, D, causal)
    in_bytes = (Q.numel() + K.numel() + V.numel()) * Q.element_size()

    def step():
        b200lab.attn_fwd(Q, K, V, causal=causal, out=O, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    n0 = b200lab.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = b200lab.launch_count() - n0
    dist.barrier()
    torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = dist.max(ms_local)
    status = b200lab.device_status()
    if status != b200lab.OK:
        raise RuntimeError(f"device status {status}: {b200lab.strerror(status)}")

    # end to end: pinned host inputs -> device, kernel, result -> pinned host
    Qh, Kh, Vh = (t.cpu().pin_memory() for t in (Q, K, V))
    Oh = torch.empty(O.shape, dtype=O.dtype, pin_memory=True)
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_step():  # the host-buffer entry: copies in, compute and copies out pipelined by chunk
        b200lab.attn_fwd_host(Qh, Kh, Vh, Oh, Q, K, V, O, causal=causal, stream=stream)

    e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist.max(e0.elapsed_time(e1) / e2e_steps)

    # the same host<->device bytes with no kernel: all copies in and out at once, every rank
    # at the same time (the floor the host-buffer call runs against)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def copies_only():
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        with torch.cuda.stream(s_in):
            Q.copy_(Qh, non_blocking=True)
            K.copy_(Kh, non_blocking=True)
            V.copy_(Vh, non_blocking=True)
        with torch.cuda.stream(s_out):
            Oh.copy_(O, non_blocking=True)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    copies_only()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        copies_only()
    e1.record(stream)
    torch.cuda.synchronize()
    floor_ms = dist.max(e0.elapsed_time(e1) / e2e_steps)

    # optional NCCL all-gather of the output shards (sharding.allgather_attention), timed
    # on its own
    allgather = None
    if dist.world > 1:
        import sharding
        for _ in range(2):
            full = sharding.allgather_attention(O, cfg["B"], cfg["Hq"])
        torch.cuda.synchronize()
        dist.barrier()
        e0.record(stream)
        for _ in range(3):
            full = sharding.allgather_attention(O, cfg["B"], cfg["Hq"])
        e1.record(stream)
        torch.cuda.synchronize()
        ag_ms = dist.max(e0.elapsed_time(e1) / 3)
        total_bytes = full.numel() * full.element_size()
        allgather = {"ms": ag_ms, "bytes_per_rank_out": O.numel() * O.element_size(),
                     "bus_gbs": total_bytes * (dist.world - 1) / dist.world / (ag_ms * 1e-3) / 1e9,
                     "kernel_plus_allgather_ms": ms + ag_ms}
        del full

    tflops = flops_total / (ms * 1e-3) / 1e12
    achieved = flops_local / (ms_local * 1e-3) / 1e12
    peak = peaks["bf16_tflops"]
    traffic = profile_traffic(f"attn_fwd_{name}")
    res = {
        "metric": BASELINE_METRIC if name == "attn_c5" else f"attn fwd TFLOP/s ({name})",
        "value": tflops, "unit": "TFLOP/s", "ms_per_step": ms,
        "flops_per_step": flops_total, "flop_convention": "causal-exec 2*B*H*S*(S+1)*D"
        if causal else "4*B*H*S^2*D",
        "dtype": "bf16" if dtype == torch.bfloat16 else "fp16",
        "config": {"workload": name, "B": cfg["B"], "Hq": cfg["Hq"], "Hkv": cfg["Hkv"], "S": S,
                   "D": D, "causal": causal, "sharding": "(batch, kv-head) units",
                   "local_shape": [B, Hq, Hkv, S, D],
                   "l2": f"inputs larger than L2 ({in_bytes / 1e6:.0f} MB per GPU)"
                   if in_bytes > 126e6 else "inputs smaller than L2 (back to back)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     # profiles/ records DRAM bytes of one full-config launch (N=1);
                     # a shard moves its units' share
                     "traffic": None if traffic is None else traffic * flops_local / flops_total},
        "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": O.numel() * O.element_size(),
                "copy_floor_ms": floor_ms, "frac_of_copy_floor": floor_ms / e2e_ms,
                "copy_floor_note": "the same copies in and out with no kernel, all ranks at once"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if allgather:
        res["allgather"] = allgather
    del Q, K, V, O, Qh, Kh, Vh, Oh, s_in, s_out
    torch.cuda.empty_cache()
    return res


# Secondary attention shapes: the BASELINE configs C1 and C2, the C5 shape at S 4096 / 8192
# with head dim 128 and 64, and short queries against a long key range (split-KV).
ATTN_CASES = {
    "attn_c1": dict(B=1, Hq=4, Hkv=4, Sq=256, Skv=256, D=128, causal=False, dtype="f16"),
    "attn_c2_d128_causal": dict(B=2, Hq=8, Hkv=8, Sq=512, Skv=512, D=128, causal=True, dtype="bf16"),
    "attn_c2_d128": dict(B=2, Hq=8, Hkv=8, Sq=512, Skv=512, D=128, causal=False, dtype="bf16"),
    "attn_c2_d64_causal": dict(B=2, Hq=8, Hkv=8, Sq=512, Skv=512, D=64, causal=True, dtype="bf16"),
    "attn_c2_d64": dict(B=2, Hq=8, Hkv=8, Sq=512, Skv=512, D=64, causal=False, dtype="bf16"),
    "attn_s4096_d128": dict(B=4, Hq=32, Hkv=8, Sq=4096, Skv=4096, D=128, causal=True, dtype="bf16"),
    "attn_s8192_d128": dict(B=4, Hq=32, Hkv=8, Sq=8192, Skv=8192, D=128, causal=True, dtype="bf16"),
    "attn_s4096_d64": dict(B=4, Hq=32, Hkv=8, Sq=4096, Skv=4096, D=64, causal=True, dtype="bf16"),
    "attn_s8192_d64": dict(B=4, Hq=32, Hkv=8, Sq=8192, Skv=8192, D=64, causal=True, dtype="bf16"),
    "attn_splitkv_q1": dict(B=1, Hq=32, Hkv=8, Sq=1, Skv=16384, D=128, causal=True, dtype="bf16"),
    "attn_splitkv_q64": dict(B=1, Hq=32, Hkv=8, Sq=64, Skv=16384, D=128, causal=True, dtype="bf16"),
}


def attn_case_flops(B, Hq, Sq, Skv, D, causal):
    """QK^T and PV FLOPs over the visible (query, key) pairs; causal masks are aligned at the
    bottom right (query i sees keys j <= Skv - Sq + i), so Sq = Skv gives 2 B H S (S+1) D."""
    if not causal:
        return 4.0 * B * Hq * Sq * Skv * D
    off = Skv - Sq
    pairs = sum(min(Skv, max(0, off + i + 1)) for i in range(Sq))
    return 4.0 * B * Hq * pairs * D


def bench_attn_case(name, shp, args, dist, peaks):
    """One attention shape through attn_fwd_sm100 (workspace preallocated), device-timed.
    Inputs smaller than L2 are timed launch by launch with L2 flushed before each; larger ones
    back to back.  Roofline: the slower of tensor peak and HBM bandwidth for the shape."""
    import torch
    import b200lab
    import workloads

    B, Hq, Hkv, Sq, Skv, D, causal = (shp[k] for k in ("B", "Hq", "Hkv", "Sq", "Skv", "D", "causal"))
    dtype = torch.float16 if shp["dtype"] == "f16" else torch.bfloat16
    units = B * Hkv
    if units % dist.world == 0:
        import sharding
        b0, nb, h0, nh = sharding.attn_shard(B, Hq, Hkv, dist.world, dist.rank)
        Bl, Hql, Hkvl, shard = nb, nh * (Hq // Hkv), nh, "(batch, kv-head) units"
        total_flops = attn_case_flops(B, Hq, Sq, Skv, D, causal)
    else:  # fewer units than GPUs: every GPU runs the whole shape
        Bl, Hql, Hkvl, shard = B, Hq, Hkv, "replicas (fewer units than GPUs)"
        total_flops = dist.world * attn_case_flops(B, Hq, Sq, Skv, D, causal)
    dev = torch.device("cuda", dist.local)
    Q, K, V = workloads.attn_inputs(Bl, Hql, Hkvl, Sq, D, dtype, seed=61 + dist.rank, device=dev, Skv=Skv)
    O = torch.empty_like(Q)
    need = int(b200lab.lib().attn_fwd_sm100_workspace(Bl, Hql, Hkvl, Sq, Skv, D, int(causal)))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev) if need else None
    stream = torch.cuda.current_stream()
    flops_local = attn_case_flops(Bl, Hql, Sq, Skv, D, causal)
    bytes_local = (Q.numel() * 2 + K.numel() + V.numel()) * Q.element_size()
    small = bytes_local < 126e6
    steps = max(3, min(args.steps, 20))

    def step():
        b200lab.attn_fwd(Q, K, V, causal=causal, out=O, workspace=ws, stream=stream)

    for _ in range(args.warmup):
        step()
    flush = L2Flush(dev) if small else None
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    n0 = b200lab.launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps if small else 1)]
    with ClockSampler(dev) as clk:
        if small:
            host_ahead(len(evs))
            for e0, e1 in evs:
                flush()
                e0.record(stream)
                step()
                e1.record(stream)
        else:
            evs[0][0].record(stream)
            for _ in range(steps):
                step()
            evs[0][1].record(stream)
        torch.cuda.synchronize()
    launches = b200lab.launch_count() - n0
    ms_local = sum(a.elapsed_time(b) for a, b in evs) / steps
    ms = dist.max(ms_local)
    status = b200lab.device_status()
    if status != b200lab.OK:
        raise RuntimeError(f"device status {status}: {b200lab.strerror(status)}")
    t_tc = flops_local / (peaks["bf16_tflops"] * 1e12)
    t_hbm = bytes_local / (peaks["hbm_gbs"] * 1e9)
    if t_tc >= t_hbm:
        roof = {"bound": "tensor", "achieved": flops_local / (ms_local * 1e-3) / 1e12,
                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": bytes_local / (ms_local * 1e-3) / 1e9,
                "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    # profiles/ records the DRAM bytes of one full-shape call (both kernels for split-KV);
    # a shard of (batch, kv-head) units moves its share, a replica the whole
    traffic = profile_traffic("attn_fwd_cases", name)
    roof["traffic"] = _scaled(traffic, (Bl * Hkvl) / (B * Hkv))
    res = {"metric": f"attn fwd TFLOP/s ({name})", "value": total_flops / (ms * 1e-3) / 1e12,
           "unit": "TFLOP/s", "us_per_step": ms * 1e3, "steps": steps,
           "flop_convention": "visible (query, key) pairs x 4 D (causal: bottom-right aligned)",
           "dtype": shp["dtype"],
           "config": {"workload": name, "B": B, "Hq": Hq, "Hkv": Hkv, "Sq": Sq, "Skv": Skv, "D": D,
                      "causal": causal, "split_kv": bool(need), "sharding": shard,
                      "l2": "L2 flushed before every launch" if small else "inputs larger than L2"},
           "roofline": roof, "gpu_launches": int(launches), "clocks": clk.summary()}
    del Q, K, V, O, ws, flush
    torch.cuda.empty_cache()
    return res


def bench_gated_attention(cfg, args, dist, peaks):
    """attn_gated_fwd_sm100 at the model's gated-attention shape, device-timed (inputs
    resident, larger than L2); (batch, kv-head) sharding as for the headline."""
    import torch
    import b200lab
    import workloads

    B, Hq, Hkv = attn_shard(cfg, dist.world, dist.rank)
    S, D, causal, dtype = cfg["S"], cfg["D"], cfg["causal"], cfg["dtype"]
    dev = torch.device("cuda", dist.local)
    Q, K, V = workloads.attn_inputs(B, Hq, Hkv, S, D, dtype, seed=52 + dist.rank, device=dev)
    G = torch.randn(Q.shape, device=dev, dtype=torch.float32).to(dtype)
    O = torch.empty_like(Q)
    stream = torch.cuda.current_stream()
    steps = max(3, min(args.steps, 10))

    def step():
        b200lab.attn_gated_fwd(Q, K, V, G, causal=causal, out=O, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    n0 = b200lab.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = b200lab.launch_count() - n0
    ms_local = e0.elapsed_time(e1) / steps
    ms = dist.max(ms_local)
    flops_total = attn_flops(cfg["B"], cfg["Hq"], S, D, causal)
    achieved = attn_flops(B, Hq, S, D, causal) / (ms_local * 1e-3) / 1e12
    res = {"metric": "gated attn fwd TFLOP/s", "value": flops_total / (ms * 1e-3) / 1e12,
           "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps,
           "config": {"workload": "attn_gated_d256", "B": cfg["B"], "Hq": cfg["Hq"], "Hkv": cfg["Hkv"],
                      "S": S, "D": D, "causal": causal, "gate": "sigmoid(G), G [B,Hq,S,D]",
                      "l2": "inputs larger than L2"},
           "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                        "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                        "traffic": _scaled(profile_traffic("attn_gated_d256"),
                                           attn_flops(B, Hq, S, D, causal) / flops_total)},
           "gpu_launches": int(launches), "clocks": clk.summary()}
    del Q, K, V, G, O
    torch.cuda.empty_cache()
    return res


def bench_gdn_decode(cfg, args, dist, peaks, state_dtype=None, weak=False):
    """GDN decode over the config's 256 steps; state_dtype fp16/bf16 runs the 16-bit-state
    entry (gdn_decode_sm100_state16), default the fp32 state.  weak: every GPU runs the
    config's B sequences (B x N in all) instead of a 1/N share of them."""
    import torch
    import b200lab
    import workloads

    Bl = cfg["B"] if weak else split_units(cfg["B"], dist.world, dist.rank)[1]
    Hqk, Hv, d, T = cfg["Hqk"], cfg["Hv"], cfg["d"], cfg["steps"]
    dtype = cfg["dtype"]
    dev = torch.device("cuda", dist.local)
    state = workloads.gdn_state(Bl, Hv, d, std=0.02, seed=3 + dist.rank, device=dev)
    sdt = state_dtype or torch.float32
    state = state.to(sdt)
    ssz = state.element_size()
    steps_in = [workloads.gdn_decode_inputs(Bl, Hqk, Hv, d, dtype, seed=1000 * dist.rank + t,
                                            device=dev) for t in range(T)]
    out = torch.empty((T, Bl, Hv, d), dtype=dtype, device=dev)
    stream = torch.cuda.current_stream()
    esz = torch.tensor([], dtype=dtype).element_size()
    bytes_step_local = (Bl * Hv * d * d * ssz * 2 + Bl * Hqk * d * esz * 2 + Bl * Hv * d * esz * 2
                        + Bl * Hv * 4 * 2)

    def run_all():
        for t in range(T):
            q, k, v, g, b = steps_in[t]
            b200lab.gdn_decode(q, k, v, g, b, state, out=out[t], stream=stream)

    run_all()  # warm-up: one pass of the 256-step sequence
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    n0 = b200lab.launch_count()
    state_bytes = state.numel() * ssz
    if state_bytes > 126e6:
        # a state larger than L2 (fp32 at 64 sequences: 134 MB): 256 steps back to back
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev) as clk:
            e0.record(stream)
            run_all()
            e1.record(stream)
            torch.cuda.synchronize()
        ms_local = e0.elapsed_time(e1) / T
    else:
        # a state that fits in L2 (16-bit, or a GPU's share of the sequences) would stay there
        # between steps: flush L2 before every step and time each step alone
        flush = L2Flush(dev)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(T)]
        with ClockSampler(dev) as clk:
            host_ahead(T, 100.0)
            for t in range(T):
                flush()
                q, k, v, g, b = steps_in[t]
                evs[t][0].record(stream)
                b200lab.gdn_decode(q, k, v, g, b, state, out=out[t], stream=stream)
                evs[t][1].record(stream)
            torch.cuda.synchronize()
        ms_local = sum(a.elapsed_time(b) for a, b in evs) / T
        del flush
    launches = b200lab.launch_count() - n0
    ms = dist.max(ms_local)
    gbs = bytes_step_local * dist.world / (ms * 1e-3) / 1e9
    achieved = bytes_step_local / (ms_local * 1e-3) / 1e9
    traffic = _scaled(profile_traffic("gdn_decode_c4" if ssz == 4 else "gdn_decode_state16_c4"),
                      Bl / cfg["B"])
    sname = {4: "fp32", 2: str(sdt).replace("torch.", "")}[ssz]
    res = {"metric": "GDN decode GB/s", "value": gbs, "unit": "GB/s", "us_per_step": ms * 1e3,
           "steps": T, "bytes_per_step": bytes_step_local * dist.world,
           "config": {"workload": "gdn_decode_c4" + ("" if ssz == 4 else f"_state_{sname}")
                      + ("_weak" if weak else ""),
                      "B": Bl * dist.world if weak else cfg["B"], "Hqk": Hqk, "Hv": Hv, "d": d,
                      "state": f"{sname} [B,Hv,128,128] in place",
                      "sharding": f"sequences, {Bl} per GPU (weak scaling)" if weak else "sequences",
                      "l2": f"state larger than L2 ({state_bytes / 1e6:.0f} MB a GPU), 256 consecutive steps"
                      if state_bytes > 126e6
                      else f"L2 flushed before every step (state {state_bytes / 1e6:.0f} MB a GPU)"},
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / peaks["hbm_gbs"], "traffic": traffic},
           "gpu_launches": int(launches), "clocks": clk.summary()}
    del state, steps_in, out
    torch.cuda.empty_cache()
    return res


def bench_gdn_prefill(cfg, args, dist, peaks, fused=False):
    """GDN chunked prefill at C3, L2 flushed before every launch.  fused: the entry with the
    pre-processing fused in (raw q, k L2-normalised in the kernels, gates and beta from
    logits: gdn_prefill_sm100_fused)."""
    import torch
    import b200lab
    import workloads

    T, Hqk, Hv, d, dtype = cfg["T"], cfg["Hqk"], cfg["Hv"], cfg["d"], cfg["dtype"]
    import sharding
    h0, Hv_l, hq0, Hqk_l = sharding.gdn_prefill_shard(Hqk, Hv, dist.world, dist.rank)
    dev = torch.device("cuda", dist.local)
    q, k, v, g, b = workloads.gdn_inputs(1, T, Hqk_l, Hv_l, d, dtype, seed=7 + dist.rank, device=dev)
    if fused:  # raw q, k (unnormalised) and the gate / beta logits with per-head parameters
        gen = torch.Generator(device=dev)
        gen.manual_seed(17 + dist.rank)
        q, k = (torch.randn(t.shape, generator=gen, device=dev).to(dtype) for t in (q, k))
        g, b = (torch.randn(t.shape, generator=gen, device=dev) for t in (g, b))
        A_log = torch.randn((Hv_l,), generator=gen, device=dev) * 0.5
        dt_bias = torch.randn((Hv_l,), generator=gen, device=dev) * 0.5
    state = torch.zeros((1, Hv_l, d, d), dtype=torch.float32, device=dev)
    out = torch.empty((1, T, Hv_l, d), dtype=dtype, device=dev)
    stream = torch.cuda.current_stream()
    ws_bytes = b200lab.gdn_prefill_workspace_bytes(1, T, Hqk_l, Hv_l, d, d)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    flush = L2Flush(dev)

    def step():
        if fused:
            b200lab.gdn_prefill_fused(q, k, v, g, b, state, A_log=A_log, dt_bias=dt_bias, out=out,
                                      workspace=ws, stream=stream)
        else:
            b200lab.gdn_prefill(q, k, v, g, b, state, out=out, workspace=ws, stream=stream)

    try:
        step()
    except b200lab.B200LabError as e:
        return {"metric": "GDN prefill tok/s", "status": str(e)}
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    n0 = b200lab.launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(dev) as clk:
        host_ahead(len(evs))
        for e0, e1 in evs:
            flush()  # inputs (106 MB) fit in L2: flush it between timed launches
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
    launches = b200lab.launch_count() - n0
    ms_local = sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps
    ms = dist.max(ms_local)
    esz = q.element_size()
    bytes_local = ((q.numel() + k.numel() + v.numel() + out.numel()) * esz
                   + (g.numel() + b.numel()) * 4 + state.numel() * 4 * 2)
    flops_local = Hv_l * T * (6 * 64 * d + 6 * d * d) + Hqk_l * T * 4 * 64 * d
    achieved = bytes_local / (ms_local * 1e-3) / 1e9
    allgather = None
    if dist.world > 1:  # o [1][T][Hv][d] on every rank: all-gather + on-device permute
        for _ in range(2):
            full = sharding.allgather_gdn_prefill(out, Hv)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = evs[0]
        e0.record(stream)
        for _ in range(3):
            full = sharding.allgather_gdn_prefill(out, Hv)
        e1.record(stream)
        torch.cuda.synchronize()
        ag_ms = dist.max(e0.elapsed_time(e1) / 3)
        nbytes = full.numel() * full.element_size()
        allgather = {"ms": ag_ms, "bus_gbs": nbytes * (dist.world - 1) / dist.world / (ag_ms * 1e-3) / 1e9,
                     "includes": "all_gather_into_tensor + head permute"}
        del full
    wl = "gdn_prefill_c3" + ("_fused" if fused else "")
    traffic = _scaled(profile_traffic(wl), Hv_l / Hv)
    if cfg.get("custom"):  # a shape of its own: the C3 summaries do not describe it
        wl, traffic = wl.replace("_c3", "") + "_custom", None
    res = {"metric": "GDN prefill tok/s", "value": T / (ms * 1e-3), "unit": "tok/s",
           "us_per_step": ms * 1e3,
           "config": {"workload": wl, "B": 1, "T": T, "Hqk": Hqk, "Hv": Hv, "d": d,
                      "chunk": 64, "sharding": "v-heads", "l2": "L2 flushed between launches"},
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / peaks["hbm_gbs"],
                        "traffic": traffic,
                        "tensor_tflops": flops_local / (ms_local * 1e-3) / 1e12},
           "gpu_launches": int(launches), "clocks": clk.summary()}
    if allgather:
        res["allgather"] = allgather
    del q, k, v, g, b, state, out, ws, flush
    torch.cuda.empty_cache()
    return res


# ----------------------------------------------------------------------------
# CPU side: the fp64 oracle restatement timed on this host
# ----------------------------------------------------------------------------
def cpu_attention_sample(cfg, budget_s, threads=0):
    """Times the oracle on rows of one (b, h) head; returns (TFLOP/s, cores, description)."""
    import numpy as np
    import torch
    import oracle
    import workloads

    S, D = cfg["S"], cfg["D"]
    Q, K, V = workloads.attn_inputs(1, 1, 1, S, D, cfg["dtype"], seed=42, device="cpu")
    q, k, v = (t.float().numpy() for t in (Q, K, V))
    cores = threads or oracle.default_threads()

    def rows_flops(rows):
        if cfg["causal"]:
            return float(sum(4.0 * (r + 1) * D for r in rows))
        return 4.0 * len(rows) * S * D

    probe = list(range(0, S, max(1, S // 256)))
    t0 = time.perf_counter()
    oracle.attn_fwd(q, k, v, 1 / math.sqrt(D), cfg["causal"], rows=probe, nthreads=threads)
    rate = rows_flops(probe) / max(time.perf_counter() - t0, 1e-6)
    full = rows_flops(range(S))
    frac = min(1.0, budget_s * rate / full)
    stride = max(1, int(round(1 / frac)))
    rows = list(range(0, S, stride))
    t0 = time.perf_counter()
    oracle.attn_fwd(q, k, v, 1 / math.sqrt(D), cfg["causal"], rows=rows, nthreads=threads)
    dt = time.perf_counter() - t0
    fl = rows_flops(rows)
    desc = (f"fp64 oracle (restated naive_attn_kernel), 1 of {cfg['B'] * cfg['Hq']} heads, "
            f"{len(rows)} of {S} query rows (every {stride}th), {fl:.3g} FLOP in {dt:.1f} s")
    return fl / dt / 1e12, cores, desc, rows, q, k, v


def cpu_gdn_prefill(cfg, threads=0):
    import numpy as np
    import oracle
    import workloads
    T, Hqk, Hv, d = cfg["T"], cfg["Hqk"], cfg["Hv"], cfg["d"]
    q, k, v, g, b = workloads.gdn_inputs(1, T, Hqk, Hv, d, cfg["dtype"], seed=7)
    arr = [t.float().numpy() for t in (q, k, v, g, b)]
    t0 = time.perf_counter()
    oracle.gdn_recurrent(*arr, np.zeros((1, Hv, d, d)), 1 / math.sqrt(d), 0, nthreads=threads)
    dt = time.perf_counter() - t0
    return {"value": T / dt, "unit": "tok/s", "cores": threads or oracle.default_threads(),
            "kind": "port", "sample": f"full config, fp64 serial recurrence, {dt:.2f} s"}


def cpu_ref_gdn_cpu(T=64):
    """The reference's own fp32 single-thread gdn_cpu (src/gdn_sm75.cu:1078-1106), compiled
    from its sources into oracle/_ref, timed at its own shape (Hq16 Hv48 d128) and LCG
    inputs: a second, labelled CPU figure beside the fp64 port."""
    import oracle
    if not oracle.ref_gdn_available():
        return {"status": "oracle/_ref not built"}
    q, k, v, g, b = oracle.ref_lcg_gdn_inputs(T)
    Sv, Hq, Hv, _ = oracle.ref_gdn_shape()
    import numpy as np
    state = np.zeros((Hv, Sv, Sv), dtype=np.float32)
    t0 = time.perf_counter()
    oracle.ref_gdn_run(q, k, v, g, b, state, T, 1 / math.sqrt(Sv))
    dt = time.perf_counter() - t0
    return {"value": T / dt, "unit": "tok/s", "cores": 1, "kind": "reference",
            "sample": f"reference gdn_cpu, T={T} at its own shape Hq{Hq} Hv{Hv} d{Sv}, fp32, "
                      f"{dt:.3f} s"}


def cpu_gdn_decode(cfg, threads=0):
    import numpy as np
    import oracle
    import workloads
    B, Hqk, Hv, d = cfg["B"], cfg["Hqk"], cfg["Hv"], cfg["d"]
    q, k, v, g, b = workloads.gdn_decode_inputs(B, Hqk, Hv, d, cfg["dtype"], seed=11)
    arr = [t.float().numpy()[:, None] for t in (q, k, v, g, b)]
    S = workloads.gdn_state(B, Hv, d).double().numpy()
    t0 = time.perf_counter()
    oracle.gdn_recurrent(*arr, S, 1 / math.sqrt(d), 0, nthreads=threads)
    dt = time.perf_counter() - t0
    nbytes = B * Hv * d * d * 4 * 2 + B * Hqk * d * 4 + B * Hv * d * 4 + B * Hv * 8
    return {"value": nbytes / dt / 1e9, "unit": "GB/s (fp32-state bytes)",
            "cores": threads or oracle.default_threads(), "kind": "port",
            "sample": f"1 of 256 steps, fp64 serial recurrence, {dt:.2f} s"}


# ----------------------------------------------------------------------------
# arms
# ----------------------------------------------------------------------------
def run_reference(args):
    """CPU implementation of the path on this host, same config/metric as our arm."""
    import workloads
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    cfg = workloads.CONFIGS.get(args.workload) if args.workload.startswith("attn") else None
    cfg = cfg or workloads.CONFIGS["attn_c5"]
    budget = max(0.5, args.cpu_budget_s / max(1, args.steps + args.warmup))
    vals = []
    desc = cores = None
    for i in range(args.warmup + args.steps):
        v, cores, desc, *_ = cpu_attention_sample(cfg, budget)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.mean(vals)
    return {"metric": BASELINE_METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": {"workload": args.workload, "B": cfg["B"],
                                            "Hq": cfg["Hq"], "Hkv": cfg["Hkv"], "S": cfg["S"],
                                            "D": cfg["D"], "causal": cfg["causal"]},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "the reference has no CPU attention; its naive_attn_kernel "
                    "(src/attn_sm75.cu:55-94) restated in fp64 C (oracle/) runs on the host cores"}


def run_ours(args):
    import torch
    import workloads

    dist = Dist(args.gpus)
    dist.init()
    peaks, peaks_src = load_peaks()
    name = args.workload
    if name in ATTN_CASES and name != "attn_c1":
        # one secondary attention shape alone, as its bench line measures it
        cfgname = "attn_c5"
    else:
        cfgname = None
    cfgname = cfgname or {"attn_c2": "attn_c2_d128", "gdn_decode": "gdn_decode_c4", "gdn_decode_state16": "gdn_decode_c4",
               "gdn_prefill": "gdn_prefill_c3", "gdn_prefill_fused": "gdn_prefill_c3"}.get(name, name)
    cfg = dict(workloads.CONFIGS[cfgname])
    if args.attn_shape:
        # smaller instance of the same kernel, for ncu captures that must stay small
        cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["S"], cfg["D"] = (int(x) for x in args.attn_shape.split(","))
        name = name + "_custom"
    if args.gdn_shape:
        cfg["T"], cfg["Hqk"], cfg["Hv"] = (int(x) for x in args.gdn_shape.split(","))
        cfg["custom"] = True
    if name in ATTN_CASES and name != "attn_c1":
        main = bench_attn_case(name, ATTN_CASES[name], args, dist, peaks)
    elif name.startswith("attn_gated"):
        main = bench_gated_attention(cfg, args, dist, peaks)
    elif name.startswith("attn"):
        main = bench_attention(name, cfg, args, dist, peaks)
    elif name == "gdn_decode":
        main = bench_gdn_decode(cfg, args, dist, peaks)
    elif name == "gdn_decode_state16":
        main = bench_gdn_decode(cfg, args, dist, peaks, state_dtype=torch.float16)
    elif name == "gdn_prefill_fused":
        main = bench_gdn_prefill(cfg, args, dist, peaks, fused=True)
    else:
        main = bench_gdn_prefill(cfg, args, dist, peaks)

    secondary = {}
    if args.secondary and name == "attn_c5" and not args.attn_shape:
        import torch
        state16 = lambda c, a, d_, p: bench_gdn_decode(c, a, d_, p, state_dtype=torch.float16)  # noqa: E731
        weak = lambda c, a, d_, p: bench_gdn_decode(c, a, d_, p, weak=True)  # noqa: E731
        fused = lambda c, a, d_, p: bench_gdn_prefill(c, a, d_, p, fused=True)  # noqa: E731
        todo = [("gdn_decode", bench_gdn_decode, workloads.CONFIGS["gdn_decode_c4"]),
                ("gdn_decode_state16", state16, workloads.CONFIGS["gdn_decode_c4"]),
                ("attn_gated_d256", bench_gated_attention, workloads.CONFIGS["attn_gated_d256"]),
                ("gdn_prefill", bench_gdn_prefill, workloads.CONFIGS["gdn_prefill_c3"]),
                ("gdn_prefill_fused", fused, workloads.CONFIGS["gdn_prefill_c3"])]
        if dist.world > 1:  # at N = 1 the weak-scaling decodes are the decode lines themselves
            todo.insert(1, ("gdn_decode_weak", weak, workloads.CONFIGS["gdn_decode_c4"]))
            weak16 = lambda c, a, d_, p: bench_gdn_decode(c, a, d_, p, state_dtype=torch.float16,  # noqa: E731
                                                          weak=True)
            todo.insert(3, ("gdn_decode_state16_weak", weak16, workloads.CONFIGS["gdn_decode_c4"]))
        for key, shp in ATTN_CASES.items():
            todo.append((key, lambda c, a, d_, p, key=key: bench_attn_case(key, c, a, d_, p), shp))
        for key, fn, c in todo:
            try:
                secondary[key] = fn(c, args, dist, peaks)
            except Exception as e:  # report, keep the headline line
                secondary[key] = {"status": f"error: {e!r}"}

    line = None
    if dist.rank == 0:
        line = {"metric": main.pop("metric"), "value": main.pop("value"), "unit": main.pop("unit"),
                "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup}
        line["ms_per_step"] = main.pop("ms_per_step", None) or main.get("us_per_step", 0) / 1e3
        line.update({"higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                     "data": "synthetic (seeded torch.Generator, config distributions)"})
        line.update(main)
        line["roofline"]["peak_source"] = f"{peaks_src} (MEASURED_PEAKS.json)" \
            if peaks_src == "measured" else "fallback (recipe constants)"
        if dist.world == 1 and name.startswith("attn") and not args.no_cpu:
            v, cores, desc, *_ = cpu_attention_sample(cfg, args.cpu_budget_s / 4)
            line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                    "sample": desc}
        if secondary:
            if dist.world == 1 and not args.no_cpu:
                for key, fn, c in (("gdn_decode", cpu_gdn_decode, workloads.CONFIGS["gdn_decode_c4"]),
                                   ("gdn_prefill", cpu_gdn_prefill, workloads.CONFIGS["gdn_prefill_c3"])):
                    if "value" in secondary.get(key, {}):
                        try:
                            secondary[key]["cpu_baseline"] = fn(c)
                        except Exception as e:
                            secondary[key]["cpu_baseline"] = {"status": repr(e)}
                if "value" in secondary.get("gdn_prefill", {}):
                    try:
                        secondary["gdn_prefill"]["cpu_baseline_reference"] = cpu_ref_gdn_cpu()
                    except Exception as e:
                        secondary["gdn_prefill"]["cpu_baseline_reference"] = {"status": repr(e)}
            line["secondary"] = secondary
        # last key of the line: a compact digest of every figure above, so that a reader who
        # keeps only the end of the output still sees them all
        line["summary"] = summary_of(line)
    dist.close()
    return line


def summary_of(line):
    """{name: [value, roofline frac]} for the headline and every secondary line, plus the
    end-to-end, copy-floor and all-gather figures, rounded to 4 significant digits."""
    def r(x):
        return None if x is None else float(f"{x:.4g}")

    out = {"n": line["n_gpus"], line["config"]["workload"]: [r(line["value"]), r(line["roofline"]["frac"])]}
    e2e = line.get("e2e", {})
    if "value" in e2e:
        out["e2e"] = [r(e2e["value"]), r(e2e.get("ms_per_step")), r(e2e.get("copy_floor_ms"))]
    if "allgather" in line:
        out["allgather"] = [r(line["allgather"]["ms"]), r(line["allgather"].get("bus_gbs"))]
    for key, sec in line.get("secondary", {}).items():
        if "value" not in sec:
            out[key] = sec.get("status", "no value")[:60]
            continue
        out[key] = [r(sec["value"]), r(sec.get("roofline", {}).get("frac"))]
        if "allgather" in sec:
            out[key + "_allgather"] = [r(sec["allgather"]["ms"]), r(sec["allgather"].get("bus_gbs"))]
    out["units"] = "[value in the line's unit, roofline frac]; e2e [TFLOP/s, ms, copy-floor ms]; " \
                   "allgather [ms, bus GB/s]"
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="attn_c5",
                    choices=["attn_c5", "attn_c1", "attn_c2", "attn_gated_d256", "gdn_decode",
                             "gdn_decode_state16", "gdn_prefill", "gdn_prefill_fused"] + [
                                 k for k in ATTN_CASES if k not in ("attn_c1",)],
                    help="the headline (attn_c5) or one secondary workload alone (for profiling)")
    ap.add_argument("--no-secondary", dest="secondary", action="store_false")
    ap.add_argument("--attn-shape", default=None, metavar="B,Hq,Hkv,S,D",
                    help="override the attention shape (profiling a smaller case)")
    ap.add_argument("--gdn-shape", default=None, metavar="T,Hqk,Hv",
                    help="override the GDN prefill shape (e.g. one GPU's share of C3 on 8 GPUs: "
                         "4096,2,4)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--cpu-budget-s", type=float, default=60.0,
                    help="approximate CPU seconds for the reference arm / cpu_baseline")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    line = run_reference(args) if args.impl == "reference" else run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
