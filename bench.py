#!/usr/bin/env python
"""Benchmark of the depthwise causal conv1d hot path on B200.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-paths]
python bench.py --profile fwd|decode|ring|spec|varlen   (4 launches of one kernel, for ncu)

Headline (the configuration the metric is quoted on): prefill of
x (batch 8, seqlen 4096, dim 8192) bf16 ~N(0,1) stored token-major and passed as its
(batch, dim, seqlen) view, weight (8192, 4) ~U(-0.5, 0.5), bias ~N(0, 0.1), SiLU. One step is one
causal_conv1d_fn call over that batch. value = algorithmic bytes (every input element read once,
every output element written once, plus weights and bias) / device time, summed over ranks.
Inputs (512 MiB) exceed L2 (126 MB), so no flush is needed between steps. e2e is the same
metric with the input in pinned host memory and the result read back to it inside every step:
the public causal_conv1d_fn is called once per 1024-token chunk of each batch row (over a window
that starts W - 1 tokens earlier, so each output has its full history), and chunks are pipelined
over three streams (upload of chunk i + 1, convolution of chunk i, download of chunk i - 1).

At N > 1 (torchrun, one rank per GPU) the layer is channel-sliced as tensor parallelism shards it:
rank r owns channels [8192 r, 8192 (r + 1)) of a layer with 8192 N channels, so per-GPU work is
fixed (weak scaling) and the kernels exchange nothing. NCCL is used once, after timing, to
all-gather a sample of every rank's outputs and compare them bit for bit with the unsharded run.

With N = 1 the other BASELINE paths are measured too ("paths"): config 2 stored channel-first,
config 2 with initial and final states and with sequence ids (the Dao-interface extras), indexed
decode (config 3) and its ring variant with the to_ring / from_ring conversions, direct-state
decode at B = 256 and 64 and ring decode at B = 64 (the shapes of the reference's published
decode numbers), the 4-step speculative verify with dense per-step states (config 4), and packed
varlen prefill (config 5) at widths 2, 3, 4 and 8, token-major and channel-first, each replayed in
a CUDA graph (no host launch gaps). Decode inputs fit in L2, so "cold" cycles 8 independent input sets whose total
exceeds L2, and "warm" repeats one set.

--impl reference times the reference's CPU algorithm (the C port of its PyTorch fallback,
oracle/cc1d_oracle.c) on the host cores, on bounded samples of the same workload.
"""

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT / "causal-conv1d-cute_b200"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "prefill/varlen achieved HBM GB/s vs ~8 TB/s; decode µs/call at bs=256"
B, L, D, W = 8, 4096, 8192, 4
E = 2  # bf16
HEADLINE_BYTES = 2 * B * L * D * E + D * W * E + D * E  # 1,073,823,744
# The kernel the headline call dispatches to (balanced shares: W = 4, 4096-token sequences).
HEADLINE_KERNEL = "fwd_channel_last_share_kernel"
L2_BYTES = 126 * 2**20
E2E_CHUNKS = 4  # token chunks per batch row in the e2e pipeline


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-paths", action="store_true")
    p.add_argument("--profile", choices=("fwd", "fwd_cf", "decode", "ring", "spec", "varlen", "varlen_cf"),
                   default=None,
                   help="run 4 launches of one kernel on a case larger than L2 (for ncu) and exit")
    p.add_argument("--width", type=int, default=W,
                   help="filter width of the --profile case (prefill and varlen cases)")
    return p.parse_args()


# ---------------------------------------------------------------------------------------------
# Peaks, clocks, profiles
# ---------------------------------------------------------------------------------------------


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(kernel):
    """dram bytes per launch of `kernel` recorded in profiles/*.md ("traffic_bytes_per_launch")."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        kname = None
        for line in f.read_text().splitlines():
            if line.startswith("kernel:"):
                kname = line.split(":", 1)[1].strip()
            if line.startswith("traffic_bytes_per_launch:") and kname == kernel:
                return int(float(line.split(":", 1)[1].strip()))
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML on a background thread."""

    REASONS = {
        "hw_slowdown": 0x8,
        "hw_thermal_slowdown": 0x40,
        "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index, period=0.01):
        self.samples = []
        self.period = period
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    handle = h
            if handle is None:
                handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nvml, self.handle = pynvml, handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.error = str(e)

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                util = n.nvmlDeviceGetUtilizationRates(self.handle).gpu
                self.samples.append((mhz, reasons, util))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.error}
        busy = [s for s in self.samples if s[2] > 0] or self.samples
        mhz = [s[0] for s in busy]
        seen = set()
        for s in busy:
            for name, bit in self.REASONS.items():
                if s[1] & bit:
                    seen.add(name)
        return {
            "sm_mhz": statistics.median(mhz) if mhz else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(seen),
            "samples": len(busy),
        }


# ---------------------------------------------------------------------------------------------
# Timing helpers
# ---------------------------------------------------------------------------------------------


def time_launches(step, steps, flush=None):
    """Run `step` `steps` times on the current stream; return (total ms, per-launch ms list).

    Each launch is bracketed by its own CUDA events (so a cold-L2 flush issued between launches is
    not counted); the total spans the first start to the last end.
    """
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return starts[0].elapsed_time(ends[-1]), per


# ---------------------------------------------------------------------------------------------
# Headline: prefill config 2
# ---------------------------------------------------------------------------------------------


def make_prefill(device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(B, L, D, device=device, dtype=torch.bfloat16, generator=g)
    w = (torch.rand(D, W, device=device, generator=g) - 0.5).to(torch.bfloat16)
    b = (torch.randn(D, device=device, generator=g) * 0.1).to(torch.bfloat16)
    return x, w, b


def run_headline(args, rank, world, device):
    import causal_conv1d_cute as C

    x, w, bias = make_prefill(device, 1234 + rank)
    xv = x.transpose(1, 2)  # (B, D, L) channel-last view
    out = torch.empty(B, L, D, device=device, dtype=torch.bfloat16).transpose(1, 2)

    def step():
        C.causal_conv1d_fn(xv, w, bias, "silu", out=out)

    for _ in range(args.warmup):
        step()
    dist_barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(device.index)
    with sampler:
        total_ms, per = time_launches(step, args.steps)
    total_ms = allreduce_max(total_ms, world, device)
    avg_launch_ms = statistics.mean(per)

    # End to end through the public API: pinned host input in, result back to pinned host memory.
    # Every batch row is cut into E2E_CHUNKS token chunks, pipelined over three streams: chunk
    # i + 1 uploads while chunk i is convolved and chunk i - 1 downloads (PCIe carries both
    # directions at once; more, smaller chunks shorten the pipeline's fill and drain). Chunk k > 0
    # of a row is convolved over the window that starts W - 1 tokens earlier (already on the
    # device), into its own output buffer whose first W - 1 rows are discarded, so every output is
    # computed from its full history. Every step moves the whole input in and the whole result
    # out; the step ends when the last chunk is back on the host.
    Lc = L // E2E_CHUNKS
    xh = torch.empty(B, L, D, dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(x)
    oh = torch.empty(B, L, D, dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    yc = torch.empty(B, E2E_CHUNKS, Lc + W - 1, D, device=device, dtype=torch.bfloat16)
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))

    def e2e_step():
        main = torch.cuda.current_stream(device)
        start = torch.cuda.Event()
        start.record(main)
        for s_ in (s_in, s_cmp, s_out):
            s_.wait_event(start)
        for i in range(B):
            for k in range(E2E_CHUNKS):
                t0, t1 = k * Lc, (k + 1) * Lc
                with torch.cuda.stream(s_in):
                    xd[i, t0:t1].copy_(xh[i, t0:t1], non_blocking=True)
                    up = torch.cuda.Event()
                    up.record(s_in)
                s_cmp.wait_event(up)
                with torch.cuda.stream(s_cmp):
                    lo = max(t0 - (W - 1), 0)
                    dst = yc[i, k, W - 1 - (t0 - lo):]
                    C.causal_conv1d_fn(xd[i : i + 1, lo:t1].transpose(1, 2), w, bias, "silu",
                                       out=dst.unsqueeze(0).transpose(1, 2))
                    done = torch.cuda.Event()
                    done.record(s_cmp)
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    oh[i, t0:t1].copy_(yc[i, k, W - 1:], non_blocking=True)
        main.wait_stream(s_out)

    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 10))
    dist_barrier(world)
    torch.cuda.synchronize()
    e2e_ms, _ = time_launches(e2e_step, e2e_steps)
    e2e_ms = allreduce_max(e2e_ms, world, device)
    torch.cuda.synchronize()
    # The result read back must equal the device result.
    assert torch.equal(oh.to(device), out.transpose(1, 2))

    value = HEADLINE_BYTES * world * args.steps / (total_ms / 1e3) / 1e9
    e2e_value = HEADLINE_BYTES * world * e2e_steps / (e2e_ms / 1e3) / 1e9
    achieved = HEADLINE_BYTES / (avg_launch_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    traffic = profiled_traffic(HEADLINE_KERNEL)
    return {
        "value": value,
        "ms_per_step": total_ms / args.steps,
        "e2e": {
            "value": e2e_value,
            "unit": "GB/s",
            "h2d_bytes_per_step": xh.numel() * xh.element_size(),
            "d2h_bytes_per_step": oh.numel() * oh.element_size(),
            "ms_per_step": e2e_ms / e2e_steps,
        },
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic,
            "peak_source": f"{peak_kind} hbm_gbs (copy, burst)",
            "kernel": HEADLINE_KERNEL,
            "algorithmic_bytes_per_launch": HEADLINE_BYTES,
            "avg_launch_us": avg_launch_ms * 1e3,
        },
        "clocks": sampler.summary(),
        "gpu_launches": args.steps,
    }


# ---------------------------------------------------------------------------------------------
# Other BASELINE paths (N = 1)
# ---------------------------------------------------------------------------------------------


def _median_us(per_ms):
    return statistics.median(per_ms) * 1e3


def graph_us(calls, reps):
    """Microseconds per call of `calls` (one callable per input set) replayed in a CUDA graph.

    All calls are captured once, back to back, and the graph is replayed `reps` times between two
    events, so host launch overhead is excluded and every call follows the previous one as it
    would inside a captured serving step.
    """
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for f in calls:
            f()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in calls:
            f()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / (reps * len(calls))


def run_paths(device, reps=50, sets=8):
    """Decode paths: `sets` independent input sets (together larger than L2) are cycled, so each
    call reads cold data ("cold"); "warm" repeats one set. Varlen inputs exceed L2 by themselves."""
    import causal_conv1d_cute as C

    g = torch.Generator(device=device).manual_seed(7)
    bf = torch.bfloat16
    res = {}
    w4 = (torch.rand(D, 4, device=device, generator=g) - 0.5).to(bf)
    bias = (torch.randn(D, device=device, generator=g) * 0.1).to(bf)

    def record(name, calls, nbytes, extra=None):
        cold = graph_us(calls, reps)
        warm = graph_us(calls[:1] * len(calls), reps)
        res[name] = {"us_cold": cold, "us_warm": warm, "bytes": nbytes,
                     "gbs_cold": nbytes / (cold * 1e3), **(extra or {})}

    # Config 2 stored channel-first: contiguous (8, 8192, 4096) (the reference's "bdl" layout).
    xcf = torch.randn(B, D, L, device=device, generator=g).to(bf)
    ocf = torch.empty_like(xcf)
    us = graph_us([lambda: C.causal_conv1d_fn(xcf, w4, bias, "silu", out=ocf)], 20)
    res["prefill_channel_first"] = {"us": us, "bytes": HEADLINE_BYTES, "gbs": HEADLINE_BYTES / (us * 1e3)}
    del xcf, ocf

    # Config 2 with the Dao-interface extras: initial states in, final states out (channel-last
    # states, as upstream allocates them). Algorithmic bytes add 2 * B * D * 3 elements.
    xs = torch.randn(B, L, D, device=device, generator=g).to(bf).transpose(1, 2)
    init = torch.randn(B, 3, D, device=device, generator=g).to(bf).transpose(1, 2)
    fin = torch.empty_like(init)
    nbytes = HEADLINE_BYTES + 2 * B * D * 3 * 2
    us = graph_us([lambda: C.causal_conv1d_fwd_states(xs, w4, bias, None, init, True, fin, "silu")], 20)
    res["prefill_states"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e3)}
    seq = torch.zeros(B, L, device=device, dtype=torch.int32)
    seq[:, L // 2:] = 1
    us = graph_us([lambda: C.causal_conv1d_fwd_states(xs, w4, bias, seq, None, False, None, "silu")], 20)
    nbytes = HEADLINE_BYTES + B * L * 4
    res["prefill_seq_idx"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e3)}
    del xs, init, fin, seq

    # Config 3: single-token indexed decode, B=256, 1024-slot cache (48 MiB per set).
    Bd, slots = 256, 1024
    calls = []
    for _ in range(sets):
        x = torch.randn(Bd, D, device=device, generator=g).to(bf)
        cache = torch.randn(slots, D, 3, device=device, generator=g).to(bf)
        idx = torch.randperm(slots, device=device, generator=g)[:Bd].to(torch.int32)
        calls.append(lambda x=x, cache=cache, idx=idx: C.causal_conv1d_update(x, cache, w4, bias, "silu", idx))
    nbytes = 2 * Bd * D * 2 + 2 * Bd * D * 3 * 2 + D * 4 * 2 + D * 2 + Bd * 4
    record("decode_indexed_b256", calls, nbytes)

    # The reference's published decode shapes (B300): direct (non-indexed) state at B = 256 and
    # B = 64, and ring decode at B = 64, for a like-for-like comparison.
    for Bq in (256, 64):
        calls = []
        for _ in range(sets):
            x = torch.randn(Bq, D, device=device, generator=g).to(bf)
            st = torch.randn(Bq, D, 3, device=device, generator=g).to(bf)
            calls.append(lambda x=x, st=st: C.causal_conv1d_update(x, st, w4, bias, "silu"))
        nbytes = 2 * Bq * D * 2 + 2 * Bq * D * 3 * 2 + D * 4 * 2 + D * 2
        record(f"decode_direct_b{Bq}", calls, nbytes)
    calls = []
    for _ in range(sets):
        x = torch.randn(64, D, device=device, generator=g).to(bf)
        ring = torch.randn(64, 3, D, device=device, generator=g).to(bf)
        seen = torch.randint(1, 8193, (64,), device=device, generator=g, dtype=torch.int32)
        calls.append(lambda x=x, ring=ring, seen=seen: C.causal_conv1d_update_ring(x, ring, w4, bias, "silu", seen))
    record("decode_ring_b64", calls, 2 * 64 * D * 2 + 4 * 64 * D * 2 + D * 4 * 2 + D * 2 + 64 * 4)

    # Config 3 ring variant: ring (256, 3, 8192), seen ~U[1, 8192].
    calls = []
    for _ in range(sets):
        x = torch.randn(Bd, D, device=device, generator=g).to(bf)
        ring = torch.randn(Bd, 3, D, device=device, generator=g).to(bf)
        seen = torch.randint(1, 8193, (Bd,), device=device, generator=g, dtype=torch.int32)
        calls.append(lambda x=x, ring=ring, seen=seen: C.causal_conv1d_update_ring(x, ring, w4, bias, "silu", seen))
    nbytes = 2 * Bd * D * 2 + 3 * Bd * D * 2 + Bd * D * 2 + D * 4 * 2 + D * 2 + Bd * 4
    record("decode_ring_b256", calls, nbytes)

    # Ring layout conversions at the config-3 ring shape (the state a prefill hands to ring
    # decode, and back): read and write 256 x 8192 x 3 elements each.
    to_calls, from_calls = [], []
    for _ in range(sets):
        st = torch.randn(Bd, D, 3, device=device, generator=g).to(bf)
        ring = torch.randn(Bd, 3, D, device=device, generator=g).to(bf)
        seen = torch.randint(1, 8193, (Bd,), device=device, generator=g, dtype=torch.int32)
        to_calls.append(lambda st=st, seen=seen: C.to_ring(st, seen))
        from_calls.append(lambda ring=ring, seen=seen: C.from_ring(ring, seen))
    nbytes = 2 * Bd * D * 3 * 2 + Bd * 4
    record("to_ring_b256", to_calls, nbytes)
    record("from_ring_b256", from_calls, nbytes)

    # Config 4: spec-decode verify, B=64, 4 steps, dense per-step states.
    Bs, S = 64, 4
    calls = []
    for _ in range(sets):
        xs = torch.randn(Bs, S, D, device=device, generator=g).to(bf).transpose(1, 2)
        st = torch.randn(Bs, D, 3, device=device, generator=g).to(bf)
        inter = torch.empty(Bs, S, D, 3, device=device, dtype=bf)
        perm = torch.randperm(Bs, device=device, generator=g).to(torch.int32)
        calls.append(lambda xs=xs, st=st, inter=inter, perm=perm:
                     C.causal_conv1d_update(xs, st, w4, bias, "silu", perm, -1, inter, perm))
    nbytes = 2 * Bs * S * D * 2 + 2 * Bs * D * 3 * 2 + Bs * S * D * 3 * 2 + D * 4 * 2 + D * 2 + 2 * Bs * 4
    record("spec_decode_b64_s4", calls, nbytes)

    # Config 5: varlen, 32 lognormal(7, 1) lengths clipped to [1, 8192], token-major x, and the
    # same batch stored channel-first.
    rng = np.random.default_rng(0)
    lens = np.clip(np.round(rng.lognormal(7, 1, 32)), 1, 8192).astype(np.int64)
    T = int(lens.sum())
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device=device, dtype=torch.int32)
    cidx = torch.from_numpy(rng.choice(512, 32, replace=False).astype(np.int32)).to(device)
    hinit = torch.from_numpy(rng.random(32) < 0.5).to(device)
    xv = torch.randn(T, D, device=device, generator=g).to(bf)
    xc = xv.t().contiguous()
    for Wv in (2, 3, 4, 8):
        wv = (torch.rand(D, Wv, device=device, generator=g) - 0.5).to(bf)
        states = torch.randn(512, D, Wv - 1, device=device, generator=g).to(bf)
        nh = int(hinit.sum())
        nbytes = 2 * D * T * 2 + D * (Wv - 1) * 2 * (32 + nh) + 4 * 33 + 4 * 32 + 32 + D * Wv * 2
        f = lambda wv=wv, states=states: C.causal_conv1d_varlen_fn(xv.t(), wv, None, qsl, cidx, hinit, states, "silu")  # noqa: E731
        us = graph_us([f], 20)
        res[f"varlen_w{Wv}"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e3), "tokens": T}
        # The same batch stored channel-first: contiguous (8192, T).
        fc = lambda wv=wv, states=states: C.causal_conv1d_varlen_fn(xc, wv, None, qsl, cidx, hinit, states, "silu")  # noqa: E731
        us = graph_us([fc], 20)
        res[f"varlen_w{Wv}_channel_first"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e3),
                                             "tokens": T}
    del xc
    return res


# ---------------------------------------------------------------------------------------------
# CPU baseline (the C port of the reference's fallback)
# ---------------------------------------------------------------------------------------------


def cpu_baseline(min_seconds=10.0):
    from oracle import native

    rng = np.random.default_rng(0)
    Ls = 256
    x = (rng.standard_normal((1, Ls, D)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    w = (rng.uniform(-0.5, 0.5, (D, W)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    b = (rng.standard_normal(D).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    native.fwd_cl_bf16(x, w, b, True)
    t0 = time.perf_counter()
    n = 0
    while True:
        native.fwd_cl_bf16(x, w, b, True)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    sample_bytes = 2 * Ls * D * E + D * W * E + D * E
    return {
        "value": sample_bytes * n / el / 1e9,
        "unit": "GB/s",
        "cores": native.threads(),
        "kind": "port",
        "sample": f"{n} calls of batch 1 x {Ls} tokens x {D} channels (W=4, bias, SiLU) of the "
                  f"config-2 workload, {el:.1f} s, oracle/cc1d_oracle.c with OpenMP",
    }


# ---------------------------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------------------------


def dist_barrier(world):
    if world > 1:
        torch.distributed.barrier()


def allreduce_max(v, world, device):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sharded_check(rank, world, device):
    """All-gather a sample of every rank's channel slice and compare with the unsharded run."""
    import causal_conv1d_cute as C

    Ls, Dg = 128, D * world
    g = torch.Generator(device=device).manual_seed(99)
    xg = torch.randn(1, Ls, Dg, device=device, generator=g).to(torch.bfloat16)
    wg = (torch.rand(Dg, W, device=device, generator=g) - 0.5).to(torch.bfloat16)
    bg = (torch.randn(Dg, device=device, generator=g) * 0.1).to(torch.bfloat16)
    lo, hi = rank * D, (rank + 1) * D
    mine = C.causal_conv1d_fn(xg[:, :, lo:hi].transpose(1, 2), wg[lo:hi], bg[lo:hi], "silu")
    mine = mine.transpose(1, 2).contiguous()
    parts = [torch.empty_like(mine) for _ in range(world)]
    torch.distributed.all_gather(parts, mine)
    ok = True
    if rank == 0:
        full = C.causal_conv1d_fn(xg.transpose(1, 2), wg, bg, "silu").transpose(1, 2)
        ok = torch.equal(torch.cat(parts, dim=2), full)
    flag = torch.tensor([1 if ok else 0], device=device)
    torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
    return bool(flag.item())


def profile_case(case, device, width=W):
    """A few launches of one kernel, sized for an ncu capture (a few hundred MB on the device)."""
    import causal_conv1d_cute as C

    g = torch.Generator(device=device).manual_seed(0)
    bf = torch.bfloat16
    w = (torch.rand(D, width, device=device, generator=g) - 0.5).to(bf)
    b = (torch.randn(D, device=device, generator=g) * 0.1).to(bf)
    if case == "fwd":  # config 2 with batch 2: 128 MiB in, 128 MiB out
        x = torch.randn(2, L, D, device=device, generator=g).to(bf)
        out = torch.empty_like(x).transpose(1, 2)
        calls = [lambda: C.causal_conv1d_fn(x.transpose(1, 2), w, b, "silu", out=out)] * 4
    elif case == "fwd_cf":  # the same batch stored channel-first (2, 8192, 4096) contiguous
        x = torch.randn(2, D, L, device=device, generator=g).to(bf)
        out = torch.empty_like(x)
        calls = [lambda: C.causal_conv1d_fn(x, w, b, "silu", out=out)] * 4
    elif case in ("decode", "ring"):  # config 3, full size
        x = torch.randn(256, D, device=device, generator=g).to(bf)
        if case == "decode":
            cache = torch.randn(1024, D, 3, device=device, generator=g).to(bf)
            idx = torch.randperm(1024, device=device, generator=g)[:256].to(torch.int32)
            calls = [lambda: C.causal_conv1d_update(x, cache, w, b, "silu", idx)] * 4
        else:
            ring = torch.randn(256, 3, D, device=device, generator=g).to(bf)
            seen = torch.randint(1, 8193, (256,), device=device, generator=g, dtype=torch.int32)
            calls = [lambda: C.causal_conv1d_update_ring(x, ring, w, b, "silu", seen)] * 4
    elif case == "spec":  # config 4, full size
        xs = torch.randn(64, 4, D, device=device, generator=g).to(bf).transpose(1, 2)
        st = torch.randn(64, D, 3, device=device, generator=g).to(bf)
        inter = torch.empty(64, 4, D, 3, device=device, dtype=bf)
        perm = torch.randperm(64, device=device, generator=g).to(torch.int32)
        calls = [lambda: C.causal_conv1d_update(xs, st, w, b, "silu", perm, -1, inter, perm)] * 4
    else:  # config 5 with 8 of its 32 lognormal sequences
        rng = np.random.default_rng(0)
        lens = np.clip(np.round(rng.lognormal(7, 1, 8)), 1, 8192).astype(np.int64)
        T = int(lens.sum())
        qsl = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device=device, dtype=torch.int32)
        xv = torch.randn(T, D, device=device, generator=g).to(bf)
        if case == "varlen_cf":  # channel-first: contiguous (8192, T); the call gets x = xv.t()
            xv = xv.t().contiguous().t()
        states = torch.randn(64, D, width - 1, device=device, generator=g).to(bf)
        cidx = torch.arange(8, device=device, dtype=torch.int32) * 3
        hinit = torch.ones(8, dtype=torch.bool, device=device)
        calls = [lambda: C.causal_conv1d_varlen_fn(xv.t(), w, None, qsl, cidx, hinit, states, "silu")] * 4
    # An L2-sized write between launches so every captured launch starts cold.
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)
    for f in calls:
        flush.fill_(1)
        f()
    torch.cuda.synchronize()
    print(json.dumps({"profile": case, "launches": len(calls)}))


def main():
    args = parse()
    if args.profile:
        profile_case(args.profile, torch.device("cuda", 0), args.width)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(world, 1)
    config = {
        "workload": "prefill_bf16_channel_last (BASELINE config 2)",
        "batch": B, "seqlen": L, "dim_per_gpu": D, "dim_global": D * n, "width": W,
        "activation": "silu", "bias": True,
        "layout": "x stored (batch, seqlen, dim), passed as its (batch, dim, seqlen) view",
        "l2": "inputs (512 MiB per GPU) larger than L2 (126 MB); no flush",
        "parallelism": f"channel-sliced tp{n}: each rank owns {D} channels, no collective in the path",
    }
    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import native

        steps = max(1, args.steps if args.steps < 50 else 20)
        per_step = []
        for i in range(min(args.warmup, 2) + steps):
            t0 = time.perf_counter()
            cb = cpu_baseline(min_seconds=0.5)
            if i >= min(args.warmup, 2):
                per_step.append(cb["value"])
        v = statistics.median(per_step)
        line = {
            "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": n,
            "steps": steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": native.threads(), "kind": "port",
                             "sample": "each step: batch 1 x 256 tokens x 8192 channels of config 2 "
                                       "for >= 0.5 s, oracle/cc1d_oracle.c (C port of the reference's "
                                       "fallback.py) with OpenMP"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line))
        return

    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    head = run_headline(args, rank, world, device)
    line = {
        "metric": METRIC,
        "value": head["value"],
        "unit": "GB/s",
        "n_gpus": n,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": config,
        "e2e": head["e2e"],
        "roofline": head["roofline"],
        "clocks": head["clocks"],
        "gpu_launches": head["gpu_launches"],
    }
    if world > 1:
        line["sharded_check"] = "bit-identical" if sharded_check(rank, world, device) else "MISMATCH"
    if rank == 0 and n == 1:
        if not args.no_paths:
            line["paths"] = run_paths(device)
        line["cpu_baseline"] = cpu_baseline()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
