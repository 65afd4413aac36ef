"""Benchmark of the per-decode-step history recall (score -> top-k -> residency plan -> stage-in).

Default workload: config 2 of the reference's headline (a 128K-token fp16
history, 64 layers, 24/4 heads, head_dim 256, pages of 256 tokens, top-32 plus
first/last page, stage-in of the selected pages' K and V from pinned host
memory into a device paged cache). One step = one decode step's recall over
all 64 layers, steady state: each step's query favours the next group of
rotating needle pages, so 3 of each layer's 32 pages turn over per step and
are staged (kvmem_b200.synth). Prints one JSON line (rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c1|c3|c4|c5] [--impl ours|reference]

N = 1: the fused step kvm_recall_step (layer chunks; the stage-in of chunk i on
a side stream overlaps the scoring of chunk i + 1).
N > 1 (torchrun, one rank per GPU): the same history partitioned by page range
over the ranks (strong scaling, kvmem_b200.shard.ShardedRecall): local scoring,
two NCCL all-gathers of small tensors per layer chunk, a replicated residency
plan, and each rank's restored pages written from its own pinned records into
the decode GPU's (rank 0's) cache over NVLink; value = token-layers of the
whole history / max-over-ranks time.
Both also report config 5 (a 1M-token q8_0 history, sharded selection) under
"c5_sharded". Config 4 (multi-lane query replay) times selection only on the
tcgen05 scorer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import csv
import ctypes as C
import io
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "select+stage-in ms/decode step @128K; KV tokens scored/s; % HBM roofline"
UNIT = "KV token-layers/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS = 1590.0
PCIE_PEAK_GBS = 63.0  # pcie__read_bytes at 55.7 GB/s read 88.4% of ncu's pcie__throughput peak


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--chunks", type=int, default=8)
    ap.add_argument("--chunks-sharded", type=int, default=4,
                    help="layer chunks of the page-range sharded step (N > 1)")
    ap.add_argument("--graph", action="store_true",
                    help="N > 1: replay the sharded step as one CUDA graph (at N = 2 it measured the same as the "
                         "eager step, 3.19 vs 3.21 ms)")
    ap.add_argument("--shard-exchange", default="lse", choices=["lse", "candidates"],
                    help="N > 1: one all-gather of the page LSE per chunk (lse) or statistics + candidates")
    ap.add_argument("--first-layers", type=int, default=1,
                    help="layers of the step's first chunk (starts the stage-in early)")
    ap.add_argument("--kmirror", default="head", choices=["head", "token"],
                    help="config 4: layout of the resident K score mirror (head-major or the engine's token-major)")
    ap.add_argument("--stage-ctas", type=int, default=128)
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU baseline and the reference GPU timings")
    ap.add_argument("--no-c5", action="store_true", help="skip the config-5 sharded-selection key")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill page-LSE capture key")
    ap.add_argument("--prefill-only", action="store_true",
                    help="time only the prefill page-LSE capture (one GPU) and print its key; for ncu captures")
    ap.add_argument("--prefill-base", type=int, default=36864,
                    help="cached tokens before the 1024-row prompt chunk of the prefill case")
    ap.add_argument("--layers", type=int, default=0, help="override the workload's layer count (profiling)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="time only the page scorer (no host history, no stage-in); for ncu captures")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 100 ms around the timed
    region, for the GPUs of `devices`, through NVML in a thread of this process (a few
    cheap driver queries per sample; `nvidia-smi -lms 200` is the fallback where NVML is
    missing).

    The timed region starts only after the first sample has arrived and the sampler
    keeps running until one sample after the region has arrived, so even a region
    shorter than the sampling period is bracketed by samples; the summary uses the
    samples taken within 250 ms of the region. A multi-rank run samples on rank 0 only,
    all ranks' GPUs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits: SW power cap, HW slowdown, SW thermal, HW thermal
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
    PERIOD_S = 0.1

    def __init__(self, devices, enabled: bool = True):
        # devices: CUDA device ordinals of this node to sample (a multi-rank run samples on
        # rank 0 only; its ranks synchronise after entering the sampler, so the sampler's
        # start-up never delays one rank's timed region against the others')
        self.devices = [devices] if isinstance(devices, int) else list(devices)
        self.enabled = enabled
        self.nvml = self.handles = None
        self.proc = None
        self.thread = None
        self.stop = False
        self.rows = []  # (host time, [index, sm MHz, max MHz, reasons...])
        self.t_begin = self.t_end = 0.0

    def _pci_ids(self):
        import torch
        out = []
        for d in self.devices:
            p = torch.cuda.get_device_properties(d)
            out.append(f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
        return out

    def _sample(self, handles, nvml):
        get_reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        for i, h in enumerate(handles):
            try:
                sm = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
                mx = nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM)
                bits = get_reasons(h)
            except Exception:
                continue
            flags = ["Active" if bits & self.BITS[k] else "Not Active"
                     for k in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")]
            self.rows.append((time.time(), [str(i), str(sm), str(mx), "", hex(bits)] + flags))

    def _nvml_loop(self, handles, nvml):
        while not self.stop:
            self._sample(handles, nvml)
            time.sleep(self.PERIOD_S)

    def _read(self):
        for line in self.proc.stdout:
            r = next(csv.reader([line]), [])
            if len(r) >= 9:
                self.rows.append((time.time(), r))

    _nvml = None  # NVML, initialised once per process (init_nvml), outside every timed region

    @classmethod
    def init_nvml(cls):
        """Initialises NVML once, early: its first initialisation stalled the work that followed
        it for some milliseconds, so it must not happen next to a timed region."""
        if cls._nvml is None:
            try:
                import pynvml as nvml
                nvml.nvmlInit()
                cls._nvml = nvml
            except Exception:
                cls._nvml = False
        return cls._nvml or None

    def _start_nvml(self) -> bool:
        import threading
        nvml = self.init_nvml()
        if nvml is None:
            return False
        try:
            handles = [nvml.nvmlDeviceGetHandleByPciBusId(pid) for pid in self._pci_ids()]
        except Exception:
            return False
        self.nvml, self.handles = nvml, handles
        self.thread = threading.Thread(target=self._nvml_loop, args=(handles, nvml), daemon=True)
        self.thread.start()
        return True

    def _start_smi(self):
        import threading
        try:
            ids = ",".join(self._pci_ids())
        except Exception:
            ids = ",".join(str(d) for d in self.devices)
        self.proc = subprocess.Popen(["nvidia-smi", f"--id={ids}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits", "-lms", "200"],
                                     stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        threading.Thread(target=self._read, daemon=True).start()

    def __enter__(self):
        self.t_begin = time.time()
        if not self.enabled:
            return self
        try:
            if not self._start_nvml():
                self._start_smi()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5.0:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.t_begin = time.time()
        return self

    def __exit__(self, *a):
        self.t_end = time.time()
        if self.thread or self.proc:
            while not any(t >= self.t_end for t, _ in self.rows) and time.time() - self.t_end < 1.0:
                time.sleep(0.01)
        if self.thread:
            self.stop = True
            self.thread.join(timeout=2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        near = [r for t, r in self.rows if self.t_begin - 0.25 <= t <= self.t_end + 0.25]
        rows = near or [r for _, r in self.rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "source": "nvml every 100 ms" if self.thread else "nvidia-smi every 200 ms"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


class NumaLocal:
    """Runs the enclosed host work on the CPU cores nearest to GPU `local` (NVML's affinity
    mask for its PCI address), so pinned host memory first touched there sits on that GPU's
    NUMA node and its PCIe reads do not cross the socket interconnect. Restores the previous
    affinity on exit (the pages stay where they were touched). A no-op where NVML or the
    affinity call is unavailable."""

    def __init__(self, local: int):
        self.local = local
        self.saved = None

    def __enter__(self):
        try:
            import pynvml
            import torch
            p = torch.cuda.get_device_properties(self.local)
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
            n = os.cpu_count() or 1
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
            cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
            allowed = os.sched_getaffinity(0)
            near = cpus & allowed
            if near and near != allowed:
                self.saved = allowed
                os.sched_setaffinity(0, near)
        except Exception:
            self.saved = None
        return self

    def __exit__(self, *a):
        if self.saved:
            try:
                os.sched_setaffinity(0, self.saved)
            except OSError:
                pass


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# --------------------------------------------------------------------------- data

# --------------------------------------------------------------------------- data

def build_history(w, seed, device, need_host=True, page_range=None):
    """K score mirror on the device and (need_host) pinned host K / V page records.

    page_range = (p0, p1): only that range of every layer (a rank of a page-range
    partition), as [L][p1 - p0 pages] on the device and in the records."""
    import torch
    from kvmem_b200 import row_bytes, synth
    rbk = row_bytes(w.k_type, w.head_dim)
    rbv = row_bytes(w.v_type, w.head_dim)
    p0, p1 = page_range or (0, w.pages)
    page_k = w.page_tokens * w.kv_heads * rbk
    page_v = w.page_tokens * w.kv_heads * rbv
    layer_k, layer_v = (p1 - p0) * page_k, (p1 - p0) * page_v
    q_base, drift = synth.make_queries(w, seed, device, drift_steps=max(8, 2 * w.rot_groups))
    k_dev = torch.empty(w.layers * layer_k, dtype=torch.uint8, device=device)
    host_k = host_v = None
    numa = NumaLocal(device.index or 0)
    if need_host:
        with numa:
            host_k = torch.empty(w.layers * layer_k, dtype=torch.uint8, pin_memory=True)
            host_v = torch.empty(w.layers * layer_v, dtype=torch.uint8, pin_memory=True)
    for l in range(w.layers):
        if w.k_type == 1:
            kl = synth.fp16_layer(w, seed, l, q_base, device).view(torch.uint8).reshape(-1)
        else:
            kl = synth.q8_0_layer(w, seed, l, q_base, device).reshape(-1)
        kl = kl[p0 * page_k:p1 * page_k]
        k_dev[l * layer_k:(l + 1) * layer_k].copy_(kl)
        if need_host:
            host_k[l * layer_k:(l + 1) * layer_k].copy_(kl)
            vl = (synth.fp16_v_layer(w, seed, l, device).view(torch.uint8).reshape(-1) if w.v_type == 1
                  else synth.q4_0_v_layer(w, seed, l, device).reshape(-1))
            host_v[l * layer_v:(l + 1) * layer_v].copy_(vl[p0 * page_v:p1 * page_v])
        del kl
    torch.cuda.synchronize()
    return dict(q_base=q_base, drift=drift, k_dev=k_dev, host_k=host_k, host_v=host_v, layer_k=layer_k,
                layer_v=layer_v, rbk=rbk, rbv=rbv, page_k=page_k, page_v=page_v, page0=p0, local_pages=p1 - p0)


def head_major_mirror(w, k_dev):
    """K of every layer re-laid head-major ([layer][kv_head][token][row]): each KV head's
    rows contiguous, so a 128-token tile is one contiguous 32 KiB run in HBM. Returns the
    mirror and its kvm_kcache."""
    import kvmem_b200 as K
    from kvmem_b200 import _abi as A
    rb = K.row_bytes(w.k_type, w.head_dim)
    T = w.pages * w.page_tokens
    mirror = k_dev.view(w.layers, T, w.kv_heads, rb).permute(0, 2, 1, 3).contiguous()
    kc = A.KCache()
    kc.data, kc.type = mirror.data_ptr(), w.k_type
    kc.token_stride, kc.head_stride, kc.layer_stride = rb, T * rb, w.kv_heads * T * rb
    kc.capacity_tokens = T
    return mirror, kc


def workload(args):
    import dataclasses
    from kvmem_b200 import synth
    w = synth.CONFIGS[args.config]
    if args.layers:
        w = dataclasses.replace(w, layers=args.layers)
    return w


def cpu_info():
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return model, os.cpu_count() or 1


def traffic_of(config):
    """DRAM bytes per scorer launch from the committed ncu summary, with its source."""
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(tp) as f:
            t = json.load(f)
        return t.get(f"page_lse_{config}"), "profiles/traffic.json: " + str(t.get("note"))
    except Exception:
        return None, None


def step_stats(w, ctx, desc, kc, qdescs, start, count, mass, sel_ids, sel_n, chunks):
    """Pages restored per step under the step-to-step query change: selection-only replays of
    `count` consecutive steps (the pool holds exactly the previous step's selection, so the
    restores of a step are its selected pages not selected the step before)."""
    import numpy as np
    restored, prev = [], None
    srows = w.layers * w.groups
    for i in range(start, start + count + 1):
        ctx.recall_step(desc, qdescs[i % len(qdescs)], kc, w.keep, w.budget, mass_mean=mass, sel_ids=sel_ids,
                        sel_n=sel_n, chunks=chunks)
        ids, n = sel_ids.cpu().numpy(), sel_n.cpu().numpy()
        cur = [set(ids[r, : n[r]].tolist()) for r in range(srows)]
        if prev is not None:
            restored.append(sum(len(c - p) for c, p in zip(cur, prev)))
        prev = cur
    return float(np.mean(restored)) if restored else 0.0


def run_ours(args, world, rank, local):
    import torch
    import kvmem_b200 as K
    w = workload(args)
    if args.kernel_only:
        return run_kernel_only(args, w, local)
    if args.config == "c4":
        return run_replay(args, w, world, rank, local)
    if args.config == "c5":
        line = sharded_selection(args, w, world, rank, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        return run_sharded_recall(args, w, world, rank, local)
    assert w.groups == 1, "stage-in geometry of this bench is per-layer selection"
    dev = torch.device("cuda", local)
    h = build_history(w, args.seed, dev)
    ctx = K.RecallContext(local)
    P, L = w.pages, w.layers
    srows = L * w.groups
    page_k, page_v = h["page_k"], h["page_v"]
    slots = w.budget
    cache_k = torch.zeros(srows * slots * page_k, dtype=torch.uint8, device=dev)
    cache_v = torch.zeros(srows * slots * page_v, dtype=torch.uint8, device=dev)
    layout = K.stage_layout([
        dict(host_base=h["host_k"].data_ptr(), host_row_stride=h["layer_k"], host_page_stride=page_k,
             dev_base=cache_k.data_ptr(), dev_row_stride=slots * page_k, dev_slot_stride=page_k, bytes=page_k),
        dict(host_base=h["host_v"].data_ptr(), host_row_stride=h["layer_v"], host_page_stride=page_v,
             dev_base=cache_v.data_ptr(), dev_row_stride=slots * page_v, dev_slot_stride=page_v, bytes=page_v)])
    pool = K.ResidencyPool(ctx, srows, P, slots)
    desc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     tokens=w.tokens, page_tokens=w.page_tokens, groups=w.groups)
    kc = K.RecallContext.make_kcache(h["k_dev"], w.k_type, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     capacity_tokens=P * w.page_tokens)
    qs = h["drift"]  # the query of step s: the rotating needle group s mod rot_groups is favoured
    qdescs = [K.RecallContext.make_query(q, w.rows) for q in qs]
    mass = torch.empty((srows, P), dtype=torch.float32, device=dev)
    sel_ids = torch.empty((srows, w.budget), dtype=torch.int32, device=dev)
    sel_n = torch.empty((srows,), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def step(i, force=False, with_pool=True, qd=None):
        ctx.recall_step(desc, qd or qdescs[i % len(qdescs)], kc, w.keep, w.budget, mass_mean=mass, sel_ids=sel_ids,
                        sel_n=sel_n, pool=pool if with_pool else None, layout=layout if with_pool else None,
                        chunks=args.chunks, stage_ctas=args.stage_ctas, force_reload=force,
                        first_layers=args.first_layers)

    def timed(n, fn):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(n):
            fn(i)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / n

    # Warm-up, then the timed steady state: every step restores the pages of the next
    # rotating needle group and evicts the previous group's.
    for i in range(args.warmup):
        step(i)
    ctx.wait(120.0)
    a0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed")
        ev0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    launches = ctx.launches - a0
    ms_step = ev0.elapsed_time(ev1) / args.steps
    ctx.check_status("timed steps")
    # The last plan's restores, gathered again alone: the stage-in half of a steady step.
    pool.stage_in(layout, ctas=args.stage_ctas)
    gather_steady_ms = timed(5, lambda i: pool.stage_in(layout, ctas=args.stage_ctas))
    start = args.warmup + args.steps

    # End to end through the C ABI with host buffers: H2D of the step's queries, the step
    # (with its stage-in), D2H of the selection.
    q_host = [q.cpu().pin_memory() for q in qs]
    q_dev = torch.empty_like(qs[0])
    qd_e2e = K.RecallContext.make_query(q_dev, w.rows)
    ids_host = torch.empty(sel_ids.shape, dtype=torch.int32, pin_memory=True)
    n_host = torch.empty(sel_n.shape, dtype=torch.int32, pin_memory=True)
    h2d = q_host[0].numel() * 4
    d2h = ids_host.numel() * 4 + n_host.numel() * 4

    def e2e_step(i):
        j = start + i
        q_dev.copy_(q_host[j % len(q_host)], non_blocking=True)
        step(j, qd=qd_e2e)
        ids_host.copy_(sel_ids, non_blocking=True)
        n_host.copy_(sel_n, non_blocking=True)

    e2e_step(0)
    start += 1
    e2e_ms = timed(args.steps, e2e_step)
    start += args.steps
    ctx.check_status("e2e steps")

    # Selection alone (score -> top-k, no residency plan or stage-in) on the same queries.
    select_ms = timed(args.steps, lambda i: step(start + i, with_pool=False))
    restored = step_stats(w, ctx, desc, kc, qdescs, start, min(args.steps, 8), mass, sel_ids, sel_n, args.chunks)

    # Cold worst case: every selected page staged every step.
    n_cold = max(3, min(10, args.steps))
    step(0, force=True)
    ms_cold = timed(n_cold, lambda i: step(i, force=True))
    cold_bytes = srows * w.budget * (page_k + page_v)

    # Stage-in alone (the gather of a full cold plan) -> link GB/s.
    g_ms = []
    for _ in range(3):
        pool.plan(sel_ids, sel_n, force_reload=True)
        g_ms.append(timed(1, lambda i: pool.stage_in(layout, ctas=args.stage_ctas)))
    gather_ms = statistics.median(g_ms)
    ref_route_ms = reference_stagein_route(w, h, pool, cache_k, cache_v, slots, dev)
    stageout_ms, out_bytes = stageout_harvest(args, w, cache_k, cache_v, slots, page_k, page_v, local)

    # Dominant kernel alone: the page log-sum-exp pass over all layers (+ its tiny normaliser).
    kbytes = L * P * w.page_tokens * w.kv_heads * h["rbk"]
    for _ in range(2):
        ctx.score_pages(desc, qdescs[0], kc, want_rows=False, out_mean=mass.view(L, w.groups, P))
    kernel_ms = timed(10, lambda i: ctx.score_pages(desc, qdescs[0], kc, want_rows=False,
                                                    out_mean=mass.view(L, w.groups, P)))
    hbm_peak, peak_src = peaks()
    achieved = kbytes / (kernel_ms * 1e-3) / 1e9
    traffic, traffic_src = traffic_of(args.config)

    token_layers = L * w.tokens
    cpu = None if args.no_cpu_baseline else cpu_baseline_port(w, h)
    ref_gpu = None if args.no_cpu_baseline else reference_gpu_timings(w, h, qs[0], dev)
    pool.close()
    ctx.close()
    del cache_k, cache_v, h
    torch.cuda.empty_cache()
    c5 = None if args.no_c5 else sharded_selection(args, workload_named("c5"), world, rank, local)
    prefill = None if args.no_prefill else prefill_capture(dev, args.prefill_base)
    line = {
        "metric": METRIC, "value": token_layers / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16" if w.k_type == 1 else "q8_0",
        "data": "synthetic: seeded on-device N(0,1) K/V with per-channel scale U(0.5,2), planted fixed and "
                "rotating needle pages",
        "config": {"workload": w.name, "layers": L, "q_heads": w.q_heads, "kv_heads": w.kv_heads,
                   "head_dim": w.head_dim, "tokens": w.tokens, "page_tokens": w.page_tokens, "pages": P,
                   "top_k": w.top_k, "keep": "first+last", "selection": "per layer",
                   "parallelism": "single GPU", "chunks": args.chunks, "first_chunk_layers": args.first_layers,
                   "l2": f"inputs larger than L2 ({kbytes / 1e9:.1f} GB of K read per step)",
                   "step": "score all pages -> top-k -> residency plan -> stage-in of non-resident pages (K+V) "
                           f"from pinned host; the query of each step favours the next rotating needle group, "
                           f"so {w.rotating} of each layer's {w.top_k} pages turn over per step"},
        "restored_pages_per_step": restored,
        "stage_bytes_per_step": restored * (page_k + page_v),
        "select_ms": select_ms, "gather_steady_ms": gather_steady_ms,
        "clocks": clk.summary(),
        "e2e": {"value": token_layers / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm",
                     "kernel": ("page_lse_mma_kernel" if w.k_type == 1 else "page_lse_q_kernel")
                               + " (+page_mass_normalize_kernel)",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "peak_source": peak_src, "traffic": traffic, "traffic_source": traffic_src,
                     "kernel_ms": kernel_ms, "algorithmic_bytes": kbytes},
        "roofline_stagein": {"bound": "pcie", "kernel": "stagein_gather_kernel (steady plan, alone)",
                             "achieved": restored * (page_k + page_v) / (gather_steady_ms * 1e-3) / 1e9,
                             "peak": PCIE_PEAK_GBS, "unit": "GB/s",
                             "frac": restored * (page_k + page_v) / (gather_steady_ms * 1e-3) / 1e9 / PCIE_PEAK_GBS,
                             "peak_source": "ncu pcie__throughput peak of PCIe Gen5 x16 on this pool "
                                            "(profiles/stagein_stageout_pcie_c2.md)"},
        "cold": {"ms_per_step": ms_cold, "stage_bytes_per_step": cold_bytes,
                 "note": "every selected page staged every step (force_reload)"},
        "stagein": {"gather_ms": gather_ms, "bytes": cold_bytes, "GB/s": cold_bytes / (gather_ms * 1e-3) / 1e9,
                    "ctas": args.stage_ctas, "link": "PCIe Gen5 x16 (mapped pinned host reads)"},
        "stagein_reference_route": {"ms": ref_route_ms, "bytes": cold_bytes,
                                    "GB/s": cold_bytes / (ref_route_ms * 1e-3) / 1e9,
                                    "route": "two host memcpys per record (store -> vector -> 32 MiB pinned slab), "
                                             "one H2D per slab, one D2D per item (the reference's slab "
                                             "route, restated; host clock)"},
        "stageout": {"ms": stageout_ms, "bytes": out_bytes, "GB/s": out_bytes / (stageout_ms * 1e-3) / 1e9,
                     "what": "K+V of one block per layer into two 32 MiB pinned slots in turn (host clock, "
                             "submit to last slot observed)", "ctas": args.stage_ctas},
        "cpu_baseline": cpu,
        "reference_gpu": ref_gpu,
        "c5_sharded": c5,
        "prefill_page_lse": prefill,
    }
    print(json.dumps(line), flush=True)


def prefill_capture(dev, base=36864):
    """Prefill page statistics, the reference's own long case (base 36864 cached tokens, a
    1024-row prompt chunk, 24 query / 4 KV heads, head_dim 256, 32 sampled rows 32i+31, pages of
    64 tokens; docs/benchmarks/ninfer-sm120-prefill-page-lse-20261114.json:43-49), bf16 instead
    of the engine's FP8 cache:
      fused     kvm_prefill_attention with capture (attention output + page LSE in one pass);
      separate  the same attention without capture, then kvm_score_pages over the 32 sampled rows
                with causal visibility as a -inf bias (the second Q.K^T pass the fusion removes);
    plus the tcgen05 attention's FLOP rate (4 * heads * head_dim * visible keys summed over rows)
    against the measured bf16 peak, and flash_attn's causal forward on the same tensors for
    context (a library kernel, not part of this repository). CUDA events, median of 10 after 3
    warm-up calls; K + V are 155 MB, above L2. `base` other than 36864 (--prefill-base) gives a
    smaller case of the same shape for ncu captures."""
    import torch

    import kvmem_b200 as K
    try:
        torch.cuda.synchronize()
        ctx = K.RecallContext(dev.index or 0)
        width, hq, hkv, dim = 1024, 24, 4, 256
        T = base + width
        g = torch.Generator(device=dev).manual_seed(11)
        q = torch.randn(width, hq, dim, device=dev, generator=g).bfloat16()
        k = torch.randn(T, hkv, dim, device=dev, generator=g).bfloat16()
        v = torch.randn(T, hkv, dim, device=dev, generator=g).bfloat16()
        samples = [32 * i + 31 for i in range(32)]
        out = torch.empty_like(q)
        lse = torch.empty(len(samples), hq, T // 64, device=dev)
        qs = q[samples].contiguous().view(1, len(samples), hq, dim)
        pos = torch.tensor([base + r for r in samples], device=dev)
        mask = torch.where(torch.arange(T, device=dev)[None, :] <= pos[:, None], 0.0, float("-inf")).float()
        sdesc = K.RecallContext.make_desc(layers=1, q_heads=hq, kv_heads=hkv, head_dim=dim, tokens=T,
                                          page_tokens=64, mask=mask)
        sq = K.RecallContext.make_query(qs, len(samples))
        sk = K.RecallContext.make_kcache(k, K.BF16, kv_heads=hkv, head_dim=dim, capacity_tokens=T)

        def med(fn, it=10):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ts = []
            for _ in range(it):
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            return statistics.median(ts)

        fused = med(lambda: ctx.prefill_attention(q, k, v, base=base, sample_rows=samples, out=out, page_lse=lse))
        attn = med(lambda: ctx.prefill_attention(q, k, v, base=base, out=out))
        stats = med(lambda: ctx.score_pages(sdesc, sq, sk, want_mean=False))
        ctx.check_status("prefill_capture")
        flops = 4.0 * hq * dim * sum(base + i + 1 for i in range(width))
        peak, src = tensor_peak()
        res = {"config": {"base": base, "width": width, "q_heads": hq, "kv_heads": hkv, "head_dim": dim,
                          "samples": len(samples), "page_tokens": 64, "dtype": "bf16"},
               "fused_ms": fused, "attention_only_ms": attn, "separate_ms": attn + stats,
               "separate_stats_ms": stats, "capture_cost_ms": fused - attn,
               "attention_tflops": flops / attn / 1e9, "fused_tflops": flops / fused / 1e9,
               "frac_of_bf16_peak": flops / fused / 1e9 / peak, "peak_tflops": peak, "peak_source": src,
               "kernel": "prefill_attn_kernel (+prefill_combine_kernel)",
               "reference_published": {"separate_ms": 31.8095, "fused_ms": 9.74842,
                                       "hardware": "RTX PRO 6000 Blackwell (sm_120a), FP8 KV",
                                       "source": "docs/benchmarks/ninfer-sm120-prefill-page-lse-20261114.json"}}
        try:
            from flash_attn import flash_attn_func
            qq, kk, vv = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
            res["flash_attn_ms"] = med(lambda: flash_attn_func(qq, kk, vv, causal=True))
        except Exception as e:  # library missing or not built for this GPU: context only
            res["flash_attn_ms"] = None
            res["flash_attn_error"] = repr(e)[:120]
        ctx.close()
        del q, k, v, out, lse, mask
        torch.cuda.empty_cache()
        return res
    except Exception as e:
        return {"error": repr(e)[:300]}


def workload_named(name):
    from kvmem_b200 import synth
    return synth.CONFIGS[name]


def reference_stagein_route(w, h, pool, cache_k, cache_v, slots, dev):
    """The reference's stage-in route for the current plan's cold set, restated: each page record
    is copied out of the store into a host vector (src/adapter/llama-memory-kvmem.cpp:4501-4502),
    then into a 32 MiB pinned slab; a full slab goes to a device staging buffer with one H2D copy
    and an event wait, then one D2D copy per item into its cache slot
    (src/adapter/llama-kvmem-stagein.cu:673-794). Python drives the item loop. Host ms."""
    import numpy as np
    import torch
    page_k, page_v = h["page_k"], h["page_v"]
    slot_of, _ = pool.read()
    slab_bytes = 32 << 20
    slab = torch.empty(slab_bytes, dtype=torch.uint8, pin_memory=True)
    slab_np = slab.numpy()
    dev_q = torch.empty(slab_bytes, dtype=torch.uint8, device=dev)
    items = []
    hk, hv = h["host_k"].numpy(), h["host_v"].numpy()
    for r in range(slot_of.shape[0]):
        for p in np.nonzero(slot_of[r] >= 0)[0]:
            s_ = int(slot_of[r, p])
            items.append((hk, r * h["layer_k"] + int(p) * page_k, cache_k, (r * slots + s_) * page_k, page_k))
            items.append((hv, r * h["layer_v"] + int(p) * page_v, cache_v, (r * slots + s_) * page_v, page_v))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    used, pending = 0, []

    def flush():
        dev_q[:used].copy_(slab[:used], non_blocking=True)
        torch.cuda.synchronize()  # the slab is reused by the next batch
        for dst, doff, off, n in pending:
            dst[doff:doff + n].copy_(dev_q[off:off + n], non_blocking=True)

    for src, soff, dst, doff, n in items:
        if used + n > slab_bytes:
            flush()
            used, pending = 0, []
        slab_np[used:used + n] = src[soff:soff + n].copy()
        pending.append((dst, doff, used, n))
        used += n
    if pending:
        flush()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) * 1e3


def stageout_harvest(args, w, cache_k, cache_v, slots, page_k, page_v, local):
    """Stage-out (harvest) of one filled block per layer: its K and V bytes from the device cache
    into the two 32 MiB pinned slots in turn -> (host ms, bytes)."""
    import torch
    import kvmem_b200 as K
    so = K.StageOut(local)
    L = w.layers

    def harvest():
        pending = -1
        for l in range(L):
            for cache, pb in ((cache_k, page_k), (cache_v, page_v)):
                src = cache.data_ptr() + l * slots * pb
                if so.enqueue(src, pb) is None:
                    slot = so.submit(ctas=args.stage_ctas)
                    so.wait(pending)
                    pending = slot
                    so.enqueue(src, pb)
        slot = so.submit(ctas=args.stage_ctas)
        so.wait(pending)
        so.wait(slot)

    harvest()
    o_ms = []
    for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        harvest()
        o_ms.append((time.perf_counter() - t0) * 1e3)
    so.close()
    return statistics.median(o_ms), L * (page_k + page_v)


def sharded_selection(args, w, world, rank, local):
    """Config 5: one 1M-token q8_0 history partitioned by page range over the ranks (strong
    scaling). A step = sharded selection on every rank: local page LSE, all-gather of softmax
    statistics, local masses, local candidates, all-gather, global top-k. No stage-in (its
    host records would be 111 GB of pinned K and V). Returns the line as a dict (rank 0)."""
    import torch
    import kvmem_b200 as K
    from kvmem_b200.shard import LseGatherSelector, ShardCompute, ShardedSelector, ShardGeometry, page_ranges
    dev = torch.device("cuda", local)
    P, L, B = w.pages, w.layers, w.page_tokens
    p0, p1 = page_ranges(P, world)[rank]
    lp = p1 - p0
    h = build_history(w, args.seed, dev, need_host=False, page_range=(p0, p1))
    page_bytes = h["page_k"]
    ctx = K.RecallContext(local)
    desc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     tokens=w.tokens, page_tokens=B, groups=w.groups)
    kc = K.RecallContext.make_kcache(h["k_dev"], w.k_type, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     capacity_tokens=lp * B)
    qds = [K.RecallContext.make_query(q, w.rows) for q in h["drift"]]
    geo = ShardGeometry(layers=L, rows=w.rows, q_heads=w.q_heads, kv_heads=w.kv_heads, groups=w.groups,
                        total_pages=P, page0=p0, local_pages=lp)
    sel = (LseGatherSelector if args.shard_exchange == "lse" else ShardedSelector)(ShardCompute(ctx))
    warm = max(3, min(args.warmup, 5))
    steps = max(5, min(args.steps, 10))
    for i in range(warm):
        sel.select(desc, qds[i % len(qds)], kc, geo, w.keep, w.budget)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0 = ctx.launches
    with ClockSampler(list(range(world)), enabled=rank == 0) as clk:
        barrier(world)  # every rank starts together, after rank 0's sampler is up
        ev0.record()
        for i in range(steps):
            sel.select(desc, qds[(warm + i) % len(qds)], kc, geo, w.keep, w.budget)
        ev1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / steps, world)
    launches = ctx.launches - a0
    ctx.check_status("sharded steps")
    # The local scorer alone (this rank's pages), for the roofline.
    ldesc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                      tokens=lp * B, page_tokens=B)
    ctx.score_pages(ldesc, qds[0], kc, want_rows=False)
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(5):
        ctx.score_pages(ldesc, qds[0], kc, want_rows=False)
    ev1.record()
    torch.cuda.synchronize()
    kernel_ms = max_over_ranks(ev0.elapsed_time(ev1) / 5, world)
    kbytes_local = L * lp * page_bytes
    hbm_peak, src = peaks()
    ctx.close()
    del h
    torch.cuda.empty_cache()
    return {
        "metric": METRIC, "value": L * w.tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q8_0" if w.k_type == 3 else "f16",
        "data": "synthetic: seeded on-device q8_0 K (codes round(N(0,1)*40), scales U(0.005,0.03)), "
                "fixed and rotating needle pages",
        "config": {"workload": w.name, "layers": L, "tokens": w.tokens, "pages": P, "top_k": w.top_k,
                   "parallelism": f"page-range shards x{world}", "pages_per_rank": lp,
                   "exchange": args.shard_exchange,
                   "step": ("sharded selection (one NCCL all-gather of the page LSE)" if args.shard_exchange == "lse"
                            else "sharded selection (two NCCL all-gathers)") + "; stage-in not included",
                   "l2": f"inputs larger than L2 ({kbytes_local / 1e9:.1f} GB of K per rank per step)"},
        "clocks": clk.summary(), "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "page_lse_q_kernel (local pages)", "kernel_ms": kernel_ms,
                     "achieved": kbytes_local / (kernel_ms * 1e-3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                     "frac": kbytes_local / (kernel_ms * 1e-3) / 1e9 / hbm_peak, "peak_source": src,
                     "algorithmic_bytes": kbytes_local,
                     "step_GBps_all_ranks": L * P * page_bytes / (ms * 1e-3) / 1e9},
    }


def chunk_schedule(layers, chunks, first):
    """Layer chunks [(l0, n)] as kvm_recall_step cuts them: a first chunk of `first` layers
    (when 0 < first < layers and chunks > 1), the rest in equal parts."""
    chunks = max(1, min(chunks, layers))
    parts, l0 = [], 0
    if 0 < first < layers and chunks > 1:
        parts.append((0, first))
        l0 = first
    rest = chunks - len(parts)
    per = -(-(layers - l0) // rest)
    while l0 < layers:
        parts.append((l0, min(per, layers - l0)))
        l0 += per
    return parts


def run_sharded_recall(args, w, world, rank, local):
    """N > 1: one history partitioned by page range over the ranks (strong scaling), the whole
    decode-step recall on every rank (kvmem_b200.shard.ShardedRecall): local page LSE, two NCCL
    all-gathers of small tensors per layer chunk, the replicated residency plan, and the stage-in
    of each rank's restored pages from its own pinned records (its own PCIe link) into the decode
    GPU's (rank 0's) paged cache through a CUDA-IPC peer mapping (NVLink); a one-element
    all-reduce ends the step. value = token-layers of the whole history / max-over-ranks ms."""
    import torch
    import torch.distributed as dist
    import kvmem_b200 as K
    from kvmem_b200.shard import (LseGatherSelector, ShardCompute, ShardedRecall, ShardedSelector, ShardGeometry,
                                  page_ranges)
    assert w.groups == 1, "stage-in geometry of this bench is per-layer selection"
    dev = torch.device("cuda", local)
    P, L, B = w.pages, w.layers, w.page_tokens
    p0, p1 = page_ranges(P, world)[rank]
    lp = p1 - p0
    h = build_history(w, args.seed, dev, page_range=(p0, p1))
    page_k, page_v = h["page_k"], h["page_v"]
    slots = w.budget
    # The decode GPU (rank 0) owns the paged cache of every layer; the others map it.
    if rank == 0:
        cache_k = torch.zeros(L * slots * page_k, dtype=torch.uint8, device=dev)
        cache_v = torch.zeros(L * slots * page_v, dtype=torch.uint8, device=dev)
        handles = [K.ipc_export(cache_k), K.ipc_export(cache_v)]
    else:
        handles = None
    box = [handles]
    dist.broadcast_object_list(box, src=0)
    if rank == 0:
        ck, cv = cache_k.data_ptr(), cache_v.data_ptr()
    else:
        ck, cv = K.ipc_open(local, box[0][0]), K.ipc_open(local, box[0][1])
    ctx = K.RecallContext(local)
    chunk_layers = chunk_schedule(L, args.chunks_sharded, args.first_layers)
    pools, layouts = [], []
    for l0, nl in chunk_layers:
        pools.append(K.ResidencyPool(ctx, nl, P, slots))
        layouts.append(K.stage_layout([
            dict(host_base=h["host_k"].data_ptr() + l0 * h["layer_k"], host_row_stride=h["layer_k"],
                 host_page_stride=page_k, dev_base=ck + l0 * slots * page_k, dev_row_stride=slots * page_k,
                 dev_slot_stride=page_k, bytes=page_k),
            dict(host_base=h["host_v"].data_ptr() + l0 * h["layer_v"], host_row_stride=h["layer_v"],
                 host_page_stride=page_v, dev_base=cv + l0 * slots * page_v, dev_row_stride=slots * page_v,
                 dev_slot_stride=page_v, bytes=page_v)]))
    geo = ShardGeometry(layers=L, rows=w.rows, q_heads=w.q_heads, kv_heads=w.kv_heads, groups=w.groups,
                        total_pages=P, page0=p0, local_pages=lp)
    selector = (LseGatherSelector if args.shard_exchange == "lse" else ShardedSelector)(ShardCompute(ctx))
    rec = ShardedRecall(selector, pools, layouts, chunk_layers, geo, stage_ctas=args.stage_ctas)
    desc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     tokens=w.tokens, page_tokens=B, groups=w.groups)
    kc = K.RecallContext.make_kcache(h["k_dev"], w.k_type, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     capacity_tokens=lp * B)
    qs = h["drift"]
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        rec.step(desc, qs[i % len(qs)], kc, w.keep, w.budget)
    torch.cuda.synchronize()
    # The step as one CUDA graph (the step's queries copied into q_static first): the host
    # then issues one launch per step instead of a few dozen library calls and collectives.
    q_static = qs[0].clone()
    graphed = args.graph and rec.capture(desc, q_static, kc, w.keep, w.budget)

    def run_step(i, q_src=None, non_blocking=False):
        q = qs[i % len(qs)] if q_src is None else q_src
        if graphed:
            q_static.copy_(q, non_blocking=non_blocking)
            return rec.replay()
        return rec.step(desc, q, kc, w.keep, w.budget)

    for i in range(2):
        run_step(i)
    torch.cuda.synchronize()
    a0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(list(range(world)), enabled=rank == 0) as clk:
        barrier(world)  # every rank starts together, after rank 0's sampler is up
        torch.cuda.nvtx.range_push("timed")
        ev0.record(stream)
        for i in range(args.steps):
            run_step(args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    launches = rec.graph_launches * args.steps if graphed else ctx.launches - a0
    ms_step = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    ctx.check_status("sharded recall steps")
    start = args.warmup + args.steps

    # Pages restored per step (every rank holds the same selection): selection differences.
    import numpy as np
    restored, prev = [], None
    for i in range(start, start + min(args.steps, 8) + 1):
        ids, n = run_step(i)
        ih, nh = ids.cpu().numpy(), n.cpu().numpy()
        cur = [set(ih[r, : nh[r]].tolist()) for r in range(L)]
        if prev is not None:
            restored.append(sum(len(c - p) for c, p in zip(cur, prev)))
        prev = cur
    start += min(args.steps, 8) + 1
    restored_per_step = float(np.mean(restored)) if restored else 0.0

    # End to end: every rank copies the step's queries from pinned host memory, rank 0 reads
    # the selection back.
    q_host = [q.cpu().pin_memory() for q in qs]
    q_dev = torch.empty_like(qs[0])
    ids_host = torch.empty((L, w.budget), dtype=torch.int32, pin_memory=True)
    n_host = torch.empty((L,), dtype=torch.int32, pin_memory=True)

    def e2e_step(j):
        if graphed:  # straight from pinned host memory into the graph's query buffer
            ids, n = run_step(j, q_src=q_host[j % len(q_host)], non_blocking=True)
        else:
            q_dev.copy_(q_host[j % len(q_host)], non_blocking=True)
            ids, n = rec.step(desc, q_dev, kc, w.keep, w.budget)
        if rank == 0:
            ids_host.copy_(ids, non_blocking=True)
            n_host.copy_(n, non_blocking=True)

    e2e_step(start)
    torch.cuda.synchronize()
    barrier(world)
    ev0.record(stream)
    for i in range(args.steps):
        e2e_step(start + 1 + i)
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    h2d = world * q_host[0].numel() * 4
    d2h = ids_host.numel() * 4 + n_host.numel() * 4

    # Breakdown: the selection alone (same chunks and collectives, no plan or stage-in), and the
    # step's collectives alone (per chunk one all-gather of the softmax statistics and one of the
    # candidates, then the step's all-reduce; same sizes), each max over ranks.
    def timed_steps(fn, n):
        torch.cuda.synchronize()
        barrier(world)
        ev0.record(stream)
        for i in range(n):
            fn(i)
        ev1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(ev0.elapsed_time(ev1) / n, world)

    select_ms = timed_steps(lambda i: rec.step(desc, qs[i % len(qs)], kc, w.keep, w.budget, stage=False),
                            args.steps)
    kcand = w.budget - len(w.keep)
    widest = max(e - b for b, e in page_ranges(P, world))
    if args.shard_exchange == "lse":  # per chunk: the page LSE of the rank's range
        bufs = [[torch.zeros(nl * w.rows * w.q_heads * widest, dtype=torch.float32, device=dev)]
                for _, nl in chunk_layers]
    else:  # per chunk: softmax statistics, then candidate scores and ids side by side
        bufs = [[torch.zeros(nl * w.rows * w.q_heads * 2, dtype=torch.float32, device=dev),
                 torch.zeros(nl * w.groups * kcand * 2, dtype=torch.int32, device=dev)] for _, nl in chunk_layers]
    outs = [[torch.empty((world,) + a.shape, dtype=a.dtype, device=dev) for a in bl] for bl in bufs]
    flag = torch.ones(1, dtype=torch.int32, device=dev)

    def collectives(_):
        for bl, ol in zip(bufs, outs):
            for a, ga in zip(bl, ol):
                dist.all_gather_into_tensor(ga, a)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)

    collectives(0)
    coll_ms = timed_steps(collectives, args.steps)

    # This rank's stage-in alone: the last step's restores of every chunk gathered again.
    def gather_again(_):
        for ci in range(len(chunk_layers)):
            pools[ci].stage_in_range(layouts[ci], p0, lp, ctas=args.stage_ctas)

    gather_again(0)
    gather_ms = timed_steps(gather_again, 5)

    # The local scorer alone (this rank's pages), for the roofline.
    ldesc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                      tokens=lp * B, page_tokens=B)
    qd0 = K.RecallContext.make_query(qs[0], w.rows)
    ctx.score_pages(ldesc, qd0, kc, want_rows=False)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(5):
        ctx.score_pages(ldesc, qd0, kc, want_rows=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    kernel_ms = max_over_ranks(ev0.elapsed_time(ev1) / 5, world)
    kbytes_local = L * lp * page_k
    hbm_peak, peak_src = peaks()
    rec.release()  # the graph holds NCCL work: drop it before the process group goes
    for p in pools:
        p.close()
    ctx.close()
    barrier(world)  # no rank writes the decode cache any more
    if rank != 0:
        K.ipc_close(local, ck)
        K.ipc_close(local, cv)
    barrier(world)
    del h
    torch.cuda.empty_cache()
    c5 = None if args.no_c5 else sharded_selection(args, workload_named("c5"), world, rank, local)
    if rank != 0:
        return
    token_layers = L * w.tokens
    print(json.dumps({
        "metric": METRIC, "value": token_layers / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16" if w.k_type == 1 else "q8_0",
        "data": "synthetic: seeded on-device N(0,1) K/V with per-channel scale U(0.5,2), planted fixed and "
                "rotating needle pages",
        "config": {"workload": w.name, "layers": L, "q_heads": w.q_heads, "kv_heads": w.kv_heads,
                   "head_dim": w.head_dim, "tokens": w.tokens, "page_tokens": B, "pages": P,
                   "top_k": w.top_k, "keep": "first+last", "selection": "per layer",
                   "parallelism": f"page-range shards x{world}", "pages_per_rank": lp, "chunks": len(chunk_layers),
                   "chunk_layers": [n for _, n in chunk_layers],
                   "l2": f"inputs larger than L2 ({kbytes_local / 1e9:.1f} GB of K per rank per step)",
                   "exchange": args.shard_exchange, "cuda_graph": graphed,
                   "step": ("per layer chunk: local page LSE, one NCCL all-gather of it, whole-row masses and "
                            "top-k on every rank" if args.shard_exchange == "lse" else
                            "per layer chunk: local page LSE, NCCL all-gather of softmax statistics, local "
                            "masses and candidates, NCCL all-gather of candidates, global top-k") +
                           ", replicated residency plan; stage-in of each rank's restored pages (K+V) from its "
                           "own pinned records into rank 0's paged cache over NVLink (CUDA IPC peer writes); "
                           "one all-reduce ends the step"},
        "restored_pages_per_step": restored_per_step,
        "stage_bytes_per_step": restored_per_step * (page_k + page_v),
        "breakdown": {"select_ms": select_ms, "collectives_ms": coll_ms, "scorer_ms": kernel_ms,
                      "gather_ms": gather_ms,
                      "collectives_per_step": len(bufs[0]) * len(chunk_layers) + 1,
                      "exchange": args.shard_exchange,
                      "note": "select_ms: the step without residency plan and stage-in; collectives_ms: its "
                              "NCCL all-gathers (page LSE, or statistics and candidates) and the closing "
                              "all-reduce alone; "
                              "scorer_ms: this rank's page LSE pass alone; gather_ms: this rank's stage-in "
                              "of one step alone (its own PCIe link, NVLink writes to the decode GPU); all "
                              "max over ranks"},
        "clocks": clk.summary(),
        "e2e": {"value": token_layers / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "page_lse_mma_kernel (local pages, +normaliser)",
                     "kernel_ms": kernel_ms, "achieved": kbytes_local / (kernel_ms * 1e-3) / 1e9,
                     "peak": hbm_peak, "unit": "GB/s",
                     "frac": kbytes_local / (kernel_ms * 1e-3) / 1e9 / hbm_peak, "peak_source": peak_src,
                     "traffic": None, "algorithmic_bytes": kbytes_local,
                     "step_GBps_all_ranks": L * P * page_k / (ms_step * 1e-3) / 1e9},
        "c5_sharded": c5,
    }), flush=True)


def cpu_baseline_port(w, h):
    """The FP64 per-token page mass of the oracle restatement (the reference's dense oracle,
    src/adapter/llama-kvmem-attention.cpp:61-94) plus the reference's picker, over all host
    cores: one layer per task (the C calls release the interpreter lock). Bounded sample: the
    first min(layers, 4 x cores) layers of one step's history (a whole config-2 step on 16+
    cores); value = token-layers / wall second."""
    import numpy as np
    from oracle import oracle as O
    model, cores = cpu_info()
    n_layers = min(w.layers, 4 * cores)
    rb = h["rbk"]
    T = w.pages * w.page_tokens
    hk = h["host_k"].numpy()
    q = h["drift"][0].cpu().numpy().astype(np.float32)
    use_ref = O.ref() is not None

    def one(l):
        k0 = hk[l * h["layer_k"]:(l + 1) * h["layer_k"]]
        m = O.page_mass(q[l:l + 1], O.F32, k0, w.k_type, layers=1, rows=w.rows, heads=w.q_heads,
                        kv_heads=w.kv_heads, dim=w.head_dim, tokens=w.tokens, page_tokens=w.page_tokens,
                        scale=1 / np.sqrt(w.head_dim), k_strides=(T * w.kv_heads * rb, w.kv_heads * rb, rb))
        O.pick_scored(w.pages, list(range(w.pages)), m[0, 0].mean(axis=0), w.keep, w.budget, use_ref=use_ref)

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=cores) as ex:
        list(ex.map(one, range(n_layers)))
    dt = time.perf_counter() - t0
    return {"value": n_layers * w.tokens / dt, "unit": UNIT, "cores": cores, "cpu_model": model, "kind": "port",
            "sample": f"{n_layers} of {w.layers} layers x {w.tokens} tokens x {w.q_heads} heads of one step: "
                      f"FP64 per-token page mass (AttentionSampler::qualify restated) + pick_scored_blocks, "
                      f"one layer per thread, {dt:.1f} s wall"}


def reference_gpu_timings(w, h, q, dev):
    """The reference's own GPU scorers (oracle/_ref/libkvref_cuda.so, compiled from its sources for
    sm_100a) on this step's inputs, host-timed per call as the reference runs them (each call
    synchronises its stream and copies its scores to the host):
      per_token: llama_kvmem_attention_cuda::score per layer, one decode row, zero mask
                 (src/adapter/llama-kvmem-attention-cuda.cu:146-193), summed over the layers;
      meank:     PageSoftmaxCuda::score over the pages' mean keys of the same K, all layers in one
                 call (kvmem/src/cuda/page_softmax.cu:202-280)."""
    import numpy as np
    import torch
    from oracle import oracle as O
    if O.ref_cuda() is None:
        return {"unavailable": "oracle/_ref/libkvref_cuda.so was not built (reference sources absent at build)"}
    L, P, T = w.layers, w.pages, w.pages * w.page_tokens
    rb = h["rbk"]
    mask = torch.zeros((1, T), dtype=torch.float32, device=dev)
    qf = q.contiguous()
    esz = 4

    def per_token_step():
        total = 0.0
        for l in range(L):
            _, ms = O.ref_attention_score(
                qf[l].data_ptr(), O.F32, dim=w.head_dim, q_rows=w.rows, heads=w.q_heads,
                q_row_stride=w.q_heads * w.head_dim * esz, q_head_stride=w.head_dim * esz,
                k_ptr=h["k_dev"].data_ptr() + l * h["layer_k"], k_type=w.k_type, tokens=w.tokens,
                kv_heads=w.kv_heads, k_token_stride=w.kv_heads * rb, k_head_stride=rb, mask_ptr=mask.data_ptr(),
                mask_type=O.F32, mask_row_stride=T * 4, scale=float(1 / np.sqrt(w.head_dim)), softcap=0.0,
                block=w.page_tokens, rows=list(range(w.rows)))
            total += ms
        return total

    per_token_step()
    pt = [per_token_step() for _ in range(2)]
    kbytes = L * P * w.page_tokens * w.kv_heads * rb
    out = {"per_token_ms": min(pt), "per_token_GBps_of_K": kbytes / (min(pt) * 1e-3) / 1e9}
    if w.k_type == 1:
        kv = h["k_dev"].view(torch.float16).view(L, P, w.page_tokens, w.kv_heads * w.head_dim)
        sums = torch.stack([kv[l].float().sum(dim=1) for l in range(L)]).cpu().numpy()
        counts = np.full(P, w.page_tokens, np.uint32)
        qn = qf.view(L, w.rows, -1).cpu().numpy()
        kw = dict(heads=w.q_heads, kv_heads=w.kv_heads, dim=w.head_dim, block=w.page_tokens, accepted=w.tokens,
                  budget=w.budget, sink=1, recent=1, fixed=w.keep)
        lr = np.full(L, w.rows, np.uint32)
        O.ref_page_softmax_cuda(dev.index or 0, sums, counts, qn, lr, **kw)
        mk = [O.ref_page_softmax_cuda(dev.index or 0, sums, counts, qn, lr, **kw)[1] for _ in range(3)]
        out["meank_ms"] = min(mk)
    O.ref_cuda().kvref_cuda_release()
    out["note"] = ("the reference's kernels compiled from its sources for sm_100a; per-token re-reads K once per "
                   "query head (no GQA reuse) and synchronises after each layer's call")
    return out

def run_kernel_only(args, w, local):
    """The page scorer alone over the workload (device-resident K), for profiling."""
    import torch
    import kvmem_b200 as K
    dev = torch.device("cuda", local)
    h = build_history(w, args.seed, dev, need_host=False)
    ctx = K.RecallContext(local)
    L, P = w.layers, w.pages
    desc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     tokens=w.tokens, page_tokens=w.page_tokens, groups=w.groups)
    if args.config == "c4" and args.kmirror == "head":
        h["k_dev"], kc = head_major_mirror(w, h["k_dev"])
    else:
        kc = K.RecallContext.make_kcache(h["k_dev"], w.k_type, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                         capacity_tokens=P * w.page_tokens)
    qd = K.RecallContext.make_query(h["q_base"], w.rows)
    mass = torch.empty((L, w.groups, P), dtype=torch.float32, device=dev)
    for _ in range(args.warmup):
        ctx.score_pages(desc, qd, kc, want_rows=False, out_mean=mass)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    ev0.record()
    for _ in range(args.steps):
        ctx.score_pages(desc, qd, kc, want_rows=False, out_mean=mass)
    ev1.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    ctx.check_status("kernel-only")
    ms = ev0.elapsed_time(ev1) / args.steps
    kbytes = L * P * w.page_tokens * w.kv_heads * h["rbk"]
    peak, src = peaks()
    print(json.dumps({"kernel_only": w.name, "layers": L, "ms": ms, "GB/s": kbytes / ms / 1e6,
                      "frac": kbytes / ms / 1e6 / peak, "peak_source": src, "launches": ctx.launches}), flush=True)
    ctx.close()



def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    except Exception:
        return FALLBACK_TFLOPS, "fallback"


def run_replay(args, w, world, rank, local):
    """Config 4: multi-lane query replay, selection only. A step scores every page
    of every (lane, layer) against the lane's 32 replayed query rows x 40 heads
    (160 vectors per KV head: the tcgen05 kernel), averages the page masses over
    the replayed rows and picks the top-24 pages per (lane, layer, KV head).
    Each rank holds its own lanes (replicas: weak scaling)."""
    import torch
    import kvmem_b200 as K
    dev = torch.device("cuda", local)
    h = build_history(w, args.seed + rank, dev, need_host=False)
    ctx = K.RecallContext(local)
    P, L = w.pages, w.layers
    srows = L * w.groups
    desc = K.RecallContext.make_desc(layers=L, q_heads=w.q_heads, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                     tokens=w.tokens, page_tokens=w.page_tokens, groups=w.groups)
    if args.kmirror == "head":
        h["k_dev"], kc = head_major_mirror(w, h["k_dev"])
    else:
        kc = K.RecallContext.make_kcache(h["k_dev"], w.k_type, kv_heads=w.kv_heads, head_dim=w.head_dim,
                                         capacity_tokens=P * w.page_tokens)
    qs = [h["q_base"]] + h["drift"]
    qdescs = [K.RecallContext.make_query(q, w.rows) for q in qs]
    mass = torch.empty((srows, P), dtype=torch.float32, device=dev)
    sel_ids = torch.empty((srows, w.budget), dtype=torch.int32, device=dev)
    sel_n = torch.empty((srows,), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def step(i, qd=None):
        ctx.recall_step(desc, qd or qdescs[i % len(qdescs)], kc, w.keep, w.budget, mass_mean=mass, sel_ids=sel_ids,
                        sel_n=sel_n, chunks=args.chunks)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    a0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(list(range(world)), enabled=rank == 0) as clk:
        barrier(world)  # every rank starts together, after rank 0's sampler is up
        torch.cuda.nvtx.range_push("timed")
        ev0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    launches = ctx.launches - a0
    ms_step = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    ctx.check_status("replay steps")

    # The page scorer alone (tcgen05 LSE pass + normaliser) for the roofline.
    kbytes = L * P * w.page_tokens * w.kv_heads * h["rbk"]
    vectors = w.rows * (w.q_heads // w.kv_heads)
    flops = 2.0 * vectors * w.head_dim * w.kv_heads * P * w.page_tokens * L
    ctx.score_pages(desc, qdescs[0], kc, want_rows=False, out_mean=mass.view(L, w.groups, P))
    torch.cuda.synchronize()
    n_k = max(3, min(10, args.steps))
    ev0.record(stream)
    for _ in range(n_k):
        ctx.score_pages(desc, qdescs[0], kc, want_rows=False, out_mean=mass.view(L, w.groups, P))
    ev1.record(stream)
    torch.cuda.synchronize()
    kernel_ms = ev0.elapsed_time(ev1) / n_k
    hbm_peak, hsrc = peaks()
    tf_peak, tsrc = tensor_peak()
    gbs = kbytes / (kernel_ms * 1e-3) / 1e9
    tfs = flops / (kernel_ms * 1e-3) / 1e12

    # End to end: H2D of the step's replayed queries from pinned host memory,
    # the step, D2H of the selection.
    q_host = [q.cpu().pin_memory() for q in qs[:2]]
    q_dev = torch.empty_like(qs[0])
    qd_e2e = K.RecallContext.make_query(q_dev, w.rows)
    ids_host = torch.empty(sel_ids.shape, dtype=torch.int32, pin_memory=True)
    n_host = torch.empty(sel_n.shape, dtype=torch.int32, pin_memory=True)
    h2d = q_host[0].numel() * 4
    d2h = ids_host.numel() * 4 + n_host.numel() * 4
    n_e = max(3, min(10, args.steps))
    for i in range(2):
        q_dev.copy_(q_host[i % 2], non_blocking=True)
        step(i, qd=qd_e2e)
    torch.cuda.synchronize()
    barrier(world)
    ev0.record(stream)
    for i in range(n_e):
        q_dev.copy_(q_host[i % 2], non_blocking=True)
        step(i, qd=qd_e2e)
        ids_host.copy_(sel_ids, non_blocking=True)
        n_host.copy_(sel_n, non_blocking=True)
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / n_e, world)
    ctx.check_status("replay e2e")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_replay(w, h)
    ctx.close()
    if rank != 0:
        return
    token_layers = L * w.tokens
    print(json.dumps({
        "metric": METRIC, "value": world * token_layers / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded on-device N(0,1) fp16 K with per-channel scale U(0.5,2), N(0,1) replay queries",
        "config": {"workload": w.name, "lanes": 8, "layers_per_lane": L // 8, "q_heads": w.q_heads,
                   "kv_heads": w.kv_heads, "head_dim": w.head_dim, "tokens_per_lane": w.tokens,
                   "page_tokens": w.page_tokens, "pages": P, "replay_rows": w.rows,
                   "vectors_per_kv_head": vectors, "top_k": w.top_k, "selection": "per (lane, layer, KV head)",
                   "k_mirror": args.kmirror + "-major",
                   "parallelism": f"lane replicas x{world}" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2 ({kbytes / 1e9:.1f} GB of K read per step)",
                   "step": "score all pages (tcgen05) -> mean over replayed rows -> top-24; no stage-in"},
        "clocks": clk.summary(),
        "e2e": {"value": world * token_layers / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm" if kbytes / hbm_peak / 1e9 >= flops / tf_peak / 1e12 else "tensor",
                     "kernel": "page_lse_tc_kernel (+page_mass_normalize_kernel)", "kernel_ms": kernel_ms,
                     "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "peak_source": hsrc, "traffic": None, "algorithmic_bytes": kbytes,
                     "tensor": {"achieved": tfs, "peak": tf_peak, "unit": "TFLOP/s", "frac": tfs / tf_peak,
                                "peak_source": tsrc, "algorithmic_flops": flops,
                                "note": "Q.K^T flops of 160 vectors per KV head, fp16 hi/lo passes not counted"}},
        "cpu_baseline": cpu,
    }), flush=True)


def cpu_baseline_replay(w, h):
    """FP64 per-token page mass of the oracle port (single thread), config 4 sample."""
    from oracle import oracle as O
    tokens = 8192
    rb = h["rbk"]
    k0 = h["k_dev"][: tokens * w.kv_heads * rb].cpu().numpy()
    q0 = h["q_base"][0:1].cpu().numpy().astype(np.float32)
    t0 = time.perf_counter()
    O.page_mass(q0, O.F32, k0, w.k_type, layers=1, rows=w.rows, heads=w.q_heads, kv_heads=w.kv_heads,
                dim=w.head_dim, tokens=tokens, page_tokens=w.page_tokens, scale=1 / np.sqrt(w.head_dim),
                groups=w.groups, k_strides=(tokens * w.kv_heads * rb, w.kv_heads * rb, rb))
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"1 (lane, layer) x {tokens} tokens x {w.rows} replay rows x {w.q_heads} heads, "
                      f"FP64 oracle restatement (AttentionSampler::qualify), {dt:.1f} s"}


# --------------------------------------------------------------------------- reference arm

def run_reference(args, world, rank, local):
    """The reference's own CPU selection path on the host cores: per layer,
    query_score_frame + page_softmax_scores (Mean-K over the pages' mean keys of the
    same K) + pick_scored_blocks, from oracle/_ref (compiled from the reference's
    sources); the C restatement stands in when that library is absent."""
    if rank != 0:
        return
    import torch
    from kvmem_b200 import synth
    from oracle import oracle as O
    w = workload(args)
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    L, P, T = w.layers, w.pages, w.pages * w.page_tokens
    q_base, drift = synth.make_queries(w, args.seed, dev, drift_steps=8)
    sums = np.empty((L, P, w.kv_heads * w.head_dim), np.float32)
    for l in range(L):
        if w.k_type == 1:
            kl = synth.fp16_layer(w, args.seed, l, q_base, dev).float()
        else:
            raw = synth.q8_0_layer(w, args.seed, l, q_base, dev).view(T, w.kv_heads, w.head_dim // 32, 34)
            d = raw[..., 0:2].contiguous().view(torch.float16).float()
            kl = (raw[..., 2:].contiguous().view(torch.int8).float() * d).view(T, w.kv_heads, w.head_dim)
        sums[l] = kl.view(P, w.page_tokens, -1).sum(dim=1).cpu().numpy()
    counts = np.full(P, w.page_tokens, np.uint32)
    queries = [q.view(L, w.rows, -1).cpu().numpy() for q in drift]
    use_ref = O.ref() is not None
    threads = os.cpu_count() or 1

    def layer_select(l, q):
        ql = np.ascontiguousarray(q[l:l + 1])
        rows = np.array([w.rows], np.uint32)
        if use_ref:
            s = O.ref_page_softmax_scores(sums[l:l + 1], counts, ql, rows, heads=w.q_heads, kv_heads=w.kv_heads,
                                          dim=w.head_dim, block=w.page_tokens, accepted=w.tokens, budget=w.budget,
                                          sink=1, recent=1, fixed=w.keep)
        else:
            f = O.query_score_frame(w.tokens, w.page_tokens, w.budget, 1, 1, w.keep)
            means = sums[l:l + 1] * (np.float32(1) / counts.astype(np.float32))[None, :, None]
            s = O.meank_scores(means, ql, rows, heads=w.q_heads, kv_heads=w.kv_heads, dim=w.head_dim,
                               score_mask=f["score_mask"])
        rc, ids = O.pick_scored(P, list(range(P)), s, w.keep, w.budget, use_ref=use_ref)
        return ids

    pool = cf.ThreadPoolExecutor(max_workers=threads)

    def one_step(i):
        q = queries[i % len(queries)]
        list(pool.map(lambda l: layer_select(l, q), range(L)))

    for i in range(args.warmup):
        one_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one_step(args.warmup + i)
    dt = (time.perf_counter() - t0) / args.steps
    value = L * w.tokens / dt
    kind = "reference" if use_ref else "port"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (same generator and seed as the GPU arm)",
        "config": {"workload": w.name, "layers": L, "pages": P, "top_k": w.top_k, "selection": "per layer"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": "full step: every layer's Mean-K page softmax + pick_scored_blocks "
                                   "(reference CPU selection path), layers spread over host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    ClockSampler.init_nvml()
    if args.prefill_only:
        import torch
        print(json.dumps({"prefill_page_lse": prefill_capture(torch.device("cuda", local), args.prefill_base)}),
              flush=True)
        return
    try:
        if args.impl == "reference":
            run_reference(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
