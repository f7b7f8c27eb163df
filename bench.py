"""Benchmark of the paged KV-cache store + batch index build on B200.

One step = one pass of the hot path over one batch: the index build of the
batch (kv_indptr, kv_indices, kv_last_page_len, qo_indptr, slot_mapping) and
the store of every layer's new K/V rows into the paged pool by that slot
mapping.  Default workload: Llama-3-8B-shaped decode (32 layers, 8 KV heads x
128, bf16, page 16), 256 sequences with context U[128, 8192], one new token
each, a pool of ~150 GB per GPU, randomly fragmented page tables.

With N GPUs (torchrun, one process per GPU) the KV heads are sharded: each
rank stores 8/N heads of every token into its own head-slice pool, and the
global batch grows to 256*N sequences, so every rank moves the same bytes
per step (weak scaling) with no inter-GPU traffic; the index build is
replicated on each rank.  `value` = store bytes moved by all ranks per step
(algorithmic: read + write of every K and V row, plus the slots) / the step
time, max over ranks.

Before timing, the first warm-up step of every workload is verified on the
device: all five index arrays against their definition (computed here with
torch ops from the lengths and page table), every written pool row against its
input row, and a seeded sample of sentinel-filled pool rows outside the step's
slots unchanged.  Inputs rotate over R sets of K/V rows and page tables
(R * per-step inputs > 2 x the 126 MB L2, distinct destination slots per set),
so neither the reads nor the scattered writes are absorbed by L2 between
steps.  The timed steps run as CUDA-graph replays (the way a serving engine
launches a decode step), queued behind a bounded device-side delay so that the
events around them time the kernels, not the host's graph launch.

The default line also carries, as sub-objects, the other workloads (ragged
prefill, Qwen2-72B decode split over the ranks' KV heads, mixed batches), each
verified the same way, and the (f)-row kernels.

  python bench.py [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import yllang_b200 as yl  # noqa: E402
from yllang_b200 import sharding, workloads  # noqa: E402

METRIC = "KV-store GB/s (% of HBM peak) + tokens/s stored; index-build µs/batch"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per step of the timed step's kernels, from one ncu
# capture of three consecutive steps with caches left warm between them (so
# each launch's DRAM writes include the write-back of the lines the previous
# launch left dirty in L2); keyed by (workload, ranks).
STEP_TRAFFIC_NCU: dict = {
    # store_decode_kernel + build_index_kernel of one decode step (256
    # sequences, 32 layers), mean of the capture's steps 2 and 3
    ("llama3_decode", 1): 66_239_872,
}
# Device-side delay queued ahead of each timed region (seconds at the maximum
# SM clock): the host enqueues the graphs while the GPU spins, so the start
# event is taken with the timed work already queued.
LEAD_SECONDS = 2e-3
# Workloads measured as sub-objects of the default line (config names of the
# workload generator); --extras overrides.
DEFAULT_EXTRAS = ("ragged_prefill", "qwen72b_decode", "mixed_ps1_hd64", "mixed_ps16_hd128", "mixed_ps64_hd256")


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_max(x: float, world: int) -> float:
    return sharding.max_over_ranks(x) if world > 1 else x


def reduce_sum(x: float, world: int) -> float:
    return sharding.sum_over_ranks(x) if world > 1 else x


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML polling thread)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons, self.period = [], 0, period_s
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            # NVML enumerates every GPU of the host: find the visible CUDA device by its PCI address
            pr = torch.cuda.get_device_properties(device_index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report that instead of clocks
            self.err = repr(e)
        self._stop = threading.Event()

    def _sample(self):
        nv = self.nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self._t.join()
            self._sample()  # at least one sample at the end of the region

    def summary(self) -> dict:
        if not self.ok:
            return {"error": getattr(self, "err", "nvml unavailable")}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": float(statistics.median(self.samples)) if self.samples else None,
                "sm_max_mhz": float(self.max_mhz), "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workload set-up
# ---------------------------------------------------------------------------
def make_batches(name: str, world: int, pool_bytes: int, rotate: int, whole_job: bool = False):
    """R batches of one workload for this rank (same lengths, different pages).
    whole_job: the batch of all `world` ranks with every KV head (what one
    host runs when it does the whole job's work)."""
    h0, h1 = sharding.head_range(0, world, 8)  # raises unless the 8 KV heads split evenly
    heads = 8 if whole_job else h1 - h0
    if name == "llama3_decode":
        layers, ps, row = 32, 16, heads * 128 * 2
        P = workloads.pool_pages_for(pool_bytes, layers, row, ps)
        mk = lambda r: workloads.llama3_decode(P, batch=256 * world, kv_heads=heads, seed_pages=2 + r)
        desc = {"workload": "llama3_8b_decode", "model_shape": "Llama-3-8B", "global_batch": 256 * world,
                "scaling": "weak"}
    elif name == "ragged_prefill":
        layers, ps, row = 32, 16, heads * 128 * 2
        P = workloads.pool_pages_for(pool_bytes, layers, row, ps)
        mk = lambda r: workloads.ragged_prefill(P, requests=64 * world, kv_heads=heads, seed_pages=2 + r)
        desc = {"workload": "ragged_prefill", "global_batch": 64 * world, "scaling": "weak"}
    elif name == "qwen72b_decode":
        layers, ps, row = 80, 16, heads * 128 * 2
        P = workloads.pool_pages_for(pool_bytes, layers, row, ps)
        mk = lambda r: workloads.qwen72b_decode(P, tp=8 // heads, batch=512, seed_pages=2 + r)
        desc = {"workload": "qwen2_72b_tp_decode", "model_shape": "Qwen2-72B", "global_batch": 512,
                "scaling": "strong"}
    elif name.startswith("mixed"):
        _, ps_s, hd_s = name.split("_")  # mixed_ps16_hd128
        ps, hd = int(ps_s[2:]), int(hd_s[2:])
        layers, row = 4, heads * hd * 2
        P = workloads.pool_pages_for(pool_bytes, layers, row, ps)
        mk = lambda r: workloads.mixed(P, page_size=ps, head_dim=hd, seed_pages=2 + r)
        desc = {"workload": name, "global_batch": 136, "scaling": "strong"}
    else:
        raise SystemExit(f"unknown workload {name}")
    batches = [mk(r) for r in range(rotate)]
    for b in batches:
        b.kv_heads = heads
    desc.update(layers=layers, kv_heads_per_gpu=heads, head_dim=batches[0].head_dim, page_size=ps,
                pool_pages_per_gpu=P, pool_gb_per_gpu=round(2 * layers * P * ps * batches[0].row_bytes / 1e9, 1))
    return batches, desc


class Step:
    """Device-resident inputs and outputs of one rotation set."""

    def __init__(self, b: workloads.Batch, dev, seed: int):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)
        self.b = b
        self.prior, self.new, self.table = t(b.prior_len), t(b.new_len), t(b.page_table)
        g = torch.Generator(device=dev).manual_seed(seed)
        E = b.kv_heads * b.head_dim
        self.k = torch.randn(b.layers, b.tokens, E, generator=g, device=dev, dtype=torch.bfloat16)
        self.v = torch.randn(b.layers, b.tokens, E, generator=g, device=dev, dtype=torch.bfloat16)
        i32 = dict(dtype=torch.int32, device=dev)
        self.out = yl.BatchIndex(torch.empty(b.batch + 1, **i32), torch.empty(b.total_pages, **i32),
                                 torch.empty(b.batch, **i32), torch.empty(b.batch + 1, **i32),
                                 torch.empty(b.tokens, dtype=torch.int64, device=dev))

    def index(self, err=None):
        yl.build_index(self.prior, self.new, self.table, self.b.page_size, num_pages=self.b.num_pages,
                       out=self.out, error_word=err)

    def store(self, k_pool, v_pool, err=None):
        yl.store_kv_cache(self.k, self.v, k_pool, v_pool, self.out.slot_mapping, error_word=err)

    def store_layer(self, layer, k_pool, v_pool, err=None):
        yl.store_kv_cache(self.k[layer], self.v[layer], k_pool[layer], v_pool[layer], self.out.slot_mapping,
                          error_word=err)

    def fused(self, k_pool, v_pool, err=None):
        yl.kv_step(self.prior, self.new, self.table, self.b.page_size, self.k, self.v, k_pool, v_pool, self.out,
                   num_pages=self.b.num_pages, error_word=err)


def input_bytes(b: workloads.Batch) -> int:
    """Device bytes of one rotation set's inputs (K/V rows + page table)."""
    return 2 * b.layers * b.tokens * b.row_bytes + b.page_table.nbytes


def plan(args, world, free_bytes, workload=None):
    """Pick the rotation count (inputs over 2.2 x L2 unless one set already is)
    and the pool size (what is left after the inputs, at most --pool-gb)."""
    probe, _ = make_batches(workload or args.workload, world, 150e9, 1)  # lengths only
    per_set = input_bytes(probe[0])
    R = args.rotate if args.rotate > 0 else max(1, min(8, math.ceil(2.2 * L2_BYTES / per_set)))
    pool_bytes = min(args.pool_gb * 1e9, free_bytes - R * per_set - 12e9)
    assert pool_bytes > 0, "not enough device memory for the inputs"
    return R, pool_bytes, per_set


def device_lead():
    """Queue a bounded device-side delay (torch's clock64 spin kernel, which
    ends on its own after the given cycles) ahead of a timed region."""
    torch.cuda._sleep(int(LEAD_SECONDS * 1.965e9))


def capture(order, launches):
    """One CUDA graph running, for every step r in `order`, the callables
    launches(r) in sequence.  No event nodes go inside the graph: an event
    record between two kernels delays the second by microseconds."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for r in order:
            for fn in launches(r):
                fn()
    return g


def time_graphs(graphs, reps=1):
    """Device time (ms) of replaying `graphs` in order, `reps` times, bracketed
    by events on the launching stream after a synchronize and a device delay
    that keeps the host's graph launch out of the interval."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    device_lead()
    start.record()
    for _ in range(reps):
        for g in graphs:
            g.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def per_launch_us(R, launches, n, reps=4):
    """Mean device time (us) of one step of `launches` over n back-to-back
    steps in a graph (replayed `reps` times after one warm-up replay)."""
    g = capture([j % R for j in range(n)], launches)
    g.replay()
    us = time_graphs([g], reps) * 1e3 / (reps * n)
    del g
    return us


def size_matched_copy_us(dev, nbytes: int, n: int = 64) -> float:
    """Device time (us) of a contiguous streaming kernel that reads nbytes / 2
    bytes and writes them to another buffer (nbytes of reads + writes, the
    step's algorithmic volume), sources and destinations rotating past L2,
    back to back in a CUDA graph: what moving the same bytes costs with no
    scatter and no index build, at this transfer size."""
    half = max(nbytes // 16, 1)  # 8-byte elements: torch's copy then moves wide vectors
    R = max(2, math.ceil(2.2 * L2_BYTES / (8 * half)))
    src = [torch.empty(half, dtype=torch.int64, device=dev) for _ in range(R)]
    dst = [torch.empty(half, dtype=torch.int64, device=dev) for _ in range(R)]
    for t in src:
        t.fill_(1)
    # torch.neg: a vectorised elementwise kernel on the SMs (a same-dtype
    # copy_ would become a copy-engine memcpy, about half as fast)
    us = per_launch_us(R, lambda r: [lambda: torch.neg(src[r], out=dst[r])], n)
    del src, dst
    return us


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class Workload:
    """One workload on this rank: R rotation sets of device inputs and
    outputs, the all-layer pool [2, L, pages * page_size, H_l * D] and the
    step's launches."""

    def __init__(self, name: str, args, shape_world: int, dev, rank: int):
        free, _ = torch.cuda.mem_get_info(dev)
        self.name = name
        self.R, pool_bytes, self.per_set = plan(args, shape_world, free, name)
        self.batches, self.desc = make_batches(name, shape_world, pool_bytes, self.R)
        b0 = self.batches[0]
        self.b0 = b0
        S = b0.num_pages * b0.page_size
        self.pool = torch.empty((2, b0.layers, S, b0.kv_heads * b0.head_dim), dtype=torch.bfloat16, device=dev)
        self.k_pool, self.v_pool = self.pool[0], self.pool[1]
        self.steps = [Step(b, dev, seed=1000 * rank + r) for r, b in enumerate(self.batches)]
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fused = args.path == "fused"

    def launches(self, r):
        s, e = self.steps[r], self.err
        if self.fused:
            return [lambda: s.fused(self.k_pool, self.v_pool, e)]
        return [lambda: s.index(e), lambda: s.store(self.k_pool, self.v_pool, e)]

    def check_err(self, when: str):
        torch.cuda.synchronize()
        bits = int(self.err.item())
        assert bits == 0, f"{self.name}: device error word {bits:#x} ({yl._abi.deverr_names(bits)}) {when}"

    def release(self):
        for n in ("pool", "k_pool", "v_pool", "steps", "batches"):
            setattr(self, n, None)
        gc.collect()
        torch.cuda.empty_cache()


def expected_index(s: Step) -> dict:
    """The five index arrays of a step by their definition, computed on the
    device with torch ops from the step's lengths and page table: page counts
    ceil((prior + new) / page_size) and their running sums, each sequence's
    first pages, its last page's fill, and the slot page * page_size + offset
    of each new token's position."""
    ps = s.b.page_size
    prior, new = s.prior.long().clamp(min=0), s.new.long().clamp(min=0)
    total = prior + new
    W = s.table.shape[1]
    pages = torch.clamp((total + ps - 1) // ps, max=W)
    zero = torch.zeros(1, dtype=torch.int64, device=prior.device)
    qo = torch.cat([zero, new.cumsum(0)])
    seq = torch.repeat_interleave(torch.arange(prior.shape[0], device=prior.device), new)
    pos = prior[seq] + torch.arange(seq.shape[0], device=prior.device) - qo[seq]
    return {"kv_indptr": torch.cat([zero, pages.cumsum(0)]),
            "kv_indices": s.table[torch.arange(W, device=prior.device)[None, :] < pages[:, None]],
            "kv_last_page_len": torch.where(pages == 0, 0, (total - 1) % ps + 1),
            "qo_indptr": qo,
            "slot_mapping": s.table[seq, pos // ps].long() * ps + pos % ps}


def verify_first_step(wl: Workload, sample_rows: int = 1 << 16, seed: int = 17) -> dict:
    """Run the workload's first step once through the timed path and check it
    on the device: every index array element, every pool row the step wrote
    (K and V of every layer) against its input row, and `sample_rows` pool
    rows outside the step's slots -- set to random sentinel values first --
    unchanged.  Raises AssertionError on any difference."""
    s = wl.steps[0]
    b = s.b
    dev = s.k.device
    L, S, E = wl.k_pool.shape
    want = expected_index(s)
    written = want["slot_mapping"]
    g = torch.Generator(device=dev).manual_seed(seed)
    flat = wl.pool.view(2 * L * S, E)
    cand = torch.randint(0, 2 * L * S, (sample_rows,), generator=g, device=dev)
    cand = cand[~torch.isin(cand % S, written)]
    sentinel = torch.randn(cand.shape[0], E, generator=g, device=dev).to(torch.bfloat16)
    flat[cand] = sentinel
    before = flat[cand].clone()  # repeated candidates keep the last sentinel written
    for fn in wl.launches(0):
        fn()
    wl.check_err("on the verified step")
    for name, w in want.items():
        got = getattr(s.out, name)
        assert torch.equal(got[:w.shape[0]].long(), w.long()), f"{wl.name}: {name} differs from its definition"
    for layer in range(L):
        assert torch.equal(wl.k_pool[layer].index_select(0, written), s.k[layer]), f"{wl.name}: K rows, layer {layer}"
        assert torch.equal(wl.v_pool[layer].index_select(0, written), s.v[layer]), f"{wl.name}: V rows, layer {layer}"
    assert torch.equal(flat[cand], before), f"{wl.name}: a pool row outside the step's slots changed"
    n_idx = sum(int(w.numel()) for w in want.values())
    return {"index_elements": n_idx, "pool_rows": 2 * L * b.tokens, "sentinel_rows": int(cand.shape[0]),
            "result": "bit-exact"}


def time_steps(wl: Workload, K: int, chunk: int, clocks=None) -> float:
    """Device time (ms) of K steps on this rank: graphs of `chunk` steps
    (rotation sets in turn) replayed back to back after a device delay."""
    C = min(K, chunk)
    q, rem = divmod(K, C)
    g_main = capture([j % wl.R for j in range(C)], wl.launches)
    g_rem = capture([(q * C + j) % wl.R for j in range(rem)], wl.launches) if rem else None
    g_main.replay()  # untimed graph warm-up
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    region = clocks if clocks is not None else _NoClocks()
    with region:
        device_lead()
        start.record()
        for _ in range(q):
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    del g_main, g_rem
    return ms


class _NoClocks:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def launches_per_step(wl: Workload) -> int:
    """Kernels of this project one timed step launches (see yl_kv_step)."""
    b = wl.b0
    index_launches = 2 if b.batch > 16384 else 1
    return index_launches + 1


def measure(wl: Workload, args, world: int, steps: int, warmup: int, clocks=None) -> dict:
    """Verify, warm up and time one workload on every rank (same collectives
    in the same order on every rank); returns this rank's view of the
    numbers, times as the max over ranks."""
    check = verify_first_step(wl)
    for w in range(1, warmup):
        for fn in wl.launches(w % wl.R):
            fn()
    wl.check_err("during warm-up")
    barrier(world)
    torch.cuda.synchronize()
    ms = time_steps(wl, steps, args.chunk, clocks)
    barrier(world)
    wl.check_err("in the timed steps")
    per_rank = [x / steps * 1e3 for x in sharding.gather_over_ranks(ms)] if world > 1 else [ms / steps * 1e3]
    step_us = max(per_rank)
    n_sep = min(max(steps, 8), 256)
    index_us = reduce_max(per_launch_us(wl.R, lambda r: [lambda: wl.steps[r].index(wl.err)], n_sep), world)
    store_us = reduce_max(per_launch_us(wl.R, lambda r: [lambda: wl.steps[r].store(wl.k_pool, wl.v_pool, wl.err)],
                                        n_sep), world)
    wl.check_err("in the kernel timings")
    b = wl.b0
    return {"verified": check, "step_us": step_us, "per_rank_step_us": per_rank, "index_us": index_us,
            "store_us": store_us, "store_bytes": b.store_bytes(), "step_bytes": b.step_bytes(),
            "index_bytes": b.index_bytes(), "tokens": b.tokens, "launches_per_step": launches_per_step(wl)}


def rank_stats(per_rank: list[float]) -> dict:
    return {"min": round(min(per_rank), 3), "median": round(statistics.median(per_rank), 3),
            "max": round(max(per_rank), 3), "all": [round(x, 3) for x in per_rank]}


def summarize(m: dict, desc: dict, world: int, peak: float) -> dict:
    """Numbers of one measured workload: whole-job GB/s and tokens/s, and the
    roofline of the timed step on one rank (its algorithmic bytes over its
    time, against the measured copy peak)."""
    per_s = m["step_us"] * 1e-6
    step_gbs = m["step_bytes"] / per_s / 1e9
    out = {"workload": desc["workload"], "scaling": desc["scaling"], "global_batch": desc["global_batch"],
           "layers": desc["layers"], "kv_heads_per_gpu": desc["kv_heads_per_gpu"], "head_dim": desc["head_dim"],
           "page_size": desc["page_size"], "tokens_per_step": m["tokens"],
           "step_us": round(m["step_us"], 3),
           "value_gbs": round(m["store_bytes"] * world / per_s / 1e9, 1),
           "tokens_per_s": round(m["tokens"] / per_s, 1),
           "step_gbs_per_gpu": round(step_gbs, 1), "frac_of_measured_hbm": round(step_gbs / peak, 4),
           "index_build_us": round(m["index_us"], 3), "store_us": round(m["store_us"], 3),
           "store_frac_of_measured_hbm": round(m["store_bytes"] / (m["store_us"] * 1e-6) / 1e9 / peak, 4),
           "verified": m["verified"]}
    if world > 1:
        out["per_rank_step_us"] = rank_stats(m["per_rank_step_us"])
    return out


# ---------------------------------------------------------------------------
# CPU baseline: the reference's path as libtorch CPU ops on the host cores
# ---------------------------------------------------------------------------
HOST_ROTATE_BYTES = 600e6  # host input sets cycled through: more than a server's last-level cache


def host_step_setup(b: workloads.Batch, pool_gb: float = 4.0):
    """Host copies of the batch for the CPU arms: the pool scaled down to
    pool_gb (same row and page size; read-only pages alias, written pages
    stay unique) and enough input sets -- K/V rows as raw bf16 bits, page
    tables with their own page ids -- that one pass over them (> 600 MB) does
    not fit a CPU's last-level cache, as the GPU arm rotates past its L2."""
    P = max(workloads.pool_pages_for(pool_gb * 1e9, b.layers, b.row_bytes, b.page_size), b.tokens + 1)
    per_set = 2 * b.layers * b.tokens * b.row_bytes
    R = max(1, min(16, int(math.ceil(HOST_ROTATE_BYTES / per_set))))
    sets = []
    for r in range(R):
        if b.name == "llama3_decode":
            hb = workloads.llama3_decode(P, batch=b.batch, kv_heads=b.kv_heads, layers=b.layers, seed_pages=2 + r)
        elif b.name == "ragged_prefill":
            hb = workloads.ragged_prefill(P, requests=b.batch, kv_heads=b.kv_heads, layers=b.layers,
                                          seed_pages=2 + r)
        else:
            hb = b
        E = hb.kv_heads * hb.head_dim
        rng = np.random.default_rng(r)
        n = hb.layers * hb.tokens * E
        k = np.frombuffer(bytearray(rng.bytes(2 * n)), np.uint16).reshape(hb.layers, hb.tokens, E)
        v = np.frombuffer(bytearray(rng.bytes(2 * n)), np.uint16).reshape(hb.layers, hb.tokens, E)
        sets.append((hb, k, v))
    hb = sets[0][0]
    pool = np.zeros((2, hb.layers, hb.num_pages * hb.page_size, hb.kv_heads * hb.head_dim), np.uint16)
    return sets, pool


def c_port_step(hb, pool, k, v, threads):
    from oracle import kvpath as orc
    out = orc.build_index(hb.prior_len, hb.new_len, hb.page_table, hb.page_size, num_pages=hb.num_pages)
    orc.store(k, v, pool[0], pool[1], out["slot_mapping"], num_slots=pool.shape[2], threads=threads)


class TorchHost:
    """The step as libtorch CPU ops (the reference's host code runs its tensor
    work through libtorch): the index arrays by vectorised torch ops and the
    store as index_copy_ of each layer's K and V rows into the [pages *
    page_size, row] pool views, on torch's intra-op threads."""

    def __init__(self, sets, pool):
        as_t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).view(torch.int16)
        self.sets = [(hb, torch.from_numpy(hb.prior_len), torch.from_numpy(hb.new_len),
                      torch.from_numpy(hb.page_table), as_t(k), as_t(v)) for hb, k, v in sets]
        self.pool = torch.from_numpy(pool).view(torch.int16)

    def step(self, r: int):
        from oracle import kvpath as orc
        hb, prior, new, table, k, v = self.sets[r % len(self.sets)]
        idx = orc.torch_build_index(prior, new, table, hb.page_size)
        orc.torch_store(k, v, self.pool[0], self.pool[1], idx["slot_mapping"])


def timed_host_steps(fn, seconds: float, min_reps: int = 3):
    """Run fn(rep) (after one untimed pass over every set) for about `seconds`;
    returns (seconds per step, steps run)."""
    reps, t0 = 0, time.perf_counter()
    while True:
        fn(reps)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds and reps >= min_reps:
            return el / reps, reps


def cpu_store_step_sample(b: workloads.Batch, seconds: float) -> dict:
    """cpu_baseline of the default line: the libtorch CPU step on all host
    threads for about `seconds`, the pool scaled to 4 GB of host memory and
    the inputs rotating past the last-level cache."""
    torch.set_num_threads(os.cpu_count() or 1)
    sets, pool = host_step_setup(b)
    th = TorchHost(sets, pool)
    for r in range(len(sets)):
        th.step(r)
    per_step, reps = timed_host_steps(th.step, seconds)
    hb = sets[0][0]
    gbs = hb.store_bytes() / per_step / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{reps} full steps of {hb.name} (B={hb.batch}, N={hb.tokens}, L={hb.layers}, "
                      f"row {hb.row_bytes} B) into a {pool.nbytes / 1e9:.1f} GB host pool: index arrays by "
                      f"libtorch CPU ops, store by index_copy_ per layer, {torch.get_num_threads()} intra-op threads, "
                      f"inputs rotating over {len(sets)} sets "
                      f"({len(sets) * 2 * hb.layers * hb.tokens * hb.row_bytes / 1e6:.0f} MB)",
            "ms_per_step": round(per_step * 1e3, 3), "hardware_concurrency": os.cpu_count()}


def ref_make2d_us(b: workloads.Batch, max_seconds: float = 5.0):
    """Time the reference's Make2DIndices (built from its sources, oracle/_ref)
    producing the decode batch's load indices (page size 1 semantics: one
    index per context token), on a sample of sequences, scaled to the batch."""
    import ctypes
    path = os.path.join(ROOT, "oracle", "_ref", "libref_index.so")
    if not os.path.exists(path):
        return None
    f = ctypes.CDLL(path).ref_make2d_indices
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.POINTER(ctypes.c_int64)]
    tot = (b.prior_len.astype(np.int64) + b.new_len)
    W = int(tot.max())
    done_elems, t0, i = 0, time.perf_counter(), 0
    while i < b.batch and time.perf_counter() - t0 < max_seconds:
        rng = np.array([[i * W, 0, int(tot[i])]], np.int64)
        out = np.zeros(int(tot[i]), np.float32)
        n = ctypes.c_int64(0)
        assert f(b.batch, W, rng.ctypes.data, 1, out.ctypes.data, out.size, ctypes.byref(n)) == 0
        done_elems += int(tot[i])
        i += 1
    el = time.perf_counter() - t0
    return {"us_per_batch": round(el / done_elems * float(tot.sum()) * 1e6, 1), "sampled_sequences": i,
            "elements_sampled": done_elems, "kind": "reference",
            "note": "reference Make2DIndices, one libtorch scalar op per element, scaled from the sample"}


def ref_gpu_store(args, b: workloads.Batch, peak: float) -> dict | None:
    """The reference's own store kernel (StoreKVCacheKernel through its
    StoreKVCache launcher, src/kvcache/store_kv_cache.cu:46-163, built from the
    reference sources for sm_100a in oracle/_ref) on this box's GPU, launched
    as the reference launches it: one call per layer (MHAKVCache::StoreKV,
    src/include/kvcache/mha_kvcache.h:76-86), int64 slots, the same batch,
    pool and input rotation as the GPU arm.  The slots come from our index
    build (the reference builds them on the host)."""
    import ctypes
    path = os.path.join(ROOT, "oracle", "_ref", "libref_store.so")
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    if not os.path.exists(path):
        return {"unavailable": "reference store harness not built (make -C oracle ref)"}
    f = ctypes.CDLL(path).ref_store_kv_cache
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 4
    if b.row_bytes not in (512, 1024, 2048, 4096):
        return {"unavailable": f"the reference's Copy<> has no {b.row_bytes}-byte rows"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = Workload(args.workload, args, 1, dev, 0)
    try:
        for s in wl.steps:
            s.index(wl.err)
        wl.check_err("building the slots for the reference store")
        L = wl.b0.layers

        def layer_calls(r):
            s = wl.steps[r]

            def call(layer):
                def go():
                    k, v = s.k[layer], s.v[layer]
                    kc, vc = wl.k_pool[layer], wl.v_pool[layer]
                    rc = f(k.shape[1] * 2, 0, 0, k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                           s.out.slot_mapping.data_ptr(), k.shape[0], k.stride(0), kc.shape[0], kc.stride(0))
                    assert rc == 0, rc
                return go
            return [call(layer) for layer in range(L)]
        for r in range(wl.R):  # eager pass: the rows land where our store puts them
            for fn in layer_calls(r):
                fn()
        torch.cuda.synchronize()
        s = wl.steps[wl.R - 1]
        slots = s.out.slot_mapping
        for layer in range(L):
            assert torch.equal(wl.k_pool[layer].index_select(0, slots), s.k[layer])
        n = max(8, min(64, args.steps))
        us = per_launch_us(wl.R, layer_calls, n, reps=2)
        nbytes = wl.b0.store_bytes()
        gbs = nbytes / (us * 1e-6) / 1e9
        return {"workload": wl.desc["workload"], "launches_per_step": L, "us_per_step": round(us, 3),
                "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
                "kernel": "StoreKVCacheKernel<2048,128,bfloat16,false> (reference source, sm_100a)",
                "timing": f"{n} steps of {L} per-layer launches in one CUDA graph, inputs rotating over {wl.R} sets",
                "checked": "pool rows at the slots equal the input rows"}
    finally:
        wl.release()


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------
def run_reference(args, world, rank):
    """The reference arm: the path on the host cores (rank 0 only), as
    libtorch CPU ops; beside it the C port, the reference's own host index
    helper and the reference's own GPU store kernel."""
    if rank != 0:
        return
    # the whole job of our arm at this world size: its global batch, every KV head
    batches, desc = make_batches(args.workload, world, 150e9, 1, whole_job=True)
    b = batches[0]
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    sets, pool = host_step_setup(b)
    th = TorchHost(sets, pool)
    hb = sets[0][0]
    times = []
    for it in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        th.step(it)
        if it >= args.warmup:
            times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    gbs = hb.store_bytes() / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 4), "higher_is_better": True,
        "scaling": desc.get("scaling", "weak"), "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded lengths and fragmented page tables, random bf16 bit patterns",
        "config": desc,
        "tokens_per_s": round(hb.tokens / per, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "hardware_concurrency": os.cpu_count(),
                         "sample": f"each step: index arrays of {hb.name} (B={hb.batch}, N={hb.tokens}, L={hb.layers}) "
                                   "by libtorch CPU ops, then index_copy_ of every layer's K and V rows into the "
                                   f"[pages * page_size, row] views of a {pool.nbytes / 1e9:.1f} GB host pool, inputs "
                                   f"rotating over {len(sets)} sets; the reference's store exists only as a CUDA "
                                   "kernel, so its semantics run as libtorch CPU ops"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    from oracle import kvpath as orc
    cthreads = orc.max_threads()

    def c_step(r):
        s_hb, k, v = sets[r % len(sets)]
        c_port_step(s_hb, pool, k, v, cthreads)
    for r in range(len(sets)):
        c_step(r)
    per_c, reps = timed_host_steps(c_step, 3.0)
    line["c_port"] = {"value": round(hb.store_bytes() / per_c / 1e9, 3), "unit": "GB/s", "cores": cthreads,
                      "ms_per_step": round(per_c * 1e3, 4), "steps": reps,
                      "what": "the C oracle's index build + pthread store, same sets and pool"}
    mk = ref_make2d_us(b, max_seconds=5.0)
    if mk:
        line["reference_make2dindices"] = mk
    if not args.no_ref_gpu:
        peak, _ = load_peaks()
        try:
            line["reference_gpu_store"] = ref_gpu_store(args, b, peak)
        except Exception as e:  # report, do not lose the CPU line
            line["reference_gpu_store"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    dev = torch.device("cuda", local)
    # replicas: every rank runs the one-GPU shapes; --shape-ranks M: one rank of
    # an M-GPU run's shapes on each GPU (a one-GPU view of a rank's work)
    shape_world = 1 if args.replicas else (args.shape_ranks or world)
    peak, peak_kind = load_peaks()
    wl = Workload(args.workload, args, shape_world, dev, rank)
    desc = dict(wl.desc)
    K = args.steps
    clocks = ClockSampler(local)  # samples during the timed region only
    m = measure(wl, args, world, K, args.warmup, clocks)
    n_layer = min(K, 16)
    L = wl.b0.layers
    layer_us = reduce_max(per_launch_us(wl.R, lambda r: [(lambda l: (lambda: wl.steps[r].store_layer(
        l, wl.k_pool, wl.v_pool, wl.err)))(layer) for layer in range(L)], n_layer), world) / L
    wl.check_err("in the per-layer store timing")
    copy_us = reduce_max(size_matched_copy_us(dev, m["step_bytes"]), world)
    e2e = None
    if not args.no_e2e:
        if wl.per_set <= 4e9:
            e2e = run_e2e(args, wl.steps[:min(wl.R, 2)], wl.k_pool, wl.v_pool, wl.err, world)
        else:
            e2e = {"value": None, "unit": "GB/s", "skipped": f"one step's inputs are {wl.per_set / 1e9:.0f} GB"}
    b0 = wl.b0
    wl.release()

    # the other workloads, every rank, in the same order
    extras = {}
    names = [n for n in (args.extras.split(",") if args.extras is not None else DEFAULT_EXTRAS) if n]
    for name in names:
        if name == args.workload:
            continue
        sub = Workload(name, args, shape_world, dev, rank)
        try:
            sm = measure(sub, args, world, min(K, args.extra_steps), 3)
            extras[name] = summarize(sm, sub.desc, world, peak)
            extras[name]["gpu_launches_per_step"] = sm["launches_per_step"]
        finally:
            sub.release()

    per_step_s = m["step_us"] * 1e-6
    total_store = reduce_sum(float(m["store_bytes"]), world)
    value = total_store / per_step_s / 1e9
    if rank != 0:
        return
    step_gbs = m["step_bytes"] / per_step_s / 1e9
    store_gbs = m["store_bytes"] / (m["store_us"] * 1e-6) / 1e9
    traffic = args.traffic if args.traffic is not None else STEP_TRAFFIC_NCU.get((args.workload, shape_world))
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(m["step_us"] / 1e3, 5), "higher_is_better": True,
        "scaling": desc.pop("scaling"), "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded lengths and fragmented page tables, K/V N(0,1) cast to bf16",
        "config": dict(desc, parallelism=(f"replicas x{world}" if args.replicas else f"kv-head shard x{world}")
                       if world > 1 else ("single GPU" if shape_world == 1
                                          else f"one rank of a kv-head shard x{shape_world}, alone"),
                       path=(("yl_kv_step (serial)" if os.environ.get("YL_STEP_MODE") == "serial"
                              else "yl_kv_step (index build and store as programmatic dependents)") if wl.fused
                             else "build_index + store_kv_cache"),
                       l2=f"inputs rotate over {wl.R} sets ({wl.R * wl.per_set / 1e6:.0f} MB > 2 x L2), "
                          "distinct destination slots per set"),
        "tokens_per_s": round(m["tokens"] / per_step_s, 1),
        "pct_hbm": round(100 * value / (peak * world), 2),
        "step_us": round(m["step_us"], 3),
        "index_build_us": round(m["index_us"], 3),
        "index_gbs": round(m["index_bytes"] / (m["index_us"] * 1e-6) / 1e9, 1),
        "verified": m["verified"],
        "roofline": {"bound": "hbm",
                     "kernel": "the timed step (yl_kv_step: index build + store of every layer)",
                     "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(step_gbs / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} hbm_gbs (copy)",
                     "algorithmic_bytes_per_launch": m["step_bytes"],
                     "launch_us": round(m["step_us"], 3),
                     "timing": f"{K} steps as CUDA-graph replays behind a device delay, events on the launching "
                               "stream, max over ranks",
                     "store_kernel": {"us": round(m["store_us"], 3), "achieved": round(store_gbs, 1),
                                      "frac": round(store_gbs / peak, 4),
                                      "algorithmic_bytes_per_launch": m["store_bytes"],
                                      "timing": "the all-layer store alone, back-to-back launches in one graph"}},
        "size_matched_copy": {"us": round(copy_us, 3), "step_over_copy": round(m["step_us"] / copy_us, 3),
                              "what": "torch's vectorised elementwise kernel streaming the step's algorithmic "
                                      "bytes (half read, half written), inputs past L2, back to back in a graph"},
        "per_layer_store": {"launches_per_step": L, "us_per_launch": round(layer_us, 3),
                            "gbs": round(m["store_bytes"] / L / (layer_us * 1e-6) / 1e9, 1)},
        "gpu_launches": K * m["launches_per_step"],
        "clocks": clocks.summary(),
        "workloads": extras,
    }
    if world > 1:
        line["per_rank_step_us"] = rank_stats(m["per_rank_step_us"])
    if e2e is not None:
        line["e2e"] = e2e
    if not args.no_gather:
        line["embedding_gather"] = bench_gather(dev, peak)
    if not args.no_qkv:
        line["qkv_norm_rope_store"] = bench_qkv(dev, peak)
    if not args.no_pool:
        line["page_allocator"] = bench_pool(dev)
    if not args.no_make2d:
        line["make2dindices"] = bench_make2d(dev, b0, peak)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_store_step_sample(b0, seconds=args.cpu_seconds)
    print(json.dumps(line), flush=True)


def bench_gather(dev, peak: float, tokens: int = 4096, sets: int = 32) -> dict:
    """The embedding lookup on the store's copy engine: Qwen3-0.6B's token
    table (151936 x 1024 bf16, 311 MB > L2), `tokens` uniformly drawn ids per
    launch, ids and outputs rotating over `sets` sets.  Algorithmic bytes per
    launch: ids + the gathered rows read + the output rows written."""
    V, E = 151936, 1024
    table = torch.randn(V, E, device=dev, dtype=torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(7)
    ids = [torch.randint(0, V, (tokens,), generator=g, device=dev, dtype=torch.int32) for _ in range(sets)]
    outs = [torch.empty(tokens, E, dtype=torch.bfloat16, device=dev) for _ in range(sets)]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for r in range(sets):
        yl.gather_rows(ids[r], table, out=outs[r], error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(outs[0], table[ids[0].long()])
    us = per_launch_us(sets, lambda r: [lambda: yl.gather_rows(ids[r], table, out=outs[r], error_word=err)], 256)
    nbytes = tokens * 4 + 2 * tokens * E * 2
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": f"qwen3-0.6b token embedding {V}x{E} bf16, {tokens} ids (int32)", "us_per_launch": round(us, 3),
            "algorithmic_bytes_per_launch": nbytes, "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
            "kernel": "gather_rows_kernel", "timing": "256 back-to-back launches in one CUDA graph; table rows may hit L2"}


def bench_make2d(dev, b: workloads.Batch, peak: float, sets: int = 4) -> dict:
    """The reference's Make2DIndices on the decode batch's load ranges
    ({row * W, 0, prior + new} per sequence: one index per context token, as
    NextBatch calls it at page size 1), one yl_make_2d_indices launch each,
    outputs rotating over `sets` buffers.  Algorithmic bytes per launch: the
    ranges read + the int64 indices written."""
    tot = b.prior_len.astype(np.int64) + b.new_len
    W = int(tot.max())
    r = np.stack([np.arange(b.batch, dtype=np.int64) * W, np.zeros(b.batch, np.int64), tot], axis=1)
    ranges = torch.from_numpy(np.ascontiguousarray(r)).to(dev)
    n = int(tot.sum())
    outs = [torch.empty(n, dtype=torch.int64, device=dev) for _ in range(sets)]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    yl.make_2d_indices(ranges, out=outs[0], error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    last = (b.batch - 1) * W + torch.arange(int(tot[-1]), device=dev)
    assert torch.equal(outs[0][:int(tot[0])], torch.arange(int(tot[0]), device=dev))
    assert torch.equal(outs[0][n - int(tot[-1]):], last)
    us = per_launch_us(sets, lambda j: [lambda: yl.make_2d_indices(ranges, out=outs[j], error_word=err)], 256)
    nbytes = b.batch * 24 + n * 8
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": f"{b.name} load ranges: {b.batch} ranges, {n} indices (int64)", "us_per_batch": round(us, 3),
            "algorithmic_bytes_per_launch": nbytes, "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
            "kernel": "make_2d_indices_kernel",
            "timing": f"256 back-to-back launches in one CUDA graph, outputs rotating over {sets} buffers "
                      f"({sets * n * 8 / 1e6:.0f} MB, may stay in L2)"}


def bench_qkv(dev, peak: float) -> dict:
    """One attention layer's input stage on the Qwen3-8B shape (32 Q heads,
    8 KV heads, head_dim 128, bf16, rope_theta 1e6): the fused Q/K RMSNorm +
    rotary + K/V store kernel against the unfused sequence of the same work
    (flashinfer's Q norm, K norm and rotary kernels, then store_kv_cache), at
    decode (256 tokens) and prefill (4096 tokens).  Inputs rotate over sets
    larger than 2 x L2.  Algorithmic bytes per launch: Q/K/V rows read, Q and
    K/V rows written, slots, positions and the tokens' cos/sin rows read."""
    from yllang_b200.attention import _flashinfer

    fi = _flashinfer()
    Hq, Hk, D = 32, 8, 128
    S = 1 << 16
    k_cache = torch.zeros(S, Hk * D, dtype=torch.bfloat16, device=dev)
    v_cache = torch.zeros_like(k_cache)
    cs = yl.rope_cos_sin_cache(32768, D, theta=1e6, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    qw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    out = {}
    for name, N in (("decode", 256), ("prefill", 4096)):
        set_bytes = N * (2 * Hq + 2 * Hk) * D * 2
        R = max(2, math.ceil(2.2 * L2_BYTES / set_bytes))
        sets = []
        for r in range(R):
            qkv = torch.randn(N, (Hq + 2 * Hk) * D, generator=g, device=dev).to(torch.bfloat16)
            q = qkv[:, :Hq * D].view(N, Hq, D)
            k = qkv[:, Hq * D:(Hq + Hk) * D].view(N, Hk, D)
            v = qkv[:, (Hq + Hk) * D:].view(N, Hk, D)
            slots = torch.randperm(S, generator=g, device=dev)[:N]
            pos = torch.randint(0, 32768, (N,), generator=g, device=dev)
            sets.append((qkv, q, k, v, slots, pos, torch.empty(N, Hq, D, dtype=torch.bfloat16, device=dev)))

        def fused(r):
            _, q, k, v, slots, pos, q_out = sets[r]
            return [lambda: yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=qw, k_weight=kw,
                                                   eps=1e-6, cos_sin_cache=cs, positions=pos, q_out=q_out)]

        def unfused(r):
            _, q, k, v, slots, pos, q_out = sets[r]
            kn = torch.empty(N, Hk, D, dtype=torch.bfloat16, device=dev)

            def rope():
                fi.rope.apply_rope_with_cos_sin_cache_inplace(pos, q_out.view(N, Hq * D), kn.view(N, Hk * D), D, cs,
                                                              is_neox=True)
            return [lambda: fi.norm.rmsnorm(q, qw, eps=1e-6, out=q_out),
                    lambda: fi.norm.rmsnorm(k, kw, eps=1e-6, out=kn), rope,
                    lambda: yl.store_kv_cache(kn.view(N, Hk * D), v.reshape(N, Hk * D), k_cache, v_cache, slots)]

        for fn in fused(0) + unfused(0):
            fn()
        torch.cuda.synchronize()
        us = per_launch_us(R, fused, 128)
        try:
            us_unfused = per_launch_us(R, unfused, 128)
            how = "4 launches in one CUDA graph"
        except Exception as e:  # a library op that cannot be captured: time it eagerly
            us_unfused = None
            how = f"not captured: {type(e).__name__}"
        nbytes = N * (2 * Hq + 4 * Hk) * D * 2 + N * 16 + N * D * 4
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"tokens": N, "us_per_launch": round(us, 3), "algorithmic_bytes_per_launch": nbytes,
                     "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
                     "unfused_us": None if us_unfused is None else round(us_unfused, 3), "unfused_timing": how}
        del sets
    out["workload"] = "qwen3-8b attention input, 32 q heads, 8 kv heads, head_dim 128, bf16, one layer"
    out["kernel"] = "qkv_norm_rope_store_kernel"
    out["unfused"] = "flashinfer rmsnorm(q), rmsnorm(k), apply_rope_with_cos_sin_cache_inplace, store_kv_cache"
    return out


def bench_pool(dev, B: int = 256, ps: int = 16, steps: int = 256) -> dict:
    """Page allocation per decode step for a Llama-3-8B-sized batch (256
    sequences, one new token each, page 16): the device pool
    (yl_reserve_pages, one launch, lengths advanced on the device) against the
    host KVCacheManager path it replaces (per-request Reserve, then the
    page-table sync to the device), timed over `steps` consecutive steps."""
    C = yl.load_extension()
    W = 80  # 512 prior + 2 * 256 timed + 256 warm-up tokens = 80 pages of 16
    P = B * W
    rng = np.random.default_rng(12)
    prior0 = rng.integers(128, 512, B).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)

    def fresh():
        pool = yl.DevicePagePool(P, dev)
        table = torch.full((B, W), -1, dtype=torch.int32, device=dev)
        pool.reserve(table, t(np.zeros(B)), t(prior0), ps)
        return pool, table, t(prior0)

    ones = torch.ones(B, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    pool, table, prior = fresh()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(steps):
            pool.reserve(table, prior, ones, ps, error_word=err)
            prior.add_(ones)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        for _ in range(steps):
            prior.add_(ones)
    # capture ran nothing; one untimed replay each, then the timed one (two
    # replays add 2 * steps / ps pages per sequence: the pool and rows hold them)
    g.replay()
    g2.replay()
    torch.cuda.synchronize()
    both = time_graphs([g]) * 1e3 / steps
    add_only = time_graphs([g2]) * 1e3 / steps
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    del g, g2

    m = C.KVCacheManager(P, B, W, ps, str(dev))
    rows = [m.AllocateTableSlot() for _ in range(B)]
    lens = prior0.astype(np.int64).copy()
    for i in range(B):
        m.Reserve(rows[i], int(lens[i]))
    m.SyncPageTable()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        lens += 1
        for i in range(B):
            m.Reserve(rows[i], int(lens[i]))
        m.SyncPageTable()
    torch.cuda.synchronize()
    host_us = (time.perf_counter() - t0) * 1e6 / steps
    return {"workload": f"decode, {B} sequences, 1 token each, page {ps}, {steps} consecutive steps",
            "device_reserve_us": round(both - add_only, 3),
            "device_timing": "one yl_reserve_pages launch per step in a CUDA graph, minus the same graph's "
                             "length update alone",
            "host_manager_us": round(host_us, 2),
            "host_timing": "wall clock of KVCacheManager.Reserve per request + SyncPageTable per step (C++ front "
                           "end called from Python)"}


def gpu_local_cpus(device_index: int) -> set[int] | None:
    """The CPUs NVML names as local to the GPU (its NUMA node), within this
    process's allowed set; None when NVML cannot say."""
    try:
        import pynvml
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(device_index)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        n = os.cpu_count() or 64
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
        cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


def run_e2e(args, steps, k_pool, v_pool, err, world):
    """The same step through the public API with host inputs: every step
    copies its K/V rows, lengths and page table from pinned host memory,
    builds the index, stores, and reads the error word back.  The process
    runs on the GPU's local CPUs while it allocates and fills the pinned
    buffers and runs the steps (so the buffers sit on the GPU's NUMA node, as
    a serving process bound to its GPU has them); the CPU set is restored
    afterwards."""
    dev = steps[0].k.device
    before = os.sched_getaffinity(0)
    local = gpu_local_cpus(dev.index if dev.index is not None else 0)
    if local is not None:
        os.sched_setaffinity(0, local)
    try:
        out = _run_e2e(args, steps, k_pool, v_pool, err, world)
    finally:
        os.sched_setaffinity(0, before)
    out["host_cpus"] = f"{len(local)} GPU-local CPUs (NVML affinity)" if local is not None else "unbound"
    return out


def _run_e2e(args, steps, k_pool, v_pool, err, world):
    R = len(steps)
    dev = steps[0].k.device
    host = []
    for s in steps:
        host.append({n: getattr(s, n).cpu().pin_memory() for n in ("k", "v", "prior", "new", "table")})
    dk = {n: torch.empty_like(getattr(steps[0], n)) for n in ("k", "v", "prior", "new", "table")}
    out = steps[0].out
    err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
    E = min(args.steps, args.e2e_steps)
    b = steps[0].b

    # K and V cross PCIe on two copy streams (two DMA engines), the small
    # inputs on the step's stream; the step waits for both copies
    main = torch.cuda.current_stream(dev)
    side = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    done = torch.cuda.Event()

    def one(r):
        h = host[r]
        for n in dk:
            if dk[n].shape != h[n].shape:
                dk[n] = torch.empty(h[n].shape, dtype=h[n].dtype, device=dev)
        done.record(main)  # the previous step has read dk["k"], dk["v"]
        for i, n in enumerate(("k", "v")):
            side[i].wait_event(done)
            with torch.cuda.stream(side[i]):
                dk[n].copy_(h[n], non_blocking=True)
            ready[i].record(side[i])
        for n in ("prior", "new", "table"):
            dk[n].copy_(h[n], non_blocking=True)
        for ev in ready:
            main.wait_event(ev)
        yl.kv_step(dk["prior"], dk["new"], dk["table"], b.page_size, dk["k"], dk["v"], k_pool, v_pool, out,
                   num_pages=b.num_pages, error_word=err)
        err_host.copy_(err, non_blocking=True)

    for r in range(min(3, R)):
        one(r)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    for j in range(E):
        one(j % R)
    end.record()
    torch.cuda.synchronize()
    ms = reduce_max(start.elapsed_time(end), world)
    h2d = sum(host[0][n].nbytes for n in ("k", "v", "prior", "new", "table"))
    per = ms / 1e3 / E
    total = reduce_sum(float(b.store_bytes()), world)
    return {"value": round(total / per / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": 4, "steps": E, "ms_per_step": round(ms / E, 4),
            "h2d_gbs": round(h2d / per / 1e9, 2),
            "bound": "the step's host-to-device copies (PCIe): h2d_gbs is their achieved rate",
            "path": "pinned host -> device copies (K and V on two copy streams), yllang_b200.kv_step, "
                    "error word -> host"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="llama3_decode")
    ap.add_argument("--path", choices=["fused", "separate"], default="fused",
                    help="timed step: yl_kv_step, or build_index + store_kv_cache as two calls")
    ap.add_argument("--rotate", type=int, default=0, help="input sets cycled through (0: enough to exceed 2.2 x L2)")
    ap.add_argument("--chunk", type=int, default=256, help="steps per captured CUDA graph")
    ap.add_argument("--pool-gb", type=float, default=150.0)
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--no-gather", action="store_true", help="skip the embedding-gather line")
    ap.add_argument("--no-qkv", action="store_true", help="skip the fused norm/rotary/store line")
    ap.add_argument("--no-pool", action="store_true", help="skip the page-allocator line")
    ap.add_argument("--no-make2d", action="store_true", help="skip the range-expansion (Make2DIndices) line")
    ap.add_argument("--replicas", action="store_true",
                    help="every rank runs the full-head one-GPU workload (a sanity check of the head-sharded run)")
    ap.add_argument("--shape-ranks", type=int, default=0,
                    help="run one rank's shapes of a kv-head shard over this many GPUs (0: the real world size)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu DRAM bytes per timed step (from the committed profile) to report")
    ap.add_argument("--extras", default=None,
                    help="comma-separated workloads measured as sub-objects (default: " + ",".join(DEFAULT_EXTRAS)
                         + "; empty: none)")
    ap.add_argument("--extra-steps", type=int, default=20, help="timed steps of each sub-workload")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="reference arm: skip timing the reference's own GPU store kernel")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # at least three untimed steps
    world, rank, local = dist_setup()
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
