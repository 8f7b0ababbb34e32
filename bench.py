"""Benchmark of the 4-bit paged decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: launched by torch.distributed.run, one process per GPU)

Workload per GPU (weak scaling): 64 sequences of a global ragged batch of
64*N sequences with lengths ~ U[128, 8192] (seeded), assigned to ranks by
longest-first bin packing on token count; Hq=32, Hkv=8, D=128, block_size 16,
pages randomly permuted in a pool sized to the tokens, int32 block tables,
K/V ~ N(0,1) fp16 quantized into the pool by the store kernel.  One step =
append 1 new token per sequence + ragged decode of every sequence, as ONE
launch (kv_append_decode_paged_batched: the split-K decode kernel quantizes
each sequence's new token itself and merges the partials in the same
launch), i.e. one attention layer of one decode step.  The pool (~290
MB/GPU) is larger than L2, so no flush is needed.

Reported: tok/s (sequences decoded per second, all GPUs), µs/step, the
decode kernel's algorithmic HBM GB/s against MEASURED_PEAKS.json, an
end-to-end figure through the public Python API with pinned host buffers,
and the CPU oracle timed on this host.  ``--impl reference`` times the
reference path's CPU restatement (oracle/kvq_oracle.c) on the same workload,
and beside it the reference's own CUDA kernels (its extension built
unmodified into oracle/_ref) driven as its vLLM adapter drives them.
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
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("µs/decode-step & achieved HBM GB/s (% of 8 TB/s) for 4-bit paged decode; "
          "tok/s @1/2/4/8")
SEQS_PER_GPU = 64
HQ, HKV, D, BS = 32, 8, 128, 16
LMIN, LMAX = 128, 8192
SEED = 1234
C5_SEQS, C5_LMIN, C5_LMAX, C5_STEPS = 256, 512, 4096, 128
C5_REF_STEPS = 16
E2E_GRAPH_STEPS = 128  # e2e steps per captured CUDA graph (the first input and last output copy of a graph cannot overlap compute)
DECODE_LAUNCHES = 2000  # decode-only launches timed back to back for the roofline (whatever --steps is)
DECODE_GRAPH_LAUNCHES = 200  # decode-only launches per captured CUDA graph
E2E_EAGER_STEPS = 500  # e2e steps issued eagerly through the public API
NOMINAL_HBM_GBS = 8000.0


# --------------------------------------------------------------------- setup
def global_lengths(world: int):
    g = torch.Generator().manual_seed(SEED)
    return torch.randint(LMIN, LMAX + 1, (SEQS_PER_GPU * world,), generator=g).tolist()


def rank_lengths(world: int, rank: int):
    from slm_turbo_b200.sharding import partition_sequences
    lengths = global_lengths(world)
    parts = partition_sequences(lengths, world)
    return [lengths[i] for i in parts[rank]]


def build_workload(lengths, rank: int):
    """Host tensors of the rank's pool: block tables, slot ids, seeded K/V, q."""
    g = torch.Generator().manual_seed(SEED + 1000 + rank)
    L1 = [L + 1 for L in lengths]  # each step appends one token at position L
    nblk = [(L + BS - 1) // BS for L in L1]
    total = sum(nblk)
    perm = torch.randperm(total, generator=g)
    bt = torch.zeros(len(lengths), max(nblk), dtype=torch.int32)
    o = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    return dict(lengths=lengths, seq_lens1=torch.tensor(L1, dtype=torch.int32), block_tables=bt,
                num_blocks=total, gen=g)


def prefill_cache(w, dev):
    """Quantize N(0,1) history tokens into the permuted pool (chunked)."""
    from slm_turbo_b200.kernels import kv_dequant as kd
    cache = torch.zeros(w["num_blocks"], BS, HKV, D + 8, dtype=torch.uint8, device=dev)
    bt = w["block_tables"].to(torch.int64)
    g = torch.Generator(device=dev).manual_seed(SEED + 7)
    for i, L in enumerate(w["lengths"]):
        t = torch.arange(L)
        slots = (bt[i, t // BS] * BS + t % BS).to(dev)
        k = torch.randn(L, HKV, D, device=dev, generator=g, dtype=torch.float32).half()
        v = torch.randn(L, HKV, D, device=dev, generator=g, dtype=torch.float32).half()
        kd.kv_quantize_store(k, v, cache, slots, BS)
    torch.cuda.synchronize(dev)
    return cache


def step_slots(w):
    bt = w["block_tables"].to(torch.int64)
    pos = torch.tensor(w["lengths"], dtype=torch.int64)
    return bt[torch.arange(len(w["lengths"])), pos // BS] * BS + pos % BS


def algorithmic_bytes(w):
    """Bytes the decode kernel must move: the packed slot of every context
    token and kv head (D/2 K + D/2 V + 8 ruler bytes), one 4-byte block-table
    entry per page, q in (fp16) and out (fp32) per query head, and the
    sequence lengths; plus the store's bytes (new K/V in, slots out)."""
    toks = int(w["seq_lens1"].sum())
    pages = sum((L + BS - 1) // BS for L in w["seq_lens1"].tolist())
    B = len(w["lengths"])
    decode = toks * HKV * (D + 8) + pages * 4 + B * HQ * D * (2 + 4) + B * 4
    store = B * HKV * D * 2 * 2 + B * HKV * (D + 8) + B * 8
    return decode, store


# -------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                r = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._h is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons)}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ profiles
def profiled_traffic(dec_bytes):
    """DRAM read+write bytes per decode launch from the committed ncu summary
    (`traffic_bytes_per_launch:` of a capture whose workload moved
    `traffic_algorithmic_bytes:`), scaled to this workload's algorithmic
    bytes (traffic grows in proportion to them); None if absent."""
    p = ROOT / "profiles" / "decode_splitk_c3.txt"
    if not p.exists():
        return None
    vals = {}
    for line in p.read_text().splitlines():
        for key in ("traffic_bytes_per_launch:", "traffic_algorithmic_bytes:"):
            if line.startswith(key):
                try:
                    vals[key] = int(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    t = vals.get("traffic_bytes_per_launch:")
    base = vals.get("traffic_algorithmic_bytes:")
    if t is None:
        return None
    return int(round(t * dec_bytes / base)) if base else t


def measured_peak():
    try:
        mp = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(mp["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except Exception:
        return 6650.0, "profiling-recipe fallback 6.65 TB/s (of fallback)"


# ---------------------------------------------------------------- CPU legs
def cpu_step_time(w_host, cache_np, reps_seconds=10.0, max_reps=50):
    """Time the oracle on this host: store of the step's tokens + decode of
    every sequence (all host threads).  Returns (seconds per step, reps, threads)."""
    import oracle
    B = len(w_host["lengths"])
    g = torch.Generator().manual_seed(99)
    q = torch.randn(B, HQ, D, generator=g).half()
    k = torch.randn(B, HKV, D, generator=g).half()
    v = torch.randn(B, HKV, D, generator=g).half()
    slots = step_slots(w_host)
    nthreads = os.cpu_count() or 1
    times = []
    t_all = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        oracle.kv_store(k, v, cache_np, slots)
        oracle.paged_decode(q, cache_np, w_host["block_tables"], w_host["seq_lens1"], BS, HKV,
                            nthreads=nthreads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > reps_seconds or len(times) >= max_reps:
            break
    return statistics.median(times), len(times), nthreads


def cpu_cache_for(w_host):
    """Fill a host pool with the oracle store (the CPU path's own setup)."""
    import oracle
    cache = np.zeros((w_host["num_blocks"], BS, HKV, D + 8), np.uint8)
    bt = w_host["block_tables"].to(torch.int64)
    g = torch.Generator().manual_seed(SEED + 7)
    for i, L in enumerate(w_host["lengths"]):
        t = torch.arange(L)
        slots = bt[i, t // BS] * BS + t % BS
        k = torch.randn(L, HKV, D, generator=g).half()
        v = torch.randn(L, HKV, D, generator=g).half()
        oracle.kv_store(k, v, cache, slots)
    return cache


# --------------------------------------------------------------------- main
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def workload_config(w, world):
    toks = int(w["seq_lens1"].sum())
    return {"workload": "C3 ragged paged 4-bit decode: per GPU 64 seqs U[128,8192] (+1 appended token/step), "
                        "Hq32/Hkv8/D128, block 16, permuted page pool, int32 block tables",
            "seqs_per_gpu": len(w["lengths"]), "global_seqs": SEQS_PER_GPU * world,
            "ctx_tokens_rank0": toks, "pool_mb_rank0": round(w["num_blocks"] * BS * HKV * (D + 8) / 1e6, 1),
            "l2": "inputs larger than L2 (page pool > 126 MB), no flush",
            "parallelism": f"seq-partition x{world} (no collective)"}


def run_reference(args):
    """CPU restatement of the reference path (oracle/kvq_oracle.c, all host
    threads) on rank 0's workload.  Each step is a bounded sample: a fixed
    subset of the sequences sized so the K+W steps take ~2 minutes at most;
    time is scaled to the full workload by context tokens."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    lengths = rank_lengths(world, 0)
    w = build_workload(lengths, 0)
    cache_np = cpu_cache_for(w)
    B = len(lengths)
    g = torch.Generator().manual_seed(99)
    q = torch.randn(B, HQ, D, generator=g).half()
    k = torch.randn(B, HKV, D, generator=g).half()
    v = torch.randn(B, HKV, D, generator=g).half()
    slots = step_slots(w)
    nthreads = os.cpu_count() or 1

    def one(idx):
        oracle.kv_store(k[idx], v[idx], cache_np, slots[idx])
        oracle.paged_decode(q[idx], cache_np, w["block_tables"][idx], w["seq_lens1"][idx], BS, HKV,
                            nthreads=nthreads)

    full = torch.arange(B)
    t0 = time.perf_counter()
    one(full)
    t_full = time.perf_counter() - t0
    budget = 100.0 / max(args.steps + args.warmup, 1)
    n = B if t_full <= budget else max(1, int(B * budget / t_full))
    idx = torch.randperm(B, generator=torch.Generator().manual_seed(5))[:n].sort().values
    toks_all = float(w["seq_lens1"].sum())
    toks_s = float(w["seq_lens1"][idx].sum())
    for _ in range(args.warmup):
        one(idx)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one(idx)
    dt = (time.perf_counter() - t0) / max(args.steps, 1) * (toks_all / toks_s)
    value = B / dt
    sample = (f"{n} of {B} rank-0 sequences per step ({int(toks_s)} of {int(toks_all)} context tokens), "
              f"time scaled by tokens; oracle/kvq_oracle.c, OpenMP {nthreads} threads, f64 attention")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": workload_config(w, world),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": nthreads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    try:
        line["reference_cuda_same_box"] = reference_cuda_same_box(w, args.steps, args.warmup)
    except Exception as exc:  # a report beside the CPU arm, never a reason to fail it
        line["reference_cuda_same_box"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    print(json.dumps(line), flush=True)
    return 0


def reference_cuda_same_box(w, steps, warmup):
    """The reference's own CUDA kernels (its extension, built unmodified into
    oracle/_ref) on this GPU, driven as its vLLM adapter drives them for one
    decode step of one layer: kv_quantize_store_cuda for the step's tokens
    (adapters/vllm_adapter.py:185-203), then seq_lens.tolist() and one
    kv_dequant_decode_per_token_paged_attention_cuda launch per request
    (:246-284).  Pool filled by the reference's own store kernel.  Timed with
    CUDA events around whole steps, host loop included."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    from oracle.build_ref import load_ref
    ref = load_ref()
    if ref is None:
        return {"unavailable": "reference extension not built into oracle/_ref"}
    _, _, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B = len(w["lengths"])
    bt = w["block_tables"].to(torch.int64)
    cache = torch.zeros(w["num_blocks"], BS, HKV, D + 8, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(SEED + 7)
    for i, L in enumerate(w["lengths"]):
        t = torch.arange(L)
        slots = (bt[i, t // BS] * BS + t % BS).to(dev)
        k = torch.randn(L, HKV, D, device=dev, generator=g, dtype=torch.float32).half()
        v = torch.randn(L, HKV, D, device=dev, generator=g, dtype=torch.float32).half()
        ref.kv_quantize_store_cuda(k, v, cache, slots, BS)
    q = torch.randn(B, HQ, D, device=dev, generator=g).half()
    k_new = torch.randn(B, HKV, D, device=dev, generator=g).half()
    v_new = torch.randn(B, HKV, D, device=dev, generator=g).half()
    slots_d = step_slots(w).to(dev)
    sl_d = w["seq_lens1"].to(dev)
    rows = [bt[r].to(dev).contiguous() for r in range(B)]
    out = torch.empty(B, HQ, D, dtype=torch.float16, device=dev)

    def step():
        ref.kv_quantize_store_cuda(k_new, v_new, cache, slots_d, BS)
        for r, L in enumerate(sl_d.tolist()):
            o = ref.kv_dequant_decode_per_token_paged_attention_cuda(
                q[r:r + 1].permute(1, 0, 2).contiguous(), cache, rows[r], int(L), BS, HKV)
            out[r] = o.permute(1, 0, 2)[0]

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    n = max(steps, 5)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / n
    return {"value": B / (ms * 1e-3), "unit": "tok/s", "ms_per_step": ms, "steps": n,
            "mode": "reference CUDA kernels (oracle/_ref, built unmodified for sm_100a) on this GPU: one "
                    "store launch + seq_lens.tolist() + one decode launch per request, as the reference "
                    "adapter runs a decode step"}


def run_ours(args):
    world, rank, local = dist_env()
    if world != args.gpus:
        args.gpus = world
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    from slm_turbo_b200.kernels import kv_dequant as kd

    lengths = rank_lengths(world, rank)
    w = build_workload(lengths, rank)
    cache = prefill_cache(w, dev)
    B = len(lengths)
    bt_d = w["block_tables"].to(dev)
    sl_d = w["seq_lens1"].to(dev)
    g = torch.Generator(device=dev).manual_seed(SEED + 11 + rank)
    q = torch.randn(B, HQ, D, device=dev, generator=g).half()
    k_new = torch.randn(B, HKV, D, device=dev, generator=g).half()
    v_new = torch.randn(B, HKV, D, device=dev, generator=g).half()
    out = torch.empty(B, HQ, D, dtype=torch.float32, device=dev)
    maxlen = int(w["seq_lens1"].max())

    def step():
        kd.kv_append_decode_paged_batched(q, k_new, v_new, cache, bt_d, sl_d, out=out, max_seq_len=maxlen)

    def decode_only():
        kd.kv_decode_paged_batched(q, cache, bt_d, sl_d, out=out, max_seq_len=maxlen)

    stream = torch.cuda.current_stream(dev)

    def barrier():
        if pg is not None:
            pg.barrier()

    def max_over_ranks(x):
        if pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up, then K timed steps (device-timed, max over ranks) ----
    # The K steps are issued as ONE replay of a CUDA graph that holds K
    # captured calls of the public API (captured before the timed region), as
    # a serving engine issues decode steps; every step does its full work.
    # The same K steps issued eagerly from Python are timed too
    # (eager_ms_per_step): there the host's per-call cost shows.
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    assert kd.read_device_errors(dev) == 0, "device error word set during warm-up"
    steps_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(steps_graph):
        for _ in range(args.steps):
            step()
    steps_graph.replay()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(dev.index)
    clk.__enter__()  # sampled across the K steps and the decode-only leg below
    ev0.record(stream)
    steps_graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms_step = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    del steps_graph
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    eager_ms_step = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)

    # ---- dominant kernel: the decode launch alone, DECODE_LAUNCHES back to back ----
    # replayed from a CUDA graph of DECODE_GRAPH_LAUNCHES captured calls, so
    # that the figure is the kernel's own (a busy host issuing launches one
    # by one from Python can leave the GPU idle between them); the same
    # launches issued eagerly are timed too (decode_eager_us)
    n_rep_dec = max(1, max(DECODE_LAUNCHES, args.steps) // DECODE_GRAPH_LAUNCHES)
    n_dec = n_rep_dec * DECODE_GRAPH_LAUNCHES
    dec_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dec_graph):
        for _ in range(DECODE_GRAPH_LAUNCHES):
            decode_only()
    dec_graph.replay()
    torch.cuda.synchronize(dev)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for _ in range(n_rep_dec):
        dec_graph.replay()
    d1.record(stream)
    torch.cuda.synchronize(dev)
    dec_ms = max_over_ranks(d0.elapsed_time(d1) / n_dec)
    del dec_graph
    d0.record(stream)
    for _ in range(n_dec):
        decode_only()
    d1.record(stream)
    torch.cuda.synchronize(dev)
    clk.__exit__()
    dec_eager_ms = max_over_ranks(d0.elapsed_time(d1) / n_dec)
    dec_bytes, store_bytes = algorithmic_bytes(w)
    peak, peak_src = measured_peak()
    achieved = dec_bytes / (dec_ms * 1e-3) / 1e9

    # ---- end to end through the public API with pinned host buffers ----
    # Each step's inputs (q, new K/V, lengths) travel in ONE pinned host ->
    # device copy and its fp32 output in one device -> host copy, on their
    # own copy streams, double-buffered: the input copy of step t+1 and the
    # output copy of step t-1 run while step t computes, as a serving loop
    # would run them.  The page pool and the block tables are the engine's
    # resident state and stay on the device.
    h_parts = [q.cpu(), k_new.cpu(), v_new.cpu(), w["seq_lens1"]]
    offs, o = [], 0
    for t in h_parts:
        offs.append(o)
        o += (t.numel() * t.element_size() + 255) // 256 * 256
    h_in = torch.empty(o, dtype=torch.uint8).pin_memory()
    for t, off in zip(h_parts, offs):
        nb = t.numel() * t.element_size()
        h_in[off:off + nb].copy_(t.contiguous().view(-1).view(torch.uint8))
    h2d = sum(t.numel() * t.element_size() for t in h_parts)
    d_in = [torch.empty(o, dtype=torch.uint8, device=dev) for _ in range(2)]

    def views(buf):
        out_v = []
        for t, off in zip(h_parts, offs):
            nb = t.numel() * t.element_size()
            out_v.append(buf[off:off + nb].view(t.dtype).view(t.shape))
        return out_v

    d_views = [views(bf) for bf in d_in]
    d_out = [torch.empty(B, HQ, D, dtype=torch.float32, device=dev) for _ in range(2)]
    h_out = [torch.empty(B, HQ, D, dtype=torch.float32).pin_memory() for _ in range(2)]
    d2h = h_out[0].numel() * h_out[0].element_size()
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of slot landed
    ev_done = [torch.cuda.Event() for _ in range(2)]   # compute of slot finished
    ev_out = [torch.cuda.Event() for _ in range(2)]    # output of slot copied out

    def e2e_run(n):
        cs = torch.cuda.current_stream(dev)  # compute stream (the capture stream under a graph)
        h2d_stream.wait_stream(cs)
        d2h_stream.wait_stream(cs)

        def copy_in(i):
            sl = i & 1
            with torch.cuda.stream(h2d_stream):
                if i >= 2:
                    h2d_stream.wait_event(ev_done[sl])  # slot's previous inputs consumed
                d_in[sl].copy_(h_in, non_blocking=True)
                ev_in[sl].record(h2d_stream)

        copy_in(0)
        for i in range(n):
            sl = i & 1
            if i + 1 < n:
                copy_in(i + 1)  # prefetch: overlaps step i's compute
            cs.wait_event(ev_in[sl])
            if i >= 2:
                cs.wait_event(ev_out[sl])  # slot's previous output read out
            dq, dk, dv, dsl = d_views[sl]
            kd.kv_append_decode_paged_batched(dq, dk, dv, cache, bt_d, dsl, out=d_out[sl], max_seq_len=maxlen)
            ev_done[sl].record(cs)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(ev_done[sl])
                h_out[sl].copy_(d_out[sl], non_blocking=True)
                ev_out[sl].record(d2h_stream)
        cs.wait_stream(h2d_stream)
        cs.wait_stream(d2h_stream)

    # (a) eager: the public API called once per step from Python, as a
    # serving loop without CUDA graphs calls it
    e2e_run(4)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_eager = max(E2E_EAGER_STEPS, args.steps)
    e0.record(stream)
    e2e_run(n_eager)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_eager_ms = max_over_ranks(e0.elapsed_time(e1) / n_eager)
    assert torch.equal(h_out[(n_eager - 1) & 1], d_out[(n_eager - 1) & 1].cpu()), "e2e output copy mismatch"

    # (b) the same steps replayed from a CUDA graph of E2E_GRAPH_STEPS
    # pipelined steps (the public API calls captured once), as a serving
    # engine runs decode; the host issues one graph launch per
    # E2E_GRAPH_STEPS steps.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        e2e_run(E2E_GRAPH_STEPS)
    graph.replay()
    torch.cuda.synchronize(dev)
    barrier()
    n_rep = max(1, args.steps // E2E_GRAPH_STEPS)
    e0.record(stream)
    for _ in range(n_rep):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / (n_rep * E2E_GRAPH_STEPS))
    last = (E2E_GRAPH_STEPS - 1) & 1
    assert torch.equal(h_out[last], d_out[last].cpu()), "e2e output copy mismatch"
    del graph
    assert kd.read_device_errors(dev) == 0, "device error word set during timing"

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cache_np = cpu_cache_for(w)
        t_cpu, reps, nthreads = cpu_step_time(w, cache_np, reps_seconds=args.cpu_seconds)
        cpu = {"value": B / t_cpu, "unit": "tok/s", "cores": nthreads, "kind": "port",
               "sample": f"full rank-0 workload ({B} seqs, store + decode), median of {reps} steps, "
                         f"oracle/kvq_oracle.c (OpenMP, f64 attention)"}

    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if rank != 0:
        return 0
    total_seqs = SEQS_PER_GPU * world  # every sequence of the global batch decodes once per step
    tok_s = total_seqs / (ms_step * 1e-3)
    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "us_per_step": ms_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": workload_config(w, world),
        "decode_us": dec_ms * 1e3, "decode_hbm_gbs": achieved, "decode_eager_us": dec_eager_ms * 1e3,
        "step": "one launch: new token quantized into the cache + decode (append fused)",
        "step_issue": f"the K steps replayed from one CUDA graph of K captured public-API calls; issued "
                      f"eagerly from Python the same K steps take {eager_ms_step * 1e3:.1f} us per step",
        "eager_ms_per_step": eager_ms_step,
        "hbm_pct_of_8tbs": 100.0 * achieved / NOMINAL_HBM_GBS,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": profiled_traffic(dec_bytes),
                     "kernel": "decode_splitk_kernel<128,1,PAGED,8,PK> (partials merged inside the launch)",
                     "algorithmic_bytes_per_launch": dec_bytes, "peak_source": peak_src,
                     "timing": f"{n_dec} decode-only launches back to back between two CUDA events, replayed "
                               f"from a CUDA graph of {DECODE_GRAPH_LAUNCHES} captured calls"},
        "e2e": {"value": total_seqs / (e2e_ms * 1e-3),
                "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "mode": f"public API (kv_append_decode_paged_batched) captured as a CUDA graph of "
                        f"{E2E_GRAPH_STEPS} steps; per step one pinned H2D of q, new K/V and lengths and "
                        "one D2H of the fp32 output, each on its own copy stream, double-buffered against "
                        "the compute; the page pool and block tables stay resident on the device",
                "ms_per_step": e2e_ms,
                "eager": {"value": total_seqs / (e2e_eager_ms * 1e-3), "unit": "tok/s",
                          "ms_per_step": e2e_eager_ms,
                          "mode": f"the same {n_eager} steps issued eagerly, one public-API call per step "
                                  "from Python (no CUDA graph)"}},
        "gpu_launches": args.steps,  # one decode_splitk_kernel (append fused) per step
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------- extra workload lines
def _dist_setup():
    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    return world, rank, dev, pg


def _timed(dev, pg, fn, steps, warmup, n_sets=1):
    """Warm-up, then `steps` calls of fn(i) replayed from one CUDA graph (the
    calls captured once, before the timed region) between CUDA events on the
    current stream, barrier + synchronize on both sides; max over ranks.
    Returns (ms per step, clocks, eager ms per step): the last is the same
    steps issued from Python, where a short kernel can be host-bound."""
    for i in range(max(warmup, 3)):
        fn(i % n_sets)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(steps):
            fn(i % n_sets)
    graph.replay()
    torch.cuda.synchronize(dev)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def max_ranks(ms):
        if pg is None:
            return ms
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(max(1, 2000 // max(steps, 1))):  # the sampler sees >= ~2000 steps
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    reps = max(1, 2000 // max(steps, 1))
    if pg is not None:
        pg.barrier()
    ms = max_ranks(e0.elapsed_time(e1) / (steps * reps))
    del graph
    e0.record(stream)
    for i in range(steps):
        fn(i % n_sets)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    eager = max_ranks(e0.elapsed_time(e1) / steps)
    return ms, clk.summary(), eager


def run_c2(args):
    """uniform batched decode over the standalone
    per-channel layout, B=16 x 2048 tokens, Hq32/Hkv8, D = --head-dim.  The
    working set of one step (34 MB at D=128) fits in L2, so the timed steps
    rotate over 4 independent input sets (136 MB) and every step reads cold
    data.  One step = one batched decode launch; sequences are split over
    ranks (weak scaling)."""
    world, rank, dev, pg = _dist_setup()
    from slm_turbo_b200.kernels import kv_dequant as kd
    B, Hq, KV, S, Dh, NSETS = 16, 32, 8, 2048, args.head_dim, 4
    g = torch.Generator(device=dev).manual_seed(SEED + 20 + rank)
    sets = []
    for _ in range(NSETS):
        k = torch.randn(B, KV, S, Dh, device=dev, generator=g).half()
        v = torch.randn(B, KV, S, Dh, device=dev, generator=g).half()
        kp, ks, kz = kd.kv_quantize_per_channel(k)
        vp, vs, vz = kd.kv_quantize_per_channel(v)
        q = torch.randn(B, Hq, Dh, device=dev, generator=g).half()
        sets.append((q, kp, ks, kz, vp, vs, vz, torch.empty(B, Hq, Dh, dtype=torch.float32, device=dev)))
        del k, v
    torch.cuda.synchronize(dev)

    def step(i):
        q, kp, ks, kz, vp, vs, vz, out = sets[i]
        kd.kv_dequant_decode_attention_batched(q, kp, ks, kz, vp, vs, vz, out=out)

    ms, clocks, eager_ms = _timed(dev, pg, step, args.steps, args.warmup, NSETS)
    assert kd.read_device_errors(dev) == 0
    byts = B * KV * S * (Dh // 2) * 2 + B * KV * Dh * 2 * 4 + B * Hq * Dh * (2 + 4)
    peak, peak_src = measured_peak()
    achieved = byts / (ms * 1e-3) / 1e9
    if pg is not None:
        pg.destroy_process_group()
    if rank != 0:
        return 0
    print(json.dumps({
        "metric": METRIC, "value": B * world / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "eager_ms_per_step": eager_ms,
        "step_issue": "steps replayed from CUDA graphs of the captured public-API calls (>= 2000 in the timed "
                      "region); eager_ms_per_step: the same steps issued from Python",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"C2 per-channel batched decode: per GPU 16 seqs x 2048, Hq32/Hkv8/D{Dh}",
                   "l2": f"{NSETS} rotating input sets ({NSETS * byts / 1e6:.0f} MB > L2)",
                   "parallelism": f"seq-partition x{world} (no collective)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": f"decode_splitk_kernel<{Dh},1,PER_CHANNEL,8,1>",
                     "algorithmic_bytes_per_launch": byts, "peak_source": peak_src},
        "e2e": None, "gpu_launches": args.steps, "clocks": clocks, "cpu_baseline": None}), flush=True)
    return 0


def run_prefill(args):
    """Row a6 / the tensor-core prefill kernel: per-channel prefill attention
    (kv_dequant_prefill_attention) of M = S = 4096 query rows over the packed
    keys/values, Hq32/Hkv8, D = --head-dim, causal.  The reference's own CUDA
    prefill kernel (oracle/_ref, unmodified) runs on the same inputs on the
    same GPU for the comparison and for an output cross-check.  Two rotating
    input sets (q + out > L2 each).  One step = one prefill launch; ranks run
    independent replicas."""
    world, rank, dev, pg = _dist_setup()
    from slm_turbo_b200.kernels import kv_dequant as kd
    H, KV, M, S, Dh, NSETS = 32, 8, 4096, 4096, args.head_dim, 2
    g = torch.Generator(device=dev).manual_seed(SEED + 40 + rank)
    sets = []
    for _ in range(NSETS):
        k = torch.randn(KV, S, Dh, device=dev, generator=g).half()
        v = torch.randn(KV, S, Dh, device=dev, generator=g).half()
        kp, ks, kz = kd.kv_quantize_per_channel(k)
        vp, vs, vz = kd.kv_quantize_per_channel(v)
        q = torch.randn(H, M, Dh, device=dev, generator=g).half()
        sets.append((q, kp, ks, kz, vp, vs, vz))
        del k, v
    torch.cuda.synchronize(dev)

    def step(i):
        kd.kv_dequant_prefill_attention(*sets[i], causal=True, num_kv_heads=KV)

    steps = min(args.steps, 50)
    ms, clocks, eager_ms = _timed(dev, pg, step, steps, args.warmup, NSETS)
    assert kd.read_device_errors(dev) == 0
    keys = sum(min(S, m + 1) for m in range(M))
    flops = 4 * Dh * H * keys  # QK^T and PV, 2 flops per multiply-add
    mp = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(mp.get("bf16_tflops", 1590.0))
    peak_src = "MEASURED_PEAKS.json bf16_tflops (of measured)" if mp else "profiling-recipe fallback (of fallback)"
    achieved = flops / (ms * 1e-3) / 1e12
    ref_line = {"unavailable": "reference extension not built into oracle/_ref"}
    try:
        from oracle.build_ref import load_ref
        ref = load_ref()
        if ref is not None and rank == 0:
            ours = kd.kv_dequant_prefill_attention(*sets[0], causal=True, num_kv_heads=KV)
            theirs = ref.kv_dequant_prefill_attention_cuda(*sets[0], 16, 64 if Dh == 64 else 32, True, True, KV)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(3):
                ref.kv_dequant_prefill_attention_cuda(*sets[i % NSETS], 16, 64 if Dh == 64 else 32, True, True, KV)
            e1.record()
            torch.cuda.synchronize(dev)
            rms = e0.elapsed_time(e1) / 3
            ref_line = {"ms_per_step": rms, "tflops": flops / (rms * 1e-3) / 1e12, "speedup_ours": rms / ms,
                        "max_abs_diff_vs_ours": float((ours - theirs).abs().max()),
                        "mode": "reference kv_dequant_prefill_attention_cuda (built unmodified, sm_100a), "
                                "3 launches between CUDA events, same inputs"}
    except Exception as exc:  # the comparison is informative, never the measured line
        ref_line = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    if pg is not None:
        pg.destroy_process_group()
    if rank != 0:
        return 0
    print(json.dumps({
        "metric": "prefill rows/s (per-channel 4-bit prefill attention)", "value": M * world / (ms * 1e-3),
        "unit": "rows/s", "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms,
        "eager_ms_per_step": eager_ms,
        "step_issue": "steps replayed from CUDA graphs of the captured public-API calls; eager_ms_per_step: "
                      "the same steps issued from Python",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"prefill (row a6): H32/KV8/D{Dh}, M=S=4096, causal, per-channel rulers",
                   "l2": f"{NSETS} rotating input sets (q 32 MB + out 64 MB each)",
                   "parallelism": f"replicas x{world} (no collective)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "kernel": f"prefill_pc_kernel<{Dh}>",
                     "algorithmic_flops_per_launch": flops, "peak_source": peak_src,
                     "note": "mma.sync m16n8k16 tiles; the peak is cuBLAS bf16 on tcgen05"},
        "reference_cuda_same_box": ref_line,
        "e2e": None, "gpu_launches": steps, "clocks": clocks, "cpu_baseline": None}), flush=True)
    return 0


def run_c4(args):
    """long-context decode, 4 sequences of 131,072 tokens,
    Hq64/Hkv8/D128, paged per-token 4-bit, block 16; split-K over the
    sequence inside a GPU, kv heads sharded over ranks (strong scaling: each
    rank holds 8/N kv heads and their 64/N query heads).  One step = append
    one token per sequence + decode."""
    world, rank, dev, pg = _dist_setup()
    from slm_turbo_b200.kernels import kv_dequant as kd
    from slm_turbo_b200.sharding import shard_kv_heads
    B, L, Hq_all, KV_all = 4, 131072, 64, 8
    heads = shard_kv_heads(KV_all, world, rank)
    kv = len(heads)
    hq = Hq_all // KV_all * kv
    nblk = (L + 1 + BS - 1) // BS
    gen = torch.Generator().manual_seed(SEED + 40)
    perm = torch.randperm(B * nblk, generator=gen)
    bt = perm.view(B, nblk).to(torch.int32).to(dev)
    cache = torch.empty(B * nblk, BS, kv, D + 8, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(SEED + 41 + rank)
    chunk = 16384
    for b in range(B):
        for t0 in range(0, L, chunk):
            t = torch.arange(t0, min(L, t0 + chunk), device=dev)
            slots = bt[b, t // BS].to(torch.int64) * BS + t % BS
            k = torch.randn(len(t), kv, D, device=dev, generator=g).half()
            v = torch.randn(len(t), kv, D, device=dev, generator=g).half()
            kd.kv_quantize_store(k, v, cache, slots, BS)
    sl = torch.full((B,), L + 1, dtype=torch.int32, device=dev)
    pos = torch.full((B,), L, dtype=torch.int64, device=dev)
    slots_new = bt[torch.arange(B, device=dev), pos // BS].to(torch.int64) * BS + pos % BS
    q = torch.randn(B, hq, D, device=dev, generator=g).half()
    k_new = torch.randn(B, kv, D, device=dev, generator=g).half()
    v_new = torch.randn(B, kv, D, device=dev, generator=g).half()
    out = torch.empty(B, hq, D, dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)

    def step(_):  # one launch: the new token of every sequence appended, then decoded
        kd.kv_append_decode_paged_batched(q, k_new, v_new, cache, bt, sl, out=out, max_seq_len=L + 1)

    ms, clocks, eager_ms = _timed(dev, pg, step, args.steps, args.warmup)
    assert kd.read_device_errors(dev) == 0
    byts = B * (L + 1) * kv * (D + 8) + B * nblk * 4 + B * hq * D * (2 + 4)
    peak, peak_src = measured_peak()
    achieved = byts / (ms * 1e-3) / 1e9
    if pg is not None:
        pg.destroy_process_group()
    if rank != 0:
        return 0
    print(json.dumps({
        "metric": METRIC, "value": B / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "eager_ms_per_step": eager_ms,
        "step_issue": "steps replayed from CUDA graphs of the captured public-API calls (>= 2000 in the timed "
                      "region); eager_ms_per_step: the same steps issued from Python",
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "C4 long-context paged 4-bit decode: 4 seqs x 131072 (+1 appended token/step), "
                               "Hq64/Hkv8/D128, block 16",
                   "kv_heads_per_gpu": kv, "pool_mb_per_gpu": round(B * nblk * BS * kv * (D + 8) / 1e6, 1),
                   "l2": "inputs larger than L2, no flush",
                   "parallelism": f"kv-head shards x{world} (no collective)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "decode_splitk_kernel<...,APPEND> (one launch per step, rank 0)",
                     "algorithmic_bytes_per_launch": byts, "peak_source": peak_src},
        "e2e": None, "gpu_launches": args.steps, "clocks": clocks, "cpu_baseline": None}), flush=True)
    return 0


C5_CHILD = r"""
import json, os, sys, time
sys.path.insert(0, sys.argv[1])
model_dir, mode, n_seqs, lmin, lmax, steps, seed = sys.argv[2], sys.argv[3], *map(int, sys.argv[4:9])
import torch
from slm_turbo_b200.adapters import vllm_adapter as ad
ad.register_plugin()
if mode == "refkern":
    # the reference's own CUDA kernels (oracle/_ref), driven as its adapter
    # drives them: one store launch, seq_lens.tolist(), one decode launch per
    # request per layer (adapters/vllm_adapter.py:185-203, 246-284)
    from oracle.build_ref import load_ref
    ref = load_ref()
    Impl = ad.QuantizedKVAttentionImpl
    def store(self, layer, key, value, kv_cache, slot_mapping):
        if kv_cache is not None and kv_cache.numel():
            ref.kv_quantize_store_cuda(key.contiguous(), value.contiguous(), kv_cache, slot_mapping,
                                       kv_cache.shape[1])
    def decode(self, query, kv_cache, md, out, n):
        for r, L in enumerate(md.seq_lens[:n].tolist()):
            if L > 0:
                o = ref.kv_dequant_decode_per_token_paged_attention_cuda(
                    query[r:r + 1].permute(1, 0, 2).contiguous(), kv_cache,
                    md.block_table[r].to(torch.int64).contiguous(), int(L), kv_cache.shape[1], kv_cache.shape[2])
                out[r] = o.permute(1, 0, 2)[0].to(out.dtype)
        return out
    Impl.do_kv_cache_update = store
    Impl._decode_attention = decode
from vllm import LLM, SamplingParams
# the reference's store and decode kernels accept fp16 only
# (kernels/kv_dequant_cuda.cu:359-360, 419-420): its arm runs the model in fp16
kw = dict(model=model_dir, load_format="dummy", skip_tokenizer_init=True,
          dtype="float16" if mode == "refkern" else "bfloat16",
          attention_backend="CUSTOM", block_size=16, max_model_len=lmax + steps + 32, max_num_seqs=n_seqs,
          max_num_batched_tokens=16384, gpu_memory_utilization=0.6, enable_prefix_caching=False, seed=0)
if mode == "ours-graph":
    kw.update(compilation_config={"mode": 0, "cudagraph_mode": "FULL_DECODE_ONLY",
                                  "cudagraph_capture_sizes": [n_seqs]})
else:
    kw.update(enforce_eager=True)
llm = LLM(**kw)
g = torch.Generator().manual_seed(seed)
lens = torch.randint(lmin, lmax + 1, (n_seqs,), generator=g).tolist()
prompts = [{"prompt_token_ids": torch.randint(3, 32000, (L,), generator=g).tolist()} for L in lens]
llm.generate(prompts[:4], SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True), use_tqdm=False)
def timed(max_tokens):
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    outs = llm.generate(prompts, SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True),
                        use_tqdm=False)
    e1.record()
    torch.cuda.synchronize()
    assert all(len(o.outputs[0].token_ids) == max_tokens for o in outs)
    return e0.elapsed_time(e1) * 1e-3, time.perf_counter() - t0
t1, w1 = timed(1)
t2, w2 = timed(1 + steps)
from slm_turbo_b200.kernels import kv_dequant as kd
err = kd.read_device_errors(torch.device("cuda", 0), reset=False)
print("RESULT " + json.dumps({"mode": mode, "prefill_s": t1, "total_s": t2, "decode_s": t2 - t1,
                              "wall_decode_s": w2 - w1, "ctx_tokens": sum(lens), "device_errors": err,
                              "decode_tok_s": n_seqs * steps / (t2 - t1)}), flush=True)
"""


def _c5_config(d):
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 2048,
           "intermediate_size": 5632, "num_hidden_layers": 22, "num_attention_heads": 32,
           "num_key_value_heads": 4, "head_dim": 64, "vocab_size": 32000, "max_position_embeddings": 8192,
           "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "hidden_act": "silu", "tie_word_embeddings": False,
           "bos_token_id": 1, "eos_token_id": 2, "torch_dtype": "bfloat16"}
    (Path(d) / "config.json").write_text(json.dumps(cfg))


def c5_engine(mode, args, steps=None):
    """Run one C5 engine (a child process: its own CUDA context and vLLM
    state) and return its RESULT dict."""
    steps = C5_STEPS if steps is None else steps
    import subprocess
    import tempfile
    world, rank, local = dist_env()
    with tempfile.TemporaryDirectory() as d:
        _c5_config(d)
        env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0", CUDA_VISIBLE_DEVICES=str(local))
        for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "LOCAL_WORLD_SIZE",
                  "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID"):
            env.pop(k, None)
        proc = subprocess.run([sys.executable, "-c", C5_CHILD, str(ROOT), d, mode, str(C5_SEQS), str(C5_LMIN),
                               str(C5_LMAX), str(steps), str(SEED + 50 + rank)],
                              env=env, capture_output=True, text=True, timeout=3000)
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")]
    if proc.returncode != 0 or not lines:
        return {"mode": mode, "failed": (proc.stdout[-1500:] + proc.stderr[-2500:])}
    return json.loads(lines[-1][len("RESULT "):])


def run_reference_c5(args):
    """C5 with the reference's own CUDA kernels (oracle/_ref) in the same vLLM
    engine, driven by its adapter's per-request decode loop (eager: the loop
    syncs seq_lens to the host every step).  Rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle.build_ref import built_path
    if built_path() is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference extension not built into oracle/_ref"}))
        return 0
    # the reference's per-request loop makes ~5,600 decode launches per step
    # (256 requests x 22 layers): a bounded sample of 16 decode steps
    r = c5_engine("refkern", args, steps=C5_REF_STEPS)
    v = r.get("decode_tok_s")
    print(json.dumps({"metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": world,
                      "steps": C5_REF_STEPS, "warmup": 1, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                      "config": {"workload": "C5 (see the ours line); reference CUDA kernels, per-request loop; "
                                             "model in fp16 (the reference kernels reject bf16)"},
                      "engine": r}), flush=True)
    return 0


def run_c5(args):
    """model-level continuous-batching decode through vLLM's
    CUSTOM backend (this package's adapter and kernels) on a random-init
    TinyLlama-shape Llama (22 layers, hidden 2048, 32/4 heads, head_dim 64,
    SwiGLU 5632, vocab 32000, bf16 weights), 256 requests per GPU with
    prompt lengths U[512, 4096], 128 decode steps, block 16.  Each GPU runs
    its own replica (data parallel; weak scaling).  decode tok/s = 256 x 128
    / (time of generate with 129 new tokens - time with 1 new token), both
    device-timed; the prefill is the difference's common part.  CUDA graphs
    for the decode steps (vLLM FULL_DECODE_ONLY, no torch.compile) and, beside
    it, the same engine eager."""
    world, rank, local = dist_env()
    res = {m: c5_engine(m, args) for m in ("ours-graph", "ours-eager")}
    vals = [res[m].get("decode_tok_s") for m in res]
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        t = torch.tensor([min(res[m].get("decode_s", float("inf")) for m in res)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        slowest = float(t.item())
        dist.destroy_process_group()
    else:
        slowest = min(res[m].get("decode_s", float("inf")) for m in res)
    if rank != 0:
        return 0
    best = max((v for v in vals if v), default=None)
    value = C5_SEQS * C5_STEPS * world / slowest if slowest != float("inf") else None
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": C5_STEPS, "warmup": 1,
        "ms_per_step": slowest / C5_STEPS * 1e3 if value else None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random token ids)",
        "config": {"workload": "C5 TinyLlama-shape model (22L, hidden 2048, 32/4 heads, D64, SwiGLU 5632, "
                               "vocab 32000, bf16), vLLM CUSTOM backend, 256 requests/GPU, prompts U[512,4096], "
                               "128 decode steps, block 16, 4-bit paged KV",
                   "parallelism": f"data-parallel replicas x{world}"},
        "best_rank0_decode_tok_s": best, "engines_rank0": res}), flush=True)
    return 0


def run_ncu_case(args):
    """A few untimed launches of one kernel on a bench workload, for an ncu
    capture (`-k regex:... -s 2 -c 1`): `decode` / `fused` = the C3 decode
    (plain, or with the step's append) on rank 0's pool, `prefill` = the
    per-channel prefill of `--workload prefill` (D = --head-dim).  Five
    launches, then a device-error check; nothing is timed or printed but a
    status line."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from slm_turbo_b200.kernels import kv_dequant as kd
    if args.ncu_case == "prefill":
        H, KV, M, S, Dh = 32, 8, 4096, 4096, args.head_dim
        g = torch.Generator(device=dev).manual_seed(SEED + 40)
        k = torch.randn(KV, S, Dh, device=dev, generator=g).half()
        v = torch.randn(KV, S, Dh, device=dev, generator=g).half()
        kp, ks, kz = kd.kv_quantize_per_channel(k)
        vp, vs, vz = kd.kv_quantize_per_channel(v)
        q = torch.randn(H, M, Dh, device=dev, generator=g).half()
        for _ in range(5):
            kd.kv_dequant_prefill_attention(q, kp, ks, kz, vp, vs, vz, causal=True, num_kv_heads=KV)
    else:
        w = build_workload(rank_lengths(1, 0), 0)
        cache = prefill_cache(w, dev)
        B = len(w["lengths"])
        bt_d, sl_d = w["block_tables"].to(dev), w["seq_lens1"].to(dev)
        g = torch.Generator(device=dev).manual_seed(SEED + 11)
        q = torch.randn(B, HQ, D, device=dev, generator=g).half()
        k_new = torch.randn(B, HKV, D, device=dev, generator=g).half()
        v_new = torch.randn(B, HKV, D, device=dev, generator=g).half()
        out = torch.empty(B, HQ, D, dtype=torch.float32, device=dev)
        maxlen = int(w["seq_lens1"].max())
        for _ in range(5):
            if args.ncu_case == "fused":
                kd.kv_append_decode_paged_batched(q, k_new, v_new, cache, bt_d, sl_d, out=out, max_seq_len=maxlen)
            else:
                kd.kv_decode_paged_batched(q, cache, bt_d, sl_d, out=out, max_seq_len=maxlen)
    torch.cuda.synchronize(dev)
    err = kd.read_device_errors(dev)
    print(f"ncu case {args.ncu_case}: 5 launches, device errors {err}")
    return 0 if err == 0 else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--workload", default="c3", choices=["c3", "c2", "c4", "c5", "prefill"],
                    help="c3 (default, the metric's config); c2 / c4 / c5 / prefill print extra lines")
    ap.add_argument("--head-dim", type=int, default=128, choices=[64, 80, 128], help="c2 and prefill only")
    ap.add_argument("--ncu-case", choices=["decode", "fused", "prefill"], default=None,
                    help="untimed launches of one kernel for an ncu capture (no JSON line)")
    args = ap.parse_args()
    if args.ncu_case:
        return run_ncu_case(args)
    if args.impl == "reference" and args.workload == "c5":
        return run_reference_c5(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c2":
        return run_c2(args)
    if args.workload == "c4":
        return run_c4(args)
    if args.workload == "c5":
        return run_c5(args)
    if args.workload == "prefill":
        return run_prefill(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
