#!/usr/bin/env python3
"""Benchmark of the DSA sparse-attention operator (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|5]

Workload (`value`): benchmark config 2 (decode, 64 query tokens per GPU, one
32768-slot sequence per token, 2.42 GB pool per GPU).  For N > 1 (torchrun,
one process per GPU) every rank serves its own 64-token batch from its own
pool — weak scaling by batch rows, no collective on the hot path; the job's
throughput is 64*N tokens / (max over ranks of the mean step time).

A step = one call of the operator over the whole batch.  Timing: CUDA events
on the launching stream around each call; the L2 is flushed before every
timed call, outside the events: a 256 MiB memset, then a 256 MiB read of a
second buffer, so every call reads its inputs from HBM and the memset's dirty
lines are written back before the call rather than during it (a memset alone
left up to 126 MB of write-back inside the next call: +6 us on config 2).  Reported:
  value         query tokens/s, whole job, inputs resident in HBM
  e2e           the same through the public Python API with pinned host
                inputs copied in and outputs copied out inside the timed
                region, every step: steps back to back over 4 rotating
                decode batches (inputs larger than L2 together), copies in,
                kernel and copies out on three streams so that one step's
                copies overlap its neighbours' kernels; wall clock over all
                steps.  `e2e_serial` = one step at a time (flush, copy in,
                call, copy out, synchronise)
  roofline      the split-KV kernel (the merge of split tokens is fused into
                it): gathered-KV bytes / its mean duration (events recorded
                by the library around that launch); `traffic` comes from the
                stored ncu capture named in `traffic_source`
  cpu_baseline  the reference's naive kernel (compiled from its source for
                CPU, oracle/_ref) on a bounded sample of the same workload
  configs       configs 1, 3, 4 and 5 at one GPU (N=1 only): us per call,
                gathered GB/s, fraction of the measured peak, tokens/s, and
                the CPU reference's tokens/s on a sample of each
  config5       config 5 strong scaling: one 1024-token batch of 256
                sequences sharded by whole sequences over the N GPUs; max over
                ranks of the mean step, job tokens/s, and each rank's kernel
                time next to its step time
  small_batches the operator on the first 1, 2, 4, 6 and 8 tokens of config 2
                (the batch sizes the reference's CUDA kernel accepts; the
                reference arm times that kernel on the same inputs)
  paged, fp8_kv, indexer, indexer_ragged, decode_step, decode_step_graph, pipelined: see their "how"
                fields
`--impl reference` runs the reference's CPU path (and, where the GPU and its
build are present, the reference's own CUDA kernel on the small batches), on
rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import gc
import importlib
import json
import os
import statistics
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
PKG = "karnbirkhera-mlsys2026-dsa_sparse_attention_b200"

METRIC = ("µs/call and gathered-KV HBM GB/s (% of 8 TB/s) at decode B=64; "
          "tokens/s at 1/2/4/8 GPUs")
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20
SMALL_BATCHES = (1, 2, 4, 6, 8)
E2E_WARMUP_STEPS = 20   # untimed end-to-end steps before the timed ones: at least this many ...
E2E_WARMUP_SECONDS = 0.5   # ... and for at least this long (the host copy rate rises over the first ~1000 copies)
INDEXER_WARMUP = 8      # untimed indexer calls: the score kernel's tile plan calibrates over them
TRAFFIC_FILE = os.path.join("profiles", "split_kernel_traffic.json")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="workload of `value` (configs 1, 3 and 4: main legs only, for profiling runs)")
    ap.add_argument("--pool-pages", type=int, default=None,
                    help="smaller page pool for profiling runs (default: the full config)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only-main", action="store_true",
                    help="profiling runs: only the config-2 value/roofline legs")
    ap.add_argument("--stop-after-indexer", action="store_true",
                    help="profiling runs: the extra legs up to the indexer's, none after (no large pools)")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", FALLBACK_BF16_TFLOPS)), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def measured_peak():
    hbm, _, kind = measured_peaks()
    return hbm, kind


def make_workload(args, world, rank, device):
    sh = importlib.import_module(f"{PKG}.sharding")
    if args.config == 2:
        kw = {} if args.pool_pages is None else {"pool_pages": args.pool_pages}
        return sh.shard_config2(world, rank, device=device, **kw)
    if args.config == 5:
        return sh.shard_config5(world, rank, device=device)
    W = importlib.import_module(f"{PKG}.workloads")
    return W.make_config(args.config, device=device)


def scaling_kind(args) -> str:
    """Config 2 gives every GPU its own 64-token batch (weak scaling);
    config 5 splits one fixed 1024-token batch over the GPUs (strong)."""
    return "strong" if args.config == 5 else "weak"


def config_dict(args, w, world):
    what = {1: "4 tokens over a 128-page pool (the CPU-runnable case)",
            2: "decode B=64 per GPU, 32768-slot sequence per token, page table = permutation of a 32768-page pool",
            3: "128 tokens, context lengths U[256, 4096], short rows padded with -1",
            4: "prefill chunk: 4096 tokens over one 131072-slot cache, local-heavy indices",
            5: "1024 tokens = 256 sequences x 4 over 131072-slot sequences, sequences sharded over GPUs"}
    d = {"workload": f"config{args.config}: " + what[args.config],
         "global_batch": 1024 if args.config == 5 else int(w.num_tokens * world),
         "tokens_per_gpu": int(w.num_tokens),
         "heads": 16, "ckv_dim": 512, "kpe_dim": 64, "topk": 2048, "page_size": 64,
         "pool_pages_per_gpu": int(w.num_pages),
         "parallelism": f"batch-rows x{world} (no collective)",
         "l2": "flushed before every timed call, outside the events: 256 MiB memset, then a 256 MiB read of a "
               "second buffer (no input lines and no dirty lines left in L2); the pipelined legs instead rotate "
               "over 4 decode batches whose gathered rows together exceed L2"}
    if args.pool_pages is not None:
        d["pool_pages_override"] = args.pool_pages
    return d


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons through NVML in a
    background thread; only samples taken while `active` is set count, so the
    summary covers the timed regions alone.  Read-only queries."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int):
        import threading
        self.samples = []
        self._active = False
        self._wake = threading.Event()   # set while a timed region runs: the thread sleeps otherwise
        self._stop = False
        self.err = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.handle = None
            try:
                uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report it instead of clocks
            self.err = f"nvml unavailable: {e}"
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def sample_now(self):
        """One sample from the calling thread (the timed loops call this
        after queueing their steps, while the GPU still runs them, so a
        short timed region has at least one sample)."""
        if self.err is not None and not hasattr(self, "handle"):
            return
        nv = self.nv
        try:
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.samples.append((nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM), reasons_fn(self.handle)))
        except Exception as e:
            self.err = str(e)

    @property
    def active(self):
        return self._active

    @active.setter
    def active(self, on):
        self._active = bool(on)
        if on:
            self._wake.set()
        else:
            self._wake.clear()

    def _run(self):
        while not self._stop:
            if not self._wake.wait(timeout=0.5):   # no wake-ups (GIL hand-offs) outside timed regions
                continue
            if self._active:
                n = len(self.samples)
                self.sample_now()
                if not self._active and len(self.samples) > n:
                    self.samples.pop()   # taken after the timed region ended
            time.sleep(0.0005)

    def stop(self):
        if self.err is not None and not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err]}
        self._stop = True
        self._wake.set()
        self.thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "NVML, timed regions only"}


def cpu_reference_rate(w, seconds: float, max_tokens: int = 64, tokens=None):
    """Query tokens/s of the reference's naive kernel compiled for CPU
    (oracle/_ref, kind "reference"), else the oracle port (kind "port"), on
    this host's cores.  The sample: the first tokens of the workload (or the
    given ones) over a compacted pool of just the rows they touch
    (result-identical; the reference's per-call fp32 cast of the whole pool,
    kernel_naive.cu:38-39, is therefore left out, which flatters it)."""
    from oracle.build_ref import load_ref
    from oracle.dsa_oracle import compact_pool, launch_sparse_attention_oracle
    torch.set_num_threads(os.cpu_count() or 1)
    ref = load_ref()
    kind = "reference" if ref is not None else "port"
    fn = ref.launch_sparse_attention_c if ref is not None else launch_sparse_attention_oracle
    sel = tokens if tokens is not None else list(range(min(max_tokens, w.num_tokens)))
    n = len(sel)
    ckv, kpe, idx = compact_pool(w.ckv_cache, w.kpe_cache, w.sparse_indices[sel])
    qn, qp = w.q_nope[sel].cpu(), w.q_pe[sel].cpu()
    ckv, kpe, idx = ckv.cpu(), kpe.cpu(), idx.cpu()
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16)
    lse = torch.empty((n, 16), dtype=torch.float32)
    fn(qn, qp, ckv, kpe, idx, w.sm_scale, out, lse)        # warm-up
    t0 = time.perf_counter()
    calls = 0
    while True:
        fn(qn, qp, ckv, kpe, idx, w.sm_scale, out, lse)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    rate = calls * n / el
    sample = (f"{n} tokens of the workload per call over a compacted pool of their {idx.ne(-1).sum().item()} "
              f"gathered rows, {calls} calls in {el:.1f} s")
    return rate, {"value": rate, "unit": "query-tokens/s", "cores": torch.get_num_threads(), "kind": kind,
                  "sample": sample, "ms_per_call": 1000.0 * el / calls}


def small_batch(w, n):
    """The first n tokens of a workload (same pool)."""
    W = importlib.import_module(f"{PKG}.workloads")
    return W.Workload(f"{w.name}_first{n}", w.q_nope[:n].contiguous(), w.q_pe[:n].contiguous(), w.ckv_cache,
                      w.kpe_cache, w.sparse_indices[:n].contiguous(), w.sm_scale, {})


class Flusher:
    def __init__(self, dev):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(L2_FLUSH_BYTES // 8, dtype=torch.int64, device=dev)

    def __call__(self):
        self.w.zero_()        # evicts every input line
        self.r.sum()          # evicts the memset's dirty lines (written back here, not in the timed call)


def time_isolated(fn, steps, stream, flush):
    """Mean device time (ms) of fn() with CUDA events on `stream`, the L2
    flushed before each call (outside the events)."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush()
        ev[i][0].record(stream)
        fn()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in ev)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = make_workload(args, 1, 0, dev)
    n = min(64, w.num_tokens)
    from oracle.build_ref import load_ref
    from oracle.dsa_oracle import compact_pool, launch_sparse_attention_oracle
    torch.set_num_threads(os.cpu_count() or 1)
    ref = load_ref()
    kind = "reference" if ref is not None else "port"
    fn = ref.launch_sparse_attention_c if ref is not None else launch_sparse_attention_oracle
    ckv, kpe, idx = compact_pool(w.ckv_cache, w.kpe_cache, w.sparse_indices[:n])
    qn, qp = w.q_nope[:n].cpu(), w.q_pe[:n].cpu()
    ckv, kpe, idx = ckv.cpu(), kpe.cpu(), idx.cpu()
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16)
    lse = torch.empty((n, 16), dtype=torch.float32)
    for _ in range(args.warmup):
        fn(qn, qp, ckv, kpe, idx, w.sm_scale, out, lse)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn(qn, qp, ckv, kpe, idx, w.sm_scale, out, lse)
        times.append(time.perf_counter() - t0)
    step = statistics.mean(times)
    rate = n / step
    world = args.gpus
    sample = (f"{n} tokens per step (the rank-0 batch of config {args.config}) over a compacted pool of "
              f"their gathered rows; CPU, {torch.get_num_threads()} threads")
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": "query-tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * step,
            "higher_is_better": True, "scaling": scaling_kind(args), "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded N(0,1) bf16, same generator and seed as the GPU arm)",
            "config": config_dict(args, w, world),
            "cpu_baseline": {"value": rate, "unit": "query-tokens/s", "cores": torch.get_num_threads(),
                             "kind": kind, "sample": sample},
            "e2e": {"value": rate, "unit": "query-tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference = methodology/checkpoints/kernel_naive.cu compiled for CPU from its source "
                    "(oracle/build_ref.py); the reference's CUDA kernel rejects num_tokens >= 9",
            "ref_cuda": reference_cuda_points(args, w) if dev == "cuda" else None}
    print(json.dumps(line), flush=True)


def reference_cuda_points(args, w):
    """The reference's own optimised CUDA kernel (solution/cuda/kernel.cu,
    compiled unchanged for sm_100a by oracle/build_ref_cuda.py) on the first
    1, 2, 4, 6 and 8 tokens of config 2, and on config 1: us per call with
    CUDA events, L2 flushed before each call.  Valid inputs only (its waits
    spin without a bound).  The library's times on the same inputs are the
    `small_batches` key of the other arm."""
    from oracle.build_ref_cuda import MAX_TOKENS, load_ref_cuda
    from oracle.dsa_oracle import reference_cuda_splits
    mod = load_ref_cuda()
    if mod is None:
        return {"unavailable": "oracle/_ref/dsa_ref_cuda.so not built"}
    W = importlib.import_module(f"{PKG}.workloads")
    dev = w.q_nope.device
    stream = torch.cuda.current_stream(dev)
    flush = Flusher(dev)
    pts = {}
    cases = [(f"n{n}", small_batch(w, n)) for n in SMALL_BATCHES if n <= MAX_TOKENS]
    cases.append(("config1", W.config1(device=dev)))
    for name, wb in cases:
        n = wb.num_tokens
        assert int(wb.sparse_indices.max()) < wb.num_pages * 64 and int(wb.sparse_indices.min()) >= -1
        out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device=dev)
        lse = torch.empty((n, 16), dtype=torch.float32, device=dev)

        def call():
            mod.launch_sparse_attention_c(*wb.args()[:5], float(wb.sm_scale), out, lse)

        for _ in range(max(args.warmup, 3)):
            call()
        ms = time_isolated(call, args.steps, stream, flush)
        S = reference_cuda_splits(n)
        pts[name] = {"tokens": n, "us_per_call": ms * 1000.0, "query_tokens_per_s": n / (ms / 1000.0),
                     "gathered_gbs": wb.gathered_bytes() / (ms / 1000.0) / 1e9, "splits": S,
                     "computes_the_operator": S <= 32}
    return {"kernel": "reference solution/cuda/kernel.cu (sparse_attention_split_kernel, fused reduce), "
                      "compiled for sm_100a", "points": pts,
            "note": "with more than 32 splits per token (num_tokens <= 4) its reduce reads 32 lanes of per-split "
                    "statistics and its output is not the operator's (kernel.cu:439-475; "
                    "tests/test_ref_cuda_gpu.py)",
            "how": "first n tokens of config 2 (2.42 GB pool) and config 1; CUDA events per call, L2 flushed"}


def kernel_events_ms(lib, lib_mod, w, out, lse, ws, stream, steps, flush):
    """Mean duration (ms) of the split-KV launch alone, from the events the
    library records around it (dsa_sparse_attention_fwd_profiled)."""
    evk = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for trio in evk:          # torch creates the CUDA event lazily, on first record
        for e in trio:
            e.record(stream)
    for i in range(steps):
        flush()
        handles = (ctypes.c_void_p * 3)(*[e.cuda_event for e in evk[i]])
        st = lib.dsa_sparse_attention_fwd_profiled(
            w.q_nope.data_ptr(), w.q_pe.data_ptr(), w.ckv_cache.data_ptr(), w.kpe_cache.data_ptr(),
            w.sparse_indices.data_ptr(), w.num_tokens, w.num_pages, w.sm_scale, out.data_ptr(), lse.data_ptr(),
            ws.data_ptr(), ws.numel(), stream.cuda_stream, handles)
        lib_mod.check(st, "fwd_profiled")
    torch.cuda.synchronize()
    return statistics.mean(e[0].elapsed_time(e[1]) for e in evk)


def config_point(dsa, lib, lib_mod, w, args, stream, flush, hbm_peak, tf_peak, cpu_tokens=None):
    """One benchmark configuration at one GPU: us per call (events around the
    public call, L2 flushed), the kernel alone (library events), gathered
    GB/s, fraction of the measured copy bandwidth, TFLOP/s, tokens/s, and the
    CPU reference's tokens/s on a sample."""
    n = w.num_tokens
    dev = w.q_nope.device
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((n, 16), dtype=torch.float32, device=dev)

    def call():
        dsa.launch_sparse_attention_c(*w.args(), out, lse)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    dsa.check_device_errors(dev)
    ms = time_isolated(call, args.steps, stream, flush)
    ws = dsa.workspace_for(dev, n)
    kms = kernel_events_ms(lib, lib_mod, w, out, lse, ws, stream, args.steps, flush)
    dsa.check_device_errors(dev)
    gathered, flops = w.gathered_bytes(), w.flops()
    d = {"tokens": n, "us_per_call": ms * 1000.0, "kernel_us": kms * 1000.0,
         "query_tokens_per_s": n / (ms / 1000.0), "gathered_bytes": gathered,
         "gathered_gbs": gathered / (kms / 1000.0) / 1e9,
         "frac_of_peak": gathered / (kms / 1000.0) / 1e9 / hbm_peak,
         "pct_of_8tbs": 100.0 * gathered / (kms / 1000.0) / 1e9 / NOMINAL_HBM_GBS,
         "tflops": flops / (kms / 1000.0) / 1e12, "frac_of_bf16_peak": flops / (kms / 1000.0) / 1e12 / tf_peak}
    if cpu_tokens is not None and not args.no_cpu_baseline:
        rate, info = cpu_reference_rate(w, min(args.cpu_seconds, 3.0), tokens=cpu_tokens)
        d["cpu_reference"] = info
    return d


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def per_rank(vals):
        """All ranks' values (list per rank), gathered to every rank."""
        if dist is None:
            return [list(vals)]
        t = torch.zeros((world, len(vals)), dtype=torch.float64, device=dev)
        t[rank] = torch.tensor(vals, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.cpu().tolist()

    dsa = importlib.import_module(PKG)
    lib_mod = importlib.import_module(f"{PKG}._lib")
    lib = lib_mod.load()
    W_mod = importlib.import_module(f"{PKG}.workloads")
    hbm_peak, tf_peak, peak_kind = measured_peaks()
    w = make_workload(args, world, rank, dev)
    n = w.num_tokens
    gathered = w.gathered_bytes()
    stream = torch.cuda.current_stream(dev)
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((n, 16), dtype=torch.float32, device=dev)
    ws = dsa.workspace_for(dev, n)
    flush_l2 = Flusher(dev)

    def call():
        dsa.launch_sparse_attention_c(*w.args(), out, lse)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    dsa.check_device_errors(dev)

    # ---- value: device time per call, inputs resident -------------------
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    # The timed host loops (the end-to-end legs) are Python: no cyclic garbage
    # collection pauses inside them, as timeit does (the run allocates no
    # reference cycles worth collecting).
    gc.collect()
    gc.disable()
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.active = True
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush_l2()
        ev[i][0].record(stream)
        call()
        ev[i][1].record(stream)
    sampler.sample_now()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    sampler.active = False
    barrier()
    step_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    step_ms_max = max_over_ranks(step_ms)
    launches_per_call = 1   # the split-KV kernel; the cross-CTA merge is fused into it
    gpu_launches = launches_per_call * args.steps

    # ---- roofline: the split-KV kernel alone, events recorded by the library
    sampler.active = True
    split_ms = kernel_events_ms(lib, lib_mod, w, out, lse, ws, stream, args.steps, flush_l2)
    sampler.sample_now()
    sampler.active = False
    split_ms_max = max_over_ranks(split_ms)

    extra = {}
    if not args.only_main and args.config in (2, 5):
        extra = run_extra_legs(args, dsa, lib, lib_mod, W_mod, w, out, lse, stream, flush_l2, world, rank, dev,
                               barrier, max_over_ranks, per_rank, hbm_peak, tf_peak)
    clocks = sampler.stop()

    # ---- CPU baseline (rank 0, N=1 only) ----------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        _, cpu = cpu_reference_rate(w, args.cpu_seconds)

    if dist is not None:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return

    tokens_total = n * world
    value = tokens_total / (step_ms_max / 1000.0)
    achieved_iso = gathered / (split_ms_max / 1000.0) / 1e9
    # The kernel's average launch duration: over the back-to-back timed region
    # when that leg ran (a launch measured alone between events also carries
    # ~6 us that an empty kernel of the same launch shape measures on this
    # pool), else the isolated launches.
    pipe = extra.get("pipelined")
    kernel_us = pipe["us_per_call"] if pipe else split_ms_max * 1000.0
    achieved = gathered / (kernel_us / 1e6) / 1e9
    traffic, traffic_src = None, None
    tp = os.path.join(REPO, TRAFFIC_FILE)
    if os.path.exists(tp):
        try:
            with open(tp) as f:
                td = json.load(f)
            traffic = td.get(f"config{args.config}_bytes_per_launch")
            traffic_src = (f"{TRAFFIC_FILE}: stored ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) "
                           f"of build {td.get('build', 'unknown')}, not measured in this run")
        except Exception:
            traffic = None
    line = {
        "metric": METRIC, "value": value, "unit": "query-tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms_max,
        "higher_is_better": True, "scaling": scaling_kind(args), "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 q/ckv/kpe, seeded index sampling; no dataset available)",
        "config": config_dict(args, w, world),
        "us_per_call": step_ms_max * 1000.0,
        "gathered_kv_bytes_per_gpu": gathered,
        "gathered_kv_gbs_per_gpu": gathered / (step_ms_max / 1000.0) / 1e9,
        "pct_of_8tbs": 100.0 * gathered / (step_ms_max / 1000.0) / 1e9 / NOMINAL_HBM_GBS,
        "roofline": {"bound": "hbm", "kernel": "dsa split-KV kernel", "achieved": achieved, "peak": hbm_peak,
                     "peak_kind": f"{peak_kind} copy bandwidth", "unit": "GB/s", "frac": achieved / hbm_peak,
                     "traffic": traffic, "traffic_source": traffic_src, "kernel_us": kernel_us,
                     "algorithmic_bytes_per_launch": gathered,
                     "pct_of_8tbs": 100.0 * achieved / NOMINAL_HBM_GBS,
                     "how": ("algorithmic gathered bytes / the split kernel's average launch duration over the "
                             "back-to-back timed region (CUDA events around all launches; 4 rotating decode batches "
                             "whose gathered rows together exceed L2, no flush)" if pipe else
                             "algorithmic gathered bytes / the mean of the library's events around each launch"),
                     "isolated": {"kernel_us": split_ms_max * 1000.0, "achieved": achieved_iso,
                                  "frac": achieved_iso / hbm_peak,
                                  "how": "the library's CUDA events around each launch, L2 flushed before it; "
                                         "includes the ~6 us an empty kernel of the same launch shape measures"}},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "gpu_launches": gpu_launches,
        "wall_s_timed_region": wall,
    }
    line.update(extra)
    if "e2e" not in line:
        line["e2e"] = None
    print(json.dumps(line), flush=True)


def run_extra_legs(args, dsa, lib, lib_mod, W_mod, w, out, lse, stream, flush_l2, world, rank, dev,
                   barrier, max_over_ranks, per_rank, hbm_peak, tf_peak):
    n = w.num_tokens
    gathered = w.gathered_bytes()
    res = {}

    # ---- the page-table-native entry point on the same problem ------------
    bt, pos, seq = (w.meta.get(k) for k in ("block_table", "positions", "seq_of_token"))
    if bt is not None:
        out_p, lse_p = torch.empty_like(out), torch.empty_like(lse)

        def call_paged():
            dsa.launch_sparse_attention_paged(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, bt, pos, w.sm_scale,
                                              out_p, lse_p, seq_of_token=seq)

        for _ in range(args.warmup):
            call_paged()
        paged_ms = max_over_ranks(time_isolated(call_paged, args.steps, stream, flush_l2))
        if not (torch.equal(out_p, out) and torch.equal(lse_p, lse)):
            raise RuntimeError("page-table-native result differs from the slot-id result")
        dsa.check_device_errors(dev)
        res["paged"] = {
            "us_per_call": paged_ms * 1000.0, "query_tokens_per_s": n * world / (paged_ms / 1000.0),
            "how": "dsa_sparse_attention_fwd_paged on the same problem: block table + positions, translated "
                   "inside the kernel; CUDA events per call, L2 flushed; result checked equal to the slot-id call"}

    # ---- FP8 KV cache variant on the same problem (656-byte rows) ---------
    fp8_mod = importlib.import_module(f"{PKG}.fp8")
    kv8 = fp8_mod.quantize_kv_fp8(w.ckv_cache, w.kpe_cache)
    out8, lse8 = torch.empty_like(out), torch.empty_like(lse)

    def call_fp8():
        fp8_mod.launch_sparse_attention_fp8_c(w.q_nope, w.q_pe, kv8, w.sparse_indices, w.sm_scale, out8, lse8)

    for _ in range(args.warmup):
        call_fp8()
    fp8_ms = max_over_ranks(time_isolated(call_fp8, args.steps, stream, flush_l2))
    dsa.check_device_errors(dev)
    fp8_bytes = gathered // 1152 * 656
    del kv8, out8, lse8
    res["fp8_kv"] = {
        "us_per_call": fp8_ms * 1000.0, "query_tokens_per_s": n * world / (fp8_ms / 1000.0),
        "gathered_bytes_per_call": fp8_bytes, "gathered_gbs": fp8_bytes / (fp8_ms / 1000.0) / 1e9,
        "frac_of_peak": fp8_bytes / (fp8_ms / 1000.0) / 1e9 / hbm_peak,
        "how": "dsa_sparse_attention_fwd_fp8 on config 2 with the pool quantised to 656-byte FP8 rows "
               "(bitwise equal to the bf16 operator on the dequantised pool); CUDA events, L2 flushed"}

    # ---- the top-k indexer that produces the attention's indices ----------
    # (warm-up of at least INDEXER_WARMUP calls: the score kernel's tile plan
    # is calibrated from the calls before)
    wi = W_mod.indexer_decode(seed=13 + rank, device=dev)
    topk_out = torch.empty((wi.batch, 2048), dtype=torch.int32, device=dev)
    for _ in range(max(args.warmup, INDEXER_WARMUP)):
        flush_l2()
        dsa.launch_topk_c(*wi.args(), topk_out)
    torch.cuda.synchronize()
    indexer_ms = max_over_ranks(time_isolated(lambda: dsa.launch_topk_c(*wi.args(), topk_out), args.steps, stream,
                                              flush_l2))
    dsa.indexer.check_errors(dev)
    ikb = wi.key_bytes()
    res["indexer"] = {
        "us_per_call": indexer_ms * 1000.0, "rows": wi.batch, "positions_per_row": 32768,
        "key_bytes_per_call": ikb, "key_gbs": ikb / (indexer_ms / 1000.0) / 1e9,
        "frac_of_peak": ikb / (indexer_ms / 1000.0) / 1e9 / hbm_peak,
        "rows_per_s_job": wi.batch * world / (indexer_ms / 1000.0),
        "how": "launch_topk_c (score kernel + top-k kernel) over a decode batch of 64 rows x 32768 "
               "positions per GPU (fp8 keys, 132 B per position); CUDA events per call, L2 flushed"}

    # ---- the indexer on ragged rows, with and without the calibrated plan --
    wr = W_mod.indexer_ragged(seed=16 + rank, device=dev)
    rg_out = torch.empty((wr.batch, 2048), dtype=torch.int32, device=dev)
    rg = {}
    for mode in (0, 1):
        dsa._lib.load().dsa_topk_indexer_set_calibrated_plan(mode)
        for _ in range(max(args.warmup, INDEXER_WARMUP)):
            flush_l2()
            dsa.launch_topk_c(*wr.args(), rg_out)
        torch.cuda.synchronize()
        rg[mode] = max_over_ranks(time_isolated(lambda: dsa.launch_topk_c(*wr.args(), rg_out), args.steps, stream,
                                                flush_l2))
    dsa.indexer.check_errors(dev)
    rkb = wr.key_bytes()
    res["indexer_ragged"] = {
        "us_per_call": rg[1] * 1000.0, "us_per_call_equal_shares": rg[0] * 1000.0, "rows": wr.batch,
        "positions": int(wr.seq_lens.sum().item()), "key_bytes_per_call": rkb,
        "key_gbs": rkb / (rg[1] / 1000.0) / 1e9, "frac_of_peak": rkb / (rg[1] / 1000.0) / 1e9 / hbm_peak,
        "how": "launch_topk_c over 64 rows of lengths uniform in [1024, 32768] (32768-position tables): the "
               "score kernel's split of the active tiles by the calibrated plan (default) against equal "
               "shares of them (dsa_topk_indexer_set_calibrated_plan(0)); CUDA events per call, L2 flushed"}
    del wr, rg_out

    # ---- decode step: indexer -> attention on its top-k -------------------
    if wi.batch == n and wi.k_index_cache.shape[0] <= w.num_pages:
        out_s, lse_s = torch.empty_like(out), torch.empty_like(lse)

        def decode_step():
            dsa.launch_topk_c(*wi.args(), topk_out)
            dsa.launch_sparse_attention_c(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, topk_out, w.sm_scale,
                                          out_s, lse_s)

        for _ in range(max(args.warmup, INDEXER_WARMUP)):
            decode_step()
        dstep_ms = max_over_ranks(time_isolated(decode_step, args.steps, stream, flush_l2))
        dsa.check_device_errors(dev)
        dsa.indexer.check_errors(dev)
        res["decode_step"] = {
            "us_per_call": dstep_ms * 1000.0, "query_tokens_per_s_job": n * world / (dstep_ms / 1000.0),
            "how": "launch_topk_c then launch_sparse_attention_c on its top-k slot ids (one DSA sparse attention "
                   "layer: indexer score + top-k + attention kernels); CUDA events per call, L2 flushed"}

        # ---- the same step captured once in a CUDA graph and replayed ------
        # thread-local capture mode: other threads of the process (the NCCL
        # process group's watchdog under torchrun) keep querying their events
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            decode_step()
        for _ in range(max(args.warmup, INDEXER_WARMUP)):
            flush_l2()
            graph.replay()
        gstep_ms = max_over_ranks(time_isolated(graph.replay, args.steps, stream, flush_l2))
        dsa.check_device_errors(dev)
        dsa.indexer.check_errors(dev)
        graph_out = out_s.clone()
        decode_step()
        if not torch.equal(graph_out, out_s):
            raise RuntimeError("graph-replayed decode step differs from the eager one")
        del graph
        res["decode_step_graph"] = {
            "us_per_call": gstep_ms * 1000.0, "query_tokens_per_s_job": n * world / (gstep_ms / 1000.0),
            "how": "the decode_step calls captured once in a CUDA graph (torch.cuda.graph) and replayed; CUDA "
                   "events per replay, L2 flushed; the last replay's output checked equal to an eager step"}
        del out_s, lse_s
    del wi, topk_out
    if args.stop_after_indexer:
        return res

    # ---- pipelined and end to end: back-to-back steps over rotating batches
    if args.config == 2:
        batches = W_mod.decode_batches(w, 4, seed=977 + rank)
        res["pipelined"] = pipelined_leg(dsa, w, batches, args, stream, barrier, max_over_ranks, hbm_peak, world)
        res["e2e"] = e2e_pipelined_leg(dsa, w, batches, args, dev, barrier, max_over_ranks, world)
        del batches
    res["e2e_serial"] = e2e_serial_leg(dsa, w, out, lse, args, dev, flush_l2, barrier, max_over_ranks, world)

    # ---- the small batches the reference's CUDA kernel accepts ------------
    if args.config == 2:
        pts = {}
        for nb in SMALL_BATCHES:
            wb = small_batch(w, nb)
            ob = torch.empty((nb, 16, 512), dtype=torch.bfloat16, device=dev)
            lb = torch.empty((nb, 16), dtype=torch.float32, device=dev)

            def call_b():
                dsa.launch_sparse_attention_c(*wb.args(), ob, lb)

            for _ in range(args.warmup):
                call_b()
            ms = max_over_ranks(time_isolated(call_b, args.steps, stream, flush_l2))
            pts[f"n{nb}"] = {"tokens": nb, "us_per_call": ms * 1000.0, "query_tokens_per_s": nb / (ms / 1000.0),
                             "gathered_gbs": wb.gathered_bytes() / (ms / 1000.0) / 1e9}
        dsa.check_device_errors(dev)
        res["small_batches"] = {"points": pts, "how": "first n tokens of config 2 (same pool), CUDA events per "
                                                      "call, L2 flushed; the reference arm's ref_cuda key times "
                                                      "the reference's CUDA kernel on the same inputs"}

    # ---- configs 1, 3, 4 and 5 at one GPU ----------------------------------
    if world == 1 and args.config == 2:
        cfgs = {}
        for c, cpu_tokens in ((1, [0, 1, 2, 3]), (3, list(range(16))), (4, [0, 1000, 2000, 3000, 4095])):
            wc = W_mod.make_config(c, device=dev)
            cfgs[f"config{c}"] = config_point(dsa, lib, lib_mod, wc, args, stream, flush_l2, hbm_peak, tf_peak,
                                              cpu_tokens)
            if c == 4:
                cfgs["config4"]["note"] = ("touched rows (positions < 6144, 7.1 MB) stay in L2: gathered GB/s "
                                           "counts algorithmic bytes and exceeds HBM; tflops / frac_of_bf16_peak "
                                           "is the relevant roofline")
            del wc
            torch.cuda.empty_cache()
        res["configs"] = cfgs

    # ---- config 5: strong scaling of one 1024-token batch -----------------
    if args.config == 2:
        res["config5"] = config5_leg(dsa, lib, lib_mod, args, stream, flush_l2, world, rank, dev, barrier,
                                     max_over_ranks, per_rank, hbm_peak)
    return res


def pipelined_leg(dsa, w, batches, args, stream, barrier, max_over_ranks, hbm_peak, world):
    """launch_sparse_attention_c back to back over the rotating decode batches
    (different queries and indices, same pool; 4 x 151 MB gathered, no L2
    flush), CUDA events around all the steps."""
    n = w.num_tokens
    gathered = w.gathered_bytes()
    outs = [(torch.empty((n, 16, 512), dtype=torch.bfloat16, device=w.q_nope.device),
             torch.empty((n, 16), dtype=torch.float32, device=w.q_nope.device)) for _ in batches]

    def call_b(k):
        qn, qp, ix = batches[k % len(batches)]
        o, l = outs[k % len(batches)]
        dsa.launch_sparse_attention_c(qn, qp, w.ckv_cache, w.kpe_cache, ix, w.sm_scale, o, l)

    for k in range(max(args.warmup, len(batches))):
        call_b(k)
    torch.cuda.synchronize()
    e_a, e_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e_a.record(stream)
    for k in range(args.steps):
        call_b(k)
    e_b.record(stream)
    torch.cuda.synchronize()
    barrier()
    dsa.check_device_errors(w.q_nope.device)
    pipe_ms = max_over_ranks(e_a.elapsed_time(e_b) / args.steps)
    return {"us_per_call": pipe_ms * 1000.0, "query_tokens_per_s_job": n * world / (pipe_ms / 1000.0),
            "gathered_gbs": gathered / (pipe_ms / 1000.0) / 1e9,
            "frac_of_peak": gathered / (pipe_ms / 1000.0) / 1e9 / hbm_peak, "batches": len(batches),
            "how": "launch_sparse_attention_c called back to back over 4 rotating decode batches of config 2 "
                   "(different queries and indices, same pool; 4 x 151 MB gathered, no L2 flush), CUDA "
                   "events around all steps"}


class _Runtime:
    """The CUDA runtime's stream-ordered copy and event calls through ctypes,
    for the host side of the end-to-end loops: one foreign call each instead
    of torch's stream context switches and copy dispatch.  The operator under
    test is still called through the public Python API every step."""

    H2D, D2H = 1, 2

    def __init__(self):
        try:
            rt = ctypes.CDLL("libcudart.so.12")
        except OSError:
            rt = ctypes.CDLL("libcudart.so")
        vp = ctypes.c_void_p
        rt.cudaMemcpyAsync.argtypes = [vp, vp, ctypes.c_size_t, ctypes.c_int, vp]
        rt.cudaEventRecord.argtypes = [vp, vp]
        rt.cudaStreamWaitEvent.argtypes = [vp, vp, ctypes.c_uint]
        rt.cudaEventCreateWithFlags.argtypes = [ctypes.POINTER(vp), ctypes.c_uint]
        rt.cudaEventDestroy.argtypes = [vp]
        self.rt = rt
        self.events = []

    def event(self):
        e = ctypes.c_void_p()
        if self.rt.cudaEventCreateWithFlags(ctypes.byref(e), 2) != 0:   # cudaEventDisableTiming
            raise RuntimeError("cudaEventCreateWithFlags failed")
        self.events.append(e)
        return e

    def copy(self, dst, src, nbytes, kind, stream):
        if self.rt.cudaMemcpyAsync(dst, src, nbytes, kind, stream) != 0:
            raise RuntimeError("cudaMemcpyAsync failed")

    def record(self, ev, stream):
        if self.rt.cudaEventRecord(ev, stream) != 0:
            raise RuntimeError("cudaEventRecord failed")

    def wait(self, stream, ev):
        if self.rt.cudaStreamWaitEvent(stream, ev, 0) != 0:
            raise RuntimeError("cudaStreamWaitEvent failed")

    def close(self):
        for e in self.events:
            self.rt.cudaEventDestroy(e)
        self.events = []


def _packed(parts):
    offs, o = [], 0
    for t in parts:
        offs.append(o)
        o += (t.numel() * t.element_size() + 255) // 256 * 256
    return offs, o


def _view(block, off, like):
    nbytes = like.numel() * like.element_size()
    return block[off:off + nbytes].view(like.dtype).view(like.shape)


def e2e_pipelined_leg(dsa, w, batches, args, dev, barrier, max_over_ranks, world):
    """End to end through the public API with pinned host buffers, as a
    serving loop runs it: every step copies its own inputs (q_nope | q_pe |
    sparse_indices, one pinned block, one copy) in and its results (output |
    lse, one block) out; steps run back to back over the 4 rotating decode
    batches, with the copies in, the kernels and the copies out on three
    streams so that the copies of one step overlap the kernels of its
    neighbours.  Events order each slot's reuse.  Wall clock over all steps;
    every result is checked against the device-resident call."""
    n = w.num_tokens
    R = len(batches)
    like_in = [batches[0][0], batches[0][1], batches[0][2]]
    in_offs, in_bytes = _packed(like_in)
    out_like = [torch.empty((n, 16, 512), dtype=torch.bfloat16), torch.empty((n, 16), dtype=torch.float32)]
    out_offs, out_bytes = _packed(out_like)
    h_in = [torch.empty(in_bytes, dtype=torch.uint8).pin_memory() for _ in range(R)]
    for b in range(R):
        for t, o in zip(batches[b], in_offs):
            _view(h_in[b], o, t).copy_(t.cpu())
    h_out = [torch.empty(out_bytes, dtype=torch.uint8).pin_memory() for _ in range(R)]
    d_in = [torch.empty(in_bytes, dtype=torch.uint8, device=dev) for _ in range(R)]
    d_out = [torch.empty(out_bytes, dtype=torch.uint8, device=dev) for _ in range(R)]
    views_in = [[_view(d_in[b], o, t) for t, o in zip(like_in, in_offs)] for b in range(R)]
    views_out = [[_view(d_out[b], o, t) for t, o in zip(out_like, out_offs)] for b in range(R)]
    s_in_t, s_out_t = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp_t = torch.cuda.current_stream(dev)   # the public call launches on the current stream
    s_in, s_out, s_comp = (ctypes.c_void_p(s.cuda_stream) for s in (s_in_t, s_out_t, s_comp_t))
    rt = _Runtime()
    ev_in = [rt.event() for _ in range(R)]       # inputs of slot b landed
    ev_comp = [rt.event() for _ in range(R)]     # kernel of slot b done (inputs free, outputs ready)
    ev_out = [rt.event() for _ in range(R)]      # outputs of slot b copied out (slot free)
    p_hin = [ctypes.c_void_p(t.data_ptr()) for t in h_in]
    p_din = [ctypes.c_void_p(t.data_ptr()) for t in d_in]
    p_hout = [ctypes.c_void_p(t.data_ptr()) for t in h_out]
    p_dout = [ctypes.c_void_p(t.data_ptr()) for t in d_out]
    h2d = sum(t.numel() * t.element_size() for t in like_in)
    d2h = n * 16 * 512 * 2 + n * 16 * 4

    # Slot b's copy-in waits for its previous copy-out, which followed its
    # previous kernel: so the kernel needs one wait (its inputs landed) and
    # every slot reuse is still ordered.
    def step(k):
        b = k % R
        if k >= R:
            rt.wait(s_in, ev_out[b])
        rt.copy(p_din[b], p_hin[b], in_bytes, rt.H2D, s_in)
        rt.record(ev_in[b], s_in)
        rt.wait(s_comp, ev_in[b])
        qn, qp, ix = views_in[b]
        o, l = views_out[b]
        dsa.launch_sparse_attention_c(qn, qp, w.ckv_cache, w.kpe_cache, ix, w.sm_scale, o, l)
        rt.record(ev_comp[b], s_comp)
        rt.wait(s_out, ev_comp[b])
        rt.copy(p_hout[b], p_dout[b], out_bytes, rt.D2H, s_out)
        rt.record(ev_out[b], s_out)

    # Warm-up: untimed, and long enough that the process's first host copies
    # are over before the timed steps: on these hosts a 1.7 MB pinned copy
    # took 78-86 us at the start of a process and 37-39 us after ~1000 copies
    # (PCIe Gen 5 throughout).  Synchronised every 50 steps so that the time
    # counts device progress, not steps queued ahead.
    k, t_w = 0, time.perf_counter()
    while True:
        step(k)
        k += 1
        if k % 50 == 0 or k >= 20000:
            torch.cuda.synchronize()
            if k >= 20000 or (k >= max(args.warmup, E2E_WARMUP_STEPS) and
                              time.perf_counter() - t_w >= E2E_WARMUP_SECONDS):
                break
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for k in range(args.steps):
        step(k)
    torch.cuda.synchronize()
    el = time.perf_counter() - t0
    barrier()
    # every slot's last result against the device-resident call on the same batch
    for b in range(R):
        qn, qp, ix = batches[b]
        ro, rl = dsa.kernel(qn, qp, w.ckv_cache, w.kpe_cache, ix, w.sm_scale)
        if not (torch.equal(_view(h_out[b], out_offs[0], out_like[0]), ro.cpu()) and
                torch.equal(_view(h_out[b], out_offs[1], out_like[1]), rl.cpu())):
            raise RuntimeError("end-to-end result differs from the device-resident call")
    rt.close()
    dsa.check_device_errors(dev)
    e2e_s = max_over_ranks(el / args.steps)
    return {"value": n * world / e2e_s, "unit": "query-tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "us_per_step": e2e_s * 1e6,
            "how": "public Python API (launch_sparse_attention_c) called back to back over 4 rotating decode "
                   "batches; every step copies its pinned host inputs (q_nope|q_pe|indices, one block) in and its "
                   "output|lse (one block) out, on separate copy streams ordered by events (copies and event "
                   "calls issued directly to the CUDA runtime); wall clock over all steps / steps; inputs of the "
                   "4 batches together exceed L2 (no flush); every slot's last result checked against the "
                   "device-resident call"}


def e2e_serial_leg(dsa, w, out, lse, args, dev, flush_l2, barrier, max_over_ranks, world):
    """One step at a time: flush, synchronise, copy the pinned inputs in,
    call the public API, copy the results out, synchronise (wall clock)."""
    n = w.num_tokens
    like_in = [w.q_nope, w.q_pe, w.sparse_indices]
    in_offs, in_bytes = _packed(like_in)
    out_like = [torch.empty((n, 16, 512), dtype=torch.bfloat16), torch.empty((n, 16), dtype=torch.float32)]
    out_offs, out_bytes = _packed(out_like)
    h_in = torch.empty(in_bytes, dtype=torch.uint8).pin_memory()
    for t, o in zip(like_in, in_offs):
        _view(h_in, o, t).copy_(t.cpu())
    h_out = torch.empty(out_bytes, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(in_bytes, dtype=torch.uint8, device=dev)
    d_out = torch.empty(out_bytes, dtype=torch.uint8, device=dev)
    d_qn, d_qp, d_idx = (_view(d_in, o, t) for t, o in zip(like_in, in_offs))
    d_o, d_l = (_view(d_out, o, t) for t, o in zip(out_like, out_offs))
    rt = _Runtime()
    s_cur = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p_hin, p_din = ctypes.c_void_p(h_in.data_ptr()), ctypes.c_void_p(d_in.data_ptr())
    p_hout, p_dout = ctypes.c_void_p(h_out.data_ptr()), ctypes.c_void_p(d_out.data_ptr())
    times = []
    barrier()
    # untimed warm-up steps first (at least E2E_WARMUP_STEPS and E2E_WARMUP_SECONDS: see e2e_pipelined_leg)
    k, t_w, warm = 0, time.perf_counter(), True
    while warm or len(times) < args.steps:
        flush_l2()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rt.copy(p_din, p_hin, in_bytes, rt.H2D, s_cur)
        dsa.launch_sparse_attention_c(d_qn, d_qp, w.ckv_cache, w.kpe_cache, d_idx, w.sm_scale, d_o, d_l)
        rt.copy(p_hout, p_dout, out_bytes, rt.D2H, s_cur)
        torch.cuda.synchronize()
        k += 1
        if not warm:
            times.append(time.perf_counter() - t0)
        elif k >= 20000 or (k >= max(args.warmup, E2E_WARMUP_STEPS) and time.perf_counter() - t_w >= E2E_WARMUP_SECONDS):
            warm = False
    if not (torch.equal(_view(h_out, out_offs[0], out_like[0]), out.cpu()) and
            torch.equal(_view(h_out, out_offs[1], out_like[1]), lse.cpu())):
        raise RuntimeError("end-to-end result differs from the device-resident call")
    e2e_s = max_over_ranks(statistics.mean(times))
    dsa.check_device_errors(dev)
    return {"value": n * world / e2e_s, "unit": "query-tokens/s", "us_per_step": e2e_s * 1e6,
            "how": "one step at a time: L2 flush, copy pinned inputs in, launch_sparse_attention_c, copy output|lse "
                   "out (copies issued directly to the CUDA runtime), synchronise; wall clock per step"}


def config5_leg(dsa, lib, lib_mod, args, stream, flush_l2, world, rank, dev, barrier, max_over_ranks, per_rank,
                hbm_peak):
    """Config 5 strong scaling: the 1024-token batch of 256 sequences x 4
    tokens over 131072-slot sequences, whole sequences per rank, each rank
    holding only its sequences' pages.  Per rank: the mean step (events around
    the public call, L2 flushed) and the mean kernel time (library events);
    job time = max over ranks of the mean step."""
    sh = importlib.import_module(f"{PKG}.sharding")
    w5 = sh.shard_config5(world, rank, device=dev)
    n5 = w5.num_tokens
    out5 = torch.empty((n5, 16, 512), dtype=torch.bfloat16, device=dev)
    lse5 = torch.empty((n5, 16), dtype=torch.float32, device=dev)

    def call5():
        dsa.launch_sparse_attention_c(*w5.args(), out5, lse5)

    for _ in range(args.warmup):
        call5()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    step_ms = time_isolated(call5, args.steps, stream, flush_l2)
    barrier()
    ws5 = dsa.workspace_for(dev, n5)
    kern_ms = kernel_events_ms(lib, lib_mod, w5, out5, lse5, ws5, stream, args.steps, flush_l2)
    dsa.check_device_errors(dev)
    gathered = w5.gathered_bytes()
    ranks = per_rank([step_ms * 1000.0, kern_ms * 1000.0, float(n5), float(gathered)])
    job_ms = max_over_ranks(step_ms)
    total_tokens = int(sum(r[2] for r in ranks))
    total_bytes = sum(r[3] for r in ranks)
    del w5, out5, lse5
    torch.cuda.empty_cache()
    return {"tokens": total_tokens, "gpus": world, "us_per_step": job_ms * 1000.0,
            "query_tokens_per_s_job": total_tokens / (job_ms / 1000.0),
            "gathered_gbs_job": total_bytes / (job_ms / 1000.0) / 1e9,
            "per_gpu_frac_of_peak": (total_bytes / world) / (job_ms / 1000.0) / 1e9 / hbm_peak,
            "per_rank": [{"rank": i, "tokens": int(r[2]), "step_us": r[0], "kernel_us": r[1]}
                         for i, r in enumerate(ranks)],
            "how": "sequences sharded over the GPUs (whole sequences, local pools, no collective); per rank: "
                   "step = CUDA events around the public call with L2 flushed before it, kernel = the library's "
                   "events around the launch; job = max over ranks of the mean step"}


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
