"""Benchmark of the B200 KIVI decode-attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config2]
                    [--impl kivi|reference]

Default workload = BASELINE config 2 (Llama-3-8B shape decode): B=64
sequences, Hq=32, Hkv=8, D=128, context U[1024, 8192], 16-token pages
scattered over a shared pool, KIVI INT4 with G=R=128, bf16 q, synthetic seeded
data.  A step = one decode-attention call for all sequences of one layer.
metric = sequence-tokens/s (B / step time), whole job.  With N GPUs the same
64 sequences are split over the ranks by token balancing (strong scaling, no
collective on the data path: every rank decodes whole sequences).

--workload config3 measures the other half of the path, quantize-on-append
64 sequences x 2048-token bf16 chunk per GPU appended to
empty sequences, metric = appended tokens/s.

--workload prefill measures chunked-prefill attention over the compressed
cache: 8 sequences per GPU with 4096 cached tokens each append a 512-token
chunk whose query rows attend causally to the whole cache, metric = query
tokens/s (the reference runs this attention token by token).

--impl reference times the reference's CPU path for the same workload: the
CPU restatement of the reference algorithm (oracle/, the reference has no CPU
implementation of this path) on all host threads, over a bounded sample of the
sequences.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "KIVI-INT4 paged decode-attn seq-tokens/s (HBM GB/s and % of peak in roofline)"
UNIT = "seq-tokens/s"
APPEND_METRIC = "KIVI-INT4 quantize-on-append appended tokens/s (config 3)"
APPEND_UNIT = "tokens/s"
PREFILL_METRIC = "KIVI-INT4 chunked-prefill attention query-tokens/s (TFLOP/s in roofline)"
PREFILL_UNIT = "query-tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="config2",
                    choices=["config2", "config3", "config4", "config4b", "config5", "prefill"])
    ap.add_argument("--impl", default="kivi", choices=["kivi", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=64, help="sequences in the CPU sample")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="token split (config4b): partials over peer memory or NCCL all-gathers")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def make_workload(wl, name: str, rank: int):
    if name == "config3":
        return wl.config3(seed=3000 + rank)
    if name == "config2":
        return wl.config2(seed=1000 + rank)
    if name in ("config4", "config4b"):
        return wl.config4(seed=4000 + rank, B=1 if name == "config4b" else 8)
    return wl.config5(seed=5000 + rank)


# ---------------------------------------------------------------------------
# cache construction on the GPU (through the public append API)
# ---------------------------------------------------------------------------
def build_gpu_cache(ops, w, dev, torch):
    fmt = ops.KiviFormat(w.D, w.group, w.residual, w.bits, w.Hkv)
    cache = ops.KiviPagedCache(fmt, w.num_pages, w.B, dev)
    bt = torch.from_numpy(w.block_tables).to(dev)
    lens = w.lengths.astype(np.int64)
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed)
    oc = torch.from_numpy(np.asarray(w.outlier_channels, np.int64)).to(dev)
    # append in batches of sequences to bound the temporary K/V memory
    per = max(1, int(2_000_000 // max(1, int(lens.mean()))))
    for s0 in range(0, w.B, per):
        s1 = min(w.B, s0 + per)
        T = int(lens[s0:s1].sum())
        k = torch.randn((T, w.Hkv, w.D), generator=gen, device=dev, dtype=torch.float32)
        v = torch.randn((T, w.Hkv, w.D), generator=gen, device=dev, dtype=torch.float32)
        if len(w.outlier_channels):
            k[:, :, oc] *= w.outlier_scale
        k = k.to(torch.bfloat16)
        v = v.to(torch.bfloat16)
        cu = torch.zeros(s1 - s0 + 1, dtype=torch.int32)
        cu[1:] = torch.from_numpy(np.cumsum(lens[s0:s1])).to(torch.int32)
        zero = torch.zeros(s1 - s0, dtype=torch.int32, device=dev)
        ops.paged_append(cache, k, v, cu.to(dev), zero, bt[s0:s1].contiguous(),
                         seq_slots=torch.arange(s0, s1, dtype=torch.int32, device=dev),
                         max_new_tokens=int(lens[s0:s1].max()))
        del k, v
    torch.cuda.synchronize()
    return cache, bt


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML from a
    background thread every ~2 ms while the timed region runs (read-only)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.stop = None
        self.th = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return self
        self.stop = threading.Event()

        def run():
            while not self.stop.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, rs))
                except Exception:
                    pass
                time.sleep(0.002)

        self.th = threading.Thread(target=run, daemon=True)
        self.th.start()
        return self

    def __exit__(self, *a):
        if self.stop is not None:
            self.stop.set()
            self.th.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        sm = [s for s, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(self.max_mhz),
                "reasons": reasons, "samples": len(sm)}


CSRC = ROOT / "truellm-engine_b200" / "csrc"
# the sources each profiled kernel is built from: an ncu figure counts only for
# the build it was taken from
KERNEL_SOURCES = {
    "decode_stream": ["tkv_stream.cu", "tkv_decode_common.cuh", "tkv_frag.cuh", "tkv_common.cuh"],
    "append": ["tkv_append.cu", "tkv_common.cuh"],
    "prefill": ["tkv_prefill.cu", "tkv_umma.cuh", "tkv_frag.cuh", "tkv_common.cuh"],
}


def source_sha(kernel: str) -> str:
    import hashlib
    h = hashlib.sha256()
    for name in KERNEL_SOURCES[kernel]:
        h.update((CSRC / name).read_bytes())
    return h.hexdigest()


def ncu_traffic(profile: str, kernel: str, key: str):
    """Per-launch DRAM traffic (dram__bytes_read + write) from the committed
    ncu summary profiles/<profile>.json, or None when there is none or it was
    taken from other kernel sources than the ones built now."""
    p = ROOT / "profiles" / f"{profile}.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    if d.get("source_sha256") != source_sha(kernel):
        return None
    return d.get(key)


# ---------------------------------------------------------------------------
# CPU timing of the reference algorithm (oracle restatement)
# ---------------------------------------------------------------------------
def cpu_sample_size(lengths, cap: int, token_budget: int = 400000) -> int:
    """Leading sequences of the CPU sample: at most `cap`, at most about
    `token_budget` context tokens (long-context workloads), at least one."""
    n, tok = 0, 0
    for L in lengths[:cap]:
        if n and tok + int(L) > token_budget:
            break
        n, tok = n + 1, tok + int(L)
    return max(1, n)

def cpu_reference_time(O, w, pool_np, ring_np, q_f32, sample, n_threads, repeats=1):
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, w.B)
    st.pool = pool_np
    st.ring = ring_np
    idx = np.arange(sample)
    bt = np.ascontiguousarray(w.block_tables[idx])
    lens = np.ascontiguousarray(w.lengths[idx])
    # the ring is indexed by batch row: use the sample's rows 0..sample-1
    t0 = time.perf_counter()
    for _ in range(repeats):
        st.decode(q_f32[idx], bt, lens, 1.0 / math.sqrt(w.D), n_threads=n_threads)
    return (time.perf_counter() - t0) / repeats


def host_cache_for_reference(O, wl, w, sample):
    """Builds the cache of the first `sample` sequences on the CPU with the
    oracle append (same seeded distribution as the GPU arm)."""
    rng = np.random.default_rng(w.seed)
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, sample)
    for b in range(sample):
        L = int(w.lengths[b])
        k, v = wl.kv_tokens(rng, L, w.Hkv, w.D, w.outlier_channels, w.outlier_scale)
        cu = np.zeros(sample + 1, np.int32)
        cu[b + 1:] = L
        lens_old = np.zeros(sample, np.int32)
        st.append(wl.to_bits(k, "bf16"), wl.to_bits(v, "bf16"), True, cu, lens_old,
                  np.ascontiguousarray(w.block_tables[:sample]))
    return st


def workload_desc(name: str, w) -> str:
    """The workload string of the JSON line's config (the same in both arms)."""
    return {"config2": f"config2: B={w.B} Hq={w.Hq} Hkv={w.Hkv} D={w.D} L~U[1024,8192]",
            "config4": f"config4 run A: B={w.B} Hq={w.Hq} Hkv={w.Hkv} D={w.D} L=131072",
            "config4b": f"config4 run B: B=1 Hq={w.Hq} Hkv={w.Hkv} D={w.D} L=131072",
            "config5": f"config5: B={w.B} Hq={w.Hq} Hkv={w.Hkv} D={w.D} L~logU[128,32768] "
                       "INT4 x128 + INT2 x128"}[name] + f" G={w.group} R={w.residual}"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as O
    O.build()
    wl = importlib.import_module("truellm-engine_b200.workloads")
    w = (wl.config4(seed=4000, B=1) if args.workload == "config4b"
         else make_workload(wl, args.workload, 0))
    sample = cpu_sample_size(w.lengths, args.cpu_sample)
    st = host_cache_for_reference(O, wl, w, sample)
    rng = np.random.default_rng(w.seed + 1)
    q = wl.bits_to_f32(wl.f32_to_bf16_bits(rng.standard_normal((w.B, w.Hq, w.D))), "bf16")
    threads = os.cpu_count() or 1
    bt = np.ascontiguousarray(w.block_tables[:sample])
    lens = np.ascontiguousarray(w.lengths[:sample])
    # each step decodes the whole sample (all 64 sequences at config 2, about
    # a second on 16 threads): at most 10 timed steps keep the arm to minutes
    steps, warmup = max(1, min(args.steps, 10)), max(1, min(args.warmup, 2))
    for _ in range(warmup):
        st.decode(q[:sample], bt, lens, 1 / math.sqrt(w.D), n_threads=threads)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        st.decode(q[:sample], bt, lens, 1 / math.sqrt(w.D), n_threads=threads)
        times.append(time.perf_counter() - t0)
    t = float(np.mean(times))
    value = sample / t
    whole = sample == w.B
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": workload_desc(args.workload, w) if whole else
                   f"{workload_desc(args.workload, w)}: sample of {sample} sequences",
                   "global_batch": sample, "mean_context": float(lens.mean())},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} of the {w.B} sequences of {args.workload} (mean "
                                   f"context {lens.mean():.0f}), CPU restatement of the "
                                   "reference algorithm: fp64 attention over the dequantised "
                                   "pages, all host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
class DecodePart:
    """One decode call of a rank's step: a cache, its q/out and tables."""

    def __init__(self, ops, wl, torch, w, dev, label):
        self.w, self.label = w, label
        self.cache, self.bt = build_gpu_cache(ops, w, dev, torch)
        self.lens = torch.from_numpy(w.lengths).to(dev)
        rng = np.random.default_rng(w.seed + 1)
        self.q_np = wl.f32_to_bf16_bits(rng.standard_normal((w.B, w.Hq, w.D)))
        self.q = torch.from_numpy(self.q_np.view(np.int16)).view(torch.bfloat16).to(dev)
        self.out = torch.empty_like(self.q)
        self.max_ctx = int(w.lengths.max())
        self.scale = 1.0 / math.sqrt(w.D)
        # workspace: split partials + counters, zeroed once (calls leave counters zero)
        self.ws = torch.zeros(ops.decode_workspace_bytes(w.B, w.Hq, w.D, self.max_ctx),
                              dtype=torch.uint8, device=dev)
        self.q_host = torch.from_numpy(self.q_np.view(np.int16)).view(torch.bfloat16).pin_memory()
        self.lens_host = torch.from_numpy(w.lengths.copy()).pin_memory()
        self.out_host = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.q_dev = torch.empty_like(self.q)
        self.lens_dev = torch.empty_like(self.lens)
        self.calls = {}  # prepared decode calls per (q, lens, stream)


def _stream_id(st) -> int:
    return st.cuda_stream if hasattr(st, "cuda_stream") else int(st)


def decode_plan(args, wl, ops, torch, dev, rank, world):
    """The rank's share of the workload: (parts, total sequences, scaling,
    layout, algorithmic bytes per step on this rank, token-split decoder)."""
    SH = importlib.import_module("truellm-engine_b200.sharding")
    name = args.workload
    if name == "config2":  # the 64 sequences, split over the ranks by token balancing
        w = make_workload(wl, name, 0)
        if world == 1:
            return ([DecodePart(ops, wl, torch, w, dev, "all")], w.B, "strong",
                    "one GPU", wl.decode_algorithmic_bytes(w), None, w)
        mine = SH.balance_sequences(w.lengths, world)[rank]
        sub = wl.subset(w, mine)
        return ([DecodePart(ops, wl, torch, sub, dev, f"{len(mine)} sequences")], w.B, "strong",
                f"token-balanced sequences x{world}", wl.decode_algorithmic_bytes(sub), None, w)
    if name == "config4":  # run A: kv heads split over the ranks, same 8 sequences
        w = make_workload(wl, name, 0)
        kvh, qh = SH.head_shard(w.Hkv, w.Hq, world, rank)
        sub = wl.subset(w, Hkv=len(kvh), Hq=len(qh))
        return ([DecodePart(ops, wl, torch, sub, dev, f"kv heads {kvh.start}-{kvh.stop - 1}")],
                w.B, "strong", f"kv-head-sharded x{world}", wl.decode_algorithmic_bytes(sub),
                None, w)
    if name == "config4b":  # run B: one sequence split by tokens over the ranks
        w = wl.config4(seed=4000, B=1)
        part = DecodePart(ops, wl, torch, w, dev, "one sequence")
        dec = SH.TokenSplitDecoder(1, w.Hq, w.D, part.max_ctx, w.residual, w.group, dev,
                                   exchange=args.exchange)
        alg = wl.token_split_bytes(w, dec.lo, dec.hi, dec.last)
        how = ("one-call decode" if world == 1 else
               "partials stored to every GPU over NVLink, then merged" if args.exchange == "peer"
               else "NCCL all-gather of partials, then merged")
        return ([part], 1, "strong", f"token-split x{world} ({how})", alg, dec, w)
    # config5: 256 sequences balanced by tokens; sequences 0-127 INT4, 128-255 INT2
    w = make_workload(wl, "config5", 0)
    mine = SH.balance_sequences(w.lengths, world)[rank]
    parts, alg = [], 0
    for bits, sel in ((4, mine[mine < w.B // 2]), (2, mine[mine >= w.B // 2])):
        if len(sel):
            sub = wl.subset(w, sel, bits=bits)
            parts.append(DecodePart(ops, wl, torch, sub, dev, f"INT{bits} x{len(sel)}"))
            alg += wl.decode_algorithmic_bytes(sub)
    return parts, w.B, "strong", f"token-balanced sequences x{world}", alg, None, w


def run_kivi(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 or args.workload == "config4b":
        import datetime
        if "MASTER_ADDR" not in os.environ:  # single process: a group of one
            os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(29500 + os.getpid() % 1000),
                              RANK="0", WORLD_SIZE="1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ops = importlib.import_module("truellm-engine_b200.ops")
    wl = importlib.import_module("truellm-engine_b200.workloads")
    parts, total_seqs, scaling, layout, alg_bytes, dec, w = decode_plan(
        args, wl, ops, torch, dev, rank, world)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    # the token split is launch-bound (range decode, reduce + publish to the
    # peers, wait + merge per step): its step is captured once in a CUDA graph
    # and replayed
    graph = None
    if dec is not None:
        p0 = parts[0]
        try:
            graph = dec.capture(p0.cache, p0.q, p0.bt, p0.lens, p0.out, scale=p0.scale, err=err)
        except Exception as e:  # capture not supported here: eager calls
            print(f"rank {rank}: CUDA graph capture failed ({e!r}); eager token split",
                  file=sys.stderr)
        stream = torch.cuda.current_stream()

    def decode(p, q, lens, st):
        if graph is not None:  # captured over p.q / p.lens
            if q is not p.q:
                p.q.copy_(q, non_blocking=True)
                p.lens.copy_(lens, non_blocking=True)
            graph.replay()
        elif dec is not None:
            dec(p.cache, q, p.bt, lens, p.out, scale=p.scale, err=err, stream=st)
        else:  # the C entry point with its arguments bound once per (buffers, stream)
            key = (q.data_ptr(), lens.data_ptr(), _stream_id(st))
            call = p.calls.get(key)
            if call is None:
                call = p.calls[key] = ops.PreparedDecode(
                    p.cache, q, p.bt, lens, p.max_ctx, p.out, p.ws, scale=p.scale, err=err,
                    stream=st)
            call()

    # parts of one step (config 5: the INT4 and the INT2 sequences) run on
    # their own streams so one launch's tail overlaps the other's work
    side = [torch.cuda.Stream() for _ in parts[1:]]

    def run_parts(fn):
        cur = torch.cuda.current_stream()  # the capture stream while a graph is captured
        if not side:
            fn(parts[0], cur)
            return
        for s_ in side:
            s_.wait_stream(cur)
        fn(parts[0], cur)
        for p, s_ in zip(parts[1:], side):
            with torch.cuda.stream(s_):
                fn(p, s_)
        for s_ in side:
            cur.wait_stream(s_)

    step_graph = None

    def step(ev=None):
        # one decode step: one decode launch per part (split + fused merge); the
        # token-split layout adds the all-gather of partials and the merge
        if ev is not None:
            ev[0].record(stream)
        if step_graph is not None:
            step_graph.replay()
        else:
            run_parts(lambda p, s_: decode(p, p.q, p.lens, s_))
        if ev is not None:
            ev[1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    # Above one GPU a rank's step is 20-90 us of GPU work, and a config-5 step
    # (two calls on two streams) costs ~50 us of Python to enqueue while every
    # rank's loop shares the host's cores: the step's launches are captured
    # once in a CUDA graph and replayed, so the host's launch rate does not
    # set the measured step.  The end-to-end leg below keeps the direct calls.
    if dec is None and (world > 1 or len(parts) > 1):
        torch.cuda.synchronize()
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                run_parts(lambda p, s_: decode(p, p.q, p.lens, s_))
            step_graph = g
            for _ in range(args.warmup):
                step()
        except Exception as e:  # capture not supported here: direct calls
            print(f"rank {rank}: CUDA graph capture failed ({e!r}); direct calls",
                  file=sys.stderr)
            step_graph = None
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the K timed steps back to back (events only around the whole run) ...
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    t_total = start.elapsed_time(stop) / 1e3
    # ... then the same K steps once more with events around each launch, for
    # the kernel time of the roofline
    for i in range(args.steps):
        step(evs[i])
    torch.cuda.synchronize()
    t_split = float(np.mean([a.elapsed_time(b) for a, b in evs])) / 1e3
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag {int(err.item()):#x}")
    t_step = t_total / args.steps
    times = torch.tensor([t_step, t_split], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_step, t_split = float(times[0]), float(times[1])

    # ---- end to end through the public API with host buffers ----
    # Every step copies its q and lengths from pinned host memory and its
    # output back.  With the plain decode call the steps are pipelined the way
    # a serving loop runs them: two buffer sets, the input copy of step i+1
    # (its own stream) and the output copy of step i-1 (another stream)
    # overlap the decode of step i; events keep each set's copy, decode and
    # read-back in order.
    pipelined = dec is None and graph is None

    def e2e_part(p, st):
        p.q_dev.copy_(p.q_host, non_blocking=True)
        p.lens_dev.copy_(p.lens_host, non_blocking=True)
        decode(p, p.q_dev, p.lens_dev, st)
        p.out_host.copy_(p.out, non_blocking=True)

    if pipelined:
        for p in parts:
            p.h2d, p.d2h = torch.cuda.Stream(), torch.cuda.Stream()
            p.sets = []
            for _ in range(2):
                q_d, l_d, o_d = (torch.empty_like(p.q), torch.empty_like(p.lens),
                                 torch.empty_like(p.out))
                p.sets.append({"q": q_d, "lens": l_d, "out": o_d,
                               "out_host": torch.empty(p.out.shape, dtype=p.out.dtype).pin_memory(),
                               "ev_in": torch.cuda.Event(), "ev_k": torch.cuda.Event(),
                               "ev_out": torch.cuda.Event(), "call": {}})
        step_no = [0]

        def e2e_pipe_part(p, st):
            b = p.sets[step_no[0] % 2]
            p.h2d.wait_event(b["ev_k"])  # the decode two steps back has read this set
            with torch.cuda.stream(p.h2d):
                b["q"].copy_(p.q_host, non_blocking=True)
                b["lens"].copy_(p.lens_host, non_blocking=True)
                b["ev_in"].record(p.h2d)
            st.wait_event(b["ev_in"])
            st.wait_event(b["ev_out"])  # its output two steps back has been read back
            key = _stream_id(st)
            if key not in b["call"]:
                b["call"][key] = ops.PreparedDecode(p.cache, b["q"], p.bt, b["lens"], p.max_ctx,
                                                    b["out"], p.ws, scale=p.scale, err=err,
                                                    stream=st)
            b["call"][key]()
            b["ev_k"].record(st)
            p.d2h.wait_event(b["ev_k"])
            with torch.cuda.stream(p.d2h):
                b["out_host"].copy_(b["out"], non_blocking=True)
                b["ev_out"].record(p.d2h)

    def e2e_step():
        if pipelined:
            run_parts(e2e_pipe_part)
            step_no[0] += 1
        else:
            run_parts(e2e_part)

    def e2e_drain():  # the timed region ends when the last read-back is done
        if pipelined:
            for p in parts:
                stream.wait_stream(p.d2h)

    for _ in range(args.warmup):
        e2e_step()
    e2e_drain()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if pipelined:
        for p in parts:
            p.h2d.wait_event(e0)
    for _ in range(args.steps):
        e2e_step()
    e2e_drain()
    e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = torch.tensor([e0.elapsed_time(e1) / 1e3 / args.steps], dtype=torch.float64,
                         device=dev)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    t_e2e = float(t_e2e[0])
    h2d = sum(p.q_host.numel() * 2 + p.lens_host.numel() * 4 for p in parts)
    d2h = sum(p.out_host.numel() * 2 for p in parts)

    peak, peak_kind = peaks()
    achieved = alg_bytes / t_split / 1e9
    traffic = (ncu_traffic(f"decode_stream_{args.workload}", "decode_stream",
                           "dram_bytes_per_launch") if world == 1 else None)
    # our kernel launches per step: the token split runs three (range decode,
    # its reduce + publish to the peers, wait + merge); otherwise one or two
    # per decode call (ops.decode_launches)
    n_launch = (3 if dec is not None and not dec.single else
                sum(ops.decode_launches(p.w.B, p.w.Hq, p.w.Hkv, p.max_ctx) for p in parts))

    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            try:
                from oracle import oracle as O
                O.build()
                p0 = parts[0]
                sample = cpu_sample_size(p0.w.lengths, args.cpu_sample)
                pool_np = p0.cache.pool.cpu().numpy()
                ring_np = p0.cache.ring.cpu().numpy().view(np.uint16)
                qf = p0.q.float().cpu().numpy()
                threads = os.cpu_count() or 1
                tc = cpu_reference_time(O, p0.w, pool_np, ring_np, qf, sample, threads)
                cpu = {"value": sample / tc, "unit": UNIT, "cores": threads, "kind": "port",
                       "sample": f"{sample} of the {p0.w.B} sequences (mean context "
                                 f"{p0.w.lengths[:sample].mean():.0f}), CPU restatement of the "
                                 "reference algorithm (fp64), all host threads"}
            except Exception as e:  # the baseline is reported, never required
                cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                       "sample": f"failed: {e!r}"[:200]}
        line = {
            "metric": METRIC, "value": total_seqs / t_step, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "int4/bf16" if args.workload != "config5" else "int4+int2/bf16",
            "data": "synthetic (seeded N(0,1) K/V, key outlier channels x8)",
            "config": {"workload": workload_desc(args.workload, w),
                       "global_batch": total_seqs, "mean_context": float(w.lengths.mean()),
                       "parallelism": layout, "rank0_parts": [p.label for p in parts],
                       "launch": ("one CUDA graph per step" if graph is not None or
                                  step_graph is not None else "direct C calls"),
                       "l2": "inputs larger than L2 (cache %.0f MB per rank)" % (alg_bytes / 1e6)},
            "gpu_launches": n_launch * args.steps,
            "e2e": {"value": total_seqs / t_e2e, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic,
                         "kernel": "decode_stream_kernel<128,%d,128>%s" % (
                             w.bits, (" (range) + stream_merge_kernel (publish) + ex_merge_kernel" if args.exchange == "peer"
                              else " (range) + stream_merge_kernel + all-gather + merge_kernel")
                             if dec is not None and not dec.single else
                             " + stream_merge_kernel" if n_launch > len(parts) else
                             " (merge fused)"),
                         "alg_bytes_per_launch": alg_bytes,
                         "kernel_ms": t_split * 1e3},
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line))
    step_graph = None
    if graph is not None:  # a graph holding collectives goes before the group
        torch.cuda.synchronize()
        del graph
    if dec is not None:  # peer mappings are released collectively
        dec.close()
    if world > 1 or dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# config 3: quantize-on-append
# ---------------------------------------------------------------------------
def append_inputs(wl, w, torch, dev):
    """Seeded bf16 K/V [B*T, Hkv, D] (keys N(0,1) with outlier channels x8)."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed)
    k = torch.randn((w.B * w.T, w.Hkv, w.D), generator=gen, device=dev, dtype=torch.float32)
    v = torch.randn((w.B * w.T, w.Hkv, w.D), generator=gen, device=dev, dtype=torch.float32)
    oc = torch.from_numpy(np.asarray(w.outlier_channels, np.int64)).to(dev)
    k[:, :, oc] *= w.outlier_scale
    return k.to(torch.bfloat16), v.to(torch.bfloat16)


def cpu_append_time(O, wl, w, sample, reps=1):
    """Oracle append of the first `sample` sequences' chunks (single thread)."""
    rng = np.random.default_rng(w.seed)
    T = sample * w.T
    k = wl.f32_to_bf16_bits(rng.standard_normal((T, w.Hkv, w.D)).astype(np.float32))
    v = wl.f32_to_bf16_bits(rng.standard_normal((T, w.Hkv, w.D)).astype(np.float32))
    cu = (np.arange(sample + 1) * w.T).astype(np.int32)
    bt = np.ascontiguousarray(w.block_tables[:sample])
    best = None
    for _ in range(reps):
        st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, sample)
        t0 = time.perf_counter()
        st.append(k, v, True, cu, np.zeros(sample, np.int32), bt)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return best


def run_append_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as O
    O.build()
    wl = importlib.import_module("truellm-engine_b200.workloads")
    w = make_workload(wl, "config3", 0)
    sample = max(1, min(args.cpu_sample // 2, w.B))
    times = [cpu_append_time(O, wl, w, sample) for _ in range(max(1, min(args.steps, 3)))]
    t = float(np.mean(times))
    value = sample * w.T / t
    line = {
        "impl": "reference", "metric": APPEND_METRIC, "value": value, "unit": APPEND_UNIT,
        "n_gpus": args.gpus, "steps": len(times), "warmup": 0, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8/f32",
        "data": "synthetic",
        "config": {"workload": f"config3: sample of {sample} sequences x {w.T} tokens"},
        "cpu_baseline": {"value": value, "unit": APPEND_UNIT, "cores": 1, "kind": "port",
                         "sample": f"{sample} of the {w.B} 2048-token chunks, CPU restatement "
                                   "of the reference quantizer and page packing, one thread"},
        "e2e": {"value": value, "unit": APPEND_UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_append(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ops = importlib.import_module("truellm-engine_b200.ops")
    wl = importlib.import_module("truellm-engine_b200.workloads")
    w = make_workload(wl, "config3", rank)
    fmt = ops.KiviFormat(w.D, w.group, w.residual, w.bits, w.Hkv)
    cache = ops.KiviPagedCache(fmt, w.num_pages, w.B, dev)
    bt = torch.from_numpy(w.block_tables).to(dev)
    k, v = append_inputs(wl, w, torch, dev)
    cu = (torch.arange(w.B + 1, dtype=torch.int32) * w.T).to(dev)
    lens0 = torch.zeros(w.B, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def step(kk, vv):
        # one call = flush kernel + residual-ring kernel (2 launches); the
        # sequences start empty every call, so each call redoes the same work
        ops.paged_append(cache, kk, vv, cu, lens0, bt, max_new_tokens=w.T, err=err,
                         stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step(k, v)
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            step(k, v)
            evs[i][1].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag {int(err.item()):#x}")
    t_step = start.elapsed_time(stop) / 1e3 / args.steps
    t_call = float(np.mean([a.elapsed_time(b) for a, b in evs])) / 1e3
    times = torch.tensor([t_step, t_call], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_step, t_call = float(times[0]), float(times[1])

    # ---- end to end: K/V from pinned host memory, error word read back ----
    k_host = k.cpu().pin_memory()
    v_host = v.cpu().pin_memory()
    err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
    k_dev, v_dev = torch.empty_like(k), torch.empty_like(v)
    n_e2e = max(3, min(args.steps, 20))

    def e2e_step():
        k_dev.copy_(k_host, non_blocking=True)
        v_dev.copy_(v_host, non_blocking=True)
        step(k_dev, v_dev)
        err_host.copy_(err, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = torch.tensor([e0.elapsed_time(e1) / 1e3 / n_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    t_e2e = float(t_e2e[0])

    alg = wl.append_algorithmic_bytes(w)
    peak, peak_kind = peaks()
    achieved = alg / t_call / 1e9
    traffic = ncu_traffic("append_config3", "append", "dram_bytes_per_call")
    if rank == 0:
        cpu = None
        if world == 1:
            try:
                from oracle import oracle as O
                O.build()
                sample = max(1, min(args.cpu_sample // 2, w.B))
                tc = cpu_append_time(O, wl, w, sample)
                cpu = {"value": sample * w.T / tc, "unit": APPEND_UNIT, "cores": 1,
                       "kind": "port",
                       "sample": f"{sample} of the {w.B} 2048-token chunks, CPU restatement of "
                                 "the reference quantizer and page packing, one thread"}
            except Exception as e:  # the baseline is reported, never required
                cpu = {"value": None, "unit": APPEND_UNIT, "cores": 1, "kind": "port",
                       "sample": f"failed: {e!r}"[:200]}
        line = {
            "metric": APPEND_METRIC, "value": world * w.B * w.T / t_step, "unit": APPEND_UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16->int4",
            "data": "synthetic (seeded N(0,1) K/V, 3 key outlier channels x8)",
            "config": {"workload": f"config3: B={w.B}/GPU x {w.T}-token bf16 chunk, Hkv={w.Hkv} "
                                   f"D={w.D} G={w.group} R={w.residual} INT{w.bits}",
                       "global_batch": world * w.B, "parallelism": f"sequence-sharded x{world}",
                       "l2": "inputs larger than L2 (%.0f MB per call)" % (alg / 1e6)},
            "gpu_launches": 2 * args.steps,
            "e2e": {"value": world * w.B * w.T / t_e2e, "unit": APPEND_UNIT,
                    "h2d_bytes_per_step": 2 * k.numel() * 2, "d2h_bytes_per_step": 4},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": "flush_groups_kernel<128,4,128> + residual_write_kernel<128>",
                         "alg_bytes_per_launch": alg, "kernel_ms": t_call * 1e3},
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# chunked prefill over the compressed cache
# ---------------------------------------------------------------------------
def prefill_inputs(ops, wl, w, torch, dev):
    """The cache after the chunk's append (history + chunk appended through the
    public API) and the chunk's seeded bf16 query rows."""
    fmt = ops.KiviFormat(w.D, w.group, w.residual, w.bits, w.Hkv)
    cache = ops.KiviPagedCache(fmt, w.num_pages, w.B, dev)
    bt = torch.from_numpy(w.block_tables).to(dev)
    L = w.hist + w.chunk
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed)
    k = torch.randn((w.B * L, w.Hkv, w.D), generator=gen, device=dev, dtype=torch.float32)
    v = torch.randn((w.B * L, w.Hkv, w.D), generator=gen, device=dev, dtype=torch.float32)
    oc = torch.from_numpy(np.asarray(w.outlier_channels, np.int64)).to(dev)
    k[:, :, oc] *= w.outlier_scale
    cu = (torch.arange(w.B + 1, dtype=torch.int32) * L).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.paged_append(cache, k.to(torch.bfloat16), v.to(torch.bfloat16), cu,
                     torch.zeros(w.B, dtype=torch.int32, device=dev), bt, max_new_tokens=L,
                     err=err)
    q = torch.randn((w.B * w.chunk, w.Hq, w.D), generator=gen, device=dev).to(torch.bfloat16)
    cu_q = (torch.arange(w.B + 1, dtype=torch.int32) * w.chunk).to(dev)
    lens = torch.full((w.B,), L, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag {int(err.item()):#x}")
    return cache, bt, q, cu_q, lens


def cpu_prefill_time(O, wl, w, threads):
    """Oracle prefill of sequence 0 (all kv heads over `threads` threads): the
    same chunk / history shape, its own seeded inputs."""
    rng = np.random.default_rng(w.seed)
    L = w.hist + w.chunk
    k = wl.f32_to_bf16_bits(rng.standard_normal((L, w.Hkv, w.D)).astype(np.float32))
    v = wl.f32_to_bf16_bits(rng.standard_normal((L, w.Hkv, w.D)).astype(np.float32))
    bt = np.ascontiguousarray(w.block_tables[:1])
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1)
    st.append(k, v, True, np.array([0, L], np.int32), np.zeros(1, np.int32), bt)
    q = wl.bits_to_f32(wl.f32_to_bf16_bits(
        rng.standard_normal((w.chunk, w.Hq, w.D)).astype(np.float32)), "bf16")
    t0 = time.perf_counter()
    st.prefill(q, np.array([0, w.chunk], np.int32), bt, np.array([L], np.int32),
               1 / math.sqrt(w.D), n_threads=threads)
    return time.perf_counter() - t0


def run_prefill_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as O
    O.build()
    wl = importlib.import_module("truellm-engine_b200.workloads")
    w = wl.prefill(seed=6000)
    threads = os.cpu_count() or 1
    times = [cpu_prefill_time(O, wl, w, threads) for _ in range(max(1, min(args.steps, 2)))]
    t = float(np.mean(times))
    value = w.chunk / t
    line = {
        "impl": "reference", "metric": PREFILL_METRIC, "value": value, "unit": PREFILL_UNIT,
        "n_gpus": args.gpus, "steps": len(times), "warmup": 0, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": f"prefill: sample of 1 sequence, {w.hist} cached + {w.chunk} "
                               "chunk tokens"},
        "cpu_baseline": {"value": value, "unit": PREFILL_UNIT, "cores": threads, "kind": "port",
                         "sample": f"1 of the {w.B} sequences (all {w.Hkv} kv heads), CPU "
                                   "restatement of the causal attention over the dequantised "
                                   "cache, fp64"},
        "e2e": {"value": value, "unit": PREFILL_UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_prefill(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ops = importlib.import_module("truellm-engine_b200.ops")
    wl = importlib.import_module("truellm-engine_b200.workloads")
    w = wl.prefill(seed=6000 + rank)
    cache, bt, q, cu_q, lens = prefill_inputs(ops, wl, w, torch, dev)
    out = torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    T = w.B * w.chunk

    def step(qq, oo):
        ops.paged_prefill(cache, qq, cu_q, bt, lens, max_q_tokens=w.chunk, out=oo, err=err,
                          stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step(q, out)
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            step(q, out)
            evs[i][1].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag {int(err.item()):#x}")
    t_step = start.elapsed_time(stop) / 1e3 / args.steps
    t_call = float(np.mean([a.elapsed_time(b) for a, b in evs])) / 1e3
    times = torch.tensor([t_step, t_call], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_step, t_call = float(times[0]), float(times[1])

    # ---- end to end: q from pinned host memory, the attention output read back ----
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_dev, o_dev = torch.empty_like(q), torch.empty_like(out)
    n_e2e = max(3, min(args.steps, 20))

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        step(q_dev, o_dev)
        out_host.copy_(o_dev, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = torch.tensor([e0.elapsed_time(e1) / 1e3 / n_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    t_e2e = float(t_e2e[0])

    flops = wl.prefill_flops(w)
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(pk.get("bf16_tflops", 1590.0))
    peak_kind = "measured (cuBLAS bf16 burst)" if "bf16_tflops" in pk else "fallback"
    achieved = flops / t_call / 1e12
    traffic = ncu_traffic("prefill_umma_chunk512", "prefill", "dram_bytes_per_launch")
    if rank == 0:
        cpu = None
        if world == 1:
            try:
                from oracle import oracle as O
                O.build()
                threads = os.cpu_count() or 1
                tc = cpu_prefill_time(O, wl, w, threads)
                cpu = {"value": w.chunk / tc, "unit": PREFILL_UNIT, "cores": threads,
                       "kind": "port",
                       "sample": f"1 of the {w.B} sequences (all {w.Hkv} kv heads), CPU "
                                 "restatement of the causal attention over the dequantised "
                                 "cache, fp64"}
            except Exception as e:  # the baseline is reported, never required
                cpu = {"value": None, "unit": PREFILL_UNIT, "cores": 1, "kind": "port",
                       "sample": f"failed: {e!r}"[:200]}
        line = {
            "metric": PREFILL_METRIC, "value": world * T / t_step, "unit": PREFILL_UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4/bf16 (f16 MMA, f32 accumulate)",
            "data": "synthetic (seeded N(0,1) K/V/q, 3 key outlier channels x8)",
            "config": {"workload": f"prefill: B={w.B}/GPU x ({w.hist} cached + {w.chunk} chunk) "
                                   f"tokens, Hq={w.Hq} Hkv={w.Hkv} D={w.D} G={w.group} "
                                   f"R={w.residual} INT{w.bits}",
                       "global_batch": world * w.B, "parallelism": f"sequence-sharded x{world}",
                       "l2": "compute-bound; the cache (%.0f MB) is read from L2 after the "
                             "first row tile" % (w.B * w.Hkv * (w.hist + w.chunk) * 136 / 1e6)},
            "gpu_launches": args.steps,
            "e2e": {"value": world * T / t_e2e, "unit": PREFILL_UNIT,
                    "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": out.numel() * 2},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "kernel": "prefill_umma_kernel<128,4,128>",
                         "flops_per_launch": flops, "kernel_ms": t_call * 1e3},
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.workload == "prefill":
        return run_prefill_reference(args) if args.impl == "reference" else run_prefill(args)
    if args.workload == "config3":
        return run_append_reference(args) if args.impl == "reference" else run_append(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_kivi(args)


if __name__ == "__main__":
    sys.exit(main())
