"""Encoder throughput benchmark (bulk document embedding of the config-4 corpus).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the config-4 corpus, 131,072 synthetic documents with token counts
clip(round(exp(N(5.0, 0.7))), 16, 512) (seed 5), sorted by length and packed
into padded batches of <= 16,384 tokens.  One step = every rank encodes
`--batches-per-step` of those batches (a seeded sample per rank, the same
count on every rank: weak scaling), through the full 12-layer XTR-base
encoder (random-init N(0, 0.02) weights quantized to Q4_K; synthetic ids).
The metric is valid (unpadded) encoder tokens per second over all ranks.

  value  device-resident inputs, one wc_t5_forward_many_device call per step
         (the handle's two compute lanes), device time of the K steps (CUDA
         events on the launching stream, barrier + synchronize on both sides,
         max over ranks)
  e2e    the public C ABI call wc_t5_forward_many with page-locked host
         buffers, one call per step: the H2D copy of ids/lengths and the D2H
         copy of the raw [B,L,128] projection and norms are inside the timed
         region
  corpus the whole corpus once, dealt to the ranks by LPT and encoded through
         witchcraft_b200.pool (strong scaling, wall clock, max over ranks)
Clocks are sampled by one nvidia-smi process (on local rank 0) for all GPUs
of the job during each timed region.
Multi-GPU: one process per GPU (torchrun), each rank a replica with its own
batches; no collective on the data path (NCCL only for the barrier and the
max-over-ranks of the timings).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "encoder tokens/sec XTR-base Q4_K (bulk embedding, config 4)"
UNIT = "tokens/s"
MAX_BATCH_TOKENS = 16384
LAUNCHES_PER_FORWARD_PER_LAYER = 7   # qkv gemm, attention, o gemm, rmsnorm, wi gemm, wo gemm, rmsnorm
# dram read+write bytes per launch of the dominant kernel (the gated-GELU GEMM
# at M = 16,384), from one ncu capture of `bench.py --profile-kernel geglu`
# (dram__bytes_read.sum + dram__bytes_write.sum); re-captured when the kernel changes
NCU_TRAFFIC_BYTES = 49352960  # 31.49 MB read + 17.86 MB written


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["bf16_tflops"], d.get("bf16_tflops_sustained"), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region: one
    sampler process (on local rank 0) covering every GPU of the job."""

    def __init__(self, indices):
        self.index = ",".join(str(i) for i in indices)
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        # one nvidia-smi process sampling every 100 ms (-lms), read line by
        # line, so a short timed region still gets several samples
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self._p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                        "--format=csv,noheader,nounits", "-lms", "100"],
                                       stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._p = None
            return self

        def run():
            for line in self._p.stdout:
                if self._stop.is_set():
                    break
                vals = [v.strip() for v in line.strip().split(",")]
                if len(vals) == 6:
                    self.rows.append((time.time(), vals))
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        # nvidia-smi's start-up (NVML initialisation) stalls CUDA calls of the
        # processes on these GPUs for a moment: let it finish before the
        # timed region starts (the first sample row marks it)
        t0 = time.time()
        while not self.rows and time.time() - t0 < 10:
            time.sleep(0.02)
        return self

    def mark(self, start: bool):
        """Bounds of the timed region: stop() reports only samples inside it."""
        if start:
            self.t_start = time.time()
        else:
            self.t_end = time.time()

    def stop(self):
        self._stop.set()
        if getattr(self, "_p", None) is not None:
            self._p.terminate()  # the sampler process this object started
            try:
                self._p.wait(timeout=5)
            except Exception:
                self._p.kill()
        if self._t:
            self._t.join(timeout=10)
        t0, t1 = getattr(self, "t_start", None), getattr(self, "t_end", None)
        rows = [v for t, v in self.rows if t0 is None or t1 is None or t0 <= t <= t1]
        window = "timed region"
        if not rows:  # a region shorter than the sampling period
            rows, window = [v for _, v in self.rows], "whole sampler run (no sample inside the timed region)"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[2 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows), "window": window}


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _plan(world: int, rank: int, per_step: int, total_steps: int, seed: int = 17):
    from witchcraft_b200 import shard
    lengths = shard.config4_lengths()
    batches = shard.plan_batches(lengths, MAX_BATCH_TOKENS)
    rng = np.random.default_rng(seed)
    order = rng.permutation(len(batches))
    need = per_step * total_steps
    # rank r walks its own disjoint slice of a seeded permutation of the corpus
    mine = [batches[order[(rank * need + i) % len(batches)]] for i in range(need)]
    return lengths, mine


def _make_inputs(lengths, batch, rng):
    B, L = len(batch.docs), batch.L
    ids = np.zeros((B, L), np.uint32)
    lens = lengths[batch.docs].astype(np.int32)
    for b, n in enumerate(lens):
        ids[b, :n] = rng.integers(3, 32128, n)
    return ids, lens


def cpu_reference_leg(model, lengths, target_s: float = 12.0, seed: int = 23, enc=None):
    """Times the reference's f32 CPU encoder algorithm, restated with torch's
    MKL GEMMs (oracle/torch_ref.py), on a bounded sample of config-4
    documents encoded one at a time as the reference's Embedder does, with
    every host core (torchrun's OMP_NUM_THREADS=1 is overridden)."""
    from oracle.torch_ref import TorchCPUEncoder
    cores = os.cpu_count() or 1
    enc = enc or TorchCPUEncoder(model, threads=cores)
    rng = np.random.default_rng(seed)
    docs = rng.choice(len(lengths), 256, replace=False)
    enc.encode_one(rng.integers(3, 32128, int(lengths[docs[0]])))  # warm the thread pool
    toks = 0
    n_docs = 0
    t0 = time.perf_counter()
    for d in docs:
        n = int(lengths[d])
        enc.encode_one(rng.integers(3, 32128, n))
        toks += n
        n_docs += 1
        if time.perf_counter() - t0 > target_s:
            break
    dt = time.perf_counter() - t0
    return {"value": toks / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n_docs} config-4 documents ({toks} tokens) encoded one at a time (batch 1, as the "
                      f"reference's Embedder does), f32, oracle/torch_ref.py (torch CPU, MKL GEMMs)"}


def run_reference(args):
    world, rank, local = _dist_env()
    if rank != 0:
        return
    from witchcraft_b200 import shard
    from witchcraft_b200.synth import make_synthetic_model
    model = make_synthetic_model(seed=0)
    lengths = shard.config4_lengths()
    from oracle.torch_ref import TorchCPUEncoder
    enc = TorchCPUEncoder(model, threads=os.cpu_count() or 1)
    vals = []
    leg = None
    for i in range(args.warmup + args.steps):
        leg = cpu_reference_leg(model, lengths, target_s=args.ref_seconds, seed=100 + i, enc=enc)
        if i >= args.warmup:
            vals.append(leg["value"])
    v = float(np.mean(vals))
    leg["value"] = v
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "config 4 bulk embedding (131,072 docs, lengths lognormal(5.0,0.7) clip [16,512]); "
                               "reference CPU arm: bounded document sample per step",
                   "model": "XTR-base Q4_K random-init", "parallelism": "cpu threads"},
        "cpu_baseline": leg,
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _gpu_indices(world: int):
    """Physical indices of the job's GPUs (local ranks 0..world-1) for nvidia-smi."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        return ids[:world]
    return list(range(world))


def run_ours(args):
    import torch
    world, rank, local = _dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from witchcraft_b200._lib import check, lib
    from witchcraft_b200.synth import make_synthetic_model
    from witchcraft_b200.t5cuda import T5EncoderModel

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t)
        return float(t.item())

    def sampler():
        # one nvidia-smi process for the whole job (local rank 0), not one per rank
        if os.environ.get("WC_BENCH_NO_CLOCKS") == "1":
            return None
        return ClockSampler(_gpu_indices(world)).start() if local == 0 else None

    model = make_synthetic_model(seed=0)
    enc = T5EncoderModel(model.gguf, model.config.to_json(), device=local)
    n_layers = model.config.num_layers
    per_step = args.batches_per_step
    lengths, mine = _plan(world, rank, per_step, args.warmup + args.steps)
    rng = np.random.default_rng(1000 + rank)
    host_inputs = [_make_inputs(lengths, b, rng) for b in mine]
    # Device-resident leg: one wc_t5_forward_many_device call per step, which
    # puts alternate batches on the handle's two compute lanes (one batch's
    # memory-bound kernels share the SMs with the other's GEMMs).
    stream = torch.cuda.Stream()
    max_rows = max(b.padded_tokens for b in mine)
    d_outs = [(torch.empty(max_rows, 128, device="cuda"), torch.empty(max_rows, device="cuda"))
              for _ in range(per_step)]
    dev = [(torch.from_numpy(ids).cuda(), torch.from_numpy(lens).cuda()) for ids, lens in host_inputs]
    torch.cuda.synchronize()

    def step(s: int):
        batch = []
        for j in range(per_step):
            ids, lens = dev[s * per_step + j]
            o, nr = d_outs[j]
            batch.append((ids.data_ptr(), lens.data_ptr(), ids.shape[0], ids.shape[1], o.data_ptr(), nr.data_ptr()))
        enc.forward_many_device(batch, stream.cuda_stream)

    # ---- device-resident timed region
    for s in range(args.warmup):
        step(s)
    # workspaces sized for the run's largest batch before the timed region
    big = max(range(len(mine)), key=lambda i: mine[i].padded_tokens)
    bi, bl = dev[big]
    enc.forward_many_device([(bi.data_ptr(), bl.data_ptr(), bi.shape[0], bi.shape[1], d_outs[k][0].data_ptr(),
                              d_outs[k][1].data_ptr()) for k in range(min(2, per_step))], stream.cuda_stream)
    enc.sync(stream.cuda_stream)
    torch.cuda.synchronize()
    clocks = sampler()
    barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.mark(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.warmup, args.warmup + args.steps):
        step(s)
    e1.record(stream)
    enc.sync(stream.cuda_stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark(False)
    barrier()
    clk = clocks.stop() if clocks else None
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms)
    timed = range(args.warmup * per_step, (args.warmup + args.steps) * per_step)
    valid_tokens = float(sum(int(host_inputs[i][1].sum()) for i in timed))
    padded_tokens = float(sum(mine[i].padded_tokens for i in timed))
    all_valid = sum_over_ranks(valid_tokens)
    value = all_valid / (ms_max / 1e3)
    launches = len(timed) * (2 + LAUNCHES_PER_FORWARD_PER_LAYER * n_layers)

    # ---- end to end through the public C ABI (pinned host buffers)
    pinned = []
    for ids, lens in host_inputs:
        B, L = ids.shape
        pi = torch.from_numpy(ids).pin_memory()
        pl = torch.from_numpy(lens).pin_memory()
        po = torch.empty(B, L, 128).pin_memory()
        pn = torch.empty(B, L).pin_memory()
        pinned.append((pi, pl, po, pn))
    l = lib()

    def e2e_step(idx):
        """One step's batches through the public pipelined call wc_t5_forward_many
        (pinned host buffers: uploads and downloads overlap the forwards)."""
        n = len(idx)
        vp = ctypes.c_void_p
        arr = lambda k: (vp * n)(*[vp(pinned[i][k].data_ptr()) for i in idx])  # noqa: E731
        Bs = (ctypes.c_int * n)(*[pinned[i][0].shape[0] for i in idx])
        Ls = (ctypes.c_int * n)(*[pinned[i][0].shape[1] for i in idx])
        check(l.wc_t5_forward_many(enc.handle, n, arr(0), arr(1), Bs, Ls, arr(2), arr(3)), enc.handle)

    warm = list(range(args.warmup * per_step))
    for s0 in range(0, len(warm), per_step):
        e2e_step(warm[s0:s0 + per_step])
    # size the handle's I/O buffers for the largest batch of the run now, not
    # inside the timed region (a larger batch reallocates them: cudaFree +
    # cudaMalloc, up to ~0.1 s)
    biggest = max(range(len(mine)), key=lambda i: mine[i].padded_tokens)
    e2e_step([biggest, biggest])
    clocks = sampler()
    barrier()
    if clocks:
        clocks.mark(True)
    t0 = time.perf_counter()
    t_steps = []
    for s0 in range(0, len(timed), per_step):
        e2e_step(timed[s0:s0 + per_step])
        t_steps.append(time.perf_counter())
    t_local = time.perf_counter() - t0
    if clocks:
        clocks.mark(False)
    barrier()
    clk_e2e = clocks.stop() if clocks else None
    t_e2e = max_over_ranks(t_local)
    t_e2e_min = -max_over_ranks(-t_local)
    if os.environ.get("WC_BENCH_DEBUG") == "1":
        dts = np.diff(np.array([t0] + t_steps)) * 1e3
        print(f"rank {rank}: e2e {t_local:.3f} s, value {ms:.1f} ms, e2e steps ms {np.round(dts, 1).tolist()}",
              file=sys.stderr, flush=True)
    h2d = sum(pinned[i][0].numel() * 4 + pinned[i][1].numel() * 4 for i in timed) / args.steps
    d2h = sum(pinned[i][2].numel() * 4 + pinned[i][3].numel() * 4 for i in timed) / args.steps
    e2e_value = all_valid / t_e2e
    del pinned

    fused = None
    if rank == 0 and not args.no_extras:
        fused = fused_weights_leg(model, dev, host_inputs, d_outs, per_step, args, lengths)

    corpus = None
    if args.corpus:
        corpus = corpus_measurement(model, enc, world, rank, local, barrier, max_over_ranks)

    result = None
    if rank == 0:
        peak, peak_sus, hbm, peak_src = _peaks()
        roof = None
        extras = {}
        if not args.no_extras:
            roof, extras = kernel_measurements(enc, args, peak, peak_src, cpu=world == 1 and not args.no_cpu,
                                               model=model)
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "config 4 bulk embedding: 131,072 docs, lengths lognormal(5.0,0.7) clip [16,512], "
                                   f"length-bucketed batches <= {MAX_BATCH_TOKENS} padded tokens, "
                                   f"{per_step} batches per rank per step",
                       "model": "XTR-base (12 x 768, d_ff 2048, 12 heads) random-init N(0,0.02) -> Q4_K",
                       "padded_tokens_per_rank_step": padded_tokens / args.steps,
                       "valid_tokens_per_rank_step": valid_tokens / args.steps,
                       "parallelism": f"replicas x{world} (no data-path collective)",
                       "value_api": "wc_t5_forward_many_device, one call per step (two compute lanes)",
                       "l2": "per-batch working set (activations of up to 16,384 tokens, ~250 MB) exceeds the 126 MB L2"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "api": "wc_t5_forward_many (page-locked host buffers, one call per step, copies overlap the forwards)",
                    "clocks": clk_e2e, "rank_seconds_min_max": [t_e2e_min, t_e2e]},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if corpus:
            result["corpus"] = corpus
        if fused:
            result["bulk_fused_q4k"] = fused
        if roof:
            result["roofline"] = roof
        result.update(extras)
        if world == 1 and not args.no_cpu:
            result["cpu_baseline"] = cpu_reference_leg(model, lengths, target_s=args.ref_seconds)
        print(json.dumps(result), flush=True)
    enc.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def fused_weights_leg(model, dev, host_inputs, d_outs, per_step, args, lengths):
    """The device-resident bulk leg on a handle created with WC_F16_WEIGHTS=0:
    the large-M GEMMs dequantise the Q4_K super-blocks in the kernel (TMA-
    staged raw blocks, dequant warps, tcgen05) instead of reading the resident
    f16 copies.  Same batches, same timing method, this rank's GPU only."""
    import torch
    from witchcraft_b200.t5cuda import T5EncoderModel
    os.environ["WC_F16_WEIGHTS"] = "0"
    try:
        enc = T5EncoderModel(model.gguf, model.config.to_json(), device=torch.cuda.current_device())
    finally:
        del os.environ["WC_F16_WEIGHTS"]
    stream = torch.cuda.Stream()

    def step(s):
        batch = []
        for j in range(per_step):
            ids, lens = dev[s * per_step + j]
            o, nr = d_outs[j]
            batch.append((ids.data_ptr(), lens.data_ptr(), ids.shape[0], ids.shape[1], o.data_ptr(), nr.data_ptr()))
        enc.forward_many_device(batch, stream.cuda_stream)
    for s in range(args.warmup):
        step(s)
    enc.sync(stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.warmup, args.warmup + args.steps):
        step(s)
    e1.record(stream)
    enc.sync(stream.cuda_stream)
    ms = e0.elapsed_time(e1)
    enc.close()
    timed = range(args.warmup * per_step, (args.warmup + args.steps) * per_step)
    valid = float(sum(int(host_inputs[i][1].sum()) for i in timed))
    return {"what": "device-resident bulk leg, Q4_K dequantised inside the large-M GEMMs (WC_F16_WEIGHTS=0)",
            "tokens_per_s": valid / (ms / 1e3), "ms_per_step": ms / args.steps}


def corpus_measurement(model, enc, world, rank, local, barrier, max_over_ranks):
    """The whole config-4 corpus (131,072 documents, about 23.8 M valid tokens)
    encoded once across the job's GPUs: batches dealt to ranks by LPT on
    padded tokens (shard.assign_batches), each rank running its share through
    the product's bulk pool (witchcraft_b200.pool: page-locked output ring,
    wc_t5_forward_many per chunk, results handed to a sink in host memory).
    Wall-clock from a barrier to the last rank's last result (max over ranks):
    strong scaling, the total work is fixed."""
    from witchcraft_b200 import shard
    from witchcraft_b200.pool import EncoderPool
    lengths = shard.config4_lengths()
    batches = shard.plan_batches(lengths, MAX_BATCH_TOKENS)
    owners = shard.assign_batches(batches, world)[rank]
    rng = np.random.default_rng(77 + rank)
    mine = []
    for i in owners:
        b = batches[i]
        lens = lengths[b.docs].astype(np.int32)
        ids = rng.integers(3, 32128, (len(lens), b.L)).astype(np.uint32)
        ids[np.arange(b.L)[None, :] >= lens[:, None]] = 0
        mine.append((ids, lens))
    valid = float(sum(int(l.sum()) for _, l in mine))
    done = [0]

    def sink(i, raw, norms):
        done[0] += 1
    with EncoderPool(lambda d: enc, [local], chunk=8, max_batch_tokens=MAX_BATCH_TOKENS,
                     close_encoders=False) as pool:
        # warm-up of the ring and the lanes, with the largest batches so the
        # handle's buffers are sized before the timed run
        pool.run(sorted(mine, key=lambda b: -b[0].size)[:8], sink)
        barrier()
        t0 = time.perf_counter()
        pool.run(mine, sink)
        t = time.perf_counter() - t0
    barrier()
    t_max = max_over_ranks(t)
    total_valid = valid
    if world > 1:
        import torch
        v = torch.tensor([valid], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(v)
        total_valid = float(v.item())
    return {"what": "whole config-4 corpus (131,072 docs) once across all ranks, LPT-dealt batches, "
                    "witchcraft_b200.pool + wc_t5_forward_many, page-locked outputs in host memory",
            "scaling": "strong", "docs": int(len(lengths)), "batches": len(batches),
            "valid_tokens": total_valid, "wall_s": t_max, "tokens_per_s": total_valid / t_max}


def _time_launches(fn, stream, reps: int, warm: int = 3) -> float:
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warm):
            fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        # a device-side delay ahead of the timed launches lets the host queue
        # all of them first, so host launch overhead cannot open gaps between
        # short kernels inside the timed region
        torch.cuda._sleep(20_000_000)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps / 1e3  # seconds per launch


def kernel_measurements(enc, args, peak, peak_src, cpu=False, model=None):
    """Per-kernel timings for the roofline: the gated-GELU GEMM (the dominant
    kernel, 44% of encoder FLOPs) at one full batch (M = 16,384) on the
    resident f16 weights the forward uses from 512 rows, plus the other GEMM
    shapes (config 2, M = 8192; the fused-dequant Q4_K kernel for comparison)
    and attention (config 3), each timed with CUDA events on its launch stream."""
    import torch
    from witchcraft_b200._lib import check, lib
    from witchcraft_b200.synth import quantize_q4k
    l = lib()
    st = torch.cuda.Stream()
    sp = ctypes.c_void_p(st.cuda_stream)
    rng = np.random.default_rng(2)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def wq(n, k):
        """(Q4_K bytes, the same weights dequantised to f16 [n][k])"""
        q = torch.from_numpy(quantize_q4k(rng.standard_normal((n, k)).astype(np.float32) * 0.02).reshape(-1)).cuda()
        h = torch.empty(n, k, device="cuda", dtype=torch.float16)
        check(l.wc_q4k_dequant_f16(P(q), q.numel() // 144, P(h), sp))
        return q, h

    w0, w1 = wq(2048, 768), wq(2048, 768)
    wqkv, wo, wattn = wq(2304, 768), wq(768, 2048), wq(768, 768)

    def gemm_case(M, K, N, epi, w, wu, fused_q4k=False):
        x = torch.randn(M, K, device="cuda").half()
        y = torch.empty(M, N, device="cuda", dtype=torch.float16 if epi in (0, 1) else torch.float32)
        k = 0 if fused_q4k else 1
        fn = l.wc_gemm_q4k if fused_q4k else l.wc_gemm_f16
        f = lambda: check(fn(P(x), M, K, P(w[k]), P(wu[k]) if wu is not None else None, N, epi, P(y), sp))  # noqa
        t = _time_launches(f, st, reps=20)
        flops = 2.0 * M * K * N * (2 if epi == 1 else 1)
        return t, flops

    t, fl = gemm_case(16384, 768, 2048, 1, w0, w1)
    achieved = fl / t / 1e12
    roof = {"bound": "tensor",
            "kernel": "gemm2_q4k_kernel<kEpiGeGLU, f16 weights> (wi_0|wi_1 + gated GELU, 2-SM), M=16384 K=768 N=2x2048",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{peak_src} dense bf16/f16 burst", "traffic": NCU_TRAFFIC_BYTES,
            "avg_launch_us": t * 1e6, "algorithmic_flop_per_launch": fl}
    micro = {}
    for name, (M, K, N, epi, w, wu, fq) in {"qkv_M8192": (8192, 768, 2304, 0, wqkv, None, False),
                                            "wi_geglu_M8192": (8192, 768, 2048, 1, w0, w1, False),
                                            "wo_M8192": (8192, 2048, 768, 3, wo, None, False),
                                            "o_M8192": (8192, 768, 768, 3, wattn, None, False),
                                            "wi_geglu_M8192_fused_q4k": (8192, 768, 2048, 1, w0, w1, True)}.items():
        t, fl = gemm_case(M, K, N, epi, w, wu, fq)
        micro[name] = {"us": t * 1e6, "tflops": fl / t / 1e12, "frac_of_peak": fl / t / 1e12 / peak}
    # attention, config 3
    B, L, H = 64, 512, 12
    lens = np.random.default_rng(4).integers(32, 513, B).astype(np.int32)
    qkv = torch.randn(B * L, 3 * H * 64, device="cuda").half()
    ao = torch.empty(B * L, H * 64, device="cuda").half()
    dl = torch.from_numpy(lens).cuda()
    bt = torch.randn(32, H, device="cuda") * 0.1
    f = lambda: check(l.wc_attention(P(qkv), B, L, H, P(dl), P(bt), 32, 128, P(ao), sp))  # noqa: E731
    t = _time_launches(f, st, reps=20)
    afl = float(sum(12 * 4 * 64 * int(n) ** 2 for n in lens))
    micro["attention_config3"] = {"us": t * 1e6, "tflops": afl / t / 1e12, "frac_of_peak": afl / t / 1e12 / peak}
    c1 = config1_measurement(enc, peak)
    extras = {"microbench": micro, "config1": c1, "query_latency": query_latency(enc), "codec": codec_measurement(),
              "index_assign": assign_measurement(), "query_scoring": query_scoring_measurement()}
    if cpu and model is not None:
        extras["cpu_configs"] = cpu_config_baselines(model, lens)
    return roof, extras


CONFIG1_FLOP_PER_TOKEN = 2.0 * (12 * 7077888 + 98304) + 12 * 3072 * 128  # 174.78 MFLOP


def config1_measurement(enc, peak, reps: int = 50):
    """Config 1: the full encoder on one B = 16 x L = 128 batch (no padding),
    device-resident, CUDA events around `reps` forwards on one stream."""
    import torch
    rng = np.random.default_rng(1)
    ids = torch.from_numpy(rng.integers(3, 32128, (16, 128)).astype(np.uint32)).cuda()
    lens = torch.full((16,), 128, dtype=torch.int32, device="cuda")
    out = torch.empty(16 * 128, 128, device="cuda")
    st = torch.cuda.Stream()
    f = lambda: enc.forward_device(ids.data_ptr(), lens.data_ptr(), 16, 128, out.data_ptr(), None, None,  # noqa
                                   st.cuda_stream)
    t = _time_launches(f, st, reps=reps)
    enc.sync(st.cuda_stream)
    tok = 16 * 128 / t
    return {"what": "full encoder, B=16 x L=128, device-resident", "tokens_per_s": tok, "ms_per_batch": t * 1e3,
            "tflops": tok * CONFIG1_FLOP_PER_TOKEN / 1e12, "frac_of_peak": tok * CONFIG1_FLOP_PER_TOKEN / 1e12 / peak}


def cpu_config_baselines(model, attn_lens, budget_s: float = 8.0):
    """The reference's f32 CPU algorithm (oracle/torch_ref.py, torch MKL on
    every host core) beside configs 1, 2, 3 and 5: the config-1 batch encoded
    one sequence at a time, the config-2 GEMMs in f32 (gated GELU included),
    config-3 attention per sequence at its valid length (softmax(QK^T + bias) V
    without scaling), and 32-token query latency p50/p99 at batch 1 and 256
    (queries encoded one by one, as the reference's Embedder does)."""
    import torch
    from oracle.torch_ref import TorchCPUEncoder
    cores = os.cpu_count() or 1
    enc = TorchCPUEncoder(model, threads=cores)
    res = {"cores": cores, "kind": "port", "impl": "oracle/torch_ref.py (torch CPU f32, MKL GEMMs)"}
    rng = np.random.default_rng(1)
    ids = rng.integers(3, 32128, (16, 128))
    enc.encode_one(ids[0])
    t0 = time.perf_counter()
    for r in ids:
        enc.encode_one(r)
    res["config1_tokens_per_s"] = 16 * 128 / (time.perf_counter() - t0)
    g = {}
    with torch.no_grad():
        for name, (M, K, N, gated) in {"qkv_M8192": (8192, 768, 2304, False), "wi_geglu_M8192": (8192, 768, 2048, True),
                                       "wo_M8192": (8192, 2048, 768, False), "o_M8192": (8192, 768, 768, False)}.items():
            x = torch.randn(M, K)
            w0 = torch.randn(N, K) * 0.02
            w1 = torch.randn(N, K) * 0.02

            def f():
                a = x @ w0.T
                if gated:
                    a = 0.5 * a * (1 + torch.tanh(0.7978845608 * (a + 0.044715 * a ** 3))) * (x @ w1.T)
                return a
            f()
            t0 = time.perf_counter()
            n = 0
            while n < 3 or (time.perf_counter() - t0 < 0.5 and n < 20):
                f()
                n += 1
            t = (time.perf_counter() - t0) / n
            g[name] = {"ms": t * 1e3, "tflops": 2.0 * M * K * N * (2 if gated else 1) / t / 1e12}
        res["config2_gemm"] = g
        H = 12
        afl = float(sum(12 * 4 * 64 * int(n) ** 2 for n in attn_lens))
        t0 = time.perf_counter()
        for L in attn_lens:
            L = int(L)
            q, k, v = (torch.randn(H, L, 64) for _ in range(3))
            bias = enc._bias(L)
            torch.softmax(q @ k.transpose(-1, -2) + bias, -1) @ v
        t = time.perf_counter() - t0
        res["config3_attention"] = {"ms": t * 1e3, "tflops": afl / t / 1e12}
    qrng = np.random.default_rng(6)
    q = {}
    for B, runs in ((1, 100), (256, 3)):
        times = []
        t_start = time.perf_counter()
        for r in range(runs):
            lens = qrng.integers(4, 33, B)
            toks = [qrng.integers(3, 32128, int(n)) for n in lens]
            t0 = time.perf_counter()
            for tk in toks:
                enc.encode_one(tk)
            times.append((time.perf_counter() - t0) * 1e3)
            if time.perf_counter() - t_start > budget_s:
                break
        q[f"b{B}"] = {"p50_ms": float(np.percentile(times, 50)), "p95_ms": float(np.percentile(times, 95)),
                      "p99_ms": float(np.percentile(times, 99)),
                      "runs": len(times)}
    res["config5_query_latency"] = q
    return res


def query_scoring_measurement(rows: int = 200000, m: int = 32, per_sub: int = 8):
    """match_centroids' candidate scoring (src/lib.rs:715-808) for one query of
    m tokens over `rows` indexed candidates (4-bit residual codes, 1024
    clusters, sub-chunks of per_sub rows, 4 sub-chunks per document): the GPU
    scorer through its host entry (copies in and out included) and the C
    oracle on one host core."""
    import torch
    from oracle import oracle as O
    from witchcraft_b200 import query as Qm
    rng = np.random.default_rng(11)
    q = rng.standard_normal((m, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    n_cent = 1024
    cs = (rng.standard_normal((m, n_cent)) * 0.2).astype(np.float32)
    codes = rng.integers(0, 256, (rows, 64), dtype=np.uint8)
    cluster = rng.integers(0, n_cent, rows).astype(np.uint32)
    n_groups = rows // per_sub
    c = Qm.Candidates(q=q, codes=codes, cluster=cluster, cscores=cs, raw=np.zeros((0, 128), np.float32),
                      group_rows=np.arange(rows, dtype=np.int64),
                      group_start=np.arange(0, rows + 1, per_sub, dtype=np.int64),
                      doc_start=np.arange(0, n_groups + 1, 4, dtype=np.int64),
                      group_keys=[(g // 4, g % 4) for g in range(n_groups)], missing=np.zeros(m, np.float32))
    table = Qm.q4_table()
    Qm.score_gpu(c, table)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        Qm.score_gpu(c, table)
    tg = (time.perf_counter() - t0) / 5
    # the scoring kernel alone on device-resident inputs (CUDA events)
    from witchcraft_b200._lib import lib
    dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dt)).cuda()  # noqa: E731
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    dq, dcodes, dcl = dev(q, np.float32), dev(codes.reshape(-1), np.uint8), dev(cluster.view(np.int32), np.int32)
    dcs, dtab = dev(cs, np.float32), dev(table, np.float32)
    dgr, dgs, dds = (dev(a, np.int64) for a in (c.group_rows, c.group_start, c.doc_start))
    dmiss = dev(c.missing, np.float32)
    out = torch.empty(n_groups, dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    f = lambda: lib().wc_score_candidates(P(dq), m, 128, P(dcodes), P(dcl), P(dcs), n_cent, P(dtab), rows, None,  # noqa
                                          P(dgr), P(dgs), P(dds), len(c.doc_start) - 1, P(dmiss), P(out),
                                          ctypes.c_void_p(st.cuda_stream))
    tk = _time_launches(f, st, reps=20)
    # bytes the kernel must read once: codes, cluster ids, row/group/doc
    # offsets, centroid scores, query, plus the scores it writes
    kbytes = (codes.nbytes + rows * 4 + rows * 8 + (n_groups + 1) * 8 + (len(c.doc_start)) * 8 + cs.nbytes + q.nbytes
              + n_groups * 4)
    _, _, hbm, _ = _peaks()
    t0 = time.perf_counter()
    O.score_candidates(q, codes, cluster, cs, table, c.raw, c.group_rows, c.group_start, c.doc_start, c.missing)
    tc = time.perf_counter() - t0
    # 2 m 128 FLOP per row: about 100 FLOP per byte read, so the FP32 FMA
    # rate, not HBM, bounds the kernel
    kflops = 2.0 * rows * m * 128
    fpk = _fp32_fma_peak_tflops()
    return {"what": "candidate scoring of one query (m tokens x rows, 4-bit residuals)", "m": m, "rows": rows,
            "gpu_ms_with_copies": tg * 1e3, "gpu_kernel_us": tk * 1e6, "kernel_bytes": kbytes,
            "kernel_gbs": kbytes / tk / 1e9, "frac_of_hbm": kbytes / tk / 1e9 / hbm, "bound": "fp32 fma",
            "kernel_tflops_fp32": kflops / tk / 1e12, "frac_of_fp32_peak": kflops / tk / 1e12 / fpk,
            "cpu_oracle_ms_1core": tc * 1e3}


def _fp32_fma_peak_tflops() -> float:
    """FP32 FMA peak: SMs x 128 lanes x 2 FLOP x the maximum SM clock."""
    import torch
    pr = torch.cuda.get_device_properties(0)
    sm_mhz = pr.clock_rate / 1e3 if hasattr(pr, "clock_rate") else 1965.0
    return pr.multi_processor_count * 128 * 2 * sm_mhz * 1e6 / 1e12


def assign_measurement(m: int = 262144, cpu_rows: int = 256):
    """matmul_argmax_batched (src/lib.rs:187-208) with the reference's center
    count k = round(16 sqrt(m)): the GPU kernel (FP32 FMA chains on the CUDA
    cores) timed with CUDA events, against the FP32 FMA peak
    (148 SMs x 128 lanes x 2 FLOP x the SM clock), and the C oracle on
    cpu_rows rows with all host threads."""
    import torch
    from oracle import oracle as O
    from witchcraft_b200 import index as I
    k = int(round(16 * m ** 0.5))
    rng = np.random.default_rng(9)
    x = rng.standard_normal((m, 128)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    c = x[rng.choice(m, k, replace=False)]
    dx, dc = torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda()
    I.assign(dx, dc)
    torch.cuda.synchronize()
    times = []
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        I.assign(dx, dc)
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
    t = min(times)
    flops = 2.0 * m * k * 128
    peak = _fp32_fma_peak_tflops()
    t0 = time.perf_counter()
    O.assign_centers(x[:cpu_rows], c)
    tc = time.perf_counter() - t0
    return {"what": "nearest-center assignment, k = round(16 sqrt(m))", "m": m, "k": k, "gpu_ms": t * 1e3,
            "gpu_tflops_fp32": flops / t / 1e12, "fp32_fma_peak_tflops": peak, "frac_of_fp32_peak": flops / t / 1e12 / peak,
            "gpu_rows_per_s": m / t, "cpu_oracle_rows_per_s": cpu_rows / tc, "cpu_threads": O.lib().oracle_num_threads()}


def codec_measurement(n_docs: int = 2048, cpu_docs: int = 256):
    """embeddings_to_packed (src/packops.rs:172-301) of config-4-length
    documents (L2-normalised synthetic rows): the GPU codec on n_docs, timed
    with CUDA events around the device entry point (inputs resident), and the
    C oracle on the first cpu_docs of them on one host core."""
    import torch
    from oracle import oracle as O
    from witchcraft_b200._lib import check, lib
    from witchcraft_b200.shard import config4_lengths
    l = lib()
    lens = config4_lengths(n_docs, seed=7)
    rng = np.random.default_rng(8)
    emb = rng.standard_normal((int(lens.sum()), 128)).astype(np.float32)
    emb /= np.linalg.norm(emb, axis=1, keepdims=True)
    rows = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    d_emb = torch.from_numpy(emb).cuda()
    cap = l.wc_packed_bound(rows.ctypes.data, n_docs, 128)
    d_out = torch.empty(cap, dtype=torch.uint8, device="cuda")
    offs = np.empty(n_docs + 1, np.int64)
    st = torch.cuda.Stream()
    sp = ctypes.c_void_p(st.cuda_stream)

    def run():
        rc = l.wc_pack_embeddings_device(ctypes.c_void_p(d_emb.data_ptr()), rows.ctypes.data, n_docs, 128,
                                         ctypes.c_void_p(d_out.data_ptr()), cap, offs.ctypes.data, sp)
        if rc != 0:
            raise RuntimeError(l.wc_codec_last_error())
    run()
    times = []
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        run()
        b.record(st)
        b.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
    t = min(times)
    n_cpu = int(rows[cpu_docs])
    t0 = time.perf_counter()
    for i in range(cpu_docs):
        O.pack_embeddings(emb[rows[i]:rows[i + 1]])
    tc = time.perf_counter() - t0
    return {"what": "embeddings_to_packed, config-4 document lengths", "docs": n_docs, "rows": int(rows[-1]),
            "gpu_rows_per_s": rows[-1] / t, "gpu_ms": t * 1e3, "bytes_per_row": offs[-1] / rows[-1],
            "cpu_oracle_rows_per_s_1core": n_cpu / tc, "cpu_sample_docs": cpu_docs}


def query_latency(enc, runs: int = 200):
    """Config 5: 32-token padded queries (lengths U[4, 32]) at batch 1 and 256,
    device-resident, one forward per timed call (CUDA events)."""
    import torch
    res = {}
    st = torch.cuda.Stream()
    for B in (1, 256):
        rng = np.random.default_rng(6)
        ids = torch.from_numpy(rng.integers(3, 32128, (B, 32)).astype(np.uint32)).cuda()
        lens = torch.from_numpy(rng.integers(4, 33, B).astype(np.int32)).cuda()
        out = torch.empty(B * 32, 128, device="cuda")
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
        for _ in range(10):
            enc.forward_device(ids.data_ptr(), lens.data_ptr(), B, 32, out.data_ptr(), None, None, st.cuda_stream)
        for a, b in ev:
            a.record(st)
            enc.forward_device(ids.data_ptr(), lens.data_ptr(), B, 32, out.data_ptr(), None, None, st.cuda_stream)
            b.record(st)
        enc.sync(st.cuda_stream)
        torch.cuda.synchronize()
        t = np.array([a.elapsed_time(b) for a, b in ev])
        # p95 is the reference's own query-latency figure (the embedder's p95)
        res[f"b{B}"] = {"p50_ms": float(np.percentile(t, 50)), "p95_ms": float(np.percentile(t, 95)),
                        "p99_ms": float(np.percentile(t, 99))}
    return res


def profile_kernel(name: str, m: int, launches: int = 5, fused_q4k: bool = False):
    """A few launches of one kernel (for an ncu capture of that kernel alone):
    the GEMMs on f16 weights as the forward runs them, or with fused_q4k the
    Q4_K-dequantising variant."""
    import torch
    from witchcraft_b200._lib import check, lib
    from witchcraft_b200.synth import quantize_q4k
    l = lib()
    rng = np.random.default_rng(2)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def wq(n, k):
        q = torch.from_numpy(quantize_q4k(rng.standard_normal((n, k)).astype(np.float32) * 0.02).reshape(-1)).cuda()
        if fused_q4k:
            return q
        h = torch.empty(n, k, device="cuda", dtype=torch.float16)
        check(l.wc_q4k_dequant_f16(P(q), q.numel() // 144, P(h), None))
        return h
    if name == "attention":
        B, L, H = 64, 512, 12
        lens = torch.from_numpy(np.random.default_rng(4).integers(32, 513, B).astype(np.int32)).cuda()
        qkv = torch.randn(B * L, 3 * H * 64, device="cuda").half()
        out = torch.empty(B * L, H * 64, device="cuda").half()
        bt = torch.randn(32, H, device="cuda") * 0.1
        f = lambda: check(l.wc_attention(P(qkv), B, L, H, P(lens), P(bt), 32, 128, P(out), None))  # noqa: E731
    else:
        K, N, epi = {"geglu": (768, 2048, 1), "qkv": (768, 2304, 0), "wo": (2048, 768, 3), "o": (768, 768, 3)}[name]
        w, wu = wq(N, K), (wq(N, K) if epi == 1 else None)
        x = torch.randn(m, K, device="cuda").half()
        y = torch.zeros(m, N, device="cuda", dtype=torch.float16 if epi in (0, 1) else torch.float32)
        fn = l.wc_gemm_q4k if fused_q4k else l.wc_gemm_f16
        f = lambda: check(fn(P(x), m, K, P(w), P(wu) if wu is not None else None, N, epi, P(y), None))  # noqa: E731
    for _ in range(launches):
        f()
    torch.cuda.synchronize()
    print(json.dumps({"profiled": name, "m": m, "launches": launches}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batches-per-step", type=int, default=8)
    ap.add_argument("--ref-seconds", type=float, default=8.0)
    ap.add_argument("--no-extras", action="store_true", help="skip per-kernel timings and query latency")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-corpus", dest="corpus", action="store_false",
                    help="skip the whole-corpus (strong scaling) encode")
    ap.add_argument("--lanes", type=int, choices=[1, 2], default=2,
                    help="device-resident leg: encoder handles on their own streams taking alternate batches")
    ap.add_argument("--profile-kernel", choices=["geglu", "qkv", "wo", "o", "attention"], default=None,
                    help="only launch one kernel a few times (for ncu)")
    ap.add_argument("--m", type=int, default=16384, help="GEMM rows for --profile-kernel")
    ap.add_argument("--fused-q4k", action="store_true", help="--profile-kernel: the Q4_K-dequantising GEMM")
    args = ap.parse_args()
    if args.profile_kernel:
        profile_kernel(args.profile_kernel, args.m, fused_q4k=args.fused_q4k)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
