"""Benchmark: batch-1 greedy decode of a TT-compressed TinyLlama-1.1B-architecture chip.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): processor_infer on the random-init TinyLlama-1.1B
architecture chip (22 layers, d_model 2048, 32 q / 4 KV heads, head_dim 64,
SwiGLU 5632, vocab 32000; every matrix N(0,0.02) bf16-rounded, TT-compressed)
with a 32-token uniform-random prompt in [3, 32000) and 128 greedy tokens,
EOS disabled: 160 tape steps.  metric = tokens processed per second (prompt +
generated, as the reference's own timing counts them).  The index stream is
2,068,840,448 B per token, far above the 126 MB L2, so every step reads its
weights from HBM.

Printed JSON line (rank 0):
  value      device time (CUDA events on the executor's stream) of the K calls
  e2e        the same calls timed on the host around the C-ABI call, prompt in
             and tokens out through host buffers
  roofline   the dominant kernel, the TT-GEMV, timed live on the config-1
             shapes (K x N in {2048x2048, 2048x5632, 5632x2048, 2048x32000},
             seeded codebooks, Gaussian-rank indices) over rotating copies
             larger than L2; bytes = K*N*2 per launch
  cpu_baseline  the compiled reference runtime (oracle/_ref) on this host,
             a bounded sample of the same chip (rank 0, N=1)
For N > 1 every rank decodes its own replica (no data-path collective):
value = all ranks' tokens / max-over-ranks time, "scaling": "weak".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from kmap_b200 import chipgen  # noqa: E402

PROMPT, GEN = 32, 128
INDEX_BYTES_PER_TOKEN = 2068840448
# dram__bytes_read.sum + dram__bytes_write.sum of one k_decode_step launch:
# 311.3 MB measured on the 2-layer TinyLlama-width chip (307.2 MB of index
# stream, ratio 1.0132), scaled to the 22-layer index stream
STEP_TRAFFIC_BYTES = 2096203116
CHIP_CACHE = os.environ.get("KLLM_CHIP_CACHE", "/tmp/kllm_chips")
TT_SHAPES = [(2048, 2048, 4096), (2048, 5632, 5461), (5632, 2048, 5461), (2048, 32000, 5461)]


def log(*a):
    print("[bench]", *a, file=sys.stderr, flush=True)


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def config0_chip(rank=0, layers=None):
    spec = chipgen.ModelSpec(**{**chipgen.TINYLLAMA_1B.__dict__})
    spec.max_seq = 2048
    if layers:
        spec.num_layers = layers
    lock = os.path.join(CHIP_CACHE, ".lock")
    os.makedirs(CHIP_CACHE, exist_ok=True)
    import fcntl
    with open(lock, "w") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        t = time.time()
        path = chipgen.ensure_chip(CHIP_CACHE, spec)
        log("chip ready in %.1fs: %s" % (time.time() - t, path))
    return path


def prompt_ids(seed=0):
    return np.random.default_rng(seed).integers(3, 32000, PROMPT).astype(np.int32)


class Clocks:
    """nvidia-smi samples (200 ms) during the timed region."""

    def __init__(self, index):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ------------------------------------------------------------ roofline ---

def ttgemv_roofline(device_index):
    """Average launch time of the TT-GEMV on the config-1 shapes, timed with
    CUDA events on the launching stream; copies rotate so that every launch
    reads its indices from HBM."""
    import torch

    import kmap_b200
    lib = kmap_b200.lib()
    dev = torch.device("cuda", device_index)
    stream = torch.cuda.current_stream(dev)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    res = []
    for K, N, C in TT_SHAPES:
        x, cb, idx = chipgen.tt_case(7, K, N, C)
        copies = max(2, int(np.ceil(3 * l2 / (K * N * 2))) + 1)
        d_idx = [torch.from_numpy(idx.view(np.int16)).to(dev) for _ in range(copies)]
        d_cb = torch.from_numpy(np.pad(cb, (0, (-len(cb)) % 4))).to(dev)
        d_x = torch.from_numpy(x).to(dev)
        d_y = torch.empty(N, dtype=torch.float32, device=dev)

        def run(i):
            rc = lib.kllm_tt_gemv(d_x.data_ptr(), 1, d_cb.data_ptr(), C, d_idx[i % copies].data_ptr(),
                                  K, N, d_y.data_ptr(), stream.cuda_stream)
            assert rc == 0, kmap_b200.last_error()

        for i in range(copies):
            run(i)
        torch.cuda.synchronize(dev)
        reps = max(3 * copies, 60)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            run(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        res.append({"K": K, "N": N, "codes": C, "us": ms * 1e3,
                    "gbs": K * N * 2 / (ms * 1e-3) / 1e9})
        del d_idx
    return res


def ttgemv_once(K, N, C, reps):
    """kllm_tt_gemv on one seeded config-1 shape, `reps` launches (for ncu)."""
    import torch

    import kmap_b200
    lib = kmap_b200.lib()
    x, cb, idx = chipgen.tt_case(7, K, N, C)
    dev = torch.device("cuda", 0)
    di = torch.from_numpy(idx.view(np.int16)).to(dev)
    dc = torch.from_numpy(np.pad(cb, (0, (-len(cb)) % 4))).to(dev)
    dx = torch.from_numpy(x).to(dev)
    dy = torch.empty(N, device=dev)
    for _ in range(reps):
        rc = lib.kllm_tt_gemv(dx.data_ptr(), 1, dc.data_ptr(), C, di.data_ptr(), K, N,
                              dy.data_ptr(), None)
        assert rc == 0, kmap_b200.last_error()
    torch.cuda.synchronize()
    log("ttgemv %dx%d ok" % (K, N))


def ttgemm_time(rows, K, N, C, reps):
    """kllm_tt_gemm on one seeded shape (prefill: `rows` prompt positions):
    mean device time over `reps` launches after one warm-up, as ms, FP32
    operations per second (one multiply and one add per weight and row) and
    rows per second."""
    import torch

    import kmap_b200
    lib = kmap_b200.lib()
    x, cb, idx = chipgen.tt_case(9, K, N, C, rows=rows)
    dev = torch.device("cuda", 0)
    di = torch.from_numpy(idx.view(np.int16)).to(dev)
    dc = torch.from_numpy(np.pad(cb, (0, (-len(cb)) % 4))).to(dev)
    dx = torch.from_numpy(x).to(dev)
    dy = torch.empty((rows, N), device=dev)
    s = torch.cuda.current_stream()
    out = {}
    for name in ("kllm_tt_gemm",):
        f = getattr(lib, name)
        call = lambda: f(dx.data_ptr(), rows, dc.data_ptr(), C, di.data_ptr(), K, N,
                         dy.data_ptr(), s.cuda_stream)
        assert call() == 0, kmap_b200.last_error()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            call()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        out[name] = {"ms": ms, "tops": 2.0 * rows * K * N / (ms * 1e-3) / 1e12,
                     "rows_per_s": rows / (ms * 1e-3)}
    log("tt-gemm %dx%dx%d codes %d: %s" % (rows, K, N, C, json.dumps(out)))
    return out


def prefill_run(steps, warmup):
    """Config-2 workload on the config-0 chip: a 2047-token uniform-random
    prompt (the chip's 2048 positions less the first generated token), batch
    1; prompt positions per second of device time, the batched prompt pass
    (kllm_infer_opts.prefill) beside the step-by-step one.  Prints one JSON
    line (not part of the default run)."""
    import kmap_b200
    kmap_b200.require_gpu()
    path = config0_chip(0)
    P = 2047
    prompt = np.random.default_rng(2).integers(3, 32000, P).astype(np.int32)
    res = {}
    first = {}
    for mode in ("batched", "step_by_step"):
        with kmap_b200.Chip(path, prefill=(mode == "batched")) as chip:
            ms = []
            for i in range(warmup + steps):
                toks = chip.infer(prompt, 1)
                if i >= warmup:
                    ms.append(chip.stats()["prefill_ms"])
            first[mode] = int(toks[0]) if len(toks) else -1
            res[mode] = {"ms": statistics.median(ms), "tok_s": P / (statistics.median(ms) * 1e-3)}
    print(json.dumps({"metric": "prefill tok/s (prompt positions per second, device time)",
                      "value": res["batched"]["tok_s"], "unit": "tok/s", "n_gpus": 1,
                      "steps": steps, "warmup": warmup, "higher_is_better": True,
                      "data": "synthetic", "dtype": "f32",
                      "config": {"workload": "TinyLlama-1.1B-arch TT chip, 2047-token prompt, "
                                             "batch 1, KV cache filled", "prompt": P},
                      "batched": res["batched"], "step_by_step": res["step_by_step"],
                      "first_token_equal": first["batched"] == first["step_by_step"]}))


# ---------------------------------------------------------------- arms ---

def reference_sample(chip, n_prompt=4, n_gen=4, threads=None):
    """Time the compiled reference runtime on a bounded sample of the chip."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    if not harness.have_ref():
        return None
    ref = harness.Ref()
    h, info = ref.chip(chip)
    p = prompt_ids()[:n_prompt]
    t = time.perf_counter()
    toks = ref.infer(h, p, n_gen)
    dt = time.perf_counter() - t
    ref.L.refh_chip_destroy(h)
    return {"value": (n_prompt + len(toks)) / dt, "seconds": dt, "tokens": n_prompt + len(toks)}


def decode_small(layers, steps, warmup):
    """Decode PROMPT + 16 tokens on a reduced-depth TinyLlama-width chip."""
    import kmap_b200
    kmap_b200.require_gpu()
    chip = kmap_b200.Chip(config0_chip(0, layers))
    p = prompt_ids()
    for _ in range(max(warmup, 1)):
        chip.infer(p, 16)
    ms, n = 0.0, 0
    for _ in range(steps):
        toks = chip.infer(p, 16)
        st = chip.stats()
        ms += st["prefill_ms"] + st["decode_ms"]
        n += PROMPT + len(toks)
    log("%d layers: %.1f us per tape step (fused=%d)" % (layers, 1e3 * ms / n, chip.stats()["fused"]))
    chip.close()


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    if not harness.have_ref():
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference runtime was not compiled into oracle/_ref"}))
        return
    chip = config0_chip()
    ref = harness.Ref()
    h, info = ref.chip(chip)
    p = prompt_ids()
    n_prompt, n_gen = 4, 4   # bounded sample per step: 8 tape steps
    for _ in range(args.warmup):
        ref.infer(h, p[:n_prompt], n_gen)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        toks = ref.infer(h, p[:n_prompt], n_gen)
        times.append(time.perf_counter() - t)
    ref.L.refh_chip_destroy(h)
    tok = (n_prompt + len(toks)) * args.steps
    v = tok / sum(times)
    cores = int(os.environ.get("OPENBLAS_NUM_THREADS", "8"))
    out = {"metric": "decode tok/s (prompt + generated tape steps per second)", "value": v,
           "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": 1e3 * sum(times) / args.steps, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "impl": "reference",
           "config": {"workload": "TinyLlama-1.1B-arch TT chip, batch-1 greedy decode; "
                      "bounded sample per step: 4 prompt + 4 generated tokens",
                      "prompt": n_prompt, "generate": n_gen},
           "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                            "sample": "4 prompt + 4 generated tape steps per step"},
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_ours(args, rank, world, local_rank):
    import kmap_b200
    kmap_b200.require_gpu()
    import torch
    torch.cuda.set_device(local_rank)
    kmap_b200.lib().kllm_set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    chip_path = config0_chip(rank)
    order = kmap_b200.ORDER_FAST if args.order == "fast" else kmap_b200.ORDER_EXACT
    chip = kmap_b200.Chip(chip_path, order=order)
    shard = args.shard and world > 1
    if shard:   # every rank holds 1/world of the columns; same prompt everywhere
        chip.connect(kmap_b200.exchange_blocks(chip.shard(rank, world)))
        dist.barrier()
    p = prompt_ids(seed=0 if shard else rank)
    t0 = time.time()
    chip.infer(p, GEN)      # first call prepares the plan (weights to HBM, graph)
    st = chip.stats()
    log("rank %d: first call %.1fs (fused=%d)" % (rank, time.time() - t0, st["fused"]))
    for _ in range(max(args.warmup - 1, 0)):
        chip.infer(p, GEN)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    dev_ms, host_s, launches, tokens = 0.0, 0.0, 0, 0
    with Clocks(local_rank) as clk:
        for _ in range(args.steps):
            t = time.perf_counter()
            toks = chip.infer(p, GEN)
            host_s += time.perf_counter() - t
            s = chip.stats()
            dev_ms += s["prefill_ms"] + s["decode_ms"]
            launches += s["launches"]
            tokens += PROMPT + len(toks)
    barrier()
    times = torch.tensor([dev_ms, host_s * 1e3], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    dev_ms_max, host_ms_max = times.tolist()
    if rank != 0:
        chip.close()
        if dist:
            dist.destroy_process_group()
        return
    streams = 1 if shard else world   # sharded: one stream over all GPUs
    value = tokens * streams / (dev_ms_max / 1e3)
    e2e = tokens * streams / (host_ms_max / 1e3)
    pk = peaks()
    hbm = pk.get("hbm_gbs")
    roof = ttgemv_roofline(local_rank)
    top = max(roof, key=lambda r: r["K"] * r["N"])
    # the dominant kernel is the decode step (one launch per tape step):
    # its algorithmic bytes are the index stream of every TT matrix
    step_us = dev_ms_max * 1e3 / tokens
    decode_gbs = INDEX_BYTES_PER_TOKEN / (step_us * 1e-6) / 1e9
    # sharded: the index stream is split over the GPUs, so their summed peak
    roof_peak = hbm * world if (shard and hbm) else hbm
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = reference_sample(chip_path)
    out = {
        "metric": "decode tok/s (prompt + generated tape steps per second)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps,
        "higher_is_better": True, "scaling": "strong" if shard else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "TinyLlama-1.1B-arch TT chip (22x2048, 32/4 heads, SwiGLU 5632, "
                   "vocab 32000, bf16-rounded N(0,0.02)), batch-1 greedy decode",
                   "prompt": PROMPT, "generate": GEN, "tape_steps_per_call": PROMPT + GEN,
                   "l2": "weights 2.07 GB/token >> 126 MB L2 (no flush needed)",
                   "parallelism": ("column-sharded over %d GPUs (NVLink peer stores in the "
                                   "decode kernel)" % world if shard else
                                   "replicas" if world > 1 else "single GPU")},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4,
                "d2h_bytes_per_step": GEN * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": decode_gbs, "peak": roof_peak, "unit": "GB/s",
                     "frac": decode_gbs / roof_peak if roof_peak else None,
                     "traffic": STEP_TRAFFIC_BYTES,
                     "kernel": "k_decode_step", "launch_us": step_us,
                     "algorithmic_bytes_per_launch": INDEX_BYTES_PER_TOKEN,
                     "order": args.order,
                     "peak_source": ("MEASURED_PEAKS.json hbm_gbs (burst copy)" if hbm
                                     else "fallback 6650 GB/s")},
        "ttgemv_microbench": {"kernel": "k_ttgemv_tma", "unit": "GB/s", "peak": hbm,
                              "shape": [top["K"], top["N"]], "achieved": top["gbs"],
                              "frac": top["gbs"] / hbm if hbm else None, "shapes": roof},
        "clocks": clk.summary(),
    }
    if cpu:
        out["cpu_baseline"] = {"value": cpu["value"], "unit": "tok/s", "cores": 8,
                               "kind": "reference",
                               "sample": "compiled reference runtime, same chip, 4 prompt + "
                                         "4 generated tape steps (%.1fs)" % cpu["seconds"]}
    print(json.dumps(out), flush=True)
    chip.close()
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", action="store_true",
                    help="with N > 1: one decode stream column-sharded over the N GPUs "
                         "(strong scaling) instead of N independent replicas")
    ap.add_argument("--order", default="exact", choices=["exact", "fast"],
                    help="TT-GEMV summation order of the decode step: the reference's "
                         "chunked order (bit-identical MATMUL_TT) or the finer split")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling aid: decode on a TinyLlama-width chip with this many "
                         "layers (small enough for a profiler), print ms per tape step, "
                         "exit (no JSON line)")
    ap.add_argument("--prefill", action="store_true",
                    help="config-2 workload: time a 2047-token prompt, batched prompt pass "
                         "beside step by step, print one JSON line and exit")
    ap.add_argument("--ttgemm-shape", type=int, nargs=4, metavar=("ROWS", "K", "N", "CODES"),
                    help="profiling aid: time kllm_tt_gemm (prefill TT-GEMM) on one seeded "
                         "shape over --steps launches, beside kllm_tt_gemv, and exit")
    ap.add_argument("--ttgemv-shape", type=int, nargs=3, metavar=("K", "N", "CODES"),
                    help="profiling aid: run kllm_tt_gemv on one seeded config-1 shape "
                         "--steps times and exit (no JSON line)")
    args = ap.parse_args()
    if args.prefill:
        prefill_run(args.steps, args.warmup)
        return
    if args.ttgemm_shape:
        ttgemm_time(*args.ttgemm_shape, reps=args.steps)
        return
    if args.ttgemv_shape:
        ttgemv_once(*args.ttgemv_shape, reps=args.steps)
        return
    if args.layers:
        decode_small(args.layers, args.steps, args.warmup)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
