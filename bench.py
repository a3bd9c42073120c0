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
  roofline   the decode step kernel (k_decode_step, one launch per tape step):
             the index stream's bytes / its mean launch time
  parity     tokens and per-step logits of one call against the compiled
             reference runtime on the same chip and prompt
  cpu_baseline  the compiled reference runtime (oracle/_ref) on this host,
             pinned to 8 cores, the full 32 + 128 workload once (rank 0, N=1)
  prefill    the 2047-token prompt pass on the same chip (N=1)
  ttgemv_microbench  kllm_tt_gemv (k_tt_fused) on the isolated MATMUL_TT
             shapes over rotating copies larger than L2
For N > 1 the N ranks run ONE decode stream column-sharded over the N GPUs
(every MATMUL_TT's columns split across ranks, NVLink peer stores inside the
decode kernel): value = that stream's tokens / max-over-ranks time,
"scaling": "strong"; "replicas" adds N independent single-GPU streams.
--impl reference: the compiled reference runtime on the host cores, each step
8 consecutive tape positions of the same 32 + 128 workload (20 steps = one
whole call).
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
# 311.1 MB measured on the 2-layer TinyLlama-width chip (307.2 MB of index
# stream, ratio 1.0126), scaled to the 22-layer index stream
STEP_TRAFFIC_BYTES = 2094968839
CHIP_CACHE = os.environ.get("KLLM_CHIP_CACHE", "/tmp/kllm_chips")
TT_SHAPES = [(2048, 2048, 4096), (2048, 5632, 5461), (5632, 2048, 5461), (2048, 32000, 5461)]


def log(*a):
    print("[bench]", *a, file=sys.stderr, flush=True)


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def tinyllama_chip(rank=0, layers=None):
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
    """Average launch time of the TT-GEMV on the benchmark shapes (TT_SHAPES), timed with
    CUDA events on the launching stream; copies rotate so that every launch
    reads its indices from HBM.  `us`: one launch per copy captured in a CUDA
    graph and replayed, so the kernels run back to back (the device time of
    a launch); `us_host_loop`: the same launches issued one by one from
    Python through the C ABI (bounded by the host's call rate for the small
    shapes)."""
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
        ms_host = e0.elapsed_time(e1) / reps
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                cs = torch.cuda.current_stream(dev)
                for i in range(copies):
                    rc = lib.kllm_tt_gemv(d_x.data_ptr(), 1, d_cb.data_ptr(), C,
                                          d_idx[i].data_ptr(), K, N, d_y.data_ptr(),
                                          cs.cuda_stream)
                    assert rc == 0, kmap_b200.last_error()
            g.replay()
            torch.cuda.synchronize(dev)
            greps = max(3, -(-reps // copies))
            e0.record(stream)
            for _ in range(greps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms, how = e0.elapsed_time(e1) / (greps * copies), "graph"
            del g
        except Exception as e:   # keep the host-loop number, say why
            log("ttgemv graph timing unavailable: %s" % e)
            ms, how = ms_host, "host loop"
        res.append({"K": K, "N": N, "codes": C, "us": ms * 1e3, "timed_by": how,
                    "gbs": K * N * 2 / (ms * 1e-3) / 1e9, "us_host_loop": ms_host * 1e3})
        del d_idx
    return res


def ttgemv_once(K, N, C, reps):
    """kllm_tt_gemv on one seeded benchmark shape, `reps` launches (for ncu)."""
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
    # the tensor-core form needs a codebook of bf16 numbers: the same codes,
    # each entry rounded to bf16
    cb16 = (cb.view(np.uint32) & np.uint32(0xffff0000)).view(np.float32)
    dc16 = torch.from_numpy(np.pad(cb16, (0, (-len(cb16)) % 4))).to(dev)
    for name in ("kllm_tt_gemm", "kllm_tt_gemm_tc"):
        f = getattr(lib, name)
        if name == "kllm_tt_gemm_tc":   # (includes building the bf16 weight and x terms)
            call = lambda: f(dx.data_ptr(), rows, dc16.data_ptr(), C, di.data_ptr(), K, N,
                             dy.data_ptr(), 3, s.cuda_stream)
        else:
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


REF_CORES = 8   # the reference's TT pool is 8 threads (compile-time fixed)


def prefill_measure(path, reps=3):
    """The 2047-token prompt on the TinyLlama-arch chip: a uniform-random
    prompt (the chip's 2048 positions less the first generated token), batch
    1.  Device time of the prompt pass -- the batched pass (TT-GEMMs and row
    kernels for positions 0..2045, then position 2046 as a decode step) and
    the step-by-step one -- and the first token's logits of both (the logits
    slot after the prompt, max_new = 0)."""
    import kmap_b200
    P = 2047
    prompt = np.random.default_rng(2).integers(3, 32000, P).astype(np.int32)
    res, first = {}, {}
    for mode in ("batched", "step_by_step"):
        with kmap_b200.Chip(path, prefill=(mode == "batched")) as chip:
            ms = []
            for i in range(1 + (reps if mode == "batched" else 1)):
                chip.infer(prompt, 0)
                if i >= 1:
                    ms.append(chip.stats()["prefill_ms"])
            first[mode] = chip.final_logits()
            m = statistics.median(ms)
            res[mode] = {"ms": m, "tok_s": P / (m * 1e-3)}
    a, b = first["batched"], first["step_by_step"]
    # one multiply and one add per weight and prompt position (the TT-GEMMs)
    ops = 2.0 * (P - 1) * INDEX_BYTES_PER_TOKEN / 2
    return {"prompt": P, "value": res["batched"]["tok_s"], "unit": "tok/s",
            "batched": res["batched"], "step_by_step": res["step_by_step"],
            "projection_fp32_ops": ops,
            "fp32_tops_whole_pass": ops / (res["batched"]["ms"] * 1e-3) / 1e12,
            "first_token": {"equal": int(np.argmax(a)) == int(np.argmax(b)),
                            "max_abs_logit_diff": float(np.max(np.abs(a - b))),
                            "allclose_1e-3_1e-4": bool(np.allclose(a, b, rtol=1e-4, atol=1e-3))}}


def prefill_run(steps, warmup):
    """The prefill measurement alone, as one JSON line."""
    import kmap_b200
    kmap_b200.require_gpu()
    r = prefill_measure(tinyllama_chip(0), reps=max(steps, 1))
    print(json.dumps({"metric": "prefill tok/s (prompt positions per second, device time)",
                      "value": r["value"], "unit": "tok/s", "n_gpus": 1, "steps": steps,
                      "warmup": warmup, "higher_is_better": True, "data": "synthetic",
                      "dtype": "f32",
                      "config": {"workload": "TinyLlama-1.1B-arch TT chip, 2047-token prompt, "
                                             "batch 1, KV cache filled", "prompt": r["prompt"]},
                      "prefill": r}))


# ---------------------------------------------------------------- arms ---

def host_cpu():
    """This host's CPU model and core counts."""
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"model": model, "nproc": os.cpu_count(),
            "affinity": len(os.sched_getaffinity(0))}


def pin_reference_cores():
    """Pin this process to REF_CORES of its allowed cores and size OpenBLAS
    to them (before the reference library loads), as taskset would."""
    allowed = sorted(os.sched_getaffinity(0))
    cores = allowed[:REF_CORES]
    os.sched_setaffinity(0, cores)
    os.environ["OPENBLAS_NUM_THREADS"] = str(len(cores))
    os.environ["OMP_NUM_THREADS"] = str(len(cores))
    return cores


def cpu_sample(out_path):
    """Child process of the GPU arm: the compiled reference runtime on
    REF_CORES pinned host cores, the whole TinyLlama-arch call (32 prompt + 128
    greedy positions) once, with every position's logits; writes an npz."""
    cores = pin_reference_cores()
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    chip = tinyllama_chip()
    ref = harness.Ref()
    h, info = ref.chip(chip)
    p = prompt_ids()
    s = ref.session(h, p, GEN)
    lg = np.zeros((PROMPT + GEN, int(info[0])), np.float32)
    t = time.perf_counter()
    n = s.run(PROMPT + GEN, lg)
    dt = time.perf_counter() - t
    toks = s.tokens()
    s.close()
    ref.L.refh_chip_destroy(h)
    np.savez(out_path, tokens=toks, logits=lg[:n], seconds=dt, positions=n,
             cores=len(cores))


def reference_baseline(chip_path):
    """Run cpu_sample in a pinned child process; None without the reference."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    if not harness.have_ref():
        return None
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "ref.npz")
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-sample", out],
                           capture_output=True, text=True)
        if r.returncode != 0 or not os.path.exists(out):
            log("reference sample failed: " + r.stderr[-2000:])
            return None
        z = np.load(out)
        return {k: z[k] for k in z.files}


def decode_small(layers, steps, warmup):
    """Decode PROMPT + 16 tokens on a reduced-depth TinyLlama-width chip."""
    import kmap_b200
    kmap_b200.require_gpu()
    chip = kmap_b200.Chip(tinyllama_chip(0, layers))
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


REF_WINDOW = 8   # tape positions per reference-arm step


def run_reference_arm(args, rank, world):
    """The compiled reference runtime on REF_CORES pinned host cores.  Each
    step runs the next REF_WINDOW positions of the TinyLlama-arch call (32 prompt +
    128 greedy positions, the reference's own greedy loop), so 20 steps time
    exactly one whole call; a new call starts after position 159."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    if not harness.have_ref():
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference runtime was not compiled into oracle/_ref"}))
        return
    cores = pin_reference_cores()
    chip = tinyllama_chip()
    ref = harness.Ref()
    h, info = ref.chip(chip)
    p = prompt_ids()
    s = ref.session(h, p, GEN)
    for _ in range(args.warmup):
        if s.run(REF_WINDOW) == 0:
            s.close()
            s = ref.session(h, p, GEN)
    s.close()
    s = ref.session(h, p, GEN)
    times, tok = [], 0
    for _ in range(args.steps):
        t = time.perf_counter()
        n = s.run(REF_WINDOW)
        if n == 0:   # the call is complete: the next one
            s.close()
            s = ref.session(h, p, GEN)
            n = s.run(REF_WINDOW)
        times.append(time.perf_counter() - t)
        tok += n
    s.close()
    ref.L.refh_chip_destroy(h)
    v = tok / sum(times)
    cpu = host_cpu()
    sample = ("compiled reference runtime (_tape_runner.c greedy loop), %d TT threads + "
              "OpenBLAS %d threads pinned to %d of %d cores (%s); each step = the next %d "
              "tape positions of the 32 + 128 call" % (REF_CORES, len(cores), len(cores),
                                                     cpu["nproc"], cpu["model"], REF_WINDOW))
    out = {"metric": "decode tok/s (prompt + generated tape steps per second)", "value": v,
           "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": 1e3 * sum(times) / args.steps, "higher_is_better": True,
           "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "impl": "reference",
           "config": {"workload": "TinyLlama-1.1B-arch TT chip (22x2048, 32/4 heads, SwiGLU "
                      "5632, vocab 32000, bf16-rounded N(0,0.02)), batch-1 greedy decode",
                      "prompt": PROMPT, "generate": GEN, "tape_steps_per_call": PROMPT + GEN,
                      "positions_per_step": REF_WINDOW, "positions_timed": tok,
                      "same_config": True},
           "host": cpu,
           "cpu_baseline": {"value": v, "unit": "tok/s", "cores": len(cores),
                            "kind": "reference", "sample": sample},
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def time_calls(chip, p, steps, clk_index):
    """K calls of the workload: device ms, host seconds, launches, tokens."""
    dev_ms, host_s, launches, tokens = 0.0, 0.0, 0, 0
    with Clocks(clk_index) as clk:
        for _ in range(steps):
            t = time.perf_counter()
            toks = chip.infer(p, GEN)
            host_s += time.perf_counter() - t
            s = chip.stats()
            dev_ms += s["prefill_ms"] + s["decode_ms"]
            launches += s["launches"]
            tokens += PROMPT + len(toks)
    return dev_ms, host_s, launches, tokens, clk.summary()


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
    chip_path = tinyllama_chip(rank)
    order = kmap_b200.ORDER_FAST if args.order == "fast" else kmap_b200.ORDER_EXACT
    t_open = time.time()
    chip = kmap_b200.Chip(chip_path, order=order)
    t_open = time.time() - t_open
    shard = world > 1 and not args.replicas
    if shard:   # every rank holds 1/world of the columns; same prompt everywhere
        chip.connect(kmap_b200.exchange_blocks(chip.shard(rank, world)))
        dist.barrier()
    p = prompt_ids(seed=0 if shard else rank)
    t0 = time.time()
    chip.infer(p, GEN)      # first call prepares the plan (weights to HBM, graph)
    t_first = time.time() - t0
    st = chip.stats()
    log("rank %d: chip open %.2fs, first call %.2fs (fused=%d)" % (rank, t_open, t_first,
                                                                  st["fused"]))
    for _ in range(max(args.warmup - 1, 0)):
        chip.infer(p, GEN)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    dev_ms, host_s, launches, tokens, clocks = time_calls(chip, p, args.steps, local_rank)
    barrier()
    times = torch.tensor([dev_ms, host_s * 1e3], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    dev_ms_max, host_ms_max = times.tolist()
    # tokens (and, on one GPU, every step's logits) of one call, for the
    # parity record (rank 0 compares); a sharded rank holds only its own
    # columns' logits rows, so N > 1 compares tokens
    lg_ours = None
    if world == 1:
        toks_ours, lg_ours = chip.infer(p, GEN, logits=True)
    else:
        toks_ours = chip.infer(p, GEN)
    replicas = None
    if shard:
        # the same workload as N independent single-GPU streams, for context
        chip.close()
        rchip = kmap_b200.Chip(chip_path, order=order)
        rp = prompt_ids(seed=rank)
        for _ in range(max(args.warmup, 1)):
            rchip.infer(rp, GEN)
        barrier()
        r_ms, _, _, r_tok, _ = time_calls(rchip, rp, args.steps, local_rank)
        barrier()
        rt = torch.tensor([r_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(rt, op=dist.ReduceOp.MAX)
        replicas = {"value": r_tok * world / (rt.item() / 1e3), "unit": "tok/s",
                    "streams": world, "scaling": "weak"}
        rchip.close()
        chip = None
    if rank != 0:
        if chip:
            chip.close()
        if dist:
            dist.destroy_process_group()
        return
    streams = 1 if shard else world   # sharded: one stream over all GPUs
    value = tokens * streams / (dev_ms_max / 1e3)
    e2e = tokens * streams / (host_ms_max / 1e3)
    pk = peaks()
    hbm = pk.get("hbm_gbs")
    # the dominant kernel is the decode step (one launch per tape step):
    # its algorithmic bytes are the index stream of every TT matrix
    step_us = dev_ms_max * 1e3 / tokens
    decode_gbs = INDEX_BYTES_PER_TOKEN / (step_us * 1e-6) / 1e9
    # sharded: the index stream is split over the GPUs, so their summed peak
    roof_peak = hbm * world if (shard and hbm) else hbm
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
                   "order": args.order,
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
                     "peak_source": ("MEASURED_PEAKS.json hbm_gbs (burst copy)%s" %
                                     (" x %d GPUs" % world if shard else "") if hbm
                                     else "fallback 6650 GB/s")},
        "clocks": clocks,
        "load": {"chip_open_s": t_open, "first_call_s": t_first,
                 "note": "kllm_chip_open (files to host), then the first processor_infer "
                         "(upload to HBM, decode layouts, graph capture, one 32 + 128 call)"},
    }
    if replicas:
        out["replicas"] = replicas
    if world == 1 and args.order == "exact" and not args.no_fast:
        # the fast summation order on the same workload, for comparison:
        # same tokens required, logits within the tolerance
        with kmap_b200.Chip(chip_path, order=kmap_b200.ORDER_FAST) as fchip:
            for _ in range(max(args.warmup, 1)):
                fchip.infer(p, GEN)
            torch.cuda.synchronize()
            f_ms, _, _, f_tok, _ = time_calls(fchip, p, args.steps, local_rank)
            f_toks, f_lg = fchip.infer(p, GEN, logits=True)
        out["fast_order"] = {"value": f_tok / (f_ms / 1e3), "unit": "tok/s",
                             "launch_us": f_ms * 1e3 / f_tok,
                             "frac": INDEX_BYTES_PER_TOKEN / (f_ms * 1e-3 / f_tok) / 1e9 / hbm
                             if hbm else None,
                             "note": "K of the narrow projections split over more warps; "
                                     "tolerance, not bit-exact MATMUL_TT",
                             "_toks": f_toks, "_lg": f_lg}
    if world == 1:
        roof = ttgemv_roofline(local_rank)
        for r in roof:
            r["frac"] = r["gbs"] / hbm if hbm else None
        top = max(roof, key=lambda r: r["K"] * r["N"])
        out["ttgemv_microbench"] = {"kernel": "k_tt_fused", "unit": "GB/s", "peak": hbm,
                                    "shape": [top["K"], top["N"]], "achieved": top["gbs"],
                                    "frac": top["frac"], "shapes": roof}
        if not args.no_prefill:
            try:
                out["prefill"] = prefill_measure(chip_path)
            except Exception as e:   # reported, not fatal for the decode line
                out["prefill"] = {"error": str(e)[:300]}
    ref = None
    if not args.no_cpu_baseline and (world == 1 or shard):
        ref = reference_baseline(chip_path)
    if ref is not None:
        n = int(ref["positions"])
        rt = ref["tokens"]
        same = len(rt) == len(toks_ours) and bool(np.array_equal(rt, toks_ours))
        out["parity"] = {"reference": "compiled reference runtime, same chip and prompt",
                         "tokens_equal": same, "tokens_compared": int(len(rt))}
        fo = out.get("fast_order")
        if fo is not None:
            rows = min(n, PROMPT + GEN - 1)
            fo["parity"] = {"tokens_equal": bool(np.array_equal(rt, fo["_toks"])),
                            "max_abs_logit_diff": float(np.abs(fo["_lg"][:rows] -
                                                               ref["logits"][:rows]).max()),
                            "logits_allclose_1e-3_1e-4": bool(np.allclose(
                                fo["_lg"][:rows], ref["logits"][:rows], rtol=1e-4, atol=1e-3))}
        if lg_ours is not None:
            rows = min(n, PROMPT + GEN - 1)   # the last step's logits pick no token
            d = np.abs(lg_ours[:rows] - ref["logits"][:rows])
            out["parity"].update({
                "max_abs_logit_diff": float(d.max()), "logit_rows": rows,
                "logits_allclose_1e-3_1e-4": bool(np.allclose(
                    lg_ours[:rows], ref["logits"][:rows], rtol=1e-4, atol=1e-3))})
        if world == 1:
            cpu = host_cpu()
            v = n / float(ref["seconds"])
            out["cpu_baseline"] = {
                "value": v, "unit": "tok/s", "cores": int(ref["cores"]), "kind": "reference",
                "sample": "compiled reference runtime on %d pinned cores of %d (%s), %d TT "
                          "threads + OpenBLAS %d: the whole 32 + 128 call once (%d positions, "
                          "%.1f s)" % (int(ref["cores"]), cpu["nproc"], cpu["model"], REF_CORES,
                                       int(ref["cores"]), n, float(ref["seconds"]))}
    if "fast_order" in out:
        out["fast_order"].pop("_toks", None)
        out["fast_order"].pop("_lg", None)
    print(json.dumps(out), flush=True)
    if chip:
        chip.close()
    if dist:
        dist.destroy_process_group()


# --------------------------------------------------------- 7B-arch decode --

L7B_PROMPT, L7B_GEN = 4096, 256
L7B_INDEX_BYTES = 13214154752   # sum of K * N * 2 over the 7B chip's 129 TT matrices


def chip_7b(local_rank):
    """The Llama-2-7B-architecture chip (32 x 4096, 32 MHA heads of 128,
    SwiGLU 11008, vocab 32000, max_seq 4352), weights drawn on the GPU."""
    import fcntl

    import torch
    spec = chipgen.ModelSpec(**{**chipgen.LLAMA2_7B.__dict__})
    os.makedirs(CHIP_CACHE, exist_ok=True)
    with open(os.path.join(CHIP_CACHE, ".lock"), "w") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        t = time.time()
        path = chipgen.ensure_chip(CHIP_CACHE, spec, device=torch.device("cuda", local_rank))
        log("7B chip ready in %.1fs: %s" % (time.time() - t, path))
    return path


def run_7b(args, rank, world, local_rank):
    """7B-arch decode: batch-1 greedy decode of 256 tokens after a 4096-token
    uniform-random prompt on the 7B-architecture chip; the prompt through
    the batched pass (tensor-core projections), then one decode step kernel
    per token, column-sharded over the N GPUs for N > 1.  value = generated
    tokens per second of decode device time; the prompt pass is reported
    beside it.  Parity: tokens and logits of a shortened run (16 prompt + 8
    generated) against the compiled reference on the same chip (rank 0)."""
    import kmap_b200
    kmap_b200.require_gpu()
    import torch
    torch.cuda.set_device(local_rank)
    kmap_b200.lib().kllm_set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local_rank))
    path = chip_7b(local_rank)
    if dist:
        dist.barrier()
    t_open = time.time()
    chip = kmap_b200.Chip(path, prefill=True)
    t_open = time.time() - t_open
    if world > 1:
        chip.connect(kmap_b200.exchange_blocks(chip.shard(rank, world)))
        dist.barrier()
    V = chip.info["vocab_size"]
    # parity run first (every rank takes part in a sharded decode)
    short = np.random.default_rng(5).integers(3, V, 16).astype(np.int32)
    toks_short = chip.infer(short, 8)
    lg_short = chip.final_logits()
    prompt = np.random.default_rng(3).integers(3, V, L7B_PROMPT).astype(np.int32)
    t0 = time.time()
    chip.infer(prompt, L7B_GEN)
    t_first = time.time() - t0
    for _ in range(max(args.warmup - 1, 0)):
        chip.infer(prompt, L7B_GEN)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    pre_ms, dec_ms, gen = 0.0, 0.0, 0
    with Clocks(local_rank) as clk:
        for _ in range(args.steps):
            toks = chip.infer(prompt, L7B_GEN)
            st = chip.stats()
            pre_ms += st["prefill_ms"]
            dec_ms += st["decode_ms"]
            gen += len(toks)
    barrier()
    tt = torch.tensor([pre_ms, dec_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    pre_ms, dec_ms = tt.tolist()
    chip.close()
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    # decode_ms covers the 256 generated tokens' steps after the prompt's
    # last position (plus the final fed token): one kernel per step
    steps_dec = L7B_GEN
    step_us = dec_ms * 1e3 / (args.steps * steps_dec)
    gbs = L7B_INDEX_BYTES / (step_us * 1e-6) / 1e9
    hbm = peaks().get("hbm_gbs")
    out = {"metric": "decode tok/s (generated tokens per second of decode device time)",
           "value": gen / (dec_ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "higher_is_better": True,
           "scaling": "strong" if world > 1 else "weak", "dtype": "f32", "data": "synthetic",
           "config": {"workload": "Llama-2-7B-arch TT chip (32x4096, 32 MHA heads of 128, "
                      "SwiGLU 11008, vocab 32000, bf16-rounded N(0,0.02) drawn on the GPU), "
                      "4096-token prompt + 256 greedy tokens, batch 1",
                      "parallelism": ("column-sharded over %d GPUs" % world if world > 1
                                      else "single GPU")},
           "prefill": {"tok_s": args.steps * (L7B_PROMPT - 1) / (pre_ms / 1e3),
                       "ms_per_prompt": pre_ms / args.steps},
           "roofline": {"bound": "hbm", "kernel": "k_decode_step", "launch_us": step_us,
                        "algorithmic_bytes_per_launch": L7B_INDEX_BYTES, "achieved": gbs,
                        "peak": hbm * world if hbm else None, "unit": "GB/s",
                        "frac": gbs / (hbm * world) if hbm else None},
           "load": {"chip_open_s": t_open, "first_call_s": t_first},
           "clocks": clk.summary()}
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    if harness.have_ref() and not args.no_cpu_baseline:
        ref = harness.Ref()
        h, info = ref.chip(path)
        s = ref.session(h, short, 8)
        lg = np.zeros((len(short) + 8, V), np.float32)
        t = time.time()
        s.run(len(short) + 8, lg)
        dt = time.time() - t
        rt = s.tokens()
        s.close()
        ref.L.refh_chip_destroy(h)
        out["parity"] = {"reference": "compiled reference runtime, same chip, 16-token prompt "
                                      "+ 8 greedy tokens (%.1f s on the host)" % dt,
                         "tokens_equal": rt.tolist() == toks_short.tolist(),
                         "final_logits_max_abs_diff": float(np.abs(lg[-1] - lg_short).max()),
                         "final_logits_allclose_1e-3_1e-4": bool(np.allclose(
                             lg_short, lg[-1], rtol=1e-4, atol=1e-3))}
    print(json.dumps(out), flush=True)
    if dist:
        dist.destroy_process_group()


B8_SEQS, B8_PROMPT, B8_GEN = 32, 1024, 128


def chip_8b(local_rank):
    """The Llama-3-8B-architecture chip (32 x 4096, 32 query / 8 kv heads of
    128, SwiGLU 14336, vocab 128256, rope theta 5e5, max_seq 1152), weights
    drawn on the GPU."""
    import fcntl

    import torch
    spec = chipgen.ModelSpec(**{**chipgen.LLAMA3_8B.__dict__})
    os.makedirs(CHIP_CACHE, exist_ok=True)
    with open(os.path.join(CHIP_CACHE, ".lock"), "w") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        t = time.time()
        path = chipgen.ensure_chip(CHIP_CACHE, spec, device=torch.device("cuda", local_rank))
        log("8B chip ready in %.1fs: %s" % (time.time() - t, path))
    return path, spec


def run_8b_batch(args, rank, world, local_rank):
    """8B-arch batched decode: greedy decode of 32 concurrent sequences (1024-token
    uniform-random prompts, 128 generated tokens each) on the
    Llama-3-8B-architecture chip.  Each sequence's prompt goes through the
    batched prompt pass into its own KV cache; every decode step then runs
    each projection once over the 32 rows (the skinny tensor-core GEMM,
    weight bytes read once per step), attention per sequence.  With N GPUs
    the sequences are divided among the ranks (independent sequences: no
    data-path collective), each rank with the whole chip.  value = generated
    tokens per second of decode device time, all sequences; e2e = the same
    tokens per second of wall time of the whole call (prompt upload, prompt
    passes, decode, token read-back).  Parity: a 4-sequence batch of short
    prompts against each sequence's single-sequence decode (the exact
    persistent step, bit-identical to the reference's MATMUL_TT) and one
    sequence against the compiled reference."""
    import kmap_b200
    kmap_b200.require_gpu()
    import torch
    torch.cuda.set_device(local_rank)
    kmap_b200.lib().kllm_set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local_rank))
    path, spec = chip_8b(local_rank)
    if dist:
        dist.barrier()
    t_open = time.time()
    chip = kmap_b200.Chip(path)
    t_open = time.time() - t_open
    V = chip.info["vocab_size"]
    rng = np.random.default_rng(11)
    prompts = [rng.integers(3, V, B8_PROMPT).astype(np.int32) for _ in range(B8_SEQS)]
    mine = prompts[rank::world]
    # parity first: short prompts, batch vs one sequence at a time
    srng = np.random.default_rng(12)
    short = [srng.integers(3, V, 16 + i).astype(np.int32) for i in range(4)]
    t0 = time.time()
    b_short = chip.infer_batch(short, 8)
    t_first = time.time() - t0
    singles = [chip.infer(p, 8) for p in short]
    for _ in range(args.warmup):
        chip.infer_batch(mine, B8_GEN)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    pre_ms, dec_ms, wall, gen = 0.0, 0.0, 0.0, 0
    with Clocks(local_rank) as clk:
        for _ in range(args.steps):
            t = time.time()
            outs = chip.infer_batch(mine, B8_GEN)
            wall += time.time() - t
            st = chip.stats()
            pre_ms += st["prefill_ms"]
            dec_ms += st["decode_ms"]
            gen += sum(len(o) for o in outs)
    launches = chip.stats().get("launches")
    barrier()
    tt = torch.tensor([pre_ms, dec_ms, wall, gen], dtype=torch.float64, device="cuda")
    if dist:
        mx = tt[:3].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        g = tt[3:].clone()
        dist.all_reduce(g, op=dist.ReduceOp.SUM)
        tt = torch.cat([mx, g])
    pre_ms, dec_ms, wall, gen = tt.tolist()
    chip.close()
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    H, F, L, Vv = spec.hidden_size, spec.intermediate_size, spec.num_layers, spec.vocab_size
    hd = H // spec.num_attention_heads
    kvd = spec.num_key_value_heads * hd
    w_bytes = 2 * (L * (H * (H + 2 * kvd) + H * H + H * 2 * F + F * H) + H * Vv)
    # k and v rows read per step, summed over the steps (n = pos + 1 per row)
    kv_rows = B8_SEQS * sum(B8_PROMPT + i for i in range(B8_GEN))
    kv_bytes = kv_rows * L * kvd * 4 * 2
    step_bytes = w_bytes + kv_bytes / B8_GEN
    step_us = dec_ms * 1e3 / (args.steps * B8_GEN)
    gbs = step_bytes / (step_us * 1e-6) / 1e9
    hbm = peaks().get("hbm_gbs")
    out = {"metric": "batched decode tok/s (generated tokens per second of decode device "
                     "time, all sequences)",
           "value": gen / (dec_ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": dec_ms / args.steps, "higher_is_better": True,
           "scaling": "strong" if world > 1 else "weak", "dtype": "bf16 tensor-core GEMM, f32",
           "data": "synthetic",
           "config": {"workload": "Llama-3-8B-arch TT chip (32x4096, 32 query / 8 kv heads of "
                      "128, SwiGLU 14336, vocab 128256, rope theta 5e5, bf16-rounded N(0,0.02) "
                      "drawn on the GPU), 32 sequences x (1024-token prompt + 128 greedy "
                      "tokens)",
                      "parallelism": ("sequences divided over %d GPUs" % world if world > 1
                                      else "single GPU"),
                      "l2": "weights 15 GB and caches 9 GB per step exceed L2"},
           "e2e": {"value": gen / wall, "unit": "tok/s",
                   "h2d_bytes_per_step": 4 * B8_SEQS * B8_PROMPT,
                   "d2h_bytes_per_step": 4 * B8_SEQS * B8_GEN,
                   "note": "wall time of kllm_chip_infer_batch: prompt passes included"},
           "prefill": {"tok_s": args.steps * B8_SEQS * (B8_PROMPT - 1) / (pre_ms / 1e3),
                       "ms_per_batch": pre_ms / args.steps},
           "roofline": {"bound": "hbm", "kernel": "one decode step of 32 sequences "
                        "(graph: skinny tcgen05 GEMMs, grouped attention, row kernels)",
                        "launch_us": step_us,
                        "algorithmic_bytes_per_launch": step_bytes,
                        "weight_bytes": w_bytes, "kv_bytes_mean": kv_bytes / B8_GEN,
                        "achieved": gbs, "peak": hbm * world if hbm else None, "unit": "GB/s",
                        "frac": gbs / (hbm * world) if hbm else None},
           "gpu_launches": launches,
           "load": {"chip_open_s": t_open, "first_call_s": t_first},
           "parity": {"batch_vs_single_sequence_tokens_equal":
                      all(a.tolist() == b.tolist() for a, b in zip(b_short, singles)),
                      "sequences": "4 prompts of 16..19 tokens + 8 greedy tokens"},
           "clocks": clk.summary()}
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import harness
    if harness.have_ref() and not args.no_cpu_baseline:
        ref = harness.Ref()
        h, info = ref.chip(path)
        t = time.time()
        rt = ref.infer(h, short[0][:8], 4)
        dt = time.time() - t
        ref.L.refh_chip_destroy(h)
        with kmap_b200.Chip(path) as c2:
            ours = c2.infer_batch([short[0][:8], short[1][:8]], 4)[0]
        out["parity"]["reference"] = ("compiled reference runtime, same chip, 8-token prompt "
                                      "+ 4 greedy tokens (%.1f s on the host)" % dt)
        out["parity"]["reference_tokens_equal"] = rt.tolist() == ours.tolist()
    print(json.dumps(out), flush=True)
    if dist:
        dist.destroy_process_group()


def batch_profile(new_tokens):
    """Profiling aid: one 8B-arch batch (32 sequences x 1024-token prompts)
    with `new_tokens` generated each; prints the prompt-pass and per-step
    device times and the launch count (no JSON line)."""
    import kmap_b200
    kmap_b200.require_gpu()
    import torch
    torch.cuda.set_device(0)
    path, _ = chip_8b(0)
    with kmap_b200.Chip(path) as chip:
        V = chip.info["vocab_size"]
        rng = np.random.default_rng(11)
        prompts = [rng.integers(3, V, B8_PROMPT).astype(np.int32) for _ in range(B8_SEQS)]
        chip.infer_batch(prompts, new_tokens)
        st = chip.stats()
    log("c4: prompt passes %.1f ms, %d steps %.3f ms each, %d launches" % (
        st["prefill_ms"], new_tokens, st["decode_ms"] / new_tokens, st["launches"]))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="with N > 1: N independent single-GPU decode streams (weak scaling) "
                         "instead of one stream column-sharded over the N GPUs")
    ap.add_argument("--no-prefill", action="store_true",
                    help="leave the prefill measurement out of the JSON line")
    ap.add_argument("--no-fast", action="store_true",
                    help="leave the fast-order comparison out of the JSON line")
    ap.add_argument("--cpu-sample", metavar="OUT", help=argparse.SUPPRESS)
    ap.add_argument("--model", default="tinyllama-1.1b", choices=["tinyllama-1.1b", "llama2-7b", "llama3-8b-batch"],
                    help="llama2-7b: the 7B-architecture decode workload (4096-token prompt, "
                         "256 tokens) as its own JSON line; llama3-8b-batch: 32 sequences "
                         "of 1024 + 128 tokens on the 8B-architecture chip")
    ap.add_argument("--order", default="exact", choices=["exact", "fast"],
                    help="TT-GEMV summation order of the decode step: the reference's "
                         "chunked order (bit-identical MATMUL_TT) or the finer split")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling aid: decode on a TinyLlama-width chip with this many "
                         "layers (small enough for a profiler), print ms per tape step, "
                         "exit (no JSON line)")
    ap.add_argument("--prefill", action="store_true",
                    help="the 2047-token prompt workload: time it through the batched prompt pass "
                         "beside step by step, print one JSON line and exit")
    ap.add_argument("--ttgemm-shape", type=int, nargs=4, metavar=("ROWS", "K", "N", "CODES"),
                    help="profiling aid: time kllm_tt_gemm (prefill TT-GEMM) on one seeded "
                         "shape over --steps launches, beside kllm_tt_gemv, and exit")
    ap.add_argument("--batch-profile", type=int, metavar="NEW",
                    help="profiling aid: one 32 x 1024-token batch on the 8B chip with NEW "
                         "tokens generated each; prints step times and exits")
    ap.add_argument("--ttgemv-shape", type=int, nargs=3, metavar=("K", "N", "CODES"),
                    help="profiling aid: run kllm_tt_gemv on one seeded benchmark shape "
                         "--steps times and exit (no JSON line)")
    args = ap.parse_args()
    if args.cpu_sample:
        cpu_sample(args.cpu_sample)
        return
    if args.prefill:
        prefill_run(args.steps, args.warmup)
        return
    if args.ttgemm_shape:
        ttgemm_time(*args.ttgemm_shape, reps=args.steps)
        return
    if args.batch_profile:
        batch_profile(args.batch_profile)
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
    if args.model == "llama2-7b":
        run_7b(args, rank, world, local_rank)
    elif args.model == "llama3-8b-batch":
        run_8b_batch(args, rank, world, local_rank)
    elif args.impl == "reference":
        run_reference_arm(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
