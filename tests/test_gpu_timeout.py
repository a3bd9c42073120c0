"""A device wait that runs out ends the decode step with a status, not a hang.

Two processes form a 2-rank column-sharded decode (rank r on GPU r, or both
on GPU 0 when only one is visible).  Rank 1 builds and connects its plan but
never runs a step, so the words rank 0's step waits for (rank 1's columns of
q, k, v and the rest) are never written.  With KLLM_WAIT_LIMIT_MS=300 the
step's polls give up: processor_infer on rank 0 returns an error naming the
status, and the GPU stays usable -- the next call in the same process (a
single-GPU chip) runs to the end with the oracle's tokens.  Only rank 0's
kernel runs; nothing waits on a kernel that is not running."""
import os
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank(rank, path, q_blocks, q_ready, out):
    import kmap_b200
    ndev = kmap_b200.device_count()
    kmap_b200.lib().kllm_set_device(rank % ndev)
    if rank == 0:
        os.environ["KLLM_WAIT_LIMIT_MS"] = "300"
    with kmap_b200.Chip(path) as chip:
        block = chip.shard(rank, 2)
        q_blocks[rank].put(block)
        other = q_blocks[1 - rank].get(timeout=120)
        blocks = [block, other] if rank == 0 else [other, block]
        chip.connect(blocks)
        if rank == 1:
            q_ready.put("connected")
            # stay connected, run nothing, until rank 0 is done
            deadline = time.time() + 120
            while "rank0" not in out and time.time() < deadline:
                time.sleep(0.05)
            return
        q_ready.get(timeout=120)
        prompt = np.array([5, 9, 13, 21], np.int32)
        t = time.time()
        err = None
        try:
            chip.infer(prompt, 4)
        except kmap_b200.KllmError as e:
            err = str(e)
        took = time.time() - t
    # the same GPU, same process: a fresh single-GPU chip runs normally
    with kmap_b200.Chip(path) as chip2:
        toks = chip2.infer(prompt, 6).tolist()
    out["rank0"] = (err, took, toks)


def test_wait_timeout_returns_status_and_gpu_stays_usable(gpu, oracle, chip_dir):
    import harness
    path = chip_dir("tl")
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    q_blocks = [mgr.Queue(), mgr.Queue()]
    q_ready = mgr.Queue()
    procs = [ctx.Process(target=_rank, args=(r, path, q_blocks, q_ready, out)) for r in (0, 1)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, took, toks = out["rank0"]
    assert err is not None and "status" in err and "timed out" in err, err
    assert took < 60, took
    oc = harness.OracleChip(oracle, path)
    toks_o, _ = oc.infer(np.array([5, 9, 13, 21], np.int32), 6)
    oc.close()
    assert toks == toks_o.tolist()
