"""Column-sharded decode on 2, 4 and 8 GPUs (each skipped with fewer).

Every rank multiplies its column groups and stores its results into both
ranks' activations over NVLink inside the decode kernel; each output
column's arithmetic is unchanged, so tokens and the final logits equal the
1-GPU run bit for bit.  A sharded context always runs the reference
summation order (the fast order is built for one GPU only)."""
import dataclasses
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp


pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, path, prompt, max_new, order, out):
    import datetime

    import torch.distributed as dist

    import kmap_b200
    kmap_b200.lib().kllm_set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        with kmap_b200.Chip(path, order=order) as chip:
            chip.connect(kmap_b200.exchange_blocks(chip.shard(rank, world)))
            dist.barrier()
            toks, lg = chip.infer(prompt, max_new, logits=True)
            out[rank] = (toks.tolist(), chip.final_logits().tolist())
            dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_sharded(path, prompt, max_new, order, world=2, limit=300):
    """One process per rank; every rank is joined with a time limit and
    killed if it is still running then (the test fails instead of waiting)."""
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, path, prompt, max_new, order, out))
             for r in range(world)]
    for p in procs:
        p.start()
    t_end = time.time() + limit
    for p in procs:
        p.join(timeout=max(1.0, t_end - time.time()))
    alive = [r for r, p in enumerate(procs) if p.is_alive()]
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(timeout=30)
    assert not alive, "ranks %s still running after %d s" % (alive, limit)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [out[r] for r in range(world)]


def _chip(chip_dir, tmp_path, name):
    from kmap_b200 import chipgen
    if name == "tinyllama2":
        spec = dataclasses.replace(chipgen.TINYLLAMA_1B, num_layers=2, max_seq=128)
        return chipgen.ensure_chip(str(tmp_path), spec)
    return chip_dir(name)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", ["tl", "tinyllama2"])
def test_sharded_decode_matches_one_gpu(gpu, chip_dir, tmp_path, name, world):
    import kmap_b200
    if kmap_b200.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    path = _chip(chip_dir, tmp_path, name)
    o = kmap_b200.ORDER_EXACT
    with kmap_b200.Chip(path, order=o) as chip:
        V = chip.info["vocab_size"]
        prompt = np.random.default_rng(5).integers(3, V, 5).astype(np.int32)
        toks1 = chip.infer(prompt, 10)
        lg1 = chip.final_logits()
    res = _run_sharded(path, prompt, 10, o, world)
    for toks, lg in res:
        assert toks == toks1.tolist()
        np.testing.assert_array_equal(np.array(lg, np.float32), lg1)


def test_sharded_fast_order_request_runs_reference_order(gpu, chip_dir, tmp_path):
    """A column-sharded context asked for the fast order builds the
    reference order: the same bits as one GPU in the reference order."""
    import kmap_b200
    if kmap_b200.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    path = _chip(chip_dir, tmp_path, "tl")
    with kmap_b200.Chip(path, order=kmap_b200.ORDER_EXACT) as chip:
        V = chip.info["vocab_size"]
        prompt = np.random.default_rng(5).integers(3, V, 5).astype(np.int32)
        toks1 = chip.infer(prompt, 10)
        lg1 = chip.final_logits()
    for toks, lg in _run_sharded(path, prompt, 10, kmap_b200.ORDER_FAST, 2):
        assert toks == toks1.tolist()
        np.testing.assert_array_equal(np.array(lg, np.float32), lg1)
