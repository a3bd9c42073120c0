"""Column-sharded decode on 2, 4 and 8 GPUs (each skipped with fewer).

Every rank multiplies its column groups and stores its results into both
ranks' activations over NVLink inside the decode kernel; each output
column's arithmetic is unchanged, so tokens and the final logits equal the
1-GPU run bit for bit (exact order), and tokens stay identical in the fast
order."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import harness

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, path, prompt, max_new, order, out):
    import torch.distributed as dist

    import kmap_b200
    kmap_b200.lib().kllm_set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        with kmap_b200.Chip(path, order=order) as chip:
            chip.connect(kmap_b200.exchange_blocks(chip.shard(rank, world)))
            dist.barrier()
            toks, lg = chip.infer(prompt, max_new, logits=True)
            out[rank] = (toks.tolist(), chip.final_logits().tolist())
            dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_sharded(path, prompt, max_new, order, world=2):
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_rank, args=(world, _free_port(), path, prompt, max_new, order, out), nprocs=world,
             join=True)
    return [out[r] for r in range(world)]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("order", ["exact", "fast"])
@pytest.mark.parametrize("name", ["tl", "tinyllama2"])
def test_sharded_decode_matches_one_gpu(gpu, chip_dir, tmp_path, name, order, world):
    import kmap_b200
    from kmap_b200 import chipgen
    if kmap_b200.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    if name == "tinyllama2":
        spec = chipgen.ModelSpec(**{**chipgen.TINYLLAMA_1B.__dict__})
        spec.num_layers = 2
        spec.max_seq = 128
        path = chipgen.ensure_chip(str(tmp_path), spec)
    else:
        path = chip_dir(name)
    o = kmap_b200.ORDER_FAST if order == "fast" else kmap_b200.ORDER_EXACT
    with kmap_b200.Chip(path, order=o) as chip:
        V = chip.info["vocab_size"]
        prompt = np.random.default_rng(5).integers(3, V, 5).astype(np.int32)
        toks1 = chip.infer(prompt, 10)
        lg1 = chip.final_logits()
    res = _run_sharded(path, prompt, 10, o, world)
    for toks, lg in res:
        assert toks == toks1.tolist()
        if order == "exact":
            np.testing.assert_array_equal(np.array(lg, np.float32), lg1)
