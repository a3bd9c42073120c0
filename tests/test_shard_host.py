"""Column-sharded decode, host side (no GPU): the block exchange over
torch.distributed with gloo at world size 2, the column-group assignment,
and the C ABI's argument and sequencing errors."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(rank, world, port, out):
    import torch.distributed as dist

    import kmap_b200
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blocks = kmap_b200.exchange_blocks(bytes([rank]) * (64 * 10))
        out[rank] = [b[0] for b in blocks] == list(range(world)) and \
            all(len(b) == 640 for b in blocks)
    finally:
        dist.destroy_process_group()


def test_exchange_blocks_gloo_world2():
    world = 2
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_exchange, args=(world, _free_port(), out), nprocs=world, join=True)
    assert out[0] and out[1]


@pytest.mark.parametrize("ngroups", [1, 7, 256, 320, 1408, 4000])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_group_assignment_covers_every_column_group_once(ngroups, world):
    # stored group i of rank r is group i * world + r of the matrix
    # (ttx_shard); a rank holds ceil((ngroups - r) / world) groups
    seen = np.zeros(ngroups, np.int32)
    for r in range(world):
        local = (ngroups - r + world - 1) // world if r < ngroups else 0
        for i in range(local):
            seen[i * world + r] += 1
    assert (seen == 1).all()


def test_shard_abi_errors(built_lib):
    import ctypes as C

    import kmap_b200
    lib = kmap_b200.lib()
    ctx = lib.tape_ctx_create(4, 1)
    try:
        assert lib.kllm_shard_set(ctx, 2, 2) == -1          # rank out of range
        assert b"rank 2 of 2" in lib.kllm_last_error()
        lib.kllm_clear_error()
        assert lib.kllm_shard_set(ctx, 1, 2) == 0
        n = C.c_size_t(0)
        assert lib.kllm_shard_export(ctx, None, 0, C.byref(n)) == -1   # no plan yet
        assert b"no fused decode plan" in lib.kllm_last_error()
        lib.kllm_clear_error()
        assert lib.kllm_shard_connect(ctx, b"\0" * 8, 8) == -1
        lib.kllm_clear_error()
    finally:
        lib.tape_ctx_destroy(ctx)
