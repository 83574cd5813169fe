"""(batch x head) sharding and the output all-gather, on CPU gloo ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_vs_sparse_attention_b200 import sharding
from oracle import attention as oracle_attention


def test_unit_range_partitions():
    for U in (1, 7, 8, 16, 64):
        for W in (1, 2, 3, 4, 8):
            seen = []
            for r in range(W):
                a, b = sharding.unit_range(U, W, r)
                assert 0 <= a <= b <= U
                seen += list(range(a, b))
            assert seen == list(range(U))
    with pytest.raises(ValueError):
        sharding.unit_range(8, 2, 2)


def _oracle_fn(q, k, v, causal, block_size, top_k):
    return torch.from_numpy(oracle_attention(q.numpy(), k.numpy(), v.numpy(), causal=causal,
                                             block_size=block_size, top_k=top_k, threads=1))


def _worker(rank, world, port, B, H, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        shape = (B, H, 128, 16)
        Q, K, V = (torch.randn(shape, generator=g) for _ in range(3))
        full = sharding.sharded_attention(Q, K, V, causal=True, block_size=16, top_k=3,
                                          attn_fn=_oracle_fn)
        local = sharding.sharded_attention(Q, K, V, causal=True, block_size=16, top_k=3,
                                           attn_fn=_oracle_fn, gather=False)
        q.put((rank, full.numpy(), local.numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,B,H", [(2, 1, 3), (2, 2, 2), (3, 1, 2)])
def test_sharded_equals_single_process(world, B, H):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, H, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(0)
    Q, K, V = (torch.randn((B, H, 128, 16), generator=g) for _ in range(3))
    want = oracle_attention(Q.numpy(), K.numpy(), V.numpy(), causal=True, block_size=16, top_k=3,
                            threads=1)
    U = B * H
    for rank, full, local in res:
        np.testing.assert_array_equal(full, want)
        a, b = sharding.unit_range(U, world, rank)
        np.testing.assert_array_equal(local[0], want.reshape(U, 128, 16)[a:b])
