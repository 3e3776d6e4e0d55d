"""The N>1 path on CPU: world_size-2 gloo ranks shard each op family's work units, compute
their shard (with the CPU oracle standing in for the kernel), and the verification
all-gather reassembles exactly the single-process result."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from ntilang_b200.dist import shard_bounds


def test_shard_bounds_cover_exactly():
    for total in (0, 1, 7, 512, 4097):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from ntilang_b200.dist import gather_rows, shard_heads, shard_rows
    from oracle import ntl_oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = np.random.default_rng(0)
        x = torch.from_numpy(g.uniform(-1, 1, size=(37, 256)).astype(np.float32))
        local = torch.from_numpy(O.cumsum_rows(shard_rows(x, rank, world).numpy()))
        full = gather_rows(local, world)
        ok_rows = np.array_equal(full.numpy().view(np.uint32), O.cumsum_rows(x.numpy()).view(np.uint32))
        a = torch.from_numpy(g.normal(size=(50, 32)).astype(np.float16))
        b = torch.from_numpy(g.normal(size=(32, 24)).astype(np.float16))
        panel = torch.from_numpy(O.gemm(shard_rows(a, rank, world).numpy(), b.numpy()))
        ok_gemm = np.allclose(gather_rows(panel, world).numpy(), O.gemm(a.numpy(), b.numpy()))
        q = torch.from_numpy(g.normal(size=(2, 3, 64, 16)).astype(np.float16))
        mine = shard_heads(q, rank, world)
        out = torch.from_numpy(O.fa2_blockwise(mine.numpy(), mine.numpy(), mine.numpy(), 0.36, False))
        full_o = gather_rows(out, world).reshape(2, 3, 64, 16)
        ok_attn = np.allclose(full_o.numpy().astype(np.float32),
                              O.fa2_blockwise(q.numpy(), q.numpy(), q.numpy(), 0.36, False).astype(np.float32))
        results[rank] = (ok_rows, ok_gemm, ok_attn)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding_and_gather():
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp

    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}
    del torch
