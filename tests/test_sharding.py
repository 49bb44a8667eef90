"""Multi-rank host logic on CPU (gloo, world size 2): token shards of the statistics sum to the whole (the fp32
accumulators are what the layer build all-reduces), row shards cover every row once, and the padded all-gather of
row shards reassembles the states."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lookatmyquant_b200.layer import row_shard
from lookatmyquant_b200.workloads import token_shard


def test_shards_partition_exactly():
    for total in (64, 1000, 4096 + 2048, 9728, 30720):
        for world in (1, 2, 3, 4, 8):
            spans = [row_shard(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(s[0] % 64 == 0 for s in spans)
    for tokens in (16384, 786432, 100000):
        for world in (1, 2, 4, 8):
            spans = [token_shard(tokens, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == tokens
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import core as O
        g = torch.Generator().manual_seed(0)
        X = torch.randn(5000, 48, generator=g).to(torch.bfloat16).float()
        w = torch.where(torch.rand(5000, generator=g) < 0.1, 10.0, 1.0)
        lo, hi = token_shard(5000, rank, world, chunk=1000)
        # this rank's fp32 accumulator Σ x (w x)ᵀ over its tokens, summed across ranks
        acc = (X[lo:hi].T @ (X[lo:hi] * w[lo:hi, None])).float()
        dist.all_reduce(acc)
        H = (acc / 5000).double().numpy()
        ref, _ = O.hessian_accumulate([X.numpy()], [w.numpy()])
        err = float(np.linalg.norm(H - ref) / np.linalg.norm(ref))
        # row shards: each rank holds its rows of a 300 x 7 "states" matrix; gather padded shards
        total, cols = 300, 7
        states = torch.arange(total * cols, dtype=torch.int16).reshape(total, cols)
        r0, r1 = row_shard(total, rank, world)
        cap = ((total + 63) // 64 + world - 1) // world * 64
        buf = torch.zeros(cap, cols, dtype=torch.int16)
        buf[: r1 - r0] = states[r0:r1]
        # collectives have no int16 type: the shards travel as bytes
        parts = [torch.empty_like(buf).view(torch.uint8) for _ in range(world)]
        dist.all_gather(parts, buf.view(torch.uint8))
        parts = [p.view(torch.int16) for p in parts]
        back = torch.cat([parts[r][: row_shard(total, r, world)[1] - row_shard(total, r, world)[0]]
                          for r in range(world)])
        q.put((rank, err, bool(torch.equal(back, states))))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, err, ok in out:
        assert err < 1e-5, (rank, err)
        assert ok, rank
