"""Multi-rank host logic on CPU (gloo, world sizes 2 and 4): token shards of the statistics sum to the whole (the fp32
accumulators are what the layer build all-reduces), row shards cover every row once, and the padded all-gather of
row shards reassembles the states; the stages' factorizations are spread over rank pairs and every rank receives
each stage's factors from its owners."""

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


def test_factor_owners_spread_stages_over_pairs():
    from lookatmyquant_b200.layer import factor_owners
    dims = [2560, 4096, 2560, 9728]  # a Qwen3-4B-class layer's stages
    assert factor_owners(dims, 2) == [(0, 1)] * 4
    eight = factor_owners(dims, 8)
    assert sorted(eight) == [(0, 1), (2, 3), (4, 5), (6, 7)]  # one pair per stage
    assert eight[3] == (0, 1)  # the largest stage first
    four = factor_owners(dims, 4)
    assert four[3] == (0, 1) and all(o == (2, 3) for o in four[:3])  # 9728³ outweighs the other three together
    for world in (2, 3, 4, 5, 8, 16):
        assert all(0 <= e < world and 0 <= q < world and e != q for e, q in factor_owners(dims, world))


def _share_worker(rank, world, port, q):
    """Every stage's owners fill their factor buffers with marks; after _share_factors every rank holds them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lookatmyquant_b200.layer import _share_factors, factor_owners
        dims = [8, 12, 8, 20]
        owners = factor_owners(dims, world)
        ok = True
        for i, n in enumerate(dims):
            e, qr = owners[i]
            Linv = torch.full((n, n), 100.0 * i + qr if rank == qr else -1.0, dtype=torch.float64)
            qst = torch.tensor([i if rank == qr else -1], dtype=torch.int32)
            U = torch.full((n, n), 100.0 * i + e if rank == e else -1.0, dtype=torch.float64)
            dead = torch.full((n,), 1 if rank == e else 7, dtype=torch.uint8)
            est = torch.tensor([i + 50 if rank == e else -1], dtype=torch.int32)
            env, L, qs = _share_factors(None, None, (Linv, qst, U, dead, est), e, qr, dist.group.WORLD)
            ok &= bool((L == 100.0 * i + qr).all()) and int(qs[0]) == i
            ok &= bool((env.U == 100.0 * i + e).all()) and bool(env.dead.all()) and int(est[0]) == i + 50
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_four_gloo_ranks_share_factors_from_their_owners():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_share_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert all(ok for _, ok in out), out


def test_measure_pieces_are_assigned_once_and_balanced():
    from lookatmyquant_b200.measure import assign_pieces, pieces
    items = pieces(range(32), 32)
    assert len(items) == 224  # the config-4 sweep: 7 linear pieces a layer
    for world in (1, 2, 3, 4, 8):
        owned = assign_pieces(items, 32, world)
        flat = sorted(k for o in owned for k in o)
        assert flat == list(range(len(items)))
        assert assign_pieces(items, 32, world) == owned  # every rank computes the same split
        cost = [sum(32 - items[k][0] + 1 for k in o) for o in owned]
        assert max(cost) - min(cost) <= 33  # within one piece's cost


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lookatmyquant_b200.measure import assign_pieces, gather_records, pieces
        items = pieces(range(3), 3)
        order = [f"{i}.{name}" for i, _, _, _, name in items]
        mine = assign_pieces(items, 3, world)[rank]
        recs = [{"item": order[k], "option": o, "dkl": float(k)} for k in mine for o in ("tr2", "tr3")]
        res = gather_records({"records": recs, "seconds in probes": 1.0 + rank, "probes": len(recs)},
                             dist.group.WORLD, order)
        q.put((rank, [r["item"] for r in res["records"]], res["probes"], res["seconds in probes"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_measure_records_gather_in_sweep_order(world):
    """The ranks' records come back on every rank in the single-rank sweep order, with the job's probe count and
    the slowest rank's time."""
    from lookatmyquant_b200.measure import pieces
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    items = pieces(range(3), 3)
    want = [f"{i}.{name}" for i, _, _, _, name in items for _ in ("tr2", "tr3")]
    for rank, got, probes, slowest in out:
        assert got == want and probes == len(want) and slowest == float(world)
