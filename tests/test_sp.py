"""Sequence parallelism: host logic on CPU (world-size-2 gloo ranks, CPU oracle
for the per-slice states) and the full algorithm emulated on one GPU."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from sgsa_b200 import sp


def test_zigzag_tiles_partition_and_balance():
    n, world = 512, 8
    tiles = [sp.zigzag_tiles(n, world, r) for r in range(world)]
    flat = sorted(t for ts in tiles for t in ts)
    assert flat == list(range(n))
    work = [sum(t + 1 for t in ts) for ts in tiles]  # causal work ~ tile index
    assert max(work) / (sum(work) / world) < 1.01
    assert all(ts == sorted(ts, reverse=True) for ts in tiles)


def _slice_states(x, t0, t1):
    """(h, M) of a token slice from the CPU oracle: final state from zero, and the
    transition (v = 0, initial state I)."""
    B, T, H, D = x["q"].shape
    sl = {n: t[:, t0:t1] for n, t in x.items()}
    _, h = oracle.sgsa_recurrent(sl["q"], sl["k"], sl["v"], sl["beta"], sl["gamma"])
    eye = np.broadcast_to(np.eye(D, dtype=np.float32), (B, H, D, D)).copy()
    _, m = oracle.sgsa_recurrent(sl["q"], sl["k"], 0 * sl["v"], sl["beta"], sl["gamma"],
                                 initial_state=eye)
    return torch.from_numpy(h), torch.from_numpy(m)


def _inputs():
    g = torch.Generator().manual_seed(0)
    B, T, H, D = 1, 96, 2, 16
    r = lambda *s: torch.randn(*s, generator=g)
    return dict(q=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
                k=torch.nn.functional.normalize(r(B, T, H, D), dim=-1), v=r(B, T, H, D),
                beta=torch.sigmoid(r(B, T, H)), gamma=0.9 + 0.1 * torch.rand(B, T, H, generator=g))


def _rank_main(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x = _inputs()
    T = x["q"].shape[1]
    tl = T // world
    h, m = _slice_states(x, rank * tl, (rank + 1) * tl)
    hs = [torch.empty_like(h) for _ in range(world)]
    ms = [torch.empty_like(m) for _ in range(world)]
    dist.all_gather(hs, h)
    dist.all_gather(ms, m)
    s_in = sp.fold_states(ms, hs)[rank]
    # this rank's slice from its folded initial state must equal the full sequence
    sl = {n: t[:, rank * tl:(rank + 1) * tl] for n, t in x.items()}
    o, _ = oracle.sgsa_recurrent(sl["q"], sl["k"], sl["v"], sl["beta"], sl["gamma"],
                                 initial_state=s_in.numpy())
    full, _ = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"])
    result[rank] = oracle.rel_l2(o, full[:, rank * tl:(rank + 1) * tl])
    dist.destroy_process_group()


def test_state_handoff_two_gloo_ranks():
    world = 2
    result = mp.Manager().dict()
    mp.spawn(_rank_main, args=(world, 29611, result), nprocs=world, join=True)
    assert all(result[r] < 1e-5 for r in range(world)), dict(result)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_sp_emulated_matches_single_gpu(world):
    from sgsa_b200 import ops
    from sgsa_b200.inputs import CONFIGS, make_inputs

    cfg = CONFIGS["b200_bf16"].scaled(name="sp", B=1, T=2048, H=2, top_k=256)
    x = {n: t.cuda() for n, t in make_inputs(cfg, seed=8).items()}
    args = (x["q"], x["k"], x["v"], x["beta"], x["gamma"], x["iq"], x["ik"], x["mix"], cfg.top_k)
    ref, st_ref = ops.sgsa_layer_fwd(*args, output_final_state=True)
    got, st = sp.sp_layer_fwd_emulated(*args, world=world, output_final_state=True)
    assert oracle.rel_l2(got.float().cpu().numpy(), ref.float().cpu().numpy()) < 2e-3
    assert oracle.rel_l2(st.cpu().numpy(), st_ref.cpu().numpy()) < 2e-3


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_plan_moves_every_tile_once(world):
    """Simulate the two all-to-alls of the plan: every rank gets the query rows of
    exactly its zigzag tiles, and every owner gets back the outputs of exactly its
    own tiles, each once."""
    n = 64 * world
    plans = [sp.ExchangePlan(n, world, r) for r in range(world)]
    for r, p in enumerate(plans):
        assert sum(p.work_count) == len(p.work) == n // world
        assert sum(p.own_count) == len(p.own) == n // world
    # query exchange: owner o sends its `own` tiles, split by own_count, to ranks s
    for r, p in enumerate(plans):
        got = []
        for o in range(world):
            po = plans[o]
            start = sum(po.own_count[:r])
            got += po.own[start:start + po.own_count[r]]
        assert got == p.work  # arrives grouped by owner, ascending = work order
    # output exchange: rank s sends its `work` tiles, split by work_count, to owners
    for r, p in enumerate(plans):
        got = []
        for s in range(world):
            ps = plans[s]
            start = sum(ps.work_count[:r])
            got += ps.work[start:start + ps.work_count[r]]
        assert got == p.own
        assert sorted(got) == list(range(r * n // world, (r + 1) * n // world))


def _a2a_main(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n_tiles, B, H = 4 * world, 2, 3
    T = n_tiles * sp.TILE
    Tl = T // world
    full = torch.arange(B * T * H, dtype=torch.float32).reshape(B, T, H, 1)
    mine = full[:, rank * Tl:(rank + 1) * Tl].contiguous()
    p = sp.ExchangePlan(n_tiles, world, rank)
    work_rows, own_rows = p.rows(p.work, False), p.rows(p.own, True)
    # queries: owners send, each rank receives its work tiles at their global rows
    fq = torch.zeros(B, T, H, 1)
    sp._all_to_all_rows(mine, own_rows, p.own_count, work_rows, p.work_count, fq, None)
    ok = torch.equal(fq[:, work_rows], full[:, work_rows])
    # outputs: each rank returns its work rows (of a full-size buffer) to their owners
    back = torch.empty(B, Tl, H, 1)
    sp._all_to_all_rows(fq, work_rows, p.work_count, own_rows, p.own_count, back, None)
    result[rank] = ok and torch.equal(back, mine)
    dist.destroy_process_group()


def test_row_all_to_all_two_gloo_ranks():
    world = 2
    result = mp.Manager().dict()
    mp.spawn(_a2a_main, args=(world, 29631, result), nprocs=world, join=True)
    assert all(result[r] for r in range(world)), dict(result)
