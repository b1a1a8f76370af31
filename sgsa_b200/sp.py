"""Sequence-parallel SGSA layer forward for long contexts (one process per GPU).

The reference has no multi-GPU path for this layer (its ops README lists
context parallelism as missing); this follows the affine-scan structure of the
chunked delta rule.  Rank r holds the contiguous token slice
[r T/N, (r+1) T/N) of every input.

Delta stage (two passes, no data-path collective but one small all-gather):
  1. local prep + scan from a zero state -> h_r, the slice's final state; a
     second scan in transition mode (v taken as zero, initial state I) ->
     M_r, the slice's state transition, so that S_out = M_r S_in + h_r;
  2. all-gather (M_r, h_r) [B, H, D, D] fp32, fold S_in(r) = M_{r-1} S_in(r-1)
     + h_{r-1}; rescan the slice from S_in(r) reusing the prep operands.
Indexer + attention: causal work grows with the query position, so the
128-query tiles are dealt to the ranks in a zigzag order (round of 2N tiles: r
and 2N-1-r) which balances it.  The keys (k, v, ik) of the whole sequence are
all-gathered; the query rows (q, iq) of each rank's zigzag tiles come from
their owners by an all-to-all (1/N of the sequence per rank); each rank's tile
outputs (fp32) go back to their owners by the reverse all-to-all, and the
owner applies the gate with its delta output.

``sp_layer_fwd`` runs on a torch.distributed NCCL group; ``sp_layer_fwd_emulated``
runs the same phases for N virtual ranks on one GPU (the tests use it).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import _lib, ops

Tensor = torch.Tensor
TILE = 128


def zigzag_tiles(n_tiles: int, world: int, rank: int) -> List[int]:
    """Query tiles of `rank`, heaviest first: tile i goes to rank p if p < N else
    2N-1-p, with p = i mod 2N."""
    mine = []
    for i in range(n_tiles):
        p = i % (2 * world)
        if (p if p < world else 2 * world - 1 - p) == rank:
            mine.append(i)
    return sorted(mine, reverse=True)


def fold_states(Ms: Sequence[Tensor], hs: Sequence[Tensor], s0: Optional[Tensor] = None):
    """Initial states of the slices: S_in(0) = s0 (or 0), S_in(r) = M_{r-1} S_in(r-1) + h_{r-1}."""
    s = torch.zeros_like(hs[0]) if s0 is None else s0.to(hs[0].dtype)
    out = [s]
    for r in range(len(hs) - 1):
        s = torch.matmul(Ms[r], s) + hs[r]
        out.append(s)
    return out


class _Delta:
    """The local delta stage of one slice, keeping its prep workspace."""

    def __init__(self, q, k, v, beta, gamma):
        self.args = [t.contiguous() for t in (q, k, v, beta, gamma)]
        B, T, H, D = q.shape
        self.shape = (B, T, H, D)
        lib = _lib.load()
        self.ws = torch.empty(max(lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, 0), 256),
                              dtype=torch.uint8, device=q.device)
        self.dt = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F32

    def _run(self, s0, flags, want_o):
        B, T, H, D = self.shape
        q = self.args[0]
        o = torch.empty(B, T, H, D, device=q.device, dtype=torch.float32) if want_o else \
            torch.empty(1, device=q.device, dtype=torch.float32)
        sT = torch.empty(B, H, D, D, device=q.device, dtype=torch.float32)
        flags |= _lib.FLAG_STORE_FINAL | _lib.FLAG_OUT_F32
        if s0 is not None:
            flags |= _lib.FLAG_HAS_INIT
        st = _lib.load().sgsa_chunk_fwd(*[t.data_ptr() for t in self.args], None, None, None,
                                         None if s0 is None else s0.data_ptr(), o.data_ptr(),
                                         sT.data_ptr(), B, T, H, D, self.dt, 64, flags,
                                         self.ws.data_ptr(), self.ws.numel(),
                                         torch.cuda.current_stream(q.device).cuda_stream)
        _lib.check(st, "sgsa_chunk_fwd")
        return o, sT

    def pass1(self):
        """(h, M): final state from zero and the slice transition."""
        B, T, H, D = self.shape
        _, h = self._run(None, 0, True)
        eye = torch.eye(D, device=self.args[0].device).expand(B, H, D, D).contiguous()
        _, M = self._run(eye, _lib.FLAG_TRANSITION | _lib.FLAG_REUSE_PREP, False)
        return h, M

    def pass2(self, s_in):
        """(o_delta fp32, final state) of the slice from its true initial state."""
        return self._run(s_in.contiguous(), _lib.FLAG_REUSE_PREP, True)


def _attention_partial(q, k, v, iq, ik, top_k, tiles, thr, out):
    """Indexer + attention (fp32, no gate) of the given query tiles into `out`."""
    qt = torch.tensor(tiles, dtype=torch.int32, device=q.device)
    ops.indexer_thresholds(iq, ik, top_k, q_tiles=qt, out=thr)
    ops.sparse_attn_thresholds(q, k, v, iq, ik, thr, q_tiles=qt, out=out)
    return out


def sp_layer_fwd_emulated(q, k, v, beta, gamma, iq, ik, mix, top_k, world: int,
                          output_final_state: bool = False):
    """The sequence-parallel algorithm for `world` virtual ranks on one GPU (full
    inputs [B, T, H, *]; T divisible by world * 128)."""
    B, T, H, D = q.shape
    Tl = T // world
    if Tl * world != T or Tl % TILE:
        raise ValueError("T must split into whole 128-token tiles per rank")
    sl = lambda t, r: t[:, r * Tl:(r + 1) * Tl]
    deltas = [_Delta(sl(q, r), sl(k, r), sl(v, r), sl(beta, r), sl(gamma, r)) for r in range(world)]
    hm = [d.pass1() for d in deltas]
    s_in = fold_states([m for _, m in hm], [h for h, _ in hm])
    od = [d.pass2(s) for d, s in zip(deltas, s_in)]
    n_tiles = T // TILE
    thr = torch.zeros(B, H, T, 4, device=q.device, dtype=torch.int32)
    o_s = torch.zeros(B, T, H, D, device=q.device, dtype=torch.float32)
    for r in range(world):  # each rank fills its zigzag tiles; the sum is the reduce-scatter
        part = torch.zeros_like(o_s)
        _attention_partial(q, k, v, iq, ik, top_k, zigzag_tiles(n_tiles, world, r), thr, part)
        o_s += part
    outs = [ops.gate_mix(sl(o_s, r), od[r][0], sl(mix, r), q.dtype) for r in range(world)]
    out = torch.cat(outs, dim=1)
    return (out, od[-1][1]) if output_final_state else out


def _gather_seq(x: Tensor, world: int, group) -> Tensor:
    """All-gather of per-rank slices [B, Tl, ...] into [B, world * Tl, ...]."""
    import torch.distributed as dist

    buf = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(buf, x.contiguous(), group=group)
    return buf.transpose(0, 1).reshape(x.shape[0], world * x.shape[1], *x.shape[2:])


class ExchangePlan:
    """Which 128-query tiles move where for the zigzag split.

    Rank r owns the contiguous tiles [r P, (r+1) P) (P = n_tiles / N) and computes
    the attention of its zigzag tiles Z_r.  Before the attention every owner sends
    the query rows (q, iq) of the tiles in Z_s to rank s; after it every rank sends
    its tiles' outputs back to their owners.  Both are all-to-all exchanges of whole
    tiles, 1/N of the sequence per rank, in these orders:
      ``work``       Z_r ascending -- grouped by owner, since owners are ascending;
      ``work_count`` tiles of Z_r per owner;
      ``own``        the tiles of r's slice that each rank s computes, s = 0 .. N-1;
      ``own_count``  their number per rank s.
    """

    def __init__(self, n_tiles: int, world: int, rank: int):
        if n_tiles % world:
            raise ValueError("the tiles must split evenly over the ranks")
        per = n_tiles // world
        self.per, self.rank, self.world = per, rank, world
        self.work = sorted(zigzag_tiles(n_tiles, world, rank))
        self.work_count = [sum(1 for t in self.work if t // per == o) for o in range(world)]
        self.own, self.own_count = [], []
        for s in range(world):
            ts = sorted(t for t in zigzag_tiles(n_tiles, world, s) if t // per == rank)
            self.own += ts
            self.own_count.append(len(ts))

    def rows(self, tiles, local: bool, device=None) -> Tensor:
        """Token rows of `tiles` (global positions, or positions in this rank's slice)."""
        off = self.rank * self.per * TILE if local else 0
        r = torch.tensor([t * TILE + i - off for t in tiles for i in range(TILE)], dtype=torch.long)
        return r if device is None else r.to(device)


def _all_to_all_rows(x: Tensor, send_rows: Tensor, send_counts, recv_rows: Tensor, recv_counts,
                     out: Tensor, group) -> None:
    """out[:, recv_rows] = the rows that the other ranks send of their x[:, send_rows]
    (dim 1 is the token dim); counts are in tiles."""
    import torch.distributed as dist

    send = x.index_select(1, send_rows).transpose(0, 1).contiguous()
    recv = torch.empty((recv_rows.numel(),) + (x.shape[0],) + tuple(x.shape[2:]), dtype=x.dtype,
                       device=x.device)
    dist.all_to_all_single(recv, send, [c * TILE for c in recv_counts],
                           [c * TILE for c in send_counts], group=group)
    out.index_copy_(1, recv_rows, recv.transpose(0, 1))


_delta_streams = {}
_plans = {}


def sp_layer_fwd(q, k, v, beta, gamma, iq, ik, mix, top_k, group=None,
                 output_final_state: bool = False, timings: Optional[dict] = None):
    """Sequence-parallel layer forward on an NCCL process group.  Inputs are this
    rank's token slice [B, Tl, H, *] (Tl a multiple of 128, equal on every rank);
    returns this slice's output (and the final state of the whole sequence on
    every rank if asked for).  ``timings`` (a dict) receives CUDA-event pairs per
    phase, to be read after a synchronisation with ``phase_ms``."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Tl, H, D = q.shape
    T = Tl * world
    dev = q.device
    comp = torch.cuda.current_stream(dev)
    dstream = _delta_streams.get(dev.index)
    if dstream is None:
        dstream = _delta_streams[dev.index] = torch.cuda.Stream(dev)
    key = (T // TILE, world, rank, dev.index)
    plan = _plans.get(key)
    if plan is None:
        p = ExchangePlan(T // TILE, world, rank)
        plan = _plans[key] = (p, p.rows(p.work, False, dev), p.rows(p.own, True, dev),
                              torch.tensor(p.work, dtype=torch.int32, device=dev))
    p, work_rows, own_rows, work_tiles = plan
    ev = (lambda name, st: _mark(timings, name, st)) if timings is not None else (lambda *a: None)

    # All collectives of a process group run in issue order on one NCCL stream, so the
    # key all-gather and the query all-to-all are issued before the delta stage's state
    # all-gather, which waits for the first delta pass: issued after it, they would
    # wait for that pass as well.
    start = torch.cuda.Event()
    start.record(comp)
    # keys of the whole sequence; queries only of this rank's zigzag tiles
    ev("key_allgather", comp)
    fk, fv, fik = [_gather_seq(t, world, group) for t in (k, v, ik)]
    ev("query_alltoall", comp)
    fq = torch.zeros(B, T, H, D, device=dev, dtype=q.dtype)  # zero rows keep max|q| exact
    fiq = torch.empty(B, T, iq.shape[2], iq.shape[3], device=dev, dtype=iq.dtype)
    _all_to_all_rows(q, own_rows, p.own_count, work_rows, p.work_count, fq, group)
    _all_to_all_rows(iq, own_rows, p.own_count, work_rows, p.work_count, fiq, group)
    # the delta stage runs on its own stream, beside the exchanges, the indexer and
    # the attention; it only joins at the gate
    dstream.wait_event(start)
    with torch.cuda.stream(dstream):
        ev("delta_pass1", dstream)
        delta = _Delta(q, k, v, beta, gamma)
        h, M = delta.pass1()
        hm = torch.stack([h, M])
        ev("state_allgather", dstream)
        allhm = torch.empty((world,) + tuple(hm.shape), dtype=hm.dtype, device=dev)
        dist.all_gather_into_tensor(allhm, hm, group=group)
        s_in = fold_states([allhm[r, 1] for r in range(world)],
                           [allhm[r, 0] for r in range(world)])
        ev("delta_pass2", dstream)
        o_delta, s_last = delta.pass2(s_in[rank])
        ev("delta_end", dstream)
    ev("indexer", comp)
    thr = torch.empty(B, iq.shape[2], T, 4, device=dev, dtype=torch.int32)
    ops.indexer_thresholds(fiq, fik, top_k, q_tiles=work_tiles.flip(0), out=thr)
    ev("attention", comp)
    o_s = torch.empty(B, T, H, D, device=dev, dtype=torch.float32)  # only the work tiles are written
    ops.sparse_attn_thresholds(fq, fk, fv, fiq, fik, thr, q_tiles=work_tiles.flip(0), out=o_s)
    ev("output_alltoall", comp)
    mine = torch.empty(B, Tl, H, D, device=dev, dtype=torch.float32)
    _all_to_all_rows(o_s, work_rows, p.work_count, own_rows, p.own_count, mine, group)
    ev("gate", comp)
    comp.wait_stream(dstream)
    o_delta.record_stream(comp)
    out = ops.gate_mix(mine, o_delta, mix, q.dtype)
    ev("end", comp)
    if not output_final_state:
        return out
    final = torch.matmul(allhm[world - 1, 1], s_in[world - 1]) + allhm[world - 1, 0]
    return out, final


def _mark(timings: dict, name: str, stream) -> None:
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    timings.setdefault("_order", []).append((name, e))


def phase_ms(timings: dict) -> dict:
    """Per-phase milliseconds from the events of one sp_layer_fwd call (synchronise
    first): each phase lasts until the next mark on the same stream."""
    marks = timings.get("_order", [])
    streams = {}
    for name, e in marks:
        streams.setdefault(name in ("delta_pass1", "state_allgather", "delta_pass2", "delta_end"),
                           []).append((name, e))
    out = {}
    for seq in streams.values():
        for (n0, e0), (_, e1) in zip(seq[:-1], seq[1:]):
            out[n0] = e0.elapsed_time(e1)
    return out
