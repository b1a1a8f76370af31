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
Indexer + attention: the keys (q, k, v, iq, ik) are all-gathered; causal work
grows with the query position, so the 128-query tiles are dealt to the ranks
in a zigzag order (round of 2N tiles: r and 2N-1-r) which balances it; each
rank writes its tiles' attention output (fp32) into a zero buffer, a
reduce-scatter (sum) hands every token's output to its owner, and the owner
applies the gate with its delta output.

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


_delta_streams = {}


def sp_layer_fwd(q, k, v, beta, gamma, iq, ik, mix, top_k, group=None,
                 output_final_state: bool = False):
    """Sequence-parallel layer forward on an NCCL process group.  Inputs are this
    rank's token slice [B, Tl, H, *] (Tl a multiple of 128, equal on every rank);
    returns this slice's output (and the final state of the whole sequence on
    every rank if asked for)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Tl, H, D = q.shape
    T = Tl * world
    comp = torch.cuda.current_stream(q.device)
    dstream = _delta_streams.get(q.device.index)
    if dstream is None:
        dstream = _delta_streams[q.device.index] = torch.cuda.Stream(q.device)
    # the delta stage runs on its own stream, beside the gathers, the indexer and the
    # attention; it only joins at the gate
    dstream.wait_stream(comp)
    # keys for the attention (the collective makes the compute stream wait for it)
    full = [_gather_seq(t, world, group) for t in (q, k, v, iq, ik)]
    with torch.cuda.stream(dstream):
        delta = _Delta(q, k, v, beta, gamma)
        h, M = delta.pass1()
        hm = torch.stack([h, M])
        allhm = torch.empty((world,) + tuple(hm.shape), dtype=hm.dtype, device=hm.device)
        dist.all_gather_into_tensor(allhm, hm, group=group)
        s_in = fold_states([allhm[r, 1] for r in range(world)],
                           [allhm[r, 0] for r in range(world)])
        o_delta, s_last = delta.pass2(s_in[rank])
    fq, fk, fv, fiq, fik = full
    thr = torch.empty(B, H, T, 4, device=q.device, dtype=torch.int32)
    o_s = torch.zeros(B, T, H, D, device=q.device, dtype=torch.float32)
    _attention_partial(fq, fk, fv, fiq, fik, top_k, zigzag_tiles(T // TILE, world, rank), thr, o_s)
    # every token's attention output to its owner (only one rank wrote it)
    o_parts = o_s.view(B, world, Tl, H, D).transpose(0, 1).contiguous()
    mine = torch.empty(B, Tl, H, D, device=q.device, dtype=torch.float32)
    dist.reduce_scatter_tensor(mine, o_parts, group=group)
    comp.wait_stream(dstream)
    o_delta.record_stream(comp)
    out = ops.gate_mix(mine, o_delta, mix, q.dtype)
    if not output_final_state:
        return out
    final = torch.matmul(allhm[world - 1, 1], s_in[world - 1]) + allhm[world - 1, 0]
    return out, final
