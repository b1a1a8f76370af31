"""Host-side operators of the SGSA layer forward on B200.

``chunk_sgsa`` keeps the signature, argument meaning and return of the
reference's public op (modelings/sgsa_ops/chunk.py:104-148), so a caller can
swap the import.  The other functions expose the rest of the layer's hot path
(indexer top-k, sparse attention + gate, the fused composite) at op level.

Every op runs the CUDA kernels of libsgsa_b200.so on the tensors' device and
current stream.  There is no CPU or Python fallback: CPU tensors, unsupported
dtypes or shapes raise.  The forward pass only is implemented; asking for a
gradient through these ops raises.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib

Tensor = torch.Tensor

_DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _dtype_code(t: Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"sgsa_b200 supports float32 and bfloat16 inputs, got {t.dtype}")
    return _DT[t.dtype]


def _dev(t: Tensor, name: str) -> Tensor:
    if not isinstance(t, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (sgsa_b200 has no CPU path)")
    return t


def _ptr(t: Optional[Tensor]):
    return None if t is None else t.data_ptr()


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _no_grad_check(*ts):
    if torch.is_grad_enabled() and any(isinstance(t, Tensor) and t.requires_grad for t in ts):
        raise NotImplementedError("sgsa_b200 implements the SGSA forward only (no backward)")


def _workspace(nbytes: int, device) -> Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


_layer_ws = {}


def _layer_workspace(nbytes: int, device) -> Tensor:
    """The layer's workspace, kept across calls per (device, stream) and grown when a
    call needs more.  Calls on one stream are ordered, so reusing it is safe; calls
    on another stream get their own."""
    dev = torch.device(device)
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    ws = _layer_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        _layer_ws.pop(key, None)
        ws = _layer_ws[key] = _workspace(nbytes, dev)
    return ws


def release_workspaces() -> None:
    """Drop the cached layer workspaces (their memory returns to torch's allocator)."""
    _layer_ws.clear()


def chunk_sgsa(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    beta: Tensor,
    gamma: Tensor,
    sparse_k: Optional[Tensor] = None,
    sparse_v: Optional[Tensor] = None,
    alpha: Optional[Tensor] = None,
    initial_state: Optional[Tensor] = None,
    chunk_size: int = 64,
    output_final_state: bool = False,
    use_triton: bool = True,
) -> Tuple[Tensor, Optional[Tensor]]:
    """Chunked Sparse-Guided State Attention core (forward).

    Same contract as the reference ``chunk_sgsa`` (modelings/sgsa_ops/chunk.py:104-148):
    q, k, v, sparse_k, sparse_v are ``[B, T, H, D]``; beta, gamma, alpha are
    ``[B, T, H]``; initial_state is ``[B, H, D, D]``; returns ``o`` in q.dtype
    and the final state in q.dtype (or None).  The sparse write is active when
    all three of sparse_k, sparse_v and alpha are given.  The device path
    always tiles by 64 tokens: ``chunk_size`` only has to be positive (the
    result does not depend on it beyond rounding), and ``use_triton`` is
    accepted for signature compatibility -- there is no other backend.
    """
    del use_triton
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    for n, t in (("q", q), ("k", k), ("v", v), ("beta", beta), ("gamma", gamma)):
        _dev(t, n)
    _no_grad_check(q, k, v, beta, gamma, sparse_k, sparse_v, alpha, initial_state)
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must share the shape [B, T, H, D]")
    B, T, H, D = q.shape
    if beta.shape != (B, T, H) or gamma.shape != (B, T, H):
        raise ValueError("beta and gamma must be [B, T, H]")
    dt = _dtype_code(q)
    has_sparse = sparse_k is not None and sparse_v is not None and alpha is not None
    flags = 0
    if has_sparse:
        if sparse_k.shape != q.shape or sparse_v.shape != q.shape or alpha.shape != (B, T, H):
            raise ValueError("sparse_k/sparse_v must be [B, T, H, D] and alpha [B, T, H]")
        flags |= _lib.FLAG_HAS_SPARSE
    cast = lambda t: None if t is None else t.to(device=q.device, dtype=q.dtype).contiguous()
    q_, k_, v_ = q.contiguous(), cast(k), cast(v)
    beta_, gamma_ = cast(beta), cast(gamma)
    sk_, sv_, al_ = (cast(sparse_k), cast(sparse_v), cast(alpha)) if has_sparse else (None,) * 3
    s0 = None
    if initial_state is not None:
        if initial_state.shape != (B, H, D, D):
            raise ValueError("initial_state must be [B, H, D, D]")
        s0 = initial_state.to(device=q.device, dtype=torch.float32).contiguous()
        flags |= _lib.FLAG_HAS_INIT
    o = torch.empty_like(q_)
    sT = None
    if output_final_state:
        sT = torch.empty(B, H, D, D, device=q.device, dtype=torch.float32)
        flags |= _lib.FLAG_STORE_FINAL
    lib = _lib.load()
    wsb = lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, flags)
    ws = _workspace(wsb, q.device)
    st = lib.sgsa_chunk_fwd(_ptr(q_), _ptr(k_), _ptr(v_), _ptr(beta_), _ptr(gamma_), _ptr(sk_),
                            _ptr(sv_), _ptr(al_), _ptr(s0), _ptr(o), _ptr(sT), B, T, H, D, dt, 64,
                            flags, _ptr(ws), ws.numel(), _stream(q))
    _lib.check(st, "sgsa_chunk_fwd", q)
    if sT is not None:
        sT = sT.to(q.dtype)
    return o, sT


def chunk_sgsa_fp32_state(q, k, v, beta, gamma, initial_state=None, sparse_k=None,
                          sparse_v=None, alpha=None, out_f32: bool = False):
    """Like ``chunk_sgsa`` but returns the final state in float32 (for hand-off
    between sequence shards) and optionally a float32 ``o``."""
    B, T, H, D = q.shape
    _dev(q, "q")
    dt = _dtype_code(q)
    has_sparse = sparse_k is not None and sparse_v is not None and alpha is not None
    flags = _lib.FLAG_STORE_FINAL | (_lib.FLAG_OUT_F32 if out_f32 else 0)
    flags |= _lib.FLAG_HAS_SPARSE if has_sparse else 0
    cast = lambda t: None if t is None else t.to(dtype=q.dtype).contiguous()
    s0 = None
    if initial_state is not None:
        s0 = initial_state.to(dtype=torch.float32).contiguous()
        flags |= _lib.FLAG_HAS_INIT
    o = torch.empty(q.shape, device=q.device, dtype=torch.float32 if out_f32 else q.dtype)
    sT = torch.empty(B, H, D, D, device=q.device, dtype=torch.float32)
    lib = _lib.load()
    ws = _workspace(lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, flags), q.device)
    args = [cast(t) for t in (q, k, v, beta, gamma)]
    sp = [cast(t) for t in (sparse_k, sparse_v, alpha)] if has_sparse else [None] * 3
    st = lib.sgsa_chunk_fwd(*[_ptr(t) for t in args], *[_ptr(t) for t in sp], _ptr(s0), _ptr(o),
                            _ptr(sT), B, T, H, D, dt, 64, flags, _ptr(ws), ws.numel(),
                            _stream(q))
    _lib.check(st, "sgsa_chunk_fwd", q)
    return o, sT


def indexer_topk(iq: Tensor, ik: Tensor, top_k: int) -> Tensor:
    """Causal per-head top-k of ``iq . ik`` -> int32 ``[B, H, T, top_k]``.

    Row t holds the min(top_k, t+1) selected key positions in ascending order,
    ties broken toward the lower position, padded with -1 (the selection of
    modelings/hybrid_dense_delta_topk.py:344-349 / modeling_sgsa.py:144-165).
    """
    _dev(iq, "iq"), _dev(ik, "ik")
    if iq.dim() != 4 or ik.shape != iq.shape:
        raise ValueError("iq and ik must share the shape [B, T, H, DI]")
    if top_k <= 0:
        raise ValueError("top_k must be positive")
    B, T, H, DI = iq.shape
    dt = _dtype_code(iq)
    iq_, ik_ = iq.contiguous(), ik.to(iq.dtype).contiguous()
    out = torch.empty(B, H, T, top_k, device=iq.device, dtype=torch.int32)
    st = _lib.load().sgsa_indexer_topk(_ptr(iq_), _ptr(ik_), _ptr(out), B, T, H, DI, top_k, dt,
                                        _stream(iq))
    _lib.check(st, "sgsa_indexer_topk", iq)
    return out


def topk_select(scores: Tensor, valid: Tensor, top_k: int) -> Tensor:
    """Row top-k of float32 ``scores [R, S]`` over columns ``[0, valid[r])``."""
    _dev(scores, "scores")
    if scores.dim() != 2:
        raise ValueError("scores must be [R, S]")
    R, S = scores.shape
    sc = scores.to(torch.float32).contiguous()
    val = valid.to(device=scores.device, dtype=torch.int32).contiguous()
    if val.shape != (R,):
        raise ValueError("valid must be [R]")
    out = torch.empty(R, top_k, device=scores.device, dtype=torch.int32)
    st = _lib.load().sgsa_topk_select(_ptr(sc), _ptr(val), _ptr(out), R, S, top_k,
                                       _stream(scores))
    _lib.check(st, "sgsa_topk_select", scores)
    return out


def sparse_attn_mix(q: Tensor, k: Tensor, v: Tensor, indices: Tensor,
                    o_delta: Optional[Tensor] = None, mix: Optional[Tensor] = None,
                    scale: Optional[float] = None) -> Tensor:
    """Softmax attention of each query over its selected rows, then the gate
    ``mix * o_s + (1 - mix) * o_delta`` (modelings/hybrid_dense_delta_topk.py:350-356,389-390).

    ``indices`` is int32 ``[B, H, T, K]`` as produced by ``indexer_topk``;
    ``mix`` is ``[B, T, H, D]`` or ``[B, T, H]``; ``o_delta`` ``[B, T, H, D]``.
    """
    for n, t in (("q", q), ("k", k), ("v", v), ("indices", indices)):
        _dev(t, n)
    B, T, H, D = q.shape
    if indices.dim() != 4 or indices.shape[0] != B or indices.shape[2] != T or \
            indices.shape[1] not in (1, H):
        raise ValueError("indices must be [B, H, T, K] or [B, 1, T, K]")
    idx_heads = indices.shape[1]
    K = indices.shape[-1]
    dt = _dtype_code(q)
    cast = lambda t: None if t is None else t.to(q.dtype).contiguous()
    q_, k_, v_ = q.contiguous(), cast(k), cast(v)
    ix = indices.to(torch.int32).contiguous()
    od = None if o_delta is None else o_delta.to(torch.float32).contiguous()
    mx = cast(mix) if o_delta is not None else None
    per_channel = int(mx is not None and mx.dim() == 4)
    out = torch.empty_like(q_)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    st = _lib.load().sgsa_sparse_attn_mix(_ptr(q_), _ptr(k_), _ptr(v_), _ptr(ix), _ptr(od),
                                           _ptr(mx), _ptr(out), B, T, H, D, K, idx_heads, sc,
                                           per_channel, dt, _stream(q))
    _lib.check(st, "sgsa_sparse_attn_mix", q)
    return out


def sgsa_layer_fwd(q: Tensor, k: Tensor, v: Tensor, beta: Tensor, gamma: Tensor, iq: Tensor,
                   ik: Tensor, mix: Tensor, top_k: int, initial_state: Optional[Tensor] = None,
                   output_final_state: bool = False, return_indices: bool = False):
    """Fused SGSA layer core: delta stage + indexer top-k + sparse attention + gate.

    Returns ``out`` (q.dtype), then the float32 final state if requested and
    the int32 indices if requested.
    """
    for n, t in (("q", q), ("k", k), ("v", v), ("beta", beta), ("gamma", gamma), ("iq", iq),
                 ("ik", ik), ("mix", mix)):
        _dev(t, n)
    _no_grad_check(q, k, v, beta, gamma, iq, ik, mix, initial_state)
    B, T, H, D = q.shape
    DI = iq.shape[-1]
    idx_heads = iq.shape[2]
    if idx_heads not in (1, H) or ik.shape != iq.shape:
        raise ValueError("iq and ik must be [B, T, H, DI] or [B, T, 1, DI] (shared indexer)")
    dt = _dtype_code(q)
    cast = lambda t: t.to(q.dtype).contiguous()
    args = [q.contiguous()] + [cast(t) for t in (k, v, beta, gamma, iq, ik, mix)]
    per_channel = int(mix.dim() == 4)
    s0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    out = torch.empty_like(args[0])
    sT = torch.empty(B, H, D, D, device=q.device, dtype=torch.float32) if output_final_state else None
    ix = torch.empty(B, idx_heads, T, top_k, device=q.device, dtype=torch.int32) \
        if return_indices else None
    lib = _lib.load()
    ws = _layer_workspace(lib.sgsa_layer_fwd_workspace_size(B, T, H, D, DI, idx_heads, top_k, dt),
                          q.device)
    st = lib.sgsa_layer_fwd(*[_ptr(t) for t in args], _ptr(s0), _ptr(out), _ptr(sT), _ptr(ix),
                            B, T, H, D, DI, idx_heads, top_k, per_channel, dt, _ptr(ws),
                            ws.numel(), _stream(q))
    _lib.check(st, "sgsa_layer_fwd", q)
    res = [out]
    if output_final_state:
        res.append(sT)
    if return_indices:
        res.append(ix)
    return res[0] if len(res) == 1 else tuple(res)


def indexer_thresholds(iq: Tensor, ik: Tensor, top_k: int, return_indices: bool = False,
                       q_tiles: Optional[Tensor] = None, out: Optional[Tensor] = None):
    """Tensor-core indexer (bf16, DI 64/128) returning the exact per-row selection as
    threshold records int32 ``[B, H, T, 4]`` (see include/sgsa_b200.h), plus the
    index rows if asked for.  ``q_tiles`` (int32, heaviest first) restricts the
    work to those 128-query tiles; ``out`` receives the records."""
    _dev(iq, "iq"), _dev(ik, "ik")
    B, T, H, DI = iq.shape
    iq_, ik_ = iq.contiguous(), ik.to(iq.dtype).contiguous()
    thr = out if out is not None else torch.empty(B, H, T, 4, device=iq.device, dtype=torch.int32)
    ix = torch.empty(B, H, T, top_k, device=iq.device, dtype=torch.int32) if return_indices else None
    qt = None if q_tiles is None else q_tiles.to(device=iq.device, dtype=torch.int32).contiguous()
    nt = 0 if qt is None else qt.numel()
    st = _lib.load().sgsa_indexer_thresholds(_ptr(iq_), _ptr(ik_), _ptr(ix), _ptr(thr), _ptr(qt),
                                              nt, B, T, H, DI, top_k, _stream(iq))
    _lib.check(st, "sgsa_indexer_thresholds", iq)
    return (thr, ix) if return_indices else thr


def sparse_attn_thresholds(q, k, v, iq, ik, thresholds, o_delta=None, mix=None, scale=None,
                           q_tiles: Optional[Tensor] = None, out: Optional[Tensor] = None,
                           out_f32: bool = False):
    """Tensor-core sparse attention + gate over the rows selected by ``thresholds``
    (bf16 output, or float32 with ``out_f32``); ``q_tiles`` as for indexer_thresholds."""
    B, T, H, D = q.shape
    DI = iq.shape[-1]
    if out is None:
        out = torch.empty(q.shape, device=q.device,
                          dtype=torch.float32 if out_f32 else q.dtype)
    od = None if o_delta is None else o_delta.to(torch.float32).contiguous()
    mx = None if mix is None else mix.to(q.dtype).contiguous()
    per_channel = int(mx is not None and mx.dim() == 4)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    qt = None if q_tiles is None else q_tiles.to(device=q.device, dtype=torch.int32).contiguous()
    nt = 0 if qt is None else qt.numel()
    norms = torch.empty(2 * B * H, device=q.device, dtype=torch.int32)  # max |q|^2, |k|^2 per head
    st = _lib.load().sgsa_sparse_attn_thresholds(
        _ptr(q), _ptr(k), _ptr(v), _ptr(iq), _ptr(ik), _ptr(thresholds), _ptr(qt), nt, _ptr(od),
        _ptr(mx), _ptr(out), B, T, H, D, DI, iq.shape[2], sc, per_channel,
        int(out.dtype == torch.float32), _ptr(norms), _stream(q))
    _lib.check(st, "sgsa_sparse_attn_thresholds", q)
    return out


_copy_streams = {}


def sgsa_layer_fwd_from_host(q, k, v, beta, gamma, iq, ik, mix, top_k, device=None,
                             out: Optional[Tensor] = None):
    """``sgsa_layer_fwd`` for inputs in host memory: returns the output in host memory.

    The host->device copies run on a copy stream in the order the stages consume
    them (indexer vectors, then q/k/v/beta/gamma, then the mix), so they overlap the
    indexer and the delta stage.  They are ordered after the previous call's copies,
    not after earlier work of the current stream, so that back-to-back calls overlap
    one call's copies with the previous call's kernels; a host input written by an
    asynchronous device->host copy must be synchronised before the call.  The output
    returns batch by batch on a second copy stream (the link is full duplex), and the
    current stream waits for it before the call returns, so a synchronisation of the
    current stream makes ``out`` valid.  Host tensors should be pinned for the copies
    to be asynchronous.
    """
    dev = torch.device(device) if device is not None else torch.device("cuda",
                                                                        torch.cuda.current_device())
    comp = torch.cuda.current_stream(dev)
    streams = _copy_streams.get(dev.index)
    if streams is None:
        streams = _copy_streams[dev.index] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    cs, os_ = streams
    host = dict(iq=iq, ik=ik, q=q, k=k, v=v, beta=beta, gamma=gamma, mix=mix)
    d, ev = {}, {}
    with torch.cuda.stream(cs):
        for n in ("iq", "ik", "q", "k", "v", "beta", "gamma", "mix"):
            d[n] = host[n].to(dev, non_blocking=True)
            ev[n] = torch.cuda.Event()
            ev[n].record(cs)
    for t in d.values():
        t.record_stream(comp)
    B, T, H, D = q.shape
    DI = iq.shape[-1]
    fused = (q.dtype == torch.bfloat16 and D == 128 and DI == 64)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    if not fused:
        comp.wait_event(ev["mix"])
        res = sgsa_layer_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"],
                             d["mix"], top_k)
        out.copy_(res, non_blocking=True)
        return out
    os_.wait_stream(comp)  # the previous user of `out` has finished with it
    comp.wait_event(ev["ik"])
    thr = indexer_thresholds(d["iq"], d["ik"], top_k)
    comp.wait_event(ev["gamma"])
    od, _ = chunk_sgsa_fp32_state(d["q"], d["k"], d["v"], d["beta"], d["gamma"], out_f32=True)
    comp.wait_event(ev["mix"])
    # attention batch by batch; each batch's output returns while the next one runs
    res = torch.empty_like(d["q"])
    for bi in range(B):
        sl = slice(bi, bi + 1)
        res[sl] = sparse_attn_thresholds(d["q"][sl], d["k"][sl], d["v"][sl], d["iq"][sl],
                                         d["ik"][sl], thr[sl], od[sl], d["mix"][sl])
        done = torch.cuda.Event()
        done.record(comp)
        os_.wait_event(done)
        with torch.cuda.stream(os_):
            out[sl].copy_(res[sl], non_blocking=True)
    res.record_stream(os_)
    comp.wait_stream(os_)
    return out


def fused_recurrent_sgsa(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    beta: Tensor,
    gamma: Tensor,
    sparse_k: Optional[Tensor] = None,
    sparse_v: Optional[Tensor] = None,
    alpha: Optional[Tensor] = None,
    initial_state: Optional[Tensor] = None,
    output_final_state: bool = False,
    use_triton: bool = True,
) -> Tuple[Tensor, Optional[Tensor]]:
    """Token-by-token SGSA forward with the signature of the reference's
    ``fused_recurrent_sgsa`` (modelings/sgsa_ops/recurrent.py:138-175): ``o`` in
    q.dtype and the final state in float32, as its Triton forward returns it
    (recurrent_fwd_triton.py:120-125).  ``use_triton`` is accepted and ignored."""
    del use_triton
    for n, t in (("q", q), ("k", k), ("v", v), ("beta", beta), ("gamma", gamma)):
        _dev(t, n)
    _no_grad_check(q, k, v, beta, gamma, sparse_k, sparse_v, alpha, initial_state)
    B, T, H, D = q.shape
    dt = _dtype_code(q)
    has_sparse = sparse_k is not None and sparse_v is not None and alpha is not None
    cast = lambda t: None if t is None else t.to(device=q.device, dtype=q.dtype).contiguous()
    args = [q.contiguous()] + [cast(t) for t in (k, v, beta, gamma)]
    sp = [cast(t) for t in (sparse_k, sparse_v, alpha)] if has_sparse else [None] * 3
    flags = _lib.FLAG_HAS_SPARSE if has_sparse else 0
    s0 = None
    if initial_state is not None:
        s0 = initial_state.to(device=q.device, dtype=torch.float32).contiguous()
        flags |= _lib.FLAG_HAS_INIT
    o = torch.empty_like(args[0])
    sT = None
    if output_final_state:
        sT = torch.empty(B, H, D, D, device=q.device, dtype=torch.float32)
        flags |= _lib.FLAG_STORE_FINAL
    st = _lib.load().sgsa_recurrent_fwd(*[_ptr(t) for t in args], *[_ptr(t) for t in sp],
                                         _ptr(s0), _ptr(o), _ptr(sT), B, T, H, D, dt, flags,
                                         _stream(q))
    _lib.check(st, "sgsa_recurrent_fwd", q)
    return o, sT


def decode_topk(iq: Tensor, ik_cache: Tensor, n: int, top_k: int) -> Tensor:
    """Top-k of ``iq [B, H, DI]`` against the first ``n`` rows of ``ik_cache
    [B, Tc, H, DI]`` -> int32 ``[B, H, top_k]`` (ascending, ties to the lowest row)."""
    _dev(iq, "iq"), _dev(ik_cache, "ik_cache")
    B, H, DI = iq.shape
    Tc = ik_cache.shape[1]
    out = torch.empty(B, H, top_k, device=iq.device, dtype=torch.int32)
    st = _lib.load().sgsa_decode_topk(_ptr(iq.contiguous()), _ptr(ik_cache), _ptr(out), B, H, Tc,
                                       int(n), DI, top_k, _dtype_code(iq), _stream(iq))
    _lib.check(st, "sgsa_decode_topk", iq)
    return out


def decode_attn_mix(q: Tensor, k_cache: Tensor, v_cache: Tensor, indices: Tensor,
                    o_delta: Optional[Tensor] = None, mix: Optional[Tensor] = None,
                    scale: Optional[float] = None) -> Tensor:
    """Attention of ``q [B, H, D]`` over its selected cache rows, then the gate."""
    B, H, D = q.shape
    Tc = k_cache.shape[1]
    K = indices.shape[-1]
    out = torch.empty_like(q)
    od = None if o_delta is None else o_delta.to(torch.float32).contiguous()
    mx = None if mix is None else mix.to(q.dtype).contiguous()
    per_channel = int(mx is not None and mx.dim() == 3)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    st = _lib.load().sgsa_decode_attn_mix(_ptr(q.contiguous()), _ptr(k_cache), _ptr(v_cache),
                                           _ptr(indices.to(torch.int32).contiguous()), _ptr(od),
                                           _ptr(mx), _ptr(out), B, H, Tc, D, K, sc, per_channel,
                                           _dtype_code(q), _stream(q))
    _lib.check(st, "sgsa_decode_attn_mix", q)
    return out


class DecodeCache:
    """Decode-time state of one SGSA layer: the delta-rule state, the K/V and
    indexer-key caches, and the top-k rows reused between refreshes.

    ``step`` runs one token: recurrent delta step, cache append, indexer top-k
    (recomputed every ``reuse`` steps and on the first step, reused otherwise --
    the top-k reuse studied in experiments/attention_topk_reuse_experiment.md:28-46),
    sparse attention over the selected rows and the gate.
    """

    def __init__(self, k_cache: Tensor, v_cache: Tensor, ik_cache: Tensor, length: int,
                 state: Tensor, top_k: int, reuse: int = 1):
        self.k, self.v, self.ik = k_cache, v_cache, ik_cache
        self.n = int(length)
        self.state = state.to(torch.float32).contiguous()
        self.top_k, self.reuse = int(top_k), max(1, int(reuse))
        self.steps = 0
        self.indices = None

    def step(self, q, k, v, beta, gamma, iq, ik, mix):
        """q, k, v [B, H, D]; beta, gamma [B, H]; iq, ik [B, H, DI]; mix [B, H, D] or [B, H]."""
        B, H, D = q.shape
        if self.n >= self.k.shape[1]:
            raise ValueError("decode cache is full")
        o_d, self.state = chunk_free_recurrent_step(q, k, v, beta, gamma, self.state)
        decode_append(self.k, self.v, self.ik, k, v, ik, self.n)
        self.n += 1
        if self.indices is None or self.steps % self.reuse == 0:
            self.indices = decode_topk(iq, self.ik, self.n, self.top_k)
        self.steps += 1
        return decode_attn_mix(q, self.k, self.v, self.indices, o_d, mix)


def decode_append(k_cache: Tensor, v_cache: Tensor, ik_cache: Tensor, k: Tensor, v: Tensor,
                  ik: Tensor, pos: int) -> None:
    """Row ``pos`` of the [B, Tc, H, *] caches from one token's k, v [B, H, D] and ik
    [B, H, DI], in one launch (the reference grows its caches by torch.cat,
    hybrid_dense_delta_topk.py:226-230)."""
    B, Tc, H, D = k_cache.shape
    DI = ik_cache.shape[-1]
    for n, t in (("k_cache", k_cache), ("v_cache", v_cache), ("ik_cache", ik_cache)):
        _dev(t, n)
        if not t.is_contiguous() or t.dtype != k_cache.dtype:
            raise ValueError(f"{n} must be contiguous and of the caches' dtype")
    cast = lambda t: t.to(k_cache.dtype).contiguous()
    k, v, ik = cast(k), cast(v), cast(ik)
    st = _lib.load().sgsa_decode_append(_ptr(k_cache), _ptr(v_cache), _ptr(ik_cache), _ptr(k),
                                        _ptr(v), _ptr(ik), B, Tc, H, D, DI, pos,
                                        _dtype_code(k_cache), _stream(k_cache))
    _lib.check(st, "sgsa_decode_append", k_cache)


def chunk_free_recurrent_step(q, k, v, beta, gamma, state):
    """One-token delta step: ``(o float32 [B, H, D], new state float32)``."""
    B, H, D = q.shape
    st = torch.empty_like(state)
    o = torch.empty(B, H, D, device=q.device, dtype=torch.float32)
    dt = _dtype_code(q)
    cast = lambda t: t.to(q.dtype).contiguous()
    flags = _lib.FLAG_HAS_INIT | _lib.FLAG_STORE_FINAL | _lib.FLAG_OUT_F32
    rc = _lib.load().sgsa_recurrent_fwd(_ptr(q.contiguous()), _ptr(cast(k)), _ptr(cast(v)),
                                         _ptr(cast(beta)), _ptr(cast(gamma)), None, None, None,
                                         _ptr(state), _ptr(o), _ptr(st), B, 1, H, D, dt, flags,
                                         _stream(q))
    _lib.check(rc, "sgsa_recurrent_fwd", q)
    return o, st


def gate_mix(o_s: Tensor, o_delta: Tensor, mix: Tensor, dtype=torch.bfloat16) -> Tensor:
    """out = mix * o_s + (1 - mix) * o_delta (o_s, o_delta float32 [..., D])."""
    D = o_s.shape[-1]
    rows = o_s.numel() // D
    out = torch.empty(o_s.shape, device=o_s.device, dtype=dtype)
    mx = mix.to(dtype).contiguous()
    per_channel = int(mx.numel() == o_s.numel())
    st = _lib.load().sgsa_gate_mix(_ptr(o_s.contiguous()), _ptr(o_delta.contiguous()), _ptr(mx),
                                    _ptr(out), rows, D, per_channel, _DT[dtype], _stream(o_s))
    _lib.check(st, "sgsa_gate_mix", o_s)
    return out


def sparse_retrieve(q: Tensor, k: Tensor, v: Tensor, indices: Tensor,
                    scale: Optional[float] = None):
    """(k_hat, v_hat) [B, T, H, D]: softmax-weighted sums of the selected k and v rows
    (SparseRetriever._token_only, modelings/modeling_sgsa.py:113-142)."""
    for n, t in (("q", q), ("k", k), ("v", v), ("indices", indices)):
        _dev(t, n)
    B, T, H, D = q.shape
    K = indices.shape[-1]
    q_, k_, v_ = q.contiguous(), k.to(q.dtype).contiguous(), v.to(q.dtype).contiguous()
    kh, vh = torch.empty_like(q_), torch.empty_like(q_)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    st = _lib.load().sgsa_sparse_retrieve(_ptr(q_), _ptr(k_), _ptr(v_),
                                           _ptr(indices.to(torch.int32).contiguous()), _ptr(kh),
                                           _ptr(vh), B, T, H, D, K, indices.shape[1], sc,
                                           _dtype_code(q), _stream(q))
    _lib.check(st, "sgsa_sparse_retrieve", q)
    return kh, vh


def sgsa_sparse_write_fwd(q, k, v, beta, gamma, alpha, top_k: int, iq=None, ik=None,
                          initial_state=None, output_final_state: bool = False):
    """The SGSA block core with the sparse write (modelings/modeling_sgsa.py:634-684
    with write_mode "direct"): top-k retrieval (scores iq . ik, by default q . k as
    in SparseRetriever.forward, modelings/modeling_sgsa.py:407-474), its k_hat / v_hat
    written into the state as the second virtual sample of each token with gain
    alpha (modelings/modeling_sgsa.py:546-609).  Returns (o, final state | None)."""
    idx = indexer_topk(q if iq is None else iq, k if ik is None else ik, top_k)
    k_hat, v_hat = sparse_retrieve(q, k, v, idx)
    return chunk_sgsa(q, k, v, beta, gamma, sparse_k=k_hat, sparse_v=v_hat, alpha=alpha,
                      initial_state=initial_state, output_final_state=output_final_state)
