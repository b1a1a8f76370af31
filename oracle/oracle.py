"""TEST INFRASTRUCTURE ONLY: ctypes front-end of the CPU parity oracle.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` import this module.  The product
package ``sgsa_b200`` never does.

Parity status: pinned against fixtures that ``tests/golden/make_golden.py``
produced by running the reference's own Python implementation
(``modelings/sgsa_ops/naive.py:10-57``, ``modelings/modeling_sgsa.py:144-165``,
``modelings/hybrid_dense_delta_topk.py:317-358,389-390``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libsgsa_oracle.so")
_lib = None

_f = ctypes.POINTER(ctypes.c_float)
_i32 = ctypes.POINTER(ctypes.c_int32)
_d = ctypes.POINTER(ctypes.c_double)
_ci = ctypes.c_int


def build(force: bool = False) -> str:
    """Compile the oracle (gcc + OpenMP) into oracle/_build/."""
    src = os.path.join(_HERE, "sgsa_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_SO)
        L.oracle_sgsa_recurrent.argtypes = [_f] * 11 + [_ci] * 6
        L.oracle_sgsa_recurrent.restype = None
        L.oracle_topk_select_f32.argtypes = [_f, _i32, _ci, _ci, _ci, _i32]
        L.oracle_topk_select_f32.restype = None
        L.oracle_indexer_topk.argtypes = [_f, _f] + [_ci] * 7 + [_i32, _d]
        L.oracle_indexer_topk.restype = None
        L.oracle_sparse_attn_mix.argtypes = [_f, _f, _f, _i32, _f, _f, _f] + [_ci] * 5 + [
            ctypes.c_double, _ci, _ci, _ci]
        L.oracle_sparse_attn_mix.restype = None
        L.oracle_num_threads.restype = ctypes.c_int
        L.oracle_set_num_threads.argtypes = [_ci]
        _lib = L
    return _lib


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


def _f32(x):
    if x is None:
        return None
    if hasattr(x, "detach"):
        x = x.detach().float().cpu().numpy()
    return np.ascontiguousarray(x, dtype=np.float32)


def _p(a, t=_f):
    return None if a is None else a.ctypes.data_as(t)


def sgsa_recurrent(q, k, v, beta, gamma, sparse_k=None, sparse_v=None, alpha=None,
                   initial_state=None, heads=None):
    """(o, final_state) of the token-by-token SGSA recurrence, float64 inside.

    ``heads=(h0, h1)`` restricts the work to a head range (other heads of the
    outputs stay zero).  Restates modelings/sgsa_ops/naive.py:39-55.
    """
    q, k, v, beta, gamma = map(_f32, (q, k, v, beta, gamma))
    sk, sv, al, s0 = map(_f32, (sparse_k, sparse_v, alpha, initial_state))
    B, T, H, D = q.shape
    if k.shape[-1] != D or v.shape[-1] != D:
        raise ValueError("SGSA requires dk == dv == q.shape[-1]")
    out = np.zeros((B, T, H, D), np.float32)
    st = np.zeros((B, H, D, D), np.float32)
    h0, h1 = heads if heads is not None else (0, H)
    lib().oracle_sgsa_recurrent(_p(q), _p(k), _p(v), _p(beta), _p(gamma), _p(sk), _p(sv), _p(al),
                                _p(s0), _p(out), _p(st), B, T, H, D, h0, h1)
    return out, st


def topk_select(scores, valid, k):
    """Row-wise top-k (ascending indices, -1 padded) of float32 scores [R, S]."""
    s = _f32(scores)
    R, S = s.shape
    val = np.ascontiguousarray(valid, dtype=np.int32)
    out = np.empty((R, k), np.int32)
    lib().oracle_topk_select_f32(_p(s), _p(val, _i32), R, S, k, _p(out, _i32))
    return out


def indexer_topk(iq, ik, k, t_range=None, return_kth=False):
    """Causal top-k indices [B, H, nq, k] (ascending, -1 padded) of iq . ik."""
    iq, ik = _f32(iq), _f32(ik)
    B, T, H, DI = iq.shape
    t0, t1 = t_range if t_range is not None else (0, T)
    nq = t1 - t0
    out = np.empty((B, H, nq, k), np.int32)
    kth = np.empty((B, H, nq), np.float64) if return_kth else None
    lib().oracle_indexer_topk(_p(iq), _p(ik), B, T, H, DI, k, t0, t1, _p(out, _i32), _p(kth, _d))
    return (out, kth) if return_kth else out


def sparse_attn_mix(q, k, v, idx, o_delta=None, mix=None, scale=None, t_range=None):
    """Gated sparse attention [B, nq, H, D] over index rows [B, H, nq, K]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, T, H, D = q.shape
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    K = idx.shape[-1]
    od, mx = _f32(o_delta), _f32(mix)
    per_channel = int(mx is not None and mx.ndim == 4)
    t0, t1 = t_range if t_range is not None else (0, T)
    out = np.empty((B, t1 - t0, H, D), np.float32)
    sc = float(scale) if scale is not None else 1.0 / np.sqrt(D)
    lib().oracle_sparse_attn_mix(_p(q), _p(k), _p(v), _p(idx, _i32), _p(od), _p(mx), _p(out),
                                 B, T, H, D, K, sc, per_channel, t0, t1)
    return out


def sgsa_layer(q, k, v, beta, gamma, iq, ik, mix, top_k, initial_state=None):
    """Composite layer forward: delta stage, indexer top-k, sparse attention, gate."""
    o_delta, st = sgsa_recurrent(q, k, v, beta, gamma, initial_state=initial_state)
    idx = indexer_topk(iq, ik, top_k)
    out = sparse_attn_mix(q, k, v, idx, o_delta, mix)
    return out, st, idx, o_delta


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def decode_topk(iq, ik_cache, n, k, return_kth=False):
    """Top-k rows (ascending, -1 padded) of iq [B,H,DI] . ik_cache[:, :n] [B,Tc,H,DI],
    float64 scores, ties to the lowest row: the decode form of the selection of
    modelings/hybrid_dense_delta_topk.py:343-349 against the cache (:226-230)."""
    iq = np.asarray(_f32(iq), np.float64)
    ikc = np.asarray(_f32(ik_cache), np.float64)[:, :n]
    s = np.einsum("bhd,bjhd->bhj", iq, ikc)
    B, H, _ = s.shape
    out = np.full((B, H, k), -1, np.int32)
    kth = np.empty((B, H))
    for b in range(B):
        for h in range(H):
            order = np.lexsort((np.arange(n), -s[b, h]))  # score desc, index asc
            m = min(k, n)
            sel = np.sort(order[:m])
            out[b, h, :m] = sel
            kth[b, h] = s[b, h, order[m - 1]]
    return (out, kth) if return_kth else out


def decode_attn_mix(q, k_cache, v_cache, idx, o_delta=None, mix=None, scale=None):
    """Softmax attention of q [B,H,D] over the selected cache rows, then the gate
    (modelings/hybrid_dense_delta_topk.py:350-356, :389-390), float64."""
    q = np.asarray(_f32(q), np.float64)
    kc = np.asarray(_f32(k_cache), np.float64)
    vc = np.asarray(_f32(v_cache), np.float64)
    B, H, D = q.shape
    sc = float(scale) if scale is not None else 1.0 / np.sqrt(D)
    out = np.zeros((B, H, D))
    for b in range(B):
        for h in range(H):
            sel = idx[b, h][idx[b, h] >= 0]
            s = kc[b, sel, h] @ q[b, h] * sc
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ vc[b, sel, h]
    if o_delta is not None:
        od = np.asarray(_f32(o_delta), np.float64)
        m = np.asarray(_f32(mix), np.float64) if mix is not None else np.ones((B, H))
        if m.ndim == 2:
            m = m[..., None]
        out = m * out + (1.0 - m) * od
    return out


def sparse_retrieve(k, v, idx, q, scale=None):
    """(k_hat, v_hat) [B, T, H, D]: softmax(q . k_j * scale) weighted sums of the
    selected k and v rows -- the retriever's token path
    (modelings/modeling_sgsa.py:113-142), float64."""
    q = np.asarray(_f32(q), np.float64)
    k = np.asarray(_f32(k), np.float64)
    v = np.asarray(_f32(v), np.float64)
    B, T, H, D = q.shape
    sc = float(scale) if scale is not None else 1.0 / np.sqrt(D)
    kh = np.zeros((B, T, H, D))
    vh = np.zeros((B, T, H, D))
    for b in range(B):
        for h in range(H):
            hh = h if idx.shape[1] == H else 0
            for t in range(T):
                sel = idx[b, hh, t][idx[b, hh, t] >= 0]
                s = k[b, sel, h] @ q[b, t, h] * sc
                p = np.exp(s - s.max())
                p /= p.sum()
                kh[b, t, h] = p @ k[b, sel, h]
                vh[b, t, h] = p @ v[b, sel, h]
    return kh, vh
