"""TEST INFRASTRUCTURE ONLY: CPU restatement of the hybrid model's prefill forward.

Only ``tests/`` and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``
use this module; ``sgsa_b200`` never imports it.

The model follows HybridDenseDeltaTopKForCausalLM (modelings/hybrid_dense_delta_topk.py):
token embedding (:447), blocks with pre-RMSNorm residual attention and SwiGLU MLP
(:394-431), a dense causal softmax-attention layer at every layer index divisible
by 4 (:398, DenseFullAttention :186-243 with RoPE :127-151), final RMSNorm and the
tied LM head (:449-453, :509-510).  The other layers are the SGSA layer of this
path (delta rule, top-k indexer, sparse attention, gate) behind one fused input
projection; its core is ``oracle.sgsa_layer``.

Computation is float64 torch on the CPU (the SGSA core: float64 inside the C
oracle on float32 inputs).  The dense block is pinned by ``tests/golden/dense_block_ref.npz``,
made by running the reference's own HybridDenseDeltaTopKBlock.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import oracle


def _d(t, dtype=torch.float64):
    return t.detach().cpu().to(dtype) if torch.is_tensor(t) else torch.as_tensor(t, dtype=dtype)


def rmsnorm(x, w, eps):
    """RMSNorm.forward (hybrid_dense_delta_topk.py:103-106)."""
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def swiglu(x, w_gate, w_up, w_down):
    """SwiGLUMLP.forward (hybrid_dense_delta_topk.py:117-119)."""
    return (torch.nn.functional.silu(x @ w_gate.T) * (x @ w_up.T)) @ w_down.T


def rope_tables(T, D, theta, pos0=0):
    """cos, sin [T, D] of _build_rope_cache (hybrid_dense_delta_topk.py:127-141)."""
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    f = torch.outer(torch.arange(pos0, pos0 + T, dtype=torch.float64), inv)
    emb = torch.cat((f, f), -1)
    return emb.cos(), emb.sin()


def apply_rope(x, cos, sin):
    """_apply_rope on [B, T, H, D] (hybrid_dense_delta_topk.py:144-151)."""
    h = x.shape[-1] // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), -1)
    return x * cos[None, :, None, :] + rot * sin[None, :, None, :]


def dense_attention(x, w_q, w_k, w_v, w_o, heads, theta):
    """DenseFullAttention.forward without cache (hybrid_dense_delta_topk.py:200-243)."""
    B, T, N = x.shape
    D = N // heads
    q = (x @ w_q.T).view(B, T, heads, D)
    k = (x @ w_k.T).view(B, T, heads, D)
    v = (x @ w_v.T).view(B, T, heads, D)
    cos, sin = (t.to(x.dtype) for t in rope_tables(T, D, theta))
    q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    s = torch.einsum("bthd,bjhd->bhtj", q, k) / math.sqrt(D)
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    a = torch.einsum("bhtj,bjhd->bthd", torch.softmax(s, -1), v)
    return a.reshape(B, T, N) @ w_o.T


def dense_block(x, w, heads, eps, theta):
    """HybridDenseDeltaTopKBlock.forward of a dense layer (hybrid_dense_delta_topk.py:406-431);
    ``w`` holds the reference's parameter names."""
    x = _d(x)
    w = {n: _d(t) for n, t in w.items()}
    h = rmsnorm(x, w["input_norm_weight"], eps)
    x = x + dense_attention(h, w["attention_q_proj_weight"], w["attention_k_proj_weight"],
                            w["attention_v_proj_weight"], w["attention_o_proj_weight"], heads,
                            theta)
    h = rmsnorm(x, w["post_attention_norm_weight"], eps)
    return x + swiglu(h, w["mlp_gate_proj_weight"], w["mlp_up_proj_weight"], w["mlp_down_proj_weight"])


def sgsa_projection(h, w_in, b_in, H, D, DI):
    """Split and transform the fused SGSA projection (the columns of ``sgsa_layer_proj``)."""
    B, T, _ = h.shape
    p = h @ w_in.T + b_in
    HD, HI = H * D, H * DI
    q = torch.nn.functional.normalize(p[..., :HD].reshape(B, T, H, D), dim=-1)
    k = torch.nn.functional.normalize(p[..., HD:2 * HD].reshape(B, T, H, D), dim=-1)
    v = p[..., 2 * HD:3 * HD].reshape(B, T, H, D)
    mix = torch.sigmoid(p[..., 3 * HD:4 * HD]).reshape(B, T, H, D)
    iq = p[..., 4 * HD:4 * HD + HI].reshape(B, T, H, DI)
    ik = p[..., 4 * HD + HI:4 * HD + 2 * HI].reshape(B, T, H, DI)
    o = 4 * HD + 2 * HI
    beta = torch.sigmoid(p[..., o:o + H]).clamp_min(1e-4)
    gamma = torch.sigmoid(p[..., o + H:o + 2 * H])
    return dict(q=q, k=k, v=v, beta=beta, gamma=gamma, iq=iq, ik=ik, mix=mix)


def model_forward(ids, weights, cfg, dtype=torch.float64):
    """Logits [B, T, V] of ``sgsa_b200.hybrid.HybridSGSAModel`` for token ids [B, T].

    ``weights`` is that model's ``weights`` dict; ``cfg`` its ``HybridConfig``;
    ``dtype`` the CPU arithmetic type of everything outside the SGSA core (float64
    for parity, float32 for the timed CPU baseline)."""
    ids = torch.as_tensor(ids).cpu()
    emb = _d(weights["embed"], dtype)
    x = emb[ids]
    H, D, DI = cfg.num_heads, cfg.head_dim, cfg.indexer_dim
    for li, lw in enumerate(weights["layers"]):
        w = {n: _d(t, dtype) for n, t in lw.items()}
        h = rmsnorm(x, w["norm1"], cfg.eps)
        if cfg.is_dense(li):
            wq, wk, wv = w["w_qkv"].chunk(3, 0)
            x = x + dense_attention(h, wq, wk, wv, w["w_o"], H, cfg.rope_theta)
        else:
            a = sgsa_projection(h, w["w_in"], w["b_in"], H, D, DI)
            out, _, _, _ = oracle.sgsa_layer(a["q"], a["k"], a["v"], a["beta"], a["gamma"],
                                             a["iq"], a["ik"], a["mix"], cfg.top_k)
            B, T = ids.shape
            x = x + torch.from_numpy(np.asarray(out)).to(dtype).reshape(B, T, -1) @ w["w_o"].T
        h = rmsnorm(x, w["norm2"], cfg.eps)
        I = cfg.intermediate_size
        x = x + swiglu(h, w["w_gu"][:I], w["w_gu"][I:], w["w_down"])
    x = rmsnorm(x, _d(weights["norm_f"], dtype), cfg.eps)
    return x @ emb.T
