"""Hybrid dense / SGSA language model: the prefill forward around the SGSA layer.

Layout of HybridDenseDeltaTopKForCausalLM (modelings/hybrid_dense_delta_topk.py:434-532):
token embedding, ``num_layers`` pre-RMSNorm blocks (attention + SwiGLU MLP, each
with a residual), final RMSNorm, LM head tied to the embedding.  A block whose
index is divisible by 4 is a dense causal softmax-attention layer with RoPE (:398,
:186-243); the others are SGSA layers: one fused input projection (q, k, v, mix,
indexer iq/ik, beta, gamma), the fused SGSA layer core of this package (delta rule,
exact top-k indexer, sparse attention over the layer's own keys, per-channel
sigmoid gate) and the output projection.

Device work per block: GEMMs through cuBLAS (``torch.addmm`` with the residual as
the accumulator input), dense attention through PyTorch's SDPA (flash kernels),
everything else in this package's kernels: ``sgsa_embed``, ``sgsa_rmsnorm``,
``sgsa_rope_qkv``, ``sgsa_layer_proj``, ``sgsa_layer_fwd``, ``sgsa_swiglu``.
Forward only (prefill), no KV cache.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from . import _lib, ops

Tensor = torch.Tensor


@dataclass(frozen=True)
class HybridConfig:
    vocab_size: int = 32000
    hidden_size: int = 2048
    intermediate_size: int = 5632
    num_layers: int = 24
    num_heads: int = 16
    top_k: int = 512
    indexer_dim: int = 64
    chunk_size: int = 64
    eps: float = 1e-6
    rope_theta: float = 10000.0
    init_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    def is_dense(self, layer: int) -> bool:
        return layer % 4 == 0

    @property
    def proj_width(self) -> int:
        """Columns of the fused SGSA projection, padded to a multiple of 8."""
        H, D, DI = self.num_heads, self.head_dim, self.indexer_dim
        n = 4 * H * D + 2 * H * DI + 2 * H
        return (n + 7) // 8 * 8


# 24 layers, hidden 2048, 16 heads x 128, SwiGLU 5632, vocab 32000, top-k 512
CONFIG_B200 = HybridConfig()
TINY = HybridConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_layers=4,
                    num_heads=4, top_k=32, indexer_dim=32, init_std=0.05)


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _dt(t):
    if t.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.DTYPE_F32
    raise ValueError(f"unsupported dtype {t.dtype}")


def rmsnorm(x: Tensor, w: Tensor, eps: float, out: Optional[Tensor] = None) -> Tensor:
    x = x.contiguous()
    out = torch.empty_like(x) if out is None else out
    st = _lib.load().sgsa_rmsnorm(_ptr(x), _ptr(w), _ptr(out), x.numel() // x.shape[-1],
                                  x.shape[-1], float(eps), _dt(x), _stream(x))
    _lib.check(st, "sgsa_rmsnorm")
    return out


def swiglu(gu: Tensor) -> Tensor:
    I = gu.shape[-1] // 2
    out = torch.empty(*gu.shape[:-1], I, dtype=gu.dtype, device=gu.device)
    st = _lib.load().sgsa_swiglu(_ptr(gu), _ptr(out), gu.numel() // gu.shape[-1], I, _dt(gu),
                                 _stream(gu))
    _lib.check(st, "sgsa_swiglu")
    return out


def rope_table(T: int, D: int, theta: float, device) -> Tensor:
    """float32 [T, D/2, 2] of (cos, sin) at position t, frequency theta^(-2j/D)."""
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    f = torch.outer(torch.arange(T, dtype=torch.float64), inv)
    return torch.stack((f.cos(), f.sin()), -1).to(torch.float32).to(device).contiguous()


def rope_qkv(qkv: Tensor, cs: Tensor, H: int, pos0: int = 0):
    """qkv [B, T, 3*H*D] -> q, k (RoPE) and v [B, T, H, D]."""
    B, T, n = qkv.shape
    D = n // (3 * H)
    q = torch.empty(B, T, H, D, dtype=qkv.dtype, device=qkv.device)
    k, v = torch.empty_like(q), torch.empty_like(q)
    st = _lib.load().sgsa_rope_qkv(_ptr(qkv), _ptr(cs), _ptr(q), _ptr(k), _ptr(v), B, T, H, D,
                                   pos0, _dt(qkv), _stream(qkv))
    _lib.check(st, "sgsa_rope_qkv")
    return q, k, v


def layer_proj(P: Tensor, H: int, D: int, DI: int) -> Dict[str, Tensor]:
    """Epilogue of the fused SGSA projection P [B, T, ld] (sgsa_layer_proj)."""
    B, T, ld = P.shape
    e = lambda *s: torch.empty(B, T, *s, dtype=P.dtype, device=P.device)
    a = dict(q=e(H, D), k=e(H, D), v=e(H, D), mix=e(H, D), iq=e(H, DI), ik=e(H, DI), beta=e(H),
             gamma=e(H))
    st = _lib.load().sgsa_layer_proj(_ptr(P), ld, *[_ptr(a[n]) for n in
                                                    ("q", "k", "v", "mix", "iq", "ik", "beta",
                                                     "gamma")],
                                     B * T, H, D, DI, _dt(P), _stream(P))
    _lib.check(st, "sgsa_layer_proj")
    return a


def embed(ids: Tensor, table: Tensor) -> Tensor:
    ids = ids.to(torch.int64).contiguous()
    out = torch.empty(*ids.shape, table.shape[1], dtype=table.dtype, device=table.device)
    st = _lib.load().sgsa_embed(_ptr(ids), _ptr(table), _ptr(out), ids.numel(), table.shape[1],
                                table.shape[0], _dt(table), _stream(table))
    _lib.check(st, "sgsa_embed")
    return out


class HybridSGSAModel:
    """Weights and prefill forward of the hybrid model on one GPU."""

    def __init__(self, cfg: HybridConfig, device="cuda", dtype=torch.bfloat16, seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        N, I, s = cfg.hidden_size, cfg.intermediate_size, cfg.init_std

        def lin(o, i):  # nn.Linear weights [out, in], normal(0, std) as _init_weights (:458-461)
            return (torch.randn(o, i, generator=g, device=self.device) * s).to(dtype)

        ones = lambda n: torch.ones(n, dtype=dtype, device=self.device)
        emb = torch.randn(cfg.vocab_size, N, generator=g, device=self.device) * s
        emb[0] = 0.0  # padding_idx row (:463-465)
        layers: List[Dict[str, Tensor]] = []
        for li in range(cfg.num_layers):
            lw = dict(norm1=ones(N), norm2=ones(N))
            if cfg.is_dense(li):
                lw["w_qkv"] = lin(3 * N, N)
            else:
                ld = cfg.proj_width
                w_in = lin(ld, N)
                w_in[4 * N + 2 * cfg.num_heads * cfg.indexer_dim + 2 * cfg.num_heads:] = 0
                lw["w_in"] = w_in
                lw["b_in"] = torch.zeros(ld, dtype=dtype, device=self.device)  # biases init 0
            lw["w_o"] = lin(N, N)
            lw["w_gu"] = lin(2 * I, N)
            lw["w_down"] = lin(N, I)
            layers.append(lw)
        self.weights = dict(embed=emb.to(dtype), norm_f=ones(N), layers=layers)
        self._rope = None

    def _rope_table(self, T: int) -> Tensor:
        if self._rope is None or self._rope.shape[0] < T:
            self._rope = rope_table(T, self.cfg.head_dim, self.cfg.rope_theta, self.device)
        return self._rope

    def dense_attention(self, h: Tensor, lw: Dict[str, Tensor], residual: Tensor) -> Tensor:
        B, T, N = h.shape
        H = self.cfg.num_heads
        qkv = torch.matmul(h, lw["w_qkv"].T)
        q, k, v = rope_qkv(qkv, self._rope_table(T), H)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                           v.transpose(1, 2), is_causal=True)
        a = a.transpose(1, 2).reshape(B * T, N)
        return torch.addmm(residual.view(B * T, N), a, lw["w_o"].T).view(B, T, N)

    def sgsa_attention(self, h: Tensor, lw: Dict[str, Tensor], residual: Tensor) -> Tensor:
        B, T, N = h.shape
        c = self.cfg
        P = torch.addmm(lw["b_in"], h.view(B * T, N), lw["w_in"].T).view(B, T, -1)
        a = layer_proj(P, c.num_heads, c.head_dim, c.indexer_dim)
        o = ops.sgsa_layer_fwd(a["q"], a["k"], a["v"], a["beta"], a["gamma"], a["iq"], a["ik"],
                               a["mix"], c.top_k)
        return torch.addmm(residual.view(B * T, N), o.view(B * T, N), lw["w_o"].T).view(B, T, N)

    def mlp(self, x: Tensor, lw: Dict[str, Tensor]) -> Tensor:
        B, T, N = x.shape
        h = rmsnorm(x, lw["norm2"], self.cfg.eps)
        gu = torch.matmul(h.view(B * T, N), lw["w_gu"].T)
        return torch.addmm(x.view(B * T, N), swiglu(gu), lw["w_down"].T).view(B, T, N)

    @torch.no_grad()
    def forward(self, ids: Tensor, last_only: bool = False, marks=None) -> Tensor:
        """Logits [B, T, V] (or [B, V] of the last position) for token ids [B, T].

        ``marks``: optional list; a (part name, CUDA event) pair is appended after
        each part of the forward (for per-part device times)."""
        c = self.cfg
        if ids.device != self.device:
            raise ValueError("token ids must be on the model's device")

        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))

        mark("start")
        x = embed(ids, self.weights["embed"])
        for li, lw in enumerate(self.weights["layers"]):
            h = rmsnorm(x, lw["norm1"], c.eps)
            if c.is_dense(li):
                x = self.dense_attention(h, lw, x)
                mark("dense_attention")
            else:
                x = self.sgsa_attention(h, lw, x)
                mark("sgsa_layer")
            x = self.mlp(x, lw)
            mark("mlp")
        if last_only:
            x = x[:, -1:].contiguous()
        x = rmsnorm(x, self.weights["norm_f"], c.eps)
        logits = torch.matmul(x, self.weights["embed"].T)
        mark("head")
        return logits[:, 0] if last_only else logits

    __call__ = forward

    def flops_per_token(self, T: int) -> float:
        """Matrix FLOPs per token of the projections, MLPs, head and dense attention."""
        c = self.cfg
        N, I = c.hidden_size, c.intermediate_size
        f = 0.0
        for li in range(c.num_layers):
            if c.is_dense(li):
                f += 2 * N * 4 * N + 2 * 2 * N * T / 2  # qkv+o, causal QK^T and PV
            else:
                f += 2 * N * (c.proj_width + N)
            f += 2 * N * 3 * I
        return f + 2 * N * c.vocab_size
