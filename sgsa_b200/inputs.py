"""Seeded synthetic inputs for the SGSA layer forward.

The reference publishes no dataset for this path; its layer is exercised on
random tensors (``tests/test_sgsa_core.py:11-22`` in the reference).  The
configurations below carry the shapes and value distributions of the
benchmark configurations:

* one CPU ``torch.Generator`` seeded once, float32 draws in the fixed order
  q, k, v, beta-logits, g-logits, iq, ik, mix-logits;
* ``q, k <- l2-normalise(., dim=-1)``, ``beta = sigmoid``, ``g = -softplus``,
  ``gamma = exp(g)``, ``mix = sigmoid`` (per channel, ``[B, T, H, D]``);
* bf16 configurations cast after the transforms, so every GPU count sees
  identical data.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class LayerConfig:
    name: str
    B: int
    T: int
    H: int
    D: int
    top_k: int
    d_idx: int
    chunk: int = 64
    dtype: torch.dtype = torch.bfloat16

    @property
    def tokens(self) -> int:
        return self.B * self.T

    def scaled(self, **kw) -> "LayerConfig":
        return replace(self, **kw)


CONFIGS = {
    "cpu_fp32": LayerConfig("cpu_fp32", B=1, T=1024, H=4, D=64, top_k=128, d_idx=32,
                            dtype=torch.float32),
    "b200_bf16": LayerConfig("b200_bf16", B=4, T=8192, H=16, D=128, top_k=512, d_idx=64),
    "long_ctx": LayerConfig("long_ctx", B=1, T=65536, H=32, D=128, top_k=2048, d_idx=64),
}


def make_inputs(cfg: LayerConfig, seed: int = 0, device="cpu"):
    """Return the dict of layer inputs for ``cfg`` (generated on the CPU)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    B, T, H, D, DI = cfg.B, cfg.T, cfg.H, cfg.D, cfg.d_idx

    def draw(*shape):
        return torch.randn(*shape, generator=g, dtype=torch.float32)

    q = F.normalize(draw(B, T, H, D), dim=-1)
    k = F.normalize(draw(B, T, H, D), dim=-1)
    v = draw(B, T, H, D)
    beta = torch.sigmoid(draw(B, T, H))
    gl = -F.softplus(draw(B, T, H))
    gamma = torch.exp(gl)
    iq = draw(B, T, H, DI)
    ik = draw(B, T, H, DI)
    mix = torch.sigmoid(draw(B, T, H, D))
    out = dict(q=q, k=k, v=v, beta=beta, gamma=gamma, iq=iq, ik=ik, mix=mix)
    out = {n: t.to(cfg.dtype) for n, t in out.items()}
    if device != "cpu":
        out = {n: t.to(device) for n, t in out.items()}
    return out


def make_inputs_slice(cfg: LayerConfig, t0: int, t1: int, seed: int = 0, block: int = 1024,
                      device="cpu"):
    """Tokens [t0, t1) of a long input drawn block by block: block i of `block`
    tokens comes from its own generator seeded (seed, i), with the distributions
    of ``make_inputs``.  Any slicing into whole blocks gives identical data, so
    every GPU count of a sequence-parallel run sees the same sequence."""
    if t0 % block or t1 % block:
        raise ValueError("slice bounds must be multiples of the block")
    parts = []
    for i in range(t0 // block, t1 // block):
        parts.append(make_inputs(replace(cfg, T=block), seed=seed * 1000003 + i))
    out = {n: torch.cat([p[n] for p in parts], dim=1) for n in parts[0]}
    if device != "cpu":
        out = {n: t.to(device) for n, t in out.items()}
    return out
