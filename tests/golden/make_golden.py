"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's OWN Python code, imported from a checkout of
FAndromedA/sgsa (read-only; pass its path as argv[1]), on seeded inputs and
writes small ``.npz`` fixtures next to this script:

* ``recurrent_tiny.npz``   -- ``naive_recurrent_sgsa`` (modelings/sgsa_ops/naive.py:10-57)
  on the reference test's own shapes (tests/test_sgsa_core.py:11-22), with and
  without sparse write, with an initial state, in float64.
* ``recurrent_cfg0.npz``   -- ``naive_recurrent_sgsa`` in float64 on the fp32
  CPU configuration (B1 T1024 H4 D64) from ``sgsa_b200.inputs``.
* ``topk_masked.npz``      -- ``SparseRetriever._masked_topk``
  (modelings/modeling_sgsa.py:144-165) on random causal scores.
* ``indexer_cfg0.npz``     -- the same selection applied to the indexer scores
  iq . ik^T of the fp32 CPU configuration (top-k 128, indexer dim 32).
* ``retriever_token.npz``  -- ``SparseRetriever._token_only`` (modelings/modeling_sgsa.py:113-142):
  the retrieval k_hat / v_hat of the sparse-write SGSA block.
* ``dense_block_ref.npz``  -- ``HybridDenseDeltaTopKBlock`` layer 0 (a dense block:
  RMSNorm, RoPE, causal softmax attention, SwiGLU; hybrid_dense_delta_topk.py:97-243,394-431).
* ``sparse_attn_ref.npz``  -- ``TopKSparseKVReuseAttention.forward``
  (modelings/hybrid_dense_delta_topk.py:330-358) with identity projections and
  identity RoPE, then the gate of hybrid_dense_delta_topk.py:389-390.

Index sets are stored sorted ascending and padded with -1 (only valid slots are
kept: hybrid_dense_delta_topk.py:346-350 pads rows shorter than k with masked
entries whose softmax weight is 0).

Usage:  python -B tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import hashlib
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().float().contiguous().numpy().tobytes()).hexdigest()


def sorted_valid(indices: torch.Tensor, valid: torch.Tensor) -> np.ndarray:
    idx = torch.where(valid, indices, torch.full_like(indices, 1 << 30))
    idx, _ = torch.sort(idx, dim=-1)
    idx = torch.where(idx == (1 << 30), torch.full_like(idx, -1), idx)
    return idx.numpy().astype(np.int32)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from modelings.sgsa_ops.naive import naive_recurrent_sgsa
    from modelings.modeling_sgsa import SparseRetriever
    from modelings.hybrid_dense_delta_topk import (HybridDenseDeltaTopKConfig,
                                                    TopKSparseKVReuseAttention)
    from sgsa_b200.inputs import CONFIGS, make_inputs

    # (1) tiny recurrence, the reference test's fixture recipe.
    torch.manual_seed(0)
    B, T, H, D = 2, 9, 3, 5
    q, k, v, sk, sv = (torch.randn(B, T, H, D, dtype=torch.float64) for _ in range(5))
    beta = torch.sigmoid(torch.randn(B, T, H, dtype=torch.float64))
    gamma = torch.sigmoid(torch.randn(B, T, H, dtype=torch.float64))
    alpha = 0.25 * torch.sigmoid(torch.randn(B, T, H, dtype=torch.float64))
    s0 = 0.1 * torch.randn(B, H, D, D, dtype=torch.float64)
    o_ns, st_ns = naive_recurrent_sgsa(q=q, k=k, v=v, beta=beta, gamma=gamma, output_final_state=True)
    o_sp, st_sp = naive_recurrent_sgsa(q=q, k=k, v=v, beta=beta, gamma=gamma, sparse_k=sk,
                                       sparse_v=sv, alpha=alpha, initial_state=s0.clone(),
                                       output_final_state=True)
    np.savez_compressed(os.path.join(HERE, "recurrent_tiny.npz"),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), sk=sk.numpy(), sv=sv.numpy(),
                        beta=beta.numpy(), gamma=gamma.numpy(), alpha=alpha.numpy(),
                        s0=s0.numpy(), o_nosparse=o_ns.numpy(), state_nosparse=st_ns.numpy(),
                        o_sparse=o_sp.numpy(), state_sparse=st_sp.numpy())

    # (2) the fp32 CPU configuration, delta stage, float64 reference run.
    cfg = CONFIGS["cpu_fp32"]
    x = make_inputs(cfg, seed=0)
    hashes = {n: sha(t) for n, t in x.items()}
    d = {n: t.double() for n, t in x.items()}
    o, st = naive_recurrent_sgsa(q=d["q"], k=d["k"], v=d["v"], beta=d["beta"], gamma=d["gamma"],
                                 output_final_state=True)
    np.savez_compressed(os.path.join(HERE, "recurrent_cfg0.npz"),
                        o=o.float().numpy(), state=st.float().numpy(),
                        input_names=np.array(list(hashes.keys())),
                        input_sha256=np.array(list(hashes.values())))

    # (3) the reference's masked top-k on random causal scores.
    torch.manual_seed(1)
    Bs, Hs, Ts, ks = 1, 2, 200, 32
    scores = torch.randn(Bs, Hs, Ts, Ts)
    valid = ~torch.triu(torch.ones(Ts, Ts, dtype=torch.bool), diagonal=1)
    valid = valid[None, None].expand(Bs, Hs, Ts, Ts)
    _, ti, tv = SparseRetriever._masked_topk(None, scores=scores, valid_mask=valid, topk=ks)
    np.savez_compressed(os.path.join(HERE, "topk_masked.npz"), scores=scores.numpy(),
                        idx=sorted_valid(ti, tv), k=ks)

    # (4) indexer selection at the fp32 CPU configuration.
    iq = d["iq"].transpose(1, 2)  # [B,H,T,DI]
    ik = d["ik"].transpose(1, 2)
    sc = torch.matmul(iq, ik.transpose(-1, -2))
    Tn = sc.shape[-1]
    valid = ~torch.triu(torch.ones(Tn, Tn, dtype=torch.bool), diagonal=1)
    valid = valid[None, None].expand_as(sc)
    _, ti, tv = SparseRetriever._masked_topk(None, scores=sc, valid_mask=valid, topk=cfg.top_k)
    np.savez_compressed(os.path.join(HERE, "indexer_cfg0.npz"), idx=sorted_valid(ti, tv).astype(np.int16))

    # (5) the reference's top-k sparse attention (identity projections / RoPE) + gate.
    torch.manual_seed(2)
    Ba, Ta, Ha, Da, ka = 1, 256, 2, 32, 64
    hcfg = HybridDenseDeltaTopKConfig(hidden_size=Ha * Da, num_attention_heads=Ha, top_k=ka)
    attn = TopKSparseKVReuseAttention(hcfg).double()
    with torch.no_grad():
        attn.q_proj.weight.copy_(torch.eye(Ha * Da, dtype=torch.float64))
        attn.o_proj.weight.copy_(torch.eye(Ha * Da, dtype=torch.float64))
    qa = torch.randn(Ba, Ta, Ha, Da, dtype=torch.float64)
    ka_ = torch.randn(Ba, Ta, Ha, Da, dtype=torch.float64)
    va = torch.randn(Ba, Ta, Ha, Da, dtype=torch.float64)
    od = torch.randn(Ba, Ta, Ha, Da, dtype=torch.float64)
    mix = torch.sigmoid(torch.randn(Ba, Ta, Ha, Da, dtype=torch.float64))
    cos = torch.ones(1, 1, Ta, Da, dtype=torch.float64)
    sin = torch.zeros(1, 1, Ta, Da, dtype=torch.float64)
    with torch.no_grad():
        topk_out = attn(hidden_states=qa.reshape(Ba, Ta, Ha * Da),
                        dense_kv=(ka_.transpose(1, 2), va.transpose(1, 2)),
                        rope=(cos, sin), attention_mask=None)
    topk_out = topk_out.view(Ba, Ta, Ha, Da)
    mixed = mix * topk_out + (1.0 - mix) * od
    np.savez_compressed(os.path.join(HERE, "sparse_attn_ref.npz"), q=qa.numpy(), k=ka_.numpy(),
                        v=va.numpy(), o_delta=od.numpy(), mix=mix.numpy(),
                        topk_out=topk_out.numpy(), out=mixed.numpy(), top_k=ka)
    # (6) the retriever's token path: k_hat / v_hat over the masked top-k
    #     (modelings/modeling_sgsa.py:113-142), self given as a plain namespace
    import types
    torch.manual_seed(3)
    Br, Tr, Hr, Dr, kr = 1, 200, 2, 32, 24
    qr, kk, vr = (torch.randn(Br, Hr, Tr, Dr, dtype=torch.float64) for _ in range(3))
    sc = torch.matmul(qr, kk.transpose(-1, -2)) / math.sqrt(Dr)
    valid = ~torch.triu(torch.ones(Tr, Tr, dtype=torch.bool), diagonal=1)
    valid = valid[None, None].expand(Br, Hr, Tr, Tr)
    ns = types.SimpleNamespace(top_k=kr, eps=1e-6)
    ns._masked_topk = lambda scores, valid_mask, topk: SparseRetriever._masked_topk(
        ns, scores=scores, valid_mask=valid_mask, topk=topk)
    res = SparseRetriever._token_only(ns, scores=sc, valid_mask=valid, k=kk, v=vr)
    np.savez_compressed(os.path.join(HERE, "retriever_token.npz"),
                        q=qr.transpose(1, 2).numpy(), k=kk.transpose(1, 2).numpy(),
                        v=vr.transpose(1, 2).numpy(), k_hat=res["k_hat"].transpose(1, 2).numpy(),
                        v_hat=res["v_hat"].transpose(1, 2).numpy(), top_k=kr)

    # (7) one dense block of the hybrid model (RMSNorm, RoPE, causal softmax attention,
    #     SwiGLU, residuals): HybridDenseDeltaTopKBlock layer 0, float64, weights std 0.1
    from modelings.hybrid_dense_delta_topk import (HybridDenseDeltaTopKBlock,
                                                    HybridDenseDeltaTopKCache,
                                                    _build_rope_cache)
    torch.manual_seed(4)
    cfgd = HybridDenseDeltaTopKConfig(vocab_size=64, hidden_size=64, intermediate_size=96,
                                      num_hidden_layers=1, num_attention_heads=2)
    blk = HybridDenseDeltaTopKBlock(cfgd, 0).double()
    with torch.no_grad():
        for prm in blk.parameters():
            prm.copy_(torch.randn_like(prm) * 0.1 + (1.0 if prm.dim() == 1 else 0.0))
        xd = torch.randn(2, 40, 64, dtype=torch.float64)
        rope = _build_rope_cache(40, cfgd.head_dim, cfgd.rope_theta, xd.device, xd.dtype)
        yd = blk(xd, rope, None, HybridDenseDeltaTopKCache(), False)
    w = {n.replace(".", "_"): prm.detach().numpy() for n, prm in blk.named_parameters()}
    np.savez_compressed(os.path.join(HERE, "dense_block_ref.npz"), x=xd.numpy(), y=yd.numpy(),
                        heads=2, eps=cfgd.layer_norm_eps, theta=cfgd.rope_theta, **w)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SGSA_REFERENCE", ""))
