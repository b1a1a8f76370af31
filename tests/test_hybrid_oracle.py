"""CPU checks of the hybrid-model oracle: the dense block against the reference's
own HybridDenseDeltaTopKBlock (golden fixture), and a tiny full-model forward."""
import os

import numpy as np
import torch

from oracle import hybrid as ohybrid
from sgsa_b200.hybrid import HybridConfig, HybridSGSAModel

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_dense_block_matches_reference():
    z = np.load(os.path.join(GOLDEN, "dense_block_ref.npz"))
    w = {n: z[n] for n in z.files if n.endswith("_weight")}
    y = ohybrid.dense_block(z["x"], w, int(z["heads"]), float(z["eps"]), float(z["theta"]))
    # the reference takes the softmax in float32 (hybrid_dense_delta_topk.py:180)
    assert np.abs(y.numpy() - z["y"]).max() < 1e-6


def test_rope_tables_rotate_pairs():
    cos, sin = ohybrid.rope_tables(5, 8, 10000.0)
    x = torch.randn(1, 5, 1, 8, dtype=torch.float64)
    y = ohybrid.apply_rope(x, cos, sin)
    # a rotation keeps the norm of every (j, j + D/2) pair
    n = lambda t: t[..., :4] ** 2 + t[..., 4:] ** 2
    assert torch.allclose(n(x), n(y))


def test_tiny_model_forward_on_cpu():
    cfg = HybridConfig(vocab_size=64, hidden_size=64, intermediate_size=96, num_layers=2,
                       num_heads=2, top_k=8, indexer_dim=32)
    m = HybridSGSAModel(cfg, device="cpu", dtype=torch.float32, seed=1)
    ids = torch.randint(0, 64, (1, 40), generator=torch.Generator().manual_seed(0))
    logits = ohybrid.model_forward(ids, m.weights, cfg)
    assert logits.shape == (1, 40, 64) and torch.isfinite(logits).all()
    # the padding row of the tied embedding is zero
    assert float(m.weights["embed"][0].abs().max()) == 0.0
