"""Configuration constants and the bench's algorithmic counts (CPU only)."""
import os
import sys

import numpy as np
import pytest

from sgsa_b200.hybrid import CONFIG_B200, HybridConfig
from sgsa_b200.inputs import CONFIGS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_hybrid_config_is_configs3():
    c = CONFIG_B200
    assert (c.num_layers, c.hidden_size, c.num_heads, c.head_dim) == (24, 2048, 16, 128)
    assert (c.intermediate_size, c.vocab_size, c.top_k, c.chunk_size) == (5632, 32000, 512, 64)
    # dense layers at every index divisible by 4 (the reference's order), SGSA layers between
    assert [li for li in range(c.num_layers) if c.is_dense(li)] == list(range(0, 24, 4))


@pytest.mark.parametrize("H,D,DI", [(16, 128, 64), (4, 64, 32), (3, 32, 32)])
def test_proj_width_covers_blocks_and_aligns(H, D, DI):
    c = HybridConfig(hidden_size=H * D, num_heads=H, indexer_dim=DI)
    need = 4 * H * D + 2 * H * DI + 2 * H
    assert c.proj_width >= need and c.proj_width % 8 == 0 and c.proj_width - need < 8


def test_algorithmic_counts_configs1():
    sys.path.insert(0, ROOT)
    import bench

    cnt = bench.algorithmic_counts(CONFIGS["b200_bf16"])
    # per layer forward at B4 T8192 H16 d128 K512 DI64
    assert abs(cnt["f_delta"] / 9.4e10 - 1) < 0.01
    assert abs(cnt["f_idx"] / 2.75e11 - 1) < 0.01
    # exact causal count (rows t < K select t + 1 keys); about B H T K 4D = 1.37e11
    sel = sum(min(512, t + 1) for t in range(8192))
    assert cnt["f_sp"] == 4 * 16 * sel * 4 * 128
    assert abs(cnt["f_sp"] / 1.37e11 - 1) < 0.04
    assert cnt["bytes_gather"] == 4 * 16 * sel * 2 * 128 * 2


def test_sparse_retrieve_shared_index_matches_per_head():
    from oracle import oracle

    g = np.random.default_rng(0)
    B, T, H, D, K = 1, 40, 3, 8, 5
    q, k, v = (g.standard_normal((B, T, H, D)).astype(np.float32) for _ in range(3))
    idx1 = oracle.indexer_topk(g.standard_normal((B, T, 1, 4)).astype(np.float32),
                               g.standard_normal((B, T, 1, 4)).astype(np.float32), K)
    kh1, vh1 = oracle.sparse_retrieve(k, v, idx1, q)
    kh2, vh2 = oracle.sparse_retrieve(k, v, np.repeat(idx1, H, axis=1), q)
    np.testing.assert_allclose(kh1, kh2, rtol=1e-12)
    np.testing.assert_allclose(vh1, vh2, rtol=1e-12)
