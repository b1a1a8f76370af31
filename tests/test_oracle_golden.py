"""The CPU oracle against fixtures produced by the reference's own code."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from sgsa_b200.inputs import CONFIGS, make_inputs

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def test_recurrent_tiny_matches_reference():
    z = load("recurrent_tiny.npz")
    o, st = oracle.sgsa_recurrent(z["q"], z["k"], z["v"], z["beta"], z["gamma"])
    assert oracle.rel_l2(o, z["o_nosparse"]) < 1e-6
    assert oracle.rel_l2(st, z["state_nosparse"]) < 1e-6
    o, st = oracle.sgsa_recurrent(z["q"], z["k"], z["v"], z["beta"], z["gamma"], z["sk"], z["sv"],
                                  z["alpha"], initial_state=z["s0"])
    assert oracle.rel_l2(o, z["o_sparse"]) < 1e-6
    assert oracle.rel_l2(st, z["state_sparse"]) < 1e-6


def test_inputs_reproduce_reference_run():
    z = load("recurrent_cfg0.npz")
    import hashlib
    x = make_inputs(CONFIGS["cpu_fp32"], seed=0)
    for n, h in zip(z["input_names"], z["input_sha256"]):
        got = hashlib.sha256(x[str(n)].float().contiguous().numpy().tobytes()).hexdigest()
        assert got == h, f"seeded input {n} differs from the one the fixture was made from"


def test_recurrent_cfg0_matches_reference():
    z = load("recurrent_cfg0.npz")
    x = make_inputs(CONFIGS["cpu_fp32"], seed=0)
    o, st = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"])
    assert oracle.rel_l2(o, z["o"]) < 1e-6
    assert oracle.rel_l2(st, z["state"]) < 1e-6


def test_masked_topk_matches_reference():
    z = load("topk_masked.npz")
    sc = z["scores"]
    B, H, T, _ = sc.shape
    k = int(z["k"])
    valid = np.tile(np.arange(1, T + 1, dtype=np.int32), B * H)
    got = oracle.topk_select(sc.reshape(B * H * T, T), valid, k).reshape(B, H, T, k)
    np.testing.assert_array_equal(got, z["idx"])


def test_indexer_cfg0_matches_reference():
    z = load("indexer_cfg0.npz")
    cfg = CONFIGS["cpu_fp32"]
    x = make_inputs(cfg, seed=0)
    got = oracle.indexer_topk(x["iq"], x["ik"], cfg.top_k)
    np.testing.assert_array_equal(got, z["idx"].astype(np.int32))


def test_sparse_attention_and_gate_match_reference():
    z = load("sparse_attn_ref.npz")
    k = int(z["top_k"])
    idx = oracle.indexer_topk(z["q"], z["k"], k)
    o = oracle.sparse_attn_mix(z["q"], z["k"], z["v"], idx)
    assert oracle.rel_l2(o, z["topk_out"]) < 1e-6
    o = oracle.sparse_attn_mix(z["q"], z["k"], z["v"], idx, z["o_delta"], z["mix"])
    assert oracle.rel_l2(o, z["out"]) < 1e-6


def test_topk_edge_cases():
    # k larger than every row, rows of length 1, exact ties -> lowest index.
    sc = np.array([[3.0, 3.0, 3.0, 1.0], [0.0, 5.0, 5.0, 5.0], [1.0, 2.0, 3.0, 4.0]], np.float32)
    got = oracle.topk_select(sc, np.array([4, 4, 1], np.int32), 2)
    np.testing.assert_array_equal(got, [[0, 1], [1, 2], [0, -1]])
    got = oracle.topk_select(sc, np.array([4, 4, 4], np.int32), 8)
    assert (got[:, :4] >= 0).all() and (got[:, 4:] == -1).all()


def test_retriever_token_path_matches_reference():
    z = load("retriever_token.npz")
    idx = oracle.indexer_topk(z["q"], z["k"], int(z["top_k"]))
    kh, vh = oracle.sparse_retrieve(z["k"], z["v"], idx, z["q"])
    assert oracle.rel_l2(kh, z["k_hat"]) < 1e-6
    assert oracle.rel_l2(vh, z["v_hat"]) < 1e-6
