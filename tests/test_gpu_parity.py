"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Tolerances (relative L2 against the float64 oracle run on the same,
already-rounded inputs): 1e-5 for float32 inputs, 2e-3 for bfloat16 inputs.
Top-k index sets must be identical; where the device and the oracle compute
scores with different rounding, a differing index is accepted only if its
score lies within a small band around the row's k-th score (a near tie).
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from sgsa_b200 import ops
from sgsa_b200.inputs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-3}


def dev(x):
    return {n: t.cuda() for n, t in x.items()}


def rand_case(B, T, H, D, dtype, seed=0, sparse=False, init=False, decay="softplus"):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)
    x = dict(q=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
             k=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
             v=r(B, T, H, D), beta=torch.sigmoid(r(B, T, H)))
    x["gamma"] = torch.exp(-torch.nn.functional.softplus(r(B, T, H))) if decay == "softplus" \
        else 0.9 + 0.1 * torch.rand(B, T, H, generator=g)
    if sparse:
        x["sparse_k"] = torch.nn.functional.normalize(r(B, T, H, D), dim=-1)
        x["sparse_v"] = r(B, T, H, D)
        x["alpha"] = 0.25 * torch.sigmoid(r(B, T, H))
    if init:
        x["initial_state"] = 0.1 * r(B, H, D, D)
    return {n: (t.to(dtype) if n != "initial_state" else t) for n, t in x.items()}


def run_chunk(x):
    d = dev(x)
    o, s = ops.chunk_sgsa(**d, output_final_state=True)
    torch.cuda.synchronize()
    return o.float().cpu().numpy(), s.float().cpu().numpy()


def oracle_chunk(x):
    return oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"], x.get("sparse_k"),
                                 x.get("sparse_v"), x.get("alpha"), x.get("initial_state"))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("sparse,init", [(False, False), (True, True)])
def test_chunk_matches_oracle(dtype, D, sparse, init):
    x = rand_case(2, 200, 3, D, dtype, seed=D, sparse=sparse, init=init)
    o, s = run_chunk(x)
    ro, rs = oracle_chunk(x)
    assert oracle.rel_l2(o, ro) < TOL[dtype]
    assert oracle.rel_l2(s, rs) < TOL[dtype]


@pytest.mark.parametrize("T,out_f32", [(1, False), (33, True), (1000, False), (1000, True)])
def test_sparse_write_tensor_core_path(T, out_f32, monkeypatch):
    """bf16, D=128 with the sparse write runs the tensor-core chunk kernels on the
    2T interleaved virtual samples (chunk_fwd.py:49-56) with the same-token mask
    (dep_mask = tau_j < tau_i).  Checked against the float64 oracle at the bf16
    tolerance and, with float32 outputs (two bf16-rounded outputs would carry two
    roundings), against the CUDA-core sparse path on the same inputs."""
    x = rand_case(2, T, 2, 128, torch.bfloat16, seed=T + 7, sparse=True, init=True)
    d = dev(x)
    o, s = ops.chunk_sgsa_fp32_state(d["q"], d["k"], d["v"], d["beta"], d["gamma"],
                                     d["initial_state"], d["sparse_k"], d["sparse_v"], d["alpha"],
                                     out_f32=out_f32)
    ro, rs = oracle_chunk(x)
    assert oracle.rel_l2(o.float().cpu().numpy(), ro) < 2e-3
    assert oracle.rel_l2(s.float().cpu().numpy(), rs) < 2e-3
    if not out_f32:
        return
    monkeypatch.setenv("SGSA_SCAN_SIMT", "1")  # the CUDA-core chunk kernels
    o2, s2 = ops.chunk_sgsa_fp32_state(d["q"], d["k"], d["v"], d["beta"], d["gamma"],
                                       d["initial_state"], d["sparse_k"], d["sparse_v"],
                                       d["alpha"], out_f32=out_f32)
    torch.cuda.synchronize()
    assert oracle.rel_l2(o.float().cpu().numpy(), o2.float().cpu().numpy()) < 2e-3
    assert oracle.rel_l2(s.float().cpu().numpy(), s2.float().cpu().numpy()) < 2e-3


@pytest.mark.parametrize("T", [1, 63, 64, 65, 130])
def test_chunk_ragged_lengths(T):
    x = rand_case(1, T, 2, 64, torch.float32, seed=T, sparse=True, init=True)
    o, s = run_chunk(x)
    ro, rs = oracle_chunk(x)
    assert oracle.rel_l2(o, ro) < 1e-5
    assert oracle.rel_l2(s, rs) < 1e-5


def test_chunk_mild_decay_long():
    # mild decay keeps the state large across many chunks (the regime the
    # reference's chunk path handles well); errors must not accumulate.
    x = rand_case(1, 2048, 2, 128, torch.float32, seed=5, decay="mild")
    o, s = run_chunk(x)
    ro, rs = oracle_chunk(x)
    assert oracle.rel_l2(o, ro) < 1e-5
    assert oracle.rel_l2(s, rs) < 1e-5


def test_chunk_cpu_config_fp32():
    cfg = CONFIGS["cpu_fp32"]
    x = make_inputs(cfg)
    d = dev(x)
    o, s = ops.chunk_sgsa(d["q"], d["k"], d["v"], d["beta"], d["gamma"], output_final_state=True)
    z = np.load("tests/golden/recurrent_cfg0.npz")
    assert oracle.rel_l2(o.cpu().numpy(), z["o"]) < 1e-5
    assert oracle.rel_l2(s.cpu().numpy(), z["state"]) < 1e-5


def test_chunk_empty_sequence_returns_initial_state():
    x = rand_case(1, 4, 2, 64, torch.float32, init=True)
    d = {n: t[:, :0].cuda() if t.dim() >= 3 and n != "initial_state" else t.cuda() for n, t in x.items()}
    o, s = ops.chunk_sgsa(**d, output_final_state=True)
    assert o.shape[1] == 0
    torch.testing.assert_close(s.cpu(), x["initial_state"])


def check_index_sets(got, want, iq, ik, kth, tol):
    """Exact equality, except that differing entries must be near-ties."""
    if np.array_equal(got, want):
        return 0
    B, H, T, K = got.shape
    bad = np.argwhere((got != want).any(-1))
    iqd = iq.double().numpy()
    ikd = ik.double().numpy()
    for b, h, t in bad:
        a = set(got[b, h, t][got[b, h, t] >= 0].tolist())
        w = set(want[b, h, t][want[b, h, t] >= 0].tolist())
        assert len(a) == len(w)
        for j in a ^ w:
            s = float(iqd[b, t, h] @ ikd[b, j, h])
            assert abs(s - kth[b, h, t]) <= tol * max(1.0, abs(kth[b, h, t])), (b, h, t, j)
    return len(bad)


def test_indexer_cpu_config_fp32_matches_reference_fixture():
    cfg = CONFIGS["cpu_fp32"]
    x = make_inputs(cfg)
    got = ops.indexer_topk(x["iq"].cuda(), x["ik"].cuda(), cfg.top_k).cpu().numpy()
    want, kth = oracle.indexer_topk(x["iq"], x["ik"], cfg.top_k, return_kth=True)
    z = np.load("tests/golden/indexer_cfg0.npz")
    np.testing.assert_array_equal(want, z["idx"].astype(np.int32))
    check_index_sets(got, want, x["iq"], x["ik"], kth, 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,DI,K", [(300, 64, 32), (1000, 128, 256), (129, 32, 128), (70, 64, 512)])
def test_indexer_matches_oracle(dtype, T, DI, K):
    g = torch.Generator().manual_seed(T + DI)
    iq = torch.randn(2, T, 3, DI, generator=g).to(dtype)
    ik = torch.randn(2, T, 3, DI, generator=g).to(dtype)
    got = ops.indexer_topk(iq.cuda(), ik.cuda(), K).cpu().numpy()
    want, kth = oracle.indexer_topk(iq, ik, K, return_kth=True)
    check_index_sets(got, want, iq.float(), ik.float(), kth, 1e-5)


def test_indexer_exact_ties_lowest_index():
    # integer-valued indexer vectors produce many exactly equal scores
    g = torch.Generator().manual_seed(3)
    iq = torch.randint(-2, 3, (1, 257, 2, 32), generator=g).float()
    ik = torch.randint(-2, 3, (1, 257, 2, 32), generator=g).float()
    for dtype in (torch.float32, torch.bfloat16):
        got = ops.indexer_topk(iq.to(dtype).cuda(), ik.to(dtype).cuda(), 16).cpu().numpy()
        want = oracle.indexer_topk(iq, ik, 16)
        np.testing.assert_array_equal(got, want)


def test_topk_select_bit_exact_on_identical_scores():
    g = torch.Generator().manual_seed(7)
    R, S, K = 300, 700, 64
    sc = torch.randn(R, S, generator=g)
    sc[::3] = torch.round(sc[::3] * 2)  # heavy ties on every third row
    sc[5] = 1.0                         # a row that is all ties
    sc[6] = -0.0
    valid = torch.randint(0, S + 1, (R,), generator=g).int()
    valid[:4] = torch.tensor([0, 1, K, K + 1])
    got = ops.topk_select(sc.cuda(), valid.cuda(), K).cpu().numpy()
    want = oracle.topk_select(sc.numpy(), valid.numpy(), K)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
def test_sparse_attn_mix_matches_oracle(dtype, D):
    T, K = 300, 48
    x = rand_case(2, T, 3, D, dtype, seed=11)
    g = torch.Generator().manual_seed(12)
    iq = torch.randn(2, T, 3, 32, generator=g)
    idx = oracle.indexer_topk(iq, iq.roll(1, 1), K)
    od = torch.randn(2, T, 3, D, generator=g)
    for mix in (torch.sigmoid(torch.randn(2, T, 3, D, generator=g)).to(dtype),
                torch.sigmoid(torch.randn(2, T, 3, generator=g)).to(dtype)):
        got = ops.sparse_attn_mix(x["q"].cuda(), x["k"].cuda(), x["v"].cuda(),
                                  torch.from_numpy(idx).cuda(), od.cuda(), mix.cuda())
        want = oracle.sparse_attn_mix(x["q"], x["k"], x["v"], idx, od, mix)
        assert oracle.rel_l2(got.float().cpu().numpy(), want) < TOL[dtype]


def test_sparse_attention_reference_fixture():
    z = np.load("tests/golden/sparse_attn_ref.npz")
    t = lambda a: torch.from_numpy(a).float().cuda()
    idx = ops.indexer_topk(t(z["q"]), t(z["k"]), int(z["top_k"]))
    got = ops.sparse_attn_mix(t(z["q"]), t(z["k"]), t(z["v"]), idx, t(z["o_delta"]), t(z["mix"]))
    assert oracle.rel_l2(got.cpu().numpy(), z["out"]) < 1e-5


@pytest.mark.parametrize("dtype,cfgname", [(torch.float32, "cpu_fp32"), (torch.bfloat16, "small_bf16")])
def test_layer_fwd_matches_oracle(dtype, cfgname):
    cfg = CONFIGS["cpu_fp32"] if cfgname == "cpu_fp32" else CONFIGS["b200_bf16"].scaled(
        name="small_bf16", B=1, T=1024, H=4)
    x = make_inputs(cfg)
    d = dev(x)
    out, st, idx = ops.sgsa_layer_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"],
                                      d["ik"], d["mix"], cfg.top_k, output_final_state=True,
                                      return_indices=True)
    ro, rs = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"])
    want_idx, kth = oracle.indexer_topk(x["iq"], x["ik"], cfg.top_k, return_kth=True)
    got_idx = idx.cpu().numpy()
    check_index_sets(got_idx, want_idx, x["iq"].float(), x["ik"].float(), kth, 1e-5)
    # score the composite on the device's own index sets so a near-tie swap
    # does not leak into the output comparison
    want = oracle.sparse_attn_mix(x["q"], x["k"], x["v"], got_idx, ro, x["mix"])
    assert oracle.rel_l2(out.float().cpu().numpy(), want) < TOL[dtype]
    assert oracle.rel_l2(st.cpu().numpy(), rs) < TOL[dtype]


def test_watchdog_clear_after_suite():
    from sgsa_b200 import _lib
    assert _lib.load().sgsa_watchdog_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("T,DI,K", [(1000, 64, 100), (777, 128, 64), (4096, 64, 512)])
def test_indexer_tc_matches_simt_bitwise_sets(T, DI, K, monkeypatch):
    """The tensor-core and CUDA-core score paths select the same sets (up to near ties)."""
    g = torch.Generator().manual_seed(T)
    iq = torch.randn(2, T, 2, DI, generator=g).bfloat16()
    ik = torch.randn(2, T, 2, DI, generator=g).bfloat16()
    got = ops.indexer_topk(iq.cuda(), ik.cuda(), K).cpu().numpy()
    want, kth = oracle.indexer_topk(iq, ik, K, return_kth=True)
    check_index_sets(got, want, iq.float(), ik.float(), kth, 1e-5)


def test_indexer_max_length_rows():
    """T = 65536 (the long-context length; 32-bit histogram path): the heaviest
    rows and a few early ones against the oracle."""
    T, DI, K = 65536, 64, 2048
    g = torch.Generator().manual_seed(99)
    iq = torch.randn(1, T, 1, DI, generator=g).bfloat16()
    ik = torch.randn(1, T, 1, DI, generator=g).bfloat16()
    got = ops.indexer_topk(iq.cuda(), ik.cuda(), K).cpu().numpy()
    for t0, t1 in ((T - 48, T), (2040, 2060), (30000, 30016)):
        want, kth = oracle.indexer_topk(iq, ik, K, t_range=(t0, t1), return_kth=True)
        sub = got[:, :, t0:t1]
        iqd, ikd = iq.double().numpy(), ik.double().numpy()
        for b, h, tt in np.argwhere((sub != want).any(-1)):
            a = set(sub[b, h, tt].tolist()) - {-1}
            w = set(want[b, h, tt].tolist()) - {-1}
            assert len(a) == len(w)
            for j in a ^ w:
                s = float(iqd[b, t0 + tt, h] @ ikd[b, j, h])
                assert abs(s - kth[b, h, tt]) <= 1e-5 * max(1.0, abs(kth[b, h, tt]))


@pytest.mark.parametrize("kind", ["negative", "huge", "tiny", "mixed"])
def test_indexer_tc_score_ranges(kind):
    """Scores outside the fast first-digit window (all negative, > 2^16, < 2^-16)
    take the plain radix path; results stay exact."""
    g = torch.Generator().manual_seed(17)
    T, DI, K = 600, 64, 64
    iq = torch.randn(1, T, 2, DI, generator=g)
    ik = torch.randn(1, T, 2, DI, generator=g)
    if kind == "negative":
        iq, ik = -iq.abs(), ik.abs()
    elif kind == "huge":
        iq, ik = iq * 1e3, ik * 1e3
    elif kind == "tiny":
        iq, ik = iq * 1e-4, ik * 1e-4
    else:
        iq[:, ::2] *= 1e3
    iq, ik = iq.bfloat16(), ik.bfloat16()
    got = ops.indexer_topk(iq.cuda(), ik.cuda(), K).cpu().numpy()
    want, kth = oracle.indexer_topk(iq, ik, K, return_kth=True)
    check_index_sets(got, want, iq.float(), ik.float(), kth, 1e-5)


@pytest.mark.parametrize("B,T,H,K", [(1, 1000, 2, 64), (2, 2048, 2, 512), (1, 4096, 1, 300)])
def test_layer_fused_attention_matches_gather_and_oracle(B, T, H, K, monkeypatch):
    """The tensor-core attention (selection applied as the indexer's exact
    per-row threshold) against the row-gather path and the oracle."""
    cfg = CONFIGS["b200_bf16"].scaled(name="fused", B=B, T=T, H=H, top_k=K)
    x = make_inputs(cfg, seed=3)
    d = dev(x)
    args = (d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"], d["mix"], K)
    fused, idx = ops.sgsa_layer_fwd(*args, return_indices=True)
    monkeypatch.setenv("SGSA_ATTN_GATHER", "1")
    gather, idx2 = ops.sgsa_layer_fwd(*args, return_indices=True)
    assert torch.equal(idx, idx2)
    assert oracle.rel_l2(fused.float().cpu().numpy(), gather.float().cpu().numpy()) < 2e-3
    ro, _ = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"])
    want = oracle.sparse_attn_mix(x["q"], x["k"], x["v"], idx.cpu().numpy(), ro, x["mix"])
    assert oracle.rel_l2(fused.float().cpu().numpy(), want) < 2e-3


def test_layer_fused_attention_with_exact_score_ties(monkeypatch):
    """Integer-valued indexer vectors make many k-th scores exact ties, so the
    threshold carries a tie cut; the fused path must still select exactly the
    rows the index-writing path selects."""
    cfg = CONFIGS["b200_bf16"].scaled(name="ties", B=1, T=1500, H=2, top_k=100)
    x = make_inputs(cfg, seed=4)
    g = torch.Generator().manual_seed(5)
    x["iq"] = torch.randint(-2, 3, x["iq"].shape, generator=g).bfloat16()
    x["ik"] = torch.randint(-2, 3, x["ik"].shape, generator=g).bfloat16()
    d = dev(x)
    args = (d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"], d["mix"], cfg.top_k)
    fused = ops.sgsa_layer_fwd(*args)
    monkeypatch.setenv("SGSA_ATTN_GATHER", "1")
    gather, idx = ops.sgsa_layer_fwd(*args, return_indices=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.indexer_topk(x["iq"], x["ik"], cfg.top_k))
    assert oracle.rel_l2(fused.float().cpu().numpy(), gather.float().cpu().numpy()) < 2e-3


@pytest.mark.parametrize("norm", [1.0, 30.0])
def test_fused_attention_bound_and_running_max(norm):
    """Unit-norm q, k take the fixed-bound softmax; norms of 30 (scores up to ~114 in
    log2 units) take the per-group running maximum.  Both against the oracle on the
    device's own index sets."""
    cfg = CONFIGS["b200_bf16"].scaled(name="bound", B=1, T=1000, H=2, top_k=128)
    x = make_inputs(cfg, seed=12)
    x["q"] = (x["q"].float() * norm).bfloat16()
    x["k"] = (x["k"].float() * norm).bfloat16()
    d = dev(x)
    thr = ops.indexer_thresholds(d["iq"], d["ik"], cfg.top_k)
    got = ops.sparse_attn_thresholds(d["q"], d["k"], d["v"], d["iq"], d["ik"], thr, out_f32=True)
    idx = ops.indexer_topk(d["iq"], d["ik"], cfg.top_k).cpu().numpy()
    want = oracle.sparse_attn_mix(x["q"], x["k"], x["v"], idx)
    assert oracle.rel_l2(got.cpu().numpy(), want) < 1e-4


def test_layer_from_host_matches_device_call():
    cfg = CONFIGS["b200_bf16"].scaled(name="host", B=2, T=1024, H=2, top_k=128)
    x = make_inputs(cfg, seed=6)
    names = ["q", "k", "v", "beta", "gamma", "iq", "ik", "mix"]
    host = [x[n].pin_memory() for n in names]
    got = ops.sgsa_layer_fwd_from_host(*host, cfg.top_k)
    torch.cuda.synchronize()
    want = ops.sgsa_layer_fwd(*[x[n].cuda() for n in names], cfg.top_k).cpu()
    assert torch.equal(got, want)


@pytest.mark.parametrize("gather", [False, True])
def test_layer_shared_indexer(gather, monkeypatch):
    """One index set per token shared by all heads (iq, ik with a single head)."""
    cfg = CONFIGS["b200_bf16"].scaled(name="shared", B=2, T=1024, H=4, top_k=128)
    x = make_inputs(cfg, seed=10)
    x["iq"], x["ik"] = x["iq"][:, :, :1].contiguous(), x["ik"][:, :, :1].contiguous()
    if gather:
        monkeypatch.setenv("SGSA_ATTN_GATHER", "1")
    d = dev(x)
    out, idx = ops.sgsa_layer_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"],
                                  d["mix"], cfg.top_k, return_indices=True)
    assert idx.shape == (2, 1, 1024, 128)
    want_idx, kth = oracle.indexer_topk(x["iq"], x["ik"], cfg.top_k, return_kth=True)
    check_index_sets(idx.cpu().numpy(), want_idx, x["iq"].float(), x["ik"].float(), kth, 1e-5)
    ro, _ = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"])
    idx_h = np.repeat(idx.cpu().numpy(), cfg.H, axis=1)
    want = oracle.sparse_attn_mix(x["q"], x["k"], x["v"], idx_h, ro, x["mix"])
    assert oracle.rel_l2(out.float().cpu().numpy(), want) < 2e-3


def test_sparse_retrieve_reference_fixture():
    z = np.load("tests/golden/retriever_token.npz")
    t = lambda a: torch.from_numpy(a).float().cuda()
    idx = ops.indexer_topk(t(z["q"]), t(z["k"]), int(z["top_k"]))
    kh, vh = ops.sparse_retrieve(t(z["q"]), t(z["k"]), t(z["v"]), idx)
    assert oracle.rel_l2(kh.cpu().numpy(), z["k_hat"]) < 1e-5
    assert oracle.rel_l2(vh.cpu().numpy(), z["v_hat"]) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])  # bf16 at 128: the tensor-core chunk kernels
def test_sparse_write_block_matches_oracle(dtype, D):
    """Retrieval (q . k top-k), k_hat / v_hat, then the delta rule with the sparse write.

    The two halves are pinned separately at the plain tolerance: the retrieval
    against the oracle's k_hat / v_hat, and the recurrence with the sparse write
    against the oracle fed the device's own (dtype-rounded) k_hat / v_hat, so the
    rounding of k_hat to the input dtype is not charged to the recurrence."""
    x = rand_case(2, 300, 2, D, dtype, seed=21, sparse=True, init=True)
    K = 32
    d = dev(x)
    o, st = ops.sgsa_sparse_write_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["alpha"],
                                      K, initial_state=d["initial_state"],
                                      output_final_state=True)
    idx_dev = ops.indexer_topk(d["q"], d["k"], K)
    idx, kth = oracle.indexer_topk(x["q"], x["k"], K, return_kth=True)
    check_index_sets(idx_dev.cpu().numpy(), idx, x["q"].float(), x["k"].float(), kth, 1e-5)
    kh_dev, vh_dev = ops.sparse_retrieve(d["q"], d["k"], d["v"], idx_dev)
    kh, vh = oracle.sparse_retrieve(x["k"], x["v"], idx_dev.cpu().numpy(), x["q"])
    assert oracle.rel_l2(kh_dev.float().cpu().numpy(), kh) < TOL[dtype]
    assert oracle.rel_l2(vh_dev.float().cpu().numpy(), vh) < TOL[dtype]
    ro, rs = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"], kh_dev.cpu(),
                                   vh_dev.cpu(), x["alpha"], x["initial_state"])
    assert oracle.rel_l2(o.float().cpu().numpy(), ro) < TOL[dtype]
    assert oracle.rel_l2(st.float().cpu().numpy(), rs) < TOL[dtype]


@pytest.mark.parametrize("dtype,cfgname", [(torch.bfloat16, "bf16"), (torch.float32, "fp32")])
def test_layer_delta_stage_in_pair_groups_is_identical(dtype, cfgname, monkeypatch):
    """A workspace cap that splits the delta stage into groups of (batch, head) pairs
    changes nothing: the same kernels run on each pair."""
    cfg = CONFIGS["b200_bf16"].scaled(name="groups", B=2, T=1024, H=3, top_k=128, dtype=dtype)
    if dtype == torch.float32:
        cfg = cfg.scaled(D=64, d_idx=32)
    x = make_inputs(cfg, seed=14)
    d = dev(x)
    args = (d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"], d["mix"], cfg.top_k)
    out, st = ops.sgsa_layer_fwd(*args, output_final_state=True)
    from sgsa_b200 import _lib
    lib = _lib.load()
    per_pair = lib.sgsa_chunk_fwd_workspace_size(1, cfg.T, 1, cfg.D, 0)
    monkeypatch.setenv("SGSA_LAYER_DELTA_CAP", str(2 * per_pair + 256))  # groups of 2 pairs
    ops.release_workspaces()
    out2, st2 = ops.sgsa_layer_fwd(*args, output_final_state=True)
    assert torch.equal(out, out2)
    assert torch.equal(st, st2)
