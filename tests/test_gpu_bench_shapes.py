"""Parity at the benchmarked shapes, and the selector on the device's own scores.

* configs[1] at full shape (B4 T8192 H16 d128, top-k 512, DI 64, bf16): the call
  bench.py times, against the float64 oracle on batch row 0 (all heads): output and
  final state within relative L2 2e-3, index sets on 256 sampled rows per head.
* configs[2] on 2 heads (T 65536, top-k 2048): final state over all 1024 chunks,
  output rows sampled across the sequence, index sets on sampled rows.
* configs[4] at full size (batch 64, 32768-token cache, H16, top-k 1024, reuse 4):
  a few decode steps, checked on sampled batch rows against a step-by-step oracle.
* The tensor-core selector on its own fp32 scores: the scores the kernel selected
  from are written out and the oracle's select on those very scores (ties to the
  lowest index, modelings/modeling_sgsa.py:155-164) must give the same index rows
  bit for bit -- no near-tie band.

Index sets against the float64 oracle are exact except for near ties of the k-th
score (|s - s_k| <= 1e-5 |s_k|), where bf16-input fp32 MMA scores and float64
scores may order two keys differently.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from sgsa_b200 import _lib, ops
from sgsa_b200.inputs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-3


def near_tie_sets(got, want, iq, ik, kth, t0, tol=1e-5):
    """got/want [B, H, n, K] for rows t0 .. t0+n; differing keys must be near ties."""
    bad = np.argwhere((got != want).any(-1))
    iqd, ikd = iq.double().numpy(), ik.double().numpy()
    for b, h, tt in bad:
        a = set(got[b, h, tt].tolist()) - {-1}
        w = set(want[b, h, tt].tolist()) - {-1}
        assert len(a) == len(w), (b, h, tt)
        for j in a ^ w:
            s = float(iqd[b, t0 + tt, h] @ ikd[b, j, h])
            assert abs(s - kth[b, h, tt]) <= tol * max(1.0, abs(kth[b, h, tt])), (b, h, t0 + tt, j)
    return len(bad)


def test_layer_configs1_full_shape():
    cfg = CONFIGS["b200_bf16"]
    x = make_inputs(cfg, seed=0)  # the inputs bench.py times on rank 0
    d = {n: t.cuda() for n, t in x.items()}
    args = (d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"], d["mix"], cfg.top_k)
    timed = ops.sgsa_layer_fwd(*args)  # exactly the benchmarked call
    out, st, idx = ops.sgsa_layer_fwd(*args, output_final_state=True, return_indices=True)
    assert torch.equal(out, timed)
    xb = {n: t[:1] for n, t in x.items()}
    ro, rs = oracle.sgsa_recurrent(xb["q"], xb["k"], xb["v"], xb["beta"], xb["gamma"])
    assert oracle.rel_l2(st[:1].cpu().numpy(), rs) < BF16_TOL
    gi = idx[:1].cpu().numpy()
    want = oracle.sparse_attn_mix(xb["q"], xb["k"], xb["v"], gi, ro, xb["mix"])
    e_out = oracle.rel_l2(out[:1].float().cpu().numpy(), want)
    assert e_out < BF16_TOL, e_out
    rows = 0
    for t0 in (511, 2000, 5000, cfg.T - 64):  # 4 x 64 = 256 rows per head
        w, kth = oracle.indexer_topk(xb["iq"], xb["ik"], cfg.top_k, t_range=(t0, t0 + 64),
                                     return_kth=True)
        near_tie_sets(gi[:, :, t0:t0 + 64], w, xb["iq"], xb["ik"], kth, t0)
        rows += 64
    assert rows >= 256


def test_layer_configs2_two_heads():
    cfg = CONFIGS["long_ctx"].scaled(name="long_h2", H=2)
    x = make_inputs(cfg, seed=0)
    d = {n: t.cuda() for n, t in x.items()}
    out, st, idx = ops.sgsa_layer_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"],
                                      d["ik"], d["mix"], cfg.top_k, output_final_state=True,
                                      return_indices=True)
    ro, rs = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"])
    assert oracle.rel_l2(st.cpu().numpy(), rs) < BF16_TOL
    gi = idx.cpu().numpy()
    of = out.float().cpu().numpy()
    for t0 in (0, 2040, 30000, cfg.T - 256):
        t1 = t0 + 256
        want = oracle.sparse_attn_mix(x["q"], x["k"], x["v"], gi[:, :, t0:t1], ro, x["mix"],
                                      t_range=(t0, t1))
        assert oracle.rel_l2(of[:, t0:t1], want) < BF16_TOL, t0
    for t0 in (2040, 40000, cfg.T - 32):
        w, kth = oracle.indexer_topk(x["iq"], x["ik"], cfg.top_k, t_range=(t0, t0 + 32),
                                     return_kth=True)
        near_tie_sets(gi[:, :, t0:t0 + 32], w, x["iq"], x["ik"], kth, t0)


def test_decode_configs4_full_size():
    """batch 64, 32768-token cache, H16, d128, top-k 1024, refresh every 4
    steps, 256 planted keys per sequence; decode steps through DecodeCache, checked on
    sampled batch rows against the oracle (selection refreshed on the same steps)."""
    B, H, D, DI, Tc, K, reuse, nplant = 64, 16, 128, 64, 32768, 1024, 4, 256
    steps = 5
    n0 = Tc - steps - 1
    g = torch.Generator(device="cuda").manual_seed(0)  # the caches are 8.6 GB each in bf16
    r = lambda *s: torch.randn(*s, generator=g, device="cuda")
    bf = torch.bfloat16
    kc = torch.nn.functional.normalize(r(B, Tc, H, D), dim=-1).to(bf)
    vc = r(B, Tc, H, D).to(bf)
    ikc = r(B, Tc, H, DI)
    pos = torch.randint(0, n0, (B, nplant), generator=g, device="cuda")
    ikc[torch.arange(B, device="cuda")[:, None], pos] = 4.0 * r(B, nplant, H, DI)
    ikc = ikc.to(bf)
    s0 = 0.1 * r(B, H, D, D)
    target = pos[torch.arange(B, device="cuda"),
                 torch.randint(0, nplant, (B,), generator=g, device="cuda")]
    rows = [0, 37]  # batch rows checked against the oracle
    kc_o, vc_o, ikc_o = kc[rows].cpu(), vc[rows].cpu(), ikc[rows].cpu()
    state = s0[rows].cpu().numpy()
    cache = ops.DecodeCache(kc, vc, ikc, n0, s0, K, reuse=reuse)
    idx = None
    hits = []
    for step in range(steps):
        q = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(bf)
        k = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(bf)
        v = r(B, H, D).to(bf)
        beta = torch.sigmoid(r(B, H)).to(bf)
        gamma = torch.exp(-torch.nn.functional.softplus(r(B, H))).to(bf)
        iq = ikc[torch.arange(B, device="cuda"), target].clone()  # aligned with a planted key
        ik = r(B, H, DI).to(bf)
        mix = torch.sigmoid(r(B, H, D)).to(bf)
        got = cache.step(q, k, v, beta, gamma, iq, ik, mix)
        hits.append((cache.indices == target[:, None, None].int()).any(-1).float().mean().item())
        sub = lambda t: t[rows].cpu()
        od, state = oracle.sgsa_recurrent(sub(q)[:, None], sub(k)[:, None], sub(v)[:, None],
                                          sub(beta)[:, None], sub(gamma)[:, None],
                                          initial_state=state)
        n = n0 + step
        kc_o[:, n], vc_o[:, n], ikc_o[:, n] = sub(k), sub(v), sub(ik)
        if step % reuse == 0:
            idx, kth = oracle.decode_topk(sub(iq), ikc_o, n + 1, K, return_kth=True)
            gi = cache.indices[rows].cpu().numpy()
            if not np.array_equal(gi, idx):  # refresh step: exact up to near ties
                s = np.einsum("bhd,bjhd->bhj", sub(iq).double().numpy(),
                              ikc_o.double().numpy()[:, :n + 1])
                for b, h in np.argwhere((gi != idx).any(-1)):
                    for j in set(gi[b, h].tolist()) ^ set(idx[b, h].tolist()):
                        assert abs(s[b, h, j] - kth[b, h]) <= 1e-5 * max(1.0, abs(kth[b, h]))
            idx = gi  # score the attention on the device's own selection
        want = oracle.decode_attn_mix(sub(q), kc_o, vc_o, idx, od[:, 0], sub(mix))
        assert oracle.rel_l2(sub(got).float().numpy(), want) < BF16_TOL
    assert min(hits) == 1.0  # every planted key retrieved on every step


def _selector_inputs(T, DI, kind, seed):
    g = torch.Generator().manual_seed(seed)
    B, H = 1, 2
    iq = torch.randn(B, T, H, DI, generator=g)
    ik = torch.randn(B, T, H, DI, generator=g)
    if kind == "shifted":  # most scores of one sign, k-th near zero (sign-unclear window)
        iq, ik = iq + 0.3, ik + 0.3
    elif kind == "ties":
        iq = torch.randint(-2, 3, iq.shape, generator=g).float()
        ik = torch.randint(-2, 3, ik.shape, generator=g).float()
    elif kind == "wide":  # rows whose score scale varies by 2^10
        iq = iq * torch.exp2(torch.randint(-5, 6, (B, T, H, 1), generator=g).float())
    elif kind == "late_keys":  # keys after the sampled first tile 2^10 larger: window misses
        ik[:, 64:] *= 1024.0
    elif kind == "cluster":  # every score close to 64: a few window bins of ~700 keys
        iq = torch.ones(B, T, H, DI) + 0.02 * iq
        ik = torch.ones(B, T, H, DI) + 0.02 * ik
    return iq.bfloat16().cuda(), ik.bfloat16().cuda()


@pytest.mark.parametrize("T,DI,K,kind", [(1024, 64, 128, "normal"), (2048, 64, 512, "normal"),
                                         (1536, 128, 256, "shifted"), (1024, 64, 100, "ties"),
                                         (777, 64, 64, "wide"), (4096, 64, 512, "normal"),
                                         (1024, 64, 128, "late_keys"), (2048, 64, 300, "cluster")])
def test_tc_selector_bit_exact_on_its_own_scores(T, DI, K, kind):
    B, H = 1, 2
    iq, ik = _selector_inputs(T, DI, kind, T + K)
    idx = torch.empty(B, H, T, K, dtype=torch.int32, device="cuda")
    sc = torch.zeros(B, H, T, T, dtype=torch.float32, device="cuda")
    lib = _lib.load()
    rc = lib.sgsa_indexer_topk_scores(iq.data_ptr(), ik.data_ptr(), idx.data_ptr(),
                                      sc.data_ptr(), B, T, H, DI, K,
                                      torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "sgsa_indexer_topk_scores")
    # the same call without the score dump selects the same rows
    assert torch.equal(idx, ops.indexer_topk(iq, ik, K))
    t = torch.arange(T, dtype=torch.int32)
    rows = sc.reshape(B * H * T, T).cpu().numpy()
    valid = np.tile((t + 1).numpy(), B * H)
    got = idx.reshape(B * H * T, K).cpu().numpy()
    long_rows = valid > K  # shorter rows keep every column (not dumped)
    want = oracle.topk_select(rows[long_rows], valid[long_rows], K)
    np.testing.assert_array_equal(got[long_rows], want)
    short = got[~long_rows]
    expect = np.where(np.arange(K)[None, :] < valid[~long_rows][:, None], np.arange(K)[None, :], -1)
    np.testing.assert_array_equal(short, expect)


def test_tc_selector_paths_are_exercised():
    """The refine pass, the plain restart and exact ties all occur on these inputs
    (counted by the kernel) -- so the bit-exact test above covers them."""
    lib = _lib.load()
    counts = (ctypes.c_ulonglong * 4)()
    seen = {}
    for kind, T, K in (("cluster", 2048, 300), ("late_keys", 1024, 128), ("ties", 1024, 100)):
        iq, ik = _selector_inputs(T, 64, kind, 5)
        _lib.check(lib.sgsa_indexer_stats(counts, 1), "stats")
        ops.indexer_topk(iq, ik, K)
        _lib.check(lib.sgsa_indexer_stats(counts, 1), "stats")
        seen[kind] = list(counts)
    assert seen["cluster"][0] > 0, seen      # refine pass
    assert seen["late_keys"][1] > 0, seen    # plain restart
    assert seen["ties"][3] > 0, seen         # exact ties at the k-th score


@pytest.mark.parametrize("T,K,kind", [(1024, 128, "normal"), (2000, 300, "ties"), (777, 64, "wide")])
def test_attention_recomputes_the_indexer_scores_bit_for_bit(T, K, kind):
    """The fused attention selects with the indexer's thresholds on scores it
    recomputes; both kernels use the same MMA sequence, so the scores must be
    bit-identical (else a near-threshold key could be selected differently)."""
    iq, ik = _selector_inputs(T, 64, kind, 7)
    B, H = iq.shape[0], iq.shape[2]
    g = torch.Generator().manual_seed(8)
    qkv = [torch.nn.functional.normalize(torch.randn(B, T, H, 128, generator=g), dim=-1)
           .bfloat16().cuda() for _ in range(3)]
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    idx = torch.empty(B, H, T, K, dtype=torch.int32, device="cuda")
    s_idx = torch.full((B, H, T, T), float("nan"), device="cuda")
    _lib.check(lib.sgsa_indexer_topk_scores(iq.data_ptr(), ik.data_ptr(), idx.data_ptr(),
                                            s_idx.data_ptr(), B, T, H, 64, K, st), "indexer")
    thr = ops.indexer_thresholds(iq, ik, K)
    out = torch.empty(B, T, H, 128, device="cuda")
    s_att = torch.full((B, H, T, T), float("nan"), device="cuda")
    _lib.check(lib.sgsa_sparse_attn_index_scores(qkv[0].data_ptr(), qkv[1].data_ptr(),
                                                 qkv[2].data_ptr(), iq.data_ptr(), ik.data_ptr(),
                                                 thr.data_ptr(), out.data_ptr(), s_att.data_ptr(),
                                                 B, T, H, st), "attention")
    torch.cuda.synchronize()
    written = ~torch.isnan(s_idx)  # rows the indexer had to select in (t + 1 > K)
    assert written.sum() > 0
    assert torch.equal(s_idx[written].view(torch.int32), s_att[written].view(torch.int32))
