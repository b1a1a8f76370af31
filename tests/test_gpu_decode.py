"""Recurrent forward and decode-time ops (through the C ABI) against the oracle.

Tolerances as in test_gpu_parity: relative L2 1e-5 (float32) / 2e-3 (bfloat16);
index sets exact up to near ties of the k-th score.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from sgsa_b200 import ops

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-3}


def _gen(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda *s: torch.randn(*s, generator=g)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("sparse", [False, True])
@pytest.mark.parametrize("T", [97, 1])  # T == 1 is the decode step's kernel
def test_fused_recurrent_matches_oracle(dtype, D, sparse, T):
    r = _gen(D + sparse)
    B, H = 2, 3
    x = dict(q=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
             k=torch.nn.functional.normalize(r(B, T, H, D), dim=-1), v=r(B, T, H, D),
             beta=torch.sigmoid(r(B, T, H)),
             gamma=torch.exp(-torch.nn.functional.softplus(r(B, T, H))))
    if sparse:
        x.update(sparse_k=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
                 sparse_v=r(B, T, H, D), alpha=0.25 * torch.sigmoid(r(B, T, H)))
    x = {n: t.to(dtype) for n, t in x.items()}
    s0 = 0.1 * r(B, H, D, D)
    o, st = ops.fused_recurrent_sgsa(**{n: t.cuda() for n, t in x.items()},
                                     initial_state=s0.cuda(), output_final_state=True)
    ro, rs = oracle.sgsa_recurrent(x["q"], x["k"], x["v"], x["beta"], x["gamma"],
                                   x.get("sparse_k"), x.get("sparse_v"), x.get("alpha"), s0)
    assert st.dtype == torch.float32
    assert oracle.rel_l2(o.float().cpu().numpy(), ro) < TOL[dtype]
    assert oracle.rel_l2(st.cpu().numpy(), rs) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,K,DI", [(700, 64, 64), (3000, 1024, 64), (50, 128, 32), (2048, 2048, 128)])
def test_decode_topk_matches_oracle(dtype, n, K, DI):
    r = _gen(n + K)
    B, H, Tc = 2, 3, max(n, 64) + 5
    iq = r(B, H, DI).to(dtype)
    ikc = r(B, Tc, H, DI).to(dtype)
    got = ops.decode_topk(iq.cuda(), ikc.cuda(), n, K).cpu().numpy()
    want, kth = oracle.decode_topk(iq, ikc, n, K, return_kth=True)
    if not np.array_equal(got, want):
        s = np.einsum("bhd,bjhd->bhj", iq.double().numpy(), ikc.double().numpy()[:, :n])
        for b, h in np.argwhere((got != want).any(-1)):
            a, w = set(got[b, h].tolist()) - {-1}, set(want[b, h].tolist()) - {-1}
            assert len(a) == len(w)
            for j in a ^ w:
                assert abs(s[b, h, j] - kth[b, h]) <= 1e-5 * max(1.0, abs(kth[b, h]))


def test_decode_topk_ties_lowest_index():
    g = torch.Generator().manual_seed(9)
    iq = torch.randint(-1, 2, (1, 2, 32), generator=g).float()
    ikc = torch.randint(-1, 2, (1, 900, 2, 32), generator=g).float()
    got = ops.decode_topk(iq.cuda(), ikc.cuda(), 900, 40).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.decode_topk(iq, ikc, 900, 40))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
def test_decode_attn_matches_oracle(dtype, D):
    r = _gen(D)
    B, H, Tc, K, n = 2, 3, 1500, 256, 1200
    q = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(dtype)
    kc = torch.nn.functional.normalize(r(B, Tc, H, D), dim=-1).to(dtype)
    vc = r(B, Tc, H, D).to(dtype)
    idx = oracle.decode_topk(r(B, H, 32), r(B, Tc, H, 32), n, K)
    idx[0, 0, 100:] = -1  # a short row
    od, mix = r(B, H, D), torch.sigmoid(r(B, H, D)).to(dtype)
    got = ops.decode_attn_mix(q.cuda(), kc.cuda(), vc.cuda(), torch.from_numpy(idx).cuda(),
                              od.cuda(), mix.cuda())
    want = oracle.decode_attn_mix(q, kc, vc, idx, od, mix)
    assert oracle.rel_l2(got.float().cpu().numpy(), want) < TOL[dtype]


@pytest.mark.parametrize("reuse", [1, 4])
def test_decode_cache_steps_match_oracle(reuse):
    """Several decode steps through DecodeCache against a step-by-step oracle that
    refreshes the selection on the same steps."""
    r = _gen(reuse)
    B, H, D, DI, Tc, n0, K = 2, 2, 128, 64, 600, 500, 64
    dtype = torch.bfloat16
    kc = torch.nn.functional.normalize(r(B, Tc, H, D), dim=-1).to(dtype)
    vc = r(B, Tc, H, D).to(dtype)
    ikc = r(B, Tc, H, DI).to(dtype)
    s0 = 0.1 * r(B, H, D, D)
    cache = ops.DecodeCache(kc.clone().cuda(), vc.clone().cuda(), ikc.clone().cuda(), n0,
                            s0.cuda(), K, reuse=reuse)
    state = s0.numpy()
    kc_o, vc_o, ikc_o = kc.clone(), vc.clone(), ikc.clone()
    idx = None
    for step in range(6):
        q = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(dtype)
        k = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(dtype)
        v = r(B, H, D).to(dtype)
        beta = torch.sigmoid(r(B, H)).to(dtype)
        gamma = torch.exp(-torch.nn.functional.softplus(r(B, H))).to(dtype)
        iq, ik = r(B, H, DI).to(dtype), r(B, H, DI).to(dtype)
        mix = torch.sigmoid(r(B, H, D)).to(dtype)
        got = cache.step(*(t.cuda() for t in (q, k, v, beta, gamma, iq, ik, mix)))
        od, state = oracle.sgsa_recurrent(q[:, None], k[:, None], v[:, None], beta[:, None],
                                          gamma[:, None], initial_state=state)
        n = n0 + step
        kc_o[:, n], vc_o[:, n], ikc_o[:, n] = k, v, ik
        if step % reuse == 0:
            idx = oracle.decode_topk(iq, ikc_o, n + 1, K)
        want = oracle.decode_attn_mix(q, kc_o, vc_o, idx, od[:, 0], mix)
        assert oracle.rel_l2(got.float().cpu().numpy(), want) < 2e-3


def test_decode_topk_at_the_longest_cache():
    """The longest cache the refresh accepts (every score of a row in shared memory)
    runs and matches the oracle; one more row is refused."""
    import ctypes

    from sgsa_b200 import _lib

    lib = _lib.load()
    n = 54 * 1024
    r = _gen(7)
    iq = r(1, 1, 64).to(torch.bfloat16)
    ikc = r(1, n, 1, 64).to(torch.bfloat16)
    got = ops.decode_topk(iq.cuda(), ikc.cuda(), n, 256).cpu().numpy()
    want, kth = oracle.decode_topk(iq, ikc, n, 256, return_kth=True)
    if not np.array_equal(got, want):
        s = np.einsum("bhd,bjhd->bhj", iq.double().numpy(), ikc.double().numpy())
        a, w = set(got[0, 0].tolist()), set(want[0, 0].tolist())
        for j in a ^ w:
            assert abs(s[0, 0, j] - kth[0, 0]) <= 1e-5 * max(1.0, abs(kth[0, 0]))
    big = torch.zeros(1, n + 1, 1, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1, 1, 256, dtype=torch.int32, device="cuda")
    rc = lib.sgsa_decode_topk(iq.cuda().data_ptr(), big.data_ptr(), out.data_ptr(), 1, 1, n + 1,
                              n + 1, 64, 256, _lib.DTYPE_BF16,
                              torch.cuda.current_stream().cuda_stream)
    assert rc == -6  # SGSA_ERR_UNSUPPORTED


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_append_matches_indexing(dtype):
    """sgsa_decode_append writes exactly row `pos` of the three caches (the same result as
    tensor indexing) and refuses a position outside the cache."""
    from sgsa_b200 import _lib

    r = _gen(11)
    B, Tc, H, D, DI = 3, 50, 4, 128, 64
    kc, vc, ikc = (r(B, Tc, H, D).to(dtype).cuda(), r(B, Tc, H, D).to(dtype).cuda(),
                   r(B, Tc, H, DI).to(dtype).cuda())
    want = [t.clone() for t in (kc, vc, ikc)]
    k, v, ik = r(B, H, D).to(dtype).cuda(), r(B, H, D).to(dtype).cuda(), r(B, H, DI).to(dtype).cuda()
    for pos in (0, 17, Tc - 1):
        ops.decode_append(kc, vc, ikc, k, v, ik, pos)
        want[0][:, pos], want[1][:, pos], want[2][:, pos] = k, v, ik
    torch.cuda.synchronize()
    for got, w in zip((kc, vc, ikc), want):
        assert torch.equal(got, w)
    lib = _lib.load()
    rc = lib.sgsa_decode_append(kc.data_ptr(), vc.data_ptr(), ikc.data_ptr(), k.data_ptr(),
                                v.data_ptr(), ik.data_ptr(), B, Tc, H, D, DI, Tc,
                                _lib.DTYPE_F32 if dtype == torch.float32 else _lib.DTYPE_BF16,
                                torch.cuda.current_stream().cuda_stream)
    assert rc != 0
