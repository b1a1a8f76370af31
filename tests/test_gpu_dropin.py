"""Drop-in proof: the reference's own SGSA layer with its chunk op swapped for ours.

The reference's SGSAStateLayer.forward (modelings/modeling_sgsa.py:522-619) calls the
module-level name ``chunk_sgsa`` on its ``torch_chunk`` backend (:583-596).  This test
replaces that name with ``sgsa_b200.chunk_sgsa`` -- the one-line integration a user
makes -- and runs the unmodified layer against the same layer on its ``python``
backend (``naive_recurrent_sgsa``, :597-609) in float64, for the write modes
"none", "direct" and "residual" (the sparse write with k_hat / v_hat).

It needs the reference installed under baseline/_ref (baseline/install_reference.sh);
without it the test is skipped.
"""
import copy
import os
import sys

import pytest
import torch

import sgsa_b200

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "modelings")):
        pytest.skip("reference not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import modelings.modeling_sgsa as m
    return m


@pytest.mark.parametrize("mode", ["none", "direct", "residual"])
@pytest.mark.parametrize("hidden,heads", [(256, 4), (512, 4)])  # head dim 64 and 128
def test_sgsa_state_layer_with_swapped_chunk_op(ref, monkeypatch, mode, hidden, heads):
    torch.manual_seed(0)
    B, T = 2, 300
    cfg = ref.SGSAConfig(hidden_size=hidden, num_attention_heads=heads, num_kv_heads=heads,
                         sgsa_write_mode=mode, linear_backend="torch_chunk")
    layer = ref.SGSAStateLayer(cfg).cuda().eval()
    py_cfg = copy.deepcopy(cfg)
    py_cfg.linear_backend = "python"
    py_layer = ref.SGSAStateLayer(py_cfg).cuda().eval()
    py_layer.load_state_dict(layer.state_dict())
    D = cfg.head_dim
    hs = torch.randn(B, T, hidden, device="cuda")
    q = torch.nn.functional.normalize(torch.randn(B, T, heads, D, device="cuda"), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, heads, D, device="cuda"), dim=-1)
    v = torch.randn(B, T, heads, D, device="cuda")
    k_hat = torch.nn.functional.normalize(torch.randn(B, T, heads, D, device="cuda"), dim=-1)
    v_hat = torch.randn(B, T, heads, D, device="cuda")
    diag = {"concentration": torch.rand(B, heads, T, device="cuda"),
            "novelty": torch.rand(B, heads, T, device="cuda")}
    calls = []

    def ours(*a, **kw):
        calls.append(1)
        return sgsa_b200.chunk_sgsa(*a, **kw)

    monkeypatch.setattr(ref, "chunk_sgsa", ours)
    with torch.no_grad():
        out, state, stats = layer(hs, q, k, v, k_hat, v_hat, diag)
        d64 = lambda t: t.double()
        want_out, want_state, _ = py_layer.double()(d64(hs), d64(q), d64(k), d64(v), d64(k_hat),
                                                    d64(v_hat), {n: d64(t) for n, t in diag.items()})
    assert calls, "the layer did not call the swapped op"
    assert float(stats["used_torch_chunk"]) == 1.0
    rel = lambda a, b: float((a.double() - b).norm() / b.norm())
    assert rel(out, want_out) < 1e-5
    assert rel(state, want_state) < 1e-5


@pytest.mark.parametrize("mode", ["none", "direct", "residual"])
def test_sgsa_state_layer_bf16_head_dim_128(ref, monkeypatch, mode):
    """The reference layer in bfloat16 with head dim 128: the swapped op takes the
    tensor-core chunk kernels (with the sparse write for "direct" / "residual").
    The bf16 layer's own projections differ from a float64 layer by more than the op's
    tolerance, so the op is checked on the exact tensors the layer hands it: its
    output and final state against the float64 oracle at the bf16 bar (2e-3)."""
    import inspect

    from oracle import oracle

    torch.manual_seed(1)
    B, T, hidden, heads = 2, 300, 512, 4
    cfg = ref.SGSAConfig(hidden_size=hidden, num_attention_heads=heads, num_kv_heads=heads,
                         sgsa_write_mode=mode, linear_backend="torch_chunk")
    layer = ref.SGSAStateLayer(cfg).cuda().eval().to(torch.bfloat16)
    D = cfg.head_dim
    bf = lambda t: t.to(torch.bfloat16)
    hs = bf(torch.randn(B, T, hidden, device="cuda"))
    q = bf(torch.nn.functional.normalize(torch.randn(B, T, heads, D, device="cuda"), dim=-1))
    k = bf(torch.nn.functional.normalize(torch.randn(B, T, heads, D, device="cuda"), dim=-1))
    v = bf(torch.randn(B, T, heads, D, device="cuda"))
    k_hat = bf(torch.nn.functional.normalize(torch.randn(B, T, heads, D, device="cuda"), dim=-1))
    v_hat = bf(torch.randn(B, T, heads, D, device="cuda"))
    diag = {"concentration": bf(torch.rand(B, heads, T, device="cuda")),
            "novelty": bf(torch.rand(B, heads, T, device="cuda"))}
    seen = []
    sig = inspect.signature(sgsa_b200.chunk_sgsa)

    def ours(*a, **kw):
        r = sgsa_b200.chunk_sgsa(*a, **kw)
        args = sig.bind(*a, **kw)
        args.apply_defaults()
        seen.append((dict(args.arguments), r))
        return r

    monkeypatch.setattr(ref, "chunk_sgsa", ours)
    with torch.no_grad():
        out, state, stats = layer(hs, q, k, v, k_hat, v_hat, diag)
    torch.cuda.synchronize()
    assert seen and float(stats["used_torch_chunk"]) == 1.0
    assert torch.isfinite(out.float()).all()
    args, (o, st) = seen[-1]
    assert args["q"].dtype == torch.bfloat16 and args["q"].shape[-1] == 128
    sparse = args.get("sparse_k") is not None
    assert sparse == (mode != "none")
    c = lambda t: None if t is None else t.detach().float().cpu()
    ro, rs = oracle.sgsa_recurrent(c(args["q"]), c(args["k"]), c(args["v"]), c(args["beta"]),
                                   c(args["gamma"]), c(args.get("sparse_k")),
                                   c(args.get("sparse_v")), c(args.get("alpha")),
                                   c(args.get("initial_state")))
    assert oracle.rel_l2(o.float().cpu().numpy(), ro) < 2e-3
    if st is not None:
        assert oracle.rel_l2(st.float().cpu().numpy(), rs) < 2e-3
