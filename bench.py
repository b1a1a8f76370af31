"""SGSA layer forward benchmark (the driver's contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one SGSA layer forward (chunked delta stage, causal top-k
indexer, sparse attention over the selected rows, gate) over the
``b200_bf16`` configuration: B=4, T=8192, H=16, d=128, top-k 512, indexer dim
64, bf16 inputs with fp32 accumulation.  Multi-GPU runs split that one
workload (strong scaling): rank r takes a contiguous block of the B*H = 64
(batch, head) pairs, which need no communication.  The line also carries
``long_ctx``: configs[2] (T 65536, H32, top-k 2048) on one GPU and, for N > 1,
sequence parallel over the N ranks (NCCL all-gather of the keys, all-to-all of
the query and output tiles) with its efficiency against the one-GPU time and
per-phase times.

``value`` is whole-job tokens/s with inputs resident in HBM (CUDA events on
the launching stream, max over ranks).  ``e2e`` is the same metric through the
public op with host (pinned) inputs: the host->device copies of all inputs and
the device->host copy of the output are inside its timed region.  The inputs
(q, k, v, iq, ik, mix: 470 MB per step) are larger than the 126 MB L2, so no
extra flush is done between steps.  ``gpu_launches`` is the library's own
launch counter over the timed region.

``--impl reference`` times the reference's CPU PyTorch path (its
naive_recurrent_sgsa from the install under baseline/_ref, plus the top-k
attention tensor operations of its hybrid model, blocked over queries) on
bounded samples of the same workload, on rank 0 only; each timed step is one
sample (2 heads of batch row 0, every query).  Without the install it times the
float64 C restatement under oracle/ and says so.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "SGSA layer fwd tokens/s"
UNIT = "tokens/s"
CONFIG_NAME = "b200_bf16"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def algorithmic_counts(cfg):
    """Per-layer-forward FLOPs and bytes of each stage: delta 6 D^2 + 2C(3D + 2D) per
    token-head, indexer 2 DI per causal pair, gathered rows 2 D bf16 values per selected pair."""
    B, T, H, D, K, DI = cfg.B, cfg.T, cfg.H, cfg.D, cfg.top_k, cfg.d_idx
    C = cfg.chunk
    f_delta = B * T * H * (6 * D * D + 2 * C * (3 * D + 2 * D))
    f_idx = B * H * T * (T + 1) * DI  # 2 * DI per causal pair, T(T+1)/2 pairs
    sel = sum(min(K, t + 1) for t in range(T))
    f_sp = B * H * sel * 4 * D
    bytes_gather = B * H * sel * (2 * D) * 2
    # tensor-core attention: indexer scores, QK^T and PV over every causal pair
    f_attn_tc = B * H * (T * (T + 1) // 2) * 2 * (DI + 2 * D)
    bytes_io = B * T * H * (2 * 3 * D + 2 * 2 * DI + 2 * D + 2 * D + 2 * 2) + 2 * B * H * D * D * 4
    return dict(f_delta=f_delta, f_idx=f_idx, f_sp=f_sp, f_attn_tc=f_attn_tc,
                bytes_gather=bytes_gather,
                bytes_io=bytes_io, selected=B * H * sel)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per (batch, head) of one
# launch at T = 8192, from ncu captures of the launches at B1 T8192 H16 (the command
# of each is in TRAFFIC_SOURCE); the traffic of these kernels grows in proportion to
# the (batch, head) pairs a launch processes.
TRAFFIC_PER_BH = {"sparse_attn_tc": (417.96e6 + 25.08e6) / 16,
                  "indexer_thresholds": (32.64e6 + 23.81e6) / 16,
                  "delta": (101.74e6 + 242.67e6 + 302.36e6 + 52.37e6) / 16}
TRAFFIC_SOURCE = ("ncu dram bytes of one launch at B1 T8192 H16 (python bench.py --only <stage> "
                  "--steps 1 --B 1 --H 16), scaled by the launch's (b, h) count")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def setup_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, local


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()


REF_DIR = os.path.join(ROOT, "baseline", "_ref")
REF_HEADS_PER_STEP = 2


def reference_available() -> bool:
    return os.path.isdir(os.path.join(REF_DIR, "modelings"))


def _reference_naive():
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from modelings.sgsa_ops.naive import naive_recurrent_sgsa
    return naive_recurrent_sgsa


def reference_cpu_sample(x, h0, h1, top_k, q_block=512):
    """One bounded sample of the reference's CPU PyTorch path, float32, on batch row 0
    and heads [h0, h1) of the workload, every query: the delta stage by the
    reference's own naive_recurrent_sgsa (modelings/sgsa_ops/naive.py:10-57); the
    selection, sparse attention and gate by the tensor operations of
    modelings/hybrid_dense_delta_topk.py:343-356,389-390 (score matmul, causal
    finfo.min mask, torch.topk, float32 softmax, gather, weighted sum, sigmoid-gate
    mix) with the indexer iq . ik choosing the rows and q . k / sqrt(d) weighting
    them, run over blocks of q_block queries (the reference's single [B,H,T,k,D]
    gather would need 137 GB at this size).  Returns (seconds, output)."""
    naive = _reference_naive()
    sl = {n: t[:1, :, h0:h1].float().contiguous() for n, t in x.items()}
    T, Hs, D = sl["q"].shape[1], sl["q"].shape[2], sl["q"].shape[3]
    t0 = time.perf_counter()
    with torch.no_grad():
        o_delta, _ = naive(sl["q"], sl["k"], sl["v"], sl["beta"], sl["gamma"])
        q, k, v = (sl[n][0].transpose(0, 1) for n in ("q", "k", "v"))     # [H, T, D]
        iq, ik = (sl[n][0].transpose(0, 1) for n in ("iq", "ik"))
        scale = 1.0 / math.sqrt(D)
        out = torch.empty(Hs, T, D)
        neg = torch.finfo(torch.float32).min
        for s0 in range(0, T, q_block):
            s1 = min(T, s0 + q_block)
            pos = torch.arange(s0, s1)[:, None]
            causal = torch.arange(s1)[None, :] <= pos                       # [Q, s1]
            idx_scores = (iq[:, s0:s1] @ ik[:, :s1].transpose(1, 2)).masked_fill(~causal, neg)
            kk = min(top_k, s1)
            _, sel = torch.topk(idx_scores, k=kk, dim=-1)                   # [H, Q, kk]
            att = (q[:, s0:s1] @ k[:, :s1].transpose(1, 2)) * scale
            att = att.gather(-1, sel).masked_fill(sel > pos, float("-inf"))
            p = torch.softmax(att, dim=-1)
            vsel = torch.gather(v[:, None].expand(-1, s1 - s0, -1, -1), 2,
                                sel[..., None].expand(-1, -1, -1, D))
            out[:, s0:s1] = (p[..., None] * vsel).sum(2)
        m = sl["mix"][0].transpose(0, 1)
        res = m * out + (1.0 - m) * o_delta[0].transpose(0, 1)
    return time.perf_counter() - t0, res


def reference_chunk_sample(x, h0, h1):
    """Seconds of the reference's own chunk_sgsa (torch path, modelings/sgsa_ops/chunk.py)
    on the same sample's delta stage; reported beside the baseline only: at this
    decay its clamped cumprods make it numerically wrong (rel-L2 ~0.8 at configs[0])."""
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from modelings.sgsa_ops import chunk_sgsa
    sl = {n: t[:1, :, h0:h1].float().contiguous() for n, t in x.items()}
    t0 = time.perf_counter()
    with torch.no_grad():
        chunk_sgsa(sl["q"], sl["k"], sl["v"], sl["beta"], sl["gamma"], use_triton=False)
    return time.perf_counter() - t0


def cpu_port_sample(cfg, x, h0, h1):
    """Seconds of the repository's float64 C restatement (oracle/) on the same sample."""
    from oracle import oracle

    oracle.set_num_threads(os.cpu_count() or 1)
    sl = {n: t[:1, :, h0:h1].contiguous() for n, t in x.items()}
    t0 = time.perf_counter()
    od, _ = oracle.sgsa_recurrent(sl["q"], sl["k"], sl["v"], sl["beta"], sl["gamma"])
    idx = oracle.indexer_topk(sl["iq"], sl["ik"], cfg.top_k)
    oracle.sparse_attn_mix(sl["q"], sl["k"], sl["v"], idx, od, sl["mix"])
    return time.perf_counter() - t0


def cpu_baseline(cfg, steps: int, warmup: int):
    """Times `steps` samples (after `warmup` untimed ones) of the reference's CPU path,
    each REF_HEADS_PER_STEP heads of batch row 0 over all T queries, so one sample is
    T * REF_HEADS_PER_STEP / H tokens' worth of the workload.  Returns the
    cpu_baseline object (value in tokens/s) and the per-step seconds."""
    from sgsa_b200.inputs import make_inputs

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x = make_inputs(cfg.scaled(B=1), seed=0)
    hs = REF_HEADS_PER_STEP
    heads = [(i * hs) % cfg.H for i in range(warmup + steps)]
    tok = cfg.T * hs / cfg.H
    if reference_available():
        for i in range(warmup):
            reference_cpu_sample(x, heads[i], heads[i] + hs, cfg.top_k)
        secs = [reference_cpu_sample(x, h, h + hs, cfg.top_k)[0] for h in heads[warmup:]]
        kind = "reference"
        what = ("the reference's CPU PyTorch path (naive_recurrent_sgsa + the top-k "
                "attention/gate tensor ops of hybrid_dense_delta_topk.py:343-356,389-390, "
                f"blocked over 512 queries), float32")
        extra = {"chunk_sgsa_s": reference_chunk_sample(x, 0, hs),
                 "chunk_sgsa_note": "reference chunk_sgsa on the same delta sample; "
                                    "numerically wrong at this decay, not the baseline"}
    else:
        for i in range(warmup):
            cpu_port_sample(cfg, x, heads[i], heads[i] + hs)
        secs = [cpu_port_sample(cfg, x, h, h + hs) for h in heads[warmup:]]
        kind = "port"
        what = "the float64 C restatement of the reference maths (oracle/)"
        extra = {"note": "reference not installed under baseline/_ref"}
    mean = statistics.mean(secs)
    sample = (f"{what} on batch row 0, {hs} of {cfg.H} heads per step (heads cycle), all "
              f"T={cfg.T} queries, top-{cfg.top_k}; {cores} threads; tokens/s = "
              f"T*{hs}/{cfg.H} / seconds per step")
    return dict(value=tok / mean, unit=UNIT, cores=cores, kind=kind, sample=sample,
                seconds_per_step=mean, steps=len(secs), **extra), secs


def run_reference(args, ws, rank):
    from sgsa_b200.inputs import CONFIGS

    if rank != 0:
        return
    cfg = CONFIGS[CONFIG_NAME]
    warm = min(args.warmup, 1)
    base, secs = cpu_baseline(cfg, max(args.steps, 1), warm)
    v = base["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws,
        "steps": len(secs), "warmup": warm, "ms_per_step": statistics.mean(secs) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, configs[1] shapes/distributions)",
        "config": {"workload": CONFIG_NAME, "B": cfg.B, "T": cfg.T, "H": cfg.H, "d": cfg.D,
                   "top_k": cfg.top_k, "d_idx": cfg.d_idx, "chunk": cfg.chunk,
                   "parallelism": "cpu, rank 0", "l2": "n/a (host)",
                   "step": f"batch row 0, {REF_HEADS_PER_STEP} heads, all {cfg.T} queries"},
        "cpu_baseline": {k: base[k] for k in ("kind", "cores", "sample", "value", "unit")},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def stage_times(cfg, d, reps=3, only=None):
    """Per-stage device time (ms) of the layer, each stage called through the C ABI."""
    from sgsa_b200 import _lib, ops

    lib = _lib.load()
    st = torch.cuda.current_stream()
    B, T, H, D = cfg.B, cfg.T, cfg.H, cfg.D
    od = torch.empty(B, T, H, D, device="cuda", dtype=torch.float32)
    ix = torch.empty(B, H, T, cfg.top_k, device="cuda", dtype=torch.int32)
    flags = _lib.FLAG_OUT_F32
    ws = torch.empty(lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, flags), device="cuda",
                     dtype=torch.uint8)
    out = torch.empty_like(d["q"])
    P = lambda t: t.data_ptr()

    def delta():
        _lib.check(lib.sgsa_chunk_fwd(P(d["q"]), P(d["k"]), P(d["v"]), P(d["beta"]), P(d["gamma"]),
                                      None, None, None, None, P(od), None, B, T, H, D,
                                      _lib.DTYPE_BF16, 64, flags, P(ws), ws.numel(), st.cuda_stream),
                   "chunk")

    def index():
        _lib.check(lib.sgsa_indexer_topk(P(d["iq"]), P(d["ik"]), P(ix), B, T, H, cfg.d_idx,
                                         cfg.top_k, _lib.DTYPE_BF16, st.cuda_stream), "indexer")

    def attn():
        _lib.check(lib.sgsa_sparse_attn_mix(P(d["q"]), P(d["k"]), P(d["v"]), P(ix), P(od),
                                            P(d["mix"]), P(out), B, T, H, D, cfg.top_k, H,
                                            1.0 / math.sqrt(D), 1, _lib.DTYPE_BF16,
                                            st.cuda_stream), "attn")

    sw = {}

    def delta_sw():
        # the delta stage with the sparse write (row f3): 2 virtual samples per token; the
        # retrieval's k_hat / v_hat stand-ins are the token's own k / v, alpha = beta
        fl = _lib.FLAG_OUT_F32 | _lib.FLAG_HAS_SPARSE
        if "ws" not in sw:
            sw["ws"] = torch.empty(lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, fl),
                                   device="cuda", dtype=torch.uint8)
        w = sw["ws"]
        _lib.check(lib.sgsa_chunk_fwd(P(d["q"]), P(d["k"]), P(d["v"]), P(d["beta"]), P(d["gamma"]),
                                      P(d["k"]), P(d["v"]), P(d["beta"]), None, P(od), None, B, T,
                                      H, D, _lib.DTYPE_BF16, 64, fl, P(w), w.numel(),
                                      st.cuda_stream), "chunk")

    def delta_sw_simt():
        os.environ["SGSA_SCAN_SIMT"] = "1"
        try:
            delta_sw()
        finally:
            del os.environ["SGSA_SCAN_SIMT"]

    thr = torch.empty(B, H, T, 4, device="cuda", dtype=torch.int32)
    norms = torch.empty(2 * B * H, device="cuda", dtype=torch.int32)

    def index_thr():
        _lib.check(lib.sgsa_indexer_thresholds(P(d["iq"]), P(d["ik"]), None, P(thr), None, 0, B,
                                               T, H, cfg.d_idx, cfg.top_k, st.cuda_stream),
                   "indexer")

    def attn_tc():
        _lib.check(lib.sgsa_sparse_attn_thresholds(P(d["q"]), P(d["k"]), P(d["v"]), P(d["iq"]),
                                                   P(d["ik"]), P(thr), None, 0, P(od), P(d["mix"]),
                                                   P(out), B, T, H, D, cfg.d_idx, H,
                                                   1.0 / math.sqrt(D), 1, 0, P(norms),
                                                   st.cuda_stream),
                   "attn_tc")

    res = {}
    # the stages as the layer runs them (fused) and the standalone index/gather pair
    stages = (("delta", delta), ("indexer_thresholds", index_thr), ("sparse_attn_tc", attn_tc),
              ("indexer_topk", index), ("sparse_attn_mix", attn),
              ("delta_sparse_write", delta_sw), ("delta_sparse_write_cuda_core", delta_sw_simt))
    if only == "sparse_attn_mix":
        index()  # the attention stage reads the indexer's output
    if only == "sparse_attn_tc":
        index_thr()
    for name, fn in stages:
        if only and name != only:
            continue
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / reps
    del ops
    return res


def run_long(args, ws, rank, local):
    """B1 T65536 H32, top-k 2048; N=1 the single-GPU layer, N>1 the
    sequence-parallel layer (contiguous T/N slices, strong scaling)."""
    from sgsa_b200 import ops, sp
    from sgsa_b200.inputs import CONFIGS, make_inputs_slice

    cfg = CONFIGS["long_ctx"]
    Tl = cfg.T // ws
    x = make_inputs_slice(cfg, rank * Tl, (rank + 1) * Tl, seed=0, device="cuda")
    args_ = (x["q"], x["k"], x["v"], x["beta"], x["gamma"], x["iq"], x["ik"], x["mix"], cfg.top_k)

    def step():
        if ws == 1:
            return ops.sgsa_layer_fwd(*args_)
        return sp.sp_layer_fwd(*args_)

    for _ in range(max(args.warmup, 1)):
        step()
    barrier(ws)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(ws)
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        barrier(ws)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    if rank == 0:
        print(json.dumps({
            "metric": "SGSA long-context layer fwd tokens/s", "workload": "long_ctx (configs[2])",
            "value": cfg.tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": ws,
            "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic, block-seeded (identical for every N)",
            "config": {"B": cfg.B, "T": cfg.T, "H": cfg.H, "d": cfg.D, "top_k": cfg.top_k,
                       "d_idx": cfg.d_idx, "parallelism": "single" if ws == 1 else f"sp{ws}"},
            "clocks": clk.summary()}), flush=True)


def run_decode(args):
    """decode with top-k reuse over a planted-retrieval cache (1 GPU)."""
    from sgsa_b200 import ops

    torch.cuda.set_device(0)
    B, H, D, DI, Tc, K, reuse, nplant = 64, 16, 128, 64, 32768, 1024, 4, 256
    if args.B:  # a smaller batch (profiling captures); the metric's configuration is B = 64
        B = args.B
    steps = args.steps
    n0 = Tc - (args.warmup + steps + 8 + 1)
    g = torch.Generator(device="cuda").manual_seed(0)
    bf = torch.bfloat16
    kc = torch.nn.functional.normalize(torch.randn(B, Tc, H, D, device="cuda", generator=g), dim=-1).to(bf)
    vc = torch.randn(B, Tc, H, D, device="cuda", generator=g).to(bf)
    ikc = torch.randn(B, Tc, H, DI, device="cuda", generator=g)
    # 256 planted keys per sequence (x4 scaled) at seeded positions of the prefilled part
    pos = torch.randint(0, n0, (B, nplant), device="cuda", generator=g)
    bidx = torch.arange(B, device="cuda")[:, None].expand(B, nplant)
    ikc[bidx, pos] = 4.0 * torch.randn(B, nplant, H, DI, device="cuda", generator=g)
    ikc = ikc.to(bf)
    state = 0.1 * torch.randn(B, H, D, D, device="cuda", generator=g)
    cache = ops.DecodeCache(kc, vc, ikc, n0, state, K, reuse=reuse)
    # each step's query is aligned to one planted key of its sequence (chosen per step)
    targets = pos[torch.arange(B, device="cuda"), torch.randint(0, nplant, (B,), device="cuda", generator=g)]

    def token(i):
        r = lambda *s: torch.randn(*s, device="cuda", generator=g)
        q = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(bf)
        k = torch.nn.functional.normalize(r(B, H, D), dim=-1).to(bf)
        iq = ikc[torch.arange(B, device="cuda"), targets].clone()
        return (q, k, r(B, H, D).to(bf), torch.sigmoid(r(B, H)).to(bf),
                torch.exp(-torch.nn.functional.softplus(r(B, H))).to(bf), iq, r(B, H, DI).to(bf),
                torch.sigmoid(r(B, H, D)).to(bf))

    toks = [token(i) for i in range(args.warmup + steps)]
    for i in range(args.warmup):
        cache.step(*toks[i])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.warmup, args.warmup + steps):
        cache.step(*toks[i])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    sel = cache.indices  # [B, H, K]
    hit = (sel == targets[:, None, None].int()).any(-1).float().mean().item()

    # Agreement with the reference on sampled batch rows over `check` more steps: the
    # reference re-scores the whole cache at every step (modelings/hybrid_dense_delta_topk.py
    # :343-349), this cache refreshes every `reuse` steps.  Exact index agreement on the
    # refresh steps, planted-key hits of both on every step, and the CPU time of the
    # reference's decode path on those rows.
    from oracle import oracle
    rows = [0, min(B - 1, B // 2 + 5)]
    check = 2 * reuse
    kc_o, vc_o, ikc_o = kc[rows].cpu(), vc[rows].cpu(), ikc[rows].cpu()
    st_o = cache.state[rows].cpu().numpy()
    n_cur = cache.n
    agree, ref_hits, our_hits = [], [], []
    cpu_s, cpu_rows = 0.0, 0
    torch.set_num_threads(os.cpu_count() or 1)
    for i in range(check):
        tk = token(steps + args.warmup + i)
        cache.step(*tk)
        sub = lambda t: t[rows].cpu()
        q, k, v, beta, gamma, iq, ik, mix = (sub(t) for t in tk)
        kc_o[:, n_cur], vc_o[:, n_cur], ikc_o[:, n_cur] = k, v, ik
        n_cur += 1
        t0 = time.perf_counter()
        od, st_o = oracle.sgsa_recurrent(q[:, None], k[:, None], v[:, None], beta[:, None],
                                         gamma[:, None], initial_state=st_o)
        ref_idx = oracle.decode_topk(iq, ikc_o, n_cur, K)
        oracle.decode_attn_mix(q, kc_o, vc_o, ref_idx, od[:, 0], mix)
        cpu_s += time.perf_counter() - t0
        cpu_rows += len(rows)
        ours = cache.indices[rows].cpu().numpy()
        tg = targets[rows].cpu().numpy()
        if (cache.steps - 1) % reuse == 0:  # a refresh step: the sets must agree
            agree.append(float((ours == ref_idx).all(-1).mean()))
        ref_hits.append(float((ref_idx == tg[:, None, None]).any(-1).mean()))
        our_hits.append(float((ours == tg[:, None, None]).any(-1).mean()))
    print(json.dumps({
        "metric": "SGSA decode tokens/s", "workload": "decode_topk_reuse (configs[4])",
        "value": B / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
        "warmup": args.warmup, "config": {"batch": B, "cache": Tc, "H": H, "d": D, "d_idx": DI,
                                          "top_k": K, "reuse": reuse, "planted": nplant},
        "retrieval_hit_rate": hit,
        "agreement": {"rows": rows, "steps": check,
                      "refresh_index_sets_equal": statistics.mean(agree) if agree else None,
                      "hit_rate_ours": statistics.mean(our_hits),
                      "hit_rate_reference": statistics.mean(ref_hits),
                      "reference": "oracle decode step: recurrence, full re-score top-k every "
                                   "step, attention + gate (float64)"},
        "cpu_baseline": {"value": cpu_rows / cpu_s, "unit": "tokens/s",
                         "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": f"{len(rows)} batch rows x {check} decode steps of the "
                                   "float64 restatement (full re-score each step)"},
        "dtype": "bf16", "data": "synthetic planted retrieval"}))


HYBRID_B, HYBRID_T = 8, 4096
HYBRID_METRIC = "hybrid model prefill tokens/s"


def cpu_hybrid_reference(cores: int, T: int = 512):
    """Time the CPU restatement of the configs[3] model (all 24 layers, full width)
    on one sequence of T tokens, float32 outside the SGSA core; returns (tokens/s,
    sample text, seconds)."""
    from oracle import hybrid as ohybrid
    from oracle import oracle
    from sgsa_b200.hybrid import CONFIG_B200, HybridSGSAModel

    oracle.set_num_threads(cores)
    torch.set_num_threads(cores)
    m = HybridSGSAModel(CONFIG_B200, device="cpu", dtype=torch.bfloat16, seed=0)
    ids = torch.randint(1, CONFIG_B200.vocab_size, (1, T), generator=torch.Generator().manual_seed(0))
    t0 = time.perf_counter()
    ohybrid.model_forward(ids, m.weights, CONFIG_B200, dtype=torch.float32)
    secs = time.perf_counter() - t0
    sample = (f"one sequence of {T} tokens through the full configs[3] model (24 layers, "
              f"hidden 2048, vocab 32000), float32 torch + float64 SGSA oracle, {cores} threads; "
              f"tokens/s = {T} / seconds")
    return T / secs, sample, secs


def run_hybrid(args, ws, rank, local):
    """hybrid model prefill, B=8 x T=4096, batch sharded over the ranks
    (B/N sequences each; strong scaling, no communication)."""
    from sgsa_b200.hybrid import CONFIG_B200, HybridSGSAModel

    if HYBRID_B % ws:
        raise SystemExit("--gpus must divide the batch of 8")
    Bl, T, cfg = HYBRID_B // ws, HYBRID_T, CONFIG_B200
    m = HybridSGSAModel(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    g = torch.Generator().manual_seed(0)
    ids_all = torch.randint(0, cfg.vocab_size, (HYBRID_B, T), generator=g)
    ids_host = ids_all[rank * Bl:(rank + 1) * Bl].contiguous()
    ids = ids_host.cuda()

    def step():
        return m(ids)

    for _ in range(max(args.warmup, 3)):
        step()
    barrier(ws)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(ws)
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        barrier(ws)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)

    # end to end: pinned token ids -> device, full prefill, last-position logits -> host
    pinned = ids_host.pin_memory()
    out_host = torch.empty(Bl, cfg.vocab_size, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        d = pinned.to("cuda", non_blocking=True)
        logits = m(d)
        out_host.copy_(logits[:, -1], non_blocking=True)

    e2e_step()
    barrier(ws)
    e2e_steps = max(1, min(args.steps, 5))
    e0.record(st)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(st)
    barrier(ws)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, ws)

    # per-part device times of one more forward
    marks = []
    m(ids, marks=marks)
    torch.cuda.synchronize()
    parts = {}
    for (_, a), (name, b) in zip(marks[:-1], marks[1:]):
        parts[name] = parts.get(name, 0.0) + a.elapsed_time(b)
    flops = m.flops_per_token(T) * Bl * T
    _, tfl, src = peaks()
    if rank == 0:
        cores = os.cpu_count() or 1
        cpu_v, sample, secs = cpu_hybrid_reference(cores)
        tokens = HYBRID_B * T
        print(json.dumps({
            "metric": HYBRID_METRIC, "workload": "hybrid_prefill (configs[3])",
            "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic token ids (uniform over the vocab), random init std 0.02",
            "config": {"workload": "hybrid_prefill", "B": HYBRID_B, "T": T,
                       "layers": cfg.num_layers, "hidden": cfg.hidden_size,
                       "heads": cfg.num_heads, "mlp": cfg.intermediate_size,
                       "vocab": cfg.vocab_size, "top_k": cfg.top_k, "d_idx": cfg.indexer_dim,
                       "layer_order": "dense at layer % 4 == 0, SGSA otherwise",
                       "parallelism": f"batch-shard x{ws}",
                       "l2": "activations > L2, no flush"},
            "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": pinned.numel() * 8 * ws,
                    "d2h_bytes_per_step": out_host.numel() * 2 * ws, "ms_per_step": e2e_ms},
            "part_ms": parts,
            "matrix_tflops": flops / (ms / 1e3) / 1e12,
            "matrix_flops_per_step_rank": flops, "peak_tflops": tfl, "peak_source": src,
            "cpu_baseline": {"value": cpu_v, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample, "seconds": secs},
            "clocks": clk.summary()}), flush=True)


def run_hybrid_reference(args, ws, rank):
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    v, sample, secs = cpu_hybrid_reference(cores)
    print(json.dumps({
        "impl": "reference", "metric": HYBRID_METRIC, "workload": "hybrid_prefill (configs[3])",
        "value": v, "unit": "tokens/s", "n_gpus": ws, "steps": 1, "warmup": 0,
        "ms_per_step": HYBRID_B * HYBRID_T / v * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic token ids, random init std 0.02",
        "config": {"workload": "hybrid_prefill", "B": HYBRID_B, "T": HYBRID_T},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample, "seconds": secs},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def run_only(args):
    """Run a single stage on a scaled configuration (for ncu captures)."""
    from sgsa_b200.inputs import CONFIGS, make_inputs

    torch.cuda.set_device(0)
    cfg = CONFIGS[CONFIG_NAME]
    kw = {n: getattr(args, n) for n in ("B", "T", "H") if getattr(args, n)}
    cfg = cfg.scaled(**kw) if kw else cfg
    d = {n: t.cuda() for n, t in make_inputs(cfg, seed=0).items()}
    res = stage_times(cfg, d, reps=args.steps, only=args.only)
    print(json.dumps({"stage": args.only, "ms": res[args.only],
                      "config": {"B": cfg.B, "T": cfg.T, "H": cfg.H}}))


def shard_of(cfg, ws: int, rank: int):
    """(b0, b1, h0, h1): rank's contiguous block of the B*H (batch, head) pairs."""
    if ws <= cfg.B:
        if cfg.B % ws:
            raise SystemExit(f"--gpus {ws} must divide the batch {cfg.B}")
        nb = cfg.B // ws
        return rank * nb, (rank + 1) * nb, 0, cfg.H
    per_b = ws // cfg.B
    if ws % cfg.B or cfg.H % per_b:
        raise SystemExit(f"--gpus {ws} must split B*H = {cfg.B}*{cfg.H} evenly")
    nh = cfg.H // per_b
    b, j = divmod(rank, per_b)
    return b, b + 1, j * nh, (j + 1) * nh


def long_ctx_run(ws, rank, local, steps=3):
    """configs[2] (B1 T65536 H32, top-k 2048): the single-GPU layer on rank 0 (the
    1-GPU reference of the efficiency) and, for N > 1, the sequence-parallel layer
    on all ranks with per-phase times of one step."""
    from sgsa_b200 import ops, sp
    from sgsa_b200.inputs import CONFIGS, make_inputs_slice

    cfg = CONFIGS["long_ctx"]
    names = ("q", "k", "v", "beta", "gamma", "iq", "ik", "mix")
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    res = {"config": {"B": cfg.B, "T": cfg.T, "H": cfg.H, "d": cfg.D, "top_k": cfg.top_k,
                      "d_idx": cfg.d_idx}, "steps": steps}
    ms1 = 0.0
    if rank == 0:
        x = make_inputs_slice(cfg, 0, cfg.T, seed=0, device="cuda")
        args_ = [x[n] for n in names] + [cfg.top_k]
        ops.sgsa_layer_fwd(*args_)
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(steps):
            ops.sgsa_layer_fwd(*args_)
        e1.record(st)
        torch.cuda.synchronize()
        ms1 = e0.elapsed_time(e1) / steps
        del x, args_
        ops.release_workspaces()
        torch.cuda.empty_cache()
    res["ms_1gpu"] = max_over_ranks(ms1, ws)
    if ws == 1:
        res["tokens_per_s_1gpu"] = cfg.tokens / (res["ms_1gpu"] / 1e3)
        return res
    Tl = cfg.T // ws
    x = make_inputs_slice(cfg, rank * Tl, (rank + 1) * Tl, seed=0, device="cuda")
    args_ = [x[n] for n in names] + [cfg.top_k]
    sp.sp_layer_fwd(*args_)
    barrier(ws)
    e0.record(st)
    for _ in range(steps):
        sp.sp_layer_fwd(*args_)
    e1.record(st)
    barrier(ws)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, ws)
    tm = {}
    sp.sp_layer_fwd(*args_, timings=tm)
    barrier(ws)
    phases = {k: max_over_ranks(v, ws) for k, v in sorted(sp.phase_ms(tm).items())}
    res.update(ms_sp=ms, parallelism=f"sp{ws}", tokens_per_s=cfg.tokens / (ms / 1e3),
               efficiency=res["ms_1gpu"] / (ws * ms), phase_ms_max_over_ranks=phases)
    return res


def run_ours(args, ws, rank, local):
    from sgsa_b200 import _lib, ops
    from sgsa_b200.inputs import CONFIGS, make_inputs

    lib = _lib.load()
    cfg = CONFIGS[CONFIG_NAME]
    b0, b1, h0, h1 = shard_of(cfg, ws, rank)
    full = make_inputs(cfg, seed=0)  # the same workload at every N; rank r takes its shard
    host = {n: t[b0:b1, :, h0:h1].contiguous() for n, t in full.items()}
    del full
    scfg = cfg.scaled(B=b1 - b0, H=h1 - h0)
    d = {n: t.cuda() for n, t in host.items()}
    names = ["q", "k", "v", "beta", "gamma", "iq", "ik", "mix"]

    def step():
        return ops.sgsa_layer_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"],
                                  d["mix"], cfg.top_k)

    for _ in range(max(args.warmup, 3)):
        step()
    barrier(ws)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(ws)
        t_start = time.perf_counter()
        n0 = lib.sgsa_kernel_launches()
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        n1 = lib.sgsa_kernel_launches()
        barrier(ws)
        # short timed regions: keep the same load (untimed) until the sampler has
        # seen at least ~1 s of it
        while time.perf_counter() - t_start < 1.0:
            step()
            torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    value = cfg.tokens / (ms / 1e3)  # the whole configs[1] workload, split over the ranks
    launches = n1 - n0
    if ws > 1:
        t = torch.tensor([launches], device="cuda", dtype=torch.int64)
        dist.all_reduce(t)
        launches = int(t.item())

    # end to end: pinned host inputs -> device -> layer -> host output
    pinned = {n: host[n].pin_memory() for n in names}
    out_host = torch.empty(scfg.B, scfg.T, scfg.H, scfg.D, dtype=scfg.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pinned.values()) * ws
    d2h = out_host.numel() * out_host.element_size() * ws

    def e2e_step():
        ops.sgsa_layer_fwd_from_host(*(pinned[n] for n in names), cfg.top_k, out=out_host)

    for _ in range(3):
        e2e_step()
    barrier(ws)
    # the host link's time varies from call to call: average over up to 20 steps (~0.3 s)
    e2e_steps = max(1, min(2 * args.steps, 20))
    e0.record(st)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(st)
    barrier(ws)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, ws)

    stages = stage_times(scfg, d)
    cnt = algorithmic_counts(scfg)
    hbm, tfl, src = peaks()
    # the dominant kernel among the stages the layer runs, and its roofline
    layer_stages = ("delta", "indexer_thresholds", "sparse_attn_tc")
    dom = max(layer_stages, key=lambda n: stages[n])
    flops = {"delta": cnt["f_delta"], "indexer_thresholds": cnt["f_idx"],
             "sparse_attn_tc": cnt["f_attn_tc"]}[dom]
    ach = flops / (stages[dom] / 1e3) / 1e12
    roof = {"kernel": dom, "bound": "tensor", "achieved": ach, "peak": tfl, "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_source"] = src
    roof["traffic"] = (TRAFFIC_PER_BH[dom] * scfg.B * scfg.H
                       if scfg.T == 8192 and dom in TRAFFIC_PER_BH else None)
    roof["traffic_source"] = TRAFFIC_SOURCE
    roof["stage_ms"] = stages
    roof["gather_equiv_gbs"] = cnt["bytes_gather"] / (stages["sparse_attn_tc"] / 1e3) / 1e9
    if dom == "indexer_thresholds":
        roof["note"] = ("the indexer's tensor work is 2*DI FLOPs per causal pair; it is bound by the "
                        "CUDA-core selection, not by the tensor cores")
    ach_attn = cnt["f_attn_tc"] / (stages["sparse_attn_tc"] / 1e3) / 1e12
    roof["sparse_attn_tc"] = {"achieved": ach_attn, "peak": tfl, "unit": "TFLOP/s",
                              "frac": ach_attn / tfl,
                              "useful_frac": cnt["f_sp"] / (stages["sparse_attn_tc"] / 1e3) / 1e12 / tfl,
                              "note": "frac counts every causal pair the kernel computes; "
                                      "useful_frac only the selected pairs (F_sp)"}
    long_ctx = long_ctx_run(ws, rank, local) if not args.no_long else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, configs[1] shapes/distributions; one workload at every N)",
            "config": {"workload": CONFIG_NAME, "B": cfg.B, "T": cfg.T, "H": cfg.H, "d": cfg.D,
                       "top_k": cfg.top_k, "d_idx": cfg.d_idx, "chunk": cfg.chunk,
                       "parallelism": "single" if ws == 1 else f"bh-shard x{ws}",
                       "shard_rank0": {"B": scfg.B, "H": scfg.H},
                       "l2": "inputs 470 MB > L2, no flush"},
            "e2e": {"value": cfg.tokens / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": launches,
            "gpu_launches_source": "sgsa_kernel_launches() counter, timed region, all ranks",
            "roofline": roof,
            "clocks": clk.summary(),
        }
        if long_ctx is not None:
            line["long_ctx"] = long_ctx
        if ws == 1 and not args.no_cpu:
            line["cpu_baseline"], _ = cpu_baseline(cfg, 3, 1)
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--only", default=None, choices=["delta", "delta_sparse_write", "indexer_topk", "sparse_attn_mix", "indexer_thresholds",
                             "sparse_attn_tc"],
                    help="profiling aid: run one stage --steps times on a (scaled) config, no JSON")
    ap.add_argument("--workload", default="layer", choices=["layer", "decode", "long", "hybrid"],
                    help="decode: configs[4] (batch 64, 32768-token cache, top-k 1024 reused "
                         "every 4 steps, planted retrieval); long: configs[2] (T 65536, "
                         "sequence parallel for N > 1); hybrid: configs[3] (24-layer "
                         "hybrid model prefill, B 8 x T 4096, batch sharded); layer "
                         "(default): configs[1]")
    ap.add_argument("--no-long", action="store_true",
                    help="skip the configs[2] long_ctx measurement of the default workload")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--B", type=int, default=None)
    ap.add_argument("--T", type=int, default=None)
    ap.add_argument("--H", type=int, default=None)
    args = ap.parse_args()
    if args.only:
        run_only(args)
        return
    if args.workload == "decode":
        run_decode(args)
        return
    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if args.workload == "hybrid":
            run_hybrid_reference(args, ws, rank)
        else:
            run_reference(args, ws, rank)
        return
    ws, rank, local = setup_dist()
    try:
        if args.workload == "long":
            run_long(args, ws, rank, local)
        elif args.workload == "hybrid":
            run_hybrid(args, ws, rank, local)
        else:
            run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
