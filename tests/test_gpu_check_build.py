"""The bounds-checked debug build (-DSGSA_CHECK, libsgsa_b200_check.so): every op of the
layer and of decode runs through it with no invariant violated, and an out-of-range
caller index is reported (and skipped) instead of being read.  Runs in a child process,
since the library variant is chosen when the package loads it (SGSA_CHECK=1)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r'''
import ctypes, torch
from sgsa_b200 import _lib, ops
from sgsa_b200.inputs import CONFIGS, make_inputs
lib = _lib.load()
assert _lib.LIB_PATH.endswith("libsgsa_b200_check.so")
def status():
    w = ctypes.c_uint(0)
    assert lib.sgsa_check_status(ctypes.byref(w), 1) == 0
    return w.value
assert status() == 0
cfg = CONFIGS["b200_bf16"].scaled(name="chk", B=1, T=1024, H=2, top_k=64)
x = {n: t.cuda() for n, t in make_inputs(cfg, seed=3).items()}
out, st, idx = ops.sgsa_layer_fwd(x["q"], x["k"], x["v"], x["beta"], x["gamma"], x["iq"], x["ik"],
                                  x["mix"], cfg.top_k, output_final_state=True, return_indices=True)
rows = ops.indexer_topk(x["iq"], x["ik"], cfg.top_k)
od, _ = ops.chunk_sgsa_fp32_state(x["q"], x["k"], x["v"], x["beta"], x["gamma"], out_f32=True)
g = ops.sparse_attn_mix(x["q"], x["k"], x["v"], rows, od, x["mix"])
# a tie-heavy indexer input drives the candidate and collect paths
iq_t = torch.ones_like(x["iq"]); ik_t = torch.ones_like(x["ik"])
ops.indexer_topk(iq_t, ik_t, cfg.top_k)
ops.indexer_thresholds(iq_t, ik_t, cfg.top_k)
# one decode step against the prefill's cache
qd, iqd = x["q"][:, -1].contiguous(), x["iq"][:, -1].contiguous()
sel = ops.decode_topk(iqd, x["ik"], cfg.T, cfg.top_k)
ops.decode_attn_mix(qd, x["k"], x["v"], sel)
sel_bad = sel.clone()
torch.cuda.synchronize()
print("clean", status())
sel_bad[0, 0, 5] = cfg.T + 1
ops.decode_attn_mix(qd, x["k"], x["v"], sel_bad)
torch.cuda.synchronize()
print("decode", status())
bad = rows.clone()
bad[0, 0, 700, 3] = cfg.T + 5
bad[0, 1, 900, 0] = -7
g_bad = ops.sparse_attn_mix(x["q"], x["k"], x["v"], bad, od, x["mix"])
pad = rows.clone()
pad[0, 0, 700, 3] = -1
pad[0, 1, 900, 0] = -1
g_pad = ops.sparse_attn_mix(x["q"], x["k"], x["v"], pad, od, x["mix"])
torch.cuda.synchronize()
print("bad", status(), bool(torch.equal(g_bad, g_pad)))
'''


@pytest.mark.gpu
def test_check_build_runs_clean_and_reports_bad_indices():
    from sgsa_b200 import build

    build.build(check=True)
    env = dict(os.environ, SGSA_CHECK="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = dict(l.split(" ", 1) for l in r.stdout.strip().splitlines() if l.startswith(("clean", "bad", "decode")))
    assert lines["clean"] == "0", r.stdout
    assert int(lines["decode"]) == 0x2, r.stdout  # the decode index check fired
    word, same = lines["bad"].split()
    assert int(word) & 0x1, r.stdout  # the gather index check fired
    assert same == "True", r.stdout   # and the bad rows were skipped like padding
