"""The device watchdog path: a bounded wait that runs out is reported on the host.

A test-support kernel waits, with a short spin limit, on a barrier that nothing
arrives at (no fault, no trap, no endless loop); the wait gives up, records its
bit and returns.  The host then reads the bit through sgsa_watchdog_status, the
debug check raises, and the context keeps working.
"""
import pytest
import torch

from sgsa_b200 import _lib, ops
from sgsa_b200.inputs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_cleared():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.sgsa_watchdog_status(st) == 0
    assert lib.sgsa_watchdog_selftest(1000, st) == 0
    assert lib.sgsa_watchdog_status(st) & 0x80
    assert lib.sgsa_watchdog_status(st) == 0  # read clears
    assert lib.sgsa_watchdog_selftest(0, st) == -1  # limit out of range


def test_debug_check_raises_and_context_survives():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.sgsa_watchdog_selftest(500, st) == 0
    with pytest.raises(_lib.SGSAError, match="watchdog"):
        _lib.check_watchdog(st, "selftest")
    # the kernels still run and the watchdog stays clear on a healthy call
    cfg = CONFIGS["b200_bf16"].scaled(name="wd", B=1, T=512, H=2, top_k=64)
    d = {n: t.cuda() for n, t in make_inputs(cfg, seed=1).items()}
    out = ops.sgsa_layer_fwd(d["q"], d["k"], d["v"], d["beta"], d["gamma"], d["iq"], d["ik"],
                             d["mix"], cfg.top_k)
    assert torch.isfinite(out.float()).all()
    _lib.check_watchdog(st, "layer")
