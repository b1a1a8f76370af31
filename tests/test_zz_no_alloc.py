"""The allocation-free chunk entry point (sgsa_chunk_fwd_noalloc) against the
regular one.

Some callers cannot allocate device memory at the moment they run the layer
(a runtime with a fixed memory plan, a locked allocator, a plugin that only
gets its inputs and outputs), so the library offers a variant whose
workspace is a scratch array built into the library.  This test calls both
entry points through the C ABI on the same inputs and compares them, twice in
a row so that a second call on the reused scratch is covered too.  The file
sorts last so that a stop-at-first-failure run has run everything else first.
"""
import ctypes

import pytest
import torch

from sgsa_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(dtype, B=2, T=300, H=3, D=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)
    x = dict(q=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
             k=torch.nn.functional.normalize(r(B, T, H, D), dim=-1),
             v=r(B, T, H, D), beta=torch.sigmoid(r(B, T, H)),
             gamma=torch.exp(-torch.nn.functional.softplus(r(B, T, H))),
             sk=torch.nn.functional.normalize(r(B, T, H, D), dim=-1), sv=r(B, T, H, D),
             alpha=0.25 * torch.sigmoid(r(B, T, H)))
    x = {n: t.to(dtype).cuda().contiguous() for n, t in x.items()}
    x["s0"] = (0.1 * r(B, H, D, D)).cuda()
    return x


def _call(lib, name, x, dtype, flags):
    B, T, H, D = x["q"].shape
    o = torch.empty_like(x["q"])
    sT = torch.empty(B, H, D, D, device="cuda")
    dt = _lib.DTYPE_F32 if dtype == torch.float32 else _lib.DTYPE_BF16
    p = [x[n].data_ptr() for n in ("q", "k", "v", "beta", "gamma", "sk", "sv", "alpha", "s0")]
    st = torch.cuda.current_stream().cuda_stream
    if name == "regular":
        ws = torch.empty(lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, flags), dtype=torch.uint8,
                         device="cuda")
        rc = lib.sgsa_chunk_fwd(*p, o.data_ptr(), sT.data_ptr(), B, T, H, D, dt, 64, flags,
                                ws.data_ptr(), ws.numel(), st)
    else:
        rc = lib.sgsa_chunk_fwd_noalloc(*p, o.data_ptr(), sT.data_ptr(), B, T, H, D, dt, 64,
                                        flags, st)
    assert rc == 0, lib.sgsa_status_string(rc)
    torch.cuda.synchronize()
    return o.float(), sT


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-3)])
def test_noalloc_matches_regular_entry_point_twice(dtype, tol):
    lib = _lib.load()
    flags = _lib.FLAG_HAS_SPARSE | _lib.FLAG_HAS_INIT | _lib.FLAG_STORE_FINAL
    for seed in (0, 1):  # two calls in a row on the shared scratch
        x = _inputs(dtype, seed=seed)
        ro, rs = _call(lib, "regular", x, dtype, flags)
        no, ns = _call(lib, "noalloc", x, dtype, flags)
        assert _rel(no, ro) <= tol
        assert _rel(ns, rs) <= tol


def test_noalloc_tensor_core_path_near_the_limit():
    """bf16, D=128, no sparse write: the tensor-core chunk kernels, whose workspace
    carries the 256-byte-aligned Qt / Kt tail, on a problem whose workspace is just
    under the 64 MiB scratch."""
    lib = _lib.load()
    B, T, H, D = 1, 4096, 7, 128
    flags = _lib.FLAG_HAS_INIT | _lib.FLAG_STORE_FINAL
    need = lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, flags)
    assert (60 << 20) < need <= (64 << 20)
    for seed in (2, 3):
        x = _inputs(torch.bfloat16, B=B, T=T, H=H, D=D, seed=seed)
        ro, rs = _call(lib, "regular", x, torch.bfloat16, flags)
        no, ns = _call(lib, "noalloc", x, torch.bfloat16, flags)
        assert _rel(no, ro) <= 2e-3
        assert _rel(ns, rs) <= 2e-3


def test_noalloc_sparse_write_on_the_tensor_cores():
    """bf16, D=128 with the sparse write: the tensor-core chunk kernels on the 2T
    interleaved samples, whose interleaved inputs also live in the scratch array."""
    lib = _lib.load()
    B, T, H, D = 1, 1000, 4, 128
    flags = _lib.FLAG_HAS_SPARSE | _lib.FLAG_HAS_INIT | _lib.FLAG_STORE_FINAL
    assert lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, flags) <= (64 << 20)
    for seed in (4, 5):
        x = _inputs(torch.bfloat16, B=B, T=T, H=H, D=D, seed=seed)
        ro, rs = _call(lib, "regular", x, torch.bfloat16, flags)
        no, ns = _call(lib, "noalloc", x, torch.bfloat16, flags)
        assert _rel(no, ro) <= 2e-3
        assert _rel(ns, rs) <= 2e-3


def test_noalloc_refuses_prep_reuse():
    """Reusing prep operands would read whatever an earlier call left in the shared
    scratch, so the flag is refused before anything is launched."""
    lib = _lib.load()
    x = _inputs(torch.bfloat16, B=1, T=128, H=1, D=128)
    p = [x[n].data_ptr() for n in ("q", "k", "v", "beta", "gamma", "sk", "sv", "alpha", "s0")]
    o = torch.empty_like(x["q"])
    sT = torch.empty(1, 1, 128, 128, device="cuda")
    for extra in (_lib.FLAG_REUSE_PREP, _lib.FLAG_REUSE_PREP | _lib.FLAG_TRANSITION):
        rc = lib.sgsa_chunk_fwd_noalloc(*p, o.data_ptr(), sT.data_ptr(), 1, 128, 1, 128,
                                        _lib.DTYPE_BF16, 64, _lib.FLAG_STORE_FINAL | extra,
                                        torch.cuda.current_stream().cuda_stream)
        assert rc == -6  # SGSA_ERR_UNSUPPORTED


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.load()
    # B*H*T large enough that the chunk workspace exceeds the 64 MiB scratch
    B, T, H, D = 4, 8192, 16, 128
    assert lib.sgsa_chunk_fwd_workspace_size(B, T, H, D, 0) > 64 << 20
    rc = lib.sgsa_chunk_fwd_noalloc(*([ctypes.c_void_p(16)] * 11), B, T, H, D, 1, 64, 0,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == -4  # SGSA_ERR_WORKSPACE, nothing launched
