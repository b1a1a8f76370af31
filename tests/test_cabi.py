"""The C-ABI library loads and exports every entry point include/sgsa_b200.h declares."""
import ctypes
import os
import re

import pytest
import torch

from sgsa_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "sgsa_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sgsa_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = header_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} missing from libsgsa_b200.so"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_host_only_entry_points(lib):
    assert lib.sgsa_version() >= 1000
    assert lib.sgsa_status_string(0) == b"ok"
    assert b"shape" in lib.sgsa_status_string(-1)
    n = lib.sgsa_chunk_fwd_workspace_size(4, 8192, 16, 128, 0)
    assert n == 4 * 16 * 128 * (4 * 64 * 128 + 64 * 64 + 64) * 4 + 256
    assert lib.sgsa_chunk_fwd_workspace_size(1, 64, 1, 96, 0) == 0  # unsupported head dim
    assert lib.sgsa_layer_fwd_workspace_size(1, 1024, 4, 64, 32, 4, 128, 0) > 0


def test_bad_arguments_rejected_before_any_launch(lib):
    # shape / dtype checks run before the device is touched
    assert lib.sgsa_chunk_fwd(*([None] * 11), 1, 64, 1, 96, 0, 64, 0, None, 0, None) == -1
    assert lib.sgsa_chunk_fwd(*([None] * 11), 1, 64, 1, 64, 0, 32, 0, None, 0, None) == -1
    assert lib.sgsa_chunk_fwd(*([None] * 11), 1, 64, 1, 64, 7, 64, 0, None, 0, None) == -2
    assert lib.sgsa_indexer_topk(None, None, None, 1, 64, 1, 48, 8, 0, None) == -1
    assert lib.sgsa_sparse_attn_mix(*([None] * 7), 1, 64, 1, 64, 0, 1, 1.0, 0, 1, None) == -1
    # empty problems are a no-op
    assert lib.sgsa_indexer_topk(None, None, None, 0, 64, 1, 64, 8, 1, None) == 0


def test_ops_refuse_cpu_tensors():
    import sgsa_b200 as sg
    x = torch.zeros(1, 8, 1, 32)
    g = torch.ones(1, 8, 1)
    with pytest.raises(ValueError, match="CUDA"):
        sg.chunk_sgsa(x, x, x, g, g)
    with pytest.raises(ValueError, match="CUDA"):
        sg.indexer_topk(x, x, 4)


def test_layer_workspace_follows_the_path(lib):
    """The fused (tensor-core) path keeps per-row selection records, never an index
    buffer; the gather path keeps B*idx_heads*T*K int32 rows."""
    GB = 1 << 30
    # B4 T8192 H16 d128, DI 64, k 512, bf16 -> fused
    fused = lib.sgsa_layer_fwd_workspace_size(4, 8192, 16, 128, 64, 16, 512, 1)
    chunk = lib.sgsa_chunk_fwd_workspace_size(4, 8192, 16, 128, 0)
    fp32_rows = 4 * 8192 * 16 * 128 * 4
    assert fused <= chunk + fp32_rows + 4 * 16 * 8192 * 16 + 4096
    # fp32 inputs take the gather path: the index rows are part of the workspace
    gather = lib.sgsa_layer_fwd_workspace_size(4, 8192, 16, 128, 64, 16, 512, 0)
    assert gather >= chunk + fp32_rows + 4 * 16 * 8192 * 512 * 4
    # B1 T65536 H32 k 2048 -> no 17 GB index buffer
    # B1 T65536 H32 k 2048 -> no 17 GB index buffer, and the delta stage's
    # per-chunk operands grouped under 1.25 GiB: under 3 GB in all
    long_ctx = lib.sgsa_layer_fwd_workspace_size(1, 65536, 32, 128, 64, 32, 2048, 1)
    assert long_ctx < 1 * 65536 * 32 * 2048 * 4
    assert long_ctx < 3 * GB
    assert lib.sgsa_layer_fwd_workspace_size(1, 1024, 4, 64, 32, 3, 128, 0) == 0  # bad idx_heads


def test_check_status_is_a_check_build_entry_point(lib):
    w = ctypes.c_uint(123)
    assert lib.sgsa_check_status(ctypes.byref(w), 0) == -6  # release build: unsupported
    assert w.value == 0
    assert lib.sgsa_check_status(None, 0) == -3


def test_bounds_checked_build_exports_the_same_symbols():
    path = build.build(check=True)
    chk = ctypes.CDLL(path)
    for n in header_functions():
        assert hasattr(chk, n), f"{n} missing from {os.path.basename(path)}"
