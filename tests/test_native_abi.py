"""The C-ABI library loads here (no GPU) and exports every entry point that
include/maba_b200.h declares; host-side validation mirrors the reference."""
import ctypes
import os
import re

import pytest
import torch

import maba_v2_architecture_b200 as mb
from maba_v2_architecture_b200 import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "maba_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MABA_API\s+[\w\s\*]+?\b(maba_\w+)\s*\(", text)))


def test_library_loads_and_abi_version():
    lib = N.lib()
    assert lib.maba_abi_version() == 1
    assert isinstance(lib.maba_last_error(), bytes)


def test_every_declared_symbol_is_exported_and_typed():
    syms = declared_symbols()
    assert len(syms) >= 12
    lib = ctypes.CDLL(str(N.LIB_PATH))
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/maba_b200.h but not exported"
        assert s in N.SIGNATURES, f"{s} has no ctypes signature in _native.py"


def test_struct_layout_matches_header():
    # void* + 2 x int32 + 6 x int64 shape + 6 x int64 stride
    assert ctypes.sizeof(N.MabaTensor) == 8 + 4 + 4 + 6 * 8 + 6 * 8


def test_workspace_queries_without_gpu():
    lib = N.lib()
    assert lib.maba_index_topk_workspace_size(1, 65536, 1024, 32) >= 65536 * 4
    assert lib.maba_dgda_prefill_workspace_size(0, 8, 10, 8192, 64, 64) == 0  # B*H fills the GPU: single pass
    assert lib.maba_dgda_prefill_workspace_size(0, 1, 10, 65536, 64, 64) > 0   # segmented


def test_cpu_tensors_are_rejected_no_fallback():
    x = torch.zeros(1, 2, 8, 4)
    with pytest.raises(RuntimeError, match="no CPU path"):
        mb.b200_dgda_prefill(x, x, x, log_alpha=x, b=x, w=x)
    with pytest.raises(RuntimeError, match="no CPU path"):
        mb.b200_compute_centroids(torch.zeros(1, 70, 8))
    with pytest.raises(RuntimeError, match="no CPU path"):
        mb.b200_index_topk(torch.zeros(1, 70, 8), torch.zeros(1, 2, 8))


def test_validation_matches_reference_errors():
    x = torch.zeros(1, 2, 8, 4)
    with pytest.raises(ValueError, match="Either alpha or log_alpha"):
        mb.b200_dgda_prefill(x, x, x, b=x, w=x)
    with pytest.raises(ValueError, match="Both b and w"):
        mb.b200_dgda_prefill(x, x, x, log_alpha=x)
    with pytest.raises(TypeError, match="Tensor dtypes must match"):
        mb.b200_dgda_prefill(x, x.double(), x, log_alpha=x, b=x, w=x)
    with pytest.raises(ValueError, match="k shape"):
        mb.b200_dgda_prefill(x, x[:, :1], x, log_alpha=x, b=x, w=x)
    with pytest.raises(ValueError, match="q must be"):
        mb.b200_dgda_step(torch.zeros(2, 3), torch.zeros(2, 3), torch.zeros(2, 3), log_alpha=torch.zeros(2, 3),
                          b=torch.zeros(2, 3), w=torch.zeros(2, 3))
    with pytest.raises(ValueError, match="top_k must be positive"):
        mb.b200_index_topk(torch.zeros(1, 4, 8), torch.zeros(1, 1, 8), top_k=0)
    with pytest.raises(ValueError, match="k_idx must be 3D"):
        mb.b200_compute_centroids(torch.zeros(4, 8))
    with pytest.raises(ValueError, match="Shape mismatch"):
        mb.b200_stream_superposition(torch.zeros(1, 2, 3, 4), torch.zeros(1, 2, 3, 5), torch.zeros(1, 2, 3, 4),
                                     gate_logits=torch.zeros(1, 3, 3))


def test_unsupported_dtype():
    x = torch.zeros(1, 2, 8, 4, dtype=torch.int32)
    with pytest.raises(TypeError, match="Unsupported dtype"):
        mb.b200_dgda_prefill(x, x, x, log_alpha=x, b=x, w=x)


def test_missing_library_message(tmp_path):
    with pytest.raises(RuntimeError, match="native library not found"):
        N.load_library(tmp_path / "nope.so")
