"""maba_index_topk_noalloc: the top-k entry point for callers that cannot
allocate device memory (a framework that owns the whole GPU memory pool, a
decode loop that must avoid cudaMalloc's implicit synchronisation, a foreign
binding that only receives device pointers).  It keeps its penalty table in a
fixed per-GPU device array instead of a caller workspace.

Checked through the C ABI against the workspace entry point (maba_index_topk)
on two calls in a row -- the second call must not see the first call's table,
which the shared array still holds -- and for the clear rejection of a request
larger than the fixed scratch.  This file sorts last so a failure here does not
hide the rest of the suite; it needs nothing from earlier tests.
"""
import ctypes

import pytest
import torch

from maba_v2_architecture_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = "cuda"


def call_noalloc(q, c, lam, top_k, block, decode, scores=True):
    B, L, _ = q.shape
    nb = c.shape[1]
    idx = torch.empty(B, L, min(top_k, nb), dtype=torch.long, device=DEV)
    sc = torch.empty(B, L, nb, dtype=q.dtype, device=DEV) if scores else None
    rc = N.lib().maba_index_topk_noalloc(N.ref(N.desc(q)), N.ref(N.desc(c)), float(lam), int(top_k), int(block),
                                         int(decode), N.ref(N.desc(idx)), N.ref(N.desc(sc)), N.stream_of(q))
    return rc, idx, sc


def call_workspace(q, c, lam, top_k, block, decode):
    """The existing entry point, through the same C ABI, with a caller workspace."""
    B, L, _ = q.shape
    nb = c.shape[1]
    idx = torch.empty(B, L, min(top_k, nb), dtype=torch.long, device=DEV)
    sc = torch.empty(B, L, nb, dtype=q.dtype, device=DEV)
    lib = N.lib()
    nbytes = lib.maba_index_topk_workspace_size(B, L, nb, top_k)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.maba_index_topk(N.ref(N.desc(q)), N.ref(N.desc(c)), float(lam), int(top_k), int(block), int(decode),
                             N.ref(N.desc(idx)), N.ref(N.desc(sc)), ws.data_ptr(), nbytes, N.stream_of(q))
    assert rc == 0, N.lib().maba_last_error()
    return idx, sc


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    g = torch.Generator().manual_seed(2025)
    cases = [  # (B, L, nb, top_k, lambda, decode): different table lengths and lambdas back to back
        (2, 4096, 64, 32, 0.3, 0),
        (1, 1000, 16, 8, 0.7, 0),
        (3, 1, 40, 32, 0.1, 1),
    ]
    for B, L, nb, top_k, lam, decode in cases:
        q = torch.randn(B, L, 64, generator=g).to(DEV)
        c = torch.randn(B, nb, 64, generator=g).to(DEV)
        rc, idx, sc = call_noalloc(q, c, lam, top_k, 64, decode)
        assert rc == 0, N.lib().maba_last_error()
        ref_idx, ref_sc = call_workspace(q, c, lam, top_k, 64, decode)
        torch.cuda.synchronize()
        # same kernels, same arithmetic: bit-identical scores and indices
        assert torch.equal(sc, ref_sc)
        assert torch.equal(idx, ref_idx)


def test_noalloc_rejects_requests_beyond_its_scratch():
    q = torch.randn(1, 70000, 8, device=DEV)
    c = torch.randn(1, 4, 8, device=DEV)
    rc, _, _ = call_noalloc(q, c, 0.5, 4, 1, 0, scores=False)  # block 1: 70,000 query blocks > 65,536 entries
    assert rc == N.ERR_UNSUPPORTED
    assert b"fixed scratch holds 65536" in N.lib().maba_last_error()
