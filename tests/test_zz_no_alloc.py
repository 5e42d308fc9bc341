"""maba_index_topk_noalloc: the top-k entry point for callers that cannot
allocate device memory (a framework that owns the whole GPU memory pool, a
decode loop that must avoid cudaMalloc's implicit synchronisation, a foreign
binding that only receives device pointers).  It keeps its scratch in a fixed
per-GPU device array instead of a caller workspace.

Checked through the C ABI against the workspace entry point (maba_index_topk)
on calls in a row -- a later call must not see what an earlier call left in
the shared array -- on each of the array's three uses: the penalty table
(every call), the centroid-norm tables of the pruned tile scan (prefill
without scores) and the partial lists of the split decode scan (decode
without scores, nb >= 2048); on a near-limit shape whose norm tables no
longer fit (it runs the unpruned scan and must give the same indices); and
for the clear rejection of a request larger than the fixed scratch.  This file
sorts last so a failure here does not hide the rest of the suite; it needs
nothing from earlier tests.
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


def call_workspace(q, c, lam, top_k, block, decode, scores=True):
    """The existing entry point, through the same C ABI, with a caller workspace."""
    B, L, _ = q.shape
    nb = c.shape[1]
    idx = torch.empty(B, L, min(top_k, nb), dtype=torch.long, device=DEV)
    sc = torch.empty(B, L, nb, dtype=q.dtype, device=DEV) if scores else None
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


def test_noalloc_pruned_and_split_paths_on_consecutive_calls():
    """Without scores_out the call also keeps the pruned scan's norm tables (prefill,
    L >= 64) or the split decode scan's partial lists (decode, nb >= 2048, B*L <= 256)
    in the shared array; back-to-back calls with different lambda, nb and batch make
    stale norms or partials from the previous call show up as wrong indices."""
    g = torch.Generator().manual_seed(77)
    cases = [  # (B, L, nb, top_k, lambda, decode, dtype)
        (2, 4096, 64, 32, 0.1, 0, torch.bfloat16),    # pruned tile scan
        (1, 4096, 4096, 32, 0.1, 1, torch.bfloat16),  # split decode: 8 splits of 512 candidates
        (1, 2048, 32, 32, 0.9, 0, torch.bfloat16),    # pruned again, other lambda / nb / B
        (4, 1, 2560, 16, 0.4, 1, torch.float32),      # split decode again, other lambda / nb / B
        (2, 4096, 64, 32, 0.1, 0, torch.bfloat16),    # the first case again after the others
    ]
    for B, L, nb, top_k, lam, decode, dt in cases:
        q = (torch.randn(B, L, 64, generator=g) / 11.3).to(DEV, dt)
        c = (torch.randn(B, nb, 64, generator=g) / 11.3).to(DEV, dt)
        rc, idx, _ = call_noalloc(q, c, lam, top_k, 64, decode, scores=False)
        assert rc == 0, N.lib().maba_last_error()
        ref_idx, _ = call_workspace(q, c, lam, top_k, 64, decode, scores=False)
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx), (B, L, nb, decode)


def test_noalloc_near_limit_falls_back_with_identical_indices():
    """nb = 65,000 fills the table almost to the limit, so the norm tables of the pruned
    scan no longer fit: the call runs the unpruned scan and must still give the
    workspace entry point's indices."""
    g = torch.Generator().manual_seed(78)
    q = (torch.randn(1, 128, 64, generator=g) / 11.3).to(DEV, torch.bfloat16)
    c = (torch.randn(1, 65000, 64, generator=g) / 11.3).to(DEV, torch.bfloat16)
    for lam in (0.1, 0.02):
        rc, idx, _ = call_noalloc(q, c, lam, 32, 64, 0, scores=False)
        assert rc == 0, N.lib().maba_last_error()
        ref_idx, _ = call_workspace(q, c, lam, 32, 64, 0, scores=False)
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)


def test_noalloc_rejects_requests_beyond_its_scratch():
    q = torch.randn(1, 70000, 8, device=DEV)
    c = torch.randn(1, 4, 8, device=DEV)
    rc, _, _ = call_noalloc(q, c, 0.5, 4, 1, 0, scores=False)  # block 1: 70,000 query blocks > 65,536 entries
    assert rc == N.ERR_UNSUPPORTED
    assert b"fixed scratch holds 65536" in N.lib().maba_last_error()
