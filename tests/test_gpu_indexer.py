"""DG-Indexer kernels (pooling, scoring + top-k) and stream superposition vs the
CPU oracle (bit-exact scores and indices) and the reference's golden outputs
(indices under the tie rule)."""
import numpy as np
import pytest
import torch

import maba_v2_architecture_b200 as mb
from helpers import RTOL_BF16, assert_rel, check_topk_rule, golden, sub
from maba_v2_architecture_b200.workloads import sa_inputs
from oracle import indexer as OI

pytestmark = pytest.mark.gpu
DEV = "cuda"


def cu(x, dtype=torch.float32):
    return torch.as_tensor(np.asarray(x)).to(DEV, dtype)


@pytest.mark.parametrize("name,block", [("needle", 64), ("tail", 64), ("hyb", 4), ("mis1", 64), ("mis63", 64),
                                        ("mis65", 64), ("mis129", 64), ("mis257", 64)])
def test_centroids(name, block):
    g = sub(golden("indexer"), f"{name}.")
    c = mb.b200_compute_centroids(cu(g["k"]), block_size=block).cpu().numpy()
    np.testing.assert_allclose(c, g["c"], rtol=1e-6, atol=1e-6)
    assert np.array_equal(c, OI.compute_centroids(g["k"], block))  # same sequential fp32 arithmetic


def test_centroids_bf16_and_strided():
    g = sub(golden("indexer"), "bf16.")
    c = mb.b200_compute_centroids(cu(g["k"], torch.bfloat16))
    assert c.dtype == torch.bfloat16
    np.testing.assert_allclose(c.float().cpu().numpy(), g["c"], atol=1e-2)
    k = torch.randn(2, 64, 300, device=DEV).transpose(1, 2)  # strided [B,L,d]
    np.testing.assert_array_equal(mb.b200_compute_centroids(k).cpu().numpy(),
                                  OI.compute_centroids(k.cpu().numpy(), 64))


@pytest.mark.parametrize("L", [64, 100, 1000, 4097])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_vectorised_pooling_matches_oracle(L, dtype):
    """Unit-stride rows take the 16-byte row-load pooling: batch 2, ragged tail blocks,
    D = 64 (centroids) and D = 128 (HCA rows).  Centroids equal the oracle's sequential
    fp32 sums bit for bit (then rounded to the output dtype); the HCA means (complete
    blocks only) match the fp64 oracle."""
    g = torch.Generator().manual_seed(L)
    k = (torch.randn(2, L, 64, generator=g) / 8).to(dtype)
    c = mb.b200_compute_centroids(k.to(DEV), block_size=64)
    ref = torch.from_numpy(OI.compute_centroids(k.float().numpy(), 64)).to(dtype)
    assert c.dtype == dtype and torch.equal(c.cpu(), ref)
    ckv = (torch.randn(2, L, 128, generator=g) / 8).to(dtype)
    for out_dtype in (None, torch.float32):
        h = mb.b200_hca_pool(ckv.to(DEV), 64, out_dtype=out_dtype)
        href = OI.hca_pool(ckv.float().numpy(), 64)
        assert tuple(h.shape) == href.shape == (2, L // 64, 128)
        tol = 1e-5 if (out_dtype == torch.float32 or dtype == torch.float32) else 1e-2
        np.testing.assert_allclose(h.float().cpu().numpy(), href, rtol=tol, atol=tol * 1e-2)


def _tk_inputs(ci, B, L):
    torch.manual_seed(400 + ci)
    return torch.randn(B, L, 64), torch.randn(B, L, 64)


@pytest.mark.parametrize("ci", range(11))
def test_topk_cases(ci):
    g = sub(golden("indexer"), f"tk{ci}.")
    B, L, top_k, lam = g["meta"].tolist()
    B, L, top_k = int(B), int(L), int(top_k)
    q, k = _tk_inputs(ci, B, L)
    c = mb.b200_compute_centroids(k.to(DEV))
    idx, sc = mb.b200_index_topk(q.to(DEV), c, lambda_dist=lam, top_k=top_k, return_scores=True)
    assert idx.dtype == torch.long and idx.shape == (B, L, min(top_k, c.shape[1]))
    cn = c.cpu().numpy()
    oidx, osc = OI.index_topk(q.numpy(), cn, lambda_dist=lam, top_k=top_k, return_scores=True)
    np.testing.assert_array_equal(sc.cpu().numpy(), osc)          # bit-exact scores (incl. -inf)
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)        # bit-exact indices (incl. filler rule)
    # against the reference's own indices: measured 0 tie-classified rows in every case
    assert check_topk_rule(g["idx"], osc, np.arange(L) // 64, top_k) == 0


def test_topk_monotone_and_clamp():
    g = sub(golden("indexer"), "mono.")
    idx = mb.b200_index_topk(cu(g["q"]), cu(g["c"]), lambda_dist=1.0, top_k=4, block_size=64)
    assert idx[0, 255].tolist() == [3, 2, 1, 0]
    q = torch.randn(2, 32, 64, device=DEV)
    c = torch.randn(2, 1, 64, device=DEV)
    idx = mb.b200_index_topk(q, c, top_k=32, block_size=64)
    assert idx.shape == (2, 32, 1) and bool((idx == 0).all())


@pytest.mark.parametrize("L", [1024, 4096])
def test_topk_needle_rank0(L):
    torch.manual_seed(42)
    k = torch.randn(1, L, 64)
    k[:, 5 * 64 + 10, 0] = 25.0
    q = torch.randn(1, L, 64) * 0.1
    q[:, -1, 0] = 5.0
    c = mb.b200_compute_centroids(k.to(DEV))
    idx = mb.b200_index_topk(q.to(DEV), c, lambda_dist=0.5, top_k=32)
    assert idx[0, -1, 0].item() == 5
    np.testing.assert_array_equal(idx[0, -1].cpu().numpy(), golden("indexer")[f"nd{L}.idx_last"])


def test_topk_decode_inline():
    g = sub(golden("indexer"), "dec.")
    w = sub(g, "w.")
    qi = (g["x"].astype(np.float32) @ w["q_idx_proj.weight"].T).astype(np.float32)
    for j in range(20):
        c = g[f"{j}.c"]
        q1 = qi[:, 50 + j:51 + j]
        idx, s = mb.b200_index_topk(cu(q1), cu(c), lambda_dist=0.5, top_k=8, block_size=16, return_scores=True,
                                    decode=True)
        oidx, osc = OI.index_topk(q1, c, lambda_dist=0.5, top_k=8, block_size=16, return_scores=True, decode=True)
        np.testing.assert_array_equal(s.cpu().numpy(), osc)
        np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
        np.testing.assert_allclose(osc, g[f"{j}.scores"], rtol=1e-5, atol=1e-5)
        check_topk_rule(g[f"{j}.idx"], osc, np.array([c.shape[1] - 1]), 8)


def test_topk_large_k_sort_path():
    q = torch.randn(2, 4096, 64)
    k = torch.randn(2, 4096, 64)
    c = mb.b200_compute_centroids(k.to(DEV))
    idx, s = mb.b200_index_topk(q.to(DEV), c, lambda_dist=0.3, top_k=40, return_scores=True)
    oidx, osc = OI.index_topk(q.numpy(), c.cpu().numpy(), lambda_dist=0.3, top_k=40, return_scores=True)
    np.testing.assert_array_equal(s.cpu().numpy(), osc)
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)


def test_topk_bf16_inputs_upcast():
    q = torch.randn(1, 700, 64).to(torch.bfloat16)
    c = torch.randn(1, 11, 64).to(torch.bfloat16)
    idx, s = mb.b200_index_topk(q.to(DEV), c.to(DEV), lambda_dist=0.5, top_k=6, return_scores=True)
    assert s.dtype == torch.bfloat16
    oidx, osc = OI.index_topk(q.float().numpy(), c.float().numpy(), lambda_dist=0.5, top_k=6, return_scores=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_array_equal(s.float().cpu().numpy(), torch.from_numpy(osc).to(torch.bfloat16).float().numpy())


def test_config2_full_size():
    """T=65,536, nb=1,024, lambda=0.1, top-32: sampled rows bit-exact vs the oracle,
    reference indices under the tie rule, structural properties on every row."""
    g = sub(golden("indexer"), "cfg2.")
    wl = sa_inputs()
    c = mb.b200_compute_centroids(wl.k_idx.to(DEV))
    assert abs(c.double().sum().item() - float(g["c_sum"])) < 1e-3
    idx = mb.b200_index_topk(wl.q_idx.to(DEV), c, lambda_dist=0.1, top_k=32, block_size=64)
    rows = g["rows"]
    oidx, osc = OI.index_topk(wl.q_idx.numpy(), c.cpu().numpy(), lambda_dist=0.1, top_k=32, return_scores=True,
                              rows=rows)
    got = idx[0, torch.as_tensor(rows, device=DEV)].cpu().numpy()
    np.testing.assert_array_equal(got, oidx[0])
    assert check_topk_rule(g["idx"][None], osc, rows // 64, 32) == 0  # measured: no tie rows
    # every row: first min(32, qb+1) entries are distinct causal blocks, fillers ascending after them
    qb = torch.arange(65536, device=DEV) // 64
    nvalid = torch.clamp(qb + 1, max=32)
    slot = torch.arange(32, device=DEV)
    i0 = idx[0]
    causal_ok = torch.where(slot[None] < nvalid[:, None], i0 <= qb[:, None], i0 == (slot[None] + 0))
    assert bool(causal_ok.all())
    srt = torch.sort(i0, dim=1).values
    assert bool((srt[:, 1:] != srt[:, :-1]).all())
    hit = (i0[wl.probe] == wl.needle_block).nonzero()
    assert (int(hit[0, 0]) if hit.numel() else -1) == int(g["needle_rank"])


def test_superposition():
    g = golden("superposition")
    t = {k: cu(g[k]) for k in ("ol", "os", "oh", "g3", "g4", "gw")}
    o3 = mb.b200_stream_superposition(t["ol"], t["os"], t["oh"], gate_logits=t["g3"])
    o4 = mb.b200_stream_superposition(t["ol"], t["os"], t["oh"], gate_logits=t["g4"])
    ow = mb.b200_stream_superposition(t["ol"], t["os"], t["oh"], gate_weights=t["gw"])
    np.testing.assert_allclose(o3.cpu().numpy(), g["o3"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(o4.cpu().numpy(), g["o4"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ow.cpu().numpy(), g["ow"], rtol=1e-5, atol=1e-6)
    ob = mb.b200_stream_superposition(*(t[k].to(torch.bfloat16) for k in ("ol", "os", "oh")),
                                      gate_logits=t["g3"].to(torch.bfloat16))
    assert ob.dtype == torch.bfloat16
    assert_rel(ob, g["o3"], RTOL_BF16, "bf16")
    # strided inputs
    olT = t["ol"].transpose(2, 3).contiguous().transpose(2, 3)
    np.testing.assert_allclose(mb.b200_stream_superposition(olT, t["os"], t["oh"], gate_logits=t["g3"]).cpu().numpy(),
                               g["o3"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", ["cfg2_bf16", "far_large_norms", "ties_lambda0", "fp32_scores_off"])
def test_topk_pruned_scan_exact(case):
    """The tile scan stops once |q| max|c| minus the smallest penalty left is strictly
    below every token's k-th best: indices stay bit-identical to the full oracle scan,
    including far blocks with large norms and exact ties (the lower index wins)."""
    g = torch.Generator().manual_seed(77)
    L, D = 8192, 64
    nb = L // 64
    lam, dt = 0.1, torch.float32
    q = torch.randn(1, L, D, generator=g) / np.sqrt(128)
    if case == "cfg2_bf16":
        c = mb.b200_compute_centroids((torch.randn(1, L, D, generator=g) / np.sqrt(128)).to(DEV)).cpu()
        dt = torch.bfloat16
    elif case == "far_large_norms":
        scale = 1.0 + 6.0 * (nb - torch.arange(nb, dtype=torch.float32)) / nb  # far blocks up to 7x larger
        c = torch.randn(1, nb, D, generator=g) * scale[None, :, None]
        lam = 0.01
    elif case == "ties_lambda0":
        c = torch.randn(1, nb, D, generator=g)
        c[:, :64] = c[:, 64:128]  # block n and n + 64 identical: equal scores, lower index first
        lam = 0.0
    else:
        c = torch.randn(1, nb, D, generator=g)
    qd, cd = q.to(dt), c.to(dt)
    idx = mb.b200_index_topk(qd.to(DEV), cd.to(DEV), lambda_dist=lam, top_k=32, block_size=64)
    rows = np.arange(0, L, 7)
    oidx = OI.index_topk(qd.float().numpy(), cd.float().numpy(), lambda_dist=lam, top_k=32, rows=rows)
    np.testing.assert_array_equal(idx[0, torch.as_tensor(rows, device=DEV)].cpu().numpy(), oidx[0])
    if case == "fp32_scores_off":
        idx2, _ = mb.b200_index_topk(qd.to(DEV), cd.to(DEV), lambda_dist=lam, top_k=32, block_size=64,
                                     return_scores=True)  # scores requested: the unpruned scan
        assert torch.equal(idx, idx2)
