"""Sequence split of one long sequence across ranks (maba_v2_architecture_b200.parallel),
checked on the CPU oracle: the in-process emulation of P ranks and a gloo world_size-2
run must both reproduce the single-sequence computation."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle.attention as oa
import oracle.dgda as od
import oracle.indexer as oi
from helpers import OracleBackend, assert_rel
from maba_v2_architecture_b200 import parallel as par


def _dgda_inputs(seed, B=1, H=2, L=192, d=64):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, d, generator=g, dtype=torch.float64) / d ** 0.5
    k = torch.nn.functional.normalize(torch.randn(B, H, L, d, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(B, H, L, d, generator=g, dtype=torch.float64)
    b = torch.sigmoid(torch.randn(B, H, L, 1, generator=g, dtype=torch.float64))
    w = torch.sigmoid(torch.randn(B, H, L, 1, generator=g, dtype=torch.float64))
    la = -torch.rand(B, H, L, d, generator=g, dtype=torch.float64) * 0.2
    return q, k, v, b, w, la


def _sa_inputs(seed, B=1, T=256, H=2, DC=128, D=64):
    g = torch.Generator().manual_seed(seed)
    qhat = torch.randn(B, T, H, DC, generator=g) * 0.1
    c = torch.randn(B, T, DC, generator=g)
    qi = torch.randn(B, T, D, generator=g)
    ki = torch.randn(B, T, D, generator=g)
    gate = torch.randn(B, T, 3, generator=g)
    return qhat, c, qi, ki, gate


def _seg(t, r, P, dim):
    n = t.shape[dim] // P
    return t.narrow(dim, r * n, n)


def test_transition_composes():
    q, k, v, b, w, la = _dgda_inputs(1, L=96)
    T = od.dgda_transition(q.numpy(), k.numpy(), v.numpy(), b=b.numpy(), w=w.numpy(), log_alpha=la.numpy())
    S0 = np.random.default_rng(0).standard_normal((1, 2, 64, 64))
    _, S_end = od.dgda_sequential(q, k, v, b=b, w=w, initial_state=S0, log_alpha=la)
    folded = par.fold_transitions([torch.from_numpy(T)], 1, torch.from_numpy(S0))
    assert_rel(folded.double(), S_end, 1e-5, "P S0 + R")


@pytest.mark.parametrize("P", [2, 3])
def test_dgda_sequence_split_emulated(P):
    q, k, v, b, w, la = _dgda_inputs(2, L=64 * P + 64 * (P == 2))
    be = OracleBackend()
    segs = [[_seg(t, r, P, 2) for t in (q, k, v, b, w, la)] for r in range(P)]
    trans = [par.dgda_segment_phase_a(*s, backend=be) for s in segs]
    outs = [par.dgda_segment_phase_b(*segs[r], trans, r, backend=be) for r in range(P)]
    o_ref, S_ref = od.dgda_sequential(q, k, v, b=b, w=w, log_alpha=la)
    assert_rel(torch.cat([o for o, _ in outs], dim=2), o_ref, 1e-5, "o")
    assert_rel(outs[-1][1], S_ref, 1e-5, "final state")


@pytest.mark.parametrize("P", [2, 3, 4])
def test_dgda_split_payload_protocol_emulated(P):
    """The exchanged payloads of sp_dgda_prefill: rank 0's final state as [S_end | 0],
    transitions of the middle ranks, zeros from the last; every rank's output pass from
    the folded state reproduces the single-sequence recurrence."""
    q, k, v, b, w, la = _dgda_inputs(9, L=64 * P)
    be = OracleBackend()
    segs = [[_seg(t, r, P, 2) for t in (q, k, v, b, w, la)] for r in range(P)]
    pays = [par.dgda_split_payload(*segs[r], r, P, backend=be) for r in range(P)]
    trans = [m for m, _ in pays]
    outs = [pays[0][1]] + [par.dgda_segment_phase_b(*segs[r], trans, r, backend=be) for r in range(1, P)]
    o_ref, S_ref = od.dgda_sequential(q, k, v, b=b, w=w, log_alpha=la)
    assert_rel(torch.cat([o for o, _ in outs], dim=2), o_ref, 1e-5, "o")
    assert_rel(outs[-1][1], S_ref, 1e-5, "final state")


@pytest.mark.parametrize("P", [2, 4])
def test_sa_sequence_split_emulated(P):
    qhat, c, qi, ki, gate = _sa_inputs(3, T=128 * P)
    p = par.SAParams(window=96, sinks=4, block=64, hca_r=64, top_k=3, lam=0.1)
    be = OracleBackend()
    parts = [par.sa_segment_phase_a(_seg(c, r, P, 1), _seg(ki, r, P, 1), p, backend=be) for r in range(P)]
    c_all, cent_all, hca_all = (list(x) for x in zip(*parts))
    res = [par.sa_segment_phase_b(_seg(qhat, r, P, 1), _seg(qi, r, P, 1), _seg(gate, r, P, 1), c_all, cent_all,
                                  hca_all, r, p, backend=be) for r in range(P)]
    cent = oi.compute_centroids(ki.numpy(), 64)
    idx_ref = oi.index_topk(qi.numpy(), cent, 0.1, 3, 64)
    assert np.array_equal(torch.cat([i for _, i in res], dim=1).numpy(), idx_ref)
    o_ref = oa.sa_attention_latent(qhat.numpy(), c.numpy(), idx_ref, gate.numpy(), 96, 4, 64, 64)
    assert_rel(torch.cat([o for o, _ in res], dim=1), o_ref, 1e-5, "latent output")


def _cut(t, bounds, r, dim):
    return t.narrow(dim, bounds[r], bounds[r + 1] - bounds[r])


def test_unequal_segments_emulated():
    """Contiguous segments of different lengths (as balanced_segments makes them)."""
    bounds = [0, 192, 256, 384]
    P = len(bounds) - 1
    be = OracleBackend()
    q, k, v, b, w, la = _dgda_inputs(7, L=bounds[-1])
    segs = [[_cut(t, bounds, r, 2) for t in (q, k, v, b, w, la)] for r in range(P)]
    trans = [par.dgda_segment_phase_a(*sg, backend=be) for sg in segs]
    outs = [par.dgda_segment_phase_b(*segs[r], trans, r, backend=be) for r in range(P)]
    o_ref, S_ref = od.dgda_sequential(q, k, v, b=b, w=w, log_alpha=la)
    assert_rel(torch.cat([o for o, _ in outs], dim=2), o_ref, 1e-5, "dgda o")
    assert_rel(outs[-1][1], S_ref, 1e-5, "dgda final state")
    qhat, c, qi, ki, gate = _sa_inputs(8, T=bounds[-1])
    p = par.SAParams(window=96, sinks=4, block=64, hca_r=64, top_k=3, lam=0.1)
    parts = [par.sa_segment_phase_a(_cut(c, bounds, r, 1), _cut(ki, bounds, r, 1), p, backend=be) for r in range(P)]
    c_all, cent_all, hca_all = (list(x) for x in zip(*parts))
    res = [par.sa_segment_phase_b(_cut(qhat, bounds, r, 1), _cut(qi, bounds, r, 1), _cut(gate, bounds, r, 1),
                                  c_all, cent_all, hca_all, r, p, backend=be) for r in range(P)]
    cent = oi.compute_centroids(ki.numpy(), 64)
    idx_ref = oi.index_topk(qi.numpy(), cent, 0.1, 3, 64)
    assert np.array_equal(torch.cat([i for _, i in res], dim=1).numpy(), idx_ref)
    o_ref = oa.sa_attention_latent(qhat.numpy(), c.numpy(), idx_ref, gate.numpy(), 96, 4, 64, 64)
    assert_rel(torch.cat([o for o, _ in res], dim=1), o_ref, 1e-5, "latent output")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balanced_segments(world):
    total, flat, slope = 1 << 20, 67.0, 1.0 / 4096
    bnd = par.balanced_segments(total, world, flat=flat, slope=slope)
    assert bnd[0] == 0 and bnd[-1] == total and len(bnd) == world + 1
    assert all(b % 64 == 0 for b in bnd) and all(x < y for x, y in zip(bnd, bnd[1:]))
    cost = [flat * (e - s) + 0.5 * slope * (e * e - s * s) for s, e in zip(bnd, bnd[1:])]
    assert max(cost) / min(cost) < 1.01
    assert bnd[1] - bnd[0] >= bnd[-1] - bnd[-2]  # later (longer-prefix) segments are shorter


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_split_bounds_equalise_rank_costs(world):
    total = 1 << 20
    bnd = par.split_bounds(total, world)
    assert bnd[0] == 0 and bnd[-1] == total and len(bnd) == world + 1
    assert all(b % 64 == 0 for b in bnd) and all(x < y for x, y in zip(bnd, bnd[1:]))
    k = 1e-3

    def cost(r, a, b):  # the model restated: attention + DGDA role + prefix receipt under the payload
        n = (b - a) * k
        attn = par.ATTN_FLAT * n + 0.5 * par.ATTN_SLOPE * ((b * k) ** 2 - (a * k) ** 2)
        if r == 0:
            return attn + par.DGDA_MS * n
        payload = par.TRANSITION * par.DGDA_MS * n if r < world - 1 else 0.0
        return attn + par.DGDA_MS * n + max(payload, par.XFER_MS * a * k)
    c = [cost(r, a, b) for r, (a, b) in enumerate(zip(bnd, bnd[1:]))]
    assert max(c) / min(c) < 1.01
    assert c == pytest.approx([par.split_cost(r, world, a, b) for r, (a, b) in enumerate(zip(bnd, bnd[1:]))])


def test_sa_split_rejects_ragged_segments():
    qhat, c, qi, ki, gate = _sa_inputs(4, T=96)
    with pytest.raises(ValueError, match="multiple of block"):
        par.sp_sa_prefill(qhat, c, qi, ki, gate, par.SAParams(), backend=OracleBackend())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, bounds):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        be = OracleBackend()
        q, k, v, b, w, la = _dgda_inputs(5, L=bounds[-1])
        o, S = par.sp_dgda_prefill(*[_cut(t, bounds, rank, 2) for t in (q, k, v, b, w, la)], backend=be)
        qhat, c, qi, ki, gate = _sa_inputs(6, T=bounds[-1])
        p = par.SAParams(window=96, sinks=4, block=64, hca_r=64, top_k=3, lam=0.1)
        so, sidx = par.sp_sa_prefill(*[_cut(t, bounds, rank, 1) for t in (qhat, c, qi, ki, gate)], p, backend=be)
        torch.save({"o": o, "S": S, "so": so, "sidx": sidx}, os.path.join(out_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bounds", [[0, 128, 256], [0, 192, 256], [0, 128, 192, 256, 384]],
                         ids=["equal", "unequal", "world4"])
def test_sequence_split_gloo(tmp_path, bounds):
    """world 2 (equal and unequal segments) and world 4 (rank 0's final state, two
    middle-rank transitions, the last rank's zeros) through the real collectives."""
    world = len(bounds) - 1
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), bounds), nprocs=world,
                       start_method="spawn")
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    q, k, v, b, w, la = _dgda_inputs(5, L=bounds[-1])
    o_ref, S_ref = od.dgda_sequential(q, k, v, b=b, w=w, log_alpha=la)
    assert_rel(torch.cat([r["o"] for r in res], dim=2), o_ref, 1e-5, "dgda o")
    assert_rel(res[-1]["S"], S_ref, 1e-5, "dgda final state")
    qhat, c, qi, ki, gate = _sa_inputs(6, T=bounds[-1])
    idx_ref = oi.index_topk(qi.numpy(), oi.compute_centroids(ki.numpy(), 64), 0.1, 3, 64)
    assert np.array_equal(torch.cat([r["sidx"] for r in res], dim=1).numpy(), idx_ref)
    o_sa = oa.sa_attention_latent(qhat.numpy(), c.numpy(), idx_ref, gate.numpy(), 96, 4, 64, 64)
    assert_rel(torch.cat([r["so"] for r in res], dim=1), o_sa, 1e-5, "sa latent output")
