"""Sequence split on the GPU: the segment transition kernel vs the oracle, the split
computation emulated on one GPU vs the unsplit kernels, and (with two or more GPUs)
the NCCL world-2 run."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import maba_v2_architecture_b200 as mb
from helpers import RTOL_BF16, RTOL_FP32, assert_rel
from maba_v2_architecture_b200 import parallel as par
from maba_v2_architecture_b200.ops import absorb_queries
from maba_v2_architecture_b200.workloads import dgda_inputs, sa_inputs
from oracle import dgda as OD

pytestmark = pytest.mark.gpu
DEV = "cuda"
KEYS = ("q", "k", "v", "b", "w", "log_alpha")


def _dgda(T, dtype, seed=0, B=1, H=2):
    d = dgda_inputs(B=B, T=T, H=H, seed=seed, per_channel=True)
    return [d[k].to(DEV, dtype) for k in KEYS]


@pytest.mark.parametrize("dtype,L,rtol", [(torch.float32, 200, RTOL_FP32), (torch.float32, 64, RTOL_FP32),
                                          (torch.bfloat16, 1000, RTOL_BF16), (torch.float16, 333, RTOL_BF16)])
def test_transition_vs_oracle(dtype, L, rtol):
    q, k, v, b, w, la = _dgda(L, dtype, seed=3)
    t = mb.b200_dgda_transition(q, k, v, b=b, w=w, log_alpha=la)
    torch.cuda.synchronize()
    want = OD.dgda_transition(*(x.double().cpu().numpy() for x in (q, k, v)), b=b.double().cpu().numpy(),
                              w=w.double().cpu().numpy(), log_alpha=la.double().cpu().numpy())
    assert t.shape == (1, 2, 64, 128) and t.dtype == torch.float32
    assert_rel(t[..., :64], want[..., :64], rtol, "R")
    assert_rel(t[..., 64:], want[..., 64:], rtol, "P")


def test_transition_chains_prefill():
    """prefill(second half, S = P S_first + R) equals the unsplit prefill."""
    q, k, v, b, w, la = _dgda(4096, torch.bfloat16, seed=4)
    o_full, S_full = mb.b200_dgda_prefill(q, k, v, None, b, w, log_alpha=la, state_dtype=torch.float32)
    P = 4
    segs = [[x.narrow(2, r * 1024, 1024) for x in (q, k, v, b, w, la)] for r in range(P)]
    trans = [par.dgda_segment_phase_a(*s) for s in segs]
    outs = [par.dgda_segment_phase_b(*segs[r], trans, r) for r in range(P)]
    torch.cuda.synchronize()
    assert_rel(torch.cat([o for o, _ in outs], dim=2), o_full, RTOL_BF16, "o")
    folded = par.fold_transitions(trans, P)[..., :64, :64]
    # two 16-bit paths (segment transitions vs the whole-sequence prefill) agree closely ...
    assert_rel(outs[-1][1], S_full, RTOL_BF16 / 4, "final state")
    assert_rel(folded, S_full, RTOL_BF16 / 4, "folded state")
    # ... and both match the fp64 recurrence on the 16-bit inputs
    ro, rS = OD.dgda_sequential(*(x.double().cpu().numpy() for x in (q, k, v)), b=b.double().cpu().numpy(),
                                w=w.double().cpu().numpy(), log_alpha=la.double().cpu().numpy())
    assert_rel(o_full, ro, RTOL_BF16, "o vs oracle")
    assert_rel(S_full, rS, RTOL_BF16, "S vs oracle")
    assert_rel(folded, rS, RTOL_BF16, "folded S vs oracle")


def _sa_parts(T, seed=5):
    wl = sa_inputs(T=T, H=4, seed=seed)
    qhat = absorb_queries(wl.q.to(DEV, torch.bfloat16), wl.w_uk.to(DEV, torch.bfloat16), wl.H, wl.dh ** -0.5)
    return (qhat, wl.c_kv.to(DEV, torch.bfloat16), wl.q_idx.to(DEV, torch.bfloat16), wl.k_idx.to(DEV, torch.bfloat16),
            wl.gate.to(DEV, torch.bfloat16))


def _sa_full(qhat, c, qi, ki, gate, p):
    cent = mb.b200_compute_centroids(ki, block_size=p.block)
    idx = mb.b200_index_topk(qi, cent, lambda_dist=p.lam, top_k=p.top_k, block_size=p.block)
    o = mb.b200_sa_attention(qhat, c, mb.b200_hca_pool(c, p.hca_r), idx, gate, window_size=p.window,
                             n_sinks=p.sinks, block_size=p.block, hca_r=p.hca_r)
    return o, idx


def test_sa_split_emulated_matches_unsplit():
    P, T = 4, 4096
    parts = _sa_parts(T)
    p = par.SAParams(lam=0.1)
    o_full, idx_full = _sa_full(*parts, p)
    qhat, c, qi, ki, gate = parts
    seg = lambda t, r: t.narrow(1, r * (T // P), T // P)  # noqa: E731
    ph = [par.sa_segment_phase_a(seg(c, r), seg(ki, r), p) for r in range(P)]
    c_all, cent_all, hca_all = (list(x) for x in zip(*ph))
    res = [par.sa_segment_phase_b(seg(qhat, r), seg(qi, r), seg(gate, r), c_all, cent_all, hca_all, r, p)
           for r in range(P)]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([i for _, i in res], dim=1), idx_full)
    assert_rel(torch.cat([o for o, _ in res], dim=1), o_full, RTOL_BF16, "latent output")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        T = 2048 * world
        q, k, v, b, w, la = (x.to(f"cuda:{rank}") for x in _dgda(T, torch.bfloat16, seed=6))
        Ls = T // world
        o, S = par.sp_dgda_prefill(*[x.narrow(2, rank * Ls, Ls) for x in (q, k, v, b, w, la)])
        parts = [x.to(f"cuda:{rank}") for x in _sa_parts(T, seed=7)]
        so, sidx = par.sp_sa_prefill(*[x.narrow(1, rank * Ls, Ls) for x in parts], par.SAParams(lam=0.1))
        torch.cuda.synchronize()
        torch.save({"o": o.cpu(), "S": S.cpu(), "so": so.cpu(), "sidx": sidx.cpu()}, os.path.join(out_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_split_nccl_world2(tmp_path):
    world = 2
    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    T = 2048 * world
    q, k, v, b, w, la = _dgda(T, torch.bfloat16, seed=6)
    o_full, S_full = mb.b200_dgda_prefill(q, k, v, None, b, w, log_alpha=la, state_dtype=torch.float32)
    assert_rel(torch.cat([r["o"] for r in res], dim=2), o_full, RTOL_BF16, "dgda o")
    assert_rel(res[-1]["S"], S_full, RTOL_FP32 * 10, "dgda state")
    o_sa, idx = _sa_full(*_sa_parts(T, seed=7), par.SAParams(lam=0.1))
    assert torch.equal(torch.cat([r["sidx"] for r in res], dim=1), idx.cpu())
    assert_rel(torch.cat([r["so"] for r in res], dim=1), o_sa, RTOL_BF16, "sa output")
