"""Multi-GPU execution of the hot path: one process per GPU, torch.distributed.

Two layouts:

* **batch sharding** -- independent sequences per rank; nothing crosses GPUs on
  the data path (``bench.py --gpus N`` runs it).
* **sequence split** -- one long sequence cut into P contiguous segments, rank r
  holding tokens [r*Ls, (r+1)*Ls) with Ls a multiple of the block size.  The
  reference never splits a sequence; this layout adds one small exchange per
  layer and keeps every result equal to the single-GPU computation:

  - DGDA: the recurrence is affine in the state, so each rank computes its
    segment's transition S_end = P S_start + R (``b200_dgda_transition``), the
    ranks all-gather the [B,H,64,128] fp32 transitions (320 KB per rank at
    H=10), each folds the preceding ones into its starting state and runs the
    output pass from it;
  - MABA-SA: a query may attend any earlier token (sparse blocks anywhere in the
    prefix, HCA over all complete blocks, the window and sinks), so the ranks
    exchange the latent rows, the block centroids and the pooled HCA rows
    (d_c=128 / d_idx=64 per token or block) as a prefix exchange -- rank j sends
    its rows to the later ranks only, into their preallocated whole-sequence
    tables; each rank then scores and attends its own queries at their
    absolute positions (``q_pos0``; the attention's queries sit at the end of
    the received prefix).

Each layout is written as local phases around one exchange so the same code
runs with NCCL (one process per GPU), with gloo on CPU (tests inject a CPU
backend), or as an emulation of the ranks inside one process.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import ops as _ops

DP = 64  # padded head dim of the transition


class B200Backend:
    """The sm_100a kernels."""

    def dgda_transition(self, q, k, v, b, w, la):
        return _ops.b200_dgda_transition(q, k, v, None, b, w, log_alpha=la)

    def dgda_prefill(self, q, k, v, b, w, la, initial_state):
        return _ops.b200_dgda_prefill(q, k, v, None, b, w, initial_state=initial_state, log_alpha=la,
                                      state_dtype=torch.float32)

    def compute_centroids(self, k_idx, block):
        return _ops.b200_compute_centroids(k_idx, block_size=block)

    def hca_pool(self, c, r):
        return _ops.b200_hca_pool(c, r)

    def index_topk_at(self, q_idx, cent, lam, top_k, block, q_pos0):
        return _ops.b200_index_topk(q_idx, cent, lambda_dist=lam, top_k=top_k, block_size=block, q_pos0=q_pos0)

    def sa_attention(self, qhat, c, hca, idx, gate, window, sinks, block, r):
        return _ops.b200_sa_attention(qhat, c, hca, idx, gate, window_size=window, n_sinks=sinks, block_size=block,
                                      hca_r=r)


def fold_transitions(trans: Sequence[torch.Tensor], upto: int, s0: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Starting state of segment `upto` from the transitions [R | P] of segments 0..upto-1."""
    t0 = trans[0]
    B, H = t0.shape[:2]
    S = torch.zeros(B, H, DP, DP, dtype=torch.float32, device=t0.device) if s0 is None else s0.float()
    for j in range(upto):
        R, P = trans[j][..., :DP].float(), trans[j][..., DP:].float()
        S = torch.matmul(P, S) + R
    return S


def _gather(t: torch.Tensor, group) -> List[torch.Tensor]:
    world = dist.get_world_size(group)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t.contiguous(), group=group)
    return out


def balanced_segments(total: int, world: int, unit: int = 64, flat: float = 67.0, slope: float = 1.0 / 4096) -> List[int]:
    """Segment boundaries [0, b_1, ..., total] (multiples of `unit`) that give every rank the
    same work under a per-token cost flat + slope * position: the three-stream attention
    grows with the position through the pooled-HCA stream (pos / (64 * 64) key tiles of 64
    per query tile and head pair) while DGDA and the other streams cost the same per token
    (`flat`, in the same tile units, from the measured single-GPU split of the step)."""
    def cost(x):
        return flat * x + 0.5 * slope * x * x
    tot = cost(total)
    bounds = [0]
    for r in range(1, world):
        target = tot * r / world
        # solve cost(x) = target for x >= 0
        a, b_, c = 0.5 * slope, flat, -target
        x = (-b_ + (b_ * b_ - 4 * a * c) ** 0.5) / (2 * a) if a > 0 else target / flat
        x = int(round(x / unit)) * unit
        bounds.append(min(max(x, bounds[-1] + unit), total - (world - r) * unit))
    bounds.append(total)
    return bounds


# measured per-token costs on one B200 (ms per 1,000 tokens, bf16, H = 10): the attention
# of a query at position p (in thousands of tokens) costs ATTN_FLAT + ATTN_SLOPE * p (the
# pooled-HCA stream grows with the prefix), the DGDA prefill DGDA_MS; a segment transition
# costs about TRANSITION times its prefill (measured on eight B200s at 1,048,576 tokens: a
# middle rank's transition 1.8-1.9x its output pass).  The MABA-SA prefix exchange took 1-2 ms
# on every rank alike (senders and receivers), so by default it does not move the bounds;
# XFER_MS per thousand received prefix tokens models an exchange that overlaps the transition.
ATTN_FLAT, ATTN_SLOPE, DGDA_MS, TRANSITION, XFER_MS = 0.0159, 7.54e-5, 0.0092, 1.9, 0.0


def split_cost(r: int, world: int, a: int, b: int, attn_flat: float = ATTN_FLAT, attn_slope: float = ATTN_SLOPE,
               dgda: float = DGDA_MS, transition: float = TRANSITION, xfer: float = XFER_MS) -> float:
    """Modelled device time (ms) of rank r holding tokens [a, b) of a split: its queries'
    attention (flat + slope * position per token), its DGDA role (rank 0 one prefill; ranks
    1..P-2 a transition, then an output pass; the last rank an output pass) and the receipt
    of the prefix tables, which overlaps the transition."""
    k = 1e-3  # costs are per thousand tokens
    n = (b - a) * k
    attn = attn_flat * n + 0.5 * attn_slope * ((b * k) ** 2 - (a * k) ** 2)
    if r == 0:
        return attn + dgda * n
    payload = transition * dgda * n if r < world - 1 else 0.0
    return attn + dgda * n + max(payload, xfer * a * k)


def split_bounds(total: int, world: int, unit: int = 64, attn_flat: float = ATTN_FLAT,
                 attn_slope: float = ATTN_SLOPE, dgda: float = DGDA_MS, transition: float = TRANSITION,
                 xfer: float = XFER_MS) -> List[int]:
    """Segment boundaries [0, b_1, ..., total] (multiples of `unit`) that equalise each rank's
    modelled share of the split prefill (split_cost).  Found by bisection on the per-rank
    budget: each rank takes the longest segment that fits it, and the last rank must fit too."""
    if world == 1:
        return [0, total]

    def cost(r, a, b):
        return split_cost(r, world, a, b, attn_flat, attn_slope, dgda, transition, xfer)

    def assign(budget):
        bounds, a = [0], 0
        for r in range(world - 1):
            lo, hi = a + unit, total - (world - 1 - r) * unit
            if lo > hi:
                return None
            if cost(r, a, lo) > budget:
                b = lo
            else:
                while hi - lo > unit:          # largest b with cost <= budget
                    mid = (lo + hi) // (2 * unit) * unit
                    if mid <= lo:
                        break
                    if cost(r, a, mid) <= budget:
                        lo = mid
                    else:
                        hi = mid
                b = hi if cost(r, a, hi) <= budget else lo
            bounds.append(b)
            a = b
        bounds.append(total)
        return bounds

    lo_b, hi_b = 0.0, cost(0, 0, total) * 2.5
    best = assign(hi_b)
    for _ in range(60):
        mid = 0.5 * (lo_b + hi_b)
        bd = assign(mid)
        if bd is not None and cost(world - 1, bd[-2], total) <= mid:
            hi_b, best = mid, bd
        else:
            lo_b = mid
    return best


# ------------------------------------------------------------------ DGDA
def dgda_segment_phase_a(q, k, v, b, w, la, backend=None):
    """Local: the segment's transition."""
    backend = backend or B200Backend()
    return backend.dgda_transition(q, k, v, b, w, la)


def dgda_segment_phase_b(q, k, v, b, w, la, trans: Sequence[torch.Tensor], rank: int, backend=None):
    """Local: output pass of segment `rank` from the state folded out of the preceding transitions."""
    backend = backend or B200Backend()
    dk, dv = q.shape[-1], v.shape[-1]
    S = fold_transitions(trans, rank)[..., :dk, :dv].contiguous()
    return backend.dgda_prefill(q, k, v, b, w, la, S)


def dgda_split_payload(q, k, v, b, w, la, rank: int, world: int, backend=None):
    """Local part before the exchange of the sequence-split DGDA prefill.  Rank 0 runs its
    prefill at once and publishes its final state as the transition [S_end | 0] (P = 0,
    so folding it yields S_end whatever came before); ranks 1..world-2 publish their
    transitions; the last rank's would never be used, so it sends zeros.
    Returns (payload [B,H,64,128] fp32, (o, S_end) for rank 0 else None)."""
    backend = backend or B200Backend()
    B, H = q.shape[:2]
    dk, dv = q.shape[-1], v.shape[-1]
    if rank == 0:
        o, S_end = backend.dgda_prefill(q, k, v, b, w, la, None)
        mine = torch.zeros(B, H, DP, 2 * DP, dtype=torch.float32, device=q.device)
        mine[..., :dk, :dv] = S_end.float().to(q.device)
        return mine, (o, S_end)
    if rank < world - 1:
        return dgda_segment_phase_a(q, k, v, b, w, la, backend), None
    return torch.zeros(B, H, DP, 2 * DP, dtype=torch.float32, device=q.device), None


def sp_dgda_prefill(q, k, v, b, w, la, group=None, backend=None):
    """Sequence-split DGDA prefill: this rank's segment of q..la ([B,H,Ls,d] views).
    Returns (o of the segment, state at the end of the segment).  One all-gather of
    the payloads of ``dgda_split_payload``; every rank r > 0 then folds the first r
    entries into its starting state and runs its output pass."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    mine, done = dgda_split_payload(q, k, v, b, w, la, rank, world, backend)
    trans = _gather(mine, group)
    if done is not None:
        return done
    return dgda_segment_phase_b(q, k, v, b, w, la, trans, rank, backend)


# ------------------------------------------------------------------ MABA-SA
@dataclass
class SAParams:
    window: int = 128
    sinks: int = 4
    block: int = 64
    hca_r: int = 64
    top_k: int = 32
    lam: float = 0.1


def sa_segment_phase_a(c_local, k_idx_local, p: SAParams, backend=None):
    """Local: the segment's latent rows, block centroids and pooled HCA rows (to be exchanged)."""
    backend = backend or B200Backend()
    return c_local, backend.compute_centroids(k_idx_local, p.block), backend.hca_pool(c_local, p.hca_r)


def sa_segment_phase_b(qhat_local, q_idx_local, gate_local, c_all: Sequence[torch.Tensor],
                       cent_all: Sequence[torch.Tensor], hca_all: Sequence[torch.Tensor], rank: int, p: SAParams,
                       backend=None):
    """Local: indexer + three-stream attention of this segment's queries over the gathered prefix.
    Block indices past the prefix (fillers) are dropped by the attention; every token they
    name lies after the query, which the reference's causal mask of the gathered tokens
    removes as well (maba_sparse/layers/sparse_attention.py:117-164)."""
    backend = backend or B200Backend()
    Ls = qhat_local.shape[1]
    start = sum(int(c.shape[1]) for c in c_all[:rank])  # segments may differ in length
    end = start + Ls
    c_prefix = torch.cat(list(c_all[: rank + 1]), dim=1)
    # The whole centroid table: future blocks score -inf, but the table's length sets
    # min(top_k, nb) and the filler indices, which then match the single-GPU indexer.
    cent = torch.cat(list(cent_all), dim=1)
    hca = torch.cat(list(hca_all[: rank + 1]), dim=1)
    idx = backend.index_topk_at(q_idx_local, cent, p.lam, p.top_k, p.block, start)
    o = backend.sa_attention(qhat_local, c_prefix, hca if hca.shape[1] else None, idx, gate_local, p.window,
                             p.sinks, p.block, p.hca_r)
    assert c_prefix.shape[1] == end
    return o, idx


def exchange_prefix(bufs: Sequence[torch.Tensor], bounds: Sequence[int], units: Sequence[int], rank: int,
                    group=None, wait: bool = True, how: str = "p2p"):
    """Prefix exchange of per-token tables between the ranks of a sequence split.

    ``bufs[i]`` is a [B, bounds[-1] // units[i], d] table (one row per ``units[i]``
    tokens) in which this rank's own rows, ``bounds[rank] // u .. bounds[rank+1] // u``,
    are already in place.  Afterwards rows ``0 .. bounds[rank+1] // u`` hold every earlier
    rank's rows too: rank j sends its rows to every later rank only (point-to-point, one
    batch), since no query attends a later segment.  Rows of later ranks are left as they
    were.  Every rank issues its sends and receives in the same order, so the batch pairs
    up; the exchange is asynchronous to the host (NCCL runs it on its own stream and the
    current stream waits for it).  With ``wait=False`` the requests are returned instead and
    the caller waits on them later (work queued on the current stream meanwhile overlaps the
    transfers).

    ``how="broadcast"`` sends each rank's rows to every rank with one broadcast per table and
    source instead (later ranks' rows too, which no query reads).  On eight B200s both forms
    took 1-3 ms for the 1,048,576-token tables (13.4 ms against 12.5-13.2 ms for the whole
    split), so the point-to-point batch, which moves fewer bytes, is the default."""
    world = len(bounds) - 1
    if how == "broadcast":
        reqs = []
        for buf, u in zip(bufs, units):
            for bi in range(buf.shape[0]):
                for j in range(world - 1):  # the last rank's rows precede no query
                    lo, hi = bounds[j] // u, bounds[j + 1] // u
                    if hi > lo:
                        reqs.append(dist.broadcast(buf[bi, lo:hi], src=j, group=group, async_op=True))
        if not wait:
            return reqs
        for req in reqs:
            req.wait()
        return None
    ops = []
    for buf, u in zip(bufs, units):
        for bi in range(buf.shape[0]):
            for j in range(world):
                if j == rank:
                    continue
                seg = j if j < rank else rank      # rows received from j, or this rank's rows sent to j
                lo, hi = bounds[seg] // u, bounds[seg + 1] // u
                if hi > lo:
                    ops.append(dist.P2POp(dist.irecv if j < rank else dist.isend, buf[bi, lo:hi], j, group))
    reqs = dist.batch_isend_irecv(ops) if ops else []
    if not wait:
        return reqs
    for req in reqs:
        req.wait()
    return None


def sa_segment_tables(c_buf: torch.Tensor, cent_buf: torch.Tensor, hca_buf: torch.Tensor, k_idx_local: torch.Tensor,
                      start: int, p: SAParams, backend=None) -> None:
    """Local: this rank's block centroids and pooled HCA rows, written into their rows of the
    whole-sequence tables (its latent rows are already in ``c_buf[:, start:start+Ls]``)."""
    backend = backend or B200Backend()
    Ls = k_idx_local.shape[1]
    nb0, nb = start // p.block, Ls // p.block
    nh0, nh = start // p.hca_r, Ls // p.hca_r
    cent_buf[:, nb0:nb0 + nb] = backend.compute_centroids(k_idx_local, p.block)
    if nh:
        hca_buf[:, nh0:nh0 + nh] = backend.hca_pool(c_buf[:, start:start + Ls], p.hca_r)


def sa_segment_attention(qhat_local, q_idx_local, gate_local, c_buf, cent_buf, hca_buf, start: int, p: SAParams,
                         backend=None):
    """Local: indexer + three-stream attention of this segment's queries (absolute positions
    start .. start+Ls-1) over the prefix rows of the whole-sequence tables.  The centroid table
    keeps its full length: future blocks score -inf whatever their rows hold, and the table's
    length sets min(top_k, nb) and the filler indices, which then match the single-GPU indexer.
    Filler blocks past the prefix are dropped by the attention; every token they name lies after
    the query, which the reference's causal mask removes as well
    (maba_sparse/layers/sparse_attention.py:117-164)."""
    backend = backend or B200Backend()
    end = start + qhat_local.shape[1]
    idx = backend.index_topk_at(q_idx_local, cent_buf, p.lam, p.top_k, p.block, start)
    nh = end // p.hca_r
    o = backend.sa_attention(qhat_local, c_buf[:, :end], hca_buf[:, :nh] if nh else None, idx, gate_local,
                             p.window, p.sinks, p.block, p.hca_r)
    return o, idx


def segment_bounds(Ls: int, group=None) -> List[int]:
    """Segment boundaries from every rank's segment length (one small all-gather)."""
    n = torch.tensor([Ls], dtype=torch.int64, device="cuda" if dist.get_backend(group) == "nccl" else "cpu")
    sizes = [int(x.item()) for x in _gather(n, group)]
    bounds = [0]
    for k in sizes:
        bounds.append(bounds[-1] + k)
    return bounds


def sp_sa_prefill(qhat_local, c_local, q_idx_local, k_idx_local, gate_local, p: SAParams, group=None,
                  backend=None, bounds: Optional[Sequence[int]] = None):
    """Sequence-split DG-Indexer + MABA-SA prefill of this rank's segment (contiguous
    segments in rank order; their lengths may differ, e.g. ``balanced_segments``; pass
    ``bounds`` when they are known to skip the size exchange).  Rank r receives only the
    latent rows, centroids and pooled rows of ranks < r."""
    B, Ls, dc = c_local.shape
    if Ls % p.block or Ls % p.hca_r:
        raise ValueError(f"segment length {Ls} must be a multiple of block {p.block} and r {p.hca_r}")
    rank = dist.get_rank(group)
    if bounds is None:
        bounds = segment_bounds(Ls, group)
    total, start = bounds[-1], bounds[rank]
    c_buf = torch.empty(B, total, dc, dtype=c_local.dtype, device=c_local.device)
    cent_buf = torch.zeros(B, total // p.block, k_idx_local.shape[2], dtype=k_idx_local.dtype,
                           device=k_idx_local.device)
    hca_buf = torch.empty(B, total // p.hca_r, dc, dtype=c_local.dtype, device=c_local.device)
    c_buf[:, start:start + Ls] = c_local
    sa_segment_tables(c_buf, cent_buf, hca_buf, k_idx_local, start, p, backend)
    exchange_prefix([c_buf, cent_buf, hca_buf], bounds, [1, p.block, p.hca_r], rank, group)
    return sa_segment_attention(qhat_local, q_idx_local, gate_local, c_buf, cent_buf, hca_buf, start, p, backend)
