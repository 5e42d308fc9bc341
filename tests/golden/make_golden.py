"""Generates the golden fixtures of tests/golden/ by running the REFERENCE
implementation (maba_sparse, pure Python/PyTorch) on seeded inputs.

Run in a checkout where the reference project is importable:

    MABA_REFERENCE=/path/to/maba-v2-architecture python tests/golden/make_golden.py

The fixtures pin the CPU oracle (oracle/) and the CUDA path: they hold the
reference's own outputs (and, for small cases, the inputs and weights; large
inputs are regenerated from their seeds by maba_v2_architecture_b200.workloads).
Nothing at test time imports the reference.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
REF = os.environ.get("MABA_REFERENCE")
if not REF:
    raise SystemExit("set MABA_REFERENCE to the reference checkout")
sys.path.insert(0, REF)

from maba_sparse.config import MabaSparseConfig  # noqa: E402
from maba_sparse.kernels.common import (  # noqa: E402
    ref_compute_centroids, ref_dgda_prefill, ref_dgda_step, ref_index_topk, ref_stream_superposition)
from maba_sparse.kernels.cpu_dgda import cpu_dgda_prefill  # noqa: E402
from maba_sparse.kernels.cpu_indexer import (  # noqa: E402
    cpu_compute_centroids, cpu_index_topk, cpu_stream_superposition)
from maba_sparse.layers.dgda import DGDALayer  # noqa: E402
from maba_sparse.layers.indexer import DGIndexer  # noqa: E402
from maba_sparse.layers.sparse_attention import MabaSparseAttention  # noqa: E402
from maba_sparse.model import MabaSparseForCausalLM  # noqa: E402

from maba_v2_architecture_b200.workloads import dgda_inputs, init_module_, sa_inputs  # noqa: E402

torch.set_num_threads(min(8, os.cpu_count() or 8))


def npy(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def save(name, **arrays):
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **{k: npy(v) for k, v in arrays.items()})
    print(f"{path.name}: {path.stat().st_size / 1024:.0f} KiB")


def state_arrays(module, prefix="w."):
    return {prefix + k: v for k, v in module.state_dict().items()}


# ---------------------------------------------------------------------------
def gen_dgda():
    out = {}
    # small mixed case with an initial state (reference sequential recurrence)
    torch.manual_seed(11)
    B, H, L, dk, dv = 2, 3, 37, 16, 8
    q = torch.randn(B, H, L, dk)
    k = F.normalize(torch.randn(B, H, L, dk), dim=-1)
    v = torch.randn(B, H, L, dv)
    alpha = torch.rand(B, H, L, dk) * 0.9 + 0.05
    b = torch.rand(B, H, L, dk)
    w = torch.rand(B, H, L, dv)
    s0 = torch.randn(B, H, dk, dv)
    o, S = ref_dgda_prefill(q, k, v, alpha, b, w, initial_state=s0)
    out.update({"small.q": q, "small.k": k, "small.v": v, "small.alpha": alpha, "small.b": b, "small.w": w,
                "small.s0": s0, "small.o": o, "small.S": S})
    # lengths around chunk boundaries, log_alpha only
    for L in (1, 7, 17, 63, 65, 129):
        torch.manual_seed(100 + L)
        q = torch.randn(1, 2, L, 32)
        k = F.normalize(torch.randn(1, 2, L, 32), dim=-1)
        v = torch.randn(1, 2, L, 32)
        la = -F.softplus(torch.randn(1, 2, L, 32) + 1.0)
        b = torch.rand(1, 2, L, 32)
        w = torch.rand(1, 2, L, 32)
        o, S = ref_dgda_prefill(q, k, v, None, b, w, log_alpha=la)
        p = f"len{L}."
        out.update({p + "q": q, p + "k": k, p + "v": v, p + "la": la, p + "b": b, p + "w": w, p + "o": o, p + "S": S})
    # extreme decays and gates (cpu_dgda tests: alpha in {0,1e-7,1e-20,1e-35,1}, b/w in {0,1})
    torch.manual_seed(101)
    B, H, L, d = 2, 2, 48, 16
    q = torch.randn(B, H, L, d)
    k = F.normalize(torch.randn(B, H, L, d), dim=-1)
    v = torch.randn(B, H, L, d)
    b = torch.rand(B, H, L, d)
    w = torch.rand(B, H, L, d)
    s0 = torch.randn(B, H, d, d)
    out.update({"ext.q": q, "ext.k": k, "ext.v": v, "ext.b": b, "ext.w": w, "ext.s0": s0})
    for i, a in enumerate((0.0, 1e-7, 1e-20, 1e-35, 1.0)):
        o, S = ref_dgda_prefill(q, k, v, torch.full_like(q, a), b, w, initial_state=s0)
        out[f"ext.alpha{i}.o"], out[f"ext.alpha{i}.S"] = o, S
    out["ext.alphas"] = torch.tensor([0.0, 1e-7, 1e-20, 1e-35, 1.0], dtype=torch.float64)
    alpha = torch.rand(B, H, L, d) * 0.9 + 0.05
    out["ext.alpha_mid"] = alpha
    for name, bv, wv in (("b0", 0.0, None), ("b1", 1.0, None), ("w0", None, 0.0), ("w1", None, 1.0)):
        bb = torch.full_like(b, bv) if bv is not None else b
        ww = torch.full_like(w, wv) if wv is not None else w
        o, S = ref_dgda_prefill(q, k, v, alpha, bb, ww, initial_state=s0)
        out[f"ext.{name}.o"], out[f"ext.{name}.S"] = o, S
    # +-100 inputs through a layer's features (tests/test_dgda_stress.py:168-190 style)
    torch.manual_seed(789)
    q = torch.randn(1, 2, 32, 32) * 100
    k = F.normalize(torch.randn(1, 2, 32, 32), dim=-1)
    v = torch.randn(1, 2, 32, 32) * 100
    b = torch.rand(1, 2, 32, 32)
    w = torch.rand(1, 2, 32, 32)
    la = -F.softplus(torch.randn(1, 2, 32, 32) * 5)
    o, S = ref_dgda_prefill(q, k, v, None, b, w, log_alpha=la)
    out.update({"stress.q": q, "stress.k": k, "stress.v": v, "stress.b": b, "stress.w": w, "stress.la": la,
                "stress.o": o, "stress.S": S})
    # config 1 (both gating variants): outputs only, inputs regenerate from the seed
    for variant, pc in (("cfg1", False), ("cfg1pc", True)):
        x = dgda_inputs(seed=0 if not pc else 10, per_channel=pc)
        o, S = ref_dgda_prefill(x["q"], x["k"], x["v"], x["alpha"], x["b"], x["w"], log_alpha=x["log_alpha"])
        out[f"{variant}.o_sub"] = o[:, :, ::8]
        out[f"{variant}.S"] = S
        out[f"{variant}.o_sum"] = o.double().sum()
        out[f"{variant}.o_abs"] = o.double().abs().sum()
        oc, Sc = cpu_dgda_prefill(x["q"], x["k"], x["v"], x["alpha"], x["b"], x["w"], chunk_size=64,
                                  log_alpha=x["log_alpha"], inversion_method="exact")
        out[f"{variant}.cpu64_maxdiff"] = (oc - o).abs().max()
    save("dgda_prefill", **out)


def gen_step():
    out = {}
    torch.manual_seed(42)
    B, H, dk, dv = 2, 4, 64, 64
    q = torch.randn(B, H, dk)
    k = F.normalize(torch.randn(B, H, dk), dim=-1)
    v = torch.randn(B, H, dv)
    a = torch.rand(B, H, dk) * 0.9 + 0.05
    b = torch.rand(B, H, dk)
    w = torch.rand(B, H, dv)
    s = torch.randn(B, H, dk, dv)
    o, S = ref_dgda_step(q, k, v, a, b, w, state=s)
    out.update({"q": q, "k": k, "v": v, "alpha": a, "b": b, "w": w, "state": s, "o": o, "S": S})
    # prefill + step continuity (tests/test_kernel_e2e.py:836-866)
    torch.manual_seed(777)
    B, H, dk, dv, L1, L2 = 1, 2, 16, 16, 8, 4
    q = torch.randn(B, H, L1 + L2, dk)
    k = F.normalize(torch.randn(B, H, L1 + L2, dk), p=2, dim=-1)
    v = torch.randn(B, H, L1 + L2, dv)
    alpha = torch.full((B, H, L1 + L2, dk), 0.9)
    b = torch.full((B, H, L1 + L2, dk), 0.5)
    w = torch.full((B, H, L1 + L2, dv), 0.5)
    fo, fs = ref_dgda_prefill(q, k, v, alpha, b, w)
    out.update({"cont.q": q, "cont.k": k, "cont.v": v, "cont.alpha": alpha, "cont.b": b, "cont.w": w,
                "cont.o": fo, "cont.S": fs})
    save("dgda_step", **out)


def gen_indexer():
    out = {}
    # needle preservation (tests/test_triton_indexer.py:147-158)
    k = torch.full((1, 256, 64), 0.01)
    k[0, 70, :] = 10.0
    out["needle.k"], out["needle.c"] = k, cpu_compute_centroids(k, block_size=64)
    # tail padding (tests/test_triton_indexer.py:160-171)
    k = torch.full((1, 100, 64), -2.0)
    out["tail.k"], out["tail.c"] = k, cpu_compute_centroids(k, block_size=64)
    # hybrid formula with block 4 (tests/test_kernel_e2e.py:427-437)
    k = torch.tensor([[[1.0, 2.0], [3.0, 4.0], [5.0, 6.0], [7.0, 8.0]]])
    out["hyb.k"], out["hyb.c"] = k, cpu_compute_centroids(k, block_size=4)
    # misaligned lengths, odd batch (tests/test_indexer_stability.py:249-316)
    for L in (1, 63, 65, 129, 257):
        torch.manual_seed(3000 + L)
        k = torch.randn(3, L, 64)
        out[f"mis{L}.k"], out[f"mis{L}.c"], out[f"mis{L}.cref"] = k, cpu_compute_centroids(k, 64), ref_compute_centroids(k, 64)
    # bf16 input (values stored as fp32)
    torch.manual_seed(5)
    kb = torch.randn(2, 300, 64).to(torch.bfloat16)
    out["bf16.k"], out["bf16.c"] = kb.float(), cpu_compute_centroids(kb, 64).float()

    # top-k parity cases (tests/test_triton_indexer.py:173-207) plus larger ones
    cases = [(1, 64, 1, 0.5), (2, 128, 2, 0.5), (3, 256, 4, 0.5), (2, 512, 8, 1.0), (1, 100, 2, 0.25),
             (2, 65, 2, 0.0), (2, 16, 2, 0.5), (1, 512, 32, 0.5), (1, 4096, 32, 0.1), (2, 2048, 32, 0.5),
             (1, 1536, 48, 0.3)]
    for ci, (B, L, top_k, lam) in enumerate(cases):
        torch.manual_seed(400 + ci)
        q = torch.randn(B, L, 64)
        k = torch.randn(B, L, 64)
        c = cpu_compute_centroids(k, 64)
        idx, sc = cpu_index_topk(q, c, lambda_dist=lam, top_k=top_k, block_size=64, return_scores=True)
        ridx = ref_index_topk(q, c, lambda_dist=lam, top_k=top_k, block_size=64)
        p = f"tk{ci}."
        # inputs regenerate from torch.manual_seed(400 + ci): q = randn(B,L,64), k = randn(B,L,64)
        out.update({p + "c": c, p + "idx": idx, p + "ref_idx": ridx, p + "meta": torch.tensor([B, L, top_k, lam])})
        if L <= 512:
            out[p + "scores"] = sc
    # monotone penalty (tests/test_triton_indexer.py:247-255)
    q = torch.ones(1, 256, 64) / 8.0
    c = torch.ones(1, 4, 64) / 8.0
    out["mono.q"], out["mono.c"] = q, c
    out["mono.idx"] = cpu_index_topk(q, c, lambda_dist=1.0, top_k=4, block_size=64)
    # needle across long contexts (tests/test_indexer_stability.py:185-223)
    for L in (1024, 4096):
        torch.manual_seed(42)
        k = torch.randn(1, L, 64)
        k[:, 5 * 64 + 10, 0] = 25.0
        q = torch.randn(1, L, 64) * 0.1
        q[:, -1, 0] = 5.0
        c = cpu_compute_centroids(k, 64)
        out[f"nd{L}.idx_last"] = cpu_index_topk(q, c, lambda_dist=0.5, top_k=32, block_size=64)[0, -1]
    # decode-time inline scoring of DGIndexer (maba_sparse/layers/indexer.py:101-112)
    torch.manual_seed(21)
    ix = DGIndexer(dim=64, d_idx=32, block_size=16, top_k=8, dist_lambda=0.5).eval()
    x = torch.randn(1, 70, 64)
    with torch.no_grad():
        ix(x[:, :50])
        dec = []
        for t in range(50, 70):
            idx, c, sc = ix(x[:, t:t + 1], return_scores=True)
            dec.append((idx, c, sc))
    out["dec.x"] = x
    out.update(state_arrays(ix, "dec.w."))
    for j, (idx, c, sc) in enumerate(dec):
        out[f"dec.{j}.idx"], out[f"dec.{j}.c"], out[f"dec.{j}.scores"] = idx, c, sc
    # config-2 scale: T=65536, nb=1024, lambda=0.1, sampled rows
    wl = sa_inputs()
    c = cpu_compute_centroids(wl.k_idx, 64)
    idx, sc = cpu_index_topk(wl.q_idx, c, lambda_dist=0.1, top_k=32, block_size=64, return_scores=True)
    g = torch.Generator().manual_seed(7)
    rows = torch.cat([torch.randint(0, 65536, (509,), generator=g), torch.tensor([63, 64, wl.probe])])
    out["cfg2.rows"] = rows
    out["cfg2.idx"] = idx[0, rows]
    out["cfg2.scores16"] = sc[0, rows[:16]]
    out["cfg2.needle"] = torch.tensor(wl.needle_block)
    out["cfg2.needle_rank"] = torch.tensor(int((idx[0, wl.probe] == wl.needle_block).nonzero()[0, 0])
                                           if (idx[0, wl.probe] == wl.needle_block).any() else -1)
    out["cfg2.c_sum"] = c.double().sum()
    save("indexer", **out)

    # superposition
    out = {}
    torch.manual_seed(9)
    ol, os_, oh = torch.randn(2, 3, 17, 16), torch.randn(2, 3, 17, 16), torch.randn(2, 3, 17, 16)
    g3, g4 = torch.randn(2, 17, 3), torch.randn(2, 3, 17, 3)
    gw = F.softmax(torch.randn(2, 17, 3), dim=-1)
    out.update({"ol": ol, "os": os_, "oh": oh, "g3": g3, "g4": g4, "gw": gw,
                "o3": cpu_stream_superposition(ol, os_, oh, gate_logits=g3),
                "o4": cpu_stream_superposition(ol, os_, oh, gate_logits=g4),
                "ow": ref_stream_superposition(ol, os_, oh, gate_weights=gw)})
    save("superposition", **out)


def record_sa(layer, x, past_c_kv=None):
    """Runs the reference layer and records its per-stream intermediates."""
    rec = {}
    orig_l, orig_s, orig_h = layer._compute_local_attention, layer._compute_sparse_attention, layer._compute_hca_attention

    def l_(q, k, v, L):
        rec["q"] = q
        o = orig_l(q, k, v, L)
        rec["ol"] = o
        return o

    def s_(q, k, v, idx, L):
        rec["idx"] = idx
        o = orig_s(q, k, v, idx, L)
        rec["os"] = o
        return o

    def h_(q, c, L):
        o = orig_h(q, c, L)
        rec["oh"] = o
        return o

    layer._compute_local_attention, layer._compute_sparse_attention, layer._compute_hca_attention = l_, s_, h_
    try:
        with torch.no_grad():
            y, c_full = layer(x, past_c_kv=past_c_kv)
            rec["gate"] = layer.stream_gate(x)
    finally:
        del layer._compute_local_attention, layer._compute_sparse_attention, layer._compute_hca_attention
    rec["y"], rec["c_full"] = y, c_full
    return rec


def gen_sa():
    out = {}
    # small layers; the config's fields win over constructor kwargs in the reference
    cases = [("a", dict(), 200, 31),
             ("b", dict(window_size=32, block_size=16, top_k=4, hca_pool_size=16), 150, 32),
             ("c", dict(window_size=48, block_size=16, top_k=8, hca_pool_size=32, dist_lambda=0.2), 300, 33)]
    for name, kw, L, seed in cases:
        cfg = MabaSparseConfig(dim=64, n_heads=2, d_head=32, kernel_size=4, chunk_size=16, eps=1e-6, **kw)
        torch.manual_seed(seed)
        layer = MabaSparseAttention(cfg).eval()
        x = torch.randn(1, L, 64)
        rec = record_sa(layer, x)
        p = f"{name}."
        out.update(state_arrays(layer, p + "w."))
        out[p + "x"] = x
        out[p + "kw"] = np.array([layer.window_size, layer.block_size, layer.top_k, layer.hca_pool_size])
        out[p + "lam"] = np.array(layer.dist_lambda)
        for key in ("q", "ol", "os", "oh", "idx", "gate", "y", "c_full"):
            out[p + key] = rec[key]
    # decode == prefill (tests/test_sparse_attention.py:256-286) with the decode outputs per step
    small = MabaSparseConfig(dim=64, n_heads=2, d_head=32, kernel_size=4, chunk_size=16, eps=1e-6, window_size=32,
                             block_size=16, top_k=4, hca_pool_size=16)
    torch.manual_seed(42)
    layer = MabaSparseAttention(small).eval()
    x = torch.randn(1, 60, 64)
    with torch.no_grad():
        y_pre, _ = layer(x[:, :40])
        past = layer.kv_down_proj(x[:, :40])
        ys = []
        for t in range(40, 60):
            yt, past = layer(x[:, t:t + 1], past_c_kv=past)
            ys.append(yt)
        layer.reset_cache()
        y_full, _ = layer(x)
    out.update(state_arrays(layer, "dec.w."))
    out["dec.kw"] = np.array([layer.window_size, layer.block_size, layer.top_k, layer.hca_pool_size])
    out["dec.x"], out["dec.y_pre"], out["dec.y_steps"], out["dec.y_full"] = x, y_pre, torch.cat(ys, 1), y_full
    # 101M-shaped layer (dim 640, 10 heads x 64, d_c 128, window 128, block 64, top-32, lambda 0.1), seeded weights
    cfg = MabaSparseConfig(dim=640, n_heads=10, d_head=64, dist_lambda=0.1)
    layer = init_module_(MabaSparseAttention(cfg), seed=123).eval()
    x = torch.randn(1, 2304, 640, generator=torch.Generator().manual_seed(124))
    rec = record_sa(layer, x)
    rows = torch.tensor([0, 1, 5, 62, 63, 64, 127, 128, 129, 700, 1500, 2047, 2048, 2200, 2303])
    out["big.rows"] = rows
    out["big.y_rows"] = rec["y"][0, rows]
    out["big.idx_rows"] = rec["idx"][0, rows]
    for key in ("ol", "os", "oh"):
        out[f"big.{key}_rows"] = rec[key][0, :, rows]
    out["big.y_sum"] = rec["y"].double().sum()
    out["big.y_abs"] = rec["y"].double().abs().sum()
    save("sa_layer", **out)


def gen_dgda_layer():
    out = {}
    small = MabaSparseConfig(dim=64, n_heads=2, d_head=32, kernel_size=4, chunk_size=16, eps=1e-6)
    torch.manual_seed(42)
    layer = DGDALayer(small).eval()
    x = torch.randn(2, 50, 64)
    with torch.no_grad():
        y, S, cs = layer(x[:, :40])
        ys = []
        for t in range(40, 50):
            yt, S, cs = layer.step(x[:, t:t + 1], state=S, conv_state=cs)
            ys.append(yt)
        yf, Sf, _ = layer(x)
    out.update(state_arrays(layer, "w."))
    out.update({"x": x, "y40": y, "y_steps": torch.cat(ys, 1), "S_steps": S, "y_full": yf, "S_full": Sf})
    save("dgda_layer", **out)


def gen_model():
    out = {}
    cfg = MabaSparseConfig(dim=64, n_heads=2, d_head=32, n_layers=4, vocab_size=512, d_emb=32,
                           intermediate_size=128, window_size=32, block_size=16, top_k=4, hca_pool_size=16,
                           dist_lambda=0.5)
    torch.manual_seed(7)
    model = MabaSparseForCausalLM(cfg).eval()
    ids = torch.randint(0, 512, (1, 90), generator=torch.Generator().manual_seed(8))
    with torch.no_grad():
        o = model(ids)
        logits = o.logits
        ps = o.past_states
        steps = []
        nxt = torch.randint(0, 512, (1, 6), generator=torch.Generator().manual_seed(9))
        for t in range(6):
            lg, ps = model.step(nxt[:, t:t + 1], past_states=ps)
            steps.append(lg)
    out.update(state_arrays(model, "w."))
    out.update({"ids": ids, "logits": logits, "next_ids": nxt, "step_logits": torch.cat(steps, 1),
                "cfg": np.array([64, 2, 32, 4, 512, 32, 128, 32, 16, 4, 16])})
    save("model", **out)


if __name__ == "__main__":
    which = sys.argv[1:] or ["dgda", "step", "indexer", "sa", "dgda_layer", "model"]
    for w in which:
        {"dgda": gen_dgda, "step": gen_step, "indexer": gen_indexer, "sa": gen_sa, "dgda_layer": gen_dgda_layer,
         "model": gen_model}[w]()
