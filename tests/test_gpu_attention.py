"""MABA-SA fused latent attention (kernel and layer) vs the CPU oracle and the
reference's golden layer outputs; DGDA layer vs the reference."""
import math

import numpy as np
import pytest
import torch

import maba_v2_architecture_b200 as mb
from helpers import RTOL_BF16, RTOL_FP32, assert_rel, golden, sub
from maba_v2_architecture_b200.config import MabaSparseConfig
from maba_v2_architecture_b200.layers import DGDALayer, MabaSparseAttention
from maba_v2_architecture_b200.workloads import init_module_, sa_inputs
from oracle import attention as OA
from oracle import indexer as OI

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rand_case(B, Lq, Lkv, H, DC, K, block, seed, gate4d=False):
    g = torch.Generator().manual_seed(seed)
    qhat = torch.randn(B, Lq, H, DC, generator=g) * 0.3
    c = torch.randn(B, Lkv, DC, generator=g)
    nb = (Lkv + block - 1) // block
    top = torch.stack([torch.stack([torch.randperm(nb + 2, generator=g)[:K] for _ in range(Lq)]) for _ in range(B)])
    gate = torch.randn(B, H, Lq, 3, generator=g) if gate4d else torch.randn(B, Lq, 3, generator=g)
    return qhat, c, top.long(), gate


@pytest.mark.parametrize("B,Lq,Lkv,H,DC,K,window,block,r,gate4d", [
    (2, 300, 300, 3, 128, 5, 48, 16, 32, False),
    (1, 50, 330, 2, 128, 6, 64, 16, 16, True),     # chunked prefill: queries at the end of a longer cache
    (1, 1, 700, 10, 128, 8, 128, 64, 64, False),   # decode-shaped
    (2, 90, 90, 4, 64, 3, 16, 8, 8, False),         # small d_c, window shorter than the prefix
    (1, 40, 40, 2, 96, 2, 128, 64, 64, False),      # everything inside the window, HCA early path only
])
def test_kernel_vs_oracle(B, Lq, Lkv, H, DC, K, window, block, r, gate4d):
    qhat, c, top, gate = rand_case(B, Lq, Lkv, H, DC, K, block, seed=B * 1000 + Lq, gate4d=gate4d)
    hca = mb.b200_hca_pool(c.to(DEV), r) if Lkv >= r else None
    out = mb.b200_sa_attention(qhat.to(DEV), c.to(DEV), hca, top.to(DEV), gate.to(DEV), window_size=window,
                               n_sinks=4, block_size=block, hca_r=r)
    ref = OA.sa_attention_latent(qhat.numpy(), c.numpy(), top.numpy(), gate.numpy(), window, 4, block, r)
    assert_rel(out, ref, RTOL_FP32, "fp32")
    outb = mb.b200_sa_attention(qhat.to(DEV, torch.bfloat16), c.to(DEV, torch.bfloat16),
                                None if hca is None else hca.to(torch.bfloat16), top.to(DEV),
                                gate.to(DEV, torch.bfloat16), window_size=window, n_sinks=4, block_size=block,
                                hca_r=r)
    assert outb.dtype == torch.bfloat16
    assert_rel(outb, ref, RTOL_BF16, "bf16")


@pytest.mark.parametrize("B,Lq,Lkv,H,K,window,sinks,gate4d,dt", [
    (1, 256, 256, 2, 4, 128, 4, False, torch.bfloat16),    # whole tiles, HCA early rows
    (2, 200, 200, 4, 6, 100, 4, False, torch.bfloat16),    # batch 2, ragged last tile, window % 64 != 0
    (1, 130, 1000, 2, 8, 128, 4, True, torch.bfloat16),    # queries at offset 870 of the cache, per-head gate
    (1, 64, 64, 2, 1, 1, 0, False, torch.bfloat16),        # window 1, no sinks, one selected block
    (1, 300, 300, 2, 32, 4096, 4, False, torch.float16),   # window covering everything, top-32, fp16
    (1, 1024, 1024, 10, 32, 128, 4, False, torch.bfloat16),  # config-2 shape, longer HCA stream
    (1, 128, 40000, 2, 32, 128, 4, False, torch.bfloat16),  # unions of ~600 blocks: running-maximum kernel
])
def test_tc_kernel_vs_oracle(B, Lq, Lkv, H, K, window, sinks, gate4d, dt):
    """The tcgen05 path (block 64, d_c 128, even H): every stream, mask and tile edge vs the oracle."""
    qhat, c, top, gate = rand_case(B, Lq, Lkv, H, 128, K, 64, seed=7 * Lq + K, gate4d=gate4d)
    cd = c.to(DEV, dt)
    hca = mb.b200_hca_pool(cd, 64) if Lkv >= 64 else None
    out = mb.b200_sa_attention(qhat.to(DEV, dt), cd, hca, top.to(DEV), gate.to(DEV, dt), window_size=window,
                               n_sinks=sinks, block_size=64, hca_r=64)
    torch.cuda.synchronize()
    assert mb._native.device_error() == 0
    ref = OA.sa_attention_latent(qhat.to(dt).float().numpy(), c.to(dt).float().numpy(), top.numpy(),
                                 gate.to(dt).float().numpy(), window, sinks, 64, 64)
    assert out.dtype == dt
    assert_rel(out, ref, RTOL_BF16, str(dt))


@pytest.mark.parametrize("scale_rows", [None, "all", "some"])
def test_tc_bound_references_and_exact_redo(scale_rows):
    """bf16 prefill takes bound-referenced exponentials; query rows whose score range
    is too wide for them (large |q| * |k|) send their tile to the running-maximum
    pass.  Both must match the oracle."""
    B, Lq, Lkv, H, K, window = 1, 512, 512, 4, 8, 128
    qhat, c, top, gate = rand_case(B, Lq, Lkv, H, 128, K, 64, seed=99)
    if scale_rows == "all":
        qhat = qhat * 60.0
    elif scale_rows == "some":
        qhat[:, 200:230] *= 80.0  # one 64-query tile misses the range condition
    dt = torch.bfloat16
    cd = c.to(DEV, dt)
    hca = mb.b200_hca_pool(cd, 64)
    out = mb.b200_sa_attention(qhat.to(DEV, dt), cd, hca, top.to(DEV), gate.to(DEV, dt), window_size=window,
                               n_sinks=4, block_size=64, hca_r=64)
    torch.cuda.synchronize()
    assert mb._native.device_error() == 0
    ref = OA.sa_attention_latent(qhat.to(dt).float().numpy(), c.to(dt).float().numpy(), top.numpy(),
                                 gate.to(dt).float().numpy(), window, 4, 64, 64)
    assert bool(torch.isfinite(out.float()).all())
    assert_rel(out, ref, RTOL_BF16, str(scale_rows))


def load_sa(name):
    g = sub(golden("sa_layer"), f"{name}.")
    window, block, top_k, r = (int(v) for v in g["kw"])
    cfg = MabaSparseConfig(dim=64, n_heads=2, d_head=32, kernel_size=4, chunk_size=16, eps=1e-6, window_size=window,
                           block_size=block, top_k=top_k, hca_pool_size=r, dist_lambda=float(g["lam"]))
    layer = MabaSparseAttention(cfg).eval().to(DEV)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in sub(g, "w.").items()})
    return g, layer


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_layer_vs_reference(name):
    g, layer = load_sa(name)
    with torch.no_grad():
        y, c_full = layer(torch.from_numpy(g["x"]).to(DEV))
    assert_rel(c_full, g["c_full"], 1e-5, "c_full")
    assert_rel(y, g["y"], RTOL_FP32, "y")


def test_layer_decode_equals_reference_steps():
    g = sub(golden("sa_layer"), "dec.")
    window, block, top_k, r = (int(v) for v in g["kw"])
    cfg = MabaSparseConfig(dim=64, n_heads=2, d_head=32, kernel_size=4, chunk_size=16, eps=1e-6, window_size=window,
                           block_size=block, top_k=top_k, hca_pool_size=r)
    layer = MabaSparseAttention(cfg).eval().to(DEV)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in sub(g, "w.").items()})
    x = torch.from_numpy(g["x"]).to(DEV)
    with torch.no_grad():
        y_pre, past = layer(x[:, :40])
        ys = []
        for t in range(40, 60):
            yt, past = layer(x[:, t:t + 1], past_c_kv=past)
            ys.append(yt)
        layer.reset_cache()
        y_full, _ = layer(x)
    assert_rel(y_pre, g["y_pre"], RTOL_FP32, "prefill")
    assert_rel(torch.cat(ys, 1), g["y_steps"], RTOL_FP32, "decode steps")
    assert_rel(y_full, g["y_full"], RTOL_FP32, "full")
    assert_rel(torch.cat(ys, 1), y_full[:, 40:], 1e-4, "decode == prefill")


def test_layer_101m_shape():
    g = sub(golden("sa_layer"), "big.")
    layer = init_module_(MabaSparseAttention(MabaSparseConfig(dim=640, n_heads=10, d_head=64, dist_lambda=0.1)),
                         seed=123).eval().to(DEV)
    x = torch.randn(1, 2304, 640, generator=torch.Generator().manual_seed(124)).to(DEV)
    with torch.no_grad():
        y, _ = layer(x)
    rows = torch.as_tensor(g["rows"], device=DEV)
    assert_rel(y[0, rows], g["y_rows"], RTOL_FP32, "y rows")
    assert abs(y.double().sum().item() - float(g["y_sum"])) <= 1e-4 * float(g["y_abs"])


def test_config2_attention_sampled_rows():
    """Config 2 (T=65,536, bf16) through indexer + fused attention; rows checked against the oracle."""
    wl = sa_inputs()
    dt = torch.bfloat16
    c_kv = wl.c_kv.to(DEV, dt)
    c = mb.b200_compute_centroids(wl.k_idx.to(DEV, dt))
    idx = mb.b200_index_topk(wl.q_idx.to(DEV, dt), c, lambda_dist=0.1, top_k=32)
    qhat = mb.ops.absorb_queries(wl.q.to(DEV, dt), wl.w_uk.to(DEV), 10, 0.125)
    hca = mb.b200_hca_pool(c_kv, 64)
    out = mb.b200_sa_attention(qhat, c_kv, hca, idx, wl.gate.to(DEV, dt))
    assert out.shape == (1, 65536, 10, 128) and bool(torch.isfinite(out.float()).all())
    rows = np.array([0, 5, 62, 63, 64, 127, 128, 2047, 2048, 4095, 33333, 65535])
    ref = OA.sa_attention_latent(qhat.float().cpu().numpy(), c_kv.float().cpu().numpy(), idx.cpu().numpy(),
                                 wl.gate.to(dt).float().numpy(), 128, 4, 64, 64, rows=rows)
    assert_rel(out[:, torch.as_tensor(rows, device=DEV)], ref, RTOL_BF16, "rows")


def test_dgda_layer_vs_reference():
    g = golden("dgda_layer")
    cfg = MabaSparseConfig(dim=64, n_heads=2, d_head=32, kernel_size=4, chunk_size=16, eps=1e-6)
    layer = DGDALayer(cfg).eval().to(DEV)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in sub(g, "w.").items()})
    x = torch.from_numpy(g["x"]).to(DEV)
    with torch.no_grad():
        y, S, cs = layer(x[:, :40])
        ys = []
        for t in range(40, 50):
            yt, S, cs = layer.step(x[:, t:t + 1], state=S, conv_state=cs)
            ys.append(yt)
        yf, Sf, _ = layer(x)
    assert_rel(y, g["y40"], RTOL_FP32, "prefill")
    assert_rel(torch.cat(ys, 1), g["y_steps"], RTOL_FP32, "steps")
    assert_rel(S, g["S_steps"], RTOL_FP32, "state after steps")
    assert_rel(yf, g["y_full"], RTOL_FP32, "full")
    assert_rel(Sf, g["S_full"], RTOL_FP32, "full state")


def test_bounded_wait_runs_out_and_reports():
    """A pipeline wait that can never complete gives up after its limit: the kernel
    returns, the device error word reads 2 (then clears), and the context stays usable."""
    from maba_v2_architecture_b200 import _native as N
    assert N.device_error() == 0
    stream = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().maba_selftest_wait_timeout(2_000_000, stream), "selftest")  # ~1 ms at 1.9 GHz
    torch.cuda.synchronize()
    assert N.device_error() == 2
    assert N.device_error() == 0
    x = torch.ones(4, device=DEV)
    assert float((x * 2).sum()) == 8.0  # the context still works


@pytest.mark.parametrize("dt,rtol", [(torch.float32, RTOL_FP32), (torch.bfloat16, RTOL_BF16)])
def test_no_hca_ablation_vs_oracle(dt, rtol):
    """ablation_mode='no_hca' zeroes the HCA stream and keeps the three-way gate
    (maba_sparse/layers/sparse_attention.py:268-271): g0*o_local + g1*o_sparse."""
    cfg = MabaSparseConfig(dim=64, n_heads=2, d_head=32, window_size=48, block_size=16, top_k=4, hca_pool_size=16,
                           dist_lambda=0.3)
    layer = init_module_(MabaSparseAttention(cfg, ablation_mode="no_hca"), seed=41).eval().to(DEV, dt)
    x = torch.randn(1, 150, 64, generator=torch.Generator().manual_seed(42)).to(DEV, dt)
    with torch.no_grad():
        c = layer.kv_down_proj(x)
        idx, _ = layer.indexer(x)
        q = layer.q_proj(x).view(1, 150, 2, 32)
        qhat = mb.ops.absorb_queries(q, layer.k_up_proj.weight, 2, layer.scale)
        out = layer.latent_attention(x, c, idx)
        gate = layer.stream_gate(x)
    st = OA.sa_streams(qhat.float().cpu().numpy(), c.float().cpu().numpy(), idx.cpu().numpy(), 48, 4, 16, 16)
    g = OA.gate_softmax(gate.float().cpu().numpy())[:, :, None, :]
    ref = g[..., 0:1] * st[0] + g[..., 1:2] * st[1]
    assert_rel(out, ref, rtol, "no_hca latent output")
