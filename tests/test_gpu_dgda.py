"""DGDA prefill / step kernels vs the CPU oracle and the reference's golden outputs."""
import numpy as np
import pytest
import torch

import maba_v2_architecture_b200 as mb
from helpers import RTOL_BF16, RTOL_FP16, RTOL_FP32, assert_rel, golden, sub
from maba_v2_architecture_b200.workloads import dgda_inputs
from oracle import dgda as OD

pytestmark = pytest.mark.gpu
DEV = "cuda"


def cu(x, dtype=torch.float32):
    return None if x is None else torch.as_tensor(np.asarray(x)).to(DEV, dtype)


def run_prefill(d, dtype=torch.float32, **kw):
    o, S = mb.b200_dgda_prefill(cu(d["q"], dtype), cu(d["k"], dtype), cu(d["v"], dtype), alpha=cu(d.get("alpha"), dtype),
                                b=cu(d["b"], dtype), w=cu(d["w"], dtype), initial_state=cu(d.get("s0"), dtype),
                                log_alpha=cu(d.get("la"), dtype), **kw)
    torch.cuda.synchronize()
    return o, S


def test_small_with_state():
    g = sub(golden("dgda_prefill"), "small.")
    o, S = run_prefill(g)
    assert o.shape == g["o"].shape and o.dtype == torch.float32 and o.is_contiguous()
    assert_rel(o, g["o"], RTOL_FP32, "o")
    assert_rel(S, g["S"], RTOL_FP32, "S")


@pytest.mark.parametrize("L", [1, 7, 17, 63, 65, 129])
def test_lengths_log_alpha_only(L):
    g = sub(golden("dgda_prefill"), f"len{L}.")
    o, S = run_prefill(g)
    assert_rel(o, g["o"], RTOL_FP32, "o")
    assert_rel(S, g["S"], RTOL_FP32, "S")


@pytest.mark.parametrize("i", range(5))
def test_extreme_decay(i):
    g = sub(golden("dgda_prefill"), "ext.")
    d = dict(g)
    d["alpha"] = np.full_like(g["q"], g["alphas"][i])
    o, S = run_prefill(d)
    assert torch.isfinite(o).all() and torch.isfinite(S).all()
    assert_rel(o, g[f"alpha{i}.o"], RTOL_FP32, "o")
    assert_rel(S, g[f"alpha{i}.S"], RTOL_FP32, "S")


@pytest.mark.parametrize("name", ["b0", "b1", "w0", "w1"])
def test_extreme_gates(name):
    g = sub(golden("dgda_prefill"), "ext.")
    d = dict(g)
    d["alpha"] = g["alpha_mid"]
    if name[0] == "b":
        d["b"] = np.full_like(g["b"], float(name[1]))
    else:
        d["w"] = np.full_like(g["w"], float(name[1]))
    o, S = run_prefill(d)
    assert_rel(o, g[f"{name}.o"], RTOL_FP32, "o")
    assert_rel(S, g[f"{name}.S"], RTOL_FP32, "S")


def test_stress_inputs():
    g = sub(golden("dgda_prefill"), "stress.")
    o, S = run_prefill(g)
    assert_rel(o, g["o"], RTOL_FP32, "o")
    assert_rel(S, g["S"], RTOL_FP32, "S")


@pytest.mark.parametrize("variant", ["cfg1", "cfg1pc"])
def test_config1_full(variant):
    """Config 1 (B=2, T=512, H=10, 64x64, fp32) against the sequential oracle and the reference."""
    x = dgda_inputs(seed=0 if variant == "cfg1" else 10, per_channel=variant == "cfg1pc")
    g = sub(golden("dgda_prefill"), f"{variant}.")
    o, S = mb.b200_dgda_prefill(x["q"].to(DEV), x["k"].to(DEV), x["v"].to(DEV), x["alpha"].to(DEV), x["b"].to(DEV),
                                x["w"].to(DEV), chunk_size=64, log_alpha=x["log_alpha"].to(DEV))
    ro, rS = OD.dgda_sequential(*(x[k].numpy() for k in ("q", "k", "v", "alpha", "b", "w")))
    assert_rel(o, ro, RTOL_FP32, "o vs oracle")
    assert_rel(S, rS, RTOL_FP32, "S vs oracle")
    assert_rel(o[:, :, ::8], g["o_sub"], RTOL_FP32, "o vs reference")
    assert_rel(S, g["S"], RTOL_FP32, "S vs reference")


@pytest.mark.parametrize("B,H,L", [(1, 2, 4096), (1, 1, 3000), (2, 3, 2500)])
def test_segmented_long_sequence(B, H, L):
    """Few heads, long sequence: the segment-parallel (affine transition) path."""
    x = dgda_inputs(B=B, T=L, H=H, seed=5, per_channel=True)
    s0 = torch.randn(B, H, 64, 64, generator=torch.Generator().manual_seed(6)) * 0.1
    o, S = mb.b200_dgda_prefill(x["q"].to(DEV), x["k"].to(DEV), x["v"].to(DEV), None, x["b"].to(DEV), x["w"].to(DEV),
                                initial_state=s0.to(DEV), log_alpha=x["log_alpha"].to(DEV))
    ro, rS = OD.dgda_sequential(*(x[k].numpy() for k in ("q", "k", "v", "alpha", "b", "w")), initial_state=s0.numpy())
    assert_rel(o, ro, RTOL_FP32, "o")
    assert_rel(S, rS, RTOL_FP32, "S")


def test_token_major_strided_inputs_and_output_layout():
    B, L, H, d = 2, 150, 3, 64
    gen = torch.Generator().manual_seed(3)
    mk = lambda: torch.randn(B, L, H, d, generator=gen)
    q, v = mk(), mk()
    k = torch.nn.functional.normalize(mk(), dim=-1)
    b, w = torch.rand(B, L, H, d, generator=gen), torch.rand(B, L, H, d, generator=gen)
    la = -torch.nn.functional.softplus(mk())
    tv = lambda t: t.to(DEV).transpose(1, 2)  # [B,H,L,d] views, non-contiguous
    o, S = mb.b200_dgda_prefill(tv(q), tv(k), tv(v), None, tv(b), tv(w), log_alpha=tv(la), out_layout="blhd")
    assert not o.is_contiguous() and o.transpose(1, 2).is_contiguous()
    tn = lambda t: t.transpose(1, 2).numpy()
    ro, rS = OD.dgda_sequential(tn(q), tn(k), tn(v), None, tn(b), tn(w), log_alpha=tn(la))
    assert_rel(o, ro, RTOL_FP32, "o")
    assert_rel(S, rS, RTOL_FP32, "S")


@pytest.mark.parametrize("dtype,rtol", [(torch.bfloat16, RTOL_BF16), (torch.float16, RTOL_FP16)])
def test_16bit_inputs(dtype, rtol):
    x = dgda_inputs(B=2, T=300, H=4, seed=8, per_channel=True)
    args = [x[k].to(DEV, dtype) for k in ("q", "k", "v", "alpha", "b", "w")]
    o, S = mb.b200_dgda_prefill(*args)
    assert o.dtype == dtype and S.dtype == dtype
    ref = {k: x[k].to(dtype).float().numpy() for k in x}
    ro, rS = OD.dgda_sequential(ref["q"], ref["k"], ref["v"], ref["alpha"], ref["b"], ref["w"])
    assert_rel(o, ro, rtol, "o")
    assert_rel(S, rS, rtol, "S")
    o2, S2 = mb.b200_dgda_prefill(*args, state_dtype=torch.float32)
    assert S2.dtype == torch.float32
    assert_rel(S2, rS, rtol, "fp32 state")


def test_fp64():
    g = sub(golden("dgda_prefill"), "small.")
    o, S = run_prefill(g, torch.float64)
    assert o.dtype == torch.float64
    ro, rS = OD.dgda_sequential(g["q"], g["k"], g["v"], g["alpha"], g["b"], g["w"], initial_state=g["s0"])
    assert_rel(o, ro, 1e-10, "o")
    assert_rel(S, rS, 1e-10, "S")


def test_chaining_through_initial_state():
    x = {k: v.to(DEV) for k, v in dgda_inputs(B=1, T=700, H=2, seed=9, per_channel=True).items()}
    cut = 333
    part = lambda s, e: [x[k][:, :, s:e] for k in ("q", "k", "v", "alpha", "b", "w")]
    o_full, S_full = mb.b200_dgda_prefill(*part(0, 700))
    o1, S1 = mb.b200_dgda_prefill(*part(0, cut))
    o2, S2 = mb.b200_dgda_prefill(*part(cut, 700), initial_state=S1)
    assert_rel(torch.cat([o1, o2], 2), o_full, RTOL_FP32, "o")
    assert_rel(S2, S_full, RTOL_FP32, "S")


def test_empty_sequence():
    z = torch.zeros(1, 2, 0, 16, device=DEV)
    s0 = torch.randn(1, 2, 16, 16, device=DEV)
    o, S = mb.b200_dgda_prefill(z, z, z, log_alpha=z, b=z, w=z, initial_state=s0)
    assert o.shape == (1, 2, 0, 16)
    torch.testing.assert_close(S, s0)


def test_step_vs_reference():
    g = golden("dgda_step")
    o, S = mb.b200_dgda_step(*(cu(g[k]) for k in ("q", "k", "v", "alpha", "b", "w")), state=cu(g["state"]))
    assert_rel(o, g["o"], 1e-5, "o")
    assert_rel(S, g["S"], 1e-5, "S")
    # 4-D [B,H,1,d] inputs
    o4, S4 = mb.b200_dgda_step(*(cu(g[k])[:, :, None] for k in ("q", "k", "v", "alpha", "b", "w")),
                               state=cu(g["state"]))
    assert o4.shape == (2, 4, 64)
    torch.testing.assert_close(o4, o)


def test_step_alpha_priority_and_log_alpha():
    g = golden("dgda_step")
    a = cu(g["alpha"])
    base = [cu(g[k]) for k in ("q", "k", "v")]
    o1, _ = mb.b200_dgda_step(*base, alpha=a, b=cu(g["b"]), w=cu(g["w"]), state=cu(g["state"]),
                              log_alpha=torch.zeros_like(a))
    o2, _ = mb.b200_dgda_step(*base, b=cu(g["b"]), w=cu(g["w"]), state=cu(g["state"]), log_alpha=torch.log(a))
    assert_rel(o1, g["o"], 1e-5, "alpha wins")
    assert_rel(o2, g["o"], 1e-5, "log_alpha")


def test_step_unroll_equals_prefill():
    x = {k: v.to(DEV) for k, v in dgda_inputs(B=2, T=40, H=3, seed=12, per_channel=True).items()}
    s0 = torch.randn(2, 3, 64, 64, device=DEV) * 0.1
    o_pre, S_pre = mb.b200_dgda_prefill(*(x[k] for k in ("q", "k", "v", "alpha", "b", "w")), initial_state=s0)
    S = s0
    outs = []
    for t in range(40):
        ot, S = mb.b200_dgda_step(*(x[k][:, :, t] for k in ("q", "k", "v", "alpha", "b", "w")), state=S)
        outs.append(ot)
    assert_rel(torch.stack(outs, 2), o_pre, RTOL_FP32, "o")
    assert_rel(S, S_pre, RTOL_FP32, "S")


def test_prefill_then_steps_continuity():
    c = sub(golden("dgda_step"), "cont.")
    t = {k: cu(c[k]) for k in ("q", "k", "v", "alpha", "b", "w")}
    o1, S = mb.b200_dgda_prefill(*(t[k][:, :, :8] for k in ("q", "k", "v", "alpha", "b", "w")))
    outs = [o1]
    for i in range(8, 12):
        ot, S = mb.b200_dgda_step(*(t[k][:, :, i] for k in ("q", "k", "v", "alpha", "b", "w")), state=S)
        outs.append(ot[:, :, None])
    assert_rel(torch.cat(outs, 2), c["o"], RTOL_FP32, "o")
    assert_rel(S, c["S"], RTOL_FP32, "S")


def test_step_bf16_with_fp32_state():
    x = dgda_inputs(B=4, T=1, H=10, seed=13, per_channel=True)
    s0 = torch.randn(4, 10, 64, 64) * 0.1
    args = [x[k][:, :, 0].to(DEV, torch.bfloat16) for k in ("q", "k", "v", "alpha", "b", "w")]
    o, S = mb.b200_dgda_step(*args, state=s0.to(DEV))
    assert S.dtype == torch.float32 and o.dtype == torch.bfloat16
    ref = [a.float().cpu().numpy() for a in args]
    ro, rS = OD.dgda_step(*ref, state=s0.numpy())
    assert_rel(o, ro, RTOL_BF16, "o")
    assert_rel(S, rS, 1e-5, "S")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,with_state", [(3, 5, True), (1, 1, False), (64, 10, True)])
def test_step_register_path_matches_generic_and_oracle(dtype, B, H, with_state):
    """fp32 state, d = 64, unit-stride rows take the register-resident kernel (one warp per
    head, B*H not a multiple of its 4 warps per CTA); a column-major state view takes the
    generic kernel.  Both against each other and the fp64 oracle."""
    x = dgda_inputs(B=B, T=1, H=H, seed=30 + B, per_channel=True)
    args = [x[k][:, :, 0].to(DEV, dtype) for k in ("q", "k", "v", "alpha", "b", "w")]
    s0 = (torch.randn(B, H, 64, 64) * 0.1) if with_state else None
    st = s0.to(DEV) if with_state else None
    o, S = mb.b200_dgda_step(*args, state=st, state_dtype=torch.float32)
    assert S.dtype == torch.float32
    if with_state:
        st_cm = st.transpose(2, 3).contiguous().transpose(2, 3)  # same values, column-major rows
        o_g, S_g = mb.b200_dgda_step(*args, state=st_cm)
        torch.testing.assert_close(S, S_g.contiguous(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(o.float(), o_g.float(), rtol=2e-2 if dtype != torch.float32 else 1e-5,
                                   atol=1e-5)
    ref = [a.double().cpu().numpy() for a in args]
    ro, rS = OD.dgda_step(*ref, state=s0.double().numpy() if with_state else None)
    assert_rel(S, rS, 1e-5, "S")
    assert_rel(o, ro, RTOL_FP32 if dtype == torch.float32 else RTOL_BF16, "o")


# ---------------------------------------------------------------- tensor-core (16-bit) chunk kernel
@pytest.mark.parametrize("dtype,rtol", [(torch.bfloat16, RTOL_BF16), (torch.float16, RTOL_FP16 * 2)])
@pytest.mark.parametrize("B,H,L", [(1, 2, 4096), (2, 10, 700), (1, 1, 129)])
def test_16bit_tensor_core_path_vs_oracle(dtype, rtol, B, H, L):
    """Token-major strided inputs (vectorised loads), single-pass and segmented launches."""
    x = dgda_inputs(B=B, T=L, H=H, seed=31 + L, per_channel=True)
    s0 = torch.randn(B, H, 64, 64, generator=torch.Generator().manual_seed(32)) * 0.1
    tm = {k: x[k].transpose(1, 2).contiguous().to(DEV, dtype) for k in ("q", "k", "v", "b", "w", "log_alpha")}
    tv = lambda t: t.transpose(1, 2)
    o, S = mb.b200_dgda_prefill(tv(tm["q"]), tv(tm["k"]), tv(tm["v"]), None, tv(tm["b"]), tv(tm["w"]),
                                initial_state=s0.to(DEV), log_alpha=tv(tm["log_alpha"]), state_dtype=torch.float32,
                                out_layout="blhd")
    ref = {k: x[k].to(dtype).float().numpy() for k in x}
    ro, rS = OD.dgda_sequential(ref["q"], ref["k"], ref["v"], None, ref["b"], ref["w"], initial_state=s0.numpy(),
                                log_alpha=ref["log_alpha"])
    assert_rel(o, ro, rtol, "o")
    assert_rel(S, rS, rtol, "S")


@pytest.mark.parametrize("i", range(5))
def test_16bit_extreme_decay(i):
    g = sub(golden("dgda_prefill"), "ext.")
    d = dict(g)
    d["alpha"] = np.full_like(g["q"], g["alphas"][i])
    o, S = run_prefill(d, torch.bfloat16)
    assert torch.isfinite(o.float()).all() and torch.isfinite(S.float()).all()
    ro, rS = OD.dgda_sequential(*(torch.as_tensor(d[k]).to(torch.bfloat16).float().numpy()
                                  for k in ("q", "k", "v", "alpha", "b", "w")),
                                initial_state=torch.as_tensor(g["s0"]).to(torch.bfloat16).float().numpy())
    assert_rel(o, ro, RTOL_BF16, "o")
    assert_rel(S, rS, RTOL_BF16, "S")


def test_16bit_unaligned_and_short_head_dims():
    """dk=dv=32 and non-unit strides: the scalar-load branch of the tensor-core kernel."""
    g = sub(golden("dgda_prefill"), "len129.")
    o, S = run_prefill(g, torch.bfloat16)
    ro, rS = OD.dgda_sequential(*(torch.as_tensor(g[k]).to(torch.bfloat16).float().numpy()
                                  for k in ("q", "k", "v")), None,
                                *(torch.as_tensor(g[k]).to(torch.bfloat16).float().numpy() for k in ("b", "w")),
                                log_alpha=torch.as_tensor(g["la"]).to(torch.bfloat16).float().numpy())
    assert_rel(o, ro, RTOL_BF16, "o")
    assert_rel(S, rS, RTOL_BF16, "S")


def test_16bit_long_sequence_full_config2_length():
    """T = 65,536, H = 10 (the bench's DGDA op): segmented path, property + sampled oracle check."""
    x = dgda_inputs(B=1, T=65536, H=10, seed=20, per_channel=True)
    dt = torch.bfloat16
    tm = {k: x[k].transpose(1, 2).contiguous().to(DEV, dt) for k in ("q", "k", "v", "b", "w", "log_alpha")}
    tv = lambda t: t.transpose(1, 2)
    o, S = mb.b200_dgda_prefill(tv(tm["q"]), tv(tm["k"]), tv(tm["v"]), None, tv(tm["b"]), tv(tm["w"]),
                                log_alpha=tv(tm["log_alpha"]), state_dtype=torch.float32, out_layout="blhd")
    assert bool(torch.isfinite(o.float()).all()) and bool(torch.isfinite(S).all())
    # chaining property: the last 4096 tokens from the state at 61,440 equal the tail of the full run
    cut = 65536 - 4096
    part = lambda s, e: [tv(tm[k][:, s:e]) for k in ("q", "k", "v")]
    _, S1 = mb.b200_dgda_prefill(*part(0, cut), None, tv(tm["b"][:, :cut]), tv(tm["w"][:, :cut]),
                                 log_alpha=tv(tm["log_alpha"][:, :cut]), state_dtype=torch.float32)
    o2, S2 = mb.b200_dgda_prefill(*part(cut, 65536), None, tv(tm["b"][:, cut:]), tv(tm["w"][:, cut:]),
                                  initial_state=S1, log_alpha=tv(tm["log_alpha"][:, cut:]),
                                  state_dtype=torch.float32)
    assert_rel(o2, o[:, :, cut:], RTOL_BF16, "tail")
    assert_rel(S2, S, RTOL_BF16, "state")
    # oracle on heads 0..1 over the first 2048 tokens (sequential fp64)
    ref = {k: x[k][:, :2, :2048].to(dt).float().numpy() for k in x}
    ro, _ = OD.dgda_sequential(ref["q"], ref["k"], ref["v"], None, ref["b"], ref["w"], log_alpha=ref["log_alpha"])
    assert_rel(o[:, :2, :2048], ro, RTOL_BF16, "prefix")


@pytest.mark.parametrize("state", ["fp32", "bf16"])
def test_16bit_chunk_parallel_windows(monkeypatch, state):
    """Chunk-parallel path over several windows (window capped at 16 chunks): the fp32
    state carried between windows reproduces the unwindowed result; a 16-bit state
    takes the segmented path instead (windows need an fp32 carry)."""
    x = dgda_inputs(B=1, T=4096, H=2, seed=11, per_channel=True)
    dt = torch.bfloat16
    args = [x[k].to(DEV, dt) for k in ("q", "k", "v")]
    kw = dict(b=x["b"].to(DEV, dt), w=x["w"].to(DEV, dt), log_alpha=x["log_alpha"].to(DEV, dt))
    sd = torch.float32 if state == "fp32" else dt
    s0 = (torch.randn(1, 2, 64, 64, generator=torch.Generator().manual_seed(3)) * 0.1).to(DEV, sd)
    o_ref, S_ref = mb.b200_dgda_prefill(*args, None, initial_state=s0, state_dtype=sd, **kw)
    monkeypatch.setenv("MABA_DGDA_WINDOW_CHUNKS", "16")
    o, S = mb.b200_dgda_prefill(*args, None, initial_state=s0, state_dtype=sd, **kw)
    torch.cuda.synchronize()
    assert_rel(o, o_ref, RTOL_BF16, "o")
    assert_rel(S, S_ref, RTOL_BF16, "S")
    ro, rS = OD.dgda_sequential(*(t.float().cpu().numpy() for t in args), b=kw["b"].float().cpu().numpy(),
                                w=kw["w"].float().cpu().numpy(), initial_state=s0.float().cpu().numpy(),
                                log_alpha=kw["log_alpha"].float().cpu().numpy())
    assert_rel(o, ro, RTOL_BF16, "o vs oracle")
    assert_rel(S, rS, RTOL_BF16, "S vs oracle")
