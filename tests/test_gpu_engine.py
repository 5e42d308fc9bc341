"""The inference engine (engine.py) against the reference model.

* the golden tiny model (tests/golden/model.npz, written by the reference
  MabaSparseForCausalLM): prefill logits and six teacher-forced decode steps;
* decode == prefill: every decode step's logits equal the prefill logits of the
  same position (float32 engine, 101M layer shapes with 4 layers, across block
  and pooling boundaries);
* the captured CUDA-graph step replays the eager step exactly;
* with a reference install present: the engine in bf16 vs the unmodified
  reference model on the CPU (same weights, bf16-rounded) at the 101M shape.
"""
import os
import sys

import numpy as np
import pytest
import torch

from helpers import RTOL_BF16, RTOL_FP32, assert_rel, golden, sub
from test_model_host import tiny_config
from maba_v2_architecture_b200.config import MabaSparseConfig, get_101m_config
from maba_v2_architecture_b200.engine import MabaEngine, ModelShape, init_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def golden_engine(dtype=torch.float32):
    g = golden("model")
    sd = {k: torch.from_numpy(v) for k, v in sub(g, "w.").items()}
    return g, MabaEngine(tiny_config(), sd, dtype=dtype)


def test_prefill_logits_vs_reference_golden():
    g, eng = golden_engine()
    logits = eng.forward(torch.from_numpy(g["ids"]).to(DEV))
    assert_rel(logits, g["logits"], RTOL_FP32, "engine prefill logits")


def test_decode_steps_vs_reference_golden():
    g, eng = golden_engine()
    sess = eng.new_session(batch=1, max_len=128)
    last = sess.prefill(torch.from_numpy(g["ids"]).to(DEV))
    assert_rel(last[:, -1], g["logits"][:, -1], RTOL_FP32, "session prefill last logits")
    nxt = torch.from_numpy(g["next_ids"]).to(DEV)
    steps = [sess.step(nxt[:, t]).clone() for t in range(nxt.shape[1])]
    assert_rel(torch.stack(steps, 1), g["step_logits"], RTOL_FP32, "engine decode steps")


def small_101m_shape(n_layers=4):
    return get_101m_config(n_layers=n_layers)


@pytest.mark.parametrize("B,T,steps", [(1, 130, 70), (2, 63, 80)])
def test_decode_equals_prefill_fp32(B, T, steps):
    """Teacher-forced decode across block (64) and pooling (64) boundaries: the logits of each step
    equal the prefill logits at that position (same weights, float32)."""
    cfg = small_101m_shape()
    eng = MabaEngine(cfg, init_state_dict(ModelShape.from_config(cfg), seed=17), dtype=torch.float32)
    ids = torch.randint(0, cfg.vocab_size, (B, T + steps), generator=torch.Generator().manual_seed(18)).to(DEV)
    full = eng.forward(ids)
    sess = eng.new_session(batch=B, max_len=T + steps + 8)
    first = sess.prefill(ids[:, :T])
    assert_rel(first[:, -1], full[:, T - 1], RTOL_FP32, "prefill last")
    got = []
    for t in range(T, T + steps):
        got.append(sess.step(ids[:, t]).clone())
    assert_rel(torch.stack(got, 1), full[:, T:T + steps], 5e-4, "decode vs prefill")


@pytest.mark.parametrize("tiny", [False, True])
def test_fused_dgda_mix_equals_two_launch_form(tiny):
    """maba_decode_dgda_mix (input GEMV + features + each head's recurrence step in the head's last
    CTA) against the two-launch form (GEMV with the features epilogue, then the state kernel); the
    101M layer shapes (d_k = d_v = 64, 10 heads) and the tiny model's (32, 2 heads)."""
    cfg = tiny_config() if tiny else small_101m_shape()
    eng = MabaEngine(cfg, init_state_dict(ModelShape.from_config(cfg), seed=31), dtype=torch.float32)
    ids = torch.randint(0, cfg.vocab_size, (3, 100), generator=torch.Generator().manual_seed(32)).to(DEV)
    fused, split = eng.new_session(batch=3, max_len=128), eng.new_session(batch=3, max_len=128)
    fused.fuse_mix, split.fuse_mix = True, False
    assert fused.launches_per_step() < split.launches_per_step()
    fused.prefill(ids[:, :70])
    split.prefill(ids[:, :70])
    for t in range(70, 100):
        a, b = fused.step(ids[:, t]).clone(), split.step(ids[:, t]).clone()
        assert_rel(a, b, 1e-5, f"fused vs split step {t}")
    for i in fused.states:
        assert_rel(fused.states[i], split.states[i], 1e-5, f"state {i}")


def test_graph_replay_matches_eager_steps():
    cfg = small_101m_shape(n_layers=8)
    sd = init_state_dict(ModelShape.from_config(cfg), seed=21)
    eng = MabaEngine(cfg, sd, dtype=torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (2, 70), generator=torch.Generator().manual_seed(22)).to(DEV)
    eager = eng.new_session(batch=2, max_len=200)
    graph = eng.new_session(batch=2, max_len=200)
    tok = eager.prefill(ids)[:, -1].argmax(-1)
    graph.prefill(ids)
    graph.ids_buf.copy_(tok)
    graph.capture()
    for _ in range(60):
        le = eager.step(tok).clone()
        tok = le.argmax(-1)
        lg = graph.replay()
        assert torch.equal(lg, le), "graph vs eager logits"
        assert torch.equal(graph.ids_buf, tok), "device argmax"
    assert int(graph.pos_dev) == 70 + 60 == graph.length
    # the bench's per-step accounting: every weight is read once per step
    weights = sum(t.numel() * t.element_size() for L in eng.layers for t in (L.w_gu, L.w_down, L.mix.w_in))
    assert graph.bytes_per_step() > weights
    assert graph.launches_per_step() == 3 + sum(2 + (7 if L.attn else 3) for L in eng.layers)


def _reference_dir():
    for path in (os.environ.get("MABA_REFERENCE"), os.path.join(REPO, "baseline", "_ref")):
        if path and os.path.isdir(os.path.join(path, "maba_sparse")):
            return path
    return None


def test_engine_bf16_vs_unmodified_reference_101m_shape():
    """The engine (bf16) vs the reference model on its CPU path in float32 with the same
    (bf16-rounded) weights, at the 101M layer shapes with 4 layers (one MABA-SA)."""
    path = _reference_dir()
    if path is None:
        pytest.skip("no reference install (baseline/_ref or MABA_REFERENCE)")
    if path not in sys.path:
        sys.path.insert(0, path)
    from maba_sparse.model import MabaSparseForCausalLM, get_101m_config as ref_cfg_fn
    rcfg = ref_cfg_fn()
    rcfg.n_layers = rcfg.num_layers = 4
    cfg = small_101m_shape()
    sd = init_state_dict(ModelShape.from_config(cfg), seed=23)
    sd16 = {k: v.to(torch.bfloat16).float() for k, v in sd.items()}
    ref = MabaSparseForCausalLM(rcfg).eval()
    ref.load_state_dict(sd16)
    ids = torch.randint(0, cfg.vocab_size, (1, 200), generator=torch.Generator().manual_seed(24))
    with torch.no_grad():
        want = ref(ids).logits
    eng = MabaEngine(cfg, sd16, dtype=torch.bfloat16)
    got = eng.forward(ids.to(DEV))
    assert_rel(got, want, RTOL_BF16, "engine bf16 vs reference")
