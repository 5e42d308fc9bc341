"""The model on the B200 layers vs the reference model's golden logits (prefill and decode)."""
import pytest
import torch

from helpers import RTOL_FP32, assert_rel, golden, sub
from test_model_host import tiny_config
from maba_v2_architecture_b200.model import MabaSparseForCausalLM

pytestmark = pytest.mark.gpu
DEV = "cuda"


def load():
    g = golden("model")
    model = MabaSparseForCausalLM(tiny_config()).to(DEV).eval()
    model.load_state_dict({k: torch.from_numpy(v) for k, v in sub(g, "w.").items()})
    return g, model


def test_prefill_logits_vs_reference():
    g, model = load()
    with torch.no_grad():
        out = model(torch.from_numpy(g["ids"]).to(DEV))
    assert_rel(out.logits, g["logits"], RTOL_FP32, "logits")


def test_decode_steps_vs_reference():
    g, model = load()
    with torch.no_grad():
        out = model(torch.from_numpy(g["ids"]).to(DEV))
        ps = out.past_states
        nxt = torch.from_numpy(g["next_ids"]).to(DEV)
        steps = []
        for t in range(nxt.shape[1]):
            lg, ps = model.step(nxt[:, t:t + 1], past_states=ps)
            steps.append(lg)
    assert_rel(torch.cat(steps, 1), g["step_logits"], RTOL_FP32, "step logits")


def test_generate_greedy_runs():
    g, model = load()
    ids = torch.from_numpy(g["ids"][:, :20]).to(DEV)
    out = model.generate(ids, max_new_tokens=5, temperature=0.0)
    assert out.shape == (1, 25)


def test_decode_session_vs_reference_steps():
    """O(1)-append decode caches + split-K decode kernels reproduce the reference decode."""
    from maba_v2_architecture_b200.decode import DecodeSession

    g, model = load()
    sess = DecodeSession(model, batch=1, max_len=128, dtype=torch.float32)
    first = sess.prefill(torch.from_numpy(g["ids"]).to(DEV))
    assert_rel(first, g["logits"][:, -1:], RTOL_FP32, "prefill last logits")
    nxt = torch.from_numpy(g["next_ids"]).to(DEV)
    steps = [sess.step(nxt[:, t:t + 1]) for t in range(nxt.shape[1])]
    assert_rel(torch.cat(steps, 1), g["step_logits"], RTOL_FP32, "session step logits")


def test_decode_session_crosses_blocks_and_matches_model_step():
    """Many steps across several block / pooling boundaries, bf16, against model.step."""
    from maba_v2_architecture_b200.decode import DecodeSession
    from maba_v2_architecture_b200.workloads import init_module_

    cfg = tiny_config()
    model = init_module_(MabaSparseForCausalLM(cfg), seed=11).to(DEV).eval()
    ids = torch.randint(0, cfg.vocab_size, (2, 70), generator=torch.Generator().manual_seed(12)).to(DEV)
    nxt = torch.randint(0, cfg.vocab_size, (2, 40), generator=torch.Generator().manual_seed(13)).to(DEV)
    with torch.no_grad():
        out = model(ids)
        ps = out.past_states
        ref = []
        for t in range(40):
            lg, ps = model.step(nxt[:, t:t + 1], past_states=ps)
            ref.append(lg)
    sess = DecodeSession(model, batch=2, max_len=128, dtype=torch.float32)
    sess.prefill(ids)
    got = [sess.step(nxt[:, t:t + 1]) for t in range(40)]
    assert_rel(torch.cat(got, 1), torch.cat(ref, 1), 1e-4, "session vs model.step")


def test_decode_kernels_long_context_vs_oracle():
    """Split-K decode attention and split decode top-k at a 65,536-token context vs the oracle."""
    import numpy as np
    import maba_v2_architecture_b200 as mb
    from oracle import attention as OA
    from oracle import indexer as OI

    gen = torch.Generator().manual_seed(14)
    L, H, DC = 65536, 10, 128
    c = (torch.randn(1, L, DC, generator=gen) / 11.3).to(DEV, torch.bfloat16)
    qhat = (torch.randn(1, 1, H, DC, generator=gen) * 0.3).to(DEV, torch.bfloat16)
    kidx = (torch.randn(1, L, 64, generator=gen) / 11.3).to(DEV, torch.bfloat16)
    qi = (torch.randn(1, 1, 64, generator=gen) / 11.3).to(DEV, torch.bfloat16)
    gate = torch.randn(1, 1, 3, generator=gen).to(DEV, torch.bfloat16)
    cent = mb.b200_compute_centroids(kidx)
    idx = mb.b200_index_topk(qi, cent, lambda_dist=0.1, top_k=32, decode=True)
    oidx = OI.index_topk(qi.float().cpu().numpy(), cent.float().cpu().numpy(), lambda_dist=0.1, top_k=32, decode=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
    hca = mb.b200_hca_pool(c, 64)
    out = mb.b200_sa_attention(qhat, c, hca, idx, gate)
    ref = OA.sa_attention_latent(qhat.float().cpu().numpy(), c.float().cpu().numpy(), idx.cpu().numpy(),
                                 gate.float().cpu().numpy(), 128, 4, 64, 64)
    assert_rel(out, ref, 2e-2, "decode attention")


def test_graph_decode_matches_eager_session():
    """The captured decode step (device-held position) replays the eager session's results."""
    from maba_v2_architecture_b200.decode import DecodeSession
    from maba_v2_architecture_b200.workloads import init_module_

    cfg = tiny_config()
    model = init_module_(MabaSparseForCausalLM(cfg), seed=21).to(DEV).eval()
    ids = torch.randint(0, cfg.vocab_size, (2, 70), generator=torch.Generator().manual_seed(22)).to(DEV)
    eager = DecodeSession(model, batch=2, max_len=200, dtype=torch.float32)
    eager.prefill(ids)
    graph = DecodeSession(model, batch=2, max_len=200, dtype=torch.float32)
    first = graph.prefill(ids)[:, -1].argmax(-1, keepdim=True)
    graph.capture(first)
    tok = first
    for _ in range(60):  # crosses block (16) and pooling (16) boundaries several times
        le = eager.step(tok)
        tok = le[:, -1].argmax(-1, keepdim=True)
        lg = graph.replay()
        assert_rel(lg, le, 1e-5, "graph vs eager logits")
        assert torch.equal(graph.ids_buf, tok)
