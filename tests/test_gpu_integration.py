"""The drop-in claim itself: the UNMODIFIED reference model (maba_sparse, installed
offline under baseline/_ref, or the directory named by MABA_REFERENCE) runs its
forward and decode steps on the sm_100a kernels after ``integration.install()``
and reproduces its own CPU results.

The expected values come from the same reference model on the CPU, computed in
this test before ``install()`` (the reference dispatcher then runs its CPU
backend: cpu_dgda_prefill / cpu_dgda_step, cpu_compute_centroids /
cpu_index_topk, and the torch attention methods of MabaSparseAttention).  After
``install()`` the model moves to the GPU with nothing else changed: the registry
ops, the patched layer methods and strict mode carry it (maba_sparse/model.py:
207-276 forward / step; layers/sparse_attention.py:221-277; layers/dgda.py:
166-287).  Skips, visibly, where no reference install is present.
"""
import os
import sys

import pytest
import torch

from helpers import RTOL_FP32, assert_rel

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_dir():
    for path in (os.environ.get("MABA_REFERENCE"), os.path.join(REPO, "baseline", "_ref")):
        if path and os.path.isdir(os.path.join(path, "maba_sparse")):
            return path
    return None


@pytest.fixture(scope="module")
def reference():
    path = _reference_dir()
    if path is None:
        pytest.skip("no reference install (baseline/_ref or MABA_REFERENCE): the drop-in check needs it")
    if path not in sys.path:
        sys.path.insert(0, path)
    import maba_sparse
    return maba_sparse


def _model(reference, seed):
    from maba_sparse.config import MabaSparseConfig
    from maba_sparse.model import MabaSparseForCausalLM

    cfg = MabaSparseConfig(dim=128, n_heads=2, d_head=64, n_layers=4, vocab_size=512, d_emb=32,
                           intermediate_size=256, window_size=64, block_size=64, top_k=4, hca_pool_size=64,
                           dist_lambda=0.5)
    torch.manual_seed(seed)
    return MabaSparseForCausalLM(cfg).eval()


@pytest.mark.parametrize("T", [150, 300])
def test_unmodified_reference_model_on_b200_kernels(reference, T, monkeypatch):
    from maba_v2_architecture_b200.integration import install, uninstall

    monkeypatch.delenv("MABA_BACKEND", raising=False)
    monkeypatch.delenv("MABA_STRICT_BACKEND", raising=False)
    model = _model(reference, seed=31 + T)
    ids = torch.randint(0, 512, (2, T), generator=torch.Generator().manual_seed(T))
    nxt = torch.randint(0, 512, (2, 5), generator=torch.Generator().manual_seed(T + 1))
    # the reference on its own CPU path
    with torch.no_grad():
        out = model(ids)
        want_logits = out.logits
        ps = out.past_states
        want_steps = []
        for t in range(nxt.shape[1]):
            lg, ps = model.step(nxt[:, t:t + 1], past_states=ps)
            want_steps.append(lg)
    for layer in model.layers:
        if hasattr(layer.mixer, "reset_cache"):
            layer.mixer.reset_cache()
    h = install()
    try:
        from maba_sparse.kernels import dispatcher as rd

        assert rd.get_backend(torch.device("cuda", 0)) == "triton"
        m = model.to("cuda")
        with torch.no_grad():
            out = m(ids.cuda())
            assert_rel(out.logits, want_logits, RTOL_FP32, "reference model forward on B200 kernels")
            ps = out.past_states
            got = []
            for t in range(nxt.shape[1]):
                lg, ps = m.step(nxt[:, t:t + 1].cuda(), past_states=ps)
                got.append(lg)
        assert_rel(torch.cat(got, 1), torch.cat(want_steps, 1), RTOL_FP32, "reference model decode steps")
    finally:
        uninstall(h)
