"""install() wires the B200 ops into a loaded reference package (host logic only).

The reference package comes from MABA_REFERENCE (a directory holding maba_sparse) or
the offline install under baseline/_ref; the test skips where neither exists.  It
checks the registry entries, the method patches, the strict-mode environment and that
uninstall() restores the reference."""
import os
import sys

import pytest
import torch

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("MABA_REFERENCE") or os.path.join(_REPO, "baseline", "_ref")


@pytest.fixture
def reference():
    if not os.path.isdir(os.path.join(REF, "maba_sparse")):
        pytest.skip("reference checkout not available")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import maba_sparse
    return maba_sparse


def test_install_and_uninstall(reference, monkeypatch):
    monkeypatch.delenv("MABA_STRICT_BACKEND", raising=False)
    monkeypatch.delenv("MABA_BACKEND", raising=False)
    from maba_sparse.kernels import dispatcher as rd
    from maba_sparse.layers.indexer import DGIndexer as RefIx
    from maba_sparse.layers.sparse_attention import MabaSparseAttention as RefSA

    import maba_v2_architecture_b200 as mb
    from maba_v2_architecture_b200.integration import install, uninstall

    before = dict(rd._KERNEL_REGISTRY.get("triton", {}))
    fwd_sa, fwd_ix = RefSA.forward, RefIx.forward
    h = install()
    try:
        assert rd.get_kernel("triton", "dgda_prefill") is mb.b200_dgda_prefill
        assert rd.get_kernel("triton", "index_topk") is mb.b200_index_topk
        assert os.environ["MABA_STRICT_BACKEND"] == "1"
        assert rd.get_backend(torch.device("cuda", 0)) == "triton"
        assert RefSA.forward is mb.MabaSparseAttention.forward
        assert RefIx.forward is mb.DGIndexer.forward
        # a reference layer now routes through the B200 path, which has no CPU implementation
        layer = RefSA(dim=64, n_heads=2, d_head=32).eval()
        with pytest.raises(RuntimeError, match="no CPU path"):
            with torch.no_grad():
                layer(torch.randn(1, 8, 64))
    finally:
        uninstall(h)
    assert RefSA.forward is fwd_sa and RefIx.forward is fwd_ix
    assert dict(rd._KERNEL_REGISTRY.get("triton", {})) == before
    assert "MABA_STRICT_BACKEND" not in os.environ
