"""Host-side registry behaviour (no GPU): the reference dispatcher's interface
(maba_sparse/kernels/dispatcher.py) with one backend and no silent fallback.
Fault injection follows the reference's fallback tests
(tests/test_dispatcher_fallbacks.py:35-175): a registry entry is replaced by a
failing fake; here the failure must surface instead of running a CPU path."""
import threading

import pytest
import torch

import maba_v2_architecture_b200.dispatcher as D


@pytest.fixture(autouse=True)
def clean_env(monkeypatch):
    monkeypatch.delenv("MABA_BACKEND", raising=False)
    D.clear_dispatcher_cache()
    yield
    D.clear_dispatcher_cache()


def test_backend_names(monkeypatch):
    assert D.get_backend() == "b200"
    assert D.get_backend(torch.device("cuda", 1)) == "b200"
    for alias in ("auto", "b200", "triton", "cuda", "GPU"):
        monkeypatch.setenv("MABA_BACKEND", alias)
        assert D.get_backend("cuda:0") == "b200"
    monkeypatch.setenv("MABA_BACKEND", "cpu")
    with pytest.raises(ValueError, match="Unsupported MABA_BACKEND"):
        D.get_backend("cuda:0")


def test_registry_has_the_five_ops():
    for op in D.OPS:
        assert callable(D.get_kernel("b200", op))
    assert D.get_kernel("b200", "nope") is None


@pytest.mark.parametrize("exc", [ZeroDivisionError, MemoryError, RuntimeError])
def test_injected_failure_propagates(monkeypatch, exc):
    def broken(**kw):
        raise exc("injected")

    monkeypatch.setitem(D._KERNEL_REGISTRY["b200"], "compute_centroids", broken)
    with pytest.raises(exc, match="injected"):
        D.dispatch_compute_centroids(torch.zeros(1, 64, 8))


def test_register_kernel_roundtrip(monkeypatch):
    calls = []

    @D.register_kernel("b200", "stream_superposition")
    def fake(**kw):
        calls.append(kw)
        return "ok"

    try:
        x = torch.zeros(1, 2, 3, 4)
        assert D.dispatch_stream_superposition(x, x, x, gate_logits=torch.zeros(1, 3, 3)) == "ok"
        assert calls and "gate_logits" in calls[0]
    finally:
        from maba_v2_architecture_b200.ops import b200_stream_superposition
        D._KERNEL_REGISTRY["b200"]["stream_superposition"] = b200_stream_superposition


def test_dispatch_validation():
    x = torch.zeros(1, 2, 8, 4)
    with pytest.raises(ValueError, match="Either alpha or log_alpha"):
        D.dispatch_dgda_prefill(x, x, x, b=x, w=x)
    with pytest.raises(ValueError, match="q_idx and centroids must be 3D"):
        D.dispatch_index_topk(torch.zeros(4, 8), torch.zeros(1, 1, 8))
    with pytest.raises(ValueError, match="block_size must be positive"):
        D.dispatch_compute_centroids(torch.zeros(1, 4, 8), block_size=0)


def test_concurrent_get_backend():
    out, errs = [], []

    def worker():
        try:
            for i in range(200):
                out.append(D.get_backend(f"cuda:{i % 8}"))
                if i % 50 == 0:
                    D.clear_dispatcher_cache()
        except Exception as e:  # pragma: no cover
            errs.append(e)

    ts = [threading.Thread(target=worker) for _ in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs and set(out) == {"b200"}
