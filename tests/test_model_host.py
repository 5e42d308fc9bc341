"""The engine's view of the model: the reference's state-dict names and shapes
(so reference checkpoints load), the 101M parameter count and the 3:1 layer
pattern (maba_sparse/model.py:62-129, 162-206)."""
import os
import sys

from helpers import golden, sub
from maba_v2_architecture_b200.config import MabaSparseConfig, get_101m_config
from maba_v2_architecture_b200.engine import TIED, ModelShape, init_state_dict, parameter_shapes

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def tiny_config():
    c = golden("model")["cfg"].tolist()
    return MabaSparseConfig(dim=c[0], n_heads=c[1], d_head=c[2], n_layers=c[3], vocab_size=c[4], d_emb=c[5],
                            intermediate_size=c[6], window_size=c[7], block_size=c[8], top_k=c[9],
                            hca_pool_size=c[10], dist_lambda=0.5)


def test_state_dict_keys_and_shapes_match_reference():
    ref = sub(golden("model"), "w.")
    shapes = parameter_shapes(ModelShape.from_config(tiny_config()))
    assert set(shapes) == set(ref)
    for k, v in shapes.items():
        assert tuple(v) == ref[k].shape, k


def test_101m_parameter_count_and_topology():
    s = ModelShape.from_config(get_101m_config())
    shapes = parameter_shapes(s)
    n = 0
    for name, shp in shapes.items():
        if name in TIED:
            continue
        k = 1
        for d in shp:
            k *= d
        n += k
    assert n == 101_282_319
    assert [s.is_attention(i) for i in range(20)] == [(i + 1) % 4 == 0 for i in range(20)]


def test_init_state_dict_ties_and_values():
    s = ModelShape.from_config(tiny_config())
    sd = init_state_dict(s, seed=3)
    assert sd["lm_head.weight"] is sd["embeddings.in_emb.weight"]
    assert float(sd["layers.0.res_gate1"][0]) == 2.0 and float(sd["final_norm.weight"][0]) == 1.0
    assert float(sd["layers.3.mixer.stream_gate.bias"].abs().sum()) == 0.0
    assert abs(float(sd["layers.0.mixer.q_proj.weight"].std()) - 0.02) < 0.005


def test_shapes_match_the_installed_reference_101m():
    """Against the unmodified reference model's own state dict, where a reference install exists."""
    import pytest
    path = next((p for p in (os.environ.get("MABA_REFERENCE"), os.path.join(REPO, "baseline", "_ref"))
                 if p and os.path.isdir(os.path.join(p, "maba_sparse"))), None)
    if path is None:
        pytest.skip("no reference install")
    if path not in sys.path:
        sys.path.insert(0, path)
    from maba_sparse.model import MabaSparseForCausalLM, get_101m_config as ref_cfg
    sd = MabaSparseForCausalLM(ref_cfg()).state_dict()
    shapes = parameter_shapes(ModelShape.from_config(ref_cfg()))
    assert set(shapes) == set(sd)
    for k, v in shapes.items():
        assert tuple(v) == tuple(sd[k].shape), k
