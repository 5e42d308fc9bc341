"""The model's module tree matches the reference's (state dicts interchange)."""
import numpy as np

from helpers import golden, sub
from maba_v2_architecture_b200.config import MabaSparseConfig, get_101m_config
from maba_v2_architecture_b200.model import MabaSparseForCausalLM


def tiny_config():
    c = golden("model")["cfg"].tolist()
    return MabaSparseConfig(dim=c[0], n_heads=c[1], d_head=c[2], n_layers=c[3], vocab_size=c[4], d_emb=c[5],
                            intermediate_size=c[6], window_size=c[7], block_size=c[8], top_k=c[9],
                            hca_pool_size=c[10], dist_lambda=0.5)


def test_state_dict_keys_and_shapes_match_reference():
    ref = sub(golden("model"), "w.")
    model = MabaSparseForCausalLM(tiny_config())
    sd = model.state_dict()
    assert set(sd) == set(ref)
    for k, v in sd.items():
        assert tuple(v.shape) == ref[k].shape, k


def test_101m_parameter_count_and_topology():
    model = MabaSparseForCausalLM(get_101m_config())
    n = sum(p.numel() for p in model.parameters())
    assert n == 101_282_319
    assert [l.is_attention for l in model.layers] == [(i + 1) % 4 == 0 for i in range(20)]
