"""Decode kernels at a long context: the split decode top-k and the split-K decode
attention (tensor-core split kernel for 16-bit d_c = 128) against the CPU oracle,
with a host-known length and at a device-held position over capacity-sized caches."""
import numpy as np
import pytest
import torch

import maba_v2_architecture_b200 as mb
from helpers import assert_rel
from oracle import attention as OA
from oracle import indexer as OI

pytestmark = pytest.mark.gpu
DEV = "cuda"


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


@pytest.mark.parametrize("L", [1000, 4159, 65536])
def test_decode_at_device_position_vs_oracle(L):
    """maba_index_topk_decode_at / maba_sa_attention_decode_at over caches sized for more than L
    tokens, the position held on the device; every stream (window + sinks, selected blocks,
    pooled rows) and the gate superposition against the oracle."""
    gen = torch.Generator().manual_seed(L)
    H, DC, cap = 10, 128, L + 300
    c_cap = torch.zeros(1, cap, DC, dtype=torch.bfloat16, device=DEV)
    k_cap = torch.zeros(1, cap, 64, dtype=torch.bfloat16, device=DEV)
    c = (torch.randn(1, L, DC, generator=gen) / 11.3).to(DEV, torch.bfloat16)
    kidx = (torch.randn(1, L, 64, generator=gen) / 11.3).to(DEV, torch.bfloat16)
    c_cap[:, :L] = c
    k_cap[:, :L] = kidx
    cent_cap = torch.zeros(1, cap // 64 + 1, 64, dtype=torch.bfloat16, device=DEV)
    cent = mb.b200_compute_centroids(kidx)
    cent_cap[:, :cent.shape[1]] = cent
    hca_cap = torch.zeros(1, cap // 64, DC, dtype=torch.bfloat16, device=DEV)
    hca = mb.b200_hca_pool(c, 64)
    hca_cap[:, :hca.shape[1]] = hca
    pos = torch.full((), L - 1, dtype=torch.long, device=DEV)
    qi = (torch.randn(1, 1, 64, generator=gen) / 11.3).to(DEV, torch.bfloat16)
    qhat = (torch.randn(1, 1, H, DC, generator=gen) * 0.3).to(DEV, torch.bfloat16)
    gate = torch.randn(1, 1, 3, generator=gen).to(DEV, torch.bfloat16)
    idx = mb.b200_index_topk_decode_at(qi, cent_cap, pos, lambda_dist=0.1, top_k=32)
    nb = (L + 63) // 64
    oidx = OI.index_topk(qi.float().cpu().numpy(), cent.float().cpu().numpy(), lambda_dist=0.1, top_k=32, decode=True)
    np.testing.assert_array_equal(idx[..., :min(32, nb)].cpu().numpy(), oidx[..., :min(32, nb)])
    out = mb.b200_sa_attention_decode_at(qhat, c_cap, hca_cap, idx, gate, pos)
    ref = OA.sa_attention_latent(qhat.float().cpu().numpy(), c.float().cpu().numpy(), idx.cpu().numpy(),
                                 gate.float().cpu().numpy(), 128, 4, 64, 64)
    assert_rel(out, ref, 2e-2, "decode attention at a device-held position")
