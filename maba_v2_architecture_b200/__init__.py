"""B200 (sm_100a) implementation of the Maba v2 inference hot path.

DGDA chunked prefill and decode step, DG-Indexer pooling + scoring + top-k,
and MABA-SA three-stream attention with gate superposition, as hand-written
CUDA kernels behind a C ABI (include/maba_b200.h, libmaba_b200.so), exposed
with the reference project's op, registry and layer interfaces.
"""
from .config import MabaSparseConfig, MabaConfig, get_101m_config
from .dispatcher import (
    clear_dispatcher_cache,
    clear_fallback_warnings,
    compute_centroids,
    dgda_prefill,
    dgda_step,
    dispatch_compute_centroids,
    dispatch_dgda_prefill,
    dispatch_dgda_step,
    dispatch_index_topk,
    dispatch_stream_superposition,
    get_backend,
    get_kernel,
    index_topk,
    register_kernel,
    stream_superposition,
)
from .layers import ConvState, DGDALayer, DGIndexer, DecoupledGatedDeltaAttention, DeltaGuidedCentroidIndexer
from .layers import MABASALayer, MabaSparseAttention
from .ops import (
    b200_compute_centroids,
    b200_decode_cache_append,
    b200_dgda_prefill,
    b200_dgda_step,
    b200_dgda_transition,
    b200_hca_pool,
    b200_index_topk,
    b200_index_topk_decode_at,
    b200_sa_attention,
    b200_sa_attention_decode_at,
    b200_stream_superposition,
)

__version__ = "0.1.0"
