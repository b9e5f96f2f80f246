"""B200-native (sm_100a) DTEM spatial routing and local attention for MergeNet.

Drop-in replacements for the reference's hot-path functions
(opentome/timm/dtem.py, opentome/utils/thetopk.py,
opentome/timm/bias_local_attn.py) backed by hand-written CUDA kernels in
``libmergenet_b200.so``.  Every function runs on CUDA tensors only.
"""
from .routing import (  # noqa: F401
    RoutePlan,
    RouteResult,
    ThreTopK,
    build_patch_spatial_adjacency,
    build_patch_spatial_neighbors,
    carrier_scatter,
    carrier_ste,
    check_status,
    dtem_select,
    dtem_select_backward,
    route_and_gather,
    sparse_neighbor_dot,
    sparse_spatial_score,
    sparse_transport_adjoint,
    sparse_weighted_transport,
    soft_topk_aux_repr,
    sparse_weighted_transport_pair,
    thre_topk_backward,
)
from .dtem import DTEMMergeBlock, build_eval_group_indices, make_merge_block  # noqa: F401
from .attention import (  # noqa: F401
    LocalAttention,
    biased_local_attention,
    cross_attention,
    local_attention_packed,
    unbiased_local_attention,
)

__version__ = "0.1.0"
