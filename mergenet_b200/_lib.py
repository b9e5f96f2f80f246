"""ctypes binding of libmergenet_b200.so (declared in include/mergenet_b200.h).

The library is built in-tree by ``python -m mergenet_b200.build``.  There is
no fallback: if the shared library is missing or fails to load, every entry
point of the package raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmergenet_b200.so"

MN_F32, MN_F16, MN_BF16 = 0, 1, 2
MN_OK = 0
MN_ERR_ARG, MN_ERR_UNSUPPORTED, MN_ERR_WORKSPACE, MN_ERR_LAUNCH = -1, -2, -3, -4
MN_INFEASIBLE_BUDGET = 1
MN_STATUS_INFEASIBLE_BUDGET, MN_STATUS_DEGENERATE_RANGE, MN_STATUS_TOO_MANY_EDGES = 1, 2, 4
MN_STATUS_TC_TIMEOUT = 256
MN_EPI_BIAS = 0
MN_EPI_BIAS_GELU = 1

_DTYPES = {torch.float32: MN_F32, torch.float16: MN_F16, torch.bfloat16: MN_BF16}

_ERRORS = {
    MN_ERR_ARG: "invalid argument",
    MN_ERR_UNSUPPORTED: "shape outside what the kernels support",
    MN_ERR_WORKSPACE: "workspace too small",
    MN_ERR_LAUNCH: "kernel launch failed",
}


class RouteDims(ctypes.Structure):
    _fields_ = [
        ("grid_h", c_int), ("grid_w", c_int), ("num_patches", c_int), ("half", c_int),
        ("k_static", c_int), ("kc", c_int), ("kin", c_int), ("radius_rows", c_int),
        ("valid_rows", c_int * 2), ("stencil_dy1", c_int), ("stencil_dy3", c_int), ("table_ints", c_int64),
    ]


_P = c_void_p
_SIGNATURES = {
    "mn_version": (c_int, []),
    "mn_neighbor_table_width": (c_int, [c_int, c_int, c_double, POINTER(c_int)]),
    "mn_neighbor_table_fill": (c_int, [c_int, c_int, c_double, c_int, _P, _P]),
    "mn_route_dims_query": (c_int, [c_int, c_int, c_double, POINTER(RouteDims)]),
    "mn_route_tables_fill": (c_int, [c_int, c_int, c_double, POINTER(RouteDims), _P]),
    "mn_route_workspace_bytes": (c_size_t, [POINTER(RouteDims), c_int, c_int]),
    "mn_route_and_gather": (c_int, [POINTER(RouteDims), _P, c_int, c_int, c_int, c_int, POINTER(c_int), c_int,
                                    c_float, c_float, _P, c_int, _P, c_int, _P, c_size_t, _P, _P, _P, _P, _P,
                                    _P, _P]),
    "mn_sparse_spatial_score": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P,
                                        _P, _P, _P, _P, _P]),
    "mn_sparse_neighbor_dot": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, _P]),
    "mn_sparse_weighted_transport": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, _P,
                                             _P]),
    "mn_sparse_transport_adjoint": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, _P,
                                            _P, _P]),
    "mn_thre_topk_workspace_bytes": (c_size_t, [c_int, c_int]),
    "mn_thre_topk": (c_int, [c_int, c_int, _P, c_int, c_float, _P, _P, c_size_t, _P, _P]),
    "mn_soft_topk_aux": (c_int, [c_int, c_int, c_int, c_int, _P, c_int64, c_int64, _P, _P, _P]),
    "mn_soft_topk_aux_backward_workspace_bytes": (c_size_t, [c_int, c_int]),
    "mn_soft_topk_aux_backward": (c_int, [c_int, c_int, c_int, c_int, _P, c_int64, c_int64, _P, _P, _P, _P, _P,
                                          c_size_t, _P]),
    "mn_carrier_ste_backward": (c_int, [c_int, c_int, c_int, c_int, _P, c_int64, c_int64, _P, c_int64, c_int64, _P,
                                        c_int, _P, _P, _P]),
    "mn_thre_topk_backward_workspace_bytes": (c_size_t, [c_int, c_int]),
    "mn_thre_topk_backward": (c_int, [c_int, c_int, _P, c_int, c_float, _P, _P, _P, c_size_t, _P, _P]),
    "mn_dtem_select_workspace_bytes": (c_size_t, [c_int, c_int]),
    "mn_dtem_select": (c_int, [c_int, c_int, c_int, _P, _P, c_int, c_float, c_float, _P, _P, c_size_t, _P, _P]),
    "mn_dtem_select_backward_workspace_bytes": (c_size_t, [c_int, c_int]),
    "mn_dtem_select_backward": (c_int, [c_int, c_int, c_int, _P, _P, c_int, c_float, c_float, _P, _P, _P, c_size_t,
                                        _P, _P]),
    "mn_dtem_select_noalloc": (c_int, [c_int, c_int, c_int, _P, _P, c_int, c_float, c_float, _P, _P, _P]),
    "mn_carrier_scatter": (c_int, [c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P]),
    "mn_local_attention": (c_int, [c_int, c_int, c_int, c_int, c_int, _P, _P, _P, c_int64, c_int64, c_int64, _P,
                                   c_int, c_int, c_int, c_float, _P, c_int, _P, _P]),
    "mn_attention": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _P, c_int64, c_int64, c_int64, _P, _P,
                             c_int64, c_int64, c_int64, c_int, c_float, _P, c_int, _P, _P]),
    "mn_add_layernorm": (c_int, [c_int64, c_int, _P, _P, _P, _P, c_float, _P, _P, _P, c_int, _P]),
    "mn_add_layernorm_f32": (c_int, [c_int64, c_int, _P, _P, _P, _P, c_float, _P, c_int, _P]),
    "mn_embed_layernorm": (c_int, [c_int, c_int, c_int, _P, _P, _P, _P, _P, c_float, _P, _P, c_int, _P]),
    "mn_patch_unfold": (c_int, [c_int, c_int, c_int, c_int, c_int, _P, _P, _P]),
    "mn_gemm_f16": (c_int, [c_int, c_int, c_int, _P, c_int64, _P, c_int64, _P, c_int, _P, c_int64, _P, _P]),
    "mn_gemm_f32_split": (c_int, [c_int, c_int, c_int, _P, _P, c_int64, _P, _P, c_int64, _P, c_float, _P, c_int64,
                                  c_int, _P, _P]),
    "mn_layernorm_split": (c_int, [c_int64, c_int, _P, _P, _P, c_float, c_float, _P, _P, _P]),
    "mn_tc_wait_selftest": (c_int, [_P, c_double, _P]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def lib():
    """The loaded library (loaded once).  Raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m mergenet_b200.build` (needs nvcc)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.mn_version() != 1:
            raise RuntimeError("libmergenet_b200.so version mismatch; rebuild it")
        _lib = handle
    return _lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def check(rc: int, what: str) -> None:
    if rc == MN_OK:
        return
    if rc == MN_INFEASIBLE_BUDGET:
        raise RuntimeError(
            f"{what}: DTEM spatial radius leaves fewer eligible donor rows than the required merge budget")
    msg = _ERRORS.get(rc, f"error {rc}")
    if rc in (MN_ERR_ARG, MN_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError("expected torch tensors")
        if not t.is_cuda:
            raise RuntimeError("mergenet_b200 kernels run on CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    return dev
