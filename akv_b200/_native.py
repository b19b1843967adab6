"""ctypes binding of ``libakv_b200.so`` (declared in include/akv_b200.h).

The library is built in-tree by ``python -m akv_b200.build``.  There is no
fallback: importing the ops without the built library raises ImportError,
and a failed launch raises RuntimeError.
"""

from __future__ import annotations

import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libakv_b200.so")

AKV_OK, AKV_ERR_INVALID, AKV_ERR_CUDA, AKV_ERR_UNSUPPORTED = 0, 1, 2, 3
AKV_ERR_OCC_MISSING_SOURCE, AKV_ERR_OCC_MISSING_COPY_SOURCE = 4, 5
AKV_F16, AKV_BF16, AKV_F32 = 0, 1, 2
GATHER_OUT64, GATHER_LITERAL, GATHER_SEG64 = 1, 2, 4
DROP_RING_UNDERFLOW, DROP_RING_OVERFLOW, DROP_BAD_RANGE, DROP_NO_ACTIVE = 1, 2, 4, 8
DROP_BAD_PAGE = 16
REPOSITION_BULK_V = 1

DTYPE_CODE = {torch.float16: AKV_F16, torch.bfloat16: AKV_BF16, torch.float32: AKV_F32}

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64

LAYOUT_CAPACITY, LAYOUT_ERROR, LAYOUT_TOO_MANY = 1, 2, 4


class LayoutBatch(ctypes.Structure):
    """struct akv_layout_batch of include/akv_b200.h, field for field."""

    _fields_ = [
        ("n_requests", _I32), ("n_tiles", _I32), ("n_tokens", _I64), ("n_repositions", _I64),
        ("n_count_cells", _I64), ("token_offsets", _P), ("token_ids", _P),
        ("token_ids_is64", _I32), ("tile_offsets", _P), ("count_offsets", _P),
        ("drop_event_offsets", _P), ("drop_insert_offsets", _P), ("drop_range_offsets", _P),
        ("drop_ranges", _P), ("reposition_offsets", _P), ("reposition_raw_boundaries", _P),
        ("positions", _P), ("keep_mask", _P), ("materialized_stage", _P),
        ("birth_positions", _P), ("birth_stages", _P), ("token_to_key", _P), ("records", _P),
        ("virtual_mask", _P), ("key_to_token", _P), ("transition_offsets", _P),
        ("transition_request_offsets", _P), ("transition_raw_tokens", _P),
        ("transition_old_positions", _P), ("transition_new_positions", _P),
        ("transition_capacity", _I64), ("effective_reposition_stages", _P),
        ("effective_repositions", _P), ("ignored_repositions", _P), ("drop_event_to_key", _P),
        ("status", _P), ("active_offsets", _P), ("raw_indices", _P), ("active_positions", _P),
        ("totals", _P), ("workspace", _P),
    ]

# name -> argument types, in the order of include/akv_b200.h
SIGNATURES = {
    "akv_version": [],
    "akv_reposition_kv_layers": [
        _P, _P, _I32, _I32, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _I64, _I64,
        _P, _P, _I32, _I64, _I32, _I32, _I64, _I64, _P, _P,
    ],
    "akv_reposition_kv_layers_ex": [
        _P, _P, _I32, _I32, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _I64, _I64,
        _P, _P, _I32, _I64, _I32, _I32, _I64, _I64, _P, _I32, _P,
    ],
    "akv_reposition_divide": [_P, _P, _P, _I64, _I32, _P],
    "akv_drop_compact_tile_tokens": [],
    "akv_drop_compact_workspace_bytes": [_I32, _I32],
    "akv_drop_compact": [
        _I32, _P, _P, _I32, _P, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _P, _P, _P, _P, _P,
        _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
    ],
    "akv_drop_compact_paged": [
        _I32, _P, _P, _I32, _P, _P, _P, _P, _P, _I64, _I32, _I32, _P, _I64, _P, _P, _P, _P, _P,
        _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
    ],
    "akv_occurrence_advance_indices": [_P, _P],
    "akv_drop_read_view": [_P, _P, _P, _I64, _P, _P, _I32, _P, _P],
    "akv_drop_compact_static_max_requests": [],
    "akv_drop_compact_static_max_tiles": [],
    "akv_drop_compact_static": [
        _I32, _P, _P, _I32, _P, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _P, _P, _P, _P, _P,
        _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
    ],
    "akv_context_decode_indices": [
        _P, _P, _I64, _P, _I32, _P, _I32, _P, _I32, _P, _I32, _P, _I32, _P, _I32, _I64, _I32,
        _P,
    ],
    "akv_context_window_lengths": [_P, _P, _I32, _P, _I32, _P, _I32, _I64, _I32, _P],
    "akv_build_decode_metadata": [
        _P, _P, _I64, _P, _P, _I64, _P, _I64, _I32, _P, _P, _P, _P, _P,
    ],
    "akv_write_row_slots": [_P, _P, _I32, _P, _I32, _P, _I32, _I64, _P],
    "akv_active_slots": [_P, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P],
    "akv_active_slots_batch": [_P, _P, _P, _I32, _P, _P, _P],
    "akv_active_slots_chunk": [],
    "akv_gather_slots_chunk": [],
    "akv_gather_slots": [_P, _P, _I32, _P, _P, _P],
    "akv_compile_layouts_max_repositions": [],
    "akv_compile_layouts_workspace_bytes": [_I32, _I64, _I64, _I64],
    "akv_compile_layouts_batch_bytes": [],
    "akv_compile_layouts": [ctypes.POINTER(LayoutBatch), _P],
    "akv_decode_attention": [
        _P, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, ctypes.c_float, _I32,
        _I32, _I32, _I32, _P, _I32, _P, _I32, _P, _P, _P, _P, _I64, _I64, _P, _P, _P,
    ],
    "akv_decode_attention_ctas_per_sm": [_I32, _I32],
    "akv_context_attention_query_block": [],
    "akv_context_attention": [
        _P, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P,
        ctypes.c_float, _I64, _I32, _I32, _I32, _P, _I32, _P, _I64, _I64, _P, _P, _I32, _P,
    ],
}
RESTYPES = {
    "akv_version": ctypes.c_char_p,
    "akv_drop_compact_tile_tokens": _I64,
    "akv_drop_compact_workspace_bytes": _I64,
    "akv_drop_compact_static_max_requests": _I64,
    "akv_drop_compact_static_max_tiles": _I64,
    "akv_compile_layouts_max_repositions": _I64,
    "akv_compile_layouts_workspace_bytes": _I64,
    "akv_compile_layouts_batch_bytes": _I64,
    "akv_decode_attention_ctas_per_sm": _I32,
    "akv_context_attention_query_block": _I64,
    "akv_active_slots_chunk": _I64,
    "akv_gather_slots_chunk": _I64,
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built; run `python -m akv_b200.build` (nvcc, sm_100a). "
            "akv_b200 has no CPU or Triton fallback."
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = RESTYPES.get(name, ctypes.c_int)
    return lib


lib = _load()


def ptr(t):
    """Device address of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device) -> ctypes.c_void_p:
    """The current torch stream of ``device`` as a cudaStream_t."""
    if _raw_stream is not None:
        if isinstance(device, int):
            return ctypes.c_void_p(_raw_stream(device))
        d = device if isinstance(device, torch.device) else torch.device(device)
        if d.type == "cuda":
            index = d.index if d.index is not None else torch.cuda.current_device()
            return ctypes.c_void_p(_raw_stream(index))
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(status: int, what: str) -> None:
    if status == AKV_OK:
        return
    if status == AKV_ERR_INVALID:
        raise ValueError(f"{what}: invalid arguments")
    if status == AKV_ERR_UNSUPPORTED:
        raise ValueError(f"{what}: unsupported configuration")
    raise RuntimeError(f"{what}: CUDA launch failed (status {status})")


def is64(t) -> int:
    if t.dtype == torch.int64:
        return 1
    if t.dtype == torch.int32:
        return 0
    raise ValueError(f"index tensors must be int32 or int64, got {t.dtype}")
