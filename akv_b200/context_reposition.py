"""Drop-in ``reposition_kv_layers`` backed by the sm_100a reposition kernel.

Same signature, argument meaning, validation and error messages as the
reference's ``reposition_kv_layers``
(akv/system/sglang/kernels/ops/attention/context_reposition.py:126-212), so
``ContextLayerCopy.apply`` and ``ContextModelBinding.reposition_existing``
(srt/layers/attention/context_backend.py:324-341, 432-472) call it unchanged.
The launch goes through the C ABI ``akv_reposition_kv_layers``.

One keyword is added: ``count_device``, an optional int32 CUDA tensor with
one element holding the number of leading transitions to process.  With it,
a transition list whose length is only known on the device (the output of
``drop_compact``) needs no device-to-host read; ``len(source_slots)`` is then
the capacity.  Callers that do not pass it get the reference's behaviour.

Slots are bounded by the exemplar pool's slot count and positions by the
cos/sin table's length: a transition outside them is skipped instead of
touching memory outside the pools, and ``error_flag`` (optional int32 CUDA
tensor) gets bit 1 (bit 2: a bulk-copy wait of ``bulk_copy_v`` ran out).

A transition whose source equals its destination is rotated in place; the
reference's contract (fresh destinations disjoint from every source) is
unchanged for everything else.
"""

from __future__ import annotations

import torch

from . import _native


def reposition_kv_layers(
    k_data_ptrs: torch.Tensor,
    v_data_ptrs: torch.Tensor,
    k_layout: torch.Tensor,
    v_layout: torch.Tensor,
    source_slots: torch.Tensor,
    destination_slots: torch.Tensor,
    position_pairs: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    *,
    is_neox_style: bool = True,
    page_size: int = 1,
    skip_unmapped: bool = False,
    rotary_dim: int | None = None,
    count_device: torch.Tensor | None = None,
    error_flag: torch.Tensor | None = None,
    bulk_copy_v: bool = False,
) -> None:
    """Rotate K and copy V across native per-layer pools in one GPU launch.

    Pointer tables hold the 64-bit base address of every layer's
    [slot, head, dim] pool; each layer has the exemplar's dtype and strides.
    The caller owns fresh, distinct destination slots disjoint from all
    source slots (or passes source == destination for an in-place rotation),
    validates positions/slots on the CPU before they reach the device, and
    keeps the KV pools and metadata alive until the stream finishes.  No
    device-to-host read, no synchronisation, no allocation.

    ``page_size``: the reference accepts 1 only (context_reposition.py:
    153-154).  Slots here are token slots (page * page_size + offset) in
    every case, so the paged pools of ``DropCompactor(page_size=...)``
    (powers of two from 4 to 128) are accepted as well; any other value
    raises the reference's error.

    ``bulk_copy_v``: move the V rows of copy transitions with TMA bulk
    copies in a second kernel (``AKV_REPOSITION_BULK_V``).  Faster when
    copies are a minority of the list, as in a Drop's mixed list of in-place
    rotations and copy-on-write, and a token's V row (local heads x head_dim
    x element size) is 512 bytes or more; slower when every transition is a
    copy, and at 128-byte rows (one KV head of head_dim 64).  Results are
    identical either way.
    """
    if page_size != 1 and (page_size < 4 or page_size > 128 or page_size & (page_size - 1)):
        raise ValueError("Context Reposition requires page_size=1")
    tensors = (
        k_data_ptrs,
        v_data_ptrs,
        k_layout,
        v_layout,
        source_slots,
        destination_slots,
        position_pairs,
        cos_sin_cache,
    )
    index = k_layout.get_device()  # -1 for a CPU tensor
    if index < 0 or any(t.get_device() != index for t in tensors):
        raise ValueError("Reposition tensors must be on one CUDA device")
    if k_layout.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("Context Reposition requires unquantized floating-point KV")
    if (
        k_layout.ndim != 3
        or v_layout.shape != k_layout.shape
        or v_layout.dtype != k_layout.dtype
    ):
        raise ValueError("Reposition requires matching native NHD K/V layouts")
    if k_layout.stride(-1) != 1 or v_layout.stride(-1) != 1:
        raise ValueError("Reposition requires contiguous head dimensions")
    if (
        k_data_ptrs.ndim != 1
        or v_data_ptrs.shape != k_data_ptrs.shape
        or k_data_ptrs.dtype not in (torch.uint64, torch.int64)
        or v_data_ptrs.dtype not in (torch.uint64, torch.int64)
        or not k_data_ptrs.is_contiguous()
        or not v_data_ptrs.is_contiguous()
    ):
        raise ValueError("Reposition requires contiguous 64-bit layer pointer tables")
    count = len(source_slots)
    if (
        source_slots.ndim != 1
        or destination_slots.shape != source_slots.shape
        or source_slots.dtype != torch.int32
        or destination_slots.dtype != torch.int32
        or not source_slots.is_contiguous()
        or not destination_slots.is_contiguous()
        or position_pairs.shape != (count, 2)
        or position_pairs.dtype != torch.int32
        or position_pairs.stride(-1) != 1
    ):
        raise ValueError("Reposition requires int32 slot vectors and [N, 2] positions")
    head_dim = k_layout.shape[-1]
    rotary_dim = head_dim if rotary_dim is None else rotary_dim
    if (
        type(rotary_dim) is not int
        or not 0 < rotary_dim <= head_dim
        or rotary_dim % 2
        or cos_sin_cache.ndim != 2
        or cos_sin_cache.shape[1] != rotary_dim
        or cos_sin_cache.stride(-1) != 1
        or not cos_sin_cache.is_floating_point()
    ):
        raise ValueError("Reposition requires a native cos/sin cache matching rotary_dim")
    if cos_sin_cache.dtype not in _native.DTYPE_CODE:
        raise ValueError("Reposition requires a native cos/sin cache matching rotary_dim")
    if error_flag is not None and (
        error_flag.get_device() != index or error_flag.dtype != torch.int32
    ):
        raise ValueError("error_flag must be an int32 tensor on the KV device")
    if count_device is not None and (
        count_device.get_device() != index
        or count_device.dtype != torch.int32
        or count_device.numel() < 1
    ):
        raise ValueError("count_device must be an int32 tensor on the KV device")
    if count == 0 or len(k_data_ptrs) == 0:
        return
    status = _native.lib.akv_reposition_kv_layers_ex(
        _native.ptr(k_data_ptrs),
        _native.ptr(v_data_ptrs),
        len(k_data_ptrs),
        _native.DTYPE_CODE[k_layout.dtype],
        k_layout.shape[1],
        head_dim,
        rotary_dim,
        k_layout.stride(0),
        k_layout.stride(1),
        v_layout.stride(0),
        v_layout.stride(1),
        _native.ptr(source_slots),
        _native.ptr(destination_slots),
        _native.ptr(position_pairs),
        position_pairs.stride(0),
        count,
        _native.ptr(count_device),
        _native.ptr(cos_sin_cache),
        _native.DTYPE_CODE[cos_sin_cache.dtype],
        cos_sin_cache.stride(0),
        int(bool(is_neox_style)),
        int(bool(skip_unmapped)),
        k_layout.shape[0],
        cos_sin_cache.shape[0],
        _native.ptr(error_flag),
        _native.REPOSITION_BULK_V if bulk_copy_v else 0,
        _native.stream_of(index),
    )
    _native.check(status, "reposition_kv_layers")


def layer_pointer_table(buffers, device=None) -> torch.Tensor:
    """uint64 device tensor of the buffers' base addresses, the table the
    native KV pool builds once per engine (context_backend.py:416-417)."""
    device = device or buffers[0].device
    return torch.tensor([b.data_ptr() for b in buffers], dtype=torch.uint64, device=device)
