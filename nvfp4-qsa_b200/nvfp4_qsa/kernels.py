"""NVFP4 paged-cache writer and QSA sparse reader: the reference's raw ops.

Same names, argument order and meaning as the reference module
``nvfp4_qsa.kernels`` (python/nvfp4_qsa/kernels.py:152-165 and :348-403), so
the vLLM backend hooks that import ``qsa_write_cache_nvfp4`` and
``qsa_sparse_paged_attention_nvfp4`` run unchanged.  Both launch hand-written
sm_100a kernels through the C ABI (include/nvfp4_qsa.h) on the current CUDA
stream and never synchronize, so they are legal inside CUDA graph capture.

Physical layout per K or V region (reference kernels.py:4-6):
  data  [blocks, page, kv_heads, head_dim / 2] uint8 (low nibble is element 2j)
  scale [blocks, page, kv_heads, head_dim / 16] uint8 holding float8_e4m3fn bytes
The global K/V scales are fixed for the lifetime of a cache.
"""
from __future__ import annotations

import contextlib
import ctypes
from functools import lru_cache

import torch

from . import _native

__all__ = [
    "qsa_sparse_paged_attention_nvfp4",
    "qsa_write_cache_nvfp4",
    "qsa_norm_rope_write_cache_nvfp4",
    "qsa_kv_proj_write_cache_nvfp4",
    "qsa_sparse_paged_attention_nvfp4_partial",
    "qsa_sparse_paged_attention_fp8",
    "qsa_sparse_paged_attention",
    "qsa_merge_partials",
    "qsa_merge_partials_strided",
    "qsa_sparse_paged_attention_nvfp4_split_kv",
    "attention_workspace_bytes",
]


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _device_ctx(device: torch.device):
    if device.type != "cuda":
        raise ValueError("NVFP4 QSA kernels require CUDA tensors")
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _check_same_device(tensors, device):
    for t in tensors:
        if t.device != device:
            raise ValueError("All NVFP4 QSA tensors must be on the same CUDA device")


def _check_write_region(source, data, scale, slot_mapping):
    """Host checks of the reference's _write_one (kernels.py:118-129)."""
    if source.dim() != 3:
        raise ValueError("NVFP4 QSA K/V must be [tokens, kv_heads, head_dim]")
    head_dim = source.shape[2]
    if source.dtype != torch.bfloat16:
        raise TypeError("NVFP4 QSA writer requires BF16 K/V")
    if data.dtype != torch.uint8 or scale.dtype != torch.uint8:
        raise TypeError("NVFP4 QSA data and scale caches must use uint8 storage")
    if slot_mapping.dtype != torch.int64:
        raise TypeError("NVFP4 QSA slot_mapping must be int64")
    if head_dim % 16 or data.shape[-1] != head_dim // 2:
        raise ValueError("invalid NVFP4 QSA packed-data shape")
    if scale.shape[-1] != head_dim // 16:
        raise ValueError("invalid NVFP4 QSA group-scale shape")
    if data.dim() != 4 or scale.dim() != 4:
        raise ValueError("NVFP4 QSA cache regions must be [blocks, page, kv_heads, bytes]")
    if source.stride(-1) != 1 or data.stride(-1) != 1 or scale.stride(-1) != 1:
        raise ValueError("NVFP4 QSA tensors need a contiguous last dimension")
    if slot_mapping.dim() != 1 or slot_mapping.shape[0] != source.shape[0] or slot_mapping.stride(0) != 1:
        raise ValueError("NVFP4 QSA slot_mapping must be a contiguous [tokens] vector")


def qsa_write_cache_nvfp4(
    key,
    value,
    key_data,
    key_scale,
    value_data,
    value_scale,
    slot_mapping,
    key_global_scale,
    value_global_scale,
):
    """Quantize and write K/V without synchronizing the serving hot path.

    One kernel launch writes both K and V (the reference launches twice).
    Tokens whose slot is negative or beyond the cache are skipped
    (kernels.py:71-77).  Valid slots must be unique: duplicates race, exactly
    as in the reference; ``PackedCache.write`` rejects them on the host.
    """
    _check_write_region(key, key_data, key_scale, slot_mapping)
    _check_write_region(value, value_data, value_scale, slot_mapping)
    if key.shape != value.shape:
        raise ValueError("NVFP4 QSA K and V must have the same shape")
    if key_data.shape[:3] != value_data.shape[:3]:
        raise ValueError("NVFP4 QSA K and V caches must share [blocks, page, kv_heads]")
    if key_data.shape[2] != key.shape[1]:
        raise ValueError("NVFP4 QSA cache kv_heads does not match K/V")
    device = key.device
    _check_same_device((value, key_data, key_scale, value_data, value_scale, slot_mapping), device)
    num_tokens, kv_heads, head_dim = key.shape
    if num_tokens == 0:
        return
    lib = _native.load()
    with _device_ctx(device):
        status = lib.nvqsa_write_cache(
            key.data_ptr(), key.stride(0), key.stride(1),
            value.data_ptr(), value.stride(0), value.stride(1),
            key_data.data_ptr(), key_data.stride(0), key_data.stride(1), key_data.stride(2),
            key_scale.data_ptr(), key_scale.stride(0), key_scale.stride(1), key_scale.stride(2),
            value_data.data_ptr(), value_data.stride(0), value_data.stride(1), value_data.stride(2),
            value_scale.data_ptr(), value_scale.stride(0), value_scale.stride(1), value_scale.stride(2),
            slot_mapping.data_ptr(), num_tokens, kv_heads, head_dim,
            key_data.shape[0], key_data.shape[1],
            float(key_global_scale), float(value_global_scale), _stream_ptr(device))
    _native.check(status, "qsa_write_cache_nvfp4")


def qsa_norm_rope_write_cache_nvfp4(
    key,
    value,
    key_data,
    key_scale,
    value_data,
    value_scale,
    slot_mapping,
    key_global_scale,
    value_global_scale,
    positions=None,
    cos_sin_cache=None,
    k_norm_weight=None,
    eps=1e-6,
    is_neox_style=True,
    norm_weight_offset=1.0,
    key_out=None,
):
    """k-norm -> RoPE -> NVFP4 quantize -> scatter in one launch, K read once.

    The reference's caller (integration/snapshot/qsa.py:618-667) runs vLLM's
    GemmaRMSNorm ``k_norm`` and rotary embedding on K and then
    ``qsa_write_cache_nvfp4``; this takes K straight from the QKV projection.
    ``k_norm_weight`` is the GemmaRMSNorm weight (``norm_weight_offset=1.0``
    multiplies by ``1 + w`` in fp32; 0.0 by ``w``) or None for no norm;
    ``cos_sin_cache`` is the rotary embedding's ``[max_position, rotary_dim]``
    cos|sin table, cast to bf16 as vLLM's native path casts it to the query
    dtype; ``positions`` is int64 ``[tokens]``.  The rotation is vLLM's bf16
    arithmetic bit for bit; the norm is fp32 with a fixed summation order and
    an IEEE square root and divide (``include/nvfp4_qsa.h``), so it can differ
    from torch's reduction by one bf16 ulp on rare elements.  ``key_out``
    (bf16 ``[tokens, kv_heads, head_dim]``) optionally receives the rotated K.
    Tokens whose position is outside the table are skipped entirely.
    """
    _check_write_region(key, key_data, key_scale, slot_mapping)
    _check_write_region(value, value_data, value_scale, slot_mapping)
    if key.shape != value.shape:
        raise ValueError("NVFP4 QSA K and V must have the same shape")
    if key_data.shape[:3] != value_data.shape[:3]:
        raise ValueError("NVFP4 QSA K and V caches must share [blocks, page, kv_heads]")
    if key_data.shape[2] != key.shape[1]:
        raise ValueError("NVFP4 QSA cache kv_heads does not match K/V")
    num_tokens, kv_heads, head_dim = key.shape
    device = key.device
    rotary_dim, max_position, cs_ptr, cs_stride, pos_ptr = 0, 0, 0, 0, 0
    if cos_sin_cache is not None:
        if positions is None:
            raise ValueError("a rotary embedding needs positions")
        if cos_sin_cache.dim() != 2 or cos_sin_cache.shape[1] % 2:
            raise ValueError("cos_sin_cache must be [max_position, rotary_dim]")
        if positions.dtype != torch.int64 or positions.dim() != 1 or positions.shape[0] != num_tokens:
            raise ValueError("positions must be an int64 [tokens] vector")
        cos_sin_cache = cos_sin_cache.to(torch.bfloat16)
        # the kernel reads each lane's cos/sin run with one vector load: a table whose rows are not
        # aligned to head_dim/16 bytes is made contiguous first
        run_bytes = head_dim // 16 if is_neox_style else max(head_dim // 32, 2)
        if (cos_sin_cache.stride(-1) != 1 or (cos_sin_cache.stride(0) * 2) % run_bytes
                or cos_sin_cache.data_ptr() % run_bytes):
            cos_sin_cache = cos_sin_cache.contiguous()
        positions = positions.contiguous()
        rotary_dim, max_position = cos_sin_cache.shape[1], cos_sin_cache.shape[0]
        cs_ptr, cs_stride, pos_ptr = cos_sin_cache.data_ptr(), cos_sin_cache.stride(0), positions.data_ptr()
        if rotary_dim > head_dim or rotary_dim % (head_dim // 16):
            raise ValueError(f"rotary_dim {rotary_dim} must be a multiple of head_dim/16 and at most head_dim")
    w_ptr = 0
    if k_norm_weight is not None:
        if k_norm_weight.numel() != head_dim:
            raise ValueError("k_norm_weight must have head_dim elements")
        k_norm_weight = k_norm_weight.reshape(head_dim).to(torch.float32).contiguous()
        w_ptr = k_norm_weight.data_ptr()
    ko_ptr, ko_st, ko_sh = 0, 0, 0
    ko_dst = None  # an unaligned key_out view is written through an aligned temporary
    if key_out is not None:
        if key_out.shape != key.shape or key_out.dtype != torch.bfloat16 or key_out.stride(-1) != 1:
            raise ValueError("key_out must be bf16 like key with a contiguous last dimension")
        ko_bytes = min(head_dim // 16, 16)
        if key_out.data_ptr() % ko_bytes or (key_out.stride(0) * 2) % ko_bytes or (key_out.stride(1) * 2) % ko_bytes:
            ko_dst, key_out = key_out, torch.empty(key.shape, dtype=torch.bfloat16, device=key_out.device)
        ko_ptr, ko_st, ko_sh = key_out.data_ptr(), key_out.stride(0), key_out.stride(1)
    extra = [t for t in (positions, cos_sin_cache, k_norm_weight, key_out) if t is not None]
    _check_same_device((value, key_data, key_scale, value_data, value_scale, slot_mapping, *extra), device)
    if num_tokens == 0:
        return key_out
    lib = _native.load()
    with _device_ctx(device):
        status = lib.nvqsa_norm_rope_write_cache(
            key.data_ptr(), key.stride(0), key.stride(1),
            value.data_ptr(), value.stride(0), value.stride(1),
            key_data.data_ptr(), key_data.stride(0), key_data.stride(1), key_data.stride(2),
            key_scale.data_ptr(), key_scale.stride(0), key_scale.stride(1), key_scale.stride(2),
            value_data.data_ptr(), value_data.stride(0), value_data.stride(1), value_data.stride(2),
            value_scale.data_ptr(), value_scale.stride(0), value_scale.stride(1), value_scale.stride(2),
            slot_mapping.data_ptr(), num_tokens, kv_heads, head_dim,
            key_data.shape[0], key_data.shape[1],
            float(key_global_scale), float(value_global_scale),
            w_ptr, float(norm_weight_offset), float(eps),
            pos_ptr, cs_ptr, cs_stride, max_position, rotary_dim, 1 if is_neox_style else 0,
            ko_ptr, ko_st, ko_sh, _stream_ptr(device))
    _native.check(status, "qsa_norm_rope_write_cache_nvfp4")
    if ko_dst is not None:
        # rows of skipped tokens stay as they were in the caller's tensor
        if positions is not None and rotary_dim > 0:
            valid = ((positions >= 0) & (positions < max_position)).view(-1, 1, 1)
            ko_dst.copy_(torch.where(valid, key_out, ko_dst))  # no host sync
        else:
            ko_dst.copy_(key_out)
        return ko_dst
    return key_out


def _aligned16(t):
    """t itself when its base and row strides are 16-byte aligned, else a copy with fresh storage."""
    if t.data_ptr() % 16 == 0 and all((st * t.element_size()) % 16 == 0 for st in t.stride()[:-1]):
        return t
    return t.clone() if t.is_contiguous() else t.contiguous()


def qsa_kv_proj_write_cache_nvfp4(
    hidden,
    key_weight,
    value_weight,
    key_data,
    key_scale,
    value_data,
    value_scale,
    slot_mapping,
    key_global_scale,
    value_global_scale,
    positions=None,
    cos_sin_cache=None,
    k_norm_weight=None,
    eps=1e-6,
    is_neox_style=True,
    norm_weight_offset=1.0,
    key_out=None,
    value_out=None,
):
    """K/V projection + k-norm + RoPE + NVFP4 quantize + scatter in one launch.

    The reference's layer (integration/snapshot/qsa.py:658-667 -> :618-640)
    computes ``qkv = hidden @ W_qkv^T`` in bf16, then k_norm and the rotary
    embedding on K, then ``qsa_write_cache_nvfp4``.  This computes the K and V
    columns of that projection on the tensor cores and encodes them straight
    from the accumulators.  ``hidden`` is bf16 ``[tokens, hidden_size]``;
    ``key_weight`` / ``value_weight`` are the bf16 ``[kv_heads * 256,
    hidden_size]`` K and V row blocks of the QKV weight (views are fine).  The
    other arguments mean what they mean for ``qsa_norm_rope_write_cache_nvfp4``;
    ``key_out`` receives the rotated K and ``value_out`` the V projection (bf16
    ``[tokens, kv_heads, 256]``, 16-byte aligned rows).  Each K and V value is
    the fp32 tensor-core sum rounded to bf16, which can differ by one bf16 ulp
    from another GEMM's; the cache bytes are those of the fused writer on
    exactly these K and V.  Returns ``(key_out, value_out)``.
    """
    if hidden.dim() != 2 or key_weight.dim() != 2 or value_weight.dim() != 2:
        raise ValueError("hidden must be [tokens, hidden_size] and the weights [kv_heads * 256, hidden_size]")
    for t in (hidden, key_weight, value_weight):
        if t.dtype != torch.bfloat16:
            raise TypeError("the K/V projection takes bf16 hidden states and weights")
        if t.stride(-1) != 1:
            raise ValueError("hidden states and weights need a contiguous last dimension")
    num_tokens, hidden_size = hidden.shape
    if key_weight.shape != value_weight.shape or key_weight.shape[1] != hidden_size:
        raise ValueError("key_weight and value_weight must both be [kv_heads * 256, hidden_size]")
    head_dim = 256
    if key_weight.shape[0] % head_dim:
        raise ValueError("the fused K/V projection supports head_dim 256")
    kv_heads = key_weight.shape[0] // head_dim
    for data, scale in ((key_data, key_scale), (value_data, value_scale)):  # the writer's checks (kernels.py:118-129)
        if data.dtype != torch.uint8 or scale.dtype != torch.uint8:
            raise TypeError("NVFP4 QSA data and scale caches must use uint8 storage")
        if data.dim() != 4 or scale.dim() != 4:
            raise ValueError("NVFP4 QSA cache regions must be [blocks, page, kv_heads, bytes]")
        if data.shape[-1] != head_dim // 2:
            raise ValueError("invalid NVFP4 QSA packed-data shape")
        if scale.shape[-1] != head_dim // 16:
            raise ValueError("invalid NVFP4 QSA group-scale shape")
        if data.stride(-1) != 1 or scale.stride(-1) != 1:
            raise ValueError("NVFP4 QSA tensors need a contiguous last dimension")
    if slot_mapping.dtype != torch.int64:
        raise TypeError("NVFP4 QSA slot_mapping must be int64")
    if slot_mapping.dim() != 1 or slot_mapping.shape[0] != num_tokens or slot_mapping.stride(0) != 1:
        raise ValueError("NVFP4 QSA slot_mapping must be a contiguous [tokens] vector")
    if key_data.shape[:3] != value_data.shape[:3] or key_data.shape[2] != kv_heads:
        raise ValueError("NVFP4 QSA K and V caches must share [blocks, page, kv_heads] with the weights' kv_heads")
    hidden = _aligned16(hidden)
    key_weight, value_weight = _aligned16(key_weight), _aligned16(value_weight)
    if key_weight.stride(0) != value_weight.stride(0):
        key_weight, value_weight = key_weight.contiguous(), value_weight.contiguous()
    device = hidden.device
    rotary_dim, max_position, cs_ptr, cs_stride, pos_ptr = 0, 0, 0, 0, 0
    if cos_sin_cache is not None:
        if positions is None:
            raise ValueError("a rotary embedding needs positions")
        if cos_sin_cache.dim() != 2 or cos_sin_cache.shape[1] % 2:
            raise ValueError("cos_sin_cache must be [max_position, rotary_dim]")
        if positions.dtype != torch.int64 or positions.dim() != 1 or positions.shape[0] != num_tokens:
            raise ValueError("positions must be an int64 [tokens] vector")
        cos_sin_cache = _aligned16(cos_sin_cache.to(torch.bfloat16))
        if cos_sin_cache.stride(-1) != 1:
            cos_sin_cache = cos_sin_cache.contiguous()
        positions = positions.contiguous()
        rotary_dim, max_position = cos_sin_cache.shape[1], cos_sin_cache.shape[0]
        cs_ptr, cs_stride, pos_ptr = cos_sin_cache.data_ptr(), cos_sin_cache.stride(0), positions.data_ptr()
        if rotary_dim > head_dim or rotary_dim % (32 if is_neox_style else 16):
            raise ValueError(f"rotary_dim {rotary_dim} must be a multiple of {32 if is_neox_style else 16} "
                             "and at most 256 for the fused K/V projection")
    w_ptr = 0
    if k_norm_weight is not None:
        if k_norm_weight.numel() != head_dim:
            raise ValueError("k_norm_weight must have head_dim elements")
        k_norm_weight = _aligned16(k_norm_weight.reshape(head_dim).to(torch.float32).contiguous())
        w_ptr = k_norm_weight.data_ptr()
    outs = []
    for o, name in ((key_out, "key_out"), (value_out, "value_out")):
        if o is None:
            outs.append((0, 0, 0))
            continue
        if o.shape != (num_tokens, kv_heads, head_dim) or o.dtype != torch.bfloat16 or o.stride(-1) != 1:
            raise ValueError(f"{name} must be bf16 [tokens, kv_heads, 256] with a contiguous last dimension")
        if o.data_ptr() % 16 or (o.stride(0) * 2) % 16 or (o.stride(1) * 2) % 16:
            raise ValueError(f"{name} needs 16-byte aligned rows")
        outs.append((o.data_ptr(), o.stride(0), o.stride(1)))
    extra = [t for t in (positions, cos_sin_cache, k_norm_weight, key_out, value_out) if t is not None]
    _check_same_device((key_weight, value_weight, key_data, key_scale, value_data, value_scale, slot_mapping,
                        *extra), device)
    if num_tokens == 0:
        return key_out, value_out
    lib = _native.load()
    with _device_ctx(device):
        status = lib.nvqsa_kv_proj_write_cache(
            hidden.data_ptr(), hidden.stride(0), num_tokens, hidden_size,
            key_weight.data_ptr(), value_weight.data_ptr(), key_weight.stride(0),
            key_data.data_ptr(), key_data.stride(0), key_data.stride(1), key_data.stride(2),
            key_scale.data_ptr(), key_scale.stride(0), key_scale.stride(1), key_scale.stride(2),
            value_data.data_ptr(), value_data.stride(0), value_data.stride(1), value_data.stride(2),
            value_scale.data_ptr(), value_scale.stride(0), value_scale.stride(1), value_scale.stride(2),
            slot_mapping.data_ptr(), kv_heads, head_dim,
            key_data.shape[0], key_data.shape[1], float(key_global_scale), float(value_global_scale),
            w_ptr, float(norm_weight_offset), float(eps),
            pos_ptr, cs_ptr, cs_stride, max_position, rotary_dim, 1 if is_neox_style else 0,
            *outs[0], *outs[1], _stream_ptr(device))
    _native.check(status, "qsa_kv_proj_write_cache_nvfp4")
    return key_out, value_out


@lru_cache(maxsize=256)
def _workspace_bytes(device_index, rows, query_heads, kv_heads, head_dim, topk):
    import ctypes

    out = ctypes.c_size_t(0)
    status = _native.load().nvqsa_sparse_attention_workspace_size(rows, query_heads, kv_heads, head_dim, topk,
                                                                  ctypes.byref(out))
    _native.check(status, "nvqsa_sparse_attention_workspace_size")
    return int(out.value)


def attention_workspace_bytes(rows, query_heads, kv_heads, head_dim, topk, device=None):
    """Scratch bytes the reader needs for this problem on ``device``."""
    device = torch.device("cuda") if device is None else torch.device(device)
    with _device_ctx(device):
        index = torch.cuda.current_device()
        return _workspace_bytes(index, int(rows), int(query_heads), int(kv_heads), int(head_dim), int(topk))


def _check_read(query, key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                token_to_request):
    if query.dim() != 3 or query.dtype != torch.bfloat16 or query.stride(-1) != 1:
        raise ValueError("NVFP4 QSA query must be bf16 [rows, query_heads, head_dim] with contiguous last dim")
    for t in (key_data, key_scale, value_data, value_scale):
        if t.dtype != torch.uint8 or t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError("NVFP4 QSA cache regions must be uint8 [blocks, page, kv_heads, bytes]")
    head_dim = query.shape[2]
    if key_data.shape[-1] != head_dim // 2 or value_data.shape[-1] != head_dim // 2:
        raise ValueError("invalid NVFP4 QSA packed-data shape")
    if key_scale.shape[-1] != head_dim // 16 or value_scale.shape[-1] != head_dim // 16:
        raise ValueError("invalid NVFP4 QSA group-scale shape")
    for t in (logical_indices, block_table, token_to_request):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("NVFP4 QSA metadata must be contiguous int32")
    if logical_indices.dim() != 2 or logical_indices.shape[0] < query.shape[0]:
        raise ValueError("NVFP4 QSA logical_indices must be [rows, topk]")
    if block_table.dim() != 2:
        raise ValueError("NVFP4 QSA block_table must be [requests, pages]")
    if token_to_request.dim() != 1 or token_to_request.shape[0] < query.shape[0]:
        raise ValueError("NVFP4 QSA token_to_request must be [rows]")


def _cache_args(key_data, key_scale, value_data, value_scale):
    return (
        key_data.data_ptr(), key_data.stride(0), key_data.stride(1), key_data.stride(2),
        key_scale.data_ptr(), key_scale.stride(0), key_scale.stride(1), key_scale.stride(2),
        value_data.data_ptr(), value_data.stride(0), value_data.stride(1), value_data.stride(2),
        value_scale.data_ptr(), value_scale.stride(0), value_scale.stride(1), value_scale.stride(2),
        key_data.shape[0], key_data.shape[1], key_data.shape[2])


def qsa_sparse_paged_attention_nvfp4(
    query,
    key_data,
    key_scale,
    value_data,
    value_scale,
    key_global_scale,
    value_global_scale,
    logical_indices,
    block_table,
    token_to_request,
    output,
    rows_per_group=1,
):
    """Sparse paged GQA decode over an NVFP4 cache; writes ``output`` in place.

    Semantics of the reference kernel (kernels.py:168-345): query heads
    ``h*G .. h*G+G-1`` use kv head ``h``; selection ``logical_indices[r, i]``
    of request ``token_to_request[r]`` is masked when the request, index,
    page or physical block is out of range; rows without a valid selection
    become zeros.  Split-KV scratch comes from the caching allocator on the
    current stream.

    ``rows_per_group`` (keyword, default 1: the reference behaviour) is a hint
    for multi-token-prediction batches: consecutive rows in groups of this
    size (2..4) that share their request and selections are served by one
    gather per record (verified on the device; groups that do not share are
    processed row by row, with the same result).
    """
    _check_read(query, key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                token_to_request)
    if output.shape != query.shape or output.dtype != torch.bfloat16 or output.stride(-1) != 1:
        raise ValueError("NVFP4 QSA output must be bf16 shaped like query with contiguous last dim")
    device = query.device
    _check_same_device((key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                        token_to_request, output), device)
    rows, query_heads, head_dim = query.shape
    if rows == 0:
        return
    topk = logical_indices.shape[1]
    kv_heads = key_data.shape[2]
    lib = _native.load()
    with _device_ctx(device):
        ws_bytes = _workspace_bytes(torch.cuda.current_device(), rows, query_heads, kv_heads, head_dim, topk)
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if ws_bytes else None
        common = (
            query.data_ptr(), query.stride(0), query.stride(1),
            *_cache_args(key_data, key_scale, value_data, value_scale),
            float(key_global_scale), float(value_global_scale),
            logical_indices.data_ptr(), topk,
            block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
            token_to_request.data_ptr(),
            output.data_ptr(), output.stride(0), output.stride(1),
            rows, query_heads, head_dim)
        tail = (workspace.data_ptr() if workspace is not None else None, ws_bytes, _stream_ptr(device))
        if rows_per_group == 1:
            status = lib.nvqsa_sparse_attention(*common, *tail)
        else:
            status = lib.nvqsa_sparse_attention_grouped(*common, int(rows_per_group), *tail)
    _native.check(status, "qsa_sparse_paged_attention_nvfp4")


def qsa_sparse_paged_attention_fp8(
    q,
    k_cache,
    v_cache,
    k_scale,
    v_scale,
    logical_indices,
    block_table,
    token_to_req,
    out=None,
):
    """FP8 sibling of the NVFP4 reader (src/qsa_fp8_harness.py:211-325); returns ``out``.

    ``k_cache`` / ``v_cache`` are float8_e4m3fn [blocks, page, kv_heads, head_dim]
    (vLLM's view of the fp8 main cache, snapshot/qsa.py:328-350); the per-tensor
    ``k_scale`` multiplies the scores and ``v_scale`` the output.  Masking and
    output rules as ``qsa_sparse_paged_attention_nvfp4``; ``out`` defaults to a
    new bf16 tensor shaped like ``q``.
    """
    if q.dim() != 3 or q.dtype != torch.bfloat16 or q.stride(-1) != 1:
        raise ValueError("QSA FP8 query must be bf16 [rows, query_heads, head_dim] with contiguous last dim")
    for t in (k_cache, v_cache):
        if t.dtype != torch.float8_e4m3fn or t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError("QSA FP8 caches must be float8_e4m3fn [blocks, page, kv_heads, head_dim]")
    if k_cache.shape != v_cache.shape or k_cache.shape[-1] != q.shape[2]:
        raise ValueError("QSA FP8 K/V caches must match each other and the query head_dim")
    for t in (logical_indices, block_table, token_to_req):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("QSA FP8 metadata must be contiguous int32")
    if out is None:
        out = torch.empty_like(q)
    if out.shape != q.shape or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("QSA FP8 output must be bf16 shaped like q with contiguous last dim")
    device = q.device
    _check_same_device((k_cache, v_cache, logical_indices, block_table, token_to_req, out), device)
    rows, query_heads, head_dim = q.shape
    if rows == 0:
        return out
    topk = logical_indices.shape[1]
    kv_heads = k_cache.shape[2]
    lib = _native.load()
    with _device_ctx(device):
        ws_bytes = _workspace_bytes(torch.cuda.current_device(), rows, query_heads, kv_heads, head_dim, topk)
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if ws_bytes else None
        status = lib.nvqsa_sparse_attention_fp8(
            q.data_ptr(), q.stride(0), q.stride(1),
            k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
            k_cache.shape[0], k_cache.shape[1], kv_heads, float(k_scale), float(v_scale),
            logical_indices.data_ptr(), topk,
            block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
            token_to_req.data_ptr(),
            out.data_ptr(), out.stride(0), out.stride(1),
            rows, query_heads, head_dim,
            workspace.data_ptr() if workspace is not None else None, ws_bytes, _stream_ptr(device))
    _native.check(status, "qsa_sparse_paged_attention_fp8")
    return out


STAMP_SLOTS = 8


def set_stamp_buffer(stamps: torch.Tensor | None) -> None:
    """Install (or, with None, remove) an int64 device buffer [units, 8] of %globaltimer stamps that every reader
    launch on its device fills per (row, kv head) unit; see nvqsa_set_stamp_buffer.  A measurement aid."""
    lib = _native.load()
    if stamps is None:
        _native.check(lib.nvqsa_set_stamp_buffer(None), "set_stamp_buffer")
        return
    if stamps.dtype != torch.int64 or not stamps.is_cuda or not stamps.is_contiguous():
        raise ValueError("stamps must be a contiguous int64 CUDA tensor")
    with _device_ctx(stamps.device):
        _native.check(lib.nvqsa_set_stamp_buffer(stamps.data_ptr()), "set_stamp_buffer")


def reset_stamps(stamps: torch.Tensor) -> None:
    """Prepare a stamp buffer for one launch: slot 0 to all ones (it takes a minimum), the others to zero."""
    stamps.zero_()
    stamps.view(-1, STAMP_SLOTS)[:, 0] = -1


def qsa_sparse_paged_attention(
    query,
    key_cache,
    value_cache,
    logical_indices,
    block_table,
    token_to_req,
    output=None,
):
    """BF16 sibling reader: QSA sparse paged decode over the bf16 main cache; returns ``output``.

    Replaces vLLM's ``qsa_sparse_paged_attention`` that the reference calls in the BF16 branch of
    ``forward_qsa`` (integration/snapshot/qsa.py:352-366).  ``key_cache`` / ``value_cache`` are bf16
    [blocks, page, kv_heads, head_dim] views (last dim contiguous; vLLM's split of a
    [blocks, kv_heads, page, 2 * head_dim] cache), scale head_dim^-0.5.  Masking and output rules as
    ``qsa_sparse_paged_attention_nvfp4``; ``output`` defaults to a new bf16 tensor shaped like ``query``.
    """
    if query.dim() != 3 or query.dtype != torch.bfloat16 or query.stride(-1) != 1:
        raise NotImplementedError("QSA requires a BF16 query [rows, query_heads, head_dim] with contiguous last dim")
    for t in (key_cache, value_cache):
        if t.dtype != torch.bfloat16:
            raise NotImplementedError("QSA requires BF16 Q/K/V")
        if t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError("QSA BF16 caches must be [blocks, page, kv_heads, head_dim] with contiguous last dim")
    if key_cache.shape != value_cache.shape or key_cache.shape[-1] != query.shape[2]:
        raise ValueError("QSA BF16 K/V caches must match each other and the query head_dim")
    for t in (logical_indices, block_table, token_to_req):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("QSA metadata must be contiguous int32")
    if output is None:
        output = torch.empty_like(query)
    if output.shape != query.shape or output.dtype != torch.bfloat16 or output.stride(-1) != 1:
        raise ValueError("QSA output must be bf16 shaped like query with contiguous last dim")
    device = query.device
    _check_same_device((key_cache, value_cache, logical_indices, block_table, token_to_req, output), device)
    rows, query_heads, head_dim = query.shape
    if rows == 0:
        return output
    topk = logical_indices.shape[1]
    kv_heads = key_cache.shape[2]
    lib = _native.load()
    el = key_cache.element_size()
    with _device_ctx(device):
        size = ctypes.c_size_t()
        _native.check(lib.nvqsa_sparse_attention_bf16_workspace_size(rows, query_heads, kv_heads, head_dim, topk,
                                                                     ctypes.byref(size)), "workspace size")
        ws_bytes = size.value
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if ws_bytes else None
        status = lib.nvqsa_sparse_attention_bf16(
            query.data_ptr(), query.stride(0), query.stride(1),
            key_cache.data_ptr(), key_cache.stride(0) * el, key_cache.stride(1) * el, key_cache.stride(2) * el,
            value_cache.data_ptr(), value_cache.stride(0) * el, value_cache.stride(1) * el,
            value_cache.stride(2) * el,
            key_cache.shape[0], key_cache.shape[1], kv_heads,
            logical_indices.data_ptr(), topk,
            block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
            token_to_req.data_ptr(),
            output.data_ptr(), output.stride(0), output.stride(1),
            rows, query_heads, head_dim,
            workspace.data_ptr() if workspace is not None else None, ws_bytes, _stream_ptr(device))
    _native.check(status, "qsa_sparse_paged_attention")
    return output


def qsa_sparse_paged_attention_nvfp4_partial(
    query,
    key_data,
    key_scale,
    value_data,
    value_scale,
    key_global_scale,
    value_global_scale,
    logical_indices,
    block_table,
    token_to_request,
    partial_out,
    partial_lse,
):
    """Un-merged reader output for split-KV across devices.

    Writes fp32 ``partial_out[rows, query_heads, head_dim]`` (softmax over this
    device's valid selections, divided by ``value_global_scale``) and
    ``partial_lse[rows, query_heads]`` = max + log2(sum), or -inf when none of
    the row's selections is valid here.  Merge with ``qsa_merge_partials``.
    """
    _check_read(query, key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                token_to_request)
    rows, query_heads, head_dim = query.shape
    if (partial_out.dtype != torch.float32 or not partial_out.is_contiguous()
            or tuple(partial_out.shape) != (rows, query_heads, head_dim)):
        raise ValueError("partial_out must be contiguous fp32 [rows, query_heads, head_dim]")
    if (partial_lse.dtype != torch.float32 or not partial_lse.is_contiguous()
            or tuple(partial_lse.shape) != (rows, query_heads)):
        raise ValueError("partial_lse must be contiguous fp32 [rows, query_heads]")
    device = query.device
    _check_same_device((key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                        token_to_request, partial_out, partial_lse), device)
    if rows == 0:
        return
    topk = logical_indices.shape[1]
    kv_heads = key_data.shape[2]
    lib = _native.load()
    with _device_ctx(device):
        ws_bytes = _workspace_bytes(torch.cuda.current_device(), rows, query_heads, kv_heads, head_dim, topk)
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if ws_bytes else None
        status = lib.nvqsa_sparse_attention_partial(
            query.data_ptr(), query.stride(0), query.stride(1),
            *_cache_args(key_data, key_scale, value_data, value_scale),
            float(key_global_scale), float(value_global_scale),
            logical_indices.data_ptr(), topk,
            block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
            token_to_request.data_ptr(),
            partial_out.data_ptr(), partial_lse.data_ptr(),
            rows, query_heads, head_dim,
            workspace.data_ptr() if workspace is not None else None, ws_bytes, _stream_ptr(device))
    _native.check(status, "qsa_sparse_paged_attention_nvfp4_partial")


def qsa_merge_partials(partial_out, partial_lse, output):
    """Log-sum-exp merge of stacked partials ``[splits, rows, heads, dim]`` into bf16 ``output``."""
    if partial_out.dim() != 4 or partial_out.dtype != torch.float32 or not partial_out.is_contiguous():
        raise ValueError("partial_out must be contiguous fp32 [splits, rows, heads, dim]")
    splits, rows, query_heads, head_dim = partial_out.shape
    if (partial_lse.dtype != torch.float32 or not partial_lse.is_contiguous()
            or tuple(partial_lse.shape) != (splits, rows, query_heads)):
        raise ValueError("partial_lse must be contiguous fp32 [splits, rows, heads]")
    if tuple(output.shape) != (rows, query_heads, head_dim) or output.dtype != torch.bfloat16 or output.stride(-1) != 1:
        raise ValueError("output must be bf16 [rows, heads, dim] with contiguous last dim")
    device = output.device
    _check_same_device((partial_out, partial_lse), device)
    if rows == 0:
        return
    lib = _native.load()
    with _device_ctx(device):
        status = lib.nvqsa_merge_partials(partial_out.data_ptr(), partial_lse.data_ptr(), splits,
                                          output.data_ptr(), output.stride(0), output.stride(1),
                                          rows, query_heads, head_dim, _stream_ptr(device))
    _native.check(status, "qsa_merge_partials")


def qsa_merge_partials_strided(partial_out, partial_lse, output):
    """``qsa_merge_partials`` for partials whose splits are not adjacent.

    ``partial_out`` [splits, rows, heads, dim] and ``partial_lse`` [splits, rows, heads]
    fp32 may have any stride on the split dimension (e.g. views of one gathered
    buffer that packs each rank's outputs and lse together); each split itself
    must be dense.
    """
    if partial_out.dim() != 4 or partial_out.dtype != torch.float32:
        raise ValueError("partial_out must be fp32 [splits, rows, heads, dim]")
    splits, rows, query_heads, head_dim = partial_out.shape
    if partial_lse.dtype != torch.float32 or tuple(partial_lse.shape) != (splits, rows, query_heads):
        raise ValueError("partial_lse must be fp32 [splits, rows, heads]")
    if (partial_out.stride()[1:] != (query_heads * head_dim, head_dim, 1)
            or partial_lse.stride()[1:] != (query_heads, 1)):
        raise ValueError("each split of partial_out / partial_lse must be dense")
    if tuple(output.shape) != (rows, query_heads, head_dim) or output.dtype != torch.bfloat16 or output.stride(-1) != 1:
        raise ValueError("output must be bf16 [rows, heads, dim] with contiguous last dim")
    device = output.device
    _check_same_device((partial_out, partial_lse), device)
    if rows == 0:
        return
    lib = _native.load()
    with _device_ctx(device):
        status = lib.nvqsa_merge_partials_strided(
            partial_out.data_ptr(), partial_out.stride(0), partial_lse.data_ptr(), partial_lse.stride(0), splits,
            output.data_ptr(), output.stride(0), output.stride(1), rows, query_heads, head_dim, _stream_ptr(device))
    _native.check(status, "qsa_merge_partials_strided")


def qsa_sparse_paged_attention_nvfp4_split_kv(
    query,
    key_data,
    key_scale,
    value_data,
    value_scale,
    key_global_scale,
    value_global_scale,
    logical_indices,
    block_table,
    token_to_request,
    output,
    exchange_ptrs,
    world,
    rank,
    parity,
):
    """Split-KV decode of one sequence across GPUs with the exchange fused into the kernel.

    ``exchange_ptrs``: the ``world`` exchange buffers (this rank's and its peers' as mapped here,
    see ``nvfp4_qsa.distributed.PeerExchange``).  Every rank makes the same call with its own cache
    pages and block table and gets the merged bf16 ``output``.
    """
    _check_read(query, key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                token_to_request)
    if output.shape != query.shape or output.dtype != torch.bfloat16 or output.stride(-1) != 1:
        raise ValueError("NVFP4 QSA output must be bf16 shaped like query with contiguous last dim")
    device = query.device
    _check_same_device((key_data, key_scale, value_data, value_scale, logical_indices, block_table,
                        token_to_request, output), device)
    rows, query_heads, head_dim = query.shape
    if rows == 0:
        return
    if len(exchange_ptrs) != world:
        raise ValueError("one exchange buffer per rank is required")
    topk = logical_indices.shape[1]
    kv_heads = key_data.shape[2]
    lib = _native.load()
    ptrs = (ctypes.c_void_p * world)(*exchange_ptrs)
    with _device_ctx(device):
        ws_bytes = _workspace_bytes(torch.cuda.current_device(), rows, query_heads, kv_heads, head_dim, topk)
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if ws_bytes else None
        status = lib.nvqsa_sparse_attention_split_kv(
            query.data_ptr(), query.stride(0), query.stride(1),
            *_cache_args(key_data, key_scale, value_data, value_scale),
            float(key_global_scale), float(value_global_scale),
            logical_indices.data_ptr(), topk,
            block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
            token_to_request.data_ptr(),
            output.data_ptr(), output.stride(0), output.stride(1),
            rows, query_heads, head_dim,
            workspace.data_ptr() if workspace is not None else None, ws_bytes,
            ctypes.cast(ptrs, ctypes.c_void_p), int(world), int(rank), int(parity), _stream_ptr(device))
    _native.check(status, "qsa_sparse_paged_attention_nvfp4_split_kv")
