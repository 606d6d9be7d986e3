"""The NVFP4 branches of the vLLM QSA attention backend, on the sm_100a kernels.

The reference's vLLM integration patch reaches this path from two hooks; both
keep their signatures, argument handling and errors here and call the C-ABI
kernels through ``nvfp4_qsa.kernels`` instead of Triton:

* ``QSANVFP4AttentionHooks.forward_qsa`` -- the attention impl's
  ``forward_qsa`` (integration/snapshot/qsa.py:263-321; public port
  integration/public/qsa.py:192-206) with its NVFP4 branch (snapshot/qsa.py:294-321):
  reject unsupported features, zero the output, take the layer's top-k buffer,
  split the uint8 cache into its four regions and run the sparse reader.
* ``write_nvfp4_kv`` -- the NVFP4 write branch of ``_run_qsa``
  (integration/snapshot/qsa.py:618-640; public/qsa.py:465-477): split the same
  cache and run the writer with the layer's fixed global scales.

The cache tensor is vLLM's [num_blocks, kv_heads, block_size, 2 * (head_size/2 +
head_size/16)] uint8 allocation: one 288-byte record (K data | K scales | V data
| V scales) per (block, kv head, token) for head_size 256.
"""
from __future__ import annotations

import torch

from . import kernels

__all__ = ["split_nvfp4_kv_cache", "QSANVFP4AttentionHooks", "write_nvfp4_kv", "is_qsa_nvfp4_dtype",
           "nvfp4_storage_dim", "nvfp4_kv_cache_spec_fields", "customize_nvfp4_spec", "nvfp4_page_bytes"]

# ---------------------------------------------------------------------------
# Cache planner accounting: the NVFP4 parts of the backend's spec methods
# (integration/snapshot/qsa.py:66-68, :187-204 and :556-566), as plain host
# arithmetic so that a serving stack sizes its pages for the 288-byte record.
# ---------------------------------------------------------------------------


def is_qsa_nvfp4_dtype(dtype) -> bool:
    """True for the QSA-owned packed E2M1 + group-scale cache dtypes (snapshot/qsa.py:66-68)."""
    return isinstance(dtype, str) and dtype in ("nvfp4", "nvfp4_4over6")


def nvfp4_storage_dim(head_dim: int) -> int:
    """Bytes of one packed K (or V) region per (token, kv head): head_dim/2 codes + head_dim/16 scales."""
    if head_dim <= 0 or head_dim % 16:
        raise ValueError(f"NVFP4 head_dim must be a positive multiple of 16, got {head_dim}")
    return head_dim // 2 + head_dim // 16


def nvfp4_kv_cache_spec_fields(block_size: int, num_kv_heads: int, head_dim: int) -> dict:
    """Fields of the per-layer cache spec the backend reports for an NVFP4 cache (snapshot/qsa.py:556-566).

    The physical width replaces the logical head size for both K and V and the
    element type is uint8, so the planner allocates [blocks, kv_heads, block_size,
    2 * storage_dim] bytes per layer (the layout ``split_nvfp4_kv_cache`` cuts).
    The reference also passes vLLM's "auto" quant mode: QSA owns writer and reader.
    """
    storage_dim = nvfp4_storage_dim(head_dim)
    return {"block_size": int(block_size), "num_kv_heads": int(num_kv_heads), "head_size": storage_dim,
            "head_size_v": storage_dim, "dtype": torch.uint8}


def customize_nvfp4_spec(spec, nvfp4_quant_mode):
    """``customize_spec`` of the backend (snapshot/qsa.py:187-204) for any dataclass spec.

    A spec whose ``kv_quant_mode`` is ``nvfp4_quant_mode`` still carries the
    logical ``head_size``; the packed K + V bytes per head slot are advertised
    through ``state_content_bytes`` (the spec multiplies by ``num_kv_heads``
    itself).  Any other spec is returned unchanged, so applying it to the final
    physical spec (quant mode "auto", 144-byte regions) is a no-op.
    """
    import dataclasses

    if getattr(spec, "kv_quant_mode", None) != nvfp4_quant_mode:
        return spec
    return dataclasses.replace(spec, state_content_bytes=2 * nvfp4_storage_dim(spec.head_size))


def nvfp4_page_bytes(block_size: int, num_kv_heads: int, head_dim: int) -> int:
    """Bytes of one cache block of one layer: block_size x kv_heads records of 2 * storage_dim bytes."""
    return int(block_size) * int(num_kv_heads) * 2 * nvfp4_storage_dim(head_dim)


def split_nvfp4_kv_cache(kv_cache: torch.Tensor, head_size: int):
    """(key_data, key_scale, value_data, value_scale) views of a vLLM NVFP4 QSA cache (snapshot/qsa.py:295-306)."""
    packed_dim = head_size // 2
    scale_dim = head_size // 16
    storage_dim = packed_dim + scale_dim
    if kv_cache.dtype != torch.uint8 or kv_cache.shape[-1] != 2 * storage_dim:
        raise RuntimeError(
            "QSA NVFP4 cache must be uint8 with packed data and fp8 "
            f"group scales (last dim {2 * storage_dim})"
        )
    packed_cache = kv_cache.transpose(1, 2)
    key_region, value_region = packed_cache.split(storage_dim, dim=-1)
    key_data, key_scale = key_region.split((packed_dim, scale_dim), dim=-1)
    value_data, value_scale = value_region.split((packed_dim, scale_dim), dim=-1)
    return key_data, key_scale, value_data, value_scale


def canonicalize_singleton_dim_strides(t: torch.Tensor) -> torch.Tensor:
    """The same view with every size-1 dim given the stride it would have in a dense layout.

    A size-1 dim is never stepped over, so its stride carries no information, but the readers check every
    stride for 16-byte alignment; vLLM applies the same normalisation before its QSA kernels
    (snapshot/qsa.py:323-325).
    """
    strides = list(t.stride())
    inner = 1
    for i in range(t.dim() - 1, -1, -1):
        if t.shape[i] == 1:
            strides[i] = inner
        inner = strides[i] * t.shape[i]
    return t.as_strided(t.shape, strides)


class QSANVFP4AttentionHooks:
    """Mixin for a vLLM attention impl of the QSA backend (snapshot/qsa.py:263-366).

    Expects the impl attributes vLLM sets: ``head_size``, ``alibi_slopes``,
    ``sinks`` and ``sliding_window``; the layer carries ``topk_indices_buffer``
    (int32 [max_tokens, topk], filled by the QSA indexer).  The main cache is
    NVFP4 unless the impl sets ``_qsa_kv_nvfp4 = False`` (fixed global scales
    ``_qsa_nvfp4_k_global`` / ``_qsa_nvfp4_v_global``, 1.0 when absent); then
    a uint8 cache with ``_qsa_kv_fp8`` goes to the FP8 sibling reader (layer
    ``_k_scale_float`` / ``_v_scale_float``) and a bf16 cache to the BF16 one.
    """

    def forward_qsa(
        self,
        layer: torch.nn.Module,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        kv_cache: torch.Tensor,
        attn_metadata,
        output: torch.Tensor,
        token_to_req: torch.Tensor,
        output_scale: torch.Tensor | None = None,
        output_block_scale: torch.Tensor | None = None,
    ) -> torch.Tensor:
        del key, value  # the cache was written by write_nvfp4_kv before this call
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("QSA does not support fused output quantization")
        if self.alibi_slopes is not None or self.sinks is not None:
            raise NotImplementedError("QSA does not support ALiBi or attention sinks")
        if self.sliding_window != (-1, -1):
            raise NotImplementedError("QSA does not support sliding-window attention")

        num_tokens = attn_metadata.num_actual_tokens
        output.zero_()
        if num_tokens == 0:
            return output

        topk_buffer = getattr(layer, "topk_indices_buffer", None)
        if topk_buffer is None:
            raise RuntimeError("QSA owner did not provide its top-k buffer")
        logical_indices = topk_buffer[:num_tokens]
        token_to_req = token_to_req[:num_tokens]
        if getattr(self, "_qsa_kv_nvfp4", True):
            key_data, key_scale, value_data, value_scale = split_nvfp4_kv_cache(kv_cache, self.head_size)
            kernels.qsa_sparse_paged_attention_nvfp4(
                query[:num_tokens],
                key_data,
                key_scale,
                value_data,
                value_scale,
                float(getattr(layer, "_qsa_nvfp4_k_global", 1.0)),
                float(getattr(layer, "_qsa_nvfp4_v_global", 1.0)),
                logical_indices,
                attn_metadata.block_table,
                token_to_req,
                output[:num_tokens],
            )
            return output

        # The BF16 and FP8 main caches (snapshot/qsa.py:323-366): K and V halves of the last dim.
        key_cache, value_cache = kv_cache.transpose(1, 2).split(self.head_size, dim=-1)
        key_cache = canonicalize_singleton_dim_strides(key_cache)
        value_cache = canonicalize_singleton_dim_strides(value_cache)
        if getattr(self, "_qsa_kv_fp8", False) and key_cache.dtype == torch.uint8:
            if query.dtype != torch.bfloat16:
                raise NotImplementedError("Qwen3.8-Flash-Next QSA requires a BF16 query")
            kernels.qsa_sparse_paged_attention_fp8(
                query[:num_tokens],
                key_cache.view(torch.float8_e4m3fn),
                value_cache.view(torch.float8_e4m3fn),
                float(getattr(layer, "_k_scale_float", 1.0)),
                float(getattr(layer, "_v_scale_float", 1.0)),
                logical_indices,
                attn_metadata.block_table,
                token_to_req,
                output[:num_tokens],
            )
            return output
        if key_cache.dtype != torch.bfloat16 or query.dtype != torch.bfloat16:
            raise NotImplementedError("Qwen3.8-Flash-Next QSA requires BF16 Q/K/V")
        kernels.qsa_sparse_paged_attention(
            query[:num_tokens],
            key_cache,
            value_cache,
            logical_indices,
            attn_metadata.block_table,
            token_to_req,
            output[:num_tokens],
        )
        return output


def write_nvfp4_kv(kv_cache: torch.Tensor, head_dim: int, key: torch.Tensor, value: torch.Tensor,
                   slot_mapping: torch.Tensor, key_global_scale: float, value_global_scale: float) -> None:
    """The NVFP4 write of ``_run_qsa``: quantise this step's K/V into the cache at ``slot_mapping``."""
    key_data, key_scale, value_data, value_scale = split_nvfp4_kv_cache(kv_cache, head_dim)
    kernels.qsa_write_cache_nvfp4(
        key,
        value,
        key_data,
        key_scale,
        value_data,
        value_scale,
        slot_mapping,
        float(key_global_scale),
        float(value_global_scale),
    )
