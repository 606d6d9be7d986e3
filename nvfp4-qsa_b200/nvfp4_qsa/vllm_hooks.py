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

__all__ = ["split_nvfp4_kv_cache", "QSANVFP4AttentionHooks", "write_nvfp4_kv"]


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


class QSANVFP4AttentionHooks:
    """Mixin for a vLLM attention impl whose main KV cache is NVFP4.

    Expects the impl attributes vLLM sets: ``head_size``, ``alibi_slopes``,
    ``sinks`` and ``sliding_window``; the layer carries ``topk_indices_buffer``
    (int32 [max_tokens, topk], filled by the QSA indexer) and the fixed global
    scales ``_qsa_nvfp4_k_global`` / ``_qsa_nvfp4_v_global`` (1.0 when absent).
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
