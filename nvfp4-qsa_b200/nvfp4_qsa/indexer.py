"""QSA indexer top-k: fill the reader's selection buffer on the GPU.

The reference's QSA layer calls its indexer with the layer's
``topk_indices_buffer[:num_tokens]`` (int32 [num_tokens, output_width]) and
checks that the selection comes back in that shape
(integration/snapshot/qsa.py:537-545, :605-616); the reader then takes it as
``logical_indices``.  The indexer module is not vendored in the reference, so
this module provides the selection step to that contract on the C-ABI kernel
``nvqsa_topk_indices``: given the indexer's per-token scores over the context,
the ``output_width`` highest-scoring positions of each token's causal context.
"""
from __future__ import annotations

import torch

from . import _native
from .kernels import _device_ctx, _stream_ptr

__all__ = ["qsa_select_topk"]


def qsa_select_topk(scores: torch.Tensor, topk_indices_buffer: torch.Tensor,
                    lengths: torch.Tensor | None = None) -> torch.Tensor:
    """Write each row's top-k positions into ``topk_indices_buffer`` and return it.

    ``scores``: fp32 [num_tokens, context] (last dim contiguous), the indexer's score of every context position
    for every query token.  ``topk_indices_buffer``: int32 [num_tokens, k] (last dim contiguous), k = the
    indexer's output width.  ``lengths``: optional int32 [num_tokens], the causal context of each token (positions
    >= lengths[i] are never selected); all ``context`` positions when omitted.  Row i receives the indices of its
    k largest scores in ascending order; ties at the k-th value go to the lowest indices; NaN ranks highest; a
    row with fewer than k valid positions gets 0 .. len - 1 followed by -1 (masked by the reader).
    """
    if scores.dim() != 2 or scores.dtype != torch.float32 or scores.stride(-1) != 1:
        raise ValueError("QSA indexer scores must be fp32 [num_tokens, context] with contiguous last dim")
    out = topk_indices_buffer
    if out.dim() != 2 or out.dtype != torch.int32 or out.stride(-1) != 1:
        raise ValueError("QSA top-k buffer must be int32 [num_tokens, output_width] with contiguous last dim")
    if out.shape[0] != scores.shape[0]:
        raise RuntimeError("QSA indexer returned an invalid selection shape")
    if lengths is not None and (lengths.dtype != torch.int32 or lengths.dim() != 1 or not lengths.is_contiguous()
                                or lengths.shape[0] < scores.shape[0]):
        raise ValueError("QSA indexer lengths must be contiguous int32 [num_tokens]")
    device = scores.device
    for t in (out,) + ((lengths,) if lengths is not None else ()):
        if t.device != device:
            raise ValueError("QSA indexer tensors must be on one device")
    rows, context = scores.shape
    k = out.shape[1]
    if rows == 0:
        return out
    lib = _native.load()
    with _device_ctx(device):
        status = lib.nvqsa_topk_indices(scores.data_ptr(), scores.stride(0),
                                        lengths.data_ptr() if lengths is not None else None, rows, context, k,
                                        out.data_ptr(), out.stride(0), _stream_ptr(device))
    _native.check(status, "qsa_select_topk")
    return out
