"""Multi-GPU decode over one box: one process per GPU, torch.distributed + NCCL.

Two ways to spread the QSA decode over GPUs:

* Independent sequences (``shard_requests``).  Each rank owns whole requests:
  their cache blocks, block-table rows, query rows and their slot of the
  output.  The reader runs alone on every rank; nothing crosses NVLink, so
  the per-GPU work is fixed as ranks are added (weak scaling).

* One long sequence, split-KV across ranks (``SplitKV``).  Rank i owns a
  contiguous range of the sequence's logical pages and holds only those
  pages' cache blocks.  Its block table keeps the sequence's full width with
  -1 in every page it does not own, so the reader's own masking rule
  (python/nvfp4_qsa/kernels.py:241-257: a selection whose physical block is
  negative contributes nothing) restricts each rank to its share of the
  selected indices with no re-indexing and no host synchronisation.  Each
  rank writes an un-merged partial -- softmax-normalised O / value_global_scale
  and the base-2 log-sum-exp per query head, the split-K layout of the
  reference's FP8 sibling (src/qsa_fp8_harness.py:183-208) -- the ranks
  exchange the partials with ONE all_gather of a packed fp32 buffer
  (rows x heads x (head_dim + 1) floats per rank, 24.7 KB for one row), and
  every rank merges the world's partials with the log-sum-exp merge kernel.
  The writer follows the same ownership: ``SplitKV.slot_mapping`` gives -1 for
  tokens on pages another rank owns, and the writer skips negative slots
  (kernels.py:71-77).

Every rank takes the same collective steps in the same order; the exchange is
the only collective on the data path.

``SplitKV.attend`` exchanges the partials with NCCL (all_gather) and merges in
a second kernel.  ``SplitKV.attend_fused`` does the exchange inside the reader
kernel itself over NVLink peer memory: the CTA that finishes this rank's
partial of a (row, kv head) stores it into every rank's exchange buffer
(``PeerExchange``: one buffer per rank, mapped into every process through CUDA
IPC handles exchanged once over the process group), raises a flag there, waits
for the other ranks' flags and merges -- one launch per layer, no NCCL call.
"""
from __future__ import annotations

from dataclasses import dataclass

import ctypes

import torch
import torch.distributed as dist

from . import _native, kernels

__all__ = ["page_range", "shard_requests", "SplitKV", "PeerExchange"]


def page_range(num_pages: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced share [lo, hi) of ``num_pages`` logical pages for ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if num_pages < 0:
        raise ValueError("num_pages must be non-negative")
    base, extra = divmod(num_pages, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_requests(num_requests: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced share [lo, hi) of independent requests for ``rank``."""
    return page_range(num_requests, world, rank)


@dataclass
class SplitKV:
    """One sequence split across ``world`` ranks by logical page ranges.

    ``num_pages`` is the sequence's block-table width (ceil(context / page)).
    The rank owns logical pages [page_lo, page_hi) and stores them in
    ``local_blocks`` cache blocks numbered 0..local_blocks-1 in the order given
    by ``block_order`` (a permutation of the owned pages, e.g. a fragmented
    allocation); identity when omitted.
    """

    num_pages: int
    page_size: int
    world: int
    rank: int
    block_order: torch.Tensor | None = None

    def __post_init__(self):
        if self.page_size < 1:
            raise ValueError("page_size must be positive")
        self.page_lo, self.page_hi = page_range(self.num_pages, self.world, self.rank)
        self.local_blocks = self.page_hi - self.page_lo
        if self.block_order is not None:
            order = torch.as_tensor(self.block_order, dtype=torch.int64).cpu()
            if order.numel() != self.local_blocks or not torch.equal(
                    torch.sort(order).values, torch.arange(self.local_blocks)):
                raise ValueError("block_order must be a permutation of the rank's local blocks")
            self.block_order = order

    def block_table(self, device=None) -> torch.Tensor:
        """int32 [1, num_pages]: local block of each owned page, -1 for pages other ranks own."""
        table = torch.full((1, self.num_pages), -1, dtype=torch.int32)
        owned = torch.arange(self.local_blocks, dtype=torch.int32)
        if self.block_order is not None:
            owned = self.block_order.to(torch.int32)
        table[0, self.page_lo:self.page_hi] = owned
        return table.to(device) if device is not None else table

    def slot_mapping(self, positions: torch.Tensor) -> torch.Tensor:
        """int64 cache slots of logical token ``positions`` on this rank; -1 where another rank owns the page."""
        pos = positions.to(torch.int64)
        page = torch.div(pos, self.page_size, rounding_mode="floor")
        table = self.block_table(pos.device).view(-1).to(torch.int64)
        inside = (pos >= 0) & (page < self.num_pages)
        blk = table[page.clamp(0, max(self.num_pages - 1, 0))]
        slot = blk * self.page_size + (pos - page * self.page_size)
        return torch.where(inside & (blk >= 0), slot, torch.full_like(slot, -1))

    # -- the decode step ------------------------------------------------------------------------------------
    def partial_buffer(self, rows: int, query_heads: int, head_dim: int, device) -> torch.Tensor:
        """Packed fp32 exchange buffer of one rank: [rows * heads * head_dim] outputs, then [rows * heads] lse,
        padded to a multiple of 4 floats so that every rank's outputs stay 16-byte aligned after the gather."""
        n = rows * query_heads * (head_dim + 1)
        return torch.empty((n + 3) // 4 * 4, dtype=torch.float32, device=device)

    @staticmethod
    def unpack(buf: torch.Tensor, rows: int, query_heads: int, head_dim: int):
        """Views (partial_out [rows, heads, dim], partial_lse [rows, heads]) of a packed buffer (last dim)."""
        n_out = rows * query_heads * head_dim
        lead = buf.shape[:-1]
        return (buf[..., :n_out].view(*lead, rows, query_heads, head_dim),
                buf[..., n_out:n_out + rows * query_heads].view(*lead, rows, query_heads))

    def exchange(self, local: torch.Tensor, group=None) -> torch.Tensor:
        """One all_gather of every rank's packed partial: returns [world, buffer] (rank order)."""
        flat = torch.empty(self.world * local.numel(), dtype=local.dtype, device=local.device)
        if self.world == 1:
            flat.copy_(local.reshape(-1))
        else:
            dist.all_gather_into_tensor(flat, local.reshape(-1), group=group)
        return flat.view(self.world, local.numel())

    def attend(self, query, key_data, key_scale, value_data, value_scale, key_global_scale, value_global_scale,
               logical_indices, token_to_request, output, block_table=None, group=None, buffer=None):
        """Split-KV decode of this sequence: local partial, one all_gather, log-sum-exp merge into ``output``.

        ``logical_indices`` is the full selection list of each row (all ranks pass the same); ``block_table``
        defaults to ``self.block_table``.  Collective: every rank of ``group`` must call it.
        """
        rows, query_heads, head_dim = query.shape
        if block_table is None:
            block_table = self.block_table(query.device)
        if buffer is None:
            buffer = self.partial_buffer(rows, query_heads, head_dim, query.device)
        part_out, part_lse = self.unpack(buffer, rows, query_heads, head_dim)
        kernels.qsa_sparse_paged_attention_nvfp4_partial(
            query, key_data, key_scale, value_data, value_scale, key_global_scale, value_global_scale,
            logical_indices, block_table, token_to_request, part_out, part_lse)
        gathered = self.exchange(buffer, group)
        outs, lses = self.unpack(gathered, rows, query_heads, head_dim)
        kernels.qsa_merge_partials_strided(outs, lses, output)
        return output

    def attend_fused(self, query, key_data, key_scale, value_data, value_scale, key_global_scale, value_global_scale,
                      logical_indices, token_to_request, output, exchange: "PeerExchange", block_table=None):
        """Split-KV decode with the exchange and merge fused into the reader kernel (no NCCL call).

        Every rank calls it with the same ``logical_indices`` and its own cache pages; all get ``output``.
        """
        if query.shape[0] != exchange.rows:
            raise ValueError("the exchange buffers were sized for a different number of rows")
        if block_table is None:
            block_table = self.block_table(query.device)
        kernels.qsa_sparse_paged_attention_nvfp4_split_kv(
            query, key_data, key_scale, value_data, value_scale, key_global_scale, value_global_scale,
            logical_indices, block_table, token_to_request, output, exchange.ptrs, exchange.world, exchange.rank,
            exchange.next_parity())
        return output


class PeerExchange:
    """Per-rank exchange buffers for ``SplitKV.attend_fused``, mapped on every rank.

    Collective (every rank of ``group`` constructs it with the same ``rows``).  Holds this
    rank's buffer (``nvqsa_exchange_alloc``) and the peers' buffers opened from their CUDA IPC
    handles, plus the parity that alternates from call to call.  ``close()`` unmaps and frees.
    """

    def __init__(self, rows: int, query_heads: int, kv_heads: int, group=None, device=None):
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("the fused split-KV exchange supports at most 8 ranks")
        self.rows = rows
        self.lib = _native.load()
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = device
        with torch.cuda.device(device):
            size = ctypes.c_size_t()
            _native.check(self.lib.nvqsa_split_kv_exchange_bytes(rows, query_heads, kv_heads, self.world,
                                                                ctypes.byref(size)), "exchange size")
            local = ctypes.c_void_p()
            _native.check(self.lib.nvqsa_exchange_alloc(size.value, ctypes.byref(local)), "exchange alloc")
            self._local = local.value
            handle = (ctypes.c_ubyte * 64)()
            _native.check(self.lib.nvqsa_ipc_get_handle(ctypes.c_void_p(self._local), handle), "ipc handle")
            handles = [bytes(handle)]
            if self.world > 1:
                gathered = [None] * self.world
                dist.all_gather_object(gathered, bytes(handle), group=group)
                handles = gathered
            self._opened = []
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._local)
                    continue
                buf = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                peer = ctypes.c_void_p()
                _native.check(self.lib.nvqsa_ipc_open_handle(buf, ctypes.byref(peer)), "ipc open")
                self._opened.append(peer.value)
                ptrs.append(peer.value)
            self.ptrs = ptrs
        self.parity = 0

    def next_parity(self) -> int:
        p = self.parity
        self.parity ^= 1
        return p

    def close(self):
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for ptr in self._opened:
                self.lib.nvqsa_ipc_close_handle(ctypes.c_void_p(ptr))
            self._opened = []
            if self._local:
                self.lib.nvqsa_exchange_free(ctypes.c_void_p(self._local))
                self._local = None
