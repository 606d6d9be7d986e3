"""CPU: host logic of the multi-GPU decode (nvfp4_qsa.distributed).

* page / request sharding covers every page once and balances the ranks;
* SplitKV's block table and slot mapping give each page to exactly one rank;
* world_size-2 gloo ranks run the split-KV exchange end to end on the CPU: each
  rank writes only its own pages (oracle writer, skipping the -1 slots
  ``SplitKV.slot_mapping`` gives it), computes its un-merged partial with the
  oracle reader over its block table, exchanges the packed partials with
  ``SplitKV.exchange`` (one all_gather), unpacks them with ``SplitKV.unpack``,
  and the log-sum-exp merge of the gathered partials equals the oracle's
  unsplit attention over the whole sequence.
The GPU kernels of the same path are checked in tests/test_gpu_split_kv.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from nvfp4_qsa import distributed as D
from nvfp4_qsa import workloads as W


@pytest.mark.parametrize("pages,world", [(0, 1), (1, 2), (7, 2), (55, 4), (55, 8), (42, 3)])
def test_page_range_partitions_every_page_once(pages, world):
    got = [D.page_range(pages, world, r) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == pages
    for (lo0, hi0), (lo1, _) in zip(got, got[1:]):
        assert hi0 == lo1
    sizes = [hi - lo for lo, hi in got]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        D.page_range(pages, world, world)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_split_kv_tables_and_slots_give_each_page_one_owner(world):
    pages, page = 11, 5
    ctx = pages * page - 3
    owners = np.zeros(pages, np.int64)
    positions = torch.arange(-2, ctx + 4)
    seen = torch.zeros(positions.numel(), dtype=torch.int64)
    for r in range(world):
        order = torch.randperm(D.page_range(pages, world, r)[1] - D.page_range(pages, world, r)[0],
                               generator=torch.Generator().manual_seed(r))
        sk = D.SplitKV(pages, page, world, r, block_order=order)
        table = sk.block_table()
        assert table.shape == (1, pages) and table.dtype == torch.int32
        own = table[0] >= 0
        owners += own.numpy()
        assert torch.equal(torch.sort(table[0][own]).values, torch.arange(sk.local_blocks, dtype=torch.int32))
        slots = sk.slot_mapping(positions)
        mine = slots >= 0
        seen += mine.to(torch.int64)
        # owned slots land in the rank's own blocks at the token's offset
        p = positions[mine]
        assert torch.equal(slots[mine] % page, p % page)
        assert torch.equal(slots[mine] // page, table[0][p // page].to(torch.int64))
    assert (owners == 1).all()
    valid = (positions >= 0) & (positions < pages * page)
    assert torch.equal(seen, valid.to(torch.int64))


def test_split_kv_rejects_a_bad_block_order():
    with pytest.raises(ValueError):
        D.SplitKV(6, 4, 2, 0, block_order=torch.tensor([0, 0, 1]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    case = W.decode_config(seed=41, context=700, topk=96, page=16, rows=2)
    pages = (700 + 15) // 16
    return case, pages


def _rank_main(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case, pages = _case()
        sk = D.SplitKV(pages, case.page, world, rank)
        storage = np.zeros((max(sk.local_blocks, 1), 2, case.page, 288), np.uint8)
        positions = torch.arange(case.key.shape[0])
        slots = sk.slot_mapping(positions).numpy()
        oracle.write_cache(case.key, case.value, storage, slots)
        out, lse = oracle.sparse_attention(case.query, storage, case.indices, sk.block_table().numpy(),
                                           case.token_to_request, return_lse=True)
        rows, qh, hd = out.shape
        buf = sk.partial_buffer(rows, qh, hd, "cpu")
        pout, plse = sk.unpack(buf, rows, qh, hd)
        pout.copy_(torch.from_numpy(out))
        plse.copy_(torch.from_numpy(lse))
        gathered = sk.exchange(buf)
        outs, lses = sk.unpack(gathered, rows, qh, hd)
        merged = oracle.merge_partials(outs.numpy(), lses.numpy())
        np.save(os.path.join(result_dir, f"merged_{rank}.npy"), merged)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_split_kv_exchange_and_merge_match_unsplit_attention(world, tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    case, pages = _case()
    storage = np.zeros((case.blocks, 2, case.page, 288), np.uint8)
    oracle.write_cache(case.key, case.value, storage, case.slots)
    expected = oracle.sparse_attention(case.query, storage, case.indices, case.block_table, case.token_to_request)
    for r in range(world):
        got = np.load(tmp_path / f"merged_{r}.npy")
        np.testing.assert_allclose(got, expected, rtol=0, atol=2e-6)


def test_merge_of_one_rank_with_no_valid_selection_ignores_it():
    # a rank that owns none of a row's selections reports lse = -inf; the merge skips it
    outs = np.stack([np.full((1, 2, 4), 7.0, np.float32), np.full((1, 2, 4), 3.0, np.float32)])
    lses = np.stack([np.full((1, 2), -np.inf, np.float32), np.zeros((1, 2), np.float32)])
    np.testing.assert_allclose(oracle.merge_partials(outs, lses), 3.0)
    lses_empty = np.full((2, 1, 2), -np.inf, np.float32)
    assert not oracle.merge_partials(outs, lses_empty).any()
