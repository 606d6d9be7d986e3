"""GPU: split-KV decode of one sequence across ranks, the kernels of nvfp4_qsa.distributed.

On one GPU the ranks are emulated in turn: rank r writes only its own pages
into its own cache (``SplitKV.slot_mapping`` gives -1 elsewhere and the writer
skips those slots), computes its un-merged partial over its masked block table
(``SplitKV.block_table``), the packed partials are stacked as the all_gather
would leave them, and the strided log-sum-exp merge kernel combines them.  The
result must match the oracle's unsplit attention within the reader tolerance
and the single-GPU reader's output.  The NCCL exchange itself is covered by the
gloo tests in tests/test_distributed_cpu.py and by ``bench.py --gpus N``.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_attention_close
from nvfp4_qsa import distributed as D
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _bits(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


def _regions(storage):
    parts = storage.transpose(1, 2).split(144, dim=-1)
    kd, ks = parts[0].split((128, 16), dim=-1)
    vd, vs = parts[1].split((128, 16), dim=-1)
    return kd, ks, vd, vs


@pytest.mark.parametrize("world,context,topk,page,rows", [
    (2, 9000, 1024, 3136, 1),     # pages split 2/1
    (4, 20000, 2048, 3136, 2),    # 7 pages over 4 ranks, two rows
    (8, 30000, 4096, 256, 1),     # many small pages, 8 ranks
    (3, 700, 96, 16, 3),          # a rank may own no selection of a row
])
def test_split_kv_ranks_merge_to_the_unsplit_result(world, context, topk, page, rows):
    dev = torch.device("cuda")
    case = W.decode_config(seed=50 + world, context=context, topk=topk, page=page, rows=rows)
    pages = (context + page - 1) // page
    key, value = _bits(case.key, dev), _bits(case.value, dev)
    q = _bits(case.query, dev)
    idx = torch.from_numpy(case.indices).to(dev)
    t2r = torch.from_numpy(case.token_to_request).to(dev)
    qh, hd = q.shape[1], q.shape[2]

    bufs = []
    for r in range(world):
        sk = D.SplitKV(pages, page, world, r,
                       block_order=torch.randperm(D.page_range(pages, world, r)[1] - D.page_range(pages, world, r)[0],
                                                  generator=torch.Generator().manual_seed(r)))
        storage = torch.zeros(max(sk.local_blocks, 1), 2, page, 288, dtype=torch.uint8, device=dev)
        kd, ks, vd, vs = _regions(storage)
        slots = sk.slot_mapping(torch.arange(context, device=dev))
        kernels.qsa_write_cache_nvfp4(key, value, kd, ks, vd, vs, slots, 1.0, 1.0)
        buf = sk.partial_buffer(rows, qh, hd, dev)
        pout, plse = sk.unpack(buf, rows, qh, hd)
        kernels.qsa_sparse_paged_attention_nvfp4_partial(q, kd, ks, vd, vs, 1.0, 1.0, idx, sk.block_table(dev), t2r,
                                                         pout, plse)
        bufs.append(buf)
    gathered = torch.stack(bufs)  # what all_gather_into_tensor leaves, viewed [world, buffer]
    outs, lses = D.SplitKV.unpack(gathered, rows, qh, hd)
    merged = torch.empty_like(q)
    kernels.qsa_merge_partials_strided(outs, lses, merged)
    torch.cuda.synchronize()

    storage_all = np.zeros((case.blocks, 2, page, 288), np.uint8)
    oracle.write_cache(case.key, case.value, storage_all, case.slots)
    expected = oracle.sparse_attention(case.query, storage_all, case.indices, case.block_table, case.token_to_request)
    assert_attention_close(merged, expected, "split-kv")

    # and the same as the one-GPU reader on the whole cache
    full = torch.from_numpy(storage_all).to(dev)
    single = torch.empty_like(q)
    kernels.qsa_sparse_paged_attention_nvfp4(q, *_regions(full), 1.0, 1.0, idx,
                                             torch.from_numpy(case.block_table).to(dev), t2r, single)
    torch.cuda.synchronize()
    assert (merged.float() - single.float()).abs().max().item() <= 2e-2


def test_strided_merge_rejects_overlapping_splits():
    dev = torch.device("cuda")
    outs = torch.zeros(2, 1, 24, 256, device=dev)
    lses = torch.zeros(2, 1, 24, device=dev)
    out = torch.empty(1, 24, 256, dtype=torch.bfloat16, device=dev)
    overlapping = outs.view(-1)[: 24 * 256 + 16].as_strided((2, 1, 24, 256), (16, 24 * 256, 256, 1))
    with pytest.raises(ValueError):
        kernels.qsa_merge_partials_strided(overlapping, lses, out)


@pytest.mark.parametrize("rows,topk", [(1, 8192), (1, 2048), (3, 4096), (40, 2048)])
def test_fused_exchange_single_rank_matches_the_reader(rows, topk):
    # world = 1: the fused path stores this rank's slot, waits for no peer and merges one slot;
    # called three times so that both flag parities are used and re-armed.
    dev = torch.device("cuda")
    context = topk + 1000
    case = W.decode_config(seed=70 + rows, context=context, topk=topk, page=3136, rows=rows)
    storage = torch.zeros(case.blocks, 2, case.page, 288, dtype=torch.uint8, device=dev)
    regs = _regions(storage)
    kernels.qsa_write_cache_nvfp4(_bits(case.key, dev), _bits(case.value, dev), *regs,
                                  torch.from_numpy(case.slots).to(dev), 1.0, 1.0)
    q = _bits(case.query, dev)
    idx = torch.from_numpy(case.indices).to(dev)
    bt = torch.from_numpy(case.block_table).to(dev)
    t2r = torch.from_numpy(case.token_to_request).to(dev)
    expected = torch.empty_like(q)
    kernels.qsa_sparse_paged_attention_nvfp4(q, *regs, 1.0, 1.0, idx, bt, t2r, expected)
    pages = (context + case.page - 1) // case.page
    sk = D.SplitKV(pages, case.page, 1, 0)
    ex = D.PeerExchange(rows, 24, 2)
    try:
        for _ in range(3):
            out = torch.full_like(q, float("nan"))
            sk.attend_fused(q, *regs, 1.0, 1.0, idx, t2r, out, ex, block_table=bt)
            torch.cuda.synchronize()
            assert torch.isfinite(out.float()).all()
            assert (out.float() - expected.float()).abs().max().item() <= 2e-2
    finally:
        ex.close()
    from nvfp4_qsa import _native
    assert _native.read_error_flags() == 0


def test_peer_wait_times_out_and_reports_without_a_fault():
    # Failure detection without a GPU fault: a two-rank exchange where rank 1 never runs.  Rank 0's
    # kernel stores its slot, raises its flag in the (local stand-in) peer buffer, waits for rank 1's
    # flag that nothing sets, gives up after its 2 s limit, raises device error bit 1 and leaves the
    # output untouched; the context stays usable.
    import ctypes
    from nvfp4_qsa import _native

    dev = torch.device("cuda")
    lib = _native.load()
    case = W.decode_config(seed=90, context=4000, topk=512, page=256, rows=1)
    storage = torch.zeros(case.blocks, 2, case.page, 288, dtype=torch.uint8, device=dev)
    regs = _regions(storage)
    kernels.qsa_write_cache_nvfp4(_bits(case.key, dev), _bits(case.value, dev), *regs,
                                  torch.from_numpy(case.slots).to(dev), 1.0, 1.0)
    q = _bits(case.query, dev)
    idx = torch.from_numpy(case.indices).to(dev)
    bt = torch.from_numpy(case.block_table).to(dev)
    t2r = torch.from_numpy(case.token_to_request).to(dev)
    size = ctypes.c_size_t()
    _native.check(lib.nvqsa_split_kv_exchange_bytes(1, 24, 2, 2, ctypes.byref(size)), "size")
    bufs = []
    for _ in range(2):
        ptr = ctypes.c_void_p()
        _native.check(lib.nvqsa_exchange_alloc(size.value, ctypes.byref(ptr)), "alloc")
        bufs.append(ptr.value)
    try:
        _native.read_error_flags(clear=True)
        out = torch.full_like(q, 7.0)
        kernels.qsa_sparse_paged_attention_nvfp4_split_kv(q, *regs, 1.0, 1.0, idx, bt, t2r, out, bufs, 2, 0, 0)
        torch.cuda.synchronize()
        assert _native.read_error_flags(clear=True) & 2
        assert (out.float() == 7.0).all()  # nothing stored after the timeout
        # the context is still usable: an ordinary call afterwards is correct
        ok = torch.empty_like(q)
        kernels.qsa_sparse_paged_attention_nvfp4(q, *regs, 1.0, 1.0, idx, bt, t2r, ok)
        torch.cuda.synchronize()
        assert torch.isfinite(ok.float()).all()
        assert _native.read_error_flags() == 0
    finally:
        for b in bufs:
            lib.nvqsa_exchange_free(ctypes.c_void_p(b))


def test_timing_stamps_are_ordered_and_leave_the_result_unchanged():
    # The opt-in %globaltimer stamps (nvqsa_set_stamp_buffer) on a split plan that merges through the workspace:
    # entry <= tiles done <= last part in <= local merge <= stored, and the output equals the unstamped launch.
    dev = torch.device("cuda")
    case = W.decode_config(seed=77, context=20000, topk=4096, page=3136, rows=1)
    storage = torch.zeros(case.blocks, 2, case.page, 288, dtype=torch.uint8, device=dev)
    regs = _regions(storage)
    kernels.qsa_write_cache_nvfp4(_bits(case.key, dev), _bits(case.value, dev), *regs,
                                  torch.from_numpy(case.slots).to(dev), 1.0, 1.0)
    q = _bits(case.query, dev)
    idx, bt, t2r = (torch.from_numpy(a).to(dev) for a in (case.indices, case.block_table, case.token_to_request))
    plain = torch.empty_like(q)
    kernels.qsa_sparse_paged_attention_nvfp4(q, *regs, 1.0, 1.0, idx, bt, t2r, plain)
    stamps = torch.zeros(2, kernels.STAMP_SLOTS, dtype=torch.int64, device=dev)
    kernels.reset_stamps(stamps)
    kernels.set_stamp_buffer(stamps)
    try:
        out = torch.empty_like(q)
        kernels.qsa_sparse_paged_attention_nvfp4(q, *regs, 1.0, 1.0, idx, bt, t2r, out)
    finally:
        kernels.set_stamp_buffer(None)
    torch.cuda.synchronize()
    assert torch.equal(out, plain)
    st = stamps.cpu()
    for u in range(2):
        s0, s1, s2, s3, s6 = (int(st[u, i]) for i in (0, 1, 2, 3, 6))
        assert 0 < s0 <= s1 <= s2 <= s3 <= s6, st[u].tolist()
