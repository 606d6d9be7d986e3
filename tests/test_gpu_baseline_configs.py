"""GPU: the reader against the float64 oracle at the full sizes of the benchmark configurations.

The oracle's cost depends only on the selected records, not on the context
length, so these cases keep the configurations' own sizes:

* config 4 (MTP = 3 decode batch): 12 sequences x 4 rows sharing each
  sequence's 2,048 sorted selections, contexts uniform in [8,192, 169,984],
  page 3,136, random block tables -- through the per-row reader and the
  grouped reader (``rows_per_group=4``);
* config 5a (one of the 12 layers of one GPU's shard): 96 sequences x 131,072
  tokens, top-2,048, page 3,136.  Every row is computed on the GPU; the
  oracle checks a sample of 8 sequences, whose blocks are copied out of the
  7.3 GB cache into a compact host copy with a renumbered block table;
* config 5b: one 169,984-token sequence with 8,192 selections -- the
  single-GPU reader, and the split-KV decomposition over 2, 4 and 8 emulated
  ranks (each rank's partial over its own pages, merged by the strided
  log-sum-exp kernel).

Tolerance: tests/gpu_util.py (max-abs 2e-2, mean-abs 2e-3 against float64).
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_attention_close, bits_to_cuda, cuda_to_bits, gpu_write, oracle_attention, regions
from nvfp4_qsa import distributed as D
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu

PAGE = 3136


def _attend(storage, q, idx, bt, t2r, rows_per_group=1):
    kd, ks, vd, vs = regions(storage)
    out = torch.full_like(q, float("nan"))
    kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2r, out,
                                             rows_per_group=rows_per_group)
    return out


def _fill_cache(blocks, seed, device="cuda"):
    """[blocks, 2, PAGE, 288] cache written by the GPU writer from N(0,1) bf16 K/V, in chunks."""
    storage = torch.zeros(blocks, 2, PAGE, 288, dtype=torch.uint8, device=device)
    kd, ks, vd, vs = regions(storage)
    gen = torch.Generator(device=device).manual_seed(seed)
    total, chunk = blocks * PAGE, 1 << 20
    for s0 in range(0, total, chunk):
        n = min(chunk, total - s0)
        kv = torch.randn(2, n, 2, 256, device=device, dtype=torch.bfloat16, generator=gen)
        slots = torch.arange(s0, s0 + n, device=device, dtype=torch.int64)
        kernels.qsa_write_cache_nvfp4(kv[0], kv[1], kd, ks, vd, vs, slots, 1.0, 1.0)
    return storage


@pytest.mark.parametrize("rows_per_group", [1, 4], ids=["per-row", "grouped"])
def test_config4_full_size(rows_per_group):
    contexts, table, blocks, slots, indices, t2r = W.mtp_config(seed=4)  # 12 x 4 rows, U[8192, 169984]
    assert contexts.min() >= 8192 and contexts.max() <= 169984 and indices.shape == (48, 2048)
    toks = int(sum(contexts))
    key = torch.randn(toks, 2, 256, device="cuda", dtype=torch.bfloat16, generator=torch.Generator("cuda").manual_seed(1))
    value = torch.randn(toks, 2, 256, device="cuda", dtype=torch.bfloat16,
                        generator=torch.Generator("cuda").manual_seed(2))
    storage = torch.zeros(blocks, 2, PAGE, 288, dtype=torch.uint8, device="cuda")
    gpu_write(storage, key, value, torch.from_numpy(np.concatenate(slots)).cuda())
    del key, value
    rng = np.random.default_rng(44)
    q = bits_to_cuda(W.f32_to_bf16_bits(rng.standard_normal((48, 24, 256), dtype=np.float32)))
    idx, bt, t2rd = (torch.from_numpy(a).cuda() for a in (indices, table, t2r))
    out = _attend(storage, q, idx, bt, t2rd, rows_per_group)
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_attention(storage, q, idx, bt, t2rd), f"config 4 rows_per_group={rows_per_group}")


def test_config5a_layer_full_size():
    seqs, ctx, topk = 96, 131072, 2048
    width = (ctx + PAGE - 1) // PAGE
    blocks = seqs * width
    storage = _fill_cache(blocks, seed=5)
    gen = torch.Generator(device="cuda").manual_seed(6)
    table = torch.randperm(blocks, device="cuda", generator=gen).to(torch.int32).view(seqs, width).contiguous()
    idx = torch.rand(seqs, ctx, device="cuda", generator=gen).topk(topk, dim=1).indices
    idx = idx.sort(dim=1).values.to(torch.int32).contiguous()
    q = torch.randn(seqs, 24, 256, device="cuda", dtype=torch.bfloat16, generator=gen)
    t2r = torch.arange(seqs, device="cuda", dtype=torch.int32)
    out = _attend(storage, q, idx, table, t2r)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    sample = torch.tensor([0, 1, 17, 42, 63, 77, 94, 95], device="cuda")
    sub_blocks = table[sample].reshape(-1).long()
    compact = storage.index_select(0, sub_blocks)          # the sampled sequences' blocks, in table order
    sub_table = torch.arange(sample.numel() * width, device="cuda", dtype=torch.int32).view(-1, width)
    sub_t2r = torch.arange(sample.numel(), device="cuda", dtype=torch.int32)
    expected = oracle_attention(compact, q[sample], idx[sample], sub_table, sub_t2r)
    assert_attention_close(out[sample], expected, "config 5a layer (8 sampled sequences of 96)")


def _config5b_case():
    return W.decode_config(seed=55, context=169984, topk=8192, page=PAGE, rows=1)


@pytest.fixture(scope="module")
def config5b():
    case = _config5b_case()
    storage = np.zeros((case.blocks, 2, PAGE, 288), np.uint8)
    oracle.write_cache(case.key, case.value, storage, case.slots)
    expected = oracle.sparse_attention(case.query, storage, case.indices, case.block_table, case.token_to_request)
    return case, storage, expected


def test_config5b_single_gpu_full_size(config5b):
    case, storage_np, expected = config5b
    storage = torch.from_numpy(storage_np).cuda()
    q = bits_to_cuda(case.query)
    idx, bt, t2r = (torch.from_numpy(a).cuda() for a in (case.indices, case.block_table, case.token_to_request))
    out = _attend(storage, q, idx, bt, t2r)
    torch.cuda.synchronize()
    assert_attention_close(out, expected, "config 5b one GPU")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config5b_split_kv_full_size(config5b, world):
    # Emulated ranks on one GPU: rank r writes only its own pages (SplitKV.slot_mapping, -1 elsewhere) from the
    # same bf16 K/V, computes its partial over its masked block table, and the strided merge combines them.
    case, _, expected = config5b
    dev = torch.device("cuda")
    pages = (169984 + PAGE - 1) // PAGE
    key, value, q = bits_to_cuda(case.key), bits_to_cuda(case.value), bits_to_cuda(case.query)
    idx = torch.from_numpy(case.indices).to(dev)
    t2r = torch.from_numpy(case.token_to_request).to(dev)
    bufs = []
    for r in range(world):
        sk = D.SplitKV(pages, PAGE, world, r)
        storage = torch.zeros(max(sk.local_blocks, 1), 2, PAGE, 288, dtype=torch.uint8, device=dev)
        kd, ks, vd, vs = regions(storage)
        kernels.qsa_write_cache_nvfp4(key, value, kd, ks, vd, vs, sk.slot_mapping(torch.arange(169984, device=dev)),
                                      1.0, 1.0)
        buf = sk.partial_buffer(1, 24, 256, dev)
        pout, plse = sk.unpack(buf, 1, 24, 256)
        kernels.qsa_sparse_paged_attention_nvfp4_partial(q, kd, ks, vd, vs, 1.0, 1.0, idx, sk.block_table(dev), t2r,
                                                         pout, plse)
        bufs.append(buf)
    outs, lses = D.SplitKV.unpack(torch.stack(bufs), 1, 24, 256)
    merged = torch.empty_like(q)
    kernels.qsa_merge_partials_strided(outs, lses, merged)
    torch.cuda.synchronize()
    assert_attention_close(merged, expected, f"config 5b split over {world} emulated ranks")
    assert not np.array_equal(cuda_to_bits(merged), np.zeros((1, 24, 256), np.uint16))
