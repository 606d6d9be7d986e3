"""GPU: the grouped (MTP) reader, nvqsa_sparse_attention_grouped.

Rows in groups of ``rows_per_group`` that share their request and selections
(the draft rows of a multi-token-prediction step) are served by one gather and
one dequantisation per record.  The result must equal the oracle within the
reader tolerance and the per-row reader's output, whether or not the groups
really share: each CTA checks its share of the index positions on the device
and processes a group that does not share row by row.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_attention_close, bits_to_cuda, gpu_write, oracle_attention, regions
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _mtp_case(seed, sequences, rows_per_seq, ctx_lo, ctx_hi, topk, heads=24):
    contexts, table, blocks, slots, indices, t2r = W.mtp_config(seed=seed, sequences=sequences,
                                                                rows_per_seq=rows_per_seq, ctx_lo=ctx_lo,
                                                                ctx_hi=ctx_hi, topk=topk)
    toks = int(sum(contexts))
    key = torch.randn(toks, 2, 256, device="cuda", dtype=torch.bfloat16,
                      generator=torch.Generator("cuda").manual_seed(seed))
    value = torch.randn(toks, 2, 256, device="cuda", dtype=torch.bfloat16,
                        generator=torch.Generator("cuda").manual_seed(seed + 1))
    storage = torch.zeros(blocks, 2, 3136, 288, dtype=torch.uint8, device="cuda")
    gpu_write(storage, key, value, torch.from_numpy(np.concatenate(slots)).cuda())
    rng = np.random.default_rng(seed + 2)
    rows = indices.shape[0]
    q = bits_to_cuda(W.f32_to_bf16_bits(rng.standard_normal((rows, heads, 256), dtype=np.float32)))
    return storage, q, indices, table, t2r


def _attend(storage, q, idx, bt, t2r, rows_per_group):
    kd, ks, vd, vs = regions(storage)
    out = torch.full_like(q, float("nan"))
    kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2r, out,
                                             rows_per_group=rows_per_group)
    return out


def _check(storage, q, indices, table, t2r, rows_per_group, what):
    idx, bt, t2rd = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (indices, table, t2r))
    grouped = _attend(storage, q, idx, bt, t2rd, rows_per_group)
    per_row = _attend(storage, q, idx, bt, t2rd, 1)
    torch.cuda.synchronize()
    assert torch.isfinite(grouped.float()).all(), what
    assert_attention_close(grouped, oracle_attention(storage, q, idx, bt, t2rd), what)
    assert (grouped.float() - per_row.float()).abs().max().item() <= 2e-2, what
    return grouped


@pytest.mark.parametrize("sequences,rows_per_seq,topk", [
    (12, 4, 2048),   # config 4 (MTP = 3), contexts reduced for the oracle
    (5, 4, 1000),    # topk not a multiple of 16: a partial last tile
    (6, 2, 2048),    # groups of two rows
    (4, 3, 4096),    # groups of three, 4 splits per group
    (3, 4, 8192),    # 8 splits (one cluster of 8) per group
])
def test_grouped_reader_matches_oracle_and_per_row(sequences, rows_per_seq, topk):
    storage, q, indices, table, t2r = _mtp_case(40 + rows_per_seq, sequences, rows_per_seq, max(4096, topk + 1000),
                                                 20000, topk)
    _check(storage, q, indices, table, t2r, rows_per_seq, f"grouped {sequences}x{rows_per_seq} topk={topk}")


@pytest.mark.parametrize("heads,rows_per_seq", [(16, 4), (32, 3), (2, 4)])
def test_grouped_reader_head_counts_and_strided_output(heads, rows_per_seq):
    # 8, 16 and 1 query heads per kv head; the output in a padded buffer (row stride not a multiple of 8)
    storage, q, indices, table, t2r = _mtp_case(90 + heads, 5, rows_per_seq, 4096, 15000, 2048, heads=heads)
    idx, bt, t2rd = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (indices, table, t2r))
    kd, ks, vd, vs = regions(storage)
    buf = torch.full((q.shape[0], heads, 260), float("nan"), dtype=torch.bfloat16, device="cuda")
    out = buf[..., :256]
    kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2rd, out,
                                             rows_per_group=rows_per_seq)
    torch.cuda.synchronize()
    assert torch.isnan(buf[..., 256:].float()).all()
    assert_attention_close(out.contiguous(), oracle_attention(storage, q, idx, bt, t2rd), f"heads {heads}")


def test_grouped_reader_ragged_last_group():
    # 10 rows in groups of 4: the last group has two rows
    storage, q, indices, table, t2r = _mtp_case(51, 5, 2, 4096, 12000, 2048)
    _check(storage, q, indices, table, t2r, 4, "ragged")


def test_groups_that_do_not_share_are_processed_row_by_row():
    storage, q, indices, table, t2r = _mtp_case(61, 6, 4, 4096, 12000, 2048)
    indices = indices.copy()
    t2r = t2r.copy()
    # group 0: row 2 differs in one index (one split's chunks only) -> that cluster falls back
    indices[2, 700] = (indices[2, 700] + 1) % 4096
    # group 1: rows have different requests with the same indices
    t2r[5] = t2r[0]
    # group 2: every row has its own selection list
    rng = np.random.default_rng(3)
    for rr in range(8, 12):
        indices[rr] = np.sort(rng.choice(4096, size=2048, replace=False))
    _check(storage, q, indices, table, t2r, 4, "mixed sharing")


def test_grouped_reader_masked_selections():
    storage, q, indices, table, t2r = _mtp_case(71, 4, 4, 4096, 9000, 2048)
    indices = indices.copy()
    indices[0:4, :100] = -1                  # negative indices (shared by the group)
    indices[4:8, 100:300] = 10 ** 7          # pages past the table width
    indices[8:12, :] = indices[8:12, :1]     # duplicates: every selection the same token
    _check(storage, q, indices, table, t2r, 4, "masked")


def test_grouped_reader_inside_cuda_graph():
    storage, q, indices, table, t2r = _mtp_case(81, 12, 4, 4096, 12000, 2048)
    idx, bt, t2rd = (torch.from_numpy(a).cuda() for a in (indices, table, t2r))
    kd, ks, vd, vs = regions(storage)
    out = torch.zeros_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2rd, out, rows_per_group=4)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2rd, out, rows_per_group=4)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_attention(storage, q, idx, bt, t2rd), "grouped graph replay")
    del g


def test_grouped_entry_rejects_bad_group_size():
    storage, q, indices, table, t2r = _mtp_case(91, 2, 4, 4096, 6000, 256)
    idx, bt, t2rd = (torch.from_numpy(a).cuda() for a in (indices, table, t2r))
    with pytest.raises(Exception):
        _attend(storage, q, idx, bt, t2rd, 5)
    from nvfp4_qsa import _native
    assert _native.read_error_flags() == 0
