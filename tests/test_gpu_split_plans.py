"""GPU: every split-KV plan of the reader against the oracle.

The reader splits each (row, kv head)'s selections over S CTAs.  With
2 <= S <= 8 the S CTAs form one thread-block cluster and rank 0 merges the
others' partials over distributed shared memory; with S > 8 the partials go
to the caller's workspace and the last CTA to arrive merges them; S = 1 is
unsplit.  The plan follows from rows x kv_heads against the SM count and from
topk (at most 1024 selections per CTA), so these cases pick batch shapes that
land on each plan, plus the partial (un-merged) entry point in cluster mode.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_attention_close, bits_to_cuda, gpu_attend, gpu_write, oracle_attention
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def _expected_splits(rows, topk, sms):
    chunks = max(1, -(-topk // 32))
    min_splits = -(-chunks // 32)
    units = rows * 2
    splits = min_splits
    if units < sms:
        splits = -(-sms // units)
    else:
        fill = 3 * sms // units
        while fill & (fill - 1):
            fill &= fill - 1
        splits = max(splits, fill)
    return max(min(splits, chunks), min_splits)


def _case(rows, topk, ctx, page, seed):
    """`rows` decode rows over min(rows, 4) requests of `ctx` tokens each, `topk` sorted selections per row."""
    rng = np.random.default_rng(seed)
    nreq = min(rows, 4)
    table, blocks, req_slots = W.paged_requests(rng, [ctx] * nreq, page)
    key = W.f32_to_bf16_bits(W.gen_values(rng, (nreq * ctx, 2, 256), "normal"))
    value = W.f32_to_bf16_bits(W.gen_values(rng, (nreq * ctx, 2, 256), "normal"))
    q = W.f32_to_bf16_bits(W.gen_values(rng, (rows, 24, 256), "normal"))
    idx = np.stack([np.sort(rng.choice(ctx, size=min(topk, ctx), replace=False)) for _ in range(rows)])
    idx = idx.astype(np.int32)
    storage = torch.zeros(blocks, 2, page, 288, dtype=torch.uint8, device="cuda")
    gpu_write(storage, bits_to_cuda(key), bits_to_cuda(value), torch.from_numpy(np.concatenate(req_slots)).cuda())
    return (storage, bits_to_cuda(q), torch.from_numpy(idx).cuda(), torch.from_numpy(table).cuda(),
            torch.from_numpy((np.arange(rows) % nreq).astype(np.int32)).cuda())


PLANS = [  # (rows, topk): the split count on a 148-SM B200 in the comment
    (80, 256),    # units 160 >= SMs, 1 split: unsplit
    (80, 2048),   # 2 splits: cluster of 2
    (25, 1024),   # units 50 -> 3 splits: cluster of 3
    (19, 1024),   # units 38 -> 4 splits: cluster of 4
    (15, 2048),   # units 30 -> 5 splits: cluster of 5
    (10, 4096),   # units 20 -> 8 splits: cluster of 8
    (80, 8192),   # 8 splits from the 1024-per-CTA limit: cluster of 8
    (3, 4096),    # units 6 -> 25 splits: global workspace, last CTA merges
    (1, 2048),    # units 2 -> 64 splits (one 32-index chunk each): global workspace
    (74, 2048),   # units 148 = SMs: 3 splits would be clusters of 3; 2 splits, cluster of 2
    (96, 3072),   # 96 chunks: 3 splits without a cluster (big batch), merged through the workspace
]


@pytest.mark.parametrize("rows,topk", PLANS, ids=[f"rows{r}-topk{t}" for r, t in PLANS])
def test_split_plan_matches_oracle(rows, topk):
    storage, q, idx, table, t2r = _case(rows, topk, ctx=max(topk + 512, 3000), page=256, seed=rows * 7919 + topk)
    out = gpu_attend(storage, q, idx, table, t2r)
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_attention(storage, q, idx, table, t2r),
                           f"rows={rows} topk={topk} splits={_expected_splits(rows, topk, _sms())}")


@pytest.mark.parametrize("rows,topk", [(25, 1024), (3, 4096)])
def test_partial_entry_point_in_cluster_and_workspace_plans(rows, topk):
    storage, q, idx, table, t2r = _case(rows, topk, ctx=2 * topk, page=256, seed=99 + rows)
    from gpu_util import regions
    kd, ks, vd, vs = regions(storage)
    po = torch.full((rows, 24, 256), float("nan"), device="cuda")
    pl = torch.full((rows, 24), float("nan"), device="cuda")
    kernels.qsa_sparse_paged_attention_nvfp4_partial(q, kd, ks, vd, vs, 1.0, 1.0, idx, table, t2r, po, pl)
    merged = torch.empty_like(q)
    kernels.qsa_merge_partials(po.unsqueeze(0).contiguous(), pl.unsqueeze(0).contiguous(), merged)
    torch.cuda.synchronize()
    assert torch.isfinite(po).all() and torch.isfinite(pl).all()
    assert_attention_close(merged, oracle_attention(storage, q, idx, table, t2r), f"partial rows={rows}")


def test_cluster_plan_inside_cuda_graph():
    storage, q, idx, table, t2r = _case(25, 1024, ctx=3000, page=256, seed=5)
    out = torch.zeros_like(q)
    from gpu_util import regions
    kd, ks, vd, vs = regions(storage)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, table, t2r, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, table, t2r, out)
    out.zero_()
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_attention(storage, q, idx, table, t2r), "graph replay")
    del g
