"""GPU: the FP8 sibling reader (nvqsa_sparse_attention_fp8) against the oracle.

The reference's FP8 variant of the QSA decode kernel (src/qsa_fp8_harness.py:42-208)
reads float8_e4m3 K and V caches [blocks, page, kv_heads, head_dim] with
per-tensor scales: k_scale multiplies the scores, v_scale the output.  The
oracle restates it in float64 (oracle.sparse_attention_fp8); the GPU output must
match within the reader tolerance for every split plan the planner picks, with
masked, duplicate and tail selections, the strided K/V views vLLM cuts from its
cache, and under CUDA-graph replay.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_attention_close, bits_to_cuda, cuda_to_bits
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _caches(blocks, page, kvh, seed, vllm_layout=False):
    g = torch.Generator("cuda").manual_seed(seed)
    if vllm_layout:
        # vLLM's fp8 main cache: one tensor [blocks, kv_heads, page, 2*hd], K and V cut as strided views
        raw = (torch.randn(blocks, kvh, page, 512, device="cuda", generator=g) * 2).to(torch.float8_e4m3fn)
        kc, vc = raw.transpose(1, 2).split(256, dim=-1)
    else:
        kc = (torch.randn(blocks, page, kvh, 256, device="cuda", generator=g) * 2).to(torch.float8_e4m3fn)
        vc = (torch.randn(blocks, page, kvh, 256, device="cuda", generator=g) * 2).to(torch.float8_e4m3fn)
    return kc, vc


def _expected(q, kc, vc, idx, bt, t2r, ks, vs):
    kb = kc.contiguous().view(torch.uint8).cpu().numpy()
    vb = vc.contiguous().view(torch.uint8).cpu().numpy()
    return oracle.sparse_attention_fp8(cuda_to_bits(q), kb, vb, idx.cpu().numpy(), bt.cpu().numpy(),
                                       t2r.cpu().numpy(), ks, vs)


def _case(rows, topk, ctx, page, seed, nreq=None, vllm_layout=False):
    rng = np.random.default_rng(seed)
    nreq = nreq or min(rows, 4)
    width = (ctx + page - 1) // page
    blocks = nreq * width
    table = rng.permutation(blocks).astype(np.int32).reshape(nreq, width)
    kc, vc = _caches(blocks, page, 2, seed, vllm_layout)
    idx = np.stack([np.sort(rng.choice(ctx, size=min(topk, ctx), replace=False)) for _ in range(rows)]).astype(np.int32)
    t2r = (np.arange(rows) % nreq).astype(np.int32)
    q = bits_to_cuda(W.f32_to_bf16_bits(rng.standard_normal((rows, 24, 256), dtype=np.float32)))
    return q, kc, vc, torch.from_numpy(idx).cuda(), torch.from_numpy(table).cuda(), torch.from_numpy(t2r).cuda()


CASES = [  # (rows, topk, ctx, page)
    (1, 2048, 32768, 3136),    # one row: many splits, clusters of 8 and the global merge
    (3, 4096, 9000, 256),      # small batch, 32 splits
    (80, 2048, 3000, 256),     # 160 units: 2 splits in clusters of 2
    (20, 1000, 5000, 16),      # topk not a multiple of 16: a partial last tile; 16-token pages
]


@pytest.mark.parametrize("rows,topk,ctx,page", CASES, ids=[f"rows{c[0]}-topk{c[1]}-page{c[3]}" for c in CASES])
def test_fp8_reader_matches_oracle(rows, topk, ctx, page):
    q, kc, vc, idx, bt, t2r = _case(rows, topk, ctx, page, seed=rows * 131 + topk)
    out = kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, 1.0, 1.0, idx, bt, t2r)
    torch.cuda.synchronize()
    assert_attention_close(out, _expected(q, kc, vc, idx, bt, t2r, 1.0, 1.0), f"fp8 rows={rows} topk={topk}")


def test_fp8_scales_and_vllm_strided_views():
    # per-tensor scales fold into the scores and the output; K and V are strided views of one cache tensor
    q, kc, vc, idx, bt, t2r = _case(6, 2048, 8000, 3136, seed=5, vllm_layout=True)
    assert kc.stride() != kc.contiguous().stride()
    for ks, vs in ((0.35, 1.7), (2.5, 0.125)):
        out = torch.full_like(q, float("nan"))
        kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, ks, vs, idx, bt, t2r, out)
        torch.cuda.synchronize()
        assert_attention_close(out, _expected(q, kc, vc, idx, bt, t2r, ks, vs), f"fp8 scales {ks} {vs}")


def test_fp8_masked_and_duplicate_selections():
    q, kc, vc, idx, bt, t2r = _case(8, 2048, 6000, 256, seed=9, nreq=2)
    idx = idx.clone()
    bt = bt.clone()
    t2r = t2r.clone()
    idx[0, :300] = -1                 # negative indices
    idx[1, 100:400] = 10 ** 7         # pages past the table width
    bt[1, 3] = -1                     # a page mapped to no block
    bt[1, 5] = 10 ** 6                # a block past the cache
    idx[2, :] = idx[2, :1]            # every selection the same token
    t2r[3] = 7                        # a request past the table: the row is zeros
    idx[4, :] = -1                    # no valid selection: zeros
    out = kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, 1.0, 1.0, idx, bt, t2r)
    torch.cuda.synchronize()
    exp = _expected(q, kc, vc, idx, bt, t2r, 1.0, 1.0)
    assert_attention_close(out, exp, "fp8 masked")
    assert not out[3].float().any() and not out[4].float().any()


def test_fp8_reader_inside_cuda_graph():
    q, kc, vc, idx, bt, t2r = _case(2, 4096, 9000, 3136, seed=13)
    out = torch.zeros_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, 1.0, 1.0, idx, bt, t2r, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, 1.0, 1.0, idx, bt, t2r, out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert_attention_close(out, _expected(q, kc, vc, idx, bt, t2r, 1.0, 1.0), "fp8 graph replay")
    del g


def test_fp8_wrapper_rejects_bad_inputs():
    q, kc, vc, idx, bt, t2r = _case(2, 256, 4000, 256, seed=3)
    with pytest.raises(ValueError, match="float8"):
        kernels.qsa_sparse_paged_attention_fp8(q, kc.view(torch.uint8), vc, 1.0, 1.0, idx, bt, t2r)
    with pytest.raises(ValueError, match="int32"):
        kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, 1.0, 1.0, idx.long(), bt, t2r)
    with pytest.raises(Exception):
        kernels.qsa_sparse_paged_attention_fp8(q, kc, vc, 0.0, 1.0, idx, bt, t2r)  # scales must be positive
    from nvfp4_qsa import _native
    assert _native.read_error_flags() == 0
