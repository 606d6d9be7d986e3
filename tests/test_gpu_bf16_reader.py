"""GPU: the BF16 sibling reader (nvqsa_sparse_attention_bf16) against the reference and the oracle.

The reference's forward_qsa sends a bf16 main cache to vLLM's
qsa_sparse_paged_attention (integration/snapshot/qsa.py:352-366).  The caches
here are laid out as vLLM allocates them, bf16 [blocks, kv_heads, page, 2*256]
split into K and V views [blocks, page, kv_heads, 256].  Checked against the
reference's own qsa_reference outputs (tests/golden/bf16_attention_cases.npz)
and, at larger sizes, against the float64 oracle, under the reader tolerance
of tests/gpu_util.py; split plans, masked and duplicate selections, pages of
16 and 3,136 tokens and graph replay are covered.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_attention_close, bits_to_cuda, cuda_to_bits
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _views(storage):
    cache = storage.transpose(1, 2)  # [blocks, page, kv_heads, 512]
    return cache[..., :256], cache[..., 256:]


def _oracle(q, storage, idx, bt, t2r):
    bits = cuda_to_bits(storage).transpose(0, 2, 1, 3)
    return oracle.sparse_attention_bf16(cuda_to_bits(q), bits[..., :256], bits[..., 256:], idx.cpu().numpy(),
                                        bt.cpu().numpy(), t2r.cpu().numpy())


def _case(seed, contexts, rows_per_req, topk, page, dist="normal"):
    rng = np.random.default_rng(seed)
    table, blocks, _ = W.paged_requests(rng, contexts, page, extra_blocks=1)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    storage = torch.randn(blocks, 2, page, 512, device="cuda", dtype=torch.bfloat16, generator=gen)
    if dist == "outliers":
        storage[..., 7::61] *= 16
    rows = len(contexts) * rows_per_req
    idx = np.full((rows, topk), -1, np.int32)
    for r in range(rows):
        ctx = int(contexts[r // rows_per_req])
        sel = np.sort(rng.choice(ctx, size=min(topk, ctx), replace=False))
        idx[r, :sel.size] = sel
    t2r = np.repeat(np.arange(len(contexts), dtype=np.int32), rows_per_req)
    q = bits_to_cuda(W.f32_to_bf16_bits(W.gen_values(rng, (rows, 24, 256), "normal")))
    return storage, q, torch.from_numpy(idx).cuda(), torch.from_numpy(table).cuda(), torch.from_numpy(t2r).cuda()


def _attend(storage, q, idx, bt, t2r):
    kc, vc = _views(storage)
    out = torch.full_like(q, float("nan"))
    kernels.qsa_sparse_paged_attention(q, kc, vc, idx, bt, t2r, out)
    torch.cuda.synchronize()
    return out


def test_bf16_golden_cases_match_reference(bf16_attention_cases):
    data, names = bf16_attention_cases
    for name in names:
        storage = bits_to_cuda(data[f"{name}__kv"])
        q = bits_to_cuda(data[f"{name}__q"])
        idx, bt, t2r = (torch.from_numpy(data[f"{name}__{k}"]).cuda() for k in ("indices", "block_table", "t2r"))
        out = _attend(storage, q, idx, bt, t2r)
        assert_attention_close(out, data[f"{name}__expected"], name)


@pytest.mark.parametrize("contexts,rows_per_req,topk,page", [
    ([32768], 1, 2048, 16),          # config 2 shape: one row, many splits (clusters + workspace merge)
    ([169984], 1, 8192, 3136),       # config 5b shape: one row, 8,192 selections
    ([9000, 5000, 20000], 2, 2048, 3136),
    ([4096] * 12, 4, 2048, 3136),    # MTP-like batch (rows of a request share nothing here)
    ([3000] * 96, 1, 2048, 3136),    # config 5a row count: 2 splits per unit in clusters
    ([700] * 5, 1, 1000, 16),        # topk not a multiple of 8: a partial last tile
    ([40] * 3, 2, 70, 16),           # topk > context: padded with -1
])
def test_bf16_reader_matches_oracle(contexts, rows_per_req, topk, page):
    storage, q, idx, bt, t2r = _case(len(contexts) * 7 + topk, contexts, rows_per_req, topk, page)
    out = _attend(storage, q, idx, bt, t2r)
    assert_attention_close(out, _oracle(q, storage, idx, bt, t2r), f"bf16 {len(contexts)}x{rows_per_req} {topk}")


def test_bf16_masked_duplicate_and_invalid_requests():
    storage, q, idx, bt, t2r = _case(91, [500, 600], 2, 256, 16, dist="outliers")
    idx[0, :3] = torch.tensor([-1, 10 ** 6, 2 ** 31 - 1], dtype=torch.int32)
    idx[1, :] = 5            # one token selected in every column
    idx[2, :] = -1           # nothing valid -> zeros
    t2r[3] = 7               # request out of range -> zeros
    out = _attend(storage, q, idx, bt, t2r)
    assert_attention_close(out, _oracle(q, storage, idx, bt, t2r), "bf16 masked")
    assert not out[2].any().item() and not out[3].any().item()


def test_bf16_reader_inside_cuda_graph():
    storage, q, idx, bt, t2r = _case(17, [8000, 6000], 3, 2048, 3136)
    kc, vc = _views(storage)
    eager = _attend(storage, q, idx, bt, t2r)
    out = torch.zeros_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qsa_sparse_paged_attention(q, kc, vc, idx, bt, t2r, out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.qsa_sparse_paged_attention(q, kc, vc, idx, bt, t2r, out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_bf16_reader_rejects_non_bf16_caches():
    storage, q, idx, bt, t2r = _case(5, [64], 1, 16, 16)
    kc, vc = _views(storage)
    with pytest.raises(NotImplementedError):
        kernels.qsa_sparse_paged_attention(q, kc.float(), vc.float(), idx, bt, t2r)
