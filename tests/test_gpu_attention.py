"""GPU: the sm_100a QSA sparse reader vs the reference's outputs and the pinned oracle.

Tolerance (north star): max-abs <= 2e-2 and mean-abs <= 2e-3 against a
float64 reference over the same dequantized K/V.  Ports the reference's
reader tests (tests/test_gpu_portable.py:33-65), its 27-cell boundary matrix
(src/boundary_matrix.py:36-57) and adversarial indices (src/sanitizer_target.py:17-22).
"""
import numpy as np
import pytest
import torch

from gpu_util import (assert_attention_close, bits_to_cuda, build_case_on_gpu, gpu_attend, gpu_write,
                      oracle_attention, regions, sha)
from nvfp4_qsa import PackedCache, kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def test_golden_attention_cases(attention_cases):
    data, names = attention_cases
    for name in names:
        storage = torch.from_numpy(data[f"{name}__storage"]).cuda()
        q = bits_to_cuda(data[f"{name}__q"])
        idx = torch.from_numpy(data[f"{name}__indices"]).cuda()
        bt = torch.from_numpy(data[f"{name}__block_table"]).cuda()
        t2r = torch.from_numpy(data[f"{name}__t2r"]).cuda()
        gk, gv = (float(s) for s in data[f"{name}__scales"])
        out = gpu_attend(storage, q, idx, bt, t2r, gk, gv)
        assert_attention_close(out, data[f"{name}__expected"], name)


def test_decode_config_matches_reference(decode_golden):
    # 1 row x 24 heads, 32,768-token cache written by the GPU writer, 2,048 sorted indices.
    case = W.decode_config(seed=2)
    storage, q, idx, bt, t2r = build_case_on_gpu(case)
    assert sha(storage) == str(decode_golden["storage_sha256"])
    out = gpu_attend(storage, q, idx, bt, t2r)
    mx, mean = assert_attention_close(out, decode_golden["expected"], "decode_config")
    assert mx < 5e-3


def test_invalid_attention_metadata_returns_finite_zero():
    # reference tests/test_gpu_portable.py:33-41
    cache = PackedCache(1)
    query = torch.ones(3, 24, 256, device="cuda", dtype=torch.bfloat16)
    indices = torch.tensor([[-1, 999], [-1, -1], [0, 1]], device="cuda", dtype=torch.int32)
    blocks = torch.tensor([[0]], device="cuda", dtype=torch.int32)
    requests = torch.tensor([0, 0, 99], device="cuda", dtype=torch.int32)
    result = cache.attend(query, indices, blocks, requests)
    assert torch.isfinite(result).all().item()
    assert not result.any().item()


def test_sparse_attention_fragmented_pages_against_cpu_dense():
    # reference tests/test_gpu_portable.py:43-65 (same tolerance, float32 dense softmax)
    torch.manual_seed(37)
    cache = PackedCache(4)
    key = torch.randn(32, 2, 256, device="cuda", dtype=torch.bfloat16)
    value = torch.randn_like(key)
    slots = torch.cat((torch.arange(32, 48), torch.arange(0, 16))).long().cuda()
    cache.write(key, value, slots)
    query = torch.randn(2, 24, 256, device="cuda", dtype=torch.bfloat16)
    indices = torch.tensor([[0, 5, 12, 17, 31], [1, 8, 15, 16, 29]], device="cuda", dtype=torch.int32)
    blocks = torch.tensor([[2, 0]], device="cuda", dtype=torch.int32)
    output = cache.attend(query, indices, blocks, torch.zeros(2, device="cuda", dtype=torch.int32)).cpu().float()
    from nvfp4_qsa import decode

    def decoded(data, scales):
        out = decode(data.contiguous().reshape(-1, 128), scales.contiguous().reshape(-1, 16),
                     torch.tensor(1.), 256).bfloat16().float().cpu()
        return out.reshape(4, 16, 2, 256)

    kd, vd = decoded(cache.kd, cache.ks), decoded(cache.vd, cache.vs)
    expected = []
    for row in range(2):
        logical = indices[row].cpu().long()
        physical = blocks[0].cpu().long()[logical // 16]
        k = kd[physical, logical % 16].repeat_interleave(12, dim=1)
        v = vd[physical, logical % 16].repeat_interleave(12, dim=1)
        logits = torch.einsum("hd,thd->ht", query[row].cpu().float(), k) / 16
        expected.append(torch.einsum("ht,thd->hd", logits.softmax(-1), v))
    torch.testing.assert_close(output, torch.stack(expected), rtol=.02, atol=.025)


def _cell(ctx, rows, topk, dist, frag=False, nreq=1, dup=False, page=16, seed=7, gk=1.0, gv=1.0):
    """Boundary cell built like src/run_validation.py:57-101, checked against the oracle."""
    rng = np.random.default_rng(seed + ctx + 31 * topk + rows)
    table, blocks, req_slots = W.paged_requests(rng, [ctx] * nreq, page, fragmented=frag)
    toks = nreq * ctx
    key = W.f32_to_bf16_bits(W.gen_values(rng, (toks, 2, 256), dist))
    value = W.f32_to_bf16_bits(W.gen_values(rng, (toks, 2, 256), dist))
    q = W.f32_to_bf16_bits(W.gen_values(rng, (rows, 24, 256), dist))
    idx = np.full((rows, topk), -1, np.int32)
    for r in range(rows):
        pos = max(1, (r + 1) * ctx // max(rows, 1))
        avail = min(pos, ctx)
        forced = np.array([f for f in (0, 1, page - 1, page, page + 1, avail - 1) if 0 <= f < avail])
        if avail <= topk:
            sel = np.arange(avail)
        else:
            sel = np.unique(np.concatenate([forced, rng.permutation(avail)[: topk - forced.size]]))[:topk]
        idx[r, : sel.size] = sel
    if dup and topk >= 2:
        idx[0, :] = 5
    t2r = (np.arange(rows) % nreq).astype(np.int32)
    storage = torch.zeros(blocks, 2, page, 288, dtype=torch.uint8, device="cuda")
    gpu_write(storage, bits_to_cuda(key), bits_to_cuda(value), torch.from_numpy(np.concatenate(req_slots)).cuda(),
              gk, gv)
    qd, idxd = bits_to_cuda(q), torch.from_numpy(idx).cuda()
    btd, t2rd = torch.from_numpy(table).cuda(), torch.from_numpy(t2r).cuda()
    out = gpu_attend(storage, qd, idxd, btd, t2rd, gk, gv)
    exp = oracle_attention(storage, qd, idxd, btd, t2rd, gk, gv)
    return assert_attention_close(out, exp, f"ctx={ctx} rows={rows} topk={topk} {dist}")


BOUNDARY_CELLS = (
    [dict(ctx=c, rows=4, topk=min(2051, c), dist="normal") for c in (1, 15, 16, 17, 1024, 8192, 32768)]
    + [dict(ctx=1024, rows=4, topk=1024, dist=d) for d in ("zeros", "normal", "heavytail", "outliers")]
    + [dict(ctx=2048, rows=q, topk=2051, dist="normal") for q in (1, 2, 3, 4)]
    + [dict(ctx=1024, rows=4, topk=1024, dist="normal", nreq=b) for b in (1, 2, 4)]
    + [dict(ctx=8192, rows=4, topk=t, dist="normal") for t in (512, 1024, 2050, 2051, 2052)]
    + [dict(ctx=2048, rows=4, topk=2051, dist="normal", frag=True),
       dict(ctx=8192, rows=8, topk=2051, dist="heavytail", frag=True, nreq=2),
       dict(ctx=2048, rows=4, topk=2051, dist="normal", dup=True),
       dict(ctx=17, rows=4, topk=17, dist="outliers")]
)


@pytest.mark.parametrize("cell", BOUNDARY_CELLS, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
def test_boundary_matrix(cell):
    _cell(**cell)


@pytest.mark.parametrize("cell", [dict(ctx=9000, rows=4, topk=2048, dist="normal", page=3136, frag=True, nreq=3),
                                  dict(ctx=3137, rows=2, topk=300, dist="heavytail", page=3136),
                                  dict(ctx=5000, rows=3, topk=64, dist="normal", page=3136, gk=3.5, gv=0.25)],
                         ids=["page3136-multireq", "page3136-boundary", "page3136-gscale"])
def test_large_pages(cell):
    _cell(**cell)


def test_adversarial_indices():
    # src/sanitizer_target.py:17-22: -1, ctx+999, 2^31-1, an all-masked row
    case = W.decode_config(seed=5, context=256, topk=64, rows=2)
    case.indices[0, :3] = [-1, 256 + 999, 2 ** 31 - 1]
    case.indices[1, :] = -1
    storage, q, idx, bt, t2r = build_case_on_gpu(case)
    out = gpu_attend(storage, q, idx, bt, t2r)
    exp = oracle_attention(storage, q, idx, bt, t2r)
    assert_attention_close(out, exp, "adversarial")
    assert not out[1].any().item()


def test_mtp_batch_against_oracle():
    # MTP=3 structure: 12 sequences x 4 rows sharing indices, page 3136 (contexts reduced for the oracle).
    contexts, table, blocks, slots, indices, t2r = W.mtp_config(seed=4, ctx_lo=4096, ctx_hi=20000, topk=2048)
    rng = np.random.default_rng(44)
    toks = int(sum(contexts))
    key = torch.randn(toks, 2, 256, device="cuda", dtype=torch.bfloat16,
                      generator=torch.Generator("cuda").manual_seed(1))
    value = torch.randn(toks, 2, 256, device="cuda", dtype=torch.bfloat16,
                        generator=torch.Generator("cuda").manual_seed(2))
    storage = torch.zeros(blocks, 2, 3136, 288, dtype=torch.uint8, device="cuda")
    gpu_write(storage, key, value, torch.from_numpy(np.concatenate(slots)).cuda())
    q = bits_to_cuda(W.f32_to_bf16_bits(rng.standard_normal((48, 24, 256), dtype=np.float32)))
    idx, bt, t2rd = (torch.from_numpy(a).cuda() for a in (indices, table, t2r))
    out = gpu_attend(storage, q, idx, bt, t2rd)
    exp = oracle_attention(storage, q, idx, bt, t2rd)
    assert_attention_close(out, exp, "mtp")


def test_partial_merge_equals_full():
    # Split-KV across devices, emulated on one GPU: each "device" sees only its pages.
    case = W.decode_config(seed=8, context=8192, topk=2048, rows=3)
    storage, q, idx, bt, t2r = build_case_on_gpu(case)
    full = gpu_attend(storage, q, idx, bt, t2r)
    kd, ks, vd, vs = regions(storage)
    parts, lses = [], []
    width = bt.shape[1]
    for shard in range(3):
        lo, hi = shard * width // 3, (shard + 1) * width // 3
        local = torch.full_like(bt, -1)
        local[:, lo:hi] = bt[:, lo:hi]
        po = torch.empty(3, 24, 256, dtype=torch.float32, device="cuda")
        pl = torch.empty(3, 24, dtype=torch.float32, device="cuda")
        kernels.qsa_sparse_paged_attention_nvfp4_partial(q, kd, ks, vd, vs, 1.0, 1.0, idx, local, t2r, po, pl)
        parts.append(po)
        lses.append(pl)
    merged = torch.empty_like(q)
    kernels.qsa_merge_partials(torch.stack(parts), torch.stack(lses), merged)
    diff = (merged.float() - full.float()).abs()
    assert diff.max().item() < 4e-3


def test_read_inside_cuda_graph():
    case = W.decode_config(seed=12, context=4096, topk=512, rows=5)
    storage, q, idx, bt, t2r = build_case_on_gpu(case)
    eager = gpu_attend(storage, q, idx, bt, t2r)
    kd, ks, vd, vs = regions(storage)
    out = torch.zeros_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2r, out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2r, out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_size_independent_properties():
    # Checks without an oracle at config 2's full size: selection order, duplicating every
    # selection, masked selections (negative / past the table) and row replication leave
    # the softmax output unchanged.
    case = W.decode_config(seed=13, context=32768, topk=2048, rows=2)
    storage, q, idx, bt, t2r = build_case_on_gpu(case)
    base = gpu_attend(storage, q, idx, bt, t2r).float()
    perm = idx[:, torch.randperm(idx.shape[1], device="cuda")].contiguous()
    assert (gpu_attend(storage, q, perm, bt, t2r).float() - base).abs().max().item() < 2e-3
    doubled = torch.cat([idx, idx], dim=1).contiguous()
    assert (gpu_attend(storage, q, doubled, bt, t2r).float() - base).abs().max().item() < 2e-3
    masked = torch.cat([torch.full_like(idx, -1), idx, torch.full_like(idx, 1 << 30)], dim=1).contiguous()
    assert (gpu_attend(storage, q, masked, bt, t2r).float() - base).abs().max().item() < 2e-3  # masked = absent
    q_rep = q[:1].repeat(6, 1, 1).contiguous()
    rep = gpu_attend(storage, q_rep, idx[:1].repeat(6, 1).contiguous(), bt, t2r[:1].repeat(6).contiguous())
    assert torch.equal(rep, rep[:1].expand_as(rep))  # identical rows -> identical bits
    assert (rep[:1].float() - base[:1]).abs().max().item() < 2e-3


def test_raw_reader_rejects_bad_metadata_types():
    st = torch.zeros(1, 2, 16, 288, dtype=torch.uint8, device="cuda")
    kd, ks, vd, vs = regions(st)
    q = torch.zeros(1, 24, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="int32"):
        kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0,
                                                 torch.zeros(1, 4, dtype=torch.int64, device="cuda"),
                                                 torch.zeros(1, 1, dtype=torch.int32, device="cuda"),
                                                 torch.zeros(1, dtype=torch.int32, device="cuda"), torch.empty_like(q))


def test_no_device_error_flags_raised():
    from nvfp4_qsa import _native
    torch.cuda.synchronize()
    assert _native.read_error_flags(clear=True) == 0


@pytest.mark.parametrize("record", [289, 290, 292, 296])
def test_reader_takes_strides_that_are_not_16_byte_multiples(record):
    # The reference's raw op takes any block/token/head strides with a contiguous last dim
    # (python/nvfp4_qsa/kernels.py:376-391): records padded to 289/290/292/296 bytes give strides whose widest
    # common alignment is 1/2/4/8 bytes; the reader copies them with plain loads of that width.
    case = W.decode_config(seed=60 + record, context=5000, topk=700, page=64, rows=3)
    compact = torch.zeros(case.blocks, 2, case.page, 288, dtype=torch.uint8, device="cuda")
    gpu_write(compact, bits_to_cuda(case.key), bits_to_cuda(case.value), torch.from_numpy(case.slots).cuda())
    padded = torch.zeros(case.blocks, 2, case.page, record, dtype=torch.uint8, device="cuda")
    view = padded[..., :288]
    view.copy_(compact)
    kd, ks, vd, vs = regions(view)
    assert kd.stride(1) == record
    q = bits_to_cuda(case.query)
    idx, bt, t2r = (torch.from_numpy(a).cuda() for a in (case.indices, case.block_table, case.token_to_request))
    out = torch.full_like(q, float("nan"))
    kernels.qsa_sparse_paged_attention_nvfp4(q, kd, ks, vd, vs, 1.0, 1.0, idx, bt, t2r, out)
    assert_attention_close(out, oracle_attention(compact, q, idx, bt, t2r), f"record {record}")
    aligned = gpu_attend(compact, q, idx, bt, t2r)
    assert (out.float() - aligned.float()).abs().max().item() <= 2e-3  # same kernel arithmetic, other copy path
