"""GPU: the K/V projection fused with the NVFP4 writer (nvqsa_kv_proj_write_cache).

The reference's layer computes qkv = hidden @ W_qkv^T in bf16, then k_norm and
the rotary embedding on K, then qsa_write_cache_nvfp4
(integration/snapshot/qsa.py:658-667 -> :618-640).  The fused kernel must give:
  1. on inputs whose dot products are exact in fp32 (so every GEMM agrees on
     the bf16 K and V), cache bytes, rotated K and V bit-identical to the C
     oracle's chain (exact projection -> oracle.norm_rope -> oracle.write_cache);
  2. on random inputs, K and V within one bf16 rounding of an fp32 projection
     computed by torch, and cache bytes and rotated K bit-identical to the
     oracle's chain run on the kernel's own projection (read back with the
     norm and rotation off: the kernel's accumulation order is fixed for a
     given shape, including the rank order of a split k-loop).
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import bits_to_cuda, cuda_to_bits, regions
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu

HD = 256


def _storage(blocks, kvh, page):
    return torch.zeros(blocks, kvh, page, 2 * (HD // 2 + HD // 16), dtype=torch.uint8, device="cuda")


def _run(hidden, wk, wv, storage, slots, pos=None, cs=None, w=None, neox=True, gk=1.0, gv=1.0, eps=1e-6,
         offset=1.0, outs=True):
    tokens, kvh = hidden.shape[0], wk.shape[0] // HD
    kd, ks, vd, vs = regions(storage)
    ko = torch.full((tokens, kvh, HD), float("nan"), dtype=torch.bfloat16, device="cuda") if outs else None
    vo = torch.full((tokens, kvh, HD), float("nan"), dtype=torch.bfloat16, device="cuda") if outs else None
    kernels.qsa_kv_proj_write_cache_nvfp4(
        hidden, wk, wv, kd, ks, vd, vs, torch.from_numpy(slots).cuda(), gk, gv,
        positions=None if pos is None else torch.from_numpy(pos).cuda(),
        cos_sin_cache=None if cs is None else bits_to_cuda(cs),
        k_norm_weight=None if w is None else torch.from_numpy(w).cuda(), eps=eps, is_neox_style=neox,
        norm_weight_offset=offset, key_out=ko, value_out=vo)
    torch.cuda.synchronize()
    return ko, vo


def _expected(kb, vb, slots, pos, cs, w, blocks, page, neox=True, gk=1.0, gv=1.0, eps=1e-6, offset=1.0):
    kr, valid = oracle.norm_rope(kb, pos, cs, w, offset, eps, neox)
    st = np.zeros((blocks, kb.shape[1], page, 2 * (HD // 2 + HD // 16)), np.uint8)
    oracle.write_cache(kr, vb, st, np.where(valid, slots, -1), gk, gv)
    return st, kr, valid


def _slots_positions(rng, tokens, blocks, page, max_pos, holes=True):
    slots = rng.permutation(blocks * page)[:tokens].astype(np.int64)
    pos = rng.integers(0, max_pos, tokens).astype(np.int64)
    if holes:
        slots[::37] = -1                    # padding tokens
        slots[5::41] = blocks * page + 3    # past the cache
        pos[7::53] = max_pos + 1            # position outside the table: token skipped
    return slots, pos


@pytest.mark.parametrize("tokens,hidden_size,kvh,rot,neox,norm", [
    (300, 1024, 2, 256, True, True),     # full rotation, ragged last tile of 128 tokens
    (128, 512, 1, 64, True, True),       # partial NeoX rotation (Qwen3-Next style), one head
    (77, 1000, 4, 64, False, True),      # GPT-J pairs, hidden not a multiple of 64 (zero-filled tail)
    (200, 768, 2, 0, True, False),       # no rotation, no norm: the plain writer on the projection
    (2400, 512, 4, 256, True, True),     # more 128-token CTAs than SMs: 256-token CTAs, ragged last one
    (3000, 256, 2, 64, True, True),      # 128-token CTAs, one wave, no k-split
    (96, 4096, 2, 64, True, True),       # a decode batch: each tile's k-blocks split over a cluster of 8 CTAs
    (1000, 640, 2, 64, False, True),     # 10 k-blocks over clusters of 4 (3, 3, 3, 1)
])
def test_exact_projection_matches_oracle_chain(tokens, hidden_size, kvh, rot, neox, norm):
    rng = np.random.default_rng(tokens + hidden_size + kvh)
    # integers times 2^-5: every dot product is exact in fp32, whatever the summation order
    x = rng.integers(-2, 3, (tokens, hidden_size)).astype(np.float32)
    wk = (rng.integers(-3, 4, (kvh * HD, hidden_size)) * 2.0 ** -5).astype(np.float32)
    wv = (rng.integers(-3, 4, (kvh * HD, hidden_size)) * 2.0 ** -5).astype(np.float32)
    kb = W.f32_to_bf16_bits((x.astype(np.float64) @ wk.T.astype(np.float64)).astype(np.float32)).reshape(tokens, kvh, HD)
    vb = W.f32_to_bf16_bits((x.astype(np.float64) @ wv.T.astype(np.float64)).astype(np.float32)).reshape(tokens, kvh, HD)
    page, max_pos = 16, 4096
    blocks = (tokens + page - 1) // page + 2
    slots, pos = _slots_positions(rng, tokens, blocks, page, max_pos)
    cs = W.f32_to_bf16_bits(W.rope_cos_sin(max_pos, rot)) if rot else None
    w = W.bf16_bits_to_f32(W.f32_to_bf16_bits((rng.standard_normal(HD) * 0.2).astype(np.float32))) if norm else None
    storage = _storage(blocks, kvh, page)
    ko, vo = _run(bits_to_cuda(W.f32_to_bf16_bits(x)), bits_to_cuda(W.f32_to_bf16_bits(wk)),
                  bits_to_cuda(W.f32_to_bf16_bits(wv)), storage, slots, pos if rot else None, cs, w, neox)
    want, kr, valid = _expected(kb, vb, slots, pos if rot else None, cs, w, blocks, page, neox)
    assert np.array_equal(storage.cpu().numpy(), want)
    assert np.array_equal(cuda_to_bits(vo), vb)
    assert np.array_equal(cuda_to_bits(ko)[valid.astype(bool)], kr[valid.astype(bool)])


@pytest.mark.parametrize("tokens", [1000, 5000])  # 128-token CTAs; 256-token CTAs (more than one wave of 128)
def test_random_projection_within_one_rounding_and_epilogue_bit_exact(tokens):
    hidden_size, kvh = 4096, 2
    rng = np.random.default_rng(17)
    g = torch.Generator(device="cuda").manual_seed(17)
    hidden = torch.randn(tokens, hidden_size, device="cuda", generator=g).to(torch.bfloat16)
    wk = (torch.randn(kvh * HD, hidden_size, device="cuda", generator=g) * hidden_size ** -0.5).to(torch.bfloat16)
    wv = (torch.randn(kvh * HD, hidden_size, device="cuda", generator=g) * hidden_size ** -0.5).to(torch.bfloat16)
    page, max_pos, rot = 64, 8192, 64
    blocks = tokens // page + 3
    slots, pos = _slots_positions(rng, tokens, blocks, page, max_pos)
    cs = W.f32_to_bf16_bits(W.rope_cos_sin(max_pos, rot))
    w = W.bf16_bits_to_f32(W.f32_to_bf16_bits((rng.standard_normal(HD) * 0.1).astype(np.float32)))

    # the projection itself: K and V with the norm and rotation off
    plain = _storage(blocks, kvh, page)
    k0, v0 = _run(hidden, wk, wv, plain, slots)
    ref_k = (hidden.float() @ wk.float().T).view(tokens, kvh, HD)
    ref_v = (hidden.float() @ wv.float().T).view(tokens, kvh, HD)
    for got, ref in ((k0, ref_k), (v0, ref_v)):
        err = (got.float() - ref).abs()
        # one bf16 rounding of an fp32 sum whose order differs: |err| <= 2^-8 |ref| + fp32 slack
        assert (err <= ref.abs() * 2.0 ** -8 + 1e-5).all()
    kb, vb = cuda_to_bits(k0), cuda_to_bits(v0)
    want_plain, _, _ = _expected(kb, vb, slots, None, None, None, blocks, page)
    assert np.array_equal(plain.cpu().numpy(), want_plain)

    # norm + rotation + writer on the same (deterministic) projection
    fused = _storage(blocks, kvh, page)
    ko, vo = _run(hidden, wk, wv, fused, slots, pos, cs, w)
    assert np.array_equal(cuda_to_bits(vo), vb)
    want, kr, valid = _expected(kb, vb, slots, pos, cs, w, blocks, page)
    assert np.array_equal(fused.cpu().numpy(), want)
    assert np.array_equal(cuda_to_bits(ko)[valid.astype(bool)], kr[valid.astype(bool)])


def test_scales_offsets_and_reference_layout_at_config_3_page():
    # slow-path global scales, a plain RMSNorm weight (offset 0), page 3136, cache views of vLLM's layout
    tokens, hidden_size, kvh = 256, 2048, 2
    rng = np.random.default_rng(23)
    x = rng.integers(-2, 3, (tokens, hidden_size)).astype(np.float32)
    wk = (rng.integers(-3, 4, (kvh * HD, hidden_size)) * 2.0 ** -6).astype(np.float32)
    wv = (rng.integers(-3, 4, (kvh * HD, hidden_size)) * 2.0 ** -6).astype(np.float32)
    kb = W.f32_to_bf16_bits((x.astype(np.float64) @ wk.T.astype(np.float64)).astype(np.float32)).reshape(tokens, kvh, HD)
    vb = W.f32_to_bf16_bits((x.astype(np.float64) @ wv.T.astype(np.float64)).astype(np.float32)).reshape(tokens, kvh, HD)
    page, blocks, max_pos, rot = 3136, 2, 100000, 256
    slots, pos = _slots_positions(rng, tokens, blocks, page, max_pos, holes=False)
    cs = W.f32_to_bf16_bits(W.rope_cos_sin(max_pos, rot))
    w = W.bf16_bits_to_f32(W.f32_to_bf16_bits((1.0 + rng.standard_normal(HD) * 0.1).astype(np.float32)))
    for gk, gv in ((1e-3, 3e4), (1.0, 1.0)):
        storage = _storage(blocks, kvh, page)
        _run(bits_to_cuda(W.f32_to_bf16_bits(x)), bits_to_cuda(W.f32_to_bf16_bits(wk)),
             bits_to_cuda(W.f32_to_bf16_bits(wv)), storage, slots, pos, cs, w, gk=gk, gv=gv, offset=0.0, outs=False)
        want, _, _ = _expected(kb, vb, slots, pos, cs, w, blocks, page, gk=gk, gv=gv, offset=0.0)
        assert np.array_equal(storage.cpu().numpy(), want), (gk, gv)


def test_weight_views_of_one_qkv_matrix():
    # K and V weights as row blocks of one [q + gate + k + v, hidden] matrix, hidden a column slice
    tokens, hidden_size, kvh = 130, 512, 2
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv_w = (torch.randn(2 * 24 * HD + 2 * kvh * HD, hidden_size, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    wk = qkv_w[2 * 24 * HD:2 * 24 * HD + kvh * HD]
    wv = qkv_w[2 * 24 * HD + kvh * HD:]
    big = torch.randn(tokens, hidden_size + 64, device="cuda", generator=g).to(torch.bfloat16)
    hidden = big[:, 64:]
    page, blocks = 16, tokens // 16 + 2
    slots = np.random.default_rng(4).permutation(blocks * page)[:tokens].astype(np.int64)
    s1, s2 = _storage(blocks, kvh, page), _storage(blocks, kvh, page)
    k1, v1 = _run(hidden, wk, wv, s1, slots)
    k2, v2 = _run(hidden.contiguous(), wk.contiguous(), wv.contiguous(), s2, slots)
    assert torch.equal(s1, s2) and torch.equal(k1, k2) and torch.equal(v1, v2)


def test_inside_cuda_graph():
    tokens, hidden_size, kvh = 384, 1024, 2
    g = torch.Generator(device="cuda").manual_seed(9)
    hidden = torch.randn(tokens, hidden_size, device="cuda", generator=g).to(torch.bfloat16)
    wk = (torch.randn(kvh * HD, hidden_size, device="cuda", generator=g) * 0.03).to(torch.bfloat16)
    wv = (torch.randn(kvh * HD, hidden_size, device="cuda", generator=g) * 0.03).to(torch.bfloat16)
    page, blocks = 32, tokens // 32 + 1
    slots = torch.from_numpy(np.random.default_rng(1).permutation(blocks * page)[:tokens].astype(np.int64)).cuda()
    eager, graphed = _storage(blocks, kvh, page), _storage(blocks, kvh, page)
    kernels.qsa_kv_proj_write_cache_nvfp4(hidden, wk, wv, *regions(eager), slots, 1.0, 1.0)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qsa_kv_proj_write_cache_nvfp4(hidden, wk, wv, *regions(graphed), slots, 1.0, 1.0)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.qsa_kv_proj_write_cache_nvfp4(hidden, wk, wv, *regions(graphed), slots, 1.0, 1.0)
    graphed.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager, graphed)
    del graph


def test_rejections_and_no_wait_ran_out():
    from nvfp4_qsa import _native
    kvh, page, blocks = 2, 16, 4
    storage = _storage(blocks, kvh, page)
    slots = torch.zeros(8, dtype=torch.int64, device="cuda")
    w = torch.zeros(kvh * HD, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):  # head_dim 128 rows
        kernels.qsa_kv_proj_write_cache_nvfp4(torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda"),
                                              w[:128], w[:128], *regions(storage), slots, 1.0, 1.0)
    with pytest.raises(ValueError):  # hidden_size 66: no row stride of 66 elements is a multiple of 16 bytes
        h = torch.zeros(8, 68, dtype=torch.bfloat16, device="cuda")[:, :66]
        kernels.qsa_kv_proj_write_cache_nvfp4(h, torch.zeros(kvh * HD, 66, dtype=torch.bfloat16, device="cuda"),
                                              torch.zeros(kvh * HD, 66, dtype=torch.bfloat16, device="cuda"),
                                              *regions(storage), slots, 1.0, 1.0)
    with pytest.raises(ValueError):  # NeoX rotation of 48 dims: not a multiple of 32
        kernels.qsa_kv_proj_write_cache_nvfp4(torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda"), w, w,
                                              *regions(storage), slots, 1.0, 1.0,
                                              positions=torch.zeros(8, dtype=torch.int64, device="cuda"),
                                              cos_sin_cache=torch.zeros(10, 48, dtype=torch.bfloat16, device="cuda"))
    torch.cuda.synchronize()
    assert _native.read_error_flags() == 0
