"""GPU: the fused k-norm -> RoPE -> NVFP4 writer (nvqsa_norm_rope_write_cache).

The reference's caller (integration/snapshot/qsa.py:618-667) runs vLLM's
GemmaRMSNorm k_norm and rotary embedding on K, then qsa_write_cache_nvfp4.
The fused writer must give (1) cache bytes and rotated K bit-identical to the
C oracle's restatement (oracle.norm_rope + oracle.write_cache), (2) cache bytes
bit-identical to the plain writer run on its own rotated K, and (3) a rotated
K within one bf16 ulp of torch's own GPU k_norm + rotary on rare elements
(torch's reduction order and rsqrt differ; the rotation itself is exact).
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import bits_to_cuda, cuda_to_bits, regions
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _inputs(seed, tokens, kvh, hd, rot, max_pos=5000, page=16, blocks=None):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((tokens, kvh, hd), dtype=np.float32) * np.exp2(rng.uniform(-2, 3, (tokens, kvh, 1)))
    k = np.where(rng.random(k.shape) < 0.02, k * 32, k).astype(np.float32)
    v = rng.standard_normal((tokens, kvh, hd), dtype=np.float32)
    blocks = blocks or (tokens + page - 1) // page + 1
    slots = rng.permutation(blocks * page)[:tokens].astype(np.int64)
    pos = rng.integers(0, max_pos, tokens).astype(np.int64)
    cs = W.f32_to_bf16_bits(W.rope_cos_sin(max_pos, rot)) if rot else None
    w = W.bf16_bits_to_f32(W.f32_to_bf16_bits((rng.standard_normal(hd) * 0.2).astype(np.float32)))
    return W.f32_to_bf16_bits(k), W.f32_to_bf16_bits(v), slots, pos, cs, w, blocks, page


def _storage(blocks, kvh, page, hd):
    return torch.zeros(blocks, kvh, page, 2 * (hd // 2 + hd // 16), dtype=torch.uint8, device="cuda")


def _fused(storage, kb, vb, slots, pos, cs, w, hd, neox=True, gk=1.0, gv=1.0, eps=1e-6, offset=1.0, key_out=True):
    kd, ks, vd, vs = regions(storage, hd)
    ko = torch.full(kb.shape, float("nan"), dtype=torch.bfloat16, device="cuda") if key_out else None
    kernels.qsa_norm_rope_write_cache_nvfp4(
        bits_to_cuda(kb), bits_to_cuda(vb), kd, ks, vd, vs, torch.from_numpy(slots).cuda(), gk, gv,
        positions=torch.from_numpy(pos).cuda(), cos_sin_cache=None if cs is None else bits_to_cuda(cs),
        k_norm_weight=None if w is None else torch.from_numpy(w).cuda(), eps=eps, is_neox_style=neox,
        norm_weight_offset=offset, key_out=ko)
    torch.cuda.synchronize()
    return ko


def _expected(kb, vb, slots, pos, cs, w, blocks, page, hd, neox=True, gk=1.0, gv=1.0, eps=1e-6, offset=1.0):
    kr, valid = oracle.norm_rope(kb, pos, cs, w, offset, eps, neox)
    st = np.zeros((blocks, kb.shape[1], page, 2 * (hd // 2 + hd // 16)), np.uint8)
    sl = np.where(valid, slots, -1)
    oracle.write_cache(kr, vb, st, sl, gk, gv)
    return st, kr, valid


CASES = [  # (head_dim, rotary_dim, neox, norm, kv_heads)
    (256, 64, True, True, 2),     # Qwen3-Next: partial rotary 0.25, GemmaRMSNorm
    (256, 256, True, True, 2),    # full rotary
    (256, 64, False, True, 2),    # GPT-J pairs
    (256, 0, True, True, 2),      # norm only
    (256, 64, True, False, 2),    # rotary only
    (256, 16, True, True, 3),     # smallest rotary for 256; odd head count (half-group lanes)
    (256, 32, True, True, 3),     # one NeoX pair of groups; odd head count (lane-per-group kernel)
    (256, 16, False, True, 1),    # GPT-J over one group; one head
    (128, 32, True, True, 1),
    (64, 64, False, True, 2),
    (64, 4, True, True, 2),
    (512, 128, True, True, 2),
]


@pytest.mark.parametrize("hd,rot,neox,norm,kvh", CASES,
                         ids=[f"hd{c[0]}-rot{c[1]}-{'neox' if c[2] else 'gptj'}-{'norm' if c[3] else 'nonorm'}-h{c[4]}"
                              for c in CASES])
def test_fused_writer_matches_oracle(hd, rot, neox, norm, kvh):
    kb, vb, slots, pos, cs, w, blocks, page = _inputs(hd + rot + kvh, 300, kvh, hd, rot)
    w = w if norm else None
    storage = _storage(blocks, kvh, page, hd)
    ko = _fused(storage, kb, vb, slots, pos, cs, w, hd, neox)
    st, kr, _ = _expected(kb, vb, slots, pos, cs, w, blocks, page, hd, neox)
    np.testing.assert_array_equal(cuda_to_bits(ko), kr)
    np.testing.assert_array_equal(storage.cpu().numpy(), st)


@pytest.mark.parametrize("gk,gv,eps,offset", [(0.37, 3e-5, 1e-6, 1.0), (1e4, 2.0, 1e-5, 0.0), (2.0 ** -118, 1.0, 0.0, 1.0)])
def test_fused_writer_scales_eps_and_plain_norm(gk, gv, eps, offset):
    kb, vb, slots, pos, cs, w, blocks, page = _inputs(7, 200, 2, 256, 64)
    storage = _storage(blocks, 2, page, 256)
    ko = _fused(storage, kb, vb, slots, pos, cs, w, 256, True, gk, gv, eps, offset)
    st, kr, _ = _expected(kb, vb, slots, pos, cs, w, blocks, page, 256, True, gk, gv, eps, offset)
    np.testing.assert_array_equal(cuda_to_bits(ko), kr)
    np.testing.assert_array_equal(storage.cpu().numpy(), st)


def test_fused_equals_plain_writer_on_its_rotated_key():
    # config 3 shape: 8,192 projection rows into a 64 x 3,136 cache
    kb, vb, slots, pos, cs, w = W.projection_config(seed=11, tokens=8192, max_position=262144)
    csb = W.f32_to_bf16_bits(cs)
    a, b = _storage(64, 2, 3136, 256), _storage(64, 2, 3136, 256)
    ko = _fused(a, kb, vb, slots, pos, csb, w, 256)
    kd, ks, vd, vs = regions(b)
    kernels.qsa_write_cache_nvfp4(ko, bits_to_cuda(vb), kd, ks, vd, vs, torch.from_numpy(slots).cuda(), 1.0, 1.0)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # and the oracle agrees on a slice of the rows
    kr, _ = oracle.norm_rope(kb[:512], pos[:512], csb, w)
    np.testing.assert_array_equal(cuda_to_bits(ko[:512]), kr)


def test_rotated_key_close_to_torch_native_path():
    """vLLM's native k_norm (ir rms_norm) and rotary embedding as torch GPU ops."""
    kb, vb, slots, pos, cs, w = W.projection_config(seed=12, tokens=4096, max_position=65536)
    csb = W.f32_to_bf16_bits(cs)
    ko = _fused(_storage(64, 2, 3136, 256), kb, vb, slots, pos, csb, w, 256)
    x = bits_to_cuda(kb).float()
    var = x.pow(2).mean(dim=-1, keepdim=True)
    y = (x * torch.rsqrt(var + 1e-6) * (torch.from_numpy(w).cuda() + 1.0)).to(torch.bfloat16)
    cos_sin = bits_to_cuda(csb).index_select(0, torch.from_numpy(pos).cuda())
    cos, sin = cos_sin.chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    rot = y[..., :64]
    x1, x2 = rot.chunk(2, dim=-1)
    ref = torch.cat((torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1), y[..., 64:]), dim=-1)
    got, want = ko.float(), ref.float()
    # a one-ulp difference in the normed K moves a rotated element by at most one ulp of its inputs
    # (|x1 c - x2 s| can be far smaller than |x1|, |x2|), so bound by the row's largest magnitude
    row = want.abs().amax(dim=-1, keepdim=True)
    tol = torch.maximum(want.abs(), got.abs()) * 2.0 ** -7 + row * 2.0 ** -7
    assert ((got - want).abs() <= tol).all()
    assert (got == want).float().mean().item() > 0.99          # and identical almost everywhere
    # the rotation alone is exact: feed torch's own normed K through a rotation-only fused call
    ko2 = torch.empty_like(ko)
    st = _storage(64, 2, 3136, 256)
    kd, ks, vd, vs = regions(st)
    kernels.qsa_norm_rope_write_cache_nvfp4(y.contiguous(), bits_to_cuda(vb), kd, ks, vd, vs,
                                            torch.from_numpy(slots).cuda(), 1.0, 1.0,
                                            positions=torch.from_numpy(pos).cuda(), cos_sin_cache=bits_to_cuda(csb),
                                            key_out=ko2)
    torch.cuda.synchronize()
    assert torch.equal(ko2.view(torch.int16), ref.contiguous().view(torch.int16))


def test_invalid_positions_and_slots_are_skipped():
    kb, vb, slots, pos, cs, w, blocks, page = _inputs(21, 64, 2, 256, 64, max_pos=1000)
    pos = pos.copy()
    slots = slots.copy()
    pos[3], pos[9], pos[20] = -1, 1000, 10 ** 12          # outside the table: token skipped entirely
    slots[5], slots[30] = -1, blocks * page + 7             # no cache slot: key_out still written
    storage = _storage(blocks, 2, page, 256)
    ko = _fused(storage, kb, vb, slots, pos, cs, w, 256)
    st, kr, valid = _expected(kb, vb, slots, pos, cs, w, blocks, page, 256)
    assert not valid[[3, 9, 20]].any() and valid.sum() == 61
    got = cuda_to_bits(ko)
    np.testing.assert_array_equal(got[valid], kr[valid])
    assert np.isnan(W.bf16_bits_to_f32(got[~valid])).all()  # untouched rows keep their NaN fill
    np.testing.assert_array_equal(storage.cpu().numpy(), st)


def test_strided_sources_unaligned_tables_and_separate_regions():
    """K/V as column slices of one qkv tensor, a cos/sin table with an odd row stride (the wrapper
    makes it contiguous),
    key_out a strided view, and separate region tensors (the general-stride path)."""
    hd, kvh, tokens, rot = 256, 2, 150, 64
    kb, vb, slots, pos, cs, w, blocks, page = _inputs(31, tokens, kvh, hd, rot, max_pos=3000)
    qkv = torch.zeros(tokens, 24 * hd + 2 * kvh * hd, dtype=torch.bfloat16, device="cuda")
    qsize = 24 * hd
    qkv[:, qsize:qsize + kvh * hd] = bits_to_cuda(kb).reshape(tokens, -1)
    qkv[:, qsize + kvh * hd:] = bits_to_cuda(vb).reshape(tokens, -1)
    key = qkv[:, qsize:qsize + kvh * hd].view(tokens, kvh, hd)
    value = qkv[:, qsize + kvh * hd:].view(tokens, kvh, hd)
    table = torch.zeros(3000, rot + 1, dtype=torch.bfloat16, device="cuda")
    table[:, :rot] = bits_to_cuda(cs)
    cos_sin = table[:, :rot]                                # row stride 65 elements
    big = torch.full((tokens, kvh, hd + 8), float("nan"), dtype=torch.bfloat16, device="cuda")
    ko = big[:, :, 4:4 + hd]                                # 8-byte offset rows: no vector stores
    kd = torch.zeros(blocks, page, kvh, hd // 2, dtype=torch.uint8, device="cuda")
    ks = torch.zeros(blocks, page, kvh, hd // 16, dtype=torch.uint8, device="cuda")
    vd, vs = torch.zeros_like(kd), torch.zeros_like(ks)
    kernels.qsa_norm_rope_write_cache_nvfp4(key, value, kd, ks, vd, vs, torch.from_numpy(slots).cuda(), 1.0, 1.0,
                                            positions=torch.from_numpy(pos).cuda(), cos_sin_cache=cos_sin,
                                            k_norm_weight=torch.from_numpy(w).cuda(), key_out=ko)
    torch.cuda.synchronize()
    st, kr, _ = _expected(kb, vb, slots, pos, cs, w, blocks, page, hd)
    np.testing.assert_array_equal(cuda_to_bits(ko), kr)
    region = hd // 2 + hd // 16
    want = torch.from_numpy(st).cuda().transpose(1, 2)
    assert torch.equal(kd, want[..., :hd // 2]) and torch.equal(ks, want[..., hd // 2:region])
    assert torch.equal(vd, want[..., region:region + hd // 2]) and torch.equal(vs, want[..., region + hd // 2:])


def test_fused_writer_inside_cuda_graph():
    kb, vb, slots, pos, cs, w, blocks, page = _inputs(41, 256, 2, 256, 64)
    storage = _storage(blocks, 2, page, 256)
    kd, ks, vd, vs = regions(storage)
    k, v = bits_to_cuda(kb), bits_to_cuda(vb)
    sl, ps, wd = (torch.from_numpy(a).cuda() for a in (slots, pos, w))
    csd = bits_to_cuda(cs)
    ko = torch.zeros_like(k)

    def call():
        kernels.qsa_norm_rope_write_cache_nvfp4(k, v, kd, ks, vd, vs, sl, 1.0, 1.0, positions=ps, cos_sin_cache=csd,
                                                k_norm_weight=wd, key_out=ko)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    storage.zero_()
    ko.zero_()
    g.replay()
    torch.cuda.synchronize()
    st, kr, _ = _expected(kb, vb, slots, pos, cs, w, blocks, page, 256)
    np.testing.assert_array_equal(cuda_to_bits(ko), kr)
    np.testing.assert_array_equal(storage.cpu().numpy(), st)
    del g


def test_fused_writer_rejects_bad_arguments():
    kb, vb, slots, pos, cs, w, blocks, page = _inputs(51, 16, 2, 256, 64)
    storage = _storage(blocks, 2, page, 256)
    kd, ks, vd, vs = regions(storage)
    k, v = bits_to_cuda(kb), bits_to_cuda(vb)
    sl, ps, csd = torch.from_numpy(slots).cuda(), torch.from_numpy(pos).cuda(), bits_to_cuda(cs)
    with pytest.raises(ValueError, match="rotary_dim"):
        kernels.qsa_norm_rope_write_cache_nvfp4(k, v, kd, ks, vd, vs, sl, 1.0, 1.0, positions=ps,
                                                cos_sin_cache=csd[:, :24])
    with pytest.raises(ValueError, match="positions"):
        kernels.qsa_norm_rope_write_cache_nvfp4(k, v, kd, ks, vd, vs, sl, 1.0, 1.0, cos_sin_cache=csd)
    with pytest.raises(ValueError, match="positions"):
        kernels.qsa_norm_rope_write_cache_nvfp4(k, v, kd, ks, vd, vs, sl, 1.0, 1.0, positions=ps.int(),
                                                cos_sin_cache=csd)
    with pytest.raises(ValueError, match="k_norm_weight"):
        kernels.qsa_norm_rope_write_cache_nvfp4(k, v, kd, ks, vd, vs, sl, 1.0, 1.0, k_norm_weight=torch.ones(
            128, device="cuda"))
    from nvfp4_qsa import _native
    lib = _native.load()
    args = [k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0), v.stride(1)]
    for t in (kd, ks, vd, vs):
        args += [t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)]
    args += [sl.data_ptr(), 16, 2, 256, blocks, page, 1.0, 1.0, 0, 1.0, 1e-6]
    # rotary_dim 24 is not a multiple of head_dim/16; a negative eps; a rotation without a table
    assert lib.nvqsa_norm_rope_write_cache(*args[:-1], -1.0, ps.data_ptr(), csd.data_ptr(), 64, 5000, 64, 1,
                                           0, 0, 0, 0) == 2
    assert lib.nvqsa_norm_rope_write_cache(*args, ps.data_ptr(), csd.data_ptr(), 64, 5000, 24, 1, 0, 0, 0, 0) == 2
    assert lib.nvqsa_norm_rope_write_cache(*args, ps.data_ptr(), 0, 64, 5000, 64, 1, 0, 0, 0, 0) == 1
    # a table row stride that breaks the vector loads (65 elements): misaligned
    assert lib.nvqsa_norm_rope_write_cache(*args, ps.data_ptr(), csd.data_ptr(), 65, 4000, 64, 1, 0, 0, 0, 0) == 4
    # a key_out row start off the 16-byte grid: misaligned (the Python wrapper goes through a temporary)
    ko = torch.empty(16, 2, 264, dtype=torch.bfloat16, device="cuda")
    assert lib.nvqsa_norm_rope_write_cache(*args, ps.data_ptr(), csd.data_ptr(), 64, 5000, 64, 1,
                                           ko.data_ptr() + 8, 528, 264, 0) == 4
    assert lib.nvqsa_norm_rope_write_cache(*args, ps.data_ptr(), csd.data_ptr(), 64, 5000, 64, 1, 0, 0, 0, 0) == 0
    torch.cuda.synchronize()
