"""CPU: the oracle's k-norm + rotary prologue of the fused writer, pinned three ways.

1. The rotation alone equals vLLM's native rotary embedding run as torch bf16
   CPU ops (rotary_embedding/base.py forward_static + common.py ApplyRotaryEmb:
   cos/sin cast to the key dtype, x1 c - x2 s and x2 c + x1 s as bf16 tensor
   arithmetic) bit for bit, NeoX and GPT-J.
2. The norm equals an independent NumPy restatement of the order the CUDA
   kernel specifies (32 lane partials of even + odd squares, pairwise at
   16..1, IEEE sqrt/divide).
3. The norm stays within one bf16 ulp of vLLM's ir rms_norm formula in torch
   (its own reduction order) and is identical on almost every element.
"""
import numpy as np
import pytest
import torch

import oracle
from nvfp4_qsa import workloads as W


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _torch_rotary(key_bf16, positions, cos_sin_bf16, neox):
    cs = cos_sin_bf16.index_select(0, torch.from_numpy(positions))
    cos, sin = cs.chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(-2), sin.unsqueeze(-2)
    rot = cos_sin_bf16.shape[1]
    x = key_bf16[..., :rot]
    if neox:
        x1, x2 = torch.chunk(x, 2, dim=-1)
    else:
        x1, x2 = x[..., ::2], x[..., 1::2]
    o1 = x1 * cos - x2 * sin
    o2 = x2 * cos + x1 * sin
    out = torch.cat((o1, o2), dim=-1) if neox else torch.stack((o1, o2), dim=-1).flatten(-2)
    return torch.cat((out, key_bf16[..., rot:]), dim=-1)


@pytest.mark.parametrize("hd,rot,neox", [(256, 64, True), (256, 64, False), (256, 256, True), (128, 32, False),
                                         (64, 4, True)])
def test_rotation_matches_torch_bf16_native_bit_for_bit(hd, rot, neox):
    rng = np.random.default_rng(hd + rot)
    kb = W.f32_to_bf16_bits(rng.standard_normal((64, 2, hd), dtype=np.float32) * 3)
    pos = rng.integers(0, 4096, 64).astype(np.int64)
    cs = W.f32_to_bf16_bits(W.rope_cos_sin(4096, rot))
    got, valid = oracle.norm_rope(kb, pos, cs, None, neox=neox)
    assert valid.all()
    want = _bits(_torch_rotary(_bf16(kb), pos, _bf16(cs), neox))
    np.testing.assert_array_equal(got, want)


def _numpy_norm(kb, w, offset, eps):
    x = W.bf16_bits_to_f32(kb).astype(np.float32)
    t, h, hd = x.shape
    e = hd // 32
    even = np.zeros((t, h, 32), np.float32)
    odd = np.zeros((t, h, 32), np.float32)
    xr = x.reshape(t, h, 32, e)
    for j in range(0, e, 2):  # squares are exact in fp32, so acc + x*x equals the fused multiply-add
        even = (even + xr[..., j] * xr[..., j]).astype(np.float32)
        odd = (odd + xr[..., j + 1] * xr[..., j + 1]).astype(np.float32)
    parts = (even + odd).astype(np.float32)
    m = 16
    while m >= 1:
        parts[..., :m] = (parts[..., :m] + parts[..., m:2 * m]).astype(np.float32)
        m //= 2
    ss = parts[..., :1]
    r = (np.float32(1.0) / np.sqrt((ss * np.float32(1.0 / hd) + np.float32(eps)).astype(np.float32))).astype(np.float32)
    y = ((x * r).astype(np.float32) * (w.astype(np.float32) + np.float32(offset))).astype(np.float32)
    return W.f32_to_bf16_bits(y)


@pytest.mark.parametrize("hd", [64, 256, 512])
def test_norm_matches_numpy_restatement_of_the_kernel_order(hd):
    rng = np.random.default_rng(hd)
    kb = W.f32_to_bf16_bits(rng.standard_normal((40, 3, hd), dtype=np.float32)
                            * np.exp2(rng.uniform(-6, 6, (40, 3, 1))).astype(np.float32))
    w = W.bf16_bits_to_f32(W.f32_to_bf16_bits((rng.standard_normal(hd) * 0.3).astype(np.float32)))
    for offset, eps in ((1.0, 1e-6), (0.0, 1e-5)):
        got, _ = oracle.norm_rope(kb, weight=w, offset=offset, eps=eps)
        np.testing.assert_array_equal(got, _numpy_norm(kb, w, offset, eps))


def test_norm_close_to_vllm_rms_norm_formula():
    kb, _, _, _, _, w = W.projection_config(seed=3, tokens=2048, max_position=16)
    got, _ = oracle.norm_rope(kb, weight=w, offset=1.0, eps=1e-6)
    x = _bf16(kb).float()
    var = x.pow(2).mean(dim=-1, keepdim=True)
    want = (x * torch.rsqrt(var + 1e-6) * (torch.from_numpy(w) + 1.0)).to(torch.bfloat16).float().numpy()
    g = W.bf16_bits_to_f32(got)
    assert np.all(np.abs(g - want) <= np.maximum(np.abs(g), np.abs(want)) * 2.0 ** -7 * 1.0001)
    assert np.mean(g == want) > 0.99


def test_positions_outside_the_table_are_not_valid():
    rng = np.random.default_rng(1)
    kb = W.f32_to_bf16_bits(rng.standard_normal((5, 2, 256), dtype=np.float32))
    cs = W.f32_to_bf16_bits(W.rope_cos_sin(100, 64))
    out, valid = oracle.norm_rope(kb, np.array([0, -1, 99, 100, 7], np.int64), cs, None)
    assert valid.tolist() == [True, False, True, False, True]
    np.testing.assert_array_equal(out[~valid], kb[~valid])
