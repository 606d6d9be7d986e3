"""CPU: argument checks of the fused k-norm + RoPE writer, in the C ABI and the Python wrapper.

Every case here is rejected (or, for an empty batch, accepted) before the library makes any
CUDA call, so the checks run without a GPU; the kernel itself is covered by
tests/test_gpu_fused_writer.py.
"""
import pytest
import torch

from nvfp4_qsa import _native, kernels

A = 0x100000  # fake device addresses: never dereferenced by the paths tested here


def _args(tokens=4, head_dim=256, kv_heads=2, blocks=4, page=16):
    rec = 2 * (head_dim // 2 + head_dim // 16)
    row = kv_heads * head_dim
    args = [A, row, head_dim, A + 0x10000, row, head_dim]
    for off in (0, head_dim // 2, head_dim // 2 + head_dim // 16, head_dim + head_dim // 16):  # record layout
        args += [A + 0x20000 + off, kv_heads * page * rec, rec, page * rec]
    args += [A + 0x80000, tokens, kv_heads, head_dim, blocks, page, 1.0, 1.0]
    return args


def _call(args, weight=A + 0x90000, offset=1.0, eps=1e-6, positions=A + 0xa0000, table=A + 0xb0000,
          stride=64, max_pos=100, rot=64, neox=1, key_out=0, ko_st=0, ko_sh=0):
    return _native.load().nvqsa_norm_rope_write_cache(*args, weight, offset, eps, positions, table, stride, max_pos,
                                                       rot, neox, key_out, ko_st, ko_sh, 0)


def test_status_codes_before_any_launch():
    a = _args()
    assert _call(_args(head_dim=100)) == 3                       # head_dim
    assert _call(a, rot=24) == 2                                 # not a multiple of head_dim / 16
    assert _call(a, rot=512) == 2                                # past head_dim
    assert _call(a, positions=0) == 1                            # rotation without positions
    assert _call(a, table=0) == 1                                # rotation without a table
    assert _call(a, stride=32) == 2                              # row shorter than rotary_dim
    assert _call(a, max_pos=0) == 2
    assert _call(a, eps=-1.0) == 2 and _call(a, eps=float("inf")) == 2
    assert _call(a, weight=A + 2) == 4                           # fp32 weights misaligned
    assert _call(a, table=A + 0xb0002) == 4                      # cos/sin runs need 16-byte rows (NeoX, hd 256)
    assert _call(a, stride=65) == 4
    assert _call(a, key_out=A + 0xc0008, ko_st=512, ko_sh=256) == 4  # key_out rows need 16-byte alignment
    assert _call(a, key_out=A + 0xc0000, ko_st=516, ko_sh=256) == 4
    assert _call(_args(tokens=0)) == 0                           # empty batch: nothing to launch


def _cpu_case(tokens=4, hd=256):
    key = torch.zeros(tokens, 2, hd, dtype=torch.bfloat16)
    kd = torch.zeros(4, 16, 2, hd // 2, dtype=torch.uint8)
    ks = torch.zeros(4, 16, 2, hd // 16, dtype=torch.uint8)
    return key, key.clone(), kd, ks, kd.clone(), ks.clone(), torch.arange(tokens, dtype=torch.int64)


def test_wrapper_rejects_bad_rotation_and_norm_arguments():
    k, v, kd, ks, vd, vs, slots = _cpu_case()
    pos = torch.zeros(4, dtype=torch.int64)
    table = torch.zeros(100, 64, dtype=torch.bfloat16)
    f = kernels.qsa_norm_rope_write_cache_nvfp4
    with pytest.raises(ValueError, match="positions"):
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, cos_sin_cache=table)
    with pytest.raises(ValueError, match="positions"):
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, positions=pos.int(), cos_sin_cache=table)
    with pytest.raises(ValueError, match="cos_sin_cache"):
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, positions=pos, cos_sin_cache=table[:, :63])
    with pytest.raises(ValueError, match="rotary_dim"):
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, positions=pos, cos_sin_cache=table[:, :24])
    with pytest.raises(ValueError, match="k_norm_weight"):
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, k_norm_weight=torch.ones(128))
    with pytest.raises(ValueError, match="key_out"):
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, key_out=torch.zeros(4, 2, 256, dtype=torch.float32))
    with pytest.raises(TypeError, match="BF16"):
        f(k.float(), v, kd, ks, vd, vs, slots, 1.0, 1.0)
    with pytest.raises(ValueError, match="CUDA"):  # valid arguments on CPU tensors: no CPU fallback
        f(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, positions=pos, cos_sin_cache=table, k_norm_weight=torch.zeros(256))
