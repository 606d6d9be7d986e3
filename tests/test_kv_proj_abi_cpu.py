"""CPU: argument checks of the fused K/V projection writer (nvqsa_kv_proj_write_cache) and its Python wrapper.

Every case below is rejected (or, for an empty batch, accepted) before the library touches device memory or
the CUDA driver, so it runs without a GPU; the pointers are placeholders that are never dereferenced.
"""
import pytest
import torch

from nvfp4_qsa import _native, kernels

A = 1 << 20  # a 16-byte aligned placeholder address


def _call(lib, hidden=A, hidden_stride=4096, tokens=8, hidden_size=4096, head_dim=256, rot=0, neox=1,
          cos_sin=0, positions=0, norm=0, eps=1e-6, key_out=0, ko_stride=512):
    return lib.nvqsa_kv_proj_write_cache(
        hidden, hidden_stride, tokens, hidden_size,
        A, A, 4096,
        A, 288 * 16 * 2, 288, 288 * 16, A + 128, 288 * 16 * 2, 288, 288 * 16,
        A + 144, 288 * 16 * 2, 288, 288 * 16, A + 272, 288 * 16 * 2, 288, 288 * 16,
        A, 2, head_dim, 4, 16, 1.0, 1.0,
        norm, 1.0, eps,
        positions, cos_sin, rot, 4096, rot, neox,
        key_out, ko_stride, 256, 0, 0, 0, None)


def test_rejections_before_any_device_access():
    lib = _native.load()
    assert _call(lib, head_dim=128) == 3                                    # head_dim 256 only
    assert _call(lib, hidden=0) == 1                                        # null hidden states
    assert _call(lib, hidden_stride=66, hidden_size=66) == 4                # 132-byte rows: not 16-byte multiples
    assert _call(lib, hidden_stride=100, hidden_size=128) == 2              # row stride shorter than a row
    assert _call(lib, rot=48, cos_sin=A, positions=A) == 2                  # NeoX halves must be whole groups
    assert _call(lib, rot=64, cos_sin=A + 8, positions=A) == 4              # cos/sin rows not 16-byte aligned
    assert _call(lib, rot=64) == 1                                          # a rotation needs positions and a table
    assert _call(lib, eps=float("nan")) == 2
    assert _call(lib, norm=A + 4) == 4                                      # norm weights read as float4
    assert _call(lib, key_out=A, ko_stride=500) == 4                        # key_out rows 16-byte aligned
    assert _call(lib, tokens=0) == 0                                        # empty batch: nothing launched


def test_wrapper_type_and_shape_checks_on_cpu_tensors():
    h = torch.zeros(4, 64, dtype=torch.bfloat16)
    w = torch.zeros(512, 64, dtype=torch.bfloat16)
    kd = torch.zeros(2, 16, 2, 128, dtype=torch.uint8)
    ks = torch.zeros(2, 16, 2, 16, dtype=torch.uint8)
    slots = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(TypeError):
        kernels.qsa_kv_proj_write_cache_nvfp4(h.float(), w, w, kd, ks, kd, ks, slots, 1.0, 1.0)
    with pytest.raises(ValueError):  # K rows of a head_dim-128 model
        kernels.qsa_kv_proj_write_cache_nvfp4(h, w[:384], w[:384], kd, ks, kd, ks, slots, 1.0, 1.0)
    with pytest.raises(ValueError):  # weights of another hidden size
        kernels.qsa_kv_proj_write_cache_nvfp4(h, w[:, :32], w[:, :32], kd, ks, kd, ks, slots, 1.0, 1.0)
    with pytest.raises(TypeError):
        kernels.qsa_kv_proj_write_cache_nvfp4(h, w, w, kd, ks, kd, ks, slots.int(), 1.0, 1.0)
    with pytest.raises(ValueError):  # the cache's kv_heads must match the weights' (2 heads of 256 rows)
        kernels.qsa_kv_proj_write_cache_nvfp4(h, w[:256], w[:256], kd, ks, kd, ks, slots, 1.0, 1.0)
    with pytest.raises(ValueError):  # NeoX rotary of 48 dims
        kernels.qsa_kv_proj_write_cache_nvfp4(h, w, w, kd, ks, kd, ks, slots, 1.0, 1.0,
                                              positions=torch.zeros(4, dtype=torch.int64),
                                              cos_sin_cache=torch.zeros(8, 48, dtype=torch.bfloat16))
