"""CPU: the vLLM backend hooks (nvfp4_qsa.vllm_hooks) with fake layer, metadata and kernels.

Checks the reference hook behaviour (integration/snapshot/qsa.py:263-321 and
:618-640) without a GPU: the rejections, output zeroing, the early return on
an empty batch, the missing top-k buffer and bad cache errors, the four region
views cut from the uint8 cache, and the exact arguments handed to the raw
kernels (recorded by monkeypatched stand-ins; nothing is computed).
"""
from types import SimpleNamespace

import pytest
import torch

from nvfp4_qsa import kernels, vllm_hooks
from nvfp4_qsa.vllm_hooks import QSANVFP4AttentionHooks, split_nvfp4_kv_cache, write_nvfp4_kv


class Impl(QSANVFP4AttentionHooks):
    def __init__(self, **kw):
        self.head_size = 256
        self.alibi_slopes = None
        self.sinks = None
        self.sliding_window = (-1, -1)
        self.__dict__.update(kw)


def _inputs(num_tokens=3, max_tokens=5, blocks=4, page=16):
    layer = SimpleNamespace(topk_indices_buffer=torch.arange(max_tokens * 8, dtype=torch.int32).view(max_tokens, 8),
                            _qsa_nvfp4_k_global=2, _qsa_nvfp4_v_global=0.5)
    query = torch.randn(max_tokens, 24, 256).bfloat16()
    kv_cache = torch.zeros(blocks, 2, page, 288, dtype=torch.uint8)
    meta = SimpleNamespace(num_actual_tokens=num_tokens, block_table=torch.zeros(2, 3, dtype=torch.int32))
    output = torch.full((max_tokens, 24, 256), 7.0).bfloat16()
    t2r = torch.zeros(max_tokens, dtype=torch.int32)
    return layer, query, kv_cache, meta, output, t2r


@pytest.fixture
def recorded(monkeypatch):
    calls = []
    monkeypatch.setattr(kernels, "qsa_sparse_paged_attention_nvfp4", lambda *a: calls.append(("read", a)))
    monkeypatch.setattr(kernels, "qsa_write_cache_nvfp4", lambda *a: calls.append(("write", a)))
    return calls


def test_split_matches_the_record_layout():
    cache = torch.arange(3 * 2 * 4 * 288, dtype=torch.int64).remainder(251).to(torch.uint8).view(3, 2, 4, 288)
    kd, ks, vd, vs = split_nvfp4_kv_cache(cache, 256)
    assert kd.shape == (3, 4, 2, 128) and ks.shape == (3, 4, 2, 16)
    assert vd.shape == (3, 4, 2, 128) and vs.shape == (3, 4, 2, 16)
    for view, off in ((kd, 0), (ks, 128), (vd, 144), (vs, 272)):
        assert view.stride() == (2 * 4 * 288, 288, 4 * 288, 1)
        assert view.data_ptr() - cache.data_ptr() == off
    assert torch.equal(vd[1, 2, 1], cache[1, 1, 2, 144:272])


@pytest.mark.parametrize("bad", [torch.zeros(2, 2, 4, 288, dtype=torch.int8), torch.zeros(2, 2, 4, 256, dtype=torch.uint8)])
def test_split_rejects_a_cache_that_is_not_nvfp4(bad):
    with pytest.raises(RuntimeError, match="last dim 288"):
        split_nvfp4_kv_cache(bad, 256)


@pytest.mark.parametrize("kw,match", [
    (dict(output_scale=torch.ones(1)), "fused output quantization"),
    (dict(output_block_scale=torch.ones(1)), "fused output quantization"),
])
def test_forward_rejects_fused_output_quantisation(recorded, kw, match):
    layer, query, cache, meta, out, t2r = _inputs()
    with pytest.raises(NotImplementedError, match=match):
        Impl().forward_qsa(layer, query, None, None, cache, meta, out, t2r, **kw)
    assert not recorded


@pytest.mark.parametrize("attrs,match", [
    (dict(alibi_slopes=torch.ones(24)), "ALiBi"),
    (dict(sinks=torch.ones(24)), "attention sinks"),
    (dict(sliding_window=(128, 0)), "sliding-window"),
])
def test_forward_rejects_unsupported_attention_features(recorded, attrs, match):
    layer, query, cache, meta, out, t2r = _inputs()
    with pytest.raises(NotImplementedError, match=match):
        Impl(**attrs).forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    assert not recorded


def test_forward_zeroes_and_returns_on_an_empty_batch(recorded):
    layer, query, cache, meta, out, t2r = _inputs(num_tokens=0)
    res = Impl().forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    assert res is out and not out.float().any() and not recorded


def test_forward_needs_the_topk_buffer(recorded):
    layer, query, cache, meta, out, t2r = _inputs()
    del layer.topk_indices_buffer
    with pytest.raises(RuntimeError, match="top-k buffer"):
        Impl().forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    assert not out.float().any()  # zeroed before the check, as in the reference


def test_forward_rejects_a_bad_cache(recorded):
    layer, query, _, meta, out, t2r = _inputs()
    with pytest.raises(RuntimeError, match="uint8"):
        Impl().forward_qsa(layer, query, None, None, torch.zeros(4, 2, 16, 288, dtype=torch.float16), meta, out, t2r)


def test_forward_hands_the_reader_the_reference_arguments(recorded):
    layer, query, cache, meta, out, t2r = _inputs(num_tokens=3)
    res = Impl().forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    assert res is out
    (kind, a), = recorded
    assert kind == "read" and len(a) == 11
    q, kd, ks, vd, vs, gk, gv, idx, bt, tr, o = a
    assert q.shape[0] == 3 and q.data_ptr() == query.data_ptr()
    assert (kd.shape, ks.shape, vd.shape, vs.shape) == ((4, 16, 2, 128), (4, 16, 2, 16), (4, 16, 2, 128), (4, 16, 2, 16))
    assert vd.data_ptr() - cache.data_ptr() == 144
    assert (gk, gv) == (2.0, 0.5) and type(gk) is float and type(gv) is float
    assert torch.equal(idx, layer.topk_indices_buffer[:3]) and bt is meta.block_table and tr.shape[0] == 3
    assert o.shape[0] == 3 and o.data_ptr() == out.data_ptr()
    assert not out.float().any()  # zeroed; the reader writes rows [0, 3)


def test_forward_defaults_the_global_scales_to_one(recorded):
    layer, query, cache, meta, out, t2r = _inputs()
    del layer._qsa_nvfp4_k_global, layer._qsa_nvfp4_v_global
    Impl().forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    assert recorded[0][1][5:7] == (1.0, 1.0)


def test_write_hook_hands_the_writer_the_reference_arguments(recorded):
    cache = torch.zeros(4, 2, 16, 288, dtype=torch.uint8)
    key = torch.randn(5, 2, 256).bfloat16()
    value = torch.randn(5, 2, 256).bfloat16()
    slots = torch.arange(5)
    write_nvfp4_kv(cache, 256, key, value, slots, 1, 3)
    (kind, a), = recorded
    assert kind == "write" and len(a) == 9
    assert a[0] is key and a[1] is value and a[6] is slots and a[7:] == (1.0, 3.0)
    assert a[4].data_ptr() - cache.data_ptr() == 144 and a[3].shape == (4, 16, 2, 16)


@pytest.fixture
def recorded_siblings(monkeypatch):
    calls = []
    monkeypatch.setattr(kernels, "qsa_sparse_paged_attention_fp8", lambda *a: calls.append(("fp8", a)))
    monkeypatch.setattr(kernels, "qsa_sparse_paged_attention", lambda *a: calls.append(("bf16", a)))
    monkeypatch.setattr(kernels, "qsa_sparse_paged_attention_nvfp4", lambda *a: calls.append(("nvfp4", a)))
    return calls


def test_forward_bf16_cache_goes_to_the_bf16_reader(recorded_siblings):
    # snapshot/qsa.py:323-366: K and V halves of a [blocks, kv_heads, page, 2 * 256] bf16 cache
    layer, query, _, meta, out, t2r = _inputs(num_tokens=2)
    cache = torch.zeros(4, 2, 16, 512, dtype=torch.bfloat16)
    Impl(_qsa_kv_nvfp4=False).forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    (kind, a), = recorded_siblings
    assert kind == "bf16" and len(a) == 7
    q, kc, vc, idx, bt, tr, o = a
    assert kc.shape == vc.shape == (4, 16, 2, 256)
    assert vc.data_ptr() - cache.data_ptr() == 256 * 2 and kc.stride() == (2 * 16 * 512, 512, 16 * 512, 1)
    assert q.shape[0] == 2 and o.shape[0] == 2 and bt is meta.block_table and torch.equal(idx, layer.topk_indices_buffer[:2])


def test_forward_fp8_cache_goes_to_the_fp8_reader(recorded_siblings):
    layer, query, _, meta, out, t2r = _inputs(num_tokens=3)
    layer._k_scale_float, layer._v_scale_float = 0.5, 2.0
    cache = torch.zeros(4, 2, 16, 512, dtype=torch.uint8)
    Impl(_qsa_kv_nvfp4=False, _qsa_kv_fp8=True).forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    (kind, a), = recorded_siblings
    assert kind == "fp8" and len(a) == 9
    assert a[1].dtype == torch.float8_e4m3fn and a[1].shape == (4, 16, 2, 256) and a[3:5] == (0.5, 2.0)


def test_forward_rejects_a_non_bf16_main_cache(recorded_siblings):
    layer, query, _, meta, out, t2r = _inputs()
    cache = torch.zeros(4, 2, 16, 512, dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="BF16 Q/K/V"):
        Impl(_qsa_kv_nvfp4=False).forward_qsa(layer, query, None, None, cache, meta, out, t2r)
    assert not recorded_siblings


def test_singleton_dims_get_dense_strides():
    t = torch.zeros(4, 1, 2, 256)[:, :, :, :]
    odd = t.as_strided(t.shape, (512, 7, 256, 1))
    fixed = vllm_hooks.canonicalize_singleton_dim_strides(odd)
    assert fixed.stride() == (512, 512, 256, 1) and fixed.data_ptr() == odd.data_ptr()


def test_hooks_module_calls_through_kernels_namespace():
    # the hooks look the raw ops up on nvfp4_qsa.kernels at call time (monkeypatch-able, one code path)
    assert vllm_hooks.kernels is kernels


# ---- cache planner accounting (snapshot/qsa.py:66-68, :187-204, :556-566) ----

def test_nvfp4_dtype_names():
    assert vllm_hooks.is_qsa_nvfp4_dtype("nvfp4") and vllm_hooks.is_qsa_nvfp4_dtype("nvfp4_4over6")
    for other in ("fp8", "auto", "bfloat16", None, torch.uint8):
        assert not vllm_hooks.is_qsa_nvfp4_dtype(other)


def test_storage_dim_and_page_bytes_match_the_record():
    assert vllm_hooks.nvfp4_storage_dim(256) == 144
    assert vllm_hooks.nvfp4_storage_dim(128) == 72
    with pytest.raises(ValueError):
        vllm_hooks.nvfp4_storage_dim(100)
    # one 3,136-token block of one layer, 2 kv heads: 3136 x 2 x 288 bytes
    assert vllm_hooks.nvfp4_page_bytes(3136, 2, 256) == 3136 * 2 * 288
    f = vllm_hooks.nvfp4_kv_cache_spec_fields(16, 2, 256)
    assert f == {"block_size": 16, "num_kv_heads": 2, "head_size": 144, "head_size_v": 144, "dtype": torch.uint8}
    # a cache allocated from those fields is what split_nvfp4_kv_cache cuts into the four regions
    cache = torch.zeros(3, f["num_kv_heads"], f["block_size"], f["head_size"] + f["head_size_v"], dtype=f["dtype"])
    kd, ks, vd, vs = split_nvfp4_kv_cache(cache, 256)
    assert kd.shape[-1] == 128 and ks.shape[-1] == 16 and vd.shape[-1] == 128 and vs.shape[-1] == 16
    assert cache.numel() == 3 * vllm_hooks.nvfp4_page_bytes(16, 2, 256)


def test_customize_spec_advertises_packed_bytes_and_is_idempotent():
    from dataclasses import dataclass

    @dataclass(frozen=True)
    class Spec:
        block_size: int
        num_kv_heads: int
        head_size: int
        kv_quant_mode: str
        state_content_bytes: int = 0

    logical = Spec(16, 2, 256, "nvfp4-mode")
    out = vllm_hooks.customize_nvfp4_spec(logical, "nvfp4-mode")
    assert out.state_content_bytes == 288 and out.head_size == 256 and logical.state_content_bytes == 0
    physical = Spec(16, 2, 144, "auto")
    assert vllm_hooks.customize_nvfp4_spec(physical, "nvfp4-mode") is physical
    bf16 = Spec(16, 2, 256, "bf16-mode")
    assert vllm_hooks.customize_nvfp4_spec(bf16, "nvfp4-mode") is bf16
