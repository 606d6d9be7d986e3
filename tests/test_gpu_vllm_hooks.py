"""GPU: the vLLM backend hooks end to end -- write_nvfp4_kv then forward_qsa -- against the oracle."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_attention_close, bits_to_cuda
from nvfp4_qsa import workloads as W
from nvfp4_qsa.vllm_hooks import QSANVFP4AttentionHooks, write_nvfp4_kv

pytestmark = pytest.mark.gpu


class Impl(QSANVFP4AttentionHooks):
    head_size = 256
    alibi_slopes = None
    sinks = None
    sliding_window = (-1, -1)


def test_hooks_write_then_attend_match_the_oracle():
    contexts, table, blocks, slots, indices, t2r = W.mtp_config(seed=8, sequences=3, rows_per_seq=2, ctx_lo=3000,
                                                               ctx_hi=7000, topk=512, page=256)
    rng = np.random.default_rng(8)
    tokens = sum(int(c) for c in contexts)
    key = W.f32_to_bf16_bits(W.gen_values(rng, (tokens, 2, 256), "outliers"))
    value = W.f32_to_bf16_bits(W.gen_values(rng, (tokens, 2, 256), "normal"))
    rows = indices.shape[0]
    query = W.f32_to_bf16_bits(W.gen_values(rng, (rows + 2, 24, 256), "normal"))  # +2 unused rows past num_tokens
    kv_cache = torch.zeros(blocks, 2, 256, 288, dtype=torch.uint8, device="cuda")
    write_nvfp4_kv(kv_cache, 256, bits_to_cuda(key), bits_to_cuda(value),
                   torch.from_numpy(np.concatenate(slots)).cuda(), 1.5, 0.75)
    layer = SimpleNamespace(topk_indices_buffer=torch.from_numpy(
        np.concatenate([indices, np.zeros((2, indices.shape[1]), np.int32)])).cuda(),
        _qsa_nvfp4_k_global=1.5, _qsa_nvfp4_v_global=0.75)
    meta = SimpleNamespace(num_actual_tokens=rows, block_table=torch.from_numpy(table).cuda())
    out = torch.full((rows + 2, 24, 256), 3.0, dtype=torch.bfloat16, device="cuda")
    t2r_d = torch.from_numpy(np.concatenate([t2r, np.zeros(2, np.int32)])).cuda()
    Impl().forward_qsa(layer, bits_to_cuda(query), None, None, kv_cache, meta, out, t2r_d)
    torch.cuda.synchronize()

    storage = np.zeros((blocks, 2, 256, 288), np.uint8)
    oracle.write_cache(key, value, storage, np.concatenate(slots), 1.5, 0.75)
    assert np.array_equal(kv_cache.cpu().numpy(), storage)  # the write hook is bit-exact
    expected = oracle.sparse_attention(query[:rows], storage, indices, table, t2r, 1.5, 0.75)
    assert_attention_close(out[:rows], expected, "hooks")
    assert not out[rows:].float().any()  # rows past num_tokens zeroed, as the reference's output.zero_()
