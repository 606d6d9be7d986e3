"""CPU: pin the C oracle (oracle/) to the reference's own outputs in tests/golden/.

The golden vectors were produced by tests/golden/make_golden.py from the
reference's src/nvfp4_oracle.py and src/qsa_ref.py.  Codec bytes must match
exactly; attention outputs to 1e-5 (both sides compute in float64).
"""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from nvfp4_qsa import workloads as W


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_codebook_roundtrip_and_nibble_order(golden_kat):
    # tests/test_cpu_contracts.py:18-24 of the reference
    values = np.array([golden_kat["codebook_values"]], np.float32)
    nib, packed, scales, _ = oracle.encode(values, 1.0)
    assert packed[0].tolist() == golden_kat["codebook_packed"]
    assert packed[0, 0] == 0x10 and packed[0, 7] == 0xFE
    assert scales[0].tolist() == golden_kat["codebook_scales"]
    np.testing.assert_array_equal(oracle.decode(packed, scales, 1.0, 16), values)


def test_midpoints_use_even_code(golden_kat):
    # tests/test_cpu_contracts.py:27-29
    mags = [oracle.e2m1_code(v) & 7 for v in golden_kat["midpoints"]]
    assert mags == golden_kat["midpoint_magnitudes"] == [0, 2, 2, 4, 4, 6, 6]


def test_zero_groups_finite(golden_kat):
    # tests/test_cpu_contracts.py:32-35
    _, packed, scales, _ = oracle.encode(np.zeros((2, 256), np.float32), 1.0)
    out = oracle.decode(packed, scales, 1.0, 256)
    assert np.isfinite(out).all() and not out.any()
    assert golden_kat["zeros_packed_nonzero"] == 0 and golden_kat["zeros_scales_nonzero"] == 0


def test_codec_cases_bit_exact(codec_cases):
    data, names = codec_cases
    for name in names:
        x, g = data[f"{name}__x"], float(data[f"{name}__g"][0])
        nib, packed, scales, stats = oracle.encode(x, g)
        np.testing.assert_array_equal(packed, data[f"{name}__packed"], err_msg=name)
        np.testing.assert_array_equal(scales, data[f"{name}__scales"], err_msg=name)
        np.testing.assert_array_equal(nib, data[f"{name}__nib"], err_msg=name)
        dec = oracle.decode(packed, scales, g, x.shape[1])
        np.testing.assert_array_equal(dec.view(np.uint32), data[f"{name}__decoded"].view(np.uint32), err_msg=name)
        ref_stats = data[f"{name}__stats"]
        assert stats["clip6_rate"] == pytest.approx(ref_stats[0], rel=1e-6, abs=1e-9), name
        assert stats["blockscale_sat_rate"] == pytest.approx(ref_stats[1], rel=1e-6, abs=1e-9), name


def test_zero_scale_groups_saturate_like_the_oracle(codec_cases):
    # The reference codec oracle (oracle.py:57) divides by clamp_min(1e-30) when a
    # group scale rounds to 0, saturating nonzero codes to +-6; its Triton writer
    # writes 0 instead.  This build follows the oracle.
    data, _ = codec_cases
    packed = data["zero_scale_groups__packed"]
    scales = data["zero_scale_groups__scales"]
    assert (scales == 0).any()
    nib_lo = packed & 0xF
    assert ((nib_lo & 7) == 7).any()


def test_e4m3_conversion_matches_torch():
    # Dense sample of [0, 448] plus every representable value and midpoint.
    rng = np.random.default_rng(5)
    reps = np.array([oracle.e4m3_to_f32(b) for b in range(0x7F)], np.float64)
    mids = (reps[:-1] + reps[1:]) / 2
    probes = np.concatenate([reps, mids, np.nextafter(mids, 0), np.nextafter(mids, 1e9),
                             rng.uniform(0, 448, 20000), rng.uniform(0, 0.02, 20000)]).astype(np.float32)
    probes = np.clip(probes, 0, 448).astype(np.float32)
    expected = torch.from_numpy(probes).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([oracle.f32_to_e4m3(float(v)) for v in probes], np.uint8)
    np.testing.assert_array_equal(got, expected)


def test_codec_config_hashes(golden_hashes):
    # Config: K/V [4096, 2, 256] N(0,1), channels 7/64/130/201 x16, g = 1.
    ref = golden_hashes["codec"]
    k, v = W.codec_config(seed=ref["seed"], tokens=ref["tokens"])
    assert sha(k) == ref["key_input_sha256"] and sha(v) == ref["value_input_sha256"]
    for name, bits in (("key", k), ("value", v)):
        x = W.bf16_bits_to_f32(bits).reshape(-1, 256)
        _, packed, scales, _ = oracle.encode(x, 1.0)
        assert sha(packed) == ref[f"{name}_packed_sha256"], name
        assert sha(scales) == ref[f"{name}_scale_sha256"], name


def test_prefill_config_storage_hash(golden_hashes):
    # Config: 8192 tokens, 2% x32 outliers, cache 64 x 3136, random free slots.
    ref = golden_hashes["prefill"]
    k, v, slots = W.prefill_config(seed=ref["seed"], tokens=ref["tokens"], blocks=ref["blocks"], page=ref["page"])
    assert sha(k) == ref["key_input_sha256"] and sha(slots) == ref["slots_sha256"]
    storage = np.zeros((ref["blocks"], 2, ref["page"], 288), np.uint8)
    oracle.write_cache(k, v, storage, slots)
    assert sha(storage) == ref["storage_sha256"]


def test_attention_cases_match_reference(attention_cases):
    data, names = attention_cases
    for name in names:
        gk, gv = (float(s) for s in data[f"{name}__scales"])
        out = oracle.sparse_attention(data[f"{name}__q"], data[f"{name}__storage"], data[f"{name}__indices"],
                                      data[f"{name}__block_table"], data[f"{name}__t2r"], gk, gv)
        np.testing.assert_allclose(out, data[f"{name}__expected"], rtol=0, atol=1e-5, err_msg=name)


def test_bf16_attention_cases_match_reference(bf16_attention_cases):
    # The BF16 sibling reader's oracle against the reference's qsa_reference on bf16 caches.
    data, names = bf16_attention_cases
    assert len(names) >= 5
    for name in names:
        kv = data[f"{name}__kv"]                      # [blocks, kv_heads, page, 512] as vLLM allocates it
        cache = kv.transpose(0, 2, 1, 3)              # [blocks, page, kv_heads, 512] view (forward_qsa's split)
        out = oracle.sparse_attention_bf16(data[f"{name}__q"], cache[..., :256], cache[..., 256:],
                                           data[f"{name}__indices"], data[f"{name}__block_table"],
                                           data[f"{name}__t2r"])
        np.testing.assert_allclose(out, data[f"{name}__expected"], rtol=0, atol=1e-5, err_msg=name)


def test_decode_config_matches_reference(decode_golden):
    case = W.decode_config(seed=2)
    storage = np.zeros((case.blocks, 2, case.page, 288), np.uint8)
    oracle.write_cache(case.key, case.value, storage, case.slots)
    assert sha(storage) == str(decode_golden["storage_sha256"])
    out = oracle.sparse_attention(case.query, storage, case.indices, case.block_table, case.token_to_request)
    np.testing.assert_allclose(out, decode_golden["expected"], rtol=0, atol=1e-5)


def test_planted_mistake_is_caught(codec_cases):
    # The checker must notice a one-bit difference: flip a nibble in the oracle's output.
    data, _ = codec_cases
    _, packed, _, _ = oracle.encode(data["normal_amp_1__x"], 1.0)
    packed = packed.copy()
    packed[3, 7] ^= 0x1
    assert not np.array_equal(packed, data["normal_amp_1__packed"])
