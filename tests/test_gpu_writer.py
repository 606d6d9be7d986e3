"""GPU: the sm_100a NVFP4 writer is bit-exact with the reference codec.

Checks against the reference's golden vectors (tests/golden/) and against the
pinned C oracle; ports the reference's writer tests (tests/test_gpu_portable.py:9-31)
and write gates W1/W4/W5 (slice5/src/w_validate.py) with byte equality in place
of decoded-value or cosine gates.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import bits_to_cuda, cuda_to_bits, gpu_write, regions, sha
from nvfp4_qsa import PackedCache, kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def oracle_storage(key_bits, value_bits, slots, blocks, page, gk=1.0, gv=1.0, head_dim=256):
    st = np.zeros((blocks, key_bits.shape[1], page, 2 * (head_dim // 2 + head_dim // 16)), np.uint8)
    oracle.write_cache(key_bits, value_bits, st, slots, gk, gv)
    return st


def test_codec_config_bytes_match_reference(golden_hashes):
    ref = golden_hashes["codec"]
    k, v = W.codec_config(seed=ref["seed"], tokens=ref["tokens"])
    cache = PackedCache(blocks=ref["tokens"] // 16)
    cache.write(bits_to_cuda(k), bits_to_cuda(v), torch.arange(ref["tokens"], dtype=torch.int64, device="cuda"))
    torch.cuda.synchronize()
    assert sha(cache.kd.reshape(-1, 128)) == ref["key_packed_sha256"]
    assert sha(cache.ks.reshape(-1, 16)) == ref["key_scale_sha256"]
    assert sha(cache.vd.reshape(-1, 128)) == ref["value_packed_sha256"]
    assert sha(cache.vs.reshape(-1, 16)) == ref["value_scale_sha256"]


def test_prefill_config_storage_matches_reference(golden_hashes):
    ref = golden_hashes["prefill"]
    k, v, slots = W.prefill_config(seed=ref["seed"], tokens=ref["tokens"], blocks=ref["blocks"], page=ref["page"])
    cache = PackedCache(blocks=ref["blocks"], page_size=ref["page"])
    cache.write(bits_to_cuda(k), bits_to_cuda(v), torch.from_numpy(slots).cuda())
    assert sha(cache.storage) == ref["storage_sha256"]


@pytest.mark.parametrize("amplitude", [0.0, 1e-4, 1.0, 10000.0])
def test_writer_amplitudes_and_slot_reuse(amplitude):
    # reference tests/test_gpu_portable.py:9-22, compared byte for byte
    rng = np.random.default_rng(42)
    key = W.f32_to_bf16_bits(rng.standard_normal((8, 2, 256), dtype=np.float32) * amplitude)
    slots = np.array([0, 1, 15, 16, 35, 63, -1, 64], np.int64)
    cache = PackedCache(4)
    cache.write(bits_to_cuda(key), bits_to_cuda(key), torch.from_numpy(slots).cuda())
    expect = oracle_storage(key, key, slots, 4, 16)
    np.testing.assert_array_equal(cache.storage.cpu().numpy(), expect)
    cache.write(torch.zeros(1, 2, 256, dtype=torch.bfloat16, device="cuda"),
                torch.zeros(1, 2, 256, dtype=torch.bfloat16, device="cuda"),
                torch.zeros(1, dtype=torch.int64, device="cuda"))
    assert not cache.kd[0, 0].any().item()


def test_guard_rejects_duplicate_and_nonfinite():
    # reference tests/test_gpu_portable.py:24-31
    cache = PackedCache(1)
    key = torch.zeros(2, 2, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="Duplicate"):
        cache.write(key, key, torch.zeros(2, dtype=torch.int64, device="cuda"))
    key[0, 0, 0] = float("nan")
    with pytest.raises(ValueError, match="Non-finite"):
        cache.write(key, key, torch.arange(2, dtype=torch.int64, device="cuda"))


def test_codec_cases_through_writer(codec_cases):
    data, names = codec_cases
    checked = 0
    for name in names:
        x, g = data[f"{name}__x"], float(data[f"{name}__g"][0])
        bits = W.f32_to_bf16_bits(x)
        if not np.array_equal(W.bf16_bits_to_f32(bits), x) or x.shape[0] % 2:
            continue  # the paged writer takes bf16 rows
        tokens = x.shape[0] // 2
        key = bits.reshape(tokens, 2, 256)
        cache = PackedCache(blocks=(tokens + 15) // 16, key_scale=g, value_scale=g)
        cache.write(bits_to_cuda(key), bits_to_cuda(key), torch.arange(tokens, dtype=torch.int64, device="cuda"))
        got_p = cache.kd.reshape(-1, 128)[: 2 * tokens].cpu().numpy()
        got_s = cache.ks.reshape(-1, 16)[: 2 * tokens].cpu().numpy()
        np.testing.assert_array_equal(got_p, data[f"{name}__packed"], err_msg=name)
        np.testing.assert_array_equal(got_s, data[f"{name}__scales"], err_msg=name)
        checked += 1
    assert checked >= 7


def test_infinite_and_tiny_values_follow_oracle():
    # +-inf saturate the group scale to 448 and the code to +-6; groups whose
    # scale rounds to zero saturate like the codec oracle (oracle.py:57).
    rng = np.random.default_rng(9)
    x = rng.standard_normal((6, 2, 256), dtype=np.float32)
    x[0, 0, 3], x[1, 1, 40], x[2, 0, 200] = np.inf, -np.inf, np.inf
    x[3:] *= 1e-6
    bits = W.f32_to_bf16_bits(x)
    slots = np.arange(6, dtype=np.int64)
    st = torch.zeros(1, 2, 16, 288, dtype=torch.uint8, device="cuda")
    gpu_write(st, bits_to_cuda(bits), bits_to_cuda(bits), torch.from_numpy(slots).cuda())
    np.testing.assert_array_equal(st.cpu().numpy(), oracle_storage(bits, bits, slots, 1, 16))


def test_slot_lifecycle_overwrite():
    # slice5/src/w_validate.py:167-200 (W4): overwrite slots, no stale bytes
    rng = np.random.default_rng(11)
    a = W.f32_to_bf16_bits(rng.standard_normal((64, 2, 256), dtype=np.float32))
    b = W.f32_to_bf16_bits(rng.standard_normal((3, 2, 256), dtype=np.float32) * 7)
    slots_a = rng.permutation(64).astype(np.int64)
    slots_b = np.array([15, 0, 47], np.int64)
    st = torch.zeros(4, 2, 16, 288, dtype=torch.uint8, device="cuda")
    gpu_write(st, bits_to_cuda(a), bits_to_cuda(a[::-1].copy()), torch.from_numpy(slots_a).cuda())
    gpu_write(st, bits_to_cuda(b), bits_to_cuda(b), torch.from_numpy(slots_b).cuda())
    exp = oracle_storage(a, a[::-1].copy(), slots_a, 4, 16)
    oracle.write_cache(b, b, exp, slots_b)
    np.testing.assert_array_equal(st.cpu().numpy(), exp)


@pytest.mark.parametrize("tokens", [1, 2, 15, 16, 17, 64, 256])
@pytest.mark.parametrize("dist", ["zeros", "normal", "heavytail", "outliers"])
def test_boundary_matrix(tokens, dist):
    # slice5/src/w_validate.py:217-253 (W5) cells, byte-exact
    rng = np.random.default_rng(1000 + tokens)
    blocks = (18 + tokens + 15) // 16 + 1
    src = W.f32_to_bf16_bits(W.gen_values(rng, (tokens, 2, 256), dist))
    g = 1.0 if dist == "zeros" else float(np.float32(2688.0 / max(np.abs(W.bf16_bits_to_f32(src)).max(), 1e-8)))
    boundary = [-1, 0, 15, 16, 17, blocks * 16 - 1]
    slots = np.array((boundary[: min(6, tokens)] + list(range(18, 18 + tokens)))[:tokens], np.int64)
    slots = slots[rng.permutation(tokens)]
    st = torch.zeros(blocks, 2, 16, 288, dtype=torch.uint8, device="cuda")
    gpu_write(st, bits_to_cuda(src), bits_to_cuda(src), torch.from_numpy(slots).cuda(), g, g)
    np.testing.assert_array_equal(st.cpu().numpy(), oracle_storage(src, src, slots, blocks, 16, g, g))


def test_generic_strides_and_separate_regions():
    # Non-canonical layout: separate padded K/V tensors, strided sources.
    rng = np.random.default_rng(21)
    big = torch.from_numpy(W.f32_to_bf16_bits(rng.standard_normal((40, 3, 384), dtype=np.float32)).view(np.int16))
    big = big.view(torch.bfloat16).cuda()
    key, value = big[:, :2, :256], big[:, 1:, 128:]
    slots = torch.from_numpy(rng.permutation(96)[:40].astype(np.int64)).cuda()
    kbuf = torch.zeros(6, 16, 2, 160, dtype=torch.uint8, device="cuda")
    vbuf = torch.zeros(6, 16, 2, 176, dtype=torch.uint8, device="cuda")
    kd, ks = kbuf[..., :128], kbuf[..., 144:160]
    vd, vs = vbuf[..., 16:144], vbuf[..., 160:176]
    kernels.qsa_write_cache_nvfp4(key, value, kd, ks, vd, vs, slots, 1.0, 2.0)
    kb, vb = cuda_to_bits(key), cuda_to_bits(value)
    exp = oracle_storage(kb, vb, slots.cpu().numpy(), 6, 16, 1.0, 2.0)
    ekd, eks, evd, evs = regions(torch.from_numpy(exp))
    np.testing.assert_array_equal(kd.cpu().numpy(), ekd.numpy())
    np.testing.assert_array_equal(ks.cpu().numpy(), eks.numpy())
    np.testing.assert_array_equal(vd.cpu().numpy(), evd.numpy())
    np.testing.assert_array_equal(vs.cpu().numpy(), evs.numpy())


@pytest.mark.parametrize("head_dim", [64, 128, 512])
def test_other_head_dims(head_dim):
    rng = np.random.default_rng(head_dim)
    src = W.f32_to_bf16_bits(W.gen_values(rng, (20, 2, head_dim), "heavytail"))
    slots = rng.permutation(32)[:20].astype(np.int64)
    width = 2 * (head_dim // 2 + head_dim // 16)
    st = torch.zeros(2, 2, 16, width, dtype=torch.uint8, device="cuda")
    gpu_write(st, bits_to_cuda(src), bits_to_cuda(src[::-1].copy()), torch.from_numpy(slots).cuda())
    exp = oracle_storage(src, src[::-1].copy(), slots, 2, 16, head_dim=head_dim)
    np.testing.assert_array_equal(st.cpu().numpy(), exp)


def test_write_inside_cuda_graph():
    rng = np.random.default_rng(5)
    src = bits_to_cuda(W.f32_to_bf16_bits(rng.standard_normal((48, 2, 256), dtype=np.float32)))
    slots = torch.from_numpy(rng.permutation(64)[:48].astype(np.int64)).cuda()
    st = torch.zeros(4, 2, 16, 288, dtype=torch.uint8, device="cuda")
    eager = torch.zeros_like(st)
    gpu_write(eager, src, src, slots)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gpu_write(st, src, src, slots)  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    st.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gpu_write(st, src, src, slots)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(st, eager)


def test_raw_op_type_errors():
    st = torch.zeros(1, 2, 16, 288, dtype=torch.uint8, device="cuda")
    kd, ks, vd, vs = regions(st)
    k = torch.zeros(1, 2, 256, dtype=torch.bfloat16, device="cuda")
    slots = torch.zeros(1, dtype=torch.int64, device="cuda")
    with pytest.raises(TypeError, match="BF16"):
        kernels.qsa_write_cache_nvfp4(k.float(), k, kd, ks, vd, vs, slots, 1.0, 1.0)
    with pytest.raises(TypeError, match="int64"):
        kernels.qsa_write_cache_nvfp4(k, k, kd, ks, vd, vs, slots.int(), 1.0, 1.0)
    with pytest.raises(ValueError, match="group-scale"):
        kernels.qsa_write_cache_nvfp4(k, k, kd, ks[..., :8], vd, vs, slots, 1.0, 1.0)


def test_division_by_six_matches_ieee_for_every_float(tmp_path):
    # The writer's group scale g * amax / 6 (oracle.py:54) uses an FMA-corrected
    # product with RN(1/6); it must equal the IEEE division for all 2^32 inputs.
    import ctypes
    import os
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    so = tmp_path / "div6_check.so"
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                    "-I", os.path.join(root, "include"), "-I", os.path.join(root, "nvfp4-qsa_b200", "csrc"),
                    os.path.join(root, "tests", "cuda", "div6_check.cu"), "-o", str(so)], check=True)
    lib = ctypes.CDLL(str(so))
    bad = ctypes.c_ulonglong(0)
    first = (ctypes.c_uint * 8)()
    assert lib.div6_check(ctypes.byref(bad), first) == 0
    assert bad.value == 0, [hex(v) for v in first]


def _scale_sweep_inputs(rng, g, tokens=96, infinities=True):
    # group amplitudes log-uniform so that g * amax / 6 sweeps the E4M3 range
    # [2^-12, 2^10] (every scale byte, subnormals and saturation included),
    # plus all-zero groups, +-inf and NaN inputs
    x = rng.standard_normal((tokens, 2, 256)).astype(np.float32)
    x /= np.maximum(np.abs(x).reshape(tokens, 2, 16, 16).max(-1, keepdims=True), 1e-30).repeat(16, -1).reshape(x.shape)
    amp = 6.0 * np.exp2(rng.uniform(-12, 10, (tokens, 2, 16))) / abs(g)
    x *= np.minimum(amp, 1e38).astype(np.float32).repeat(16, -1)
    x[::7, 0, :16] = 0.0
    if infinities:
        x[3, 1, 20] = np.inf
        x[5, 0, 100] = -np.inf
    x[9, 1, 200] = np.nan
    return W.f32_to_bf16_bits(x)


@pytest.mark.parametrize("gk,gv", [(1.0, 1.0), (0.37, 3e-5), (1e4, 2.0 ** -117), (2.0 ** -118, 1e30), (-2.0, 5e8),
                                   (2.0 ** 100, 2.0 ** 101), (-(2.0 ** -117), 1.5), (3e38, 0.0)])
def test_global_scales_across_the_scale_table_paths(gk, gv):
    # The per-CTA table g / max(e4m3(b), 1e-30) is built from g / k by exact
    # power-of-two scaling when 2^-117 <= |g| <= 2^100 and by direct division
    # otherwise; both must give the oracle's bytes, including groups whose
    # out_scale overflows to inf (zero groups with g >= 3.4e8 -> NaN -> code 0).
    # g = 0 gets no infinite inputs: 0 * inf is a NaN scale whose sign IEEE
    # leaves open (x86 gives 0xff, the GPU 0x7f; both decode to NaN).
    rng = np.random.default_rng(abs(hash((gk, gv))) % 2 ** 32)
    kb = _scale_sweep_inputs(rng, gk if gk != 0 else 1.0, infinities=gk != 0)
    vb = _scale_sweep_inputs(rng, gv if gv != 0 else 1.0, infinities=gv != 0)
    slots = rng.permutation(128)[:96].astype(np.int64)
    st = torch.zeros(8, 2, 16, 288, dtype=torch.uint8, device="cuda")
    gpu_write(st, bits_to_cuda(kb), bits_to_cuda(vb), torch.from_numpy(slots).cuda(), gk, gv)
    np.testing.assert_array_equal(st.cpu().numpy(), oracle_storage(kb, vb, slots, 8, 16, gk, gv))


@pytest.mark.parametrize("page", [1, 3, 7, 16, 1000, 3136, 65537])
def test_page_sizes_and_slot_edges(page):
    # slot -> (block, offset) is a multiply-shift division by the page size;
    # the last valid slot, one past it and negative slots at every page size
    rng = np.random.default_rng(page)
    blocks = max(2, 64 // page + 1)
    n = blocks * page
    tokens = 40
    src = W.f32_to_bf16_bits(rng.standard_normal((tokens, 2, 256), dtype=np.float32))
    # distinct slots below the last one, then the last valid slot, one past the cache and a negative slot
    slots = np.concatenate([rng.permutation(n - 1)[:tokens - 4], [n - 1, n, n + page, -1]]).astype(np.int64)
    slots = slots[rng.permutation(tokens)]
    st = torch.zeros(blocks, 2, page, 288, dtype=torch.uint8, device="cuda")
    gpu_write(st, bits_to_cuda(src), bits_to_cuda(src), torch.from_numpy(slots).cuda())
    np.testing.assert_array_equal(st.cpu().numpy(), oracle_storage(src, src, slots, blocks, page))


def test_block_stride_above_two_gib_takes_the_64_bit_path():
    # one block of 3.8M tokens: the block stride (2 x 3.8M x 288 B) exceeds 2^31,
    # so the writer uses 64-bit index arithmetic and the 64-bit slot division
    page = 3_800_000
    st = torch.zeros(1, 2, page, 288, dtype=torch.uint8, device="cuda")
    assert st.stride(0) > 2 ** 31
    rng = np.random.default_rng(17)
    tokens = 48
    src = W.f32_to_bf16_bits(rng.standard_normal((tokens, 2, 256), dtype=np.float32))
    slots = rng.choice(page, tokens, replace=False).astype(np.int64)
    slots[0], slots[1] = page - 1, page  # the last slot, and one past the cache (skipped)
    gpu_write(st, bits_to_cuda(src), bits_to_cuda(src), torch.from_numpy(slots).cuda())
    exp = oracle_storage(src, src, np.arange(tokens, dtype=np.int64), (tokens + 15) // 16, 16)
    exp = exp.transpose(0, 2, 1, 3).reshape(-1, 2, 288)[:tokens]
    valid = slots < page
    got = st[0].transpose(0, 1)[torch.from_numpy(slots[valid]).cuda()].cpu().numpy()
    np.testing.assert_array_equal(got, exp[valid])
    del st
    torch.cuda.empty_cache()


def test_negative_products_that_underflow_to_zero_get_code_zero():
    # y = x * out_scale rounds to -0 for a tiny negative x in a group whose
    # out_scale is tiny (small g, saturated scale): the oracle's sign is y < 0,
    # so the code is +0 (0x0), not -0 (0x8).  A fused x * s + 0 would keep the
    # sign of the exact product and write 0x8.
    x = np.zeros((4, 2, 256), np.float32)
    x[:, :, 0] = 2.0 ** 32  # amax: g * amax / 6 saturates the scale to 448
    x[:, :, 1] = -(2.0 ** -133)  # bf16 subnormal
    x[:, :, 2] = -(2.0 ** -126)
    x[:, :, 3] = -(2.0 ** -120)
    x[:, :, 4] = 2.0 ** -133
    x[:, :, 5] = -0.0
    x[:, :, 16:] = np.random.default_rng(3).standard_normal((4, 2, 240))
    bits = W.f32_to_bf16_bits(x)
    slots = np.arange(4, dtype=np.int64)
    for g in (2.0 ** -20, 2.0 ** -118, 1.0):  # slow path (table by scaling, by division); fast path with -0
        st = torch.zeros(1, 2, 16, 288, dtype=torch.uint8, device="cuda")
        gpu_write(st, bits_to_cuda(bits), bits_to_cuda(bits), torch.from_numpy(slots).cuda(), g, g)
        exp = oracle_storage(bits, bits, slots, 1, 16, g, g)
        if g == 2.0 ** -20:  # x0 -> +6 (code 7), x1, x2 underflow to -0 -> code 0, x3 rounds to -2^-149 -> 0x8
            assert exp[0, 0, 0, 0] == 0x07 and exp[0, 0, 0, 1] == 0x80 and exp[0, 0, 0, 2] == 0x00
        np.testing.assert_array_equal(st.cpu().numpy(), exp, err_msg=f"g={g}")


@pytest.mark.parametrize("kv_heads", [1, 3, 4])
def test_record_layout_with_other_head_counts(kv_heads):
    # one head (the upper half-warp idle), an odd count (the last pair has one head) and two pairs per token
    rng = np.random.default_rng(100 + kv_heads)
    tokens, blocks, page = 300, 24, 16
    key = W.f32_to_bf16_bits(rng.standard_normal((tokens, kv_heads, 256), dtype=np.float32) * 3)
    value = W.f32_to_bf16_bits(rng.standard_normal((tokens, kv_heads, 256), dtype=np.float32))
    slots = rng.permutation(blocks * page)[:tokens].astype(np.int64)
    slots[::37] = -1
    cache = PackedCache(blocks, page_size=page, kv_heads=kv_heads)
    cache.write(bits_to_cuda(key), bits_to_cuda(value), torch.from_numpy(slots).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.storage.cpu().numpy(), oracle_storage(key, value, slots, blocks, page))


@pytest.mark.parametrize("record", [289, 290, 292, 296])
def test_writer_takes_strides_that_are_not_word_multiples(record):
    # The reference's writer takes any block/token/head strides with a contiguous last dim
    # (python/nvfp4_qsa/kernels.py:132-150); records padded to 289..296 bytes make the packed rows unaligned to
    # the lane's 4-byte store, so the writer stores bytes.  The bytes must equal the canonical layout's.
    k, v, slots = W.prefill_config(seed=9, tokens=1024, blocks=8, page=256)
    compact = torch.zeros(8, 2, 256, 288, dtype=torch.uint8, device="cuda")
    gpu_write(compact, bits_to_cuda(k), bits_to_cuda(v), torch.from_numpy(slots).cuda())
    padded = torch.zeros(8, 2, 256, record, dtype=torch.uint8, device="cuda")
    gpu_write(padded[..., :288], bits_to_cuda(k), bits_to_cuda(v), torch.from_numpy(slots).cuda())
    torch.cuda.synchronize()
    assert torch.equal(padded[..., :288], compact)
    assert not padded[..., 288:].any()
