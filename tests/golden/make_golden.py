#!/usr/bin/env python3
"""Generate the golden vectors in tests/golden/ from the REFERENCE implementation.

Runs where a checkout of the reference is available, named by --reference PATH
or $NVQSA_REFERENCE (one of the two is required).  It imports the reference's
own CPU code:
  src/nvfp4_oracle.py  encode / decode / global_scale_for / _round_e2m1_magnitude
  src/qsa_ref.py       qsa_reference (float64 sparse paged GQA)
and records their outputs on seeded inputs (numpy PCG64, see
nvfp4_qsa/workloads.py) so that machines without the reference (the GPU box)
can check bit-exactness.  Cache bytes for attention cases are assembled by
scattering the reference encoder's per-(token, head) bytes into the
[blocks, kv_heads, page, 288] layout of python/nvfp4_qsa/cache.py:20-24.

Outputs: kat.json, codec_cases.npz, config_hashes.json, attention_cases.npz,
bf16_attention_cases.npz, decode_config.npz.  Re-running with the same reference reproduces them exactly.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "nvfp4-qsa_b200"))
from nvfp4_qsa import workloads as W  # noqa: E402

HD, KVH, QH = 256, 2, 24


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits_to_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class Ref:
    def __init__(self, root: Path):
        sys.path.insert(0, str(root / "src"))
        import nvfp4_oracle  # noqa: F401
        import qsa_ref  # noqa: F401
        self.o = sys.modules["nvfp4_oracle"]
        self.q = sys.modules["qsa_ref"]

    def encode_bits(self, bits: np.ndarray, g: float):
        """bf16 bits [..., n] -> (nib, packed, scale, stats) from the reference encoder."""
        x = bits_to_tensor(bits.reshape(-1, bits.shape[-1])).float()
        nib, packed, scale, stats = self.o.encode(x, torch.tensor(np.float32(g)))
        return nib.numpy(), packed.numpy(), scale.numpy(), stats

    def storage(self, key_bits, value_bits, slots, blocks, page, gk=1.0, gv=1.0):
        """Reference bytes scattered into a [blocks, kvh, page, 288] uint8 cache."""
        tokens, kvh, hd = key_bits.shape
        st = np.zeros((blocks, kvh, page, 2 * (hd // 2 + hd // 16)), np.uint8)
        region = hd // 2 + hd // 16
        for r, (bits, g) in enumerate(((key_bits, gk), (value_bits, gv))):
            _, packed, scale, _ = self.encode_bits(bits, g)
            packed = packed.reshape(tokens, kvh, hd // 2)
            scale = scale.reshape(tokens, kvh, hd // 16)
            for t in range(tokens):
                s = int(slots[t])
                if s < 0 or s // page >= blocks:
                    continue
                b, o = divmod(s, page)
                st[b, :, o, r * region:r * region + hd // 2] = packed[t]
                st[b, :, o, r * region + hd // 2:(r + 1) * region] = scale[t]
        return st

    def decoded_caches(self, storage, gk=1.0, gv=1.0):
        blocks, kvh, page, _ = storage.shape
        region = HD // 2 + HD // 16
        out = []
        for r, g in ((0, gk), (1, gv)):
            packed = torch.from_numpy(storage[..., r * region:r * region + HD // 2].reshape(-1, HD // 2).copy())
            scale = torch.from_numpy(storage[..., r * region + HD // 2:(r + 1) * region].reshape(-1, HD // 16).copy())
            dec = self.o.decode(packed, scale, torch.tensor(np.float32(g)), HD)
            out.append(dec.reshape(blocks, kvh, page, HD).transpose(1, 2).contiguous())
        return out

    def attention(self, q_bits, storage, indices, block_table, t2r, page, gk=1.0, gv=1.0):
        kc, vc = self.decoded_caches(storage, gk, gv)
        q = bits_to_tensor(q_bits).float()
        rows = q.shape[0]
        out = np.zeros((rows, q.shape[1], HD), np.float32)
        for r in range(rows):  # rows with an out-of-range request are zeros (kernels.py:209-210, 245-246)
            req = int(t2r[r])
            if req < 0 or req >= block_table.shape[0]:
                continue
            res = self.q.qsa_reference(q[r:r + 1], kc, vc, torch.from_numpy(indices[r:r + 1].astype(np.int64)),
                                       torch.from_numpy(block_table.astype(np.int64)),
                                       torch.tensor([req]), page)
            out[r] = res["out"][0].numpy()
        return out


def make_kat(ref: Ref):
    values = torch.tensor([[0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6]])
    _, packed, scales, _ = ref.o.encode(values, torch.tensor(1.0))
    mid = torch.tensor([.25, .75, 1.25, 1.75, 2.5, 3.5, 5.0])
    _, zp, zs, _ = ref.o.encode(torch.zeros(2, 256), torch.tensor(1.0))
    return {
        "codebook_values": values[0].tolist(),
        "codebook_packed": packed[0].tolist(),
        "codebook_scales": scales[0].tolist(),
        "midpoints": mid.tolist(),
        "midpoint_magnitudes": ref.o._round_e2m1_magnitude(mid).tolist(),
        "zeros_packed_nonzero": int(zp.count_nonzero()),
        "zeros_scales_nonzero": int(zs.count_nonzero()),
    }


def codec_inputs():
    """Named fp32 inputs [rows, 256] and global scales for the flat codec."""
    rng = np.random.default_rng(1234)
    cases = {}
    for amp in (0.0, 1e-4, 1.0, 1e4):  # tests/test_gpu_portable.py:9 amplitudes
        x = W.bf16_bits_to_f32(W.f32_to_bf16_bits(rng.standard_normal((16, HD), dtype=np.float32) * amp))
        cases[f"normal_amp_{amp:g}"] = (x, 1.0)
    for dist in ("heavytail", "outliers", "normal"):
        x = W.bf16_bits_to_f32(W.f32_to_bf16_bits(W.gen_values(rng, (16, HD), dist)))
        g = float((448.0 * 6.0) / np.float32(max(np.abs(x).max(), 1e-8)))
        cases[f"{dist}_gscale"] = (x, float(np.float32(g)))
    # exact E2M1 midpoints at scale 1 (group amax 6 -> block scale exactly 1)
    mids = np.array([6.0, .25, .75, 1.25, 1.75, 2.5, 3.5, 5.0, -.25, -.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0],
                    np.float32)
    ties = np.stack([mids * (2.0 ** k) for k in range(-4, 12)]).astype(np.float32)
    cases["ties_pow2"] = (np.tile(ties, (1, HD // 16)), 1.0)
    # plain fp32 (not bf16-representable) values with a non-unit global scale
    cases["fp32_g3"] = (rng.standard_normal((16, HD), dtype=np.float32) * 3, 3.0)
    # infinities: the group scale saturates to 448, inf -> +-6
    inf = rng.standard_normal((4, HD), dtype=np.float32)
    inf[0, 3], inf[1, 40], inf[2, 17], inf[3, 255] = np.inf, -np.inf, np.inf, -np.inf
    cases["infinities"] = (inf, 1.0)
    # subnormal-scale groups: scale rounds to 0 -> oracle saturates codes (oracle.py:57)
    tiny = rng.standard_normal((4, HD), dtype=np.float32) * 1e-6
    cases["zero_scale_groups"] = (tiny, 1.0)
    return cases


def make_codec_cases(ref: Ref):
    arrays = {}
    for name, (x, g) in codec_inputs().items():
        nib, packed, scale, stats = ref.o.encode(torch.from_numpy(x), torch.tensor(np.float32(g)))
        dec = ref.o.decode(packed, scale, torch.tensor(np.float32(g)), HD)
        arrays[f"{name}__x"] = x
        arrays[f"{name}__g"] = np.array([g], np.float32)
        arrays[f"{name}__nib"] = nib.numpy()
        arrays[f"{name}__packed"] = packed.numpy()
        arrays[f"{name}__scales"] = scale.numpy()
        arrays[f"{name}__decoded"] = dec.numpy()
        arrays[f"{name}__stats"] = np.array([stats["clip6_rate"], stats["blockscale_sat_rate"]], np.float64)
    np.savez_compressed(HERE / "codec_cases.npz", **arrays)
    return sorted({k.split("__")[0] for k in arrays})


def make_config_hashes(ref: Ref):
    out = {}
    k, v = W.codec_config(seed=0)
    out["codec"] = {"seed": 0, "tokens": 4096, "key_input_sha256": sha(k), "value_input_sha256": sha(v)}
    for name, bits in (("key", k), ("value", v)):
        _, packed, scale, stats = ref.encode_bits(bits, 1.0)
        out["codec"][f"{name}_packed_sha256"] = sha(packed)
        out["codec"][f"{name}_scale_sha256"] = sha(scale)
        out["codec"][f"{name}_stats"] = stats
        out["codec"][f"{name}_packed_row0"] = packed[0].tolist()
        out["codec"][f"{name}_scale_row0"] = scale[0].tolist()
    k, v, slots = W.prefill_config(seed=3)
    storage = ref.storage(k, v, slots, 64, 3136)
    out["prefill"] = {"seed": 3, "tokens": 8192, "blocks": 64, "page": 3136,
                      "key_input_sha256": sha(k), "value_input_sha256": sha(v), "slots_sha256": sha(slots),
                      "storage_sha256": sha(storage), "storage_nonzero": int(np.count_nonzero(storage))}
    return out


def attention_case(ref, name, key, value, slots, blocks, page, q, idx, bt, t2r, gk=1.0, gv=1.0):
    storage = ref.storage(key, value, slots, blocks, page, gk, gv)
    exp = ref.attention(q, storage, idx, bt, t2r, page, gk, gv)
    return {f"{name}__storage": storage, f"{name}__q": q, f"{name}__indices": idx.astype(np.int32),
            f"{name}__block_table": bt.astype(np.int32), f"{name}__t2r": t2r.astype(np.int32),
            f"{name}__scales": np.array([gk, gv], np.float32), f"{name}__expected": exp}


def make_attention_cases(ref: Ref):
    arrays = {}
    rng = np.random.default_rng(37)
    # fragmented pages (tests/test_gpu_portable.py:43-65 shape): 4 blocks of 16, two rows
    key = W.f32_to_bf16_bits(rng.standard_normal((32, KVH, HD), dtype=np.float32))
    value = W.f32_to_bf16_bits(rng.standard_normal((32, KVH, HD), dtype=np.float32))
    slots = np.concatenate([np.arange(32, 48), np.arange(0, 16)]).astype(np.int64)
    q = W.f32_to_bf16_bits(rng.standard_normal((2, QH, HD), dtype=np.float32))
    idx = np.array([[0, 5, 12, 17, 31], [1, 8, 15, 16, 29]], np.int32)
    arrays.update(attention_case(ref, "fragmented", key, value, slots, 4, 16, q, idx,
                                 np.array([[2, 0]]), np.zeros(2)))
    # invalid metadata -> zeros (tests/test_gpu_portable.py:33-41)
    q1 = W.f32_to_bf16_bits(np.ones((3, QH, HD), np.float32))
    arrays.update(attention_case(ref, "invalid_metadata", key[:1] * 0, value[:1] * 0, np.array([0], np.int64), 1, 16,
                                 q1, np.array([[-1, 999], [-1, -1], [0, 1]]), np.array([[0]]), np.array([0, 0, 99])))
    # boundary and adversarial cells (src/boundary_matrix.py:36-57, src/sanitizer_target.py:17-22)
    cells = [
        ("ctx17_outliers", 17, 4, 17, "outliers", 1, False, False, 1.0, 1.0),
        ("topk_gt_ctx_heavytail", 64, 2, 70, "heavytail", 1, True, False, 1.0, 1.0),
        ("adversarial_multireq", 256, 4, 64, "normal", 2, True, True, 1.0, 1.0),
        ("duplicates_gscale", 300, 3, 96, "normal", 1, False, False, 2.5, 0.75),
        ("zeros_dist", 64, 2, 32, "zeros", 1, False, False, 1.0, 1.0),
    ]
    for cell_seed, (name, ctx, rows, topk, dist, nreq, frag, adversarial, gk, gv) in enumerate(cells, start=101):
        crng = np.random.default_rng(cell_seed)
        table, blocks, req_slots = W.paged_requests(crng, [ctx] * nreq, 16, extra_blocks=1, fragmented=frag)
        toks = nreq * ctx
        key = W.f32_to_bf16_bits(W.gen_values(crng, (toks, KVH, HD), dist))
        value = W.f32_to_bf16_bits(W.gen_values(crng, (toks, KVH, HD), dist))
        slots = np.concatenate(req_slots)
        q = W.f32_to_bf16_bits(W.gen_values(crng, (rows, QH, HD), "normal"))
        t2r = (np.arange(rows) % nreq).astype(np.int32)
        idx = np.full((rows, topk), -1, np.int32)
        for r in range(rows):
            forced = [0, 1, 15, 16, 17, ctx - 1]
            pool = crng.permutation(ctx)[:topk]
            sel = np.unique(np.concatenate([[f for f in forced if f < ctx], pool]))[:topk]
            idx[r, :sel.size] = sel
        if name.startswith("duplicates"):
            idx[0, :] = 5  # one logical token selected in every column (boundary_matrix.py:19-20)
            idx[1, : topk // 2] = idx[1, topk // 2: 2 * (topk // 2)]
        if adversarial:
            idx[0, 0], idx[0, 1], idx[0, 2] = -1, ctx + 999, 2 ** 31 - 1
            idx[1, :] = -1
            t2r[3] = -1
        arrays.update(attention_case(ref, name, key, value, slots, blocks, 16, q, idx, table, t2r, gk, gv))
    np.savez_compressed(HERE / "attention_cases.npz", **arrays)
    return sorted({k.split("__")[0] for k in arrays})


def make_bf16_attention_cases(ref: Ref):
    """The BF16 sibling reader's pin: src/qsa_ref.py:qsa_reference on bf16 caches (no quantisation).

    Each case stores the raw cache as vLLM allocates it, bf16 bits [blocks, kv_heads, page, 2 * 256] (K then V
    per token), whose K / V views [blocks, page, kv_heads, 256] are what the reader takes.
    """
    arrays = {}
    cells = [
        ("bf16_fragmented", 32, 2, 5, "normal", 1, True, False, False),
        ("bf16_ctx17_outliers", 17, 4, 17, "outliers", 1, False, False, False),
        ("bf16_adversarial_multireq", 256, 4, 64, "normal", 2, True, True, False),
        ("bf16_duplicates", 300, 3, 96, "normal", 1, False, False, True),
        ("bf16_heavytail_topk_gt_ctx", 64, 2, 70, "heavytail", 1, True, False, False),
    ]
    for cell_seed, (name, ctx, rows, topk, dist, nreq, frag, adversarial, dup) in enumerate(cells, start=301):
        crng = np.random.default_rng(cell_seed)
        page = 16
        table, blocks, req_slots = W.paged_requests(crng, [ctx] * nreq, page, extra_blocks=1, fragmented=frag)
        toks = nreq * ctx
        key = W.f32_to_bf16_bits(W.gen_values(crng, (toks, KVH, HD), dist))
        value = W.f32_to_bf16_bits(W.gen_values(crng, (toks, KVH, HD), dist))
        kv = np.zeros((blocks, KVH, page, 2 * HD), np.uint16)
        slots = np.concatenate(req_slots)
        kv[slots // page, :, slots % page, :HD] = key
        kv[slots // page, :, slots % page, HD:] = value
        q = W.f32_to_bf16_bits(W.gen_values(crng, (rows, QH, HD), "normal"))
        t2r = (np.arange(rows) % nreq).astype(np.int32)
        idx = np.full((rows, topk), -1, np.int32)
        for r in range(rows):
            forced = [0, 1, 15, 16, 17, ctx - 1]
            pool = crng.permutation(ctx)[:topk]
            sel = np.unique(np.concatenate([[f for f in forced if f < ctx], pool]))[:topk]
            idx[r, :sel.size] = sel
        if dup:
            idx[0, :] = 5
            idx[1, : topk // 2] = idx[1, topk // 2: 2 * (topk // 2)]
        if adversarial:
            idx[0, 0], idx[0, 1], idx[0, 2] = -1, ctx + 999, 2 ** 31 - 1
            idx[1, :] = -1
            t2r[3] = -1
        cache = bits_to_tensor(kv).transpose(1, 2)  # [blocks, page, kvh, 512] view, as forward_qsa splits it
        kc, vc = cache[..., :HD], cache[..., HD:]
        qt = bits_to_tensor(q)
        out = np.zeros((rows, QH, HD), np.float32)
        for r in range(rows):  # rows with an out-of-range request are zeros
            req = int(t2r[r])
            if req < 0 or req >= table.shape[0]:
                continue
            res = ref.q.qsa_reference(qt[r:r + 1], kc, vc, torch.from_numpy(idx[r:r + 1].astype(np.int64)),
                                      torch.from_numpy(table.astype(np.int64)), torch.tensor([req]), page)
            out[r] = res["out"][0].numpy()
        arrays.update({f"{name}__kv": kv, f"{name}__q": q, f"{name}__indices": idx,
                       f"{name}__block_table": table.astype(np.int32), f"{name}__t2r": t2r,
                       f"{name}__expected": out})
    np.savez_compressed(HERE / "bf16_attention_cases.npz", **arrays)
    return sorted({k.split("__")[0] for k in arrays})


def make_decode_config(ref: Ref):
    case = W.decode_config(seed=2)
    storage = ref.storage(case.key, case.value, case.slots, case.blocks, case.page)
    exp = ref.attention(case.query, storage, case.indices, case.block_table, case.token_to_request, case.page)
    np.savez_compressed(HERE / "decode_config.npz", expected=exp, storage_sha256=np.array(sha(storage)),
                        query=case.query, indices=case.indices)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NVQSA_REFERENCE"),
                    help="checkout of badbat4560/nvfp4-qsa (default: $NVQSA_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference PATH or NVQSA_REFERENCE")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = Ref(Path(args.reference))
    manifest = {"generator": "tests/golden/make_golden.py", "reference_files": [
        "src/nvfp4_oracle.py", "src/qsa_ref.py"], "torch": torch.__version__, "numpy": np.__version__}
    (HERE / "kat.json").write_text(json.dumps(make_kat(ref), indent=1) + "\n")
    manifest["codec_cases"] = make_codec_cases(ref)
    (HERE / "config_hashes.json").write_text(json.dumps(make_config_hashes(ref), indent=1) + "\n")
    manifest["attention_cases"] = make_attention_cases(ref)
    manifest["bf16_attention_cases"] = make_bf16_attention_cases(ref)
    make_decode_config(ref)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
