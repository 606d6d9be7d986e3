"""Seeded synthetic workloads for the benchmark configurations.

No public dataset is involved in this path; inputs are drawn with numpy's
PCG64 generator (bit-stable across machines, unlike some vectorised CPU
samplers), rounded to bf16 with round-to-nearest-even, and described by the
value distributions of the reference's harnesses (src/run_validation.py:73-86,
slice5/src/w_validate.py:203-214) and the benchmark configurations:

  codec      [4096, 2, 256] N(0,1), channels 7/64/130/201 x16, g = 1
  decode     1 row, 24 heads; cache of 32,768 tokens; 2,048 sorted indices
  prefill    [8192, 2, 256] N(0,1) with 2% of values x32; cache 64 x 3,136;
             slots = seeded permutation of the free slots
  mtp        12 sequences x 4 rows, context U[8,192, 169,984], page 3,136
  scale-out  96 sequences x 131,072 tokens x 12 layers; or one
             169,984-token sequence with 8,192 selections
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

HEAD_DIM = 256
KV_HEADS = 2
QUERY_HEADS = 24
RECORD_BYTES = 2 * (HEAD_DIM // 2 + HEAD_DIM // 16)  # 288 bytes per (token, kv head)
CODEC_OUTLIER_CHANNELS = (7, 64, 130, 201)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round-to-nearest-even, NaN kept quiet."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = np.where(nan, (u >> 16) | 0x40, rounded)
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def gen_values(rng: np.random.Generator, shape, dist: str = "normal") -> np.ndarray:
    """fp32 values with the reference harnesses' distributions."""
    if dist == "zeros":
        return np.zeros(shape, np.float32)
    if dist == "normal":
        return rng.standard_normal(shape, dtype=np.float32)
    if dist == "heavytail":  # 2% of values + N(0, 8)
        base = rng.standard_normal(shape, dtype=np.float32)
        spike = (rng.random(shape) < 0.02) * rng.standard_normal(shape, dtype=np.float32) * 8
        return (base + spike).astype(np.float32)
    if dist == "outliers":  # 0.5% of values +30 on 0.1 * N(0, 1)
        base = rng.standard_normal(shape, dtype=np.float32) * 0.1
        return (base + (rng.random(shape) < 0.005) * 30.0).astype(np.float32)
    raise ValueError(dist)


def codec_config(seed: int = 0, tokens: int = 4096):
    """Codec round-trip config: (K bits, V bits) bf16 [tokens, 2, 256]."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(2):
        x = rng.standard_normal((tokens, KV_HEADS, HEAD_DIM), dtype=np.float32)
        x[..., list(CODEC_OUTLIER_CHANNELS)] *= 16.0
        out.append(f32_to_bf16_bits(x))
    return out[0], out[1]


def prefill_config(seed: int = 3, tokens: int = 8192, blocks: int = 64, page: int = 3136):
    """Prefill write config: (K bits, V bits, slot_mapping int64)."""
    rng = np.random.default_rng(seed)
    kv = []
    for _ in range(2):
        x = rng.standard_normal((tokens, KV_HEADS, HEAD_DIM), dtype=np.float32)
        x = np.where(rng.random(x.shape) < 0.02, x * 32.0, x).astype(np.float32)
        kv.append(f32_to_bf16_bits(x))
    slots = rng.permutation(blocks * page)[:tokens].astype(np.int64)
    return kv[0], kv[1], slots


def rope_cos_sin(max_position: int, rotary_dim: int, base: float = 1.0e7) -> np.ndarray:
    """float32 [max_position, rotary_dim] cos | sin table built like vLLM's RotaryEmbedding cache.

    inv_freq = base^(-2i / rotary_dim), angle = position * inv_freq; the writer
    and vLLM's native path use it cast to bf16.  base 1e7 is Qwen3-Next's rope_theta.
    """
    inv = 1.0 / (base ** (np.arange(0, rotary_dim, 2, dtype=np.float64) / rotary_dim))
    ang = np.outer(np.arange(max_position, dtype=np.float64), inv).astype(np.float32)
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)


def projection_config(seed: int = 5, tokens: int = 8192, blocks: int = 64, page: int = 3136,
                      max_position: int = 262144, rotary_dim: int = 64):
    """K/V as they leave the QKV projection, before k_norm and RoPE (config 3's shape).

    Returns (K bits, V bits, slots int64, positions int64, cos_sin float32
    [max_position, rotary_dim], k_norm weight float32 [256]).  K rows carry a
    per-head magnitude spread like un-normalised projections (RMS 0.5 to 8),
    2 % outliers x32; the GemmaRMSNorm weight is small around 0 (scale 1 + w).
    """
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((tokens, KV_HEADS, HEAD_DIM), dtype=np.float32)
    k *= np.exp2(rng.uniform(-1, 3, (tokens, KV_HEADS, 1))).astype(np.float32)
    k = np.where(rng.random(k.shape) < 0.02, k * 32.0, k).astype(np.float32)
    v = rng.standard_normal((tokens, KV_HEADS, HEAD_DIM), dtype=np.float32)
    v = np.where(rng.random(v.shape) < 0.02, v * 32.0, v).astype(np.float32)
    slots = rng.permutation(blocks * page)[:tokens].astype(np.int64)
    positions = rng.integers(0, max_position, tokens).astype(np.int64)
    weight = bf16_bits_to_f32(f32_to_bf16_bits((rng.standard_normal(HEAD_DIM) * 0.1).astype(np.float32)))
    return (f32_to_bf16_bits(k), f32_to_bf16_bits(v), slots, positions, rope_cos_sin(max_position, rotary_dim),
            weight)


@dataclass
class DecodeCase:
    """A paged sparse-decode problem (CPU arrays; K/V as bf16 bits)."""

    key: np.ndarray            # uint16 [cache_tokens, kv_heads, head_dim]
    value: np.ndarray
    slots: np.ndarray          # int64 [cache_tokens]: token i of request r -> physical slot
    query: np.ndarray          # uint16 [rows, query_heads, head_dim]
    indices: np.ndarray        # int32 [rows, topk]
    block_table: np.ndarray    # int32 [requests, width]
    token_to_request: np.ndarray  # int32 [rows]
    blocks: int
    page: int


def paged_requests(rng, contexts, page, extra_blocks=0, fragmented=True):
    """Disjoint random block assignments for requests with the given contexts.

    Returns (block_table int32 [R, W], blocks, slots_per_request list of int64
    arrays mapping logical token -> physical slot)."""
    widths = [(c + page - 1) // page for c in contexts]
    total = sum(widths) + extra_blocks
    perm = rng.permutation(total) if fragmented else np.arange(total)
    width = max(widths) if widths else 1
    table = np.full((len(contexts), max(width, 1)), -1, np.int32)
    slots = []
    cursor = 0
    for r, (c, w) in enumerate(zip(contexts, widths)):
        blocks_r = perm[cursor:cursor + w].astype(np.int64)
        cursor += w
        table[r, :w] = blocks_r
        tok = np.arange(c, dtype=np.int64)
        slots.append(blocks_r[tok // page] * page + tok % page)
    return table, total, slots


def decode_config(seed: int = 2, context: int = 32768, topk: int = 2048, page: int = 16, rows: int = 1,
                  dist: str = "normal") -> DecodeCase:
    """Single-sequence sparse decode: `rows` query rows of one request."""
    rng = np.random.default_rng(seed)
    table, blocks, slots = paged_requests(rng, [context], page)
    key = f32_to_bf16_bits(gen_values(rng, (context, KV_HEADS, HEAD_DIM), dist))
    value = f32_to_bf16_bits(gen_values(rng, (context, KV_HEADS, HEAD_DIM), dist))
    query = f32_to_bf16_bits(gen_values(rng, (rows, QUERY_HEADS, HEAD_DIM), dist))
    idx = np.stack([np.sort(rng.choice(context, size=min(topk, context), replace=False)) for _ in range(rows)])
    if idx.shape[1] < topk:
        idx = np.concatenate([idx, np.full((rows, topk - idx.shape[1]), -1)], axis=1)
    return DecodeCase(key, value, slots[0], query, idx.astype(np.int32), table, np.zeros(rows, np.int32), blocks,
                      page)


def mtp_config(seed: int = 4, sequences: int = 12, rows_per_seq: int = 4, ctx_lo: int = 8192,
               ctx_hi: int = 169984, topk: int = 2048, page: int = 3136):
    """MTP decode batch metadata: contexts, block table, indices (shared per sequence)."""
    rng = np.random.default_rng(seed)
    contexts = rng.integers(ctx_lo, ctx_hi + 1, size=sequences)
    table, blocks, slots = paged_requests(rng, list(contexts), page)
    idx = np.stack([np.sort(rng.choice(int(c), size=topk, replace=False)) for c in contexts]).astype(np.int32)
    indices = np.repeat(idx, rows_per_seq, axis=0)
    t2r = np.repeat(np.arange(sequences, dtype=np.int32), rows_per_seq)
    return contexts, table, blocks, slots, indices, t2r
