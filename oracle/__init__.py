"""TEST INFRASTRUCTURE ONLY: CPU checker for the NVFP4 QSA CUDA path.

ctypes wrapper around ``oracle/nvfp4_oracle.c``, a plain-C restatement of the
reference's codec oracle (python/nvfp4_qsa/oracle.py:25-92), its paged writer
contract (python/nvfp4_qsa/kernels.py:46-165) and its sparse reader contract
(python/nvfp4_qsa/kernels.py:168-403; float64 math as src/qsa_ref.py:12-52).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` leg may
import this package, and only as the checker (or the timed CPU baseline).  The
product package ``nvfp4-qsa_b200/nvfp4_qsa`` never imports it.

Parity of this restatement is pinned to the reference itself by the vectors in
``tests/golden/`` (made by ``tests/golden/make_golden.py`` from the reference's
own Python code) and checked by ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from ctypes import c_float, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "nvfp4_oracle.c"
LIB = HERE / "_build" / "liboracle_nvfp4.so"

E2M1_GRID = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
E2M1_MAX = 6.0
E4M3_MAX = 448.0
GROUP = 16


def build(force: bool = False) -> Path:
    """Compile the C restatement with gcc (IEEE float, no contraction)."""
    if not force and LIB.exists() and LIB.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
           "-std=c11", str(SOURCE), "-o", str(tmp), "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"gcc failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        P, I64, I32, F = c_void_p, c_int64, c_int32, c_float
        lib.orc_f32_to_e4m3.restype = ctypes.c_uint8
        lib.orc_f32_to_e4m3.argtypes = [F]
        lib.orc_e4m3_to_f32.restype = F
        lib.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        lib.orc_e2m1_code.restype = ctypes.c_uint8
        lib.orc_e2m1_code.argtypes = [F]
        lib.orc_encode_rows.restype = None
        lib.orc_encode_rows.argtypes = [P, I64, I64, I32, F, P, P, P, P]
        lib.orc_decode_rows.restype = None
        lib.orc_decode_rows.argtypes = [P, P, I64, I64, I32, F, P]
        lib.orc_write_cache.restype = None
        lib.orc_write_cache.argtypes = [P, I64, I64, P, I64, I64,
                                        P, I64, I64, I64, P, I64, I64, I64,
                                        P, I64, I64, I64, P, I64, I64, I64,
                                        P, I64, I32, I32, I64, I64, F, F]
        lib.orc_sparse_attention.restype = None
        lib.orc_sparse_attention.argtypes = [P, I64, I64,
                                             P, I64, I64, I64, P, I64, I64, I64,
                                             P, I64, I64, I64, P, I64, I64, I64,
                                             I64, I64, I32, F, F,
                                             P, I64, P, I64, I64, P, P, I64, I32, I32, P]
        lib.orc_sparse_attention_fp8.restype = None
        lib.orc_sparse_attention_fp8.argtypes = [P, I64, I64, P, I64, I64, I64, P, I64, I64, I64,
                                                 I64, I64, I32, F, F,
                                                 P, I64, P, I64, I64, P, P, I64, I32, I32, P]
        lib.orc_sparse_attention_bf16.restype = None
        lib.orc_sparse_attention_bf16.argtypes = [P, I64, I64, P, I64, I64, I64, P, I64, I64, I64,
                                                  I64, I64, I32,
                                                  P, I64, P, I64, I64, P, P, I64, I32, I32, P]
        lib.orc_norm_rope.restype = None
        lib.orc_norm_rope.argtypes = [P, I64, I64, I64, I32, I32, P, F, F, P, P, I64, I64, I32, I32, P, P]
        lib.orc_set_threads.restype = None
        lib.orc_set_threads.argtypes = [c_int]
        lib.orc_get_threads.restype = c_int
        lib.orc_get_threads.argtypes = []
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def set_threads(n: int) -> None:
    _load().orc_set_threads(int(n))


def get_threads() -> int:
    return int(_load().orc_get_threads())


def f32_to_e4m3(x: float) -> int:
    return int(_load().orc_f32_to_e4m3(float(x)))


def e4m3_to_f32(b: int) -> float:
    return float(_load().orc_e4m3_to_f32(int(b)))


def e2m1_code(y: float) -> int:
    return int(_load().orc_e2m1_code(float(y)))


def encode(x2d, global_scale: float, block_size: int = GROUP):
    """oracle.py:47-69 on numpy fp32 [m, n]: (nibbles, packed, scale_u8, stats)."""
    x = np.ascontiguousarray(np.asarray(x2d, dtype=np.float32))
    m, n = x.shape
    nib = np.empty((m, n), np.uint8)
    packed = np.empty((m, n // 2), np.uint8)
    scales = np.empty((m, n // block_size), np.uint8)
    counts = np.zeros(2, np.int64)
    _load().orc_encode_rows(_ptr(x), m, n, block_size, float(np.float32(global_scale)), _ptr(nib), _ptr(packed),
                            _ptr(scales), _ptr(counts))
    total, groups = m * n, m * (n // block_size)
    stats = {"clip6_rate": counts[0] / total if total else math.nan,
             "blockscale_sat_rate": counts[1] / groups if groups else math.nan}
    return nib, packed, scales, stats


def decode(packed, scale_u8, global_scale: float, n: int, block_size: int = GROUP):
    """oracle.py:72-85: fp32 [m, n]."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scale_u8 = np.ascontiguousarray(scale_u8, dtype=np.uint8)
    m = packed.shape[0]
    out = np.empty((m, n), np.float32)
    _load().orc_decode_rows(_ptr(packed), _ptr(scale_u8), m, n, block_size, float(np.float32(global_scale)), _ptr(out))
    return out


def cache_regions(storage: np.ndarray, head_dim: int = 256):
    """Split a uint8 [blocks, kv_heads, page, 2*(hd/2+hd/16)] storage like cache.py:20-24.

    Returns four (array, (block, token, head) byte strides, byte offset) tuples
    describing key_data, key_scale, value_data, value_scale.
    """
    blocks, kvh, page, width = storage.shape
    region = head_dim // 2 + head_dim // 16
    sb, sh, st = storage.strides[0], storage.strides[1], storage.strides[2]
    offs = (0, head_dim // 2, region, region + head_dim // 2)
    return [(off, (sb, st, sh)) for off in offs]


def write_cache(key_bits: np.ndarray, value_bits: np.ndarray, storage: np.ndarray, slots: np.ndarray,
                key_global_scale: float = 1.0, value_global_scale: float = 1.0) -> None:
    """Writer contract (kernels.py:46-165) into a packed storage array, in place."""
    key_bits = np.ascontiguousarray(key_bits, dtype=np.uint16)
    value_bits = np.ascontiguousarray(value_bits, dtype=np.uint16)
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    assert storage.flags["C_CONTIGUOUS"] and storage.dtype == np.uint8
    tokens, kvh, hd = key_bits.shape
    blocks, _, page, _ = storage.shape
    regs = cache_regions(storage, hd)
    base = _ptr(storage)
    args = []
    for off, (sb, st, sh) in regs:
        args += [base + off, sb, st, sh]
    _load().orc_write_cache(_ptr(key_bits), kvh * hd, hd, _ptr(value_bits), kvh * hd, hd, *args, _ptr(slots),
                            tokens, kvh, hd, blocks, page, float(key_global_scale), float(value_global_scale))


def norm_rope(key_bits: np.ndarray, positions=None, cos_sin_bits=None, weight=None, offset: float = 1.0,
              eps: float = 1e-6, neox: bool = True):
    """K-norm + rotary embedding of bf16 K bits [tokens, kv_heads, head_dim] (the writer's fused prologue).

    Returns (bf16 bits [tokens, kv_heads, head_dim], valid [tokens] bool); rows of
    tokens whose position is outside the table are returned unchanged and not valid.
    """
    key_bits = np.ascontiguousarray(key_bits, dtype=np.uint16)
    tokens, kvh, hd = key_bits.shape
    out = key_bits.copy()
    valid = np.ones(tokens, np.uint8)
    rot, max_pos, cs_ptr, cs_stride, pos_ptr = 0, 0, None, 0, None
    if cos_sin_bits is not None:
        cos_sin_bits = np.ascontiguousarray(cos_sin_bits, dtype=np.uint16)
        positions = np.ascontiguousarray(positions, dtype=np.int64)
        max_pos, rot = cos_sin_bits.shape
        cs_ptr, cs_stride, pos_ptr = _ptr(cos_sin_bits), rot, _ptr(positions)
    w_ptr = None
    if weight is not None:
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        w_ptr = _ptr(weight)
    _load().orc_norm_rope(_ptr(key_bits), kvh * hd, hd, tokens, kvh, hd, w_ptr, float(offset), float(eps),
                          pos_ptr, cs_ptr, cs_stride, max_pos, rot, 1 if neox else 0, _ptr(out), _ptr(valid))
    return out, valid.astype(bool)


def sparse_attention(q_bits: np.ndarray, storage: np.ndarray, indices: np.ndarray, block_table: np.ndarray,
                     token_to_request: np.ndarray, key_global_scale: float = 1.0,
                     value_global_scale: float = 1.0, return_lse: bool = False):
    """Reader contract (kernels.py:168-345) in float64; returns fp32 [rows, qh, hd].

    With ``return_lse`` also returns each head's base-2 log-sum-exp of the scaled
    scores (fp32 [rows, qh], -inf where no selection is valid): the split-KV
    partial format (src/qsa_fp8_harness.py:183-208) that merge_partials combines.
    """
    q_bits = np.ascontiguousarray(q_bits, dtype=np.uint16)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    block_table = np.ascontiguousarray(block_table, dtype=np.int32)
    token_to_request = np.ascontiguousarray(token_to_request, dtype=np.int32)
    assert storage.flags["C_CONTIGUOUS"] and storage.dtype == np.uint8
    rows, qh, hd = q_bits.shape
    blocks, kvh, page, _ = storage.shape
    out = np.zeros((rows, qh, hd), np.float32)
    lse = np.full((rows, qh), -np.inf, np.float32)
    regs = cache_regions(storage, hd)
    base = _ptr(storage)
    args = []
    for off, (sb, st, sh) in regs:
        args += [base + off, sb, st, sh]
    topk = indices.shape[1] if indices.ndim == 2 else 0
    _load().orc_sparse_attention(_ptr(q_bits), qh * hd, hd, *args, blocks, page, kvh, float(key_global_scale),
                                 float(value_global_scale), _ptr(indices), topk, _ptr(block_table),
                                 block_table.shape[0], block_table.shape[1], _ptr(token_to_request), _ptr(out),
                                 rows, qh, hd, _ptr(lse) if return_lse else None)
    return (out, lse) if return_lse else out


def sparse_attention_fp8(q_bits: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, indices: np.ndarray,
                         block_table: np.ndarray, token_to_request: np.ndarray, k_scale: float = 1.0,
                         v_scale: float = 1.0, return_lse: bool = False):
    """FP8 sibling reader (src/qsa_fp8_harness.py:42-208) in float64; returns fp32 [rows, qh, hd].

    ``k_cache`` / ``v_cache``: uint8 views of float8_e4m3fn [blocks, page, kv_heads, head_dim], C-contiguous.
    Scores are scaled by head_dim^-0.5 * k_scale and outputs multiplied by v_scale.
    """
    q_bits = np.ascontiguousarray(q_bits, dtype=np.uint16)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    block_table = np.ascontiguousarray(block_table, dtype=np.int32)
    token_to_request = np.ascontiguousarray(token_to_request, dtype=np.int32)
    for c in (k_cache, v_cache):
        assert c.flags["C_CONTIGUOUS"] and c.dtype == np.uint8 and c.shape == k_cache.shape
    rows, qh, hd = q_bits.shape
    blocks, page, kvh, _ = k_cache.shape
    sb, st, sh = page * kvh * hd, kvh * hd, hd
    out = np.zeros((rows, qh, hd), np.float32)
    lse = np.full((rows, qh), -np.inf, np.float32)
    topk = indices.shape[1] if indices.ndim == 2 else 0
    _load().orc_sparse_attention_fp8(_ptr(q_bits), qh * hd, hd, _ptr(k_cache), sb, st, sh, _ptr(v_cache), sb, st, sh,
                                     blocks, page, kvh, float(k_scale), float(v_scale), _ptr(indices), topk,
                                     _ptr(block_table), block_table.shape[0], block_table.shape[1],
                                     _ptr(token_to_request), _ptr(out), rows, qh, hd,
                                     _ptr(lse) if return_lse else None)
    return (out, lse) if return_lse else out


def sparse_attention_bf16(q_bits: np.ndarray, k_cache_bits: np.ndarray, v_cache_bits: np.ndarray,
                          indices: np.ndarray, block_table: np.ndarray, token_to_request: np.ndarray,
                          return_lse: bool = False):
    """BF16 sibling reader (src/qsa_ref.py:12-52 on a bf16 cache) in float64; returns fp32 [rows, qh, hd].

    ``k_cache_bits`` / ``v_cache_bits``: uint16 bf16 bit patterns [blocks, page, kv_heads, head_dim], any
    strides with a contiguous last dim (e.g. the K and V halves of a [blocks, page, kv_heads, 2 * hd] array).
    """
    q_bits = np.ascontiguousarray(q_bits, dtype=np.uint16)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    block_table = np.ascontiguousarray(block_table, dtype=np.int32)
    token_to_request = np.ascontiguousarray(token_to_request, dtype=np.int32)
    for c in (k_cache_bits, v_cache_bits):
        assert c.dtype == np.uint16 and c.ndim == 4 and c.strides[-1] == 2 and c.shape == k_cache_bits.shape
    rows, qh, hd = q_bits.shape
    blocks, page, kvh, _ = k_cache_bits.shape
    out = np.zeros((rows, qh, hd), np.float32)
    lse = np.full((rows, qh), -np.inf, np.float32)
    topk = indices.shape[1] if indices.ndim == 2 else 0
    ks, vs = k_cache_bits.strides, v_cache_bits.strides
    _load().orc_sparse_attention_bf16(_ptr(q_bits), qh * hd, hd, k_cache_bits.ctypes.data, ks[0], ks[1], ks[2],
                                      v_cache_bits.ctypes.data, vs[0], vs[1], vs[2], blocks, page, kvh,
                                      _ptr(indices), topk, _ptr(block_table), block_table.shape[0],
                                      block_table.shape[1], _ptr(token_to_request), _ptr(out), rows, qh, hd,
                                      _ptr(lse) if return_lse else None)
    return (out, lse) if return_lse else out


def topk_indices(scores: np.ndarray, k: int, lengths=None) -> np.ndarray:
    """The indexer top-k contract in NumPy: per row, the indices of the k largest of scores[row, :len] in
    ascending order, ties at the k-th value to the lowest indices, NaN highest, -1 padding past len."""
    scores = np.asarray(scores, dtype=np.float32)
    rows, context = scores.shape
    out = np.full((rows, k), -1, np.int32)
    for r in range(rows):
        n = context if lengths is None else int(min(max(lengths[r], 0), context))
        s = scores[r, :n].astype(np.float64)
        key = np.where(np.isnan(s), np.inf, s)
        # largest first; equal keys in index order (stable sort on -key); NaN (inf here) above +inf
        order = np.lexsort((np.arange(n), -key, ~np.isnan(s)))
        sel = np.sort(order[:k])
        out[r, :sel.size] = sel
    return out


def merge_partials(part_out: np.ndarray, part_lse: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of split partials (src/qsa_fp8_harness.py:308-321 semantics).

    part_out: [splits, rows, qh, hd] normalised outputs; part_lse: [splits, rows, qh]
    base-2 lse (-inf for empty splits).  Returns float64 [rows, qh, hd]; rows whose
    splits are all empty are zero.
    """
    o = np.asarray(part_out, np.float64)
    l = np.asarray(part_lse, np.float64)
    m = l.max(axis=0)
    safe_m = np.where(np.isfinite(m), m, 0.0)
    w = np.where(np.isfinite(l), np.exp2(l - safe_m[None]), 0.0)
    den = w.sum(axis=0)
    num = (w[..., None] * o).sum(axis=0)
    return np.where(den[..., None] > 0, num / np.where(den > 0, den, 1.0)[..., None], 0.0)
