"""Helpers shared by the GPU tests (no test functions here)."""
import hashlib

import numpy as np
import torch

import oracle
from nvfp4_qsa import kernels
from nvfp4_qsa import workloads as W

# North-star attention tolerance vs an FP32/64 reference over the same dequantized K/V.
TOL_MAX_ABS = 2e-2
TOL_MEAN_ABS = 2e-3


def sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.contiguous().cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits_to_cuda(bits: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def cuda_to_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def regions(storage: torch.Tensor, head_dim: int = 256):
    """(kd, ks, vd, vs) views of a [blocks, kvh, page, 2*(hd/2+hd/16)] storage (cache.py:20-24)."""
    region = head_dim // 2 + head_dim // 16
    parts = storage.transpose(1, 2).split(region, dim=-1)
    kd, ks = parts[0].split((head_dim // 2, head_dim // 16), dim=-1)
    vd, vs = parts[1].split((head_dim // 2, head_dim // 16), dim=-1)
    return kd, ks, vd, vs


def gpu_write(storage: torch.Tensor, key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor, gk=1.0, gv=1.0):
    kd, ks, vd, vs = regions(storage, key.shape[-1])
    kernels.qsa_write_cache_nvfp4(key, value, kd, ks, vd, vs, slots, gk, gv)


def gpu_attend(storage, query, indices, block_table, t2r, gk=1.0, gv=1.0):
    kd, ks, vd, vs = regions(storage)
    out = torch.full_like(query, float("nan"))
    kernels.qsa_sparse_paged_attention_nvfp4(query, kd, ks, vd, vs, gk, gv, indices, block_table, t2r, out)
    return out


def assert_attention_close(out: torch.Tensor, expected: np.ndarray, what=""):
    """North-star tolerance on the error beyond the bf16 output's own rounding.

    The output is bf16 (as in the reference kernel), whose rounding alone is up
    to 2^-8 |x|: 0.06 for outputs near 30 in the outlier distributions.  That
    share is discounted before the max-abs 2e-2 / mean-abs 2e-3 gates apply.
    """
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    diff = np.abs(got - expected)
    excess = np.maximum(diff - np.abs(expected) * 2.0 ** -8, 0.0)
    assert excess.max() <= TOL_MAX_ABS, f"{what}: max_abs {diff.max():.3e} (beyond bf16 rounding {excess.max():.3e})"
    assert excess.mean() <= TOL_MEAN_ABS, f"{what}: mean_abs {diff.mean():.3e} (beyond bf16 {excess.mean():.3e})"
    return float(diff.max()), float(diff.mean())


def build_case_on_gpu(case: W.DecodeCase, device="cuda"):
    """Write a DecodeCase with the GPU writer; return (storage, q, idx, table, t2r) on device."""
    storage = torch.zeros(case.blocks, 2, case.page, 288, dtype=torch.uint8, device=device)
    gpu_write(storage, bits_to_cuda(case.key, device), bits_to_cuda(case.value, device),
              torch.from_numpy(case.slots).to(device))
    return (storage, bits_to_cuda(case.query, device), torch.from_numpy(case.indices).to(device),
            torch.from_numpy(case.block_table).to(device), torch.from_numpy(case.token_to_request).to(device))


def oracle_attention(storage: torch.Tensor, q: torch.Tensor, idx, table, t2r, gk=1.0, gv=1.0):
    return oracle.sparse_attention(cuda_to_bits(q), storage.cpu().numpy(), idx.cpu().numpy(), table.cpu().numpy(),
                                   t2r.cpu().numpy(), gk, gv)
