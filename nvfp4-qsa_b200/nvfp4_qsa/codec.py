"""NVFP4 codec API (encode / decode / global_scale_for / quant_dequant) on the GPU.

Same functions, arguments and return values as the reference's codec module
(python/nvfp4_qsa/oracle.py:25-92), computed by the sm_100a kernels in
csrc/codec.cu through the C ABI.  Inputs may live on the CPU or a CUDA device;
the work runs on CUDA (the input's device, else the current device) and the
results are returned on the input's device.  There is no CPU implementation:
without CUDA these functions raise RuntimeError.

Format: FP4 = E2M1, magnitudes [0, .5, 1, 1.5, 2, 3, 4, 6], nibble = sign<<3 |
index; one E4M3 scale per ``block_size`` values; fp32 global scale g:
  scale  = e4m3(clamp(g * group_amax / 6, -448, 448))
  codes  = round_e2m1(clamp(x * g / scale, -6, 6)), packed low = element 2j
  decode = grid[code] * sign * (scale / g)
"""
from __future__ import annotations

import torch

from . import _native

E2M1_GRID = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
E2M1_MAX = 6.0
E4M3_MAX = 448.0
GROUP = 16


def _work_device(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("nvfp4_qsa codec runs on CUDA; no CUDA device is available (no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def global_scale_for(x: torch.Tensor) -> torch.Tensor:
    """Per-tensor fp32 global scale (448 * 6) / amax(|x|) (reference oracle.py:25-27)."""
    amax = x.abs().amax().clamp_min(1e-8).float()
    return (E4M3_MAX * E2M1_MAX) / amax


def encode(x2d: torch.Tensor, global_scale: torch.Tensor, block_size: int = GROUP):
    """x2d: [M, N] (N % block_size == 0). Returns (nibbles[M,N] uint8,
    packed[M,N//2] uint8, block_scale_fp8[M,N//block_size] uint8 view,
    saturation stats dict)."""
    m, n = x2d.shape
    if block_size < 2 or block_size % 2 or n % block_size:
        raise ValueError("encode needs an even block_size dividing the row length")
    dev = _work_device(x2d)
    x = x2d.to(device=dev, dtype=torch.float32).contiguous()
    g = torch.as_tensor(global_scale).reshape(1).to(device=dev, dtype=torch.float32)
    nib = torch.empty((m, n), dtype=torch.uint8, device=dev)
    packed = torch.empty((m, n // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((m, n // block_size), dtype=torch.uint8, device=dev)
    counts = torch.zeros(2, dtype=torch.int64, device=dev)
    if m and n:
        with torch.cuda.device(dev):
            status = _native.load().nvqsa_encode_rows(
                x.data_ptr(), m, n, block_size, g.data_ptr(), nib.data_ptr(), packed.data_ptr(),
                scales.data_ptr(), counts.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        _native.check(status, "nvfp4_qsa.encode")
    clip, sat = counts.tolist()
    total, groups = m * n, m * (n // block_size)
    stats = {"clip6_rate": clip / total if total else float("nan"),
             "blockscale_sat_rate": sat / groups if groups else float("nan")}
    home = x2d.device
    return nib.to(home), packed.to(home), scales.to(home), stats


def decode(packed: torch.Tensor, scale_u8: torch.Tensor, global_scale: torch.Tensor,
           n: int, block_size: int = GROUP) -> torch.Tensor:
    """Inverse of encode -> float32 [M, N]."""
    if block_size < 2 or block_size % 2 or n % block_size:
        raise ValueError("decode needs an even block_size dividing the row length")
    dev = _work_device(packed)
    m = packed.shape[0]
    p = packed.to(device=dev, dtype=torch.uint8).contiguous()
    s = scale_u8.to(device=dev).view(torch.uint8).contiguous()
    if p.numel() != m * n // 2 or s.numel() != m * n // block_size:
        raise ValueError("packed / scale sizes do not match [M, n]")
    g = torch.as_tensor(global_scale).reshape(1).to(device=dev, dtype=torch.float32)
    out = torch.empty((m, n), dtype=torch.float32, device=dev)
    if m and n:
        with torch.cuda.device(dev):
            status = _native.load().nvqsa_decode_rows(
                p.data_ptr(), s.data_ptr(), m, n, block_size, g.data_ptr(), out.data_ptr(),
                torch.cuda.current_stream(dev).cuda_stream)
        _native.check(status, "nvfp4_qsa.decode")
    return out.to(packed.device)


def quant_dequant(x2d: torch.Tensor, block_size: int = GROUP):
    """(x_hat, packed, scale_u8, global_scale, nibbles, stats) with g = global_scale_for(x2d)."""
    g = global_scale_for(x2d)
    nib, packed, scale_u8, sat = encode(x2d, g, block_size)
    xhat = decode(packed, scale_u8, g, x2d.shape[1], block_size)
    return xhat, packed, scale_u8, float(g.item()), nib, sat
