"""GPU: the nvfp4_qsa.encode / decode API (csrc/codec.cu) equals the reference codec."""
import numpy as np
import pytest
import torch

import nvfp4_qsa
from nvfp4_qsa import oracle as compat

pytestmark = pytest.mark.gpu


def test_codec_cases_bit_exact(codec_cases):
    data, names = codec_cases
    for name in names:
        x = torch.from_numpy(data[f"{name}__x"]).cuda()
        g = torch.tensor(float(data[f"{name}__g"][0]))
        nib, packed, scales, stats = nvfp4_qsa.encode(x, g)
        np.testing.assert_array_equal(packed.cpu().numpy(), data[f"{name}__packed"], err_msg=name)
        np.testing.assert_array_equal(scales.cpu().numpy(), data[f"{name}__scales"], err_msg=name)
        np.testing.assert_array_equal(nib.cpu().numpy(), data[f"{name}__nib"], err_msg=name)
        dec = nvfp4_qsa.decode(packed, scales, g, x.shape[1])
        np.testing.assert_array_equal(dec.cpu().numpy().view(np.uint32),
                                      data[f"{name}__decoded"].view(np.uint32), err_msg=name)
        ref = data[f"{name}__stats"]
        assert stats["clip6_rate"] == pytest.approx(ref[0], rel=1e-6, abs=1e-9), name
        assert stats["blockscale_sat_rate"] == pytest.approx(ref[1], rel=1e-6, abs=1e-9), name


def test_codebook_kat_on_cpu_tensors(golden_kat):
    # CPU tensors in, CPU tensors out; the work runs on CUDA (reference test_cpu_contracts.py:18-35)
    values = torch.tensor([golden_kat["codebook_values"]])
    _, packed, scales, _ = compat.encode(values, torch.tensor(1.0))
    assert packed.device.type == "cpu"
    assert packed[0].tolist() == golden_kat["codebook_packed"]
    assert torch.equal(compat.decode(packed, scales, torch.tensor(1.0), 16), values)
    _, data, sc, _ = nvfp4_qsa.encode(torch.zeros(2, 256), torch.tensor(1.0))
    out = nvfp4_qsa.decode(data, sc, torch.tensor(1.0), 256)
    assert torch.isfinite(out).all() and not out.count_nonzero()


def test_quant_dequant_and_block_size_32():
    x = torch.randn(64, 512, device="cuda")
    xhat, packed, scales, g, nib, sat = compat.quant_dequant(x)
    assert xhat.shape == x.shape and scales.shape == (64, 32)
    assert (xhat - x).abs().max().item() < 0.5 * x.abs().max().item()
    _, p32, s32, _ = nvfp4_qsa.encode(x, torch.tensor(g), block_size=32)
    assert s32.shape == (64, 16) and p32.shape == (64, 256)
    assert nvfp4_qsa.global_scale_for(x).item() == pytest.approx(2688.0 / x.abs().max().item(), rel=1e-6)


@pytest.mark.parametrize("g", [1.0, 2.0 ** -10])
def test_signed_zeros_and_underflowing_products(g):
    # -0 inputs and negative products that underflow to -0 get code 0 (the
    # oracle's sign is y < 0); tiny negative products that round to a nonzero
    # subnormal keep code 8
    import oracle
    x = np.zeros((2, 32), np.float32)
    x[:, 0] = 2688.0 / g  # group scale saturates at 448
    x[:, 1:6] = [-1e-45, -0.0, -1e-40, -(2.0 ** -140), -(2.0 ** -126)]
    x[1, 16:] = -0.0  # an all -0 group
    x[0, 16:] = np.random.default_rng(2).standard_normal(16)
    nib, packed, scales, _ = nvfp4_qsa.encode(torch.from_numpy(x).cuda(), torch.tensor(g))
    enib, epacked, escales, _ = oracle.encode(x, g)
    assert enib[0, 1] == 0 and enib[0, 2] == 0  # -1e-45 underflows, -0 stays zero
    assert enib[0, 5] == 8  # -2^-126 * s rounds to a nonzero subnormal at both g
    np.testing.assert_array_equal(scales.cpu().numpy(), escales)
    np.testing.assert_array_equal(packed.cpu().numpy(), epacked)
    np.testing.assert_array_equal(nib.cpu().numpy(), enib)
