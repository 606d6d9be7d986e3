"""GPU: the no-allocation reader entry point matches the regular one.

nvqsa_sparse_attention_noalloc serves callers that may not allocate device
memory at call time (fixed-buffer hosts, serving loops under a no-allocation
rule, plugins whose framework owns every allocation): instead of a
caller-provided workspace it keeps its split-KV partials in a static 16 MiB
device buffer.  This test calls it through the C ABI twice in a row, on
different inputs, and compares each result with nvqsa_sparse_attention's on
the same inputs.  The file is named to be collected last.
"""
import numpy as np
import pytest
import torch

from nvfp4_qsa import _native, kernels
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu

# Same bf16 output-rounding-aware tolerance as the other reader tests; the two
# entry points run the same kernels, so the results are expected to match bitwise.
TOL_MAX_ABS = 2e-2


def _storage_case(seed):
    case = W.decode_config(seed=seed, context=4096, topk=640, rows=3)
    dev = torch.device("cuda")
    storage = torch.zeros(case.blocks, 2, case.page, 288, dtype=torch.uint8, device=dev)
    parts = storage.transpose(1, 2).split(144, dim=-1)
    kd, ks = parts[0].split((128, 16), dim=-1)
    vd, vs = parts[1].split((128, 16), dim=-1)

    def bits(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)

    kernels.qsa_write_cache_nvfp4(bits(case.key), bits(case.value), kd, ks, vd, vs,
                                  torch.from_numpy(case.slots).to(dev), 1.0, 1.0)
    return (case, (kd, ks, vd, vs), bits(case.query), torch.from_numpy(case.indices).to(dev),
            torch.from_numpy(case.block_table).to(dev), torch.from_numpy(case.token_to_request).to(dev))


def _noalloc_call(lib, q, regions, idx, bt, t2r, out):
    kd, ks, vd, vs = regions
    return lib.nvqsa_sparse_attention_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1),
        kd.data_ptr(), kd.stride(0), kd.stride(1), kd.stride(2),
        ks.data_ptr(), ks.stride(0), ks.stride(1), ks.stride(2),
        vd.data_ptr(), vd.stride(0), vd.stride(1), vd.stride(2),
        vs.data_ptr(), vs.stride(0), vs.stride(1), vs.stride(2),
        kd.shape[0], kd.shape[1], kd.shape[2], 1.0, 1.0,
        idx.data_ptr(), idx.shape[1], bt.data_ptr(), bt.shape[0], bt.shape[1], t2r.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        q.shape[0], q.shape[1], q.shape[2], torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_regular_entry_point_on_two_calls():
    lib = _native.load()
    for seed in (31, 32):  # two calls in a row share the static buffer
        case, regions, q, idx, bt, t2r = _storage_case(seed)
        assert kernels.attention_workspace_bytes(q.shape[0], 24, 2, 256, idx.shape[1]) > 0  # exercises the scratch
        expected = torch.empty_like(q)
        kernels.qsa_sparse_paged_attention_nvfp4(q, *regions, 1.0, 1.0, idx, bt, t2r, expected)
        got = torch.full_like(q, float("nan"))
        status = _noalloc_call(lib, q, regions, idx, bt, t2r, got)
        assert status == 0, _native.status_text(status)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        diff = (got.float() - expected.float()).abs().max().item()
        assert diff <= TOL_MAX_ABS, diff


def test_noalloc_back_to_back_on_one_stream():
    # The serving pattern: two calls with different inputs and outputs queued on one stream with no host
    # synchronisation between them.  The second call's counter reset and reader launch are stream-ordered
    # after the first call's kernel, which uses the same static buffer.
    lib = _native.load()
    cases = [_storage_case(seed) for seed in (34, 35)]
    outs = [torch.full_like(c[2], float("nan")) for c in cases]
    torch.cuda.synchronize()
    for (case, regions, q, idx, bt, t2r), got in zip(cases, outs):
        status = _noalloc_call(lib, q, regions, idx, bt, t2r, got)
        assert status == 0, _native.status_text(status)
    torch.cuda.synchronize()
    for (case, regions, q, idx, bt, t2r), got in zip(cases, outs):
        expected = torch.empty_like(q)
        kernels.qsa_sparse_paged_attention_nvfp4(q, *regions, 1.0, 1.0, idx, bt, t2r, expected)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert (got.float() - expected.float()).abs().max().item() <= TOL_MAX_ABS


def test_noalloc_rejects_problems_beyond_its_buffer():
    lib = _native.load()
    case, regions, q, idx, bt, t2r = _storage_case(33)
    rows, topk = 4096, 16384  # 16 splits (beyond a cluster) x 4096 rows x 24 heads x 1 KiB of partials > 16 MiB
    assert kernels.attention_workspace_bytes(rows, 24, 2, 256, topk) > (16 << 20)
    big_q = torch.zeros(rows, 24, 256, dtype=torch.bfloat16, device="cuda")
    big_idx = torch.zeros(rows, topk, dtype=torch.int32, device="cuda")
    big_t2r = torch.zeros(rows, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(big_q)
    status = _noalloc_call(lib, big_q, regions, big_idx, bt, big_t2r, out)
    assert status == 9 and "scratch" in _native.status_text(status)
    torch.cuda.synchronize()
    assert not out.any().item()  # rejected before any launch
