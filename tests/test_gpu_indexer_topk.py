"""GPU: the indexer top-k kernel (nvqsa_topk_indices) against torch.topk and the NumPy contract.

Bit-exact index sets: against torch.topk on seeded scores without ties, and against oracle.topk_indices
(ties to the lowest index, NaN highest, -1 padding past a row's causal length) on scores with ties, NaN and
infinities.  Sizes include the decode shapes: 96 rows x 131,072 positions and one row of 169,984, k = 2,048.
The selection then drives the reader end to end.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_attention_close, build_case_on_gpu, gpu_attend, oracle_attention
from nvfp4_qsa import indexer
from nvfp4_qsa import workloads as W

pytestmark = pytest.mark.gpu


def _select(scores, k, lengths=None):
    out = torch.full((scores.shape[0], k), -7, dtype=torch.int32, device=scores.device)
    indexer.qsa_select_topk(scores, out, lengths)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("rows,context,k", [(96, 131072, 2048), (1, 169984, 2048), (48, 20000, 2048),
                                            (5, 3000, 1000), (7, 2049, 2048), (3, 100, 7)])
def test_topk_matches_torch_topk(rows, context, k):
    g = torch.Generator(device="cuda").manual_seed(rows + context)
    s = torch.randn(rows, context, device="cuda", generator=g)
    got = _select(s, k)
    want = torch.topk(s, k, dim=1).indices.sort(dim=1).values.to(torch.int32)
    assert torch.equal(got, want)


def test_topk_ties_nan_inf_and_lengths_match_the_contract():
    g = torch.Generator(device="cuda").manual_seed(3)
    s = torch.randint(-4, 5, (6, 5000), device="cuda", generator=g).float()  # heavy ties
    s[1, 100] = float("nan")
    s[1, 4000] = float("inf")
    s[2, :] = 0.0
    s[2, 1::2] = -0.0  # equal to +0: ties in index order regardless of sign
    s[3, 50:60] = float("-inf")
    lengths = torch.tensor([5000, 4500, 3000, 2048, 10, 0], dtype=torch.int32, device="cuda")
    got = _select(s, 2048, lengths)
    want = oracle.topk_indices(s.cpu().numpy(), 2048, lengths.cpu().numpy())
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("rows,context,levels", [(8, 131072, 5), (1, 169984, 3), (3, 40000, 1)])
def test_topk_heavy_ties_at_decode_sizes(rows, context, levels):
    # few distinct values: the candidate lists overflow and the selection takes the re-scan path
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + levels)
    s = torch.randint(0, levels, (rows, context), device="cuda", generator=g).float()
    s[0, 12345] = 9.0
    lengths = torch.full((rows,), context, dtype=torch.int32, device="cuda")
    lengths[-1] = context - 777
    got = _select(s, 2048, lengths)
    want = oracle.topk_indices(s.cpu().numpy(), 2048, lengths.cpu().numpy())
    assert np.array_equal(got.cpu().numpy(), want)


def test_topk_top_keys_concentrated_in_one_range():
    # increasing / decreasing scores put every selected key in one warp's range: that warp's list overflows
    base = torch.arange(50000, device="cuda", dtype=torch.float32)
    s = torch.stack([base, -base, base.flip(0) * 0.5, torch.zeros_like(base)])
    got = _select(s, 2048)
    want = oracle.topk_indices(s.cpu().numpy(), 2048)
    assert np.array_equal(got.cpu().numpy(), want)


def test_topk_unaligned_rows_and_padded_output():
    # rows that start off a 16-byte boundary (scalar loads) and an output buffer wider than its rows' k
    g = torch.Generator(device="cuda").manual_seed(11)
    base = torch.randn(5, 20011, device="cuda", generator=g)
    s = base[:, 3:20003]  # row stride 20011: no row 16-byte aligned except by chance
    buf = torch.full((5, 2100), -9, dtype=torch.int32, device="cuda")
    indexer.qsa_select_topk(s, buf[:, :2048])
    torch.cuda.synchronize()
    want = torch.topk(s, 2048, dim=1).indices.sort(dim=1).values.to(torch.int32)
    assert torch.equal(buf[:, :2048], want)
    assert (buf[:, 2048:] == -9).all()


def test_selection_drives_the_reader():
    # scores from the indexer side -> top-2048 -> the reader: equals the reader on the same indices
    case = W.decode_config(seed=21, context=16384, topk=2048, page=3136, rows=4)
    storage, q, _, bt, t2r = build_case_on_gpu(case)
    g = torch.Generator(device="cuda").manual_seed(5)
    scores = torch.randn(4, 16384, device="cuda", generator=g)
    lengths = torch.tensor([16384, 12000, 9000, 2000], dtype=torch.int32, device="cuda")
    idx = _select(scores, 2048, lengths)
    assert (idx[3, 2000:] == -1).all() and (idx[3, :2000] == torch.arange(2000, device="cuda")).all()
    out = gpu_attend(storage, q, idx, bt, t2r)
    assert_attention_close(out, oracle_attention(storage, q, idx, bt, t2r), "indexer -> reader")
