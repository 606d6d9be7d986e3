"""CPU: the indexer top-k contract (oracle.topk_indices) against torch.topk, and the wrapper's checks.

The selection buffer contract is the reference's (integration/snapshot/qsa.py:537-545, :605-616): int32
[num_tokens, output_width] logical indices for the reader, -1 where masked.  torch.topk is the selection the
contract is checked against where scores have no ties; ties go to the lowest index.
"""
import numpy as np
import pytest
import torch

import oracle
from nvfp4_qsa import indexer


@pytest.mark.parametrize("rows,context,k", [(4, 1000, 64), (2, 5000, 2048), (3, 40, 40), (1, 17, 5)])
def test_oracle_matches_torch_topk_without_ties(rows, context, k):
    g = torch.Generator().manual_seed(rows * 1000 + context)
    s = torch.randn(rows, context, generator=g)
    want = torch.topk(s, k, dim=1).indices.sort(dim=1).values.numpy()
    assert np.array_equal(oracle.topk_indices(s.numpy(), k), want)


def test_oracle_tie_nan_and_length_rules():
    s = np.array([[2, 7, 7, 7, 1, 7], [np.nan, 0, np.inf, -np.inf, np.nan, 3]], np.float32)
    assert oracle.topk_indices(s, 3).tolist() == [[1, 2, 3], [0, 2, 4]]
    assert oracle.topk_indices(s, 4, lengths=[3, 0]).tolist() == [[0, 1, 2, -1], [-1, -1, -1, -1]]
    z = np.array([[0.0, -0.0, 0.0, -0.0, -1.0]], np.float32)  # -0 equals +0: index order decides
    assert oracle.topk_indices(z, 3).tolist() == [[0, 1, 2]]


def test_wrapper_rejects_bad_buffers():
    s = torch.zeros(3, 10)
    with pytest.raises(ValueError):
        indexer.qsa_select_topk(s.double(), torch.zeros(3, 4, dtype=torch.int32))
    with pytest.raises(ValueError):
        indexer.qsa_select_topk(s, torch.zeros(3, 4, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="invalid selection shape"):
        indexer.qsa_select_topk(s, torch.zeros(2, 4, dtype=torch.int32))
