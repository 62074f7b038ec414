"""Acceptance-walk oracle pinned to the reference's accept_batch outputs (tests/golden/accept.npz)."""
from __future__ import annotations

import numpy as np
import pytest

from golden_cases import load_npz
from oracle import accept as accept_oracle


def _golden():
    z = load_npz("accept.npz")
    return z, accept_oracle.accept_batch(z["logits"], z["token_ids"], z["parents"], z["depths"],
                                         z["offsets"], int(z["max_depth"]))


def test_oracle_matches_reference_walks():
    z, results = _golden()
    assert len(results) == len(z["offsets"]) - 1
    for r, res in enumerate(results):
        length = int(z["accepted_length"][r]) + 1
        assert res["path"] == z["path"][r, :length].tolist()
        assert res["accepted_length"] == int(z["accepted_length"][r])
        assert res["correction"] == int(z["correction"][r])
        assert res["outputs"] == z["outputs"][r, :length].tolist()


def test_duplicate_siblings_last_child_wins():
    # The reference's own known answer (tests/test_jetspec_serving_ops.py:37-56).
    _, results = _golden()
    assert results[0]["path"] == [0, 2, 4]


def test_depth_cap_and_single_node_tree():
    z, results = _golden()
    assert results[-1]["accepted_length"] == int(z["max_depth"])  # chain deeper than the cap
    assert results[1]["path"] == [0] and results[1]["accepted_length"] == 0


def test_inconsistent_depths_raise():
    z = load_npz("accept.npz")
    depths = z["depths"].copy()
    depths[2] = 5  # node 2 of the first tree is on its accepted path
    with pytest.raises(RuntimeError, match="canonical tail"):
        accept_oracle.accept_batch(z["logits"], z["token_ids"], z["parents"], depths,
                                   z["offsets"], int(z["max_depth"]))


def test_argmax_ties_and_nan_follow_torch():
    import torch
    row = np.array([[1.0, 3.0, 3.0, 2.0], [0.0, np.nan, 5.0, np.nan]], dtype=np.float32)
    assert np.argmax(row, axis=-1).tolist() == torch.from_numpy(row).argmax(-1).tolist() == [1, 1]
