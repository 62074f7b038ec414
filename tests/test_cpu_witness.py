"""The argmax-flip witness (verify_step.argmax_flip_witness) against the reference's own
results on seeded logits (golden fixture from tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import torch

from golden_cases import load_npz
from jetspec_b200.verify_step import argmax_flip_witness


def test_witness_matches_the_reference_golden():
    z = load_npz("witness.npz")
    result = argmax_flip_witness(torch.from_numpy(z["actual"]), torch.from_numpy(z["reference"]))
    assert result["argmax_flips"] == int(z["argmax_flips"])
    assert result["large_margin_violations"] == int(z["large_margin_violations"])
    rows = result["rows"]
    assert [r["argmax_flipped"] for r in rows] == z["flipped"].tolist()
    assert [r["large_margin_violation"] for r in rows] == z["violation"].tolist()
    assert [r["flip_within_error_envelope"] is True for r in rows] == z["within"].tolist()
    assert [r["actual_argmax"] for r in rows] == z["actual_argmax"].tolist()
    assert [r["reference_argmax"] for r in rows] == z["reference_argmax"].tolist()
    np.testing.assert_array_equal([r["logits_inf_delta"] for r in rows], z["delta"])
    np.testing.assert_array_equal([r["reference_top2_margin"] for r in rows], z["margin"])


def test_witness_rejects_mismatched_shapes():
    import pytest

    with pytest.raises(ValueError):
        argmax_flip_witness(torch.zeros(2, 5), torch.zeros(2, 6))
