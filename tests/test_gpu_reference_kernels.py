"""This package's kernels against the reference's own Triton kernels on the same B200.

The reference package installed under baseline/_ref carries the kernels this package
replaces; on the GPU they run natively (its CPU path is only the Triton interpreter).

* bf16 probabilities: packed_tree_attention_gqa against the reference's grouped kernel
  (tree_gqa.py:114-140), configs 1-3 and the page-boundary prefix sweep.
* fp32 probabilities and fp32 operands: the dispatcher's "reference" backend against the
  reference's scalar fp32 kernel (_packed_paged_tree_fp32, paged_backend.py:116-213,
  through tree_attention.py:40-62), within the reference's fp32 bound.
"""
from __future__ import annotations

from pathlib import Path
import sys

import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import workloads

from helpers import BF16_MAX_ABS, BF16_MEAN_ABS, FP32_BOUND, PREFIX_LENGTHS, ragged_batch

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "nanovllm").is_dir(),
                                 reason="reference package not installed under baseline/_ref")]
DEVICE = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ref():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from nanovllm.speculative.jetspec import tree_attention, tree_gqa

    return tree_gqa.packed_tree_attention_gqa, tree_attention.packed_tree_attention_reference


def _close(ours, theirs, max_abs, mean_abs=None):
    assert torch.isfinite(ours).all() and torch.isfinite(theirs).all()
    diff = (ours.float() - theirs.float()).abs()
    assert diff.max().item() <= max_abs, diff.max().item()
    if mean_abs is not None:
        assert diff.mean().item() <= mean_abs, diff.mean().item()
    return diff.max().item()


@pytest.mark.parametrize("name", ("config1", "config2", "config3"))
def test_bf16_probabilities_match_the_reference_grouped_kernel(ref, name):
    ref_gqa, _ = ref
    batch = workloads.CONFIGS[name]()
    q, k, v = workloads.make_tensors(batch, DEVICE, poison=False, generator_device="cuda")
    meta = batch.metadata(DEVICE)
    scale = batch.head_dim ** -0.5
    ours = jb.packed_tree_attention_gqa(q, k, v, meta, scale, batch.groups)
    theirs = ref_gqa(q, k, v, meta, scale, batch.groups)
    _close(ours, theirs, BF16_MAX_ABS, BF16_MEAN_ABS)


def test_prefix_sweep_matches_the_reference_grouped_kernel(ref):
    ref_gqa, _ = ref
    batch = ragged_batch(PREFIX_LENGTHS, counts=(63, 31, 47, 1, 16, 5, 64, 2, 9, 33))
    q, k, v = workloads.make_tensors(batch, DEVICE)
    meta = batch.metadata(DEVICE)
    scale = batch.head_dim ** -0.5
    _close(jb.packed_tree_attention_gqa(q, k, v, meta, scale, batch.groups),
           ref_gqa(q, k, v, meta, scale, batch.groups), BF16_MAX_ABS, BF16_MEAN_ABS)


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
def test_fp32_arithmetic_matches_the_reference_fp32_kernel(ref, dtype):
    _, ref_fp32 = ref
    batch = ragged_batch((65, 0, 257, 1024), counts=(63, 31, 47, 16))
    q, k, v = workloads.make_tensors(batch, DEVICE, dtype=dtype)
    meta = batch.metadata(DEVICE)
    scale = batch.head_dim ** -0.5
    ours = jb.packed_tree_attention(q, k, v, meta, scale, batch.groups, backend="reference",
                                    output_dtype=torch.float32)
    theirs = ref_fp32(q, k, v, meta, scale, batch.groups, output_dtype=torch.float32)
    bound = FP32_BOUND * max(1.0, theirs.abs().max().item())
    _close(ours, theirs, bound)
