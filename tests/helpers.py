"""Fixtures shared by the tests: reference-style ragged batches and oracle comparison."""
from __future__ import annotations

import numpy as np
import torch

import jetspec_b200 as jb
from jetspec_b200 import workloads
from oracle import tree_attention as attn_oracle

# Tolerances of the bf16 contract: max-abs and mean-abs against the fp32 oracle.
BF16_MAX_ABS = 2e-2
BF16_MEAN_ABS = 2e-3
# fp32-output / fp32-probability contract: the reference's FP32 attention bound.
FP32_BOUND = 1e-4

# Page-boundary sweep of the reference's qualification harness.
PREFIX_LENGTHS = (0, 1, 63, 64, 65, 255, 256, 257, 1024, 2048)


def ragged_batch(prefixes, counts=(63, 31, 47), *, kv_heads=2, groups=4, head_dim=128,
                 seed=317, window=None, block_size=256, num_blocks=None):
    """Random topological trees at scattered scratch slots over shuffled prefix pages."""
    rng = np.random.default_rng(seed)
    parents = [workloads.random_parents(rng, int(c), window) for c in counts]
    accepted = [3] * len(counts)
    return workloads.build_batch(prefixes, parents, block_size=block_size, num_kv_heads=kv_heads,
                                 groups=groups, head_dim=head_dim, seed=seed,
                                 accepted_lengths=accepted, num_blocks=num_blocks)


def oracle_output(batch, q, k_pool, v_pool, scale=None, requests=None):
    scale = batch.head_dim ** -0.5 if scale is None else scale
    return attn_oracle.masked_sdpa(q, k_pool, v_pool, batch.prefix_lens,
                                   batch.block_tables, batch.tree_slots, batch.parents, scale,
                                   batch.groups, requests=requests)


def assert_bf16_close(actual, expected, rows=None):
    actual = actual.float().cpu()
    if rows is not None:
        actual, expected = actual[rows], expected[rows]
    assert torch.isfinite(actual).all(), "non-finite output: a poisoned row was read"
    diff = (actual - expected).abs()
    assert diff.max().item() <= BF16_MAX_ABS, f"max-abs {diff.max().item():.3e}"
    assert diff.mean().item() <= BF16_MEAN_ABS, f"mean-abs {diff.mean().item():.3e}"
    return diff


def assert_fp32_close(actual, expected):
    actual = actual.float().cpu()
    assert torch.isfinite(actual).all()
    bound = FP32_BOUND * max(1.0, expected.abs().max().item())
    diff = (actual - expected).abs().max().item()
    assert diff <= bound, f"max-abs {diff:.3e} > {bound:.3e}"
    rms = (actual - expected).square().mean().sqrt() / expected.square().mean().sqrt()
    assert rms.item() <= FP32_BOUND, f"relative RMS {rms.item():.3e}"


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (a.shape == b.shape and a.dtype == b.dtype
            and torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8)))


def run_gqa(batch, q, k_pool, v_pool, meta=None, **kwargs):
    meta = batch.metadata(q.device) if meta is None else meta
    return jb.packed_tree_attention_gqa(q, k_pool, v_pool, meta, batch.head_dim ** -0.5,
                                        batch.groups, **kwargs)
