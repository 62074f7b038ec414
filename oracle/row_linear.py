"""CPU restatement of the row-parallel linear and its all-reduce (test infrastructure only).

Follows RowParallelLinear (nanovllm/layers/linear.py:131-156): rank r holds columns
[r K/W, (r+1) K/W) of the input and of the weight (weight_loader, :139-147, narrows the
input dimension by tp_rank); forward (:153-156) computes y_r = F.linear(x_r, W_r, bias on
rank 0 only), rounded to the layer's dtype, and dist.all_reduce sums the y_r over the
ranks.  Pinned against the reference run under gloo ranks (tests/golden/row_linear.npz).
"""
from __future__ import annotations

import numpy as np


def round_bf16(values) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returned as float32."""
    bits = np.asarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    return bits.astype(np.uint32).view(np.float32)


def bf16_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


def round_to(values, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(values)
    if dtype == "f16":
        return np.asarray(values, dtype=np.float32).astype(np.float16).astype(np.float32)
    raise ValueError(dtype)


def rank_partials(x, weight, bias, world: int, dtype: str = "bf16") -> list[np.ndarray]:
    """y_r of every rank: x [M, K], weight [N, K] (full, unsharded), bias [N] or None."""
    x = np.asarray(x, dtype=np.float64)
    weight = np.asarray(weight, dtype=np.float64)
    k = x.shape[1]
    if k % world:
        raise ValueError("input features must divide by the world size")
    shard = k // world
    partials = []
    for r in range(world):
        y = x[:, r * shard:(r + 1) * shard] @ weight[:, r * shard:(r + 1) * shard].T
        if r == 0 and bias is not None:
            y = y + np.asarray(bias, dtype=np.float64)
        partials.append(round_to(y.astype(np.float32), dtype))
    return partials


def row_parallel_linear(x, weight, bias, world: int, dtype: str = "bf16") -> np.ndarray:
    """The all-reduced output, summed in float64 and rounded once to the dtype."""
    partials = rank_partials(x, weight, bias, world, dtype)
    return round_to(np.sum(np.stack(partials).astype(np.float64), axis=0).astype(np.float32),
                    dtype)


def tolerance(x, weight, bias, world: int, dtype: str = "bf16") -> np.ndarray:
    """Per-element bound on |y - row_parallel_linear| for any implementation that sums
    each rank's products in float32 (in any order), rounds each partial and the sum once:
    one unit in the last place of every partial and of the result, plus the float32
    accumulation bound gamma_K * sum |x_i w_i| (gamma_K ~ K 2^-24) of each partial."""
    eps = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    partials = rank_partials(x, weight, bias, world, dtype)
    total = row_parallel_linear(x, weight, bias, world, dtype)
    shard = np.asarray(x).shape[1] // world
    absdot = np.abs(np.asarray(x, dtype=np.float64)) @ np.abs(np.asarray(weight, np.float64)).T
    return (eps * (np.sum(np.abs(np.stack(partials)), axis=0) + np.abs(total)) +
            shard * 2.0 ** -24 * absdot + 1e-6)
