"""Fused HF-order RoPE + node scatter on the CPU: the oracle against the reference
kernel's golden output (bit for bit) and the wrapper's argument checks."""
from __future__ import annotations

import pytest
import torch

from golden_cases import load_rope_case
from jetspec_b200.tree_fusion import rope_scatter
from oracle import rope as rope_oracle


@pytest.mark.parametrize("dtype_name", ["bf16", "f32"])
def test_eager_rope_oracle_matches_reference_kernel_bitwise(dtype_name):
    q, k, v, positions, cache, slots, out, kv_after = load_rope_case(dtype_name)
    pools = torch.zeros((2, 4, 256) + tuple(k.shape[1:]), dtype=k.dtype)
    got = rope_oracle.rope_scatter(q, k, v, positions, cache, pools[0], pools[1], slots)
    assert torch.equal(got.view(torch.uint8), out.view(torch.uint8))
    rows = pools[:, slots // 256, slots % 256]
    assert torch.equal(rows.contiguous().view(torch.uint8), kv_after.contiguous().view(torch.uint8))


def test_rope_scatter_checks_match_reference():
    q, k, v, positions, cache, slots, _, _ = load_rope_case("bf16")
    pools = torch.zeros((2, 4, 256) + tuple(k.shape[1:]), dtype=k.dtype)
    with pytest.raises(ValueError, match="CUDA tensors"):
        rope_scatter(q, k, v, positions, cache, pools[0], pools[1], slots)
    with pytest.raises(ValueError, match="even head geometry"):
        rope_scatter(q[..., :127], k[..., :127], v[..., :127], positions, cache[..., :127],
                     pools[0][..., :127], pools[1][..., :127], slots)
    with pytest.raises(ValueError, match="BF16 or FP32"):
        rope_scatter(q.half(), k.half(), v.half(), positions, cache, pools[0].half(),
                     pools[1].half(), slots)
    with pytest.raises(ValueError, match="integer"):
        rope_scatter(q, k, v, positions.float(), cache, pools[0], pools[1], slots)
    with pytest.raises(ValueError, match="cos/sin cache"):
        rope_scatter(q, k, v, positions, cache[:, 0, :64], pools[0], pools[1], slots)
    with pytest.raises(ValueError, match="KV pools"):
        rope_scatter(q, k, v, positions, cache, pools[0][..., :64], pools[1][..., :64], slots)
