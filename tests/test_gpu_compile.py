"""A torch.compile'd caller traces through the launchers without a graph break.

The reference compiles parts of its model (nanovllm/layers/layernorm.py,
rotary_embedding.py); a compiled verifier step that calls the tree attention, the
tree-node store and the commit must see them as operators (jetspec_b200::*), not as
opaque ctypes calls.  fullgraph=True turns any graph break into an error; the compiled
results must equal the eager ones bit for bit.
"""
from __future__ import annotations

import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import workloads

from helpers import bits_equal, ragged_batch

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)


def test_compiled_step_has_no_graph_break_and_matches_eager():
    batch = ragged_batch((1024, 0, 257), counts=(63, 31, 47))
    q, k, v = workloads.make_tensors(batch, DEVICE)
    meta = batch.metadata(DEVICE)
    scale = batch.head_dim ** -0.5
    gen = torch.Generator(device=DEVICE).manual_seed(3)
    k_nodes = (torch.randn((batch.total_queries, 2, 128), generator=gen, device=DEVICE) * scale).bfloat16()
    v_nodes = (torch.randn((batch.total_queries, 2, 128), generator=gen, device=DEVICE) * scale).bfloat16()
    pool = torch.stack([k, v]).unsqueeze(1).clone()  # [2, 1, blocks, bs, heads, dim]
    src = meta.tree_slots[:5].clone()
    dst = torch.tensor(batch.owned_pages[0][-1:], device=DEVICE) * 256 + torch.arange(5, device=DEVICE)

    def step(q, pool):
        jb.store_kvcache(k_nodes, v_nodes, pool[0, 0], pool[1, 0], meta.tree_slots)
        out = jb.packed_tree_attention_gqa(q, pool[0, 0], pool[1, 0], meta, scale, batch.groups)
        jb.copy_accepted_kv(pool, src, dst, 256)
        return out

    eager_pool = pool.clone()
    expected = step(q, eager_pool)
    compiled = torch.compile(step, fullgraph=True, backend="aot_eager")
    got_pool = pool.clone()
    got = compiled(q, got_pool)
    torch.cuda.synchronize()
    assert bits_equal(got, expected)
    assert bits_equal(got_pool, eager_pool)
