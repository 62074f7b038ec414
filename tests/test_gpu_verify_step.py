"""The reference's own verifier with this package patched in (integration.ReferencePatch).

The reference package installed under baseline/_ref supplies the model code
(nanovllm/models/qwen3.py), its metadata builder, its Triton kernels (the unpatched arm)
and its acceptance walk; the patch routes the RoPE scatter, the tree attention, the
row-parallel projections and the acceptance walk through this package.

* Stage 1: one Qwen3 decoder layer (random weights) on the config-3 serving mix (64
  requests, contexts log-uniform in [512, 16384], trees of 16 to 128 nodes): the RoPE-ed
  queries and the scattered tree-node K/V equal the unpatched layer's bit for bit, the
  tree attention inside the layer matches the fp32 masked-SDPA oracle within the bf16
  contract, and the layer outputs agree.
* Stage 2: config 5 itself, the full 36-layer Qwen3-8B (random weights), 32 requests of
  2048-token contexts with 64-node trees, tensor parallelism 1: the greedy accepted paths
  of the patched verifier equal the unpatched reference's on identical inputs, paths of up
  to 8 accepted nodes having been planted through the reference's own greedy tokens;
  a request whose path differs must trace back to a greedy flip that the reference's
  argmax-flip witness (restated in verify_step.py) explains as a near-tie.
"""
from __future__ import annotations

from pathlib import Path
import socket
import sys

import numpy as np
import pytest
import torch

from helpers import BF16_MAX_ABS, BF16_MEAN_ABS, assert_bf16_close

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "nanovllm").is_dir(),
                                 reason="reference package not installed under baseline/_ref")]
DEVICE = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def reference():
    """The reference package importable, and a one-rank process group (its layers read
    the tensor-parallel rank and size when they are built)."""
    import torch.distributed as dist

    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    created = False
    if not dist.is_initialized():
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=1)
        created = True
    torch.cuda.set_device(DEVICE)
    yield
    if created:
        dist.destroy_process_group()


class Recorder:
    """Wraps an attention entry point and keeps (q, out) of every call."""

    def __init__(self, fn):
        self.fn, self.calls = fn, []

    def __call__(self, q, *args, **kwargs):
        out = self.fn(q, *args, **kwargs)
        self.calls.append((q.clone(), out.clone()))
        return out


def test_stage1_decoder_layer_config3(reference):
    import nanovllm.speculative.jetspec.paged_backend as ref_backend
    from jetspec_b200 import verify_step, workloads
    from jetspec_b200.integration import ReferencePatch
    from oracle import tree_attention as attn_oracle

    config = verify_step.qwen3_8b_config(num_layers=1)
    model = verify_step.build_reference_model(config, DEVICE)
    verify_step.set_target_kernels(model, "fused_rope_gqa")
    mix = workloads.config3()
    inputs = verify_step.make_inputs(config, DEVICE, requests=mix.num_requests,
                                     context=mix.prefix_lens, nodes=mix.node_counts, seed=1003)
    layer = model.model.layers[0]
    kp, vp = inputs.kv_pool[0, 0], inputs.kv_pool[1, 0]
    slots = inputs.metadata.tree_slots
    with torch.inference_mode():
        hidden = model.model.embed_tokens(inputs.tokens)

        def run():
            out = layer.forward_packed_tree(inputs.positions, hidden, kp, vp, inputs.metadata)
            torch.cuda.synchronize()
            return out, kp[slots // 256, slots % 256].clone(), vp[slots // 256, slots % 256].clone()

        original = ref_backend.packed_tree_attention
        ref_rec = Recorder(original)
        ref_backend.packed_tree_attention = ref_rec
        try:
            ref_out, ref_k, ref_v = run()
        finally:
            ref_backend.packed_tree_attention = original
        with ReferencePatch(model):
            ours_fn = ref_backend.packed_tree_attention
            our_rec = Recorder(ours_fn)
            ref_backend.packed_tree_attention = our_rec
            try:
                our_out, our_k, our_v = run()
            finally:
                ref_backend.packed_tree_attention = ours_fn
    assert ref_backend.packed_tree_attention is original
    (ref_q, ref_attn), = ref_rec.calls
    (our_q, our_attn), = our_rec.calls
    # The fused RoPE + scatter is bit-exact: same rotated queries, same node K/V.
    assert torch.equal(our_q, ref_q)
    assert torch.equal(our_k, ref_k) and torch.equal(our_v, ref_v)
    # The attention inside the layer against the fp32 oracle on sampled requests (the
    # longest context, the largest tree and two more), and against the reference kernel.
    order = np.argsort(mix.prefix_lens)
    sample = sorted({int(order[-1]), int(np.argmax(mix.node_counts)), 0, 17})
    expected = attn_oracle.masked_sdpa(our_q, kp, vp, inputs.prefix_lens, inputs.block_tables,
                                       [list(inputs.metadata.tree_slot_ids[a:b]) for a, b in
                                        zip(inputs.offsets[:-1], inputs.offsets[1:])],
                                       inputs.parents, layer.self_attn.scaling, 4, requests=sample)
    rows = torch.cat([torch.arange(inputs.offsets[r], inputs.offsets[r + 1]) for r in sample])
    assert_bf16_close(our_attn.cpu(), expected, rows=rows)
    assert_bf16_close(ref_attn.cpu(), expected, rows=rows)
    diff = (our_attn.float() - ref_attn.float()).abs()
    assert diff.max().item() <= BF16_MAX_ABS and diff.mean().item() <= BF16_MEAN_ABS
    # Layer outputs: the only difference is the attention's rounding, through o_proj.
    rel = ((our_out.float() - ref_out.float()).norm() / ref_out.float().norm()).item()
    assert torch.isfinite(our_out).all() and rel <= 1e-2, rel


def test_stage2_config5_accepted_paths(reference):
    """Config 5 at TP 1, four verifiers on the same round, on the numerically stable
    synthetic Qwen3-8B (verify_step.build_reference_model):

    * fp32 probabilities (the numerics the reference qualifies against): the reference with
      its fp32-probability kernels (target_kernels "fused_rope") against the same code with
      this package patched in;
    * bf16 probabilities (the reference's fastest, shipped path, "fused_rope_gqa") against
      the same code patched.

    Both pairs must accept identical greedy paths (and corrections) for every request;
    the reference's own two backends against each other are reported beside them.
    """
    from jetspec_b200 import verify_step
    from jetspec_b200.integration import ReferencePatch

    config = verify_step.qwen3_8b_config(num_layers=36)
    model = verify_step.build_reference_model(config, DEVICE)
    verify_step.set_target_kernels(model, "fused_rope_gqa")
    inputs = verify_step.make_inputs(config, DEVICE, requests=32, context=2048, nodes=64)
    rng = np.random.default_rng(55)
    planted = rng.integers(0, 9, size=32).tolist()
    verify_step.plant_paths(model, inputs, planted)

    def run(kernels, patched):
        verify_step.set_target_kernels(model, kernels)
        if patched:
            with ReferencePatch(model):
                logits = verify_step.verify_logits(model, inputs)
                return logits, verify_step.accept(logits, inputs)
        logits = verify_step.verify_logits(model, inputs)
        return logits, verify_step.accept(logits, inputs)

    ref_logits, ref_acc = run("fused_rope_gqa", False)
    our_logits, our_acc = run("fused_rope_gqa", True)
    ref32_logits, ref32_acc = run("fused_rope", False)
    our32_logits, our32_acc = run("fused_rope", True)
    verify_step.set_target_kernels(model, "fused_rope_gqa")
    torch.cuda.synchronize()
    # The planted paths are what the shipped reference accepts (at least that deep).
    for r, result in enumerate(ref_acc):
        depth = max(inputs.trees[r].host_depths)
        assert result["accepted_length"] >= min(planted[r], depth), (r, result, planted[r])
    fp32 = verify_step.divergence_report(our32_acc, ref32_acc, our32_logits, ref32_logits, inputs)
    ours = verify_step.divergence_report(our_acc, ref_acc, our_logits, ref_logits, inputs)
    spread = verify_step.divergence_report(ref32_acc, ref_acc, ref32_logits, ref_logits, inputs)
    print(f"config5 fp32-probability, patched vs reference: {fp32}")
    print(f"config5 bf16-probability, patched vs shipped: {ours}")
    print(f"config5 reference fp32-probability vs shipped: {spread}")
    for row in fp32["divergent"] + ours["divergent"]:
        assert row["flipped"] and row["consistent"], row
    assert fp32["paths_identical"] == fp32["requests"], fp32
    assert ours["paths_identical"] == ours["requests"], ours
