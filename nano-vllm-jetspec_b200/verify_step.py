"""Config 5: one full Qwen3-8B tree-verification step through the reference's own verifier.

The model is the reference's ``Qwen3ForCausalLM`` (nanovllm/models/qwen3.py) built with
its own layers and filled through its own weight loaders (``weight_loader`` of every
parameter, with the checkpoint-name mapping of nanovllm/utils/loader.py and
``packed_modules_mapping``, qwen3.py:643-649), from seeded synthetic bf16 tensors in the
Hugging Face layout: there is no checkpoint here.  A step is the reference's packed
verify (``Qwen3Model.forward_packed_tree``, qwen3.py:620-656, attention seam :226-241),
``lm_head`` logits, the greedy acceptance walk (``accept_batch``, serving_ops.py:55-90)
and the accepted-only KV commit (``copy_accepted_kv``, state.py:64-86), on R requests with
C-token contexts and T-node random-parent trees.  The reference arm runs it as shipped
(``target_kernels="fused_rope_gqa"``: its Triton RoPE scatter and grouped tree kernel,
F.linear + NCCL all-reduce); this package's arm runs the same code with
``integration.ReferencePatch`` applied.

Importing this module needs the reference package (``nanovllm``) on ``sys.path``.
"""
from __future__ import annotations

from dataclasses import dataclass
import math
from types import SimpleNamespace
import zlib

import numpy as np
import torch
import torch.distributed as dist

from .packed_metadata import ancestor_mask_from_parents
from .workloads import random_parents

BLOCK = 256


def qwen3_8b_config(num_layers: int = 36):
    """Qwen3-8B's architecture (hidden 4096, 32 q / 8 kv heads of 128, q/k RMSNorm, RoPE
    theta 1e6, SwiGLU 12288, vocabulary 151936, untied head)."""
    from transformers import Qwen3Config

    return Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                       num_hidden_layers=num_layers, num_attention_heads=32,
                       num_key_value_heads=8, head_dim=128, hidden_act="silu",
                       max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1000000.0,
                       attention_bias=False, tie_word_embeddings=False)


def _hf_weights(config):
    """(checkpoint name, global shape, kind) of every tensor of the model."""
    h, inter, d = config.hidden_size, config.intermediate_size, config.head_dim
    q, kv = config.num_attention_heads * d, config.num_key_value_heads * d
    yield "model.embed_tokens.weight", (config.vocab_size, h), "dense"
    for i in range(config.num_hidden_layers):
        pre = f"model.layers.{i}."
        for name, shape in (("self_attn.q_proj.weight", (q, h)), ("self_attn.k_proj.weight", (kv, h)),
                            ("self_attn.v_proj.weight", (kv, h)), ("self_attn.o_proj.weight", (h, q)),
                            ("mlp.gate_proj.weight", (inter, h)), ("mlp.up_proj.weight", (inter, h)),
                            ("mlp.down_proj.weight", (h, inter))):
            yield pre + name, shape, "dense"
        for name, shape in (("input_layernorm.weight", (h,)),
                            ("post_attention_layernorm.weight", (h,)),
                            ("self_attn.q_norm.weight", (d,)), ("self_attn.k_norm.weight", (d,))):
            yield pre + name, shape, "norm"
    yield "model.norm.weight", (h,), "norm"
    yield "lm_head.weight", (config.vocab_size, h), "dense"


def build_reference_model(config, device, seed: int = 5, std: float = 0.02,
                          embed_std: float | None = 1.0, residual_std: float | None = None,
                          head_std: float | None = None):
    """The reference's Qwen3ForCausalLM on ``device`` (bf16), weights loaded through its
    own weight loaders from seeded synthetic checkpoint tensors: dense weights
    N(0, std^2), norm weights 1, the output head N(0, head_std^2) (default std), and a
    numerically stable residual stream: the embedding N(0, embed_std^2) (default 1, a
    unit-scale stream) and the projections that write into it (o_proj, down_proj)
    N(0, residual_std^2), by default std / sqrt(2 x layers) / 32, so that each layer
    adds a small update.  With every weight N(0, 0.02^2) instead, the 36-layer random
    network is chaotic: any rounding difference (the reference's own two attention
    backends against each other, as much as this package against either) grows to a few
    tenths at the logits and flips greedy choices at near-ties, which says nothing about
    either implementation; trained models are not chaotic in that way.  Every rank
    generates the same global tensor per name, so tensor-parallel shards agree.  Needs
    torch.distributed initialised (the reference's layers read the rank and world size
    when built)."""
    from nanovllm.models.qwen3 import Qwen3ForCausalLM

    previous = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            model = Qwen3ForCausalLM(config)
    finally:
        torch.set_default_dtype(previous)
    mapping = getattr(model, "packed_modules_mapping", {})
    gen = torch.Generator(device=device)
    with torch.no_grad():
        for name, shape, kind in _hf_weights(config):
            if kind == "norm":
                tensor = torch.ones(shape, dtype=torch.bfloat16, device=device)
            else:
                gen.manual_seed(seed * 1_000_003 + zlib.crc32(name.encode()))
                scale = std
                if "o_proj" in name or "down_proj" in name:
                    scale = (std / math.sqrt(2 * config.num_hidden_layers) / 32
                             if residual_std is None else residual_std)
                elif "embed_tokens" in name and embed_std is not None:
                    scale = embed_std
                elif name == "lm_head.weight" and head_std is not None:
                    scale = head_std
                tensor = (torch.randn(shape, generator=gen, device=device) * scale).bfloat16()
            for key, (target, shard) in mapping.items():
                if key in name:
                    param = model.get_parameter(name.replace(key, target))
                    param.weight_loader(param, tensor, shard)
                    break
            else:
                param = model.get_parameter(name)
                loader = getattr(param, "weight_loader", None)
                if loader is None:
                    param.data.copy_(tensor)
                else:
                    loader(param, tensor)
            del tensor
    model.eval()
    if dist.is_initialized() and dist.get_world_size() > 1:
        for layer in model.model.layers:
            layer.mlp.forward_dense = _dense_mlp_rank_width(layer.mlp)
    return model


def _dense_mlp_rank_width(mlp):
    """``Qwen3MLP.forward_dense`` (qwen3.py:348-355) with the gate / up split at this
    rank's width.  The reference splits the merged gate_up weight at
    ``output_sizes[0]``, the global intermediate size, which is right only at tensor
    parallelism 1 (its packed verifier requires TP 1, llm_engine.py:355-356); a rank holds
    output_sizes[0] / TP rows of each half, so the split point is half the rank's rows.
    Applied to both arms of a TP > 1 run; at TP 1 the reference's method runs unchanged."""
    import torch.nn.functional as F

    def forward_dense(x):
        weight, bias = mlp.gate_up_proj.weight, mlp.gate_up_proj.bias
        width = weight.shape[0] // 2
        gate = F.linear(x, weight[:width], None if bias is None else bias[:width])
        up = F.linear(x, weight[width:], None if bias is None else bias[width:])
        return mlp.down_proj(F.silu(gate) * up)

    return forward_dense


@dataclass
class VerifyInputs:
    """One round of packed verification: trees, pool, metadata and draft tokens."""
    prefix_lens: list
    parents: list
    block_tables: list
    arena_pages: list
    commit_pages: list
    kv_pool: torch.Tensor
    metadata: object
    tokens: torch.Tensor
    positions: torch.Tensor
    trees: list
    max_depth: int

    @property
    def offsets(self):
        return self.metadata.query_offsets


def _depths(parents):
    depth = [0] * len(parents)
    for i in range(1, len(parents)):
        depth[i] = depth[parents[i]] + 1
    return depth


def make_inputs(config, device, *, requests: int = 32, context: int | list = 2048,
                nodes: int | list = 64, window: int = 8, seed: int = 1005,
                kv_heads: int | None = None, max_depth: int = 16) -> VerifyInputs:
    """Config 5's round: ``requests`` contexts of ``context`` tokens (or a list of
    per-request lengths) whose K/V sit in the paged pool [2, layers, pages, 256, kv_heads,
    128] (a shuffled page order), trees of ``nodes`` (or per-request counts) random-parent
    nodes (parent of i uniform in [max(0, i - window), i - 1]) whose scratch pages come
    from the same pool, random draft tokens, RoPE positions prefix + depth, and the
    metadata the reference builds for its serving rounds
    (``PackedTreeMetadata.from_host_trees``).  Prefix K ~ N(0, 1) and V ~ N(0, 1.28^2)
    (the scales q/k RMSNorm and a 0.02-std v_proj give); under tensor parallelism each
    rank holds its heads' slice of the same global pool."""
    from nanovllm.speculative.jetspec.packed_metadata import PackedTreeMetadata

    heads = config.num_key_value_heads if kv_heads is None else kv_heads
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    rng = np.random.default_rng(seed)
    contexts = [int(context)] * requests if np.isscalar(context) else [int(c) for c in context]
    counts = [int(nodes)] * requests if np.isscalar(nodes) else [int(n) for n in nodes]
    parents = [random_parents(rng, n, window) for n in counts]
    arena_count = -(-sum(counts) // BLOCK)
    commit_count = requests  # one page for each request's accepted tail
    total_pages = sum(-(-c // BLOCK) for c in contexts) + arena_count + commit_count + 1
    order = rng.permutation(total_pages).tolist()
    tables, commit_pages = [], []
    cursor = 0
    for c in contexts:
        tables.append(order[cursor:cursor + -(-c // BLOCK)])
        cursor += -(-c // BLOCK)
    arena = order[cursor:cursor + arena_count]
    cursor += arena_count
    for _ in range(requests):
        commit_pages.append(order[cursor])
        cursor += 1
    layers = config.num_hidden_layers
    pool = torch.empty((2, layers, total_pages, BLOCK, heads, config.head_dim),
                       dtype=torch.bfloat16, device=device)
    gen = torch.Generator(device=device).manual_seed(seed + 31)
    for axis, std in ((0, 1.0), (1, 1.28)):
        for layer in range(layers):
            # The global pool's heads, this rank's slice: identical across TP degrees.
            full = torch.randn((total_pages, BLOCK, config.num_key_value_heads, config.head_dim),
                               generator=gen, device=device)
            lo = rank * heads if world * heads == config.num_key_value_heads else 0
            pool[axis, layer].copy_((full[:, :, lo:lo + heads] * std).bfloat16())
            del full
    trees = []
    for tree in parents:
        depth = _depths(tree)
        trees.append(SimpleNamespace(
            num_nodes=len(tree), host_parents=list(tree), host_depths=depth,
            host_ancestor=torch.from_numpy(ancestor_mask_from_parents(tree))))
    metadata = PackedTreeMetadata.from_host_trees(
        contexts, tables, trees, arena, BLOCK, device=device,
        request_ids=list(range(requests)))
    tokens = torch.from_numpy(rng.integers(0, config.vocab_size, size=sum(counts))).to(device)
    positions = torch.tensor([c + d for c, t in zip(contexts, trees) for d in t.host_depths],
                             dtype=torch.int64, device=device)
    out = VerifyInputs(contexts, parents, tables, arena, commit_pages, pool, metadata,
                       tokens, positions, trees, max_depth)
    refresh_trees(out)
    return out


def refresh_trees(inputs: VerifyInputs) -> None:
    """(Re)derive the host topology the acceptance walk reads (child maps with the
    reference's last-sibling-wins rule, serving_ops.py:30-40) from the current tokens,
    and per-tree device views of the token / parent / depth vectors."""
    tokens = inputs.tokens.tolist()
    device = inputs.tokens.device
    packed_parents = torch.tensor([p for ps in inputs.parents for p in ps], device=device)
    packed_depths = torch.tensor([d for t in inputs.trees for d in t.host_depths], device=device)
    offsets = inputs.offsets
    for r, tree in enumerate(inputs.trees):
        lo, hi = offsets[r], offsets[r + 1]
        host = tokens[lo:hi]
        children = [dict() for _ in range(tree.num_nodes)]
        for node, parent in enumerate(tree.host_parents):
            if parent >= 0:
                children[parent][host[node]] = node
        tree.host_token_ids = host
        tree.child_maps = children
        tree.token_ids = inputs.tokens[lo:hi]
        tree.parent_indices = packed_parents[lo:hi]
        tree.depth = packed_depths[lo:hi]


def verify_logits(model, inputs: VerifyInputs) -> torch.Tensor | None:
    """The reference verifier's forward: packed Target pass, then lm_head (logits on rank
    0 under tensor parallelism, None elsewhere)."""
    with torch.inference_mode():
        hidden, _ = model.model.forward_packed_tree(inputs.tokens, inputs.positions,
                                                    inputs.kv_pool, inputs.metadata)
        return model.compute_logits(hidden)


def set_target_kernels(model, kernels: str = "fused_rope_gqa") -> None:
    """The reference's per-layer kernel switches (batch_runtime.py:126-132)."""
    for layer in model.model.layers:
        layer.self_attn._jetspec_tree_fusion = kernels != "reference"
        layer.self_attn._jetspec_tree_gqa = kernels == "fused_rope_gqa"


def accept(logits, inputs: VerifyInputs):
    """``accept_batch`` as the reference's runtime calls it (batch_runtime.py:551-553),
    looked up at call time so that a ReferencePatch takes effect."""
    from nanovllm.speculative.jetspec import serving_ops

    return serving_ops.accept_batch(logits, inputs.trees, inputs.offsets, inputs.max_depth)


def commit(inputs: VerifyInputs, results) -> int:
    """The accepted nodes' K/V into the canonical slots after each prefix, through the
    reference's ``copy_accepted_kv`` (looked up at call time)."""
    from nanovllm.speculative.jetspec import state

    src, dst = [], []
    slots = inputs.metadata.tree_slot_ids
    for r, result in enumerate(results):
        base = inputs.offsets[r]
        for i, node in enumerate(result["path"]):
            src.append(slots[base + node])
            dst.append(inputs.commit_pages[r] * BLOCK + i)
    device = inputs.kv_pool.device
    return state.copy_accepted_kv(inputs.kv_pool, torch.tensor(src, device=device),
                                  torch.tensor(dst, device=device), BLOCK)


def plant_paths(model, inputs: VerifyInputs, lengths) -> None:
    """Make request r's deepest chain accepted for ``lengths[r]`` steps under the model
    that runs (the reference verifier): one forward per depth, each setting the draft
    token of the next chain node to the current greedy token of its parent.  A node's
    logits depend only on its own and its ancestors' tokens, so earlier plants stay valid.
    Under tensor parallelism rank 0 decides and broadcasts the tokens."""
    chains = []
    for tree in inputs.trees:
        depth = tree.host_depths
        node = int(np.argmax(depth))
        chain = []
        while node != -1:
            chain.append(node)
            node = tree.host_parents[node]
        chains.append(chain[::-1])
    steps = max(min(int(n), len(c) - 1) for n, c in zip(lengths, chains))
    for step in range(steps):
        logits = verify_logits(model, inputs)
        if logits is not None:
            greedy = logits.argmax(-1)
            for r, (n, chain) in enumerate(zip(lengths, chains)):
                if step < min(int(n), len(chain) - 1):
                    lo = inputs.offsets[r]
                    inputs.tokens[lo + chain[step + 1]] = greedy[lo + chain[step]]
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.broadcast(inputs.tokens, src=0)
    refresh_trees(inputs)


def first_divergence(a, b):
    """Per request, the first path position where two acceptance results differ (None
    when the paths are equal)."""
    out = []
    for x, y in zip(a, b):
        px, py = x["path"], y["path"]
        if px == py and x["correction"] == y["correction"]:
            out.append(None)
            continue
        k = 0
        while k < min(len(px), len(py)) and px[k] == py[k]:
            k += 1
        out.append(k)
    return out


def argmax_flip_witness(logits_a: torch.Tensor, logits_b: torch.Tensor) -> dict:
    """The reference's argmax-flip consistency witness (restating
    benchmarks/jetspec_numeric_oracles.py:171-217): with delta = ||A - B||_inf between two
    logits rows (B the reference), a reference winner whose margin over the runner-up
    exceeds 2 delta cannot lose in A.  A row whose argmax differs is "consistent" when
    both the reference's top-2 margin and the gap between B's winner and A's winner
    (measured in B) are at most 2 delta; an inconsistent flip is a large-margin violation.
    Ties follow torch.argmax's first-index rule.  It explains greedy accepted-path
    differences between two verifiers as near-ties; it does not show that delta is small.
    """
    a = logits_a.detach().cpu().double()
    b = logits_b.detach().cpu().double()
    if a.shape != b.shape or a.ndim < 1 or a.shape[-1] < 2:
        raise ValueError("logits must have equal shapes with vocabulary size >= 2")
    if not (torch.isfinite(a).all() and torch.isfinite(b).all()):
        raise ValueError("logits must be finite")
    a = a.reshape(-1, a.shape[-1])
    b = b.reshape(-1, b.shape[-1])
    rows, flips, violations = [], 0, 0
    winners_a = a.argmax(-1)
    winners_b = b.argmax(-1)
    top2 = torch.topk(b, k=2, dim=-1).values
    deltas = (a - b).abs().amax(-1)
    for index in range(a.shape[0]):
        wa, wb = int(winners_a[index]), int(winners_b[index])
        margin = float(top2[index, 0] - top2[index, 1])
        delta = float(deltas[index])
        gap = float(b[index, wb] - b[index, wa])
        flipped = wa != wb
        consistent = margin <= 2 * delta and gap <= 2 * delta
        violation = flipped and not consistent
        flips += int(flipped)
        violations += int(violation)
        rows.append({"row": index, "actual_argmax": wa, "reference_argmax": wb,
                     "argmax_flipped": flipped, "logits_inf_delta": delta,
                     "reference_top2_margin": margin, "two_delta": 2 * delta,
                     "reference_winner_vs_actual_winner_gap": gap,
                     "flip_within_error_envelope": consistent if flipped else None,
                     "large_margin_violation": violation})
    return {"rows_checked": len(rows), "argmax_flips": flips,
            "large_margin_violations": violations,
            "all_flip_witnesses_consistent": violations == 0, "rows": rows}


def divergence_report(actual, reference, actual_logits, reference_logits, inputs) -> dict:
    """Accepted-path agreement of two verifiers on the same round: identical requests, and
    for each divergent one the argmax-flip witness at the node where the paths part (the
    last common node, whose greedy token differs)."""
    divergent = first_divergence(actual, reference)
    rows = []
    for r, k in enumerate(divergent):
        if k is None:
            continue
        row = inputs.offsets[r] + reference[r]["path"][k - 1]
        w = argmax_flip_witness(actual_logits[row:row + 1], reference_logits[row:row + 1])
        rows.append({"request": r, "path_index": k, "flipped": w["argmax_flips"] == 1,
                     "consistent": w["all_flip_witnesses_consistent"],
                     "delta": w["rows"][0]["logits_inf_delta"],
                     "margin": w["rows"][0]["reference_top2_margin"]})
    return {"paths_identical": sum(d is None for d in divergent), "requests": len(divergent),
            "logits_max_abs_diff": float((actual_logits.float() - reference_logits.float()).abs().max()),
            "divergent": rows}
