"""Drop-in wiring of this package into the reference's verifier (the nanovllm package).

The reference looks up its hot-path operators as module attributes at call time:

* ``rope_scatter_prevalidated`` / ``rope_scatter`` - imported inside
  ``Qwen3Attention.forward_paged_tree`` from nanovllm/speculative/jetspec/tree_fusion.py
  (call site nanovllm/models/qwen3.py:226-236);
* ``packed_tree_attention`` - imported there from
  nanovllm/speculative/jetspec/paged_backend.py (qwen3.py:237-241, 261-265);
* ``packed_tree_attention_gqa`` - imported by the dispatcher from
  nanovllm/speculative/jetspec/tree_gqa.py (paged_backend.py:273-276);
* ``copy_accepted_kv`` - a module global of nanovllm/speculative/jetspec/state.py, called at
  state.py:502 and :888;
* ``accept_batch`` - imported inside ``BatchRuntime._accept_batch`` from
  nanovllm/speculative/jetspec/serving_ops.py (batch_runtime.py:551-553);
* ``store_kvcache`` - a module global of nanovllm/layers/attention.py (call site :123);

so replacing those attributes routes every later call through this package with no edit
of the reference's source.  The row-parallel projections are module instances built when
the model is constructed (``o_proj`` and ``down_proj``, nanovllm/layers/linear.py:131-156);
``swap_row_parallel`` replaces each instance in a built model by this package's
``RowParallelLinear`` sharing the same weight tensor.  ``ReferencePatch`` applies both and
undoes them on exit.
"""
from __future__ import annotations

import importlib

import torch

from . import accept as _accept
from . import attention as _attention
from . import paged_backend as _paged_backend
from . import row_linear as _row_linear
from . import state as _state
from . import tree_fusion as _tree_fusion
from . import tree_gqa as _tree_gqa

# (reference module, attribute) -> this package's replacement.
PATCH_SITES = {
    ("nanovllm.speculative.jetspec.tree_fusion", "rope_scatter_prevalidated"):
        _tree_fusion.rope_scatter_prevalidated,
    ("nanovllm.speculative.jetspec.tree_fusion", "rope_scatter"): _tree_fusion.rope_scatter,
    ("nanovllm.speculative.jetspec.paged_backend", "packed_tree_attention"):
        _paged_backend.packed_tree_attention,
    ("nanovllm.speculative.jetspec.tree_gqa", "packed_tree_attention_gqa"):
        _tree_gqa.packed_tree_attention_gqa,
    ("nanovllm.speculative.jetspec.state", "copy_accepted_kv"): _state.copy_accepted_kv,
    ("nanovllm.speculative.jetspec.serving_ops", "accept_batch"): _accept.accept_batch,
    ("nanovllm.layers.attention", "store_kvcache"): _attention.store_kvcache,
}


def swap_row_parallel(model: torch.nn.Module) -> list:
    """Replace every reference RowParallelLinear inside ``model`` by this package's,
    sharing the weight (and bias) tensors; returns the undo list."""
    reference = importlib.import_module("nanovllm.layers.linear").RowParallelLinear
    undo = []
    for parent in list(model.modules()):
        for name, child in list(parent.named_children()):
            if not isinstance(child, reference):
                continue
            ours = _row_linear.RowParallelLinear.__new__(_row_linear.RowParallelLinear)
            torch.nn.Module.__init__(ours)
            ours.tp_size, ours.tp_rank, ours.tp_dim = child.tp_size, child.tp_rank, 1
            ours.weight = child.weight
            if child.bias is not None:
                ours.bias = child.bias
            else:
                ours.register_parameter("bias", None)
            setattr(parent, name, ours)
            undo.append((parent, name, child))
    return undo


class ReferencePatch:
    """Context manager: route the reference's hot path through this package.

    ``with ReferencePatch(model):`` patches the operator sites of ``PATCH_SITES`` and, when
    ``model`` is given and ``row_parallel`` is true, swaps its row-parallel projections; on
    exit every original is put back.  The reference package (``nanovllm``) must be
    importable.
    """

    def __init__(self, model: torch.nn.Module | None = None, *, row_parallel: bool = True):
        self.model = model
        self.row_parallel = row_parallel
        self._saved: list = []
        self._swapped: list = []

    def __enter__(self):
        for (module_name, attr), replacement in PATCH_SITES.items():
            module = importlib.import_module(module_name)
            self._saved.append((module, attr, getattr(module, attr)))
            setattr(module, attr, replacement)
        if self.model is not None and self.row_parallel:
            self._swapped = swap_row_parallel(self.model)
        return self

    def __exit__(self, *exc):
        for parent, name, original in reversed(self._swapped):
            setattr(parent, name, original)
        for module, attr, original in reversed(self._saved):
            setattr(module, attr, original)
        self._saved, self._swapped = [], []
        return False
