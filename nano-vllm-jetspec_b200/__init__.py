"""B200-native (sm_100a) JetSpec tree-verification hot path.

Public operators keep the reference's Python signatures so the nano-vLLM JetSpec
verifier, scratch arena and block tables work unchanged:

* packed_tree_attention_gqa  - nanovllm/speculative/jetspec/tree_gqa.py:114
* packed_tree_attention      - nanovllm/speculative/jetspec/paged_backend.py:240
* store_kvcache              - nanovllm/layers/attention.py:38
* copy_accepted_kv           - nanovllm/speculative/jetspec/state.py:64
* PackedTreeMetadata         - nanovllm/speculative/jetspec/packed_metadata.py:16
* rope_scatter(_prevalidated) - nanovllm/speculative/jetspec/tree_fusion.py:172-199
* accept_batch               - nanovllm/speculative/jetspec/serving_ops.py:55 (plus the
                               device-side accept_walk)
* RowParallelLinear          - nanovllm/layers/linear.py:131 (GEMM + all-reduce fused)

All compute runs in libjetspec_b200.so (hand-written CUDA for sm_100a) through a C ABI
(include/jetspec_b200.h).  There is no CPU or library fallback: without the built
library every operator raises LibraryMissingError.
"""
from ._lib import KernelLaunchError, LibraryMissingError, load_library, read_device_errors
from . import ops  # noqa: F401  (registers the jetspec_b200:: custom operators)
from .accept import accept_batch, accept_walk
from .attention import store_kvcache
from .packed_metadata import PackedTreeMetadata, ancestor_mask_from_parents
from .row_linear import RowParallelLinear, row_parallel_linear
from .paged_backend import packed_tree_attention, packed_tree_attention_reference
from .sharding import KvHeadShard, shard_for_rank
from .state import _slots_for_blocks, copy_accepted_kv
from .tree_fusion import rope_scatter, rope_scatter_prevalidated, scatter_tree_kv
from .tree_gqa import packed_tree_attention_gqa

__all__ = [
    "KernelLaunchError", "LibraryMissingError", "load_library", "read_device_errors",
    "store_kvcache", "PackedTreeMetadata", "ancestor_mask_from_parents",
    "packed_tree_attention", "packed_tree_attention_reference", "KvHeadShard",
    "shard_for_rank", "copy_accepted_kv", "scatter_tree_kv", "rope_scatter",
    "rope_scatter_prevalidated", "packed_tree_attention_gqa", "accept_batch", "accept_walk",
    "RowParallelLinear", "row_parallel_linear",
]
