"""CPU oracle for the JetSpec tree-verification path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this package.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm use it, always as the checker or as the timed
CPU restatement of the reference's own CPU path, never as a kernel substitute.

* tree_attention.masked_sdpa     - the reference's PyTorch masked-SDPA oracle in fp32
  (prefix gather through the block table, ancestor mask, GQA expansion, SDPA).
* tree_attention.parent_chain_fp64 - independent fp64 attention of one node over its
  prefix + root-to-node chain (no mask, no bias, no paging).
* kv_cache.store_kvcache / copy_accepted_kv - byte-level numpy restatements of the
  paged KV store and the accepted-only commit.

Parity is pinned against fixtures produced by running the reference itself
(tests/golden/make_golden.py): its scalar FP32 Triton kernel under the Triton CPU
interpreter, its fp64 oracle, its store_kvcache kernel and its copy_accepted_kv.
"""
