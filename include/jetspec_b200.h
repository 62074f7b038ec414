/*
 * jetspec_b200.h -- C ABI of the B200 (sm_100a) JetSpec tree-verification kernels.
 *
 * Everything here is plain C: POD parameter structs holding device pointers, element
 * strides and sizes, plus a cudaStream_t.  No PyTorch (or other framework) type
 * appears in any signature.  Every launcher enqueues work on the given stream and
 * returns immediately: it never synchronises and never allocates device memory.
 * jt_tree_attn_launch, jt_kv_store_launch and jt_kv_commit_launch may be called inside
 * CUDA-graph stream capture.  Return value: JT_OK (0) or a negative JT_ERR_* code;
 * jt_last_error() then holds a one-line message (thread-local).
 *
 * Paths below are relative to the nano-vllm-jetspec reference project.
 */
#ifndef JETSPEC_B200_H
#define JETSPEC_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JT_ABI_VERSION 1

enum JtStatus {
  JT_OK = 0,
  JT_ERR_INVALID = -1,     /* bad geometry / dtype / stride / null pointer */
  JT_ERR_WORKSPACE = -2,   /* workspace missing or smaller than jt_tree_attn_workspace_size */
  JT_ERR_CUDA = -3,        /* a CUDA runtime call failed (message has the CUDA error) */
  JT_ERR_UNSUPPORTED = -4  /* valid request this build does not implement */
};

enum JtDtype { JT_BF16 = 0, JT_F16 = 1, JT_F32 = 2 };

/* Flags for JtTreeAttnParams.flags */
#define JT_FLAG_FP32_PROBABILITY 1u  /* PV with near-fp32 probabilities (hi+lo bf16 split)  */
#define JT_FLAG_PORTABLE_CORE 2u     /* force the warp-level mma.sync core (A/B testing)     */

/*
 * Packed ragged tree attention over a paged KV cache.
 *
 * Replaces the Triton launch inside packed_tree_attention_gqa
 * (nanovllm/speculative/jetspec/tree_gqa.py:114-140, kernel :32-111) and the packed
 * dispatcher's backends (nanovllm/speculative/jetspec/paged_backend.py:240-306).
 *
 * Semantics per packed query row i of request r (local node j), query head hq,
 * kv head h = hq / groups: keys are positions 0..P_r+T_r-1 of the request
 * (prefix pages from block_tables, then the T_r tree nodes at tree_slots); key
 * position p is visible iff p < P_r, or p = P_r+n with n <= j and
 * qq_bias[qq_bias_offsets[r] + j*T_r + n] == 0.  Scores are (q.k)*scale with fp32
 * accumulation, softmax in fp32, probabilities rounded to the input dtype for the
 * PV product (unless JT_FLAG_FP32_PROBABILITY), output = acc / sum.
 *
 * Metadata arrays are the device tensors of PackedTreeMetadata
 * (nanovllm/speculative/jetspec/packed_metadata.py:16-33).  Strides are in elements;
 * the last dimension of q, out, k_pool and v_pool must be contiguous, the row
 * strides must be multiples of 8 elements and every base 16-byte aligned.
 */
typedef struct JtTreeAttnParams {
  void* out;                       /* [total_queries, q_heads, head_dim], out_dtype      */
  const void* q;                   /* [total_queries, q_heads, head_dim], dtype          */
  const void* k_pool;              /* [num_blocks, block_size, kv_heads, head_dim]      */
  const void* v_pool;              /* same geometry as k_pool                           */
  const int32_t* cu_seqlens_q;     /* [num_requests + 1]                                */
  const int32_t* query_to_request; /* [total_queries]                                   */
  const int32_t* query_local_row;  /* [total_queries]                                   */
  const int32_t* prefix_lens;      /* [num_requests]                                    */
  const int32_t* node_counts;      /* [num_requests]                                    */
  const int32_t* block_tables;     /* [num_requests, table_width] (row stride below)     */
  const int64_t* tree_slots;       /* [total_queries] physical slot = page*bs + offset  */
  const float* qq_bias;            /* [sum T_r^2] 0 / -inf                              */
  const int64_t* qq_bias_offsets;  /* [num_requests + 1]                                */
  int32_t num_requests;
  int32_t total_queries;
  int32_t num_kv_heads;
  int32_t groups;                  /* query heads per kv head                           */
  int32_t head_dim;                /* 64 or 128                                         */
  int32_t block_size;              /* tokens per page                                   */
  int32_t table_width;             /* columns of block_tables                           */
  int32_t dtype;                   /* JT_BF16 or JT_F16                                 */
  int32_t out_dtype;               /* dtype or JT_F32                                   */
  uint32_t flags;                  /* JT_FLAG_*                                         */
  int64_t num_blocks;              /* pages in the pool                                 */
  int64_t q_stride0, q_stride1;
  int64_t out_stride0, out_stride1;
  int64_t table_stride0;
  int64_t k_stride0, k_stride1, k_stride2;
  int64_t v_stride0, v_stride1, v_stride2;
  float scale;
  int32_t split_keys;              /* 0 = automatic; else keys per split (multiple of 1024) */
  void* workspace;                 /* device scratch, >= jt_tree_attn_workspace_size     */
  size_t workspace_bytes;
} JtTreeAttnParams;

/* Bytes of device workspace jt_tree_attn_launch needs for this geometry.  Depends only
 * on (num_requests, total_queries, num_kv_heads, groups, head_dim), never on prefix
 * lengths or node counts, so one workspace serves every CUDA-graph replay of a shape. */
int jt_tree_attn_workspace_size(int32_t num_requests, int32_t total_queries,
                                int32_t num_kv_heads, int32_t groups, int32_t head_dim,
                                size_t* bytes);

int jt_tree_attn_launch(const JtTreeAttnParams* params, cudaStream_t stream);

/*
 * jt_tree_attn_launch without a caller-provided workspace: it allocates nothing.
 * No counterpart in the reference (which always allocates through PyTorch).
 *
 * For callers that cannot allocate device memory: a host that binds only this C ABI
 * and owns all device memory through its own fixed arenas can pass the tensors it holds
 * but has no allocator to obtain scratch from.  The scratch comes from one file-scope
 * device array of 32 MiB (every GPU that loads the library holds it until exit); the
 * split-KV partial results are confined to 16 MiB of it, so the device plan uses
 * coarser splits than jt_tree_attn_launch.  Geometries whose scratch exceeds 32 MiB
 * are rejected with JT_ERR_WORKSPACE.  `workspace` / `workspace_bytes` are ignored.
 *
 * Every call made outside stream capture looks up the array's device address
 * (cudaGetSymbolAddress, in the current device and context) and records it for that
 * context; a call made during capture uses the record and is refused (JT_ERR_INVALID)
 * when no call has been made in the current context yet, so make the first call on a
 * device before any stream capture.  All calls share the array and the plan kernel
 * re-initialises what must start at zero on every call, but calls that overlap on the
 * GPU (different streams, or concurrent graph replays) race on it: serialise them.
 */
int jt_tree_attn_launch_noalloc(const JtTreeAttnParams* params, cudaStream_t stream);

/*
 * Paged KV store: for token i with slot s = slot_mapping[i] (skipped when s < 0),
 * k_cache[s / block_size, s % block_size, :, :] = key[i]; same for value.
 *
 * Replaces store_kvcache (nanovllm/layers/attention.py:38-45, kernel :15-35) and the
 * tree-node scratch write in forward_paged_tree (nanovllm/models/qwen3.py:255-258).
 */
typedef struct JtKvStoreParams {
  const void* key;      /* [num_tokens, kv_heads, head_dim] */
  const void* value;
  void* k_cache;        /* [num_blocks, block_size, kv_heads, head_dim] */
  void* v_cache;
  const void* slot_mapping;   /* [num_tokens] int32 or int64 */
  int32_t slot_is_int64;
  int32_t num_tokens;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t elem_bytes;   /* 2 or 4 */
  int32_t block_size;
  int64_t num_blocks;
  int64_t key_stride0, key_stride1;
  int64_t value_stride0, value_stride1;
  int64_t k_stride0, k_stride1, k_stride2;
  int64_t v_stride0, v_stride1, v_stride2;
} JtKvStoreParams;

int jt_kv_store_launch(const JtKvStoreParams* params, cudaStream_t stream);

/*
 * Accepted-only KV commit across both KV axes and every layer of a 6-D pool
 * [2, layers, num_blocks, block_size, kv_heads, head_dim]:
 *   pool[:, :, dst//bs, dst%bs] = pool[:, :, src//bs, src%bs]   (gather before scatter)
 *
 * Replaces copy_accepted_kv (nanovllm/speculative/jetspec/state.py:64-86).  Every read
 * of an (axis, layer) plane completes before any write to it (a cooperative launch with a
 * grid barrier between the gather and the scatter, the planes taken in groups that fit
 * the grid's shared memory), so overlapping source/destination sets behave like the
 * reference's materialised copy.  jt_kv_commit_max_slots() is the largest slot count one
 * call accepts on the current device (one 16-byte word per slot staged per SM x 12288:
 * about 1.8 million slots on a 148-SM B200; 12288 when no device is visible).
 */
typedef struct JtKvCommitParams {
  void* kv_pool;
  const void* source_slots;       /* [num_slots] int32 or int64 */
  const void* destination_slots;  /* [num_slots] int32 or int64 */
  int32_t slot_is_int64;
  int32_t num_slots;
  int32_t num_layers;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t elem_bytes;
  int32_t block_size;
  int64_t num_blocks;
  int64_t stride_axis, stride_layer, stride_block, stride_offset, stride_head; /* elements */
} JtKvCommitParams;

int jt_kv_commit_launch(const JtKvCommitParams* params, cudaStream_t stream);
int32_t jt_kv_commit_max_slots(void);

/*
 * HF-order RoPE of Q and K with the tree-node K/V scatter, in one launch:
 *   out[r, h]                    = rope(q[r, h], positions[r])      every query head h
 *   k_pool[s / bs, s % bs, kh]   = rope(k[r, kh], positions[r])     s = node_slots[r]
 *   v_pool[s / bs, s % bs, kh]   = v[r, kh]
 * rope(x) = [x1*cos - x2*sin, x2*cos + x1*sin] over the two halves of the head dim, with
 * cos/sin = cache[positions[r], :dim/2] and [dim/2:] converted to the operand type, and
 * every product rounded to the operand type before the add / subtract (eager PyTorch
 * order; no fused multiply-add).  Bit-exact with rope_scatter_prevalidated
 * (nanovllm/speculative/jetspec/tree_fusion.py:181-199, kernel :31-83).  The caller
 * guarantees in-range positions, unique in-range slots and non-aliasing buffers (the
 * prevalidated contract); out-of-range slots are skipped and flagged in the device error
 * word.  All strides in elements.
 */
typedef struct JtRopeScatterParams {
  const void* q;             /* [rows, q_heads, dim]  bf16 or fp32 */
  const void* k;             /* [rows, kv_heads, dim] */
  const void* v;             /* [rows, kv_heads, dim] */
  const void* positions;     /* [rows] int32 or int64 */
  const void* cos_sin_cache; /* [max_position, dim] (cos | sin), bf16 or fp32 */
  const void* node_slots;    /* [rows] int32 or int64 */
  void* out;                 /* [rows, q_heads, dim] rotated Q */
  void* k_pool;              /* [pages, page_size, kv_heads, dim] */
  void* v_pool;
  int32_t dtype;             /* JT_BF16 or JT_F32 (q, k, v, out, pools) */
  int32_t cache_dtype;       /* JT_BF16 or JT_F32 */
  int32_t positions_is_int64, slots_is_int64;
  int32_t rows, q_heads, kv_heads, head_dim, page_size;
  int64_t num_pages;
  int64_t q_stride0, q_stride1, q_stride2;
  int64_t k_stride0, k_stride1, k_stride2;
  int64_t v_stride0, v_stride1, v_stride2;
  int64_t positions_stride, slots_stride, cache_stride0, cache_stride_last;
  int64_t out_stride0, out_stride1, out_stride2;
  int64_t kp_stride0, kp_stride1, kp_stride2, kp_stride3;
  int64_t vp_stride0, vp_stride1, vp_stride2, vp_stride3;
} JtRopeScatterParams;

int jt_rope_scatter_launch(const JtRopeScatterParams* params, cudaStream_t stream);

/*
 * Greedy acceptance walk over the packed verification trees (replaces the argmax
 * download and host walk of accept_batch, nanovllm/speculative/jetspec/serving_ops.py:55-90,
 * called from batch_runtime.py:551-553).  Per request r (nodes offsets[r]..offsets[r+1]-1,
 * root first): path = [0]; while len(path) <= max_depth, follow the child c of the last
 * node n with parent_indices[c] == n and token_ids[c] == argmax(logits[n]) (the last such
 * child when siblings repeat a token); correction = argmax(logits[last node]).  argmax is
 * torch.argmax's: NaN ranks highest, ties go to the lowest index.  Only the logits rows of
 * the nodes on the path are read.  Outputs: path[r, :] (node indices, -1 padded),
 * accepted_length[r] = len(path) - 1, correction[r], outputs[r, :] = token_ids[path[1:]]
 * followed by the correction (-1 padded).  Depths along the path that are not 0, 1, 2, ...
 * (when depths is given) set device error bit 0.
 */
typedef struct JtAcceptWalkParams {
  const void* logits;              /* [Q, vocab] bf16, f16 or f32 (row stride below)      */
  const int64_t* token_ids;        /* [Q] draft token of each node                        */
  const int64_t* parent_indices;   /* [Q] request-local parent, -1 for the root           */
  const int64_t* depths;           /* [Q] or NULL (no depth check)                        */
  const int32_t* offsets;          /* [R + 1] packed node offsets (cu_seqlens_q)           */
  int32_t* path;                   /* [R, path_stride]                                    */
  int32_t* accepted_length;        /* [R]                                                 */
  int64_t* correction;             /* [R]                                                 */
  int64_t* outputs;                /* [R, path_stride]                                    */
  int64_t logits_stride0;          /* elements between logits rows                        */
  int32_t logits_dtype;            /* JT_BF16, JT_F16 or JT_F32                           */
  int32_t vocab, num_requests, max_depth, path_stride;  /* path_stride >= max_depth + 1  */
  int32_t num_nodes;               /* Q: rows of logits / entries of the node arrays; a
                                      request whose offsets leave [0, Q] is skipped and
                                      flagged (device error bit 0)                      */
} JtAcceptWalkParams;

int jt_accept_walk_launch(const JtAcceptWalkParams* params, cudaStream_t stream);

/*
 * Device-side build of the packed verification metadata (the fields of
 * PackedTreeMetadata, nanovllm/speculative/jetspec/packed_metadata.py:16-33, as
 * from_host_trees builds them, :128-198) from compact topology: per request its node count
 * and each node's request-local parent (parents[0] = -1, every parent before its child),
 * plus the round's arena pages (scratch slot of packed node q = arena_pages[q / block_size]
 * * block_size + q % block_size).  Writes cu_seqlens_q, query_to_request, query_local_row,
 * tree_slots, qq_bias (0 where node j sees node n: n is j or an ancestor of j; -inf
 * elsewhere) and qq_bias_offsets.  A parent out of order sets device error bit 0 and
 * leaves the node seeing only itself.
 */
typedef struct JtMetadataBuildParams {
  const int32_t* node_counts;  /* [R]                                               */
  const int32_t* parents;      /* [Q] request-local parent indices                  */
  const int32_t* arena_pages;  /* [ceil(Q / block_size)] scratch pages of the round */
  int32_t* cu_seqlens_q;       /* [R + 1]                                           */
  int32_t* query_to_request;   /* [Q]                                               */
  int32_t* query_local_row;    /* [Q]                                               */
  int64_t* tree_slots;         /* [Q]                                               */
  float* qq_bias;              /* [sum of T_r^2]                                    */
  int64_t* qq_bias_offsets;    /* [R + 1]                                           */
  int32_t num_requests, block_size;
  int32_t max_nodes;           /* max T_r (<= 1024): sizes the kernel's shared memory */
  int32_t num_nodes;           /* Q = sum of node_counts (entries of parents)        */
  int32_t num_pages;           /* entries of arena_pages; ceil(Q / block_size) needed */
} JtMetadataBuildParams;

int jt_metadata_build_launch(const JtMetadataBuildParams* params, cudaStream_t stream);

/*
 * Row-parallel linear with its all-reduce fused in: out = sum over the group's ranks of
 * x_r W_r^T (+ bias, added once).  Replaces RowParallelLinear.forward
 * (nanovllm/layers/linear.py:153-156: F.linear on the rank's input shard with the bias on
 * rank 0 only, then dist.all_reduce of the [M, N] result), used by the Qwen3 o_proj and
 * down_proj.  One launch per rank, on each rank's own GPU; every rank of the group makes
 * the same call (same m, n, k, dtype, epoch).  x [m, k] (row stride x_stride), weight
 * [n, k] (nn.Linear layout, row stride w_stride), out [m, n] contiguous, bias [n] or NULL;
 * bf16 or f16; n a multiple of 32, k a multiple of 8.  For world > 1, workspaces[r] is
 * rank r's workspace (jt_row_linear_workspace_size bytes, zeroed once when allocated,
 * 256-byte aligned) as this process addresses it (its own, and the peers' opened through
 * jt_ipc_open_handle).  epoch 0 (the usual value) takes the call's epoch from a counter in
 * the rank's workspace that the kernel advances itself, so a captured launch replays
 * correctly; a nonzero epoch (1, 2, 3, ... on every rank, never mixed with 0 on one
 * workspace) is used as given (consecutive calls take consecutive epochs: a pair of ranks
 * alternates its receive slots with the epoch's parity).  A rank whose peers do not arrive
 * within wait_limit_cycles (0: about ten seconds) flags device error bit 2 and leaves its output
 * incomplete.
 */
typedef struct JtRowLinearParams {
  const void* x;
  const void* weight;
  const void* bias;          /* [n] or NULL; only rank 0's is added                   */
  void* out;
  int64_t m, n, k;
  int64_t x_stride, w_stride;
  int32_t dtype;             /* JT_BF16 or JT_F16                                     */
  int32_t rank, world;       /* 1 <= world <= 8                                       */
  void* const* workspaces;   /* [world], or NULL when world == 1                      */
  uint32_t epoch;
  int64_t wait_limit_cycles;
} JtRowLinearParams;

int jt_row_linear_launch(const JtRowLinearParams* params, cudaStream_t stream);
/* Bytes of one rank's exchange workspace (0 for world == 1, -1 for invalid sizes). */
int64_t jt_row_linear_workspace_size(int64_t m, int64_t n, int32_t world);
/* Test form on one GPU: one cooperative launch plays every rank of a group whose inputs,
 * outputs and workspaces all live on the current device; ranks[i].rank == i. */
int jt_row_linear_emulate(const JtRowLinearParams* ranks, int32_t count, cudaStream_t stream);
/* Workspace plumbing: a zeroed cudaMalloc allocation (its IPC handle maps its first byte),
 * and the CUDA IPC handle exchange between the ranks' processes (64-byte handles). */
int jt_device_alloc_zeroed(int64_t bytes, void** ptr);
int jt_device_free(void* ptr);
int jt_ipc_get_handle(const void* ptr, void* handle);
int jt_ipc_open_handle(const void* handle, void** ptr);
int jt_ipc_close_handle(void* ptr);

/*
 * Failure detection without a GPU fault: runs one thread that waits, with the kernels'
 * bounded-wait routine and a limit of limit_cycles, on an mbarrier nothing arrives on.
 * Synchronous (diagnostics).  out[0] = 1 if the wait claimed completion (a failure),
 * out[1] = the abort flag the wait raised (expected 1), out[2] = cycles spent waiting.
 * Afterwards jt_read_device_errors reports bit 2 (timeout), and the context stays usable.
 */
int jt_selftest_bounded_wait(int64_t limit_cycles, int32_t* out);

/* Library information / diagnostics. */
int32_t jt_abi_version(void);
const char* jt_last_error(void);
/* Reads and clears the device-side error word of the current device (synchronises;
 * diagnostics only).  Bit 0: a slot/page index outside the pool was skipped;
 * bit 1: a tree larger than the kernel's mask capacity was skipped; bit 2: a bounded
 * pipeline wait ran out (the launch's output is invalid). */
int jt_read_device_errors(uint32_t* errors);

#ifdef __cplusplus
}
#endif

#endif /* JETSPEC_B200_H */
