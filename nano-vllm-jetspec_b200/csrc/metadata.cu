// Device-side build of the packed verification metadata from compact tree topology.
//
// The reference builds PackedTreeMetadata on the host (from_host_trees,
// nanovllm/speculative/jetspec/packed_metadata.py:128-198): per request a T x T float
// bias matrix (0 where a node sees another, -inf elsewhere) from the tree's ancestor mask,
// plus offsets, request / row indices and the scratch slots of the round's arena pages,
// then uploads them.  The bias matrices dominate (config 3: ~1.4 MB of the upload and the
// host's numpy work).  Here the host uploads only node counts, prefix lengths, block
// tables, parents (one int32 each) and the arena page list in one copy, and one kernel
// derives every field on the device: one CTA per request builds its ancestor rows in
// shared memory in topological order (row j = row parent(j) | {j}, one lane per 32-bit
// word) and expands them to the bias matrix with coalesced stores.
#include "common.cuh"

namespace {

__device__ uint32_t g_meta_errors;

constexpr int kMetaThreads = 256;

__global__ void __launch_bounds__(kMetaThreads)
    metadata_build_kernel(JtMetadataBuildParams p) {
  extern __shared__ uint32_t rows[];  // [nodes][words] ancestor bitmask of this request
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  int64_t node_off = 0, bias_off = 0;
  for (int i = tid; i < r; i += kMetaThreads) {
    const int64_t c = p.node_counts[i];
    node_off += c;
    bias_off += c * c;
  }
  for (int o = 16; o > 0; o >>= 1) {
    node_off += __shfl_xor_sync(0xffffffffu, node_off, o);
    bias_off += __shfl_xor_sync(0xffffffffu, bias_off, o);
  }
  __shared__ int64_t s_off[2][kMetaThreads / 32];
  if (lane == 0) {
    s_off[0][tid >> 5] = node_off;
    s_off[1][tid >> 5] = bias_off;
  }
  __syncthreads();
  node_off = bias_off = 0;
  for (int w = 0; w < kMetaThreads / 32; ++w) {
    node_off += s_off[0][w];
    bias_off += s_off[1][w];
  }
  const int nodes = p.node_counts[r];
  const int words = (nodes + 31) / 32;
  if (tid == 0) {
    p.cu_seqlens_q[r] = static_cast<int32_t>(node_off);
    p.qq_bias_offsets[r] = bias_off;
    if (r == p.num_requests - 1) {
      p.cu_seqlens_q[r + 1] = static_cast<int32_t>(node_off + nodes);
      p.qq_bias_offsets[r + 1] = bias_off + static_cast<int64_t>(nodes) * nodes;
    }
  }
  const int64_t pages_needed = (node_off + nodes + p.block_size - 1) / p.block_size;
  if (nodes < 1 || nodes > p.max_nodes || node_off + nodes > p.num_nodes ||
      pages_needed > p.num_pages) {
    // The shared-memory rows are sized for max_nodes, and parents / arena pages must hold
    // the request: otherwise it is skipped and flagged.
    if (tid == 0) atomicOr(&g_meta_errors, JT_DEVERR_TREE_TOO_LARGE);
    return;
  }
  const int32_t* parents = p.parents + node_off;
  for (int j = tid; j < nodes; j += kMetaThreads) {
    const int64_t q = node_off + j;
    p.query_to_request[q] = r;
    p.query_local_row[q] = j;
    p.tree_slots[q] = static_cast<int64_t>(p.arena_pages[q / p.block_size]) * p.block_size +
                      q % p.block_size;
  }
  // Ancestor rows in topological order (every parent precedes its child); a parent outside
  // [0, j) leaves the node seeing only itself and is flagged.
  if (tid < 32) {
    for (int j = 0; j < nodes; ++j) {
      const int parent = j == 0 ? -1 : parents[j];
      const bool ok = j == 0 ? parents[0] == -1 : (parent >= 0 && parent < j);
      if (!ok && lane == 0) atomicOr(&g_meta_errors, JT_DEVERR_OUT_OF_RANGE);
      for (int k = lane; k < words; k += 32) {
        uint32_t v = (ok && j > 0) ? rows[parent * words + k] : 0u;
        if (k == (j >> 5)) v |= 1u << (j & 31);
        rows[j * words + k] = v;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  float* bias = p.qq_bias + bias_off;
  const int64_t cells = static_cast<int64_t>(nodes) * nodes;
  for (int64_t e = tid; e < cells; e += kMetaThreads) {
    const int j = static_cast<int>(e / nodes), n = static_cast<int>(e - static_cast<int64_t>(j) * nodes);
    const bool visible = (rows[j * words + (n >> 5)] >> (n & 31)) & 1u;
    bias[e] = visible ? 0.0f : -INFINITY;
  }
}

}  // namespace

int jt_read_errors_meta(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_meta_errors, sizeof(uint32_t)),
                         "read metadata error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_meta_errors, &zero, sizeof(uint32_t)),
                       "clear metadata error word");
}

extern "C" int jt_metadata_build_launch(const JtMetadataBuildParams* pp, cudaStream_t stream) {
  if (pp == nullptr) return jt_fail(JT_ERR_INVALID, "metadata_build: null params");
  const JtMetadataBuildParams& p = *pp;
  if (p.num_requests < 1 || p.block_size < 1 || p.max_nodes < 1 || p.max_nodes > 1024 ||
      p.num_nodes < 1 || p.num_pages < 1)
    return jt_fail(JT_ERR_INVALID, "metadata_build: invalid geometry (1 <= max_nodes <= 1024)");
  if (!p.node_counts || !p.parents || !p.arena_pages || !p.cu_seqlens_q ||
      !p.query_to_request || !p.query_local_row || !p.tree_slots || !p.qq_bias ||
      !p.qq_bias_offsets)
    return jt_fail(JT_ERR_INVALID, "metadata_build: null tensor pointer");
  const size_t smem = static_cast<size_t>(p.max_nodes) * ((p.max_nodes + 31) / 32) * 4;
  int rc = jt_cuda_check(cudaFuncSetAttribute(metadata_build_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(smem)),
                         "metadata smem attribute");
  if (rc != JT_OK) return rc;
  metadata_build_kernel<<<p.num_requests, kMetaThreads, smem, stream>>>(p);
  return jt_cuda_check(cudaGetLastError(), "metadata_build launch");
}
