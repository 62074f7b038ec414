// Paged KV writes around tree verification:
//   * jt_kv_store_launch  - warp-per-token indexed store into the paged pool
//     (store_kvcache, nanovllm/layers/attention.py:15-45; tree-node scatter,
//     nanovllm/models/qwen3.py:255-258).
//   * jt_kv_commit_launch - accepted-only commit across K/V and every layer
//     (copy_accepted_kv, nanovllm/speculative/jetspec/state.py:64-86).
// Both are pure byte movers: results are bit-identical to the reference's copies.
#include "common.cuh"

namespace {

__device__ uint32_t g_kv_errors;

constexpr int kStoreThreads = 256;
constexpr int kCommitThreads = 256;
constexpr int kCommitSmemCap = 192 * 1024;  // bytes of staging per commit CTA

__device__ __forceinline__ int64_t load_slot(const void* base, int is64, int64_t i) {
  return is64 ? static_cast<const int64_t*>(base)[i]
              : static_cast<int64_t>(static_cast<const int32_t*>(base)[i]);
}

// One warp per token.  Each lane moves 16-byte words (VEC == 16) or single
// elements (VEC == elem_bytes) for layouts that are not 16-byte aligned.
template <int VEC>
__global__ void __launch_bounds__(kStoreThreads) kv_store_kernel(JtKvStoreParams p) {
  const int64_t token = (static_cast<int64_t>(blockIdx.x) * kStoreThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (token >= p.num_tokens) return;
  const int64_t slot = load_slot(p.slot_mapping, p.slot_is_int64, token);
  if (slot < 0) return;  // padding slot (-1) is skipped, as in the reference
  const int64_t page = slot / p.block_size;
  const int64_t offset = slot - page * p.block_size;
  if (page >= p.num_blocks) {
    if (lane == 0) atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
    return;
  }
  const int eb = p.elem_bytes;
  const int words_per_head = p.head_dim * eb / VEC;
  const int words = p.num_kv_heads * words_per_head;
  const char* ksrc = static_cast<const char*>(p.key) + token * p.key_stride0 * eb;
  const char* vsrc = static_cast<const char*>(p.value) + token * p.value_stride0 * eb;
  char* kdst = static_cast<char*>(p.k_cache) + (page * p.k_stride0 + offset * p.k_stride1) * eb;
  char* vdst = static_cast<char*>(p.v_cache) + (page * p.v_stride0 + offset * p.v_stride1) * eb;
  for (int w = lane; w < words; w += 32) {
    const int h = w / words_per_head;
    const int c = (w - h * words_per_head) * VEC;
    const char* ks = ksrc + h * p.key_stride1 * eb + c;
    const char* vs = vsrc + h * p.value_stride1 * eb + c;
    char* kd = kdst + h * p.k_stride2 * eb + c;
    char* vd = vdst + h * p.v_stride2 * eb + c;
    if constexpr (VEC == 16) {
      const int4 kv = __ldg(reinterpret_cast<const int4*>(ks));
      const int4 vv = __ldg(reinterpret_cast<const int4*>(vs));
      *reinterpret_cast<int4*>(kd) = kv;
      *reinterpret_cast<int4*>(vd) = vv;
    } else if constexpr (VEC == 4) {
      *reinterpret_cast<uint32_t*>(kd) = *reinterpret_cast<const uint32_t*>(ks);
      *reinterpret_cast<uint32_t*>(vd) = *reinterpret_cast<const uint32_t*>(vs);
    } else {
      *reinterpret_cast<uint16_t*>(kd) = *reinterpret_cast<const uint16_t*>(ks);
      *reinterpret_cast<uint16_t*>(vd) = *reinterpret_cast<const uint16_t*>(vs);
    }
  }
}

// One CTA per (axis, layer, kv head, chunk of the head's row).  The CTA first gathers
// its chunk of every accepted source slot into shared memory, then scatters to the
// destinations: no write of a plane can precede a read of the same plane, so the
// copy is overlap-safe like the reference's materialised gather + scatter.
__global__ void __launch_bounds__(kCommitThreads)
    kv_commit_kernel(JtKvCommitParams p, int chunk_bytes, int chunks_per_head) {
  extern __shared__ __align__(16) unsigned char staging[];
  int plane = blockIdx.x;
  const int chunk = plane % chunks_per_head;
  plane /= chunks_per_head;
  const int head = plane % p.num_kv_heads;
  plane /= p.num_kv_heads;
  const int layer = plane % p.num_layers;
  const int axis = plane / p.num_layers;
  const int eb = p.elem_bytes;
  char* base = static_cast<char*>(p.kv_pool) +
               (axis * p.stride_axis + layer * p.stride_layer + head * p.stride_head) * eb +
               chunk * chunk_bytes;
  const int words = chunk_bytes / 16;
  const int total = p.num_slots * words;
  const int64_t pool_slots = p.num_blocks * p.block_size;
  for (int i = threadIdx.x; i < total; i += kCommitThreads) {
    const int s = i / words;
    const int w = i - s * words;
    const int64_t slot = load_slot(p.source_slots, p.slot_is_int64, s);
    int4 value = make_int4(0, 0, 0, 0);
    if (slot >= 0 && slot < pool_slots) {
      const int64_t page = slot / p.block_size;
      const int64_t off = slot - page * p.block_size;
      value = *reinterpret_cast<const int4*>(
          base + (page * p.stride_block + off * p.stride_offset) * eb + w * 16);
    } else if (w == 0) {
      atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
    }
    reinterpret_cast<int4*>(staging)[i] = value;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += kCommitThreads) {
    const int s = i / words;
    const int w = i - s * words;
    const int64_t slot = load_slot(p.destination_slots, p.slot_is_int64, s);
    const int64_t src = load_slot(p.source_slots, p.slot_is_int64, s);
    if (slot < 0 || slot >= pool_slots || src < 0 || src >= pool_slots) {
      if (w == 0) atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
      continue;
    }
    const int64_t page = slot / p.block_size;
    const int64_t off = slot - page * p.block_size;
    *reinterpret_cast<int4*>(base + (page * p.stride_block + off * p.stride_offset) * eb +
                             w * 16) = reinterpret_cast<const int4*>(staging)[i];
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride16(int64_t stride, int eb) { return ((stride * eb) & 15) == 0; }

// Largest staging chunk (64, 32 or 16 bytes of each head row) that keeps all
// num_slots rows of one plane within the shared-memory budget; 0 if none fits.
int commit_chunk_bytes(int row_bytes, int num_slots) {
  for (int cb = 64; cb >= 16; cb >>= 1) {
    if (row_bytes % cb != 0) continue;
    if (static_cast<int64_t>(num_slots) * cb <= kCommitSmemCap) return cb;
  }
  return 0;
}

}  // namespace

int jt_read_errors_kv(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_kv_errors, sizeof(uint32_t)),
                         "read kv error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_kv_errors, &zero, sizeof(uint32_t)),
                       "clear kv error word");
}

extern "C" int jt_kv_store_launch(const JtKvStoreParams* p, cudaStream_t stream) {
  if (p == nullptr) return jt_fail(JT_ERR_INVALID, "kv_store: null params");
  if (p->num_tokens < 0 || p->num_kv_heads <= 0 || p->head_dim <= 0 || p->block_size <= 0 ||
      p->num_blocks <= 0)
    return jt_fail(JT_ERR_INVALID, "kv_store: invalid geometry");
  if (p->elem_bytes != 2 && p->elem_bytes != 4)
    return jt_fail(JT_ERR_INVALID, "kv_store: element size must be 2 or 4 bytes");
  if (p->num_tokens == 0) return JT_OK;
  if (!p->key || !p->value || !p->k_cache || !p->v_cache || !p->slot_mapping)
    return jt_fail(JT_ERR_INVALID, "kv_store: null tensor pointer");
  const int eb = p->elem_bytes;
  const bool vec = aligned16(p->key) && aligned16(p->value) && aligned16(p->k_cache) &&
                   aligned16(p->v_cache) && ((p->head_dim * eb) % 16 == 0) &&
                   stride16(p->key_stride0, eb) && stride16(p->key_stride1, eb) &&
                   stride16(p->value_stride0, eb) && stride16(p->value_stride1, eb) &&
                   stride16(p->k_stride0, eb) && stride16(p->k_stride1, eb) &&
                   stride16(p->k_stride2, eb) && stride16(p->v_stride0, eb) &&
                   stride16(p->v_stride1, eb) && stride16(p->v_stride2, eb);
  const int64_t threads = static_cast<int64_t>(p->num_tokens) * 32;
  const unsigned blocks = static_cast<unsigned>((threads + kStoreThreads - 1) / kStoreThreads);
  if (vec)
    kv_store_kernel<16><<<blocks, kStoreThreads, 0, stream>>>(*p);
  else if (eb == 4)
    kv_store_kernel<4><<<blocks, kStoreThreads, 0, stream>>>(*p);
  else
    kv_store_kernel<2><<<blocks, kStoreThreads, 0, stream>>>(*p);
  return jt_cuda_check(cudaGetLastError(), "kv_store launch");
}

extern "C" int32_t jt_kv_commit_max_slots(void) { return kCommitSmemCap / 16; }

extern "C" int jt_kv_commit_launch(const JtKvCommitParams* p, cudaStream_t stream) {
  if (p == nullptr) return jt_fail(JT_ERR_INVALID, "kv_commit: null params");
  if (p->num_slots < 0 || p->num_layers <= 0 || p->num_kv_heads <= 0 || p->head_dim <= 0 ||
      p->block_size <= 0 || p->num_blocks <= 0)
    return jt_fail(JT_ERR_INVALID, "kv_commit: invalid geometry");
  if (p->elem_bytes != 2 && p->elem_bytes != 4)
    return jt_fail(JT_ERR_INVALID, "kv_commit: element size must be 2 or 4 bytes");
  if (p->num_slots == 0) return JT_OK;
  if (!p->kv_pool || !p->source_slots || !p->destination_slots)
    return jt_fail(JT_ERR_INVALID, "kv_commit: null tensor pointer");
  const int eb = p->elem_bytes;
  const int row_bytes = p->head_dim * eb;
  if (!aligned16(p->kv_pool) || row_bytes % 16 != 0 || !stride16(p->stride_axis, eb) ||
      !stride16(p->stride_layer, eb) || !stride16(p->stride_block, eb) ||
      !stride16(p->stride_offset, eb) || !stride16(p->stride_head, eb))
    return jt_fail(JT_ERR_INVALID,
                   "kv_commit: pool rows must be 16-byte aligned with 16-byte multiple strides");
  const int cb = commit_chunk_bytes(row_bytes, p->num_slots);
  if (cb == 0)
    return jt_fail(JT_ERR_UNSUPPORTED, "kv_commit: %d slots exceed the per-call limit of %d",
                   p->num_slots, jt_kv_commit_max_slots());
  const int chunks = row_bytes / cb;
  const int64_t planes = 2LL * p->num_layers * p->num_kv_heads * chunks;
  if (planes > 0x7fffffff) return jt_fail(JT_ERR_INVALID, "kv_commit: too many planes");
  const int smem = p->num_slots * cb;
  int rc = jt_cuda_check(cudaFuncSetAttribute(kv_commit_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kCommitSmemCap),
                         "kv_commit smem attribute");
  if (rc != JT_OK) return rc;
  kv_commit_kernel<<<static_cast<unsigned>(planes), kCommitThreads, smem, stream>>>(*p, cb,
                                                                                     chunks);
  return jt_cuda_check(cudaGetLastError(), "kv_commit launch");
}
