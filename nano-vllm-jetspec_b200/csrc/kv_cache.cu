// Paged KV writes around tree verification:
//   * jt_kv_store_launch  - warp-per-token indexed store into the paged pool
//     (store_kvcache, nanovllm/layers/attention.py:15-45; tree-node scatter,
//     nanovllm/models/qwen3.py:255-258).
//   * jt_kv_commit_launch - accepted-only commit across K/V and every layer
//     (copy_accepted_kv, nanovllm/speculative/jetspec/state.py:64-86).
// Both are pure byte movers: results are bit-identical to the reference's copies.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

__device__ uint32_t g_kv_errors;

constexpr int kStoreThreads = 256;
constexpr int kCommitThreads = 512;
constexpr int kCommitUnroll = 4;
constexpr int kCommitSmemCap = 192 * 1024;  // bytes of staging per commit CTA
constexpr int kLocalThreads = 512;          // plane-local commit CTAs
constexpr int kLocalUnroll = 4;             // a plane of up to 2048 units in one round
constexpr int kLocalMinPlanes = 32;         // fewer planes: the grid-wide form spreads wider

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

// Accepted-only commit over the whole GPU.  The copy is cut into 16-byte units, one per
// (K/V axis, layer, slot, kv head, 16-byte word of the head row), ordered so that
// neighbouring threads move neighbouring bytes of one slot's rows.  A "plane" is the
// set of units of one (axis, layer, head chunk, word chunk) over EVERY slot: a write to
// a plane can only clobber a source row of the same plane, so the reference's
// gather-before-scatter semantics hold if every unit of a plane is read before any unit
// of that plane is written.  Planes are processed in groups that fit the shared memory of
// the whole grid: each CTA gathers its share of the group's units into shared memory,
// the grid synchronises (cooperative launch: every CTA is resident), and each CTA
// scatters the units it gathered; the next group starts after a second grid barrier.
// The grid spans the GPU whatever the number of layers and heads, so a commit of many
// slots on a single KV head (one GPU of a KV-head-sharded group) is as parallel as one
// over all heads.
struct CommitGeom {
  int heads_per_plane;   // divides num_kv_heads
  int words_per_plane;   // divides the 16-byte words of a head row
  int words_per_row;     // 16-byte words of one head row
  int planes;            // 2 * layers * (heads / heads_per_plane) * (words / words_per_plane)
  int planes_per_group;
  int groups;
  int plane_units;       // num_slots * heads_per_plane * words_per_plane
};

__device__ __forceinline__ char* commit_unit_address(const JtKvCommitParams& p,
                                                     const CommitGeom& g, int plane,
                                                     int rem, const void* slots,
                                                     int64_t pool_slots, bool* ok) {
  const int unit_cols = g.heads_per_plane * g.words_per_plane;
  const int s = rem / unit_cols;
  const int r2 = rem - s * unit_cols;
  const int head_in = r2 / g.words_per_plane;
  const int word_in = r2 - head_in * g.words_per_plane;
  const int word_chunks = g.words_per_row / g.words_per_plane;
  const int head_chunks = p.num_kv_heads / g.heads_per_plane;
  const int wchunk = plane % word_chunks;
  int rest = plane / word_chunks;
  const int hchunk = rest % head_chunks;
  rest /= head_chunks;
  const int layer = rest % p.num_layers;
  const int axis = rest / p.num_layers;
  const int head = hchunk * g.heads_per_plane + head_in;
  const int word = wchunk * g.words_per_plane + word_in;
  const int64_t slot = load_slot(slots, p.slot_is_int64, s);
  *ok = slot >= 0 && slot < pool_slots;
  if (!*ok) return nullptr;
  const int64_t page = slot / p.block_size;
  const int64_t off = slot - page * p.block_size;
  return static_cast<char*>(p.kv_pool) +
         (axis * p.stride_axis + layer * p.stride_layer + page * p.stride_block +
          off * p.stride_offset + static_cast<int64_t>(head) * p.stride_head) *
             p.elem_bytes +
         static_cast<int64_t>(word) * 16;
}

__global__ void __launch_bounds__(kCommitThreads) kv_commit_kernel(JtKvCommitParams p,
                                                                   CommitGeom g) {
  extern __shared__ __align__(16) int4 staging[];
  cg::grid_group grid = cg::this_grid();
  const int64_t pool_slots = p.num_blocks * p.block_size;
  for (int grp = 0; grp < g.groups; ++grp) {
    const int plane0 = grp * g.planes_per_group;
    const int planes_here = min(g.planes_per_group, g.planes - plane0);
    const int64_t units = static_cast<int64_t>(planes_here) * g.plane_units;
    const int64_t per = (units + gridDim.x - 1) / gridDim.x;
    const int64_t u0 = min(units, static_cast<int64_t>(blockIdx.x) * per);
    const int n = static_cast<int>(min(units, u0 + per) - u0);
    // Gather: kCommitUnroll loads in flight per thread before they are staged.
    for (int base = threadIdx.x; base < n; base += kCommitThreads * kCommitUnroll) {
      int4 v[kCommitUnroll];
#pragma unroll
      for (int k = 0; k < kCommitUnroll; ++k) {
        const int i = base + k * kCommitThreads;
        v[k] = make_int4(0, 0, 0, 0);
        if (i < n) {
          const int64_t u = u0 + i;
          const int plane = plane0 + static_cast<int>(u / g.plane_units);
          const int rem = static_cast<int>(u % g.plane_units);
          bool ok = false;
          const char* src =
              commit_unit_address(p, g, plane, rem, p.source_slots, pool_slots, &ok);
          if (ok) v[k] = *reinterpret_cast<const int4*>(src);
          else atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
        }
      }
#pragma unroll
      for (int k = 0; k < kCommitUnroll; ++k) {
        const int i = base + k * kCommitThreads;
        if (i < n) staging[i] = v[k];
      }
    }
    grid.sync();  // every read of this group's planes precedes every write to them
    for (int i = threadIdx.x; i < n; i += kCommitThreads) {
      const int64_t u = u0 + i;
      const int plane = plane0 + static_cast<int>(u / g.plane_units);
      const int rem = static_cast<int>(u % g.plane_units);
      bool src_ok = false, dst_ok = false;
      commit_unit_address(p, g, plane, rem, p.source_slots, pool_slots, &src_ok);
      char* dst = commit_unit_address(p, g, plane, rem, p.destination_slots, pool_slots, &dst_ok);
      if (src_ok && dst_ok) *reinterpret_cast<int4*>(dst) = staging[i];
      else if (!dst_ok) atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
    }
    if (grp + 1 < g.groups) grid.sync();  // this group's writes precede the next reads
  }
}

// Plane-local form: when every plane's units fit one CTA's shared memory and there are
// enough planes to spread over the GPU, each CTA takes whole planes (a grid-stride loop):
// it gathers a plane's units, synchronises its own threads and scatters them.  Planes
// cover disjoint bytes, so no CTA waits for another: an ordinary launch, no grid barrier.
__global__ void __launch_bounds__(kLocalThreads) kv_commit_local_kernel(JtKvCommitParams p,
                                                                        CommitGeom g) {
  extern __shared__ __align__(16) int4 staging[];
  const int64_t pool_slots = p.num_blocks * p.block_size;
  const int n = g.plane_units;
  for (int plane = blockIdx.x; plane < g.planes; plane += gridDim.x) {
    for (int base = threadIdx.x; base < n; base += kLocalThreads * kLocalUnroll) {
      int4 v[kLocalUnroll];
#pragma unroll
      for (int k = 0; k < kLocalUnroll; ++k) {
        const int i = base + k * kLocalThreads;
        v[k] = make_int4(0, 0, 0, 0);
        if (i < n) {
          bool ok = false;
          const char* src = commit_unit_address(p, g, plane, i, p.source_slots, pool_slots, &ok);
          if (ok) v[k] = *reinterpret_cast<const int4*>(src);
          else atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
        }
      }
#pragma unroll
      for (int k = 0; k < kLocalUnroll; ++k) {
        const int i = base + k * kLocalThreads;
        if (i < n) staging[i] = v[k];
      }
    }
    __syncthreads();  // every read of this plane precedes every write to it
    for (int i = threadIdx.x; i < n; i += kLocalThreads) {
      bool src_ok = false, dst_ok = false;
      commit_unit_address(p, g, plane, i, p.source_slots, pool_slots, &src_ok);
      char* dst = commit_unit_address(p, g, plane, i, p.destination_slots, pool_slots, &dst_ok);
      if (src_ok && dst_ok) *reinterpret_cast<int4*>(dst) = staging[i];
      else if (!dst_ok) atomicOr(&g_kv_errors, JT_DEVERR_OUT_OF_RANGE);
    }
    __syncthreads();  // the staging is free for the next plane
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride16(int64_t stride, int eb) { return ((stride * eb) & 15) == 0; }

// SM count of the current device (0 when there is none).
int commit_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

// Units one launch can stage at once: one CTA per SM, kCommitSmemCap bytes each.
int64_t commit_capacity_units(int sms) {
  return static_cast<int64_t>(std::max(sms, 1)) * (kCommitSmemCap / 16);
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

extern "C" int32_t jt_kv_commit_max_slots(void) {
  // One plane of one head-row word per slot must fit the grid's staging.
  const int64_t cap = commit_capacity_units(commit_sms());
  return static_cast<int32_t>(std::min<int64_t>(cap, 0x7fffffff));
}

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
  const int sms = commit_sms();
  if (sms <= 0) return jt_fail(JT_ERR_CUDA, "kv_commit: no CUDA device");
  const int64_t capacity = commit_capacity_units(sms);
  const int words = row_bytes / 16;
  const int64_t n = p->num_slots;
  // Plane-local form: planes of one head and one 32-byte sector of its row while a plane
  // stays within one round of loads (n <= 1024), else of one 16-byte word (half the
  // rounds), each gathered and scattered by one CTA; one word when the sector planes are
  // too few or do not fit.
  for (int wp : {2, 1}) {
    if (words % wp != 0 || (wp == 2 && n * 2 > kLocalThreads * kLocalUnroll)) continue;
    const int64_t planes = 2LL * p->num_layers * p->num_kv_heads * (words / wp);
    const int64_t staging = n * wp * 16;
    if (planes < kLocalMinPlanes || planes > 0x7fffffff || staging > kCommitSmemCap) continue;
    CommitGeom g{};
    g.heads_per_plane = 1;
    g.words_per_plane = wp;
    g.words_per_row = words;
    g.planes = static_cast<int>(planes);
    g.plane_units = static_cast<int>(n * wp);
    g.planes_per_group = g.planes;
    g.groups = 1;
    const int smem = static_cast<int>(staging);
    int rc = jt_cuda_check(cudaFuncSetAttribute(kv_commit_local_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kCommitSmemCap),
                           "kv_commit smem attribute");
    if (rc != JT_OK) return rc;
    const int grid = static_cast<int>(std::min<int64_t>(planes, 8LL * sms));
    kv_commit_local_kernel<<<grid, kLocalThreads, smem, stream>>>(*p, g);
    return jt_cuda_check(cudaGetLastError(), "kv_commit launch");
  }
  // Grid-wide form: the largest planes that fit the grid's staging (all heads and words
  // of a slot, else one head's row, else one 16-byte word of it).
  CommitGeom g{};
  if (n * p->num_kv_heads * words <= capacity) {
    g.heads_per_plane = p->num_kv_heads;
    g.words_per_plane = words;
  } else if (n * words <= capacity) {
    g.heads_per_plane = 1;
    g.words_per_plane = words;
  } else if (n <= capacity) {
    g.heads_per_plane = 1;
    g.words_per_plane = 1;
  } else {
    return jt_fail(JT_ERR_UNSUPPORTED, "kv_commit: %d slots exceed the per-call limit of %d",
                   p->num_slots, jt_kv_commit_max_slots());
  }
  g.words_per_row = words;
  const int64_t planes = 2LL * p->num_layers * (p->num_kv_heads / g.heads_per_plane) *
                         (words / g.words_per_plane);
  if (planes > 0x7fffffff) return jt_fail(JT_ERR_INVALID, "kv_commit: too many planes");
  g.planes = static_cast<int>(planes);
  g.plane_units = static_cast<int>(n * g.heads_per_plane * g.words_per_plane);
  g.planes_per_group = static_cast<int>(std::min<int64_t>(planes, capacity / g.plane_units));
  g.groups = (g.planes + g.planes_per_group - 1) / g.planes_per_group;
  const int64_t group_units = static_cast<int64_t>(g.planes_per_group) * g.plane_units;
  // Enough CTAs for about kCommitThreads * kCommitUnroll units each, at most one per SM
  // (every CTA must be resident for the grid barrier).
  const int64_t want = (group_units + kCommitThreads * kCommitUnroll - 1) /
                       (kCommitThreads * kCommitUnroll);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sms, want)));
  const int64_t per_cta = (group_units + grid - 1) / grid;
  const int smem = static_cast<int>(per_cta * 16);
  if (smem > kCommitSmemCap)
    return jt_fail(JT_ERR_UNSUPPORTED, "kv_commit: staging of %d bytes per CTA", smem);
  int rc = jt_cuda_check(cudaFuncSetAttribute(kv_commit_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kCommitSmemCap),
                         "kv_commit smem attribute");
  if (rc != JT_OK) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kCommitThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return jt_cuda_check(cudaLaunchKernelEx(&cfg, kv_commit_kernel, *p, g), "kv_commit launch");
}
