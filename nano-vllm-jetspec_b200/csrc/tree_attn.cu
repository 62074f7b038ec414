// Packed ragged GQA tree-verification attention over a paged KV cache (sm_100a).
//
// Replaces the Triton kernel _packed_tree_gqa_dot and its launcher
// (nanovllm/speculative/jetspec/tree_gqa.py:32-140).  Same semantics: for every packed
// tree node, each of the `groups` query heads of one KV head attends to the request's
// prefix (through its block table) plus the tree nodes its ancestor bias admits;
// scores and softmax in fp32, probabilities rounded to the operand type for PV.
//
// Structure (two launches on the caller's stream, both graph-capturable):
//   1. plan kernel   - block 0 builds the work list from the DEVICE prefix lengths and
//                      node counts (split-KV plan, longest-first order, partial-slot
//                      offsets); the other blocks turn qq_bias rows into ancestor
//                      bitmasks (one warp per tree node, one ballot per 32 nodes).
//   2. attention     - persistent CTAs pull work items (request, split, kv head,
//                      m-block) from an atomic queue.  One item = BM score rows
//                      (BM/groups tree nodes x groups query heads of one KV head)
//                      against a contiguous key range, streamed in 64-key tiles
//                      through a 3-stage cp.async ring with 16-byte loads.  QK^T and
//                      PV run on tensor cores (m16n8k16, fp32 accumulate); online
//                      softmax in fp32 registers.  Items of split requests write
//                      unnormalised partials; the last CTA of a (request, head,
//                      m-block) merges them (counter in the workspace).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace {

__device__ uint32_t g_attn_errors;

constexpr int kTileKeys = 64;     // keys per KV tile
constexpr int kStages = 3;        // cp.async ring depth
constexpr int kMaxMaskWords = 32; // tree nodes per request <= 1024
constexpr int kPlanThreads = 256;
constexpr int kBuckets = 256;  // item-order buckets: 8 per octave of key counts
static_assert(kBuckets == kPlanThreads, "one bucket per plan thread in the bucket scan");
constexpr int kSplitCandidates = 16;  // split lengths 1024 << c
constexpr int kSplitBase = 1024;
// Planning costs in 128-key tile times, measured: the fixed cost of one work item (query
// tile load, pipeline fill, epilogue) and the extra cost of a split plan (fp32 partials,
// the release fence and counter of every split item, the merging loads).
#ifndef JT_ITEM_COST_TILES
#define JT_ITEM_COST_TILES 2
#endif
constexpr int kItemCostTiles = JT_ITEM_COST_TILES;
#ifndef JT_MERGE_COST_TILES
#define JT_MERGE_COST_TILES 16
#endif
constexpr int kMergeCostTiles = JT_MERGE_COST_TILES;
// Longest prefix (block-table capacity) for which a one-item-per-CTA launch without a plan
// beats a split plan (the plan's estimate gives splits no gain below about 32 tiles).
constexpr int64_t kSingleLaunchMaxKeys = 4096;
constexpr int64_t kPartialBudgetBytes = 256ll << 20;

// ---- workspace layout ---------------------------------------------------------------
struct Layout {
  int bm;           // score rows per item (64 or 128)
  int counter_stride;  // split counters per (request, kv head, m-block): 1, or 2 per row
  int mask_words;   // 32-bit words of ancestor bitmask per tree node
  int max_items;
  int max_slots;    // partial-result slots (split items)
  size_t off_header, off_req, off_items, off_counters, off_masks, off_part_o, off_part_ml;
  size_t total;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int choose_bm(int32_t num_requests, int32_t total_queries, int32_t groups) {
  // 128-row items (8 warps) once the average request carries >= 128 score rows per KV
  // head; otherwise 64-row items (4 warps).  Depends only on the launch shape.
  return static_cast<int64_t>(total_queries) * groups >= 128ll * num_requests ? 128 : 64;
}

Layout make_layout(int32_t R, int32_t Q, int32_t H, int32_t G, int32_t D,
                   int64_t partial_budget = kPartialBudgetBytes, int bm = 0,
                   bool row_counters = false) {
  Layout L{};
  L.bm = bm > 0 ? bm : choose_bm(R, Q, G);
  L.mask_words = static_cast<int>(std::min<int64_t>((std::max<int32_t>(Q, 1) + 31) / 32,
                                                    kMaxMaskWords));
  const int64_t mblocks_bound = (static_cast<int64_t>(Q) * G) / L.bm + R;
  const int64_t per_slot = static_cast<int64_t>(L.bm) * D * 4;
  int64_t slots = std::min<int64_t>(4 * mblocks_bound * H, partial_budget / per_slot);
  slots = std::max<int64_t>(slots, 1);
  L.max_slots = static_cast<int>(slots);
  L.max_items = static_cast<int>(mblocks_bound * H + slots);
  size_t o = 0;
  L.off_header = o;   o = align_up(o + 64, 256);
  L.off_req = o;      o = align_up(o + sizeof(int4) * static_cast<size_t>(R), 256);
  L.off_items = o;    o = align_up(o + sizeof(int4) * static_cast<size_t>(L.max_items), 256);
  // Split counters: one per (request, kv head, m-block) for the portable core, one per
  // score row and output half for the tcgen05 core (whose rows and halves finish
  // independently).
  const size_t counter_stride = row_counters ? 2 * static_cast<size_t>(L.bm) : 1;
  L.counter_stride = static_cast<int>(counter_stride);
  L.off_counters = o;
  o = align_up(o + sizeof(int) * static_cast<size_t>(L.max_slots) * counter_stride, 256);
  L.off_masks = o;
  o = align_up(o + sizeof(uint32_t) * static_cast<size_t>(Q) * L.mask_words, 256);
  L.off_part_o = o;   o = align_up(o + static_cast<size_t>(per_slot) * L.max_slots, 256);
  L.off_part_ml = o;  // (max, sum) per row; per row and output half for the tcgen05 core
  o = align_up(o + sizeof(float2) * static_cast<size_t>(L.bm) * L.max_slots * (row_counters ? 2 : 1),
               256);
  L.total = o;
  return L;
}

struct DevLayout {
  int* header;      // [0] queue head, [1] item count, [2] split keys
  int4* req;        // per request: n_split, partial base, counter base, m-blocks
  int4* items;      // request, split, kv head, m-block
  int* counters;
  uint32_t* masks;
  float* part_o;
  float2* part_ml;
  int bm, mask_words, max_items, max_slots;
  int counter_stride;  // split counters per (request, kv head, m-block): 1, or 2 per row
};

DevLayout device_layout(const Layout& L, void* ws) {
  char* b = static_cast<char*>(ws);
  DevLayout d;
  d.header = reinterpret_cast<int*>(b + L.off_header);
  d.req = reinterpret_cast<int4*>(b + L.off_req);
  d.items = reinterpret_cast<int4*>(b + L.off_items);
  d.counters = reinterpret_cast<int*>(b + L.off_counters);
  d.masks = reinterpret_cast<uint32_t*>(b + L.off_masks);
  d.part_o = reinterpret_cast<float*>(b + L.off_part_o);
  d.part_ml = reinterpret_cast<float2*>(b + L.off_part_ml);
  d.bm = L.bm;
  d.mask_words = L.mask_words;
  d.max_items = L.max_items;
  d.max_slots = L.max_slots;
  d.counter_stride = L.counter_stride;
  return d;
}

// ---- plan kernel --------------------------------------------------------------------
__device__ __forceinline__ int request_mblocks(int nodes, int groups, int bm) {
  return static_cast<int>((static_cast<int64_t>(nodes) * groups + bm - 1) / bm);
}

// Bucket of an item with `keys` keys in the longest-first order: the octave
// floor(log2(keys)) and the next three bits below it (exact below 8 keys), so items within
// 12.5 % of each other share a bucket.
__device__ __forceinline__ int key_bucket(int keys) {
  keys = max(keys, 1);
  const int e = 31 - __clz(keys);
  return e < 3 ? e * 8 : e * 8 + ((keys >> (e - 3)) & 7);
}

__device__ __forceinline__ int request_splits(int prefix, int split_keys) {
  return prefix > split_keys ? (prefix + split_keys - 1) / split_keys : 1;
}

__global__ void __launch_bounds__(kPlanThreads)
    tree_plan_kernel(JtTreeAttnParams p, DevLayout w, int num_ctas) {
  // The tcgen05 attention kernel is launched as a programmatic dependent: it may start its
  // prologue now and waits (griddepcontrol.wait) for this grid's completion before it reads
  // the plan.
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int tid = threadIdx.x;
  if (blockIdx.x > 0) {
    // Ancestor bitmask of one packed tree node per warp.
    const int q = (blockIdx.x - 1) * (kPlanThreads / 32) + (tid >> 5);
    const int lane = tid & 31;
    if (q >= p.total_queries) return;
    const int r = p.query_to_request[q];
    const int j = p.query_local_row[q];
    const int nodes = p.node_counts[r];
    if (nodes > w.mask_words * 32) {
      if (lane == 0) atomicOr(&g_attn_errors, JT_DEVERR_TREE_TOO_LARGE);
      return;
    }
    const float* bias = p.qq_bias + p.qq_bias_offsets[r] + static_cast<int64_t>(j) * nodes;
    // Only the words that hold this tree's nodes: the attention kernels never read a word
    // at or past ceil(nodes / 32) (a key past the request's last node is out of range).
    const int words = (nodes + 31) / 32;
    for (int word = 0; word < words; ++word) {
      const int n = word * 32 + lane;
      const bool visible = n < nodes && n <= j && bias[n] == 0.0f;
      const uint32_t bits = __ballot_sync(0xffffffffu, visible);
      if (lane == 0) w.masks[static_cast<int64_t>(q) * w.mask_words + word] = bits;
    }
    return;
  }

  __shared__ int cand_red[kPlanThreads / 32][4][kSplitCandidates];
  __shared__ int64_t cand_est[kSplitCandidates];
  __shared__ int cand_ok[kSplitCandidates];
  __shared__ int bucket_count[kBuckets];
  __shared__ int bucket_start[kBuckets];
  __shared__ int s_split;
  __shared__ int s_carry[2];
  __shared__ int warp_tot[2][kPlanThreads / 32];

  const int R = p.num_requests, G = p.groups, H = p.num_kv_heads, bm = w.bm;
  const int cap = w.mask_words * 32;
  const int warp = tid >> 5, lane = tid & 31;

  // Per candidate split length S = 1024 << c: the partial slots it needs, the total work
  // in tile times (tiles of every item plus a fixed cost per item) and the longest item.
  // Candidates are visited one at a time (few registers); each thread's first request is
  // kept in registers across them.
  const int r0 = tid;
  const int nodes0 = r0 < R ? p.node_counts[r0] : 0;
  const int prefix0 = r0 < R ? p.prefix_lens[r0] : 0;
#pragma unroll 1
  for (int c = 0; c < kSplitCandidates; ++c) {
    const int len = kSplitBase << c;
    // Reduced in 32 bits: each thread's terms are clamped to 2^24, so a warp's sum stays
    // below 2^29 and a clamped slot count still exceeds any partial budget.
    unsigned c_slots = 0, c_work = 0, c_long = 0, c_full = 0;
    for (int r = tid; r < R; r += kPlanThreads) {
      const int nodes = r == r0 ? nodes0 : p.node_counts[r];
      const int prefix = r == r0 ? prefix0 : p.prefix_lens[r];
      if (nodes < 1 || nodes > cap || prefix < 0) continue;
      const int mb = request_mblocks(nodes, G, bm);
      const int ns = request_splits(prefix, len);
      const int last_keys = prefix + nodes - (ns - 1) * len;
      const int tiles = (ns - 1) * (len / 128) + (last_keys + 127) / 128;
      const int64_t work = static_cast<int64_t>(mb) * H * (tiles + ns * kItemCostTiles);
      c_work = static_cast<unsigned>(min(static_cast<int64_t>(c_work) + work, static_cast<int64_t>(1) << 24));
      c_long = max(c_long, static_cast<unsigned>(max(ns > 1 ? len / 128 : 0, (last_keys + 127) / 128)));
      if (ns > 1) {
        c_slots = static_cast<unsigned>(
            min(static_cast<int64_t>(c_slots) + static_cast<int64_t>(ns) * mb * H,
                static_cast<int64_t>(1) << 24));
        c_full = static_cast<unsigned>(
            min(static_cast<int64_t>(c_full) + static_cast<int64_t>(ns - 1) * mb * H,
                static_cast<int64_t>(1) << 24));
      }
    }
    c_slots = __reduce_add_sync(0xffffffffu, min(c_slots, 1u << 24));
    c_work = min(c_work, 1u << 24);
    c_work = __reduce_add_sync(0xffffffffu, c_work);
    c_long = __reduce_max_sync(0xffffffffu, c_long);
    c_full = __reduce_add_sync(0xffffffffu, min(c_full, 1u << 24));
    if (lane == 0) {
      cand_red[warp][0][c] = static_cast<int>(c_slots);
      cand_red[warp][1][c] = static_cast<int>(c_work);
      cand_red[warp][2][c] = static_cast<int>(c_long);
      cand_red[warp][3][c] = static_cast<int>(c_full);
    }
  }
  if (tid < kBuckets) bucket_count[tid] = 0;
  __syncthreads();
  if (tid < kSplitCandidates) {
    // Candidate `tid`: partial slots, and the estimated makespan in tile times: longest-
    // first list scheduling finishes within max(average load, longest item), and no
    // sooner than the waves its full-length split items take on their own (items of one
    // length fill the CTAs wave by wave); plus the fixed cost of a split plan.
    int64_t sl = 0, wk = 0, lg = 0, fl = 0;
#pragma unroll
    for (int k = 0; k < kPlanThreads / 32; ++k) {
      sl += cand_red[k][0][tid];
      wk += cand_red[k][1][tid];
      lg = max(lg, static_cast<int64_t>(cand_red[k][2][tid]));
      fl += cand_red[k][3][tid];
    }
    const int64_t full_len = (kSplitBase << tid) / 128 + kItemCostTiles;
    cand_ok[tid] = sl <= w.max_slots;
    cand_est[tid] = max(max((wk + num_ctas - 1) / num_ctas, lg + kItemCostTiles),
                        (fl + num_ctas - 1) / num_ctas * full_len) +
                    (sl > 0 ? kMergeCostTiles : 0);
  }
  __syncthreads();
  if (tid == 0) {
    // Explicit split (1024 times a power of two): the first candidate at least that long
    // whose partials fit the budget.  Automatic: the smallest estimate within the budget;
    // ties go to the longer split.  The last candidate (longer than any prefix: no split)
    // always fits.  Shorter splits need more partials, so the scan stops at the first
    // candidate over budget.
    int split = kSplitBase << (kSplitCandidates - 1);
    int64_t best_est = -1;
    for (int c = kSplitCandidates - 1; c >= 0 && cand_ok[c]; --c) {
      const int len = kSplitBase << c;
      if (p.split_keys > 0) {
        if (len >= p.split_keys) split = len;
      } else if (best_est < 0 || cand_est[c] < best_est) {
        best_est = cand_est[c];
        split = len;
      }
    }
    s_split = split;
    s_carry[0] = s_carry[1] = 0;
  }
  __syncthreads();
  const int split = s_split;

  // Per-request split count plus exclusive scans of partial slots and counters.
  for (int base = 0; base < R; base += kPlanThreads) {
    const int r = base + tid;
    int n_split = 1, mb = 0, slots = 0, counters = 0;
    if (r < R) {
      const int nodes = p.node_counts[r];
      const int prefix = p.prefix_lens[r];
      if (nodes >= 1 && nodes <= cap && prefix >= 0) {
        mb = request_mblocks(nodes, G, bm);
        n_split = request_splits(prefix, split);
        if (n_split > 1) {
          slots = n_split * mb * H;
          counters = mb * H;
        }
      } else {
        n_split = 0;  // skipped request (flagged by the mask blocks)
      }
    }
    int a = slots, b = counters;
    for (int o = 1; o < 32; o <<= 1) {
      const int ya = __shfl_up_sync(0xffffffffu, a, o);
      const int yb = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) { a += ya; b += yb; }
    }
    if (lane == 31) { warp_tot[0][warp] = a; warp_tot[1][warp] = b; }
    __syncthreads();
    int pa = s_carry[0], pb = s_carry[1];
    for (int k = 0; k < warp; ++k) { pa += warp_tot[0][k]; pb += warp_tot[1][k]; }
    if (r < R) w.req[r] = make_int4(n_split, pa + a - slots, pb + b - counters, mb);
    __syncthreads();
    if (tid == kPlanThreads - 1) { s_carry[0] = pa + a; s_carry[1] = pb + b; }
    __syncthreads();
  }
  // Reset split counters for this launch.
  for (int64_t i = tid; i < static_cast<int64_t>(s_carry[1]) * w.counter_stride; i += kPlanThreads)
    w.counters[i] = 0;

  // Longest-first item order: bucket units (request, split) by key_bucket(keys).
  for (int r = tid; r < R; r += kPlanThreads) {
    const int4 info = w.req[r];
    if (info.x == 0) continue;
    const int prefix = p.prefix_lens[r], nodes = p.node_counts[r];
    for (int s = 0; s < info.x; ++s) {
      const int keys = (s + 1 < info.x) ? split : prefix + nodes - s * split;
      atomicAdd(&bucket_count[key_bucket(keys)], info.w * H);
    }
  }
  __syncthreads();
  {
    // Bucket starts in descending bucket order: an exclusive scan with thread t on
    // bucket kBuckets-1-t (warp shuffles, then the warp totals).
    const int b = kBuckets - 1 - tid;
    const int cnt = bucket_count[b];
    int x = cnt;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[0][warp] = x;
    __syncthreads();
    int base = 0;
    for (int k = 0; k < warp; ++k) base += warp_tot[0][k];
    bucket_start[b] = base + x - cnt;
    if (tid == kPlanThreads - 1) {
      const int run = base + x;
      w.header[1] = run <= w.max_items ? run : 0;
      if (run > w.max_items) atomicOr(&g_attn_errors, JT_DEVERR_OUT_OF_RANGE);
      w.header[0] = 0;
      w.header[2] = split;
    }
  }
  __syncthreads();
  for (int r = tid; r < R; r += kPlanThreads) {
    const int4 info = w.req[r];
    if (info.x == 0) continue;
    const int prefix = p.prefix_lens[r], nodes = p.node_counts[r];
    for (int s = 0; s < info.x; ++s) {
      const int keys = (s + 1 < info.x) ? split : prefix + nodes - s * split;
      const int pos = atomicAdd(&bucket_start[key_bucket(keys)], info.w * H);
      if (pos + info.w * H > w.max_items) continue;
      for (int h = 0; h < H; ++h)
        for (int m = 0; m < info.w; ++m) w.items[pos + h * info.w + m] = make_int4(r, s, h, m);
    }
  }
}

// ---- attention kernel ---------------------------------------------------------------
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  // 16-byte chunk XOR swizzle: conflict-free cp.async writes and ldmatrix reads.
  return static_cast<uint32_t>(row * (D * 2) + ((chunk ^ (row & 7)) << 4));
}

template <typename Elem, int WARPS, int D, bool FP32P>
struct AttnKernel {
  static constexpr int kThreads = WARPS * 32;
  static constexpr int kBM = WARPS * 16;
  static constexpr int kRowBytes = D * 2;
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  static constexpr int kQBytes = kBM * kRowBytes;
  static constexpr int kTileBytes = kTileKeys * kRowBytes;
  static constexpr int kSmem = kQBytes + 2 * kStages * kTileBytes;
  static constexpr int kNT = kTileKeys / 8;  // score n-tiles per warp
  static constexpr int kDT = D / 8;          // output n-tiles per warp
  static constexpr int kKS = D / 16;         // k-steps over head_dim
};

template <typename Elem, int WARPS, int D, bool FP32P>
__global__ void __launch_bounds__(WARPS * 32)
    tree_attn_kernel(JtTreeAttnParams p, DevLayout w) {
  using K = AttnKernel<Elem, WARPS, D, FP32P>;
  using Mma = jt::MmaOp<Elem>;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_item;
  __shared__ int s_last;
  const uint32_t sbase = jt::smem_u32(smem);
  const uint32_t sq = sbase;
  const uint32_t sk = sbase + K::kQBytes;
  const uint32_t sv = sk + kStages * K::kTileBytes;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, t4 = lane & 3;
  const int G = p.groups, H = p.num_kv_heads, bs = p.block_size;
  const int num_items = w.header[1];
  const int split_keys = w.header[2];
  const float scale_log2 = p.scale * 1.4426950408889634f;
  const int64_t pool_slots = p.num_blocks * static_cast<int64_t>(bs);
  const char* kbase = static_cast<const char*>(p.k_pool);
  const char* vbase = static_cast<const char*>(p.v_pool);

  for (;;) {
    if (tid == 0) s_item = atomicAdd(&w.header[0], 1);
    __syncthreads();
    const int item = s_item;
    if (item >= num_items) break;
    const int4 it = w.items[item];
    const int r = it.x, split = it.y, h = it.z, mb = it.w;
    const int4 info = w.req[r];
    const int n_split = info.x, mblocks = info.w;
    const int P = p.prefix_lens[r];
    const int T = p.node_counts[r];
    const int q_start = p.cu_seqlens_q[r];
    const int row0 = mb * K::kBM;
    const int key_begin = split * split_keys;
    int key_end;
    if (split + 1 < n_split) {
      key_end = key_begin + split_keys;
    } else {
      // Tree nodes after the last one any row of this block can see are pruned.
      const int vis_nodes = min(T, (row0 + K::kBM + G - 1) / G);
      key_end = P + vis_nodes;
    }
    const int n_tiles = (key_end - key_begin + kTileKeys - 1) / kTileKeys;
    const int32_t* table = p.block_tables + static_cast<int64_t>(r) * p.table_stride0;

    // --- async loads ------------------------------------------------------------------
    auto load_q = [&]() {
      for (int c = tid; c < K::kBM * K::kChunks; c += K::kThreads) {
        const int row = c / K::kChunks, ch = c - row * K::kChunks;
        const int gm = row0 + row;
        const int j = gm / G, g = gm - j * G;
        const bool ok = j < T;
        const char* src = static_cast<const char*>(p.q);
        if (ok)
          src += ((static_cast<int64_t>(q_start + j) * p.q_stride0) +
                  static_cast<int64_t>(h * G + g) * p.q_stride1 + ch * 8) * 2;
        jt::cp_async_16(sq + swz<D>(row, ch), src, ok ? 16 : 0);
      }
    };
    auto load_kv = [&](int tile, int stage) {
      const int kb = key_begin + tile * kTileKeys;
      for (int c = tid; c < kTileKeys * K::kChunks; c += K::kThreads) {
        const int row = c / K::kChunks, ch = c - row * K::kChunks;
        const int pos = kb + row;
        int64_t page = 0, off = 0;
        bool ok = pos < key_end;
        if (ok) {
          int64_t slot = -1;
          if (pos < P) {
            const int col = pos / bs;
            if (col < p.table_width) slot = static_cast<int64_t>(__ldg(table + col)) * bs + pos % bs;
          } else {
            slot = __ldg(p.tree_slots + q_start + (pos - P));
          }
          if (slot < 0 || slot >= pool_slots) {
            ok = false;
            if (ch == 0) atomicOr(&g_attn_errors, JT_DEVERR_OUT_OF_RANGE);
          } else {
            page = slot / bs;
            off = slot - page * bs;
          }
        }
        const char* ks = kbase;
        const char* vs = vbase;
        if (ok) {
          ks += (page * p.k_stride0 + off * p.k_stride1 + static_cast<int64_t>(h) * p.k_stride2 +
                 ch * 8) * 2;
          vs += (page * p.v_stride0 + off * p.v_stride1 + static_cast<int64_t>(h) * p.v_stride2 +
                 ch * 8) * 2;
        }
        const uint32_t o = static_cast<uint32_t>(stage * K::kTileBytes) + swz<D>(row, ch);
        jt::cp_async_16(sk + o, ks, ok ? 16 : 0);
        jt::cp_async_16(sv + o, vs, ok ? 16 : 0);
      }
    };

    load_q();
#pragma unroll
    for (int st = 0; st < kStages - 1; ++st) {
      if (st < n_tiles) load_kv(st, st);
      jt::cp_async_commit();
    }

    // Per-thread score rows: g4 and g4 + 8 of this warp's 16.
    int row_j[2];
    bool row_ok[2];
    const uint32_t* row_mask[2];
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      const int gm = row0 + warp * 16 + g4 + hrow * 8;
      row_j[hrow] = gm / G;
      row_ok[hrow] = row_j[hrow] < T;
      row_mask[hrow] = w.masks + static_cast<int64_t>(q_start + (row_ok[hrow] ? row_j[hrow] : 0)) *
                                    w.mask_words;
    }

    uint32_t qf[K::kKS][4];
    float o_acc[K::kDT][4];
#pragma unroll
    for (int i = 0; i < K::kDT; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};

    for (int tile = 0; tile < n_tiles; ++tile) {
      jt::cp_async_wait<kStages - 2>();
      __syncthreads();
      if (tile == 0) {
#pragma unroll
        for (int ks = 0; ks < K::kKS; ++ks) {
          const int row = warp * 16 + (lane & 15);
          const int ch = ks * 2 + (lane >> 4);
          jt::ldmatrix_x4(qf[ks], sq + swz<D>(row, ch));
        }
      }
      {
        const int nxt = tile + kStages - 1;
        if (nxt < n_tiles) load_kv(nxt, nxt % kStages);
        jt::cp_async_commit();
      }
      const int stage = tile % kStages;
      const uint32_t ks_base = sk + stage * K::kTileBytes;
      const uint32_t vs_base = sv + stage * K::kTileBytes;

      // S = Q K^T for this warp's 16 rows x 64 keys.
      float s[K::kNT][4];
#pragma unroll
      for (int i = 0; i < K::kNT; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < K::kKS; ++ks) {
#pragma unroll
        for (int np = 0; np < K::kNT / 2; ++np) {
          uint32_t b[4];
          const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int ch = ks * 2 + ((lane >> 3) & 1);
          jt::ldmatrix_x4(b, ks_base + swz<D>(key, ch));
          Mma::run(s[2 * np], qf[ks], b[0], b[1]);
          Mma::run(s[2 * np + 1], qf[ks], b[2], b[3]);
        }
      }

      // Scale into the log2 domain and mask.
      const int kb = key_begin + tile * kTileKeys;
      const bool full = kb + kTileKeys <= min(P, key_end);
#pragma unroll
      for (int nt = 0; nt < K::kNT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = s[nt][e] * scale_log2;
          if (!full) {
            const int hrow = e >> 1;
            const int pos = kb + nt * 8 + t4 * 2 + (e & 1);
            bool vis = row_ok[hrow] && pos < key_end;
            if (vis && pos >= P) {
              const int n = pos - P;
              vis = (__ldg(row_mask[hrow] + (n >> 5)) >> (n & 31)) & 1u;
            }
            if (!vis) v = -INFINITY;
          }
          s[nt][e] = v;
        }
      }

      // Online softmax (row max over the quad, guarded exponent base).
      float alpha[2], m_use[2];
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < K::kNT; ++nt)
          mx = fmaxf(mx, fmaxf(s[nt][2 * hrow], s[nt][2 * hrow + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[hrow], mx);
        m_use[hrow] = m_new == -INFINITY ? 0.f : m_new;
        alpha[hrow] = jt::fast_exp2(m_run[hrow] - m_use[hrow]);
        m_run[hrow] = m_new;
      }
      float rsum[2] = {0.f, 0.f};
      uint32_t pa[K::kNT / 2][4];
      uint32_t pl[FP32P ? K::kNT / 2 : 1][4];
#pragma unroll
      for (int nt = 0; nt < K::kNT; ++nt) {
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          pr[e] = jt::fast_exp2(s[nt][e] - m_use[e >> 1]);
          rsum[e >> 1] += pr[e];
        }
        const int kk = nt >> 1, hi = (nt & 1) * 2;
        pa[kk][hi + 0] = Mma::pack(pr[0], pr[1]);
        pa[kk][hi + 1] = Mma::pack(pr[2], pr[3]);
        if constexpr (FP32P) {
          const float2 r01 = Mma::unpack(pa[kk][hi + 0]);
          const float2 r23 = Mma::unpack(pa[kk][hi + 1]);
          pl[kk][hi + 0] = Mma::pack(pr[0] - r01.x, pr[1] - r01.y);
          pl[kk][hi + 1] = Mma::pack(pr[2] - r23.x, pr[3] - r23.y);
        }
      }
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) l_run[hrow] = l_run[hrow] * alpha[hrow] + rsum[hrow];
#pragma unroll
      for (int dt = 0; dt < K::kDT; ++dt) {
        o_acc[dt][0] *= alpha[0];
        o_acc[dt][1] *= alpha[0];
        o_acc[dt][2] *= alpha[1];
        o_acc[dt][3] *= alpha[1];
      }

      // O += P V.
#pragma unroll
      for (int kk = 0; kk < K::kNT / 2; ++kk) {
#pragma unroll
        for (int dp = 0; dp < K::kDT / 2; ++dp) {
          uint32_t b[4];
          const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int ch = dp * 2 + (lane >> 4);
          jt::ldmatrix_x4_trans(b, vs_base + swz<D>(key, ch));
          Mma::run(o_acc[2 * dp], pa[kk], b[0], b[1]);
          Mma::run(o_acc[2 * dp + 1], pa[kk], b[2], b[3]);
          if constexpr (FP32P) {
            Mma::run(o_acc[2 * dp], pl[kk], b[0], b[1]);
            Mma::run(o_acc[2 * dp + 1], pl[kk], b[2], b[3]);
          }
        }
      }
    }
    jt::cp_async_wait<0>();

    // Row sums across the quad.
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      l_run[hrow] += __shfl_xor_sync(0xffffffffu, l_run[hrow], 1);
      l_run[hrow] += __shfl_xor_sync(0xffffffffu, l_run[hrow], 2);
    }

    auto store_row = [&](int gm, int d, float x0, float x1) {
      const int j = gm / G, g = gm - j * G;
      if (j >= T) return;
      const int64_t off = static_cast<int64_t>(q_start + j) * p.out_stride0 +
                          static_cast<int64_t>(h * G + g) * p.out_stride1 + d;
      if (p.out_dtype == JT_F32) {
        *reinterpret_cast<float2*>(static_cast<float*>(p.out) + off) = make_float2(x0, x1);
      } else {
        *reinterpret_cast<uint32_t*>(static_cast<Elem*>(p.out) + off) = Mma::pack(x0, x1);
      }
    };

    if (n_split == 1) {
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const float inv = 1.f / l_run[hrow];
        const int gm = row0 + warp * 16 + g4 + hrow * 8;
#pragma unroll
        for (int dt = 0; dt < K::kDT; ++dt)
          store_row(gm, dt * 8 + t4 * 2, o_acc[dt][2 * hrow] * inv,
                    o_acc[dt][2 * hrow + 1] * inv);
      }
    } else {
      // Unnormalised partial + (max, sum); the last CTA of this group merges.
      const int64_t slot = info.y + (static_cast<int64_t>(h) * mblocks + mb) * n_split + split;
      float* po = w.part_o + slot * K::kBM * D;
      float2* pml = w.part_ml + slot * K::kBM;
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const int row = warp * 16 + g4 + hrow * 8;
#pragma unroll
        for (int dt = 0; dt < K::kDT; ++dt)
          *reinterpret_cast<float2*>(po + row * D + dt * 8 + t4 * 2) =
              make_float2(o_acc[dt][2 * hrow], o_acc[dt][2 * hrow + 1]);
        if (t4 == 0) pml[row] = make_float2(m_run[hrow], l_run[hrow]);
      }
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        int* counter = w.counters + info.z + h * mblocks + mb;
        const int done = atomicAdd(counter, 1);
        s_last = done == n_split - 1;
        if (s_last) *counter = 0;
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        const int64_t slot0 = info.y + (static_cast<int64_t>(h) * mblocks + mb) * n_split;
        for (int idx = tid; idx < K::kBM * (D / 4); idx += K::kThreads) {
          const int row = idx / (D / 4), d4 = (idx - row * (D / 4)) * 4;
          if ((row0 + row) / G >= T) continue;
          float mmax = -INFINITY;
          for (int s2 = 0; s2 < n_split; ++s2)
            mmax = fmaxf(mmax, __ldcg(w.part_ml + (slot0 + s2) * K::kBM + row).x);
          const float mref = mmax == -INFINITY ? 0.f : mmax;
          float den = 0.f;
          float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int s2 = 0; s2 < n_split; ++s2) {
            const float2 ml = __ldcg(w.part_ml + (slot0 + s2) * K::kBM + row);
            const float wgt = jt::fast_exp2(ml.x - mref);
            const float4 o = __ldcg(reinterpret_cast<const float4*>(
                w.part_o + ((slot0 + s2) * K::kBM + row) * D + d4));
            den += wgt * ml.y;
            num.x += wgt * o.x;
            num.y += wgt * o.y;
            num.z += wgt * o.z;
            num.w += wgt * o.w;
          }
          const float inv = 1.f / den;
          store_row(row0 + row, d4, num.x * inv, num.y * inv);
          store_row(row0 + row, d4 + 2, num.z * inv, num.w * inv);
        }
      }
    }
    __syncthreads();
  }
}

#include "attn_tcgen05.cuh"

// ---- host side ----------------------------------------------------------------------
struct DeviceInfo {
  int sms = 0;
};
DeviceInfo g_devices[64];

int device_sms(int* sms) {
  int dev = 0;
  int rc = jt_cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != JT_OK) return rc;
  if (dev < 0 || dev >= 64) return jt_fail(JT_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  if (g_devices[dev].sms == 0) {
    int v = 0;
    rc = jt_cuda_check(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev),
                       "SM count");
    if (rc != JT_OK) return rc;
    g_devices[dev].sms = v;
  }
  *sms = g_devices[dev].sms;
  return JT_OK;
}

template <typename Elem, int WARPS, int D, bool FP32P>
int launch_attn(const JtTreeAttnParams& p, const Layout& L, const DevLayout& d,
                cudaStream_t stream) {
  using K = AttnKernel<Elem, WARPS, D, FP32P>;
  auto kernel = tree_attn_kernel<Elem, WARPS, D, FP32P>;
  int rc = jt_cuda_check(
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, K::kSmem),
      "attention smem attribute");
  if (rc != JT_OK) return rc;
  int sms = 0;
  rc = device_sms(&sms);
  if (rc != JT_OK) return rc;
  int per_sm = 0;
  rc = jt_cuda_check(
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, K::kThreads, K::kSmem),
      "attention occupancy");
  if (rc != JT_OK) return rc;
  per_sm = std::max(per_sm, 1);
  const int num_ctas = sms * per_sm;
  const int plan_blocks = 1 + (p.total_queries + kPlanThreads / 32 - 1) / (kPlanThreads / 32);
  tree_plan_kernel<<<plan_blocks, kPlanThreads, 0, stream>>>(p, d, num_ctas);
  rc = jt_cuda_check(cudaGetLastError(), "plan launch");
  if (rc != JT_OK) return rc;
  const int grid = std::min(num_ctas, L.max_items);
  kernel<<<grid, K::kThreads, K::kSmem, stream>>>(p, d);
  return jt_cuda_check(cudaGetLastError(), "attention launch");
}

template <typename Elem, int D>
int dispatch_bm(const JtTreeAttnParams& p, const Layout& L, const DevLayout& d,
                cudaStream_t stream) {
  const bool fp32p = (p.flags & JT_FLAG_FP32_PROBABILITY) != 0;
  if (L.bm == 128)
    return fp32p ? launch_attn<Elem, 8, D, true>(p, L, d, stream)
                 : launch_attn<Elem, 8, D, false>(p, L, d, stream);
  return fp32p ? launch_attn<Elem, 4, D, true>(p, L, d, stream)
               : launch_attn<Elem, 4, D, false>(p, L, d, stream);
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// ---- tcgen05 path -------------------------------------------------------------------
constexpr int kTcItemRows = tc::kM;  // score rows per tcgen05 work item (one query tile)

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult query{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &query) ==
            cudaSuccess &&
        query == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 4-D map over a paged pool [blocks, block_size, kv_heads, 128] (strides in elements) with
// a 64-dim x 64-token box and the 128-byte swizzle of the MMA operand layout.
bool encode_pool_map(CUtensorMap* map, const void* pool, int32_t dtype, int64_t blocks,
                     int32_t block_size, int32_t heads, int64_t s0, int64_t s1, int64_t s2) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(tc::kD), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(block_size),
                              static_cast<cuuint64_t>(blocks)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(s2 * 2), static_cast<cuuint64_t>(s1 * 2),
                                 static_cast<cuuint64_t>(s0 * 2)};
  const cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(tc::kN), 1};
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  const CUresult rc = encode(map,
                             dtype == JT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             4, const_cast<void*>(pool), dims, strides, box, elem,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return rc == CUDA_SUCCESS;
}

// 3-D map over the packed queries [total_queries, heads, 128] (strides in elements): a box
// is 128/groups nodes x the groups query heads of one KV head x 64 dims, i.e. 128 score
// rows of a query tile in (node, group) order, with the MMA operand's 128-byte swizzle.
bool encode_query_map(CUtensorMap* map, const JtTreeAttnParams& p) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const int heads = p.num_kv_heads * p.groups;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(tc::kD), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(p.total_queries)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.q_stride1 * 2),
                                 static_cast<cuuint64_t>(p.q_stride0 * 2)};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(p.groups),
                             static_cast<cuuint32_t>(tc::kM / p.groups)};
  const cuuint32_t elem[3] = {1, 1, 1};
  const CUresult rc = encode(map,
                             p.dtype == JT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             3, const_cast<void*>(p.q), dims, strides, box, elem,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return rc == CUDA_SUCCESS;
}

// The tcgen05 core covers head_dim 128, pages that hold whole 128-key tiles, group counts
// that divide a 128-row query tile into whole nodes, 16-byte aligned query rows (TMA) and
// outputs whose rows allow 16-byte stores; anything else runs on the portable core.
bool tcgen05_eligible(const JtTreeAttnParams& p) {
  if (p.flags & JT_FLAG_PORTABLE_CORE) return false;
  if (p.head_dim != tc::kD || p.block_size % tc::kN != 0) return false;
  if (p.groups > tc::kM || tc::kM % p.groups != 0) return false;
  if ((p.out_stride0 | p.out_stride1) % 8 != 0) return false;
  if ((p.q_stride0 | p.q_stride1) % 8 != 0 || !al16(p.q)) return false;
  // Compute-capability major per device, queried once (0: not queried yet).
  static std::atomic<int> cc_major[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  int major = cc_major[dev].load(std::memory_order_relaxed);
  if (major == 0) {
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return false;
    cc_major[dev].store(major, std::memory_order_relaxed);
  }
  return major == 10 && tensor_map_encoder() != nullptr;
}

template <typename Elem, bool FP32P>
int launch_tc(const JtTreeAttnParams& p, const Layout& L, const DevLayout& d,
              const CUtensorMap& qmap, const CUtensorMap& kmap, const CUtensorMap& vmap,
              cudaStream_t stream) {
  auto kernel = tc::tree_attn_tc_kernel<Elem, FP32P>;
  int rc = jt_cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              tc::kSmemBytes),
                         "tcgen05 attention smem attribute");
  if (rc != JT_OK) return rc;
  int sms = 0;
  rc = device_sms(&sms);
  if (rc != JT_OK) return rc;
  // Small batches run as one launch: when even the largest possible number of work items
  // (every request's query tiles of every KV head) fits one wave of CTAs and the block
  // table cannot address more than kSingleLaunchMaxKeys keys (beyond that a split plan can
  // win), each CTA takes one item and builds its own ancestor bitmasks; the plan kernel
  // and its launch latency go away.  Both bounds come from the launch shape alone, so the
  // choice is the same on every replay of a captured graph.
  const int64_t item_bound =
      (static_cast<int64_t>(p.total_queries) * p.groups / tc::kM + p.num_requests) *
      p.num_kv_heads;
  const int64_t key_bound = static_cast<int64_t>(p.table_width) * p.block_size;
  if (item_bound <= sms && key_bound <= kSingleLaunchMaxKeys && p.split_keys == 0) {
    kernel<<<static_cast<int>(item_bound), tc::kThreads, tc::kSmemBytes, stream>>>(
        p, d, qmap, kmap, vmap, 1);
    return jt_cuda_check(cudaGetLastError(), "tcgen05 attention launch");
  }
  const int plan_blocks = 1 + (p.total_queries + kPlanThreads / 32 - 1) / (kPlanThreads / 32);
  tree_plan_kernel<<<plan_blocks, kPlanThreads, 0, stream>>>(p, d, sms);
  rc = jt_cuda_check(cudaGetLastError(), "plan launch");
  if (rc != JT_OK) return rc;
  // Programmatic dependent launch: the attention grid's prologue (barrier setup, TMEM
  // allocation) overlaps the plan kernel; the kernel waits for the plan before using it.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(std::min(sms, L.max_items));
  cfg.blockDim = dim3(tc::kThreads);
  cfg.dynamicSmemBytes = tc::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return jt_cuda_check(cudaLaunchKernelEx(&cfg, kernel, p, d, qmap, kmap, vmap, 0),
                       "tcgen05 attention launch");
}

int dispatch_tc(const JtTreeAttnParams& p, const Layout& L, const DevLayout& d,
                cudaStream_t stream) {
  CUtensorMap qmap, kmap, vmap;
  if (!encode_query_map(&qmap, p))
    return jt_fail(JT_ERR_CUDA, "tree_attn: cuTensorMapEncodeTiled rejected the query layout");
  if (!encode_pool_map(&kmap, p.k_pool, p.dtype, p.num_blocks, p.block_size, p.num_kv_heads,
                       p.k_stride0, p.k_stride1, p.k_stride2) ||
      !encode_pool_map(&vmap, p.v_pool, p.dtype, p.num_blocks, p.block_size, p.num_kv_heads,
                       p.v_stride0, p.v_stride1, p.v_stride2))
    return jt_fail(JT_ERR_CUDA, "tree_attn: cuTensorMapEncodeTiled rejected the KV pool layout");
  const bool fp32p = (p.flags & JT_FLAG_FP32_PROBABILITY) != 0;
  if (p.dtype == JT_BF16)
    return fp32p ? launch_tc<__nv_bfloat16, true>(p, L, d, qmap, kmap, vmap, stream)
                 : launch_tc<__nv_bfloat16, false>(p, L, d, qmap, kmap, vmap, stream);
  return fp32p ? launch_tc<__half, true>(p, L, d, qmap, kmap, vmap, stream)
               : launch_tc<__half, false>(p, L, d, qmap, kmap, vmap, stream);
}

}  // namespace

int jt_read_errors_attn(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_attn_errors, sizeof(uint32_t)),
                         "read attention error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_attn_errors, &zero, sizeof(uint32_t)),
                       "clear attention error word");
}

extern "C" int jt_tree_attn_workspace_size(int32_t num_requests, int32_t total_queries,
                                           int32_t num_kv_heads, int32_t groups,
                                           int32_t head_dim, size_t* bytes) {
  if (bytes == nullptr) return jt_fail(JT_ERR_INVALID, "workspace_size: null output");
  if (num_requests < 1 || total_queries < 1 || num_kv_heads < 1 || groups < 1 ||
      head_dim < 1)
    return jt_fail(JT_ERR_INVALID, "workspace_size: invalid geometry");
  size_t total = make_layout(num_requests, total_queries, num_kv_heads, groups, head_dim).total;
  if (head_dim == tc::kD)
    total = std::max(total, make_layout(num_requests, total_queries, num_kv_heads, groups,
                                        head_dim, kPartialBudgetBytes, kTcItemRows, true)
                                .total);
  *bytes = total;
  return JT_OK;
}

namespace {

// Checks every launch argument except the workspace (shared by both entry points).
int validate_params(const JtTreeAttnParams& p) {
  if (p.num_requests < 1 || p.total_queries < 1 || p.num_kv_heads < 1 || p.groups < 1 ||
      p.block_size < 1 || p.num_blocks < 1 || p.table_width < 1)
    return jt_fail(JT_ERR_INVALID, "tree_attn: invalid geometry");
  if (p.head_dim != 64 && p.head_dim != 128)
    return jt_fail(JT_ERR_UNSUPPORTED, "tree_attn: head_dim %d not in {64, 128}", p.head_dim);
  if (p.dtype != JT_BF16 && p.dtype != JT_F16 && p.dtype != JT_F32)
    return jt_fail(JT_ERR_UNSUPPORTED, "tree_attn: operands must be bf16, f16 or f32");
  if (p.out_dtype != p.dtype && p.out_dtype != JT_F32)
    return jt_fail(JT_ERR_INVALID, "tree_attn: output dtype must match input or be f32");
  if (!p.out || !p.q || !p.k_pool || !p.v_pool || !p.cu_seqlens_q || !p.query_to_request ||
      !p.query_local_row || !p.prefix_lens || !p.node_counts || !p.block_tables ||
      !p.tree_slots || !p.qq_bias || !p.qq_bias_offsets)
    return jt_fail(JT_ERR_INVALID, "tree_attn: null tensor pointer");
  if (!al16(p.q) || !al16(p.k_pool) || !al16(p.v_pool) || !al16(p.out) ||
      (p.q_stride0 | p.q_stride1 | p.k_stride0 | p.k_stride1 | p.k_stride2 | p.v_stride0 |
       p.v_stride1 | p.v_stride2) % 8 != 0 ||
      (p.out_stride0 | p.out_stride1) % 2 != 0)
    return jt_fail(JT_ERR_INVALID,
                   "tree_attn: q/k/v need 16-byte aligned bases and rows (strides multiple "
                   "of 8 elements); out strides must be even");
  if (p.split_keys < 0 ||
      (p.split_keys > 0 && (p.split_keys % 1024 != 0 ||
                            ((p.split_keys / 1024) & (p.split_keys / 1024 - 1)) != 0)))
    return jt_fail(JT_ERR_INVALID,
                   "tree_attn: split_keys must be 0 or 1024 times a power of two");
  return JT_OK;
}

// Plans and launches with a workspace laid out for `partial_budget` bytes of split-KV
// partial results (the plan coarsens splits to stay within it).
int run_tree_attn(const JtTreeAttnParams& p, int64_t partial_budget, cudaStream_t stream) {
  const bool tc_core = tcgen05_eligible(p);
  const Layout L = make_layout(p.num_requests, p.total_queries, p.num_kv_heads, p.groups,
                               p.head_dim, partial_budget, tc_core ? kTcItemRows : 0, tc_core);
  if (p.workspace == nullptr || p.workspace_bytes < L.total || !al16(p.workspace))
    return jt_fail(JT_ERR_WORKSPACE, "tree_attn: workspace of %zu bytes required (got %zu)",
                   L.total, p.workspace_bytes);
  const DevLayout d = device_layout(L, p.workspace);
  if (tc_core) return dispatch_tc(p, L, d, stream);
  if (p.dtype == JT_BF16)
    return p.head_dim == 128 ? dispatch_bm<__nv_bfloat16, 128>(p, L, d, stream)
                             : dispatch_bm<__nv_bfloat16, 64>(p, L, d, stream);
  return p.head_dim == 128 ? dispatch_bm<__half, 128>(p, L, d, stream)
                           : dispatch_bm<__half, 64>(p, L, d, stream);
}

}  // namespace

extern "C" int jt_tree_attn_launch(const JtTreeAttnParams* pp, cudaStream_t stream) {
  if (pp == nullptr) return jt_fail(JT_ERR_INVALID, "tree_attn: null params");
  const int rc = validate_params(*pp);
  if (rc != JT_OK) return rc;
  // fp32 operands: the CUDA-core kernel, which needs no workspace.
  if (pp->dtype == JT_F32) return jt_tree_attn_f32_launch(*pp, stream);
  return run_tree_attn(*pp, kPartialBudgetBytes, stream);
}

// ---- entry point without allocation ------------------------------------------------
// Some callers cannot allocate device memory: an engine that binds this library only
// through its C ABI and owns every byte of device memory through its own fixed arenas
// (a cgo / JNI / ctypes host with a frozen memory budget) can pass the tensors it holds
// but has no allocator to hand out a workspace.  jt_tree_attn_launch_noalloc serves them
// from this file-scope device array instead.  Every GPU that loads the library holds it
// until the process exits.
namespace {

constexpr size_t kStaticWorkspaceBytes = 32u << 20;     // per device
constexpr int64_t kStaticPartialBudget = 16ll << 20;    // split-KV partials within it

__device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

// Device address of g_static_workspace.  In host code the symbol names a host-side
// stand-in, not device memory, so the address comes from cudaGetSymbolAddress with the
// device current.  The address belongs to the module loaded in the CURRENT context: a
// host that switches contexts (cuCtxCreate / cuCtxSetCurrent) or resets the device
// (cudaDeviceReset, after which the module is loaded again) sees another address.  So
// outside stream capture every call looks the address up afresh (a table lookup in the
// runtime once the module is loaded) and records it with the context it belongs to;
// during capture, where lookups are best avoided, the recorded address is used only if it
// was recorded in the same context, and the call is refused otherwise.  The record is
// guarded by a mutex: several host threads may call at once.
struct StaticWorkspaceRecord {
  CUcontext ctx;
  void* ptr;
};
StaticWorkspaceRecord g_static_workspace_rec[64];
std::mutex g_static_workspace_mutex;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult query{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &query) ==
            cudaSuccess &&
        query == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(ptr);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  return fn;
}

int static_workspace(cudaStream_t stream, void** out) {
  int dev = 0;
  int rc = jt_cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != JT_OK) return rc;
  if (dev < 0 || dev >= 64) return jt_fail(JT_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  // The capture query is a runtime call on the stream: it also makes the runtime's
  // context current in this thread, so the context can be named afterwards.  Nothing
  // below may synchronise or allocate while a stream is being captured.
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  const bool capturing = cudaStreamIsCapturing(stream, &status) != cudaSuccess ||
                         status != cudaStreamCaptureStatusNone;
  if (capturing) (void)cudaGetLastError();  // clear a refused query's (non-sticky) error
  void* fresh = nullptr;
  if (!capturing) {
    rc = jt_cuda_check(cudaGetSymbolAddress(&fresh, g_static_workspace),
                       "cudaGetSymbolAddress(static workspace)");
    if (rc != JT_OK) return rc;
  }
  CUcontext ctx = nullptr;
  const CtxGetCurrentFn get_ctx = ctx_get_current();
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return jt_fail(JT_ERR_CUDA, "tree_attn_noalloc: cannot read the current CUDA context");
  std::lock_guard<std::mutex> lock(g_static_workspace_mutex);
  StaticWorkspaceRecord& rec = g_static_workspace_rec[dev];
  if (!capturing) {
    rec.ctx = ctx;
    rec.ptr = fresh;
  } else if (rec.ptr == nullptr || rec.ctx != ctx) {
    return jt_fail(JT_ERR_INVALID,
                   "tree_attn_noalloc: under stream capture before any call in this CUDA "
                   "context; make one call outside capture first");
  }
  *out = rec.ptr;
  return JT_OK;
}

}  // namespace

extern "C" int jt_tree_attn_launch_noalloc(const JtTreeAttnParams* pp, cudaStream_t stream) {
  if (pp == nullptr) return jt_fail(JT_ERR_INVALID, "tree_attn_noalloc: null params");
  int rc = validate_params(*pp);
  if (rc != JT_OK) return rc;
  if (pp->dtype == JT_F32) return jt_tree_attn_f32_launch(*pp, stream);  // no scratch at all
  const bool tc_core = tcgen05_eligible(*pp);
  const Layout L = make_layout(pp->num_requests, pp->total_queries, pp->num_kv_heads,
                               pp->groups, pp->head_dim, kStaticPartialBudget,
                               tc_core ? kTcItemRows : 0, tc_core);
  if (L.total > kStaticWorkspaceBytes)
    return jt_fail(JT_ERR_WORKSPACE,
                   "tree_attn_noalloc: this geometry needs %zu bytes of scratch, above the "
                   "static capacity of %zu bytes; use jt_tree_attn_launch with a workspace",
                   L.total, kStaticWorkspaceBytes);
  void* scratch = nullptr;
  rc = static_workspace(stream, &scratch);
  if (rc != JT_OK) return rc;
  JtTreeAttnParams p = *pp;
  p.workspace = scratch;
  p.workspace_bytes = kStaticWorkspaceBytes;
  return run_tree_attn(p, kStaticPartialBudget, stream);
}

// ---- bounded-wait self-test ---------------------------------------------------------
namespace {
__device__ int g_wait_selftest[3];
}  // namespace

extern "C" int jt_selftest_bounded_wait(int64_t limit_cycles, int32_t* out) {
  if (out == nullptr || limit_cycles < 1 || limit_cycles > (1ll << 32))
    return jt_fail(JT_ERR_INVALID, "selftest_bounded_wait: limit must be in [1, 2^32] cycles");
  int* dev = nullptr;
  int rc = jt_cuda_check(cudaGetSymbolAddress(reinterpret_cast<void**>(&dev), g_wait_selftest),
                         "self-test buffer");
  if (rc != JT_OK) return rc;
  tc::wait_selftest_kernel<<<1, 32>>>(limit_cycles, dev);
  rc = jt_cuda_check(cudaGetLastError(), "self-test launch");
  if (rc != JT_OK) return rc;
  rc = jt_cuda_check(cudaDeviceSynchronize(), "self-test run");
  if (rc != JT_OK) return rc;
  int host[3] = {0, 0, 0};
  rc = jt_cuda_check(cudaMemcpyFromSymbol(host, g_wait_selftest, sizeof(host)), "self-test read");
  if (rc != JT_OK) return rc;
  for (int i = 0; i < 3; ++i) out[i] = host[i];
  return JT_OK;
}
