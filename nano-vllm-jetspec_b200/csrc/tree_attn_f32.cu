// fp32-operand packed tree attention on the CUDA cores (sm_100a).
//
// The reference's dispatcher runs its "auto", "reference" and "prefix" backends on fp32
// q / k / v as well as bf16 / f16 (nanovllm/speculative/jetspec/paged_backend.py:240-306,
// tree_attention.py:40-62): one (query, query head) program with fp32 multiply, fp32
// reductions and an fp32 online softmax over 64-key tiles (_packed_paged_tree_fp32,
// paged_backend.py:116-213).  This kernel keeps that arithmetic class (every product and
// sum in fp32, no tensor-core rounding of the operands) but shares each K/V tile among all
// query heads of one KV head and a tile of tree nodes: one CTA = 64 score rows (64/G nodes
// x the G query heads of one KV head) of one request against the request's keys, in
// 32-key fp32 tiles double-buffered through shared memory with 16-byte cp.async.
//
// Thread (ty, tx) of 16 x 16 owns score rows 4ty..4ty+3; in QK^T it computes keys tx and
// tx + 16 of the tile, in PV output dims {4tx..4tx+3} (and {64+4tx..64+4tx+3} when D is
// 128).  A row's 16 owners are one half-warp, so row maxima and sums are half-warp
// shuffles.  P goes through shared memory (key-major) between the two products.
//
// Grid: (floor(Q / nodes_per_tile) + R, Hkv) programs, a function of the launch shape
// only (CUDA-graph capturable); request r owns programs [floor(cu[r] / n) + r,
// floor(cu[r+1] / n) + r + 1), found by binary search, and programs past the request's
// last node tile exit at once (the reference GQA launcher's grid rule, tree_gqa.py:45-50).
#include "common.cuh"

namespace {

__device__ uint32_t g_f32_errors;

constexpr int kRows = 64;      // score rows per CTA
constexpr int kKeys = 32;      // keys per K/V tile
constexpr int kThreads = 256;

template <int D>
struct F32Tile {
  static constexpr int kRowFloats = D + 4;           // padded K/V row (conflict-free LDS.128)
  static constexpr int kQFloats = kRows * D;
  static constexpr int kKVFloats = kKeys * kRowFloats;
  static constexpr int kPStride = kRows + 4;        // P row (2-way bank conflicts at most)
  static constexpr int kPFloats = kKeys * kPStride;  // P, key-major
  static constexpr int kSmemBytes = (kQFloats + 4 * kKVFloats + kPFloats) * 4;
  static constexpr int kChunks = D / 4;              // 16-byte chunks per row
  static constexpr int kDimsPerThread = D / 16;      // PV output dims per thread
};

template <int D>
__global__ void __launch_bounds__(kThreads)
    tree_attn_f32_kernel(const JtTreeAttnParams p, const int nodes_per_tile) {
  using L = F32Tile<D>;
  extern __shared__ __align__(16) float smem[];
  float* sq = smem;
  float* skv = smem + L::kQFloats;                   // [2 stages][K, V]
  float* sp = skv + 4 * L::kKVFloats;

  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int h = blockIdx.y, G = p.groups, nt = nodes_per_tile;
  // Request owning this program (largest r with floor(cu[r] / nt) + r <= program).
  const int program = blockIdx.x;
  int lo = 0, hi = p.num_requests - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.cu_seqlens_q[mid] / nt + mid <= program) lo = mid;
    else hi = mid - 1;
  }
  const int r = lo;
  const int q_start = p.cu_seqlens_q[r];
  const int tile = program - (q_start / nt + r);
  const int T = p.node_counts[r];
  const int P = p.prefix_lens[r];
  const int j0 = tile * nt;
  if (tile < 0 || j0 >= T || P < 0) return;
  const int key_end = P + min(T, j0 + nt);
  const int n_tiles = (key_end + kKeys - 1) / kKeys;
  const int bs = p.block_size;
  const int64_t pool_slots = p.num_blocks * static_cast<int64_t>(bs);
  const int32_t* table = p.block_tables + static_cast<int64_t>(r) * p.table_stride0;
  const float* bias = p.qq_bias + p.qq_bias_offsets[r];

  // Query tile: row rr = (node j0 + rr / G, head h * G + rr % G); rows past the tree are 0.
  for (int c = tid; c < kRows * L::kChunks; c += kThreads) {
    const int rr = c / L::kChunks, ch = c - rr * L::kChunks;
    const int j = j0 + rr / G, g = rr % G;
    const bool ok = rr / G < nt && j < T;
    const float* src = static_cast<const float*>(p.q);
    if (ok)
      src += static_cast<int64_t>(q_start + j) * p.q_stride0 +
             static_cast<int64_t>(h * G + g) * p.q_stride1 + ch * 4;
    jt::cp_async_16(jt::smem_u32(sq + rr * D + ch * 4), src, ok ? 16 : 0);
  }
  auto load_tile = [&](int t, int stage) {
    float* sk = skv + (2 * stage) * L::kKVFloats;
    float* sv = sk + L::kKVFloats;
    for (int c = tid; c < kKeys * L::kChunks; c += kThreads) {
      const int key = c / L::kChunks, ch = c - key * L::kChunks;
      const int pos = t * kKeys + key;
      int64_t slot = -1;
      if (pos < key_end) {
        if (pos < P) {
          const int col = pos / bs;
          if (col < p.table_width) slot = static_cast<int64_t>(__ldg(table + col)) * bs + pos % bs;
        } else {
          slot = __ldg(p.tree_slots + q_start + (pos - P));
        }
        if (slot < 0 || slot >= pool_slots) {
          if (ch == 0) atomicOr(&g_f32_errors, JT_DEVERR_OUT_OF_RANGE);
          slot = -1;
        }
      }
      const float* ks = static_cast<const float*>(p.k_pool);
      const float* vs = static_cast<const float*>(p.v_pool);
      if (slot >= 0) {
        const int64_t pg = slot / bs, o = slot - pg * bs;
        ks += pg * p.k_stride0 + o * p.k_stride1 + static_cast<int64_t>(h) * p.k_stride2 + ch * 4;
        vs += pg * p.v_stride0 + o * p.v_stride1 + static_cast<int64_t>(h) * p.v_stride2 + ch * 4;
      }
      jt::cp_async_16(jt::smem_u32(sk + key * L::kRowFloats + ch * 4), ks, slot >= 0 ? 16 : 0);
      jt::cp_async_16(jt::smem_u32(sv + key * L::kRowFloats + ch * 4), vs, slot >= 0 ? 16 : 0);
    }
  };
  load_tile(0, 0);
  jt::cp_async_commit();

  // This thread's four score rows: node index (request-local) and validity.
  int row_node[4];
  bool row_ok[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = 4 * ty + i;
    row_node[i] = j0 + rr / G;
    row_ok[i] = rr / G < nt && row_node[i] < T;
  }
  const float scale_log2 = p.scale * 1.4426950408889634f;
  float m_run[4], l_run[4];
  float acc[4][L::kDimsPerThread];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int d = 0; d < L::kDimsPerThread; ++d) acc[i][d] = 0.f;
  }

  for (int t = 0; t < n_tiles; ++t) {
    const int stage = t & 1;
    if (t + 1 < n_tiles) load_tile(t + 1, stage ^ 1);
    jt::cp_async_commit();
    jt::cp_async_wait<1>();
    __syncthreads();
    const float* sk = skv + (2 * stage) * L::kKVFloats;
    const float* sv = sk + L::kKVFloats;
    // S = Q K^T for rows 4ty..4ty+3 and keys tx, tx + 16 (fp32 FMA over the head dim).
    float s[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.f;
#pragma unroll 4
    for (int d4 = 0; d4 < L::kChunks; ++d4) {
      float4 kv[2];
#pragma unroll
      for (int jk = 0; jk < 2; ++jk)
        kv[jk] = *reinterpret_cast<const float4*>(sk + (tx + 16 * jk) * L::kRowFloats + 4 * d4);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 qv = *reinterpret_cast<const float4*>(sq + (4 * ty + i) * D + 4 * d4);
#pragma unroll
        for (int jk = 0; jk < 2; ++jk) {
          s[i][jk] = fmaf(qv.x, kv[jk].x, s[i][jk]);
          s[i][jk] = fmaf(qv.y, kv[jk].y, s[i][jk]);
          s[i][jk] = fmaf(qv.z, kv[jk].z, s[i][jk]);
          s[i][jk] = fmaf(qv.w, kv[jk].w, s[i][jk]);
        }
      }
    }
    // Visibility, online softmax (log2 units), P to shared memory.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float x[2];
#pragma unroll
      for (int jk = 0; jk < 2; ++jk) {
        const int pos = t * kKeys + tx + 16 * jk;
        bool visible = row_ok[i] && pos < key_end;
        if (visible && pos >= P) {
          const int n = pos - P;
          visible = n <= row_node[i] &&
                    __ldg(bias + static_cast<int64_t>(row_node[i]) * T + n) == 0.0f;
        }
        x[jk] = visible ? s[i][jk] * scale_log2 : -INFINITY;
      }
      float mx = fmaxf(x[0], x[1]);
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run[i], mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = jt::fast_exp2(m_run[i] - m_use);
      const float p0 = jt::fast_exp2(x[0] - m_use), p1 = jt::fast_exp2(x[1] - m_use);
      float rs = p0 + p1;
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
      l_run[i] = l_run[i] * alpha + rs;
      m_run[i] = m_new;
#pragma unroll
      for (int d = 0; d < L::kDimsPerThread; ++d) acc[i][d] *= alpha;
      sp[tx * L::kPStride + 4 * ty + i] = p0;
      sp[(tx + 16) * L::kPStride + 4 * ty + i] = p1;
    }
    __syncthreads();
    // O += P V over the tile's keys.
#pragma unroll 4
    for (int key = 0; key < kKeys; ++key) {
      const float4 pv = *reinterpret_cast<const float4*>(sp + key * L::kPStride + 4 * ty);
      const float pr[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int half = 0; half < L::kDimsPerThread / 4; ++half) {
        const float4 v = *reinterpret_cast<const float4*>(sv + key * L::kRowFloats + 64 * half + 4 * tx);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[i][4 * half + 0] = fmaf(pr[i], v.x, acc[i][4 * half + 0]);
          acc[i][4 * half + 1] = fmaf(pr[i], v.y, acc[i][4 * half + 1]);
          acc[i][4 * half + 2] = fmaf(pr[i], v.z, acc[i][4 * half + 2]);
          acc[i][4 * half + 3] = fmaf(pr[i], v.w, acc[i][4 * half + 3]);
        }
      }
    }
    __syncthreads();  // the stage and P are rewritten next iteration
  }
  jt::cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!row_ok[i]) continue;
    const int rr = 4 * ty + i;
    float* dst = static_cast<float*>(p.out) + static_cast<int64_t>(q_start + row_node[i]) * p.out_stride0 +
                 static_cast<int64_t>(h * G + rr % G) * p.out_stride1;
#pragma unroll
    for (int half = 0; half < L::kDimsPerThread / 4; ++half) {
      float4 o;
      o.x = acc[i][4 * half + 0] / l_run[i];
      o.y = acc[i][4 * half + 1] / l_run[i];
      o.z = acc[i][4 * half + 2] / l_run[i];
      o.w = acc[i][4 * half + 3] / l_run[i];
      *reinterpret_cast<float4*>(dst + 64 * half + 4 * tx) = o;
    }
  }
}

template <int D>
int launch_f32(const JtTreeAttnParams& p, cudaStream_t stream) {
  using L = F32Tile<D>;
  const int nodes_per_tile = kRows / p.groups;
  auto kernel = tree_attn_f32_kernel<D>;
  int rc = jt_cuda_check(
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes),
      "fp32 attention smem attribute");
  if (rc != JT_OK) return rc;
  const dim3 grid(static_cast<unsigned>(p.total_queries / nodes_per_tile + p.num_requests),
                  static_cast<unsigned>(p.num_kv_heads));
  kernel<<<grid, kThreads, L::kSmemBytes, stream>>>(p, nodes_per_tile);
  return jt_cuda_check(cudaGetLastError(), "fp32 attention launch");
}

}  // namespace

int jt_read_errors_f32(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_f32_errors, sizeof(uint32_t)),
                         "read fp32 attention error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_f32_errors, &zero, sizeof(uint32_t)),
                       "clear fp32 attention error word");
}

// Launch of the fp32 path for parameters already checked by the entry point: fp32 q, k,
// v and out, groups dividing 64, head_dim 64 or 128, 16-byte aligned rows.
int jt_tree_attn_f32_launch(const JtTreeAttnParams& p, cudaStream_t stream) {
  if (p.groups > kRows || kRows % p.groups != 0)
    return jt_fail(JT_ERR_UNSUPPORTED, "tree_attn: fp32 operands need groups dividing 64 (got %d)",
                   p.groups);
  if ((p.q_stride0 | p.q_stride1 | p.k_stride0 | p.k_stride1 | p.k_stride2 | p.v_stride0 |
       p.v_stride1 | p.v_stride2 | p.out_stride0 | p.out_stride1) % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(p.out) & 15u) != 0)
    return jt_fail(JT_ERR_INVALID,
                   "tree_attn: fp32 operands need 16-byte aligned rows (strides multiple of 4)");
  return p.head_dim == 128 ? launch_f32<128>(p, stream) : launch_f32<64>(p, stream);
}
