// HF-order RoPE of Q and K fused with the tree-node K/V scatter (sm_100a).
//
// One CTA per packed row.  Its threads cover (head, rotation pair) tasks: every query
// head's pairs (d, d + dim/2) produce the rotated Q row; the KV heads' pairs also rotate
// K into the pool slot and copy V.  The arithmetic keeps eager PyTorch's rounding points:
// each product is rounded to the operand type, then the add / subtract, then the result
// (explicit __fmul_rn / __fadd_rn / __fsub_rn, so nothing contracts into an FMA).
#include "common.cuh"

namespace {

constexpr int kRopeThreads = 256;

__device__ uint32_t g_rope_errors;

template <typename T>
struct Scalar;
template <>
struct Scalar<__nv_bfloat16> {
  __device__ __forceinline__ static float load(const void* p, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  __device__ __forceinline__ static void store(void* p, int64_t i, float x) {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  }
};
template <>
struct Scalar<float> {
  __device__ __forceinline__ static float load(const void* p, int64_t i) {
    return static_cast<const float*>(p)[i];
  }
  __device__ __forceinline__ static float round(float x) { return x; }
  __device__ __forceinline__ static void store(void* p, int64_t i, float x) {
    static_cast<float*>(p)[i] = x;
  }
};

__device__ __forceinline__ int64_t load_index(const void* p, int64_t i, int is64) {
  return is64 ? static_cast<const int64_t*>(p)[i] : static_cast<const int32_t*>(p)[i];
}

__device__ __forceinline__ float load_cache(const JtRopeScatterParams& p, int64_t i) {
  return p.cache_dtype == JT_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.cos_sin_cache)[i])
                                  : static_cast<const float*>(p.cos_sin_cache)[i];
}

// rope of the pair (x1, x2) with (cos, sin): products rounded, then sum / difference.
template <typename T>
__device__ __forceinline__ void rotate(float x1, float x2, float c, float s, float& r1,
                                       float& r2) {
  using S = Scalar<T>;
  const float a = S::round(__fmul_rn(x1, c));
  const float b = S::round(__fmul_rn(x2, s));
  const float cc = S::round(__fmul_rn(x2, c));
  const float d = S::round(__fmul_rn(x1, s));
  r1 = __fsub_rn(a, b);
  r2 = __fadd_rn(cc, d);
}

template <typename T>
__global__ void __launch_bounds__(kRopeThreads) rope_scatter_kernel(const JtRopeScatterParams p) {
  using S = Scalar<T>;
  const int row = blockIdx.x;
  const int half = p.head_dim / 2;
  const int64_t position = load_index(p.positions, row * p.positions_stride, p.positions_is_int64);
  const int64_t cache_row = position * p.cache_stride0;
  const int q_tasks = p.q_heads * half;
  const int k_tasks = p.kv_heads * half;
  const int v_tasks = p.kv_heads * p.head_dim;
  int64_t page = -1, offset = 0;
  {
    const int64_t slot = load_index(p.node_slots, row * p.slots_stride, p.slots_is_int64);
    const int64_t capacity = p.num_pages * static_cast<int64_t>(p.page_size);
    if (slot >= 0 && slot < capacity) {
      page = slot / p.page_size;
      offset = slot - page * p.page_size;
    } else if (threadIdx.x == 0) {
      atomicOr(&g_rope_errors, JT_DEVERR_OUT_OF_RANGE);
    }
  }
  for (int task = threadIdx.x; task < q_tasks + k_tasks + v_tasks; task += kRopeThreads) {
    if (task < q_tasks + k_tasks) {
      const bool is_q = task < q_tasks;
      const int t = is_q ? task : task - q_tasks;
      const int head = t / half, d = t - head * half;
      // cos / sin converted to the operand type first (cache.to(dtype)).
      const float c = S::round(load_cache(p, cache_row + d * p.cache_stride_last));
      const float s = S::round(load_cache(p, cache_row + (d + half) * p.cache_stride_last));
      float r1, r2;
      if (is_q) {
        const int64_t base = row * p.q_stride0 + head * p.q_stride1;
        rotate<T>(S::load(p.q, base + d * p.q_stride2), S::load(p.q, base + (d + half) * p.q_stride2),
                  c, s, r1, r2);
        const int64_t ob = row * p.out_stride0 + head * p.out_stride1;
        S::store(p.out, ob + d * p.out_stride2, r1);
        S::store(p.out, ob + (d + half) * p.out_stride2, r2);
      } else {
        if (page < 0) continue;
        const int64_t base = row * p.k_stride0 + head * p.k_stride1;
        rotate<T>(S::load(p.k, base + d * p.k_stride2), S::load(p.k, base + (d + half) * p.k_stride2),
                  c, s, r1, r2);
        const int64_t kb = page * p.kp_stride0 + offset * p.kp_stride1 + head * p.kp_stride2;
        S::store(p.k_pool, kb + d * p.kp_stride3, r1);
        S::store(p.k_pool, kb + (d + half) * p.kp_stride3, r2);
      }
    } else {
      if (page < 0) continue;
      const int t = task - q_tasks - k_tasks;
      const int head = t / p.head_dim, d = t - head * p.head_dim;
      const int64_t src = row * p.v_stride0 + head * p.v_stride1 + d * p.v_stride2;
      const int64_t dst = page * p.vp_stride0 + offset * p.vp_stride1 + head * p.vp_stride2 +
                          d * p.vp_stride3;
      if constexpr (sizeof(T) == 2)
        static_cast<__nv_bfloat16*>(p.v_pool)[dst] = static_cast<const __nv_bfloat16*>(p.v)[src];
      else
        static_cast<float*>(p.v_pool)[dst] = static_cast<const float*>(p.v)[src];
    }
  }
}

}  // namespace

int jt_read_errors_rope(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_rope_errors, sizeof(uint32_t)),
                         "read rope error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_rope_errors, &zero, sizeof(uint32_t)),
                       "clear rope error word");
}

extern "C" int jt_rope_scatter_launch(const JtRopeScatterParams* p, cudaStream_t stream) {
  if (p == nullptr) return jt_fail(JT_ERR_INVALID, "rope_scatter: null params");
  if (p->rows < 0 || p->q_heads < 1 || p->kv_heads < 1 || p->q_heads % p->kv_heads != 0 ||
      p->head_dim < 2 || p->head_dim % 2 != 0 || p->head_dim > 256 || p->page_size < 1 ||
      p->num_pages < 1)
    return jt_fail(JT_ERR_INVALID, "rope_scatter: invalid geometry");
  if ((p->dtype != JT_BF16 && p->dtype != JT_F32) ||
      (p->cache_dtype != JT_BF16 && p->cache_dtype != JT_F32))
    return jt_fail(JT_ERR_UNSUPPORTED, "rope_scatter: operands must be bf16 or fp32");
  if (p->rows == 0) return JT_OK;
  if (!p->q || !p->k || !p->v || !p->positions || !p->cos_sin_cache || !p->node_slots ||
      !p->out || !p->k_pool || !p->v_pool)
    return jt_fail(JT_ERR_INVALID, "rope_scatter: null tensor pointer");
  if (p->dtype == JT_BF16)
    rope_scatter_kernel<__nv_bfloat16><<<p->rows, kRopeThreads, 0, stream>>>(*p);
  else
    rope_scatter_kernel<float><<<p->rows, kRopeThreads, 0, stream>>>(*p);
  return jt_cuda_check(cudaGetLastError(), "rope_scatter launch");
}
