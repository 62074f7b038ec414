// Greedy acceptance walk over the packed verification trees, on the device.
//
// The reference takes the argmax of every tree node's logits ([Q, vocab]), downloads the
// Q token ids and walks each tree on the host (accept_batch,
// nanovllm/speculative/jetspec/serving_ops.py:55-90): from the root, follow the child
// whose draft token equals the current node's greedy token (the last such child when
// siblings repeat a token), up to max_depth steps; the correction token is the greedy
// token of the last node on the path.  Only the argmaxes of the nodes on the path are
// ever read, so this kernel computes them lazily: one CTA per request reduces the logits
// row of the current node, searches the node's children for the greedy token, and moves
// on.  A verification round with accepted paths of a few nodes reads a few rows per
// request instead of all Q rows (config 3: ~48 MB instead of 1.18 GB), and the result
// stays on the device for the accepted-KV commit (no host round trip between them).
//
// argmax follows torch.argmax: NaN ranks above every number and ties go to the lowest
// index.  The depth check of the reference (depths along the path equal 0, 1, 2, ...)
// sets JT_DEVERR_OUT_OF_RANGE instead of raising; a parent index outside the request is
// skipped the same way.
#include <type_traits>

#include "common.cuh"

namespace {

__device__ uint32_t g_accept_errors;

constexpr int kAcceptThreads = 1024;  // 128 KB of a logits row in flight per CTA

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}

// NaN-propagating max ("NaN ranks highest"), two lanes at a time for 16-bit types.
__device__ __forceinline__ uint32_t vmax2(uint32_t a, uint32_t b, __nv_bfloat16) {
  const __nv_bfloat162 r = __hmax2_nan(*reinterpret_cast<__nv_bfloat162*>(&a),
                                       *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t vmax2(uint32_t a, uint32_t b, __half) {
  const __half2 r = __hmax2_nan(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;\n" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float lo_f32(uint32_t v, __nv_bfloat16) {
  return __uint_as_float(v << 16);
}
__device__ __forceinline__ float hi_f32(uint32_t v, __nv_bfloat16) {
  return __uint_as_float(v & 0xffff0000u);
}
__device__ __forceinline__ float lo_f32(uint32_t v, __half) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xffffu)));
}
__device__ __forceinline__ float hi_f32(uint32_t v, __half) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
}

// Block-wide NaN-propagating max of one float per thread (every thread gets it).
__device__ float block_max_nan(float v, float* s_val) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) s_val[warp] = v;
  __syncthreads();
  v = s_val[0];
  for (int w = 1; w < kAcceptThreads / 32; ++w) v = fmax_nan(v, s_val[w]);
  __syncthreads();
  return v;
}
__device__ int block_min(int v, int* s_idx) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) s_idx[warp] = v;
  __syncthreads();
  v = s_idx[0];
  for (int w = 1; w < kAcceptThreads / 32; ++w) v = min(v, s_idx[w]);
  __syncthreads();
  return v;
}

__device__ __forceinline__ bool same(float a, float m) { return a == m || (a != a && m != m); }

// argmax of one logits row, over the whole block; every thread gets the result.  Pass 1:
// the row's max (NaN highest) with packed max instructions while streaming the row;
// pass 2: the first index holding it (the row is now in L2).
template <typename T>
__device__ int row_argmax(const T* row, int vocab, float* s_val, int* s_idx) {
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte load
  const int tid = threadIdx.x;
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  const int nvec = aligned ? vocab / kVec : 0;
  const uint4* vrow = reinterpret_cast<const uint4*>(row);
  float best = -INFINITY;
  constexpr int kInFlight = 8;
  if constexpr (sizeof(T) == 2) {
    uint32_t m2 = 0xff80ff80u;  // two -inf (bf16); for f16 0xfc00 pairs below
    if constexpr (std::is_same<T, __half>::value) m2 = 0xfc00fc00u;
    int v = tid;
    for (; v + (kInFlight - 1) * kAcceptThreads < nvec; v += kInFlight * kAcceptThreads) {
      uint4 x[kInFlight];
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) x[u] = __ldcg(vrow + v + u * kAcceptThreads);
#pragma unroll
      for (int u = 0; u < kInFlight; ++u)
        m2 = vmax2(vmax2(m2, vmax2(x[u].x, x[u].y, T()), T()), vmax2(x[u].z, x[u].w, T()), T());
    }
    for (; v < nvec; v += kAcceptThreads) {
      const uint4 x = __ldcg(vrow + v);
      m2 = vmax2(vmax2(m2, vmax2(x.x, x.y, T()), T()), vmax2(x.z, x.w, T()), T());
    }
    best = fmax_nan(lo_f32(m2, T()), hi_f32(m2, T()));
  } else {
    for (int v = tid; v < nvec; v += kAcceptThreads) {
      const uint4 x = __ldcg(vrow + v);
      best = fmax_nan(fmax_nan(fmax_nan(best, __uint_as_float(x.x)), __uint_as_float(x.y)),
                      fmax_nan(__uint_as_float(x.z), __uint_as_float(x.w)));
    }
  }
  for (int idx = nvec * kVec + tid; idx < vocab; idx += kAcceptThreads)
    best = fmax_nan(best, to_f32(row[idx]));
  const float m = block_max_nan(best, s_val);
  // Pass 2: the lowest index whose value is the maximum (an equal NaN counts as equal).
  int first = 0x7fffffff;
  for (int v = tid; v < nvec && first == 0x7fffffff; v += kAcceptThreads) {
    const uint4 x = __ldcg(vrow + v);
    const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
    for (int k = kVec - 1; k >= 0; --k)
      if (same(to_f32(e[k]), m)) first = v * kVec + k;
  }
  for (int idx = nvec * kVec + tid; idx < vocab && first == 0x7fffffff; idx += kAcceptThreads)
    if (same(to_f32(row[idx]), m)) first = idx;
  return block_min(first, s_idx);
}

template <typename T>
__global__ void __launch_bounds__(kAcceptThreads)
    accept_walk_kernel(JtAcceptWalkParams p) {
  __shared__ float s_val[kAcceptThreads / 32];
  __shared__ int s_idx[33];
  __shared__ int s_child;
  const int r = blockIdx.x, tid = threadIdx.x;
  const int lo = p.offsets[r], hi = p.offsets[r + 1];
  // A request outside [0, num_nodes] is treated as empty (skipped and flagged), so no
  // row or node entry beyond the arrays is ever read.
  const int nodes = (lo >= 0 && hi <= p.num_nodes) ? hi - lo : 0;
  int32_t* path = p.path + static_cast<int64_t>(r) * p.path_stride;
  int64_t* outputs = p.outputs + static_cast<int64_t>(r) * p.path_stride;
  for (int i = tid; i < p.path_stride; i += kAcceptThreads) {
    path[i] = -1;
    outputs[i] = -1;
  }
  if (nodes < 1) {
    if (tid == 0) {
      p.accepted_length[r] = -1;
      p.correction[r] = -1;
      atomicOr(&g_accept_errors, JT_DEVERR_OUT_OF_RANGE);
    }
    return;
  }
  const T* logits = static_cast<const T*>(p.logits);
  int node = 0, len = 1;
  bool depth_ok = p.depths == nullptr || p.depths[lo] == 0;
  __syncthreads();
  if (tid == 0) path[0] = 0;
  int greedy = 0;
  for (;;) {
    greedy = row_argmax<T>(logits + static_cast<int64_t>(lo + node) * p.logits_stride0, p.vocab,
                           s_val, s_idx);
    if (len > p.max_depth) break;
    // Children of `node` carrying the greedy token; the last one wins (the reference's
    // child maps are filled in node order, later siblings overwriting earlier ones).
    if (tid == 0) s_child = -1;
    __syncthreads();
    int child = -1;
    for (int j = tid; j < nodes; j += kAcceptThreads)
      if (p.parent_indices[lo + j] == node && p.token_ids[lo + j] == greedy) child = j;
    for (int o = 16; o > 0; o >>= 1) child = max(child, __shfl_xor_sync(0xffffffffu, child, o));
    if ((tid & 31) == 0 && child >= 0) atomicMax(&s_child, child);
    __syncthreads();
    child = s_child;
    __syncthreads();
    if (child < 0) break;
    if (p.depths != nullptr && p.depths[lo + child] != len) depth_ok = false;
    if (tid == 0) {
      path[len] = child;
      outputs[len - 1] = p.token_ids[lo + child];
    }
    node = child;
    ++len;
  }
  if (tid == 0) {
    outputs[len - 1] = greedy;
    p.accepted_length[r] = len - 1;
    p.correction[r] = greedy;
    if (!depth_ok) atomicOr(&g_accept_errors, JT_DEVERR_OUT_OF_RANGE);
  }
}

}  // namespace

int jt_read_errors_accept(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_accept_errors, sizeof(uint32_t)),
                         "read acceptance error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_accept_errors, &zero, sizeof(uint32_t)),
                       "clear acceptance error word");
}

extern "C" int jt_accept_walk_launch(const JtAcceptWalkParams* pp, cudaStream_t stream) {
  if (pp == nullptr) return jt_fail(JT_ERR_INVALID, "accept_walk: null params");
  const JtAcceptWalkParams& p = *pp;
  if (p.num_requests < 1 || p.vocab < 1 || p.max_depth < 0 || p.num_nodes < 1 ||
      p.path_stride < p.max_depth + 1 || p.logits_stride0 < p.vocab)
    return jt_fail(JT_ERR_INVALID, "accept_walk: invalid geometry");
  if (!p.logits || !p.token_ids || !p.parent_indices || !p.offsets || !p.path ||
      !p.accepted_length || !p.correction || !p.outputs)
    return jt_fail(JT_ERR_INVALID, "accept_walk: null tensor pointer");
  if (p.logits_dtype != JT_BF16 && p.logits_dtype != JT_F16 && p.logits_dtype != JT_F32)
    return jt_fail(JT_ERR_UNSUPPORTED, "accept_walk: logits must be bf16, f16 or f32");
  const dim3 grid(p.num_requests);
  if (p.logits_dtype == JT_BF16)
    accept_walk_kernel<__nv_bfloat16><<<grid, kAcceptThreads, 0, stream>>>(p);
  else if (p.logits_dtype == JT_F16)
    accept_walk_kernel<__half><<<grid, kAcceptThreads, 0, stream>>>(p);
  else
    accept_walk_kernel<float><<<grid, kAcceptThreads, 0, stream>>>(p);
  return jt_cuda_check(cudaGetLastError(), "accept_walk launch");
}
