// Blackwell (sm_100a) tree-attention core: tcgen05 tensor cores with TMEM accumulators.
//
// Included by tree_attn.cu inside its anonymous namespace (uses DevLayout, the plan's
// work items and g_attn_errors).  One persistent CTA per SM; work items come from the
// device plan in longest-first order and are strided over the CTAs.  An item is up to
// two 128-row query tiles (256 score rows = 256/groups tree nodes x groups query heads)
// of one (request, KV head, key split).  Warp roles:
//
//   warp 0       MMA issuer (one thread) and TMEM owner (512 columns)
//   warps 1-3    loaders: TMA for full prefix tiles (64 keys inside one page, 128-byte
//                swizzle), cp.async for query tiles and for tiles that touch the tree
//                nodes (scattered scratch slots), written in the same swizzled layout
//   warps 4-7    softmax + epilogue of query tile 0 (one thread per score row)
//   warps 8-11   softmax + epilogue of query tile 1
//
// Per 64-key tile j and query tile i: S_i = Q_i K_j^T (tcgen05.mma, A and B from shared
// memory, fp32 accumulator in TMEM); the softmax warps read S_i from TMEM, apply the
// tree mask, update the fp32 online softmax and write P_i (rounded to the operand type)
// back to TMEM; O_i += P_i V_j (tcgen05.mma with A from TMEM, B = V in shared memory,
// MN-major).  The two query tiles ping-pong: while one tile's softmax runs, the tensor
// core works on the other tile.  The running max is only moved (and O rescaled in TMEM)
// when it grows by more than 2^8, so P stays <= 256 and the rescale is rare.
//
// Every mbarrier wait is bounded; a wait that runs out sets JT_DEVERR_TIMEOUT and an
// abort flag, after which all roles run to the end without waiting, drain their own
// asynchronous copies and MMAs, and the CTA frees its TMEM and exits.

namespace tc {

constexpr int kN = 64;        // keys per KV tile
constexpr int kD = 128;       // head dim
constexpr int kM = 128;       // rows per query tile (MMA M)
constexpr int kStages = 4;    // KV ring depth
constexpr int kThreads = 384;
constexpr int kQTileBytes = kM * kD * 2;   // 32 KB: two 64-dim halves of [128 rows][128 B]
constexpr int kQHalfBytes = kM * 128;
constexpr int kKVBytes = kN * kD * 2;      // 16 KB: two 64-dim halves of [64 keys][128 B]
constexpr int kKVHalfBytes = kN * 128;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kQTileBytes;
constexpr int kOffV = kOffK + kStages * kKVBytes;
constexpr int kOffBar = kOffV + kStages * kKVBytes;
constexpr int kNumBars = 2 * kStages + 2 + 4 * 2 + 1;
constexpr int kOffRows = kOffBar + 8 * 32;              // 64 x (K, V) row byte offsets
constexpr int kOffMisc = kOffRows + 64 * 2 * 8;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;        // + alignment slack
constexpr long long kWaitLimit = 4000000000ll;          // cycles (~2 s) per wait

// TMEM column map (512 columns x 128 lanes x 32 bit).
__host__ __device__ constexpr uint32_t col_o(int i) { return 128u * i; }          // O_i: 128 cols
__host__ __device__ constexpr uint32_t col_s(int i) { return 256u + 64u * i; }    // S_i: 64 cols
__host__ __device__ constexpr uint32_t col_p(int i) { return 384u + 32u * i; }    // P_i: 32 cols
__host__ __device__ constexpr uint32_t col_pl(int i) { return 448u + 32u * i; }   // P_i low part

// Barrier indices.
constexpr int kBarKvFull = 0;
constexpr int kBarKvEmpty = kStages;
constexpr int kBarQFull = 2 * kStages;
constexpr int kBarQEmpty = kBarQFull + 1;
constexpr int kBarSFull = kBarQEmpty + 1;    // [2]
constexpr int kBarPFull = kBarSFull + 2;     // [2]
constexpr int kBarODone = kBarPFull + 2;     // [2]
constexpr int kBarOFree = kBarODone + 2;     // [2]
constexpr int kBarDrain = kBarOFree + 2;

// ---- PTX wrappers ------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the completion of the phase with the given parity.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          bool abortable = true) {
  if (mbar_try(bar, parity)) return true;
  const long long start = clock64();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (abortable && *abort) return false;
    if (clock64() - start > kWaitLimit) {
      *abort = 1;
      atomicOr(&g_attn_errors, JT_DEVERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::f16 with an fp32 accumulator.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool bf16, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31]));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// Byte offset of 16-byte chunk `chunk` (0..15 over 128 dims) of row `row` in a tile made
// of two 64-dim halves of `rows` x 128 B, with the 128-byte swizzle the MMA expects.
__device__ __forceinline__ uint32_t swz128(int row, int chunk, int rows) {
  const int half = chunk >> 3, c = chunk & 7;
  return static_cast<uint32_t>(half * rows * 128 + row * 128 + ((c ^ (row & 7)) << 4));
}

struct Item {
  int r, split, h, tp, n_split, mblocks, slot_base, counter_base;
  int P, T, q_start, key_begin, key_end, n_tiles, nq;
};

__device__ __forceinline__ Item decode(const JtTreeAttnParams& p, const DevLayout& w, int index,
                                       int split_keys) {
  Item it;
  const int4 e = w.items[index];
  it.r = e.x;
  it.split = e.y;
  it.h = e.z;
  it.tp = e.w;
  const int4 info = w.req[it.r];
  it.n_split = info.x;
  it.slot_base = info.y;
  it.counter_base = info.z;
  it.mblocks = info.w;
  it.P = p.prefix_lens[it.r];
  it.T = p.node_counts[it.r];
  it.q_start = p.cu_seqlens_q[it.r];
  const int G = p.groups;
  const int rows = it.T * G - it.tp * 2 * kM;
  it.nq = rows > kM ? 2 : 1;
  it.key_begin = it.split * split_keys;
  if (it.split + 1 < it.n_split) {
    it.key_end = it.key_begin + split_keys;
  } else {
    const int last_row = it.tp * 2 * kM + it.nq * kM - 1;
    it.key_end = it.P + min(it.T, last_row / G + 1);
  }
  it.n_tiles = (it.key_end - it.key_begin + kN - 1) / kN;
  return it;
}

template <typename Elem, bool FP32P>
__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_tc_kernel(const JtTreeAttnParams p, const DevLayout w,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
  using Mma = jt::MmaOp<Elem>;
  constexpr bool kBf16 = std::is_same<Elem, __nv_bfloat16>::value;
  constexpr uint32_t kIdescQK = instr_desc(kM, kN, kBf16, false);
  constexpr uint32_t kIdescPV = instr_desc(kM, kD, kBf16, true);

  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = jt::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw);
  auto bar = [&](int i) { return base + kOffBar + 8u * static_cast<uint32_t>(i); };
  int64_t* row_off = reinterpret_cast<int64_t*>(sbase + kOffRows);  // [64][2]
  volatile int* misc = reinterpret_cast<volatile int*>(sbase + kOffMisc);
  // misc[0]: TMEM base, misc[1]: abort, misc[2..3]: split-merge flags
  volatile int* abort = misc + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t count = 1;
      if (i == kBarPFull || i == kBarPFull + 1 || i == kBarOFree || i == kBarOFree + 1) count = 128;
      mbar_init(bar(i), count);
    }
    misc[1] = 0;
    misc[2] = misc[3] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(
                     base + kOffMisc)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = static_cast<uint32_t>(misc[0]);

  const int num_items = w.header[1];
  const int split_keys = w.header[2];
  const int G = p.groups, bs = p.block_size;

  if (warp == 0) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t kv_count = 0, q_count = 0, pf[2] = {0, 0}, of[2] = {0, 0};
      const uint32_t sq0 = base + kOffQ;
      for (int index = blockIdx.x; index < num_items; index += gridDim.x) {
        const Item it = decode(p, w, index, split_keys);
        mbar_wait(bar(kBarQFull), q_count & 1, abort);
        ++q_count;
        tc_fence_after();
        auto issue_qk = [&](int i, int stage) {
          const uint32_t qa = sq0 + i * kQTileBytes;
          const uint32_t ka = base + kOffK + stage * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk & 3) * 32;
            const uint64_t a = smem_desc(qa + (kk >> 2) * kQHalfBytes + off, 16, 1024);
            const uint64_t b = smem_desc(ka + (kk >> 2) * kKVHalfBytes + off, 16, 1024);
            mma_ss(tmem + col_s(i), a, b, kIdescQK, kk > 0 ? 1u : 0u);
          }
          tc_commit(bar(kBarSFull + i));
        };
        auto issue_pv = [&](int i, int stage, bool accumulate) {
          const uint32_t va = base + kOffV + stage * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            const uint64_t b = smem_desc(va + kk * 2048, kKVHalfBytes, 1024);
            mma_ts(tmem + col_o(i), tmem + col_p(i) + kk * 8, b, kIdescPV,
                   (accumulate || kk > 0) ? 1u : 0u);
            if constexpr (FP32P)
              mma_ts(tmem + col_o(i), tmem + col_pl(i) + kk * 8, b, kIdescPV, 1u);
          }
          tc_commit(bar(kBarODone + i));
        };
        {
          const int stage = kv_count % kStages;
          mbar_wait(bar(kBarKvFull + stage), (kv_count / kStages) & 1, abort);
          tc_fence_after();
          for (int i = 0; i < it.nq; ++i) issue_qk(i, stage);
          if (it.n_tiles == 1) tc_commit(bar(kBarQEmpty));
        }
        for (int t = 0; t < it.n_tiles; ++t) {
          const int stage = kv_count % kStages;
          for (int i = 0; i < it.nq; ++i) {
            if (t == 0 && of[i] > 0) mbar_wait(bar(kBarOFree + i), (of[i] - 1) & 1, abort);
            mbar_wait(bar(kBarPFull + i), pf[i] & 1, abort);
            ++pf[i];
            tc_fence_after();
            issue_pv(i, stage, t > 0);
            if (t + 1 < it.n_tiles) {
              const int next = (kv_count + 1) % kStages;
              if (i == 0) {
                mbar_wait(bar(kBarKvFull + next), ((kv_count + 1) / kStages) & 1, abort);
                tc_fence_after();
              }
              issue_qk(i, next);
              if (t + 2 == it.n_tiles && i == it.nq - 1) tc_commit(bar(kBarQEmpty));
            }
          }
          tc_commit(bar(kBarKvEmpty + stage));
          ++kv_count;
        }
        for (int i = 0; i < it.nq; ++i) ++of[i];
      }
      // Drain: every MMA this thread issued has completed before TMEM is released.
      tc_commit(bar(kBarDrain));
      mbar_wait(bar(kBarDrain), 0, abort, false);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------------ loaders
    const int ltid = tid - 32;
    uint32_t kv_count = 0, q_count = 0;
    uint32_t filled = 0;       // stages whose last fill went through TMA (drain bookkeeping)
    uint32_t last_parity = 0;  // bit s: phase parity of stage s's last TMA fill
    const char* kbase = static_cast<const char*>(p.k_pool);
    const char* vbase = static_cast<const char*>(p.v_pool);
    const int64_t pool_slots = p.num_blocks * static_cast<int64_t>(bs);
    for (int index = blockIdx.x; index < num_items; index += gridDim.x) {
      const Item it = decode(p, w, index, split_keys);
      const int32_t* table = p.block_tables + static_cast<int64_t>(it.r) * p.table_stride0;
      // Query tiles (cp.async, swizzled).  Rows past the request's nodes are zero.
      if (q_count > 0) mbar_wait(bar(kBarQEmpty), (q_count - 1) & 1, abort);
      const int qrows = it.nq * kM;
      for (int c = ltid; c < qrows * 16; c += 96) {
        const int row = c >> 4, chunk = c & 15;
        const int gm = it.tp * 2 * kM + row;
        const int j = gm / G, g = gm - j * G;
        const bool ok = j < it.T;
        const char* src = static_cast<const char*>(p.q);
        if (ok)
          src += (static_cast<int64_t>(it.q_start + j) * p.q_stride0 +
                  static_cast<int64_t>(it.h * G + g) * p.q_stride1 + chunk * 8) * 2;
        const uint32_t dst = base + kOffQ + (row >> 7) * kQTileBytes + swz128(row & 127, chunk, kM);
        jt::cp_async_16(dst, src, ok ? 16 : 0);
      }
      asm volatile("cp.async.wait_all;\n" ::: "memory");
      fence_proxy_async();
      named_sync(2, 96);
      if (ltid == 0) mbar_arrive(bar(kBarQFull));
      ++q_count;

      for (int t = 0; t < it.n_tiles; ++t) {
        const int stage = kv_count % kStages;
        const uint32_t parity = (kv_count / kStages) & 1;
        const int kb = it.key_begin + t * kN;
        const bool full = kb + kN <= min(it.P, it.key_end);
        const uint32_t kdst = base + kOffK + stage * kKVBytes;
        const uint32_t vdst = base + kOffV + stage * kKVBytes;
        if (full) {
          if (ltid == 0) {
            if (kv_count >= kStages) mbar_wait(bar(kBarKvEmpty + stage), parity ^ 1, abort);
            const int page = __ldg(table + kb / bs);
            const int off = kb % bs;
            mbar_arrive_tx(bar(kBarKvFull + stage), 2 * kKVBytes);
            tma_load_4d(kdst, &kmap, 0, it.h, off, page, bar(kBarKvFull + stage));
            tma_load_4d(kdst + kKVHalfBytes, &kmap, 64, it.h, off, page, bar(kBarKvFull + stage));
            tma_load_4d(vdst, &vmap, 0, it.h, off, page, bar(kBarKvFull + stage));
            tma_load_4d(vdst + kKVHalfBytes, &vmap, 64, it.h, off, page, bar(kBarKvFull + stage));
            filled |= 1u << stage;
            last_parity = (last_parity & ~(1u << stage)) | (parity << stage);
          }
        } else {
          if (kv_count >= kStages) mbar_wait(bar(kBarKvEmpty + stage), parity ^ 1, abort);
          if (ltid < kN) {
            const int pos = kb + ltid;
            int64_t ko = -1, vo = -1;
            if (pos < it.key_end) {
              int64_t slot = -1;
              if (pos < it.P) {
                const int col = pos / bs;
                if (col < p.table_width)
                  slot = static_cast<int64_t>(__ldg(table + col)) * bs + pos % bs;
              } else {
                slot = __ldg(p.tree_slots + it.q_start + (pos - it.P));
              }
              if (slot >= 0 && slot < pool_slots) {
                const int64_t page = slot / bs, off = slot - page * bs;
                ko = (page * p.k_stride0 + off * p.k_stride1 +
                      static_cast<int64_t>(it.h) * p.k_stride2) * 2;
                vo = (page * p.v_stride0 + off * p.v_stride1 +
                      static_cast<int64_t>(it.h) * p.v_stride2) * 2;
              } else {
                atomicOr(&g_attn_errors, JT_DEVERR_OUT_OF_RANGE);
              }
            }
            row_off[2 * ltid] = ko;
            row_off[2 * ltid + 1] = vo;
          }
          named_sync(2, 96);
          for (int c = ltid; c < kN * 16; c += 96) {
            const int row = c >> 4, chunk = c & 15;
            const int64_t ko = row_off[2 * row], vo = row_off[2 * row + 1];
            const uint32_t o = swz128(row, chunk, kN);
            jt::cp_async_16(kdst + o, ko >= 0 ? kbase + ko + chunk * 16 : kbase, ko >= 0 ? 16 : 0);
            jt::cp_async_16(vdst + o, vo >= 0 ? vbase + vo + chunk * 16 : vbase, vo >= 0 ? 16 : 0);
          }
          asm volatile("cp.async.wait_all;\n" ::: "memory");
          fence_proxy_async();
          named_sync(2, 96);
          if (ltid == 0) {
            mbar_arrive(bar(kBarKvFull + stage));
            filled &= ~(1u << stage);
          }
        }
        ++kv_count;
      }
    }
    // Drain: the TMA copies this thread issued have landed before the CTA exits.
    if (ltid == 0) {
      for (int s = 0; s < kStages; ++s)
        if (filled & (1u << s)) mbar_wait(bar(kBarKvFull + s), (last_parity >> s) & 1u, abort, false);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int i = (warp - 4) >> 2;          // query tile of this warpgroup
    const int t128 = tid - 128 - i * 128;   // row within the query tile
    const uint32_t lane_base = static_cast<uint32_t>((t128 >> 5) * 32) << 16;
    const float scale_log2 = p.scale * 1.4426950408889634f;
    uint32_t sf = 0, od = 0;
    for (int index = blockIdx.x; index < num_items; index += gridDim.x) {
      const Item it = decode(p, w, index, split_keys);
      if (i >= it.nq) continue;
      const int gm = it.tp * 2 * kM + i * kM + t128;
      const int j = gm / G, g = gm - j * G;
      const bool row_ok = j < it.T;
      const uint32_t* mask_row =
          w.masks + static_cast<int64_t>(it.q_start + (row_ok ? j : 0)) * w.mask_words;
      float m_run = -INFINITY, l_run = 0.f;
      for (int t = 0; t < it.n_tiles; ++t) {
        mbar_wait(bar(kBarSFull + i), sf & 1, abort);
        ++sf;
        tc_fence_after();
        uint32_t sraw[2][32];
        tmem_ld32(tmem + lane_base + col_s(i), sraw[0]);
        tmem_ld32(tmem + lane_base + col_s(i) + 32, sraw[1]);
        tmem_wait_ld();
        const int kb = it.key_begin + t * kN;
        const bool full = kb + kN <= min(it.P, it.key_end);
        float s[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(sraw[c >> 5][c & 31]) * scale_log2;
        if (!full) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int pos = kb + c;
            bool vis = row_ok && pos < it.key_end;
            if (vis && pos >= it.P) {
              const int n = pos - it.P;
              vis = (__ldg(mask_row + (n >> 5)) >> (n & 31)) & 1u;
            }
            if (!vis) s[c] = -INFINITY;
          }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) mx = fmaxf(mx, s[c]);
        // Lazy max: move only when it grows by more than 8 (log2 units).
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_run + 8.f) {
          if (m_run != -INFINITY) {
            alpha = jt::fast_exp2(m_run - mx);
            rescale = true;
          }
          m_run = mx;
        }
        const float m_use = m_run == -INFINITY ? 0.f : m_run;
        float rsum = 0.f;
        uint32_t ph[32];
        uint32_t pl[FP32P ? 32 : 1];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p0 = jt::fast_exp2(s[2 * c] - m_use);
          const float p1 = jt::fast_exp2(s[2 * c + 1] - m_use);
          rsum += p0 + p1;
          ph[c] = Mma::pack(p0, p1);
          if constexpr (FP32P) {
            const float2 r = Mma::unpack(ph[c]);
            pl[c] = Mma::pack(p0 - r.x, p1 - r.y);
          }
        }
        l_run = l_run * alpha + rsum;
        if (t > 0) {
          mbar_wait(bar(kBarODone + i), od & 1, abort);
          ++od;
          tc_fence_after();
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
            for (int chunk = 0; chunk < 4; ++chunk) {
              uint32_t o[32];
              const uint32_t ta = tmem + lane_base + col_o(i) + chunk * 32;
              tmem_ld32(ta, o);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st32(ta, o);
            }
          }
        }
        tmem_st32(tmem + lane_base + col_p(i), ph);
        if constexpr (FP32P) {
          uint32_t lo[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) lo[c] = pl[c];
          tmem_st32(tmem + lane_base + col_pl(i), lo);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(kBarPFull + i));
      }
      // Epilogue: last PV done -> O / l, or an unnormalised partial for split items.
      mbar_wait(bar(kBarODone + i), od & 1, abort);
      ++od;
      tc_fence_after();
      const bool split_item = it.n_split > 1;
      const int64_t slot = it.slot_base +
                           (static_cast<int64_t>(it.h) * it.mblocks + it.tp) * it.n_split + it.split;
      const int item_row = i * kM + t128;
      const float inv = 1.f / l_run;
#pragma unroll 1
      for (int chunk = 0; chunk < 4; ++chunk) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + col_o(i) + chunk * 32, o);
        tmem_wait_ld();
        if (split_item) {
          float4* dst = reinterpret_cast<float4*>(w.part_o + (slot * (2 * kM) + item_row) * kD +
                                                  chunk * 32);
#pragma unroll
          for (int c = 0; c < 8; ++c)
            dst[c] = make_float4(__uint_as_float(o[4 * c]), __uint_as_float(o[4 * c + 1]),
                                 __uint_as_float(o[4 * c + 2]), __uint_as_float(o[4 * c + 3]));
        } else if (row_ok) {
          const int64_t off = static_cast<int64_t>(it.q_start + j) * p.out_stride0 +
                              static_cast<int64_t>(it.h * G + g) * p.out_stride1 + chunk * 32;
          if (p.out_dtype == JT_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off);
#pragma unroll
            for (int c = 0; c < 8; ++c)
              dst[c] = make_float4(__uint_as_float(o[4 * c]) * inv, __uint_as_float(o[4 * c + 1]) * inv,
                                   __uint_as_float(o[4 * c + 2]) * inv,
                                   __uint_as_float(o[4 * c + 3]) * inv);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<Elem*>(p.out) + off);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              dst[c] = make_uint4(
                  Mma::pack(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                  Mma::pack(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                  Mma::pack(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                  Mma::pack(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar(kBarOFree + i));
      if (split_item) {
        w.part_ml[slot * (2 * kM) + item_row] = make_float2(m_run, l_run);
        __threadfence();
        const int barrier_id = it.nq == 2 ? 1 : 3;
        const int members = it.nq * kM;
        named_sync(barrier_id, members);
        // Flag slot by the item's position in this CTA's sequence (same for both tiles).
        volatile int* flag = misc + 2 + (((index - static_cast<int>(blockIdx.x)) /
                                         static_cast<int>(gridDim.x)) & 1);
        if (i == 0 && t128 == 0) {
          int* counter = w.counters + it.counter_base + it.h * it.mblocks + it.tp;
          const int done = atomicAdd(counter, 1);
          const int last = done == it.n_split - 1;
          if (last) *counter = 0;
          *flag = last;
        }
        named_sync(barrier_id, members);
        if (*flag && row_ok) {
          __threadfence();
          const int64_t slot0 =
              it.slot_base + (static_cast<int64_t>(it.h) * it.mblocks + it.tp) * it.n_split;
          float mmax = -INFINITY;
          for (int s2 = 0; s2 < it.n_split; ++s2)
            mmax = fmaxf(mmax, __ldcg(w.part_ml + (slot0 + s2) * (2 * kM) + item_row).x);
          const float mref = mmax == -INFINITY ? 0.f : mmax;
          float den = 0.f;
          for (int s2 = 0; s2 < it.n_split; ++s2) {
            const float2 ml = __ldcg(w.part_ml + (slot0 + s2) * (2 * kM) + item_row);
            den += jt::fast_exp2(ml.x - mref) * ml.y;
          }
          const float dinv = 1.f / den;
          const int64_t off = static_cast<int64_t>(it.q_start + j) * p.out_stride0 +
                              static_cast<int64_t>(it.h * G + g) * p.out_stride1;
          for (int d = 0; d < kD; d += 4) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s2 = 0; s2 < it.n_split; ++s2) {
              const float wv =
                  jt::fast_exp2(__ldcg(w.part_ml + (slot0 + s2) * (2 * kM) + item_row).x - mref);
              const float4 o = __ldcg(reinterpret_cast<const float4*>(
                  w.part_o + ((slot0 + s2) * (2 * kM) + item_row) * kD + d));
              acc.x += wv * o.x;
              acc.y += wv * o.y;
              acc.z += wv * o.z;
              acc.w += wv * o.w;
            }
            if (p.out_dtype == JT_F32) {
              *reinterpret_cast<float4*>(static_cast<float*>(p.out) + off + d) =
                  make_float4(acc.x * dinv, acc.y * dinv, acc.z * dinv, acc.w * dinv);
            } else {
              *reinterpret_cast<uint2*>(static_cast<Elem*>(p.out) + off + d) =
                  make_uint2(Mma::pack(acc.x * dinv, acc.y * dinv), Mma::pack(acc.z * dinv, acc.w * dinv));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem) : "memory");
  }
}

}  // namespace tc
