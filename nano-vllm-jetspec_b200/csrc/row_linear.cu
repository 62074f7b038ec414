// Row-parallel linear with its all-reduce fused in: y = sum over ranks of x_r W_r^T (+ bias).
//
// The reference's RowParallelLinear.forward (nanovllm/layers/linear.py:153-156) runs
// F.linear on this rank's input shard (bias on rank 0 only) and then dist.all_reduce on
// the [M, N] result; the Qwen3 o_proj (qwen3.py:59, :97 ... :302) and down_proj (:334,
// :345) are its callers.  Here one persistent kernel per GPU does both:
//
//   warp 0      TMA producer: x [BM rows x 64 K] and W [256 rows x 64 K] tiles, 128-byte
//               swizzle, into a ring of stages
//   warp 1      tcgen05.mma issuer (kind::f16, M128 N256 K16) and TMEM owner
//
// Two tile shapes.  Tall (one GPU): 256 x 256 output tiles, two MMAs per K step (the two
// 128-row halves of the x tile share each W tile, half the W stream per flop), the fp32
// tile in all 512 TMEM columns, 3 stages of 64 KB.  Short (a group of GPUs): 128 x 256
// tiles, two 256-column accumulators so the epilogue and exchange of one tile overlap the
// MMAs of the next, 4 stages of 48 KB: with twice the tiles, the partial and result
// transfers of the first tiles run while the GEMM of the later ones still does.
//   warps 2-5   epilogue: TMEM -> registers -> bf16/f16 partial tile, stored straight into
//               the tile owner's receive slot (a peer GPU's memory over NVLink, or this
//               GPU's), then a release flag in the owner's memory
//   warps 6-13  exchange: for the tiles this rank owns (tile t belongs to rank t % world)
//               wait for every rank's partial, sum them in fp32, round once, write the
//               tile to this rank's output and into every other rank's inbox, and raise
//               a done flag there; then copy the tiles other ranks own from this rank's
//               inbox into its output as each one is done
//
// A pair of GPUs (world == 2) exchanges in one hop instead: every rank's epilogue stores
// its partial tile into its own and its peer's receive slot (double-buffered by the call's
// epoch parity), and the exchange warps of both ranks sum the two partials of the tiles
// their CTA computed, in rank order, and write their own output: the same bytes cross
// NVLink as with an owner (one partial each way per tile), without the second hop of the
// results, the owner's done flag and the inbox copy.
//
// The all-reduce therefore moves the reduce-scatter + all-gather volume ((world-1)/world of
// the output out and back per rank), tile by tile while the GEMM is still running, and
// without a separate collective launch; every transfer over NVLink is a posted store
// (partials to their owner, results to the inboxes), every load is from this GPU's memory.
// Flags carry the call's epoch (the host increments it per call), so nothing is reset
// between calls; a rank's receive slots and inbox are rewritten only after it finished
// reading them in the previous call (a rank sends its next partial only after leaving the
// previous call, which it does after copying its whole inbox, and an owner pushes a result
// only after every rank's next partial for that tile arrived).  Every wait is
// bounded: a flag that does not arrive within the limit sets JT_DEVERR_TIMEOUT and the
// exchange warps skip the rest of their work.  No load uses cluster multicast.
//
// With world == 1 the epilogue writes the output directly (plain F.linear).  For tests on
// one GPU, one launch can play every rank of a group (jt_row_linear_emulate): its CTAs
// are split between the ranks, each with its own inputs, and the launch is cooperative so
// that all of them are resident at once (a CTA waits only on CTAs of the same launch).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace {

__device__ uint32_t g_rowlin_errors;

namespace rl {

constexpr int kBN = 256, kBK = 64;  // output tile width, K step; MMAs are M128
constexpr int kBTileBytes = kBN * kBK * 2;  // 32 KB
constexpr int kThreads = 448;
constexpr int kExchangeThreads = 256;  // warps 6-13
constexpr int kMaxRanks = 8;
// The tall tile (256 rows) on one GPU, the short one (128 rows) in a group of GPUs.
#ifndef JT_RL_TALL_WORLD_MAX
#define JT_RL_TALL_WORLD_MAX 1
#endif
__host__ __device__ constexpr bool tall_for(int world) { return world <= JT_RL_TALL_WORLD_MAX; }

template <bool kTall>
struct Shape {
  static constexpr int kBM = kTall ? 256 : 128;         // output tile rows
  static constexpr int kStages = kTall ? 3 : 4;
  static constexpr int kAccBufs = kTall ? 1 : 2;        // fp32 accumulators in TMEM
  static constexpr int kATileBytes = kBM * kBK * 2;     // 32 / 16 KB
  static constexpr int kAHalfBytes = kATileBytes / 2;   // rows 128..255 of a tall x tile
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kATileBytes;
  static constexpr int kOffBar = kOffB + kStages * kBTileBytes;
  static constexpr int kOffMisc = kOffBar + 16 * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack
  static constexpr int kTileElems = kBM * kBN;          // elements per partial / result tile
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};
__host__ __device__ constexpr int tile_rows(int world) { return tall_for(world) ? 256 : 128; }
constexpr long long kLocalWaitLimit = 4000000000ll;  // cycles per pipeline wait

// Barriers.
constexpr int kBarFull = 0;       // [stages] TMA bytes
constexpr int kBarEmpty = 4;      // [stages] MMA commit
constexpr int kBarAccFull = 8;    // [accumulators] MMA commit after a tile's last K step
constexpr int kBarAccEmpty = 10;  // [accumulators] 4 epilogue warps
constexpr int kBarDrain = 12;
constexpr int kNumBars = 13;

struct Args {
  int64_t M, N, K;
  int32_t world, ranks_in_launch, base_rank, grid_per_rank;
  int32_t m_tiles, n_tiles, tiles, owned_max;
  uint32_t epoch;
  long long wait_limit;
  const void* bias[kMaxRanks];   // per rank of this launch (nullptr: no bias)
  void* out[kMaxRanks];          // per rank of this launch, [M, N] row-major
  unsigned char* ws[kMaxRanks];  // per rank of the group, as addressable from this GPU
};

// Workspace of one rank: a 256-byte control block (u32 call counter at 0, u32 CTA exit
// counter at 4), [ready: tiles x world u32][done: tiles u32] (256-byte aligned), then the
// receive slots [owned_max][world][tile], then the inbox [tiles][tile] where the owners of
// the other tiles put the reduced results.
// A pair (world == 2) uses receive slots [tiles][epoch parity][world][tile] after the
// flags instead, and no inbox.
constexpr int kCtrlBytes = 256;
#ifndef JT_RL_PAIR_EXCHANGE
#define JT_RL_PAIR_EXCHANGE 1
#endif
__host__ __device__ constexpr bool pair_exchange(int world) {
  return JT_RL_PAIR_EXCHANGE != 0 && world == 2;
}
__host__ __device__ inline int64_t ws_flag_bytes(int tiles, int world) {
  return kCtrlBytes + ((static_cast<int64_t>(tiles) * (world + 1) * 4) + 255) / 256 * 256;
}
__host__ __device__ inline int64_t ws_recv_offset(int tiles, int world) {
  return ws_flag_bytes(tiles, world);
}
__host__ __device__ inline int64_t ws_result_offset(int tiles, int world, int owned_max,
                                                    int tile_elems) {
  return ws_recv_offset(tiles, world) +
         static_cast<int64_t>(owned_max) * world * tile_elems * 2;
}
__host__ __device__ inline int64_t ws_total(int tiles, int world, int owned_max,
                                            int tile_elems) {
  if (pair_exchange(world))
    return ws_recv_offset(tiles, world) + static_cast<int64_t>(tiles) * 2 * world * tile_elems * 2;
  return ws_result_offset(tiles, world, owned_max, tile_elems) +
         static_cast<int64_t>(tiles) * tile_elems * 2;
}
// Receive slot of (tile, source rank) in a pair's workspace for the call's epoch parity.
__host__ __device__ inline int64_t ws_pair_slot(int tiles, int world, int t, uint32_t epoch,
                                                int src, int tile_elems) {
  return ws_recv_offset(tiles, world) +
         ((static_cast<int64_t>(t) * 2 + (epoch & 1u)) * world + src) * tile_elems * 2;
}

// ---- PTX wrappers --------------------------------------------------------------------
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
// Bounded wait for the phase with the given parity; a wait that runs out flags a timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const long long start = clock64();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (clock64() - start > kLocalWaitLimit) {
      atomicOr(&g_rowlin_errors, JT_DEVERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_commit_warp(uint32_t bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(
          bar)
      : "memory");
}
__device__ __forceinline__ void mma_ss_warp(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// K-major operand in shared memory with the 128-byte swizzle: rows of 128 B, 8-row groups
// 1024 B apart (descriptor version 1 for sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(16u >> 4) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}
// kind::f16 instruction descriptor, fp32 accumulate, both operands K-major.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
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
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
// Flags shared with other GPUs: release stores, acquire loads at system scope.
__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
// Bounded wait until a flag reaches the epoch (flags only grow; a difference below 2^31
// counts as reached).  Returns false, and flags a timeout, when the limit runs out or an
// earlier wait of this CTA already did.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t epoch, long long limit,
                                          volatile int* abort) {
  if (static_cast<int>(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const long long start = clock64();
  for (;;) {
    if (static_cast<int>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if (*abort) return false;
    if (clock64() - start > limit) {
      *abort = 1;
      atomicOr(&g_rowlin_errors, JT_DEVERR_TIMEOUT);
      return false;
    }
  }
}

template <bool kBf16>
struct Conv;
template <>
struct Conv<true> {
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static float2 unpack(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
  }
};
template <>
struct Conv<false> {
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static float2 unpack(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2*>(&v));
  }
};

}  // namespace rl

namespace rl {

struct Maps {
  CUtensorMap x[kMaxRanks];  // [M, K] input shard of each rank of this launch
  CUtensorMap w[kMaxRanks];  // [N, K] weight shard of each rank of this launch
};

__device__ __forceinline__ uint32_t* ready_flags(unsigned char* ws) {
  return reinterpret_cast<uint32_t*>(ws + kCtrlBytes);
}
__device__ __forceinline__ uint32_t* done_flags(unsigned char* ws, int tiles, int world) {
  return ready_flags(ws) + static_cast<int64_t>(tiles) * world;
}

// 16-byte chunk `ch` (0..8191 of a tall tile, 0..4095 of a short one) of a partial /
// result tile: chunks are stored so that the 32 lanes of an epilogue warp write 512
// contiguous bytes (one row per lane, 8 columns per chunk); this maps a chunk back to its
// row and first column inside the tile (chunk = half * 4096 + quadrant * 1024 + column
// group * 128 + i * 32 + lane; a short tile has only half 0).
__device__ __forceinline__ void chunk_coords(int ch, int& row, int& col) {
  const int lane = ch & 31, i = (ch >> 5) & 3, c = (ch >> 7) & 7, q = (ch >> 10) & 3;
  row = (ch >> 12) * 128 + q * 32 + lane;
  col = c * 32 + i * 8;
}

template <bool kBf16, bool kTall>
__global__ void __launch_bounds__(kThreads, 1)
    row_linear_kernel(const __grid_constant__ Args a, const __grid_constant__ Maps maps) {
  using Cv = Conv<kBf16>;
  using S = Shape<kTall>;
  constexpr int kBM = S::kBM, kStages = S::kStages, kTileElems = S::kTileElems;
  constexpr int kATileBytes = S::kATileBytes, kOffA = S::kOffA, kOffB = S::kOffB;
  constexpr uint32_t kIdesc = instr_desc(128, kBN, kBf16);  // one 128-row block per MMA
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = jt::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + S::kOffBar;
#define RL_BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))
  volatile int* misc = reinterpret_cast<volatile int*>(sbase + S::kOffMisc);
  volatile int* abort = misc + 1;  // misc[0]: TMEM base
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lr = blockIdx.x % a.ranks_in_launch;  // rank of this launch the CTA works for
  const int cta = blockIdx.x / a.ranks_in_launch;
  const int rank = a.base_rank + lr;
  const int world = a.world;
  const int k_blocks = static_cast<int>((a.K + kBK - 1) / kBK);

  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(RL_BAR(i), (i == kBarAccEmpty || i == kBarAccEmpty + 1) ? 4u : 1u);
    misc[1] = 0;
    // The call's epoch: given by the host, or (0) one past this rank's call counter, which
    // the last CTA of the previous call advanced (stream order makes it visible here).
    misc[2] = static_cast<int>(
        a.epoch != 0 || world == 1
            ? a.epoch
            : *reinterpret_cast<volatile uint32_t*>(a.ws[rank]) + 1u);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(
                     base + S::kOffMisc)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = static_cast<uint32_t>(misc[0]);
  const uint32_t epoch = static_cast<uint32_t>(misc[2]);

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t r = 0;
      for (int t = cta; t < a.tiles; t += a.grid_per_rank) {
        const int m0 = (t % a.m_tiles) * kBM, n0 = (t / a.m_tiles) * kBN;
        for (int kb = 0; kb < k_blocks; ++kb, ++r) {
          const int s = static_cast<int>(r % kStages);
          mbar_wait(RL_BAR(kBarEmpty + s), ((r / kStages) & 1u) ^ 1u);
          mbar_arrive_tx(RL_BAR(kBarFull + s), S::kStageBytes);
          tma_load_2d(base + kOffA + s * kATileBytes, &maps.x[lr], kb * kBK, m0,
                      RL_BAR(kBarFull + s));
          tma_load_2d(base + kOffB + s * kBTileBytes, &maps.w[lr], kb * kBK, n0,
                      RL_BAR(kBarFull + s));
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    uint32_t r = 0, acc = 0;
    const uint64_t adesc0 = smem_desc(base + kOffA), bdesc0 = smem_desc(base + kOffB);
    for (int t = cta; t < a.tiles; t += a.grid_per_rank, ++acc) {
      // An accumulator is free once the epilogue read it (tall: the one 512-column
      // accumulator; short: accumulators alternate, 256 columns each).
      const uint32_t buf = kTall ? 0u : (acc & 1u), use = kTall ? acc : (acc >> 1);
      mbar_wait(RL_BAR(kBarAccEmpty + buf), (use & 1u) ^ 1u);
      tc_fence_after();
      const uint32_t d = tmem + buf * static_cast<uint32_t>(kBN);
      for (int kb = 0; kb < k_blocks; ++kb, ++r) {
        const int s = static_cast<int>(r % kStages);
        mbar_wait(RL_BAR(kBarFull + s), (r / kStages) & 1u);
        tc_fence_after();
        const uint64_t ad = adesc0 + static_cast<uint64_t>((s * kATileBytes) >> 4);
        const uint64_t bd = bdesc0 + static_cast<uint64_t>((s * kBTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {  // 16 K elements = 32 bytes along the row
          const uint32_t accumulate = (kb > 0 || kk > 0) ? 1u : 0u;
          mma_ss_warp(d, ad + 2 * kk, bd + 2 * kk, kIdesc, accumulate);
          if constexpr (kTall)
            mma_ss_warp(tmem + static_cast<uint32_t>(kBN), ad + (S::kAHalfBytes >> 4) + 2 * kk,
                        bd + 2 * kk, kIdesc, accumulate);
        }
        tc_commit_warp(RL_BAR(kBarEmpty + s));
      }
      tc_commit_warp(RL_BAR(kBarAccFull + buf));
    }
    // Drain: every MMA this warp issued has completed before TMEM is released.
    tc_commit_warp(RL_BAR(kBarDrain));
    mbar_wait(RL_BAR(kBarDrain), 0);
  } else if (warp < 6) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may read
    const uint16_t* bias = static_cast<const uint16_t*>(a.bias[lr]);
    uint32_t acc = 0;
    for (int t = cta; t < a.tiles; t += a.grid_per_rank, ++acc) {
      const int m0 = (t % a.m_tiles) * kBM, n0 = (t / a.m_tiles) * kBN;
      const int owner = t % world, j = t / world;
      const uint32_t buf = kTall ? 0u : (acc & 1u), use = kTall ? acc : (acc >> 1);
      mbar_wait(RL_BAR(kBarAccFull + buf), use & 1u);
      tc_fence_after();
      const bool pair = pair_exchange(world);
      unsigned char* slot = nullptr;
      unsigned char* slot_peer = nullptr;
      if (pair) {
        const int64_t off = ws_pair_slot(a.tiles, world, t, epoch, rank, kTileElems);
        slot = a.ws[rank] + off;
        slot_peer = a.ws[rank ^ 1] + off;
      } else if (world > 1) {
        slot = a.ws[owner] + ws_recv_offset(a.tiles, world) +
               (static_cast<int64_t>(j) * world + rank) * kTileElems * 2;
      }
#pragma unroll 1
      for (int hc = 0; hc < (kBM / 128) * (kBN / 32); ++hc) {  // (half, 32-column group)
        const int h = hc >> 3, c = hc & 7;
        const int64_t m = m0 + h * 128 + q * 32 + lane;
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) +
                      static_cast<uint32_t>((h + static_cast<int>(buf)) * kBN + c * 32),
                  v);
        tmem_wait_ld();
        const int64_t n = n0 + c * 32;
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float lo = __uint_as_float(v[2 * i]), hi = __uint_as_float(v[2 * i + 1]);
          if (bias != nullptr && n < a.N) {
            const float2 b = Cv::unpack(*reinterpret_cast<const uint32_t*>(bias + n + 2 * i));
            lo += b.x;
            hi += b.y;
          }
          packed[i] = Cv::pack(lo, hi);
        }
        if (world == 1) {
          if (m < a.M && n < a.N) {
            uint4* o = reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.out[lr]) +
                                                (m * a.N + n) * 2);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              o[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                packed[4 * i + 3]);
          }
        } else {
          const int64_t ch0 = h * 4096 + (q * 8 + c) * 128 + lane;
          uint4* o = reinterpret_cast<uint4*>(slot) + ch0;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[32 * i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                   packed[4 * i + 3]);
          if (pair) {
            uint4* op = reinterpret_cast<uint4*>(slot_peer) + ch0;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              op[32 * i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                      packed[4 * i + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(RL_BAR(kBarAccEmpty + buf));
      if (world > 1) {
        // Every epilogue thread's stores of this partial are visible system-wide before
        // the owner's ready flag for (tile, this rank) is raised.
        __threadfence_system();
        named_sync(2, 128);
        if (pair) {
          if ((warp == 2 || warp == 3) && lane == 0)
            st_release_sys(ready_flags(a.ws[rank ^ (warp - 2)]) +
                               static_cast<int64_t>(t) * world + rank,
                           epoch);
        } else if (warp == 2 && lane == 0) {
          st_release_sys(ready_flags(a.ws[owner]) + static_cast<int64_t>(t) * world + rank,
                         epoch);
        }
      }
    }
  } else if (pair_exchange(world)) {
    // ---------------------------------------------------------------- pair exchange
    // The tiles this CTA computed: wait for both partials, sum them in rank order (the
    // same order, hence the same bits, on both ranks), write this rank's output.
    const int et = tid - 192;  // 0..255
    unsigned char* mine = a.ws[rank];
    for (int t = cta; t < a.tiles; t += a.grid_per_rank) {
      if (et < world)
        wait_flag(ready_flags(mine) + static_cast<int64_t>(t) * world + et, epoch,
                  a.wait_limit, abort);
      named_sync(1, kExchangeThreads);
      if (*abort) continue;
      const int m0 = (t % a.m_tiles) * kBM, n0 = (t / a.m_tiles) * kBN;
      const uint4* slots = reinterpret_cast<const uint4*>(
          mine + ws_pair_slot(a.tiles, world, t, epoch, 0, kTileElems));
#pragma unroll 1
      for (int c0 = et; c0 < kTileElems / 8; c0 += 4 * kExchangeThreads) {
        uint4 in0[4], in1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          in0[u] = __ldcg(slots + c0 + kExchangeThreads * u);
          in1[u] = __ldcg(slots + kTileElems / 8 + c0 + kExchangeThreads * u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t w0[4] = {in0[u].x, in0[u].y, in0[u].z, in0[u].w};
          const uint32_t w1[4] = {in1[u].x, in1[u].y, in1[u].z, in1[u].w};
          uint32_t r4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f0 = Cv::unpack(w0[e]), f1 = Cv::unpack(w1[e]);
            r4[e] = Cv::pack(f0.x + f1.x, f0.y + f1.y);
          }
          int row, col;
          chunk_coords(c0 + kExchangeThreads * u, row, col);
          const int64_t m = m0 + row, n = n0 + col;
          if (m < a.M && n < a.N)
            *reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.out[lr]) +
                                      (m * a.N + n) * 2) = make_uint4(r4[0], r4[1], r4[2], r4[3]);
        }
      }
    }
  } else if (world > 1) {
    // ---------------------------------------------------------------- exchange
    const int et = tid - 192;  // 0..255
    unsigned char* mine = a.ws[rank];
    const int64_t inbox_off = ws_result_offset(a.tiles, world, a.owned_max, kTileElems);
    const int owned = (a.tiles - rank + world - 1) / world;  // tiles j * world + rank
    for (int j = cta; j < owned; j += a.grid_per_rank) {
      const int t = j * world + rank;
      if (et < world)
        wait_flag(ready_flags(mine) + static_cast<int64_t>(t) * world + et, epoch,
                  a.wait_limit, abort);
      named_sync(1, kExchangeThreads);
      if (!*abort) {
        const int m0 = (t % a.m_tiles) * kBM, n0 = (t / a.m_tiles) * kBN;
        const uint4* slots = reinterpret_cast<const uint4*>(
            mine + ws_recv_offset(a.tiles, world) +
            static_cast<int64_t>(j) * world * kTileElems * 2);
        const int64_t inbox_tile = inbox_off + static_cast<int64_t>(t) * kTileElems * 2;
#pragma unroll 1
        for (int c0 = et; c0 < kTileElems / 8; c0 += 4 * kExchangeThreads) {
          float sum[4][8];
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int e = 0; e < 8; ++e) sum[u][e] = 0.f;
#pragma unroll 2
          for (int s = 0; s < world; ++s) {
            uint4 in[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              in[u] = __ldcg(slots + static_cast<int64_t>(s) * (kTileElems / 8) + c0 +
                             kExchangeThreads * u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint32_t w4[4] = {in[u].x, in[u].y, in[u].z, in[u].w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = Cv::unpack(w4[e]);
                sum[u][2 * e] += f.x;
                sum[u][2 * e + 1] += f.y;
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int ch = c0 + kExchangeThreads * u;
            const uint4 o = make_uint4(Cv::pack(sum[u][0], sum[u][1]), Cv::pack(sum[u][2], sum[u][3]),
                                       Cv::pack(sum[u][4], sum[u][5]), Cv::pack(sum[u][6], sum[u][7]));
            for (int r = 0; r < world; ++r)  // posted stores into the other ranks' inboxes
              if (r != rank) reinterpret_cast<uint4*>(a.ws[r] + inbox_tile)[ch] = o;
            int row, col;
            chunk_coords(ch, row, col);
            const int64_t m = m0 + row, n = n0 + col;
            if (m < a.M && n < a.N)
              *reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.out[lr]) +
                                        (m * a.N + n) * 2) = o;
          }
        }
      }
      __threadfence_system();
      named_sync(1, kExchangeThreads);
      if (et < world && et != rank && !*abort)
        st_release_sys(done_flags(a.ws[et], a.tiles, world) + t, epoch);
    }
    // Tiles other ranks own: copy each from this rank's inbox once its owner is done.
    uint32_t* done = done_flags(mine, a.tiles, world);
    for (int t = cta; t < a.tiles; t += a.grid_per_rank) {
      const int owner = t % world;
      if (owner == rank) continue;
      if (et == 0) wait_flag(done + t, epoch, a.wait_limit, abort);
      named_sync(1, kExchangeThreads);
      if (*abort) continue;
      const int m0 = (t % a.m_tiles) * kBM, n0 = (t / a.m_tiles) * kBN;
      const uint4* src =
          reinterpret_cast<const uint4*>(mine + inbox_off + static_cast<int64_t>(t) * kTileElems * 2);
#pragma unroll 1
      for (int c0 = et; c0 < kTileElems / 8; c0 += 8 * kExchangeThreads) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldcg(src + c0 + kExchangeThreads * u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          int row, col;
          chunk_coords(c0 + kExchangeThreads * u, row, col);
          const int64_t m = m0 + row, n = n0 + col;
          if (m < a.M && n < a.N)
            *reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.out[lr]) +
                                      (m * a.N + n) * 2) = v[u];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem)
                 : "memory");
  }
  if (tid == 0 && world > 1 && a.epoch == 0) {
    // Every CTA of this rank read the counter at its start; the last one to leave
    // advances it for the next call.
    uint32_t* ctrl = reinterpret_cast<uint32_t*>(a.ws[rank]);
    __threadfence();
    if (atomicAdd(ctrl + 1, 1u) == static_cast<uint32_t>(a.grid_per_rank - 1)) {
      atomicExch(ctrl + 1, 0u);
      __threadfence();
      atomicAdd(ctrl, 1u);
    }
  }
#undef RL_BAR
}

}  // namespace rl

PFN_cuTensorMapEncodeTiled_v12000 rl_tensor_map_encoder() {
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

// 2-D K-major map [rows, cols] (row stride in elements) with a 64-column x box_rows box and
// the 128-byte swizzle; elements outside the matrix read as zero.
bool encode_kmajor(CUtensorMap* map, const void* ptr, int32_t dtype, int64_t rows, int64_t cols,
                   int64_t row_stride, int box_rows) {
  auto encode = rl_tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(rl::kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map,
                dtype == JT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                2, const_cast<void*>(ptr), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int rl_tiles(int64_t m, int64_t n, int bm, int* m_tiles, int* n_tiles) {
  const int64_t mt = (m + bm - 1) / bm, nt = (n + rl::kBN - 1) / rl::kBN;
  if (mt * nt > (1ll << 30)) return jt_fail(JT_ERR_INVALID, "row_linear: output too large");
  *m_tiles = static_cast<int>(mt);
  *n_tiles = static_cast<int>(nt);
  return JT_OK;
}

// Checks one rank's call (every check the kernel relies on) and encodes its maps.
int rl_check_rank(const JtRowLinearParams& p, CUtensorMap* xmap, CUtensorMap* wmap) {
  if (p.dtype != JT_BF16 && p.dtype != JT_F16)
    return jt_fail(JT_ERR_INVALID, "row_linear: dtype must be bf16 or f16");
  if (p.m < 1 || p.n < 32 || p.n % 32 != 0 || p.k < 8 || p.k % 8 != 0)
    return jt_fail(JT_ERR_INVALID,
                   "row_linear: need m >= 1, n a positive multiple of 32, k a positive multiple "
                   "of 8 (m=%lld n=%lld k=%lld)",
                   static_cast<long long>(p.m), static_cast<long long>(p.n),
                   static_cast<long long>(p.k));
  if (p.world < 1 || p.world > rl::kMaxRanks || p.rank < 0 || p.rank >= p.world)
    return jt_fail(JT_ERR_INVALID, "row_linear: rank %d of world %d (1 <= world <= 8)", p.rank,
                   p.world);
  if (!p.x || !p.weight || !p.out)
    return jt_fail(JT_ERR_INVALID, "row_linear: null x / weight / out");
  if (!al16(p.x) || !al16(p.weight) || !al16(p.out) || (p.bias && (reinterpret_cast<uintptr_t>(p.bias) & 3u)))
    return jt_fail(JT_ERR_INVALID, "row_linear: x, weight and out need 16-byte alignment");
  if (p.x_stride < p.k || p.x_stride % 8 != 0 || p.w_stride < p.k || p.w_stride % 8 != 0)
    return jt_fail(JT_ERR_INVALID,
                   "row_linear: row strides must be >= k and multiples of 8 elements");
  if (p.world > 1) {
    if (p.workspaces == nullptr)
      return jt_fail(JT_ERR_INVALID, "row_linear: world > 1 needs the ranks' workspaces");
    for (int r = 0; r < p.world; ++r)
      if (p.workspaces[r] == nullptr || (reinterpret_cast<uintptr_t>(p.workspaces[r]) & 255u))
        return jt_fail(JT_ERR_INVALID, "row_linear: workspace %d null or not 256-byte aligned", r);
  }
  if (!encode_kmajor(xmap, p.x, p.dtype, p.m, p.k, p.x_stride, rl::tile_rows(p.world)) ||
      !encode_kmajor(wmap, p.weight, p.dtype, p.n, p.k, p.w_stride, rl::kBN))
    return jt_fail(JT_ERR_CUDA, "row_linear: cuTensorMapEncodeTiled rejected x or weight");
  return JT_OK;
}

// ranks[0..count) are the ranks this launch plays (count 1, or the whole group).
int rl_launch(const JtRowLinearParams* ranks, int count, cudaStream_t stream) {
  const JtRowLinearParams& p0 = ranks[0];
  rl::Args a{};
  rl::Maps maps{};
  for (int i = 0; i < count; ++i) {
    const JtRowLinearParams& p = ranks[i];
    int rc = rl_check_rank(p, &maps.x[i], &maps.w[i]);
    if (rc != JT_OK) return rc;
    if (i > 0 && (p.m != p0.m || p.n != p0.n || p.k != p0.k || p.dtype != p0.dtype ||
                  p.world != p0.world || p.epoch != p0.epoch || p.rank != p0.rank + i))
      return jt_fail(JT_ERR_INVALID, "row_linear: emulated ranks must share the geometry and "
                                     "be given in rank order");
    a.bias[i] = p.rank == 0 ? p.bias : nullptr;  // the bias is added once, by rank 0
    a.out[i] = p.out;
  }
  int m_tiles = 0, n_tiles = 0;
  const bool tall = rl::tall_for(p0.world);
  int rc = rl_tiles(p0.m, p0.n, rl::tile_rows(p0.world), &m_tiles, &n_tiles);
  if (rc != JT_OK) return rc;
  a.M = p0.m;
  a.N = p0.n;
  a.K = p0.k;
  a.world = p0.world;
  a.ranks_in_launch = count;
  a.base_rank = p0.rank;
  a.m_tiles = m_tiles;
  a.n_tiles = n_tiles;
  a.tiles = m_tiles * n_tiles;
  a.owned_max = (a.tiles + a.world - 1) / a.world;
  a.epoch = p0.epoch;
  a.wait_limit = p0.wait_limit_cycles > 0 ? p0.wait_limit_cycles : 20000000000ll;
  for (int r = 0; r < p0.world && p0.world > 1; ++r)
    a.ws[r] = static_cast<unsigned char*>(p0.workspaces[r]);
  // Per-device facts, looked up once: the SM count and the kernels' shared-memory opt-in.
  static int sm_count[64] = {0};
  int dev = 0;
  rc = jt_cuda_check(cudaGetDevice(&dev), "row_linear: device");
  if (rc != JT_OK) return rc;
  if (dev < 0 || dev >= 64) return jt_fail(JT_ERR_INVALID, "row_linear: device index");
  const bool bf16 = p0.dtype == JT_BF16;
  auto kernel = tall ? (bf16 ? rl::row_linear_kernel<true, true> : rl::row_linear_kernel<false, true>)
                     : (bf16 ? rl::row_linear_kernel<true, false> : rl::row_linear_kernel<false, false>);
  const int smem = tall ? rl::Shape<true>::kSmemBytes : rl::Shape<false>::kSmemBytes;
  if (sm_count[dev] == 0) {
    int sms = 0;
    rc = jt_cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                       "row_linear: SM count");
    if (rc != JT_OK) return rc;
    for (auto k : {rl::row_linear_kernel<true, true>, rl::row_linear_kernel<false, true>}) {
      rc = jt_cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              rl::Shape<true>::kSmemBytes),
                         "row_linear: smem attribute");
      if (rc != JT_OK) return rc;
    }
    for (auto k : {rl::row_linear_kernel<true, false>, rl::row_linear_kernel<false, false>}) {
      rc = jt_cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              rl::Shape<false>::kSmemBytes),
                         "row_linear: smem attribute");
      if (rc != JT_OK) return rc;
    }
    sm_count[dev] = sms;
  }
  const int sms = sm_count[dev];
  if (sms < count) return jt_fail(JT_ERR_INVALID, "row_linear: more ranks than SMs");
  a.grid_per_rank = std::min(a.tiles, sms / count);
  // Cooperative: every CTA is resident at once (an exchange warp waits on other CTAs).
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(a.grid_per_rank * count));
  cfg.blockDim = dim3(rl::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return jt_cuda_check(cudaLaunchKernelEx(&cfg, kernel, a, maps), "row_linear launch");
}

}  // namespace

int jt_read_errors_rowlin(uint32_t* bits) {
  uint32_t zero = 0;
  int rc = jt_cuda_check(cudaMemcpyFromSymbol(bits, g_rowlin_errors, sizeof(uint32_t)),
                         "read row_linear error word");
  if (rc != JT_OK) return rc;
  return jt_cuda_check(cudaMemcpyToSymbol(g_rowlin_errors, &zero, sizeof(uint32_t)),
                       "clear row_linear error word");
}

extern "C" int64_t jt_row_linear_workspace_size(int64_t m, int64_t n, int32_t world) {
  if (m < 1 || n < 1 || world < 1 || world > rl::kMaxRanks) return -1;
  if (world == 1) return 0;
  int m_tiles = 0, n_tiles = 0;
  const int bm = rl::tile_rows(world);
  if (rl_tiles(m, n, bm, &m_tiles, &n_tiles) != JT_OK) return -1;
  const int tiles = m_tiles * n_tiles;
  return rl::ws_total(tiles, world, (tiles + world - 1) / world, bm * rl::kBN);
}

extern "C" int jt_row_linear_launch(const JtRowLinearParams* p, cudaStream_t stream) {
  if (p == nullptr) return jt_fail(JT_ERR_INVALID, "row_linear: null params");
  return rl_launch(p, 1, stream);
}

extern "C" int jt_row_linear_emulate(const JtRowLinearParams* ranks, int32_t count,
                                     cudaStream_t stream) {
  if (ranks == nullptr || count < 1 || count > rl::kMaxRanks)
    return jt_fail(JT_ERR_INVALID, "row_linear_emulate: 1..8 rank params");
  if (ranks[0].rank != 0 || ranks[0].world != count)
    return jt_fail(JT_ERR_INVALID, "row_linear_emulate: give every rank of the group, rank 0 first");
  return rl_launch(ranks, count, stream);
}

extern "C" int jt_device_alloc_zeroed(int64_t bytes, void** ptr) {
  if (ptr == nullptr || bytes < 1) return jt_fail(JT_ERR_INVALID, "device_alloc: bad arguments");
  *ptr = nullptr;
  int rc = jt_cuda_check(cudaMalloc(ptr, static_cast<size_t>(bytes)), "device_alloc");
  if (rc != JT_OK) return rc;
  rc = jt_cuda_check(cudaMemset(*ptr, 0, static_cast<size_t>(bytes)), "device_alloc: zero");
  if (rc != JT_OK) {
    cudaFree(*ptr);
    *ptr = nullptr;
  }
  return rc;
}

extern "C" int jt_device_free(void* ptr) {
  return jt_cuda_check(cudaFree(ptr), "device_free");
}

extern "C" int jt_ipc_get_handle(const void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) return jt_fail(JT_ERR_INVALID, "ipc_get_handle: null");
  cudaIpcMemHandle_t h;
  int rc = jt_cuda_check(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "ipc_get_handle");
  if (rc != JT_OK) return rc;
  memcpy(handle, &h, sizeof(h));
  return JT_OK;
}

extern "C" int jt_ipc_open_handle(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return jt_fail(JT_ERR_INVALID, "ipc_open_handle: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return jt_cuda_check(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                       "ipc_open_handle");
}

extern "C" int jt_ipc_close_handle(void* ptr) {
  return jt_cuda_check(cudaIpcCloseMemHandle(ptr), "ipc_close_handle");
}
