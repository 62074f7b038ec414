// Blackwell (sm_100a) tree-attention core: tcgen05 tensor cores with TMEM accumulators.
//
// Included by tree_attn.cu inside its anonymous namespace (uses DevLayout, the plan's
// work items and g_attn_errors).  One persistent CTA per SM pulls work items from the
// device plan's queue (longest first).  An item is one 128-row query tile (128/groups
// tree nodes x groups query heads) of one (request, KV head, key split), streamed against
// 128-key K/V tiles.  The query tiles of one request and KV head are adjacent in the
// queue, so CTAs on neighbouring SMs stream the same K/V tiles at about the same time and
// all but the first read them from L2.  Warp roles:
//
//   warp 0       MMA issuer (one thread) and TMEM owner (512 columns)
//   warps 1-3    loaders: TMA for the query tile and for prefix K/V tiles (128 keys inside
//                one page, 128-byte swizzle), cp.async for tiles that touch the tree
//                nodes (scattered scratch slots), written in the same swizzled layout
//   warps 4-11   softmax + epilogue: warpgroup c (warps 4+4c..7+4c) owns keys 64c..64c+63
//                of every key tile and output columns 64c..64c+63; thread t owns score
//                row t (its TMEM lane)
//
// TMEM holds O (128 columns) and three S buffers (128 columns each).  Per key tile t:
// S = Q K_t^T (tcgen05.mma M128 N128 K16, both operands in shared memory) into buffer
// t % 3; the softmax reads its half of S, swaps half-row maxima with the other warpgroup,
// and writes P (rounded to the operand type) over the S columns it read; O += P V_t
// (tcgen05.mma with A from TMEM, V MN-major in shared memory).  With three S buffers the
// QKs run up to three tiles ahead of the softmax, which therefore never waits for the
// tensor core; it only waits for the previous PV before it rescales O, and the running
// max moves (O rescaled in TMEM) only when it grows by more than 2^8, so P stays <= 256
// and rescales are rare.  K and V tiles share one five-slot ring filled in the MMA's
// consumption order.
//
// Every mbarrier wait is bounded and every waiter consumes every phase of the barriers it
// waits on, in order (parity waits are unambiguous only within one phase), except the
// softmax's waits on the per-buffer PV barriers, which it takes only before a rescale and
// at the epilogue; the argument that each of those waits is exactly one phase behind sits
// beside it.  A wait that
// runs out sets JT_DEVERR_TIMEOUT and an abort flag; all roles then leave their loops,
// drain their own asynchronous copies and MMAs, and the CTA frees its TMEM and exits.

namespace tc {

constexpr int kN = 128;       // keys per KV tile
constexpr int kD = 128;       // head dim
constexpr int kM = 128;       // rows per query tile (MMA M)
constexpr int kRing = 5;      // K/V ring slots (32 KB each), filled in consumption order
constexpr int kSBufs = 3;     // S buffers in TMEM
constexpr int kAhead = 3;     // QKs issued ahead of the PVs (= kSBufs)
constexpr int kThreads = 384;
constexpr int kQTileBytes = kM * kD * 2;   // 32 KB: two 64-dim halves of [128 rows][128 B]
constexpr int kQHalfBytes = kM * 128;
constexpr int kKVBytes = kN * kD * 2;      // 32 KB: two 64-dim halves of [128 keys][128 B]
constexpr int kKVHalfBytes = kN * 128;
constexpr int kOffQ = 0;
constexpr int kOffRing = kOffQ + kQTileBytes;
constexpr int kOffBar = kOffRing + kRing * kKVBytes;
constexpr int kOffMisc = kOffBar + 8 * 32;
constexpr int kOffXl = kOffMisc + 64;                   // [2 halves][128] row sums
constexpr int kOffXm = kOffXl + 2 * kM * 4;             // [tile parity][2 halves][128] maxima
constexpr int kOffItem = kOffXm + 4 * kM * 4;           // [2] decoded work items (16 ints)
constexpr int kMaskWordsMax = 32;                       // tree nodes per request <= 1024
constexpr int kOffMask = kOffItem + 2 * 64;             // single-launch mode: the item's
                                                        // ancestor bitmasks [128][32] words
constexpr int kSmemBytes = kOffMask + kM * kMaskWordsMax * 4 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
constexpr long long kWaitLimit = 4000000000ll;          // cycles (~2 s) per wait

// TMEM column map (512 columns x 128 lanes x 32 bit): O, then the S buffers.
__host__ __device__ constexpr uint32_t col_o() { return 0u; }
__host__ __device__ constexpr uint32_t col_s(int b) { return 128u + 128u * b; }
// P of keys 16kk..16kk+15 (operand-type pairs, 8 columns) inside an S buffer: each softmax
// warpgroup writes the probabilities of its 64 keys inside the S columns it owns (keys
// 0..63 -> columns 0..31, keys 64..127 -> columns 64..95); fp32-probability low parts
// follow 32 columns later.
__host__ __device__ constexpr uint32_t col_p(int kk) {
  return kk < 4 ? 8u * kk : 64u + 8u * (kk - 4);
}

// Barrier indices.
constexpr int kBarFull = 0;                    // [kRing]  loader warps (+ TMA bytes)
constexpr int kBarEmpty = 5;                   // [kRing]  MMA commit after the slot's MMAs
constexpr int kBarQFull = 10;                  // loader thread 0 (+ TMA bytes)
constexpr int kBarQEmpty = 11;                 // MMA commit after an item's last QK
constexpr int kBarSFull = 12;                  // [kSBufs] MMA commit per QK
constexpr int kBarPFull = 15;                  // [kSBufs] 8 softmax warps
constexpr int kBarPvDone = 18;                 // [kSBufs] MMA commit per PV (by P's S buffer)
constexpr int kBarOFree = 21;                  // 8 softmax warps after the epilogue
constexpr int kBarMx = 22;                     // 8 softmax warps: half maxima swapped
constexpr int kBarLx = 23;                     // 8 softmax warps: half row sums swapped
constexpr int kSoftmaxWarps = 8;
constexpr int kBarDrain = 24;
constexpr int kBarItemFull = 25;               // [2] work-item ring
constexpr int kBarItemEmpty = 27;              // [2]
constexpr int kNumBars = 29;
constexpr int kItemConsumers = 12;             // every warp of the CTA reads each item
constexpr int kGatherThreads = 64;             // warps 2-3: cp.async tree tiles
constexpr int kFullArrivals = 2;               // per ring fill: TMA (arrive_tx + arrive) or
                                               // one arrival per gather warp
static_assert(kNumBars * 8 <= 8 * 32, "barrier area");

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
                                          bool abortable = true,
                                          long long limit = kWaitLimit) {
  if (mbar_try(bar, parity)) return true;
  const long long start = clock64();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (abortable && *abort) return false;
    if (clock64() - start > limit) {
      *abort = 1;
      atomicOr(&g_attn_errors, JT_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// Warp-wide arrival: the lanes synchronise (bar.warp.sync orders their earlier memory and
// tcgen05-fenced operations before lane 0's arrival), then lane 0 arrives for the warp.
__device__ __forceinline__ void warp_arrive(uint32_t bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}
// Warp-wide wait: every lane polls the phase itself (no divergent branch to reconverge).
__device__ __forceinline__ void warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  mbar_wait(bar, parity, abort);
  __syncwarp();
}

// Release store / bounded acquire wait on a shared-memory position counter.
__device__ __forceinline__ void st_release_shared(uint32_t addr, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_shared(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
// Waits until the counter reaches `target` (counters only grow; a difference of less than
// 2^31 counts as reached).  Bounded like the mbarrier waits.
__device__ __forceinline__ bool wait_shared_at_least(uint32_t addr, uint32_t target,
                                                     volatile int* abort) {
  if (static_cast<int>(ld_acquire_shared(addr) - target) >= 0) return true;
  const long long start = clock64();
  for (;;) {
    if (static_cast<int>(ld_acquire_shared(addr) - target) >= 0) return true;
    if (*abort) return false;
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

// Warp-wide forms: every lane of the warp executes them with identical operands and
// elect.sync picks one lane (always the same one for a fully active warp) to issue, so the
// operands stay warp-uniform and the issuing lane is the one whose MMAs each commit tracks.
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
__device__ __forceinline__ void mma_ts_warp(uint32_t d, uint32_t a_tmem, uint64_t b,
                                            uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
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
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                 "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(
                   taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
               "r"(v[7]));
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

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// Byte offset of 16-byte chunk `chunk` (0..15 over 128 dims) of row `row` in a tile made
// of two 64-dim halves of `rows` x 128 B, with the 128-byte swizzle the MMA expects.
__device__ __forceinline__ uint32_t swz128(int row, int chunk, int rows) {
  const int half = chunk >> 3, c = chunk & 7;
  return static_cast<uint32_t>(half * rows * 128 + row * 128 + ((c ^ (row & 7)) << 4));
}

// Visibility of the 32 keys at positions p0..p0+31 for one score row: bit b is set when
// position p0+b is a prefix key, or a tree node inside [P, key_end) whose ancestor bit
// (from the row's bitmask) is set.
__device__ __forceinline__ uint32_t visible_bits(int p0, int P, int key_end, int T,
                                                 const uint32_t* mask_row) {
  uint32_t bits = 0;
  const int pre = min(P, key_end) - p0;  // prefix keys in this word
  if (pre >= 32) return 0xffffffffu;
  if (pre > 0) bits = (1u << pre) - 1u;
  const int n0 = p0 - P;        // node index of bit 0
  const int end = key_end - p0;  // bits below `end` are inside the key range
  if (end > 0 && n0 + 31 >= 0) {
    const int lo = max(0, -n0);  // first bit that is a tree node
    const int nb = n0 + lo;      // its node index
    const int widx = nb >> 5, sh = nb & 31;
    uint32_t word = mask_row[widx] >> sh;
    if (sh != 0 && (widx + 1) * 32 < T) word |= mask_row[widx + 1] << (32 - sh);
    word <<= lo;
    bits |= word & (end >= 32 ? 0xffffffffu : ((1u << end) - 1u));
  }
  return bits;
}

struct Item {
  int r, split, h, tp, n_split, mblocks, slot_base, counter_base;
  int P, T, q_start, key_begin, key_end, n_tiles;
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
  it.key_begin = it.split * split_keys;
  if (it.split + 1 < it.n_split) {
    it.key_end = it.key_begin + split_keys;
  } else {
    const int last_row = it.tp * kM + kM - 1;
    it.key_end = it.P + min(it.T, last_row / p.groups + 1);
  }
  it.n_tiles = (it.key_end - it.key_begin + kN - 1) / kN;
  return it;
}

// Single-launch mode (no plan kernel, one item per CTA, no split): item `index` in the
// plan's order for a split-free plan (requests in order, then KV head, then query tile).
// Returns false past the last item; a request whose tree exceeds the mask capacity is
// skipped and flagged, as the plan kernel does.
__device__ __forceinline__ bool static_item(const JtTreeAttnParams& p, int index, int cap,
                                            Item& it) {
  for (int r = 0; r < p.num_requests; ++r) {
    const int nodes = p.node_counts[r];
    const int prefix = p.prefix_lens[r];
    if (nodes < 1 || prefix < 0) continue;
    if (nodes > cap) {
      if (threadIdx.x == 0) atomicOr(&g_attn_errors, JT_DEVERR_TREE_TOO_LARGE);
      continue;
    }
    const int mb = (nodes * p.groups + kM - 1) / kM;
    if (index < mb * p.num_kv_heads) {
      it.r = r;
      it.split = 0;
      it.h = index / mb;
      it.tp = index - it.h * mb;
      it.n_split = 1;
      it.mblocks = mb;
      it.slot_base = 0;
      it.counter_base = 0;
      it.P = prefix;
      it.T = nodes;
      it.q_start = p.cu_seqlens_q[r];
      it.key_begin = 0;
      it.key_end = prefix + min(nodes, (it.tp * kM + kM - 1) / p.groups + 1);
      it.n_tiles = (it.key_end + kN - 1) / kN;
      return true;
    }
    index -= mb * p.num_kv_heads;
  }
  return false;
}

// Gathers one 128-key K or V tile that touches tree nodes (scattered scratch slots) into
// its ring stage, one cp.async row per gather thread and step (rows past key_end are
// zero-filled), and waits for the rows to land; the caller then arrives on the stage's
// full barrier.
__device__ __forceinline__ void gather_kv_tile(const JtTreeAttnParams& p, const Item& it,
                                               const int32_t* table, int kb, int gtid,
                                               uint32_t dst, const char* pool, int64_t s0,
                                               int64_t s1, int64_t s2, int64_t pool_slots) {
  const int bs = p.block_size;
  for (int row = gtid; row < kN; row += kGatherThreads) {
    const int pos = kb + row;
    int64_t off = -1;
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
        const int64_t pg = slot / bs, o = slot - pg * bs;
        off = (pg * s0 + o * s1 + static_cast<int64_t>(it.h) * s2) * 2;
      } else {
        atomicOr(&g_attn_errors, JT_DEVERR_OUT_OF_RANGE);
      }
    }
#pragma unroll
    for (int chunk = 0; chunk < 16; ++chunk)
      jt::cp_async_16(dst + swz128(row, chunk, kN), off >= 0 ? pool + off + chunk * 16 : pool,
                      off >= 0 ? 16 : 0);
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  fence_proxy_async();
}
// Softmax helpers for one score row (the calling thread's TMEM lane) of one 128-key tile.
// `vk` describes the tile for masked tiles: keys kb..kb+127, prefix P, range end, nodes T
// and the row's ancestor bitmask (row_ok false masks the whole row).
struct TileKeys {
  int kb, P, key_end, T;
  const uint32_t* mask_row;
  bool row_ok;
};

template <bool kMasked>
__device__ __forceinline__ uint32_t chunk_visibility(const TileKeys& vk, int h) {
  if constexpr (!kMasked) return 0xffffffffu;
  return vk.row_ok ? visible_bits(vk.kb + 32 * h, vk.P, vk.key_end, vk.T, vk.mask_row) : 0u;
}

// Exponentials of score pairs on the FMA pipe, relieving the MUFU unit (16 results per
// clock per SM) that otherwise bounds the softmax.  2^x = 2^j * 2^f with j = rint(x) taken
// from the float rounding trick (x + 1.5 * 2^23) and 2^f, f in [-0.5, 0.5], from a cubic
// fitted to minimise the relative error on that interval (Lawson / minimax fit; max
// relative error 8.4e-5, far below the bf16 rounding of P).  j is added straight into the
// exponent field; x is clamped at -125 so the result stays a normal number or zero.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x = make_float2(fmaxf(x.x, -125.f), fmaxf(x.y, -125.f));
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 j = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __fadd2_rn(x, make_float2(-j.x, -j.y));
  float2 q = __ffma2_rn(make_float2(0.05521299f, 0.05521299f), f,
                        make_float2(0.24271414f, 0.24271414f));
  q = __ffma2_rn(q, f, make_float2(0.69326216f, 0.69326216f));
  q = __ffma2_rn(q, f, make_float2(0.9999196f, 0.9999196f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// Pairs per 16 whose exponentials go to the FMA pipe in unmasked tiles (0, 1, 2, 4, 8).
#ifndef JT_EXP2_POLY_PAIRS
#define JT_EXP2_POLY_PAIRS 4
#endif
constexpr int kPolyPairs = JT_EXP2_POLY_PAIRS;
__host__ __device__ constexpr bool poly_pair(int c) {
  return kPolyPairs > 0 && (c % (16 / (kPolyPairs > 0 ? kPolyPairs : 1))) ==
                               (16 / (kPolyPairs > 0 ? kPolyPairs : 1)) - 1;
}
// Softmax of one score row for one key half.  The two softmax warpgroups share every
// 128-key tile: warpgroup `c` owns keys 64c..64c+63, i.e. S columns 64c..64c+63, and only
// ever reads or writes those.  Each thread loads its 64 scores (two 32-column TMEM loads,
// one wait), publishes its half's max in `xm` and meets the other warpgroup on `mx_bar`
// (a rendezvous of the eight softmax warps), so both derive the same running max.  The running max is
// lazy: it moves only when the tile max exceeds it by more than 8 (log2 units).  P =
// exp2(s * scale_log2 - m), rounded to the operand type, goes to this half's columns
// (col_p).  Returns the fp32 sum of this half's P; `alpha` is the factor the older O and
// partial sum must take.
template <typename Elem, bool FP32P, bool kMasked>
__device__ __forceinline__ float softmax_half(uint32_t s_addr, int c, const TileKeys& vk,
                                              float scale_log2, float& m_run, float& alpha,
                                              float* xm_mine, const float* xm_other,
                                              uint32_t mx_bar, uint32_t mx_parity,
                                              volatile int* abort) {
  using Mma = jt::MmaOp<Elem>;
  const int own = 64 * c;
  uint32_t v[64];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    tmem_ld32(s_addr + own + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * h));
  uint32_t vw[2];
  if constexpr (kMasked) {
#pragma unroll
    for (int h = 0; h < 2; ++h) vw[h] = chunk_visibility<true>(vk, 2 * c + h);
  }
  tmem_wait_ld();
  if constexpr (kMasked) {
#pragma unroll
    for (int k = 0; k < 64; ++k)
      if (!((vw[k >> 5] >> (k & 31)) & 1u)) v[k] = __float_as_uint(-INFINITY);
  }
  float m8[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m8[k] = fmaxf(__uint_as_float(v[k]), __uint_as_float(v[k + 8]));
#pragma unroll
  for (int k0 = 16; k0 < 64; k0 += 16)
#pragma unroll
    for (int k = 0; k < 8; ++k)
      m8[k] = max3f(m8[k], __uint_as_float(v[k0 + k]), __uint_as_float(v[k0 + k + 8]));
  const float half_max = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]),
                               fmaxf(m8[6], m8[7]));
  *xm_mine = half_max;
  warp_arrive(mx_bar);
  warp_wait(mx_bar, mx_parity, abort);
  // Raw max; scale > 0 keeps the order.
  const float mx = fmaxf(half_max, *xm_other) * scale_log2;
  alpha = 1.f;
  if (mx > m_run + 8.f) {
    if (m_run != -INFINITY) alpha = jt::fast_exp2(m_run - mx);
    m_run = mx;
  }
  const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
  const float2 scale2 = make_float2(scale_log2, scale_log2);
  const float2 neg2 = make_float2(neg_m, neg_m);
  float2 r2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  const uint32_t p_addr = s_addr + col_p(4 * c);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t ph[16];
    uint32_t pl[FP32P ? 16 : 1];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float2 x = __ffma2_rn(
          make_float2(__uint_as_float(v[32 * h + 2 * k]), __uint_as_float(v[32 * h + 2 * k + 1])),
          scale2, neg2);
      float2 e;
      if (!kMasked && !FP32P && poly_pair(k))
        e = exp2_poly2(x);
      else
        e = make_float2(jt::fast_exp2(x.x), jt::fast_exp2(x.y));
      r2[k & 1] = __fadd2_rn(r2[k & 1], e);
      ph[k] = Mma::pack(e.x, e.y);
      if constexpr (FP32P) {
        const float2 r = Mma::unpack(ph[k]);
        pl[k] = Mma::pack(e.x - r.x, e.y - r.y);
      }
    }
    tmem_st16(p_addr + 16 * h, ph);
    if constexpr (FP32P) tmem_st16(p_addr + 32 + 16 * h, pl);
  }
  return (r2[0].x + r2[1].x) + (r2[0].y + r2[1].y);
}

// Zero P for this warpgroup's 64 keys (rows of a warp with no live row).
template <bool FP32P>
__device__ __forceinline__ void write_zero_half(uint32_t s_addr, int c) {
  uint32_t z[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) z[k] = 0u;
  const uint32_t p_addr = s_addr + col_p(4 * c);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    tmem_st16(p_addr + 16 * h, z);
    if constexpr (FP32P) tmem_st16(p_addr + 32 + 16 * h, z);
  }
}
template <typename Elem, bool FP32P>
__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_tc_kernel(const JtTreeAttnParams p, const DevLayout w,
                        const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const int single_launch) {
  using Mma = jt::MmaOp<Elem>;
  constexpr bool kBf16 = std::is_same<Elem, __nv_bfloat16>::value;
  constexpr uint32_t kIdescQK = instr_desc(kM, kN, kBf16, false);
  constexpr uint32_t kIdescPV = instr_desc(kM, kD, kBf16, true);

  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = jt::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + kOffBar;
#define JT_BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))
  volatile int* misc = reinterpret_cast<volatile int*>(sbase + kOffMisc);
  // misc[0]: TMEM base, misc[1]: abort, misc[2]: ring positions free to gather into
  volatile int* abort = misc + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t count = 1;
      if ((i >= kBarPFull && i < kBarPFull + kSBufs) || i == kBarOFree || i == kBarMx ||
          i == kBarLx)
        count = kSoftmaxWarps;
      if (i == kBarItemEmpty || i == kBarItemEmpty + 1) count = kItemConsumers;
      if (i >= kBarFull && i < kBarFull + kRing) count = kFullArrivals;
      mbar_init(JT_BAR(i), count);
    }
    misc[1] = 0;
    misc[2] = 0;  // ring_free
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

  // Launched as a programmatic dependent of the plan kernel: everything above overlapped
  // the plan; from here on the plan's output (and, through it, every earlier launch on the
  // stream) is complete and visible.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const int G = p.groups, bs = p.block_size;
  // Single-launch mode (small batches, chosen on the host from the launch shape): no plan
  // kernel ran; this CTA's only item comes from static_item, and the ancestor bitmasks of
  // its tree rows are built here into shared memory (the plan's mask blocks, for one item).
  const bool single = single_launch != 0;
  Item s_it{};
  const bool s_has = single && static_item(p, blockIdx.x, w.mask_words * 32, s_it);
  const uint32_t* smask = reinterpret_cast<const uint32_t*>(sbase + kOffMask);
  if (s_has) {
    uint32_t* masks = reinterpret_cast<uint32_t*>(sbase + kOffMask);
    const int rows = kM / G, j0 = s_it.tp * rows;
    const int words = (s_it.T + 31) / 32;
    const float* bias = p.qq_bias + p.qq_bias_offsets[s_it.r];
    for (int task = warp; task < rows * words; task += kThreads / 32) {
      const int jj = task / words, wd = task - jj * words;
      const int jrow = j0 + jj, n = wd * 32 + lane;
      const bool visible = jrow < s_it.T && n < s_it.T && n <= jrow &&
                           bias[static_cast<int64_t>(jrow) * s_it.T + n] == 0.0f;
      const uint32_t bits = __ballot_sync(0xffffffffu, visible);
      if (lane == 0) masks[jj * kMaskWordsMax + wd] = bits;
    }
    __syncthreads();
  }
  const int num_items = single ? 0 : w.header[1];
  const int split_keys = single ? 0 : w.header[2];

  // Work items: lane 0 of the TMA warp takes the next one from the device queue, decodes
  // it and publishes the decoded item through a two-entry ring in shared memory, one item
  // ahead of its own loads, so no role waits on the decode's global-memory chain at an
  // item boundary.  Every lane reads each entry; the warp takes it as an item only when
  // every lane did, so the end of the queue, or an abort, reads as no item for all lanes.
  volatile int* item_ring = reinterpret_cast<volatile int*>(sbase + kOffItem);
  auto publish = [&](uint32_t seq) {
    const int slot = seq & 1;
    if (seq >= 2) mbar_wait(JT_BAR(kBarItemEmpty + slot), ((seq >> 1) - 1) & 1, abort);
    volatile int* e = item_ring + 16 * slot;
    int index = num_items;
    if (single) index = (seq == 0 && s_has && !*abort) ? 0 : 1;
    else if (!*abort) index = atomicAdd(&w.header[0], 1);
    if (single ? index == 0 : index < num_items) {
      const Item it = single ? s_it : decode(p, w, index, split_keys);
      const int f[14] = {it.r, it.split, it.h, it.tp, it.n_split, it.mblocks, it.slot_base,
                         it.counter_base, it.P, it.T, it.q_start, it.key_begin, it.key_end,
                         it.n_tiles};
#pragma unroll
      for (int k = 0; k < 14; ++k) e[k] = f[k];
      e[15] = 1;
    } else {
      e[15] = 0;
    }
    mbar_arrive(JT_BAR(kBarItemFull + slot));
  };
  auto next_item = [&](uint32_t seq, Item& it) -> bool {
    const int slot = seq & 1;
    int f[15];
#pragma unroll
    for (int k = 0; k < 15; ++k) f[k] = 0;
    // Every lane waits for the entry and reads it; lane 0 releases it once all have.
    if (mbar_wait(JT_BAR(kBarItemFull + slot), (seq >> 1) & 1, abort) && !*abort) {
      volatile int* e = item_ring + 16 * slot;
      f[14] = e[15];
#pragma unroll
      for (int k = 0; k < 14; ++k) f[k] = e[k];
    }
    // One verdict per warp: an item only when every lane read it.
    f[14] = __all_sync(0xffffffffu, f[14] != 0) ? 1 : 0;
    if (lane == 0) mbar_arrive(JT_BAR(kBarItemEmpty + slot));
    it.r = f[0]; it.split = f[1]; it.h = f[2]; it.tp = f[3]; it.n_split = f[4];
    it.mblocks = f[5]; it.slot_base = f[6]; it.counter_base = f[7]; it.P = f[8]; it.T = f[9];
    it.q_start = f[10]; it.key_begin = f[11]; it.key_end = f[12]; it.n_tiles = f[13];
    return f[14] != 0;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ MMA issuer
    // Per item: QK 0..2 into S buffers g%3 (g counts tiles over all items), then per tile
    // t: PV t (once the softmax published P t) and QK t+3.  tcgen05.mma instructions of
    // one thread execute in issue order, so PV t has read P t out of its S buffer before
    // QK t+3 overwrites that buffer.
    // The whole warp runs this loop with warp-uniform values; elect.sync inside the MMA
    // and commit wrappers picks the issuing lane.  Descriptors are built once: within a
    // tile they differ only in the start-address field (16-byte units), so each MMA adds
    // a compile-time constant.
    uint32_t ring = 0, q_count = 0, g0 = 0;
    bool o_used = false;
    uint32_t of_par = 0;
    const uint64_t q_desc = smem_desc(base + kOffQ, 16, 1024);
    const uint64_t ring_k_desc = smem_desc(base + kOffRing, 16, 1024);
    const uint64_t ring_v_desc = smem_desc(base + kOffRing, kKVHalfBytes, 1024);
    for (uint32_t seq = 0;; ++seq) {
      Item it;
      if (!next_item(seq, it)) break;
      const int n = it.n_tiles;
      mbar_wait(JT_BAR(kBarQFull), q_count & 1, abort);
      ++q_count;
      tc_fence_after();
      auto take = [&]() -> int {
        const int slot = ring % kRing;
        mbar_wait(JT_BAR(kBarFull + slot), (ring / kRing) & 1, abort);
        tc_fence_after();
        return slot;
      };
      auto release = [&](int slot) {
        tc_commit_warp(JT_BAR(kBarEmpty + slot));
        ++ring;
      };
      auto issue_qk = [&](int t) {
        const int slot = take();
        const int b = (g0 + t) % kSBufs;
        const uint64_t kd = ring_k_desc + static_cast<uint64_t>(slot * (kKVBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk & 3) * 32;
          mma_ss_warp(tmem + col_s(b), q_desc + ((kk >> 2) * kQHalfBytes + off) / 16,
                      kd + ((kk >> 2) * kKVHalfBytes + off) / 16, kIdescQK, kk > 0 ? 1u : 0u);
        }
        tc_commit_warp(JT_BAR(kBarSFull + b));
        release(slot);
        if (t == n - 1) tc_commit_warp(JT_BAR(kBarQEmpty));
      };
      for (int t = 0; t < min(kAhead, n); ++t) issue_qk(t);
      for (int t = 0; t < n; ++t) {
        const int g = g0 + t;
        const int b = g % kSBufs;
        const int slot = take();
        if (t == 0 && o_used) {
          // O still holds the previous item until its epilogue has read it.
          mbar_wait(JT_BAR(kBarOFree), of_par, abort);
          of_par ^= 1u;
        }
        mbar_wait(JT_BAR(kBarPFull + b), (g / kSBufs) & 1, abort);
        tc_fence_after();
        // O += P V (P inside S buffer b in TMEM, V MN-major in shared memory).
        const uint32_t pa = tmem + col_s(b);
        const uint64_t vd = ring_v_desc + static_cast<uint64_t>(slot * (kKVBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          mma_ts_warp(tmem + col_o(), pa + col_p(kk), vd + kk * (2048 / 16), kIdescPV,
                      (t > 0 || kk > 0) ? 1u : 0u);
          if constexpr (FP32P)
            mma_ts_warp(tmem + col_o(), pa + col_p(kk) + 32, vd + kk * (2048 / 16), kIdescPV, 1u);
        }
        tc_commit_warp(JT_BAR(kBarPvDone + b));
        release(slot);
        if (t + kAhead < n) issue_qk(t + kAhead);
      }
      g0 += n;
      o_used = true;
    }
    // Drain: every MMA the issuing lane started has completed before TMEM is released.
    tc_commit_warp(JT_BAR(kBarDrain));
    mbar_wait(JT_BAR(kBarDrain), 0, abort, false);
  } else if (warp < 4) {
    // ------------------------------------------------------------------ loaders
    // Warp 1 publishes the work items, issues every TMA load (query tiles, prefix K/V
    // tiles) and is the only waiter on the ring's empty barriers: it waits for every ring
    // position in order (so it is never a phase behind or ahead on any slot) and then
    // publishes the position as free in `ring_free`.  Warps 2-3 gather the tiles that touch
    // tree nodes with cp.async, each once `ring_free` has reached its position, so a gather
    // waiting for its rows never holds back the TMA loads behind it.  Both walk the same
    // fill sequence: the MMA's consumption order, K 0..2, then V t and K t+3 per tile.
    const bool tma_warp = warp == 1;
    const int gtid = tid - 64;  // gather thread index (warps 2-3)
    uint32_t ring = 0, q_fills = 0;
    uint32_t filled = 0;       // bit s: the last fill of ring slot s was TMA
    uint32_t last_parity = 0;  // bit s: phase parity of that fill
    const int64_t pool_slots = p.num_blocks * static_cast<int64_t>(bs);
    const uint32_t ring_free = base + kOffMisc + 8;  // misc[2]: last free ring position + 1
    if (tma_warp && lane == 0) publish(0);
    for (uint32_t seq = 0;; ++seq) {
      Item it;
      if (!next_item(seq, it)) break;
      const int n = it.n_tiles;
      const int32_t* table = p.block_tables + static_cast<int64_t>(it.r) * p.table_stride0;
      // Query tile: one TMA box of 128/groups nodes x groups heads x 64 dims per half, once
      // the previous item's last QK has read the buffer.  Rows past the request's nodes
      // hold other requests' queries (or zeros past the end); their score rows are never
      // written out.
      if (tma_warp && lane == 0) {
        if (seq > 0) mbar_wait(JT_BAR(kBarQEmpty), (seq - 1) & 1, abort);
        mbar_arrive_tx(JT_BAR(kBarQFull), kQTileBytes);
        const int node = it.q_start + it.tp * (kM / G);
        tma_load_3d(base + kOffQ, &qmap, 0, it.h * G, node, JT_BAR(kBarQFull));
        tma_load_3d(base + kOffQ + kQHalfBytes, &qmap, 64, it.h * G, node, JT_BAR(kBarQFull));
        ++q_fills;
      }
      auto fill = [&](bool is_v, int t) {
        const int kb = it.key_begin + t * kN;
        // A prefix tile inside one page (tiles never straddle pages: block_size is a
        // multiple of 128 and every key range starts on a tile boundary) goes by TMA.
        const bool full = kb + kN <= min(it.P, it.key_end);
        const int slot = ring % kRing;
        const uint32_t parity = (ring / kRing) & 1;
        const uint32_t dst = base + kOffRing + slot * kKVBytes;
        const uint32_t full_bar = JT_BAR(kBarFull + slot);
        if (tma_warp) {
          if (lane == 0) {
            if (ring >= kRing) mbar_wait(JT_BAR(kBarEmpty + slot), parity ^ 1, abort);
            if (full) {
              const int page = __ldg(table + kb / bs);
              const CUtensorMap* map = is_v ? &vmap : &kmap;
              mbar_arrive_tx(full_bar, kKVBytes);
              tma_load_4d(dst, map, 0, it.h, kb % bs, page, full_bar);
              tma_load_4d(dst + kKVHalfBytes, map, 64, it.h, kb % bs, page, full_bar);
              mbar_arrive(full_bar);
            } else {
              st_release_shared(ring_free, ring + 1);
            }
          }
        } else if (!full) {
          wait_shared_at_least(ring_free, ring + 1, abort);
          const char* pool = static_cast<const char*>(is_v ? p.v_pool : p.k_pool);
          const int64_t s0 = is_v ? p.v_stride0 : p.k_stride0;
          const int64_t s1 = is_v ? p.v_stride1 : p.k_stride1;
          const int64_t s2 = is_v ? p.v_stride2 : p.k_stride2;
          gather_kv_tile(p, it, table, kb, gtid, dst, pool, s0, s1, s2, pool_slots);
          __syncwarp();
          if (lane == 0) mbar_arrive(full_bar);
        }
        const uint32_t bit = 1u << slot;
        if (full) { filled |= bit; last_parity = (last_parity & ~bit) | (parity ? bit : 0u); }
        else filled &= ~bit;
        ++ring;
      };
      for (int t = 0; t < min(kAhead, n); ++t) fill(false, t);
      for (int t = 0; t < n; ++t) {
        // The next item is claimed and published while this one still has about four
        // tiles to go: early enough for its query tile and first K tiles to be loaded
        // before the MMA reaches them, late enough not to hold work another CTA could take.
        if (tma_warp && lane == 0 && t == max(0, n - 4)) publish(seq + 1);
        fill(true, t);
        if (t + kAhead < n) fill(false, t + kAhead);
      }
    }
    // Drain: the TMA copies this warp issued have landed before the CTA exits.
    if (tma_warp && lane == 0) {
      for (int s = 0; s < kRing; ++s)
        if (filled & (1u << s))
          mbar_wait(JT_BAR(kBarFull + s), (last_parity >> s) & 1u, abort, false);
      if (q_fills > 0) mbar_wait(JT_BAR(kBarQFull), (q_fills - 1) & 1u, abort, false);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int c = (warp - 4) >> 2;           // key / output column half of this warpgroup
    const int t128 = tid - 128 - c * 128;    // score row (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>((t128 >> 5) * 32) << 16;
    float* xl = reinterpret_cast<float*>(sbase + kOffXl);  // [half][row] row sums
    // [tile parity][half][row] half maxima: alternating buffers, so a warpgroup that runs a
    // tile ahead never overwrites a value the other warpgroup has yet to read.
    float* xm = reinterpret_cast<float*>(sbase + kOffXm);
    const float scale_log2 = p.scale * 1.4426950408889634f;
    // Operand-type rows whose 32-column pieces start on 32-byte boundaries take 32-byte
    // stores.
    const bool wide_out = (reinterpret_cast<uintptr_t>(p.out) & 31u) == 0 &&
                          (p.out_stride0 | p.out_stride1) % 16 == 0;
    uint32_t g0 = 0, mx_par = 0, lx_par = 0;
    for (uint32_t seq = 0;; ++seq) {
      Item it;
      if (!next_item(seq, it)) break;
      const int n = it.n_tiles;
      const int gm = it.tp * kM + t128;
      const int j = gm / G, g = gm - j * G;
      const bool row_ok = j < it.T;
      const bool warp_live = __any_sync(0xffffffffu, row_ok);
      const uint32_t* mask_row =
          single ? smask + (row_ok ? j - it.tp * (kM / G) : 0) * kMaskWordsMax
                 : w.masks + static_cast<int64_t>(it.q_start + (row_ok ? j : 0)) * w.mask_words;
      float m_run = -INFINITY;  // running max in log2 units (scaled scores)
      float l_run = 0.f;        // this half's partial row sum
      const uint32_t o_addr = tmem + lane_base + col_o();
      for (int t = 0; t < n; ++t) {
        const int gt = g0 + t;
        const int b = gt % kSBufs;
        const int kb = it.key_begin + t * kN;
        const bool full = kb + kN <= min(it.P, it.key_end);
        const TileKeys vk{kb, it.P, it.key_end, it.T, mask_row, row_ok};
        const uint32_t s_addr = tmem + lane_base + col_s(b);
        warp_wait(JT_BAR(kBarSFull + b), (gt / kSBufs) & 1, abort);
        tc_fence_after();
        float alpha = 1.f, rsum = 0.f;
        float* xm_mine = xm + ((gt & 1) * 2 + c) * kM + t128;
        const float* xm_other = xm + ((gt & 1) * 2 + (c ^ 1)) * kM + t128;
        if (warp_live) {
          rsum = full ? softmax_half<Elem, FP32P, false>(s_addr, c, vk, scale_log2, m_run,
                                                         alpha, xm_mine, xm_other,
                                                         JT_BAR(kBarMx), mx_par, abort)
                      : softmax_half<Elem, FP32P, true>(s_addr, c, vk, scale_log2, m_run,
                                                        alpha, xm_mine, xm_other,
                                                        JT_BAR(kBarMx), mx_par, abort);
        } else {
          // No live row in this warp: zero P, but still meet the other warpgroup.
          warp_arrive(JT_BAR(kBarMx));
          warp_wait(JT_BAR(kBarMx), mx_par, abort);
          write_zero_half<FP32P>(s_addr, c);
        }
        mx_par ^= 1u;
        l_run = l_run * alpha + rsum;
        if (t > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          // Rescale this warp's O rows once PV t-1 has completed.  A warp that needs no
          // rescale publishes P t at once, so PV t never waits for PV t-1 in the common
          // case.  The wait is for exactly one phase of PvDone[(gt-1) % 3]: its previous
          // phase (PV gt-4) completed before QK gt, whose S this warp has read, and its next
          // one (PV gt+2) needs this warp's P gt+2.
          const int gp = gt - 1;
          warp_wait(JT_BAR(kBarPvDone + gp % kSBufs), (gp / kSBufs) & 1, abort);
          tc_fence_after();
#pragma unroll 1
          for (int chunk = 0; chunk < 2; ++chunk) {
            uint32_t o[32];
            tmem_ld32(o_addr + 64 * c + chunk * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            tmem_st32(o_addr + 64 * c + chunk * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive(JT_BAR(kBarPFull + b));
      }
      // Epilogue: wait for the item's last PV, swap the half row sums, then each
      // warpgroup writes its 64 output columns.
      {
        const int gl = g0 + n - 1;  // same one-phase argument as the rescale wait
        warp_wait(JT_BAR(kBarPvDone + gl % kSBufs), (gl / kSBufs) & 1, abort);
      }
      xl[c * kM + t128] = l_run;
      warp_arrive(JT_BAR(kBarLx));
      warp_wait(JT_BAR(kBarLx), lx_par, abort);
      lx_par ^= 1u;
      const float l_fin = l_run + xl[(c ^ 1) * kM + t128];
      tc_fence_after();
      const bool split_item = it.n_split > 1;
      const int64_t slot = it.slot_base +
                           (static_cast<int64_t>(it.h) * it.mblocks + it.tp) * it.n_split + it.split;
      const float inv = 1.f / l_fin;
#pragma unroll 1
      for (int chunk = 0; chunk < 2; ++chunk) {
        uint32_t o[32];
        tmem_ld32(o_addr + 64 * c + chunk * 32, o);
        tmem_wait_ld();
        const int col = 64 * c + 32 * chunk;
        if (split_item) {
          // Column-group-major partials, [slot][32 groups of 4 columns][128 rows]: the 32
          // lanes of a warp store 512 contiguous bytes per instruction.
          float4* dst = reinterpret_cast<float4*>(w.part_o) +
                        (slot * (kD / 4) + col / 4) * kM + t128;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            dst[k * kM] = make_float4(__uint_as_float(o[4 * k]), __uint_as_float(o[4 * k + 1]),
                                      __uint_as_float(o[4 * k + 2]), __uint_as_float(o[4 * k + 3]));
        } else if (row_ok) {
          const int64_t off = static_cast<int64_t>(it.q_start + j) * p.out_stride0 +
                              static_cast<int64_t>(it.h * G + g) * p.out_stride1 + col;
          if (p.out_dtype == JT_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              dst[k] = make_float4(__uint_as_float(o[4 * k]) * inv, __uint_as_float(o[4 * k + 1]) * inv,
                                   __uint_as_float(o[4 * k + 2]) * inv,
                                   __uint_as_float(o[4 * k + 3]) * inv);
          } else if (wide_out) {
            // 32-byte stores: each fills a whole sector, half the store transactions.
            Elem* dst = static_cast<Elem*>(p.out) + off;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              uint32_t v8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                v8[e] = Mma::pack(__uint_as_float(o[16 * k + 2 * e]) * inv,
                                  __uint_as_float(o[16 * k + 2 * e + 1]) * inv);
              asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"l"(
                               dst + 16 * k),
                           "r"(v8[0]), "r"(v8[1]), "r"(v8[2]), "r"(v8[3]), "r"(v8[4]), "r"(v8[5]),
                           "r"(v8[6]), "r"(v8[7])
                           : "memory");
            }
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<Elem*>(p.out) + off);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              dst[k] = make_uint4(
                  Mma::pack(__uint_as_float(o[8 * k]) * inv, __uint_as_float(o[8 * k + 1]) * inv),
                  Mma::pack(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv),
                  Mma::pack(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv),
                  Mma::pack(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv));
          }
        }
      }
      tc_fence_before();
      warp_arrive(JT_BAR(kBarOFree));
      if (split_item) {
        // Per-(row, half) merge: each half publishes its 64 columns and its own copy of the
        // row's max (log2 units) and sum, then bumps the (row, half) counter; the arrival
        // that completes it (this half of every split) merges those 64 columns.  Nothing
        // waits: rows and halves finish independently.
        w.part_ml[(slot * 2 + c) * kM + t128] = make_float2(m_run, l_fin);
        __threadfence();
        int* counter = w.counters +
                       (static_cast<int64_t>(it.counter_base) + it.h * it.mblocks + it.tp) * 2 * kM +
                       c * kM + t128;
        const int done = atomicAdd(counter, 1);
        if (done == it.n_split - 1) {
          *counter = 0;
          __threadfence();
          if (row_ok) {
            // Online merge over the splits, two splits' loads in flight per round: the
            // running max moves as new splits arrive and the accumulated columns are
            // rescaled, so no separate pass over the maxima is needed.
            const int64_t slot0 =
                it.slot_base + (static_cast<int64_t>(it.h) * it.mblocks + it.tp) * it.n_split;
            const int ns = it.n_split;
            const int64_t off = static_cast<int64_t>(it.q_start + j) * p.out_stride0 +
                                static_cast<int64_t>(it.h * G + g) * p.out_stride1 + 64 * c;
            const float4* po = reinterpret_cast<const float4*>(w.part_o);
#pragma unroll 1
            for (int part = 0; part < 2; ++part) {
              const int cg0 = 16 * c + 8 * part;  // first 4-column group of this part
              float acc[32];
#pragma unroll
              for (int k = 0; k < 32; ++k) acc[k] = 0.f;
              float den = 0.f, mrun = -INFINITY;
#pragma unroll 1
              for (int s2 = 0; s2 < ns; s2 += 2) {
                const bool two = s2 + 1 < ns;
                const float2 mla = __ldcg(w.part_ml + ((slot0 + s2) * 2 + c) * kM + t128);
                const float2 mlb = two ? __ldcg(w.part_ml + ((slot0 + s2 + 1) * 2 + c) * kM + t128)
                                       : make_float2(-INFINITY, 0.f);
                float4 va[8], vb[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  va[k] = __ldcg(po + ((slot0 + s2) * (kD / 4) + cg0 + k) * kM + t128);
                  vb[k] = two ? __ldcg(po + ((slot0 + s2 + 1) * (kD / 4) + cg0 + k) * kM + t128)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                const float mnew = fmaxf(mrun, fmaxf(mla.x, mlb.x));
                const float mref = mnew == -INFINITY ? 0.f : mnew;
                const float sc = mrun == -INFINITY ? 0.f : jt::fast_exp2(mrun - mref);
                const float wa = jt::fast_exp2(mla.x - mref);
                const float wb = two ? jt::fast_exp2(mlb.x - mref) : 0.f;
                den = den * sc + wa * mla.y + wb * mlb.y;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  acc[4 * k] = acc[4 * k] * sc + wa * va[k].x + wb * vb[k].x;
                  acc[4 * k + 1] = acc[4 * k + 1] * sc + wa * va[k].y + wb * vb[k].y;
                  acc[4 * k + 2] = acc[4 * k + 2] * sc + wa * va[k].z + wb * vb[k].z;
                  acc[4 * k + 3] = acc[4 * k + 3] * sc + wa * va[k].w + wb * vb[k].w;
                }
                mrun = mnew;
              }
              const float dinv = 1.f / den;
              if (p.out_dtype == JT_F32) {
                float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off + 32 * part);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                  dst[k] = make_float4(acc[4 * k] * dinv, acc[4 * k + 1] * dinv,
                                       acc[4 * k + 2] * dinv, acc[4 * k + 3] * dinv);
              } else {
                uint4* dst = reinterpret_cast<uint4*>(static_cast<Elem*>(p.out) + off + 32 * part);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  dst[k] = make_uint4(Mma::pack(acc[8 * k] * dinv, acc[8 * k + 1] * dinv),
                                      Mma::pack(acc[8 * k + 2] * dinv, acc[8 * k + 3] * dinv),
                                      Mma::pack(acc[8 * k + 4] * dinv, acc[8 * k + 5] * dinv),
                                      Mma::pack(acc[8 * k + 6] * dinv, acc[8 * k + 7] * dinv));
              }
            }
          }
        }
      }
      g0 += n;
    }
  }
#undef JT_BAR

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem) : "memory");
  }
}

// Self-test of the bounded wait (failure detection without a GPU fault): one thread waits
// on an mbarrier nothing arrives on, with a short limit.  The wait must give up, raise the
// CTA's abort flag and the timeout error bit, and the kernel must return normally.
// out[0]: 1 if the wait claimed completion (a failure); out[1]: the abort flag afterwards;
// out[2]: cycles spent in the wait (saturated).
__global__ void wait_selftest_kernel(long long limit, int* out) {
  __shared__ __align__(8) unsigned long long bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  const uint32_t addr = jt::smem_u32(&bar);
  mbar_init(addr, 1);
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  const long long t0 = clock64();
  const bool ok = mbar_wait(addr, 0, &abort_flag, true, limit);
  const long long spent = clock64() - t0;
  out[0] = ok ? 1 : 0;
  out[1] = abort_flag;
  out[2] = static_cast<int>(spent < 0x7fffffffll ? spent : 0x7fffffffll);
}

}  // namespace tc
