// Batched 16-bit GEMM for the Newton-Schulz orthogonaliser, written for sm_100a:
//   * tcgen05.mma kind::f16 (bf16 or binary16 operands) accumulating fp32 in
//     tensor memory, two 256-column accumulators so the epilogue of one tile
//     overlaps the main loop of the next; 128 x 256 tiles on one CTA
//     (cta_group::1) or 256 x 256 tiles on a CTA pair (cta_group::2);
//   * operands staged by TMA (cp.async.bulk.tensor, 128-byte swizzle; every
//     CTA loads its own tiles) through an mbarrier ring; either operand may be
//     K-major or MN-major, so tall matrices are consumed in their stored layout;
//   * a persistent grid (one CTA or CTA pair per SM slot) walking a static tile schedule;
//     symmetric outputs compute only tiles that touch the upper triangle and
//     mirror them in the epilogue;
//   * warp roles: warp 0 = TMA producer, warp 1 = MMA issuer (and TMEM owner),
//     warps 2-9 = epilogue (two per TMEM lane quadrant, half the columns each;
//     warps 2-5 only, whole rows, for outputs with row sums).
// Every wait is bounded: on expiry the CTA raises the device error word,
// drains its own copies and MMAs (again bounded), frees TMEM and returns.
// A CUDA-core kernel covers shapes the tensor-core path does not take
// (min(M,N) < 128, unaligned strides) with the same epilogues.
#include "b2o_common.cuh"
#include "b2o_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace b2o {

namespace tc {

constexpr int BM = 128, BN = 256, BK = 64;     // BM: rows of one CTA's accumulator
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int TMEM_COLS = 512;                  // 2 accumulators x 256 fp32 columns
// Epilogue staging: per epilogue warp two slots of two 32x32 16-bit tiles
// (direct and mirrored), 64-byte rows in the TMA 64-byte swizzle, written by
// TMA stores; while one slot's stores drain the next chunk fills the other.
constexpr int EPI_TILE_BYTES = 32 * 32 * 2;
constexpr int EPI_WARP_BYTES = 2 * 2 * EPI_TILE_BYTES;  // 8 KB
// Epilogue warps: two per TMEM lane quadrant (each moves half of the 256
// accumulator columns), except for outputs with row sums, whose partials are
// per 256-column tile and row, kept whole by one warp per quadrant.
template <int RSQ> struct EpiWarps { static constexpr int value = RSQ ? 4 : 8; };
// PAIR = 1: one CTA computes a 128 x 256 tile (stages of 16 + 32 KB).
// PAIR = 2: a CTA pair (cluster of 2, tcgen05 cta_group::2) computes a
// 256 x 256 tile; each CTA stages its 128 rows of A and its 128 columns of B
// (stages of 16 + 16 KB), halving the operand bytes each SM pulls per MMA.
// The operand ring takes what shared memory leaves beside the epilogue staging.
template <int PAIR, int EW> struct Geo {
  static constexpr int B_ROWS = BN / PAIR;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_BYTES = EW * EPI_WARP_BYTES;
  static constexpr int STAGES = PAIR == 1 ? (EW == 8 ? 3 : 4) : (EW == 8 ? 5 : 6);
  static constexpr int STAGE_AREA = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGE_AREA + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int TILE_M = BM * PAIR;
  static constexpr int THREADS = 64 + 32 * EW;  // TMA warp, MMA warp, epilogue warps
};
static_assert(Geo<1, 4>::SMEM_BYTES <= 232448 && Geo<1, 8>::SMEM_BYTES <= 232448, "shared memory");
static_assert(Geo<2, 4>::SMEM_BYTES <= 232448 && Geo<2, 8>::SMEM_BYTES <= 232448, "shared memory");
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

struct Params {
  int M, N, K, batch;
  int tile_m;  // rows per output tile: 128 (one CTA) or 256 (CTA pair)
  int a_kmajor, b_kmajor, sym, in_half;
  int tiles_m, tiles_n, tiles_per_batch, total_tiles, nk;
  Epilogue e;
  int* err;
};

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. Returns false when the CTA is aborting (this wait ran out or
// another role of the CTA gave up).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      *abort_flag = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Byte offset of 16-bit element (row, col) in a 32x32 staging tile stored with
// 64-byte rows under the TMA 64-byte swizzle (16-byte chunk index XOR bits 1-2 of the row).
__device__ __forceinline__ uint32_t stage_off(int row, int col) {
  const uint32_t chunk = static_cast<uint32_t>(col >> 3) ^ ((static_cast<uint32_t>(row) >> 1) & 3u);
  return static_cast<uint32_t>(row) * 64u + (chunk << 4) + (static_cast<uint32_t>(col & 7) << 1);
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx_cluster(uint32_t caddr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(caddr), "r"(bytes) : "memory");
}
// TMA load whose completion is signalled on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                 uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(mbar_cluster)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on the mbarrier at this offset in both CTAs of the pair once all
// prior cta_group::2 MMAs of this thread have completed.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 128-byte-swizzled shared-memory matrix descriptor (sm_100 layout: start
// address, leading/stride byte offsets, version 1, layout type 2 = SW128).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// Issues a 32-column TMEM load into r (completes at tmem_ld_wait()).
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* out) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r[i]);
}

// Tile t of the schedule -> (batch, tile_m, tile_n). Symmetric outputs keep
// the tiles whose column range reaches the diagonal block of their rows.
__device__ __forceinline__ void tile_coords(const Params& p, int t, int& b, int& tm, int& tn) {
  b = t / p.tiles_per_batch;
  int local = t - b * p.tiles_per_batch;
  if (!p.sym) {
    tn = local / p.tiles_m;   // consecutive CTAs share the B column block
    tm = local - tn * p.tiles_m;
    return;
  }
  tn = 0;
  while (true) {
    const int cnt = min(p.tiles_m, (tn * BN + BN - 1) / p.tile_m + 1);
    if (local < cnt) { tm = local; return; }
    local -= cnt;
    ++tn;
  }
}

// ----------------------------------------------------------- epilogue ------
__device__ __forceinline__ void load_row32(const uint16_t* base, int64_t ld, int row, int col0, int M, int N,
                                           bool vec, int half, float* out) {
  if (vec) {
    const uint4* src = reinterpret_cast<const uint4*>(base + static_cast<int64_t>(row) * ld + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 v = src[q];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        out[q * 8 + 2 * h] = h16_to_f32(static_cast<uint16_t>(w[h] & 0xFFFFu), half);
        out[q * 8 + 2 * h + 1] = h16_to_f32(static_cast<uint16_t>(w[h] >> 16), half);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int col = col0 + j;
      out[j] = (row < M && col < N) ? h16_to_f32(base[static_cast<int64_t>(row) * ld + col], half) : 0.f;
    }
  }
}

template <int KIND>
__device__ __forceinline__ float epi_value(const Params& p, float acc, float c, float sc, int row, int col) {
  if (KIND == 0) return acc * sc;
  if (KIND == 1) return fmaf(p.e.gamma, acc, fmaf(p.e.beta, c, row == col ? p.e.alpha : 0.f));
  if (KIND == 2) return round_bf16(round_bf16(p.e.beta * c) + round_bf16(p.e.gamma * round_bf16(acc)));
  return round_bf16(round_bf16(p.e.alpha * c) + round_bf16(acc));
}
// Two values rounded to the 16-bit output type, packed low/high.
template <int DHALF>
__device__ __forceinline__ uint32_t pack2(float x0, float x1) {
  if (DHALF) {
    const __half2 h = __floats2half2_rn(x0, x1);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <int DHALF>
__device__ __forceinline__ float unpack_lo(uint32_t w) {
  return DHALF ? f16_to_f32(static_cast<uint16_t>(w & 0xFFFFu)) : bf16_to_f32(static_cast<uint16_t>(w & 0xFFFFu));
}
template <int DHALF>
__device__ __forceinline__ float unpack_hi(uint32_t w) {
  return DHALF ? f16_to_f32(static_cast<uint16_t>(w >> 16)) : bf16_to_f32(static_cast<uint16_t>(w >> 16));
}

template <int KIND, int DHALF, int SYM, int RSQ, int PAIR>
__global__ void __launch_bounds__((Geo<PAIR, EpiWarps<RSQ>::value>::THREADS), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ Params p) {
  constexpr int EW = EpiWarps<RSQ>::value;
  using G = Geo<PAIR, EW>;
  constexpr int STAGES = G::STAGES;
  constexpr int STAGE_BYTES = G::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + G::STAGE_AREA;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_smem + G::EPI_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR == 2 ? cluster_rank() : 0u;  // 0 = the CTA that issues the MMAs
  const int unit = blockIdx.x / PAIR;                       // tile-schedule slot (CTA or CTA pair)
  const int nunits = gridDim.x / PAIR;

  if (threadIdx.x == 0) {
    // full: one expect-tx arrival per CTA of the pair (counted on the MMA CTA);
    // tempty: every epilogue thread of the pair releases the accumulator
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full_bar[s], PAIR); mbar_init(&empty_bar[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull_bar[a], 1); mbar_init(&tempty_bar[a], 32 * EW * PAIR); }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    if (PAIR == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  fence_before_sync();
  __syncthreads();
  if (PAIR == 2) cluster_sync();  // the peer's barriers exist before any remote arrival
  fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // the set-up above overlaps the previous kernel's tail; no global memory is
  // touched before the previous kernel has completed
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[STAGES];  // phase of the last load issued into each stage
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
      bool ok = true;
      for (int t = unit; t < p.total_tiles && ok; t += nunits) {
        int b, tm, tn;
        tile_coords(p, t, b, tm, tn);
        const int arow = tm * G::TILE_M + static_cast<int>(rank) * BM;    // this CTA's rows of A
        const int bcol = tn * BN + static_cast<int>(rank) * G::B_ROWS;     // this CTA's columns of B
        for (int kb = 0; kb < p.nk; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t a_dst = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_dst = a_dst + A_BYTES;
          if (PAIR == 1) {
            mbar_expect_tx(&full_bar[stage], STAGE_BYTES);
            if (p.a_kmajor) {
              tma_load_3d(a_dst, &tmA, kb * BK, arow, b, &full_bar[stage]);
            } else {
              tma_load_3d(a_dst, &tmA, arow, kb * BK, b, &full_bar[stage]);
              tma_load_3d(a_dst + 8192, &tmA, arow + 64, kb * BK, b, &full_bar[stage]);
            }
            if (p.b_kmajor) {
              tma_load_3d(b_dst, &tmB, kb * BK, bcol, b, &full_bar[stage]);
            } else {
#pragma unroll
              for (int q = 0; q < G::B_ROWS / 64; ++q)
                tma_load_3d(b_dst + q * 8192, &tmB, bcol + q * 64, kb * BK, b, &full_bar[stage]);
            }
          } else {
            const uint32_t fb = map_to_rank(smem_u32(&full_bar[stage]), 0);
            mbar_expect_tx_cluster(fb, STAGE_BYTES);
            if (p.a_kmajor) {
              tma_load_3d_pair(a_dst, &tmA, kb * BK, arow, b, fb);
            } else {
              tma_load_3d_pair(a_dst, &tmA, arow, kb * BK, b, fb);
              tma_load_3d_pair(a_dst + 8192, &tmA, arow + 64, kb * BK, b, fb);
            }
            if (p.b_kmajor) {
              tma_load_3d_pair(b_dst, &tmB, kb * BK, bcol, b, fb);
            } else {
#pragma unroll
              for (int q = 0; q < G::B_ROWS / 64; ++q)
                tma_load_3d_pair(b_dst + q * 8192, &tmB, bcol + q * 64, kb * BK, b, fb);
            }
          }
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if ((!ok || *abort_flag) && rank == 0) {
        // Drain: wait (bounded) until the last loads issued into each stage
        // (by both CTAs of a pair: they signal this CTA's barriers) have
        // landed, so no copy into shared memory outlives the kernel.
        const uint64_t t0 = globaltimer();
        for (int s = 0; s < STAGES; ++s) {
          if (last_phase[s] < 0) continue;
          while (!mbar_try_wait(&full_bar[s], static_cast<uint32_t>(last_phase[s]))) {
            if (globaltimer() - t0 > kTimeoutNs) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer ---
    if (lane == 0 && rank == 0) {
      const uint32_t fmt = p.in_half ? 0u : 1u;  // kind::f16 operand format: 0 = f16, 1 = bf16
      const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(!p.a_kmajor) << 15) |
                             (static_cast<uint32_t>(!p.b_kmajor) << 16) | (static_cast<uint32_t>(BN >> 3) << 17) |
                             (static_cast<uint32_t>(G::TILE_M >> 4) << 24);
      const uint32_t a_lbo = p.a_kmajor ? 16u : 8192u;
      const uint32_t b_lbo = p.b_kmajor ? 16u : 8192u;
      const uint32_t a_kstep = p.a_kmajor ? 32u : 2048u;
      const uint32_t b_kstep = p.b_kmajor ? 32u : 2048u;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = unit; t < p.total_tiles && ok; t += nunits, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        fence_after_sync();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < p.nk; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          fence_after_sync();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = make_desc(a_addr + kk * a_kstep, a_lbo, 1024u);
            const uint64_t bd = make_desc(b_addr + kk * b_kstep, b_lbo, 1024u);
            if (PAIR == 2) mma_bf16_pair(tmem_d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else mma_bf16(tmem_d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          // frees the stage (in every CTA of the pair) once these MMAs retire
          if (PAIR == 2) mma_commit_pair_both(&empty_bar[stage]);
          else mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        // accumulator ready for the epilogue warps of every CTA of the pair
        if (PAIR == 2) mma_commit_pair_both(&tfull_bar[acc]);
        else mma_commit(&tfull_bar[acc]);
      }
      // Make sure every MMA this thread issued has retired before TMEM is freed.
      if (PAIR == 2) mma_commit_pair_local(drain_bar);
      else mma_commit(drain_bar);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (globaltimer() - t0 > kTimeoutNs) { *abort_flag = 1; break; }
      }
    }
  } else {
    // --------------------------------------------------------- epilogue ---
    // Each warp owns TMEM lanes [32*quad, 32*quad+32), i.e. 32 output rows, and
    // a contiguous range of the 256 columns (all of them with 4 epilogue warps,
    // one half with 8), moved out 32 columns at a time: tcgen05.ld -> epilogue arithmetic in
    // registers -> swizzled staging tile in shared memory -> TMA store (which
    // clips rows/columns outside the matrix). Symmetric outputs skip chunks
    // below the diagonal, store chunks above it twice (direct and mirrored)
    // and symmetrise the diagonal chunk in shared memory before one store.
    const int quad = warp & 3;
    constexpr int CPW = (BN / 32) / (EW / 4);     // chunks of 32 columns per warp
    const int ch_lo = ((warp - 2) >> 2) * CPW;    // this warp's first chunk
    const uint32_t st_base = smem_u32(epi_smem) + static_cast<uint32_t>(warp - 2) * EPI_WARP_BYTES;
    const uint32_t tempty0 = PAIR == 2 ? map_to_rank(smem_u32(&tempty_bar[0]), 0) : 0u;
    const uint32_t tempty1 = PAIR == 2 ? map_to_rank(smem_u32(&tempty_bar[1]), 0) : 0u;
    int local = 0;
    const Epilogue& e = p.e;
    const bool vec_c = e.C && ((e.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(e.C) & 15) == 0) &&
                       ((e.strideC & 7) == 0);
    constexpr bool want_rsq = RSQ != 0;
    for (int t = unit; t < p.total_tiles; t += nunits, ++local) {
      int b, tm, tn;
      tile_coords(p, t, b, tm, tn);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag)) break;
      fence_after_sync();
      const int r0 = tm * G::TILE_M + static_cast<int>(rank) * BM + quad * 32;
      const int row = r0 + lane;
      const float sc = e.scale ? e.alpha * e.scale[b] : e.alpha;
      const uint16_t* Cb = e.C ? e.C + static_cast<int64_t>(b) * e.strideC : nullptr;
      float rsq = 0.f;
      // chunks this warp moves out (warp-uniform): inside the matrix and, for
      // symmetric outputs, on or above the diagonal
      uint32_t todo = 0;
#pragma unroll
      for (int ch = ch_lo; ch < ch_lo + CPW; ++ch) {
        const int c0 = tn * BN + ch * 32;
        const bool skip = (c0 >= p.N) || (r0 >= p.M) || (SYM && (c0 + 32 <= r0));
        if (!skip) todo |= 1u << ch;
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
      uint32_t cur[32], nxt[32];
      // C rows (KIND != 0) are fetched one chunk ahead, like the accumulator,
      // so their L2 latency overlaps the current chunk's arithmetic and stores
      uint4 craw[4], cnext[4];
      auto c_fetch = [&](int chn, uint4* dst) {
        const int cc0 = tn * BN + chn * 32;
        if (KIND != 0 && row < p.M && vec_c && cc0 + 32 <= p.N) {
          const uint4* src = reinterpret_cast<const uint4*>(Cb + static_cast<int64_t>(row) * e.ldc + cc0);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = src[q];
        }
      };
      int ch = todo ? __ffs(todo) - 1 : -1;
      if (ch >= 0) {
        __syncwarp();
        tmem_ld32_issue(tbase + ch * 32, cur);
        c_fetch(ch, craw);
        tmem_ld_wait();
      }
      int slot = 0;
#pragma unroll 1
      while (ch >= 0) {
        const uint32_t rest = todo & ~((2u << ch) - 1u);
        const int nch = rest ? __ffs(rest) - 1 : -1;
        if (nch >= 0) {
          tmem_ld32_issue(tbase + nch * 32, nxt);  // overlaps this chunk's work
          c_fetch(nch, cnext);
        }
        const int c0 = tn * BN + ch * 32;
        const bool diag = SYM && (c0 == r0);
        float cv[32];
        if (KIND != 0) {
          if (row >= p.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) cv[j] = 0.f;
          } else if (vec_c && (c0 + 32 <= p.N)) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t w[4] = {craw[q].x, craw[q].y, craw[q].z, craw[q].w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                cv[q * 8 + 2 * h] = h16_to_f32(static_cast<uint16_t>(w[h] & 0xFFFFu), DHALF);
                cv[q * 8 + 2 * h + 1] = h16_to_f32(static_cast<uint16_t>(w[h] >> 16), DHALF);
              }
            }
          } else {
            load_row32(Cb, e.ldc, row, c0, p.M, p.N, false, DHALF, cv);
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float x0 = epi_value<KIND>(p, __uint_as_float(cur[j]), KIND != 0 ? cv[j] : 0.f, sc, row, c0 + j);
          const float x1 =
              epi_value<KIND>(p, __uint_as_float(cur[j + 1]), KIND != 0 ? cv[j + 1] : 0.f, sc, row, c0 + j + 1);
          pk[j >> 1] = pack2<DHALF>(x0, x1);
          if (want_rsq) {
            const float y0 = unpack_lo<DHALF>(pk[j >> 1]), y1 = unpack_hi<DHALF>(pk[j >> 1]);
            if (c0 + j < p.N) rsq = fmaf(y0, y0, rsq);
            if (c0 + j + 1 < p.N) rsq = fmaf(y1, y1, rsq);
          }
        }
        const uint32_t st_direct = st_base + static_cast<uint32_t>(slot) * 2u * EPI_TILE_BYTES;
        const uint32_t st_mirror = st_direct + EPI_TILE_BYTES;
        // the stores issued from this slot two chunks ago must have read it
        if (lane == 0) bulk_wait_read1();
        __syncwarp();
        if (!diag) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_shared_v4(st_direct + stage_off(lane, q * 8), pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          if (SYM) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint16_t h = static_cast<uint16_t>(j & 1 ? (pk[j >> 1] >> 16) : (pk[j >> 1] & 0xFFFFu));
              st_shared_u16(st_mirror + stage_off(j, lane), h);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j >= lane) {
              const uint16_t h = static_cast<uint16_t>(j & 1 ? (pk[j >> 1] >> 16) : (pk[j >> 1] & 0xFFFFu));
              st_shared_u16(st_direct + stage_off(lane, j), h);
              st_shared_u16(st_direct + stage_off(j, lane), h);
            }
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmD, st_direct, c0, r0, b);
          if (SYM && !diag) tma_store_3d(&tmD, st_mirror, r0, c0, b);
          bulk_commit();
        }
        slot ^= 1;
        if (nch >= 0) {
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) cur[j] = nxt[j];
          if (KIND != 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q) craw[q] = cnext[q];
          }
        }
        ch = nch;
      }
      fence_before_sync();
      if (PAIR == 2) mbar_arrive_cluster(acc ? tempty1 : tempty0);
      else mbar_arrive(&tempty_bar[acc]);
      if (want_rsq && row < p.M)
        e.rowsq[(static_cast<int64_t>(b) * p.tiles_n + tn) * p.M + row] = rsq;
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  fence_before_sync();
  __syncthreads();
  pdl_trigger();  // this CTA's work is done: the next kernel may start launching
  if (PAIR == 2) cluster_sync();  // the pair's MMAs, loads and remote arrivals are finished
  if (threadIdx.x == 0 && *abort_flag) atomicOr(p.err, kErrWaitTimeout);
  (void)DHALF;
  if (warp == 1) {
    __syncwarp();
    fence_after_sync();
    if (PAIR == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                   : "memory");
  }
}

// ------------------------------------------------------ host-side setup ---
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// A tensor map is a pure function of its encode arguments (address, type,
// dims, strides, box, swizzle, promotion), so encoded maps are kept and
// reused: a step encodes the same ~90 maps every time it runs.
struct MapKey {
  uint64_t addr;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  int dtype, swizzle, promo;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(MapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};
static_assert(sizeof(MapKey) % 8 == 0, "MapKey hashes whole words");

static int encode_cached(CUtensorMap* map, CUtensorMapDataType dtype, void* addr, const cuuint64_t* dims,
                         const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
                         CUtensorMapL2promotion promo, const char* what) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey k;
  std::memset(&k, 0, sizeof(k));  // padding bytes take part in the comparison
  k.addr = reinterpret_cast<uint64_t>(addr);
  for (int i = 0; i < 3; ++i) { k.dims[i] = dims[i]; k.box[i] = box[i]; }
  for (int i = 0; i < 2; ++i) k.strides[i] = strides[i];
  k.dtype = static_cast<int>(dtype); k.swizzle = static_cast<int>(swz); k.promo = static_cast<int>(promo);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(k);
    if (it != cache.end()) { *map = it->second; return 0; }
  }
  auto fn = encode_fn();
  if (!fn) { set_error("gemm: cuTensorMapEncodeTiled unavailable"); return -1; }
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, addr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(std::string("gemm: ") + what + " tensor map failed with code " + std::to_string(static_cast<int>(r)));
    return -1;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() >= 8192) cache.clear();
  cache.emplace(k, *map);
  return 0;
}

// rows_box: MN extent of one box for K-major operands (128 for A, 256 for B).
static int make_map(CUtensorMap* map, const Operand& op, int mn, int K, int batch, int rows_box) {
  cuuint64_t dims[3];
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(op.ld) * 2, static_cast<cuuint64_t>(op.stride) * 2};
  cuuint32_t box[3];
  if (op.kmajor) {
    dims[0] = K; dims[1] = mn; box[0] = BK; box[1] = rows_box;
  } else {
    dims[0] = mn; dims[1] = K; box[0] = 64; box[1] = BK;
  }
  dims[2] = batch; box[2] = 1;
  if (batch == 1) strides[1] = strides[0] * dims[1];  // any valid stride
  return encode_cached(map, op.half ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                       const_cast<uint16_t*>(op.ptr), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "operand");
}

// Output map: rows of D (ldd apart) x columns, 32 x 32 boxes, 64-byte swizzle.
static int make_store_map(CUtensorMap* map, const Epilogue& E, int M, int N, int batch) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(E.ldd) * 2, static_cast<cuuint64_t>(E.strideD) * 2};
  if (batch == 1) strides[1] = strides[0] * dims[1];
  cuuint32_t box[3] = {32, 32, 1};
  return encode_cached(map, E.d_half ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, E.D, dims,
                       strides, box, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, "output");
}

}  // namespace tc

// ------------------------------------------------------------- CUDA cores --
// One CTA computes a 256-column row segment of one output row.
__global__ void __launch_bounds__(256) gemm_simt_kernel(Operand A, Operand B, Epilogue E, int M, int N, int K) {
  pdl_wait();
  const int tn = blockIdx.x, row = blockIdx.y, b = blockIdx.z;
  const int col = tn * 256 + threadIdx.x;
  const uint16_t* Ab = A.ptr + static_cast<int64_t>(b) * A.stride;
  const uint16_t* Bb = B.ptr + static_cast<int64_t>(b) * B.stride;
  float acc = 0.f;
  if (col < N) {
    for (int k = 0; k < K; ++k) {
      const float a = h16_to_f32(A.kmajor ? Ab[static_cast<int64_t>(row) * A.ld + k] : Ab[static_cast<int64_t>(k) * A.ld + row], A.half);
      const float bb = h16_to_f32(B.kmajor ? Bb[static_cast<int64_t>(col) * B.ld + k] : Bb[static_cast<int64_t>(k) * B.ld + col], B.half);
      acc = fmaf(a, bb, acc);
    }
  }
  float sq = 0.f;
  if (col < N) {
    const float c = E.C ? h16_to_f32(E.C[static_cast<int64_t>(b) * E.strideC + static_cast<int64_t>(row) * E.ldc + col], E.d_half) : 0.f;
    float x;
    switch (E.kind) {
      case 0: x = acc * (E.scale ? E.alpha * E.scale[b] : E.alpha); break;
      case 1: x = fmaf(E.gamma, acc, fmaf(E.beta, c, row == col ? E.alpha : 0.f)); break;
      case 2: x = round_bf16(round_bf16(E.beta * c) + round_bf16(E.gamma * round_bf16(acc))); break;
      default: x = round_bf16(round_bf16(E.alpha * c) + round_bf16(acc)); break;
    }
    const uint16_t o = f32_to_h16(x, E.d_half);
    E.D[static_cast<int64_t>(b) * E.strideD + static_cast<int64_t>(row) * E.ldd + col] = o;
    const float xr = h16_to_f32(o, E.d_half);
    sq = xr * xr;
  }
  if (E.rowsq) {
    __shared__ float red[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < 8; ++w) t += red[w];
      const int tiles_n = (N + 255) / 256;
      E.rowsq[(static_cast<int64_t>(b) * tiles_n + tn) * M + row] = t;
    }
  }
}

int gemm_simt(const Operand& A, const Operand& B, const Epilogue& E, int M, int N, int K, int batch,
              cudaStream_t stream) {
  dim3 grid((N + 255) / 256, M, batch);
  if (grid.y > 65535u || grid.z > 65535u) { set_error("gemm_simt: problem too large"); return -1; }
  launch_pdl(gemm_simt_kernel, grid, dim3(256), 0, stream, A, B, E, M, N, K);
  count_launch();
  return check_launch("gemm_simt");
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Optional CUDA-event timing of every tensor-core GEMM launch (off by default):
// the benchmark reads the summed device time and the algorithmic FLOPs of the
// launches (symmetric outputs counted at half).
GemmTimer& GemmTimer::instance() {
  static GemmTimer t;
  return t;
}
void GemmTimer::before(cudaStream_t st, double flops) {
  if (!enabled) return;
  std::lock_guard<std::mutex> lk(mu);
  cudaEvent_t a, b;
  if (cudaEventCreate(&a) != cudaSuccess) return;
  if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return; }
  cudaEventRecord(a, st);
  pending.push_back({a, b, flops});
}
void GemmTimer::after(cudaStream_t st) {
  if (!enabled) return;
  std::lock_guard<std::mutex> lk(mu);
  if (!pending.empty()) cudaEventRecord(pending.back().b, st);
}
int GemmTimer::read(double* ms, double* flops, int64_t* launches) {
  std::lock_guard<std::mutex> lk(mu);
  double t = 0.0, f = 0.0;
  for (auto& e : pending) {
    cudaEventSynchronize(e.b);
    float x = 0.f;
    if (cudaEventElapsedTime(&x, e.a, e.b) == cudaSuccess) t += x;
    f += e.flops;
    cudaEventDestroy(e.a);
    cudaEventDestroy(e.b);
  }
  if (ms) *ms = t;
  if (flops) *flops = f;
  if (launches) *launches = static_cast<int64_t>(pending.size());
  pending.clear();
  return 0;
}

bool gemm_tc_supported(const Operand& A, const Operand& B, const Epilogue& E, int M, int N, int K) {
  if (M < tc::BM || N < 128 || K < tc::BK) return false;
  if (!al16(A.ptr) || !al16(B.ptr)) return false;
  if ((A.ld & 7) || (B.ld & 7) || (A.stride & 7) || (B.stride & 7)) return false;
  if (!al16(E.D) || (E.ldd & 7) || (E.strideD & 7)) return false;  // TMA store of the output
  return true;
}

int gemm(const Operand& A, const Operand& B, const Epilogue& E, int M, int N, int K, int batch, int sym,
         cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) { set_error("gemm: empty problem"); return -1; }
  if (!A.ptr || !B.ptr || !E.D) { set_error("gemm: null operand"); return -1; }
  if (E.kind < 0 || E.kind > 3) { set_error("gemm: bad epilogue"); return -1; }
  if (E.kind != 0 && !E.C) { set_error("gemm: epilogue needs C"); return -1; }
  if (sym && M != N) { set_error("gemm: symmetric output needs M == N"); return -1; }
  if (sym && E.rowsq) { set_error("gemm: row sums are not produced for symmetric outputs"); return -1; }
  if (A.half != B.half) { set_error("gemm: A and B must have the same element type"); return -1; }
  if ((E.kind == 2 || E.kind == 3) && (E.d_half || A.half)) {
    set_error("gemm: the quintic epilogues restate bf16 arithmetic and need bf16 data"); return -1;
  }
  if (!gemm_tc_supported(A, B, E, M, N, K)) return gemm_simt(A, B, E, M, N, K, batch, stream);

  // A CTA pair (256-row tiles) once there are rows for both CTAs.
  const int pair = (M >= 256) ? 2 : 1;
  tc::Params p;
  memset(&p, 0, sizeof(p));
  p.M = M; p.N = N; p.K = K; p.batch = batch;
  p.tile_m = tc::BM * pair;
  p.a_kmajor = A.kmajor; p.b_kmajor = B.kmajor; p.sym = sym; p.in_half = A.half;
  p.tiles_m = (M + p.tile_m - 1) / p.tile_m;
  p.tiles_n = (N + tc::BN - 1) / tc::BN;
  if (sym) {
    int cnt = 0;
    for (int tn = 0; tn < p.tiles_n; ++tn) cnt += std::min(p.tiles_m, (tn * tc::BN + tc::BN - 1) / p.tile_m + 1);
    p.tiles_per_batch = cnt;
  } else {
    p.tiles_per_batch = p.tiles_m * p.tiles_n;
  }
  const int64_t total = static_cast<int64_t>(p.tiles_per_batch) * batch;
  if (total > (1ll << 30)) { set_error("gemm: too many tiles"); return -1; }
  p.total_tiles = static_cast<int>(total);
  p.nk = (K + tc::BK - 1) / tc::BK;
  p.e = E;
  p.err = device_error_word();
  if (!p.err) { set_error("gemm: no device error word"); return -1; }
  // rowsq partials are laid out per 256-column tile of the output
  if (E.rowsq && p.tiles_n != (N + 255) / 256) { set_error("gemm: row-sum layout"); return -1; }

  CUtensorMap ma, mb, md;
  if (tc::make_map(&ma, A, M, K, batch, tc::BM)) return -1;
  if (tc::make_map(&mb, B, N, K, batch, tc::BN / pair)) return -1;
  if (tc::make_store_map(&md, E, M, N, batch)) return -1;

  using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const tc::Params);
#define B2O_K(K_, H_, S_, R_) {tc::gemm_tc_kernel<K_, H_, S_, R_, 1>, tc::gemm_tc_kernel<K_, H_, S_, R_, 2>}
  // [kind][d_half][sym][rowsq][pair-1]; invalid combinations are rejected above
  static const KernelFn table[4][2][2][2][2] = {
      {{{B2O_K(0, 0, 0, 0), B2O_K(0, 0, 0, 1)}, {B2O_K(0, 0, 1, 0), {nullptr, nullptr}}},
       {{B2O_K(0, 1, 0, 0), B2O_K(0, 1, 0, 1)}, {B2O_K(0, 1, 1, 0), {nullptr, nullptr}}}},
      {{{B2O_K(1, 0, 0, 0), B2O_K(1, 0, 0, 1)}, {B2O_K(1, 0, 1, 0), {nullptr, nullptr}}},
       {{B2O_K(1, 1, 0, 0), B2O_K(1, 1, 0, 1)}, {B2O_K(1, 1, 1, 0), {nullptr, nullptr}}}},
      {{{B2O_K(2, 0, 0, 0), B2O_K(2, 0, 0, 1)}, {B2O_K(2, 0, 1, 0), {nullptr, nullptr}}},
       {{{nullptr, nullptr}, {nullptr, nullptr}}, {{nullptr, nullptr}, {nullptr, nullptr}}}},
      {{{B2O_K(3, 0, 0, 0), B2O_K(3, 0, 0, 1)}, {B2O_K(3, 0, 1, 0), {nullptr, nullptr}}},
       {{{nullptr, nullptr}, {nullptr, nullptr}}, {{nullptr, nullptr}, {nullptr, nullptr}}}},
  };
#undef B2O_K
  const KernelFn fn = table[E.kind][E.d_half ? 1 : 0][sym ? 1 : 0][E.rowsq ? 1 : 0][pair - 1];
  if (!fn) { set_error("gemm: unsupported epilogue combination"); return -1; }
  const bool ew8 = !E.rowsq;  // tc::EpiWarps
  const int smem_bytes = pair == 1 ? (ew8 ? tc::Geo<1, 8>::SMEM_BYTES : tc::Geo<1, 4>::SMEM_BYTES)
                                   : (ew8 ? tc::Geo<2, 8>::SMEM_BYTES : tc::Geo<2, 4>::SMEM_BYTES);
  const int threads = ew8 ? tc::Geo<1, 8>::THREADS : tc::Geo<1, 4>::THREADS;
  static std::mutex attr_mu;
  static std::vector<std::pair<int, const void*>> configured;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(attr_mu);
    const std::pair<int, const void*> key{dev, reinterpret_cast<const void*>(fn)};
    if (std::find(configured.begin(), configured.end(), key) == configured.end()) {
      cudaError_t ce = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
      if (ce != cudaSuccess) { set_error(std::string("gemm: smem attribute: ") + cudaGetErrorString(ce)); return ce; }
      configured.push_back(key);
    }
  }
  const int units = std::min(p.total_tiles, num_sms() / pair);
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(units * pair, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pair;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  GemmTimer::instance().before(stream, 2.0 * M * N * K * batch * (sym ? 0.5 : 1.0));
  cudaError_t le = cudaLaunchKernelEx(&cfg, fn, ma, mb, md, p);
  GemmTimer::instance().after(stream);
  if (le != cudaSuccess) { set_error(std::string("gemm_tc launch: ") + cudaGetErrorString(le)); return le; }
  count_launch();
  return check_launch("gemm_tc");
}

}  // namespace b2o
