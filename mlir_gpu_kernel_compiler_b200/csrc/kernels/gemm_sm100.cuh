// Persistent, warp-specialised tcgen05 GEMM for sm_100a with a fused pointwise epilogue.
//
//   C[b, i, j] = sum_k A[b, i, k] * B[b, k, j]   (B stored [N,K] K-major, or [K,N] N-major)
//   then the plan's epilogue DAG on the f32 accumulator, stored in the output dtype.
//
// Plan semantics: tensorjit/backends/cuda_backend.py:299-429 (matmul + _epilogue_lines).
//
// Roles (192 threads, one CTA per SM, tiles handed out round-robin):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per stage into
//               128B-swizzled shared memory, completion tracked by mbarrier tx bytes.
//   warp 1      TMEM allocator + MMA issuer: the warp runs the loop converged and one lane
//               picked by elect.sync issues
//               tcgen05.mma.cta_group::1.kind::f16 (128 x BN x 16) four times per stage
//               into a TMEM accumulator; tcgen05.commit frees the smem stage, and
//               a final commit per tile signals the epilogue.
//   warps 2..   epilogue (EPI_WARPS = 4 or 8): tcgen05.ld 32 columns at a time
//               (lane = output row; with 8 warps, two warps share a TMEM lane quadrant
//               and split the tile's columns), generated epilogue functor (bias /
//               GELU / residual ...), 16-byte stores.
// The accumulator is double-buffered in TMEM (2 x BN columns), so the epilogue of
// tile t overlaps the main loop of tile t+1.
//
// Every wait is bounded: after TJ_WAIT_NS of no progress the waiting thread raises
// a CTA-wide abort flag and writes the device status word; all roles then drain
// their in-flight copies / MMAs (again bounded), TMEM is freed, and the kernel
// returns.  No trap, no unbounded spin.
//
// No TMA multicast is used anywhere (loads are plain per-CTA tiled copies).
#pragma once
#include <cuda.h>

#include "tj_common.cuh"

#ifndef TJ_WAIT_NS
#define TJ_WAIT_NS 4000000000ull  // 4 s without progress = failure
#endif

namespace tjg {

TJ_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

TJ_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
TJ_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
TJ_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
TJ_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity` of `bar`.  Returns false on abort / timeout.
TJ_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status, int where,
                      uint64_t budget_ns = TJ_WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tj_globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort_flag) return false;
      if (tj_globaltimer() - t0 > budget_ns) {
        *abort_flag = 1;
        tj_report(status, TJ_STATUS_WAIT_TIMEOUT, where);
        return false;
      }
    }
  }
}

// bounded wait by a whole warp; false (for every lane) unless every lane saw the phase
TJ_DEV bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status, int where,
                           uint64_t budget_ns = TJ_WAIT_NS) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, status, where, budget_ns));
}

TJ_DEV void tma_prefetch(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
TJ_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
TJ_DEV void tma_load_3d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// TMA store of a [box] tile from shared memory (bulk-group completion; out-of-range
// coordinates of the box are clipped by the hardware, so ragged edges are never written).
TJ_DEV void tma_store_3d(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
TJ_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
TJ_DEV void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
TJ_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
TJ_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// UMMA shared-memory matrix descriptor, 128-byte swizzle (sm100 descriptor version 1).
TJ_DEV uint64_t desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f32 accumulation.
constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

TJ_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
TJ_DEV void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Instruction descriptor for kind::tf32 with f32 accumulation (A and B K-major).
constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}
// Warp-converged forms: every lane of the issuing warp executes them with the same
// (warp-uniform) operands and one lane chosen by elect.sync issues the instruction, so the
// descriptors stay in uniform registers (issuing from a lane-0-only branch instead costs
// per-thread -> uniform register moves on every MMA).
TJ_DEV void umma_f16_elect(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
TJ_DEV void umma_tf32_elect(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
TJ_DEV void umma_commit_elect(uint32_t bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar)
      : "memory");
}
TJ_DEV void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
TJ_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols) : "memory");
}
TJ_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
TJ_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
TJ_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TJ_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive f32 columns: thread `lane` receives its row's 32 values.
TJ_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  // the wait names every destination register so no use can be scheduled before it
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Grouped raster over (m, n) tiles inside one batch: GROUP_M m-tiles share the
// same B columns while the whole group sweeps N, so concurrently running CTAs
// reuse A and B tiles through L2.
// Tile order of the persistent kernels: batch by batch; inside a batch, bands of group_n column
// tiles (0 = one band over all of N) are swept one after the other, and inside a band groups of
// group_m row tiles, row tile fastest.  A band keeps its B panels in L2 for the whole sweep over
// the rows, so with a wide K the weights are read from DRAM once per band instead of once per
// wave of row tiles; each A panel is then read once per band.
TJ_DEV void tile_coords(long t, int m_tiles, int n_tiles, int group_m, int group_n, long& b, int& mt, int& nt) {
  const long per_batch = static_cast<long>(m_tiles) * n_tiles;
  b = t / per_batch;
  long r = t - b * per_batch;
  const int gn = (group_n > 0 && group_n < n_tiles) ? group_n : n_tiles;
  const long per_band = static_cast<long>(m_tiles) * gn;  // every band but the last is full
  const int band = static_cast<int>(r / per_band);
  const int n_first = band * gn;
  const int bw = min(n_tiles - n_first, gn);
  r -= static_cast<long>(band) * per_band;
  const long per_group = static_cast<long>(group_m) * bw;
  const int g = static_cast<int>(r / per_group);
  const int first_m = g * group_m;
  const int gsize = min(m_tiles - first_m, group_m);
  const int in_g = static_cast<int>(r - static_cast<long>(g) * per_group);
  mt = first_m + in_g % gsize;
  nt = n_first + in_g / gsize;
}

TJ_DEV void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
TJ_DEV void tma_load_5d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
// Tiled load of a rank-R tensor map at coordinates c[0..R-1].
template <int R>
TJ_DEV void tma_load_nd(uint32_t dst, const CUtensorMap* m, uint32_t bar, const int (&c)[5]) {
  static_assert(R >= 2 && R <= 5, "tensor map rank");
  if constexpr (R == 2) tma_load_2d(dst, m, bar, c[0], c[1]);
  if constexpr (R == 3) tma_load_3d(dst, m, bar, c[0], c[1], c[2]);
  if constexpr (R == 4) tma_load_4d(dst, m, bar, c[0], c[1], c[2], c[3]);
  if constexpr (R == 5) tma_load_5d(dst, m, bar, c[0], c[1], c[2], c[3], c[4]);
}

// Plain coalesced stores of one epilogue warp's staged block: 32 rows x (32 * nch) columns of
// 16-bit outputs, chunk c of the block in stage buffer c (32 rows x 64 bytes each, 16-byte
// pieces swizzled as the TMA-store path writes them: piece ^= (row >> 1) & 3).  With two chunks
// a row is one 128-byte segment (8 lanes, 4 rows per instruction); with one, 64 bytes (4 lanes,
// 8 rows).  Used instead of TMA stores for outputs that may be another GPU's memory, where
// whole-line writes matter most.  Cfg::store16(prm, b, i, j, v) stores 8 elements at (i, j)
// (nothing for rows >= M or columns >= N).
template <class Cfg, class P>
TJ_DEV void staged_store_rows(const P& prm, const uint8_t* stage, uint32_t out_stage, int nch, long b, long row_base,
                              long j0, int lane) {
  if (nch == 2) {
    const int piece = lane & 7;
    const uint8_t* buf = stage + (piece >> 2) * out_stage;
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int row = rr * 4 + (lane >> 3);
      const uint4 v = *reinterpret_cast<const uint4*>(buf + row * 64 + (((piece & 3) ^ ((row >> 1) & 3)) << 4));
      Cfg::store16(prm, b, row_base + row, j0 + piece * 8, v);
    }
  } else {
    const int piece = lane & 3;
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const int row = rr * 8 + (lane >> 2);
      const uint4 v = *reinterpret_cast<const uint4*>(stage + row * 64 + ((piece ^ ((row >> 1) & 3)) << 4));
      Cfg::store16(prm, b, row_base + row, j0 + piece * 8, v);
    }
  }
}

// Cfg provides:
//   static constexpr int BN, STAGES, M, N, K, GROUP_M, GROUP_N, EPI_WARPS, KSPLIT, NSEG; static constexpr long BATCH;
//   (NSEG > 1: static __device__ int segment(int nt), seg_tile0(int g) map a column tile to its B operand)
//   static constexpr bool BF16, B_MN_MAJOR, TMA_STORE, STAGED_STORE, STAGE_LAST;  using OutT = <output type>;
//   static constexpr int A_RANK, B_RANK (2: the operand through a 2-D map [K, mats * rows]; 3..5:
//   read from a transpose's source, with static __device__ void a_coords(long ab, int m0, int k0,
//   int (&c)[5]) / b_coords(long bb, int n0, int k0, int (&c)[5]); B_FOLDED marks the folded B);
//   static __device__ void batch_map(long b, long& a_batch, long& b_batch);
//   template <class P> static __device__ void epilogue(const P& prm, long b, long i, long j0, const float (&acc)[32]);
//     (direct 16-byte stores), or with TMA_STORE:
//   template <class P> static __device__ void epilogue_vals(const P& prm, long b, long i, long j0,
//                                                           const float (&acc)[32], float (&out)[32]);
//     (values only; the kernel stages them in shared memory and stores 32 x 32 tiles with TMA),
//   or with STAGED_STORE: epilogue_vals and store16 (staged, then plain coalesced stores);
//   STAGE_LAST (f32 outputs, partial sums): also epilogue_vals and store4(prm, b, i, j, float4),
//   used on the CTA's last tile (staged in the idle pipeline memory), epilogue on the others
template <class Cfg, class P>
__device__ __forceinline__ void gemm_sm100(const P& prm, int* status, int kernel_id) {
  // 3xTF32 mode (f32 operands): the stage holds hi and lo copies of A and B (written by the
  // split pre-pass), and every k-step issues hi*hi + hi*lo + lo*hi into the f32 accumulator.
  constexpr bool X3 = Cfg::TF32X3;
  constexpr int ESZ = X3 ? 4 : 2;
  constexpr int BM = 128, BK = 128 / ESZ;  // one 128-byte swizzle row of K per stage
  constexpr int UK = 32 / ESZ;             // K of one MMA instruction (16 x 16-bit or 8 x tf32)
  constexpr int OPC = X3 ? 2 : 1;          // operand copies per stage
  constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES;
  constexpr uint32_t A_BYTES = BM * 128;
  constexpr uint32_t B_BYTES = BN * 128;
  constexpr uint32_t STAGE_BYTES = OPC * (A_BYTES + B_BYTES);
  static_assert(!X3 || (!Cfg::B_MN_MAJOR && !Cfg::TMA_STORE), "3xTF32 mode: K-major B, direct stores");
  static_assert(!X3 || (Cfg::A_RANK == 2 && !Cfg::B_FOLDED), "3xTF32 mode reads its copies through 2-D maps");
  constexpr int m_tiles = (Cfg::M + BM - 1) / BM;
  constexpr int n_tiles = (Cfg::N + BN - 1) / BN;
  constexpr int k_blocks = (Cfg::K + BK - 1) / BK;
  // split-K: work item w = (tile w / KSPLIT, k slice w % KSPLIT of KPB k-blocks); the epilogue
  // receives batch index b + slice * BATCH (a partial-sum slice of the workspace)
  constexpr int KSPLIT = Cfg::KSPLIT;
  constexpr int KPB = (k_blocks + KSPLIT - 1) / KSPLIT;
  static_assert(KSPLIT >= 1 && (KSPLIT - 1) * KPB < k_blocks, "every k slice has work");
  constexpr long num_tiles = Cfg::BATCH * m_tiles * n_tiles * KSPLIT;
  constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  constexpr uint32_t IDESC = X3 ? idesc_tf32(BM, BN) : idesc_f16(Cfg::BF16, BM, BN, false, Cfg::B_MN_MAJOR);
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(!Cfg::B_MN_MAJOR || BN % 64 == 0, "N-major B needs BN multiple of 64");
  constexpr int EPI_WARPS = Cfg::EPI_WARPS;
  static_assert(EPI_WARPS == 4 || (EPI_WARPS == 8 && BN % 64 == 0), "epilogue warps");
  constexpr int EPI_COLS = BN / (EPI_WARPS / 4);  // columns of the tile one epilogue warp covers

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                              // stage s: [A (hi)][A lo]
  uint8_t* sB = smem + STAGES * OPC * A_BYTES;     // stage s: [B (hi)][B lo]
  // TMA-store staging: per epilogue warp two 32 x 32 output tiles (64-byte rows, 64B swizzle)
  uint8_t* sOut = sB + STAGES * OPC * B_BYTES;
  constexpr bool STAGED = Cfg::STAGED_STORE;
  static_assert(!(STAGED && (Cfg::TMA_STORE || X3)), "one store path");
  constexpr uint32_t OUT_STAGE = (Cfg::TMA_STORE || STAGED) ? 32 * 32 * 2 : 0;
  // f32 outputs (and split-K partial sums): on the CTA's last tile the pipeline's stage memory is
  // idle once the tile's MMAs have completed, so the epilogue stages its 32 x EPI_COLS block
  // there and writes whole row segments instead of 16 bytes into each of 32 rows per store
  constexpr bool STAGE_LAST = Cfg::STAGE_LAST;
  static_assert(!STAGE_LAST || (!Cfg::TMA_STORE && !STAGED), "one store path");
  static_assert(!STAGE_LAST || EPI_WARPS * 32 * EPI_COLS * 4 <= STAGES * STAGE_BYTES, "staging fits the stages");
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + EPI_WARPS * 2 * OUT_STAGE);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const CUtensorMap* tmA = &prm.tm[0];
  const CUtensorMap* tmB = &prm.tm[1];

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 32 * Cfg::EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch(tmA);
    for (int g = 0; g < Cfg::NSEG; ++g) tma_prefetch(&prm.tm[1 + g]);
    if constexpr (Cfg::TMA_STORE || X3) tma_prefetch(&prm.tm[2]);
    if constexpr (X3) tma_prefetch(&prm.tm[3]);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  tj_pdl_wait();  // the previous kernel of the program is complete and its writes are visible

  // stages the producer filled (and the phase it filled them in): on an abort, the
  // copies still in flight are waited for before shared memory is released
  uint32_t issued_phase[STAGES];
  bool pending[STAGES];
#pragma unroll
  for (int s = 0; s < STAGES; ++s) pending[s] = false;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
#ifdef TJ_TEST_STALL_FIRST_LOAD
      // Failure-path test build only: the first stage is never filled, so the MMA warp's
      // bounded wait on it must run out and report through the status words.
      bool stall_pending = true;
#endif
      for (long w = blockIdx.x; w < num_tiles && ok; w += gridDim.x) {
        const long t = w / KSPLIT;
        const int kb0 = static_cast<int>(w % KSPLIT) * KPB, kb1 = min(kb0 + KPB, k_blocks);
        long b;
        int mt, nt;
        tile_coords(t, m_tiles, n_tiles, Cfg::GROUP_M, Cfg::GROUP_N, b, mt, nt);
        long ab, bb;
        Cfg::batch_map(b, ab, bb);
        const int a_row = static_cast<int>(ab * Cfg::M + static_cast<long>(mt) * BM);
        // several B operands side by side along N (GEMMs sharing A): segment g owns the
        // column tiles from seg_tile0(g), its B rows start at 0 in its own tensor map
        const CUtensorMap* tb = tmB;
        int n0 = nt * BN;
        if constexpr (Cfg::NSEG > 1) {
          const int g = Cfg::segment(nt);
          tb = &prm.tm[1 + g];
          n0 = (nt - Cfg::seg_tile0(g)) * BN;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, status, kernel_id * 16 + 1)) {
            ok = false;
            break;
          }
#ifdef TJ_TEST_STALL_FIRST_LOAD
          if (stall_pending) {
            stall_pending = false;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
#endif
#ifdef TJ_CHECKED
          // checked build: the tile walk stays inside the operands (a TMA load outside them would
          // only zero-fill, so a wrong walk would otherwise go unnoticed); on a violation the CTA
          // aborts like on a timeout
          if (!tj_check(kb * BK < Cfg::K && mt * BM < Cfg::M && ab >= 0 && ab < Cfg::A_MATS && bb >= 0 &&
                            bb < Cfg::B_MATS && n0 >= 0 && n0 < Cfg::N,
                        status, kernel_id * 16 + 15, -1, static_cast<long>(kb))) {
            *abort_flag = 1;
            ok = false;
            break;
          }
#endif
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_expect_tx(fb, STAGE_BYTES);
          uint8_t* a_st = sA + stage * OPC * A_BYTES;
          uint8_t* b_st = sB + stage * OPC * B_BYTES;
          if constexpr (Cfg::A_RANK > 2) {
            // A read in place from a transpose's source: rank-3..5 map, coordinates from the Cfg
            int ac[5] = {0, 0, 0, 0, 0};
            Cfg::a_coords(ab, mt * BM, kb * BK, ac);
            tma_load_nd<Cfg::A_RANK>(smem_u32(a_st), tmA, fb, ac);
          } else {
            tma_load_2d(smem_u32(a_st), tmA, fb, kb * BK, a_row);
          }
          if constexpr (Cfg::B_FOLDED && !Cfg::B_MN_MAJOR) {
            // K-major B read in place from a transpose's source
            int bc[5] = {0, 0, 0, 0, 0};
            Cfg::b_coords(bb, n0, kb * BK, bc);
            tma_load_nd<Cfg::B_RANK>(smem_u32(b_st), tb, fb, bc);
          } else if constexpr (!Cfg::B_MN_MAJOR) {
            tma_load_2d(smem_u32(b_st), tb, fb, kb * BK, static_cast<int>(bb * Cfg::N + n0));
          } else if constexpr (Cfg::B_FOLDED) {
            // N-major B read in place from a transpose's source: the same 64 x 64 chunks
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) {
              int bc[5] = {0, 0, 0, 0, 0};
              Cfg::b_coords(bb, n0 + 64 * c, kb * BK, bc);
              tma_load_nd<Cfg::B_RANK>(smem_u32(b_st + c * (BK * 128)), tmB, fb, bc);
            }
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(smem_u32(b_st + c * (BK * 128)), tmB, fb, n0 + 64 * c, kb * BK, static_cast<int>(bb));
          }
          if constexpr (X3) {
            tma_load_2d(smem_u32(a_st + A_BYTES), &prm.tm[2], fb, kb * BK, a_row);
            tma_load_2d(smem_u32(b_st + B_BYTES), &prm.tm[3], fb, kb * BK, static_cast<int>(bb * Cfg::N + n0));
          }
          pending[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the warp runs the loop converged, elect.sync issues ----------------
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    bool issued_any = false;
    // smem descriptors of stage 0; a stage / k step adds (byte offset >> 4) to the start address
    const uint64_t da0 = desc_sw128(smem_u32(sA), 16, 1024);
    const uint64_t db0 = Cfg::B_MN_MAJOR ? desc_sw128(smem_u32(sB), BK * 128, 1024) : desc_sw128(smem_u32(sB), 16, 1024);
    for (long w = blockIdx.x; w < num_tiles && ok; w += gridDim.x, ++it) {
      const int kb0 = static_cast<int>(w % KSPLIT) * KPB, kb1 = min(kb0 + KPB, k_blocks);
      const int buf = it & 1;
      if (!mbar_wait_warp(smem_u32(&tempty[buf]), ((it >> 1) & 1) ^ 1u, abort_flag, status, kernel_id * 16 + 2)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_warp(smem_u32(&full[stage]), phase, abort_flag, status, kernel_id * 16 + 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a0 = da0 + ((stage * OPC * A_BYTES) >> 4);
        const uint64_t b0 = db0 + ((stage * OPC * B_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < BK / UK; ++kk) {
          const uint64_t ad = a0 + 2 * kk;  // 32 bytes of K per step
          const uint64_t bd = Cfg::B_MN_MAJOR ? b0 + ((kk * UK * 128) >> 4) : b0 + 2 * kk;
          if constexpr (!X3) {
            umma_f16_elect(d, ad, bd, IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
          } else {
            umma_tf32_elect(d, ad, bd, IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
            umma_tf32_elect(d, ad, bd + (B_BYTES >> 4), IDESC, 1u);
            umma_tf32_elect(d, ad + (A_BYTES >> 4), bd, IDESC, 1u);
          }
        }
        umma_commit_elect(smem_u32(&empty[stage]));
        issued_any = true;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit_elect(smem_u32(&tfull[buf]));
    }
    if (!ok && issued_any) {
      // abort: wait for the MMAs already issued before TMEM / smem go away
      umma_commit_elect(smem_u32(drain));
      volatile int no_abort = 0;
      mbar_wait_warp(smem_u32(drain), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
    }
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;                      // TMEM lane quadrant this warp may access
    const int col0 = ((warp - 2) / 4) * EPI_COLS;  // first tile column this warp covers
    uint8_t* stage_out = sOut + (warp - 2) * 2 * OUT_STAGE;
    int sbuf = 0;
    int it = 0;
    for (long w = blockIdx.x; w < num_tiles; w += gridDim.x, ++it) {
      const long t = w / KSPLIT;
      long b;
      int mt, nt;
      tile_coords(t, m_tiles, n_tiles, Cfg::GROUP_M, Cfg::GROUP_N, b, mt, nt);
      b += (w % KSPLIT) * Cfg::BATCH;  // partial-sum slice (KSPLIT > 1)
      const int buf = it & 1;
      const bool ok = mbar_wait(smem_u32(&tfull[buf]), (it >> 1) & 1, abort_flag, status, kernel_id * 16 + 4);
      if (!__all_sync(0xffffffffu, ok)) break;  // the warp leaves together: tcgen05.ld is warp-collective
      tc_fence_after();
      const long i = static_cast<long>(mt) * BM + q * 32 + lane;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + col0);
      if constexpr (STAGE_LAST) {
        if (w + gridDim.x >= num_tiles) {
          // this CTA's last tile: no further loads or MMAs will touch the stage memory
          float* st = reinterpret_cast<float*>(smem) + (warp - 2) * 32 * EPI_COLS;
          constexpr int PR = EPI_COLS / 4;  // 16-byte pieces per staged row (swizzle: piece ^ (row & 7))
#pragma unroll 1
          for (int c = 0; c < EPI_COLS / 32; ++c) {
            TJ_CHECKED_ONLY(if (!tj_check(buf * BN + col0 + c * 32 + 32 <= static_cast<int>(TMEM_COLS), status,
                                          kernel_id * 16 + 15, -2, c)) break;)
            float acc[32];
            tmem_ld32(tbase + c * 32, acc);
            float vals[32];
            Cfg::epilogue_vals(prm, b, i, static_cast<long>(nt) * BN + col0 + c * 32, acc, vals);
#pragma unroll
            for (int cc = 0; cc < 8; ++cc)
              *reinterpret_cast<float4*>(st + lane * EPI_COLS + (((c * 8 + cc) ^ (lane & 7)) << 2)) =
                  make_float4(vals[4 * cc], vals[4 * cc + 1], vals[4 * cc + 2], vals[4 * cc + 3]);
          }
          __syncwarp();
          const long row_base = static_cast<long>(mt) * BM + q * 32;
          const long col_base = static_cast<long>(nt) * BN + col0;
#pragma unroll 4
          for (int it = 0; it < PR; ++it) {  // one 16-byte piece per lane: PR iterations cover 32 rows
            const int idx = it * 32 + lane;
            const int row = idx / PR, p = idx % PR;
            const float4 v = *reinterpret_cast<const float4*>(st + row * EPI_COLS + ((p ^ (row & 7)) << 2));
            Cfg::store4(prm, b, row_base + row, col_base + p * 4, v);
          }
          tc_fence_before();
          mbar_arrive(smem_u32(&tempty[buf]));
          continue;
        }
      }
#pragma unroll 1
      for (int c = 0; c < EPI_COLS / 32; ++c) {
        // checked build: the accumulator columns read lie inside this CTA's TMEM allocation
        TJ_CHECKED_ONLY(if (!tj_check(buf * BN + col0 + c * 32 + 32 <= static_cast<int>(TMEM_COLS), status,
                                      kernel_id * 16 + 15, -2, c)) break;)
        float acc[32];
        tmem_ld32(tbase + c * 32, acc);
        const long j0 = static_cast<long>(nt) * BN + col0 + c * 32;
        if constexpr (STAGED) {
          float vals[32];
          Cfg::epilogue_vals(prm, b, i, j0, acc, vals);
          if ((c & 1) == 0) __syncwarp();  // the previous block's stage reads are done
          uint8_t* dst = stage_out + (c & 1) * OUT_STAGE + lane * 64;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const uint4 v = tj_pack(vals + 8 * cc, static_cast<const typename Cfg::OutT*>(nullptr));
            *reinterpret_cast<uint4*>(dst + ((cc ^ ((lane >> 1) & 3)) << 4)) = v;
          }
          if ((c & 1) || c == EPI_COLS / 32 - 1) {
            __syncwarp();
            const int nch = (c & 1) + 1;
            staged_store_rows<Cfg>(prm, stage_out, OUT_STAGE, nch, b, static_cast<long>(mt) * BM + q * 32,
                                   j0 - 32 * (nch - 1), lane);
          }
        } else if constexpr (!Cfg::TMA_STORE) {
          Cfg::epilogue(prm, b, i, j0, acc);
        } else {
          float vals[32];
          Cfg::epilogue_vals(prm, b, i, j0, acc, vals);
          if (lane == 0) bulk_wait_read1();  // the store issued two chunks ago has left this buffer
          __syncwarp();
          uint8_t* dst = stage_out + sbuf * OUT_STAGE + lane * 64;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const uint4 v = tj_pack(vals + 8 * cc, static_cast<const typename Cfg::OutT*>(nullptr));
            // 64B swizzle: 16-byte chunk index ^= (row >> 1) & 3  (bank-conflict free, matches the tensor map)
            *reinterpret_cast<uint4*>(dst + ((cc ^ ((lane >> 1) & 3)) << 4)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&prm.tm[2], smem_u32(stage_out + sbuf * OUT_STAGE), static_cast<int>(j0),
                         mt * BM + q * 32, static_cast<int>(b));
            bulk_commit();
          }
          sbuf ^= 1;
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[buf]));
    }
    if constexpr (Cfg::TMA_STORE) {
      if (lane == 0) bulk_wait_all();  // every store complete before shared memory is released
      __syncwarp();
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // abort: every copy the producer issued lands before this CTA's shared memory is released
    for (int s = 0; s < STAGES; ++s)
      if (pending[s]) {
        volatile int no_abort = 0;
        mbar_wait(smem_u32(&full[s]), issued_phase[s], &no_abort, status, kernel_id * 16 + 5, 200000000ull);
      }
  }
  // the next kernel of the program may launch once every CTA is here (it still waits for this
  // grid's completion before touching memory); triggered at the end, not at the start, so a
  // persistent kernel does not hold a launched dependent for its whole run
  tj_pdl_launch_dependents();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}


}  // namespace tjg
