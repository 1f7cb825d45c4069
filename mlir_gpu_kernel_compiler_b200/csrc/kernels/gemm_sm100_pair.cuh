// CTA-pair (cta_group::2) variant of the persistent tcgen05 GEMM: one cluster of two CTAs on
// two SMs computes a 256 x BN tile with a single tcgen05.mma.cta_group::2 stream.
//
//   CTA r of the pair holds A rows [m0 + 128 r, +128) and B rows [n0 + r BN/2, +BN/2) of every
//   stage in its own shared memory (same offsets in both CTAs).  The leader (r = 0) issues
//   the MMAs; the hardware reads the two A halves and the two B halves from both SMs, and
//   each CTA's TMEM receives its own 128 accumulator rows x BN columns.  Per SM and k-block
//   this loads 16 KB of A + BN*64 B of B for 128 x BN x 64 MACs: half the B traffic of the
//   single-CTA kernel for the same tile width, which is what lets BN = 256 run 6 stages deep.
//   With Cfg::NSEG > 1 (GEMMs sharing A) each column tile reads its own segment's B map, as
//   in the single-CTA kernel.
//
// Synchronisation (all waits bounded; TJ_WAIT_NS):
//   full[s]    leader only, 1 arrival: the leader's producer arrive.expect_tx's the bytes of
//              both CTAs on its own barrier; each CTA's TMA loads (.cta_group::2) complete
//              there.  The peer's producer only issues loads: a remote arrive with
//              release.cluster semantics on every k-block serialised each iteration behind
//              the previous loads (about 0.8 us per k-block).
//   empty[s]   in both CTAs; the leader's tcgen05.commit multicasts to both (mask 0b11).
//   tfull[b]   in both CTAs; commit multicast after the last k-block of a tile.
//   tempty[b]  leader only, 2 x EPI_WARPS arrivals (one elected lane per epilogue warp of
//              either CTA, remote arrive for the peer).
// An abort in one CTA is forwarded to the other CTA's flag through distributed shared memory.
// No TMA multicast: every load reads global memory into the issuing CTA's own buffer.
#pragma once
#include "gemm_sm100.cuh"

namespace tjg {

TJ_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of this cluster
TJ_DEV uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
TJ_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
TJ_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
TJ_DEV void mbar_expect_tx_remote(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
               "r"(bytes)
               : "memory");
}
TJ_DEV void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// Bounded wait for barriers that also receive arrivals from the peer CTA (the arrivals are
// release.cluster; the data they guard is read by the tensor core after
// tcgen05.fence::after_thread_sync).  A timeout raises this CTA's abort flag and the peer's.
TJ_DEV bool mbar_wait_pair(uint32_t bar, uint32_t parity, volatile int* abort_flag, uint32_t peer_abort, int* status,
                           int where, uint64_t budget_ns = TJ_WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tj_globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort_flag) return false;
      if (tj_globaltimer() - t0 > budget_ns) {
        *abort_flag = 1;
        st_cluster_u32(peer_abort, 1u);
        tj_report(status, TJ_STATUS_WAIT_TIMEOUT, where);
        return false;
      }
    }
  }
}

TJ_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, uint32_t leader_bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(leader_bar), "r"(c0), "r"(c1)
      : "memory");
}
TJ_DEV void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at this shared offset in both CTAs of the pair once the MMAs issued so far complete
TJ_DEV void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n .reg .b16 m;\n mov.b16 m, 3;\n"
      " tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n}\n" ::"r"(
          bar)
      : "memory");
}
// warp-converged forms (all lanes execute, one lane chosen by elect.sync issues)
TJ_DEV void umma_f16_pair_elect(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
TJ_DEV void umma_commit_pair_elect(uint32_t bar) {
  asm volatile(
      "{\n .reg .b16 m;\n .reg .pred e;\n mov.b16 m, 3;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n}\n" ::"r"(
          bar)
      : "memory");
}
TJ_DEV void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
TJ_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
TJ_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

template <class Cfg, class P>
__device__ __forceinline__ void gemm_sm100_pair(const P& prm, int* status, int kernel_id) {
  constexpr int BM = 256, BK = 64;  // pair tile rows; each CTA holds 128
  constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES;
  constexpr int BN_HALF = BN / 2;
  constexpr uint32_t A_BYTES = 128 * BK * 2;
  constexpr uint32_t B_BYTES = BN_HALF * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;  // per CTA
  constexpr int m_tiles = (Cfg::M + BM - 1) / BM;
  constexpr int n_tiles = (Cfg::N + BN - 1) / BN;
  constexpr int k_blocks = (Cfg::K + BK - 1) / BK;
  constexpr long num_tiles = Cfg::BATCH * m_tiles * n_tiles;
  constexpr uint32_t TMEM_COLS = (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512));
  constexpr uint32_t IDESC = idesc_f16(Cfg::BF16, BM, BN, false, false);
  static_assert(BN == 128 || BN == 256, "pair kernel tile width");
  static_assert(!Cfg::B_MN_MAJOR, "pair kernel needs a K-major B");
  constexpr int EPI_WARPS = Cfg::EPI_WARPS;
  static_assert(EPI_WARPS == 8, "pair kernel uses 8 epilogue warps");
  constexpr int EPI_COLS = BN / 2;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * B_BYTES;
  constexpr bool STAGED = Cfg::STAGED_STORE;   // plain coalesced stores through the stage
  static_assert(!Cfg::STAGE_LAST, "last-tile staging is a single-CTA kernel path");
  static_assert(Cfg::A_RANK == 2 && !Cfg::B_FOLDED, "operands read from a transpose's source: single-CTA path");
  static_assert(!(STAGED && Cfg::TMA_STORE), "one store path");
  constexpr uint32_t OUT_STAGE = (Cfg::TMA_STORE || STAGED) ? 32 * 32 * 2 : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + EPI_WARPS * 2 * OUT_STAGE);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const uint32_t peer = rank ^ 1u;
  const long cluster_id = blockIdx.x / 2;
  const long num_clusters = gridDim.x / 2;
  const CUtensorMap* tmA = &prm.tm[0];
  const CUtensorMap* tmB = &prm.tm[1];
  const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int*>(abort_flag)), peer);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 2 * EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch(tmA);
    for (int g = 0; g < Cfg::NSEG; ++g) tma_prefetch(&prm.tm[1 + g]);
    if constexpr (Cfg::TMA_STORE) tma_prefetch(&prm.tm[2]);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any remote access
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  tj_pdl_wait();  // the previous kernel of the program is complete and its writes are visible

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
#ifdef TJ_TEST_STALL_FIRST_LOAD
      // Failure-path test build only: neither CTA fills its first stage, so the leader's MMA
      // wait on it must run out, raise both CTAs' abort flags and report through the status.
      bool stall_pending = true;
#endif
      for (long t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        long b;
        int mt, nt;
        tile_coords(t, m_tiles, n_tiles, Cfg::GROUP_M, Cfg::GROUP_N, b, mt, nt);
        long ab, bb;
        Cfg::batch_map(b, ab, bb);
        const int a_row = static_cast<int>(ab * Cfg::M + static_cast<long>(mt) * BM + rank * 128);
        int b_row = static_cast<int>(bb * Cfg::N + static_cast<long>(nt) * BN + rank * BN_HALF);
        const CUtensorMap* tmBt = tmB;
        if constexpr (Cfg::NSEG > 1) {
          // several B operands side by side along N (GEMMs sharing A): segment g owns the
          // column tiles from seg_tile0(g), its B rows start at 0 in its own tensor map
          const int g = Cfg::segment(nt);
          tmBt = &prm.tm[1 + g];
          b_row = (nt - Cfg::seg_tile0(g)) * BN + static_cast<int>(rank) * BN_HALF;
        }
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_pair(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, peer_abort, status,
                              kernel_id * 16 + 1)) {
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
          // checked build: the tile walk stays inside the operands; a violation aborts both CTAs
          if (!tj_check(kb * BK < Cfg::K && mt * BM < Cfg::M && ab >= 0 && ab < Cfg::A_MATS && bb >= 0 &&
                            bb < Cfg::B_MATS && nt * BN < Cfg::N,
                        status, kernel_id * 16 + 15, -1, static_cast<long>(kb))) {
            *abort_flag = 1;
            st_cluster_u32(peer_abort, 1u);
            ok = false;
            break;
          }
#endif
          const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_expect_tx(smem_u32(&full[stage]), 2 * STAGE_BYTES);
          tma_load_2d_pair(smem_u32(sA + stage * A_BYTES), tmA, leader_full, kb * BK, a_row);
          tma_load_2d_pair(smem_u32(sB + stage * B_BYTES), tmBt, leader_full, kb * BK, b_row);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (leader CTA; the warp runs the loop converged) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      const uint64_t da0 = desc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t db0 = desc_sw128(smem_u32(sB), 16, 1024);
      auto wait_all = [&](uint32_t bar, uint32_t parity, int where) {
        return __all_sync(0xffffffffu, mbar_wait_pair(bar, parity, abort_flag, peer_abort, status, where));
      };
      for (long t = cluster_id; t < num_tiles && ok; t += num_clusters, ++it) {
        const int buf = it & 1;
        if (!wait_all(smem_u32(&tempty[buf]), ((it >> 1) & 1) ^ 1u, kernel_id * 16 + 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!wait_all(smem_u32(&full[stage]), phase, kernel_id * 16 + 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a0 = da0 + ((stage * A_BYTES) >> 4);
          const uint64_t b0 = db0 + ((stage * B_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_pair_elect(d, a0 + 2 * kk, b0 + 2 * kk, IDESC, (kb | kk) != 0 ? 1u : 0u);
          umma_commit_pair_elect(smem_u32(&empty[stage]));
          issued_any = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair_elect(smem_u32(&tfull[buf]));
      }
      if (!ok && issued_any) {
        umma_commit_pair_elect(smem_u32(drain));
        volatile int no_abort = 0;
        mbar_wait_warp(smem_u32(drain), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
      }
    }
  } else {
    // ---------------- epilogue warps (both CTAs) ----------------
    const int q = warp & 3;
    const int col0 = ((warp - 2) / 4) * EPI_COLS;
    uint8_t* stage_out = sOut + (warp - 2) * 2 * OUT_STAGE;
    int sbuf = 0;
    int it = 0;
    for (long t = cluster_id; t < num_tiles; t += num_clusters, ++it) {
      long b;
      int mt, nt;
      tile_coords(t, m_tiles, n_tiles, Cfg::GROUP_M, Cfg::GROUP_N, b, mt, nt);
      const int buf = it & 1;
      const bool ok = mbar_wait_pair(smem_u32(&tfull[buf]), (it >> 1) & 1, abort_flag, peer_abort, status,
                                     kernel_id * 16 + 4);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int row0 = mt * BM + static_cast<int>(rank) * 128 + q * 32;
      const long i = row0 + lane;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + col0);
#pragma unroll 1
      for (int c = 0; c < EPI_COLS / 32; ++c) {
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
            staged_store_rows<Cfg>(prm, stage_out, OUT_STAGE, nch, b, row0, j0 - 32 * (nch - 1), lane);
          }
        } else if constexpr (!Cfg::TMA_STORE) {
          Cfg::epilogue(prm, b, i, j0, acc);
        } else {
          float vals[32];
          Cfg::epilogue_vals(prm, b, i, j0, acc, vals);
          if (lane == 0) bulk_wait_read1();
          __syncwarp();
          uint8_t* dst = stage_out + sbuf * OUT_STAGE + lane * 64;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const uint4 v = tj_pack(vals + 8 * cc, static_cast<const typename Cfg::OutT*>(nullptr));
            *reinterpret_cast<uint4*>(dst + ((cc ^ ((lane >> 1) & 3)) << 4)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&prm.tm[2], smem_u32(stage_out + sbuf * OUT_STAGE), static_cast<int>(j0), row0,
                         static_cast<int>(b));
            bulk_commit();
          }
          sbuf ^= 1;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&tempty[buf]), 0));
    }
    if constexpr (Cfg::TMA_STORE) {
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA leaves while its partner may still touch its shared memory
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0) {
    // abort: copies this CTA issued signal the leader's barriers, so give any still in
    // flight a bounded grace period to land before shared memory is released
    const uint64_t t0 = tj_globaltimer();
    while (tj_globaltimer() - t0 < 2000000ull) __nanosleep(1000);
  }
  __syncthreads();
  // the next kernel of the program may launch once every CTA is here (it still waits for this
  // grid's completion before touching memory); triggered at the end, not at the start, so a
  // persistent kernel does not hold a launched dependent for its whole run
  tj_pdl_launch_dependents();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

}  // namespace tjg
