// Fused attention for sm_100a, one softmax thread per query row: O = softmax(scale * Q K^T) V.
//
// One CTA owns two 128-row query tiles of one (batch, head) and streams 64-key blocks of K and V
// through a TMA ring (384 threads):
//   warp 0       TMA producer: both Q tiles once, then K_j / V_j (64 keys x 64) per stage.
//   warps 1, 2   MMA issuers for tile 0 / tile 1:  S_t(j) = Q_t K_j^T into S_t[j % 2] (TMEM),
//                O_t += P_t(j) V_j with P_t[j % 2] read from TMEM as the A operand.
//   warp 3       idle after setup.
//   warps 4-7    softmax of tile 0, warps 8-11 of tile 1: thread = query row = TMEM lane; each
//                handles the row's 64 scores of a block alone (no partner thread, no exchange).
// S and P are double-buffered per tile, so the tensor core computes S_t(j+1) while the softmax
// of block j runs, and P_t(j + 1) can be written while P_t(j) V is still in flight.  Every
// barrier is per buffer, so no waiter is ever more than one phase behind.
//
// TMEM (512 columns): S_t[b] at 64 (2 t + b), O_t at 256 + 64 t, P_t[b] at 384 + 32 (2 t + b)
// (64 keys of bf16/f16 packed two per column).
//
// Softmax per block: wait S_t(j), load the 64 scores, release the S buffer, block max, lazy
// rescale (the running max m moves only when the block max exceeds it by more than 8 in log2
// units; O_t is then scaled in TMEM once the previous P V has finished), p = 2^(s c - m) with the
// scale folded into c, sum, P into TMEM, arrive.  O is divided by the row sum once at the end.
// Every wait is bounded (TJ_WAIT_NS); on an abort all roles leave their loops, in-flight copies
// and MMAs are drained (bounded), TMEM is freed and the kernel returns.  No TMA multicast.
#pragma once
#include "attention_sm100.cuh"

namespace tja {

// Cfg: as attention_sm100 (SQ, SK, D, DV, STAGES, QR, KR, VR, EMU, DESYNC, NAP, BATCH, BF16, C, T,
// q_coords / k_coords / v_coords / out_offset; O_NUMEL in a checked build).  The K and V tensor
// maps have 64-row boxes (the Q map 128).
template <class Cfg, class P>
__device__ __forceinline__ void attention_row_sm100(const P& prm, typename Cfg::T* __restrict__ out, int* status,
                                                    int kernel_id) {
  using T = typename Cfg::T;
  constexpr int BM = 128, BN = 64, D = Cfg::D, DV = Cfg::DV, STAGES = Cfg::STAGES;
  static_assert(D == 64 && DV == 64, "head dimension 64");
  constexpr uint32_t Q_BYTES = BM * D * 2;   // 16 KB
  constexpr uint32_t K_BYTES = BN * D * 2;   // 8 KB
  constexpr uint32_t V_BYTES = BN * DV * 2;  // 8 KB
  constexpr int NB = (Cfg::SK + BN - 1) / BN;
  constexpr int LAST_VALID = Cfg::SK - (NB - 1) * BN;
  constexpr int QPAIRS = (Cfg::SQ + 2 * BM - 1) / (2 * BM);
  constexpr int SM_THREADS = 128;  // softmax threads per tile
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t O_COL = 256, P_COL = 384;
  constexpr uint32_t IDESC_S = idesc_f16(Cfg::BF16, BM, BN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16(Cfg::BF16, BM, DV, false, true);
  constexpr float RESCALE_THRESHOLD = 8.0f;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * Q_BYTES;
  uint8_t* sV = sK + STAGES * K_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + STAGES * V_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;  // [tile][buffer]
  uint64_t* s_free = s_full + 4;         // [tile][buffer]
  uint64_t* p_ready = s_free + 4;        // [tile][buffer]
  uint64_t* o_done = p_ready + 4;        // [tile][buffer]: P_t(j) V_j complete, j % 2 = buffer
  uint64_t* drain = o_done + 4;          // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long bh = blockIdx.x / QPAIRS;
  const int q0 = (blockIdx.x % QPAIRS) * 2 * BM;
  const int ntiles = (Cfg::SQ - q0 > BM) ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&kv_empty[s]), ntiles);  // one commit per tile's MMA warp
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&s_free[i]), SM_THREADS);
      mbar_init(smem_u32(&p_ready[i]), SM_THREADS);
      mbar_init(smem_u32(&o_done[i]), 1);
    }
    mbar_init(smem_u32(&drain[0]), 1);
    mbar_init(smem_u32(&drain[1]), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch(&prm.tm[0]);
    tma_prefetch(&prm.tm[1]);
    tma_prefetch(&prm.tm[2]);
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

  bool q_pending = false;
  uint32_t pending = 0, issued_phase = 0;  // producer: stages with copies possibly in flight

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int c[5];
#ifdef TJ_CHECKED
      if (!tj_check(bh >= 0 && bh < Cfg::BATCH && q0 < Cfg::SQ, status, kernel_id * 16 + 15, -1, bh)) *abort_flag = 1;
#endif
      mbar_expect_tx(smem_u32(q_full), ntiles * Q_BYTES);
      for (int t = 0; t < ntiles; ++t) {
        Cfg::q_coords(bh, q0 + t * BM, c);
        tma_load_nd<Cfg::QR>(smem_u32(sQ + t * Q_BYTES), &prm.tm[0], smem_u32(q_full), c);
      }
      q_pending = true;
      for (int j = 0; j < NB; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait_nap<Cfg::NAP>(smem_u32(&kv_empty[s]), ph ^ 1u, abort_flag, status, kernel_id * 16 + 1)) break;
#ifdef TJ_TEST_STALL_FIRST_LOAD
        if (j == 0) continue;  // failure-path test build: K_0 / V_0 never arrive
#endif
        mbar_expect_tx(smem_u32(&k_full[s]), K_BYTES);
        Cfg::k_coords(bh, j * BN, c);
        tma_load_nd<Cfg::KR>(smem_u32(sK + s * K_BYTES), &prm.tm[1], smem_u32(&k_full[s]), c);
        mbar_expect_tx(smem_u32(&v_full[s]), V_BYTES);
        Cfg::v_coords(bh, j * BN, c);
        tma_load_nd<Cfg::VR>(smem_u32(sV + s * V_BYTES), &prm.tm[2], smem_u32(&v_full[s]), c);
        pending |= 1u << s;
        issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuers: warp 1 for tile 0, warp 2 for tile 1 ----------------
    const int t = warp - 1;
    bool ok = t < ntiles;
    bool issued_any = false;
    if (ok)
      ok = mbar_wait_warp_nap<Cfg::NAP>(smem_u32(q_full), 0, abort_flag, status, kernel_id * 16 + 2) &&
           mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&k_full[0]), 0, abort_flag, status, kernel_id * 16 + 2);
    const uint64_t dq = desc_sw128(smem_u32(sQ + t * Q_BYTES), 16, 1024);
    const uint64_t dk0 = desc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = desc_sw128(smem_u32(sV), BN * 128, 1024);
    const uint32_t tS = tmem_base + 64 * (2 * t);      // S_t[b] at + 64 b
    const uint32_t tO = tmem_base + O_COL + 64 * t;
    const uint32_t tP = tmem_base + P_COL + 32 * (2 * t);  // P_t[b] at + 32 b
    auto issue_s = [&](int j) {
      const int s = j % STAGES, b = j & 1;
      const uint64_t kb = dk0 + ((s * K_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) umma_f16_elect(tS + 64 * b, dq + 2 * kk, kb + 2 * kk, IDESC_S, kk > 0);
      umma_commit_elect(smem_u32(&s_full[2 * t + b]));
      issued_any = true;
    };
    auto issue_pv = [&](int j) {
      const int s = j % STAGES, b = j & 1;
      const uint64_t vb = dv0 + ((s * V_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        umma_f16_ts_elect(tO, tP + 32 * b + kk * 8, vb + ((kk * 16 * 128) >> 4), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
      umma_commit_elect(smem_u32(&o_done[2 * t + b]));
      umma_commit_elect(smem_u32(&kv_empty[s]));  // this tile is done with K_j and V_j
      issued_any = true;
    };
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < NB && ok; ++j) {
      if (j + 1 < NB) {
        // S_t(j+1) into buffer (j+1) % 2 once K_{j+1} is in and the softmax has read S_t(j-1)
        const int j1 = j + 1;
        if (!mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&k_full[j1 % STAGES]), (j1 / STAGES) & 1, abort_flag, status,
                                          kernel_id * 16 + 3) ||
            (j1 >= 2 && !mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&s_free[2 * t + (j1 & 1)]), ((j1 - 2) >> 1) & 1,
                                                      abort_flag, status, kernel_id * 16 + 4))) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(j1);
      }
      if (!mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&v_full[j % STAGES]), (j / STAGES) & 1, abort_flag, status,
                                        kernel_id * 16 + 3) ||
          !mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&p_ready[2 * t + (j & 1)]), (j >> 1) & 1, abort_flag, status,
                                        kernel_id * 16 + 5)) {
        ok = false;
        break;
      }
      tc_fence_after();
      issue_pv(j);
    }
    if (!ok && issued_any) {
      umma_commit_elect(smem_u32(&drain[t]));
      volatile int no_abort = 0;
      mbar_wait_warp(smem_u32(&drain[t]), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
    }
  } else if (warp >= 4) {
    // ---------------- softmax: warps 4-7 tile 0, warps 8-11 tile 1; thread = query row ----------------
    const int t = (warp - 4) >> 2;
    const int q = warp & 3;        // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;   // row of the tile = TMEM lane
    if (t < ntiles) {
      const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
      const uint32_t tS = tmem_base + lane_off + 64 * (2 * t);
      const uint32_t tO = tmem_base + lane_off + O_COL + 64 * t;
      const uint32_t tP = tmem_base + lane_off + P_COL + 32 * (2 * t);
      float m = -INFINITY, l = 0.0f;
      bool ok = true;
      if (Cfg::DESYNC && t == 1)  // start tile 1 one key block behind tile 0
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&p_ready[0]), 0, abort_flag, status, kernel_id * 16 + 11));
      for (int j = 0; j < NB && ok; ++j) {
        const int b = j & 1;
        ok = mbar_wait(smem_u32(&s_full[2 * t + b]), (j >> 1) & 1, abort_flag, status, kernel_id * 16 + 7);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld64(tS + 64 * b, sr);
        tc_fence_before();
        mbar_arrive(smem_u32(&s_free[2 * t + b]));  // the tensor core may write S_t(j + 2) here
        float x[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(sr[i]);
        if (j == NB - 1 && LAST_VALID < BN) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= LAST_VALID) x[i] = -INFINITY;
        }
        float mx0 = x[0], mx1 = x[1], mx2 = x[2], mx3 = x[3];
#pragma unroll
        for (int i = 4; i < 60; i += 8) {
          mx0 = fmax3(mx0, x[i], x[i + 4]);
          mx1 = fmax3(mx1, x[i + 1], x[i + 5]);
          mx2 = fmax3(mx2, x[i + 2], x[i + 6]);
          mx3 = fmax3(mx3, x[i + 3], x[i + 7]);
        }
        mx0 = fmax3(mx0, x[60], x[61]);
        mx1 = fmax3(mx1, x[62], x[63]);
        const float mblk = fmax3(mx0, mx1, fmaxf(mx2, mx3)) * Cfg::C;
        float alpha = 1.0f;
        bool rescale = false;
        if (mblk > m + RESCALE_THRESHOLD) {  // also the first block (m = -inf -> alpha = 0)
          alpha = ex2_approx(m - mblk);
          l *= alpha;
          m = mblk;
          rescale = j > 0;  // O_t holds nothing before block 0's P V
        }
        // P_t[b] was last read by P_t(j - 2) V: wait until that has completed
        if (j >= 2) {
          const bool w = mbar_wait(smem_u32(&o_done[2 * t + b]), ((j - 2) >> 1) & 1, abort_flag, status,
                                   kernel_id * 16 + 8);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
        }
        float l0 = 0.f, l1 = 0.f;
        uint32_t pk[16];
        exp_pairs<0, T, Cfg::EMU>(x, Cfg::C, m, pk, l0, l1);
        tmem_st16(tP + 32 * b, pk);
        uint32_t pk2[16];
        exp_pairs<16, T, Cfg::EMU>(x, Cfg::C, m, pk2, l0, l1);
        tmem_st16(tP + 32 * b + 16, pk2);
        l += l0 + l1;
        if (__any_sync(0xffffffffu, rescale)) {
          // O_t *= alpha once P_t(j - 1) V has finished (P_t(j) V is not issued before this arrives)
          const bool w = mbar_wait(smem_u32(&o_done[2 * t + (b ^ 1)]), ((j - 1) >> 1) & 1, abort_flag, status,
                                   kernel_id * 16 + 9);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32_wait(tO + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&p_ready[2 * t + b]));
      }
      if (ok) {
        constexpr int LB = (NB - 1) & 1;
        ok = mbar_wait(smem_u32(&o_done[2 * t + LB]), ((NB - 1) >> 1) & 1, abort_flag, status, kernel_id * 16 + 10);
        if (__all_sync(0xffffffffu, ok)) {
          tc_fence_after();
          const int row = q0 + t * BM + r;
          const float inv = 1.0f / l;
          bool store = row < Cfg::SQ;
#ifdef TJ_CHECKED
          if (store)
            store = tj_check(Cfg::out_offset(bh, row) >= 0 && Cfg::out_offset(bh, row) + DV <= Cfg::O_NUMEL, status,
                             kernel_id * 16 + 15, -3, row);
#endif
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            if (store) {
              T* orow = out + Cfg::out_offset(bh, row) + c * 32;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 w;
                w.x = pack2<T>(o[8 * v + 0] * inv, o[8 * v + 1] * inv);
                w.y = pack2<T>(o[8 * v + 2] * inv, o[8 * v + 3] * inv);
                w.z = pack2<T>(o[8 * v + 4] * inv, o[8 * v + 5] * inv);
                w.w = pack2<T>(o[8 * v + 6] * inv, o[8 * v + 7] * inv);
                *reinterpret_cast<uint4*>(orow + 8 * v) = w;
              }
            }
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // abort: every copy the producer issued lands before this CTA's shared memory is released
    volatile int no_abort = 0;
    if (q_pending) mbar_wait(smem_u32(q_full), 0, &no_abort, status, kernel_id * 16 + 14, 200000000ull);
    for (int s = 0; s < STAGES; ++s) {
      if (!((pending >> s) & 1u)) continue;
      const uint32_t ph = (issued_phase >> s) & 1u;
      mbar_wait(smem_u32(&k_full[s]), ph, &no_abort, status, kernel_id * 16 + 14, 200000000ull);
      mbar_wait(smem_u32(&v_full[s]), ph, &no_abort, status, kernel_id * 16 + 14, 200000000ull);
    }
  }
  // the next kernel of the program may launch once every CTA is here (it still waits for this
  // grid's completion before touching memory); triggered at the end, not at the start, so a
  // persistent kernel does not hold a launched dependent for its whole run
  tj_pdl_launch_dependents();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace tja
