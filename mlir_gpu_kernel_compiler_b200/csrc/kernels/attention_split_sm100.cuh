// Fused attention for sm_100a, split-row variant: O = softmax(scale * Q K^T) V.
//
// Same roles, tiles and TMA ring as attention_sm100.cuh (one CTA = two 128-row query tiles of
// one head, K/V blocks of 128 keys, 640 threads), but the two softmax threads that share a
// query row no longer exchange their half-row maxima every key block.  Each of them keeps its
// own running max m_h and sum l_h over ITS 64 keys of every block and accumulates its own
// output O_h = sum_j P_h(j) V_h(j) in TMEM (the P V product is split along the keys: the first
// four k-steps of the MMA go to O_0, the last four to O_1).  Softmax is linear in those
// partial results, so once all key blocks are done the row is combined exactly:
//     m = max(m_0, m_1),  a_h = 2^(m_h - m),  O = (a_0 O_0 + a_1 O_1) / (a_0 l_0 + a_1 l_1)
// with one exchange of (m_h, l_h) through shared memory per row instead of one per block.
//
// TMEM (512 columns): S_0 [0,128) S_1 [128,256) O_0,h0 [256,320) O_0,h1 [320,384)
//                     O_1,h0 [384,448) O_1,h1 [448,512).
// P_t,h (64 keys, bf16/f16 packed two per column) is written over the first 32 columns of the
// half row's own scores in S_t, which that thread has already loaded.  The MMA warp therefore
// issues S_t(j+1) only after P_t(j) V_j has completed (it waits on its own commit barrier);
// the other tile's softmax keeps the MUFU busy meanwhile.
//
// Per key block a softmax thread: waits for S_t(j), loads its 64 scores, takes the half-row
// max, rescales lazily (m_h moves only when the block max exceeds it by more than 8 in log2
// units; O_h is then scaled in TMEM after the previous P V has finished), computes
// p = 2^(s c - m_h), stores its 32 P columns and arrives on p_ready.  Every wait is bounded
// (TJ_WAIT_NS); on an abort all roles leave their loops, in-flight copies and MMAs are drained
// (bounded), TMEM is freed and the kernel returns.  No TMA multicast.
#pragma once
#include "attention_sm100.cuh"

namespace tja {

// Cfg: as attention_sm100 (SQ, SK, D, DV, STAGES, QR, KR, VR, EMU, DESYNC, ALT, BATCH, BF16, C, T,
// q_coords / k_coords / v_coords / out_offset; O_NUMEL in a checked build).
template <class Cfg, class P>
__device__ __forceinline__ void attention_split_sm100(const P& prm, typename Cfg::T* __restrict__ out, int* status,
                                                      int kernel_id) {
  using T = typename Cfg::T;
  constexpr int BM = 128, BN = 128, D = Cfg::D, DV = Cfg::DV, STAGES = Cfg::STAGES;
  static_assert(D == 64 && DV == 64, "head dimension 64");
  constexpr uint32_t Q_BYTES = BM * D * 2;
  constexpr uint32_t K_BYTES = BN * D * 2;
  constexpr uint32_t V_BYTES = BN * DV * 2;
  constexpr int NB = (Cfg::SK + BN - 1) / BN;
  constexpr int LAST_VALID = Cfg::SK - (NB - 1) * BN;
  constexpr int QPAIRS = (Cfg::SQ + 2 * BM - 1) / (2 * BM);
  constexpr int SM_THREADS = 256;  // softmax threads per tile
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t O_COL = 2 * BN;  // O_t,h at O_COL + (2 t + h) * DV
  constexpr uint32_t IDESC_S = idesc_f16(Cfg::BF16, BM, BN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16(Cfg::BF16, BM, DV, false, true);
  constexpr float RESCALE_THRESHOLD = 8.0f;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * Q_BYTES;
  uint8_t* sV = sK + STAGES * K_BYTES;
  float* xm = reinterpret_cast<float*>(sV + STAGES * V_BYTES);  // [2 tiles][2 halves][128 rows]: m_h
  float* xl = xm + 2 * 2 * BM;                                   // [2 tiles][2 halves][128 rows]: l_h
  uint64_t* bars = reinterpret_cast<uint64_t*>(xl + 2 * 2 * BM);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;  // [2]
  uint64_t* p_ready = s_full + 2;        // [2]
  uint64_t* o_done = p_ready + 2;        // [2]
  uint64_t* drain = o_done + 2;          // [2]
  uint64_t* xbar = drain + 2;            // [2 tiles x 4 lane quadrants]: the final (m, l) exchange
  uint64_t* turn = xbar + 8;             // [2] (ALT)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(turn + 2);
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
      mbar_init(smem_u32(&kv_empty[s]), ntiles);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&p_ready[t]), SM_THREADS);
      mbar_init(smem_u32(&o_done[t]), 1);
      mbar_init(smem_u32(&drain[t]), 1);
    }
    for (int i = 0; i < 8; ++i) mbar_init(smem_u32(&xbar[i]), 64);
    mbar_init(smem_u32(&turn[0]), SM_THREADS);
    mbar_init(smem_u32(&turn[1]), SM_THREADS);
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
  uint32_t pending = 0, issued_phase = 0;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (as in attention_sm100) ----------------
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
        if (!mbar_wait(smem_u32(&kv_empty[s]), ph ^ 1u, abort_flag, status, kernel_id * 16 + 1)) break;
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
      ok = mbar_wait_warp(smem_u32(q_full), 0, abort_flag, status, kernel_id * 16 + 2) &&
           mbar_wait_warp(smem_u32(&k_full[0]), 0, abort_flag, status, kernel_id * 16 + 2);
    const uint64_t dq = desc_sw128(smem_u32(sQ + t * Q_BYTES), 16, 1024);
    const uint64_t dk0 = desc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = desc_sw128(smem_u32(sV), BN * 128, 1024);
    const uint32_t tS = tmem_base + t * BN;
    const uint32_t tO = tmem_base + O_COL + 2 * t * DV;  // O_t,h0; O_t,h1 follows at + DV
    auto issue_s = [&](int s) {
      const uint64_t b = dk0 + ((s * K_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) umma_f16_elect(tS, dq + 2 * kk, b + 2 * kk, IDESC_S, kk > 0);
      umma_commit_elect(smem_u32(&s_full[t]));
      issued_any = true;
    };
    // O_t,h += P_t,h(j) V_h(j): keys [64 h, 64 h + 64) of the block; P_t,h sits in the first 32
    // columns of the half row's scores (TMEM column S_t + 64 h)
    auto issue_pv = [&](int s, bool acc) {
      const uint64_t b = dv0 + ((s * V_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const int h = kk >> 2, k4 = kk & 3;
        umma_f16_ts_elect(tO + h * DV, tS + h * 64 + k4 * 8, b + ((kk * 16 * 128) >> 4), IDESC_O,
                          (acc || k4 > 0) ? 1u : 0u);
      }
      umma_commit_elect(smem_u32(&o_done[t]));
      issued_any = true;
    };
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < NB && ok; ++j) {
      const int s = j % STAGES;
      if (!mbar_wait_warp(smem_u32(&v_full[s]), (j / STAGES) & 1, abort_flag, status, kernel_id * 16 + 3) ||
          !mbar_wait_warp(smem_u32(&p_ready[t]), j & 1, abort_flag, status, kernel_id * 16 + 5)) {
        ok = false;
        break;
      }
      tc_fence_after();
      issue_pv(s, j > 0);
      umma_commit_elect(smem_u32(&kv_empty[s]));  // this tile is done with K_j and V_j
      if (j + 1 < NB) {
        // S_t(j+1) overwrites P_t(j): wait until P_t(j) V_j has completed
        const int s1 = (j + 1) % STAGES;
        if (!mbar_wait_warp(smem_u32(&k_full[s1]), ((j + 1) / STAGES) & 1, abort_flag, status, kernel_id * 16 + 3) ||
            !mbar_wait_warp(smem_u32(&o_done[t]), j & 1, abort_flag, status, kernel_id * 16 + 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(s1);
      }
    }
    if (!ok && issued_any) {
      umma_commit_elect(smem_u32(&drain[t]));
      volatile int no_abort = 0;
      mbar_wait_warp(smem_u32(&drain[t]), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
    }
  } else if (warp >= 4) {
    // ---------------- softmax warps: warps 4-11 tile 0, 12-19 tile 1 ----------------
    const int t = (warp - 4) >> 3;         // query tile
    const int h = ((warp - 4) >> 2) & 1;   // half of the 128 key columns
    const int q = warp & 3;                // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;           // row of the tile = TMEM lane
    const uint32_t pair_bar = smem_u32(&xbar[t * 4 + q]);
    if (t < ntiles) {
      const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
      const uint32_t tS = tmem_base + lane_off + t * BN + h * 64;    // this half's scores; its P over the first 32
      const uint32_t tO = tmem_base + lane_off + O_COL + 2 * t * DV;  // O_t,h0 (O_t,h1 at + DV)
      float m = -INFINITY, l = 0.0f;
      bool ok = true;
      const bool alt = Cfg::ALT && ntiles == 2;
      if (Cfg::DESYNC && !alt && t == 1)  // start tile 1 one key block behind tile 0
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&p_ready[0]), 0, abort_flag, status, kernel_id * 16 + 11));
      for (int j = 0; j < NB && ok; ++j) {
        ok = mbar_wait(smem_u32(&s_full[t]), j & 1, abort_flag, status, kernel_id * 16 + 7);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld64(tS, sr);
        float x[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(sr[i]);
        if (j == NB - 1 && LAST_VALID < BN) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (h * 64 + i >= LAST_VALID) x[i] = -INFINITY;
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
        // lazy rescale of this half's statistics; the first block always sets m (alpha = 0 then)
        float alpha = 1.0f;
        bool rescale = false;
        if (mblk > m + RESCALE_THRESHOLD) {
          alpha = ex2_approx(m - mblk);
          l *= alpha;
          m = mblk;
          rescale = j > 0;  // O_t,h holds nothing before block 0's P V
        }
        // a half row whose first block is all padding keeps m = -inf: its p are 0
        const float mu = (m == -INFINITY) ? 0.0f : m;
        if (alt && (t == 1 || j > 0)) {
          const bool w = mbar_wait(smem_u32(&turn[t]), (t == 1 ? j : j - 1) & 1, abort_flag, status,
                                   kernel_id * 16 + 13);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
        }
        float l0 = 0.f, l1 = 0.f;
        uint32_t pk[16];
        exp_pairs<0, T, Cfg::EMU>(x, Cfg::C, mu, pk, l0, l1);
        tmem_st16(tS, pk);
        if (alt) mbar_arrive(smem_u32(&turn[t ^ 1]));
        uint32_t pk2[16];
        exp_pairs<16, T, Cfg::EMU>(x, Cfg::C, mu, pk2, l0, l1);
        tmem_st16(tS + 16, pk2);
        l += l0 + l1;
        if (__any_sync(0xffffffffu, rescale)) {
          // O_t,h *= alpha.  No P V is in flight: S_t(j) was issued after P_t(j-1) V completed.
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(tO + h * DV + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32_wait(tO + h * DV + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&p_ready[t]));
      }
      if (ok) {
        // combine the two half rows: m = max(m_0, m_1), O = (a_0 O_0 + a_1 O_1) / (a_0 l_0 + a_1 l_1)
        xm[(t * 2 + h) * BM + r] = m;
        xl[(t * 2 + h) * BM + r] = l;
        mbar_arrive(pair_bar);
        ok = mbar_wait(pair_bar, 0, abort_flag, status, kernel_id * 16 + 12) &&
             mbar_wait(smem_u32(&o_done[t]), (NB - 1) & 1, abort_flag, status, kernel_id * 16 + 9);
        if (__all_sync(0xffffffffu, ok)) {
          const float m0 = xm[(t * 2) * BM + r], m1 = xm[(t * 2 + 1) * BM + r];
          const float l0 = xl[(t * 2) * BM + r], l1 = xl[(t * 2 + 1) * BM + r];
          const float mm = fmaxf(m0, m1);
          const float a0 = (m0 == -INFINITY) ? 0.0f : ex2_approx(m0 - mm);
          const float a1 = (m1 == -INFINITY) ? 0.0f : ex2_approx(m1 - mm);
          const float inv = 1.0f / (a0 * l0 + a1 * l1);
          const float w0 = a0 * inv, w1 = a1 * inv;
          tc_fence_after();
          const int row = q0 + t * BM + r;
          float o0[32], o1[32];
          tmem_ld32(tO + h * 32, o0);       // O_t,h0, this thread's 32 output columns
          tmem_ld32(tO + DV + h * 32, o1);  // O_t,h1, the same columns
          bool store = row < Cfg::SQ;
#ifdef TJ_CHECKED
          if (store)
            store = tj_check(Cfg::out_offset(bh, row) >= 0 && Cfg::out_offset(bh, row) + h * 32 + 32 <= Cfg::O_NUMEL,
                             status, kernel_id * 16 + 15, -3, row);
#endif
          if (store) {
            T* orow = out + Cfg::out_offset(bh, row) + h * 32;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) f[u] = fmaf(o0[8 * v + u], w0, o1[8 * v + u] * w1);
              uint4 w;
              w.x = pack2<T>(f[0], f[1]);
              w.y = pack2<T>(f[2], f[3]);
              w.z = pack2<T>(f[4], f[5]);
              w.w = pack2<T>(f[6], f[7]);
              *reinterpret_cast<uint4*>(orow + 8 * v) = w;
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
    if (q_pending) mbar_wait(smem_u32(q_full), 0, &no_abort, status, kernel_id * 16 + 10, 200000000ull);
    for (int s = 0; s < STAGES; ++s) {
      if (!((pending >> s) & 1u)) continue;
      const uint32_t ph = (issued_phase >> s) & 1u;
      mbar_wait(smem_u32(&k_full[s]), ph, &no_abort, status, kernel_id * 16 + 10, 200000000ull);
      mbar_wait(smem_u32(&v_full[s]), ph, &no_abort, status, kernel_id * 16 + 10, 200000000ull);
    }
  }
  // the next kernel of the program may launch once every CTA is here (it still waits for this
  // grid's completion before touching memory); triggered at the end, not at the start, so a
  // persistent kernel does not hold a launched dependent for its whole run
  tj_pdl_launch_dependents();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace tja
