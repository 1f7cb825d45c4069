// Fused attention for sm_100a, four softmax threads per query row and two CTAs per SM:
// O = softmax(scale * Q K^T) V.
//
// One CTA owns ONE 128-row query tile of one (batch, head) and uses 256 TMEM columns (S 128,
// O 64, P 64), so two CTAs share an SM and their softmax warps interleave freely (576 threads,
// 56 registers each):
//   warp 0       TMA producer: Q once, then K_j / V_j (128 keys x 64) through a 2-stage ring.
//   warp 1       MMA issuer and TMEM owner: S(j) = Q K_j^T, then O += P(j) V_j (P from TMEM).
//   warps 2-17   softmax: the thread for (query row r, quarter h) handles keys [32 h, 32 h + 32)
//                of every block: loads its 32 scores, takes the quarter max, exchanges the four
//                quarter maxima of the row through shared memory (one 128-arrival mbarrier per TMEM
//                lane quadrant, one phase per block), rescales lazily (the running max moves only
//                when the block max exceeds it by more than 8 in log2 units; O is then scaled in
//                TMEM), computes p = 2^(s c - m), stores its 16 P columns, and at the end divides
//                its 16 O columns by the row sum (the four quarter sums exchanged the same way).
// Each SM thus runs 32 softmax warps (8 per scheduler) instead of 16, each with half the scores
// per block of the two-threads-per-row kernel.  Every wait is bounded (TJ_WAIT_NS); on an abort all
// roles leave their loops, in-flight copies and MMAs are drained (bounded), TMEM is freed and the
// kernel returns.  No TMA multicast.
#pragma once
#include "attention_sm100.cuh"

namespace tja {

// Cfg: as attention_sm100 (SQ, SK, D, DV, STAGES, QR, KR, VR, EMU, NAP, BATCH, BF16, C, T, q_coords /
// k_coords / v_coords / out_offset; O_NUMEL in a checked build).
template <class Cfg, class P>
__device__ __forceinline__ void attention_quad_sm100(const P& prm, typename Cfg::T* __restrict__ out, int* status,
                                                     int kernel_id) {
  using T = typename Cfg::T;
  constexpr int BM = 128, BN = 128, D = Cfg::D, DV = Cfg::DV, STAGES = Cfg::STAGES;
  static_assert(D == 64 && DV == 64, "head dimension 64");
  constexpr uint32_t Q_BYTES = BM * D * 2;
  constexpr uint32_t K_BYTES = BN * D * 2;
  constexpr uint32_t V_BYTES = BN * DV * 2;
  constexpr int NB = (Cfg::SK + BN - 1) / BN;
  constexpr int LAST_VALID = Cfg::SK - (NB - 1) * BN;
  constexpr int QTILES = (Cfg::SQ + BM - 1) / BM;
  constexpr int SM_THREADS = 512;  // softmax threads (4 per row)
  constexpr uint32_t TMEM_COLS = 256;
  constexpr uint32_t O_COL = BN, P_COL = BN + DV;  // S [0,128) O [128,192) P [192,256)
  constexpr uint32_t IDESC_S = idesc_f16(Cfg::BF16, BM, BN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16(Cfg::BF16, BM, DV, false, true);
  constexpr float RESCALE_THRESHOLD = 8.0f;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;
  uint8_t* sV = sK + STAGES * K_BYTES;
  float* xv = reinterpret_cast<float*>(sV + STAGES * V_BYTES);  // [2 parities][4 quarters][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xv + 2 * 4 * BM);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_ready = s_free + 1;
  uint64_t* o_done = p_ready + 1;
  uint64_t* drain = o_done + 1;
  uint64_t* xbar = drain + 1;  // [4 lane quadrants]: the row exchange of the four quarters
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long bh = blockIdx.x / QTILES;
  const int q0 = (blockIdx.x % QTILES) * BM;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&kv_empty[s]), 1);
    }
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(s_free), SM_THREADS);
    mbar_init(smem_u32(p_ready), SM_THREADS);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(drain), 1);
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&xbar[i]), 128);
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
      // ---------------- TMA producer ----------------
      int c[5];
#ifdef TJ_CHECKED
      if (!tj_check(bh >= 0 && bh < Cfg::BATCH && q0 < Cfg::SQ, status, kernel_id * 16 + 15, -1, bh)) *abort_flag = 1;
#endif
      mbar_expect_tx(smem_u32(q_full), Q_BYTES);
      Cfg::q_coords(bh, q0, c);
      tma_load_nd<Cfg::QR>(smem_u32(sQ), &prm.tm[0], smem_u32(q_full), c);
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
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    bool ok = mbar_wait_warp_nap<Cfg::NAP>(smem_u32(q_full), 0, abort_flag, status, kernel_id * 16 + 2) &&
              mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&k_full[0]), 0, abort_flag, status, kernel_id * 16 + 2);
    bool issued_any = false;
    const uint64_t dq = desc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dk0 = desc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = desc_sw128(smem_u32(sV), BN * 128, 1024);
    const uint32_t tS = tmem_base, tO = tmem_base + O_COL, tP = tmem_base + P_COL;
    auto issue_s = [&](int s) {
      const uint64_t b = dk0 + ((s * K_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) umma_f16_elect(tS, dq + 2 * kk, b + 2 * kk, IDESC_S, kk > 0);
      umma_commit_elect(smem_u32(s_full));
      issued_any = true;
    };
    auto issue_pv = [&](int s, bool acc) {
      const uint64_t b = dv0 + ((s * V_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        umma_f16_ts_elect(tO, tP + kk * 8, b + ((kk * 16 * 128) >> 4), IDESC_O, (acc || kk > 0) ? 1u : 0u);
      umma_commit_elect(smem_u32(o_done));
      issued_any = true;
    };
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < NB && ok; ++j) {
      const int s = j % STAGES;
      if (j + 1 < NB) {
        const int s1 = (j + 1) % STAGES;
        if (!mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&k_full[s1]), ((j + 1) / STAGES) & 1, abort_flag, status,
                                          kernel_id * 16 + 3) ||
            !mbar_wait_warp_nap<Cfg::NAP>(smem_u32(s_free), j & 1, abort_flag, status, kernel_id * 16 + 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(s1);
      }
      if (!mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&v_full[s]), (j / STAGES) & 1, abort_flag, status,
                                        kernel_id * 16 + 3) ||
          !mbar_wait_warp_nap<Cfg::NAP>(smem_u32(p_ready), j & 1, abort_flag, status, kernel_id * 16 + 5)) {
        ok = false;
        break;
      }
      tc_fence_after();
      issue_pv(s, j > 0);
      umma_commit_elect(smem_u32(&kv_empty[s]));
    }
    if (!ok && issued_any) {
      umma_commit_elect(smem_u32(drain));
      volatile int no_abort = 0;
      mbar_wait_warp(smem_u32(drain), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
    }
  } else {
    // ---------------- softmax: warps 2-17, thread = (query row, quarter of the 128 keys) ----------------
    const int h = (warp - 2) >> 2;  // quarter of the key block
    const int q = warp & 3;         // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;    // row of the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + 32 * h;
    const uint32_t tO = tmem_base + lane_off + O_COL + 16 * h;
    const uint32_t tP = tmem_base + lane_off + P_COL + 16 * h;
    const uint32_t xb = smem_u32(&xbar[q]);
    float m = 0.0f, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < NB && ok; ++j) {
      ok = mbar_wait(smem_u32(s_full), j & 1, abort_flag, status, kernel_id * 16 + 7);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[32];
      tmem_ld32(tS, x);
      tc_fence_before();
      mbar_arrive(smem_u32(s_free));  // the tensor core may overwrite S now
      if (j == NB - 1 && LAST_VALID < BN) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (h * 32 + i >= LAST_VALID) x[i] = -INFINITY;
      }
      float mx0 = fmax3(x[0], x[1], x[2]), mx1 = fmax3(x[3], x[4], x[5]);
#pragma unroll
      for (int i = 6; i < 30; i += 4) {
        mx0 = fmax3(mx0, x[i], x[i + 1]);
        mx1 = fmax3(mx1, x[i + 2], x[i + 3]);
      }
      mx0 = fmax3(mx0, x[30], x[31]);
      // the four quarter maxima of the row (shared memory, double-buffered by block parity)
      float* slot = xv + (j & 1) * 4 * BM;
      slot[h * BM + r] = fmaxf(mx0, mx1);
      mbar_arrive(xb);
      const bool w = mbar_wait(xb, j & 1, abort_flag, status, kernel_id * 16 + 12);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      const float mblk = fmaxf(fmaxf(slot[r], slot[BM + r]), fmaxf(slot[2 * BM + r], slot[3 * BM + r])) * Cfg::C;
      float alpha = 1.0f;
      bool rescale = false;
      if (j == 0) {
        m = mblk;
      } else if (mblk > m + RESCALE_THRESHOLD) {
        alpha = ex2_approx(m - mblk);
        l *= alpha;
        m = mblk;
        rescale = true;
      }
      // P and O are operands of the previous P V: wait until it has finished
      if (j > 0) {
        const bool w2 = mbar_wait(smem_u32(o_done), (j - 1) & 1, abort_flag, status, kernel_id * 16 + 8);
        if (!__all_sync(0xffffffffu, w2)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      uint32_t pk[16];
      float l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float a0 = fmaf(x[2 * k], Cfg::C, -m), a1 = fmaf(x[2 * k + 1], Cfg::C, -m);
        const bool emu = k < Cfg::EMU;
        const float p0 = emu ? ex2_poly(a0) : ex2_approx(a0);
        const float p1 = emu ? ex2_poly(a1) : ex2_approx(a1);
        l0 += p0;
        l1 += p1;
        pk[k] = pack2<T>(p0, p1);
      }
      tmem_st16(tP, pk);
      l += l0 + l1;
      if (__any_sync(0xffffffffu, rescale)) {
        float o[16];
        uint32_t ow[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15}, [%16];\ntcgen05.wait::ld.sync.aligned;"
            : "=r"(ow[0]), "=r"(ow[1]), "=r"(ow[2]), "=r"(ow[3]), "=r"(ow[4]), "=r"(ow[5]), "=r"(ow[6]), "=r"(ow[7]),
              "=r"(ow[8]), "=r"(ow[9]), "=r"(ow[10]), "=r"(ow[11]), "=r"(ow[12]), "=r"(ow[13]), "=r"(ow[14]),
              "=r"(ow[15])
            : "r"(tO)
            : "memory");
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[i] = __uint_as_float(ow[i]) * alpha;
          ow[i] = __float_as_uint(o[i]);
        }
        tmem_st16(tO, ow);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(p_ready));
    }
    if (ok) {
      // row sum = the four quarter sums (same m)
      float* slot = xv + (NB & 1) * 4 * BM;
      slot[h * BM + r] = l;
      mbar_arrive(xb);
      ok = mbar_wait(xb, NB & 1, abort_flag, status, kernel_id * 16 + 12) &&
           mbar_wait(smem_u32(o_done), (NB - 1) & 1, abort_flag, status, kernel_id * 16 + 9);
      if (__all_sync(0xffffffffu, ok)) {
        const float inv = 1.0f / (slot[r] + slot[BM + r] + slot[2 * BM + r] + slot[3 * BM + r]);
        tc_fence_after();
        uint32_t ow[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15}, [%16];\ntcgen05.wait::ld.sync.aligned;"
            : "=r"(ow[0]), "=r"(ow[1]), "=r"(ow[2]), "=r"(ow[3]), "=r"(ow[4]), "=r"(ow[5]), "=r"(ow[6]), "=r"(ow[7]),
              "=r"(ow[8]), "=r"(ow[9]), "=r"(ow[10]), "=r"(ow[11]), "=r"(ow[12]), "=r"(ow[13]), "=r"(ow[14]),
              "=r"(ow[15])
            : "r"(tO)
            : "memory");
        const int row = q0 + r;
        bool store = row < Cfg::SQ;
#ifdef TJ_CHECKED
        if (store)
          store = tj_check(Cfg::out_offset(bh, row) >= 0 && Cfg::out_offset(bh, row) + h * 16 + 16 <= Cfg::O_NUMEL,
                           status, kernel_id * 16 + 15, -3, row);
#endif
        if (store) {
          T* orow = out + Cfg::out_offset(bh, row) + h * 16;
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            uint4 wv;
            wv.x = pack2<T>(__uint_as_float(ow[8 * v + 0]) * inv, __uint_as_float(ow[8 * v + 1]) * inv);
            wv.y = pack2<T>(__uint_as_float(ow[8 * v + 2]) * inv, __uint_as_float(ow[8 * v + 3]) * inv);
            wv.z = pack2<T>(__uint_as_float(ow[8 * v + 4]) * inv, __uint_as_float(ow[8 * v + 5]) * inv);
            wv.w = pack2<T>(__uint_as_float(ow[8 * v + 6]) * inv, __uint_as_float(ow[8 * v + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + 8 * v) = wv;
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
