// Fused attention for sm_100a: O = softmax(scale * Q K^T) V, one launch per plan pattern
//
//   S = matmul(Q, K, trans_b) [* scale]  ->  row softmax over the key axis  ->  O = matmul(P, V)
//
// which tensorjit plans as three kernels (matmul, row, matmul; the reference backend runs
// them as tensorjit/backends/cuda_backend.py:299-429 and :163-297) that write and re-read the
// [.., Sq, Sk] score and probability matrices through HBM.  Here S and P never leave the SM:
// S lives in TMEM, P (bf16/f16, unnormalised) in shared memory, and the row statistics in
// registers (online softmax: running max m and running sum l per query row; O is divided by
// l once at the end).
//
// One CTA owns two 128-row query tiles of one (batch, head) and streams the K/V blocks of
// that head through a 3-stage TMA ring shared by both tiles.  Roles (384 threads; the
// register budget of 12 warps, 168 per thread, holds a softmax thread's 128 scores without spills):
//   warp 0      TMA producer: both Q tiles once, then K_j / V_j (128 keys x 64) per stage.
//   warp 1      TMEM owner + MMA issuer (one lane):
//                 S_t(j) = Q_t K_j^T      tcgen05.mma 128x128x16 x4   -> TMEM cols [128t, 128t+128)
//                 O_t   += P_t(j) V_j      tcgen05.mma 128x64x16  x8   -> TMEM cols [256+64t, +64)
//               S_t(j+1) is issued as soon as softmax t has read S_t(j) out of TMEM, so the
//               tensor core computes the next scores while the exponentials of block j run.
//   warps 2-3   idle after setup.
//   warps 4-7   softmax for tile 0, warps 8-11 for tile 1 (thread = query row = TMEM lane):
//               tcgen05.ld S row, row max, lazy rescale, p = 2^(s*c - m) (c = scale*log2 e),
//               row sum, P row -> shared memory (K-major, 128B swizzle: the A operand layout
//               of the P V MMA), then the final O / l, stored straight to global memory.
// Lazy rescale: the running max m moves only when a block's max exceeds it by more than
// 8 (log2 units), so p <= 2^8 and the O accumulator is rescaled in TMEM (ld, scale, st)
// only on those rare steps; the result is the same softmax since O and l share m.
//
// Every wait is bounded (TJ_WAIT_NS without progress -> CTA abort flag + device status
// word); on an abort all roles leave their loops together, copies and MMAs in flight are
// drained (bounded), TMEM is freed and the kernel returns.  No TMA multicast.
#pragma once
#include "gemm_sm100.cuh"

namespace tja {
using namespace tjg;

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

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32; 2^-inf = 0).
TJ_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 32 consecutive f32 columns, no wait (the caller waits once for several loads).
TJ_DEV void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Four 32-column loads (128 columns of one lane quadrant) and one wait that names every
// destination register, so no use of them can be scheduled before the data has landed.
TJ_DEV void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
  tmem_ld32_async(taddr, r);
  tmem_ld32_async(taddr + 32, r + 32);
  tmem_ld32_async(taddr + 64, r + 64);
  tmem_ld32_async(taddr + 96, r + 96);
#define TJA_R8(i) "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]), "+r"(r[i + 5]), \
                  "+r"(r[i + 6]), "+r"(r[i + 7])
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : TJA_R8(0), TJA_R8(8), TJA_R8(16), TJA_R8(24), TJA_R8(32), TJA_R8(40), TJA_R8(48), TJA_R8(56),
                 TJA_R8(64), TJA_R8(72), TJA_R8(80), TJA_R8(88), TJA_R8(96), TJA_R8(104), TJA_R8(112), TJA_R8(120)
               :
               : "memory");
#undef TJA_R8
}

// 32 lanes x 32 consecutive f32 columns from registers into TMEM, then wait for the store.
TJ_DEV void tmem_st32_wait(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

template <class T> TJ_DEV uint32_t pack2(float lo, float hi);
template <> TJ_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return tj_pack_bf16x2(lo, hi); }
template <> TJ_DEV uint32_t pack2<__half>(float lo, float hi) { return tj_pack_f16x2(lo, hi); }

// Cfg provides:
//   static constexpr int SQ, SK, D, DV, STAGES, QR, KR, VR (tensor-map ranks);
//   static constexpr long BATCH;  static constexpr bool BF16;  static constexpr float C (scale * log2 e, > 0);
//   using T = element type (__nv_bfloat16 / __half);
//   static __device__ void q_coords(long bh, int s0, int (&c)[5]);   (and k_coords, v_coords)
//   static __device__ long out_offset(long bh, long s);              (element offset of O[bh, s, 0])
// prm.tm[0..2] = Q, K, V tensor maps (box: 64 x 128 rows, 128B swizzle); prm.p[out_arg] = O.
template <class Cfg, class P>
__device__ __forceinline__ void attention_sm100(const P& prm, typename Cfg::T* __restrict__ out, int* status,
                                                int kernel_id) {
  using T = typename Cfg::T;
  constexpr int BM = 128, BN = 128, D = Cfg::D, DV = Cfg::DV, STAGES = Cfg::STAGES;
  static_assert(D == 64 && DV == 64, "head dimension 64");
  constexpr uint32_t Q_BYTES = BM * D * 2;   // 16 KB, [128 rows][64] 128B-swizzled
  constexpr uint32_t K_BYTES = BN * D * 2;   // 16 KB
  constexpr uint32_t V_BYTES = BN * DV * 2;  // 16 KB, [128 keys][64 dv] (N-major B operand)
  constexpr uint32_t P_BYTES = BM * BN * 2;  // 32 KB, two [128][64] K-major chunks
  constexpr int NB = (Cfg::SK + BN - 1) / BN;
  constexpr int LAST_VALID = Cfg::SK - (NB - 1) * BN;  // valid keys in the last block
  constexpr int QPAIRS = (Cfg::SQ + 2 * BM - 1) / (2 * BM);
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t IDESC_S = idesc_f16(Cfg::BF16, BM, BN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16(Cfg::BF16, BM, DV, false, true);
  constexpr float RESCALE_THRESHOLD = 8.0f;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // 2 x Q_BYTES
  uint8_t* sP = sQ + 2 * Q_BYTES;            // 2 x P_BYTES
  uint8_t* sK = sP + 2 * P_BYTES;            // STAGES x K_BYTES
  uint8_t* sV = sK + STAGES * K_BYTES;       // STAGES x V_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + STAGES * V_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;  // [2]
  uint64_t* s_free = s_full + 2;         // [2]
  uint64_t* p_ready = s_free + 2;        // [2]
  uint64_t* o_done = p_ready + 2;        // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
      mbar_init(smem_u32(&kv_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&s_free[t]), 128);
      mbar_init(smem_u32(&p_ready[t]), 128);
      mbar_init(smem_u32(&o_done[t]), 1);
    }
    mbar_init(smem_u32(drain), 1);
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

  // producer bookkeeping for the abort drain: stages with copies possibly in flight
  bool q_pending = false;
  uint32_t pending = 0, issued_phase = 0;  // bit s: stage s filled / parity it was filled in

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int c[5];
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
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, status, kernel_id * 16 + 2) &&
                mbar_wait(smem_u32(&k_full[0]), 0, abort_flag, status, kernel_id * 16 + 2);
      bool issued_any = false;
      auto issue_s = [&](int t, int s) {
        const uint32_t a0 = smem_u32(sQ + t * Q_BYTES), b0 = smem_u32(sK + s * K_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem_base + t * BN, desc_sw128(a0 + kk * 32, 16, 1024), desc_sw128(b0 + kk * 32, 16, 1024), IDESC_S,
                   kk > 0 ? 1u : 0u);
        umma_commit(smem_u32(&s_full[t]));
        issued_any = true;
      };
      auto issue_pv = [&](int t, int s, bool acc) {
        const uint32_t a0 = smem_u32(sP + t * P_BYTES), b0 = smem_u32(sV + s * V_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16(tmem_base + 2 * BN + t * DV, desc_sw128(a0 + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024),
                   desc_sw128(b0 + kk * 16 * 128, BN * 128, 1024), IDESC_O, (acc || kk > 0) ? 1u : 0u);
        umma_commit(smem_u32(&o_done[t]));
        issued_any = true;
      };
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < ntiles; ++t) issue_s(t, 0);
      }
      for (int j = 0; j < NB && ok; ++j) {
        const int s = j % STAGES;
        if (j + 1 < NB) {
          const int s1 = (j + 1) % STAGES;
          if (!mbar_wait(smem_u32(&k_full[s1]), ((j + 1) / STAGES) & 1, abort_flag, status, kernel_id * 16 + 3)) {
            ok = false;
            break;
          }
          for (int t = 0; t < ntiles && ok; ++t) {
            if (!mbar_wait(smem_u32(&s_free[t]), j & 1, abort_flag, status, kernel_id * 16 + 4)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(t, s1);
          }
          if (!ok) break;
        }
        if (!mbar_wait(smem_u32(&v_full[s]), (j / STAGES) & 1, abort_flag, status, kernel_id * 16 + 3)) {
          ok = false;
          break;
        }
        for (int t = 0; t < ntiles && ok; ++t) {
          if (!mbar_wait(smem_u32(&p_ready[t]), j & 1, abort_flag, status, kernel_id * 16 + 5)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, s, j > 0);
        }
        if (!ok) break;
        umma_commit(smem_u32(&kv_empty[s]));  // K_j and V_j are free once every MMA so far is done
      }
      if (!ok && issued_any) {
        umma_commit(smem_u32(drain));
        volatile int no_abort = 0;
        mbar_wait(smem_u32(drain), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax warps ----------------
    const int t = (warp - 4) >> 2;  // query tile
    const int q = warp & 3;         // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;    // row of the tile = TMEM lane
    if (t < ntiles) {
      const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
      const uint32_t tS = tmem_base + lane_off + t * BN;
      const uint32_t tO = tmem_base + lane_off + 2 * BN + t * DV;
      uint8_t* prow = sP + t * P_BYTES + r * 128;
      const int sw = r & 7;
      float m = 0.0f, l = 0.0f;
      bool ok = true;
      for (int j = 0; j < NB; ++j) {
        ok = mbar_wait(smem_u32(&s_full[t]), j & 1, abort_flag, status, kernel_id * 16 + 7);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld128(tS, sr);
        tc_fence_before();
        mbar_arrive(smem_u32(&s_free[t]));  // the tensor core may overwrite S_t now
        float x[128];
#pragma unroll
        for (int i = 0; i < 128; ++i) x[i] = __uint_as_float(sr[i]);
        if (j == NB - 1 && LAST_VALID < BN) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= LAST_VALID) x[i] = -INFINITY;
        }
        float mx0 = x[0], mx1 = x[1], mx2 = x[2], mx3 = x[3];
#pragma unroll
        for (int i = 4; i < 128; i += 4) {
          mx0 = fmaxf(mx0, x[i]);
          mx1 = fmaxf(mx1, x[i + 1]);
          mx2 = fmaxf(mx2, x[i + 2]);
          mx3 = fmaxf(mx3, x[i + 3]);
        }
        const float mblk = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * Cfg::C;
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
        // p = 2^(x*c - m), packed to the element type; the row sum uses the packed values
        uint32_t pk[64];
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float p0 = ex2_approx(fmaf(x[2 * i], Cfg::C, -m));
          const float p1 = ex2_approx(fmaf(x[2 * i + 1], Cfg::C, -m));
          l0 += p0;
          l1 += p1;
          pk[i] = pack2<T>(p0, p1);
        }
        l += l0 + l1;
        // P_t and O_t are the previous P V MMA's operands: wait until it has finished
        if (j > 0) {
          ok = mbar_wait(smem_u32(&o_done[t]), (j - 1) & 1, abort_flag, status, kernel_id * 16 + 8);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int h = 0; h < DV / 32; ++h) {
              float o[32];
              tmem_ld32(tO + h * 32, o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= alpha;
              tmem_st32_wait(tO + h * 32, o);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          // keys 8u..8u+7: chunk u/8 (64 keys), 16-byte unit (u%8) ^ (row%8) of the row
          uint8_t* dst = prow + (u >> 3) * (BM * 128) + (((u & 7) ^ sw) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
        fence_proxy_async_smem();  // generic-proxy P writes -> visible to the tensor core
        tc_fence_before();
        mbar_arrive(smem_u32(&p_ready[t]));
      }
      if (ok) {
        ok = mbar_wait(smem_u32(&o_done[t]), (NB - 1) & 1, abort_flag, status, kernel_id * 16 + 9);
        if (__all_sync(0xffffffffu, ok)) {
          tc_fence_after();
          const int row = q0 + t * BM + r;
          const float inv = 1.0f / l;
          T* orow = out + Cfg::out_offset(bh, row);
#pragma unroll
          for (int h = 0; h < DV / 32; ++h) {
            float o[32];
            tmem_ld32(tO + h * 32, o);
            if (row < Cfg::SQ) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 w;
                w.x = pack2<T>(o[8 * v + 0] * inv, o[8 * v + 1] * inv);
                w.y = pack2<T>(o[8 * v + 2] * inv, o[8 * v + 3] * inv);
                w.z = pack2<T>(o[8 * v + 4] * inv, o[8 * v + 5] * inv);
                w.w = pack2<T>(o[8 * v + 6] * inv, o[8 * v + 7] * inv);
                *reinterpret_cast<uint4*>(orow + h * 32 + 8 * v) = w;
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
    if (q_pending) mbar_wait(smem_u32(q_full), 0, &no_abort, status, kernel_id * 16 + 10, 200000000ull);
    for (int s = 0; s < STAGES; ++s) {
      if (!((pending >> s) & 1u)) continue;
      const uint32_t ph = (issued_phase >> s) & 1u;
      mbar_wait(smem_u32(&k_full[s]), ph, &no_abort, status, kernel_id * 16 + 10, 200000000ull);
      mbar_wait(smem_u32(&v_full[s]), ph, &no_abort, status, kernel_id * 16 + 10, 200000000ull);
    }
  }
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace tja
