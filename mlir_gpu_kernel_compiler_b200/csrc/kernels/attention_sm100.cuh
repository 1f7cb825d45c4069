// Fused attention for sm_100a: O = softmax(scale * Q K^T) V, one launch per plan pattern
//
//   S = matmul(Q, K, trans_b) [* scale]  ->  row softmax over the key axis  ->  O = matmul(P, V)
//
// which tensorjit plans as three kernels (matmul, row, matmul; the reference backend runs
// them as tensorjit/backends/cuda_backend.py:299-429 and :163-297) that write and re-read the
// [.., Sq, Sk] score and probability matrices through HBM.  Here S and P never leave the SM:
// S and P (bf16/f16, unnormalised) live in TMEM and the row statistics in registers (online
// softmax: running max m and running sum l per query row; O is divided by l once at the end).
//
// One CTA owns two 128-row query tiles of one (batch, head) and streams the K/V blocks of
// that head through a TMA ring shared by both tiles.  Roles (640 threads):
//   warp 0      TMA producer: both Q tiles once, then K_j / V_j (128 keys x 64) per stage.
//   warps 1, 2  MMA issuers for tile 0 / tile 1 (warp 1 also owns TMEM); each runs its loop
//               converged and elect.sync picks the lane that issues each tcgen05.mma / commit:
//                 S_t(j) = Q_t K_j^T    128x128x16 x4, A and B from smem -> TMEM S_t
//                 O_t   += P_t(j) V_j    128x64x16  x8, A = P_t from TMEM -> TMEM O_t
//               S_t(j+1) is issued as soon as softmax t has read S_t(j) out of TMEM, so the
//               tensor core computes the next scores while the exponentials of block j run;
//               one issuer per tile keeps each tile's chain independent of the other's.
//   warp 3      idle after setup.
//   warps 4-11  softmax for tile 0, warps 12-19 for tile 1.  A query row (TMEM lane) is shared
//               by two threads in warps w and w+4 (same lane quadrant), one per half of the
//               128 key columns: tcgen05.ld of its 64 scores, half-row max, the two halves'
//               maxima exchanged through shared memory (one 64-arrival mbarrier per warp pair,
//               one phase per key block, so the wait stays bounded), lazy rescale,
//               p = 2^(s*c - m) (c = scale * log2 e), the half-row sum, 64 P values -> its 32
//               P columns in TMEM; at the end the two half sums are combined and each thread
//               stores its 32 columns of O / l.
// Two threads per row gives 16 softmax warps (4 per SM sub-partition), enough independent
// work to keep the MUFU busy through the TMEM-load and row-max phases of the other warps.
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

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32; 2^-inf = 0).
TJ_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x without MUFU, for the share of exponentials moved to the FMA/ALU pipes:
// x = j + f with j = round(x) (added to the exponent field) and f in [-0.5, 0.5], where
// 2^f is a degree-3 polynomial whose coefficients were fitted here for minimal relative
// error on that interval (Lawson-weighted least squares; max relative error 7.7e-5, below
// half an ulp of the bf16/f16 probabilities it feeds).  Valid for x <= 127; x < -126
// (including -inf for masked keys) returns 2^-126 * 2^f, i.e. 0 after rounding to bf16/f16.
TJ_DEV float ex2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;  // 1.5 * 2^23: x rounded to an integer in the low mantissa bits
  const float f = x - (t - 12582912.0f);
  const float p = fmaf(fmaf(fmaf(0.05522261559963226f, f, 0.24261537194252014f), f, 0.6932516098022461f), f,
                       0.9999275803565979f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// max of three (one PTX max.f32 with three sources, sm_100)
TJ_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Bounded wait that sleeps NAP_NS between polls: for the producer and MMA warps, which wait most
// of the time on the softmax warps; their polls would otherwise take issue slots from the
// softmax warps sharing their scheduler.  NAP_NS = 0 is the plain bounded wait.
template <int NAP_NS>
TJ_DEV bool mbar_wait_nap(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status, int where) {
  if constexpr (NAP_NS == 0) {
    return mbar_wait(bar, parity, abort_flag, status, where);
  } else {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = tj_globaltimer();
    for (uint32_t it = 1;; ++it) {
      __nanosleep(NAP_NS);
      if (mbar_try_wait(bar, parity)) return true;
      if ((it & 7u) == 0) {
        if (*abort_flag) return false;
        if (tj_globaltimer() - t0 > TJ_WAIT_NS) {
          *abort_flag = 1;
          tj_report(status, TJ_STATUS_WAIT_TIMEOUT, where);
          return false;
        }
      }
    }
  }
}
template <int NAP_NS>
TJ_DEV bool mbar_wait_warp_nap(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status, int where) {
  return __all_sync(0xffffffffu, mbar_wait_nap<NAP_NS>(bar, parity, abort_flag, status, where));
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

// Two 32-column loads (64 columns of one lane quadrant) and one wait that names every
// destination register, so no use of them can be scheduled before the data has landed.
TJ_DEV void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  tmem_ld32_async(taddr, r);
  tmem_ld32_async(taddr + 32, r + 32);
#define TJA_R8(i) "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]), "+r"(r[i + 5]), \
                  "+r"(r[i + 6]), "+r"(r[i + 7])
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : TJA_R8(0), TJA_R8(8), TJA_R8(16), TJA_R8(24), TJA_R8(32), TJA_R8(40), TJA_R8(48), TJA_R8(56)
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

// the same for 32 packed words (two bf16/f16 per column)
TJ_DEV void tmem_st32_wait(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// D (TMEM) += A (TMEM) * B (smem descriptor), kind::f16; A is M x 16 with row i in lane i and
// two 16-bit elements per 32-bit column (8 columns per instruction).  Issued by one elected
// lane of a converged warp.
TJ_DEV void umma_f16_ts_elect(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}


// Two f32 values in one 64-bit register pair, for the packed f32x2 FMA / add of sm_100 (each
// lane rounds exactly like fmaf / a plain round-to-nearest add, so results are bit-identical).
TJ_DEV uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
TJ_DEV void f2_unpack(uint64_t v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
TJ_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
TJ_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <class T> TJ_DEV uint32_t pack2(float lo, float hi);
template <> TJ_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return tj_pack_bf16x2(lo, hi); }
template <> TJ_DEV uint32_t pack2<__half>(float lo, float hi) { return tj_pack_f16x2(lo, hi); }

// p = 2^(x*c - m) for the column pairs [I0, I0 + 16) of a 64-column half row, packed two per
// word to the element type; l0 / l1 accumulate the sum of the even / odd columns.  EMU of
// every 16 pairs use ex2_poly (FMA pipe), the rest ex2.approx (MUFU).  F2: the scale-and-shift
// and the running sums as packed f32x2 operations (half the FMA / add instructions, same bits).
template <int I0, class T, int EMU, bool F2 = false>
TJ_DEV void exp_pairs(const float (&x)[64], float c, float m, uint32_t (&pk)[16], float& l0, float& l1) {
  if constexpr (F2) {
    const uint64_t cc = f2_pack(c, c), nm = f2_pack(-m, -m);
    uint64_t ll = f2_pack(l0, l1);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int i = I0 + k;
      float a0, a1;
      f2_unpack(f2_fma(f2_pack(x[2 * i], x[2 * i + 1]), cc, nm), a0, a1);
      const bool emu = (i & 15) < EMU;
      const float p0 = emu ? ex2_poly(a0) : ex2_approx(a0);
      const float p1 = emu ? ex2_poly(a1) : ex2_approx(a1);
      ll = f2_add(ll, f2_pack(p0, p1));
      pk[k] = pack2<T>(p0, p1);
    }
    f2_unpack(ll, l0, l1);
    return;
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int i = I0 + k;
    const float a0 = fmaf(x[2 * i], c, -m), a1 = fmaf(x[2 * i + 1], c, -m);
    const bool emu = (i & 15) < EMU;
    const float p0 = emu ? ex2_poly(a0) : ex2_approx(a0);
    const float p1 = emu ? ex2_poly(a1) : ex2_approx(a1);
    l0 += p0;
    l1 += p1;
    pk[k] = pack2<T>(p0, p1);
  }
}

// exp_pairs that also tracks the maximum of the 32 scores it reads (two chains, h0 / h1)
template <int I0, class T, int EMU>
TJ_DEV void exp_pairs_max(const float (&x)[64], float c, float m, uint32_t (&pk)[16], float& l0, float& l1,
                          float& h0, float& h1) {
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int i = I0 + k;
    if (k & 1)
      h1 = fmax3(h1, x[2 * i], x[2 * i + 1]);
    else
      h0 = fmax3(h0, x[2 * i], x[2 * i + 1]);
    const float a0 = fmaf(x[2 * i], c, -m), a1 = fmaf(x[2 * i + 1], c, -m);
    const bool emu = (i & 15) < EMU;
    const float p0 = emu ? ex2_poly(a0) : ex2_approx(a0);
    const float p1 = emu ? ex2_poly(a1) : ex2_approx(a1);
    l0 += p0;
    l1 += p1;
    pk[k] = pack2<T>(p0, p1);
  }
}

// 16 consecutive 32-bit columns of one lane quadrant from registers into TMEM, then wait.
TJ_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
TJ_DEV void tmem_st16_wait(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};\n"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// 16 columns from registers into TMEM without waiting (tcgen05.wait::st before the data is used)
TJ_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// Cfg provides:
//   static constexpr int SQ, SK, D, DV, STAGES, QR, KR, VR (tensor-map ranks);
//   static constexpr int EMU (exponentials of every 16 column pairs computed by ex2_poly, 0..16);
//   static constexpr bool DESYNC (tile 1 starts one key block behind tile 0);
//   static constexpr bool ALT (the two tiles' exponential phases alternate, one mbarrier token each);
//   static constexpr int NAP (ns the producer and MMA warps sleep between polls; 0 = none);
//   static constexpr bool SPEC (exponentials with the current row max while the block's max is
//   exchanged; recomputed when it moved by more than the rescale threshold);
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
  constexpr int NB = (Cfg::SK + BN - 1) / BN;
  constexpr int LAST_VALID = Cfg::SK - (NB - 1) * BN;  // valid keys in the last block
  constexpr int QPAIRS = (Cfg::SQ + 2 * BM - 1) / (2 * BM);
  constexpr int SM_THREADS = 256;  // softmax threads per tile (8 warps)
  // TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,320) O_1 [320,384)
  //               P_0 [384,448) P_1 [448,512) (128 keys of bf16/f16 packed two per column)
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t P_COL = 2 * BN + 2 * DV;
  constexpr uint32_t IDESC_S = idesc_f16(Cfg::BF16, BM, BN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16(Cfg::BF16, BM, DV, false, true);
  constexpr float RESCALE_THRESHOLD = 8.0f;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // 2 x Q_BYTES
  uint8_t* sK = sQ + 2 * Q_BYTES;            // STAGES x K_BYTES
  uint8_t* sV = sK + STAGES * K_BYTES;       // STAGES x V_BYTES
  float* xmax = reinterpret_cast<float*>(sV + STAGES * V_BYTES);  // [2 parity][2 tiles][2 halves][128 rows]
  float* xsum = xmax + 2 * 2 * 2 * BM;                             // [2 tiles][2 halves][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xsum + 2 * 2 * BM);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;  // [2]
  uint64_t* s_free = s_full + 2;         // [2]
  uint64_t* p_ready = s_free + 2;        // [2]
  uint64_t* o_done = p_ready + 2;        // [2]
  uint64_t* drain = o_done + 2;          // [2]
  uint64_t* xbar = drain + 2;            // [2 tiles x 4 lane quadrants]: half-row exchange
  uint64_t* turn = xbar + 8;             // [2] (ALT): tile t may start its exponentials
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
      mbar_init(smem_u32(&kv_empty[s]), ntiles);  // one commit per tile's MMA warp
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&s_free[t]), SM_THREADS);
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

  // producer bookkeeping for the abort drain: stages with copies possibly in flight
  bool q_pending = false;
  uint32_t pending = 0, issued_phase = 0;  // bit s: stage s filled / parity it was filled in

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int c[5];
#ifdef TJ_CHECKED
      // checked build: this CTA's (batch x head) and query rows lie inside the operands
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
        // Failure-path test build only: K_0 / V_0 are never loaded, so the MMA warps' bounded
        // wait on them must run out and report through the status words.
        if (j == 0) continue;
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
    // smem descriptors built once; stepping through K adds (byte offset >> 4) to the
    // start-address field, so each MMA costs one 64-bit add on warp-uniform values
    const uint64_t dq = desc_sw128(smem_u32(sQ + t * Q_BYTES), 16, 1024);
    const uint64_t dk0 = desc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = desc_sw128(smem_u32(sV), BN * 128, 1024);
    const uint32_t tS = tmem_base + t * BN, tO = tmem_base + 2 * BN + t * DV, tP = tmem_base + P_COL + t * (BN / 2);
    auto issue_s = [&](int s) {
      const uint64_t b = dk0 + ((s * K_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) umma_f16_elect(tS, dq + 2 * kk, b + 2 * kk, IDESC_S, kk > 0);
      umma_commit_elect(smem_u32(&s_full[t]));
      issued_any = true;
    };
    auto issue_pv = [&](int s, bool acc) {
      const uint64_t b = dv0 + ((s * V_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        umma_f16_ts_elect(tO, tP + kk * 8, b + ((kk * 16 * 128) >> 4), IDESC_O, (acc || kk > 0) ? 1u : 0u);
      umma_commit_elect(smem_u32(&o_done[t]));
      issued_any = true;
    };
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    // per key block j: S_t(j+1) as soon as softmax t has read S_t(j) out of TMEM, then
    // O_t += P_t(j) V_j once softmax t has written P_t(j)
    for (int j = 0; j < NB && ok; ++j) {
      const int s = j % STAGES;
      if (j + 1 < NB) {
        const int s1 = (j + 1) % STAGES;
        if (!mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&k_full[s1]), ((j + 1) / STAGES) & 1, abort_flag, status,
                                          kernel_id * 16 + 3) ||
            !mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&s_free[t]), j & 1, abort_flag, status, kernel_id * 16 + 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(s1);
      }
      if (!mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&v_full[s]), (j / STAGES) & 1, abort_flag, status,
                                        kernel_id * 16 + 3) ||
          !mbar_wait_warp_nap<Cfg::NAP>(smem_u32(&p_ready[t]), j & 1, abort_flag, status, kernel_id * 16 + 5)) {
        ok = false;
        break;
      }
      tc_fence_after();
      issue_pv(s, j > 0);
      umma_commit_elect(smem_u32(&kv_empty[s]));  // this tile is done with K_j and V_j
    }
    if (!ok && issued_any) {
      umma_commit_elect(smem_u32(&drain[t]));
      volatile int no_abort = 0;
      mbar_wait_warp(smem_u32(&drain[t]), 0, &no_abort, status, kernel_id * 16 + 6, 200000000ull);
    }
  } else if (warp >= 4) {
    // ---------------- softmax warps ----------------
    const int t = (warp - 4) >> 3;         // query tile
    const int h = ((warp - 4) >> 2) & 1;   // half of the 128 key columns
    const int q = warp & 3;                // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;           // row of the tile = TMEM lane
    const uint32_t pair_bar = smem_u32(&xbar[t * 4 + q]);  // shared by warps w and w+4
    if (t < ntiles) {
      const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
      const uint32_t tS = tmem_base + lane_off + t * BN + h * 64;
      const uint32_t tO = tmem_base + lane_off + 2 * BN + t * DV + h * 32;
      const uint32_t tP = tmem_base + lane_off + P_COL + t * (BN / 2) + h * 32;
      float* my_max = xmax + (t * 2 + h) * BM + r;         // + parity * 4 * BM
      const float* other_max = xmax + (t * 2 + (h ^ 1)) * BM + r;
      float m = 0.0f, l = 0.0f;
      bool ok = true;
      static_assert(!(Cfg::ALT && Cfg::SPEC), "ALT and SPEC are exclusive");
      const bool alt = Cfg::ALT && ntiles == 2;
      if (Cfg::DESYNC && !alt && t == 1) {
        // start tile 1 one key block behind tile 0
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&p_ready[0]), 0, abort_flag, status, kernel_id * 16 + 11));
      }
      for (int j = 0; j < NB && ok; ++j) {
        ok = mbar_wait(smem_u32(&s_full[t]), j & 1, abort_flag, status, kernel_id * 16 + 7);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld64(tS, sr);
        tc_fence_before();
        mbar_arrive(smem_u32(&s_free[t]));  // the tensor core may overwrite S_t now
        float x[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(sr[i]);
        if (j == NB - 1 && LAST_VALID < BN) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (h * 64 + i >= LAST_VALID) x[i] = -INFINITY;
        }
        float l0 = 0.f, l1 = 0.f;
        uint32_t pk[16];
        float alpha = 1.0f;
        bool rescale = false;
        // exchange of the half-row maxima (shared memory, double-buffered by block parity;
        // the arrive releases the store, the completed phase acquires the partner's)
        auto row_max = [&](float hmax, float& mblk) -> bool {
          my_max[(j & 1) * 4 * BM] = hmax;
          mbar_arrive(pair_bar);
          const bool w = mbar_wait(pair_bar, j & 1, abort_flag, status, kernel_id * 16 + 12);
          if (!__all_sync(0xffffffffu, w)) return false;
          mblk = fmaxf(hmax, other_max[(j & 1) * 4 * BM]) * Cfg::C;
          return true;
        };
        // P_t and O_t are operands of the previous P V MMA: wait until it has finished
        auto wait_prev_pv = [&]() -> bool {
          if (j == 0) return true;
          const bool w = mbar_wait(smem_u32(&o_done[t]), (j - 1) & 1, abort_flag, status, kernel_id * 16 + 8);
          if (!__all_sync(0xffffffffu, w)) return false;
          tc_fence_after();
          return true;
        };
        if (!Cfg::SPEC || j == 0) {
          // half-row max first: four independent chains of 3-input maxima
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
          float mblk;
          if (!row_max(fmax3(mx0, mx1, fmaxf(mx2, mx3)), mblk)) {
            ok = false;
            break;
          }
          if (j == 0) {
            m = mblk;
          } else if (mblk > m + RESCALE_THRESHOLD) {
            alpha = ex2_approx(m - mblk);
            l *= alpha;
            m = mblk;
            rescale = true;
          }
          // ALT: the two tiles take turns on the MUFU, so one tile's exponentials overlap the
          // other's TMEM load / row max / exchange instead of both contending at once
          if (alt && (t == 1 || j > 0)) {
            const bool w = mbar_wait(smem_u32(&turn[t]), (t == 1 ? j : j - 1) & 1, abort_flag, status,
                                     kernel_id * 16 + 13);
            if (!__all_sync(0xffffffffu, w)) {
              ok = false;
              break;
            }
          }
          exp_pairs<0, T, Cfg::EMU, Cfg::F2>(x, Cfg::C, m, pk, l0, l1);
          if (!wait_prev_pv()) {
            ok = false;
            break;
          }
          tmem_st16(tP, pk);
          // hand the MUFU to the other tile half-way: its warps wake up while this tile's
          // second half still keeps the unit busy
          if (alt) mbar_arrive(smem_u32(&turn[t ^ 1]));
          uint32_t pk2[16];
          exp_pairs<16, T, Cfg::EMU, Cfg::F2>(x, Cfg::C, m, pk2, l0, l1);
          tmem_st16(tP + 16, pk2);
          tmem_wait_st();
        } else {
          // speculative: the exponentials use the current m while the half-row max is
          // tracked alongside; when the exchanged row max moved by more than the threshold
          // (rare), the block is recomputed with the new m from the scores still in registers
          float hm0 = -INFINITY, hm1 = -INFINITY;
          exp_pairs_max<0, T, Cfg::EMU>(x, Cfg::C, m, pk, l0, l1, hm0, hm1);
          if (!wait_prev_pv()) {
            ok = false;
            break;
          }
          tmem_st16_wait(tP, pk);
          exp_pairs_max<16, T, Cfg::EMU>(x, Cfg::C, m, pk, l0, l1, hm0, hm1);
          tmem_st16_wait(tP + 16, pk);
          float mblk;
          if (!row_max(fmaxf(hm0, hm1), mblk)) {
            ok = false;
            break;
          }
          if (mblk > m + RESCALE_THRESHOLD) {
            alpha = ex2_approx(m - mblk);
            l *= alpha;
            m = mblk;
            rescale = true;
          }
          if (__any_sync(0xffffffffu, rescale)) {
            l0 = 0.f;
            l1 = 0.f;
            exp_pairs<0, T, Cfg::EMU>(x, Cfg::C, m, pk, l0, l1);
            tmem_st16_wait(tP, pk);
            exp_pairs<16, T, Cfg::EMU>(x, Cfg::C, m, pk, l0, l1);
            tmem_st16_wait(tP + 16, pk);
          }
        }
        l += l0 + l1;
        if (__any_sync(0xffffffffu, rescale)) {
          // O_t *= alpha on the rows whose running max moved (this thread's 32 columns)
          float o[32];
          tmem_ld32(tO, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32_wait(tO, o);
        }
        tc_fence_before();
        mbar_arrive(smem_u32(&p_ready[t]));
      }
      if (ok) {
        // row sum = the two halves' sums (same m)
        xsum[(t * 2 + h) * BM + r] = l;
        mbar_arrive(pair_bar);
        ok = mbar_wait(pair_bar, NB & 1, abort_flag, status, kernel_id * 16 + 12) &&
             mbar_wait(smem_u32(&o_done[t]), (NB - 1) & 1, abort_flag, status, kernel_id * 16 + 9);
        if (__all_sync(0xffffffffu, ok)) {
          l += xsum[(t * 2 + (h ^ 1)) * BM + r];
          tc_fence_after();
          const int row = q0 + t * BM + r;
          const float inv = 1.0f / l;
          float o[32];
          tmem_ld32(tO, o);
          bool store = row < Cfg::SQ;
#ifdef TJ_CHECKED
          // checked build: this thread's 32 output columns lie inside O
          if (store)
            store = tj_check(Cfg::out_offset(bh, row) >= 0 && Cfg::out_offset(bh, row) + h * 32 + 32 <= Cfg::O_NUMEL,
                             status, kernel_id * 16 + 15, -3, row);
#endif
          if (store) {
            T* orow = out + Cfg::out_offset(bh, row) + h * 32;
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
