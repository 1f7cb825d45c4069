// tj_b200_linear_f32_noalloc: the f32 linear layer C = A * B^T (3xTF32 on tcgen05) for callers
// that cannot allocate device memory.
//
// Who needs it: code that runs inside a host application which owns every byte of device
// memory (a plugin or custom operator handed raw buffers by a framework's allocator), and
// code on paths where an allocation may block or fail at the worst moment (a latency-bound
// serving loop, a thread that must not take the driver's allocation locks).  Such callers can
// pass inputs and outputs but cannot call cudaMalloc for a workspace.
//
// The regular path (tj_b200_run on a compiled program) keeps the 3xTF32 hi/lo operand copies
// in the program's arena, which tj_b200_program_create allocates.  This entry point does the
// same computation -- split both operands into TF32 hi/lo parts, then
// C = A_hi B_hi^T + A_hi B_lo^T + A_lo B_hi^T with f32 accumulation in TMEM -- but its scratch
// is the file-scope array below, so a call allocates nothing (no cudaMalloc, cudaFree or
// allocating library routine).
//
// Limits and sharing rules:
//   * each operand may hold at most TJ_NOALLOC_MAX_OPERAND (2^21) elements: M*K <= 2^21 and
//     N*K <= 2^21; larger calls are rejected with TJ_ERR_INVALID and a message.  The array
//     (4 x 2^21 floats = 32 MiB) lives on every GPU that loads this library until exit.
//   * K must be a multiple of 4 (16-byte rows for the tensor-memory copies); A, B, C must be
//     16-byte aligned, row-major and contiguous.
//   * every call shares the array and the status words, which keep the previous call's
//     contents; the status words are cleared at the start of each call and the operand copies
//     are rewritten before they are read.  Calls whose work overlaps on the GPU (two streams,
//     or two host threads with different streams) race on the array: serialise them.
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current) and the driver's cuTensorMapEncodeTiled
//     entry point; make that first call before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "../../include/tj_b200.h"
#include "kernels/gemm_sm100.cuh"

// defined in tj_b200_runtime.cpp (same library, not exported)
void tj_b200_internal_set_error(const char* msg);

#define TJ_NOALLOC_MAX_OPERAND (1u << 21)
#define TJ_NOALLOC_MAX_DEVICES 64

// [A hi | A lo | B hi | B lo], each up to TJ_NOALLOC_MAX_OPERAND floats
static __device__ __align__(256) float tj_noalloc_scratch[4 * TJ_NOALLOC_MAX_OPERAND];
static __device__ __align__(16) int tj_noalloc_status[4];

namespace {

constexpr int NA_BM = 128, NA_BN = 64, NA_BK = 32, NA_STAGES = 4;  // BK: 32 f32 = one 128-byte swizzle row
constexpr uint32_t NA_A_BYTES = NA_BM * 128, NA_B_BYTES = NA_BN * 128;
constexpr uint32_t NA_STAGE_BYTES = 2 * (NA_A_BYTES + NA_B_BYTES);
constexpr int NA_SMEM = 1024 + NA_STAGES * NA_STAGE_BYTES + (2 * NA_STAGES + 6) * 8 + 16;

struct NoallocParams {
  float* C;
  int* status;
  int M, N, K;
  int pad;
  CUtensorMap tm[4];  // A hi, B hi, A lo, B lo (all in tj_noalloc_scratch)
};

__global__ void __launch_bounds__(256) noalloc_split(const float4* __restrict__ x, float4* __restrict__ hi,
                                                      float4* __restrict__ lo, long n4) {
  for (long i = static_cast<long>(blockIdx.x) * 256 + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * 256) {
    const float4 v = __ldg(x + i);
    float4 h;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xffffe000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xffffe000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xffffe000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xffffe000u);
    hi[i] = h;
    lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

// Persistent 3xTF32 GEMM with runtime shapes: 1 TMA warp, 1 MMA warp, 4 epilogue warps,
// 128 x 64 tiles, 4 stages, TMEM double-buffered; every wait bounded (TJ_WAIT_NS).
__global__ void __launch_bounds__(192, 1) noalloc_gemm(const __grid_constant__ NoallocParams p) {
  using namespace tjg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + NA_STAGES * 2 * NA_A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + NA_STAGES * 2 * NA_B_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + NA_STAGES;
  uint64_t* tfull = bars + 2 * NA_STAGES;
  uint64_t* tempty = bars + 2 * NA_STAGES + 2;
  uint64_t* drain = bars + 2 * NA_STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * NA_STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t TMEM_COLS = 2 * NA_BN;
  constexpr uint32_t IDESC = idesc_tf32(NA_BM, NA_BN);

  const int m_tiles = (p.M + NA_BM - 1) / NA_BM, n_tiles = (p.N + NA_BN - 1) / NA_BN;
  const int k_blocks = (p.K + NA_BK - 1) / NA_BK;
  const long num_tiles = static_cast<long>(m_tiles) * n_tiles;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NA_STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 128);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < 4; ++i) tma_prefetch(&p.tm[i]);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  uint32_t issued_phase[NA_STAGES];
  bool pending[NA_STAGES];
  for (int s = 0; s < NA_STAGES; ++s) pending[s] = false;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
#ifdef TJ_TEST_STALL_FIRST_LOAD
      // Failure-path test build only: the first stage is never filled, so the MMA warp's
      // bounded wait on it runs out and the status words report it.
      bool stall_pending = true;
#endif
      for (long t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int mt = static_cast<int>(t % m_tiles), nt = static_cast<int>(t / m_tiles);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.status, 1)) {
            ok = false;
            break;
          }
#ifdef TJ_TEST_STALL_FIRST_LOAD
          if (stall_pending) {
            stall_pending = false;
            if (++stage == NA_STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
#endif
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_expect_tx(fb, NA_STAGE_BYTES);
          uint8_t* a_st = sA + stage * 2 * NA_A_BYTES;
          uint8_t* b_st = sB + stage * 2 * NA_B_BYTES;
          tma_load_2d(smem_u32(a_st), &p.tm[0], fb, kb * NA_BK, mt * NA_BM);
          tma_load_2d(smem_u32(b_st), &p.tm[1], fb, kb * NA_BK, nt * NA_BN);
          tma_load_2d(smem_u32(a_st + NA_A_BYTES), &p.tm[2], fb, kb * NA_BK, mt * NA_BM);
          tma_load_2d(smem_u32(b_st + NA_B_BYTES), &p.tm[3], fb, kb * NA_BK, nt * NA_BN);
          pending[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == NA_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true, issued_any = false;
      for (long t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!mbar_wait(smem_u32(&tempty[buf]), ((it >> 1) & 1) ^ 1u, abort_flag, p.status, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * NA_BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.status, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * 2 * NA_A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * 2 * NA_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < NA_BK / 8; ++kk) {
            const uint64_t ah = desc_sw128(a0 + kk * 32, 16, 1024), al = desc_sw128(a0 + NA_A_BYTES + kk * 32, 16, 1024);
            const uint64_t bh = desc_sw128(b0 + kk * 32, 16, 1024), bl = desc_sw128(b0 + NA_B_BYTES + kk * 32, 16, 1024);
            umma_tf32(d, ah, bh, IDESC, (kb | kk) != 0 ? 1u : 0u);
            umma_tf32(d, ah, bl, IDESC, 1u);
            umma_tf32(d, al, bh, IDESC, 1u);
          }
          umma_commit(smem_u32(&empty[stage]));
          issued_any = true;
          if (++stage == NA_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(smem_u32(&tfull[buf]));
      }
      if (!ok && issued_any) {
        umma_commit(smem_u32(drain));
        volatile int no_abort = 0;
        mbar_wait(smem_u32(drain), 0, &no_abort, p.status, 6, 200000000ull);
      }
    }
  } else {
    const int q = warp & 3;
    int it = 0;
    for (long t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int mt = static_cast<int>(t % m_tiles), nt = static_cast<int>(t / m_tiles);
      const int buf = it & 1;
      const bool ok = mbar_wait(smem_u32(&tfull[buf]), (it >> 1) & 1, abort_flag, p.status, 4);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const long i = static_cast<long>(mt) * NA_BM + q * 32 + lane;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * NA_BN);
#pragma unroll 1
      for (int c = 0; c < NA_BN / 32; ++c) {
        float acc[32];
        tmem_ld32(tbase + c * 32, acc);
        const long j0 = static_cast<long>(nt) * NA_BN + c * 32;
        if (i < p.M) {
          float* row = p.C + i * static_cast<long>(p.N);
          if (j0 + 32 <= p.N && (p.N & 3) == 0) {
#pragma unroll
            for (int u = 0; u < 32; u += 4) *reinterpret_cast<float4*>(row + j0 + u) = make_float4(acc[u], acc[u + 1], acc[u + 2], acc[u + 3]);
          } else {
            for (int u = 0; u < 32 && j0 + u < p.N; ++u) row[j0 + u] = acc[u];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[buf]));
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0 && lane == 0 && *abort_flag) {
    for (int s = 0; s < NA_STAGES; ++s)
      if (pending[s]) {
        volatile int no_abort = 0;
        mbar_wait(smem_u32(&full[s]), issued_phase[s], &no_abort, p.status, 5, 200000000ull);
      }
  }
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

int na_fail(int code, const char* msg) {
  tj_b200_internal_set_error(msg);  // reported by tj_b200_last_error()
  return code;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceSetup {
  std::once_flag once;
  int rc = TJ_OK;
  std::string why;
  float* scratch = nullptr;
  int* status = nullptr;
  int num_sms = 0;
};
DeviceSetup g_setup[TJ_NOALLOC_MAX_DEVICES];
EncodeFn g_encode = nullptr;
std::once_flag g_encode_once;

// Per-device set-up (first call on a device, with that device current): the device address
// of the file-scope scratch array and status words, and the kernel's shared-memory opt-in.
void setup_device(DeviceSetup& s) {
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, tj_noalloc_scratch);
  if (e != cudaSuccess) {
    s.rc = TJ_ERR_CUDA;
    s.why = std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e);
    return;
  }
  s.scratch = static_cast<float*>(ptr);
  e = cudaGetSymbolAddress(&ptr, tj_noalloc_status);
  if (e != cudaSuccess) {
    s.rc = TJ_ERR_CUDA;
    s.why = std::string("cudaGetSymbolAddress(status) failed: ") + cudaGetErrorString(e);
    return;
  }
  s.status = static_cast<int*>(ptr);
  e = cudaFuncSetAttribute(noalloc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, NA_SMEM);
  if (e != cudaSuccess) {
    s.rc = TJ_ERR_CUDA;
    s.why = std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(e);
    return;
  }
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess || s.num_sms <= 0) {
    s.rc = TJ_ERR_CUDA;
    s.why = std::string("multiprocessor count query failed: ") + cudaGetErrorString(e);
  }
}

// The calling thread's device, with its set-up done (first use on a device runs it).
int current_setup(DeviceSetup** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail(TJ_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= TJ_NOALLOC_MAX_DEVICES) return na_fail(TJ_ERR_INVALID, "device index out of range");
  DeviceSetup& s = g_setup[dev];
  std::call_once(s.once, [&] { setup_device(s); });
  if (s.rc != TJ_OK) return na_fail(s.rc, s.why.c_str());
  *out = &s;
  return TJ_OK;
}

bool encode(CUtensorMap* m, float* base, int rows, int K, int box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 4};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int tj_b200_linear_f32_noalloc(const float* A, const float* B, float* C, int32_t M, int32_t N,
                                          int32_t K, void* stream) {
  if (!A || !B || !C) return na_fail(TJ_ERR_INVALID, "tj_b200_linear_f32_noalloc: NULL pointer");
  if (M <= 0 || N <= 0 || K <= 0 || K % 4 != 0)
    return na_fail(TJ_ERR_INVALID, "tj_b200_linear_f32_noalloc: need M, N, K > 0 and K % 4 == 0");
  if (static_cast<uint64_t>(M) * K > TJ_NOALLOC_MAX_OPERAND || static_cast<uint64_t>(N) * K > TJ_NOALLOC_MAX_OPERAND)
    return na_fail(TJ_ERR_INVALID,
                   "tj_b200_linear_f32_noalloc: operand too large for the static scratch (M*K and N*K must each "
                   "be <= 2097152 elements)");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) & 15)
    return na_fail(TJ_ERR_INVALID, "tj_b200_linear_f32_noalloc: A, B and C must be 16-byte aligned");
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeFn>(fn);
  });
  if (!g_encode) return na_fail(TJ_ERR_NO_DRIVER, "cuTensorMapEncodeTiled is unavailable");
  DeviceSetup* sp = nullptr;
  const int rc = current_setup(&sp);
  if (rc != TJ_OK) return rc;
  DeviceSetup& s = *sp;

  float* a_hi = s.scratch;
  float* a_lo = s.scratch + TJ_NOALLOC_MAX_OPERAND;
  float* b_hi = s.scratch + 2 * TJ_NOALLOC_MAX_OPERAND;
  float* b_lo = s.scratch + 3 * TJ_NOALLOC_MAX_OPERAND;
  NoallocParams prm{};
  prm.C = C;
  prm.status = s.status;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  if (!encode(&prm.tm[0], a_hi, M, K, NA_BM) || !encode(&prm.tm[1], b_hi, N, K, NA_BN) ||
      !encode(&prm.tm[2], a_lo, M, K, NA_BM) || !encode(&prm.tm[3], b_lo, N, K, NA_BN))
    return na_fail(TJ_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(s.status, 0, sizeof(int) * 4, st);  // status words start at zero every call
  if (e != cudaSuccess) return na_fail(TJ_ERR_CUDA, cudaGetErrorString(e));
  const long na4 = static_cast<long>(M) * K / 4, nb4 = static_cast<long>(N) * K / 4;
  const long split_ctas = 8L * s.num_sms;
  noalloc_split<<<static_cast<int>(std::min<long>((na4 + 255) / 256, split_ctas)), 256, 0, st>>>(
      reinterpret_cast<const float4*>(A), reinterpret_cast<float4*>(a_hi), reinterpret_cast<float4*>(a_lo), na4);
  noalloc_split<<<static_cast<int>(std::min<long>((nb4 + 255) / 256, split_ctas)), 256, 0, st>>>(
      reinterpret_cast<const float4*>(B), reinterpret_cast<float4*>(b_hi), reinterpret_cast<float4*>(b_lo), nb4);
  const long tiles = static_cast<long>((M + NA_BM - 1) / NA_BM) * ((N + NA_BN - 1) / NA_BN);
  noalloc_gemm<<<static_cast<int>(std::min<long>(tiles, s.num_sms)), 192, NA_SMEM, st>>>(prm);
  e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail(TJ_ERR_CUDA, cudaGetErrorString(e));
  return TJ_OK;
}

// The failure record of the allocation-free GEMM: a bounded wait in it that ran out leaves
// its (code, site) in the shared status words instead of stopping the GPU.  This waits for
// `stream`, copies the words back, clears them, and reports code 0 when nothing failed.
extern "C" int tj_b200_linear_f32_noalloc_status(int32_t* code, int32_t* where, void* stream) {
  if (!code || !where) return na_fail(TJ_ERR_INVALID, "tj_b200_linear_f32_noalloc_status: NULL pointer");
  *code = 0;
  *where = 0;
  DeviceSetup* sp = nullptr;
  const int rc = current_setup(&sp);
  if (rc != TJ_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int words[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(words, sp->status, sizeof(words), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && words[0] != 0) {
    e = cudaMemsetAsync(sp->status, 0, sizeof(words), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return na_fail(TJ_ERR_CUDA, cudaGetErrorString(e));
  *code = words[0];
  *where = words[1];
  return words[0] != 0 ? TJ_ERR_DEVICE_STATUS : TJ_OK;
}
