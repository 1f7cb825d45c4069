// Shared device helpers for the generated sm_100a kernels of the tensorjit B200 backend.
//
// Arithmetic follows the reference's CUDA expression table
// (tensorjit/backends/common.py:65-88): every value is f32 inside a kernel,
// loads convert to f32 and stores round f32 -> storage type to nearest even
// (tensorjit/backends/cuda_backend.py:46-54).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define TJ_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// scalar conversions
// ---------------------------------------------------------------------------
TJ_DEV float tj_f32(float x) { return x; }
TJ_DEV float tj_f32(int x) { return (float)x; }
TJ_DEV float tj_f32(__half x) { return __half2float(x); }
TJ_DEV float tj_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> TJ_DEV T tj_from(float x);
template <> TJ_DEV float tj_from<float>(float x) { return x; }
template <> TJ_DEV int tj_from<int>(float x) { return (int)x; }
template <> TJ_DEV __half tj_from<__half>(float x) { return __float2half_rn(x); }
template <> TJ_DEV __nv_bfloat16 tj_from<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// ---------------------------------------------------------------------------
// 16-byte vector loads/stores: VEC = 16 / sizeof(T) elements
// ---------------------------------------------------------------------------
template <typename T> struct TjVec { static constexpr int N = 16 / sizeof(T); };

TJ_DEV uint4 tj_ld16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// streaming load for data read exactly once
TJ_DEV uint4 tj_ld16_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
TJ_DEV void tj_st16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// hi part of the TF32 split of 3xTF32 operands: v with its 13 low mantissa bits cleared (the
// lo part v - hi is exact in f32)
TJ_DEV float tj_tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xffffe000u); }

TJ_DEV void tj_unpack(uint4 v, float* f, const float*) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}
TJ_DEV void tj_unpack(uint4 v, float* f, const __nv_bfloat16*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
TJ_DEV void tj_unpack(uint4 v, float* f, const __half*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
TJ_DEV uint4 tj_pack(const float* f, const float*) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}
TJ_DEV uint32_t tj_pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
TJ_DEV uint4 tj_pack(const float* f, const __nv_bfloat16*) {
  return make_uint4(tj_pack_bf16x2(f[0], f[1]), tj_pack_bf16x2(f[2], f[3]), tj_pack_bf16x2(f[4], f[5]),
                    tj_pack_bf16x2(f[6], f[7]));
}
TJ_DEV uint32_t tj_pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
TJ_DEV uint4 tj_pack(const float* f, const __half*) {
  return make_uint4(tj_pack_f16x2(f[0], f[1]), tj_pack_f16x2(f[2], f[3]), tj_pack_f16x2(f[4], f[5]),
                    tj_pack_f16x2(f[6], f[7]));
}
template <typename T> TJ_DEV void tj_load_vec(const T* p, float* f) { tj_unpack(tj_ld16(p), f, (const T*)nullptr); }
template <typename T> TJ_DEV void tj_load_vec_stream(const T* p, float* f) {
  tj_unpack(tj_ld16_stream(p), f, (const T*)nullptr);
}
template <typename T> TJ_DEV void tj_store_vec(T* p, const float* f) { tj_st16(p, tj_pack(f, (const T*)nullptr)); }

// ---------------------------------------------------------------------------
// op semantics (tensorjit/backends/common.py:65-88, CUDA variant)
// ---------------------------------------------------------------------------
TJ_DEV float tj_gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
TJ_DEV float tj_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
TJ_DEV float tj_silu(float x) { return x / (1.0f + expf(-x)); }
TJ_DEV float tj_rsqrt(float x) { return 1.0f / sqrtf(x); }
TJ_DEV float tj_relu(float x) { return fmaxf(x, 0.0f); }
TJ_DEV float tj_where(float c, float a, float b) { return c != 0.0f ? a : b; }
TJ_DEV float tj_sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
// GELU for half-precision outputs: x * Phi(x) with Phi(x) = 1 / (1 + 2^(-x P(x^2))), where
// x P(x^2) is an odd degree-7 polynomial fitted here to log2 e * logit(Phi(x)) on |x| <= 5
// (Lawson-weighted least squares for minimal maximum error; the degree-3 logistic fit of
// Bowling et al. 2009, "A logistic approximation to the cumulative normal distribution",
// is the starting form).  Since sigma(g) has a relative error of about |g - logit Phi|, the GELU
// relative error is <= 3.8e-4 for x >= 0 and <= 1.4e-3 for x < 0 (below half an ulp of bf16,
// the negative tail included; absolute error <= 1.7e-4); the polynomial is monotone, so large
// |x| give x or -0.  Ten instructions (two MUFU) instead of erff's or an erf approximation's twenty; the
// epilogues of GEMMs with half-precision outputs are issue-bound on this.
TJ_DEV float tj_gelu_fast(float x) {
  const float y = x * x;
  const float p = fmaf(fmaf(fmaf(1.303200679103611e-05f, y, -0.0014235572889447212f), y, 0.10939675569534302f), y,
                       2.2976467609405518f);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-x * p));
  return __fdividef(x, 1.0f + e);
}
TJ_DEV float tj_silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
template <int W> TJ_DEV float tj_group_sum(float v) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int W> TJ_DEV float tj_group_max(float v) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// device status word: the first failing kernel records (code, where)
// ---------------------------------------------------------------------------
enum : int { TJ_STATUS_WAIT_TIMEOUT = 1, TJ_STATUS_BOUNDS = 2 };
TJ_DEV void tj_report(int* status, int code, int where) {
  if (status && atomicCAS(status, 0, code) == 0) status[1] = where;
}
// Programmatic dependent launch: the runtime lets a program's next kernel start while this one
// finishes.  Every kernel lets its dependents launch as soon as it starts (its own blocks are all
// resident or done by then), and waits for the previous kernel's completion and memory before
// its first global access; only set-up (barriers, TMEM allocation, descriptor prefetch) overlaps.
// Both are no-ops for a kernel launched without the attribute.
TJ_DEV void tj_pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
TJ_DEV void tj_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TJ_DEV uint64_t tj_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// checked build (-DTJ_CHECKED, TENSORJIT_B200_CHECKED=1): the generated kernels declare their
// global operands as bounded views instead of raw pointers, so every computed element index of
// a load or store is compared with the operand's element count first.  A violation skips the
// access (loads read 0) and records (TJ_STATUS_BOUNDS, kernel * 16 + 15) in the program's
// status words, with the operand's argument index and the offending element offset in words 2
// and 3.  The unchecked build never sees these types.
// ---------------------------------------------------------------------------
#ifdef TJ_CHECKED
TJ_DEV void tj_report_bounds(int* status, int where, int arg, long off) {
  if (status && atomicCAS(status, 0, TJ_STATUS_BOUNDS) == 0) {
    status[1] = where;
    status[2] = arg;
    status[3] = static_cast<int>(off > 0x7fffffffL ? 0x7fffffffL : (off < -0x7fffffffL ? -0x7fffffffL : off));
  }
}
// element reference through a view: reads give 0 and writes are dropped when out of bounds
template <class T> struct tj_ref {
  T* p;
  bool ok;
  TJ_DEV tj_ref& operator=(T v) {
    if (ok) *p = v;
    return *this;
  }
  TJ_DEV operator T() const { return ok ? *p : T(); }
};
// a view plus an element offset (what `view + off` yields; vector accesses check all 16 bytes)
template <class T> struct tj_cptr {
  T* p;
  long n;
  int* status;
  int where, arg;
  long off;
  TJ_DEV tj_cptr operator+(long d) const { return tj_cptr{p, n, status, where, arg, off + d}; }
  TJ_DEV bool check(long len) const {
    const bool ok = off >= 0 && off + len <= n;
    if (!ok) tj_report_bounds(status, where, arg, off);
    return ok;
  }
  TJ_DEV tj_ref<T> operator[](long i) const { return (*this + i).deref(); }
  TJ_DEV tj_ref<T> deref() const {
    const bool ok = check(1);
    return tj_ref<T>{p + (ok ? off : 0), ok};
  }
};
template <class T> struct tj_view {
  T* p;
  long n;
  int* status;
  int where, arg;
  TJ_DEV tj_cptr<T> operator+(long d) const { return tj_cptr<T>{p, n, status, where, arg, d}; }
  TJ_DEV tj_ref<T> operator[](long i) const { return (*this + i).deref(); }
};
template <typename T> TJ_DEV void tj_load_vec(tj_cptr<const T> q, float* f) {
  if (!q.check(TjVec<T>::N)) {
#pragma unroll
    for (int i = 0; i < TjVec<T>::N; ++i) f[i] = 0.0f;
    return;
  }
  tj_load_vec(q.p + q.off, f);
}
template <typename T> TJ_DEV void tj_load_vec_stream(tj_cptr<const T> q, float* f) { tj_load_vec(q, f); }
template <typename T> TJ_DEV void tj_store_vec(tj_cptr<T> q, const float* f) {
  if (q.check(TjVec<T>::N)) tj_store_vec(q.p + q.off, f);
}
template <typename T> TJ_DEV void tj_st16(tj_cptr<T> q, uint4 v) {
  if (q.check(static_cast<int>(16 / sizeof(T)))) tj_st16(q.p + q.off, v);
}
// a condition the generated code asserts (a TMA coordinate, a TMEM column): false = violation
TJ_DEV bool tj_check(bool ok, int* status, int where, int arg, long what) {
  if (!ok) tj_report_bounds(status, where, arg, what);
  return ok;
}
#define TJ_CHECKED_ONLY(...) __VA_ARGS__
#else
#define TJ_CHECKED_ONLY(...)
#endif
