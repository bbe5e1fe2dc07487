// Shared device/host helpers for the greyhound_b200 C-ABI library.
//
// Everything here is plumbing: dtype codes, 16-byte vector loads of the three
// logits dtypes the reference accepts (fp16 / bf16 / fp32,
// src/greyhound/kernels/cross_entropy.py:180), the (max, sum-exp) merge used
// by every row reduction, status codes and the per-thread last-error string.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/greyhound_b200.h"

namespace gh {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegInf = -__builtin_huge_valf();

// ---- host-side error bookkeeping (defined in capi.cu) ----------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
void count_launch(int n = 1);
// Enqueue the copy of a non-zero workspace status word into this device's
// sticky error slot (gh_take_device_errors); GH_OK when status is NULL.
int publish_status(const int* status, cudaStream_t st);

// Kernel classes for the optional event timing (gh_profile_enable / _read).
enum ProfClass {
  PROF_GEMM_LOGITS_CE = 0,  // logits GEMM with the fused CE epilogue
  PROF_GEMM_DW = 1,
  PROF_GEMM_DH = 2,
  PROF_DLOGITS = 3,         // the small kernels between the GEMMs (q fix-up, alpha * H, or the dlogits pass)
  PROF_ROWS = 4,            // standalone CE / SLS row kernels
  PROF_GEMM_OTHER = 5,
  PROF_NUM = 6
};
// RAII: records an event pair around the launches in its scope when timing is on.
struct ProfScope {
  ProfScope(int cls, cudaStream_t st);
  ~ProfScope();
  int cls_;
  cudaStream_t st_;
  void* a_;
};

inline int elt_size(int dtype) {
  switch (dtype) {
    case GH_F16: case GH_BF16: return 2;
    case GH_F32: case GH_I32: return 4;
    case GH_I64: return 8;
    default: return 0;
  }
}

// ---- element conversion ----------------------------------------------------
template <typename T> struct Elt;
template <> struct Elt<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// A 16-byte vector of T, unpacked to / packed from fp32.
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  uint4 raw;
  __device__ __forceinline__ void to_float(float (&f)[N]) const {
    const T* p = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = Elt<T>::to_f(p[i]);
  }
  __device__ __forceinline__ void from_float(const float (&f)[N]) {
    T* p = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = Elt<T>::from_f(f[i]);
  }
};

// Streaming 16-byte global load that keeps the line in L2 (evict_last hint
// is not needed: the default policy already keeps a just-read row for the
// second pass; ld.global.nc avoids L1 allocation churn).
__device__ __forceinline__ uint4 ld16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// Load that is the last use of the line: no L1 allocation.
__device__ __forceinline__ uint4 ld16_last(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// 32-byte (256-bit) accesses, sm_100: half the memory instructions of 16-byte ones.
struct U8 {
  uint32_t w[8];
};
__device__ __forceinline__ U8 ld32(const void* p) {
  U8 v;
  asm volatile("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                 "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}
// First read of a row that will be read again soon: keep it in L2.
__device__ __forceinline__ U8 ld32_keep(const void* p) {
  U8 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::evict_last.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                 "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}
__device__ __forceinline__ U8 ld32_last(const void* p) {
  U8 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                 "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st32(void* p, const U8& v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
               "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
               : "memory");
}
// Store that must not displace lines still waiting to be re-read (the
// gradient written by a row kernel whose input row is re-read from L2).
__device__ __forceinline__ void st32_stream(void* p, const U8& v) {
  asm volatile("st.global.L1::no_allocate.L2::evict_first.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p),
               "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]),
               "r"(v.w[7])
               : "memory");
}
template <typename T>
struct Vec32 {
  static constexpr int N = 32 / sizeof(T);
  U8 raw;
  __device__ __forceinline__ void to_float(float (&f)[N]) const {
    const T* p = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = Elt<T>::to_f(p[i]);
  }
  __device__ __forceinline__ void from_float(const float (&f)[N]) {
    T* p = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = Elt<T>::from_f(f[i]);
  }
};
__device__ __forceinline__ void st16(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
// Store of a value nobody reads back soon: streaming (evict-first).
__device__ __forceinline__ void st16_cs(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Running (max, sum) of exp2 terms, in log2 units: the pair represents
// s * 2^m. Merging two pairs rescales the smaller-max side. An empty side is
// (-inf, 0); merging two empty sides stays empty (no inf - inf).
struct MS {
  float m;
  float s;
};
__device__ __forceinline__ MS ms_empty() { return {kNegInf, 0.f}; }
__device__ __forceinline__ MS ms_merge(MS a, MS b) {
  float m = fmaxf(a.m, b.m);
  if (m == kNegInf) return {kNegInf, 0.f};
  float s = a.s * fast_exp2(a.m - m) + b.s * fast_exp2(b.m - m);
  return {m, s};
}
// Fold a block of already-scaled values t[i] = x[i]*log2e into the pair.
template <int N>
__device__ __forceinline__ MS ms_fold(MS a, const float (&t)[N]) {
  float bm = t[0];
#pragma unroll
  for (int i = 1; i < N; ++i) bm = fmaxf(bm, t[i]);
  float m = fmaxf(a.m, bm);
  if (m == kNegInf) return a;
  float s = a.s * fast_exp2(a.m - m);
#pragma unroll
  for (int i = 0; i < N; ++i) s += fast_exp2(t[i] - m);
  return {m, s};
}
// Same for raw (unscaled) values x[i]: the max is taken on x and the scale
// folded into one FFMA per element, exp2(x * log2e - m).
template <int N>
__device__ __forceinline__ MS ms_fold_raw(MS a, const float (&x)[N]) {
  float bm = x[0];
#pragma unroll
  for (int i = 1; i < N; ++i) bm = fmaxf(bm, x[i]);
  const float m = fmaxf(a.m, bm * kLog2e);
  if (m == kNegInf) return a;
  float s = a.s * fast_exp2(a.m - m);
#pragma unroll
  for (int i = 0; i < N; ++i) s += fast_exp2(fmaf(x[i], kLog2e, -m));
  return {m, s};
}
__device__ __forceinline__ MS ms_fold1(MS a, float t) {
  float m = fmaxf(a.m, t);
  if (m == kNegInf) return a;
  return {m, a.s * fast_exp2(a.m - m) + fast_exp2(t - m)};
}

__device__ __forceinline__ MS warp_merge(MS v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    MS o;
    o.m = __shfl_xor_sync(0xffffffffu, v.m, off);
    o.s = __shfl_xor_sync(0xffffffffu, v.s, off);
    v = ms_merge(v, o);
  }
  return v;
}

// Block-wide merge; every thread receives the result. `scratch` holds
// 2 * (blockDim/32) floats.
template <int THREADS>
__device__ __forceinline__ MS block_merge(MS v, float* scratch) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_merge(v);
  if (lane == 0) { scratch[warp] = v.m; scratch[W + warp] = v.s; }
  __syncthreads();
  MS r = ms_empty();
  if (lane < W) { r.m = scratch[lane]; r.s = scratch[W + lane]; }
  r = warp_merge(r);
  __syncthreads();  // scratch may be reused right after
  return r;
}

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < W ? scratch[lane] : 0.f;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
  __syncthreads();
  return r;
}

// Split [0, n) of a row that starts at byte address `addr` into a scalar head
// (up to the first 16-byte boundary), a run of whole 16-byte vectors and a
// scalar tail. Handles the odd vocab sizes the reference tests use (257, 97).
struct RowSplit {
  int64_t head;   // scalar elements before the first vector
  int64_t nvec;   // number of 16-byte vectors
  int64_t tail0;  // first element of the scalar tail
};
__device__ __forceinline__ RowSplit row_split(uintptr_t addr, int64_t n, int elt, int vbytes = 16) {
  RowSplit r;
  int64_t mis = (int64_t)(addr & (vbytes - 1));
  int64_t head = mis == 0 ? 0 : (vbytes - mis) / elt;
  if (head > n) head = n;
  r.head = head;
  const int per = vbytes / elt;
  r.nvec = (n - head) / per;
  r.tail0 = head + r.nvec * per;
  return r;
}

}  // namespace gh
