// Row-reduction building blocks shared by the standalone row kernels and the
// linear cross-entropy pipeline: per-thread (max, sum-exp) partials over a
// row segment, the gradient write of a row segment, zero fill, and the small
// fixed-order reduction kernels for the loss sums.
#pragma once

#include "common.cuh"

namespace gh {
namespace {

constexpr int kUnroll = 2;  // x 32-byte vectors in flight per thread

// This thread's (max, sum) partial over x[0, n), in log2 units.
// KEEP: the row is read again right after (CE): first-read loads marked
// evict_last so the re-read hits L2.
template <typename T, int THREADS, int UNROLL, bool KEEP = false>
__device__ __forceinline__ MS row_partial(const T* __restrict__ x, int64_t n) {
  constexpr int PER = 32 / sizeof(T);
  const RowSplit sp = row_split(reinterpret_cast<uintptr_t>(x), n, sizeof(T), 32);
  MS acc = ms_empty();
  const int tid = threadIdx.x;
  for (int64_t i = tid; i < sp.head; i += THREADS)
    acc = ms_fold1(acc, Elt<T>::to_f(x[i]) * kLog2e);
  for (int64_t i = sp.tail0 + tid; i < n; i += THREADS)
    acc = ms_fold1(acc, Elt<T>::to_f(x[i]) * kLog2e);
  const U8* xv = reinterpret_cast<const U8*>(x + sp.head);
  int64_t i = tid;
  for (; i + (int64_t)(UNROLL - 1) * THREADS < sp.nvec; i += (int64_t)UNROLL * THREADS) {
    Vec32<T> r[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) r[u].raw = KEEP ? ld32_keep(xv + i + u * THREADS) : ld32(xv + i + u * THREADS);
    float t[UNROLL * PER];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      float f[PER];
      r[u].to_float(f);
#pragma unroll
      for (int k = 0; k < PER; ++k) t[u * PER + k] = f[k];
    }
    acc = ms_fold_raw<UNROLL * PER>(acc, t);
  }
  for (; i < sp.nvec; i += THREADS) {
    Vec32<T> r;
    r.raw = KEEP ? ld32_keep(xv + i) : ld32(xv + i);
    float f[PER];
    r.to_float(f);
    acc = ms_fold_raw<PER>(acc, f);
  }
  return acc;
}

// y[c] = exp2(x[c] * log2e - mm) * coef - (c == lab ? sub : 0) for c in [0, n).
// x and y share their 16-byte misalignment (checked on the host). y may be x.
// REV: walk the vectors from the end of the row, i.e. re-read first what the
// preceding pass loaded last (the lines most likely still in L2).
template <typename T, int THREADS, int UNROLL, bool REV = false>
__device__ __forceinline__ void row_grad(const T* x, T* y, int64_t n, int64_t lab,
                                         float mm, float coef, float sub) {
  constexpr int PER = 32 / sizeof(T);
  const RowSplit sp = row_split(reinterpret_cast<uintptr_t>(x), n, sizeof(T), 32);
  const int tid = threadIdx.x;
  auto scalar = [&](int64_t c) {
    float g = fast_exp2(Elt<T>::to_f(x[c]) * kLog2e - mm) * coef;
    if (c == lab) g -= sub;
    y[c] = Elt<T>::from_f(g);
  };
  for (int64_t c = tid; c < sp.head; c += THREADS) scalar(c);
  for (int64_t c = sp.tail0 + tid; c < n; c += THREADS) scalar(c);
  const U8* xv = reinterpret_cast<const U8*>(x + sp.head);
  U8* yv = reinterpret_cast<U8*>(y + sp.head);
  const int64_t lab_rel = lab - sp.head;  // label position relative to the vector run
  // vector holding the label (or -1): one compare per vector, not per element
  const int64_t lab_vec = (lab_rel >= 0 && lab_rel < sp.nvec * PER) ? lab_rel / PER : -1;
  const int lab_k = (int)(lab_rel - (lab_vec < 0 ? 0 : lab_vec) * PER);
  auto vi = [&](int64_t j) { return REV ? sp.nvec - 1 - j : j; };
  int64_t i = tid;
  for (; i + (int64_t)(UNROLL - 1) * THREADS < sp.nvec; i += (int64_t)UNROLL * THREADS) {
    Vec32<T> r[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) r[u].raw = ld32_last(xv + vi(i + u * THREADS));
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      float f[PER];
      r[u].to_float(f);
#pragma unroll
      for (int k = 0; k < PER; ++k) f[k] = fast_exp2(fmaf(f[k], kLog2e, -mm)) * coef;
      if (vi(i + u * THREADS) == lab_vec) {
#pragma unroll
        for (int k = 0; k < PER; ++k)
          if (k == lab_k) f[k] -= sub;
      }
      Vec32<T> o;
      o.from_float(f);
      st32_stream(yv + vi(i + u * THREADS), o.raw);
    }
  }
  for (; i < sp.nvec; i += THREADS) {
    Vec32<T> r;
    r.raw = ld32_last(xv + vi(i));
    float f[PER];
    r.to_float(f);
#pragma unroll
    for (int k = 0; k < PER; ++k) f[k] = fast_exp2(fmaf(f[k], kLog2e, -mm)) * coef;
    if (vi(i) == lab_vec) {
#pragma unroll
      for (int k = 0; k < PER; ++k)
        if (k == lab_k) f[k] -= sub;
    }
    Vec32<T> o;
    o.from_float(f);
    st32_stream(yv + vi(i), o.raw);
  }
}

template <typename T, int THREADS>
__device__ __forceinline__ void row_zero(T* y, int64_t n) {
  constexpr int PER = 16 / sizeof(T);
  const RowSplit sp = row_split(reinterpret_cast<uintptr_t>(y), n, sizeof(T));
  const int tid = threadIdx.x;
  for (int64_t c = tid; c < sp.head; c += THREADS) y[c] = Elt<T>::from_f(0.f);
  for (int64_t c = sp.tail0 + tid; c < n; c += THREADS) y[c] = Elt<T>::from_f(0.f);
  uint4* yv = reinterpret_cast<uint4*>(y + sp.head);
  for (int64_t i = tid; i < sp.nvec; i += THREADS) st16(yv + i, make_uint4(0, 0, 0, 0));
  (void)PER;
}

template <typename I>
__device__ __forceinline__ int64_t load_index(const I* p, int64_t r) { return (int64_t)p[r]; }

// Count of labels != ignore_index -> scale = 1 / max(count, 1)
// (ops/cross_entropy.py:63-66, clamp(min=1) then reciprocal).
// An optional caller-provided device factor multiplies the result.
__global__ void __launch_bounds__(1024)
mean_scale_kernel(const int64_t* __restrict__ labels, int64_t rows, int64_t ignore,
                  const float* extra, float* scale) {
  __shared__ float scratch[32];
  float c = 0.f;
  for (int64_t r = threadIdx.x; r < rows; r += 1024) c += labels[r] != ignore ? 1.f : 0.f;
  c = block_sum<1024>(c, scratch);
  if (threadIdx.x == 0) *scale = (extra ? *extra : 1.f) / fmaxf(c, 1.f);
}

// Fixed-order sums of the per-row loss terms; n_valid counts label != ignore.
__global__ void __launch_bounds__(1024)
ce_finalize_kernel(const float* __restrict__ row_ce, const float* __restrict__ row_z,
                   const int64_t* __restrict__ labels, int64_t rows, int64_t ignore,
                   float* ce_sum, float* z_sum, float* n_valid) {
  __shared__ float scratch[32];
  float ce = 0.f, z = 0.f, c = 0.f;
  for (int64_t r = threadIdx.x; r < rows; r += 1024) {
    ce += row_ce[r];
    z += row_z[r];
    c += labels[r] != ignore ? 1.f : 0.f;
  }
  ce = block_sum<1024>(ce, scratch);
  z = block_sum<1024>(z, scratch);
  c = block_sum<1024>(c, scratch);
  if (threadIdx.x == 0) { *ce_sum = ce; *z_sum = z; *n_valid = c; }
}

}  // namespace
}  // namespace gh
