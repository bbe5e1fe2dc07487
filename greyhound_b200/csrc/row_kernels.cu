// Bandwidth-bound row kernels: cross-entropy with logits gradient, selective
// log-softmax forward, and its backward.
//
// Semantics follow the reference CuTe-DSL kernels:
//   CE+grad  src/greyhound/kernels/cross_entropy.py:20-108
//            lse = max + log(sum exp(x - max)); ce = lse - x[label];
//            z = lse^2; n_valid += 1 for label != ignore_index;
//            grad = softmax * (1 + 2 z_mult lse) - onehot(label), 0 if ignored
//   SLS fwd  src/greyhound/kernels/logprobs.py:20-88   out = x[index] - lse
//   SLS bwd  new (the reference raises, ops/logprobs.py:30)
//
// Design (B200): 16-byte vector loads/stores, fp32 online (max, sum-exp)
// accumulated in log2 units with ex2.approx, no float atomics. Two launch
// shapes:
//   * "fused": one CTA per row (grid-strided over rows). The row is read
//     twice; the second read hits L2 because at most 2 CTAs/SM x 148 SMs rows
//     (76 MB of bf16 rows at V=128256) are in flight against a 126 MB L2.
//   * "split": for few rows (< 2 x SMs) each row is cut into chunks handled by
//     separate CTAs; a stats kernel writes per-chunk (max, sum) partials and
//     the label logit, a second kernel merges them and writes the gradient.
// Per-row loss terms go to workspace arrays; one single-CTA kernel sums them
// in a fixed order, so results are bit-reproducible run to run.
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "row_ops.cuh"

namespace gh {
namespace {

constexpr int kFusedThreads = 512;
constexpr int kSplitThreads = 256;

// ---------------------------------------------------------------------------
// CE, fused shape: one CTA per row.
template <typename T, int THREADS, int UNROLL>
__global__ void __launch_bounds__(THREADS, 2)
ce_fused_kernel(const T* __restrict__ logits, T* dlogits, const int64_t* __restrict__ labels,
                int64_t rows, int64_t V, float zmul, int64_t ignore, const float* scale_ptr,
                float* row_ce, float* row_z, float* lse_out, int* status) {
  __shared__ float scratch[2 * THREADS / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* x = logits + row * V;
    const int64_t lab = labels[row];
    bool valid = lab != ignore;
    const bool bad = valid && (lab < 0 || lab >= V);
    valid = valid && !bad;
    // Read the label logit before the barrier inside block_merge: with an
    // in-place gradient other threads overwrite it right after.
    float x_lab = 0.f;
    if (threadIdx.x == 0 && valid) x_lab = Elt<T>::to_f(x[lab]);
    MS tot = block_merge<THREADS>(row_partial<T, THREADS, UNROLL, true>(x, V), scratch);
    const float lse2 = tot.m + fast_log2(tot.s);
    const float lse = lse2 * kLn2;
    if (threadIdx.x == 0) {
      if (bad) atomicOr(status, GH_DEV_BAD_LABEL);
      row_ce[row] = valid ? lse - x_lab : 0.f;
      row_z[row] = valid ? lse * lse : 0.f;
      if (lse_out) lse_out[row] = lse;
    }
    if (dlogits != nullptr) {
      T* y = dlogits + row * V;
      if (!valid) {
        row_zero<T, THREADS>(y, V);
      } else {
        const float scale = scale_ptr ? *scale_ptr : 1.f;
        const float coef = scale * (1.f + 2.f * zmul * lse) / tot.s;
        row_grad<T, THREADS, UNROLL, true>(x, y, V, lab, tot.m, coef, scale);
      }
    }
  }
}

// Split shape, kernel 1: per-(chunk,row) partial stats + label logit.
// part layout: [rows][splits] of float2 (m, s); xlab[rows].
template <typename T, typename I, int THREADS>
__global__ void __launch_bounds__(THREADS)
split_stats_kernel(const T* __restrict__ logits, const I* __restrict__ labels, int64_t rows,
                   int64_t V, int64_t chunk, int splits, float2* part, float* xlab) {
  __shared__ float scratch[2 * THREADS / 32];
  const int64_t row = blockIdx.y;
  const int split = blockIdx.x;
  const int64_t c0 = (int64_t)split * chunk;
  const int64_t c1 = c0 + chunk < V ? c0 + chunk : V;
  const T* x = logits + row * V;
  MS acc = c0 < c1 ? row_partial<T, THREADS, kUnroll>(x + c0, c1 - c0) : ms_empty();
  MS tot = block_merge<THREADS>(acc, scratch);
  if (threadIdx.x == 0) {
    part[row * splits + split] = make_float2(tot.m, tot.s);
    const int64_t lab = load_index(labels, row);
    if (lab >= c0 && lab < c1) xlab[row] = Elt<T>::to_f(x[lab]);
  }
}

// Merge a row's `splits` partials; every thread gets the total.
template <int THREADS>
__device__ __forceinline__ MS merge_parts(const float2* part, int splits, float* scratch) {
  MS acc = ms_empty();
  for (int j = threadIdx.x; j < splits; j += THREADS) {
    float2 p = part[j];
    acc = ms_merge(acc, MS{p.x, p.y});
  }
  return block_merge<THREADS>(acc, scratch);
}

// Split shape, kernel 2 (CE): merge partials, write loss terms and gradient.
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
ce_split_grad_kernel(const T* logits, T* dlogits, const int64_t* __restrict__ labels,
                     int64_t rows, int64_t V, int64_t chunk, int splits, const float2* part,
                     const float* xlab, float zmul, int64_t ignore, const float* scale_ptr,
                     float* row_ce, float* row_z, float* lse_out, int* status) {
  __shared__ float scratch[2 * THREADS / 32];
  const int64_t row = blockIdx.y;
  const int split = blockIdx.x;
  MS tot = merge_parts<THREADS>(part + row * splits, splits, scratch);
  const float lse = (tot.m + fast_log2(tot.s)) * kLn2;
  const int64_t lab = labels[row];
  bool valid = lab != ignore;
  const bool bad = valid && (lab < 0 || lab >= V);
  valid = valid && !bad;
  if (split == 0 && threadIdx.x == 0) {
    if (bad) atomicOr(status, GH_DEV_BAD_LABEL);
    row_ce[row] = valid ? lse - xlab[row] : 0.f;
    row_z[row] = valid ? lse * lse : 0.f;
    if (lse_out) lse_out[row] = lse;
  }
  if (dlogits == nullptr) return;
  const int64_t c0 = (int64_t)split * chunk;
  if (c0 >= V) return;
  const int64_t n = c0 + chunk < V ? chunk : V - c0;
  T* y = dlogits + row * V + c0;
  if (!valid) {
    row_zero<T, THREADS>(y, n);
    return;
  }
  const float scale = scale_ptr ? *scale_ptr : 1.f;
  const float coef = scale * (1.f + 2.f * zmul * lse) / tot.s;
  row_grad<T, THREADS, kUnroll>(logits + row * V + c0, y, n, lab - c0, tot.m, coef, scale);
}

// ---------------------------------------------------------------------------
// Selective log-softmax forward, fused shape.
template <typename T, typename I, typename O, int THREADS, int UNROLL>
__global__ void __launch_bounds__(THREADS, 2)
sls_fused_kernel(const T* __restrict__ logits, const I* __restrict__ index, int64_t rows,
                 int64_t V, O* out, float* lse_out, int* status) {
  __shared__ float scratch[2 * THREADS / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* x = logits + row * V;
    const int64_t idx = load_index(index, row);
    const bool ok = idx >= 0 && idx < V;
    float x_idx = 0.f;
    if (threadIdx.x == 0 && ok) x_idx = Elt<T>::to_f(x[idx]);
    MS tot = block_merge<THREADS>(row_partial<T, THREADS, UNROLL>(x, V), scratch);
    if (threadIdx.x == 0) {
      const float lse = (tot.m + fast_log2(tot.s)) * kLn2;
      if (!ok) atomicOr(status, GH_DEV_BAD_LABEL);
      out[row] = Elt<O>::from_f(ok ? x_idx - lse : __int_as_float(0x7fc00000));
      if (lse_out) lse_out[row] = lse;
    }
  }
}

// Selective log-softmax forward, split shape kernel 2.
template <typename I, typename O, int THREADS>
__global__ void __launch_bounds__(THREADS)
sls_split_finish_kernel(const I* __restrict__ index, int64_t rows, int64_t V, int splits,
                        const float2* part, const float* xlab, O* out, float* lse_out,
                        int* status) {
  __shared__ float scratch[2 * THREADS / 32];
  const int64_t row = blockIdx.x;
  MS tot = merge_parts<THREADS>(part + row * splits, splits, scratch);
  if (threadIdx.x == 0) {
    const float lse = (tot.m + fast_log2(tot.s)) * kLn2;
    const int64_t idx = load_index(index, row);
    const bool ok = idx >= 0 && idx < V;
    if (!ok) atomicOr(status, GH_DEV_BAD_LABEL);
    out[row] = Elt<O>::from_f(ok ? xlab[row] - lse : __int_as_float(0x7fc00000));
    if (lse_out) lse_out[row] = lse;
  }
}

// Selective log-softmax backward: grid (rows, chunks).
//   grad[v] = g * ([v == idx] - exp(x[v] - lse))
template <typename T, typename I, typename G, int THREADS>
__global__ void __launch_bounds__(THREADS)
sls_bwd_kernel(const T* __restrict__ logits, const I* __restrict__ index,
               const float* __restrict__ lse, const G* __restrict__ grad_out, int64_t rows,
               int64_t V, int64_t chunk, T* grad) {
  const int64_t row = blockIdx.x;
  const int64_t c0 = (int64_t)blockIdx.y * chunk;
  if (c0 >= V) return;
  const int64_t n = c0 + chunk < V ? chunk : V - c0;
  const float g = Elt<G>::to_f(grad_out[row]);
  const int64_t idx = load_index(index, row);
  const float lse2 = lse[row] * kLog2e;
  // exp2(t - lse2) * (-g) - (c == idx ? -g : 0)
  row_grad<T, THREADS, kUnroll>(logits + row * V + c0, grad + row * V + c0, n, idx - c0, lse2,
                                -g, -g);
}

// Logits gradient from precomputed row logsumexp (grid (rows, chunks)):
//   g[v] = exp(x[v] - lse) * (1 + 2 z lse) * scale - scale * [v == label - offset]
// rows whose label equals ignore_index get zeros. Used by the linear-CE path
// after the row statistics are complete (locally or across vocab shards).
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
logits_grad_kernel(const T* logits, T* dlogits, const int64_t* __restrict__ labels,
                   const float* __restrict__ lse, int64_t rows, int64_t V, int64_t chunk,
                   float zmul, int64_t ignore, int64_t offset, const float* scale_ptr) {
  const int64_t row = blockIdx.x;
  const int64_t c0 = (int64_t)blockIdx.y * chunk;
  if (c0 >= V) return;
  const int64_t n = c0 + chunk < V ? chunk : V - c0;
  const int64_t lab = labels[row];
  T* y = dlogits + row * V + c0;
  if (lab == ignore) {
    row_zero<T, THREADS>(y, n);
    return;
  }
  const float l = lse[row];
  const float scale = scale_ptr ? *scale_ptr : 1.f;
  const float coef = scale * (1.f + 2.f * zmul * l);
  row_grad<T, THREADS, kUnroll>(logits + row * V + c0, y, n, lab - offset - c0, l * kLog2e, coef,
                                scale);
}

// ---------------------------------------------------------------------------
// Host side.

struct WsLayout {
  size_t status = 0;   // int
  size_t scale = 4;    // float
  size_t row_ce, row_z, xlab, part, total;
};

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cached[64] = {0};
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Plan {
  bool fused;
  int splits;
  int64_t chunk;
};

Plan plan_rows(int64_t rows, int64_t V, int elt) {
  Plan p;
  const int sms = num_sms();
  if (rows >= 2 * sms || V <= 2048) {
    p.fused = true;
    p.splits = 1;
    p.chunk = V;
    return p;
  }
  int64_t want = (4 * (int64_t)sms + rows - 1) / rows;  // CTAs per row
  int64_t max_by_size = (V + 2047) / 2048;               // >= 2048 elements per chunk
  int64_t s = want < max_by_size ? want : max_by_size;
  if (s < 1) s = 1;
  if (s > 1024) s = 1024;
  const int per = 16 / elt;
  int64_t chunk = (V + s - 1) / s;
  chunk = (chunk + per - 1) / per * per;  // keep chunk starts vector-aligned
  s = (V + chunk - 1) / chunk;
  p.fused = false;
  p.splits = (int)s;
  p.chunk = chunk;
  return p;
}

WsLayout layout(int64_t rows, const Plan& p) {
  WsLayout w;
  size_t off = 256;
  w.row_ce = off; off = align256(off + sizeof(float) * rows);
  w.row_z = off;  off = align256(off + sizeof(float) * rows);
  w.xlab = off;   off = align256(off + sizeof(float) * rows);
  w.part = off;   off = align256(off + sizeof(float2) * rows * (p.fused ? 0 : p.splits));
  w.total = off;
  return w;
}

template <typename T>
int launch_ce(const void* logits, void* dlogits, const int64_t* labels, int64_t rows, int64_t V,
              float zmul, int64_t ignore, int mean, const float* gscale, float* ce_sum,
              float* z_sum, float* n_valid, float* lse_out, char* ws,
              const Plan& p, const WsLayout& w, cudaStream_t st) {
  int* status = reinterpret_cast<int*>(ws + w.status);
  float* scale = reinterpret_cast<float*>(ws + w.scale);
  float* row_ce = reinterpret_cast<float*>(ws + w.row_ce);
  float* row_z = reinterpret_cast<float*>(ws + w.row_z);
  const T* x = static_cast<const T*>(logits);
  T* y = static_cast<T*>(dlogits);
  int launches = 0;
  cudaMemsetAsync(status, 0, sizeof(int), st);
  if (mean && y) {
    mean_scale_kernel<<<1, 1024, 0, st>>>(labels, rows, ignore, gscale, scale);
    ++launches;
  }
  const float* sp = (mean && y) ? scale : gscale;
  ProfScope prof(PROF_ROWS, st);
  if (rows > 0) {
    if (p.fused) {
      int64_t grid = rows;
      const int64_t cap = (int64_t)num_sms() * 2 * 64;
      if (grid > cap) grid = cap;
      // 32-byte vectors in flight per thread: 3 (measured at cfg2: 2 -> 5.02,
      // 3 -> 5.19, 4 -> 4.84 TB/s, the last spilling registers);
      // GREYHOUND_B200_CE_UNROLL = 2 or 4 selects the others
      const char* ue = getenv("GREYHOUND_B200_CE_UNROLL");
      const int un = ue && *ue ? atoi(ue) : 3;
      if (un == 3)
        ce_fused_kernel<T, kFusedThreads, 3><<<(unsigned)grid, kFusedThreads, 0, st>>>(
            x, y, labels, rows, V, zmul, ignore, sp, row_ce, row_z, lse_out, status);
      else if (un == 4)
        ce_fused_kernel<T, kFusedThreads, 4><<<(unsigned)grid, kFusedThreads, 0, st>>>(
            x, y, labels, rows, V, zmul, ignore, sp, row_ce, row_z, lse_out, status);
      else
        ce_fused_kernel<T, kFusedThreads, kUnroll><<<(unsigned)grid, kFusedThreads, 0, st>>>(
            x, y, labels, rows, V, zmul, ignore, sp, row_ce, row_z, lse_out, status);
      ++launches;
    } else {
      float2* part = reinterpret_cast<float2*>(ws + w.part);
      float* xlab = reinterpret_cast<float*>(ws + w.xlab);
      dim3 grid(p.splits, (unsigned)rows);
      split_stats_kernel<T, int64_t, kSplitThreads><<<grid, kSplitThreads, 0, st>>>(
          x, labels, rows, V, p.chunk, p.splits, part, xlab);
      ce_split_grad_kernel<T, kSplitThreads><<<grid, kSplitThreads, 0, st>>>(
          x, y, labels, rows, V, p.chunk, p.splits, part, xlab, zmul, ignore, sp, row_ce, row_z,
          lse_out, status);
      launches += 2;
    }
  }
  ce_finalize_kernel<<<1, 1024, 0, st>>>(row_ce, row_z, labels, rows, ignore, ce_sum, z_sum,
                                         n_valid);
  ++launches;
  count_launch(launches);
  return check_launch("gh_ce_fwd_grad");
}

template <typename T, typename I, typename O>
int launch_sls(const void* logits, const void* index, int64_t rows, int64_t V, void* out,
               float* lse_out, char* ws, const Plan& p, const WsLayout& w, cudaStream_t st) {
  int* status = reinterpret_cast<int*>(ws + w.status);
  const T* x = static_cast<const T*>(logits);
  const I* idx = static_cast<const I*>(index);
  O* o = static_cast<O*>(out);
  cudaMemsetAsync(status, 0, sizeof(int), st);
  if (rows == 0) return check_launch("gh_sls_fwd");
  ProfScope prof(PROF_ROWS, st);
  if (p.fused) {
    int64_t grid = rows;
    const int64_t cap = (int64_t)num_sms() * 2 * 64;
    if (grid > cap) grid = cap;
    sls_fused_kernel<T, I, O, kFusedThreads, kUnroll><<<(unsigned)grid, kFusedThreads, 0, st>>>(
        x, idx, rows, V, o, lse_out, status);
    count_launch(1);
  } else {
    float2* part = reinterpret_cast<float2*>(ws + w.part);
    float* xlab = reinterpret_cast<float*>(ws + w.xlab);
    dim3 grid(p.splits, (unsigned)rows);
    split_stats_kernel<T, I, kSplitThreads><<<grid, kSplitThreads, 0, st>>>(
        x, idx, rows, V, p.chunk, p.splits, part, xlab);
    sls_split_finish_kernel<I, O, kSplitThreads><<<(unsigned)rows, kSplitThreads, 0, st>>>(
        idx, rows, V, p.splits, part, xlab, o, lse_out, status);
    count_launch(2);
  }
  return check_launch("gh_sls_fwd");
}

template <typename T, typename I, typename G>
int launch_sls_bwd(const void* logits, const void* index, const float* lse, const void* g,
                   int64_t rows, int64_t V, void* grad, cudaStream_t st) {
  if (rows == 0) return GH_OK;
  const int sms = num_sms();
  int64_t want = (8 * (int64_t)sms + rows - 1) / rows;
  int64_t max_by_size = (V + 4095) / 4096;
  int64_t s = want < max_by_size ? want : max_by_size;
  if (s < 1) s = 1;
  const int per = 16 / (int)sizeof(T);
  int64_t chunk = (V + s - 1) / s;
  chunk = (chunk + per - 1) / per * per;
  s = (V + chunk - 1) / chunk;
  dim3 grid((unsigned)rows, (unsigned)s);
  sls_bwd_kernel<T, I, G, kSplitThreads><<<grid, kSplitThreads, 0, st>>>(
      static_cast<const T*>(logits), static_cast<const I*>(index), lse,
      static_cast<const G*>(g), rows, V, chunk, static_cast<T*>(grad));
  count_launch(1);
  return check_launch("gh_sls_bwd");
}

bool is_float_dtype(int d) { return d == GH_F16 || d == GH_BF16 || d == GH_F32; }

template <typename T>
int launch_logits_grad(const void* logits, void* dlogits, const int64_t* labels, const float* lse,
                       int64_t rows, int64_t V, float zmul, int64_t ignore, int64_t offset,
                       const float* scale, cudaStream_t st) {
  if (rows == 0) return GH_OK;
  const int sms = num_sms();
  int64_t want = (8 * (int64_t)sms + rows - 1) / rows;
  int64_t max_by_size = (V + 4095) / 4096;
  int64_t s = want < max_by_size ? want : max_by_size;
  if (s < 1) s = 1;
  const int per = 16 / (int)sizeof(T);
  int64_t chunk = (V + s - 1) / s;
  chunk = (chunk + per - 1) / per * per;
  s = (V + chunk - 1) / chunk;
  dim3 grid((unsigned)rows, (unsigned)s);
  logits_grad_kernel<T, kSplitThreads><<<grid, kSplitThreads, 0, st>>>(
      static_cast<const T*>(logits), static_cast<T*>(dlogits), labels, lse, rows, V, chunk, zmul,
      ignore, offset, scale);
  count_launch(1);
  return check_launch("gh_logits_grad");
}

}  // namespace
}  // namespace gh

using namespace gh;

extern "C" size_t gh_ce_workspace_bytes(int64_t rows, int64_t vocab, int dtype) {
  int elt = elt_size(dtype);
  if (elt == 0 || rows < 0 || vocab <= 0) return 0;
  Plan p = plan_rows(rows, vocab, elt);
  return layout(rows, p).total;
}

extern "C" size_t gh_sls_workspace_bytes(int64_t rows, int64_t vocab, int dtype) {
  return gh_ce_workspace_bytes(rows, vocab, dtype);
}

// publish: end with publish_status (the pinned error slots are allocated on
// first use, so the allocation-free entry point passes false).
static int ce_fwd_grad_impl(const void* logits, void* dlogits, const int64_t* labels, int64_t rows, int64_t vocab,
                            int dtype, float z_loss_multiplier, int64_t ignore_index, int mean_reduction,
                            const float* grad_scale, float* ce_sum, float* z_sum, float* n_valid, float* lse_out,
                            void* workspace, size_t workspace_bytes, void* stream, bool publish) {
  if (!is_float_dtype(dtype)) return set_error(GH_ETYPE, "unsupported logits dtype code %d", dtype);
  if (rows < 0 || vocab <= 0) return set_error(GH_EINVAL, "bad shape rows=%lld vocab=%lld",
                                                (long long)rows, (long long)vocab);
  if ((rows > 0 && (!logits || !labels)) || !ce_sum || !z_sum || !n_valid || !workspace)
    return set_error(GH_EINVAL, "null pointer argument");
  const int elt = elt_size(dtype);
  if (dlogits && ((reinterpret_cast<uintptr_t>(dlogits) - reinterpret_cast<uintptr_t>(logits)) & 15))
    return set_error(GH_EINVAL, "dlogits must share the 16-byte alignment of logits");
  Plan p = plan_rows(rows, vocab, elt);
  WsLayout w = layout(rows, p);
  if (workspace_bytes < w.total)
    return set_error(GH_EWORKSPACE, "workspace too small: %zu < %zu", workspace_bytes, w.total);
  if (!p.fused && rows > 65535) p.fused = true;  // grid.y limit; unreachable by plan_rows
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int rc;
  switch (dtype) {
    case GH_BF16:
      rc = launch_ce<__nv_bfloat16>(logits, dlogits, labels, rows, vocab, z_loss_multiplier, ignore_index,
                                    mean_reduction, grad_scale, ce_sum, z_sum, n_valid, lse_out, ws, p, w, st);
      break;
    case GH_F16:
      rc = launch_ce<__half>(logits, dlogits, labels, rows, vocab, z_loss_multiplier, ignore_index, mean_reduction,
                             grad_scale, ce_sum, z_sum, n_valid, lse_out, ws, p, w, st);
      break;
    default:
      rc = launch_ce<float>(logits, dlogits, labels, rows, vocab, z_loss_multiplier, ignore_index, mean_reduction,
                            grad_scale, ce_sum, z_sum, n_valid, lse_out, ws, p, w, st);
      break;
  }
  if (rc || !publish) return rc;
  return publish_status(reinterpret_cast<int*>(ws + w.status), st);
}

extern "C" int gh_ce_fwd_grad(const void* logits, void* dlogits, const int64_t* labels,
                              int64_t rows, int64_t vocab, int dtype, float z_loss_multiplier,
                              int64_t ignore_index, int mean_reduction,
                              const float* grad_scale, float* ce_sum, float* z_sum,
                              float* n_valid, float* lse_out, void* workspace, size_t workspace_bytes,
                              void* stream) {
  return ce_fwd_grad_impl(logits, dlogits, labels, rows, vocab, dtype, z_loss_multiplier, ignore_index,
                          mean_reduction, grad_scale, ce_sum, z_sum, n_valid, lse_out, workspace, workspace_bytes,
                          stream, true);
}

template <typename T, typename I>
static int sls_dispatch_out(const void* logits, const void* index, int64_t rows, int64_t V,
                            void* out, int out_dtype, float* lse_out, char* ws, const Plan& p,
                            const WsLayout& w, cudaStream_t st) {
  switch (out_dtype) {
    case GH_BF16: return launch_sls<T, I, __nv_bfloat16>(logits, index, rows, V, out, lse_out, ws, p, w, st);
    case GH_F16: return launch_sls<T, I, __half>(logits, index, rows, V, out, lse_out, ws, p, w, st);
    case GH_F32: return launch_sls<T, I, float>(logits, index, rows, V, out, lse_out, ws, p, w, st);
    default: return set_error(GH_ETYPE, "unsupported output dtype code %d", out_dtype);
  }
}

template <typename T>
static int sls_dispatch_idx(const void* logits, const void* index, int index_dtype, int64_t rows,
                            int64_t V, void* out, int out_dtype, float* lse_out, char* ws,
                            const Plan& p, const WsLayout& w, cudaStream_t st) {
  if (index_dtype == GH_I64)
    return sls_dispatch_out<T, int64_t>(logits, index, rows, V, out, out_dtype, lse_out, ws, p, w, st);
  return sls_dispatch_out<T, int32_t>(logits, index, rows, V, out, out_dtype, lse_out, ws, p, w, st);
}

extern "C" int gh_sls_fwd(const void* logits, const void* index, int index_dtype, int64_t rows,
                          int64_t vocab, int dtype, void* out, int out_dtype, float* lse_out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!is_float_dtype(dtype)) return set_error(GH_ETYPE, "unsupported logits dtype code %d", dtype);
  if (index_dtype != GH_I32 && index_dtype != GH_I64)
    return set_error(GH_ETYPE, "expected int32 or int64 index, got dtype code %d", index_dtype);
  if (!is_float_dtype(out_dtype)) return set_error(GH_ETYPE, "unsupported output dtype code %d", out_dtype);
  if (rows < 0 || vocab <= 0) return set_error(GH_EINVAL, "expected non-empty vocabulary dimension");
  if ((rows > 0 && (!logits || !index || !out)) || !workspace)
    return set_error(GH_EINVAL, "null pointer argument");
  Plan p = plan_rows(rows, vocab, elt_size(dtype));
  WsLayout w = layout(rows, p);
  if (workspace_bytes < w.total)
    return set_error(GH_EWORKSPACE, "workspace too small: %zu < %zu", workspace_bytes, w.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int rc;
  switch (dtype) {
    case GH_BF16: rc = sls_dispatch_idx<__nv_bfloat16>(logits, index, index_dtype, rows, vocab, out, out_dtype, lse_out, ws, p, w, st); break;
    case GH_F16: rc = sls_dispatch_idx<__half>(logits, index, index_dtype, rows, vocab, out, out_dtype, lse_out, ws, p, w, st); break;
    default: rc = sls_dispatch_idx<float>(logits, index, index_dtype, rows, vocab, out, out_dtype, lse_out, ws, p, w, st); break;
  }
  return rc ? rc : publish_status(reinterpret_cast<int*>(ws + w.status), st);
}

template <typename T, typename I>
static int sls_bwd_dispatch_g(const void* logits, const void* index, const float* lse,
                              const void* g, int gd, int64_t rows, int64_t V, void* grad,
                              cudaStream_t st) {
  switch (gd) {
    case GH_BF16: return launch_sls_bwd<T, I, __nv_bfloat16>(logits, index, lse, g, rows, V, grad, st);
    case GH_F16: return launch_sls_bwd<T, I, __half>(logits, index, lse, g, rows, V, grad, st);
    case GH_F32: return launch_sls_bwd<T, I, float>(logits, index, lse, g, rows, V, grad, st);
    default: return set_error(GH_ETYPE, "unsupported grad_out dtype code %d", gd);
  }
}

template <typename T>
static int sls_bwd_dispatch_i(const void* logits, const void* index, int id, const float* lse,
                              const void* g, int gd, int64_t rows, int64_t V, void* grad,
                              cudaStream_t st) {
  if (id == GH_I64) return sls_bwd_dispatch_g<T, int64_t>(logits, index, lse, g, gd, rows, V, grad, st);
  return sls_bwd_dispatch_g<T, int32_t>(logits, index, lse, g, gd, rows, V, grad, st);
}

extern "C" int gh_sls_bwd(const void* logits, const void* index, int index_dtype, const float* lse,
                          const void* grad_out, int grad_dtype, int64_t rows, int64_t vocab,
                          int dtype, void* grad_logits, void* stream) {
  if (!is_float_dtype(dtype)) return set_error(GH_ETYPE, "unsupported logits dtype code %d", dtype);
  if (index_dtype != GH_I32 && index_dtype != GH_I64)
    return set_error(GH_ETYPE, "expected int32 or int64 index, got dtype code %d", index_dtype);
  if (rows < 0 || vocab <= 0) return set_error(GH_EINVAL, "expected non-empty vocabulary dimension");
  if (rows > 0 && (!logits || !index || !lse || !grad_out || !grad_logits))
    return set_error(GH_EINVAL, "null pointer argument");
  if ((reinterpret_cast<uintptr_t>(grad_logits) - reinterpret_cast<uintptr_t>(logits)) & 15)
    return set_error(GH_EINVAL, "grad_logits must share the 16-byte alignment of logits");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GH_BF16: return sls_bwd_dispatch_i<__nv_bfloat16>(logits, index, index_dtype, lse, grad_out, grad_dtype, rows, vocab, grad_logits, st);
    case GH_F16: return sls_bwd_dispatch_i<__half>(logits, index, index_dtype, lse, grad_out, grad_dtype, rows, vocab, grad_logits, st);
    default: return sls_bwd_dispatch_i<float>(logits, index, index_dtype, lse, grad_out, grad_dtype, rows, vocab, grad_logits, st);
  }
}

extern "C" int gh_logits_grad(const void* logits, void* dlogits, const int64_t* labels,
                              const float* lse, int64_t rows, int64_t vocab, int dtype,
                              float z_loss_multiplier, int64_t ignore_index, int64_t label_offset,
                              const float* grad_scale, void* stream) {
  if (!is_float_dtype(dtype)) return set_error(GH_ETYPE, "unsupported logits dtype code %d", dtype);
  if (rows < 0 || vocab <= 0) return set_error(GH_EINVAL, "bad shape");
  if (rows > 0 && (!logits || !dlogits || !labels || !lse))
    return set_error(GH_EINVAL, "null pointer argument");
  if ((reinterpret_cast<uintptr_t>(dlogits) - reinterpret_cast<uintptr_t>(logits)) & 15)
    return set_error(GH_EINVAL, "dlogits must share the 16-byte alignment of logits");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GH_BF16: return launch_logits_grad<__nv_bfloat16>(logits, dlogits, labels, lse, rows, vocab, z_loss_multiplier, ignore_index, label_offset, grad_scale, st);
    case GH_F16: return launch_logits_grad<__half>(logits, dlogits, labels, lse, rows, vocab, z_loss_multiplier, ignore_index, label_offset, grad_scale, st);
    default: return launch_logits_grad<float>(logits, dlogits, labels, lse, rows, vocab, z_loss_multiplier, ignore_index, label_offset, grad_scale, st);
  }
}

// out[i] = in[i] * (*g): the backward of an op whose gradients were computed
// in the forward (ops/*: grad * grad_output), vectorised, g read on the device.
namespace gh {
namespace {
template <typename T>
__global__ void __launch_bounds__(256) scale_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t n,
                                                    const float* __restrict__ g) {
  constexpr int PER = 16 / sizeof(T);
  const float s = *g;
  const int64_t nvec = n / PER;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    Vec16<T> v;
    v.raw = ld16(reinterpret_cast<const uint4*>(in) + i);
    float f[PER];
    v.to_float(f);
#pragma unroll
    for (int k = 0; k < PER; ++k) f[k] *= s;
    v.from_float(f);
    st16_cs(reinterpret_cast<uint4*>(out) + i, v.raw);
  }
  for (int64_t i = nvec * PER + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = Elt<T>::from_f(Elt<T>::to_f(in[i]) * s);
}
}  // namespace
}  // namespace gh

extern "C" int gh_scale(const void* in, void* out, int64_t n, int dtype, const float* g, void* stream) {
  if (!is_float_dtype(dtype)) return set_error(GH_ETYPE, "unsupported dtype code %d", dtype);
  if (n < 0 || (n > 0 && (!in || !out || !g))) return set_error(GH_EINVAL, "bad arguments");
  if (n == 0) return GH_OK;
  if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(GH_EINVAL, "gh_scale needs 16-byte aligned buffers");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = num_sms();
  int64_t blocks = (n / (16 / elt_size(dtype)) + 255) / 256;
  if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
  if (blocks < 1) blocks = 1;
  switch (dtype) {
    case GH_BF16: scale_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), n, g); break;
    case GH_F16: scale_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __half*>(in), static_cast<__half*>(out), n, g); break;
    default: scale_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(in), static_cast<float*>(out), n, g); break;
  }
  count_launch(1);
  return check_launch("gh_scale");
}

// ---------------------------------------------------------------------------
// Allocation-free variant of gh_ce_fwd_grad.
//
// Some callers cannot allocate device memory at all at the point where they
// need the loss: code running under an allocator that forbids it, custom
// runtimes with their own pool that does not hand out scratch, or a host
// language binding with no device allocator of its own. For them the scratch
// lives in a fixed, library-owned device array instead of a caller workspace.
// Every GPU that loads this library holds the array (GH_CE_NOALLOC_SCRATCH_BYTES)
// until the process exits.
namespace gh {
namespace {
constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_ce_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array for the current device. The array's
// host-side name is only a stand-in, so the address is looked up once per
// device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(GH_EUNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ce_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(GH_ECUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GH_OK;
}
}  // namespace
}  // namespace gh

extern "C" size_t gh_ce_noalloc_scratch_bytes(void) { return gh::kNoAllocScratchBytes; }

extern "C" int gh_ce_fwd_grad_noalloc(const void* logits, void* dlogits, const int64_t* labels, int64_t rows,
                                      int64_t vocab, int dtype, float z_loss_multiplier, int64_t ignore_index,
                                      int mean_reduction, const float* grad_scale, float* ce_sum, float* z_sum,
                                      float* n_valid, float* lse_out, void* stream) {
  const size_t need = gh_ce_workspace_bytes(rows, vocab, dtype);
  if (need == 0 && (!is_float_dtype(dtype)))
    return set_error(GH_ETYPE, "unsupported logits dtype code %d", dtype);
  if (need > kNoAllocScratchBytes)
    return set_error(GH_EWORKSPACE,
                     "gh_ce_fwd_grad_noalloc: %lld rows x %lld vocab need %zu scratch bytes, more than the "
                     "fixed %zu; use gh_ce_fwd_grad with a caller workspace",
                     (long long)rows, (long long)vocab, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return ce_fwd_grad_impl(logits, dlogits, labels, rows, vocab, dtype, z_loss_multiplier, ignore_index,
                          mean_reduction, grad_scale, ce_sum, z_sum, n_valid, lse_out, scratch,
                          kNoAllocScratchBytes, stream, false);
}

extern "C" int gh_ce_noalloc_status(int* host_out, void* stream) {
  if (!host_out) return set_error(GH_EINVAL, "null pointer argument");
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // the status word sits at offset 0 of the shared scratch (as in any workspace)
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(host_out, scratch, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "gh_ce_noalloc_status: %s", cudaGetErrorString(e));
  return GH_OK;
}
