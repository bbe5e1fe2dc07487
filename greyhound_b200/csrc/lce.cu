// Chunked linear cross-entropy on the tcgen05 GEMM, plus the generic GEMM
// entry point used by the bring-your-own-loss path.
//
// Per row chunk [s, e) (the reference loop, src/greyhound/ops/chunked_linear_loss.py:79-101,
// with the CE callback of src/greyhound/ops/chunked_linear_cross_entropy.py:43-59):
//   1. logits GEMM with the fused CE epilogue: bf16 logits tile to the
//      workspace + per-(row, 256-column tile) (max, sum-exp) + target logit
//   2. row combine: exact logsumexp per row, per-row ce / z terms
//   3. logits -> dlogits in place: softmax * (1 + 2 z lse) * s - s * onehot
//      (s = 1/max(n_valid,1) for the mean, folded in here instead of two
//      mul_ passes over grad_input / grad_weight afterwards)
//   4. dW GEMM (dlogits^T @ H), written as [V, D]; fp32 or weight-dtype
//      accumulation across chunks through the epilogue addend
//   5. dH GEMM (dlogits @ W), rows [s, e) of grad_input
// and once at the end a fixed-order reduction of the per-row loss terms.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "row_ops.cuh"
#include "tc_gemm.cuh"

namespace gh {
namespace {

using gemm::BK;
using gemm::BM;
using gemm::BN;

// ---------------------------------------------------------------------------
// Tensor maps

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D map over a row-major matrix [outer, inner] with row pitch `ld`
// elements, box {64, box_outer}, 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t inner, int64_t outer, int64_t ld,
             int box_outer) {
  // A host thread that has made no runtime call yet (autograd's backward
  // thread for device 0, for one) has no current context, and the driver
  // call below needs one: bind the current device's primary context.
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  auto enc = get_encode();
  if (!enc) return set_error(GH_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const int elt = elt_size(dtype);
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((ld * elt) & 15))
    return set_error(GH_EUNSUPPORTED, "GEMM operand needs a 16-byte aligned base and row pitch (pitch %lld elements)",
                     (long long)ld);
  CUtensorMapDataType dt = dtype == GH_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t gstride[1] = {(cuuint64_t)(ld * elt)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(GH_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GH_OK;
}

int num_sms_dev() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cached[64] = {0};
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

// One GEMM operand: pointer, pitch, majorness.
struct Operand {
  const void* ptr;
  int64_t ld;
  int mn_major;  // 0: [rows, K] K contiguous; 1: [K, rows] rows contiguous
};

template <typename T, int A_MN, int B_MN, int EPI, typename OutT, int PAIR, int NSUB = 1>
int launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, gemm::Params& p, int max_ctas, cudaStream_t st) {
  auto kern = gemm::tc_gemm_kernel<T, A_MN, B_MN, EPI, OutT, PAIR, NSUB>;
  constexpr int SMEM = gemm::Geo<PAIR, NSUB>::SMEM;
  static int max_units[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return set_error(GH_EUNSUPPORTED, "device index >= 64");
  if (!max_units[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    int units = num_sms_dev() / PAIR;
    if (PAIR > 1) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(units * PAIR);
      cfg.blockDim = dim3(gemm::THREADS);
      cfg.dynamicSmemBytes = SMEM;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = PAIR;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0 && n < units) units = n;
      cudaGetLastError();
    }
    max_units[dev] = units;
  }
  int units = max_units[dev];
  if (max_ctas > 0 && max_ctas / PAIR < units) units = max_ctas / PAIR > 0 ? max_ctas / PAIR : 1;
  if (p.num_tiles < units) units = p.num_tiles;
  if (units <= 0) return GH_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(units * PAIR);
  cfg.blockDim = dim3(gemm::THREADS);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = PAIR;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "tc_gemm launch: %s", cudaGetErrorString(e));
  count_launch(1);
  return check_launch("tc_gemm");
}

// Dispatch on majorness, pairing and tile width for a fixed (T, EPI, OutT).
template <typename T, int EPI, typename OutT>
int launch_gemm_mm(const CUtensorMap& ta, const CUtensorMap& tb, int a_mn, int b_mn, int pair, int nsub,
                   gemm::Params& p, int max_ctas, cudaStream_t st) {
  if (pair == 2 && nsub == 2) {
    if constexpr (sizeof(OutT) == 2 && EPI != gemm::EPI_LCE_Q) {
      if (p.add_f32 || p.add_same) return set_error(GH_EUNSUPPORTED, "512-column GEMM tile with an addend");
      if (!a_mn && !b_mn) return launch_gemm_t<T, 0, 0, EPI, OutT, 2, 2>(ta, tb, p, max_ctas, st);
      if (!a_mn && b_mn) return launch_gemm_t<T, 0, 1, EPI, OutT, 2, 2>(ta, tb, p, max_ctas, st);
      if (a_mn && !b_mn) return launch_gemm_t<T, 1, 0, EPI, OutT, 2, 2>(ta, tb, p, max_ctas, st);
      return launch_gemm_t<T, 1, 1, EPI, OutT, 2, 2>(ta, tb, p, max_ctas, st);
    } else {
      return set_error(GH_EUNSUPPORTED, "512-column GEMM tile with an fp32 output");
    }
  }
  if (pair == 2) {
    if (!a_mn && !b_mn) return launch_gemm_t<T, 0, 0, EPI, OutT, 2>(ta, tb, p, max_ctas, st);
    if (!a_mn && b_mn) return launch_gemm_t<T, 0, 1, EPI, OutT, 2>(ta, tb, p, max_ctas, st);
    if (a_mn && !b_mn) return launch_gemm_t<T, 1, 0, EPI, OutT, 2>(ta, tb, p, max_ctas, st);
    return launch_gemm_t<T, 1, 1, EPI, OutT, 2>(ta, tb, p, max_ctas, st);
  }
  if (!a_mn && !b_mn) return launch_gemm_t<T, 0, 0, EPI, OutT, 1>(ta, tb, p, max_ctas, st);
  if (!a_mn && b_mn) return launch_gemm_t<T, 0, 1, EPI, OutT, 1>(ta, tb, p, max_ctas, st);
  if (a_mn && !b_mn) return launch_gemm_t<T, 1, 0, EPI, OutT, 1>(ta, tb, p, max_ctas, st);
  return launch_gemm_t<T, 1, 1, EPI, OutT, 1>(ta, tb, p, max_ctas, st);
}

// 2-CTA tiles (256 rows) once there are more than 128 rows.
inline int pick_pair(int64_t M) { return M > BM ? 2 : 1; }

// Tile width of a paired GEMM: 512 columns (NSUB = 2) unless the coarser
// tiles would leave a last wave much emptier than 256-column tiles do. The
// wide tile is credited with 6 % (its measured energy saving at the power
// cap). Outputs that need an fp32 epilogue (fp32 output, an addend) keep 256
// columns: only 16-bit outputs can be parked in registers to free TMEM early.
// The linear-CE epilogue (logits + statistics, ~4k cycles per 32-column chunk
// next to the MMAs) also keeps 256 columns: with 512 the tensor pipe waited
// ~18 % of each tile for it (measured), while two 256-column accumulators
// hide it completely. GREYHOUND_B200_GEMM_WIDE=0 forces 256 columns, =2
// forces 512 wherever the output allows it.
inline int wide_mode() {
  static int mode = [] {
    const char* e = getenv("GREYHOUND_B200_GEMM_WIDE");
    return e && *e ? atoi(e) : 1;
  }();
  return mode;
}
// Tiling of one GEMM: tile width (nsub) and split-K slices (ksplit).
struct Tiling {
  int nsub = 1, ksplit = 1;
};
// Split-K (2 slices, 512-column tiles; the slices write two 16-bit partials
// that a small kernel adds) when the caller provides the second output and
// the unsplit wide tiles would leave a short last wave: dH at the Llama-3-8B
// head (8192 x 4096 output) has 256 wide tiles for 74 pair units (a 46 %
// last wave) but 512 split units (6.9 full waves). Charged 1 % for the add.
inline Tiling pick_tiling(int64_t M, int64_t N, int64_t K, int pair, int units, bool fp32_epilogue,
                          bool lce_epilogue, bool split_ok = false) {
  Tiling t;
  if (pair != 2 || N <= BN || fp32_epilogue) return t;
  const int mode = wide_mode();
  if (mode != 1) {
    t.nsub = mode == 2 ? 2 : 1;
    return t;
  }
  if (lce_epilogue) return t;
  auto eff = [&](int64_t tn, int64_t ks) {
    const int64_t tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + tn - 1) / tn) * ks;
    const int64_t waves = (tiles + units - 1) / units;
    // useful columns per computed column (a partial last tile computes zeros)
    const double fill = (double)N / (double)(((N + tn - 1) / tn) * tn);
    return (double)tiles / (double)(waves * units) * fill;
  };
  const double narrow = eff(BN, 1), wide = eff(2 * BN, 1) * 1.06;
  // each slice keeps at least 4 stage rounds of k-steps
  const bool can_split = split_ok && (K + BK - 1) / BK >= 2 * 16;
  const double wide_split = can_split ? eff(2 * BN, 2) * 1.06 * 0.99 : 0.0;
  if (wide_split > wide * 1.02 && wide_split > narrow) {
    t.nsub = 2;
    t.ksplit = 2;
  } else if (wide >= narrow) {
    t.nsub = 2;
  }
  return t;
}
inline int pick_nsub(int64_t M, int64_t N, int pair, int units, bool fp32_epilogue, bool lce_epilogue) {
  return pick_tiling(M, N, 0, pair, units, fp32_epilogue, lce_epilogue).nsub;
}

// Tensor maps of both operands for a GEMM of M x N x K with pairing `pair`.
int make_operand_maps(CUtensorMap* ta, CUtensorMap* tb, int dtype, const Operand& A, const Operand& B, int64_t M,
                      int64_t N, int64_t K, int pair) {
  int rc;
  if (A.mn_major) rc = make_map(ta, A.ptr, dtype, M, K, A.ld, BK);
  else rc = make_map(ta, A.ptr, dtype, K, M, A.ld, BM);
  if (rc) return rc;
  if (B.mn_major) rc = make_map(tb, B.ptr, dtype, N, K, B.ld, BK);
  else rc = make_map(tb, B.ptr, dtype, K, N, B.ld, BN / pair);
  return rc;
}

void set_tiles(gemm::Params& p, int64_t M, int64_t N, int64_t K, int pair, int nsub = 1, int ksplit = 1) {
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_m = (int)((M + BM * pair - 1) / (BM * pair));
  p.num_n = (int)((N + BN * nsub - 1) / (BN * nsub));
  p.ksplit = ksplit;
  p.num_tiles = p.num_m * p.num_n * ksplit;
}

// Generic: D[M,N] = scale * A B^T (+ addend), D written as out_dtype with pitch ldo.
// L2 policies of one GEMM: operand loads (0 none, 1 evict_first, 2 evict_last)
// and evict-first output stores.
struct Hints {
  int a = 0, b = 0, out = 0;
};
// Logits GEMM tile order: groups of 16 m-tiles (4096 rows, 32 MB of H at
// D = 4096) sweep all vocab tiles before the next group starts. Measured at
// the Llama-3-8B head (ncu, DRAM read per launch): m-fastest 11.5-16 GB,
// groups of 4 / 8 / 12 / 24: 28 / 19 / 8.4 / 10 GB, groups of 16: 4.0-6.9 GB
// and 7-9 % less time. The dW GEMM keeps the n-fastest order (other orders
// and groupings read more).
constexpr int kLogitsGroup = 16;
// GREYHOUND_B200_LOGITS_GROUP overrides it (tuning sweeps)
inline int logits_group() {
  const char* e = getenv("GREYHOUND_B200_LOGITS_GROUP");
  const int g = e && *e ? atoi(e) : kLogitsGroup;
  return g >= 1 ? g : kLogitsGroup;
}
// dW / logits-style GEMMs: the 2 GB dlogits (or W) stream must not evict the
// small H operand that every tile re-reads.
constexpr Hints kStreamA_KeepB{1, 2, 1};
constexpr Hints kKeepA_StreamB{2, 1, 1};

// out[r, c] = out[r, c] + part[r, c] (16-bit, fp32 add, one rounding) over
// rows of pitch ld: the second split-K slice folded into the first.
template <typename T>
__global__ void __launch_bounds__(256) add_partial_kernel(T* out, const T* __restrict__ part, int64_t rows,
                                                          int64_t cols, int64_t ld) {
  constexpr int PER = 16 / sizeof(T);
  const int64_t vpr = cols / PER;  // whole vectors per row (rows are 16-byte aligned)
  const int64_t nvec = rows * vpr;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const int64_t r = i / vpr, c = (i - r * vpr) * PER;
    Vec16<T> a, b;
    a.raw = *reinterpret_cast<const uint4*>(out + r * ld + c);
    b.raw = ld16_last(part + r * ld + c);
    float fa[PER], fb[PER];
    a.to_float(fa);
    b.to_float(fb);
#pragma unroll
    for (int k = 0; k < PER; ++k) fa[k] += fb[k];
    a.from_float(fa);
    st16(out + r * ld + c, a.raw);
  }
  const int64_t tail = cols - vpr * PER;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * tail; i += stride) {
    const int64_t r = i / tail, c = vpr * PER + (i - r * tail);
    out[r * ld + c] = Elt<T>::from_f(Elt<T>::to_f(out[r * ld + c]) + Elt<T>::to_f(part[r * ld + c]));
  }
}

template <typename T>
int add_partial(void* out, const void* part, int64_t rows, int64_t cols, int64_t ld, int max_ctas, cudaStream_t st) {
  const int sms = num_sms_dev();
  int grid = 4 * (max_ctas > 0 && max_ctas < sms ? max_ctas : sms);
  add_partial_kernel<T><<<grid, 256, 0, st>>>(static_cast<T*>(out), static_cast<const T*>(part), rows, cols, ld);
  count_launch(1);
  return check_launch("add_partial");
}

// Output rows split into bands stored on the ranks that reduce them
// (gemm::Params::peer_out).
struct PeerOut {
  int n = 0;
  int64_t rows = 0;
  int first = 0;  // band whose tiles this GEMM computes first
  void* ptr[gemm::kMaxPeers] = {};
};

int run_gemm(int dtype, const Operand& A, const Operand& B, int64_t M, int64_t N, int64_t K, void* out,
             int out_dtype, int64_t ldo, const float* add_f32, const void* add_same, int64_t ldadd,
             const float* scale, int raster, int max_ctas, cudaStream_t st, int* status,
             int prof_class = PROF_GEMM_OTHER, Hints hints = Hints{}, void* split_out = nullptr,
             const float* row_scale = nullptr, const PeerOut* peers = nullptr) {
  if (M <= 0 || N <= 0) return GH_OK;
  if (K <= 0) return set_error(GH_EINVAL, "GEMM needs K >= 1");
  ProfScope prof(prof_class, st);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return set_error(GH_EINVAL, "GEMM dimension too large");
  const int pair = pick_pair(M);
  int units = num_sms_dev() / 2;
  if (max_ctas > 0 && max_ctas / 2 < units) units = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
  const bool split_ok = split_out && out_dtype != GH_F32 &&
                        ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(split_out) |
                          (uintptr_t)(ldo * elt_size(out_dtype))) & 15) == 0;
  const Tiling tl = pick_tiling(M, N, K, pair, units, out_dtype == GH_F32 || add_f32 || add_same, false, split_ok);
  const int nsub = tl.nsub;
  CUtensorMap ta, tb;
  int rc = make_operand_maps(&ta, &tb, dtype, A, B, M, N, K, pair);
  if (rc) return rc;
  gemm::Params p{};
  set_tiles(p, M, N, K, pair, nsub, tl.ksplit);
  p.out2 = tl.ksplit > 1 ? split_out : nullptr;
  p.raster = raster;
  p.group = 1;
  // tile-order override for the gradient GEMMs, "raster,group"
  // (GREYHOUND_B200_DW_ORDER / GREYHOUND_B200_DH_ORDER; tuning sweeps)
  if (prof_class == PROF_GEMM_DW || prof_class == PROF_GEMM_DH) {
    const char* e = getenv(prof_class == PROF_GEMM_DW ? "GREYHOUND_B200_DW_ORDER" : "GREYHOUND_B200_DH_ORDER");
    int r = -1, g = 1;
    if (e && *e && sscanf(e, "%d,%d", &r, &g) >= 1 && r >= 0 && r <= 3 && g >= 1) {
      p.raster = r;
      p.group = g;
    }
  }
  p.out = out;
  p.ldo = ldo;
  const int oelt = elt_size(out_dtype);
  p.vec_ok = ((reinterpret_cast<uintptr_t>(out) | (uintptr_t)(ldo * oelt)) & 15) == 0;
  if (add_f32) p.vec_ok &= ((reinterpret_cast<uintptr_t>(add_f32) | (uintptr_t)(ldadd * 4)) & 15) == 0;
  if (add_same) p.vec_ok &= ((reinterpret_cast<uintptr_t>(add_same) | (uintptr_t)(ldadd * oelt)) & 15) == 0;
  p.add_f32 = add_f32;
  p.add_same = add_same;
  p.ldadd = ldadd;
  p.scale = scale;
  p.row_scale = row_scale;
  if (peers && peers->n > 0) {
    if (out_dtype == GH_F32 || split_out || peers->n > gemm::kMaxPeers || peers->rows % (2 * BM))
      return set_error(GH_EUNSUPPORTED, "peer output: 16-bit output, no split-K, <= %d bands of a multiple of %d rows",
                       gemm::kMaxPeers, 2 * BM);
    p.npeer = peers->n;
    // start on band `first` (raster 1 walks the output rows band by band)
    if (raster == 1) p.tile_rot = (int)(((int64_t)peers->first * (peers->rows / (BM * pair)) * p.num_n) % p.num_tiles);
    p.peer_rows = peers->rows;
    for (int i = 0; i < peers->n; ++i) {
      p.peer_out[i] = peers->ptr[i];
      if (reinterpret_cast<uintptr_t>(peers->ptr[i]) & 15) p.vec_ok = 0;
    }
  }
  p.status = status;
  p.a_hint = hints.a;
  p.b_hint = hints.b;
  p.out_evict_first = hints.out;
  if (dtype == GH_BF16) {
    if (out_dtype == GH_F32) return launch_gemm_mm<__nv_bfloat16, gemm::EPI_STORE, float>(ta, tb, A.mn_major, B.mn_major, pair, nsub, p, max_ctas, st);
    if (out_dtype == GH_BF16) {
      rc = launch_gemm_mm<__nv_bfloat16, gemm::EPI_STORE, __nv_bfloat16>(ta, tb, A.mn_major, B.mn_major, pair, nsub, p, max_ctas, st);
      return rc || tl.ksplit == 1 ? rc : add_partial<__nv_bfloat16>(out, split_out, M, N, ldo, max_ctas, st);
    }
  } else if (dtype == GH_F16) {
    if (out_dtype == GH_F32) return launch_gemm_mm<__half, gemm::EPI_STORE, float>(ta, tb, A.mn_major, B.mn_major, pair, nsub, p, max_ctas, st);
    if (out_dtype == GH_F16) {
      rc = launch_gemm_mm<__half, gemm::EPI_STORE, __half>(ta, tb, A.mn_major, B.mn_major, pair, nsub, p, max_ctas, st);
      return rc || tl.ksplit == 1 ? rc : add_partial<__half>(out, split_out, M, N, ldo, max_ctas, st);
    }
  }
  return set_error(GH_ETYPE, "unsupported GEMM dtype combination (%d -> %d)", dtype, out_dtype);
}

// ---------------------------------------------------------------------------
// Linear-CE helper kernels

// Exact per-row logsumexp from the epilogue's per-tile (max, sum) pairs and
// the per-row loss terms (kernels/cross_entropy.py:84-92). Block = 32 rows x
// 8 warps: lane <-> row (coalesced reads of the [tile][row] partials), warps
// split the tiles, then one merge across warps.
// shard mode (stats3 != nullptr): rows hold only a vocab shard; write
// (lse_shard, 1, target logit or -inf) for the cross-shard exchange instead of
// loss terms.
constexpr int kCombineWarps = 8;
// q mode (qm != nullptr): the logits GEMM stored q = e^x per 128-column group
// (or raw logits, flagged in qm); also write alpha[r], the factor that turns
// the row's stored values into its logits gradient (s (1 + 2 z lse) e^-lse
// for a q row, s for a row the fix-up pass rewrites, 0 for an ignored row),
// and rowflag[r] = 1 when the row needs that fix-up.
struct QOut {
  const uint8_t* qm;
  const float* scale;  // s (nullptr: 1)
  float zmul;
  float* alpha;
  int* rowflag;
};

__global__ void __launch_bounds__(32 * kCombineWarps)
lce_combine_kernel(const float2* __restrict__ stats, int num_n, int64_t rows, const float* __restrict__ xt,
                   const int64_t* __restrict__ labels, int64_t label_offset, int64_t V, int64_t ignore,
                   float* lse_out, float* row_ce, float* row_z, float* stats3, int* status, QOut qo) {
  __shared__ float sm[kCombineWarps][32], ss[kCombineWarps][32];
  __shared__ int sf[kCombineWarps][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * 32 + lane;
  MS acc = ms_empty();
  int flag = 0;
  if (r < rows)
    for (int j = w; j < num_n; j += kCombineWarps) {
      const float2 p = stats[(int64_t)j * rows + r];
      acc = ms_merge(acc, MS{p.x, p.y});
      if (qo.qm) {
        // a group is only written when it has columns inside the vocabulary
        flag |= qo.qm[((int64_t)j * 2) * rows + r];
        if ((int64_t)j * BN + BN / 2 < V) flag |= qo.qm[((int64_t)j * 2 + 1) * rows + r];
      }
    }
  sm[w][lane] = acc.m;
  ss[w][lane] = acc.s;
  sf[w][lane] = flag;
  __syncthreads();
  if (w != 0 || r >= rows) return;
  for (int k = 1; k < kCombineWarps; ++k) {
    acc = ms_merge(acc, MS{sm[k][lane], ss[k][lane]});
    flag |= sf[k][lane];
  }
  const float lse = (acc.m + fast_log2(acc.s)) * kLn2;
  const int64_t t = labels[r];
  const int64_t loc = t - label_offset;
  if (stats3) {
    const bool inside = t != ignore && loc >= 0 && loc < V;
    stats3[3 * r + 0] = lse;
    stats3[3 * r + 1] = 1.f;
    stats3[3 * r + 2] = inside ? xt[r] : kNegInf;
    return;
  }
  bool valid = t != ignore;
  if (valid && (loc < 0 || loc >= V)) {
    atomicOr(status, GH_DEV_BAD_LABEL);
    valid = false;
  }
  lse_out[r] = lse;
  row_ce[r] = valid ? lse - xt[r] : 0.f;
  row_z[r] = valid ? lse * lse : 0.f;
  if (qo.qm) {
    const float s = qo.scale ? *qo.scale : 1.f;
    const float f = 1.f + 2.f * qo.zmul * lse;
    flag |= fabsf(f) < 1e-3f;
    qo.alpha[r] = !valid ? 0.f : flag ? s : s * f * fast_exp2(-lse * kLog2e);
    qo.rowflag[r] = valid && flag;
  }
}

// Fix-up of the rows that q mode cannot represent: a group whose largest
// logit lies outside the exponent window (stored raw), or a row whose z-loss
// factor 1 + 2 z lse is about 0. The row is rewritten as its logits gradient
// divided by s, (1 + 2 z lse) e^(x - lse) - onehot, from raw logits where a
// group holds them and from q = e^x elsewhere; its alpha is s. Grid (rows);
// rows without the flag return at once.
template <typename T>
__global__ void __launch_bounds__(256)
lce_q_fixup_kernel(T* q, int64_t ld, const uint8_t* __restrict__ qm, const int* __restrict__ rowflag,
                   const float* __restrict__ lse, const int64_t* __restrict__ labels, int64_t label_offset,
                   int64_t rows, int64_t V, float zmul) {
  const int64_t row = blockIdx.x;
  if (!rowflag[row]) return;
  const float l = lse[row];
  const float l2 = l * kLog2e;
  const float f = 1.f + 2.f * zmul * l;
  const int64_t t = labels[row] - label_offset;
  T* y = q + row * ld;
  for (int64_t c = threadIdx.x; c < V; c += blockDim.x) {
    const int64_t grp = (c >> 8) * 2 + ((c >> 7) & 1);
    const float v = Elt<T>::to_f(y[c]);
    float p;
    if (qm[grp * rows + row]) p = fast_exp2(fmaf(v, kLog2e, -l2));
    else p = v > 0.f ? fast_exp2(fast_log2(v) - l2) : 0.f;
    y[c] = Elt<T>::from_f(f * p - (c == t ? 1.f : 0.f));
  }
}

// out[r, :] = alpha[r] * H[r, :]: the dW GEMM's second operand in q mode.
template <typename T>
__global__ void __launch_bounds__(256)
scale_rows_kernel(const T* __restrict__ H, const float* __restrict__ alpha, int64_t rows, int64_t D,
                  T* __restrict__ out) {
  constexpr int PER = 16 / sizeof(T);
  const int64_t vpr = D / PER;
  const int64_t n = rows * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vpr;
    const float a = alpha[r];
    Vec16<T> v;
    v.raw = ld16(reinterpret_cast<const uint4*>(H) + i);
    float f[PER];
    v.to_float(f);
#pragma unroll
    for (int k = 0; k < PER; ++k) f[k] *= a;
    v.from_float(f);
    st16(reinterpret_cast<uint4*>(out) + i, v.raw);
  }
}

// Target column of the q-mode rows that the fix-up pass does not rewrite:
// q[r, t] = e^x_t - e^lse / (1 + 2 z lse), so that alpha[r] * q[r, t] =
// s (1 + 2 z lse) p_t - s, the reference's logits gradient at the target.
// Computed from the fp32 target logit (not from the rounded q), so the
// difference keeps its precision when p_t is close to 1 and is rounded once.
template <typename T>
__global__ void __launch_bounds__(256)
lce_q_target_kernel(T* q, int64_t ld, const int64_t* __restrict__ labels, const float* __restrict__ xt,
                    const float* __restrict__ lse, const int* __restrict__ rowflag, const float* __restrict__ alpha,
                    int64_t rows, int64_t V, int64_t ignore, float zmul) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int64_t t = labels[r];
  if (t == ignore || t < 0 || t >= V || rowflag[r] || alpha[r] == 0.f) return;
  const float l = lse[r];
  const float v = fast_exp2(xt[r] * kLog2e) - fast_exp2(l * kLog2e) / (1.f + 2.f * zmul * l);
  q[r * ld + t] = Elt<T>::from_f(v);
}

// In-place logits -> dlogits over a pitched [rows, ld] buffer; grid (rows, chunks).
// Rows with target == ignore get zeros. In shard mode the one-hot term is only
// subtracted when the target falls in this shard's columns; otherwise a target
// outside [0, V) marks a bad label (zero row, flagged by the combine kernel).
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
lce_dlogits_kernel(T* logits, int64_t ld, const int64_t* __restrict__ labels, int64_t label_offset, int shard,
                   const float* __restrict__ lse, int64_t V, int64_t chunk, float zmul, int64_t ignore,
                   const float* scale_ptr) {
  const int64_t row = blockIdx.x;
  const int64_t c0 = (int64_t)blockIdx.y * chunk;
  if (c0 >= V) return;
  const int64_t n = c0 + chunk < V ? chunk : V - c0;
  const int64_t t = labels[row];
  const int64_t loc = t - label_offset;
  T* y = logits + row * ld + c0;
  if (t == ignore || (!shard && (loc < 0 || loc >= V))) {
    row_zero<T, THREADS>(y, n);
    return;
  }
  const float l = lse[row];
  const float scale = scale_ptr ? *scale_ptr : 1.f;
  const float coef = scale * (1.f + 2.f * zmul * l);
  row_grad<T, THREADS, kUnroll>(y, y, n, loc - c0, l * kLog2e, coef, scale);
}

struct LceLayout {
  size_t status = 0, scale = 64;
  size_t logits, stats, xt, lse, row_ce, row_z, acc, dh2, total;
  // q mode only
  size_t qmode = 0, alpha = 0, rowflag = 0, hs = 0;
  int64_t chunk, ldl;
  int num_n;
  bool need_acc;
  bool q = false;
};

// q mode: the logits GEMM stores q = e^x (bf16) instead of the logits, and
// the gradient GEMMs apply the per-row factor and the one-hot term, so no
// pass reads and rewrites the [chunk, V] buffer. bf16 only (fp16's exponent
// range cannot hold e^x); GREYHOUND_B200_LCE_Q=0 switches it off.
inline bool q_mode_for(int dtype) {
  const char* e = getenv("GREYHOUND_B200_LCE_Q");
  return (e && *e ? atoi(e) : 1) && dtype == GH_BF16;
}

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

LceLayout lce_layout(int64_t N, int64_t D, int64_t V, int64_t chunk, int dtype, int fp32_accum,
                     bool loss_only = false) {
  LceLayout L;
  if (chunk <= 0 || chunk > N) chunk = N;
  L.chunk = chunk;
  L.ldl = (V + 7) / 8 * 8;  // 16-byte row pitch for TMA
  L.num_n = (int)((V + BN - 1) / BN);
  const int elt = elt_size(dtype);
  size_t off = 256;
  L.logits = off;
  if (!loss_only) off = al256(off + (size_t)chunk * L.ldl * elt);
  L.stats = off;  off = al256(off + sizeof(float2) * (size_t)L.num_n * chunk);
  L.xt = off;     off = al256(off + sizeof(float) * chunk);
  L.lse = off;    off = al256(off + sizeof(float) * chunk);
  L.row_ce = off; off = al256(off + sizeof(float) * N);
  L.row_z = off;  off = al256(off + sizeof(float) * N);
  const int64_t nchunks = N > 0 ? (N + chunk - 1) / chunk : 0;
  L.need_acc = !loss_only && fp32_accum && nchunks > 1;
  L.acc = off;
  if (L.need_acc) off = al256(off + sizeof(float) * (size_t)D * V);
  // second split-K partial of a chunk's dH [chunk, D]
  L.dh2 = off;
  if (!loss_only) off = al256(off + (size_t)chunk * D * elt);
  L.q = !loss_only && q_mode_for(dtype);
  if (L.q) {
    L.qmode = off;   off = al256(off + (size_t)L.num_n * 2 * chunk);
    L.alpha = off;   off = al256(off + sizeof(float) * chunk);
    L.rowflag = off; off = al256(off + sizeof(int) * chunk);
    L.hs = off;      off = al256(off + (size_t)chunk * D * elt);
  }
  L.total = off;
  return L;
}

template <typename T>
int lce_dlogits(T* logits, int64_t ld, const int64_t* labels, const float* lse, int64_t rows, int64_t V,
                float zmul, int64_t ignore, const float* scale, cudaStream_t st, int64_t label_offset = 0,
                int shard = 0) {
  if (rows <= 0) return GH_OK;
  const int sms = num_sms_dev();
  int64_t want = (8 * (int64_t)sms + rows - 1) / rows;
  int64_t max_by_size = (V + 4095) / 4096;
  int64_t s = want < max_by_size ? want : max_by_size;
  if (s < 1) s = 1;
  const int per = 16 / (int)sizeof(T);
  int64_t chunk = (V + s - 1) / s;
  chunk = (chunk + per - 1) / per * per;
  s = (V + chunk - 1) / chunk;
  dim3 grid((unsigned)rows, (unsigned)s);
  ProfScope prof(PROF_DLOGITS, st);
  lce_dlogits_kernel<T, 256><<<grid, 256, 0, st>>>(logits, ld, labels, label_offset, shard, lse, V, chunk, zmul,
                                                   ignore, scale);
  count_launch(1);
  return check_launch("lce_dlogits");
}

template <typename T>
int lce_run(const void* H, const void* W, const int64_t* target, int64_t N, int64_t D, int64_t V, int dtype,
            float zmul, int64_t ignore, int mean, const float* grad_scale, const LceLayout& L, int flags,
            void* grad_input, void* grad_weight, float* ce_sum, float* z_sum, float* n_valid, char* ws,
            cudaStream_t st) {
  int* status = reinterpret_cast<int*>(ws + L.status);
  float* scale = reinterpret_cast<float*>(ws + L.scale);
  T* logits = reinterpret_cast<T*>(ws + L.logits);
  float2* stats = reinterpret_cast<float2*>(ws + L.stats);
  float* xt = reinterpret_cast<float*>(ws + L.xt);
  float* lse = reinterpret_cast<float*>(ws + L.lse);
  float* row_ce = reinterpret_cast<float*>(ws + L.row_ce);
  float* row_z = reinterpret_cast<float*>(ws + L.row_z);
  float* acc = reinterpret_cast<float*>(ws + L.acc);
  const bool with_grad = grad_input || grad_weight || (flags & GH_LCE_GRADS_LATER);
  const bool fp32_accum = L.need_acc;
  // q mode is decided by the layout alone (dtype and GREYHOUND_B200_LCE_Q),
  // so the calls that continue this one from the workspace agree with it
  const bool q = L.q && with_grad;
  const bool q_dw = q && (grad_weight || (flags & (GH_LCE_KEEP_DW_OPERAND | GH_LCE_GRADS_LATER)));
  uint8_t* qmode = reinterpret_cast<uint8_t*>(ws + L.qmode);
  float* alpha = reinterpret_cast<float*>(ws + L.alpha);
  int* rowflag = reinterpret_cast<int*>(ws + L.rowflag);
  T* hs = reinterpret_cast<T*>(ws + L.hs);
  int rc = GH_OK;
  cudaMemsetAsync(status, 0, sizeof(int), st);
  const float* sp = grad_scale;
  if (with_grad && mean) {
    mean_scale_kernel<<<1, 1024, 0, st>>>(target, N, ignore, grad_scale, scale);
    count_launch(1);
    sp = scale;
  }
  const int64_t nchunks = (N + L.chunk - 1) / L.chunk;
  const int sms = num_sms_dev();
  for (int64_t c = 0; c < nchunks; ++c) {
    const int64_t s0 = c * L.chunk;
    const int64_t rows = (s0 + L.chunk <= N) ? L.chunk : N - s0;
    const T* Hc = static_cast<const T*>(H) + s0 * D;
    const int64_t* tc = target + s0;
    // 1. logits GEMM + fused CE statistics
    {
      const int pair = pick_pair(rows);
      // the q store runs on 256-column tiles only
      const int nsub = q ? 1 : pick_nsub(rows, V, pair, sms / 2, false, true);
      CUtensorMap ta, tb;
      if ((rc = make_operand_maps(&ta, &tb, dtype, Operand{Hc, D, 0}, Operand{W, D, 0}, rows, V, D, pair)))
        return rc;
      gemm::Params p{};
      set_tiles(p, rows, V, D, pair, nsub);
      p.raster = 2;
      p.group = logits_group();
      p.out = with_grad ? logits : nullptr;  // forward only: statistics, no logits
      p.ldo = L.ldl;
      p.vec_ok = ((L.ldl * (int64_t)sizeof(T)) & 15) == 0;
      p.labels = tc;
      p.a_hint = kKeepA_StreamB.a;
      p.b_hint = kKeepA_StreamB.b;
      p.out_evict_first = kKeepA_StreamB.out;
      p.stats = stats;
      p.xt = xt;
      p.status = status;
      p.qmode = qmode;
      ProfScope prof(PROF_GEMM_LOGITS_CE, st);
      if (q) rc = launch_gemm_mm<T, gemm::EPI_LCE_Q, T>(ta, tb, 0, 0, pair, nsub, p, sms, st);
      else rc = launch_gemm_mm<T, gemm::EPI_LCE, T>(ta, tb, 0, 0, pair, nsub, p, sms, st);
      if (rc) return rc;
    }
    // 2. per-row logsumexp and loss terms (q mode: also the per-row factor)
    lce_combine_kernel<<<(unsigned)((rows + 31) / 32), 32 * kCombineWarps, 0, st>>>(
        stats, L.num_n, rows, xt, tc, 0, V, ignore, lse, row_ce + s0, row_z + s0, nullptr, status,
        q ? QOut{qmode, sp, zmul, alpha, rowflag} : QOut{nullptr, nullptr, 0.f, nullptr, nullptr});
    count_launch(1);
    if ((rc = check_launch("lce_combine"))) return rc;
    if (!with_grad) continue;
    if (q) {
      // 3q. rows q mode cannot represent are rewritten (most CTAs return at
      //     once), the target column of the others gets its one-hot term,
      //     and H is scaled by alpha for the dW GEMM
      ProfScope prof(PROF_DLOGITS, st);
      lce_q_fixup_kernel<T><<<(unsigned)rows, 256, 0, st>>>(logits, L.ldl, qmode, rowflag, lse, tc, 0, rows, V, zmul);
      lce_q_target_kernel<T><<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(logits, L.ldl, tc, xt, lse, rowflag,
                                                                             alpha, rows, V, ignore, zmul);
      count_launch(2);
      if (q_dw) {
        scale_rows_kernel<T><<<4 * sms, 256, 0, st>>>(Hc, alpha, rows, D, hs);
        count_launch(1);
      }
      if ((rc = check_launch("lce_q_prep"))) return rc;
    } else {
      // 3. dlogits in place
      if ((rc = lce_dlogits<T>(logits, L.ldl, tc, lse, rows, V, zmul, ignore, sp, st))) return rc;
    }
    // 4. dW[V, D] (+)= dlogits_c^T @ H_c  (row-major [V, D] = the op's [D, V]
    //    gradient as a transposed view, so autograd can hand it to W.grad as is)
    if (grad_weight) {
      const bool first = c == 0, last = c == nchunks - 1;
      Operand A{logits, L.ldl, 1};
      Operand B{Hc, D, 1};
      void* out;
      int out_dtype;
      const float* add_f32 = nullptr;
      const void* add_same = nullptr;
      if (fp32_accum) {
        out = last ? grad_weight : (void*)acc;
        out_dtype = last ? dtype : GH_F32;
        add_f32 = first ? nullptr : acc;
      } else {
        out = grad_weight;
        out_dtype = dtype;
        add_same = first ? nullptr : grad_weight;
      }
      if (q) B = Operand{hs, D, 1};
      if ((rc = run_gemm(dtype, A, B, V, D, rows, out, out_dtype, D, add_f32, add_same, D, nullptr, 1, sms, st,
                         status, PROF_GEMM_DW, kStreamA_KeepB)))
        return rc;
    }
    // 5. dH rows [s0, s0 + rows) = dlogits_c @ W
    if (grad_input && !((flags & GH_LCE_DEFER_LAST_DH) && c == nchunks - 1)) {
      Operand A{logits, L.ldl, 0};
      Operand B{W, D, 1};
      if ((rc = run_gemm(dtype, A, B, rows, D, V, static_cast<T*>(grad_input) + s0 * D, dtype, D, nullptr, nullptr,
                         0, nullptr, 1, sms, st, status, PROF_GEMM_DH, Hints{}, ws + L.dh2, q ? alpha : nullptr)))
        return rc;
    }
  }
  ce_finalize_kernel<<<1, 1024, 0, st>>>(row_ce, row_z, target, N, ignore, ce_sum, z_sum, n_valid);
  count_launch(1);
  if ((rc = check_launch("lce_finalize"))) return rc;
  return publish_status(status, st);
}

// ---------------------------------------------------------------------------
// Vocab-parallel phases (one vocab shard of W per rank; all rows in one chunk).

template <typename T>
int shard_stats_run(const void* H, const void* W, const int64_t* target, int64_t N, int64_t D, int64_t Vs,
                    int64_t vstart, int dtype, float* stats3, const LceLayout& L, char* ws, cudaStream_t st) {
  int* status = reinterpret_cast<int*>(ws + L.status);
  T* logits = reinterpret_cast<T*>(ws + L.logits);
  float2* stats = reinterpret_cast<float2*>(ws + L.stats);
  float* xt = reinterpret_cast<float*>(ws + L.xt);
  cudaMemsetAsync(status, 0, sizeof(int), st);
  const int pair = pick_pair(N);
  const int nsub = pick_nsub(N, Vs, pair, num_sms_dev() / 2, false, true);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_operand_maps(&ta, &tb, dtype, Operand{H, D, 0}, Operand{W, D, 0}, N, Vs, D, pair))) return rc;
  gemm::Params p{};
  set_tiles(p, N, Vs, D, pair, nsub);
  p.raster = 2;
  p.group = kLogitsGroup;
  p.out = logits;
  p.ldo = L.ldl;
  p.vec_ok = ((L.ldl * (int64_t)sizeof(T)) & 15) == 0;
  p.labels = target;
  p.label_offset = vstart;
  p.a_hint = kKeepA_StreamB.a;
  p.b_hint = kKeepA_StreamB.b;
  p.out_evict_first = kKeepA_StreamB.out;
  p.stats = stats;
  p.xt = xt;
  p.status = status;
  {
    ProfScope prof(PROF_GEMM_LOGITS_CE, st);
    rc = launch_gemm_mm<T, gemm::EPI_LCE, T>(ta, tb, 0, 0, pair, nsub, p, num_sms_dev(), st);
    if (rc) return rc;
  }
  lce_combine_kernel<<<(unsigned)((N + 31) / 32), 32 * kCombineWarps, 0, st>>>(
      stats, L.num_n, N, xt, target, vstart, Vs, INT64_MIN, nullptr, nullptr, nullptr, stats3, status,
      QOut{nullptr, nullptr, 0.f, nullptr, nullptr});
  count_launch(1);
  if ((rc = check_launch("lce_shard_combine"))) return rc;
  return publish_status(status, st);
}

template <typename T>
int shard_grads_run(const void* H, const void* W, const int64_t* target, const float* lse, int64_t N, int64_t D,
                    int64_t Vs, int64_t vstart, int dtype, float zmul, int64_t ignore, const float* grad_scale,
                    void* grad_input, void* grad_weight, const LceLayout& L, char* ws, cudaStream_t st) {
  int* status = reinterpret_cast<int*>(ws + L.status);
  T* logits = reinterpret_cast<T*>(ws + L.logits);
  const int sms = num_sms_dev();
  int rc;
  if ((rc = lce_dlogits<T>(logits, L.ldl, target, lse, N, Vs, zmul, ignore, grad_scale, st, vstart, 1))) return rc;
  if (grad_weight) {
    if ((rc = run_gemm(dtype, Operand{logits, L.ldl, 1}, Operand{H, D, 1}, Vs, D, N, grad_weight, dtype, D, nullptr,
                       nullptr, 0, nullptr, 1, sms, st, status, PROF_GEMM_DW, kStreamA_KeepB)))
      return rc;
  }
  if (grad_input) {
    if ((rc = run_gemm(dtype, Operand{logits, L.ldl, 0}, Operand{W, D, 1}, N, D, Vs, grad_input, dtype, D, nullptr,
                       nullptr, 0, nullptr, 1, sms, st, status, PROF_GEMM_DH)))
      return rc;
  }
  return publish_status(status, st);
}

}  // namespace
}  // namespace gh

using namespace gh;

extern "C" size_t gh_lce_workspace_bytes(int64_t N, int64_t D, int64_t V, int64_t chunk_rows, int dtype,
                                         int fp32_grad_weight_accum) {
  if (N < 0 || D <= 0 || V <= 0 || elt_size(dtype) != 2) return 0;
  return lce_layout(N, D, V, chunk_rows, dtype, fp32_grad_weight_accum).total;
}

extern "C" size_t gh_lce_loss_workspace_bytes(int64_t N, int64_t D, int64_t V, int64_t chunk_rows, int dtype) {
  if (N < 0 || D <= 0 || V <= 0 || elt_size(dtype) != 2) return 0;
  return lce_layout(N, D, V, chunk_rows, dtype, 0, true).total;
}

extern "C" int gh_lce_fwd_bwd(const void* H, const void* W, const int64_t* target, int64_t N, int64_t D, int64_t V,
                              int dtype, float z_loss_multiplier, int64_t ignore_index, int mean_reduction,
                              const float* grad_scale, int64_t chunk_rows, int fp32_grad_weight_accum, int flags,
                              void* grad_input, void* grad_weight, float* ce_sum, float* z_sum, float* n_valid,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16)
    return set_error(GH_ETYPE, "linear cross-entropy kernels take bf16 or fp16 operands (dtype code %d)", dtype);
  if (N < 0 || D <= 0 || V <= 0) return set_error(GH_EINVAL, "bad shape N=%lld D=%lld V=%lld", (long long)N,
                                                   (long long)D, (long long)V);
  if (D % 8) return set_error(GH_EUNSUPPORTED, "hidden size must be a multiple of 8 (got %lld)", (long long)D);
  if (!H || !W || !target || !ce_sum || !z_sum || !n_valid || !workspace)
    return set_error(GH_EINVAL, "null pointer argument");
  const bool later = flags & GH_LCE_GRADS_LATER;
  const bool loss_only = !grad_input && !grad_weight && !later;
  if (later && (grad_input || grad_weight))
    return set_error(GH_EINVAL, "GH_LCE_GRADS_LATER takes no gradient buffers");
  LceLayout L = lce_layout(N, D, V, chunk_rows, dtype, fp32_grad_weight_accum, loss_only);
  if (later && N > L.chunk)
    return set_error(GH_EUNSUPPORTED, "GH_LCE_GRADS_LATER needs all rows in one chunk");
  if (workspace_bytes < L.total)
    return set_error(GH_EWORKSPACE, "workspace too small: %zu < %zu", workspace_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  if (N == 0) {
    ce_finalize_kernel<<<1, 1024, 0, st>>>(nullptr, nullptr, target, 0, ignore_index, ce_sum, z_sum, n_valid);
    count_launch(1);
    return check_launch("lce_finalize");
  }
  if (dtype == GH_BF16)
    return lce_run<__nv_bfloat16>(H, W, target, N, D, V, dtype, z_loss_multiplier, ignore_index, mean_reduction,
                                  grad_scale, L, flags, grad_input, grad_weight, ce_sum, z_sum, n_valid, ws, st);
  return lce_run<__half>(H, W, target, N, D, V, dtype, z_loss_multiplier, ignore_index, mean_reduction, grad_scale,
                         L, flags, grad_input, grad_weight, ce_sum, z_sum, n_valid, ws, st);
}

extern "C" int gh_lce_dh_last_chunk(const void* W, int64_t N, int64_t D, int64_t V, int dtype, int64_t chunk_rows,
                                    int fp32_grad_weight_accum, int64_t row_begin, int64_t row_end,
                                    const float* scale, void* grad_input, void* workspace, size_t workspace_bytes,
                                    int max_ctas, void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "bf16 or fp16 expected");
  if (N <= 0) return GH_OK;
  if (!W || !grad_input || !workspace) return set_error(GH_EINVAL, "null pointer argument");
  LceLayout L = lce_layout(N, D, V, chunk_rows, dtype, fp32_grad_weight_accum);
  if (workspace_bytes < L.total) return set_error(GH_EWORKSPACE, "workspace too small");
  char* ws = static_cast<char*>(workspace);
  const int64_t nchunks = (N + L.chunk - 1) / L.chunk;
  const int64_t s0 = (nchunks - 1) * L.chunk;
  const int64_t rows = N - s0;
  if (row_end < 0 || row_end > rows) row_end = rows;
  if (row_begin < 0) row_begin = 0;
  if (row_begin >= row_end) return GH_OK;
  const int elt = elt_size(dtype);
  Operand A{ws + L.logits + (size_t)row_begin * L.ldl * elt, L.ldl, 0};
  Operand B{W, D, 1};
  // the q-mode decision gh_lce_fwd_bwd made for this workspace: the rows'
  // factor alpha then multiplies the product
  const bool q = L.q;
  // each row range has its own rows of the split-K partial buffer, so the two
  // ranges may run concurrently
  int* status = reinterpret_cast<int*>(ws + L.status);
  const int rc = run_gemm(dtype, A, B, row_end - row_begin, D, V,
                          static_cast<char*>(grad_input) + (s0 + row_begin) * D * elt, dtype, D, nullptr, nullptr, 0,
                          scale, 1, max_ctas, static_cast<cudaStream_t>(stream), status, PROF_GEMM_DH, Hints{},
                          ws + L.dh2 + (size_t)row_begin * D * elt,
                          q ? reinterpret_cast<const float*>(ws + L.alpha) + row_begin : nullptr);
  return rc ? rc : publish_status(status, static_cast<cudaStream_t>(stream));
}

extern "C" int gh_lce_dw_peers(const void* H, int64_t N, int64_t D, int64_t V, int dtype, int64_t chunk_rows,
                               int fp32_grad_weight_accum, const float* scale, void* const* band_out, int nbands,
                               int64_t band_rows, int first_band, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "bf16 or fp16 expected");
  if (N < 0 || D <= 0 || V <= 0) return set_error(GH_EINVAL, "bad shape");
  if (!H || !band_out || !workspace) return set_error(GH_EINVAL, "null pointer argument");
  if (nbands <= 0 || nbands > gemm::kMaxPeers || band_rows <= 0 || band_rows % (2 * BM) ||
      (int64_t)nbands * band_rows < V)
    return set_error(GH_EINVAL, "need 1..%d bands of a multiple of %d rows covering the vocabulary",
                     gemm::kMaxPeers, 2 * BM);
  LceLayout L = lce_layout(N, D, V, chunk_rows, dtype, fp32_grad_weight_accum);
  if (workspace_bytes < L.total) return set_error(GH_EWORKSPACE, "workspace too small");
  if (N > L.chunk) return set_error(GH_EUNSUPPORTED, "band-stored weight gradient needs all rows in one chunk");
  if (N == 0) return GH_OK;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  PeerOut po;
  po.n = nbands;
  po.rows = band_rows;
  po.first = first_band >= 0 && first_band < nbands ? first_band : 0;
  for (int i = 0; i < nbands; ++i) po.ptr[i] = band_out[i];
  // q mode: gh_lce_fwd_bwd(..., GH_LCE_KEEP_DW_OPERAND or GH_LCE_GRADS_LATER)
  // left alpha * H in the workspace
  Operand A{ws + L.logits, L.ldl, 1};
  Operand B = L.q ? Operand{ws + L.hs, D, 1} : Operand{H, D, 1};
  int* status = reinterpret_cast<int*>(ws + L.status);
  const int rc = run_gemm(dtype, A, B, V, D, N, nullptr, dtype, D, nullptr, nullptr, 0, scale, 1, num_sms_dev(), st,
                          status, PROF_GEMM_DW, kStreamA_KeepB, nullptr, nullptr, &po);
  return rc ? rc : publish_status(status, st);
}

extern "C" int gh_gemm(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major,
                       int64_t M, int64_t N, int64_t K, int dtype, void* out, int64_t ldo, int out_dtype,
                       const void* addend, int64_t ld_add, const float* scale, int* status, void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "GEMM operands must be bf16 or fp16");
  if (M < 0 || N < 0 || K <= 0) return set_error(GH_EINVAL, "bad GEMM shape");
  Operand a{A, lda, a_mn_major ? 1 : 0};
  Operand b{B, ldb, b_mn_major ? 1 : 0};
  const float* add_f32 = out_dtype == GH_F32 ? static_cast<const float*>(addend) : nullptr;
  const void* add_same = out_dtype == GH_F32 ? nullptr : addend;
  const int raster = M >= N ? 1 : 0;
  const int rc = run_gemm(dtype, a, b, M, N, K, out, out_dtype, ldo, add_f32, add_same, ld_add, scale, raster, 0,
                          static_cast<cudaStream_t>(stream), status);
  return rc ? rc : publish_status(status, static_cast<cudaStream_t>(stream));
}

extern "C" size_t gh_lce_shard_workspace_bytes(int64_t N, int64_t D, int64_t V_shard, int dtype) {
  if (N < 0 || D <= 0 || V_shard <= 0 || elt_size(dtype) != 2) return 0;
  return lce_layout(N, D, V_shard, N, dtype, 0).total;
}

extern "C" int gh_lce_shard_stats(const void* H, const void* W_shard, const int64_t* target, int64_t N, int64_t D,
                                  int64_t V_shard, int64_t vocab_start, int dtype, float* stats3, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "bf16 or fp16 expected (dtype code %d)", dtype);
  if (N < 0 || D <= 0 || V_shard <= 0) return set_error(GH_EINVAL, "bad shape");
  if (D % 8) return set_error(GH_EUNSUPPORTED, "hidden size must be a multiple of 8");
  if (N == 0) return GH_OK;
  if (!H || !W_shard || !target || !stats3 || !workspace) return set_error(GH_EINVAL, "null pointer argument");
  LceLayout L = lce_layout(N, D, V_shard, N, dtype, 0);
  if (workspace_bytes < L.total) return set_error(GH_EWORKSPACE, "workspace too small: %zu < %zu", workspace_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  if (dtype == GH_BF16)
    return shard_stats_run<__nv_bfloat16>(H, W_shard, target, N, D, V_shard, vocab_start, dtype, stats3, L, ws, st);
  return shard_stats_run<__half>(H, W_shard, target, N, D, V_shard, vocab_start, dtype, stats3, L, ws, st);
}

extern "C" int gh_lce_shard_grads(const void* H, const void* W_shard, const int64_t* target, const float* lse,
                                  int64_t N, int64_t D, int64_t V_shard, int64_t vocab_start, int dtype,
                                  float z_loss_multiplier, int64_t ignore_index, const float* grad_scale,
                                  void* grad_input_partial, void* grad_weight_shard, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "bf16 or fp16 expected (dtype code %d)", dtype);
  if (N < 0 || D <= 0 || V_shard <= 0) return set_error(GH_EINVAL, "bad shape");
  if (N == 0) return GH_OK;
  if (!H || !W_shard || !target || !lse || !workspace) return set_error(GH_EINVAL, "null pointer argument");
  LceLayout L = lce_layout(N, D, V_shard, N, dtype, 0);
  if (workspace_bytes < L.total) return set_error(GH_EWORKSPACE, "workspace too small: %zu < %zu", workspace_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  if (dtype == GH_BF16)
    return shard_grads_run<__nv_bfloat16>(H, W_shard, target, lse, N, D, V_shard, vocab_start, dtype,
                                          z_loss_multiplier, ignore_index, grad_scale, grad_input_partial,
                                          grad_weight_shard, L, ws, st);
  return shard_grads_run<__half>(H, W_shard, target, lse, N, D, V_shard, vocab_start, dtype, z_loss_multiplier,
                                 ignore_index, grad_scale, grad_input_partial, grad_weight_shard, L, ws, st);
}

extern "C" int gh_lce_shard_dw(const void* H, int64_t N, int64_t D, int64_t V_shard, int dtype,
                               void* grad_weight_shard, void* workspace, size_t workspace_bytes, int max_ctas,
                               void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "bf16 or fp16 expected (dtype code %d)", dtype);
  if (N < 0 || D <= 0 || V_shard <= 0) return set_error(GH_EINVAL, "bad shape");
  if (N == 0) return GH_OK;
  if (!H || !grad_weight_shard || !workspace) return set_error(GH_EINVAL, "null pointer argument");
  LceLayout L = lce_layout(N, D, V_shard, N, dtype, 0);
  if (workspace_bytes < L.total) return set_error(GH_EWORKSPACE, "workspace too small: %zu < %zu", workspace_bytes, L.total);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + L.status);
  const int rc = run_gemm(dtype, Operand{ws + L.logits, L.ldl, 1}, Operand{H, D, 1}, V_shard, D, N, grad_weight_shard,
                          dtype, D, nullptr, nullptr, 0, nullptr, 1, max_ctas, static_cast<cudaStream_t>(stream),
                          status, PROF_GEMM_DW, kStreamA_KeepB);
  return rc ? rc : publish_status(status, static_cast<cudaStream_t>(stream));
}

extern "C" int gh_gemm_selftest_stall(void* scratch, size_t scratch_bytes, int* status, int wait_ms, void* stream) {
  if (!scratch || !status || scratch_bytes < (size_t)(128 * 64 + 256 * 64 + 128 * 256) * 2)
    return set_error(GH_EINVAL, "gh_gemm_selftest_stall: scratch of at least 112 KB and a status word are required");
  if ((reinterpret_cast<uintptr_t>(scratch) & 15)) return set_error(GH_EINVAL, "scratch must be 16-byte aligned");
  if (wait_ms <= 0 || wait_ms > 10000) return set_error(GH_EINVAL, "wait_ms must be in (0, 10000]");
  char* base = static_cast<char*>(scratch);
  CUtensorMap ta, tb;
  int rc = make_operand_maps(&ta, &tb, GH_BF16, Operand{base, 64, 0}, Operand{base + 128 * 64 * 2, 64, 0}, 128, 256,
                             64, 1);
  if (rc) return rc;
  gemm::Params p{};
  set_tiles(p, 128, 256, 64, 1);
  p.raster = 0;
  p.group = 1;
  p.out = base + (128 * 64 + 256 * 64) * 2;
  p.ldo = 256;
  p.vec_ok = 1;
  p.status = status;
  p.wait_limit_ns = (uint64_t)wait_ms * 1000000ull;
  p.debug_no_loads = 1;
  rc = launch_gemm_t<__nv_bfloat16, 0, 0, gemm::EPI_STORE, __nv_bfloat16, 1>(ta, tb, p, 1,
                                                                           static_cast<cudaStream_t>(stream));
  return rc ? rc : publish_status(status, static_cast<cudaStream_t>(stream));
}
