// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M, N] = sum_k A[m, k] * B[n, k]     (bf16 / fp16 operands, fp32 accumulate in TMEM)
//
// A and B are each either K-major (k contiguous: X[r * ld + k]) or MN-major
// (m/n contiguous: X[k * ld + r]); this covers the three GEMMs of the linear
// cross-entropy:
//   logits  = H @ W^T        A = H [C, D] K-major,        B = W [V, D] K-major
//   dH      = dlogits @ W    A = dlogits [C, V] K-major,  B = W [V, D] MN-major
//   dW      = dlogits^T @ H  A = dlogits [C, V] MN-major, B = H [C, D] MN-major
//
// CTA: 256 threads, one CTA per SM, persistent over output tiles of
// 128 x 256 (static round-robin over a rasterised tile order).
//   warp 0      TMA producer: 4-stage ring of (A 128x64, B 256x64) tiles,
//               128-byte swizzle, completion on mbarriers
//   warp 1      MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=16) per stage,
//               tcgen05.commit frees the smem stage / publishes the tile
//   warp 2      TMEM allocator (512 columns = two 128x256 fp32 accumulators)
//   warps 4-7   epilogue: tcgen05.ld (32 lanes x 32 columns) -> registers ->
//               fused epilogue -> global; double-buffered TMEM lets the
//               epilogue of tile i overlap the MMAs of tile i+1
// Epilogues: plain store (optional scale and fp32 / same-type addend), or the
// linear-CE epilogue (bf16 logits + per-(row, 256-column tile) max / sum-exp
// + target logit), which replaces the reference's separate CE row pass
// (src/greyhound/kernels/cross_entropy.py:20-108) for the logits tile.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "tc_primitives.cuh"

namespace gh {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;           // 64 x 2 B = one 128-byte swizzle row
constexpr int THREADS = 256;
constexpr int TMEM_COLS = 2 * BN;

enum Epi { EPI_STORE = 0, EPI_LCE = 1 };

struct Params {
  int M, N, K;
  int num_m, num_n, num_tiles;   // num_m counts tiles of Geo<PAIR>::TM rows
  int raster;           // 0: m-tile fastest, 1: n-tile fastest,
                        // 2: groups of `group` m-tiles (m fastest inside), 3: same for n
  int group;
  // EPI_STORE
  void* out;
  int64_t ldo;
  int vec_ok;           // 16-byte aligned rows (vector stores allowed)
  const float* add_f32; // optional fp32 addend [M, ldadd]
  const void* add_same; // optional addend in the output type [M, ldadd]
  int64_t ldadd;
  const float* scale;   // optional device scalar multiplying the product
  // EPI_LCE (out == nullptr: statistics only, no logits written)
  const int64_t* labels;  // [M] (chunk rows), compared against the column index
  int64_t label_offset;   // first vocab id of this GEMM's columns (vocab shards)
  float2* stats;          // [num_n][M] (max, sum-exp) in log2 units
  float* xt;              // [M] target logit (written by the tile holding it)
  int* status;            // device error word (bit 2: pipeline timeout)
  // L2 policy of each operand's TMA loads (0 none, 1 evict_first, 2 evict_last)
  // and of the epilogue stores (1: evict_first for a large streamed output)
  int a_hint, b_hint, out_evict_first;
  // Pipeline wait limit (0: 10 s). Self-test only: debug_no_loads makes the
  // producer issue nothing, so the waits run out and the kernel must return
  // with status bit 4 instead of hanging.
  uint64_t wait_limit_ns;
  int debug_no_loads;
};

// Tile order. The grouped orders bound how much of the re-read operand is live
// at once (a group of m-tiles shares one pass over all n-tiles), so it stays
// in L2 instead of being fetched from DRAM once per band.
__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& mt, int& nt) {
  if (p.raster == 0) {
    mt = tile % p.num_m;
    nt = tile / p.num_m;
  } else if (p.raster == 1) {
    nt = tile % p.num_n;
    mt = tile / p.num_n;
  } else if (p.raster == 2) {
    const int per = p.group * p.num_n;
    const int g = tile / per, r = tile % per;
    const int rem = p.num_m - g * p.group;
    const int gm = rem < p.group ? rem : p.group;
    mt = g * p.group + r % gm;
    nt = r / gm;
  } else {
    const int per = p.group * p.num_m;
    const int g = tile / per, r = tile % per;
    const int rem = p.num_n - g * p.group;
    const int gn = rem < p.group ? rem : p.group;
    nt = g * p.group + r % gn;
    mt = r / gn;
  }
}

template <typename T> struct AbType;
template <> struct AbType<__nv_bfloat16> { static constexpr int v = 1; };
template <> struct AbType<__half> { static constexpr int v = 0; };

// Store 32 consecutive fp32 values of one output row as OutT.
template <typename OutT>
__device__ __forceinline__ void store_row32(OutT* dst, int col0, int N, const float (&v)[32], bool vec_ok,
                                            bool evict_first = false) {
  constexpr int PER = 16 / sizeof(OutT);
  if (vec_ok && col0 + 32 <= N) {
#pragma unroll
    for (int q = 0; q < 32 / PER; ++q) {
      Vec16<OutT> o;
      float f[PER];
#pragma unroll
      for (int k = 0; k < PER; ++k) f[k] = v[q * PER + k];
      o.from_float(f);
      if (evict_first) st16_cs(dst + col0 + q * PER, o.raw);
      else st16(dst + col0 + q * PER, o.raw);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) dst[col0 + j] = Elt<OutT>::from_f(v[j]);
  }
}

template <typename OutT>
__device__ __forceinline__ void load_row32(const OutT* src, int col0, int N, float (&v)[32], bool vec_ok) {
  constexpr int PER = 16 / sizeof(OutT);
  if (vec_ok && col0 + 32 <= N) {
#pragma unroll
    for (int q = 0; q < 32 / PER; ++q) {
      Vec16<OutT> r;
      r.raw = *reinterpret_cast<const uint4*>(src + col0 + q * PER);
      float f[PER];
      r.to_float(f);
#pragma unroll
      for (int k = 0; k < PER; ++k) v[q * PER + k] = f[k];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = col0 + j < N ? Elt<OutT>::to_f(src[col0 + j]) : 0.f;
  }
}

// Geometry of one configuration. PAIR = 1: one CTA computes a 128 x 256 tile.
// PAIR = 2: a 2-CTA cluster computes a 256 x 256 tile with tcgen05.mma
// cta_group::2; each CTA stages its 128 rows of A and 128 of the 256 B rows,
// and holds its 128 accumulator rows in its own TMEM.
template <int PAIR>
struct Geo {
  static constexpr int TM = BM * PAIR;            // tile rows
  static constexpr int B_ROWS = BN / PAIR;        // B rows staged per CTA
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STG = PAIR == 2 ? 6 : 4;   // pipeline depth
  static constexpr int SMEM = STG * (A_BYTES + B_BYTES) + 1024 + 256;
};

template <typename T, int A_MN, int B_MN, int EPI, typename OutT, int PAIR>
__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  using G = Geo<PAIR>;
  constexpr int STG = G::STG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STG * G::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STG * G::B_BYTES);
  uint64_t* empty = full + STG;
  uint64_t* tfull = empty + STG;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR == 2 ? tc::cluster_ctarank() : 0;
  const int unit = blockIdx.x / PAIR;         // cluster index
  const int nunits = gridDim.x / PAIR;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 4 * PAIR);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::tma_prefetch_desc(&tmA);
    tc::tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    if (PAIR == 2) tc::tmem_alloc_pair(tmem_holder, TMEM_COLS);
    else tc::tmem_alloc(tmem_holder, TMEM_COLS);
  }
  __syncthreads();
  if (PAIR == 2) tc::cluster_sync();  // peer barriers initialised before any remote arrive
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int nkb = (p.K + BK - 1) / BK;
  const uint64_t lim = p.wait_limit_ns ? p.wait_limit_ns : 10000000000ull;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs of a pair) ----------------
      const uint64_t pol_a = tc::l2_policy(p.a_hint), pol_b = tc::l2_policy(p.b_hint);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = p.debug_no_loads ? p.num_tiles : unit; tile < p.num_tiles; tile += nunits) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        const int ma = mt * G::TM + (int)rank * BM;         // this CTA's A rows
        const int nb = nt * BN + (int)rank * G::B_ROWS;     // this CTA's B rows
        for (int kb = 0; kb < nkb; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, abort_flag, lim)) goto producer_done;
          uint8_t* a = sA + stage * G::A_BYTES;
          uint8_t* b = sB + stage * G::B_BYTES;
          const int k0 = kb * BK;
          if (PAIR == 1) {
            tc::mbar_arrive_expect_tx(&full[stage], G::A_BYTES + G::B_BYTES);
            if (A_MN) {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) tc::tma_load_2d_hint(a + j * (BK * 128), &tmA, &full[stage], ma + j * 64, k0, pol_a);
            } else {
              tc::tma_load_2d_hint(a, &tmA, &full[stage], k0, ma, pol_a);
            }
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < G::B_ROWS / 64; ++j)
                tc::tma_load_2d_hint(b + j * (BK * 128), &tmB, &full[stage], nb + j * 64, k0, pol_b);
            } else {
              tc::tma_load_2d_hint(b, &tmB, &full[stage], k0, nb, pol_b);
            }
          } else {
            // both CTAs' copies complete on the leader's full barrier
            if (rank == 0) tc::mbar_arrive_expect_tx(&full[stage], 2 * (G::A_BYTES + G::B_BYTES));
            const uint32_t fb = tc::mapa_shared(tc::smem_u32(&full[stage]), 0);
            if (A_MN) {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) tc::tma_load_2d_pair_hint(a + j * (BK * 128), &tmA, fb, ma + j * 64, k0, pol_a);
            } else {
              tc::tma_load_2d_pair_hint(a, &tmA, fb, k0, ma, pol_a);
            }
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < G::B_ROWS / 64; ++j)
                tc::tma_load_2d_pair_hint(b + j * (BK * 128), &tmB, fb, nb + j * 64, k0, pol_b);
            } else {
              tc::tma_load_2d_pair_hint(b, &tmB, fb, k0, nb, pol_b);
            }
          }
          if (++stage == STG) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (pair leader) ----------------
      constexpr uint32_t idesc = tc::instr_desc_f16(AbType<T>::v, A_MN, B_MN, G::TM, BN);
      // K-major: 8-row groups of 128 B rows at 1024 B; K step of 16 = +32 B.
      // MN-major: 64-element column blocks at BK*128 B (LBO); K groups of 8
      // rows at 1024 B (SBO); K step of 16 = +2048 B.
      constexpr uint32_t a_lbo = A_MN ? BK * 128 : 16, a_sbo = 1024;
      constexpr uint32_t b_lbo = B_MN ? BK * 128 : 16, b_sbo = 1024;
      constexpr uint32_t a_kstep = A_MN ? 2048 : 32, b_kstep = B_MN ? 2048 : 32;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = unit; tile < p.num_tiles; tile += nunits) {
        if (!tc::mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, lim)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, abort_flag, lim)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t a0 = tc::smem_u32(sA + stage * G::A_BYTES);
          const uint32_t b0 = tc::smem_u32(sB + stage * G::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = tc::smem_desc_sw128(a0 + k * a_kstep, a_lbo, a_sbo);
            const uint64_t bd = tc::smem_desc_sw128(b0 + k * b_kstep, b_lbo, b_sbo);
            if (PAIR == 2) tc::mma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else tc::mma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          if (PAIR == 2) tc::mma_commit_pair_mc(&empty[stage], 0x3);
          else tc::mma_commit(&empty[stage]);
          if (++stage == STG) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (PAIR == 2) tc::mma_commit_pair_mc(&tfull[acc], 0x3);
        else tc::mma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue ----------------
    const int q = warp - 4;  // TMEM lane quarter this warp may access
    const uint32_t tempty_leader0 = tc::mapa_shared(tc::smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = tc::mapa_shared(tc::smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = unit; tile < p.num_tiles; tile += nunits) {
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int m0 = mt * G::TM + (int)rank * BM, n0 = nt * BN;
      if (!tc::mbar_wait(&tfull[acc], acc_phase, abort_flag, lim)) break;
      tc::tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (EPI == EPI_LCE) {
        const int64_t lab = row_ok ? p.labels[row] - p.label_offset : -1;
        const int64_t lab_rel = lab - n0;  // label column inside this tile, if any
        float m_run = kNegInf, s_run = 0.f;
        OutT* orow = reinterpret_cast<OutT*>(p.out) + (int64_t)row * p.ldo;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tc::tmem_ld32(tbase + c * 32, r);
          tc::tmem_ld_wait();
          float x[32];
          float cm = kNegInf;
          const int col0 = n0 + c * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            // the logits tensor holds the product rounded to the input dtype
            // (as the reference's cuBLAS output); statistics use those values
            x[j] = Elt<OutT>::to_f(Elt<OutT>::from_f(__uint_as_float(r[j])));
            if (col0 + j < p.N) cm = fmaxf(cm, x[j]);
            if ((int64_t)(c * 32 + j) == lab_rel) p.xt[row] = x[j];
          }
          const float cm2 = cm * kLog2e;
          const float mnew = fmaxf(m_run, cm2);
          float acc_s = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.N) acc_s += fast_exp2(fmaf(x[j], kLog2e, -mnew));
          s_run = (m_run == kNegInf ? 0.f : s_run * fast_exp2(m_run - mnew)) + acc_s;
          m_run = mnew;
          if (row_ok && p.out) store_row32<OutT>(orow, col0, p.N, x, p.vec_ok, p.out_evict_first);
        }
        if (row_ok) p.stats[(int64_t)nt * p.M + row] = make_float2(m_run, s_run);
      } else {
        const float scale = p.scale ? *p.scale : 1.f;
        OutT* orow = reinterpret_cast<OutT*>(p.out) + (int64_t)row * p.ldo;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tc::tmem_ld32(tbase + c * 32, r);
          tc::tmem_ld_wait();
          const int col0 = n0 + c * 32;
          if (row_ok && col0 < p.N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * scale;
            if (p.add_f32) {
              float a[32];
              load_row32<float>(p.add_f32 + (int64_t)row * p.ldadd, col0, p.N, a, p.vec_ok);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += a[j];
            } else if (p.add_same) {
              float a[32];
              load_row32<OutT>(reinterpret_cast<const OutT*>(p.add_same) + (int64_t)row * p.ldadd, col0, p.N, a,
                               p.vec_ok);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += a[j];
            }
            store_row32<OutT>(orow, col0, p.N, v, p.vec_ok, p.out_evict_first);
          }
        }
      }
      // release this accumulator buffer to the (leader's) MMA warp
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR == 2) tc::mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        else tc::mbar_arrive(&tempty[acc]);
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }
  __syncthreads();
  if (PAIR == 2) tc::cluster_sync();  // no CTA leaves while its peer may still signal it
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicOr(p.status, 4);
  if (warp == 2) {
    tc::tc_fence_after();
    if (PAIR == 2) tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace gh
