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
// CTA: 320 threads, one CTA per SM, persistent over output tiles of
// 128 x 256 (static round-robin over a rasterised tile order); CTA pairs
// (cta_group::2) share 256 x 256 or 256 x 512 tiles (see Geo below).
//   warp 0      TMA producer: ring of (A 128x64, B 256x64) stages,
//               128-byte swizzle, completion on mbarriers
//   warp 1      MMA issuer: 4 x tcgen05.mma (K=16) per stage and accumulator,
//               tcgen05.commit frees the smem stage / publishes the tile
//   warps 2-9   epilogue: tcgen05.ld (32 lanes x 32 columns) -> registers ->
//               fused epilogue -> global (stores staged through shared
//               memory so each instruction writes whole row segments);
//               double-buffered TMEM lets the epilogue of tile i overlap the
//               MMAs of tile i+1. Warp 2 also allocates TMEM (512 columns =
//               two 128x256 fp32 accumulators, or the two halves of one
//               128x512 accumulator).
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
constexpr int THREADS = 320;     // warp 0 producer, 1 MMA, 2-9 epilogue (warp 2 also owns TMEM)
constexpr int EPI_WARP0 = 2;
constexpr int EPI_WARPS = 8;
constexpr int EPI_CHUNKS = BN / 32 / (EPI_WARPS / 4);  // 32-column chunks per warp per half
constexpr int TMEM_COLS = 2 * BN;

enum Epi { EPI_STORE = 0, EPI_LCE = 1, EPI_LCE_Q = 2 };
constexpr int kMaxPeers = 8;

// Exponent window of the unnormalised-probability store (EPI_LCE_Q), in log2
// units: a row group whose largest logit x satisfies
// kQLo <= x * log2(e) <= kQHi stores q = 2^(x log2 e) = e^x (at most 2^80,
// so sums over the vocabulary and the dH accumulator stay far inside fp32,
// and the largest term is far above bf16's smallest normal). Other groups
// store the raw logits and are rewritten by a fix-up pass once the row's
// logsumexp is known.
constexpr float kQHi = 80.f;
constexpr float kQLo = -80.f;

struct Params {
  int M, N, K;
  int num_m, num_n, num_tiles;   // num_m counts tiles of Geo<PAIR>::TM rows
  int raster;           // 0: m-tile fastest, 1: n-tile fastest,
                        // 2: groups of `group` m-tiles (m fastest inside), 3: same for n
  int group;
  // EPI_STORE
  void* out;
  int64_t ldo;
  // split-K (EPI_STORE): ksplit slices of K per output tile (0 or 1: none);
  // slice 0 writes `out`, slice 1 writes `out2` (same pitch), the host sums
  int ksplit;
  void* out2;
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
  // EPI_LCE_Q: per (256-column tile, 128-column group, row) byte, 1 when
  // that group of the row holds raw logits instead of q ([num_n][2][M])
  uint8_t* qmode;
  // EPI_STORE: optional per-row factor multiplying the product ([M] fp32)
  const float* row_scale;
  // EPI_STORE, 16-bit output: when npeer > 0 the output rows are split into
  // bands of peer_rows rows (a multiple of the tile height) and band b is
  // stored at peer_out[b] (row r at peer_out[b] + (r - b * peer_rows) * ldo),
  // which may be another GPU's memory: the GEMM's tiles go straight to the
  // rank that reduces that band (a reduce-scatter fused into the epilogue).
  int npeer;
  // tile order rotated by this many tiles (band-store GEMMs start on their
  // own rank's band, so the ranks do not all write to one owner at a time)
  int tile_rot;
  int64_t peer_rows;
  void* peer_out[kMaxPeers];
  // L2 policy of each operand's TMA loads (0 none, 1 evict_first, 2 evict_last)
  // and of the epilogue stores (1: evict_first for a large streamed output)
  int a_hint, b_hint, out_evict_first;
  // Pipeline wait limit (0: 10 s). Self-test only: debug_no_loads makes the
  // producer issue nothing, so the waits run out and the kernel must return
  // with status bit 4 instead of hanging.
  uint64_t wait_limit_ns;
  int debug_no_loads;
};

// Output base of the tile whose first row is m0: the band owner's buffer,
// offset so that indexing it with the global row lands in that band.
template <typename OutT>
__device__ __forceinline__ OutT* tile_out_base(const Params& p, void* pout, int m0) {
  if (p.npeer <= 0) return reinterpret_cast<OutT*>(pout);
  int b = (int)(m0 / p.peer_rows);
  if (b >= p.npeer) b = p.npeer - 1;
  return reinterpret_cast<OutT*>(p.peer_out[b]) - (int64_t)b * p.peer_rows * p.ldo;
}

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

// One work unit: output tile (mt, nt) and its K slice [kb0, kb1) of 64-wide
// k-steps. Split-K units of slice ks follow all units of slice ks - 1.
struct TileK {
  int mt, nt, ks, kb0, kb1;
};
__device__ __forceinline__ TileK tile_k(const Params& p, int tile, int nkb) {
  TileK t;
  const int nsplit = p.ksplit > 1 ? p.ksplit : 1;
  const int per_slice = p.num_m * p.num_n;
  if (p.tile_rot) tile = (tile + p.tile_rot) % p.num_tiles;
  t.ks = nsplit > 1 ? tile / per_slice : 0;
  tile_coords(p, tile - t.ks * per_slice, t.mt, t.nt);
  const int per = (nkb + nsplit - 1) / nsplit;
  t.kb0 = t.ks * per;
  t.kb1 = t.kb0 + per < nkb ? t.kb0 + per : nkb;
  return t;
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

// Store one warp's 32 rows x 32 columns (lane = row, v = that row's values)
// through a 2 KB shared-memory transpose, so each global store instruction
// writes 8 rows x 64 contiguous bytes instead of 32 rows x 16 bytes. The 16-byte
// pieces of a row are XOR-swizzled by (row >> 1) & 3, which keeps both the
// row-wise writes and the column-wise reads free of bank conflicts. Ragged
// column edges and unaligned outputs take the per-row path.
template <typename OutT>
__device__ __forceinline__ void store_chunk(OutT* out, int64_t ldo, int row0, int M, int col0, int N,
                                            const float (&v)[32], uint8_t* buf, int lane, bool vec_ok,
                                            bool evict_first) {
  constexpr int PER = 16 / sizeof(OutT);  // elements per 16-byte piece
  constexpr int PASSES = 32 / PER / 4;    // 4 pieces (64 B) per row per pass
  if (!vec_ok || col0 + 32 > N) {
    if (row0 + lane < M) store_row32<OutT>(out + (int64_t)(row0 + lane) * ldo, col0, N, v, vec_ok, evict_first);
    return;
  }
#pragma unroll
  for (int pass = 0; pass < PASSES; ++pass) {
#pragma unroll
    for (int pc = 0; pc < 4; ++pc) {
      Vec16<OutT> o;
      float f[PER];
#pragma unroll
      for (int k = 0; k < PER; ++k) f[k] = v[(pass * 4 + pc) * PER + k];
      o.from_float(f);
      *reinterpret_cast<uint4*>(buf + lane * 64 + 16 * (pc ^ ((lane >> 1) & 3))) = o.raw;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = j * 8 + (lane >> 2), pc = lane & 3;
      const uint4 w = *reinterpret_cast<const uint4*>(buf + r * 64 + 16 * (pc ^ ((r >> 1) & 3)));
      if (row0 + r < M) {
        OutT* dst = out + (int64_t)(row0 + r) * ldo + col0 + (pass * 4 + pc) * PER;
        if (evict_first) st16_cs(dst, w);
        else st16(dst, w);
      }
    }
    __syncwarp();
  }
}

// Two values rounded to a 16-bit type and packed into one word (first value
// in the low half), and the inverse.
template <typename OutT> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
template <typename OutT> __device__ __forceinline__ void unpack2(uint32_t w, float& a, float& b);
template <> __device__ __forceinline__ void unpack2<__nv_bfloat16>(uint32_t w, float& a, float& b) {
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xffff0000u);
}
template <> __device__ __forceinline__ void unpack2<__half>(uint32_t w, float& a, float& b) {
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tcvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(a), "=f"(b)
      : "r"(w));
}

// store_chunk for 32 already-packed 16-bit values per row (w: 16 words).
template <typename OutT>
__device__ __forceinline__ void store_chunk_packed(OutT* out, int64_t ldo, int row0, int M, int col0, int N,
                                                   const uint32_t* w, uint8_t* buf, int lane, bool vec_ok,
                                                   bool evict_first) {
  static_assert(sizeof(OutT) == 2, "packed stores are for 16-bit outputs");
  if (!vec_ok || col0 + 32 > N) {
    if (row0 + lane < M) {
      unsigned short* dst = reinterpret_cast<unsigned short*>(out + (int64_t)(row0 + lane) * ldo + col0);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (col0 + 2 * j < N) dst[2 * j] = (unsigned short)(w[j] & 0xffffu);
        if (col0 + 2 * j + 1 < N) dst[2 * j + 1] = (unsigned short)(w[j] >> 16);
      }
    }
    return;
  }
#pragma unroll
  for (int pc = 0; pc < 4; ++pc)
    *reinterpret_cast<uint4*>(buf + lane * 64 + 16 * (pc ^ ((lane >> 1) & 3))) =
        make_uint4(w[4 * pc], w[4 * pc + 1], w[4 * pc + 2], w[4 * pc + 3]);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = j * 8 + (lane >> 2), pc = lane & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(buf + r * 64 + 16 * (pc ^ ((r >> 1) & 3)));
    if (row0 + r < M) {
      OutT* dst = out + (int64_t)(row0 + r) * ldo + col0 + pc * 8;
      if (evict_first) st16_cs(dst, v);
      else st16(dst, v);
    }
  }
  __syncwarp();
}

// Fold 16 logits starting at column cs into the running (max, sum-exp) pair
// in log2 units. `full`: all 16 columns are < N (the common case: no
// per-element predicates).
__device__ __forceinline__ void lce_fold16(const float (&x)[16], bool full, int cs, int N, float& m_run, float& s_run) {
  float cm;
  if (full) {
    float t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = fmaxf(x[2 * j], x[2 * j + 1]);
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = fmaxf(t[2 * j], t[2 * j + 1]);
    cm = fmaxf(fmaxf(t[0], t[1]), fmaxf(t[2], t[3]));
  } else {
    cm = kNegInf;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (cs + j < N) cm = fmaxf(cm, x[j]);
  }
  const float mnew = fmaxf(m_run, cm * kLog2e);
  float a0 = 0.f, a1 = 0.f;
  if (full) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      a0 += fast_exp2(fmaf(x[j], kLog2e, -mnew));
      a1 += fast_exp2(fmaf(x[j + 1], kLog2e, -mnew));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (cs + j < N) a0 += fast_exp2(fmaf(x[j], kLog2e, -mnew));
  }
  s_run = (m_run == kNegInf ? 0.f : s_run * fast_exp2(m_run - mnew)) + (a0 + a1);
  m_run = mnew;
}

// If the target column (lab_rel, relative to the 256-column half) lies in
// 32-column chunk c, write its 16-bit logit (from the packed words w) to *xt_row.
template <typename OutT>
__device__ __forceinline__ void lce_target_from_chunk(const uint32_t* w, int c, int64_t lab_rel, float* xt_row) {
  const int64_t li = lab_rel - c * 32;
  if ((uint64_t)li < 32u) {
    // one select per word, written so the compiler cannot turn the chain
    // into an indexed load (that would move w to local memory)
    uint32_t word = 0;
    const int wi = (int)(li >> 1);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      asm("{\n\t.reg .pred p;\n\tsetp.eq.s32 p, %2, %3;\n\tselp.b32 %0, %1, %0, p;\n\t}"
          : "+r"(word)
          : "r"(w[j]), "r"(wi), "r"(j));
    float lo, hi;
    unpack2<OutT>(word, lo, hi);
    *xt_row = (li & 1) ? hi : lo;
  }
}

// Fold 32 packed 16-bit logits (columns c * 32 .. c * 32 + 31 of a 256-column
// half starting at n0) into the running pair and record the target logit if
// it lies in this chunk (lab_rel: target column relative to n0). Two
// 16-column sub-chunks keep few values live.
template <typename OutT>
__device__ __forceinline__ void lce_fold_chunk(const uint32_t* w, int c, int n0, int N, int64_t lab_rel,
                                               float* xt_row, float& m_run, float& s_run) {
  const int col0 = n0 + c * 32;
  const bool full = col0 + 32 <= N;
#pragma unroll
  for (int sc = 0; sc < 2; ++sc) {
    float x[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) unpack2<OutT>(w[sc * 8 + j], x[2 * j], x[2 * j + 1]);
    lce_fold16(x, full, col0 + sc * 16, N, m_run, s_run);
  }
  lce_target_from_chunk<OutT>(w, c, lab_rel, xt_row);
}

// Geometry of one configuration. PAIR = 1: one CTA computes a 128 x 256 tile.
// PAIR = 2: a 2-CTA cluster computes a 256 x 256 tile with tcgen05.mma
// cta_group::2; each CTA stages its 128 rows of A and 128 of the 256 B rows,
// and holds its 128 accumulator rows in its own TMEM.
// NSUB = 2 (pairs only): the pair tile is 256 x 512, two N = 256 MMAs per K
// step share each staged A tile, so a CTA moves 48 KB from L2 per 8.4 MFLOP
// instead of 32 KB per 4.2 MFLOP. Operand traffic from L2 is about a quarter
// of the GEMM's energy and the GEMM runs at the power cap, so the wider tile
// buys clock. The 128 x 512 fp32 accumulator fills all of TMEM, so the
// halves are published and released separately: a tile's last STG k-steps
// finish half 0 first (the epilogue drains it while half 1 finishes) and the
// next tile's first STG k-steps run on half 0 while half 1 is drained.
template <int PAIR, int NSUB = 1>
struct Geo {
  static_assert(NSUB == 1 || PAIR == 2, "the 512-column tile needs a CTA pair");
  static constexpr int TM = BM * PAIR;            // tile rows
  static constexpr int TN = BN * NSUB;            // tile columns
  static constexpr int HB = BN / PAIR;            // B rows per CTA per 256-column half
  static constexpr int B_ROWS = HB * NSUB;        // B rows staged per CTA
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int HALF_BYTES = HB * BK * 2;  // one half's B tile
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STG = NSUB == 2 ? 4 : (PAIR == 2 ? 6 : 4);   // pipeline depth
  // operand stages, 1 KB alignment slack, barriers (256 B), epilogue exchange
  // (2 x 128 float2) and one 2 KB store-staging buffer per epilogue warp
  static constexpr int SMEM = STG * (A_BYTES + B_BYTES) + 1024 + 256 + 2 * BM * 8 + EPI_WARPS * 2048;
};

template <typename T, int A_MN, int B_MN, int EPI, typename OutT, int PAIR, int NSUB>
__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  using G = Geo<PAIR, NSUB>;
  static_assert(NSUB == 1 || sizeof(OutT) == 2, "the 512-column tile parks 16-bit outputs only");
  static_assert(EPI != EPI_LCE_Q || NSUB == 1, "the q store runs on 256-column tiles");
  constexpr int STG = G::STG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STG * G::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STG * G::B_BYTES);
  uint64_t* empty = full + STG;
  uint64_t* tfull = empty + STG;
  uint64_t* tempty = tfull + 2;
  uint64_t* xready = tempty + 2;  // group 1's (max, sum) of a half is in xchg[b]
  uint64_t* xdone = xready + 2;   // group 0 has read xchg[b]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(xdone + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float2* xchg = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(full) + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* stage_out = reinterpret_cast<uint8_t*>(xchg + 2 * BM) + (warp >= EPI_WARP0 ? (warp - EPI_WARP0) * 2048 : 0);
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
      tc::mbar_init(&tempty[b], EPI_WARPS * PAIR);
      tc::mbar_init(&xready[b], 4);
      tc::mbar_init(&xdone[b], 4);
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
        const TileK tk = tile_k(p, tile, nkb);
        const int ma = tk.mt * G::TM + (int)rank * BM;      // this CTA's A rows
        const int nb = tk.nt * G::TN + (int)rank * G::HB;   // this CTA's B rows (first half)
        for (int kb = tk.kb0; kb < tk.kb1; ++kb) {
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
#pragma unroll
            for (int h = 0; h < NSUB; ++h) {
              uint8_t* bh = b + h * G::HALF_BYTES;
              const int nbh = nb + h * BN;
              if (B_MN) {
#pragma unroll
                for (int j = 0; j < G::HB / 64; ++j)
                  tc::tma_load_2d_pair_hint(bh + j * (BK * 128), &tmB, fb, nbh + j * 64, k0, pol_b);
              } else {
                tc::tma_load_2d_pair_hint(bh, &tmB, fb, k0, nbh, pol_b);
              }
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
      if (NSUB == 2) {
        // One 512-column accumulator: half h at columns [h * BN, h * BN + BN).
        // The first `pre` k-steps run on half 0 only and keep their stages;
        // once the epilogue has released half 1 they are replayed on it and
        // freed, then both halves advance together.
        auto issue = [&](int st_, int h, bool first) {
          const uint32_t a0 = tc::smem_u32(sA + st_ * G::A_BYTES);
          const uint32_t b0 = tc::smem_u32(sB + st_ * G::B_BYTES + h * G::HALF_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = tc::smem_desc_sw128(a0 + k * a_kstep, a_lbo, a_sbo);
            const uint64_t bd = tc::smem_desc_sw128(b0 + k * b_kstep, b_lbo, b_sbo);
            tc::mma_f16_pair(tmem_base + h * BN, ad, bd, idesc, !(first && k == 0));
          }
        };
        // k-steps [0, pre) open a tile on half 0 while the epilogue still
        // drains half 1 of the previous tile; k-steps [nkt - tail, nkt) close
        // it half 0 first, so the epilogue starts on half 0 while the tensor
        // pipe finishes half 1.
        for (int tile = unit; tile < p.num_tiles; tile += nunits) {
          const TileK tk = tile_k(p, tile, nkb);
          const int nkt = tk.kb1 - tk.kb0;  // k-steps of this unit
          const int pre = nkt < STG ? nkt : STG;
          const int tail = nkt - pre < STG ? nkt - pre : STG;
          if (!tc::mbar_wait(&tempty[0], acc_phase ^ 1, abort_flag, lim)) break;
          tc::tc_fence_after();
          bool ok = true;
          int s = stage;
          uint32_t ph = phase;
          for (int kb = 0; kb < pre; ++kb) {
            if (!tc::mbar_wait(&full[s], ph, abort_flag, lim)) { ok = false; break; }
            tc::tc_fence_after();
            issue(s, 0, kb == 0);
            if (++s == STG) { s = 0; ph ^= 1; }
          }
          if (!ok) break;
          if (!tc::mbar_wait(&tempty[1], acc_phase ^ 1, abort_flag, lim)) break;
          tc::tc_fence_after();
          for (int kb = 0; kb < pre; ++kb) {
            issue(stage, 1, kb == 0);
            tc::mma_commit_pair_mc(&empty[stage], 0x3);
            if (++stage == STG) { stage = 0; phase ^= 1; }
          }
          for (int kb = pre; kb < nkt - tail; ++kb) {
            if (!tc::mbar_wait(&full[stage], phase, abort_flag, lim)) { ok = false; break; }
            tc::tc_fence_after();
            issue(stage, 0, false);
            issue(stage, 1, false);
            tc::mma_commit_pair_mc(&empty[stage], 0x3);
            if (++stage == STG) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          s = stage;
          ph = phase;
          for (int kb = 0; kb < tail; ++kb) {
            if (!tc::mbar_wait(&full[s], ph, abort_flag, lim)) { ok = false; break; }
            tc::tc_fence_after();
            issue(s, 0, false);
            if (++s == STG) { s = 0; ph ^= 1; }
          }
          if (!ok) break;
          tc::mma_commit_pair_mc(&tfull[0], 0x3);
          for (int kb = 0; kb < tail; ++kb) {
            issue(stage, 1, false);
            tc::mma_commit_pair_mc(&empty[stage], 0x3);
            if (++stage == STG) { stage = 0; phase ^= 1; }
          }
          tc::mma_commit_pair_mc(&tfull[1], 0x3);
          acc_phase ^= 1;
        }
      } else
      for (int tile = unit; tile < p.num_tiles; tile += nunits) {
        const TileK tk = tile_k(p, tile, nkb);
        const int nkt = tk.kb1 - tk.kb0;
        if (!tc::mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, lim)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nkt; ++kb) {
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
  } else if (warp >= EPI_WARP0) {
    // ---------------- epilogue ----------------
    // Two groups of four warps; warp w reads TMEM lanes 32 * (w % 4) and group
    // g takes columns [g * 128, g * 128 + 128) of each 256-column block. In
    // the plain-store path TMEM loads run one 32-column chunk ahead of the
    // math; the CE paths load 16 columns at a time to stay within registers.
    const int q = warp & 3;
    const int g = (warp - EPI_WARP0) >> 2;
    const uint32_t tempty_leader0 = tc::mapa_shared(tc::smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = tc::mapa_shared(tc::smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int xbuf = 0;
    uint32_t xphase = 0;  // bit b: phase of xready[b]
    bool stop = false;
    for (int tile = unit; tile < p.num_tiles && !stop; tile += nunits) {
      const TileK tk = tile_k(p, tile, nkb);
      const int mt = tk.mt, nt = tk.nt;
      void* const pout = tk.ks ? p.out2 : p.out;  // this K slice's output
      const int m0 = mt * G::TM + (int)rank * BM;
      if (NSUB == 1) {
        if (!tc::mbar_wait(&tfull[acc], acc_phase, abort_flag, lim)) break;
        tc::tc_fence_after();
      }
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      // Both groups hold (max, sum) partials of the same rows for one
      // 256-column block; group 1 hands its pair to group 0 through
      // xchg[xbuf], and group 0 writes the merged statistics of block `sub`.
      // xready / xdone order the two sides of each buffer's every use.
      auto stats_exchange_at = [&](int sub, float m, float sm) -> bool {
        float2* xs = xchg + xbuf * BM;
        const uint32_t ph = (xphase >> xbuf) & 1u;
        bool ok = true;
        if (g == 1) {
          if ((ok = tc::mbar_wait(&xdone[xbuf], ph ^ 1u, abort_flag, lim))) {
            xs[q * 32 + lane] = make_float2(m, sm);
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&xready[xbuf]);
          }
        } else if ((ok = tc::mbar_wait(&xready[xbuf], ph, abort_flag, lim))) {
          const float2 o = xs[q * 32 + lane];
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&xdone[xbuf]);
          const MS t = ms_merge(MS{m, sm}, MS{o.x, o.y});
          if (row_ok) p.stats[(int64_t)(nt * NSUB + sub) * p.M + row] = make_float2(t.m, t.s);
        }
        xphase ^= 1u << xbuf;
        xbuf ^= 1;
        return ok;
      };
      if constexpr (NSUB == 2) {
        {
          // 512-column tile, 16-bit output. Each warp drains its 4 chunks of a
          // half from TMEM, finishes the first at once and parks the other 3
          // as packed 16-bit values in registers, then releases the half: the
          // MMAs get TMEM back after ~1/4 of the epilogue work. The parked
          // chunks (CE statistics and the stores, whose shared-memory traffic
          // competes with the MMAs' operand reads) are done afterwards while
          // the next tile's MMAs run.
          constexpr int PW = (EPI_CHUNKS - 1) * 16;  // parked words per half
          uint32_t pk[2][PW];
          float hm[2] = {kNegInf, kNegInf}, hs[2] = {0.f, 0.f};
          const float scale = (EPI == EPI_STORE && p.scale ? *p.scale : 1.f) *
                              (EPI == EPI_STORE && p.row_scale && row_ok ? p.row_scale[row] : 1.f);
          const int64_t lab = (EPI == EPI_LCE && row_ok) ? p.labels[row] - p.label_offset : -1;
          float* xt_row = EPI == EPI_LCE ? p.xt + row : nullptr;
          OutT* out = tile_out_base<OutT>(p, pout, mt * G::TM);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!tc::mbar_wait(&tfull[h], acc_phase, abort_flag, lim)) { stop = true; break; }
            tc::tc_fence_after();
            const int n0 = nt * G::TN + h * BN;
            if (n0 < p.N) {
              const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + h * BN + g * EPI_CHUNKS * 32;
              __syncwarp();
#pragma unroll
              for (int i = 0; i < EPI_CHUNKS; ++i) {
                uint32_t w[16];
#pragma unroll
                for (int sc = 0; sc < 2; ++sc) {
                  uint32_t r[16];
                  tc::tmem_ld16_wait(tb + i * 32 + sc * 16, r);
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                    const uint32_t v =
                        pack2<OutT>(__uint_as_float(r[2 * j]) * scale, __uint_as_float(r[2 * j + 1]) * scale);
                    if (i == 0) w[sc * 8 + j] = v;
                    else pk[h][(i - 1) * 16 + sc * 8 + j] = v;
                  }
                }
                if (i == 0) {
                  const int c = g * EPI_CHUNKS;
                  if (EPI == EPI_LCE) lce_fold_chunk<OutT>(w, c, n0, p.N, lab - n0, xt_row, hm[h], hs[h]);
                  if (out)
                    store_chunk_packed<OutT>(out, p.ldo, m0 + q * 32, p.M, n0 + c * 32, p.N, w, stage_out, lane,
                                             p.vec_ok, p.out_evict_first);
                }
              }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_cluster(h ? tempty_leader1 : tempty_leader0);
          }
          if (stop) break;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int n0 = nt * G::TN + h * BN;
            if (n0 >= p.N) continue;
#pragma unroll
            for (int i = 1; i < EPI_CHUNKS; ++i) {
              const int c = g * EPI_CHUNKS + i;
              if (EPI == EPI_LCE) lce_fold_chunk<OutT>(&pk[h][(i - 1) * 16], c, n0, p.N, lab - n0, xt_row, hm[h], hs[h]);
              if (out)
                store_chunk_packed<OutT>(out, p.ldo, m0 + q * 32, p.M, n0 + c * 32, p.N, &pk[h][(i - 1) * 16],
                                         stage_out, lane, p.vec_ok, p.out_evict_first);
            }
            if (EPI == EPI_LCE) {
              // group 1 hands its (max, sum) to group 0, which writes the half's stats
              if (!stats_exchange_at(h, hm[h], hs[h])) stop = true;
            }
          }
          acc_phase ^= 1;
        }
      } else {
#pragma unroll 1
      for (int h = 0; h < NSUB; ++h) {
        if (NSUB == 2) {  // each half is published on its own barrier
          if (!tc::mbar_wait(&tfull[h], acc_phase, abort_flag, lim)) { stop = true; break; }
          tc::tc_fence_after();
        }
        const int n0 = nt * G::TN + h * BN;
        const int sub = NSUB == 2 ? h : acc;  // accumulator (half) index
        const int c0 = g * EPI_CHUNKS;        // first 32-column chunk of this group
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + sub * BN + c0 * 32;
        if (n0 < p.N) {
          __syncwarp();
          if constexpr (EPI == EPI_LCE_Q) {
            static_assert(NSUB == 1 && sizeof(OutT) == 2, "the q store runs on 256-column tiles, 16-bit output");
            const int64_t lab = row_ok ? p.labels[row] - p.label_offset : -1;
            const int64_t lab_rel = lab - n0;
            // Pass 1: the window decision for this row's 128 columns of the
            // tile, from the fp32 accumulator.
            float cmax = kNegInf;
#pragma unroll 1
            for (int i = 0; i < EPI_CHUNKS; ++i) {
              uint32_t r[32];
              tc::tmem_ld32(tbase + i * 32, r);
              tc::tmem_ld_wait(r);
              const int col0 = n0 + (c0 + i) * 32;
              if (col0 + 32 <= p.N) {
#pragma unroll
                for (int j = 0; j < 32; ++j) cmax = fmaxf(cmax, __uint_as_float(r[j]));
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.N) cmax = fmaxf(cmax, __uint_as_float(r[j]));
              }
            }
            const bool any_col = n0 + c0 * 32 < p.N;
            const float cml = cmax * kLog2e;
            const bool raw = any_col && !(cml <= kQHi && cml >= kQLo);  // NaN: raw
            if (row_ok && any_col) p.qmode[((int64_t)(nt * NSUB + h) * 2 + g) * p.M + row] = raw ? 1 : 0;
            // Pass 2: round to bf16 (the reference's logits dtype), record the
            // target logit, then store q = e^x (or the raw logit) and fold the
            // statistics: sum q directly (pair (0, sum)) or, for raw groups,
            // the running (max, sum) of the plain CE epilogue.
            float m_run = kNegInf, s_run = 0.f, s_q = 0.f;
#pragma unroll 1
            for (int i = 0; i < EPI_CHUNKS; ++i) {
              const int c = c0 + i;
              const int col0 = n0 + c * 32;
              uint32_t w[16];
#pragma unroll
              for (int sc = 0; sc < 2; ++sc) {
                uint32_t r[16];
                tc::tmem_ld16_wait(tbase + i * 32 + sc * 16, r);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  w[sc * 8 + j] = pack2<OutT>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
              }
              lce_target_from_chunk<OutT>(w, c, lab_rel, p.xt + row);
              const bool full = col0 + 32 <= p.N;
              if (raw) {
#pragma unroll
                for (int sc = 0; sc < 2; ++sc) {
                  float x[16];
#pragma unroll
                  for (int j = 0; j < 8; ++j) unpack2<OutT>(w[sc * 8 + j], x[2 * j], x[2 * j + 1]);
                  lce_fold16(x, full, col0 + sc * 16, p.N, m_run, s_run);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  float a, b;
                  unpack2<OutT>(w[j], a, b);
                  a = fast_exp2(a * kLog2e);
                  b = fast_exp2(b * kLog2e);
                  if (!full) {
                    if (col0 + 2 * j >= p.N) a = 0.f;
                    if (col0 + 2 * j + 1 >= p.N) b = 0.f;
                  }
                  s_q += a + b;
                  w[j] = pack2<OutT>(a, b);
                }
              }
              if (pout)
                store_chunk_packed<OutT>(reinterpret_cast<OutT*>(pout), p.ldo, m0 + q * 32, p.M, col0, p.N, w,
                                         stage_out, lane, p.vec_ok, p.out_evict_first);
            }
            if (!raw) {
              m_run = s_q > 0.f ? 0.f : kNegInf;
              s_run = s_q;
            }
            if (!stats_exchange_at(h, m_run, s_run)) stop = true;
          } else if constexpr (EPI == EPI_LCE) {
            const int64_t lab = row_ok ? p.labels[row] - p.label_offset : -1;
            const int64_t lab_rel = lab - n0;  // label column inside this half, if any
            float m_run = kNegInf, s_run = 0.f;
#pragma unroll 1
            for (int i = 0; i < EPI_CHUNKS; ++i) {
              const int c = c0 + i;
              // the logits tensor holds the product rounded to the input dtype
              // (as the reference's cuBLAS output); statistics use those values
              uint32_t w[16];
#pragma unroll
              for (int sc = 0; sc < 2; ++sc) {
                uint32_t r[16];
                tc::tmem_ld16_wait(tbase + i * 32 + sc * 16, r);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  w[sc * 8 + j] = pack2<OutT>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
              }
              lce_fold_chunk<OutT>(w, c, n0, p.N, lab_rel, p.xt + row, m_run, s_run);
              if (pout)
                store_chunk_packed<OutT>(reinterpret_cast<OutT*>(pout), p.ldo, m0 + q * 32, p.M, n0 + c * 32, p.N, w,
                                         stage_out, lane, p.vec_ok, p.out_evict_first);
            }
            // group 1 hands its (max, sum) to group 0, which writes the half's stats
            if (!stats_exchange_at(h, m_run, s_run)) stop = true;
          } else {
            const float scale = (p.scale ? *p.scale : 1.f) * (p.row_scale && row_ok ? p.row_scale[row] : 1.f);
            uint32_t ra[32], rb[32];
            tc::tmem_ld32(tbase, ra);
#pragma unroll
            for (int i = 0; i < EPI_CHUNKS; ++i) {
              uint32_t(&r)[32] = (i & 1) ? rb : ra;
              tc::tmem_ld_wait(r);
              if (i + 1 < EPI_CHUNKS) tc::tmem_ld32(tbase + (i + 1) * 32, (i & 1) ? ra : rb);
              const int col0 = n0 + (c0 + i) * 32;
              if (col0 < p.N) {
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * scale;
                if (!row_ok) {
                } else if (p.add_f32) {
                  float a[32];
                  load_row32<float>(p.add_f32 + (int64_t)row * p.ldadd, col0, p.N, a, p.vec_ok);
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] += a[j];
                } else if (p.add_same) {
                  float a[32];
                  load_row32<OutT>(reinterpret_cast<const OutT*>(p.add_same) + (int64_t)row * p.ldadd, col0, p.N,
                                   a, p.vec_ok);
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] += a[j];
                }
                store_chunk<OutT>(tile_out_base<OutT>(p, pout, mt * G::TM), p.ldo, m0 + q * 32, p.M, col0, p.N, v,
                                  stage_out, lane, p.vec_ok, p.out_evict_first);
              }
            }
          }
        }
        // release this accumulator buffer (half) to the (leader's) MMA warp
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR == 2) tc::mbar_arrive_cluster(sub ? tempty_leader1 : tempty_leader0);
          else tc::mbar_arrive(&tempty[sub]);
        }
        if (stop) break;
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  }
  // stores to another GPU's memory are visible there before the grid is done
  if (p.npeer > 0 && warp >= EPI_WARP0) __threadfence_system();
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
