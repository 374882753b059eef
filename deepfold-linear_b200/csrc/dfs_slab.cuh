// dfs_slab.cuh -- pieces shared by the resident forward and backward kernels.
//
// A CTA owns a 64-row slab of one N x N problem.  In registers the slab is laid
// out as E[r][k] = element (kRpw*warp + r, 32*k + lane): each of the kWarps warps
// holds kRpw rows, each lane the columns congruent to it mod 32.  Row reductions
// are lane reductions (reduce4_rows), column reductions go through shared memory
// and, across the cluster, through distributed shared memory.
#pragma once

#include "dfs_kernels.cuh"

namespace dfs {

// Drain an M=64 fp32 accumulator (TMEM columns [col_base, col_base+NP)) into the
// 64 x NP 128B-swizzled staging buffer, multiplied by `scale`.  TMEM row m of an
// M=64 MMA sits in lane (m % 16) + 32 (m / 16); a warp may only read the lane
// quarter warp % 4, so the kWarps/4 warps sharing a quarter split the 32-column
// chunks.  Caller synchronises before and after.
template <int NP>
DFS_DEV void drain_m64(float* Ts, uint32_t tbase, uint32_t col_base, float scale, int warp, int lane) {
  const int q = warp & 3, grp = warp >> 2;
#pragma unroll 1
  for (int ch = grp; ch < NP / 32; ch += kWarps / 4) {
    const int col0 = 32 * ch;
    float v[32];
    tmem_ld32(tbase + (static_cast<uint32_t>(32 * q) << 16) + col_base + col0, v);
    if (lane < 16) {
      const int row = 16 * q + lane, r = row & 7;
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(Ts) +
                                              ((((col0 >> 5) * 8 + (row >> 3)) << 10) + (r << 7)));
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4)
        dst[c4 ^ r] = make_float4(v[4 * c4] * scale, v[4 * c4 + 1] * scale, v[4 * c4 + 2] * scale,
                                  v[4 * c4 + 3] * scale);
    }
  }
}

// Column owned by thread tid = 32 warp + lane (tid < NP) in the CTA column
// reductions below: a permutation of 0..NP-1 inside each warp.
DFS_DEV int col_of_thread(int warp, int lane) { return 32 * warp + 4 * (lane & 7) + (lane >> 3); }

// CTA total of the per-warp column partials red[w * NP + j] (w < kWarps) for
// column col_of_thread(warp, lane); call from the threads tid < NP only
// (whole warps).  Lane l of warp w takes quad q = 8w + (l & 7) (columns
// 4q..4q+3) and sums the warp partials 4g..4g+3, g = l >> 3, so that each
// quarter-warp reads 128 contiguous bytes (no bank conflicts); a reduce-scatter
// over the 4 lanes of the quad (xor 16, xor 8: 3 shuffles) leaves lane l with
// column 4q + g.  Summation order is fixed: every CTA gets identical bits.
template <int NP>
DFS_DEV float colsum16(const float* red, int warp, int lane) {
  static_assert(kWarps == 16, "four warp partials per lane of a quad");
  const int qd = 8 * warp + (lane & 7), g4 = lane >> 3;
  const float* rp = red + (4 * g4) * NP + 4 * qd;
  float4 s4 = *reinterpret_cast<const float4*>(rp);
#pragma unroll
  for (int w = 1; w < 4; ++w) {
    const float4 x = *reinterpret_cast<const float4*>(rp + w * NP);
    s4 = make_float4(s4.x + x.x, s4.y + x.y, s4.z + x.z, s4.w + x.w);
  }
  const bool hi = (g4 & 2) != 0, odd = (g4 & 1) != 0;
  const float k0 = hi ? s4.z : s4.x, k1 = hi ? s4.w : s4.y;  // columns 2h, 2h+1 kept
  const float o0 = hi ? s4.x : s4.z, o1 = hi ? s4.y : s4.w;  // the other half, sent
  const float a0 = k0 + __shfl_xor_sync(0xffffffffu, o0, 16);
  const float a1 = k1 + __shfl_xor_sync(0xffffffffu, o1, 16);
  const float kk = odd ? a1 : a0, oo = odd ? a0 : a1;
  return kk + __shfl_xor_sync(0xffffffffu, oo, 8);
}

template <int NS>
DFS_DEV void stage_to_regs(float (&E)[kRpw][NS], const float* Ts, int warp, int lane) {
#pragma unroll
  for (int r = 0; r < kRpw; ++r)
#pragma unroll
    for (int k = 0; k < NS; ++k) E[r][k] = Ts[sw_off(kRpw * warp + r, 32 * k + lane, 64) >> 2];
}

template <int NS>
DFS_DEV void regs_to_stage(const float (&E)[kRpw][NS], float* Ts, int warp, int lane) {
#pragma unroll
  for (int r = 0; r < kRpw; ++r)
#pragma unroll
    for (int k = 0; k < NS; ++k) Ts[sw_off(kRpw * warp + r, 32 * k + lane, 64) >> 2] = E[r][k];
}

// Position / geometry terms of the cost, folded into the slab as
// S' -= (pos_weight[h, bins_ij] + w_h dist_ij / (r_h + dist_ij)) * s_scale
// (src/deepfold/model/kernels/sinkhorn_kernel.py:107-127).
struct BiasArgs {
  const float* pos_weight;   // (H, 68) or null
  BinSource bins;            // position bins (table or compute_bins inputs)
  const float* xrow;         // smem, 3 x 64 row coordinates (x, y, z planes)
  const float* xcol;         // smem, 3 x NP column coordinates
  bool geo;                  // geometry term present
  float w_h, r_0, s_scale;   // r_0: this head's geometry scale r_h
  int bb, hh, N, row0;
  bool transposed;           // slab rows are cost columns (bins read as [col][row])
};

// Subtract the bias terms from the staged 64 x NP slab S' (128B-swizzled, see
// sw_off).  A rolled loop over the tile: the code stays small, consecutive
// threads touch consecutive columns (coalesced bin reads).
template <int NP>
DFS_DEV void add_cost_bias_stage(float* Ts, const BiasArgs& a, int tid) {
#pragma unroll 1
  for (int idx = tid; idx < 64 * NP; idx += kThreads) {
    const int li = idx / NP, gj = idx - li * NP, gi = a.row0 + li;
    if (gi >= a.N || gj >= a.N) continue;
    float bias = 0.0f;
    if (a.pos_weight) {
      const unsigned bin = static_cast<unsigned>(a.transposed ? bin_at(a.bins, a.bb, a.N, gj, gi)
                                                              : bin_at(a.bins, a.bb, a.N, gi, gj));
      // bins outside [0, 68) add nothing
      bias += bin < 68u ? a.pos_weight[a.hh * 68 + bin] : 0.0f;
    }
    if (a.geo) {
      const float d0 = a.xrow[li] - a.xcol[gj], d1 = a.xrow[64 + li] - a.xcol[NP + gj],
                  d2 = a.xrow[128 + li] - a.xcol[2 * NP + gj];
      const float dist = sqrtf(d0 * d0 + d1 * d1 + d2 * d2 + 1e-8f);
      bias += a.w_h * dist / (a.r_0 + dist);
    }
    Ts[sw_off(li, gj, 64) >> 2] -= bias * a.s_scale;
  }
}

// Dense cost rows [row0, row0+64) of a (., N, N) fp32 matrix into the staging
// tile as S' = -C * s_scale (zero outside N x N).
template <int NP>
DFS_DEV void dense_cost_to_stage(float* Ts, const float* Cm, size_t bh, int N, int row0, float s_scale, int tid) {
#pragma unroll 1
  for (int idx = tid; idx < 64 * NP; idx += kThreads) {
    const int li = idx / NP, gj = idx - li * NP, gi = row0 + li;
    Ts[sw_off(li, gj, 64) >> 2] = (gi < N && gj < N) ? -__ldg(Cm + (bh * N + gi) * N + gj) * s_scale : 0.0f;
  }
}

// 16-byte chunk of elements of type T widened to fp32.
template <typename T>
struct Chunk16 {
  static constexpr int kElems = 16 / static_cast<int>(sizeof(T));
};
DFS_DEV void widen(const uint4& raw, float (&v)[8], __nv_bfloat16*) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(h[q]);
    v[2 * q] = f.x;
    v[2 * q + 1] = f.y;
  }
}
DFS_DEV void widen(const uint4& raw, float (&v)[8], __half*) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __half22float2(h[q]);
    v[2 * q] = f.x;
    v[2 * q + 1] = f.y;
  }
}
DFS_DEV void widen(const uint4& raw, float (&v)[4], float*) {
  v[0] = __uint_as_float(raw.x);
  v[1] = __uint_as_float(raw.y);
  v[2] = __uint_as_float(raw.z);
  v[3] = __uint_as_float(raw.w);
}

// Rows [row_first, row_first+ROWS) of a row-major (., DH) tensor of T (rows at
// or beyond N read as zero) into a 128B-swizzled fp32 operand buffer: with
// TR = false element (i, c) lands at (i, c) of a buffer with ROWS rows, with
// TR = true at (c, i) of a buffer with DH rows (the K-major operand holding the
// transpose).  Each thread moves 16-byte chunks and issues all of its loads
// before consuming any, so the tile costs one global-memory round trip.
template <int DH, int ROWS, bool TR, typename T, int NT = kThreads>
DFS_DEV void load_tile(float* dst, const T* src, int row_first, int N, int tid) {
  constexpr int kThreads = NT;              // threads taking part
  constexpr int EPC = Chunk16<T>::kElems;   // elements per chunk
  constexpr int CPR = DH / EPC;             // chunks per row
  constexpr int TOTAL = ROWS * CPR;
  constexpr int BATCH = (TOTAL + kThreads - 1) / kThreads;
  uint4 raw[BATCH];
  // chunk c -> (row i, chunk-in-row ch): row-major order for the plain tile
  // (coalesced reads, 16-byte stores); column-major order for the transposed
  // one, so that the 32 lanes of a warp store 32 consecutive columns of one
  // output row (conflict-free)
  auto row_of = [](int c) { return TR ? c % ROWS : c / CPR; };
  auto chunk_of = [](int c) { return TR ? c / ROWS : c % CPR; };
#pragma unroll
  for (int b = 0; b < BATCH; ++b) {
    const int c = tid + kThreads * b;
    const int gi = row_first + row_of(c);
    raw[b] = make_uint4(0u, 0u, 0u, 0u);
    if ((TOTAL % kThreads == 0 || c < TOTAL) && gi < N)
      raw[b] = __ldg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(gi) * DH) + chunk_of(c));
  }
#pragma unroll
  for (int b = 0; b < BATCH; ++b) {
    const int c = tid + kThreads * b;
    if (TOTAL % kThreads != 0 && c >= TOTAL) break;
    const int i = row_of(c), c0 = chunk_of(c) * EPC;
    float v[EPC];
    widen(raw[b], v, static_cast<T*>(nullptr));
    if (!TR) {
#pragma unroll
      for (int q = 0; q < EPC / 4; ++q)
        *reinterpret_cast<float4*>(dst + (sw_off(i, c0 + 4 * q, ROWS) >> 2)) =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int q = 0; q < EPC; ++q) dst[sw_off(c0 + q, i, DH) >> 2] = v[q];
    }
  }
}

template <int DH, int ROWS, bool TR, int NT = kThreads>
DFS_DEV void load_tile_any(float* dst, const void* src, int dtype, size_t base_row, int row_first, int N,
                           int tid) {
  if (dtype == DFS_BF16)
    load_tile<DH, ROWS, TR, __nv_bfloat16, NT>(dst, reinterpret_cast<const __nv_bfloat16*>(src) + base_row * DH,
                                               row_first, N, tid);
  else if (dtype == DFS_F16)
    load_tile<DH, ROWS, TR, __half, NT>(dst, reinterpret_cast<const __half*>(src) + base_row * DH, row_first, N,
                                        tid);
  else
    load_tile<DH, ROWS, TR, float, NT>(dst, reinterpret_cast<const float*>(src) + base_row * DH, row_first, N,
                                       tid);
}

// Load rows [row_first, row_first+ROWS) of a (., DH) tensor into a
// 128B-swizzled fp32 operand buffer with ROWS rows (rows beyond N are zero).
template <int DH, int ROWS>
DFS_DEV void load_operand(float* dst, const void* src, int dtype, size_t base_row, int row_first, int N, int tid) {
  load_tile_any<DH, ROWS, false>(dst, src, dtype, base_row, row_first, N, tid);
}

// Transposed load: element (row gi, c) of a (., DH) tensor goes to (row c,
// column gi - row_first) of a 128B-swizzled buffer with DH rows and ROWS
// columns, i.e. the K-major operand holding the tensor's transpose.
template <int DH, int ROWS>
DFS_DEV void load_operand_t(float* dst, const void* src, int dtype, size_t base_row, int row_first, int N,
                            int tid) {
  load_tile_any<DH, ROWS, true>(dst, src, dtype, base_row, row_first, N, tid);
}

// fp32 variants for already-fp32 tensors (upstream gradients).
template <int DH, int ROWS>
DFS_DEV void load_operand_f32(float* dst, const float* src, size_t base_row, int row_first, int N, int tid) {
  load_tile<DH, ROWS, false>(dst, src + base_row * DH, row_first, N, tid);
}
template <int DH, int ROWS>
DFS_DEV void load_operand_f32_t(float* dst, const float* src, size_t base_row, int row_first, int N, int tid) {
  load_tile<DH, ROWS, true>(dst, src + base_row * DH, row_first, N, tid);
}

// Bulk prefetch into L2 of rows [row0, min(row0+64, N)) of a row-major
// (., DH) tensor with `esize`-byte elements (one instruction per tensor; the
// caller guarantees 16-byte alignment, which DH * esize a multiple of 16 keeps).
DFS_DEV void prefetch_slab_l2(const void* base, size_t base_row, int row0, int N, int DH, int esize) {
  const int rows = min(64, N - row0);
  if (rows <= 0) return;
  const char* p = reinterpret_cast<const char*>(base) + (base_row + row0) * static_cast<size_t>(DH) * esize;
  const uint32_t bytes = static_cast<uint32_t>(rows) * DH * esize;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Issue D (TMEM, M=64 rows x NN columns) = A (64 x KD, K-major) * B (NN x KD,
// K-major)^T, both 128B-swizzled fp32 buffers read as tf32, B stored with NN
// rows (one elected thread).  The descriptors are built once; each K step
// advances their start-address field (bits 0-13, 16-byte units, no carry for
// shared-memory addresses) by a compile-time offset, so issuing costs a few
// instructions per MMA.
template <int NN, int KD>
DFS_DEV void issue_abt(uint32_t d_tmem, const float* A, const float* Bm) {
  constexpr int NH = NN > 256 ? 2 : 1;
  constexpr int NCH = NN / NH;
  constexpr uint32_t idesc = idesc_tf32(64, NCH, 0, 0);
  const uint64_t a0 = sw128_desc(smem_u32(A), 16, 1024), b0 = sw128_desc(smem_u32(Bm), 16, 1024);
#pragma unroll
  for (int h2 = 0; h2 < NH; ++h2) {
#pragma unroll
    for (int kk = 0; kk < KD / 8; ++kk) {
      const uint64_t ao = static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
      const uint64_t bo = static_cast<uint64_t>(((kk >> 2) * NN * 128 + (h2 * NCH / 8) * 1024 + (kk & 3) * 32) >> 4);
      mma_tf32(d_tmem + h2 * NCH, a0 + ao, b0 + bo, idesc, kk > 0 ? 1u : 0u);
    }
  }
}

// D (TMEM, MA rows x NN columns, MA = 64 or 128) (+)= A (MA x KD) * B (NN x KD)^T,
// both K-major 128B-swizzled fp32 buffers (A stored with MA rows, B with NN
// rows) read as tf32; `accumulate` = false starts the accumulator.  With
// MA = 128, row m of the result is TMEM lane m.  One elected thread.
template <int MA, int NN, int KD>
DFS_DEV void issue_mma(uint32_t d_tmem, const float* A, const float* Bm, bool accumulate) {
  static_assert((MA == 64 || MA == 128) && NN % 16 == 0 && NN <= 256 && KD % 8 == 0, "UMMA shape");
  constexpr uint32_t idesc = idesc_tf32(MA, NN, 0, 0);
  const uint64_t a0 = sw128_desc(smem_u32(A), 16, 1024), b0 = sw128_desc(smem_u32(Bm), 16, 1024);
#pragma unroll
  for (int kk = 0; kk < KD / 8; ++kk) {
    const uint64_t ao = static_cast<uint64_t>(((kk >> 2) * MA * 128 + (kk & 3) * 32) >> 4);
    const uint64_t bo = static_cast<uint64_t>(((kk >> 2) * NN * 128 + (kk & 3) * 32) >> 4);
    mma_tf32(d_tmem, a0 + ao, b0 + bo, idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

// As issue_abt for a narrow result (NN <= 256) with a long K: the K steps are
// dealt round-robin to NACC independent accumulators at TMEM columns
// d_tmem + a * NN (a < NACC), so consecutive MMAs do not wait on each other's
// accumulation; the reader sums the NACC partials.
template <int NN, int KD, int NACC>
DFS_DEV void issue_abt_split(uint32_t d_tmem, const float* A, const float* Bm) {
  static_assert(NN <= 256 && (KD / 8) % NACC == 0, "narrow result, K steps divisible by NACC");
  constexpr uint32_t idesc = idesc_tf32(64, NN, 0, 0);
  const uint64_t a0 = sw128_desc(smem_u32(A), 16, 1024), b0 = sw128_desc(smem_u32(Bm), 16, 1024);
#pragma unroll
  for (int kk = 0; kk < KD / 8; ++kk) {
    const uint64_t ao = static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
    const uint64_t bo = static_cast<uint64_t>(((kk >> 2) * NN * 128 + (kk & 3) * 32) >> 4);
    mma_tf32(d_tmem + (kk % NACC) * NN, a0 + ao, b0 + bo, idesc, kk >= NACC ? 1u : 0u);
  }
}

// Issue S = Q K^T for the slab (one elected thread): A = Q slab (64 x DH,
// K-major), B = K (NP x DH, K-major), D = TMEM columns [0, NP).
template <int NP, int DH>
DFS_DEV void issue_qk(uint32_t tbase, const float* Qs, const float* Ks) {
  issue_abt<NP, DH>(tbase, Qs, Ks);
}

// Drain an M=64 result of DH columns held as NACC partial accumulators (TMEM
// columns [col + a*DH, col + (a+1)*DH), see issue_abt_split) to a row-major
// global (rows, DH) tensor, rows row0.. (< N), scaled.  Warps 0-3 (one per
// TMEM lane quarter) read 16 columns at a time.
template <int DH, int NACC>
DFS_DEV void drain_rows_to_global(uint32_t tbase, uint32_t col, float* out, size_t row_base, int row0, int N,
                                  float scale, int warp, int lane) {
  if (warp >= 4) return;
  const uint32_t lanes = static_cast<uint32_t>(32 * warp) << 16;
  const int gi = row0 + 16 * warp + lane;
#pragma unroll
  for (int g = 0; g < DH / 16; ++g) {
    float v[16];
    tmem_ld16(tbase + lanes + col + 16 * g, v);
#pragma unroll
    for (int a = 1; a < NACC; ++a) {
      float t[16];
      tmem_ld16(tbase + lanes + col + a * DH + 16 * g, t);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += t[i];
    }
    if (lane < 16 && gi < N) {
      float4* dst = reinterpret_cast<float4*>(out + (row_base + gi) * DH + 16 * g);
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4)
        dst[c4] = make_float4(v[4 * c4] * scale, v[4 * c4 + 1] * scale, v[4 * c4 + 2] * scale,
                              v[4 * c4 + 3] * scale);
    }
  }
}

}  // namespace dfs
