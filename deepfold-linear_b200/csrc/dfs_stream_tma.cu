// dfs_stream_tma.cu -- TMA-staged, warp-specialised row passes of the streamed
// path for sm_100a.
//
// Three passes dominate a streamed call: the Sinkhorn half-update (a row
// log-sum-exp, run twice per iteration: rows, then the same pass on S^T), the
// row statistics of the transport output, and the plan-vector product of the
// IFT conjugate-gradient solve (twice per CG iteration).  All three stream the
// columns of S = A B^T past a block of 128 rows and reduce each row on the fly:
//
//   LSE       f_i = kappa (a_i - LSE_j(x_ij)),          x = S' + g_j  (log2 units)
//   ROWSTATS  m_i = f_i + max_j x_ij, R_i = sum_j exp2(x_ij - max_j x_ij)
//   MATVEC    y_i = c_i sum_j exp2(x_ij + f_i) v_j
//
// (S' = S log2(e) / (eps sqrt d); a masked column has g_j = -inf.)  One CTA per
// block of 128 rows; its ten warps split the work so that no thread that does
// arithmetic ever waits on global memory:
//
//   warp 8      producer: one TMA load of the row block (A), then column tiles
//               of B (128 rows of the column operand) into a ring of NS stages,
//               with the tile's column bias (and vector) staged beside it
//   warp 9      MMA: S tile = A B_tile^T, tcgen05.mma kind::f16 (bf16 / fp16
//               operands, exactly the reference's products of bf16 inputs) or
//               kind::tf32 (fp32 operands), fp32 into one of two TMEM buffers
//   warps 0-7   epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (thread =
//               row) and columns 64 (w / 4) .. + 63 of every tile with
//               tcgen05.ld, folding them into a running reduction per row;
//               the two halves of each row are merged at the end
//
// Two epilogue warps per lane quadrant, and two CTAs per SM, give every SM
// sub-partition four warps of exp2 / FMA work to interleave.
//
// The MMA of tile t+1 runs while the epilogue works on tile t.  Operands are
// K-major with 128-byte swizzle, the layout TMA writes for a box 128 bytes wide;
// a 256-byte row (fp32, d = 64) is two such boxes side by side.  The kernels
// cover 128- and 256-byte operand rows (d = 64, or fp32 with d = 32); other
// shapes, and operands not aligned to 16 bytes, keep the register-staged
// kernels of dfs_stream.cu / dfs_stream_bwd.cu.
#include <cstdlib>
#include <mutex>

#include "dfs_tma.cuh"

namespace dfs {

constexpr int kTThreads = 320;  // warps 0-7 epilogue, 8 producer, 9 MMA
constexpr int kTEpi = 256;      // epilogue threads
constexpr int kTProducer = 8, kTMma = 9;
constexpr float kLag = 16.0f;   // log2 headroom of the lagged exponent reference
constexpr int kMaxSplit = 8;    // column splits of a row block (small grids)
constexpr int kSplitCtas = 4096;  // CTAs of a split launch at most (their partials' scratch)
// bf16 / fp16 passes: the 32 elements of a chunk are worked in 16 pairs with the
// packed fp32 pair instructions (one FMA / ADD issue per two elements); the
// pairs whose bit is set in kPolyPairs take their exponentials as a polynomial
// on the FMA pipes (ex2_poly2) instead of the MUFU, whose throughput bounds
// these passes -- 4 of 16 pairs (8 of 32 elements) balance the MUFU's 8 cycles
// per warp instruction against the issue slots the rest of the chunk needs.
#ifndef DFS_POLY_PAIRS
#define DFS_POLY_PAIRS 0x1111u  // pairs 0, 4, 8, 12
#endif
constexpr unsigned kPolyPairs = DFS_POLY_PAIRS;
constexpr int kTCols = 128;     // columns per tile

struct TileParams {
  CUtensorMap tmA;         // row operand, (BH, N, d) viewed as the 3-D tensor {d, N, BH}
  CUtensorMap tmB;         // column operand, same view
  const float* eps;        // (H,)
  const float* mask;       // (B, N) nonzero = valid, or null
  const float* col_bias;   // (BH, N) potential of the columns, log2 units
  const float* col_vec;    // MATVEC: (BH, N) the vector v
  const float* row_bias;   // ROWSTATS, MATVEC: (BH, N) potential of the rows, log2 units
  const float* row_marg;   // LSE: (BH, N) natural-log marginal of the rows
  const float* row_scale;  // MATVEC: (BH, N) factor c_i, or null (1)
  const int32_t* done;     // MATVEC: (BH) skip problems whose flag is nonzero, or null
  float* row_out;          // LSE: potential (log2); ROWSTATS: m; MATVEC: y
  float* row_out_nat;      // LSE: the potential in natural-log units, or null
  float* row_R;            // ROWSTATS: R
  int32_t* status;         // DFS_ERR_DEVICE_TIMEOUT is OR-ed in if a wait gives up, or null
  // peer exchange (LSE): every GPU's copy of row_out, their arrival counters,
  // and this GPU's counter with the count to wait for before reading
  int npeers;
  float* peer_out[DFS_MAX_PEERS];
  unsigned long long* peer_cnt[DFS_MAX_PEERS];
  const unsigned long long* wait_cnt;
  unsigned long long wait_for;
  const int2* extent;      // (B) valid extents of the mask, or null (scan the mask)
  float* part;             // nsplit > 1: (CTA, 3, 128) partial results of the column splits
  unsigned* counter;       // nsplit > 1: (BH * row blocks) arrival counters, zero between launches
  int B, H, N;
  int row_begin, row_end;  // rows this launch handles
  int nsplit;              // CTAs per row block, each over a contiguous share of the column tiles
  float lam;
  float qk_scale;          // 1/sqrt(d) of the cost
  CostTerms ct;            // optional position / geometry terms in this pass's orientation
};

// TERMS: the variant with the optional cost terms (a 3-stage ring when rows are
// 128 bytes, to make room for the staged column coordinates and bin weights)
template <int DT, int D, bool TERMS = false>
struct TileCfg {
  static constexpr int ESZ = DT == DFS_F32 ? 4 : 2;
  static constexpr int RB = D * ESZ;       // bytes per operand row
  static_assert(RB == 128 || RB == 256, "128- or 256-byte operand rows");
  static constexpr int G = RB / 128;       // 128-byte swizzle atoms across a row
  static constexpr int KSTEPS = RB / 32;   // one MMA per 32 bytes of K
  static constexpr uint32_t GROUP = 128u * 128u;  // bytes of one atom column of a 128-row tile
  static constexpr uint32_t TILE = 128u * RB;     // bytes of a 128-row tile
  static constexpr int NS = RB == 128 ? (TERMS ? 3 : 4) : 2;  // stages of the column-tile ring
  static constexpr uint32_t OFF_A = 0;
  static constexpr uint32_t OFF_B = OFF_A + TILE;
  static constexpr uint32_t OFF_CB = OFF_B + NS * TILE;   // NS x 128 column bias
  static constexpr uint32_t OFF_CV = OFF_CB + NS * 512u;  // NS x 128 column vector
  static constexpr uint32_t OFF_CX = OFF_CV + NS * 512u;                 // TERMS: NS x 3 x 128 column coordinates
  static constexpr uint32_t OFF_PW = OFF_CX + (TERMS ? NS * 1536u : 0u);  // TERMS: 69 scaled bin weights (+ pad)
  static constexpr uint32_t OFF_MRG = OFF_PW + (TERMS ? 288u : 0u);       // 3 x 128 partials of the second half, a flag
  // bf16 / fp16 operands: the column bias rides in the MMA as one more K = 16
  // slice (A: ones, B: the bias in three bf16 parts), in the no-swizzle
  // core-matrix layout, 128 rows x 32 bytes = 4 KB per tile
  static constexpr bool kExt = DT != DFS_F32;
  static constexpr uint32_t EXT = 4096u;
  static constexpr uint32_t OFF_AX = OFF_MRG + 1536u + 16u + 112u;  // 128-byte aligned
  static constexpr uint32_t OFF_BX = OFF_AX + (kExt ? EXT : 0u);
  static constexpr uint32_t OFF_BAR = OFF_BX + (kExt ? NS * EXT : 0u);
  static constexpr uint32_t NBAR = 2 * NS + 5;            // full, empty, sfull x2, sempty x2, afull
  static constexpr uint32_t OFF_SLOT = OFF_BAR + 8 * NBAR;
  static constexpr uint32_t OFF_RED = OFF_SLOT + 16;
  static constexpr uint32_t NEED = OFF_RED + 4u * 2 * (kTThreads / 32) + 1024;  // + alignment slack
  // at least 80 KB: at most two CTAs per SM, whose 2 x 256 TMEM columns always fit
  static constexpr uint32_t SMEM = NEED > 81920u ? NEED : 81920u;
  static_assert(NEED <= 113u * 1024u, "two CTAs per SM");
};

// Rows [row0, row0 + 128) of problem `prob` into a tile buffer (G boxes of 128
// bytes x 128 rows; rows beyond N arrive as zeros).
template <int DT, int D>
DFS_DEV void tma_tile(uint32_t dst, const CUtensorMap* tm, int row0, int prob, uint32_t bar) {
  using C = TileCfg<DT, D>;
#pragma unroll
  for (int g = 0; g < C::G; ++g) tma_load_3d(dst + g * C::GROUP, tm, g * (128 / C::ESZ), row0, prob, bar);
}

// S (128 x 128, TMEM) = A (128 x d) B (128 x d)^T from two K-major swizzled tiles.
template <int DT, int D>
DFS_DEV void tile_mma(uint32_t d_tmem, uint32_t a_s, uint32_t b_s) {
  using C = TileCfg<DT, D>;
  const uint64_t a0 = sw128_desc(a_s, 16, 1024), b0 = sw128_desc(b_s, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < C::KSTEPS; ++kk) {
    const uint64_t off = static_cast<uint64_t>(((kk >> 2) * C::GROUP + (kk & 3) * 32) >> 4);
    if constexpr (DT == DFS_F32)
      mma_tf32(d_tmem, a0 + off, b0 + off, idesc_tf32(128, kTCols, 0, 0), kk > 0 ? 1u : 0u);
    else
      mma_f16(d_tmem, a0 + off, b0 + off, idesc_f16(128, kTCols, DT == DFS_BF16), kk > 0 ? 1u : 0u);
  }
}

template <int MODE, int DT, int D, bool TERMS>
__global__ void __launch_bounds__(kTThreads, 2) tile_kernel(const __grid_constant__ TileParams p) {
  using C = TileCfg<DT, D, TERMS>;
  // launched as a programmatic dependent of the previous kernel on the stream:
  // its grid is set up while that kernel drains; nothing is read before this
  // wait returns, i.e. before the previous kernel's results are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the next pass on the stream may now be launched and rasterised into the
  // slots this grid's last wave frees; its first instruction is the same wait,
  // so it reads nothing before this grid has finished
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sA = smem_u32(base + C::OFF_A), sB = smem_u32(base + C::OFF_B);
  float* cbs = reinterpret_cast<float*>(base + C::OFF_CB);
  float* cvs = reinterpret_cast<float*>(base + C::OFF_CV);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::OFF_BAR);  // [NS] tile staged
  uint64_t* empty = full + C::NS;                                      // [NS] tile consumed
  uint64_t* sfull = empty + C::NS;                                     // [2] S buffer written
  uint64_t* sempty = sfull + 2;                                        // [2] S buffer read
  uint64_t* afull = sempty + 2;                                        // row block staged
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + C::OFF_SLOT);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  const int blk = blockIdx.x / p.nsplit, sp = blockIdx.x % p.nsplit;
  const int prob = blk / nrb, rb = blk % nrb;
  if (MODE == TL_MATVEC && p.done != nullptr && p.done[prob] != 0) return;  // uniform over the CTA
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const size_t bh = static_cast<size_t>(prob);
  const int r0 = p.row_begin + 128 * rb;
  // only column tiles holding a valid point are visited (a masked column adds
  // exactly nothing); a block without a valid row visits none
  int vlo, vhi;
  valid_extent<kTThreads>(p.extent, p.mask, bb, N, reinterpret_cast<int*>(base + C::OFF_RED), vlo, vhi);
  const int rhi = min(min(r0 + 128, p.row_end), N);
  const bool live = max(r0, vlo) < min(rhi, vhi);
  if (!live) {
    // No valid row in this block: its rows' results are the masked-row values.
    // The block's first CTA writes them (in a peer exchange to every GPU, after
    // the same wait as any CTA, with the block's one signal); every CTA of the
    // block returns before any set-up.
    if (sp == 0) {
      int derr = 0;
      if (p.wait_cnt != nullptr && tid == 0) {
        uint64_t t0 = 0;
        for (uint32_t it = 0; ld_acquire_sys_u64(p.wait_cnt) < p.wait_for; ++it) {
          if (it == 0) t0 = global_ns();
          else if ((it & 63u) == 0 && global_ns() - t0 > kWaitNs) { derr = 1; break; }
          __nanosleep(64);
        }
      }
      __syncthreads();
      for (int i = tid; i < rhi - r0; i += kTThreads) {
        const size_t o = bh * N + r0 + i;
        if constexpr (MODE == TL_LSE) {
          if (p.npeers > 0) {
            for (int k = 0; k < p.npeers; ++k) p.peer_out[k][o] = 0.0f;
          } else {
            p.row_out[o] = 0.0f;
          }
          if (p.row_out_nat) p.row_out_nat[o] = 0.0f;
        } else {
          p.row_out[o] = 0.0f;
          if constexpr (MODE == TL_ROWSTATS) p.row_R[o] = 0.0f;
        }
      }
      if (MODE == TL_LSE && p.npeers > 0) {
        __threadfence_system();
        __syncthreads();
        if (tid == 0)
          for (int k = 0; k < p.npeers; ++k) atomicAdd_system(p.peer_cnt[k], 1ull);
      }
      if (derr && tid == 0 && p.status != nullptr) atomicOr(p.status, DFS_ERR_DEVICE_TIMEOUT);
    }
    return;
  }
  // this CTA's contiguous share of the row block's column tiles
  const int t_all = live ? (vhi + kTCols - 1) / kTCols - vlo / kTCols : 0;
  const int t_q = t_all / p.nsplit, t_r = t_all % p.nsplit;
  const int t_begin = (live ? vlo / kTCols : 0) + sp * t_q + min(sp, t_r);
  const int ntiles = t_q + (sp < t_r ? 1 : 0);

  if (warp == 0) tmem_alloc(tslot, 256);
  if (tid == 32 * kTProducer) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 32);     // every producer lane (bias stores); the TMA bytes as transactions
      mbar_init(&empty[s], 1 + 8);  // MMA completion + the 8 epilogue warps (bias reads)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], 8);
    }
    mbar_init(afull, 1);
    fence_mbar_init();
  }
  if constexpr (C::kExt) {
    // extension operand A: rows [1, 1, 1, 0 ...] (B rows are written whole by
    // the producer, per tile)
    uint32_t* ax = reinterpret_cast<uint32_t*>(base + C::OFF_AX);
    const uint32_t one = DT == DFS_BF16 ? 0x3F80u : 0x3C00u;
    for (int i = tid; i < static_cast<int>(C::EXT / 4); i += kTThreads) {
      // 32-bit word i holds elements (2i, 2i+1) of the layout: element k of row r sits at
      // ((r / 8) * 2 + k / 8) * 64 + (r % 8) * 8 + k % 8 (in 2-byte units)
      const int e = 2 * i, kchunk = (e >> 6) & 1, k = (kchunk << 3) | (e & 7);
      const uint32_t lo = k < 3 ? one : 0u, hi = (k + 1) < 3 ? one : 0u;
      ax[i] = lo | (hi << 16);
    }
    fence_async_smem();
  }
  int err = 0;
  if (p.wait_cnt != nullptr && tid == 0) {
    // peer exchange: the potentials this phase reads are complete on this GPU
    // once every GPU's previous phase has raised the counter (bounded wait)
    uint64_t t0 = 0;
    for (uint32_t it = 0; ld_acquire_sys_u64(p.wait_cnt) < p.wait_for; ++it) {
      if (it == 0) t0 = global_ns();
      else if ((it & 63u) == 0 && global_ns() - t0 > kWaitNs) { err = 1; break; }
      __nanosleep(64);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  bool final_cta_of_block = true;  // this CTA writes the block's results (column splits: the last one)
  if (warp == kTProducer) {
    // ------------------------------------------------------------ producer
    if (ntiles > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(smem_u32(afull), C::TILE);
        tma_tile<DT, D>(sA, &p.tmA, r0, prob, smem_u32(afull));
      }
      const float inv_scale = p.eps[hh] / (kLog2e * p.qk_scale);  // 1 / scale
      (void)inv_scale;
      // the tile's column bias (and vector), 4 columns per lane, fetched one tile
      // ahead so that their global latency overlaps the wait for a free stage
      float pc[4], pw[4], px[3][4];
      const float* xg = TERMS ? p.ct.x : nullptr;  // geometry term: the columns' coordinates, staged beside the tile
      auto fetch = [&](int u) {
        const int c0 = (t_begin + u) * kTCols;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j = c0 + lane + 32 * q;
          const bool cin = j < N;
          const bool cok = cin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
          pc[q] = cok ? __ldcg(p.col_bias + bh * N + j) : -INFINITY;  // L2: peers may have written it
          if constexpr (MODE == TL_MATVEC) pw[q] = cin ? p.col_vec[bh * N + j] : 0.0f;
          if (xg != nullptr) {
#pragma unroll
            for (int c = 0; c < 3; ++c) px[c][q] = cin ? xg[(static_cast<size_t>(bb) * N + j) * 3 + c] : 0.0f;
          }
        }
      };
      fetch(0);
#pragma unroll 1
      for (int u = 0; u < ntiles; ++u) {
        const int s = u % C::NS;
        if (u >= C::NS && !mbar_wait(&empty[s], ((u / C::NS) - 1) & 1)) err = 1;
        const int c0 = (t_begin + u) * kTCols;
        if (lane == 0) {
          mbar_expect_tx(smem_u32(&full[s]), C::TILE);
          tma_tile<DT, D>(sB + s * C::TILE, &p.tmB, c0, prob, smem_u32(&full[s]));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = lane + 32 * q;
          if constexpr (C::kExt) {
            // bias / scale as three bf16 / fp16 parts hi + mid + lo (a masked column: -inf, 0, 0)
            const float y = pc[q] * inv_scale;
            float r1 = 0.0f, r2 = 0.0f;
            uint32_t h0, h1, h2;
            if constexpr (DT == DFS_BF16) {
              const __nv_bfloat16 b0 = __float2bfloat16_rn(y);
              const bool fin = y > -1e30f;
              r1 = fin ? y - __bfloat162float(b0) : 0.0f;
              const __nv_bfloat16 b1 = __float2bfloat16_rn(r1);
              r2 = fin ? r1 - __bfloat162float(b1) : 0.0f;
              const __nv_bfloat16 b2 = __float2bfloat16_rn(r2);
              h0 = __bfloat16_as_ushort(b0);
              h1 = __bfloat16_as_ushort(b1);
              h2 = __bfloat16_as_ushort(b2);
            } else {
              const __half b0 = __float2half_rn(y);
              const bool fin = y > -1e30f;
              r1 = fin ? y - __half2float(b0) : 0.0f;
              const __half b1 = __float2half_rn(r1);
              r2 = fin ? r1 - __half2float(b1) : 0.0f;
              const __half b2 = __float2half_rn(r2);
              h0 = __half_as_ushort(b0);
              h1 = __half_as_ushort(b1);
              h2 = __half_as_ushort(b2);
            }
            // row c: elements 0-7 (core matrix of K chunk 0) and 8-15 (chunk 1, zeros)
            uint4* row = reinterpret_cast<uint4*>(base + C::OFF_BX + s * C::EXT + (c >> 3) * 256 + (c & 7) * 16);
            row[0] = make_uint4(h0 | (h1 << 16), h2, 0u, 0u);
            row[8] = make_uint4(0u, 0u, 0u, 0u);
          } else {
            cbs[s * 128 + c] = pc[q];
          }
          if constexpr (MODE == TL_MATVEC) cvs[s * 128 + c] = pw[q];
          if (TERMS && xg != nullptr) {
            float* cx = reinterpret_cast<float*>(base + C::OFF_CX) + s * 384;
#pragma unroll
            for (int k = 0; k < 3; ++k) cx[k * 128 + c] = px[k][q];
          }
        }
        if constexpr (C::kExt) fence_async_smem();  // the MMA reads the extension rows
        mbar_arrive(&full[s]);
        if (u + 1 < ntiles) fetch(u + 1);
      }
      // the last stages' releases: every MMA completion has arrived before exit
      for (int u = max(0, ntiles - C::NS); u < ntiles; ++u)
        if (!mbar_wait(&empty[u % C::NS], (u / C::NS) & 1)) err = 1;
    }
  } else if (warp == kTMma) {
    // ------------------------------------------------------------ MMA issuer
    if (ntiles > 0) {
      if (!mbar_wait(afull, 0)) err = 1;
#pragma unroll 1
      for (int u = 0; u < ntiles; ++u) {
        const int s = u % C::NS, b = u & 1;
        if (!mbar_wait(&full[s], (u / C::NS) & 1)) err = 1;
        if (u >= 2 && !mbar_wait(&sempty[b], ((u >> 1) - 1) & 1)) err = 1;
        tc_fence_after();
        if (lane == 0) {
          tile_mma<DT, D>(tbase + b * kTCols, sA, sB + s * C::TILE);
          if constexpr (C::kExt)  // + the column bias: ones x (bias parts), K = 16
            mma_f16(tbase + b * kTCols, noswz_desc(smem_u32(base + C::OFF_AX), 128, 256),
                    noswz_desc(smem_u32(base + C::OFF_BX + s * C::EXT), 128, 256),
                    idesc_f16(128, kTCols, DT == DFS_BF16), 1u);
          mma_commit(&sfull[b]);
          mma_commit(&empty[s]);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3, half = warp >> 2;
    const int lrow = 32 * quad + lane, row = r0 + lrow;
    const bool rin = row < p.row_end && row < N;
    const bool rok = rin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + row] != 0.0f);
    const float eps_h = p.eps[hh];
    const float scale = kLog2e * p.qk_scale / eps_h;
    const float fi = (MODE != TL_LSE && rin) ? __ldcg(p.row_bias + bh * N + row) : 0.0f;
    const uint32_t tlane = static_cast<uint32_t>(32 * quad) << 16;
    // optional cost terms: bin weights scaled to -log2(e)/eps in shared memory
    // (entry 68, the table's "no bin", is 0), this row's coordinates
    const bool use_bins = TERMS && p.ct.bins != nullptr, use_geo = TERMS && p.ct.x != nullptr;
    constexpr bool has_terms = TERMS;
    float* pws = reinterpret_cast<float*>(base + C::OFF_PW);
    const float* cxs = reinterpret_cast<const float*>(base + C::OFF_CX);
    float xi0 = 0.0f, xi1 = 0.0f, xi2 = 0.0f, wS = 0.0f, r_h = 1.0f;
    const uint8_t* brow = nullptr;
    if constexpr (has_terms) {
      const float nsc = -kLog2e / eps_h;
      if (use_bins && tid <= kBinCount) pws[tid] = tid < kBinCount ? p.ct.pos_weight[hh * kBinCount + tid] * nsc : 0.0f;
      if (use_geo) {
        wS = p.ct.w_dist[hh] * nsc;
        r_h = geo_scale(p.ct, hh);
        if (rin) {
          const float* xr = p.ct.x + (static_cast<size_t>(bb) * N + row) * 3;
          xi0 = xr[0];
          xi1 = xr[1];
          xi2 = xr[2];
        }
      }
      if (use_bins && rin) brow = p.ct.bins + (static_cast<size_t>(bb) * N + row) * p.ct.bin_stride;
      asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory");  // pws written
    }
    // running reference, exact maximum and sum of exp2(x - reference) of this
    // half's columns (LSE, ROWSTATS)
    float m = kNeg, mt = kNeg, sum = 0.0f;
    float acc = 0.0f;            // MATVEC
#pragma unroll 1
    for (int u = 0; u < ntiles; ++u) {
      const int s = u % C::NS, b = u & 1;
      // this row's bins of the tile's columns of this half (64 bytes), loaded ahead of the waits
      uint4 bq[4] = {};
      if (TERMS && brow != nullptr) {
        const uint4* src = reinterpret_cast<const uint4*>(brow + (t_begin + u) * kTCols + 64 * half);
#pragma unroll
        for (int q = 0; q < 4; ++q) bq[q] = __ldg(src + q);
      }
      if (!mbar_wait(&full[s], (u / C::NS) & 1)) err = 1;  // the producer's bias stores
      if (!mbar_wait(&sfull[b], (u >> 1) & 1)) err = 1;
      tc_fence_after();
      // the second chunk's TMEM load overlaps the first chunk's arithmetic
      uint32_t r0v[32], r1v[32];
      tmem_ld32_async(tbase + tlane + b * kTCols + 64 * half, r0v);
      tmem_wait_ld(r0v);
      tmem_ld32_async(tbase + tlane + b * kTCols + 64 * half + 32, r1v);
      // with cost terms: x = S' + column bias (+ row bias for MATVEC) + term, then the
      // plain reductions below on x
      auto chunk_terms = [&](uint32_t (&rv32)[32], int ch) {
        const float* cb = cbs + s * 128 + 32 * ch;
        const float* xs = cxs + s * 384 + 32 * ch;
        const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bq[2 * (ch & 1)]);
        float x[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          float t = C::kExt ? 0.0f : cb[k];
          if constexpr (MODE == TL_MATVEC) t += fi;
          if (use_bins) t += pws[(bw[k >> 2] >> (8 * (k & 3))) & 0xffu];
          if (use_geo) {
            const float d0 = xi0 - xs[k], d1 = xi1 - xs[128 + k], d2 = xi2 - xs[256 + k];
            const float dist = sqrtf(fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, 1e-8f))));
            t = fmaf(wS, __fdividef(dist, r_h + dist), t);
          }
          x[k] = fmaf(__uint_as_float(rv32[k]), scale, t);
        }
        if constexpr (MODE == TL_MATVEC) {
          const float* cv = cvs + s * 128 + 32 * ch;
          float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int k = 0; k < 32; ++k) a[k & 3] = fmaf(ex2(x[k]), cv[k], a[k & 3]);
          acc += (a[0] + a[1]) + (a[2] + a[3]);
        } else {
          float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int k = 0; k < 32; ++k) a[k & 3] += ex2(x[k] - m);
          float cm = kNeg;
#pragma unroll
          for (int k = 0; k < 32; ++k) cm = fmaxf(cm, x[k]);
          mt = fmaxf(mt, cm);
          if (cm > m + kLag) {
            a[0] = a[1] = a[2] = a[3] = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; ++k) a[k & 3] += ex2(x[k] - cm);
            sum *= ex2(m - cm);
            m = cm;
          }
          sum += (a[0] + a[1]) + (a[2] + a[3]);
        }
      };
      auto chunk = [&](uint32_t (&rv32)[32], int ch) {
        if constexpr (has_terms) {
          chunk_terms(rv32, ch);
        } else {
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(rv32[k]);
        const float* cb = cbs + s * 128 + 32 * ch;
        if constexpr (MODE == TL_MATVEC && C::kExt) {
          // v = S + g / scale (the column bias came with the MMA); element pairs
          const float* cv = cvs + s * 128 + 32 * ch;
          const float2 sc2 = make_float2(scale, scale), fi2 = make_float2(fi, fi);
          float2 a0 = make_float2(0.0f, 0.0f), a1 = a0;
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float2 x = __ffma2_rn(make_float2(v[k], v[k + 1]), sc2, fi2);
            const float2 e = ((kPolyPairs >> (k >> 1)) & 1u) ? ex2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
            const float2 w = *reinterpret_cast<const float2*>(cv + k);
            if ((k >> 1) & 1) a1 = __ffma2_rn(e, w, a1);
            else a0 = __ffma2_rn(e, w, a0);
          }
          acc += (a0.x + a1.x) + (a0.y + a1.y);
        } else if constexpr (MODE == TL_MATVEC) {
          const float* cv = cvs + s * 128 + 32 * ch;
          float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int k = 0; k < 32; ++k) a[k & 3] = fmaf(ex2(fmaf(v[k], scale, cb[k] + fi)), cv[k], a[k & 3]);
          acc += (a[0] + a[1]) + (a[2] + a[3]);
        } else if constexpr (C::kExt) {
          // v = S + g / scale: x - m = v scale - m is one FMA per element; the
          // chunk maximum is taken on v (scale > 0).  Same lagged reference as below.
          // element pairs: x = v scale - m by one packed FMA, the pair's
          // exponentials (MUFU or polynomial), two packed partial sums
          const float2 sc2 = make_float2(scale, scale);
          float2 nm2 = make_float2(-m, -m);
          float2 a0 = make_float2(0.0f, 0.0f), a1 = a0;
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float2 x = __ffma2_rn(make_float2(v[k], v[k + 1]), sc2, nm2);
            const float2 e = ((kPolyPairs >> (k >> 1)) & 1u) ? ex2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
            if ((k >> 1) & 1) a1 = __fadd2_rn(a1, e);
            else a0 = __fadd2_rn(a0, e);
          }
          const float cm = max32(v) * scale;
          mt = fmaxf(mt, cm);
          if (cm > m + kLag) {
            a0 = a1 = make_float2(0.0f, 0.0f);
            nm2 = make_float2(-cm, -cm);
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
              const float2 x = __ffma2_rn(make_float2(v[k], v[k + 1]), sc2, nm2);
              const float2 e = make_float2(ex2(x.x), ex2(x.y));
              if ((k >> 1) & 1) a1 = __fadd2_rn(a1, e);
              else a0 = __fadd2_rn(a0, e);
            }
            sum *= ex2(m - cm);
            m = cm;
          }
          sum += (a0.x + a1.x) + (a0.y + a1.y);
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = fmaf(v[k], scale, cb[k]);
          // exponents against the running reference m (a maximum of the earlier
          // columns), so they need not wait for this chunk's maximum, which is
          // reduced alongside; a chunk whose maximum exceeds m by more than kLag
          // (the first one, and rarely any other) moves the reference and is
          // summed again.  The sum then stays within [1, N 2^kLag].
          float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int k = 0; k < 32; ++k) a[k & 3] += ex2(v[k] - m);
          float mx[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) mx[q] = fmaxf(fmaxf(v[4 * q], v[4 * q + 1]), fmaxf(v[4 * q + 2], v[4 * q + 3]));
          const float cm = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
          mt = fmaxf(mt, cm);
          if (cm > m + kLag) {
            a[0] = a[1] = a[2] = a[3] = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; ++k) a[k & 3] += ex2(v[k] - cm);
            sum *= ex2(m - cm);
            m = cm;
          }
          sum += (a[0] + a[1]) + (a[2] + a[3]);
        }
        }  // no cost terms
      };
      chunk(r0v, 2 * half);
      tmem_wait_ld(r1v);
      chunk(r1v, 2 * half + 1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sempty[b]);
        mbar_arrive(&empty[s]);
      }
    }
    // merge the two column halves of each row (epilogue threads only)
    float* mrg = reinterpret_cast<float*>(base + C::OFF_MRG);
    if (half == 1) {
      mrg[lrow] = MODE == TL_MATVEC ? acc : m;
      mrg[128 + lrow] = sum;
      mrg[256 + lrow] = mt;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory");
    bool final_cta = true;
    if (half == 0) {
      if constexpr (MODE == TL_MATVEC) {
        acc += mrg[lrow];
      } else {
        const float m2 = mrg[lrow], s2 = mrg[128 + lrow];
        const float mm = fmaxf(m, m2);
        sum = sum * ex2(m - mm) + s2 * ex2(m2 - mm);
        m = mm;
        mt = fmaxf(mt, mrg[256 + lrow]);
      }
    }
    if (p.nsplit > 1) {
      // column-split row block: publish this CTA's partials; the last CTA of the
      // block to arrive merges all of them and re-arms the counter
      // this CTA's partials: 3 x 128 floats at its grid index (blk * nsplit + sp)
      float* mine = p.part + static_cast<size_t>(blockIdx.x) * 384;
      if (half == 0 && rin) {
        mine[lrow] = MODE == TL_MATVEC ? acc : m;
        mine[128 + lrow] = sum;
        mine[256 + lrow] = mt;
      }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory");
      volatile int* flag = reinterpret_cast<volatile int*>(mrg + 384);
      if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counter[blk], 1u);
        const int last = prev == static_cast<unsigned>(p.nsplit - 1);
        if (last) p.counter[blk] = 0u;  // every CTA of this block has arrived
        *flag = last;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory");
      final_cta = *flag != 0;
      final_cta_of_block = final_cta;
      if (final_cta) {
        __threadfence();
        if (half == 0 && rin) {
          m = kNeg;
          sum = 0.0f;
          mt = kNeg;
          acc = 0.0f;
          for (int q = 0; q < p.nsplit; ++q) {
            const float* pq = p.part + (static_cast<size_t>(blk) * p.nsplit + q) * 384;
            const float a0 = __ldcg(pq + lrow);
            const float a1 = __ldcg(pq + 128 + lrow);
            const float a2 = __ldcg(pq + 256 + lrow);
            if constexpr (MODE == TL_MATVEC) {
              acc += a0;
            } else {
              const float mm = fmaxf(m, a0);
              sum = sum * ex2(m - mm) + a1 * ex2(a0 - mm);
              m = mm;
              mt = fmaxf(mt, a2);
            }
          }
        }
      }
    }
    if (final_cta && half == 0 && rin) {
      const size_t o = bh * N + row;
      if constexpr (MODE == TL_MATVEC) {
        p.row_out[o] = rok ? acc * (p.row_scale != nullptr ? p.row_scale[o] : 1.0f) : 0.0f;
      } else {
        if constexpr (MODE == TL_LSE) {
          const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
          float f = 0.0f;
          if (rok && sum > 0.0f) f = kap * (p.row_marg[o] * kLog2e - (m + lg2(sum)));
          if (p.npeers > 0) {
            for (int k = 0; k < p.npeers; ++k) p.peer_out[k][o] = f;  // NVLink stores, own copy included
          } else {
            p.row_out[o] = f;
          }
          if (p.row_out_nat) p.row_out_nat[o] = f * kLn2;
        } else {
          // the row maximum itself and the sum relative to it
          p.row_out[o] = rok ? mt + fi : 0.0f;
          p.row_R[o] = rok ? sum * ex2(m - mt) : 0.0f;
        }
      }
    }
  }
  if (MODE == TL_LSE && p.npeers > 0 && final_cta_of_block && warp < kTEpi / 32) {
    // every GPU's copy of this block's rows is written (the epilogue threads'
    // stores, ordered before thread 0's system-scope fence by the barrier;
    // the fence is cumulative): raise every counter once.  Only the CTA that
    // wrote the block's potentials fences; the other column splits wrote only
    // local partials, already ordered for the merging CTA.
    asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory");
    if (tid == 0) {
      __threadfence_system();
      for (int k = 0; k < p.npeers; ++k) atomicAdd_system(p.peer_cnt[k], 1ull);
    }
  }
  if (err && p.status != nullptr) atomicOr(p.status, DFS_ERR_DEVICE_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// ---------------------------------------------------------------- host side
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

}  // namespace

bool tmap_available() { return encode_fn() != nullptr; }

bool make_tmap(CUtensorMap* tm, const void* ptr, int dtype, int inner, int rows, int BH, int box_inner,
               int box_rows) {
  const int esz = dtype == DFS_F32 ? 4 : 2;
  if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || box_inner * esz != 128) return false;
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const CUtensorMapDataType ty = dtype == DFS_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == DFS_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(BH)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(inner) * esz, static_cast<cuuint64_t>(rows) * inner * esz};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(tm, ty, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

template <int MODE, int DT, int D, bool TERMS>
cudaError_t launch_tile_mdd(const TileParams& p, cudaStream_t st) {
  using C = TileCfg<DT, D, TERMS>;
  auto kern = tile_kernel<MODE, DT, D, TERMS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  return launch_dependent(kern, dim3(p.B * p.H * nrb * p.nsplit), dim3(kTThreads), C::SMEM, st, p);
}

template <int MODE, bool TERMS>
cudaError_t launch_tile_mt(int dtype, int d, const TileParams& p, cudaStream_t st) {
  if (d == 64) {
    if (dtype == DFS_BF16) return launch_tile_mdd<MODE, DFS_BF16, 64, TERMS>(p, st);
    if (dtype == DFS_F16) return launch_tile_mdd<MODE, DFS_F16, 64, TERMS>(p, st);
    return launch_tile_mdd<MODE, DFS_F32, 64, TERMS>(p, st);
  }
  return launch_tile_mdd<MODE, DFS_F32, 32, TERMS>(p, st);
}

template <int MODE>
cudaError_t launch_tile_m(int dtype, int d, const TileParams& p, cudaStream_t st) {
  if (p.ct.bins != nullptr || p.ct.x != nullptr) return launch_tile_mt<MODE, true>(dtype, d, p, st);
  return launch_tile_mt<MODE, false>(dtype, d, p, st);
}

}  // namespace

// Raises up to DFS_MAX_PEERS counters once each (pointers by value: no device
// array to stage).
__global__ void peer_signal_one(unsigned long long* c0, unsigned long long* c1, unsigned long long* c2,
                                unsigned long long* c3, unsigned long long* c4, unsigned long long* c5,
                                unsigned long long* c6, unsigned long long* c7, int n) {
  unsigned long long* c[8] = {c0, c1, c2, c3, c4, c5, c6, c7};
  __threadfence_system();
  for (int k = 0; k < n && k < 8; ++k) atomicAdd_system(c[k], 1ull);
}

cudaError_t peer_signal(unsigned long long* const* cnt, int n, cudaStream_t st) {
  struct Ptrs {
    unsigned long long* c[DFS_MAX_PEERS];
  } ptrs{};
  for (int k = 0; k < n && k < DFS_MAX_PEERS; ++k) ptrs.c[k] = cnt[k];
  peer_signal_one<<<1, 1, 0, st>>>(ptrs.c[0], ptrs.c[1], ptrs.c[2], ptrs.c[3], ptrs.c[4], ptrs.c[5], ptrs.c[6],
                                   ptrs.c[7], n);
  return cudaGetLastError();
}

__global__ void extent_kernel(const float* mask, int N, int2* out) {
  __shared__ int red[16];
  int lo, hi;
  valid_extent<256>(mask, blockIdx.x, N, red, lo, hi);
  if (threadIdx.x == 0) out[blockIdx.x] = make_int2(lo, hi);
}

cudaError_t compute_extents(const float* mask, int B, int N, int2* out, cudaStream_t st) {
  if (mask == nullptr || B <= 0) return cudaSuccess;
  extent_kernel<<<B, 256, 0, st>>>(mask, N, out);
  return cudaGetLastError();
}

namespace {
// CTAs whose partials the split scratch of a (B, H, N) problem holds: every row
// block split kMaxSplit ways, capped at kSplitCtas
size_t split_ctas(int B, int H, int N) {
  const size_t all = static_cast<size_t>(B) * H * ((N + 127) / 128) * kMaxSplit;
  return all < static_cast<size_t>(kSplitCtas) ? all : static_cast<size_t>(kSplitCtas);
}
}  // namespace

size_t tile_split_bytes(int B, int H, int N) {
  return sizeof(float) * 384 * split_ctas(B, H, N) + sizeof(unsigned) * static_cast<size_t>(B) * H * ((N + 127) / 128);
}

cudaError_t tile_split_reset(float* split, int B, int H, int N, cudaStream_t st) {
  return cudaMemsetAsync(split + 384 * split_ctas(B, H, N), 0,
                         sizeof(unsigned) * static_cast<size_t>(B) * H * ((N + 127) / 128), st);
}

bool tile_path_ok(int dtype, int d, int N, const void* a, const void* b) {
  const bool shape = (d == 64 || (d == 32 && dtype == DFS_F32)) && N >= 128;  // boxes of 128 rows
  return shape && a != nullptr && b != nullptr &&
         ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u) == 0 && encode_fn() != nullptr;
}

cudaError_t launch_tile_pass(int mode, const TileArgs& t, cudaStream_t st) {
  if (t.row_end <= t.row_begin) return cudaSuccess;
  TileParams p{};
  const int box_inner = t.dtype == DFS_F32 ? 32 : 64;  // 128 bytes
  if (!make_tmap(&p.tmA, t.A, t.dtype, t.d, t.N, t.B * t.H, box_inner, 128) ||
      !make_tmap(&p.tmB, t.Bop, t.dtype, t.d, t.N, t.B * t.H, box_inner, 128))
    return cudaErrorInvalidValue;
  p.eps = t.eps;
  p.mask = t.mask;
  p.col_bias = t.col_bias;
  p.col_vec = t.col_vec;
  p.row_bias = t.row_bias;
  p.row_marg = t.row_marg;
  p.row_scale = t.row_scale;
  p.done = t.done;
  p.row_out = t.row_out;
  p.row_out_nat = t.row_out_nat;
  p.row_R = t.row_R;
  p.status = t.status;
  p.B = t.B;
  p.H = t.H;
  p.N = t.N;
  p.row_begin = t.row_begin;
  p.row_end = t.row_end;
  p.lam = t.lam;
  p.qk_scale = t.qk_scale;
  p.ct = t.ct;
  p.npeers = t.npeers;
  for (int k = 0; k < DFS_MAX_PEERS; ++k) {
    p.peer_out[k] = t.peer_out[k];
    p.peer_cnt[k] = t.peer_cnt[k];
  }
  p.wait_cnt = t.wait_cnt;
  p.wait_for = t.wait_for;
  p.extent = t.extent;
  // Column splits: a row block's column tiles shared by nsplit CTAs, which
  // publish (reference, sum, max) partials that the block's last CTA merges.
  // The count aims at about 3.5 waves of CTAs (two per SM) while each CTA keeps
  // enough tiles to amortise its set-up and the merge (16 of long rows, 4 of
  // short ones).  Measured on the N = 8192 half-update (B = 1, H = 16) over the
  // row ranges of 1/2/4/8 GPUs, the best counts were 1, 2, 4 and 2-4 (1024, 512,
  // 256 and 128 row blocks); this rule picks 1, 2, 4, 4.  DFS_TILE_SPLITS (1-8)
  // overrides it, within the scratch's capacity.
  p.nsplit = 1;
  if (t.split != nullptr) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long slots = 2L * sms;
    const long blocks = static_cast<long>(t.B) * t.H * ((t.row_end - t.row_begin + 127) / 128);
    const int tiles = (t.N + kTCols - 1) / kTCols;
    const long cap = static_cast<long>(split_ctas(t.B, t.H, t.N));
    const int min_tiles = tiles >= 32 ? 16 : 4;
    const int max_ns = static_cast<int>(min(static_cast<long>(max(1, min(kMaxSplit, tiles / min_tiles))),
                                            blocks > 0 ? max(1L, cap / blocks) : 1L));
    const long want = blocks > 0 ? (7 * slots) / (2 * blocks) : 1;
    p.nsplit = static_cast<int>(max(1L, min(want, static_cast<long>(max_ns))));
    if (const char* ov = getenv("DFS_TILE_SPLITS")) {
      const int n = atoi(ov);
      const long fit = blocks > 0 ? cap / blocks : 1;
      if (n >= 1) p.nsplit = static_cast<int>(max(1L, min(static_cast<long>(min(n, min(kMaxSplit, tiles))), fit)));
    }
    if (p.nsplit > 1) {
      p.part = t.split;
      p.counter = reinterpret_cast<unsigned*>(t.split + 384 * cap);
    }
  }
  if (mode == TL_LSE) return launch_tile_m<TL_LSE>(t.dtype, t.d, p, st);
  if (mode == TL_ROWSTATS) return launch_tile_m<TL_ROWSTATS>(t.dtype, t.d, p, st);
  return launch_tile_m<TL_MATVEC>(t.dtype, t.d, p, st);
}

}  // namespace dfs
