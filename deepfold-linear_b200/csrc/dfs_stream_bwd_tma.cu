// dfs_stream_bwd_tma.cu -- TMA-staged, warp-specialised tile passes of the
// streamed IFT backward for sm_100a (d = 32 or 64, N >= 128).
//
// The four passes that recompute both S = A B^T and dT = A2 B2^T tile by tile
// (the notation and formulas are those of dfs_stream_bwd.cu):
//
//   BT_ROW  rows i:     m_i, R_i, D_i = sum_j T_ij dT_ij               (online max)
//   BT_COL  columns j:  c_j = sum_i P_ij, g_v_j = sum_i T_ij (dT_ij - D_i),
//                       dV_j = sum_i T_ij dO_i                          (T tile -> MMA)
//   BT_DQ   rows i:     dQ_i = sum_j dS_ij K_j / (eps sqrt d)           (dS tile -> MMA)
//   BT_DK   columns j:  dK_j = sum_i dS_ij Q_i / (eps sqrt d)           (dS tile -> MMA)
//   BT_OUT  rows i:     O_i = sum_j T_ij V_j, x_centroid_i = sum_j T_ij x_j
//                       (the forward's transport output; S only, no dT)   (T tile -> MMA)
//
// dV is accumulated by the column-statistics pass, which already holds T_norm,
// so the last pass needs only dS.  All operands are fp32 copies made once per
// backward by the prep step (Q, K, V converted, dO as given, and the
// transposes Q^T, K^T, dO^T), so every MMA is kind::tf32 on K-major tiles that
// TMA writes directly in the 128-byte-swizzled layout the tensor core reads.
//
// One CTA per block of 128 rows and 20 warps:
//   warp 16     producer: the two row operands once (TMA, 128-row boxes); per
//               column tile of 64, the two column operands (64-row boxes) and
//               the tile's per-column vectors (fetched a tile ahead) into a
//               2-stage ring
//   warp 18     producer: the transposed accumulation operand, second 2-stage ring
//   warp 17     MMA: S and dT of each tile into one of two TMEM buffers (64 + 64
//               columns each)
//   warp 19     MMA: accumulation of each dS or T tile (shared memory) times the
//               transposed tile into a d-column TMEM accumulator, so that it
//               never waits behind the next tile's operands
//   warps 0-15  epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (thread =
//               row) and columns 16 (w / 4) .. + 15 of each tile, keeps the
//               running per-row reductions and writes its part of the dS / T
//               tile; the four column parts of each row are merged at the end.
#include "dfs_kernels.cuh"
#include "dfs_tma.cuh"

namespace dfs {

constexpr int kBEpiWarps = 16;
constexpr int kBTThreads = 32 * (kBEpiWarps + 4);  // 640
constexpr int kBProd = 16, kBMma = 17, kBProd3 = 18, kBMma3 = 19;
constexpr int kBTW = 64;  // columns per tile

enum BTileMode { BT_ROW = 0, BT_COL = 1, BT_DQ = 2, BT_DK = 3, BT_OUT = 4 };

struct BTileParams {
  CUtensorMap tmA, tmA2;  // row operands: fp32 (BH, N, d), boxes 32 x 128 rows
  CUtensorMap tmB, tmB2;  // column operands: fp32 (BH, N, d), boxes 32 x 64 rows
  CUtensorMap tmB3;       // accumulation operand: fp32 (BH, d, N) transposed, boxes 32 x d
  const float* eps;
  const float* mask;
  const float* tv[5];     // per-tile-column vectors (BH, N); bit k of pot_mask: -inf where masked
  int pot_mask;
  const float* xvec;      // per-tile-column 3-vectors (B or BH, N, 3), or null
  int xvec_per_head;
  const float* rv[5];     // per-row vectors (BH, N)
  const float* rxvec;     // per-row 3-vectors, or null
  int rxvec_per_head;
  float* out0;            // per-row results (ROW: m, R, D; COL: c, g_v)
  float* out1;
  float* out2;
  float* acc;             // (BH, N, d) accumulated result (COL: dV; DQ: dQ; DK: dK)
  float acc_scale;        // < 0: 1 / (eps_h sqrt d)
  int32_t* status;
  const int2* extent;     // (B) valid extents of the mask, or null (scan the mask)
  int B, H, N, row_begin, row_end;
  float qk_scale;         // 1/sqrt(d) of the cost
  CostTerms ct;           // optional position / geometry terms in this pass's orientation
  CostGradOut cg;         // DQ / DK / COL: shares of the shared-parameter gradients (null: none)
};

// Fixed point of the per-warp bin histograms: a warp's largest |dC| so far
// maps below 2^kHistBits, so the sum of its at most 32 rows x 16 columns x
// 1024 tiles (2^19) terms stays below 2^59.  A larger maximum later shifts the
// sums right (deterministically) to the new scale.
constexpr int kHistBits = 40;

template <int MODE, int D, bool TERMS = false>
struct BTileCfg {
  static constexpr bool kAcc = MODE != BT_ROW;
  static constexpr bool kDT = MODE != BT_OUT;        // second product dT = A2 B2^T
  static constexpr int G = D / 32;                   // 128-byte atoms across an fp32 row
  static constexpr uint32_t ATILE = 128u * D * 4;    // 128-row operand
  static constexpr uint32_t BTILE = 64u * D * 4;     // 64-row operand
  static constexpr uint32_t B3TILE = 64u * D * 4;    // d rows x 64 columns
  static constexpr int NS = 2, NS3 = 2;
  static constexpr int NVEC = TERMS ? 11 : 8;        // tv0..4, x 3-vector (+ the columns' coordinates)
  static constexpr uint32_t VEC = NVEC * kBTW * 4;
  static constexpr uint32_t OFF_A = 0;
  static constexpr uint32_t OFF_A2 = ATILE;
  static constexpr uint32_t OFF_B = (kDT ? 2 : 1) * ATILE;            // stage s: B, then B2
  static constexpr uint32_t SB = (kDT ? 2 : 1) * BTILE;               // bytes of a ring stage
  static constexpr uint32_t OFF_B3 = OFF_B + NS * SB;
  static constexpr uint32_t OFF_DS = OFF_B3 + (kAcc ? NS3 * B3TILE : 0u);   // 128 x 64 fp32
  // BT_OUT: T_norm enters the product as two tiles, its tf32 part and the fp32
  // remainder, so that O = T_norm V carries ~2^-20 relative error, not tf32's 2^-11
  static constexpr bool kSplitT = MODE == BT_OUT;
  static constexpr uint32_t OFF_DS2 = OFF_DS + (kAcc ? 128u * kBTW * 4 : 0u);
  static constexpr uint32_t OFF_VEC = OFF_DS2 + (kSplitT ? 128u * kBTW * 4 : 0u);
  static constexpr int NMRG = TERMS ? 5 : 3;                          // values merged per row (dx, dw, dr)
  static constexpr uint32_t OFF_MRG = OFF_VEC + NS * VEC;                // 3 parts x NMRG values x 128
  static constexpr uint32_t OFF_PW = OFF_MRG + 3 * NMRG * 128 * 4;       // TERMS: 69 scaled bin weights
  static constexpr bool kHist = TERMS && MODE == BT_DQ;
  static constexpr uint32_t OFF_HIST = OFF_PW + (TERMS ? 288u : 0u);     // DQ: 16 warps x 68 int64 bin sums
  static constexpr uint32_t OFF_HF = OFF_HIST + (kHist ? kBEpiWarps * 68u * 8u : 0u);  // DQ: 16 x 68 floats
  static constexpr uint32_t OFF_BAR = OFF_HF + (kHist ? kBEpiWarps * 68u * 4u : 0u);
  static constexpr uint32_t NBAR = 2 * NS + 2 * NS3 + 4 + 3;          // + sfull/sempty x2, ds x2, a
  static constexpr uint32_t OFF_SLOT = OFF_BAR + 8 * NBAR;
  static constexpr uint32_t OFF_RED = OFF_SLOT + 16;
  static constexpr uint32_t SMEM = OFF_RED + 4u * 2 * (kBTThreads / 32) + 1024;
  static_assert(SMEM <= 232448u, "shared memory");
};

template <int MODE, int D, bool TERMS>
__global__ void __launch_bounds__(kBTThreads, 1) btile_kernel(const __grid_constant__ BTileParams p) {
  using C = BTileCfg<MODE, D, TERMS>;
  constexpr bool kAcc = C::kAcc, kDT = C::kDT;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch (see launch_dependent)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the next pass may launch (it waits first)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sA = reinterpret_cast<float*>(base + C::OFF_A);
  float* sA2 = reinterpret_cast<float*>(base + C::OFF_A2);
  float* sDS = reinterpret_cast<float*>(base + C::OFF_DS);
  float* vecs = reinterpret_cast<float*>(base + C::OFF_VEC);
  float* mrg = reinterpret_cast<float*>(base + C::OFF_MRG);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::OFF_BAR);  // [NS] column operands + vectors staged
  uint64_t* empty = full + C::NS;                                      // [NS] consumed (MMA + epilogue)
  uint64_t* full3 = empty + C::NS;                                     // [NS3] transposed operand staged
  uint64_t* empty3 = full3 + C::NS3;                                   // [NS3] consumed (accumulation MMA)
  uint64_t* sfull = empty3 + C::NS3;                                   // [2] S, dT written
  uint64_t* sempty = sfull + 2;                                        // [2] S, dT read
  uint64_t* dsfull = sempty + 2;                                       // dS / T tile written
  uint64_t* dsempty = dsfull + 1;                                      // dS / T tile consumed
  uint64_t* afull = dsempty + 1;                                       // row operands staged
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + C::OFF_SLOT);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  const int prob = blockIdx.x / nrb, rb = blockIdx.x % nrb;
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const size_t bh = static_cast<size_t>(prob);
  const int r0 = p.row_begin + 128 * rb;
  // only the column tiles holding a valid point are visited (a masked column
  // contributes exactly nothing); a block without a valid row visits none
  int vlo, vhi;
  valid_extent<kBTThreads>(p.extent, p.mask, bb, N, reinterpret_cast<int*>(base + C::OFF_RED), vlo, vhi);
  const int rhi = min(min(r0 + 128, p.row_end), N);
  const bool live = max(r0, vlo) < min(rhi, vhi);
  if (!live) {
    // no valid row: the block's results are the masked-row zeros, written
    // before any set-up
    for (int i = tid; i < rhi - r0; i += kBTThreads) {
      const size_t o = bh * N + r0 + i;
      if constexpr (MODE == BT_ROW) {
        p.out0[o] = 0.0f;
        p.out1[o] = 0.0f;
        p.out2[o] = 0.0f;
      } else if constexpr (MODE == BT_COL) {
        p.out0[o] = 0.0f;
        p.out1[o] = 0.0f;
      } else if constexpr (MODE == BT_OUT) {
        if (p.out0 != nullptr) {
          p.out0[o * 3] = 0.0f;
          p.out0[o * 3 + 1] = 0.0f;
          p.out0[o * 3 + 2] = 0.0f;
        }
      }
      if constexpr (kAcc) {
        if (p.acc != nullptr) {
          float4* dst = reinterpret_cast<float4*>(p.acc + o * D);
#pragma unroll
          for (int q = 0; q < D / 4; ++q) dst[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      // this block's shares of the shared-parameter gradients (summed later)
      if (p.cg.dx != nullptr) {
        p.cg.dx[o * 3] = 0.0f;
        p.cg.dx[o * 3 + 1] = 0.0f;
        p.cg.dx[o * 3 + 2] = 0.0f;
      }
      if constexpr (MODE == BT_DQ) {
        if (p.cg.dw != nullptr) p.cg.dw[o] = 0.0f;
        if (p.cg.dr != nullptr) p.cg.dr[o] = 0.0f;
      }
    }
    if constexpr (C::kHist) {
      if (p.cg.dpos != nullptr && p.ct.bins != nullptr && tid < kBinCount) {
        const int nrb_all = (p.row_end - p.row_begin + 127) / 128;
        p.cg.dpos[(bh * nrb_all + rb) * kBinCount + tid] = 0.0f;
      }
    }
    return;
  }
  const int t_begin = live ? vlo / kBTW : 0;
  const int ntiles = live ? (vhi + kBTW - 1) / kBTW - t_begin : 0;

  if (warp == 0) tmem_alloc(tslot, 512);
  if (tid == 32 * kBProd) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 32);
      mbar_init(&empty[s], 1 + kBEpiWarps);
    }
    for (int s = 0; s < C::NS3; ++s) {
      mbar_init(&full3[s], 1);
      mbar_init(&empty3[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], kBEpiWarps);
    }
    mbar_init(dsfull, kBEpiWarps);
    mbar_init(dsempty, 1);
    mbar_init(afull, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  // TMEM columns: S [128 b, 128 b + 64), dT [128 b + 64, 128 b + 128), accumulator [256, 256 + d)
  const uint32_t t_acc = tbase + 256;
  int err = 0;

  if (warp == kBProd) {
    // ------------------------------------------------------------ producer: row operands, ring 1
    if (ntiles > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(smem_u32(afull), (kDT ? 2 : 1) * C::ATILE);
#pragma unroll
        for (int g = 0; g < C::G; ++g) {
          tma_load_3d(smem_u32(sA) + g * 128u * 128u, &p.tmA, 32 * g, r0, prob, smem_u32(afull));
          if constexpr (kDT)
            tma_load_3d(smem_u32(sA2) + g * 128u * 128u, &p.tmA2, 32 * g, r0, prob, smem_u32(afull));
        }
      }
      // the per-column vectors of a tile (2 columns per lane), fetched one tile
      // ahead so that their global latency overlaps the wait for a free stage
      float pv[2][C::NVEC];
      auto fetch = [&](int u) {
        const int c0 = (t_begin + u) * kBTW;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = c0 + lane + 32 * h;
          const bool cin = j < N;
          const bool cok = cin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
#pragma unroll
          for (int k = 0; k < 5; ++k) {
            float v = (cin && p.tv[k] != nullptr) ? p.tv[k][bh * N + j] : 0.0f;
            pv[h][k] = (((p.pot_mask >> k) & 1) && !cok) ? -INFINITY : v;
          }
#pragma unroll
          for (int x = 0; x < 3; ++x)
            pv[h][5 + x] = (p.xvec != nullptr && cin)
                               ? p.xvec[((p.xvec_per_head ? bh : static_cast<size_t>(bb)) * N + j) * 3 + x]
                               : 0.0f;
          if constexpr (TERMS) {
#pragma unroll
            for (int x = 0; x < 3; ++x)
              pv[h][8 + x] = (p.ct.x != nullptr && cin) ? p.ct.x[(static_cast<size_t>(bb) * N + j) * 3 + x] : 0.0f;
          }
        }
      };
      fetch(0);
#pragma unroll 1
      for (int u = 0; u < ntiles; ++u) {
        const int s = u % C::NS;
        const int c0 = (t_begin + u) * kBTW;
        if (u >= C::NS && !mbar_wait(&empty[s], ((u / C::NS) - 1) & 1)) err = 1;
        if (lane == 0) {
          const uint32_t dst = smem_u32(base + C::OFF_B + s * C::SB);
          mbar_expect_tx(smem_u32(&full[s]), C::SB);
#pragma unroll
          for (int g = 0; g < C::G; ++g) {
            tma_load_3d(dst + g * 64u * 128u, &p.tmB, 32 * g, c0, prob, smem_u32(&full[s]));
            if constexpr (kDT)
              tma_load_3d(dst + C::BTILE + g * 64u * 128u, &p.tmB2, 32 * g, c0, prob, smem_u32(&full[s]));
          }
        }
        float* vb = vecs + s * (C::VEC / 4);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int k = 0; k < C::NVEC; ++k) vb[k * kBTW + lane + 32 * h] = pv[h][k];
        mbar_arrive(&full[s]);
        if (u + 1 < ntiles) fetch(u + 1);
      }
      // every MMA completion has arrived before the CTA exits
      for (int u = max(0, ntiles - C::NS); u < ntiles; ++u)
        if (!mbar_wait(&empty[u % C::NS], (u / C::NS) & 1)) err = 1;
    }
  } else if (warp == kBProd3) {
    // ------------------------------------------------------------ producer: transposed operand ring
    if (kAcc && ntiles > 0) {
#pragma unroll 1
      for (int u = 0; u < ntiles; ++u) {
        const int s3 = u % C::NS3, c0 = (t_begin + u) * kBTW;
        if (u >= C::NS3 && !mbar_wait(&empty3[s3], ((u / C::NS3) - 1) & 1)) err = 1;
        if (lane == 0) {
          const uint32_t dst = smem_u32(base + C::OFF_B3 + s3 * C::B3TILE);
          mbar_arrive_expect_tx(smem_u32(&full3[s3]), C::B3TILE);
          // two boxes of 32 columns (K) x d rows: the K-major layout of the (d x 64) operand
          tma_load_3d(dst, &p.tmB3, c0, 0, prob, smem_u32(&full3[s3]));
          tma_load_3d(dst + D * 128u, &p.tmB3, c0 + 32, 0, prob, smem_u32(&full3[s3]));
        }
        __syncwarp();
      }
      for (int u = max(0, ntiles - C::NS3); u < ntiles; ++u)
        if (!mbar_wait(&empty3[u % C::NS3], (u / C::NS3) & 1)) err = 1;
    }
  } else if (warp == kBMma) {
    // ------------------------------------------------------------ MMA: S and dT
    if (ntiles > 0) {
      if (!mbar_wait(afull, 0)) err = 1;
#pragma unroll 1
      for (int u = 0; u < ntiles; ++u) {
        const int s = u % C::NS, b = u & 1;
        if (!mbar_wait(&full[s], (u / C::NS) & 1)) err = 1;
        if (u >= 2 && !mbar_wait(&sempty[b], ((u >> 1) - 1) & 1)) err = 1;
        tc_fence_after();
        if (lane == 0) {
          const float* sB = reinterpret_cast<const float*>(base + C::OFF_B + s * C::SB);
          issue_mma<128, kBTW, D>(tbase + 128 * b, sA, sB, false);
          if constexpr (kDT) issue_mma<128, kBTW, D>(tbase + 128 * b + kBTW, sA2, sB + C::BTILE / 4, false);
          mma_commit(&sfull[b]);
          mma_commit(&empty[s]);
        }
        __syncwarp();
      }
    }
  } else if (warp == kBMma3) {
    // ------------------------------------------------------------ MMA: accumulation of the dS / T tiles
    if (kAcc && ntiles > 0) {
#pragma unroll 1
      for (int v = 0; v < ntiles; ++v) {
        const int s3 = v % C::NS3;
        if (!mbar_wait(dsfull, v & 1)) err = 1;
        if (!mbar_wait(&full3[s3], (v / C::NS3) & 1)) err = 1;
        tc_fence_after();
        if (lane == 0) {
          const float* sB3 = reinterpret_cast<const float*>(base + C::OFF_B3 + s3 * C::B3TILE);
          issue_mma<128, D, kBTW>(t_acc, sDS, sB3, v > 0);
          if constexpr (C::kSplitT)
            issue_mma<128, D, kBTW>(t_acc, reinterpret_cast<const float*>(base + C::OFF_DS2), sB3, true);
          mma_commit(dsempty);
          mma_commit(&empty3[s3]);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3, part = warp >> 2;
    const int lrow = 32 * quad + lane, row = r0 + lrow;
    const bool rin = row < p.row_end && row < N;
    const bool rok = rin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + row] != 0.0f);
    const float eps_h = p.eps[hh];
    const float scale = kLog2e * p.qk_scale / eps_h;
    float rv[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) rv[k] = (rin && p.rv[k] != nullptr) ? p.rv[k][bh * N + row] : 0.0f;
    const bool has_x = p.xvec != nullptr && p.rxvec != nullptr;
    float rx[3] = {0.0f, 0.0f, 0.0f};
    if (has_x && rin) {
      const size_t o = (p.rxvec_per_head ? bh : static_cast<size_t>(bb)) * N + row;
#pragma unroll
      for (int c = 0; c < 3; ++c) rx[c] = p.rxvec[o * 3 + c];
    }
    const uint32_t tlane = static_cast<uint32_t>(32 * quad) << 16;
    // optional cost terms: bin weights scaled to -log2(e)/eps (entry 68: 0), this
    // row's coordinates; gradient shares of the shared cost parameters
    float* pws = reinterpret_cast<float*>(base + C::OFF_PW);
    const bool use_bins = TERMS && p.ct.bins != nullptr, use_geo = TERMS && p.ct.x != nullptr;
    float xi[3] = {0.0f, 0.0f, 0.0f}, wS = 0.0f, w_h = 0.0f, r_h = 1.0f;
    const uint8_t* brow = nullptr;
    // this row's dx, dw and dr shares (this part); gdr sums dC dist / (r_h + dist)^2
    float gdx[3] = {0.0f, 0.0f, 0.0f}, gdw = 0.0f, gdr = 0.0f;
    const bool want_geo_grad = TERMS && use_geo && (p.cg.dx != nullptr || p.cg.dw != nullptr || p.cg.dr != nullptr) &&
                               (MODE == BT_DQ || MODE == BT_DK);
    const bool want_hist = C::kHist && use_bins && p.cg.dpos != nullptr;
    const bool want_cent_grad = MODE == BT_COL && p.cg.dx != nullptr && p.xvec != nullptr;
    const float inv_eps = 1.0f / eps_h;
    unsigned long long* whist = reinterpret_cast<unsigned long long*>(base + C::OFF_HIST) + warp * 68;
    int e_cur = -1000;  // exponent of this warp's histogram scale (-1000: nothing added yet)
    if constexpr (TERMS) {
      const float nsc = -kLog2e * inv_eps;
      if (use_bins && tid <= kBinCount) pws[tid] = tid < kBinCount ? p.ct.pos_weight[hh * kBinCount + tid] * nsc : 0.0f;
      if (use_geo) {
        w_h = p.ct.w_dist[hh];
        r_h = geo_scale(p.ct, hh);
        wS = w_h * nsc;
        if (rin) {
#pragma unroll
          for (int c = 0; c < 3; ++c) xi[c] = p.ct.x[(static_cast<size_t>(bb) * N + row) * 3 + c];
        }
      }
      if (use_bins && rin) brow = p.ct.bins + (static_cast<size_t>(bb) * N + row) * p.ct.bin_stride;
      if (want_hist)
        for (int b2 = lane; b2 < 68; b2 += 32) whist[b2] = 0ull;
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kBEpiWarps) : "memory");  // pws written
    }
    // running results of this column part (BT_OUT: the three x_centroid sums)
    float m = MODE == BT_OUT ? 0.0f : kNeg, s0 = 0.0f, s1 = 0.0f;
    const float out_fm = rv[0] - rv[1];              // BT_OUT: f_i - m_i
    const float out_inv = 1.0f / (rv[2] + 1e-6f);    // BT_OUT: 1 / (R_i + 1e-6)
    const bool col_x = p.xvec != nullptr;
#pragma unroll 1
    for (int u = 0; u < ntiles; ++u) {
      const int s = u % C::NS, b = u & 1;
      uint4 bq = make_uint4(0u, 0u, 0u, 0u);  // this row's 16 bins of the tile's part (loaded ahead)
      if (TERMS && brow != nullptr) bq = __ldg(reinterpret_cast<const uint4*>(brow + (t_begin + u) * kBTW + 16 * part));
      if (!mbar_wait(&full[s], (u / C::NS) & 1)) err = 1;  // vectors
      if (!mbar_wait(&sfull[b], (u >> 1) & 1)) err = 1;
      tc_fence_after();
      float sv[16], dv[16];
      tmem_ld16(tbase + tlane + 128 * b + 16 * part, sv);
      if constexpr (kDT) tmem_ld16(tbase + tlane + 128 * b + kBTW + 16 * part, dv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[b]);
      const float* vb = vecs + s * (C::VEC / 4) + 16 * part;
      // the cost terms of this row's 16 columns (log2 units), 0 without terms
      float tm[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) tm[k] = 0.0f;
      if constexpr (TERMS) {
        const uint32_t bw[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          float t = 0.0f;
          if (use_bins) t = pws[(bw[k >> 2] >> (8 * (k & 3))) & 0xffu];
          if (use_geo) {
            const float d0 = xi[0] - vb[8 * kBTW + k], d1 = xi[1] - vb[9 * kBTW + k], d2 = xi[2] - vb[10 * kBTW + k];
            const float dist = sqrtf(fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, 1e-8f))));
            t = fmaf(wS, __fdividef(dist, r_h + dist), t);
          }
          tm[k] = t;
        }
      }
      // adds this column's term (compile-time nothing without TERMS)
      auto with_term = [&](float x, int k) {
        if constexpr (TERMS) return x + tm[k];
        else return x;
      };
      float dt[16];
      if constexpr (kDT) {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          dt[k] = dv[k];
          if (has_x) dt[k] += rx[0] * vb[5 * kBTW + k] + rx[1] * vb[6 * kBTW + k] + rx[2] * vb[7 * kBTW + k];
        }
      }
      float out[16];  // dS or T values of this row's 16 columns (accumulating modes)
      if constexpr (MODE == BT_ROW) {
        // rv0 = f_i; tv0 = g_j
#pragma unroll
        for (int k = 0; k < 16; ++k) sv[k] = with_term(fmaf(sv[k], scale, vb[k] + rv[0]), k);
        float mx[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) mx[q] = fmaxf(fmaxf(sv[4 * q], sv[4 * q + 1]), fmaxf(sv[4 * q + 2], sv[4 * q + 3]));
        const float mn = fmaxf(m, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
        const float resc = ex2(m - mn);
        float r[2] = {s0 * resc, 0.0f}, pd[2] = {s1 * resc, 0.0f};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float e = ex2(sv[k] - mn);
          r[k & 1] += e;
          pd[k & 1] = fmaf(e, dt[k], pd[k & 1]);
        }
        m = mn;
        s0 = r[0] + r[1];
        s1 = pd[0] + pd[1];
      } else if constexpr (MODE == BT_COL) {
        // thread = column j: rv0 = g_j; tile i: tv0 = f, tv1 = f - m, tv2 = 1/(R+1e-6), tv3 = D
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float sc = with_term(fmaf(sv[k], scale, rv[0]), k);
          const float P = ex2(sc + vb[k]);
          const float T = ex2(sc + vb[kBTW + k]) * vb[2 * kBTW + k];
          s0 += P;
          s1 = fmaf(T, dt[k] - vb[3 * kBTW + k], s1);
          out[k] = rok ? T : 0.0f;
        }
        if (want_cent_grad) {  // centroid share: dx_j += sum_i T_ij dxc_i (dxc staged as the tile's 3-vectors)
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            gdx[0] = fmaf(out[k], vb[5 * kBTW + k], gdx[0]);
            gdx[1] = fmaf(out[k], vb[6 * kBTW + k], gdx[1]);
            gdx[2] = fmaf(out[k], vb[7 * kBTW + k], gdx[2]);
          }
        }
      } else if constexpr (MODE == BT_DQ) {
        // rv0 = f, rv1 = f - m, rv2 = 1/(R+1e-6), rv3 = D, rv4 = w1; tv0 = g, tv1 = w2
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float sc = with_term(fmaf(sv[k], scale, vb[k]), k);
          const float P = ex2(sc + rv[0]);
          const float T = ex2(sc + rv[1]) * rv[2];
          out[k] = rok ? T * (dt[k] - rv[3]) - P * (rv[4] + vb[kBTW + k]) : 0.0f;
        }
      } else if constexpr (MODE == BT_OUT) {
        // rv0 = f, rv1 = m, rv2 = R (rows); tv0 = g, tv 5..7 = x_j
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float T = rok ? ex2(with_term(fmaf(sv[k], scale, vb[k]) + out_fm, k)) * out_inv : 0.0f;
          out[k] = T;
          if (col_x) {
            m = fmaf(T, vb[5 * kBTW + k], m);
            s0 = fmaf(T, vb[6 * kBTW + k], s0);
            s1 = fmaf(T, vb[7 * kBTW + k], s1);
          }
        }
      } else {
        // thread = column j: rv0 = g_j, rv1 = w2_j; tile i: tv0 = f, tv1 = f - m, tv2 = 1/(R+1e-6),
        // tv3 = D, tv4 = w1
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float sc = with_term(fmaf(sv[k], scale, rv[0]), k);
          const float P = ex2(sc + vb[k]);
          const float T = ex2(sc + vb[kBTW + k]) * vb[2 * kBTW + k];
          out[k] = rok ? T * (dt[k] - vb[3 * kBTW + k]) - P * (vb[4 * kBTW + k] + rv[1]) : 0.0f;
        }
      }
      if constexpr (TERMS && (MODE == BT_DQ || MODE == BT_DK)) {
        // gradient shares from dS (natural units; dC = -dS / eps): geometry per row
        // (DQ: rows i, columns j; DK: rows j, columns i -- dist and c are symmetric)
        if (want_geo_grad) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float dC = -out[k] * inv_eps;
            const float d0 = xi[0] - vb[8 * kBTW + k], d1 = xi[1] - vb[9 * kBTW + k], d2 = xi[2] - vb[10 * kBTW + k];
            const float dist = sqrtf(fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, 1e-8f))));
            const float rd = __fdividef(1.0f, r_h + dist);
            if (MODE == BT_DQ) {
              const float t = dC * dist * rd;
              gdw += t;
              gdr = fmaf(t, rd, gdr);
            }
            const float cf = __fdividef(dC * w_h * r_h * rd * rd, dist);
            gdx[0] = fmaf(cf, d0, gdx[0]);
            gdx[1] = fmaf(cf, d1, gdx[1]);
            gdx[2] = fmaf(cf, d2, gdx[2]);
          }
        }
        if constexpr (C::kHist) {
          if (want_hist) {
            float amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(out[k]));
            amax = warp_max(amax * inv_eps);
            if (amax > 0.0f) {
              int e = 0;
              frexpf(amax, &e);  // amax < 2^e, the same in every lane
              if (e > e_cur) {
                if (e_cur > -1000) {
                  const int sh = min(e - e_cur, 63);
                  for (int b2 = lane; b2 < 68; b2 += 32)
                    whist[b2] = static_cast<unsigned long long>(static_cast<long long>(whist[b2]) >> sh);
                }
                e_cur = e;
                __syncwarp();
              }
              const float hsc = ldexpf(1.0f, kHistBits - e_cur);
              const uint32_t bw[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const unsigned bin = (bw[k >> 2] >> (8 * (k & 3))) & 0xffu;
                const long long q = __float2ll_rn(-out[k] * inv_eps * hsc);
                if (bin < static_cast<unsigned>(kBinCount) && q != 0)
                  atomicAdd(&whist[bin], static_cast<unsigned long long>(q));
              }
              __syncwarp();
            }
          }
        }
      }
      if constexpr (kAcc) {
        if (u >= 1 && !mbar_wait(dsempty, (u - 1) & 1)) err = 1;  // accumulation MMA of tile u-1 done
        if constexpr (C::kSplitT) {
          // tf32 part (the 10 mantissa bits the tensor core reads) and the remainder
          float* sDS2 = reinterpret_cast<float*>(base + C::OFF_DS2);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              hi[e] = __uint_as_float(__float_as_uint(out[4 * q + e]) & 0xFFFFE000u);
              lo[e] = out[4 * q + e] - hi[e];
            }
            const uint32_t o4 = sw_off(lrow, 16 * part + 4 * q, 128) >> 2;
            *reinterpret_cast<float4*>(sDS + o4) = make_float4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<float4*>(sDS2 + o4) = make_float4(lo[0], lo[1], lo[2], lo[3]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float4*>(sDS + (sw_off(lrow, 16 * part + 4 * q, 128) >> 2)) =
                make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(dsfull);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // ---- per-row results: merge the four column parts
    if constexpr (MODE == BT_ROW || MODE == BT_COL || MODE == BT_OUT) {
      if (part > 0) {
        float* mp = mrg + (part - 1) * C::NMRG * 128;
        mp[lrow] = m;
        mp[128 + lrow] = s0;
        mp[256 + lrow] = s1;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kBEpiWarps) : "memory");
      if (part == 0 && rin) {
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          const float* mp = mrg + q * C::NMRG * 128;
          if constexpr (MODE == BT_ROW) {
            const float m2 = mp[lrow], mm = fmaxf(m, m2);
            const float a = ex2(m - mm), c = ex2(m2 - mm);
            s0 = s0 * a + mp[128 + lrow] * c;
            s1 = s1 * a + mp[256 + lrow] * c;
            m = mm;
          } else {
            if constexpr (MODE == BT_OUT) m += mp[lrow];
            s0 += mp[128 + lrow];
            s1 += mp[256 + lrow];
          }
        }
        const size_t o = bh * N + row;
        if constexpr (MODE == BT_OUT) {
          if (p.out0 != nullptr) {  // x_centroid
            p.out0[o * 3] = rok ? m : 0.0f;
            p.out0[o * 3 + 1] = rok ? s0 : 0.0f;
            p.out0[o * 3 + 2] = rok ? s1 : 0.0f;
          }
        } else if constexpr (MODE == BT_ROW) {
          p.out0[o] = rok ? m : 0.0f;                 // m
          p.out1[o] = rok ? s0 : 0.0f;                // R
          p.out2[o] = rok ? s1 / (s0 + 1e-6f) : 0.0f;  // D
        } else {
          p.out0[o] = rok ? s0 : 0.0f;  // c
          p.out1[o] = rok ? s1 : 0.0f;  // g_v
        }
      }
    }
    // ---- shares of the shared-parameter gradients: merge the four column parts per row
    if constexpr (TERMS || MODE == BT_COL) {
      if (p.cg.dx != nullptr || p.cg.dw != nullptr || p.cg.dr != nullptr) {
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kBEpiWarps) : "memory");  // mrg free again
        constexpr int NV = C::NMRG;
        if (part > 0) {
          float* mp = mrg + (part - 1) * C::NMRG * 128;
          mp[lrow] = gdx[0];
          mp[128 + lrow] = gdx[1];
          mp[256 + lrow] = gdx[2];
          if constexpr (NV == 5) {
            mp[384 + lrow] = gdw;
            mp[512 + lrow] = gdr;
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kBEpiWarps) : "memory");
        if (part == 0 && rin) {
#pragma unroll
          for (int q = 0; q < 3; ++q) {
            const float* mp = mrg + q * C::NMRG * 128;
            gdx[0] += mp[lrow];
            gdx[1] += mp[128 + lrow];
            gdx[2] += mp[256 + lrow];
            if constexpr (NV == 5) {
              gdw += mp[384 + lrow];
              gdr += mp[512 + lrow];
            }
          }
          const size_t o = bh * N + row;
          if (p.cg.dx != nullptr) {
            p.cg.dx[o * 3] = rok ? gdx[0] : 0.0f;
            p.cg.dx[o * 3 + 1] = rok ? gdx[1] : 0.0f;
            p.cg.dx[o * 3 + 2] = rok ? gdx[2] : 0.0f;
          }
          if (MODE == BT_DQ && p.cg.dw != nullptr) p.cg.dw[o] = rok ? gdw : 0.0f;
          if (MODE == BT_DQ && p.cg.dr != nullptr) p.cg.dr[o] = rok ? -w_h * gdr : 0.0f;
        }
      }
    }
    if constexpr (C::kHist) {
      // the bin sums: each warp's histogram to floats, then the 16 warps in order
      if (want_hist) {
        float* hf = reinterpret_cast<float*>(base + C::OFF_HF);
        const float back = e_cur > -1000 ? ldexpf(1.0f, e_cur - kHistBits) : 0.0f;
        for (int b2 = lane; b2 < 68; b2 += 32)
          hf[warp * 68 + b2] = static_cast<float>(static_cast<double>(static_cast<long long>(whist[b2])) * back);
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kBEpiWarps) : "memory");
        if (tid < kBinCount) {
          float t = 0.0f;
          for (int w = 0; w < kBEpiWarps; ++w) t += hf[w * 68 + tid];
          const int nrb_all = (p.row_end - p.row_begin + 127) / 128;
          p.cg.dpos[(bh * nrb_all + rb) * kBinCount + tid] = t;
        }
      }
    }
    // ---- accumulated result: part p of each quadrant writes columns [16 p, 16 p + 16)
    if constexpr (kAcc) {
      if (ntiles > 0 && !mbar_wait(dsempty, (ntiles - 1) & 1)) err = 1;  // last accumulation MMA done
      tc_fence_after();
      float sc = p.acc_scale;
      if (sc < 0.0f) sc = p.qk_scale / eps_h;
      if (16 * part < D) {
        float v[16];
        tmem_ld16(t_acc + tlane + 16 * part, v);
        if (rin && p.acc != nullptr) {
          float4* dst = reinterpret_cast<float4*>(p.acc + (bh * N + row) * D + 16 * part);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = rok ? make_float4(v[4 * q] * sc, v[4 * q + 1] * sc, v[4 * q + 2] * sc, v[4 * q + 3] * sc)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  }
  if (err && p.status != nullptr) atomicOr(p.status, DFS_ERR_DEVICE_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

// fp32 copies for the tile passes: row-major (BH, N, d) and transposed (BH, d, N),
// either may be null.  One block per 32 rows of one problem.
__global__ void bt_prep_kernel(const void* src, int dtype, float* row_out, float* t_out, int N, int d) {
  __shared__ float tile[32][65];
  const int bh = blockIdx.y, n0 = blockIdx.x * 32;
  const size_t base = static_cast<size_t>(bh) * N * d;
  for (int e = threadIdx.x; e < 32 * d; e += blockDim.x) {
    const int r = e / d, c = e % d, n = n0 + r;
    float v = 0.0f;
    if (n < N) {
      v = load_f32(src, base + static_cast<size_t>(n) * d + c, dtype);
      if (row_out != nullptr) row_out[base + static_cast<size_t>(n) * d + c] = v;
    }
    tile[r][c] = v;
  }
  __syncthreads();
  if (t_out == nullptr) return;
  for (int e = threadIdx.x; e < 32 * d; e += blockDim.x) {
    const int c = e / 32, r = e % 32, n = n0 + r;
    if (n < N) t_out[base + static_cast<size_t>(c) * N + n] = tile[r][c];
  }
}

// ---------------------------------------------------------------- host side
namespace {

template <int MODE, int D, bool TERMS>
cudaError_t launch_bt_md(const BTileParams& p, cudaStream_t st) {
  using C = BTileCfg<MODE, D, TERMS>;
  auto kern = btile_kernel<MODE, D, TERMS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  return launch_dependent(kern, dim3(p.B * p.H * nrb), dim3(kBTThreads), C::SMEM, st, p);
}

template <int MODE>
cudaError_t launch_bt_m(int d, const BTileParams& p, cudaStream_t st) {
  if (p.ct.bins != nullptr || p.ct.x != nullptr)
    return d == 64 ? launch_bt_md<MODE, 64, true>(p, st) : launch_bt_md<MODE, 32, true>(p, st);
  return d == 64 ? launch_bt_md<MODE, 64, false>(p, st) : launch_bt_md<MODE, 32, false>(p, st);
}

}  // namespace

size_t bt_copies_bytes(int B, int H, int N, int d) {
  return 7 * sizeof(float) * static_cast<size_t>(B) * H * N * d + 256;
}

bool bt_path_ok(int d, int N, const void* ws) {
  // N % 4: the transposed copies' rows (N floats) must be a multiple of 16 bytes for TMA
  return (d == 32 || d == 64) && N >= 128 && N % 4 == 0 && ws != nullptr && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0 &&
         tmap_available();
}

BtCopies bt_copies(float* region, int B, int H, int N, int d) {
  float* r = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(region) + 255) & ~uintptr_t(255));
  const size_t n = static_cast<size_t>(B) * H * N * d;
  BtCopies c;
  c.Qf = r;
  c.Kf = r + n;
  c.Vf = r + 2 * n;
  c.dOf = r + 3 * n;
  c.QT = r + 4 * n;
  c.KT = r + 5 * n;
  c.dOT = r + 6 * n;
  return c;
}

cudaError_t bt_convert(const void* src, int dtype, float* row_out, float* t_out, int BH, int N, int d,
                       cudaStream_t st) {
  bt_prep_kernel<<<dim3((N + 31) / 32, BH), 256, 0, st>>>(src, dtype, row_out, t_out, N, d);
  return cudaGetLastError();
}

cudaError_t bt_prep(const BwdParams& bp, const BtCopies& c, cudaStream_t st) {
  const dim3 grid((bp.N + 31) / 32, bp.B * bp.H);
  bt_prep_kernel<<<grid, 256, 0, st>>>(bp.Q, bp.in_dtype, c.Qf, c.QT, bp.N, bp.d);
  bt_prep_kernel<<<grid, 256, 0, st>>>(bp.K, bp.in_dtype, c.Kf, c.KT, bp.N, bp.d);
  bt_prep_kernel<<<grid, 256, 0, st>>>(bp.V, bp.in_dtype, c.Vf, nullptr, bp.N, bp.d);
  bt_prep_kernel<<<grid, 256, 0, st>>>(bp.dO, DFS_F32, c.dOf, c.dOT, bp.N, bp.d);
  return cudaGetLastError();
}

cudaError_t launch_bt_pass(int mode, const BtArgs& a, cudaStream_t st) {
  if (a.row_end <= a.row_begin) return cudaSuccess;
  BTileParams p{};
  const int BH = a.B * a.H;
  const bool dt = mode != BT_OUT;
  const bool ok = make_tmap(&p.tmA, a.A, DFS_F32, a.d, a.N, BH, 32, 128) &&
                  (!dt || make_tmap(&p.tmA2, a.A2, DFS_F32, a.d, a.N, BH, 32, 128)) &&
                  make_tmap(&p.tmB, a.Bop, DFS_F32, a.d, a.N, BH, 32, kBTW) &&
                  (!dt || make_tmap(&p.tmB2, a.B2, DFS_F32, a.d, a.N, BH, 32, kBTW)) &&
                  (mode == BT_ROW || make_tmap(&p.tmB3, a.B3, DFS_F32, a.N, a.d, BH, 32, a.d));
  if (!ok) return cudaErrorInvalidValue;
  p.eps = a.eps;
  p.qk_scale = a.qk_scale;
  p.mask = a.mask;
  for (int k = 0; k < 5; ++k) {
    p.tv[k] = a.tv[k];
    p.rv[k] = a.rv[k];
  }
  p.pot_mask = a.pot_mask;
  p.xvec = a.xvec;
  p.xvec_per_head = a.xvec_per_head;
  p.rxvec = a.rxvec;
  p.rxvec_per_head = a.rxvec_per_head;
  p.out0 = a.out0;
  p.out1 = a.out1;
  p.out2 = a.out2;
  p.acc = a.acc;
  p.acc_scale = a.acc_scale;
  p.status = a.status;
  p.extent = a.extent;
  p.B = a.B;
  p.H = a.H;
  p.N = a.N;
  p.row_begin = a.row_begin;
  p.row_end = a.row_end;
  p.ct = a.ct;
  p.cg = a.cg;
  switch (mode) {
    case BT_ROW: return launch_bt_m<BT_ROW>(a.d, p, st);
    case BT_COL: return launch_bt_m<BT_COL>(a.d, p, st);
    case BT_DQ: return launch_bt_m<BT_DQ>(a.d, p, st);
    case BT_DK: return launch_bt_m<BT_DK>(a.d, p, st);
    default: return launch_bt_m<BT_OUT>(a.d, p, st);
  }
}

}  // namespace dfs
