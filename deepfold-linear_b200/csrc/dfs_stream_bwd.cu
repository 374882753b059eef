// dfs_stream_bwd.cu -- streamed IFT backward for sm_100a (any N, d = 32 or 64).
//
// The same gradient as the cluster-resident backward (csrc/dfs_bwd.cu): with
// the forward's fixed point (f, g), P = exp2(x), x = S' + f_i + g_j (log2 units),
// T_norm = exp2(x - m_i) / (R_i + 1e-6), dT = dO V^T (+ dxc x^T),
// D_i = sum_j T_norm dT, E = T_norm o (dT - D), the IFT system is solved on the
// Schur complement of its row block by conjugate gradient, and
// dS = E - P o (w1 (+) w2) gives dQ = dS K and dK = dS^T Q (scaled by
// 1/(eps sqrt d)), dV = T_norm^T dO.  Nothing of size N x N is stored: every
// pass below recomputes its tiles of S (and of dT) with tcgen05 MMAs.
//
// Tile passes (one CTA = 128 rows of one problem, one thread per row = TMEM
// lane, column tiles of 64):
//   SB_ROW     rows:    m, R, D                    (S, dT tiles)
//   SB_COL     columns: c = P^T 1, g_v = E^T 1      (S^T, dT^T tiles; roles swapped)
//   SB_MATVEC  y_i = scale_i sum_j P_ij v_j        (either orientation)
//   SB_DQ      rows:    dQ += dS K                  (dS tile -> third MMA)
//   SB_DKV     columns: dK += dS^T Q, dV += T_norm^T dO
// Per-problem vector steps (setup of the CG system, one CG iteration, the
// null-space shift and marginal gradients) run as one CTA per problem.
#include <mutex>
#include <type_traits>

#include "dfs_tma.cuh"

namespace dfs {

constexpr int kBThreads = 128;
constexpr int kBTile = 64;

enum StreamBwdMode { SB_ROW = 0, SB_COL = 1, SB_MATVEC = 2, SB_DQ = 3, SB_DKV = 4 };

struct StreamBwdParams {
  // operands, each (BH, N, d) row-major, of type dtype unless marked fp32
  const void* Aop; int a_f32;     // rows of S = A B^T
  const void* Bop; int b_f32;     // columns
  const void* A2op; int a2_f32;   // rows of the second product (dT)
  const void* B2op; int b2_f32;   // columns of the second product
  const void* B3op; int b3_f32;   // SB_DQ / SB_DKV: first accumulation MMA, stored transposed
  const void* B4op; int b4_f32;   // SB_DKV: second accumulation MMA, stored transposed
  int dtype;
  const float* eps;
  const float* mask;              // (B, N) or null
  const float* tv[8];             // per-column-position vectors (BH, N), see each mode
  const float* xvec;              // (B, N, 3) per-position 3-vectors (x_res or dxc), or null
  int xvec_per_head;              // xvec is (BH, N, 3) (dxc) rather than (B, N, 3) (x_res)
  const float* rv[8];             // per-row vectors (BH, N)
  const float* rxvec;             // (B or BH, N, 3) per-row 3-vectors, or null
  int rxvec_per_head;
  const int32_t* done;            // (BH) skip the problem when nonzero (converged CG), or null
  float* out0;                    // (BH, N) results per row
  float* out1;
  float* out2;
  float* acc0;                    // (BH, N, d) accumulated results
  float* acc1;
  float acc_scale0, acc_scale1;
  int B, H, N;
  int row_begin, row_end;
  float qk_scale;                 // 1/sqrt(d) of the cost
};

template <int MODE, int D>
struct SBCfg {
  static constexpr bool kDT = MODE == SB_ROW || MODE == SB_COL || MODE == SB_DQ || MODE == SB_DKV;
  static constexpr bool kAcc = MODE == SB_DQ || MODE == SB_DKV;
  static constexpr bool kTwo = MODE == SB_DKV;
  static constexpr int TW = kBTile;
  static constexpr uint32_t OFF_A = 0;                                        // 128 x D
  static constexpr uint32_t OFF_A2 = OFF_A + 4u * 128 * D;                    // 128 x D
  static constexpr uint32_t OFF_B = OFF_A2 + (kDT ? 4u * 128 * D : 0u);       // TW x D
  static constexpr uint32_t OFF_B2 = OFF_B + 4u * TW * D;                     // TW x D
  static constexpr uint32_t OFF_B3 = OFF_B2 + (kDT ? 4u * TW * D : 0u);       // D x TW
  static constexpr uint32_t OFF_B4 = OFF_B3 + (kAcc ? 4u * D * TW : 0u);      // D x TW
  static constexpr uint32_t OFF_DS = OFF_B4 + (kTwo ? 4u * D * TW : 0u);      // 128 x TW
  static constexpr uint32_t OFF_TT = OFF_DS + (kAcc ? 4u * 128 * TW : 0u);    // 128 x TW
  static constexpr uint32_t OFF_TV = OFF_TT + (kTwo ? 4u * 128 * TW : 0u);    // 11 x TW vectors
  static constexpr uint32_t OFF_BAR = OFF_TV + 4u * 11 * TW;
  static constexpr uint32_t NEED = OFF_BAR + 64 + 1024;
  static constexpr uint32_t SMEM = NEED > 81920u ? NEED : 81920u;  // <= 2 CTAs / SM (TMEM 2 x 256)
  static_assert(NEED <= 232448u, "shared memory");
};

template <int MODE, int D>
__global__ void __launch_bounds__(kBThreads) stream_bwd_kernel(const StreamBwdParams p) {
  using Cfg = SBCfg<MODE, D>;
  constexpr int TW = Cfg::TW;
  constexpr bool kDT = Cfg::kDT, kAcc = Cfg::kAcc, kTwo = Cfg::kTwo;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* As = reinterpret_cast<float*>(base + Cfg::OFF_A);
  float* A2s = reinterpret_cast<float*>(base + Cfg::OFF_A2);
  float* Bs = reinterpret_cast<float*>(base + Cfg::OFF_B);
  float* B2s = reinterpret_cast<float*>(base + Cfg::OFF_B2);
  float* B3s = reinterpret_cast<float*>(base + Cfg::OFF_B3);
  float* B4s = reinterpret_cast<float*>(base + Cfg::OFF_B4);
  float* dSs = reinterpret_cast<float*>(base + Cfg::OFF_DS);
  float* TTs = reinterpret_cast<float*>(base + Cfg::OFF_TT);
  float* tvs = reinterpret_cast<float*>(base + Cfg::OFF_TV);  // [11][TW]: tv0..7, x 3-vector
  uint64_t* mbar = reinterpret_cast<uint64_t*>(base + Cfg::OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + Cfg::OFF_BAR + 16);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  const int prob = blockIdx.x / nrb, rb = blockIdx.x % nrb;
  if (p.done != nullptr && p.done[prob] != 0) return;  // uniform over the CTA
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const size_t bh = static_cast<size_t>(prob);
  const int r0 = p.row_begin + 128 * rb, row = r0 + tid;
  const float eps_h = p.eps[hh];
  const float scale = kLog2e * p.qk_scale / eps_h;
  const bool rin = row < p.row_end && row < N;
  const bool rok = rin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + row] != 0.0f);
  int err = 0;
  // Only the column tiles that hold a valid point are visited (a masked column
  // has a -inf potential: P = T_norm = 0 there, so it adds exactly nothing);
  // a block with no valid row visits none and writes the masked-row values.
  int vlo, vhi;
  valid_extent<kBThreads>(p.mask, bb, N, reinterpret_cast<int*>(base + Cfg::OFF_BAR + 32), vlo, vhi);
  const int rhi = min(min(r0 + 128, p.row_end), N);
  const bool live = max(r0, vlo) < min(rhi, vhi);
  const int t_begin = live ? vlo / TW : 0;
  const int ntiles = live ? (vhi + TW - 1) / TW - t_begin : 0;

  if (warp == 0) tmem_alloc(tslot, 256);
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
  }
  auto ldt = [&](float* dst, const void* src, int is_f32, int row_first, auto rows_tag, auto tr_tag) {
    constexpr int ROWS = decltype(rows_tag)::value;
    constexpr bool TR = decltype(tr_tag)::value;
    load_tile_any<D, ROWS, TR, kBThreads>(dst, src, is_f32 ? static_cast<int>(DFS_F32) : p.dtype, bh * N,
                                          row_first, N, tid);
  };
  using R128 = std::integral_constant<int, 128>;
  using RTW = std::integral_constant<int, TW>;
  using NoT = std::false_type;
  using Tr = std::true_type;
  ldt(As, p.Aop, p.a_f32, r0, R128{}, NoT{});
  if constexpr (kDT) ldt(A2s, p.A2op, p.a2_f32, r0, R128{}, NoT{});
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tlane = static_cast<uint32_t>(32 * warp) << 16;
  // TMEM columns: S [0, TW), dT [TW, 2 TW), accumulators [2 TW, 2 TW + D), [2 TW + D, 2 TW + 2 D)
  const uint32_t t_s = tbase, t_dt = tbase + TW, t_a0 = tbase + 2 * TW, t_a1 = tbase + 2 * TW + D;

  float rv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) rv[k] = (rin && p.rv[k] != nullptr) ? p.rv[k][bh * N + row] : 0.0f;
  float rx[3] = {0.0f, 0.0f, 0.0f};
  if (p.rxvec != nullptr && rin) {
    const size_t o = (p.rxvec_per_head ? bh : static_cast<size_t>(bb)) * N + row;
#pragma unroll
    for (int c = 0; c < 3; ++c) rx[c] = p.rxvec[o * 3 + c];
  }
  const bool has_x = p.xvec != nullptr && p.rxvec != nullptr;
  float s0 = 0.0f, s1 = 0.0f, mrun = -1.0e30f;  // running results

  uint32_t ph0 = 0, ph1 = 0;
  auto wait_bar = [&](int b) {
    const uint32_t par = b == 0 ? ph0 : ph1;
    if (!mbar_wait(&mbar[b], par)) err |= DFS_ERR_DEVICE_TIMEOUT;
    if (b == 0) ph0 ^= 1u; else ph1 ^= 1u;
    tc_fence_after();
  };

#pragma unroll 1
  for (int u = 0; u < ntiles; ++u) {
    const int c0 = (t_begin + u) * TW;
    if (kAcc && u > 0) wait_bar(1);  // accumulation MMAs of tile t-1 done: their operands are free
    // ---- stage the tile
    ldt(Bs, p.Bop, p.b_f32, c0, RTW{}, NoT{});
    if constexpr (kDT) ldt(B2s, p.B2op, p.b2_f32, c0, RTW{}, NoT{});
    if constexpr (kAcc) ldt(B3s, p.B3op, p.b3_f32, c0, RTW{}, Tr{});
    if constexpr (kTwo) ldt(B4s, p.B4op, p.b4_f32, c0, RTW{}, Tr{});
    if (tid < TW) {
      const int j = c0 + tid;
      const bool cin = j < N;
      const bool cok = cin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float v = (cin && p.tv[k] != nullptr) ? p.tv[k][bh * N + j] : 0.0f;
        // tv0 (and for SB_COL / SB_DKV tv1) are potentials: -inf on invalid columns zeroes P, T
        const bool pot = k == 0 || (k == 1 && (MODE == SB_COL || MODE == SB_DKV));
        if (pot && !cok) v = -INFINITY;
        tvs[k * TW + tid] = v;
      }
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        float v = 0.0f;
        if (has_x && cin) {
          const size_t o = (p.xvec_per_head ? bh : static_cast<size_t>(bb)) * N + j;
          v = p.xvec[o * 3 + c];
        }
        tvs[(8 + c) * TW + tid] = v;
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      issue_mma<128, TW, D>(t_s, As, Bs, false);
      if constexpr (kDT) issue_mma<128, TW, D>(t_dt, A2s, B2s, false);
      mma_commit(&mbar[0]);
    }
    wait_bar(0);

    // ---- epilogue: 2 chunks of 32 columns
#pragma unroll 1
    for (int ch = 0; ch < TW / 32; ++ch) {
      float sv[32], dv[32];
      tmem_ld32(t_s + tlane + 32 * ch, sv);
      if constexpr (kDT) tmem_ld32(t_dt + tlane + 32 * ch, dv);
      const float* tv0 = tvs + 32 * ch;
      if constexpr (MODE == SB_ROW) {
        // rv0 = f; tv0 = g; dT += dxc_i . x_j (rx = dxc_i, tv 8..10 = x_j)
        float cm = -1.0e30f;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          sv[k] = fmaf(sv[k], scale, tv0[k] + rv[0]);
          cm = fmaxf(cm, sv[k]);
        }
        const float mn = fmaxf(mrun, cm), resc = ex2(mrun - mn);
        float r = s0 * resc, pd = s1 * resc;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          float dt = dv[k];
          if (has_x) dt += rx[0] * tv0[8 * TW + k] + rx[1] * tv0[9 * TW + k] + rx[2] * tv0[10 * TW + k];
          const float e = ex2(sv[k] - mn);
          r += e;
          pd = fmaf(e, dt, pd);
        }
        mrun = mn;
        s0 = r;
        s1 = pd;
      } else if constexpr (MODE == SB_COL) {
        // thread = column j: rv0 = g_j, rx = x_j; tile i: tv0 = f, tv1 = f - m, tv2 = 1/(R+1e-6),
        // tv3 = D, tv 8..10 = dxc_i
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float sc = sv[k] * scale + rv[0];
          const float P = ex2(sc + tv0[k]);
          const float T = ex2(sc + tv0[TW + k]) * tv0[2 * TW + k];
          float dt = dv[k];
          if (has_x) dt += rx[0] * tv0[8 * TW + k] + rx[1] * tv0[9 * TW + k] + rx[2] * tv0[10 * TW + k];
          s0 += P;
          s1 = fmaf(T, dt - tv0[3 * TW + k], s1);
        }
      } else if constexpr (MODE == SB_MATVEC) {
        // rv0 = row potential; tv0 = column potential, tv1 = the vector
#pragma unroll
        for (int k = 0; k < 32; ++k) s0 = fmaf(ex2(fmaf(sv[k], scale, tv0[k] + rv[0])), tv0[TW + k], s0);
      } else if constexpr (MODE == SB_DQ) {
        // rv0 = f, rv1 = f - m, rv2 = 1/(R+1e-6), rv3 = D, rv4 = w1; tv0 = g, tv1 = w2, tv 8..10 = x_j;
        // rx = dxc_i
        float ds[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float sc = fmaf(sv[k], scale, tv0[k]);
          const float P = ex2(sc + rv[0]);
          const float T = ex2(sc + rv[1]) * rv[2];
          float dt = dv[k];
          if (has_x) dt += rx[0] * tv0[8 * TW + k] + rx[1] * tv0[9 * TW + k] + rx[2] * tv0[10 * TW + k];
          ds[k] = rok ? T * (dt - rv[3]) - P * (rv[4] + tv0[TW + k]) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(dSs + (sw_off(tid, 32 * ch + 4 * q, 128) >> 2)) =
              make_float4(ds[4 * q], ds[4 * q + 1], ds[4 * q + 2], ds[4 * q + 3]);
      } else {  // SB_DKV
        // thread = column j: rv0 = g_j, rv1 = w2_j, rx = x_j; tile i: tv0 = f, tv1 = f - m,
        // tv2 = 1/(R+1e-6), tv3 = D, tv4 = w1, tv 8..10 = dxc_i
        float ds[32], tt[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float sc = sv[k] * scale + rv[0];
          const float P = ex2(sc + tv0[k]);
          const float T = ex2(sc + tv0[TW + k]) * tv0[2 * TW + k];
          float dt = dv[k];
          if (has_x) dt += rx[0] * tv0[8 * TW + k] + rx[1] * tv0[9 * TW + k] + rx[2] * tv0[10 * TW + k];
          ds[k] = rok ? T * (dt - tv0[3 * TW + k]) - P * (tv0[4 * TW + k] + rv[1]) : 0.0f;
          tt[k] = rok ? T : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          *reinterpret_cast<float4*>(dSs + (sw_off(tid, 32 * ch + 4 * q, 128) >> 2)) =
              make_float4(ds[4 * q], ds[4 * q + 1], ds[4 * q + 2], ds[4 * q + 3]);
          *reinterpret_cast<float4*>(TTs + (sw_off(tid, 32 * ch + 4 * q, 128) >> 2)) =
              make_float4(tt[4 * q], tt[4 * q + 1], tt[4 * q + 2], tt[4 * q + 3]);
        }
      }
    }
    // every thread is done with the tile's vectors and TMEM S / dT; dS and T tiles are written
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if constexpr (kAcc) {
      if (tid == 0) {
        issue_mma<128, D, TW>(t_a0, dSs, B3s, u > 0);
        if constexpr (kTwo) issue_mma<128, D, TW>(t_a1, TTs, B4s, u > 0);
        mma_commit(&mbar[1]);
      }
    }
  }

  // ---------------------------------------------------------------- results
  if constexpr (kAcc) {
    if (ntiles > 0) wait_bar(1);  // (no tile: every row is masked and written as 0)
#pragma unroll
    for (int a = 0; a < (kTwo ? 2 : 1); ++a) {
      float* dst_base = a == 0 ? p.acc0 : p.acc1;
      float sc = a == 0 ? p.acc_scale0 : p.acc_scale1;
      if (sc < 0.0f) sc = p.qk_scale / eps_h;  // dS -> dQ, dK
#pragma unroll
      for (int g = 0; g < D / 16; ++g) {
        float v[16];
        tmem_ld16((a == 0 ? t_a0 : t_a1) + tlane + 16 * g, v);
        if (rin && dst_base != nullptr) {
          float4* dst = reinterpret_cast<float4*>(dst_base + (bh * N + row) * D + 16 * g);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = rok ? make_float4(v[4 * q] * sc, v[4 * q + 1] * sc, v[4 * q + 2] * sc, v[4 * q + 3] * sc)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  } else if (rin) {
    const size_t o = bh * N + row;
    if constexpr (MODE == SB_ROW) {
      p.out0[o] = rok ? mrun : 0.0f;                       // m
      p.out1[o] = rok ? s0 : 0.0f;                         // R
      p.out2[o] = rok ? s1 / (s0 + 1e-6f) : 0.0f;          // D
    } else if constexpr (MODE == SB_COL) {
      p.out0[o] = rok ? s0 : 0.0f;                         // c
      p.out1[o] = rok ? s1 : 0.0f;                         // g_v
    } else {
      p.out0[o] = rok ? s0 * (p.rv[1] != nullptr ? rv[1] : 1.0f) : 0.0f;
    }
  }
  (void)err;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

template <int MODE, int D>
static cudaError_t launch_sb_md(const StreamBwdParams& p, cudaStream_t st) {
  using Cfg = SBCfg<MODE, D>;
  auto kern = stream_bwd_kernel<MODE, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  if (e != cudaSuccess) return e;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  kern<<<p.B * p.H * nrb, kBThreads, Cfg::SMEM, st>>>(p);
  return cudaGetLastError();
}

template <int D>
static cudaError_t launch_sb_d(int mode, const StreamBwdParams& p, cudaStream_t st) {
  switch (mode) {
    case SB_ROW: return launch_sb_md<SB_ROW, D>(p, st);
    case SB_COL: return launch_sb_md<SB_COL, D>(p, st);
    case SB_MATVEC: return launch_sb_md<SB_MATVEC, D>(p, st);
    case SB_DQ: return launch_sb_md<SB_DQ, D>(p, st);
    default: return launch_sb_md<SB_DKV, D>(p, st);
  }
}

cudaError_t launch_stream_bwd_pass(int mode, int d, const StreamBwdParams& p, cudaStream_t st) {
  if (p.row_end <= p.row_begin) return cudaSuccess;
  if (d == 32) return launch_sb_d<32>(mode, p, st);
  if (d == 64) return launch_sb_d<64>(mode, p, st);
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- vector steps
// Workspace slots (each (BH, N) fp32) and per-problem scalars.
enum {
  WS_F = 0, WS_G, WS_M, WS_R, WS_D, WS_FM, WS_INVR, WS_C, WS_GV, WS_D1I, WS_B1, WS_D2, WS_D2I,
  WS_X2, WS_R2, WS_P2, WS_S2, WS_U2, WS_W2, WS_T, WS_S, WS_W1, WS_NUM
};
// SC_LOOP: problem 0's entry holds the round count (int32) of the
// device-terminated CG loop (sb_loopcond_kernel)
enum { SC_GAM = 0, SC_ALPHA, SC_BETA, SC_TOL2, SC_RR, SC_LOOP = 7, SC_NUM = 8 };

constexpr int kVThreads = 256;

struct VecParams {
  float* ws;
  float* sc;        // (BH, SC_NUM)
  int32_t* done;    // (BH)
  int32_t* iters;   // (BH)
  const float* eps;
  const float* mask;
  const float* log_u;
  const float* log_v;
  float* dlog_mu;
  float* dlog_nu;
  int32_t* cg_iters;
  float* cg_residual;
  int32_t* status;
  float lam, rtol, atol;
  int B, H, N, max_iter;
};

DFS_DEV bool pos_ok(const VecParams& p, int bb, int i) {
  return i < p.N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * p.N + i] != 0.0f);
}

// deterministic block sums of up to 3 values (fixed order)
DFS_DEV void block_sum3(float& a, float& b, float& c, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  c = warp_sum(c);
  __syncthreads();
  if (lane == 0) {
    red[warp] = a;
    red[8 + warp] = b;
    red[16 + warp] = c;
  }
  __syncthreads();
  a = b = c = 0.0f;
#pragma unroll
  for (int w = 0; w < kVThreads / 32; ++w) {
    a += red[w];
    b += red[8 + w];
    c += red[16 + w];
  }
}

// phase 0: potentials into log2 units (elementwise over BH N)
__global__ void sb_prep_kernel(VecParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  const size_t n = static_cast<size_t>(p.B) * p.H * p.N;
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int pos = static_cast<int>(i % p.N), prob = static_cast<int>(i / p.N), bb = prob / p.H;
  const bool ok = pos_ok(p, bb, pos);
  p.ws[WS_F * n + i] = ok ? p.log_u[i] * kLog2e : 0.0f;
  p.ws[WS_G * n + i] = ok ? p.log_v[i] * kLog2e : 0.0f;
}

// after SB_ROW: f - m, 1/(R + 1e-6), the row block d1 = r/kappa (r = R 2^m) and
// b1 = dL/df = rowsum(E) = D (1 - R/(R + 1e-6))
__global__ void sb_rowderive_kernel(VecParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  const size_t n = static_cast<size_t>(p.B) * p.H * p.N;
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int pos = static_cast<int>(i % p.N), prob = static_cast<int>(i / p.N), bb = prob / p.H, hh = prob % p.H;
  const float eps_h = p.eps[hh];
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
  const bool ok = pos_ok(p, bb, pos);
  const float m = p.ws[WS_M * n + i], R = p.ws[WS_R * n + i], D = p.ws[WS_D * n + i];
  const float inv = 1.0f / (R + 1e-6f);
  const float r = R * ex2(m);
  p.ws[WS_FM * n + i] = ok ? p.ws[WS_F * n + i] - m : 0.0f;
  p.ws[WS_INVR * n + i] = ok ? inv : 0.0f;
  p.ws[WS_D1I * n + i] = (ok && r > 0.0f) ? kap / r : 0.0f;
  p.ws[WS_B1 * n + i] = ok ? D * (1.0f - R * inv) : 0.0f;
  p.ws[WS_T * n + i] = 0.0f;
}

// after SB_COL (one CTA per problem): d2 = c/kappa, the kappa = 1 projection of
// the right-hand side onto the range of the singular system, and t = D1^-1 b1
__global__ void __launch_bounds__(kVThreads) sb_setup_kernel(VecParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  __shared__ float red[32];
  const size_t n = static_cast<size_t>(p.B) * p.H * p.N;
  const int prob = blockIdx.x, bb = prob / p.H, hh = prob % p.H, N = p.N;
  const size_t o = static_cast<size_t>(prob) * N;
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + p.eps[hh]);
  float* ws = p.ws;
  float sb1 = 0.0f, sb2 = 0.0f, nv = 0.0f;
  for (int i = threadIdx.x; i < N; i += kVThreads) {
    const bool ok = pos_ok(p, bb, i);
    const float c = ws[WS_C * n + o + i];
    const float d2 = (ok && c > 0.0f) ? c / kap : 0.0f;
    ws[WS_D2 * n + o + i] = d2;
    ws[WS_D2I * n + o + i] = d2 > 0.0f ? 1.0f / d2 : 0.0f;
    const float b2 = ok ? ws[WS_GV * n + o + i] : 0.0f;
    ws[WS_GV * n + o + i] = b2;
    sb1 += ws[WS_B1 * n + o + i];
    sb2 += b2;
    nv += ok ? 1.0f : 0.0f;
  }
  block_sum3(sb1, sb2, nv, red);
  const float sh = (kap >= 1.0f && nv > 0.0f) ? (sb1 - sb2) / (2.0f * nv) : 0.0f;
  for (int i = threadIdx.x; i < N; i += kVThreads) {
    const bool ok = pos_ok(p, bb, i);
    const float b1 = ok ? ws[WS_B1 * n + o + i] - sh : 0.0f;
    ws[WS_B1 * n + o + i] = b1;
    ws[WS_GV * n + o + i] = ok ? ws[WS_GV * n + o + i] + sh : 0.0f;
    ws[WS_T * n + o + i] = ws[WS_D1I * n + o + i] * b1;
  }
  if (threadIdx.x == 0) {
    p.done[prob] = 0;
    p.iters[prob] = 0;
  }
}

// after s = P^T D1^-1 b1: the reduced right-hand side r2 = b2 - s; x2 = 0; u2 = D2^-1 r2
__global__ void sb_cginit_kernel(VecParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  const size_t n = static_cast<size_t>(p.B) * p.H * p.N;
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int pos = static_cast<int>(i % p.N), prob = static_cast<int>(i / p.N), bb = prob / p.H;
  const bool ok = pos_ok(p, bb, pos);
  const float r2 = ok ? p.ws[WS_GV * n + i] - p.ws[WS_S * n + i] : 0.0f;
  p.ws[WS_R2 * n + i] = r2;
  p.ws[WS_U2 * n + i] = r2 * p.ws[WS_D2I * n + i];
  p.ws[WS_X2 * n + i] = 0.0f;
  p.ws[WS_P2 * n + i] = 0.0f;
  p.ws[WS_S2 * n + i] = 0.0f;
}

// One Chronopoulos-Gear step (one CTA per problem), after s = P^T D1^-1 P u2:
// w2 = D2 u2 - s, the dots (r,u), (w,u), (r,r), the convergence test and the
// scalars, then the vector updates for the next product (same recurrence as
// the resident backward).
__global__ void __launch_bounds__(kVThreads) sb_cgstep_kernel(VecParams p, int first) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  __shared__ float red[32];
  const int prob = blockIdx.x;
  if (p.done[prob]) return;
  const size_t n = static_cast<size_t>(p.B) * p.H * p.N;
  const int bb = prob / p.H, N = p.N;
  const size_t o = static_cast<size_t>(prob) * N;
  float* ws = p.ws;
  float* sc = p.sc + static_cast<size_t>(prob) * SC_NUM;
  float ru = 0.0f, wu = 0.0f, rr = 0.0f;
  for (int i = threadIdx.x; i < N; i += kVThreads) {
    const bool ok = pos_ok(p, bb, i);
    const float u = ws[WS_U2 * n + o + i];
    const float w = ok ? ws[WS_D2 * n + o + i] * u - ws[WS_S * n + o + i] : 0.0f;
    ws[WS_W2 * n + o + i] = w;
    const float r = ws[WS_R2 * n + o + i];
    ru += r * u;
    wu += w * u;
    rr += r * r;
  }
  block_sum3(ru, wu, rr, red);
  float gam = sc[SC_GAM], alpha = sc[SC_ALPHA], beta = sc[SC_BETA];
  int result = 0;  // 0: continue, 1: converged, 2: stopped unconverged (cap or breakdown)
  if (first) {
    const float nrm0 = sqrtf(fmaxf(rr, 0.0f));
    const float tol = fmaxf(p.atol, p.rtol * nrm0);
    if (threadIdx.x == 0) sc[SC_TOL2] = tol * tol;
    if (!(nrm0 > tol)) result = 1;
    else if (!(wu > 0.0f) || p.max_iter <= 0) result = 2;
    gam = ru;
    alpha = wu > 0.0f ? ru / wu : 0.0f;
    beta = 0.0f;
  } else {
    const int it = p.iters[prob] + 1;
    if (threadIdx.x == 0) p.iters[prob] = it;
    if (rr <= sc[SC_TOL2]) {
      result = 1;
    } else {
      beta = ru / gam;
      const float den = wu - beta * ru / alpha;
      if (!(den > 0.0f) || !(den < 3.0e38f) || it >= p.max_iter) {
        result = 2;
      } else {
        alpha = ru / den;
        gam = ru;
      }
    }
  }
  if (threadIdx.x == 0) {
    sc[SC_GAM] = gam;
    sc[SC_ALPHA] = alpha;
    sc[SC_BETA] = beta;
    sc[SC_RR] = rr;
    if (result) p.done[prob] = result;
  }
  const bool stop = result != 0;
  if (stop) return;
  for (int i = threadIdx.x; i < N; i += kVThreads) {
    const float pp = ws[WS_U2 * n + o + i] + beta * ws[WS_P2 * n + o + i];
    const float ss = ws[WS_W2 * n + o + i] + beta * ws[WS_S2 * n + o + i];
    ws[WS_P2 * n + o + i] = pp;
    ws[WS_S2 * n + o + i] = ss;
    ws[WS_X2 * n + o + i] += alpha * pp;
    const float r = ws[WS_R2 * n + o + i] - alpha * ss;
    ws[WS_R2 * n + o + i] = r;
    ws[WS_U2 * n + o + i] = r * ws[WS_D2I * n + o + i];
  }
}

// Condition of the device-terminated CG loop (a WHILE node of a CUDA graph
// whose body is one CG round): 1 while some problem's solve still runs.  The
// round count is capped independently of the flags (every solve stops within
// max_iter rounds by itself), so the loop ends after at most max_rounds
// rounds whatever the flags say.  `reset`: the launch before the loop.
__global__ void sb_loopcond_kernel(const int32_t* done, int nprob, int32_t* rounds, int max_rounds, int reset,
                                   cudaGraphConditionalHandle cond) {
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  int mine = 0;
  for (int i = threadIdx.x; i < nprob; i += blockDim.x) mine |= done[i] == 0;
  if (mine) any = 1;  // every writer stores the same value
  __syncthreads();
  if (threadIdx.x == 0) {
    const int r = reset ? 0 : rounds[0] + 1;
    rounds[0] = r;
    cudaGraphSetConditional(cond, (any != 0 && r < max_rounds) ? 1u : 0u);
  }
}

// After q = P x2 (in WS_S): w1 = D1^-1 (b1 - q); for kappa = 1 the null-space
// shift t = -sum(r w1)/sum(r); marginal gradients; CG report (one CTA per problem).
__global__ void __launch_bounds__(kVThreads) sb_final_kernel(VecParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  __shared__ float red[32];
  const int prob = blockIdx.x, bb = prob / p.H, hh = prob % p.H, N = p.N;
  const size_t n = static_cast<size_t>(p.B) * p.H * N;
  const size_t o = static_cast<size_t>(prob) * N;
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + p.eps[hh]);
  float* ws = p.ws;
  float srw = 0.0f, sr = 0.0f, unused = 0.0f;
  for (int i = threadIdx.x; i < N; i += kVThreads) {
    const bool ok = pos_ok(p, bb, i);
    const float d1i = ws[WS_D1I * n + o + i];
    const float w1 = ok ? d1i * (ws[WS_B1 * n + o + i] - ws[WS_S * n + o + i]) : 0.0f;
    ws[WS_W1 * n + o + i] = w1;
    const float r = d1i > 0.0f ? kap / d1i : 0.0f;
    srw += r * w1;
    sr += r;
  }
  block_sum3(srw, sr, unused, red);
  const float tshift = (kap >= 1.0f && sr > 0.0f) ? -srw / sr : 0.0f;
  for (int i = threadIdx.x; i < N; i += kVThreads) {
    const bool ok = pos_ok(p, bb, i);
    const float d1i = ws[WS_D1I * n + o + i];
    const float r = d1i > 0.0f ? kap / d1i : 0.0f;
    if (p.dlog_mu) p.dlog_mu[o + i] = ok ? r * (ws[WS_W1 * n + o + i] + tshift) : 0.0f;
    if (p.dlog_nu) p.dlog_nu[o + i] = ok ? ws[WS_C * n + o + i] * (ws[WS_X2 * n + o + i] - tshift) : 0.0f;
  }
  if (threadIdx.x == 0) {
    if (p.cg_iters) p.cg_iters[prob] = p.iters[prob];
    if (p.cg_residual) p.cg_residual[prob] = sqrtf(fmaxf(p.sc[static_cast<size_t>(prob) * SC_NUM + SC_RR], 0.0f));
    if (p.done[prob] != 1 && p.status) atomicOr(p.status, DFS_WARN_CG_NOT_CONVERGED);
  }
}

// Slots, per-problem scalars, CG flags and iteration counts, then the fp32
// operand copies of the TMA-staged tile passes, the column-split scratch, the
// mask's valid extents; with cost terms, the bin tables (position term) and
// the shares of the shared-parameter gradients (CostGradWs below).
namespace {
size_t rnd256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
// dx shares of the three gradient passes (rows, columns, centroid), the per-row
// dw share, the per-CTA bin sums, the per-row dr share
size_t costgrad_floats(int B, int H, int N) {
  const size_t n = static_cast<size_t>(B) * H * N, bh = static_cast<size_t>(B) * H;
  return 3 * 3 * n + n + bh * ((N + 127) / 128) * kBinCount + n;
}
}  // namespace

size_t stream_bwd_workspace(int B, int H, int N, int d, int terms) {
  const size_t n = static_cast<size_t>(B) * H * N, bh = static_cast<size_t>(B) * H;
  size_t bytes = sizeof(float) * (WS_NUM * n + SC_NUM * bh) + 2 * sizeof(int32_t) * bh + 256 +
                 bt_copies_bytes(B, H, N, d) + 256 + tile_split_bytes(B, H, N) + 64 + sizeof(int2) * static_cast<size_t>(B);
  if (terms & DFS_TERM_POS) bytes += 256 + 2 * rnd256(cost_bins_bytes(B, N));
  if (terms) bytes += 256 + sizeof(float) * costgrad_floats(B, H, N);
  return bytes;
}

// Sums of the gradient shares in a fixed order: dx_res over heads (the row,
// column and centroid shares whose bits are set in `shares`), dw_dist over
// batch elements and rows, dpos_weight over batch elements and row blocks,
// dr_head over batch elements and rows.
__global__ void stream_costgrad_finalize(const float* dx_row, const float* dx_col, const float* dx_t,
                                         const float* dw, const float* dpos, const float* dr, int shares, int B,
                                         int H, int N, float* dx_res, float* dw_dist, float* dpos_weight,
                                         float* dr_head) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int nrb = (N + 127) / 128;
  const int ndx = dx_res != nullptr ? B * N * 3 : 0;
  const int ndw = dw_dist != nullptr ? H : 0;
  const int npos = dpos_weight != nullptr ? H * kBinCount : 0;
  const int ndr = dr_head != nullptr ? H : 0;
  if (t < ndx) {
    const int b = t / (N * 3), rem = t % (N * 3);
    float s = 0.0f;
    for (int h = 0; h < H; ++h) {
      const size_t o = (static_cast<size_t>(b) * H + h) * N * 3 + rem;
      if (shares & 1) s += dx_row[o];
      if (shares & 2) s += dx_col[o];
      if (shares & 4) s += dx_t[o];
    }
    dx_res[t] = s;
  } else if (t < ndx + ndw) {
    const int h = t - ndx;
    float s = 0.0f;
    for (int b = 0; b < B; ++b)
      for (int i = 0; i < N; ++i) s += dw[(static_cast<size_t>(b) * H + h) * N + i];
    dw_dist[h] = s;
  } else if (t < ndx + ndw + npos) {
    const int u = t - ndx - ndw, h = u / kBinCount, bin = u % kBinCount;
    float s = 0.0f;
    for (int b = 0; b < B; ++b)
      for (int r = 0; r < nrb; ++r) s += dpos[((static_cast<size_t>(b) * H + h) * nrb + r) * kBinCount + bin];
    dpos_weight[u] = s;
  } else if (t < ndx + ndw + npos + ndr) {
    const int h = t - ndx - ndw - npos;
    float s = 0.0f;
    for (int b = 0; b < B; ++b)
      for (int i = 0; i < N; ++i) s += dr[(static_cast<size_t>(b) * H + h) * N + i];
    dr_head[h] = s;
  }
}

constexpr bool same_slot(int a, int b) { return a == b; }
static_assert(same_slot(WS_F, DFS_WS_BWD_F) && same_slot(WS_G, DFS_WS_BWD_G) && same_slot(WS_M, DFS_WS_BWD_M) &&
                  same_slot(WS_R, DFS_WS_BWD_R) && same_slot(WS_D, DFS_WS_BWD_D) && same_slot(WS_C, DFS_WS_BWD_C) &&
                  same_slot(WS_GV, DFS_WS_BWD_GV) && same_slot(WS_T, DFS_WS_BWD_T) && same_slot(WS_S, DFS_WS_BWD_S) &&
                  same_slot(WS_NUM, DFS_WS_BWD_NSLOTS) && same_slot(SC_NUM, DFS_WS_BWD_NSCALARS),
              "workspace slots named in include/dfsink.h");

// One phase of the streamed backward on rows (or, for the column phases,
// columns) [r0, r1): the whole problem on a single GPU, a range per GPU when
// rows are sharded.  Phases without a range work on every position, from the
// all-gathered vectors.  The order, and the vectors each range phase produces
// (which a sharded run all-gathers before the next phase):
//   BWD_PREP                     f, g in log2 units
//   BWD_ROWSTATS   rows          m, R, D
//   BWD_ROWDERIVE                f - m, 1/(R+1e-6), D1^-1, b1
//   BWD_COLSTATS   columns       c, g_v
//   BWD_SETUP                    D2, kappa = 1 projection, t = D1^-1 b1
//   BWD_PT_T       columns       s = P^T t
//   BWD_CGINIT                   reduced right-hand side, u2
//   then (max_iter + 1) x { BWD_P_U rows: t = D1^-1 P u2;  BWD_PT_T columns: s = P^T t;
//                           BWD_CGSTEP_FIRST (first time) / BWD_CGSTEP }
//   BWD_P_X        rows          s = P x2
//   BWD_FINAL                    w1, null-space shift, dlog_mu, dlog_nu, CG report
//   BWD_DQ         rows          dQ
//   BWD_DKV        columns       dK, dV
static TileArgs tile_args(const BwdParams& bp, int r0, int r1, float* split, const int2* ext) {
  TileArgs ta{};
  ta.split = split;
  ta.extent = ext;
  ta.dtype = bp.in_dtype;
  ta.d = bp.d;
  ta.eps = bp.eps;
  ta.mask = bp.mask;
  ta.status = bp.status;
  ta.B = bp.B;
  ta.H = bp.H;
  ta.N = bp.N;
  ta.row_begin = r0;
  ta.row_end = r1;
  ta.lam = bp.lam;
  ta.qk_scale = bp.qk_scale;
  return ta;
}

cudaError_t stream_bwd_op(int op, const BwdParams& bp, float* wsp, int r0, int r1, cudaStream_t st) {
  const int B = bp.B, H = bp.H, N = bp.N, d = bp.d;
  const size_t n = static_cast<size_t>(B) * H * N, nbh = static_cast<size_t>(B) * H;
  VecParams v{};
  v.ws = wsp;
  v.sc = wsp + WS_NUM * n;
  v.done = reinterpret_cast<int32_t*>(v.sc + SC_NUM * nbh);
  v.iters = v.done + nbh;
  v.eps = bp.eps;
  v.mask = bp.mask;
  v.log_u = bp.log_u;
  v.log_v = bp.log_v;
  v.dlog_mu = bp.dlog_mu;
  v.dlog_nu = bp.dlog_nu;
  v.cg_iters = bp.cg_iters;
  v.cg_residual = bp.cg_residual;
  v.status = bp.status;
  v.lam = bp.lam;
  v.rtol = bp.cg_rtol;
  v.atol = bp.cg_atol;
  v.B = B;
  v.H = H;
  v.N = N;
  v.max_iter = bp.cg_max_iter;
  float* ws = wsp;
  auto slot = [&](int k) { return ws + static_cast<size_t>(k) * n; };
  const unsigned eblocks = static_cast<unsigned>((n + 255) / 256);
  const unsigned pblocks = static_cast<unsigned>(nbh);

  // TMA-staged tile passes on fp32 copies placed after the CG state
  const bool bt = bt_path_ok(d, N, wsp);
  const BtCopies cp = bt_copies(reinterpret_cast<float*>(v.iters + nbh), B, H, N, d);
  // column-split scratch of the plan-vector products, after the copies
  float* split = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(cp.dOT + static_cast<size_t>(n) * d) + 255) & ~uintptr_t(255));
  // the mask's valid extent per batch element, after the split scratch
  int2* extents = reinterpret_cast<int2*>(
      (reinterpret_cast<uintptr_t>(split) + tile_split_bytes(B, H, N) + 63) & ~uintptr_t(63));
  const int2* ext = bp.mask != nullptr ? extents : nullptr;
  // cost-term tables and gradient shares, after the extents
  uint8_t* bins = nullptr;
  uint8_t* bins_t = nullptr;
  float* cgw = nullptr;
  {
    uint8_t* q8 = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(extents + B) + 255) & ~uintptr_t(255));
    if (bp.cost_terms & DFS_TERM_POS) {
      bins = q8;
      bins_t = bins + rnd256(cost_bins_bytes(B, N));
      q8 = bins_t + rnd256(cost_bins_bytes(B, N));
    }
    if (bp.cost_terms) cgw = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(q8) + 255) & ~uintptr_t(255));
  }
  const bool geo = bp.x_res != nullptr && bp.w_dist != nullptr;
  auto terms = [&](bool transposed) {
    return cost_terms_of(bp.pos_weight, geo ? bp.x_res : nullptr, bp.w_dist, bp.r_0, bp.r_head, N, bins, bins_t,
                         transposed);
  };
  float* cg_dx_row = cgw;
  float* cg_dx_col = cgw ? cgw + 3 * n : nullptr;
  float* cg_dx_t = cgw ? cgw + 6 * n : nullptr;
  float* cg_dw = cgw ? cgw + 9 * n : nullptr;
  float* cg_dpos = cgw ? cgw + 10 * n : nullptr;
  float* cg_dr = cgw ? cg_dpos + static_cast<size_t>(B) * H * ((N + 127) / 128) * kBinCount : nullptr;
  const bool want_dx = cgw != nullptr && bp.dx_res != nullptr;
  BtArgs ba{};
  ba.d = d;
  ba.eps = bp.eps;
  ba.qk_scale = bp.qk_scale;
  ba.mask = bp.mask;
  ba.status = bp.status;
  ba.B = B;
  ba.H = H;
  ba.N = N;
  ba.row_begin = r0;
  ba.row_end = r1;
  ba.extent = ext;

  StreamBwdParams q{};
  q.dtype = bp.in_dtype;
  q.eps = bp.eps;
  q.qk_scale = bp.qk_scale;
  q.mask = bp.mask;
  q.B = B;
  q.H = H;
  q.N = N;
  q.row_begin = r0;
  q.row_end = r1;
  switch (op) {
    case DFS_OP_BWD_PREP: {
      cudaError_t e = launch_dependent(sb_prep_kernel, dim3(eblocks), dim3(256), 0, st, v);
      if (e == cudaSuccess && bt) e = bt_prep(bp, cp, st);
      if (e == cudaSuccess) e = tile_split_reset(split, B, H, N, st);
      if (e == cudaSuccess) e = compute_extents(bp.mask, B, N, extents, st);
      if (e == cudaSuccess && bins != nullptr && bins_given(bin_source(bp)))
        e = build_cost_bins(bin_source(bp), B, N, bins, bins_t, st);
      return e;
    }
    case DFS_OP_BWD_ROWSTATS:  // m, R, D
      if (bt) {
        ba.A = cp.Qf; ba.A2 = cp.dOf; ba.Bop = cp.Kf; ba.B2 = cp.Vf;
        ba.tv[0] = slot(WS_G); ba.pot_mask = 1;
        ba.rv[0] = slot(WS_F);
        ba.xvec = bp.dxc ? bp.x_res : nullptr; ba.xvec_per_head = 0;
        ba.rxvec = bp.dxc; ba.rxvec_per_head = 1;
        ba.out0 = slot(WS_M); ba.out1 = slot(WS_R); ba.out2 = slot(WS_D);
        ba.ct = terms(false);
        return launch_bt_pass(BTP_ROW, ba, st);
      }
      q.Aop = bp.Q; q.Bop = bp.K; q.A2op = bp.dO; q.a2_f32 = 1; q.B2op = bp.V;
      q.tv[0] = slot(WS_G);
      q.rv[0] = slot(WS_F);
      q.xvec = bp.dxc ? bp.x_res : nullptr; q.xvec_per_head = 0;
      q.rxvec = bp.dxc; q.rxvec_per_head = 1;
      q.out0 = slot(WS_M); q.out1 = slot(WS_R); q.out2 = slot(WS_D);
      return launch_stream_bwd_pass(SB_ROW, d, q, st);
    case DFS_OP_BWD_ROWDERIVE:
      return launch_dependent(sb_rowderive_kernel, dim3(eblocks), dim3(256), 0, st, v);
    case DFS_OP_BWD_COLSTATS:  // c, g_v (and, on the TMA-staged path, dV = T_norm^T dO)
      if (bt) {
        ba.A = cp.Kf; ba.A2 = cp.Vf; ba.Bop = cp.Qf; ba.B2 = cp.dOf; ba.B3 = cp.dOT;
        ba.tv[0] = slot(WS_F); ba.tv[1] = slot(WS_FM); ba.tv[2] = slot(WS_INVR); ba.tv[3] = slot(WS_D);
        ba.pot_mask = 3;
        ba.rv[0] = slot(WS_G);
        ba.xvec = bp.dxc; ba.xvec_per_head = 1;
        ba.rxvec = bp.dxc ? bp.x_res : nullptr; ba.rxvec_per_head = 0;
        ba.out0 = slot(WS_C); ba.out1 = slot(WS_GV);
        ba.acc = bp.dV; ba.acc_scale = 1.0f;
        ba.ct = terms(true);
        if (want_dx && bp.dxc != nullptr) ba.cg.dx = cg_dx_t;  // centroid share T_norm^T dxc
        return launch_bt_pass(BTP_COL, ba, st);
      }
      q.Aop = bp.K; q.Bop = bp.Q; q.A2op = bp.V; q.B2op = bp.dO; q.b2_f32 = 1;
      q.tv[0] = slot(WS_F); q.tv[1] = slot(WS_FM); q.tv[2] = slot(WS_INVR); q.tv[3] = slot(WS_D);
      q.rv[0] = slot(WS_G);
      q.xvec = bp.dxc; q.xvec_per_head = 1;
      q.rxvec = bp.dxc ? bp.x_res : nullptr; q.rxvec_per_head = 0;
      q.out0 = slot(WS_C); q.out1 = slot(WS_GV);
      return launch_stream_bwd_pass(SB_COL, d, q, st);
    case DFS_OP_BWD_SETUP:
      return launch_dependent(sb_setup_kernel, dim3(pblocks), dim3(kVThreads), 0, st, v);
    case DFS_OP_BWD_CGINIT:
      return launch_dependent(sb_cginit_kernel, dim3(eblocks), dim3(256), 0, st, v);
    case DFS_OP_BWD_P_U:   // t = D1^-1 P u2 (problems whose CG has stopped are skipped)
    case DFS_OP_BWD_P_X:   // s = P x2
      if (tile_path_ok(bp.in_dtype, d, N, bp.Q, bp.K)) {
        TileArgs ta = tile_args(bp, r0, r1, split, ext);
        ta.A = bp.Q; ta.Bop = bp.K;
        ta.col_bias = slot(WS_G); ta.col_vec = slot(op == DFS_OP_BWD_P_U ? WS_U2 : WS_X2);
        ta.row_bias = slot(WS_F); ta.row_scale = op == DFS_OP_BWD_P_U ? slot(WS_D1I) : nullptr;
        ta.done = op == DFS_OP_BWD_P_U ? v.done : nullptr;
        ta.row_out = slot(op == DFS_OP_BWD_P_U ? WS_T : WS_S);
        ta.ct = terms(false);
        return launch_tile_pass(TL_MATVEC, ta, st);
      }
      q.Aop = bp.Q; q.Bop = bp.K;
      q.tv[0] = slot(WS_G); q.tv[1] = slot(op == DFS_OP_BWD_P_U ? WS_U2 : WS_X2);
      q.rv[0] = slot(WS_F); q.rv[1] = op == DFS_OP_BWD_P_U ? slot(WS_D1I) : nullptr;
      q.done = op == DFS_OP_BWD_P_U ? v.done : nullptr;
      q.out0 = slot(op == DFS_OP_BWD_P_U ? WS_T : WS_S);
      return launch_stream_bwd_pass(SB_MATVEC, d, q, st);
    case DFS_OP_BWD_PT_T:  // s = P^T t (skips stopped problems once the CG has started)
      if (tile_path_ok(bp.in_dtype, d, N, bp.K, bp.Q)) {
        TileArgs ta = tile_args(bp, r0, r1, split, ext);
        ta.A = bp.K; ta.Bop = bp.Q;
        ta.col_bias = slot(WS_F); ta.col_vec = slot(WS_T);
        ta.row_bias = slot(WS_G);
        ta.done = v.done;
        ta.row_out = slot(WS_S);
        ta.ct = terms(true);
        return launch_tile_pass(TL_MATVEC, ta, st);
      }
      q.Aop = bp.K; q.Bop = bp.Q;
      q.tv[0] = slot(WS_F); q.tv[1] = slot(WS_T);
      q.rv[0] = slot(WS_G);
      q.done = v.done;
      q.out0 = slot(WS_S);
      return launch_stream_bwd_pass(SB_MATVEC, d, q, st);
    case DFS_OP_BWD_CGSTEP_FIRST:
    case DFS_OP_BWD_CGSTEP:
      return launch_dependent(sb_cgstep_kernel, dim3(pblocks), dim3(kVThreads), 0, st, v,
                              op == DFS_OP_BWD_CGSTEP_FIRST ? 1 : 0);
    case DFS_OP_BWD_FINAL:
      return launch_dependent(sb_final_kernel, dim3(pblocks), dim3(kVThreads), 0, st, v);
    case DFS_OP_BWD_DQ:    // dQ = dS K / (eps_h sqrt d)
      if (bt) {
        ba.A = cp.Qf; ba.A2 = cp.dOf; ba.Bop = cp.Kf; ba.B2 = cp.Vf; ba.B3 = cp.KT;
        ba.tv[0] = slot(WS_G); ba.tv[1] = slot(WS_X2); ba.pot_mask = 1;
        ba.rv[0] = slot(WS_F); ba.rv[1] = slot(WS_FM); ba.rv[2] = slot(WS_INVR); ba.rv[3] = slot(WS_D);
        ba.rv[4] = slot(WS_W1);
        ba.xvec = bp.dxc ? bp.x_res : nullptr; ba.xvec_per_head = 0;
        ba.rxvec = bp.dxc; ba.rxvec_per_head = 1;
        ba.acc = bp.dQ; ba.acc_scale = -1.0f;
        ba.ct = terms(false);
        if (want_dx && geo) ba.cg.dx = cg_dx_row;
        if (cgw != nullptr && bp.dw_dist != nullptr && geo) ba.cg.dw = cg_dw;
        if (cgw != nullptr && bp.dr_head != nullptr && geo) ba.cg.dr = cg_dr;
        if (cgw != nullptr && bp.dpos_weight != nullptr && bins != nullptr) ba.cg.dpos = cg_dpos;
        return launch_bt_pass(BTP_DQ, ba, st);
      }
      q.Aop = bp.Q; q.Bop = bp.K; q.A2op = bp.dO; q.a2_f32 = 1; q.B2op = bp.V; q.B3op = bp.K;
      q.tv[0] = slot(WS_G); q.tv[1] = slot(WS_X2);
      q.rv[0] = slot(WS_F); q.rv[1] = slot(WS_FM); q.rv[2] = slot(WS_INVR); q.rv[3] = slot(WS_D);
      q.rv[4] = slot(WS_W1);
      q.xvec = bp.dxc ? bp.x_res : nullptr; q.xvec_per_head = 0;
      q.rxvec = bp.dxc; q.rxvec_per_head = 1;
      q.acc0 = bp.dQ;
      q.acc_scale0 = -1.0f;  // negative: 1/(eps_h sqrt d) of the problem's head
      return launch_stream_bwd_pass(SB_DQ, d, q, st);
    case DFS_OP_BWD_DKV:   // dK = dS^T Q / (eps_h sqrt d), dV = T_norm^T dO (dV already done on the TMA path)
      if (bt) {
        ba.A = cp.Kf; ba.A2 = cp.Vf; ba.Bop = cp.Qf; ba.B2 = cp.dOf; ba.B3 = cp.QT;
        ba.tv[0] = slot(WS_F); ba.tv[1] = slot(WS_FM); ba.tv[2] = slot(WS_INVR); ba.tv[3] = slot(WS_D);
        ba.tv[4] = slot(WS_W1); ba.pot_mask = 3;
        ba.rv[0] = slot(WS_G); ba.rv[1] = slot(WS_X2);
        ba.xvec = bp.dxc; ba.xvec_per_head = 1;
        ba.rxvec = bp.dxc ? bp.x_res : nullptr; ba.rxvec_per_head = 0;
        ba.acc = bp.dK; ba.acc_scale = -1.0f;
        ba.ct = terms(true);
        if (want_dx && geo) ba.cg.dx = cg_dx_col;
        cudaError_t e = launch_bt_pass(BTP_DK, ba, st);
        if (e != cudaSuccess || cgw == nullptr) return e;
        // the shared-parameter gradients from the shares of the DQ, DK and COL passes
        const int shares = (want_dx && geo ? 3 : 0) | (want_dx && bp.dxc != nullptr ? 4 : 0);
        float* dx_out = want_dx ? bp.dx_res : nullptr;
        float* dw_out = geo ? bp.dw_dist : nullptr;
        float* dpos_out = bins != nullptr ? bp.dpos_weight : nullptr;
        float* dr_out = geo ? bp.dr_head : nullptr;
        if (dx_out != nullptr && shares == 0) {  // x_res enters neither the cost nor the loss
          if ((e = cudaMemsetAsync(dx_out, 0, sizeof(float) * B * N * 3, st)) != cudaSuccess) return e;
          dx_out = nullptr;
        }
        const int cnt =
            (dx_out ? B * N * 3 : 0) + (dw_out ? H : 0) + (dpos_out ? H * kBinCount : 0) + (dr_out ? H : 0);
        if (cnt == 0) return cudaSuccess;
        stream_costgrad_finalize<<<(cnt + 255) / 256, 256, 0, st>>>(cg_dx_row, cg_dx_col, cg_dx_t, cg_dw, cg_dpos,
                                                                    cg_dr, shares, B, H, N, dx_out, dw_out,
                                                                    dpos_out, dr_out);
        return cudaGetLastError();
      }
      q.Aop = bp.K; q.Bop = bp.Q; q.A2op = bp.V; q.B2op = bp.dO; q.b2_f32 = 1;
      q.B3op = bp.Q; q.B4op = bp.dO; q.b4_f32 = 1;
      q.tv[0] = slot(WS_F); q.tv[1] = slot(WS_FM); q.tv[2] = slot(WS_INVR); q.tv[3] = slot(WS_D);
      q.tv[4] = slot(WS_W1);
      q.rv[0] = slot(WS_G); q.rv[1] = slot(WS_X2);
      q.xvec = bp.dxc; q.xvec_per_head = 1;
      q.rxvec = bp.dxc ? bp.x_res : nullptr; q.rxvec_per_head = 0;
      q.acc0 = bp.dK;
      q.acc1 = bp.dV;
      q.acc_scale0 = -1.0f;
      q.acc_scale1 = 1.0f;
      return launch_stream_bwd_pass(SB_DKV, d, q, st);
    default:
      return cudaErrorInvalidValue;
  }
}

// The whole streamed backward on one GPU: every phase over all rows.
namespace {

// A private stream per device on which the CG loop's body is recorded (stream
// capture records launches without running them; the caller's stream may be
// the legacy default stream, which cannot be captured).
constexpr int kCaptureDevices = 64;
cudaStream_t capture_stream(int dev) {
  static std::mutex mu;
  static cudaStream_t streams[kCaptureDevices] = {};
  if (dev < 0 || dev >= kCaptureDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (streams[dev] == nullptr) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return nullptr;
    if (cur != dev && cudaSetDevice(dev) != cudaSuccess) return nullptr;
    cudaStream_t s = nullptr;
    const cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (cur != dev) cudaSetDevice(cur);
    if (e != cudaSuccess) return nullptr;
    streams[dev] = s;
  }
  return streams[dev];
}

// CG rounds 1 .. max_iter as one CUDA graph launched on `st`: a kernel that
// sets the loop condition, then a WHILE node whose body is one round
// (t = D1^-1 P u, s = P^T t, the CG step, the condition again).  The loop stops
// on the device as soon as every problem's solve has stopped, so no launches
// run after convergence and the host never waits.  Returns false (and leaves
// nothing queued) when the runtime cannot build or launch such a graph; the
// caller then issues the rounds one by one.
bool cg_loop_graph(const BwdParams& bp, float* wsp, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return false;  // inside the caller's own capture: plain launches
  }
  int dev = 0;
  if (cudaStreamGetDevice(st, &dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  cudaStream_t cap = capture_stream(dev);
  if (cap == nullptr) return false;
  static std::mutex capture_mu;  // one recording at a time on the shared capture streams
  std::lock_guard<std::mutex> lock(capture_mu);
  const size_t n = static_cast<size_t>(bp.B) * bp.H * bp.N, nbh = static_cast<size_t>(bp.B) * bp.H;
  float* sc = wsp + WS_NUM * n;
  int32_t* done = reinterpret_cast<int32_t*>(sc + SC_NUM * nbh);
  int32_t* rounds = reinterpret_cast<int32_t*>(sc + SC_LOOP);
  const int nprob = static_cast<int>(nbh), max_rounds = bp.cg_max_iter;
  cudaGraph_t g = nullptr, body = nullptr;
  cudaGraphExec_t ex = nullptr;
  cudaGraphNode_t first = nullptr, loop = nullptr;
  bool ok = cudaGraphCreate(&g, 0) == cudaSuccess;
  cudaGraphConditionalHandle cond = 0;
  ok = ok && cudaGraphConditionalHandleCreate(&cond, g, 0, cudaGraphCondAssignDefault) == cudaSuccess;
  if (ok) {
    int reset = 1;
    void* args[] = {&done, const_cast<int*>(&nprob), &rounds, const_cast<int*>(&max_rounds), &reset, &cond};
    cudaKernelNodeParams kp = {};
    kp.func = reinterpret_cast<void*>(sb_loopcond_kernel);
    kp.gridDim = dim3(1);
    kp.blockDim = dim3(256);
    kp.kernelParams = args;
    ok = cudaGraphAddKernelNode(&first, g, nullptr, 0, &kp) == cudaSuccess;
  }
  if (ok) {
    cudaGraphNodeParams np = {};
    np.type = cudaGraphNodeTypeConditional;
    np.conditional.handle = cond;
    np.conditional.type = cudaGraphCondTypeWhile;
    np.conditional.size = 1;
    ok = cudaGraphAddNode(&loop, g, &first, 1, &np) == cudaSuccess;
    if (ok) body = np.conditional.phGraph_out[0];
  }
  if (ok) ok = cudaStreamBeginCaptureToGraph(cap, body, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed) ==
               cudaSuccess;
  if (ok) {
    cudaError_t e = stream_bwd_op(DFS_OP_BWD_P_U, bp, wsp, 0, bp.N, cap);
    if (e == cudaSuccess) e = stream_bwd_op(DFS_OP_BWD_PT_T, bp, wsp, 0, bp.N, cap);
    if (e == cudaSuccess) e = stream_bwd_op(DFS_OP_BWD_CGSTEP, bp, wsp, 0, bp.N, cap);
    if (e == cudaSuccess) {
      sb_loopcond_kernel<<<1, 256, 0, cap>>>(done, nprob, rounds, max_rounds, 0, cond);
      e = cudaGetLastError();
    }
    cudaGraph_t captured = nullptr;
    const cudaError_t ee = cudaStreamEndCapture(cap, &captured);
    ok = e == cudaSuccess && ee == cudaSuccess;
  }
  if (ok) ok = cudaGraphInstantiate(&ex, g, 0) == cudaSuccess;
  if (ok) ok = cudaGraphLaunch(ex, st) == cudaSuccess;
  // an executable graph destroyed while in flight is freed once it completes
  if (ex != nullptr) cudaGraphExecDestroy(ex);
  if (g != nullptr) cudaGraphDestroy(g);
  if (!ok) cudaGetLastError();  // the failure is handled by the caller's fallback
  return ok;
}

}  // namespace

// The same device-terminated loop for one rank of a row-sharded run: each round
// runs the plan products on this rank's rows, gathers their slots (t, then s)
// from every rank through peer memory, and takes the CG step.  The stop flags
// come from the gathered vectors, identical on every rank, so every rank's
// loop runs the same rounds; the gathers' waits count on the device, so the
// recorded graph needs no per-round argument and the host never waits.
bool cg_loop_graph_peer(const BwdParams& bp, float* wsp, int r0, int r1, const PeerInfo& pi, size_t counter_offset,
                        cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return false;
  }
  int dev = 0;
  if (cudaStreamGetDevice(st, &dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  cudaStream_t cap = capture_stream(dev);
  if (cap == nullptr) return false;
  static std::mutex capture_mu;
  std::lock_guard<std::mutex> lock(capture_mu);
  const size_t n = static_cast<size_t>(bp.B) * bp.H * bp.N, nbh = static_cast<size_t>(bp.B) * bp.H;
  float* sc = wsp + WS_NUM * n;
  int32_t* done = reinterpret_cast<int32_t*>(sc + SC_NUM * nbh);
  int32_t* rounds = reinterpret_cast<int32_t*>(sc + SC_LOOP);
  const int nprob = static_cast<int>(nbh), max_rounds = bp.cg_max_iter;
  const size_t slot_bytes = sizeof(float) * n;
  cudaGraph_t g = nullptr, body = nullptr;
  cudaGraphExec_t ex = nullptr;
  cudaGraphNode_t first = nullptr, loop = nullptr;
  bool ok = cudaGraphCreate(&g, 0) == cudaSuccess;
  cudaGraphConditionalHandle cond = 0;
  ok = ok && cudaGraphConditionalHandleCreate(&cond, g, 0, cudaGraphCondAssignDefault) == cudaSuccess;
  if (ok) {
    int reset = 1;
    void* args[] = {&done, const_cast<int*>(&nprob), &rounds, const_cast<int*>(&max_rounds), &reset, &cond};
    cudaKernelNodeParams kp = {};
    kp.func = reinterpret_cast<void*>(sb_loopcond_kernel);
    kp.gridDim = dim3(1);
    kp.blockDim = dim3(256);
    kp.kernelParams = args;
    ok = cudaGraphAddKernelNode(&first, g, nullptr, 0, &kp) == cudaSuccess;
  }
  if (ok) {
    cudaGraphNodeParams np = {};
    np.type = cudaGraphNodeTypeConditional;
    np.conditional.handle = cond;
    np.conditional.type = cudaGraphCondTypeWhile;
    np.conditional.size = 1;
    ok = cudaGraphAddNode(&loop, g, &first, 1, &np) == cudaSuccess;
    if (ok) body = np.conditional.phGraph_out[0];
  }
  if (ok) ok = cudaStreamBeginCaptureToGraph(cap, body, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed) ==
               cudaSuccess;
  if (ok) {
    cudaError_t e = stream_bwd_op(DFS_OP_BWD_P_U, bp, wsp, r0, r1, cap);
    if (e == cudaSuccess)
      e = peer_gather_rows(pi, WS_T * slot_bytes, nprob, bp.N, 1, r0, r1, counter_offset, bp.status, cap);
    if (e == cudaSuccess) e = stream_bwd_op(DFS_OP_BWD_PT_T, bp, wsp, r0, r1, cap);
    if (e == cudaSuccess)
      e = peer_gather_rows(pi, WS_S * slot_bytes, nprob, bp.N, 1, r0, r1, counter_offset, bp.status, cap);
    if (e == cudaSuccess) e = stream_bwd_op(DFS_OP_BWD_CGSTEP, bp, wsp, 0, bp.N, cap);
    if (e == cudaSuccess) {
      sb_loopcond_kernel<<<1, 256, 0, cap>>>(done, nprob, rounds, max_rounds, 0, cond);
      e = cudaGetLastError();
    }
    cudaGraph_t captured = nullptr;
    const cudaError_t ee = cudaStreamEndCapture(cap, &captured);
    ok = e == cudaSuccess && ee == cudaSuccess;
  }
  if (ok) ok = cudaGraphInstantiate(&ex, g, 0) == cudaSuccess;
  if (ok) ok = cudaGraphLaunch(ex, st) == cudaSuccess;
  if (ex != nullptr) cudaGraphExecDestroy(ex);
  if (g != nullptr) cudaGraphDestroy(g);
  if (!ok) cudaGetLastError();
  return ok;
}

cudaError_t launch_stream_bwd(const BwdParams& bp, float* wsp, cudaStream_t st) {
  const int N = bp.N;
  cudaError_t e = cudaSuccess;
  auto run = [&](int op) {
    if (e == cudaSuccess) e = stream_bwd_op(op, bp, wsp, 0, N, st);
  };
  run(DFS_OP_BWD_PREP);
  run(DFS_OP_BWD_ROWSTATS);
  run(DFS_OP_BWD_ROWDERIVE);
  run(DFS_OP_BWD_COLSTATS);
  run(DFS_OP_BWD_SETUP);
  run(DFS_OP_BWD_PT_T);   // s = P^T D1^-1 b1 (no problem has stopped yet)
  run(DFS_OP_BWD_CGINIT);
  run(DFS_OP_BWD_P_U);    // the first CG round
  run(DFS_OP_BWD_PT_T);
  run(DFS_OP_BWD_CGSTEP_FIRST);
  // rounds 1 .. max_iter: a device-terminated loop, or one by one where the
  // runtime cannot run it (rounds after convergence then exit early per problem)
  if (e == cudaSuccess && bp.cg_max_iter > 0 && !cg_loop_graph(bp, wsp, st)) {
    for (int it = 1; it <= bp.cg_max_iter; ++it) {
      run(DFS_OP_BWD_P_U);
      run(DFS_OP_BWD_PT_T);
      run(DFS_OP_BWD_CGSTEP);
    }
  }
  run(DFS_OP_BWD_P_X);
  run(DFS_OP_BWD_FINAL);
  run(DFS_OP_BWD_DQ);
  run(DFS_OP_BWD_DKV);
  return e;
}

}  // namespace dfs
