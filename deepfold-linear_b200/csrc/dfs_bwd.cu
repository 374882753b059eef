// dfs_bwd.cu -- resident flash-Sinkhorn backward for sm_100a: implicit-function
// theorem adjoint solved by conjugate gradient on the device.
//
// Same cluster decomposition as the forward: cluster rank c owns rows
// [64c, 64c+64) ("row slab") and, for the transposed half of the work, the
// same range of columns ("column slab").  With the fixed point (f, g) from the
// forward, P = exp(f + S + g), r = P 1, c = P^T 1 and the kappa-damped updates
// f = kappa (a - LSE_j(S + g)), g = kappa (b - LSE_i(S + f)), the adjoint of
// the fixed-point map is the symmetric PSD system
//
//     [ diag(r)/kappa   P            ] [w1]   [ dL/df ]
//     [ P^T             diag(c)/kappa] [w2] = [ dL/dg ]
//
// whose solution gives dL/dS = E - P o (w1 (+) w2), dL/dlog_mu = r o w1 and
// dL/dlog_nu = c o w2, where E = T_norm o (dT - D) is the direct gradient through
// the transport output, dT = dO V^T (+ dxc x^T), D = rowsum(T_norm o dT).
// For kappa = 1 the system is singular along (1, -1): the right-hand side is
// projected onto its range and the null-space component of w removed (dL/dS
// does not depend on it).  At a converged forward this equals the reference's
// unrolled K-step gradient (src/deepfold/model/kernels/sinkhorn_kernel.py:2086-2382).
//
// Phases (all MMAs tcgen05 kind::tf32, K-major operands, accumulators in TMEM):
//   1  row slab:    S = Q_s K^T -> P, r, T_norm           (registers)
//   2               dT = dO_s V^T -> E (in shared memory), D; one cluster
//                   exchange of the column sums c = P^T 1 and g_v = E^T 1
//   3  CG:          on the Schur complement of the row block (preconditioner
//                   D2), Chronopoulos-Gear form: per iteration one P / P^T
//                   product pair, one cluster exchange, three CTA barriers
//   4               all-gather w1, f, 1/rowsum, D; marginal gradients
//   5               dS = E - P (w1 + w2);  dQ = dS K
//   6  column slab: S^T = K_s Q^T -> P^T                     (registers)
//   7               dT^T = V_s dO^T,  dV = T_norm^T dO
//   8               dS^T = T_norm^T (dT^T - D) - P^T (w1 + w2);  dK = dS^T Q
// Every row or column is owned by exactly one CTA: no atomics, deterministic.
// Element loops over the register slab are branch-free; optional terms (dxc,
// bias) are separate rolled passes over the shared-memory tile.
//
// Gradients of the shared cost parameters (sinkhorn_kernel.py:2366-2382 of the
// reference returns them): with dC = -dS / eps,
//   dw_h    = sum_ij dC_ij dist_ij / (r_h + dist_ij)
//   dr_h    = -w_h sum_ij dC_ij dist_ij / (r_h + dist_ij)^2
//   dx_i    = sum_j dC_ij c_ij (x_i - x_j) + sum_j dC_ji c_ji (x_i - x_j) + (T_norm^T dxc)_i,
//             c_ij = w_h r_h / ((r_h + dist_ij)^2 dist_ij)
//   dpos[h, b] = sum over the entries with bins_ij = b of dC_ij
// (r_h = r_head[h], or r_0) are accumulated from the staged dS tile of phase 5
// (row part, dw, dr, bins), the
// staged T_norm^T of phase 7 (centroid part) and the staged dS^T of phase 8
// (column part), per slab row and per CTA into the workspace; the bin histogram
// is summed in 64-bit fixed point (scale from the tile's largest |dC|), so its
// integer atomics are exact and order-free.  resident_costgrad_finalize sums the
// partials over heads, CTAs and batch elements in a fixed order.
#include "dfs_slab.cuh"

namespace dfs {

// column-indexed vectors; FA/INV/DD/W1 hold all N rows after the all-gather
enum { BC_G = 0, BC_OK, BC_U2, BC_SOL2, BC_FA, BC_INV, BC_DD, BC_W1, BC_CC, BC_X0, BC_X1, BC_X2, BC_NUM };
// slab-row vectors: coordinates and per-row values kept out of registers
enum { BR_X0 = 0, BR_X1, BR_X2, BR_INV, BR_D, BR_F, BR_NUM };

template <int C, int DH>
struct BwdCfg {
  static constexpr int NP = 64 * C;
  static constexpr int NS = NP / 32;
  static constexpr uint32_t OFF_T = 0;                                // 64 x NP fp32 staging
  static constexpr uint32_t OFF_SA = OFF_T + 256u * NP;               // 64 x DH slab operand
  static constexpr uint32_t OFF_DA = OFF_SA + 256u * DH;              // 64 x DH dO slab
  static constexpr uint32_t OFF_KV = OFF_DA + 256u * DH;              // NP x DH operand / partials
  // exchange rounds: phase 2 (2 NP + 4 floats), CG (NP + 4), phase 4 (260)
  static constexpr int RS = (2 * NP > 256 ? 2 * NP : 256) + 8;
  static constexpr uint32_t OFF_XR = OFF_KV + 4u * NP * DH;           // 2 x C x RS receive slots
  static constexpr uint32_t OFF_STG = OFF_XR + 8u * C * RS;           // 2 x RS stages
  static constexpr uint32_t OFF_COL = OFF_STG + 8u * RS;              // column / all-row vectors
  static constexpr uint32_t OFF_ROW = OFF_COL + 4u * BC_NUM * NP;     // slab-row vectors
  static constexpr uint32_t OFF_MISC = OFF_ROW + 4u * BR_NUM * 64;    // 192 floats, barriers
  static constexpr uint32_t SMEM_NEED = OFF_MISC + 1024 + 1024;
  static constexpr uint32_t SMEM = SMEM_NEED > 122880u ? SMEM_NEED : 122880u;
  static_assert(SMEM <= 232448u, "exceeds the 227 KB of shared memory a CTA can use");
  static_assert(kWarps * 2u * NP * 4 <= 4u * NP * DH, "column partials must fit the K/V region");
  static_assert(NP + DH <= 512, "TMEM columns");
  static_assert(8u * C * RS >= 1600u + 4u * 2 * kWarps, "cost-gradient scratch must fit the exchange slots");
};

// Workspace of the shared-parameter gradients (floats): per (batch, head,
// point) the three dx partials, then per (batch, head, CTA) the dw partial, the
// 68 position-bin partials and the dr partial.
struct CostGradWs {
  float* dx;    // (B*H, N, 3)
  float* dw;    // (B*H, C)
  float* dpos;  // (B*H, C, 68)
  float* dr;    // (B*H, C)
};
__host__ __device__ inline CostGradWs costgrad_ws(float* ws, int B, int H, int N) {
  const size_t bh = static_cast<size_t>(B) * H, C = (N + 63) / 64;
  CostGradWs w;
  w.dx = ws;
  w.dw = ws + bh * N * 3;
  w.dpos = w.dw + bh * C;
  w.dr = w.dpos + bh * C * 68;
  return w;
}
constexpr int kBins = 68;

template <int C, int DH>
__global__ void __launch_bounds__(kThreads, 1) resident_bwd_kernel(const BwdParams p) {
  using Cfg = BwdCfg<C, DH>;
  constexpr int NP = Cfg::NP, NS = Cfg::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* Ts = reinterpret_cast<float*>(base + Cfg::OFF_T);
  float* SA = reinterpret_cast<float*>(base + Cfg::OFF_SA);
  float* DA = reinterpret_cast<float*>(base + Cfg::OFF_DA);
  float* KV = reinterpret_cast<float*>(base + Cfg::OFF_KV);
  float* colv = reinterpret_cast<float*>(base + Cfg::OFF_COL);
  float* rowv = reinterpret_cast<float*>(base + Cfg::OFF_ROW);
  float* misc = reinterpret_cast<float*>(base + Cfg::OFF_MISC);  // [0,64) and [64,128): per-warp sums
  uint64_t* mbar = reinterpret_cast<uint64_t*>(base + Cfg::OFF_MISC + 768);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + Cfg::OFF_MISC + 784);
  BulkExchange<C, Cfg::RS> ex{reinterpret_cast<float*>(base + Cfg::OFF_XR),
                              reinterpret_cast<float*>(base + Cfg::OFF_STG),
                              reinterpret_cast<uint64_t*>(base + Cfg::OFF_MISC + 800), 0, 0u, 0, false};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int crank = static_cast<int>(cluster_rank());
  ex.rank = crank;
  const int prob = blockIdx.x / C;
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const int row0 = 64 * crank;
  const size_t bh = static_cast<size_t>(bb) * p.H + hh;
  const float eps_h = p.eps[hh];
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
  const float s_scale = kLog2e / eps_h;
  const float qk_scale = s_scale * p.qk_scale;
  const float grad_scale = p.qk_scale / eps_h;   // dS -> dQ, dK
  const float w_h = p.w_dist ? p.w_dist[hh] : 0.0f;
  const float r_h = p.r_head != nullptr ? p.r_head[hh] : p.r_0;  // geometry scale of this head
  int err = 0;
  uint32_t mma_phase = 0;

  auto mma_wait = [&]() {
    if (!mbar_wait(mbar, mma_phase & 1)) err |= DFS_ERR_DEVICE_TIMEOUT;
    ++mma_phase;
    tc_fence_after();
  };
  // all generic-proxy smem writes done and visible to the tensor core, TMEM
  // reads of earlier accumulators finished
  auto operands_ready = [&]() {
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  // sum of the 16 per-warp partials slot[0..15] (broadcast float4 loads, fixed order)
  auto sum16 = [](const float* slot) -> float {
    const float4 a = *reinterpret_cast<const float4*>(slot), b = *reinterpret_cast<const float4*>(slot + 4),
                 c = *reinterpret_cast<const float4*>(slot + 8), d = *reinterpret_cast<const float4*>(slot + 12);
    return (((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w))) +
           (((c.x + c.y) + (c.z + c.w)) + ((d.x + d.y) + (d.z + d.w)));
  };
  // CTA-wide sums of three per-thread values with one barrier; `slot` is one of
  // the two 64-float regions of misc, laid out [value][warp].  Per warp: a
  // 4-value transpose-reduce (6 shuffles) leaves lanes 0, 8, 16 with the warp
  // totals; after the barrier each warp loads the 16 partials of each value
  // (32-bit loads, one wavefront) and finishes with a 4-level xor butterfly,
  // which gives every lane (and every CTA, for identical inputs) the same bits.
  auto cta_sum3 = [&](float a, float b, float c, float* slot, float& A, float& B, float& Cs) {
    const float v4[4] = {a, b, c, 0.0f};
    const float v = reduce4_rows<false>(v4, lane);  // lane l: total of value (l >> 3) & 3
    if ((lane & 7) == 0 && lane < 24) slot[(lane >> 3) * 16 + warp] = v;
    __syncthreads();
    const int l16 = lane & 15;
    float x = slot[l16], y = slot[16 + l16], z = slot[32 + l16];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      x += __shfl_xor_sync(0xffffffffu, x, o);
      y += __shfl_xor_sync(0xffffffffu, y, o);
      z += __shfl_xor_sync(0xffffffffu, z, o);
    }
    A = x;
    B = y;
    Cs = z;
  };

  // ---------------------------------------------------------------- setup
  if (tid == 0) {  // this CTA's slab of every operand into L2
    const int es = p.in_dtype == DFS_F32 ? 4 : 2;
    prefetch_slab_l2(p.Q, bh * N, row0, N, DH, es);
    prefetch_slab_l2(p.K, bh * N, row0, N, DH, es);
    prefetch_slab_l2(p.V, bh * N, row0, N, DH, es);
    prefetch_slab_l2(p.dO, bh * N, row0, N, DH, 4);
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  if (tid == 0) {
    mbar_init(mbar, 1);
    ex.init();
    fence_mbar_init();
  }
  const bool colt = tid < NP;  // column threads (whole warps)
  const int jc = col_of_thread(warp, lane);
  if (colt) {
    const bool ok = jc < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + jc] != 0.0f);
    colv[BC_OK * NP + jc] = ok ? 1.0f : 0.0f;
    colv[BC_G * NP + jc] = ok ? p.log_v[bh * N + jc] * kLog2e : 0.0f;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      colv[(BC_X0 + c) * NP + jc] =
          (p.x_res && jc < N) ? p.x_res[(static_cast<size_t>(bb) * N + jc) * 3 + c] : 0.0f;
  }
  if (tid < 64) {
    const int gi = row0 + tid;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      rowv[(BR_X0 + c) * 64 + tid] =
          (p.x_res && gi < N) ? p.x_res[(static_cast<size_t>(bb) * N + gi) * 3 + c] : 0.0f;
  }
  load_operand<DH, 64>(SA, p.Q, p.in_dtype, bh * N, row0, N, tid);
  load_operand<DH, NP>(KV, p.K, p.in_dtype, bh * N, 0, N, tid);
  load_operand_f32<DH, 64>(DA, p.dO, bh * N, row0, N, tid);
  operands_ready();
  if constexpr (C > 1) cluster_sync();  // every CTA's exchange mbarriers initialised
  const uint32_t tbase = *tslot;

  const bool bias_on = p.pos_weight != nullptr || (p.x_res != nullptr && w_h != 0.0f);
  // subtract the position / geometry terms from the staged S' (built here so
  // that none of it occupies registers in between)
  auto add_bias = [&](bool transposed) {
    BiasArgs bias;
    bias.pos_weight = p.pos_weight;
    bias.bins = bin_source(p);
    bias.xrow = rowv + BR_X0 * 64;
    bias.xcol = colv + BC_X0 * NP;
    bias.geo = p.x_res != nullptr && w_h != 0.0f;
    bias.w_h = w_h;
    bias.r_0 = r_h;
    bias.s_scale = s_scale;
    bias.bb = bb;
    bias.hh = hh;
    bias.N = N;
    bias.row0 = row0;
    bias.transposed = transposed;
    add_cost_bias_stage<NP>(Ts, bias, tid);
  };

  const int rho = (lane >> 3) & 3;  // row whose totals this lane holds after reduce4_rows
  const int li_own = kRpw * warp + rho, grow = row0 + li_own;
  const bool rok = grow < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + grow] != 0.0f);
  const bool own = ((lane & 7) == 0) & rok;  // one lane per valid row for row sums
  uint32_t rokm = 0, cokm = 0;
#pragma unroll
  for (int r = 0; r < kRpw; ++r) {
    const int gi = row0 + kRpw * warp + r;
    const bool ok = gi < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + gi] != 0.0f);
    rokm |= ok ? (1u << r) : 0u;
  }
#pragma unroll
  for (int k = 0; k < NS; ++k) cokm |= (colv[BC_OK * NP + 32 * k + lane] != 0.0f) ? (1u << k) : 0u;
  const float fr = rok ? p.log_u[bh * N + grow] * kLog2e : 0.0f;
  if ((lane & 7) == 0) rowv[BR_F * 64 + li_own] = fr;
  // sum of a per-row value over this warp's 4 rows (lanes 0, 8, 16, 24 hold
  // one copy each); lane 0 ends with the warp total
  auto rows_sum = [&](float v) -> float {
    v = own ? v : 0.0f;
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    return v;
  };

  // ---------------------------------------------------------------- phase 1
  if (tid == 0) {
    issue_qk<NP, DH>(tbase, SA, KV);
    mma_commit(mbar);
  }
  mma_wait();
  drain_m64<NP>(Ts, tbase, 0, qk_scale, warp, lane);
  __syncthreads();
  if (bias_on) {
    add_bias(false);
    __syncthreads();
  }
  float P[kRpw][NS];
  stage_to_regs<NS>(P, Ts, warp, lane);
  float rsum_r, inv_r;
  {
    float fall[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) fall[r] = __shfl_sync(0xffffffffu, fr, 8 * r);
    float a[kRpw], m[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) a[r] = m[r] = 0.0f;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float g = colv[BC_G * NP + 32 * k + lane];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const bool ok = ((rokm >> r) & (cokm >> k) & 1u) != 0u;
        const float e = ex2(P[r][k] + fall[r] + g);
        P[r][k] = ok ? e : 0.0f;
        a[r] += P[r][k];
        m[r] = fmaxf(m[r], P[r][k]);
      }
    }
    rsum_r = reduce4_rows<false>(a, lane);
    const float pm = reduce4_rows<true>(m, lane);
    const float iv = 1.0f / (rsum_r + 1e-6f * pm);
    inv_r = (rok & (rsum_r > 0.0f)) ? iv : 0.0f;
    if (!isfinite(rsum_r)) err |= DFS_ERR_NUMERIC;
  }

  // ---------------------------------------------------------------- phase 2
  __syncthreads();  // Ts (S) fully read
  load_operand<DH, NP>(KV, p.V, p.in_dtype, bh * N, 0, N, tid);
  operands_ready();
  if (tid == 0) {
    issue_abt<NP, DH>(tbase, DA, KV);  // dT = dO_s V^T
    mma_commit(mbar);
  }
  mma_wait();
  drain_m64<NP>(Ts, tbase, 0, 1.0f, warp, lane);
  __syncthreads();
  if (p.dxc) {  // dT[i][j] += dxc_i . x_j
#pragma unroll 1
    for (int idx = tid; idx < 64 * NP; idx += kThreads) {
      const int li = idx / NP, gj = idx - li * NP, gi = row0 + li;
      if (gi < N) {
        const float* dx = p.dxc + (bh * N + gi) * 3;
        Ts[sw_off(li, gj, 64) >> 2] += dx[0] * colv[BC_X0 * NP + gj] + dx[1] * colv[BC_X1 * NP + gj] +
                                       dx[2] * colv[BC_X2 * NP + gj];
      }
    }
    __syncthreads();
  }
  float* red = KV;  // V is no longer needed: 2 x kWarps x NP column partials (P and E)
  float fbar_r, D_r;
  {
    float inv[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) inv[r] = __shfl_sync(0xffffffffu, inv_r, 8 * r);
    float accD[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) s = fmaf(P[r][k], Ts[sw_off(kRpw * warp + r, 32 * k + lane, 64) >> 2], s);
      accD[r] = s;
    }
    D_r = inv_r * reduce4_rows<false>(accD, lane);  // D = sum_j T_norm dT
    float D[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) D[r] = __shfl_sync(0xffffffffu, D_r, 8 * r);
    float re[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) re[r] = 0.0f;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int j = 32 * k + lane;
      float cp = 0.0f, ce = 0.0f;
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const uint32_t o = sw_off(kRpw * warp + r, j, 64) >> 2;
        const float e = P[r][k] * inv[r] * (Ts[o] - D[r]);
        Ts[o] = e;
        ce += e;
        cp += P[r][k];
        re[r] += e;
      }
      red[warp * NP + j] = cp;
      red[kWarps * NP + warp * NP + j] = ce;
    }
    fbar_r = reduce4_rows<false>(re, lane);
    if ((lane & 7) == 0) {
      rowv[BR_INV * 64 + li_own] = inv_r;
      rowv[BR_D * 64 + li_own] = D_r;
    }
  }
  {
    const float sf = rows_sum(fbar_r), sr = rows_sum(rsum_r);
    if (lane == 0) {
      misc[warp] = sf;
      misc[16 + warp] = sr;
    }
  }
  __syncthreads();
  if (colt) {
    ex.stage()[jc] = colsum16<NP>(red, warp, lane);
    ex.stage()[NP + jc] = colsum16<NP>(red + kWarps * NP, warp, lane);
  }
  if (tid == kThreads - 32) {  // last warp: no column work (NP <= 384 < 512)
    ex.stage()[2 * NP] = sum16(misc);
    ex.stage()[2 * NP + 1] = sum16(misc + 16);
  }
  if (!ex.exchange(tid, 4u * (2 * NP + 4))) err |= DFS_ERR_DEVICE_TIMEOUT;
  float cc = 0.0f, gv = 0.0f, okc = 0.0f;
  if (colt) {
    cc = ex.from(0)[jc];
    gv = ex.from(0)[NP + jc];
#pragma unroll
    for (int c = 1; c < C; ++c) {
      cc += ex.from(c)[jc];
      gv += ex.from(c)[NP + jc];
    }
    okc = colv[BC_OK * NP + jc];
    colv[BC_CC * NP + jc] = cc;
  }
  float sum_fbar = 0.0f, sum_r = 0.0f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    sum_fbar += ex.from(c)[2 * NP];
    sum_r += ex.from(c)[2 * NP + 1];
  }
  ex.next();

  // ---------------------------------------------------------------- phase 3 (CG)
  // The Jacobi-preconditioned block system is 2-cyclic, so CG on it takes
  // twice the iterations of CG on its Schur complement
  //     S w2 = b2 - P^T D1^-1 b1,   S = D2 - P^T D1^-1 P,   preconditioner D2,
  // followed by w1 = D1^-1 (b1 - P w2).  Rows are CTA-local, so one S
  // product costs one cluster exchange (the column partials of P^T t).
  const bool cok = okc != 0.0f;
  const float d1 = (rok & (rsum_r > 0.0f)) ? rsum_r / kap : 0.0f;
  const float d1i = d1 > 0.0f ? 1.0f / d1 : 0.0f;
  const float d2 = (cok & (cc > 0.0f)) ? cc / kap : 0.0f;
  const float d2i = d2 > 0.0f ? 1.0f / d2 : 0.0f;
  float b1 = rok ? fbar_r : 0.0f;
  float b2 = cok ? gv : 0.0f;
  if (kap >= 1.0f) {  // project [b1; b2] onto the range of the singular system
    float s2, nv, unused;
    cta_sum3(b2, cok ? 1.0f : 0.0f, 0.0f, misc + 64, s2, nv, unused);
    const float sh = nv > 0.0f ? (sum_fbar - s2) / (2.0f * nv) : 0.0f;
    b1 = rok ? b1 - sh : 0.0f;
    b2 = cok ? b2 + sh : 0.0f;
  }

  // P x for a column vector x (value of column thread jc); returns the row
  // value (held by all 8 lanes of the row's group).  One barrier.
  auto p_apply = [&](float xcol) -> float {
    if (colt) colv[BC_U2 * NP + jc] = xcol;
    __syncthreads();
    float acc[kRpw] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float xk = colv[BC_U2 * NP + 32 * k + lane];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) acc[r] = fmaf(P[r][k], xk, acc[r]);
    }
    return reduce4_rows<false>(acc, lane);
  };
  // P^T t for a row vector t (held by the row's lanes); returns the value of
  // column jc (column threads).  One barrier and one cluster exchange.
  auto pt_apply = [&](float trow) -> float {
    float ta[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) ta[r] = __shfl_sync(0xffffffffu, trow, 8 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      float sk = 0.0f;
#pragma unroll
      for (int r = 0; r < kRpw; ++r) sk = fmaf(P[r][k], ta[r], sk);
      red[warp * NP + 32 * k + lane] = sk;
    }
    __syncthreads();
    if (colt) ex.stage()[jc] = colsum16<NP>(red, warp, lane);
    if (!ex.exchange(tid, 4u * (NP + 4))) err |= DFS_ERR_DEVICE_TIMEOUT;
    float t = 0.0f;
    if (colt) {
      t = ex.from(0)[jc];
#pragma unroll
      for (int c = 1; c < C; ++c) t += ex.from(c)[jc];
    }
    ex.next();
    return t;
  };
  // S x = D2 x - P^T D1^-1 P x
  auto schur = [&](float xcol) -> float {
    const float q = p_apply(xcol);
    const float s = pt_apply(rok ? q * d1i : 0.0f);
    const float y = d2 * xcol - s;
    return cok ? y : 0.0f;
  };

  // Chronopoulos-Gear CG (one fused CTA reduction of (r,u), (w,u), (r,r) per
  // iteration); every CTA holds all columns, so these dots need no exchange
  // and are bit-identical across the cluster (uniform control flow).
  const float bs = pt_apply(rok ? b1 * d1i : 0.0f);
  float res2 = cok ? b2 - bs : 0.0f;
  float x2 = 0.0f, p2 = 0.0f, s2v = 0.0f, u2 = res2 * d2i;
  float w2 = schur(u2), ru, wu, rr;
  cta_sum3(res2 * u2, w2 * u2, res2 * res2, misc + 64, ru, wu, rr);
  const float nrm0 = sqrtf(fmaxf(rr, 0.0f));
  const float tol = fmaxf(p.cg_atol, p.cg_rtol * nrm0);
  const float tol2 = tol * tol;
  int iters = 0;
  bool conv = !(nrm0 > tol) || !(wu > 0.0f);
  float gam = ru, alpha = (wu > 0.0f) ? ru / wu : 0.0f, beta = 0.0f;
#pragma unroll 1
  for (int it = 0; it < p.cg_max_iter && !conv; ++it) {
    p2 = u2 + beta * p2;
    s2v = w2 + beta * s2v;
    x2 += alpha * p2;
    res2 -= alpha * s2v;
    u2 = res2 * d2i;
    w2 = schur(u2);
    cta_sum3(res2 * u2, w2 * u2, res2 * res2, misc + 64, ru, wu, rr);
    iters = it + 1;
    if (rr <= tol2) {
      conv = true;
      break;
    }
    // CG scalars: fast divisions (a few ulp) are ample here
    beta = __fdividef(ru, gam);
    const float den = wu - beta * __fdividef(ru, alpha);
    if (!(den > 0.0f) | !(den < 3.0e38f)) break;
    alpha = __fdividef(ru, den);
    gam = ru;
  }
  const float resn = sqrtf(fmaxf(rr, 0.0f));
  if (!conv) err |= DFS_WARN_CG_NOT_CONVERGED;
  if (crank == 0 && tid == 0) {
    if (p.cg_iters) p.cg_iters[bh] = iters;
    if (p.cg_residual) p.cg_residual[bh] = resn;
  }
  // back-substitution for the row block
  float x1;
  {
    const float q = p_apply(x2);
    x1 = rok ? d1i * (b1 - q) : 0.0f;
  }

  // ---------------------------------------------------------------- phase 4
  // all-gather w1, f, 1/rowsum, D of every row; for kappa = 1 remove the
  // null-space component so that sum(dlog_mu) = sum(dlog_nu) = 0
  float tshift = 0.0f;
  {
    float* st = ex.stage();
    if ((lane & 7) == 0) {
      st[li_own] = rok ? x1 : 0.0f;
      st[64 + li_own] = rowv[BR_F * 64 + li_own];
      st[128 + li_own] = rowv[BR_INV * 64 + li_own];
      st[192 + li_own] = rowv[BR_D * 64 + li_own];
    }
    const float a = rows_sum(rsum_r * x1);
    if (lane == 0) misc[warp] = a;
    __syncthreads();
    if (tid == 0) st[256] = sum16(misc);
    if (!ex.exchange(tid, 4u * 260)) err |= DFS_ERR_DEVICE_TIMEOUT;
    if (colt) {
      const float* src = ex.from(jc >> 6);
      const int o = jc & 63;
      colv[BC_W1 * NP + jc] = src[o];
      colv[BC_FA * NP + jc] = src[64 + o];
      colv[BC_INV * NP + jc] = src[128 + o];
      colv[BC_DD * NP + jc] = src[192 + o];
      colv[BC_SOL2 * NP + jc] = x2;
    }
    float tot = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) tot += ex.from(c)[256];
    ex.next();
    if (kap >= 1.0f) tshift = sum_r > 0.0f ? -tot / sum_r : 0.0f;
  }
  if (p.dlog_mu && (lane & 7) == 0 && grow < N) p.dlog_mu[bh * N + grow] = rok ? rsum_r * (x1 + tshift) : 0.0f;
  if (p.dlog_nu && colt && jc >= row0 && jc < row0 + 64 && jc < N)
    p.dlog_nu[bh * N + jc] = cok ? colv[BC_CC * NP + jc] * (x2 - tshift) : 0.0f;
  __syncthreads();

  // ---------------------------------------------------------------- phase 5 (dQ)
  {
    float xa[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) xa[r] = __shfl_sync(0xffffffffu, x1, 8 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int j = 32 * k + lane;
      const float xs = colv[BC_SOL2 * NP + j];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const uint32_t o = sw_off(kRpw * warp + r, j, 64) >> 2;
        Ts[o] = fmaf(-P[r][k], xa[r] + xs, Ts[o]);
      }
    }
  }
  load_operand_t<DH, NP>(KV, p.K, p.in_dtype, bh * N, 0, N, tid);  // K^T (DH x NP)
  operands_ready();
  if (tid == 0) {
    issue_abt_split<DH, NP, kGradAcc>(tbase, Ts, KV);  // dQ = dS K
    mma_commit(mbar);
  }
  // shared-parameter gradients from the staged dS while the tensor core reads it
  // (the exchange buffers are free from here on: cg_* scratch lives there)
  const bool geo_grad = p.x_res != nullptr && (p.dw_dist != nullptr || p.dr_head != nullptr ||
                                               (p.dx_res != nullptr && w_h != 0.0f));
  const BinSource bsrc = bin_source(p);
  const bool pos_grad = p.dpos_weight != nullptr && bins_given(bsrc);
  const bool cost_grad = geo_grad || pos_grad || p.dx_res != nullptr;
  float* cg_dx = reinterpret_cast<float*>(base + Cfg::OFF_XR);                                // 3 x 64
  unsigned long long* cg_hist = reinterpret_cast<unsigned long long*>(base + Cfg::OFF_XR + 1024);  // 68
  float* cg_red = reinterpret_cast<float*>(base + Cfg::OFF_XR + 1600);                        // 32
  const float inv_eps = 1.0f / eps_h;
  // dx share sum_j dC_ij c_ij (x_row - x_col) of the staged tile's slab rows
  // (lanes over the N columns), added to cg_dx; with `bins`, the tile's dw and
  // dr partials (returned, per thread) and fixed-point histogram (scale `hscale`)
  auto geo_rows = [&](bool transposed, bool with_bins, float hscale) -> float2 {
    float dw = 0.0f, dr = 0.0f;
#pragma unroll 1
    for (int r = 0; r < kRpw; ++r) {
      const int li = kRpw * warp + r, gi = row0 + li;
      float ax = 0.0f, ay = 0.0f, az = 0.0f;
      if (gi < N) {
        const float x0 = rowv[BR_X0 * 64 + li], x1 = rowv[BR_X1 * 64 + li], x2 = rowv[BR_X2 * 64 + li];
        const bool hist = pos_grad && with_bins;
#pragma unroll 2
        for (int j = lane; j < N; j += 32) {
          const float dC = -Ts[sw_off(li, j, 64) >> 2] * inv_eps;
          if (geo_grad) {
            const float d0 = x0 - colv[BC_X0 * NP + j], d1 = x1 - colv[BC_X1 * NP + j], d2 = x2 - colv[BC_X2 * NP + j];
            const float dist = sqrtf(d0 * d0 + d1 * d1 + d2 * d2 + 1e-8f);
            const float rd = 1.0f / (r_h + dist);
            if (with_bins) {
              const float t = dC * dist * rd;
              dw += t;
              dr = fmaf(t, rd, dr);
            }
            const float cf = dC * w_h * r_h * rd * rd / dist;
            ax = fmaf(cf, d0, ax);
            ay = fmaf(cf, d1, ay);
            az = fmaf(cf, d2, az);
          }
          if (hist) {
            const unsigned bin = static_cast<unsigned>(bin_at(bsrc, bb, N, gi, j));  // outside [0, 68): nothing
            const long long q = __float2ll_rn(dC * hscale);
            if (bin < static_cast<unsigned>(kBins)) atomicAdd(&cg_hist[bin], static_cast<unsigned long long>(q));
          }
        }
      }
      ax = warp_sum(ax);
      ay = warp_sum(ay);
      az = warp_sum(az);
      if (lane == 0) {
        cg_dx[li] += ax;
        cg_dx[64 + li] += ay;
        cg_dx[128 + li] += az;
      }
    }
    (void)transposed;
    return make_float2(dw, dr);
  };
  if (cost_grad) {
    for (int i = tid; i < 3 * 64; i += kThreads) cg_dx[i] = 0.0f;
    for (int i = tid; i < kBins; i += kThreads) cg_hist[i] = 0ull;
    // fixed-point scale of the histogram: the tile's largest |dC| maps to 2^46,
    // so that the sum of up to 64 x 384 < 2^15 terms stays below 2^62
    float hscale = 0.0f;
    if (pos_grad) {
      float mx = 0.0f;
#pragma unroll 1
      for (int idx = tid; idx < 64 * NP; idx += kThreads) mx = fmaxf(mx, fabsf(Ts[sw_off(idx / NP, idx % NP, 64) >> 2]));
      mx = warp_max(mx);
      if (lane == 0) cg_red[warp] = mx;
    }
    __syncthreads();
    if (pos_grad) {
      float mx = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, cg_red[w]);
      mx *= inv_eps;
      int ex = 0;
      frexpf(mx, &ex);  // mx < 2^ex
      hscale = mx > 0.0f ? ldexpf(1.0f, 46 - ex) : 0.0f;
    }
    const float2 dwp = geo_rows(false, true, hscale);
    __syncthreads();  // cg_red reused
    const float dws = warp_sum(dwp.x), drs = warp_sum(dwp.y);
    if (lane == 0) {
      cg_red[warp] = dws;
      cg_red[kWarps + warp] = drs;
    }
    __syncthreads();
    const size_t cta = static_cast<size_t>(prob) * C + crank;
    const CostGradWs cw = costgrad_ws(p.ws, p.B, p.H, N);
    if (tid == 0 && p.dw_dist != nullptr) {
      float s = 0.0f;
      for (int w = 0; w < kWarps; ++w) s += cg_red[w];
      cw.dw[cta] = s;
    }
    if (tid == 32 && p.dr_head != nullptr) {
      float s = 0.0f;
      for (int w = 0; w < kWarps; ++w) s += cg_red[kWarps + w];
      cw.dr[cta] = -w_h * s;
    }
    if (pos_grad && tid < kBins)
      cw.dpos[cta * kBins + tid] =
          hscale > 0.0f ? static_cast<float>(static_cast<double>(static_cast<long long>(cg_hist[tid])) / hscale) : 0.0f;
  }
  mma_wait();
  if (p.dQ) drain_rows_to_global<DH, kGradAcc>(tbase, 0, p.dQ, bh * N, row0, N, grad_scale, warp, lane);

  // ---------------------------------------------------------------- phase 6
  tc_fence_before();
  __syncthreads();
  load_operand<DH, 64>(SA, p.K, p.in_dtype, bh * N, row0, N, tid);  // K slab
  load_operand<DH, NP>(KV, p.Q, p.in_dtype, bh * N, 0, N, tid);     // Q (all rows)
  operands_ready();
  if (tid == 0) {
    issue_qk<NP, DH>(tbase, SA, KV);  // S^T for the column slab
    mma_commit(mbar);
  }
  mma_wait();
  drain_m64<NP>(Ts, tbase, 0, qk_scale, warp, lane);
  __syncthreads();
  if (bias_on) {
    add_bias(true);
    __syncthreads();
  }
  stage_to_regs<NS>(P, Ts, warp, lane);
  {
    // slab rows r are columns j of the cost, lanes run over rows i
    float gj[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) gj[r] = colv[BC_G * NP + row0 + kRpw * warp + r];
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float fi = colv[BC_FA * NP + 32 * k + lane];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const bool ok = ((rokm >> r) & (cokm >> k) & 1u) != 0u;
        const float e = ex2(P[r][k] + gj[r] + fi);
        P[r][k] = ok ? e : 0.0f;
      }
    }
  }

  // ---------------------------------------------------------------- phase 7 (dV)
  __syncthreads();  // Ts (S^T) fully read
  load_operand<DH, 64>(SA, p.V, p.in_dtype, bh * N, row0, N, tid);   // V slab
  load_operand_f32<DH, NP>(KV, p.dO, bh * N, 0, N, tid);              // dO (all rows)
  operands_ready();
  if (tid == 0) {
    issue_abt<NP, DH>(tbase, SA, KV);  // dT^T = V_s dO^T
    mma_commit(mbar);
  }
#pragma unroll
  for (int k = 0; k < NS; ++k) {  // T_norm^T into the staging buffer (not read by that MMA)
    const int i = 32 * k + lane;
    const float inv = colv[BC_INV * NP + i];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) Ts[sw_off(kRpw * warp + r, i, 64) >> 2] = P[r][k] * inv;
  }
  if (cost_grad && p.dx_res != nullptr && p.dxc != nullptr) {
    // centroid share (T_norm^T dxc)_j for the slab rows j (each warp its own rows,
    // from its own stores above)
    __syncwarp();
#pragma unroll 1
    for (int r = 0; r < kRpw; ++r) {
      const int lj = kRpw * warp + r;
      float ax = 0.0f, ay = 0.0f, az = 0.0f;
      for (int i = lane; i < N; i += 32) {
        const float t = Ts[sw_off(lj, i, 64) >> 2];
        const float* dx = p.dxc + (bh * N + i) * 3;
        ax = fmaf(t, dx[0], ax);
        ay = fmaf(t, dx[1], ay);
        az = fmaf(t, dx[2], az);
      }
      ax = warp_sum(ax);
      ay = warp_sum(ay);
      az = warp_sum(az);
      if (lane == 0) {
        cg_dx[lj] += ax;
        cg_dx[64 + lj] += ay;
        cg_dx[128 + lj] += az;
      }
    }
  }
  mma_wait();
  __syncthreads();
  load_operand_f32_t<DH, NP>(KV, p.dO, bh * N, 0, N, tid);            // dO^T (DH x NP)
  operands_ready();
  if (tid == 0) {
    issue_abt_split<DH, NP, kGradAcc>(tbase + NP, Ts, KV);  // dV = T_norm^T dO
    mma_commit(mbar);
  }
  mma_wait();
  if (p.dV) drain_rows_to_global<DH, kGradAcc>(tbase, NP, p.dV, bh * N, row0, N, 1.0f, warp, lane);

  // ---------------------------------------------------------------- phase 8 (dK)
  tc_fence_before();
  __syncthreads();
  drain_m64<NP>(Ts, tbase, 0, 1.0f, warp, lane);  // dT^T
  __syncthreads();
  if (p.dxc) {  // dT^T[j][i] += dxc_i . x_j
#pragma unroll 1
    for (int idx = tid; idx < 64 * NP; idx += kThreads) {
      const int lj = idx / NP, gi = idx - lj * NP;
      if (gi < N) {
        const float* dx = p.dxc + (bh * N + gi) * 3;
        Ts[sw_off(lj, gi, 64) >> 2] += dx[0] * rowv[BR_X0 * 64 + lj] + dx[1] * rowv[BR_X1 * 64 + lj] +
                                       dx[2] * rowv[BR_X2 * 64 + lj];
      }
    }
    __syncthreads();
  }
  {
    float sol2j[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) sol2j[r] = colv[BC_SOL2 * NP + row0 + kRpw * warp + r];
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int i = 32 * k + lane;
      const float inv = colv[BC_INV * NP + i], Di = colv[BC_DD * NP + i], w1i = colv[BC_W1 * NP + i];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const uint32_t o = sw_off(kRpw * warp + r, i, 64) >> 2;
        Ts[o] = P[r][k] * fmaf(inv, Ts[o] - Di, -(w1i + sol2j[r]));
      }
    }
  }
  load_operand_t<DH, NP>(KV, p.Q, p.in_dtype, bh * N, 0, N, tid);  // Q^T (DH x NP)
  operands_ready();
  if (tid == 0) {
    issue_abt_split<DH, NP, kGradAcc>(tbase, Ts, KV);  // dK = dS^T Q
    mma_commit(mbar);
  }
  if (cost_grad && p.dx_res != nullptr) {
    // column share: slab rows are cost columns j, lanes run over the rows i;
    // dx_j += sum_i dC_ij c_ij (x_j - x_i) (dist and c are symmetric in i, j)
    if (geo_grad && w_h != 0.0f) geo_rows(true, false, 0.0f);
    __syncthreads();
    if (tid < 64 && row0 + tid < N) {
      const CostGradWs cw = costgrad_ws(p.ws, p.B, p.H, N);
      float* o = cw.dx + (bh * N + row0 + tid) * 3;
      o[0] = cg_dx[tid];
      o[1] = cg_dx[64 + tid];
      o[2] = cg_dx[128 + tid];
    }
  }
  mma_wait();
  if (p.dK) drain_rows_to_global<DH, kGradAcc>(tbase, 0, p.dK, bh * N, row0, N, grad_scale, warp, lane);

  // ---------------------------------------------------------------- teardown
  if (err && p.status) atomicOr(p.status, err);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
  cluster_sync();  // peers may read this CTA's exchange buffers until here
}

// Sums of the shared-parameter gradient partials in a fixed order: dx_res over
// heads, dw_dist and dpos_weight over batch elements and CTAs.
__global__ void resident_costgrad_finalize(const BwdParams p, int C) {
  const CostGradWs cw = costgrad_ws(p.ws, p.B, p.H, p.N);
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int ndx = p.dx_res != nullptr ? p.B * p.N * 3 : 0;
  const int ndw = p.dw_dist != nullptr ? p.H : 0;
  const int npos = p.dpos_weight != nullptr ? p.H * kBins : 0;
  const int ndr = p.dr_head != nullptr ? p.H : 0;
  if (t < ndx) {
    const int b = t / (p.N * 3), rem = t % (p.N * 3);
    float s = 0.0f;
    for (int h = 0; h < p.H; ++h) s += cw.dx[(static_cast<size_t>(b) * p.H + h) * p.N * 3 + rem];
    p.dx_res[t] = s;
  } else if (t < ndx + ndw) {
    const int h = t - ndx;
    float s = 0.0f;
    for (int b = 0; b < p.B; ++b)
      for (int c = 0; c < C; ++c) s += cw.dw[(static_cast<size_t>(b) * p.H + h) * C + c];
    p.dw_dist[h] = s;
  } else if (t < ndx + ndw + npos) {
    const int u = t - ndx - ndw, h = u / kBins, bin = u % kBins;
    float s = 0.0f;
    for (int b = 0; b < p.B; ++b)
      for (int c = 0; c < C; ++c) s += cw.dpos[((static_cast<size_t>(b) * p.H + h) * C + c) * kBins + bin];
    p.dpos_weight[u] = s;
  } else if (t < ndx + ndw + npos + ndr) {
    const int h = t - ndx - ndw - npos;
    float s = 0.0f;
    for (int b = 0; b < p.B; ++b)
      for (int c = 0; c < C; ++c) s += cw.dr[(static_cast<size_t>(b) * p.H + h) * C + c];
    p.dr_head[h] = s;
  }
}

template <int C, int DH>
static cudaError_t launch_bwd_cd(const BwdParams& p, cudaStream_t st) {
  using Cfg = BwdCfg<C, DH>;
  auto kern = resident_bwd_kernel<C, DH>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C * p.B * p.H);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_resident_bwd(const BwdParams& p, cudaStream_t st) {
  const int C = (p.N + 63) / 64;
  if (p.d != 32) return cudaErrorInvalidValue;
  cudaError_t e;
  switch (C) {
    case 1: e = launch_bwd_cd<1, 32>(p, st); break;
    case 2: e = launch_bwd_cd<2, 32>(p, st); break;
    case 3: e = launch_bwd_cd<3, 32>(p, st); break;
    case 4: e = launch_bwd_cd<4, 32>(p, st); break;
    case 5: e = launch_bwd_cd<5, 32>(p, st); break;
    case 6: e = launch_bwd_cd<6, 32>(p, st); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  const int n = (p.dx_res ? p.B * p.N * 3 : 0) + (p.dw_dist ? p.H : 0) + (p.dpos_weight ? p.H * kBins : 0) +
                (p.dr_head ? p.H : 0);
  if (n == 0) return cudaSuccess;
  resident_costgrad_finalize<<<(n + 255) / 256, 256, 0, st>>>(p, C);
  return cudaGetLastError();
}

size_t resident_bwd_smem(int N, int d) {
  const int C = (N + 63) / 64;
  if (d != 32 || C < 1 || C > 6) return 0;
  switch (C) {
    case 1: return BwdCfg<1, 32>::SMEM;
    case 2: return BwdCfg<2, 32>::SMEM;
    case 3: return BwdCfg<3, 32>::SMEM;
    case 4: return BwdCfg<4, 32>::SMEM;
    case 5: return BwdCfg<5, 32>::SMEM;
    default: return BwdCfg<6, 32>::SMEM;
  }
}

size_t resident_bwd_workspace(int B, int H, int N, int) {
  const size_t bh = static_cast<size_t>(B) * H, C = (N + 63) / 64;
  return sizeof(float) * (bh * N * 3 + 2 * bh * C + bh * C * kBins);
}

}  // namespace dfs
