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
//   2               dT = dO_s V^T -> E, D; one cluster exchange gives c = P^T 1,
//                   g_v = E^T 1 and all-gathers f, 1/rowsum and D
//   3  CG:          Jacobi-preconditioned, Chronopoulos-Gear form, one matvec and
//                   one fused cluster reduction per iteration, no host sync
//   4               w1 all-gathered; marginal gradients
//   5               dS = E - P (w1 + w2);  dQ = dS K
//   6  column slab: S^T = K_s Q^T -> P^T, T_norm^T           (registers)
//   7               dV = T_norm^T dO,  dT^T = V_s dO^T
//   8               dS^T = T_norm^T (dT^T - D) - P^T (w1 + w2);  dK = dS^T Q
// Every row or column is owned by exactly one CTA: no atomics, deterministic.
#include "dfs_slab.cuh"

namespace dfs {

template <int C, int DH>
struct BwdCfg {
  static constexpr int NP = 64 * C;
  static constexpr int NS = NP / 32;
  static constexpr uint32_t OFF_T = 0;                                // 64 x NP fp32 staging
  static constexpr uint32_t OFF_SA = OFF_T + 256u * NP;               // 64 x DH slab operand
  static constexpr uint32_t OFF_DA = OFF_SA + 256u * DH;              // 64 x DH dO slab
  static constexpr uint32_t OFF_KV = OFF_DA + 256u * DH;              // NP x DH operand / partials
  // one-off exchange of phase 2 (single buffer) and the CG / all-gather
  // exchanges (double buffered), see ClusterExchange
  static constexpr int RSA = 2 * NP + 3 * 64 + 8;
  static constexpr int RSB = NP + 8;
  static constexpr uint32_t OFF_XA = OFF_KV + 4u * NP * DH;           // C x RSA
  static constexpr uint32_t OFF_XB = OFF_XA + 4u * C * RSA;           // 2 x C x RSB
  static constexpr uint32_t OFF_COL = OFF_XB + 8u * C * RSB;          // column / all-row vectors
  static constexpr uint32_t OFF_ROW = OFF_COL + 4u * 12 * NP;         // slab-row vectors
  static constexpr uint32_t OFF_MISC = OFF_ROW + 4u * 4 * 64;
  static constexpr uint32_t SMEM_NEED = OFF_MISC + 1024 + 1024;
  static constexpr uint32_t SMEM = SMEM_NEED > 122880u ? SMEM_NEED : 122880u;
  static_assert(SMEM <= 232448u, "exceeds the 227 KB of shared memory a CTA can use");
  static_assert(kWarps * 2u * NP * 4 <= 4u * NP * DH, "column partials must fit the K/V region");
  static_assert(NP + DH <= 512, "TMEM columns");
};

// column-indexed vectors; FA/INV/DD/W1 hold all N rows after the all-gathers
enum { BC_G = 0, BC_OK, BC_U2, BC_SOL2, BC_FA, BC_INV, BC_DD, BC_W1, BC_X0, BC_X1, BC_X2, BC_NUM };
enum { BR_X0 = 0, BR_X1, BR_X2 };

template <int C, int DH>
__global__ void __launch_bounds__(kThreads, 1) resident_bwd_kernel(const BwdParams p) {
  using Cfg = BwdCfg<C, DH>;
  constexpr int NP = Cfg::NP, NS = Cfg::NS;
  constexpr int MC = (NP + kThreads - 1) / kThreads;  // columns per thread for vector work (j = tid + kThreads m)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* Ts = reinterpret_cast<float*>(base + Cfg::OFF_T);
  float* SA = reinterpret_cast<float*>(base + Cfg::OFF_SA);
  float* DA = reinterpret_cast<float*>(base + Cfg::OFF_DA);
  float* KV = reinterpret_cast<float*>(base + Cfg::OFF_KV);
  ClusterExchange<C, Cfg::RSA> exa{reinterpret_cast<float*>(base + Cfg::OFF_XA), 0, 0};
  ClusterExchange<C, Cfg::RSB> exb{reinterpret_cast<float*>(base + Cfg::OFF_XB), 0, 0};
  float* colv = reinterpret_cast<float*>(base + Cfg::OFF_COL);
  float* rowv = reinterpret_cast<float*>(base + Cfg::OFF_ROW);
  float* misc = reinterpret_cast<float*>(base + Cfg::OFF_MISC);       // 192 scalars (per-warp slots of 16)
  uint64_t* mbar = reinterpret_cast<uint64_t*>(base + Cfg::OFF_MISC + 768);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + Cfg::OFF_MISC + 784);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int crank = static_cast<int>(cluster_rank());
  exa.rank = exb.rank = crank;
  constexpr int OWN = NP / 4;  // threads that own 4 consecutive columns for the exchanges
  const int j4 = 4 * tid;
  const int prob = blockIdx.x / C;
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const int row0 = 64 * crank;
  const size_t bh = static_cast<size_t>(bb) * p.H + hh;
  const float eps_h = p.eps[hh];
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
  const float s_scale = kLog2e / eps_h;
  const float qk_scale = s_scale * rsqrtf(static_cast<float>(DH));
  const float grad_scale = rsqrtf(static_cast<float>(DH)) / eps_h;   // dS -> dQ, dK
  const float w_h = p.w_dist ? p.w_dist[hh] : 0.0f;
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

  // ---------------------------------------------------------------- setup
  if (warp == 0) tmem_alloc(tslot, 512);
  if (tid == 0) {
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  for (int j = tid; j < NP; j += kThreads) {
    const bool ok = j < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
    colv[BC_OK * NP + j] = ok ? 1.0f : 0.0f;
    colv[BC_G * NP + j] = ok ? p.log_v[bh * N + j] * kLog2e : 0.0f;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      colv[(BC_X0 + c) * NP + j] = (p.x_res && j < N) ? p.x_res[(static_cast<size_t>(bb) * N + j) * 3 + c] : 0.0f;
  }
  for (int i = tid; i < 64; i += kThreads) {
    const int gi = row0 + i;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      rowv[(BR_X0 + c) * 64 + i] = (p.x_res && gi < N) ? p.x_res[(static_cast<size_t>(bb) * N + gi) * 3 + c] : 0.0f;
  }
  load_operand<DH>(SA, p.Q, p.in_dtype, bh * N, row0, 64, N, tid, kThreads);
  load_operand<DH>(KV, p.K, p.in_dtype, bh * N, 0, NP, N, tid, kThreads);
  load_operand_f32<DH>(DA, p.dO, bh * N, row0, 64, N, tid, kThreads);
  operands_ready();
  const uint32_t tbase = *tslot;

  BiasArgs bias;
  bias.pos_weight = p.pos_weight;
  bias.pos_bins = p.pos_bins;
  bias.xrow = rowv + BR_X0 * 64;
  bias.xcol = colv + BC_X0 * NP;
  bias.geo = p.x_res != nullptr && w_h != 0.0f;
  bias.w_h = w_h;
  bias.r_0 = p.r_0;
  bias.s_scale = s_scale;
  bias.bb = bb;
  bias.hh = hh;
  bias.N = N;
  bias.row0 = row0;
  bias.transposed = false;
  const bool bias_on = p.pos_weight != nullptr || bias.geo;

  const int rho = (lane >> 3) & 3;
  const int grow = row0 + kRpw * warp + rho;
  const bool rok = grow < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + grow] != 0.0f);
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

  // ---------------------------------------------------------------- phase 1
  if (tid == 0) {
    issue_qk<NP, DH>(tbase, SA, KV);
    mma_commit(mbar);
  }
  mma_wait();
  __syncthreads();
  drain_m64<NP>(Ts, tbase, 0, qk_scale, warp, lane);
  __syncthreads();
  if (bias_on) {
    add_cost_bias_stage<NP>(Ts, bias, tid);
    __syncthreads();
  }
  float P[kRpw][NS];
  stage_to_regs<NS>(P, Ts, warp, lane);
  {
    float fall[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) fall[r] = __shfl_sync(0xffffffffu, fr, 8 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float g = colv[BC_G * NP + 32 * k + lane];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const bool ok = ((rokm >> r) & 1u) && ((cokm >> k) & 1u);
        P[r][k] = ok ? ex2(P[r][k] + fall[r] + g) : 0.0f;
      }
    }
  }
  float rsum_r, inv_r;
  {
    float a[kRpw], m[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      a[r] = 0.0f;
      m[r] = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        a[r] += P[r][k];
        m[r] = fmaxf(m[r], P[r][k]);
      }
    }
    rsum_r = reduce4_rows<false>(a, lane);
    const float pm = reduce4_rows<true>(m, lane);
    inv_r = (rok && rsum_r > 0.0f) ? 1.0f / (rsum_r + 1e-6f * pm) : 0.0f;
    if (!isfinite(rsum_r)) err |= DFS_ERR_NUMERIC;
  }

  // ---------------------------------------------------------------- phase 2
  __syncthreads();
  load_operand<DH>(KV, p.V, p.in_dtype, bh * N, 0, NP, N, tid, kThreads);
  operands_ready();
  if (tid == 0) {
    issue_abt<NP, DH>(tbase, DA, KV, NP);  // dT = dO_s V^T
    mma_commit(mbar);
  }
  mma_wait();
  __syncthreads();
  drain_m64<NP>(Ts, tbase, 0, 1.0f, warp, lane);
  __syncthreads();
  float* red = KV;  // V is no longer needed: 2 x kWarps x NP column partials (P and E)
  float fbar_r, D_r;
  {
    float inv[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) inv[r] = __shfl_sync(0xffffffffu, inv_r, 8 * r);
    float dxr[3][kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      const int gi = row0 + kRpw * warp + r;
#pragma unroll
      for (int c = 0; c < 3; ++c) dxr[c][r] = (p.dxc && gi < N) ? p.dxc[(bh * N + gi) * 3 + c] : 0.0f;
    }
    float accD[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      accD[r] = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const int j = 32 * k + lane;
        float dt = Ts[sw_off(kRpw * warp + r, j, 64) >> 2];
        if (p.dxc)
          dt += dxr[0][r] * colv[BC_X0 * NP + j] + dxr[1][r] * colv[BC_X1 * NP + j] +
                dxr[2][r] * colv[BC_X2 * NP + j];
        accD[r] += P[r][k] * inv[r] * dt;
      }
    }
    D_r = reduce4_rows<false>(accD, lane);
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
        float dt = Ts[o];
        if (p.dxc)
          dt += dxr[0][r] * colv[BC_X0 * NP + j] + dxr[1][r] * colv[BC_X1 * NP + j] +
                dxr[2][r] * colv[BC_X2 * NP + j];
        const float e = P[r][k] * inv[r] * (dt - D[r]);
        Ts[o] = e;
        ce += e;
        cp += P[r][k];
        re[r] += e;
      }
      red[warp * NP + j] = cp;
      red[kWarps * NP + warp * NP + j] = ce;
    }
    fbar_r = reduce4_rows<false>(re, lane);
  }
  {
    const bool own = (lane & 7) == 0 && rok;
    const float sf = warp_sum(own ? fbar_r : 0.0f);
    const float sr = warp_sum(own ? rsum_r : 0.0f);
    if (lane == 0) {
      misc[warp] = sf;
      misc[16 + warp] = sr;
    }
  }
  __syncthreads();
  if (tid < OWN) {
    float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f), b4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float4 x = *reinterpret_cast<const float4*>(red + w * NP + j4);
      const float4 y = *reinterpret_cast<const float4*>(red + kWarps * NP + w * NP + j4);
      a4 = make_float4(a4.x + x.x, a4.y + x.y, a4.z + x.z, a4.w + x.w);
      b4 = make_float4(b4.x + y.x, b4.y + y.y, b4.z + y.z, b4.w + y.w);
    }
    exa.put4(j4, a4);
    exa.put4(NP + j4, b4);
  }
  if ((lane & 7) == 0) {  // this slab's rows for the all-gathers
    const int li = kRpw * warp + rho;
    exa.put(2 * NP + li, fr);
    exa.put(2 * NP + 64 + li, inv_r);
    exa.put(2 * NP + 128 + li, D_r);
  }
  if (tid == 0) {
    float a = 0.0f, b = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      a += misc[w];
      b += misc[16 + w];
    }
    exa.put4(2 * NP + 192, make_float4(a, b, 0.0f, 0.0f));
  }
  exa.sync();
  float cc[MC], gv[MC];
  bool okc[MC];
  float sum_fbar = 0.0f, sum_r = 0.0f;
#pragma unroll
  for (int m = 0; m < MC; ++m) {
    const int j = tid + kThreads * m;
    cc[m] = gv[m] = 0.0f;
    okc[m] = j < NP && colv[BC_OK * NP + j] != 0.0f;
    if (j < NP) {
#pragma unroll
      for (int c = 0; c < C; ++c) {
        cc[m] += exa.from(c)[j];
        gv[m] += exa.from(c)[NP + j];
      }
      const float* src = exa.from(j >> 6);
      colv[BC_FA * NP + j] = src[2 * NP + (j & 63)];
      colv[BC_INV * NP + j] = src[2 * NP + 64 + (j & 63)];
      colv[BC_DD * NP + j] = src[2 * NP + 128 + (j & 63)];
    }
  }
#pragma unroll
  for (int c = 0; c < C; ++c) {
    sum_fbar += exa.from(c)[2 * NP + 192];
    sum_r += exa.from(c)[2 * NP + 193];
  }
  __syncthreads();

  // ---------------------------------------------------------------- phase 3 (CG)
  auto cta_sum = [&](float v, int slot) -> float {  // identical in every CTA
    v = warp_sum(v);
    if (lane == 0) misc[slot + warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += misc[slot + w];
    return s;
  };
  const float d1 = (rok && rsum_r > 0.0f) ? rsum_r / kap : 0.0f;
  float d2[MC];
#pragma unroll
  for (int m = 0; m < MC; ++m) d2[m] = (okc[m] && cc[m] > 0.0f) ? cc[m] / kap : 0.0f;
  float b1 = rok ? fbar_r : 0.0f;
  float b2[MC];
#pragma unroll
  for (int m = 0; m < MC; ++m) b2[m] = okc[m] ? gv[m] : 0.0f;
  if (kap >= 1.0f) {  // project [b1; b2] onto the range of the singular system
    float s2 = 0.0f, nv = 0.0f;
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      s2 += b2[m];
      nv += okc[m] ? 1.0f : 0.0f;
    }
    s2 = cta_sum(s2, 32);
    nv = cta_sum(nv, 48);
    const float sh = nv > 0.0f ? (sum_fbar - s2) / (2.0f * nv) : 0.0f;
    if (rok) b1 -= sh;
#pragma unroll
    for (int m = 0; m < MC; ++m)
      if (okc[m]) b2[m] += sh;
  }

  float w1;
  float w2[MC];
  // w = A u for the block system; returns the global dots (res.u, w.u, res.res)
  auto matvec = [&](float u1, const float (&u2)[MC], float res1, const float (&res2)[MC], float& ru,
                    float& wu, float& rr) {
#pragma unroll
    for (int m = 0; m < MC; ++m)
      if (tid + kThreads * m < NP) colv[BC_U2 * NP + tid + kThreads * m] = u2[m];
    __syncthreads();
    float acc[kRpw];
    float u2k[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) u2k[k] = colv[BC_U2 * NP + 32 * k + lane];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) s += P[r][k] * u2k[k];
      acc[r] = s;
    }
    const float pu = reduce4_rows<false>(acc, lane);
    w1 = rok ? d1 * u1 + pu : 0.0f;
    float u1a[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) u1a[r] = __shfl_sync(0xffffffffu, u1, 8 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      float s = 0.0f;
#pragma unroll
      for (int r = 0; r < kRpw; ++r) s += P[r][k] * u1a[r];
      red[warp * NP + 32 * k + lane] = s;
    }
    const bool own = (lane & 7) == 0 && rok;
    const float a0 = warp_sum(own ? res1 * u1 : 0.0f);
    const float a1 = warp_sum(own ? w1 * u1 : 0.0f);
    const float a2 = warp_sum(own ? res1 * res1 : 0.0f);
    if (lane == 0) {
      misc[64 + warp] = a0;
      misc[80 + warp] = a1;
      misc[96 + warp] = a2;
    }
    __syncthreads();
    if (tid < OWN) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float4 x = *reinterpret_cast<const float4*>(red + w * NP + j4);
        s4 = make_float4(s4.x + x.x, s4.y + x.y, s4.z + x.z, s4.w + x.w);
      }
      exb.put4(j4, s4);
      if (tid == 0) {
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          s0 += misc[64 + w];
          s1 += misc[80 + w];
          s2 += misc[96 + w];
        }
        exb.put4(NP, make_float4(s0, s1, s2, 0.0f));
      }
    }
    exb.sync();
    float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f;
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      const int j = tid + kThreads * m;
      float t = 0.0f;
      if (j < NP) {
#pragma unroll
        for (int c = 0; c < C; ++c) t += exb.from(c)[j];
      }
      w2[m] = okc[m] ? t + d2[m] * u2[m] : 0.0f;
      c0 += res2[m] * u2[m];
      c1 += w2[m] * u2[m];
      c2 += res2[m] * res2[m];
    }
    float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float4 d = *reinterpret_cast<const float4*>(exb.from(c) + NP);
      g0 += d.x;
      g1 += d.y;
      g2 += d.z;
    }
    exb.next();
    c0 = cta_sum(c0, 112);
    c1 = cta_sum(c1, 128);
    c2 = cta_sum(c2, 144);
    __syncthreads();
    ru = g0 + c0;
    wu = g1 + c1;
    rr = g2 + c2;
  };

  float x1 = 0.0f, res1 = b1, p1 = 0.0f, s1 = 0.0f;
  float x2[MC], res2[MC], p2[MC], s2v[MC], u2[MC];
#pragma unroll
  for (int m = 0; m < MC; ++m) {
    x2[m] = 0.0f;
    res2[m] = b2[m];
    p2[m] = s2v[m] = 0.0f;
    u2[m] = d2[m] > 0.0f ? res2[m] / d2[m] : 0.0f;
  }
  float u1 = d1 > 0.0f ? res1 / d1 : 0.0f;
  float ru, wu, rr;
  matvec(u1, u2, res1, res2, ru, wu, rr);
  const float nrm0 = sqrtf(fmaxf(rr, 0.0f));
  const float tol = fmaxf(p.cg_atol, p.cg_rtol * nrm0);
  float resn = nrm0;
  int iters = 0;
  bool conv = !(nrm0 > tol) || !(wu > 0.0f);
  float gam = ru, alpha = (wu > 0.0f) ? ru / wu : 0.0f, beta = 0.0f;
#pragma unroll 1
  for (int it = 0; it < p.cg_max_iter && !conv; ++it) {
    p1 = u1 + beta * p1;
    s1 = w1 + beta * s1;
    x1 += alpha * p1;
    res1 -= alpha * s1;
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      p2[m] = u2[m] + beta * p2[m];
      s2v[m] = w2[m] + beta * s2v[m];
      x2[m] += alpha * p2[m];
      res2[m] -= alpha * s2v[m];
      u2[m] = d2[m] > 0.0f ? res2[m] / d2[m] : 0.0f;
    }
    u1 = d1 > 0.0f ? res1 / d1 : 0.0f;
    matvec(u1, u2, res1, res2, ru, wu, rr);
    iters = it + 1;
    resn = sqrtf(fmaxf(rr, 0.0f));
    if (resn <= tol) {
      conv = true;
      break;
    }
    beta = ru / gam;
    const float den = wu - beta * ru / alpha;
    if (!(den > 0.0f) || !isfinite(den)) break;
    alpha = ru / den;
    gam = ru;
  }
  if (!conv) err |= DFS_WARN_CG_NOT_CONVERGED;
  if (crank == 0 && tid == 0) {
    if (p.cg_iters) p.cg_iters[bh] = iters;
    if (p.cg_residual) p.cg_residual[bh] = resn;
  }

  // ---------------------------------------------------------------- phase 4
  // all-gather w1; for kappa = 1 remove the null-space component so that
  // sum(dlog_mu) = sum(dlog_nu) = 0
  float tshift = 0.0f;
  {
    const bool own = (lane & 7) == 0 && rok;
    const float a = warp_sum(own ? rsum_r * x1 : 0.0f);
    if (lane == 0) misc[160 + warp] = a;
    __syncthreads();
    if ((lane & 7) == 0) exb.put(kRpw * warp + rho, x1);
    if (tid == 0) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += misc[160 + w];
      exb.put(64, t);
    }
    exb.sync();
    for (int i = tid; i < NP; i += kThreads) colv[BC_W1 * NP + i] = exb.from(i >> 6)[i & 63];
    float tot = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) tot += exb.from(c)[64];
    exb.next();
    if (kap >= 1.0f) tshift = sum_r > 0.0f ? -tot / sum_r : 0.0f;
  }
  if (p.dlog_mu && (lane & 7) == 0 && grow < N) p.dlog_mu[bh * N + grow] = rok ? rsum_r * (x1 + tshift) : 0.0f;
#pragma unroll
  for (int m = 0; m < MC; ++m) {
    const int j = tid + kThreads * m;
    if (j < NP) colv[BC_SOL2 * NP + j] = x2[m];
    if (p.dlog_nu && j >= row0 && j < row0 + 64 && j < N)
      p.dlog_nu[bh * N + j] = okc[m] ? cc[m] * (x2[m] - tshift) : 0.0f;
  }
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
        Ts[o] = Ts[o] - P[r][k] * (xa[r] + xs);
      }
    }
  }
  load_operand_t<DH>(KV, p.K, p.in_dtype, bh * N, 0, NP, N, tid, kThreads);  // K^T (DH x NP)
  operands_ready();
  if (tid == 0) {
    issue_abt<DH, NP>(tbase, Ts, KV, DH);  // dQ = dS K
    mma_commit(mbar);
  }
  mma_wait();
  if (p.dQ) drain_rows_to_global<DH>(tbase, 0, p.dQ, bh * N, row0, N, grad_scale, warp, lane);

  // ---------------------------------------------------------------- phase 6
  tc_fence_before();
  __syncthreads();
  load_operand<DH>(SA, p.K, p.in_dtype, bh * N, row0, 64, N, tid, kThreads);  // K slab
  load_operand<DH>(KV, p.Q, p.in_dtype, bh * N, 0, NP, N, tid, kThreads);     // Q (all rows)
  operands_ready();
  if (tid == 0) {
    issue_qk<NP, DH>(tbase, SA, KV);  // S^T for the column slab
    mma_commit(mbar);
  }
  mma_wait();
  __syncthreads();
  drain_m64<NP>(Ts, tbase, 0, qk_scale, warp, lane);
  __syncthreads();
  if (bias_on) {
    bias.transposed = true;
    add_cost_bias_stage<NP>(Ts, bias, tid);
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
      const int i = 32 * k + lane;
      const float fi = colv[BC_FA * NP + i];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const bool ok = ((rokm >> r) & 1u) && ((cokm >> k) & 1u);
        P[r][k] = ok ? ex2(P[r][k] + gj[r] + fi) : 0.0f;
      }
    }
  }

  // ---------------------------------------------------------------- phase 7 (dV)
  __syncthreads();
  load_operand<DH>(SA, p.V, p.in_dtype, bh * N, row0, 64, N, tid, kThreads);   // V slab
  load_operand_f32<DH>(KV, p.dO, bh * N, 0, NP, N, tid, kThreads);              // dO (all rows)
  operands_ready();
  if (tid == 0) {
    issue_abt<NP, DH>(tbase, SA, KV, NP);  // dT^T = V_s dO^T
    mma_commit(mbar);
  }
#pragma unroll
  for (int k = 0; k < NS; ++k) {  // T_norm^T into the staging buffer (not read by that MMA)
    const int i = 32 * k + lane;
    const float inv = colv[BC_INV * NP + i];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) Ts[sw_off(kRpw * warp + r, i, 64) >> 2] = P[r][k] * inv;
  }
  mma_wait();
  __syncthreads();
  load_operand_f32_t<DH>(KV, p.dO, bh * N, 0, NP, N, tid, kThreads);            // dO^T (DH x NP)
  operands_ready();
  if (tid == 0) {
    issue_abt<DH, NP>(tbase + NP, Ts, KV, DH);  // dV = T_norm^T dO
    mma_commit(mbar);
  }
  mma_wait();
  if (p.dV) drain_rows_to_global<DH>(tbase, NP, p.dV, bh * N, row0, N, 1.0f, warp, lane);

  // ---------------------------------------------------------------- phase 8 (dK)
  tc_fence_before();
  __syncthreads();
  drain_m64<NP>(Ts, tbase, 0, 1.0f, warp, lane);  // dT^T
  __syncthreads();
  {
    float xj[3][kRpw], sol2j[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      const int j = row0 + kRpw * warp + r;
      sol2j[r] = colv[BC_SOL2 * NP + j];
#pragma unroll
      for (int c = 0; c < 3; ++c) xj[c][r] = colv[(BC_X0 + c) * NP + j];
    }
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int i = 32 * k + lane;
      const float inv = colv[BC_INV * NP + i], Di = colv[BC_DD * NP + i], w1i = colv[BC_W1 * NP + i];
      float dx0 = 0.0f, dx1 = 0.0f, dx2 = 0.0f;
      if (p.dxc && i < N) {
        dx0 = p.dxc[(bh * N + i) * 3 + 0];
        dx1 = p.dxc[(bh * N + i) * 3 + 1];
        dx2 = p.dxc[(bh * N + i) * 3 + 2];
      }
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const uint32_t o = sw_off(kRpw * warp + r, i, 64) >> 2;
        float dt = Ts[o];
        if (p.dxc) dt += dx0 * xj[0][r] + dx1 * xj[1][r] + dx2 * xj[2][r];
        Ts[o] = P[r][k] * inv * (dt - Di) - P[r][k] * (w1i + sol2j[r]);
      }
    }
  }
  load_operand_t<DH>(KV, p.Q, p.in_dtype, bh * N, 0, NP, N, tid, kThreads);  // Q^T (DH x NP)
  operands_ready();
  if (tid == 0) {
    issue_abt<DH, NP>(tbase, Ts, KV, DH);  // dK = dS^T Q
    mma_commit(mbar);
  }
  mma_wait();
  if (p.dK) drain_rows_to_global<DH>(tbase, 0, p.dK, bh * N, row0, N, grad_scale, warp, lane);

  // ---------------------------------------------------------------- teardown
  if (err && p.status) atomicOr(p.status, err);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
  cluster_sync();  // peers may read this CTA's exchange buffers until here
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
  switch (C) {
    case 1: return launch_bwd_cd<1, 32>(p, st);
    case 2: return launch_bwd_cd<2, 32>(p, st);
    case 3: return launch_bwd_cd<3, 32>(p, st);
    case 4: return launch_bwd_cd<4, 32>(p, st);
    case 5: return launch_bwd_cd<5, 32>(p, st);
    case 6: return launch_bwd_cd<6, 32>(p, st);
    default: return cudaErrorInvalidValue;
  }
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

size_t resident_bwd_workspace(int, int, int, int) { return 0; }

}  // namespace dfs
