// dfs_fwd.cu -- resident flash-Sinkhorn forward for sm_100a.
//
// One thread-block cluster per (batch, head) problem, C CTAs per cluster, each
// CTA owning a 64-row slab of the N x N problem (N <= 64*C).
//
//   1. S = Q K^T is computed once per slab with tcgen05.mma (tf32 operands from
//      128B-swizzled shared memory, fp32 accumulator in TMEM) and kept in TMEM.
//   2. The slab is moved into registers (8 warps x 8 rows, lane = column mod 32)
//      and turned into a stabilised kernel matrix E = exp2(S' + f + g - alpha - beta)
//      with every row and column maximum equal to 1 ("absorption").
//   3. Each Sinkhorn iteration is then FMA work on E: the row update reduces
//      E v over the slab's own columns, the column update reduces E^T u over the
//      slab's rows and combines the C per-CTA partial sums (max, sum-exp) through
//      distributed shared memory with one cluster barrier.  Potentials are kept
//      in log2 units in fp32, so the iteration is exactly the reference's
//      log-domain update  f = kappa (a - LSE_j(S + g)),  g = kappa (b - LSE_i(S + f))
//      (src/deepfold/model/sinkhorn.py:82-96); E is re-absorbed whenever the
//      potentials drift far enough from the last absorption to risk underflow.
//   4. The transport plan T_norm = exp(score - rowmax) / (sum + 1e-6)
//      (src/deepfold/model/kernels/sinkhorn_kernel.py:1329-1493) is written to
//      shared memory and O = T_norm V is one more tcgen05.mma chain.
#include "dfs_slab.cuh"

namespace dfs {

template <int C, int DH>
struct FwdCfg {
  static constexpr int NP = 64 * C;          // padded N (columns and rows)
  static constexpr int NS = NP / 32;         // column slots per lane
  static constexpr int KA = DH / 32;         // 32-column atoms across the head dim
  static constexpr uint32_t OFF_T = 0;                              // 64 x NP
  static constexpr uint32_t OFF_Q = OFF_T + 256u * NP;              // 64 x DH
  static constexpr uint32_t OFF_KV = OFF_Q + 256u * DH;             // NP x DH (K, then V)
  static constexpr uint32_t OFF_RED = OFF_KV + 4u * NP * DH;        // 8 x NP
  static constexpr int RS = NP + 8;                                 // exchange slot (floats)
  static constexpr uint32_t OFF_XCH = OFF_RED + 32u * NP;           // 2 x C x RS receive buffers
  static constexpr uint32_t OFF_COL = OFF_XCH + 8u * C * RS;        // 10 x NP column vectors
  static constexpr uint32_t OFF_ROW = OFF_COL + 40u * NP;           // 4 x 64 row vectors
  static constexpr uint32_t OFF_MISC = OFF_ROW + 4u * 4 * 64;       // scalars, barrier
  // at least 120 KB so that only one CTA fits per SM and its 512 TMEM columns
  // never wait for another CTA of the same cluster
  static constexpr uint32_t SMEM_NEED = OFF_MISC + 512 + 1024;      // + alignment slack
  static constexpr uint32_t SMEM = SMEM_NEED > 122880u ? SMEM_NEED : 122880u;
  static_assert(SMEM <= 232448u, "exceeds the 227 KB of shared memory a CTA can use");
};

// column-vector slots (each NP floats)
enum { CV_G = 0, CV_BT, CV_GABS, CV_BNU, CV_OK, CV_GN, CV_X0, CV_X1, CV_X2, CV_NUM };
// row-vector slots (each 64 floats)
enum { RV_X0 = 0, RV_X1, RV_X2, RV_NUM };

template <int C, int DH>
__global__ void __launch_bounds__(256, 1) resident_fwd_kernel(const FwdParams p) {
  using Cfg = FwdCfg<C, DH>;
  constexpr int NP = Cfg::NP, NS = Cfg::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* Ts = reinterpret_cast<float*>(base + Cfg::OFF_T);
  float* Qs = reinterpret_cast<float*>(base + Cfg::OFF_Q);
  float* KVs = reinterpret_cast<float*>(base + Cfg::OFF_KV);
  float* red = reinterpret_cast<float*>(base + Cfg::OFF_RED);
  ClusterExchange<C, Cfg::RS> ex{reinterpret_cast<float*>(base + Cfg::OFF_XCH), 0, 0};
  float* colv = reinterpret_cast<float*>(base + Cfg::OFF_COL);
  float* rowv = reinterpret_cast<float*>(base + Cfg::OFF_ROW);
  float* misc = reinterpret_cast<float*>(base + Cfg::OFF_MISC);     // [0..63] scalars
  uint64_t* mbar = reinterpret_cast<uint64_t*>(base + Cfg::OFF_MISC + 256);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + Cfg::OFF_MISC + 272);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int crank = static_cast<int>(cluster_rank());
  ex.rank = crank;
  constexpr int OWN = NP / 4;  // threads that own 4 consecutive columns for vector work
  const int j4 = 4 * tid;
  const int prob = blockIdx.x / C;
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const int row0 = 64 * crank;
  const size_t bh = static_cast<size_t>(bb) * p.H + hh;
  const float eps_h = p.eps[hh];
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
  const float s_scale = kLog2e / eps_h;            // S' = S * log2(e),  S = -C / eps
  const float qk_scale = s_scale * rsqrtf(static_cast<float>(DH));
  const float w_h = p.w_dist ? p.w_dist[hh] : 0.0f;
  int err = 0;

  // ---------------------------------------------------------------- setup
  if (warp == 0) tmem_alloc(tslot, 512);
  if (tid == 0) {
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  // column vectors
  for (int j = tid; j < NP; j += 256) {
    const bool ok = j < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
    colv[CV_OK * NP + j] = ok ? 1.0f : 0.0f;
    colv[CV_BNU * NP + j] = ok ? p.log_nu[bh * N + j] * kLog2e : 0.0f;
    colv[CV_G * NP + j] = (ok && p.log_v_init) ? p.log_v_init[bh * N + j] * kLog2e : 0.0f;
    if (p.x_res) {
#pragma unroll
      for (int c = 0; c < 3; ++c)
        colv[(CV_X0 + c) * NP + j] = j < N ? p.x_res[(static_cast<size_t>(bb) * N + j) * 3 + c] : 0.0f;
    }
  }
  if (p.x_res) {
    for (int i = tid; i < 64; i += 256) {
      const int gi = row0 + i;
#pragma unroll
      for (int c = 0; c < 3; ++c)
        rowv[(RV_X0 + c) * 64 + i] = gi < N ? p.x_res[(static_cast<size_t>(bb) * N + gi) * 3 + c] : 0.0f;
    }
  }
  if (p.cost_mode == DFS_COST_QK) {
    load_operand<DH>(Qs, p.Q, p.in_dtype, bh * N, row0, 64, N, tid, 256);
    load_operand<DH>(KVs, p.K, p.in_dtype, bh * N, 0, NP, N, tid, 256);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  uint32_t mma_phase = 0;

  if (p.cost_mode == DFS_COST_QK) {
    if (tid == 0) {
      issue_qk<NP, DH>(tbase, Qs, KVs);
      mma_commit(mbar);
    }
    if (!mbar_wait(mbar, mma_phase & 1)) err |= DFS_ERR_DEVICE_TIMEOUT;
    ++mma_phase;
    tc_fence_after();
    __syncthreads();
  }
  // K is no longer needed (S stays in TMEM): load V over it for the output MMA.
  if (p.O != nullptr) load_operand_t<DH>(KVs, p.V, p.in_dtype, bh * N, 0, NP, N, tid, 256);

  // ---------------------------------------------------------------- registers
  float E[8][NS];
  const int rho = (lane >> 2) & 7;                 // row whose totals this lane holds
  const int lrow = 8 * warp + rho, grow = row0 + lrow;
  const bool rok = grow < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + grow] != 0.0f);
  const float ar = rok ? p.log_mu[bh * N + grow] * kLog2e : 0.0f;
  float fr = (rok && p.log_u_init) ? p.log_u_init[bh * N + grow] * kLog2e : 0.0f;
  float atr = 0.0f, fabs_r = 0.0f;
  float wk[NS];
  uint32_t cokm = 0;                               // bit k: column 32k+lane valid

  // S' (log2 units, bias terms included, invalid entries kNeg) into E.
  BiasArgs bias;
  bias.pos_weight = p.pos_weight;
  bias.pos_bins = p.pos_bins;
  bias.xrow = rowv + RV_X0 * 64;
  bias.xcol = colv + CV_X0 * NP;
  bias.geo = p.x_res != nullptr && w_h != 0.0f;
  bias.w_h = w_h;
  bias.r_0 = p.r_0;
  bias.s_scale = s_scale;
  bias.bb = bb;
  bias.hh = hh;
  bias.N = N;
  bias.row0 = row0;
  bias.transposed = false;
  auto load_S = [&]() {
    if (p.cost_mode == DFS_COST_QK) {
      __syncthreads();
      drain_m64<NP>(Ts, tbase, 0, qk_scale, warp, lane);
      __syncthreads();
      stage_to_regs<NS>(E, Ts, warp, lane);
      __syncthreads();
    } else {
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int gi = row0 + 8 * warp + r;
#pragma unroll
        for (int k = 0; k < NS; ++k) {
          const int gj = 32 * k + lane;
          E[r][k] = (gi < N && gj < N) ? -p.C[(bh * N + gi) * N + gj] * s_scale : 0.0f;
        }
      }
    }
    add_cost_bias<NS>(E, bias, warp, lane);
  };

  // Recompute the stabilised kernel matrix from S' and the current potentials.
  auto absorb = [&]() {
    load_S();
    float fall[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) fall[r] = __shfl_sync(0xffffffffu, fr, 4 * r);
    uint32_t rokm = 0;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int gi = row0 + 8 * warp + r;
      const bool ok = gi < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + gi] != 0.0f);
      rokm |= ok ? (1u << r) : 0u;
    }
    float gk[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) gk[k] = colv[CV_G * NP + 32 * k + lane];
    float mx[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      mx[r] = kNeg;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const bool ok = ((rokm >> r) & 1u) && ((cokm >> k) & 1u);
        E[r][k] = ok ? E[r][k] + fall[r] + gk[k] : kNeg;
        mx[r] = fmaxf(mx[r], E[r][k]);
      }
    }
    float alpha_r = reduce8_rows<true>(mx, lane);
    if (!rok) alpha_r = 0.0f;
    float alpha[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) alpha[r] = __shfl_sync(0xffffffffu, alpha_r, 4 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      float cm = kNeg;
#pragma unroll
      for (int r = 0; r < 8; ++r) cm = fmaxf(cm, E[r][k] - alpha[r]);
      red[warp * NP + 32 * k + lane] = cm;
    }
    __syncthreads();
    if (tid < OWN) {
      float4 m = make_float4(kNeg, kNeg, kNeg, kNeg);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float4 x = *reinterpret_cast<const float4*>(red + w * NP + j4);
        m = make_float4(fmaxf(m.x, x.x), fmaxf(m.y, x.y), fmaxf(m.z, x.z), fmaxf(m.w, x.w));
      }
      ex.put4(j4, m);
    }
    ex.sync();
    if (tid < OWN) {
      float m[4] = {kNeg, kNeg, kNeg, kNeg};
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const float4 x = *reinterpret_cast<const float4*>(ex.from(c) + j4);
        m[0] = fmaxf(m[0], x.x);
        m[1] = fmaxf(m[1], x.y);
        m[2] = fmaxf(m[2], x.z);
        m[3] = fmaxf(m[3], x.w);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = j4 + q;
        const float beta = colv[CV_OK * NP + j] != 0.0f ? m[q] : 0.0f;
        colv[CV_GN * NP + j] = beta;  // beta (temporary)
        colv[CV_BT * NP + j] = beta - colv[CV_G * NP + j];
        colv[CV_GABS * NP + j] = colv[CV_G * NP + j];
      }
    }
    ex.next();
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float beta = colv[CV_GN * NP + 32 * k + lane];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const bool ok = ((rokm >> r) & 1u) && ((cokm >> k) & 1u);
        E[r][k] = ok ? ex2(E[r][k] - alpha[r] - beta) : 0.0f;
      }
      wk[k] = colv[CV_BT * NP + 32 * k + lane] + colv[CV_G * NP + 32 * k + lane];
    }
    atr = alpha_r - fr;
    fabs_r = fr;
    __syncthreads();
  };

  // Row update: f = kappa (a - LSE_j(S + g)); returns the new f of row rho.
  auto row_pass = [&](float* rowmax_out, float* v_out) -> float {
    // wk = beta + (g - g_abs) <= kDrift (beta <= 0 and the drift is bounded by
    // re-absorption), so exp2(wk) needs no shift
    float v[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) v[k] = ((cokm >> k) & 1u) ? ex2(wk[k]) : 0.0f;
    float acc[8], amx[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float s = 0.0f, m = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const float t = E[r][k] * v[k];
        s += t;
        if (rowmax_out) m = fmaxf(m, t);
      }
      acc[r] = s;
      amx[r] = m;
    }
    const float s = reduce8_rows<false>(acc, lane);
    if (rowmax_out) *rowmax_out = reduce8_rows<true>(amx, lane);
    if (v_out) {
#pragma unroll
      for (int k = 0; k < NS; ++k) v_out[k] = v[k];
    }
    if (rowmax_out) return s;
    const float L = atr + lg2(s);
    return rok ? kap * (ar - L) : 0.0f;
  };

  // Column update from the new row potential fn; writes g_new into CV_GN.
  // Returns a cluster-uniform flag: 1 if the result must be recomputed after
  // re-absorption (underflow / drift), plus the L-inf changes for early stop.
  auto col_pass = [&](float fn, float fprev, float& dfmax) -> int {
    const float t = rok ? fn + atr : kNeg;
    const float mu = warp_max(t);
    const float u_r = rok ? ex2(t - mu) : 0.0f;
    float u[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) u[r] = __shfl_sync(0xffffffffu, u_r, 4 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      float cs = 0.0f;
#pragma unroll
      for (int r = 0; r < 8; ++r) cs += E[r][k] * u[r];
      red[warp * NP + 32 * k + lane] = cs;
    }
    const float df = warp_max(rok ? fabsf(fn - fprev) : 0.0f);
    const float dabs = warp_max(rok ? fabsf(fn - fabs_r) : 0.0f);
    if (lane == 0) {
      misc[warp] = mu;
      misc[8 + warp] = df;
      misc[16 + warp] = dabs;
    }
    __syncthreads();
    if (tid < OWN) {  // CTA partial of 4 columns, shifted to the CTA max, to every CTA
      float mc = kNeg;
#pragma unroll
      for (int w = 0; w < 8; ++w) mc = fmaxf(mc, misc[w]);
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float fw = ex2(misc[w] - mc);
        const float4 x = *reinterpret_cast<const float4*>(red + w * NP + j4);
        s4.x += x.x * fw;
        s4.y += x.y * fw;
        s4.z += x.z * fw;
        s4.w += x.w * fw;
      }
      ex.put4(j4, s4);
      if (tid == 0) {
        float dfl = 0.0f, dal = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          dfl = fmaxf(dfl, misc[8 + w]);
          dal = fmaxf(dal, misc[16 + w]);
        }
        ex.put4(NP, make_float4(mc, dfl, dal, 0.0f));
      }
    }
    ex.sync();
    float mall = kNeg, dfg = 0.0f, dag = 0.0f;
    float mcs[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float4 sc = *reinterpret_cast<const float4*>(ex.from(c) + NP);
      mcs[c] = sc.x;
      mall = fmaxf(mall, sc.x);
      dfg = fmaxf(dfg, sc.y);
      dag = fmaxf(dag, sc.z);
    }
    int bad = 0;
    if (tid < OWN) {
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const float wf = ex2(mcs[c] - mall);
        const float4 x = *reinterpret_cast<const float4*>(ex.from(c) + j4);
        tot[0] += x.x * wf;
        tot[1] += x.y * wf;
        tot[2] += x.z * wf;
        tot[3] += x.w * wf;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = j4 + q;
        float gn = 0.0f;
        if (colv[CV_OK * NP + j] != 0.0f) {
          if (!(tot[q] > 1e-30f) || !(tot[q] < 3e38f)) bad = 1;
          gn = kap * (colv[CV_BNU * NP + j] - (colv[CV_BT * NP + j] + mall + lg2(tot[q])));
        }
        colv[CV_GN * NP + j] = gn;
      }
    }
    ex.next();
    // cluster-uniform: every CTA combined the same exchanged values
    bad = __syncthreads_or(bad);
    dfmax = dfg;
    return (bad || dag > kDrift) ? 1 : 0;
  };

  // column-valid bits for this lane
#pragma unroll
  for (int k = 0; k < NS; ++k) cokm |= (colv[CV_OK * NP + 32 * k + lane] != 0.0f) ? (1u << k) : 0u;

  absorb();

  // ---------------------------------------------------------------- iterations
  float gdrift = 0.0f;
#pragma unroll 1
  for (int it = 0; it < p.K_iter; ++it) {
    if (gdrift > kDrift) absorb();
    const float fprev = fr;
    const float fn = row_pass(nullptr, nullptr);
    float dfmax;
    int redo = col_pass(fn, fprev, dfmax);
    if (redo) {
      fr = fn;   // absorb around the new row potential, then repeat the column update
      absorb();
      redo = col_pass(fn, fprev, dfmax);
      if (redo) {
        // drift alone is harmless right after absorption; only underflow is fatal
        bool anybad = false;
        for (int j = tid; j < NP; j += 256)
          if (!isfinite(colv[CV_GN * NP + j])) anybad = true;
        if (__syncthreads_or(anybad)) err |= DFS_ERR_NUMERIC;
      }
    }
    fr = fn;
    // commit g; track its change (early stop) and its drift since absorption
    float drift = 0.0f, dgl = 0.0f;
    if (tid < OWN) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = j4 + q;
        const float g = colv[CV_GN * NP + j];
        dgl = fmaxf(dgl, fabsf(g - colv[CV_G * NP + j]));
        colv[CV_G * NP + j] = g;
        drift = fmaxf(drift, fabsf(g - colv[CV_GABS * NP + j]));
      }
    }
    drift = warp_max(drift);
    dgl = warp_max(dgl);
    if (lane == 0) {
      misc[32 + warp] = drift;
      misc[40 + warp] = dgl;
    }
    __syncthreads();
    gdrift = 0.0f;
    float dgmax = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      gdrift = fmaxf(gdrift, misc[32 + w]);
      dgmax = fmaxf(dgmax, misc[40 + w]);
    }
#pragma unroll
    for (int k = 0; k < NS; ++k) wk[k] = colv[CV_BT * NP + 32 * k + lane] + colv[CV_G * NP + 32 * k + lane];
    if (p.threshold > 0.0f && ((it + 1) % p.check_every) == 0) {
      // threshold is in natural-log units, potentials here in log2 units
      if (fmaxf(dfmax, dgmax) * kLn2 < p.threshold) break;
    }
  }

  // ---------------------------------------------------------------- outputs
  if (p.O != nullptr || p.x_centroid != nullptr || p.T_out != nullptr) {
    float rmax;
    float v[NS];
    const float s = row_pass(&rmax, v);
    const float inv_r = (rok && s > 0.0f) ? 1.0f / (s + 1e-6f * rmax) : 0.0f;
    float inv[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) inv[r] = __shfl_sync(0xffffffffu, inv_r, 4 * r);
    __syncthreads();
    float xa[3][8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      xa[0][r] = xa[1][r] = xa[2][r] = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const float t = E[r][k] * v[k] * inv[r];
        Ts[sw_off(8 * warp + r, 32 * k + lane, 64) >> 2] = t;
        if (p.T_out != nullptr) {
          const int gi = row0 + 8 * warp + r, gj = 32 * k + lane;
          if (gi < N && gj < N) p.T_out[(bh * N + gi) * N + gj] = t;
        }
        if (p.x_centroid != nullptr) {
          xa[0][r] += t * colv[CV_X0 * NP + 32 * k + lane];
          xa[1][r] += t * colv[CV_X1 * NP + 32 * k + lane];
          xa[2][r] += t * colv[CV_X2 * NP + 32 * k + lane];
        }
      }
    }
    if (p.x_centroid != nullptr) {
      float xr[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) xr[c] = reduce8_rows<false>(xa[c], lane);
      if ((lane & 3) == 0 && grow < N) {
#pragma unroll
        for (int c = 0; c < 3; ++c) p.x_centroid[(bh * N + grow) * 3 + c] = rok ? xr[c] : 0.0f;
      }
    }
    if (p.O != nullptr) {
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (tid == 0) {
        issue_abt<DH, NP>(tbase + NP, Ts, KVs, DH);  // O = T_norm (V^T)^T
        mma_commit(mbar);
      }
      if (!mbar_wait(mbar, mma_phase & 1)) err |= DFS_ERR_DEVICE_TIMEOUT;
      ++mma_phase;
      tc_fence_after();
      drain_rows_to_global<DH>(tbase, NP, p.O, bh * N, row0, N, 1.0f, warp, lane);
    }
  }
  if ((lane & 3) == 0 && grow < N) p.log_u[bh * N + grow] = rok ? fr * kLn2 : 0.0f;
  for (int j = row0 + tid; j < row0 + 64 && j < N; j += 256)
    p.log_v[bh * N + j] = colv[CV_OK * NP + j] != 0.0f ? colv[CV_G * NP + j] * kLn2 : 0.0f;

  // ---------------------------------------------------------------- teardown
  if (err && p.status) atomicOr(p.status, err);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
  cluster_sync();  // peers may still read this CTA's exchange buffers until here
}

// ---------------------------------------------------------------- launcher
template <int C, int DH>
static cudaError_t launch_fwd_cd(const FwdParams& p, cudaStream_t st) {
  using Cfg = FwdCfg<C, DH>;
  auto kern = resident_fwd_kernel<C, DH>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C * p.B * p.H);
  cfg.blockDim = dim3(256);
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

template <int DH>
static cudaError_t launch_fwd_d(const FwdParams& p, int C, cudaStream_t st) {
  switch (C) {
    case 1: return launch_fwd_cd<1, DH>(p, st);
    case 2: return launch_fwd_cd<2, DH>(p, st);
    case 3: return launch_fwd_cd<3, DH>(p, st);
    case 4: return launch_fwd_cd<4, DH>(p, st);
    case 5: return launch_fwd_cd<5, DH>(p, st);
    case 6: return launch_fwd_cd<6, DH>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_resident_fwd(const FwdParams& p, cudaStream_t st) {
  const int C = (p.N + 63) / 64;
  if (p.d == 32) return launch_fwd_d<32>(p, C, st);
  return cudaErrorInvalidValue;
}

size_t resident_fwd_smem(int N, int d) {
  const int C = (N + 63) / 64;
  if (d != 32 || C < 1 || C > 6) return 0;
  switch (C) {
    case 1: return FwdCfg<1, 32>::SMEM;
    case 2: return FwdCfg<2, 32>::SMEM;
    case 3: return FwdCfg<3, 32>::SMEM;
    case 4: return FwdCfg<4, 32>::SMEM;
    case 5: return FwdCfg<5, 32>::SMEM;
    default: return FwdCfg<6, 32>::SMEM;
  }
}

}  // namespace dfs
