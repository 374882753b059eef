// dfs_fwd.cu -- resident flash-Sinkhorn forward for sm_100a.
//
// One thread-block cluster per (batch, head) problem, C CTAs per cluster, each
// CTA owning a 64-row slab of the N x N problem (N <= 64*C), 16 warps x 4 rows.
//
//   1. S = Q K^T is computed once per slab with tcgen05.mma (tf32 operands from
//      128B-swizzled shared memory, fp32 accumulator in TMEM) and kept in TMEM.
//   2. The slab is moved into registers (lane = column mod 32) and turned into a
//      stabilised kernel matrix E = exp2(S' + f + g - alpha - beta) whose row and
//      column maxima are 1 ("absorption").  The shifts stay fixed until the next
//      absorption, so an iteration needs no max reductions.
//   3. Each Sinkhorn iteration is FMA work on E: the row update reduces E v over
//      the slab's columns (lane-local sums + 6 shuffles), the column update
//      reduces E^T u per warp, sums the 16 warp partials per CTA and the C CTA
//      partials with one push-style all-to-all through distributed shared
//      memory.  Potentials are kept in log2 units in fp32, so the iteration is
//      exactly the reference's log-domain update
//          f = kappa (a - LSE_j(S + g)),  g = kappa (b - LSE_i(S + f))
//      (src/deepfold/model/sinkhorn.py:82-96).  E is rebuilt from S (still in
//      TMEM) when the potentials drift far enough from the last absorption to
//      threaten the fp32 range, or if a column sum left it.
//   4. The transport plan T_norm = exp(score - rowmax) / (sum + 1e-6)
//      (src/deepfold/model/kernels/sinkhorn_kernel.py:1329-1493) is written to
//      shared memory and O = T_norm V is one more tcgen05.mma chain.
#include "dfs_slab.cuh"

namespace dfs {

// column-vector slots (each NP floats); G0/G1 alternate as current / next g
// CV_V holds v = exp2(beta + g - g_abs), the column factor of the row update
enum { CV_G0 = 0, CV_G1, CV_BT, CV_GABS, CV_BNU, CV_OK, CV_V, CV_X0, CV_X1, CV_X2, CV_NUM };
// slab-row vector slots (each 64 floats)
enum { RV_X0 = 0, RV_X1, RV_X2, RV_NUM };
// int slots: [MI_ALPHA] CTA max of alpha (ordered ints, shared-memory atomicMax);
// [MI_FL + s] flag word of iteration parity s (atomicOr of warp-reduced bits)
enum { MI_ALPHA = 0, MI_FL = 1 };
// flag bits: FL_FDRIFT / FL_FNC are this CTA's rows (|f - f_abs| > kDrift,
// |f - f_prev| >= threshold), the _C variants the same over the whole cluster,
// FL_GDRIFT / FL_GNC the columns (identical in every CTA)
enum : unsigned { FL_FDRIFT = 1u, FL_FNC = 2u, FL_GDRIFT = 4u, FL_GNC = 8u, FL_FDRIFT_C = 16u, FL_FNC_C = 32u };

template <int C, int DH>
struct FwdCfg {
  static constexpr int NP = 64 * C;          // padded N (columns and rows)
  static constexpr int NS = NP / 32;         // column slots per lane
  static constexpr uint32_t OFF_T = 0;                              // 64 x NP
  static constexpr uint32_t OFF_Q = OFF_T + 256u * NP;              // 64 x DH
  static constexpr uint32_t OFF_KV = OFF_Q + 256u * DH;             // NP x DH (K, then V^T)
  static constexpr uint32_t OFF_RED = OFF_KV + 4u * NP * DH;        // kWarps x NP
  static constexpr int RS = NP + 8;                                 // exchange slot (floats)
  static constexpr uint32_t XBYTES = 4u * (NP + 4);                 // bytes exchanged per round
  static constexpr uint32_t OFF_XCH = OFF_RED + 4u * kWarps * NP;   // 2 x C x RS receive slots
  static constexpr uint32_t OFF_STG = OFF_XCH + 8u * C * RS;         // 2 x RS stages
  static constexpr uint32_t OFF_COL = OFF_STG + 8u * RS;
  static constexpr uint32_t OFF_ROW = OFF_COL + 4u * CV_NUM * NP;
  static constexpr uint32_t OFF_MISC = OFF_ROW + 4u * RV_NUM * 64;  // 32 ints, barrier, TMEM slot
  // at least 120 KB so that only one CTA fits per SM and its 512 TMEM columns
  // never wait for another CTA of the same cluster
  static constexpr uint32_t SMEM_NEED = OFF_MISC + 256 + 1024;      // + alignment slack
  static constexpr uint32_t SMEM = SMEM_NEED > 122880u ? SMEM_NEED : 122880u;
  static_assert(SMEM <= 232448u, "exceeds the 227 KB of shared memory a CTA can use");
};

template <int C, int DH>
__global__ void __launch_bounds__(kThreads, 1) resident_fwd_kernel(const FwdParams p) {
  using Cfg = FwdCfg<C, DH>;
  constexpr int NP = Cfg::NP, NS = Cfg::NS;
  constexpr int OWN = NP / 4;  // threads that own 4 consecutive columns for vector work
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* Ts = reinterpret_cast<float*>(base + Cfg::OFF_T);
  float* Qs = reinterpret_cast<float*>(base + Cfg::OFF_Q);
  float* KVs = reinterpret_cast<float*>(base + Cfg::OFF_KV);
  float* red = reinterpret_cast<float*>(base + Cfg::OFF_RED);
  float* colv = reinterpret_cast<float*>(base + Cfg::OFF_COL);
  float* rowv = reinterpret_cast<float*>(base + Cfg::OFF_ROW);
  int* mi = reinterpret_cast<int*>(base + Cfg::OFF_MISC);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(base + Cfg::OFF_MISC + 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + Cfg::OFF_MISC + 144);
  BulkExchange<C, Cfg::RS> ex{reinterpret_cast<float*>(base + Cfg::OFF_XCH),
                              reinterpret_cast<float*>(base + Cfg::OFF_STG),
                              reinterpret_cast<uint64_t*>(base + Cfg::OFF_MISC + 160), 0, 0u, 0, false};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int crank = static_cast<int>(cluster_rank());
  ex.rank = crank;
  const int j4 = 4 * tid;
  const int prob = blockIdx.x / C;
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const int row0 = 64 * crank;
  const size_t bh = static_cast<size_t>(bb) * p.H + hh;
  const float eps_h = p.eps[hh];
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
  int err = 0;

  // ---------------------------------------------------------------- setup
  if (tid == 0 && p.cost_mode == DFS_COST_QK) {  // this CTA's slab of every operand into L2
    const int es = p.in_dtype == DFS_F32 ? 4 : 2;
    prefetch_slab_l2(p.Q, bh * N, row0, N, DH, es);
    prefetch_slab_l2(p.K, bh * N, row0, N, DH, es);
    if (p.V) prefetch_slab_l2(p.V, bh * N, row0, N, DH, es);
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  if (tid == 0) {
    mbar_init(mbar, 1);
    ex.init();
    fence_mbar_init();
  }
  if (tid < 32) mi[tid] = 0;
  for (int j = tid; j < NP; j += kThreads) {
    const bool ok = j < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
    colv[CV_OK * NP + j] = ok ? 1.0f : 0.0f;
    colv[CV_BNU * NP + j] = ok ? p.log_nu[bh * N + j] * kLog2e : 0.0f;
    colv[CV_G0 * NP + j] = (ok && p.log_v_init) ? p.log_v_init[bh * N + j] * kLog2e : 0.0f;
    if (p.x_res) {
#pragma unroll
      for (int c = 0; c < 3; ++c)
        colv[(CV_X0 + c) * NP + j] = j < N ? p.x_res[(static_cast<size_t>(bb) * N + j) * 3 + c] : 0.0f;
    }
  }
  if (p.x_res && tid < 64) {
    const int gi = row0 + tid;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      rowv[(RV_X0 + c) * 64 + tid] = gi < N ? p.x_res[(static_cast<size_t>(bb) * N + gi) * 3 + c] : 0.0f;
  }
  if (p.cost_mode == DFS_COST_QK) {
    load_operand<DH, 64>(Qs, p.Q, p.in_dtype, bh * N, row0, N, tid);
    load_operand<DH, NP>(KVs, p.K, p.in_dtype, bh * N, 0, N, tid);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (C > 1) cluster_sync();  // every CTA's exchange mbarriers initialised
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
  // K is no longer needed (S stays in TMEM): V^T goes over it for the output MMA.
  if (p.O != nullptr) load_operand_t<DH, NP>(KVs, p.V, p.in_dtype, bh * N, 0, N, tid);

  // ---------------------------------------------------------------- registers
  float E[kRpw][NS];
  const int rho = (lane >> 3) & 3;                 // row whose totals this lane holds
  const int grow = row0 + kRpw * warp + rho;
  const bool rok = grow < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + grow] != 0.0f);
  const bool row_owner = (lane & 7) == 0;
  const float ar = rok ? p.log_mu[bh * N + grow] * kLog2e : 0.0f;
  float fr = (rok && p.log_u_init) ? p.log_u_init[bh * N + grow] * kLog2e : 0.0f;
  float atr = 0.0f, fabs_r = 0.0f, mall = 0.0f;
  uint32_t cokm = 0, rokm = 0;
  int gcur = CV_G0;
#pragma unroll
  for (int r = 0; r < kRpw; ++r) {
    const int gi = row0 + kRpw * warp + r;
    const bool ok = gi < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + gi] != 0.0f);
    rokm |= ok ? (1u << r) : 0u;
  }

  // S' = S log2(e) (S = -C / eps, bias terms included) into E.  Everything it
  // needs besides E is recomputed from the parameters here, so that none of it
  // occupies registers across the iterations.
  auto load_S = [&]() {
    const int pq = blockIdx.x / C, hq = pq % p.H, bq = pq / p.H;
    const int r0 = 64 * static_cast<int>(cluster_rank());
    const float ssc = kLog2e / p.eps[hq];
    const float wq = p.w_dist ? p.w_dist[hq] : 0.0f;
    __syncthreads();
    if (p.cost_mode == DFS_COST_QK)
      drain_m64<NP>(Ts, *tslot, 0, ssc * p.qk_scale, warp, lane);
    else
      dense_cost_to_stage<NP>(Ts, p.C, static_cast<size_t>(bq) * p.H + hq, p.N, r0, ssc, tid);
    if (p.pos_weight != nullptr || (p.x_res != nullptr && wq != 0.0f)) {
      BiasArgs bias;
      bias.pos_weight = p.pos_weight;
      bias.bins = bin_source(p);
      bias.xrow = rowv + RV_X0 * 64;
      bias.xcol = colv + CV_X0 * NP;
      bias.geo = p.x_res != nullptr && wq != 0.0f;
      bias.w_h = wq;
      bias.r_0 = p.r_head != nullptr ? p.r_head[hq] : p.r_0;
      bias.s_scale = ssc;
      bias.bb = bq;
      bias.hh = hq;
      bias.N = p.N;
      bias.row0 = r0;
      bias.transposed = false;
      __syncthreads();
      add_cost_bias_stage<NP>(Ts, bias, tid);
    }
    __syncthreads();
    stage_to_regs<NS>(E, Ts, warp, lane);
  };

  // Rebuild the stabilised kernel matrix from S' and the potentials (fr, G[gcur]).
  auto absorb = [&]() {
    if (tid == 0) mi[MI_ALPHA] = float_to_ordered(kNeg);
    load_S();  // starts with a barrier
    float fall[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) fall[r] = __shfl_sync(0xffffffffu, fr, 8 * r);
    float mx[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) mx[r] = kNeg;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float gk = colv[gcur * NP + 32 * k + lane];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const bool ok = ((rokm >> r) & 1u) && ((cokm >> k) & 1u);
        E[r][k] = ok ? E[r][k] + fall[r] + gk : kNeg;
        mx[r] = fmaxf(mx[r], E[r][k]);
      }
    }
    float alpha_r = reduce4_rows<true>(mx, lane);
    if (!rok) alpha_r = 0.0f;
    float alpha[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) alpha[r] = __shfl_sync(0xffffffffu, alpha_r, 8 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      float cm = kNeg;
#pragma unroll
      for (int r = 0; r < kRpw; ++r)
        if (((rokm >> r) & 1u) && ((cokm >> k) & 1u)) cm = fmaxf(cm, E[r][k] - alpha[r]);
      red[warp * NP + 32 * k + lane] = cm;
    }
    if (row_owner && rok) atomicMax(&mi[MI_ALPHA], float_to_ordered(alpha_r));
    __syncthreads();
    if (tid < OWN) {
      float4 m = make_float4(kNeg, kNeg, kNeg, kNeg);
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float4 x = *reinterpret_cast<const float4*>(red + w * NP + j4);
        m = make_float4(fmaxf(m.x, x.x), fmaxf(m.y, x.y), fmaxf(m.z, x.z), fmaxf(m.w, x.w));
      }
      *reinterpret_cast<float4*>(ex.stage() + j4) = m;
      if (tid == 0) ex.stage()[NP] = ordered_to_float(mi[MI_ALPHA]);
    }
    if (!ex.exchange(tid, Cfg::XBYTES)) err |= DFS_ERR_DEVICE_TIMEOUT;
    float* beta_tmp = colv + (CV_G0 + CV_G1 - gcur) * NP;  // the next-g buffer is free here
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
        beta_tmp[j] = beta;
        colv[CV_V * NP + j] = colv[CV_OK * NP + j] != 0.0f ? ex2(beta) : 0.0f;
        colv[CV_BT * NP + j] = beta - colv[gcur * NP + j];
        colv[CV_GABS * NP + j] = colv[gcur * NP + j];
      }
    }
    mall = kNeg;
#pragma unroll
    for (int c = 0; c < C; ++c) mall = fmaxf(mall, ex.from(c)[NP]);
    ex.next();
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int j = 32 * k + lane;
      const float beta = beta_tmp[j];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const bool ok = ((rokm >> r) & 1u) && ((cokm >> k) & 1u);
        E[r][k] = ok ? ex2(E[r][k] - alpha[r] - beta) : 0.0f;
      }
    }
    atr = rok ? alpha_r - fr : 0.0f;
    fabs_r = fr;
    __syncthreads();
  };

  // Hot-loop code below is written without short-circuit logic or conditional
  // calls (bitwise & on bools, selects after unconditional arithmetic): each
  // divergent branch region costs far more than the arithmetic it guards.

  // v = exp2(beta + g - g_abs) <= exp2(kDrift): beta <= 0 and the drift is
  // bounded by re-absorption, so the row sums need no further shift.
  auto load_v = [&](float (&v)[NS]) {
#pragma unroll
    for (int k = 0; k < NS; ++k) v[k] = colv[CV_V * NP + 32 * k + lane];
  };
  // Row update: f = kappa (a - LSE_j(S + g)) for row rho.
  auto row_pass = [&]() -> float {
    float v[NS];
    load_v(v);
    float acc[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) s = fmaf(E[r][k], v[k], s);
      acc[r] = s;
    }
    const float s = reduce4_rows<false>(acc, lane);
    const float f = kap * (ar - (atr + lg2(s)));
    return rok ? f : 0.0f;
  };

  // Column update from the new row potential fn into G[next] and v; returns a
  // cluster-uniform "must re-absorb and repeat" flag.  Drift / convergence
  // flags of the iteration go to mi[MI_FL + set].
  auto col_pass = [&](float fn, float fprev, int set, bool chk) -> int {
    const float ue = ex2(fn + atr - mall);
    const float u_r = rok ? ue : 0.0f;
    float u[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) u[r] = __shfl_sync(0xffffffffu, u_r, 8 * r);
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      float cs = 0.0f;
#pragma unroll
      for (int r = 0; r < kRpw; ++r) cs = fmaf(E[r][k], u[r], cs);
      red[warp * NP + 32 * k + lane] = cs;
    }
    {
      const bool own = row_owner & rok;
      const unsigned fb = static_cast<unsigned>(own & (fabsf(fn - fabs_r) > kDrift)) * FL_FDRIFT |
                          static_cast<unsigned>(own & chk & (fabsf(fn - fprev) * kLn2 >= p.threshold)) * FL_FNC;
      const unsigned wb = __reduce_or_sync(0xffffffffu, fb);
      if (lane == 0 && wb) atomicOr(&mi[MI_FL + set], static_cast<int>(wb));
    }
    __syncthreads();
    if (tid == 0) mi[MI_FL + (set ^ 1)] = 0;  // the other parity, for the next iteration
    // From here each thread tid < NP works on one column jc (colsum16).
    const bool colt = tid < NP;  // warp-uniform (NP is a multiple of 64)
    const int jc = col_of_thread(warp, lane);
    float c_ok = 0.0f, c_bnu = 0.0f, c_bt = 0.0f, c_gab = 0.0f, c_gc = 0.0f;
    if (colt) {
      const float ctot = colsum16<NP>(red, warp, lane);
      ex.stage()[jc] = ctot;
      // this column's constants, loaded before the exchange
      c_ok = colv[CV_OK * NP + jc];
      c_bnu = colv[CV_BNU * NP + jc];
      c_bt = colv[CV_BT * NP + jc];
      c_gab = colv[CV_GABS * NP + jc];
      c_gc = colv[gcur * NP + jc];
    }
    if (tid == 0) ex.stage()[NP] = __int_as_float(mi[MI_FL + set]);  // this CTA's row flags
    if (!ex.exchange(tid, Cfg::XBYTES)) err |= DFS_ERR_DEVICE_TIMEOUT;
    int bad = 0;
    unsigned gb = 0;
    if (warp == 0 && lane < C) gb = (__float_as_uint(ex.from(lane)[NP]) & (FL_FDRIFT | FL_FNC)) << 4;
    if (colt) {
      float t = ex.from(0)[jc];
#pragma unroll
      for (int c = 1; c < C; ++c) t += ex.from(c)[jc];
      const bool ok = c_ok != 0.0f;
      bad = static_cast<int>(ok & !((t > 1e-30f) & (t < 3e38f)));
      const float g = kap * (c_bnu - (c_bt + mall + lg2(t)));
      const float e = ex2(c_bt + g);
      colv[(CV_G0 + CV_G1 - gcur) * NP + jc] = ok ? g : 0.0f;
      // the row update of the next iteration reads v (all reads of this
      // iteration's v finished before the first barrier above)
      colv[CV_V * NP + jc] = ok ? e : 0.0f;
      gb |= static_cast<unsigned>(ok & (fabsf(g - c_gab) > kDrift)) * FL_GDRIFT |
            static_cast<unsigned>(ok & chk & (fabsf(g - c_gc) * kLn2 >= p.threshold)) * FL_GNC;
      const unsigned wb = __reduce_or_sync(0xffffffffu, gb);
      if (lane == 0 && wb) atomicOr(&mi[MI_FL + set], static_cast<int>(wb));
    }
    ex.next();
    return __syncthreads_or(bad);  // every CTA combined the same values: cluster-uniform
  };

  // column-valid bits for this lane
#pragma unroll
  for (int k = 0; k < NS; ++k) cokm |= (colv[CV_OK * NP + 32 * k + lane] != 0.0f) ? (1u << k) : 0u;

  // ---------------------------------------------------------------- iterations
  // absorb() has a single call site (the loop must fit the instruction cache):
  // the first absorption, re-absorption on drift, the emergency absorption
  // before a repeated column update and the one before the outputs all enter
  // through the top of this loop.  All control flow is cluster-uniform.
  const bool want_out = p.O != nullptr || p.x_centroid != nullptr || p.T_out != nullptr;
  bool need_absorb = true, redo = false, finishing = p.K_iter <= 0;
  float fn = 0.0f, fprev = 0.0f;
  int it = 0;
  const bool use_thr = p.threshold > 0.0f;
  int chk_left = p.check_every;  // iterations until the next convergence check
#pragma unroll 1
  for (;;) {
    if (__builtin_expect(need_absorb, 0)) {
      absorb();
      need_absorb = false;
      if (finishing) break;
    }
    const int set = it & 1;
    const bool chk = use_thr & (chk_left == 1);
    if (!redo) {
      fprev = fr;
      fn = row_pass();
    }
    const int bad = col_pass(fn, fprev, set, chk);
    if (__builtin_expect(bad != 0, 0)) {
      if (!redo) {
        // a column sum left the fp32 range: absorb around the new row
        // potential (and the previous, valid g) and repeat the column update
        if (tid == 0) mi[MI_FL + set] = 0;
        fr = fn;
        redo = need_absorb = true;
        continue;
      }
      err |= DFS_ERR_NUMERIC;
    }
    redo = false;
    const unsigned fl = static_cast<unsigned>(mi[MI_FL + set]);
    fr = fn;
    gcur = CV_G0 + CV_G1 - gcur;
    need_absorb = (fl & (FL_FDRIFT_C | FL_GDRIFT)) != 0;
    ++it;
    chk_left = chk ? p.check_every : chk_left - 1;
    const bool stop = (chk & ((fl & (FL_FNC_C | FL_GNC)) == 0)) | (it >= p.K_iter);
    if (__builtin_expect(stop, 0)) {
      finishing = true;
      need_absorb = need_absorb & want_out;
      if (!need_absorb) break;
    }
  }

  // ---------------------------------------------------------------- outputs
  if (want_out) {
    float v[NS];
    load_v(v);
    float acc[kRpw], amx[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      float sr = 0.0f, m = 0.0f;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const float t = E[r][k] * v[k];
        sr += t;
        m = fmaxf(m, t);
      }
      acc[r] = sr;
      amx[r] = m;
    }
    const float s = reduce4_rows<false>(acc, lane);
    const float rmax = reduce4_rows<true>(amx, lane);
    const float inv_r = (rok && s > 0.0f) ? 1.0f / (s + 1e-6f * rmax) : 0.0f;
    float inv[kRpw];
#pragma unroll
    for (int r = 0; r < kRpw; ++r) inv[r] = __shfl_sync(0xffffffffu, inv_r, 8 * r);
#pragma unroll
    for (int r = 0; r < kRpw; ++r)
#pragma unroll
      for (int k = 0; k < NS; ++k) E[r][k] *= v[k] * inv[r];  // E now holds T_norm
    __syncthreads();
    regs_to_stage<NS>(E, Ts, warp, lane);
    if (p.x_centroid != nullptr) {
      float xa[3][kRpw];
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int r = 0; r < kRpw; ++r) {
          float acc = 0.0f;
#pragma unroll
          for (int k = 0; k < NS; ++k) acc += E[r][k] * colv[(CV_X0 + c) * NP + 32 * k + lane];
          xa[c][r] = acc;
        }
      float xr[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) xr[c] = reduce4_rows<false>(xa[c], lane);
      if (row_owner && grow < N) {
#pragma unroll
        for (int c = 0; c < 3; ++c) p.x_centroid[(bh * N + grow) * 3 + c] = rok ? xr[c] : 0.0f;
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (p.T_out != nullptr) {  // materialised plan (dense compute_transport_output only)
#pragma unroll 1
      for (int idx = tid; idx < 64 * NP; idx += kThreads) {
        const int li = idx / NP, gj = idx % NP, gi = row0 + li;
        if (gi < N && gj < N) p.T_out[(bh * N + gi) * N + gj] = Ts[sw_off(li, gj, 64) >> 2];
      }
    }
    if (p.O != nullptr) {
      if (tid == 0) {
        issue_abt_split<DH, NP, kGradAcc>(tbase + NP, Ts, KVs);  // O = T_norm (V^T)^T
        mma_commit(mbar);
      }
      if (!mbar_wait(mbar, mma_phase & 1)) err |= DFS_ERR_DEVICE_TIMEOUT;
      ++mma_phase;
      tc_fence_after();
      drain_rows_to_global<DH, kGradAcc>(tbase, NP, p.O, bh * N, row0, N, 1.0f, warp, lane);
    }
  }
  if (row_owner && grow < N) p.log_u[bh * N + grow] = rok ? fr * kLn2 : 0.0f;
  for (int j = row0 + tid; j < row0 + 64 && j < N; j += kThreads)
    p.log_v[bh * N + j] = colv[CV_OK * NP + j] != 0.0f ? colv[gcur * NP + j] * kLn2 : 0.0f;

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
