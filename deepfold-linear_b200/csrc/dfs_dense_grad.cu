// dfs_dense_grad.cu -- gradients of the dense-cost entry points.
//
// The reference differentiates sinkhorn_solve by autograd through its K
// iterations (src/deepfold/model/sinkhorn.py:17-112: "plain autograd through K
// iterations") and compute_transport_output through its dense tensor ops
// (sinkhorn.py:115-198).  Here both are explicit reverse passes over C.
//
// sinkhorn_solve.  The forward (dfs_dense_iterate) keeps every iterate in a
// history, slot 2i = u_i and slot 2i + 1 = v_i for i = 0 .. K (u_0, v_0 the warm
// start), one (B, H, N) block per slot.  Iteration i is
//   u_i = kappa (a - LSE_j X_ij),  X_ij = -C_ij / eps + v_i-1,j + cb_j
//   v_i = kappa (b - LSE_r Y_rj),  Y_rj = -C_rj / eps + u_i,r + rb_r
// (a = log_mu, b = log_nu, cb / rb the -1e9 mask biases), so with the adjoints
// gu_i, gv_i of the potentials and the softmax weights recovered from the
// stored potentials (LSE = a - u / kappa, resp. b - v / kappa):
//   Pc_rj = exp(Y_rj - b_j + v_i,j / kappa)       (column softmax of step i)
//   Pr_rj = exp(X_rj - a_r + u_i,r / kappa)       (row softmax of step i)
//   gu_i,r   = [i = K] gu_up,r - kappa sum_j gv_i,j Pc_rj
//   gv_i-1,j = -kappa sum_r gu_i,r Pr_rj         (gv_K: the upstream adjoint)
//   dC_rj   += kappa / eps (gv_i,j Pc_rj + gu_i,r Pr_rj)
//   dlog_mu  = kappa sum_i gu_i,   dlog_nu = kappa sum_i gv_i (i >= 1),
//   dlog_v_init = gv_0,  dlog_u_init = 0 (u_0 is never read) unless K = 0.
// The reverse iterations only form the adjoints -- gu_i from gv_i (a row
// reduction) and gv_i-1 from gu_i (a column reduction): one read of C per
// iteration for N <= 8192 (rev_fused_kernel), else a row pass (one warp per
// row) and a column pass (one CTA per 128 columns) of 4 bytes per element
// each -- and keep every gu_i, gv_i; then one tiled pass forms
//   dC_rj = kappa / eps sum_i (gv_i,j Pc_i,rj + gu_i,r Pr_i,rj)
// from them, reading C and writing dC once: 2K exponentials per element, so
// that pass is bound by the exponentials, not by HBM.
// The upstream adjoints of the returned potentials are multiplied by the mask
// first: the forward zeroes padded potentials after the loop.
//
// compute_transport_output.  With T_norm materialised (the forward returns it)
// and dTn = dL/dT_norm formed by the caller (gO V^T + gxc x^T + the gradient of
// T_norm itself: plain batched GEMMs), the softmax backward of T_norm =
// T / (sum T + 1e-6), T = exp(score - rowmax) is, per row,
//   dscore_rj = Tn_rj (dTn_rj - sum_k dTn_rk Tn_rk)
// (the row sum S cancels), dC = -dscore / eps, dlog_v_j = sum_r dscore_rj, and
// dlog_u = 0 exactly (log_u_r cancels in score - rowmax; the rowmax path, which
// autograd routes to the argmax column, carries sum_j dT_rj T_rj = A 1e-6 /
// (S + 1e-6)^2 and is dropped: a 1e-6-relative term).
#include "dfs_kernels.cuh"
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "dfs_tma.cuh"  // ex2_poly2

namespace dfs {
namespace {

constexpr float kMaskBias = -1e9f;
constexpr int kRevThreads = 256;  // 8 warps

__device__ __forceinline__ float kappa_of(float lam, float eps) { return isinf(lam) ? 1.0f : lam / (lam + eps); }

__device__ __forceinline__ float bias_of(const float* mask, int b, int N, int j) {
  return mask == nullptr ? 0.0f : (1.0f - mask[static_cast<size_t>(b) * N + j]) * kMaskBias;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The reverse passes recover a softmax weight from stored potentials, e.g.
// exp(Y - b + v / kappa) with v = kappa (b - LSE).  On a padded entry whose
// marginal is a large negative number (the reference pads log_mu / log_nu with
// -1e9) that difference cancels to within ~1e2 and the exponent may reach
// +1e2; such an entry always meets a zero adjoint, so the exponent is capped at
// 64: the product is 0 instead of 0 * inf.  Valid entries have exponents <= ~0.
__device__ __forceinline__ float ex2c(float x) { return ex2f(fminf(x, 64.0f)); }

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

unsigned grid_for(size_t work_items, size_t per_cta) {
  const size_t g = (work_items + per_cta - 1) / per_cta;
  const size_t cap = 148u * 16u;
  return static_cast<unsigned>(g < 1 ? 1 : (g > cap ? cap : g));
}

struct RevArgs {
  const float* C;
  const float* eps;
  const float* mu;      // log_mu (B,H,N)
  const float* nu;      // log_nu
  const float* mask;    // (B,N) or null
  const float* u;       // u_i
  const float* v;       // column pass: v_i-1
  const float* g;       // column pass: gu_i
  const float2* yg;     // row pass: per column j of v_i, ((v_i,j / kappa - b_j) log2e, gv_i,j)
  const float* gup;     // row pass, i = K: masked upstream adjoint of u_K (else null)
  float* gout;          // row pass: gu_i; column pass: gv_i-1 as a plain vector (null: not wanted)
  float2* ygout;        // column pass: gv_i-1 paired with v_i-1's exponent term, as yg (null: not wanted)
  float* dsum;          // row pass: dlog_mu; column pass: dlog_nu (null: not accumulated)
  int B, H, N;
  float lam;
  int first;            // row pass i = K: dlog_mu written, not accumulated
};

// Row pass of iteration i: gu_i,r = [i = K] gu_up,r - kappa sum_j gv_i,j Pc_rj,
// one warp per row r, 16-byte loads over j when the rows are 16-byte aligned.
template <bool VEC>
__global__ void __launch_bounds__(kRevThreads) rev_row_kernel(const RevArgs a) {
  const int lane = threadIdx.x & 31;
  const size_t rows = static_cast<size_t>(a.B) * a.H * a.N;
  const size_t warp0 = (static_cast<size_t>(blockIdx.x) * kRevThreads + threadIdx.x) >> 5;
  const size_t nwarps = (static_cast<size_t>(gridDim.x) * kRevThreads) >> 5;
  const int N = a.N;
  for (size_t r = warp0; r < rows; r += nwarps) {
    const size_t prob = r / N;
    const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H), i = static_cast<int>(r % N);
    const float eps = a.eps[h], kap = kappa_of(a.lam, eps);
    const float sc = -kLog2e / eps;
    // exponent of Pc: C sc + (u_i,r + rb_r) log2e + (v_i,j / kappa - b_j) log2e
    const float yr = (a.u[r] + bias_of(a.mask, b, N, i)) * kLog2e;
    const float* c = a.C + r * N;
    const float* yg = reinterpret_cast<const float*>(a.yg + prob * N);  // (y, g) pairs
    float acc = 0.0f;
    auto elem = [&](float cj, float yj, float gj) { acc = fmaf(gj, ex2c(fmaf(cj, sc, yj + yr)), acc); };
    if constexpr (VEC) {
      auto group = [&](const float4& cv, int j) {
        const float4 p0 = ld4(yg + 2 * j), p1 = ld4(yg + 2 * j + 4);
        elem(cv.x, p0.x, p0.y);
        elem(cv.y, p0.z, p0.w);
        elem(cv.z, p1.x, p1.y);
        elem(cv.w, p1.z, p1.w);
      };
      int j = 4 * lane;
      for (; j + 384 < N; j += 512) {  // four 16-byte loads of C in flight per lane
        float4 cv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) cv[q] = __ldcs(reinterpret_cast<const float4*>(c + j + 128 * q));
#pragma unroll
        for (int q = 0; q < 4; ++q) group(cv[q], j + 128 * q);
      }
      for (; j < N; j += 128) group(__ldcs(reinterpret_cast<const float4*>(c + j)), j);
    } else {
      for (int j = lane; j < N; j += 32) elem(__ldcs(c + j), yg[2 * j], yg[2 * j + 1]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const float gu = (a.gup != nullptr ? a.gup[r] : 0.0f) - kap * acc;
      a.gout[r] = gu;
      if (a.dsum != nullptr) a.dsum[r] = a.first ? kap * gu : a.dsum[r] + kap * gu;
    }
  }
}

// Column pass of iteration i: gv_i-1,j = -kappa sum_r gu_i,r Pr_rj.  CTA = COLS
// columns of one problem, warp w takes rows w, w + 8, ...; per-column partial
// sums added over the warps in a fixed order (deterministic).
template <bool VEC>
__global__ void __launch_bounds__(kRevThreads) rev_col_kernel(const RevArgs a) {
  constexpr int COLS = VEC ? 128 : 32, PER = VEC ? 4 : 1;
  __shared__ float sacc[8][COLS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = a.N;
  const int cblocks = (N + COLS - 1) / COLS;
  const size_t prob = blockIdx.x / cblocks;
  const int j0 = (blockIdx.x % cblocks) * COLS;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float eps = a.eps[h], kap = kappa_of(a.lam, eps), ikap = 1.0f / kap;
  const float sc = -kLog2e / eps;
  const int j = j0 + PER * lane;
  float cb[PER], acc[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    cb[q] = (j + q < N) ? (a.v[prob * N + j + q] + bias_of(a.mask, b, N, j + q)) * kLog2e : 0.0f;
    acc[q] = 0.0f;
  }
  if (j < N) {
    const float* cbase = a.C + prob * N * static_cast<size_t>(N) + j;
    const float* ur = a.u + prob * N;
    const float* mur = a.mu + prob * N;
    const float* gur = a.g + prob * N;
    auto row = [&](int i, const float4& cv) {
      const float gu = gur[i];
      const float xr = (ur[i] * ikap - mur[i]) * kLog2e;  // u_i,r / kappa - a_r
      acc[0] = fmaf(gu, ex2c(fmaf(cv.x, sc, cb[0]) + xr), acc[0]);
      if constexpr (VEC) {
        acc[1] = fmaf(gu, ex2c(fmaf(cv.y, sc, cb[1]) + xr), acc[1]);
        acc[2] = fmaf(gu, ex2c(fmaf(cv.z, sc, cb[2]) + xr), acc[2]);
        acc[3] = fmaf(gu, ex2c(fmaf(cv.w, sc, cb[3]) + xr), acc[3]);
      }
    };
    auto load = [&](int i) {
      if constexpr (VEC) return __ldcs(reinterpret_cast<const float4*>(cbase + static_cast<size_t>(i) * N));
      else return make_float4(__ldcs(cbase + static_cast<size_t>(i) * N), 0.0f, 0.0f, 0.0f);
    };
    int i = warp;
    for (; i + 24 < N; i += 32) {  // four row segments in flight per thread
      float4 cv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) cv[u] = load(i + 8 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) row(i + 8 * u, cv[u]);
    }
    for (; i < N; i += 8) row(i, load(i));
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) sacc[warp][PER * lane + q] = acc[q];
  __syncthreads();
  for (int t = threadIdx.x; t < COLS; t += kRevThreads) {
    const int jj = j0 + t;
    if (jj >= N) continue;
    float sum = 0.0f;
    for (int w = 0; w < 8; ++w) sum += sacc[w][t];
    const float gv = -kap * sum;
    const size_t o = prob * N + jj;
    if (a.gout != nullptr) a.gout[o] = gv;
    if (a.ygout != nullptr) a.ygout[o] = make_float2((a.v[o] * ikap - a.nu[o]) * kLog2e, gv);
    if (a.dsum != nullptr) a.dsum[o] += kap * gv;
  }
}

// One reverse iteration in one read of C (N <= kRevFuseMaxN): the row pass and
// the column pass above fused as dense_fused_kernel fuses the forward.  A CTA
// takes rows [r0, r1) of one problem, eight at a time: each warp finishes its
// row's gu_i,r (pass A, the row pass's reduction); then the CTA re-reads the
// same rows (from L2) and adds gu_i,r Pr_rj into per-column sums kept in shared
// memory (pass B), thread t owning columns 4t + 1024k.  Each CTA writes its
// column sums; rev_fused_merge adds a problem's CTA sums in CTA order into
// gv_i-1 (and its exponent pair, dlog_nu).
constexpr int kRevFuseMaxN = 8192;

struct RevPlan {
  int S;    // CTAs per problem
  int rpu;  // rows per CTA, a multiple of 8
};

RevPlan rev_plan(int BH, int N, int slots) {
  RevPlan p;
  p.S = std::max(1, std::min(slots / std::max(BH, 1), (N + 7) / 8));
  p.rpu = ((N + p.S - 1) / p.S + 7) / 8 * 8;
  p.S = (N + p.rpu - 1) / p.rpu;
  return p;
}

size_t rev_fuse_smem(int N) { return static_cast<size_t>(2) * N * sizeof(float) + 16 * sizeof(float); }

template <bool VEC>
__global__ void __launch_bounds__(kRevThreads) rev_fused_kernel(const RevArgs a, RevPlan plan, float* part) {
  extern __shared__ __align__(16) float rsm[];
  const int N = a.N;
  float* cacc = rsm;          // column sums of gu_r Pr_rj
  float* cbv = rsm + N;       // (v_i-1,j + cb_j) log2e
  float* gw = rsm + 2 * N;    // this group's gu_r
  float* xw = gw + 8;         // this group's (u_i,r / kappa - a_r) log2e
  const size_t prob = blockIdx.x / plan.S;
  const int r0 = static_cast<int>(blockIdx.x % plan.S) * plan.rpu, r1 = min(N, r0 + plan.rpu);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float eps = a.eps[h], kap = kappa_of(a.lam, eps), ikap = 1.0f / kap;
  const float sc = -kLog2e / eps;
  const float* cprob = a.C + prob * static_cast<size_t>(N) * N;
  const float* yg = reinterpret_cast<const float*>(a.yg + prob * N);  // (y, g) pairs of v_i
  for (int j = threadIdx.x; j < N; j += kRevThreads) {
    cacc[j] = 0.0f;
    cbv[j] = (a.v[prob * N + j] + bias_of(a.mask, b, N, j)) * kLog2e;
  }
  for (int g0 = r0; g0 < r1; g0 += 8) {
    // pass A: gu of row g0 + warp
    const int ri = g0 + warp;
    if (ri < r1) {
      const size_t r = prob * N + ri;
      const float yr = (a.u[r] + bias_of(a.mask, b, N, ri)) * kLog2e;
      const float* c = cprob + static_cast<size_t>(ri) * N;
      float acc = 0.0f;
      auto elem = [&](float cj, float yj, float gj) { acc = fmaf(gj, ex2c(fmaf(cj, sc, yj + yr)), acc); };
      if constexpr (VEC) {
        auto group = [&](const float4& cv, int j) {
          const float4 p0 = ld4(yg + 2 * j), p1 = ld4(yg + 2 * j + 4);
          elem(cv.x, p0.x, p0.y);
          elem(cv.y, p0.z, p0.w);
          elem(cv.z, p1.x, p1.y);
          elem(cv.w, p1.z, p1.w);
        };
        int j = 4 * lane;
        for (; j + 384 < N; j += 512) {
          float4 cv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) cv[q] = ld4(c + j + 128 * q);  // plain loads: kept in L2 for pass B
#pragma unroll
          for (int q = 0; q < 4; ++q) group(cv[q], j + 128 * q);
        }
        for (; j < N; j += 128) group(ld4(c + j), j);
      } else {
        for (int j = lane; j < N; j += 32) elem(c[j], yg[2 * j], yg[2 * j + 1]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        const float gu = (a.gup != nullptr ? a.gup[r] : 0.0f) - kap * acc;
        a.gout[r] = gu;
        if (a.dsum != nullptr) a.dsum[r] = a.first ? kap * gu : a.dsum[r] + kap * gu;
        gw[warp] = gu;
        xw[warp] = (a.u[r] * ikap - a.mu[r]) * kLog2e;
      }
    } else if (lane == 0) {
      gw[warp] = 0.0f;  // no row: weight 0 (its capped exponential stays finite)
      xw[warp] = 0.0f;
    }
    __syncthreads();
    // pass B: gu_r Pr_rj of the group's rows into the column sums
    const int nr = min(8, r1 - g0);
    if constexpr (VEC) {
      for (int j = 4 * threadIdx.x; j < N; j += 4 * kRevThreads) {
        float4 s4 = *reinterpret_cast<float4*>(cacc + j);
        const float4 cb = *reinterpret_cast<const float4*>(cbv + j);
        for (int w0 = 0; w0 < 8; w0 += 4) {
          float4 cv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int row = g0 + min(w0 + q, nr - 1);  // rows past the range re-read a valid row, weight 0
            cv[q] = __ldcs(reinterpret_cast<const float4*>(cprob + static_cast<size_t>(row) * N + j));
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float g = gw[w0 + q], x = xw[w0 + q];
            s4.x = fmaf(g, ex2c(fmaf(cv[q].x, sc, cb.x) + x), s4.x);
            s4.y = fmaf(g, ex2c(fmaf(cv[q].y, sc, cb.y) + x), s4.y);
            s4.z = fmaf(g, ex2c(fmaf(cv[q].z, sc, cb.z) + x), s4.z);
            s4.w = fmaf(g, ex2c(fmaf(cv[q].w, sc, cb.w) + x), s4.w);
          }
        }
        *reinterpret_cast<float4*>(cacc + j) = s4;
      }
    } else {
      for (int j = threadIdx.x; j < N; j += kRevThreads) {
        float s1 = cacc[j];
        for (int w = 0; w < nr; ++w)
          s1 = fmaf(gw[w], ex2c(fmaf(__ldcs(cprob + static_cast<size_t>(g0 + w) * N + j), sc, cbv[j]) + xw[w]), s1);
        cacc[j] = s1;
      }
    }
    __syncthreads();  // gw / xw are rewritten by the next group
  }
  float* pp = part + static_cast<size_t>(blockIdx.x) * N;
  for (int j = threadIdx.x; j < N; j += kRevThreads) pp[j] = cacc[j];
}

// gv_i-1,j = -kappa sum over the problem's CTAs (in CTA order) of their column sums
__global__ void rev_fused_merge(const RevArgs a, RevPlan plan, const float* part) {
  const int N = a.N;
  const size_t n = static_cast<size_t>(a.B) * a.H * N;
  for (size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < n;
       o += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t prob = o / N;
    const int j = static_cast<int>(o % N);
    const float* p = part + prob * plan.S * static_cast<size_t>(N) + j;
    float sum = p[0];
    for (int k = 1; k < plan.S; ++k) sum += p[static_cast<size_t>(k) * N];
    const float kap = kappa_of(a.lam, a.eps[prob % a.H]), ikap = 1.0f / kap;
    const float gv = -kap * sum;
    if (a.ygout != nullptr) a.ygout[o] = make_float2((a.v[o] * ikap - a.nu[o]) * kLog2e, gv);
    if (a.gout != nullptr) a.gout[o] = gv;
    if (a.dsum != nullptr) a.dsum[o] += kap * gv;
  }
}

// The cost gradient from every iteration's adjoints at once (after the reverse
// passes): dC_rj = sum_i w_i,j Pc_i,rj + w'_i,r Pr_i,rj over i = 1 .. K, with
// the per-row and per-column parts of each exponent and weight staged in
// shared memory.  A CTA takes a 64 x 64 tile of one problem, thread t the
// rows 4 (t / 16) .. + 3 and columns 4 (t % 16) .. + 3 (16-byte loads and
// stores of C and dC), and walks the iterations in chunks of kDcChunk.  Each
// element costs 2K exponentials and one read of C and one write of dC, so the
// pass is bound by the exponentials: pairs of elements run on the packed fp32
// instructions, and the exponentials of the pairs kDcPolyPairs selects are
// evaluated on the FMA pipes (ex2_poly2) instead of the MUFU.
constexpr int kDcTile = 64, kDcChunk = 16;
// POLY: bit p (of the 8 element pairs of a term) puts pair p's exponentials on
// the FMA pipes.  The default share is set from a sweep on the B200; the
// environment variable DFS_DC_POLY (0, 2, 3 or 4 pairs of 8) overrides it.
constexpr int kDcPolyDefault = 0;

struct DcArgs {
  const float* C;
  const float* eps;
  const float* mu;
  const float* nu;
  const float* mask;
  const float* hist;   // slot 2i = u_i, 2i + 1 = v_i
  const float* gu;     // gu_i at gu + (i - 1) ns, i = 1 .. K
  const float* gv;     // (y, gv_i) pairs: gv_i,o at gv[2 ((i - 1) ns + o) + 1]
  size_t ns;           // stride of the scratch slots (floats; n rounded up to 64)
  float* dC;
  int B, H, N, K;
  float lam;
  const float* shift;  // factored pass: s, s', t, t' planes of ns floats (row / column maxima, log2 units)
  const unsigned* rng; // factored pass: per problem 4 largest ranges (float bits); null: exact pass only
  const float* fac;    // factored pass: A, A', B, B' planes of K x ns floats (iteration i at (i - 1) ns)
};

// Each term of the cost gradient factors over rows and columns:
//   Pc_i,rj = exp2(c_rj sc) 2^(U_i,r) 2^(Vc_i,j),  Pr_i,rj = exp2(c_rj sc) 2^(Ur_i,r) 2^(Vr_i,j),
// so dC_rj = exp2(c sc + s_r + t_j) sum_i A_i,r B_i,j + exp2(c sc + s'_r + t'_j) sum_i A'_i,r B'_i,j
// with A = 2^(U - s), B = w 2^(Vc - t), A' = w' 2^(Ur - s'), B' = 2^(Vr - t'), the shifts s, t
// (s', t') each row's / column's maximum over the iterations: a rank-2K product, 2K FMAs and two
// exponentials per element instead of 2K exponentials.  Every factor lies in [2^-range, 1] (times
// its weight); while the largest row range plus the largest column range of a problem stays within
// kDcRange, no factor or product leaves the normal fp32 range and the final scale stays below
// 2^kDcRange (the largest term of each kind is <= 1: a softmax weight).  Problems beyond it (far
// from converged potentials at a tiny eps) take the exact pass.
constexpr float kDcRange = 64.0f;

__device__ __forceinline__ bool dc_fast(const unsigned* r) {
  return __uint_as_float(r[0]) + __uint_as_float(r[2]) <= kDcRange &&
         __uint_as_float(r[1]) + __uint_as_float(r[3]) <= kDcRange;  // NaN: exact pass
}

// Shifts, ranges and factors: one thread per (problem, row) and per (problem,
// column); padded points get shift 0 and factors 0 and take no part in the
// ranges.  The ranges are reduced over the warp before the atomic when the
// whole warp holds one problem's rows (or columns).
__global__ void dc_factor_kernel(const DcArgs a, float* shift, unsigned* rng, float* fac) {
  const int N = a.N;
  const size_t n = static_cast<size_t>(a.B) * a.H * N;
  const size_t kn = static_cast<size_t>(a.K) * a.ns;
  const size_t total = 2 * n, stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t span = (total + stride - 1) / stride * stride;  // every lane runs the same trip count
  for (size_t e = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < span; e += stride) {
    const bool live = e < total;
    const bool row = e < n;
    const size_t o = live ? (row ? e : e - n) : 0;
    const size_t prob = o / N;
    const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H), q = static_cast<int>(o % N);
    const float kap = kappa_of(a.lam, a.eps[h]), ikap = 1.0f / kap, cdc = kap / a.eps[h];
    const bool valid = live && (a.mask == nullptr || a.mask[static_cast<size_t>(b) * N + q] != 0.0f);
    // row: x0 = U = u_i log2e, x1 = Ur = (u_i / kappa - a) log2e; column: x0 = Vc = (v_i / kappa - b) log2e,
    // x1 = Vr = v_i-1 log2e (the mask biases are 0 on valid points)
    auto xs = [&](int i, float& x0, float& x1) {
      if (row) {
        const float u = a.hist[static_cast<size_t>(2 * i) * n + o];
        x0 = u * kLog2e;
        x1 = (u * ikap - a.mu[o]) * kLog2e;
      } else {
        x0 = (a.hist[static_cast<size_t>(2 * i + 1) * n + o] * ikap - a.nu[o]) * kLog2e;
        x1 = a.hist[static_cast<size_t>(2 * i - 1) * n + o] * kLog2e;
      }
    };
    float m0 = -INFINITY, l0 = INFINITY, m1 = -INFINITY, l1 = INFINITY;
    if (valid) {
      for (int i = 1; i <= a.K; ++i) {
        float x0, x1;
        xs(i, x0, x1);
        m0 = fmaxf(m0, x0);
        l0 = fminf(l0, x0);
        m1 = fmaxf(m1, x1);
        l1 = fminf(l1, x1);
      }
    }
    if (live) {
      shift[(row ? 0 : 2) * a.ns + o] = valid ? m0 : 0.0f;
      shift[(row ? 1 : 3) * a.ns + o] = valid ? m1 : 0.0f;
      // factors: rows A = 2^(U - s), A' = w' 2^(Ur - s'); columns B = w 2^(Vc - t), B' = 2^(Vr - t')
      float* f0 = fac + (row ? 0 : 2) * kn + o;
      float* f1 = fac + (row ? 1 : 3) * kn + o;
      for (int i = 1; i <= a.K; ++i) {
        float v0 = 0.0f, v1 = 0.0f;
        if (valid) {
          float x0, x1;
          xs(i, x0, x1);
          const size_t so = static_cast<size_t>(i - 1) * a.ns + o;
          const float w = cdc * (row ? a.gu[so] : a.gv[2 * so + 1]);
          v0 = ex2f(x0 - m0);
          v1 = ex2f(x1 - m1);
          if (row) v1 *= w;
          else v0 *= w;
        }
        f0[static_cast<size_t>(i - 1) * a.ns] = v0;
        f1[static_cast<size_t>(i - 1) * a.ns] = v1;
      }
    }
    // ranges: >= 0, or NaN / inf for non-finite potentials (kept as +inf: the exact pass)
    const float r0 = m0 - l0, r1 = m1 - l1;
    unsigned u0 = valid ? (isnan(r0) ? 0x7f800000u : __float_as_uint(r0)) : 0u;
    unsigned u1 = valid ? (isnan(r1) ? 0x7f800000u : __float_as_uint(r1)) : 0u;
    const unsigned long long key = live ? prob * 2 + (row ? 0 : 1) : ~0ull;
    const unsigned long long key0 = __shfl_sync(0xffffffffu, key, 0);
    if (__all_sync(0xffffffffu, key == key0)) {
      u0 = __reduce_max_sync(0xffffffffu, u0);
      u1 = __reduce_max_sync(0xffffffffu, u1);
      if ((threadIdx.x & 31) == 0 && live && (u0 | u1)) {
        atomicMax(rng + 4 * prob + (row ? 0 : 2), u0);
        atomicMax(rng + 4 * prob + (row ? 1 : 3), u1);
      }
    } else if (valid) {
      atomicMax(rng + 4 * prob + (row ? 0 : 2), u0);
      atomicMax(rng + 4 * prob + (row ? 1 : 3), u1);
    }
  }
}

// The factored cost-gradient pass: same tiles and thread layout as the exact
// pass below, the factors of kDcChunk iterations staged per chunk.
template <bool VEC>
__global__ void __launch_bounds__(256, 3) dense_dc_fact_kernel(const DcArgs a) {
  __shared__ float4 srow[2][kDcChunk][kDcTile / 4];  // A, A' for 64 rows
  __shared__ float4 scol[2][kDcChunk][kDcTile / 4];  // B, B' for 64 columns
  const int N = a.N;
  const int tiles = (N + kDcTile - 1) / kDcTile;
  const size_t prob = blockIdx.x / (static_cast<size_t>(tiles) * tiles);
  if (!dc_fast(a.rng + 4 * prob)) return;  // uniform over the CTA: the exact pass takes this problem
  const int tr = static_cast<int>((blockIdx.x / tiles) % tiles), tc = static_cast<int>(blockIdx.x % tiles);
  const int r0 = tr * kDcTile, c0 = tc * kDcTile;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float sc = -kLog2e / a.eps[h];
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  const int row0 = r0 + 4 * rg, col0 = c0 + 4 * cg;
  const float* mk = a.mask == nullptr ? nullptr : a.mask + static_cast<size_t>(b) * N;
  float2 acc1[4][2], acc2[4][2];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) acc1[rr][0] = acc1[rr][1] = acc2[rr][0] = acc2[rr][1] = make_float2(0.0f, 0.0f);
  // the tile of C, read first so that its HBM latency overlaps the staging and the products
  const float* cbase = a.C + prob * static_cast<size_t>(N) * N;
  float c[4][4];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const int r = row0 + rr;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) c[rr][cc] = 0.0f;
    if constexpr (VEC) {
      if (r < N && col0 < N) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(cbase + static_cast<size_t>(r) * N + col0));
        c[rr][0] = v.x, c[rr][1] = v.y, c[rr][2] = v.z, c[rr][3] = v.w;
      }
    } else {
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        if (r < N && col0 + cc < N) c[rr][cc] = __ldcs(cbase + static_cast<size_t>(r) * N + col0 + cc);
    }
  }
  const size_t kn = static_cast<size_t>(a.K) * a.ns;
  for (int i0 = 1; i0 <= a.K; i0 += kDcChunk) {
    const int nk = min(kDcChunk, a.K - i0 + 1);
    __syncthreads();
    // copy the chunk's factors: plane pl (A, A', B, B'), iteration k, 64 rows or columns
    if constexpr (VEC) {
      for (int e = threadIdx.x; e < 4 * kDcChunk * (kDcTile / 4); e += 256) {
        const int pl = e / (kDcChunk * (kDcTile / 4)), rem = e % (kDcChunk * (kDcTile / 4));
        const int k = rem / (kDcTile / 4), p4 = rem % (kDcTile / 4);
        const int q = (pl < 2 ? r0 : c0) + 4 * p4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k < nk && q < N)
          v = *reinterpret_cast<const float4*>(a.fac + pl * kn + static_cast<size_t>(i0 + k - 1) * a.ns + prob * N + q);
        (pl < 2 ? srow[pl][k] : scol[pl - 2][k])[p4] = v;
      }
    } else {
      for (int e = threadIdx.x; e < 4 * kDcChunk * kDcTile; e += 256) {
        const int pl = e / (kDcChunk * kDcTile), rem = e % (kDcChunk * kDcTile);
        const int k = rem / kDcTile, p = rem % kDcTile;
        const int q = (pl < 2 ? r0 : c0) + p;
        const float v = (k < nk && q < N) ? a.fac[pl * kn + static_cast<size_t>(i0 + k - 1) * a.ns + prob * N + q] : 0.0f;
        reinterpret_cast<float*>(pl < 2 ? &srow[pl][k][0] : &scol[pl - 2][k][0])[p] = v;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < nk; ++k) {
      const float4 A = srow[0][k][rg], A1 = srow[1][k][rg];
      const float4 Bv = scol[0][k][cg], B1 = scol[1][k][cg];
      const float Aa[4] = {A.x, A.y, A.z, A.w}, A1a[4] = {A1.x, A1.y, A1.z, A1.w};
      const float2 bp[2] = {make_float2(Bv.x, Bv.y), make_float2(Bv.z, Bv.w)};
      const float2 b1p[2] = {make_float2(B1.x, B1.y), make_float2(B1.z, B1.w)};
#pragma unroll
      for (int rr = 0; rr < 4; ++rr)
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          acc1[rr][h2] = __ffma2_rn(make_float2(Aa[rr], Aa[rr]), bp[h2], acc1[rr][h2]);
          acc2[rr][h2] = __ffma2_rn(make_float2(A1a[rr], A1a[rr]), b1p[h2], acc2[rr][h2]);
        }
    }
  }
  // scale by exp2(c sc + shifts) and store; padded rows / columns exactly 0
  float* dbase = a.dC + prob * static_cast<size_t>(N) * N;
  float t0[4], t1[4];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int j = col0 + cc;
    t0[cc] = j < N ? a.shift[2 * a.ns + prob * N + j] : 0.0f;
    t1[cc] = j < N ? a.shift[3 * a.ns + prob * N + j] : 0.0f;
  }
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const int r = row0 + rr;
    if (r >= N) continue;
    const float s0 = a.shift[prob * N + r], s1 = a.shift[a.ns + prob * N + r];
    const bool rok = mk == nullptr || mk[r] != 0.0f;
    const float p1[4] = {acc1[rr][0].x, acc1[rr][0].y, acc1[rr][1].x, acc1[rr][1].y};
    const float p2[4] = {acc2[rr][0].x, acc2[rr][0].y, acc2[rr][1].x, acc2[rr][1].y};
    float out[4];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int j = col0 + cc;
      const bool ok = rok && j < N && (mk == nullptr || mk[j] != 0.0f);
      const float base = c[rr][cc] * sc;
      const float v = ex2f(fminf(base + s0 + t0[cc], 126.0f)) * p1[cc] + ex2f(fminf(base + s1 + t1[cc], 126.0f)) * p2[cc];
      out[cc] = ok ? v : 0.0f;
    }
    if constexpr (VEC) {
      if (col0 < N)
        __stcs(reinterpret_cast<float4*>(dbase + static_cast<size_t>(r) * N + col0),
               make_float4(out[0], out[1], out[2], out[3]));
    } else {
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        if (col0 + cc < N) dbase[static_cast<size_t>(r) * N + col0 + cc] = out[cc];
    }
  }
}

__device__ __forceinline__ float2 ex2c2(float2 x, bool poly) {
  x.x = fminf(x.x, 64.0f);
  x.y = fminf(x.y, 64.0f);
  if (poly) return ex2_poly2(x);
  return make_float2(ex2f(x.x), ex2f(x.y));
}

template <bool VEC, unsigned POLY>
__global__ void __launch_bounds__(256) dense_dc_kernel(const DcArgs a) {
  __shared__ float4 srow[3][kDcChunk][kDcTile / 4];  // U, Ur, w' for 64 rows (4 per float4)
  __shared__ float4 scol[3][kDcChunk][kDcTile / 4];  // Vc, Vr, w for 64 columns
  const int N = a.N;
  const int tiles = (N + kDcTile - 1) / kDcTile;
  const size_t total = static_cast<size_t>(a.B) * a.H * tiles * tiles;
  // grid-stride over the tiles (a few CTAs per SM): the tiles of problems the
  // factored pass takes are skipped without a CTA launch each
  for (size_t tile = blockIdx.x; tile < total; tile += gridDim.x) {
  const size_t prob = tile / (static_cast<size_t>(tiles) * tiles);
  if (a.rng != nullptr && dc_fast(a.rng + 4 * prob)) continue;  // uniform over the CTA: the factored pass has it
  const int tr = static_cast<int>((tile / tiles) % tiles), tc = static_cast<int>(tile % tiles);
  const int r0 = tr * kDcTile, c0 = tc * kDcTile;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float eps = a.eps[h], kap = kappa_of(a.lam, eps), ikap = 1.0f / kap;
  const float sc = -kLog2e / eps, cdc = kap / eps;
  const size_t n = static_cast<size_t>(a.B) * a.H * N;
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  const int row0 = r0 + 4 * rg, col0 = c0 + 4 * cg;
  const float* cbase = a.C + prob * static_cast<size_t>(N) * N;
  // base exponents c sc of the thread's 4 x 4 elements, -inf outside the problem
  float2 base[4][2], acc[4][2];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const int r = row0 + rr;
    float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if constexpr (VEC) {
      if (r < N && col0 < N) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(cbase + static_cast<size_t>(r) * N + col0));
        c[0] = v.x, c[1] = v.y, c[2] = v.z, c[3] = v.w;
      }
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int j = col0 + cc;
      if constexpr (!VEC) {
        if (r < N && j < N) c[cc] = __ldcs(cbase + static_cast<size_t>(r) * N + j);
      }
      const float x = (r < N && j < N) ? c[cc] * sc : -INFINITY;
      if (cc & 1) base[rr][cc >> 1].y = x;
      else base[rr][cc >> 1].x = x;
    }
    acc[rr][0] = acc[rr][1] = make_float2(0.0f, 0.0f);
  }
  for (int i0 = 1; i0 <= a.K; i0 += kDcChunk) {
    const int nk = min(kDcChunk, a.K - i0 + 1);
    __syncthreads();  // the previous chunk's reads are done
    // stage: thread t fills one (term, row / column) entry per step
    for (int e = threadIdx.x; e < 2 * kDcChunk * kDcTile; e += 256) {
      const int side = e / (kDcChunk * kDcTile), rem = e % (kDcChunk * kDcTile);
      const int k = rem / kDcTile, p = rem % kDcTile;
      float x0 = 0.0f, x1 = 0.0f, x2 = 0.0f;
      const int q = (side == 0 ? r0 : c0) + p;
      if (k < nk && q < N) {
        const int i = i0 + k;
        const size_t o = prob * N + q;
        const float bias = bias_of(a.mask, b, N, q);
        if (side == 0) {  // row r = q: U = (u_i + rb) log2e, Ur = (u_i / kappa - a) log2e, w' = kappa / eps gu_i
          const float u = a.hist[static_cast<size_t>(2 * i) * n + o];
          x0 = (u + bias) * kLog2e;
          x1 = (u * ikap - a.mu[o]) * kLog2e;
          x2 = cdc * a.gu[static_cast<size_t>(i - 1) * a.ns + o];
        } else {          // column j = q: Vc = (v_i / kappa - b) log2e, Vr = (v_i-1 + cb) log2e, w = kappa / eps gv_i
          const float v = a.hist[static_cast<size_t>(2 * i + 1) * n + o];
          x0 = (v * ikap - a.nu[o]) * kLog2e;
          x1 = (a.hist[static_cast<size_t>(2 * i - 1) * n + o] + bias) * kLog2e;
          x2 = cdc * a.gv[2 * (static_cast<size_t>(i - 1) * a.ns + o) + 1];
        }
      }
      float* dst = reinterpret_cast<float*>(side == 0 ? &srow[0][k][0] : &scol[0][k][0]);
      const size_t plane = static_cast<size_t>(kDcChunk) * kDcTile;  // floats per value plane
      dst[p] = x0;
      dst[plane + p] = x1;
      dst[2 * plane + p] = x2;
    }
    __syncthreads();
    for (int k = 0; k < nk; ++k) {
      const float4 U = srow[0][k][rg], Ur = srow[1][k][rg], Wr = srow[2][k][rg];
      const float4 Vc = scol[0][k][cg], Vr = scol[1][k][cg], Wc = scol[2][k][cg];
      const float Ua[4] = {U.x, U.y, U.z, U.w}, Ura[4] = {Ur.x, Ur.y, Ur.z, Ur.w};
      const float Wra[4] = {Wr.x, Wr.y, Wr.z, Wr.w};
      const float2 vc[2] = {make_float2(Vc.x, Vc.y), make_float2(Vc.z, Vc.w)};
      const float2 vr[2] = {make_float2(Vr.x, Vr.y), make_float2(Vr.z, Vr.w)};
      const float2 wc[2] = {make_float2(Wc.x, Wc.y), make_float2(Wc.z, Wc.w)};
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int pair = rr * 2 + h2;  // 8 pairs per term
          // column-softmax term: exp2(c sc + U_r + Vc_j) weighted by w_j
          const float2 xc = __fadd2_rn(base[rr][h2], __fadd2_rn(make_float2(Ua[rr], Ua[rr]), vc[h2]));
          const float2 pc = ex2c2(xc, (POLY >> pair) & 1u);
          acc[rr][h2] = __ffma2_rn(wc[h2], pc, acc[rr][h2]);
          // row-softmax term: exp2(c sc + Ur_r + Vr_j) weighted by w'_r
          const float2 xr = __fadd2_rn(base[rr][h2], __fadd2_rn(make_float2(Ura[rr], Ura[rr]), vr[h2]));
          const float2 pr = ex2c2(xr, (POLY >> (pair ^ 1)) & 1u);
          acc[rr][h2] = __ffma2_rn(make_float2(Wra[rr], Wra[rr]), pr, acc[rr][h2]);
        }
      }
    }
  }
  // padded rows and columns: exactly 0, as autograd gives them (their terms are
  // 0 or, on the FMA pipes, 2^-125-sized)
  if (a.mask != nullptr) {
    const float* mk = a.mask + static_cast<size_t>(b) * N;
#pragma unroll
    for (int rr = 0; rr < 4; ++rr)
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int r = row0 + rr, j = col0 + cc;
        const bool keep = r < N && j < N && mk[r] != 0.0f && mk[j] != 0.0f;
        float2& x = acc[rr][cc >> 1];
        if (!keep) (cc & 1 ? x.y : x.x) = 0.0f;
      }
  }
  float* dbase = a.dC + prob * static_cast<size_t>(N) * N;
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const int r = row0 + rr;
    if (r >= N) continue;
    if constexpr (VEC) {
      if (col0 < N)
        __stcs(reinterpret_cast<float4*>(dbase + static_cast<size_t>(r) * N + col0),
               make_float4(acc[rr][0].x, acc[rr][0].y, acc[rr][1].x, acc[rr][1].y));
    } else {
      const float v[4] = {acc[rr][0].x, acc[rr][0].y, acc[rr][1].x, acc[rr][1].y};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        if (col0 + cc < N) dbase[static_cast<size_t>(r) * N + col0 + cc] = v[cc];
    }
  }
  }  // tiles
}

// u_0, v_0 of the history from the warm start (zeros without one)
__global__ void hist_init_kernel(const float* lui, const float* lvi, float* u0, float* v0, size_t n) {
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    u0[k] = lui != nullptr ? lui[k] : 0.0f;
    v0[k] = lvi != nullptr ? lvi[k] : 0.0f;
  }
}

// largest |u_i - u_i-1| and |v_i - v_i-1| over the batch (the reference's stop
// test, sinkhorn.py:99-103), as float bits (non-negative floats order like
// their bit patterns)
__global__ void hist_change_kernel(const float* u, const float* up, const float* v, const float* vp, size_t n,
                                   unsigned* out) {
  float m = 0.0f;
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fmaxf(fabsf(u[k] - up[k]), fabsf(v[k] - vp[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// the returned potentials: slot K, padded entries zeroed (sinkhorn.py:107-110),
// non-finite valid entries flagged
__global__ void hist_out_kernel(const float* uK, const float* vK, const float* mask, float* lu, float* lv, int H,
                                int N, size_t n, int32_t* status) {
  int bad = 0;
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float m = mask != nullptr ? mask[(k / (static_cast<size_t>(H) * N)) * N + k % N] : 1.0f;
    const float u = uK[k] * m, v = vK[k] * m;
    lu[k] = u;
    lv[k] = v;
    bad |= !isfinite(u) || !isfinite(v);
  }
  if (bad && status != nullptr) atomicOr(status, DFS_ERR_NUMERIC);
}

// out = g * mask, and dsum = kappa out when dsum is given
__global__ void masked_adjoint_kernel(const float* g, const float* mask, const float* eps, float lam, int H, int N,
                                      size_t n, float* out, float* dsum) {
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t bh = k / N;
    const float m = mask != nullptr ? mask[(bh / H) * N + k % N] : 1.0f;
    const float x = g != nullptr ? g[k] * m : 0.0f;
    out[k] = x;
    if (dsum != nullptr) dsum[k] = kappa_of(lam, eps[bh % H]) * x;
  }
}

// transport backward, pass 1: one warp per row, dC_rj = -Tn_rj (dTn_rj - <dTn_r, Tn_r>) / eps in place of dTn
template <bool VEC>
__global__ void __launch_bounds__(kRevThreads) tbwd_row_kernel(const float* Tn, float* dT, const float* eps, int H, int N,
                                                            size_t rows) {
  const int lane = threadIdx.x & 31;
  const size_t warp0 = (static_cast<size_t>(blockIdx.x) * kRevThreads + threadIdx.x) >> 5;
  const size_t nwarps = (static_cast<size_t>(gridDim.x) * kRevThreads) >> 5;
  for (size_t r = warp0; r < rows; r += nwarps) {
    const float* t = Tn + r * N;
    float* d = dT + r * N;
    float dot = 0.0f;
    if constexpr (VEC) {
      for (int j = 4 * lane; j < N; j += 128) {
        const float4 a = ld4(t + j), g = ld4(d + j);
        dot = fmaf(a.x, g.x, dot);
        dot = fmaf(a.y, g.y, dot);
        dot = fmaf(a.z, g.z, dot);
        dot = fmaf(a.w, g.w, dot);
      }
    } else {
      for (int j = lane; j < N; j += 32) dot = fmaf(t[j], d[j], dot);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float s = -1.0f / eps[(r / N) % H];
    // the second sweep re-reads the row just read: it is served from L1 / L2
    if constexpr (VEC) {
      for (int j = 4 * lane; j < N; j += 128) {
        const float4 a = ld4(t + j);
        float4 g = ld4(d + j);
        g.x = s * a.x * (g.x - dot);
        g.y = s * a.y * (g.y - dot);
        g.z = s * a.z * (g.z - dot);
        g.w = s * a.w * (g.w - dot);
        __stcs(reinterpret_cast<float4*>(d + j), g);
      }
    } else {
      for (int j = lane; j < N; j += 32) d[j] = s * t[j] * (d[j] - dot);
    }
  }
}

// transport backward, pass 2: dlog_v_j = sum_r dscore_rj = -eps sum_r dC_rj
template <bool VEC>
__global__ void __launch_bounds__(kRevThreads) tbwd_col_kernel(const float* dC, const float* eps, int H, int N,
                                                            float* dlv) {
  constexpr int COLS = VEC ? 128 : 32, PER = VEC ? 4 : 1;
  __shared__ float sacc[8][COLS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cblocks = (N + COLS - 1) / COLS;
  const size_t prob = blockIdx.x / cblocks;
  const int j0 = (blockIdx.x % cblocks) * COLS;
  const int j = j0 + PER * lane;
  float acc[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) acc[q] = 0.0f;
  if (j < N) {
    const float* base = dC + prob * N * static_cast<size_t>(N) + j;
    for (int i = warp; i < N; i += 8) {
      if constexpr (VEC) {
        const float4 x = __ldcs(reinterpret_cast<const float4*>(base + static_cast<size_t>(i) * N));
        acc[0] += x.x;
        acc[1] += x.y;
        acc[2] += x.z;
        acc[3] += x.w;
      } else {
        acc[0] += __ldcs(base + static_cast<size_t>(i) * N);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) sacc[warp][PER * lane + q] = acc[q];
  __syncthreads();
  const float e = eps[prob % H];
  for (int t = threadIdx.x; t < COLS; t += kRevThreads) {
    const int jj = j0 + t;
    if (jj >= N) continue;
    float sum = 0.0f;
    for (int w = 0; w < 8; ++w) sum += sacc[w][t];
    dlv[prob * N + jj] = -e * sum;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Scratch of the reverse (floats), slots of ns = n rounded up to 64 floats
// (every slot 256-byte aligned): gu_i (iters slots), (y, gv_i) pairs (2 iters),
// the masked upstream adjoint of u_K (1), the factored pass's shifts (4) and
// factors (4 iters), 4 x BH per-problem ranges (rounded up to 64), then the
// one-read reverse iterations' column sums.
size_t dense_bwd_slot(size_t n) { return (n + 63) / 64 * 64; }
// column sums of the one-read reverse iterations: N floats per CTA, at most max(BH, 148 SMs x 8) CTAs
size_t rev_part_floats(int B, int H, int N) {
  return N > kRevFuseMaxN ? 0 : static_cast<size_t>(std::max(B * H, 148 * 8)) * N;
}
size_t dense_bwd_scratch_floats(int B, int H, int N, int iters) {
  const size_t n = static_cast<size_t>(B) * H * N;
  return static_cast<size_t>(7 * iters + 5) * dense_bwd_slot(n) + dense_bwd_slot(4 * static_cast<size_t>(B) * H) +
         rev_part_floats(B, H, N);
}

// ((v_K / kappa - b) log2e, gv_K) pairs from the masked upstream adjoint of v_K; dlog_nu = kappa gv_K
__global__ void ygv_init_kernel(const float* g, const float* vK, const float* nu, const float* mask, const float* eps,
                                float lam, int H, int N, size_t n, float2* yg, float* dnu) {
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t bh = k / N;
    const float m = mask != nullptr ? mask[(bh / H) * N + k % N] : 1.0f;
    const float kap = kappa_of(lam, eps[bh % H]);
    const float x = g != nullptr ? g[k] * m : 0.0f;
    yg[k] = make_float2((vK[k] / kap - nu[k]) * kLog2e, x);
    if (dnu != nullptr) dnu[k] = kap * x;
  }
}

}  // namespace

cudaError_t launch_dense_solve_bwd(int B, int H, int N, int iters, float lam, const float* C, const float* eps,
                                   const float* mu, const float* nu, const float* mask, const float* hist,
                                   const float* g_lu, const float* g_lv, float* dC, float* dmu, float* dnu,
                                   float* dlui, float* dlvi, float* scratch, cudaStream_t st) {
  const size_t n = static_cast<size_t>(B) * H * N;
  const size_t ns = dense_bwd_slot(n);
  const unsigned ge = grid_for(n, 256);
  cudaError_t e = cudaSuccess;
  if (iters == 0) {  // the outputs are the (masked) warm start itself
    if (dlui) masked_adjoint_kernel<<<ge, 256, 0, st>>>(g_lu, mask, eps, lam, H, N, n, dlui, nullptr);
    if (dlvi) masked_adjoint_kernel<<<ge, 256, 0, st>>>(g_lv, mask, eps, lam, H, N, n, dlvi, nullptr);
    if (dC && (e = cudaMemsetAsync(dC, 0, n * N * sizeof(float), st)) != cudaSuccess) return e;
    if (dmu && (e = cudaMemsetAsync(dmu, 0, n * sizeof(float), st)) != cudaSuccess) return e;
    if (dnu && (e = cudaMemsetAsync(dnu, 0, n * sizeof(float), st)) != cudaSuccess) return e;
    return cudaGetLastError();
  }
  auto gu = [&](int i) { return scratch + static_cast<size_t>(i - 1) * ns; };
  auto gvy = [&](int i) { return reinterpret_cast<float2*>(scratch + static_cast<size_t>(iters + 2 * (i - 1)) * ns); };
  float* gup = scratch + static_cast<size_t>(3 * iters) * ns;
  auto slot = [&](int k) { return hist + static_cast<size_t>(k) * n; };
  ygv_init_kernel<<<ge, 256, 0, st>>>(g_lv, slot(2 * iters + 1), nu, mask, eps, lam, H, N, n, gvy(iters), dnu);
  masked_adjoint_kernel<<<ge, 256, 0, st>>>(g_lu, mask, eps, lam, H, N, n, gup, nullptr);
  if (dlui && (e = cudaMemsetAsync(dlui, 0, n * sizeof(float), st)) != cudaSuccess) return e;
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const bool vec = (N % 4) == 0 && aligned16(C) && (dC == nullptr || aligned16(dC));
  const unsigned grow = grid_for(n, kRevThreads / 32);
  const int cols = vec ? 128 : 32;
  const unsigned gcol = static_cast<unsigned>(B) * H * static_cast<unsigned>((N + cols - 1) / cols);
  // one read of C per reverse iteration for N <= kRevFuseMaxN
  float* rpart = scratch + static_cast<size_t>(7 * iters + 5) * ns + dense_bwd_slot(4 * static_cast<size_t>(B) * H);
  const size_t rpart_floats = rev_part_floats(B, H, N);
  RevPlan plan{0, 0};
  if (rpart_floats != 0) {
    const size_t smem = rev_fuse_smem(N);
    auto kern = vec ? rev_fused_kernel<true> : rev_fused_kernel<false>;
    int nb = 0, dev = 0, sms = 148;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))) ==
            cudaSuccess &&
        (e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kRevThreads, smem)) == cudaSuccess &&
        (e = cudaGetDevice(&dev)) == cudaSuccess)
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    plan = rev_plan(B * H, N, std::max(1, nb) * sms);
    while (static_cast<size_t>(B) * H * plan.S * N > rpart_floats && plan.S > 1)
      plan = rev_plan(B * H, N, B * H * (plan.S - 1));
  }
  for (int i = iters; i >= 1 && e == cudaSuccess; --i) {
    RevArgs a{};
    a.C = C;
    a.eps = eps;
    a.mu = mu;
    a.nu = nu;
    a.mask = mask;
    a.B = B;
    a.H = H;
    a.N = N;
    a.lam = lam;
    // row pass: gu_i from gv_i
    a.u = slot(2 * i);
    a.yg = gvy(i);
    a.gup = i == iters ? gup : nullptr;
    a.gout = gu(i);
    a.dsum = dmu;
    a.first = i == iters;
    const bool want_gv = i > 1 || dlvi != nullptr;  // gv_0 is wanted only as the warm start's gradient
    if (plan.S > 0 && want_gv) {
      // row and column pass in one read of C: gu_i, then gv_i-1 from the CTAs' column sums
      a.v = slot(2 * i - 1);
      a.gout = gu(i);
      a.ygout = nullptr;
      const size_t smem = rev_fuse_smem(N);
      if (vec) rev_fused_kernel<true><<<static_cast<unsigned>(B * H * plan.S), kRevThreads, smem, st>>>(a, plan, rpart);
      else rev_fused_kernel<false><<<static_cast<unsigned>(B * H * plan.S), kRevThreads, smem, st>>>(a, plan, rpart);
      RevArgs m = a;
      m.gout = i > 1 ? nullptr : dlvi;
      m.ygout = i > 1 ? gvy(i - 1) : nullptr;
      m.dsum = i > 1 ? dnu : nullptr;
      rev_fused_merge<<<ge, 256, 0, st>>>(m, plan, rpart);
      e = cudaGetLastError();
      continue;
    }
    if (vec) rev_row_kernel<true><<<grow, kRevThreads, 0, st>>>(a);
    else rev_row_kernel<false><<<grow, kRevThreads, 0, st>>>(a);
    // column pass: gv_i-1 from gu_i (the adjoint of the warm start at i = 1)
    RevArgs c = a;
    c.v = slot(2 * i - 1);
    c.g = gu(i);
    c.yg = nullptr;
    c.gup = nullptr;
    c.gout = i > 1 ? nullptr : dlvi;
    c.ygout = i > 1 ? gvy(i - 1) : nullptr;
    c.dsum = i > 1 ? dnu : nullptr;
    c.first = 0;
    if (want_gv) {
      if (vec) rev_col_kernel<true><<<gcol, kRevThreads, 0, st>>>(c);
      else rev_col_kernel<false><<<gcol, kRevThreads, 0, st>>>(c);
    }
    e = cudaGetLastError();
  }
  if (e != cudaSuccess || dC == nullptr) return e;
  // the factored pass for the problems whose potentials stay within kDcRange, the exact one for the rest
  // (DFS_DENSE_DC=exact in the environment: the exact pass for every problem)
  const char* mode = std::getenv("DFS_DENSE_DC");
  const bool factored = mode == nullptr || std::strcmp(mode, "exact") != 0;
  float* shift = scratch + static_cast<size_t>(3 * iters + 1) * ns;
  float* fac = shift + 4 * ns;
  unsigned* rng = reinterpret_cast<unsigned*>(fac + static_cast<size_t>(4 * iters) * ns);
  DcArgs d{C, eps, mu, nu, mask, hist, gu(1), reinterpret_cast<const float*>(gvy(1)), ns, dC, B, H, N, iters, lam,
           nullptr, nullptr, nullptr};
  if (factored) {
    if ((e = cudaMemsetAsync(rng, 0, 4 * static_cast<size_t>(B) * H * sizeof(unsigned), st)) != cudaSuccess)
      return e;
    d.shift = shift;
    d.rng = rng;
    d.fac = fac;
    dc_factor_kernel<<<grid_for(2 * n, 256), 256, 0, st>>>(d, shift, rng, fac);
  }
  const size_t tiles = static_cast<size_t>((N + kDcTile - 1) / kDcTile);
  const unsigned gdc = static_cast<unsigned>(static_cast<size_t>(B) * H * tiles * tiles);
  static const int poly = [] {
    const char* v = std::getenv("DFS_DC_POLY");
    return v != nullptr ? std::atoi(v) : kDcPolyDefault;
  }();
  auto go = [&](auto kern) { kern<<<gdc, 256, 0, st>>>(d); };
  if (factored) vec ? go(dense_dc_fact_kernel<true>) : go(dense_dc_fact_kernel<false>);
  const unsigned gex = static_cast<unsigned>(std::min<size_t>(gdc, 148u * 2u));  // the exact pass: grid-stride
  auto go_ex = [&](auto kern) { kern<<<gex, 256, 0, st>>>(d); };
  switch (poly) {
    case 2: vec ? go_ex(dense_dc_kernel<true, 0x11u>) : go_ex(dense_dc_kernel<false, 0x11u>); break;
    case 3: vec ? go_ex(dense_dc_kernel<true, 0x15u>) : go_ex(dense_dc_kernel<false, 0x15u>); break;
    case 4: vec ? go_ex(dense_dc_kernel<true, 0x55u>) : go_ex(dense_dc_kernel<false, 0x55u>); break;
    default: vec ? go_ex(dense_dc_kernel<true, 0x00u>) : go_ex(dense_dc_kernel<false, 0x00u>); break;
  }
  return cudaGetLastError();
}

}  // namespace dfs

using namespace dfs;

namespace {
bool dims_ok(int B, int H, int N) {
  return B > 0 && H > 0 && N > 0 && N <= (1 << 16) && static_cast<long long>(B) * H <= (1 << 24);
}
int status_of(cudaError_t e) { return e == cudaSuccess ? DFS_OK : DFS_ERR_CUDA; }
}  // namespace

extern "C" size_t dfs_dense_work_bytes(int B, int H, int N) {
  return dims_ok(B, H, N) ? dense_fuse_part_bytes(B, H, N) : 0;
}

extern "C" int dfs_dense_iterate(int B, int H, int N, float lam, const float* C, const float* eps,
                                 const float* log_mu, const float* log_nu, const float* log_u_init,
                                 const float* log_v_init, const float* mask, float* hist, int it_begin, int it_end,
                                 float* log_u, float* log_v, float* change, void* work, int32_t* status,
                                 void* stream) {
  if (!dims_ok(B, H, N) || C == nullptr || eps == nullptr || log_mu == nullptr || log_nu == nullptr ||
      hist == nullptr || log_u == nullptr || log_v == nullptr || it_begin < 0 || it_end < it_begin ||
      !(lam > 0.0f) || (work == nullptr && dense_fuse_part_bytes(B, H, N) != 0) ||
      (reinterpret_cast<uintptr_t>(work) & 15u) != 0)
    return DFS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t n = static_cast<size_t>(B) * H * N;
  const unsigned ge = grid_for(n, 256);
  if (it_begin == 0) hist_init_kernel<<<ge, 256, 0, st>>>(log_u_init, log_v_init, hist, hist + n, n);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess)
    e = launch_dense_iterations(C, eps, log_mu, log_nu, mask, B, H, N, lam, hist, it_begin, it_end,
                                static_cast<float*>(work), dense_fuse_part_bytes(B, H, N), st);
  const float* uK = hist + static_cast<size_t>(2 * it_end) * n;
  if (e == cudaSuccess && change != nullptr) {
    if ((e = cudaMemsetAsync(change, 0, sizeof(float), st)) == cudaSuccess && it_end > 0)
      hist_change_kernel<<<ge, 256, 0, st>>>(uK, uK - 2 * n, uK + n, uK - n, n, reinterpret_cast<unsigned*>(change));
  }
  if (e == cudaSuccess) {
    hist_out_kernel<<<ge, 256, 0, st>>>(uK, uK + n, mask, log_u, log_v, H, N, n, status);
    e = cudaGetLastError();
  }
  return status_of(e);
}

extern "C" size_t dfs_dense_solve_bwd_scratch(int B, int H, int N, int iters) {
  if (!dims_ok(B, H, N) || iters < 0) return 0;
  return dense_bwd_scratch_floats(B, H, N, iters) * sizeof(float);
}

extern "C" int dfs_dense_solve_bwd(int B, int H, int N, int iters, float lam, const float* C, const float* eps,
                                   const float* log_mu, const float* log_nu, const float* mask, const float* hist,
                                   const float* g_log_u, const float* g_log_v, float* dC, float* dlog_mu,
                                   float* dlog_nu, float* dlog_u_init, float* dlog_v_init, float* scratch,
                                   void* stream) {
  if (!dims_ok(B, H, N) || C == nullptr || eps == nullptr || log_mu == nullptr || log_nu == nullptr ||
      hist == nullptr || scratch == nullptr || iters < 0 || !(lam > 0.0f))
    return DFS_ERR_INVALID_ARGUMENT;
  return status_of(launch_dense_solve_bwd(B, H, N, iters, lam, C, eps, log_mu, log_nu, mask, hist, g_log_u, g_log_v,
                                          dC, dlog_mu, dlog_nu, dlog_u_init, dlog_v_init, scratch,
                                          static_cast<cudaStream_t>(stream)));
}

extern "C" int dfs_dense_transport_bwd(int B, int H, int N, const float* T_norm, float* dT, const float* eps,
                                       float* dlog_v, void* stream) {
  if (!dims_ok(B, H, N) || T_norm == nullptr || dT == nullptr || eps == nullptr) return DFS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t rows = static_cast<size_t>(B) * H * N;
  const bool vec = (N % 4) == 0 && aligned16(T_norm) && aligned16(dT);
  const unsigned grow = grid_for(rows, kRevThreads / 32);
  if (vec) tbwd_row_kernel<true><<<grow, kRevThreads, 0, st>>>(T_norm, dT, eps, H, N, rows);
  else tbwd_row_kernel<false><<<grow, kRevThreads, 0, st>>>(T_norm, dT, eps, H, N, rows);
  if (dlog_v != nullptr) {
    const int cols = vec ? 128 : 32;
    const unsigned gcol = static_cast<unsigned>(B) * H * static_cast<unsigned>((N + cols - 1) / cols);
    if (vec) tbwd_col_kernel<true><<<gcol, kRevThreads, 0, st>>>(dT, eps, H, N, dlog_v);
    else tbwd_col_kernel<false><<<gcol, kRevThreads, 0, st>>>(dT, eps, H, N, dlog_v);
  }
  return status_of(cudaGetLastError());
}
