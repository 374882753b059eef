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
//   gv_i-1,j = [i - 1 = K] ... - kappa sum_r gu_i,r Pr_rj
//   dC_rj   += kappa / eps (gv_i,j Pc_rj + gu_i,r Pr_rj)
//   dlog_mu  = kappa sum_i gu_i,   dlog_nu = kappa sum_i gv_i (i >= 1),
//   dlog_v_init = gv_0,  dlog_u_init = 0 (u_0 is never read) unless K = 0.
// The reverse runs as 2K HBM passes over C, alternating
//   row pass i (one warp per row r):  gu_i from gv_i (a row reduction), and dC
//        gets both the column-softmax term of step i and the row-softmax term
//        of step i + 1 (known since the previous pass: it needs gu_i+1, u_i+1
//        and v_i), so dC is read and written once per iteration -- 12 bytes
//        per element, 8 in the first pass, which writes dC without reading it;
//   column pass i (one CTA per 128 columns): gv_i-1 from gu_i (a column
//        reduction), reading C only -- 4 bytes per element; the last (i = 1)
//        also adds the row-softmax term of step 1 into dC.
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
  const float* u;       // row pass: u_i; column pass: u_i
  const float* v;       // row pass: v_i; column pass: v_i-1
  const float* g;       // row pass: gv_i; column pass: gu_i
  const float* gup;     // row pass, i = K: masked upstream adjoint of u_K (else null)
  const float* u1;      // row pass, i < K: u_i+1 (else null: no row-softmax term)
  const float* gu1;     // row pass, i < K: gu_i+1
  float* gout;          // row pass: gu_i; column pass: gv_i-1
  float* dC;            // null: C needs no gradient
  float* dsum;          // row pass: dlog_mu; column pass: dlog_nu (null: not accumulated)
  int B, H, N;
  float lam;
  int first;            // row pass: the first (i = K) -- dC and dlog_mu written, not accumulated
  int dc_rows;          // column pass: add the row-softmax term of this step into dC (i = 1)
};

// Row pass of iteration i: one warp per row r, 16-byte loads over j when the
// rows are 16-byte aligned.
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
    const float eps = a.eps[h], kap = kappa_of(a.lam, eps), ikap = 1.0f / kap;
    const float sc = -kLog2e / eps, cdc = kap / eps;
    const float rb = bias_of(a.mask, b, N, i);
    // column-softmax exponent: C sc + (u_i,r + rb_r) log2e + (v_i,j / kappa - b_j) log2e
    const float yr = (a.u[r] + rb) * kLog2e;
    // row-softmax exponent of step i + 1: C sc + (v_i,j + cb_j) log2e + (u_i+1,r / kappa - a_r) log2e
    const bool rowterm = a.u1 != nullptr;
    const float xr = rowterm ? (a.u1[r] * ikap - a.mu[r]) * kLog2e : 0.0f;
    const float wr = rowterm ? cdc * a.gu1[r] : 0.0f;
    const float* c = a.C + r * N;
    float* dc = a.dC == nullptr ? nullptr : a.dC + r * N;
    const float* v = a.v + prob * N;
    const float* nu = a.nu + prob * N;
    const float* gv = a.g + prob * N;
    const float* mk = a.mask == nullptr ? nullptr : a.mask + static_cast<size_t>(b) * N;
    float acc = 0.0f;
    auto elem = [&](float cj, float vj, float nj, float gj, float cbj, float& dcj) {
      const float base = cj * sc;
      const float pc = ex2c(base + fmaf(vj * ikap - nj, kLog2e, yr));
      const float t = gj * pc;
      acc += t;
      float d = cdc * t;
      if (rowterm) d = fmaf(wr, ex2c(base + fmaf(vj + cbj, kLog2e, xr)), d);
      dcj = a.first ? d : dcj + d;
    };
    if constexpr (VEC) {
      for (int j = 4 * lane; j < N; j += 128) {
        const float4 cv = __ldcs(reinterpret_cast<const float4*>(c + j));
        const float4 vv = ld4(v + j), nv = ld4(nu + j), gw = ld4(gv + j);
        float4 cb = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (mk != nullptr) {
          const float4 m = ld4(mk + j);
          cb = make_float4((1.0f - m.x) * kMaskBias, (1.0f - m.y) * kMaskBias, (1.0f - m.z) * kMaskBias,
                           (1.0f - m.w) * kMaskBias);
        }
        float4 dv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (dc != nullptr && !a.first) dv = __ldcs(reinterpret_cast<const float4*>(dc + j));
        elem(cv.x, vv.x, nv.x, gw.x, cb.x, dv.x);
        elem(cv.y, vv.y, nv.y, gw.y, cb.y, dv.y);
        elem(cv.z, vv.z, nv.z, gw.z, cb.z, dv.z);
        elem(cv.w, vv.w, nv.w, gw.w, cb.w, dv.w);
        if (dc != nullptr) __stcs(reinterpret_cast<float4*>(dc + j), dv);
      }
    } else {
      for (int j = lane; j < N; j += 32) {
        float dv = (dc != nullptr && !a.first) ? dc[j] : 0.0f;
        elem(__ldcs(c + j), v[j], nu[j], gv[j], bias_of(a.mask, b, N, j), dv);
        if (dc != nullptr) dc[j] = dv;
      }
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

// Column pass of iteration i: CTA = COLS columns of one problem, warp w takes
// rows w, w + 8, ...; per-column partial sums added over the warps in a fixed
// order (deterministic).
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
  const float sc = -kLog2e / eps, cdc = kap / eps;
  const int j = j0 + PER * lane;
  float cb[PER], acc[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    cb[q] = (j + q < N) ? (a.v[prob * N + j + q] + bias_of(a.mask, b, N, j + q)) * kLog2e : 0.0f;
    acc[q] = 0.0f;
  }
  float* dcb = a.dc_rows && a.dC != nullptr ? a.dC + prob * N * static_cast<size_t>(N) + j : nullptr;
  if (j < N) {
    const float* cbase = a.C + prob * N * static_cast<size_t>(N) + j;
    const float* ur = a.u + prob * N;
    const float* mur = a.mu + prob * N;
    const float* gur = a.g + prob * N;
    for (int i = warp; i < N; i += 8) {
      const float gu = gur[i];
      const float xr = (ur[i] * ikap - mur[i]) * kLog2e;  // u_i,r / kappa - a_r
      const size_t off = static_cast<size_t>(i) * N;
      if constexpr (VEC) {
        const float4 cv = __ldcs(reinterpret_cast<const float4*>(cbase + off));
        const float p0 = ex2c(fmaf(cv.x, sc, cb[0]) + xr), p1 = ex2c(fmaf(cv.y, sc, cb[1]) + xr);
        const float p2 = ex2c(fmaf(cv.z, sc, cb[2]) + xr), p3 = ex2c(fmaf(cv.w, sc, cb[3]) + xr);
        acc[0] = fmaf(gu, p0, acc[0]);
        acc[1] = fmaf(gu, p1, acc[1]);
        acc[2] = fmaf(gu, p2, acc[2]);
        acc[3] = fmaf(gu, p3, acc[3]);
        if (dcb != nullptr) {
          const float w = cdc * gu;
          float4 dv = __ldcs(reinterpret_cast<const float4*>(dcb + off));
          dv.x = fmaf(w, p0, dv.x);
          dv.y = fmaf(w, p1, dv.y);
          dv.z = fmaf(w, p2, dv.z);
          dv.w = fmaf(w, p3, dv.w);
          __stcs(reinterpret_cast<float4*>(dcb + off), dv);
        }
      } else {
        const float p = ex2c(fmaf(__ldcs(cbase + off), sc, cb[0]) + xr);
        acc[0] = fmaf(gu, p, acc[0]);
        if (dcb != nullptr) dcb[off] = fmaf(cdc * gu, p, dcb[off]);
      }
    }
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
    a.gout[o] = gv;
    if (a.dsum != nullptr) a.dsum[o] += kap * gv;
  }
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

}  // namespace

// The reverse of iterations iters .. 1 (scratch: 3 x BH x N floats -- gv, and gu
// for two consecutive iterations, since a row pass reads gu_i+1 while it writes gu_i).
cudaError_t launch_dense_solve_bwd(int B, int H, int N, int iters, float lam, const float* C, const float* eps,
                                   const float* mu, const float* nu, const float* mask, const float* hist,
                                   const float* g_lu, const float* g_lv, float* dC, float* dmu, float* dnu,
                                   float* dlui, float* dlvi, float* scratch, cudaStream_t st) {
  const size_t n = static_cast<size_t>(B) * H * N;
  float* gv = scratch;
  float* gu[2] = {scratch + n, scratch + 2 * n};
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
  // gv_K = the masked upstream adjoint of v_K, dlog_nu = kappa gv_K; gu_up masked into gu[1]
  masked_adjoint_kernel<<<ge, 256, 0, st>>>(g_lv, mask, eps, lam, H, N, n, gv, dnu);
  masked_adjoint_kernel<<<ge, 256, 0, st>>>(g_lu, mask, eps, lam, H, N, n, gu[iters & 1 ? 0 : 1], nullptr);
  if (dlui && (e = cudaMemsetAsync(dlui, 0, n * sizeof(float), st)) != cudaSuccess) return e;
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const bool vec = (N % 4) == 0 && aligned16(C) && (dC == nullptr || aligned16(dC));
  const unsigned grow = grid_for(n, kRevThreads / 32);
  const int cols = vec ? 128 : 32;
  const unsigned gcol = static_cast<unsigned>(B) * H * static_cast<unsigned>((N + cols - 1) / cols);
  auto slot = [&](int k) { return hist + static_cast<size_t>(k) * n; };
  for (int i = iters; i >= 1 && e == cudaSuccess; --i) {
    // gu_i goes to gu[i & 1]; gu_i+1 (or the masked upstream at i = K) sits in gu[(i + 1) & 1]
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
    a.dC = dC;
    a.u = slot(2 * i);
    a.v = slot(2 * i + 1);
    a.g = gv;
    a.gup = i == iters ? gu[(i + 1) & 1] : nullptr;
    a.u1 = i == iters ? nullptr : slot(2 * i + 2);
    a.gu1 = i == iters ? nullptr : gu[(i + 1) & 1];
    a.gout = gu[i & 1];
    a.dsum = dmu;
    a.first = i == iters;
    if (vec) rev_row_kernel<true><<<grow, kRevThreads, 0, st>>>(a);
    else rev_row_kernel<false><<<grow, kRevThreads, 0, st>>>(a);
    // column pass: gv_i-1 from gu_i; the adjoint of the warm start at i = 1
    RevArgs c = a;
    c.u = slot(2 * i);
    c.v = slot(2 * i - 1);
    c.g = gu[i & 1];
    c.gup = c.u1 = c.gu1 = nullptr;
    c.gout = i > 1 ? gv : (dlvi != nullptr ? dlvi : gv);
    c.dsum = i > 1 ? dnu : nullptr;
    c.first = 0;
    c.dc_rows = i == 1;
    if (vec) rev_col_kernel<true><<<gcol, kRevThreads, 0, st>>>(c);
    else rev_col_kernel<false><<<gcol, kRevThreads, 0, st>>>(c);
    e = cudaGetLastError();
  }
  return e;
}

}  // namespace dfs

using namespace dfs;

namespace {
bool dims_ok(int B, int H, int N) {
  return B > 0 && H > 0 && N > 0 && N <= (1 << 16) && static_cast<long long>(B) * H <= (1 << 24);
}
int status_of(cudaError_t e) { return e == cudaSuccess ? DFS_OK : DFS_ERR_CUDA; }
}  // namespace

extern "C" int dfs_dense_iterate(int B, int H, int N, float lam, const float* C, const float* eps,
                                 const float* log_mu, const float* log_nu, const float* log_u_init,
                                 const float* log_v_init, const float* mask, float* hist, int it_begin, int it_end,
                                 float* log_u, float* log_v, float* change, int32_t* status, void* stream) {
  if (!dims_ok(B, H, N) || C == nullptr || eps == nullptr || log_mu == nullptr || log_nu == nullptr ||
      hist == nullptr || log_u == nullptr || log_v == nullptr || it_begin < 0 || it_end < it_begin ||
      !(lam > 0.0f))
    return DFS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t n = static_cast<size_t>(B) * H * N;
  const unsigned ge = grid_for(n, 256);
  if (it_begin == 0) hist_init_kernel<<<ge, 256, 0, st>>>(log_u_init, log_v_init, hist, hist + n, n);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess)
    e = launch_dense_iterations(C, eps, log_mu, log_nu, mask, B, H, N, lam, hist, it_begin, it_end, st);
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
