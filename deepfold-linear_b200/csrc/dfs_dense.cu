// dfs_dense.cu -- Sinkhorn on a caller-given dense cost C (B, H, N, N) fp32 for
// problems the cluster-resident kernels do not hold (N > 384, or a V head dim
// above 32): the dense entry points sinkhorn_solve and compute_transport_output
// of the reference (src/deepfold/model/sinkhorn.py:17-112, 115-198).
//
// The cost is the input here, so every pass is a stream over C in HBM (4 bytes
// per pair) with a handful of flops per pair: no tensor-core work exists to
// reshape it into.  The passes are coalesced 16-byte loads (4-byte ones when a
// row of C is not 16-byte aligned), sized so that one launch covers the GPU:
//   row update     one warp per row i: LSE_j(-C_ij / eps + log_v_j + colbias_j)
//   column update  one CTA per 128 (or 32) columns j, its 8 warps over
//                  interleaved rows i, per-column online (max, sum) merged in
//                  shared memory: LSE_i(-C_ij / eps + log_u_i + rowbias_i)
//   transport      one warp per row, 8 rows per CTA: pass 1 the row's max and
//                  sum, pass 2 T_norm_ij per column, O_i += T_norm_ij V_j with
//                  the CTA's V tile staged in shared memory, x_centroid.
// For N <= 8192 one iteration is one read of C instead (dense_fused_kernel):
// a CTA finishes the row updates of eight rows and folds the same rows, re-read
// from L1 / L2, into per-column partials kept in shared memory; a small kernel
// merges the CTAs' partials into the column update.
// The arithmetic follows the reference's formulas -- log K = -C / eps, masks as
// additive -1e9 biases, kappa = lam / (lam + eps) (1 for lam = inf), T =
// exp(score - rowmax), T_norm = T / (sum T + 1e-6), padded rows of T_norm and
// padded potentials zeroed -- in log2 units with ex2 on the MUFU (below), so
// that a pass costs about one FMA and one exponential per element and is bound
// by HBM, not by the arithmetic.
//
// Early stopping (threshold > 0): on every check_every-th iteration the passes
// record each problem's largest |change| of log_u and log_v; a one-CTA kernel
// then marks the problems whose change is below the threshold done, and the
// later passes skip them -- each (batch, head) problem stops on its own, as on
// the resident path.
#include <algorithm>

#include "dfs_kernels.cuh"

namespace dfs {
namespace {

constexpr float kMaskBias = -1e9f;
constexpr int kDenseThreads = 256;  // 8 warps

struct DenseArgs {
  const float* C;
  const float* eps;
  const float* mu;      // log_mu (B,H,N)
  const float* nu;      // log_nu
  const float* mask;    // (B,N) or null
  float* lu;            // log_u (B,H,N): state and result
  float* lv;            // log_v
  unsigned* diff;       // (2, BH) largest |change| as float bits (check iterations)
  int* done;            // (BH) converged problems
  float* rmax;          // transport row statistics (B,H,N): exact maximum of the score, log2 units
  float* rsum;          // and the sum of exp2(score - maximum)
  int B, H, N;
  float lam;
  int check;            // this pass records |change|
};

__device__ __forceinline__ float kappa_of(float lam, float eps) { return isinf(lam) ? 1.0f : lam / (lam + eps); }

__device__ __forceinline__ float bias_of(const float* mask, int b, int N, int j) {
  return mask == nullptr ? 0.0f : (1.0f - mask[static_cast<size_t>(b) * N + j]) * kMaskBias;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The passes work in log2 units: x = (-C / eps + potential + bias) log2(e) is one
// FMA per element, c * (-log2(e) / eps) + (potential + bias) log2(e), and each
// exponential one ex2 on the MUFU.  The running reference m lags the maximum by
// up to kLag: a group of four elements moves it only when its own maximum
// exceeds m + kLag, so the sum of exp2(x - m) stays within [1, N 2^kLag] and the
// common case has no branch.  The result is ln(sum exp(...)) = (m + log2 s) ln 2.
constexpr float kLag = 16.0f;  // (kLog2e, kLn2: dfs_device.cuh)

__device__ __forceinline__ void lse_push4(float& m, float& s, float x0, float x1, float x2, float x3) {
  const float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
  if (mx > m + kLag) {  // the first group with a finite value, and rarely any other
    s *= ex2f(m - mx);  // m = -inf first: exp2(-inf) = 0
    m = mx;
  }
  if (m > -INFINITY) s += (ex2f(x0 - m) + ex2f(x1 - m)) + (ex2f(x2 - m) + ex2f(x3 - m));
}
__device__ __forceinline__ void lse_push1(float& m, float& s, float x) {
  if (x > m + kLag) {
    s *= ex2f(m - x);
    m = x;
  }
  if (m > -INFINITY) s += ex2f(x - m);
}
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * ex2f(m - m2) + s2;
    m = m2;
  } else if (m2 > -INFINITY) {
    s += s2 * ex2f(m2 - m);
  }
}

__device__ __forceinline__ void record_change(unsigned* slot, float a) {
  // non-negative floats order like their bit patterns (NaN ends above every number)
  atomicMax(slot, __float_as_uint(a));
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// f_i = kappa (log_mu_i - LSE_j(-C_ij / eps + g_j + colbias_j)), one warp per row.
// STAT: the transport's row statistics instead, on the score f_i - C_ij / eps +
// g_j + colbias_j (log2 units): its exact maximum into a.rmax and the sum of
// exp2(score - maximum) into a.rsum.
template <bool VEC, bool STAT>
__global__ void __launch_bounds__(kDenseThreads) dense_row_kernel(const DenseArgs a) {
  const int lane = threadIdx.x & 31;
  const size_t rows = static_cast<size_t>(a.B) * a.H * a.N;
  const size_t warp0 = (static_cast<size_t>(blockIdx.x) * kDenseThreads + threadIdx.x) >> 5;
  const size_t nwarps = (static_cast<size_t>(gridDim.x) * kDenseThreads) >> 5;
  const int N = a.N;
  for (size_t r = warp0; r < rows; r += nwarps) {
    const size_t prob = r / N;
    if (a.done != nullptr && a.done[prob]) continue;  // uniform over the warp
    const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
    const float eps = a.eps[h];
    const float sc = -kLog2e / eps;
    const float* c = a.C + r * N;
    const float* g = a.lv + prob * N;
    const float* mk = a.mask == nullptr ? nullptr : a.mask + static_cast<size_t>(b) * N;
    const float ui = STAT ? a.lu[r] : 0.0f;
    float m = -INFINITY, s = 0.0f, mt = -INFINITY;
    if constexpr (VEC) {
      // four 16-byte loads of C in flight per lane before any is consumed
      auto group = [&](const float4& cv, int j) {
        float4 t = ld4(g + j);
        if constexpr (STAT) {
          t.x += ui;
          t.y += ui;
          t.z += ui;
          t.w += ui;
        }
        if (mk != nullptr) {
          const float4 mv = ld4(mk + j);
          t.x += (1.0f - mv.x) * kMaskBias;
          t.y += (1.0f - mv.y) * kMaskBias;
          t.z += (1.0f - mv.z) * kMaskBias;
          t.w += (1.0f - mv.w) * kMaskBias;
        }
        const float x0 = fmaf(cv.x, sc, t.x * kLog2e), x1 = fmaf(cv.y, sc, t.y * kLog2e),
                    x2 = fmaf(cv.z, sc, t.z * kLog2e), x3 = fmaf(cv.w, sc, t.w * kLog2e);
        if constexpr (STAT) mt = fmaxf(mt, fmaxf(fmaxf(x0, x1), fmaxf(x2, x3)));
        lse_push4(m, s, x0, x1, x2, x3);
      };
      int j = 4 * lane;
      for (; j + 384 < N; j += 512) {
        float4 cv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) cv[u] = __ldcs(reinterpret_cast<const float4*>(c + j + 128 * u));
#pragma unroll
        for (int u = 0; u < 4; ++u) group(cv[u], j + 128 * u);
      }
      for (; j < N; j += 128) group(__ldcs(reinterpret_cast<const float4*>(c + j)), j);
    } else {
      for (int j = lane; j < N; j += 32) {
        const float x = fmaf(__ldcs(c + j), sc, (ui + g[j] + bias_of(a.mask, b, N, j)) * kLog2e);
        if constexpr (STAT) mt = fmaxf(mt, x);
        lse_push1(m, s, x);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      lse_merge(m, s, m2, s2);
      if constexpr (STAT) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
    }
    if constexpr (STAT) {
      if (lane == 0) {
        a.rmax[r] = mt;
        a.rsum[r] = mt > -INFINITY ? s * ex2f(m - mt) : 0.0f;
      }
      continue;
    }
    if (lane == 0) {
      const size_t i = r;
      const float f = kappa_of(a.lam, eps) * (a.mu[i] - (m + __log2f(s)) * kLn2);
      if (a.check) record_change(a.diff + prob, fabsf(f - a.lu[i]));
      a.lu[i] = f;
    }
  }
}

// g_j = kappa (log_nu_j - LSE_i(-C_ij / eps + f_i + rowbias_i)); CTA = COLS
// columns of one problem, warp w takes rows w, w + 8, ...
template <bool VEC>
__global__ void __launch_bounds__(kDenseThreads) dense_col_kernel(const DenseArgs a) {
  constexpr int COLS = VEC ? 128 : 32, PER = VEC ? 4 : 1;
  __shared__ float sm[8][COLS], ss[8][COLS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = a.N;
  const int cblocks = (N + COLS - 1) / COLS;
  const size_t prob = blockIdx.x / cblocks;
  const int j0 = (blockIdx.x % cblocks) * COLS;
  if (a.done != nullptr && a.done[prob]) return;  // uniform over the CTA
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float eps = a.eps[h];
  const float sc = -kLog2e / eps;
  const float* f = a.lu + prob * N;
  float m[PER], s[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    m[q] = -INFINITY;
    s[q] = 0.0f;
  }
  const int j = j0 + PER * lane;
  if (j < N) {
    const float* cb = a.C + prob * N * static_cast<size_t>(N) + j;
    auto row = [&](int i, const float4& cv) {
      const float ti = (f[i] + bias_of(a.mask, b, N, i)) * kLog2e;
      lse_push1(m[0], s[0], fmaf(cv.x, sc, ti));
      if constexpr (VEC) {
        lse_push1(m[1], s[1], fmaf(cv.y, sc, ti));
        lse_push1(m[2], s[2], fmaf(cv.z, sc, ti));
        lse_push1(m[3], s[3], fmaf(cv.w, sc, ti));
      }
    };
    auto load = [&](int i) {
      if constexpr (VEC) return __ldcs(reinterpret_cast<const float4*>(cb + static_cast<size_t>(i) * N));
      else return make_float4(__ldcs(cb + static_cast<size_t>(i) * N), 0.0f, 0.0f, 0.0f);
    };
    // rows warp, warp + 8, ...: four loads in flight per thread before any is
    // consumed, and each column's four new values pushed as one group
    int i = warp;
    for (; i + 24 < N; i += 32) {
      float4 cv[4];
      float ti[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) cv[u] = load(i + 8 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) ti[u] = (f[i + 8 * u] + bias_of(a.mask, b, N, i + 8 * u)) * kLog2e;
      lse_push4(m[0], s[0], fmaf(cv[0].x, sc, ti[0]), fmaf(cv[1].x, sc, ti[1]), fmaf(cv[2].x, sc, ti[2]),
                fmaf(cv[3].x, sc, ti[3]));
      if constexpr (VEC) {
        lse_push4(m[1], s[1], fmaf(cv[0].y, sc, ti[0]), fmaf(cv[1].y, sc, ti[1]), fmaf(cv[2].y, sc, ti[2]),
                  fmaf(cv[3].y, sc, ti[3]));
        lse_push4(m[2], s[2], fmaf(cv[0].z, sc, ti[0]), fmaf(cv[1].z, sc, ti[1]), fmaf(cv[2].z, sc, ti[2]),
                  fmaf(cv[3].z, sc, ti[3]));
        lse_push4(m[3], s[3], fmaf(cv[0].w, sc, ti[0]), fmaf(cv[1].w, sc, ti[1]), fmaf(cv[2].w, sc, ti[2]),
                  fmaf(cv[3].w, sc, ti[3]));
      }
    }
    for (; i < N; i += 8) row(i, load(i));
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    sm[warp][PER * lane + q] = m[q];
    ss[warp][PER * lane + q] = s[q];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < COLS; t += kDenseThreads) {
    const int jj = j0 + t;
    if (jj >= N) continue;
    float mm = sm[0][t], sv = ss[0][t];
    for (int w = 1; w < 8; ++w) lse_merge(mm, sv, sm[w][t], ss[w][t]);
    const size_t o = prob * N + jj;
    const float g = kappa_of(a.lam, eps) * (a.nu[o] - (mm + __log2f(sv)) * kLn2);
    if (a.check) record_change(a.diff + static_cast<size_t>(a.B) * a.H + prob, fabsf(g - a.lv[o]));
    a.lv[o] = g;
  }
}

// problems whose largest change of this check is below the threshold are done
__global__ void dense_check_kernel(unsigned* diff, int* done, int BH, float threshold) {
  for (int p = threadIdx.x; p < BH; p += blockDim.x) {
    const float du = __uint_as_float(diff[p]), dv = __uint_as_float(diff[BH + p]);
    if (fmaxf(du, dv) < threshold) done[p] = 1;  // NaN compares false: keeps iterating
    diff[p] = 0u;
    diff[BH + p] = 0u;
  }
}

// start values (warm start or zeros) into the outputs, per-problem state cleared
__global__ void dense_init_kernel(const float* lui, const float* lvi, float* lu, float* lv, size_t n, unsigned* diff,
                                  int* done, int BH) {
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    lu[k] = lui != nullptr ? lui[k] : 0.0f;
    lv[k] = lvi != nullptr ? lvi[k] : 0.0f;
    if (k < static_cast<size_t>(BH)) {
      diff[k] = 0u;
      diff[BH + k] = 0u;
      done[k] = 0;
    }
  }
}

// padded potentials zeroed (sinkhorn.py:107-110); non-finite valid ones flagged
__global__ void dense_finish_kernel(const float* mask, float* lu, float* lv, int B, int H, int N, int32_t* status) {
  const size_t n = static_cast<size_t>(B) * H * N;
  int bad = 0;
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(k / (static_cast<size_t>(H) * N)), i = static_cast<int>(k % N);
    if (mask != nullptr) {
      const float mv = mask[static_cast<size_t>(b) * N + i];
      lu[k] *= mv;
      lv[k] *= mv;
    }
    bad |= !isfinite(lu[k]) || !isfinite(lv[k]);
  }
  if (bad && status != nullptr) atomicOr(status, DFS_ERR_NUMERIC);
}

}  // namespace

namespace {

// compute_transport_output (sinkhorn.py:152-195) on a dense cost, after the
// row statistics (dense_row_kernel<., true>: each row's exact score maximum mt
// and sum of exp2(score - mt)).  A CTA takes 128 rows of one problem and walks
// the columns in chunks of 64.  Per chunk: T_norm_ij = exp2(score_ij - mt_i) /
// (sum_i + 1e-6) (0 on a padded row) from coalesced 16-byte loads of C (thread
// t: rows t / 16 + 16 m, columns 4 (t % 16) ...), written out when T_norm is
// asked for, added into the rows' centroid partials and staged in shared memory
// beside the chunk's 64 rows of V; then O = T_norm V as a register-blocked
// product, thread t accumulating rows t / 8 + 32 m (m < 4) and head dims
// DPT (t % 8) .. + DPT - 1 with packed pair FMAs: per four columns, four 16-byte
// reads of T and 4 DPT / 4 of V, each one shared-memory wavefront per warp, for
// 8 DPT pair FMAs (64 at DPT = 8), so the product is bound by the FMA pipes.
struct DenseOutArgs {
  const float* C;
  const float* V;     // (B,H,N,d) fp32 or null
  const float* x;     // (B,N,3) or null
  const float* eps;
  const float* mask;
  const float* lu;
  const float* lv;
  const float* rmax;  // row statistics of the score (log2 units)
  const float* rsum;
  float* O;           // (B,H,N,d)
  float* T;           // (B,H,N,N) or null
  float* xc;          // (B,H,N,3) or null
  int B, H, N, d;
};

constexpr int kOutRows = 128, kOutCols = 64, kOutTS = kOutCols + 4;  // T tile row stride (floats)
constexpr int kOutTR = kOutRows / 16, kOutPR = kOutRows / 32;  // rows per thread: T side, product side

template <int DPT>
size_t dense_out_smem() {
  return sizeof(float) * (static_cast<size_t>(kOutRows) * kOutTS + static_cast<size_t>(kOutCols) * 8 * DPT);
}

template <int DPT, bool VEC>  // DPT: O's head dims per thread (d <= 8 DPT)
__global__ void __launch_bounds__(kDenseThreads) dense_out_kernel(const DenseOutArgs a) {
  constexpr int DP = 8 * DPT;
  extern __shared__ float4 smo4[];
  float* Ts = reinterpret_cast<float*>(smo4);     // [128][68]
  float* Vs = Ts + kOutRows * kOutTS;             // [64][DP] (dims beyond d zero)
  const int tid = threadIdx.x, lane = tid & 31;
  const int N = a.N, d = a.d;
  const int rblocks = (N + kOutRows - 1) / kOutRows;
  const size_t prob = blockIdx.x / rblocks;
  const int i0 = (blockIdx.x % rblocks) * kOutRows;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float sc = -kLog2e / a.eps[h];
  const float* g = a.lv + prob * N;
  const float* xb = a.x != nullptr ? a.x + static_cast<size_t>(b) * N * 3 : nullptr;
  // T side: rows lrow0 + 16 m (m < kOutTR), columns 4 c4 .. + 3 of each chunk
  const int lrow0 = tid >> 4, c4 = tid & 15;
  float ui[kOutTR], mt[kOutTR], inv[kOutTR], cx[kOutTR], cy[kOutTR], cz[kOutTR];
#pragma unroll
  for (int m = 0; m < kOutTR; ++m) {
    const int i = i0 + lrow0 + 16 * m;
    const size_t r = prob * N + (i < N ? i : 0);
    const bool ok = i < N;
    ui[m] = ok ? a.lu[r] : 0.0f;
    mt[m] = ok ? a.rmax[r] : 0.0f;
    const float rm = (!ok) ? 0.0f : (a.mask == nullptr ? 1.0f : a.mask[static_cast<size_t>(b) * N + i]);
    inv[m] = ok ? rm / (a.rsum[r] + 1e-6f) : 0.0f;
    cx[m] = cy[m] = cz[m] = 0.0f;
  }
  // product side: rows rg + 32 m (m < kOutPR), dims DPT dg .. + DPT - 1
  const int rg = tid >> 3, dg = tid & 7;
  float2 acc[kOutPR][DPT / 2];
#pragma unroll
  for (int m = 0; m < kOutPR; ++m)
#pragma unroll
    for (int q = 0; q < DPT / 2; ++q) acc[m][q] = make_float2(0.0f, 0.0f);
  for (int j0 = 0; j0 < N; j0 += kOutCols) {
    const int jc = j0 + 4 * c4;  // this thread's 4 columns
    float gb[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) gb[e] = (jc + e < N) ? (g[jc + e] + bias_of(a.mask, b, N, jc + e)) : 0.0f;
    __syncthreads();  // the previous chunk's product is done with Ts / Vs
#pragma unroll
    for (int m = 0; m < kOutTR; ++m) {
      const int li = lrow0 + 16 * m, i = i0 + li;
      const float* crow = a.C + (prob * N + (i < N ? i : 0)) * static_cast<size_t>(N);
      float cv[4];
      if (VEC && i < N && jc + 4 <= N) {
        const float4 c = __ldcs(reinterpret_cast<const float4*>(crow + jc));
        cv[0] = c.x; cv[1] = c.y; cv[2] = c.z; cv[3] = c.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) cv[e] = (i < N && jc + e < N) ? __ldcs(crow + jc + e) : 0.0f;
      }
      float t[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = jc + e;
        // the reference's T / (sum + 1e-6), then the padded-row factor (in inv)
        t[e] = (i < N && j < N) ? ex2f(fmaf(cv[e], sc, (ui[m] + gb[e]) * kLog2e) - mt[m]) * inv[m] : 0.0f;
        if (xb != nullptr && j < N) {
          cx[m] = fmaf(t[e], xb[3 * j], cx[m]);
          cy[m] = fmaf(t[e], xb[3 * j + 1], cy[m]);
          cz[m] = fmaf(t[e], xb[3 * j + 2], cz[m]);
        }
      }
      *reinterpret_cast<float4*>(Ts + li * kOutTS + 4 * c4) = make_float4(t[0], t[1], t[2], t[3]);
      if (a.T != nullptr && i < N) {
        float* trow = a.T + (prob * N + i) * static_cast<size_t>(N);
        if (VEC && jc + 4 <= N) {
          __stcs(reinterpret_cast<float4*>(trow + jc), make_float4(t[0], t[1], t[2], t[3]));
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (jc + e < N) __stcs(trow + jc + e, t[e]);
        }
      }
    }
    if (a.V == nullptr) continue;  // uniform: no O asked for
    const float* vsrc = a.V + (prob * N + j0) * static_cast<size_t>(d);
    const int rows = min(kOutCols, N - j0);
    // every CTA of a problem reads all of V (from L2): 16-byte loads where the rows allow
    if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(a.V) & 15u) == 0) {
      const int d4 = d >> 2, DP4 = DP / 4;
      for (int e = tid; e < kOutCols * DP4; e += kDenseThreads) {
        const int c = e / DP4, k4 = e - c * DP4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < rows && k4 < d4) v = __ldg(reinterpret_cast<const float4*>(vsrc + static_cast<size_t>(c) * d) + k4);
        reinterpret_cast<float4*>(Vs)[e] = v;
      }
    } else {
      for (int e = tid; e < kOutCols * DP; e += kDenseThreads) {
        const int c = e / DP, k = e - c * DP;
        Vs[e] = (c < rows && k < d) ? __ldg(vsrc + static_cast<size_t>(c) * d + k) : 0.0f;
      }
    }
    __syncthreads();
    // rows rg + 32 m: the four rows a warp reads start on banks 16 w + {0, 4, 8, 12}
    // (row stride 68 floats), so each 16-byte read of four columns of T is one
    // wavefront; V's 8 head-dim groups are one more per 16-byte read
    const float* tb = Ts + rg * kOutTS;
    const float* vb = Vs + DPT * dg;
#pragma unroll 2
    for (int c = 0; c < kOutCols; c += 4) {
      float4 tq[kOutPR];
#pragma unroll
      for (int m = 0; m < kOutPR; ++m) tq[m] = *reinterpret_cast<const float4*>(tb + 32 * m * kOutTS + c);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float2 v[DPT / 2];
#pragma unroll
        for (int q = 0; q < DPT / 4; ++q) {
          const float4 v4 = *reinterpret_cast<const float4*>(vb + (c + cc) * DP + 4 * q);
          v[2 * q] = make_float2(v4.x, v4.y);
          v[2 * q + 1] = make_float2(v4.z, v4.w);
        }
#pragma unroll
        for (int m = 0; m < kOutPR; ++m) {
          const float tv = cc == 0 ? tq[m].x : (cc == 1 ? tq[m].y : (cc == 2 ? tq[m].z : tq[m].w));
          const float2 t2 = make_float2(tv, tv);
#pragma unroll
          for (int q = 0; q < DPT / 2; ++q) acc[m][q] = __ffma2_rn(t2, v[q], acc[m][q]);
        }
      }
    }
  }
  if (a.xc != nullptr) {
    // the 16 threads of a row are consecutive lanes of one warp
#pragma unroll
    for (int m = 0; m < kOutTR; ++m) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        cx[m] += __shfl_xor_sync(0xffffffffu, cx[m], o);
        cy[m] += __shfl_xor_sync(0xffffffffu, cy[m], o);
        cz[m] += __shfl_xor_sync(0xffffffffu, cz[m], o);
      }
      const int i = i0 + lrow0 + 16 * m;
      if (c4 == 0 && i < N) {
        const size_t r = prob * N + i;
        a.xc[r * 3] = cx[m];
        a.xc[r * 3 + 1] = cy[m];
        a.xc[r * 3 + 2] = cz[m];
      }
    }
  }
  (void)lane;
  if (a.O != nullptr) {
#pragma unroll
    for (int m = 0; m < kOutPR; ++m) {
      const int i = i0 + rg + 32 * m;
      if (i >= N) continue;
      float* orow = a.O + (prob * N + i) * static_cast<size_t>(d);
#pragma unroll
      for (int q = 0; q < DPT / 2; ++q) {
        const int k = DPT * dg + 2 * q;
        if (k < d) orow[k] = acc[m][q].x;
        if (k + 1 < d) orow[k + 1] = acc[m][q].y;
      }
    }
  }
}

// One Sinkhorn iteration in one read of C (N <= kFuseMaxN).  A CTA takes rows
// [r0, r1) of one problem, eight at a time (one per warp):
//   pass A  each warp finishes its row's update u_i (the row LSE over j, four
//           16-byte loads of C in flight per lane, as dense_row_kernel);
//   pass B  the CTA re-reads the same eight rows -- just fetched, so from L1 /
//           L2, not HBM -- with thread t owning columns 4t + 1024k, and folds
//           them into its columns' online (max, sum) of the column update,
//           kept in shared memory across all the CTA's rows.
// Each CTA then writes its columns' partial (max, sum); dense_fused_merge adds
// the CTA partials of a problem into v_i.  HBM traffic per iteration: C once
// (4 bytes per element) plus 8 bytes per column per CTA of partials, against
// 8 bytes per element for the separate row and column passes.
constexpr int kFuseMaxN = 8192;

struct FusePlan {
  int S;    // CTAs (row ranges) per problem
  int rpu;  // rows per CTA, a multiple of 8
};

// CTAs per problem: as many as fill the GPU once (no partial second wave)
FusePlan fuse_plan(int BH, int N, int slots) {
  FusePlan p;
  p.S = std::max(1, std::min(slots / std::max(BH, 1), (N + 7) / 8));
  p.rpu = ((N + p.S - 1) / p.S + 7) / 8 * 8;
  p.S = (N + p.rpu - 1) / p.rpu;
  return p;
}

size_t fuse_smem(int N) { return static_cast<size_t>(2) * N * sizeof(float) + 16 * sizeof(float); }

template <bool VEC>
__global__ void __launch_bounds__(kDenseThreads) dense_fused_kernel(const DenseArgs a, FusePlan plan, float* part) {
  extern __shared__ __align__(16) float fsm[];
  const int N = a.N;
  float* cm = fsm;          // column running maximum (log2 units)
  float* cs = fsm + N;      // column sum of exp2(x - max)
  float* tw = fsm + 2 * N;  // this group's row terms (u_r + rowbias_r) log2e
  const size_t prob = blockIdx.x / plan.S;
  const int r0 = static_cast<int>(blockIdx.x % plan.S) * plan.rpu, r1 = min(N, r0 + plan.rpu);
  if (a.done != nullptr && a.done[prob]) return;  // uniform over the CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const float eps = a.eps[h];
  const float sc = -kLog2e / eps, kap = kappa_of(a.lam, eps);
  const float* g = a.lv + prob * N;
  const float* mk = a.mask == nullptr ? nullptr : a.mask + static_cast<size_t>(b) * N;
  const float* cprob = a.C + prob * static_cast<size_t>(N) * N;
  for (int j = threadIdx.x; j < N; j += kDenseThreads) {
    cm[j] = -INFINITY;
    cs[j] = 0.0f;
  }
  for (int g0 = r0; g0 < r1; g0 += 8) {
    // pass A: row update of row g0 + warp
    const int ri = g0 + warp;
    if (ri < r1) {
      const float* c = cprob + static_cast<size_t>(ri) * N;
      float m = -INFINITY, s = 0.0f;
      if constexpr (VEC) {
        auto group = [&](const float4& cv, int j) {
          float4 t = ld4(g + j);
          if (mk != nullptr) {
            const float4 mv = ld4(mk + j);
            t.x += (1.0f - mv.x) * kMaskBias;
            t.y += (1.0f - mv.y) * kMaskBias;
            t.z += (1.0f - mv.z) * kMaskBias;
            t.w += (1.0f - mv.w) * kMaskBias;
          }
          lse_push4(m, s, fmaf(cv.x, sc, t.x * kLog2e), fmaf(cv.y, sc, t.y * kLog2e), fmaf(cv.z, sc, t.z * kLog2e),
                    fmaf(cv.w, sc, t.w * kLog2e));
        };
        int j = 4 * lane;
        for (; j + 384 < N; j += 512) {
          float4 cv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) cv[u] = ld4(c + j + 128 * u);  // plain loads: kept in L2 for pass B
#pragma unroll
          for (int u = 0; u < 4; ++u) group(cv[u], j + 128 * u);
        }
        for (; j < N; j += 128) group(ld4(c + j), j);
      } else {
        for (int j = lane; j < N; j += 32) lse_push1(m, s, fmaf(c[j], sc, (g[j] + bias_of(a.mask, b, N, j)) * kLog2e));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
        lse_merge(m, s, m2, s2);
      }
      if (lane == 0) {
        const size_t i = prob * N + ri;
        const float f = kap * (a.mu[i] - (m + __log2f(s)) * kLn2);
        if (a.check) record_change(a.diff + prob, fabsf(f - a.lu[i]));
        a.lu[i] = f;
        tw[warp] = (f + bias_of(a.mask, b, N, ri)) * kLog2e;
      }
    } else if (lane == 0) {
      tw[warp] = -INFINITY;  // no row: contributes nothing
    }
    __syncthreads();
    // pass B: the group's rows into the column accumulators
    const int nr = min(8, r1 - g0);
    if constexpr (VEC) {
      for (int j = 4 * threadIdx.x; j < N; j += 4 * kDenseThreads) {
        float4 mm = *reinterpret_cast<float4*>(cm + j), ss = *reinterpret_cast<float4*>(cs + j);
        for (int w0 = 0; w0 < 8; w0 += 4) {
          float4 cv[4];
          float t[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int w = w0 + u;
            const int row = g0 + min(w, nr - 1);  // rows past the range re-read a valid row, weighted -inf
            cv[u] = __ldcs(reinterpret_cast<const float4*>(cprob + static_cast<size_t>(row) * N + j));
            t[u] = tw[w];
          }
          lse_push4(mm.x, ss.x, fmaf(cv[0].x, sc, t[0]), fmaf(cv[1].x, sc, t[1]), fmaf(cv[2].x, sc, t[2]),
                    fmaf(cv[3].x, sc, t[3]));
          lse_push4(mm.y, ss.y, fmaf(cv[0].y, sc, t[0]), fmaf(cv[1].y, sc, t[1]), fmaf(cv[2].y, sc, t[2]),
                    fmaf(cv[3].y, sc, t[3]));
          lse_push4(mm.z, ss.z, fmaf(cv[0].z, sc, t[0]), fmaf(cv[1].z, sc, t[1]), fmaf(cv[2].z, sc, t[2]),
                    fmaf(cv[3].z, sc, t[3]));
          lse_push4(mm.w, ss.w, fmaf(cv[0].w, sc, t[0]), fmaf(cv[1].w, sc, t[1]), fmaf(cv[2].w, sc, t[2]),
                    fmaf(cv[3].w, sc, t[3]));
        }
        *reinterpret_cast<float4*>(cm + j) = mm;
        *reinterpret_cast<float4*>(cs + j) = ss;
      }
    } else {
      for (int j = threadIdx.x; j < N; j += kDenseThreads) {
        float mm = cm[j], ss = cs[j];
        for (int w = 0; w < nr; ++w)
          lse_push1(mm, ss, fmaf(__ldcs(cprob + static_cast<size_t>(g0 + w) * N + j), sc, tw[w]));
        cm[j] = mm;
        cs[j] = ss;
      }
    }
    __syncthreads();  // tw is rewritten by the next group
  }
  float* pm = part + static_cast<size_t>(blockIdx.x) * 2 * N;
  for (int j = threadIdx.x; j < N; j += kDenseThreads) {
    pm[j] = cm[j];
    pm[N + j] = cs[j];
  }
}

// v_j = kappa (log_nu_j - LSE), the LSE merged from the problem's CTA partials
// in CTA order (deterministic)
__global__ void dense_fused_merge(const DenseArgs a, FusePlan plan, const float* part, float* lv_out) {
  const int N = a.N;
  const size_t n = static_cast<size_t>(a.B) * a.H * N;
  for (size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < n;
       o += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t prob = o / N;
    if (a.done != nullptr && a.done[prob]) continue;
    const int j = static_cast<int>(o % N);
    const float* p = part + prob * plan.S * 2 * static_cast<size_t>(N) + j;
    float m = p[0], s = p[N];
    for (int k = 1; k < plan.S; ++k)
      lse_merge(m, s, p[2 * static_cast<size_t>(k) * N], p[(2 * static_cast<size_t>(k) + 1) * N]);
    const float v = kappa_of(a.lam, a.eps[prob % a.H]) * (a.nu[o] - (m + __log2f(s)) * kLn2);
    if (a.check) record_change(a.diff + static_cast<size_t>(a.B) * a.H + prob, fabsf(v - lv_out[o]));
    lv_out[o] = v;
  }
}

unsigned grid_for(size_t work_items, size_t per_cta) {
  const size_t g = (work_items + per_cta - 1) / per_cta;
  const size_t cap = 148u * 16u;  // 16 CTAs of 256 threads per SM at most: a few waves, grid-stride beyond
  return static_cast<unsigned>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

namespace {
size_t r256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
}  // namespace

// partials of the fused iteration: 2 x N floats per CTA, at most max(BH, 148 SMs x 8 CTAs) CTAs
size_t dense_fuse_part_bytes(int B, int H, int N) {
  if (N > kFuseMaxN) return 0;
  return static_cast<size_t>(std::max(B * H, 148 * 8)) * 2 * N * sizeof(float);
}

size_t dense_fwd_workspace(int B, int H, int N) {
  // diff (2 x BH unsigned) and done (BH int); the transport's row statistics
  // (2 x BH x N floats); each region 256-byte aligned.  The one-read iteration's
  // partials follow when the caller's workspace holds them too (dense_fuse_part_bytes).
  return r256(static_cast<size_t>(3) * B * H * 4) + r256(static_cast<size_t>(2) * B * H * N * 4);
}

namespace {
// One iteration: u_i into a.lu from v_i-1 in a.lv, v_i into lv_out -- fused
// (one read of C) when part is given and N <= kFuseMaxN, else the separate
// row and column passes.
cudaError_t dense_iteration(const DenseArgs& a, float* lv_out, float* part, size_t part_bytes, bool vec,
                            cudaStream_t st) {
  const int BH = a.B * a.H;
  const size_t n = static_cast<size_t>(BH) * a.N;
  if (part != nullptr && a.N <= kFuseMaxN) {
    const size_t smem = fuse_smem(a.N);
    auto kern = vec ? dense_fused_kernel<true> : dense_fused_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    int nb = 0, dev = 0, sms = 148;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kDenseThreads, smem);
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    FusePlan plan = fuse_plan(BH, a.N, std::max(1, nb) * sms);
    while (static_cast<size_t>(BH) * plan.S * 2 * a.N * sizeof(float) > part_bytes && plan.S > 1)
      plan = fuse_plan(BH, a.N, BH * (plan.S - 1));  // fewer CTAs per problem to fit the partials
    kern<<<static_cast<unsigned>(BH) * plan.S, kDenseThreads, smem, st>>>(a, plan, part);
    dense_fused_merge<<<grid_for(n, 256), 256, 0, st>>>(a, plan, part, lv_out);
    return cudaGetLastError();
  }
  const unsigned grow = grid_for(n, kDenseThreads / 32);
  const int cols = vec ? 128 : 32;
  const unsigned gcol = static_cast<unsigned>(BH) * static_cast<unsigned>((a.N + cols - 1) / cols);
  if (vec) dense_row_kernel<true, false><<<grow, kDenseThreads, 0, st>>>(a);
  else dense_row_kernel<false, false><<<grow, kDenseThreads, 0, st>>>(a);
  DenseArgs c = a;
  c.lv = lv_out;
  if (vec) dense_col_kernel<true><<<gcol, kDenseThreads, 0, st>>>(c);
  else dense_col_kernel<false><<<gcol, kDenseThreads, 0, st>>>(c);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_dense_fwd(const FwdParams& q, void* ws, size_t ws_bytes, cudaStream_t st) {
  const int BH = q.B * q.H;
  const size_t n = static_cast<size_t>(BH) * q.N;
  unsigned* diff = static_cast<unsigned*>(ws);
  int* done = reinterpret_cast<int*>(diff + 2 * static_cast<size_t>(BH));
  float* rmax = reinterpret_cast<float*>(static_cast<char*>(ws) + r256(static_cast<size_t>(3) * BH * 4));
  float* rsum = rmax + n;
  // the one-read iterations when the workspace also holds their partials, else two passes per iteration
  const size_t base = dense_fwd_workspace(q.B, q.H, q.N);
  const size_t part_bytes = dense_fuse_part_bytes(q.B, q.H, q.N);
  float* part = part_bytes != 0 && ws_bytes >= base + part_bytes
                    ? reinterpret_cast<float*>(static_cast<char*>(ws) + base)
                    : nullptr;
  const bool vec = (q.N % 4) == 0 && (reinterpret_cast<uintptr_t>(q.C) & 15u) == 0;
  dense_init_kernel<<<grid_for(n, 256), 256, 0, st>>>(q.log_u_init, q.log_v_init, q.log_u, q.log_v, n, diff, done,
                                                       BH);
  cudaError_t e = cudaGetLastError();
  DenseArgs a{q.C, q.eps, q.log_mu, q.log_nu, q.mask, q.log_u, q.log_v, diff, q.threshold > 0.0f ? done : nullptr,
              rmax, rsum, q.B, q.H, q.N, q.lam, 0};
  const unsigned grow = grid_for(n, kDenseThreads / 32);
  for (int it = 0; it < q.K_iter && e == cudaSuccess; ++it) {
    a.check = q.threshold > 0.0f && ((it + 1) % q.check_every) == 0;
    e = dense_iteration(a, q.log_v, part, part_bytes, vec, st);
    if (a.check) dense_check_kernel<<<1, 256, 0, st>>>(diff, done, BH, q.threshold);
    if (e == cudaSuccess) e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  if (q.O != nullptr || q.T_out != nullptr || q.x_centroid != nullptr) {
    DenseArgs sa = a;
    sa.done = nullptr;  // every problem's outputs
    if (vec) dense_row_kernel<true, true><<<grow, kDenseThreads, 0, st>>>(sa);
    else dense_row_kernel<false, true><<<grow, kDenseThreads, 0, st>>>(sa);
    DenseOutArgs o{q.C, q.O != nullptr ? static_cast<const float*>(q.V) : nullptr, q.x_res, q.eps, q.mask,
                   q.log_u, q.log_v, rmax, rsum, q.O, q.T_out, q.x_centroid, q.B, q.H, q.N, q.d};
    const unsigned g = static_cast<unsigned>(BH) * static_cast<unsigned>((q.N + kOutRows - 1) / kOutRows);
    auto go = [&](auto kern, size_t smem) {
      cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e2 == cudaSuccess) {
        kern<<<g, kDenseThreads, smem, st>>>(o);
        e2 = cudaGetLastError();
      }
      return e2;
    };
    const int dpt = q.d <= 32 ? 4 : (q.d <= 64 ? 8 : 16);
    if (dpt == 4) e = vec ? go(dense_out_kernel<4, true>, dense_out_smem<4>()) : go(dense_out_kernel<4, false>, dense_out_smem<4>());
    else if (dpt == 8) e = vec ? go(dense_out_kernel<8, true>, dense_out_smem<8>()) : go(dense_out_kernel<8, false>, dense_out_smem<8>());
    else e = vec ? go(dense_out_kernel<16, true>, dense_out_smem<16>()) : go(dense_out_kernel<16, false>, dense_out_smem<16>());
    if (e != cudaSuccess) return e;
  }
  dense_finish_kernel<<<grid_for(n, 256), 256, 0, st>>>(q.mask, q.log_u, q.log_v, q.B, q.H, q.N, q.status);
  return cudaGetLastError();
}

// Iterations it_begin + 1 .. it_end of the plain loop (no early stop) on a
// history of potentials (slot 2i = log_u after iteration i, slot 2i + 1 =
// log_v), each iteration reading its inputs from the previous slots: the
// forward that the dense gradients (dfs_dense_grad.cu) reverse.
cudaError_t launch_dense_iterations(const float* C, const float* eps, const float* mu, const float* nu,
                                    const float* mask, int B, int H, int N, float lam, float* hist, int it_begin,
                                    int it_end, float* part, size_t part_bytes, cudaStream_t st) {
  const size_t n = static_cast<size_t>(B) * H * N;
  const bool vec = (N % 4) == 0 && (reinterpret_cast<uintptr_t>(C) & 15u) == 0;
  DenseArgs a{C, eps, mu, nu, mask, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, B, H, N, lam, 0};
  cudaError_t e = cudaSuccess;
  for (int it = it_begin + 1; it <= it_end && e == cudaSuccess; ++it) {
    a.lu = hist + static_cast<size_t>(2 * it) * n;      // u_it (written)
    a.lv = hist + static_cast<size_t>(2 * it - 1) * n;  // v_it-1 (read)
    e = dense_iteration(a, hist + static_cast<size_t>(2 * it + 1) * n, part, part_bytes, vec, st);  // v_it
  }
  return e;
}

}  // namespace dfs
