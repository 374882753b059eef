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
// The arithmetic follows the reference's: log K = -C / eps (an IEEE division),
// masks as additive -1e9 biases, kappa = lam / (lam + eps) (1 for lam = inf),
// T = exp(score - rowmax), T_norm = T / (sum T + 1e-6), padded rows of T_norm
// and padded potentials zeroed.
//
// Early stopping (threshold > 0): on every check_every-th iteration the passes
// record each problem's largest |change| of log_u and log_v; a one-CTA kernel
// then marks the problems whose change is below the threshold done, and the
// later passes skip them -- each (batch, head) problem stops on its own, as on
// the resident path.
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
  int B, H, N;
  float lam;
  int check;            // this pass records |change|
};

__device__ __forceinline__ float kappa_of(float lam, float eps) { return isinf(lam) ? 1.0f : lam / (lam + eps); }

__device__ __forceinline__ float bias_of(const float* mask, int b, int N, int j) {
  return mask == nullptr ? 0.0f : (1.0f - mask[static_cast<size_t>(b) * N + j]) * kMaskBias;
}

// online log-sum-exp state: running max m and sum s of exp(x - m)
__device__ __forceinline__ void lse_push(float& m, float& s, float x) {
  if (x > m) {
    s = s * expf(m - x) + 1.0f;  // m = -inf first: exp(-inf) = 0
    m = x;
  } else if (x > -INFINITY) {  // (-inf, -inf): nothing to add
    s += expf(x - m);
  }
}
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * expf(m - m2) + s2;
    m = m2;
  } else if (m2 > -INFINITY) {
    s += s2 * expf(m2 - m);
  }
}

__device__ __forceinline__ void record_change(unsigned* slot, float a) {
  // non-negative floats order like their bit patterns (NaN ends above every number)
  atomicMax(slot, __float_as_uint(a));
}

// f_i = kappa (log_mu_i - LSE_j(-C_ij / eps + g_j + colbias_j)), one warp per row
template <bool VEC>
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
    const float* c = a.C + r * N;
    const float* g = a.lv + prob * N;
    float m = -INFINITY, s = 0.0f;
    if constexpr (VEC) {
      for (int j = 4 * lane; j < N; j += 128) {
        const float4 cv = __ldcs(reinterpret_cast<const float4*>(c + j));
        const float4 gv = *reinterpret_cast<const float4*>(g + j);
        lse_push(m, s, -cv.x / eps + gv.x + bias_of(a.mask, b, N, j));
        lse_push(m, s, -cv.y / eps + gv.y + bias_of(a.mask, b, N, j + 1));
        lse_push(m, s, -cv.z / eps + gv.z + bias_of(a.mask, b, N, j + 2));
        lse_push(m, s, -cv.w / eps + gv.w + bias_of(a.mask, b, N, j + 3));
      }
    } else {
      for (int j = lane; j < N; j += 32) lse_push(m, s, -__ldcs(c + j) / eps + g[j] + bias_of(a.mask, b, N, j));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      lse_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const size_t i = r;
      const float f = kappa_of(a.lam, eps) * (a.mu[i] - (m + logf(s)));
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
  const float* f = a.lu + prob * N;
  float m[PER], s[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    m[q] = -INFINITY;
    s[q] = 0.0f;
  }
  const int j = j0 + PER * lane;
  for (int i = warp; i < N; i += 8) {
    const float* c = a.C + (prob * N + i) * N;
    const float fi = f[i] + bias_of(a.mask, b, N, i);
    if constexpr (VEC) {
      if (j < N) {
        const float4 cv = __ldcs(reinterpret_cast<const float4*>(c + j));
        lse_push(m[0], s[0], -cv.x / eps + fi);
        lse_push(m[1], s[1], -cv.y / eps + fi);
        lse_push(m[2], s[2], -cv.z / eps + fi);
        lse_push(m[3], s[3], -cv.w / eps + fi);
      }
    } else {
      if (j < N) lse_push(m[0], s[0], -__ldcs(c + j) / eps + fi);
    }
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
    const float g = kappa_of(a.lam, eps) * (a.nu[o] - (mm + logf(sv)));
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

// compute_transport_output (sinkhorn.py:152-195) on a dense cost: one warp per
// row, 8 rows per CTA.  score_ij = log_u_i + (-C_ij / eps) + log_v_j + colbias_j;
// pass 1: the row's max m and sum s of exp(score - m); pass 2 per tile of 32
// columns: T_norm_ij = exp(score_ij - m) / (s + 1e-6) (0 on a padded row),
// written when asked for, O_i += T_norm_ij V_j (the tile of V staged in shared
// memory once per CTA, lane k accumulating dims k, k + 32, ...), centroid
// sum_j T_norm_ij x_j.  DV = ceil(d / 32) accumulators per lane.
struct DenseOutArgs {
  const float* C;
  const float* V;     // (B,H,N,d) fp32 or null
  const float* x;     // (B,N,3) or null
  const float* eps;
  const float* mask;
  const float* lu;
  const float* lv;
  float* O;           // (B,H,N,d)
  float* T;           // (B,H,N,N) or null
  float* xc;          // (B,H,N,3) or null
  int B, H, N, d;
};

template <int DV>
__global__ void __launch_bounds__(kDenseThreads) dense_out_kernel(const DenseOutArgs a) {
  extern __shared__ float vt[];  // [32][d] tile of V
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = a.N, d = a.d;
  const int rblocks = (N + 7) / 8;
  const size_t prob = blockIdx.x / rblocks;
  const int i = (blockIdx.x % rblocks) * 8 + warp;
  const int b = static_cast<int>(prob / a.H), h = static_cast<int>(prob % a.H);
  const bool row_ok = i < N;  // rows past N still help stage V
  const float eps = a.eps[h];
  const size_t r = prob * N + (row_ok ? i : 0);
  const float* c = a.C + r * N;
  const float* g = a.lv + prob * N;
  const float ui = row_ok ? a.lu[r] : 0.0f;
  float m = -INFINITY, s = 0.0f;
  if (row_ok)
    for (int j = lane; j < N; j += 32) lse_push(m, s, ui + (-c[j] / eps) + g[j] + bias_of(a.mask, b, N, j));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  const float rmask = (a.mask == nullptr || !row_ok) ? 1.0f : a.mask[static_cast<size_t>(b) * N + i];
  float acc[DV];
#pragma unroll
  for (int q = 0; q < DV; ++q) acc[q] = 0.0f;
  float cx = 0.0f, cy = 0.0f, cz = 0.0f;
  const float* xb = a.x != nullptr ? a.x + static_cast<size_t>(b) * N * 3 : nullptr;
  for (int j0 = 0; j0 < N; j0 += 32) {
    const int j = j0 + lane;
    float t = 0.0f;
    if (row_ok && j < N) {
      // the reference's T / (sum + 1e-6), then the padded-row factor
      t = expf(ui + (-c[j] / eps) + g[j] + bias_of(a.mask, b, N, j) - m) / (s + 1e-6f) * rmask;
      if (a.T != nullptr) __stcs(a.T + r * N + j, t);
      if (xb != nullptr) {
        cx += t * xb[3 * j];
        cy += t * xb[3 * j + 1];
        cz += t * xb[3 * j + 2];
      }
    }
    if (a.V != nullptr) {
      __syncthreads();
      const float* vsrc = a.V + (prob * N + j0) * d;
      const int rows = min(32, N - j0);
      for (int e = threadIdx.x; e < 32 * d; e += kDenseThreads) vt[e] = e < rows * d ? vsrc[e] : 0.0f;
      __syncthreads();
#pragma unroll 4
      for (int cc = 0; cc < 32; ++cc) {
        const float tc = __shfl_sync(0xffffffffu, t, cc);
#pragma unroll
        for (int q = 0; q < DV; ++q) {
          const int k = lane + 32 * q;
          if (k < d) acc[q] = fmaf(tc, vt[cc * d + k], acc[q]);
        }
      }
    }
  }
  if (!row_ok) return;
  if (a.O != nullptr)
#pragma unroll
    for (int q = 0; q < DV; ++q) {
      const int k = lane + 32 * q;
      if (k < d) a.O[r * d + k] = acc[q];
    }
  if (a.xc != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      cx += __shfl_xor_sync(0xffffffffu, cx, o);
      cy += __shfl_xor_sync(0xffffffffu, cy, o);
      cz += __shfl_xor_sync(0xffffffffu, cz, o);
    }
    if (lane == 0) {
      a.xc[r * 3] = cx;
      a.xc[r * 3 + 1] = cy;
      a.xc[r * 3 + 2] = cz;
    }
  }
}

unsigned grid_for(size_t work_items, size_t per_cta) {
  const size_t g = (work_items + per_cta - 1) / per_cta;
  const size_t cap = 148u * 16u;  // 16 CTAs of 256 threads per SM at most: a few waves, grid-stride beyond
  return static_cast<unsigned>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

size_t dense_fwd_workspace(int B, int H) {
  // diff (2 x BH unsigned) and done (BH int), 256-byte rounded
  return (static_cast<size_t>(3) * B * H * 4 + 255) & ~static_cast<size_t>(255);
}

cudaError_t launch_dense_fwd(const FwdParams& q, void* ws, cudaStream_t st) {
  const int BH = q.B * q.H;
  const size_t n = static_cast<size_t>(BH) * q.N;
  unsigned* diff = static_cast<unsigned*>(ws);
  int* done = reinterpret_cast<int*>(diff + 2 * static_cast<size_t>(BH));
  const bool vec = (q.N % 4) == 0 && (reinterpret_cast<uintptr_t>(q.C) & 15u) == 0;
  dense_init_kernel<<<grid_for(n, 256), 256, 0, st>>>(q.log_u_init, q.log_v_init, q.log_u, q.log_v, n, diff, done,
                                                       BH);
  cudaError_t e = cudaGetLastError();
  DenseArgs a{q.C, q.eps, q.log_mu, q.log_nu, q.mask, q.log_u, q.log_v, diff, q.threshold > 0.0f ? done : nullptr,
              q.B, q.H, q.N, q.lam, 0};
  const unsigned grow = grid_for(n, kDenseThreads / 32);
  const int cols = vec ? 128 : 32;
  const unsigned gcol = static_cast<unsigned>(BH) * static_cast<unsigned>((q.N + cols - 1) / cols);
  for (int it = 0; it < q.K_iter && e == cudaSuccess; ++it) {
    a.check = q.threshold > 0.0f && ((it + 1) % q.check_every) == 0;
    if (vec) dense_row_kernel<true><<<grow, kDenseThreads, 0, st>>>(a);
    else dense_row_kernel<false><<<grow, kDenseThreads, 0, st>>>(a);
    if (vec) dense_col_kernel<true><<<gcol, kDenseThreads, 0, st>>>(a);
    else dense_col_kernel<false><<<gcol, kDenseThreads, 0, st>>>(a);
    if (a.check) dense_check_kernel<<<1, 256, 0, st>>>(diff, done, BH, q.threshold);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  if (q.O != nullptr || q.T_out != nullptr || q.x_centroid != nullptr) {
    DenseOutArgs o{q.C, q.O != nullptr ? static_cast<const float*>(q.V) : nullptr, q.x_res, q.eps, q.mask,
                   q.log_u, q.log_v, q.O, q.T_out, q.x_centroid, q.B, q.H, q.N, q.d};
    const unsigned g = static_cast<unsigned>(BH) * static_cast<unsigned>((q.N + 7) / 8);
    const size_t smem = static_cast<size_t>(32) * q.d * sizeof(float);
    const int dv = (q.d + 31) / 32;
    if (dv <= 1) dense_out_kernel<1><<<g, kDenseThreads, smem, st>>>(o);
    else if (dv == 2) dense_out_kernel<2><<<g, kDenseThreads, smem, st>>>(o);
    else dense_out_kernel<4><<<g, kDenseThreads, smem, st>>>(o);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  dense_finish_kernel<<<grid_for(n, 256), 256, 0, st>>>(q.mask, q.log_u, q.log_v, q.B, q.H, q.N, q.status);
  return cudaGetLastError();
}

}  // namespace dfs
