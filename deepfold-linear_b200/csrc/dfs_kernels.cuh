// dfs_kernels.cuh -- parameter blocks and launchers shared by the C ABI layer and
// the kernels of libdfsink.
#pragma once

#include "dfs_device.cuh"

namespace dfs {

// Resident kernels: 16 warps per CTA, each warp owning 4 rows of the 64-row slab.
constexpr int kThreads = 512;
constexpr int kWarps = 16;
constexpr int kRpw = 4;
// Independent TMEM accumulators for the narrow (d-column) MMAs with K = N.
constexpr int kGradAcc = 1;

// Potential drift (log2 units) since the last absorption beyond which the
// stabilised kernel matrix is rebuilt: row/column sums then stay above 2^-60.
constexpr float kDrift = 30.0f;

DFS_DEV float load_f32(const void* p, size_t i, int dtype) {
  if (dtype == DFS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == DFS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

struct FwdParams {
  const void* Q;
  const void* K;
  const void* V;
  const float* C;
  const float* x_res;
  const float* pos_weight;
  const int32_t* pos_bins;
  const float* eps;
  const float* w_dist;
  const float* log_mu;
  const float* log_nu;
  const float* log_u_init;
  const float* log_v_init;
  const float* mask;
  float* O;
  float* x_centroid;
  float* log_u;
  float* log_v;
  int32_t* status;
  float* T_out;
  int B, H, N, d, in_dtype, cost_mode, K_iter, check_every;
  float lam, r_0, threshold;
};

struct BwdParams {
  const void* Q;
  const void* K;
  const void* V;
  const float* x_res;
  const float* pos_weight;
  const int32_t* pos_bins;
  const float* eps;
  const float* w_dist;
  const float* log_mu;
  const float* log_nu;
  const float* mask;
  const float* log_u;
  const float* log_v;
  const float* dO;
  const float* dxc;
  float* dQ;
  float* dK;
  float* dV;
  float* dlog_mu;
  float* dlog_nu;
  float* dx_res;
  float* dpos_weight;
  float* dw_dist;
  int32_t* cg_iters;
  float* cg_residual;
  int32_t* status;
  float* ws;               // workspace: per-CTA partials of the shared-parameter grads
  int B, H, N, d, in_dtype, cg_max_iter;
  float lam, r_0, cg_rtol, cg_atol;
};

cudaError_t launch_resident_fwd(const FwdParams& p, cudaStream_t st);
size_t resident_fwd_smem(int N, int d);
cudaError_t launch_stream_fwd(const FwdParams& p, float* ws, cudaStream_t st);
cudaError_t stream_fwd_op(int op, const FwdParams& p, float* ws, int r0, int r1, cudaStream_t st);
cudaError_t stream_bwd_op(int op, const BwdParams& p, float* ws, int r0, int r1, cudaStream_t st);
size_t stream_fwd_workspace(int B, int H, int N);
cudaError_t launch_resident_bwd(const BwdParams& p, cudaStream_t st);
cudaError_t launch_stream_bwd(const BwdParams& p, float* ws, cudaStream_t st);
size_t stream_bwd_workspace(int B, int H, int N);
size_t resident_bwd_smem(int N, int d);
size_t resident_bwd_workspace(int B, int H, int N, int d);
cudaError_t launch_selftest_mma(int which, const float* A, const float* B, float* D, int M, int N, int K,
                                cudaStream_t st);

}  // namespace dfs
