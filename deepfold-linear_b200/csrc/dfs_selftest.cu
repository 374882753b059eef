// dfs_selftest.cu -- checks the tcgen05.mma operand arrangement the Sinkhorn
// kernels rely on, against plain matrix products computed by the caller.  All
// operands are fp32 (read by the tensor core as tf32), staged in 128B-swizzled
// shared memory K-major, exactly as the production kernels stage them, and the
// MMA chain is issued by the same helper (issue_abt):
//
//   which 0:  D[64 x N] = A[64 x K] B[N x K]^T     (S = Q K^T, O = T_norm V, dQ = dS K, ...)
//
// (which 1 and 2 are kept for ABI stability and run the same product.)
#include "dfs_slab.cuh"

namespace dfs {

__global__ void __launch_bounds__(128, 1)
    selftest_mma_kernel(int which, const float* A, const float* B, float* D, int M, int N, int K) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t mbar;
  __shared__ uint32_t tslot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // A and B regions of 96 KB each (checked by dfs_selftest_mma)
  float* As = reinterpret_cast<float*>(base);
  float* Bs = reinterpret_cast<float*>(base + 98304);
  if (warp == 0) tmem_alloc(&tslot, 512);
  if (tid == 0) {
    mbar_init(&mbar, 1);
    fence_mbar_init();
  }
  for (int e = tid; e < M * K; e += 128) As[sw_off(e / K, e % K, M) >> 2] = A[e];
  for (int e = tid; e < N * K; e += 128) Bs[sw_off(e / K, e % K, N) >> 2] = B[e];
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tslot;
  int err = 0;
  if (tid == 0) {
    // N and K are runtime values here: dispatch to the compile-time shapes the
    // kernels use
    if (N == 32 && K == 384) issue_abt<32, 384>(tbase, As, Bs);
    else if (N == 192 && K == 32) issue_abt<192, 32>(tbase, As, Bs);
    else if (N == 256 && K == 64) issue_abt<256, 64>(tbase, As, Bs);
    else if (N == 384 && K == 32) issue_abt<384, 32>(tbase, As, Bs);
    else if (N == 64 && K == 128) issue_abt<64, 128>(tbase, As, Bs);
    else err = 2;
    mma_commit(&mbar);
  }
  if (!mbar_wait(&mbar, 0)) err = 1;
  err = __syncthreads_or(err);
  tc_fence_after();
  // M = 64: row m sits in TMEM lane (m % 16) + 32 (m / 16)
  for (int c0 = 0; c0 < N; c0 += 32) {
    float v[32];
    tmem_ld32(tbase + (static_cast<uint32_t>(32 * warp) << 16) + c0, v);
    const int row = lane < 16 ? 16 * warp + lane : -1;
    if (row >= 0 && row < M) {
      for (int c = 0; c < 32 && c0 + c < N; ++c) D[row * N + c0 + c] = err ? __int_as_float(0x7fc00000) : v[c];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

cudaError_t launch_selftest_mma(int which, const float* A, const float* B, float* D, int M, int N, int K,
                                cudaStream_t st) {
  const size_t smem = 98304 * 2 + 1024;
  cudaError_t e = cudaFuncSetAttribute(selftest_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  selftest_mma_kernel<<<1, 128, smem, st>>>(which, A, B, D, M, N, K);
  return cudaGetLastError();
}

}  // namespace dfs
