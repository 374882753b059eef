// dfs_pad.cu -- head dims the kernels are not instantiated for.
//
// The kernels are compiled for head dims 32 and 64.  A problem with another
// head dim d <= 64 runs on the next instantiated one, dk = 32 or 64, with the
// operands zero-padded along d: the padding adds exact zeros to every product
// Q K^T, dO V^T and T_norm V, so the padded problem has the same cost, plan and
// potentials, and the padded columns of O, dQ, dK, dV come out 0 (they are
// dropped).  The logit scale stays 1/sqrt(d) of the caller's d (FwdParams /
// BwdParams::qk_scale).  The copies live in the caller's workspace.
#include "dfs_kernels.cuh"

namespace dfs {

namespace {

template <typename T>
__global__ void pad_kernel(const T* __restrict__ src, T* __restrict__ dst, size_t rows, int d, int dk) {
  const size_t n = rows * static_cast<size_t>(dk);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / dk;
    const int c = static_cast<int>(i - r * dk);
    dst[i] = c < d ? src[r * d + c] : T(0);
  }
}

__global__ void unpad_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t rows, int d, int dk) {
  const size_t n = rows * static_cast<size_t>(d);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / d;
    const int c = static_cast<int>(i - r * d);
    dst[i] = src[r * dk + c];
  }
}

unsigned grid_for(size_t n) {
  const size_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 148u * 16u ? (b > 0 ? b : 1) : 148u * 16u);
}

}  // namespace

int kernel_head_dim(int d) { return d <= 0 ? 0 : d <= 32 ? 32 : d <= 64 ? 64 : 0; }

cudaError_t pad_rows(const void* src, void* dst, int esize, size_t rows, int d, int dk, cudaStream_t st) {
  const unsigned g = grid_for(rows * static_cast<size_t>(dk));
  if (esize == 2)
    pad_kernel<unsigned short><<<g, 256, 0, st>>>(static_cast<const unsigned short*>(src),
                                                  static_cast<unsigned short*>(dst), rows, d, dk);
  else
    pad_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(src), static_cast<float*>(dst), rows, d, dk);
  return cudaGetLastError();
}

cudaError_t unpad_rows(const float* src, float* dst, size_t rows, int d, int dk, cudaStream_t st) {
  unpad_kernel<<<grid_for(rows * static_cast<size_t>(d)), 256, 0, st>>>(src, dst, rows, d, dk);
  return cudaGetLastError();
}

}  // namespace dfs
