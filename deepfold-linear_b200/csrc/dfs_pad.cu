// dfs_pad.cu -- operand transforms that run a problem on the instantiated
// kernels: head dims other than 32 / 64, and fp32 operands at full precision.
//
// Padding.  The kernels are compiled for head dims 32 and 64.  A problem with
// another head dim d <= 64 runs on the next instantiated one, dk = 32 or 64,
// with the operands zero-padded along d: the padding adds exact zeros to every
// product Q K^T, dO V^T and T_norm V, so the padded problem has the same cost,
// plan and potentials, and the padded columns of O, dQ, dK, dV are dropped.
//
// fp32 split.  Tensor-core products of fp32 operands run as tf32 (10 explicit
// mantissa bits), which costs ~1e-3 relative accuracy in the logits.  For fp32
// inputs with 3 d <= 32 the library instead writes each operand as a sum of two
// bf16 parts, x = hi + lo (hi = bf16(x), lo = bf16(x - hi); 16 mantissa bits),
// and concatenates the parts along the contraction dimension:
//     Q' = [Qhi Qhi Qlo],  K' = [Khi Klo Khi],  V' = [Vhi Vlo 0],  dO' = [dO dO 0]
// so that Q' K'^T = Qhi Khi^T + Qhi Klo^T + Qlo Khi^T (every product exact,
// fp32 accumulation; only Qlo Klo^T, ~2^-16 relative, is dropped) and
// dO' V'^T = dO V^T.  The problem then runs as a bf16 problem of head dim 3d.
// Its outputs fold back: O = O'[0:d] + O'[d:2d], dQ = dQ'[0:d] + dQ'[d:2d]
// (dS Khi + dS Klo), dK = dK'[0:d] + dK'[2d:3d], dV = dV'[0:d].  The logit
// scale stays 1/sqrt(d) (FwdParams / BwdParams::qk_scale).  All copies live in
// the caller's workspace.
#include "dfs_kernels.cuh"

namespace dfs {

namespace {

unsigned grid_for(size_t n) {
  const size_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 148u * 16u ? (b > 0 ? b : 1) : 148u * 16u);
}

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

// dst (rows, dk) bf16: column block b < 3 of width d holds part parts[b] of
// src (rows, d) fp32 (0: zero, 1: hi, 2: lo); columns from 3d on are zero
__global__ void split_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, size_t rows, int d,
                             int dk, int3 parts) {
  const size_t n = rows * static_cast<size_t>(dk);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / dk;
    const int c = static_cast<int>(i - r * dk);
    const int blk = c / d;
    const int part = blk == 0 ? parts.x : blk == 1 ? parts.y : blk == 2 ? parts.z : 0;
    float v = 0.0f;
    if (part != 0) {
      const float x = src[r * d + (c - blk * d)];
      const float hi = __bfloat162float(__float2bfloat16_rn(x));
      v = part == 1 ? hi : x - hi;
    }
    dst[i] = __float2bfloat16_rn(v);
  }
}

// dst (rows, dk) fp32: `copies` copies of src (rows, d) side by side, zeros after
__global__ void dup_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t rows, int d, int dk,
                           int copies) {
  const size_t n = rows * static_cast<size_t>(dk);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / dk;
    const int c = static_cast<int>(i - r * dk);
    dst[i] = c < copies * d ? src[r * d + c % d] : 0.0f;
  }
}

// dst (rows, d) = sum over the column blocks b (width d) of src (rows, dk) whose
// bit is set in `blocks`
__global__ void fold_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t rows, int d, int dk,
                            int blocks) {
  const size_t n = rows * static_cast<size_t>(d);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / d;
    const int c = static_cast<int>(i - r * d);
    float v = 0.0f;
    for (int b = 0; b < 3; ++b)
      if ((blocks >> b) & 1) v += src[r * dk + b * d + c];
    dst[i] = v;
  }
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

cudaError_t split_rows(const float* src, void* dst, size_t rows, int d, int dk, int p0, int p1, int p2,
                       cudaStream_t st) {
  split_kernel<<<grid_for(rows * static_cast<size_t>(dk)), 256, 0, st>>>(
      src, static_cast<__nv_bfloat16*>(dst), rows, d, dk, make_int3(p0, p1, p2));
  return cudaGetLastError();
}

cudaError_t dup_rows(const float* src, float* dst, size_t rows, int d, int dk, int copies, cudaStream_t st) {
  dup_kernel<<<grid_for(rows * static_cast<size_t>(dk)), 256, 0, st>>>(src, dst, rows, d, dk, copies);
  return cudaGetLastError();
}

cudaError_t fold_rows(const float* src, float* dst, size_t rows, int d, int dk, int blocks, cudaStream_t st) {
  fold_kernel<<<grid_for(rows * static_cast<size_t>(d)), 256, 0, st>>>(src, dst, rows, d, dk, blocks);
  return cudaGetLastError();
}

}  // namespace dfs
