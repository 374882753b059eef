// dfs_stream.cu -- streamed flash-Sinkhorn kernels for sm_100a (any N, d = 32 or 64).
//
// Problems too large for the cluster-resident kernels recompute the log-kernel
// tile by tile instead of keeping it on chip (the flash-attention pattern, as the
// reference's Triton kernels do, src/deepfold/model/kernels/sinkhorn_kernel.py:
// 59-129 and 1107-1493).  One CTA owns a block of 128 rows of one (batch, head)
// problem; its 128 threads own one row each (= TMEM lane, so every per-row
// reduction is thread-local) and stream the columns in tiles of 128:
//
//   S tile = A_blk B_tile^T       tcgen05.mma kind::tf32, M=128 N=128 K=d, fp32 in TMEM
//   epilogue (per row, per tile)  x = S log2(e)/(eps sqrt d) + column bias (+ row bias)
//
// with the next tile's operand load and MMA overlapping the current epilogue
// (two TMEM accumulators, two shared-memory operand buffers).  The half-update
// of Sinkhorn is a row log-sum-exp, and the column half-update is the same
// kernel with the operands' roles swapped (A = K, B = Q, bias = f), so both
// halves, and a row-sharded multi-GPU run, use one kernel:
//
//   SM_LSE       f_i = kappa (a_i - LSE_j(x_ij)),   x = S' + g_j      (log2 units)
//   SM_ROWSTATS  m_i = max_j x_ij, R_i = sum_j exp2(x_ij - m_i),  x = S' + f_i + g_j
//   SM_OUT       T_norm = exp2(x - m_i) / (R_i + 1e-6); O = T_norm V (second MMA,
//                K = the tile's columns), x_centroid = T_norm x
//
// T_norm and its 1e-6 follow compute_transport_output (src/deepfold/model/
// sinkhorn.py:152-195).
#include "dfs_slab.cuh"

namespace dfs {

constexpr int kSThreads = 128;  // one thread per row of a block
constexpr int kSTile = 128;     // columns per streamed tile

enum StreamMode { SM_LSE = 0, SM_ROWSTATS = 1, SM_OUT = 2 };

struct StreamParams {
  const void* Aop;        // (BH, N, d): rows of S = A B^T
  const void* Bop;        // (BH, N, d): columns
  const void* Vop;        // SM_OUT: (BH, N, d) values
  int dtype;
  const float* eps;       // (H,)
  const float* mask;      // (B, N) 1 = real point, or null
  const float* col_bias;  // (BH, N) potential of the columns, log2 units
  const float* row_bias;  // (BH, N) potential of the rows, log2 units (ROWSTATS, OUT)
  const float* row_marg;  // (BH, N) natural-log marginal of the rows (LSE)
  float* row_out;         // LSE: new row potential, log2 units; ROWSTATS: m
  float* row_out_nat;     // LSE: the same potential in natural-log units, or null
  float* row_R;           // ROWSTATS: out; OUT: in
  const float* row_m;     // OUT: m
  float* O;               // OUT: (BH, N, d) fp32
  const float* x_res;     // OUT: (B, N, 3) or null
  float* x_centroid;      // OUT: (BH, N, 3) or null
  int B, H, N;
  int row_begin, row_end; // rows this launch handles ([0, N) unless sharded)
  float lam;
  float qk_scale;         // 1/sqrt(d) of the cost
};

template <int MODE, int D>
struct StreamCfg {
  static constexpr bool kOut = MODE == SM_OUT;
  static constexpr int NBUF = kOut ? 1 : 2;  // operand / accumulator buffers
  static constexpr uint32_t OFF_A = 0;                                   // 128 x D
  static constexpr uint32_t OFF_B = OFF_A + 4u * 128 * D;               // NBUF x 128 x D
  static constexpr uint32_t OFF_T = OFF_B + 4u * NBUF * 128 * D;        // OUT: 128 x 128
  static constexpr uint32_t OFF_VT = OFF_T + (kOut ? 4u * 128 * 128 : 0u);  // OUT: D x 128
  static constexpr uint32_t OFF_CB = OFF_VT + (kOut ? 4u * D * 128 : 0u);   // 3 x 128 column bias
  static constexpr uint32_t OFF_XC = OFF_CB + 4u * 3 * 128;            // OUT: 3 x 128 coordinates
  static constexpr uint32_t OFF_BAR = OFF_XC + 4u * 3 * 128;           // 2 mbarriers, TMEM slot
  static constexpr uint32_t SMEM_NEED = OFF_BAR + 64 + 1024;           // + alignment slack
  // at least 80 KB: at most two CTAs per SM, whose 2 x 256 TMEM columns always fit
  static constexpr uint32_t SMEM = SMEM_NEED > 81920u ? SMEM_NEED : 81920u;
  static_assert(SMEM <= 232448u, "shared memory");
};

constexpr float kNegBig = -1.0e30f;  // finite "minus infinity" for running maxima

template <int MODE, int D>
__global__ void __launch_bounds__(kSThreads) stream_kernel(const StreamParams p) {
  using Cfg = StreamCfg<MODE, D>;
  constexpr bool kOut = Cfg::kOut;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* As = reinterpret_cast<float*>(base + Cfg::OFF_A);
  float* Bs = reinterpret_cast<float*>(base + Cfg::OFF_B);
  float* Ts = reinterpret_cast<float*>(base + Cfg::OFF_T);
  float* Vt = reinterpret_cast<float*>(base + Cfg::OFF_VT);
  float* cb = reinterpret_cast<float*>(base + Cfg::OFF_CB);
  float* xc = reinterpret_cast<float*>(base + Cfg::OFF_XC);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(base + Cfg::OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + Cfg::OFF_BAR + 16);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  const int prob = blockIdx.x / nrb, rb = blockIdx.x % nrb;
  const int bb = prob / p.H, hh = prob % p.H;
  const int N = p.N;
  const size_t bh = static_cast<size_t>(prob);
  const int r0 = p.row_begin + 128 * rb, row = r0 + tid;
  const float eps_h = p.eps[hh];
  const float scale = kLog2e * p.qk_scale / eps_h;
  const float kap = isinf(p.lam) ? 1.0f : p.lam / (p.lam + eps_h);
  const bool rin = row < p.row_end && row < N;
  const bool rok = rin && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + row] != 0.0f);
  int err = 0;
  // Only the column tiles that hold a valid point are visited: a masked column
  // contributes exactly nothing (its bias is -inf), so the others are skipped,
  // and a block with no valid row visits none (its rows' results are the
  // masked-row values).
  int vlo, vhi;
  valid_extent<kSThreads>(p.mask, bb, N, reinterpret_cast<int*>(base + Cfg::OFF_BAR + 32), vlo, vhi);
  const int rhi = min(min(r0 + 128, p.row_end), N);
  const bool live = max(r0, vlo) < min(rhi, vhi);
  const int t_begin = live ? vlo / kSTile : 0;
  const int ntiles = live ? (vhi + kSTile - 1) / kSTile - t_begin : 0;

  if (warp == 0) tmem_alloc(tslot, 256);
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
  }
  load_tile_any<D, 128, false, kSThreads>(As, p.Aop, p.dtype, bh * N, r0, N, tid);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tlane = static_cast<uint32_t>(32 * warp) << 16;

  const float fi = (MODE == SM_LSE || !rin) ? 0.0f : p.row_bias[bh * N + row];
  float m = kNegBig, s = 0.0f;  // running max and sum (LSE, ROWSTATS)
  float mi = 0.0f, inv = 0.0f;  // OUT
  if constexpr (kOut) {
    if (rin) {
      mi = p.row_m[bh * N + row];
      inv = 1.0f / (p.row_R[bh * N + row] + 1e-6f);
    }
  }
  float cx = 0.0f, cy = 0.0f, cz = 0.0f;  // centroid accumulators

  // operands of tile t into buffer b; column bias into slot t % 3 (read by the
  // epilogue of tile t, two barriers after the last read of that slot)
  auto stage = [&](int t, int b) {
    const int c0 = t * kSTile;
    load_tile_any<D, 128, false, kSThreads>(Bs + b * 128 * D, p.Bop, p.dtype, bh * N, c0, N, tid);
    const int j = c0 + tid;
    const bool cok = j < N && (p.mask == nullptr || p.mask[static_cast<size_t>(bb) * N + j] != 0.0f);
    cb[(t % 3) * 128 + tid] = cok ? p.col_bias[bh * N + j] : -INFINITY;
    if constexpr (kOut) {
      load_tile_any<D, 128, true, kSThreads>(Vt, p.Vop, p.dtype, bh * N, c0, N, tid);  // V^T (D x 128)
      if (p.x_centroid != nullptr) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
          xc[c * 128 + tid] = j < N ? p.x_res[(static_cast<size_t>(bb) * N + j) * 3 + c] : 0.0f;
      }
    }
  };
  auto issue_s = [&](int b) {
    if (tid == 0) {
      issue_mma<128, kSTile, D>(tbase + b * kSTile, As, Bs + b * 128 * D, false);
      mma_commit(&mbar[b]);
    }
  };
  uint32_t ph0 = 0, ph1 = 0;
  auto wait_bar = [&](int b) {
    const uint32_t par = b == 0 ? ph0 : ph1;
    if (!mbar_wait(&mbar[b], par)) err |= DFS_ERR_DEVICE_TIMEOUT;
    if (b == 0) ph0 ^= 1u; else ph1 ^= 1u;
    tc_fence_after();
  };

  // per-row epilogue of one tile: 4 chunks of 32 columns from TMEM
  auto epilogue = [&](int t, int b) {
    const float* cbt = cb + (t % 3) * 128;
#pragma unroll 1
    for (int ch = 0; ch < kSTile / 32; ++ch) {
      float v[32];
      tmem_ld32(tbase + tlane + b * kSTile + 32 * ch, v);
      if constexpr (MODE == SM_LSE || MODE == SM_ROWSTATS) {
        float cm = kNegBig;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          v[k] = fmaf(v[k], scale, cbt[32 * ch + k] + fi);
          cm = fmaxf(cm, v[k]);
        }
        const float mn = fmaxf(m, cm);
        float acc = s * ex2(m - mn);
#pragma unroll
        for (int k = 0; k < 32; ++k) acc += ex2(v[k] - mn);
        m = mn;
        s = acc;
      } else {
        float tv[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float x = fmaf(v[k], scale, cbt[32 * ch + k] + fi);
          tv[k] = rok ? ex2(x - mi) * inv : 0.0f;
        }
        if (p.x_centroid != nullptr) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            cx = fmaf(tv[k], xc[32 * ch + k], cx);
            cy = fmaf(tv[k], xc[128 + 32 * ch + k], cy);
            cz = fmaf(tv[k], xc[256 + 32 * ch + k], cz);
          }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(Ts + (sw_off(tid, 32 * ch + 4 * q, 128) >> 2)) =
              make_float4(tv[4 * q], tv[4 * q + 1], tv[4 * q + 2], tv[4 * q + 3]);
      }
    }
  };

  if constexpr (!kOut) {
    if (ntiles > 0) {
      stage(t_begin, 0);
      fence_async_smem();
      __syncthreads();
      issue_s(0);
    }
#pragma unroll 1
    for (int u = 0; u < ntiles; ++u) {
      const int t = t_begin + u, b = u & 1;
      if (u + 1 < ntiles) stage(t + 1, b ^ 1);  // buffer b^1: its MMA (tile t-1) completed
      fence_async_smem();
      wait_bar(b);
      tc_fence_before();
      __syncthreads();  // tile t+1 staged by all; epilogue t-1 (TMEM b^1) finished by all
      tc_fence_after();
      if (u + 1 < ntiles) issue_s(b ^ 1);
      epilogue(t, b);
    }
  } else {
    // one buffer: S tile -> T_norm tile (shared memory) -> O += T_norm V
#pragma unroll 1
    for (int u = 0; u < ntiles; ++u) {
      const int t = t_begin + u;
      if (u > 0) wait_bar(1);  // O MMA of tile t-1 done: T and V^T buffers free
      stage(t, 0);
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      issue_s(0);
      wait_bar(0);
      epilogue(t, 0);
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (tid == 0) {
        issue_mma<128, D, kSTile>(tbase + kSTile, Ts, Vt, u > 0);
        mma_commit(&mbar[1]);
      }
    }
    if (ntiles > 0) wait_bar(1);  // (no tile: every row is masked, O is written as 0)
  }

  // ---------------------------------------------------------------- results
  if constexpr (MODE == SM_LSE) {
    if (rin) {
      float f = 0.0f;
      if (rok && s > 0.0f) f = kap * (p.row_marg[bh * N + row] * kLog2e - (m + lg2(s)));
      p.row_out[bh * N + row] = f;
      if (p.row_out_nat) p.row_out_nat[bh * N + row] = f * kLn2;
    }
  } else if constexpr (MODE == SM_ROWSTATS) {
    if (rin) {
      p.row_out[bh * N + row] = rok ? m : 0.0f;
      p.row_R[bh * N + row] = rok ? s : 0.0f;
    }
  } else {
#pragma unroll
    for (int g = 0; g < D / 16; ++g) {
      float v[16];
      tmem_ld16(tbase + tlane + kSTile + 16 * g, v);
      if (rin) {
        float4* dst = reinterpret_cast<float4*>(p.O + (bh * N + row) * D + 16 * g);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = rok ? make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3])
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (p.x_centroid != nullptr && rin) {
      float* xo = p.x_centroid + (bh * N + row) * 3;
      xo[0] = rok ? cx : 0.0f;
      xo[1] = rok ? cy : 0.0f;
      xo[2] = rok ? cz : 0.0f;
    }
  }
  (void)err;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// initial potentials from an optional natural-log warm start: log2 units into
// the workspace, natural units into the output (so K_iter = 0 returns them)
__global__ void stream_init_kernel(float* out2, float* out_nat, const float* init, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = init ? init[i] : 0.0f;
  out2[i] = v * kLog2e;
  out_nat[i] = v;
}

template <int MODE, int D>
static cudaError_t launch_stream_md(const StreamParams& p, cudaStream_t st) {
  using Cfg = StreamCfg<MODE, D>;
  auto kern = stream_kernel<MODE, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  if (e != cudaSuccess) return e;
  const int nrb = (p.row_end - p.row_begin + 127) / 128;
  kern<<<p.B * p.H * nrb, kSThreads, Cfg::SMEM, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_stream(int mode, int d, const StreamParams& p, cudaStream_t st) {
  if (p.row_end <= p.row_begin) return cudaSuccess;
  if (d == 32) {
    if (mode == SM_LSE) return launch_stream_md<SM_LSE, 32>(p, st);
    if (mode == SM_ROWSTATS) return launch_stream_md<SM_ROWSTATS, 32>(p, st);
    return launch_stream_md<SM_OUT, 32>(p, st);
  }
  if (d == 64) {
    if (mode == SM_LSE) return launch_stream_md<SM_LSE, 64>(p, st);
    if (mode == SM_ROWSTATS) return launch_stream_md<SM_ROWSTATS, 64>(p, st);
    return launch_stream_md<SM_OUT, 64>(p, st);
  }
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- cost-term tables
int cost_bin_stride(int N) { return (N + 127) / 128 * 128; }
size_t cost_bins_bytes(int B, int N) { return static_cast<size_t>(B) * N * cost_bin_stride(N); }

// position bins (a (B, N, N) int32 table, or compute_bins' inputs evaluated
// per pair) -> table (B, N, stride) uint8 and its transpose (entry [b][j][i] =
// bins[b][i][j]); bins outside [0, 68) and the padding columns hold 68, whose
// weight the passes take as 0.  32 x 32 tiles through shared memory, one block
// per tile of the (stride x stride) square.
__global__ void cost_bins_kernel(const BinSource src, int N, int stride, uint8_t* __restrict__ t,
                                 uint8_t* __restrict__ tt) {
  __shared__ uint8_t tile[32][33];
  const size_t b = blockIdx.z;
  const int i0 = blockIdx.y * 32, j0 = blockIdx.x * 32, tx = threadIdx.x;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int i = i0 + r, j = j0 + tx;
    uint8_t v = kBinCount;
    if (i < N && j < N) {
      const unsigned x = static_cast<unsigned>(bin_at(src, b, N, i, j));
      v = x < static_cast<unsigned>(kBinCount) ? static_cast<uint8_t>(x) : static_cast<uint8_t>(kBinCount);
    }
    if (i < N && j < stride) t[(b * N + i) * stride + j] = v;
    tile[r][tx] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int j = j0 + r, i = i0 + tx;
    if (j < N && i < stride) tt[(b * N + j) * stride + i] = tile[tx][r];
  }
}

cudaError_t build_cost_bins(const BinSource& src, int B, int N, uint8_t* bins, uint8_t* bins_t, cudaStream_t st) {
  const int stride = cost_bin_stride(N);
  cost_bins_kernel<<<dim3(stride / 32, stride / 32, B), dim3(32, 8), 0, st>>>(src, N, stride, bins, bins_t);
  return cudaGetLastError();
}

// compute_bins (position_encoding.py:7-52) into an int32 table: one thread per
// pair, rows of a block's 256 consecutive pairs of one batch element
__global__ void compute_bins_kernel(const BinSource src, int B, int N, int32_t* __restrict__ out) {
  const size_t nn = static_cast<size_t>(N) * N, total = nn * B;
  for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < total;
       k += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t b = k / nn, r = k - b * nn;
    const int i = static_cast<int>(r / N), j = static_cast<int>(r - static_cast<size_t>(i) * N);
    out[k] = bin_at(src, b, N, i, j);
  }
}

cudaError_t compute_bins_table(const int32_t* chain, const int32_t* gidx, const uint8_t* bond, int B, int N,
                               int32_t* out, cudaStream_t st) {
  const size_t total = static_cast<size_t>(B) * N * N;
  if (total == 0) return cudaSuccess;
  const size_t blocks = (total + 255) / 256;
  const unsigned g = static_cast<unsigned>(blocks < 148u * 32u ? blocks : 148u * 32u);
  compute_bins_kernel<<<g, 256, 0, st>>>(BinSource{nullptr, chain, gidx, bond}, B, N, out);
  return cudaGetLastError();
}

namespace {
float* align256(float* p) {
  return reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
}
size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
}  // namespace

// f, g (log2), m, R; then fp32 copies Q, K (row-major) and V^T (transposed)
// for the TMA-staged transport-output pass
// ... then the column-split scratch, a 64-byte slot whose first 8 bytes are
// the peer-exchange arrival counter, the mask's valid extent per batch element,
// and, with the position term, the uint8 bin table and its transpose
size_t stream_fwd_workspace(int B, int H, int N, int d, int terms) {
  const size_t n = static_cast<size_t>(B) * H * N;
  size_t bytes = 4 * sizeof(float) * n + 256 + 3 * sizeof(float) * n * d + 256 + tile_split_bytes(B, H, N) + 128 +
                 sizeof(int2) * static_cast<size_t>(B);
  if (terms & DFS_TERM_POS) bytes += 256 + 2 * round256(cost_bins_bytes(B, N));
  return bytes;
}

// The cost terms of a pass from the forward / backward inputs: `transposed` for
// the passes on S^T (their rows are the cost's columns).
CostTerms cost_terms_of(const float* pos_weight, const float* x_res, const float* w_dist, float r_0,
                        const float* r_head, int N, const uint8_t* bins, const uint8_t* bins_t, bool transposed) {
  CostTerms c{};
  if (pos_weight != nullptr && bins != nullptr) {
    c.bins = transposed ? bins_t : bins;
    c.bin_stride = cost_bin_stride(N);
    c.pos_weight = pos_weight;
  }
  if (x_res != nullptr && w_dist != nullptr) {
    c.x = x_res;
    c.w_dist = w_dist;
  }
  c.r_0 = r_0;
  c.r_head = r_head;
  return c;
}

// One phase of the streamed forward on rows [r0, r1) (the whole problem for a
// single GPU; a row range per GPU when the rows are sharded, with the
// potentials all-gathered between phases).  Workspace slots, (BH, N) fp32 each:
// f, g (log2 units), m, R.
//   FWD_INIT  f, g (and log_u, log_v) from the warm starts, all positions
//   FWD_ROWS  f = kappa (a - LSE_j(S' + g)) for rows [r0, r1); also log_u there
//   FWD_COLS  g = kappa (b - LSE_i(S' + f)) for columns [r0, r1); also log_v there
//   FWD_OUT   row statistics, O and x_centroid for rows [r0, r1)
cudaError_t stream_fwd_op(int op, const FwdParams& fp, float* ws, int r0, int r1, cudaStream_t st,
                          const PeerInfo* peers) {
  const size_t n = static_cast<size_t>(fp.B) * fp.H * fp.N;
  float* fw = ws;
  float* gw = ws + n;
  float* mw = ws + 2 * n;
  float* Rw = ws + 3 * n;
  float* copies = align256(ws + 4 * n);                            // Q, K, V^T fp32
  float* split = align256(copies + 3 * n * static_cast<size_t>(fp.d));  // column-split scratch
  unsigned long long* counter = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(split) + tile_split_bytes(fp.B, fp.H, fp.N) + 63) & ~uintptr_t(63));
  // the same byte offset in another GPU's workspace
  auto at_peer = [&](int k, const void* own) {
    return static_cast<char*>(peers->ws[k]) + (static_cast<const char*>(own) - reinterpret_cast<char*>(ws));
  };
  int2* extents = reinterpret_cast<int2*>(reinterpret_cast<char*>(counter) + 64);
  uint8_t* bins = nullptr;  // position-bin tables (row orientation, transposed)
  uint8_t* bins_t = nullptr;
  if (fp.cost_terms & DFS_TERM_POS) {
    bins = reinterpret_cast<uint8_t*>(align256(reinterpret_cast<float*>(extents + fp.B)));
    bins_t = bins + round256(cost_bins_bytes(fp.B, fp.N));
  }
  auto terms = [&](bool transposed) {
    return cost_terms_of(fp.pos_weight, fp.x_res, fp.w_dist, fp.r_0, fp.r_head, fp.N, bins, bins_t, transposed);
  };
  unsigned long long* cnts[DFS_MAX_PEERS] = {};
  if (peers != nullptr)
    for (int k = 0; k < peers->npeers; ++k) cnts[k] = reinterpret_cast<unsigned long long*>(at_peer(k, counter));
  if (op == DFS_OP_FWD_INIT) {
    const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
    stream_init_kernel<<<blocks, 256, 0, st>>>(fw, fp.log_u, fp.log_u_init, n);
    stream_init_kernel<<<blocks, 256, 0, st>>>(gw, fp.log_v, fp.log_v_init, n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = tile_split_reset(split, fp.B, fp.H, fp.N, st);
    if (e == cudaSuccess) e = compute_extents(fp.mask, fp.B, fp.N, extents, st);
    if (e == cudaSuccess && bins != nullptr && bins_given(bin_source(fp)))
      e = build_cost_bins(bin_source(fp), fp.B, fp.N, bins, bins_t, st);
    if (e == cudaSuccess && peers != nullptr) e = peer_signal(cnts, peers->npeers, st);
    return e;
  }
  StreamParams p{};
  p.dtype = fp.in_dtype;
  p.eps = fp.eps;
  p.mask = fp.mask;
  p.B = fp.B;
  p.H = fp.H;
  p.N = fp.N;
  p.row_begin = r0;
  p.row_end = r1;
  p.lam = fp.lam;
  p.qk_scale = fp.qk_scale;
  // the TMA-staged kernels take the row passes whenever they cover the operands
  const bool tma = tile_path_ok(fp.in_dtype, fp.d, fp.N, fp.Q, fp.K);
  TileArgs ta{};
  ta.dtype = fp.in_dtype;
  ta.d = fp.d;
  ta.eps = fp.eps;
  ta.mask = fp.mask;
  ta.status = fp.status;
  ta.B = fp.B;
  ta.H = fp.H;
  ta.N = fp.N;
  ta.row_begin = r0;
  ta.row_end = r1;
  ta.lam = fp.lam;
  ta.qk_scale = fp.qk_scale;
  ta.split = split;
  ta.extent = fp.mask != nullptr ? extents : nullptr;
  if (peers != nullptr) {
    if (!tma) return cudaErrorNotSupported;
    ta.wait_cnt = counter;
    ta.wait_for = peers->wait_for;
  }
  if (tma && (op == DFS_OP_FWD_ROWS || op == DFS_OP_FWD_COLS)) {
    const bool rows = op == DFS_OP_FWD_ROWS;  // the column half-update is the row pass on S^T
    ta.A = rows ? fp.Q : fp.K;
    ta.Bop = rows ? fp.K : fp.Q;
    ta.col_bias = rows ? gw : fw;
    ta.row_marg = rows ? fp.log_mu : fp.log_nu;
    ta.row_out = rows ? fw : gw;
    ta.row_out_nat = rows ? fp.log_u : fp.log_v;
    ta.ct = terms(!rows);
    if (peers != nullptr) {
      ta.npeers = peers->npeers;
      for (int k = 0; k < peers->npeers; ++k) {
        ta.peer_out[k] = reinterpret_cast<float*>(at_peer(k, ta.row_out));
        ta.peer_cnt[k] = cnts[k];
      }
    }
    return launch_tile_pass(TL_LSE, ta, st);
  }
  if (op == DFS_OP_FWD_ROWS) {
    p.Aop = fp.Q;
    p.Bop = fp.K;
    p.col_bias = gw;
    p.row_marg = fp.log_mu;
    p.row_out = fw;
    p.row_out_nat = fp.log_u;
    return launch_stream(SM_LSE, fp.d, p, st);
  }
  if (op == DFS_OP_FWD_COLS) {  // the same kernel on S^T = K Q^T
    p.Aop = fp.K;
    p.Bop = fp.Q;
    p.col_bias = fw;
    p.row_marg = fp.log_nu;
    p.row_out = gw;
    p.row_out_nat = fp.log_v;
    return launch_stream(SM_LSE, fp.d, p, st);
  }
  if (op == DFS_OP_FWD_OUT) {
    if (fp.O == nullptr) return cudaSuccess;
    p.Aop = fp.Q;
    p.Bop = fp.K;
    p.col_bias = gw;
    p.row_bias = fw;
    p.row_out = mw;
    p.row_R = Rw;
    cudaError_t e;
    if (tma) {
      ta.A = fp.Q;
      ta.Bop = fp.K;
      ta.col_bias = gw;
      ta.row_bias = fw;
      ta.row_out = mw;
      ta.row_R = Rw;
      ta.ct = terms(false);
      e = launch_tile_pass(TL_ROWSTATS, ta, st);
      if (e != cudaSuccess) return e;
      if (bt_path_ok(fp.d, fp.N, ws)) {
        // O = T_norm V by the TMA-staged tile pass on fp32 copies of Q, K and V^T
        float* cp = copies;
        const size_t nd = n * fp.d;
        float* Qf = cp;
        float* Kf = cp + nd;
        float* VT = cp + 2 * nd;
        const int BH = fp.B * fp.H;
        e = bt_convert(fp.Q, fp.in_dtype, Qf, nullptr, BH, fp.N, fp.d, st);
        if (e == cudaSuccess) e = bt_convert(fp.K, fp.in_dtype, Kf, nullptr, BH, fp.N, fp.d, st);
        if (e == cudaSuccess) e = bt_convert(fp.V, fp.in_dtype, nullptr, VT, BH, fp.N, fp.d, st);
        if (e != cudaSuccess) return e;
        BtArgs ba{};
        ba.A = Qf;
        ba.Bop = Kf;
        ba.B3 = VT;
        ba.d = fp.d;
        ba.eps = fp.eps;
        ba.qk_scale = fp.qk_scale;
        ba.mask = fp.mask;
        ba.tv[0] = gw;
        ba.pot_mask = 1;
        ba.xvec = fp.x_centroid != nullptr ? fp.x_res : nullptr;
        ba.rv[0] = fw;
        ba.rv[1] = mw;
        ba.rv[2] = Rw;
        ba.out0 = fp.x_centroid;
        ba.acc = fp.O;
        ba.acc_scale = 1.0f;
        ba.status = fp.status;
        ba.extent = ta.extent;
        ba.ct = terms(false);
        ba.B = fp.B;
        ba.H = fp.H;
        ba.N = fp.N;
        ba.row_begin = r0;
        ba.row_end = r1;
        return launch_bt_pass(BTP_OUT, ba, st);
      }
    } else {
      e = launch_stream(SM_ROWSTATS, fp.d, p, st);
    }
    if (e != cudaSuccess) return e;
    p.Vop = fp.V;
    p.row_m = mw;
    p.O = fp.O;
    p.x_res = fp.x_res;
    p.x_centroid = fp.x_centroid;
    return launch_stream(SM_OUT, fp.d, p, st);
  }
  return cudaErrorInvalidValue;
}

// Full streamed forward on one GPU: K_iter x (row half-update, column
// half-update), then the transport output.
cudaError_t launch_stream_fwd(const FwdParams& fp, float* ws, cudaStream_t st) {
  cudaError_t e = stream_fwd_op(DFS_OP_FWD_INIT, fp, ws, 0, fp.N, st);
  for (int it = 0; e == cudaSuccess && it < fp.K_iter; ++it) {
    e = stream_fwd_op(DFS_OP_FWD_ROWS, fp, ws, 0, fp.N, st);
    if (e == cudaSuccess) e = stream_fwd_op(DFS_OP_FWD_COLS, fp, ws, 0, fp.N, st);
  }
  if (e == cudaSuccess) e = stream_fwd_op(DFS_OP_FWD_OUT, fp, ws, 0, fp.N, st);
  return e;
}

}  // namespace dfs
