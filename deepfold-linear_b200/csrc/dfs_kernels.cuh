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

// Where the position bins of a problem come from: a (B, N, N) int32 table, or
// the inputs of the reference's compute_bins (src/deepfold/model/
// position_encoding.py:7-52), evaluated per pair:
//   same chain, no bond:  clamp(gidx_i - gidx_j, -32, 32) + 32    (0 .. 64)
//   other chain, no bond: 65;  same chain, bond: 66;  other chain, bond: 67
struct BinSource {
  const int32_t* table;   // (B, N, N) or null
  const int32_t* chain;   // (B, N) chain id, with gidx and bond when table is null
  const int32_t* gidx;    // (B, N) global residue index
  const uint8_t* bond;    // (B, N, N) covalent bond adjacency, 0 / 1
};
DFS_DEV_HOST_INLINE bool bins_given(const BinSource& s) { return s.table != nullptr || s.chain != nullptr; }
// bin of pair (i, j) of batch element b; values outside [0, 68) come from a table only
DFS_DEV int bin_at(const BinSource& s, size_t b, int N, int i, int j) {
  const size_t ij = (b * N + i) * static_cast<size_t>(N) + j;
  if (s.table != nullptr) return s.table[ij];
  const size_t bi = b * N + i, bj = b * N + j;
  const bool same = s.chain[bi] == s.chain[bj];
  if (s.bond[ij] != 0) return same ? 66 : 67;
  if (!same) return 65;
  const long long sep = static_cast<long long>(s.gidx[bi]) - s.gidx[bj];
  return static_cast<int>(sep < -32 ? 0 : sep > 32 ? 64 : sep + 32);
}

DFS_DEV float load_f32(const void* p, size_t i, int dtype) {
  if (dtype == DFS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == DFS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// Optional cost terms on the streamed passes.  Each element (r, c) of a pass
// (rows r, columns c of S = A B^T; for the passes on S^T the rows are the cost's
// columns) adds, in log2 units,
//     pwS[bins(r, c)] + wS * t(r, c),  t = dist / (r_h + dist),
//     dist = sqrt(|x_r - x_c|^2 + 1e-8)            (sinkhorn_kernel.py:59-129)
// with pwS = -pos_weight[h] log2(e) / eps_h and wS = -w_h log2(e) / eps_h.  The
// bins come from a per-call uint8 table in the pass's orientation (rows of
// kBinRow bytes; entries outside [0, 68), and the padding, hold 68, a bin
// whose weight is 0); the distance is computed from the coordinates.
constexpr int kBinCount = 68;
struct CostTerms {
  const uint8_t* bins;      // (B, N, bin_stride) uint8 in the pass's orientation, or null
  int bin_stride;           // bytes per row of the table (N rounded up to 128)
  const float* pos_weight;  // (H, 68) with bins
  const float* x;           // (B, N, 3) coordinates with the geometry term, or null
  const float* w_dist;      // (H,) with x
  float r_0;
  const float* r_head;      // (H,) per-head geometry scale r_h, or null: r_0
};
// geometry scale of head h
DFS_DEV float geo_scale(const CostTerms& t, int h) { return t.r_head != nullptr ? t.r_head[h] : t.r_0; }
// Shares of the shared-parameter gradients written by the streamed gradient
// passes (null: not wanted), summed by stream_costgrad_finalize.
struct CostGradOut {
  float* dx;    // (BH, N, 3) this pass's share of dx per row
  float* dw;    // (BH, N) per-row share of dw_dist
  float* dr;    // (BH, N) per-row share of sum dC dist / (r_h + dist)^2 (dr_head = -w_h times it)
  float* dpos;  // (BH, row blocks, 68) per-CTA bin sums
};

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
  float qk_scale;          // 1/sqrt(d) of the caller's head dim (kernels may run d zero-padded)
  int cost_terms;          // DFS_TERM_* declared by the problem (workspace layout of the streamed path)
  const float* r_head;     // (H,) per-head geometry scale, or null: r_0
  const int32_t* chain_id; // position bins from compute_bins' inputs (with pos_bins null)
  const int32_t* global_idx;
  const uint8_t* bond_matrix;
};
DFS_DEV_HOST_INLINE BinSource bin_source(const FwdParams& p) {
  return BinSource{p.pos_bins, p.chain_id, p.global_idx, p.bond_matrix};
}

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
  float qk_scale;          // 1/sqrt(d) of the caller's head dim (kernels may run d zero-padded)
  int cost_terms;          // DFS_TERM_* declared by the problem (workspace layout of the streamed path)
  const float* r_head;     // (H,) per-head geometry scale, or null: r_0
  float* dr_head;          // (H,) gradient of r_head (or of r_0 per head), or null
  const int32_t* chain_id; // position bins from compute_bins' inputs (with pos_bins null)
  const int32_t* global_idx;
  const uint8_t* bond_matrix;
};
DFS_DEV_HOST_INLINE BinSource bin_source(const BwdParams& p) {
  return BinSource{p.pos_bins, p.chain_id, p.global_idx, p.bond_matrix};
}

cudaError_t launch_resident_fwd(const FwdParams& p, cudaStream_t st);
size_t resident_fwd_smem(int N, int d);
cudaError_t launch_stream_fwd(const FwdParams& p, float* ws, cudaStream_t st);
// dense-cost forward streamed from the caller's C (problems outside the
// resident kernels' range): potentials, O / T_norm / x_centroid, early stop
size_t dense_fwd_workspace(int B, int H, int N);
cudaError_t launch_dense_fwd(const FwdParams& p, void* ws, size_t ws_bytes, cudaStream_t st);
size_t dense_fuse_part_bytes(int B, int H, int N);
cudaError_t launch_dense_iterations(const float* C, const float* eps, const float* mu, const float* nu,
                                    const float* mask, int B, int H, int N, float lam, float* hist, int it_begin,
                                    int it_end, float* part, size_t part_bytes, cudaStream_t st);
// Peer exchange of a row-sharded forward: every GPU's workspace (same layout,
// 256-byte aligned bases) and the cumulative arrival count the phase waits for.
struct PeerInfo {
  int npeers, self;
  void* ws[DFS_MAX_PEERS];
  unsigned long long wait_for;
};
cudaError_t stream_fwd_op(int op, const FwdParams& p, float* ws, int r0, int r1, cudaStream_t st,
                          const PeerInfo* peers = nullptr);
cudaError_t stream_bwd_op(int op, const BwdParams& p, float* ws, int r0, int r1, cudaStream_t st);
// Peer-memory gather of the rows [r0, r1) of a slot (P x N x width floats at
// slot_offset of every GPU's buffer pi.ws[k]); counters at counter_offset
// (arrivals, push completion, expected count: device-relative waits).
cudaError_t peer_gather_rows(const PeerInfo& pi, size_t slot_offset, int P, int N, int width, int row_begin,
                             int row_end, size_t counter_offset, int32_t* status, cudaStream_t st);
// The row-sharded backward's CG rounds 1 .. max_iter as one CUDA graph with a
// device-terminated WHILE loop (plan products on rows [r0, r1), peer gathers
// of their slots, the CG step); false when no such graph could be built.
bool cg_loop_graph_peer(const BwdParams& bp, float* ws, int r0, int r1, const PeerInfo& pi, size_t counter_offset,
                        cudaStream_t st);
size_t stream_fwd_workspace(int B, int H, int N, int d, int terms = 0);
cudaError_t launch_resident_bwd(const BwdParams& p, cudaStream_t st);
cudaError_t launch_stream_bwd(const BwdParams& p, float* ws, cudaStream_t st);
size_t stream_bwd_workspace(int B, int H, int N, int d, int terms = 0);
// Per-call tables of the cost terms (dfs_stream.cu): bytes of one uint8 bin
// table, and the launch that builds the table and its transpose.
size_t cost_bins_bytes(int B, int N);
int cost_bin_stride(int N);
cudaError_t build_cost_bins(const BinSource& src, int B, int N, uint8_t* bins, uint8_t* bins_t, cudaStream_t st);
// compute_bins of the reference into a (B, N, N) int32 table
cudaError_t compute_bins_table(const int32_t* chain, const int32_t* gidx, const uint8_t* bond, int B, int N,
                               int32_t* out, cudaStream_t st);
// The cost terms of a pass from the operator's inputs (position term when
// pos_weight and the tables are given, geometry term when x_res and w_dist
// are): `transposed` for the passes on S^T, whose rows are the cost's columns.
CostTerms cost_terms_of(const float* pos_weight, const float* x_res, const float* w_dist, float r_0,
                        const float* r_head, int N,
                        const uint8_t* bins, const uint8_t* bins_t, bool transposed);
size_t resident_bwd_smem(int N, int d);
size_t resident_bwd_workspace(int B, int H, int N, int d);
// TMA-staged row passes of the streamed path (dfs_stream_tma.cu): one launch
// reduces every row of [row_begin, row_end) over all columns of S = A B^T.
enum TilePass { TL_LSE = 0, TL_ROWSTATS = 1, TL_MATVEC = 2 };
struct TileArgs {
  const void* A;           // (BH, N, d) row operand
  const void* Bop;         // (BH, N, d) column operand
  int dtype, d;
  const float* eps;
  const float* mask;
  const float* col_bias;   // (BH, N) column potential, log2 units
  const float* col_vec;    // MATVEC: v
  const float* row_bias;   // ROWSTATS, MATVEC: row potential, log2 units
  const float* row_marg;   // LSE: natural-log row marginal
  const float* row_scale;  // MATVEC: per-row factor, or null
  const int32_t* done;     // MATVEC: per-problem skip flags, or null
  float* row_out;
  float* row_out_nat;
  float* row_R;
  int32_t* status;
  const int2* extent;      // (B) valid extents of the mask (compute_extents), or null: scan the mask
  float* split;            // tile_split_bytes() of scratch for column splits (counters zeroed
                           // by tile_split_reset), or null: one CTA per row block
  // peer exchange (LSE only): row_out's slot in every GPU's workspace, their arrival
  // counters, and this GPU's counter to wait on before reading (npeers = 0: none)
  int npeers;
  float* peer_out[DFS_MAX_PEERS];
  unsigned long long* peer_cnt[DFS_MAX_PEERS];
  const unsigned long long* wait_cnt;
  unsigned long long wait_for;
  int B, H, N, row_begin, row_end;
  float lam;
  float qk_scale;          // 1/sqrt(d) of the cost
  CostTerms ct;            // optional cost terms in this pass's orientation (bins / x null: none)
};
size_t tile_split_bytes(int B, int H, int N);
// Per batch element, the smallest range [lo, hi) of positions holding every
// valid point of the mask ([0, 0) when none is valid), into out[B].
cudaError_t compute_extents(const float* mask, int B, int N, int2* out, cudaStream_t st);
// Raises each of the n counters once (system-scope release), one thread.
cudaError_t peer_signal(unsigned long long* const* cnt, int n, cudaStream_t st);
cudaError_t tile_split_reset(float* split, int B, int H, int N, cudaStream_t st);
// True when the TMA-staged kernels cover this operand type, head dim, length
// (N >= 128) and the two operand addresses (16-byte aligned); otherwise the
// register-staged kernels run the pass.
bool tile_path_ok(int dtype, int d, int N, const void* a, const void* b);
// True when the driver provides cuTensorMapEncodeTiled (the TMA-staged passes).
bool tmap_available();
cudaError_t launch_tile_pass(int mode, const TileArgs& t, cudaStream_t st);

// TMA-staged tile passes of the streamed backward (dfs_stream_bwd_tma.cu) on
// fp32 copies of the operands kept in the backward workspace.
struct BtCopies {
  float* Qf;   // (BH, N, d) row-major fp32 copies
  float* Kf;
  float* Vf;
  float* dOf;
  float* QT;   // (BH, d, N) transposed fp32 copies
  float* KT;
  float* dOT;
};
struct BtArgs {
  const float* A;    // row operands (BH, N, d): S = A B^T, dT = A2 B2^T
  const float* A2;
  const float* Bop;  // column operands (BH, N, d)
  const float* B2;
  const float* B3;   // transposed accumulation operand (BH, d, N)
  int d;
  const float* eps;
  const float* mask;
  const float* tv[5];
  int pot_mask;
  const float* xvec;
  int xvec_per_head;
  const float* rv[5];
  const float* rxvec;
  int rxvec_per_head;
  float* out0;
  float* out1;
  float* out2;
  float* acc;
  float acc_scale;
  int32_t* status;
  const int2* extent;      // (B) valid extents of the mask, or null
  int B, H, N, row_begin, row_end;
  float qk_scale;          // 1/sqrt(d) of the cost
  CostTerms ct;            // optional cost terms in this pass's orientation
  CostGradOut cg;          // DQ / DK / COL: shares of the shared-parameter gradients, or null
};
enum BtPass { BTP_ROW = 0, BTP_COL = 1, BTP_DQ = 2, BTP_DK = 3, BTP_OUT = 4 };
size_t bt_copies_bytes(int B, int H, int N, int d);
bool bt_path_ok(int d, int N, const void* ws);
BtCopies bt_copies(float* region, int B, int H, int N, int d);
cudaError_t bt_prep(const BwdParams& bp, const BtCopies& c, cudaStream_t st);
// fp32 copies of one (BH, N, d) operand: row-major and / or transposed (either may be null)
cudaError_t bt_convert(const void* src, int dtype, float* row_out, float* t_out, int BH, int N, int d,
                       cudaStream_t st);
cudaError_t launch_bt_pass(int mode, const BtArgs& a, cudaStream_t st);

// Operand transforms (dfs_pad.cu): the instantiated head dim a problem of head
// dim d runs on (0 when d > 64); zero padding of (rows, d) to (rows, dk);
// the bf16 hi / lo split of fp32 operands into column blocks (part 0 zero,
// 1 hi, 2 lo); side-by-side copies of fp32 rows; the sum of selected column
// blocks of width d (bit b of `blocks`: block b) back into (rows, d).
int kernel_head_dim(int d);
cudaError_t pad_rows(const void* src, void* dst, int esize, size_t rows, int d, int dk, cudaStream_t st);
cudaError_t split_rows(const float* src, void* dst, size_t rows, int d, int dk, int p0, int p1, int p2,
                       cudaStream_t st);
cudaError_t dup_rows(const float* src, float* dst, size_t rows, int d, int dk, int copies, cudaStream_t st);
cudaError_t fold_rows(const float* src, float* dst, size_t rows, int d, int dk, int blocks, cudaStream_t st);

cudaError_t launch_selftest_mma(int which, const float* A, const float* B, float* D, int M, int N, int K,
                                cudaStream_t st);

}  // namespace dfs
