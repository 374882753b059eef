// dfs_abi.cu -- the extern "C" entry points of libdfsink.so (include/dfsink.h):
// argument validation, workspace sizing and kernel dispatch.  Nothing here
// allocates device memory.
#include <cmath>
#include <cstring>

#include "dfs_kernels.cuh"

using namespace dfs;

namespace {

bool dims_ok(const dfs_problem* p) {
  return p && p->B > 0 && p->H > 0 && p->N > 0 && p->d > 0 && p->K_iter >= 0 &&
         (p->in_dtype == DFS_BF16 || p->in_dtype == DFS_F16 || p->in_dtype == DFS_F32) &&
         (p->cost_mode == DFS_COST_QK || p->cost_mode == DFS_COST_DENSE) &&
         !(p->lam <= 0.0f) && !std::isnan(p->lam) && (p->threshold <= 0.0f || p->check_every > 0);
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? DFS_OK : DFS_ERR_CUDA; }

// the kernels read Q, K, V and dO in 16-byte chunks
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cluster-resident kernels (S kept on chip): d <= 32, N <= 384; streamed
// kernels (S recomputed tile by tile): d <= 64, N <= kStreamMaxN.  The kernels
// are instantiated for head dims 32 and 64.  Operands are transformed on copies
// at the front of the workspace (dfs_pad.cu) when
//   XF_PAD      the head dim is another one: zero-padded to the next one;
//   XF_SPLIT_QK fp32 Q, K, V whose tripled head dim stays in the same kernel
//               family (3 d <= 32 for d <= 32, i.e. d <= 10; 3 d <= 64 for
//               32 < d <= 64 never holds): bf16 hi / lo parts along the
//               contraction dimension (exact products instead of tf32 ones);
//   XF_SPLIT_V  fp32 V of the dense-cost path with 2 d <= 32: V = [Vhi Vlo].
constexpr int kResidentMaxN = 384;
constexpr int kStreamMaxN = 1 << 16;
enum { XF_NONE = 0, XF_PAD = 1, XF_SPLIT_QK = 2, XF_SPLIT_V = 3 };
// the fp32 split of a problem (XF_SPLIT_QK / XF_SPLIT_V), or XF_NONE
int split_kind(const dfs_problem* p) {
  if (p->in_dtype == DFS_F32 && p->cost_mode == DFS_COST_QK && 3 * p->d <= 32) return XF_SPLIT_QK;
  if (p->in_dtype == DFS_F32 && p->cost_mode == DFS_COST_DENSE && 2 * p->d <= 32) return XF_SPLIT_V;
  return XF_NONE;
}
int kdim(const dfs_problem* p);
bool dense_streamed(const dfs_problem* p);
int xform(const dfs_problem* p) {
  if (dense_streamed(p)) return XF_NONE;  // reads C and fp32 V as given
  const int x = split_kind(p);
  if (x != XF_NONE) return x;
  return kdim(p) != p->d ? XF_PAD : XF_NONE;
}
// position / geometry terms of a streamed problem (bits of dfs_problem.cost_terms)
bool streamed_terms(const dfs_problem* p) {
  return p->cost_mode == DFS_COST_QK && p->N > kResidentMaxN && (p->cost_terms & (DFS_TERM_POS | DFS_TERM_GEO)) != 0;
}
int kdim(const dfs_problem* p) {
  const int x = split_kind(p);
  const int k = kernel_head_dim(x == XF_SPLIT_QK ? 3 * p->d : x == XF_SPLIT_V ? 2 * p->d : p->d);
  // streamed problems with cost terms run on the TMA-staged passes, built for
  // 128- and 256-byte operand rows: head dim 64 (zero-padded from d <= 32)
  return (k == 32 && streamed_terms(p)) ? 64 : k;
}
bool padded(const dfs_problem* p) { return xform(p) != XF_NONE; }
bool resident(const dfs_problem* p) { return kdim(p) == 32 && p->N <= kResidentMaxN; }
bool streamed(const dfs_problem* p) { return kdim(p) != 0 && p->N <= kStreamMaxN; }
// dense cost outside the resident range: the HBM passes over C (dfs_dense.cu),
// fp32 V of head dim up to 128
constexpr int kDenseMaxD = 128;
bool dense_streamed(const dfs_problem* p) {
  return p->cost_mode == DFS_COST_DENSE && !(kdim(p) == 32 && p->N <= kResidentMaxN) && p->d <= kDenseMaxD &&
         p->N <= kStreamMaxN;
}

size_t elem_bytes(int dtype) { return dtype == DFS_F32 ? 4 : 2; }
size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
size_t padded_elems(const dfs_problem* p) { return static_cast<size_t>(p->B) * p->H * p->N * kdim(p); }
// element type of the kernels' Q, K, V: bf16 parts when split
int kernel_dtype(const dfs_problem* p) {
  const int x = xform(p);
  return (x == XF_SPLIT_QK || x == XF_SPLIT_V) ? DFS_BF16 : p->in_dtype;
}
// transformed copies at the front of the workspace: Q, K, V (kernel type), then
// O (forward) or dO, dQ, dK, dV (backward), fp32; each region 256-byte aligned
size_t pad_fwd_bytes(const dfs_problem* p) {
  if (!padded(p)) return 0;
  const size_t nd = padded_elems(p);
  return 3 * round256(nd * elem_bytes(kernel_dtype(p))) + round256(nd * 4);
}
size_t pad_bwd_bytes(const dfs_problem* p) {
  if (!padded(p)) return 0;
  const size_t nd = padded_elems(p);
  return 3 * round256(nd * elem_bytes(kernel_dtype(p))) + 4 * round256(nd * 4);
}

// Transformed copy of one operand (Q: which = 0, K: 1, V: 2) into dst.
cudaError_t transform_operand(const dfs_problem* p, int which, const void* src, void* dst, size_t rows,
                              cudaStream_t st) {
  const int x = xform(p), dk = kdim(p);
  if (x == XF_SPLIT_QK) {
    static const int parts[3][3] = {{1, 1, 2}, {1, 2, 1}, {1, 2, 0}};  // Q' = [hi hi lo], K' = [hi lo hi], V' = [hi lo 0]
    return split_rows(static_cast<const float*>(src), dst, rows, p->d, dk, parts[which][0], parts[which][1],
                      parts[which][2], st);
  }
  if (x == XF_SPLIT_V) return split_rows(static_cast<const float*>(src), dst, rows, p->d, dk, 1, 2, 0, st);
  return pad_rows(src, dst, static_cast<int>(elem_bytes(p->in_dtype)), rows, p->d, dk, st);
}
// Output column blocks summed back into (rows, d): O and dQ take blocks 0 and 1
// of a split problem, dK blocks 0 and 2, dV block 0; padded problems block 0.
int fold_blocks(const dfs_problem* p, char what) {
  const int x = xform(p);
  if (x == XF_NONE || x == XF_PAD) return 1;
  if (what == 'O' || what == 'Q') return 3;
  if (what == 'K') return 5;
  return 1;
}

FwdParams fwd_params(const dfs_problem* p, const dfs_fwd_args* a) {
  FwdParams q;
  std::memset(&q, 0, sizeof(q));
  q.Q = a->Q; q.K = a->K; q.V = a->V; q.C = a->C;
  q.x_res = a->x_res; q.pos_weight = a->pos_weight; q.pos_bins = a->pos_bins;
  q.eps = a->eps; q.w_dist = a->w_dist; q.log_mu = a->log_mu; q.log_nu = a->log_nu;
  q.log_u_init = a->log_u_init; q.log_v_init = a->log_v_init; q.mask = a->mask;
  q.O = a->O; q.x_centroid = a->x_centroid; q.log_u = a->log_u; q.log_v = a->log_v;
  q.status = a->status;
  q.T_out = a->T_norm;
  q.B = p->B; q.H = p->H; q.N = p->N; q.d = p->d; q.in_dtype = p->in_dtype;
  q.cost_mode = p->cost_mode; q.K_iter = p->K_iter; q.check_every = p->check_every > 0 ? p->check_every : 1;
  q.lam = p->lam; q.r_0 = p->r_0; q.threshold = p->threshold;
  q.qk_scale = 1.0f / std::sqrt(static_cast<float>(p->d));
  q.cost_terms = p->cost_terms;
  q.r_head = a->r_head;
  q.chain_id = a->chain_id;
  q.global_idx = a->global_idx;
  q.bond_matrix = a->bond_matrix;
  return q;
}

BwdParams bwd_params(const dfs_problem* p, const dfs_cg_params* cg, const dfs_bwd_args* a, void* workspace) {
  BwdParams q;
  std::memset(&q, 0, sizeof(q));
  q.Q = a->Q; q.K = a->K; q.V = a->V;
  q.x_res = a->x_res; q.pos_weight = a->pos_weight; q.pos_bins = a->pos_bins;
  q.eps = a->eps; q.w_dist = a->w_dist; q.log_mu = a->log_mu; q.log_nu = a->log_nu; q.mask = a->mask;
  q.log_u = a->log_u; q.log_v = a->log_v; q.dO = a->dO; q.dxc = a->dxc;
  q.dQ = a->dQ; q.dK = a->dK; q.dV = a->dV; q.dlog_mu = a->dlog_mu; q.dlog_nu = a->dlog_nu;
  q.dx_res = a->dx_res; q.dpos_weight = a->dpos_weight; q.dw_dist = a->dw_dist;
  q.cg_iters = a->cg_iters; q.cg_residual = a->cg_residual; q.status = a->status;
  q.ws = static_cast<float*>(workspace);
  q.B = p->B; q.H = p->H; q.N = p->N; q.d = p->d; q.in_dtype = p->in_dtype;
  q.cg_max_iter = cg->max_iter; q.cg_rtol = cg->rtol; q.cg_atol = cg->atol;
  q.lam = p->lam; q.r_0 = p->r_0;
  q.qk_scale = 1.0f / std::sqrt(static_cast<float>(p->d));
  q.cost_terms = p->cost_terms;
  q.r_head = a->r_head;
  q.dr_head = a->dr_head;
  q.chain_id = a->chain_id;
  q.global_idx = a->global_idx;
  q.bond_matrix = a->bond_matrix;
  return q;
}

// position bins: the int32 table, or all three compute_bins inputs, or nothing
bool bins_args_ok(const int32_t* table, const int32_t* chain, const int32_t* gidx, const uint8_t* bond) {
  const int parts = (chain != nullptr) + (gidx != nullptr) + (bond != nullptr);
  return parts == 0 || (parts == 3 && table == nullptr);
}
bool has_bins(const int32_t* table, const int32_t* chain) { return table != nullptr || chain != nullptr; }

// argument checks shared by dfs_fwd and the forward phases
int check_fwd_args(const dfs_problem* p, const dfs_fwd_args* a) {
  if (!dims_ok(p) || !a) return DFS_ERR_INVALID_ARGUMENT;
  if (!a->eps || !a->log_mu || !a->log_nu || !a->log_u || !a->log_v) return DFS_ERR_INVALID_ARGUMENT;
  if (p->cost_mode == DFS_COST_QK && (!a->Q || !a->K)) return DFS_ERR_INVALID_ARGUMENT;
  if (p->cost_mode == DFS_COST_DENSE && !a->C) return DFS_ERR_INVALID_ARGUMENT;
  if (a->O && !a->V) return DFS_ERR_INVALID_ARGUMENT;
  if (!bins_args_ok(a->pos_bins, a->chain_id, a->global_idx, a->bond_matrix)) return DFS_ERR_INVALID_ARGUMENT;
  if (a->pos_weight && !has_bins(a->pos_bins, a->chain_id)) return DFS_ERR_INVALID_ARGUMENT;
  if (a->x_centroid && !a->x_res) return DFS_ERR_INVALID_ARGUMENT;
  if (dense_streamed(p)) {
    // fp32 V (the dense entry points' values), no position / geometry terms (C holds the whole cost)
    if (a->V && p->in_dtype != DFS_F32) return DFS_ERR_UNSUPPORTED;
    if (a->pos_weight || a->w_dist) return DFS_ERR_INVALID_ARGUMENT;
    return DFS_OK;
  }
  if (!resident(p) && !streamed(p)) return DFS_ERR_UNSUPPORTED;
  // the kernels read the operands in 16-byte chunks (padded ones are copies)
  if (!padded(p) && (!aligned16(a->O) || !aligned16(a->Q) || !aligned16(a->K) || !aligned16(a->V)))
    return DFS_ERR_INVALID_ARGUMENT;
  return DFS_OK;
}

// The position / geometry terms of the streamed path run on the TMA-staged
// passes only: N >= 128 and N % 4 == 0 (the transposed fp32 copies), operand
// rows of 128 or 256 bytes.
bool terms_path_ok(const dfs_problem* p) {
  const int dk = kdim(p);
  const int dt = kernel_dtype(p);
  return p->N >= 128 && p->N % 4 == 0 && (dk == 64 || dt == DFS_F32) && tmap_available();
}

// streamed path: QK cost with masks, marginals, kappa, warm starts and the
// position / geometry terms the problem declares; early stopping and the dense
// plan are resident-only
int check_stream_fwd(const dfs_problem* p, const dfs_fwd_args* a, void* workspace, size_t workspace_bytes) {
  if (p->cost_mode != DFS_COST_QK || p->threshold > 0.0f || a->T_norm || (a->x_centroid && !a->O))
    return DFS_ERR_UNSUPPORTED;
  const bool pos = a->pos_weight != nullptr, geo = a->x_res != nullptr && a->w_dist != nullptr;
  if ((pos && !(p->cost_terms & DFS_TERM_POS)) || (geo && !(p->cost_terms & DFS_TERM_GEO)))
    return DFS_ERR_INVALID_ARGUMENT;  // the workspace layout depends on the declared terms
  if ((pos || geo) && !terms_path_ok(p)) return DFS_ERR_UNSUPPORTED;
  if (workspace == nullptr || workspace_bytes < stream_fwd_workspace(p->B, p->H, p->N, kdim(p), p->cost_terms) ||
      !aligned16(workspace))
    return DFS_ERR_WORKSPACE;
  return DFS_OK;
}

int check_bwd_args(const dfs_problem* p, const dfs_cg_params* cg, const dfs_bwd_args* a) {
  if (!dims_ok(p) || !a || !cg) return DFS_ERR_INVALID_ARGUMENT;
  if (p->cost_mode != DFS_COST_QK) return DFS_ERR_UNSUPPORTED;
  if (!a->Q || !a->K || !a->V || !a->eps || !a->log_mu || !a->log_nu || !a->log_u || !a->log_v || !a->dO)
    return DFS_ERR_INVALID_ARGUMENT;
  if (!bins_args_ok(a->pos_bins, a->chain_id, a->global_idx, a->bond_matrix)) return DFS_ERR_INVALID_ARGUMENT;
  if (a->pos_weight && !has_bins(a->pos_bins, a->chain_id)) return DFS_ERR_INVALID_ARGUMENT;
  if (a->dxc && !a->x_res) return DFS_ERR_INVALID_ARGUMENT;
  if ((a->dx_res || a->dw_dist) && !a->x_res) return DFS_ERR_INVALID_ARGUMENT;
  if (a->dr_head && (!a->x_res || !a->w_dist)) return DFS_ERR_INVALID_ARGUMENT;
  if (a->dpos_weight && !has_bins(a->pos_bins, a->chain_id)) return DFS_ERR_INVALID_ARGUMENT;
  if (cg->max_iter < 0) return DFS_ERR_INVALID_ARGUMENT;
  if (!resident(p) && !streamed(p)) return DFS_ERR_UNSUPPORTED;
  if (!padded(p) && (!aligned16(a->Q) || !aligned16(a->K) || !aligned16(a->V) || !aligned16(a->dO) ||
                     !aligned16(a->dQ) || !aligned16(a->dK) || !aligned16(a->dV)))
    return DFS_ERR_INVALID_ARGUMENT;
  return DFS_OK;
}

// streamed path: the declared position / geometry terms and the gradients of
// x_res, pos_weight, w_dist (their shares need the declared workspace)
int check_stream_bwd(const dfs_problem* p, const dfs_bwd_args* a, void* workspace, size_t workspace_bytes) {
  const bool pos = a->pos_weight != nullptr, geo = a->x_res != nullptr && a->w_dist != nullptr;
  if ((pos && !(p->cost_terms & DFS_TERM_POS)) || (geo && !(p->cost_terms & DFS_TERM_GEO)))
    return DFS_ERR_INVALID_ARGUMENT;
  const bool shared_grads =
      a->dx_res != nullptr || a->dpos_weight != nullptr || a->dw_dist != nullptr || a->dr_head != nullptr;
  if (shared_grads && p->cost_terms == 0) return DFS_ERR_INVALID_ARGUMENT;
  if ((pos || geo || shared_grads) && !terms_path_ok(p)) return DFS_ERR_UNSUPPORTED;
  if (workspace == nullptr || workspace_bytes < stream_bwd_workspace(p->B, p->H, p->N, kdim(p), p->cost_terms) ||
      !aligned16(workspace))
    return DFS_ERR_WORKSPACE;
  return DFS_OK;
}

}  // namespace

extern "C" {

int dfs_abi_version(void) { return DFS_ABI_VERSION; }

const char* dfs_status_string(int s) {
  switch (s) {
    case DFS_OK: return "ok";
    case DFS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DFS_ERR_UNSUPPORTED: return "shape, dtype or option not supported by the kernels";
    case DFS_ERR_WORKSPACE: return "workspace too small";
    case DFS_ERR_CUDA: return "CUDA runtime error";
    case DFS_ERR_DEVICE_TIMEOUT: return "device: bounded wait gave up";
    case DFS_ERR_NUMERIC: return "device: non-finite potentials after re-stabilisation";
    case DFS_WARN_CG_NOT_CONVERGED: return "device: CG reached max_iter";
    default: return "several device status bits set";
  }
}

int dfs_max_n(int d) { return kernel_head_dim(d) != 0 ? kStreamMaxN : 0; }

int dfs_workspace_size(const dfs_problem* p, size_t* fwd_bytes, size_t* bwd_bytes) {
  if (!dims_ok(p)) return DFS_ERR_INVALID_ARGUMENT;
  if (dense_streamed(p)) {
    if (fwd_bytes) *fwd_bytes = dense_fwd_workspace(p->B, p->H, p->N);
    if (bwd_bytes) *bwd_bytes = 0;  // no backward on the dense-cost path
    return DFS_OK;
  }
  if (!resident(p) && !streamed(p)) return DFS_ERR_UNSUPPORTED;
  const bool res = resident(p);
  const int dk = kdim(p);
  if (fwd_bytes) *fwd_bytes = pad_fwd_bytes(p) + (res ? 0 : stream_fwd_workspace(p->B, p->H, p->N, dk, p->cost_terms));
  if (bwd_bytes)
    *bwd_bytes = pad_bwd_bytes(p) + (res ? resident_bwd_workspace(p->B, p->H, p->N, dk)
                                         : stream_bwd_workspace(p->B, p->H, p->N, dk, p->cost_terms));
  return DFS_OK;
}

int dfs_fwd(const dfs_problem* p, const dfs_fwd_args* a, void* workspace, size_t workspace_bytes,
            void* stream) {
  int rc = check_fwd_args(p, a);
  if (rc != DFS_OK) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dense_streamed(p)) {
    if (workspace == nullptr || workspace_bytes < dense_fwd_workspace(p->B, p->H, p->N) || !aligned16(workspace))
      return DFS_ERR_WORKSPACE;
    return cuda_status(launch_dense_fwd(fwd_params(p, a), workspace, workspace_bytes, st));
  }
  // padded head dim: copies at the front of the workspace, the kernels' share after them
  const size_t pad = pad_fwd_bytes(p);
  if (pad > 0 && (workspace == nullptr || workspace_bytes < pad || !aligned16(workspace))) return DFS_ERR_WORKSPACE;
  char* const ws = static_cast<char*>(workspace);
  void* const kws = pad > 0 ? static_cast<void*>(ws + pad) : workspace;
  const size_t kbytes = workspace_bytes - pad;
  if (!resident(p) && (rc = check_stream_fwd(p, a, kws, kbytes)) != DFS_OK) return rc;
  FwdParams q = fwd_params(p, a);
  const size_t rows = static_cast<size_t>(p->B) * p->H * p->N;
  float* Op = nullptr;
  if (pad > 0) {
    const int dk = kdim(p);
    const size_t opb = round256(padded_elems(p) * elem_bytes(kernel_dtype(p)));
    char* Qp = ws;
    char* Kp = ws + opb;
    char* Vp = ws + 2 * opb;
    Op = reinterpret_cast<float*>(ws + 3 * opb);
    cudaError_t e = cudaSuccess;
    if (a->Q) e = transform_operand(p, 0, a->Q, Qp, rows, st);
    if (e == cudaSuccess && a->K) e = transform_operand(p, 1, a->K, Kp, rows, st);
    if (e == cudaSuccess && a->V) e = transform_operand(p, 2, a->V, Vp, rows, st);
    if (e != cudaSuccess) return DFS_ERR_CUDA;
    q.d = dk;
    q.in_dtype = kernel_dtype(p);
    q.Q = a->Q ? Qp : nullptr;
    q.K = a->K ? Kp : nullptr;
    q.V = a->V ? Vp : nullptr;
    q.O = a->O ? Op : nullptr;
  }
  const cudaError_t e = resident(p) ? launch_resident_fwd(q, st) : launch_stream_fwd(q, static_cast<float*>(kws), st);
  if (e != cudaSuccess) return DFS_ERR_CUDA;
  if (pad > 0 && a->O) return cuda_status(fold_rows(Op, a->O, rows, p->d, kdim(p), fold_blocks(p, 'O'), st));
  return DFS_OK;
}

int dfs_bwd(const dfs_problem* p, const dfs_cg_params* cg, const dfs_bwd_args* a, void* workspace,
            size_t workspace_bytes, void* stream) {
  int rc = check_bwd_args(p, cg, a);
  if (rc != DFS_OK) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t pad = pad_bwd_bytes(p);
  if (pad > 0 && (workspace == nullptr || workspace_bytes < pad || !aligned16(workspace))) return DFS_ERR_WORKSPACE;
  char* const ws = static_cast<char*>(workspace);
  void* const kws = pad > 0 ? static_cast<void*>(ws + pad) : workspace;
  const size_t kbytes = workspace_bytes - pad;
  if (!resident(p)) {
    if ((rc = check_stream_bwd(p, a, kws, kbytes)) != DFS_OK) return rc;
  } else {
    // the resident kernels use the workspace only for the partials of the
    // shared-parameter gradients
    const bool shared = a->dx_res != nullptr || a->dpos_weight != nullptr || a->dw_dist != nullptr ||
                        a->dr_head != nullptr;
    const size_t need = shared ? resident_bwd_workspace(p->B, p->H, p->N, kdim(p)) : 0;
    if (need > 0 && (kws == nullptr || kbytes < need)) return DFS_ERR_WORKSPACE;
  }
  BwdParams q = bwd_params(p, cg, a, kws);
  const size_t rows = static_cast<size_t>(p->B) * p->H * p->N;
  float* grads[3] = {nullptr, nullptr, nullptr};  // padded dQ, dK, dV
  if (pad > 0) {
    const int dk = kdim(p);
    const size_t opb = round256(padded_elems(p) * elem_bytes(kernel_dtype(p)));
    const size_t fb = round256(padded_elems(p) * 4);
    char* Qp = ws;
    char* Kp = ws + opb;
    char* Vp = ws + 2 * opb;
    float* dOp = reinterpret_cast<float*>(ws + 3 * opb);
    for (int k = 0; k < 3; ++k) grads[k] = reinterpret_cast<float*>(ws + 3 * opb + (k + 1) * fb);
    cudaError_t e = transform_operand(p, 0, a->Q, Qp, rows, st);
    if (e == cudaSuccess) e = transform_operand(p, 1, a->K, Kp, rows, st);
    if (e == cudaSuccess) e = transform_operand(p, 2, a->V, Vp, rows, st);
    // dO' = [dO dO 0] against V' = [Vhi Vlo 0] (split), or dO zero-padded
    if (e == cudaSuccess) e = dup_rows(a->dO, dOp, rows, p->d, dk, xform(p) == XF_SPLIT_QK ? 2 : 1, st);
    if (e != cudaSuccess) return DFS_ERR_CUDA;
    q.d = dk;
    q.in_dtype = kernel_dtype(p);
    q.Q = Qp;
    q.K = Kp;
    q.V = Vp;
    q.dO = dOp;
    q.dQ = a->dQ ? grads[0] : nullptr;
    q.dK = a->dK ? grads[1] : nullptr;
    q.dV = a->dV ? grads[2] : nullptr;
  }
  const cudaError_t e = resident(p) ? launch_resident_bwd(q, st) : launch_stream_bwd(q, static_cast<float*>(kws), st);
  if (e != cudaSuccess) return DFS_ERR_CUDA;
  if (pad > 0) {
    float* outs[3] = {a->dQ, a->dK, a->dV};
    const char what[3] = {'Q', 'K', 'V'};
    for (int k = 0; k < 3; ++k)
      if (outs[k] && fold_rows(grads[k], outs[k], rows, p->d, kdim(p), fold_blocks(p, what[k]), st) != cudaSuccess)
        return DFS_ERR_CUDA;
  }
  return DFS_OK;
}

int dfs_stream_op(int op, const dfs_problem* p, const dfs_cg_params* cg, const dfs_fwd_args* fa,
                  const dfs_bwd_args* ba, int row_begin, int row_end, void* workspace, size_t workspace_bytes,
                  void* stream) {
  // the phases keep no padded copies between calls (head dims 32 and 64 only) and
  // take no position / geometry terms (their gradient shares need one GPU's rows)
  if (!dims_ok(p) || !streamed(p) || padded(p) || (p->cost_terms & (DFS_TERM_POS | DFS_TERM_GEO)))
    return dims_ok(p) ? DFS_ERR_UNSUPPORTED : DFS_ERR_INVALID_ARGUMENT;
  if (row_begin < 0 || row_end < row_begin || row_end > p->N) return DFS_ERR_INVALID_ARGUMENT;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if (op >= DFS_OP_FWD_INIT && op <= DFS_OP_FWD_OUT) {
    if ((rc = check_fwd_args(p, fa)) != DFS_OK) return rc;
    if ((rc = check_stream_fwd(p, fa, workspace, workspace_bytes)) != DFS_OK) return rc;
    return cuda_status(stream_fwd_op(op, fwd_params(p, fa), static_cast<float*>(workspace), row_begin, row_end, st));
  }
  if (op >= DFS_OP_BWD_PREP && op <= DFS_OP_BWD_DKV) {
    if ((rc = check_bwd_args(p, cg, ba)) != DFS_OK) return rc;
    if ((rc = check_stream_bwd(p, ba, workspace, workspace_bytes)) != DFS_OK) return rc;
    return cuda_status(
        stream_bwd_op(op, bwd_params(p, cg, ba, workspace), static_cast<float*>(workspace), row_begin, row_end, st));
  }
  return DFS_ERR_INVALID_ARGUMENT;
}

int dfs_stream_cg_loop_peer(const dfs_problem* p, const dfs_cg_params* cg, const dfs_bwd_args* ba, int row_begin,
                            int row_end, void* workspace, size_t workspace_bytes, const dfs_peer_set* peers,
                            size_t counter_offset, void* stream) {
  if (!dims_ok(p) || !streamed(p) || padded(p) || (p->cost_terms & (DFS_TERM_POS | DFS_TERM_GEO)))
    return dims_ok(p) ? DFS_ERR_UNSUPPORTED : DFS_ERR_INVALID_ARGUMENT;
  if (row_begin < 0 || row_end < row_begin || row_end > p->N || peers == nullptr) return DFS_ERR_INVALID_ARGUMENT;
  if (peers->npeers < 1 || peers->npeers > DFS_MAX_PEERS || peers->self < 0 || peers->self >= peers->npeers ||
      peers->ws[peers->self] != workspace || (counter_offset & 7u) != 0 || counter_offset < workspace_bytes)
    return DFS_ERR_INVALID_ARGUMENT;
  for (int k = 0; k < peers->npeers; ++k)
    if (peers->ws[k] == nullptr || (reinterpret_cast<uintptr_t>(peers->ws[k]) & 255u) != 0)
      return DFS_ERR_INVALID_ARGUMENT;
  int rc;
  if ((rc = check_bwd_args(p, cg, ba)) != DFS_OK) return rc;
  if ((rc = check_stream_bwd(p, ba, workspace, workspace_bytes)) != DFS_OK) return rc;
  PeerInfo pi{};
  pi.npeers = peers->npeers;
  pi.self = peers->self;
  for (int k = 0; k < peers->npeers; ++k) pi.ws[k] = peers->ws[k];
  return cg_loop_graph_peer(bwd_params(p, cg, ba, workspace), static_cast<float*>(workspace), row_begin, row_end, pi,
                            counter_offset, static_cast<cudaStream_t>(stream))
             ? DFS_OK
             : DFS_ERR_UNSUPPORTED;
}

int dfs_peer_alloc(size_t bytes, void** ptr, dfs_ipc_handle* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return DFS_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return DFS_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return DFS_ERR_CUDA;
  }
  static_assert(sizeof(h) == sizeof(handle->bytes), "IPC handle size");
  memcpy(handle->bytes, &h, sizeof(h));
  *ptr = p;
  return DFS_OK;
}

int dfs_peer_open(const dfs_ipc_handle* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return DFS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? DFS_OK : DFS_ERR_CUDA;
}

int dfs_peer_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? DFS_OK : DFS_ERR_CUDA; }

int dfs_peer_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? DFS_OK : DFS_ERR_CUDA; }

int dfs_stream_op_peer(int op, const dfs_problem* p, const dfs_fwd_args* fa, int row_begin, int row_end,
                       void* workspace, size_t workspace_bytes, const dfs_peer_set* peers, void* stream) {
  if (!dims_ok(p) || !streamed(p) || padded(p) || (p->cost_terms & (DFS_TERM_POS | DFS_TERM_GEO)))
    return dims_ok(p) ? DFS_ERR_UNSUPPORTED : DFS_ERR_INVALID_ARGUMENT;
  if (op < DFS_OP_FWD_INIT || op > DFS_OP_FWD_OUT || peers == nullptr) return DFS_ERR_INVALID_ARGUMENT;
  if (row_begin < 0 || row_end < row_begin || row_end > p->N) return DFS_ERR_INVALID_ARGUMENT;
  if (peers->npeers < 1 || peers->npeers > DFS_MAX_PEERS || peers->self < 0 || peers->self >= peers->npeers)
    return DFS_ERR_INVALID_ARGUMENT;
  if (peers->ws[peers->self] != workspace) return DFS_ERR_INVALID_ARGUMENT;
  for (int k = 0; k < peers->npeers; ++k)
    if (peers->ws[k] == nullptr || (reinterpret_cast<uintptr_t>(peers->ws[k]) & 255u) != 0)
      return DFS_ERR_INVALID_ARGUMENT;
  int rc;
  if ((rc = check_fwd_args(p, fa)) != DFS_OK) return rc;
  if ((rc = check_stream_fwd(p, fa, workspace, workspace_bytes)) != DFS_OK) return rc;
  if (!tile_path_ok(p->in_dtype, p->d, p->N, fa->Q, fa->K)) return DFS_ERR_UNSUPPORTED;
  PeerInfo pi{};
  pi.npeers = peers->npeers;
  pi.self = peers->self;
  for (int k = 0; k < peers->npeers; ++k) pi.ws[k] = peers->ws[k];
  pi.wait_for = peers->wait_for;
  return cuda_status(stream_fwd_op(op, fwd_params(p, fa), static_cast<float*>(workspace), row_begin, row_end,
                                   static_cast<cudaStream_t>(stream), &pi));
}

int dfs_compute_bins(int B, int N, const int32_t* chain_id, const int32_t* global_idx,
                     const uint8_t* bond_matrix, int32_t* out, void* stream) {
  if (B < 0 || N < 0) return DFS_ERR_INVALID_ARGUMENT;
  if (static_cast<size_t>(B) * N == 0) return DFS_OK;
  if (!chain_id || !global_idx || !bond_matrix || !out) return DFS_ERR_INVALID_ARGUMENT;
  return cuda_status(compute_bins_table(chain_id, global_idx, bond_matrix, B, N, out,
                                        static_cast<cudaStream_t>(stream)));
}

int dfs_selftest_mma(int which, const float* A, const float* B, float* D, int M, int N, int K, void* stream) {
  if (!A || !B || !D || which < 0 || which > 2) return DFS_ERR_INVALID_ARGUMENT;
  if (M != 64 || K <= 0 || K % 8 || N <= 0 || N > 384 || N % 32) return DFS_ERR_INVALID_ARGUMENT;
  const size_t abytes = static_cast<size_t>(M) * K * 4, bbytes = static_cast<size_t>(N) * K * 4;
  if (abytes > 98304 || bbytes > 98304) return DFS_ERR_UNSUPPORTED;
  return cuda_status(launch_selftest_mma(which, A, B, D, M, N, K, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
