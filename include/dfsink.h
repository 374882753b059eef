/*
 * dfsink.h -- C ABI of the B200 flash-Sinkhorn library (libdfsink.so).
 *
 * One (batch, head) pair is one optimal-transport problem.  For each problem
 * the library runs the log-domain (un)balanced Sinkhorn iteration of the
 * reference (vv137/deepfold-linear) on the log-kernel S = -C/eps with
 *     C_ij = -q_i.k_j/sqrt(d) + pos_weight[h, bins_ij] + w_h * dist_ij/(r_h+dist_ij),
 * (r_h = r_head[h] when given, else the problem's r_0),
 * produces the row-normalised transport output O = T_norm V (and the optional
 * centroid T_norm x), and differentiates it with the implicit-function theorem,
 * solving the adjoint system by conjugate gradient on the device.
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise; every tensor is
 *     dense row-major (C-contiguous) with the shape given beside it.  With head
 *     dim 32 or 64, Q, K, V, dO, O, dQ, dK and dV must be 16-byte aligned.
 *   - The caller owns all memory.  No entry point allocates device memory; the
 *     scratch a call needs is passed in as `workspace` (size from
 *     dfs_workspace_size).
 *   - Calls are asynchronous on `stream` (a cudaStream_t passed as void*).  The
 *     return value reports argument errors and launch errors only.  Errors found
 *     on the device (a bounded wait that gave up, non-finite potentials) are
 *     OR-ed into the int32 word `status` (device memory, may be NULL) and can be
 *     read after the stream is synchronised.
 *   - Entry points are thread-safe; concurrent calls on different streams need
 *     separate `status` words and workspaces.
 *   - Natural-log potentials (log_u, log_v) in and out, as in the reference.
 */
#ifndef DFSINK_H
#define DFSINK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFS_ABI_VERSION 2

/* return / status codes */
enum {
  DFS_OK = 0,
  DFS_ERR_INVALID_ARGUMENT = 1, /* null pointer where one is required, bad sizes   */
  DFS_ERR_UNSUPPORTED = 2,      /* shape or dtype outside the kernels' range       */
  DFS_ERR_WORKSPACE = 3,        /* workspace smaller than dfs_workspace_size       */
  DFS_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed           */
  DFS_ERR_DEVICE_TIMEOUT = 8,   /* device: a bounded wait gave up (bit in status)  */
  DFS_ERR_NUMERIC = 16,         /* device: potentials not finite after re-scaling  */
  DFS_WARN_CG_NOT_CONVERGED = 32/* device: some CG solve hit max_iter (soft)       */
};

/* element type of Q, K, V */
enum { DFS_BF16 = 0, DFS_F16 = 1, DFS_F32 = 2 };

/* where the cost comes from */
enum {
  DFS_COST_QK = 0,    /* C = -QK^T/sqrt(d) (+ position / geometry terms)          */
  DFS_COST_DENSE = 1  /* C read from a dense (B,H,N,N) fp32 tensor                */
};

typedef struct {
  int32_t B, H, N, d;     /* problems are (B, H); N points per side; head dim d  */
  int32_t in_dtype;       /* DFS_BF16 / DFS_F16 / DFS_F32 for Q, K, V             */
  int32_t cost_mode;      /* DFS_COST_QK / DFS_COST_DENSE                          */
  int32_t K_iter;         /* Sinkhorn iterations (row update then column update)  */
  int32_t check_every;    /* early-stop test period (used when threshold > 0)     */
  float lam;              /* marginal penalty; kappa = lam/(lam+eps); +inf -> 1   */
  float r_0;              /* geometry scale r_0                                    */
  float threshold;        /* L-inf early-stop tolerance on the potentials; <= 0 off */
  int32_t cost_terms;     /* DFS_TERM_* bits: the optional cost terms the calls pass */
} dfs_problem;

/* dfs_problem.cost_terms: which optional inputs the calls of this problem pass.
 * The streamed kernels (N > 384 or head dim > 32) keep per-call tables for them
 * in the workspace, so dfs_workspace_size must know; a streamed call whose
 * arguments carry a term its problem does not declare is rejected with
 * DFS_ERR_INVALID_ARGUMENT.  (0 = none, the plain -QK^T/sqrt(d) cost.) */
enum {
  DFS_TERM_POS = 1,   /* pos_weight / pos_bins: position-bin term                 */
  DFS_TERM_GEO = 2,   /* x_res with w_dist: geometry term                         */
  DFS_TERM_XRES = 4   /* x_res given (centroid; its gradient dx_res)              */
};

typedef struct {
  /* inputs */
  const void* Q;            /* (B,H,N,d) in_dtype, DFS_COST_QK                       */
  const void* K;            /* (B,H,N,d) in_dtype, DFS_COST_QK                       */
  const void* V;            /* (B,H,N,d) in_dtype, or NULL when O is NULL            */
  const float* C;           /* (B,H,N,N) dense cost, DFS_COST_DENSE                  */
  const float* x_res;       /* (B,N,3) or NULL: no geometry term, no centroid        */
  const float* pos_weight;  /* (H,68) or NULL: no position term                      */
  const int32_t* pos_bins;  /* (B,N,N) int32 in [0,68); with pos_weight, this or the */
                            /* compute_bins inputs at the end of this structure      */
  const float* eps;         /* (H,) entropic regularisation                          */
  const float* w_dist;      /* (H,) geometry weight, or NULL                         */
  const float* log_mu;      /* (B,H,N) log row marginals                             */
  const float* log_nu;      /* (B,H,N) log column marginals                          */
  const float* log_u_init;  /* (B,H,N) warm start or NULL                            */
  const float* log_v_init;  /* (B,H,N) warm start or NULL                            */
  const float* mask;        /* (B,N) 1 = real point, 0 = padding; or NULL            */
  /* outputs */
  float* O;                 /* (B,H,N,d) O = T_norm V (padded rows 0), or NULL       */
  float* x_centroid;        /* (B,H,N,3) T_norm x, or NULL                           */
  float* log_u;             /* (B,H,N) row potential, padded entries 0               */
  float* log_v;             /* (B,H,N) column potential, padded entries 0            */
  int32_t* status;          /* device int32, error bits OR-ed in; or NULL            */
  float* T_norm;            /* (B,H,N,N) row-normalised plan, or NULL (materialises  */
                            /* the plan: only for the dense compute_transport_output)*/
  const float* r_head;      /* (H,) per-head geometry scale r_h (> 0), or NULL: r_0  */
  /* position bins computed in the kernels from the inputs of compute_bins, in   */
  /* place of pos_bins (which must then be NULL): all three or none              */
  const int32_t* chain_id;     /* (B,N) chain identifier per point                 */
  const int32_t* global_idx;   /* (B,N) global residue index                       */
  const uint8_t* bond_matrix;  /* (B,N,N) covalent bond adjacency, 0 / 1           */
} dfs_fwd_args;

typedef struct {
  float rtol;               /* CG stops when ||r|| <= max(atol, rtol*||r0||)        */
  float atol;
  int32_t max_iter;         /* CG iteration cap                                      */
  int32_t reserved;
} dfs_cg_params;

typedef struct {
  /* forward inputs (same tensors as the forward call) */
  const void* Q; const void* K; const void* V;
  const float* x_res; const float* pos_weight; const int32_t* pos_bins;
  const float* eps; const float* w_dist;
  const float* log_mu; const float* log_nu;
  const float* mask;
  /* forward outputs */
  const float* log_u;       /* (B,H,N) from dfs_fwd                                  */
  const float* log_v;       /* (B,H,N) from dfs_fwd                                  */
  /* upstream gradients */
  const float* dO;          /* (B,H,N,d) dL/dO (after the gate), fp32                */
  const float* dxc;         /* (B,H,N,3) dL/dx_centroid, or NULL                     */
  /* gradients (written, not accumulated); NULL = not wanted */
  float* dQ; float* dK; float* dV;      /* (B,H,N,d) fp32                           */
  float* dlog_mu; float* dlog_nu;       /* (B,H,N)                                  */
  float* dx_res;            /* (B,N,3)                                               */
  float* dpos_weight;       /* (H,68)                                                */
  float* dw_dist;           /* (H,)                                                  */
  /* per-problem CG report, (B*H) each, or NULL */
  int32_t* cg_iters;
  float* cg_residual;
  int32_t* status;
  /* per-head geometry scale (same as the forward's) and its gradient */
  const float* r_head;      /* (H,) r_h, or NULL: r_0                                */
  float* dr_head;           /* (H,) dL/dr_h, or NULL; needs x_res and w_dist         */
  /* in place of pos_bins, as in dfs_fwd_args */
  const int32_t* chain_id; const int32_t* global_idx; const uint8_t* bond_matrix;
} dfs_bwd_args;

/* Library ABI version (DFS_ABI_VERSION of the build). */
int dfs_abi_version(void);

/* Text for a status code or an OR of device status bits. */
const char* dfs_status_string(int status);

/* Largest N accepted for head dim d (0 if d is unsupported: d > 64).  d <= 32
 * and N <= 384 run on the cluster-resident kernels (the log-kernel stays on
 * chip); larger N and 32 < d <= 64 run on the streamed kernels, which
 * recompute it tile by tile and need a workspace (dfs_workspace_size).  The
 * kernels are built for head dims 32 and 64; any other d <= 64 (e.g. the
 * reference tests' d = 8) runs on zero-padded copies of the operands made in
 * the workspace (padding adds exact zeros to every product; the logit scale
 * stays 1/sqrt(d)), and the padded columns of O and of the gradients are
 * dropped.  fp32 Q, K, V with d <= 10 are likewise rewritten in the
 * workspace as bf16 hi / lo parts along the contraction dimension
 * ([Qhi Qhi Qlo] [Khi Klo Khi]^T), so that their tensor-core products are exact
 * bf16 products (about 2^-16 relative) rather than tf32 ones (2^-11); the
 * results are folded back to head dim d. */
int dfs_max_n(int d);

/* Bytes of device workspace dfs_fwd / dfs_bwd need for problem p. */
int dfs_workspace_size(const dfs_problem* p, size_t* fwd_bytes, size_t* bwd_bytes);

/* Forward: Sinkhorn potentials and transport output.
 * Replaces FlashSinkhornFunction.forward
 *   (src/deepfold/model/kernels/sinkhorn_kernel.py:1923-2084) and, with
 *   DFS_COST_DENSE and O == NULL, the loop of sinkhorn_solve
 *   (src/deepfold/model/sinkhorn.py:17-112). */
int dfs_fwd(const dfs_problem* p, const dfs_fwd_args* a, void* workspace,
            size_t workspace_bytes, void* stream);

/* Backward: implicit-function-theorem gradients via device-side conjugate
 * gradient.  Replaces FlashSinkhornFunction.backward
 *   (src/deepfold/model/kernels/sinkhorn_kernel.py:2086-2382), whose unrolled
 *   K-step adjoint it equals at a converged fixed point. */
int dfs_bwd(const dfs_problem* p, const dfs_cg_params* cg, const dfs_bwd_args* a,
            void* workspace, size_t workspace_bytes, void* stream);

/* ---- Gradients of the dense-cost entry points ----
 * The reference differentiates sinkhorn_solve and compute_transport_output by
 * autograd through their dense tensor ops (src/deepfold/model/sinkhorn.py:
 * 17-112, 115-198).  These three calls give the same gradients as explicit
 * passes over C.  All tensors are fp32, contiguous, on the stream's device;
 * shapes are (B,H,N,N) for C, (B,H,N) for potentials and marginals, (H,) for
 * eps, (B,N) for mask (may be NULL).  N <= 65536.
 *
 * dfs_dense_iterate: iterations it_begin+1 .. it_end of sinkhorn_solve's loop
 * (sinkhorn.py:82-96, without its early stop), every iterate kept in `hist`,
 * (2K + 2) x B*H*N floats for K iterations in all: slot 2i holds log_u after
 * iteration i, slot 2i+1 log_v (slot 0 / 1 the warm start, written from
 * log_u_init / log_v_init -- zeros when NULL -- when it_begin == 0).
 * log_u / log_v receive slot it_end with padded entries zeroed
 * (sinkhorn.py:107-110).  change (1 float, may be NULL) receives the largest
 * |change| of log_u and log_v in iteration it_end over the whole batch: the
 * reference's stop test (sinkhorn.py:99-103), which the caller evaluates
 * between calls to stop where the reference stops. */
int dfs_dense_iterate(int B, int H, int N, float lam, const float* C, const float* eps, const float* log_mu,
                      const float* log_nu, const float* log_u_init, const float* log_v_init, const float* mask,
                      float* hist, int it_begin, int it_end, float* log_u, float* log_v, float* change,
                      void* work, int32_t* status, void* stream);

/* Bytes of the 16-byte aligned `work` buffer dfs_dense_iterate needs: the
 * per-CTA column partials of its one-read iterations (N <= 8192); 0 beyond,
 * where work may be NULL.  For dfs_fwd with DFS_COST_DENSE, dfs_workspace_size
 * reports the minimum (each iteration then reads C twice); a workspace of that
 * size rounded up to 256 plus these bytes makes each iteration one read of C. */
size_t dfs_dense_work_bytes(int B, int H, int N);

/* dfs_dense_solve_bwd: the adjoint of `iters` iterations recorded in hist by
 * dfs_dense_iterate.  g_log_u / g_log_v: gradients of the returned log_u /
 * log_v (NULL: zero).  Writes dC, dlog_mu, dlog_nu, dlog_u_init, dlog_v_init
 * (each may be NULL when not wanted).  scratch: dfs_dense_solve_bwd_scratch bytes, 256-byte aligned.  eps and lam
 * get no gradient (eps is a fixed per-head constant in the reference). */
/* Bytes of scratch dfs_dense_solve_bwd needs (0 for invalid sizes): about
 * (7 iters + 5) x 4 bytes per (batch, head, point), plus for N <= 8192 the
 * one-read reverse iterations' column sums, 4 N bytes for each of up to
 * max(B*H, 1184) CTAs. */
size_t dfs_dense_solve_bwd_scratch(int B, int H, int N, int iters);

int dfs_dense_solve_bwd(int B, int H, int N, int iters, float lam, const float* C, const float* eps,
                        const float* log_mu, const float* log_nu, const float* mask, const float* hist,
                        const float* g_log_u, const float* g_log_v, float* dC, float* dlog_mu, float* dlog_nu,
                        float* dlog_u_init, float* dlog_v_init, float* scratch, void* stream);

/* dfs_dense_transport_bwd: the softmax backward of compute_transport_output's
 * T_norm (sinkhorn.py:163-176).  dT holds dL/dT_norm (B,H,N,N) on entry -- the
 * caller forms it from the gradients of o, x_centroid and T_norm (plain
 * batched products with V and x_res) -- and dL/dC on return; dlog_v
 * (may be NULL) receives dL/dlog_v.  dL/dlog_u is zero: log_u cancels in
 * score - rowmax. */
int dfs_dense_transport_bwd(int B, int H, int N, const float* T_norm, float* dT, const float* eps, float* dlog_v,
                            void* stream);

/* Position bins of the reference's compute_bins (src/deepfold/model/
 * position_encoding.py:7-52) into a (B,N,N) int32 table `out`:
 *   same chain, no bond: clamp(gidx_i - gidx_j, -32, 32) + 32;  other chain, no
 *   bond: 65;  same chain, bond: 66;  other chain, bond: 67.
 * chain_id, global_idx (B,N) int32; bond_matrix (B,N,N) uint8 (0 / 1).  The
 * forward and backward can evaluate the same per pair instead (the chain_id /
 * global_idx / bond_matrix arguments), without the N x N int32 table. */
int dfs_compute_bins(int B, int N, const int32_t* chain_id, const int32_t* global_idx,
                     const uint8_t* bond_matrix, int32_t* out, void* stream);

/* ---------------------------------------------------------------------------
 * Row-sharded runs (several GPUs per problem).  dfs_stream_op runs one phase of
 * the streamed forward or backward on a range of rows [row_begin, row_end) (for
 * the column phases: of columns).  dfs_fwd / dfs_bwd on one GPU are exactly
 * these phases over all rows, in the order below; a run sharded over G GPUs
 * gives each GPU one range and all-gathers the workspace vectors a range phase
 * produced (listed per phase) before the next phase.  Every GPU holds Q, K, V,
 * dO and the marginals in full.  The workspace is dfs_workspace_size's
 * fwd_bytes (forward phases) or bwd_bytes (backward phases); its vectors are
 * (B*H, N) fp32 slots at slot * B*H*N floats (numbers below).
 *
 * Forward: FWD_INIT; K_iter x { FWD_ROWS (gather slot F and log_u),
 *          FWD_COLS (gather slot G and log_v) }; FWD_OUT (O, x_centroid rows).
 * Backward: BWD_PREP; BWD_ROWSTATS (gather M, R, D); BWD_ROWDERIVE;
 *          BWD_COLSTATS (gather C, GV; writes the dV rows where the TMA-staged
 *          passes run: d = 32 or 64, N >= 128, N % 4 == 0); BWD_SETUP; BWD_PT_T (gather S);
 *          BWD_CGINIT; (max_iter + 1) x { BWD_P_U (gather T); BWD_PT_T (gather S);
 *          BWD_CGSTEP_FIRST the first time, BWD_CGSTEP after };
 *          BWD_P_X (gather S); BWD_FINAL; BWD_DQ (dQ rows); BWD_DKV (dK rows, and
 *          dV rows where BWD_COLSTATS did not write them).
 * --------------------------------------------------------------------------- */
enum {
  DFS_OP_FWD_INIT = 0, DFS_OP_FWD_ROWS = 1, DFS_OP_FWD_COLS = 2, DFS_OP_FWD_OUT = 3,
  DFS_OP_BWD_PREP = 10, DFS_OP_BWD_ROWSTATS = 11, DFS_OP_BWD_ROWDERIVE = 12, DFS_OP_BWD_COLSTATS = 13,
  DFS_OP_BWD_SETUP = 14, DFS_OP_BWD_PT_T = 15, DFS_OP_BWD_CGINIT = 16, DFS_OP_BWD_P_U = 17,
  DFS_OP_BWD_CGSTEP_FIRST = 18, DFS_OP_BWD_CGSTEP = 19, DFS_OP_BWD_P_X = 20, DFS_OP_BWD_FINAL = 21,
  DFS_OP_BWD_DQ = 22, DFS_OP_BWD_DKV = 23
};
/* workspace slots gathered between phases */
enum { DFS_WS_FWD_F = 0, DFS_WS_FWD_G = 1 };
enum {
  DFS_WS_BWD_F = 0, DFS_WS_BWD_G = 1, DFS_WS_BWD_M = 2, DFS_WS_BWD_R = 3, DFS_WS_BWD_D = 4,
  DFS_WS_BWD_C = 7, DFS_WS_BWD_GV = 8, DFS_WS_BWD_T = 19, DFS_WS_BWD_S = 20,
  /* after the DFS_WS_BWD_NSLOTS vector slots come DFS_WS_BWD_NSCALARS floats per
   * problem, then one int32 CG stop flag per problem (nonzero once that
   * problem's solve has stopped; identical on every GPU of a sharded run) */
  DFS_WS_BWD_NSLOTS = 22, DFS_WS_BWD_NSCALARS = 8
};

/* One phase of the streamed path on rows (columns) [row_begin, row_end).
 * Forward phases read `fa` (and ignore `cg`, `ba`), backward phases `cg` and
 * `ba`.  Any N the streamed kernels accept, head dims 32 and 64 only (the phases
 * keep no padded copies between calls).  New for
 * multi-GPU row sharding of long sequences; the reference has no sharded path. */
int dfs_stream_op(int op, const dfs_problem* p, const dfs_cg_params* cg, const dfs_fwd_args* fa,
                  const dfs_bwd_args* ba, int row_begin, int row_end, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Size of the library's fixed device scratch used by dfs_fwd_static: 16 MiB.
 * dfs_workspace_size's fwd_bytes is the authority on what a problem needs: the
 * streamed forward takes 112 + 12 d bytes per (batch, head, point) -- potentials
 * and row statistics, fp32 operand copies, the column-split partials -- plus
 * 4 bytes per block of 128 rows and under 1 KB fixed, i.e. B*H*N up to about
 * 19,000 points at d = 64 or 33,000 at d = 32; head dims other than 32 and 64
 * add their zero-padded copies.  Cluster-resident problems (N <= 384, d = 32)
 * need none; dense-cost problems need 8 bytes per (batch, head, point). */
#define DFS_STATIC_SCRATCH_BYTES (16u << 20)

/* Forward for callers that cannot allocate device memory.  No counterpart in
 * the reference.  Same arguments and results as dfs_fwd, but the workspace the
 * streamed kernels need is a fixed DFS_STATIC_SCRATCH_BYTES array of device
 * memory that the library itself holds (on every GPU that loads it, until the
 * process exits), so the call allocates nothing.  It serves callers that only
 * receive their buffers from another runtime or framework and have no
 * allocator to ask for a workspace.
 *   - Problems whose forward workspace exceeds DFS_STATIC_SCRATCH_BYTES are
 *     rejected with DFS_ERR_WORKSPACE before anything runs.
 *   - The device that owns `stream` must be current.  The first call on a
 *     device looks up the scratch's device address once (cudaGetSymbolAddress),
 *     so make that first call before any stream capture on the device.
 *   - All calls on a device share the one scratch: calls whose work overlaps on
 *     the GPU (different streams with no ordering between them) race and must
 *     be serialised by the caller.  Nothing in it needs to start at zero. */
int dfs_fwd_static(const dfs_problem* p, const dfs_fwd_args* a, void* stream);

/* ---------------------------------------------------------------------------
 * Peer exchange for row-sharded forwards (one process per GPU, GPUs linked by
 * NVLink / NVSwitch).  Instead of gathering the potential slices with a
 * collective after every half-iteration, the half-update kernel of each GPU
 * stores its new potentials straight into the forward workspace of every GPU
 * of the run and raises an arrival counter there; the next phase waits on its
 * own counter before it reads.  The workspaces are device buffers shared
 * between the processes through CUDA IPC: each process allocates its own with
 * dfs_peer_alloc (zero-filled), the processes exchange the 64-byte handles
 * (an all-gather), and each maps the others' with dfs_peer_open.  New for
 * multi-GPU row sharding; the reference has no sharded path.
 * --------------------------------------------------------------------------- */
#define DFS_MAX_PEERS 8
typedef struct { unsigned char bytes[64]; } dfs_ipc_handle;

int dfs_peer_alloc(size_t bytes, void** ptr, dfs_ipc_handle* handle);
int dfs_peer_open(const dfs_ipc_handle* handle, void** ptr);
int dfs_peer_close(void* ptr);  /* unmaps a buffer mapped by dfs_peer_open */
int dfs_peer_free(void* ptr);   /* frees a buffer from dfs_peer_alloc */

typedef struct {
  int32_t npeers;           /* GPUs in the run (<= DFS_MAX_PEERS), this one included */
  int32_t self;             /* this GPU's index in ws[] */
  void* ws[DFS_MAX_PEERS];  /* every GPU's forward workspace (own one included), same problem */
  uint64_t wait_for;        /* arrivals the phase waits for on its own counter before reading */
} dfs_peer_set;

/* One forward phase (DFS_OP_FWD_*) with peer exchange.  FWD_INIT also raises
 * every GPU's counter once (a later call's stores then wait until this call
 * has started everywhere, i.e. the previous call has finished); FWD_ROWS and
 * FWD_COLS store the new potentials of rows [row_begin, row_end) into every
 * workspace and raise every counter once per block of 128 rows of each
 * problem; FWD_ROWS, FWD_COLS and FWD_OUT first wait until their own counter
 * reaches peers->wait_for (bounded: a timeout sets DFS_ERR_DEVICE_TIMEOUT in
 * the status word).  Counters accumulate for the life of the workspace, so all
 * GPUs must pass the same cumulative wait_for sequence.  Only where the
 * TMA-staged passes run (d = 64, or fp32 with d = 32; N >= 128; 16-byte aligned
 * operands); elsewhere DFS_ERR_UNSUPPORTED. */
int dfs_stream_op_peer(int op, const dfs_problem* p, const dfs_fwd_args* fa, int row_begin, int row_end,
                       void* workspace, size_t workspace_bytes, const dfs_peer_set* peers, void* stream);

/* Peer-memory gather of row slices, for the phases of a row-sharded backward
 * (or any buffer every GPU of the run holds at the same layout, e.g. one
 * shared through dfs_peer_alloc / dfs_peer_open; peers->ws[k] are the
 * buffers' bases, 256-byte aligned).  The slot at byte slot_offset holds P
 * problems x N rows x `width` floats; this GPU's rows [row_begin, row_end) of
 * every problem are stored into every other GPU's buffer, then every GPU's
 * arrival counter (a uint64 at byte counter_offset of its buffer; the 8 bytes
 * after it are the push's completion counter, zero between calls, then the
 * expected count; 24 bytes in all, zero at allocation) is raised
 * once; finally the stream waits until this GPU's own counter reaches its
 * expected count plus npeers (bounded: a timeout sets DFS_ERR_DEVICE_TIMEOUT in
 * *status).  The expected count is a uint64 at counter_offset + 16 that the
 * wait itself advances, so all GPUs must run the same gathers on a buffer in
 * the same order; peers->wait_for is not used.  Replaces, for the row-sharded path, the
 * all-gather collective between phases; the reference has no sharded path. */
int dfs_peer_gather_rows(const dfs_peer_set* peers, size_t slot_offset, int P, int N, int width, int row_begin,
                         int row_end, size_t counter_offset, int32_t* status, void* stream);

/* The CG rounds after the first (what the loop of DFS_OP_BWD_P_U, the gather
 * of slot DFS_WS_BWD_T, DFS_OP_BWD_PT_T, the gather of DFS_WS_BWD_S and
 * DFS_OP_BWD_CGSTEP would do, up to cg->max_iter rounds) for one GPU of a
 * row-sharded backward, as one CUDA graph launched on `stream` whose WHILE loop
 * stops on the device once every problem's solve has stopped: the host neither
 * waits nor reads flags.  The backward workspace must be the buffer every GPU
 * shares (peers->ws[self] == workspace) with the dfs_peer_gather_rows counters
 * at counter_offset (>= workspace_bytes); every GPU calls it at the same point.
 * DFS_ERR_UNSUPPORTED when no such graph can be built (inside the caller's own
 * stream capture, or a runtime without conditional graph nodes): the caller
 * then runs the rounds phase by phase.  New for multi-GPU row sharding. */
int dfs_stream_cg_loop_peer(const dfs_problem* p, const dfs_cg_params* cg, const dfs_bwd_args* ba, int row_begin,
                            int row_end, void* workspace, size_t workspace_bytes, const dfs_peer_set* peers,
                            size_t counter_offset, void* stream);

/* TEST-ONLY entry point, not part of the operator surface: runs one of the
 * three tcgen05 MMA operand layouts the kernels use on caller-provided data
 * (D = A B^T, M = 64), so the test suite can check each layout against a
 * plain matrix product.  No counterpart in the reference. */
int dfs_selftest_mma(int which, const float* A, const float* B, float* D,
                     int M, int N, int K, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DFSINK_H */
