// dfs_torch.cpp -- native autograd glue between PyTorch and libdfsink.
//
// FlashSinkhornFn is the autograd function behind deepfold's flash_sinkhorn
// (reference: FlashSinkhornFunction, src/deepfold/model/kernels/
// sinkhorn_kernel.py:1923-2382); BalancedTransportFn the one behind
// balanced_sinkhorn_transport(_dual) (flash_sinkhorn_transport.py:287-545).  Its forward and backward validate shapes,
// allocate outputs with the caching allocator and call dfs_fwd / dfs_bwd of the
// C ABI on the current stream; nothing here computes.  Doing this in C++
// rather than Python keeps the per-call host cost to a few allocations, so the
// GPU, not the interpreter, bounds a training step.
//
// Errors the kernels find on the device (a bounded wait that gave up,
// non-finite potentials, a CG solve that hit its iteration cap) are OR-ed into
// a sticky status word per device.  Reading it at once would synchronise every
// call; instead the word is read back asynchronously and picked up by the next
// call, and the bits go to Python through take_status, where the op raises
// RuntimeError for an error bit and warns for DFS_WARN_CG_NOT_CONVERGED (see
// DeviceStatus below).
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <limits>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "dfsink.h"

namespace {

using at::Tensor;
using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

// Errors are thrown as std::runtime_error (pybind11 raises RuntimeError) with
// the message built here: a TORCH_CHECK whose message formats a number crashed
// the process in this torch build, inside any extension.
[[noreturn]] void fail(const std::string& msg) { throw std::runtime_error(msg); }
void require(bool ok, const char* msg) {
  if (!ok) fail(msg);
}

void check_rc(int rc, const char* what) {
  if (rc != DFS_OK)
    fail(std::string(what) + " failed: " + dfs_status_string(rc) + " (code " + std::to_string(rc) + ")");
}

int dtype_code(at::ScalarType t) {
  if (t == at::kBFloat16) return DFS_BF16;
  if (t == at::kHalf) return DFS_F16;
  return DFS_F32;
}

Tensor f32(const c10::optional<Tensor>& t) {
  if (!t.has_value() || !t->defined()) return Tensor();
  return t->contiguous().to(at::kFloat);
}

template <typename T>
T* ptr_or_null(const Tensor& t) {
  return t.defined() ? static_cast<T*>(t.data_ptr()) : nullptr;
}

// Most recent backward's per-problem CG report (device tensors).  Held in a
// heap object that is never destroyed: tensors and CUDA events must not be
// torn down by static destructors after the CUDA runtime has shut down.
std::vector<Tensor>& last_report() {
  static auto* r = new std::vector<Tensor>();
  return *r;
}

// Makes a device current for a scope and restores the previous one, with the
// plain runtime calls.
struct DeviceSwitch {
  int prev = -1;
  explicit DeviceSwitch(const at::Device& dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev.index()) cudaSetDevice(dev.index());
  }
  ~DeviceSwitch() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
  DeviceSwitch(const DeviceSwitch&) = delete;
  DeviceSwitch& operator=(const DeviceSwitch&) = delete;
};

// ---------------------------------------------------------------- device status
// One sticky int32 status word per device: every forward and backward call
// hands it to the library, whose kernels OR their error bits into it.  After a
// call, if no read-back is in flight, the word is copied to pinned host memory
// on the call's stream and an event recorded; the next call (or check_status)
// reads the copy once its event has completed, and on a nonzero value clears
// the word and raises (errors) or warns (DFS_WARN_CG_NOT_CONVERGED).  So a
// call costs at most one 4-byte copy and no synchronisation.  All of it lives
// in never-destroyed heap objects (see last_report).
constexpr int kMaxDevices = 64;
struct DeviceStatus {
  Tensor word;            // (1,) int32 on the device, sticky
  int32_t* mirror = nullptr;  // pinned host copy
  cudaEvent_t copied = nullptr;
  bool in_flight = false;
};
std::mutex g_status_mu;
DeviceStatus* g_status[kMaxDevices] = {};

DeviceStatus& device_status(const at::Device& dev) {
  const int i = dev.index();
  require(i >= 0 && i < kMaxDevices, "device index out of range");
  if (g_status[i] == nullptr) {
    auto* ds = new DeviceStatus();
    ds->word = at::zeros({1}, at::TensorOptions().device(dev).dtype(at::kInt));
    require(cudaHostAlloc(reinterpret_cast<void**>(&ds->mirror), sizeof(int32_t), cudaHostAllocDefault) ==
                cudaSuccess, "cudaHostAlloc failed");
    *ds->mirror = 0;
    require(cudaEventCreateWithFlags(&ds->copied, cudaEventDisableTiming) == cudaSuccess, "cudaEventCreate failed");
    g_status[i] = ds;
  }
  return *g_status[i];
}

// After a call on `stream` (the current device's): start a read-back of the
// word unless one is in flight.  Caller holds g_status_mu.
void start_readback(DeviceStatus& ds, cudaStream_t stream) {
  if (ds.in_flight) return;
  if (cudaMemcpyAsync(ds.mirror, ds.word.data_ptr<int32_t>(), sizeof(int32_t), cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaEventRecord(ds.copied, stream) != cudaSuccess)
    return;
  ds.in_flight = true;
}

// Read the status word of a device (wait: its value once all work on the
// device has finished, read synchronously; otherwise the last completed
// read-back, or 0).  A nonzero value clears the word.  Returns the bits.
int poll_device_status(const at::Device& dev, bool wait) {
  std::lock_guard<std::mutex> lock(g_status_mu);
  DeviceStatus& ds = device_status(dev);
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  if (wait) {
    // an in-flight read-back may predate the latest calls (a call starts none
    // while one is in flight): drain the device and read the word itself
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(ds.mirror, ds.word.data_ptr<int32_t>(), sizeof(int32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
      return 0;
  } else if (!ds.in_flight || cudaEventQuery(ds.copied) != cudaSuccess) {
    return 0;
  }
  ds.in_flight = false;
  const int v = *ds.mirror;
  if (v != 0) {
    *ds.mirror = 0;
    cudaMemsetAsync(ds.word.data_ptr<int32_t>(), 0, sizeof(int32_t), stream);
  }
  return v;
}

// Status bits picked up by the checks inside calls (the backward runs on
// autograd's worker threads, away from Python), handed to Python by
// take_status: the op's Python wrapper raises for error bits and warns for
// DFS_WARN_CG_NOT_CONVERGED after each call, so no exception is thrown from
// here.
std::atomic<int> g_seen{0};

// The check at the start of every forward and backward.
void check_device_status(const at::Device& dev) { g_seen.fetch_or(poll_device_status(dev, false)); }

// For Python: the status bits of the current device (see poll_device_status)
// together with the bits kept by the checks inside calls; all are cleared.
int take_status(bool wait) {
  const int v = poll_device_status(at::Device(at::kCUDA, c10::cuda::current_device()), wait);
  return v | g_seen.exchange(0);
}

// DFS_TERM_* bits of the optional inputs a call passes (the streamed kernels
// size their workspace by them)
int32_t cost_terms_of(const Tensor& pw, const Tensor& pb, const Tensor& xr, const Tensor& wd,
                      const Tensor& chain = Tensor()) {
  int32_t t = 0;
  if (pw.defined() && (pb.defined() || chain.defined())) t |= DFS_TERM_POS;
  if (xr.defined() && wd.defined()) t |= DFS_TERM_GEO;
  if (xr.defined()) t |= DFS_TERM_XRES;
  return t;
}

struct FlashSinkhornFn : public torch::autograd::Function<FlashSinkhornFn> {
  // Arguments (positions in the gradient list backward returns): 0 Q, 1 K, 2 V,
  // 3 x_res, 4 pos_weight, 5 pos_bins, 6 eps, 7 w_dist, 8 log_mu, 9 log_nu,
  // 10 log_u_init, 11 log_v_init, 12 mask, 13 K_iter, 14 lam, 15 r_0, 16 cg_rtol,
  // 17 cg_atol, 18 cg_max_iter, 19 chain_id, 20 global_idx, 21 bond_matrix (the
  // inputs of compute_bins, in place of pos_bins).  needs_input_grad counts only
  // the tensors that were passed (absent optionals are no autograd edge), so the
  // forward records each argument's edge index.
  static variable_list forward(AutogradContext* ctx, Tensor Q, Tensor K, Tensor V, c10::optional<Tensor> x_res,
                               c10::optional<Tensor> pos_weight, c10::optional<Tensor> pos_bins, Tensor eps,
                               c10::optional<Tensor> w_dist, Tensor log_mu, Tensor log_nu,
                               c10::optional<Tensor> log_u_init, c10::optional<Tensor> log_v_init,
                               c10::optional<Tensor> mask, int64_t K_iter, double lam, double r_0,
                               double cg_rtol, double cg_atol, int64_t cg_max_iter,
                               c10::optional<Tensor> chain_id, c10::optional<Tensor> global_idx,
                               c10::optional<Tensor> bond_matrix) {
    require(Q.is_cuda() && K.is_cuda() && V.is_cuda(),
                "deepfold B200 Sinkhorn ops run on CUDA tensors only (no CPU path)");
    require(Q.dim() == 4 && K.sizes() == Q.sizes() && V.sizes() == Q.sizes(),
                "Q, K, V must share the shape (B, H, N, d)");
    require(K.device() == Q.device() && V.device() == Q.device(), "Q, K, V must be on one device");
    const int64_t B = Q.size(0), H = Q.size(1), N = Q.size(2), d = Q.size(3);
    if (N > dfs_max_n(static_cast<int>(d)))
      fail("N=" + std::to_string(N) + ", d=" + std::to_string(d) +
           " is outside the kernels' range (head dim <= 64, N <= " + std::to_string(dfs_max_n(static_cast<int>(d))) +
           ")");
    const DeviceSwitch guard(Q.device());  // launches, attributes and streams of Q's device
    check_device_status(Q.device());
    const auto st = Q.scalar_type();
    const auto cdt = (st == at::kBFloat16 || st == at::kHalf || st == at::kFloat) ? st : at::kFloat;
    const Tensor Qc = Q.contiguous().to(cdt), Kc = K.contiguous().to(cdt), Vc = V.contiguous().to(cdt);
    const Tensor xr = f32(x_res), pw = f32(pos_weight);
    Tensor pb, ch, gx, bd;
    if (pw.defined() && pos_bins.has_value() && pos_bins->defined()) pb = pos_bins->contiguous().to(at::kInt);
    const bool bins_inputs = chain_id.has_value() && chain_id->defined();
    if (pw.defined() && !pb.defined() && bins_inputs) {
      require(global_idx.has_value() && global_idx->defined() && bond_matrix.has_value() && bond_matrix->defined(),
              "chain_id, global_idx and bond_matrix are given together");
      require(chain_id->dim() == 2 && chain_id->size(0) == B && chain_id->size(1) == N &&
                  global_idx->sizes() == chain_id->sizes() && bond_matrix->dim() == 3 &&
                  bond_matrix->size(0) == B && bond_matrix->size(1) == N && bond_matrix->size(2) == N,
              "chain_id, global_idx must be (B, N) and bond_matrix (B, N, N)");
      ch = chain_id->contiguous().to(at::kInt);
      gx = global_idx->contiguous().to(at::kInt);
      bd = bond_matrix->contiguous().to(at::kByte);
    }
    const Tensor epsc = eps.contiguous().to(at::kFloat), wd = f32(w_dist);
    const Tensor lmu = log_mu.contiguous().to(at::kFloat), lnu = log_nu.contiguous().to(at::kFloat);
    const Tensor lui = f32(log_u_init), lvi = f32(log_v_init), mk = f32(mask);
    const auto fo = Q.options().dtype(at::kFloat);
    Tensor O = at::empty({B, H, N, d}, fo);
    Tensor xc = xr.defined() ? at::empty({B, H, N, 3}, fo) : Tensor();
    const Tensor pot = at::empty({2, B, H, N}, fo);
    Tensor lu = pot[0], lv = pot[1];
    Tensor status = device_status(Q.device()).word;

    dfs_problem prob{};
    prob.B = static_cast<int32_t>(B);
    prob.H = static_cast<int32_t>(H);
    prob.N = static_cast<int32_t>(N);
    prob.d = static_cast<int32_t>(d);
    prob.in_dtype = dtype_code(cdt);
    prob.cost_mode = DFS_COST_QK;
    prob.K_iter = static_cast<int32_t>(K_iter);
    prob.check_every = 2;
    prob.lam = static_cast<float>(lam);
    prob.r_0 = static_cast<float>(r_0);
    prob.cost_terms = cost_terms_of(pw, pb, xr, wd, ch);
    ctx->saved_data["cost_terms"] = static_cast<int64_t>(prob.cost_terms);
    dfs_fwd_args a{};
    a.Q = Qc.data_ptr();
    a.K = Kc.data_ptr();
    a.V = Vc.data_ptr();
    a.x_res = ptr_or_null<const float>(xr);
    a.pos_weight = ptr_or_null<const float>(pw);
    a.pos_bins = ptr_or_null<const int32_t>(pb);
    a.eps = epsc.data_ptr<float>();
    a.w_dist = ptr_or_null<const float>(wd);
    a.log_mu = lmu.data_ptr<float>();
    a.log_nu = lnu.data_ptr<float>();
    a.log_u_init = ptr_or_null<const float>(lui);
    a.log_v_init = ptr_or_null<const float>(lvi);
    a.mask = ptr_or_null<const float>(mk);
    a.chain_id = ptr_or_null<const int32_t>(ch);
    a.global_idx = ptr_or_null<const int32_t>(gx);
    a.bond_matrix = ptr_or_null<const uint8_t>(bd);
    a.O = O.data_ptr<float>();
    a.x_centroid = ptr_or_null<float>(xc);
    a.log_u = lu.data_ptr<float>();
    a.log_v = lv.data_ptr<float>();
    a.status = status.data_ptr<int32_t>();
    size_t fwd_ws = 0, bwd_ws = 0;  // the streamed path (large N, d = 64) needs scratch
    check_rc(dfs_workspace_size(&prob, &fwd_ws, &bwd_ws), "dfs_workspace_size");
    Tensor ws = fwd_ws ? at::empty({static_cast<int64_t>((fwd_ws + 3) / 4)}, fo) : Tensor();
    const at::cuda::CUDAStream cstream = at::cuda::getCurrentCUDAStream(Q.device().index());
    check_rc(dfs_fwd(&prob, &a, ws.defined() ? ws.data_ptr() : nullptr, fwd_ws, cstream.stream()), "dfs_fwd");
    {
      std::lock_guard<std::mutex> lock(g_status_mu);
      start_readback(device_status(Q.device()), cstream.stream());
    }

    ctx->save_for_backward({Qc, Kc, Vc, xr, pw, pb, epsc, wd, lmu, lnu, mk, lu, lv, ch, gx, bd});
    ctx->saved_data["K_iter"] = K_iter;
    ctx->saved_data["lam"] = lam;
    ctx->saved_data["r_0"] = r_0;
    ctx->saved_data["cg_rtol"] = cg_rtol;
    ctx->saved_data["cg_atol"] = cg_atol;
    ctx->saved_data["cg_max_iter"] = cg_max_iter;
    ctx->saved_data["fwd_status"] = status;
    ctx->saved_data["in_dtype"] = static_cast<int64_t>(Q.scalar_type());
    auto dtype_of = [](const c10::optional<Tensor>& t) {
      return static_cast<int64_t>(t.has_value() && t->defined() ? t->scalar_type() : at::kFloat);
    };
    ctx->saved_data["x_dtype"] = dtype_of(x_res);
    ctx->saved_data["pw_dtype"] = dtype_of(pos_weight);
    ctx->saved_data["wd_dtype"] = dtype_of(w_dist);
    int64_t edge = 3;  // Q, K, V are edges 0..2
    auto next_edge = [&](bool present) -> int64_t { return present ? edge++ : -1; };
    ctx->saved_data["e_x"] = next_edge(x_res.has_value());
    ctx->saved_data["e_pw"] = next_edge(pos_weight.has_value());
    next_edge(pos_bins.has_value());
    next_edge(true);  // eps
    ctx->saved_data["e_wd"] = next_edge(w_dist.has_value());
    ctx->saved_data["e_mu"] = next_edge(true);
    ctx->saved_data["e_nu"] = next_edge(true);
    ctx->mark_non_differentiable({lu, lv});
    // no zero tensors for the outputs whose gradient is absent (the potentials):
    // the backward takes undefined gradients as zero
    ctx->set_materialize_grads(false);
    // autograd outputs must be defined tensors: without x_res there is no centroid
    if (xc.defined()) return {O, xc, lu, lv};
    return {O, lu, lv};
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    const DeviceSwitch guard(saved[0].device());
    check_device_status(saved[0].device());
    const Tensor &Qc = saved[0], &Kc = saved[1], &Vc = saved[2], &xr = saved[3], &pw = saved[4],
                 &pb = saved[5], &epsc = saved[6], &wd = saved[7], &lmu = saved[8], &lnu = saved[9],
                 &mk = saved[10], &lu = saved[11], &lv = saved[12], &ch = saved[13], &gx = saved[14],
                 &bd = saved[15];
    auto needs = [&](const char* key) {
      const int64_t e = ctx->saved_data[key].toInt();
      return e >= 0 && ctx->needs_input_grad(static_cast<size_t>(e));
    };
    const int64_t B = Qc.size(0), H = Qc.size(1), N = Qc.size(2), d = Qc.size(3);
    const auto fo = Qc.options().dtype(at::kFloat);
    const Tensor dOc = grads[0].defined() ? grads[0].contiguous().to(at::kFloat) : at::zeros({B, H, N, d}, fo);
    const Tensor dxc = (xr.defined() && grads[1].defined()) ? grads[1].contiguous().to(at::kFloat) : Tensor();
    // dQ, dK, dV in one buffer: one allocation, and one cast to the inputs' dtype
    const Tensor gbuf = at::empty({3, B, H, N, d}, fo);
    const bool want_q = ctx->needs_input_grad(0), want_k = ctx->needs_input_grad(1), want_v = ctx->needs_input_grad(2);
    float* const g0 = gbuf.data_ptr<float>();
    const int64_t nd = B * H * N * d;
    Tensor dmu = needs("e_mu") ? at::empty({B, H, N}, fo) : Tensor();
    Tensor dnu = needs("e_nu") ? at::empty({B, H, N}, fo) : Tensor();
    // gradients of the shared cost parameters (reference: sinkhorn_kernel.py:2366-2382)
    Tensor dxr = (needs("e_x") && xr.defined()) ? at::empty({B, N, 3}, fo) : Tensor();
    Tensor dpw = (needs("e_pw") && pw.defined() && (pb.defined() || ch.defined())) ? at::empty({H, 68}, fo)
                                                                                   : Tensor();
    Tensor dwd = (needs("e_wd") && wd.defined() && xr.defined()) ? at::empty({H}, fo) : Tensor();
    // CG report: iterations (int32) then residuals (fp32) per problem
    const Tensor rep = at::empty({2, B * H}, Qc.options().dtype(at::kInt));
    Tensor status = device_status(Qc.device()).word;

    dfs_problem prob{};
    prob.B = static_cast<int32_t>(B);
    prob.H = static_cast<int32_t>(H);
    prob.N = static_cast<int32_t>(N);
    prob.d = static_cast<int32_t>(d);
    prob.in_dtype = dtype_code(Qc.scalar_type());
    prob.cost_mode = DFS_COST_QK;
    prob.K_iter = static_cast<int32_t>(ctx->saved_data["K_iter"].toInt());
    prob.check_every = 2;
    prob.lam = static_cast<float>(ctx->saved_data["lam"].toDouble());
    prob.r_0 = static_cast<float>(ctx->saved_data["r_0"].toDouble());
    prob.cost_terms = static_cast<int32_t>(ctx->saved_data["cost_terms"].toInt());
    dfs_cg_params cg{};
    cg.rtol = static_cast<float>(ctx->saved_data["cg_rtol"].toDouble());
    cg.atol = static_cast<float>(ctx->saved_data["cg_atol"].toDouble());
    cg.max_iter = static_cast<int32_t>(ctx->saved_data["cg_max_iter"].toInt());
    dfs_bwd_args a{};
    a.Q = Qc.data_ptr();
    a.K = Kc.data_ptr();
    a.V = Vc.data_ptr();
    a.x_res = ptr_or_null<const float>(xr);
    a.pos_weight = ptr_or_null<const float>(pw);
    a.pos_bins = ptr_or_null<const int32_t>(pb);
    a.eps = epsc.data_ptr<float>();
    a.w_dist = ptr_or_null<const float>(wd);
    a.log_mu = lmu.data_ptr<float>();
    a.log_nu = lnu.data_ptr<float>();
    a.mask = ptr_or_null<const float>(mk);
    a.chain_id = ptr_or_null<const int32_t>(ch);
    a.global_idx = ptr_or_null<const int32_t>(gx);
    a.bond_matrix = ptr_or_null<const uint8_t>(bd);
    a.log_u = lu.data_ptr<float>();
    a.log_v = lv.data_ptr<float>();
    a.dO = dOc.data_ptr<float>();
    a.dxc = ptr_or_null<const float>(dxc);
    a.dQ = want_q ? g0 : nullptr;
    a.dK = want_k ? g0 + nd : nullptr;
    a.dV = want_v ? g0 + 2 * nd : nullptr;
    a.dlog_mu = ptr_or_null<float>(dmu);
    a.dlog_nu = ptr_or_null<float>(dnu);
    a.dx_res = ptr_or_null<float>(dxr);
    a.dpos_weight = ptr_or_null<float>(dpw);
    a.dw_dist = ptr_or_null<float>(dwd);
    a.cg_iters = rep.data_ptr<int32_t>();
    a.cg_residual = reinterpret_cast<float*>(rep.data_ptr<int32_t>() + B * H);
    a.status = status.data_ptr<int32_t>();
    size_t fwd_ws = 0, bwd_ws = 0;
    check_rc(dfs_workspace_size(&prob, &fwd_ws, &bwd_ws), "dfs_workspace_size");
    Tensor ws = bwd_ws ? at::empty({static_cast<int64_t>((bwd_ws + 3) / 4)}, fo) : Tensor();
    const at::cuda::CUDAStream cstream = at::cuda::getCurrentCUDAStream(Qc.device().index());
    check_rc(dfs_bwd(&prob, &cg, &a, ws.defined() ? ws.data_ptr() : nullptr, bwd_ws, cstream.stream()), "dfs_bwd");
    {
      std::lock_guard<std::mutex> lock(g_status_mu);
      start_readback(device_status(Qc.device()), cstream.stream());
    }
    last_report() = {rep, status, ctx->saved_data["fwd_status"].toTensor()};

    // gradients in the dtype of the forward's inputs (one cast for the three)
    const auto in_dt = static_cast<at::ScalarType>(ctx->saved_data["in_dtype"].toInt());
    const Tensor gcast = gbuf.to(in_dt);
    variable_list out(22);
    out[0] = want_q ? gcast[0] : Tensor();
    out[1] = want_k ? gcast[1] : Tensor();
    out[2] = want_v ? gcast[2] : Tensor();
    out[3] = dxr.defined() ? dxr.to(static_cast<at::ScalarType>(ctx->saved_data["x_dtype"].toInt())) : dxr;
    out[4] = dpw.defined() ? dpw.to(static_cast<at::ScalarType>(ctx->saved_data["pw_dtype"].toInt())) : dpw;
    out[7] = dwd.defined() ? dwd.to(static_cast<at::ScalarType>(ctx->saved_data["wd_dtype"].toInt())) : dwd;
    out[8] = dmu;
    out[9] = dnu;
    return out;
  }
};

// Balanced Sinkhorn transport of the reference's trunk block
// (BalancedSinkhornFn / BalancedSinkhornDualFn, src/deepfold/model/kernels/
// flash_sinkhorn_transport.py:287-545): cosine cost
//     C_ij = (1 - w_h)(1 - q_i.k_j) + w_h dist_ij / (r_h + dist_ij),
//     w_h = sigmoid(alpha_h),  r_h = max(|r_param_h|, 0.1),
// K_iter x (column update, row update) with uniform marginals, then
// x_centroid = T_norm x and (dual) h_centroid = T_norm V.  It runs on the same
// library calls as flash_sinkhorn, after a change of parameters:
//   - the constant (1 - w_h) of C shifts every logit of a problem equally and
//     cancels in T_norm (the potentials absorb it), so only
//     -C/eps = (1-w) q.k / eps - w g / eps matters, which is the library's
//     cost -C'/eps' with C' = -q.k/sqrt(D) + w' g at
//         eps' = eps / ((1 - w) sqrt(D)),   w' = w / ((1 - w) sqrt(D))
//     (D the head dim the library runs, the larger of d and V's width, the
//     narrower operands zero-padded -- exact for every product);
//   - the per-head r_h is the library's r_head;
//   - the reference updates the columns first.  The library's iteration is
//     rows first, so the first call runs it on the transposed problem (Q and K
//     swapped; the geometry term, the masks and the uniform marginals are
//     symmetric), whose rows are the original columns: K_iter x (column, row)
//     exactly.  A second call with K_iter = 0 and those potentials as warm
//     starts writes T_norm x and T_norm V;
//   - the marginals: 1/n_b per valid point.  The reference's device path uses
//     one batch-mean constant instead; a constant change of the marginals only
//     shifts the column potential and leaves T_norm unchanged.
// The backward is the library's implicit-function gradient at those
// potentials; the gradients of alpha_h and r_h follow by the chain rule:
//     dL/dalpha_h = w_h (-sum_{b,i} q_i.dq_i + dw'_h / sqrt(D)),
//     dL/dr_param_h = dL/dr_h sign(r_param_h) [|r_param_h| >= 0.1]
// (the first because dL/dS summed over a problem is 0: a constant logit shift
// changes nothing).  Padded rows (mask 0) of both outputs are 0.
struct BalancedTransportFn : public torch::autograd::Function<BalancedTransportFn> {
  // Arguments: 0 Q, 1 K, 2 x_res, 3 V (optional), 4 eps, 5 alpha_h, 6 r_h,
  // 7 mask (optional), 8 K_iter, 9 cg_rtol, 10 cg_atol, 11 cg_max_iter.
  static variable_list forward(AutogradContext* ctx, Tensor Q, Tensor K, Tensor x_res, c10::optional<Tensor> V,
                               Tensor eps, Tensor alpha_h, Tensor r_h, c10::optional<Tensor> mask, int64_t K_iter,
                               double cg_rtol, double cg_atol, int64_t cg_max_iter) {
    require(Q.is_cuda() && K.is_cuda() && x_res.is_cuda(),
            "deepfold B200 Sinkhorn ops run on CUDA tensors only (no CPU path)");
    require(Q.dim() == 4 && K.sizes() == Q.sizes(), "Q_s and K_s must share the shape (B, H, N, d_h)");
    const int64_t B = Q.size(0), H = Q.size(1), N = Q.size(2), d = Q.size(3);
    require(x_res.dim() == 3 && x_res.size(0) == B && x_res.size(1) == N && x_res.size(2) == 3,
            "x_res must have the shape (B, N, 3)");
    const bool dual = V.has_value() && V->defined();
    const int64_t dv = dual ? V->size(3) : d;
    if (dual)
      require(V->dim() == 4 && V->size(0) == B && V->size(1) == H && V->size(2) == N,
              "V_h must have the shape (B, H, N, D_V)");
    const int64_t D = std::max(d, dv);
    if (D > 64 || N > dfs_max_n(static_cast<int>(D)))
      fail("N=" + std::to_string(N) + ", head dim " + std::to_string(D) +
           " is outside the kernels' range (head dim <= 64)");
    require(eps.numel() == H && alpha_h.numel() == H && r_h.numel() == H, "eps, alpha_h and r_h must have H entries");
    require(K_iter >= 0, "K_iter must be >= 0");
    if (mask.has_value() && mask->defined())
      require(mask->dim() == 2 && mask->size(0) == B && mask->size(1) == N, "mask must have the shape (B, N)");
    const DeviceSwitch guard(Q.device());
    check_device_status(Q.device());
    const auto st = Q.scalar_type();
    const auto cdt = (st == at::kBFloat16 || st == at::kHalf || st == at::kFloat) ? st : at::kFloat;
    auto widen = [&](const Tensor& t) {
      const Tensor c = t.contiguous().to(cdt);
      return t.size(3) < D ? at::constant_pad_nd(c, {0, D - t.size(3)}).contiguous() : c;
    };
    const Tensor Qc = widen(Q), Kc = widen(K);
    const Tensor Vc = dual ? widen(*V) : Tensor();
    const auto fo = Q.options().dtype(at::kFloat);
    const Tensor xr = x_res.contiguous().to(at::kFloat);
    const Tensor w = at::sigmoid(alpha_h.reshape({H}).to(at::kFloat));
    const Tensor rh = r_h.reshape({H}).to(at::kFloat);
    const Tensor r = at::clamp_min(at::abs(rh), 0.1).contiguous();
    const double qs = 1.0 / std::sqrt(static_cast<double>(D));
    const Tensor epsp = (eps.reshape({H}).to(at::kFloat) * qs / (1.0 - w)).contiguous();
    const Tensor wdp = (w * qs / (1.0 - w)).contiguous();
    Tensor mk, counts;
    if (mask.has_value() && mask->defined()) {
      mk = (mask->to(at::kFloat) > 0.5).to(at::kFloat).contiguous();
      counts = at::clamp_min(mk.sum(1), 1.0);
    } else {
      counts = at::full({B}, static_cast<double>(N), fo);
    }
    const Tensor lm = (-at::log(counts)).view({B, 1, 1}).expand({B, H, N}).contiguous();
    Tensor lu_t = at::empty({B, H, N}, fo), lv_t = at::empty({B, H, N}, fo);
    Tensor lu = at::empty({B, H, N}, fo), lv = at::empty({B, H, N}, fo);
    Tensor O = at::empty({B, H, N, D}, fo), xc = at::empty({B, H, N, 3}, fo);
    Tensor status = device_status(Q.device()).word;

    dfs_problem prob{};
    prob.B = static_cast<int32_t>(B);
    prob.H = static_cast<int32_t>(H);
    prob.N = static_cast<int32_t>(N);
    prob.d = static_cast<int32_t>(D);
    prob.in_dtype = dtype_code(cdt);
    prob.cost_mode = DFS_COST_QK;
    prob.K_iter = static_cast<int32_t>(K_iter);
    prob.check_every = 2;
    prob.lam = std::numeric_limits<float>::infinity();
    prob.r_0 = 1.0f;  // unused: r_head is given
    prob.cost_terms = DFS_TERM_GEO | DFS_TERM_XRES;
    size_t fwd_ws = 0, bwd_ws = 0;
    check_rc(dfs_workspace_size(&prob, &fwd_ws, &bwd_ws), "dfs_workspace_size");
    Tensor ws = fwd_ws ? at::empty({static_cast<int64_t>((fwd_ws + 3) / 4)}, fo) : Tensor();
    const at::cuda::CUDAStream cstream = at::cuda::getCurrentCUDAStream(Q.device().index());
    // 1. the potentials: rows of the transposed problem are the original columns
    dfs_fwd_args a{};
    a.Q = Kc.data_ptr();
    a.K = Qc.data_ptr();
    a.x_res = xr.data_ptr<float>();
    a.eps = epsp.data_ptr<float>();
    a.w_dist = wdp.data_ptr<float>();
    a.r_head = r.data_ptr<float>();
    a.log_mu = lm.data_ptr<float>();
    a.log_nu = lm.data_ptr<float>();
    a.mask = ptr_or_null<const float>(mk);
    a.log_u = lv_t.data_ptr<float>();  // column potential of the original problem
    a.log_v = lu_t.data_ptr<float>();
    a.status = status.data_ptr<int32_t>();
    check_rc(dfs_fwd(&prob, &a, ws.defined() ? ws.data_ptr() : nullptr, fwd_ws, cstream.stream()), "dfs_fwd");
    // 2. T_norm x and T_norm V from those potentials (the single variant passes Q
    //    as V and drops O: the streamed kernels write x_centroid with O)
    dfs_problem out_prob = prob;
    out_prob.K_iter = 0;
    dfs_fwd_args o{};
    o.Q = Qc.data_ptr();
    o.K = Kc.data_ptr();
    o.V = dual ? Vc.data_ptr() : Qc.data_ptr();
    o.x_res = a.x_res;
    o.eps = a.eps;
    o.w_dist = a.w_dist;
    o.r_head = a.r_head;
    o.log_mu = a.log_mu;
    o.log_nu = a.log_nu;
    o.log_u_init = lu_t.data_ptr<float>();
    o.log_v_init = lv_t.data_ptr<float>();
    o.mask = a.mask;
    o.O = O.data_ptr<float>();
    o.x_centroid = xc.data_ptr<float>();
    o.log_u = lu.data_ptr<float>();
    o.log_v = lv.data_ptr<float>();
    o.status = a.status;
    check_rc(dfs_fwd(&out_prob, &o, ws.defined() ? ws.data_ptr() : nullptr, fwd_ws, cstream.stream()), "dfs_fwd");
    {
      std::lock_guard<std::mutex> lock(g_status_mu);
      start_readback(device_status(Q.device()), cstream.stream());
    }

    ctx->save_for_backward({Qc, Kc, Vc, xr, epsp, wdp, r, lm, mk, lu, lv, w, rh});
    ctx->saved_data["K_iter"] = K_iter;
    ctx->saved_data["cg_rtol"] = cg_rtol;
    ctx->saved_data["cg_atol"] = cg_atol;
    ctx->saved_data["cg_max_iter"] = cg_max_iter;
    ctx->saved_data["fwd_status"] = status;
    ctx->saved_data["d"] = d;
    ctx->saved_data["dv"] = dv;
    ctx->saved_data["q_dtype"] = static_cast<int64_t>(Q.scalar_type());
    ctx->saved_data["x_dtype"] = static_cast<int64_t>(x_res.scalar_type());
    ctx->saved_data["v_dtype"] = static_cast<int64_t>(dual ? V->scalar_type() : Q.scalar_type());
    ctx->saved_data["a_dtype"] = static_cast<int64_t>(alpha_h.scalar_type());
    ctx->saved_data["r_dtype"] = static_cast<int64_t>(r_h.scalar_type());
    int64_t edge = 3;  // Q, K, x_res are edges 0..2
    ctx->saved_data["e_v"] = dual ? edge++ : int64_t(-1);
    if (V.has_value() && !dual) ++edge;
    ++edge;  // eps
    ctx->saved_data["e_alpha"] = edge++;
    ctx->saved_data["e_r"] = edge++;
    // outputs in fp32 (float64 for float64 inputs), as the reference's device path
    // returns them (it computes on fp32 copies)
    const auto out_dt = st == at::kDouble ? at::kDouble : at::kFloat;
    const Tensor xo = xc.to(out_dt);
    if (!dual) return {xo};
    return {xo, O.narrow(3, 0, dv).to(out_dt)};
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    const DeviceSwitch guard(saved[0].device());
    check_device_status(saved[0].device());
    const Tensor &Qc = saved[0], &Kc = saved[1], &Vc = saved[2], &xr = saved[3], &epsp = saved[4],
                 &wdp = saved[5], &r = saved[6], &lm = saved[7], &mk = saved[8], &lu = saved[9], &lv = saved[10],
                 &w = saved[11], &rh = saved[12];
    const bool dual = Vc.defined();
    auto needs = [&](const char* key) {
      const int64_t e = ctx->saved_data[key].toInt();
      return e >= 0 && ctx->needs_input_grad(static_cast<size_t>(e));
    };
    const int64_t B = Qc.size(0), H = Qc.size(1), N = Qc.size(2), D = Qc.size(3);
    const int64_t d = ctx->saved_data["d"].toInt(), dv = ctx->saved_data["dv"].toInt();
    const auto fo = Qc.options().dtype(at::kFloat);
    const bool want_alpha = needs("e_alpha"), want_r = needs("e_r");
    const Tensor dxc = grads[0].defined() ? grads[0].contiguous().to(at::kFloat) : Tensor();
    Tensor dO;
    if (dual && grads.size() > 1 && grads[1].defined()) {
      dO = grads[1].contiguous().to(at::kFloat);
      if (dv < D) dO = at::constant_pad_nd(dO, {0, D - dv}).contiguous();
    } else {
      dO = at::zeros({B, H, N, D}, fo);
    }
    Tensor dQ = (ctx->needs_input_grad(0) || want_alpha) ? at::empty({B, H, N, D}, fo) : Tensor();
    Tensor dK = ctx->needs_input_grad(1) ? at::empty({B, H, N, D}, fo) : Tensor();
    Tensor dV = (dual && needs("e_v")) ? at::empty({B, H, N, D}, fo) : Tensor();
    Tensor dx = ctx->needs_input_grad(2) ? at::empty({B, N, 3}, fo) : Tensor();
    Tensor dwd = want_alpha ? at::empty({H}, fo) : Tensor();
    Tensor dr = want_r ? at::empty({H}, fo) : Tensor();
    const Tensor rep = at::empty({2, B * H}, Qc.options().dtype(at::kInt));  // CG iterations, residuals
    Tensor status = device_status(Qc.device()).word;

    dfs_problem prob{};
    prob.B = static_cast<int32_t>(B);
    prob.H = static_cast<int32_t>(H);
    prob.N = static_cast<int32_t>(N);
    prob.d = static_cast<int32_t>(D);
    prob.in_dtype = dtype_code(Qc.scalar_type());
    prob.cost_mode = DFS_COST_QK;
    prob.K_iter = static_cast<int32_t>(ctx->saved_data["K_iter"].toInt());
    prob.check_every = 2;
    prob.lam = std::numeric_limits<float>::infinity();
    prob.r_0 = 1.0f;
    prob.cost_terms = DFS_TERM_GEO | DFS_TERM_XRES;
    dfs_cg_params cg{};
    cg.rtol = static_cast<float>(ctx->saved_data["cg_rtol"].toDouble());
    cg.atol = static_cast<float>(ctx->saved_data["cg_atol"].toDouble());
    cg.max_iter = static_cast<int32_t>(ctx->saved_data["cg_max_iter"].toInt());
    dfs_bwd_args a{};
    a.Q = Qc.data_ptr();
    a.K = Kc.data_ptr();
    a.V = dual ? Vc.data_ptr() : Qc.data_ptr();
    a.x_res = xr.data_ptr<float>();
    a.eps = epsp.data_ptr<float>();
    a.w_dist = wdp.data_ptr<float>();
    a.r_head = r.data_ptr<float>();
    a.log_mu = lm.data_ptr<float>();
    a.log_nu = lm.data_ptr<float>();
    a.mask = ptr_or_null<const float>(mk);
    a.log_u = lu.data_ptr<float>();
    a.log_v = lv.data_ptr<float>();
    a.dO = dO.data_ptr<float>();
    a.dxc = ptr_or_null<const float>(dxc);
    a.dQ = ptr_or_null<float>(dQ);
    a.dK = ptr_or_null<float>(dK);
    a.dV = ptr_or_null<float>(dV);
    a.dx_res = ptr_or_null<float>(dx);
    a.dw_dist = ptr_or_null<float>(dwd);
    a.dr_head = ptr_or_null<float>(dr);
    a.cg_iters = rep.data_ptr<int32_t>();
    a.cg_residual = reinterpret_cast<float*>(rep.data_ptr<int32_t>() + B * H);
    a.status = status.data_ptr<int32_t>();
    size_t fwd_ws = 0, bwd_ws = 0;
    check_rc(dfs_workspace_size(&prob, &fwd_ws, &bwd_ws), "dfs_workspace_size");
    Tensor ws = bwd_ws ? at::empty({static_cast<int64_t>((bwd_ws + 3) / 4)}, fo) : Tensor();
    const at::cuda::CUDAStream cstream = at::cuda::getCurrentCUDAStream(Qc.device().index());
    check_rc(dfs_bwd(&prob, &cg, &a, ws.defined() ? ws.data_ptr() : nullptr, bwd_ws, cstream.stream()), "dfs_bwd");
    {
      std::lock_guard<std::mutex> lock(g_status_mu);
      start_readback(device_status(Qc.device()), cstream.stream());
    }
    last_report() = {rep, status, ctx->saved_data["fwd_status"].toTensor()};

    auto as = [&](const Tensor& g, const char* key) {
      return g.to(static_cast<at::ScalarType>(ctx->saved_data[key].toInt()));
    };
    variable_list out(12);
    if (dQ.defined() && ctx->needs_input_grad(0)) out[0] = as(dQ.narrow(3, 0, d), "q_dtype");
    if (dK.defined()) out[1] = as(dK.narrow(3, 0, d), "q_dtype");
    if (dx.defined()) out[2] = as(dx, "x_dtype");
    if (dV.defined()) out[3] = as(dV.narrow(3, 0, dv), "v_dtype");
    if (want_alpha) {
      const Tensor qdq = (Qc.to(at::kFloat) * dQ).sum({0, 2, 3});
      out[5] = as(w * (dwd * (1.0 / std::sqrt(static_cast<double>(D))) - qdq), "a_dtype");
    }
    if (want_r) out[6] = as(dr * at::sign(rh) * (at::abs(rh) >= 0.1).to(at::kFloat), "r_dtype");
    return out;
  }
};

std::vector<Tensor> balanced_transport_autograd(Tensor Q, Tensor K, Tensor x_res, c10::optional<Tensor> V,
                                                Tensor eps, Tensor alpha_h, Tensor r_h, c10::optional<Tensor> mask,
                                                int64_t K_iter, double cg_rtol, double cg_atol, int64_t cg_max_iter) {
  return BalancedTransportFn::apply(Q, K, x_res, V, eps, alpha_h, r_h, mask, K_iter, cg_rtol, cg_atol, cg_max_iter);
}

std::vector<Tensor> flash_sinkhorn_autograd(Tensor Q, Tensor K, Tensor V, c10::optional<Tensor> x_res,
                                            c10::optional<Tensor> pos_weight, c10::optional<Tensor> pos_bins,
                                            Tensor eps, c10::optional<Tensor> w_dist, Tensor log_mu,
                                            Tensor log_nu, c10::optional<Tensor> log_u_init,
                                            c10::optional<Tensor> log_v_init, c10::optional<Tensor> mask,
                                            int64_t K_iter, double lam, double r_0, double cg_rtol,
                                            double cg_atol, int64_t cg_max_iter, c10::optional<Tensor> chain_id,
                                            c10::optional<Tensor> global_idx, c10::optional<Tensor> bond_matrix) {
  return FlashSinkhornFn::apply(Q, K, V, x_res, pos_weight, pos_bins, eps, w_dist, log_mu, log_nu, log_u_init,
                                log_v_init, mask, K_iter, lam, r_0, cg_rtol, cg_atol, cg_max_iter, chain_id,
                                global_idx, bond_matrix);
}

// compute_bins of the reference on the device: (B, N, N) int32
Tensor compute_bins_cuda(Tensor chain_id, Tensor global_idx, Tensor bond_matrix) {
  require(chain_id.is_cuda() && global_idx.is_cuda() && bond_matrix.is_cuda(),
          "compute_bins runs on CUDA tensors only (no CPU path)");
  require(chain_id.dim() == 2 && global_idx.sizes() == chain_id.sizes() && bond_matrix.dim() == 3 &&
              bond_matrix.size(0) == chain_id.size(0) && bond_matrix.size(1) == chain_id.size(1) &&
              bond_matrix.size(2) == chain_id.size(1),
          "compute_bins: chain_id, global_idx (B, N) and bond_matrix (B, N, N)");
  const DeviceSwitch guard(chain_id.device());
  const int64_t B = chain_id.size(0), N = chain_id.size(1);
  const Tensor ch = chain_id.contiguous().to(at::kInt), gx = global_idx.contiguous().to(at::kInt);
  const Tensor bd = bond_matrix.contiguous().to(at::kByte);
  Tensor out = at::empty({B, N, N}, chain_id.options().dtype(at::kInt));
  const at::cuda::CUDAStream cstream = at::cuda::getCurrentCUDAStream(chain_id.device().index());
  check_rc(dfs_compute_bins(static_cast<int>(B), static_cast<int>(N), ch.data_ptr<int32_t>(), gx.data_ptr<int32_t>(),
                            bd.data_ptr<uint8_t>(), out.data_ptr<int32_t>(), cstream.stream()),
           "dfs_compute_bins");
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "native autograd glue for libdfsink (flash Sinkhorn forward / IFT backward)";
  m.def("flash_sinkhorn", &flash_sinkhorn_autograd,
        "FlashSinkhornFn.apply: returns [O, x_centroid, log_u, log_v], or [O, log_u, log_v] without x_res",
        py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("x_res"), py::arg("pos_weight"), py::arg("pos_bins"),
        py::arg("eps"), py::arg("w_dist"), py::arg("log_mu"), py::arg("log_nu"), py::arg("log_u_init"),
        py::arg("log_v_init"), py::arg("mask"), py::arg("K_iter"), py::arg("lam"), py::arg("r_0"),
        py::arg("cg_rtol"), py::arg("cg_atol"), py::arg("cg_max_iter"), py::arg("chain_id") = py::none(),
        py::arg("global_idx") = py::none(), py::arg("bond_matrix") = py::none());
  m.def("compute_bins", &compute_bins_cuda, "compute_bins of the reference on the device: (B, N, N) int32");
  m.def("balanced_transport", &balanced_transport_autograd,
        "BalancedTransportFn.apply: returns [x_centroid], or [x_centroid, h_centroid] with V");
  m.def("last_report", []() { return last_report(); },
        "[report (2, B*H) int32: CG iterations, then the residuals' fp32 bits; status, fwd_status] of the most "
        "recent backward (status: the device's sticky status word, the OR of every call's bits since the last "
        "check)");
  m.def("take_status", &take_status, py::arg("wait") = true,
        "status bits of the current device's calls since the last read (after the stream drains with "
        "wait=True), plus warning bits seen by the checks inside calls; the bits are cleared");
}
