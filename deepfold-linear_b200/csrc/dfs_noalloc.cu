// dfs_noalloc.cu -- dfs_fwd_static: the forward for callers that cannot
// allocate device memory.
//
// Problems beyond the cluster-resident range (N > 384 or d = 64) run on the
// streamed kernels, which need a scratch workspace (dfs_workspace_size).  Some
// callers have no way to provide one: a C or FFI host program that receives
// its input and output buffers from another runtime and holds no allocator of
// its own, or an application whose device memory is entirely owned by a
// framework's memory pool, where a cudaMalloc of its own would synchronise the
// device and compete with that pool.  For them this file keeps one fixed
// scratch array in device memory, sized DFS_STATIC_SCRATCH_BYTES, that the
// library owns; dfs_fwd_static hands it to the regular forward in place of a
// caller workspace and allocates nothing itself.
//
// The array exists on every GPU that loads this library, for the life of the
// process.  Every call on a device shares it: two calls whose work overlaps on
// that GPU (different streams without ordering between them) race on it.
// Nothing in the forward's workspace has to start at zero -- every slot is
// written before it is read -- so no clearing is needed between calls.
#include <mutex>

#include "dfs_kernels.cuh"

namespace {

// The scratch itself.  In host code this name is only a stand-in for the
// device array, never an address a kernel may use: kernels get the device
// address fetched with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_fwd_scratch[DFS_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};  // device address of g_fwd_scratch, per device

// Device address of the scratch on the current device; looked up once per
// device (the first call there), with that device current.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DFS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fwd_scratch) != cudaSuccess || p == nullptr) return DFS_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DFS_OK;
}

}  // namespace

extern "C" int dfs_fwd_static(const dfs_problem* p, const dfs_fwd_args* a, void* stream) {
  size_t need = 0;
  const int rc = dfs_workspace_size(p, &need, nullptr);
  if (rc != DFS_OK) return rc;
  if (need > DFS_STATIC_SCRATCH_BYTES) return DFS_ERR_WORKSPACE;  // beyond the fixed scratch
  void* ws = nullptr;
  if (need > 0) {
    const int src = scratch_address(&ws);
    if (src != DFS_OK) return src;
  }
  return dfs_fwd(p, a, ws, need, stream);
}
