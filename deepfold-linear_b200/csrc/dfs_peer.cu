// dfs_peer.cu -- peer-memory gather of row slices between the GPUs of a
// row-sharded run (dfs_peer_gather_rows in include/dfsink.h).
//
// Every GPU holds the same buffer layout (a workspace shared through CUDA IPC):
// a slot of P problems x N rows x `width` floats.  Each GPU owns rows
// [row_begin, row_end) of every problem; a gather makes every GPU's copy whole.
// Two launches on the caller's stream:
//   push    this GPU's rows into every other GPU's buffer over NVLink (plain
//           stores, 16-byte when the rows allow it); each CTA then fences at
//           system scope (thread 0, after a barrier: the fence is cumulative
//           over the CTA's stores) and arrives on a completion counter in this
//           GPU's buffer; the last CTA re-arms it, fences again and raises
//           every GPU's arrival counter once;
//   wait    one thread: adds npeers to this GPU's expected count (kept beside
//           its arrival counter) and spins until the arrival counter reaches
//           it, bounded by kWaitNs (a timeout sets DFS_ERR_DEVICE_TIMEOUT in
//           the status word and returns).  Every GPU runs the same gathers in
//           the same order, so the counts stay in step without the host: a
//           gather's launches take no per-call argument and can be recorded
//           once into a CUDA graph (the row-sharded CG loop does).
// A later kernel on the stream starts after the wait kernel has seen every
// GPU's arrival, so it reads every GPU's rows.  No collective library is
// involved; the exchange costs two short launches instead of an all-gather.
#include <algorithm>

#include "dfs_kernels.cuh"

namespace dfs {
namespace {

struct PushArgs {
  float* dst[DFS_MAX_PEERS];               // every other GPU's slot base (null: skip)
  unsigned long long* arrive[DFS_MAX_PEERS];  // every GPU's arrival counter
  unsigned* done;                          // this GPU's completion counter of the push CTAs
  const float* src;                        // this GPU's slot base
  int npeers;
  int P;
  size_t row_floats;                       // floats per problem (N * width)
  size_t first;                            // first float of this GPU's rows within a problem
  size_t count;                            // floats of this GPU's rows within a problem
};

template <bool VEC>
__global__ void __launch_bounds__(256) peer_push_kernel(const PushArgs a) {
  const size_t per = VEC ? a.count / 4 : a.count;  // units per problem
  const size_t total = per * a.P;
  for (size_t u = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t p = u / per, k = u - p * per;
    const size_t off = p * a.row_floats + a.first + (VEC ? 4 * k : k);
    if constexpr (VEC) {
      const float4 v = *reinterpret_cast<const float4*>(a.src + off);
      for (int q = 0; q < a.npeers; ++q)
        if (a.dst[q] != nullptr) *reinterpret_cast<float4*>(a.dst[q] + off) = v;
    } else {
      const float v = a.src[off];
      for (int q = 0; q < a.npeers; ++q)
        if (a.dst[q] != nullptr) a.dst[q][off] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's stores (ordered before by the barrier) are performed everywhere
    const unsigned prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {  // every CTA's stores are performed: re-arm, then raise every counter
      *a.done = 0u;
      __threadfence_system();
      for (int q = 0; q < a.npeers; ++q) atomicAdd_system(a.arrive[q], 1ull);
    }
  }
}

__global__ void peer_wait_kernel(const unsigned long long* cnt, unsigned long long* expected, int npeers,
                                 int32_t* status) {
  const unsigned long long want = *expected + static_cast<unsigned long long>(npeers);
  *expected = want;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(cnt) : "memory");
    if (v >= want) return;
    if (it == 0) t0 = global_ns();
    else if ((it & 63u) == 0 && global_ns() - t0 > kWaitNs) break;
    __nanosleep(128);
  }
  if (status != nullptr) atomicOr(status, DFS_ERR_DEVICE_TIMEOUT);
}

}  // namespace

cudaError_t peer_gather_rows(const PeerInfo& pi, size_t slot_offset, int P, int N, int width, int row_begin,
                             int row_end, size_t counter_offset, int32_t* status, cudaStream_t st) {
  PushArgs a{};
  a.npeers = pi.npeers;
  for (int k = 0; k < pi.npeers; ++k)
    a.dst[k] = k == pi.self ? nullptr : reinterpret_cast<float*>(static_cast<char*>(pi.ws[k]) + slot_offset);
  a.src = reinterpret_cast<const float*>(static_cast<const char*>(pi.ws[pi.self]) + slot_offset);
  a.P = P;
  a.row_floats = static_cast<size_t>(N) * width;
  a.first = static_cast<size_t>(row_begin) * width;
  a.count = static_cast<size_t>(row_end - row_begin) * width;
  for (int k = 0; k < pi.npeers; ++k)
    a.arrive[k] = reinterpret_cast<unsigned long long*>(static_cast<char*>(pi.ws[k]) + counter_offset);
  char* own = static_cast<char*>(pi.ws[pi.self]) + counter_offset;
  a.done = reinterpret_cast<unsigned*>(own + 8);
  // 16-byte stores when every problem's segment starts and ends on a 16-byte boundary
  const bool vec = (slot_offset % 16) == 0 && (a.row_floats % 4) == 0 && (a.first % 4) == 0 && (a.count % 4) == 0;
  const size_t units = (vec ? a.count / 4 : a.count) * P;
  const unsigned grid = static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>((units + 255) / 256, 148u * 4u)));
  if (vec) peer_push_kernel<true><<<grid, 256, 0, st>>>(a);
  else peer_push_kernel<false><<<grid, 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  peer_wait_kernel<<<1, 1, 0, st>>>(a.arrive[pi.self], reinterpret_cast<unsigned long long*>(own + 16), pi.npeers,
                                    status);
  return cudaGetLastError();
}

}  // namespace dfs

using namespace dfs;

namespace {
bool peer_set_ok(const dfs_peer_set* peers) {
  if (peers == nullptr || peers->npeers < 1 || peers->npeers > DFS_MAX_PEERS || peers->self < 0 ||
      peers->self >= peers->npeers)
    return false;
  for (int k = 0; k < peers->npeers; ++k)
    if (peers->ws[k] == nullptr || (reinterpret_cast<uintptr_t>(peers->ws[k]) & 255u) != 0) return false;
  return true;
}
PeerInfo peer_info(const dfs_peer_set* peers) {
  PeerInfo pi{};
  pi.npeers = peers->npeers;
  pi.self = peers->self;
  for (int k = 0; k < peers->npeers; ++k) pi.ws[k] = peers->ws[k];
  pi.wait_for = 0;
  return pi;
}
}  // namespace

extern "C" int dfs_peer_gather_rows(const dfs_peer_set* peers, size_t slot_offset, int P, int N, int width,
                                    int row_begin, int row_end, size_t counter_offset, int32_t* status,
                                    void* stream) {
  if (!peer_set_ok(peers) || P <= 0 || N <= 0 || width <= 0 || row_begin < 0 || row_end < row_begin ||
      row_end > N || (slot_offset & 3u) != 0 || (counter_offset & 7u) != 0)
    return DFS_ERR_INVALID_ARGUMENT;
  return peer_gather_rows(peer_info(peers), slot_offset, P, N, width, row_begin, row_end, counter_offset, status,
                          static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? DFS_OK
             : DFS_ERR_CUDA;
}
