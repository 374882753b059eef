// dfs_device.cuh -- sm_100a building blocks shared by the flash-Sinkhorn kernels:
// tcgen05 tensor-memory allocation, MMA issue and loads, mbarriers with bounded
// waits, thread-block-cluster barriers and distributed-shared-memory access,
// and the 128-byte-swizzled shared-memory operand layout the MMAs read.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/dfsink.h"

#define DFS_DEV __device__ __forceinline__
#define DFS_DEV_HOST_INLINE __host__ __device__ inline

namespace dfs {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNeg = -1e30f;          // "minus infinity" that keeps x - y finite
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits give up after 2 s

DFS_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DFS_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
DFS_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

DFS_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Wait until the phase with the given parity has completed.  Gives up after
// kWaitNs and returns false, so a lost arrival can never hang the GPU.
DFS_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if (it == 0) t0 = global_ns();
    else if ((it & 255u) == 0 && global_ns() - t0 > kWaitNs) return false;
  }
}

// ---------------------------------------------------------------- fences
DFS_DEV void fence_async_smem() {  // generic-proxy smem writes -> visible to tcgen05
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
DFS_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DFS_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------- TMEM
// Executed by one full warp.
DFS_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
DFS_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (warp-collective).
DFS_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

DFS_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- UMMA
// Shared-memory matrix descriptor for a 128B-swizzled operand.
// For K-major operands lbo is unused (16); sbo is the 8-row-group stride (1024).
// For MN-major operands lbo is the stride between 32-element MN groups and sbo
// the stride between 8-row K groups.
DFS_DEV uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::tf32, fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                                  // D = F32
         | (2u << 7) | (2u << 10)                   // A, B = TF32
         | (static_cast<uint32_t>(a_mn_major) << 15) | (static_cast<uint32_t>(b_mn_major) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D(tmem) (+)= A(smem) * B(smem), issued by one thread.
DFS_DEV void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
DFS_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Byte offset of element (row, col) of an fp32 matrix with `rows` rows (a
// multiple of 8) stored as 128B-swizzled atoms of 8 rows x 32 columns; atom
// (col/32, row/8) sits at ((col/32)*(rows/8) + row/8) * 1024.  Inside an atom the
// 16-byte chunk index is XOR-ed with the row index, the layout tcgen05 reads
// with SWIZZLE_128B descriptors.  Read K-major along columns (sbo = 1024) or
// MN-major along columns (lbo = rows*128, sbo = 1024).
DFS_DEV uint32_t sw_off(int row, int col, int rows) {
  const int r = row & 7;
  return static_cast<uint32_t>((((col >> 5) * (rows >> 3) + (row >> 3)) << 10) + (r << 7) +
                               ((((col >> 2) & 7) ^ r) << 4) + ((col & 3) << 2));
}

// ---------------------------------------------------------------- cluster
DFS_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
DFS_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
DFS_DEV uint32_t dsmem_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
DFS_DEV void dsmem_st(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
DFS_DEV void dsmem_st4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// Push-style all-to-all over distributed shared memory.  Every CTA of the
// cluster owns a receive buffer recv[2][C][RS] (floats); a CTA publishes its
// values into slot [buf][its rank] of every CTA with remote stores (which do
// not stall the writer), one cluster barrier orders them, and readers then use
// their own copy with ordinary shared-memory loads.  The two buffers alternate:
// a CTA can only start the next exchange after every peer has arrived at the
// barrier of this one, i.e. has finished reading the previous one.
template <int C, int RS>
struct ClusterExchange {
  float* recv;
  int buf;
  int rank;
  DFS_DEV uint32_t slot_addr(int off) const { return smem_u32(recv + (buf * C + rank) * RS + off); }
  // a cluster of one CTA exchanges through its own shared memory and a CTA barrier
  DFS_DEV void put(int off, float v) const {
    if constexpr (C == 1) {
      recv[buf * RS + off] = v;
    } else {
      const uint32_t a = slot_addr(off);
#pragma unroll
      for (int c = 0; c < C; ++c) dsmem_st(dsmem_addr(a, static_cast<uint32_t>(c)), v);
    }
  }
  DFS_DEV void put4(int off, float4 v) const {
    if constexpr (C == 1) {
      *reinterpret_cast<float4*>(recv + buf * RS + off) = v;
    } else {
      const uint32_t a = slot_addr(off);
#pragma unroll
      for (int c = 0; c < C; ++c) dsmem_st4(dsmem_addr(a, static_cast<uint32_t>(c)), v);
    }
  }
  // four values to CTA `dst` only
  DFS_DEV void put4_to(int dst, int off, float4 v) const {
    if constexpr (C == 1)
      *reinterpret_cast<float4*>(recv + buf * RS + off) = v;
    else
      dsmem_st4(dsmem_addr(slot_addr(off), static_cast<uint32_t>(dst)), v);
  }
  // one value to CTA `dst` only (callers spread the C destinations over lanes)
  DFS_DEV void put_to(int dst, int off, float v) const {
    if constexpr (C == 1)
      recv[buf * RS + off] = v;
    else
      dsmem_st(dsmem_addr(slot_addr(off), static_cast<uint32_t>(dst)), v);
  }
  DFS_DEV const float* from(int src) const { return recv + (buf * C + src) * RS; }
  DFS_DEV void sync() const {
    if constexpr (C == 1)
      __syncthreads();
    else
      cluster_sync();
  }
  DFS_DEV void next() { buf ^= 1; }
};

DFS_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bulk copy of `bytes` from this CTA's shared memory into the shared memory of a
// CTA of the cluster; completion is counted in bytes on that CTA's mbarrier.
DFS_DEV void bulk_copy_to_cluster(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t dst_bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "r"(src), "r"(bytes), "r"(dst_bar)
               : "memory");
}

// Cluster all-to-all through bulk asynchronous copies.  Every CTA stages its
// contribution in local shared memory; after a CTA barrier one thread copies
// the stage into this CTA's receive slot in every CTA (one cp.async.bulk per
// destination, completion counted in bytes on the destination's mbarrier) and
// every thread waits on its own CTA's mbarrier.  Stages, receive buffers and
// mbarriers are double-buffered by round parity.  Reuse is safe without further
// synchronisation: a CTA rewrites stage / receive buffer b two rounds later,
// and completing the round in between requires every peer's copy of that
// round, which each peer issues only after it has received (so read) the
// earlier round.  A cluster of one CTA exchanges through its stage and the
// CTA barrier alone.
template <int C, int RS>
struct BulkExchange {
  float* recv;        // [2][C][RS] floats
  float* stg;         // [2][RS] floats
  uint64_t* bar;      // [2] mbarriers, arrival count 1
  int buf;
  uint32_t phase;     // bit b: parity of bar[b]'s next completion
  int rank;
  bool dead;          // a wait timed out: later waits return at once

  DFS_DEV void init() const {  // one thread; then fence_mbar_init and a cluster barrier
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
  }
  DFS_DEV float* stage() const { return stg + buf * RS; }
  DFS_DEV const float* from(int src) const {
    if constexpr (C == 1)
      return stg + buf * RS;
    else
      return recv + (buf * C + src) * RS;
  }
  // All threads, after writing this round's stage: exchange `bytes` (a multiple
  // of 16) of it.  Returns false if the wait timed out.
  DFS_DEV bool exchange(int tid, uint32_t bytes) {
    if constexpr (C == 1) {
      __syncthreads();
      return true;
    } else {
      fence_async_smem();  // stage writes -> visible to the bulk-copy engine
      __syncthreads();
      const uint32_t b = smem_u32(&bar[buf]);
      if (tid == 0) {
        mbar_arrive_expect_tx(b, C * bytes);
        const uint32_t dst = smem_u32(recv + (buf * C + rank) * RS), src = smem_u32(stage());
#pragma unroll
        for (int c = 0; c < C; ++c)
          bulk_copy_to_cluster(dsmem_addr(dst, static_cast<uint32_t>(c)), src, bytes,
                               dsmem_addr(b, static_cast<uint32_t>(c)));
      }
      const uint32_t par = (phase >> buf) & 1u;
      phase ^= 1u << buf;
      if (dead) return false;
      if (!mbar_wait(&bar[buf], par)) {
        dead = true;
        return false;
      }
      return true;
    }
  }
  DFS_DEV void next() { buf ^= 1; }
};

DFS_DEV float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ---------------------------------------------------------------- misc
DFS_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
DFS_DEV float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
DFS_DEV float load_as_f32(const void* p, size_t i, int dtype) {
  if (dtype == DFS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == DFS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

DFS_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
DFS_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Reduce 4 per-lane partials (one per row of the warp's 4-row block) across the
// 32 lanes.  Lane l ends with the total of row (l >> 3) & 3.  6 shuffles.
template <bool kMax>
DFS_DEV float reduce4_rows(const float (&a)[4], int lane) {
  const bool hi4 = lane & 16, hi3 = lane & 8;
  float b[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = hi4 ? a[i] : a[i + 2];
    const float keep = hi4 ? a[i + 2] : a[i];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
    b[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
  float d;
  {
    const float send = hi3 ? b[0] : b[1];
    const float keep = hi3 ? b[1] : b[0];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 8);
    d = kMax ? fmaxf(keep, recv) : keep + recv;
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) {
    const float e = __shfl_xor_sync(0xffffffffu, d, o);
    d = kMax ? fmaxf(d, e) : d + e;
  }
  return d;
}

// Order-preserving map between floats and ints, for atomicMax on floats of any sign.
DFS_DEV int float_to_ordered(float x) {
  const int i = __float_as_int(x);
  return i >= 0 ? i : (i ^ 0x7fffffff);
}
DFS_DEV float ordered_to_float(int i) { return __int_as_float(i >= 0 ? i : (i ^ 0x7fffffff)); }

// Reduce 8 per-lane partials (one per row of the warp's 8-row block) across the
// 32 lanes.  Lane l ends with the total of row (l >> 2) & 7.  9 shuffles.
template <bool kMax>
DFS_DEV float reduce8_rows(float (&a)[8], int lane) {
  const bool hi4 = lane & 16, hi3 = lane & 8, hi2 = lane & 4;
  float b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = hi4 ? a[i] : a[i + 4];
    const float keep = hi4 ? a[i + 4] : a[i];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
    b[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
  float c[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = hi3 ? b[i] : b[i + 2];
    const float keep = hi3 ? b[i + 2] : b[i];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 8);
    c[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
  float d;
  {
    const float send = hi2 ? c[0] : c[1];
    const float keep = hi2 ? c[1] : c[0];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 4);
    d = kMax ? fmaxf(keep, recv) : keep + recv;
  }
  float e = __shfl_xor_sync(0xffffffffu, d, 2);
  d = kMax ? fmaxf(d, e) : d + e;
  e = __shfl_xor_sync(0xffffffffu, d, 1);
  d = kMax ? fmaxf(d, e) : d + e;
  return d;
}

// [lo, hi): the smallest range of positions that holds every valid point of
// batch element bb under a (B, N) mask (nonzero = valid); [0, N) without a
// mask, [0, 0) when no point is valid.  Block-wide: every thread of a CTA of NT
// threads calls it; red is 2 * NT / 32 ints of shared memory.
template <int NT>
DFS_DEV void valid_extent(const float* mask, int bb, int N, int* red, int& lo, int& hi) {
  if (mask == nullptr) {
    lo = 0;
    hi = N;
    return;
  }
  const float* mrow = mask + static_cast<size_t>(bb) * N;
  int l = N, h = -1;
#pragma unroll 4
  for (int j = threadIdx.x; j < N; j += NT) {
    const bool v = mrow[j] != 0.0f;
    l = v ? min(l, j) : l;
    h = v ? j : h;
  }
  l = __reduce_min_sync(0xffffffffu, l);
  h = __reduce_max_sync(0xffffffffu, h);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    red[warp] = l;
    red[NT / 32 + warp] = h;
  }
  __syncthreads();
  l = N;
  h = -1;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    l = min(l, red[w]);
    h = max(h, red[NT / 32 + w]);
  }
  __syncthreads();  // red may be reused
  lo = h < 0 ? 0 : l;
  hi = h + 1;
}

// The same extent from a per-batch table computed once per call (ext != null,
// mask != null): two loads instead of a scan of the mask and two CTA barriers.
template <int NT>
DFS_DEV void valid_extent(const int2* ext, const float* mask, int bb, int N, int* red, int& lo, int& hi) {
  if (ext != nullptr && mask != nullptr) {
    const int2 e = ext[bb];
    lo = e.x;
    hi = e.y;
    return;
  }
  valid_extent<NT>(mask, bb, N, red, lo, hi);
}

}  // namespace dfs
