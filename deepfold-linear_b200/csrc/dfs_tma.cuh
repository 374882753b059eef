// dfs_tma.cuh -- TMA staging helpers shared by the warp-specialised streamed
// kernels (dfs_stream_tma.cu, dfs_stream_bwd_tma.cu).
#pragma once

#include <cuda.h>

#include "dfs_slab.cuh"

namespace dfs {

// Instruction descriptor, kind::f16 (fp16 or bf16 operands), fp32 accumulate,
// both operands K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

DFS_DEV void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

// tcgen05.ld of 32 columns without waiting: the registers are valid only after
// tmem_wait_ld on the same array (which carries them as operands, so no use
// can be scheduled before the wait).
DFS_DEV void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
DFS_DEV void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])::"memory");
}

// Shared-memory matrix descriptor of a K-major operand without swizzle: core
// matrices of 8 rows x 16 bytes stored contiguously (128 bytes), lbo = byte
// stride between core matrices adjacent in K, sbo = between those adjacent in
// M / N.
DFS_DEV uint64_t noswz_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100; layout type 0 = no swizzle
  return d;
}

// 2^x on the FMA and integer pipes, to take part of the exponentials off the
// MUFU (which runs 16 of them per clock per SM against 128 FMAs).  Cody-Waite
// style: x = j + f with j = round(x) by the 1.5 * 2^23 rounding trick (j lands
// in the low mantissa bits of t) and f in [-0.5, 0.5]; 2^f by a degree-5
// polynomial whose coefficients are a relative-error minimax fit on
// [-0.5, 0.5] (iteratively reweighted least squares in float64, rounded to
// fp32); 2^j by adding j to the exponent field.  Maximum relative error
// 2.1e-7 over [-125, 16] (fp32 evaluation with FMA), about that of ex2.approx.
// x is clamped below at -125 so the result stays a normal float: there it
// returns 2^-125 (about 2.4e-38) instead of a smaller value or zero, which is
// below the rounding of any sum it joins whose largest term is >= 1.
DFS_DEV float ex2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;
  const float j = t - 12582912.0f;
  const float f = x - j;
  float p = fmaf(0.00132764445f, f, 0.00967553724f);
  p = fmaf(p, f, 0.0555071346f);
  p = fmaf(p, f, 0.240221202f);
  p = fmaf(p, f, 0.693146944f);
  p = fmaf(p, f, 1.00000012f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// ex2_poly on two values at once with the packed fp32 pair instructions of
// sm_100 (fma.rn.f32x2 / add.rn.f32x2: one issue slot for two lanes' worth of
// FMA work): the same operations in the same order and rounding, so each
// result is bit-identical to ex2_poly's.
DFS_DEV float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.0f, 12582912.0f));
  const float2 j = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);  // x - j, exact
  float2 p = __ffma2_rn(make_float2(0.00132764445f, 0.00132764445f), f,
                        make_float2(0.00967553724f, 0.00967553724f));
  p = __ffma2_rn(p, f, make_float2(0.0555071346f, 0.0555071346f));
  p = __ffma2_rn(p, f, make_float2(0.240221202f, 0.240221202f));
  p = __ffma2_rn(p, f, make_float2(0.693146944f, 0.693146944f));
  p = __ffma2_rn(p, f, make_float2(1.00000012f, 1.00000012f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// max of three floats in one instruction (sm_100), NaN operands ignored as fmaxf does
DFS_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// maximum of 32 values: 17 three- and two-input max instructions
DFS_DEV float max32(const float (&v)[32]) {
  float t[11];
#pragma unroll
  for (int i = 0; i < 10; ++i) t[i] = fmax3(v[3 * i], v[3 * i + 1], v[3 * i + 2]);
  t[10] = fmaxf(v[30], v[31]);
  const float u0 = fmax3(t[0], t[1], t[2]), u1 = fmax3(t[3], t[4], t[5]), u2 = fmax3(t[6], t[7], t[8]);
  const float u3 = fmaxf(t[9], t[10]);
  return fmaxf(fmax3(u0, u1, u2), u3);
}

// 64-bit load with system-scope acquire (a counter raised by other GPUs).
DFS_DEV unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Adds `bytes` to the transaction count of the current phase without arriving.
DFS_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

DFS_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// TMA load of the box at element coordinates (x, y, z) into shared memory,
// completion counted in bytes on `bar`.  No multicast.
DFS_DEV void tma_load_3d(uint32_t dst, const CUtensorMap* tm, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Launches a kernel as a programmatic dependent of the previous work on the
// stream (programmatic stream serialization): its grid may be launched and set
// up while the previous kernel's last CTAs run.  Every kernel launched this way
// executes griddepcontrol.wait as its first instruction, before it reads or
// writes anything; the tile passes then trigger their own dependents
// (griddepcontrol.launch_dependents) at once, so the next pass is launched when
// every CTA of this one has started and passed its wait -- at most two grids
// overlap, and the later one only waits until the earlier has finished.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// Tensor map of a row-major (BH, rows, inner) tensor of `dtype` elements as the
// 3-D tensor {inner, rows, BH}, boxes of box_inner x box_rows x 1 elements with
// 128-byte swizzle (box_inner x element size must be 128 bytes).  False when
// the address is not 16-byte aligned or the driver refuses the map.
bool make_tmap(CUtensorMap* tm, const void* ptr, int dtype, int inner, int rows, int BH, int box_inner, int box_rows);
// True when cuTensorMapEncodeTiled could be obtained from the driver.
bool tmap_available();

}  // namespace dfs
