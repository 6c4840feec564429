// Shared device helpers for the b200 kernels: mbarriers with bounded waits,
// TMA tile loads, tcgen05 (TMEM alloc / MMA / commit / load), programmatic
// dependent launch and cluster (DSMEM) primitives.  sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define DEVI __device__ __forceinline__

namespace laya {

// Status word codes written by kernels (host maps them to errors).
enum : uint32_t {
  kStatusOk = 0,
  kStatusGemmFullTimeout = 1,
  kStatusGemmEmptyTimeout = 2,
  kStatusGemmDoneTimeout = 3,
  kStatusAttnTimeout = 4,
};

// e4m3 row scale = max(amax * fl(1/448), 1e-12).  The reference's FP8 path
// multiplies by the fp32 reciprocal of 448 rather than dividing (PyTorch's CUDA
// division of a tensor by a scalar and Triton's division by a constant both
// lower to that product), which differs from amax / 448 in the last bit for
// some inputs; the golden vectors of its FP8Linear pin this form.
constexpr float kInvE4m3Max = 1.0f / 448.0f;

// Every spin on an mbarrier gives up after this many nanoseconds, records an
// error in the status word and lets the kernel unwind.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

DEVI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DEVI uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

DEVI void record_status(uint32_t* status, uint32_t code) {
  if (status) atomicCAS(status, 0u, code);
}

// ---------------------------------------------------------------- mbarrier
DEVI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

DEVI void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DEVI void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

DEVI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

DEVI bool mbar_try(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false after
// `limit_ns` (default kWaitLimitNs) without completion.
DEVI bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try(addr, parity)) return true;
    if (globaltimer() - t0 > limit_ns) return false;
  }
}

// Wait limit of a launch: its parameter block's override in microseconds, or
// the default.
DEVI uint64_t wait_limit(uint32_t override_us) {
  return override_us ? (uint64_t)override_us * 1000ull : kWaitLimitNs;
}

// ---------------------------------------------------------------- TMA
DEVI void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 3-D tile load ([batch][rows][cols] tensors: rows past a batch entry's end
// read as zeros instead of the next entry's first rows).
DEVI void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Tile store from shared memory (rows beyond the tensor's extent are clipped).
DEVI void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
DEVI void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
DEVI void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
DEVI void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

DEVI uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

DEVI uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

DEVI void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------- PDL
DEVI void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DEVI void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
DEVI void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
DEVI void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
DEVI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
DEVI void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f8f6f4 (e4m3 x e4m3, fp32 accumulate).
DEVI void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Block-scaled NVFP4: e2m1 x e2m1 with ue4m3 scales every 16 elements, the
// scale factors read from TMEM.
DEVI void umma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa_tmem,
                    uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %6, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%4], [%5], p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// Copy 128 lanes x 16 bytes of scale factors from shared memory into TMEM
// (one 32x128b block per warp quarter, replicated as the MMA expects).
DEVI void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

DEVI void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns per warp.
DEVI void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
DEVI void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
DEVI void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout TMA writes (8-row groups 1024 bytes apart).
DEVI uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // 128-byte swizzle
  return d;
}

// Instruction descriptors (M = 128 TMEM lanes, N = token tile).
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---------------------------------------------------------------- cluster
DEVI void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
DEVI uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
DEVI float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
DEVI float4 ld_dsmem_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
// 2^x on the SFU (flushes results below 2^-126 to zero; 2^-inf = 0).
DEVI float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk j of row r in a 128-byte-swizzled tile (rows
// of 128 bytes, 8-row groups 1024 bytes apart), the layout TMA writes and the
// MMA's sw128 descriptors read.
DEVI uint32_t sw128_offset(int r, int j) { return (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4); }

// Asynchronous store into another CTA's shared memory (cluster address) that
// counts its bytes on that CTA's mbarrier (cluster address).
DEVI void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(addr), "f"(v),
               "r"(bar)
               : "memory");
}
DEVI void st_async_f32x4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
               : "memory");
}
// mbarrier wait that also acquires what other CTAs of the cluster stored
// with st.async before completing its transaction bytes; false after limit_ns.
DEVI bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if (globaltimer() - t0 > limit_ns) return false;
  }
}
DEVI uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// ---------------------------------------------------------------- numerics
DEVI float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Exact (erf) GELU in fp32, as torch's F.gelu(approximate="none").
DEVI float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

// Two fp32 values -> two e4m3 bytes (round to nearest even, saturate).
DEVI uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two fp32 values -> one byte of two e2m1 nibbles (lo in bits 0-3).
DEVI uint8_t f32x2_to_e2m1x2(float lo, float hi) {
  uint16_t r;
  asm("{\n .reg .b8 q;\n cvt.rn.satfinite.e2m1x2.f32 q, %1, %2;\n mov.b16 %0, {q, 0};\n}\n"
      : "=h"(r)
      : "f"(hi), "f"(lo));
  return (uint8_t)(r & 0xFF);
}

// x / d rounded to nearest, given inv = 1/d rounded to nearest, by two
// residual corrections of the product x * inv (Markstein's FMA division,
// IBM J. Res. Dev. 34(1):111-119, 1990): after the first step the quotient is
// faithful, and a correction of a faithful quotient with an exact residual
// r = x - q*d and a correctly rounded reciprocal yields the correctly rounded
// quotient.  Valid for normal d and quotients that neither overflow nor
// underflow; the quantisers divide by scales >= 1e-12 with |x| <= 448 * d.
DEVI float div_rn_by(float x, float d, float inv) {
  float q = x * inv;
  q = fmaf(fmaf(-q, d, x), inv, q);
  return fmaf(fmaf(-q, d, x), inv, q);
}

// Value of a non-negative e4m3 code (sign bit clear; 4 exponent bits, bias 7,
// 3 mantissa bits), built from its bits: subnormals m * 2^-9, normals
// (1 + m/8) * 2^(e-7) as an fp32 with exponent e + 120.
DEVI float e4m3_value(uint32_t code) {
  const uint32_t e = (code >> 3) & 0xF, m = code & 7;
  return e == 0 ? (float)m * 0.001953125f : __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// NVFP4 scale-block byte offset of (row, 16-element block g): blocks of
// `rows_per_block` rows x 4 scale columns (512 bytes, byte (r%32)*16 + (r/32)*4
// + g%4), the layout tcgen05.cp.32x128b.warpx4 moves into TMEM.
DEVI size_t sf_offset(int row, int g, int rows_per_block, int col_blocks) {
  const int rb = row / rows_per_block, r = row % rows_per_block;
  return ((size_t)rb * col_blocks + (g >> 2)) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (g & 3);
}

DEVI float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DEVI float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace laya
