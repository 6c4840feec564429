// NVFP4 projections: e2m1 values with one ue4m3 scale per 16 elements, an
// fp32 outer scale per weight tensor and per activation row.  Follows the
// reference's NVFP4 experiment (experiments/frontier/nvfp4.py:29-92: 2^-9
// scale floor, cvt.rn.satfinite rounding, the 128x4 scale-block layout of
// :55-62) with the weight outer scale per tensor instead of per row.
//
// Kernel: tcgen05.mma kind::mxf4nvf4.block_scale.scale_vec::4X.  Per 128-byte
// k-block (256 elements) a stage holds the A tile (128 weight rows), the B
// tile (BN tokens), and the four 512-byte scale blocks of each operand; the
// MMA thread moves the scale blocks into TMEM with tcgen05.cp (32x128b,
// replicated to the four lane quarters) and issues 4 MMAs of K=64.  The
// accumulator epilogue and cluster split-K reduction are the shared ones.
//
// Scale layout in global memory (weights and activations alike): blocks of
// 128 rows x 4 scale columns, 512 bytes, byte (r%32)*16 + (r/32)*4 + j; block
// (row_block, col_block) at ((row_block * col_blocks) + col_block) * 512, the
// column blocks padded to a multiple of 4 (one k-block) with zero scales.
// Activation row blocks hold one token tile (BN <= 128 tokens) each.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "gemm_epilogue.cuh"

#include <mutex>

namespace laya {

namespace {

DEVI void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Smem descriptor of one 512-byte scale block (32 rows x 16 bytes, no swizzle).
DEVI uint64_t sf_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;          // leading byte offset (one 16-byte column)
  d |= (uint64_t)(128 >> 4) << 32; // 8-row core matrices are 128 bytes apart
  d |= (uint64_t)1 << 46;          // sm_100 descriptor version; layout type 0 = no swizzle
  return d;
}

__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  // e2m1 x e2m1 (format 1), ue4m3 scales (bit 23 = 0), K-major, fp32 accumulate
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

}  // namespace

template <int BN, int STAGES>
struct Nvf4Cfg {
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int SF_BYTES = 2048;  // four 512-byte scale blocks per operand per k-block
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + 2 * SF_BYTES;
  static constexpr int PIPE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int PART_BYTES = BN >= 128 ? BN * 128 * 4 + BN * 128 * 2 + BN * 4 : BN * 128 * 4;
  static constexpr int MAIN_BYTES = PIPE_BYTES > PART_BYTES ? PIPE_BYTES : PART_BYTES;
  static constexpr int SMEM = MAIN_BYTES + 256 + 1024;
  static constexpr int TMEM_NEED = BN + STAGES * 32;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128 : TMEM_NEED <= 256 ? 256 : 512;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(BN >= 128 ? 256 : 128, BN == 128 ? 2 : 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap omap, const uint8_t* __restrict__ wsf,
                      const uint8_t* __restrict__ xsf, int sf_kbs, const GemmParams p) {
  using C = Nvf4Cfg<BN, STAGES>;
  // All shared memory of the projection kernels is this dynamic block (a
  // static __shared__ variable in the epilogue made the TMA-store epilogue
  // fault with an illegal address; the cause was not established).
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* sSFA = sB + STAGES * C::B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * C::SF_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::MAIN_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint64_t* rbar = done + 1;  // residual tile load of the TMA epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  uint32_t* failed = tmem_slot + 1;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile_n = blockIdx.x, tile_m = blockIdx.y;
  const int split = gridDim.z, rank = blockIdx.z;
  const int kb0 = (int)((long long)rank * p.kblocks / split);
  const int kb1 = (int)((long long)(rank + 1) * p.kblocks / split);
  const int nkb = kb1 - kb0;

  griddep_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(rbar, 1);
    *failed = 0;
    fence_mbar_init();
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint8_t* wsf_tile = wsf + (size_t)tile_n * sf_kbs * C::SF_BYTES;
  const uint8_t* xsf_tile = xsf + (size_t)tile_m * sf_kbs * C::SF_BYTES;
  int issued = 0;
  if (tid == 0) {
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int pre = nkb < STAGES ? nkb : STAGES;
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], C::STAGE_BYTES);
      tma_load_2d(sA + i * C::A_BYTES, &wmap, &full[i], (kb0 + i) * 128, tile_n * 128, pol_w);
      bulk_load(sSFA + i * C::SF_BYTES, wsf_tile + (size_t)(kb0 + i) * C::SF_BYTES, C::SF_BYTES, &full[i], pol_w);
    }
    griddep_wait();
    for (int i = 0; i < pre; ++i) {
      tma_load_2d(sB + i * C::B_BYTES, &xmap, &full[i], (kb0 + i) * 128, tile_m * BN, pol_x);
      bulk_load(sSFB + i * C::SF_BYTES, xsf_tile + (size_t)(kb0 + i) * C::SF_BYTES, C::SF_BYTES, &full[i], pol_x);
    }
    issued = pre;
    for (int i = pre; i < nkb; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(&empty[s], ((i / STAGES) - 1) & 1)) {
        record_status(p.status, kStatusGemmEmptyTimeout);
        atomicExch(failed, 1u);
        break;
      }
      mbar_expect_tx(&full[s], C::STAGE_BYTES);
      tma_load_2d(sA + s * C::A_BYTES, &wmap, &full[s], (kb0 + i) * 128, tile_n * 128, pol_w);
      bulk_load(sSFA + s * C::SF_BYTES, wsf_tile + (size_t)(kb0 + i) * C::SF_BYTES, C::SF_BYTES, &full[s], pol_w);
      tma_load_2d(sB + s * C::B_BYTES, &xmap, &full[s], (kb0 + i) * 128, tile_m * BN, pol_x);
      bulk_load(sSFB + s * C::SF_BYTES, xsf_tile + (size_t)(kb0 + i) * C::SF_BYTES, C::SF_BYTES, &full[s], pol_x);
      issued = i + 1;
    }
  } else if (tid == 32) {
    const uint32_t idesc = idesc_nvf4(128, BN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
        record_status(p.status, kStatusGemmFullTimeout);
        atomicExch(failed, 1u);
        break;
      }
      tc_fence_after();
      const uint32_t t_sfa = tmem + (uint32_t)(BN + s * 32);
      const uint32_t t_sfb = t_sfa + 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tmem_cp_32x128b_warpx4(t_sfa + 4 * j, sf_desc(smem_u32(sSFA + s * C::SF_BYTES + 512 * j)));
        tmem_cp_32x128b_warpx4(t_sfb + 4 * j, sf_desc(smem_u32(sSFB + s * C::SF_BYTES + 512 * j)));
      }
      const uint64_t ad = sw128_desc(smem_u32(sA + s * C::A_BYTES));
      const uint64_t bd = sw128_desc(smem_u32(sB + s * C::B_BYTES));
#pragma unroll
      for (int j = 0; j < 4; ++j)  // K = 64 elements = 32 bytes per MMA
        umma_nvf4(tmem, ad + 2 * j, bd + 2 * j, idesc, t_sfa + 4 * j, t_sfb + 4 * j, (i | j) != 0);
      // Only stages that the producer refills get a release; the last STAGES
      // k-blocks are covered by `done`, so no arrive is left in flight when
      // the CTA exits.
      if (i + STAGES < nkb) umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();

  griddep_wait();
  if (!mbar_wait(done, 0)) {
    record_status(p.status, kStatusGemmDoneTimeout);
    atomicExch(failed, 1u);
  }
  tc_fence_after();
  const bool wide = split == 1 && p.tma_epilogue && BN >= 128;
  if constexpr (BN >= 128) {
    if (wide) tile_epilogue_wide<BN, kKindNvfp4, 256>(p, &omap, tmem, smem, tile_n, tile_m);
  }
  if (!wide) tile_epilogue<BN, kKindNvfp4>(p, tmem, reinterpret_cast<float*>(smem), tile_n, tile_m, split, rank);

  // ---- teardown: drain copies still in flight after a failure, free TMEM
  if (tid == 0 && *failed) {
    for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
      mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------- quantisers


// One warp per row: 16-element blocks -> ue4m3 scale + 16 e2m1 nibbles.
// outer > 0: fixed outer scale (weights, per tensor); outer <= 0: per-row
// outer = max(amax/(6*448), 1e-20) written to row_outer (activations).
DEVI void nvfp4_row(const __nv_bfloat16* src, int k, float outer, float* row_outer, uint8_t* q, uint8_t* sf, int row,
                    int rows_per_block, int col_blocks, int lane) {
  if (outer <= 0.f) {
    float amax = 0.f;
    for (int c = lane * 8; c < k; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(__bfloat162float(e[j])));
    }
    amax = warp_max(amax);
    outer = fmaxf(amax / (6.0f * 448.0f), 1e-20f);
    if (lane == 0 && row_outer) *row_outer = outer;
  }
  for (int g = lane; g < k / 16; g += 32) {
    float x[16];
    const uint4 u0 = *reinterpret_cast<const uint4*>(src + g * 16);
    const uint4 u1 = *reinterpret_cast<const uint4*>(src + g * 16 + 8);
    const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&u0);
    const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&u1);
    float bmax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = __bfloat162float(e0[j]);
      x[8 + j] = __bfloat162float(e1[j]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) bmax = fmaxf(bmax, fabsf(x[j]));
    const float sc = fmaxf(bmax / (6.0f * outer), 0.001953125f);  // 2^-9 floor
    const uint8_t sc8 = (uint8_t)(f32x2_to_e4m3x2(sc, 0.f) & 0xFF);
    // decode the e4m3 scale exactly (1 sign, 4 exponent, 3 mantissa bits, bias 7)
    const float scale = e4m3_value(sc8);
    const float denom = scale * outer;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      w0 |= (uint32_t)f32x2_to_e2m1x2(x[j] / denom, x[j + 1] / denom) << (4 * j);
      w1 |= (uint32_t)f32x2_to_e2m1x2(x[8 + j] / denom, x[8 + j + 1] / denom) << (4 * j);
    }
    *reinterpret_cast<uint2*>(q + g * 8) = make_uint2(w0, w1);
    sf[sf_offset(row, g, rows_per_block, col_blocks)] = sc8;
  }
}

__global__ void __launch_bounds__(256) nvfp4_amax_kernel(const __nv_bfloat16* w, size_t n, unsigned int* amax_bits) {
  float m = 0.f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(w[i])));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

__global__ void __launch_bounds__(256) nvfp4_pack_weight_kernel(const __nv_bfloat16* w, int rows, int k,
                                                                const unsigned int* amax_bits, uint8_t* q,
                                                                uint8_t* sf, int col_blocks, float* tensor_scale) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const float outer = fmaxf(__uint_as_float(*amax_bits) / (6.0f * 448.0f), 1e-20f);
  if (row == 0 && lane == 0) *tensor_scale = outer;
  if (row >= rows) return;
  nvfp4_row(w + (size_t)row * k, k, outer, nullptr, q + (size_t)row * (k / 2), sf, row, 128, col_blocks, lane);
}

// Activation quantiser: one CTA of 128 threads per row (k <= 1024*MAXC), the
// same values as nvfp4_row with a per-row outer scale.  Each thread holds
// elements [8t + 1024i, +8) in registers (every load in flight at once), so a
// 16-element block is split over a thread pair and its maximum takes one
// shuffle; the row maximum is a warp then CTA reduction; quotients use the
// FMA-corrected division (correctly rounded).
template <int MAXC>
__global__ void __launch_bounds__(128) quant_nvfp4_kernel(const QuantParams p, int rows_per_block, int col_blocks) {
  __shared__ float s_max[4];
  griddep_launch_dependents();
  griddep_wait();
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (row >= p.rows) return;
  const __nv_bfloat16* src = p.src + (size_t)row * p.k;
  uint4 u[MAXC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid * 8 + 1024 * i;
    u[i] = c < p.k ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(__bfloat162float(e[j])));
  }
  amax = warp_max(amax);
  if (lane == 0) s_max[warp] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(s_max[0], s_max[1]), fmaxf(s_max[2], s_max[3]));
  const float outer = fmaxf(amax / (6.0f * 448.0f), 1e-20f);
  if (tid == 0) p.scale[row] = outer;
  const float o6 = 6.0f * outer, inv_o6 = 1.0f / o6;
  uint8_t* q = p.q + (size_t)row * (p.k / 2);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid * 8 + 1024 * i;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
    float x[8], bmax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = __bfloat162float(e[j]);
      bmax = fmaxf(bmax, fabsf(x[j]));
    }
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));  // the thread pair of one 16-element block
    if (c >= p.k) continue;
    const float sc = fmaxf(div_rn_by(bmax, o6, inv_o6), 0.001953125f);  // 2^-9 floor
    const uint8_t sc8 = (uint8_t)(f32x2_to_e4m3x2(sc, 0.f) & 0xFF);
    const float scale = e4m3_value(sc8);
    const float denom = scale * outer, inv_d = 1.0f / denom;
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; j += 2)
      w |= (uint32_t)f32x2_to_e2m1x2(div_rn_by(x[j], denom, inv_d), div_rn_by(x[j + 1], denom, inv_d)) << (4 * j);
    *reinterpret_cast<uint32_t*>(q + c / 2) = w;
    if ((tid & 1) == 0) p.sf[sf_offset(row, c / 16, rows_per_block, col_blocks)] = sc8;
  }
}

// The same quantisation with one warp per row, for large row counts (from
// 2,048 rows): chunk c = lane + 32 i of 8 elements, so a 16-element block is
// the chunk pair of lanes (2m, 2m+1) and its maximum takes one shuffle.
// Arithmetic identical to quant_nvfp4_kernel.
template <int CPL>
__global__ void __launch_bounds__(256) quant_nvfp4_warp_kernel(const QuantParams p, int rows_per_block,
                                                               int col_blocks) {
  griddep_launch_dependents();
  griddep_wait();
  const int lane = threadIdx.x & 31, row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int chunks = p.k / 8;
  const __nv_bfloat16* src = p.src + (size_t)row * p.k;
  uint4 u[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    u[i] = c < chunks ? reinterpret_cast<const uint4*>(src)[c] : make_uint4(0, 0, 0, 0);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(__bfloat162float(e[j])));
  }
  amax = warp_max(amax);
  const float outer = fmaxf(amax / (6.0f * 448.0f), 1e-20f);
  if (lane == 0) p.scale[row] = outer;
  const float o6 = 6.0f * outer, inv_o6 = 1.0f / o6;
  uint8_t* q = p.q + (size_t)row * (p.k / 2);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
    float x[8], bmax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = __bfloat162float(e[j]);
      bmax = fmaxf(bmax, fabsf(x[j]));
    }
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));  // the lane pair of one 16-element block
    if (c >= chunks) continue;
    const float sc = fmaxf(div_rn_by(bmax, o6, inv_o6), 0.001953125f);  // 2^-9 floor
    const uint8_t sc8 = (uint8_t)(f32x2_to_e4m3x2(sc, 0.f) & 0xFF);
    const float scale = e4m3_value(sc8);
    const float denom = scale * outer, inv_d = 1.0f / denom;
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; j += 2)
      w |= (uint32_t)f32x2_to_e2m1x2(div_rn_by(x[j], denom, inv_d), div_rn_by(x[j + 1], denom, inv_d)) << (4 * j);
    reinterpret_cast<uint32_t*>(q)[c] = w;
    if ((lane & 1) == 0) p.sf[sf_offset(row, c / 2, rows_per_block, col_blocks)] = sc8;
  }
}

// ------------------------------------------------------------- host side

namespace {
template <int BN, int STAGES>
cudaError_t launch_nvf4(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap, const uint8_t* wsf,
                        const uint8_t* xsf,
                        int sf_kbs, const GemmParams& p, int tiles_n, int tiles_m, int split, cudaStream_t stream,
                        bool pdl) {
  using C = Nvf4Cfg<BN, STAGES>;
  auto kern = gemm_nvfp4_kernel<BN, STAGES>;
  static std::mutex mu;
  static uint64_t ready = 0;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(ready >> dev & 1)) {
      err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
      if (err == cudaSuccess) err = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (err != cudaSuccess) return err;
      ready |= uint64_t(1) << dev;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles_n, tiles_m, split);
  cfg.blockDim = dim3(BN >= 128 ? 256 : 128, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (split > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = split;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, wmap, xmap, omap, wsf, xsf, sf_kbs, p);
}
}  // namespace

cudaError_t launch_gemm_nvfp4(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap,
                              const uint8_t* wsf,
                              const uint8_t* xsf, int sf_kbs, const GemmParams& p, int bn, int split,
                              cudaStream_t stream, bool pdl) {
  const int tiles_n = p.N / 128;
  const int tiles_m = (p.M + bn - 1) / bn;
  if (p.N % 128 || split < 1 || split > 16 || split > p.kblocks) return cudaErrorInvalidValue;
  switch (bn) {
    case 16: return launch_nvf4<16, 4>(wmap, xmap, omap, wsf, xsf, sf_kbs, p, tiles_n, tiles_m, split, stream, pdl);
    case 32: return launch_nvf4<32, 4>(wmap, xmap, omap, wsf, xsf, sf_kbs, p, tiles_n, tiles_m, split, stream, pdl);
    case 64: return launch_nvf4<64, 3>(wmap, xmap, omap, wsf, xsf, sf_kbs, p, tiles_n, tiles_m, split, stream, pdl);
    case 128: return launch_nvf4<128, 3>(wmap, xmap, omap, wsf, xsf, sf_kbs, p, tiles_n, tiles_m, split, stream, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_nvfp4_pack_weight(const __nv_bfloat16* w, int rows, int k, unsigned int* amax_scratch, uint8_t* q,
                                     uint8_t* sf, int col_blocks, float* tensor_scale, cudaStream_t stream) {
  cudaError_t err = cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int), stream);
  if (err != cudaSuccess) return err;
  nvfp4_amax_kernel<<<296, 256, 0, stream>>>(w, (size_t)rows * k, amax_scratch);
  nvfp4_pack_weight_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(w, rows, k, amax_scratch, q, sf, col_blocks,
                                                              tensor_scale);
  return cudaGetLastError();
}

cudaError_t launch_quant_nvfp4(const QuantParams& p, int rows_per_block, int col_blocks, cudaStream_t stream,
                               bool pdl) {
  if (p.k % 16 || p.k > 4096) return cudaErrorInvalidValue;
  QuantParams q = p;
  void* args[] = {&q, &rows_per_block, &col_blocks};
  if (p.rows >= 2048) {  // a warp per row (same switch as the FP8 quantiser and the LayerNorm rows)
    const int cpl = (p.k / 8 + 31) / 32;
    const void* wk = cpl <= 4    ? (const void*)quant_nvfp4_warp_kernel<4>
                     : cpl <= 8  ? (const void*)quant_nvfp4_warp_kernel<8>
                     : cpl <= 12 ? (const void*)quant_nvfp4_warp_kernel<12>
                                 : (const void*)quant_nvfp4_warp_kernel<16>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.rows + 7) / 8, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, wk, args);
  }
  const void* kern = p.k <= 1024   ? (const void*)quant_nvfp4_kernel<1>
                     : p.k <= 2048 ? (const void*)quant_nvfp4_kernel<2>
                     : p.k <= 3072 ? (const void*)quant_nvfp4_kernel<3>
                                   : (const void*)quant_nvfp4_kernel<4>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.rows, 1, 1);  // one CTA of 128 threads per row
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

}  // namespace laya
