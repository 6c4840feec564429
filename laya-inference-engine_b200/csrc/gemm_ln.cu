// Projection with its LayerNorm applied on load (batch 1, 32 < tokens <= 64,
// bf16): the encoder's attn_norm / mlp_norm (add_norm,
// src/laya_blackwell/model.py:15-19,90,97) fused into the QKV and Wi
// projections (model.py:91,100) that consume them, so the batch-1 chain has no
// separate LayerNorm launch inside the encoder.
//
// The residual projection before it (Wo2, or Wo with fused attention) writes
// per (token, 128-column tile) statistics of the updated residual rows; this
// kernel merges them per token (Chan et al.'s pairwise update: mean of the
// tile means, M2 = sum of tile M2 + 128 * sum of squared mean deviations),
// then normalises its K slice of the fp32 rows, LN(h) * w rounded to bf16 as
// add_norm does, straight into the MMA's B operand in the 128-byte-swizzled
// K-major layout.  Every weight tile of the CTA's K slice is loaded before
// the programmatic-dependent-launch wait (no stage reuse: at most eight K
// blocks per CTA), the MMA and the split-K epilogue (store with the rotary
// embedding for QKV, GEGLU for Wi) are the projection GEMM's.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "gemm_epilogue.cuh"

#include <mutex>

namespace laya {

namespace {
constexpr int kLnBN = 64;           // token tile: the whole sequence
constexpr int kLnMaxKb = 8;         // K blocks per CTA, all resident
constexpr int kLnMaxTiles = 8;      // 128-column statistics tiles per row (K <= 1024)
constexpr int kLnA = 128 * 128;     // weight tile: 128 rows x 64 bf16
constexpr int kLnX = kLnBN * 128;   // normalised operand: 64 tokens x 64 bf16
constexpr int kLnThreads = 256;
constexpr int kLnPerThread = 6;     // 8-column chunks normalised per thread per round

// Operand region (weights + normalised tiles, or the split-K partial).
__host__ __device__ constexpr int ln_main(int nkb) {
  return nkb * (kLnA + kLnX) > kLnBN * 128 * 4 ? nkb * (kLnA + kLnX) : kLnBN * 128 * 4;
}
// + LayerNorm weight slice, row mean / rstd, barriers, 1024-byte alignment slack
__host__ __device__ constexpr int ln_smem(int nkb) {
  return ln_main(nkb) + kLnMaxKb * 64 * 4 + 2 * kLnBN * 4 + 256 + 1024;
}
}  // namespace

__global__ void __launch_bounds__(kLnThreads, 2)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap wmap, const GemmParams p, const LnParams ln, int nkb_max) {
  // All shared memory is this dynamic block (see gemm.cu).
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sX = smem + nkb_max * kLnA;
  float* s_w = reinterpret_cast<float*>(smem + ln_main(nkb_max));
  float* s_mean = s_w + kLnMaxKb * 64;
  float* s_rstd = s_mean + kLnBN;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_rstd + kLnBN);
  uint64_t* done = full + kLnMaxKb;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  uint32_t* failed = tmem_slot + 1;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile_n = blockIdx.x;
  const int split = gridDim.z, rank = blockIdx.z;
  const int kb0 = (int)((long long)rank * p.kblocks / split);
  const int kb1 = (int)((long long)(rank + 1) * p.kblocks / split);
  const int nkb = kb1 - kb0;  // <= nkb_max <= kLnMaxKb (checked by the launcher)

  griddep_launch_dependents();
  if (tid == 0) {
    for (int i = 0; i < kLnMaxKb; ++i) mbar_init(&full[i], 1);
    mbar_init(done, 1);
    *failed = 0;
    fence_mbar_init();
    prefetch_tensormap(&wmap);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kLnBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {  // the whole weight slice, before the dependency wait
    const uint64_t pol_w = policy_evict_first();
    for (int i = 0; i < nkb; ++i) {
      mbar_expect_tx(&full[i], kLnA);
      tma_load_2d(sA + i * kLnA, &wmap, &full[i], (kb0 + i) * 64, tile_n * 128, pol_w);
    }
  }
  for (int i = tid; i < nkb * 64; i += kLnThreads) s_w[i] = ln.w[kb0 * 64 + i];  // constant
  griddep_wait();

  // normalised operand: chunk c = (K block j, token r, 8 columns q)
  const int nchunks = nkb * kLnBN * 8;
  for (int base = 0; base < nchunks; base += kLnThreads * kLnPerThread) {
    float4 hv[kLnPerThread][2];
#pragma unroll
    for (int u = 0; u < kLnPerThread; ++u) {
      const int c = base + tid + u * kLnThreads;
      const int j = c >> 9, r = (c >> 3) & (kLnBN - 1), q = c & 7;
      hv[u][0] = hv[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < nchunks && r < p.M) {
        const float* src = ln.h + (size_t)r * ln.ldh + (kb0 + j) * 64 + q * 8;
        hv[u][0] = *reinterpret_cast<const float4*>(src);
        hv[u][1] = *reinterpret_cast<const float4*>(src + 4);
      }
    }
    if (base == 0) {
      // row statistics of the CTA's tokens (Chan et al.'s merge of the tile
      // partials), while the first round's loads are in flight
      if (tid < kLnBN) {
        float mean = 0.f, rstd = 0.f;
        if (tid < p.M) {
          const float2* st = ln.stats + (size_t)tid * ln.ntiles;
          float2 part[kLnMaxTiles];
#pragma unroll
          for (int t = 0; t < kLnMaxTiles; ++t) part[t] = t < ln.ntiles ? st[t] : make_float2(0.f, 0.f);
          float sum = 0.f;
#pragma unroll
          for (int t = 0; t < kLnMaxTiles; ++t) sum += t < ln.ntiles ? part[t].x : 0.f;
          mean = sum / (float)ln.ntiles;
          float m2 = 0.f;
#pragma unroll
          for (int t = 0; t < kLnMaxTiles; ++t) {
            const float dm = part[t].x - mean;
            if (t < ln.ntiles) m2 += part[t].y + 128.f * dm * dm;
          }
          rstd = rsqrtf(m2 / (float)(ln.ntiles * 128) + ln.eps);
        }
        s_mean[tid] = mean;
        s_rstd[tid] = rstd;
      }
      __syncthreads();  // s_w, s_mean, s_rstd
    }
#pragma unroll
    for (int u = 0; u < kLnPerThread; ++u) {
      const int c = base + tid + u * kLnThreads;
      if (c >= nchunks) continue;
      const int j = c >> 9, r = (c >> 3) & (kLnBN - 1), q = c & 7;
      const float mean = s_mean[r], rstd = s_rstd[r];
      const float* w = s_w + j * 64 + q * 8;
      const float x[8] = {hv[u][0].x, hv[u][0].y, hv[u][0].z, hv[u][0].w,
                          hv[u][1].x, hv[u][1].y, hv[u][1].z, hv[u][1].w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float y0 = ((x[2 * e] - mean) * rstd) * w[2 * e];
        const float y1 = ((x[2 * e + 1] - mean) * rstd) * w[2 * e + 1];
        __nv_bfloat162 v = __floats2bfloat162_rn(y0, y1);
        o[e] = *reinterpret_cast<uint32_t*>(&v);
      }
      *reinterpret_cast<uint4*>(sX + j * kLnX + r * 128 + ((q ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  fence_proxy_async_smem();  // the operand was written by threads, the MMA reads it
  __syncthreads();

  if (tid == 32) {
    const uint32_t idesc = idesc_bf16(128, kLnBN);
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&full[i], 0)) {
        record_status(p.status, kStatusGemmFullTimeout);
        atomicExch(failed, 1u);
        break;
      }
      tc_fence_after();
      const uint64_t ad = sw128_desc(smem_u32(sA + i * kLnA));
      const uint64_t bd = sw128_desc(smem_u32(sX + i * kLnX));
#pragma unroll
      for (int k = 0; k < 4; ++k) umma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0);
    }
    umma_commit(done);
  }
  __syncwarp();
  if (!mbar_wait(done, 0)) {
    record_status(p.status, kStatusGemmDoneTimeout);
    atomicExch(failed, 1u);
  }
  tc_fence_after();
  tile_epilogue<kLnBN, kKindBf16>(p, tmem, reinterpret_cast<float*>(smem), tile_n, 0, split, rank);

  // teardown: drain weight copies still in flight after a failure, free TMEM
  if (tid == 0 && *failed)
    for (int i = 0; i < nkb; ++i) mbar_wait(&full[i], 0);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kLnBN);
}

cudaError_t launch_gemm_ln(const CUtensorMap& wmap, const GemmParams& p, const LnParams& ln, int split,
                           cudaStream_t stream, bool pdl) {
  if (p.N % 128 || p.M <= 32 || p.M > kLnBN || p.K % 128 || p.kblocks * 64 != p.K || ln.ntiles * 128 != p.K ||
      ln.ntiles > kLnMaxTiles ||
      split < 1 || split > 16 || split > p.kblocks || (p.epilogue != kEpiStore && p.epilogue != kEpiGeglu) ||
      !ln.h || !ln.w || !ln.stats)
    return cudaErrorInvalidValue;
  const int nkb_max = (p.kblocks + split - 1) / split;
  if (nkb_max > kLnMaxKb) return cudaErrorInvalidValue;
  static std::mutex mu;
  static uint64_t ready = 0;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(ready >> dev & 1)) {
      err = cudaFuncSetAttribute(gemm_ln_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ln_smem(kLnMaxKb));
      if (err == cudaSuccess)
        err = cudaFuncSetAttribute(gemm_ln_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (err != cudaSuccess) return err;
      ready |= uint64_t(1) << dev;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.N / 128, 1, split);
  cfg.blockDim = dim3(kLnThreads, 1, 1);
  cfg.dynamicSmemBytes = ln_smem(nkb_max);
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
  return cudaLaunchKernelEx(&cfg, gemm_ln_kernel, wmap, p, ln, nkb_max);
}

}  // namespace laya
