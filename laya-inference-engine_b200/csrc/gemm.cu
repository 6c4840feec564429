// Projection GEMM for every Linear of the Laya forward, on tcgen05 tensor
// cores.  Replaces the reference's cuBLAS / Triton / torch._scaled_mm calls
// (src/laya_blackwell/model.py:91,97,100-101,64-69,114;
//  src/laya_blackwell/quantization.py:88-101).
//
// Orientation ("swap AB"): out[m][n] = sum_k X[m][k] * W[n][k].  The weight
// tile (128 rows of W) is the MMA's A operand and sits on the 128 TMEM lanes;
// the token tile (BN rows of X) is the MMA's N dimension.  At batch 1 the
// token count is 64, so the 128-wide MMA M axis is always full.
//
// Pipeline per CTA: thread 0 issues TMA loads (weights first, before the
// programmatic-dependent-launch wait, because weights never depend on the
// previous kernel), thread 32 issues tcgen05.mma into a TMEM accumulator,
// then the epilogue threads move the accumulator out of TMEM.
//
// Split-K: a thread-block cluster of S CTAs shares one output tile, each CTA
// reducing a slice of K.  After the MMAs every CTA parks its fp32 partial in an
// L2 scratch (or, when none is given, its own shared memory), the cluster
// synchronises once, and CTA r sums rows {j, j+64 : j in its token share} over
// all S partials in rank order 0..S-1, so the result is deterministic.  The
// pairing of row j with row j+64 lets the GEGLU epilogue see act and gate of
// one output column together (the packer interleaves Wi in blocks of 64); in
// the QKV tiles rows j and j+32 pair instead, for the rotary embedding.
// Unsplit 128-token tiles use the 256-thread wide epilogue with a TMA store.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "gemm_epilogue.cuh"

#include <cstdio>
#include <mutex>

namespace laya {

template <int BN, int KIND, int STAGES>
struct GemmCfg {
  static constexpr int A_BYTES = 128 * 128;   // 128 weight rows x 128 bytes of K
  static constexpr int B_BYTES = BN * 128;    // BN token rows x 128 bytes of K
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PIPE_BYTES = STAGES * STAGE_BYTES;
  // split-K partial, or the wide epilogue's fp32 tile + bf16 output + row scales
  static constexpr int PART_BYTES = BN >= 128 ? BN * 128 * 4 + BN * 128 * 2 + BN * 4 : BN * 128 * 4;
  static constexpr int MAIN_BYTES = PIPE_BYTES > PART_BYTES ? PIPE_BYTES : PART_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = MAIN_BYTES + BAR_BYTES + 1024;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int K_ELEMS = KIND == kKindBf16 ? 64 : 128;
};

// LNST: the residual epilogue also writes LayerNorm row statistics
// (p.ln_stats) for a following projection that normalises on load.
template <int BN, int KIND, int STAGES, bool LNST = false>
__global__ void __launch_bounds__(BN >= 128 ? 256 : 128, BN == 128 ? 2 : 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ CUtensorMap omap, const GemmParams p) {
  using C = GemmCfg<BN, KIND, STAGES>;
  // All shared memory of the projection kernels is this dynamic block (a
  // static __shared__ variable in the epilogue made the TMA-store epilogue
  // fault with an illegal address; the cause was not established).
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::MAIN_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint64_t* rbar = done + 1;  // residual tile load of the TMA residual epilogue
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

  const uint64_t limit = wait_limit(p.wait_limit_us);
  int issued = 0;  // producer: loads issued (for the drain on failure)
  if (tid == 0) {
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int pre = nkb < STAGES ? nkb : STAGES;
    for (int i = 0; i < pre; ++i) {
      if (i + 1 == p.test_withhold) continue;  // test hook: nothing completes this stage
      mbar_expect_tx(&full[i], C::STAGE_BYTES);
      tma_load_2d(sA + i * C::A_BYTES, &wmap, &full[i], (kb0 + i) * C::K_ELEMS, tile_n * 128, pol_w);
    }
    griddep_wait();
    for (int i = 0; i < pre; ++i)
      if (i + 1 != p.test_withhold)
        tma_load_2d(sB + i * C::B_BYTES, &xmap, &full[i], (kb0 + i) * C::K_ELEMS, tile_m * BN, pol_x);
    issued = pre;
    for (int i = pre; i < nkb; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, limit)) {
        record_status(p.status, kStatusGemmEmptyTimeout);
        atomicExch(failed, 1u);
        break;
      }
      mbar_expect_tx(&full[s], C::STAGE_BYTES);
      tma_load_2d(sA + s * C::A_BYTES, &wmap, &full[s], (kb0 + i) * C::K_ELEMS, tile_n * 128, pol_w);
      tma_load_2d(sB + s * C::B_BYTES, &xmap, &full[s], (kb0 + i) * C::K_ELEMS, tile_m * BN, pol_x);
      issued = i + 1;
    }
  } else if (tid == 32) {
    const uint32_t idesc = KIND == kKindBf16 ? idesc_bf16(128, BN) : idesc_e4m3(128, BN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(&full[s], (i / STAGES) & 1, limit)) {
        record_status(p.status, kStatusGemmFullTimeout);
        atomicExch(failed, 1u);
        break;
      }
      tc_fence_after();
      const uint64_t ad = sw128_desc(smem_u32(sA + s * C::A_BYTES));
      const uint64_t bd = sw128_desc(smem_u32(sB + s * C::B_BYTES));
#pragma unroll
      for (int k = 0; k < 4; ++k) {  // 4 MMAs of 32 bytes of K each; +2 = 32 bytes in the descriptor
        if (KIND == kKindBf16)
          umma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0);
        else
          umma_f8(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0);
      }
      // Only stages that the producer refills get a release; the last STAGES
      // k-blocks are covered by `done`, so no arrive is left in flight when
      // the CTA exits.
      if (i + STAGES < nkb) umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();

  // ---- epilogue: TMEM -> shared partial [BN][128] fp32 -> cluster reduction
  griddep_wait();
  if (!mbar_wait(done, 0, limit)) {
    record_status(p.status, kStatusGemmDoneTimeout);
    atomicExch(failed, 1u);
  }
  tc_fence_after();
  const bool wide = split == 1 && p.tma_epilogue && BN >= 128;
  // unsplit 64-token residual tiles: residual rows in and out by TMA
  const bool tres = BN == 64 && !LNST && split == 1 && p.tma_epilogue && p.epilogue == kEpiResidual;
  if constexpr (BN >= 128) {
    if (wide) tile_epilogue_wide<BN, KIND, 256>(p, &omap, tmem, smem, tile_n, tile_m);
  }
  if constexpr (BN == 64 && !LNST) {
    static_assert(C::MAIN_BYTES >= BN * 1024 + BN * 4, "TMA residual epilogue: accumulator, residual and scale tiles");
    if (tres && !tile_epilogue_resid_tma<BN, KIND>(p, &omap, tmem, smem, rbar, tile_n, tile_m, limit)) {
      record_status(p.status, kStatusGemmDoneTimeout);
      atomicExch(failed, 1u);
    }
  }
  if (!wide && !tres)
    tile_epilogue<BN, KIND, LNST>(p, tmem, reinterpret_cast<float*>(smem), tile_n, tile_m, split, rank);

  // ---- teardown: drain copies still in flight after a failure, free TMEM
  if (tid == 0 && *failed) {
    for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
      mbar_wait(&full[i % STAGES], (i / STAGES) & 1, limit);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------ host side

namespace {

template <int BN, int KIND, int STAGES, bool LNST = false>
cudaError_t launch_one(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap, const GemmParams& p,
                       int tiles_n,
                       int tiles_m, int split, cudaStream_t stream, bool pdl) {
  using C = GemmCfg<BN, KIND, STAGES>;
  auto kern = gemm_kernel<BN, KIND, STAGES, LNST>;
  // Function attributes are per device: set them once for each device used.
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
  return cudaLaunchKernelEx(&cfg, kern, wmap, xmap, omap, p);
}

template <int KIND>
cudaError_t dispatch_bn(int bn, const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap,
                        const GemmParams& p, int tn,
                        int tm, int split, cudaStream_t st, bool pdl) {
  switch (bn) {
    case 16: return launch_one<16, KIND, 4>(wmap, xmap, omap, p, tn, tm, split, st, pdl);
    case 32: return launch_one<32, KIND, 4>(wmap, xmap, omap, p, tn, tm, split, st, pdl);
    case 64: return launch_one<64, KIND, 4>(wmap, xmap, omap, p, tn, tm, split, st, pdl);
    case 128: return launch_one<128, KIND, 3>(wmap, xmap, omap, p, tn, tm, split, st, pdl);
    case 256: return launch_one<256, KIND, 4>(wmap, xmap, omap, p, tn, tm, split, st, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

// Token tile and split-K factor for one projection.  Small token counts use
// one token tile of the smallest MMA width that covers them and split K over
// a cluster until about one wave of CTAs is in flight (weight streaming);
// large token counts use 128-token tiles (about 97 KB of shared memory, so
// two CTAs share an SM and one's epilogue overlaps the other's mainloop;
// measured faster than 256-token tiles at one CTA per SM for 1.5k and 8k
// tokens, and than 64-token tiles wherever the 128-token grid fills the GPU).
void gemm_plan(int M, int N, int kblocks, int sm_count, int* bn_out, int* split_out) {
  (void)N;
  int bn;
  if (M <= 16) bn = 16;
  else if (M <= 32) bn = 32;
  else if (M <= 64) bn = 64;
  else  // 128-token tiles, or 64 when those would leave SMs idle (C3's 512
        // tokens: 1.893 -> 1.805 ms per forward; C2's 1,536: 2.459 -> 2.426)
    bn = (N / 128) * ((M + 127) / 128) < sm_count ? 64 : 128;
  const int tiles = (N / 128) * ((M + bn - 1) / bn);
  *bn_out = bn;
  // token tiles of <= 64 fit two CTAs per SM: split until about two per SM
  // (measured 937 -> 933 us per batch-1 forward)
  *split_out = gemm_split(tiles, kblocks, bn <= 64 ? 2 * sm_count : sm_count, 8);
  // 128-token tiles that leave SMs idle and run a long K loop (Wo2 at 1.5k
  // tokens: 96 tiles x 21 K blocks) split K in two: C2 2.58 -> 2.51 ms (the
  // same for Wo's 8 K blocks measured slower, 2.55 ms)
  if (bn == 128 && *split_out == 1 && tiles < sm_count && kblocks >= 16) *split_out = 2;
}

int gemm_token_tile(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

int gemm_k_elems(int kind) { return kind == kKindBf16 ? 64 : 128; }

// Split-K factor: fill about one wave of the 148 SMs with CTAs when the tile
// grid alone is too small, at least two K blocks per CTA when possible.
int gemm_split(int tiles, int kblocks, int sm_count, int max_split) {
  if (tiles >= sm_count) return 1;
  int s = sm_count / tiles;
  if (s > max_split) s = max_split;
  if (s > kblocks) s = kblocks;
  if (s < 1) s = 1;
  return s;
}

cudaError_t launch_gemm(int kind, const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap,
                        const GemmParams& p, int bn, int split, cudaStream_t stream, bool pdl) {
  const int tiles_n = p.N / 128;
  const int tiles_m = (p.M + bn - 1) / bn;
  if (p.N % 128 || split < 1 || split > 16 || split > p.kblocks) return cudaErrorInvalidValue;
  if (p.ln_stats) {  // batch-1 residual projection feeding a normalise-on-load projection
    if (kind != kKindBf16 || bn != 64 || p.epilogue != kEpiResidual || p.bias || (split == 1 && p.tma_epilogue))
      return cudaErrorInvalidValue;
    // six stages: every weight tile of the CTA's K slice (at most six at
    // batch 1) is requested before the dependency wait; the grid is small
    // enough that one CTA per SM loses nothing (931.8 -> 927.8 us per C1 forward)
    return launch_one<64, kKindBf16, 6, true>(wmap, xmap, omap, p, tiles_n, tiles_m, split, stream, pdl);
  }
  if (kind == kKindBf16) return dispatch_bn<kKindBf16>(bn, wmap, xmap, omap, p, tiles_n, tiles_m, split, stream, pdl);
  if (kind == kKindFp8) return dispatch_bn<kKindFp8>(bn, wmap, xmap, omap, p, tiles_n, tiles_m, split, stream, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace laya
