// Fused attention + output projection for one short sequence (batch 1,
// 32 < s <= 64, bf16): the encoder's SDPA (src/laya_blackwell/model.py:92-96)
// computed inside the split-K CTAs of the Wo projection (model.py:97) that
// consume it, so the attention output never leaves shared memory and the
// layer saves one dependent launch.
//
// Each CTA of the Wo grid owns one 128-row weight tile and a K slice of whole
// heads (a K block of 64 bf16 is one head).  After the weight tiles are in
// flight (before the programmatic-dependent-launch wait), it copies q, k and v
// of two heads at a time from the QKV buffer (already rotated by the QKV
// projection's epilogue) with cp.async; warps 0-3 and 4-7 each compute one
// head's attention for the 64 query positions with register-level
// tensor-core tiles (attention_tile.cuh: at 64 tokens shorter than a
// tensor-memory round trip) and write the bf16 output straight into the MMA's
// B operand stage, in the 128-byte-swizzled K-major layout a TMA load would
// have produced.  The MMA, the split-K reduction and the residual epilogue are
// the projection GEMM's; the epilogue also writes the LayerNorm statistics of
// the updated residual rows for the MLP projection, which normalises on load.
// Every CTA recomputes its heads for its own weight tile: at 64 tokens that is
// cheaper than a separate launch.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "gemm_epilogue.cuh"
#include "attention_tile.cuh"

#include <mutex>

namespace laya {

namespace {
using namespace attn;

constexpr int kFaBN = 64;                    // token tile: the whole sequence
constexpr int kFaStages = 4;                 // most heads (K blocks) per CTA
constexpr int kFaThreads = 256;              // two heads in flight, four warps each
constexpr int kFaA = 128 * 128;              // weight tile: 128 rows x 64 bf16
constexpr int kFaB = kFaBN * 128;            // attention output: 64 tokens x 64 bf16
constexpr int kFaTile = AQ * LDS * 2;        // one staged Q / K / V tile
constexpr int kFaPipe = kFaStages * (kFaA + kFaB) + 2 * 3 * kFaTile;
constexpr int kFaPart = kFaBN * 128 * 4;     // split-K partial when kept in shared memory
constexpr int kFaMain = kFaPipe > kFaPart ? kFaPipe : kFaPart;
constexpr int kFaSmem = kFaMain + 256 + 1024;
}  // namespace

__global__ void __launch_bounds__(kFaThreads, 1)
    gemm_attn_kernel(const __grid_constant__ CUtensorMap wmap, const GemmParams p, const AttnParams a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_kvalid[AK];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kFaStages * kFaA;
  __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(sB + kFaStages * kFaB);  // [2 heads][Q, K, V]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kFaMain);
  uint64_t* done = full + kFaStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  uint32_t* failed = tmem_slot + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile_n = blockIdx.x;
  const int split = gridDim.z, rank = blockIdx.z;
  const int kb0 = (int)((long long)rank * p.kblocks / split);
  const int kb1 = (int)((long long)(rank + 1) * p.kblocks / split);
  const int nkb = kb1 - kb0;  // <= kFaStages (checked by the launcher)

  griddep_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < kFaStages; ++s) mbar_init(&full[s], 1);
    mbar_init(done, 1);
    *failed = 0;
    fence_mbar_init();
    prefetch_tensormap(&wmap);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kFaBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {  // every weight tile of the slice, before the dependency wait
    const uint64_t pol_w = policy_evict_first();
    for (int i = 0; i < nkb; ++i) {
      mbar_expect_tx(&full[i], kFaA);
      tma_load_2d(sA + i * kFaA, &wmap, &full[i], (kb0 + i) * 64, tile_n * 128, pol_w);
    }
  }
  griddep_wait();

  const int slot = warp >> 2, qw = warp & 3;  // head slot, query quarter
  const int g = lane >> 2, t4 = lane & 3;
  const int qp0 = qw * 16 + g < a.s ? qw * 16 + g : -1;
  const int qp1 = qw * 16 + g + 8 < a.s ? qw * 16 + g + 8 : -1;
  for (int j0 = 0; j0 < nkb; j0 += 2) {
    // q, k, v of heads kb0+j0 and kb0+j0+1: 2 x 3 x 64 rows x 8 chunks of 16 bytes
    for (int it = tid; it < 2 * 3 * AQ * 8; it += kFaThreads) {
      const int hs = it / (3 * AQ * 8), rem = it % (3 * AQ * 8);
      const int part = rem / (AQ * 8), r = (rem >> 3) & (AQ - 1), c = (rem & 7) * 8;
      const bool ok = j0 + hs < nkb && r < a.s;
      const __nv_bfloat16* src = ok ? a.qkv + (size_t)r * a.ld_qkv + part * a.d + (kb0 + j0 + hs) * 64 + c : a.qkv;
      cp_async16(stage + (hs * 3 + part) * AQ * LDS + r * LDS + c, src, ok);
    }
    if (j0 == 0 && tid < AK) cp_async4(&s_kvalid[tid], a.key_valid + (tid < a.s ? tid : 0), tid < a.s);
    cp_commit();
    cp_wait_all();
    __syncthreads();
    const int j = j0 + slot;
    if (j < nkb) {
      const __nv_bfloat16* sQ = stage + slot * 3 * AQ * LDS;
      uint32_t qf[4][4];
      load_q_frags(qf, sQ, qw, lane);
      Acc acc;
      acc_init(acc);
      attend_tile(acc, qf, sQ + AQ * LDS, sQ + 2 * AQ * LDS, s_kvalid, 0, a.window, qp0, qp1, lane);
      // normalised bf16 rows -> B stage j: token row r holds 8 chunks of 16
      // bytes, chunk c stored at position c ^ (r & 7) (128-byte swizzle)
      uint8_t* ob = sB + j * kFaB;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float l = acc.lrow[r];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int row = qw * 16 + g + 8 * r;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<uint32_t*>(ob + row * 128 + ((nt ^ (row & 7)) << 4) + t4 * 4) =
              pack_bf16(acc.o[nt][2 * r] * inv, acc.o[nt][2 * r + 1] * inv);
      }
    }
    __syncthreads();  // the staging tiles are refilled for the next pair of heads
  }
  fence_proxy_async_smem();  // the B stages were written by threads, the MMA reads them
  __syncthreads();

  if (tid == 32) {
    const uint32_t idesc = idesc_bf16(128, kFaBN);
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&full[i], 0)) {
        record_status(p.status, kStatusGemmFullTimeout);
        atomicExch(failed, 1u);
        break;
      }
      tc_fence_after();
      const uint64_t ad = sw128_desc(smem_u32(sA + i * kFaA));
      const uint64_t bd = sw128_desc(smem_u32(sB + i * kFaB));
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
  tile_epilogue<kFaBN, kKindBf16, true>(p, tmem, reinterpret_cast<float*>(smem), tile_n, 0, split, rank);

  // teardown: drain weight copies still in flight after a failure, free TMEM
  if (tid == 0 && *failed)
    for (int i = 0; i < nkb; ++i) mbar_wait(&full[i], 0);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kFaBN);
}

cudaError_t launch_gemm_attn(const CUtensorMap& wmap, const GemmParams& p, const AttnParams& a, int split,
                             cudaStream_t stream, bool pdl) {
  if (p.N % 128 || p.M <= 32 || p.M > kFaBN || a.s != p.M || split < 1 || split > 16 || split > p.kblocks ||
      p.kblocks * 64 != p.K || p.K != a.d || p.epilogue != kEpiResidual || a.q_pos || a.nq != a.s ||
      !p.ln_stats || p.bias)
    return cudaErrorInvalidValue;
  if ((p.kblocks + split - 1) / split > kFaStages) return cudaErrorInvalidValue;
  static std::mutex mu;
  static uint64_t ready = 0;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(ready >> dev & 1)) {
      err = cudaFuncSetAttribute(gemm_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem);
      if (err == cudaSuccess)
        err = cudaFuncSetAttribute(gemm_attn_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (err != cudaSuccess) return err;
      ready |= uint64_t(1) << dev;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.N / 128, 1, split);
  cfg.blockDim = dim3(kFaThreads, 1, 1);
  cfg.dynamicSmemBytes = kFaSmem;
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
  return cudaLaunchKernelEx(&cfg, gemm_attn_kernel, wmap, p, a);
}

}  // namespace laya
