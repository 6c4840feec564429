// Shared tail of the projection GEMMs (bf16, fp8 and nvfp4 mainloops): the
// epilogue arithmetic and the split-K reduction of a 128-row x BN-token fp32
// accumulator from TMEM across a thread-block cluster.
#pragma once
#include "common.cuh"
#include "params.h"

namespace laya {

// Epilogue for 4 consecutive weight rows n_lo..n_lo+3 and their partners
// n_lo+64..n_lo+67 of one token m (lo/hi hold the fp32 accumulators).
template <int KIND>
DEVI void epilogue_quad(const GemmParams& p, int m, int n_lo, int geglu_col, float4 lo, float4 hi) {
  float l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
  const int n_hi = n_lo + 64;
  if (KIND == kKindFp8) {
    const float sa = p.a_scale[m];
    const float4 wl = *reinterpret_cast<const float4*>(p.w_scale + n_lo);
    const float4 wh = *reinterpret_cast<const float4*>(p.w_scale + n_hi);
    const float wlv[4] = {wl.x, wl.y, wl.z, wl.w}, whv[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      l[e] = (l[e] * sa) * wlv[e];
      h[e] = (h[e] * sa) * whv[e];
    }
  } else if (KIND == kKindNvfp4) {
    const float sa = p.a_scale[m] * p.w_tensor_scale;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      l[e] *= sa;
      h[e] *= sa;
    }
  }
  if (p.epilogue == kEpiGeglu) {
    __nv_bfloat16 o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = bf16_round(l[e]), g = bf16_round(h[e]);
      o[e] = __float2bfloat16_rn(bf16_round(gelu_erf(a)) * g);
    }
    *reinterpret_cast<uint2*>(p.out + (size_t)m * p.ldo + geglu_col) = *reinterpret_cast<uint2*>(o);
    return;
  }
  if (p.bias) {
    const uint2 bl = *reinterpret_cast<const uint2*>(p.bias + n_lo);
    const uint2 bh = *reinterpret_cast<const uint2*>(p.bias + n_hi);
    const __nv_bfloat16* bla = reinterpret_cast<const __nv_bfloat16*>(&bl);
    const __nv_bfloat16* bha = reinterpret_cast<const __nv_bfloat16*>(&bh);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      l[e] += __bfloat162float(bla[e]);
      h[e] += __bfloat162float(bha[e]);
    }
  }
  if (p.epilogue == kEpiResidual) {
    float4* rl = reinterpret_cast<float4*>(p.resid + (size_t)m * p.ldr + n_lo);
    float4* rh = reinterpret_cast<float4*>(p.resid + (size_t)m * p.ldr + n_hi);
    float4 a = *rl, b = *rh;
    a.x += bf16_round(l[0]); a.y += bf16_round(l[1]); a.z += bf16_round(l[2]); a.w += bf16_round(l[3]);
    b.x += bf16_round(h[0]); b.y += bf16_round(h[1]); b.z += bf16_round(h[2]); b.w += bf16_round(h[3]);
    *rl = a;
    *rh = b;
    return;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (p.epilogue == kEpiRelu) {
      l[e] = fmaxf(l[e], 0.f);
      h[e] = fmaxf(h[e], 0.f);
    } else if (p.epilogue == kEpiGelu) {
      l[e] = gelu_erf(bf16_round(l[e]));
      h[e] = gelu_erf(bf16_round(h[e]));
    }
  }
  __nv_bfloat16 ol[4], oh[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    ol[e] = __float2bfloat16_rn(l[e]);
    oh[e] = __float2bfloat16_rn(h[e]);
  }
  __nv_bfloat16* o = p.out + (size_t)m * p.ldo;
  *reinterpret_cast<uint2*>(o + n_lo) = *reinterpret_cast<uint2*>(ol);
  *reinterpret_cast<uint2*>(o + n_hi) = *reinterpret_cast<uint2*>(oh);
}

// TMEM accumulator -> shared partial -> cluster reduction -> epilogue.
// Called by all 128 threads after the MMA-done barrier completed.
// `part` is this CTA's shared scratch of at least BN*128 floats (the
// pipeline region, free once every MMA has completed).
template <int BN, int KIND>
DEVI void tile_epilogue(const GemmParams& p, uint32_t tmem, float* part, int tile_n, int tile_m, int split,
                        int rank) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  if (BN >= 32) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(lane_addr + c, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) part[(c + j) * 128 + tid] = __uint_as_float(r[j]);
    }
  } else {
    uint32_t r[16];
    tmem_ld16(lane_addr, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) part[j * 128 + tid] = __uint_as_float(r[j]);
  }
  tc_fence_before();
  if (split > 1)
    cluster_sync_all();
  else
    __syncthreads();

  // ---- reduction over the cluster and the epilogue.  CTA `rank` owns the
  // tokens [t0, t1) of the tile; a thread takes 4 consecutive rows (and their
  // +64 partners) of one token and sums the S partials in rank order with
  // 16-byte DSMEM loads issued back to back.
  const int t0 = rank * BN / split, t1 = (rank + 1) * BN / split, nt = t1 - t0;
  const uint32_t part_addr = smem_u32(part);
  for (int item = tid; item < nt * 16; item += 128) {
    const int tl = t0 + (item >> 4);
    const int q4 = (item & 15) * 4;
    const int m = tile_m * BN + tl;
    if (m >= p.M) continue;
    const int off = tl * 128 + q4;
    float4 lo, hi;
    if (split == 1) {
      lo = *reinterpret_cast<const float4*>(part + off);
      hi = *reinterpret_cast<const float4*>(part + off + 64);
    } else {
      lo = make_float4(0.f, 0.f, 0.f, 0.f);
      hi = lo;
      // all remote loads of up to 8 peers are issued before any add
      for (int q0 = 0; q0 < split; q0 += 8) {
        float4 va[8], vb[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (q0 + u < split) {
            const uint32_t base = mapa_shared(part_addr, (uint32_t)(q0 + u));
            va[u] = ld_dsmem_f32x4(base + off * 4);
            vb[u] = ld_dsmem_f32x4(base + (off + 64) * 4);
          }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (q0 + u < split) {
            lo.x += va[u].x; lo.y += va[u].y; lo.z += va[u].z; lo.w += va[u].w;
            hi.x += vb[u].x; hi.y += vb[u].y; hi.z += vb[u].z; hi.w += vb[u].w;
          }
      }
    }
    epilogue_quad<KIND>(p, m, tile_n * 128 + q4, tile_n * 64 + q4, lo, hi);
  }
  if (split > 1) cluster_sync_all();

}

}  // namespace laya
