// Shared tail of the projection kernels (bf16, fp8 and nvfp4 mainloops, the
// fused attention and LayerNorm-on-load kernels): the epilogue arithmetic
// (scales, bias, RoPE, activations, GEGLU, residual, LayerNorm statistics),
// the split-K reduction of a 128-row x BN-token fp32 accumulator from TMEM
// across a thread-block cluster, and the wide epilogue of unsplit tiles.
#pragma once
#include "common.cuh"
#include "params.h"

namespace laya {

// Global operands of one epilogue item that do not depend on the split-K
// partials: the activation row scale, the residual rows (residual epilogues)
// and the rotary table entries (rotary tiles).  Loaded together with the
// partials so that an item costs one memory round trip.
struct EpiPre {
  float sa;
  float4 ra, rb;  // residual rows n_lo.., n_lo+64..
  float4 c0, s0;  // cos / sin at d0 (the tables repeat their first 32
                  // columns, so these serve d0+32 as well)
};

template <int KIND>
DEVI EpiPre epi_prefetch(const GemmParams& p, int m, int n_lo, bool residual, bool rope) {
  EpiPre e;
  e.sa = KIND == kKindBf16 ? 1.f : p.a_scale[m];
  if (residual) {
    e.ra = __ldcg(reinterpret_cast<const float4*>(p.resid + (size_t)m * p.ldr + n_lo));
    e.rb = __ldcg(reinterpret_cast<const float4*>(p.resid + (size_t)m * p.ldr + n_lo + 64));
  }
  if (rope) {
    const int pos = m % p.rope_seq, d0 = n_lo & 63;
    e.c0 = *reinterpret_cast<const float4*>(p.rope_cos + (size_t)pos * 64 + d0);
    e.s0 = *reinterpret_cast<const float4*>(p.rope_sin + (size_t)pos * 64 + d0);
  }
  return e;
}

// Epilogue for 4 consecutive weight rows n_lo..n_lo+3 and their partners
// n_lo+64..n_lo+67 of one token m (lo/hi hold the fp32 accumulators).
template <int KIND>
DEVI void epilogue_quad(const GemmParams& p, int m, int n_lo, int geglu_col, float4 lo, float4 hi, const EpiPre& pre) {
  float l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
  const int n_hi = n_lo + 64;
  if (KIND == kKindFp8) {
    const float sa = pre.sa;
    const float4 wl = *reinterpret_cast<const float4*>(p.w_scale + n_lo);
    const float4 wh = *reinterpret_cast<const float4*>(p.w_scale + n_hi);
    const float wlv[4] = {wl.x, wl.y, wl.z, wl.w}, whv[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      l[e] = (l[e] * sa) * wlv[e];
      h[e] = (h[e] * sa) * whv[e];
    }
  } else if (KIND == kKindNvfp4) {
    const float sa = pre.sa * p.w_tensor_scale;
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
    float4 a = pre.ra, b = pre.rb;
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

// Rotary epilogue (plain store) for rows n_lo..n_lo+3 of a q or k head
// (n_lo & 63 < 32) and their rotation partners n_lo+32..n_lo+35 of token m:
// bf16(qkv) rotated in fp32 without FMA contraction, as rope_qkv does
// (kernels.py:62-93), at the token's position m % rope_seq.
template <int KIND>
DEVI void epilogue_rope(const GemmParams& p, int m, int n_lo, float4 lo, float4 hi, const EpiPre& pre) {
  float l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
  const int n_hi = n_lo + 32;
  if (KIND == kKindFp8) {
    const float sa = pre.sa;
    const float4 wl = *reinterpret_cast<const float4*>(p.w_scale + n_lo);
    const float4 wh = *reinterpret_cast<const float4*>(p.w_scale + n_hi);
    const float wlv[4] = {wl.x, wl.y, wl.z, wl.w}, whv[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      l[e] = (l[e] * sa) * wlv[e];
      h[e] = (h[e] * sa) * whv[e];
    }
  } else if (KIND == kKindNvfp4) {
    const float sa = pre.sa * p.w_tensor_scale;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      l[e] *= sa;
      h[e] *= sa;
    }
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
  // cos / sin at d0 + 32 equal those at d0 (the rotary embedding's
  // cat(freqs, freqs), built so by rope_tables)
  const float4 c0 = pre.c0, s0 = pre.s0;
  const float cl[4] = {c0.x, c0.y, c0.z, c0.w}, sl[4] = {s0.x, s0.y, s0.z, s0.w};
  const float* ch = cl;
  const float* sh = sl;
  __nv_bfloat16 ol[4], oh[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = bf16_round(l[e]), b = bf16_round(h[e]);
    ol[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(a, cl[e]), __fmul_rn(-b, sl[e])));
    oh[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(b, ch[e]), __fmul_rn(a, sh[e])));
  }
  __nv_bfloat16* o = p.out + (size_t)m * p.ldo;
  *reinterpret_cast<uint2*>(o + n_lo) = *reinterpret_cast<uint2*>(ol);
  *reinterpret_cast<uint2*>(o + n_hi) = *reinterpret_cast<uint2*>(oh);
}

// TMEM accumulator -> partial (L2 scratch p.partials, or the shared scratch
// `part`) -> cluster reduction -> epilogue.  Called by all threads of the CTA
// after the MMA-done barrier completed: warps 0-3 read the TMEM lane quarters
// (in 256-thread CTAs warps 4-7 read the same quarters' upper token columns),
// and every thread takes part in the reduction.  `part` is at least BN*128
// floats of shared memory (the pipeline region, free once every MMA has
// completed).
// LNST: residual epilogue that also writes the LayerNorm statistics of the
// updated rows (p.ln_stats; bf16 projections without bias).
template <int BN, int KIND, bool LNST = false>
DEVI void tile_epilogue(const GemmParams& p, uint32_t tmem, float* part, int tile_n, int tile_m, int split,
                        int rank) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  // Split-K partials go to a global (L2) scratch when one is given: peers then
  // read them after the cluster barrier, and no closing barrier is needed to
  // keep a CTA's shared memory alive for its readers.
  const bool gpath = split > 1 && p.partials != nullptr;
  if (gpath) part = p.partials + ((size_t)(tile_m * gridDim.x + tile_n) * split + rank) * BN * 128;
  // CTA `rank` owns the tokens [t0, t1) of the tile in the reduction below.
  const int t0 = rank * BN / split, t1 = (rank + 1) * BN / split, nt = t1 - t0;
  if (BN >= 64 && blockDim.x >= 256) {
    // two warps per TMEM lane quarter (warp w reads lanes 32*(w%4)..), each
    // dumping half of the token columns
    if (warp < 8) {
      const int lq = warp & 3, c0 = (warp >> 2) * (BN / 2);
      const uint32_t qaddr = tmem + ((uint32_t)(lq * 32) << 16);
#pragma unroll 1
      for (int c = c0; c < c0 + BN / 2; c += 32) {
        uint32_t r[32];
        tmem_ld32(qaddr + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) part[(c + j) * 128 + lq * 32 + (tid & 31)] = __uint_as_float(r[j]);
      }
    }
  } else if (tid >= 128) {
    // only warps 0-3 own TMEM lanes
  } else if (BN >= 32) {
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

  // ---- reduction over the cluster and the epilogue: a thread (of all the
  // CTA's threads) takes 4 consecutive rows of one token and their partners
  // (+64: the GEGLU gate; +32 in the rotary tiles of q and k: the rotation
  // partner) and sums the S partials in rank order with 16-byte loads issued
  // back to back, together with the item's other global operands.
  const uint32_t part_addr = smem_u32(part);
  const bool rope = tile_n * 128 < p.rope_cols;
  const int pair = rope ? 32 : 64;
  const bool residual = LNST || p.epilogue == kEpiResidual;
  for (int item = tid; item < nt * 16; item += blockDim.x) {
    const int tl = t0 + (item >> 4);
    const int q4 = rope ? ((item >> 3) & 1) * 64 + (item & 7) * 4 : (item & 15) * 4;
    const int m = tile_m * BN + tl;
    if (m >= p.M) continue;
    const int off = tl * 128 + q4;
    const EpiPre pre = epi_prefetch<KIND>(p, m, tile_n * 128 + q4, residual, rope);
    float4 lo, hi;
    if (split == 1) {
      lo = *reinterpret_cast<const float4*>(part + off);
      hi = *reinterpret_cast<const float4*>(part + off + pair);
    } else {
      lo = make_float4(0.f, 0.f, 0.f, 0.f);
      hi = lo;
      // all remote loads of up to 8 peers are issued before any add
      for (int q0 = 0; q0 < split; q0 += 8) {
        float4 va[8], vb[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (q0 + u < split) {
            if (gpath) {  // L2 loads (the cluster barrier ordered the peers' stores)
              const float* src = p.partials + ((size_t)(tile_m * gridDim.x + tile_n) * split + q0 + u) * BN * 128 + off;
              va[u] = __ldcg(reinterpret_cast<const float4*>(src));
              vb[u] = __ldcg(reinterpret_cast<const float4*>(src + pair));
            } else {
              const uint32_t base = mapa_shared(part_addr, (uint32_t)(q0 + u));
              va[u] = ld_dsmem_f32x4(base + off * 4);
              vb[u] = ld_dsmem_f32x4(base + (off + pair) * 4);
            }
          }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (q0 + u < split) {
            lo.x += va[u].x; lo.y += va[u].y; lo.z += va[u].z; lo.w += va[u].w;
            hi.x += vb[u].x; hi.y += vb[u].y; hi.z += vb[u].z; hi.w += vb[u].w;
          }
      }
    }
    if (LNST) {
      // residual update, then the tile statistics of token m: its 16 items
      // are 16 consecutive threads (a 16-lane half warp)
      float4* rl = reinterpret_cast<float4*>(p.resid + (size_t)m * p.ldr + tile_n * 128 + q4);
      float4* rh = rl + 16;
      float4 a = pre.ra, b = pre.rb;
      a.x += bf16_round(lo.x); a.y += bf16_round(lo.y); a.z += bf16_round(lo.z); a.w += bf16_round(lo.w);
      b.x += bf16_round(hi.x); b.y += bf16_round(hi.y); b.z += bf16_round(hi.z); b.w += bf16_round(hi.w);
      *rl = a;
      *rh = b;
      const unsigned half = 0xFFFFu << (tid & 16);
      float sum = (a.x + a.y + a.z + a.w) + (b.x + b.y + b.z + b.w);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(half, sum, o);
      const float mean = sum * (1.0f / 128.0f);
      float m2 = 0.f;
      {
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) m2 += (v[e] - mean) * (v[e] - mean);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) m2 += __shfl_xor_sync(half, m2, o);
      if ((tid & 15) == 0) p.ln_stats[(size_t)m * gridDim.x + tile_n] = make_float2(mean, m2);
      continue;
    }
    if (rope)
      epilogue_rope<KIND>(p, m, tile_n * 128 + q4, lo, hi, pre);
    else
      epilogue_quad<KIND>(p, m, tile_n * 128 + q4, tile_n * 64 + q4, lo, hi, pre);
  }
  if (split > 1 && !gpath) cluster_sync_all();

}

// Epilogue of an unsplit tile with THREADS (256) threads.  The eight warps,
// two per TMEM lane quarter, dump the raw fp32 accumulator into shared memory
// as P[token][128 weight rows]; then every thread takes (token, 4 rows)
// items (rotary tiles: a token's rows r, r+32, r+64, r+96 that share one
// cos / sin pair), applies the precision's scales, bias and activation, and either
// writes the bf16 result into a shared [token][features] tile that one TMA
// store copies out (store / ReLU / GELU / GEGLU), or updates the fp32
// residual in global memory with 16-byte loads issued eight items at a time.
// Spreading the arithmetic (erf for GELU) over eight warps instead of the
// four TMEM warps keeps two warps per SM sub-partition busy.
template <int BN, int KIND, int THREADS>
DEVI void tile_epilogue_wide(const GemmParams& p, const CUtensorMap* omap, uint32_t tmem, uint8_t* smem, int tile_n,
                             int tile_m) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const int m_base = tile_m * BN;
  const int ep = p.epilogue;
  float* P = reinterpret_cast<float*>(smem);
  __nv_bfloat16* O = reinterpret_cast<__nv_bfloat16*>(smem + BN * 512);
  float* S = reinterpret_cast<float*>(smem + BN * 512 + BN * 256);
  static_assert(THREADS == 256 && BN >= 64, "wide epilogue: two warpgroups, 64+ token columns");
  {
    // two warps per TMEM lane quarter (warp w reads lanes 32*(w%4)..), each
    // dumping half of the token columns
    const int lq = warp & 3, c0 = (warp >> 2) * (BN / 2);
    const uint32_t lane_addr = tmem + ((uint32_t)(lq * 32) << 16);
#pragma unroll 1
    for (int c = c0; c < c0 + BN / 2; c += 32) {
      uint32_t v[32];
      tmem_ld32(lane_addr + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) P[(c + j) * 128 + lq * 32 + (tid & 31)] = __uint_as_float(v[j]);
    }
  }
  if (KIND != kKindBf16)
    for (int i = tid; i < BN; i += THREADS) S[i] = m_base + i < p.M ? p.a_scale[m_base + i] : 0.f;
  __syncthreads();
  const float tsc = KIND == kKindNvfp4 ? p.w_tensor_scale : 1.f;
  // item = (token, quad): rows 4q..4q+3 (GEGLU: act rows 4q..4q+3 of 64, gate rows +64)
  const int quads = ep == kEpiGeglu ? 16 : 32;
  const int items = BN * quads;
  if (ep == kEpiResidual) {
    constexpr int BATCH = 8;
    for (int i0 = tid; i0 < items; i0 += THREADS * BATCH) {
      float4 res[BATCH];
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        const int it = i0 + u * THREADS;
        const int tok = it >> 5, q = it & 31, m = m_base + tok;
        if (it < items && m < p.M)
          res[u] = *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.ldr + tile_n * 128 + 4 * q);
      }
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        const int it = i0 + u * THREADS;
        const int tok = it >> 5, q = it & 31, m = m_base + tok;
        if (it >= items || m >= p.M) continue;
        const int n = tile_n * 128 + 4 * q;
        float4 a = *reinterpret_cast<const float4*>(P + tok * 128 + 4 * q);
        float x[4] = {a.x, a.y, a.z, a.w};
        if (KIND == kKindFp8) {
          const float4 w = *reinterpret_cast<const float4*>(p.w_scale + n);
          const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] = (x[e] * S[tok]) * ww[e];
        } else if (KIND == kKindNvfp4) {
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] *= S[tok] * tsc;
        }
        if (p.bias) {
          const uint2 bu = *reinterpret_cast<const uint2*>(p.bias + n);
          const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&bu);
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] += __bfloat162float(bb[e]);
        }
        float4 r = res[u];
        r.x += bf16_round(x[0]);
        r.y += bf16_round(x[1]);
        r.z += bf16_round(x[2]);
        r.w += bf16_round(x[3]);
        *reinterpret_cast<float4*>(p.resid + (size_t)m * p.ldr + n) = r;
      }
    }
    __syncthreads();
    return;
  }
  if (tile_n * 128 + 128 <= p.rope_cols) {
    // rotary tile (two q or k heads): a thread takes rows r0..r0+3 (d0 < 32),
    // their partners r0+32.., and the same two row groups of the second head
    // (+64), for tokens tid/8, +32, ...: one cos / sin quad serves all four,
    // since the tables repeat their first 32 columns (the rotary embedding's
    // cat(freqs, freqs), built so by rope_tables), and a thread's four tokens
    // are loaded in one batch.
    const int r0 = 4 * (tid & 7);
    float ws[4][4];
#pragma unroll
    for (int gq = 0; gq < 4; ++gq) {
      ws[gq][0] = ws[gq][1] = ws[gq][2] = ws[gq][3] = 1.f;
      if (KIND == kKindFp8) {
        const float4 a = *reinterpret_cast<const float4*>(p.w_scale + tile_n * 128 + r0 + 32 * gq);
        ws[gq][0] = a.x; ws[gq][1] = a.y; ws[gq][2] = a.z; ws[gq][3] = a.w;
      }
    }
    constexpr int RT = BN / (THREADS / 8);  // tokens per thread
    float4 c0[RT], s0[RT];
#pragma unroll
    for (int u = 0; u < RT; ++u) {
      const int pos = (m_base + (tid >> 3) + u * (THREADS / 8)) % p.rope_seq;
      c0[u] = *reinterpret_cast<const float4*>(p.rope_cos + (size_t)pos * 64 + r0);
      s0[u] = *reinterpret_cast<const float4*>(p.rope_sin + (size_t)pos * 64 + r0);
    }
#pragma unroll
    for (int u = 0; u < RT; ++u) {
      const int tok = (tid >> 3) + u * (THREADS / 8);
      const float cl[4] = {c0[u].x, c0[u].y, c0[u].z, c0[u].w};
      const float sl[4] = {s0[u].x, s0[u].y, s0[u].z, s0[u].w};
      const float* ch = cl;
      const float* sh = sl;
      const float sc = KIND == kKindNvfp4 ? S[tok] * tsc : KIND == kKindFp8 ? S[tok] : 1.f;
#pragma unroll
      for (int hd = 0; hd < 2; ++hd) {
        const float4 la = *reinterpret_cast<const float4*>(P + tok * 128 + 64 * hd + r0);
        const float4 ha = *reinterpret_cast<const float4*>(P + tok * 128 + 64 * hd + r0 + 32);
        float l[4] = {la.x, la.y, la.z, la.w}, h[4] = {ha.x, ha.y, ha.z, ha.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (KIND == kKindFp8) {
            l[e] = (l[e] * sc) * ws[2 * hd][e];
            h[e] = (h[e] * sc) * ws[2 * hd + 1][e];
          } else if (KIND == kKindNvfp4) {
            l[e] *= sc;
            h[e] *= sc;
          }
        }
        // bf16(qkv) rotated in fp32 without FMA, as rope_qkv does (kernels.py:62-93)
        __nv_bfloat16 ol[4], oh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16_round(l[e]), b = bf16_round(h[e]);
          ol[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(a, cl[e]), __fmul_rn(-b, sl[e])));
          oh[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(b, ch[e]), __fmul_rn(a, sh[e])));
        }
        *reinterpret_cast<uint2*>(O + tok * 128 + 64 * hd + r0) = *reinterpret_cast<uint2*>(ol);
        *reinterpret_cast<uint2*>(O + tok * 128 + 64 * hd + r0 + 32) = *reinterpret_cast<uint2*>(oh);
      }
    }
  } else {
  // THREADS is a multiple of `quads`, so every item of a thread covers the
  // same 4 rows: the per-row constants (weight scales, bias, the rotation
  // partner) are loaded once, and the rotary tables of a thread's tokens are
  // loaded KB tokens at a time ahead of the arithmetic (a load per item
  // left the loop latency-bound).
  static_assert(THREADS % 32 == 0, "wide epilogue: whole warps");
  const int q = tid % quads, r0 = 4 * q, n = tile_n * 128 + r0;
  const int tok_step = THREADS / quads;
  const bool rot = n < p.rope_cols;
  const int d0 = r0 & 63, pr = d0 < 32 ? r0 + 32 : r0 - 32;
  float wx[4] = {1.f, 1.f, 1.f, 1.f}, wg[4] = {1.f, 1.f, 1.f, 1.f}, wy[4] = {1.f, 1.f, 1.f, 1.f};
  if (KIND == kKindFp8) {
    const float4 a = *reinterpret_cast<const float4*>(p.w_scale + n);
    wx[0] = a.x; wx[1] = a.y; wx[2] = a.z; wx[3] = a.w;
    if (ep == kEpiGeglu) {
      const float4 b = *reinterpret_cast<const float4*>(p.w_scale + n + 64);
      wg[0] = b.x; wg[1] = b.y; wg[2] = b.z; wg[3] = b.w;
    }
    if (rot) {
      const float4 c = *reinterpret_cast<const float4*>(p.w_scale + tile_n * 128 + pr);
      wy[0] = c.x; wy[1] = c.y; wy[2] = c.z; wy[3] = c.w;
    }
  }
  float bx[4] = {0.f, 0.f, 0.f, 0.f};
  const bool has_bias = p.bias != nullptr && !rot && ep != kEpiGeglu;
  if (has_bias) {
    const uint2 bu = *reinterpret_cast<const uint2*>(p.bias + n);
    const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&bu);
#pragma unroll
    for (int e = 0; e < 4; ++e) bx[e] = __bfloat162float(bb[e]);
  }
  constexpr int KB = 4;  // 8 measured no faster (and spills with fp8's weight scales)
  for (int tb = tid / quads; tb < BN; tb += KB * tok_step) {
    float4 cv[KB], sv[KB];
    if (rot) {
#pragma unroll
      for (int u = 0; u < KB; ++u) {
        const int tok = tb + u * tok_step;
        const int pos = (m_base + (tok < BN ? tok : 0)) % p.rope_seq;
        cv[u] = *reinterpret_cast<const float4*>(p.rope_cos + (size_t)pos * 64 + d0);
        sv[u] = *reinterpret_cast<const float4*>(p.rope_sin + (size_t)pos * 64 + d0);
      }
    }
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const int tok = tb + u * tok_step;
      if (tok >= BN) break;
      float x[4], g[4];
      {
        const float4 a = *reinterpret_cast<const float4*>(P + tok * 128 + r0);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        g[0] = g[1] = g[2] = g[3] = 0.f;
        if (ep == kEpiGeglu) {
          const float4 b = *reinterpret_cast<const float4*>(P + tok * 128 + 64 + r0);
          g[0] = b.x; g[1] = b.y; g[2] = b.z; g[3] = b.w;
        }
      }
      if (KIND == kKindFp8) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x[e] = (x[e] * S[tok]) * wx[e];
          g[e] = (g[e] * S[tok]) * wg[e];
        }
      } else if (KIND == kKindNvfp4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x[e] *= S[tok] * tsc;
          g[e] *= S[tok] * tsc;
        }
      }
      __nv_bfloat16 o[4];
      if (rot) {
        // bf16(qkv) rotated in fp32 without FMA, as rope_qkv does (kernels.py:62-93)
        const float4 pb = *reinterpret_cast<const float4*>(P + tok * 128 + pr);
        float y[4] = {pb.x, pb.y, pb.z, pb.w};
        if (KIND == kKindFp8) {
#pragma unroll
          for (int e = 0; e < 4; ++e) y[e] = (y[e] * S[tok]) * wy[e];
        } else if (KIND == kKindNvfp4) {
#pragma unroll
          for (int e = 0; e < 4; ++e) y[e] *= S[tok] * tsc;
        }
        const float cs[4] = {cv[u].x, cv[u].y, cv[u].z, cv[u].w};
        const float sn[4] = {sv[u].x, sv[u].y, sv[u].z, sv[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16_round(x[e]), b = bf16_round(y[e]);
          const float rotp = __fmul_rn(d0 < 32 ? -b : b, sn[e]);
          o[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(a, cs[e]), rotp));
        }
        *reinterpret_cast<uint2*>(O + tok * 128 + r0) = *reinterpret_cast<uint2*>(o);
      } else if (ep == kEpiGeglu) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          o[e] = __float2bfloat16_rn(bf16_round(gelu_erf(bf16_round(x[e]))) * bf16_round(g[e]));
        *reinterpret_cast<uint2*>(O + tok * 64 + r0) = *reinterpret_cast<uint2*>(o);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float y = has_bias ? x[e] + bx[e] : x[e];
          if (ep == kEpiRelu) y = fmaxf(y, 0.f);
          else if (ep == kEpiGelu) y = gelu_erf(bf16_round(y));
          o[e] = __float2bfloat16_rn(y);
        }
        *reinterpret_cast<uint2*>(O + tok * 128 + r0) = *reinterpret_cast<uint2*>(o);
      }
    }
  }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    tma_store_2d(omap, O, ep == kEpiGeglu ? tile_n * 64 : tile_n * 128, m_base);
    bulk_commit();
    bulk_wait_read0();
  }
  __syncthreads();
}


// Residual epilogue of an unsplit 64-token tile (128 threads): the fp32
// residual tile [64 tokens][128 columns] comes in with one TMA load, issued
// while the warps move the accumulator out of TMEM, is updated in shared
// memory (r += bf16(scaled accumulator + bias), the same arithmetic as
// epilogue_quad) and goes back with one TMA store; rows past p.M are clipped
// by the tensor map.  A thread keeps one column quad (its weight scales and
// bias) for all its tokens.  Returns false when the residual tile did not
// arrive within `limit` (nothing is stored then; thread 0 waits once more,
// bounded, so that a late copy does not land after the CTA has exited).
template <int BN, int KIND>
DEVI bool tile_epilogue_resid_tma(const GemmParams& p, const CUtensorMap* rmap, uint32_t tmem, uint8_t* smem,
                                  uint64_t* rbar, int tile_n, int tile_m, uint64_t limit) {
  static_assert(BN == 64, "TMA residual epilogue: 64-token tiles");
  const int tid = threadIdx.x, warp = tid >> 5;
  const int m_base = tile_m * BN;
  float* P = reinterpret_cast<float*>(smem);                // [BN][128] accumulator
  float* R = reinterpret_cast<float*>(smem + BN * 512);     // [BN][128] residual rows
  float* S = reinterpret_cast<float*>(smem + BN * 1024);    // [BN] activation row scales
  if (tid == 0) {
    mbar_expect_tx(rbar, BN * 512);
    tma_load_2d(R, rmap, rbar, tile_n * 128, m_base, policy_evict_last());
  }
  if (warp < 4) {
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t v[32];
      tmem_ld32(lane_addr + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) P[(c + j) * 128 + warp * 32 + (tid & 31)] = __uint_as_float(v[j]);
    }
  }
  if (KIND != kKindBf16)
    for (int i = tid; i < BN; i += blockDim.x) S[i] = m_base + i < p.M ? p.a_scale[m_base + i] : 0.f;
  const int q = tid & 31, n = tile_n * 128 + 4 * q;
  float ws[4] = {1.f, 1.f, 1.f, 1.f}, bx[4] = {0.f, 0.f, 0.f, 0.f};
  if (KIND == kKindFp8) {
    const float4 a = *reinterpret_cast<const float4*>(p.w_scale + n);
    ws[0] = a.x; ws[1] = a.y; ws[2] = a.z; ws[3] = a.w;
  }
  if (p.bias) {
    const uint2 bu = *reinterpret_cast<const uint2*>(p.bias + n);
    const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&bu);
#pragma unroll
    for (int e = 0; e < 4; ++e) bx[e] = __bfloat162float(bb[e]);
  }
  const float tsc = KIND == kKindNvfp4 ? p.w_tensor_scale : 1.f;
  // one CTA-wide verdict on the residual tile (the barrier also publishes P
  // and S), so that every thread takes the same path
  const bool ok = __syncthreads_and(mbar_wait(rbar, 0, limit)) != 0;
  if (ok) {
    for (int tok = tid >> 5; tok < BN; tok += blockDim.x >> 5) {
      const float4 a = *reinterpret_cast<const float4*>(P + tok * 128 + 4 * q);
      float x[4] = {a.x, a.y, a.z, a.w};
      if (KIND == kKindFp8) {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = (x[e] * S[tok]) * ws[e];
      } else if (KIND == kKindNvfp4) {
        const float sc = S[tok] * tsc;
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] *= sc;
      }
      if (p.bias) {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] += bx[e];
      }
      float4* rp = reinterpret_cast<float4*>(R + tok * 128 + 4 * q);
      float4 r = *rp;
      r.x += bf16_round(x[0]);
      r.y += bf16_round(x[1]);
      r.z += bf16_round(x[2]);
      r.w += bf16_round(x[3]);
      *rp = r;
    }
    fence_proxy_async_smem();
  }
  __syncthreads();
  if (ok && tid == 0) {
    tma_store_2d(rmap, R, tile_n * 128, m_base);
    bulk_commit();
    bulk_wait_read0();
  }
  if (!ok && tid == 0) mbar_wait(rbar, 0, limit);  // a late tile still lands before the CTA exits
  __syncthreads();
  return ok;
}

}  // namespace laya
