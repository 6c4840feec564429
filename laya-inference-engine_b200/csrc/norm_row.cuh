// One LayerNorm row of the Laya forward (one warp, d = 128*NV fp32 values in
// registers): the embedding gather, add_norm, the type-embedding add and an
// optional second LayerNorm, with fp32 / bf16 / e4m3 / NVFP4 outputs.
//
// Reference: add_norm and the embedding LN (src/laya_blackwell/model.py:15-19,
// 84,90,97,102-104,59,68), _quantize_rows (quantization.py:20-29).  LayerNorm
// uses the two-pass mean / centred variance in fp32.
#pragma once
#include "common.cuh"
#include "params.h"

namespace laya {

template <int NV>
DEVI void row_layernorm(float4 (&x)[NV], int d, float eps, const float* w, const float* b, int lane) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (x[i].x + x[i].y) + (x[i].z + x[i].w);
  const float mean = warp_sum(s) / (float)d;
  float v = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = x[i].x - mean, bb = x[i].y - mean, c = x[i].z - mean, e = x[i].w - mean;
    v += (a * a + bb * bb) + (c * c + e * e);
  }
  const float var = warp_sum(v) / (float)d;
  const float rstd = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = (lane + 32 * i) * 4;
    const float4 ww = *reinterpret_cast<const float4*>(w + col);
    float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
    if (b) bb = *reinterpret_cast<const float4*>(b + col);
    x[i].x = (x[i].x - mean) * rstd * ww.x + bb.x;
    x[i].y = (x[i].y - mean) * rstd * ww.y + bb.y;
    x[i].z = (x[i].z - mean) * rstd * ww.z + bb.z;
    x[i].w = (x[i].w - mean) * rstd * ww.w + bb.w;
  }
}

// Normalise output row `row` (a warp, lane = lane index).
template <int NV>
DEVI void norm_row(const NormParams& p, int row, int lane) {
  const float* src;
  if (p.tok_ids)
    src = p.src + (size_t)p.tok_ids[row] * p.ld_src;
  else
    src = p.src + (size_t)(p.row_map ? p.row_map[row] : row) * p.ld_src;
  float4 x[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) x[i] = reinterpret_cast<const float4*>(src)[lane + 32 * i];
  row_layernorm<NV>(x, p.d, p.eps, p.w, p.b, lane);
  if (p.add_table) {
    const float* a = p.add_table + (size_t)p.add_idx[row / p.add_div] * p.d;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float4 t = reinterpret_cast<const float4*>(a)[lane + 32 * i];
      x[i].x += t.x;
      x[i].y += t.y;
      x[i].z += t.z;
      x[i].w += t.w;
    }
  }
  if (p.out_f32) {
    float4* dst = reinterpret_cast<float4*>(p.out_f32 + (size_t)row * p.ld_out_f32);
#pragma unroll
    for (int i = 0; i < NV; ++i) dst[lane + 32 * i] = x[i];
  }
  if (p.second_w) row_layernorm<NV>(x, p.d, p.eps, p.second_w, p.second_b, lane);
  if (!p.out_bf16 && !p.out_fp8 && !p.out_x4) return;
  // bf16 of the row (also the FP8 quantiser's input, as in the reference where
  // _quantize_rows reads the bf16 normed activations).
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    x[i].x = bf16_round(x[i].x);
    x[i].y = bf16_round(x[i].y);
    x[i].z = bf16_round(x[i].z);
    x[i].w = bf16_round(x[i].w);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w))));
  }
  if (p.out_bf16) {
    __nv_bfloat16* dst = p.out_bf16 + (size_t)row * p.d;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      __nv_bfloat162 a = __floats2bfloat162_rn(x[i].x, x[i].y);
      __nv_bfloat162 c = __floats2bfloat162_rn(x[i].z, x[i].w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&a);
      u.y = *reinterpret_cast<uint32_t*>(&c);
      *reinterpret_cast<uint2*>(dst + (lane + 32 * i) * 4) = u;
    }
  }
  if (p.out_fp8) {
    amax = warp_max(amax);
    const float scale = fmaxf(amax * kInvE4m3Max, 1e-12f), inv = 1.0f / scale;
    uint8_t* dst = p.out_fp8 + (size_t)row * p.d;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float a = fminf(fmaxf(div_rn_by(x[i].x, scale, inv), -448.f), 448.f);
      const float bq = fminf(fmaxf(div_rn_by(x[i].y, scale, inv), -448.f), 448.f);
      const float c = fminf(fmaxf(div_rn_by(x[i].z, scale, inv), -448.f), 448.f);
      const float e = fminf(fmaxf(div_rn_by(x[i].w, scale, inv), -448.f), 448.f);
      const uint32_t lo = f32x2_to_e4m3x2(a, bq), hi = f32x2_to_e4m3x2(c, e);
      *reinterpret_cast<uint32_t*>(dst + (lane + 32 * i) * 4) = lo | (hi << 16);
    }
    if (lane == 0) p.out_fp8_scale[row] = scale;
  }
  if (p.out_x4) {
    // NVFP4 (the activation quantiser's values): outer = max(amax/(6*448),
    // 1e-20) per row; a 16-element block is 4 lanes' chunks, its e4m3 scale
    // max(bmax/(6*outer), 2^-9), values e2m1(x / (scale*outer)).
    amax = warp_max(amax);
    const float outer = fmaxf(amax / (6.0f * 448.0f), 1e-20f);
    if (lane == 0) p.out_x4_outer[row] = outer;
    const float o6 = 6.0f * outer, inv_o6 = 1.0f / o6;
    uint8_t* q = p.out_x4 + (size_t)row * (p.d / 2);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float bmax = fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w)));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
      const float sc = fmaxf(div_rn_by(bmax, o6, inv_o6), 0.001953125f);  // 2^-9 floor
      const uint8_t sc8 = (uint8_t)(f32x2_to_e4m3x2(sc, 0.f) & 0xFF);
      const float scale = e4m3_value(sc8);
      const float denom = scale * outer, inv_d = 1.0f / denom;
      const int col = (lane + 32 * i) * 4;
      const uint32_t lo = f32x2_to_e2m1x2(div_rn_by(x[i].x, denom, inv_d), div_rn_by(x[i].y, denom, inv_d));
      const uint32_t hi = f32x2_to_e2m1x2(div_rn_by(x[i].z, denom, inv_d), div_rn_by(x[i].w, denom, inv_d));
      *reinterpret_cast<uint16_t*>(q + col / 2) = (uint16_t)(lo | (hi << 8));
      if ((lane & 3) == 0) p.out_x4_sf[sf_offset(row, col / 16, p.x4_rows_per_block, p.x4_col_blocks)] = sc8;
    }
  }
}

// ---- one CTA per row: d/8 threads, thread t holds columns [8t, 8t+8)
// (d a multiple of 256).  The same arithmetic as norm_row with the
// reductions done across the CTA; used where a warp per row leaves a short
// batch's rows as long serial chains (the quantised outputs).

// Sum of v over the CTA (nw warps); `red` is nw floats of shared memory.
DEVI float cta_sum(float v, float* red, int nw) {
  v = warp_sum(v);
  __syncthreads();  // red is free (previous use finished)
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

DEVI float cta_max(float v, float* red, int nw) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = 0.f;
  for (int i = 0; i < nw; ++i) m = fmaxf(m, red[i]);
  return m;
}

DEVI void cta_layernorm(float (&x)[8], int d, float eps, const float* w, const float* b, int col, float* red,
                        int nw) {
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 8; e += 4) s += (x[e] + x[e + 1]) + (x[e + 2] + x[e + 3]);
  const float mean = cta_sum(s, red, nw) / (float)d;
  float v = 0.f;
#pragma unroll
  for (int e = 0; e < 8; e += 4) {
    const float a0 = x[e] - mean, a1 = x[e + 1] - mean, a2 = x[e + 2] - mean, a3 = x[e + 3] - mean;
    v += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
  }
  const float var = cta_sum(v, red, nw) / (float)d;
  const float rstd = rsqrtf(var + eps);
  const float4 w0 = *reinterpret_cast<const float4*>(w + col), w1 = *reinterpret_cast<const float4*>(w + col + 4);
  float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
  if (b) {
    b0 = *reinterpret_cast<const float4*>(b + col);
    b1 = *reinterpret_cast<const float4*>(b + col + 4);
  }
  const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = (x[e] - mean) * rstd * ww[e] + bb[e];
}

// Normalise row `row` with the CTA (blockDim.x == p.d / 8); `red` holds
// blockDim.x / 32 floats.
DEVI void norm_row_cta(const NormParams& p, int row, float* red) {
  const int t = threadIdx.x, nw = blockDim.x >> 5, col = t * 8;
  const float* src;
  if (p.tok_ids)
    src = p.src + (size_t)p.tok_ids[row] * p.ld_src;
  else
    src = p.src + (size_t)(p.row_map ? p.row_map[row] : row) * p.ld_src;
  float x[8];
  {
    const float4 a = *reinterpret_cast<const float4*>(src + col), b = *reinterpret_cast<const float4*>(src + col + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
  cta_layernorm(x, p.d, p.eps, p.w, p.b, col, red, nw);
  if (p.add_table) {
    const float* a = p.add_table + (size_t)p.add_idx[row / p.add_div] * p.d + col;
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] += a[e];
  }
  if (p.out_f32) {
    float* dst = p.out_f32 + (size_t)row * p.ld_out_f32 + col;
    *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
  }
  if (p.second_w) cta_layernorm(x, p.d, p.eps, p.second_w, p.second_b, col, red, nw);
  if (!p.out_bf16 && !p.out_fp8 && !p.out_x4) return;
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    x[e] = bf16_round(x[e]);
    amax = fmaxf(amax, fabsf(x[e]));
  }
  if (p.out_bf16) {
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 v = __floats2bfloat162_rn(x[2 * e], x[2 * e + 1]);
      o[e] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(p.out_bf16 + (size_t)row * p.d + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (!p.out_fp8 && !p.out_x4) return;
  amax = cta_max(amax, red, nw);
  if (p.out_fp8) {
    const float scale = fmaxf(amax * kInvE4m3Max, 1e-12f), inv = 1.0f / scale;
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = fminf(fmaxf(div_rn_by(x[4 * j + e], scale, inv), -448.f), 448.f);
      w[j] = (uint32_t)f32x2_to_e4m3x2(v[0], v[1]) | ((uint32_t)f32x2_to_e4m3x2(v[2], v[3]) << 16);
    }
    *reinterpret_cast<uint2*>(p.out_fp8 + (size_t)row * p.d + col) = make_uint2(w[0], w[1]);
    if (t == 0) p.out_fp8_scale[row] = scale;
  }
  if (p.out_x4) {
    // NVFP4 as the activation quantiser: a 16-element block is a thread pair
    const float outer = fmaxf(amax / (6.0f * 448.0f), 1e-20f);
    if (t == 0) p.out_x4_outer[row] = outer;
    const float o6 = 6.0f * outer, inv_o6 = 1.0f / o6;
    float bmax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) bmax = fmaxf(bmax, fabsf(x[e]));
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
    const float sc = fmaxf(div_rn_by(bmax, o6, inv_o6), 0.001953125f);  // 2^-9 floor
    const uint8_t sc8 = (uint8_t)(f32x2_to_e4m3x2(sc, 0.f) & 0xFF);
    const float denom = e4m3_value(sc8) * outer, inv_d = 1.0f / denom;
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 8; e += 2)
      w |= (uint32_t)f32x2_to_e2m1x2(div_rn_by(x[e], denom, inv_d), div_rn_by(x[e + 1], denom, inv_d)) << (4 * e);
    *reinterpret_cast<uint32_t*>(p.out_x4 + (size_t)row * (p.d / 2) + col / 2) = w;
    if ((t & 1) == 0) p.out_x4_sf[sf_offset(row, col / 16, p.x4_rows_per_block, p.x4_col_blocks)] = sc8;
  }
}

}  // namespace laya
