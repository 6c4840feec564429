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
    const float scale = fmaxf(amax / 448.0f, 1e-12f), inv = 1.0f / scale;
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

}  // namespace laya
