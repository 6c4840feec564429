// Row-wise kernels of the Laya forward: LayerNorm (with the embedding
// gather, the type-embedding add and an optional second LayerNorm fused on the
// same row), per-row FP8 activation quantisation, the head's row gather and
// the decision tail (scorer logits, masked softmax, entropy, top-2, act_head).
//
// Reference: add_norm and the embedding LN (src/laya_blackwell/model.py:15-19,84,
// 90,97,102-104,59,68), _quantize_rows (quantization.py:20-29), the select
// gather (model.py:64-66,106) and the tail (model.py:113-123).
//
// One warp owns one row (the LayerNorm row code is in norm_row.cuh);
// reductions are warp shuffles.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "norm_row.cuh"

namespace laya {

template <int NV>
__global__ void __launch_bounds__(256) norm_kernel(const NormParams p) {
  griddep_launch_dependents();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  norm_row<NV>(p, row, lane);
}

// One CTA of d/8 threads per row (d a multiple of 256): see norm_row_cta.
__global__ void __launch_bounds__(128) norm_cta_kernel(const NormParams p) {
  __shared__ float red[4];
  griddep_launch_dependents();
  griddep_wait();
  if ((int)blockIdx.x >= p.rows) return;
  norm_row_cta(p, blockIdx.x, red);
}

// Per-row e4m3 quantisation of a bf16 matrix (quantization.py:20-29).  One
// CTA of 128 threads per row (k <= 1024*MAXC): each thread holds its chunks of
// 8 in registers with every load in flight at once, the row maximum is a warp
// then CTA reduction, and quotients use the FMA-corrected division.  Four
// warps per row keep a short batch's rows from being one long serial chain.
template <int MAXC>
__global__ void __launch_bounds__(128) quant_fp8_kernel(const QuantParams p) {
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
  const float scale = fmaxf(amax * kInvE4m3Max, 1e-12f), inv = 1.0f / scale;
  uint8_t* dst = p.q + (size_t)row * p.k;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid * 8 + 1024 * i;
    if (c >= p.k) continue;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        v[t] = fminf(fmaxf(div_rn_by(__bfloat162float(e[4 * j + t]), scale, inv), -448.f), 448.f);
      w[j] = (uint32_t)f32x2_to_e4m3x2(v[0], v[1]) | ((uint32_t)f32x2_to_e4m3x2(v[2], v[3]) << 16);
    }
    *reinterpret_cast<uint2*>(dst + c) = make_uint2(w[0], w[1]);
  }
  if (tid == 0) p.scale[row] = scale;
}

// The same quantisation with one warp per row, for large row counts (from
// 2,048 rows, where one CTA per row runs in several waves): chunk
// c = lane + 32 i of 8 elements, every load in flight at once, the row
// maximum a warp reduction.  Arithmetic identical to quant_fp8_kernel.
template <int CPL>
__global__ void __launch_bounds__(256) quant_fp8_warp_kernel(const QuantParams p) {
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
  const float scale = fmaxf(amax * kInvE4m3Max, 1e-12f), inv = 1.0f / scale;
  uint8_t* dst = p.q + (size_t)row * p.k;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c >= chunks) continue;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        v[t] = fminf(fmaxf(div_rn_by(__bfloat162float(e[4 * j + t]), scale, inv), -448.f), 448.f);
      w[j] = (uint32_t)f32x2_to_e4m3x2(v[0], v[1]) | ((uint32_t)f32x2_to_e4m3x2(v[2], v[3]) << 16);
    }
    reinterpret_cast<uint2*>(dst)[c] = make_uint2(w[0], w[1]);
  }
  if (lane == 0) p.scale[row] = scale;
}

// dst[r] = src[map[r]] for fp32 rows of width d (multiple of 4).
__global__ void __launch_bounds__(256) gather_rows_kernel(float* dst, const float* src, const int* map, int rows,
                                                           int d) {
  griddep_launch_dependents();
  griddep_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* s = reinterpret_cast<const float4*>(src + (size_t)map[row] * d);
  float4* o = reinterpret_cast<float4*>(dst + (size_t)row * d);
  for (int c = lane; c < d / 4; c += 32) o[c] = s[c];
}

// Decision tail (model.py:113-122).  Grid (questions, kTailCtas): every CTA
// recomputes the question's logits and softmax features (cheap) and a slice
// of act_head's first layer; the last CTA of a question to finish (atomic
// arrival count, no spinning) applies the second layer and resets the count.
constexpr int kTailCtas = 16;

__global__ void __launch_bounds__(256) tail_kernel(const TailParams p) {
  extern __shared__ float tsm[];
  float* s_logit = tsm;                       // [k]
  float* s_x = tsm + 256;                     // [d + 4] (bf16-rounded act_head input)
  __shared__ unsigned int s_last;
  griddep_launch_dependents();
  griddep_wait();
  const int q = blockIdx.x, part = blockIdx.y, nparts = gridDim.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  // scorer[3]: logit_j = bf16(z_j . w + b), masked to -1e4
  for (int j = warp; j < p.k; j += nw) {
    const __nv_bfloat16* z = p.z + ((size_t)q * p.k + j) * p.d;
    float acc = 0.f;
    for (int c = lane * 8; c < p.d; c += 256) {
      const uint4 zu = *reinterpret_cast<const uint4*>(z + c);
      const uint4 wu = *reinterpret_cast<const uint4*>(p.fc2_w + c);
      const __nv_bfloat16* za = reinterpret_cast<const __nv_bfloat16*>(&zu);
      const __nv_bfloat16* wa = reinterpret_cast<const __nv_bfloat16*>(&wu);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += __bfloat162float(za[e]) * __bfloat162float(wa[e]);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const float l = bf16_round(acc + __bfloat162float(p.fc2_b[0]));
      s_logit[j] = p.marker_mask[q * p.k + j] ? l : -1e4f;
    }
  }
  const float* cls = p.h_sel + (size_t)q * (1 + p.k) * p.d;
  for (int c = tid; c < p.d; c += blockDim.x) s_x[c] = bf16_round(cls[c]);
  __syncthreads();
  if (tid == 0) {
    float mx = -INFINITY;
    int count = 0;
    for (int j = 0; j < p.k; ++j) {
      mx = fmaxf(mx, s_logit[j]);
      count += p.marker_mask[q * p.k + j] != 0;
    }
    float sum = 0.f;
    for (int j = 0; j < p.k; ++j) sum += expf(s_logit[j] - mx);
    float ent = 0.f, t1 = -1.f, t2 = -1.f;
    for (int j = 0; j < p.k; ++j) {
      const float pj = expf(s_logit[j] - mx) / sum;
      ent += pj * logf(fmaxf(pj, 1e-9f));
      if (pj > t1) {
        t2 = t1;
        t1 = pj;
      } else if (pj > t2) {
        t2 = pj;
      }
      if (part == 0) p.logits[q * p.k + j] = s_logit[j];
    }
    const float cnt = (float)(count < 2 ? 2 : count);
    ent = -ent / logf(cnt);
    s_x[p.d + 0] = bf16_round(t1);
    s_x[p.d + 1] = bf16_round(t1 - t2);
    s_x[p.d + 2] = bf16_round(ent);
    s_x[p.d + 3] = bf16_round(cnt / 255.0f);
  }
  __syncthreads();
  // act_head[0..1] for this CTA's slice: a1 = bf16(gelu(bf16(W1 x + b1)))
  const int din = p.d + 4;
  const int per = (p.act_hidden + nparts - 1) / nparts;
  const int u0 = part * per, u1 = min(p.act_hidden, u0 + per);
  for (int u = u0 + warp; u < u1; u += nw) {
    const __nv_bfloat16* wr = p.a1_w + (size_t)u * din;
    float acc = 0.f;
    for (int c = lane; c < din; c += 32) acc += __bfloat162float(wr[c]) * s_x[c];
    acc = warp_sum(acc);
    if (lane == 0) p.a1[(size_t)q * p.act_hidden + u] = bf16_round(gelu_erf(bf16_round(acc + __bfloat162float(p.a1_b[u]))));
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&p.arrivals[q], 1u) == (unsigned)(nparts - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // act_head[2]: act = bf16(W2 a1 + b2)
  if (warp < 2) {
    const __nv_bfloat16* wr = p.a2_w + (size_t)warp * p.act_hidden;
    const float* a1 = p.a1 + (size_t)q * p.act_hidden;
    float acc = 0.f;
    for (int c = lane; c < p.act_hidden; c += 32) acc += __bfloat162float(wr[c]) * __ldcg(a1 + c);
    acc = warp_sum(acc);
    if (lane == 0) p.act[q * 2 + warp] = bf16_round(acc + __bfloat162float(p.a2_b[warp]));
  }
  if (tid == 0) p.arrivals[q] = 0;
}

// Per-output-row e4m3 weight quantisation (quantization.py:62-73), bf16 in.
__global__ void __launch_bounds__(256) pack_fp8_rows_kernel(const __nv_bfloat16* w, uint8_t* q, float* scale, int rows,
                                                            int k) {
  QuantParams p;
  p.rows = rows;
  p.k = k;
  p.src = w;
  p.q = q;
  p.scale = scale;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __nv_bfloat16* src = p.src + (size_t)row * k;
  float amax = 0.f;
  for (int c = lane; c < k; c += 32) amax = fmaxf(amax, fabsf(__bfloat162float(src[c])));
  amax = warp_max(amax);
  const float s = fmaxf(amax * kInvE4m3Max, 1e-12f);
  for (int c = lane * 2; c < k; c += 64) {
    const float a = fminf(fmaxf(__bfloat162float(src[c]) / s, -448.f), 448.f);
    const float b = fminf(fmaxf(__bfloat162float(src[c + 1]) / s, -448.f), 448.f);
    *reinterpret_cast<uint16_t*>(q + (size_t)row * k + c) = f32x2_to_e4m3x2(a, b);
  }
  if (lane == 0) scale[row] = s;
}

// ------------------------------------------------------------------ launchers
namespace {
// One warp per row, `rows_per_block` rows (warps) per CTA.
// Row count from which the row kernels with quantised outputs use a warp
// per row instead of a CTA per row.
constexpr int kWarpRowsFrom = 2048;

cudaError_t launch_rows(const void* kern, void** args, int rows, size_t smem, cudaStream_t stream, bool pdl,
                        int rows_per_block = 8) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((rows + rows_per_block - 1) / rows_per_block, 1, 1);
  cfg.blockDim = dim3(32 * rows_per_block, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, kern, args);
}
}  // namespace

cudaError_t launch_norm(const NormParams& p, cudaStream_t stream, bool pdl) {
  if (p.d % 128 || p.d > 1024 || p.d < 128) return cudaErrorInvalidValue;
  NormParams q = p;
  void* args[] = {&q};
  const void* kern = nullptr;
  switch (p.d / 128) {
    case 1: kern = (const void*)norm_kernel<1>; break;
    case 2: kern = (const void*)norm_kernel<2>; break;
    case 3: kern = (const void*)norm_kernel<3>; break;
    case 4: kern = (const void*)norm_kernel<4>; break;
    case 5: kern = (const void*)norm_kernel<5>; break;
    case 6: kern = (const void*)norm_kernel<6>; break;
    case 7: kern = (const void*)norm_kernel<7>; break;
    case 8: kern = (const void*)norm_kernel<8>; break;
  }
  if ((p.out_fp8 || p.out_x4) && p.d % 256 == 0 && p.rows < kWarpRowsFrom) {
    // quantised outputs carry much more per-row work: one CTA per row while
    // that fits in about one wave; from 2,048 rows a warp per row
    // (8,192-token FP8 forward: 9.03 -> 8.83 ms)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.rows, 1, 1);
    cfg.blockDim = dim3(p.d / 8, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, (const void*)norm_cta_kernel, args);
  }
  return launch_rows(kern, args, p.rows, 0, stream, pdl, p.out_x4 ? 4 : 8);
}

cudaError_t launch_quant_fp8(const QuantParams& p, cudaStream_t stream, bool pdl) {
  if (p.k % 8 || p.k > 4096) return cudaErrorInvalidValue;
  QuantParams q = p;
  void* args[] = {&q};
  if (p.rows >= kWarpRowsFrom) {  // a warp per row (see launch_norm)
    const int cpl = (p.k / 8 + 31) / 32;
    const void* wk = cpl <= 4    ? (const void*)quant_fp8_warp_kernel<4>
                     : cpl <= 8  ? (const void*)quant_fp8_warp_kernel<8>
                     : cpl <= 12 ? (const void*)quant_fp8_warp_kernel<12>
                                 : (const void*)quant_fp8_warp_kernel<16>;
    return launch_rows(wk, args, p.rows, 0, stream, pdl, 8);
  }
  const void* kern = p.k <= 1024   ? (const void*)quant_fp8_kernel<1>
                     : p.k <= 2048 ? (const void*)quant_fp8_kernel<2>
                     : p.k <= 3072 ? (const void*)quant_fp8_kernel<3>
                                   : (const void*)quant_fp8_kernel<4>;
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

cudaError_t launch_gather_rows(float* dst, const float* src, const int* map, int rows, int d, cudaStream_t stream,
                               bool pdl) {
  void* args[] = {&dst, &src, &map, &rows, &d};
  return launch_rows((const void*)gather_rows_kernel, args, rows, 0, stream, pdl);
}

cudaError_t launch_tail(const TailParams& p, int batch, cudaStream_t stream, bool pdl) {
  if (p.k > 256) return cudaErrorInvalidValue;
  TailParams q = p;
  void* args[] = {&q};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(batch, kTailCtas, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = (256 + p.d + 8) * sizeof(float);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, (const void*)tail_kernel, args);
}

cudaError_t launch_pack_fp8_rows(const __nv_bfloat16* w, uint8_t* q, float* scale, int rows, int k,
                                 cudaStream_t stream) {
  pack_fp8_rows_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(w, q, scale, rows, k);
  return cudaGetLastError();
}

}  // namespace laya
