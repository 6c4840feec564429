// Token tables (the reference's fast-mode token_tables.py:13-38, an option
// there too): for every vocabulary id the embedding LayerNorm row (fp32, the
// residual stream's first value) and its layer-0 QKV projection (bf16, before
// the rotary embedding) are computed once with the engine's own kernels; a
// forward then starts with one gather that copies a token's rows and rotates
// q and k at the token's position, in place of the embedding norm and the
// layer-0 QKV projection.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "attention_tile.cuh"

namespace laya {

// One warp per token row t: h[t] = table_h[id], qkv[t] = rope(table_qkv[id])
// with position t % seq on q and k (layer 0 is a global layer).
__global__ void __launch_bounds__(256) token_gather_kernel(const TokenGatherParams p) {
  griddep_launch_dependents();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int id = p.ids[row], pos = row % p.seq, d = p.d;
  const float4* hs = reinterpret_cast<const float4*>(p.table_h + (size_t)id * d);
  float4* hd = reinterpret_cast<float4*>(p.h + (size_t)row * p.ldh);
  for (int c = lane; c < d / 4; c += 32) hd[c] = hs[c];
  const __nv_bfloat16* qs = p.table_qkv + (size_t)id * 3 * d;
  __nv_bfloat16* qd = p.qkv + (size_t)row * p.ldqkv;
  // q and k: per head, chunk c (8 dims, c < 4) with its partner c + 4
  const int heads = d / 64;
  const float* cs = p.cos + (size_t)pos * 64;
  const float* sn = p.sin + (size_t)pos * 64;
  for (int u = lane; u < 2 * heads * 4; u += 32) {
    const int col = (u / 4) * 64 + (u % 4) * 8;  // region (q, k) and head folded: heads are 64 apart
    uint4 lo = *reinterpret_cast<const uint4*>(qs + col);
    uint4 hi = *reinterpret_cast<const uint4*>(qs + col + 32);
    attn::rope8(lo, hi, cs, sn, (u % 4) * 8);
    *reinterpret_cast<uint4*>(qd + col) = lo;
    *reinterpret_cast<uint4*>(qd + col + 32) = hi;
  }
  for (int c = lane; c < d / 8; c += 32)
    *reinterpret_cast<uint4*>(qd + 2 * d + c * 8) = *reinterpret_cast<const uint4*>(qs + 2 * d + c * 8);
}

cudaError_t launch_token_gather(const TokenGatherParams& p, cudaStream_t stream, bool pdl) {
  if (p.d % 64 || p.rows < 1 || p.seq < 1) return cudaErrorInvalidValue;
  TokenGatherParams q = p;
  void* args[] = {&q};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.rows + 7) / 8, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, (const void*)token_gather_kernel, args);
}

}  // namespace laya
