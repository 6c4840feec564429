// Host-side launchers of the b200 kernels (all take the stream to enqueue on
// and whether to allow programmatic dependent launch on the previous kernel).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include "params.h"

namespace laya {

int gemm_token_tile(int M);
void gemm_plan(int M, int N, int kblocks, int sm_count, int* bn, int* split);
int gemm_k_elems(int kind);
int gemm_split(int tiles, int kblocks, int sm_count, int max_split);
cudaError_t launch_gemm(int kind, const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap,
                        const GemmParams& p, int bn, int split, cudaStream_t stream, bool pdl);

// Fused attention + residual output projection for one sequence of
// 32 < s <= 64 tokens (bf16, q and k already rotated): attention of the CTA's
// heads computed in shared memory as the B operand (gemm_attn.cu).
cudaError_t launch_gemm_attn(const CUtensorMap& wmap, const GemmParams& p, const AttnParams& a, int split,
                             cudaStream_t stream, bool pdl);
// Projection (store / GEGLU epilogue) of LN(h) for one sequence of
// 32 < s <= 64 tokens (bf16): the LayerNorm is applied while the operand is
// built, from the row statistics of the previous residual projection
// (gemm_ln.cu).
cudaError_t launch_gemm_ln(const CUtensorMap& wmap, const GemmParams& p, const LnParams& ln, int split,
                           cudaStream_t stream, bool pdl);
cudaError_t launch_gemm_nvfp4(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap,
                              const uint8_t* wsf,
                              const uint8_t* xsf, int sf_kbs, const GemmParams& p, int bn, int split,
                              cudaStream_t stream, bool pdl);
cudaError_t launch_nvfp4_pack_weight(const __nv_bfloat16* w, int rows, int k, unsigned int* amax_scratch, uint8_t* q,
                                     uint8_t* sf, int col_blocks, float* tensor_scale, cudaStream_t stream);
cudaError_t launch_quant_nvfp4(const QuantParams& p, int rows_per_block, int col_blocks, cudaStream_t stream,
                               bool pdl);
// Attention of `heads` heads of `batch` sequences on tcgen05 tensor cores;
// qkv_map: 3-D map of p.qkv as [batch][s][ld_qkv] bf16, box 64 x 64 x 1,
// 128-byte swizzle.  At most 512 keys visible to any 128-query tile.
cudaError_t launch_attention(const AttnParams& p, const CUtensorMap& qkv_map, int batch, int heads,
                             cudaStream_t stream, bool pdl);
// Chunks of 64 keys the widest query tile of p sees (the kernel takes <= 8).
int attention_chunks(const AttnParams& p);
// CTAs that share one query tile's key chunks (1 or 2) for a grid of
// base_ctas (tile, head, sequence) CTAs on sm_count SMs.
int attention_split(int base_ctas, int chunks, int sm_count);
cudaError_t launch_norm(const NormParams& p, cudaStream_t stream, bool pdl);
cudaError_t launch_quant_fp8(const QuantParams& p, cudaStream_t stream, bool pdl);
cudaError_t launch_gather_rows(float* dst, const float* src, const int* map, int rows, int d, cudaStream_t stream,
                               bool pdl);
cudaError_t launch_tail(const TailParams& p, int batch, cudaStream_t stream, bool pdl);
cudaError_t launch_token_gather(const TokenGatherParams& p, cudaStream_t stream, bool pdl);
cudaError_t launch_pack_fp8_rows(const __nv_bfloat16* w, uint8_t* q, float* scale, int rows, int k,
                                 cudaStream_t stream);

}  // namespace laya
