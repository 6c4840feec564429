// Kernel parameter blocks shared by the host runtime and the kernels.
#pragma once
#include <stdint.h>
#include <cuda_bf16.h>

namespace laya {

// Epilogues of the projection GEMM.  v is the fp32 accumulator after the
// precision's scales; every bf16() is a round-to-nearest-even to bf16.
enum GemmEpilogue : int {
  kEpiStore = 0,     // out[m][n] = bf16(v + bias[n])
  kEpiRelu = 1,      // out[m][n] = bf16(relu(v + bias[n]))
  kEpiGelu = 2,      // out[m][n] = bf16(gelu(bf16(v + bias[n])))
  kEpiGeglu = 3,     // tile rows 0-63 act, 64-127 gate: out[m][j] = bf16(bf16(gelu(bf16(act))) * bf16(gate))
  kEpiResidual = 4,  // resid[m][n] += bf16(v + bias[n])   (fp32 residual stream)
};

enum GemmKind : int { kKindBf16 = 0, kKindFp8 = 1, kKindNvfp4 = 2 };

struct NormParams {
  int rows;
  int d;
  float eps;
  // Source rows: embedding table gathered by token id, or an fp32 matrix
  // (optionally through a row map).
  const int* tok_ids;       // [rows] or null
  const float* src;         // fp32 [*, ld_src] (table when tok_ids != null)
  int ld_src;
  const int* row_map;       // [rows] source row per output row, or null
  const float* w;           // LayerNorm weight [d]
  const float* b;           // LayerNorm bias [d] or null
  // y = LN(x) * w + b (+ add_table[add_idx[row / add_div]])
  const float* add_table;   // [*, d] or null
  const int* add_idx;
  int add_div;
  float* out_f32;           // y (fp32) or null; may alias src (in place)
  int ld_out_f32;
  // bf16 output: bf16(y) when second_w == null; otherwise bf16(LN2(y)) with
  // second_w / second_b (a second LayerNorm fused on the same row).
  const float* second_w;
  const float* second_b;
  __nv_bfloat16* out_bf16;  // [rows][d] or null
  uint8_t* out_fp8;         // e4m3 per-row quantisation of the bf16 output, or null
  float* out_fp8_scale;     // [rows]
  // NVFP4 quantisation of the bf16 output (per-row outer scale), laid out for
  // a projection with `x4_rows_per_block`-token tiles, or null
  uint8_t* out_x4;          // e2m1 [rows][d/2]
  uint8_t* out_x4_sf;       // e4m3 block scales (tiled)
  float* out_x4_outer;      // [rows]
  int x4_rows_per_block;
  int x4_col_blocks;
};

struct GemmParams {
  int M;          // token rows
  int N;          // weight rows (features) -- multiple of 128
  int K;          // reduction length in elements
  int kblocks;    // number of K blocks
  int epilogue;   // GemmEpilogue
  __nv_bfloat16* out;       // bf16 output [M][ldo]
  int ldo;
  float* resid;             // fp32 residual [M][ldr] (kEpiResidual)
  int ldr;
  const __nv_bfloat16* bias;  // [N] or null
  const float* a_scale;     // fp8/nvfp4: per-token fp32 scale [M]
  const float* w_scale;     // fp8: per-feature fp32 scale [N]
  float w_tensor_scale;     // nvfp4: weight tensor scale
  uint32_t* status;         // device-visible status word
  // 1: unsplit tiles use the TMA epilogue (the kernel's omap describes the
  // output: bf16 [M][ldo] with a (128 | 64 for GEGLU) x BN box, or the fp32
  // residual [M][ldr] with a 128 x BN box).
  int tma_epilogue;
  // Rotary embedding applied in the wide epilogue to output columns
  // [0, rope_cols) (q and k of a QKV projection): position = row % rope_seq,
  // tables [max_len][64].  rope_cols = 0 disables it.
  const float* rope_cos;
  const float* rope_sin;
  int rope_seq;
  int rope_cols;
  float* partials;           // global split-K partials [tiles][split][BN][128] floats, or null
  // Residual projections feeding a LayerNorm that the next projection applies
  // on load: per (token, 128-column tile) statistics of the updated residual
  // row, (mean, sum of squared deviations) over the tile, at
  // [token * (N / 128) + tile].
  float2* ln_stats;
  // Test hooks (zero in every normal launch): wait_limit_us shortens every
  // bounded wait of the launch; test_withhold = 1 + the index of a prefetched
  // pipeline stage whose loads are never issued, so the waits on it run out
  // (gemm_kernel only).
  uint32_t wait_limit_us;
  int test_withhold;
};

// LayerNorm applied by a projection to its fp32 input rows while building the
// bf16 operand (batch-1 path): LN(h) * w with the row statistics merged from
// the per-tile partials the previous residual projection wrote.
struct LnParams {
  const float* h;           // fp32 [M][ldh] residual rows
  int ldh;
  const float* w;           // LayerNorm weight [K]
  const float2* stats;      // [M][ntiles] (mean, M2) over 128-column tiles
  int ntiles;               // K / 128
  float eps;
};


// Forward start from the token tables (token_tables.cu).
struct TokenGatherParams {
  int rows;                        // tokens
  int seq;                         // tokens per sequence (position = row % seq)
  int d;
  const int* ids;                  // [rows]
  const float* table_h;            // [vocab][d] embedding LayerNorm rows
  const __nv_bfloat16* table_qkv;  // [vocab][3d] layer-0 QKV rows, q / k not rotated
  const float* cos;                // [max_len][64] global rotary tables
  const float* sin;
  float* h;                        // [rows][ldh]
  int ldh;
  __nv_bfloat16* qkv;              // [rows][ldqkv]
  int ldqkv;
};

struct AttnParams {
  const __nv_bfloat16* qkv;  // [tokens][ld_qkv]; q at col h*64, k at d + h*64, v at 2d + h*64
  int ld_qkv;
  int d;                     // heads * 64
  int s;                     // keys per sequence
  int nq;                    // queries per sequence
  const int* q_pos;          // [b][nq] query positions, or null (query i at position i)
  const int* key_valid;      // [b][s] 1 = visible key
  int window;                // -1 global; else |q - k| <= window
  __nv_bfloat16* out;        // [b*nq][ld_out]
  int ld_out;
  uint32_t* status;          // device-visible status word (bounded waits)
  uint32_t wait_limit_us;    // 0: the default limit
};

struct QuantParams {
  int rows;
  int k;
  const __nv_bfloat16* src;  // [rows][k]
  uint8_t* q;                // e4m3 [rows][k]  (fp8) or e2m1 [rows][k/2] (nvfp4)
  float* scale;              // per-row fp32 scale (fp8) / outer (nvfp4)
  uint8_t* sf;               // nvfp4 block scales in the MMA's tiled layout
  int sf_cols;               // nvfp4: padded scale columns per row group
};

struct TailParams {
  int k;                     // options per question
  int d;
  int act_hidden;
  const __nv_bfloat16* z;    // gelu(scorer.fc1) rows [b*k][d]
  const __nv_bfloat16* fc2_w;  // [d]
  const __nv_bfloat16* fc2_b;  // [1]
  const int* marker_mask;    // [b][k]
  const float* h_sel;        // [b*(1+k)][d]; row 0 of each question is CLS
  const __nv_bfloat16* a1_w;   // [act_hidden][d+4]
  const __nv_bfloat16* a1_b;
  const __nv_bfloat16* a2_w;   // [2][act_hidden]
  const __nv_bfloat16* a2_b;
  float* logits;             // [b][k]
  float* act;                // [b][2]
  float* a1;                 // scratch [b][act_hidden]: act_head layer-1 outputs
  unsigned int* arrivals;    // [b] CTA arrival counters, zero between launches
};

}  // namespace laya
