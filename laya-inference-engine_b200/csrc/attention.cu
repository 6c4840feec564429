// Fused RoPE attention for the encoder (global and radius-64 local layers)
// and the head's key-padded attention.  Replaces rope_qkv + SDPA
// (src/laya_blackwell/model.py:92-96 and :62-67, kernels.py:62-93).
//
// One CTA = 64 queries of one (sequence, head); 4 warps x 16 queries, tensor
// cores through mma.sync m16n8k16 (bf16, fp32 accumulate).  Local layers only
// visit key tiles inside [q-64, q+64] (compute skipping, not just masking).
// Scores and the online softmax are fp32; P is rounded to bf16 for the P.V
// product (as FlashAttention does); a query that sees no key returns zeros
// (SDPA's result for a fully masked row).
//
// Two load paths:
//  * attention_kernel: Q and K are rotated while they are staged (batch-1
//    shapes, where the QKV projection's split-K epilogue does not rotate):
//    y = bf16(fl(a*cos) + fl(b*sin)) in fp32 without FMA contraction.
//  * attention_async_kernel: the QKV projection already rotated q and k in its
//    epilogue, so Q, K, V and the key-validity words are copied with cp.async
//    (zero-filled past the sequence), the next key tile's copies in flight while
//    the current tile is computed.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "attention_tile.cuh"

namespace laya {

namespace {
using namespace attn;

// Normalise and store this warp's 16 output rows.
DEVI void store_rows(const Acc& acc, const AttnParams& p, int b, int q0, int h, int warp, int lane) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = acc.lrow[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int qi = q0 + warp * 16 + g + 8 * r;
    if (qi < p.nq) {
      __nv_bfloat16* dst = p.out + ((size_t)b * p.nq + qi) * p.ld_out + h * 64;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
        *reinterpret_cast<uint32_t*>(dst + nt * 8 + 2 * t4) =
            pack_bf16(acc.o[nt][2 * r] * inv, acc.o[nt][2 * r + 1] * inv);
    }
  }
}

// Key range of the CTA's query tile: all keys, or the tiles covering
// [q0 - window, q_last + window] on local layers.
DEVI void key_range(const AttnParams& p, int q0, int& kbeg, int& kend) {
  kbeg = 0;
  kend = p.s;
  if (p.window >= 0) {  // queries of this tile are positions q0 .. q0+63
    const int qmax = min(q0 + AQ, p.nq) - 1;
    kbeg = max(0, q0 - p.window);
    kend = min(p.s, qmax + p.window + 1);
    kbeg = (kbeg / AK) * AK;
  }
}

}  // namespace

__global__ void __launch_bounds__(128) attention_kernel(const AttnParams p) {
  __shared__ __align__(16) __nv_bfloat16 sQ[AQ * LDS];
  __shared__ __align__(16) __nv_bfloat16 sK[AK * LDS];
  __shared__ __align__(16) __nv_bfloat16 sV[AK * LDS];
  __shared__ int s_qpos[AQ];
  __shared__ int s_kvalid[AK];

  griddep_launch_dependents();
  const int q0 = blockIdx.x * AQ, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  griddep_wait();

  if (tid < AQ) {
    const int qi = q0 + tid;
    s_qpos[tid] = qi < p.nq ? (p.q_pos ? p.q_pos[b * p.nq + qi] : qi) : -1;
  }
  __syncthreads();
  const size_t seq_base = (size_t)b * p.s;
  for (int it = tid; it < AQ * 4; it += 128) {
    const int r = it >> 2, c = (it & 3) * 8;
    const int pos = s_qpos[r];
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    if (pos >= 0) {
      const __nv_bfloat16* src = p.qkv + (seq_base + pos) * p.ld_qkv + h * 64;
      lo = *reinterpret_cast<const uint4*>(src + c);
      hi = *reinterpret_cast<const uint4*>(src + c + 32);
      if (p.cos) rope8(lo, hi, p.cos + (size_t)pos * 64, p.sin + (size_t)pos * 64, c);
    }
    *reinterpret_cast<uint4*>(&sQ[r * LDS + c]) = lo;
    *reinterpret_cast<uint4*>(&sQ[r * LDS + c + 32]) = hi;
  }
  int kbeg, kend;
  key_range(p, q0, kbeg, kend);
  __syncthreads();

  uint32_t qf[4][4];
  load_q_frags(qf, sQ, warp, lane);
  const int g = lane >> 2;
  const int qpos0 = s_qpos[warp * 16 + g], qpos1 = s_qpos[warp * 16 + g + 8];
  Acc acc;
  acc_init(acc);

  for (int k0 = kbeg; k0 < kend; k0 += AK) {
    __syncthreads();
    for (int it = tid; it < AK * 4; it += 128) {
      const int r = it >> 2, c = (it & 3) * 8;
      const int kp = k0 + r;
      uint4 klo = make_uint4(0, 0, 0, 0), khi = klo, vlo = klo, vhi = klo;
      if (kp < p.s) {
        const __nv_bfloat16* row = p.qkv + (seq_base + kp) * p.ld_qkv;
        const __nv_bfloat16* ks = row + p.d + h * 64;
        const __nv_bfloat16* vs = row + 2 * p.d + h * 64;
        klo = *reinterpret_cast<const uint4*>(ks + c);
        khi = *reinterpret_cast<const uint4*>(ks + c + 32);
        vlo = *reinterpret_cast<const uint4*>(vs + c);
        vhi = *reinterpret_cast<const uint4*>(vs + c + 32);
        if (p.cos) rope8(klo, khi, p.cos + (size_t)kp * 64, p.sin + (size_t)kp * 64, c);
      }
      *reinterpret_cast<uint4*>(&sK[r * LDS + c]) = klo;
      *reinterpret_cast<uint4*>(&sK[r * LDS + c + 32]) = khi;
      *reinterpret_cast<uint4*>(&sV[r * LDS + c]) = vlo;
      *reinterpret_cast<uint4*>(&sV[r * LDS + c + 32]) = vhi;
    }
    if (tid < AK) s_kvalid[tid] = (k0 + tid < p.s) ? (p.key_valid[seq_base + k0 + tid] != 0) : 0;
    __syncthreads();
    attend_tile(acc, qf, sK, sV, s_kvalid, k0, p.window, qpos0, qpos1, lane);
  }
  store_rows(acc, p, b, q0, h, warp, lane);
}

__global__ void __launch_bounds__(128) attention_async_kernel(const AttnParams p) {
  __shared__ __align__(16) __nv_bfloat16 sQ[AQ * LDS];
  __shared__ __align__(16) __nv_bfloat16 sK[2][AK * LDS];
  __shared__ __align__(16) __nv_bfloat16 sV[2][AK * LDS];
  __shared__ __align__(16) int s_kvalid[2][AK];
  __shared__ int s_qpos[AQ];

  griddep_launch_dependents();
  const int q0 = blockIdx.x * AQ, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  griddep_wait();

  if (tid < AQ) {
    const int qi = q0 + tid;
    s_qpos[tid] = qi < p.nq ? (p.q_pos ? p.q_pos[b * p.nq + qi] : qi) : -1;
  }
  __syncthreads();
  const size_t seq_base = (size_t)b * p.s;
  // Q: 64 rows x 8 chunks of 16 bytes
  for (int it = tid; it < AQ * 8; it += 128) {
    const int r = it >> 3, c = (it & 7) * 8;
    const int pos = s_qpos[r];
    const __nv_bfloat16* src = pos >= 0 ? p.qkv + (seq_base + pos) * p.ld_qkv + h * 64 + c : p.qkv;
    cp_async16(&sQ[r * LDS + c], src, pos >= 0);
  }
  int kbeg, kend;
  key_range(p, q0, kbeg, kend);
  const int ntiles = (kend - kbeg + AK - 1) / AK;
  auto issue_tile = [&](int t) {
    const int k0 = kbeg + t * AK, buf = t & 1;
    for (int it = tid; it < AK * 8; it += 128) {
      const int r = it >> 3, c = (it & 7) * 8;
      const int kp = k0 + r;
      const bool ok = kp < p.s;
      const __nv_bfloat16* row = ok ? p.qkv + (seq_base + kp) * p.ld_qkv : p.qkv;
      cp_async16(&sK[buf][r * LDS + c], row + p.d + h * 64 + c, ok);
      cp_async16(&sV[buf][r * LDS + c], row + 2 * p.d + h * 64 + c, ok);
    }
    if (tid < AK) {
      const bool ok = k0 + tid < p.s;
      cp_async4(&s_kvalid[buf][tid], ok ? p.key_valid + seq_base + k0 + tid : p.key_valid, ok);
    }
    cp_commit();
  };
  if (ntiles > 0) issue_tile(0);  // first group also carries Q
  else cp_commit();

  const int g = lane >> 2;
  const int qpos0 = s_qpos[warp * 16 + g], qpos1 = s_qpos[warp * 16 + g + 8];
  Acc acc;
  acc_init(acc);
  uint32_t qf[4][4];
  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) {
      issue_tile(t + 1);
      cp_wait_all_but_one();
    } else {
      cp_wait_all();
    }
    __syncthreads();
    if (t == 0) load_q_frags(qf, sQ, warp, lane);
    attend_tile(acc, qf, sK[t & 1], sV[t & 1], s_kvalid[t & 1], kbeg + t * AK, p.window, qpos0, qpos1, lane);
    __syncthreads();  // buffer t & 1 is refilled by the copies issued in the next iteration
  }
  cp_wait_all();
  store_rows(acc, p, b, q0, h, warp, lane);
}

cudaError_t launch_attention(const AttnParams& p, int batch, int heads, cudaStream_t stream, bool pdl) {
  if (p.window >= 0 && p.q_pos) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.nq + AQ - 1) / AQ, heads, batch);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (p.cos) return cudaLaunchKernelEx(&cfg, attention_kernel, p);
  return cudaLaunchKernelEx(&cfg, attention_async_kernel, p);
}

}  // namespace laya
