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
//  * attention_split_kernel: the same copies with eight warps, for grids of
//    fewer CTAs than SMs: warps 0-3 take the even key tiles and warps 4-7 the
//    odd ones, each group with its own online softmax, merged at the end; the
//    next pair of tiles is copied while the current pair is computed.
#include "common.cuh"
#include "params.h"
#include "launch.h"
#include "attention_tile.cuh"

#include <mutex>

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

// Shared memory of attention_split_kernel: Q, two stages x two key groups of
// K and V tiles, their key-validity words, the query positions.
constexpr int kSplitThreads = 256;
constexpr int kTileBytes = AK * LDS * 2;
constexpr int kSplitSmem = AQ * LDS * 2 + 8 * kTileBytes + 4 * AK * 4 + AQ * 4;

__global__ void __launch_bounds__(kSplitThreads) attention_split_kernel(const AttnParams p) {
  extern __shared__ __align__(16) uint8_t att_smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(att_smem);
  // K tile of (stage st, group gr) at sKV + (st * 2 + gr) * 2 tiles, V right after it
  __nv_bfloat16* sKV = sQ + AQ * LDS;
  int* s_kvalid = reinterpret_cast<int*>(att_smem + AQ * LDS * 2 + 8 * kTileBytes);  // [stage][group][AK]
  int* s_qpos = s_kvalid + 4 * AK;

  griddep_launch_dependents();
  const int q0 = blockIdx.x * AQ, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = warp >> 2, qw = warp & 3;  // key group, query quarter
  griddep_wait();

  if (tid < AQ) {
    const int qi = q0 + tid;
    s_qpos[tid] = qi < p.nq ? (p.q_pos ? p.q_pos[b * p.nq + qi] : qi) : -1;
  }
  __syncthreads();
  const size_t seq_base = (size_t)b * p.s;
  // Q: 64 rows x 8 chunks of 16 bytes
  for (int it = tid; it < AQ * 8; it += kSplitThreads) {
    const int r = it >> 3, c = (it & 7) * 8;
    const int pos = s_qpos[r];
    const __nv_bfloat16* src = pos >= 0 ? p.qkv + (seq_base + pos) * p.ld_qkv + h * 64 + c : p.qkv;
    cp_async16(&sQ[r * LDS + c], src, pos >= 0);
  }
  int kbeg, kend;
  key_range(p, q0, kbeg, kend);
  const int ntiles = (kend - kbeg + AK - 1) / AK;
  const int npairs = (ntiles + 1) / 2;
  // step j: key tile 2j for group 0, 2j+1 for group 1, into stage j & 1
  auto issue_pair = [&](int j) {
    const int st = j & 1;
    for (int it = tid; it < 2 * AK * 8; it += kSplitThreads) {
      const int gr = it / (AK * 8), r = (it >> 3) & (AK - 1), c = (it & 7) * 8;
      const int t = 2 * j + gr;
      if (t >= ntiles) continue;
      const int kp = kbeg + t * AK + r;
      const bool ok = kp < p.s;
      const __nv_bfloat16* row = ok ? p.qkv + (seq_base + kp) * p.ld_qkv : p.qkv;
      __nv_bfloat16* sK = sKV + (st * 2 + gr) * 2 * AK * LDS;
      cp_async16(&sK[r * LDS + c], row + p.d + h * 64 + c, ok);
      cp_async16(&sK[AK * LDS + r * LDS + c], row + 2 * p.d + h * 64 + c, ok);
    }
    if (tid < 2 * AK) {
      const int gr = tid / AK, t = 2 * j + gr, kp = kbeg + t * AK + (tid & (AK - 1));
      if (t < ntiles) {
        const bool ok = kp < p.s;
        cp_async4(&s_kvalid[(st * 2 + gr) * AK + (tid & (AK - 1))], ok ? p.key_valid + seq_base + kp : p.key_valid, ok);
      }
    }
    cp_commit();
  };
  if (npairs > 0) issue_pair(0);  // first group also carries Q
  else cp_commit();

  const int g = lane >> 2;
  const int qpos0 = s_qpos[qw * 16 + g], qpos1 = s_qpos[qw * 16 + g + 8];
  Acc acc;
  acc_init(acc);
  uint32_t qf[4][4];
  for (int j = 0; j < npairs; ++j) {
    if (j + 1 < npairs) {
      issue_pair(j + 1);
      cp_wait_all_but_one();
    } else {
      cp_wait_all();
    }
    __syncthreads();
    if (j == 0) load_q_frags(qf, sQ, qw, lane);
    const int t = 2 * j + grp, st = j & 1;
    if (t < ntiles) {
      const __nv_bfloat16* sK = sKV + (st * 2 + grp) * 2 * AK * LDS;
      attend_tile(acc, qf, sK, sK + AK * LDS, s_kvalid + (st * 2 + grp) * AK, kbeg + t * AK, p.window, qpos0, qpos1,
                  lane);
    }
    __syncthreads();  // stage j & 1 is refilled by the copies issued in the next step
  }
  cp_wait_all();
  __syncthreads();
  // merge the two key groups' online-softmax states (same fragment layout):
  // m = max(m0, m1), l and O rescaled by exp2(m_i - m)
  float* xch = reinterpret_cast<float*>(sKV) + (qw * 32 + lane) * 36;
  if (grp == 1) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) xch[nt * 4 + e] = acc.o[nt][e];
    xch[32] = acc.mrow[0];
    xch[33] = acc.mrow[1];
    xch[34] = acc.lrow[0];
    xch[35] = acc.lrow[1];
  }
  __syncthreads();
  if (grp == 0) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float m1 = xch[32 + r], l1 = xch[34 + r], m0 = acc.mrow[r];
      const float m = fmaxf(m0, m1);
      const float c0 = m == -INFINITY ? 0.f : exp2f(m0 - m);
      const float c1 = m == -INFINITY ? 0.f : exp2f(m1 - m);
      acc.lrow[r] = acc.lrow[r] * c0 + l1 * c1;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        acc.o[nt][2 * r] = acc.o[nt][2 * r] * c0 + xch[nt * 4 + 2 * r] * c1;
        acc.o[nt][2 * r + 1] = acc.o[nt][2 * r + 1] * c0 + xch[nt * 4 + 2 * r + 1] * c1;
      }
      acc.mrow[r] = m;
    }
    store_rows(acc, p, b, q0, h, qw, lane);
  }
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
  // Fewer CTAs than SMs (long sequences at small batch): split the key tiles
  // over two warp groups (measured 2.07 -> 1.85 ms per C3 forward); with
  // several CTAs per SM the four-warp kernel is faster (C2: 2.62 vs 2.75 ms).
  static std::mutex mu;
  static uint64_t ready = 0;
  static int sms[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(ready >> dev & 1)) {
      err = cudaFuncSetAttribute(attention_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmem);
      if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (err != cudaSuccess) return err;
      ready |= uint64_t(1) << dev;
    }
  }
  const long long ctas = (long long)cfg.gridDim.x * cfg.gridDim.y * cfg.gridDim.z;
  if (ctas > sms[dev]) return cudaLaunchKernelEx(&cfg, attention_async_kernel, p);
  cfg.blockDim = dim3(kSplitThreads, 1, 1);
  cfg.dynamicSmemBytes = kSplitSmem;
  return cudaLaunchKernelEx(&cfg, attention_split_kernel, p);
}

}  // namespace laya
