// Attention tile arithmetic of the fused batch-1 attention + output
// projection (gemm_attn.cu): 64 queries x 64 keys of one head, four warps of
// 16 queries, register-level tensor-core tiles (mma.sync m16n8k16, bf16 in,
// fp32 accumulate), online softmax in fp32 with P rounded to bf16 for P.V (as
// FlashAttention does); and the rotary embedding of staged rows (rope_qkv,
// kernels.py:62-93) used by the token-table gather.  Every batched shape runs
// attention on tcgen05 instead (attention.cu); at 64 tokens these tiles are
// shorter than a tensor-memory round trip.
#pragma once
#include "common.cuh"

namespace laya {
namespace attn {
constexpr int AQ = 64;    // queries per CTA
constexpr int AK = 64;    // keys per tile
constexpr int LDS = 72;   // padded shared row (bf16 elements)

DEVI void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
DEVI void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
DEVI void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
DEVI uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

DEVI void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
DEVI void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
DEVI void cp_wait_all_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
DEVI void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Rotate 8 dims [c, c+8) (c < 32) together with their partners [c+32, c+40).
DEVI void rope8(uint4& lo, uint4& hi, const float* cs, const float* sn, int c) {
  __nv_bfloat16* xl = reinterpret_cast<__nv_bfloat16*>(&lo);
  __nv_bfloat16* xh = reinterpret_cast<__nv_bfloat16*>(&hi);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = __bfloat162float(xl[e]);
    const float b = __bfloat162float(xh[e]);
    const float yl = __fadd_rn(__fmul_rn(a, cs[c + e]), __fmul_rn(-b, sn[c + e]));
    const float yh = __fadd_rn(__fmul_rn(b, cs[c + e + 32]), __fmul_rn(a, sn[c + e + 32]));
    xl[e] = __float2bfloat16_rn(yl);
    xh[e] = __float2bfloat16_rn(yh);
  }
}

// Per-warp state of the online softmax for its 16 queries.
struct Acc {
  float o[8][4];
  float mrow[2], lrow[2];
};

DEVI void acc_init(Acc& a) {
#pragma unroll
  for (int i = 0; i < 8; ++i) a.o[i][0] = a.o[i][1] = a.o[i][2] = a.o[i][3] = 0.f;
  a.mrow[0] = a.mrow[1] = -INFINITY;
  a.lrow[0] = a.lrow[1] = 0.f;
}

// Q fragments of this warp's 16 rows (4 k-steps of 16 dims).
DEVI void load_q_frags(uint32_t (&qf)[4][4], const __nv_bfloat16* sQ, int warp, int lane) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
    ldsm_x4(qf[ks], &sQ[(warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LDS + ks * 16 + (lane >> 4) * 8]);
}

// One key tile (64 keys from position k0): scores, masking (key validity and
// window), online-softmax update, O += P V.
DEVI void attend_tile(Acc& acc, const uint32_t (&qf)[4][4], const __nv_bfloat16* sK, const __nv_bfloat16* sV,
                      const int* kvalid, int k0, int window, int qpos0, int qpos1, int lane) {
  const int t4 = lane & 3;
  const float kScaleLog2 = 0.125f * 1.4426950408889634f;
  float sc[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t kb[4];
      ldsm_x4(kb, &sK[(nt * 8 + (lane & 7)) * LDS + kk * 32 + (lane >> 3) * 8]);
      mma16816(sc[nt], qf[2 * kk], kb[0], kb[1]);
      mma16816(sc[nt], qf[2 * kk + 1], kb[2], kb[3]);
    }
  }
  float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int kl = nt * 8 + 2 * t4 + (e & 1);
      const int kp = k0 + kl;
      const int qp = (e >> 1) ? qpos1 : qpos0;
      bool vis = kvalid[kl] != 0 && qp >= 0;
      if (window >= 0) vis = vis && abs(qp - kp) <= window;
      const float v = vis ? sc[nt][e] * kScaleLog2 : -INFINITY;
      sc[nt][e] = v;
      tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
    tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
    const float mnew = fmaxf(acc.mrow[r], tmax[r]);
    const float msafe = mnew == -INFINITY ? 0.f : mnew;
    const float corr = exp2f(acc.mrow[r] - msafe);
    acc.lrow[r] *= corr;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      acc.o[nt][2 * r] *= corr;
      acc.o[nt][2 * r + 1] *= corr;
    }
    acc.mrow[r] = mnew;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(sc[nt][2 * r] - msafe);
      const float p1 = exp2f(sc[nt][2 * r + 1] - msafe);
      sc[nt][2 * r] = p0;
      sc[nt][2 * r + 1] = p1;
      acc.lrow[r] += p0 + p1;
    }
  }
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    uint32_t pa[4];
    pa[0] = pack_bf16(sc[2 * ks][0], sc[2 * ks][1]);
    pa[1] = pack_bf16(sc[2 * ks][2], sc[2 * ks][3]);
    pa[2] = pack_bf16(sc[2 * ks + 1][0], sc[2 * ks + 1][1]);
    pa[3] = pack_bf16(sc[2 * ks + 1][2], sc[2 * ks + 1][3]);
#pragma unroll
    for (int nt2 = 0; nt2 < 4; ++nt2) {
      uint32_t vb[4];
      ldsm_x4_t(vb, &sV[(ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LDS + nt2 * 16 + (lane >> 4) * 8]);
      mma16816(acc.o[2 * nt2], pa, vb[0], vb[1]);
      mma16816(acc.o[2 * nt2 + 1], pa, vb[2], vb[3]);
    }
  }
}

}  // namespace attn
}  // namespace laya
