// Fused attention for the encoder (global and radius-64 local layers) and the
// head's key-padded attention, on tcgen05 tensor cores.  Replaces SDPA in
// src/laya_blackwell/model.py:92-96 (encoder) and :62-67 (head), whose fast
// paths are the reference's FA2 kernel (fast/native/global_attention.cu:12-68)
// and its window attention (fast/padded_rope.py:45-92).  q and k arrive
// rotated: the QKV projection's epilogue applies the rotary embedding.
//
// One CTA = 128 queries (the 128 TMEM lanes) of one (sequence, head) against
// every key those queries can see: all keys of the sequence on global layers,
// keys [q0 - 64, q0 + 127 + 64] on local layers.  The span is at most 512
// keys, so the whole score row of a query fits in TMEM (512 fp32 columns) and
// the softmax is exact and two-pass, with no running-max rescaling of O:
//
//  * warp 0, lane 0: TMA loads of Q (128 rows), every K and V chunk of 64
//    keys (the [batch][seq][3*hidden] map reads rows past the sequence as
//    zeros), then the MMAs: S = Q K^T per 128 keys (M=128, N=128, K=64) into
//    TMEM columns [0, keys), and for each 64-key chunk O += P V (M=128, N=64,
//    K=64; V is the MN-major B operand straight from its TMA tile) into TMEM
//    columns [0, 64), which chunk 0's scores free before its P is released.
//  * warp 1: key-validity bits (one word per 32 keys) and, for the head's
//    selected query rows, the gather of Q into the swizzled layout.
//  * split CTAs: when the (query tile, head, sequence) grid is smaller than
//    the GPU (one long sequence), a cluster of 2 CTAs (the code takes up to
//    4) shares each query tile, each CTA taking a contiguous share of its key
//    chunks.  The CTAs
//    push each row's max to one another (st.async into the peers' shared
//    memory, counted on their mbarriers), so all use the row's true max; each
//    then sums p and accumulates O over its own keys, and CTA r of n gathers
//    columns [64r/n, 64(r+1)/n) of O and the row sums from the others, adding
//    the n partials in rank order.
//  * warps 2-9: two threads per query row (warps 2-5 and 6-9 cover the four
//    TMEM lane quarters twice), each owning 32 of every 64 key columns.
//    Pass 1 reads the row's scores from TMEM and takes the max over visible
//    keys; pass 2 reads them again, computes p = 2^(s*log2(e)/8 - max), sums
//    p in fp32 and writes it as two bf16 tiles, hi = bf16(p) and
//    lo = bf16(p - hi) (128-byte swizzle, double-buffered, in the Q and K
//    space the score MMAs have finished with); the two halves' max and sum
//    meet in shared memory; the epilogue scales O by 1/sum and each thread
//    stores 32 of the row's 64 bf16 outputs.  A warp whose 32 rows all lie
//    past the last query keeps only the barrier protocol.
//
// Numerics: scores and the softmax in fp32; P.V as hi.V + lo.V, which carries
// p to about 16 significant bits (V is bf16, so each product is exact in the
// fp32 accumulator) instead of rounding it to bf16 as FlashAttention does:
// the result tracks an fp32-probability softmax (the reference's CPU path,
// which its golden outputs come from) to within fp32 summation order.  A query
// that sees no key returns zeros (SDPA's result for a fully masked row).
//
// Every mbarrier wait is bounded; on expiry the CTA records
// kStatusAttnTimeout, waits (bounded) for its own copies and MMAs, frees TMEM
// and returns.  TMEM is allocated after griddepcontrol.wait (so the
// projection before it has released its columns) and the next kernel is
// released only after the allocation (so it cannot take columns first and
// then wait on this grid).
#include "common.cuh"
#include "params.h"
#include "launch.h"

#include <mutex>

namespace laya {

namespace {

constexpr int kTq = 128;          // queries per CTA (TMEM lanes)
constexpr int kKc = 64;           // keys per chunk (one TMA box, one P tile)
constexpr int kMaxChunks = 8;     // 512 keys: the TMEM columns of one score row
constexpr int kThreads = 320;     // warp 0 TMA + MMA, warp 1 setup, warps 2-9 softmax
constexpr int kSoftmaxThreads = 256;
constexpr uint32_t kQBytes = kTq * 128;
constexpr uint32_t kChunkBytes = kKc * 128;
constexpr uint32_t kPBytes = kTq * 128;
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
// O += P V: bf16 x bf16 -> fp32, M = 128, N = 64, B (V) MN-major.
constexpr uint32_t kIdescPV = idesc_bf16(128, 64) | (1u << 16);

// Shared memory (from a 1024-aligned base): Q, the K region, the V chunks,
// the partial O columns received from the other CTAs of a split tile, then
// barriers, key bits, the TMEM slot and the row reductions.  Once every score
// MMA has completed, Q and the K region hold the four P tiles (hi and lo, two
// buffers), hence a K region of at least 6 chunks.
constexpr int kMaxSplit = 4;
constexpr uint32_t kBarBytes = 6144;
struct Layout {
  uint32_t k, v, recv, bars, total;
};
__host__ __device__ constexpr uint32_t kregion(int chunks) { return (chunks > 6 ? chunks : 6) * kChunkBytes; }
__host__ __device__ constexpr uint32_t recv_bytes(int split) { return (split - 1) * kTq * (64 / split) * 4; }
__host__ __device__ constexpr Layout layout(int chunks, int split) {
  return Layout{kQBytes, kQBytes + kregion(chunks), kQBytes + kregion(chunks) + chunks * kChunkBytes,
                kQBytes + kregion(chunks) + chunks * kChunkBytes + recv_bytes(split),
                kQBytes + kregion(chunks) + chunks * kChunkBytes + recv_bytes(split) + kBarBytes};
}
struct Bars {
  uint64_t q, k[kMaxChunks], v[kMaxChunks], s[kMaxChunks / 2], p[2], pv[2], o;
  uint64_t xm, xo;  // split tiles: the other CTAs' row maxima / O columns and sums arrived
  uint32_t key_bits[2 * kMaxChunks];
  uint32_t tmem_slot, failed;
  float red_max[2][kTq], red_sum[2][kTq];  // the two half-rows' max and sum
  float peer_max[kMaxSplit - 1][kTq], peer_sum[kMaxSplit - 1][kTq];
};
static_assert(sizeof(Bars) <= kBarBytes, "barrier block");

// Slot of sender s in receiver r's arrays (the receiver itself has none).
__host__ __device__ constexpr int peer_slot(int s, int r) { return s < r ? s : s - 1; }

// Keys [kbeg, kend) that the CTA's queries q0 .. q0+127 can see.
__host__ __device__ inline void key_span(const AttnParams& p, int q0, int& kbeg, int& kend) {
  kbeg = 0;
  kend = p.s;
  if (p.window >= 0) {
    const int qmax = (q0 + kTq < p.nq ? q0 + kTq : p.nq) - 1;
    kbeg = q0 - p.window > 0 ? q0 - p.window : 0;
    kend = qmax + p.window + 1 < p.s ? qmax + p.window + 1 : p.s;
  }
}

DEVI uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Named barrier of the softmax warps.
DEVI void softmax_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxThreads) : "memory"); }

// Keys base .. base+31 (relative to kbeg) that a row seeing keys [lo, hi]
// sees: the key-validity bits restricted to that range.
DEVI uint32_t visible_mask(uint32_t bits, int base, int lo, int hi) {
  const int a = lo - base, z = hi - base;
  if (a > 31 || z < 0 || a > z) return 0u;
  const uint32_t from = a <= 0 ? 0xffffffffu : 0xffffffffu << a;
  const uint32_t to = z >= 31 ? 0xffffffffu : 0xffffffffu >> (31 - z);
  return bits & from & to;
}

DEVI float ex2(float x) { return ex2_approx(x); }

// Max over the visible scores of 32 consecutive keys.
DEVI float masked_max(const uint32_t (&r)[32], uint32_t vis, float m) {
  if (vis == 0xffffffffu) {
#pragma unroll
    for (int e = 0; e < 32; ++e) m = fmaxf(m, __uint_as_float(r[e]));
    return m;
  }
#pragma unroll
  for (int e = 0; e < 32; ++e) m = fmaxf(m, (vis >> e) & 1u ? __uint_as_float(r[e]) : -INFINITY);
  return m;
}

// bf16 pairs of (a, b) and of their remainders (a - bf16(a), b - bf16(b)).
DEVI void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack2(a - __low2float(h), b - __high2float(h));
}

// p = 2^(s * scale - ms) for visible keys, 0 otherwise; adds p to l and packs
// the bf16 pairs of p into ph[0..15] and of its remainder into pl.
DEVI void probs(const uint32_t (&r)[32], uint32_t vis, float ms, float& l, uint32_t* ph, uint32_t* pl) {
  float p[32];
  if (vis == 0xffffffffu) {
#pragma unroll
    for (int e = 0; e < 32; ++e) p[e] = ex2(__uint_as_float(r[e]) * kScaleLog2 - ms);
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) p[e] = ex2((vis >> e) & 1u ? __uint_as_float(r[e]) * kScaleLog2 - ms : -INFINITY);
  }
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    l += p[e] + p[e + 1];
    split2(p[e], p[e + 1], ph[e >> 1], pl[e >> 1]);
  }
}


}  // namespace

template <int SPLIT>
__global__ void __launch_bounds__(kThreads, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap qkv_map, const AttnParams p, int max_chunks) {
  constexpr int W = 64 / SPLIT;  // output columns gathered by each CTA of a split tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = layout(max_chunks, SPLIT);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + L.k;
  uint8_t* sV = smem + L.v;
  float* recv = reinterpret_cast<float*>(smem + L.recv);  // [SPLIT-1][kTq][W]
  Bars& B = *reinterpret_cast<Bars*>(smem + L.bars);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = SPLIT > 1 ? (int)(blockIdx.x % SPLIT) : 0;
  const int q0 = (blockIdx.x / SPLIT) * kTq, h = blockIdx.y, b = blockIdx.z;
  int kbeg, kend;
  key_span(p, q0, kbeg, kend);
  {  // this CTA's share of the tile's key chunks
    const int all = (kend - kbeg + kKc - 1) / kKc;
    const int c0 = rank * all / SPLIT, c1 = (rank + 1) * all / SPLIT;
    const int end = kbeg + c1 * kKc < kend ? kbeg + c1 * kKc : kend;
    kbeg += c0 * kKc;
    kend = end > kbeg ? end : kbeg;
  }
  const int nk = kend - kbeg;
  const int chunks = (nk + kKc - 1) / kKc;
  const int blocks = (chunks + 1) / 2;
  const uint32_t tcols = chunks <= 1 ? 64 : chunks <= 2 ? 128 : chunks <= 4 ? 256 : 512;
  const uint64_t limit = wait_limit(p.wait_limit_us);

  if (tid == 0) {
    mbar_init(&B.q, 1);
    for (int i = 0; i < kMaxChunks; ++i) {
      mbar_init(&B.k[i], 1);
      mbar_init(&B.v[i], 1);
    }
    for (int i = 0; i < kMaxChunks / 2; ++i) mbar_init(&B.s[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.p[i], kSoftmaxThreads);
      mbar_init(&B.pv[i], 1);
    }
    mbar_init(&B.o, 1);
    B.failed = 0;
    if (SPLIT > 1) {  // the bytes the other CTAs will push
      mbar_init(&B.xm, 1);
      mbar_init(&B.xo, 1);
      mbar_expect_tx(&B.xm, (SPLIT - 1) * kTq * 4);
      mbar_expect_tx(&B.xo, (SPLIT - 1) * kTq * (W + 1) * 4);
    }
    fence_mbar_init();
    prefetch_tensormap(&qkv_map);
  }
  if (SPLIT > 1)
    cluster_sync_all();  // every CTA's barriers exist before any st.async
  else
    __syncthreads();
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      if (!p.q_pos && chunks > 0) {
        mbar_expect_tx(&B.q, kQBytes);
        tma_load_3d(sQ, &qkv_map, &B.q, h * 64, q0, b, pol);
        tma_load_3d(sQ + kQBytes / 2, &qkv_map, &B.q, h * 64, q0 + 64, b, pol);
      }
      for (int c = 0; c < chunks; ++c) {
        mbar_expect_tx(&B.k[c], kChunkBytes);
        tma_load_3d(sK + c * kChunkBytes, &qkv_map, &B.k[c], p.d + h * 64, kbeg + c * kKc, b, pol);
      }
      for (int c = 0; c < chunks; ++c) {
        mbar_expect_tx(&B.v[c], kChunkBytes);
        tma_load_3d(sV + c * kChunkBytes, &qkv_map, &B.v[c], 2 * p.d + h * 64, kbeg + c * kKc, b, pol);
      }
    }
    __syncwarp();
    tmem_alloc(&B.tmem_slot, tcols);
    tmem_relinquish();
  } else if (warp == 1) {
    // all loads first (one latency, not one per word), then the ballots
    int valid[2 * kMaxChunks];
    const int* kv = p.key_valid + (size_t)b * p.s + kbeg + lane;
#pragma unroll
    for (int w = 0; w < 2 * kMaxChunks; ++w) valid[w] = kbeg + 32 * w + lane < kend ? kv[32 * w] : 0;
#pragma unroll
    for (int w = 0; w < 2 * kMaxChunks; ++w) {
      const uint32_t bits = __ballot_sync(0xffffffffu, valid[w] != 0);
      if (lane == 0 && w < 2 * chunks) B.key_bits[w] = bits;
    }
    if (p.q_pos && chunks > 0) {  // selected query rows (head layer): gather Q, zeros past nq
      for (int it = lane; it < kTq * 8; it += 32) {
        const int r = it >> 3, j = it & 7, qi = q0 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (qi < p.nq) {
          const int pos = p.q_pos[b * p.nq + qi];
          v = *reinterpret_cast<const uint4*>(p.qkv + ((size_t)b * p.s + pos) * p.ld_qkv + h * 64 + j * 8);
        }
        *reinterpret_cast<uint4*>(sQ + sw128_offset(r, j)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.q);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch_dependents();
  const uint32_t tmem = B.tmem_slot;

  if (tid == 0) {
    // ---- MMA issue: scores for every 128 keys, then O += P V per chunk
    bool ok = chunks == 0 || mbar_wait(&B.q, 0, limit);
    const uint64_t qd = sw128_desc(smem_u32(sQ));
    for (int j = 0; ok && j < blocks; ++j) {
      ok = mbar_wait(&B.k[2 * j], 0, limit) && (2 * j + 1 >= chunks || mbar_wait(&B.k[2 * j + 1], 0, limit));
      if (!ok) break;
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(128, 2 * j + 1 < chunks ? 128 : 64);
      const uint64_t kd = sw128_desc(smem_u32(sK + 2 * j * kChunkBytes));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + j * 128, qd + 2 * kk, kd + 2 * kk, idesc, kk != 0);
      umma_commit(&B.s[j]);
    }
    for (int c = 0; ok && c < chunks; ++c) {
      ok = mbar_wait(&B.p[c & 1], (c >> 1) & 1, limit) && mbar_wait(&B.v[c], 0, limit);
      if (!ok) break;
      tc_fence_after();
      const uint64_t hd = sw128_desc(smem_u32(sQ + (c & 1) * 2 * kPBytes));
      const uint64_t ld = sw128_desc(smem_u32(sQ + ((c & 1) * 2 + 1) * kPBytes));
      const uint64_t vd = sw128_desc(smem_u32(sV + c * kChunkBytes));
      // K steps of 16: 32 bytes along P's rows, 16 rows (2048 bytes) down V
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        umma_f16(tmem, hd + 2 * kk, vd + 128 * kk, kIdescPV, (c | kk) != 0);
        umma_f16(tmem, ld + 2 * kk, vd + 128 * kk, kIdescPV, 1);
      }
      umma_commit(&B.pv[c & 1]);
    }
    if (!ok) {
      record_status(p.status, kStatusAttnTimeout);
      atomicExch(&B.failed, 1u);
    }
    umma_commit(&B.o);
  } else if (warp >= 2) {
    // ---- softmax: two threads per query row (TMEM lane = row), thread `half`
    // owning columns [32 * half, 32 * half + 32) of every 64-key chunk
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane, qi = q0 + row;
    int qp = -1;
    if (qi < p.nq) qp = p.q_pos ? p.q_pos[b * p.nq + qi] : qi;
    int lo = 0, hi = nk - 1;  // visible keys relative to kbeg
    if (qp < 0) {
      lo = 1;
      hi = 0;
    } else if (p.window >= 0) {
      lo = max(lo, qp - p.window - kbeg);
      hi = min(hi, qp + p.window - kbeg);
    }
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + 32 * half;
    // a warp whose 32 rows are all past the last query only keeps the barrier
    // protocol: its rows of P and O are never stored, so they are not computed
    const bool live = __any_sync(0xffffffffu, qp >= 0);
    bool ok = true;
    float m = -INFINITY;
    for (int j = 0; live && j < blocks; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&B.s[j], 0, limit));
      if (!ok) break;
      tc_fence_after();
      const int c0 = 2 * j, base0 = c0 * kKc + 32 * half, base1 = base0 + kKc;
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c0 * kKc, r0);
      if (c0 + 1 < chunks) tmem_ld32(taddr + (c0 + 1) * kKc, r1);
      tmem_wait_ld();
      m = masked_max(r0, visible_mask(B.key_bits[base0 >> 5], base0, lo, hi), m);
      if (c0 + 1 < chunks) m = masked_max(r1, visible_mask(B.key_bits[base1 >> 5], base1, lo, hi), m);
    }
    B.red_max[half][row] = m;
    softmax_sync();
    m = fmaxf(B.red_max[0][row], B.red_max[1][row]);
    if (SPLIT > 1) {  // the row's max over every CTA of the tile
      if (half == 0)
        for (int r = 0; r < SPLIT; ++r)
          if (r != rank)
            st_async_f32(mapa_shared(smem_u32(&B.peer_max[peer_slot(rank, r)][row]), r), m,
                         mapa_shared(smem_u32(&B.xm), r));
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&B.xm, 0, limit))) ok = false;
#pragma unroll
      for (int s = 0; s < SPLIT - 1; ++s) m = fmaxf(m, B.peer_max[s][row]);
    }
    const float ms = m == -INFINITY ? 0.f : m * kScaleLog2;
    float l = 0.f;
    for (int c = 0; ok && c < chunks; ++c) {
      const int buf = c & 1;
      if (c >= 2) {  // the P.V of chunk c - 2 has released this buffer
        ok = __all_sync(0xffffffffu, mbar_wait(&B.pv[buf], ((c - 2) >> 1) & 1, limit));
        if (!ok) break;
        tc_fence_after();
      }
      if (live) {
        const int base = c * kKc + 32 * half;
        uint32_t r[32], ph[16], pl[16];
        tmem_ld32(taddr + c * kKc, r);
        tmem_wait_ld();
        probs(r, visible_mask(B.key_bits[base >> 5], base, lo, hi), ms, l, ph, pl);
        uint8_t* tile = sQ + buf * 2 * kPBytes;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t off = sw128_offset(row, 4 * half + j);
          *reinterpret_cast<uint4*>(tile + off) = make_uint4(ph[4 * j], ph[4 * j + 1], ph[4 * j + 2], ph[4 * j + 3]);
          *reinterpret_cast<uint4*>(tile + kPBytes + off) =
              make_uint4(pl[4 * j], pl[4 * j + 1], pl[4 * j + 2], pl[4 * j + 3]);
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      mbar_arrive(&B.p[buf]);
    }
    B.red_sum[half][row] = l;
    softmax_sync();
    l = B.red_sum[0][row] + B.red_sum[1][row];
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&B.o, 0, limit));
    // this CTA's O for the thread's 32 columns (zeros without keys)
    uint32_t r[32];
    if (ok && live && chunks > 0) {
      tc_fence_after();
      tmem_ld32(taddr, r);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = 0u;
    }
    if (SPLIT > 1) {
      // push the columns other CTAs gather, and the row sum; then gather ours
#pragma unroll
      for (int t = 0; t < 32 / W; ++t) {
        const int owner = (32 * half) / W + t;
        if (owner == rank) continue;
        const uint32_t dst = mapa_shared(smem_u32(recv + ((size_t)peer_slot(rank, owner) * kTq + row) * W), owner);
        const uint32_t bar = mapa_shared(smem_u32(&B.xo), owner);
#pragma unroll
        for (int j = 0; j < W; j += 4)
          st_async_f32x4(dst + 4 * j, __uint_as_float(r[t * W + j]), __uint_as_float(r[t * W + j + 1]),
                         __uint_as_float(r[t * W + j + 2]), __uint_as_float(r[t * W + j + 3]), bar);
      }
      if (half == 0)
        for (int q = 0; q < SPLIT; ++q)
          if (q != rank)
            st_async_f32(mapa_shared(smem_u32(&B.peer_sum[peer_slot(rank, q)][row]), q), l,
                         mapa_shared(smem_u32(&B.xo), q));
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&B.xo, 0, limit))) ok = false;
      const int mine = (rank * W) / 32, cofs = (rank * W) % 32;
      if (ok && half == mine && qi < p.nq) {
        // this CTA's partial, then the others' in rank order
        float lt = l;
        for (int q = 0; q < SPLIT; ++q)
          if (q != rank) lt += B.peer_sum[peer_slot(q, rank)][row];
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.out + ((size_t)b * p.nq + qi) * p.ld_out + h * 64 + rank * W);
#pragma unroll
        for (int j8 = 0; j8 < W / 8; ++j8) {
          float o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = __uint_as_float(cofs ? r[(32 - W) + 8 * j8 + j] : r[8 * j8 + j]);
          for (int q = 0; q < SPLIT; ++q) {
            if (q == rank) continue;
            const float4* src = reinterpret_cast<const float4*>(recv + ((size_t)peer_slot(q, rank) * kTq + row) * W + 8 * j8);
            const float4 a = src[0], c = src[1];
            o[0] += a.x; o[1] += a.y; o[2] += a.z; o[3] += a.w;
            o[4] += c.x; o[5] += c.y; o[6] += c.z; o[7] += c.w;
          }
          dst[j8] = make_uint4(pack2(o[0] * inv, o[1] * inv), pack2(o[2] * inv, o[3] * inv),
                               pack2(o[4] * inv, o[5] * inv), pack2(o[6] * inv, o[7] * inv));
        }
      }
    } else if (ok && live && qi < p.nq) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.out + ((size_t)b * p.nq + qi) * p.ld_out + h * 64 + 32 * half);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t* x = r + 8 * j;
        dst[j] = make_uint4(pack2(__uint_as_float(x[0]) * inv, __uint_as_float(x[1]) * inv),
                            pack2(__uint_as_float(x[2]) * inv, __uint_as_float(x[3]) * inv),
                            pack2(__uint_as_float(x[4]) * inv, __uint_as_float(x[5]) * inv),
                            pack2(__uint_as_float(x[6]) * inv, __uint_as_float(x[7]) * inv));
      }
    }
    if (!ok) {
      record_status(p.status, kStatusAttnTimeout);
      atomicExch(&B.failed, 1u);
    }
  }

  // ---- teardown: after a failure, wait (bounded) for this CTA's copies and
  // MMAs before its shared memory and TMEM are released; a split tile's CTAs
  // leave together, after every push into their shared memory
  __syncthreads();
  if (SPLIT > 1) cluster_sync_all();
  if (tid == 0 && B.failed) {
    if (!p.q_pos && chunks > 0) mbar_wait(&B.q, 0, limit);
    for (int c = 0; c < chunks; ++c) {
      mbar_wait(&B.k[c], 0, limit);
      mbar_wait(&B.v[c], 0, limit);
    }
    mbar_wait(&B.o, 0, limit);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

// ------------------------------------------------------------------ host side

int attention_chunks(const AttnParams& p) {
  int most = 0;
  for (int q0 = 0; q0 < p.nq; q0 += kTq) {
    int kbeg, kend;
    key_span(p, q0, kbeg, kend);
    const int c = (kend - kbeg + kKc - 1) / kKc;
    most = c > most ? c : most;
  }
  return most;
}

namespace {

template <int SPLIT>
cudaError_t launch_split(const AttnParams& p, const CUtensorMap& qkv_map, int batch, int heads, int chunks,
                         cudaStream_t stream, bool pdl) {
  const int share = (chunks + SPLIT - 1) / SPLIT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(((p.nq + kTq - 1) / kTq) * SPLIT, heads, batch);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = layout(share, SPLIT).total + 1024;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (SPLIT > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = SPLIT;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, attention_tc_kernel<SPLIT>, qkv_map, p, share);
}

template <int SPLIT>
cudaError_t prepare_split() {
  cudaError_t err = cudaFuncSetAttribute(attention_tc_kernel<SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)layout(kMaxChunks, SPLIT).total + 1024);
  // all of the unified L1 / shared storage as shared memory, so that two
  // CTAs of up to four chunks each fit on one SM
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(attention_tc_kernel<SPLIT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared);
  return err;
}

}  // namespace

int attention_split(int base_ctas, int chunks, int sm_count) {
  // Fewer (tile, head, sequence) CTAs than SMs: share each tile's chunks over
  // a pair of CTAs, at least two chunks each on the widest tile.  Measured on
  // C3 (64 tiles x heads, 4 or 8 chunks): pairs 1.757 ms per forward, no
  // split 1.769, clusters of 4 for the 8-chunk global layers 1.801 (their two
  // exchanges cost more than the shorter second pass saves).
  return base_ctas < sm_count && chunks >= 4 ? 2 : 1;
}

cudaError_t launch_attention(const AttnParams& p, const CUtensorMap& qkv_map, int batch, int heads,
                             cudaStream_t stream, bool pdl) {
  if ((p.window >= 0 && p.q_pos) || p.nq < 1 || p.s < 1 || batch < 1 || heads < 1) return cudaErrorInvalidValue;
  const int chunks = attention_chunks(p);
  if (chunks < 1 || chunks > kMaxChunks) return cudaErrorInvalidValue;
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
      err = prepare_split<1>();
      if (err == cudaSuccess) err = prepare_split<2>();
      if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (err != cudaSuccess) return err;
      ready |= uint64_t(1) << dev;
    }
  }
  const long long base = (long long)((p.nq + kTq - 1) / kTq) * heads * batch;
  switch (attention_split(base > (1 << 30) ? (1 << 30) : (int)base, chunks, sms[dev])) {
    case 2:
      return launch_split<2>(p, qkv_map, batch, heads, chunks, stream, pdl);
    default:
      return launch_split<1>(p, qkv_map, batch, heads, chunks, stream, pdl);
  }
}

}  // namespace laya
