// Host runtime behind the C ABI (include/laya_b200.h): weight arena and
// packing, activation arena, per-shape CUDA-graph slots with pinned I/O,
// serving lanes sharing the weights, token tables, and the forward's launch
// sequence (with the batch-1 fusions: attention inside Wo, LayerNorm applied
// on load by QKV / Wi).
//
// The forward mirrors FastDecisionModel.forward
// (src/laya_blackwell/model.py:72-123); the slot / fill / replay logic mirrors
// BlackwellEngine._slot / _fill / run_prepared (src/laya_blackwell/engine.py:
// 140-214) and the fast mode's in-graph copies (src/laya_blackwell/fast/
// host.py:192-199, fast/native/host.cpp:15-80).
#include "laya_b200.h"
#include "common.cuh"
#include "launch.h"
#include "params.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

using namespace laya;

namespace {
thread_local std::string g_create_error;
}  // namespace

namespace laya {
// Message of the last failed engine-less call on this thread (create, tail).
std::string& create_error_message() { return g_create_error; }
}  // namespace laya

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct Error {
  std::string msg;
};

[[noreturn]] void fail(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  throw Error{buf};
}

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail("%s: %s", what, cudaGetErrorString(e));
}

enum Dtype { kBf16 = 0, kF32 = 1 };

struct ParamInfo {
  size_t elems;
  int dtype;
  size_t offset;  // bytes into the weight arena
  int rows, cols;
  bool uploaded;
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// K-major 2D tensor map with 128-byte swizzle: rows x cols elements of
// `esize` bytes (cols*esize a multiple of 16), box = (128 bytes) x box_rows.
CUtensorMap make_map(const void* ptr, int rows, int cols, int esize, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) fail("cuTensorMapEncodeTiled is unavailable");
  CUtensorMap m;
  const CUtensorMapDataType dt = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * esize};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esize), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail("cuTensorMapEncodeTiled failed (%d) rows=%d cols=%d", (int)r, rows, cols);
  return m;
}

// [batch][seq][ld] bf16 rows (the QKV projection's output) for the attention
// kernel: box 64 columns (one head) x 64 rows x 1, 128-byte swizzle; rows past
// a sequence's end read as zeros.
CUtensorMap make_seq_map(const void* ptr, int batch, int seq, int ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) fail("cuTensorMapEncodeTiled is unavailable");
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)seq, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)seq * ld * 2};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail("cuTensorMapEncodeTiled failed (%d) for a %dx%dx%d sequence map", (int)r, batch, seq, ld);
  return m;
}

// Plain (unswizzled) 2D map for the TMA epilogue: a [rows][ld] row-major
// buffer of `esize`-byte elements, box = box_cols x box_rows.  Returns false
// when the driver rejects the geometry (the caller then uses the register
// epilogue).
bool make_plain_map(CUtensorMap* m, const void* ptr, int rows, int ld, int esize, int box_cols, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const CUtensorMapDataType dt = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * esize};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// One projection weight as the GEMM consumes it.
struct Proj {
  int N = 0, K = 0, kind = kKindBf16;
  const void* w = nullptr;           // bf16 [N][K], e4m3 [N][K] or packed e2m1 [N][K/2]
  const float* w_scale = nullptr;    // fp8 per-row scales
  const uint8_t* wsf = nullptr;      // nvfp4 scale blocks
  float w_tensor_scale = 1.f;        // nvfp4 per-tensor outer scale
  const __nv_bfloat16* bias = nullptr;
  CUtensorMap map;
};

struct Shape {
  int b, s, k, unmasked;
};

// Capacity of the split-K partial scratch (floats): larger reductions fall
// back to distributed shared memory.
constexpr size_t kPartialFloats = (size_t)16 * 1024 * 1024;

// Compact per-shape layout of the int32 input words and fp32 output words, so
// each step copies only what the shape needs.
struct IoLayout {
  size_t ids, valid, qtype, mmask, selsrc, selpos, score, words;
  size_t logits, act, out_words;
};

IoLayout io_layout(const Shape& sh) {
  IoLayout L{};
  const size_t b = sh.b, T = (size_t)sh.b * sh.s, R = (size_t)sh.b * (1 + sh.k), BK = (size_t)sh.b * sh.k;
  size_t o = 0;
  L.ids = o; o += T;
  L.valid = o; o += T;
  L.qtype = o; o += b;
  L.mmask = o; o += BK;
  L.selsrc = o; o += R;
  L.selpos = o; o += R;
  L.score = o; o += BK;
  L.words = o;
  L.logits = 0;
  L.act = BK;
  L.out_words = BK + 2 * b;
  return L;
}

// Kernel categories for partial replays (timing of one kernel family).
enum : int { kCatGemm = 1, kCatAttention = 2, kCatRows = 4, kCatQuant = 8, kCatAll = 15 };

struct Slot {
  Shape sh;
  cudaGraphExec_t io_exec = nullptr;   // H2D + kernels + D2H
  cudaGraphExec_t dev_exec[16] = {};    // kernels only, by category mask
  int kernels = 0;
  bool live = false;
};

// Weight memory shared by an engine and its lanes; freed with the last one.
struct WeightShare {
  std::mutex mu;
  int refs = 1;
  uint8_t* warena = nullptr;
  uint8_t* qarena = nullptr;
  float* table_h = nullptr;             // token tables (optional)
  __nv_bfloat16* table_qkv = nullptr;
};

}  // namespace

struct laya_b200_engine {
  int device = 0;
  laya_b200_config cfg{};
  int precision = -1;
  int sm_count = 148;
  bool finalized = false;
  std::string last_error;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;

  std::map<std::string, ParamInfo> params;
  uint8_t* warena = nullptr;
  size_t warena_bytes = 0;
  uint8_t* qarena = nullptr;  // packed low-precision encoder weights
  size_t qarena_bytes = 0;
  WeightShare* weights = nullptr;  // owner of warena / qarena (shared with lanes)
  // token tables: embedding LayerNorm rows [vocab][d] and layer-0 QKV rows
  // [vocab][3d] (before the rotary embedding), or null
  float* table_h = nullptr;
  __nv_bfloat16* table_qkv = nullptr;

  // activations
  uint8_t* aarena = nullptr;
  size_t aarena_bytes = 0;
  int max_tokens = 0, max_rows_sel = 0, max_rows_score = 0;
  float* h = nullptr;
  __nv_bfloat16 *n = nullptr, *qkv = nullptr, *attn = nullptr, *g = nullptr;
  uint8_t *n8 = nullptr, *a8 = nullptr, *g8 = nullptr;
  float *n8s = nullptr, *a8s = nullptr, *g8s = nullptr;
  float* hsel = nullptr;
  __nv_bfloat16 *asel = nullptr, *nsel = nullptr, *fsel = nullptr, *msc = nullptr, *zsc = nullptr;
  float *gcos = nullptr, *gsin = nullptr, *lcos = nullptr, *lsin = nullptr;
  uint8_t* x4 = nullptr;            // nvfp4 activation values [T][max(d,I)/2]
  uint8_t* x4sf = nullptr;          // nvfp4 activation scale blocks
  float* x4o = nullptr;             // nvfp4 per-row outer scales [T]
  int x4_col_blocks = 0;
  float* gpart = nullptr;           // split-K partials of the cluster reduction (kPartialFloats)
  float2* lnst = nullptr;           // LayerNorm tile statistics [T][hidden/128] (batch-1 path)
  float* a1 = nullptr;              // tail scratch [max_batch][act_hidden]
  unsigned int* arrivals = nullptr; // tail arrival counters [max_batch]
  // device inputs / outputs (int32 staging layout)
  int32_t* d_in = nullptr;
  float* d_out = nullptr;
  int32_t* h_in = nullptr;  // pinned
  float* h_out = nullptr;   // pinned
  size_t in_words = 0, out_words = 0;
  uint32_t* status_host = nullptr;  // mapped pinned
  uint32_t* status_dev = nullptr;

  // projections
  std::vector<Proj> wqkv, wo, wi, wo2;
  std::vector<Proj> in_proj, out_proj, lin1, lin2;
  Proj sc_fc1;

  std::vector<Slot> slots;
  int launches = 0;  // counter while enqueuing
  // Diagnostic mode (environment LAYA_B200_SYNC_CHECK=1 at create): run()
  // enqueues the forward without a graph and synchronises after every
  // launch, so a device error names the launch that raised it.
  bool sync_check = false;
  // The slot whose inputs the device staging buffer holds (set by run): a
  // kernels-only replay of another slot would read another shape's layout.
  int inputs_slot = -1;
  // Test hook (laya_b200_test_withhold_stage): wait limit in microseconds for
  // the next run's first generic projection, whose first stage is withheld;
  // 0 = not armed.
  uint32_t test_withhold_us = 0;

  std::vector<cudaEvent_t> timing_events;
};

namespace {

// -------------------------------------------------------------- param table
// Same order and shapes as laya_b200.weights.param_table.
std::vector<std::tuple<std::string, int, int, int>> param_table(const laya_b200_config& c) {
  std::vector<std::tuple<std::string, int, int, int>> t;  // name, rows, cols, dtype
  const int d = c.hidden, I = c.intermediate, V = c.vocab, F = c.head_ff, A = c.act_hidden;
  t.emplace_back("embed.tok", V, d, kF32);
  t.emplace_back("embed.norm.w", 1, d, kF32);
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "enc." + std::to_string(i) + ".";
    if (i > 0) t.emplace_back(p + "attn_norm.w", 1, d, kF32);
    t.emplace_back(p + "wqkv", 3 * d, d, kBf16);
    t.emplace_back(p + "wo", d, d, kBf16);
    t.emplace_back(p + "mlp_norm.w", 1, d, kF32);
    t.emplace_back(p + "wi", 2 * I, d, kBf16);
    t.emplace_back(p + "wo2", d, I, kBf16);
  }
  t.emplace_back("final_norm.w", 1, d, kF32);
  t.emplace_back("type_emb", c.num_qtypes, d, kF32);
  for (int j = 0; j < c.head_layers; ++j) {
    const std::string p = "head." + std::to_string(j) + ".";
    t.emplace_back(p + "norm1.w", 1, d, kF32);
    t.emplace_back(p + "norm1.b", 1, d, kF32);
    t.emplace_back(p + "in_proj.w", 3 * d, d, kBf16);
    t.emplace_back(p + "in_proj.b", 1, 3 * d, kBf16);
    t.emplace_back(p + "out_proj.w", d, d, kBf16);
    t.emplace_back(p + "out_proj.b", 1, d, kBf16);
    t.emplace_back(p + "norm2.w", 1, d, kF32);
    t.emplace_back(p + "norm2.b", 1, d, kF32);
    t.emplace_back(p + "linear1.w", F, d, kBf16);
    t.emplace_back(p + "linear1.b", 1, F, kBf16);
    t.emplace_back(p + "linear2.w", d, F, kBf16);
    t.emplace_back(p + "linear2.b", 1, d, kBf16);
  }
  t.emplace_back("scorer.norm.w", 1, d, kF32);
  t.emplace_back("scorer.norm.b", 1, d, kF32);
  t.emplace_back("scorer.fc1.w", d, d, kBf16);
  t.emplace_back("scorer.fc1.b", 1, d, kBf16);
  t.emplace_back("scorer.fc2.w", 1, d, kBf16);
  t.emplace_back("scorer.fc2.b", 1, 1, kBf16);
  t.emplace_back("act.fc1.w", A, d + 4, kBf16);
  t.emplace_back("act.fc1.b", 1, A, kBf16);
  t.emplace_back("act.fc2.w", 2, A, kBf16);
  t.emplace_back("act.fc2.b", 1, 2, kBf16);
  return t;
}

template <class T>
T* wptr(laya_b200_engine* e, const std::string& name) {
  auto it = e->params.find(name);
  if (it == e->params.end()) fail("no parameter %s", name.c_str());
  return reinterpret_cast<T*>(e->warena + it->second.offset);
}

void validate_cfg(const laya_b200_config& c) {
  if (c.head_dim != 64) fail("head_dim must be 64");
  if (c.hidden != c.heads * c.head_dim) fail("hidden must equal heads*head_dim");
  if (c.hidden % 128 || c.hidden < 128 || c.hidden > 1024) fail("hidden must be a multiple of 128 in [128, 1024]");
  if (c.intermediate % 64 || c.intermediate <= 0) fail("intermediate must be a positive multiple of 64");
  if (c.head_ff % 128 || c.head_ff <= 0) fail("head_ff must be a positive multiple of 128");
  if (c.hidden / c.head_heads != 64 || c.hidden % c.head_heads) fail("head attention needs 64-wide heads");
  if (c.layers < 1 || c.vocab < 1 || c.num_qtypes < 1 || c.head_layers < 0) fail("bad layer / vocab counts");
  if (c.max_len < 1 || c.max_len > 512) fail("max_len must be in [1, 512] (attention keeps a query's scores in TMEM)");
  if (c.global_every < 1 || c.local_window < 0) fail("bad attention pattern");
  if (c.act_hidden < 32 || c.act_hidden > 1024 || c.act_hidden % 32) fail("act_hidden must be a multiple of 32");
  if (c.max_batch < 1 || c.max_options < 2 || c.max_options > 256) fail("max_batch >= 1, 2 <= max_options <= 256");
}

// Rotary tables like transformers' default rope: inv_freq in fp32, the angle
// pos*inv_freq in fp32, cos/sin of that fp32 angle.
// Columns i and i + 32 hold the same angle (cat(freqs, freqs)); the QKV
// epilogue's rotary tiles rely on it and read only the first 32.
void rope_tables(float theta, int max_len, std::vector<float>& cs, std::vector<float>& sn) {
  cs.assign((size_t)max_len * 64, 0.f);
  sn.assign((size_t)max_len * 64, 0.f);
  float inv[32];
  for (int i = 0; i < 32; ++i) inv[i] = 1.0f / std::pow(theta, (float)(2 * i) / 64.0f);
  for (int p = 0; p < max_len; ++p)
    for (int i = 0; i < 64; ++i) {
      const float ang = (float)p * inv[i & 31];
      cs[(size_t)p * 64 + i] = (float)std::cos((double)ang);
      sn[(size_t)p * 64 + i] = (float)std::sin((double)ang);
    }
}

// ------------------------------------------------------------ the forward
struct Fwd {
  laya_b200_engine* e;
  cudaStream_t st;
  int mask = kCatAll;  // enqueue only kernels of these categories
  bool first = true;
  bool eager_check = false;  // synchronise and check after every launch
  uint32_t test_withhold_us = 0;  // test hook for the next generic projection launch

  bool on(int cat) const { return (mask & cat) != 0; }
  bool pdl() {
    const bool r = !first;
    first = false;
    return r;
  }
  void count(cudaError_t err, const char* what) {
    ck(err, what);
    ck(cudaGetLastError(), what);
    e->launches++;
    if (eager_check) {
      const cudaError_t r = cudaStreamSynchronize(st);
      if (r != cudaSuccess) fail("launch %d (%s): %s", e->launches, what, cudaGetErrorString(r));
    }
  }

  // Returns true when the epilogue applied the rotary embedding (cos / sin
  // given, plain store) to the output's q and k columns.
  bool gemm(const Proj& w, const void* x, const float* x_scale, int M, int epi, __nv_bfloat16* out, int ldo,
            float* resid, int ldr, const float* rope_cos = nullptr, const float* rope_sin = nullptr,
            int rope_seq = 0, bool ln_stats = false) {
    const int kb = (w.K + gemm_k_elems(w.kind) - 1) / gemm_k_elems(w.kind);
    int bn = 0, split = 1;
    gemm_plan(M, w.N, kb, e->sm_count, &bn, &split);
    if (!on(kCatGemm)) return rope_cos && epi == kEpiStore;
    const int esize = w.kind == kKindBf16 ? 2 : 1;
    CUtensorMap xmap = make_map(x, M, w.K, esize, bn);
    GemmParams p{};
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.kblocks = kb;
    p.epilogue = epi;
    p.out = out;
    p.ldo = ldo;
    p.resid = resid;
    p.ldr = ldr;
    p.bias = w.bias;
    p.a_scale = x_scale;
    p.w_scale = w.w_scale;
    p.status = e->status_dev;
    CUtensorMap omap;
    memset(&omap, 0, sizeof(omap));
    if (split > 1 && (size_t)(w.N / 128) * ((M + bn - 1) / bn) * split * bn * 128 <= kPartialFloats)
      p.partials = e->gpart;
    // unsplit 128-token tiles store through a TMA tile map; unsplit 64-token
    // residual tiles move their residual rows with one
    if (split == 1 && (bn >= 128 || (bn == 64 && epi == kEpiResidual && !ln_stats))) {
      p.tma_epilogue = output_map(&omap, p, bn);
      if (!p.tma_epilogue) fail("output tensor map rejected for a %dx%d projection", M, w.N);
    }
    const bool rotated = rope_cos && epi == kEpiStore;
    if (rotated) {
      p.rope_cos = rope_cos;
      p.rope_sin = rope_sin;
      p.rope_seq = rope_seq;
      p.rope_cols = 2 * (w.N / 3);
    }
    if (ln_stats) p.ln_stats = e->lnst;
    if (test_withhold_us) {  // test hook: this launch's first stage is never loaded
      p.test_withhold = 1;
      p.wait_limit_us = test_withhold_us;
      test_withhold_us = 0;
    }
    count(launch_gemm(w.kind, w.map, xmap, omap, p, bn, split, st, pdl()), "gemm launch");
    return rotated;
  }

  // Attention fused into the residual output projection (bf16, one sequence of
  // 32 < s <= 64 tokens with q and k already rotated, each CTA's K slice at
  // most four heads).  Returns false,
  // launching nothing, when the shape does not qualify.
  bool gemm_attn(const Proj& w, const AttnParams& a, int M) {
    if (w.kind != kKindBf16 || a.q_pos || a.nq != a.s || a.s != M || M <= 32 || M > 64 || w.K % 64)
      return false;
    const int kb = w.K / 64;
    int bn = 0, split = 1;
    gemm_plan(M, w.N, kb, e->sm_count, &bn, &split);
    if (bn != 64 || (kb + split - 1) / split > 4) return false;
    if (!on(kCatGemm)) return true;
    GemmParams p{};
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.kblocks = kb;
    p.epilogue = kEpiResidual;
    p.resid = e->h;
    p.ldr = e->cfg.hidden;
    p.bias = w.bias;
    p.status = e->status_dev;
    if (split > 1 && (size_t)(w.N / 128) * split * bn * 128 <= kPartialFloats) p.partials = e->gpart;
    p.ln_stats = e->lnst;
    count(launch_gemm_attn(w.map, p, a, split, st, pdl()), "fused attention launch");
    return true;
  }

  // Batch-1 LayerNorm on load: the plan of a bf16 projection of the hidden
  // rows qualifies (64-token tile, at most eight K blocks per CTA).
  bool ln_plan(const Proj& w, int M) const {
    const int d = e->cfg.hidden;
    if (w.kind != kKindBf16 || M <= 32 || M > 64 || w.K != d || d % 128 || d > 1024 || w.bias) return false;
    const int kb = w.K / 64;
    return (kb + ln_split(w.N, kb) - 1) / ln_split(w.N, kb) <= 8;
  }
  // Split-K factor of the normalise-on-load projections: the largest of
  // 8, 6, 4, 3, 2 that keeps the grid within two CTAs per SM (their operand is
  // built by the CTA's threads, so more CTAs build it in parallel: measured
  // 935 vs 1004 us per forward against one CTA per SM; a cluster of 7 packed
  // badly, 1100 us).
  int ln_split(int N, int kb) const {
    const int tiles = N / 128;
    for (int s : {8, 6, 4, 3, 2})
      if (s <= kb && tiles * s <= 2 * e->sm_count) return s;
    return 1;
  }

  // Projection of LN(h) (weight ln_w) with the statistics the previous
  // residual projection wrote; store (+ rotary) or GEGLU epilogue.
  void gemm_ln(const Proj& w, const float* ln_w, int M, int epi, __nv_bfloat16* out, int ldo,
               const float* rope_cos = nullptr, const float* rope_sin = nullptr, int rope_seq = 0) {
    if (!on(kCatGemm)) return;
    const int kb = w.K / 64, bn = 64, split = ln_split(w.N, kb);
    GemmParams p{};
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.kblocks = kb;
    p.epilogue = epi;
    p.out = out;
    p.ldo = ldo;
    p.status = e->status_dev;
    if (split > 1 && (size_t)(w.N / 128) * split * bn * 128 <= kPartialFloats) p.partials = e->gpart;
    if (rope_cos && epi == kEpiStore) {
      p.rope_cos = rope_cos;
      p.rope_sin = rope_sin;
      p.rope_seq = rope_seq;
      p.rope_cols = 2 * (w.N / 3);
    }
    LnParams ln{};
    ln.h = e->h;
    ln.ldh = e->cfg.hidden;
    ln.w = ln_w;
    ln.stats = e->lnst;
    ln.ntiles = e->cfg.hidden / 128;
    ln.eps = e->cfg.norm_eps;
    count(launch_gemm_ln(w.map, p, ln, split, st, pdl()), "layernorm gemm launch");
  }

  // NVFP4 projection: quantise the bf16 operand per row (scale blocks laid
  // out for the GEMM's token tile), then the block-scaled GEMM.
  // Token tile, split-K and K blocks of an NVFP4 projection.
  void nv4_plan(const Proj& w, int M, int* bn, int* split, int* kb) const {
    *kb = (w.K + 255) / 256;
    gemm_plan(M, w.N, *kb, e->sm_count, bn, split);
    if (*bn > 128) {
      *bn = 128;
      const int tiles = (w.N / 128) * ((M + *bn - 1) / *bn);
      *split = gemm_split(tiles, *kb, e->sm_count, 8);
    }
  }

  // NVFP4 output of a LayerNorm feeding projection w (M token rows).
  void nv4_norm_out(NormParams& p, const Proj& w, int M) const {
    int bn = 0, split = 1, kb = 0;
    nv4_plan(w, M, &bn, &split, &kb);
    p.out_x4 = e->x4;
    p.out_x4_sf = e->x4sf;
    p.out_x4_outer = e->x4o;
    p.x4_rows_per_block = bn;
    p.x4_col_blocks = 4 * kb;
  }

  // `quantized`: the LayerNorm before it already wrote the NVFP4 operand.
  bool gemm_nv4(const Proj& w, const __nv_bfloat16* x, int M, int epi, __nv_bfloat16* out, int ldo, float* resid,
                int ldr, const float* rope_cos = nullptr, const float* rope_sin = nullptr, int rope_seq = 0,
                bool quantized = false) {
    int bn = 0, split = 1, kb = 0;
    nv4_plan(w, M, &bn, &split, &kb);
    const bool wide = split == 1 && bn >= 128;
    if (on(kCatQuant) && !quantized) {
      QuantParams q{};
      q.rows = M;
      q.k = w.K;
      q.src = x;
      q.q = e->x4;
      q.scale = e->x4o;
      q.sf = e->x4sf;
      count(launch_quant_nvfp4(q, bn, 4 * kb, st, pdl()), "nvfp4 quant launch");
    }
    if (!on(kCatGemm)) return rope_cos && epi == kEpiStore;
    CUtensorMap xmap = make_map(e->x4, M, w.K / 2, 1, bn);
    GemmParams p{};
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.kblocks = kb;
    p.epilogue = epi;
    p.out = out;
    p.ldo = ldo;
    p.resid = resid;
    p.ldr = ldr;
    p.a_scale = e->x4o;
    p.w_tensor_scale = w.w_tensor_scale;
    p.status = e->status_dev;
    CUtensorMap omap;
    memset(&omap, 0, sizeof(omap));
    if (wide) {
      p.tma_epilogue = output_map(&omap, p, bn);
      if (!p.tma_epilogue) fail("output tensor map rejected for a %dx%d projection", M, w.N);
    }
    const bool rotated = rope_cos && epi == kEpiStore;
    if (rotated) {
      p.rope_cos = rope_cos;
      p.rope_sin = rope_sin;
      p.rope_seq = rope_seq;
      p.rope_cols = 2 * (w.N / 3);
    }
    count(launch_gemm_nvfp4(w.map, xmap, omap, w.wsf, e->x4sf, kb, p, bn, split, st, pdl()), "nvfp4 gemm launch");
    return rotated;
  }

  // Output tensor map of the TMA epilogue (unsplit tiles).
  static int output_map(CUtensorMap* m, const GemmParams& p, int bn) {
    if (p.epilogue == kEpiResidual) return make_plain_map(m, p.resid, p.M, p.ldr, 4, 128, bn) ? 1 : 0;
    const int cols = p.epilogue == kEpiGeglu ? 64 : 128;
    return make_plain_map(m, p.out, p.M, p.ldo, 2, cols, bn) ? 1 : 0;
  }

  void norm(NormParams p) {
    if (!on(kCatRows)) return;
    p.eps = e->cfg.norm_eps;
    p.d = e->cfg.hidden;
    count(launch_norm(p, st, pdl()), "norm launch");
  }

  void attention(AttnParams p, int batch, int heads) {
    if (!on(kCatAttention)) return;
    const int chunks = attention_chunks(p);
    if (chunks < 1 || chunks > 8) fail("attention over %d keys: at most 512 per query tile", chunks * 64);
    p.status = e->status_dev;
    const CUtensorMap map = make_seq_map(p.qkv, batch, p.s, p.ld_qkv);
    count(launch_attention(p, map, batch, heads, st, pdl()), "attention launch");
  }

  // Token-table rows [v0, v0 + n): the embedding LayerNorm of those ids and
  // their layer-0 QKV projection (no rotary embedding), with the precision's
  // own operand path, into E.h / E.qkv rows [0, n).
  void token_table_rows(const int* iota, int v0, int n) {
    laya_b200_engine& E = *e;
    const bool fp8 = E.precision == LAYA_B200_FP8, nv4 = E.precision == LAYA_B200_NVFP4;
    const int d = E.cfg.hidden;
    NormParams p{};
    p.rows = n;
    p.tok_ids = iota + v0;
    p.src = wptr<float>(e, "embed.tok");
    p.ld_src = d;
    p.w = wptr<float>(e, "embed.norm.w");
    p.out_f32 = E.h;
    p.ld_out_f32 = d;
    if (fp8) {
      p.out_fp8 = E.n8;
      p.out_fp8_scale = E.n8s;
    } else if (nv4) {
      nv4_norm_out(p, E.wqkv[0], n);
    } else {
      p.out_bf16 = E.n;
    }
    norm(p);
    if (nv4)
      gemm_nv4(E.wqkv[0], E.n, n, kEpiStore, E.qkv, 3 * d, nullptr, 0, nullptr, nullptr, 0, true);
    else
      gemm(E.wqkv[0], fp8 ? (const void*)E.n8 : (const void*)E.n, E.n8s, n, kEpiStore, E.qkv, 3 * d, nullptr, 0);
  }

  void run(const Shape& sh) {
    laya_b200_engine& E = *e;
    const laya_b200_config& c = E.cfg;
    const int b = sh.b, s = sh.s, k = sh.k, d = c.hidden, I = c.intermediate, F = c.head_ff;
    const int T = b * s, R = b * (1 + k), BK = b * k;
    const bool fp8 = E.precision == LAYA_B200_FP8;
    const bool nv4 = E.precision == LAYA_B200_NVFP4;
    const IoLayout L = io_layout(sh);
    const int32_t* in = E.d_in;
    const int* ids = in + L.ids;
    const int* valid = in + L.valid;
    const int* qtype = in + L.qtype;
    const int* mmask = in + L.mmask;
    const int* selsrc = in + L.selsrc;
    const int* selpos = in + L.selpos;
    const int* score_rows = in + L.score;

    // Token tables: one gather gives h and the rotated layer-0 qkv.
    const bool tables = E.table_h != nullptr && c.layers > 0;
    if (tables && on(kCatRows)) {
      TokenGatherParams g{};
      g.rows = T;
      g.seq = s;
      g.d = d;
      g.ids = ids;
      g.table_h = E.table_h;
      g.table_qkv = E.table_qkv;
      g.cos = E.gcos;
      g.sin = E.gsin;
      g.h = E.h;
      g.ldh = d;
      g.qkv = E.qkv;
      g.ldqkv = 3 * d;
      count(launch_token_gather(g, st, pdl()), "token gather launch");
    }
    // enc.embeddings: gather + LayerNorm; layer 0 consumes bf16(h) (model.py:84,87-88)
    if (!tables) {
      NormParams p{};
      p.rows = T;
      p.tok_ids = ids;
      p.src = wptr<float>(e, "embed.tok");
      p.ld_src = d;
      p.w = wptr<float>(e, "embed.norm.w");
      p.out_f32 = E.h;
      p.ld_out_f32 = d;
      if (fp8) {
        p.out_fp8 = E.n8;
        p.out_fp8_scale = E.n8s;
      } else if (nv4 && c.layers > 0) {
        nv4_norm_out(p, E.wqkv[0], T);
      } else {
        p.out_bf16 = E.n;
      }
      norm(p);
    }
    // LayerNorm feeding the encoder projection w: bf16, e4m3 + row scales, or
    // the NVFP4 operand laid out for w's token tile.
    auto enc_norm = [&](const std::string& wname, const Proj& w) {
      NormParams p{};
      p.rows = T;
      p.src = E.h;
      p.ld_src = d;
      p.w = wptr<float>(e, wname);
      if (fp8) {
        p.out_fp8 = E.n8;
        p.out_fp8_scale = E.n8s;
      } else if (nv4) {
        nv4_norm_out(p, w, T);
      } else {
        p.out_bf16 = E.n;
      }
      return p;
    };
    // final_norm(h + pending) + type_emb(qtype) (model.py:102-104), fused with
    // the first head layer's norm1 (model.py:59).
    NormParams final_norm{};
    final_norm.rows = T;
    final_norm.src = E.h;
    final_norm.ld_src = d;
    final_norm.w = wptr<float>(e, "final_norm.w");
    final_norm.add_table = wptr<float>(e, "type_emb");
    final_norm.add_idx = qtype;
    final_norm.add_div = s;
    final_norm.out_f32 = E.h;
    final_norm.ld_out_f32 = d;
    if (c.head_layers > 0) {
      final_norm.second_w = wptr<float>(e, "head.0.norm1.w");
      final_norm.second_b = wptr<float>(e, "head.0.norm1.b");
      final_norm.out_bf16 = E.n;
    }
    if (c.layers == 0) norm(final_norm);
    // Each residual projection (Wo, Wo2) is followed by add_norm
    // (model.py:15-19): mlp_norm after Wo, the next layer's attn_norm (or the
    // final norm) after Wo2.
    // One short sequence in bf16 (the latency path): attention runs inside the
    // Wo projection, and attn_norm / mlp_norm inside the QKV / Wi projections,
    // from row statistics written by the residual projection before them.
    const bool short_bf16 = !fp8 && !nv4 && b == 1 && c.layers > 0 && ln_plan(E.wqkv[0], T) &&
                            ln_plan(E.wi[0], T);
    for (int i = 0; i < c.layers; ++i) {
      const std::string pre = "enc." + std::to_string(i) + ".";
      const bool glob = (i % c.global_every) == 0;
      const float* rc = glob ? E.gcos : E.lcos;
      const float* rs = glob ? E.gsin : E.lsin;
      // The rotary embedding runs in the projection's epilogue (the token
      // tables hold layer 0's rotated q and k).
      bool rotated = true;
      if (tables && i == 0) {
        // layer-0 qkv came from the token tables
      } else if (short_bf16 && i > 0)
        gemm_ln(E.wqkv[i], wptr<float>(e, pre + "attn_norm.w"), T, kEpiStore, E.qkv, 3 * d, rc, rs, s);
      else
        rotated = nv4 ? gemm_nv4(E.wqkv[i], E.n, T, kEpiStore, E.qkv, 3 * d, nullptr, 0, rc, rs, s, true)
                      : gemm(E.wqkv[i], fp8 ? (const void*)E.n8 : (const void*)E.n, E.n8s, T, kEpiStore, E.qkv,
                             3 * d, nullptr, 0, rc, rs, s);
      AttnParams a{};
      a.qkv = E.qkv;
      a.ld_qkv = 3 * d;
      a.d = d;
      a.s = s;
      a.nq = s;
      a.key_valid = valid;
      if (!rotated) fail("layer %d: the QKV projection did not apply the rotary embedding", i);
      a.window = glob ? -1 : c.local_window;
      a.out = E.attn;
      a.ld_out = d;
      const bool fused = !fp8 && !nv4 && b == 1 && gemm_attn(E.wo[i], a, T);
      if (short_bf16 && !fused) fail("batch-1 plan: the attention projection did not fuse");
      if (!fused) {
        attention(a, b, c.heads);
        if (fp8 && on(kCatQuant)) {
          QuantParams q{};
          q.rows = T;
          q.k = d;
          q.src = E.attn;
          q.q = E.a8;
          q.scale = E.a8s;
          count(launch_quant_fp8(q, st, pdl()), "quant launch");
        }
        if (nv4)
          gemm_nv4(E.wo[i], E.attn, T, kEpiResidual, nullptr, 0, E.h, d);
        else
          gemm(E.wo[i], fp8 ? (const void*)E.a8 : (const void*)E.attn, E.a8s, T, kEpiResidual, nullptr, 0, E.h, d);
      }
      if (short_bf16)
        gemm_ln(E.wi[i], wptr<float>(e, pre + "mlp_norm.w"), T, kEpiGeglu, E.g, I);
      else {
        norm(enc_norm(pre + "mlp_norm.w", E.wi[i]));
        if (nv4)
          gemm_nv4(E.wi[i], E.n, T, kEpiGeglu, E.g, I, nullptr, 0, nullptr, nullptr, 0, true);
        else
          gemm(E.wi[i], fp8 ? (const void*)E.n8 : (const void*)E.n, E.n8s, T, kEpiGeglu, E.g, I, nullptr, 0);
      }
      if (fp8 && on(kCatQuant)) {
        QuantParams q{};
        q.rows = T;
        q.k = I;
        q.src = E.g;
        q.q = E.g8;
        q.scale = E.g8s;
        count(launch_quant_fp8(q, st, pdl()), "quant launch");
      }
      const bool last = i + 1 == c.layers;
      if (nv4)
        gemm_nv4(E.wo2[i], E.g, T, kEpiResidual, nullptr, 0, E.h, d);
      else
        gemm(E.wo2[i], fp8 ? (const void*)E.g8 : (const void*)E.g, E.g8s, T, kEpiResidual, nullptr, 0, E.h, d,
             nullptr, nullptr, 0, short_bf16 && !last);
      // add_norm after Wo2: the next layer's attn_norm (applied by its QKV
      // projection on the batch-1 path), or the final norm
      if (last)
        norm(final_norm);
      else if (!short_bf16)
        norm(enc_norm("enc." + std::to_string(i + 1) + ".attn_norm.w", E.wqkv[i + 1]));
    }
    // Head layers (model.py:58-70): norm1 of layer j > 0 follows the previous
    // layer's linear2, norm2 follows out_proj.
    for (int j = 0; j < c.head_layers; ++j) {
      const std::string pre = "head." + std::to_string(j) + ".";
      const bool last = j == c.head_layers - 1;
      gemm(E.in_proj[j], E.n, nullptr, T, kEpiStore, E.qkv, 3 * d, nullptr, 0);
      AttnParams a{};
      a.qkv = E.qkv;
      a.ld_qkv = 3 * d;
      a.d = d;
      a.s = s;
      a.key_valid = valid;
      a.window = -1;
      a.ld_out = d;
      float* hrows = E.h;
      int rows = T;
      __nv_bfloat16* arows = E.attn;
      __nv_bfloat16* nrows = E.n;
      __nv_bfloat16* frows = E.g;
      if (!last) {
        a.nq = s;
        a.out = E.attn;
        attention(a, b, c.head_heads);
      } else {  // only CLS and marker rows leave the last head layer (model.py:64-66)
        a.nq = 1 + k;
        a.q_pos = selpos;
        a.out = E.asel;
        attention(a, b, c.head_heads);
        if (on(kCatRows)) count(launch_gather_rows(E.hsel, E.h, selsrc, R, d, st, pdl()), "gather launch");
        hrows = E.hsel;
        rows = R;
        arows = E.asel;
        nrows = E.nsel;
        frows = E.fsel;
      }
      NormParams norm2{};
      norm2.rows = rows;
      norm2.src = hrows;
      norm2.ld_src = d;
      norm2.w = wptr<float>(e, pre + "norm2.w");
      norm2.b = wptr<float>(e, pre + "norm2.b");
      norm2.out_bf16 = nrows;
      gemm(E.out_proj[j], arows, nullptr, rows, kEpiResidual, nullptr, 0, hrows, d);
      norm(norm2);
      gemm(E.lin1[j], nrows, nullptr, rows, kEpiRelu, frows, F, nullptr, 0);
      if (last) {
        gemm(E.lin2[j], frows, nullptr, rows, kEpiResidual, nullptr, 0, hrows, d);
      } else {  // norm1 of the next layer, on the same T rows
        const std::string nxt = "head." + std::to_string(j + 1) + ".";
        NormParams norm1{};
        norm1.rows = T;
        norm1.src = E.h;
        norm1.ld_src = d;
        norm1.w = wptr<float>(e, nxt + "norm1.w");
        norm1.b = wptr<float>(e, nxt + "norm1.b");
        norm1.out_bf16 = E.n;
        gemm(E.lin2[j], frows, nullptr, rows, kEpiResidual, nullptr, 0, hrows, d);
        norm(norm1);
      }
    }
    if (c.head_layers == 0 && on(kCatRows))
      count(launch_gather_rows(E.hsel, E.h, selsrc, R, d, st, pdl()), "gather launch");
    // scorer: LN -> bf16 -> Linear -> GELU (model.py:113-114)
    {
      NormParams p{};
      p.rows = BK;
      p.src = E.hsel;
      p.ld_src = d;
      p.row_map = score_rows;
      p.w = wptr<float>(e, "scorer.norm.w");
      p.b = wptr<float>(e, "scorer.norm.b");
      p.out_bf16 = E.msc;
      norm(p);
    }
    gemm(E.sc_fc1, E.msc, nullptr, BK, kEpiGelu, E.zsc, d, nullptr, 0);
    if (on(kCatRows)) {
      TailParams t{};
      t.k = k;
      t.d = d;
      t.act_hidden = c.act_hidden;
      t.z = E.zsc;
      t.fc2_w = wptr<__nv_bfloat16>(e, "scorer.fc2.w");
      t.fc2_b = wptr<__nv_bfloat16>(e, "scorer.fc2.b");
      t.marker_mask = mmask;
      t.h_sel = E.hsel;
      t.a1_w = wptr<__nv_bfloat16>(e, "act.fc1.w");
      t.a1_b = wptr<__nv_bfloat16>(e, "act.fc1.b");
      t.a2_w = wptr<__nv_bfloat16>(e, "act.fc2.w");
      t.a2_b = wptr<__nv_bfloat16>(e, "act.fc2.b");
      t.logits = E.d_out + L.logits;
      t.act = E.d_out + L.act;
      t.a1 = E.a1;
      t.arrivals = E.arrivals;
      count(launch_tail(t, b, st, pdl()), "tail launch");
    }
  }
};

Proj make_proj(laya_b200_engine* e, const std::string& wname, const std::string& bname, int kind,
               const void* qweights, const float* qscale) {
  const ParamInfo& pi = e->params.at(wname);
  Proj p;
  p.N = pi.rows;
  p.K = pi.cols;
  p.kind = kind;
  p.bias = bname.empty() ? nullptr : wptr<__nv_bfloat16>(e, bname);
  if (kind == kKindBf16) {
    p.w = e->warena + pi.offset;
    p.map = make_map(p.w, p.N, p.K, 2, 128);
  } else if (kind == kKindFp8) {
    p.w = qweights;
    p.w_scale = qscale;
    p.map = make_map(p.w, p.N, p.K, 1, 128);
  } else {  // nvfp4: packed e2m1 [N][K/2]
    p.w = qweights;
    p.map = make_map(p.w, p.N, p.K / 2, 1, 128);
  }
  return p;
}

void free_slot(Slot& s) {
  if (s.io_exec) cudaGraphExecDestroy(s.io_exec);
  for (auto& g : s.dev_exec)
    if (g) cudaGraphExecDestroy(g);
  s = Slot{};
}

// Capture one forward (kernels of the categories in `mask`) into a graph;
// with_io adds the H2D copy of the shape's inputs and the D2H copy of its
// outputs around the kernels.
cudaGraphExec_t capture_graph(laya_b200_engine* e, const Shape& sh, int mask, bool with_io, int* kernels) {
  const IoLayout L = io_layout(sh);
  cudaGraph_t graph = nullptr;
  ck(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    if (with_io)
      ck(cudaMemcpyAsync(e->d_in, e->h_in, L.words * 4, cudaMemcpyHostToDevice, e->stream), "H2D");
    e->launches = 0;
    Fwd f{e, e->stream, mask};
    f.run(sh);
    if (kernels) *kernels = e->launches;
    if (with_io)
      ck(cudaMemcpyAsync(e->h_out, e->d_out, L.out_words * 4, cudaMemcpyDeviceToHost, e->stream), "D2H");
  } catch (...) {
    cudaStreamEndCapture(e->stream, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  ck(cudaStreamEndCapture(e->stream, &graph), "end capture");
  cudaGraphExec_t exec = nullptr;
  cudaError_t err = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  ck(err, "graph instantiate");
  return exec;
}

int guard(laya_b200_engine* e, const std::function<void()>& fn) {
  try {
    if (!e) fail("engine is NULL");
    ck(cudaSetDevice(e->device), "cudaSetDevice");
    fn();
    e->last_error.clear();
    return 0;
  } catch (const Error& err) {
    if (e) e->last_error = err.msg;
    return 1;
  } catch (const std::exception& ex) {
    if (e) e->last_error = ex.what();
    return 1;
  }
}

}  // namespace

// Stream, activation arena, RoPE tables, I/O staging and status word of one
// engine or lane (everything but the weights).
void alloc_runtime(laya_b200_engine* e) {
  ck(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream");
  ck(cudaEventCreate(&e->ev0), "event");
  ck(cudaEventCreate(&e->ev1), "event");
  // activations
  const laya_b200_config& c = e->cfg;
  const int d = c.hidden, I = c.intermediate, F = c.head_ff;
  const size_t T = (size_t)c.max_batch * c.max_len;
  const size_t R = (size_t)c.max_batch * (1 + c.max_options);
  const size_t BK = (size_t)c.max_batch * c.max_options;
  e->max_tokens = (int)T;
  e->x4_col_blocks = 4 * ((std::max(d, I) + 255) / 256);
  const size_t gw = (size_t)(I > F ? I : F);
  std::vector<std::pair<void**, size_t>> bufs = {
      {(void**)&e->h, T * d * 4},         {(void**)&e->n, T * d * 2},
      {(void**)&e->qkv, T * 3 * d * 2},   {(void**)&e->attn, T * d * 2},
      {(void**)&e->g, T * gw * 2},        {(void**)&e->n8, T * d},
      {(void**)&e->a8, T * d},            {(void**)&e->g8, T * I},
      {(void**)&e->n8s, T * 4},           {(void**)&e->a8s, T * 4},
      {(void**)&e->g8s, T * 4},           {(void**)&e->hsel, R * d * 4},
      {(void**)&e->asel, R * d * 2},      {(void**)&e->nsel, R * d * 2},
      {(void**)&e->fsel, R * F * 2},      {(void**)&e->msc, BK * d * 2},
      {(void**)&e->zsc, BK * d * 2},      {(void**)&e->gcos, (size_t)c.max_len * 64 * 4},
      {(void**)&e->gsin, (size_t)c.max_len * 64 * 4}, {(void**)&e->lcos, (size_t)c.max_len * 64 * 4},
      {(void**)&e->lsin, (size_t)c.max_len * 64 * 4},
      {(void**)&e->a1, (size_t)c.max_batch * c.act_hidden * 4},
      {(void**)&e->gpart, kPartialFloats * 4},
      {(void**)&e->lnst, T * (size_t)(d / 128) * 8},
      {(void**)&e->x4, T * (size_t)(d > I ? d : I) / 2},
      {(void**)&e->x4sf, ((T + 15) / 16) * (size_t)(4 * ((std::max(d, I) + 255) / 256)) * 512},
      {(void**)&e->x4o, T * 4},
      {(void**)&e->arrivals, (size_t)c.max_batch * 4},
  };
  size_t aoff = 0;
  for (auto& b : bufs) aoff = align_up(aoff + b.second, 1024);
  e->aarena_bytes = aoff;
  ck(cudaMalloc(&e->aarena, aoff), "activation arena");
  ck(cudaMemset(e->aarena, 0, aoff), "activation memset");
  aoff = 0;
  for (auto& b : bufs) {
    *b.first = e->aarena + aoff;
    aoff = align_up(aoff + b.second, 1024);
  }
  std::vector<float> cs, sn;
  rope_tables(c.rope_theta_global, c.max_len, cs, sn);
  ck(cudaMemcpy(e->gcos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope upload");
  ck(cudaMemcpy(e->gsin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope upload");
  rope_tables(c.rope_theta_local, c.max_len, cs, sn);
  ck(cudaMemcpy(e->lcos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope upload");
  ck(cudaMemcpy(e->lsin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope upload");
  // I/O staging capacity: the layout of the largest shape
  const IoLayout cap = io_layout(Shape{c.max_batch, c.max_len, c.max_options, 0});
  e->in_words = cap.words;
  e->out_words = cap.out_words;
  ck(cudaMalloc(&e->d_in, e->in_words * 4), "input buffer");
  ck(cudaMemset(e->d_in, 0, e->in_words * 4), "input memset");
  ck(cudaMalloc(&e->d_out, e->out_words * 4), "output buffer");
  ck(cudaHostAlloc(&e->h_in, e->in_words * 4, cudaHostAllocDefault), "pinned input");
  ck(cudaHostAlloc(&e->h_out, e->out_words * 4, cudaHostAllocDefault), "pinned output");
  ck(cudaHostAlloc(&e->status_host, 64, cudaHostAllocMapped), "status word");
  memset(e->status_host, 0, 64);
  ck(cudaHostGetDevicePointer((void**)&e->status_dev, e->status_host, 0), "status pointer");
}

extern "C" {

int laya_b200_create(int device, const laya_b200_config* cfg, laya_b200_engine** out) {
  if (!out || !cfg) {
    g_create_error = "null argument";
    return 1;
  }
  *out = nullptr;
  std::unique_ptr<laya_b200_engine> e(new laya_b200_engine());
  try {
    validate_cfg(*cfg);
    int n = 0;
    ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    if (device < 0 || device >= n) fail("device %d out of range (%d visible)", device, n);
    e->device = device;
    e->cfg = *cfg;
    ck(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    ck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10) fail("the b200 engine needs an sm_100 GPU; found %s (SM%d%d)", prop.name, prop.major, prop.minor);
    e->sm_count = prop.multiProcessorCount;
    {
      const char* v = getenv("LAYA_B200_SYNC_CHECK");
      e->sync_check = v && v[0] == '1';
    }
    // weights
    size_t off = 0;
    for (auto& t : param_table(*cfg)) {
      ParamInfo pi{};
      pi.rows = std::get<1>(t);
      pi.cols = std::get<2>(t);
      pi.dtype = std::get<3>(t);
      pi.elems = (size_t)pi.rows * pi.cols;
      pi.offset = off;
      off = align_up(off + pi.elems * (pi.dtype == kF32 ? 4 : 2), 256);
      e->params[std::get<0>(t)] = pi;
    }
    e->warena_bytes = off;
    e->weights = new WeightShare();
    ck(cudaMalloc(&e->weights->warena, off), "weight arena");
    e->warena = e->weights->warena;
    alloc_runtime(e.get());
    if (!get_encode_fn()) fail("cuTensorMapEncodeTiled is unavailable");
  } catch (const Error& err) {
    g_create_error = err.msg;
    laya_b200_destroy(e.release());
    return 1;
  }
  *out = e.release();
  return 0;
}

int laya_b200_create_lane(laya_b200_engine* parent, laya_b200_engine** out) {
  if (!out || !parent) {
    g_create_error = "null argument";
    return 1;
  }
  *out = nullptr;
  if (!parent->finalized) {
    g_create_error = "finalize the weights before creating a lane";
    return 1;
  }
  std::unique_ptr<laya_b200_engine> e(new laya_b200_engine());
  try {
    ck(cudaSetDevice(parent->device), "cudaSetDevice");
    e->device = parent->device;
    e->cfg = parent->cfg;
    e->sm_count = parent->sm_count;
    e->sync_check = parent->sync_check;
    e->precision = parent->precision;
    e->params = parent->params;
    {
      std::lock_guard<std::mutex> lock(parent->weights->mu);
      parent->weights->refs++;
    }
    e->weights = parent->weights;
    e->warena = parent->warena;
    e->warena_bytes = parent->warena_bytes;
    e->qarena = parent->qarena;
    e->qarena_bytes = parent->qarena_bytes;
    e->wqkv = parent->wqkv;
    e->wo = parent->wo;
    e->wi = parent->wi;
    e->wo2 = parent->wo2;
    e->in_proj = parent->in_proj;
    e->out_proj = parent->out_proj;
    e->lin1 = parent->lin1;
    e->lin2 = parent->lin2;
    e->sc_fc1 = parent->sc_fc1;
    e->table_h = parent->table_h;
    e->table_qkv = parent->table_qkv;
    e->finalized = true;
    alloc_runtime(e.get());
  } catch (const Error& err) {
    g_create_error = err.msg;
    laya_b200_destroy(e.release());
    return 1;
  }
  *out = e.release();
  return 0;
}

int laya_b200_build_token_tables(laya_b200_engine* e) {
  return guard(e, [&] {
    if (!e->finalized) fail("finalize the weights before building token tables");
    if (e->table_h) return;
    const laya_b200_config& c = e->cfg;
    if (c.layers < 1) fail("token tables need an encoder layer");
    const size_t V = (size_t)c.vocab, d = (size_t)c.hidden;
    WeightShare* w = e->weights;
    ck(cudaMalloc(&w->table_h, V * d * 4), "token table (norm rows)");
    ck(cudaMalloc(&w->table_qkv, V * 3 * d * 2), "token table (qkv rows)");
    std::vector<int> iota(V);
    for (size_t v = 0; v < V; ++v) iota[v] = (int)v;
    int* d_iota = nullptr;
    ck(cudaMalloc(&d_iota, V * 4), "token table ids");
    try {
      ck(cudaMemcpy(d_iota, iota.data(), V * 4, cudaMemcpyHostToDevice), "token table ids");
      const int chunk = e->max_tokens;
      for (size_t v0 = 0; v0 < V; v0 += chunk) {
        const int n = (int)std::min((size_t)chunk, V - v0);
        Fwd f{e, e->stream, kCatAll};
        f.token_table_rows(d_iota, (int)v0, n);
        ck(cudaMemcpyAsync(w->table_h + v0 * d, e->h, (size_t)n * d * 4, cudaMemcpyDeviceToDevice, e->stream),
           "token table copy");
        ck(cudaMemcpyAsync(w->table_qkv + v0 * 3 * d, e->qkv, (size_t)n * 3 * d * 2, cudaMemcpyDeviceToDevice,
                           e->stream),
           "token table copy");
      }
      ck(cudaStreamSynchronize(e->stream), "token tables");
    } catch (...) {
      cudaFree(d_iota);
      throw;
    }
    cudaFree(d_iota);
    if (e->status_host[0]) {
      e->status_host[0] = 0;
      fail("a device-side wait timed out while building the token tables");
    }
    e->table_h = w->table_h;
    e->table_qkv = w->table_qkv;
    e->inputs_slot = -1;  // the staging buffers were used for the tables
  });
}

int laya_b200_set_weight(laya_b200_engine* e, const char* name, const void* host, size_t bytes) {
  return guard(e, [&] {
    if (!name || !host) fail("null argument");
    if (e->finalized) fail("weights are already finalized");
    auto it = e->params.find(name);
    if (it == e->params.end()) fail("unknown parameter %s", name);
    ParamInfo& pi = it->second;
    const size_t want = pi.elems * (pi.dtype == kF32 ? 4 : 2);
    if (bytes != want) fail("parameter %s: expected %zu bytes, got %zu", name, want, bytes);
    uint8_t* dst = e->warena + pi.offset;
    const std::string n(name);
    const bool is_wi = n.size() > 3 && n.compare(n.size() - 3, 3, ".wi") == 0 && n.rfind("enc.", 0) == 0;
    if (is_wi) {
      // Interleave act/gate rows in blocks of 64 so that each 128-row GEMM
      // tile holds act rows j and their gate rows j+64 (GEGLU epilogue).
      const int I = e->cfg.intermediate, K = pi.cols;
      const size_t rowb = (size_t)K * 2;
      const uint8_t* src = static_cast<const uint8_t*>(host);
      for (int t = 0; t < I / 64; ++t) {
        ck(cudaMemcpy(dst + (size_t)(128 * t) * rowb, src + (size_t)(64 * t) * rowb, 64 * rowb,
                      cudaMemcpyHostToDevice),
           "weight upload");
        ck(cudaMemcpy(dst + (size_t)(128 * t + 64) * rowb, src + (size_t)(I + 64 * t) * rowb, 64 * rowb,
                      cudaMemcpyHostToDevice),
           "weight upload");
      }
    } else {
      ck(cudaMemcpy(dst, host, bytes, cudaMemcpyHostToDevice), "weight upload");
    }
    pi.uploaded = true;
  });
}

int laya_b200_finalize(laya_b200_engine* e, int precision) {
  return guard(e, [&] {
    if (e->finalized) fail("already finalized");
    for (auto& kv : e->params)
      if (!kv.second.uploaded) fail("parameter %s was not uploaded", kv.first.c_str());
    if (precision != LAYA_B200_BF16 && precision != LAYA_B200_FP8 && precision != LAYA_B200_NVFP4)
      fail("unknown precision %d", precision);
    const laya_b200_config& c = e->cfg;
    const int kind = precision == LAYA_B200_FP8 ? kKindFp8 : precision == LAYA_B200_NVFP4 ? kKindNvfp4 : kKindBf16;
    if (kind == kKindNvfp4 && (c.hidden % 16 || c.intermediate % 16)) fail("NVFP4 needs K divisible by 16");
    if (kind != kKindBf16 && c.intermediate > 4096)
      fail("FP8 and NVFP4 need intermediate <= 4096 (row quantiser width)");
    std::vector<std::pair<std::string, size_t>> qoff;  // weight name -> offset of e4m3 bytes, scales follow
    if (kind == kKindFp8) {
      size_t off = 0;
      for (int i = 0; i < c.layers; ++i)
        for (const char* nm : {"wqkv", "wo", "wi", "wo2"}) {
          const std::string name = "enc." + std::to_string(i) + "." + nm;
          const ParamInfo& pi = e->params.at(name);
          qoff.emplace_back(name, off);
          off = align_up(off + pi.elems, 256);
          off = align_up(off + (size_t)pi.rows * 4, 256);
        }
      e->qarena_bytes = off;
      ck(cudaMalloc(&e->qarena, off), "packed weight arena");
      e->weights->qarena = e->qarena;
      for (auto& q : qoff) {
        const ParamInfo& pi = e->params.at(q.first);
        uint8_t* wq = e->qarena + q.second;
        float* ws = reinterpret_cast<float*>(e->qarena + align_up(q.second + pi.elems, 256));
        ck(launch_pack_fp8_rows(reinterpret_cast<const __nv_bfloat16*>(e->warena + pi.offset), wq, ws, pi.rows,
                                pi.cols, e->stream),
           "fp8 packer");
      }
      ck(cudaStreamSynchronize(e->stream), "fp8 packer");
    }
    // NVFP4: per weight [e2m1 N*K/2 | scale blocks (N/128) x 4*ceil(K/256) x 512 | tensor scale]
    struct Nv4 {
      std::string name;
      size_t q, sf, ts;
      int col_blocks;
    };
    std::vector<Nv4> nv4;
    if (kind == kKindNvfp4) {
      size_t off = 0;
      for (int i = 0; i < c.layers; ++i)
        for (const char* nm : {"wqkv", "wo", "wi", "wo2"}) {
          const std::string name = "enc." + std::to_string(i) + "." + nm;
          const ParamInfo& pi = e->params.at(name);
          Nv4 w{name, off, 0, 0, 4 * ((pi.cols + 255) / 256)};
          off = align_up(off + pi.elems / 2, 256);
          w.sf = off;
          off = align_up(off + (size_t)(pi.rows / 128) * w.col_blocks * 512, 256);
          w.ts = off;
          off = align_up(off + 4, 256);
          nv4.push_back(w);
        }
      const size_t scratch = off;
      off = align_up(off + 4, 256);
      e->qarena_bytes = off;
      ck(cudaMalloc(&e->qarena, off), "packed weight arena");
      e->weights->qarena = e->qarena;
      ck(cudaMemset(e->qarena, 0, off), "packed weight arena");  // zero scale padding
      for (auto& w : nv4) {
        const ParamInfo& pi = e->params.at(w.name);
        ck(launch_nvfp4_pack_weight(reinterpret_cast<const __nv_bfloat16*>(e->warena + pi.offset), pi.rows, pi.cols,
                                    reinterpret_cast<unsigned int*>(e->qarena + scratch), e->qarena + w.q,
                                    e->qarena + w.sf, w.col_blocks, reinterpret_cast<float*>(e->qarena + w.ts),
                                    e->stream),
           "nvfp4 packer");
      }
      ck(cudaStreamSynchronize(e->stream), "nvfp4 packer");
    }
    auto enc_proj = [&](const std::string& name) {
      if (kind == kKindBf16) return make_proj(e, name, "", kKindBf16, nullptr, nullptr);
      if (kind == kKindNvfp4) {
        for (auto& w : nv4)
          if (w.name == name) {
            Proj p = make_proj(e, name, "", kKindNvfp4, e->qarena + w.q, nullptr);
            p.wsf = e->qarena + w.sf;
            ck(cudaMemcpy(&p.w_tensor_scale, e->qarena + w.ts, 4, cudaMemcpyDeviceToHost), "tensor scale");
            return p;
          }
        fail("no packed weights for %s", name.c_str());
      }
      for (auto& q : qoff)
        if (q.first == name) {
          const ParamInfo& pi = e->params.at(name);
          return make_proj(e, name, "", kKindFp8, e->qarena + q.second,
                           reinterpret_cast<const float*>(e->qarena + align_up(q.second + pi.elems, 256)));
        }
      fail("no packed weights for %s", name.c_str());
    };
    for (int i = 0; i < c.layers; ++i) {
      const std::string p = "enc." + std::to_string(i) + ".";
      e->wqkv.push_back(enc_proj(p + "wqkv"));
      e->wo.push_back(enc_proj(p + "wo"));
      e->wi.push_back(enc_proj(p + "wi"));
      e->wo2.push_back(enc_proj(p + "wo2"));
    }
    for (int j = 0; j < c.head_layers; ++j) {
      const std::string p = "head." + std::to_string(j) + ".";
      e->in_proj.push_back(make_proj(e, p + "in_proj.w", p + "in_proj.b", kKindBf16, nullptr, nullptr));
      e->out_proj.push_back(make_proj(e, p + "out_proj.w", p + "out_proj.b", kKindBf16, nullptr, nullptr));
      e->lin1.push_back(make_proj(e, p + "linear1.w", p + "linear1.b", kKindBf16, nullptr, nullptr));
      e->lin2.push_back(make_proj(e, p + "linear2.w", p + "linear2.b", kKindBf16, nullptr, nullptr));
    }
    e->sc_fc1 = make_proj(e, "scorer.fc1.w", "scorer.fc1.b", kKindBf16, nullptr, nullptr);
    e->precision = precision;
    e->finalized = true;
  });
}

int laya_b200_capture(laya_b200_engine* e, int batch, int seq, int options, int unmasked, int* slot) {
  return guard(e, [&] {
    if (!e->finalized) fail("finalize the weights before capturing");
    if (!slot) fail("null slot pointer");
    const laya_b200_config& c = e->cfg;
    if (batch < 1 || batch > c.max_batch) fail("batch %d outside [1, %d]", batch, c.max_batch);
    if (seq < 1 || seq > c.max_len) fail("seq %d outside [1, %d]", seq, c.max_len);
    if (options < 2 || options > c.max_options) fail("options %d outside [2, %d]", options, c.max_options);
    Slot s;
    s.sh = Shape{batch, seq, options, unmasked ? 1 : 0};
    try {
      s.io_exec = capture_graph(e, s.sh, kCatAll, true, &s.kernels);
      s.dev_exec[kCatAll] = capture_graph(e, s.sh, kCatAll, false, nullptr);
    } catch (...) {
      free_slot(s);
      throw;
    }
    s.live = true;
    for (size_t i = 0; i < e->slots.size(); ++i)
      if (!e->slots[i].live) {
        e->slots[i] = s;
        *slot = (int)i;
        if (e->inputs_slot == (int)i) e->inputs_slot = -1;
        return;
      }
    e->slots.push_back(s);
    *slot = (int)e->slots.size() - 1;
  });
}

int laya_b200_release(laya_b200_engine* e, int slot) {
  return guard(e, [&] {
    if (slot < 0 || slot >= (int)e->slots.size() || !e->slots[slot].live) fail("no slot %d", slot);
    ck(cudaStreamSynchronize(e->stream), "sync");
    free_slot(e->slots[slot]);
    if (e->inputs_slot == slot) e->inputs_slot = -1;
  });
}

int laya_b200_run(laya_b200_engine* e, int slot, const int64_t* input_ids, const int64_t* attention_mask,
                  const int64_t* marker_pos, const uint8_t* marker_mask, const int64_t* qtype, float* logits,
                  float* act) {
  return guard(e, [&] {
    if (slot < 0 || slot >= (int)e->slots.size() || !e->slots[slot].live) fail("no slot %d", slot);
    if (!input_ids || !attention_mask || !marker_pos || !marker_mask || !qtype || !logits || !act)
      fail("null buffer");
    const Slot& sl = e->slots[slot];
    const int b = sl.sh.b, s = sl.sh.s, k = sl.sh.k;
    const laya_b200_config& c = e->cfg;
    const IoLayout L = io_layout(sl.sh);
    int32_t* w = e->h_in;
    // Pack and validate on the host; nothing out of range reaches a kernel.
    for (int i = 0; i < b * s; ++i) {
      const int64_t id = input_ids[i];
      if (id < 0 || id >= c.vocab) fail("input_ids[%d]=%lld outside [0, %d)", i, (long long)id, c.vocab);
      w[L.ids + i] = (int32_t)id;
      w[L.valid + i] = attention_mask[i] != 0;
    }
    for (int q = 0; q < b; ++q) {
      if (qtype[q] < 0 || qtype[q] >= c.num_qtypes) fail("qtype[%d]=%lld out of range", q, (long long)qtype[q]);
      w[L.qtype + q] = (int32_t)qtype[q];
      w[L.selsrc + q * (1 + k)] = q * s;
      w[L.selpos + q * (1 + k)] = 0;
      for (int j = 0; j < k; ++j) {
        const int64_t pos = marker_pos[q * k + j];
        if (pos < 0 || pos >= s) fail("marker_pos[%d][%d]=%lld outside [0, %d)", q, j, (long long)pos, s);
        w[L.mmask + q * k + j] = marker_mask[q * k + j] != 0;
        w[L.selsrc + q * (1 + k) + 1 + j] = q * s + (int32_t)pos;
        w[L.selpos + q * (1 + k) + 1 + j] = (int32_t)pos;
        w[L.score + q * k + j] = q * (1 + k) + 1 + j;
      }
    }
    // The copy below overwrites the staging buffer with this slot's layout:
    // until it has completed, no slot's inputs are known to be resident.
    e->inputs_slot = -1;
    const uint32_t withhold_us = e->test_withhold_us;
    e->test_withhold_us = 0;
    if (e->sync_check || withhold_us) {
      ck(cudaMemcpyAsync(e->d_in, e->h_in, L.words * 4, cudaMemcpyHostToDevice, e->stream), "H2D");
      e->launches = 0;
      Fwd f{e, e->stream, kCatAll};
      f.eager_check = e->sync_check;
      f.test_withhold_us = withhold_us;
      f.run(sl.sh);
      if (withhold_us && f.test_withhold_us) fail("test hook: the forward has no generic projection launch");
      ck(cudaMemcpyAsync(e->h_out, e->d_out, L.out_words * 4, cudaMemcpyDeviceToHost, e->stream), "D2H");
    } else {
      ck(cudaGraphLaunch(sl.io_exec, e->stream), "graph launch");
    }
    ck(cudaStreamSynchronize(e->stream), "forward");
    e->inputs_slot = slot;
    const uint32_t st = __atomic_load_n(e->status_host, __ATOMIC_ACQUIRE);
    if (st) {
      e->status_host[0] = 0;
      fail("a device-side wait timed out (status %u); the results of this call are invalid", st);
    }
    memcpy(logits, e->h_out + L.logits, sizeof(float) * b * k);
    memcpy(act, e->h_out + L.act, sizeof(float) * b * 2);
  });
}

int laya_b200_replay_device(laya_b200_engine* e, int slot, int iterations, int kernel_mask, float* ms_each) {
  return guard(e, [&] {
    if (slot < 0 || slot >= (int)e->slots.size() || !e->slots[slot].live) fail("no slot %d", slot);
    if (iterations < 1 || !ms_each || kernel_mask < 1 || kernel_mask > kCatAll) fail("bad arguments");
    if (e->inputs_slot != slot)
      fail("slot %d: the device inputs belong to another slot; run this slot once before replaying it", slot);
    Slot& sl = e->slots[slot];
    if (!sl.dev_exec[kernel_mask]) sl.dev_exec[kernel_mask] = capture_graph(e, sl.sh, kernel_mask, false, nullptr);
    while ((int)e->timing_events.size() < iterations + 1) {
      cudaEvent_t ev;
      ck(cudaEventCreate(&ev), "event");
      e->timing_events.push_back(ev);
    }
    ck(cudaEventRecord(e->timing_events[0], e->stream), "event");
    for (int i = 0; i < iterations; ++i) {
      ck(cudaGraphLaunch(sl.dev_exec[kernel_mask], e->stream), "graph launch");
      ck(cudaEventRecord(e->timing_events[i + 1], e->stream), "event");
    }
    ck(cudaEventSynchronize(e->timing_events[iterations]), "replay");
    for (int i = 0; i < iterations; ++i)
      ck(cudaEventElapsedTime(&ms_each[i], e->timing_events[i], e->timing_events[i + 1]), "elapsed");
    if (e->status_host[0]) {
      e->status_host[0] = 0;
      fail("a device-side wait timed out during replay");
    }
  });
}

int laya_b200_test_withhold_stage(laya_b200_engine* e, int wait_limit_us) {
  return guard(e, [&] {
    if (wait_limit_us < 1 || wait_limit_us > 1000000) fail("wait_limit_us must be in [1, 1000000]");
    e->test_withhold_us = (uint32_t)wait_limit_us;
  });
}

int laya_b200_kernel_count(laya_b200_engine* e, int slot, int* count) {
  return guard(e, [&] {
    if (slot < 0 || slot >= (int)e->slots.size() || !e->slots[slot].live || !count) fail("no slot %d", slot);
    *count = e->slots[slot].kernels;
  });
}

int laya_b200_read_buffer(laya_b200_engine* e, const char* name, void* dst, size_t bytes) {
  return guard(e, [&] {
    if (!name || !dst) fail("null argument");
    const laya_b200_config& c = e->cfg;
    const size_t T = (size_t)c.max_batch * c.max_len, d = c.hidden;
    const size_t R = (size_t)c.max_batch * (1 + c.max_options), BK = (size_t)c.max_batch * c.max_options;
    const std::string n(name);
    const void* src = nullptr;
    size_t cap = 0;
    if (n == "h") { src = e->h; cap = T * d * 4; }
    else if (n == "n") { src = e->n; cap = T * d * 2; }
    else if (n == "qkv") { src = e->qkv; cap = T * 3 * d * 2; }
    else if (n == "attn") { src = e->attn; cap = T * d * 2; }
    else if (n == "g") { src = e->g; cap = T * (size_t)(c.intermediate > c.head_ff ? c.intermediate : c.head_ff) * 2; }
    else if (n == "hsel") { src = e->hsel; cap = R * d * 4; }
    else if (n == "asel") { src = e->asel; cap = R * d * 2; }
    else if (n == "msc") { src = e->msc; cap = BK * d * 2; }
    else if (n == "zsc") { src = e->zsc; cap = BK * d * 2; }
    else if (n == "n8" && e->n8) { src = e->n8; cap = T * d; }
    else if (n == "n8s" && e->n8s) { src = e->n8s; cap = T * 4; }
    else if (n == "a8" && e->a8) { src = e->a8; cap = T * d; }
    else if (n == "a8s" && e->a8s) { src = e->a8s; cap = T * 4; }
    else if (n == "g8" && e->g8) { src = e->g8; cap = T * (size_t)c.intermediate; }
    else if (n == "g8s" && e->g8s) { src = e->g8s; cap = T * 4; }
    else if (n == "x4" && e->x4) { src = e->x4; cap = T * (size_t)std::max(d, (size_t)c.intermediate) / 2; }
    else if (n == "x4sf" && e->x4sf) {
      src = e->x4sf;
      cap = ((T + 15) / 16) * (size_t)(4 * ((std::max(d, (size_t)c.intermediate) + 255) / 256)) * 512;
    }
    else if (n == "x4o" && e->x4o) { src = e->x4o; cap = T * 4; }
    else fail("unknown buffer %s", name);
    if (bytes > cap) fail("buffer %s holds %zu bytes, %zu requested", name, cap, bytes);
    ck(cudaStreamSynchronize(e->stream), "sync");
    ck(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost), "read buffer");
  });
}

const char* laya_b200_last_error(laya_b200_engine* e) {
  return e ? e->last_error.c_str() : g_create_error.c_str();
}

int laya_b200_destroy(laya_b200_engine* e) {
  if (!e) return 0;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& s : e->slots) free_slot(s);
  if (e->weights) {
    int left;
    {
      std::lock_guard<std::mutex> lock(e->weights->mu);
      left = --e->weights->refs;
    }
    if (left == 0) {
      cudaFree(e->weights->warena);
      cudaFree(e->weights->qarena);
      cudaFree(e->weights->table_h);
      cudaFree(e->weights->table_qkv);
      delete e->weights;
    }
  }
  cudaFree(e->aarena);
  cudaFree(e->d_in);
  cudaFree(e->d_out);
  if (e->h_in) cudaFreeHost(e->h_in);
  if (e->h_out) cudaFreeHost(e->h_out);
  if (e->status_host) cudaFreeHost(e->status_host);
  for (auto ev : e->timing_events) cudaEventDestroy(ev);
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
  return 0;
}

}  // extern "C"
