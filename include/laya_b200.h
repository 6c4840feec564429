/* C ABI of the b200 Laya decision engine (liblaya_b200.so).
 *
 * Plain pointers and sizes only; every function returns 0 on success and a
 * nonzero status on failure, never throws across the boundary, and leaves a
 * message readable through laya_b200_last_error().  One engine owns one GPU:
 * its weights, activation arena, CUDA-graph slots, streams and pinned I/O
 * buffers.  Calls on one engine must be serialised by the caller (the Python
 * B200Engine holds a lock, as BlackwellEngine does at
 * src/laya_blackwell/engine.py:84,192).  Different engines (different GPUs)
 * may be driven from different threads concurrently.
 */
#ifndef LAYA_B200_H
#define LAYA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LAYA_B200_API __attribute__((visibility("default")))
#else
#define LAYA_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct laya_b200_engine laya_b200_engine;

/* Network shape.  Mirrors the checkpoint's encoder config and the Laya head
 * that FastDecisionModel reads (src/laya_blackwell/model.py:37-56,82-83). */
typedef struct laya_b200_config {
  int32_t layers, hidden, heads, head_dim, intermediate, vocab, max_len;
  int32_t local_window;   /* radius: local layers see |q-k| <= local_window (model.py:82-83) */
  int32_t global_every;   /* layer i is global iff i % global_every == 0 */
  float rope_theta_global, rope_theta_local, norm_eps;
  int32_t head_layers, head_heads, head_ff, num_qtypes, act_hidden;
  int32_t max_batch;      /* largest padded batch any captured shape may use */
  int32_t max_options;    /* largest padded option count */
} laya_b200_config;

enum { LAYA_B200_BF16 = 0, LAYA_B200_FP8 = 1, LAYA_B200_NVFP4 = 2 };

/* Replaces the model construction of BlackwellEngine.__init__
 * (src/laya_blackwell/engine.py:74-104): select the GPU, validate the shape,
 * allocate the weight and activation arenas. */
LAYA_B200_API int laya_b200_create(int device, const laya_b200_config* cfg, laya_b200_engine** out);

/* Upload one parameter by its table name (e.g. "enc.3.wqkv"), host bytes in
 * the storage dtype (bf16 bit patterns for Linear weights/biases, fp32 for
 * embeddings and LayerNorms), replacing FastDecisionModel's bf16 casts
 * (model.py:28-35).  Sizes are checked against the table. */
LAYA_B200_API int laya_b200_set_weight(laya_b200_engine* e, const char* name, const void* host, size_t bytes);

/* Check that every parameter was uploaded, run the offline packer for the
 * precision (LAYA_B200_FP8: per-output-row e4m3 like
 * quantization.py:62-73; LAYA_B200_NVFP4: e2m1 + e4m3/16 + fp32 tensor
 * scale) and build the weight tensor maps. */
LAYA_B200_API int laya_b200_finalize(laya_b200_engine* e, int precision);

/* Token tables (the reference fast mode's token_tables.py:13-38): compute,
 * for every vocabulary id, the embedding LayerNorm row (fp32) and its layer-0
 * QKV projection (bf16, before the rotary embedding) with the engine's own
 * kernels and precision, so that a forward starts with one gather in place of
 * the embedding norm and the layer-0 QKV projection.  Costs vocab * hidden *
 * 10 bytes of device memory (515 MB for the Laya shape), shared with lanes
 * created afterwards.  Call after finalize; slots captured before the call
 * keep their old launch sequence. */
LAYA_B200_API int laya_b200_build_token_tables(laya_b200_engine* e);

/* Serving lanes (the multi-stream lanes of the reference's serving
 * experiments, experiments/latency/serving/README.md:6-14; no counterpart in
 * its engine API): a new engine handle on the parent's GPU that shares the
 * parent's finalized weights and has its own stream, activations, I/O staging
 * and graph slots, so requests on different lanes run concurrently.  Every
 * call takes a lane like an engine; the shared weights are freed with the last
 * of the parent and its lanes.  Calls on one lane must be serialised by the
 * caller, calls on different lanes may overlap. */
LAYA_B200_API int laya_b200_create_lane(laya_b200_engine* parent, laya_b200_engine** lane);

/* Capture the forward for one padded shape into CUDA graphs (the analogue
 * of BlackwellEngine._slot, engine.py:161-187).  `unmasked` mirrors the
 * graph key's flag (engine.py:132-138); results do not depend on it. */
LAYA_B200_API int laya_b200_capture(laya_b200_engine* e, int batch, int seq, int options, int unmasked, int* slot);

/* Drop a captured slot (LRU eviction, engine.py:167-169). */
LAYA_B200_API int laya_b200_release(laya_b200_engine* e, int slot);

/* One forward on host buffers: pack into pinned memory, replay the graph
 * (H2D copy, kernels, D2H copy), synchronise, write the outputs.  Inputs are
 * the padded arrays of BlackwellEngine._fill (engine.py:140-153):
 * input_ids/attention_mask [batch][seq] int64, marker_pos [batch][options]
 * int64, marker_mask [batch][options] uint8, qtype [batch] int64.  Outputs:
 * logits [batch][options] fp32 (masked options = -1e4), act [batch][2] fp32
 * (model.py:115,122).  Replaces engine.py:205-212 and host.cpp:64-73. */
LAYA_B200_API int laya_b200_run(laya_b200_engine* e, int slot, const int64_t* input_ids, const int64_t* attention_mask,
                  const int64_t* marker_pos, const uint8_t* marker_mask, const int64_t* qtype, float* logits,
                  float* act);

/* Measurement helper: replay the kernels-only graph `iterations` times back
 * to back on the inputs already resident on the device (from the last run)
 * and write each replay's device time in milliseconds (CUDA events on the
 * engine's stream) to ms_each[iterations].  kernel_mask selects the kernel
 * families in the replayed graph: 1 projections (GEMM), 2 attention, 4 row
 * kernels (norms, gather, tail), 8 activation quantisers (FP8 / NVFP4);
 * 15 is the whole forward.
 * Partial masks compute garbage and exist only to time one family. */
LAYA_B200_API int laya_b200_replay_device(laya_b200_engine* e, int slot, int iterations, int kernel_mask,
                                          float* ms_each);

/* Test hook with no counterpart in the reference (failure detection): the
 * next laya_b200_run on this engine enqueues its forward without a graph, and
 * the first generic projection launch in it never loads its first pipeline
 * stage and limits each of its waits to wait_limit_us microseconds (1 ..
 * 1,000,000).  Nothing completes that stage's barrier, so the kernel's
 * bounded waits run out: it records a timeout in the engine's status word,
 * drains its own copies, frees its tensor memory and returns, and the run
 * fails with a "device-side wait timed out" error.  The engine stays usable;
 * later runs are unaffected. */
LAYA_B200_API int laya_b200_test_withhold_stage(laya_b200_engine* e, int wait_limit_us);

/* Number of kernels one forward of the slot launches. */
LAYA_B200_API int laya_b200_kernel_count(laya_b200_engine* e, int slot, int* count);

/* Test hook with no counterpart in the reference: copy the first `bytes` of
 * a named activation buffer ("h", "n", "qkv", "attn", "g", "hsel", "msc",
 * "zsc"; with FP8 also the e4m3 codes and per-row scales "n8", "n8s", "a8",
 * "a8s", "g8", "g8s"; with NVFP4 the last quantised operand "x4" (e2m1
 * nibbles), "x4sf" (e4m3 block scales, tiled) and "x4o" (per-row outer
 * scales)) to host memory after synchronising, so kernel-level tests can
 * compare intermediate results with a CPU oracle. */
LAYA_B200_API int laya_b200_read_buffer(laya_b200_engine* e, const char* name, void* dst, size_t bytes);

/* Arguments of laya_b200_tail_noalloc: device pointers the caller owns. */
typedef struct laya_b200_tail_args {
  int32_t questions;         /* 1..64 */
  int32_t options;           /* padded option count k, 2..256 */
  int32_t hidden;            /* d */
  int32_t act_hidden;        /* act_head width; questions * act_hidden <= 65536 */
  const void* z;             /* bf16 [questions*options][hidden]: gelu(scorer.fc1) of the option rows;
                                16-byte aligned */
  const void* fc2_w;         /* bf16 [hidden]: scorer.fc2 weight; 16-byte aligned */
  const void* fc2_b;         /* bf16 [1] */
  const int32_t* marker_mask;/* int32 [questions][options], nonzero = real option */
  const float* h_sel;        /* fp32 [questions*(1+options)][hidden]: CLS row then option rows */
  const void* a1_w;          /* bf16 [act_hidden][hidden+4]: act_head[0] */
  const void* a1_b;          /* bf16 [act_hidden] */
  const void* a2_w;          /* bf16 [2][act_hidden]: act_head[2] */
  const void* a2_b;          /* bf16 [2] */
  float* logits;             /* out fp32 [questions][options], masked options = -1e4 */
  float* act;                /* out fp32 [questions][2] */
} laya_b200_tail_args;

/* No counterpart in the reference.  The decision tail (scorer logits, masked
 * softmax features, act_head) for callers that cannot allocate device memory
 * -- a host that owns every device buffer through its own allocator or pool,
 * or a worker restricted to launching on memory it was handed.  It calls no
 * cudaMalloc, cudaFree or allocating library routine: its scratch lives in a
 * fixed 256 KiB file-scope __device__ array that every GPU loading this
 * library keeps until process exit, which limits a call to 64 questions and
 * questions * act_hidden <= 65536; larger calls are rejected.  The first call
 * on a device looks up that array's device address (once per device, with
 * the device current), so make it before any stream capture.  All calls on a
 * device share the array and it keeps the last call's contents; the call
 * clears its counters itself, and calls whose kernels overlap on the GPU
 * race.  `stream` is a cudaStream_t (NULL: the legacy default stream); the
 * launch is asynchronous.  Errors: nonzero return, message from
 * laya_b200_last_error(NULL) on the calling thread. */
LAYA_B200_API int laya_b200_tail_noalloc(const laya_b200_tail_args* args, void* stream);

/* Last error message of the engine (or of the last failed create when e is
 * NULL).  The pointer stays valid until the next call on the engine. */
LAYA_B200_API const char* laya_b200_last_error(laya_b200_engine* e);

/* Synchronise, free every device resource.  Safe on NULL. */
LAYA_B200_API int laya_b200_destroy(laya_b200_engine* e);

#ifdef __cplusplus
}
#endif
#endif
