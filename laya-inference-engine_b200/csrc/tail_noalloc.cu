// Decision tail without any device allocation (laya_b200_tail_noalloc).
//
// Some callers cannot allocate device memory at all: a host process that
// embeds this library behind a fixed memory budget handed out by its own
// allocator, a plugin that runs inside another framework's capture or memory
// pool, or a sandboxed worker whose CUDA calls are restricted to launches on
// buffers it was given.  For them this entry point runs the same decision
// tail as the engine (scorer logits, masked softmax features, act_head) on
// buffers the caller passes in, and keeps the kernel's scratch (act_head's
// first-layer outputs and the per-question arrival counters) in a file-scope
// __device__ array that the module carries, so no cudaMalloc, cudaFree or
// allocating library call happens on this path.
//
// The array is kTailScratchBytes (256 KiB + 256 B) and every GPU that loads
// this library holds it until the process exits.  It bounds one call to
// kTailMaxQuestions questions and questions * act_hidden <= kTailMaxA1 floats.
// All calls on a device share it and it keeps the last call's contents: each
// call clears the arrival counters it uses before the launch, and calls whose
// kernels overlap on the GPU (different streams without ordering) race on it.
#include "laya_b200.h"
#include "common.cuh"
#include "launch.h"
#include "params.h"

#include <mutex>
#include <string>

namespace laya {
std::string& create_error_message();
}

namespace {

constexpr int kTailMaxQuestions = 64;
constexpr int kTailMaxA1 = 64 * 1024;  // floats of act_head layer-1 outputs per call
constexpr size_t kTailCountersOffset = (size_t)kTailMaxA1 * sizeof(float);
constexpr size_t kTailScratchBytes = kTailCountersOffset + 256;

static __device__ __align__(256) unsigned char g_tail_scratch[kTailScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_tail_scratch on the current device, looked up once per
// device.  The name g_tail_scratch in host code is only a host-side stand-in;
// kernels must be given this address.
void* scratch_address(int device) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[device]) {
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_tail_scratch);
    if (err != cudaSuccess) return nullptr;
    g_scratch_ptr[device] = ptr;
  }
  return g_scratch_ptr[device];
}

}  // namespace

extern "C" int laya_b200_tail_noalloc(const laya_b200_tail_args* a, void* stream) {
  std::string& msg = laya::create_error_message();
  auto reject = [&](const std::string& m) {
    msg = m;
    return 1;
  };
  if (!a) return reject("null arguments");
  if (a->questions < 1 || a->questions > kTailMaxQuestions)
    return reject("questions must be in [1, " + std::to_string(kTailMaxQuestions) + "]");
  if (a->options < 2 || a->options > 256) return reject("options must be in [2, 256]");
  if (a->hidden < 32 || a->hidden % 8 || a->hidden > 4096) return reject("hidden must be a multiple of 8 in [32, 4096]");
  if (a->act_hidden < 1 || a->act_hidden > 1024) return reject("act_hidden must be in [1, 1024]");
  if ((long long)a->questions * a->act_hidden > kTailMaxA1)
    return reject("questions * act_hidden exceeds the scratch array (" + std::to_string(kTailMaxA1) + " floats)");
  if (!a->z || !a->fc2_w || !a->fc2_b || !a->marker_mask || !a->h_sel || !a->a1_w || !a->a1_b || !a->a2_w ||
      !a->a2_b || !a->logits || !a->act)
    return reject("null buffer");
  // z and fc2_w are read 16 bytes at a time by the kernel: a pointer from a
  // caller's pool that is only 8-byte aligned would fault on the GPU, so it is
  // refused here instead.
  if ((reinterpret_cast<uintptr_t>(a->z) | reinterpret_cast<uintptr_t>(a->fc2_w)) & 15)
    return reject("z and fc2_w must be 16-byte aligned device pointers");
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return reject(std::string("cudaGetDevice: ") + cudaGetErrorString(err));
  if (device < 0 || device >= kMaxDevices) return reject("device ordinal out of range");
  unsigned char* scratch = static_cast<unsigned char*>(scratch_address(device));
  if (!scratch) return reject("cudaGetSymbolAddress failed for the tail scratch array");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int* arrivals = reinterpret_cast<unsigned int*>(scratch + kTailCountersOffset);
  err = cudaMemsetAsync(arrivals, 0, sizeof(unsigned int) * a->questions, st);
  if (err != cudaSuccess) return reject(std::string("clearing the arrival counters: ") + cudaGetErrorString(err));
  laya::TailParams t{};
  t.k = a->options;
  t.d = a->hidden;
  t.act_hidden = a->act_hidden;
  t.z = static_cast<const __nv_bfloat16*>(a->z);
  t.fc2_w = static_cast<const __nv_bfloat16*>(a->fc2_w);
  t.fc2_b = static_cast<const __nv_bfloat16*>(a->fc2_b);
  t.marker_mask = a->marker_mask;
  t.h_sel = a->h_sel;
  t.a1_w = static_cast<const __nv_bfloat16*>(a->a1_w);
  t.a1_b = static_cast<const __nv_bfloat16*>(a->a1_b);
  t.a2_w = static_cast<const __nv_bfloat16*>(a->a2_w);
  t.a2_b = static_cast<const __nv_bfloat16*>(a->a2_b);
  t.logits = a->logits;
  t.act = a->act;
  t.a1 = reinterpret_cast<float*>(scratch);
  t.arrivals = arrivals;
  err = laya::launch_tail(t, a->questions, st, false);
  if (err != cudaSuccess) return reject(std::string("tail launch: ") + cudaGetErrorString(err));
  msg.clear();
  return 0;
}
