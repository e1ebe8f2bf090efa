// Split-KV decode attention whose split partials live in a fixed, library-owned device array, for
// callers that cannot allocate device memory themselves.
//
// Who needs it: a host that hands a plugin only its input and output buffers and owns every other
// allocation (an inference-server backend with its own memory pool, say), and latency-critical
// loops that must not call cudaMalloc / cudaFree, which can synchronise the whole device. Such a
// caller cannot provide the `workspace` that ipe_decode_attention asks for.
//
// The scratch below is a file-scope __device__ array: every GPU that loads the library holds
// kStaticScratchBytes of it until the process exits. In host code its name is only a host-side
// stand-in for the symbol, never a device address, so the host asks the runtime for the real
// address (cudaGetSymbolAddress) once per device, with that device current, and passes that
// pointer to the kernels.
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace ipe {
size_t decode_attention_workspace_bytes(int batch, int q_heads, int capacity);
int report_failure(int status, const char* message);
}  // namespace ipe

namespace {

constexpr size_t kStaticScratchBytes = size_t(2) << 20;  // 2 MiB per GPU
static __device__ __align__(256) float g_split_kv_scratch[kStaticScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;

// Address of the scratch on the current device; looked up on the first call per device.
float* scratch_on_current_device(int* status) {
  static std::mutex mu;
  static float* addresses[kMaxDevices] = {};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    *status = ipe::report_failure(IPE_ERR_CUDA, "ipe_decode_attention_static_scratch: cudaGetDevice failed");
    return nullptr;
  }
  if (device < 0 || device >= kMaxDevices) {
    *status = ipe::report_failure(IPE_ERR_UNSUPPORTED, "ipe_decode_attention_static_scratch: device ordinal >= 64");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addresses[device]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_split_kv_scratch);
    if (e != cudaSuccess || !p) {
      *status = ipe::report_failure(IPE_ERR_CUDA,
                                    "ipe_decode_attention_static_scratch: cudaGetSymbolAddress of the scratch failed");
      return nullptr;
    }
    addresses[device] = static_cast<float*>(p);
  }
  return addresses[device];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int ipe_decode_attention_static_scratch(const void* q, const void* k_cache, const void* v_cache, void* out,
                                                   int batch, int q_heads, int kv_heads, int capacity, int length,
                                                   const int64_t* state, void* stream) {
  if (!q || !k_cache || !v_cache || !out)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_decode_attention_static_scratch: null pointer");
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || capacity < 1 || q_heads % kv_heads)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_decode_attention_static_scratch: bad sizes");
  const int group = q_heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return ipe::report_failure(IPE_ERR_UNSUPPORTED,
                               "ipe_decode_attention_static_scratch: 1, 2, 4 or 8 query heads per KV head");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_decode_attention_static_scratch: pointers must be 16-byte aligned");
  if (!state && (length < 1 || length > capacity))
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_decode_attention_static_scratch: length outside 1..capacity");
  if (ipe::decode_attention_workspace_bytes(batch, q_heads, capacity) > kStaticScratchBytes)
    return ipe::report_failure(IPE_ERR_UNSUPPORTED,
                               "ipe_decode_attention_static_scratch: batch x q_heads x capacity needs more than the "
                               "2 MiB static scratch; use ipe_decode_attention with a caller workspace");
  int status = IPE_OK;
  float* scratch = scratch_on_current_device(&status);
  if (!scratch) return status;
  cudaError_t e = ipe::launch_decode_attention(q, k_cache, v_cache, out, batch, q_heads, kv_heads, capacity, length,
                                               state, scratch, ipe::device_error_word_ptr(),
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return ipe::report_failure(IPE_ERR_CUDA, cudaGetErrorString(e));
  return IPE_OK;
}
