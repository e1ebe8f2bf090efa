// The extern "C" boundary: host-side argument checks, then the launchers of the kernel files.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "tensor_map.h"

namespace ipe {
size_t decode_attention_workspace_bytes(int batch, int q_heads, int capacity);
}

namespace {

thread_local char g_message[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return IPE_OK;
  return fail(IPE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One error word per device: the first device-side failure code since the last reset.
__device__ int g_device_error;

int* device_error_word() {
  static std::mutex mu;
  static int* words[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    words[dev] = static_cast<int*>(p);
  }
  return words[dev];
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

namespace ipe {
// Lets entry points defined in other files set the calling thread's ipe_last_error() message.
int report_failure(int status, const char* message) { return fail(status, "%s", message); }
int* device_error_word_ptr() { return device_error_word(); }
}  // namespace ipe

extern "C" {

const char* ipe_last_error(void) { return g_message; }

int ipe_abi_version(void) { return 1; }

int ipe_device_error(int reset, int* out_code) {
  if (!out_code) return fail(IPE_ERR_ARGUMENT, "ipe_device_error: out_code is null");
  int* word = device_error_word();
  if (!word) return fail(IPE_ERR_CUDA, "ipe_device_error: no device error word");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "ipe_device_error");
  e = cudaMemcpy(out_code, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "ipe_device_error");
  if (reset) {
    e = cudaMemset(word, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "ipe_device_error");
  }
  return IPE_OK;
}

int ipe_rmsnorm(const void* x, const void* weight, void* out, int64_t rows, int width, float eps, int dtype,
                void* stream) {
  if (!x || !weight || !out) return fail(IPE_ERR_ARGUMENT, "ipe_rmsnorm: null pointer");
  if (rows < 0 || width < 1) return fail(IPE_ERR_ARGUMENT, "ipe_rmsnorm: rows %lld width %d", (long long)rows, width);
  if (dtype != 0 && dtype != 1) return fail(IPE_ERR_ARGUMENT, "ipe_rmsnorm: dtype %d", dtype);
  if (rows == 0) return IPE_OK;
  if (rows > 0x7fffffff) return fail(IPE_ERR_UNSUPPORTED, "ipe_rmsnorm: too many rows");
  ipe::launch_rmsnorm(x, weight, out, rows, width, eps, dtype == 0, as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_rmsnorm");
}

int ipe_embed(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
              void* stream) {
  if (!ids || !table || !out) return fail(IPE_ERR_ARGUMENT, "ipe_embed: null pointer");
  if (count < 0 || vocab < 1 || hidden < 8 || hidden % 8) return fail(IPE_ERR_ARGUMENT, "ipe_embed: bad sizes");
  if (!aligned16(table) || !aligned16(out)) return fail(IPE_ERR_ARGUMENT, "ipe_embed: table/out not 16-byte aligned");
  if (count == 0) return IPE_OK;
  ipe::launch_embed(ids, count, table, vocab, hidden, out, device_error_word(), as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_embed");
}

int ipe_qk_norm_rope_append(const void* qkv, int batch, int tokens, int q_heads, int kv_heads,
                            const void* q_norm_weight, const void* k_norm_weight, const void* cos_table,
                            const void* sin_table, int start, const int64_t* state, void* q_out, void* k_cache,
                            void* v_cache, int capacity, float eps, void* stream) {
  if (!qkv || !q_norm_weight || !k_norm_weight || !cos_table || !sin_table || !q_out || !k_cache || !v_cache)
    return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append: null pointer");
  if (batch < 1 || tokens < 1 || q_heads < 1 || kv_heads < 1 || q_heads % kv_heads || capacity < 1)
    return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append: bad sizes");
  if (!state && (start < 0 || start + tokens > capacity))
    return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append: positions %d..%d outside capacity %d", start,
                start + tokens - 1, capacity);
  ipe::launch_qk_norm_rope_append(qkv, batch, tokens, q_heads, kv_heads, q_norm_weight, k_norm_weight, cos_table,
                                  sin_table, start, state, q_out, k_cache, v_cache, capacity, eps,
                                  device_error_word(), as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_qk_norm_rope_append");
}

static int gemv_checks(const char* name, const void* x, const void* w, const void* out, int batch, int k, int rows) {
  if (!x || !w || !out) return fail(IPE_ERR_ARGUMENT, "%s: null pointer", name);
  if (batch < 1 || batch > 16) return fail(IPE_ERR_UNSUPPORTED, "%s: batch %d outside 1..16", name, batch);
  if (k < 128 || k % 128) return fail(IPE_ERR_UNSUPPORTED, "%s: in_features %d is not a multiple of 128", name, k);
  if (rows < 1) return fail(IPE_ERR_ARGUMENT, "%s: out_features %d", name, rows);
  if (rows % 32) return fail(IPE_ERR_UNSUPPORTED, "%s: out_features %d is not a multiple of 32", name, rows);
  if (!aligned16(x) || !aligned16(w)) return fail(IPE_ERR_ARGUMENT, "%s: operands must be 16-byte aligned", name);
  return IPE_OK;
}

static int run_gemv(const char* name, ipe::GemvArgs a, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  a.err = device_error_word();
  const size_t need = ipe::gemv_workspace_bytes(a);
  if (need && (!workspace || workspace_bytes < need))
    return fail(IPE_ERR_ARGUMENT, "%s: a zero-filled workspace of %zu bytes is needed", name, need);
  const char* message = nullptr;
  cudaError_t e = ipe::launch_gemv(a, workspace, stream, &message);
  if (e != cudaSuccess && message) return fail(IPE_ERR_CUDA, "%s: %s", name, message);
  return cuda_status(e, name);
}

size_t ipe_decode_tiles_bytes(int rows, int in_features, int gate_up_pair) {
  if (rows < 1 || in_features < 128 || in_features % 128) return 0;
  return ipe::decode_tiles_bytes(rows, in_features, gate_up_pair != 0);
}

int ipe_decode_tiles(const void* w, const void* w_up, void* tiles, int rows, int in_features, void* stream) {
  if (!w || !tiles) return fail(IPE_ERR_ARGUMENT, "ipe_decode_tiles: null pointer");
  if (rows < 1 || in_features < 128 || in_features % 128)
    return fail(IPE_ERR_UNSUPPORTED, "ipe_decode_tiles: in_features %d is not a multiple of 128", in_features);
  if (w_up ? rows % 16 : rows % 32)
    return fail(IPE_ERR_UNSUPPORTED, "ipe_decode_tiles: rows %d must be a multiple of %d", rows, w_up ? 16 : 32);
  if (!aligned16(w) || !aligned16(tiles) || (w_up && !aligned16(w_up)))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_tiles: pointers must be 16-byte aligned");
  return cuda_status(ipe::launch_decode_tiles(w, w_up, tiles, rows, in_features, as_stream(stream)),
                     "ipe_decode_tiles");
}

size_t ipe_decode_linear_workspace(int batch, int weight_rows, int in_features) {
  if (batch < 1 || batch > 16 || weight_rows < 1 || in_features < 128 || in_features % 128) return 0;
  ipe::GemvArgs a{};
  a.batch = batch;
  a.rows = weight_rows;
  a.k = in_features;
  size_t most = 0;
  for (int epi : {ipe::kGemvStore, ipe::kGemvSiluMul}) {
    a.epilogue = epi;
    const size_t need = ipe::gemv_workspace_bytes(a);
    if (need > most) most = need;
  }
  return most;
}

int ipe_rmsnorm_qkv(const void* x, const void* norm_weight, const void* w_qkv, void* qkv_out, int batch, int hidden,
                    int qkv_rows, float eps, void* workspace, size_t workspace_bytes, void* stream) {
  int s = gemv_checks("ipe_rmsnorm_qkv", x, w_qkv, qkv_out, batch, hidden, qkv_rows);
  if (s) return s;
  if (!norm_weight || !aligned16(norm_weight)) return fail(IPE_ERR_ARGUMENT, "ipe_rmsnorm_qkv: norm_weight");
  ipe::GemvArgs a{};
  a.x = x; a.x_stride = hidden; a.norm_weight = norm_weight; a.eps = eps; a.w = w_qkv; a.rows = qkv_rows; a.k = hidden;
  a.batch = batch; a.out = qkv_out; a.out_stride = qkv_rows; a.epilogue = ipe::kGemvStore;
  return run_gemv("ipe_rmsnorm_qkv", a, workspace, workspace_bytes, as_stream(stream));
}

int ipe_linear_residual(const void* act, const void* w, void* x, int batch, int in_features, int out_features,
                        void* workspace, size_t workspace_bytes, void* stream) {
  int s = gemv_checks("ipe_linear_residual", act, w, x, batch, in_features, out_features);
  if (s) return s;
  ipe::GemvArgs a{};
  a.x = act; a.x_stride = in_features; a.w = w; a.rows = out_features; a.k = in_features; a.batch = batch;
  a.out = x; a.out_stride = out_features; a.epilogue = ipe::kGemvResidual;
  return run_gemv("ipe_linear_residual", a, workspace, workspace_bytes, as_stream(stream));
}

int ipe_linear_partial(const void* act, const void* w, float* out, int batch, int in_features, int out_features,
                       void* workspace, size_t workspace_bytes, void* stream) {
  int s = gemv_checks("ipe_linear_partial", act, w, out, batch, in_features, out_features);
  if (s) return s;
  ipe::GemvArgs a{};
  a.x = act; a.x_stride = in_features; a.w = w; a.rows = out_features; a.k = in_features; a.batch = batch;
  a.out = out; a.out_stride = out_features; a.epilogue = ipe::kGemvPartial;
  return run_gemv("ipe_linear_partial", a, workspace, workspace_bytes, as_stream(stream));
}

int ipe_add_partial(void* x, const float* sum, int64_t count, void* stream) {
  if (!x || !sum) return fail(IPE_ERR_ARGUMENT, "ipe_add_partial: null pointer");
  if (count < 0) return fail(IPE_ERR_ARGUMENT, "ipe_add_partial: count %lld", static_cast<long long>(count));
  if (count == 0) return IPE_OK;
  ipe::launch_add_partial(x, sum, count, as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_add_partial");
}

int ipe_rmsnorm_gate_up_silu(const void* x, const void* norm_weight, const void* w_gate_up, void* act_out, int batch,
                             int hidden, int intermediate, float eps, void* workspace, size_t workspace_bytes,
                             void* stream) {
  int s = gemv_checks("ipe_rmsnorm_gate_up_silu", x, w_gate_up, act_out, batch, hidden, 2 * intermediate);
  if (s) return s;
  if (intermediate % IPE_GATE_UP_GROUP)
    return fail(IPE_ERR_UNSUPPORTED, "ipe_rmsnorm_gate_up_silu: intermediate %d is not a multiple of %d", intermediate,
                IPE_GATE_UP_GROUP);
  if (!norm_weight || !aligned16(norm_weight)) return fail(IPE_ERR_ARGUMENT, "ipe_rmsnorm_gate_up_silu: norm_weight");
  ipe::GemvArgs a{};
  a.x = x; a.x_stride = hidden; a.norm_weight = norm_weight; a.eps = eps; a.w = w_gate_up; a.rows = 2 * intermediate;
  a.k = hidden; a.batch = batch; a.out = act_out; a.out_stride = intermediate; a.epilogue = ipe::kGemvSiluMul;
  return run_gemv("ipe_rmsnorm_gate_up_silu", a, workspace, workspace_bytes, as_stream(stream));
}

int ipe_lm_head_parts(int vocab) { return vocab < 1 ? 0 : (vocab + 31) / 32; }

int ipe_lm_head(const void* x, int64_t x_row_stride, const void* norm_weight, const void* embed, float* logits,
                float* partials, int batch, int hidden, int vocab, float eps, float temperature, uint64_t seed,
                const int64_t* state, void* stream) {
  int s = gemv_checks("ipe_lm_head", x, embed, logits, batch, hidden, vocab);
  if (s) return s;
  if (!partials || !norm_weight || !aligned16(norm_weight)) return fail(IPE_ERR_ARGUMENT, "ipe_lm_head: null pointer");
  if (x_row_stride < hidden || x_row_stride % 8) return fail(IPE_ERR_ARGUMENT, "ipe_lm_head: x_row_stride");
  if (!(temperature >= 0.f)) return fail(IPE_ERR_ARGUMENT, "ipe_lm_head: temperature must be >= 0");
  ipe::GemvArgs a{};
  a.x = x; a.x_stride = x_row_stride; a.norm_weight = norm_weight; a.eps = eps; a.w = embed; a.rows = vocab;
  a.k = hidden; a.batch = batch; a.out = logits; a.out_stride = vocab; a.partials = partials;
  a.temperature = temperature; a.seed = seed; a.state = state; a.epilogue = ipe::kGemvLogits;
  return run_gemv("ipe_lm_head", a, nullptr, 0, as_stream(stream));
}

int ipe_lm_head_shard(const void* x, int64_t x_row_stride, const void* norm_weight, const void* embed_tiles,
                      float* logits, float* partials, int batch, int hidden, int vocab_rows, int vocab_offset,
                      float eps, float temperature, uint64_t seed, const int64_t* state, void* stream) {
  int s = gemv_checks("ipe_lm_head_shard", x, embed_tiles, logits, batch, hidden, vocab_rows);
  if (s) return s;
  if (!partials || !norm_weight || !aligned16(norm_weight))
    return fail(IPE_ERR_ARGUMENT, "ipe_lm_head_shard: null pointer");
  if (vocab_offset < 0 || vocab_offset % 32) return fail(IPE_ERR_ARGUMENT, "ipe_lm_head_shard: vocab_offset %d", vocab_offset);
  if (x_row_stride < hidden || x_row_stride % 8) return fail(IPE_ERR_ARGUMENT, "ipe_lm_head_shard: x_row_stride");
  if (!(temperature >= 0.f)) return fail(IPE_ERR_ARGUMENT, "ipe_lm_head_shard: temperature must be >= 0");
  ipe::GemvArgs a{};
  a.x = x; a.x_stride = x_row_stride; a.norm_weight = norm_weight; a.eps = eps; a.w = embed_tiles; a.rows = vocab_rows;
  a.k = hidden; a.batch = batch; a.out = logits; a.out_stride = vocab_rows; a.partials = partials;
  a.temperature = temperature; a.seed = seed; a.state = state; a.epilogue = ipe::kGemvLogits;
  a.row_offset = vocab_offset;
  return run_gemv("ipe_lm_head_shard", a, nullptr, 0, as_stream(stream));
}

int ipe_sample(const float* partials, const float* logits, int batch, int vocab, float temperature, int64_t* state,
               int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens, void* stream) {
  if (!partials || !logits || !tokens || !logprobs) return fail(IPE_ERR_ARGUMENT, "ipe_sample: null pointer");
  if (batch < 1 || batch > 16 || vocab < 1 || stride < 1) return fail(IPE_ERR_ARGUMENT, "ipe_sample: bad sizes");
  if (!(temperature >= 0.f)) return fail(IPE_ERR_ARGUMENT, "ipe_sample: temperature must be >= 0");
  ipe::launch_sample(partials, ipe_lm_head_parts(vocab), logits, batch, vocab, temperature, state, tokens, logprobs,
                     stride, next_tokens, as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_sample");
}

int ipe_sample_records(const float* partials, int parts, int batch, float temperature, int64_t* state,
                       int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens, void* stream) {
  if (!partials || !tokens || !logprobs) return fail(IPE_ERR_ARGUMENT, "ipe_sample_records: null pointer");
  if (parts < 1 || batch < 1 || batch > 16 || stride < 1) return fail(IPE_ERR_ARGUMENT, "ipe_sample_records: bad sizes");
  if (!(temperature >= 0.f)) return fail(IPE_ERR_ARGUMENT, "ipe_sample_records: temperature must be >= 0");
  ipe::launch_sample(partials, parts, nullptr, batch, 0, temperature, state, tokens, logprobs, stride, next_tokens,
                     as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_sample_records");
}

int ipe_sample_logits(const float* logits, int64_t rows, int vocab, float temperature, uint64_t seed,
                      int64_t* tokens, float* logprobs, void* stream) {
  if (!logits || !tokens || !logprobs) return fail(IPE_ERR_ARGUMENT, "ipe_sample_logits: null pointer");
  if (rows < 0 || rows > 0x7fffffff || vocab < 1) return fail(IPE_ERR_ARGUMENT, "ipe_sample_logits: bad sizes");
  if (!(temperature >= 0.f)) return fail(IPE_ERR_ARGUMENT, "ipe_sample_logits: temperature must be >= 0");
  if (rows == 0) return IPE_OK;
  ipe::launch_sample_logits(logits, rows, vocab, temperature, seed, tokens, logprobs, 1, as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_sample_logits");
}

size_t ipe_decode_attention_workspace(int batch, int q_heads, int capacity) {
  if (batch < 1 || q_heads < 1 || capacity < 1) return 0;
  return ipe::decode_attention_workspace_bytes(batch, q_heads, capacity);
}

static int attention_checks(const char* name, const void* q, const void* k, const void* v, const void* out, int batch,
                            int q_heads, int kv_heads, int capacity) {
  if (!q || !k || !v || !out) return fail(IPE_ERR_ARGUMENT, "%s: null pointer", name);
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || capacity < 1) return fail(IPE_ERR_ARGUMENT, "%s: bad sizes", name);
  if (q_heads % kv_heads) return fail(IPE_ERR_ARGUMENT, "%s: q_heads %% kv_heads != 0", name);
  const int group = q_heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return fail(IPE_ERR_UNSUPPORTED, "%s: %d query heads per KV head (1, 2, 4 or 8 supported)", name, group);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(IPE_ERR_ARGUMENT, "%s: pointers must be 16-byte aligned", name);
  return IPE_OK;
}

int ipe_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int batch, int q_heads,
                         int kv_heads, int capacity, int length, const int64_t* state, void* workspace,
                         size_t workspace_bytes, void* stream) {
  int s = attention_checks("ipe_decode_attention", q, k_cache, v_cache, out, batch, q_heads, kv_heads, capacity);
  if (s) return s;
  if (!state && (length < 1 || length > capacity))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_attention: length %d outside 1..%d", length, capacity);
  if (!workspace || workspace_bytes < ipe_decode_attention_workspace(batch, q_heads, capacity))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_attention: workspace of %zu bytes needed",
                ipe_decode_attention_workspace(batch, q_heads, capacity));
  return cuda_status(ipe::launch_decode_attention(q, k_cache, v_cache, out, batch, q_heads, kv_heads, capacity, length,
                                                  state, static_cast<float*>(workspace), device_error_word(),
                                                  as_stream(stream)),
                     "ipe_decode_attention");
}

size_t ipe_decode_attention_qkv_workspace(int batch, int q_heads, int kv_heads, int capacity) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || capacity < 1) return 0;
  return ipe::fused_decode_workspace_bytes(batch, q_heads, kv_heads, capacity);
}

int ipe_decode_attention_qkv(const void* qkv, const void* q_norm_weight, const void* k_norm_weight,
                             const void* cos_table, const void* sin_table, int start, const int64_t* state,
                             void* k_cache, void* v_cache, void* out, int batch, int q_heads, int kv_heads,
                             int capacity, float eps, void* workspace, size_t workspace_bytes, void* stream) {
  int s = attention_checks("ipe_decode_attention_qkv", qkv, k_cache, v_cache, out, batch, q_heads, kv_heads, capacity);
  if (s) return s;
  if (!q_norm_weight || !k_norm_weight || !cos_table || !sin_table)
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_attention_qkv: null pointer");
  if (!state && (start < 0 || start >= capacity))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_attention_qkv: position %d outside 0..%d", start, capacity - 1);
  const size_t need = ipe::fused_decode_workspace_bytes(batch, q_heads, kv_heads, capacity);
  if (!workspace || workspace_bytes < need)
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_attention_qkv: a zero-filled workspace of %zu bytes is needed", need);
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(workspace))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_attention_qkv: caches and workspace must be 16-byte aligned (bulk copies)");
  return cuda_status(ipe::launch_decode_attention_fused(qkv, q_norm_weight, k_norm_weight, cos_table, sin_table, state,
                                                        start, k_cache, v_cache, out, batch, q_heads, kv_heads,
                                                        capacity, eps, workspace, device_error_word(),
                                                        as_stream(stream)),
                     "ipe_decode_attention_qkv");
}

int ipe_prefill_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int batch, int q_heads,
                          int kv_heads, int tokens, int capacity, void* stream) {
  int s = attention_checks("ipe_prefill_attention", q, k_cache, v_cache, out, batch, q_heads, kv_heads, capacity);
  if (s) return s;
  if (tokens < 1 || tokens > capacity)
    return fail(IPE_ERR_ARGUMENT, "ipe_prefill_attention: tokens %d outside 1..%d", tokens, capacity);
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(IPE_ERR_ARGUMENT, "ipe_prefill_attention: q, caches and out must be 16-byte aligned (TMA)");
  return cuda_status(ipe::launch_prefill_attention_tc(q, k_cache, v_cache, out, batch, q_heads, kv_heads, tokens,
                                                      capacity, device_error_word(), as_stream(stream)),
                     "ipe_prefill_attention");
}

int ipe_gemm(const void* a, const void* b, void* c, int m, int n, int k, int epilogue, const void* residual,
             void* stream) {
  if (!a || !b || !c) return fail(IPE_ERR_ARGUMENT, "ipe_gemm: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(IPE_ERR_ARGUMENT, "ipe_gemm: m %d n %d k %d", m, n, k);
  if (n % 128 || k % 64) return fail(IPE_ERR_UNSUPPORTED, "ipe_gemm: n %% 128 and k %% 64 must be 0 (n %d k %d)", n, k);
  if (epilogue < IPE_EPI_STORE || epilogue > IPE_EPI_PARTIAL) return fail(IPE_ERR_ARGUMENT, "ipe_gemm: epilogue");
  if (epilogue == IPE_EPI_RESIDUAL && (!residual || !aligned16(residual)))
    return fail(IPE_ERR_ARGUMENT, "ipe_gemm: residual epilogue needs an aligned residual");
  if (!aligned16(a) || !aligned16(b) || !aligned16(c)) return fail(IPE_ERR_ARGUMENT, "ipe_gemm: unaligned operand");
  const char* message = nullptr;
  cudaError_t e = ipe::launch_gemm(a, b, c, m, n, k, epilogue, residual, device_error_word(), as_stream(stream),
                                   &message);
  if (e != cudaSuccess && message) return fail(IPE_ERR_CUDA, "ipe_gemm: %s", message);
  return cuda_status(e, "ipe_gemm");
}

// ----------------------------------------------------------------------- fp32 (plumbing) path

int ipe_gemm_f32(const void* a, const void* w, void* c, int m, int n, int k, int epilogue, const void* residual,
                 void* stream) {
  if (!a || !w || !c) return fail(IPE_ERR_ARGUMENT, "ipe_gemm_f32: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(IPE_ERR_ARGUMENT, "ipe_gemm_f32: m %d n %d k %d", m, n, k);
  if (epilogue < IPE_EPI_STORE || epilogue > IPE_EPI_LOGITS) return fail(IPE_ERR_ARGUMENT, "ipe_gemm_f32: epilogue");
  if (epilogue == IPE_EPI_SILU_MUL && n % (2 * IPE_GATE_UP_GROUP))
    return fail(IPE_ERR_UNSUPPORTED, "ipe_gemm_f32: gate/up rows %d are not whole groups of %d", n, 2 * IPE_GATE_UP_GROUP);
  if (epilogue == IPE_EPI_RESIDUAL && !residual)
    return fail(IPE_ERR_ARGUMENT, "ipe_gemm_f32: residual epilogue needs a residual");
  return cuda_status(ipe::launch_gemm_f32(a, w, c, m, n, k, epilogue, residual, as_stream(stream)), "ipe_gemm_f32");
}

int ipe_embed_f32(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
                  void* stream) {
  if (!ids || !table || !out) return fail(IPE_ERR_ARGUMENT, "ipe_embed_f32: null pointer");
  if (count < 0 || vocab < 1 || hidden < 1) return fail(IPE_ERR_ARGUMENT, "ipe_embed_f32: bad sizes");
  if (count == 0) return IPE_OK;
  ipe::launch_embed_f32(ids, count, table, vocab, hidden, out, device_error_word(), as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_embed_f32");
}

int ipe_qk_norm_rope_append_f32(const void* qkv, int batch, int tokens, int q_heads, int kv_heads,
                                const void* q_norm_weight, const void* k_norm_weight, const void* cos_table,
                                const void* sin_table, int start, void* q_out, void* k_cache, void* v_cache,
                                int capacity, float eps, void* stream) {
  if (!qkv || !q_norm_weight || !k_norm_weight || !cos_table || !sin_table || !q_out || !k_cache || !v_cache)
    return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append_f32: null pointer");
  if (batch < 1 || tokens < 1 || q_heads < 1 || kv_heads < 1 || q_heads % kv_heads || capacity < 1)
    return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append_f32: bad sizes");
  if (start < 0 || start + tokens > capacity)
    return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append_f32: positions %d..%d outside capacity %d", start,
                start + tokens - 1, capacity);
  for (const void* p : {qkv, static_cast<const void*>(q_out), static_cast<const void*>(k_cache),
                        static_cast<const void*>(v_cache)})
    if (!aligned16(p)) return fail(IPE_ERR_ARGUMENT, "ipe_qk_norm_rope_append_f32: unaligned operand");
  ipe::launch_qk_norm_rope_append_f32(qkv, batch, tokens, q_heads, kv_heads, q_norm_weight, k_norm_weight, cos_table,
                                      sin_table, start, q_out, k_cache, v_cache, capacity, eps, device_error_word(),
                                      as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_qk_norm_rope_append_f32");
}

int ipe_attention_f32(const void* q, const void* k_cache, const void* v_cache, void* out, int batch, int q_heads,
                      int kv_heads, int tokens, int capacity, int start, void* stream) {
  if (!q || !k_cache || !v_cache || !out) return fail(IPE_ERR_ARGUMENT, "ipe_attention_f32: null pointer");
  if (batch < 1 || tokens < 1 || q_heads < 1 || kv_heads < 1 || q_heads % kv_heads || capacity < 1)
    return fail(IPE_ERR_ARGUMENT, "ipe_attention_f32: bad sizes");
  if (start < 0 || start + tokens > capacity)
    return fail(IPE_ERR_ARGUMENT, "ipe_attention_f32: positions %d..%d outside capacity %d", start, start + tokens - 1,
                capacity);
  if (!aligned16(k_cache) || !aligned16(v_cache)) return fail(IPE_ERR_ARGUMENT, "ipe_attention_f32: unaligned cache");
  return cuda_status(ipe::launch_attention_f32(q, k_cache, v_cache, out, batch, q_heads, kv_heads, tokens, capacity,
                                               start, as_stream(stream)),
                     "ipe_attention_f32");
}

// ---------------------------------------------------------------- NVLink peer-memory all-reduce

size_t ipe_comm_bytes(size_t slot_bytes) { return ipe::comm_region_bytes(slot_bytes); }

size_t ipe_comm_slot_offset(int slot, size_t slot_bytes) {
  return slot == 0 || slot == 1 ? ipe::comm_slot_offset(slot, slot_bytes) : 0;
}

int ipe_comm_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(IPE_ERR_ARGUMENT, "ipe_comm_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  return cuda_status(e, "ipe_comm_alloc");
}

int ipe_comm_free(void* ptr) { return cuda_status(cudaFree(ptr), "ipe_comm_free"); }

int ipe_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return fail(IPE_ERR_ARGUMENT, "ipe_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e == cudaSuccess) std::memcpy(handle, &h, sizeof(h));
  return cuda_status(e, "ipe_ipc_handle");
}

int ipe_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(IPE_ERR_ARGUMENT, "ipe_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipe_ipc_open");
}

int ipe_ipc_close(void* ptr) { return cuda_status(cudaIpcCloseMemHandle(ptr), "ipe_ipc_close"); }

int ipe_allreduce_residual(void* x, int64_t count, const void* peers, int world, int rank, int slot,
                           size_t slot_bytes, void* stream) {
  if (!x || !peers) return fail(IPE_ERR_ARGUMENT, "ipe_allreduce_residual: null pointer");
  if (world < 1 || world > 32 || rank < 0 || rank >= world || (slot != 0 && slot != 1))
    return fail(IPE_ERR_ARGUMENT, "ipe_allreduce_residual: rank %d of %d, slot %d", rank, world, slot);
  if (count < 1 || static_cast<size_t>(count) * sizeof(float) > slot_bytes)
    return fail(IPE_ERR_ARGUMENT, "ipe_allreduce_residual: %lld values do not fit a %zu-byte slot",
                static_cast<long long>(count), slot_bytes);
  ipe::launch_allreduce_residual(x, count, static_cast<const uint64_t*>(peers), world, rank, slot, slot_bytes,
                                 device_error_word(), as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_allreduce_residual");
}

size_t ipe_decode_step_workspace(int batch, int q_heads, int kv_heads, int capacity) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || capacity < 1) return 0;
  return ipe::decode_step_workspace_bytes(batch, q_heads, kv_heads, capacity);
}

int ipe_decode_step_grid(void) { return ipe::sm_count(); }

size_t ipe_decode_step_comm_bytes(int tp_world, int batch, int hidden) {
  if (tp_world < 1 || batch < 1 || hidden < 1) return 0;
  return ipe::decode_step_comm_bytes(tp_world, batch, hidden);
}

int ipe_decode_step(const ipe_decode_step_desc* d, void* stream) {
  if (!d) return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: null descriptor");
  if (!d->layer_descs || !d->embed || !d->lm_head_tiles || !d->final_norm || !d->cos_table || !d->sin_table ||
      !d->state || !d->tokens || !d->x || !d->qkv || !d->attn || !d->act || !d->logits || !d->partials ||
      !d->workspace)
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: null pointer in the descriptor");
  const void* const operands[] = {d->embed, d->lm_head_tiles, d->final_norm, d->cos_table, d->sin_table, d->x,
                                  d->qkv,   d->attn,          d->act,        d->logits,    d->workspace,
                                  d->layer_descs};
  for (const void* p : operands)
    if (!aligned16(p)) return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: descriptor pointers must be 16-byte aligned");
  if (d->layers < 1 || d->batch < 1 || d->batch > 16 || d->capacity < 1 || d->vocab < 1 || d->q_heads < 1 ||
      d->kv_heads < 1 || d->q_heads % d->kv_heads)
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: bad sizes");
  const int group = d->q_heads / d->kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return fail(IPE_ERR_UNSUPPORTED, "ipe_decode_step: %d query heads per KV head", group);
  if (d->hidden % 128 || d->intermediate % 128 || d->vocab % 32)
    return fail(IPE_ERR_UNSUPPORTED, "ipe_decode_step: hidden / intermediate must be multiples of 128, vocab of 32");
  if (d->history_tokens && (!d->history_logprobs || d->history_stride < 1))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: history needs logprobs and a stride");
  if (d->tp_world > 1 && (d->tp_world > 32 || d->tp_rank < 0 || d->tp_rank >= d->tp_world || !d->tp_peers ||
                         !d->x_alt || !aligned16(d->x_alt) || d->vocab_total < d->vocab || d->vocab_offset < 0 ||
                         d->vocab_offset % 32))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: tensor-parallel fields");
  if (d->workspace_bytes < ipe_decode_step_workspace(d->batch, d->q_heads, d->kv_heads, d->capacity))
    return fail(IPE_ERR_ARGUMENT, "ipe_decode_step: workspace of %zu bytes needed",
                ipe_decode_step_workspace(d->batch, d->q_heads, d->kv_heads, d->capacity));
  const char* message = nullptr;
  cudaError_t e = ipe::launch_decode_step(*d, device_error_word(), as_stream(stream), &message);
  if (e != cudaSuccess && message) return fail(IPE_ERR_CUDA, "ipe_decode_step: %s", message);
  return cuda_status(e, "ipe_decode_step");
}

int ipe_state_set(int64_t* state, int index, int64_t value, void* stream) {
  if (!state || index < 0 || index >= IPE_STATE_WORDS) return fail(IPE_ERR_ARGUMENT, "ipe_state_set: bad arguments");
  ipe::launch_state_update(state, index, value, false, as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_state_set");
}

int ipe_state_add(int64_t* state, int index, int64_t delta, void* stream) {
  if (!state || index < 0 || index >= IPE_STATE_WORDS) return fail(IPE_ERR_ARGUMENT, "ipe_state_add: bad arguments");
  ipe::launch_state_update(state, index, delta, true, as_stream(stream));
  return cuda_status(cudaGetLastError(), "ipe_state_add");
}

}  // extern "C"
