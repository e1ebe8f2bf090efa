// Internal launchers shared by the kernel translation units and the C-ABI layer (capi.cu).
// Arguments are validated by the C-ABI layer before any of these is called.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "ipe_b200.h"

namespace ipe {

void launch_rmsnorm(const void* x, const void* w, void* out, int64_t rows, int width, float eps, bool bf16_io,
                    cudaStream_t stream);
void launch_embed(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
                  int* err, cudaStream_t stream);
void launch_qk_norm_rope_append(const void* qkv, int batch, int tokens, int q_heads, int kv_heads, const void* qn,
                                const void* kn, const void* cos_t, const void* sin_t, int start, const int64_t* state,
                                void* q_out, void* k_cache, void* v_cache, int capacity, float eps, int* err,
                                cudaStream_t stream);
void launch_state_update(int64_t* state, int index, int64_t value, bool add, cudaStream_t stream);

// Decode weight-streaming linear layers (gemv.cu).
enum GemvEpilogue : int { kGemvStore = 0, kGemvResidual = 1, kGemvSiluMul = 2, kGemvLogits = 3, kGemvPartial = 4 };
struct GemvArgs {
  const void* x;           // bf16 activations, row b at x + b * x_stride
  int64_t x_stride;
  const void* norm_weight;  // RMSNorm weight for the norm-fused epilogues (width k)
  float eps;
  const void* w;  // decode tiles of the bf16 [rows, k] weight (ipe_decode_tiles)
  int rows;       // weight rows (for SiLU: 2 * intermediate, interleaved in groups of 64)
  int k;
  int batch;
  void* out;  // bf16 (store / residual in-out / silu) or fp32 logits
  int64_t out_stride;
  float* partials;  // logits: sampling partial records, one per 32 rows
  float temperature;
  uint64_t seed;
  const int64_t* state;
  int epilogue;
  int* err;
  float* slots;    // split-K partial tiles (set by launch_gemv from the workspace)
  int* counters;   // split-K arrival counters, zero between launches
  int row_offset;  // logits: global vocabulary ID of weight row 0 (a vocabulary shard)
};
// Bytes of the decode tile layout of a [rows, k] matrix (pair: two [rows, k] gate/up matrices).
size_t decode_tiles_bytes(int rows, int k, bool pair);
cudaError_t launch_decode_tiles(const void* w, const void* w2, void* out, int rows, int k, cudaStream_t stream);
// Workspace bytes launch_gemv needs for `a` (0 when K is not split); zero-filled before first use.
size_t gemv_workspace_bytes(const GemvArgs& a);
cudaError_t launch_gemv(GemvArgs a, void* workspace, cudaStream_t stream, const char** message);

void launch_sample(const float* partials, int parts, const float* logits, int batch, int vocab, float temperature,
                   int64_t* state, int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens,
                   cudaStream_t stream);

void launch_sample_logits(const float* logits, int64_t rows, int vocab, float temperature, uint64_t seed,
                          int64_t* tokens, float* logprobs, int64_t stride, cudaStream_t stream);

// Attention (attention_decode.cu, attention_prefill_tc.cu).
int decode_attention_chunk();
cudaError_t launch_decode_attention(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                    int kv_heads, int capacity, int length, const int64_t* state, float* workspace,
                                    int* err, cudaStream_t stream);
// The calling device's error word (the first device-side failure code since the last reset), or null.
int* device_error_word_ptr();
size_t fused_decode_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity);
cudaError_t launch_decode_attention_fused(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_t,
                                          const void* sin_t, const int64_t* state, int start, void* k_cache,
                                          void* v_cache, void* out, int batch, int q_heads, int kv_heads, int capacity,
                                          float eps, void* workspace, int* err, cudaStream_t stream);
cudaError_t launch_prefill_attention_tc(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                        int kv_heads, int tokens, int capacity, int* err, cudaStream_t stream);

// Whole decode step (decode_step.cu).
size_t decode_step_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity);
cudaError_t launch_decode_step(const ipe_decode_step_desc& d, int* err, cudaStream_t stream, const char** message);

// tcgen05 GEMM (gemm_tcgen05.cu). Returns a CUDA error or cudaSuccess; *message set on failure.
cudaError_t launch_gemm(const void* a, const void* b, void* c, int m, int n, int k, int epilogue,
                        const void* residual, int* err, cudaStream_t stream, const char** message);

// fp32 (plumbing) path, fp32.cu
cudaError_t launch_gemm_f32(const void* a, const void* w, void* c, int m, int n, int k, int epilogue,
                            const void* residual, cudaStream_t stream);
void launch_embed_f32(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
                      int* err, cudaStream_t stream);
void launch_qk_norm_rope_append_f32(const void* qkv, int batch, int tokens, int q_heads, int kv_heads, const void* qn,
                                    const void* kn, const void* cos_t, const void* sin_t, int start, void* q_out,
                                    void* k_cache, void* v_cache, int capacity, float eps, int* err,
                                    cudaStream_t stream);
cudaError_t launch_attention_f32(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                 int kv_heads, int tokens, int capacity, int start, cudaStream_t stream);

void launch_add_partial(void* x, const float* sum, int64_t count, cudaStream_t stream);

// NVLink peer-memory all-reduce, allreduce.cu
size_t comm_region_bytes(size_t slot_bytes);
size_t comm_slot_offset(int slot, size_t slot_bytes);
void launch_allreduce_residual(void* x, int64_t count, const uint64_t* peers, int world, int rank, int slot,
                               size_t slot_bytes, int* err, cudaStream_t stream);

size_t decode_step_comm_bytes(int world, int batch, int hidden);

}  // namespace ipe
