// Internal launchers shared by the kernel translation units and the C-ABI layer (capi.cu).
// Arguments are validated by the C-ABI layer before any of these is called.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

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
enum GemvEpilogue : int { kGemvStore = 0, kGemvResidual = 1, kGemvSiluMul = 2, kGemvLogits = 3 };
struct GemvArgs {
  const void* x;           // bf16 activations, row b at x + b * x_stride
  int64_t x_stride;
  const void* norm_weight;  // non-null: RMSNorm x rows first (width k)
  float eps;
  const void* w;  // bf16 [rows, k]
  int rows;       // weight rows (for SiLU: 2 * intermediate, interleaved in groups of 64)
  int k;
  int batch;
  void* out;  // bf16 (store / residual in-out / silu) or fp32 logits
  int64_t out_stride;
  float* partials;  // logits: sampling partial records
  float temperature;
  uint64_t seed;
  const int64_t* state;
  int epilogue;
  int* err;
};
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream);
int gemv_rows_per_block(int epilogue);
size_t gemv_smem_bytes(const GemvArgs& a);

void launch_sample(const float* partials, int parts, const float* logits, int batch, int vocab, float temperature,
                   int64_t* state, int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens,
                   cudaStream_t stream);

void launch_sample_logits(const float* logits, int64_t rows, int vocab, float temperature, uint64_t seed,
                          int64_t* tokens, float* logprobs, int64_t stride, cudaStream_t stream);

// Attention (attention_decode.cu, attention_prefill.cu).
int decode_attention_chunk();
cudaError_t launch_decode_attention(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                    int kv_heads, int capacity, int length, const int64_t* state, float* workspace,
                                    cudaStream_t stream);
cudaError_t launch_prefill_attention(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                     int kv_heads, int tokens, int capacity, cudaStream_t stream);

// tcgen05 GEMM (gemm_tcgen05.cu). Returns a CUDA error or cudaSuccess; *message set on failure.
cudaError_t launch_gemm(const void* a, const void* b, void* c, int m, int n, int k, int epilogue,
                        const void* residual, int* err, cudaStream_t stream, const char** message);

}  // namespace ipe
