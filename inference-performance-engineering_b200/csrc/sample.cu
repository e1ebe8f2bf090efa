// Sampling kernels: the fused sampler that reduces the LM head's per-block records, and the
// standalone sampler over a logits matrix held by the caller (reference src/ipe/engine.py:28-41).
#include "common.cuh"
#include "launch.h"
#include "sampling.cuh"

namespace ipe {
namespace {

__global__ void __launch_bounds__(1024) sample_kernel(const float* __restrict__ partials, int parts,
                                                      const float* __restrict__ logits, int B, int V,
                                                      float temperature_arg, int64_t* state, int64_t* tokens,
                                                      float* logprobs, int64_t stride, int64_t* next_tokens) {
  __shared__ Stat shared[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_row = 32 / B;  // warps per batch row (B <= 16)
  const int b = warp / per_row, sub = warp % per_row;
  const int64_t step = state ? state[IPE_STATE_STEP] : 0;
  const float temperature = state ? __int_as_float(static_cast<int>(state[IPE_STATE_TEMPERATURE])) : temperature_arg;
  Stat st = empty_stat();
  if (b < B) {
    for (int p = sub * 32 + lane; p < parts; p += per_row * 32)
      st = merge(st, load_stat(partials + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) st = merge(st, shfl_xor_stat(st, o));
  if (lane == 0) shared[warp] = st;
  __syncthreads();
  if (threadIdx.x < B) {
    const int row = threadIdx.x;
    Stat r = shared[row * per_row];
    for (int i = 1; i < per_row; ++i) r = merge(r, shared[row * per_row + i]);
    const int token = temperature > 0.f ? r.garg : r.arg;
    // the chosen token's logit: from the logits when given, else from the records (the argmax's is
    // the maximum, the Gumbel winner's is carried with it)
    const float logit = logits ? logits[static_cast<int64_t>(row) * V + token] : (temperature > 0.f ? r.gl : r.m);
    const float lp = (logit - r.m) - logf(r.s);
    tokens[row * stride + step] = token;
    logprobs[row * stride + step] = lp;
    if (next_tokens) next_tokens[row] = token;
  }
  __syncthreads();
  if (threadIdx.x == 0 && state) state[IPE_STATE_STEP] = step + 1;
}

// Token and untempered log-probability per row of a logits matrix [rows, V]: one CTA per row.
// Gumbel noise for (seed, row, vocab id) when temperature > 0.
__global__ void __launch_bounds__(256) sample_logits_kernel(const float* __restrict__ logits, int V, float temperature,
                                                            uint64_t seed, int64_t* tokens, float* logprobs,
                                                            int64_t stride) {
  const int64_t row = blockIdx.x;
  const float* l = logits + row * V;
  Stat st = empty_stat();
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = l[v];
    Stat y{x, 1.f, v, -INFINITY, 0x7fffffff, 0.f};
    if (temperature > 0.f) {
      const uint32_t r = philox_word(static_cast<uint32_t>(v), static_cast<uint32_t>(row),
                                     static_cast<uint32_t>(row >> 32), 0xffffffffu, static_cast<uint32_t>(seed),
                                     static_cast<uint32_t>(seed >> 32));
      const float u = static_cast<float>(r >> 8) * (1.0f / 16777216.0f);
      y.gs = x / temperature - logf(-logf(u));
      y.garg = v;
      y.gl = x;
    }
    st = merge(st, y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) st = merge(st, shfl_xor_stat(st, o));
  __shared__ Stat shared[8];
  if ((threadIdx.x & 31) == 0) shared[threadIdx.x >> 5] = st;
  __syncthreads();
  if (threadIdx.x == 0) {
    Stat r = shared[0];
    for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) r = merge(r, shared[i]);
    const int token = temperature > 0.f ? r.garg : r.arg;
    tokens[row * stride] = token;
    logprobs[row * stride] = (l[token] - r.m) - logf(r.s);
  }
}

}  // namespace

void launch_sample(const float* partials, int parts, const float* logits, int batch, int vocab, float temperature,
                   int64_t* state, int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens,
                   cudaStream_t stream) {
  sample_kernel<<<1, 1024, 0, stream>>>(partials, parts, logits, batch, vocab, temperature, state, tokens, logprobs,
                                        stride, next_tokens);
}

}  // namespace ipe

namespace ipe {
void launch_sample_logits(const float* logits, int64_t rows, int vocab, float temperature, uint64_t seed,
                          int64_t* tokens, float* logprobs, int64_t stride, cudaStream_t stream) {
  sample_logits_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(logits, vocab, temperature, seed, tokens,
                                                                        logprobs, stride);
}
}  // namespace ipe
