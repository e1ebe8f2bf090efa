// Small memory-bound kernels: RMSNorm rows, embedding gather, per-head q/k norm + RoPE + KV append,
// and the device step-state updates.
#include "common.cuh"
#include "launch.h"

namespace ipe {

// ------------------------------------------------------------------------------- rms_norm rows
// One CTA per row. fp32 statistics; at bf16 the normalised value is rounded before the weight
// multiply and the product is rounded again (reference src/ipe/ops.py:23-33).
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                           T* __restrict__ out, int width, float eps) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * width;
  T* orow = out + row * width;
  float ss = 0.f;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float v = static_cast<float>(xr[i]);
    ss += v * v;
  }
  __shared__ float part[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) part[0] = v;
  }
  __syncthreads();
  const float rstd = rsqrtf(part[0] / static_cast<float>(width) + eps);
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float n = static_cast<float>(xr[i]) * rstd;
    if constexpr (sizeof(T) == 2) {
      orow[i] = __float2bfloat16_rn(static_cast<float>(w[i]) * bf16_round(n));
    } else {
      orow[i] = static_cast<float>(w[i]) * n;
    }
  }
}

void launch_rmsnorm(const void* x, const void* w, void* out, int64_t rows, int width, float eps, bool bf16_io,
                    cudaStream_t stream) {
  if (bf16_io) {
    rmsnorm_rows_kernel<bf16><<<static_cast<unsigned>(rows), 256, 0, stream>>>(
        static_cast<const bf16*>(x), static_cast<const bf16*>(w), static_cast<bf16*>(out), width, eps);
  } else {
    rmsnorm_rows_kernel<float><<<static_cast<unsigned>(rows), 256, 0, stream>>>(
        static_cast<const float*>(x), static_cast<const float*>(w), static_cast<float*>(out), width, eps);
  }
}

// ------------------------------------------------------------------------------- embedding
__global__ void __launch_bounds__(256) embed_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ table,
                                                    int64_t vocab, int hidden, bf16* __restrict__ out, int* err) {
  const int64_t row = blockIdx.x;
  const int64_t id = ids[row];
  uint4* dst = reinterpret_cast<uint4*>(out + row * hidden);
  const int vecs = hidden / 8;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report(err, kErrTokenRange);
    for (int i = threadIdx.x; i < vecs; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * hidden);
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) dst[i] = ldg16(src + i);
}

void launch_embed(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
                  int* err, cudaStream_t stream) {
  embed_kernel<<<static_cast<unsigned>(count), 256, 0, stream>>>(ids, static_cast<const bf16*>(table), vocab, hidden,
                                                                  static_cast<bf16*>(out), err);
}

// ------------------------------------------------------------------- q/k norm + RoPE + append
// One warp per (token, head slot); slots are q heads, then k heads, then v heads. Lane l holds
// elements 4l..4l+3 of the 128-wide head, so the rotate-half partner (d +- 64) is lane l ^ 16.
__global__ void __launch_bounds__(256) qk_norm_rope_append_kernel(
    const bf16* __restrict__ qkv, int tokens, int q_heads, int kv_heads, const bf16* __restrict__ q_norm_w,
    const bf16* __restrict__ k_norm_w, const bf16* __restrict__ cos_t, const bf16* __restrict__ sin_t, int start,
    const int64_t* __restrict__ state, bf16* __restrict__ q_out, bf16* __restrict__ k_cache,
    bf16* __restrict__ v_cache, int capacity, float eps, int64_t total_warps, int* err) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (warp >= total_warps) return;
  const int lane = threadIdx.x & 31;
  const int slots = q_heads + 2 * kv_heads;
  const int slot = static_cast<int>(warp % slots);
  const int64_t row = warp / slots;  // b * tokens + t
  const int t = static_cast<int>(row % tokens);
  const int b = static_cast<int>(row / tokens);
  const int base = state ? static_cast<int>(state[IPE_STATE_POS]) : start;
  const int pos = base + t;
  if (pos < 0 || pos >= capacity) {
    if (lane == 0) report(err, kErrPositionRange);
    return;
  }
  const int d0 = lane * 4;
  const bf16* src = qkv + row * (static_cast<int64_t>(slots) * 128) + slot * 128 + d0;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float x[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                __uint_as_float(raw.y & 0xffff0000u)};
  if (slot >= q_heads + kv_heads) {  // value head: copy into the cache
    const int h = slot - q_heads - kv_heads;
    bf16* dst = v_cache + ((static_cast<int64_t>(b) * kv_heads + h) * capacity + pos) * 128 + d0;
    *reinterpret_cast<uint2*>(dst) = raw;
    return;
  }
  const bool is_q = slot < q_heads;
  const bf16* nw = is_q ? q_norm_w : k_norm_w;
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / 128.f + eps);
  float h[4], p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = bf16_round(__bfloat162float(nw[d0 + i]) * bf16_round(x[i] * rstd));
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, h[i], 16);
  const bf16* cr = cos_t + static_cast<int64_t>(pos) * 128 + d0;
  const bf16* sr = sin_t + static_cast<int64_t>(pos) * 128 + d0;
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float rot = d0 < 64 ? -p[i] : p[i];
    const float t1 = bf16_round(h[i] * __bfloat162float(cr[i]));
    const float t2 = bf16_round(rot * __bfloat162float(sr[i]));
    o[i] = t1 + t2;
  }
  uint2 packed = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
  bf16* dst;
  if (is_q) {
    dst = q_out + ((static_cast<int64_t>(b) * q_heads + slot) * tokens + t) * 128 + d0;
  } else {
    const int h2 = slot - q_heads;
    dst = k_cache + ((static_cast<int64_t>(b) * kv_heads + h2) * capacity + pos) * 128 + d0;
  }
  *reinterpret_cast<uint2*>(dst) = packed;
}

void launch_qk_norm_rope_append(const void* qkv, int batch, int tokens, int q_heads, int kv_heads, const void* qn,
                                const void* kn, const void* cos_t, const void* sin_t, int start, const int64_t* state,
                                void* q_out, void* k_cache, void* v_cache, int capacity, float eps, int* err,
                                cudaStream_t stream) {
  const int64_t warps = static_cast<int64_t>(batch) * tokens * (q_heads + 2 * kv_heads);
  const unsigned blocks = static_cast<unsigned>((warps + 7) / 8);
  qk_norm_rope_append_kernel<<<blocks, 256, 0, stream>>>(
      static_cast<const bf16*>(qkv), tokens, q_heads, kv_heads, static_cast<const bf16*>(qn),
      static_cast<const bf16*>(kn), static_cast<const bf16*>(cos_t), static_cast<const bf16*>(sin_t), start, state,
      static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache), capacity, eps, warps, err);
}

// ------------------------------------------------------------------------------- step state
__global__ void state_update_kernel(int64_t* state, int index, int64_t value, int add) {
  if (add) state[index] += value;
  else state[index] = value;
}

void launch_state_update(int64_t* state, int index, int64_t value, bool add, cudaStream_t stream) {
  state_update_kernel<<<1, 1, 0, stream>>>(state, index, value, add ? 1 : 0);
}

// ------------------------------------------------------------------ residual add of a summed part
// x = bf16(x + bf16(sum)): the residual update of a layer whose product was summed in fp32 over
// tensor-parallel ranks, with the rounding points of the unsplit layer.
__global__ void __launch_bounds__(256) add_partial_kernel(bf16* __restrict__ x, const float* __restrict__ sum,
                                                          int64_t count) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < count) x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) + bf16_round(sum[i]));
}

void launch_add_partial(void* x, const float* sum, int64_t count, cudaStream_t stream) {
  add_partial_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(static_cast<bf16*>(x), sum,
                                                                                      count);
}

}  // namespace ipe
