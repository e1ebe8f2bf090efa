// Split-KV flash-decode for grouped-query attention over the preallocated cache.
//
// Pass 1: one CTA per (chunk of kChunk keys, KV head, batch row) scores the chunk against every
// query head that shares the KV head (the K and V rows are read once for the group), and writes
// the chunk's unnormalised output with its running max and sum. Pass 2 merges the chunks per
// (batch row, query head). The key count comes from the device step state when one is given, so
// the grid is sized by capacity and chunks past the current length exit at once.
#include "common.cuh"
#include "launch.h"

namespace ipe {
namespace {

constexpr int kChunk = 32;   // keys per CTA
constexpr int kThreads = 128;
constexpr int kRecord = 128 + 2;  // floats per (batch, head, chunk) partial: o[128], max, sum
constexpr float kScale = 0.08838834764831845f;  // 128 ** -0.5

template <int G>
__global__ void __launch_bounds__(kThreads) decode_chunk_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                                const bf16* __restrict__ vc, float* __restrict__ ws,
                                                                int q_heads, int kv_heads, int capacity, int length_arg,
                                                                const int64_t* __restrict__ state, int chunks_max) {
  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int length = state ? static_cast<int>(state[IPE_STATE_POS]) + 1 : length_arg;
  const int key0 = chunk * kChunk;
  if (key0 >= length) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  __shared__ float qs[G][128];
  __shared__ float sc[G][kChunk];
  __shared__ float red[8][G][128];
  __shared__ float stat[G][2];

  for (int i = threadIdx.x; i < G * 128; i += kThreads) {
    const int g = i / 128, d = i % 128;
    qs[g][d] = __bfloat162float(q[(static_cast<int64_t>(b) * q_heads + kvh * G + g) * 128 + d]);
  }
  __syncthreads();

  const int64_t head_base = (static_cast<int64_t>(b) * kv_heads + kvh) * capacity;
  // Scores: warp w handles keys key0 + 8w .. +7; 4 lanes per key, 32 dims per lane.
  {
    const int kk = warp * 8 + (lane >> 2);
    const int part = lane & 3;
    const int key = key0 + kk;
    float dot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) dot[g] = 0.f;
    if (key < length) {
      const bf16* kr = kc + (head_base + key) * 128 + part * 32;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        float f[8];
        unpack8(ldg16(kr + v * 8), f);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < 8; ++i) dot[g] += f[i] * qs[g][part * 32 + v * 8 + i];
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 1);
      dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 2);
    }
    if (part == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g][kk] = key < length ? dot[g] * kScale : -INFINITY;
    }
  }
  __syncthreads();
  // Softmax statistics per query head: warp w handles heads w, w + 4; lane = key.
  for (int g = warp; g < G; g += kThreads / 32) {
    const float s = sc[g][lane];
    const float m = warp_max(s);
    const float p = s == -INFINITY ? 0.f : expf(s - m);
    const float l = warp_sum(p);
    sc[g][lane] = p;
    if (lane == 0) {
      stat[g][0] = m;
      stat[g][1] = l;
    }
  }
  __syncthreads();
  // P V: thread (key group kg = tid / 16, dim chunk dc = tid % 16) over keys kg, kg+8, kg+16, kg+24.
  {
    const int kg = threadIdx.x >> 4, dc = threadIdx.x & 15;
    float o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
#pragma unroll
    for (int j = 0; j < kChunk / 8; ++j) {
      const int kk = kg + 8 * j;
      const int key = key0 + kk;
      if (key < length) {
        float f[8];
        unpack8(ldg16(vc + (head_base + key) * 128 + dc * 8), f);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float p = sc[g][kk];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[g][i] += p * f[i];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) red[kg][g][dc * 8 + i] = o[g][i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * 128; i += kThreads) {
    const int g = i / 128, d = i % 128;
    float s = 0.f;
#pragma unroll
    for (int kg = 0; kg < 8; ++kg) s += red[kg][g][d];
    float* rec = ws + ((static_cast<int64_t>(b) * q_heads + kvh * G + g) * chunks_max + chunk) * kRecord;
    rec[d] = s;
    if (d == 0) {
      rec[128] = stat[g][0];
      rec[129] = stat[g][1];
    }
  }
}

__global__ void __launch_bounds__(128) decode_combine_kernel(const float* __restrict__ ws, bf16* __restrict__ out,
                                                             int q_heads, int length_arg,
                                                             const int64_t* __restrict__ state, int chunks_max) {
  const int head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int length = state ? static_cast<int>(state[IPE_STATE_POS]) + 1 : length_arg;
  const int chunks = (length + kChunk - 1) / kChunk;
  const float* base = ws + (static_cast<int64_t>(b) * q_heads + head) * chunks_max * kRecord;
  float m = -INFINITY;
  for (int c = 0; c < chunks; ++c) m = fmaxf(m, base[c * kRecord + 128]);
  float l = 0.f, o = 0.f;
  for (int c = 0; c < chunks; ++c) {
    const float* rec = base + c * kRecord;
    const float e = expf(rec[128] - m);
    l += rec[129] * e;
    o += rec[d] * e;
  }
  out[(static_cast<int64_t>(b) * q_heads + head) * 128 + d] = __float2bfloat16_rn(o / l);
}

// ------------------------------------------------------------------------------------------
// Fused decode step attention, used by the engine: per-head q_norm / k_norm and RoPE of this
// step's q and k straight from the QKV projection output, the K/V append at the current
// position, split-KV attention, and the cross-chunk merge by the last chunk CTA of each
// (row, KV head) to arrive (an arrival counter, reset by that CTA). The merge sums chunks in
// chunk order, so results do not depend on arrival order.

struct FusedArgs {
  const bf16* qkv;  // [batch, (q_heads + 2 * kv_heads) * 128]
  const bf16* q_norm;
  const bf16* k_norm;
  const bf16* cos_t;  // [capacity, 128]
  const bf16* sin_t;
  const int64_t* state;
  int start;
  bf16* k_cache;  // [batch, kv_heads, capacity, 128] of this layer
  bf16* v_cache;
  bf16* out;  // [batch, q_heads * 128]
  float* records;  // [batch, q_heads, chunks_max, kRecord]
  int* counters;   // [batch * kv_heads], zero between launches
  int q_heads, kv_heads, capacity, chunks_max;
  float eps;
  int* err;
};

// RMSNorm over the 128-wide head held 4 elements per lane, then split-half RoPE at `pos`
// (reference rounding: bf16 normalised value, bf16 weight product, bf16 x*cos, rot*sin and sum).
__device__ __forceinline__ void norm_rope4(float (&x)[4], const bf16* w, const bf16* cos_t, const bf16* sin_t, int pos,
                                           int lane, float eps) {
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / 128.f + eps);
  const int d0 = lane * 4;
  float h[4], p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = bf16_round(__bfloat162float(w[d0 + i]) * bf16_round(x[i] * r));
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, h[i], 16);
  const bf16* cr = cos_t + static_cast<int64_t>(pos) * 128 + d0;
  const bf16* sr = sin_t + static_cast<int64_t>(pos) * 128 + d0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float rot = d0 < 64 ? -p[i] : p[i];
    x[i] = bf16_round(bf16_round(h[i] * __bfloat162float(cr[i])) + bf16_round(rot * __bfloat162float(sr[i])));
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads) fused_decode_kernel(const FusedArgs a) {
  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float qs[G][128];
  __shared__ float sc[G][kChunk];
  __shared__ float red[8][G][128];
  __shared__ float stat[G][2];
  __shared__ int last;
  extern __shared__ float weight[];  // [G][chunks_max] merge weights (last CTA only)

  pdl_trigger();
  pdl_wait();
  const int pos = a.state ? static_cast<int>(a.state[IPE_STATE_POS]) : a.start;
  if (pos < 0 || pos >= a.capacity) {
    if (threadIdx.x == 0 && chunk == 0) report(a.err, kErrPositionRange);
    return;
  }
  const int length = pos + 1;
  const int key0 = chunk * kChunk;
  if (key0 >= length) return;
  const int chunks = (length + kChunk - 1) / kChunk;
  const int slots = a.q_heads + 2 * a.kv_heads;
  const bf16* row = a.qkv + static_cast<int64_t>(b) * slots * 128;
  const int64_t head_base = (static_cast<int64_t>(b) * a.kv_heads + kvh) * a.capacity;

  // q heads of this group (warp w: heads w, w + 4), normalised and rotated.
  for (int gi = warp; gi < G; gi += kThreads / 32) {
    const uint2 raw = ldcg8(row + (kvh * G + gi) * 128 + lane * 4);
    float x[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                  __uint_as_float(raw.y & 0xffff0000u)};
    norm_rope4(x, a.q_norm, a.cos_t, a.sin_t, pos, lane, a.eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) qs[gi][lane * 4 + i] = x[i];
  }
  // The chunk holding this step's position appends its K (normalised, rotated) and V rows.
  if (chunk == chunks - 1 && warp == (kThreads / 32) - 1) {
    const uint2 kraw = ldcg8(row + (a.q_heads + kvh) * 128 + lane * 4);
    const uint2 vraw = ldcg8(row + (a.q_heads + a.kv_heads + kvh) * 128 + lane * 4);
    float x[4] = {__uint_as_float(kraw.x << 16), __uint_as_float(kraw.x & 0xffff0000u),
                  __uint_as_float(kraw.y << 16), __uint_as_float(kraw.y & 0xffff0000u)};
    norm_rope4(x, a.k_norm, a.cos_t, a.sin_t, pos, lane, a.eps);
    *reinterpret_cast<uint2*>(a.k_cache + (head_base + pos) * 128 + lane * 4) =
        make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    *reinterpret_cast<uint2*>(a.v_cache + (head_base + pos) * 128 + lane * 4) = vraw;
  }
  __syncthreads();

  // Scores: warp w handles keys key0 + 8w .. +7; 4 lanes per key, 32 dims per lane.
  {
    const int kk = warp * 8 + (lane >> 2);
    const int part = lane & 3;
    const int key = key0 + kk;
    float dot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) dot[g] = 0.f;
    if (key < length) {
      const bf16* kr = a.k_cache + (head_base + key) * 128 + part * 32;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        float f[8];
        unpack8(ldcg16(kr + v * 8), f);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < 8; ++i) dot[g] += f[i] * qs[g][part * 32 + v * 8 + i];
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 1);
      dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 2);
    }
    if (part == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g][kk] = key < length ? dot[g] * kScale : -INFINITY;
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += kThreads / 32) {
    const float s = sc[g][lane];
    const float m = warp_max(s);
    const float p = s == -INFINITY ? 0.f : expf(s - m);
    const float l = warp_sum(p);
    sc[g][lane] = p;
    if (lane == 0) {
      stat[g][0] = m;
      stat[g][1] = l;
    }
  }
  __syncthreads();
  {
    const int kg = threadIdx.x >> 4, dc = threadIdx.x & 15;
    float o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
#pragma unroll
    for (int j = 0; j < kChunk / 8; ++j) {
      const int kk = kg + 8 * j;
      const int key = key0 + kk;
      if (key < length) {
        float f[8];
        unpack8(ldcg16(a.v_cache + (head_base + key) * 128 + dc * 8), f);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float p = sc[g][kk];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[g][i] += p * f[i];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) red[kg][g][dc * 8 + i] = o[g][i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * 128; i += kThreads) {
    const int g = i / 128, d = i % 128;
    float s = 0.f;
#pragma unroll
    for (int kg = 0; kg < 8; ++kg) s += red[kg][g][d];
    float* rec = a.records + ((static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * a.chunks_max + chunk) * kRecord;
    __stcg(rec + d, s);
    if (d == 0) {
      __stcg(rec + 128, stat[g][0]);
      __stcg(rec + 129, stat[g][1]);
    }
  }
  // Arrival: the last chunk CTA of this (row, KV head) merges every chunk.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* counter = a.counters + b * a.kv_heads + kvh;
    const int prior = atomicAdd(counter, 1);
    last = prior == chunks - 1;
    if (last) *counter = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Per head: lanes compute the chunk weights exp(m_c - M) / L, then every thread sums its dims.
  for (int g = warp; g < G; g += kThreads / 32) {
    const float* base = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * a.chunks_max * kRecord;
    float m = -INFINITY;
    for (int c = lane; c < chunks; c += 32) m = fmaxf(m, __ldcg(base + c * kRecord + 128));
    m = warp_max(m);
    float l = 0.f;
    for (int c = lane; c < chunks; c += 32) {
      const float e = expf(__ldcg(base + c * kRecord + 128) - m);
      l += __ldcg(base + c * kRecord + 129) * e;
      weight[g * a.chunks_max + c] = e;
    }
    l = warp_sum(l);
    for (int c = lane; c < chunks; c += 32) weight[g * a.chunks_max + c] /= l;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * 128; i += kThreads) {
    const int g = i / 128, d = i % 128;
    const float* base = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * a.chunks_max * kRecord;
    float o = 0.f;
    const float* wg = weight + g * a.chunks_max;
    for (int c = 0; c < chunks; ++c) o += wg[c] * __ldcg(base + c * kRecord + d);
    a.out[(static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * 128 + d] = __float2bfloat16_rn(o);
  }
}

template <int G>
void launch_chunks(dim3 grid, const bf16* q, const bf16* k, const bf16* v, float* ws, int q_heads, int kv_heads,
                   int capacity, int length, const int64_t* state, int chunks_max, cudaStream_t stream) {
  decode_chunk_kernel<G><<<grid, kThreads, 0, stream>>>(q, k, v, ws, q_heads, kv_heads, capacity, length, state,
                                                        chunks_max);
}

}  // namespace

int decode_attention_chunk() { return kChunk; }

cudaError_t launch_decode_attention(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                    int kv_heads, int capacity, int length, const int64_t* state, float* ws,
                                    cudaStream_t stream) {
  const int chunks_max = (capacity + kChunk - 1) / kChunk;
  const int group = q_heads / kv_heads;
  const dim3 grid(chunks_max, kv_heads, batch);
  auto qq = static_cast<const bf16*>(q);
  auto kk = static_cast<const bf16*>(k);
  auto vv = static_cast<const bf16*>(v);
  switch (group) {
    case 1: launch_chunks<1>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, stream); break;
    case 2: launch_chunks<2>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, stream); break;
    case 4: launch_chunks<4>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, stream); break;
    case 8: launch_chunks<8>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, stream); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_combine_kernel<<<dim3(q_heads, batch), 128, 0, stream>>>(ws, static_cast<bf16*>(out), q_heads, length, state,
                                                                   chunks_max);
  return cudaGetLastError();
}

size_t fused_decode_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity) {
  const int chunks_max = (capacity + kChunk - 1) / kChunk;
  const size_t counters = (static_cast<size_t>(batch) * kv_heads * sizeof(int) + 255) / 256 * 256;
  return counters + static_cast<size_t>(batch) * q_heads * chunks_max * kRecord * sizeof(float);
}

template <int G>
cudaError_t launch_fused(const FusedArgs& a, int batch, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(G) * a.chunks_max * sizeof(float);
  auto kernel = fused_decode_kernel<G>;
  if (smem > 16 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(kernel, dim3(a.chunks_max, a.kv_heads, batch), dim3(kThreads), smem, stream, a);
}

cudaError_t launch_decode_attention_fused(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_t,
                                          const void* sin_t, const int64_t* state, int start, void* k_cache,
                                          void* v_cache, void* out, int batch, int q_heads, int kv_heads, int capacity,
                                          float eps, void* workspace, int* err, cudaStream_t stream) {
  FusedArgs a{};
  a.qkv = static_cast<const bf16*>(qkv);
  a.q_norm = static_cast<const bf16*>(q_norm);
  a.k_norm = static_cast<const bf16*>(k_norm);
  a.cos_t = static_cast<const bf16*>(cos_t);
  a.sin_t = static_cast<const bf16*>(sin_t);
  a.state = state;
  a.start = start;
  a.k_cache = static_cast<bf16*>(k_cache);
  a.v_cache = static_cast<bf16*>(v_cache);
  a.out = static_cast<bf16*>(out);
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.capacity = capacity;
  a.chunks_max = (capacity + kChunk - 1) / kChunk;
  a.eps = eps;
  a.err = err;
  a.counters = static_cast<int*>(workspace);
  const size_t counters = (static_cast<size_t>(batch) * kv_heads * sizeof(int) + 255) / 256 * 256;
  a.records = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + counters);
  switch (q_heads / kv_heads) {
    case 1: return launch_fused<1>(a, batch, stream);
    case 2: return launch_fused<2>(a, batch, stream);
    case 4: return launch_fused<4>(a, batch, stream);
    case 8: return launch_fused<8>(a, batch, stream);
    default: return cudaErrorInvalidValue;
  }
}

size_t decode_attention_workspace_bytes(int batch, int q_heads, int capacity) {
  const int chunks_max = (capacity + kChunk - 1) / kChunk;
  return static_cast<size_t>(batch) * q_heads * chunks_max * kRecord * sizeof(float);
}

}  // namespace ipe
