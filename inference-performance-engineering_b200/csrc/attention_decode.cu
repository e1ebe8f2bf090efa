// Split-KV flash-decode for grouped-query attention over the preallocated cache.
//
// Pass 1: one CTA per (chunk of kChunk keys, KV head, batch row) scores the chunk against every
// query head that shares the KV head (the K and V rows are read once for the group), and writes
// the chunk's unnormalised output with its running max and sum. Pass 2 merges the chunks per
// (batch row, query head). The key count comes from the device step state when one is given, so
// the grid is sized by capacity and chunks past the current length exit at once.
#include "common.cuh"
#include "decode_attention.cuh"
#include "launch.h"
#include "tensor_map.h"

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
                                                                const int64_t* __restrict__ state, int chunks_max,
                                                                int* err) {
  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int length = state ? static_cast<int>(state[IPE_STATE_POS]) + 1 : length_arg;
  // a device position outside the cache: nothing is read or written (the host checks a host length)
  if (length < 1 || length > capacity) {
    if (chunk == 0 && kvh == 0 && b == 0 && threadIdx.x == 0) report(err, kErrPositionRange);
    return;
  }
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
                                                             int q_heads, int capacity, int length_arg,
                                                             const int64_t* __restrict__ state, int chunks_max) {
  const int head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int length = state ? static_cast<int>(state[IPE_STATE_POS]) + 1 : length_arg;
  if (length < 1 || length > capacity) return;  // reported by the chunk kernel; the output is left as it was
  const int chunks = min((length + kChunk - 1) / kChunk, chunks_max);
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
// Fused decode-step attention (decode_attention.cuh): one CTA per (split, KV head, batch row).
template <int G>
__global__ void __launch_bounds__(kAttnThreads) fused_decode_kernel(const FusedArgs a) {
  extern __shared__ __align__(16) float scratch[];
  __shared__ uint64_t bars[kAttnSlotsMax + 1];
  if (threadIdx.x == 0) {
    attn_ring_init(bars);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int pos = a.state ? static_cast<int>(a.state[IPE_STATE_POS]) : a.start;
  if (pos < 0 || pos >= a.capacity) {
    if (threadIdx.x == 0 && split == 0) report(a.err, kErrPositionRange);
    return;
  }
  const AttnSplit sp = attn_split(pos, a.max_splits);
  if (split >= sp.splits) return;
  AttnSeq seq;
  attention_item<G>(a, split, kvh, b, pos, sp, AttnSmem<G>(scratch, bars, kAttnSlotsMax), seq, threadIdx.x);
}

template <int G>
void launch_chunks(dim3 grid, const bf16* q, const bf16* k, const bf16* v, float* ws, int q_heads, int kv_heads,
                   int capacity, int length, const int64_t* state, int chunks_max, int* err, cudaStream_t stream) {
  decode_chunk_kernel<G><<<grid, kThreads, 0, stream>>>(q, k, v, ws, q_heads, kv_heads, capacity, length, state,
                                                        chunks_max, err);
}

}  // namespace

int decode_attention_chunk() { return kChunk; }

cudaError_t launch_decode_attention(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                    int kv_heads, int capacity, int length, const int64_t* state, float* ws,
                                    int* err, cudaStream_t stream) {
  const int chunks_max = (capacity + kChunk - 1) / kChunk;
  const int group = q_heads / kv_heads;
  const dim3 grid(chunks_max, kv_heads, batch);
  auto qq = static_cast<const bf16*>(q);
  auto kk = static_cast<const bf16*>(k);
  auto vv = static_cast<const bf16*>(v);
  switch (group) {
    case 1: launch_chunks<1>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, err, stream); break;
    case 2: launch_chunks<2>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, err, stream); break;
    case 4: launch_chunks<4>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, err, stream); break;
    case 8: launch_chunks<8>(grid, qq, kk, vv, ws, q_heads, kv_heads, capacity, length, state, chunks_max, err, stream); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_combine_kernel<<<dim3(q_heads, batch), 128, 0, stream>>>(ws, static_cast<bf16*>(out), q_heads, capacity,
                                                                   length, state, chunks_max);
  return cudaGetLastError();
}

size_t fused_decode_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity) {
  (void)capacity;  // records are per split, and splits are bounded by kAttnSplitsMax
  const size_t counters = (static_cast<size_t>(batch) * kv_heads * sizeof(int) + 255) / 256 * 256;
  return counters + static_cast<size_t>(batch) * q_heads * kAttnSplitsMax * kAttnRecord * sizeof(float);
}

template <int G>
cudaError_t launch_fused(const FusedArgs& a, int batch, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(attn_smem_floats<G>(kAttnSlotsMax)) * sizeof(float);
  auto kernel = fused_decode_kernel<G>;
  if (smem > 40 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(kernel, dim3(a.max_splits, a.kv_heads, batch), dim3(kAttnThreads), smem, stream, a);
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
  a.max_splits = std::min(attn_max_splits(2 * sm_count(), batch, kv_heads), attn_merge_splits(q_heads / kv_heads, kAttnSlotsMax));
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
