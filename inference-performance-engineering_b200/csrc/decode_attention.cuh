// One work item of decode-step attention, shared by the standalone fused kernel and the persistent
// decode-step kernel: 128 threads (4 warps) handle one (32-key chunk, KV head, batch row).
//
// The item normalises (q_norm) and rotates this step's query heads of the group straight from the
// QKV projection output; the chunk that holds the current position also normalises / rotates the
// step's key and appends K and V to the cache. Scores, an fp32 softmax over the chunk and P.V go to
// a partial record; the last chunk of each (row, KV head) to arrive (an atomic counter it resets)
// merges all chunk records in chunk order, so the result does not depend on arrival order.
#pragma once

#include "common.cuh"

namespace ipe {

constexpr int kAttnChunk = 32;                       // keys per item
constexpr int kAttnThreads = 128;                    // threads per item
constexpr int kAttnRecord = 128 + 2;                 // floats per record: o[128], max, sum
constexpr float kAttnScale = 0.08838834764831845f;  // 128 ** -0.5
constexpr int kAttnBarrier = 2;                      // named barrier id used by an item

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
  bf16* out;       // [batch, q_heads * 128]
  float* records;  // [batch, q_heads, chunks_max, kAttnRecord]
  int* counters;   // [batch * kv_heads], zero between launches
  int q_heads, kv_heads, capacity, chunks_max;
  float eps;
  int* err;
};

// Shared-memory scratch of one item: floats, see attn_smem_floats.
template <int G>
struct AttnSmem {
  float* qs;      // [G][128]
  float* sc;      // [G][kAttnChunk]
  float* red;     // [8][G][128]
  float* stat;    // [G][2]
  float* weight;  // [G][chunks_max]
  int* last;
  __device__ AttnSmem(float* base, int chunks_max)
      : qs(base), sc(qs + G * 128), red(sc + G * kAttnChunk), stat(red + 8 * G * 128), weight(stat + 2 * G),
        last(reinterpret_cast<int*>(weight + G * chunks_max)) {}
};

template <int G>
__host__ __device__ constexpr int attn_smem_floats(int chunks_max) {
  return G * 128 + G * kAttnChunk + 8 * G * 128 + 2 * G + G * chunks_max + 4;
}

__device__ __forceinline__ void attn_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kAttnBarrier), "n"(kAttnThreads) : "memory");
}

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

// One item. tid in [0, 128). pos: this step's position (length = pos + 1); the caller skips
// chunks at or past the length. Every thread of the item must call it.
template <int G>
__device__ void attention_item(const FusedArgs& a, int chunk, int kvh, int b, int pos, const AttnSmem<G>& s, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int length = pos + 1;
  const int key0 = chunk * kAttnChunk;
  const int chunks = (length + kAttnChunk - 1) / kAttnChunk;
  const int slots = a.q_heads + 2 * a.kv_heads;
  const bf16* row = a.qkv + static_cast<int64_t>(b) * slots * 128;
  const int64_t head_base = (static_cast<int64_t>(b) * a.kv_heads + kvh) * a.capacity;

  // q heads of this group (warp w: heads w, w + 4), normalised and rotated.
  for (int gi = warp; gi < G; gi += kAttnThreads / 32) {
    const uint2 raw = ldcg8(row + (kvh * G + gi) * 128 + lane * 4);
    float x[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                  __uint_as_float(raw.y & 0xffff0000u)};
    norm_rope4(x, a.q_norm, a.cos_t, a.sin_t, pos, lane, a.eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) s.qs[gi * 128 + lane * 4 + i] = x[i];
  }
  // The chunk holding this step's position appends its K (normalised, rotated) and V rows.
  if (chunk == chunks - 1 && warp == (kAttnThreads / 32) - 1) {
    const uint2 kraw = ldcg8(row + (a.q_heads + kvh) * 128 + lane * 4);
    const uint2 vraw = ldcg8(row + (a.q_heads + a.kv_heads + kvh) * 128 + lane * 4);
    float x[4] = {__uint_as_float(kraw.x << 16), __uint_as_float(kraw.x & 0xffff0000u),
                  __uint_as_float(kraw.y << 16), __uint_as_float(kraw.y & 0xffff0000u)};
    norm_rope4(x, a.k_norm, a.cos_t, a.sin_t, pos, lane, a.eps);
    *reinterpret_cast<uint2*>(a.k_cache + (head_base + pos) * 128 + lane * 4) =
        make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    *reinterpret_cast<uint2*>(a.v_cache + (head_base + pos) * 128 + lane * 4) = vraw;
  }
  attn_sync();

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
          for (int i = 0; i < 8; ++i) dot[g] += f[i] * s.qs[g * 128 + part * 32 + v * 8 + i];
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 1);
      dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 2);
    }
    if (part == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) s.sc[g * kAttnChunk + kk] = key < length ? dot[g] * kAttnScale : -INFINITY;
    }
  }
  attn_sync();
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    const float sv = s.sc[g * kAttnChunk + lane];
    const float m = warp_max(sv);
    const float p = sv == -INFINITY ? 0.f : expf(sv - m);
    const float l = warp_sum(p);
    s.sc[g * kAttnChunk + lane] = p;
    if (lane == 0) {
      s.stat[2 * g] = m;
      s.stat[2 * g + 1] = l;
    }
  }
  attn_sync();
  {
    const int kg = tid >> 4, dc = tid & 15;
    float o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
#pragma unroll
    for (int j = 0; j < kAttnChunk / 8; ++j) {
      const int kk = kg + 8 * j;
      const int key = key0 + kk;
      if (key < length) {
        float f[8];
        unpack8(ldcg16(a.v_cache + (head_base + key) * 128 + dc * 8), f);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float p = s.sc[g * kAttnChunk + kk];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[g][i] += p * f[i];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) s.red[(kg * G + g) * 128 + dc * 8 + i] = o[g][i];
  }
  attn_sync();
  for (int i = tid; i < G * 128; i += kAttnThreads) {
    const int g = i / 128, d = i % 128;
    float sum = 0.f;
#pragma unroll
    for (int kg = 0; kg < 8; ++kg) sum += s.red[(kg * G + g) * 128 + d];
    float* rec =
        a.records + ((static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * a.chunks_max + chunk) * kAttnRecord;
    __stcg(rec + d, sum);
    if (d == 0) {
      __stcg(rec + 128, s.stat[2 * g]);
      __stcg(rec + 129, s.stat[2 * g + 1]);
    }
  }
  // Arrival: the last chunk of this (row, KV head) merges every chunk.
  __threadfence();
  attn_sync();
  if (tid == 0) {
    int* counter = a.counters + b * a.kv_heads + kvh;
    const int prior = atomicAdd(counter, 1);
    *s.last = prior == chunks - 1;
    if (*s.last) *counter = 0;
  }
  attn_sync();
  if (!*s.last) return;
  __threadfence();
  // Per head: lanes compute the chunk weights exp(m_c - M) / L, then every thread sums its dims.
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    const float* base = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * a.chunks_max * kAttnRecord;
    float m = -INFINITY;
    for (int c = lane; c < chunks; c += 32) m = fmaxf(m, __ldcg(base + c * kAttnRecord + 128));
    m = warp_max(m);
    float l = 0.f;
    for (int c = lane; c < chunks; c += 32) {
      const float e = expf(__ldcg(base + c * kAttnRecord + 128) - m);
      l += __ldcg(base + c * kAttnRecord + 129) * e;
      s.weight[g * a.chunks_max + c] = e;
    }
    l = warp_sum(l);
    for (int c = lane; c < chunks; c += 32) s.weight[g * a.chunks_max + c] /= l;
  }
  attn_sync();
  for (int i = tid; i < G * 128; i += kAttnThreads) {
    const int g = i / 128, d = i % 128;
    const float* base = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * a.chunks_max * kAttnRecord;
    const float* wg = s.weight + g * a.chunks_max;
    float o = 0.f;
    for (int c = 0; c < chunks; ++c) o += wg[c] * __ldcg(base + c * kAttnRecord + d);
    a.out[(static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * 128 + d] = __float2bfloat16_rn(o);
  }
  attn_sync();  // the item's shared scratch may be reused right after
}

}  // namespace ipe
