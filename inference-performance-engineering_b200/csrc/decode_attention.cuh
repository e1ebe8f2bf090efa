// One work item of decode-step attention, shared by the standalone fused kernel and the persistent
// decode-step kernel: 128 threads (4 warps) handle one (KV-head, batch row, split) triple, a split
// being `span` consecutive keys (a multiple of 32) of the positions 0 .. pos.
//
// The item normalises (q_norm) and rotates this step's query heads of the group straight from the
// QKV projection output; the split that holds the current position also normalises / rotates the
// step's key and appends K and V to the cache (its own scores read the new key from shared
// memory). Keys stream in 32-key sub-chunks whose K and V rows are loaded one sub-chunk ahead into
// registers; an fp32 online softmax carries the running max and sum across sub-chunks. A single
// split writes the output directly; with several, each writes a partial record (unnormalised o,
// max, sum) and the last split of each (row, KV head) to arrive (an atomic counter it resets)
// merges all records in split order, so the result does not depend on arrival order.
#pragma once

#include "common.cuh"

namespace ipe {

constexpr int kAttnChunk = 32;                       // keys per sub-chunk
constexpr int kAttnThreads = 128;                    // threads per item
constexpr int kAttnRecord = 128 + 2;                 // floats per record: o[128], max, sum
constexpr int kAttnSplitsMax = 32;                   // splits per (row, KV head) at most
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
  float* records;  // [batch, q_heads, kAttnSplitsMax, kAttnRecord]
  int* counters;   // [batch * kv_heads], zero between launches
  int q_heads, kv_heads, capacity, max_splits;
  float eps;
  int* err;
  uint64_t* trace;  // nullable: this item's milestones go to trace[0] (q ready, first K / V requested) and trace[1] (P.V done)
};

// How the keys 0 .. pos are split: `splits` spans of `span` keys (the last one shorter).
struct AttnSplit {
  int splits, span;
};

__host__ __device__ inline AttnSplit attn_split(int pos, int max_splits) {
  const int chunks = pos / kAttnChunk + 1;
  const int per = (chunks + max_splits - 1) / max_splits;  // sub-chunks per split
  return {(chunks + per - 1) / per, per * kAttnChunk};
}

// Splits per (row, KV head) so that batch * kv_heads * splits items about fill `ctas` CTAs.
__host__ __device__ inline int attn_max_splits(int ctas, int batch, int kv_heads) {
  const int s = ctas / (batch * kv_heads);
  return s < 1 ? 1 : (s > kAttnSplitsMax ? kAttnSplitsMax : s);
}

// Shared-memory scratch of one item: floats, see attn_smem_floats.
template <int G>
struct AttnSmem {
  float* qs;      // [G][128]
  float* sc;      // [2][G][kAttnChunk]
  float* red;     // [8][G][128]
  float* stat;    // [G][2] running max, sum
  float* alpha;   // [G] rescale of this sub-chunk
  float* knew;    // [128] this step's key (normalised, rotated, bf16 values)
  float* vnew;    // [128] this step's value
  float* weight;  // [G][kAttnSplitsMax]
  int* last;
  __device__ explicit AttnSmem(float* base)
      : qs(base), sc(qs + G * 128), red(sc + 2 * G * kAttnChunk), stat(red + 8 * G * 128), alpha(stat + 2 * G),
        knew(alpha + G), vnew(knew + 128), weight(vnew + 128),
        last(reinterpret_cast<int*>(weight + G * kAttnSplitsMax)) {}
};

template <int G>
__host__ __device__ constexpr int attn_smem_floats() {
  return G * 128 + 2 * G * kAttnChunk + 8 * G * 128 + 3 * G + 256 + G * kAttnSplitsMax + 4;
}

__device__ __forceinline__ void attn_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kAttnBarrier), "n"(kAttnThreads) : "memory");
}

__device__ __forceinline__ void unpack4(uint2 raw, float (&x)[4]) {
  x[0] = __uint_as_float(raw.x << 16);
  x[1] = __uint_as_float(raw.x & 0xffff0000u);
  x[2] = __uint_as_float(raw.y << 16);
  x[3] = __uint_as_float(raw.y & 0xffff0000u);
}

// RMSNorm over the 128-wide head held 4 elements per lane, then split-half RoPE with this lane's
// cos / sin values (reference rounding: bf16 normalised value, bf16 weight product, bf16 x*cos,
// rot*sin and sum).
__device__ __forceinline__ void norm_rope4(float (&x)[4], const bf16* w, const float (&c)[4], const float (&s)[4],
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
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float rot = d0 < 64 ? -p[i] : p[i];
    x[i] = bf16_round(bf16_round(h[i] * c[i]) + bf16_round(rot * s[i]));
  }
}

// K rows for the score layout (key c0 + 8 warp + lane/4, dims 32 (lane%4) ..) and V rows for the
// P.V layout (keys c0 + tid/16 + 8j, dims 8 (tid%16) ..) of the sub-chunk at c0. Keys at or past
// `end` and the key at `pos` (not yet in the cache) are not loaded.
__device__ __forceinline__ void load_kv(const bf16* k_head, const bf16* v_head, int c0, int end, int pos, int tid,
                                        uint4 (&kr)[4], uint4 (&vr)[4]) {
  const int warp = tid >> 5, lane = tid & 31;
  const int key = c0 + warp * 8 + (lane >> 2);
  const bool kin = key < end && key != pos;
#pragma unroll
  for (int v = 0; v < 4; ++v)
    kr[v] = kin ? ldcg16(k_head + static_cast<int64_t>(key) * 128 + (lane & 3) * 32 + v * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int kv = c0 + (tid >> 4) + 8 * j;
    vr[j] = kv < end && kv != pos ? ldcg16(v_head + static_cast<int64_t>(kv) * 128 + (tid & 15) * 8)
                                  : make_uint4(0, 0, 0, 0);
  }
}

// One item. tid in [0, 128). pos: this step's position (length = pos + 1); sp from attn_split;
// split < sp.splits. Every thread of the item must call it.
template <int G>
__device__ void attention_item(const FusedArgs& a, int split, int kvh, int b, int pos, AttnSplit sp,
                               const AttnSmem<G>& s, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int begin = split * sp.span;
  const int end = min(begin + sp.span, pos + 1);
  const int slots = a.q_heads + 2 * a.kv_heads;
  const bf16* row = a.qkv + static_cast<int64_t>(b) * slots * 128;
  const int64_t head_base = (static_cast<int64_t>(b) * a.kv_heads + kvh) * a.capacity;
  const bf16* k_head = a.k_cache + head_base * 128;
  const bf16* v_head = a.v_cache + head_base * 128;
  const bool appends = end == pos + 1;

  // Everything this item reads first, issued together: q (and, appending, k / v) rows, this
  // position's cos / sin, and the first sub-chunk of K and V.
  uint2 qraw[(G + 3) / 4];
#pragma unroll
  for (int i = 0; i < (G + 3) / 4; ++i) {
    const int gi = warp + 4 * i;
    qraw[i] = gi < G ? ldcg8(row + (kvh * G + gi) * 128 + lane * 4) : make_uint2(0, 0);
  }
  const bool append_warp = appends && warp == 3;
  const uint2 kraw = append_warp ? ldcg8(row + (a.q_heads + kvh) * 128 + lane * 4) : make_uint2(0, 0);
  const uint2 vraw = append_warp ? ldcg8(row + (a.q_heads + a.kv_heads + kvh) * 128 + lane * 4) : make_uint2(0, 0);
  float cs[4], sn[4];
  unpack4(*reinterpret_cast<const uint2*>(a.cos_t + static_cast<int64_t>(pos) * 128 + lane * 4), cs);
  unpack4(*reinterpret_cast<const uint2*>(a.sin_t + static_cast<int64_t>(pos) * 128 + lane * 4), sn);
  uint4 kr[4], vr[4];
  load_kv(k_head, v_head, begin, end, pos, tid, kr, vr);

#pragma unroll
  for (int i = 0; i < (G + 3) / 4; ++i) {
    const int gi = warp + 4 * i;
    if (gi >= G) continue;
    float x[4];
    unpack4(qraw[i], x);
    norm_rope4(x, a.q_norm, cs, sn, lane, a.eps);
#pragma unroll
    for (int e = 0; e < 4; ++e) s.qs[gi * 128 + lane * 4 + e] = x[e];
  }
  if (append_warp) {
    float x[4], v[4];
    unpack4(kraw, x);
    unpack4(vraw, v);
    norm_rope4(x, a.k_norm, cs, sn, lane, a.eps);
    *reinterpret_cast<uint2*>(a.k_cache + (head_base + pos) * 128 + lane * 4) =
        make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    *reinterpret_cast<uint2*>(a.v_cache + (head_base + pos) * 128 + lane * 4) = vraw;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s.knew[lane * 4 + e] = x[e];  // already bf16 values
      s.vnew[lane * 4 + e] = v[e];
    }
  }
  if (tid < G) {
    s.stat[2 * tid] = -INFINITY;
    s.stat[2 * tid + 1] = 0.f;
  }
  attn_sync();
  if (a.trace && tid == 0) a.trace[0] = globaltimer_ns();

  const int kg = tid >> 4, dc = tid & 15;
  float o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) o[g][i] = 0.f;

  int buf = 0;
  for (int c0 = begin; c0 < end; c0 += kAttnChunk, buf ^= 1) {
    uint4 kn[4], vn[4];
    if (c0 + kAttnChunk < end) load_kv(k_head, v_head, c0 + kAttnChunk, end, pos, tid, kn, vn);
    float* sc = s.sc + buf * G * kAttnChunk;
    // Scores: 4 lanes per key, 32 dims per lane.
    {
      const int kk = warp * 8 + (lane >> 2);
      const int part = lane & 3;
      const int key = c0 + kk;
      float dot[G];
#pragma unroll
      for (int g = 0; g < G; ++g) dot[g] = 0.f;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        float f[8];
        if (key == pos) {
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = s.knew[part * 32 + v * 8 + i];
        } else {
          unpack8(kr[v], f);
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < 8; ++i) dot[g] += f[i] * s.qs[g * 128 + part * 32 + v * 8 + i];
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 1);
        dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 2);
      }
      if (part == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g * kAttnChunk + kk] = key < end ? dot[g] * kAttnScale : -INFINITY;
      }
    }
    attn_sync();
    // Online softmax per head: running max / sum, this sub-chunk's probabilities and rescale.
    for (int g = warp; g < G; g += kAttnThreads / 32) {
      const float sv = sc[g * kAttnChunk + lane];
      const float m_old = s.stat[2 * g];
      const float m = fmaxf(m_old, warp_max(sv));
      const float p = sv == -INFINITY ? 0.f : expf(sv - m);
      const float l = warp_sum(p);
      sc[g * kAttnChunk + lane] = p;
      if (lane == 0) {
        const float al = m_old == -INFINITY ? 0.f : expf(m_old - m);
        s.alpha[g] = al;
        s.stat[2 * g] = m;
        s.stat[2 * g + 1] = s.stat[2 * g + 1] * al + l;
      }
    }
    attn_sync();
    // P.V: thread (key group kg, dims 8 dc ..), keys kg + 8j.
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float al = s.alpha[g];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[g][i] *= al;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = kg + 8 * j;
      const int key = c0 + kk;
      float f[8];
      if (key == pos) {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = s.vnew[dc * 8 + i];
      } else {
        unpack8(vr[j], f);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = sc[g * kAttnChunk + kk];  // 0 past the end
#pragma unroll
        for (int i = 0; i < 8; ++i) o[g][i] += p * f[i];
      }
    }
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      kr[v] = kn[v];
      vr[v] = vn[v];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) s.red[(kg * G + g) * 128 + dc * 8 + i] = o[g][i];
  attn_sync();
  if (a.trace && tid == 0) a.trace[1] = globaltimer_ns();

  if (sp.splits == 1) {
    for (int i = tid; i < G * 128; i += kAttnThreads) {
      const int g = i / 128, d = i % 128;
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) sum += s.red[(k * G + g) * 128 + d];
      a.out[(static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * 128 + d] =
          __float2bfloat16_rn(sum / s.stat[2 * g + 1]);
    }
    attn_sync();  // the item's shared scratch may be reused right after
    return;
  }
  for (int i = tid; i < G * 128; i += kAttnThreads) {
    const int g = i / 128, d = i % 128;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += s.red[(k * G + g) * 128 + d];
    float* rec =
        a.records + ((static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * kAttnSplitsMax + split) * kAttnRecord;
    __stcg(rec + d, sum);
    if (d == 0) {
      __stcg(rec + 128, s.stat[2 * g]);
      __stcg(rec + 129, s.stat[2 * g + 1]);
    }
  }
  // Arrival: the last split of this (row, KV head) merges every split. The records written by
  // every thread are ordered before thread 0's acq_rel fence by the barrier (release); the last
  // arriver's fence after its counter update orders the merge's reads after it (acquire), and the
  // barrier passes that on to the other threads.
  attn_sync();
  if (tid == 0) {
    int* counter = a.counters + b * a.kv_heads + kvh;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    const int prior = atomicAdd(counter, 1);
    *s.last = prior == sp.splits - 1;
    if (*s.last) {
      *counter = 0;
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
  }
  attn_sync();
  if (!*s.last) return;
  // Per head (one lane per split): weights exp(m_s - M) / L, then every thread sums its dims.
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    const float* base = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * kAttnSplitsMax * kAttnRecord;
    const bool in = lane < sp.splits;
    const float ms = in ? __ldcg(base + lane * kAttnRecord + 128) : -INFINITY;
    const float ls = in ? __ldcg(base + lane * kAttnRecord + 129) : 0.f;
    const float m = warp_max(ms);
    const float e = in ? expf(ms - m) : 0.f;
    const float l = warp_sum(ls * e);
    s.weight[g * kAttnSplitsMax + lane] = e / l;
  }
  attn_sync();
  for (int i = tid; i < G * 128; i += kAttnThreads) {
    const int g = i / 128, d = i % 128;
    const float* base = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * kAttnSplitsMax * kAttnRecord;
    const float* wg = s.weight + g * kAttnSplitsMax;
    float acc = 0.f;
    for (int c0 = 0; c0 < sp.splits; c0 += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = c0 + u < sp.splits ? __ldcg(base + (c0 + u) * kAttnRecord + d) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u < sp.splits) acc += wg[c0 + u] * v[u];
    }
    a.out[(static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * 128 + d] = __float2bfloat16_rn(acc);
  }
  attn_sync();  // the item's shared scratch may be reused right after
}

}  // namespace ipe
