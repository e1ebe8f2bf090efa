// One work item of decode-step attention, shared by the standalone fused kernel and the persistent
// decode-step kernel: 128 threads (4 warps) handle one (KV-head, batch row, split) triple, a split
// being `span` consecutive keys (a multiple of 32) of the positions 0 .. pos.
//
// The item normalises (q_norm) and rotates this step's query heads of the group straight from the
// QKV projection output; the split that holds the current position also normalises / rotates the
// step's key and appends K and V to the cache, and writes them into its last sub-chunk's rows.
// Keys stream in 32-key sub-chunks: every thread copies its share of each sub-chunk's K and V rows
// (16 KB, 16-byte cp.async into XOR-swizzled 256-byte rows) into a ring of up to kAttnSlotsMax
// shared-memory slots, all of them in flight from the item's start. Both products run on the
// tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate, the G query heads as the 8-wide N):
// scores S = K q^T from ldmatrix fragments of the key rows; P.V as O^T = V^T P^T from transposed
// ldmatrix fragments of the value rows, with P split into two bf16 terms (high part and the
// remainder) so its fp32 value carries over to about 16 significant bits. An fp32 online softmax
// carries the running max and sum across sub-chunks. A single split writes the output directly;
// with several, each writes a partial record (unnormalised o, max, sum) and the last split of each
// (row, KV head) to arrive (an atomic counter it resets) copies every split's record into the free
// ring in one bulk copy per head and merges them in split order, so the result does not depend on
// arrival order.
#pragma once

#include "common.cuh"

namespace ipe {

constexpr int kAttnChunk = 32;                       // keys per sub-chunk
constexpr int kAttnThreads = 128;                    // threads per item
constexpr int kAttnRecord = 128 + 4;                 // floats per record: o[128], max, sum, 2 unused (528 bytes)
constexpr int kAttnSlotBytes = 2 * kAttnChunk * 128 * 2;  // one ring slot: a sub-chunk's K rows, then its V rows
constexpr int kAttnSlotsMax = 4;                      // ring slots at most
constexpr int kAttnSlotsMin = 2;  // at least: a slot is refilled one sub-chunk after it was read
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
  uint64_t wait_ns;  // bound of every mbarrier wait (0: kWaitLimitNs)
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

// Splits a merge can take: every split's record of the G heads fits in the ring of `slots` slots.
__host__ __device__ constexpr int attn_merge_splits(int group, int slots) {
  return slots * kAttnSlotBytes / (group * kAttnRecord * 4) < kAttnSplitsMax
             ? slots * kAttnSlotBytes / (group * kAttnRecord * 4)
             : kAttnSplitsMax;
}

// Shared-memory scratch of one item (16-byte aligned base): the ring, then floats, see
// attn_smem_floats. The ring's mbarriers live outside the scratch (the scratch is shared with
// other phases of the decode-step kernel): `bars` holds kAttnSlotsMax + 1 of them, one per slot
// (an arrival per thread of the item and fill) and one for the merge's bulk copies (attn_ring_init).
// A slot holds a sub-chunk's 32 K rows, then its 32 V rows, 256 bytes each; the 16-byte chunk c of
// row r sits at chunk c ^ (r & 7) (ring_offset), so the 8 rows one ldmatrix matrix reads at the
// same columns fall in 8 different bank groups.
template <int G>
struct AttnSmem {
  unsigned char* ring;  // [slots][2][kAttnChunk][256 bytes]
  float* qs;            // [G][128]
  float* sc;            // [2][G][kAttnChunk]
  float* stat;          // [G][2] running max, sum
  float* alpha;         // [G] rescale of this sub-chunk
  float* weight;        // [G][kAttnSplitsMax]
  int* last;
  uint64_t* bars;
  int slots;
  __device__ AttnSmem(float* base, uint64_t* bars_, int slots_)
      : ring(reinterpret_cast<unsigned char*>(base)), qs(base + slots_ * (kAttnSlotBytes / 4)), sc(qs + G * 128),
        stat(sc + 2 * G * kAttnChunk), alpha(stat + 2 * G), weight(alpha + G),
        last(reinterpret_cast<int*>(weight + G * kAttnSplitsMax)),
        bars(bars_), slots(slots_) {}
};

template <int G>
__host__ __device__ constexpr int attn_smem_floats(int slots) {
  return slots * (kAttnSlotBytes / 4) + G * 128 + 2 * G * kAttnChunk + 3 * G + G * kAttnSplitsMax + 4;
}

// Ring fills and merges of this CTA so far: the parities of the next waits. Every thread of the
// item keeps its own copy, updated identically.
struct AttnSeq {
  uint32_t fills = 0, merges = 0;
};

// Thread 0 initialises the ring's mbarriers; the caller then orders the initialisation before use
// (fence_barrier_init and a CTA barrier).
__device__ __forceinline__ void attn_ring_init(uint64_t* bars) {
  for (int i = 0; i < kAttnSlotsMax; ++i) mbar_init(&bars[i], kAttnThreads);
  mbar_init(&bars[kAttnSlotsMax], 1);
}

// Byte offset of 16-byte chunk c (0..15) of row r in one half (K or V) of a ring slot.
__device__ __forceinline__ uint32_t ring_offset(int r, int c) {
  return static_cast<uint32_t>(r * 256 + ((c ^ (r & 7)) << 4));
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

// One item. tid in [0, 128). pos: this step's position (length = pos + 1); sp from attn_split with
// sp.splits <= attn_merge_splits(G, s.slots); split < sp.splits; s.slots >= kAttnSlotsMin (slot
// (i - 1) % slots is refilled with sub-chunk i - 1 + slots after the scores of sub-chunk i, so
// sub-chunk i was issued before anyone waits for it only with two slots or more). Every thread of
// the item must call it, with the same seq. The K / V caches must be 16-byte aligned.
template <int G>
__device__ void attention_item(const FusedArgs& a, int split, int kvh, int b, int pos, AttnSplit sp,
                               const AttnSmem<G>& s, AttnSeq& seq, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int begin = split * sp.span;
  const int end = min(begin + sp.span, pos + 1);
  const int slots = a.q_heads + 2 * a.kv_heads;
  const bf16* row = a.qkv + static_cast<int64_t>(b) * slots * 128;
  const int64_t head_base = (static_cast<int64_t>(b) * a.kv_heads + kvh) * a.capacity;
  const bf16* k_head = a.k_cache + head_base * 128;
  const bf16* v_head = a.v_cache + head_base * 128;
  const bool appends = end == pos + 1;
  const uint64_t wait_ns = a.wait_ns ? a.wait_ns : kWaitLimitNs;
  if (s.slots < kAttnSlotsMin || sp.splits > attn_merge_splits(G, s.slots) ||
      ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 15u)) {
    // host checks keep this from happening (the decode step's caches come from device descriptors)
    if (tid == 0) report(a.err, kErrShape);
    return;
  }

  // The K / V ring: sub-chunk i of the split (keys begin + 32 i ..) goes to slot (fills + i) % slots,
  // each thread copying 8 of its 1024 16-byte chunks and arriving on the slot's barrier once they
  // have landed. Keys not yet in the cache (past the split, or the appended key) are zero-filled
  // without a read; the appending warp writes the appended key's and value's row before its scores.
  const int nsub = (end - begin + kAttnChunk - 1) / kAttnChunk;
  const int cached_end = appends ? pos : end;
  const uint32_t ring = smem_addr(s.ring);
  auto issue = [&](int i) {  // every thread
    const uint32_t n = seq.fills + static_cast<uint32_t>(i);
    const uint32_t slot = n % static_cast<uint32_t>(s.slots);
    const int c0 = begin + i * kAttnChunk;
    const uint32_t kdst = ring + slot * kAttnSlotBytes;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = tid + kAttnThreads * u;  // row idx / 16, chunk idx % 16
      const int r = idx >> 4, c = idx & 15;
      const bool in = c0 + r < cached_end;
      const int64_t src = (in ? static_cast<int64_t>(c0 + r) : 0) * 128 + c * 8;
      cp_async16(kdst + ring_offset(r, c), k_head + src, in ? 16u : 0u);
      cp_async16(kdst + kAttnSlotBytes / 2 + ring_offset(r, c), v_head + src, in ? 16u : 0u);
    }
    cp_async_mbar_arrive(&s.bars[slot]);
  };
  for (int i = 0; i < min(s.slots, nsub); ++i) issue(i);

  // Everything else this item reads first, issued together: q (and, appending, k / v) rows and
  // this position's cos / sin.
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
  uint2 knew_raw = make_uint2(0, 0);  // the appended key's 4 dims of this lane (bf16)
  if (append_warp) {
    float x[4];
    unpack4(kraw, x);
    norm_rope4(x, a.k_norm, cs, sn, lane, a.eps);
    knew_raw = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    *reinterpret_cast<uint2*>(a.k_cache + (head_base + pos) * 128 + lane * 4) = knew_raw;
    *reinterpret_cast<uint2*>(a.v_cache + (head_base + pos) * 128 + lane * 4) = vraw;
  }
  if (tid < G) {
    s.stat[2 * tid] = -INFINITY;
    s.stat[2 * tid + 1] = 0.f;
  }
  attn_sync();
  if (a.trace && tid == 0) a.trace[0] = globaltimer_ns();

  // MMA lane roles: g = lane / 4 (a row of the A fragment, a column of B), t = lane % 4.
  const int g = lane >> 2, t = lane & 3;
  // q^T as the B operand of the scores (k = dims, n = heads): head g's dims 16 s + 2t (+1, +8, +9).
  uint32_t qf[8][2];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const float* q = s.qs + g * 128 + ks * 16 + 2 * t;
    qf[ks][0] = g < G ? pack_bf16x2(q[0], q[1]) : 0u;  // bf16 values already: packing is exact
    qf[ks][1] = g < G ? pack_bf16x2(q[8], q[9]) : 0u;
  }
  // O^T accumulators: dims 32 warp + 16 mt + g (+8), heads 2t, 2t + 1.
  float o[2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  for (int i = 0; i < nsub; ++i) {
    const int c0 = begin + i * kAttnChunk;
    const uint32_t n = seq.fills + static_cast<uint32_t>(i);
    const uint32_t slot = n % static_cast<uint32_t>(s.slots);
    mbar_wait(&s.bars[slot], (n / static_cast<uint32_t>(s.slots)) & 1u, a.err, wait_ns);
    const uint32_t kb = ring + slot * kAttnSlotBytes;
    const uint32_t vb = kb + kAttnSlotBytes / 2;
    float* sc = s.sc + (i & 1) * G * kAttnChunk;
    if (appends && i == nsub - 1) {  // the appended key and value into their (zero-filled) rows
      if (append_warp) {
        const int r = pos - c0;
        const uint32_t off = ring_offset(r, lane >> 1) + (lane & 1) * 8;
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(kb + off), "r"(knew_raw.x), "r"(knew_raw.y) : "memory");
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(vb + off), "r"(vraw.x), "r"(vraw.y) : "memory");
      }
      attn_sync();
    }
    // Scores: warp w < 2 takes keys 16 w .. 16 w + 15 (the MMA's M) over the 128 dims (8 k-steps).
    if (warp < 2) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      const int lr = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(a0, a1, a2, a3, kb + ring_offset(lr, 2 * ks + (lane >> 4)));
        mma16816(d, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
      }
      // d: keys 16 w + g (+8), heads 2t, 2t + 1
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kk = 16 * warp + g + 8 * (e >> 1), head = 2 * t + (e & 1);
        if (head < G) sc[head * kAttnChunk + kk] = c0 + kk < end ? d[e] * kAttnScale : -INFINITY;
      }
    }
    attn_sync();
    // every thread is past its P.V reads of sub-chunk i - 1: its slot takes sub-chunk i - 1 + slots
    if (i >= 1 && i - 1 + s.slots < nsub) issue(i - 1 + s.slots);
    // Online softmax per head: running max / sum, this sub-chunk's probabilities and rescale.
    for (int h = warp; h < G; h += kAttnThreads / 32) {
      const float sv = sc[h * kAttnChunk + lane];
      const float m_old = s.stat[2 * h];
      const float m = fmaxf(m_old, warp_max(sv));
      const float p = sv == -INFINITY ? 0.f : expf(sv - m);
      const float l = warp_sum(p);
      sc[h * kAttnChunk + lane] = p;
      if (lane == 0) {
        const float al = m_old == -INFINITY ? 0.f : expf(m_old - m);
        s.alpha[h] = al;
        s.stat[2 * h] = m;
        s.stat[2 * h + 1] = s.stat[2 * h + 1] * al + l;
      }
    }
    attn_sync();
    // P.V as O^T += V^T P^T: warp w takes dims 32 w .. 32 w + 31 (two M tiles), the 32 keys as two
    // k-steps; P^T (k = keys, n = heads) as a high and a low bf16 part.
    {
      const float al0 = 2 * t < G ? s.alpha[2 * t] : 0.f;
      const float al1 = 2 * t + 1 < G ? s.alpha[2 * t + 1] : 0.f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
        float pv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pv[e] = g < G ? sc[g * kAttnChunk + 16 * kt + 2 * t + (e & 1) + 8 * (e >> 1)] : 0.f;
        float hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hi[e] = bf16_round(pv[e]);
          lo[e] = pv[e] - hi[e];
        }
        const uint32_t bh0 = pack_bf16x2(hi[0], hi[1]), bh1 = pack_bf16x2(hi[2], hi[3]);
        const uint32_t bl0 = pack_bf16x2(lo[0], lo[1]), bl1 = pack_bf16x2(lo[2], lo[3]);
        // V^T fragments: matrix j of ldmatrix = value rows 16 kt + 8 (j / 2) .., dims 16 m + 8 (j % 2) ..
        const int vr = 16 * kt + (lane & 7) + 8 * (lane >> 4);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(a0, a1, a2, a3, vb + ring_offset(vr, 2 * (2 * warp + mt) + ((lane >> 3) & 1)));
          mma16816(o[mt], a0, a1, a2, a3, bh0, bh1);
          mma16816(o[mt], a0, a1, a2, a3, bl0, bl1);
        }
      }
    }
  }
  seq.fills += static_cast<uint32_t>(nsub);
  if (a.trace && tid == 0) a.trace[1] = globaltimer_ns();

  // o[mt][e]: dim 32 warp + 16 mt + g + 8 (e >> 1), head 2t + (e & 1) (heads past G hold zeros).
  if (sp.splits == 1) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 32 * warp + 16 * mt + g + 8 * (e >> 1), head = 2 * t + (e & 1);
        if (head < G)
          a.out[(static_cast<int64_t>(b) * a.q_heads + kvh * G + head) * 128 + d] =
              __float2bfloat16_rn(o[mt][e] / s.stat[2 * head + 1]);
      }
    attn_sync();  // the item's shared scratch may be reused right after
    return;
  }
  {
    float* rec0 = a.records + ((static_cast<int64_t>(b) * a.q_heads + kvh * G) * kAttnSplitsMax + split) * kAttnRecord;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 32 * warp + 16 * mt + g + 8 * (e >> 1), head = 2 * t + (e & 1);
        if (head < G) __stcg(rec0 + static_cast<int64_t>(head) * kAttnSplitsMax * kAttnRecord + d, o[mt][e]);
      }
    if (tid < G) {
      __stcg(rec0 + static_cast<int64_t>(tid) * kAttnSplitsMax * kAttnRecord + 128, s.stat[2 * tid]);
      __stcg(rec0 + static_cast<int64_t>(tid) * kAttnSplitsMax * kAttnRecord + 129, s.stat[2 * tid + 1]);
    }
  }
  // the merge's bulk copies (async proxy) may overwrite the ring this thread's copies filled
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  // Arrival: the last split of this (row, KV head) merges every split. The records written by
  // every thread are ordered before thread 0's acq_rel fence by the barrier (release); the last
  // arriver's fence after its counter update orders its reads after it (acquire), and the proxy
  // fence extends that to its bulk copies of the records into the ring (free again: every thread
  // is past its last P.V read).
  attn_sync();
  const int S = sp.splits;
  const uint32_t head_bytes = static_cast<uint32_t>(S) * kAttnRecord * 4u;
  const float* rec0 = a.records + (static_cast<int64_t>(b) * a.q_heads + kvh * G) * kAttnSplitsMax * kAttnRecord;
  if (tid == 0) {
    int* counter = a.counters + b * a.kv_heads + kvh;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    const int prior = atomicAdd(counter, 1);
    *s.last = prior == S - 1;
    if (*s.last) {
      *counter = 0;
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      asm volatile("fence.proxy.async.global;" ::: "memory");
      mbar_expect_tx(&s.bars[kAttnSlotsMax], static_cast<uint32_t>(G) * head_bytes);
      for (int g = 0; g < G; ++g)
        bulk_copy(ring + g * head_bytes, rec0 + static_cast<int64_t>(g) * kAttnSplitsMax * kAttnRecord, head_bytes,
                  &s.bars[kAttnSlotsMax]);
    }
  }
  attn_sync();
  if (!*s.last) return;
  mbar_wait(&s.bars[kAttnSlotsMax], seq.merges & 1u, a.err, wait_ns);
  ++seq.merges;
  const float* R = reinterpret_cast<const float*>(s.ring);  // [G][S][kAttnRecord]
  // Per head (one lane per split): weights exp(m_s - M) / L, then every thread sums its dims.
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    const bool in = lane < S;
    const float ms = in ? R[(g * S + lane) * kAttnRecord + 128] : -INFINITY;
    const float ls = in ? R[(g * S + lane) * kAttnRecord + 129] : 0.f;
    const float m = warp_max(ms);
    const float e = in ? expf(ms - m) : 0.f;
    const float l = warp_sum(ls * e);
    s.weight[g * kAttnSplitsMax + lane] = e / l;
  }
  attn_sync();
  for (int i = tid; i < G * 128; i += kAttnThreads) {
    const int g = i / 128, d = i % 128;
    const float* wg = s.weight + g * kAttnSplitsMax;
    const float* rg = R + g * S * kAttnRecord + d;
    float acc = 0.f;
    for (int c = 0; c < S; ++c) acc += wg[c] * rg[c * kAttnRecord];
    a.out[(static_cast<int64_t>(b) * a.q_heads + kvh * G + g) * 128 + d] = __float2bfloat16_rn(acc);
  }
  attn_sync();  // the item's shared scratch may be reused right after
}

}  // namespace ipe
