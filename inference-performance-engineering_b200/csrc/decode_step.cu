// One whole decode step in one persistent kernel: embedding, every layer's QKV projection
// (RMSNorm fused), attention (q/k norm + RoPE + KV append + split-KV), o_proj + residual,
// RMSNorm + gate/up + SiLU*up, down_proj + residual, the final norm + tied LM head with fp32
// logits and sampling records, and (optionally) the sampled token fed back for the next step.
//
// Why one kernel: every weight byte of the step is known before the step starts, so the weight
// stream does not depend on activations. Each CTA (one per SM, cooperative launch) has a producer
// warp that walks its share of ALL phases' decode tiles back to back with bulk copies into
// per-consumer-warp shared-memory slots and never waits for a phase boundary; ahead of those
// copies it issues L2 prefetches of the same units, of the K / V rows its attention items will
// read, and of the norm weights. The 4 consumer warps wait only where the data requires it: at a
// bounded-spin grid barrier after each phase (the next phase needs the full activation vector),
// then they stage that vector in shared memory and consume tiles that are usually already there.
//
// Work split: a phase's units (a 32-row block, or a 16-row half block where that evens out the
// bytes per CTA, always over the whole K: no split-K) are dealt round-robin over the CTAs,
// continuing where the previous phase stopped; within a CTA a unit's tiles go round-robin to the
// consumer warps, whose partial sums are reduced in a fixed order through shared memory
// (deterministic). Attention runs as (split, KV head, row) items over the CTAs. Every spin (grid
// barrier, mbarrier) is bounded; a timeout sets the device error word and an abort flag and the
// kernel winds down.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "decode_attention.cuh"
#include "launch.h"
#include "sampling.cuh"
#include "stream_tile.cuh"
#include "tensor_map.h"

namespace ipe {
namespace {

constexpr int kConsumers = 4;
constexpr int kMaxSlotsPerWarp = 8;
constexpr int kMaxStages = kConsumers * kMaxSlotsPerWarp;  // 8 KB slots (bounded by shared memory)
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kCThreads = 32 * kConsumers;
constexpr int kPad = 32;
constexpr int kStepBarrier = 1;  // named barrier id of the consumer warps
constexpr size_t kSmemMax = 226 * 1024;  // dynamic shared memory; the rest holds static arrays

struct StepArgs {
  ipe_decode_step_desc d;
  unsigned* grid_bar;  // [0] arrivals, [1] abort flag
  int* attn_counters;
  float* attn_records;
  int* err;
  int slots;                // ring slots per consumer warp
  int max_splits;           // attention splits per (row, KV head)
  unsigned prefetch_bytes;  // how far the L2 prefetch runs ahead of the shared-memory copies
  int evict_first;          // weight copies mark their L2 lines evict-first
  int halves;               // half-row-block units allowed
  // tensor parallelism (d.tp_world > 1): byte offsets in a communication region
  size_t recv_x;            // [2 slots][world][batch][hidden] fp32 parts of o_proj / down_proj
  size_t recv_rec;          // [world][parts_max][batch][IPE_PARTIAL_WORDS] LM-head records
  int parts_max;            // LM-head records per rank (the largest shard's)
};

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kStepBarrier), "n"(kCThreads) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier among the consumer warps of all CTAs. Returns false when the step is aborted.
// trace (this CTA's row of the step trace, or null) receives the arrival and release times.
__device__ bool grid_sync(const StepArgs& a, unsigned index, int tid, int* abort_smem, uint64_t* trace) {
  consumers_sync();
  if (tid == 0) {
    if (trace) trace[1 + 5 * (index - 1)] = globaltimer_ns();
    __threadfence();
    atomicAdd(&a.grid_bar[0], 1u);
    const unsigned target = index * gridDim.x;
    uint64_t start = 0;
    for (unsigned i = 0;; ++i) {
      if (ld_acquire(&a.grid_bar[0]) >= target) break;
      if (ld_acquire(&a.grid_bar[1])) {
        *abort_smem = 1;
        break;
      }
      if ((i & 63u) == 63u) {
        const uint64_t now = globaltimer_ns();
        if (start == 0) start = now;
        else if (now - start > kWaitLimitNs) {
          report(a.err, kErrWaitTimeout);
          atomicExch(&a.grid_bar[1], 1u);
          *abort_smem = 1;
          break;
        }
      }
      __nanosleep(64);
    }
    __threadfence();
    if (trace) trace[2 + 5 * (index - 1)] = globaltimer_ns();
  }
  consumers_sync();
  return *abort_smem == 0;
}

// --------------------------------------------------------------------- tensor parallelism
// Communication region of a rank (see ipe_decode_step_comm_bytes): u32 flag[r] at byte 4 r (the
// last epoch rank r announced here), the epoch counter at byte 128, then the receive buffers.
constexpr size_t kTpFlags = 0;
constexpr size_t kTpCounter = 128;
constexpr size_t kTpRecv = 256;

__device__ __forceinline__ unsigned char* tp_region(const ipe_decode_step_desc& d, int r) {
  return reinterpret_cast<unsigned char*>(static_cast<const uint64_t*>(d.tp_peers)[r]);
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// A grid barrier that is also an exchange with the other ranks: every CTA makes its pushes to the
// peers visible and arrives; CTA 0, once all have arrived, announces `epoch` to every peer and
// waits (bounded) for every peer's announcement, then releases this GPU's CTAs. After it, every
// rank's pushes of the phase are in this rank's receive buffers. epoch matters in CTA 0 only.
__device__ bool grid_sync_tp(const StepArgs& a, unsigned index, int tid, int* abort_smem, unsigned epoch) {
  consumers_sync();
  if (tid == 0) {
    const ipe_decode_step_desc& d = a.d;
    __threadfence_system();
    atomicAdd(&a.grid_bar[0], 1u);
    bool ok = true;
    uint64_t start = 0;
    auto waiting = [&](unsigned i) {  // false once the step is aborted or the wait limit passed
      __nanosleep(32);
      if ((i & 63u) != 63u) return true;
      if (ld_acquire(&a.grid_bar[1])) return false;
      const uint64_t now = globaltimer_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitLimitNs) {
        report(a.err, kErrWaitTimeout);
        atomicExch(&a.grid_bar[1], 1u);
        return false;
      }
      return true;
    };
    if (blockIdx.x == 0) {
      const unsigned target = index * gridDim.x;
      for (unsigned i = 0; ok && ld_acquire(&a.grid_bar[0]) < target; ++i) ok = waiting(i);
      if (ok) {
        __threadfence_system();
        for (int r = 0; r < d.tp_world; ++r)
          if (r != d.tp_rank) st_release_sys(reinterpret_cast<unsigned*>(tp_region(d, r) + kTpFlags) + d.tp_rank, epoch);
        const unsigned* flags = reinterpret_cast<const unsigned*>(tp_region(d, d.tp_rank) + kTpFlags);
        for (int r = 0; r < d.tp_world && ok; ++r) {
          if (r == d.tp_rank) continue;
          for (unsigned i = 0; ok && static_cast<int>(ld_acquire_sys(flags + r) - epoch) < 0; ++i) ok = waiting(i);
        }
      }
      if (ok) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&a.grid_bar[2]), "r"(index) : "memory");
    } else {
      for (unsigned i = 0; ok && ld_acquire(&a.grid_bar[2]) < index; ++i) ok = waiting(i);
    }
    if (!ok) *abort_smem = 1;
    __threadfence();
  }
  consumers_sync();
  return *abort_smem == 0;
}

// First unit of this CTA in a phase that starts dealing at `cursor`.
__device__ __forceinline__ int first_unit(int cursor) {
  const int g = static_cast<int>(gridDim.x);
  return (static_cast<int>(blockIdx.x) - cursor % g + g) % g;
}

// A weight phase as units dealt round-robin over the CTAs: a unit is one row block (32 rows, whole
// K, 8 KB tiles) or, when that lowers the most bytes any CTA streams in the phase, one 16-row half
// of a row block (4 KB half tiles).
struct PhaseShape {
  const unsigned char* tiles;
  int units;
  int ku;  // tiles per unit
  bool half;
};

__device__ __forceinline__ PhaseShape make_phase(const void* tiles, int row_blocks, int ku, bool may_halve) {
  const int g = static_cast<int>(gridDim.x);
  const bool half = may_halve && (2 * row_blocks + g - 1) / g < 2 * ((row_blocks + g - 1) / g);
  return {static_cast<const unsigned char*>(tiles), half ? 2 * row_blocks : row_blocks, ku, half};
}

// Slot bookkeeping of one consumer warp's ring share: slot index and how often it wrapped.
struct SlotCursor {
  int slot = 0, fill = 0;
  __device__ __forceinline__ void advance(int slots) {
    if (++slot == slots) {
      slot = 0;
      ++fill;
    }
  }
};

// Position of a walk over this CTA's units of the step, in stream order.
struct UnitWalk {
  int layer = 0, kind = 0, cursor = 0, unit = 0;
  bool in_phase = false, done = false;
  PhaseShape ph{};
};

template <int NT, int G, bool ACT_SMEM>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const StepArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int S = a.slots;
  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kConsumers * S * kTileBytes);
  uint64_t* empty = full + kMaxStages;
  float* rstd = reinterpret_cast<float*>(empty + kMaxStages);  // [16]
  int* abort_smem = reinterpret_cast<int*>(rstd + 16);
  float* red = reinterpret_cast<float*>(abort_smem + 4);  // [kConsumers][32][8 * NT]
  float* scratch = red + kConsumers * 32 * 8 * NT;        // activations or attention scratch
  bf16* xs = reinterpret_cast<bf16*>(scratch);

  const ipe_decode_step_desc& d = a.d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = d.batch, H = d.hidden, I = d.intermediate;
  const int Q = d.q_heads * 128, QKV = (d.q_heads + 2 * d.kv_heads) * 128;
  const int G_ = static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kConsumers * S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_smem = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // kind: 0 QKV, 1 o_proj, 2 gate/up, 3 down_proj; layer == layers: the LM head.
  auto phase_shape = [&](int layer, int kind) -> PhaseShape {
    if (layer == d.layers) return make_phase(d.lm_head_tiles, (d.vocab + 31) / 32, H / kTileK, false);
    const ipe_layer_desc& L = d.layer_descs[layer];
    switch (kind) {
      case 0: return make_phase(L.qkv_tiles, QKV / 32, H / kTileK, a.halves != 0);
      case 1: return make_phase(L.o_tiles, H / 32, Q / kTileK, a.halves != 0);
      case 2: return make_phase(L.gate_up_tiles, I / 16, H / kTileK, false);
      default: return make_phase(L.down_tiles, H / 32, I / kTileK, a.halves != 0);
    }
  };

  // Next unit of a walk (w.ph and w.unit describe it); entered_layer is set to the layer whose QKV
  // phase the walk just entered (else -1).
  auto next_unit = [&](UnitWalk& w, int& entered_layer) -> bool {
    entered_layer = -1;
    while (!w.done) {
      if (!w.in_phase) {
        w.ph = phase_shape(w.layer, w.kind);
        w.unit = first_unit(w.cursor);
        w.in_phase = true;
        if (w.kind == 0 && w.layer < d.layers) entered_layer = w.layer;
      } else {
        w.unit += G_;
      }
      if (w.unit < w.ph.units) return true;
      w.cursor = (w.cursor + w.ph.units) % G_;
      w.in_phase = false;
      if (w.layer == d.layers) w.done = true;
      else if (++w.kind == 4) {
        w.kind = 0;
        ++w.layer;
      }
    }
    return false;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    // Bulk copies of this CTA's tiles into the consumer warps' ring slots (tile t of a unit to
    // warp t % 4), and, prefetch_bytes ahead of them, L2 prefetches of the same units plus the
    // K / V rows this CTA's attention items of each layer will read. The per-tile path is kept
    // short: one thread issues every copy of the SM.
    if (lane == 0) {
      const uint32_t ring_base = smem_addr(ring);
      const uint64_t policy = evict_first_policy();
      const int pos = static_cast<int>(d.state[IPE_STATE_POS]);
      if (pos < 0 || pos >= d.capacity) return;  // the consumers leave too; nothing was issued
      const AttnSplit sp = attn_split(pos, a.max_splits);
      auto prefetch_kv = [&](int layer) {
        const ipe_layer_desc& L = d.layer_descs[layer];
        // the layer's norm weights too (the stages that read them are on the critical path); a
        // bulk prefetch needs a 16-byte aligned start, so an unaligned vector is left to the loads
        auto prefetch_vec = [&](const void* p, uint32_t bytes) {
          if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) prefetch_l2(p, bytes);
        };
        prefetch_vec(L.input_layernorm, static_cast<uint32_t>(H) * 2u);
        prefetch_vec(L.post_attention_layernorm, static_cast<uint32_t>(H) * 2u);
        prefetch_vec(L.q_norm, 256u);
        prefetch_vec(L.k_norm, 256u);
        if (layer == d.layers - 1) prefetch_vec(d.final_norm, static_cast<uint32_t>(H) * 2u);
        const int items = sp.splits * d.kv_heads * B;
        for (int it = static_cast<int>(blockIdx.x); it < items; it += G_) {
          const int split = it % sp.splits, rest = it / sp.splits;  // rest = row * kv_heads + head
          const int begin = split * sp.span, end = min(begin + sp.span, pos + 1);
          const int64_t row0 = static_cast<int64_t>(rest) * d.capacity + begin;
          for (int k0 = 0; k0 < end - begin; k0 += 64) {  // 64 rows = 16 KB a prefetch
            const uint32_t bytes = static_cast<uint32_t>(min(64, end - begin - k0)) * 256u;
            prefetch_l2(static_cast<const bf16*>(L.k_cache) + (row0 + k0) * 128, bytes);
            prefetch_l2(static_cast<const bf16*>(L.v_cache) + (row0 + k0) * 128, bytes);
          }
        }
      };
      // A unit's tiles are one contiguous range of ku whole tiles (a half unit reads half of each).
      auto prefetch_unit = [&](const UnitWalk& w) {
        const int rb = w.ph.half ? w.unit >> 1 : w.unit;
        const unsigned char* base = w.ph.tiles + static_cast<int64_t>(rb) * w.ph.ku * kTileBytes;
        for (int t = 0; t < w.ph.ku; t += 8) {  // 8 tiles = 64 KB a prefetch
          const uint32_t bytes = static_cast<uint32_t>(min(8, w.ph.ku - t)) * kTileBytes;
          prefetch_l2(base + static_cast<int64_t>(t) * kTileBytes, bytes);
        }
      };
      UnitWalk main_walk, ahead;
      uint64_t issued = 0, prefetched = 0;
      SlotCursor sc[kConsumers];
      bool ok = true;
      int entered;
      while (ok && next_unit(main_walk, entered)) {
        const PhaseShape& ph = main_walk.ph;
        const uint32_t bytes = ph.half ? kTileBytes / 2 : kTileBytes;
        while (prefetched < issued + a.prefetch_bytes) {
          int player;
          if (!next_unit(ahead, player)) break;
          if (player >= 0) prefetch_kv(player);
          prefetch_unit(ahead);
          prefetched += static_cast<uint64_t>(ahead.ph.ku) * (ahead.ph.half ? kTileBytes / 2 : kTileBytes);
        }
        const int rb = ph.half ? main_walk.unit >> 1 : main_walk.unit;
        const unsigned char* src = ph.tiles + static_cast<int64_t>(rb) * ph.ku * kTileBytes +
                                   (ph.half ? (main_walk.unit & 1) * (kTileBytes / 2) : 0);
        for (int t0 = 0; t0 < ph.ku && ok; t0 += kConsumers) {
#pragma unroll
          for (int w = 0; w < kConsumers; ++w) {
            const int t = t0 + w;
            if (t >= ph.ku || !ok) continue;
            const int slot = w * S + sc[w].slot;
            if (sc[w].fill > 0 && !mbar_wait(&empty[slot], (sc[w].fill - 1) & 1, a.err)) {
              ok = false;
              continue;
            }
            mbar_expect_tx(&full[slot], bytes);
            if (a.evict_first)
              bulk_copy_hint(ring_base + slot * kTileBytes, src + static_cast<int64_t>(t) * kTileBytes, bytes,
                             &full[slot], policy);
            else
              bulk_copy(ring_base + slot * kTileBytes, src + static_cast<int64_t>(t) * kTileBytes, bytes,
                        &full[slot]);
            sc[w].advance(S);
          }
        }
        issued += static_cast<uint64_t>(ph.ku) * bytes;
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cw = warp - 1, tid = threadIdx.x - 32;
  const int g = lane >> 2, t = lane & 3;
  SlotCursor mine;
  int cursor = 0;
  unsigned barrier_index = 0;
  int64_t* state = d.state;
  uint64_t* trace = d.trace ? d.trace + static_cast<int64_t>(blockIdx.x) * IPE_TRACE_WORDS(d.layers) : nullptr;
  if (trace && tid == 0) trace[0] = globaltimer_ns();
  // trace word k (2: staged, 3: first tile ready, 4: last tile ready) of the current phase
  auto mark = [&](int k) {
    if (trace && tid == 0) trace[1 + 5 * (barrier_index - 1) + k] = globaltimer_ns();
  };
  // tensor parallelism: this rank's region, and the epoch of its exchanges (CTA 0, thread 0)
  const bool tp = d.tp_world > 1;
  unsigned char* my_region = tp ? tp_region(d, d.tp_rank) : nullptr;
  unsigned tp_epoch = (tp && blockIdx.x == 0 && tid == 0) ? *reinterpret_cast<const unsigned*>(my_region + kTpCounter) : 0u;
  const size_t x_part_bytes = static_cast<size_t>(B) * H * sizeof(float);
  const size_t rec_rank_bytes = static_cast<size_t>(a.parts_max) * B * IPE_PARTIAL_WORDS * sizeof(float);
  __shared__ float red_ss[4 * 16];  // tensor-parallel staging: [warp][row] sums of squares
  int tp_slot = 0;                  // receive slot of the current row-parallel phase

  // Embedding: x[b] = embed[tokens[b]] (out-of-range IDs give zeros and set device error 1).
  {
    const int vecs = H / 8;
    bf16* x = static_cast<bf16*>(d.x);
    for (int i = static_cast<int>(blockIdx.x) * kCThreads + tid; i < B * vecs; i += G_ * kCThreads) {
      const int b = i / vecs, v = i % vecs;
      const int64_t id = d.tokens[b];
      uint4 val = make_uint4(0, 0, 0, 0);
      if (id >= 0 && id < (d.vocab_total > 0 ? d.vocab_total : d.vocab))
        val = ldg16(static_cast<const bf16*>(d.embed) + id * H + v * 8);
      else if (v == 0) report(a.err, kErrTokenRange);
      *reinterpret_cast<uint4*>(x + static_cast<int64_t>(b) * H + v * 8) = val;
    }
  }
  if (!grid_sync(a, ++barrier_index, tid, abort_smem, trace)) return;

  // Stage the activation rows of a phase (optionally RMS-normalised) in shared memory; without
  // shared staging only the RMS scales are kept and tiles read activations from global memory.
  auto stage = [&](const bf16* src, const bf16* norm_w, int K) {
    stage_rows(src, K, norm_w, d.eps, B, K, xs, K + kPad, rstd, cw, kConsumers, lane, ACT_SMEM);
    consumers_sync();
    mark(2);
  };

  // (tensor parallel) The residual stream after a row-parallel layer, x = bf16(x_old + bf16(sum
  // over the ranks, in rank order, of the parts in receive slot `slot`)) (slot < 0: x_old as is),
  // staged in shared memory, RMS-normalised with norm_w when non-null; chunk i of it also goes to
  // x_new (when non-null) from CTA i % grid, so the next residual base is whole after the next
  // barrier. Every CTA runs it, with or without units. Needs hidden % 256 == 0.
  auto stage_tp = [&](const bf16* x_old, bf16* x_new, int slot, const bf16* norm_w) {
    const int chunks = H / 8, total = B * chunks;
    const float* parts = slot >= 0 ? reinterpret_cast<const float*>(my_region + a.recv_x + slot * d.tp_world * x_part_bytes)
                                   : nullptr;
    if (norm_w && lane == 0)
      for (int b = 0; b < B; ++b) red_ss[cw * 16 + b] = 0.f;
    for (int i = tid; i < total; i += kCThreads) {  // warp-uniform rows: chunks is a multiple of 32
      const int b = i / chunks, c = i % chunks;
      float f[8];
      unpack8(ldcg16(x_old + static_cast<int64_t>(b) * H + c * 8), f);
      if (parts) {
        float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < d.tp_world; ++r) {
          const float4* q = reinterpret_cast<const float4*>(parts + (static_cast<int64_t>(r) * B + b) * H + c * 8);
          const float4 lo = __ldcv(q), hi = __ldcv(q + 1);  // pushed by the peers: read fresh
          sum[0] += lo.x; sum[1] += lo.y; sum[2] += lo.z; sum[3] += lo.w;
          sum[4] += hi.x; sum[5] += hi.y; sum[6] += hi.z; sum[7] += hi.w;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = bf16_round(f[e] + bf16_round(sum[e]));
      }
      const uint4 packed = pack8(f);
      if (x_new && i % G_ == static_cast<int>(blockIdx.x))
        *reinterpret_cast<uint4*>(x_new + static_cast<int64_t>(b) * H + c * 8) = packed;
      *reinterpret_cast<uint4*>(xs + b * (H + kPad) + c * 8) = packed;
      if (norm_w) {
        float sq = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) sq += f[e] * f[e];
        sq = warp_sum(sq);
        if (lane == 0) red_ss[cw * 16 + b] += sq;
      }
    }
    if (norm_w) {
      consumers_sync();
      for (int i = tid; i < total; i += kCThreads) {
        const int b = i / chunks, c = i % chunks;
        const float r = rsqrtf((red_ss[b] + red_ss[16 + b] + red_ss[32 + b] + red_ss[48 + b]) / static_cast<float>(H) +
                               d.eps);
        float f[8], w[8];
        unpack8(*reinterpret_cast<const uint4*>(xs + b * (H + kPad) + c * 8), f);
        unpack8(ldg16(norm_w + c * 8), w);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = w[e] * bf16_round(f[e] * r);
        *reinterpret_cast<uint4*>(xs + b * (H + kPad) + c * 8) = pack8(f);
      }
    }
    consumers_sync();
    mark(2);
  };

  // (tensor parallel) A row-parallel unit's fp32 sums into every rank's receive slot tp_slot.
  auto push_parts = [&](const float (&acc)[2][NT][4], int rb, int first_half, int halves) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h >= halves) break;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = rb * 32 + (first_half + h) * 16 + g + 8 * (e >> 1);
          const int b = 8 * j + 2 * t + (e & 1);
          if (b >= B || n >= H) continue;
          for (int r = 0; r < d.tp_world; ++r) {
            float* dst = reinterpret_cast<float*>(tp_region(d, r) + a.recv_x +
                                                  (static_cast<size_t>(tp_slot) * d.tp_world + d.tp_rank) * x_part_bytes);
            dst[b * H + n] = acc[h][j][e];
          }
        }
    }
  };

  // (tensor parallel) The LM-head records of row block rb into every rank's record buffer.
  auto push_records = [&](int rb) {
    __syncwarp();
    for (int l = lane; l < B * IPE_PARTIAL_WORDS; l += 32) {
      const int64_t index = static_cast<int64_t>(rb) * B * IPE_PARTIAL_WORDS + l;
      const float v = d.partials[index];
      for (int r = 0; r < d.tp_world; ++r)
        reinterpret_cast<float*>(tp_region(d, r) + a.recv_rec + d.tp_rank * rec_rank_bytes)[index] = v;
    }
  };

  // One weight phase: this CTA's units, tiles round-robin over the consumer warps.
  auto run_phase = [&](auto epi_tag, const PhaseShape& ph, const bf16* src, const bf16* norm_w, int K,
                       const EpilogueArgs& ea) -> bool {
    constexpr int EPI = decltype(epi_tag)::value;
    float my_rstd[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) my_rstd[j] = (!ACT_SMEM && norm_w && 8 * j + g < B) ? rstd[8 * j + g] : 1.f;
    bool ok = true, first = true;
    for (int u = first_unit(cursor); u < ph.units; u += G_) {
      float acc[2][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[h][j][0] = acc[h][j][1] = acc[h][j][2] = acc[h][j][3] = 0.f;
      for (int tt = cw; tt < ph.ku && ok; tt += kConsumers) {
        const int slot = cw * S + mine.slot;
        const int k0 = tt * kTileK;
        uint4 xv[4][NT];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const int b = 8 * j + g;
            const int kk = k0 + c * 32 + 8 * t;
            if (b >= B) {
              xv[c][j] = make_uint4(0, 0, 0, 0);
            } else if constexpr (ACT_SMEM) {
              xv[c][j] = *reinterpret_cast<const uint4*>(xs + b * (K + kPad) + kk);
            } else {
              uint4 raw = ldcg16(src + static_cast<int64_t>(b) * K + kk);
              if (norm_w) {
                float f[8], wf[8];
                unpack8(raw, f);
                unpack8(ldg16(norm_w + kk), wf);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * my_rstd[j]);
                raw = pack8(f);
              }
              xv[c][j] = raw;
            }
          }
        if (!mbar_wait(&full[slot], mine.fill & 1, a.err)) {
          ok = false;
          break;
        }
        if (trace) {
          if (first) mark(3);
          mark(4);
          first = false;
        }
        if (ph.half) consume_half<NT>(acc, smem_addr(ring + slot * kTileBytes), xv, g, t);
        else consume_tile<NT>(acc, smem_addr(ring + slot * kTileBytes), xv, g, t);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        mine.advance(S);
      }
      if (ph.half) {  // the two column chains of a half unit
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[0][j][e] += acc[1][j][e];
      }
      // Fixed-order reduction of the warps' partial sums, then the epilogue by warp 0.
      float* part = red + (cw * 32 + lane) * 8 * NT;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) part[(h * NT + j) * 4 + e] = acc[h][j][e];
      consumers_sync();
      if (cw == 0) {
#pragma unroll
        for (int w = 1; w < kConsumers; ++w) {
          const float* other = red + (w * 32 + lane) * 8 * NT;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[h][j][e] += other[(h * NT + j) * 4 + e];
        }
        if (EPI == kGemvResidual && tp) {  // a row-parallel layer: push this rank's part
          if (ph.half) push_parts(acc, u >> 1, u & 1, 1);
          else push_parts(acc, u, 0, 2);
        } else if (ph.half) {
          if constexpr (EPI == kGemvStore || EPI == kGemvResidual)
            row_block_epilogue<EPI, NT>(acc, u >> 1, lane, ea, u & 1, 1);
        } else {
          row_block_epilogue<EPI, NT>(acc, u, lane, ea);
          if (EPI == kGemvLogits && tp) push_records(u);
        }
      }
      consumers_sync();
      if (!ok) return false;
    }
    cursor = (cursor + ph.units) % G_;
    return true;
  };

  using EpiStore = std::integral_constant<int, kGemvStore>;
  using EpiResidual = std::integral_constant<int, kGemvResidual>;
  using EpiSilu = std::integral_constant<int, kGemvSiluMul>;
  using EpiLogits = std::integral_constant<int, kGemvLogits>;

  bf16* x = static_cast<bf16*>(d.x);
  bf16* qkv = static_cast<bf16*>(d.qkv);
  bf16* attn = static_cast<bf16*>(d.attn);
  bf16* act = static_cast<bf16*>(d.act);
  const int pos = static_cast<int>(state[IPE_STATE_POS]);
  if (pos < 0 || pos >= d.capacity) {
    if (blockIdx.x == 0 && tid == 0) report(a.err, kErrPositionRange);
    return;  // every CTA sees the same position and leaves before the next barrier
  }
  const AttnSplit sp = attn_split(pos, a.max_splits);

  for (int layer = 0; layer < d.layers; ++layer) {
    const ipe_layer_desc& L = d.layer_descs[layer];
    // QKV projection (input RMSNorm fused); tensor parallel: after the previous layer's down_proj
    // parts, the residual stream moves from x to x_alt
    if (tp) stage_tp(x, static_cast<bf16*>(d.x_alt), layer == 0 ? -1 : 1, static_cast<const bf16*>(L.input_layernorm));
    else stage(x, static_cast<const bf16*>(L.input_layernorm), H);
    if (!run_phase(EpiStore{}, phase_shape(layer, 0), x, static_cast<const bf16*>(L.input_layernorm), H,
                   EpilogueArgs{qkv, QKV, QKV, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!grid_sync(a, ++barrier_index, tid, abort_smem, trace)) return;
    // attention: items (split, KV head, row) over the CTAs
    {
      FusedArgs fa{};
      fa.qkv = qkv;
      fa.q_norm = static_cast<const bf16*>(L.q_norm);
      fa.k_norm = static_cast<const bf16*>(L.k_norm);
      fa.cos_t = static_cast<const bf16*>(d.cos_table);
      fa.sin_t = static_cast<const bf16*>(d.sin_table);
      fa.k_cache = static_cast<bf16*>(L.k_cache);
      fa.v_cache = static_cast<bf16*>(L.v_cache);
      fa.out = attn;
      fa.records = a.attn_records;
      fa.counters = a.attn_counters;
      fa.q_heads = d.q_heads;
      fa.kv_heads = d.kv_heads;
      fa.capacity = d.capacity;
      fa.max_splits = a.max_splits;
      fa.eps = d.eps;
      fa.err = a.err;
      const int items = sp.splits * d.kv_heads * B;
      const AttnSmem<G> sm(scratch);
      for (int it = static_cast<int>(blockIdx.x); it < items; it += G_) {
        const int split = it % sp.splits, rest = it / sp.splits;
        // the first item's milestones: K / V requested and q ready, scores and P.V done, merged
        fa.trace = trace && it == static_cast<int>(blockIdx.x) ? trace + 1 + 5 * (barrier_index - 1) + 2 : nullptr;
        attention_item<G>(fa, split, rest % d.kv_heads, rest / d.kv_heads, pos, sp, sm, tid);
        mark(4);
      }
    }
    if (!grid_sync(a, ++barrier_index, tid, abort_smem, trace)) return;
    // o_proj + residual (tensor parallel: this rank's part, pushed to every rank)
    stage(attn, nullptr, Q);
    tp_slot = 0;
    if (!run_phase(EpiResidual{}, phase_shape(layer, 1), attn, nullptr, Q,
                   EpilogueArgs{x, H, H, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!(tp ? grid_sync_tp(a, ++barrier_index, tid, abort_smem, ++tp_epoch)
             : grid_sync(a, ++barrier_index, tid, abort_smem, trace)))
      return;
    // post-attention RMSNorm + gate/up + SiLU * up (tensor parallel: the residual stream moves back
    // from x_alt to x with the o_proj parts)
    if (tp) stage_tp(static_cast<const bf16*>(d.x_alt), x, 0, static_cast<const bf16*>(L.post_attention_layernorm));
    else stage(x, static_cast<const bf16*>(L.post_attention_layernorm), H);
    if (!run_phase(EpiSilu{}, phase_shape(layer, 2), x, static_cast<const bf16*>(L.post_attention_layernorm), H,
                   EpilogueArgs{act, I, 2 * I, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!grid_sync(a, ++barrier_index, tid, abort_smem, trace)) return;
    // down_proj + residual (tensor parallel: this rank's part, pushed to every rank)
    stage(act, nullptr, I);
    tp_slot = 1;
    if (!run_phase(EpiResidual{}, phase_shape(layer, 3), act, nullptr, I,
                   EpilogueArgs{x, H, H, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!(tp ? grid_sync_tp(a, ++barrier_index, tid, abort_smem, ++tp_epoch)
             : grid_sync(a, ++barrier_index, tid, abort_smem, trace)))
      return;
  }
  // final RMSNorm + tied LM head: fp32 logits and one sampling record per 32 vocabulary rows
  // (tensor parallel: this rank's vocabulary rows, records pushed to every rank)
  if (tp) {
    stage_tp(x, nullptr, 1, static_cast<const bf16*>(d.final_norm));
    // neutral records for this rank's padding up to the largest shard's record count
    const int parts_mine = (d.vocab + 31) / 32;
    for (int l = tid; l < (a.parts_max - parts_mine) * B; l += kCThreads) {
      if (blockIdx.x != 0) break;
      const int64_t index = (static_cast<int64_t>(parts_mine) * B + l) * IPE_PARTIAL_WORDS;
      const float rec[IPE_PARTIAL_WORDS] = {-INFINITY, 0.f, -INFINITY, 0.f, __int_as_float(0x7fffffff),
                                            __int_as_float(0x7fffffff), 0.f, 0.f};
      for (int r = 0; r < d.tp_world; ++r)
        for (int w = 0; w < IPE_PARTIAL_WORDS; ++w)
          reinterpret_cast<float*>(tp_region(d, r) + a.recv_rec + d.tp_rank * rec_rank_bytes)[index + w] = rec[w];
    }
  } else {
    stage(x, static_cast<const bf16*>(d.final_norm), H);
  }
  {
    EpilogueArgs ea{d.logits, d.vocab, d.vocab, B, d.partials, state, 0.f, 0};
    ea.row_offset = d.vocab_offset;
    if (!run_phase(EpiLogits{}, phase_shape(d.layers, 0), x, static_cast<const bf16*>(d.final_norm), H, ea)) return;
  }
  if (!(tp ? grid_sync_tp(a, ++barrier_index, tid, abort_smem, ++tp_epoch)
           : grid_sync(a, ++barrier_index, tid, abort_smem, trace)))
    return;
  if (trace && tid == 0) trace[IPE_TRACE_WORDS(d.layers) - 1] = globaltimer_ns();
  if (blockIdx.x != 0) return;

  // Sampling (CTA 0): token and untempered log-probability per row, fed back as the next input.
  // Tensor parallel: over every rank's records (the same on every rank); the chosen token's logit
  // then comes from the records.
  const int parts = tp ? d.tp_world * a.parts_max : (d.vocab + 31) / 32;
  const float* records = tp ? reinterpret_cast<const float*>(my_region + a.recv_rec) : d.partials;
  if (d.history_tokens) {
    const float temperature = __int_as_float(static_cast<int>(state[IPE_STATE_TEMPERATURE]));
    const int64_t step = state[IPE_STATE_STEP];
    for (int b = cw; b < B; b += kConsumers) {
      Stat st = empty_stat();
      for (int p = lane; p < parts; p += 32)
        st = merge(st, tp ? Stat{__ldcv(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS),
                                 __ldcv(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS + 1),
                                 __float_as_int(__ldcv(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS + 4)),
                                 __ldcv(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS + 2),
                                 __float_as_int(__ldcv(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS + 5)),
                                 __ldcv(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS + 3)}
                          : load_stat(records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) st = merge(st, shfl_xor_stat(st, o));
      if (lane == 0) {
        const int token = temperature > 0.f ? st.garg : st.arg;
        const float logit = tp ? (temperature > 0.f ? st.gl : st.m)
                               : __ldcg(d.logits + static_cast<int64_t>(b) * d.vocab + token);
        d.history_tokens[b * d.history_stride + step] = token;
        d.history_logprobs[b * d.history_stride + step] = (logit - st.m) - logf(st.s);
        d.tokens[b] = token;
      }
    }
  }
  consumers_sync();
  if (tid == 0) {
    if (d.history_tokens) state[IPE_STATE_STEP] += 1;
    state[IPE_STATE_POS] = pos + 1;
    if (tp) *reinterpret_cast<unsigned*>(my_region + kTpCounter) = tp_epoch;  // the exchanges of the next step
  }
}


template <int NT, int G, bool ACT>
cudaError_t launch_variant(const StepArgs& a, size_t smem, cudaStream_t stream) {
  auto kernel = decode_step_kernel<NT, G, ACT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemMax));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(sm_count());
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
  attribute[0].val.cooperative = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, a);
}

template <int NT, bool ACT>
cudaError_t by_group(const StepArgs& a, size_t smem, cudaStream_t stream) {
  switch (a.d.q_heads / a.d.kv_heads) {
    case 1: return launch_variant<NT, 1, ACT>(a, smem, stream);
    case 2: return launch_variant<NT, 2, ACT>(a, smem, stream);
    case 4: return launch_variant<NT, 4, ACT>(a, smem, stream);
    case 8: return launch_variant<NT, 8, ACT>(a, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

// Tuning of the weight stream, fixed per process (measured on B200 with Qwen3-1.7B at batch 1, a
// 512-token context: these defaults gave the shortest step): ring slots per consumer warp
// (IPE_STEP_SLOTS, 4), the L2 prefetch distance per CTA in KB (IPE_STEP_PREFETCH_KB, 128; larger
// distances lengthened the latency-bound phases), weight copies marked L2 evict-first
// (IPE_STEP_EVICT_FIRST, 1), and half-row-block units (IPE_STEP_HALF, 1).
struct StepTuning {
  int slots = 4;
  unsigned prefetch_kb = 128;
  int evict_first = 1;
  int halves = 1;
};

const StepTuning& tuning() {
  static const StepTuning t = [] {
    StepTuning r;
    if (const char* v = std::getenv("IPE_STEP_SLOTS")) r.slots = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_PREFETCH_KB")) r.prefetch_kb = static_cast<unsigned>(std::atoi(v));
    if (const char* v = std::getenv("IPE_STEP_EVICT_FIRST")) r.evict_first = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_HALF")) r.halves = std::atoi(v);
    return r;
  }();
  return t;
}

size_t fixed_smem(int nt, int slots) {
  return 1024 + static_cast<size_t>(kConsumers) * slots * kTileBytes + 2 * kMaxStages * 8 + 16 * 4 + 16 +
         static_cast<size_t>(kConsumers) * 32 * 8 * nt * 4;
}

size_t attn_bytes(int group) {
  switch (group) {
    case 1: return attn_smem_floats<1>() * 4;
    case 2: return attn_smem_floats<2>() * 4;
    case 4: return attn_smem_floats<4>() * 4;
    default: return attn_smem_floats<8>() * 4;
  }
}

}  // namespace

size_t decode_step_comm_bytes(int world, int batch, int hidden, int vocab_rows_max) {
  const size_t parts_max = (static_cast<size_t>(vocab_rows_max) + 31) / 32;
  const size_t recv_x = (2ull * world * batch * hidden * sizeof(float) + 255) / 256 * 256;
  return 256 + recv_x + static_cast<size_t>(world) * parts_max * batch * IPE_PARTIAL_WORDS * sizeof(float);
}

size_t decode_step_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity) {
  (void)capacity;  // attention records are per split, at most kAttnSplitsMax of them
  const size_t counters = (static_cast<size_t>(batch) * kv_heads * sizeof(int) + 255) / 256 * 256;
  return 256 + counters + static_cast<size_t>(batch) * q_heads * kAttnSplitsMax * kAttnRecord * sizeof(float);
}

cudaError_t launch_decode_step(const ipe_decode_step_desc& d, int* err, cudaStream_t stream, const char** message) {
  StepArgs a{};
  a.d = d;
  a.err = err;
  a.max_splits = attn_max_splits(sm_count(), d.batch, d.kv_heads);
  unsigned char* ws = static_cast<unsigned char*>(d.workspace);
  a.grid_bar = reinterpret_cast<unsigned*>(ws);
  a.attn_counters = reinterpret_cast<int*>(ws + 256);
  const size_t counters = (static_cast<size_t>(d.batch) * d.kv_heads * sizeof(int) + 255) / 256 * 256;
  a.attn_records = reinterpret_cast<float*>(ws + 256 + counters);
  const int nt = d.batch <= 8 ? 1 : 2;
  const int group = d.q_heads / d.kv_heads;
  const size_t act = static_cast<size_t>(d.batch) *
                     (std::max(std::max(d.hidden, d.intermediate), d.q_heads * 128) + kPad) * 2;
  const size_t attn = attn_bytes(group);
  // Activations stay in shared memory when that leaves room for 4 slots per consumer warp.
  const bool act_smem = fixed_smem(nt, 4) + std::max(act, attn) <= kSmemMax;
  const size_t scratch = act_smem ? std::max(act, attn) : attn;
  int slots = std::min(kMaxSlotsPerWarp, std::max(2, tuning().slots));
  while (slots > 2 && fixed_smem(nt, slots) + scratch > kSmemMax) --slots;
  a.slots = slots;
  a.prefetch_bytes = tuning().prefetch_kb * 1024u;
  a.evict_first = tuning().evict_first;
  a.halves = tuning().halves;
  const size_t smem = fixed_smem(nt, slots) + scratch;
  if (smem > kSmemMax) {
    *message = "decode-step scratch does not fit in shared memory";
    return cudaErrorInvalidValue;
  }
  if (d.tp_world > 1) {
    if (!act_smem || d.hidden % 256) {
      *message = "tensor parallel: needs hidden % 256 == 0 and the activations in shared memory (a smaller batch)";
      return cudaErrorInvalidValue;
    }
    const int blocks = (d.vocab_total + 31) / 32;
    a.parts_max = (blocks + d.tp_world - 1) / d.tp_world;
    a.recv_x = 256;
    a.recv_rec = a.recv_x + (2ull * d.tp_world * d.batch * d.hidden * sizeof(float) + 255) / 256 * 256;
  }
  // the grid barrier counts arrivals from zero every step ([0] arrivals, [1] abort, [2] release)
  cudaError_t e = cudaMemsetAsync(a.grid_bar, 0, 4 * sizeof(unsigned), stream);
  if (e != cudaSuccess) return e;
  if (nt == 1) return act_smem ? by_group<1, true>(a, smem, stream) : by_group<1, false>(a, smem, stream);
  return act_smem ? by_group<2, true>(a, smem, stream) : by_group<2, false>(a, smem, stream);
}

}  // namespace ipe
