// One whole decode step in one persistent kernel: embedding, every layer's QKV projection
// (RMSNorm fused), attention (q/k norm + RoPE + KV append + split-KV), o_proj + residual,
// RMSNorm + gate/up + SiLU*up, down_proj + residual, the final norm + tied LM head with fp32
// logits and sampling records, and (optionally) the sampled token fed back for the next step.
//
// Why one kernel: every weight byte of the step is known before the step starts, so the weight
// stream does not depend on activations. Each CTA (one per SM, cooperative launch) has a producer
// thread that walks its share of ALL phases' weights back to back and never waits for a phase
// boundary: a unit's weights are one contiguous run of half tiles (stream_tile.cuh), streamed in
// 32 KB bulk copies into a ring of shared-memory stages that all four consumer warps read. Copies
// that large are what lets one SM's copy engine keep up with its share of HBM (8 KB copies cap the
// whole GPU near 4.9 TB/s, 32 KB ones reach 7.3 TB/s). Nothing is prefetched into L2 by default
// (weights past the ring, or each layer's K / V rows): every such prefetch measured slower, as it
// lengthens the L2 round trips of the phase boundaries. The consumer warps wait only where the
// data requires it:
// at a bounded-spin grid barrier after each phase (the next phase needs the full activation
// vector), then they stage that vector in shared memory and consume stages that are usually
// already there.
//
// Work split: a phase's units (a 32-row block, or a 16-row half block where that evens out the
// bytes per CTA, always over the whole K: no split-K) are dealt round-robin over the CTAs,
// continuing where the previous phase stopped; within a stage, warp w takes half tiles w and
// w + 4, and the warps' partial sums are reduced in a fixed order through shared memory
// (deterministic). Attention runs as (split, KV head, row) items over the CTAs. Every spin (grid
// barrier, mbarrier) is bounded; a timeout sets the device error word and an abort flag, the
// kernel winds down, and the producer waits for its copies in flight before it leaves.
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
constexpr int kStageTiles = 8;                             // half tiles per stage (2 per consumer warp)
constexpr int kStageBytes = kStageTiles * kHalfTileBytes;  // 32 KB: one bulk copy
constexpr int kMaxStages = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kCThreads = 32 * kConsumers;
constexpr int kPad = 32;
constexpr int kStepBarrier = 1;  // named barrier id of the consumer warps
constexpr int kReadyWord = 32;   // first per-KV-head readiness counter in the barrier words
constexpr int kReadyHeadsMax = 32;  // the barrier words hold 64 counters; KV heads beyond use the barrier
constexpr size_t kSmemMax = 226 * 1024;  // dynamic shared memory; the rest holds static arrays

struct StepArgs {
  ipe_decode_step_desc d;
  unsigned* grid_bar;  // [0] arrivals, [1] abort flag, [kReadyWord + h] QKV rows of KV head h written (x 16)
  int* attn_counters;
  float* attn_records;
  int* err;
  int stages;               // 32 KB ring stages
  int max_splits;           // attention splits per (row, KV head)
  int attn_slots;           // attention K / V ring slots (16 KB each, at the start of the scratch)
  int prefetch_kv;          // the producer prefetches each layer's K / V rows (and norm weights) into L2
  int l2_ahead;             // the producer keeps this many stages past its copies prefetched into L2
  int evict_first;          // weight copies mark their L2 lines evict-first
  int halves;               // half-row-block units allowed
  int act_cols;             // without ACT_SMEM: RMS-normalised phases with K <= act_cols still stage in shared memory
  int bulk_stage;           // with ACT_SMEM: phases without a norm stage their rows by bulk copies (batch > 1)
  int qkv_ready;            // per-KV-head readiness counters replace the grid barrier after the QKV phase
  unsigned xres_off;        // bulk staging: byte offset from the scratch of a copy of the residual rows x (0: none)
  int light_fences;         // grid barrier arrival: 2 release reduction, 1 acq_rel fence + atomic, 0 full fences
  int overlap_epilogue;     // warps 1-3 start the next unit while warp 0 runs this unit's epilogue
  float* cta_records;       // [grid][batch][IPE_PARTIAL_WORDS]: each CTA's merge of its LM-head records
  uint64_t wait_ns;         // bound of every spin-wait
  // tensor parallelism (d.tp_world > 1): byte offsets in a communication region
  size_t recv_x;            // [2 slots][world][batch][hidden / 16][8 lines] parts of o_proj / down_proj
  size_t recv_rec;          // [world][grid][batch][3 lines] the CTAs' merged LM-head records
};

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kStepBarrier), "n"(kCThreads) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier among the consumer warps of all CTAs (the index-th of the step). Returns false when
// the step is aborted. tr (this barrier's words in this CTA's row of the step trace, or null)
// receives the arrival and release times.
__device__ bool grid_sync(const StepArgs& a, unsigned index, int tid, int* abort_smem, uint64_t* tr) {
  consumers_sync();
  if (tid == 0) {
    if (tr) tr[0] = globaltimer_ns();
    // release: the consumer warps' writes (ordered before by the named barrier) before the arrival.
    // light_fences 2: one release reduction (no returned value to wait for) and a poll of the count
    // alone, the abort flag checked with the clock every 64 polls; 1: an acq_rel fence, then the
    // atomic; 0: full fences on both sides.
    const bool red_arrive = a.light_fences == 2;
    if (red_arrive) {
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(&a.grid_bar[0]), "r"(1u) : "memory");
    } else {
      if (a.light_fences) asm volatile("fence.acq_rel.gpu;" ::: "memory");
      else __threadfence();
      atomicAdd(&a.grid_bar[0], 1u);
    }
    const unsigned target = index * gridDim.x;
    uint64_t start = 0;
    for (unsigned i = 0;; ++i) {
      if (ld_acquire(&a.grid_bar[0]) >= target) break;
      if ((!red_arrive || (i & 63u) == 63u) && ld_acquire(&a.grid_bar[1])) {
        *abort_smem = 1;
        break;
      }
      if ((i & 63u) == 63u) {
        const uint64_t now = globaltimer_ns();
        if (start == 0) start = now;
        else if (now - start > a.wait_ns) {
          report(a.err, kErrWaitTimeout);
          atomicExch(&a.grid_bar[1], 1u);
          *abort_smem = 1;
          break;
        }
      }
      if (!red_arrive) __nanosleep(64);
    }
    // the acquire load that saw the count already orders this CTA's later reads (through the
    // named barrier below); the full fence is kept as the measured alternative
    if (!a.light_fences) __threadfence();
    if (tr) tr[1] = globaltimer_ns();
  }
  consumers_sync();
  return *abort_smem == 0;
}

// --------------------------------------------------------------------- tensor parallelism
// Communication region of a rank (ipe_decode_step_comm_bytes): the epoch counter at byte 128 (the
// last exchange epoch of the previous step), then the receive buffers. Every value a peer sends is
// a flagged element: one naturally aligned 64-bit word {value (low 32 bits), epoch (high 32 bits)},
// and a 16-byte line holds two of them. Lines are written and read as vectors of two 64-bit
// elements; the memory model makes each 64-bit element a single-copy-atomic access (a vector is not
// atomic as a whole), so a reader that sees the current epoch in an element holds that element's
// value. The exchange needs no fence and no barrier; each exchange has its own epoch, so an element
// from an earlier one never passes.
constexpr size_t kTpCounter = 128;
constexpr size_t kTpRecv = 256;
constexpr size_t kTpLine = 16;
constexpr size_t kTpRecordBytes = 3 * kTpLine;  // sampling record words 0..5: {m, s} {gs, gl} {arg, garg}

__device__ __forceinline__ unsigned char* tp_region(const ipe_decode_step_desc& d, int r) {
  return reinterpret_cast<unsigned char*>(static_cast<const uint64_t*>(d.tp_peers)[r]);
}

// Two flagged elements {w0, epoch} and {w1, epoch}, each one 64-bit access.
__device__ __forceinline__ void st_line(void* p, uint32_t w0, uint32_t w1, unsigned epoch) {
  const uint64_t e0 = (static_cast<uint64_t>(epoch) << 32) | w0;
  const uint64_t e1 = (static_cast<uint64_t>(epoch) << 32) | w1;
  asm volatile("st.volatile.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(e0), "l"(e1) : "memory");
}

// The line's elements as {value 0, epoch 0, value 1, epoch 1}.
__device__ __forceinline__ uint4 ld_line(const void* p) {
  uint64_t e0, e1;
  asm volatile("ld.volatile.global.v2.b64 {%0, %1}, [%2];" : "=l"(e0), "=l"(e1) : "l"(p) : "memory");
  return make_uint4(static_cast<uint32_t>(e0), static_cast<uint32_t>(e0 >> 32), static_cast<uint32_t>(e1),
                    static_cast<uint32_t>(e1 >> 32));
}

__device__ __forceinline__ bool line_ready(const uint4& v, unsigned epoch) { return v.y == epoch && v.w == epoch; }

// Re-reads the line at p until it carries `epoch` and returns it; once the step is aborted or the
// wait limit passed (the error word is set and every CTA is told to leave), returns the last read,
// which the caller sees is not ready.
__device__ __noinline__ uint4 wait_line(const StepArgs& a, const void* p, unsigned epoch) {
  uint64_t start = 0;
  for (unsigned i = 0;; ++i) {
    const uint4 v = ld_line(p);
    if (line_ready(v, epoch)) return v;
    if ((i & 63u) == 63u) {
      if (ld_acquire(&a.grid_bar[1])) return v;
      const uint64_t now = globaltimer_ns();
      if (start == 0) start = now;
      else if (now - start > a.wait_ns) {
        report(a.err, kErrWaitTimeout);
        atomicExch(&a.grid_bar[1], 1u);
        return v;
      }
    }
    __nanosleep(32);
  }
}

// The staging of a tensor-parallel phase (see stage_tp in the kernel), kept out of line so that
// its registers do not weigh on the weight-streaming loop.
struct TpStage {
  const bf16* x_old;
  bf16* x_new;
  const unsigned char* parts;  // this rank's receive slot (world parts), or null: x_old as is
  const bf16* norm_w;          // nullable
  bf16* xs;                    // shared [batch][hidden + kPad]
  float* red_ss;               // shared [4 warps][16 rows]
  size_t part_bytes;
  unsigned epoch;
  int* abort_smem;
};

__device__ __noinline__ void tp_stage(const StepArgs& a, const TpStage& st, int tid) {
  const ipe_decode_step_desc& d = a.d;
  const int B = d.batch, H = d.hidden, G_ = static_cast<int>(gridDim.x);
  const int lane = tid & 31, cw = tid >> 5;
  const int chunks = H / 16, total = B * chunks;
  bool ok = true;
  if (st.norm_w && lane == 0)
    for (int b = 0; b < B; ++b) st.red_ss[cw * 16 + b] = 0.f;
  // the norm weights of this thread's first 16-column chunk, fetched with the rows and parts (with
  // hidden = 16 * 128 every chunk of the thread has these columns)
  const int k_first = tid % chunks;
  uint4 w_first[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (st.norm_w) {
    w_first[0] = ldg16(st.norm_w + k_first * 16);
    w_first[1] = ldg16(st.norm_w + k_first * 16 + 8);
  }
  for (int i = tid; i < total; i += kCThreads) {  // warp-uniform rows: chunks is a multiple of 32
    const int b = i / chunks, k = i % chunks;
    const bf16* xo = st.x_old + static_cast<int64_t>(b) * H + k * 16;
    float f[16];
    unpack8(ldcg16(xo), f);
    unpack8(ldcg16(xo + 8), f + 8);
    if (st.parts) {
      float sum[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) sum[e] = 0.f;
      for (int r = 0; r < d.tp_world; ++r) {
        const unsigned char* lines = st.parts + r * st.part_bytes + (static_cast<size_t>(b) * chunks + k) * 8 * kTpLine;
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = ld_line(lines + q * kTpLine);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (!line_ready(v[q], st.epoch) && ok) {
            v[q] = wait_line(a, lines + q * kTpLine, st.epoch);
            ok = line_ready(v[q], st.epoch);
          }
          sum[q] += __uint_as_float(v[q].x);
          sum[q + 8] += __uint_as_float(v[q].z);
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = bf16_round(f[e] + bf16_round(sum[e]));
    }
    const uint4 lo = pack8(f), hi = pack8(f + 8);
    if (st.x_new && i % G_ == static_cast<int>(blockIdx.x)) {
      bf16* xn = st.x_new + static_cast<int64_t>(b) * H + k * 16;
      *reinterpret_cast<uint4*>(xn) = lo;
      *reinterpret_cast<uint4*>(xn + 8) = hi;
    }
    *reinterpret_cast<uint4*>(st.xs + b * (H + kPad) + k * 16) = lo;
    *reinterpret_cast<uint4*>(st.xs + b * (H + kPad) + k * 16 + 8) = hi;
    if (st.norm_w) {
      float sq = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) sq += f[e] * f[e];
      sq = warp_sum(sq);
      if (lane == 0) st.red_ss[cw * 16 + b] += sq;
    }
  }
  if (!ok) *st.abort_smem = 1;
  if (st.norm_w) {
    consumers_sync();
    // the same 16-column chunks as above: the norm weights are mostly in registers already
    for (int i = tid; i < total; i += kCThreads) {
      const int b = i / chunks, k = i % chunks;
      const float* ss = st.red_ss;
      const float r = rsqrtf((ss[b] + ss[16 + b] + ss[32 + b] + ss[48 + b]) / static_cast<float>(H) + d.eps);
      bf16* row = st.xs + b * (H + kPad) + k * 16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float f[8], w[8];
        unpack8(*reinterpret_cast<const uint4*>(row + 8 * h), f);
        unpack8(k == k_first ? w_first[h] : ldg16(st.norm_w + k * 16 + 8 * h), w);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = w[e] * bf16_round(f[e] * r);
        *reinterpret_cast<uint4*>(row + 8 * h) = pack8(f);
      }
    }
  }
  consumers_sync();
}

// Row b's merge, over this lane's share (p = lane, lane + 32, ...) of `parts` flagged records at
// recs, 4 records in flight. ok is cleared when a record does not arrive (the step is aborted).
struct MergedRecords {
  Stat st;
  bool ok;
};

__device__ __noinline__ MergedRecords tp_merge_records(const StepArgs& a, const unsigned char* recs, int parts, int b,
                                                       int lane, unsigned epoch) {
  const int B = a.d.batch;
  MergedRecords m{empty_stat(), true};
  for (int p0 = lane; p0 < parts; p0 += 4 * 32) {
    uint4 v[4][3];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (p0 + 32 * k < parts)
          v[k][q] = ld_line(recs + (static_cast<size_t>(p0 + 32 * k) * B + b) * kTpRecordBytes + q * kTpLine);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int p = p0 + 32 * k;
      if (p >= parts) break;
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (!line_ready(v[k][q], epoch) && m.ok) {
          v[k][q] = wait_line(a, recs + (static_cast<size_t>(p) * B + b) * kTpRecordBytes + q * kTpLine, epoch);
          m.ok = line_ready(v[k][q], epoch);
        }
      m.st = merge(m.st, Stat{__uint_as_float(v[k][0].x), __uint_as_float(v[k][0].z), static_cast<int>(v[k][2].x),
                              __uint_as_float(v[k][1].x), static_cast<int>(v[k][2].z), __uint_as_float(v[k][1].z)});
    }
  }
  return m;
}

// This lane's activation vectors for the tile whose columns start at k0 (batch columns 8j + g):
// from the staged rows xs (row stride K + pad) or, without staging, from src in global memory with
// the RMS scale and norm weight applied (the reference's two roundings). Rows past the batch are 0.
template <int NT>
__device__ __forceinline__ void load_activations(uint4 (&xv)[4][NT], int k0, bool staged, const bf16* xs,
                                                 const bf16* src, const bf16* norm_w, const float (&rstd)[NT], int K,
                                                 int pad, int B, int g, int t) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int b = 8 * j + g;
      const int kk = k0 + c * 32 + 8 * t;
      if (b >= B) {
        xv[c][j] = make_uint4(0, 0, 0, 0);
      } else if (staged) {
        xv[c][j] = *reinterpret_cast<const uint4*>(xs + b * (K + pad) + kk);
      } else {
        uint4 raw = ldcg16(src + static_cast<int64_t>(b) * K + kk);
        if (norm_w) {
          float f[8], wf[8];
          unpack8(raw, f);
          unpack8(ldg16(norm_w + kk), wf);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * rstd[j]);
          raw = pack8(f);
        }
        xv[c][j] = raw;
      }
    }
}

// Slot bookkeeping of the ring: stage index and how often it wrapped.
struct SlotCursor {
  int slot = 0, fill = 0;
  __device__ __forceinline__ void advance(int slots) {
    if (++slot == slots) {
      slot = 0;
      ++fill;
    }
  }
};

// The LM head's unit epilogue with one lane per vocabulary row: red holds the four consumer warps'
// sums in the MMA fragment layout (lane g * 4 + t holds rows h * 16 + g + 8 * (e >> 1), batch column
// 8 j + 2 t + (e & 1) at [(h * NT + j) * 4 + e]). Per batch row b: lane l adds the warps' sums of row
// rb * 32 + l in warp order and rounds it to bf16 (the reference's bf16 logits, widened), stores it,
// and the warp reduces the row block's sampling record (max, sum of exp(l - max), lowest argmax,
// and with a temperature the Gumbel maximum, its ID and logit) with one exp per lane.
template <int NT>
__device__ __forceinline__ void logits_epilogue(const float* red, int rb, int lane, const EpilogueArgs& a) {
  float* logits = static_cast<float*>(a.out);
  const float temperature = __int_as_float(static_cast<int>(a.state[IPE_STATE_TEMPERATURE]));
  const uint64_t seed = static_cast<uint64_t>(a.state[IPE_STATE_SEED]);
  const int64_t step = a.state[IPE_STATE_STEP];
  const int h = lane >> 4, g = lane & 7, e_hi = (lane >> 3) & 1;
  const int n = rb * 32 + lane;
  const bool live = n < a.rows;
  for (int b = 0; b < a.batch; ++b) {
    const int j = b >> 3, t = (b & 7) >> 1, e = 2 * e_hi + (b & 1);
    const float* src = red + (g * 4 + t) * 8 * NT + (h * NT + j) * 4 + e;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) sum += src[w * 32 * 8 * NT];
    const float l = live ? bf16_round(sum) : -INFINITY;
    if (live) logits[static_cast<int64_t>(b) * a.out_stride + n] = l;
    const int id = n + a.row_offset;
    const float m = warp_max(l);
    const float sx = warp_sum(live ? expf(l - m) : 0.f);
    int arg = (live && l == m) ? id : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) arg = min(arg, __shfl_xor_sync(0xffffffffu, arg, o));
    float gs = -INFINITY, gl = 0.f;
    int garg = 0x7fffffff;
    if (temperature > 0.f) {
      const float score = live ? l / temperature - logf(-logf(uniform01(seed, id, b, step))) : -INFINITY;
      const float best = warp_max(score);
      garg = (live && score == best) ? id : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) garg = min(garg, __shfl_xor_sync(0xffffffffu, garg, o));
      gl = __shfl_sync(0xffffffffu, l, (garg - a.row_offset - rb * 32) & 31);
      gs = best;
    }
    if (lane == 0) {
      float* rec = a.partials + (static_cast<int64_t>(rb) * a.batch + b) * IPE_PARTIAL_WORDS;
      rec[0] = m;
      rec[1] = sx;
      rec[2] = gs;
      rec[3] = gl;
      rec[4] = __int_as_float(arg);
      rec[5] = __int_as_float(garg);
    }
  }
}

// First unit of this CTA in a phase that starts dealing at `cursor`.
__device__ __forceinline__ int first_unit(int cursor) {
  const int g = static_cast<int>(gridDim.x);
  return (static_cast<int>(blockIdx.x) - cursor % g + g) % g;
}

// A weight phase as units dealt round-robin over the CTAs: a unit is one row block (32 rows, whole
// K: its two halves' runs of half tiles, one after the other) or, when that lowers the most bytes
// any CTA streams in the phase, one 16-row half of a row block (one run).
struct PhaseShape {
  const unsigned char* tiles;
  int units;
  int ku;  // k tiles (128 columns) per row
  bool half;
  __device__ __forceinline__ int half_tiles() const { return half ? ku : 2 * ku; }
  // the unit's run of half tiles: row block rb, starting at half (u & 1) of a half unit
  __device__ __forceinline__ const unsigned char* run(int u) const {
    return tiles + (half ? half_tile_offset(u >> 1, u & 1, 0, ku) : half_tile_offset(u, 0, 0, ku));
  }
};

__device__ __forceinline__ PhaseShape make_phase(const void* tiles, int row_blocks, int ku, bool may_halve) {
  const int g = static_cast<int>(gridDim.x);
  const bool half = may_halve && (2 * row_blocks + g - 1) / g < 2 * ((row_blocks + g - 1) / g);
  return {static_cast<const unsigned char*>(tiles), half ? 2 * row_blocks : row_blocks, ku, half};
}

// Position of a walk over this CTA's units of the step, in stream order.
struct UnitWalk {
  int layer = 0, kind = 0, cursor = 0, unit = 0;
  bool in_phase = false, done = false;
  PhaseShape ph{};
};

// Position of a walk over this CTA's ring stages of the step (up to 32 KB of one unit's run each).
struct StageWalk {
  UnitWalk w;
  const unsigned char* run = nullptr;
  int n_ht = 0, s0 = 0;
};

// TP: a tensor-parallel rank (tp_world > 1; needs ACT_SMEM), compiled apart so that the one-GPU
// variants carry none of its code.
template <int NT, int G, bool ACT_SMEM, bool TP>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const StepArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int S = a.stages;
  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(S) * kStageBytes);
  uint64_t* empty = full + kMaxStages;
  float* rstd = reinterpret_cast<float*>(empty + kMaxStages);  // [16]
  int* abort_smem = reinterpret_cast<int*>(rstd + 16);
  float* red = reinterpret_cast<float*>(abort_smem + 4);  // [2 units][kConsumers][32][8 * NT]
  // the layer descriptors, copied once: every phase reads its operands' addresses from here
  ipe_layer_desc* descs = reinterpret_cast<ipe_layer_desc*>(red + 2 * kConsumers * 32 * 8 * NT);
  float* scratch = reinterpret_cast<float*>(descs + a.d.layers);  // activations or attention scratch (16-byte aligned)
  bf16* xres = reinterpret_cast<bf16*>(reinterpret_cast<unsigned char*>(scratch) + a.xres_off);  // if xres_off
  bf16* xs = reinterpret_cast<bf16*>(scratch);

  const ipe_decode_step_desc& d = a.d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = d.batch, H = d.hidden, I = d.intermediate;
  const int Q = d.q_heads * 128, QKV = (d.q_heads + 2 * d.kv_heads) * 128;
  const int G_ = static_cast<int>(gridDim.x);

  __shared__ uint64_t stage_bar;  // completion of the bulk copies that stage activation rows
  __shared__ uint64_t attn_bars[kAttnSlotsMax + 1];  // the attention items' K / V ring and merge copies
  __shared__ uint64_t desc_bar;                      // completion of the layer descriptors' copy
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    mbar_init(&stage_bar, 1);
    attn_ring_init(attn_bars);
    mbar_init(&desc_bar, 1);
    *abort_smem = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bytes = static_cast<uint32_t>(a.d.layers) * sizeof(ipe_layer_desc);
    mbar_expect_tx(&desc_bar, bytes);
    bulk_copy(smem_addr(descs), a.d.layer_descs, bytes, &desc_bar);
  }

  // kind: 0 QKV, 1 o_proj, 2 gate/up, 3 down_proj; layer == layers: the LM head.
  auto phase_shape = [&](int layer, int kind) -> PhaseShape {
    if (layer == d.layers) return make_phase(d.lm_head_tiles, (d.vocab + 31) / 32, H / kTileK, false);
    const ipe_layer_desc& L = descs[layer];
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
    // One thread issues every copy of the SM: each unit's run in stages of up to 8 half tiles
    // (32 KB), one bulk copy per stage, into the ring in order. Entering a layer's QKV phase, it
    // also prefetches into L2 the K / V rows this CTA's attention items of the layer will read and
    // the layer's norm weights (they are on the critical path of the next stages and items).
    if (lane == 0) {
      const uint32_t ring_base = smem_addr(ring);
      const uint64_t policy = evict_first_policy();
      const int pos = static_cast<int>(d.state[IPE_STATE_POS]);
      // the descriptors' copy (this thread issued it) lands before anything reads them or it leaves
      if (!mbar_wait(&desc_bar, 0, a.err, a.wait_ns)) atomicExch(&a.grid_bar[1], 1u);
      if (pos < 0 || pos >= d.capacity) return;  // the consumers leave too; nothing else was issued
      const AttnSplit sp = attn_split(pos, a.max_splits);
      auto prefetch_kv = [&](int layer) {
        const ipe_layer_desc& L = descs[layer];
        // a bulk prefetch needs a 16-byte aligned start, so an unaligned vector is left to the loads
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
      // The L2 window: stages past the ring's copies are prefetched into L2, a.l2_ahead of them, so
      // that HBM keeps streaming while the ring is full and the consumers wait at a phase boundary;
      // the copies then read those stages from L2 (and mark them evict-first).
      StageWalk pf;
      auto prefetch_next = [&]() {
        while (pf.s0 >= pf.n_ht) {
          int entered_pf;
          if (!next_unit(pf.w, entered_pf)) return;
          pf.run = pf.w.ph.run(pf.w.unit);
          pf.n_ht = pf.w.ph.half_tiles();
          pf.s0 = 0;
        }
        const uint32_t bytes = static_cast<uint32_t>(min(kStageTiles, pf.n_ht - pf.s0)) * kHalfTileBytes;
        prefetch_l2(pf.run + static_cast<int64_t>(pf.s0) * kHalfTileBytes, bytes);
        pf.s0 += kStageTiles;
      };
      for (int i = 0; i < a.l2_ahead; ++i) prefetch_next();
      UnitWalk walk;
      SlotCursor rc;  // the ring position of the next copy
      bool ok = true;
      int entered;
      while (ok && next_unit(walk, entered)) {
        if (entered >= 0 && a.prefetch_kv) prefetch_kv(entered);
        const PhaseShape& ph = walk.ph;
        const unsigned char* run = ph.run(walk.unit);
        const int n_ht = ph.half_tiles();
        for (int s0 = 0; s0 < n_ht; s0 += kStageTiles) {
          const uint32_t bytes = static_cast<uint32_t>(min(kStageTiles, n_ht - s0)) * kHalfTileBytes;
          if (rc.fill > 0 && !mbar_wait(&empty[rc.slot], (rc.fill - 1) & 1, a.err, a.wait_ns)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[rc.slot], bytes);
          const uint32_t dst = ring_base + rc.slot * kStageBytes;
          const unsigned char* src = run + static_cast<int64_t>(s0) * kHalfTileBytes;
          if (a.evict_first) bulk_copy_hint(dst, src, bytes, &full[rc.slot], policy);
          else bulk_copy(dst, src, bytes, &full[rc.slot]);
          rc.advance(S);
          if (a.l2_ahead > 0) prefetch_next();
        }
      }
      // Every copy issued has landed before the thread leaves (on an aborted step the consumers may
      // have left early): stage s was filled fills(s) times; wait for the last of them.
      for (int st = 0; st < S; ++st) {
        const int fills = rc.fill + (st < rc.slot ? 1 : 0);
        if (fills > 0) mbar_wait(&full[st], (fills - 1) & 1, a.err, a.wait_ns);
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cw = warp - 1, tid = threadIdx.x - 32;
  const int g = lane >> 2, t = lane & 3;
  SlotCursor mine;  // the ring position of the next stage (every consumer warp reads every stage)
  int cursor = 0;
  // phase ends so far (each a grid barrier, or in tensor-parallel steps after a row-parallel phase
  // the end of this CTA's pushes), and grid barriers so far
  unsigned barrier_index = 0, syncs = 0;
  unsigned red_flip = 0;  // units consumed so far: which partial-sum buffer the next one uses
  int64_t* state = d.state;
  uint64_t* trace = d.trace ? d.trace + static_cast<int64_t>(blockIdx.x) * IPE_TRACE_WORDS(d.layers) : nullptr;
  if (trace && tid == 0) trace[0] = globaltimer_ns();
  // trace word k (2: staged, 3: first tile ready, 4: last tile ready) of the current phase
  auto mark = [&](int k) {
    if (trace && tid == 0) trace[1 + 5 * (barrier_index - 1) + k] = globaltimer_ns();
  };
  // the end of a phase: a grid barrier, or (tensor parallel, after a row-parallel phase) none: the
  // readers of the pushed parts poll them
  auto phase_end = [&](bool barrier) -> bool {
    ++barrier_index;
    uint64_t* tr = trace ? trace + 1 + 5 * (barrier_index - 1) : nullptr;
    if (barrier) return grid_sync(a, ++syncs, tid, abort_smem, tr);
    if (tr && tid == 0) tr[0] = tr[1] = globaltimer_ns();
    return true;
  };
  // tensor parallelism: this rank's region and the epoch of the current exchange. Every CTA reads
  // the counter before the first grid barrier; CTA 0 advances it at the end of the step.
  constexpr bool tp = TP;
  unsigned char* my_region = tp ? tp_region(d, d.tp_rank) : nullptr;
  unsigned tp_epoch = tp ? *reinterpret_cast<const volatile unsigned*>(my_region + kTpCounter) : 0u;
  const size_t x_part_bytes = static_cast<size_t>(B) * H / 2 * kTpLine;  // one rank's part: 2 values a line
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
  if (!phase_end(true)) return;

  // Whether a phase of reduction width K keeps its activation rows in shared memory: always with
  // ACT_SMEM; otherwise (a batch whose widest rows do not fit) an RMS-normalised phase whose K fits
  // in the scratch (measured at batch 16: staging beats per-tile normalisation there, while the
  // phases without a norm are faster reading their activations from L2 tile by tile).
  auto act_in_smem = [&](int K, bool normed) -> bool { return ACT_SMEM || (normed && K <= a.act_cols); };

  // Stage the B activation rows (row b at src + b * cols, no norm) in shared memory (rows of
  // cols + kPad) with one bulk copy per row, all on one mbarrier, so the batch costs one round trip
  // instead of one per row per warp. Callers have synchronised the consumer warps since the last
  // reads of xs; returns with them synchronised again. A copy that never lands sets the device
  // error and aborts the step. (Measured: with a norm, the per-lane loads of stage_rows, which
  // fetch rows and weights together, stay faster.)
  unsigned stage_parity = 0;
  // With res (the residual rows x of an o_proj / down_proj phase) and a residual copy in shared
  // memory (xres), those rows arrive on the same mbarrier, so the phase's residual epilogues read
  // shared memory instead of making an L2 round trip per unit.
  auto stage_bulk = [&](const bf16* src, int cols, const bf16* res) {
    const int64_t src_stride = cols;
    const int xs_cols = cols;
    if (tid == 0) {
      // generic writes of xs (this CTA) and of src (every CTA) come before the async-proxy copies
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("fence.proxy.async.global;" ::: "memory");
      const uint32_t bytes = static_cast<uint32_t>(cols) * 2u;
      const uint32_t res_bytes = res ? static_cast<uint32_t>(H) * 2u : 0u;
      mbar_expect_tx(&stage_bar, (bytes + res_bytes) * static_cast<uint32_t>(B));
      for (int b = 0; b < B; ++b)
        bulk_copy(smem_addr(xs + b * (xs_cols + kPad)), src + b * src_stride, bytes, &stage_bar);
      if (res)
        for (int b = 0; b < B; ++b) bulk_copy(smem_addr(xres + b * H), res + b * H, res_bytes, &stage_bar);
    }
    if (!mbar_wait(&stage_bar, stage_parity, a.err, a.wait_ns)) {
      atomicExch(&a.grid_bar[1], 1u);  // every CTA leaves at its next barrier
      *abort_smem = 1;
    }
    stage_parity ^= 1u;
    consumers_sync();
  };

  // Stage the activation rows of a phase (optionally RMS-normalised) in shared memory; without
  // shared staging only the RMS scales are kept and tiles read activations from global memory.
  // One RMS-normalised row (batch 1, K <= 2048) staged by all four consumer warps, two 16-byte
  // vectors and their weights per lane, the warps' sums of squares added in warp order through
  // shared memory: the one-warp path of stage_rows leaves three warps idle on the critical path.
  auto stage_one_normed = [&](const bf16* src, const bf16* norm_w, int K) {
    const int chunks = K / 8;
    uint4 v[2], w[2];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = u * kCThreads + tid;
      v[u] = c < chunks ? ldcg16(src + c * 8) : make_uint4(0, 0, 0, 0);
      w[u] = c < chunks ? ldg16(norm_w + c * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float f[8];
      unpack8(v[u], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
    }
    ss = warp_sum(ss);
    if (lane == 0) red_ss[cw] = ss;
    consumers_sync();
    const float r = rsqrtf((red_ss[0] + red_ss[1] + red_ss[2] + red_ss[3]) / static_cast<float>(K) + d.eps);
    if (tid == 0) rstd[0] = r;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = u * kCThreads + tid;
      if (c >= chunks) continue;
      float f[8], wf[8];
      unpack8(v[u], f);
      unpack8(w[u], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * r);
      *reinterpret_cast<uint4*>(xs + c * 8) = pack8(f);
    }
  };

  auto stage = [&](const bf16* src, const bf16* norm_w, int K, const bf16* res = nullptr) {
    if (!TP && B == 1 && norm_w && K <= 2 * 8 * kCThreads && K % 8 == 0 && act_in_smem(K, true)) {
      stage_one_normed(src, norm_w, K);
      consumers_sync();
      mark(2);
      return;
    }
    if (ACT_SMEM && a.bulk_stage && !norm_w) {
      stage_bulk(src, K, a.xres_off ? res : nullptr);
      mark(2);
      return;
    }
    stage_rows(src, K, norm_w, d.eps, B, K, xs, K + kPad, rstd, cw, kConsumers, lane,
               act_in_smem(K, norm_w != nullptr));
    consumers_sync();
    mark(2);
  };

  // (tensor parallel) The residual stream after a row-parallel layer, x = bf16(x_old + bf16(sum
  // over the ranks, in rank order, of their parts in receive slot `slot`)) (slot < 0: x_old as
  // is), staged in shared memory, RMS-normalised with norm_w when non-null; 16-column chunk i of it
  // also goes to x_new (when non-null) from CTA i % grid, so the next residual base is whole after
  // the next grid barrier. The parts are polled line by line (epoch tp_epoch). Every CTA runs it,
  // with or without units. Needs hidden % 512 == 0. false when the step is aborted.
  //
  // A part is [batch][hidden / 16][8 lines]: line q of 16-column group k of row b holds columns
  // 16 k + q and 16 k + q + 8 (the pair one lane of the row-block epilogue owns).
  auto stage_tp = [&](const bf16* x_old, bf16* x_new, int slot, const bf16* norm_w) -> bool {
    TpStage st{x_old,     x_new, slot >= 0 ? my_region + a.recv_x + static_cast<size_t>(slot) * d.tp_world * x_part_bytes
                                           : nullptr,
               norm_w,    xs,    red_ss,
               x_part_bytes, tp_epoch, abort_smem};
    tp_stage(a, st, tid);
    mark(2);
    return *abort_smem == 0;
  };

  // (tensor parallel) A row-parallel unit's fp32 sums, as flagged lines, into every rank's receive
  // slot tp_slot (this rank's part).
  auto push_parts = [&](const float (&acc)[2][NT][4], int rb, int first_half, int halves) {
    const int chunks = H / 16;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h >= halves) break;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int b = 8 * j + 2 * t + e;
          if (b >= B) continue;
          const size_t off = a.recv_x + (static_cast<size_t>(tp_slot) * d.tp_world + d.tp_rank) * x_part_bytes +
                             ((static_cast<size_t>(b) * chunks + rb * 2 + first_half + h) * 8 + g) * kTpLine;
          for (int r = 0; r < d.tp_world; ++r)
            st_line(tp_region(d, r) + off, __float_as_uint(acc[h][j][e]), __float_as_uint(acc[h][j][e + 2]), tp_epoch);
        }
    }
  };

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
  const bool res_smem = ACT_SMEM && !TP && a.bulk_stage && a.xres_off != 0;
  AttnSeq attn_seq;  // the attention ring's fills and merges so far (the same in every consumer thread)
  const bool qkv_ready = !TP && a.qkv_ready;

  if (!mbar_wait(&desc_bar, 0, a.err, a.wait_ns)) {
    atomicExch(&a.grid_bar[1], 1u);  // every CTA leaves at its next barrier
    *abort_smem = 1;
  }
  // The step as a sequence of phases, one code path for every weight phase (a single copy of the
  // tile loop in the kernel, whatever the epilogue): phase p of layer p / 5 is QKV (0), attention
  // (1), o_proj (2), gate/up (3), down_proj (4); phase 5 * layers is the LM head.
  const int n_phases = 5 * d.layers + 1;
  int lm_first = 0;
  for (int p = 0; p < n_phases; ++p) {
    const int layer = p / 5, kind = p == 5 * d.layers ? 5 : p % 5;
    const ipe_layer_desc& L = descs[layer < d.layers ? layer : 0];
    if (kind == 1) {
      // attention: items (split, KV head, row) over the CTAs
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
      fa.wait_ns = a.wait_ns;
      const int items = sp.splits * d.kv_heads * B;
      const AttnSmem<G> sm(scratch, attn_bars, a.attn_slots);
      for (int it = static_cast<int>(blockIdx.x); it < items; it += G_) {
        const int split = it % sp.splits, rest = it / sp.splits;
        if (qkv_ready) {
          // every QKV row of this item's KV head written: (G + 2) x 128 rows a layer, 16 a tick
          if (tid == 0) {
            const unsigned target = static_cast<unsigned>((G + 2) * 8 * (layer + 1));
            const unsigned* word = &a.grid_bar[kReadyWord + rest % d.kv_heads];
            uint64_t start = 0;
            for (unsigned i = 0;; ++i) {
              if (ld_acquire(word) >= target) break;
              if ((i & 63u) == 63u) {
                if (ld_acquire(&a.grid_bar[1])) {
                  *abort_smem = 1;
                  break;
                }
                const uint64_t now = globaltimer_ns();
                if (start == 0) start = now;
                else if (now - start > a.wait_ns) {
                  report(a.err, kErrWaitTimeout);
                  atomicExch(&a.grid_bar[1], 1u);
                  *abort_smem = 1;
                  break;
                }
              }
            }
          }
          consumers_sync();
          if (*abort_smem != 0) return;
        }
        // the first item's milestones: K / V requested and q ready, scores and P.V done, merged
        fa.trace = trace && it == static_cast<int>(blockIdx.x) ? trace + 1 + 5 * (barrier_index - 1) + 2 : nullptr;
        attention_item<G>(fa, split, rest % d.kv_heads, rest / d.kv_heads, pos, sp, sm, attn_seq, tid);
        mark(4);
      }
      if (!phase_end(true)) return;
      continue;
    }
    // The weight phase's input rows, normalisation, epilogue and whether a grid barrier ends it.
    // Tensor parallel: the residual stream alternates between x and x_alt around the row-parallel
    // phases (o_proj, down_proj), whose parts go to every rank and end without a barrier.
    const bf16* src;
    const bf16* norm_w;
    int K, epi;
    EpilogueArgs ea{x, H, H, B, nullptr, nullptr, 0.f, 0};
    bool barrier = true;
    switch (kind) {
      case 0:
        src = x, norm_w = static_cast<const bf16*>(L.input_layernorm), K = H, epi = kGemvStore;
        ea = EpilogueArgs{qkv, QKV, QKV, B, nullptr, nullptr, 0.f, 0};
        barrier = !qkv_ready;  // the attention items wait for their own head's rows instead
        break;
      case 2:
        src = attn, norm_w = nullptr, K = Q, epi = kGemvResidual, barrier = !tp;
        tp_slot = 0;
        ++tp_epoch;
        break;
      case 3:
        src = x, norm_w = static_cast<const bf16*>(L.post_attention_layernorm), K = H, epi = kGemvSiluMul;
        ea = EpilogueArgs{act, I, 2 * I, B, nullptr, nullptr, 0.f, 0};
        break;
      case 4:
        src = act, norm_w = nullptr, K = I, epi = kGemvResidual, barrier = !tp;
        tp_slot = 1;
        ++tp_epoch;
        break;
      default:  // the final RMSNorm + tied LM head: fp32 logits and one sampling record per 32 rows
        src = x, norm_w = static_cast<const bf16*>(d.final_norm), K = H, epi = kGemvLogits;
        ea = EpilogueArgs{d.logits, d.vocab, d.vocab, B, d.partials, state, 0.f, 0};
        ea.row_offset = d.vocab_offset;
        break;
    }
    if (epi == kGemvResidual && res_smem) ea.res_smem = xres;  // x += bf16(sum), x from its staged copy
    if (tp && norm_w) {
      const bool ok_stage = kind == 0   ? stage_tp(x, static_cast<bf16*>(d.x_alt), layer == 0 ? -1 : 1, norm_w)
                            : kind == 3 ? stage_tp(static_cast<const bf16*>(d.x_alt), x, 0, norm_w)
                                        : stage_tp(x, nullptr, 1, norm_w);
      if (!ok_stage) return;
      if (kind == 5) ++tp_epoch;
    } else {
      stage(src, norm_w, K, epi == kGemvResidual ? x : nullptr);
    }
    const PhaseShape ph = phase_shape(layer, kind == 5 ? 0 : kind - (kind > 1 ? 1 : 0));
    if (kind == 5) lm_first = first_unit(cursor);

    // This CTA's units of the phase; within a stage, warp w takes half tiles w and w + 4.
    const bool smem_act = act_in_smem(K, norm_w != nullptr);
    float my_rstd[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) my_rstd[j] = (!smem_act && norm_w && 8 * j + g < B) ? rstd[8 * j + g] : 1.f;
    bool first = true;
    const int n_ht = ph.half_tiles();
    int units_here = 0;
    for (int u = first_unit(cursor); u < ph.units; u += G_, ++units_here) {
      // per half (full unit: half 0, half 1; half unit: [0]) CH independent MMA chains
      constexpr int CH = NT == 1 ? 4 : 2;
      float acc4[2][CH][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < CH; ++c)
#pragma unroll
          for (int j = 0; j < NT; ++j) acc4[h][c][j][0] = acc4[h][c][j][1] = acc4[h][c][j][2] = acc4[h][c][j][3] = 0.f;
      for (int s0 = 0; s0 < n_ht; s0 += kStageTiles) {
        const int slot = mine.slot;
        const uint32_t base = smem_addr(ring + static_cast<size_t>(slot) * kStageBytes);
        // this warp's half tiles of the stage are w and w + 4; the first one's activations are
        // loaded before the wait. Every warp waits for every fill of every stage, with a tile in it
        // or not, so no warp's parity wait can run a phase ahead of the barrier.
        uint4 xv[4][NT];
        const int j0 = s0 + cw;
        const int h0 = (!ph.half && j0 >= ph.ku) ? 1 : 0;
        if (j0 < n_ht) load_activations<NT>(xv, (j0 - h0 * ph.ku) * kTileK, smem_act, xs, src, norm_w, my_rstd, K, kPad,
                                            B, g, t);
        if (!mbar_wait(&full[slot], mine.fill & 1, a.err, a.wait_ns)) {
          *abort_smem = 1;  // every warp leaves the phase together, after the barrier below
          break;
        }
        if (trace) {
          if (first) mark(3);
          mark(4);
          first = false;
        }
        if (j0 < n_ht) {
          if (h0 == 0) consume_half_chains<NT, CH>(acc4[0], base + cw * kHalfTileBytes, xv, g, t);
          else consume_half_chains<NT, CH>(acc4[1], base + cw * kHalfTileBytes, xv, g, t);
        }
        const int j1 = j0 + kConsumers;
        if (j1 < n_ht) {
          const int h1 = (!ph.half && j1 >= ph.ku) ? 1 : 0;
          load_activations<NT>(xv, (j1 - h1 * ph.ku) * kTileK, smem_act, xs, src, norm_w, my_rstd, K, kPad, B, g, t);
          if (h1 == 0) consume_half_chains<NT, CH>(acc4[0], base + (cw + kConsumers) * kHalfTileBytes, xv, g, t);
          else consume_half_chains<NT, CH>(acc4[1], base + (cw + kConsumers) * kHalfTileBytes, xv, g, t);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        mine.advance(S);
      }
      // The warps' sums per half (half unit: [0]) go to shared memory, then one warp adds them in a
      // fixed order and runs the epilogue: a different warp for each unit (this CTA's k-th unit of
      // the phase: warp k % 4), so that no warp falls behind the others by more than one epilogue
      // (every stage waits for all four). Units alternate between two partial-sum buffers; with
      // overlap_epilogue the other warps go on to the next unit's stages meanwhile, and the barrier
      // after the next unit's partials orders the epilogue's reads of this buffer before its reuse.
      float* red_u = red + (red_flip++ & 1u) * (kConsumers * 32 * 8 * NT);
      {
        float* part = red_u + (cw * 32 + lane) * 8 * NT;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float sum = acc4[h][0][j][e];
#pragma unroll
              for (int c = 1; c < CH; ++c) sum += acc4[h][c][j][e];
              part[(h * NT + j) * 4 + e] = sum;
            }
      }
      consumers_sync();
      if (*abort_smem != 0) return;
      if (cw == units_here % kConsumers && epi == kGemvLogits) {
        logits_epilogue<NT>(red_u, u, lane, ea);
      } else if (cw == units_here % kConsumers) {
        float acc[2][NT][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float sum = 0.f;
#pragma unroll
              for (int w = 0; w < kConsumers; ++w) sum += red_u[(w * 32 + lane) * 8 * NT + (h * NT + j) * 4 + e];
              acc[h][j][e] = sum;
            }
        const int rb = ph.half ? u >> 1 : u, first_half = ph.half ? (u & 1) : 0, halves = ph.half ? 1 : 2;
        if (epi == kGemvResidual && tp) push_parts(acc, rb, first_half, halves);  // this rank's part
        else if (epi == kGemvStore) {
          row_block_epilogue<kGemvStore, NT>(acc, rb, lane, ea, first_half, halves);
          if (qkv_ready) {  // this unit's QKV rows are written: count them (16 rows a tick) for their KV head
            __syncwarp();
            if (lane == 0) {
              const int r0 = rb * 32 + first_half * 16, kvr = d.kv_heads * 128;
              const int h = r0 < Q ? r0 / (Q / d.kv_heads) : (r0 < Q + kvr ? (r0 - Q) / 128 : (r0 - Q - kvr) / 128);
              asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(&a.grid_bar[kReadyWord + h]),
                           "r"(static_cast<unsigned>(halves))
                           : "memory");
            }
          }
        }
        else if (epi == kGemvResidual) row_block_epilogue<kGemvResidual, NT>(acc, rb, lane, ea, first_half, halves);
        else row_block_epilogue<kGemvSiluMul, NT>(acc, rb, lane, ea);
      }
      if (!a.overlap_epilogue) consumers_sync();
    }
    if (a.overlap_epilogue) consumers_sync();  // the last epilogue of the phase is done
    cursor = (cursor + ph.units) % G_;
    // the attention ring's bulk copies overwrite the scratch this phase staged: every thread's
    // generic writes of it go before them
    if (kind == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (kind != 5 && !phase_end(barrier)) return;
  }
  {
    const PhaseShape lm = phase_shape(d.layers, 0);
    // rows over the consumer warps; this CTA's units lane-strided, then the lanes in a fixed tree
    for (int b = cw; b < B; b += kConsumers) {
      Stat st = empty_stat();
      for (int u = lm_first + lane * G_; u < lm.units; u += 32 * G_)
        st = merge(st, load_stat(d.partials + (static_cast<int64_t>(u) * B + b) * IPE_PARTIAL_WORDS));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) st = merge(st, shfl_xor_stat(st, o));
      if (lane == 0) {
        if (tp) {
          const size_t off = a.recv_rec + ((static_cast<size_t>(d.tp_rank) * G_ + blockIdx.x) * B + b) * kTpRecordBytes;
          for (int r = 0; r < d.tp_world; ++r) {
            unsigned char* dst = tp_region(d, r) + off;
            st_line(dst, __float_as_uint(st.m), __float_as_uint(st.s), tp_epoch);
            st_line(dst + kTpLine, __float_as_uint(st.gs), __float_as_uint(st.gl), tp_epoch);
            st_line(dst + 2 * kTpLine, static_cast<uint32_t>(st.arg), static_cast<uint32_t>(st.garg), tp_epoch);
          }
        } else {
          float* rec = a.cta_records + (static_cast<int64_t>(blockIdx.x) * B + b) * IPE_PARTIAL_WORDS;
          rec[0] = st.m;
          rec[1] = st.s;
          rec[2] = st.gs;
          rec[3] = st.gl;
          rec[4] = __int_as_float(st.arg);
          rec[5] = __int_as_float(st.garg);
        }
      }
    }
  }
  // Tensor parallel: no barrier; CTA 0 polls every rank's records, each pushed after its
  // epilogues read the step state, so the state may change once they are all in.
  if (!phase_end(!tp)) return;
  if (trace && tid == 0) trace[IPE_TRACE_WORDS(d.layers) - 2] = globaltimer_ns();
  if (blockIdx.x != 0) return;

  // Sampling (CTA 0): token and untempered log-probability per row, fed back as the next input.
  // Tensor parallel: over every rank's records (the same on every rank); the chosen token's logit
  // then comes from the records.
  const int parts = tp ? d.tp_world * G_ : G_;  // the CTAs' merged records
  bool ok = true;
  if (d.history_tokens) {
    const float temperature = __int_as_float(static_cast<int>(state[IPE_STATE_TEMPERATURE]));
    const int64_t step = state[IPE_STATE_STEP];
    for (int b = cw; b < B; b += kConsumers) {
      Stat st = empty_stat();
      if (tp) {
        const MergedRecords m = tp_merge_records(a, my_region + a.recv_rec, parts, b, lane, tp_epoch);
        st = m.st;
        ok = ok && m.ok;
      } else {
        for (int p = lane; p < parts; p += 32)
          st = merge(st, load_stat(a.cta_records + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) st = merge(st, shfl_xor_stat(st, o));
      if (lane == 0 && ok) {
        const int token = temperature > 0.f ? st.garg : st.arg;
        const float logit = tp ? (temperature > 0.f ? st.gl : st.m)
                               : __ldcg(d.logits + static_cast<int64_t>(b) * d.vocab + token);
        d.history_tokens[b * d.history_stride + step] = token;
        d.history_logprobs[b * d.history_stride + step] = (logit - st.m) - logf(st.s);
        d.tokens[b] = token;
      }
    }
  }
  if (!ok) *abort_smem = 1;
  consumers_sync();
  if (tid == 0 && *abort_smem == 0) {
    if (d.history_tokens) state[IPE_STATE_STEP] += 1;
    state[IPE_STATE_POS] = pos + 1;
    if (tp) *reinterpret_cast<unsigned*>(my_region + kTpCounter) = tp_epoch;  // the next step's epochs follow
  }
  if (trace && tid == 0) trace[IPE_TRACE_WORDS(d.layers) - 1] = globaltimer_ns();
}


template <int NT, int G, bool ACT, bool TP>
cudaError_t launch_variant(const StepArgs& a, size_t smem, cudaStream_t stream) {
  auto kernel = decode_step_kernel<NT, G, ACT, TP>;
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

template <int NT, bool ACT, bool TP>
cudaError_t by_group(const StepArgs& a, size_t smem, cudaStream_t stream) {
  switch (a.d.q_heads / a.d.kv_heads) {
    case 1: return launch_variant<NT, 1, ACT, TP>(a, smem, stream);
    case 2: return launch_variant<NT, 2, ACT, TP>(a, smem, stream);
    case 4: return launch_variant<NT, 4, ACT, TP>(a, smem, stream);
    case 8: return launch_variant<NT, 8, ACT, TP>(a, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

// Tuning of the weight stream, fixed per process (measured on B200 with Qwen3-1.7B at batch 1, a
// 512-token context): 32 KB ring stages (IPE_STEP_STAGES, 6, fewer when the activations need the
// room), the producer's L2 prefetch of each layer's K / V rows and norm weights
// (IPE_STEP_PREFETCH_KV, 0), weight copies marked L2 evict-first (IPE_STEP_EVICT_FIRST, 1),
// half-row-block units (IPE_STEP_HALF, 1), bulk-copy staging of the o_proj / down_proj rows with
// the residual rows beside them (IPE_STEP_BULK, 1), the grid barrier's arrival
// (IPE_STEP_LIGHT_FENCES, 2: a release reduction and a poll of the count alone; batch 1 / 4 / 16
// 1127.9 / 1397.2 / 3073.5 -> 1100.8 / 1374.2 / 3048.5 us per step against 1, an acq_rel fence and
// an atomic with a poll that also read the abort flag every time; one box, alternating runs), the unit epilogue overlapped with the next unit's tiles
// (IPE_STEP_OVERLAP, 1), per-KV-head readiness counters instead of the grid barrier after the QKV
// phase (IPE_STEP_QKV_READY, 1: batch 1 / 4 / 16 1129.3 / 1416.6 / 3078.6 -> 1118.8 / 1399.1 /
// 3064.0 us per step, one box, alternating runs), a cap on the attention splits per (row, KV head)
// (IPE_STEP_ATTN_SPLITS, 0 = none: as many as fill the grid measured fastest, batch 1 1119.1 us
// against 1147.6 with 9 and 1174.2 with 6), the attention items' K / V ring slots at most (IPE_STEP_ATTN_SLOTS, 4;
// as many as fit beside the weight stages), and the stages the producer keeps prefetched into L2
// past its copies (IPE_STEP_L2_AHEAD, 0). With the attention items streaming their K / V rows
// through their own ring, both prefetches off measured fastest (batch 1 / 4 / 16: 1116.4 / 1390.8
// / 3184.8 us per step against 1136.8 / 1404.3 / 3234.1 with both on, one box, medians of 3 and
// 2 runs): the per-layer K / V burst delayed the grid barrier that precedes it.
struct StepTuning {
  int stages = 6;
  int prefetch_kv = 0;
  int evict_first = 1;
  int halves = 1;
  int bulk = 1;
  int light_fences = 2;
  int overlap_epilogue = 1;
  int attn_slots = 4;
  int l2_ahead = 0;
  int qkv_ready = 1;
  int attn_splits = 0;
};

const StepTuning& tuning() {
  static const StepTuning t = [] {
    StepTuning r;
    if (const char* v = std::getenv("IPE_STEP_STAGES")) r.stages = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_PREFETCH_KV")) r.prefetch_kv = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_EVICT_FIRST")) r.evict_first = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_HALF")) r.halves = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_BULK")) r.bulk = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_LIGHT_FENCES")) r.light_fences = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_OVERLAP")) r.overlap_epilogue = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_ATTN_SLOTS")) r.attn_slots = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_L2_AHEAD")) r.l2_ahead = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_QKV_READY")) r.qkv_ready = std::atoi(v);
    if (const char* v = std::getenv("IPE_STEP_ATTN_SPLITS")) r.attn_splits = std::atoi(v);
    return r;
  }();
  return t;
}

// The dynamic shared memory before the scratch: alignment slack, the ring, its barriers, the RMS
// scales, the abort flag, the partial sums and the layer descriptors.
size_t fixed_smem(int nt, int stages, int layers) {
  return 1024 + static_cast<size_t>(stages) * kStageBytes + 2 * kMaxStages * 8 + 16 * 4 + 16 +
         2 * static_cast<size_t>(kConsumers) * 32 * 8 * nt * 4 + static_cast<size_t>(layers) * sizeof(ipe_layer_desc);
}
static_assert(sizeof(ipe_layer_desc) % 16 == 0, "layer descriptors keep the scratch 16-byte aligned");

size_t attn_bytes(int group, int slots) {
  switch (group) {
    case 1: return attn_smem_floats<1>(slots) * 4;
    case 2: return attn_smem_floats<2>(slots) * 4;
    case 4: return attn_smem_floats<4>(slots) * 4;
    default: return attn_smem_floats<8>(slots) * 4;
  }
}

}  // namespace

// Receive slots of the row-parallel parts: 2 slots x world parts x batch x hidden / 2 lines.
size_t tp_parts_bytes(int world, int batch, int hidden) {
  return (2ull * world * batch * (hidden / 2) * kTpLine + 255) / 256 * 256;
}

size_t decode_step_comm_bytes(int world, int batch, int hidden) {
  return kTpRecv + tp_parts_bytes(world, batch, hidden) +
         static_cast<size_t>(world) * sm_count() * batch * kTpRecordBytes;
}

// [256 barrier words][attention counters][attention records][the CTAs' merged LM-head records]
size_t decode_step_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity) {
  (void)capacity;  // attention records are per split, at most kAttnSplitsMax of them
  const size_t counters = (static_cast<size_t>(batch) * kv_heads * sizeof(int) + 255) / 256 * 256;
  const size_t records =
      (static_cast<size_t>(batch) * q_heads * kAttnSplitsMax * kAttnRecord * sizeof(float) + 255) / 256 * 256;
  return 256 + counters + records + static_cast<size_t>(sm_count()) * batch * IPE_PARTIAL_WORDS * sizeof(float);
}

cudaError_t launch_decode_step(const ipe_decode_step_desc& d, int* err, cudaStream_t stream, const char** message) {
  StepArgs a{};
  a.d = d;
  a.err = err;
  a.wait_ns = d.wait_limit_ns > 0 ? static_cast<uint64_t>(d.wait_limit_ns) : kWaitLimitNs;
  unsigned char* ws = static_cast<unsigned char*>(d.workspace);
  a.grid_bar = reinterpret_cast<unsigned*>(ws);
  a.attn_counters = reinterpret_cast<int*>(ws + 256);
  const size_t counters = (static_cast<size_t>(d.batch) * d.kv_heads * sizeof(int) + 255) / 256 * 256;
  a.attn_records = reinterpret_cast<float*>(ws + 256 + counters);
  const size_t records =
      (static_cast<size_t>(d.batch) * d.q_heads * kAttnSplitsMax * kAttnRecord * sizeof(float) + 255) / 256 * 256;
  a.cta_records = reinterpret_cast<float*>(ws + 256 + counters + records);
  const int nt = d.batch <= 8 ? 1 : 2;
  const int group = d.q_heads / d.kv_heads;
  const size_t act = static_cast<size_t>(d.batch) *
                     (std::max(std::max(d.hidden, d.intermediate), d.q_heads * 128) + kPad) * 2;
  const size_t attn1 = attn_bytes(group, kAttnSlotsMin);
  // Activations stay in shared memory when that leaves room for 4 ring stages. When
  // the widest rows do not fit (a larger batch), the RMS-normalised phases (QKV, gate/up, the LM
  // head; reduction width `hidden`) still stage theirs if those fit.
  const bool act_smem = fixed_smem(nt, 4, d.layers) + std::max(act, attn1) <= kSmemMax;
  const size_t act_h = static_cast<size_t>(d.batch) * (d.hidden + kPad) * 2;
  const bool act_h_smem = !act_smem && fixed_smem(nt, 4, d.layers) + std::max(act_h, attn1) <= kSmemMax;
  a.act_cols = act_h_smem ? d.hidden : 0;
  // Bulk staging copies whole rows of the attention output and the SiLU product: 16-byte aligned
  // buffers and widths.
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  a.bulk_stage = tuning().bulk && d.tp_world <= 1 && aligned(d.attn) && aligned(d.act) && d.intermediate % 8 == 0 &&
                 (d.q_heads * 128) % 8 == 0;
  // The scratch: the activation rows or the attention scratch (whichever is larger), then, with
  // bulk-staged o_proj / down_proj phases, a copy of the residual rows when that still leaves 4
  // ring stages.
  const size_t act_part = act_smem ? act : act_h_smem ? act_h : 0;
  const size_t xres_bytes = static_cast<size_t>(d.batch) * d.hidden * 2;
  auto round16 = [](size_t v) { return (v + 15) / 16 * 16; };
  auto base_scratch = [&](int slots) { return std::max(act_part, attn_bytes(group, slots)); };
  const bool xres = act_smem && a.bulk_stage && aligned(d.x) && d.hidden % 8 == 0 &&
                    fixed_smem(nt, 4, d.layers) + round16(base_scratch(kAttnSlotsMin)) + xres_bytes <= kSmemMax;
  auto scratch_with = [&](int slots) { return xres ? round16(base_scratch(slots)) + xres_bytes : base_scratch(slots); };
  int stages = std::min(kMaxStages, std::max(2, tuning().stages));
  while (stages > 2 && fixed_smem(nt, stages, d.layers) + scratch_with(kAttnSlotsMin) > kSmemMax) --stages;
  a.stages = stages;
  // The attention ring (kAttnSlotsMin slots at least) grows into what the weight stages leave.
  int slots = kAttnSlotsMin;
  while (slots < std::min(kAttnSlotsMax, std::max(kAttnSlotsMin, tuning().attn_slots)) &&
         fixed_smem(nt, stages, d.layers) + scratch_with(slots + 1) <= kSmemMax)
    ++slots;
  a.attn_slots = slots;
  a.max_splits = std::min(attn_max_splits(sm_count(), d.batch, d.kv_heads), attn_merge_splits(group, slots));
  if (tuning().attn_splits > 0) a.max_splits = std::min(a.max_splits, tuning().attn_splits);
  a.xres_off = xres ? static_cast<unsigned>(round16(base_scratch(slots))) : 0u;
  const size_t scratch = scratch_with(slots);
  a.prefetch_kv = tuning().prefetch_kv;
  a.l2_ahead = std::max(0, std::min(64, tuning().l2_ahead));
  a.qkv_ready = tuning().qkv_ready && d.tp_world <= 1 && d.kv_heads <= kReadyHeadsMax;
  a.evict_first = tuning().evict_first;
  a.halves = tuning().halves;
  a.light_fences = tuning().light_fences;
  a.overlap_epilogue = tuning().overlap_epilogue;
  const size_t smem = fixed_smem(nt, stages, d.layers) + scratch;
  if (smem > kSmemMax) {
    *message = "decode-step scratch does not fit in shared memory";
    return cudaErrorInvalidValue;
  }
  if (d.tp_world > 1) {
    if (!act_smem || d.hidden % 512) {
      *message = "tensor parallel: needs hidden % 512 == 0 and the activations in shared memory (a smaller batch)";
      return cudaErrorInvalidValue;
    }
    a.recv_x = kTpRecv;
    a.recv_rec = a.recv_x + tp_parts_bytes(d.tp_world, d.batch, d.hidden);
  }
  // the grid barrier counts arrivals from zero every step ([0] arrivals, [1] abort)
  cudaError_t e = cudaMemsetAsync(a.grid_bar, 0, (a.qkv_ready ? 64 : 2) * sizeof(unsigned), stream);
  if (e != cudaSuccess) return e;
  if (d.tp_world > 1) return nt == 1 ? by_group<1, true, true>(a, smem, stream) : by_group<2, true, true>(a, smem, stream);
  if (nt == 1) return act_smem ? by_group<1, true, false>(a, smem, stream) : by_group<1, false, false>(a, smem, stream);
  return act_smem ? by_group<2, true, false>(a, smem, stream) : by_group<2, false, false>(a, smem, stream);
}

}  // namespace ipe
