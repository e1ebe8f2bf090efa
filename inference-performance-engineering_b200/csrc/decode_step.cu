// One whole decode step in one persistent kernel: embedding, every layer's QKV projection
// (RMSNorm fused), attention (q/k norm + RoPE + KV append + split-KV), o_proj + residual,
// RMSNorm + gate/up + SiLU*up, down_proj + residual, the final norm + tied LM head with fp32
// logits and sampling records, and (optionally) the sampled token fed back for the next step.
//
// Why one kernel: every weight byte of the step is known before the step starts, so the weight
// stream does not depend on activations. Each CTA (one per SM, cooperative launch) has a producer
// warp that walks its share of ALL phases' decode tiles back to back with 8 KB bulk copies into
// per-consumer-warp shared-memory slots, and never waits for a phase boundary; the HBM stream
// continues across the whole step. The 4 consumer warps wait only where the data requires it: at
// a bounded-spin grid barrier after each phase (the next phase needs the full activation vector),
// then they stage that vector in shared memory and consume tiles that are usually already there.
//
// Work split: a phase's row blocks (32 weight rows each, whole K, no split-K) are dealt
// round-robin over the CTAs, continuing where the previous phase stopped so every CTA streams
// the same number of row blocks per step; within a CTA a row block's tiles go round-robin to the
// consumer warps, whose partial sums are reduced in a fixed order through shared memory
// (deterministic). Every spin (grid barrier, mbarrier) is bounded; a timeout sets the device error
// word and an abort flag and the kernel winds down.
#include <algorithm>
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
constexpr int kSlotsPerWarp = 4;
constexpr int kStages = kConsumers * kSlotsPerWarp;  // 16 x 8 KB = 128 KB of weights in flight
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kCThreads = 32 * kConsumers;
constexpr int kPad = 32;
constexpr int kStepBarrier = 1;  // named barrier id of the consumer warps
constexpr size_t kSmemMax = 227 * 1024;

struct StepArgs {
  ipe_decode_step_desc d;
  unsigned* grid_bar;  // [0] arrivals, [1] abort flag
  int* attn_counters;
  float* attn_records;
  int* err;
  int chunks_max;
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
__device__ bool grid_sync(const StepArgs& a, unsigned index, int tid, int* abort_smem) {
  consumers_sync();
  if (tid == 0) {
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
  }
  consumers_sync();
  return *abort_smem == 0;
}

// First row block of this CTA in a phase that starts dealing at `cursor`.
__device__ __forceinline__ int first_row_block(int cursor) {
  const int g = static_cast<int>(gridDim.x);
  return (static_cast<int>(blockIdx.x) - cursor % g + g) % g;
}

struct PhaseShape {
  const unsigned char* tiles;
  int row_blocks;
  int ku;  // tiles per row block
};

template <int NT, int G, bool ACT_SMEM>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const StepArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * kTileBytes);
  uint64_t* empty = full + kStages;
  float* rstd = reinterpret_cast<float*>(empty + kStages);  // [16]
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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_smem = 0;
    fence_barrier_init();
  }
  __syncthreads();

  auto phase_shape = [&](int layer, int kind) -> PhaseShape {
    if (layer == d.layers) return {static_cast<const unsigned char*>(d.lm_head_tiles), (d.vocab + 31) / 32, H / kTileK};
    const ipe_layer_desc& L = d.layer_descs[layer];
    switch (kind) {
      case 0: return {static_cast<const unsigned char*>(L.qkv_tiles), QKV / 32, H / kTileK};
      case 1: return {static_cast<const unsigned char*>(L.o_tiles), H / 32, Q / kTileK};
      case 2: return {static_cast<const unsigned char*>(L.gate_up_tiles), I / 16, H / kTileK};
      default: return {static_cast<const unsigned char*>(L.down_tiles), H / 32, I / kTileK};
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t ring_base = smem_addr(ring);
      int kcount[kConsumers] = {0, 0, 0, 0};
      int cursor = 0;
      bool ok = true;
      for (int layer = 0; layer <= d.layers && ok; ++layer) {
        for (int kind = 0; kind < (layer == d.layers ? 1 : 4) && ok; ++kind) {
          const PhaseShape ph = phase_shape(layer, kind);
          for (int rb = first_row_block(cursor); rb < ph.row_blocks && ok; rb += G_) {
            const unsigned char* src = ph.tiles + static_cast<int64_t>(rb) * ph.ku * kTileBytes;
            for (int t0 = 0; t0 < ph.ku && ok; t0 += kConsumers) {
#pragma unroll
              for (int w = 0; w < kConsumers; ++w) {
                const int t = t0 + w;
                if (t >= ph.ku || !ok) continue;
                const int k = kcount[w]++;
                const int slot = w * kSlotsPerWarp + (k & (kSlotsPerWarp - 1));
                const int fill = k / kSlotsPerWarp;
                if (fill > 0 && !mbar_wait(&empty[slot], (fill - 1) & 1, a.err)) {
                  ok = false;
                  continue;
                }
                mbar_expect_tx(&full[slot], kTileBytes);
                bulk_copy(ring_base + slot * kTileBytes, src + static_cast<int64_t>(t) * kTileBytes, kTileBytes,
                          &full[slot]);
              }
            }
          }
          cursor = (cursor + ph.row_blocks) % G_;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cw = warp - 1, tid = threadIdx.x - 32;
  const int g = lane >> 2, t = lane & 3;
  int kcount = 0, cursor = 0;
  unsigned barrier_index = 0;
  int64_t* state = d.state;

  // Embedding: x[b] = embed[tokens[b]] (out-of-range IDs give zeros and set device error 1).
  {
    const int vecs = H / 8;
    bf16* x = static_cast<bf16*>(d.x);
    for (int i = static_cast<int>(blockIdx.x) * kCThreads + tid; i < B * vecs; i += G_ * kCThreads) {
      const int b = i / vecs, v = i % vecs;
      const int64_t id = d.tokens[b];
      uint4 val = make_uint4(0, 0, 0, 0);
      if (id >= 0 && id < d.vocab) val = ldg16(static_cast<const bf16*>(d.embed) + id * H + v * 8);
      else if (v == 0) report(a.err, kErrTokenRange);
      *reinterpret_cast<uint4*>(x + static_cast<int64_t>(b) * H + v * 8) = val;
    }
  }
  if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;

  // Stage the activation rows of a phase (optionally RMS-normalised) in shared memory; without
  // shared staging only the RMS scales are kept and tiles read activations from global memory.
  auto stage = [&](const bf16* src, const bf16* norm_w, int K) {
    for (int b = cw; b < B; b += kConsumers) {
      const bf16* xr = src + static_cast<int64_t>(b) * K;
      float r = 1.f;
      if (norm_w) {
        float ss = 0.f;
        for (int c = lane; c < K / 8; c += 32) {
          float f[8];
          unpack8(ldcg16(xr + c * 8), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
        }
        ss = warp_sum(ss);
        r = rsqrtf(ss / static_cast<float>(K) + d.eps);
        if (lane == 0) rstd[b] = r;
      }
      if constexpr (ACT_SMEM) {
        for (int c = lane; c < K / 8; c += 32) {
          uint4 v = ldcg16(xr + c * 8);
          if (norm_w) {
            float f[8], wf[8];
            unpack8(v, f);
            unpack8(ldg16(norm_w + c * 8), wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * r);
            v = pack8(f);
          }
          *reinterpret_cast<uint4*>(xs + b * (K + kPad) + c * 8) = v;
        }
      }
    }
    consumers_sync();
  };

  // One weight phase: this CTA's row blocks, tiles round-robin over the consumer warps.
  auto run_phase = [&](auto epi_tag, const PhaseShape& ph, const bf16* src, const bf16* norm_w, int K,
                       const EpilogueArgs& ea) -> bool {
    constexpr int EPI = decltype(epi_tag)::value;
    float my_rstd[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) my_rstd[j] = (!ACT_SMEM && norm_w && 8 * j + g < B) ? rstd[8 * j + g] : 1.f;
    bool ok = true;
    for (int rb = first_row_block(cursor); rb < ph.row_blocks; rb += G_) {
      float acc[2][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[h][j][0] = acc[h][j][1] = acc[h][j][2] = acc[h][j][3] = 0.f;
      for (int tt = cw; tt < ph.ku && ok; tt += kConsumers) {
        const int k = kcount++;
        const int slot = cw * kSlotsPerWarp + (k & (kSlotsPerWarp - 1));
        const int fill = k / kSlotsPerWarp;
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
        if (!mbar_wait(&full[slot], fill & 1, a.err)) {
          ok = false;
          break;
        }
        consume_tile<NT>(acc, smem_addr(ring + slot * kTileBytes), xv, g, t);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      // Fixed-order reduction of the warps' partial sums, then the epilogue by warp 0.
      float* mine = red + (cw * 32 + lane) * 8 * NT;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) mine[(h * NT + j) * 4 + e] = acc[h][j][e];
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
        row_block_epilogue<EPI, NT>(acc, rb, lane, ea);
      }
      consumers_sync();
      if (!ok) return false;
    }
    cursor = (cursor + ph.row_blocks) % G_;
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

  for (int layer = 0; layer < d.layers; ++layer) {
    const ipe_layer_desc& L = d.layer_descs[layer];
    // QKV projection (input RMSNorm fused)
    stage(x, static_cast<const bf16*>(L.input_layernorm), H);
    if (!run_phase(EpiStore{}, phase_shape(layer, 0), x, static_cast<const bf16*>(L.input_layernorm), H,
                   EpilogueArgs{qkv, QKV, QKV, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;
    // attention: items (chunk, KV head, row) over the CTAs
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
      fa.chunks_max = a.chunks_max;
      fa.eps = d.eps;
      fa.err = a.err;
      const int chunks = pos / kAttnChunk + 1;
      const int items = chunks * d.kv_heads * B;
      const AttnSmem<G> sm(scratch, a.chunks_max);
      for (int it = static_cast<int>(blockIdx.x); it < items; it += G_) {
        const int chunk = it % chunks, rest = it / chunks;
        attention_item<G>(fa, chunk, rest % d.kv_heads, rest / d.kv_heads, pos, sm, tid);
      }
    }
    if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;
    // o_proj + residual
    stage(attn, nullptr, Q);
    if (!run_phase(EpiResidual{}, phase_shape(layer, 1), attn, nullptr, Q,
                   EpilogueArgs{x, H, H, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;
    // post-attention RMSNorm + gate/up + SiLU * up
    stage(x, static_cast<const bf16*>(L.post_attention_layernorm), H);
    if (!run_phase(EpiSilu{}, phase_shape(layer, 2), x, static_cast<const bf16*>(L.post_attention_layernorm), H,
                   EpilogueArgs{act, I, 2 * I, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;
    // down_proj + residual
    stage(act, nullptr, I);
    if (!run_phase(EpiResidual{}, phase_shape(layer, 3), act, nullptr, I,
                   EpilogueArgs{x, H, H, B, nullptr, nullptr, 0.f, 0}))
      return;
    if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;
  }
  // final RMSNorm + tied LM head: fp32 logits and one sampling record per 32 vocabulary rows
  stage(x, static_cast<const bf16*>(d.final_norm), H);
  if (!run_phase(EpiLogits{}, phase_shape(d.layers, 0), x, static_cast<const bf16*>(d.final_norm), H,
                 EpilogueArgs{d.logits, d.vocab, d.vocab, B, d.partials, state, 0.f, 0}))
    return;
  if (!grid_sync(a, ++barrier_index, tid, abort_smem)) return;
  if (blockIdx.x != 0) return;

  // Sampling (CTA 0): token and untempered log-probability per row, fed back as the next input.
  const int parts = (d.vocab + 31) / 32;
  if (d.history_tokens) {
    const float temperature = __int_as_float(static_cast<int>(state[IPE_STATE_TEMPERATURE]));
    const int64_t step = state[IPE_STATE_STEP];
    for (int b = cw; b < B; b += kConsumers) {
      Stat st{-INFINITY, 0.f, 0x7fffffff, -INFINITY, 0x7fffffff};
      for (int p = lane; p < parts; p += 32) {
        const float* rec = d.partials + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS;
        st = merge(st, Stat{__ldcg(rec), __ldcg(rec + 1), __float_as_int(__ldcg(rec + 4)), __ldcg(rec + 2),
                            __float_as_int(__ldcg(rec + 5))});
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        Stat y{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
               __shfl_xor_sync(0xffffffffu, st.arg, o), __shfl_xor_sync(0xffffffffu, st.gs, o),
               __shfl_xor_sync(0xffffffffu, st.garg, o)};
        st = merge(st, y);
      }
      if (lane == 0) {
        const int token = temperature > 0.f ? st.garg : st.arg;
        const float logit = __ldcg(d.logits + static_cast<int64_t>(b) * d.vocab + token);
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

size_t fixed_smem(int nt) {
  return 1024 + static_cast<size_t>(kStages) * kTileBytes + 2 * kStages * 8 + 16 * 4 + 16 +
         static_cast<size_t>(kConsumers) * 32 * 8 * nt * 4;
}

size_t attn_bytes(int group, int chunks_max) {
  switch (group) {
    case 1: return attn_smem_floats<1>(chunks_max) * 4;
    case 2: return attn_smem_floats<2>(chunks_max) * 4;
    case 4: return attn_smem_floats<4>(chunks_max) * 4;
    default: return attn_smem_floats<8>(chunks_max) * 4;
  }
}

}  // namespace

size_t decode_step_workspace_bytes(int batch, int q_heads, int kv_heads, int capacity) {
  const int chunks_max = (capacity + kAttnChunk - 1) / kAttnChunk;
  const size_t counters = (static_cast<size_t>(batch) * kv_heads * sizeof(int) + 255) / 256 * 256;
  return 256 + counters + static_cast<size_t>(batch) * q_heads * chunks_max * kAttnRecord * sizeof(float);
}

cudaError_t launch_decode_step(const ipe_decode_step_desc& d, int* err, cudaStream_t stream, const char** message) {
  StepArgs a{};
  a.d = d;
  a.err = err;
  a.chunks_max = (d.capacity + kAttnChunk - 1) / kAttnChunk;
  unsigned char* ws = static_cast<unsigned char*>(d.workspace);
  a.grid_bar = reinterpret_cast<unsigned*>(ws);
  a.attn_counters = reinterpret_cast<int*>(ws + 256);
  const size_t counters = (static_cast<size_t>(d.batch) * d.kv_heads * sizeof(int) + 255) / 256 * 256;
  a.attn_records = reinterpret_cast<float*>(ws + 256 + counters);
  const int nt = d.batch <= 8 ? 1 : 2;
  const int group = d.q_heads / d.kv_heads;
  const size_t act = static_cast<size_t>(d.batch) *
                     (std::max(std::max(d.hidden, d.intermediate), d.q_heads * 128) + kPad) * 2;
  const size_t attn = attn_bytes(group, a.chunks_max);
  const bool act_smem = fixed_smem(nt) + std::max(act, attn) <= kSmemMax;
  const size_t smem = fixed_smem(nt) + (act_smem ? std::max(act, attn) : attn);
  if (smem > kSmemMax) {
    *message = "attention scratch for this capacity does not fit in shared memory";
    return cudaErrorInvalidValue;
  }
  // the grid barrier counts arrivals from zero every step
  cudaError_t e = cudaMemsetAsync(a.grid_bar, 0, 2 * sizeof(unsigned), stream);
  if (e != cudaSuccess) return e;
  if (nt == 1) return act_smem ? by_group<1, true>(a, smem, stream) : by_group<1, false>(a, smem, stream);
  return act_smem ? by_group<2, true>(a, smem, stream) : by_group<2, false>(a, smem, stream);
}

}  // namespace ipe
