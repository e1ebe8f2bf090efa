// Device pieces shared by the weight-streaming kernels (per-op GEMV and the decode-step kernel):
// the decode-tile format, bulk copies into shared memory, the tensor-core consumption of one tile,
// and the linear-layer epilogues with the reference's rounding points.
//
// Decode tiles: a matrix is cut into row blocks of 32 output rows (for SiLU*up: 16 gate rows, then
// the 16 matching up rows) and each row block into two 16-row halves. A half tile is 16 rows x 128
// reduction columns = 4 KB, laid out [64-column box (2)][row (16)][128 bytes]; in odd rows the two
// 64-byte halves of each 128-byte row segment are swapped (16-byte chunk c stored at c ^ 4). The
// consumers' 16-byte loads are served 8 lanes at a time: lanes (row 2p or 2p + 1, chunk t of a
// 64-byte half) then cover all 32 banks once, with no bank conflict. Half tiles are stored half-major within a row block:
// [row block][half (2)][k tile (K / 128)][4 KB], so a half's whole reduction range, and a row
// block's two halves one after the other, are each one contiguous run of memory that streams in a
// few large bulk copies (a copy's fixed cost makes copies below 16 KB slow: 8 KB copies cap the
// stream near 4.9 TB/s on B200, 32 KB copies reach 7.3 TB/s).
#pragma once

#include "common.cuh"
#include "launch.h"
#include "sampling.cuh"

namespace ipe {

constexpr int kTileBytes = 8192;  // a row block's two half tiles of one 128-column range
constexpr int kHalfTileBytes = 4096;  // 16 rows x 128 bf16
constexpr int kTileBoxBytes = 2048;  // 16 rows x 64 bf16
constexpr int kTileK = 128;

// Stored position of 16-byte chunk `chunk` (0..7) of a tile row: odd rows swap their 64-byte halves.
__host__ __device__ __forceinline__ int swizzle(int chunk, int row) { return chunk ^ ((row & 1) << 2); }

// Byte offset of half tile (row block rb, half h, k tile k) in a matrix with ku k tiles per row.
__host__ __device__ __forceinline__ int64_t half_tile_offset(int64_t rb, int h, int k, int ku) {
  return ((rb * 2 + h) * ku + k) * static_cast<int64_t>(kHalfTileBytes);
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// L2 policy that evicts the lines it covers first (data read once).
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// acc[h][j] += rows (h, g / g+8) of a row block's two half tiles for one k tile, gathered at base
// (half 0) and base + kHalfTileBytes (half 1), x activations xv[c][j] (batch columns 8j..8j+7) over
// the 128 columns. The MMA's K order is permuted identically for A (weights, 16-byte chunk of 8
// consecutive columns per thread) and B (activations, the same 8 columns), so the dot products are
// unchanged while every read is one contiguous 16 bytes.
template <int NT>
__device__ __forceinline__ void consume_tile(float (&acc)[2][NT][4], uint32_t base, const uint4 (&xv)[4][NT], int g,
                                             int t) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int chunk = (c & 1) * 4 + t;
    uint4 w[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = g + 8 * r;
        w[h][r] = lds128(base + h * kHalfTileBytes + (c >> 1) * kTileBoxBytes + row * 128 + (swizzle(chunk, row) << 4));
      }
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        mma16816(acc[h][j], w[h][0].x, w[h][1].x, w[h][0].y, w[h][1].y, xv[c][j].x, xv[c][j].y);
        mma16816(acc[h][j], w[h][0].z, w[h][1].z, w[h][0].w, w[h][1].w, xv[c][j].z, xv[c][j].w);
      }
  }
}

// The same over one 16-row half of a tile, copied alone (4 KB, [box (2)][row (16)][128 bytes]) to
// base: columns 0..63 accumulate into acc[0], 64..127 into acc[1] (two independent MMA chains);
// the caller adds acc[1] into acc[0] when the unit is complete.
template <int NT>
__device__ __forceinline__ void consume_half(float (&acc)[2][NT][4], uint32_t base, const uint4 (&xv)[4][NT], int g,
                                             int t) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int chunk = (c & 1) * 4 + t;
    uint4 w[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      w[r] = lds128(base + (c >> 1) * kTileBoxBytes + row * 128 + (swizzle(chunk, row) << 4));
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      mma16816(acc[c >> 1][j], w[0].x, w[1].x, w[0].y, w[1].y, xv[c][j].x, xv[c][j].y);
      mma16816(acc[c >> 1][j], w[0].z, w[1].z, w[0].w, w[1].w, xv[c][j].z, xv[c][j].w);
    }
  }
}

// acc[m % CH][j] += the 16 rows (g / g+8) of one 4 KB half tile at base x activations xv[c][j]
// over its 128 columns (the same K permutation as consume_tile), the tile's eight MMAs m = 2c + s
// spread over CH independent accumulator chains: a chain of dependent mma.sync waits out the
// instruction's latency at every step, so one long chain per warp limits how fast a warp can
// consume a stage; the caller sums the chains in a fixed order.
template <int NT, int CH>
__device__ __forceinline__ void consume_half_chains(float (&acc)[CH][NT][4], uint32_t base, const uint4 (&xv)[4][NT],
                                                    int g, int t) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int chunk = (c & 1) * 4 + t;
    uint4 w[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      w[r] = lds128(base + (c >> 1) * kTileBoxBytes + row * 128 + (swizzle(chunk, row) << 4));
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      mma16816(acc[(2 * c) % CH][j], w[0].x, w[1].x, w[0].y, w[1].y, xv[c][j].x, xv[c][j].y);
      mma16816(acc[(2 * c + 1) % CH][j], w[0].z, w[1].z, w[0].w, w[1].w, xv[c][j].z, xv[c][j].w);
    }
  }
}

// Stage B activation rows (row b at src + b * src_stride, K wide) in shared memory xs (row stride
// xs_stride), RMS-normalised with weight norm_w when it is non-null: bf16(w * bf16(x * rstd)), the
// reference's two roundings. rstd[b] receives the scale. The nwarps calling warps issue 8
// independent 16-byte loads per lane (and the norm weight's alongside) before using any, so a row
// of up to 2048 columns costs one L2 round trip. to_smem = false computes rstd only. Callers
// synchronise.
__device__ __forceinline__ void stage_rows(const bf16* src, int64_t src_stride, const bf16* norm_w, float eps, int B,
                                           int K, bf16* xs, int xs_stride, float* rstd, int warp_id, int nwarps,
                                           int lane, bool to_smem) {
  const int chunks = K / 8;
  if (norm_w) {
    const bool one_round = chunks <= 256;
    for (int b = warp_id; b < B; b += nwarps) {
      const bf16* xr = src + b * src_stride;
      uint4 v[8], wv[8];
      float ss = 0.f;
      for (int base = 0; base < chunks; base += 256) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = base + u * 32 + lane;
          v[u] = c < chunks ? ldcg16(xr + c * 8) : make_uint4(0, 0, 0, 0);
          if (one_round && to_smem) wv[u] = c < chunks ? ldg16(norm_w + c * 8) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float f[8];
          unpack8(v[u], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
        }
      }
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / static_cast<float>(K) + eps);
      if (lane == 0) rstd[b] = r;
      if (!to_smem) continue;
      for (int base = 0; base < chunks; base += 256) {
        if (!one_round) {  // the row did not fit one round: load this round again
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = base + u * 32 + lane;
            v[u] = c < chunks ? ldcg16(xr + c * 8) : make_uint4(0, 0, 0, 0);
            wv[u] = c < chunks ? ldg16(norm_w + c * 8) : make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = base + u * 32 + lane;
          if (c >= chunks) continue;
          float f[8], wf[8];
          unpack8(v[u], f);
          unpack8(wv[u], wf);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * r);
          *reinterpret_cast<uint4*>(xs + b * xs_stride + c * 8) = pack8(f);
        }
      }
    }
  } else if (to_smem) {
    const int total = B * chunks, step = nwarps * 32;
    for (int base = warp_id * 32 + lane; base < total; base += step * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * step;
        v[u] = i < total ? ldcg16(src + (i / chunks) * src_stride + (i % chunks) * 8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * step;
        if (i < total) *reinterpret_cast<uint4*>(xs + (i / chunks) * xs_stride + (i % chunks) * 8) = v[u];
      }
    }
  }
}

struct EpilogueArgs {
  void* out;  // bf16 (store / residual in-out / silu) or fp32 (logits, partial sums)
  int64_t out_stride;
  int rows;   // weight rows (logits: this shard's vocabulary rows)
  int batch;
  float* partials;  // logits: one sampling record per row block and batch row
  const int64_t* state;
  float temperature;
  uint64_t seed;
  int row_offset = 0;  // logits: global vocabulary ID of row 0 (a vocabulary shard)
  const bf16* res_smem = nullptr;  // residual: a shared-memory copy of out's rows (row stride out_stride), or null
};

// Row block rb's outputs from the complete fp32 sums acc (lane layout of mma m16n8: rows
// h*16 + g + 8*(e>>1), batch column 8j + 2t + (e&1)). Reads of the residual use L2-only loads.
// Store / residual also take a single 16-row half: rows rb*32 + 16*first_half + ..., `halves` of
// them (acc[0] holding the first).
template <int EPI, int NT>
__device__ __forceinline__ void row_block_epilogue(const float (&acc)[2][NT][4], int rb, int lane,
                                                   const EpilogueArgs& a, int first_half = 0, int halves = 2) {
  const int g = lane >> 2, t = lane & 3, B = a.batch;
  if constexpr (EPI == kGemvStore || EPI == kGemvResidual) {
    bf16* out = static_cast<bf16*>(a.out);
    // residual from global memory (batch 8-16 in the decode step): every value is read before any
    // is written, so the reads overlap in one L2 round trip instead of waiting, one by one, behind
    // stores the compiler cannot prove disjoint (batch 16: 3193.8 -> 3073.4 us per step). A residual
    // staged in shared memory keeps the one pass (its reads are short either way).
    float res[2][NT][4];
    if (EPI == kGemvResidual && !a.res_smem) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = rb * 32 + (first_half + h) * 16 + g + 8 * (e >> 1);
            const int b = 8 * j + 2 * t + (e & 1);
            res[h][j][e] = 0.f;
            if (h >= halves || b >= B || n >= a.rows) continue;
            res[h][j][e] = ldcg_bf16(out + b * a.out_stride + n);
          }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h >= halves) break;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = rb * 32 + (first_half + h) * 16 + g + 8 * (e >> 1);
          const int b = 8 * j + 2 * t + (e & 1);
          if (b >= B || n >= a.rows) continue;
          bf16* dst = out + b * a.out_stride + n;
          if constexpr (EPI == kGemvStore) *dst = __float2bfloat16_rn(acc[h][j][e]);
          else {
            const float rv = a.res_smem ? __bfloat162float(a.res_smem[b * a.out_stride + n]) : res[h][j][e];
            *dst = __float2bfloat16_rn(rv + bf16_round(acc[h][j][e]));
          }
        }
    }
  } else if constexpr (EPI == kGemvSiluMul) {
    bf16* out = static_cast<bf16*>(a.out);
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = rb * 16 + g + 8 * (e >> 1);
        const int b = 8 * j + 2 * t + (e & 1);
        if (b >= B) continue;
        const float gate = bf16_round(acc[0][j][e]);
        const float up = bf16_round(acc[1][j][e]);
        const float act = bf16_round(gate / (1.0f + expf(-gate)));
        out[b * a.out_stride + col] = __float2bfloat16_rn(act * up);
      }
  } else if constexpr (EPI == kGemvPartial) {  // fp32 sums, unrounded (a tensor-parallel shard's part)
    float* out = static_cast<float*>(a.out);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h >= halves) break;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = rb * 32 + (first_half + h) * 16 + g + 8 * (e >> 1);
          const int b = 8 * j + 2 * t + (e & 1);
          if (b < B && n < a.rows) out[b * a.out_stride + n] = acc[h][j][e];
        }
    }
  } else {  // fp32 logits + per-row-block sampling records
    float* logits = static_cast<float*>(a.out);
    const float temperature =
        a.state ? __int_as_float(static_cast<int>(a.state[IPE_STATE_TEMPERATURE])) : a.temperature;
    const uint64_t seed = a.state ? static_cast<uint64_t>(a.state[IPE_STATE_SEED]) : a.seed;
    const int64_t step = a.state ? a.state[IPE_STATE_STEP] : 0;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int b = 8 * j + 2 * t + c;
        Stat st = empty_stat();
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int n = rb * 32 + h * 16 + g + 8 * r;
            if (b < B && n < a.rows) {
              const float l = bf16_round(acc[h][j][2 * r + c]);
              logits[b * a.out_stride + n] = l;
              const int id = n + a.row_offset;  // global vocabulary ID
              Stat y{l, 1.f, id, -INFINITY, 0x7fffffff, 0.f};
              if (temperature > 0.f) {
                y.gs = l / temperature - logf(-logf(uniform01(seed, id, b, step)));
                y.garg = id;
                y.gl = l;
              }
              st = merge(st, y);
            }
          }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) st = merge(st, shfl_xor_stat(st, o));
        if (g == 0 && b < B) {
          float* rec = a.partials + (static_cast<int64_t>(rb) * B + b) * IPE_PARTIAL_WORDS;
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

}  // namespace ipe
