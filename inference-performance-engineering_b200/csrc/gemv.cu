// Decode linear layers: persistent, bulk-copy-fed weight-streaming GEMV for 1..16 activation rows.
//
// Weight layout ("decode tiles", built once by ipe_decode_tiles, see stream_tile.cuh): 4 KB half
// tiles of 16 rows x 128 columns stored [row block][half][k tile]. This kernel consumes a row
// block's two halves of one k tile together: each 8 KB slot is filled by two 4 KB copies.
//
// Work: each row block's K range is split into `ksplit` pieces; pieces are dealt in contiguous
// ranges to one CTA per SM, and within a CTA round-robin to its 4 consumer warps. One producer
// thread streams the CTA's tiles with 8 KB cp.async.bulk copies into shared-memory slots
// (mbarrier full/empty pairs), 3 slots owned by each consumer warp, so ~96 KB of weights are in
// flight per SM. A slot has exactly one consumer, which waits for its fills in order: a parity
// wait is then never more than one phase ahead of the barrier (a shared ring would let a fast
// warp wait two phases ahead, where the parity aliases). Activations
// (normalised once per CTA for the norm-fused layers) sit in shared memory; consumer warps read
// their slot with conflict-free 16-byte loads and feed mma.sync m16n8k16 (weights = A,
// activations = B, the same K permutation on both sides so every read is a contiguous 16 bytes).
// With ksplit > 1, pieces write fp32 partial tiles to the workspace and the last piece of a row
// block to arrive (an atomic counter) sums them in piece order - deterministic - applies the
// epilogue with the reference's rounding points and resets the counter.
//
// Launched with programmatic dependent launch: the producer streams weights before the previous
// kernel has finished; consumers wait (griddepcontrol.wait) before reading activations.
#include "common.cuh"
#include "launch.h"
#include "sampling.cuh"
#include "stream_tile.cuh"
#include "tensor_map.h"

namespace ipe {
namespace {

constexpr int kConsumers = 4;
constexpr int kSlotsPerWarp = 3;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kSubK = kTileK;
constexpr int kMaxStages = kConsumers * kSlotsPerWarp;
constexpr int kPad = 32;  // bf16 elements of padding per staged activation row
constexpr size_t kCounterBytes = 32768;  // arrival counters for up to 8192 row blocks
constexpr size_t kSmemLimit = 200 * 1024;
constexpr size_t kFixedSmem = 1024 + 2 * kMaxStages * 8 + 16 * 4 + 64;

struct Plan {
  int row_blocks;
  int ksplit;
  int piece_k;  // columns per piece, a multiple of kSubK
  int pieces;
  int stages;
  int act_smem;  // activations staged in shared memory (else read from global per tile)
  int64_t tiles;  // tiles in the weight buffer: row_blocks * (k / kSubK)
  size_t smem;
};

template <int NT, int EPI, bool NORM, bool ACT_SMEM>
__global__ void __launch_bounds__(kThreads, 2) stream_gemv_kernel(const GemvArgs a, const Plan plan) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = plan.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + stages * kTileBytes);
  uint64_t* empty = full + kMaxStages;
  float* rstd = reinterpret_cast<float*>(empty + kMaxStages);
  bf16* xs = reinterpret_cast<bf16*>(rstd + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int p0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * plan.pieces / G);
  const int p1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * plan.pieces / G);
  const int npieces = p1 - p0;
  const int subs = plan.piece_k / kSubK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer (weights only)
    if (lane == 0) {
      // Piece p's tiles are p * subs .. p * subs + subs - 1 (a row block's pieces are adjacent), so
      // the walk is pointer arithmetic only: the single issuing thread must stay far ahead. Warp w's
      // k-th tile goes to its slot w * kSlotsPerWarp + k % kSlotsPerWarp as fill k / kSlotsPerWarp.
      const uint32_t ring_base = smem_addr(ring);
      const int units_per_row = a.k / kSubK;
      bool ok = true;
      for (int q0 = 0, k0 = 0; q0 < npieces && ok; q0 += kConsumers, k0 += subs) {
        const int gs = min(kConsumers, npieces - q0);
        for (int s = 0; s < subs && ok; ++s) {
          const int k = k0 + s;
          const int fill = k / kSlotsPerWarp, sub = k - fill * kSlotsPerWarp;
          for (int w = 0; w < gs; ++w) {
            const int64_t tile = static_cast<int64_t>(p0 + q0 + w) * subs + s;
            if (tile < 0 || tile >= plan.tiles) {  // never expected: refuse the copy, report
              report(a.err, kErrShape);
              ok = false;
              break;
            }
            const int slot = w * kSlotsPerWarp + sub;
            if (fill > 0 && !mbar_wait(&empty[slot], (fill - 1) & 1, a.err)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&full[slot], kTileBytes);
            const unsigned char* w_base = static_cast<const unsigned char*>(a.w);
            const int64_t rb = tile / units_per_row, kt = tile % units_per_row;
            bulk_copy(ring_base + slot * kTileBytes, w_base + half_tile_offset(rb, 0, kt, units_per_row),
                      kHalfTileBytes, &full[slot]);
            bulk_copy(ring_base + slot * kTileBytes + kHalfTileBytes, w_base + half_tile_offset(rb, 1, kt, units_per_row),
                      kHalfTileBytes, &full[slot]);
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int cw = warp - 1;
  const int g = lane >> 2, t = lane & 3;
  const int B = a.batch, K = a.k;
  const int xs_stride = K + kPad;
  const bf16* __restrict__ x = static_cast<const bf16*>(a.x);
  const bf16* __restrict__ nw = static_cast<const bf16*>(a.norm_weight);
  pdl_wait();
  if constexpr (NORM || ACT_SMEM) {
    for (int b = cw; b < B; b += kConsumers) {
      const bf16* xr = x + b * a.x_stride;
      float r = 1.f;
      if constexpr (NORM) {
        float ss = 0.f;
        for (int c = lane; c < K / 8; c += 32) {
          float f[8];
          unpack8(ldcg16(xr + c * 8), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
        }
        ss = warp_sum(ss);
        r = rsqrtf(ss / static_cast<float>(K) + a.eps);
        if (lane == 0) rstd[b] = r;
      }
      if constexpr (ACT_SMEM) {
        for (int c = lane; c < K / 8; c += 32) {
          uint4 v = ldcg16(xr + c * 8);
          if constexpr (NORM) {
            float f[8], wf[8];
            unpack8(v, f);
            unpack8(ldg16(nw + c * 8), wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * r);
            v = pack8(f);
          }
          *reinterpret_cast<uint4*>(xs + b * xs_stride + c * 8) = v;
        }
      }
    }
    named_barrier(1, kConsumers * 32);
  }
  float my_rstd[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) my_rstd[j] = (NORM && !ACT_SMEM && 8 * j + g < B) ? rstd[8 * j + g] : 0.f;

  for (int q = 0; q * kConsumers < npieces; ++q) {
    const int gs = min(kConsumers, npieces - q * kConsumers);
    if (cw >= gs) continue;
    const int piece = p0 + q * kConsumers + cw;
    const int rb = piece / plan.ksplit, ks = piece % plan.ksplit;
    float acc[2][NT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < NT; ++j) acc[h][j][0] = acc[h][j][1] = acc[h][j][2] = acc[h][j][3] = 0.f;
    bool ok = true;
    for (int s = 0; s < subs; ++s) {
      const int k = q * subs + s;  // this warp's k-th tile
      const int fill = k / kSlotsPerWarp;
      const int slot = cw * kSlotsPerWarp + (k - fill * kSlotsPerWarp);
      const int k0 = ks * plan.piece_k + s * kSubK;
      uint4 xv[4][NT];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int b = 8 * j + g;
          const int k = k0 + c * 32 + 8 * t;
          if (b >= B) {
            xv[c][j] = make_uint4(0, 0, 0, 0);
          } else if constexpr (ACT_SMEM) {
            xv[c][j] = *reinterpret_cast<const uint4*>(xs + b * xs_stride + k);
          } else {
            const uint4 raw = ldcg16(x + b * a.x_stride + k);
            if constexpr (NORM) {
              float f[8], wf[8];
              unpack8(raw, f);
              unpack8(ldg16(nw + k), wf);
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = wf[e] * bf16_round(f[e] * my_rstd[j]);
              xv[c][j] = pack8(f);
            } else {
              xv[c][j] = raw;
            }
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
    if (!ok) break;

    // ---------------------------------------------------------------- split-K reduction
    if (plan.ksplit > 1) {
      float* slotbuf = a.slots + (static_cast<int64_t>(piece) * 32 + lane) * (8 * NT);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j)
          __stcg(reinterpret_cast<float4*>(slotbuf + (h * NT + j) * 4),
                 make_float4(acc[h][j][0], acc[h][j][1], acc[h][j][2], acc[h][j][3]));
      __threadfence();
      __syncwarp();
      int prior = 0;
      if (lane == 0) prior = atomicAdd(&a.counters[rb], 1);
      prior = __shfl_sync(0xffffffffu, prior, 0);
      if (prior != plan.ksplit - 1) continue;
      __threadfence();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[h][j][0] = acc[h][j][1] = acc[h][j][2] = acc[h][j][3] = 0.f;
      for (int p = 0; p < plan.ksplit; ++p) {
        const float* src = a.slots + (static_cast<int64_t>(rb * plan.ksplit + p) * 32 + lane) * (8 * NT);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (h * NT + j) * 4));
            acc[h][j][0] += v.x;
            acc[h][j][1] += v.y;
            acc[h][j][2] += v.z;
            acc[h][j][3] += v.w;
          }
      }
      if (lane == 0) a.counters[rb] = 0;
    }

    // ---------------------------------------------------------------- epilogue
    EpilogueArgs ea{a.out, a.out_stride, a.rows, B, a.partials, a.state, a.temperature, a.seed, a.row_offset};
    row_block_epilogue<EPI, NT>(acc, rb, lane, ea);
  }
}

Plan make_plan(const GemvArgs& a) {
  Plan p{};
  p.row_blocks = a.epilogue == kGemvSiluMul ? a.rows / 32 : (a.rows + 31) / 32;
  const int units = a.k / kSubK;  // tiles per row block
  const int sms = sm_count();
  int split = 1;
  if (a.epilogue != kGemvLogits) {
    // Smallest power-of-two split that gives every SM >= 8 pieces and <= 5% imbalance.
    for (int s = 1; s <= units; s *= 2) {
      if (units % s) break;
      split = s;
      const int64_t pieces = static_cast<int64_t>(p.row_blocks) * s;
      const double per = static_cast<double>(pieces) / sms;
      const double balance = per / static_cast<double>((pieces + sms - 1) / sms);
      if (pieces >= 8LL * sms && balance >= 0.95) break;
    }
  }
  p.ksplit = split;
  p.piece_k = a.k / split;
  p.pieces = p.row_blocks * split;
  p.tiles = static_cast<int64_t>(p.row_blocks) * units;
  const size_t act = static_cast<size_t>(a.batch) * (a.k + kPad) * 2;
  p.stages = kMaxStages;
  p.act_smem = kFixedSmem + static_cast<size_t>(kMaxStages) * kTileBytes + act + 16 <= kSmemLimit;
  p.smem = kFixedSmem + static_cast<size_t>(p.stages) * kTileBytes + (p.act_smem ? act + 16 : 0);
  return p;
}

template <int NT, int EPI, bool NORM, bool ACT>
cudaError_t launch_one(const GemvArgs& a, const Plan& plan, cudaStream_t stream) {
  auto kernel = stream_gemv_kernel<NT, EPI, NORM, ACT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemLimit + 1024));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int grid = plan.pieces < sm_count() ? plan.pieces : sm_count();
  return launch_pdl(kernel, dim3(grid), dim3(kThreads), plan.smem, stream, a, plan);
}

template <int NT, bool ACT>
cudaError_t dispatch(const GemvArgs& a, const Plan& plan, cudaStream_t stream) {
  switch (a.epilogue) {
    case kGemvStore: return launch_one<NT, kGemvStore, true, ACT>(a, plan, stream);
    case kGemvResidual: return launch_one<NT, kGemvResidual, false, ACT>(a, plan, stream);
    case kGemvSiluMul: return launch_one<NT, kGemvSiluMul, true, ACT>(a, plan, stream);
    case kGemvPartial: return launch_one<NT, kGemvPartial, false, ACT>(a, plan, stream);
    default: return launch_one<NT, kGemvLogits, true, ACT>(a, plan, stream);
  }
}

// ------------------------------------------------------------------------------ tile builder
// One thread per 16-byte chunk of the tiled output.
__global__ void decode_tiles_kernel(const bf16* __restrict__ w, const bf16* __restrict__ w2, bf16* __restrict__ out,
                                    int rows, int k, int64_t chunks) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= chunks) return;
  // idx = ((((rb * 2 + h) * ku_row + ku) * 2 + j) * 16 + r) * 8 + pc (half_tile_offset / 16)
  const int pc = static_cast<int>(idx & 7);
  const int r = static_cast<int>((idx >> 3) & 15);
  const int j = static_cast<int>((idx >> 7) & 1);
  const int64_t half_tile = idx >> 8;
  const int ku_row = k / kSubK;
  const int ku = static_cast<int>(half_tile % ku_row);
  const int h = static_cast<int>((half_tile / ku_row) & 1);
  const int64_t rb = half_tile / ku_row / 2;
  const int lc = swizzle(pc, r);  // the logical chunk stored at physical chunk pc (self-inverse)
  const int col = ku * kSubK + j * 64 + lc * 8;
  int64_t row;
  const bf16* src;
  if (w2) {  // gate / up pair: half 0 from w, half 1 from w2, rows 16 rb + r
    row = rb * 16 + r;
    src = h == 0 ? w : w2;
  } else {
    row = rb * 32 + h * 16 + r;
    src = w;
  }
  uint4 v = make_uint4(0, 0, 0, 0);
  if (row < rows) v = *reinterpret_cast<const uint4*>(src + row * k + col);
  *reinterpret_cast<uint4*>(out + idx * 8) = v;
}

}  // namespace

size_t gemv_workspace_bytes(const GemvArgs& a) {
  const Plan p = make_plan(a);
  if (p.ksplit == 1) return 0;
  const int nt = a.batch <= 8 ? 1 : 2;
  return kCounterBytes + static_cast<size_t>(p.pieces) * 32 * 8 * nt * sizeof(float);
}

size_t decode_tiles_bytes(int rows, int k, bool pair) {
  const int64_t blocks = pair ? (rows + 15) / 16 : (rows + 31) / 32;
  return static_cast<size_t>(blocks) * (k / kSubK) * kTileBytes;
}

cudaError_t launch_decode_tiles(const void* w, const void* w2, void* out, int rows, int k, cudaStream_t stream) {
  const int64_t chunks = static_cast<int64_t>(decode_tiles_bytes(rows, k, w2 != nullptr) / 16);
  const unsigned blocks = static_cast<unsigned>((chunks + 255) / 256);
  decode_tiles_kernel<<<blocks, 256, 0, stream>>>(static_cast<const bf16*>(w), static_cast<const bf16*>(w2),
                                                   static_cast<bf16*>(out), rows, k, chunks);
  return cudaGetLastError();
}

cudaError_t launch_gemv(GemvArgs a, void* workspace, cudaStream_t stream, const char** message) {
  const Plan plan = make_plan(a);
  if (plan.row_blocks > static_cast<int>(kCounterBytes / sizeof(int)) && plan.ksplit > 1) {
    *message = "too many row blocks for the split-K counters";
    return cudaErrorInvalidValue;
  }
  if (plan.ksplit > 1) {
    a.counters = static_cast<int*>(workspace);
    a.slots = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kCounterBytes);
  }
  if (a.batch <= 8) return plan.act_smem ? dispatch<1, true>(a, plan, stream) : dispatch<1, false>(a, plan, stream);
  return plan.act_smem ? dispatch<2, true>(a, plan, stream) : dispatch<2, false>(a, plan, stream);
}

}  // namespace ipe
