// Persistent tensor-core GEMM for sm_100a: C = epilogue(A @ B^T), A [M, K] and B [N, K] bf16,
// both K-contiguous, fp32 accumulation in tensor memory (TMEM).
//
// Warp roles per CTA (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x64 A and BNx64 B tiles (128-byte swizzle) into a kStages ring
//   warp 1      TMEM allocator and MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16)
//               and commits each stage back to the producer and each finished tile to the epilogue
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (one TMEM lane = one output row),
//               reference rounding, fused residual / SiLU*up / fp32-logit writes
// Two accumulator buffers in TMEM let the epilogue of tile i overlap the MMAs of tile i+1.
// Every mbarrier wait is bounded; a timeout sets the device error word and the CTA winds down.
#include <cstdlib>

#include "common.cuh"
#include "launch.h"
#include "tensor_map.h"

namespace ipe {
namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // two accumulator buffers
  static constexpr size_t kSmem = 1024 /*align*/ + static_cast<size_t>(kStages) * kStageBytes + 256;
};

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

template <int BN>
__device__ __forceinline__ uint32_t instr_desc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                                                          const __grid_constant__ CUtensorMap map_b, void* c,
                                                          const bf16* residual, int M, int N, int K, int* err) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tmem_full = empty + C::kStages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM, num_n = N / BN;
  const int tiles_total = num_m * num_n;
  const int kblocks = K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;  // bit s: parity of the last phase armed on full[s] + 1 flag in bit 16+s
      for (int tile = blockIdx.x; tile < tiles_total && !*abort_flag; tile += gridDim.x) {
        const int m = tile % num_m, n = tile / num_m;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err)) {
            *abort_flag = 1;
            break;
          }
          mbar_expect_tx(&full[stage], C::kStageBytes);
          const uint32_t sa = smem_addr(tiles + stage * C::kStageBytes);
          tma_load_2d(sa, &map_a, &full[stage], kb * kBK, m * kBM);
          tma_load_2d(sa + C::kABytes, &map_b, &full[stage], kb * kBK, n * BN);
          armed = (armed & ~(1u << stage)) | (phase << stage) | (1u << (16 + stage));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // Let copies already in flight land before the CTA's shared memory goes away.
        for (int s = 0; s < C::kStages; ++s)
          if (armed & (1u << (16 + s))) mbar_wait(&full[s], (armed >> s) & 1u, err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t idesc = instr_desc<BN>();
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < tiles_total && !*abort_flag; tile += gridDim.x) {
      if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, err)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = smem_addr(tiles + stage * C::kStageBytes);
          const uint64_t da = smem_desc_sw128(sa);
          const uint64_t db = smem_desc_sw128(sa + C::kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle atom (encoded >> 4).
            umma(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tmem_full[acc]);
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < tiles_total && !*abort_flag; tile += gridDim.x) {
      const int m = tile % num_m, n = tile / num_m;
      if (!mbar_wait(&tmem_full[acc], acc_phase, err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = m * kBM + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      const bool live = row < M;
      if constexpr (EPI == IPE_EPI_SILU_MUL) {
        bf16* out = static_cast<bf16*>(c) + static_cast<int64_t>(row) * (N / 2);
#pragma unroll 1
        for (int grp = 0; grp < BN / 128; ++grp) {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float gate[32], up[32];
            tmem_ld32(taddr + grp * 128 + h * 32, gate);
            tmem_ld32(taddr + grp * 128 + 64 + h * 32, up);
            if (live) {
              const int j0 = (n * BN + grp * 128) / 2 + h * 32;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                float r[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const float gv = bf16_round(gate[v * 8 + i]);
                  const float act = bf16_round(gv / (1.0f + expf(-gv)));
                  r[i] = act * bf16_round(up[v * 8 + i]);
                }
                *reinterpret_cast<uint4*>(out + j0 + v * 8) = pack8(r);
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          float v[32];
          tmem_ld32(taddr + cc * 32, v);
          if (!live) continue;
          const int col = n * BN + cc * 32;
          if constexpr (EPI == IPE_EPI_LOGITS) {
            float* out = static_cast<float*>(c) + static_cast<int64_t>(row) * N + col;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<float4*>(out + 4 * q) =
                  make_float4(bf16_round(v[4 * q]), bf16_round(v[4 * q + 1]), bf16_round(v[4 * q + 2]),
                              bf16_round(v[4 * q + 3]));
          } else if constexpr (EPI == IPE_EPI_PARTIAL) {  // unrounded fp32 sums
            float* out = static_cast<float*>(c) + static_cast<int64_t>(row) * N + col;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<float4*>(out + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
            bf16* out = static_cast<bf16*>(c) + static_cast<int64_t>(row) * N + col;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float r[8];
              if constexpr (EPI == IPE_EPI_RESIDUAL) {
                float res[8];
                unpack8(*reinterpret_cast<const uint4*>(residual + static_cast<int64_t>(row) * N + col + 8 * q), res);
#pragma unroll
                for (int i = 0; i < 8; ++i) r[i] = res[i] + bf16_round(v[8 * q + i]);
              } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) r[i] = v[8 * q + i];
              }
              *reinterpret_cast<uint4*>(out + 8 * q) = pack8(r);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::kTmemCols));
  }
}

// ------------------------------------------------------------------------------ host side
bool make_map(CUtensorMap* map, const void* ptr, int rows, int k, int box_rows) {
  return make_map_2d(map, ptr, rows, k, box_rows, kBK);
}

template <int BN, int EPI>
cudaError_t run(const CUtensorMap& ma, const CUtensorMap& mb, void* c, const void* residual, int m, int n, int k,
                int* err, cudaStream_t stream) {
  auto kernel = gemm_kernel<BN, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(Cfg<BN>::kSmem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int tiles = ((m + kBM - 1) / kBM) * (n / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kernel<<<grid, kThreads, Cfg<BN>::kSmem, stream>>>(ma, mb, c, static_cast<const bf16*>(residual), m, n, k, err);
  return cudaGetLastError();
}

template <int BN>
cudaError_t run_epi(int epi, const CUtensorMap& ma, const CUtensorMap& mb, void* c, const void* residual, int m, int n,
                    int k, int* err, cudaStream_t stream) {
  switch (epi) {
    case IPE_EPI_STORE: return run<BN, IPE_EPI_STORE>(ma, mb, c, residual, m, n, k, err, stream);
    case IPE_EPI_RESIDUAL: return run<BN, IPE_EPI_RESIDUAL>(ma, mb, c, residual, m, n, k, err, stream);
    case IPE_EPI_SILU_MUL: return run<BN, IPE_EPI_SILU_MUL>(ma, mb, c, residual, m, n, k, err, stream);
    case IPE_EPI_PARTIAL: return run<BN, IPE_EPI_PARTIAL>(ma, mb, c, residual, m, n, k, err, stream);
    default: return run<BN, IPE_EPI_LOGITS>(ma, mb, c, residual, m, n, k, err, stream);
  }
}

// 64-column tiles: every epilogue but SiLU*up (its gate / up pairs span 128 columns).
cudaError_t run_epi64(int epi, const CUtensorMap& ma, const CUtensorMap& mb, void* c, const void* residual, int m,
                      int n, int k, int* err, cudaStream_t stream) {
  switch (epi) {
    case IPE_EPI_STORE: return run<64, IPE_EPI_STORE>(ma, mb, c, residual, m, n, k, err, stream);
    case IPE_EPI_RESIDUAL: return run<64, IPE_EPI_RESIDUAL>(ma, mb, c, residual, m, n, k, err, stream);
    case IPE_EPI_PARTIAL: return run<64, IPE_EPI_PARTIAL>(ma, mb, c, residual, m, n, k, err, stream);
    case IPE_EPI_LOGITS: return run<64, IPE_EPI_LOGITS>(ma, mb, c, residual, m, n, k, err, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// Output-tile width: the one with the least wave-quantised time, ceil(tiles / SMs) x BN, weighted
// by the tile's relative cost per column (a wider tile re-reads A less: 0.8 for 256, 1.15 for 64;
// fitted to B200 timings of Qwen3-1.7B's layer GEMMs at M = 512 and 4096). At M = 512, o_proj and
// down_proj (N = 2048) take 64-column tiles: 128 tiles instead of 64 on 148 SMs (-11% and -6%). The
// SiLU*up epilogue pairs gate / up columns inside 128-column groups, so it takes 128 or 256.
// IPE_GEMM_BN forces a width where it is valid.
int pick_bn(int m, int n, int epilogue) {
  static const int forced = [] {
    const char* v = std::getenv("IPE_GEMM_BN");
    return v ? std::atoi(v) : 0;
  }();
  const int widths[3] = {256, 128, 64};
  const float weight[3] = {0.8f, 1.0f, 1.15f};
  auto valid = [&](int bn) { return n % bn == 0 && (epilogue != IPE_EPI_SILU_MUL || bn >= 128); };
  if ((forced == 64 || forced == 128 || forced == 256) && valid(forced)) return forced;
  const int64_t m_tiles = (m + kBM - 1) / kBM;
  int best = 0;
  float best_cost = 0.f;
  for (int i = 0; i < 3; ++i) {
    if (!valid(widths[i])) continue;
    const int64_t tiles = m_tiles * (n / widths[i]);
    const int64_t waves = (tiles + sm_count() - 1) / sm_count();
    const float cost = static_cast<float>(waves) * widths[i] * weight[i];
    if (best == 0 || cost < best_cost) {
      best = widths[i];
      best_cost = cost;
    }
  }
  return best;
}

cudaError_t launch_gemm(const void* a, const void* b, void* c, int m, int n, int k, int epilogue, const void* residual,
                        int* err, cudaStream_t stream, const char** message) {
  const int bn = pick_bn(m, n, epilogue);
  if (bn == 0) {
    *message = "no output-tile width divides n";
    return cudaErrorInvalidValue;
  }
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, m, k, kBM) || !make_map(&mb, b, n, k, bn)) {
    *message = "cuTensorMapEncodeTiled failed (driver entry point missing or bad operand layout)";
    return cudaErrorInvalidValue;
  }
  if (bn == 256) return run_epi<256>(epilogue, ma, mb, c, residual, m, n, k, err, stream);
  if (bn == 128) return run_epi<128>(epilogue, ma, mb, c, residual, m, n, k, err, stream);
  return run_epi64(epilogue, ma, mb, c, residual, m, n, k, err, stream);
}

}  // namespace ipe
