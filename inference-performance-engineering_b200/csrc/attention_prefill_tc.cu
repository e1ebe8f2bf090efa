// Causal grouped-query flash attention over a prompt (prefill) on the 5th-generation tensor cores:
// S = Q K^T and O += P V as tcgen05.mma (bf16 in, fp32 accumulators in tensor memory), tiles
// brought in by TMA. Replaces ops.attention for T > 1 (src/ipe/ops.py:78-101), head_dim 128.
//
// One CTA per (128 queries, query head, batch row), 192 threads, one CTA per SM:
//   warp 0     TMA producer: the Q tile once, then K_j and V_j (128 keys x 128, as two 64-column
//              128-byte-swizzled halves) into a 4-slot ring. The K / V maps are 3-D
//              [batch * kv_heads][tokens][128] over the caches, so rows at or past `tokens` read as
//              zeros (the NaN-filled cache beyond the prompt is never loaded).
//   warp 1     TMEM allocator (512 columns: S0, S1, O) and MMA issuer: S_{j+1} = Q K_{j+1}^T into
//              the free S buffer before O += P_j V_j, so the tensor cores work on tile j+1 while
//              the softmax warps finish tile j. V is the MN-major B operand (transpose-B bit), as
//              stored; P is the K-major A operand written by the softmax warps.
//   warps 2-5  softmax, one query row per thread (TMEM lane = row): tcgen05.ld of the S row,
//              causal mask on the diagonal tile, fp32 online softmax in the base-2 domain with the
//              128^-0.5 scale folded in, P rounded to bf16 into shared memory (the same swizzle
//              TMA writes), O rescaled in TMEM (tcgen05.ld / st) only when a row's max moved, and
//              at the end O / l rounded to bf16 to the [batch, tokens, q_heads * 128] output.
// Arithmetic: fp32 scores, fp32 softmax statistics, bf16 P, fp32 P V accumulation, one rounding
// of O / l.
// Query blocks are scheduled heaviest first (the causal work grows with the block index). Every
// mbarrier wait is bounded; a timeout sets the device error word and the CTA winds down.
#include "common.cuh"
#include "launch.h"
#include "tensor_map.h"

namespace ipe {
namespace {

constexpr int kBM = 128, kBN = 128, kD = 128;
constexpr int kThreads = 192;
constexpr int kHalf = kBM * 64 * 2;  // one 128-row x 64-column bf16 block: 16 KB
constexpr int kTile = 2 * kHalf;     // 128 x 128 bf16: 32 KB
constexpr int kStages = 4;
constexpr int kTmemCols = 512;       // S0 [0, 128), S1 [128, 256), O [256, 384)
constexpr uint32_t kColO = 256;
constexpr float kScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;  // 128^-0.5 * log2(e)
constexpr size_t kSmem = 1024 + static_cast<size_t>(2 + kStages) * kTile + 256;

// K-major operand, 128-byte swizzle: 8-row groups 1024 bytes apart (the stride dimension).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
  return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// MN-major operand (V: the N = head-dim columns contiguous), 128-byte swizzle: the two 64-column
// halves kHalf bytes apart (leading dimension), 8-key groups 1024 bytes apart (stride dimension).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr) {
  return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(kHalf >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 D, bf16 A and B, M = 128, N = 128; B transposed (MN-major)
// when transpose_b.
__device__ __forceinline__ uint32_t instr_desc(bool transpose_b) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (transpose_b ? (1u << 16) : 0u) | (static_cast<uint32_t>(kBN >> 3) << 17) |
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

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one row per lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
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

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                                const __grid_constant__ CUtensorMap map_v, bf16* __restrict__ out, int q_heads,
                                int kv_heads, int tokens, int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* s_q = smem;
  unsigned char* s_p = smem + kTile;
  unsigned char* ring = smem + 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kStages * kTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [2]
  uint64_t* s_empty = s_full + 2;         // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // heaviest blocks first
  const int head = blockIdx.y, b = blockIdx.z;
  const int kvh = head / (q_heads / kv_heads);
  const int n_tiles = qb + 1;  // causal: key tiles 0..qb (kBN == kBM)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
      const int q_slice = b * q_heads + head, kv_slice = b * kv_heads + kvh;
      mbar_expect_tx(q_full, kTile);
      tma_load_3d(smem_addr(s_q), &map_q, q_full, 0, qb * kBM, q_slice);
      tma_load_3d(smem_addr(s_q) + kHalf, &map_q, q_full, 64, qb * kBM, q_slice);
      uint32_t armed = 0;  // bit s: parity armed on kv_full[s]; bit 16 + s: armed at all
      for (int i = 0; i < 2 * n_tiles && !*abort_flag; ++i) {  // K_0, V_0, K_1, V_1, ...
        const int s = i % kStages;
        const uint32_t phase = (i / kStages) & 1;
        if (!mbar_wait(&kv_empty[s], phase ^ 1, err)) {
          *abort_flag = 1;
          break;
        }
        const CUtensorMap* map = (i & 1) ? &map_v : &map_k;
        const uint32_t dst = smem_addr(ring + s * kTile);
        mbar_expect_tx(&kv_full[s], kTile);
        tma_load_3d(dst, map, &kv_full[s], 0, (i >> 1) * kBN, kv_slice);
        tma_load_3d(dst + kHalf, map, &kv_full[s], 64, (i >> 1) * kBN, kv_slice);
        armed = (armed & ~(1u << s)) | (phase << s) | (1u << (16 + s));
      }
      // copies in flight land before the CTA's shared memory goes away
      mbar_wait(q_full, 0, err);
      if (*abort_flag)
        for (int s = 0; s < kStages; ++s)
          if (armed & (1u << (16 + s))) mbar_wait(&kv_full[s], (armed >> s) & 1u, err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t idesc_s = instr_desc(false), idesc_o = instr_desc(true);
    bool ok = mbar_wait(q_full, 0, err);
    auto issue_s = [&](int j) -> bool {  // S[j % 2] = Q K_j^T
      const int i = 2 * j, s = i % kStages;
      if (!mbar_wait(&kv_full[s], (i / kStages) & 1, err)) return false;
      if (!mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1, err)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_addr(s_q), ka = smem_addr(ring + s * kTile);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf;  // 64-column half, then +32 bytes per 16 columns
          umma(tmem_base + (j & 1) * kBN, desc_kmajor(qa + off) + 2 * (kk & 3), desc_kmajor(ka + off) + 2 * (kk & 3),
               idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&kv_empty[s]);
        umma_commit(&s_full[j & 1]);
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](int j) -> bool {  // O (+)= P_j V_j
      const int i = 2 * j + 1, s = i % kStages;
      if (!mbar_wait(&kv_full[s], (i / kStages) & 1, err)) return false;
      if (!mbar_wait(p_full, j & 1, err)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pa = smem_addr(s_p), va = smem_addr(ring + s * kTile);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {  // 16 keys per MMA
          umma(tmem_base + kColO, desc_kmajor(pa + (kk >> 2) * kHalf) + 2 * (kk & 3), desc_mnmajor(va + kk * 16 * 128),
               idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[s]);
        umma_commit(o_done);
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s(0);
    for (int j = 0; j < n_tiles && ok && !*abort_flag; ++j) {
      if (j + 1 < n_tiles) ok = issue_s(j + 1);
      if (ok) ok = issue_pv(j);
    }
    if (!ok) *abort_flag = 1;
  } else {
    // ------------------------------------------------------------------ softmax
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. + 31
    const int row = quarter * 32 + lane;
    const int qrow = qb * kBM + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // waits are taken by every lane and agreed on, so the warp-collective tcgen05 loads and stores
    // below always run converged
    auto wait_all = [&](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity, err)); };
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (!wait_all(&s_full[j & 1], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tmem_ld32(tmem_base + lane_off + (j & 1) * kBN + c * 32, s + c * 32);
      tc_fence_before();
      mbar_arrive(&s_empty[j & 1]);
      if (j == qb) {  // diagonal tile: key j * 128 + c is later than query qb * 128 + row when c > row
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c > row) s[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN; ++c) mx = fmaxf(mx, s[c]);
      const float m_new = fmaxf(m_run, mx);
      const float corr = exp2f((m_run - m_new) * kScaleLog2);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        s[c] = exp2f((s[c] - m_new) * kScaleLog2);
        sum += s[c];
      }
      l_run = l_run * corr + sum;
      m_run = m_new;
      if (j > 0 && !wait_all(o_done, (j - 1) & 1)) {  // P V_{j-1} done: P free, O settled
        ok = false;
        break;
      }
      tc_fence_after();
      // P row -> shared memory, K-major with the 128-byte swizzle (16-byte chunk ^ row % 8)
      const uint32_t prow = smem_addr(s_p) + row * 128;
#pragma unroll
      for (int c = 0; c < kBN / 8; ++c) {
        const uint32_t addr = prow + (c >> 3) * kHalf + ((((c & 7) ^ (row & 7))) << 4);
        const uint4 v = pack8(s + 8 * c);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
      if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {  // rescale O where a row's max moved
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          tmem_ld32(tmem_base + lane_off + kColO + c * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= corr;
          tmem_st32(tmem_base + lane_off + kColO + c * 32, o);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor cores
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && wait_all(o_done, (n_tiles - 1) & 1)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      bf16* dst = out + (static_cast<int64_t>(b) * tokens + qrow) * (static_cast<int64_t>(q_heads) * kD) + head * kD;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        float o[32];
        tmem_ld32(tmem_base + lane_off + kColO + c * 32, o);
        if (qrow < tokens) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float r[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] = o[8 * q + e] * inv;
            *reinterpret_cast<uint4*>(dst + c * 32 + 8 * q) = pack8(r);
          }
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
  }
}

}  // namespace

cudaError_t launch_prefill_attention_tc(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                        int kv_heads, int tokens, int capacity, int* err, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  if (!make_map_3d(&mq, q, kD, tokens, batch * q_heads, tokens, kBM, 64) ||
      !make_map_3d(&mk, k, kD, tokens, batch * kv_heads, capacity, kBN, 64) ||
      !make_map_3d(&mv, v, kD, tokens, batch * kv_heads, capacity, kBN, 64))
    return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const dim3 grid((tokens + kBM - 1) / kBM, q_heads, batch);
  prefill_attention_tc_kernel<<<grid, kThreads, kSmem, stream>>>(mq, mk, mv, static_cast<bf16*>(out), q_heads,
                                                                 kv_heads, tokens, err);
  return cudaGetLastError();
}

}  // namespace ipe
