// Causal flash-attention over a prompt (prefill), grouped-query, head_dim 128.
//
// One CTA per (64 queries, query head, batch row); 4 warps of 16 query rows each. K and V tiles of
// 64 keys are double-buffered in XOR-swizzled shared memory with cp.async; S = Q K^T and O += P V
// run on mma.sync m16n8k16 (bf16 in, fp32 accumulate) with an fp32 online softmax. P is rounded to
// bf16 for the P V product, as flash kernels do. Keys at positions >= tokens are zero-filled so
// padded query rows never read stale cache contents.
#include "common.cuh"
#include "launch.h"

namespace ipe {
namespace {

constexpr int kBM = 64, kBN = 64, kD = 128;
constexpr int kThreads = 128;
constexpr float kScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;  // 128^-0.5 * log2(e)
constexpr int kTileBytes = kBM * kD * 2;                                     // 16 KB

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset inside a [64][128] bf16 tile
  return static_cast<uint32_t>(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int size = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(size));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Copy rows [row0, row0+64) x 128 of a [rows][128] bf16 matrix into a swizzled tile; rows >= limit are zeros.
__device__ __forceinline__ void load_tile(uint32_t tile, const bf16* src, int row0, int limit) {
  for (int i = threadIdx.x; i < kBM * 16; i += kThreads) {
    const int r = i >> 4, c = i & 15;
    const bool valid = row0 + r < limit;
    const bf16* p = src + static_cast<int64_t>(valid ? row0 + r : 0) * kD + c * 8;
    cp_async16(tile + swz(r, c), p, valid);
  }
}

__global__ void __launch_bounds__(kThreads, 2) prefill_attention_kernel(const bf16* __restrict__ q,
                                                                       const bf16* __restrict__ kc,
                                                                       const bf16* __restrict__ vc,
                                                                       bf16* __restrict__ out, int q_heads,
                                                                       int kv_heads, int tokens, int capacity) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int qt = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  const int kvh = head / (q_heads / kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t s_q = smem_addr(smem);
  const uint32_t s_k[2] = {s_q + kTileBytes, s_q + 2 * kTileBytes};
  const uint32_t s_v[2] = {s_q + 3 * kTileBytes, s_q + 4 * kTileBytes};

  const bf16* qbase = q + (static_cast<int64_t>(b) * q_heads + head) * tokens * kD;
  const bf16* kbase = kc + (static_cast<int64_t>(b) * kv_heads + kvh) * capacity * kD;
  const bf16* vbase = vc + (static_cast<int64_t>(b) * kv_heads + kvh) * capacity * kD;
  const int q0 = qt * kBM;
  const int n_tiles = qt + 1;  // causal: key tiles 0..qt

  load_tile(s_q, qbase, q0, tokens);
  load_tile(s_k[0], kbase, 0, tokens);
  load_tile(s_v[0], vbase, 0, tokens);
  cp_commit();

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int kt = 0; kt < n_tiles; ++kt) {
    const int st = kt & 1;
    if (kt + 1 < n_tiles) {
      load_tile(s_k[st ^ 1], kbase, (kt + 1) * kBN, tokens);
      load_tile(s_v[st ^ 1], vbase, (kt + 1) * kBN, tokens);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(s_q + swz(r, c), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = n * 8 + (lane & 7);
        const int c = ks * 2 + (lane >> 3);
        ldsm_x4(s_k[st] + swz(r, c), b0, b1, b2, b3);
        mma16816(s[n], qf[ks], b0, b1);
        mma16816(s[n], qf[ks + 1], b2, b3);
      }
    }
    // Causal mask on the diagonal tile (keys > query), then the online softmax.
    if (kt == qt) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int key = kt * kBN + n * 8 + 2 * t + (i & 1);
          const int qrow = q0 + warp * 16 + g + 8 * (i >> 1);
          if (key > qrow) s[n][i] = -INFINITY;
        }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * h], s[n][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[h], mx);
      corr[h] = exp2f((m_run[h] - m_new) * kScaleLog2);
      m_run[h] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float p0 = exp2f((s[n][2 * h] - m_new) * kScaleLog2);
        const float p1 = exp2f((s[n][2 * h + 1] - m_new) * kScaleLog2);
        s[n][2 * h] = p0;
        s[n][2 * h + 1] = p1;
        sum += p0 + p1;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l_run[h] = l_run[h] * corr[h] + sum;
    }
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= corr[0];
      o[d][1] *= corr[0];
      o[d][2] *= corr[1];
      o[d][3] *= corr[1];
    }
    // O += P V: P from registers (bf16), V via transposed ldmatrix.
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
      pa[1] = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
      pa[2] = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      pa[3] = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
      for (int d = 0; d < 16; d += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = d + (lane >> 4);
        ldsm_x4_t(s_v[st] + swz(r, c), b0, b1, b2, b3);
        mma16816(o[d], pa, b0, b1);
        mma16816(o[d + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();

  // Normalise and store rows g and g + 8 of this warp: out[b][query][head * 128 + d].
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qrow = q0 + warp * 16 + g + 8 * h;
    if (qrow >= tokens) continue;
    const float inv = 1.f / l_run[h];
    bf16* dst = out + (static_cast<int64_t>(b) * tokens + qrow) * (q_heads * kD) + head * kD;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      *reinterpret_cast<uint32_t*>(dst + d * 8 + 2 * t) = pack_bf16x2(o[d][2 * h] * inv, o[d][2 * h + 1] * inv);
    }
  }
}

}  // namespace

cudaError_t launch_prefill_attention(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                     int kv_heads, int tokens, int capacity, cudaStream_t stream) {
  const size_t smem = 5 * kTileBytes;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const dim3 grid((tokens + kBM - 1) / kBM, q_heads, batch);
  prefill_attention_kernel<<<grid, kThreads, smem, stream>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                                                             static_cast<const bf16*>(v), static_cast<bf16*>(out),
                                                             q_heads, kv_heads, tokens, capacity);
  return cudaGetLastError();
}

}  // namespace ipe
