// Reference-precision kernels: the dense Qwen3 path at dtype float32, as the reference computes it
// with TF32 disabled (src/ipe/forward.py:42-43): fp32 storage, fp32 FMA arithmetic, no bf16
// rounding points and no tensor cores. They serve Engine / forward_full at dtype=torch.float32
// (the plumbing configuration); throughput is not their purpose, so they favour simple, exact
// structure over the streaming and tcgen05 machinery of the bf16 path.
#include "common.cuh"
#include "launch.h"

namespace ipe {
namespace {

constexpr int kTile = 64;    // output tile edge of the fp32 GEMM
constexpr int kTileK = 16;   // reduction slice staged per step
constexpr float kScale = 0.08838834764831845f;  // 128 ** -0.5

// C[m, n] = epilogue(sum_k A[m, k] * W[n, k]), A [M, K], W [N, K] row-major fp32. One 256-thread CTA
// per 64 x 64 output tile (for SiLU*up: 64 activation columns, whose 64 gate rows and 64 up rows
// sit together in W, rows 128 j .. 128 j + 127 for columns 64 j ..); each thread owns 4 x 4
// outputs and sums each 16-wide k slice into a fresh partial before adding it to the total.
template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, const float* __restrict__ W,
                                                       float* C, int M, int N, int K, const float* R) {
  __shared__ float as[kTileK][kTile + 4];
  __shared__ float ws[kTileK][kTile + 4];
  __shared__ float us[kTileK][kTile + 4];  // the up rows (SiLU*up only)
  const int tm = blockIdx.y * kTile, tn = blockIdx.x * kTile;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  // rows of W feeding this tile: gate rows (and up rows) for SiLU*up, else the output columns
  const int w_row0 = EPI == kGemvSiluMul ? 2 * tn : tn;
  const int w_rows = EPI == kGemvSiluMul ? 2 * N : N;  // N is the activation width for SiLU*up
  float acc[4][4] = {}, acc_up[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kTileK) {
    for (int i = threadIdx.x; i < kTile * kTileK; i += 256) {
      const int r = i / kTileK, kk = i % kTileK;
      const bool kin = k0 + kk < K;
      as[kk][r] = tm + r < M && kin ? A[static_cast<int64_t>(tm + r) * K + k0 + kk] : 0.f;
      ws[kk][r] = w_row0 + r < w_rows && kin ? W[static_cast<int64_t>(w_row0 + r) * K + k0 + kk] : 0.f;
      if constexpr (EPI == kGemvSiluMul)
        us[kk][r] = w_row0 + kTile + r < w_rows && kin ? W[static_cast<int64_t>(w_row0 + kTile + r) * K + k0 + kk] : 0.f;
    }
    __syncthreads();
    // two-level summation: this slice's 16 products into a fresh partial, then into the total,
    // so rounding error grows with K / 16 + 16 rather than with K
    float part[4][4] = {}, part_up[4][4] = {};
#pragma unroll
    for (int kk = 0; kk < kTileK; ++kk) {
      float a[4], b[4], u[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = as[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
        if constexpr (EPI == kGemvSiluMul) u[i] = us[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          part[i][j] = fmaf(a[i], b[j], part[i][j]);
          if constexpr (EPI == kGemvSiluMul) part_up[i][j] = fmaf(a[i], u[j], part_up[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] += part[i][j];
        if constexpr (EPI == kGemvSiluMul) acc_up[i][j] += part_up[i][j];
      }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = tm + ty * 4 + i, col = tn + tx * 4 + j;
      if (row >= M || col >= N) continue;
      const int64_t o = static_cast<int64_t>(row) * N + col;
      if constexpr (EPI == kGemvResidual) {
        C[o] = R[o] + acc[i][j];
      } else if constexpr (EPI == kGemvSiluMul) {
        const float gate = acc[i][j];
        C[o] = gate / (1.0f + expf(-gate)) * acc_up[i][j];
      } else {
        C[o] = acc[i][j];
      }
    }
}

__global__ void __launch_bounds__(256) embed_f32_kernel(const int64_t* __restrict__ ids, const float* __restrict__ table,
                                                        int64_t vocab, int hidden, float* __restrict__ out,
                                                        int64_t total, int* err) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int64_t row = i / hidden;
  const int col = static_cast<int>(i % hidden);
  const int64_t id = ids[row];
  if (id < 0 || id >= vocab) {
    if (col == 0) report(err, kErrTokenRange);
    out[i] = 0.f;
    return;
  }
  out[i] = table[id * hidden + col];
}

// One warp per (token, head slot): q heads, k heads, v heads; lane l holds elements 4l .. 4l+3, so
// the rotate-half partner (d +- 64) is lane l ^ 16. RMSNorm over the head and RoPE in fp32
// (src/ipe/ops.py:36-63 at dtype float32), then the cache append.
__global__ void __launch_bounds__(256) qk_norm_rope_append_f32_kernel(
    const float* __restrict__ qkv, int tokens, int q_heads, int kv_heads, const float* __restrict__ q_norm_w,
    const float* __restrict__ k_norm_w, const float* __restrict__ cos_t, const float* __restrict__ sin_t, int start,
    float* __restrict__ q_out, float* __restrict__ k_cache, float* __restrict__ v_cache, int capacity, float eps,
    int64_t total_warps, int* err) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (warp >= total_warps) return;
  const int lane = threadIdx.x & 31;
  const int slots = q_heads + 2 * kv_heads;
  const int slot = static_cast<int>(warp % slots);
  const int64_t row = warp / slots;
  const int t = static_cast<int>(row % tokens);
  const int b = static_cast<int>(row / tokens);
  const int pos = start + t;
  if (pos < 0 || pos >= capacity) {
    if (lane == 0) report(err, kErrPositionRange);
    return;
  }
  const int d0 = lane * 4;
  const float4 raw = *reinterpret_cast<const float4*>(qkv + row * (static_cast<int64_t>(slots) * 128) + slot * 128 + d0);
  float x[4] = {raw.x, raw.y, raw.z, raw.w};
  if (slot >= q_heads + kv_heads) {
    const int h = slot - q_heads - kv_heads;
    *reinterpret_cast<float4*>(v_cache + ((static_cast<int64_t>(b) * kv_heads + h) * capacity + pos) * 128 + d0) = raw;
    return;
  }
  const bool is_q = slot < q_heads;
  const float* nw = is_q ? q_norm_w : k_norm_w;
  const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float rstd = rsqrtf(ss / 128.f + eps);
  float h[4], p[4], o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = nw[d0 + i] * (x[i] * rstd);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, h[i], 16);
  const float* cr = cos_t + static_cast<int64_t>(pos) * 128 + d0;
  const float* sr = sin_t + static_cast<int64_t>(pos) * 128 + d0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float rot = d0 < 64 ? -p[i] : p[i];
    o[i] = h[i] * cr[i] + rot * sr[i];
  }
  float* dst = is_q ? q_out + ((static_cast<int64_t>(b) * q_heads + slot) * tokens + t) * 128 + d0
                    : k_cache + ((static_cast<int64_t>(b) * kv_heads + (slot - q_heads)) * capacity + pos) * 128 + d0;
  *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
}

// One 128-thread CTA per (query token t, query head, row): query t at position start + t attends
// cache keys 0 .. start + t (causal; a decode step is tokens = 1). GQA: query head j reads KV head
// j / (q_heads / kv_heads). fp32 scores, softmax and P.V.
__global__ void __launch_bounds__(128) attention_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                            const float* __restrict__ v, float* __restrict__ out,
                                                            int q_heads, int kv_heads, int tokens, int capacity,
                                                            int start) {
  extern __shared__ float sm[];
  float* qs = sm;         // [128]
  float* sc = sm + 128;   // [keys]
  __shared__ float red[4];
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (q_heads / kv_heads);
  const int keys = start + t + 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  qs[tid] = q[((static_cast<int64_t>(b) * q_heads + h) * tokens + t) * 128 + tid];
  __syncthreads();
  const float* kh = k + (static_cast<int64_t>(b) * kv_heads + kvh) * capacity * 128;
  const float* vh = v + (static_cast<int64_t>(b) * kv_heads + kvh) * capacity * 128;
  float m = -INFINITY;
  for (int j = tid; j < keys; j += 128) {
    const float4* kr = reinterpret_cast<const float4*>(kh + static_cast<int64_t>(j) * 128);
    float dot = 0.f;
    for (int d0 = 0; d0 < 32; d0 += 4) {  // 16 products per partial, then into the total
      float part = 0.f;
#pragma unroll
      for (int d = d0; d < d0 + 4; ++d) {
        const float4 kv4 = kr[d];
        part = fmaf(qs[4 * d], kv4.x, part);
        part = fmaf(qs[4 * d + 1], kv4.y, part);
        part = fmaf(qs[4 * d + 2], kv4.z, part);
        part = fmaf(qs[4 * d + 3], kv4.w, part);
      }
      dot += part;
    }
    sc[j] = dot * kScale;
    m = fmaxf(m, sc[j]);
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float l = 0.f;
  for (int j = tid; j < keys; j += 128) {
    const float p = expf(sc[j] - m);
    sc[j] = p;
    l += p;
  }
  l = warp_sum(l);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  l = red[0] + red[1] + red[2] + red[3];
  float o = 0.f;
  for (int j0 = 0; j0 < keys; j0 += 16) {  // blocks of 16 keys, then into the total
    float part = 0.f;
    for (int j = j0; j < min(j0 + 16, keys); ++j) part = fmaf(sc[j], vh[static_cast<int64_t>(j) * 128 + tid], part);
    o += part;
  }
  out[(static_cast<int64_t>(b) * tokens + t) * (q_heads * 128) + h * 128 + tid] = o / l;
}

}  // namespace

cudaError_t launch_gemm_f32(const void* a, const void* w, void* c, int m, int n, int k, int epilogue,
                            const void* residual, cudaStream_t stream) {
  const int cols = epilogue == kGemvSiluMul ? n / 2 : n;  // n: rows of w
  const dim3 grid((cols + kTile - 1) / kTile, (m + kTile - 1) / kTile);
  auto A = static_cast<const float*>(a);
  auto W = static_cast<const float*>(w);
  auto C = static_cast<float*>(c);
  auto R = static_cast<const float*>(residual);
  switch (epilogue) {
    case kGemvStore:
    case kGemvLogits: gemm_f32_kernel<kGemvStore><<<grid, 256, 0, stream>>>(A, W, C, m, cols, k, R); break;
    case kGemvResidual: gemm_f32_kernel<kGemvResidual><<<grid, 256, 0, stream>>>(A, W, C, m, cols, k, R); break;
    case kGemvSiluMul: gemm_f32_kernel<kGemvSiluMul><<<grid, 256, 0, stream>>>(A, W, C, m, cols, k, R); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

void launch_embed_f32(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
                      int* err, cudaStream_t stream) {
  const int64_t total = count * hidden;
  embed_f32_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      ids, static_cast<const float*>(table), vocab, hidden, static_cast<float*>(out), total, err);
}

void launch_qk_norm_rope_append_f32(const void* qkv, int batch, int tokens, int q_heads, int kv_heads, const void* qn,
                                    const void* kn, const void* cos_t, const void* sin_t, int start, void* q_out,
                                    void* k_cache, void* v_cache, int capacity, float eps, int* err,
                                    cudaStream_t stream) {
  const int64_t warps = static_cast<int64_t>(batch) * tokens * (q_heads + 2 * kv_heads);
  qk_norm_rope_append_f32_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(
      static_cast<const float*>(qkv), tokens, q_heads, kv_heads, static_cast<const float*>(qn),
      static_cast<const float*>(kn), static_cast<const float*>(cos_t), static_cast<const float*>(sin_t), start,
      static_cast<float*>(q_out), static_cast<float*>(k_cache), static_cast<float*>(v_cache), capacity, eps, warps,
      err);
}

cudaError_t launch_attention_f32(const void* q, const void* k, const void* v, void* out, int batch, int q_heads,
                                 int kv_heads, int tokens, int capacity, int start, cudaStream_t stream) {
  const size_t smem = (128 + static_cast<size_t>(start + tokens)) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  attention_f32_kernel<<<dim3(tokens, q_heads, batch), 128, smem, stream>>>(
      static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
      static_cast<float*>(out), q_heads, kv_heads, tokens, capacity, start);
  return cudaGetLastError();
}

}  // namespace ipe
