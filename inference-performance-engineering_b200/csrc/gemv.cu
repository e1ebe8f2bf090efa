// Decode linear layers: weight-streaming GEMV for 1..16 activation rows on the tensor pipe.
//
// Each CTA owns 16 (or 32) weight rows and the whole reduction dimension; its 8 warps split K in
// 32-wide chunks. A thread streams 16-byte pieces of two weight rows with L1-bypassing loads and
// feeds them to mma.sync m16n8k16 as the A operand; the activations are the B operand. The MMA's
// K order is permuted the same way for A and B (physical k = 8*tig + j), which keeps every weight
// load a contiguous 16 bytes while the dot product is unchanged. Per-warp partial tiles are
// summed through shared memory and the epilogue applies the reference's rounding points.
#include "common.cuh"
#include "launch.h"

namespace ipe {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kPadElems = 32;  // 64-byte pad per staged activation row: conflict-free 16-byte reads

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11): first word.
__device__ __forceinline__ uint32_t philox_word(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                                uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

// Uniform on [0, 1) with 24 random bits, for (vocab id, batch row, sampled-token index).
__device__ __forceinline__ float uniform01(uint64_t seed, int n, int b, int64_t step) {
  const uint32_t r = philox_word(static_cast<uint32_t>(n), static_cast<uint32_t>(b), static_cast<uint32_t>(step),
                                 static_cast<uint32_t>(step >> 32), static_cast<uint32_t>(seed),
                                 static_cast<uint32_t>(seed >> 32));
  return static_cast<float>(r >> 8) * (1.0f / 16777216.0f);
}

template <int RT, int EPI>
__device__ __forceinline__ int weight_row(int block, int rt, int r) {
  if constexpr (EPI == kGemvSiluMul) {
    // 16 intermediate rows j0..j0+15 per block: gate rows, then the matching up rows.
    const int j0 = block * 16;
    return (j0 / IPE_GATE_UP_GROUP) * (2 * IPE_GATE_UP_GROUP) + (j0 % IPE_GATE_UP_GROUP) + rt * IPE_GATE_UP_GROUP + r;
  } else {
    return block * 16 * RT + rt * 16 + r;
  }
}

template <int NT, int RT, bool NORM, int EPI, int U>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = a.k, B = a.batch;
  const bf16* __restrict__ x = static_cast<const bf16*>(a.x);
  const bf16* __restrict__ w = static_cast<const bf16*>(a.w);
  const int xs_stride = K + kPadElems;
  bf16* xs = reinterpret_cast<bf16*>(smem);
  float* red = reinterpret_cast<float*>(smem + (NORM ? static_cast<size_t>(B) * xs_stride * 2 : 0));
  constexpr int kRows = RT * 16, kCols = NT * 8, kOut = kRows * kCols;
  float* fin = red + kWarps * kOut;

  if constexpr (NORM) {
    // Stage rms_norm(x) rows in shared memory with the reference's two roundings.
    const bf16* __restrict__ nw = static_cast<const bf16*>(a.norm_weight);
    for (int b = warp; b < B; b += kWarps) {
      const bf16* xr = x + b * a.x_stride;
      float ss = 0.f;
      for (int c = lane; c < K / 8; c += 32) {
        float f[8];
        unpack8(ldg16(xr + c * 8), f);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
      }
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss / static_cast<float>(K) + a.eps);
      for (int c = lane; c < K / 8; c += 32) {
        float f[8], wf[8], h[8];
        unpack8(ldg16(xr + c * 8), f);
        unpack8(ldg16(nw + c * 8), wf);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = wf[i] * bf16_round(f[i] * rstd);
        *reinterpret_cast<uint4*>(xs + b * xs_stride + c * 8) = pack8(h);
      }
    }
    __syncthreads();
  }

  int rows_idx[RT][2];
  bool rows_ok[RT][2];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = weight_row<RT, EPI>(blockIdx.x, rt, g + 8 * h);
      rows_ok[rt][h] = r < a.rows;
      rows_idx[rt][h] = rows_ok[rt][h] ? r : 0;
    }
  }

  float acc[RT][NT][4];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[rt][j][i] = 0.f;

  const int chunks = K / 32;
  for (int c0 = warp; c0 < chunks; c0 += kWarps * U) {
    uint4 wv[U][RT][2];
    uint4 xv[U][NT];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * kWarps;
      const bool live = c < chunks;
      const int k = c * 32 + 8 * t;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          wv[u][rt][h] = (live && rows_ok[rt][h]) ? ldg_stream(w + static_cast<int64_t>(rows_idx[rt][h]) * K + k)
                                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int b = 8 * j + g;
        if (live && b < B) {
          if constexpr (NORM) xv[u][j] = *reinterpret_cast<const uint4*>(xs + b * xs_stride + k);
          else xv[u][j] = ldg16(x + b * a.x_stride + k);
        } else {
          xv[u][j] = make_uint4(0, 0, 0, 0);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          mma16816(acc[rt][j], wv[u][rt][0].x, wv[u][rt][1].x, wv[u][rt][0].y, wv[u][rt][1].y, xv[u][j].x,
                   xv[u][j].y);
          mma16816(acc[rt][j], wv[u][rt][0].z, wv[u][rt][1].z, wv[u][rt][0].w, wv[u][rt][1].w, xv[u][j].z,
                   xv[u][j].w);
        }
  }

  // Cross-warp reduction: red[warp][row][col], col = batch row.
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rt * 16 + g + 8 * (i >> 1);
        const int col = 8 * j + 2 * t + (i & 1);
        red[(warp * kRows + r) * kCols + col] = acc[rt][j][i];
      }
  __syncthreads();
  for (int o = threadIdx.x; o < kOut; o += kThreads) {
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < kWarps; ++v) s += red[v * kOut + o];
    fin[o] = s;
  }
  __syncthreads();

  if constexpr (EPI == kGemvStore || EPI == kGemvResidual) {
    bf16* out = static_cast<bf16*>(a.out);
    for (int o = threadIdx.x; o < kOut; o += kThreads) {
      const int r = o / kCols, b = o % kCols;
      const int n = weight_row<RT, EPI>(blockIdx.x, r / 16, r % 16);
      if (b >= B || n >= a.rows) continue;
      bf16* dst = out + b * a.out_stride + n;
      if constexpr (EPI == kGemvStore) {
        *dst = __float2bfloat16_rn(fin[o]);
      } else {
        *dst = __float2bfloat16_rn(__bfloat162float(*dst) + bf16_round(fin[o]));
      }
    }
  } else if constexpr (EPI == kGemvSiluMul) {
    bf16* out = static_cast<bf16*>(a.out);
    for (int o = threadIdx.x; o < 16 * kCols; o += kThreads) {
      const int r = o / kCols, b = o % kCols;
      if (b >= B) continue;
      const float gate = bf16_round(fin[r * kCols + b]);
      const float up = bf16_round(fin[(16 + r) * kCols + b]);
      const float act = bf16_round(gate / (1.0f + expf(-gate)));
      out[b * a.out_stride + blockIdx.x * 16 + r] = __float2bfloat16_rn(act * up);
    }
  } else {  // logits + sampling partials
    float* logits = static_cast<float*>(a.out);
    for (int o = threadIdx.x; o < kOut; o += kThreads) {
      const int r = o / kCols, b = o % kCols;
      const int n = weight_row<RT, EPI>(blockIdx.x, r / 16, r % 16);
      const float l = bf16_round(fin[o]);
      fin[o] = l;
      if (b < B && n < a.rows) logits[b * a.out_stride + n] = l;
    }
    __syncthreads();
    if (threadIdx.x < B) {
      const int b = threadIdx.x;
      const int n0 = weight_row<RT, EPI>(blockIdx.x, 0, 0);
      const int valid = min(kRows, a.rows - n0);
      float m = -INFINITY;
      int arg = n0;
      for (int r = 0; r < valid; ++r) {
        const float l = fin[r * kCols + b];
        if (l > m) {
          m = l;
          arg = n0 + r;
        }
      }
      float s = 0.f;
      if (m > -INFINITY)
        for (int r = 0; r < valid; ++r) s += expf(fin[r * kCols + b] - m);
      float gs = -INFINITY;
      int garg = n0;
      const float temperature = a.state ? __int_as_float(static_cast<int>(a.state[IPE_STATE_TEMPERATURE])) : a.temperature;
      if (temperature > 0.f) {
        const uint64_t seed = a.state ? static_cast<uint64_t>(a.state[IPE_STATE_SEED]) : a.seed;
        const int64_t step = a.state ? a.state[IPE_STATE_STEP] : 0;
        for (int r = 0; r < valid; ++r) {
          const float u = uniform01(seed, n0 + r, b, step);
          const float score = fin[r * kCols + b] / temperature - logf(-logf(u));
          if (score > gs) {
            gs = score;
            garg = n0 + r;
          }
        }
      }
      float* rec = a.partials + (static_cast<int64_t>(blockIdx.x) * B + b) * IPE_PARTIAL_WORDS;
      rec[0] = m;
      rec[1] = s;
      rec[2] = gs;
      rec[3] = 0.f;
      rec[4] = __int_as_float(arg);
      rec[5] = __int_as_float(garg);
    }
  }
}

template <int NT, int RT, bool NORM, int EPI, int U>
cudaError_t launch_one(const GemvArgs& a, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes(a);
  auto kernel = gemv_kernel<NT, RT, NORM, EPI, U>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int per_block = EPI == kGemvSiluMul ? 16 : 16 * RT;
  const int logical_rows = EPI == kGemvSiluMul ? a.rows / 2 : a.rows;
  const unsigned blocks = static_cast<unsigned>((logical_rows + per_block - 1) / per_block);
  kernel<<<blocks, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <int NT>
cudaError_t dispatch(const GemvArgs& a, cudaStream_t stream) {
  switch (a.epilogue) {
    case kGemvStore:
      return launch_one<NT, 1, true, kGemvStore, 4>(a, stream);
    case kGemvResidual:
      return launch_one<NT, 1, false, kGemvResidual, 4>(a, stream);
    case kGemvSiluMul:
      return launch_one<NT, 2, true, kGemvSiluMul, 2>(a, stream);
    default:
      return launch_one<NT, 2, true, kGemvLogits, 2>(a, stream);
  }
}

// -------------------------------------------------------------------------------- sampling
struct Stat {
  float m, s;
  int arg;
  float gs;
  int garg;
};

__device__ __forceinline__ Stat merge(Stat x, const Stat& y) {
  if (y.m > x.m) {
    x.s = (x.m == -INFINITY ? 0.f : x.s * expf(x.m - y.m)) + y.s;
    x.m = y.m;
    x.arg = y.arg;
  } else if (y.m > -INFINITY) {
    x.s += y.s * expf(y.m - x.m);
    if (y.m == x.m && y.arg < x.arg) x.arg = y.arg;
  }
  if (y.gs > x.gs || (y.gs == x.gs && y.garg < x.garg)) {
    x.gs = y.gs;
    x.garg = y.garg;
  }
  return x;
}

__global__ void __launch_bounds__(1024) sample_kernel(const float* __restrict__ partials, int parts,
                                                      const float* __restrict__ logits, int B, int V,
                                                      float temperature_arg, int64_t* state, int64_t* tokens,
                                                      float* logprobs, int64_t stride, int64_t* next_tokens) {
  __shared__ Stat shared[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_row = 32 / B;  // warps per batch row (B <= 16)
  const int b = warp / per_row, sub = warp % per_row;
  const int64_t step = state ? state[IPE_STATE_STEP] : 0;
  const float temperature = state ? __int_as_float(static_cast<int>(state[IPE_STATE_TEMPERATURE])) : temperature_arg;
  Stat st{-INFINITY, 0.f, 0x7fffffff, -INFINITY, 0x7fffffff};
  if (b < B) {
    for (int p = sub * 32 + lane; p < parts; p += per_row * 32) {
      const float* rec = partials + (static_cast<int64_t>(p) * B + b) * IPE_PARTIAL_WORDS;
      st = merge(st, Stat{rec[0], rec[1], __float_as_int(rec[4]), rec[2], __float_as_int(rec[5])});
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stat y{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
           __shfl_xor_sync(0xffffffffu, st.arg, o), __shfl_xor_sync(0xffffffffu, st.gs, o),
           __shfl_xor_sync(0xffffffffu, st.garg, o)};
    st = merge(st, y);
  }
  if (lane == 0) shared[warp] = st;
  __syncthreads();
  if (threadIdx.x < B) {
    const int row = threadIdx.x;
    Stat r = shared[row * per_row];
    for (int i = 1; i < per_row; ++i) r = merge(r, shared[row * per_row + i]);
    const int token = temperature > 0.f ? r.garg : r.arg;
    const float logit = logits[static_cast<int64_t>(row) * V + token];
    const float lp = (logit - r.m) - logf(r.s);
    tokens[row * stride + step] = token;
    logprobs[row * stride + step] = lp;
    if (next_tokens) next_tokens[row] = token;
  }
  __syncthreads();
  if (threadIdx.x == 0 && state) state[IPE_STATE_STEP] = step + 1;
}

// Token and untempered log-probability per row of a logits matrix [rows, V]: one CTA per row.
// Gumbel noise for (seed, row, vocab id) when temperature > 0.
__global__ void __launch_bounds__(256) sample_logits_kernel(const float* __restrict__ logits, int V, float temperature,
                                                            uint64_t seed, int64_t* tokens, float* logprobs,
                                                            int64_t stride) {
  const int64_t row = blockIdx.x;
  const float* l = logits + row * V;
  Stat st{-INFINITY, 0.f, 0x7fffffff, -INFINITY, 0x7fffffff};
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = l[v];
    Stat y{x, 1.f, v, -INFINITY, 0x7fffffff};
    if (temperature > 0.f) {
      const uint32_t r = philox_word(static_cast<uint32_t>(v), static_cast<uint32_t>(row),
                                     static_cast<uint32_t>(row >> 32), 0xffffffffu, static_cast<uint32_t>(seed),
                                     static_cast<uint32_t>(seed >> 32));
      const float u = static_cast<float>(r >> 8) * (1.0f / 16777216.0f);
      y.gs = x / temperature - logf(-logf(u));
      y.garg = v;
    }
    st = merge(st, y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stat y{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
           __shfl_xor_sync(0xffffffffu, st.arg, o), __shfl_xor_sync(0xffffffffu, st.gs, o),
           __shfl_xor_sync(0xffffffffu, st.garg, o)};
    st = merge(st, y);
  }
  __shared__ Stat shared[8];
  if ((threadIdx.x & 31) == 0) shared[threadIdx.x >> 5] = st;
  __syncthreads();
  if (threadIdx.x == 0) {
    Stat r = shared[0];
    for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) r = merge(r, shared[i]);
    const int token = temperature > 0.f ? r.garg : r.arg;
    tokens[row * stride] = token;
    logprobs[row * stride] = (l[token] - r.m) - logf(r.s);
  }
}

}  // namespace

int gemv_rows_per_block(int epilogue) { return epilogue == kGemvStore || epilogue == kGemvResidual ? 16 : 32; }

size_t gemv_smem_bytes(const GemvArgs& a) {
  const int nt = a.batch <= 8 ? 1 : 2;
  const int rt = (a.epilogue == kGemvStore || a.epilogue == kGemvResidual) ? 1 : 2;
  const bool norm = a.epilogue != kGemvResidual;
  const size_t out = static_cast<size_t>(rt) * 16 * nt * 8;
  size_t bytes = (kWarps + 1) * out * sizeof(float);
  if (norm) bytes += static_cast<size_t>(a.batch) * (a.k + kPadElems) * 2;
  return bytes;
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream) {
  return a.batch <= 8 ? dispatch<1>(a, stream) : dispatch<2>(a, stream);
}

void launch_sample(const float* partials, int parts, const float* logits, int batch, int vocab, float temperature,
                   int64_t* state, int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens,
                   cudaStream_t stream) {
  sample_kernel<<<1, 1024, 0, stream>>>(partials, parts, logits, batch, vocab, temperature, state, tokens, logprobs,
                                        stride, next_tokens);
}

}  // namespace ipe

namespace ipe {
void launch_sample_logits(const float* logits, int64_t rows, int vocab, float temperature, uint64_t seed,
                          int64_t* tokens, float* logprobs, int64_t stride, cudaStream_t stream) {
  sample_logits_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(logits, vocab, temperature, seed, tokens,
                                                                        logprobs, stride);
}
}  // namespace ipe
