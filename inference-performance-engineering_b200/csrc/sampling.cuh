// Counter-based random numbers and the mergeable sampling statistic shared by the LM-head epilogue
// and the sampling kernels.
#pragma once

#include "common.cuh"

namespace ipe {

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

// Mergeable sampling statistic over a set of logits: max m, sum of exp(l - m) s, argmax arg (lowest
// ID on ties), and the Gumbel maximum gs with its ID garg and logit gl.
struct Stat {
  float m, s;
  int arg;
  float gs;
  int garg;
  float gl;
};

// The neutral statistic (merging it changes nothing).
__device__ __forceinline__ Stat empty_stat() { return Stat{-INFINITY, 0.f, 0x7fffffff, -INFINITY, 0x7fffffff, 0.f}; }

// The statistic of lane (lane ^ o).
__device__ __forceinline__ Stat shfl_xor_stat(const Stat& st, int o) {
  return Stat{__shfl_xor_sync(0xffffffffu, st.m, o),   __shfl_xor_sync(0xffffffffu, st.s, o),
              __shfl_xor_sync(0xffffffffu, st.arg, o), __shfl_xor_sync(0xffffffffu, st.gs, o),
              __shfl_xor_sync(0xffffffffu, st.garg, o), __shfl_xor_sync(0xffffffffu, st.gl, o)};
}

// The record of one statistic (IPE_PARTIAL_WORDS floats): m, s, gs, gl, arg, garg as int bits.
__device__ __forceinline__ Stat load_stat(const float* rec) {
  return Stat{__ldcg(rec), __ldcg(rec + 1), __float_as_int(__ldcg(rec + 4)), __ldcg(rec + 2),
              __float_as_int(__ldcg(rec + 5)), __ldcg(rec + 3)};
}

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
    x.gl = y.gl;
  }
  return x;
}


}  // namespace ipe
