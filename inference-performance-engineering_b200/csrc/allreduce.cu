// One-shot all-reduce of a tensor-parallel layer's fp32 parts over NVLink peer memory, fused with
// the residual add that follows it (x = bf16(x + bf16(sum over ranks))). Replaces the NCCL
// all-reduce of the decode step, whose ~20 us per call dominates a batch-1 step at 56 calls.
//
// Each rank owns a communication region (ipe_comm_alloc), mapped into its peers through CUDA IPC:
//   [0, 128)            u32 flag[r]: the last epoch rank r announced to this rank (world <= 32)
//   [128, 256)          u32 epoch counter of this rank's calls
//   [256, 256 + 2 S)    two slots of S bytes: this rank's fp32 part (slot 0 and slot 1 alternate
//                       between consecutive calls, so a slot is rewritten only after every peer
//                       has finished reading it: each peer announced the call in between)
// A call: thread 0 takes epoch = counter + 1, fences at system scope (the part in this rank's slot,
// written by the preceding kernel, becomes visible to the peers) and stores the epoch into every
// peer's flag[me]; it then waits, bounded, until every peer's flag in its own region reaches the
// epoch. All threads then read every rank's slot (peer loads over NVLink), sum in rank order (the
// same bits on every rank), and apply the residual. No multicast, no NCCL.
#include "common.cuh"
#include "launch.h"

namespace ipe {
namespace {

constexpr size_t kFlagsOffset = 0;
constexpr size_t kCounterOffset = 128;
constexpr size_t kSlotsOffset = 256;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(1024) allreduce_residual_kernel(bf16* __restrict__ x, int64_t count,
                                                                  const uint64_t* __restrict__ peers, int world,
                                                                  int rank, int slot, size_t slot_bytes, int* err) {
  __shared__ unsigned epoch_smem;
  __shared__ int ok_smem;
  unsigned char* mine = reinterpret_cast<unsigned char*>(peers[rank]);
  unsigned* counter = reinterpret_cast<unsigned*>(mine + kCounterOffset);
  if (threadIdx.x == 0) {
    const unsigned epoch = *counter + 1;
    epoch_smem = epoch;
    __threadfence_system();
    for (int r = 0; r < world; ++r) {
      if (r == rank) continue;
      unsigned* flags = reinterpret_cast<unsigned*>(reinterpret_cast<unsigned char*>(peers[r]) + kFlagsOffset);
      st_release_sys(flags + rank, epoch);
    }
    // wait for every peer's announcement of this epoch (bounded)
    const unsigned* my_flags = reinterpret_cast<const unsigned*>(mine + kFlagsOffset);
    int ok = 1;
    uint64_t start = 0;
    for (int r = 0; r < world && ok; ++r) {
      if (r == rank) continue;
      for (unsigned i = 0;; ++i) {
        if (static_cast<int>(ld_acquire_sys(my_flags + r) - epoch) >= 0) break;
        if ((i & 63u) == 63u) {
          const uint64_t now = globaltimer_ns();
          if (start == 0) start = now;
          else if (now - start > kWaitLimitNs) {
            report(err, kErrWaitTimeout);
            ok = 0;
            break;
          }
        }
        __nanosleep(32);
      }
    }
    ok_smem = ok;
    *counter = epoch;
  }
  __syncthreads();
  if (!ok_smem) return;  // a peer did not arrive: x is left as it was, the error word is set
  const size_t slot_offset = kSlotsOffset + static_cast<size_t>(slot) * slot_bytes;
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
    float sum = 0.f;
    for (int r = 0; r < world; ++r) {
      const float* part = reinterpret_cast<const float*>(reinterpret_cast<const unsigned char*>(peers[r]) + slot_offset);
      sum += __ldcv(part + i);  // volatile: the peers' parts are read fresh every call
    }
    x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) + bf16_round(sum));
  }
}

}  // namespace

size_t comm_region_bytes(size_t slot_bytes) { return kSlotsOffset + 2 * ((slot_bytes + 255) / 256 * 256); }

size_t comm_slot_offset(int slot, size_t slot_bytes) {
  return kSlotsOffset + static_cast<size_t>(slot) * ((slot_bytes + 255) / 256 * 256);
}

void launch_allreduce_residual(void* x, int64_t count, const uint64_t* peers, int world, int rank, int slot,
                               size_t slot_bytes, int* err, cudaStream_t stream) {
  allreduce_residual_kernel<<<1, 1024, 0, stream>>>(static_cast<bf16*>(x), count, peers, world, rank, slot,
                                                    (slot_bytes + 255) / 256 * 256, err);
}

}  // namespace ipe
