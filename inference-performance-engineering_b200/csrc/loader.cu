// Direct-to-device reads of tensor payloads from a checkpoint file (safetensors stores each tensor
// as one contiguous little-endian byte range), replacing the reference's per-tensor
// mmap -> .to(dtype) -> .to(device) copies (src/ipe/weights.py:154-161).
//
// The ranges are read in file order through two pinned staging buffers: while the GPU copies one
// buffer into its destination (cudaMemcpyAsync on the caller's stream), the host reads the next
// chunk of the file into the other, so disk (or page-cache) reads overlap the host-to-device
// transfer and no pageable copy is made. A buffer is refilled only after the copy that read it
// has finished (an event per buffer). The call returns after the last copy has finished, so the
// destinations are complete and the staging memory can be released.
#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include "common.cuh"

namespace ipe {
int report_failure(int status, const char* message);
}

namespace {

struct Staging {
  unsigned char* buffer[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool pending[2] = {false, false};

  ~Staging() {
    for (int i = 0; i < 2; ++i) {
      if (done[i]) {
        if (pending[i]) cudaEventSynchronize(done[i]);
        cudaEventDestroy(done[i]);
      }
      if (buffer[i]) cudaFreeHost(buffer[i]);
    }
  }
};

struct File {
  int fd = -1;
  ~File() {
    if (fd >= 0) close(fd);
  }
};

int io_failure(const char* what, const char* path) {
  char message[512];
  snprintf(message, sizeof(message), "ipe_read_to_device: %s %s: %s", what, path, strerror(errno));
  return ipe::report_failure(IPE_ERR_IO, message);
}

int cuda_failure(cudaError_t e, const char* what) {
  char message[512];
  snprintf(message, sizeof(message), "ipe_read_to_device: %s: %s", what, cudaGetErrorString(e));
  return ipe::report_failure(IPE_ERR_CUDA, message);
}

// Reads exactly `bytes` at `offset` (pread may return short counts).
bool read_fully(int fd, unsigned char* dst, size_t bytes, uint64_t offset) {
  while (bytes > 0) {
    const ssize_t got = pread(fd, dst, bytes, static_cast<off_t>(offset));
    if (got < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    if (got == 0) {
      errno = EIO;  // the file ended early
      return false;
    }
    dst += got;
    bytes -= static_cast<size_t>(got);
    offset += static_cast<uint64_t>(got);
  }
  return true;
}

}  // namespace

extern "C" int ipe_read_to_device(const char* path, int count, const uint64_t* offsets, const uint64_t* sizes,
                                  void* const* destinations, size_t staging_bytes, void* stream) {
  if (!path || count < 0 || (count > 0 && (!offsets || !sizes || !destinations)))
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: null pointer or negative count");
  if (staging_bytes < 4096)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: staging_bytes below 4096");
  File file;
  file.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (file.fd < 0) return io_failure("cannot open", path);
  struct stat st;
  if (fstat(file.fd, &st) != 0) return io_failure("cannot stat", path);
  const uint64_t file_bytes = static_cast<uint64_t>(st.st_size);
  for (int i = 0; i < count; ++i) {
    if (sizes[i] > 0 && !destinations[i])
      return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: null destination");
    if (offsets[i] > file_bytes || sizes[i] > file_bytes - offsets[i]) {
      char message[512];
      snprintf(message, sizeof(message), "ipe_read_to_device: range %d [%llu, +%llu) is outside %s (%llu bytes)", i,
               static_cast<unsigned long long>(offsets[i]), static_cast<unsigned long long>(sizes[i]), path,
               static_cast<unsigned long long>(file_bytes));
      return ipe::report_failure(IPE_ERR_ARGUMENT, message);
    }
  }
  if (count == 0) return IPE_OK;
#ifdef POSIX_FADV_SEQUENTIAL
  posix_fadvise(file.fd, 0, 0, POSIX_FADV_SEQUENTIAL);
#endif
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  Staging staging;
  for (int b = 0; b < 2; ++b) {
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&staging.buffer[b]), staging_bytes, cudaHostAllocDefault);
    if (e != cudaSuccess) return cuda_failure(e, "pinned staging buffer");
    e = cudaEventCreateWithFlags(&staging.done[b], cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_failure(e, "staging event");
  }
  int next = 0;
  for (int i = 0; i < count; ++i) {
    unsigned char* dst = static_cast<unsigned char*>(destinations[i]);
    for (uint64_t done = 0; done < sizes[i];) {
      const size_t chunk = static_cast<size_t>(std::min<uint64_t>(staging_bytes, sizes[i] - done));
      if (staging.pending[next]) {  // the copy that last read this buffer must have finished
        const cudaError_t e = cudaEventSynchronize(staging.done[next]);
        staging.pending[next] = false;
        if (e != cudaSuccess) return cuda_failure(e, "waiting for a staging copy");
      }
      if (!read_fully(file.fd, staging.buffer[next], chunk, offsets[i] + done)) return io_failure("cannot read", path);
      cudaError_t e = cudaMemcpyAsync(dst + done, staging.buffer[next], chunk, cudaMemcpyHostToDevice, s);
      if (e == cudaSuccess) e = cudaEventRecord(staging.done[next], s);
      if (e != cudaSuccess) return cuda_failure(e, "host-to-device copy");
      staging.pending[next] = true;
      done += chunk;
      next ^= 1;
    }
  }
  for (int b = 0; b < 2; ++b) {
    if (!staging.pending[b]) continue;
    const cudaError_t e = cudaEventSynchronize(staging.done[b]);
    staging.pending[b] = false;
    if (e != cudaSuccess) return cuda_failure(e, "waiting for the last copies");
  }
  return IPE_OK;
}
