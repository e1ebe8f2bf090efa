// Direct-to-device reads of tensor payloads from a checkpoint file (safetensors stores each tensor
// as one contiguous little-endian byte range), replacing the reference's per-tensor
// mmap -> .to(dtype) -> .to(device) copies (src/ipe/weights.py:154-161).
//
// The ranges (of one or more files) are cut into chunks of at most staging_bytes, taken in list
// order by `threads` reader threads. Each reader has two pinned staging buffers (carved from one
// pinned allocation per call, since each allocation has a fixed cost): while the GPU copies one into its
// destination (cudaMemcpyAsync on the caller's stream), the reader fills the other from the file,
// so file (or page-cache) reads run in parallel and overlap the host-to-device transfer, and no
// pageable copy is made. A buffer is refilled only after the copy that read it has finished (an
// event per buffer). The call returns after every copy has finished, so the destinations are
// complete and the staging memory is released.
#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace ipe {
int report_failure(int status, const char* message);
}

namespace {

struct Staging {
  unsigned char* buffer[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool pending[2] = {false, false};

  ~Staging() {  // the buffers are views of the job's pinned block
    for (int i = 0; i < 2; ++i)
      if (done[i]) {
        if (pending[i]) cudaEventSynchronize(done[i]);
        cudaEventDestroy(done[i]);
      }
  }
};

int io_failure(const char* what, const char* path) {
  char message[512];
  snprintf(message, sizeof(message), "ipe_read_to_device: %s %s: %s", what, path, strerror(errno));
  return ipe::report_failure(IPE_ERR_IO, message);
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

namespace {

// One chunk of one range: bytes [offset, offset + bytes) of file `fd` to destination dst.
struct Chunk {
  int fd;
  uint64_t offset;
  size_t bytes;
  unsigned char* dst;
};

// The shared state of one call: the chunk list, the next chunk to take, the first failure.
struct Job {
  int device;
  cudaStream_t stream;
  size_t staging_bytes;
  unsigned char* staging;  // threads x 2 pinned buffers of staging_bytes
  std::vector<Chunk> chunks;
  std::atomic<size_t> next{0};
  std::atomic<bool> failed{false};
  std::mutex mu;
  int status = IPE_OK;
  std::string message;

  void fail(int code, const std::string& what) {
    std::lock_guard<std::mutex> lock(mu);
    if (status == IPE_OK) {
      status = code;
      message = what;
    }
    failed = true;
  }
};

// A reader: takes chunks in list order, reads each into one of its two pinned buffers (after the
// copy that last read that buffer finished) and queues its copy on the job's stream.
void reader(Job* job, int index, const std::vector<std::string>* paths, const std::vector<int>* fds) {
  if (cudaSetDevice(job->device) != cudaSuccess) {
    job->fail(IPE_ERR_CUDA, "cudaSetDevice in a reader thread");
    return;
  }
  Staging staging;  // the buffers belong to the job; the events and the final wait are this reader's
  for (int b = 0; b < 2; ++b) {
    staging.buffer[b] = job->staging + (2 * static_cast<size_t>(index) + b) * job->staging_bytes;
    const cudaError_t e = cudaEventCreateWithFlags(&staging.done[b], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      job->fail(IPE_ERR_CUDA, std::string("staging event: ") + cudaGetErrorString(e));
      staging.buffer[0] = staging.buffer[1] = nullptr;
      return;
    }
  }
  int next = 0;
  while (!job->failed) {
    const size_t i = job->next.fetch_add(1);
    if (i >= job->chunks.size()) break;
    const Chunk& c = job->chunks[i];
    if (staging.pending[next]) {
      const cudaError_t e = cudaEventSynchronize(staging.done[next]);
      staging.pending[next] = false;
      if (e != cudaSuccess) {
        job->fail(IPE_ERR_CUDA, std::string("waiting for a staging copy: ") + cudaGetErrorString(e));
        break;
      }
    }
    if (!read_fully(c.fd, staging.buffer[next], c.bytes, c.offset)) {
      size_t f = 0;
      while (f < fds->size() && (*fds)[f] != c.fd) ++f;
      job->fail(IPE_ERR_IO, std::string("cannot read ") + (f < paths->size() ? (*paths)[f] : "?") + ": " +
                                strerror(errno));
      break;
    }
    cudaError_t e = cudaMemcpyAsync(c.dst, staging.buffer[next], c.bytes, cudaMemcpyHostToDevice, job->stream);
    if (e == cudaSuccess) e = cudaEventRecord(staging.done[next], job->stream);
    if (e != cudaSuccess) {
      job->fail(IPE_ERR_CUDA, std::string("host-to-device copy: ") + cudaGetErrorString(e));
      break;
    }
    staging.pending[next] = true;
    next ^= 1;
  }
  for (int b = 0; b < 2; ++b) {  // wait for this reader's copies; the job frees the buffers
    if (staging.pending[b]) cudaEventSynchronize(staging.done[b]);
    staging.pending[b] = false;
    staging.buffer[b] = nullptr;
  }
}

struct Files {
  std::vector<int> fds;
  ~Files() {
    for (int fd : fds)
      if (fd >= 0) close(fd);
  }
};

}  // namespace

extern "C" int ipe_read_to_device(int files, const char* const* paths, int count, const int* file_of,
                                  const uint64_t* offsets, const uint64_t* sizes, void* const* destinations,
                                  size_t staging_bytes, int threads, void* stream) {
  if (files < 1 || !paths || count < 0 || (count > 0 && (!file_of || !offsets || !sizes || !destinations)))
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: null pointer or bad counts");
  if (staging_bytes < 4096)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: staging_bytes below 4096");
  if (threads < 1 || threads > 64)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: threads outside 1..64");
  Files open_files;
  std::vector<std::string> names;
  std::vector<uint64_t> file_bytes;
  for (int f = 0; f < files; ++f) {
    if (!paths[f]) return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: null path");
    names.emplace_back(paths[f]);
    const int fd = open(paths[f], O_RDONLY | O_CLOEXEC);
    if (fd < 0) return io_failure("cannot open", paths[f]);
    open_files.fds.push_back(fd);
    struct stat st;
    if (fstat(fd, &st) != 0) return io_failure("cannot stat", paths[f]);
    file_bytes.push_back(static_cast<uint64_t>(st.st_size));
#ifdef POSIX_FADV_SEQUENTIAL
    posix_fadvise(fd, 0, 0, POSIX_FADV_SEQUENTIAL);
#endif
  }
  Job job;
  job.stream = static_cast<cudaStream_t>(stream);
  job.staging_bytes = staging_bytes;
  for (int i = 0; i < count; ++i) {
    const int f = file_of[i];
    if (f < 0 || f >= files) return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: file index out of range");
    if (sizes[i] > 0 && !destinations[i])
      return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: null destination");
    if (offsets[i] > file_bytes[f] || sizes[i] > file_bytes[f] - offsets[i]) {
      char message[512];
      snprintf(message, sizeof(message), "ipe_read_to_device: range %d [%llu, +%llu) is outside %s (%llu bytes)", i,
               static_cast<unsigned long long>(offsets[i]), static_cast<unsigned long long>(sizes[i]), paths[f],
               static_cast<unsigned long long>(file_bytes[f]));
      return ipe::report_failure(IPE_ERR_ARGUMENT, message);
    }
    for (uint64_t done = 0; done < sizes[i]; done += staging_bytes)
      job.chunks.push_back({open_files.fds[f], offsets[i] + done,
                            static_cast<size_t>(std::min<uint64_t>(staging_bytes, sizes[i] - done)),
                            static_cast<unsigned char*>(destinations[i]) + done});
  }
  if (job.chunks.empty()) return IPE_OK;
  if (cudaGetDevice(&job.device) != cudaSuccess)
    return ipe::report_failure(IPE_ERR_CUDA, "ipe_read_to_device: cudaGetDevice failed");
  const int n = static_cast<int>(std::min<size_t>(threads, job.chunks.size()));
  // one pinned allocation for every reader's two buffers (each allocation has a fixed cost)
  cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&job.staging), 2 * static_cast<size_t>(n) * staging_bytes,
                                cudaHostAllocDefault);
  if (e != cudaSuccess) {
    const std::string message = std::string("ipe_read_to_device: pinned staging buffers: ") + cudaGetErrorString(e);
    return ipe::report_failure(IPE_ERR_CUDA, message.c_str());
  }
  std::vector<std::thread> workers;
  workers.reserve(n);
  for (int t = 0; t < n; ++t) workers.emplace_back(reader, &job, t, &names, &open_files.fds);
  for (std::thread& w : workers) w.join();
  cudaFreeHost(job.staging);  // every reader waited for its copies
  if (job.status != IPE_OK) {
    const std::string message = "ipe_read_to_device: " + job.message;
    return ipe::report_failure(job.status, message.c_str());
  }
  return IPE_OK;
}
