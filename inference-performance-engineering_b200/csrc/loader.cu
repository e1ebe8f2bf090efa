// Direct-to-device reads of tensor payloads from a checkpoint file (safetensors stores each tensor
// as one contiguous little-endian byte range), replacing the reference's per-tensor
// mmap -> .to(dtype) -> .to(device) copies (src/ipe/weights.py:154-161).
//
// The ranges are cut into chunks of at most staging_bytes, taken in file order by `threads` reader
// threads. Each reader owns two pinned staging buffers: while the GPU copies one into its
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

// One chunk of one range: bytes [offset, offset + bytes) of the file to destination dst.
struct Chunk {
  uint64_t offset;
  size_t bytes;
  unsigned char* dst;
};

// The shared state of one call: the chunk list, the next chunk to take, the first failure.
struct Job {
  int fd;
  const char* path;
  int device;
  cudaStream_t stream;
  size_t staging_bytes;
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
void reader(Job* job) {
  if (cudaSetDevice(job->device) != cudaSuccess) {
    job->fail(IPE_ERR_CUDA, "cudaSetDevice in a reader thread");
    return;
  }
  Staging staging;
  for (int b = 0; b < 2; ++b) {
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&staging.buffer[b]), job->staging_bytes, cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&staging.done[b], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      job->fail(IPE_ERR_CUDA, std::string("pinned staging buffer: ") + cudaGetErrorString(e));
      return;
    }
  }
  int next = 0;
  while (!job->failed) {
    const size_t index = job->next.fetch_add(1);
    if (index >= job->chunks.size()) break;
    const Chunk& c = job->chunks[index];
    if (staging.pending[next]) {
      const cudaError_t e = cudaEventSynchronize(staging.done[next]);
      staging.pending[next] = false;
      if (e != cudaSuccess) {
        job->fail(IPE_ERR_CUDA, std::string("waiting for a staging copy: ") + cudaGetErrorString(e));
        break;
      }
    }
    if (!read_fully(job->fd, staging.buffer[next], c.bytes, c.offset)) {
      job->fail(IPE_ERR_IO, std::string("cannot read ") + job->path + ": " + strerror(errno));
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
  // ~Staging waits for this reader's copies before releasing its buffers
}

}  // namespace

extern "C" int ipe_read_to_device(const char* path, int count, const uint64_t* offsets, const uint64_t* sizes,
                                  void* const* destinations, size_t staging_bytes, int threads, void* stream) {
  if (!path || count < 0 || (count > 0 && (!offsets || !sizes || !destinations)))
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: null pointer or negative count");
  if (staging_bytes < 4096)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: staging_bytes below 4096");
  if (threads < 1 || threads > 64)
    return ipe::report_failure(IPE_ERR_ARGUMENT, "ipe_read_to_device: threads outside 1..64");
  File file;
  file.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (file.fd < 0) return io_failure("cannot open", path);
  struct stat st;
  if (fstat(file.fd, &st) != 0) return io_failure("cannot stat", path);
  const uint64_t file_bytes = static_cast<uint64_t>(st.st_size);
  Job job;
  job.fd = file.fd;
  job.path = path;
  job.stream = static_cast<cudaStream_t>(stream);
  job.staging_bytes = staging_bytes;
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
    for (uint64_t done = 0; done < sizes[i]; done += staging_bytes)
      job.chunks.push_back({offsets[i] + done, static_cast<size_t>(std::min<uint64_t>(staging_bytes, sizes[i] - done)),
                            static_cast<unsigned char*>(destinations[i]) + done});
  }
  if (job.chunks.empty()) return IPE_OK;
  if (cudaGetDevice(&job.device) != cudaSuccess)
    return ipe::report_failure(IPE_ERR_CUDA, "ipe_read_to_device: cudaGetDevice failed");
#ifdef POSIX_FADV_SEQUENTIAL
  posix_fadvise(file.fd, 0, 0, POSIX_FADV_SEQUENTIAL);
#endif
  const int n = static_cast<int>(std::min<size_t>(threads, job.chunks.size()));
  std::vector<std::thread> workers;
  workers.reserve(n);
  for (int t = 0; t < n; ++t) workers.emplace_back(reader, &job);
  for (std::thread& w : workers) w.join();
  if (job.status != IPE_OK) {
    const std::string message = "ipe_read_to_device: " + job.message;
    return ipe::report_failure(job.status, message.c_str());
  }
  return IPE_OK;
}
