// Expert-file reader: byte ranges of one file -> device (or host) memory.
//
// The reference streams expert slices from SSD with a Python thread pool of os.preadv calls straight
// into unified memory (engine/mimo_stream/store.py:14-82: ExpertStore.jobs gives (fd, offset, view)
// per slot tensor, IOPool runs them, F_NOCACHE and read-ahead off).  Here the HBM pools are filled
// once at load time, so the reader is a bulk copier: reader threads pread the ranges in chunks into
// pinned staging buffers (two per thread, so one chunk's host->device copy overlaps the next read;
// the buffers are kept for the next call), each thread copying on its own stream.  O_DIRECT is used
// for chunks whose offset and size are multiples of 4 KiB (every expert slice of a converted file is
// 16 KiB aligned), buffered reads for the rest or when the filesystem refuses O_DIRECT.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdint>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/mimo_moe.h"

namespace {

constexpr int64_t kDirectAlign = 4096;

struct Chunk {
  int64_t off, n;
  char* dst;
};

// pread until n bytes or an error/EOF; returns bytes read, or -errno.
int64_t read_full(int fd, char* buf, int64_t n, int64_t off) {
  int64_t got = 0;
  while (got < n) {
    const ssize_t r = pread(fd, buf + got, (size_t)(n - got), (off_t)(off + got));
    if (r < 0) {
      if (errno == EINTR) continue;
      return -errno;
    }
    if (r == 0) break;
    got += r;
  }
  return got;
}

bool direct_ok(const Chunk& c, const char* buf) {
  return c.off % kDirectAlign == 0 && c.n % kDirectAlign == 0 && ((uintptr_t)buf % kDirectAlign) == 0;
}

// Pinned staging buffers outlive a call (allocating pinned memory costs more than reading a layer
// from the page cache): a process-wide free list of buffers of one size, refilled on demand.
struct StagingPool {
  std::mutex mu;
  int64_t bytes = 0;
  std::vector<char*> free_list;

  char* take(int64_t n) {
    {
      std::lock_guard<std::mutex> g(mu);
      if (n != bytes) {  // a new chunk size: drop the old buffers (none are in use between calls)
        for (char* b : free_list) cudaFreeHost(b);
        free_list.clear();
        bytes = n;
      }
      if (!free_list.empty()) {
        char* b = free_list.back();
        free_list.pop_back();
        return b;
      }
    }
    char* b = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&b), (size_t)n, cudaHostAllocDefault) != cudaSuccess) return nullptr;
    return b;
  }
  void give(char* b, int64_t n) {
    std::lock_guard<std::mutex> g(mu);
    if (n == bytes && free_list.size() < 64) free_list.push_back(b);
    else cudaFreeHost(b);
  }
};

StagingPool& staging() {
  static StagingPool* pool = new StagingPool();  // never destroyed: no CUDA calls at process exit
  return *pool;
}

// One call at a time per process shares the pool's chunk size.
std::mutex& read_call_mutex() {
  static std::mutex m;
  return m;
}

}  // namespace

extern "C" int mimo_moe_read_file_spans(const char* path, const mimo_moe_file_span* spans, int32_t n,
                                        int32_t threads, int64_t chunk_bytes, int32_t direct, int32_t dst_host,
                                        void* stream) {
  if (!path || (n > 0 && !spans) || n < 0 || threads < 1 || threads > 64 || chunk_bytes < kDirectAlign ||
      chunk_bytes % kDirectAlign)
    return MIMO_EINVAL;
  std::vector<Chunk> chunks;
  for (int32_t i = 0; i < n; ++i) {
    const mimo_moe_file_span& s = spans[i];
    if (s.file_offset < 0 || s.nbytes < 0 || (s.nbytes > 0 && !s.dst)) return MIMO_EINVAL;
    for (int64_t o = 0; o < s.nbytes; o += chunk_bytes)
      chunks.push_back({s.file_offset + o, std::min(chunk_bytes, s.nbytes - o), static_cast<char*>(s.dst) + o});
  }
  if (chunks.empty()) return MIMO_OK;
  const int fd_buf = open(path, O_RDONLY | O_CLOEXEC);
  if (fd_buf < 0) return MIMO_EIO;
  int fd_direct = -1;
  if (direct && !dst_host) fd_direct = open(path, O_RDONLY | O_CLOEXEC | O_DIRECT);
  std::atomic<bool> use_direct{fd_direct >= 0};

  std::atomic<int> err{MIMO_OK};
  std::atomic<size_t> next{0};
  auto fail = [&](int code) {
    int expect = MIMO_OK;
    err.compare_exchange_strong(expect, code);
  };
  const int nthreads = (int)std::min<size_t>((size_t)threads, chunks.size());

  if (dst_host) {  // plain reads straight into the caller's host memory
    auto worker = [&]() {
      for (size_t i; err.load() == MIMO_OK && (i = next.fetch_add(1)) < chunks.size();) {
        const Chunk& c = chunks[i];
        if (read_full(fd_buf, c.dst, c.n, c.off) != c.n) fail(MIMO_EIO);
      }
    };
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) pool.emplace_back(worker);
    for (auto& th : pool) th.join();
    close(fd_buf);
    return err.load();
  }

  std::lock_guard<std::mutex> serial(read_call_mutex());
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    close(fd_buf);
    if (fd_direct >= 0) close(fd_direct);
    return MIMO_ECUDA;
  }
  // the pools may reuse memory that work already queued on the caller's stream still touches
  cudaEvent_t entry = nullptr;
  if (cudaEventCreateWithFlags(&entry, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventRecord(entry, static_cast<cudaStream_t>(stream)) != cudaSuccess) {
    close(fd_buf);
    if (fd_direct >= 0) close(fd_direct);
    return MIMO_ECUDA;
  }
  auto worker = [&]() {
    if (cudaSetDevice(dev) != cudaSuccess) return fail(MIMO_ECUDA);
    cudaStream_t st = nullptr;
    char* buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool pending[2] = {false, false};
    bool ok = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamWaitEvent(st, entry, 0) == cudaSuccess;
    for (int b = 0; b < 2 && ok; ++b)
      ok = (buf[b] = staging().take(chunk_bytes)) != nullptr &&
           cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) fail(MIMO_ECUDA);
    int b = 0;
    for (size_t i; ok && err.load() == MIMO_OK && (i = next.fetch_add(1)) < chunks.size(); b ^= 1) {
      const Chunk& c = chunks[i];
      if (pending[b] && cudaEventSynchronize(done[b]) != cudaSuccess) {
        fail(MIMO_ECUDA);
        break;
      }
      int64_t r = -1;
      if (use_direct.load() && direct_ok(c, buf[b])) {
        r = read_full(fd_direct, buf[b], c.n, c.off);
        if (r == -EINVAL) use_direct.store(false);  // filesystem without O_DIRECT: buffered from here on
      }
      if (r < 0) r = read_full(fd_buf, buf[b], c.n, c.off);
      if (r != c.n) {
        fail(MIMO_EIO);
        break;
      }
      if (cudaMemcpyAsync(c.dst, buf[b], (size_t)c.n, cudaMemcpyHostToDevice, st) != cudaSuccess ||
          cudaEventRecord(done[b], st) != cudaSuccess) {
        fail(MIMO_ECUDA);
        break;
      }
      pending[b] = true;
    }
    if (st && cudaStreamSynchronize(st) != cudaSuccess) fail(MIMO_ECUDA);
    for (int k = 0; k < 2; ++k) {
      if (done[k]) cudaEventDestroy(done[k]);
      if (buf[k]) staging().give(buf[k], chunk_bytes);  // its copy completed: the stream was synchronised
    }
    if (st) cudaStreamDestroy(st);
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < nthreads; ++t) pool.emplace_back(worker);
  for (auto& th : pool) th.join();
  cudaEventDestroy(entry);
  close(fd_buf);
  if (fd_direct >= 0) close(fd_direct);
  return err.load();
}
