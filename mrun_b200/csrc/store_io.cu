// On-disk store reading: byte ranges of QStore files (weights.i8, scales.f32, extras.f32) and
// expert page files straight into caller memory (normally pinned host buffers that feed
// host->device copies).
//
// The reference reads these files through numpy memory maps: every first touch is a 4 KiB
// page fault, the mapped pages count toward the process's resident memory until they are
// dropped, and one copy thread tops out near 17 GB/s (engine/kernels/qstore.py:622-660 moves
// to three numpy copy threads; engine/qwen3_moe_cuda.py:925-951 switches the bulk warm-up
// to unbuffered reads for the RSS reason). Here a range is split into chunks read by
// parallel pread(2) calls on one file descriptor: no mapping, no fault per page, and the
// kernel's page cache and read-ahead stay in play. Optional posix_fadvise calls announce
// the next predicted range (WILLNEED) and drop the pages of a range once it has been read
// (DONTNEED), as the reference's _drop_mmap_pages does for its mappings.
//
// Host code only: no device memory is touched here.
#include "common.cuh"

#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <thread>
#include <vector>

namespace mrb {

struct StoreFile {
  int fd;
  uint64_t size;
};

constexpr uint64_t SIO_CHUNK = 4ull << 20;  // bytes per read call
constexpr int SIO_MAX_THREADS = 64;

// Read [off, off + n) into dst; 0 on success, else the errno (EIO for an early end of file).
static int pread_full(int fd, uint64_t off, uint64_t n, unsigned char* dst) {
  while (n > 0) {
    const size_t want = (size_t)std::min<uint64_t>(n, SIO_CHUNK);
    const ssize_t got = pread(fd, dst, want, (off_t)off);
    if (got < 0) {
      if (errno == EINTR) continue;
      return errno;
    }
    if (got == 0) return EIO;
    dst += got;
    off += (uint64_t)got;
    n -= (uint64_t)got;
  }
  return 0;
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_store_file_open(const char* path, void** handle, uint64_t* size) {
  if (!path || !handle || !size) return fail(MRB_ERR_ARG, "store_file_open: null pointer");
  *handle = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(MRB_ERR_IO, "store_file_open: %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    const int e = errno;
    close(fd);
    return fail(MRB_ERR_IO, "store_file_open: %s: %s", path, strerror(e));
  }
  if (!S_ISREG(st.st_mode)) {
    close(fd);
    return fail(MRB_ERR_ARG, "store_file_open: %s is not a regular file", path);
  }
  StoreFile* f = new StoreFile{fd, (uint64_t)st.st_size};
  *handle = f;
  *size = f->size;
  clear_error();
  return MRB_OK;
}

extern "C" int mrb_store_file_close(void* handle) {
  if (!handle) return MRB_OK;
  StoreFile* f = static_cast<StoreFile*>(handle);
  const int rc = close(f->fd);
  delete f;
  if (rc != 0) return fail(MRB_ERR_IO, "store_file_close: %s", strerror(errno));
  return MRB_OK;
}

extern "C" int mrb_store_file_read(void* handle, uint64_t offset, uint64_t bytes, void* dst, int threads,
                                   int drop_after) {
  if (!handle) return fail(MRB_ERR_ARG, "store_file_read: null handle");
  StoreFile* f = static_cast<StoreFile*>(handle);
  if (bytes == 0) return MRB_OK;
  if (!dst) return fail(MRB_ERR_ARG, "store_file_read: null destination");
  if (offset > f->size || bytes > f->size - offset)
    return fail(MRB_ERR_ARG, "store_file_read: range [%llu, %llu) beyond the file's %llu bytes",
                (unsigned long long)offset, (unsigned long long)(offset + bytes), (unsigned long long)f->size);
  // pieces of at least two chunks per thread; the first thread is the caller
  const uint64_t pieces = (bytes + 2 * SIO_CHUNK - 1) / (2 * SIO_CHUNK);
  const int nt = (int)std::max<uint64_t>(1, std::min<uint64_t>(pieces, (uint64_t)std::clamp(threads, 1, SIO_MAX_THREADS)));
  unsigned char* out = static_cast<unsigned char*>(dst);
  int err = 0;
  if (nt == 1) {
    err = pread_full(f->fd, offset, bytes, out);
  } else {
    // equal contiguous shares, split on chunk boundaries
    const uint64_t share = ((bytes / nt + SIO_CHUNK - 1) / SIO_CHUNK) * SIO_CHUNK;
    std::vector<int> errs(nt, 0);
    std::vector<std::thread> pool;
    pool.reserve(nt - 1);
    for (int t = 1; t < nt; ++t) {
      const uint64_t lo = std::min(bytes, share * t), hi = std::min(bytes, share * (t + 1));
      if (lo >= hi) break;
      pool.emplace_back([&, t, lo, hi]() { errs[t] = pread_full(f->fd, offset + lo, hi - lo, out + lo); });
    }
    errs[0] = pread_full(f->fd, offset, std::min(bytes, share), out);
    for (auto& th : pool) th.join();
    for (int e : errs)
      if (e) err = e;
  }
  if (err) return fail(MRB_ERR_IO, "store_file_read: %s", strerror(err));
  if (drop_after) posix_fadvise(f->fd, (off_t)offset, (off_t)bytes, POSIX_FADV_DONTNEED);
  clear_error();
  return MRB_OK;
}

extern "C" int mrb_store_file_advise(void* handle, uint64_t offset, uint64_t bytes, int will_need) {
  if (!handle) return fail(MRB_ERR_ARG, "store_file_advise: null handle");
  StoreFile* f = static_cast<StoreFile*>(handle);
  if (bytes == 0 || offset >= f->size) return MRB_OK;
  bytes = std::min(bytes, f->size - offset);
  const int rc = posix_fadvise(f->fd, (off_t)offset, (off_t)bytes, will_need ? POSIX_FADV_WILLNEED : POSIX_FADV_DONTNEED);
  if (rc != 0) return fail(MRB_ERR_IO, "store_file_advise: %s", strerror(rc));
  return MRB_OK;
}
