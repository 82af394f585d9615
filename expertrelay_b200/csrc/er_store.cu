// er_store.cu -- the expert store's experts.bin read into host memory.
//
// Reference: store/unbuffered_io.py (read_at, :135-149) and
// store/expert_reader.py (ExpertStoreReader.read_into, :92-101). An expert is
// one record of record_size bytes at a 4096-aligned offset of experts.bin,
// loaded with exactly one read that bypasses the OS page cache, into a
// 4096-aligned buffer; offset, size and address must all be multiples of
// 4096 and a short read is an error. The reference does this with Win32
// FILE_FLAG_NO_BUFFERING only; here it is Linux O_DIRECT, with a plain
// buffered read where the filesystem refuses O_DIRECT (tmpfs, some
// overlays) -- same bytes, only the page cache differs.
//
// read_many runs several reads at once on a few threads (an NVMe drive needs
// many requests in flight to reach its bandwidth); each read still covers one
// whole record, so the "one read per expert" property holds. The destination
// is normally pinned (page-locked) host memory, from where the HBM expert
// cache copies records to the GPU.
#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <string>
#include <thread>
#include <vector>

#include "er_internal.cuh"

namespace {

constexpr uint64_t kStoreAlign = 4096;  // store/unbuffered_io.py ALIGNMENT

}  // namespace

struct er_store {
  int fd = -1;
  int direct = 0;
  uint64_t bytes = 0;
};

using er::fail;

// One pread loop of nbytes at offset: retries EINTR and partial reads, fails
// on an error or end of file before nbytes.
static int store_read_one(const er_store* s, uint64_t offset, uint64_t nbytes, void* dst) {
  if (offset % kStoreAlign || nbytes % kStoreAlign || (uintptr_t)dst % kStoreAlign)
    return fail(ER_EINVAL, "unaligned unbuffered read: offset=%llu nbytes=%llu address=%p",
                (unsigned long long)offset, (unsigned long long)nbytes, dst);
  uint64_t done = 0;
  char* out = static_cast<char*>(dst);
  while (done < nbytes) {
    const ssize_t got = pread(s->fd, out + done, nbytes - done, (off_t)(offset + done));
    if (got < 0) {
      if (errno == EINTR) continue;
      return fail(ER_EIO, "read of %llu bytes at offset %llu failed: %s", (unsigned long long)nbytes,
                  (unsigned long long)offset, strerror(errno));
    }
    if (got == 0)
      return fail(ER_EIO, "short read at offset %llu: %llu of %llu bytes", (unsigned long long)offset,
                  (unsigned long long)done, (unsigned long long)nbytes);
    done += (uint64_t)got;
  }
  return ER_OK;
}

extern "C" int er_store_open(const char* path, int flags, er_store** out) {
  if (!path || !out) return fail(ER_EINVAL, "er_store_open: null argument");
  *out = nullptr;
  int direct = (flags & ER_STORE_BUFFERED) ? 0 : 1;
  int fd = -1;
  if (direct) {
    fd = open(path, O_RDONLY | O_DIRECT | O_CLOEXEC);
    if (fd < 0 && errno == EINVAL) direct = 0;  // the filesystem has no O_DIRECT
  }
  if (!direct) fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(ER_EIO, "er_store_open(%s): %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    const int e = errno;
    close(fd);
    return fail(ER_EIO, "er_store_open(%s): fstat: %s", path, strerror(e));
  }
  er_store* s = new er_store;
  s->fd = fd;
  s->direct = direct;
  s->bytes = (uint64_t)st.st_size;
  *out = s;
  return ER_OK;
}

extern "C" int er_store_close(er_store* s) {
  if (!s) return ER_OK;
  if (s->fd >= 0) close(s->fd);
  delete s;
  return ER_OK;
}

extern "C" int er_store_info(const er_store* s, uint64_t* file_bytes, int* direct) {
  if (!s) return fail(ER_EINVAL, "er_store_info: null store");
  if (file_bytes) *file_bytes = s->bytes;
  if (direct) *direct = s->direct;
  return ER_OK;
}

extern "C" int er_store_read(er_store* s, uint64_t offset, uint64_t nbytes, void* dst) {
  if (!s || !dst) return fail(ER_EINVAL, "er_store_read: null argument");
  return store_read_one(s, offset, nbytes, dst);
}

extern "C" int er_store_read_many(er_store* s, int count, const uint64_t* offsets, uint64_t nbytes,
                                  void* const* dsts, int threads, int* failed) {
  if (failed) *failed = -1;
  if (!s || count < 0 || (count > 0 && (!offsets || !dsts)))
    return fail(ER_EINVAL, "er_store_read_many: bad arguments (count %d)", count);
  for (int i = 0; i < count; ++i)  // every read checked before any starts
    if (offsets[i] % kStoreAlign || nbytes % kStoreAlign || (uintptr_t)dsts[i] % kStoreAlign) {
      if (failed) *failed = i;
      return fail(ER_EINVAL, "unaligned unbuffered read: offset=%llu nbytes=%llu address=%p",
                  (unsigned long long)offsets[i], (unsigned long long)nbytes, dsts[i]);
    }
  if (threads < 1) threads = 1;
  if (threads > count) threads = count;
  if (threads <= 1) {
    for (int i = 0; i < count; ++i)
      if (int rc = store_read_one(s, offsets[i], nbytes, dsts[i])) {
        if (failed) *failed = i;
        return rc;
      }
    return ER_OK;
  }
  std::atomic<int> next{0};
  std::atomic<int> first_bad{-1};
  std::vector<int> status(count, ER_OK);
  std::string bad_msg;  // the failing read's message (recorded on its worker thread)
  auto worker = [&]() {
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= count || first_bad.load() >= 0) return;
      status[i] = store_read_one(s, offsets[i], nbytes, dsts[i]);
      if (status[i] != ER_OK) {
        int expect = -1;
        if (first_bad.compare_exchange_strong(expect, i)) bad_msg = er_last_error();
      }
    }
  };
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int t = 0; t < threads; ++t) pool.emplace_back(worker);
  for (auto& t : pool) t.join();
  const int bad = first_bad.load();
  if (bad >= 0) {
    if (failed) *failed = bad;
    return fail(status[bad], "er_store_read_many: read %d: %s", bad, bad_msg.c_str());
  }
  return ER_OK;
}
