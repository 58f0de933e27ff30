// NCCL profiler plugin: records the host-side start and stop of every collective and
// point-to-point operation into a per-process shared-memory ring that the fail-slow detector
// reads (detect/nccl_profile_reader.py).  Loaded through NCCL's official plugin interface:
//
//   NCCL_PROFILER_PLUGIN=/path/libresihp_nccl_profiler.so
//   RESIHP_NCCL_PROF_DIR=/dev/shm      (ring file: resihp_nccl_<pid>.ring)
//
// Ring layout (little endian): header {u32 magic "RESH", u32 version, u32 capacity,
// u32 record_size, u64 head}; then `capacity` records {u64 start_ns, u64 end_ns, u64 comm_id,
// u64 count, i32 rank, i32 nranks, i32 type, i32 peer, char func[24], u64 seq}.  A writer
// claims slot `head++`, fills it, then publishes seq = index + 1 (release); a reader accepts a
// record only when seq matches.  Profiling problems never fail the job: init degrades to a
// zero activation mask.
#include <fcntl.h>
#include <sys/mman.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "nccl_profiler_abi.h"

namespace {

constexpr uint32_t kMagic = 0x52455348u;  // "RESH"
constexpr uint32_t kVersion = 1;
constexpr uint32_t kCapacity = 65536;
constexpr int kFuncLen = 24;

struct Record {
  uint64_t start_ns;
  uint64_t end_ns;
  uint64_t comm_id;
  uint64_t count;
  int32_t rank;
  int32_t nranks;
  int32_t type;
  int32_t peer;
  char func[kFuncLen];
  std::atomic<uint64_t> seq;
};

struct Header {
  uint32_t magic;
  uint32_t version;
  uint32_t capacity;
  uint32_t record_size;
  std::atomic<uint64_t> head;
};

static_assert(sizeof(Record) == 4 * 8 + 4 * 4 + kFuncLen + 8, "record layout");
static_assert(sizeof(Header) == 4 * 4 + 8, "header layout");

struct Comm {
  uint64_t id;
  int rank;
  int nranks;
};

struct Event {
  const Comm* comm;
  uint64_t start_ns;
  uint64_t count;
  int type;
  int peer;
  char func[kFuncLen];
};

class Ring {
 public:
  bool acquire() {
    std::lock_guard<std::mutex> g(mu_);
    if (header_ == nullptr && !open()) return false;
    ++refs_;
    return true;
  }

  void release() {
    std::lock_guard<std::mutex> g(mu_);
    if (refs_ > 0 && --refs_ == 0 && header_ != nullptr) {
      munmap(header_, bytes_);
      header_ = nullptr;
      records_ = nullptr;
    }
  }

  void write(const Event& ev, uint64_t end_ns) {
    Header* h = header_;
    if (h == nullptr) return;
    const uint64_t idx = h->head.fetch_add(1, std::memory_order_acq_rel);
    Record& r = records_[idx % kCapacity];
    r.seq.store(0, std::memory_order_relaxed);
    std::atomic_thread_fence(std::memory_order_release);
    r.start_ns = ev.start_ns;
    r.end_ns = end_ns;
    r.comm_id = ev.comm->id;
    r.count = ev.count;
    r.rank = ev.comm->rank;
    r.nranks = ev.comm->nranks;
    r.type = ev.type;
    r.peer = ev.peer;
    std::memcpy(r.func, ev.func, kFuncLen);
    r.seq.store(idx + 1, std::memory_order_release);
  }

 private:
  bool open() {
    const char* dir = std::getenv("RESIHP_NCCL_PROF_DIR");
    char path[1024];
    std::snprintf(path, sizeof(path), "%s/resihp_nccl_%d.ring", dir ? dir : "/dev/shm", static_cast<int>(getpid()));
    bytes_ = sizeof(Header) + static_cast<size_t>(kCapacity) * sizeof(Record);
    const int fd = ::open(path, O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return false;
    if (ftruncate(fd, static_cast<off_t>(bytes_)) != 0) {
      close(fd);
      return false;
    }
    void* p = mmap(nullptr, bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return false;
    std::memset(p, 0, bytes_);
    header_ = static_cast<Header*>(p);
    records_ = reinterpret_cast<Record*>(static_cast<char*>(p) + sizeof(Header));
    header_->version = kVersion;
    header_->capacity = kCapacity;
    header_->record_size = sizeof(Record);
    header_->head.store(0, std::memory_order_relaxed);
    std::atomic_thread_fence(std::memory_order_release);
    header_->magic = kMagic;  // published last: a reader that sees the magic sees a valid header
    return true;
  }

  std::mutex mu_;
  Header* header_ = nullptr;
  Record* records_ = nullptr;
  size_t bytes_ = 0;
  int refs_ = 0;
};

Ring g_ring;

uint64_t monotonic_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}

void copy_name(char (&dst)[kFuncLen], const char* src) {
  std::strncpy(dst, src ? src : "?", kFuncLen - 1);
  dst[kFuncLen - 1] = '\0';
}

ncclResult_t plugin_init(void** context, uint64_t commId, int* mask, const char*, int, int nranks, int rank,
                         ncclDebugLogger_t) {
  *context = nullptr;
  *mask = 0;
  if (!g_ring.acquire()) return ncclSuccess;  // no ring: profile nothing, never fail the job
  Comm* c = new (std::nothrow) Comm{commId, rank, nranks};
  if (c == nullptr) {
    g_ring.release();
    return ncclSystemError;
  }
  *context = c;
  *mask = ncclProfileColl | ncclProfileP2p;
  return ncclSuccess;
}

ncclResult_t plugin_start(void* context, void** handle, ncclProfilerEventDescr_v5_t* d) {
  *handle = nullptr;
  if (context == nullptr || d == nullptr) return ncclSuccess;
  if (d->type != static_cast<uint64_t>(ncclProfileColl) && d->type != static_cast<uint64_t>(ncclProfileP2p))
    return ncclSuccess;
  Event* ev = new (std::nothrow) Event();
  if (ev == nullptr) return ncclSuccess;
  ev->comm = static_cast<const Comm*>(context);
  ev->type = static_cast<int>(d->type);
  if (d->type == static_cast<uint64_t>(ncclProfileColl)) {
    copy_name(ev->func, d->coll.func);
    ev->count = d->coll.count;
    ev->peer = -1;
  } else {
    copy_name(ev->func, d->p2p.func);
    ev->count = d->p2p.count;
    ev->peer = d->p2p.peer;
  }
  ev->start_ns = monotonic_ns();
  *handle = ev;
  return ncclSuccess;
}

ncclResult_t plugin_stop(void* handle) {
  Event* ev = static_cast<Event*>(handle);
  if (ev == nullptr) return ncclSuccess;
  g_ring.write(*ev, monotonic_ns());
  delete ev;
  return ncclSuccess;
}

ncclResult_t plugin_state(void*, ncclProfilerEventState_v5_t, ncclProfilerEventStateArgs_v5_t*) {
  return ncclSuccess;
}

ncclResult_t plugin_finalize(void* context) {
  if (context != nullptr) {
    delete static_cast<Comm*>(context);
    g_ring.release();
  }
  return ncclSuccess;
}

}  // namespace

extern "C" {
__attribute__((visibility("default"))) ncclProfiler_v5_t ncclProfiler_v5 = {
    "resihp", plugin_init, plugin_start, plugin_stop, plugin_state, plugin_finalize,
};
}
