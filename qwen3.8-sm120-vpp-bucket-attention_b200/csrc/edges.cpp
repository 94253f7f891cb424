// Peer-to-peer copy-engine boundary edges on one node.
//
// Data path: the sender's copy stream copies a message's two planes from its
// local source slot straight into the receiver's destination slot (an IPC
// mapping of the receiver's arena) with cudaMemcpyAsync, which the copy
// engines carry over NVLink; no host staging.  Completion is signalled with an
// interprocess CUDA event recorded after the copies; the receiver's compute
// stream waits on that event, so no host thread waits for the data itself.
//
// Control path (per directed edge, a small POSIX shared-memory page owned by
// the receiver), generalising the READY/ACK words of the reference's
// segmented DMA edge (src/qwen_infra/vpp/native/dma_edge.cpp:21-46):
//   grant[seq % 8]  receiver -> sender: "destination slot p is yours for seq"
//   header[seq % 8] the 96-byte wire header of seq, written before publish
//   published       sender -> receiver: seqs [0, published) have their copies
//                   enqueued and their completion event recorded
//   failed          either side gives up; every wait checks it
// Every host wait has a deadline.
#include <cuda_runtime_api.h>
#include <fcntl.h>
#include <sched.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <string>

namespace qvpp {

constexpr std::uint64_t kCtrlMagic = 0x51565050434e5431ull;  // "QVPPCNT1"
constexpr int kRing = 8;

struct EdgeControl {
  alignas(64) std::atomic<std::uint64_t> grant[kRing];
  alignas(64) std::atomic<std::uint64_t> published;
  alignas(64) std::atomic<std::uint32_t> failed;
  alignas(64) std::uint8_t header[kRing][96];
  alignas(64) std::atomic<std::uint64_t> magic;
};

struct ControlPage {
  EdgeControl* ctrl = nullptr;
  std::string name;
  bool owner = false;
};

enum : int { kOk = 0, kErr = -1, kTimeout = -2, kFailed = -3 };

namespace {

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void backoff(unsigned& spins) {
  ++spins;
  if (spins < 64) return;
  if (spins < 256) {
    sched_yield();
    return;
  }
  timespec ts{0, spins < 4096 ? 2000 : 50000};
  nanosleep(&ts, nullptr);
}

template <class Pred>
int wait_until(EdgeControl* c, double timeout_s, Pred done) {
  const double deadline = now_s() + timeout_s;
  unsigned spins = 0;
  while (!done()) {
    if (c->failed.load(std::memory_order_acquire)) return kFailed;
    if ((spins & 63) == 0 && now_s() > deadline) return kTimeout;
    backoff(spins);
  }
  return kOk;
}

}  // namespace

ControlPage* ctrl_create(const char* name) {
  const int fd = shm_open(name, O_CREAT | O_EXCL | O_RDWR, 0600);
  if (fd < 0) return nullptr;
  if (ftruncate(fd, sizeof(EdgeControl)) != 0) {
    close(fd);
    shm_unlink(name);
    return nullptr;
  }
  void* p = mmap(nullptr, sizeof(EdgeControl), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    shm_unlink(name);
    return nullptr;
  }
  std::memset(p, 0, sizeof(EdgeControl));
  auto* page = new ControlPage{static_cast<EdgeControl*>(p), name, true};
  page->ctrl->magic.store(kCtrlMagic, std::memory_order_release);
  return page;
}

ControlPage* ctrl_open(const char* name, double timeout_s) {
  const double deadline = now_s() + timeout_s;
  unsigned spins = 0;
  int fd = -1;
  while ((fd = shm_open(name, O_RDWR, 0600)) < 0) {
    if (now_s() > deadline) return nullptr;
    spins += 4096;
    backoff(spins);
  }
  struct stat st {};
  while (fstat(fd, &st) == 0 && (std::size_t)st.st_size < sizeof(EdgeControl)) {
    if (now_s() > deadline) {
      close(fd);
      return nullptr;
    }
    backoff(spins);
  }
  void* p = mmap(nullptr, sizeof(EdgeControl), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return nullptr;
  auto* c = static_cast<EdgeControl*>(p);
  while (c->magic.load(std::memory_order_acquire) != kCtrlMagic) {
    if (now_s() > deadline) {
      munmap(p, sizeof(EdgeControl));
      return nullptr;
    }
    backoff(spins);
  }
  return new ControlPage{c, name, false};
}

void ctrl_close(ControlPage* page) {
  if (!page) return;
  munmap(page->ctrl, sizeof(EdgeControl));
  if (page->owner) shm_unlink(page->name.c_str());
  delete page;
}

int ctrl_grant(ControlPage* page, std::uint64_t seq, std::uint32_t physical) {
  if (!page || physical > 0xFF) return kErr;
  page->ctrl->grant[seq % kRing].store(((seq + 1) << 8) | physical, std::memory_order_release);
  return kOk;
}

int ctrl_wait_grant(ControlPage* page, std::uint64_t seq, double timeout_s, std::uint32_t* physical) {
  if (!page || !physical) return kErr;
  EdgeControl* c = page->ctrl;
  std::uint64_t v = 0;
  const int rc = wait_until(c, timeout_s, [&] {
    v = c->grant[seq % kRing].load(std::memory_order_acquire);
    return (v >> 8) == seq + 1;
  });
  if (rc == kOk) *physical = std::uint32_t(v & 0xFF);
  return rc;
}

int ctrl_publish(ControlPage* page, std::uint64_t seq, const std::uint8_t* wire) {
  if (!page || !wire) return kErr;
  EdgeControl* c = page->ctrl;
  if (c->published.load(std::memory_order_relaxed) != seq) return kErr;  // strictly in order
  std::memcpy(c->header[seq % kRing], wire, 96);
  c->published.store(seq + 1, std::memory_order_release);
  return kOk;
}

int ctrl_wait_published(ControlPage* page, std::uint64_t seq, double timeout_s, std::uint8_t* wire_out) {
  if (!page) return kErr;
  EdgeControl* c = page->ctrl;
  const int rc = wait_until(c, timeout_s, [&] { return c->published.load(std::memory_order_acquire) > seq; });
  if (rc == kOk && wire_out) std::memcpy(wire_out, c->header[seq % kRing], 96);
  return rc;
}

int ctrl_peek_published(ControlPage* page, std::uint64_t* count) {
  if (!page || !count) return kErr;
  *count = page->ctrl->published.load(std::memory_order_acquire);
  return kOk;
}

void ctrl_fail(ControlPage* page) {
  if (page) page->ctrl->failed.store(1, std::memory_order_release);
}

int ctrl_failed(ControlPage* page) { return page ? int(page->ctrl->failed.load(std::memory_order_acquire)) : 1; }

// Enqueue one message's copies on `stream`: the residual plane after its ready
// event, then the hidden plane after its own, each split into segments of at
// most `segment` bytes; then record the interprocess completion event and the
// local "source slot free" event.
int copy_message(cudaStream_t stream, cudaEvent_t residual_ready, cudaEvent_t hidden_ready, const void* src_hidden,
                 const void* src_residual, void* dst_hidden, void* dst_residual, std::uint64_t bytes,
                 std::uint64_t segment, cudaEvent_t ipc_done, cudaEvent_t local_done) {
  if (segment == 0) segment = bytes ? bytes : 1;
  cudaError_t e = cudaSuccess;
  const struct {
    cudaEvent_t ready;
    const void* src;
    void* dst;
  } planes[2] = {{residual_ready, src_residual, dst_residual}, {hidden_ready, src_hidden, dst_hidden}};
  for (const auto& pl : planes) {
    if (pl.ready && (e = cudaStreamWaitEvent(stream, pl.ready, 0)) != cudaSuccess) return int(e);
    for (std::uint64_t off = 0; off < bytes; off += segment) {
      const std::uint64_t n = bytes - off < segment ? bytes - off : segment;
      e = cudaMemcpyAsync(static_cast<char*>(pl.dst) + off, static_cast<const char*>(pl.src) + off, n,
                          cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return int(e);
    }
  }
  if (ipc_done && (e = cudaEventRecord(ipc_done, stream)) != cudaSuccess) return int(e);
  if (local_done && (e = cudaEventRecord(local_done, stream)) != cudaSuccess) return int(e);
  return 0;
}

}  // namespace qvpp
