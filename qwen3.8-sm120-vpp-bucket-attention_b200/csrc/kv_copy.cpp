// KV page copy engine: see kv_copy.h.  C ABI at the end (qv_kvcopy_*).
#include "kv_copy.h"

#include <algorithm>
#include <stdexcept>
#include <unordered_map>

namespace qvpp {
namespace {

std::uint64_t now_ns() {
  return (std::uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

bool event_done(cudaEvent_t e) {
  const cudaError_t s = cudaEventQuery(e);
  if (s == cudaErrorNotReady) return false;
  cuda_check(s, "KV copy event");
  return true;
}

constexpr auto kJobDeadline = std::chrono::seconds(120);

}  // namespace

std::vector<KvUnit> kv_plan_units(const std::vector<std::uint64_t>& device_bytes, std::uint64_t host_bytes,
                                  const std::int64_t* rows, std::int64_t n, const std::int64_t* gates,
                                  std::int64_t flag_count, std::uint32_t max_runs) {
  if (!rows || n < 1 || (std::uint64_t)n > max_runs) throw std::invalid_argument("expected 1..max_runs copy runs");
  std::vector<KvUnit> units;
  std::unordered_map<std::int64_t, std::size_t> by_gate;
  for (std::int64_t i = 0; i < n; ++i) {
    const std::int64_t* r = rows + 7 * i;
    if (r[0] < 0 || (std::uint64_t)r[0] >= device_bytes.size() || r[1] < 0 || r[2] < 0 || r[3] <= 0 || r[4] <= 0 ||
        r[5] < 0 || r[6] < 0)
      throw std::invalid_argument("invalid copy run (tensor index, offsets, bytes, fragments or strides)");
    const std::uint64_t dev_total = device_bytes[(std::size_t)r[0]];
    const std::uint64_t off = (std::uint64_t)r[1], hoff = (std::uint64_t)r[2], bytes = (std::uint64_t)r[3];
    if (off > dev_total || bytes > dev_total - off || hoff > host_bytes || bytes > host_bytes - hoff)
      throw std::invalid_argument("copy run escapes its device buffer or the host pool");
    const std::uint64_t frags = (std::uint64_t)r[4], ds = (std::uint64_t)r[5], hs = (std::uint64_t)r[6];
    if (frags > 1 && (ds < bytes || hs < bytes || frags - 1 > (dev_total - off - bytes) / ds ||
                      frags - 1 > (host_bytes - hoff - bytes) / hs))
      throw std::invalid_argument("copy run strides or fragment count escape the device buffer or the host pool");
    KvRun run{(std::uint64_t)r[0], off, hoff, bytes, frags, ds, hs};
    if (frags > 1 && ds == bytes && hs == bytes) {  // contiguous on both sides: one piece
      run.bytes *= frags;
      run.fragments = 1;
    }
    const std::int64_t gate = gates ? gates[2 * i] : -1, epoch = gates ? gates[2 * i + 1] : 0;
    if (gates && (gate < 0 || gate >= flag_count || epoch <= 0))
      throw std::invalid_argument("invalid page gate or epoch");
    auto found = by_gate.emplace(gate, units.size());
    if (found.second) {
      units.emplace_back();
      units.back().gate = gate;
      units.back().epoch = epoch;
    }
    KvUnit& u = units[found.first->second];
    if (u.epoch != epoch) throw std::invalid_argument("one page gate cannot mix epochs");
    u.bytes += run.bytes * run.fragments;
    if (run.fragments == 1 && !u.runs.empty()) {
      KvRun& last = u.runs.back();
      if (last.fragments == 1 && last.tensor == run.tensor && last.device + last.bytes == run.device &&
          last.host + last.bytes == run.host) {
        last.bytes += run.bytes;
        continue;
      }
    }
    u.runs.push_back(run);
  }
  return units;
}

KvCopyEngine::KvCopyEngine(int device, std::vector<std::pair<std::uint8_t*, std::uint64_t>> buffers,
                           std::uint8_t* host, std::uint64_t host_bytes, std::uint64_t segment,
                           std::uint32_t max_jobs, std::uint32_t max_runs, bool pitched)
    : device_(device),
      buffers_(std::move(buffers)),
      host_(host),
      host_bytes_(host_bytes),
      segment_(segment),
      max_runs_(max_runs),
      pitched_(pitched),
      jobs_(max_jobs) {
  if (!(segment == (4ull << 20) || segment == (8ull << 20) || segment == (16ull << 20)) || max_jobs < 1 ||
      max_jobs > 8 || max_runs < 1 || max_runs > (1u << 20))
    throw std::invalid_argument("segment must be 4, 8 or 16 MiB, 1..8 jobs, 1..2^20 runs per job");
  if (buffers_.empty() || buffers_.size() > 64 || !host_ || !host_bytes_)
    throw std::invalid_argument("expected 1..64 device buffers and a host pool");
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  for (const auto& b : buffers_) {
    cudaPointerAttributes at{};
    cuda_check(cudaPointerGetAttributes(&at, b.first), "device buffer attributes");
    if (at.type != cudaMemoryTypeDevice || at.device != device_)
      throw std::invalid_argument("device buffers must live on the engine's device");
  }
  cudaPointerAttributes at{};
  cuda_check(cudaPointerGetAttributes(&at, host_), "host pool attributes");
  if (at.type != cudaMemoryTypeHost) throw std::invalid_argument("the host pool must be pinned (no pageable copies)");
  try {
    cuda_check(cudaStreamCreateWithFlags(&store_stream_, cudaStreamNonBlocking), "store stream");
    cuda_check(cudaStreamCreateWithFlags(&load_stream_, cudaStreamNonBlocking), "load stream");
    for (auto& j : jobs_) {
      cuda_check(cudaEventCreateWithFlags(&j.dependency, cudaEventDisableTiming), "event");
      cuda_check(cudaEventCreate(&j.begin), "event");
      cuda_check(cudaEventCreate(&j.segment), "event");
    }
    worker_ = std::thread([this] { loop(); });
  } catch (...) {
    destroy_events();
    throw;
  }
}

void KvCopyEngine::check() const {
  if (error_) std::rethrow_exception(error_);
  if (closed_ || stopping_) throw std::runtime_error("KV copy engine is closed");
}

bool KvCopyEngine::eligible(const KvUnit& u, bool store) const {
  if (u.cursor >= u.runs.size()) return false;
  if (store || u.gate < 0) return true;
  return __atomic_load_n(flags_ + u.gate, __ATOMIC_ACQUIRE) == u.epoch;
}

// One step of a job; true when it made progress.  Caller holds the mutex.
bool KvCopyEngine::advance(Job& j) {
  if (std::chrono::steady_clock::now() - j.admitted > kJobDeadline)
    throw std::runtime_error("KV copy job deadline expired");
  if (j.phase == Job::Copying) {
    if (!event_done(j.segment)) return false;
    j.bytes += j.issued_bytes;
    ++j.segments;
    j.phase = Job::Queued;
    j.last_done_ns = now_ns();
    for (const auto& is : j.issued) {
      KvUnit& u = j.units[is.first];
      u.done += is.second;
      if (u.done > u.bytes) throw std::runtime_error("KV copy unit completion overflow");
      if (j.store && u.gate >= 0 && u.done == u.bytes)
        __atomic_store_n(flags_ + u.gate, u.epoch, __ATOMIC_RELEASE);
    }
  }
  if (j.phase != Job::Queued) return false;
  // Cancellation stops what was not issued; copies in flight always finish.
  if (j.cancelled ||
      std::all_of(j.units.begin(), j.units.end(), [](const KvUnit& u) { return u.cursor == u.runs.size(); })) {
    j.phase = Job::Done;
    completed_.notify_all();
    return true;
  }
  if (!std::any_of(j.units.begin(), j.units.end(), [&](const KvUnit& u) { return eligible(u, j.store); }))
    return false;
  const cudaStream_t stream = j.store ? store_stream_ : load_stream_;
  if (!j.waited) {  // the producer's work before submission precedes every copy
    cuda_check(cudaStreamWaitEvent(stream, j.dependency, 0), "wait producer event");
    j.waited = true;
  }
  if (!j.started) {
    cuda_check(cudaEventRecord(j.begin, stream), "record begin");
    j.started = true;
    j.first_issue_ns = now_ns();
  }
  j.issued.clear();
  std::uint64_t budget = segment_;
  std::uint32_t calls = 0;
  const cudaMemcpyKind kind = j.store ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
  while (budget && calls < max_runs_) {
    // Ready pages may pass a unit still waiting for its gate.
    auto found = std::find_if(j.units.begin(), j.units.end(), [&](const KvUnit& u) { return eligible(u, j.store); });
    if (found == j.units.end()) break;
    KvUnit& u = *found;
    const std::size_t index = (std::size_t)(found - j.units.begin());
    const KvRun& run = u.runs[u.cursor];
    const std::uint64_t width = std::min(budget, run.bytes - u.offset);
    const std::uint64_t nrows =
        (pitched_ && u.offset == 0 && budget >= run.bytes) ? std::min(run.fragments - u.fragment, budget / run.bytes)
                                                           : 1;
    std::uint8_t* dev = buffers_[run.tensor].first + run.device + u.fragment * run.device_stride + u.offset;
    std::uint8_t* hst = host_ + run.host + u.fragment * run.host_stride + u.offset;
    void* dst = j.store ? (void*)hst : (void*)dev;
    const void* src = j.store ? (const void*)dev : (const void*)hst;
    if (nrows > 1) {
      const std::uint64_t dpitch = j.store ? run.host_stride : run.device_stride;
      const std::uint64_t spitch = j.store ? run.device_stride : run.host_stride;
      cuda_check(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, nrows, kind, stream), "strided copy");
    } else {
      cuda_check(cudaMemcpyAsync(dst, src, width, kind, stream), "copy");
    }
    ++calls;
    const std::uint64_t bytes = width * nrows;
    if (!j.issued.empty() && j.issued.back().first == index) j.issued.back().second += bytes;
    else j.issued.emplace_back(index, bytes);
    u.offset += width;
    budget -= bytes;
    if (u.offset == run.bytes) {
      u.fragment += nrows;
      u.offset = 0;
      if (u.fragment == run.fragments) {
        ++u.cursor;
        u.fragment = 0;
      }
    }
  }
  cuda_check(cudaEventRecord(j.segment, stream), "record segment");
  j.issued_bytes = segment_ - budget;
  j.phase = Job::Copying;
  return true;
}

void KvCopyEngine::loop() noexcept {
  try {
    cuda_check(cudaSetDevice(device_), "cudaSetDevice");
    std::unique_lock<std::mutex> lock(mutex_);
    for (;;) {
      if (stopping_) break;
      bool pending = false, progressed = false;
      for (auto& j : jobs_)
        if (j.phase == Job::Queued || j.phase == Job::Copying) {
          pending = true;
          progressed = advance(j) || progressed;
        }
      if (!progressed) {
        if (pending) {
          work_.wait_for(lock, std::chrono::microseconds(50));
        } else {
          work_.wait(lock, [&] {
            return stopping_ || std::any_of(jobs_.begin(), jobs_.end(), [](const Job& j) {
                     return j.phase == Job::Queued || j.phase == Job::Copying;
                   });
          });
        }
      }
    }
  } catch (...) {
    std::lock_guard<std::mutex> lock(mutex_);
    error_ = std::current_exception();
    stopping_ = true;
    completed_.notify_all();
    work_.notify_all();
  }
}

bool KvCopyEngine::submit(std::uint64_t id, std::uint64_t generation, const std::int64_t* rows, std::int64_t n,
                          bool store, cudaStream_t producer, const std::int64_t* gates) {
  std::lock_guard<std::mutex> lock(mutex_);
  check();
  if (id <= last_id_) throw std::invalid_argument("KV copy ids must increase; a retired job cannot be resubmitted");
  if (gates && !flags_) throw std::invalid_argument("page gates need set_ready() first");
  auto free_job = std::find_if(jobs_.begin(), jobs_.end(), [](const Job& j) { return j.phase == Job::Empty; });
  if (free_job == jobs_.end()) return false;  // bounded: the caller retries after poll()
  std::vector<std::uint64_t> sizes;
  for (const auto& b : buffers_) sizes.push_back(b.second);
  std::vector<KvUnit> units = kv_plan_units(sizes, host_bytes_, rows, n, gates, flag_count_, max_runs_);
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  Job& j = *free_job;
  cuda_check(cudaEventRecord(j.dependency, producer), "record producer event");
  j.id = id;
  j.generation = generation;
  j.store = store;
  j.units = std::move(units);
  j.bytes = j.segments = j.issued_bytes = 0;
  j.first_issue_ns = j.last_done_ns = 0;
  j.cancelled = j.started = j.waited = false;
  j.issued.clear();
  j.admitted = std::chrono::steady_clock::now();
  j.phase = Job::Queued;
  last_id_ = id;
  work_.notify_one();
  return true;
}

void KvCopyEngine::set_ready(std::int64_t* flags, std::int64_t n) {
  std::lock_guard<std::mutex> lock(mutex_);
  check();
  if (flags_ || last_id_ || !flags || n < 1 || n > 64 * 4096 || (reinterpret_cast<std::uintptr_t>(flags) & 7))
    throw std::invalid_argument("ready flags: bounded, aligned, attached once before the first submission");
  flags_ = flags;
  flag_count_ = n;
}

bool KvCopyEngine::cancel(std::uint64_t id, std::uint64_t generation) {
  std::lock_guard<std::mutex> lock(mutex_);
  check();
  for (auto& j : jobs_)
    if (j.phase != Job::Empty && j.id == id && j.generation == generation) {
      if (j.phase != Job::Done) j.cancelled = true;
      work_.notify_one();
      return true;
    }
  return false;
}

std::vector<KvResult> KvCopyEngine::poll() {
  std::lock_guard<std::mutex> lock(mutex_);
  check();
  std::vector<KvResult> out;
  for (auto& j : jobs_)
    if (j.phase == Job::Done) {
      float ms = 0.0f;
      if (j.started && j.segments) cuda_check(cudaEventElapsedTime(&ms, j.begin, j.segment), "elapsed");
      out.push_back({j.id, j.generation, j.bytes, j.segments, j.cancelled, ms, j.first_issue_ns, j.last_done_ns});
      j.phase = Job::Empty;
      j.units.clear();
      j.issued.clear();
    }
  return out;
}

std::vector<KvResult> KvCopyEngine::snapshot() {
  std::lock_guard<std::mutex> lock(mutex_);
  check();
  std::vector<KvResult> out;
  for (const auto& j : jobs_)
    if (j.phase != Job::Empty)
      out.push_back({j.id, j.generation, j.bytes, j.segments, j.cancelled, 0.0f, j.first_issue_ns, j.last_done_ns});
  return out;
}

bool KvCopyEngine::wait(const std::vector<std::uint64_t>& ids, std::uint32_t timeout_ms) {
  if (!timeout_ms || timeout_ms > 120000) throw std::invalid_argument("wait timeout must be 1..120000 ms");
  std::unique_lock<std::mutex> lock(mutex_);
  check();
  const bool done = completed_.wait_for(lock, std::chrono::milliseconds(timeout_ms), [&] {
    return error_ || std::all_of(ids.begin(), ids.end(), [&](std::uint64_t id) {
             return std::none_of(jobs_.begin(), jobs_.end(), [&](const Job& j) {
               return j.id == id && (j.phase == Job::Queued || j.phase == Job::Copying);
             });
           });
  });
  check();
  return done;
}

bool KvCopyEngine::drain(std::uint32_t timeout_ms) {
  if (!timeout_ms || timeout_ms > 120000) throw std::invalid_argument("drain timeout must be 1..120000 ms");
  std::unique_lock<std::mutex> lock(mutex_);
  check();
  const bool done = completed_.wait_for(lock, std::chrono::milliseconds(timeout_ms), [&] {
    return error_ || std::all_of(jobs_.begin(), jobs_.end(),
                                 [](const Job& j) { return j.phase == Job::Empty || j.phase == Job::Done; });
  });
  check();
  return done;
}

void KvCopyEngine::close() {
  {
    std::lock_guard<std::mutex> lock(mutex_);
    check();
    if (!std::all_of(jobs_.begin(), jobs_.end(), [](const Job& j) { return j.phase == Job::Empty; }))
      throw std::runtime_error("drain and poll every KV copy job before close");
    stopping_ = true;
  }
  work_.notify_all();
  if (worker_.joinable()) worker_.join();
  destroy_events();
  closed_ = true;
}

void KvCopyEngine::destroy_events() noexcept {
  cudaSetDevice(device_);
  for (auto& j : jobs_)
    for (cudaEvent_t* e : {&j.dependency, &j.begin, &j.segment})
      if (*e) {
        cudaEventDestroy(*e);
        *e = nullptr;
      }
  for (cudaStream_t* s : {&store_stream_, &load_stream_})
    if (*s) {
      cudaStreamDestroy(*s);
      *s = nullptr;
    }
}

KvCopyEngine::~KvCopyEngine() {
  if (closed_) return;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    stopping_ = true;
  }
  work_.notify_all();
  if (worker_.joinable()) worker_.join();
  // Copies may still reference the pools: let them finish before the streams go.
  for (cudaStream_t s : {store_stream_, load_stream_})
    if (s) cudaStreamSynchronize(s);
  destroy_events();
}

}  // namespace qvpp

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
#include <cstring>

namespace {
thread_local std::string g_kv_error;

// -1: invalid arguments (nothing happened); -4: engine failure (terminal:
// CUDA error, job deadline, use after close).
int kv_fail(const std::exception& e) {
  g_kv_error = e.what();
  return dynamic_cast<const std::invalid_argument*>(&e) ? -1 : -4;
}

struct QvKvCopyResultC {
  std::uint64_t job_id, generation, bytes, segments;
  std::int32_t cancelled;
  float device_ms;
  std::uint64_t first_issue_ns, last_done_ns;
};

int fill(const std::vector<qvpp::KvResult>& r, QvKvCopyResultC* out, int cap) {
  const int n = (int)std::min<std::size_t>(r.size(), (std::size_t)std::max(cap, 0));
  for (int i = 0; i < n; ++i)
    out[i] = {r[i].job_id, r[i].generation, r[i].bytes, r[i].segments, r[i].cancelled ? 1 : 0, r[i].device_ms,
              r[i].first_issue_ns, r[i].last_done_ns};
  return (int)r.size();
}
}  // namespace

extern "C" {

const char* qv_kvcopy_last_error(void) { return g_kv_error.c_str(); }

void* qv_kvcopy_create(int device, void* const* buffers, const std::uint64_t* buffer_bytes, int count, void* host,
                       std::uint64_t host_bytes, std::uint64_t segment_bytes, std::uint32_t max_jobs,
                       std::uint32_t max_runs, int pitched) {
  try {
    if (!buffers || !buffer_bytes || count < 1) throw std::invalid_argument("expected device buffers");
    std::vector<std::pair<std::uint8_t*, std::uint64_t>> b;
    for (int i = 0; i < count; ++i) b.emplace_back(static_cast<std::uint8_t*>(buffers[i]), buffer_bytes[i]);
    return new qvpp::KvCopyEngine(device, std::move(b), static_cast<std::uint8_t*>(host), host_bytes, segment_bytes,
                                  max_jobs, max_runs, pitched != 0);
  } catch (const std::exception& e) {
    kv_fail(e);
    return nullptr;
  }
}

void qv_kvcopy_destroy(void* engine) { delete static_cast<qvpp::KvCopyEngine*>(engine); }

int qv_kvcopy_submit(void* engine, std::uint64_t id, std::uint64_t generation, const std::int64_t* runs,
                     std::int64_t count, int store, void* producer_stream, const std::int64_t* gates) {
  try {
    return static_cast<qvpp::KvCopyEngine*>(engine)->submit(id, generation, runs, count, store != 0,
                                                            static_cast<cudaStream_t>(producer_stream), gates)
               ? 1
               : 0;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_set_ready(void* engine, std::int64_t* flags, std::int64_t count) {
  try {
    static_cast<qvpp::KvCopyEngine*>(engine)->set_ready(flags, count);
    return 0;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_cancel(void* engine, std::uint64_t id, std::uint64_t generation) {
  try {
    return static_cast<qvpp::KvCopyEngine*>(engine)->cancel(id, generation) ? 1 : 0;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_poll(void* engine, QvKvCopyResultC* out, int cap) {
  try {
    return fill(static_cast<qvpp::KvCopyEngine*>(engine)->poll(), out, cap);
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_snapshot(void* engine, QvKvCopyResultC* out, int cap) {
  try {
    return fill(static_cast<qvpp::KvCopyEngine*>(engine)->snapshot(), out, cap);
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_wait(void* engine, const std::uint64_t* ids, int count, std::uint32_t timeout_ms) {
  try {
    std::vector<std::uint64_t> v(ids, ids + std::max(count, 0));
    return static_cast<qvpp::KvCopyEngine*>(engine)->wait(v, timeout_ms) ? 0 : -2;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_drain(void* engine, std::uint32_t timeout_ms) {
  try {
    return static_cast<qvpp::KvCopyEngine*>(engine)->drain(timeout_ms) ? 0 : -2;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_close(void* engine) {
  try {
    static_cast<qvpp::KvCopyEngine*>(engine)->close();
    return 0;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

int qv_kvcopy_plan(const std::uint64_t* buffer_bytes, int count, std::uint64_t host_bytes, const std::int64_t* runs,
                   std::int64_t rows, const std::int64_t* gates, std::int64_t flag_count, std::uint32_t max_runs,
                   std::int64_t* units_out, std::int64_t* pieces_out, std::uint64_t* bytes_out) {
  try {
    std::vector<std::uint64_t> sizes(buffer_bytes, buffer_bytes + std::max(count, 0));
    const auto units = qvpp::kv_plan_units(sizes, host_bytes, runs, rows, gates, flag_count, max_runs);
    std::int64_t pieces = 0;
    std::uint64_t bytes = 0;
    for (const auto& u : units) {
      pieces += (std::int64_t)u.runs.size();
      bytes += u.bytes;
    }
    if (units_out) *units_out = (std::int64_t)units.size();
    if (pieces_out) *pieces_out = pieces;
    if (bytes_out) *bytes_out = bytes;
    return 0;
  } catch (const std::exception& e) {
    return kv_fail(e);
  }
}

}  // extern "C"
