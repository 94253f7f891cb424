// KV page copy engine (offload / reload of paged KV between device byte
// buffers and one pinned host pool) -- the B200 counterpart of the
// reference's KvCopy (src/qwen_infra/vpp/native/kv_copy.h:10-45,
// kv_copy.cpp:62-401).
//
// A job is a list of copy runs [tensor, device offset, host offset, bytes,
// fragments, device stride, host stride]: `fragments` pieces of `bytes` each,
// strided on both sides.  Runs sharing a page gate form one unit; a store
// (device -> host) publishes its gate (flags[gate] = epoch, release) once all
// of the unit's bytes have landed, a load (host -> device) starts a unit only
// once flags[gate] == epoch (acquire).  One progress thread moves each job in
// segments of at most `segment` bytes on its own stream per direction: every
// run piece is one cudaMemcpyAsync, a strided run of whole fragments one
// cudaMemcpy2DAsync, and a segment ends with an event the thread polls.
// Jobs wait on an event recorded on the producer stream at submission.
#pragma once

#include <cuda_runtime_api.h>

#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <exception>
#include <mutex>
#include <string>
#include <thread>
#include <utility>
#include <vector>

namespace qvpp {

struct KvRun {  // one copy run after validation (contiguous runs collapsed)
  std::uint64_t tensor, device, host, bytes, fragments, device_stride, host_stride;
};

struct KvUnit {  // the runs of one page gate
  std::vector<KvRun> runs;
  std::size_t cursor = 0;
  std::uint64_t fragment = 0, offset = 0, bytes = 0, done = 0;
  std::int64_t gate = -1, epoch = 0;
};

struct KvResult {
  std::uint64_t job_id, generation, bytes, segments;
  bool cancelled;
  float device_ms;
  std::uint64_t first_issue_ns, last_done_ns;
};

// Validates rows [N, 7] (and gates [N, 2] when given) against the storage
// sizes; throws std::invalid_argument with the reason.  Contiguous strided
// runs collapse to one piece; adjacent single-piece runs of one gate merge.
std::vector<KvUnit> kv_plan_units(const std::vector<std::uint64_t>& device_bytes, std::uint64_t host_bytes,
                                  const std::int64_t* rows, std::int64_t n, const std::int64_t* gates,
                                  std::int64_t flag_count, std::uint32_t max_runs);

class KvCopyEngine {
 public:
  KvCopyEngine(int device, std::vector<std::pair<std::uint8_t*, std::uint64_t>> buffers, std::uint8_t* host,
               std::uint64_t host_bytes, std::uint64_t segment, std::uint32_t max_jobs, std::uint32_t max_runs,
               bool pitched);
  ~KvCopyEngine();
  bool submit(std::uint64_t id, std::uint64_t generation, const std::int64_t* rows, std::int64_t n, bool store,
              cudaStream_t producer, const std::int64_t* gates);
  void set_ready(std::int64_t* flags, std::int64_t n);
  bool cancel(std::uint64_t id, std::uint64_t generation);
  std::vector<KvResult> poll();
  std::vector<KvResult> snapshot();
  bool wait(const std::vector<std::uint64_t>& ids, std::uint32_t timeout_ms);
  bool drain(std::uint32_t timeout_ms);
  void close();

 private:
  struct Job {
    enum Phase { Empty, Queued, Copying, Done } phase = Empty;
    std::uint64_t id = 0, generation = 0, bytes = 0, segments = 0, issued_bytes = 0;
    std::vector<KvUnit> units;
    std::vector<std::pair<std::size_t, std::uint64_t>> issued;  // (unit, bytes) of the segment in flight
    bool store = false, cancelled = false, started = false, waited = false;
    cudaEvent_t dependency = nullptr, begin = nullptr, segment = nullptr;
    std::chrono::steady_clock::time_point admitted;
    std::uint64_t first_issue_ns = 0, last_done_ns = 0;
  };
  bool eligible(const KvUnit& u, bool store) const;
  bool advance(Job& j);
  void loop() noexcept;
  void check() const;
  void destroy_events() noexcept;

  int device_;
  std::vector<std::pair<std::uint8_t*, std::uint64_t>> buffers_;
  std::uint8_t* host_;
  std::uint64_t host_bytes_, segment_, last_id_ = 0;
  std::uint32_t max_runs_;
  bool pitched_;
  std::int64_t* flags_ = nullptr;
  std::int64_t flag_count_ = 0;
  cudaStream_t store_stream_ = nullptr, load_stream_ = nullptr;
  std::vector<Job> jobs_;
  mutable std::mutex mutex_;
  std::condition_variable work_, completed_;
  std::thread worker_;
  std::exception_ptr error_;
  bool stopping_ = false, closed_ = false;
};

}  // namespace qvpp
