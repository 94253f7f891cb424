// Boundary slot bookkeeping (host metadata only; no memory is allocated here).
//
// SlotRing: one directed edge's logical ring of `slot_count` message slots.
// Each message walks Free -> Reserved -> Produced -> Transferring -> Consuming
// -> Free (source side skips Consuming, destination side skips Produced);
// tickets carry (ring id, sequence, generation, slot), so a completion that
// names an older generation of a reused slot is rejected.  A ring never
// resumes after stop(): a skipped sequence would leave a hole in the peer's
// receive order.  Semantics follow src/qwen_infra/vpp/native/slot_pool.cpp.
//
// PhysicalLeases: the rank-shared physical arena (2 source or 3 destination
// slots) that logical tickets of several edges lease one at a time.
#pragma once

#include <array>
#include <cstdint>
#include <optional>
#include <stdexcept>

#include "wire.h"

namespace qvpp {

enum class Role : int { Source = 0, Destination = 1 };
enum class SlotState : int { Free = 0, Reserved, Produced, Transferring, Consuming };

struct Ticket {
  std::uint64_t ring_id = 0, sequence = 0, generation = 0;
  std::uint32_t slot_id = 0;
};

struct SlotError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

class PhysicalLeases {
 public:
  explicit PhysicalLeases(std::uint32_t slots);
  bool available() const noexcept { return live_ < slots_; }
  std::uint32_t acquire(const Ticket&);
  void release(std::uint32_t physical, const Ticket&);
  void note_stall() noexcept { ++stalls_; }
  std::uint32_t live() const noexcept { return live_; }
  std::uint32_t peak_live() const noexcept { return peak_; }
  std::uint64_t stalls() const noexcept { return stalls_; }

 private:
  std::uint32_t slots_, live_ = 0, peak_ = 0;
  std::uint64_t stalls_ = 0;
  std::array<std::optional<Ticket>, 7> owner_{};
};

class SlotRing {
 public:
  SlotRing(Role, Layout, std::uint64_t epoch, std::uint32_t src_stage);
  SlotRing(const SlotRing&) = delete;
  SlotRing& operator=(const SlotRing&) = delete;

  std::optional<Ticket> try_acquire(const Boundary&);
  const Boundary& descriptor(const Ticket&) const;
  SlotState state(const Ticket&) const;

  void producer_recorded(const Ticket&);     // source: Reserved -> Produced
  void transfer_recorded(const Ticket&);     // source: Produced -> Transferring; destination: Reserved -> Transferring
  void consumer_recorded(const Ticket&);     // destination: Transferring -> Consuming
  void source_read_complete(const Ticket&);  // source: Transferring -> Free
  void consumer_complete(const Ticket&);     // destination: Consuming -> Free
  void discard_received(const Ticket&);      // destination: Transferring -> Free
  void stop() noexcept { stopped_ = true; }
  void release_unsubmitted(const Ticket&);   // after stop(): Reserved -> Free

  std::uint32_t live() const noexcept { return live_; }
  std::uint32_t peak_live() const noexcept { return peak_; }
  std::uint64_t next_sequence() const noexcept { return next_; }

 private:
  struct Entry {
    Boundary desc{};
    SlotState state = SlotState::Free;
  };
  const Entry& entry(const Ticket&) const;
  void move(const Ticket&, Role required, SlotState from, SlotState to);

  Role role_;
  Layout layout_;
  std::uint64_t epoch_, id_, next_ = 0;
  std::uint32_t src_stage_, live_ = 0, peak_ = 0;
  bool stopped_ = false;
  std::array<Entry, 7> entries_{};
};

}  // namespace qvpp
