// Host-side bookkeeping of stage-boundary slots (metadata only: the slots'
// device memory lives in the arenas that the Python transport allocates).
//
// A directed wire edge owns a logical ring of up to 7 message slots.  Every
// message's slot walks a small state machine.  The legal moves are one table
// (`kMoves` in slot_pool.cpp) keyed by (side of the edge, event); the event
// names what the host just did:
//
//   event            source side                 destination side
//   Produced         Reserved -> Produced        (not allowed)
//   TransferIssued   Produced -> Transferring    Reserved -> Transferring
//   ConsumerIssued   (not allowed)               Transferring -> Consuming
//   SourceReadDone   Transferring -> Free        (not allowed)
//   ConsumerDone     (not allowed)               Consuming -> Free
//   Discarded        (not allowed)               Transferring -> Free
//   Abandoned        Reserved -> Free            Reserved -> Free   (stopped rings only)
//
// A message enters the ring (Free -> Reserved) only in edge-sequence order, so
// the receive order on the peer has no holes; a stopped ring never admits
// again (a fresh epoch must be created).  Tickets carry (ring, sequence,
// generation, slot): an event that names an older generation of a reused slot
// is refused.  Protocol: src/qwen_infra/vpp/native/slot_pool.h:9-75 (states,
// ordering and generation rules of the reference's rings and leases).
//
// LeaseArena: the rank-shared physical arena (2 source or 3 destination
// slots) that tickets of several edges borrow one at a time.
#pragma once

#include <array>
#include <cstdint>
#include <optional>
#include <stdexcept>

#include "wire.h"

namespace qvpp {

enum class Role : int { Source = 0, Destination = 1 };
enum class SlotState : int { Free = 0, Reserved, Produced, Transferring, Consuming };

// Host events on a reserved slot (values are the ABI's op codes).
enum class SlotEvent : int {
  Produced = 0,
  TransferIssued = 1,
  ConsumerIssued = 2,
  SourceReadDone = 3,
  ConsumerDone = 4,
  Discarded = 5,
  Abandoned = 6,
};
constexpr int kSlotEvents = 7;
constexpr std::uint32_t kMaxSlots = 7;

struct Ticket {
  std::uint64_t ring_id = 0, sequence = 0, generation = 0;
  std::uint32_t slot_id = 0;
  bool operator==(const Ticket& o) const noexcept {
    return ring_id == o.ring_id && sequence == o.sequence && generation == o.generation && slot_id == o.slot_id;
  }
};

struct SlotError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

// Current and high-water occupancy.
struct Occupancy {
  std::uint32_t now = 0, peak = 0;
  void up() noexcept { peak = ++now > peak ? now : peak; }
  void down() noexcept { --now; }
};

class LeaseArena {
 public:
  explicit LeaseArena(std::uint32_t capacity);
  bool available() const noexcept { return busy_mask_ != full_mask_; }
  std::uint32_t acquire(const Ticket&);
  void release(std::uint32_t physical, const Ticket&);
  void note_stall() noexcept { ++stalls_; }
  std::uint32_t live() const noexcept { return use_.now; }
  std::uint32_t peak_live() const noexcept { return use_.peak; }
  std::uint64_t stalls() const noexcept { return stalls_; }

 private:
  std::uint32_t capacity_, full_mask_, busy_mask_ = 0;
  Occupancy use_;
  std::uint64_t stalls_ = 0;
  std::array<Ticket, kMaxSlots> holder_{};
};

class SlotRing {
 public:
  SlotRing(Role, Layout, std::uint64_t epoch, std::uint32_t src_stage);
  SlotRing(const SlotRing&) = delete;
  SlotRing& operator=(const SlotRing&) = delete;

  // Reserve the slot of the next message; empty when that slot is still busy.
  std::optional<Ticket> try_acquire(const Boundary&);
  const Boundary& descriptor(const Ticket&) const;
  SlotState state(const Ticket&) const;
  void apply(const Ticket&, SlotEvent);
  void stop() noexcept { stopped_ = true; }

  std::uint32_t live() const noexcept { return use_.now; }
  std::uint32_t peak_live() const noexcept { return use_.peak; }
  std::uint64_t next_sequence() const noexcept { return expected_; }

 private:
  struct Record {
    Boundary desc{};
    SlotState state = SlotState::Free;
  };
  Record& locate(const Ticket&);
  const Record& locate(const Ticket& t) const { return const_cast<SlotRing*>(this)->locate(t); }

  Role side_;
  Layout layout_;
  std::uint64_t epoch_, ring_id_, expected_ = 0;
  std::uint32_t src_stage_;
  bool stopped_ = false;
  Occupancy use_;
  std::array<Record, kMaxSlots> slots_{};
};

}  // namespace qvpp
