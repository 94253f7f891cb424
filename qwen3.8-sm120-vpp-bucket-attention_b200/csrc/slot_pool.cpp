#include "slot_pool.h"

#include <atomic>

namespace qvpp {
namespace {

std::atomic<std::uint64_t> g_ring_ids{1};

[[noreturn]] void refuse(const char* why) { throw SlotError(why); }

// One legal move: the state the slot must be in, the state it goes to, and
// whether the ring must have been stopped first.
struct Move {
  bool allowed;
  SlotState from, to;
  bool only_when_stopped;
};
constexpr Move kNone{false, SlotState::Free, SlotState::Free, false};
constexpr Move mv(SlotState from, SlotState to, bool stopped = false) { return Move{true, from, to, stopped}; }

// kMoves[event][side]: side 0 = source, 1 = destination.
constexpr Move kMoves[kSlotEvents][2] = {
    /* Produced       */ {mv(SlotState::Reserved, SlotState::Produced), kNone},
    /* TransferIssued */ {mv(SlotState::Produced, SlotState::Transferring),
                          mv(SlotState::Reserved, SlotState::Transferring)},
    /* ConsumerIssued */ {kNone, mv(SlotState::Transferring, SlotState::Consuming)},
    /* SourceReadDone */ {mv(SlotState::Transferring, SlotState::Free), kNone},
    /* ConsumerDone   */ {kNone, mv(SlotState::Consuming, SlotState::Free)},
    /* Discarded      */ {kNone, mv(SlotState::Transferring, SlotState::Free)},
    /* Abandoned      */ {mv(SlotState::Reserved, SlotState::Free, true),
                          mv(SlotState::Reserved, SlotState::Free, true)},
};

}  // namespace

// ---- LeaseArena -------------------------------------------------------------

LeaseArena::LeaseArena(std::uint32_t capacity)
    : capacity_(capacity), full_mask_(capacity >= 1 && capacity <= kMaxSlots ? (1u << capacity) - 1u : 0u) {
  if (capacity < 1 || capacity > kMaxSlots) refuse("a lease arena holds 1 to 7 physical slots");
}

std::uint32_t LeaseArena::acquire(const Ticket& t) {
  if (!available()) refuse("every physical slot of the arena is leased");
  for (std::uint32_t bits = busy_mask_; bits; bits &= bits - 1) {
    const Ticket& h = holder_[__builtin_ctz(bits)];
    if (h.ring_id == t.ring_id && h.slot_id == t.slot_id) refuse("this logical slot already holds a physical lease");
  }
  const std::uint32_t physical = __builtin_ctz(~busy_mask_);  // lowest free slot
  busy_mask_ |= 1u << physical;
  holder_[physical] = t;
  use_.up();
  return physical;
}

void LeaseArena::release(std::uint32_t physical, const Ticket& t) {
  if (physical >= capacity_) refuse("physical slot index past the arena");
  if (!(busy_mask_ >> physical & 1u) || !(holder_[physical] == t))
    refuse("lease returned by a ticket that does not hold it");
  busy_mask_ &= ~(1u << physical);
  use_.down();
}

// ---- SlotRing ---------------------------------------------------------------

SlotRing::SlotRing(Role side, Layout layout, std::uint64_t epoch, std::uint32_t src_stage)
    : side_(side), layout_(layout), epoch_(epoch), ring_id_(g_ring_ids.fetch_add(1)), src_stage_(src_stage) {
  if (side != Role::Source && side != Role::Destination) refuse("ring side must be source or destination");
  make_boundary(layout_, epoch_, 0, 0, src_stage_, 0);  // checks the layout, epoch and edge
}

std::optional<Ticket> SlotRing::try_acquire(const Boundary& d) {
  if (stopped_) refuse("ring was stopped; a new epoch needs a new ring");
  validate_boundary(layout_, d);
  if (d.epoch != epoch_ || d.src_stage != src_stage_) refuse("message belongs to another epoch or edge");
  if (d.edge_sequence != expected_) refuse("message admitted out of edge-sequence order");
  Record& r = slots_[d.slot_id];
  if (r.state != SlotState::Free) return std::nullopt;
  r.desc = d;
  r.state = SlotState::Reserved;
  ++expected_;
  use_.up();
  return Ticket{ring_id_, d.edge_sequence, d.generation, d.slot_id};
}

SlotRing::Record& SlotRing::locate(const Ticket& t) {
  if (t.ring_id != ring_id_ || t.slot_id >= layout_.slot_count) refuse("ticket was issued by another ring");
  Record& r = slots_[t.slot_id];
  if (r.state == SlotState::Free || r.desc.edge_sequence != t.sequence || r.desc.generation != t.generation)
    refuse("ticket no longer names a live message (retired or older generation)");
  return r;
}

const Boundary& SlotRing::descriptor(const Ticket& t) const { return locate(t).desc; }
SlotState SlotRing::state(const Ticket& t) const { return locate(t).state; }

void SlotRing::apply(const Ticket& t, SlotEvent ev) {
  const int e = static_cast<int>(ev);
  if (e < 0 || e >= kSlotEvents) refuse("unknown slot event");
  const Move& m = kMoves[e][side_ == Role::Source ? 0 : 1];
  if (!m.allowed) refuse("event does not apply to this side of the edge");
  if (m.only_when_stopped && !stopped_) refuse("a reserved message may be abandoned only after the ring stopped");
  Record& r = locate(t);
  if (r.state != m.from) refuse("event does not apply in the slot's current state");
  r.state = m.to;
  if (m.to == SlotState::Free) use_.down();
}

}  // namespace qvpp
