#include "slot_pool.h"

#include <algorithm>
#include <atomic>

namespace qvpp {
namespace {

std::atomic<std::uint64_t> g_next_ring{1};

void need(bool ok, const char* what) {
  if (!ok) throw SlotError(what);
}

bool same_ticket(const Ticket& a, const Ticket& b) {
  return a.ring_id == b.ring_id && a.sequence == b.sequence && a.generation == b.generation &&
         a.slot_id == b.slot_id;
}

}  // namespace

PhysicalLeases::PhysicalLeases(std::uint32_t slots) : slots_(slots) {
  need(slots >= 1 && slots <= owner_.size(), "invalid physical arena capacity");
}

std::uint32_t PhysicalLeases::acquire(const Ticket& t) {
  need(available(), "physical arena has no free lease");
  for (const auto& o : owner_)
    need(!o || o->ring_id != t.ring_id || o->slot_id != t.slot_id, "logical ticket already has a physical lease");
  for (std::uint32_t i = 0; i < slots_; ++i) {
    if (!owner_[i]) {
      owner_[i] = t;
      ++live_;
      peak_ = std::max(peak_, live_);
      return i;
    }
  }
  throw std::logic_error("physical lease accounting mismatch");
}

void PhysicalLeases::release(std::uint32_t physical, const Ticket& t) {
  need(physical < slots_, "physical lease outside arena");
  need(owner_[physical].has_value() && same_ticket(*owner_[physical], t),
       "physical lease completion belongs to another ticket/generation");
  owner_[physical].reset();
  --live_;
}

SlotRing::SlotRing(Role role, Layout layout, std::uint64_t epoch, std::uint32_t src_stage)
    : role_(role), layout_(layout), epoch_(epoch), id_(g_next_ring.fetch_add(1)), src_stage_(src_stage) {
  make_boundary(layout_, epoch_, 0, 0, src_stage_, 0);  // validates epoch, edge and layout
  need(role == Role::Source || role == Role::Destination, "invalid pool role");
}

std::optional<Ticket> SlotRing::try_acquire(const Boundary& d) {
  need(!stopped_, "role stopped; create a new role epoch, do not resume");
  validate_boundary(layout_, d);
  need(d.epoch == epoch_ && d.src_stage == src_stage_, "wrong role epoch or edge");
  need(d.edge_sequence == next_, "out-of-order boundary admission");
  Entry& e = entries_[d.slot_id];
  if (e.state != SlotState::Free) return std::nullopt;
  e.desc = d;
  e.state = SlotState::Reserved;
  ++next_;
  ++live_;
  peak_ = std::max(peak_, live_);
  return Ticket{id_, d.edge_sequence, d.generation, d.slot_id};
}

const SlotRing::Entry& SlotRing::entry(const Ticket& t) const {
  need(t.ring_id == id_ && t.slot_id < layout_.slot_count, "ticket belongs to another pool");
  const Entry& e = entries_[t.slot_id];
  need(e.state != SlotState::Free && e.desc.edge_sequence == t.sequence && e.desc.generation == t.generation,
       "stale completion or retired ticket");
  return e;
}

const Boundary& SlotRing::descriptor(const Ticket& t) const { return entry(t).desc; }
SlotState SlotRing::state(const Ticket& t) const { return entry(t).state; }

void SlotRing::move(const Ticket& t, Role required, SlotState from, SlotState to) {
  need(role_ == required && entry(t).state == from, "invalid slot transition");
  entries_[t.slot_id].state = to;
  if (to == SlotState::Free) --live_;
}

void SlotRing::producer_recorded(const Ticket& t) { move(t, Role::Source, SlotState::Reserved, SlotState::Produced); }
void SlotRing::transfer_recorded(const Ticket& t) {
  move(t, role_, role_ == Role::Source ? SlotState::Produced : SlotState::Reserved, SlotState::Transferring);
}
void SlotRing::consumer_recorded(const Ticket& t) {
  move(t, Role::Destination, SlotState::Transferring, SlotState::Consuming);
}
void SlotRing::source_read_complete(const Ticket& t) {
  move(t, Role::Source, SlotState::Transferring, SlotState::Free);
}
void SlotRing::consumer_complete(const Ticket& t) {
  move(t, Role::Destination, SlotState::Consuming, SlotState::Free);
}
void SlotRing::discard_received(const Ticket& t) {
  move(t, Role::Destination, SlotState::Transferring, SlotState::Free);
}
void SlotRing::release_unsubmitted(const Ticket& t) {
  need(stopped_, "unsent sequence can only be abandoned at fatal role shutdown");
  move(t, role_, SlotState::Reserved, SlotState::Free);
}

}  // namespace qvpp
