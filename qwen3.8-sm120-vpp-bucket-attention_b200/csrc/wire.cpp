#include "wire.h"

#include <cstring>
#include <limits>

namespace qvpp {
namespace {

constexpr std::uint32_t kMagic = 0x31505056u;  // bytes "VPP1"
constexpr std::uint16_t kVersion = 1;
constexpr std::uint16_t kKindDualBf16 = 1;

void check(bool ok, const char* what) {
  if (!ok) throw WireError(what);
}

void store_le(Wire& w, std::size_t at, std::uint64_t v, unsigned n) {
  for (unsigned i = 0; i < n; ++i) w[at + i] = std::uint8_t((v >> (8 * i)) & 0xFFu);
}

std::uint64_t load_le(const Wire& w, std::size_t at, unsigned n) {
  std::uint64_t v = 0;
  for (unsigned i = 0; i < n; ++i) v |= std::uint64_t(w[at + i]) << (8 * i);
  return v;
}

}  // namespace

std::uint32_t Topology::stage_rank(std::uint32_t stage) const {
  check(ranks >= 1 && stage < stages(), "virtual stage index outside 0 .. 2G-1");
  return stage < ranks ? stage : stages() - 1 - stage;
}

bool Topology::is_wire_edge(std::uint32_t src, std::uint32_t dst) const {
  return ranks >= 2 && dst == src + 1 && dst < stages() && src != ranks - 1;
}

std::vector<std::uint32_t> Topology::source_stages() const {
  std::vector<std::uint32_t> out;
  for (std::uint32_t s = 0; s + 1 < stages(); ++s)
    if (is_wire_edge(s, s + 1)) out.push_back(s);
  return out;
}

std::uint32_t Topology::edge_index(std::uint32_t src, std::uint32_t dst) const {
  check(is_wire_edge(src, dst), "stage pair is not a wire edge of the folded layout");
  return src < ranks ? src : src - 1;
}

void Layout::validate() const {
  check(token_capacity > 0 && token_capacity <= 16384, "slot token capacity must be 1 .. 16384");
  check(slot_count > 0 && slot_count <= 7, "ring must hold 1 to 7 slots");
  check(hidden > 0 && hidden % 8 == 0, "hidden size must be a positive multiple of 8");
  check(topo.ranks >= 2 && topo.ranks <= 64, "rank count must be 2 .. 64");
}

void validate_boundary(const Layout& layout, const Boundary& d) {
  layout.validate();
  layout.topo.edge_index(d.src_stage, d.dst_stage);
  check(d.epoch != 0, "epoch 0 is reserved");
  check(d.edge_sequence != std::numeric_limits<std::uint64_t>::max(),
        "edge sequence would overflow; start a new epoch (sequences never wrap)");
  check(d.slot_id == d.edge_sequence % layout.slot_count, "slot id is not sequence mod ring size");
  check(d.generation == d.edge_sequence / layout.slot_count + 1, "generation is not sequence / ring size + 1");
  check(d.valid_tokens <= layout.token_capacity, "valid tokens exceed the slot capacity");
  const std::uint64_t bytes = std::uint64_t(d.valid_tokens) * layout.hidden * 2;
  check(d.hidden.offset_bytes == 0 && d.hidden.valid_bytes == bytes, "hidden plane span does not match the layout");
  check(d.residual.offset_bytes == layout.plane_bytes() && d.residual.valid_bytes == bytes, "residual plane span does not match the layout");
}

Boundary make_boundary(const Layout& layout, std::uint64_t epoch, std::int64_t batch, std::uint64_t sequence,
                       std::uint32_t src, std::uint32_t rows) {
  layout.validate();
  Boundary d;
  d.epoch = epoch;
  d.batch_id = batch;
  d.edge_sequence = sequence;
  d.generation = sequence / layout.slot_count + 1;
  d.src_stage = src;
  d.dst_stage = src + 1;
  d.slot_id = std::uint32_t(sequence % layout.slot_count);
  d.valid_tokens = rows;
  const std::uint64_t bytes = std::uint64_t(rows) * layout.hidden * 2;
  d.hidden = {0, bytes};
  d.residual = {layout.plane_bytes(), bytes};
  validate_boundary(layout, d);
  return d;
}

Wire encode_boundary(const Layout& layout, const Boundary& d) {
  validate_boundary(layout, d);
  Wire w{};
  store_le(w, 0, kMagic, 4);
  store_le(w, 4, kVersion, 2);
  store_le(w, 6, kKindDualBf16, 2);
  store_le(w, 8, d.epoch, 8);
  std::uint64_t batch_bits;
  std::memcpy(&batch_bits, &d.batch_id, 8);
  store_le(w, 16, batch_bits, 8);
  store_le(w, 24, d.edge_sequence, 8);
  store_le(w, 32, d.generation, 8);
  store_le(w, 40, d.src_stage, 4);
  store_le(w, 44, d.dst_stage, 4);
  store_le(w, 48, d.slot_id, 4);
  store_le(w, 52, d.valid_tokens, 4);
  store_le(w, 56, d.hidden.offset_bytes, 8);
  store_le(w, 64, d.hidden.valid_bytes, 8);
  store_le(w, 72, d.residual.offset_bytes, 8);
  store_le(w, 80, d.residual.valid_bytes, 8);
  // bytes 88..95 stay zero (reserved)
  return w;
}

Boundary decode_boundary(const Layout& layout, const Wire& w) {
  check(load_le(w, 0, 4) == kMagic && load_le(w, 4, 2) == kVersion && load_le(w, 6, 2) == kKindDualBf16 &&
            load_le(w, 88, 8) == 0,
        "wire header magic, version or kind not recognised");
  Boundary d;
  d.epoch = load_le(w, 8, 8);
  const std::uint64_t bits = load_le(w, 16, 8);
  std::memcpy(&d.batch_id, &bits, 8);
  d.edge_sequence = load_le(w, 24, 8);
  d.generation = load_le(w, 32, 8);
  d.src_stage = std::uint32_t(load_le(w, 40, 4));
  d.dst_stage = std::uint32_t(load_le(w, 44, 4));
  d.slot_id = std::uint32_t(load_le(w, 48, 4));
  d.valid_tokens = std::uint32_t(load_le(w, 52, 4));
  d.hidden = {load_le(w, 56, 8), load_le(w, 64, 8)};
  d.residual = {load_le(w, 72, 8), load_le(w, 80, 8)};
  validate_boundary(layout, d);
  return d;
}

Boundary match_boundary(const Layout& layout, const Wire& w, std::uint64_t epoch, std::int64_t batch,
                        std::uint64_t sequence, std::uint32_t src) {
  Boundary d = decode_boundary(layout, w);
  check(d.epoch == epoch && d.batch_id == batch && d.edge_sequence == sequence && d.src_stage == src,
        "header names another epoch, batch, sequence or edge than expected");
  return d;
}

std::vector<std::uint64_t> rank_boundary_budget(const Layout& layout) {
  layout.validate();
  const std::uint64_t family = std::uint64_t(layout.slot_count) * layout.slot_bytes();
  std::vector<std::uint64_t> bytes(layout.topo.ranks, 0);
  for (std::uint32_t src : layout.topo.source_stages()) {
    bytes[layout.topo.stage_rank(src)] += family;
    bytes[layout.topo.stage_rank(src + 1)] += family;
  }
  return bytes;
}

}  // namespace qvpp
