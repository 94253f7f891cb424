// Stage-boundary wire header and the folded edge topology for G ranks.
//
// A boundary message moves the dual-bf16 planes (hidden, residual) of one
// chunk from virtual stage s to stage s+1 on another rank.  Its 96-byte
// little-endian header keeps the reference's field layout and validation
// rules (src/qwen_infra/vpp/native/interface.cpp:74-169): magic "VPP1",
// version 1, kind 1 (dual bf16), slot = sequence % ring slots, generation =
// sequence / ring slots + 1, planes [0, rows*H*2) and [plane bytes, +rows*H*2).
// The edge set is generalised from the fixed 8 stages / 4 ranks to 2G / G.
#pragma once

#include <array>
#include <cstdint>
#include <stdexcept>
#include <vector>

namespace qvpp {

struct Span {
  std::uint64_t offset_bytes = 0;
  std::uint64_t valid_bytes = 0;
};

struct Boundary {
  std::uint64_t epoch = 0;
  std::int64_t batch_id = 0;  // negative ids are allowed (warm-up batches)
  std::uint64_t edge_sequence = 0;
  std::uint64_t generation = 0;
  std::uint32_t src_stage = 0, dst_stage = 0, slot_id = 0, valid_tokens = 0;
  Span hidden, residual;
};

struct Topology {
  std::uint32_t ranks = 4;
  std::uint32_t stages() const { return 2 * ranks; }
  std::uint32_t stage_rank(std::uint32_t stage) const;
  bool is_wire_edge(std::uint32_t src, std::uint32_t dst) const;
  std::uint32_t edge_index(std::uint32_t src, std::uint32_t dst) const;  // 0 .. 2G-3
  std::vector<std::uint32_t> source_stages() const;
};

struct Layout {
  std::uint32_t token_capacity = 0;  // rows per plane (<= 16384)
  std::uint32_t slot_count = 0;      // ring slots of one edge (1 .. 7)
  std::uint32_t hidden = 5120;
  Topology topo;
  void validate() const;
  std::uint64_t plane_bytes() const { return std::uint64_t(token_capacity) * hidden * 2; }
  std::uint64_t slot_bytes() const { return 2 * plane_bytes(); }
};

using Wire = std::array<std::uint8_t, 96>;

struct WireError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

Boundary make_boundary(const Layout&, std::uint64_t epoch, std::int64_t batch, std::uint64_t sequence,
                       std::uint32_t src_stage, std::uint32_t rows);
void validate_boundary(const Layout&, const Boundary&);
Wire encode_boundary(const Layout&, const Boundary&);
Boundary decode_boundary(const Layout&, const Wire&);
Boundary match_boundary(const Layout&, const Wire&, std::uint64_t epoch, std::int64_t batch,
                        std::uint64_t sequence, std::uint32_t src_stage);
// Bytes of all edge rings touching each rank (source + destination families).
std::vector<std::uint64_t> rank_boundary_budget(const Layout&);

}  // namespace qvpp
