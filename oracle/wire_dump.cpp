// Test-infrastructure driver: links the reference's own wire codec
// (src/qwen_infra/vpp/native/interface.cpp, compiled where it lies) and prints
// the 96-byte headers it encodes for a fixed set of descriptors as JSON, plus
// which malformed inputs it rejects.  Built into oracle/_ref/ by build_ref.py.
#include <cstdio>
#include <exception>
#include <vector>

#include "interface.h"

using namespace vpp;

static void hex(const WireBoundary& w) {
  std::printf("\"");
  for (auto b : w) std::printf("%02x", b);
  std::printf("\"");
}

int main() {
  struct Case { std::uint32_t cap, slots; std::uint64_t epoch; std::int64_t batch; std::uint64_t seq;
                std::uint32_t src, rows; };
  std::vector<Case> cases = {
      {2048, 2, 1, 12, 0, 0, 513},  {2048, 2, 1, 12, 0, 6, 513},  {2048, 7, 1, 0, 0, 1, 1024},
      {2048, 7, 3, -5, 9, 5, 17},   {16384, 7, 2, 123456789, 1000, 4, 16384}, {512, 3, 7, 0, 2, 2, 0},
      {4096, 7, 1, 63, 63, 6, 4096}};
  std::printf("{\"encoded\": [");
  for (std::size_t i = 0; i < cases.size(); ++i) {
    const auto& c = cases[i];
    BoundaryLayout layout{c.cap, c.slots};
    auto d = make_boundary(layout, c.epoch, c.batch, c.seq, c.src, c.rows);
    std::printf("%s{\"cap\": %u, \"slots\": %u, \"epoch\": %llu, \"batch\": %lld, \"seq\": %llu, \"src\": %u, "
                "\"rows\": %u, \"wire\": ",
                i ? ", " : "", c.cap, c.slots, (unsigned long long)c.epoch, (long long)c.batch,
                (unsigned long long)c.seq, c.src, c.rows);
    hex(encode_boundary(layout, d));
    std::printf("}");
  }
  // Rejections the codec must reproduce.
  struct Bad { const char* name; std::uint32_t cap, slots; std::uint64_t epoch; std::uint32_t src, rows; };
  std::vector<Bad> bad = {{"fold_edge", 2048, 7, 1, 3, 1}, {"last_stage", 2048, 7, 1, 7, 1},
                          {"zero_epoch", 2048, 7, 0, 0, 1}, {"over_capacity", 2048, 7, 1, 0, 2049},
                          {"zero_capacity", 0, 7, 1, 0, 0}, {"eight_slots", 2048, 8, 1, 0, 1}};
  std::printf("], \"rejected\": {");
  for (std::size_t i = 0; i < bad.size(); ++i) {
    bool rejected = false;
    try {
      make_boundary(BoundaryLayout{bad[i].cap, bad[i].slots}, bad[i].epoch, 0, 0, bad[i].src, bad[i].rows);
    } catch (const std::exception&) {
      rejected = true;
    }
    std::printf("%s\"%s\": %s", i ? ", " : "", bad[i].name, rejected ? "true" : "false");
  }
  auto budget = rank_boundary_budget(BoundaryLayout{2048, 7});
  std::printf("}, \"budget_2048_7\": [%llu, %llu, %llu, %llu]}\n", (unsigned long long)budget[0],
              (unsigned long long)budget[1], (unsigned long long)budget[2], (unsigned long long)budget[3]);
  return 0;
}
