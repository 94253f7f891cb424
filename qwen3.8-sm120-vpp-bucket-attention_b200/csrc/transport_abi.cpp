// C ABI of the stage-boundary transport library (declarations:
// include/qwen_vpp_native.h).  Errors: functions return 0 on success and a
// negative code otherwise; qv_last_error() gives the message of the last
// failure on this thread.
#include <cuda_runtime_api.h>

#include <cstring>
#include <exception>
#include <string>

#include "slot_pool.h"
#include "wire.h"

namespace qvpp {
struct ControlPage;
ControlPage* ctrl_create(const char* name);
ControlPage* ctrl_open(const char* name, double timeout_s);
void ctrl_close(ControlPage* page);
int ctrl_grant(ControlPage*, std::uint64_t seq, std::uint32_t physical);
int ctrl_wait_grant(ControlPage*, std::uint64_t seq, double timeout_s, std::uint32_t* physical);
int ctrl_publish(ControlPage*, std::uint64_t seq, const std::uint8_t* wire);
int ctrl_wait_published(ControlPage*, std::uint64_t seq, double timeout_s, std::uint8_t* wire_out);
int ctrl_peek_published(ControlPage*, std::uint64_t* count);
void ctrl_fail(ControlPage*);
int ctrl_failed(ControlPage*);
int copy_message(cudaStream_t, cudaEvent_t, cudaEvent_t, const void*, const void*, void*, void*, std::uint64_t,
                 std::uint64_t, cudaEvent_t, cudaEvent_t);
}  // namespace qvpp

using namespace qvpp;

namespace {
thread_local std::string g_error;

int fail(const std::exception& e) {
  g_error = e.what();
  return -1;
}

Layout make_layout(std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden) {
  Layout l;
  l.token_capacity = cap;
  l.slot_count = slots;
  l.hidden = hidden;
  l.topo.ranks = ranks;
  return l;
}

struct QvBoundaryC {
  std::uint64_t epoch;
  std::int64_t batch_id;
  std::uint64_t edge_sequence, generation;
  std::uint32_t src_stage, dst_stage, slot_id, valid_tokens;
  std::uint64_t hidden_offset, hidden_bytes, residual_offset, residual_bytes;
};

QvBoundaryC to_c(const Boundary& d) {
  return QvBoundaryC{d.epoch, d.batch_id, d.edge_sequence, d.generation, d.src_stage, d.dst_stage, d.slot_id,
                     d.valid_tokens, d.hidden.offset_bytes, d.hidden.valid_bytes, d.residual.offset_bytes,
                     d.residual.valid_bytes};
}

Boundary from_c(const QvBoundaryC& c) {
  Boundary d;
  d.epoch = c.epoch;
  d.batch_id = c.batch_id;
  d.edge_sequence = c.edge_sequence;
  d.generation = c.generation;
  d.src_stage = c.src_stage;
  d.dst_stage = c.dst_stage;
  d.slot_id = c.slot_id;
  d.valid_tokens = c.valid_tokens;
  d.hidden = {c.hidden_offset, c.hidden_bytes};
  d.residual = {c.residual_offset, c.residual_bytes};
  return d;
}

struct QvTicketC {
  std::uint64_t ring_id, sequence, generation;
  std::uint32_t slot_id;
};

Ticket ticket_from(const QvTicketC* t) { return Ticket{t->ring_id, t->sequence, t->generation, t->slot_id}; }

}  // namespace

extern "C" {

const char* qv_last_error(void) { return g_error.c_str(); }

int qv_make_boundary(std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden,
                     std::uint64_t epoch, std::int64_t batch, std::uint64_t seq, std::uint32_t src,
                     std::uint32_t rows, QvBoundaryC* out) {
  try {
    *out = to_c(make_boundary(make_layout(cap, slots, ranks, hidden), epoch, batch, seq, src, rows));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_encode_boundary(std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden,
                       const QvBoundaryC* d, std::uint8_t* wire) {
  try {
    const Wire w = encode_boundary(make_layout(cap, slots, ranks, hidden), from_c(*d));
    std::memcpy(wire, w.data(), 96);
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_decode_boundary(std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden,
                       const std::uint8_t* wire, QvBoundaryC* out) {
  try {
    Wire w;
    std::memcpy(w.data(), wire, 96);
    *out = to_c(decode_boundary(make_layout(cap, slots, ranks, hidden), w));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_match_boundary(std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden,
                      const std::uint8_t* wire, std::uint64_t epoch, std::int64_t batch, std::uint64_t seq,
                      std::uint32_t src, QvBoundaryC* out) {
  try {
    Wire w;
    std::memcpy(w.data(), wire, 96);
    *out = to_c(match_boundary(make_layout(cap, slots, ranks, hidden), w, epoch, batch, seq, src));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_rank_boundary_budget(std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden,
                            std::uint64_t* out) {
  try {
    const auto b = rank_boundary_budget(make_layout(cap, slots, ranks, hidden));
    for (std::size_t i = 0; i < b.size(); ++i) out[i] = b[i];
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_edge_index(std::uint32_t ranks, std::uint32_t src, std::uint32_t dst) {
  try {
    Topology t;
    t.ranks = ranks;
    return int(t.edge_index(src, dst));
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ---- slot rings ------------------------------------------------------------
void* qv_ring_create(int role, std::uint32_t cap, std::uint32_t slots, std::uint32_t ranks, std::uint32_t hidden,
                     std::uint64_t epoch, std::uint32_t src_stage) {
  try {
    return new SlotRing(Role(role), make_layout(cap, slots, ranks, hidden), epoch, src_stage);
  } catch (const std::exception& e) {
    fail(e);
    return nullptr;
  }
}

void qv_ring_destroy(void* r) { delete static_cast<SlotRing*>(r); }

// 1 = acquired, 0 = ring slot busy, -1 = error
int qv_ring_try_acquire(void* r, const QvBoundaryC* d, QvTicketC* out) {
  try {
    auto t = static_cast<SlotRing*>(r)->try_acquire(from_c(*d));
    if (!t) return 0;
    *out = QvTicketC{t->ring_id, t->sequence, t->generation, t->slot_id};
    return 1;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// op: a SlotEvent value (0 produced, 1 transfer issued, 2 consumer issued,
//     3 source read done, 4 consumer done, 5 discarded, 6 abandoned)
int qv_ring_transition(void* r, const QvTicketC* t, int op) {
  try {
    if (op < 0 || op >= kSlotEvents) throw SlotError("unknown slot event");
    static_cast<SlotRing*>(r)->apply(ticket_from(t), SlotEvent(op));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_ring_state(void* r, const QvTicketC* t) {
  try {
    return int(static_cast<SlotRing*>(r)->state(ticket_from(t)));
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int qv_ring_descriptor(void* r, const QvTicketC* t, QvBoundaryC* out) {
  try {
    *out = to_c(static_cast<SlotRing*>(r)->descriptor(ticket_from(t)));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

void qv_ring_stop(void* r) { static_cast<SlotRing*>(r)->stop(); }
std::uint32_t qv_ring_live(void* r) { return static_cast<SlotRing*>(r)->live(); }
std::uint32_t qv_ring_peak_live(void* r) { return static_cast<SlotRing*>(r)->peak_live(); }
std::uint64_t qv_ring_next_sequence(void* r) { return static_cast<SlotRing*>(r)->next_sequence(); }

// ---- physical leases --------------------------------------------------------
void* qv_leases_create(std::uint32_t slots) {
  try {
    return new LeaseArena(slots);
  } catch (const std::exception& e) {
    fail(e);
    return nullptr;
  }
}
void qv_leases_destroy(void* l) { delete static_cast<LeaseArena*>(l); }
int qv_leases_available(void* l) { return static_cast<LeaseArena*>(l)->available() ? 1 : 0; }
int qv_leases_acquire(void* l, const QvTicketC* t) {
  try {
    return int(static_cast<LeaseArena*>(l)->acquire(ticket_from(t)));
  } catch (const std::exception& e) {
    return fail(e);
  }
}
int qv_leases_release(void* l, std::uint32_t physical, const QvTicketC* t) {
  try {
    static_cast<LeaseArena*>(l)->release(physical, ticket_from(t));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}
void qv_leases_note_stall(void* l) { static_cast<LeaseArena*>(l)->note_stall(); }
std::uint32_t qv_leases_live(void* l) { return static_cast<LeaseArena*>(l)->live(); }
std::uint32_t qv_leases_peak_live(void* l) { return static_cast<LeaseArena*>(l)->peak_live(); }
std::uint64_t qv_leases_stalls(void* l) { return static_cast<LeaseArena*>(l)->stalls(); }

// ---- edge control pages -----------------------------------------------------
void* qv_ctrl_create(const char* name) {
  void* p = ctrl_create(name);
  if (!p) g_error = std::string("cannot create control page ") + name;
  return p;
}
void* qv_ctrl_open(const char* name, double timeout_s) {
  void* p = ctrl_open(name, timeout_s);
  if (!p) g_error = std::string("cannot open control page ") + name;
  return p;
}
void qv_ctrl_close(void* p) { ctrl_close(static_cast<ControlPage*>(p)); }
int qv_ctrl_grant(void* p, std::uint64_t seq, std::uint32_t physical) {
  return ctrl_grant(static_cast<ControlPage*>(p), seq, physical);
}
int qv_ctrl_wait_grant(void* p, std::uint64_t seq, double timeout_s, std::uint32_t* physical) {
  return ctrl_wait_grant(static_cast<ControlPage*>(p), seq, timeout_s, physical);
}
int qv_ctrl_publish(void* p, std::uint64_t seq, const std::uint8_t* wire) {
  return ctrl_publish(static_cast<ControlPage*>(p), seq, wire);
}
int qv_ctrl_wait_published(void* p, std::uint64_t seq, double timeout_s, std::uint8_t* wire_out) {
  return ctrl_wait_published(static_cast<ControlPage*>(p), seq, timeout_s, wire_out);
}
int qv_ctrl_peek_published(void* p, std::uint64_t* count) {
  return ctrl_peek_published(static_cast<ControlPage*>(p), count);
}
void qv_ctrl_fail(void* p) { ctrl_fail(static_cast<ControlPage*>(p)); }
int qv_ctrl_failed(void* p) { return ctrl_failed(static_cast<ControlPage*>(p)); }

// ---- device memory / events shared between the rank processes -------------
static int bind(int device) {
  int cur = -1;
  cudaGetDevice(&cur);
  return cur == device ? 0 : int(cudaSetDevice(device));
}

int qv_arena_alloc(int device, std::uint64_t bytes, void** ptr, std::uint8_t* handle) {
  if (int e = bind(device)) return e;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return int(e);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) return int(e);
  std::memcpy(handle, &h, sizeof(h));
  return 0;
}

int qv_arena_free(int device, void* ptr) {
  if (int e = bind(device)) return e;
  return int(cudaFree(ptr));
}

int qv_arena_open(int device, const std::uint8_t* handle, void** ptr) {
  if (int e = bind(device)) return e;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return int(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int qv_arena_close(int device, void* ptr) {
  if (int e = bind(device)) return e;
  return int(cudaIpcCloseMemHandle(ptr));
}

int qv_ipc_event_create(int device, void** event, std::uint8_t* handle) {
  if (int e = bind(device)) return e;
  cudaEvent_t ev;
  cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming | cudaEventInterprocess);
  if (e != cudaSuccess) return int(e);
  cudaIpcEventHandle_t h;
  e = cudaIpcGetEventHandle(&h, ev);
  if (e != cudaSuccess) return int(e);
  std::memcpy(handle, &h, sizeof(h));
  *event = ev;
  return 0;
}

int qv_ipc_event_open(int device, const std::uint8_t* handle, void** event) {
  if (int e = bind(device)) return e;
  cudaIpcEventHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaEvent_t ev;
  const cudaError_t e = cudaIpcOpenEventHandle(&ev, h);
  if (e == cudaSuccess) *event = ev;
  return int(e);
}

int qv_event_destroy(int device, void* event) {
  if (int e = bind(device)) return e;
  return int(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
}

// 0 = complete, 1 = still pending, otherwise a cudaError_t value
int qv_event_query(void* event) {
  const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
  if (e == cudaSuccess) return 0;
  if (e == cudaErrorNotReady) return 1;
  return int(e);
}

// ---- copy engine ------------------------------------------------------------
int qv_copy_message(int device, void* stream, void* residual_ready, void* hidden_ready, const void* src_hidden,
                    const void* src_residual, void* dst_hidden, void* dst_residual, std::uint64_t bytes,
                    std::uint64_t segment, void* ipc_done, void* local_done) {
  if (int e = bind(device)) return e;
  return copy_message(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(residual_ready),
                      static_cast<cudaEvent_t>(hidden_ready), src_hidden, src_residual, dst_hidden, dst_residual,
                      bytes, segment, static_cast<cudaEvent_t>(ipc_done), static_cast<cudaEvent_t>(local_done));
}

int qv_stream_wait_event(int device, void* stream, void* event) {
  if (int e = bind(device)) return e;
  return int(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
}

}  // extern "C"
