/*
 * C ABI of the stage-boundary transport (host C++ over the CUDA runtime).
 * Returns 0 on success, a negative code on failure (qv_last_error() has the
 * message); waits return -2 on deadline and -3 when the peer flagged failure.
 *
 * Interfaces replaced (paths inside the reference project):
 *   qv_make/encode/decode/match_boundary, qv_rank_boundary_budget, qv_edge_index
 *       <- src/qwen_infra/vpp/native/interface.h:40-55 (boundary/check_boundary,
 *          bindings.cpp), generalised from 8 stages on 4 ranks to 2G on G
 *   qv_ring_*   <- SlotPool            (native/slot_pool.h:36-75)
 *   qv_leases_* <- PhysicalSlotLeases  (native/slot_pool.h:18-32)
 *   qv_ctrl_*   <- DmaEdge control page READY/ACK words (native/dma_edge.cpp:21-46),
 *                  here credits (grant) and publication for a peer-to-peer copy
 *   qv_copy_message <- DmaEdge D2H/H2D segment copies (native/dma_edge.cpp:135-194),
 *                  here one device-to-device copy per plane segment over NVLink
 *   qv_kvcopy_*  <- KvCopy (native/kv_copy.h:10-45, kv_copy.cpp:62-401): KV page
 *                  offload / reload between device byte buffers and a pinned host
 *                  pool, one cudaMemcpyAsync (or cudaMemcpy2DAsync for a strided
 *                  run of whole fragments) per piece instead of batched copies
 */
#ifndef QWEN_VPP_NATIVE_H
#define QWEN_VPP_NATIVE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct QvBoundary {
  uint64_t epoch;
  int64_t batch_id;
  uint64_t edge_sequence, generation;
  uint32_t src_stage, dst_stage, slot_id, valid_tokens;
  uint64_t hidden_offset, hidden_bytes, residual_offset, residual_bytes;
} QvBoundary;

typedef struct QvTicket {
  uint64_t ring_id, sequence, generation;
  uint32_t slot_id;
} QvTicket;

const char* qv_last_error(void);

int qv_make_boundary(uint32_t capacity, uint32_t slots, uint32_t ranks, uint32_t hidden, uint64_t epoch,
                     int64_t batch, uint64_t sequence, uint32_t src_stage, uint32_t rows, QvBoundary* out);
int qv_encode_boundary(uint32_t capacity, uint32_t slots, uint32_t ranks, uint32_t hidden, const QvBoundary* d,
                       uint8_t wire[96]);
int qv_decode_boundary(uint32_t capacity, uint32_t slots, uint32_t ranks, uint32_t hidden, const uint8_t wire[96],
                       QvBoundary* out);
int qv_match_boundary(uint32_t capacity, uint32_t slots, uint32_t ranks, uint32_t hidden, const uint8_t wire[96],
                      uint64_t epoch, int64_t batch, uint64_t sequence, uint32_t src_stage, QvBoundary* out);
int qv_rank_boundary_budget(uint32_t capacity, uint32_t slots, uint32_t ranks, uint32_t hidden, uint64_t* out);
int qv_edge_index(uint32_t ranks, uint32_t src_stage, uint32_t dst_stage);

/* role: 0 source, 1 destination.  try_acquire: 1 acquired, 0 busy, -1 error.
 * transition op: 0 producer_recorded, 1 transfer_recorded, 2 consumer_recorded,
 * 3 source_read_complete, 4 consumer_complete, 5 discard_received,
 * 6 release_unsubmitted (only after qv_ring_stop). */
void* qv_ring_create(int role, uint32_t capacity, uint32_t slots, uint32_t ranks, uint32_t hidden, uint64_t epoch,
                     uint32_t src_stage);
void qv_ring_destroy(void* ring);
int qv_ring_try_acquire(void* ring, const QvBoundary* d, QvTicket* out);
int qv_ring_transition(void* ring, const QvTicket* t, int op);
int qv_ring_state(void* ring, const QvTicket* t);
int qv_ring_descriptor(void* ring, const QvTicket* t, QvBoundary* out);
void qv_ring_stop(void* ring);
uint32_t qv_ring_live(void* ring);
uint32_t qv_ring_peak_live(void* ring);
uint64_t qv_ring_next_sequence(void* ring);

void* qv_leases_create(uint32_t slots);
void qv_leases_destroy(void* leases);
int qv_leases_available(void* leases);
int qv_leases_acquire(void* leases, const QvTicket* t);
int qv_leases_release(void* leases, uint32_t physical, const QvTicket* t);
void qv_leases_note_stall(void* leases);
uint32_t qv_leases_live(void* leases);
uint32_t qv_leases_peak_live(void* leases);
uint64_t qv_leases_stalls(void* leases);

/* Control page of one directed edge (POSIX shared memory, created by the receiver). */
void* qv_ctrl_create(const char* name);
void* qv_ctrl_open(const char* name, double timeout_s);
void qv_ctrl_close(void* page);
int qv_ctrl_grant(void* page, uint64_t sequence, uint32_t physical_slot);
int qv_ctrl_wait_grant(void* page, uint64_t sequence, double timeout_s, uint32_t* physical_slot);
int qv_ctrl_publish(void* page, uint64_t sequence, const uint8_t wire[96]);
int qv_ctrl_wait_published(void* page, uint64_t sequence, double timeout_s, uint8_t wire_out[96]);
int qv_ctrl_peek_published(void* page, uint64_t* count);
void qv_ctrl_fail(void* page);
int qv_ctrl_failed(void* page);

/* Device memory and events shared between rank processes (CUDA IPC); the
 * device index is made current first.  Returns cudaError_t values. */
int qv_arena_alloc(int device, uint64_t bytes, void** ptr, uint8_t handle[64]);
int qv_arena_free(int device, void* ptr);
int qv_arena_open(int device, const uint8_t handle[64], void** ptr);
int qv_arena_close(int device, void* ptr);
int qv_ipc_event_create(int device, void** event, uint8_t handle[64]);
int qv_ipc_event_open(int device, const uint8_t handle[64], void** event);
int qv_event_destroy(int device, void* event);
int qv_event_query(void* event); /* 0 complete, 1 pending, else a cudaError_t */

/* Enqueue residual then hidden plane copies (segments of `segment_bytes`) on
 * `stream` after their ready events; record `ipc_done` and `local_done`.
 * Returns a cudaError_t value. */
int qv_copy_message(int device, void* stream, void* residual_ready, void* hidden_ready, const void* src_hidden,
                    const void* src_residual, void* dst_hidden, void* dst_residual, uint64_t plane_bytes,
                    uint64_t segment_bytes, void* ipc_done, void* local_done);
int qv_stream_wait_event(int device, void* stream, void* event);

/* ---- KV page copy engine ---------------------------------------------------
 * Copy runs are int64 rows [tensor, device offset, host offset, bytes,
 * fragments, device stride, host stride]; gates (optional) int64 rows [flag
 * index, epoch > 0]: a store publishes flags[gate] = epoch (release) when all
 * of its gate's bytes landed on the host, a load starts a gate's runs once
 * flags[gate] == epoch (acquire).  segment_bytes 4, 8 or 16 MiB; 1..8 jobs;
 * runs per job (and copy calls per segment) <= max_runs <= 2^20.  The host
 * pool must be pinned.  Errors: NULL, -1 (invalid arguments, nothing done)
 * or -4 (engine failure: CUDA error, job deadline, closed; terminal), with
 * qv_kvcopy_last_error(). */
typedef struct QvKvCopyResult {
  uint64_t job_id, generation, bytes, segments;
  int32_t cancelled;
  float device_ms;
  uint64_t first_issue_ns, last_done_ns;
} QvKvCopyResult;

const char* qv_kvcopy_last_error(void);
void* qv_kvcopy_create(int device, void* const* buffers, const uint64_t* buffer_bytes, int count, void* host,
                       uint64_t host_bytes, uint64_t segment_bytes, uint32_t max_jobs, uint32_t max_runs, int pitched);
void qv_kvcopy_destroy(void* engine);
/* 1 admitted, 0 every job slot busy (poll, then retry), -1 invalid. ids increase. */
int qv_kvcopy_submit(void* engine, uint64_t id, uint64_t generation, const int64_t* runs, int64_t count, int store,
                     void* producer_stream, const int64_t* gates);
int qv_kvcopy_set_ready(void* engine, int64_t* flags, int64_t count);
int qv_kvcopy_cancel(void* engine, uint64_t id, uint64_t generation); /* 1 found, 0 not */
/* Finished jobs (harvested) / live jobs (not harvested): returns the count,
 * writes at most cap results. */
int qv_kvcopy_poll(void* engine, QvKvCopyResult* out, int cap);
int qv_kvcopy_snapshot(void* engine, QvKvCopyResult* out, int cap);
int qv_kvcopy_wait(void* engine, const uint64_t* ids, int count, uint32_t timeout_ms); /* 0, -2 deadline */
int qv_kvcopy_drain(void* engine, uint32_t timeout_ms);                             /* 0, -2 deadline */
int qv_kvcopy_close(void* engine);
/* Host-only validation of a job's runs (no device use): units (gates), pieces
 * after collapsing contiguous runs, and bytes. */
int qv_kvcopy_plan(const uint64_t* buffer_bytes, int count, uint64_t host_bytes, const int64_t* runs, int64_t rows,
                   const int64_t* gates, int64_t flag_count, uint32_t max_runs, int64_t* units_out,
                   int64_t* pieces_out, uint64_t* bytes_out);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_VPP_NATIVE_H */
