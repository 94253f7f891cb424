// Paged-KV prefill attention for callers that cannot allocate device memory.
//
// The regular path (qi_kv_dequant + qi_prefill_attention) needs a caller-
// provided scratch buffer for the f16 K / V^T it reads.  Some callers cannot
// call cudaMalloc at that point: a custom allocator callback, a plugin host
// that hands out only input/output buffers, or a process whose memory budget
// is already fully reserved by its framework.  This entry point keeps that scratch in a
// fixed, statically sized device array instead, so a call allocates nothing.
//
// Cost and limits:
//   * every GPU that loads this library holds kScratchBytes (32 MiB) of device
//     memory for this array, plus the attention kernel's key-range split
//     workspace (kSplitBytes, about 21 MB), until the process exits;
//   * a call is limited to what fits in it: Hkv * tokens * D * 2 bytes of K
//     plus Hkv * D * round_up(tokens, 64) * 2 bytes of V^T (27B shape, 8 KV
//     heads x 128: up to 8192 tokens of history + chunk); larger requests are
//     rejected with cudaErrorInvalidValue before anything is launched;
//   * all calls share the one array, so calls whose work overlaps on the GPU
//     (different streams without ordering between them) race on it; order
//     them on one stream.  Nothing in the scratch array has to start at zero:
//     every byte the attention reads is written by the dequantisation of the
//     same call.  The split workspace's arrival counters must start even;
//     every call clears them first (cudaMemsetAsync, which allocates nothing).
//   * the first call on a device looks the array's device address up (with
//     that device current) and caches it.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "qwen_infra_b200.h"

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;
__device__ __align__(256) unsigned char g_attention_scratch[kScratchBytes];

// Key-range split workspace of the attention kernel (QiAttention.workspace):
// room for 80 split units of head_dim 128 (the kernel splits at most half
// the SM count; a device with more than 160 SMs gets fewer splits).  Zero at
// load, as the kernel requires; the kernel keeps its counters consistent.
constexpr size_t kSplitBytes = size_t(4096) + size_t(80) * 2 * 256 * 2 * 4 + size_t(80) * 2 * 256 * 128 * 4;
__device__ __align__(256) unsigned char g_split_workspace[kSplitBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
void* g_split_addr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device (looked up once
// per device; the host-side symbol itself is not a device address).
cudaError_t scratch_address(int device, void** out, void** split) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[device]) {
    void *ptr = nullptr, *ws = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_attention_scratch);
    if (e != cudaSuccess) return e;
    e = cudaGetSymbolAddress(&ws, g_split_workspace);
    if (e != cudaSuccess) return e;
    g_scratch_addr[device] = ptr;
    g_split_addr[device] = ws;
  }
  *out = g_scratch_addr[device];
  *split = g_split_addr[device];
  return cudaSuccess;
}

}  // namespace

extern "C" int qi_paged_prefill_attention_noalloc(const QiKvView* kv, const int32_t* block_table, const void* q,
                                                  int64_t q_row, void* out, int64_t out_row, int rows, int history,
                                                  int qheads, const float* k_global, const float* v_global,
                                                  float softmax_scale, int* status, cudaStream_t stream) {
  if (!kv || !block_table || !q || !out || rows < 1 || history < 0 || qheads < 1)
    return (int)cudaErrorInvalidValue;
  QI_BIND(stream, q);
  const int64_t tokens = (int64_t)history + rows;
  const int64_t vt_row = (tokens + 63) / 64 * 64;
  const int64_t k_bytes = (int64_t)kv->kvheads * tokens * kv->head_dim * 2;
  const int64_t k_span = (k_bytes + 255) / 256 * 256;
  const int64_t vt_bytes = (int64_t)kv->kvheads * kv->head_dim * vt_row * 2;
  if (kv->kvheads < 1 || kv->head_dim < 1 || k_span + vt_bytes > (int64_t)kScratchBytes)
    return (int)cudaErrorInvalidValue;
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return (int)e;
  if (device < 0 || device >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  void *scratch = nullptr, *split = nullptr;
  e = scratch_address(device, &scratch, &split);
  if (e != cudaSuccess) return (int)e;
  unsigned char* base = static_cast<unsigned char*>(scratch);
  QiAttention a{};
  a.q = q;
  a.k = base;
  a.vt = base + k_span;
  a.out = out;
  a.k_global = k_global;
  a.v_global = v_global;
  a.status = status;
  a.rows = rows;
  a.history = history;
  a.kv_tokens = (int)tokens;
  a.qheads = qheads;
  a.kvheads = kv->kvheads;
  a.head_dim = kv->head_dim;
  a.q_row = q_row;
  a.out_row = out_row;
  a.vt_row = vt_row;
  a.softmax_scale = softmax_scale;
  a.workspace = split;
  a.workspace_bytes = (int64_t)kSplitBytes;
  // Check both launches' arguments before touching the shared array: a
  // rejected call must not overwrite scratch that an earlier call may still
  // be reading.
  if (!qi::kv_dequant_request_valid(kv, block_table, 0, (int)tokens, a.k, tokens, a.vt, vt_row) ||
      !qi::attention_request_valid(&a))
    return (int)cudaErrorInvalidValue;
  e = cudaMemsetAsync(split, 0, 4096, stream);  // arrival counters of the split units
  if (e != cudaSuccess) return (int)e;
  int rc = qi_kv_dequant(kv, block_table, (int)tokens, base, base + k_span, vt_row, stream);
  if (rc) return rc;
  return qi_prefill_attention(&a, stream);
}
