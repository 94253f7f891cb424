// Bucket decode attention over the paged NVFP4 KV cache (one query token per
// request), the decode-side counterpart of the reference's native-XQA task
// backend (src/qwen_infra/kernels/nvfp4_bucket_xqa.cu:79-288,
// nvfp4_bucket_xqa.py:19-69) on this build's cache format: 16-token pages,
// [pages, page, Hkv, D/2] e2m1 codes + [pages, page, Hkv, D/16] e4m3 scales,
// the cache the prefill path appends to.
//
// Plan (qi_decode_assign): the KV of each request is cut into 256-token tiles
// and the tiles into tasks, in one of the reference's three modes: intervals
// (requests laid end to end, buckets of `budget` tiles), cyclic (`splits`
// tasks per request, task s taking tiles s, s+splits, ...), aligned (the
// smallest budget whose per-request ceil(tiles/budget) tasks fit in `ctas`).
//
// Compute (qi_decode_attention): one CTA per (task slot, KV head), 128
// threads, thread t <-> key t of a 128-key block <-> TMEM lane t.  HBM-bound:
// a key costs D/2 + D/16 bytes of K and as much of V per KV head, and the
// group of G = Hq/Hkv query heads makes 4*G*D flops of it -- too many for the
// CUDA cores at HBM speed, so both products run on tcgen05:
//   S^T[keys, 64] = K . Qt^T: kind::mxf4nvf4 straight on the cached K codes
//                            (A, shared memory) and block scales (TMEM), with
//                            the query group written as a sum of four NVFP4
//                            terms (B: 4 terms x 16 heads); per head the four
//                            term columns combine in registers with their
//                            power-of-two global scales;
//   O^T[D, G]  += V^T . P^T: A = V (dequantised to f16) from shared memory in
//                            its natural [key][D] order, read MN-major (no
//                            transpose), B = P (f16) from shared memory.
// Two K = 64 block-scaled MMAs make S where the f16 form needs eight K = 16
// ones.  Neither HBM nor the MMAs bound the kernel: each CTA's block is a
// serial chain (load issue, V dequantisation, S, softmax, P, PV) and three
// CTAs per SM overlap three chains.  The softmax
// runs in the log2 domain with a running max per head (CTA-wide reductions
// through shared memory), P is rounded to f16 for the PV product and the
// running sum takes the unrounded exponentials.  A request served by several
// tasks writes unnormalised partials (O, m, l); the last task to finish (per
// request and KV head) merges them in slot order, so the result does not
// depend on the order the CTAs ran in.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "qwen_infra_b200.h"

using namespace qi;

namespace {

constexpr int kD = 128;          // head dim served
constexpr int kBlock = 128;      // keys per MMA block
constexpr int kTile = 256;       // tokens per plan unit
constexpr int kMaxGroup = 16;    // query heads per KV head (MMA N = 16)
constexpr int kThreads = 128;
constexpr int kMaxBatch = 32;
constexpr int kMaxCtas = 340;
constexpr float kMaxLag = 8.0f;  // log2 headroom of the deferred softmax maximum

constexpr int kQTerms = 4;        // NVFP4 terms of the query group (B rows 16 t + j)

// TMEM columns (128 allocated): S^T (4 terms x 16 heads), O^T, block scales
// of K (A) and of the query terms (B), 4 columns per K = 64 MMA each.
constexpr uint32_t kColS = 0, kColO = 64, kColSfa = 80, kColSfb = 88, kTmemCols = 128;

// Shared memory (offsets from the 1024-aligned base).
constexpr uint32_t kOffV = 0;                  // V block, MN-major SW128: 2 D-halves x 16 KB
constexpr uint32_t kVHalf = 16384;
// K codes and query terms share one SW128 region of 128-byte rows: row r
// holds key r's 64 code bytes in its first half (16-byte chunks 0-3 before the
// swizzle) and, for r < 64, query-term row r in its second half (chunks 4-7).
constexpr uint32_t kOffK = 32768;
constexpr uint32_t kQHalf = 64;                // byte offset of the query terms within a row
constexpr uint32_t kOffP = kOffK + 16384;      // P operand:   2 K-blocks x (16 rows x 128 B)
constexpr uint32_t kOffSfk = kOffP + 4096;     // K scales of the block, [key][8] bytes
constexpr uint32_t kOffSfq = kOffSfk + 1024;   // query-term scales, [64 rows][8] bytes
constexpr uint32_t kOffRed = kOffSfq + 512;    // float [4][16] reductions + [kQTerms][4] term maxima
constexpr uint32_t kOffMisc = kOffRed + (4 * kMaxGroup + 4 * kQTerms) * 4;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack

// ---------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------
__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

__global__ void __launch_bounds__(128) assign_kernel(const int32_t* __restrict__ lengths, QiDecodeTask* tasks,
                                                     QiDecodeRange* requests, QiDecodeBucket* buckets,
                                                     int32_t* header, int batch, int ctas, int table_width,
                                                     int page_size, int mode) {
  __shared__ int prefix[kMaxBatch + 1], base[kMaxBatch + 1], first[kMaxBatch];
  __shared__ int s_budget, s_splits, s_slots;
  if (threadIdx.x == 0) {
    prefix[0] = base[0] = 0;
    const int cap = table_width * page_size;  // lengths past the page table are clamped (and flagged by compute)
    for (int r = 0; r < batch; ++r) prefix[r + 1] = prefix[r] + cdiv(min(max(0, lengths[r]), cap), kTile);
    int budget = max(2, cdiv(prefix[batch], ctas));
    if (mode == 2) {  // smallest budget with sum ceil(n / budget) <= ctas (monotone: bisect)
      int lo = 1, hi = 1;
      for (int r = 0; r < batch; ++r) hi = max(hi, prefix[r + 1] - prefix[r]);
      while (lo < hi) {
        const int mid = (lo + hi) / 2;
        int count = 0;
        for (int r = 0; r < batch; ++r) count += cdiv(prefix[r + 1] - prefix[r], mid);
        if (count <= ctas) hi = mid; else lo = mid + 1;
      }
      budget = lo;
    }
    const int splits = min(max(1, ctas / batch), cdiv(table_width * page_size, kTile));
    int max_count = 0;
    for (int r = 0; r < batch; ++r) {
      const int n = prefix[r + 1] - prefix[r];
      first[r] = prefix[r] / budget;
      const int count = mode == 1 ? splits
                        : mode == 2 ? cdiv(n, budget)
                                    : (n ? (prefix[r + 1] - 1) / budget - first[r] + 1 : 0);
      requests[r] = QiDecodeRange{base[r], count};
      base[r + 1] = base[r] + count;
      max_count = max(max_count, count);
    }
    s_budget = budget;
    s_splits = splits;
    s_slots = base[batch];
    header[0] = mode == 1 ? splits : budget;
    header[1] = base[batch];
    header[2] = mode ? base[batch] : cdiv(prefix[batch], budget);
    header[3] = max_count;
  }
  __syncthreads();
  const int budget = s_budget, splits = s_splits, slots = s_slots;
  for (int slot = threadIdx.x; slot < slots; slot += blockDim.x) {
    int r = 0;
    while (r + 1 < batch && base[r + 1] <= slot) ++r;
    const int ordinal = slot - base[r], n = prefix[r + 1] - prefix[r];
    if (mode == 1) {
      tasks[slot] = QiDecodeTask{r, ordinal, n, splits};
    } else if (mode == 2) {
      const int count = base[r + 1] - base[r];
      tasks[slot] = QiDecodeTask{r, ordinal * n / count, (ordinal + 1) * n / count, 1};
    } else {
      const int bucket = first[r] + ordinal;
      const int lo = max(prefix[r], bucket * budget) - prefix[r];
      const int hi = min(prefix[r + 1], (bucket + 1) * budget) - prefix[r];
      tasks[slot] = QiDecodeTask{r, lo, hi, 1};
    }
  }
  // Buckets: the task slots each persistent CTA runs (intervals mode), one
  // slot per CTA (aligned mode), none (cyclic mode).
  for (int b = threadIdx.x; b < ctas; b += blockDim.x) {
    if (mode == 2) {
      buckets[b] = b < slots ? QiDecodeBucket{b, b + 1} : QiDecodeBucket{0, 0};
      continue;
    }
    const int lo = b * budget, hi = min(prefix[batch], lo + budget);
    if (mode == 1 || lo >= hi) {
      buckets[b] = QiDecodeBucket{0, 0};
      continue;
    }
    int fr = 0;
    while (fr + 1 < batch && prefix[fr + 1] <= lo) ++fr;
    int lr = fr;
    while (lr + 1 < batch && prefix[lr + 1] < hi) ++lr;
    buckets[b] = QiDecodeBucket{base[fr] + b - first[fr], base[lr] + b - first[lr] + 1};
  }
}

// ---------------------------------------------------------------------------
// Compute helpers
// ---------------------------------------------------------------------------

// 32 lanes x 8 columns (register i -> column taddr + i).
__device__ __forceinline__ void tmem_st8w(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
// Loads without the wait (the caller issues tcgen05.wait::ld once for several).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D (+)= A . B, both from shared memory.
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// S: kind::mxf4nvf4, M = 128 keys, N = 4 terms x 16 heads.  PV: kind::f16,
// f16 A and B, fp32 accumulator, M = 128, N = 16, bit 15: A is MN-major (V
// read in its natural [key][D] order).
constexpr uint32_t kIdescS = idesc_nvfp4(kQTerms * kMaxGroup);
constexpr uint32_t kIdescO =
    (1u << 4) | (1u << 15) | ((uint32_t)(kMaxGroup >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

// Byte offset of element (row, k) in a K-major SW128 operand of 16 rows whose
// K extent is split into 64-element blocks of 2 KB (16 rows x 128 B).
__device__ __forceinline__ uint32_t kmajor16_offset(int row, int k) {
  const int kb = k >> 6, kk = k & 63;
  const int chunk = (kk >> 3) ^ (row & 7);
  return kb * 2048 + (row >> 3) * 1024 + (row & 7) * 128 + chunk * 16 + (kk & 7) * 2;
}

// ---------------------------------------------------------------------------
// Compute
// ---------------------------------------------------------------------------
struct DecodeArgs {
  const __nv_bfloat16* q;
  const uint8_t *kc, *vc, *ks, *vs;
  int64_t data_page, data_row, data_head, sf_page, sf_row, sf_head;
  const int32_t* table;
  const int32_t* lengths;
  const QiDecodeTask* tasks;
  const QiDecodeRange* requests;
  const QiDecodeBucket* buckets;
  const int32_t* header;
  int32_t* semaphores;
  float* part_o;   // [capacity][Hkv][16][D]
  float* part_ml;  // [capacity][Hkv][16][2]
  void* out;
  const __nv_bfloat16* gate;
  const float* out_scale;
  const float *k_global, *v_global;
  int* status;
  int batch, table_width, page_size, page_shift, kvheads, qheads, group, persistent;
  float softmax_scale;
};

// The block's bytes one thread loads.  Loads are coalesced 256-bit vectors:
// thread (warp w, lane l) reads the 32-byte half l % 2 of key rows
// 32 w + 16 j + l / 2 (j = 0, 1), so one warp instruction covers 16 keys x 64
// contiguous bytes (a key per thread would touch 32 lines per instruction and
// load-issue would throttle).  Even lanes also read the key's K scales, odd
// lanes its V scales (one instruction for both).
struct BlockBytes {
  uint4 k[2][2], v[2][2];  // [j][16-byte chunk of the 32-byte half]
  uint2 s[2];
};

__device__ __forceinline__ int load_key_index(int warp, int lane, int j) { return warp * 32 + j * 16 + (lane >> 1); }

__device__ __forceinline__ void ld256(const uint8_t* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.cs.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w)
               : "l"(p));
}
__device__ __forceinline__ uint2 ld64(const uint8_t* p) {
  uint2 r;
  asm volatile("ld.global.cs.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// Page id of a key (-1 past the length).  Looked up two blocks ahead of use,
// so the dependent table load never stalls the key loads.
__device__ __forceinline__ int page_of(const DecodeArgs& a, int r, int key, int length) {
  return key < length ? __ldg(a.table + (int64_t)r * a.table_width + (key >> a.page_shift)) : -1;
}
__device__ __forceinline__ void block_pages(const DecodeArgs& a, int r, int base, int length, int warp, int lane,
                                            int* pg) {
#pragma unroll
  for (int j = 0; j < 2; ++j) pg[j] = page_of(a, r, base + load_key_index(warp, lane, j), length);
}

__device__ __forceinline__ void load_block(const DecodeArgs& a, int h, int base, const int* pg, int warp, int lane,
                                           BlockBytes& bb) {
  const int hf = lane & 1;
  const uint8_t* sbuf = hf ? a.vs : a.ks;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if (pg[j] >= 0) {
      const int entry = (base + load_key_index(warp, lane, j)) & (a.page_size - 1);
      const int64_t d = (int64_t)pg[j] * a.data_page + (int64_t)entry * a.data_row + (int64_t)h * a.data_head + hf * 32;
      const int64_t s = (int64_t)pg[j] * a.sf_page + (int64_t)entry * a.sf_row + (int64_t)h * a.sf_head;
      ld256(a.kc + d, bb.k[j][0], bb.k[j][1]);
      ld256(a.vc + d, bb.v[j][0], bb.v[j][1]);
      bb.s[j] = ld64(sbuf + s);
    } else {
      bb.k[j][0] = bb.k[j][1] = bb.v[j][0] = bb.v[j][1] = make_uint4(0, 0, 0, 0);
      bb.s[j] = make_uint2(0, 0);
    }
  }
}

// Next 128-key block of a task after (tile, sub): the second block of a tile
// while inside the length, else the first block of the next tile.
__device__ __forceinline__ void next_block(int& tile, int& sub, int stride, int length) {
  if (sub == 0 && tile * kTile + kBlock < length) {
    sub = 1;
  } else {
    tile += stride;
    sub = 0;
  }
}

__device__ __forceinline__ float ex2f(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Final value of output element (query head `qh`, dimension d) of request r.
__device__ __forceinline__ void store_out(const DecodeArgs& a, int r, int qh, int d, float v) {
  const int64_t i = ((int64_t)r * a.qheads + qh) * kD + d;
  if (a.gate) {
    const float ob = bf16r(v);
    const float sg = bf16r(sigmoid_f(__bfloat162float(a.gate[i])));
    const float gv = bf16r(__fmul_rn(ob, sg));
    static_cast<uint8_t*>(a.out)[i] = (uint8_t)f_to_e4m3(__fdiv_rn(gv, *a.out_scale));
  } else {
    static_cast<__nv_bfloat16*>(a.out)[i] = __float2bfloat16_rn(v);
  }
}

// Three CTAs per SM (shared memory); a fourth, with 128 registers a thread,
// measured slower.
template <int GP>
__global__ void __launch_bounds__(kThreads, 3) decode_kernel(const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(sm + kOffRed);  // [4 warps][16]
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + kOffMisc);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_o + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 2);
  float* cg = reinterpret_cast<float*>(sm + kOffMisc + 32);  // [kQTerms] scale2 / g_t of the current task

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x % a.kvheads, owner = blockIdx.x / a.kvheads;
  const int G = a.group;

  // A request with no keys gets zeros (written by the CTA whose owner index is
  // that request, which also clears the request's semaphore).
  const int cap = a.table_width * a.page_size;
  if (owner < a.batch && a.lengths[owner] <= 0) {
    for (int i = tid; i < G * kD; i += kThreads) {
      const int64_t o = ((int64_t)owner * a.qheads + h * G + i / kD) * kD + (i % kD);
      if (a.gate) static_cast<uint8_t*>(a.out)[o] = 0;
      else static_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(0.0f);
    }
    if (tid == 0) a.semaphores[owner * a.kvheads + h] = 0;
  }

  int slot_begin, slot_end;
  const int count = a.header[1];
  if (a.persistent) {
    const QiDecodeBucket b = a.buckets[owner];
    slot_begin = b.begin;
    slot_end = min(b.end, count);
  } else {
    slot_begin = owner;
    slot_end = owner < count ? owner + 1 : owner;
  }
  if (slot_begin >= slot_end) return;  // CTA-uniform

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  {  // P rows past the group stay zero
    uint4* p = reinterpret_cast<uint4*>(sm + kOffP);
    p[tid] = make_uint4(0, 0, 0, 0);
    p[tid + kThreads] = make_uint4(0, 0, 0, 0);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t sV = smem_u32(sm + kOffV), sK = smem_u32(sm + kOffK), sQ = sK + kQHalf, sP = smem_u32(sm + kOffP);
  const float scale2 = __fmul_rn(__fmul_rn(a.softmax_scale, *a.k_global), 1.4426950408889634f);
  const float vglob = *a.v_global;
  uint32_t phase_s = 0, phase_o = 0;
  bool ok = true;

  for (int slot = slot_begin; ok && slot < slot_end; ++slot) {
    const QiDecodeTask task = a.tasks[slot];
    const int r = task.request, L = min(a.lengths[r], cap);
    if (L <= 0) continue;  // CTA-uniform
    if (a.lengths[r] > cap && tid == 0 && h == 0 && slot == a.requests[r].first) report(a.status, QI_STATUS_BAD_LENGTH);
    const QiDecodeRange range = a.requests[r];

    // The query group as a sum of kQTerms NVFP4 rows, the B operand of the S
    // product: row n = 16 t + j holds term t of query head j (rows of heads
    // >= G are zero).  Term t quantises the residual the earlier terms left,
    // per 16 elements, with a power-of-two global scale
    // g_t = 2^floor(log2(2688 / amax_t)) (amax over the whole group), so its
    // values code * scale / g_t are exact in fp32 and each term removes about
    // 3.5 bits of the residual: four leave ~1e-4 of the group's largest value.
    // S = sum_t (K . term_t) / g_t, combined per head in registers
    // (cg[t] = scale2 / g_t).  Thread <-> (head j = tid / 8, block b = tid % 8).
    {
      const int j = tid >> 3, b = tid & 7;
      float rv[16];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (j < G) raw = *reinterpret_cast<const uint4*>(a.q + ((int64_t)r * a.qheads + h * G + j) * kD + b * 16 + i * 8);
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(b2[e]);
          rv[i * 8 + 2 * e] = f.x;
          rv[i * 8 + 2 * e + 1] = f.y;
        }
      }
      float* tred = red + 4 * kMaxGroup;  // [kQTerms][4 warps]
#pragma unroll
      for (int t = 0; t < kQTerms; ++t) {
        float am = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(rv[e]));
        am = warp_max_butterfly(am);
        if (lane == 0) tred[t * 4 + warp] = am;
        __syncthreads();
        const float amax = fmaxf(fmaxf(tred[t * 4], tred[t * 4 + 1]), fmaxf(tred[t * 4 + 2], tred[t * 4 + 3]));
        uint2 packed = make_uint2(0, 0);
        uint32_t sf = 0;
        float ig = 0.0f;
        if (amax > 0.0f) {  // CTA-uniform
          const float y = fminf(fmaxf(__fdiv_rn(2688.0f, amax), 0x1p-100f), 0x1p100f);
          const float g = __uint_as_float(__float_as_uint(y) & 0x7F800000u);  // 2^floor(log2 y)
          ig = __uint_as_float((254u << 23) - __float_as_uint(g));            // 1 / g, exact
          sf = nvfp4_quant16(rv, g, packed);
          const float sc = e4m3_to_f(sf);
          uint32_t hv[8];
          e2m1x8_to_f16x8(packed.x, hv);
          e2m1x8_to_f16x8(packed.y, hv + 4);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint32_t bits = (e & 1) ? hv[e >> 1] >> 16 : hv[e >> 1] & 0xFFFFu;
            const float cv = __half2float(__ushort_as_half((unsigned short)bits));
            rv[e] = __fsub_rn(rv[e], __fmul_rn(__fmul_rn(cv, sc), ig));
          }
        }
        if (tid == 0) cg[t] = __fmul_rn(ig, scale2);
        const int n = t * kMaxGroup + j;
        *reinterpret_cast<uint2*>(sm + kOffK + (n >> 3) * 1024 + (n & 7) * 128 + (((4 + (b >> 1)) ^ (n & 7)) * 16) +
                                  (b & 1) * 8) = packed;
        sm[kOffSfq + n * 8 + b] = (uint8_t)sf;
      }
      __syncthreads();
      // Term scales -> TMEM in the MMA's scale layout: lane l of every lane
      // quarter, column 4 kk + c, holds the four scales (K block kk) of row
      // l + 32 c; rows 64..127 do not exist (N = 64) and stay zero.
      uint32_t v[8];
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          v[kk * 4 + c] = c < 2 ? *reinterpret_cast<const uint32_t*>(sm + kOffSfq + (lane + 32 * c) * 8 + kk * 4) : 0u;
      __syncwarp();
      tmem_st8w(tmem + lane_base + kColSfb, v);
    }

    float m_run[GP], l_thr[GP];
#pragma unroll
    for (int j = 0; j < GP; ++j) m_run[j] = -INFINITY, l_thr[j] = 0.0f;
    bool first_pv = true;

    // Blocks of the task: tiles begin, begin + stride, ... < end; two
    // 128-key blocks per tile while inside the length.  Block i's bytes are
    // loaded into registers during block i - 1, issued right after block
    // i - 1's S product (the load issue overlaps the MMA), and their page ids
    // are looked up during block i - 2.
    int tile = task.begin, sub = 0;
    bool have = tile < task.end;
    int t1 = tile, s1 = sub;  // the blocks 1 and 2 after the current one
    next_block(t1, s1, task.stride, L);
    int t2 = t1, s2 = s1;
    next_block(t2, s2, task.stride, L);
    BlockBytes bb;
    int pg1[2] = {-1, -1};  // page ids of the block after the current one
    if (have) {
      int pg0[2];
      block_pages(a, r, tile * kTile, L, warp, lane, pg0);
      load_block(a, h, tile * kTile, pg0, warp, lane, bb);
      if (t1 < task.end) block_pages(a, r, t1 * kTile + s1 * kBlock, L, warp, lane, pg1);
    }
    while (have) {
      const int key = tile * kTile + sub * kBlock + tid;
      const bool valid = key < L;
      const bool have_next = t1 < task.end;

      // K codes -> shared memory (A operand, row = key, 128-byte swizzle),
      // K scales -> the exchange table.  The previous block's S product has
      // finished with both (its barrier was waited on).
      const int hf = lane & 1;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kr = load_key_index(warp, lane, j);
        uint8_t* krow = sm + kOffK + (kr >> 3) * 1024 + (kr & 7) * 128;
        *reinterpret_cast<uint4*>(krow + (((2 * hf) ^ (kr & 7)) * 16)) = bb.k[j][0];
        *reinterpret_cast<uint4*>(krow + (((2 * hf + 1) ^ (kr & 7)) * 16)) = bb.k[j][1];
        if (hf == 0) *reinterpret_cast<uint2*>(sm + kOffSfk + kr * 8) = bb.s[j];
      }
      // The previous PV product still reads V and P.
      if (!first_pv) {
        ok = mbar_wait(bar_o, phase_o, abort_flag, a.status);
        phase_o ^= 1;
      }
      ok = __syncthreads_and(ok);
      if (!ok) break;
      {  // K scales -> TMEM: lane l of each quarter, column 4 kk + c <- key l + 32 c
        uint32_t v[8];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            v[kk * 4 + c] = *reinterpret_cast<const uint32_t*>(sm + kOffSfk + (lane + 32 * c) * 8 + kk * 4);
        tmem_st8w(tmem + lane_base + kColSfa, v);
      }
      // V -> shared memory as f16, natural [key][D] order, 128-byte swizzle:
      // a thread's 32 bytes of a key are the 64 elements of D-half hf (scale
      // groups 4 hf .. 4 hf + 3: word hf of the V scales its odd partner lane
      // loaded).
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kr = load_key_index(warp, lane, j);
        const uint32_t sx = __shfl_sync(0xffffffffu, bb.s[j].x, lane | 1);
        const uint32_t sy = __shfl_sync(0xffffffffu, bb.s[j].y, lane | 1);
        const uint32_t sw = hf ? sy : sx;
        const uint32_t s01 = e4m3x2_to_f16x2(sw & 0xFFFFu), s23 = e4m3x2_to_f16x2(sw >> 16);
        uint8_t* row = sm + kOffV + hf * kVHalf + (kr >> 3) * 1024 + (kr & 7) * 128;
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // 16-byte code chunk: 32 elements, groups 2 q, 2 q + 1
          const uint4 cv = bb.v[j][q];
          const uint32_t words[4] = {cv.x, cv.y, cv.z, cv.w};
          uint32_t pairs[16];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int group = 2 * q + (w >> 1);
            const uint32_t s2 = splat_half(group < 2 ? s01 : s23, group & 1);
            uint32_t f[4];
            e2m1x8_to_f16x8(words[w], f);
#pragma unroll
            for (int e = 0; e < 4; ++e) pairs[w * 4 + e] = hmul2u(f[e], s2);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(row + (((4 * q + c) ^ (kr & 7)) * 16)) =
                make_uint4(pairs[4 * c], pairs[4 * c + 1], pairs[4 * c + 2], pairs[4 * c + 3]);
        }
      }
      __syncwarp();
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          mma_nvfp4(tmem + kColS, sdesc_kmajor_sw128(sK + kk * 32), sdesc_kmajor_sw128(sQ + kk * 32), kIdescS,
                    tmem + kColSfa + kk * 4, tmem + kColSfb + kk * 4, (uint32_t)kk);
        tc_commit(bar_s);
      }
      // The next block's loads, issued while the S product runs.
      if (have_next) {
        load_block(a, h, t1 * kTile + s1 * kBlock, pg1, warp, lane, bb);
        if (t2 < task.end) block_pages(a, r, t2 * kTile + s2 * kBlock, L, warp, lane, pg1);
        else pg1[0] = pg1[1] = -1;
      }
      __syncwarp();
      ok = mbar_wait(bar_s, phase_s, abort_flag, a.status);
      phase_s ^= 1;
      __syncwarp();
      tc_fence_after();
      // S per head: the four term columns, each times scale2 / g_t.
      // (GP = 16 reads one term per round trip to stay within the registers.)
      constexpr int kTermsPerLoad = GP == 16 ? 1 : 2;
      float sv[16];
#pragma unroll
      for (int t0 = 0; t0 < kQTerms; t0 += kTermsPerLoad) {
        uint32_t d[kTermsPerLoad][GP];
#pragma unroll
        for (int u = 0; u < kTermsPerLoad; ++u) {
          if constexpr (GP == 16) tmem_ld16_async(tmem + lane_base + kColS + (t0 + u) * kMaxGroup, d[u]);
          else tmem_ld8_async(tmem + lane_base + kColS + (t0 + u) * kMaxGroup, d[u]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < GP; ++j)
#pragma unroll
          for (int u = 0; u < kTermsPerLoad; ++u)
            sv[j] = t0 + u == 0 ? __fmul_rn(__uint_as_float(d[0][j]), cg[0])
                                : __fmaf_rn(__uint_as_float(d[u][j]), cg[t0 + u], sv[j]);
      }
      // Deferred maximum: the running maxima m stay while no score of the
      // block exceeds them by more than 8 (P <= 2^8, exact enough in f16);
      // otherwise (and on a task's first block) all heads move to the block
      // maximum through a CTA-wide reduction and O is rescaled.
      bool grow = first_pv;
#pragma unroll
      for (int j = 0; j < GP; ++j) {
        sv[j] = valid ? sv[j] : -INFINITY;
        grow |= sv[j] > m_run[j] + kMaxLag;
      }
      if (__syncthreads_or(grow || !ok)) {
        ok = __syncthreads_and(ok);
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          const float mx = warp_max_butterfly(sv[j]);
          if (lane == 0) red[warp * 16 + j] = mx;
        }
        __syncthreads();
        bool rescale = false;
        float alpha[GP];
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          const float bm = fmaxf(fmaxf(red[j], red[16 + j]), fmaxf(red[32 + j], red[48 + j]));
          const float mn = fmaxf(m_run[j], bm);
          alpha[j] = m_run[j] == -INFINITY ? 0.0f : ex2f(m_run[j] - mn);
          rescale |= alpha[j] != 1.0f;
          l_thr[j] = __fmul_rn(l_thr[j], alpha[j]);
          m_run[j] = mn;
        }
        if (!first_pv && rescale) {  // CTA-uniform: every thread read the same maxima
          float o[16];
          tmem_ld16(tmem + lane_base + kColO, o);
#pragma unroll
          for (int j = 0; j < GP; ++j) o[j] = __fmul_rn(o[j], alpha[j]);
          tmem_st16(tmem + lane_base + kColO, o);
        }
      }
#pragma unroll
      for (int j = 0; j < GP; ++j) {
        const float p = valid ? ex2f(sv[j] - m_run[j]) : 0.0f;
        l_thr[j] = __fadd_rn(l_thr[j], p);
        sv[j] = p;
      }
#pragma unroll
      for (int j = 0; j < GP; ++j)
        *reinterpret_cast<__half*>(sm + kOffP + kmajor16_offset(j, tid)) = __float2half_rn(sv[j]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < kBlock / 16; ++s)
          mma_ss(tmem + kColO, sdesc_mnmajor_sw128(sV + s * 2048, kVHalf, 1024),
                 sdesc_kmajor_sw128(sP + (s >> 2) * 2048 + (s & 3) * 32), kIdescO, (!first_pv || s > 0) ? 1u : 0u);
        tc_commit(bar_o);
      }
      __syncwarp();
      first_pv = false;
      tile = t1, sub = s1, have = have_next;
      t1 = t2, s1 = s2;
      next_block(t2, s2, task.stride, L);
    }
    if (!ok) break;
    if (!first_pv) {
      ok = mbar_wait(bar_o, phase_o, abort_flag, a.status);
      phase_o ^= 1;
      tc_fence_after();
    }
    ok = __syncthreads_and(ok);
    if (!ok) break;

    // Row sums: per head over the 128 threads (fixed butterfly + fixed order).
#pragma unroll
    for (int j = 0; j < GP; ++j) {
      const float s = warp_sum_butterfly(l_thr[j]);
      if (lane == 0) red[warp * 16 + j] = s;
    }
    __syncthreads();
    float lsum[GP];
#pragma unroll
    for (int j = 0; j < GP; ++j) lsum[j] = __fadd_rn(__fadd_rn(red[j], red[16 + j]), __fadd_rn(red[32 + j], red[48 + j]));
    float o[16];
    if (!first_pv) {
      tmem_ld16(tmem + lane_base + kColO, o);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = 0.0f;
    }
    const int d = tid;
    if (range.count == 1) {
#pragma unroll
      for (int j = 0; j < GP; ++j)
        if (j < G) store_out(a, r, h * G + j, d, __fmul_rn(o[j], __fdiv_rn(vglob, lsum[j])));
    } else {
      float* po = a.part_o + ((int64_t)slot * a.kvheads + h) * 16 * kD;
      float* pml = a.part_ml + ((int64_t)slot * a.kvheads + h) * 16 * 2;
#pragma unroll
      for (int j = 0; j < GP; ++j)
        if (j < G) __stcg(po + j * kD + d, o[j]);
#pragma unroll
      for (int j = 0; j < GP; ++j)
        if (j < G && d == j) {
          __stcg(pml + 2 * j, m_run[j]);
          __stcg(pml + 2 * j + 1, lsum[j]);
        }
      __threadfence();
      __syncthreads();
      if (tid == 0) *s_last = atomicAdd(a.semaphores + r * a.kvheads + h, 1) == range.count - 1;
      __syncthreads();
      if (*s_last) {
        __threadfence();
        for (int j = 0; j < G; ++j) {
          float mx = -INFINITY;
          for (int i = range.first; i < range.first + range.count; ++i)
            mx = fmaxf(mx, __ldcg(a.part_ml + (((int64_t)i * a.kvheads + h) * 16 + j) * 2));
          float acc = 0.0f, lt = 0.0f;
          for (int i = range.first; i < range.first + range.count; ++i) {
            const float* ml = a.part_ml + (((int64_t)i * a.kvheads + h) * 16 + j) * 2;
            const float mi = __ldcg(ml);
            const float w = mi == -INFINITY ? 0.0f : ex2f(mi - mx);
            lt = __fadd_rn(lt, __fmul_rn(w, __ldcg(ml + 1)));
            acc = __fadd_rn(acc, __fmul_rn(w, __ldcg(a.part_o + (((int64_t)i * a.kvheads + h) * 16 + j) * kD + d)));
          }
          store_out(a, r, h * G + j, d, __fmul_rn(acc, __fdiv_rn(vglob, lt)));
        }
        if (tid == 0) atomicExch(a.semaphores + r * a.kvheads + h, 0);
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and shared memory are reused by the next slot
    tc_fence_after();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

template <class Kernel>
static cudaError_t configure(Kernel kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

// Resident CTAs per SM of one kernel from its own limits: registers
// (256-register warp granules), shared memory (plus the 1 KB the system
// reserves per CTA) and tensor memory (512 columns).  (The runtime occupancy
// query does not know the tensor-memory limit.)
template <class Kernel>
static int resident_ctas(Kernel kernel, int* regs, int* local) {
  cudaError_t e = configure(kernel);
  if (e != cudaSuccess) return -(int)e;
  cudaFuncAttributes attr;
  e = cudaFuncGetAttributes(&attr, kernel);
  if (e != cudaSuccess) return -(int)e;
  int dev = 0, smem_sm = 0, regs_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
  const int warp_regs = (attr.numRegs * 32 + 255) / 256 * 256;
  *regs = attr.numRegs;
  *local = (int)attr.localSizeBytes;
  return std::min(std::min(regs_sm / (warp_regs * (kThreads / 32)), smem_sm / ((int)kSmemBytes + 1024)),
                  512 / (int)kTmemCols);
}

extern "C" {

static int decode_check(const QiDecode* p) {
  if (!p || p->batch < 1 || p->batch > kMaxBatch || p->ctas < p->batch || p->ctas > kMaxCtas ||
      p->table_width < 1 || p->mode < 0 || p->mode > 2 || (p->persistent && p->mode != 0))
    return (int)cudaErrorInvalidValue;
  const QiKvView& kv = p->kv;
  // Pages of a power-of-two token count (the page of a key is a shift).
  if (kv.head_dim != kD || kv.kvheads < 1 || kv.page_size < 1 || (kv.page_size & (kv.page_size - 1)) ||
      p->qheads < kv.kvheads ||
      p->qheads % kv.kvheads || p->qheads / kv.kvheads > kMaxGroup ||
      (int64_t)p->table_width * kv.page_size > (int64_t)0x7fffffff - (kTile - 1))
    return (int)cudaErrorInvalidValue;
  if (!p->lengths || !p->tasks || !p->requests || !p->buckets || !p->header) return (int)cudaErrorInvalidValue;
  return 0;
}

int qi_decode_assign(const QiDecode* p, cudaStream_t stream) {
  if (const int e = decode_check(p)) return e;
  QI_BIND(stream, p->tasks);
  assign_kernel<<<1, 128, 0, stream>>>(p->lengths, p->tasks, p->requests, p->buckets, p->header, p->batch, p->ctas,
                                       p->table_width, p->kv.page_size, p->mode);
  return (int)cudaPeekAtLastError();
}

int qi_decode_attention(const QiDecode* p, cudaStream_t stream) {
  if (const int e = decode_check(p)) return e;
  const QiKvView& kv = p->kv;
  if (!p->q || !kv.k_cache || !kv.v_cache || !kv.k_scales || !kv.v_scales || !p->block_table || !p->semaphores ||
      !p->scratch || !p->out || !p->k_global || !p->v_global || (p->gate && !p->out_scale))
    return (int)cudaErrorInvalidValue;
  // 32-byte code loads, 8-byte scale loads, 16-byte Q loads.
  auto a32 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 31) == 0; };
  auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  auto a8 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 7) == 0; };
  if (!a32(kv.k_cache) || !a32(kv.v_cache) || kv.data_page % 32 || kv.data_row % 32 || kv.data_head % 32 ||
      !a8(kv.k_scales) || !a8(kv.v_scales) || kv.sf_page % 8 || kv.sf_row % 8 || kv.sf_head % 8 || !a16(p->q) ||
      !a16(p->scratch) || (reinterpret_cast<uintptr_t>(p->out) & 1) || (reinterpret_cast<uintptr_t>(p->gate) & 1))
    return (int)cudaErrorInvalidValue;
  QI_BIND(stream, p->out);
  const int capacity = p->ctas + p->batch - 1;
  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(p->q);
  a.kc = static_cast<const uint8_t*>(kv.k_cache);
  a.vc = static_cast<const uint8_t*>(kv.v_cache);
  a.ks = static_cast<const uint8_t*>(kv.k_scales);
  a.vs = static_cast<const uint8_t*>(kv.v_scales);
  a.data_page = kv.data_page, a.data_row = kv.data_row, a.data_head = kv.data_head;
  a.sf_page = kv.sf_page, a.sf_row = kv.sf_row, a.sf_head = kv.sf_head;
  a.table = p->block_table;
  a.lengths = p->lengths;
  a.tasks = p->tasks;
  a.requests = p->requests;
  a.buckets = p->buckets;
  a.header = p->header;
  a.semaphores = p->semaphores;
  a.part_o = static_cast<float*>(p->scratch);
  a.part_ml = a.part_o + (int64_t)capacity * kv.kvheads * kMaxGroup * kD;
  a.out = p->out;
  a.gate = static_cast<const __nv_bfloat16*>(p->gate);
  a.out_scale = p->out_scale;
  a.k_global = p->k_global;
  a.v_global = p->v_global;
  a.status = p->status;
  a.batch = p->batch, a.table_width = p->table_width, a.page_size = kv.page_size;
  a.page_shift = 0;
  while ((1 << a.page_shift) < kv.page_size) ++a.page_shift;
  a.kvheads = kv.kvheads, a.qheads = p->qheads, a.group = p->qheads / kv.kvheads;
  a.persistent = p->persistent;
  a.softmax_scale = p->softmax_scale;
  const int splits = std::min(std::max(1, p->ctas / p->batch), (p->table_width * kv.page_size + kTile - 1) / kTile);
  const int slots = p->persistent || p->mode == 2 ? p->ctas : p->mode == 1 ? p->batch * splits : capacity;
  const dim3 grid(slots * kv.kvheads);
  static bool configured[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
  const int gi = a.group <= 8 ? 0 : 1;
  if (!configured[dev][gi]) {
    const cudaError_t e = gi == 0 ? configure(decode_kernel<8>) : configure(decode_kernel<16>);
    if (e != cudaSuccess) return (int)e;
    configured[dev][gi] = true;
  }
  if (gi == 0) decode_kernel<8><<<grid, kThreads, kSmemBytes, stream>>>(a);
  else decode_kernel<16><<<grid, kThreads, kSmemBytes, stream>>>(a);
  return (int)cudaPeekAtLastError();
}

int qi_decode_resources(int* values) {
  if (!values) return (int)cudaErrorInvalidValue;
  int regs8 = 0, local8 = 0, regs16 = 0, local16 = 0;
  const int r8 = resident_ctas(decode_kernel<8>, &regs8, &local8);
  if (r8 < 0) return -r8;
  const int r16 = resident_ctas(decode_kernel<16>, &regs16, &local16);
  if (r16 < 0) return -r16;
  values[0] = (int)sizeof(QiDecode);
  values[1] = regs8;
  values[2] = (int)kSmemBytes;
  values[3] = std::max(local8, local16);
  values[4] = r8;
  values[5] = (int)sizeof(QiDecodeTask);
  values[6] = (int)sizeof(QiDecodeRange);
  values[7] = (int)sizeof(QiDecodeBucket);
  values[8] = regs16;
  values[9] = r16;
  return 0;
}

uint64_t qi_decode_scratch_bytes(int capacity, int kvheads) {
  if (capacity < 1 || capacity > kMaxCtas + kMaxBatch - 1 || kvheads < 1 || kvheads > 64) return 0;
  return (uint64_t)capacity * kvheads * kMaxGroup * (kD + 2) * sizeof(float);
}

}  // extern "C"
