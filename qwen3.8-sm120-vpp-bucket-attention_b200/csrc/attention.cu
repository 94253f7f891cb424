// Chunked causal GQA prefill attention on tcgen05 (sm_100a).
//
// Operands: Q from the QK-norm/RoPE producer (bf16, converted to f16 in shared
// memory - exact for normalised queries), K and V^T from qi_kv_dequant as f16
// (e2m1 x e4m3 products are exact in f16); the fp32 global multipliers of K
// and V are folded into the softmax scale and the output normalisation.  S and
// O accumulate in fp32 in tensor memory; P = 2^(s*scale*log2e - m) is formed
// in fp32 (MUFU ex2), packed to f16 pairs and written back into the S columns
// of tensor memory, from where the PV MMA reads it as its A operand (no
// shared-memory round trip).
//
// One CTA = 256 query rows (two 128-row tiles Q0, Q1) of one query head; 10 warps:
//   warp 0      : TMA producer (Q once; K and V^T tiles of 128 keys, 2 stages),
//   warp 1      : TMEM allocator + the single MMA-issuing thread,
//   warps 2..5  : softmax of Q0 (one query row per thread = TMEM lane),
//   warps 6..9  : softmax of Q1.
// The MMA order is PV0_j, S0_{j+1}, PV1_j, S1_{j+1}, so the tensor cores run
// one tile's PV and next QK^T while the other tile's softmax runs (ping-pong).  The
// running max is only moved (and O rescaled in TMEM) when it grows by more than
// 2^8, which keeps rescales rare; P may then reach 256, well inside f16.
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "qwen_infra_b200.h"

using namespace qi;

namespace {

constexpr int TQ = 128, TK = 128, NQ = 2;
constexpr int ATOM = 128 * 128;            // one 128-row x 128-byte swizzle column (16 KB)
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int HD>
struct Geometry {
  static constexpr int Q_TILE = (HD / 64) * ATOM;  // [128 rows x HD] 16-bit
  static constexpr int K_BYTES = (HD / 64) * ATOM;  // [128 keys x HD]
  static constexpr int V_ATOM = HD * 128;           // [HD rows x 64 keys]
  static constexpr int V_BYTES = 2 * V_ATOM;
  static constexpr int SMEM = NQ * Q_TILE + 2 * K_BYTES + 2 * V_BYTES + 1024 + 256;
  static constexpr uint32_t S_COL0 = 0, S_COL1 = 128, O_COL0 = 256, O_COL1 = 256 + HD;
};

struct AttnParams {
  int rows, history, kv_tokens, qheads, group;
  int64_t out_row;
  __nv_bfloat16* out;
  const float* k_global;
  const float* v_global;
  float softmax_scale;
  int* status;
  int q_blocks;
  // Key-range split of the lightest units (see split_plan): CTAs with
  // blockIdx >= split_first each take half of the key tiles of one unit and
  // combine through the workspace.
  int split_first;
  unsigned* ws_count;  // [slots] arrival counters (parity = which piece is last)
  float* ws_ml;        // [slots][2][NQ*TQ][2] (m, l) per row and piece
  float* ws_o;         // [slots][2][NQ*TQ][HD] unnormalised O per row and piece
  // Paged NVFP4 K/V (the paged kernel only): codes [page][entry][kv head][D/2]
  // and E4M3 scales [..][D/16] through byte strides; keys past kv_tokens read
  // as zeros.
  const uint8_t *kc, *vc, *ksf, *vsf;
  const int32_t* block_table;
  int page_shift;
  int64_t data_page, data_row, data_head, sf_page, sf_row, sf_head;
};

// Workspace of the key-range split for `slots` split units of head_dim hd.
// The arrival counters persist across launches, so they sit at a fixed place
// (the first 4 KB, up to 1024 slots) whatever a launch's split count; the
// (m, l) and O halves after them are rewritten by every launch that reads them.
constexpr int kMaxSlots = 1024;
__host__ __device__ constexpr int64_t ws_count_bytes(int) { return (int64_t)kMaxSlots * 4; }
__host__ __device__ constexpr int64_t ws_ml_bytes(int slots) { return (int64_t)slots * 2 * NQ * TQ * 2 * 4; }
__host__ __device__ constexpr int64_t ws_o_bytes(int slots, int hd) { return (int64_t)slots * 2 * NQ * TQ * hd * 4; }
__host__ __device__ constexpr int64_t ws_bytes(int slots, int hd) {
  return ws_count_bytes(slots) + ws_ml_bytes(slots) + ws_o_bytes(slots, hd);
}

// kind::f16 with F16 A and B (format 0) and an fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// D (+)= A . B with A read from tensor memory (lane = row, consecutive K pairs
// packed in each 32-bit column) and B from shared memory.
QI_DEV void mma_f16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

QI_DEV uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
QI_DEV float ex2_f32(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// 32 lanes x 32 columns load without the completion wait (callers issue several
// and then one tcgen05.wait::ld).
QI_DEV void tmem_ld32_nowait(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
QI_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Packed fp32 pair arithmetic (one instruction for two lanes' worth of work).
QI_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
QI_DEV float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
QI_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
QI_DEV void tmem_st32u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// Max of 64 values in four independent chains (short dependency chains).
QI_DEV float max64(const float* v) {
  float a = fmax3(v[0], v[1], v[2]), b = fmax3(v[3], v[4], v[5]), c = fmax3(v[6], v[7], v[8]),
        d = fmax3(v[9], v[10], v[11]);
#pragma unroll
  for (int i = 12; i < 60; i += 8) {
    a = fmax3(a, v[i], v[i + 1]);
    b = fmax3(b, v[i + 2], v[i + 3]);
    c = fmax3(c, v[i + 4], v[i + 5]);
    d = fmax3(d, v[i + 6], v[i + 7]);
  }
  a = fmax3(a, v[60], v[61]);
  b = fmax3(b, v[62], v[63]);
  return fmax3(fmaxf(a, b), c, d);
}

QI_DEV void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 32 output columns of one row as bf16: a * norm, or (a*wa + b*wb) * norm
// when a second half b is given (lower-key half first).
QI_DEV void store_out_row(__nv_bfloat16* dst, const float* a, float norm, const float* b, float wa, float wb) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float x0 = a[2 * i], x1 = a[2 * i + 1];
    if (b) {
      x0 = __fadd_rn(__fmul_rn(x0, wa), __fmul_rn(b[2 * i], wb));
      x1 = __fadd_rn(__fmul_rn(x1, wa), __fmul_rn(b[2 * i + 1], wb));
    }
    __nv_bfloat162 h2 = __floats2bfloat162_rn(x0 * norm, x1 * norm);
    w[i] = *reinterpret_cast<uint32_t*>(&h2);
  }
  uint4* o = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

// Roles.  f16 kernel (PAGED = false, 10 warps): warp 0 TMA producer, warp 1
// TMEM allocator + MMA thread, warps 2..9 softmax.  Paged kernel (16 warps =
// 4 warpgroups, one warp of each per SM sub-partition): warpgroup 0 the KV
// producers (thread 0 also loads Q by TMA), warpgroups 1 and 2 the softmax of
// the two query tiles, warp 12 the TMEM allocator + MMA thread (warps 13..15
// idle).  The launch gives every thread 128 registers; setmaxnreg then moves
// them to the softmax: producers 120, warpgroup 3 72, softmax 160 (per
// sub-partition 120 + 2 x 160 + 72 = 512; per CTA 128 x 120 + 256 x 160 +
// 128 x 72 = 65,536 = 512 x 128).  This split compiles without spills.
template <bool PAGED>
struct Roles {
  static constexpr int kThreads = PAGED ? 512 : 320;
  static constexpr int kSoftFirst = PAGED ? 128 : 64;  // first softmax thread
  static constexpr int kMmaWarp = PAGED ? 12 : 1;
  static constexpr int kProducerWarps = PAGED ? 4 : 1;
};

// Paged producer: one thread handles QPK = HD/32 (key, 32-value quarter)
// items of K and as many of V per key tile (mapping: paged_key / paged_quarter).  A tile's codes and scales are
// loaded into registers one tile ahead; converting them writes f16 K and V
// into the same shared-memory tiles the MMAs read: row kr of 128 bytes per
// 64-value half of D, 16-byte chunks swizzled by kr & 7 (K-major K, MN-major V).
template <int HD>
struct PagedTile {
  static constexpr int QPK = HD / 32;
  uint4 kc[QPK], vc[QPK];
  uint32_t ks[QPK], vs[QPK];
};

// Item i of producer thread t: key i * (128/QPK) + (t / 32) * KPW + t % KPW,
// quarter (t % 32) / KPW, KPW = 32/QPK keys per warp and pass.  Consecutive
// lanes take consecutive keys, so each quarter-warp's eight 16-byte shared
// stores land on eight different swizzle positions (no bank conflict), and a
// warp's loads still cover whole 64-byte key rows.
template <int HD>
QI_DEV int paged_key(int i, int t) {
  constexpr int QPK = HD / 32, KPW = 32 / QPK;
  return i * (128 / QPK) + (t >> 5) * KPW + (t & 31) % KPW;
}
template <int HD>
QI_DEV int paged_quarter(int t) {
  constexpr int KPW = 32 / (HD / 32);
  return (t & 31) / KPW;
}

template <int HD>
QI_DEV void paged_fetch(const AttnParams& p, int kvh, int kbase, int t, PagedTile<HD>& b) {
  constexpr int QPK = HD / 32;
  const int qd = paged_quarter<HD>(t);
  const int page_mask = (1 << p.page_shift) - 1;
#pragma unroll
  for (int i = 0; i < QPK; ++i) {
    const int token = kbase + paged_key<HD>(i, t);
    if (token < p.kv_tokens) {
      const int64_t page = __ldg(p.block_table + (token >> p.page_shift)), entry = token & page_mask;
      const int64_t dofs = page * p.data_page + entry * p.data_row + (int64_t)kvh * p.data_head + qd * 16;
      const int64_t sofs = page * p.sf_page + entry * p.sf_row + (int64_t)kvh * p.sf_head + qd * 2;
      b.kc[i] = __ldg(reinterpret_cast<const uint4*>(p.kc + dofs));
      b.vc[i] = __ldg(reinterpret_cast<const uint4*>(p.vc + dofs));
      b.ks[i] = __ldg(reinterpret_cast<const unsigned short*>(p.ksf + sofs));
      b.vs[i] = __ldg(reinterpret_cast<const unsigned short*>(p.vsf + sofs));
    } else {
      b.kc[i] = b.vc[i] = make_uint4(0, 0, 0, 0);
      b.ks[i] = b.vs[i] = 0;
    }
  }
}

// e2m1 x e4m3 -> f16 (exact) into a [D/64][128 keys][128 B] swizzled tile.
template <int HD>
QI_DEV void paged_put(const uint4* codes, const uint32_t* scales, uint8_t* tile, int t) {
  constexpr int QPK = HD / 32;
  const int qd = paged_quarter<HD>(t);
#pragma unroll
  for (int i = 0; i < QPK; ++i) {
    const int kr = paged_key<HD>(i, t);
    const uint32_t s2 = e4m3x2_to_f16x2(scales[i] & 0xFFFFu);
    const uint32_t words[4] = {codes[i].x, codes[i].y, codes[i].z, codes[i].w};
    uint8_t* row = tile + (qd >> 1) * (128 * 128) + kr * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // 16-byte output chunk c: elements 8c .. 8c+7 of the quarter
      uint32_t f[4];
      e2m1x8_to_f16x8(words[c], f);
      const uint32_t sc = splat_half(s2, c >> 1);
      const int chunk = ((qd & 1) * 4 + c) ^ (kr & 7);
      *reinterpret_cast<uint4*>(row + chunk * 16) =
          make_uint4(hmul2u(f[0], sc), hmul2u(f[1], sc), hmul2u(f[2], sc), hmul2u(f[3], sc));
    }
  }
}

template <int HD, bool PAGED>
__global__ void __launch_bounds__(Roles<PAGED>::kThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, AttnParams p) {
  using G = Geometry<HD>;
  using R = Roles<PAGED>;
  constexpr int Q_TILE = G::Q_TILE, K_BYTES = G::K_BYTES, V_BYTES = G::V_BYTES, V_ATOM = G::V_ATOM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;              // NQ tiles
  uint8_t* sK = sQ + NQ * Q_TILE;  // 2 stages
  uint8_t* sV = sK + 2 * K_BYTES;  // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * V_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* q_ready = bars + 1;
  uint64_t* k_full = bars + 2;    // [2]
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [NQ]
  uint64_t* p_full = bars + 12;   // [NQ]
  uint64_t* pv_done = bars + 14;  // [NQ]
  uint64_t* p_half = bars + 16;   // [NQ] P of keys 0..63 of the tile stored
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bid = blockIdx.x;
  // Unit = (query block, head); units run heaviest (latest query block) first.
  // CTAs from split_first on take one half of the key tiles of a split unit.
  const int slot = bid < p.split_first ? -1 : (bid - p.split_first) >> 1;
  const int piece = bid < p.split_first ? -1 : (bid - p.split_first) & 1;
  const int unit = bid < p.split_first ? bid : p.split_first + slot;
  const int qb = p.q_blocks - 1 - unit / p.qheads;
  const int head = unit % p.qheads;
  const int kvh = head / p.group;
  const int q0 = qb * (NQ * TQ);
  const int last_row = min(q0 + NQ * TQ, p.rows) - 1;
  const int unit_tiles = (p.history + last_row + 1 + TK - 1) / TK;
  const int j_first = piece == 1 ? unit_tiles / 2 : 0;  // first key tile of this CTA
  const int ntiles = piece == 0 ? unit_tiles / 2 : unit_tiles - j_first;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tq);
    if constexpr (!PAGED) {
      prefetch_tensormap(&tk);
      prefetch_tensormap(&tv);
    }
    mbar_init(q_full, 1);
    mbar_init(q_ready, NQ * 4);  // one arrival per softmax warp
    for (int i = 0; i < 2; ++i) {
      // TMA: one expect_tx arrival; paged: one arrival per producer warp
      mbar_init(&k_full[i], R::kProducerWarps);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], R::kProducerWarps);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < NQ; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per softmax warp
      mbar_init(&p_half[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == R::kMmaWarp) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Role bodies (one per kind of warp), dispatched below by warpgroup.
  auto mma_role = [&]() {
    if (lane == 0) {
      // Issue order: S0_0 S1_0 | PV0_0 S0_1 PV1_0 S1_1 | PV0_1 S0_2 ... (each PV
      // in two halves of 64 keys, the first as soon as its P is stored) so that
      // the softmax of one tile overlaps the other tile's PV + S pair.  S_t(j+1)
      // overwrites the TMEM columns that PV_t(j), issued just before it by this
      // thread, reads P_t(j) from; tcgen05.mma operations issued by one thread
      // execute in order, so the read precedes the overwrite.  The commit that
      // signals S_t(j+1) covers PV_t(j) as well, so the softmax may rescale O
      // once it sees S_t(j+1).
      // PV reads V^T K-major (f16 kernel) or V in its natural [key][D] order
      // as an MN-major B operand (paged kernel: instruction-descriptor bit 16).
      constexpr uint32_t idesc_s = idesc_f16(128), idesc_o = idesc_f16(HD) | (PAGED ? (1u << 16) : 0u);
      const uint32_t q_base = smem_u32(sQ);
      bool ok = mbar_wait(q_ready, 0, abort_flag, p.status);
      tc_fence_after();
      auto issue_s = [&](int t, int j) {
        const uint32_t k_base = smem_u32(sK + (j & 1) * K_BYTES);
        const uint32_t d_s = tmem + (t ? G::S_COL1 : G::S_COL0);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM + (kk & 3) * 32;
          mma_bf16(d_s, sdesc_kmajor_sw128(q_base + t * Q_TILE + off), sdesc_kmajor_sw128(k_base + off), idesc_s,
                   kk ? 1u : 0u);
        }
        tc_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j, int h) {  // keys 64h .. 64h+63 of the tile
        const uint32_t v_base = smem_u32(sV + (j & 1) * V_BYTES);
        const uint32_t a_p = tmem + (t ? G::S_COL1 : G::S_COL0), d_o = tmem + (t ? G::O_COL1 : G::O_COL0);
#pragma unroll
        for (int kk = 4 * h; kk < 4 * h + 4; ++kk) {
          uint64_t vdesc;
          if constexpr (PAGED) {
            // 16 keys = 16 rows of 128 B; the D halves 16 KB apart; 8-row groups 1 KB apart
            vdesc = sdesc_mnmajor_sw128(v_base + kk * 2048, 128 * 128, 1024);
          } else {
            vdesc = sdesc_kmajor_sw128(v_base + (kk >> 2) * V_ATOM + (kk & 3) * 32);
          }
          mma_f16_ts(d_o, a_p + kk * 8, vdesc, idesc_o, (j | kk) ? 1u : 0u);
        }
      };
      if (ok && (ok = mbar_wait(&k_full[0], 0, abort_flag, p.status))) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        tc_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j & 1;
        const bool more = j + 1 < ntiles;
        if (!(ok = mbar_wait(&v_full[s], (j >> 1) & 1, abort_flag, p.status))) break;
        if (more && !(ok = mbar_wait(&k_full[s ^ 1], ((j + 1) >> 1) & 1, abort_flag, p.status))) break;
        if (!(ok = mbar_wait(&p_half[0], j & 1, abort_flag, p.status))) break;
        tc_fence_after();
        issue_pv(0, j, 0);
        if (!(ok = mbar_wait(&p_full[0], j & 1, abort_flag, p.status))) break;
        tc_fence_after();
        issue_pv(0, j, 1);
        if (more) issue_s(0, j + 1);
        if (!(ok = mbar_wait(&p_half[1], j & 1, abort_flag, p.status))) break;
        tc_fence_after();
        issue_pv(1, j, 0);
        if (!(ok = mbar_wait(&p_full[1], j & 1, abort_flag, p.status))) break;
        tc_fence_after();
        issue_pv(1, j, 1);
        tc_commit(&v_empty[s]);
        if (more) {
          issue_s(1, j + 1);
          tc_commit(&k_empty[s ^ 1]);
        }
      }
      if (ok) {
        tc_commit(&pv_done[0]);
        tc_commit(&pv_done[1]);
      }
    }
  };
  auto softmax_role = [&]() {
    const int t = (warp - R::kSoftFirst / 32) >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;       // TMEM lane quarter
    const int r = quarter * 32 + lane;  // row within the tile == TMEM lane
    const int qrow = q0 + t * TQ + r;
    const int qpos = p.history + qrow;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_addr = lane_base + (t ? G::S_COL1 : G::S_COL0);
    const uint32_t o_addr = lane_base + (t ? G::O_COL1 : G::O_COL0);
    // Convert this warpgroup's Q tile from bf16 to f16 in place (layout unchanged).
    bool ok = mbar_wait(q_full, 0, abort_flag, p.status);
    if (ok) {
      uint4* q4 = reinterpret_cast<uint4*>(sQ + t * Q_TILE);
      for (int i = (int)threadIdx.x - R::kSoftFirst - t * 128; i < Q_TILE / 16; i += 128) {
        uint4 v = q4[i];
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[e]));
          w[e] = pack_f16x2(f.x, f.y);
        }
        q4[i] = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_ready);
    const float scale2 = __fmul_rn(__fmul_rn(p.softmax_scale, *p.k_global), 1.4426950408889634f);
    float m_used = -INFINITY, l_run = 0.0f;
    for (int j = 0; ok && j < ntiles; ++j) {
      ok = mbar_wait(&s_full[t], j & 1, abort_flag, p.status);
      if (!ok) break;
      tc_fence_after();
      // Two passes over S in TMEM (64 columns at a time) keep the live
      // registers low: pass 1 finds the row max, pass 2 forms P = 2^(s*scale2 - m)
      // and writes it back as f16 pairs over the columns just read.
      const int kbase = (j_first + j) * TK;
      const bool diagonal = kbase + TK - 1 > qpos;
      float mx = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float sv[64];
        __syncwarp();
        tmem_ld32_nowait(s_addr + h * 64, sv);
        tmem_ld32_nowait(s_addr + h * 64 + 32, sv + 32);
        tmem_wait_ld();
        if (diagonal) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (kbase + h * 64 + c > qpos) sv[c] = -INFINITY;
        }
        mx = fmaxf(mx, max64(sv));
      }
      const float m_tile = mx * scale2;
      float corr = 1.0f;
      bool rescale = false;
      if (m_used == -INFINITY) {
        // First tile with a visible key for this row (key 0 is visible to every
        // row; in the upper half of a split unit a row may see no key at all
        // for a while, and then m_used stays -inf and P stays 0).
        m_used = m_tile;
      } else if (m_tile > m_used + kRescaleThreshold) {
        corr = ex2_f32(m_used - m_tile);
        m_used = m_tile;
        rescale = true;
      }
      // PV_t of the previous key tile has completed (the commit that signalled
      // this S_t covers it), so O may be rescaled -- before the first half of
      // P is published, since PV_t(j) starts on it.
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float ov[32];
          tmem_ld32(o_addr + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= corr;
          tmem_st32(o_addr + c * 32, ov);
        }
      }
      const float m_sub = m_used == -INFINITY ? 0.0f : m_used;
      const float2 sc2 = make_float2(scale2, scale2), nm2 = make_float2(-m_sub, -m_sub);
      float2 acc = make_float2(0.0f, 0.0f), acc_b = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float sv[64];
        uint32_t pw[32];
        __syncwarp();
        tmem_ld32_nowait(s_addr + h * 64, sv);
        tmem_ld32_nowait(s_addr + h * 64 + 32, sv + 32);
        tmem_wait_ld();
        if (diagonal) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (kbase + h * 64 + c > qpos) sv[c] = -INFINITY;
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float2 d = ffma2(make_float2(sv[2 * c], sv[2 * c + 1]), sc2, nm2);
          // All exponentials on MUFU: the softmax is latency-bound here, and
          // moving a share to an FMA-pipe polynomial (Cody-Waite split plus a
          // cubic) measured slower at every share tried (1/8 .. 1/2).
          const float2 e = make_float2(ex2_f32(d.x), ex2_f32(d.y));
          if (c & 1) acc_b = fadd2(acc_b, e); else acc = fadd2(acc, e);
          pw[c] = pack_f16x2(e.x, e.y);
        }
        // P for keys [64h, 64h+64) -> S columns [32h, 32h+32); pass 2 of the
        // second half reads columns 64..127, which this store does not touch.
        tmem_st32u(s_addr + h * 32, pw);
        // Publish each half as soon as it is stored: the MMA thread runs the
        // PV of keys 0..63 while the second half is being computed.
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(h == 0 ? &p_half[t] : &p_full[t]);
      }
      const float sum = (acc.x + acc.y) + (acc_b.x + acc_b.y);
      l_run = l_run * corr + sum;
    }
    if (ok) ok = mbar_wait(&pv_done[t], 0, abort_flag, p.status);
    tc_fence_after();
    const int prow = t * TQ + r;  // row within the unit
    __nv_bfloat16* orow = p.out + (int64_t)qrow * p.out_row + (int64_t)head * HD;
    if (piece < 0) {
      if (ok) {
        const float norm = __fdiv_rn(*p.v_global, l_run);
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float ov[32];
          __syncwarp();
          tmem_ld32(o_addr + c * 32, ov);
          if (qrow < p.rows) store_out_row(orow + c * 32, ov, norm, nullptr, 0.0f, 0.0f);
        }
      }
    } else {
      // Split unit: publish this half's (m, l, O), then the CTA that arrives
      // second combines both halves (its own from TMEM, the other's from the
      // workspace).  No CTA waits for another.  Both pieces always arrive,
      // so the counter's parity stays right even after an aborted launch.
      float* my_o = p.ws_o + ((int64_t)(slot * 2 + piece) * NQ * TQ + prow) * HD;
      float* my_ml = p.ws_ml + ((int64_t)(slot * 2 + piece) * NQ * TQ + prow) * 2;
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float ov[32];
          __syncwarp();
          tmem_ld32(o_addr + c * 32, ov);
          float4* dst = reinterpret_cast<float4*>(my_o + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) __stcg(dst + i, make_float4(ov[4 * i], ov[4 * i + 1], ov[4 * i + 2], ov[4 * i + 3]));
        }
        __stcg(reinterpret_cast<float2*>(my_ml), make_float2(m_used, l_run));
      }
      __threadfence();
      named_bar_sync(1, NQ * TQ);
      volatile int* last_flag = abort_flag + 1;
      if (threadIdx.x == R::kSoftFirst) {
        const unsigned old = atomicAdd(p.ws_count + slot, 1u);
        __threadfence();
        *last_flag = (int)(old & 1u);
      }
      named_bar_sync(1, NQ * TQ);
      if (*last_flag && ok) {
        const int other = piece ^ 1;
        const float* ot_o = p.ws_o + ((int64_t)(slot * 2 + other) * NQ * TQ + prow) * HD;
        const float2 ot_ml = __ldcg(reinterpret_cast<const float2*>(p.ws_ml + ((int64_t)(slot * 2 + other) * NQ * TQ + prow) * 2));
        // Combine in piece order (lower keys first) whichever CTA is last.
        const float m0 = piece == 0 ? m_used : ot_ml.x, m1 = piece == 0 ? ot_ml.x : m_used;
        const float l0 = piece == 0 ? l_run : ot_ml.y, l1 = piece == 0 ? ot_ml.y : l_run;
        const float mm = fmaxf(m0, m1);
        const float w0 = m0 == -INFINITY ? 0.0f : ex2_f32(m0 - mm);
        const float w1 = m1 == -INFINITY ? 0.0f : ex2_f32(m1 - mm);
        const float norm = __fdiv_rn(*p.v_global, __fadd_rn(__fmul_rn(l0, w0), __fmul_rn(l1, w1)));
        const float w_own = piece == 0 ? w0 : w1, w_other = piece == 0 ? w1 : w0;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float ov[32], xv[32];
          __syncwarp();
          tmem_ld32(o_addr + c * 32, ov);
          const float4* src = reinterpret_cast<const float4*>(ot_o + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 v = __ldcg(src + i);
            xv[4 * i] = v.x, xv[4 * i + 1] = v.y, xv[4 * i + 2] = v.z, xv[4 * i + 3] = v.w;
          }
          if (qrow < p.rows) {
            if (piece == 0)
              store_out_row(orow + c * 32, ov, norm, xv, w_own, w_other);
            else
              store_out_row(orow + c * 32, xv, norm, ov, w_other, w_own);
          }
        }
      }
    }
  };
  if constexpr (PAGED) {
    if (warp < 4) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 120;");
      const int t = threadIdx.x;  // 0 .. 127
      if (t == 0) {
        mbar_expect_tx(q_full, NQ * Q_TILE);
  #pragma unroll
        for (int qt = 0; qt < NQ; ++qt)
  #pragma unroll
          for (int a = 0; a < HD / 64; ++a)
            tma_load_2d(sQ + qt * Q_TILE + a * ATOM, &tq, q_full, head * HD + 64 * a, q0 + qt * TQ);
      }
      // Tile j: wait until the MMAs that read stage j & 1 two tiles ago are
      // done, convert, make the generic-proxy writes visible to the tensor
      // cores, then one arrival per warp.  Tile j + 1 is loaded first.
      auto step = [&](PagedTile<HD>& cur, PagedTile<HD>& nxt, int j) -> bool {
        if (j + 1 < ntiles) paged_fetch<HD>(p, kvh, (j_first + j + 1) * TK, t, nxt);
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status)) return false;
        paged_put<HD>(cur.kc, cur.ks, sK + s * K_BYTES, t);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&k_full[s]);
        if (j >= 2 && !mbar_wait(&v_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status)) return false;
        paged_put<HD>(cur.vc, cur.vs, sV + s * V_BYTES, t);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&v_full[s]);
        return true;
      };
      PagedTile<HD> ta, tb;
      if (ntiles > 0) paged_fetch<HD>(p, kvh, j_first * TK, t, ta);
      for (int j = 0; j < ntiles; j += 2) {
        if (!step(ta, tb, j)) break;
        if (j + 1 < ntiles && !step(tb, ta, j + 1)) break;
      }
    } else if (warp >= 12) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 72;");
      if (warp == 12) mma_role();  // warps 13..15 only take part in the CTA barriers
    } else {
      asm volatile("setmaxnreg.inc.sync.aligned.u32 160;");
      softmax_role();
    }
  } else {
    if (warp == 0) {
      if (lane == 0) {
        mbar_expect_tx(q_full, NQ * Q_TILE);
  #pragma unroll
        for (int t = 0; t < NQ; ++t)
  #pragma unroll
          for (int a = 0; a < HD / 64; ++a)
            tma_load_2d(sQ + t * Q_TILE + a * ATOM, &tq, q_full, head * HD + 64 * a, q0 + t * TQ);
        for (int j = 0; j < ntiles; ++j) {
          const int s = j & 1;
          if (j >= 2 && !mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status)) break;
          mbar_expect_tx(&k_full[s], K_BYTES);
  #pragma unroll
          for (int a = 0; a < HD / 64; ++a)
            tma_load_3d(sK + s * K_BYTES + a * ATOM, &tk, &k_full[s], 64 * a, (j_first + j) * TK, kvh);
          if (j >= 2 && !mbar_wait(&v_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status)) break;
          mbar_expect_tx(&v_full[s], V_BYTES);
          tma_load_3d(sV + s * V_BYTES, &tv, &v_full[s], (j_first + j) * TK, 0, kvh);
          tma_load_3d(sV + s * V_BYTES + V_ATOM, &tv, &v_full[s], (j_first + j) * TK + 64, 0, kvh);
        }
      }
    } else if (warp == 1) {
      mma_role();
    } else {
      softmax_role();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == R::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 16-bit tensor with up to 3 dims; box {64 (128 B), box1, 1}, 128-byte swizzle.
bool make_map16(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, uint32_t box1) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[3], s[2];
  cuuint32_t box[3] = {64, box1, 1}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) d[i] = dims[i];
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  return fn(map, type, rank, const_cast<void*>(base), d, s, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int sm_count(int dev) {
  static int sms[64] = {};
  if (!sms[dev]) {
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count < 1) return 0;
    sms[dev] = count;
  }
  return sms[dev];
}

// How many of the lightest units to split into two key-range halves.  One CTA
// per SM (the kernel holds all 512 TMEM columns), so `units` CTAs run in
// ceil(units / sms) waves and the last wave is partly idle; splitting that
// wave's units in two halves its length.  With fewer units than SMs, split as
// many as there are idle SMs.  Every split unit needs >= 2 key tiles.
// split_plan never splits more than half the SM count.
int max_split_slots(int sms) { return sms / 2; }

// Short units are not split: below kMinSplitTiles key tiles the second CTA's
// fixed cost (Q load, first QK^T, the combine) outweighs the shorter wave.
constexpr int kMinSplitTiles = 24;

int split_plan(int units, int sms, int lightest_tiles, int slots_available) {
  if (sms < 1 || lightest_tiles < kMinSplitTiles) return 0;
  int k = 0;
  if (units < sms) {
    k = units < sms - units ? units : sms - units;
  } else {
    const int r = units % sms;
    if (r > 0 && r <= sms / 2) k = r;
  }
  return k < slots_available ? k : slots_available;
}

// Key-range split plan, workspace carve-up and launch, shared by both kernels.
template <int HD, bool PAGED>
int run_attention(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, AttnParams p,
                  void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  static bool configured[64] = {};
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  if (cur_dev < 0 || cur_dev >= 64) return (int)cudaErrorInvalidDevice;
  const int sms = sm_count(cur_dev);
  if (!configured[cur_dev]) {
    const cudaError_t e = cudaFuncSetAttribute(attn_kernel<HD, PAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               Geometry<HD>::SMEM);
    if (e != cudaSuccess) return (int)e;
    configured[cur_dev] = true;
  }
  p.q_blocks = (p.rows + NQ * TQ - 1) / (NQ * TQ);
  const int units = p.q_blocks * p.qheads;
  int slots_available = 0;
  if (workspace && workspace_bytes > 0) {
    int lo = 0, hi = units < kMaxSlots ? units : kMaxSlots;  // largest slot count whose workspace fits
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (ws_bytes(mid, HD) <= workspace_bytes) lo = mid; else hi = mid - 1;
    }
    slots_available = lo;
  }
  const int lightest_tiles = (p.history + (p.rows < NQ * TQ ? p.rows : NQ * TQ) + TK - 1) / TK;
  const int split = split_plan(units, sms, lightest_tiles, slots_available);
  p.split_first = units - split;
  if (split) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    p.ws_count = reinterpret_cast<unsigned*>(ws);
    p.ws_ml = reinterpret_cast<float*>(ws + ws_count_bytes(split));
    p.ws_o = reinterpret_cast<float*>(ws + ws_count_bytes(split) + ws_ml_bytes(split));
  }
  attn_kernel<HD, PAGED><<<units + split, Roles<PAGED>::kThreads, Geometry<HD>::SMEM, stream>>>(mq, mk, mv, p);
  return (int)cudaPeekAtLastError();
}

template <int HD>
bool make_q_map(CUtensorMap* mq, const void* q, int64_t q_row, int rows) {
  const uint64_t qd[2] = {(uint64_t)q_row, (uint64_t)rows};
  const uint64_t qs[1] = {(uint64_t)q_row * 2};
  return make_map16(mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, 2, qd, qs, 128);
}

template <int HD>
int launch_attention(const QiAttention* a, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  const uint64_t kd[3] = {(uint64_t)HD, (uint64_t)a->kv_tokens, (uint64_t)a->kvheads};
  const uint64_t ks[2] = {(uint64_t)HD * 2, (uint64_t)a->kv_tokens * HD * 2};
  const uint64_t vd[3] = {(uint64_t)a->kv_tokens, (uint64_t)HD, (uint64_t)a->kvheads};
  const uint64_t vs[2] = {(uint64_t)a->vt_row * 2, (uint64_t)a->vt_row * HD * 2};
  if (!make_q_map<HD>(&mq, a->q, a->q_row, a->rows) ||
      !make_map16(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a->k, 3, kd, ks, 128) ||
      !make_map16(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a->vt, 3, vd, vs, HD))
    return (int)cudaErrorInvalidValue;
  AttnParams p{};
  p.rows = a->rows;
  p.history = a->history;
  p.kv_tokens = a->kv_tokens;
  p.qheads = a->qheads;
  p.group = a->qheads / a->kvheads;
  p.out_row = a->out_row;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.k_global = a->k_global;
  p.v_global = a->v_global;
  p.softmax_scale = a->softmax_scale;
  p.status = a->status;
  return run_attention<HD, false>(mq, mk, mv, p, a->workspace, a->workspace_bytes, stream);
}

template <int HD>
int launch_paged_attention(const QiPagedAttention* a, cudaStream_t stream) {
  CUtensorMap mq;
  CUtensorMap unused{};
  if (!make_q_map<HD>(&mq, a->q, a->q_row, a->rows)) return (int)cudaErrorInvalidValue;
  const QiKvView& kv = a->kv;
  AttnParams p{};
  p.rows = a->rows;
  p.history = a->history;
  p.kv_tokens = a->history + a->rows;
  p.qheads = a->qheads;
  p.group = a->qheads / kv.kvheads;
  p.out_row = a->out_row;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.k_global = a->k_global;
  p.v_global = a->v_global;
  p.softmax_scale = a->softmax_scale;
  p.status = a->status;
  p.kc = static_cast<const uint8_t*>(kv.k_cache);
  p.vc = static_cast<const uint8_t*>(kv.v_cache);
  p.ksf = static_cast<const uint8_t*>(kv.k_scales);
  p.vsf = static_cast<const uint8_t*>(kv.v_scales);
  p.block_table = a->block_table;
  p.page_shift = __builtin_ctz((unsigned)kv.page_size);
  p.data_page = kv.data_page;
  p.data_row = kv.data_row;
  p.data_head = kv.data_head;
  p.sf_page = kv.sf_page;
  p.sf_row = kv.sf_row;
  p.sf_head = kv.sf_head;
  return run_attention<HD, true>(mq, unused, unused, p, a->workspace, a->workspace_bytes, stream);
}

}  // namespace

namespace qi {
bool attention_request_valid(const QiAttention* a) {
  if (!a || a->rows < 1 || a->history < 0 || (a->head_dim != 64 && a->head_dim != 128) || a->qheads < 1 ||
      a->kvheads < 1 || a->qheads % a->kvheads || !a->q || !a->k || !a->vt || !a->out || !a->k_global ||
      !a->v_global)
    return false;
  const int64_t hd = a->head_dim;
  if (a->kv_tokens < a->history + a->rows || a->vt_row < a->kv_tokens || a->vt_row % 8 || a->q_row % 8 ||
      a->out_row % 8 || a->q_row < a->qheads * hd || a->out_row < a->qheads * hd)
    return false;
  return aligned16(a->q) && aligned16(a->k) && aligned16(a->vt) && aligned16(a->out) &&
         !(a->workspace && (reinterpret_cast<uintptr_t>(a->workspace) & 255));
}
bool paged_attention_request_valid(const QiPagedAttention* a) {
  if (!a || a->rows < 1 || a->history < 0 || a->qheads < 1 || !a->q || !a->out || !a->block_table ||
      !a->k_global || !a->v_global)
    return false;
  const QiKvView& kv = a->kv;
  if ((kv.head_dim != 64 && kv.head_dim != 128) || kv.kvheads < 1 || a->qheads % kv.kvheads || kv.page_size < 1 ||
      (kv.page_size & (kv.page_size - 1)) || !kv.k_cache || !kv.v_cache || !kv.k_scales || !kv.v_scales)
    return false;
  const int64_t hd = kv.head_dim;
  if ((int64_t)a->history + a->rows > (int64_t)1 << 30 || a->q_row % 8 || a->out_row % 8 ||
      a->q_row < a->qheads * hd || a->out_row < a->qheads * hd)
    return false;
  // 16-byte code loads and 2-byte scale loads per 32 values of a key
  return aligned16(a->q) && aligned16(a->out) && aligned16(kv.k_cache) && aligned16(kv.v_cache) &&
         !(kv.data_page % 16) && !(kv.data_row % 16) && !(kv.data_head % 16) &&
         !(reinterpret_cast<uintptr_t>(kv.k_scales) & 1) && !(reinterpret_cast<uintptr_t>(kv.v_scales) & 1) &&
         !(kv.sf_page % 2) && !(kv.sf_row % 2) && !(kv.sf_head % 2) &&
         !(a->workspace && (reinterpret_cast<uintptr_t>(a->workspace) & 255));
}
}  // namespace qi

extern "C" int qi_prefill_attention(const QiAttention* a, cudaStream_t stream) {
  QI_BIND(stream, a ? a->q : nullptr);
  if (!attention_request_valid(a)) return (int)cudaErrorInvalidValue;
  return a->head_dim == 64 ? launch_attention<64>(a, stream) : launch_attention<128>(a, stream);
}

extern "C" int qi_paged_prefill_attention(const QiPagedAttention* a, cudaStream_t stream) {
  QI_BIND(stream, a ? a->q : nullptr);
  if (!paged_attention_request_valid(a)) return (int)cudaErrorInvalidValue;
  return a->kv.head_dim == 64 ? launch_paged_attention<64>(a, stream) : launch_paged_attention<128>(a, stream);
}

extern "C" int qi_prefill_attention_workspace_bytes(int head_dim, int64_t* bytes) {
  if (!bytes || (head_dim != 64 && head_dim != 128)) return (int)cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
  const int sms = sm_count(dev);
  if (!sms) return (int)cudaErrorInvalidDevice;
  *bytes = ws_bytes(max_split_slots(sms), head_dim);
  return 0;
}
