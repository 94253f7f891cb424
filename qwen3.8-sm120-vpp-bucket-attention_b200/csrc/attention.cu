// Chunked causal GQA prefill attention on tcgen05 (sm_100a), bf16 operands,
// fp32 accumulators in tensor memory and an fp32 online softmax.
//
// Input K / V^T come from the paged NVFP4 cache through qi_kv_dequant (values
// e2m1 * e4m3, exact in bf16); the fp32 global multipliers of K and V are
// folded into the softmax scale and the output normalisation.
//
// One CTA = 128 query rows of one query head; 6 warps:
//   warp 0     : TMA producer (Q once; K and V^T tiles of 128 keys, 2 stages),
//   warp 1     : TMEM allocator + single MMA thread: S_j = Q K_j^T into one of
//                two S buffers, O += P_{j-1} V_{j-1} (P from shared memory),
//   warps 2..5 : softmax, one query row per thread (TMEM lane): online max /
//                sum, O rescale in TMEM, P written to smem in the 128-byte
//                swizzled K-major layout the MMA reads; final O / l epilogue.
// S_{j+1} is computed by the tensor cores while the softmax works on S_j.
#include <mutex>

#include "common.cuh"
#include "qwen_infra_b200.h"

using namespace qi;

namespace {

constexpr int TQ = 128, TK = 128;
constexpr int ATOM = 128 * 128;  // one 128-row x 128-byte swizzle column (16 KB)
constexpr uint32_t S_COL0 = 0, S_COL1 = 128, O_COL = 256, TMEM_COLS = 512;

template <int HD>
struct Geometry {
  static constexpr int Q_BYTES = (HD / 64) * ATOM;  // HD/64 columns of [128 rows x 128 B]
  static constexpr int K_BYTES = (HD / 64) * ATOM;
  static constexpr int V_ATOM = HD * 128;  // one 64-key column of V^T: [HD rows x 128 B]
  static constexpr int V_BYTES = 2 * V_ATOM;
  static constexpr int P_BYTES = 2 * ATOM;
  static constexpr int SMEM = Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + P_BYTES + 1024 + 256;
};

struct AttnParams {
  int rows, history, kv_tokens, qheads, group;
  int64_t out_row;
  __nv_bfloat16* out;
  const float* k_global;
  const float* v_global;
  float softmax_scale;
  int* status;
  int q_tiles;
};

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, AttnParams p) {
  using G = Geometry<HD>;
  constexpr int Q_BYTES = G::Q_BYTES, K_BYTES = G::K_BYTES, V_BYTES = G::V_BYTES, P_BYTES = G::P_BYTES;
  constexpr int V_ATOM = G::V_ATOM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;
  uint8_t* sV = sK + 2 * K_BYTES;
  uint8_t* sP = sV + 2 * V_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* o_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bid = blockIdx.x;
  const int qt = p.q_tiles - 1 - bid / p.qheads;  // heaviest (latest) query tiles first
  const int head = bid % p.qheads;
  const int kvh = head / p.group;
  const int q0 = qt * TQ;
  const int last_row = min(q0 + TQ, p.rows) - 1;
  const int ntiles = (p.history + last_row + 1 + TK - 1) / TK;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tq);
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, Q_BYTES);
#pragma unroll
      for (int a = 0; a < HD / 64; ++a) tma_load_2d(sQ + a * ATOM, &tq, q_full, head * HD + 64 * a, q0);
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status)) break;
        mbar_expect_tx(&k_full[s], K_BYTES);
#pragma unroll
        for (int a = 0; a < HD / 64; ++a) tma_load_3d(sK + s * K_BYTES + a * ATOM, &tk, &k_full[s], 64 * a, j * TK, kvh);
        if (j >= 2 && !mbar_wait(&v_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status)) break;
        mbar_expect_tx(&v_full[s], V_BYTES);
        tma_load_3d(sV + s * V_BYTES, &tv, &v_full[s], j * TK, 0, kvh);
        tma_load_3d(sV + s * V_BYTES + V_ATOM, &tv, &v_full[s], j * TK + 64, 0, kvh);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16(128), idesc_o = idesc_bf16(HD);
      const uint32_t q_base = smem_u32(sQ), p_base = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          const int s = j & 1;
          if (!(ok = mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t k_base = smem_u32(sK + s * K_BYTES);
          const uint32_t d_s = tmem + (s ? S_COL1 : S_COL0);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * ATOM + (kk & 3) * 32;
            mma_bf16(d_s, sdesc_kmajor_sw128(q_base + off), sdesc_kmajor_sw128(k_base + off), idesc_s, kk ? 1u : 0u);
          }
          tc_commit(&s_full[s]);
          tc_commit(&k_empty[s]);
        }
        if (j >= 1) {
          const int jp = j - 1, s = jp & 1;
          if (!(ok = mbar_wait(p_full, jp & 1, abort_flag, p.status))) break;
          if (!(ok = mbar_wait(&v_full[s], (jp >> 1) & 1, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t v_base = smem_u32(sV + s * V_BYTES);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t poff = (kk >> 2) * ATOM + (kk & 3) * 32, voff = (kk >> 2) * V_ATOM + (kk & 3) * 32;
            mma_bf16(tmem + O_COL, sdesc_kmajor_sw128(p_base + poff), sdesc_kmajor_sw128(v_base + voff), idesc_o,
                     (jp | kk) ? 1u : 0u);
          }
          tc_commit(o_done);
          tc_commit(&v_empty[s]);
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile == TMEM lane
    const int qpos = p.history + q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float scale2 = __fmul_rn(__fmul_rn(p.softmax_scale, *p.k_global), 1.4426950408889634f);
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    uint8_t* prow = sP + r * 128;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      ok = mbar_wait(&s_full[s], (j >> 1) & 1, abort_flag, p.status);
      if (!ok) break;
      tc_fence_after();
      float sv[128];
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_base + (s ? S_COL1 : S_COL0) + c * 32, sv + c * 32);
      const int kbase = j * TK;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const float x = (kbase + c <= qpos) ? sv[c] * scale2 : -INFINITY;
        sv[c] = x;
        mx = fmaxf(mx, x);
      }
      const float m_new = fmaxf(m_run, mx);
      const float corr = (m_run == -INFINITY) ? 0.0f : exp2f(m_run - m_new);
      float sum = 0.0f;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const float e = (sv[c] == -INFINITY) ? 0.0f : exp2f(sv[c] - m_new);
        sv[c] = e;
        sum += e;
      }
      l_run = l_run * corr + sum;
      m_run = m_new;
      if (j >= 1) {
        // PV_{j-1} must be complete before O is rescaled and P overwritten.
        ok = mbar_wait(o_done, (j - 1) & 1, abort_flag, p.status);
        if (!ok) break;
        tc_fence_after();
        const bool need = __any_sync(0xffffffffu, corr != 1.0f);
        if (need) {
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float ov[32];
            tmem_ld32(lane_base + O_COL + c * 32, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= corr;
            tmem_st32(lane_base + O_COL + c * 32, ov);
          }
        }
      }
      // P row -> smem, 128-byte swizzle: 16-byte chunk c16 of row r lands at c16 ^ (r % 8).
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(sv[ch * 8 + 2 * i], sv[ch * 8 + 2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&h2);
        }
        const int atom = ch >> 3, c16 = ch & 7;
        *reinterpret_cast<uint4*>(prow + atom * ATOM + ((c16 ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) ok = mbar_wait(o_done, (ntiles - 1) & 1, abort_flag, p.status);
    tc_fence_after();
    if (ok) {
      const float norm = __fdiv_rn(*p.v_global, l_run);
      const int qrow = q0 + r;
      __nv_bfloat16* orow = p.out + (int64_t)qrow * p.out_row + (int64_t)head * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        float ov[32];
        __syncwarp();
        tmem_ld32(lane_base + O_COL + c * 32, ov);
        if (qrow < p.rows) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(ov[2 * i] * norm, ov[2 * i + 1] * norm);
            w[i] = *reinterpret_cast<uint32_t*>(&h2);
          }
          uint4* o = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
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

// bf16 tensor with up to 3 dims; box {64 (128 B), box1, 1}, 128-byte swizzle.
bool make_map_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                   uint32_t box1) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[3], s[2];
  cuuint32_t box[3] = {64, box1, 1}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) d[i] = dims[i];
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int HD>
int launch_attention(const QiAttention* a, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  const uint64_t qd[2] = {(uint64_t)a->q_row, (uint64_t)a->rows};
  const uint64_t qs[1] = {(uint64_t)a->q_row * 2};
  const uint64_t kd[3] = {(uint64_t)HD, (uint64_t)a->kv_tokens, (uint64_t)a->kvheads};
  const uint64_t ks[2] = {(uint64_t)HD * 2, (uint64_t)a->kv_tokens * HD * 2};
  const uint64_t vd[3] = {(uint64_t)a->kv_tokens, (uint64_t)HD, (uint64_t)a->kvheads};
  const uint64_t vs[2] = {(uint64_t)a->vt_row * 2, (uint64_t)a->vt_row * HD * 2};
  if (!make_map_bf16(&mq, a->q, 2, qd, qs, 128) || !make_map_bf16(&mk, a->k, 3, kd, ks, 128) ||
      !make_map_bf16(&mv, a->vt, 3, vd, vs, HD))
    return (int)cudaErrorInvalidValue;
  static bool configured[64] = {};
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  if (cur_dev < 0 || cur_dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!configured[cur_dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, Geometry<HD>::SMEM);
    if (e != cudaSuccess) return (int)e;
    configured[cur_dev] = true;
  }
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
  p.q_tiles = (a->rows + TQ - 1) / TQ;
  attn_kernel<HD><<<p.q_tiles * a->qheads, 192, Geometry<HD>::SMEM, stream>>>(mq, mk, mv, p);
  return (int)cudaPeekAtLastError();
}

}  // namespace

extern "C" int qi_prefill_attention(const QiAttention* a, cudaStream_t stream) {
  QI_BIND(stream, a ? a->q : nullptr);
  if (!a || a->rows < 1 || a->history < 0 || (a->head_dim != 64 && a->head_dim != 128) || a->qheads < 1 ||
      a->kvheads < 1 || a->qheads % a->kvheads || !a->q || !a->k || !a->vt || !a->out || !a->k_global ||
      !a->v_global)
    return (int)cudaErrorInvalidValue;
  const int64_t hd = a->head_dim;
  if (a->kv_tokens < a->history + a->rows || a->vt_row < a->kv_tokens || a->vt_row % 8 || a->q_row % 8 ||
      a->out_row % 8 || a->q_row < a->qheads * hd || a->out_row < a->qheads * hd)
    return (int)cudaErrorInvalidValue;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->vt) || !aligned16(a->out)) return (int)cudaErrorInvalidValue;
  return a->head_dim == 64 ? launch_attention<64>(a, stream) : launch_attention<128>(a, stream);
}
