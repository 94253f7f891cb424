// Block-scaled NVFP4 (kind::mxf4nvf4, 16-element E4M3 scales) and E4M3
// (kind::f8f6f4) GEMMs on the 5th-generation tensor cores of sm_100a.
//
//   D[m, n] = sum_k A[m, k] * B[n, k]     (A: activations, B: weights, both K-major)
//
// Persistent, warp-specialised: one CTA per SM walks 128 x 256 output tiles
// (M tiles fastest, so the CTAs in flight share weight tiles through L2 and
// each weight byte is read from HBM about once).
//   warp 0      : TMA producer (A and B tiles, 128-byte swizzle; block scales by
//                 untiled bulk copies of whole 512-byte swizzle atoms) running
//                 ahead across tile boundaries through a 4-stage smem ring,
//   warp 1      : TMEM allocator and the single thread issuing tcgen05.cp (scale
//                 factors smem -> TMEM, own columns per stage) and tcgen05.mma,
//   warps 2..9  : epilogue: two warps per TMEM lane quarter, each reading half
//                 of the tile's columns; the accumulator is released as soon as
//                 it is in registers, so the fused epilogue math and the global
//                 stores overlap the next tile's MMAs.
#include <mutex>

#include "common.cuh"
#include "qwen_infra_b200.h"

using namespace qi;

namespace {

constexpr int BM = 128, BN = 256, BKB = 128;  // K tile: 128 bytes (256 E2M1 or 128 E4M3 values)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKB;
constexpr int B_BYTES = BN * BKB;
constexpr int SFA_BYTES = 2048;  // 128 rows x 16 scales (4 atoms of 512 B)
constexpr int SFB_BYTES = 4096;  // 256 rows x 16 scales
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int THREADS = 320;
constexpr int EPI_THREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
// Scale factors get their own TMEM columns per pipeline stage (16 for A, 32
// for B), so copying the next stage's scales never waits on MMAs that still
// read the previous ones.
constexpr uint32_t ACC_COL = 0, SFA_COL = 256, SFB_COL = 256 + STAGES * 16;

struct Params {
  int m, n, kt;  // kt: number of 128-byte K tiles
  int m_tiles, n_tiles;
  const uint8_t* sfa;
  const uint8_t* sfb;
  int64_t sfa_block, sfb_block;  // bytes per 128-row block of the scale buffers
  const float* alpha;
  float alpha_value;
  const float* row_scale;
  const float* col_scale;
  void* out;
  int64_t ldo;
  uint8_t* act_q;
  uint8_t* act_sf;
  const float* act_global;
  int64_t act_ld;
  int act_gp;  // padded scale groups per row of the SwiGLU output
  int* status;
};

template <bool kFp4, int kEpi>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * SFB_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_THREADS);
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
      const uint32_t tx = A_BYTES + B_BYTES + (kFp4 ? SFA_BYTES + SFB_BYTES : 0);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * BM, n0 = (tile / p.m_tiles) * BN;
        for (int kt = 0; kt < p.kt; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !(ok = mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, abort_flag, p.status))) break;
          mbar_expect_tx(&full[s], tx);
          tma_load_2d(sA + s * A_BYTES, &tma_a, &full[s], kt * BKB, m0);
          tma_load_2d(sB + s * B_BYTES, &tma_b, &full[s], kt * BKB, n0);
          if constexpr (kFp4) {
            bulk_load(sSFA + s * SFA_BYTES, p.sfa + (int64_t)(m0 >> 7) * p.sfa_block + (int64_t)kt * 2048, 2048,
                      &full[s]);
            bulk_load(sSFB + s * SFB_BYTES, p.sfb + (int64_t)(n0 >> 7) * p.sfb_block + (int64_t)kt * 2048, 2048,
                      &full[s]);
            bulk_load(sSFB + s * SFB_BYTES + 2048,
                      p.sfb + (int64_t)((n0 >> 7) + 1) * p.sfb_block + (int64_t)kt * 2048, 2048, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = kFp4 ? idesc_nvfp4(BN) : idesc_e4m3(BN);
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++tcount) {
        // The accumulator is single-buffered: wait until the epilogue holds the
        // previous tile in registers.
        if (tcount > 0 && !(ok = mbar_wait(acc_empty, (tcount - 1) & 1, abort_flag, p.status))) break;
        tc_fence_after();
        for (int kt = 0; kt < p.kt; ++kt, ++it) {
          const int s = it % STAGES;
          if (!(ok = mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * A_BYTES), b_base = smem_u32(sB + s * B_BYTES);
          if constexpr (kFp4) {
            // All of this stage's scale factors first, then its four MMAs.
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t sfa_t = tmem + SFA_COL + s * 16 + kk * 4, sfb_t = tmem + SFB_COL + s * 32 + kk * 8;
              tc_cp_sf(sfa_t, sdesc_sf_atom(smem_u32(sSFA + s * SFA_BYTES + kk * 512)));
              tc_cp_sf(sfb_t, sdesc_sf_atom(smem_u32(sSFB + s * SFB_BYTES + kk * 512)));
              tc_cp_sf(sfb_t + 4, sdesc_sf_atom(smem_u32(sSFB + s * SFB_BYTES + 2048 + kk * 512)));
            }
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adesc = sdesc_kmajor_sw128(a_base + kk * 32);
            const uint64_t bdesc = sdesc_kmajor_sw128(b_base + kk * 32);
            const uint32_t acc = (kt | kk) ? 1u : 0u;
            if constexpr (kFp4) {
              mma_nvfp4(tmem + ACC_COL, adesc, bdesc, idesc, tmem + SFA_COL + s * 16 + kk * 4,
                        tmem + SFB_COL + s * 32 + kk * 8, acc);
            } else {
              mma_f8(tmem + ACC_COL, adesc, bdesc, idesc, acc);
            }
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(acc_full);
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes [32*(w%4), +32) = tile rows; the two
    // warps of a lane quarter split the tile's columns in halves.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float alpha = p.alpha ? *p.alpha : p.alpha_value;
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tcount) {
      const int m0 = (tile % p.m_tiles) * BM, n0 = (tile / p.m_tiles) * BN;
      const int row = m0 + quarter * 32 + lane;
      const bool in_range = row < p.m;
      const bool ok = mbar_wait(acc_full, tcount & 1, abort_flag, p.status);
      tc_fence_after();
      float v[128];
      if (ok) {
        __syncwarp();
        if constexpr (kEpi == QI_EPI_SWIGLU_NVFP4) {
          // gate columns [64h, 64h+64) into v[0..64), up columns [128+64h, ...) into v[64..128)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32(tmem + lane_off + ACC_COL + half * 64 + c * 32, v + c * 32);
            tmem_ld32(tmem + lane_off + ACC_COL + 128 + half * 64 + c * 32, v + 64 + c * 32);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_off + ACC_COL + half * 128 + c * 32, v + c * 32);
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty);  // the accumulator may now take the next tile
      if (!ok) break;
      if (!in_range) continue;
      if constexpr (kEpi == QI_EPI_SWIGLU_NVFP4) {
        const float g = *p.act_global;
        const int64_t gp = p.act_gp;
        const int ch0 = (n0 >> 1) + half * 64;  // first output channel of this thread's half
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float gg = bf16r(__fmul_rn(v[j], alpha));
          const float uu = bf16r(__fmul_rn(v[64 + j], alpha));
          v[j] = bf16r(__fmul_rn(silu_f(gg), uu));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint2 packed;
          const uint32_t code = nvfp4_quant16(v + 16 * q, g, packed);
          const int ch = ch0 + 16 * q;
          *reinterpret_cast<uint2*>(p.act_q + (int64_t)row * p.act_ld + (ch >> 1)) = packed;
          p.act_sf[sf_offset(row, ch >> 4, gp)] = (uint8_t)code;
        }
      } else if constexpr (kEpi == QI_EPI_F32) {
        float* o = static_cast<float*>(p.out) + (int64_t)row * p.ldo + n0 + half * 128;
#pragma unroll
        for (int j = 0; j < 128; j += 4)
          *reinterpret_cast<float4*>(o + j) = make_float4(__fmul_rn(v[j], alpha), __fmul_rn(v[j + 1], alpha),
                                                          __fmul_rn(v[j + 2], alpha), __fmul_rn(v[j + 3], alpha));
      } else {
        const int col0 = n0 + half * 128;
        float rs = 1.0f;
        if constexpr (kEpi == QI_EPI_BF16_ROWCOL) rs = p.row_scale[row];
        uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + col0);
#pragma unroll
        for (int j = 0; j < 128; j += 8) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float a, b;
            if constexpr (kEpi == QI_EPI_BF16_ROWCOL) {
              a = __fmul_rn(__fmul_rn(v[j + 2 * i], rs), p.col_scale[col0 + j + 2 * i]);
              b = __fmul_rn(__fmul_rn(v[j + 2 * i + 1], rs), p.col_scale[col0 + j + 2 * i + 1]);
            } else {
              a = __fmul_rn(v[j + 2 * i], alpha);
              b = __fmul_rn(v[j + 2 * i + 1], alpha);
            }
            __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
            w[i] = *reinterpret_cast<uint32_t*>(&h2);
          }
          o[j / 8] = make_uint4(w[0], w[1], w[2], w[3]);
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

// ---- host side ------------------------------------------------------------

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

// 2-D byte matrix [rows, row_bytes] with a (128 B x box_rows) box, 128-byte swizzle.
bool make_map_u8(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kFp4, int kEpi>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, cudaStream_t stream) {
  static bool configured[64] = {};
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  if (cur_dev < 0 || cur_dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!configured[cur_dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_kernel<kFp4, kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    configured[cur_dev] = true;
  }
  static int sms[64] = {};
  if (!sms[cur_dev]) {
    int count = 0;
    const cudaError_t e = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, cur_dev);
    if (e != cudaSuccess) return (int)e;
    sms[cur_dev] = count;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < sms[cur_dev] ? tiles : sms[cur_dev];
  gemm_kernel<kFp4, kEpi><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
  return (int)cudaPeekAtLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int qi_gemm(const QiGemm* g, cudaStream_t stream) {
  QI_BIND(stream, g ? g->a : nullptr);
  if (!g || g->m < 1 || g->n < BN || g->n % BN || !g->a || !g->b) return (int)cudaErrorInvalidValue;
  const bool fp4 = g->kind == QI_GEMM_NVFP4;
  if (!fp4 && g->kind != QI_GEMM_E4M3) return (int)cudaErrorInvalidValue;
  const int64_t k_bytes = fp4 ? g->k / 2 : g->k;
  if (g->k < 1 || k_bytes % BKB || !aligned16(g->a) || !aligned16(g->b)) return (int)cudaErrorInvalidValue;
  if (fp4 && (!g->sfa || !g->sfb || !aligned16(g->sfa) || !aligned16(g->sfb))) return (int)cudaErrorInvalidValue;
  Params p{};
  p.m = g->m;
  p.n = g->n;
  p.kt = (int)(k_bytes / BKB);
  p.m_tiles = (g->m + BM - 1) / BM;
  p.n_tiles = g->n / BN;
  p.sfa = static_cast<const uint8_t*>(g->sfa);
  p.sfb = static_cast<const uint8_t*>(g->sfb);
  const int64_t gp = ((g->k / 16) + 3) / 4 * 4;
  p.sfa_block = 128 * gp;
  p.sfb_block = 128 * gp;
  p.alpha = g->alpha;
  p.alpha_value = g->alpha_value;
  p.row_scale = g->row_scale;
  p.col_scale = g->col_scale;
  p.out = g->out;
  p.ldo = g->ldo;
  p.act_q = static_cast<uint8_t*>(g->act_q);
  p.act_sf = static_cast<uint8_t*>(g->act_sf);
  p.act_global = g->act_global;
  p.act_ld = g->act_ld;
  p.act_gp = (int)((((g->n / 2) / 16) + 3) / 4 * 4);
  p.status = g->status;
  switch (g->epilogue) {
    case QI_EPI_BF16:
    case QI_EPI_F32:
      if (!g->out || g->ldo < g->n || g->ldo % 8) return (int)cudaErrorInvalidValue;
      break;
    case QI_EPI_BF16_ROWCOL:
      if (!g->out || g->ldo < g->n || g->ldo % 8 || !g->row_scale || !g->col_scale) return (int)cudaErrorInvalidValue;
      break;
    case QI_EPI_SWIGLU_NVFP4:
      if (!g->act_q || !g->act_sf || !g->act_global || g->act_ld < g->n / 4 || g->act_ld % 8)
        return (int)cudaErrorInvalidValue;
      break;
    default:
      return (int)cudaErrorInvalidValue;
  }
  CUtensorMap ma, mb;
  if (!make_map_u8(&ma, g->a, k_bytes, g->m, BM) || !make_map_u8(&mb, g->b, k_bytes, g->n, BN))
    return (int)cudaErrorInvalidValue;
  if (fp4) {
    switch (g->epilogue) {
      case QI_EPI_BF16: return launch<true, QI_EPI_BF16>(ma, mb, p, stream);
      case QI_EPI_F32: return launch<true, QI_EPI_F32>(ma, mb, p, stream);
      case QI_EPI_SWIGLU_NVFP4: return launch<true, QI_EPI_SWIGLU_NVFP4>(ma, mb, p, stream);
      default: return (int)cudaErrorInvalidValue;
    }
  }
  switch (g->epilogue) {
    case QI_EPI_BF16: return launch<false, QI_EPI_BF16>(ma, mb, p, stream);
    case QI_EPI_F32: return launch<false, QI_EPI_F32>(ma, mb, p, stream);
    case QI_EPI_BF16_ROWCOL: return launch<false, QI_EPI_BF16_ROWCOL>(ma, mb, p, stream);
    default: return (int)cudaErrorInvalidValue;
  }
}

int qi_gemm_resources(int* out) {
  if (!out) return (int)cudaErrorInvalidValue;
  cudaFuncAttributes a{};
  const cudaError_t e = cudaFuncGetAttributes(&a, gemm_kernel<true, QI_EPI_BF16>);
  if (e != cudaSuccess) return (int)e;
  out[0] = SMEM_BYTES;
  out[1] = a.numRegs;
  out[2] = THREADS;
  return 0;
}

}  // extern "C"
