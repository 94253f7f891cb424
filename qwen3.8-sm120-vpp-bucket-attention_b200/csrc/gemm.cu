// Block-scaled NVFP4 (kind::mxf4nvf4, 16-element E4M3 scales) and E4M3
// (kind::f8f6f4) GEMMs on the 5th-generation tensor cores of sm_100a.
//
//   D[m, n] = sum_k A[m, k] * B[n, k]     (A: activations, B: weights, both K-major)
//
// All three kernels are persistent and warp-specialised: a CTA (or CTA pair)
// per SM walks the output tiles (M tiles fastest, so the CTAs in flight share
// weight tiles through L2 and each weight byte is read from HBM about once);
// a TMA producer runs ahead across tile boundaries through a shared-memory
// ring; one thread issues tcgen05.mma into a 256-column TMEM accumulator; the
// epilogue warps (two per TMEM lane quarter, each on half of the tile's
// columns) release the accumulator as soon as it is in registers, so the
// fused epilogue math and the global stores overlap the next tile's MMAs.
//   gemm_sfw_kernel   NVFP4, 128 x 256 tiles, block scales written to TMEM by
//                     four scale-writer warps (tcgen05.st), 16 warps;
//   gemm_pair_kernel  E4M3 with M > 128: CTA pairs, 2-SM MMAs, 256 x 256 tiles;
//   gemm_kernel       E4M3 with M <= 128: 128 x 256 tiles, 10 warps.
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
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;  // NVFP4 stage
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int THREADS = 320;     // gemm_kernel and gemm_pair_kernel
constexpr int EPI_THREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_COL = 0;

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

// In-warp transpose of a 32 x 32 matrix of 32-bit words: lane l holds row l
// in x[0..31] on entry and column l (word l of rows 0..31) on exit; five
// butterfly stages of shfl_xor, each exchanging half the words with the lane
// whose bit s differs.
__device__ __forceinline__ void warp_transpose32(uint32_t* x, int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if ((j & s) == 0) {  // compile-time pair (j, j|s); selects keep both in registers
        const uint32_t lo = x[j], hi = x[j | s];
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, upper ? lo : hi, s);
        x[j] = upper ? recv : lo;
        x[j | s] = upper ? hi : recv;
      }
    }
  }
}

// Fused epilogue of one warp's 32 tile rows (row0 .. row0+31, this thread's
// row is row0 + lane): v holds the thread's 128 accumulator columns (half h of
// the 256-column tile starting at n0; for SwiGLU the 64 gate and 64 up
// columns of output channels (n0/2 + 64h ..)).  bf16 outputs leave the warp
// transposed, so that every store instruction writes 128 contiguous bytes of
// one row (a row per thread would make each 16-byte store touch 32 rows:
// measured, those stores cost the NVFP4 GEMM ~20% through the shared L1 /
// shared-memory data path).  Rows at or past p.m are not stored.
template <int kEpi>
__device__ __forceinline__ void epilogue_rows(const Params& p, float* v, int row0, int lane, int n0, int half,
                                              float alpha) {
  const int row = row0 + lane;
  if constexpr (kEpi == QI_EPI_SWIGLU_NVFP4) {
    if (row >= p.m) return;
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
    if (row >= p.m) return;
    float* o = static_cast<float*>(p.out) + (int64_t)row * p.ldo + n0 + half * 128;
#pragma unroll
    for (int j = 0; j < 128; j += 4)
      *reinterpret_cast<float4*>(o + j) = make_float4(__fmul_rn(v[j], alpha), __fmul_rn(v[j + 1], alpha),
                                                      __fmul_rn(v[j + 2], alpha), __fmul_rn(v[j + 3], alpha));
  }
}

// bf16 epilogues: the thread's 128 accumulator columns arrive 32 at a time,
// each block scaled and packed into bf16 pairs at once (so at most 32 fp32
// values and 64 words are live), then the accumulator is released and the
// packed row is stored transposed through the warp.
template <int kEpi>
__device__ __forceinline__ void pack_bf16_block(const Params& p, const float* v, uint32_t* w, int row, int col0,
                                                int c0, float alpha) {
  float rs = 1.0f;
  if constexpr (kEpi == QI_EPI_BF16_ROWCOL) rs = row < p.m ? p.row_scale[row] : 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float x0, x1;
    if constexpr (kEpi == QI_EPI_BF16_ROWCOL) {
      x0 = __fmul_rn(__fmul_rn(v[2 * i], rs), p.col_scale[col0 + c0 + 2 * i]);
      x1 = __fmul_rn(__fmul_rn(v[2 * i + 1], rs), p.col_scale[col0 + c0 + 2 * i + 1]);
    } else {
      x0 = __fmul_rn(v[2 * i], alpha);
      x1 = __fmul_rn(v[2 * i + 1], alpha);
    }
    __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
    w[i] = *reinterpret_cast<uint32_t*>(&h2);
  }
}

__device__ __forceinline__ void store_bf16_transposed(const Params& p, uint32_t* w, int row0, int lane, int col0) {
#pragma unroll
  for (int b = 0; b < 2; ++b) {  // two blocks of 32 words = 64 bf16 columns
    uint32_t* x = w + 32 * b;
    warp_transpose32(x, lane);  // lane now holds word `lane` (columns 2 lane, 2 lane + 1) of rows row0 + j
    uint32_t* base = reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(p.out) + col0 + 64 * b) + lane;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (row0 + j < p.m) base[(int64_t)(row0 + j) * (p.ldo >> 1)] = x[j];
  }
}

// One tile's epilogue for one thread (TMEM row = tile row row0 + lane):
// read the accumulator, call release() (the accumulator may take the next
// tile), then the fused math and stores.  ok must be warp-uniform.
template <int kEpi, class Release>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t acc_row, bool ok, int row0, int lane, int n0,
                                              int half, float alpha, Release release) {
  if constexpr (kEpi == QI_EPI_BF16 || kEpi == QI_EPI_BF16_ROWCOL) {
    const int col0 = n0 + half * 128;
    uint32_t w[64];
    if (ok) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(acc_row + half * 128 + c * 32, v);
        pack_bf16_block<kEpi>(p, v, w + 16 * c, row0 + lane, col0, c * 32, alpha);
      }
    }
    release();
    if (ok) store_bf16_transposed(p, w, row0, lane, col0);
  } else {
    float v[128];
    if (ok) {
      if constexpr (kEpi == QI_EPI_SWIGLU_NVFP4) {
        // gate columns [64h, 64h+64) into v[0..64), up columns [128+64h, ...) into v[64..128)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(acc_row + half * 64 + c * 32, v + c * 32);
          tmem_ld32(acc_row + 128 + half * 64 + c * 32, v + 64 + c * 32);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(acc_row + half * 128 + c * 32, v + c * 32);
      }
    }
    release();
    if (ok) epilogue_rows<kEpi>(p, v, row0, lane, n0, half, alpha);
  }
}

template <int kEpi>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
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
      constexpr uint32_t tx = A_BYTES + B_BYTES;
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
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(BN);
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
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f8(tmem + ACC_COL, sdesc_kmajor_sw128(a_base + kk * 32), sdesc_kmajor_sw128(b_base + kk * 32), idesc,
                   (kt | kk) ? 1u : 0u);
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
      // warp-uniform: the epilogue's transposed stores are warp-collective
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, tcount & 1, abort_flag, p.status));
      tc_fence_after();
      __syncwarp();
      epilogue_tile<kEpi>(p, tmem + lane_off + ACC_COL, ok, row - lane, lane, n0, half, alpha, [&] {
        tc_fence_before();
        mbar_arrive(acc_empty);  // the accumulator may now take the next tile
      });
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- block-scaled variant with scale-writer warps ----------------------------
//
// tcgen05.cp copies of the block scales run in the tensor pipe in series with
// the MMAs (measured: 4 NVFP4 MMAs of a K tile 513 clk alone, 946 clk with the
// 12 copies that feed them).  Here four warps write the scales into TMEM with
// tcgen05.st instead (the same replicated 4 x 32-lane layout the copies
// produce), through their own TMEM ring, and the MMAs run without
// interruption.  The scales have their own shared-memory ring and producer
// thread too, one stage deeper than the A/B ring: the scale writers used to
// start only when a stage's A/B data had landed, and their latency came on
// top of it (a clock trace of the MMA thread: 2961 of 18898 clk per QKV tile
// spent waiting for scales).  16 warps, registers rebalanced with setmaxnreg:
//   warps 0..3   (56 regs): warp 0 A/B TMA producer, warp 1 TMEM allocator +
//                           MMA issuer, warp 2 scale producer,
//   warps 4..7   (72 regs): scale writers, one per TMEM lane quarter,
//   warps 8..15 (192 regs): epilogue, two warps per lane quarter.

constexpr int S_THREADS = 512;
constexpr int S_SST = 5;               // shared-memory scale stages
constexpr int NSF = 5;                 // TMEM scale stages
constexpr int S_SMEM = STAGES * (A_BYTES + B_BYTES) + S_SST * (SFA_BYTES + SFB_BYTES) + 1024 /*align*/ +
                       256 /*barriers*/;
static_assert(S_SMEM + 64 <= 227 * 1024, "scale-writer GEMM exceeds shared memory");
constexpr uint32_t S_SF_COL = 256;     // stage t: columns S_SF_COL + 48t .. +48
constexpr int S_SF_STAGE_COLS = 48;    // 16 for A (4 MMAs x 4), 32 for B (4 MMAs x 2 halves x 4)
static_assert(S_SF_COL + NSF * S_SF_STAGE_COLS <= TMEM_COLS, "scale stages exceed TMEM");
static_assert(56 * 128 + 72 * 128 + 192 * 256 <= 128 * S_THREADS, "register split exceeds the launch budget");

QI_DEV void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <int kEpi>
__global__ void __launch_bounds__(S_THREADS, 1)
    gemm_sfw_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;   // [S_SST]
  uint8_t* sSFB = sSFA + S_SST * SFA_BYTES;  // [S_SST]
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + S_SST * SFB_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* sc_full = empty + STAGES;     // [S_SST] scales in shared memory
  uint64_t* sc_empty = sc_full + S_SST;   // [S_SST]
  uint64_t* sf_full = sc_empty + S_SST;   // [NSF] scales in TMEM
  uint64_t* sf_empty = sf_full + NSF;     // [NSF]
  uint64_t* acc_full = sf_empty + NSF;
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
    for (int s = 0; s < S_SST; ++s) {
      mbar_init(&sc_full[s], 1);
      mbar_init(&sc_empty[s], 4);  // one arrival per scale-writer warp
    }
    for (int t = 0; t < NSF; ++t) {
      mbar_init(&sf_full[t], 4);  // one arrival per scale-writer warp
      mbar_init(&sf_empty[t], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);  // one arrival per epilogue warp
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    if (warp == 0 && lane == 0) {
      constexpr uint32_t tx = A_BYTES + B_BYTES;
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
        }
      }
    } else if (warp == 2 && lane == 0) {
      // Scale producer: each K tile's A and B block scales (6 KB) into the
      // scale ring, as far ahead as the scale writers free its stages.
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * BM, n0 = (tile / p.m_tiles) * BN;
        for (int kt = 0; kt < p.kt; ++kt, ++it) {
          const int s = it % S_SST;
          if (it >= S_SST && !(ok = mbar_wait(&sc_empty[s], ((it / S_SST) - 1) & 1, abort_flag, p.status))) break;
          mbar_expect_tx(&sc_full[s], SFA_BYTES + SFB_BYTES);
          bulk_load(sSFA + s * SFA_BYTES, p.sfa + (int64_t)(m0 >> 7) * p.sfa_block + (int64_t)kt * 2048, 2048,
                    &sc_full[s]);
          bulk_load(sSFB + s * SFB_BYTES, p.sfb + (int64_t)(n0 >> 7) * p.sfb_block + (int64_t)kt * 2048, 2048,
                    &sc_full[s]);
          bulk_load(sSFB + s * SFB_BYTES + 2048, p.sfb + (int64_t)((n0 >> 7) + 1) * p.sfb_block + (int64_t)kt * 2048,
                    2048, &sc_full[s]);
        }
      }
    } else if (warp == 1 && lane == 0) {
      const uint32_t idesc = idesc_nvfp4(BN);
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++tcount) {
        if (tcount > 0 && !(ok = mbar_wait(acc_empty, (tcount - 1) & 1, abort_flag, p.status))) break;
        tc_fence_after();
        for (int kt = 0; kt < p.kt; ++kt, ++it) {
          const int s = it % STAGES, t = it % NSF;
          if (!(ok = mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, p.status))) break;
          if (!(ok = mbar_wait(&sf_full[t], (it / NSF) & 1, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * A_BYTES), b_base = smem_u32(sB + s * B_BYTES);
          const uint32_t sf = tmem + S_SF_COL + t * S_SF_STAGE_COLS;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_nvfp4(tmem + ACC_COL, sdesc_kmajor_sw128(a_base + kk * 32), sdesc_kmajor_sw128(b_base + kk * 32), idesc,
                      sf + kk * 4, sf + 16 + kk * 8, (kt | kk) ? 1u : 0u);
          tc_commit(&empty[s]);
          tc_commit(&sf_empty[t]);
        }
        if (ok) tc_commit(acc_full);
      }
    }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;");
    // Scale writer for TMEM lanes [32q, 32q+32): lane l of every 512-byte
    // atom (32 chunks of 16 bytes) goes to TMEM lane 32q + l, replicated in
    // each quarter as the MMA reads it.  Stage layout (columns): A atoms kk at
    // 4kk; B atoms for output columns 0..127 at 16 + 8kk, 128..255 at 20 + 8kk.
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + S_SF_COL;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
      for (int kt = 0; kt < p.kt; ++kt, ++it) {
        const int s = it % S_SST, t = it % NSF;
        if (!(ok = mbar_wait(&sc_full[s], (it / S_SST) & 1, abort_flag, p.status))) break;
        if (it >= NSF && !(ok = mbar_wait(&sf_empty[t], ((it / NSF) - 1) & 1, abort_flag, p.status))) break;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t v[S_SF_STAGE_COLS];
        const uint4* a4 = reinterpret_cast<const uint4*>(sSFA + s * SFA_BYTES);
        const uint4* b4 = reinterpret_cast<const uint4*>(sSFB + s * SFB_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint4 xa = a4[kk * 32 + lane], xb0 = b4[kk * 32 + lane], xb1 = b4[128 + kk * 32 + lane];
          v[4 * kk] = xa.x, v[4 * kk + 1] = xa.y, v[4 * kk + 2] = xa.z, v[4 * kk + 3] = xa.w;
          v[16 + 8 * kk] = xb0.x, v[17 + 8 * kk] = xb0.y, v[18 + 8 * kk] = xb0.z, v[19 + 8 * kk] = xb0.w;
          v[20 + 8 * kk] = xb1.x, v[21 + 8 * kk] = xb1.y, v[22 + 8 * kk] = xb1.z, v[23 + 8 * kk] = xb1.w;
        }
        const uint32_t dst = lane_base + t * S_SF_STAGE_COLS;
        tmem_st16(dst, v);
        tmem_st16(dst + 16, v + 16);
        tmem_st16(dst + 32, v + 32);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sf_full[t]);
          mbar_arrive(&sc_empty[s]);  // the shared-memory stage was read into registers above
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 192;");
    const int quarter = warp & 3;
    const int half = (warp - 8) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float alpha = p.alpha ? *p.alpha : p.alpha_value;
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tcount) {
      const int m0 = (tile % p.m_tiles) * BM, n0 = (tile / p.m_tiles) * BN;
      const int row = m0 + quarter * 32 + lane;
      bool ok = mbar_wait(acc_full, tcount & 1, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      __syncwarp();
      epilogue_tile<kEpi>(p, tmem + lane_off + ACC_COL, ok, row - lane, lane, n0, half, alpha, [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);  // the accumulator may now take the next tile
      });
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- paired-CTA (2-SM) variant ----------------------------------------------
//
// E4M3 GEMMs with two or more 128-row blocks.  A cluster of two CTAs on a TPC
// computes 256 x 256 output tiles with cta_group::2 MMAs (M = 256): each CTA
// stages its own 128 rows of A and its own 128 rows of B, so per SM the
// tensor cores read half the B operand bytes of the 1-SM kernel (measured
// about 7% faster on the O projection).  The leader (cluster rank 0) issues
// the MMAs; both CTAs' TMA loads signal the leader's stage barrier; the
// leader's commits arrive on both CTAs' barriers; both epilogues release the
// accumulator to the leader.  No load uses cluster multicast.

constexpr int P_STAGES = 6;
constexpr int P_A = 128 * BKB, P_B = 128 * BKB;
constexpr int P_STAGE = P_A + P_B;
constexpr int P_SMEM = P_STAGES * P_STAGE + 1024 /*align*/ + 256 /*barriers*/;

QI_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
QI_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the same shared variable in CTA `rank` of the cluster.
QI_DEV uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
  return out;
}
// Wait with cluster-scope acquire (arrivals may come from the peer CTA).
QI_DEV bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
QI_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((++spins & 63) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - start > kWaitLimitNs) {
        *abort = 1;
        report(status, kStatusWaitTimeout);
        return false;
      }
    }
  }
}
QI_DEV void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// TMA tile loads of a CTA pair: data into this CTA's shared memory, completion
// bytes counted on the leader's barrier (cluster address).  No multicast.
QI_DEV void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t leader_bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(leader_bar), "r"(c0), "r"(c1)
      : "memory");
}
QI_DEV void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
QI_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Commit of the leader's MMAs arriving on the barrier at this offset in both CTAs.
QI_DEV void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
QI_DEV void mma_f8_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Instruction descriptors with M = 256 (the pair's rows).
__host__ __device__ constexpr uint32_t with_m256(uint32_t idesc128) {
  return (idesc128 & ~(0x1Fu << 24)) | ((uint32_t)(256 >> 4) << 24);
}

template <int kEpi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + P_STAGES * P_A;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + P_STAGES * P_B);
  uint64_t* empty = full + P_STAGES;
  uint64_t* acc_full = empty + P_STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: leader
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int m_tiles2 = (p.m + 255) / 256;
  const int tiles = m_tiles2 * p.n_tiles;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * (EPI_THREADS / 32));  // one arrival per epilogue warp of both CTAs
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = 2u * (P_A + P_B);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += pairs) {
        const int m0 = (tile % m_tiles2) * 256 + (int)rank * 128, nb = (tile / m_tiles2) * BN;
        for (int kt = 0; kt < p.kt; ++kt, ++it) {
          const int s = it % P_STAGES;
          if (it >= P_STAGES &&
              !(ok = mbar_wait_cluster(&empty[s], ((it / P_STAGES) - 1) & 1, abort_flag, p.status)))
            break;
          const uint32_t lbar = cluster_addr(&full[s], 0);
          if (rank == 0) mbar_expect_tx(&full[s], tx);
          tma_load_2d_pair(sA + s * P_A, &tma_a, lbar, kt * BKB, m0);
          tma_load_2d_pair(sB + s * P_B, &tma_b, lbar, kt * BKB, nb + (int)rank * 128);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = with_m256(idesc_e4m3(BN));
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += pairs, ++tcount) {
        if (tcount > 0 && !(ok = mbar_wait_cluster(acc_empty, (tcount - 1) & 1, abort_flag, p.status))) break;
        tc_fence_after();
        for (int kt = 0; kt < p.kt; ++kt, ++it) {
          const int s = it % P_STAGES;
          if (!(ok = mbar_wait_cluster(&full[s], (it / P_STAGES) & 1, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * P_A), b_base = smem_u32(sB + s * P_B);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f8_pair(tmem + ACC_COL, sdesc_kmajor_sw128(a_base + kk * 32), sdesc_kmajor_sw128(b_base + kk * 32),
                        idesc, (kt | kk) ? 1u : 0u);
          tc_commit_pair(&empty[s]);
        }
        if (ok) tc_commit_pair(acc_full);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float alpha = p.alpha ? *p.alpha : p.alpha_value;
    const uint32_t leader_acc_empty = cluster_addr(acc_empty, 0);
    uint32_t tcount = 0;
    for (int tile = pair; tile < tiles; tile += pairs, ++tcount) {
      const int m0 = (tile % m_tiles2) * 256 + (int)rank * 128, n0 = (tile / m_tiles2) * BN;
      const int row = m0 + quarter * 32 + lane;
      // warp-uniform: the epilogue's transposed stores are warp-collective
      const bool ok = __all_sync(0xffffffffu, mbar_wait_cluster(acc_full, tcount & 1, abort_flag, p.status));
      tc_fence_after();
      __syncwarp();
      epilogue_tile<kEpi>(p, tmem + lane_off + ACC_COL, ok, row - lane, lane, n0, half, alpha, [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(leader_acc_empty);  // the accumulator may take the next tile
      });
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the other may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
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

template <int kEpi>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, cudaStream_t stream) {
  static bool configured[64] = {};
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  if (cur_dev < 0 || cur_dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!configured[cur_dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_kernel<kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
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
  gemm_kernel<kEpi><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
  return (int)cudaPeekAtLastError();
}

template <int kEpi>
int launch_sfw(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, cudaStream_t stream) {
  static bool configured[64] = {};
  static int sms[64] = {};
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  if (cur_dev < 0 || cur_dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!configured[cur_dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_sfw_kernel<kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S_SMEM + 64);
    if (e != cudaSuccess) return (int)e;
    e = cudaDeviceGetAttribute(&sms[cur_dev], cudaDevAttrMultiProcessorCount, cur_dev);
    if (e != cudaSuccess) return (int)e;
    configured[cur_dev] = true;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < sms[cur_dev] ? tiles : sms[cur_dev];
  gemm_sfw_kernel<kEpi><<<grid, S_THREADS, S_SMEM + 64, stream>>>(ma, mb, p);
  return (int)cudaPeekAtLastError();
}

template <int kEpi>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, cudaStream_t stream) {
  static bool configured[64] = {};
  static int max_pairs[64] = {};
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  if (cur_dev < 0 || cur_dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!configured[cur_dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         P_SMEM);
    if (e != cudaSuccess) return (int)e;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cur_dev);
    if (e != cudaSuccess) return (int)e;
    // Clusters that can be resident at once (pairs of SMs on a TPC).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = P_SMEM;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_kernel<kEpi>, &cfg) != cudaSuccess ||
        clusters < 1) {
      cudaGetLastError();
      clusters = sms / 2;
    }
    max_pairs[cur_dev] = clusters;
    configured[cur_dev] = true;
  }
  const int tiles = ((p.m + 255) / 256) * p.n_tiles;
  const int pairs = tiles < max_pairs[cur_dev] ? tiles : max_pairs[cur_dev];
  gemm_pair_kernel<kEpi><<<2 * pairs, THREADS, P_SMEM, stream>>>(ma, mb, p);
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
  if (fp4) {
    // Block-scaled: scale factors written to TMEM by warps (see gemm_sfw_kernel).
    if (!make_map_u8(&ma, g->a, k_bytes, g->m, BM) || !make_map_u8(&mb, g->b, k_bytes, g->n, BN))
      return (int)cudaErrorInvalidValue;
    switch (g->epilogue) {
      case QI_EPI_BF16: return launch_sfw<QI_EPI_BF16>(ma, mb, p, stream);
      case QI_EPI_F32: return launch_sfw<QI_EPI_F32>(ma, mb, p, stream);
      case QI_EPI_SWIGLU_NVFP4: return launch_sfw<QI_EPI_SWIGLU_NVFP4>(ma, mb, p, stream);
      default: return (int)cudaErrorInvalidValue;
    }
  }
  // E4M3.  Two or more 128-row blocks: paired CTAs (2-SM MMA, 256 x 256 tiles).
  if (g->m > BM) {
    if (!make_map_u8(&ma, g->a, k_bytes, g->m, 128) || !make_map_u8(&mb, g->b, k_bytes, g->n, 128))
      return (int)cudaErrorInvalidValue;
    switch (g->epilogue) {
      case QI_EPI_BF16: return launch_pair<QI_EPI_BF16>(ma, mb, p, stream);
      case QI_EPI_F32: return launch_pair<QI_EPI_F32>(ma, mb, p, stream);
      case QI_EPI_BF16_ROWCOL: return launch_pair<QI_EPI_BF16_ROWCOL>(ma, mb, p, stream);
      default: return (int)cudaErrorInvalidValue;
    }
  }
  if (!make_map_u8(&ma, g->a, k_bytes, g->m, BM) || !make_map_u8(&mb, g->b, k_bytes, g->n, BN))
    return (int)cudaErrorInvalidValue;
  switch (g->epilogue) {
    case QI_EPI_BF16: return launch<QI_EPI_BF16>(ma, mb, p, stream);
    case QI_EPI_F32: return launch<QI_EPI_F32>(ma, mb, p, stream);
    case QI_EPI_BF16_ROWCOL: return launch<QI_EPI_BF16_ROWCOL>(ma, mb, p, stream);
    default: return (int)cudaErrorInvalidValue;
  }
}

int qi_gemm_resources(int* out) {
  if (!out) return (int)cudaErrorInvalidValue;
  cudaFuncAttributes a{};
  const cudaError_t e = cudaFuncGetAttributes(&a, gemm_sfw_kernel<QI_EPI_BF16>);
  if (e != cudaSuccess) return (int)e;
  out[0] = S_SMEM + 64;
  out[1] = a.numRegs;
  out[2] = S_THREADS;
  return 0;
}

}  // extern "C"
