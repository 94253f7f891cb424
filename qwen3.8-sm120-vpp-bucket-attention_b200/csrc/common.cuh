// Shared device helpers for the sm_100a kernels of the folded-VPP prefill path:
// exactly-rounded fp32 arithmetic, NVFP4 / FP8 conversions, mbarrier / TMA /
// tcgen05 wrappers (inline PTX) and bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qwen_infra_b200.h"

#define QI_DEV __device__ __forceinline__

namespace qi {

// ---------------------------------------------------------------------------
// Status words written by kernels (never a trap): OR-ed into a device int.
// ---------------------------------------------------------------------------
enum : int {
  kStatusOk = 0,
  kStatusBadKvScale = 1 << 0,   // non-finite or non-positive K/V global scale
  kStatusWaitTimeout = 1 << 1,  // an mbarrier wait gave up
  kStatusBadSlot = 1 << 2,      // a KV slot outside the cache (reported, skipped)
};

// The kernel library links its own (static) CUDA runtime, whose current
// device is independent of the caller's runtime.  Every entry point makes the
// device of its stream (or, for a default stream, of its first operand)
// current before it launches.
inline cudaError_t bind_device(cudaStream_t stream, const void* operand) {
  int dev = -1;
  const uintptr_t h = reinterpret_cast<uintptr_t>(stream);
  if (h > 2) {
    const cudaError_t e = cudaStreamGetDevice(stream, &dev);
    if (e != cudaSuccess) return e;
  } else if (operand) {
    cudaPointerAttributes attr{};
    const cudaError_t e = cudaPointerGetAttributes(&attr, operand);
    if (e != cudaSuccess) return e;
    dev = attr.device;
  }
  if (dev < 0) return cudaSuccess;
  int cur = -1;
  cudaGetDevice(&cur);
  return cur == dev ? cudaSuccess : cudaSetDevice(dev);
}

#define QI_BIND(stream, ptr)                                   \
  do {                                                         \
    const cudaError_t qi_bind_e = qi::bind_device(stream, ptr); \
    if (qi_bind_e != cudaSuccess) return (int)qi_bind_e;       \
  } while (0)

QI_DEV void report(int* status, int code) {
  if (status) atomicOr(status, code);
}

// ---------------------------------------------------------------------------
// fp32 helpers: one IEEE rounding per operation, never contracted.
// ---------------------------------------------------------------------------
QI_DEV float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// Two values rounded to bf16 (RN-even) with one packed conversion.
QI_DEV void bf16r2(float& a, float& b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));  // first source -> upper half
  a = __uint_as_float(r << 16);
  b = __uint_as_float(r & 0xFFFF0000u);
}

QI_DEV float e4m3_to_f(uint32_t c) {
  const uint32_t e = (c >> 3) & 0xF, m = c & 7;
  float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20)) : __fmul_rn((float)m, 0.001953125f);
  return (c & 0x80) ? -v : v;
}

QI_DEV uint32_t f_to_e4m3(float x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  return r & 0xFFu;
}
// Two E4M3 codes in one conversion: lo in bits 0-7, hi in bits 8-15.
QI_DEV uint32_t f2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Eight fp32 values -> eight E2M1 codes packed in 32 bits, element 0 in the
// lowest nibble (cvt.e2m1x2 puts its FIRST source operand in the high nibble).
QI_DEV uint32_t f8_to_e2m1x8(const float* v) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

QI_DEV uint32_t f2_to_e2m1x2(float lo, float hi) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.u32.u8 %0, b0;\n\t}"
      : "=r"(out)
      : "f"(lo), "f"(hi));
  return out & 0xFFu;
}

// sigmoid and SiLU with CUDA's expf, as the reference calls it
// (nvfp4_bucket_xqa.cu:57: 1/(1+expf(-g)); vLLM's SiLU-and-mul: g/(1+expf(-g))).
// Each division and addition is one IEEE fp32 operation.
QI_DEV float sigmoid_f(float g) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))); }
QI_DEV float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

QI_DEV float warp_sum_butterfly(float v) {
#pragma unroll
  for (int d = 16; d; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}
QI_DEV float warp_max_butterfly(float v) {
#pragma unroll
  for (int d = 16; d; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// Byte offset of the E4M3 scale of (row, 16-element group) in the 128x4
// swizzled block-scale layout; `gp` is groups per row padded to 4.
QI_DEV int64_t sf_offset(int64_t row, int64_t group, int64_t gp) {
  return (row >> 7) * (128 * gp) + (group >> 2) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 +
         (group & 3);
}

// NVFP4 quantisation of 16 values with a (quantisation-direction) global scale
// g: scale = e4m3(min(amax*g*(1/6), 448)), codes = e2m1(v*g/scale).  Returns
// the scale byte; writes 8 packed bytes.
QI_DEV uint32_t nvfp4_quant16(const float* v, float g, uint2& packed) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
  const float pre = fminf(__fmul_rn(__fmul_rn(amax, g), 0x1.555556p-3f), 448.0f);
  const uint32_t sf = f_to_e4m3(pre);
  const float scale = e4m3_to_f(sf);
  const float inv = scale > 0.0f ? __fdiv_rn(g, scale) : 0.0f;
  float t[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) t[j] = __fmul_rn(v[j], inv);
  packed.x = f8_to_e2m1x8(t);
  packed.y = f8_to_e2m1x8(t + 8);
  return sf;
}

// ---------------------------------------------------------------------------
// Shared memory / mbarrier / TMA
// ---------------------------------------------------------------------------
QI_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

QI_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
QI_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
QI_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
QI_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
QI_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
QI_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after `limit_ns` (or at once when another role of the
// CTA already gave up, signalled through *abort), records the failure and
// returns false.  No wait in these kernels can spin forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s; the longest launch is ~10 ms
QI_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
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

QI_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
QI_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses and size).
QI_DEV void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
QI_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
QI_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, tensor memory)
// ---------------------------------------------------------------------------
QI_DEV void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
QI_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
QI_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QI_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 format, version 1).  K-major
// operand staged by TMA with 128-byte swizzle: rows of 128 B, 8-row groups
// 1024 B apart (SBO), LBO unused (1).
QI_DEV uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major operand with 128-byte swizzle: 64-element MN chunks of 128 B,
// 8 K-rows per 1 KB atom; LBO = stride between MN chunks, SBO = stride
// between 8-row K groups.
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

QI_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
QI_DEV void mma_nvfp4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}
QI_DEV void mma_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
QI_DEV void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptors (M = 128, K-major A and B).
// kind::mxf4nvf4: A/B E2M1 (format 1), UE4M3 scales (bit 23 = 0).
__host__ __device__ constexpr uint32_t idesc_nvfp4(int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// kind::f8f6f4: A/B E4M3 (format 0), fp32 accumulator (c_format 1).
__host__ __device__ constexpr uint32_t idesc_e4m3(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// kind::f16: A/B BF16 (format 1), fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets lane
// (warp's quarter * 32 + i), columns [col, col + 32).
QI_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
QI_DEV void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

QI_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// NVFP4 / E4M3 -> f16 conversions of the cached K/V values (exact in f16).
// Two e2m1 codes (one byte, low nibble = even element) -> f16x2 (even in the
// low half); four bytes of a word at once.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t* out) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
      : "r"(w));
}
// Two e4m3 scale bytes (low byte first) -> f16x2.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  uint32_t out;
  asm("{\n\t.reg .b16 h;\n\t"
      "cvt.u16.u32 h, %1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, h;\n\t}"
      : "=r"(out)
      : "r"(two));
  return out;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// f16x2 with the low (sel = 0) or high (sel = 1) half of `pair` in both halves.
__device__ __forceinline__ uint32_t splat_half(uint32_t pair, int sel) {
  return sel ? __byte_perm(pair, 0, 0x3232) : __byte_perm(pair, 0, 0x1010);
}

// Host-side request checks shared by entry points that combine several
// launches (the allocation-free attention): every argument is checked before
// the first launch, so a rejected call launches nothing.
bool attention_request_valid(const QiAttention* a);
bool paged_attention_request_valid(const QiPagedAttention* a);
bool kv_dequant_request_valid(const QiKvView* kv, const int32_t* block_table, int first, int tokens,
                              const void* k_out, int64_t k_capacity, const void* vt_out, int64_t vt_row);

}  // namespace qi
