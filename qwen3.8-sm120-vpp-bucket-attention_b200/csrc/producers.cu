// HBM-bound producers of one decoder layer (sm_100a):
//   * residual add + RMSNorm -> NVFP4 pack with 128x4-swizzled E4M3 scales,
//   * the same norm with a bf16 output (final norm of the last stage),
//   * QK-norm + NeoX RoPE + gate split + NVFP4 paged KV append,
//   * attention output x sigmoid(gate) -> FP8 E4M3 with a per-token scale,
//   * weight quantisers (NVFP4 per 16 + global, FP8 per output channel),
//   * paged NVFP4 KV -> contiguous bf16 K and transposed V for attention.
// Every fp32 step is an explicitly rounded IEEE operation; the reduction trees
// are fixed, so the CPU restatement reproduces the quantised bytes exactly.
#include <cuda_fp16.h>

#include "common.cuh"
#include "qwen_infra_b200.h"

using namespace qi;

namespace {

struct alignas(16) BF8 {
  __nv_bfloat162 v[4];
};

QI_DEV void load16_bf16(const __nv_bfloat16* p, float* out) {
  const uint4 a = reinterpret_cast<const uint4*>(p)[0];
  const uint4 b = reinterpret_cast<const uint4*>(p)[1];
  const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 fa = __bfloat1622float2(pa[i]);
    float2 fb = __bfloat1622float2(pb[i]);
    out[2 * i] = fa.x;
    out[2 * i + 1] = fa.y;
    out[8 + 2 * i] = fb.x;
    out[8 + 2 * i + 1] = fb.y;
  }
}

QI_DEV void store16_bf16(__nv_bfloat16* p, const float* v) {
  uint4 a, b;
  __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&a);
  __nv_bfloat162* pb = reinterpret_cast<__nv_bfloat162*>(&b);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    pa[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    pb[i] = __floats2bfloat162_rn(v[8 + 2 * i], v[8 + 2 * i + 1]);
  }
  reinterpret_cast<uint4*>(p)[0] = a;
  reinterpret_cast<uint4*>(p)[1] = b;
}

// Block-wide sum over per-thread partials: warp xor-butterfly, then a second
// butterfly over the zero-padded per-warp sums.  Result broadcast to all.
QI_DEV float block_sum(float v, float* scratch32) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum_butterfly(v);
  if (lane == 0) scratch32[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < nwarps ? scratch32[lane] : 0.0f;
    w = warp_sum_butterfly(w);
    if (lane == 0) scratch32[32] = w;
  }
  __syncthreads();
  return scratch32[32];
}

QI_DEV float block_max(float v, float* scratch32) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  v = warp_max_butterfly(v);
  if (lane == 0) scratch32[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < nwarps ? scratch32[lane] : 0.0f;
    w = warp_max_butterfly(w);
    if (lane == 0) scratch32[32] = w;
  }
  __syncthreads();
  return scratch32[32];
}

// One CTA per row, thread t owns elements [16t, 16t+16) (= scale group t).
// The kernel waits on its loads with too few warps (a CTA per row, the block
// reduction between the loads and the stores), and at 34 registers a thread
// four 10-warp CTAs fill an SM's register file; capped at 32 (no spills),
// five do.
template <bool kQuant>
__global__ void __maxnreg__(32) norm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ residual,
                            const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ gscale,
                            uint8_t* __restrict__ q, uint8_t* __restrict__ sf, __nv_bfloat16* __restrict__ updated,
                            __nv_bfloat16* __restrict__ y_out, int hidden, float eps, float woff) {
  __shared__ float scratch[33];
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const int groups = hidden >> 4;
  const bool active = t < groups;
  float h[16];
  float ss = 0.0f;
  if (active) {
    const int64_t base = row * hidden + 16 * t;
    load16_bf16(x + base, h);
    if (residual) {
      float r[16];
      load16_bf16(residual + base, r);
#pragma unroll
      for (int j = 0; j < 16; ++j) h[j] = __fadd_rn(h[j], r[j]);
    }
    // the reference's per-thread order: h0^2, h8^2, h1^2, h9^2, ... h7^2, h15^2
    // (nvfp4_norm_pack.cu:23-27: each step adds one element of each 8-half)
    ss = __fmul_rn(h[0], h[0]);
    ss = __fadd_rn(ss, __fmul_rn(h[8], h[8]));
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      ss = __fadd_rn(ss, __fmul_rn(h[j], h[j]));
      ss = __fadd_rn(ss, __fmul_rn(h[j + 8], h[j + 8]));
    }
    if (updated) store16_bf16(updated + base, h);
  }
  const float total = block_sum(ss, scratch);
  // CUDA's rsqrtf, as the reference calls it (nvfp4_norm_pack.cu:39)
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(total, (float)hidden), eps));
  if (!active) return;
  float w[16], y[16];
  load16_bf16(gamma + 16 * t, w);
#pragma unroll
  for (int j = 0; j < 16; ++j) y[j] = bf16r(__fmul_rn(__fmul_rn(h[j], inv), __fadd_rn(w[j], woff)));
  if constexpr (kQuant) {
    uint2 packed;
    const uint32_t code = nvfp4_quant16(y, *gscale, packed);
    reinterpret_cast<uint2*>(q + row * (hidden >> 1))[t] = packed;
    const int64_t gp = (groups + 3) & ~3;
    sf[sf_offset(row, t, gp)] = (uint8_t)code;
  } else {
    store16_bf16(y_out + row * hidden + 16 * t, y);
  }
}

// QK-norm + RoPE + gate split + NVFP4 paged append.  One CTA per row.  A head
// of D values is handled by L = D/16 lanes: lane `sub` of the head owns the 8
// consecutive elements [8 sub, 8 sub + 8) of each rotary half (16-byte loads
// and stores), so a warp takes 32/L heads at once and the row's heads are
// split into warp tasks (Q heads first, then K heads, each K task also
// appending its V head).
//
// The sum of squares follows the reference kernel's tree exactly
// (nvfp4_attention_front.cu:72-82): pair t = (element t, element t + D/2) is
// one reference thread with partial x^2 + y^2; 32 consecutive pairs form a
// reference warp reduced by shfl_down (16, 8, 4, 2, 1), and the warp partials
// by a second shfl_down tree over lanes padded with zeros.  Pair t = 8 sub + e
// lives in lane `sub`, element e, so: the 16-step pairs lanes sub and sub ^ 2,
// the 8-step sub and sub ^ 1, the 4/2/1 steps stay inside the lane, and the
// warp partials sit in subs 0, 4, 8, 12.  Then rsqrtf as the reference.
QI_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
QI_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

QI_DEV void unpack8_bf16(const uint4& a, float* out) {
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = bf16_lo(w[i]);
    out[2 * i + 1] = bf16_hi(w[i]);
  }
}
// Element e (compile-time in unrolled loops) of 8 packed bf16 values.
QI_DEV float bf16_at(const uint4& a, int e) {
  const uint32_t w = e < 2 ? a.x : e < 4 ? a.y : e < 6 ? a.z : a.w;
  return (e & 1) ? bf16_hi(w) : bf16_lo(w);
}

QI_DEV void load8_bf16(const __nv_bfloat16* p, float* out) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = bf16_lo(w[i]);
    out[2 * i + 1] = bf16_hi(w[i]);
  }
}

QI_DEV void store8_bf16(__nv_bfloat16* p, const float* v) {
  uint4 a;
  __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) pa[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = a;
}

QI_DEV void load8_trig(const void* base, int64_t off, bool is_float, float* out) {
  if (is_float) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off + 4);
    out[0] = a.x, out[1] = a.y, out[2] = a.z, out[3] = a.w;
    out[4] = b.x, out[5] = b.y, out[6] = b.z, out[7] = b.w;
  } else {
    load8_bf16(static_cast<const __nv_bfloat16*>(base) + off, out);
  }
}

// Sum of squares of one head over its L lanes in the reference's tree order.
template <int L>
QI_DEV float head_sum_squares(const float* x, const float* y) {
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(__fmul_rn(x[e], x[e]), __fmul_rn(y[e], y[e]));
  if constexpr (L >= 4) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], __shfl_xor_sync(0xffffffffu, v[e], 2));  // pairs t, t+16
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], __shfl_xor_sync(0xffffffffu, v[e], 1));  // t, t+8
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = __fadd_rn(v[e], v[e + 4]);
  v[0] = __fadd_rn(v[0], v[2]);
  v[1] = __fadd_rn(v[1], v[3]);
  float p = __fadd_rn(v[0], v[1]);  // this reference warp's partial, valid in subs 0, 4, 8, 12
  if constexpr (L == 16) {
    p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 8));  // warps w, w + 2
    p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 4));  // then w, w + 1
  } else if constexpr (L == 8) {
    p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 4));
  }
  const int lane = threadIdx.x & 31;
  return __shfl_sync(0xffffffffu, p, lane & ~(L - 1));  // from the head's sub 0
}

// NVFP4 of 8 values of one lane; the 16-element group spans lanes sub, sub^1.
// scale = e4m3(amax / (6 g)), code = e2m1(v * 1/(scale g))
// (nvfp4_attention_front.cu:45-66).  Returns the 4 code bytes; the scale byte
// goes to *scale_code.
QI_DEV uint32_t kv_quant8(const float* v, float g, uint32_t* scale_code) {
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const uint32_t code = f_to_e4m3(__fdiv_rn(amax, __fmul_rn(6.0f, g)));
  const float scale = e4m3_to_f(code);
  const float inverse = scale > 0.0f ? __fdiv_rn(1.0f, __fmul_rn(scale, g)) : 0.0f;
  float t[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) t[e] = __fmul_rn(v[e], inverse);
  *scale_code = code;
  return f8_to_e2m1x8(t);
}

// One warp per task: a task is 32/L heads of one kind (Q heads, or K heads
// with their V heads), so a row has ceil(Hq/HPW) + ceil(Hkv/HPW) tasks and
// blockIdx.y picks a group of `warpsPerCta` of them.  Every load a warp needs
// (its heads' values, the V values of a K task, cos/sin and its norm weight)
// is issued before any arithmetic, so each warp has all its bytes in flight
// at once; only the weights of the task's own kind are held.
// Capped at 64 registers (three spilled words; 74 uncapped): five 6-warp CTAs
// per SM instead of four -- the kernel is latency-bound, so warps are speed.
template <int D>
__global__ void __maxnreg__(64) front_kernel(QiFront p) {
  constexpr int HALF = D / 2, L = D / 16, HPW = 32 / L;
  const int lane = threadIdx.x & 31;
  const int sub = lane % L, hsel = lane / L;
  const int64_t row = blockIdx.x;
  const int d0 = sub * 8;
  const int q_tasks = (p.qheads + HPW - 1) / HPW;
  const int tasks = q_tasks + (p.kvheads + HPW - 1) / HPW;
  const int task = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (task >= tasks) return;  // whole warp
  const bool is_k = task >= q_tasks;
  int64_t slot = -1;
  if (is_k) {
    if (row >= p.slot_rows) return;  // nothing to append for this row
    slot = p.slot_long ? static_cast<const int64_t*>(p.slots)[row] : static_cast<const int32_t*>(p.slots)[row];
    if (slot < 0) return;  // padding token
  }
  const int local = (is_k ? task - q_tasks : task) * HPW + hsel;
  const bool live = local < (is_k ? p.kvheads : p.qheads);
  const __nv_bfloat16* qkv = static_cast<const __nv_bfloat16*>(p.qkv);
  const int64_t base =
      row * p.input_row + (is_k ? (int64_t)p.qheads * 2 * D + (int64_t)local * D : (int64_t)local * 2 * D);
  const int64_t vbase = row * p.input_row + (int64_t)p.qheads * 2 * D + (int64_t)p.kvheads * D + (int64_t)local * D;
  // bf16 operands stay packed (4 registers per 8 values) until they are used:
  // the kernel is latency-bound, so registers are warps.
  uint4 xr = make_uint4(0, 0, 0, 0), yr = xr, vxr = xr, vyr = xr;
  if (live) {
    xr = *reinterpret_cast<const uint4*>(qkv + base + d0);
    yr = *reinterpret_cast<const uint4*>(qkv + base + HALF + d0);
    if (is_k) {
      vxr = *reinterpret_cast<const uint4*>(qkv + vbase + d0);
      vyr = *reinterpret_cast<const uint4*>(qkv + vbase + HALF + d0);
    }
  }
  const int64_t pos = p.pos_long ? static_cast<const int64_t*>(p.positions)[row]
                                 : static_cast<const int32_t*>(p.positions)[row];
  float cs[8], sn[8];
  const __nv_bfloat16* wsrc = static_cast<const __nv_bfloat16*>(is_k ? p.k_weight : p.q_weight);
  const uint4 w0r = *reinterpret_cast<const uint4*>(wsrc + d0), w1r = *reinterpret_cast<const uint4*>(wsrc + HALF + d0);
  load8_trig(p.cos_sin, pos * p.cos_row + d0, p.cos_float, cs);
  load8_trig(p.cos_sin, pos * p.cos_row + HALF + d0, p.cos_float, sn);
  float x[8], y[8];
  unpack8_bf16(xr, x);
  unpack8_bf16(yr, y);
  const float total = head_sum_squares<L>(x, y);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(total, (float)D), p.eps));  // nvfp4_attention_front.cu:81
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = bf16r(__fmul_rn(__fmul_rn(x[e], inv), __fadd_rn(bf16_at(w0r, e), p.weight_offset)));
    const float b = bf16r(__fmul_rn(__fmul_rn(y[e], inv), __fadd_rn(bf16_at(w1r, e), p.weight_offset)));
    x[e] = bf16r(__fsub_rn(__fmul_rn(a, cs[e]), __fmul_rn(b, sn[e])));
    y[e] = bf16r(__fadd_rn(__fmul_rn(b, cs[e]), __fmul_rn(a, sn[e])));
  }
  if (!is_k) {
    if (!live) return;
    __nv_bfloat16* q = static_cast<__nv_bfloat16*>(p.q) + row * p.q_row + (int64_t)local * D;
    store8_bf16(q + d0, x);
    store8_bf16(q + HALF + d0, y);
    if (p.gate) {
      __nv_bfloat16* g = static_cast<__nv_bfloat16*>(p.gate) + row * p.gate_row + (int64_t)local * D;
      *reinterpret_cast<uint4*>(g + d0) = *reinterpret_cast<const uint4*>(qkv + base + D + d0);
      *reinterpret_cast<uint4*>(g + HALF + d0) = *reinterpret_cast<const uint4*>(qkv + base + D + HALF + d0);
    }
    return;
  }
  if (slot >= (int64_t)p.pages * p.page_size) {
    if (lane == 0) report(p.status, kStatusBadSlot);
    return;
  }
  const float kg = *p.k_global, vg = *p.v_global;
  if (!(isfinite(kg) && kg > 0.0f && isfinite(vg) && vg > 0.0f)) {
    if (lane == 0) report(p.status, kStatusBadKvScale);
    return;
  }
  const int64_t page = slot / p.page_size, entry = slot % p.page_size;
  const int64_t data = page * p.data_page + entry * p.data_row + (int64_t)local * p.data_head;
  const int64_t sfo = page * p.sf_page + entry * p.sf_row + (int64_t)local * p.sf_head;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    uint8_t* codes = static_cast<uint8_t*>(which ? p.v_cache : p.k_cache) + data;
    uint8_t* scales = static_cast<uint8_t*>(which ? p.v_scales : p.k_scales) + sfo;
    uint32_t sx, sy;
    // K: the normed, rotated values; V: the raw projection values
    float vx[8], vy[8];
    if (which) {
      unpack8_bf16(vxr, vx);
      unpack8_bf16(vyr, vy);
    }
    const uint32_t cx = kv_quant8(which ? vx : x, which ? vg : kg, &sx);
    const uint32_t cy = kv_quant8(which ? vy : y, which ? vg : kg, &sy);
    if (live) {
      *reinterpret_cast<uint32_t*>(codes + (d0 >> 1)) = cx;
      *reinterpret_cast<uint32_t*>(codes + ((HALF + d0) >> 1)) = cy;
      if ((sub & 1) == 0) {
        scales[d0 >> 4] = (uint8_t)sx;
        scales[(HALF + d0) >> 4] = (uint8_t)sy;
      }
    }
  }
}

// The gate of column c sits at gate + row * gate_row + (c / head_dim) *
// head_stride + c % head_dim: a compact [rows, cols] gate (head_dim = cols),
// or the gate halves read in place from the QKV projection's per-head
// [q(D) | gate(D)] blocks (head_dim = D, head_stride = 2D).
// With static_scale (the reference's form: one per-tensor scale) the row
// maximum is not taken and scale_out is not written.
// Capped at 40 registers (one spilled word): three CTAs of 512 threads per SM
// instead of two -- the kernel is latency- and XU-bound, so warps are speed.
__global__ void __maxnreg__(40) gate_fp8_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ gate,
                                int64_t out_row, int64_t gate_row, int head_dim, int64_t head_stride,
                                uint8_t* __restrict__ fp8, int64_t fp8_row, float* __restrict__ scale_out, int cols,
                                const float* __restrict__ static_scale) {
  __shared__ float scratch[33];
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const bool active = 16 * t < cols;
  float v[16];
  float amax = 0.0f;
  if (active) {
    float o[16], g[16];
    load16_bf16(out + row * out_row + 16 * t, o);
    load16_bf16(gate + row * gate_row + (int64_t)(16 * t / head_dim) * head_stride + (16 * t) % head_dim, g);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      float s0 = sigmoid_f(g[j]), s1 = sigmoid_f(g[j + 1]);
      bf16r2(s0, s1);
      float v0 = __fmul_rn(o[j], s0), v1 = __fmul_rn(o[j + 1], s1);
      bf16r2(v0, v1);
      v[j] = v0, v[j + 1] = v1;
      amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
    }
  }
  float scale;
  if (static_scale) {
    scale = *static_scale;
  } else {
    amax = block_max(amax, scratch);
    scale = fmaxf(__fdiv_rn(amax, 448.0f), 1.17549435e-38f);
    if (t == 0) scale_out[row] = scale;
  }
  if (!active) return;
  uint32_t w[4];
  if (static_scale) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = f2_to_e4m3x2(__fdiv_rn(v[4 * k], scale), __fdiv_rn(v[4 * k + 1], scale)) |
             (f2_to_e4m3x2(__fdiv_rn(v[4 * k + 2], scale), __fdiv_rn(v[4 * k + 3], scale)) << 16);
  } else {
    // v / scale correctly rounded from one reciprocal per row, by Markstein's
    // correction step (IBM J. Res. Dev. 34(1), 1990): y = RN(1/s),
    // q = RN(v y), r = v - s q (exact with an FMA), RN(q + r y) = RN(v / s)
    // whenever the quotient is a normal number.  Here |v| <= 448 s, so it
    // never overflows; a quotient below the normal range encodes to e4m3
    // zero either way.
    const float y = __frcp_rn(scale);
    auto quot = [&](float a) {
      const float q0 = __fmul_rn(a, y);
      return __fmaf_rn(__fmaf_rn(-q0, scale, a), y, q0);
    };
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = f2_to_e4m3x2(quot(v[4 * k]), quot(v[4 * k + 1])) |
             (f2_to_e4m3x2(quot(v[4 * k + 2]), quot(v[4 * k + 3])) << 16);
  }
  reinterpret_cast<uint4*>(fp8 + row * fp8_row)[t] = make_uint4(w[0], w[1], w[2], w[3]);
}

// SiLU-and-mul + NVFP4 of the gate_up GEMM output.  gu is bf16 [rows, 2I]
// with gate and up interleaved in 128-column blocks (block b: gate channels
// 128b.. at columns 256b.., up at 256b+128..), already bf16(acc * alpha).
// One thread per (row, 16-channel scale group): act = bf16(silu(gate) * up),
// then the NVFP4 quantisation with global scale g.  Grid: rows x I/16 threads
// in blocks of 256 (high occupancy: the SiLU is ~50 exact fp32 operations per
// element).
__global__ void __launch_bounds__(256) swiglu_nvfp4_kernel(const __nv_bfloat16* __restrict__ gu, int64_t gu_row,
                                                           int rows, int groups, const float* __restrict__ gscale,
                                                           uint8_t* __restrict__ q, int64_t q_row,
                                                           uint8_t* __restrict__ sf, int64_t gp) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)rows * groups) return;
  const int64_t row = idx / groups;
  const int grp = (int)(idx - row * groups);
  const int ch = grp * 16;
  const int64_t col = (int64_t)(ch >> 7) * 256 + (ch & 127);
  float g[16], u[16], v[16];
  load16_bf16(gu + row * gu_row + col, g);
  load16_bf16(gu + row * gu_row + col + 128, u);
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = bf16r(__fmul_rn(silu_f(g[j]), u[j]));
  uint2 packed;
  const uint32_t code = nvfp4_quant16(v, *gscale, packed);
  *reinterpret_cast<uint2*>(q + row * q_row + (ch >> 1)) = packed;
  sf[sf_offset(row, grp, gp)] = (uint8_t)code;
}

// Weight quantiser: fp32 [rows, K] -> NVFP4 (same arithmetic as the producer).
__global__ void nvfp4_quant_kernel(const float* __restrict__ w, int64_t rows, int k, const float* __restrict__ g,
                                   uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  const int64_t groups = k >> 4;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * groups) return;
  const int64_t row = idx / groups, grp = idx % groups;
  float v[16];
  const float4* src = reinterpret_cast<const float4*>(w + row * k + grp * 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 f = src[i];
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
  uint2 packed;
  const uint32_t code = nvfp4_quant16(v, *g, packed);
  reinterpret_cast<uint2*>(q + row * (k >> 1))[grp] = packed;
  sf[sf_offset(row, grp, (groups + 3) & ~3)] = (uint8_t)code;
}

// Weight quantiser: fp32 [rows, K] -> E4M3 with scale[row] = max(amax/448, FLT_MIN).
__global__ void fp8_rows_kernel(const float* __restrict__ w, int k, uint8_t* __restrict__ q,
                                float* __restrict__ scale_out) {
  __shared__ float scratch[33];
  const int64_t row = blockIdx.x;
  float amax = 0.0f;
  for (int c = threadIdx.x; c < k; c += blockDim.x) amax = fmaxf(amax, fabsf(w[row * k + c]));
  amax = block_max(amax, scratch);
  const float scale = fmaxf(__fdiv_rn(amax, 448.0f), 1.17549435e-38f);
  if (threadIdx.x == 0) scale_out[row] = scale;
  for (int c = threadIdx.x; c < k; c += blockDim.x) q[row * k + c] = (uint8_t)f_to_e4m3(__fdiv_rn(w[row * k + c], scale));
}

// Paged NVFP4 K/V of one KV head -> contiguous f16 K [tokens, D] and V^T
// [D, vt_row].  CTA = 64 tokens of one head; thread = (token, 32-value
// quarter of D=128 / half of D=64): one 16-byte code load and one 2-byte scale
// load per K and V, K stored with 16-byte stores (each token's row is written
// by its threads as one contiguous run), V staged transposed in shared memory
// and stored as 128-byte V^T row segments in 16-byte pieces.  Values:
// e2m1 x e4m3, exact in f16 (at most 6 significant bits, magnitudes 2^-10 ..
// 2688), so the product is taken in f16: a code byte maps to its two e2m1
// values as f16 through a 256-entry table in shared memory, times the scale
// converted to f16.  The fp32 global multipliers are applied by the attention.
template <int D>
__global__ void __launch_bounds__(256) kv_dequant_kernel(const uint8_t* __restrict__ kc, const uint8_t* __restrict__ vc,
                                                         const uint8_t* __restrict__ ksf, const uint8_t* __restrict__ vsf,
                                                         const int32_t* __restrict__ block_table, int first, int tokens,
                                                         int page_size,
                                                         int64_t data_page, int64_t data_row, int64_t data_head,
                                                         int64_t sf_page, int64_t sf_row, int64_t sf_head,
                                                         __half* __restrict__ k_out, __half* __restrict__ vt_out,
                                                         int64_t k_head_stride, int64_t vt_head_stride, int64_t vt_row) {
  constexpr int PARTS = D / 32;          // threads per token
  constexpr int TOK = 256 / PARTS;       // tokens per pass of the CTA
  constexpr int VT_PITCH = 64 + 8;       // halves per V^T row in shared memory (16-byte aligned rows)
  __shared__ __align__(16) __half vtile[D][VT_PITCH];
  __shared__ __half2 pair_lut[256];  // code byte -> (low-nibble value, high-nibble value)
  {
    constexpr float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const uint32_t b = threadIdx.x, lo = b & 0xF, hi = b >> 4;
    const float vlo = (lo & 8) ? -mag[lo & 7] : mag[lo & 7], vhi = (hi & 8) ? -mag[hi & 7] : mag[hi & 7];
    pair_lut[b] = __floats2half2_rn(vlo, vhi);
  }
  __syncthreads();
  const int head = blockIdx.y;
  const int t0 = first + blockIdx.x * 64;
  const int part = threadIdx.x % PARTS;
  for (int tl = threadIdx.x / PARTS; tl < 64; tl += TOK) {
    const int tok = t0 + tl;
    uint4 kcode = make_uint4(0, 0, 0, 0), vcode = kcode;
    uint32_t kscale = 0, vscale = 0;
    if (tok < tokens) {
      const int64_t page = block_table[tok / page_size], entry = tok % page_size;
      const int64_t dbase = page * data_page + entry * data_row + (int64_t)head * data_head + part * 16;
      const int64_t sbase = page * sf_page + entry * sf_row + (int64_t)head * sf_head + part * 2;
      kcode = __ldg(reinterpret_cast<const uint4*>(kc + dbase));
      vcode = __ldg(reinterpret_cast<const uint4*>(vc + dbase));
      kscale = __ldg(reinterpret_cast<const unsigned short*>(ksf + sbase));
      vscale = __ldg(reinterpret_cast<const unsigned short*>(vsf + sbase));
    }
    const uint32_t kw[4] = {kcode.x, kcode.y, kcode.z, kcode.w}, vw[4] = {vcode.x, vcode.y, vcode.z, vcode.w};
    uint4 kout[4];
    __half2* ko = reinterpret_cast<__half2*>(kout);
#pragma unroll
    for (int g = 0; g < 2; ++g) {  // two 16-value scale groups
      const __half ksh = __float2half_rn(e4m3_to_f((kscale >> (8 * g)) & 0xFF));
      const __half vsh = __float2half_rn(e4m3_to_f((vscale >> (8 * g)) & 0xFF));
      const __half2 ks2 = __halves2half2(ksh, ksh), vs2 = __halves2half2(vsh, vsh);
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const uint32_t kb = kw[2 * g + w], vb = vw[2 * g + w];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          ko[(2 * g + w) * 4 + j / 2] = __hmul2(pair_lut[(kb >> (4 * j)) & 0xFF], ks2);
          const __half2 v2 = __hmul2(pair_lut[(vb >> (4 * j)) & 0xFF], vs2);
          const int d = part * 32 + (2 * g + w) * 8 + j;
          vtile[d][tl] = __low2half(v2);
          vtile[d + 1][tl] = __high2half(v2);
        }
      }
    }
    if (tok < tokens) {
      uint4* dst = reinterpret_cast<uint4*>(k_out + head * k_head_stride + (int64_t)tok * D + part * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = kout[i];
    }
  }
  __syncthreads();
  // V^T: row d gets this CTA's 64 tokens (128 bytes) as 8 pieces of 16 bytes.
  const int valid = min(64, (int)(vt_row - t0));  // vt_row is a multiple of 64, so 64
  for (int i = threadIdx.x; i < D * 8; i += blockDim.x) {
    const int d = i / 8, piece = i % 8;
    if (piece * 8 < valid)
      *reinterpret_cast<uint4*>(vt_out + head * vt_head_stride + (int64_t)d * vt_row + t0 + piece * 8) =
          *reinterpret_cast<const uint4*>(&vtile[d][piece * 8]);
  }
}

// Element-wise conversion check: E2M1 codes of in[i] (pairs packed as the
// kernels pack them), E4M3 codes, and expf / sigmoid of in[i].
__global__ void convert_probe_kernel(const float* __restrict__ in, uint8_t* __restrict__ e2m1_pairs,
                                     uint8_t* __restrict__ e4m3, float* __restrict__ ex, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = in[i];
  e4m3[i] = (uint8_t)f_to_e4m3(v);
  ex[2 * i] = expf(v);
  ex[2 * i + 1] = sigmoid_f(v);
  if ((i & 1) == 0 && i + 1 < n) e2m1_pairs[i >> 1] = (uint8_t)f2_to_e2m1x2(v, in[i + 1]);
  if ((i & 7) == 0 && i + 7 < n) {
    float v8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v8[j] = in[i + j];
    reinterpret_cast<uint32_t*>(e2m1_pairs + (n >> 1))[i >> 3] = f8_to_e2m1x8(v8);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

namespace qi {
bool kv_dequant_request_valid(const QiKvView* kv, const int32_t* block_table, int first, int tokens,
                              const void* k_out, int64_t k_capacity, const void* vt_out, int64_t vt_row) {
  if (!kv || !block_table || tokens < 1 || first < 0 || first % 64 || first >= tokens || !k_out || !vt_out ||
      k_capacity < tokens || vt_row < tokens || vt_row % 64)
    return false;
  if (!kv->k_cache || !kv->v_cache || !kv->k_scales || !kv->v_scales || kv->kvheads < 1 || kv->page_size < 1 ||
      (kv->head_dim != 64 && kv->head_dim != 128))
    return false;
  // 16-byte code loads and 2-byte scale loads per 32 values of a token
  return aligned16(kv->k_cache) && aligned16(kv->v_cache) && !(kv->data_page % 16) && !(kv->data_row % 16) &&
         !(kv->data_head % 16) && !(reinterpret_cast<uintptr_t>(kv->k_scales) & 1) &&
         !(reinterpret_cast<uintptr_t>(kv->v_scales) & 1) && !(kv->sf_page % 2) && !(kv->sf_row % 2) &&
         !(kv->sf_head % 2) && aligned16(k_out) && aligned16(vt_out);
}
}  // namespace qi

extern "C" {

int qi_norm_pack(const void* x, const void* residual, const void* gamma, const float* global_scale, void* q,
                 void* scales, void* updated, int rows, int hidden, float eps, float weight_offset,
                 cudaStream_t stream) {
  QI_BIND(stream, x);
  if (rows < 1 || hidden < 64 || hidden % 64 || hidden > 16384 || !x || !gamma || !global_scale || !q || !scales)
    return (int)cudaErrorInvalidValue;
  if (!aligned16(x) || (residual && !aligned16(residual)) || (updated && !aligned16(updated)) || !aligned16(gamma) ||
      (reinterpret_cast<uintptr_t>(q) & 7))
    return (int)cudaErrorInvalidValue;
  const int threads = ((hidden / 16) + 31) / 32 * 32;
  norm_kernel<true><<<rows, threads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
      static_cast<const __nv_bfloat16*>(gamma), global_scale, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales),
      static_cast<__nv_bfloat16*>(updated), nullptr, hidden, eps, weight_offset);
  return (int)cudaPeekAtLastError();
}

int qi_rms_norm(const void* x, const void* residual, const void* gamma, void* out, void* updated, int rows,
                int hidden, float eps, float weight_offset, cudaStream_t stream) {
  QI_BIND(stream, x);
  if (rows < 1 || hidden < 64 || hidden % 64 || hidden > 16384 || !x || !gamma || !out)
    return (int)cudaErrorInvalidValue;
  if (!aligned16(x) || (residual && !aligned16(residual)) || !aligned16(out) || !aligned16(gamma) ||
      (updated && !aligned16(updated)))
    return (int)cudaErrorInvalidValue;
  const int threads = ((hidden / 16) + 31) / 32 * 32;
  norm_kernel<false><<<rows, threads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
      static_cast<const __nv_bfloat16*>(gamma), nullptr, nullptr, nullptr, static_cast<__nv_bfloat16*>(updated),
      static_cast<__nv_bfloat16*>(out), hidden, eps, weight_offset);
  return (int)cudaPeekAtLastError();
}

int nvfp4_norm_pack_launch(const void* x, const void* r, const void* w, const void* global, void* q, void* scale,
                           void* updated, int rows, cudaStream_t stream) {
  if (rows < 1 || rows > 8192 || !x || !r || !w || !global || !q || !scale || !updated)
    return (int)cudaErrorInvalidValue;
  return qi_norm_pack(x, r, w, static_cast<const float*>(global), q, scale, updated, rows, 5120, 1e-6f, 1.0f, stream);
}

int nvfp4_norm_pack_metadata(int* out) {
  if (!out) return (int)cudaErrorInvalidValue;
  cudaFuncAttributes attr{};
  const cudaError_t status = cudaFuncGetAttributes(&attr, norm_kernel<true>);
  if (status != cudaSuccess) return (int)status;
  out[0] = attr.numRegs;
  out[1] = (int)attr.sharedSizeBytes;
  out[2] = (int)attr.localSizeBytes;
  return 0;
}

int qi_qk_rope_kv_append(const QiFront* p, cudaStream_t stream) {
  QI_BIND(stream, p ? p->qkv : nullptr);
  if (!p || p->rows < 1 || p->qheads < 1 || p->kvheads < 1 || !p->qkv || !p->q_weight || !p->k_weight ||
      !p->cos_sin || !p->positions || !p->q || p->page_size < 1 || p->pages < 0)
    return (int)cudaErrorInvalidValue;
  if (p->qheads % p->kvheads) return (int)cudaErrorInvalidValue;
  if (p->slot_rows > 0 && (!p->slots || !p->k_global || !p->v_global || !p->k_cache || !p->v_cache ||
                           !p->k_scales || !p->v_scales))
    return (int)cudaErrorInvalidValue;
  if (p->slot_rows > p->rows) return (int)cudaErrorInvalidValue;
  // 16-byte loads / stores of 8 bf16 values (and of 8 fp32 cos/sin values),
  // 4-byte code stores
  const int d = p->head_dim;
  if (!aligned16(p->qkv) || !aligned16(p->q) || (p->gate && !aligned16(p->gate)) || !aligned16(p->cos_sin) ||
      !aligned16(p->q_weight) || !aligned16(p->k_weight) || p->input_row % 8 || p->q_row % 8 ||
      (p->gate && p->gate_row % 8) || p->cos_row % (p->cos_float ? 4 : 8))
    return (int)cudaErrorInvalidValue;
  if (p->slot_rows > 0 &&
      ((reinterpret_cast<uintptr_t>(p->k_cache) & 3) || (reinterpret_cast<uintptr_t>(p->v_cache) & 3) ||
       p->data_page % 4 || p->data_row % 4 || p->data_head % 4))
    return (int)cudaErrorInvalidValue;
  if (d != 64 && d != 128 && d != 256) return (int)cudaErrorInvalidValue;
  const int hpw = 32 / (d / 16);
  const int tasks = (p->qheads + hpw - 1) / hpw + (p->kvheads + hpw - 1) / hpw;
  // one warp per task; the row's tasks split evenly over 1..8-warp CTAs
  const int groups = (tasks + 7) / 8;
  const int warps = (tasks + groups - 1) / groups;
  const dim3 grid(p->rows, groups);
  switch (d) {
    case 64: front_kernel<64><<<grid, warps * 32, 0, stream>>>(*p); break;
    case 128: front_kernel<128><<<grid, warps * 32, 0, stream>>>(*p); break;
    default: front_kernel<256><<<grid, warps * 32, 0, stream>>>(*p); break;
  }
  return (int)cudaPeekAtLastError();
}

int qi_qk_rope_kv_append_resources(int* out) {
  if (!out) return (int)cudaErrorInvalidValue;
  cudaFuncAttributes a{};
  int occupancy = 0;
  cudaError_t e = cudaFuncGetAttributes(&a, front_kernel<128>);
  if (e != cudaSuccess) return (int)e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occupancy, front_kernel<128>, 192, 0);
  if (e != cudaSuccess) return (int)e;
  out[0] = (int)sizeof(QiFront);
  out[1] = a.numRegs;
  out[2] = (int)a.sharedSizeBytes;
  out[3] = (int)a.localSizeBytes;
  out[4] = occupancy;
  return 0;
}

int nvfp4_attention_front(RefFront f, cudaStream_t stream) {
  // The reference's D256 ABI: no MRoPE, rotary covering the whole head.
  if (f.rows < 1 || f.qheads < 1 || f.kvheads < 1 || f.rotary != 256 || f.mrope_h || f.mrope_w)
    return (int)cudaErrorInvalidValue;
  QiFront p{};
  p.qkv = f.qkv;
  p.q_weight = f.qw;
  p.k_weight = f.kw;
  p.cos_sin = f.cos_sin;
  p.positions = f.positions;
  p.slots = f.slots;
  p.k_global = f.k_scale;
  p.v_global = f.v_scale;
  p.k_cache = f.k;
  p.v_cache = f.v;
  p.k_scales = f.ks;
  p.v_scales = f.vs;
  p.q = f.q;
  p.gate = f.gate;
  p.status = nullptr;
  p.rows = f.rows;
  p.qheads = f.qheads;
  p.kvheads = f.kvheads;
  p.head_dim = 256;
  p.slot_rows = f.slot_rows;
  p.pages = f.pages;
  p.page_size = f.page_size;
  p.cos_float = f.cos_float;
  p.pos_long = f.pos_long;
  p.slot_long = f.slot_long;
  p.input_row = f.input_row;
  p.cos_row = f.cos_row;
  p.q_row = (int64_t)f.qheads * 256;
  p.gate_row = (int64_t)f.qheads * 256;
  p.data_page = f.data_page;
  p.data_row = f.data_row;
  p.data_head = f.data_head;
  p.sf_page = f.sf_page;
  p.sf_row = f.sf_row;
  p.sf_head = f.sf_head;
  p.eps = f.epsilon;
  p.weight_offset = 1.0f;
  if (f.pos_t != 1) return (int)cudaErrorInvalidValue;
  return qi_qk_rope_kv_append(&p, stream);
}

int nvfp4_attention_front_resources(int* out) {
  if (!out) return (int)cudaErrorInvalidValue;
  const int rc = qi_qk_rope_kv_append_resources(out);
  if (rc) return rc;
  out[0] = (int)sizeof(RefFront);
  return 0;
}

int qi_swiglu_nvfp4(const void* gate_up, int64_t gu_row, int rows, int inter, const float* global_scale, void* q,
                    int64_t q_row, void* scales, cudaStream_t stream) {
  QI_BIND(stream, gate_up);
  if (rows < 1 || inter < 128 || inter % 128 || gu_row < 2 * (int64_t)inter || gu_row % 8 || q_row < inter / 2 ||
      q_row % 8 || !gate_up || !global_scale || !q || !scales)
    return (int)cudaErrorInvalidValue;
  if (!aligned16(gate_up) || (reinterpret_cast<uintptr_t>(q) & 7)) return (int)cudaErrorInvalidValue;
  const int groups = inter / 16;
  const int64_t gp = ((int64_t)groups + 3) / 4 * 4;
  const int64_t threads = (int64_t)rows * groups;
  swiglu_nvfp4_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(gate_up), gu_row, rows, groups, global_scale, static_cast<uint8_t*>(q), q_row,
      static_cast<uint8_t*>(scales), gp);
  return (int)cudaPeekAtLastError();
}

static int gate_fp8_launch(const void* out, const void* gate, int64_t out_row, int64_t gate_row,
                           int64_t gate_head_stride, int head_dim, void* fp8, int64_t fp8_row, float* scale,
                           const float* static_scale, int rows, int cols, cudaStream_t stream) {
  QI_BIND(stream, out);
  if (rows < 1 || cols < 16 || cols % 16 || cols > 16384 || !out || !gate || !fp8 || !(scale || static_scale) ||
      head_dim < 16 ||
      head_dim % 16 || cols % head_dim || gate_head_stride < 0 || gate_head_stride % 8 ||
      (cols > head_dim && gate_head_stride < head_dim))
    return (int)cudaErrorInvalidValue;
  if (!aligned16(out) || !aligned16(gate) || !aligned16(fp8) || out_row % 8 || gate_row % 8 || fp8_row % 16)
    return (int)cudaErrorInvalidValue;
  const int threads = ((cols / 16) + 31) / 32 * 32;
  gate_fp8_kernel<<<rows, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(out),
                                                static_cast<const __nv_bfloat16*>(gate), out_row, gate_row, head_dim,
                                                gate_head_stride, static_cast<uint8_t*>(fp8), fp8_row, scale, cols,
                                                static_scale);
  return (int)cudaPeekAtLastError();
}

int qi_gate_fp8_heads(const void* out, const void* gate, int64_t out_row, int64_t gate_row, int64_t gate_head_stride,
                      int head_dim, void* fp8, int64_t fp8_row, float* scale, int rows, int cols,
                      cudaStream_t stream) {
  if (!scale) return (int)cudaErrorInvalidValue;
  return gate_fp8_launch(out, gate, out_row, gate_row, gate_head_stride, head_dim, fp8, fp8_row, scale, nullptr, rows,
                         cols, stream);
}

int qi_gate_fp8_static(const void* out, const void* gate, int64_t out_row, int64_t gate_row,
                       int64_t gate_head_stride, int head_dim, void* fp8, int64_t fp8_row, const float* scale,
                       int rows, int cols, cudaStream_t stream) {
  if (!scale) return (int)cudaErrorInvalidValue;
  return gate_fp8_launch(out, gate, out_row, gate_row, gate_head_stride, head_dim, fp8, fp8_row, nullptr, scale, rows,
                         cols, stream);
}

int qi_gate_fp8(const void* out, const void* gate, int64_t out_row, int64_t gate_row, void* fp8, int64_t fp8_row,
                float* scale, int rows, int cols, cudaStream_t stream) {
  return qi_gate_fp8_heads(out, gate, out_row, gate_row, 0, cols, fp8, fp8_row, scale, rows, cols, stream);
}

int qi_nvfp4_quantize(const float* w, int64_t rows, int k, const float* global_scale, void* q, void* scales,
                      cudaStream_t stream) {
  QI_BIND(stream, w);
  if (rows < 1 || k < 64 || k % 64 || !w || !global_scale || !q || !scales || !aligned16(w))
    return (int)cudaErrorInvalidValue;
  const int64_t work = rows * (k / 16);
  const int threads = 256;
  const int64_t blocks = (work + threads - 1) / threads;
  if (blocks > 0x7fffffff) return (int)cudaErrorInvalidValue;
  nvfp4_quant_kernel<<<(unsigned)blocks, threads, 0, stream>>>(w, rows, k, global_scale, static_cast<uint8_t*>(q),
                                                               static_cast<uint8_t*>(scales));
  return (int)cudaPeekAtLastError();
}

int qi_fp8_quantize_rows(const float* w, int rows, int k, void* q, float* scales, cudaStream_t stream) {
  QI_BIND(stream, w);
  if (rows < 1 || k < 1 || !w || !q || !scales) return (int)cudaErrorInvalidValue;
  fp8_rows_kernel<<<rows, 256, 0, stream>>>(w, k, static_cast<uint8_t*>(q), scales);
  return (int)cudaPeekAtLastError();
}

int qi_kv_dequant_range(const QiKvView* kv, const int32_t* block_table, int first, int tokens, void* k_out,
                        int64_t k_capacity, void* vt_out, int64_t vt_row, cudaStream_t stream) {
  QI_BIND(stream, k_out);
  if (!kv_dequant_request_valid(kv, block_table, first, tokens, k_out, k_capacity, vt_out, vt_row))
    return (int)cudaErrorInvalidValue;
  const dim3 grid((tokens - first + 63) / 64, kv->kvheads);
  const int64_t ks = k_capacity * kv->head_dim, vs = (int64_t)kv->head_dim * vt_row;
#define QI_KVD(DD)                                                                                                  \
  kv_dequant_kernel<DD><<<grid, 256, 0, stream>>>(                                                                  \
      static_cast<const uint8_t*>(kv->k_cache), static_cast<const uint8_t*>(kv->v_cache),                          \
      static_cast<const uint8_t*>(kv->k_scales), static_cast<const uint8_t*>(kv->v_scales), block_table, first,    \
      tokens, kv->page_size, kv->data_page, kv->data_row, kv->data_head, kv->sf_page, kv->sf_row, kv->sf_head,     \
      static_cast<__half*>(k_out), static_cast<__half*>(vt_out), ks, vs, vt_row)
  switch (kv->head_dim) {
    case 64: QI_KVD(64); break;
    case 128: QI_KVD(128); break;
    default: return (int)cudaErrorInvalidValue;
  }
#undef QI_KVD
  return (int)cudaPeekAtLastError();
}

int qi_kv_dequant(const QiKvView* kv, const int32_t* block_table, int tokens, void* k_out, void* vt_out,
                  int64_t vt_row, cudaStream_t stream) {
  return qi_kv_dequant_range(kv, block_table, 0, tokens, k_out, tokens, vt_out, vt_row, stream);
}

int qi_convert_probe(const float* in, void* e2m1_pairs, void* e4m3, float* ex, int n, cudaStream_t stream) {
  QI_BIND(stream, in);
  if (!in || !e2m1_pairs || !e4m3 || !ex || n < 8 || n % 8) return (int)cudaErrorInvalidValue;
  convert_probe_kernel<<<(n + 255) / 256, 256, 0, stream>>>(in, static_cast<uint8_t*>(e2m1_pairs),
                                                             static_cast<uint8_t*>(e4m3), ex, n);
  return (int)cudaPeekAtLastError();
}

int qi_abi_struct_sizes(int* out) {
  if (!out) return (int)cudaErrorInvalidValue;
  out[0] = (int)sizeof(RefFront);
  out[1] = (int)sizeof(QiFront);
  out[2] = (int)sizeof(QiGemm);
  out[3] = (int)sizeof(QiKvView);
  out[4] = (int)sizeof(QiAttention);
  out[5] = (int)sizeof(QiDecode);
  out[6] = (int)sizeof(QiPagedAttention);
  return 0;
}

}  // extern "C"
