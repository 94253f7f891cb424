// LM head + greedy sampling of the bank's output token (P+1).
//
// The reference samples one token per request with temperature 0
// (src/qwen_infra/cli.py:145, on logical rank 0: vpp/runner.py:324-352) from
// the final-normed hidden state of each request's last prompt token.  Here:
// logits[r, v] = <hidden[r], W[v]> over a bf16 LM head [V, H] (NVFP4
// checkpoints keep the LM head unquantised), token[r] = argmax_v logits[r, v]
// with the lowest index on ties.
//
// Memory-bound GEMV (R <= 8 rows against V x H bf16 weights: 1.56 GB read for
// the 27B shape, one pass for all rows): CUDA cores, no tensor cores.  Each
// warp takes 8 vocabulary rows; lane l accumulates the 16-byte chunks l,
// l+32, ... of the row in order with explicitly rounded fp32 multiply and add,
// then the 32 lane sums are combined by an xor butterfly, so the logits are
// reproducible bit for bit on the CPU.  The argmax is folded into 64-bit keys
// (order-preserving float bits, then the complement of the index) and merged
// with atomicMax; the last CTA to finish turns the keys into token ids and
// resets the workspace to zero, so one launch does it all.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "qwen_infra_b200.h"

using namespace qi;

namespace {

constexpr int kWarps = 8, kRowsPerWarp = 8, kMaxRows = 8;
constexpr int kVocabPerCta = kWarps * kRowsPerWarp;

__device__ __forceinline__ uint64_t argmax_key(float v, int idx) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // monotone in v
  return ((uint64_t)ord << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(kWarps * 32) lm_head_kernel(const __nv_bfloat16* __restrict__ hidden,
                                                               int64_t hidden_row, int rows, int dim,
                                                               const __nv_bfloat16* __restrict__ w, int vocab,
                                                               float* __restrict__ logits, uint64_t* keys,
                                                               unsigned* counter, int* __restrict__ tokens) {
  extern __shared__ uint4 sh[];  // hidden rows, bf16, [rows][dim]
  __shared__ uint64_t warp_best[kWarps][kMaxRows];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = dim / 8;  // 16-byte chunks per row
  for (int i = threadIdx.x; i < rows * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i - r * chunks;
    sh[i] = reinterpret_cast<const uint4*>(hidden + (int64_t)r * hidden_row)[c];
  }
  __syncthreads();
  uint64_t best[kMaxRows];
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) best[r] = 0;
  const int v0 = blockIdx.x * kVocabPerCta + warp * kRowsPerWarp;
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int v = v0 + i;
    if (v >= vocab) break;
    const uint4* wr = reinterpret_cast<const uint4*>(w + (int64_t)v * dim);
    float acc[kMaxRows];
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) acc[r] = 0.0f;
    for (int c = lane; c < chunks; c += 32) {
      const uint4 wv = __ldg(wr + c);
      const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv);
      float wf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(wp[e]);
        wf[2 * e] = f.x, wf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        if (r >= rows) break;
        const uint4 hv = sh[r * chunks + c];
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hp[e]);
          acc[r] = __fadd_rn(acc[r], __fmul_rn(wf[2 * e], f.x));
          acc[r] = __fadd_rn(acc[r], __fmul_rn(wf[2 * e + 1], f.y));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) {
      if (r >= rows) break;
      const float logit = warp_sum_butterfly(acc[r]);  // identical in every lane
      if (logits && lane == r) logits[(int64_t)r * vocab + v] = logit;
      if (logit == logit) {  // NaN never wins
        const uint64_t k = argmax_key(logit, v);
        best[r] = k > best[r] ? k : best[r];
      }
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) warp_best[warp][r] = best[r];
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    uint64_t k = 0;
    for (int i = 0; i < kWarps; ++i) k = warp_best[i][threadIdx.x] > k ? warp_best[i][threadIdx.x] : k;
    if (k) atomicMax(reinterpret_cast<unsigned long long*>(keys + threadIdx.x), (unsigned long long)k);
  }
  // Last CTA out: keys -> token ids, then leave the workspace zeroed.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (is_last) {
    __threadfence();
    if (threadIdx.x < rows) {
      const uint64_t k = atomicExch(reinterpret_cast<unsigned long long*>(keys + threadIdx.x), 0ull);
      tokens[threadIdx.x] = k ? (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu)) : -1;
    }
    if (threadIdx.x == 0) atomicExch(counter, 0u);
  }
}

}  // namespace

extern "C" {

int qi_lm_head_argmax(const void* hidden, int64_t hidden_row, int rows, int dim, const void* weight, int vocab,
                      float* logits, void* workspace, int* tokens, cudaStream_t stream) {
  QI_BIND(stream, hidden);
  if (!hidden || !weight || !workspace || !tokens || rows < 1 || rows > kMaxRows || dim < 8 || dim % 8 ||
      dim > 8192 || vocab < 1 || hidden_row < dim || hidden_row % 8)
    return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(hidden) & 15) || (reinterpret_cast<uintptr_t>(weight) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 7))
    return (int)cudaErrorInvalidValue;
  const size_t smem = (size_t)rows * dim * 2;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxRows * 8192 * 2);
    if (e != cudaSuccess) return (int)e;
    configured[dev] = true;
  }
  uint64_t* keys = static_cast<uint64_t*>(workspace);
  unsigned* counter = reinterpret_cast<unsigned*>(keys + kMaxRows);
  const int grid = (vocab + kVocabPerCta - 1) / kVocabPerCta;
  lm_head_kernel<<<grid, kWarps * 32, smem, stream>>>(static_cast<const __nv_bfloat16*>(hidden), hidden_row, rows,
                                                       dim, static_cast<const __nv_bfloat16*>(weight), vocab, logits,
                                                       keys, counter, tokens);
  return (int)cudaPeekAtLastError();
}

int qi_lm_head_workspace_bytes(void) { return (int)(kMaxRows * sizeof(uint64_t) + 8); }

}  // extern "C"
