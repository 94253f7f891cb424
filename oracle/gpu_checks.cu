// GPU-side helpers of the oracle (TEST INFRASTRUCTURE ONLY; built into
// oracle/_ref/ by oracle/build_ref.py with the reference's producer flags:
// -O3 --fmad=false -arch=sm_100a).
//
// * qo_rsqrtf / qo_expf: CUDA's own rsqrtf and expf evaluated on an array, so
//   that the CPU restatement in oracle/producers.py can use the exact values
//   the reference kernels get from these two functions (black-box outputs; the
//   restatement never re-derives them).
// * qo_gate_fp8_static: the reference's FP8 epilogue restated element-wise
//   from src/qwen_infra/kernels/nvfp4_bucket_xqa.cu:56-62 (bf16 sigmoid of the
//   gate with expf, bf16 product, E4M3 with a static scale), so that the
//   product's gate kernel can be compared byte for byte with the reference's
//   arithmetic.  The reference kernel itself is the decode attention, which
//   only runs on sm_120 here.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace {

__global__ void rsqrtf_kernel(const float* in, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = rsqrtf(in[i]);
}

__global__ void expf_kernel(const float* in, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = expf(in[i]);
}

__global__ void gate_fp8_ref_kernel(const __nv_bfloat16* values, const __nv_bfloat16* gates, const float* scale_ptr,
                                    uint8_t* fp8, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float scale = *scale_ptr;
  const float gate = __bfloat162float(gates[i]);
  const float sigmoid = __bfloat162float(__float2bfloat16_rn(1.f / (1.f + expf(-gate))));
  const float gated = __bfloat162float(__float2bfloat16_rn(__bfloat162float(values[i]) * sigmoid));
  const __nv_fp8_e4m3 value(gated / scale);
  fp8[i] = value.__x;
}

int grid(int n) { return (n + 255) / 256; }

}  // namespace

extern "C" {

int qo_rsqrtf(const float* in, float* out, int n, cudaStream_t stream) {
  if (!in || !out || n < 1) return (int)cudaErrorInvalidValue;
  rsqrtf_kernel<<<grid(n), 256, 0, stream>>>(in, out, n);
  return (int)cudaPeekAtLastError();
}

int qo_expf(const float* in, float* out, int n, cudaStream_t stream) {
  if (!in || !out || n < 1) return (int)cudaErrorInvalidValue;
  expf_kernel<<<grid(n), 256, 0, stream>>>(in, out, n);
  return (int)cudaPeekAtLastError();
}

int qo_gate_fp8_static(const void* values, const void* gates, const float* scale, void* fp8, int n,
                       cudaStream_t stream) {
  if (!values || !gates || !scale || !fp8 || n < 1) return (int)cudaErrorInvalidValue;
  gate_fp8_ref_kernel<<<grid(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(values),
                                                   static_cast<const __nv_bfloat16*>(gates), scale,
                                                   static_cast<uint8_t*>(fp8), n);
  return (int)cudaPeekAtLastError();
}

}  // extern "C"
