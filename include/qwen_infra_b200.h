/*
 * C ABI of the B200-native folded-VPP prefill kernels (sm_100a).
 *
 * Every entry point takes device pointers, sizes and strides, enqueues on the
 * given stream and returns a cudaError_t value (0 = success); invalid
 * arguments return cudaErrorInvalidValue (1) before anything is launched.
 * Device-detected problems are never a trap: kernels OR a code into the
 * optional `status` word (QI_STATUS_* below), which the caller reads back.
 *
 * Interfaces replaced (paths inside the reference project,
 * Nicko-F/qwen3.8-sm120-vpp-bucket-attention):
 *   nvfp4_norm_pack_launch / _metadata  <- src/qwen_infra/kernels/nvfp4_norm_pack.cu:68-85
 *   nvfp4_attention_front / _resources  <- src/qwen_infra/kernels/nvfp4_attention_front.cu:12-23,114-127
 *   qi_norm_pack          generalises nvfp4_norm_pack_launch (any H % 64 == 0, optional residual)
 *   qi_rms_norm           final norm of the last virtual stage (vpp/model.py:112-114)
 *   qi_qk_rope_kv_append  generalises nvfp4_attention_front (D in {64,128,256}, status word)
 *   qi_gate_fp8           store_final_fp8, src/qwen_infra/kernels/nvfp4_bucket_xqa.cu:48-66,
 *                         with a per-token scale
 *   qi_gemm               FlashInfer mm_fp4 called at src/qwen_infra/vpp/producer.py:29-45,
 *                         vLLM scaled_fp4_quant at producer.py:200-206 (fused epilogue),
 *                         and the FP8 O projection (kernels/nvfp4_attention_fusion.py:46)
 *   qi_kv_dequant +
 *   qi_prefill_attention  FlashInfer paged prefill attention selected at src/qwen_infra/config.py:80
 *   qi_nvfp4_quantize / qi_fp8_quantize_rows  weight preparation (checkpoint NVFP4 / FP8 layouts)
 */
#ifndef QWEN_INFRA_B200_H
#define QWEN_INFRA_B200_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QI_STATUS_BAD_KV_SCALE 1
#define QI_STATUS_WAIT_TIMEOUT 2
#define QI_STATUS_BAD_SLOT 4
#define QI_STATUS_BAD_LENGTH 8 /* decode: a length past its page-table row (clamped) */

/* ---- fused residual + RMSNorm -> NVFP4 --------------------------------- */

/* Reference ABI (nvfp4_norm_pack.cu:68): H = 5120, Gemma (1+w), eps 1e-6.
 * x, r, updated: bf16 [rows, 5120]; w: bf16 [5120]; global: fp32 device
 * scalar; q: u8 [rows, 2560]; scale: u8 [ceil(rows/128)*128, 320] swizzled. */
int nvfp4_norm_pack_launch(const void* x, const void* r, const void* w, const void* global, void* q,
                           void* scale, void* updated, int rows, cudaStream_t stream);
int nvfp4_norm_pack_metadata(int* out); /* out[3]: registers, static smem, local bytes */

/* Any hidden % 64 == 0 (<= 16384).  residual may be NULL (first layer);
 * updated may be NULL.  weight_offset = 1 for the Gemma (1+w) form, 0 for w. */
int qi_norm_pack(const void* x, const void* residual, const void* gamma, const float* global_scale, void* q,
                 void* scales, void* updated, int rows, int hidden, float eps, float weight_offset,
                 cudaStream_t stream);

/* Same norm, bf16 normalised output [rows, hidden]. */
int qi_rms_norm(const void* x, const void* residual, const void* gamma, void* out, void* updated, int rows,
                int hidden, float eps, float weight_offset, cudaStream_t stream);

/* ---- QK-norm + RoPE + gate split + NVFP4 paged KV append --------------- */

/* Byte-for-byte the reference's parameter struct (nvfp4_attention_front.cu:12-23). */
typedef struct RefFront {
  const void *qkv, *qw, *kw;
  const void *cos_sin, *positions, *slots;
  const float *k_scale, *v_scale;
  uint8_t *k, *v, *ks, *vs;
  void *q, *gate;
  int rows, qheads, kvheads, rotary, slot_rows, pages, page_size;
  int cos_float, pos_long, slot_long, mrope_h, mrope_w;
  int64_t input_row, cos_row, pos_m, pos_t;
  int64_t data_page, data_row, data_head, sf_page, sf_row, sf_head;
  float epsilon;
} RefFront;

/* Reference ABI: head_dim 256, rotary == 256 (MRoPE sections rejected). */
int nvfp4_attention_front(RefFront p, cudaStream_t stream);
int nvfp4_attention_front_resources(int* out); /* sizeof, regs, smem, local, occupancy */

/* qkv row: per Q head [q(D) | gate(D)], then K heads, then V heads (bf16).
 * cos_sin [maxpos, D]: cos in [0, D/2), sin in [D/2, D).  Caches:
 * data [pages, page_size, Hkv, D/2] u8 and scales [.., D/16] E4M3 addressed
 * through the strides below (bytes).  k_global / v_global are the fp32
 * dequantisation multipliers: scale = e4m3(amax / (6 g)). */
typedef struct QiFront {
  const void *qkv, *q_weight, *k_weight, *cos_sin, *positions, *slots;
  const float *k_global, *v_global;
  void *k_cache, *v_cache, *k_scales, *v_scales, *q, *gate;
  int* status;
  int rows, qheads, kvheads, head_dim, slot_rows, pages, page_size;
  int cos_float, pos_long, slot_long;
  int64_t input_row, cos_row, q_row, gate_row;
  int64_t data_page, data_row, data_head, sf_page, sf_row, sf_head;
  float eps, weight_offset;
} QiFront;

int qi_qk_rope_kv_append(const QiFront* p, cudaStream_t stream);
int qi_qk_rope_kv_append_resources(int* out);

/* ---- SiLU-and-mul + NVFP4 of the gate_up GEMM output -------------------
 * Replaces the reference's act_fn + scaled_fp4_quant(is_sf_swizzled_layout=True)
 * after gate_up_proj (src/qwen_infra/producer.py:200-206).  gate_up: bf16
 * [rows, 2*inter] (row stride gu_row elements) as written by qi_gemm with the
 * gate/up weight rows interleaved in 128-row blocks; out: codes [rows, inter/2]
 * (row stride q_row bytes) and swizzled scales (128 x 4 layout) of K = inter.
 * act = bf16(silu(gate) * up); scale = e4m3(min(amax*g/6, 448)). */
int qi_swiglu_nvfp4(const void* gate_up, int64_t gu_row, int rows, int inter, const float* global_scale, void* q,
                    int64_t q_row, void* scales, cudaStream_t stream);

/* ---- LM head + greedy sampling of the output token ----------------------
 * Replaces the reference's LM head and temperature-0 sampling of the one
 * output token (src/qwen_infra/cli.py:145; logical rank 0, vpp/runner.py:324-352).
 * hidden: bf16 [rows, dim] final-normed (row stride hidden_row elements);
 * weight: bf16 [vocab, dim]; logits: optional fp32 [rows, vocab] (NULL: not
 * written); tokens: int32 [rows], argmax with the lowest index on ties (-1 if
 * every logit is NaN).  rows <= 8, dim % 8 == 0, dim <= 8192.  workspace:
 * qi_lm_head_workspace_bytes() bytes, 8-byte aligned, zero-filled before the
 * first call and left zero by every call; calls that overlap on the GPU need
 * separate workspaces. */
int qi_lm_head_argmax(const void* hidden, int64_t hidden_row, int rows, int dim, const void* weight, int vocab,
                      float* logits, void* workspace, int* tokens, cudaStream_t stream);
int qi_lm_head_workspace_bytes(void);

/* ---- attention output x sigmoid(gate) -> FP8 (per-token scale) --------- */
int qi_gate_fp8(const void* out, const void* gate, int64_t out_row, int64_t gate_row, void* fp8, int64_t fp8_row,
                float* scale, int rows, int cols, cudaStream_t stream);
/* The same with the gate read per head: column c at gate + row * gate_row +
 * (c / head_dim) * gate_head_stride + c % head_dim (elements), e.g. in place in
 * the QKV projection output (gate = qkv + D, gate_head_stride = 2D), which
 * spares the front kernel its gate copy. */
int qi_gate_fp8_heads(const void* out, const void* gate, int64_t out_row, int64_t gate_row, int64_t gate_head_stride,
                      int head_dim, void* fp8, int64_t fp8_row, float* scale, int rows, int cols,
                      cudaStream_t stream);
/* The reference's own form of the epilogue (store_final_fp8,
 * nvfp4_bucket_xqa.cu:48-66): one static per-tensor scale read from the
 * device scalar `scale`, fp8 = e4m3_satfinite(bf16(out * bf16(sigmoid(gate))) / scale);
 * no per-token scale is written.  Gate addressing as qi_gate_fp8_heads. */
int qi_gate_fp8_static(const void* out, const void* gate, int64_t out_row, int64_t gate_row,
                       int64_t gate_head_stride, int head_dim, void* fp8, int64_t fp8_row, const float* scale,
                       int rows, int cols, cudaStream_t stream);

/* ---- tcgen05 GEMM: D[m, n] = A[m, k] . B[n, k]^T ------------------------ */
#define QI_GEMM_NVFP4 0 /* kind::mxf4nvf4, E2M1 with 16-element E4M3 block scales */
#define QI_GEMM_E4M3 1  /* kind::f8f6f4, E4M3 x E4M3 */

#define QI_EPI_BF16 0          /* out bf16 = acc * alpha */
#define QI_EPI_F32 1           /* out fp32 = acc * alpha */
#define QI_EPI_SWIGLU_NVFP4 2  /* 256-col tile = 128 gate + 128 up cols -> NVFP4 act */
#define QI_EPI_BF16_ROWCOL 3   /* out bf16 = acc * row_scale[m] * col_scale[n] */

typedef struct QiGemm {
  int kind, epilogue;
  int m, n, k; /* k in elements; n % 256 == 0; k % 256 == 0 (NVFP4) / % 128 (E4M3) */
  const void *a, *b;     /* row-major, K contiguous; NVFP4 packs two codes per byte */
  const void *sfa, *sfb; /* swizzled block scales of A and B (NVFP4) */
  const float* alpha;    /* device scalar, or NULL to use alpha_value */
  float alpha_value;
  const float *row_scale, *col_scale;
  void* out;
  int64_t ldo; /* elements */
  void *act_q, *act_sf;  /* QI_EPI_SWIGLU_NVFP4: [m, n/4] bytes and swizzled scales of K = n/2 */
  const float* act_global;
  int64_t act_ld; /* bytes */
  int* status;
} QiGemm;

int qi_gemm(const QiGemm* g, cudaStream_t stream);
int qi_gemm_resources(int* out); /* dynamic smem bytes, regs, threads */

/* ---- paged NVFP4 KV -> bf16 K / V^T and causal GQA prefill attention ---- */
typedef struct QiKvView {
  const void *k_cache, *v_cache, *k_scales, *v_scales;
  int kvheads, head_dim, page_size;
  int64_t data_page, data_row, data_head, sf_page, sf_row, sf_head;
} QiKvView;

/* k_out f16 [Hkv, tokens, D]; vt_out f16 [Hkv, D, vt_row] (vt_row % 64 == 0); the
 * values are the exact e2m1 x e4m3 products (global multipliers not applied). */
int qi_kv_dequant(const QiKvView* kv, const int32_t* block_table, int tokens, void* k_out, void* vt_out,
                  int64_t vt_row, cudaStream_t stream);
/* Tokens [first, tokens) only (first % 64 == 0), into K buffers of
 * k_capacity >= tokens rows per head (k_out f16 [Hkv, k_capacity, D]): a
 * caller that keeps the f16 K / V^T of a request across its chunks
 * dequantises each chunk's new tokens once (tokens past `tokens` in the last
 * 64-token group are written as zeros). */
int qi_kv_dequant_range(const QiKvView* kv, const int32_t* block_table, int first, int tokens, void* k_out,
                        int64_t k_capacity, void* vt_out, int64_t vt_row, cudaStream_t stream);

typedef struct QiAttention {
  const void* q;         /* bf16 [rows, Hq*D] (row stride q_row elements) */
  const void* k;         /* f16 [Hkv, kv_tokens, D] (from qi_kv_dequant) */
  const void* vt;        /* f16 [Hkv, D, vt_row] */
  void* out;             /* bf16 [rows, Hq*D] (row stride out_row) */
  const float *k_global, *v_global;
  int* status;
  int rows, history, kv_tokens, qheads, kvheads, head_dim;
  int64_t q_row, out_row, vt_row;
  float softmax_scale;
  /* Optional key-range split workspace (256-byte aligned, zero-filled before
   * its first use; the kernel leaves its counters consistent, so it is reused
   * as is).  With it, the units of the last, partly idle wave of CTAs are
   * split into two key-range halves that combine in the kernel; NULL or too
   * small: no split.  Calls that overlap on the GPU need separate workspaces. */
  void* workspace;
  int64_t workspace_bytes;
} QiAttention;

int qi_prefill_attention(const QiAttention* p, cudaStream_t stream);

/* Bytes of QiAttention.workspace that allow every split the current device's
 * SM count can ask for at this head_dim. */
int qi_prefill_attention_workspace_bytes(int head_dim, int64_t* bytes);

/* Causal GQA prefill attention straight over the paged NVFP4 cache: the
 * kernel's producer warps load each 128-key tile's E2M1 codes and E4M3 scales
 * through the block table and convert them to f16 in shared memory (no
 * dequantised copy of the cache in HBM).  `rows` queries at positions
 * history .. history+rows-1 attend keys 0 .. history+rows-1 of the request
 * whose pages block_table lists (ceil((history+rows)/page_size) entries).
 * page_size a power of two; head_dim 64 or 128; workspace as in QiAttention.
 * Replaces the FlashInfer paged prefill selected at src/qwen_infra/config.py:80. */
typedef struct QiPagedAttention {
  const void* q; /* bf16 [rows, Hq*D] (row stride q_row elements) */
  void* out;     /* bf16 [rows, Hq*D] (row stride out_row) */
  QiKvView kv;
  const int32_t* block_table;
  const float *k_global, *v_global;
  int* status;
  int rows, history, qheads;
  int64_t q_row, out_row;
  float softmax_scale;
  void* workspace;
  int64_t workspace_bytes;
} QiPagedAttention;

int qi_paged_prefill_attention(const QiPagedAttention* p, cudaStream_t stream);

/* qi_kv_dequant + qi_prefill_attention in one call that allocates nothing, for
 * callers that cannot allocate device memory (an allocator callback, or a
 * plugin host that only hands out input and output buffers).  No counterpart in the reference project.  The f16 K / V^T scratch
 * lives in a 32 MiB static device array (and the attention split workspace in
 * a second one of about 21 MB) that every GPU loading this library holds until
 * exit; history + rows is limited to what fits (Hkv * D * 4 bytes
 * per token, plus V^T padding to 64 tokens: 8192 tokens for 8 KV heads of 128),
 * larger calls return cudaErrorInvalidValue.  All calls share the array:
 * calls that overlap on the GPU race, so order them on one stream.  The first
 * call on a device looks up the array's device address.  q / out / strides as
 * in QiAttention. */
int qi_paged_prefill_attention_noalloc(const QiKvView* kv, const int32_t* block_table, const void* q,
                                       int64_t q_row, void* out, int64_t out_row, int rows, int history,
                                       int qheads, const float* k_global, const float* v_global,
                                       float softmax_scale, int* status, cudaStream_t stream);

/* ---- bucket decode attention ------------------------------------------------
 * One query token per request attends its paged NVFP4 K/V (the cache above),
 * the KV cut into 256-token tiles and the tiles into tasks.  Replaces the
 * reference's native-XQA task backend: nvfp4_xqa_assign / nvfp4_xqa_compute /
 * nvfp4_xqa_resources / nvfp4_xqa_scratch_bytes
 * (src/qwen_infra/kernels/nvfp4_bucket_xqa.cu:255-288) with its XQATask /
 * XQARange / XQABucket records (:15-17), plan semantics of
 * kernels/nvfp4_bucket_xqa.py:19-69, on 16-token pages and head_dim 128. */
typedef struct QiDecodeTask { int32_t request, begin, end, stride; } QiDecodeTask; /* tiles begin..end step stride */
typedef struct QiDecodeRange { int32_t first, count; } QiDecodeRange;              /* a request's task slots */
typedef struct QiDecodeBucket { int32_t begin, end; } QiDecodeBucket;              /* a persistent CTA's slots */

typedef struct QiDecode {
  const void* q;                 /* bf16 [batch, qheads, 128], 16-byte aligned */
  QiKvView kv;                   /* head_dim 128, power-of-two page_size; code base and strides % 32, scale % 8 */
  const int32_t* block_table;    /* [batch, table_width] page ids */
  const int32_t* lengths;        /* [batch] keys per request, 0 .. table_width * page_size */
  QiDecodeTask* tasks;           /* [ctas + batch - 1]  plan, written by qi_decode_assign */
  QiDecodeRange* requests;       /* [batch] */
  QiDecodeBucket* buckets;       /* [ctas] */
  int32_t* header;               /* [4]: budget (splits when cyclic), tasks, active CTAs, max tasks per request */
  int32_t* semaphores;           /* [batch * Hkv] zero before the first call; calls leave them zero */
  void* scratch;                 /* qi_decode_scratch_bytes(ctas + batch - 1, Hkv) bytes, 16-byte aligned */
  void* out;                     /* bf16 [batch, qheads, 128]; e4m3 bytes of the same shape with gate */
  const void* gate;              /* NULL, or bf16 [batch, qheads * 128]: gated FP8 output */
  const float* out_scale;        /* with gate: static fp32 output scale */
  const float *k_global, *v_global; /* cache dequantisation multipliers */
  int* status;
  int batch, ctas, table_width;  /* 1..32 requests, batch <= ctas <= 340 task slots */
  int mode;                      /* 0 intervals, 1 cyclic, 2 aligned */
  int persistent;                /* mode 0 only: ctas CTAs each run their bucket of slots */
  int qheads;                    /* qheads / Hkv <= 16 */
  float softmax_scale;
} QiDecode;

int qi_decode_assign(const QiDecode* p, cudaStream_t stream);
int qi_decode_attention(const QiDecode* p, cudaStream_t stream);
/* values[10]: sizeof(QiDecode), registers, shared bytes, local bytes, resident
 * CTAs per SM (groups of <= 8 query heads per KV head), sizeof(QiDecodeTask),
 * sizeof(QiDecodeRange), sizeof(QiDecodeBucket), registers and resident CTAs
 * per SM of the kernel for groups of 9..16. */
int qi_decode_resources(int* values);
uint64_t qi_decode_scratch_bytes(int capacity, int kvheads);

/* ---- weight preparation ------------------------------------------------- */
int qi_nvfp4_quantize(const float* w, int64_t rows, int k, const float* global_scale, void* q, void* scales,
                      cudaStream_t stream);
int qi_fp8_quantize_rows(const float* w, int rows, int k, void* q, float* scales, cudaStream_t stream);

/* Conversion probe (tests): e2m1_pairs gets n/2 bytes packed pairwise and then
 * n/2 bytes packed eight at a time; e4m3[n]; ex[2n] = (expf, sigmoid) pairs. */
int qi_convert_probe(const float* in, void* e2m1_pairs, void* e4m3, float* ex, int n, cudaStream_t stream);

/* Host-only: sizeof(RefFront, QiFront, QiGemm, QiKvView, QiAttention, QiDecode, QiPagedAttention)
 * for ABI checks (out[7]). */
int qi_abi_struct_sizes(int* out);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_INFRA_B200_H */
