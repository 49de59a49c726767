/*
 * otf_b200.h -- C ABI of the B200 (sm_100a) quantized-decode library.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t passed as void*, launches asynchronously on that stream and
 * returns an int status (OTF_OK == 0).  Nothing allocates device memory except
 * otf_ar_create (the tensor-parallel receive buffers, once per process group);
 * outputs are caller-owned.  Half-precision tensors are IEEE binary16 bit
 * patterns (uint16_t).  No exceptions cross this boundary.
 *
 * Layouts are the reference package's own (otf_llm, GT-Labs-AI/otf-llm-engine):
 *   packed  uint8 [N, K/4]   code k of row n at bits 2*(k%4) of byte k/4
 *                            (pack_2bit_uint8, otf_llm/symmetric_2bit_engine.py:100-107)
 *   scales  fp16  [N, K/G]   per-group scale (symmetric_2bit_engine.py:190)
 *   zeros   fp16  [N, K/G]   per-group offset, asymmetric layers only
 *                            (otf_llm/otf_2bit_quantizer.py:65-71)
 *   outlier_vals fp16 [N, k] and outlier_idx int64 [k]: fp16 anchor columns
 *                            (symmetric_2bit_engine.py:200-206, :230-232)
 *   weight_int8 int8 [V, D], scales fp16 [V, 1] (symmetric_2bit_engine.py:17-91)
 */
#ifndef OTF_B200_H
#define OTF_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define OTF_API __attribute__((visibility("default")))
#else
#define OTF_API
#endif

/* Status codes. */
#define OTF_OK 0
#define OTF_ERR_INVALID 1      /* bad pointer, size, stride or alignment */
#define OTF_ERR_UNSUPPORTED 2  /* shape/codebook this build cannot run */
#define OTF_ERR_CUDA 3         /* a CUDA runtime call failed (see otf_last_cuda_error) */
#define OTF_ERR_DEVICE 4       /* current device is not sm_100 */

/* Input transforms of otf2b_linear_group (applied to x while the kernel stages it). */
#define OTF_XOP_NONE 0
#define OTF_XOP_RMSNORM 1   /* x <- aux * fp16(x * rsqrt(mean(x^2) + eps)); aux may be NULL (ones) */
#define OTF_XOP_SILU_MUL 2  /* x <- fp16(fp16(silu(x)) * aux) */

/* Flags for otf2b_linear. */
#define OTF_AR_NONE 0
#define OTF_AR_PRODUCE 1
#define OTF_AR_CONSUME 2
#define OTF_AR_MAX_WORLD 8
#define OTF_AR_HANDLE_BYTES 64  /* one cudaIpcMemHandle_t */

#define OTF_FLAG_CLAMP 1u          /* clamp output to [-65504, 65504] (SymmetricOTF2BitLinear) */
#define OTF_FLAG_FORCE_GENERIC 2u  /* use the portable CUDA-core kernel (testing) */

/* Library version as 10000*major + 100*minor + patch. */
OTF_API int otf_version(void);

/* Human-readable name of a status code. */
OTF_API const char* otf_status_string(int status);

/* Last CUDA error code seen by this thread inside the library (cudaError_t as int). */
OTF_API int otf_last_cuda_error(void);

/*
 * Device-side failure flag of the pipelined kernels (synchronous).  Every wait inside a
 * kernel is bounded; if one gives up (a pipeline that never completes), the kernel sets
 * this flag instead of hanging.  The attention kernels set it too when the device-side
 * position is outside [0, max_pos) (they then write nothing).  Returns 1 if set, 0 if not,
 * -1 on a CUDA error; with clear != 0 the flag is reset.  No counterpart in the reference
 * (it has no pipelines).
 */
OTF_API int otf_device_error(int clear);

/*
 * One 2-bit quantized linear layer:
 *   y[m,n] = sum_k fp16(x[m,k]*mask[k]) * (codebook[q[n,k]] * scales[n,k/G] + zeros[n,k/G])
 *            + bias[n] + sum_j x[m, outlier_idx[j]] * outlier_vals[n,j] + residual[m,n]
 * accumulated in fp32 and stored as fp16, clamped to +-65504 when OTF_FLAG_CLAMP is set.
 *
 * Replaces the reference's whole forward for this layer: the mask multiply and
 * dispatch of triton_symmetric_2bit_gemm (otf_llm/otf_triton_2bit_kernel.py:164-194),
 * its native op sym2bit_gemv_cuda / sym2bit_gemv_warp_kernel (:23-113), the LUT
 * fallback (:146-161, :188-194), and the bias / outlier / clamp tail of
 * SymmetricOTF2BitLinear.forward (otf_llm/symmetric_2bit_engine.py:214-235) and
 * OTF2BitLinear.forward (otf_llm/otf_2bit_quantizer.py:193-221, zeros honoured).
 *
 * x: fp16 [M, ldx]; y: fp16 [M, ldy]; codebook: HOST pointer to 4 floats.
 * zeros, mask, outlier_idx/outlier_vals (n_outliers may be 0), bias and residual may be
 * NULL.  residual (fp16 [M, ld_residual]) is this package's fusion of the decoder's
 * skip connection; the reference added it in a separate torch op.
 * The fast path needs a codebook with c0 + c3 == c1 + c2 (every symmetric one),
 * G a multiple of 32, K a multiple of G and 16-byte aligned packed rows;
 * other shapes run a portable CUDA-core kernel.
 */
OTF_API int otf2b_linear(const void* x, int64_t ldx,
                         const uint8_t* packed, int64_t ld_packed,
                         const void* scales, int64_t ld_scales,
                         const void* zeros, int64_t ld_zeros,
                         const float* codebook,
                         const void* mask,
                         const int64_t* outlier_idx, int64_t n_outliers,
                         const void* outlier_vals, int64_t ld_outlier_vals,
                         const void* bias,
                         const void* residual, int64_t ld_residual,
                         void* y, int64_t ldy,
                         int64_t M, int64_t N, int64_t K, int64_t group_size,
                         uint32_t flags, void* stream);

/*
 * Batched and prefill 2-bit linear on the 5th-generation tensor cores: same arguments,
 * layouts and semantics as otf2b_linear, any M >= 1, any codebook.  The weights are
 * dequantised to fp16 exactly as the reference's LUT path does (fp16(c[q] * s), or fp32
 * s*c[q] + z rounded to fp16 for the asymmetric layout) and multiplied by tcgen05.mma
 * (fp32 accumulation in tensor memory).  Symmetric layers with G in {32, 64} write the
 * dequantised weights into tensor memory and feed them as the MMA's A operand (TMA brings
 * codes, scales and x); the others stage fp16 tiles in shared memory.  The fp16 anchors
 * are extra K tiles of the same accumulation.  otf2b_linear routes M >= 9 here by itself
 * (the tensor-memory form; the shared-memory form from M >= 32).
 * Needs 16-byte aligned x rows (ldx % 8 == 0), code rows (ld_packed % 16 == 0) and mask,
 * even scale strides and G in {32, 64, 128, 256}; OTF_ERR_UNSUPPORTED otherwise.
 * Replaces: the LUT dequant + torch matmul of triton_symmetric_2bit_gemm for M > 1
 * (otf_llm/otf_triton_2bit_kernel.py:188-194) and OTF2BitLinear.forward's batched path
 * (otf_llm/otf_2bit_quantizer.py:193-221).
 */
OTF_API int otf2b_gemm_mma(const void* x, int64_t ldx,
                           const uint8_t* packed, int64_t ld_packed,
                           const void* scales, int64_t ld_scales,
                           const void* zeros, int64_t ld_zeros,
                           const float* codebook,
                           const void* mask,
                           const int64_t* outlier_idx, int64_t n_outliers,
                           const void* outlier_vals, int64_t ld_outlier_vals,
                           const void* bias,
                           const void* residual, int64_t ld_residual,
                           void* y, int64_t ldy,
                           int64_t M, int64_t N, int64_t K, int64_t group_size,
                           uint32_t flags, void* stream);

/*
 * One layer of a grouped decode launch (batch 1).  Fields mean what the arguments of
 * otf2b_linear mean; x_op transforms x while the kernel stages it (this package's fusion
 * of the Llama decoder step around the reference's projections):
 *   OTF_XOP_RMSNORM   x <- x_aux * fp16(x * rsqrt(mean(x^2) + eps))   (x_aux: fp16 [K] or NULL)
 *   OTF_XOP_SILU_MUL  x <- fp16(fp16(silu(x)) * x_aux)               (x_aux: fp16 [K])
 * The layer's mask applies after the transform; anchors use the transformed, unmasked x.
 */
typedef struct otf2b_layer {
  const void* x;
  int64_t ldx;
  const uint8_t* packed;
  int64_t ld_packed;
  const void* scales;
  int64_t ld_scales;
  const void* zeros;
  int64_t ld_zeros;
  const float* codebook; /* host pointer to 4 floats */
  const void* mask;
  const int64_t* outlier_idx;
  int64_t n_outliers;
  const void* outlier_vals;
  int64_t ld_outlier_vals;
  const void* bias;
  const void* residual;
  int64_t ld_residual;
  void* y;
  int64_t ldy;
  int64_t N, K, group_size;
  uint32_t flags;
  int32_t x_op;
  const void* x_aux;
  float eps;
  /* Tensor-parallel peer all-reduce (see otf_ar_create; ar == NULL: none).
   *   ar_mode OTF_AR_PRODUCE: the finished rows (fp32, after bias, anchors and residual,
   *     before the clamp) go to receive buffer ar_buf of every rank instead of y; the
   *     layer must be launched alone (n_layers == 1).
   *   ar_mode OTF_AR_CONSUME: x is the sum over ranks of receive buffer ar_buf (rounded to
   *     fp16, clamped), read after every rank has produced all K rows into it; x itself is
   *     not read.  ar_out (fp16 [K], may be NULL) receives that sum once per launch. */
  void* ar;
  int32_t ar_mode;
  int32_t ar_buf;
  void* ar_out;
} otf2b_layer;

/*
 * Up to 4 layers in one launch (q/k/v, or gate/up, of a decoder step).  Layers with the
 * same K, group size and zero-point use share one grid; otherwise they launch one after
 * another.  The reference launched each projection separately
 * (otf_llm/symmetric_2bit_engine.py:214-235 per module call).
 */
OTF_API int otf2b_linear_group(const otf2b_layer* layers, int n_layers, void* stream);

/*
 * Symmetric 2-bit quantizer (replaces Symmetric2BitQuantizer.quantize_tensor,
 * otf_llm/symmetric_2bit_engine.py:109-169; packing as pack_2bit_uint8, :100-107).
 * w: [N, ldw] of w_dtype (OTF_DTYPE_*), ldw a multiple of 4, w aligned to 4 elements.
 * Column impact ||w[:, c]||_2 (* act[c] when act, fp32 [K], is not NULL); the n_outliers
 * largest columns (descending, ties to the lower index) go to outlier_idx (int64 [n_outliers])
 * and outliers (fp16 [N, ldo], column j = fp16(w[:, outlier_idx[j]])), and count as zero in
 * the fit.  Per group of group_size (16, 32, 64, 128 or 256) columns: RMS start and five
 * rounds of nearest-centroid codes + least-squares scale over codebook (4 fp32 values in host
 * memory; NULL = the reference's -1.52, -0.45, 0.45, 1.52).  packed: uint8 [N, ldp] (four
 * codes per byte, code j at bits 2*(j%4)); scales: fp16 [N, lds].  n_outliers = 0 needs no
 * workspace; otherwise workspace (256-byte aligned) of otf2b_quantize_workspace_bytes(N, K).
 * Sums run in a fixed order, so a scale can differ from the torch reference by one fp16 ulp
 * where its fp32 value lies next to an fp16 rounding boundary; codes, indices and anchor
 * values follow the reference.
 */
#define OTF_DTYPE_F16 0
#define OTF_DTYPE_BF16 1
#define OTF_DTYPE_F32 2
OTF_API int64_t otf2b_quantize_workspace_bytes(int64_t N, int64_t K);
OTF_API int otf2b_quantize(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int64_t group_size,
                           const float* act, int64_t n_outliers, const float* codebook, void* workspace,
                           int64_t workspace_bytes, uint8_t* packed, int64_t ldp, void* scales, int64_t lds,
                           void* outliers, int64_t ldo, int64_t* outlier_idx, void* stream);

/*
 * Unpack 2-bit codes to one byte per code: codes[n,k] = q[n,k] in {0..3}.
 * The inverse of pack_2bit_uint8 (otf_llm/symmetric_2bit_engine.py:100-107) and the
 * code-extraction step of unpack_2bit_uint8 (otf_llm/otf_2bit_quantizer.py:58-63).
 * Used to prove bit-exact unpacking.  codes: uint8 [N, ld_codes].
 */
OTF_API int otf2b_unpack_codes(const uint8_t* packed, int64_t ld_packed, int64_t N, int64_t K,
                               uint8_t* codes, int64_t ld_codes, void* stream);

/*
 * INT8 shared-vocabulary LM head:
 *   logits[m,v] = scales[v] * sum_d x[m,d] * w[v,d]   (fp32, NaN -> 0, clamped to +-65504)
 * Replaces QuantizedLinearHead.forward (otf_llm/symmetric_2bit_engine.py:75-91).
 * x: fp16 [M, ldx]; w: int8 [V, ldw]; scales: fp16 [V]; logits: fp32 [M, ldl].
 * With 16-byte aligned weight rows (D a multiple of 16) one launch serves up to 8 rows of x
 * (4 at D = 8192), reading the weights once for all of them; each row's logits are
 * bit-identical to a call with that row alone.
 */
OTF_API int otf_i8_head(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scales,
                        float* logits, int64_t ldl, int64_t M, int64_t V, int64_t D, void* stream);

/*
 * Greedy decode step on the INT8 head: argmax[m] = the first index of the largest logit of
 * row m (torch.argmax semantics over QuantizedLinearHead.forward's output, after its
 * nan_to_num), int64 [M], 8-byte aligned; it is also the kernel's reduction buffer.
 * logits may be NULL (then they are not stored).  No reference counterpart as one call:
 * replaces QuantizedLinearHead.forward (otf_llm/symmetric_2bit_engine.py:75-91) followed by
 * torch.argmax over its logits (greedy decoding).
 */
OTF_API int otf_i8_head_argmax(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scales,
                               float* logits, int64_t ldl, int64_t* argmax, int64_t M, int64_t V, int64_t D,
                               void* stream);

/*
 * INT8 embedding gather: out[t,:] = fp16(w[ids[t],:]) * scales[ids[t]] in fp16,
 * bit-identical to QuantizedEmbedding.forward (otf_llm/symmetric_2bit_engine.py:41-47).
 * Ids outside [0, V) produce a zero row and set *bad_ids (device int32, may be NULL) to 1.
 * ids: int64 [n]; out: fp16 [n, ldo].
 */
OTF_API int otf_i8_embed(const int64_t* ids, int64_t n, const int8_t* w, int64_t ldw, const void* scales,
                         void* out, int64_t ldo, int64_t V, int64_t D, int32_t* bad_ids, void* stream);

/*
 * RMSNorm over the last dimension, Llama semantics (transformers LlamaRMSNorm, the norm
 * the reference runner keeps from HF, otf_llm/run_symmetric_2bit.py:139-147):
 *   out[m,:] = w * fp16( x[m,:] * rsqrt(mean(x[m,:]^2) + eps) )   (statistics in fp32)
 * x, w, out: fp16.  w may be NULL (all ones).
 */
OTF_API int otf_rmsnorm(const void* x, int64_t ldx, const void* w, float eps, void* out, int64_t ldo,
                        int64_t M, int64_t K, void* stream);

/*
 * Gated activation of the Llama MLP: out = fp16( fp16(silu(g)) * u ), elementwise over n
 * fp16 values (act_fn(gate_proj(x)) * up_proj(x) in transformers LlamaMLP).
 */
OTF_API int otf_silu_mul(const void* g, const void* u, void* out, int64_t n, void* stream);

/*
 * Tensor-parallel peer all-reduce over NVLink (one process per GPU).  No reference
 * counterpart as a library: it replaces the NCCL all_reduce after each row-parallel
 * o_proj / down_proj that tensor parallelism adds around the reference's
 * SymmetricOTF2BitLinear (otf_llm/symmetric_2bit_engine.py:214-235).
 *
 * otf_ar_create allocates this rank's receive region (two buffers of world x max_elems
 * fp32 slots plus arrival counters) on the current device and writes its CUDA IPC handle
 * (OTF_AR_HANDLE_BYTES) to ipc_handle; the caller exchanges the handles (e.g. an
 * all-gather over the process group) and passes all of them, in rank order, to
 * otf_ar_open, which maps every peer's region.  Producers write rows straight into every
 * peer's region and then add the row count to the peer's arrival counter (release, system
 * scope); a consumer waits until the counter reaches world x rows (bounded: on time-out it
 * raises the otf_device_error flag and carries on), sums the world slots in rank order
 * (identical on every rank) and, as the last consumer CTA of its launch, resets the
 * counter.  Consecutive exchanges must alternate buffers 0 and 1.
 */
typedef struct otf_ar otf_ar;
OTF_API int otf_ar_create(int rank, int world, int64_t max_elems, void* ipc_handle, otf_ar** out);
OTF_API int otf_ar_open(otf_ar* ar, const void* all_handles);
OTF_API int otf_ar_destroy(otf_ar* ar);
/* Push an fp16 vector x[n] (this rank's partial sum) into buffer buf of every rank. */
OTF_API int otf_ar_push(otf_ar* ar, int buf, const void* x, int64_t n, void* stream);
/* Wait for all ranks' n rows in buffer buf and write their fp16 sum to out[n]. */
OTF_API int otf_ar_finish(otf_ar* ar, int buf, void* out, int64_t n, void* stream);

/*
 * A whole batch-1 decode step of a Llama-shaped 2-bit decoder stack in ONE persistent
 * launch (one CTA per SM): per layer RMSNorm -> q/k/v -> (single-position attention:
 * the output of each query head is its KV head's v) -> o + residual -> RMSNorm ->
 * gate/up -> fp16(silu(g)) * u -> down + residual, every projection the fused
 * 2-bit linear of otf2b_linear (mask, anchors, bias, clamp).  Stages are separated by a
 * device-wide barrier; each warp streams its share of every stage's weight tiles through
 * its own copy ring, so the next stage's weights arrive while the barrier and the
 * activation staging run.  No reference counterpart as one call: it replaces the
 * per-module SymmetricOTF2BitLinear.forward calls (otf_llm/symmetric_2bit_engine.py:
 * 214-235) that HF's LlamaDecoderLayer makes for one generated token
 * (otf_llm/run_symmetric_2bit.py:150-187 injects them).
 */
typedef struct otf2b_proj {
  const uint8_t* packed;     /* uint8 [N, ld_packed], ld_packed % 16 == 0 */
  int64_t ld_packed;
  const void* scales;        /* fp16 [N, ld_scales], ld_scales even */
  int64_t ld_scales;
  const void* mask;          /* fp16 [K] or NULL */
  const int64_t* outlier_idx;
  int64_t n_outliers;
  const void* outlier_vals;  /* fp16 [N, ld_outlier_vals] */
  int64_t ld_outlier_vals;
  const void* bias;          /* fp16 [N] or NULL */
  int64_t N, K;
} otf2b_proj;

typedef struct otf2b_decoder_layer {
  otf2b_proj q, k, v, o, gate, up, down;
  const void* input_norm;    /* fp16 [hidden] or NULL (ones) */
  const void* post_norm;     /* fp16 [hidden] or NULL (ones) */
} otf2b_decoder_layer;

typedef struct otf2b_decode_dims {
  int64_t n_layers, hidden, intermediate, heads, kv_heads, head_dim, group_size;
  float eps;
  float codebook[4];         /* affine: c3 - c2 == c1 - c0 */
} otf2b_decode_dims;

/* Bytes of the caller-owned device workspace for these dimensions (16-byte aligned). */
OTF_API int64_t otf2b_decode_workspace_bytes(const otf2b_decode_dims* dims);
/* Validate the layers (host array) and copy their descriptors into the workspace
 * (synchronous; once per stack).  OTF_ERR_UNSUPPORTED for shapes the kernel does not take. */
OTF_API int otf2b_decode_prepare(const otf2b_decoder_layer* layers, const otf2b_decode_dims* dims, void* workspace,
                                 int64_t workspace_bytes);
/* One decode step: h (fp16 [hidden], 16-byte aligned) is the residual stream in and out. */
OTF_API int otf2b_decode_step(const otf2b_decode_dims* dims, void* h, void* workspace, void* stream);

/*
 * Decode attention for a decoder stack with a KV cache (batch 1, grouped-query heads).
 * Replaces the attention of HF's LlamaAttention that the reference runner keeps around its
 * injected projections (otf_llm/run_symmetric_2bit.py:150-187); no reference counterpart
 * as a library.  pos: int32 [1] in device memory, the position of the token being decoded.
 *
 * otf_rope_kv: rotate q (fp16 [heads, head_dim]) and k (fp16 [kv_heads, head_dim]) in place
 * with cos_sin (fp16 [max_pos, 2, head_dim]: HF's cos then sin rows, halves duplicated;
 * rotate_half form, fp16 arithmetic) and write k and v to row pos of the caches
 * (fp16 [max_pos, kv_heads * head_dim]).
 * otf_attn_decode: out (fp16 [heads * head_dim]) = softmax(q k^T * scale) v over cache rows
 * 0..pos, query head j reading KV head j / (heads / kv_heads) (<= 8); split over groups of
 * 64 positions, fp32 arithmetic.  head_dim 64 or 128.  workspace: caller-owned, zeroed once,
 * otf_attn_workspace_bytes(...) bytes.
 * otf_pos_advance: *pos += 1 (the last launch of a token step).
 * Every attention entry point reads pos on the device: a position outside [0, max_pos)
 * writes nothing (no cache row, no output) and raises the otf_device_error flag.
 */
OTF_API int otf_rope_kv(void* q, void* k, const void* v, const void* cos_sin, const int32_t* pos, void* k_cache,
                        void* v_cache, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_pos,
                        void* stream);
OTF_API int64_t otf_attn_workspace_bytes(int64_t kv_heads, int64_t head_dim, int64_t max_pos);
OTF_API int otf_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int32_t* pos, void* out,
                            float scale, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_pos,
                            void* workspace, int64_t workspace_bytes, void* stream);
OTF_API int otf_pos_advance(int32_t* pos, void* stream);
/*
 * otf_rope_kv followed by otf_attn_decode in one launch: q, k, v as the q/k/v projections
 * wrote them (unrotated), the caches get row pos (rotated k, v), out as otf_attn_decode.
 * Same workspace (otf_attn_workspace_bytes).  With 1, 2, 3, 4 or 8 query heads per KV head the
 * splits of a KV head form one thread-block cluster (at most 16 CTAs, 8 for 8 query heads per
 * KV head) and merge over distributed shared memory (the workspace is then not touched); the
 * other ratios, and the batched form, merge through the workspace.  Both merges give the same
 * results within fp32 rounding.
 */
OTF_API int otf_attn_rope_decode(const void* q, const void* k, const void* v, const void* cos_sin, const int32_t* pos,
                                 void* k_cache, void* v_cache, void* out, float scale, int64_t heads,
                                 int64_t kv_heads, int64_t head_dim, int64_t max_pos, void* workspace,
                                 int64_t workspace_bytes, void* stream);

/*
 * otf_attn_rope_decode for `batch` independent sequences in one launch (batched greedy decoding;
 * no counterpart in the reference, whose runner decodes one sequence with HF attention):
 * sequence b reads q + b*ldq, k + b*ldkv, v + b*ldkv, position pos[b], its caches at
 * k_cache/v_cache + b*cache_stride elements (cache_stride >= max_pos * kv_heads * head_dim), and
 * writes out + b*ldo.  workspace: caller-owned, zeroed once, otf_attn_workspace_bytes_batch(...).
 * otf_pos_advance_batch: pos[i] += 1 for i < n.
 */
OTF_API int64_t otf_attn_workspace_bytes_batch(int64_t kv_heads, int64_t head_dim, int64_t max_pos, int64_t batch);
OTF_API int otf_attn_rope_decode_batch(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv,
                                       const void* cos_sin, const int32_t* pos, void* k_cache, void* v_cache,
                                       int64_t cache_stride, void* out, int64_t ldo, float scale, int64_t heads,
                                       int64_t kv_heads, int64_t head_dim, int64_t max_pos, int64_t batch,
                                       void* workspace, int64_t workspace_bytes, void* stream);
OTF_API int otf_pos_advance_batch(int32_t* pos, int64_t n, void* stream);

/*
 * Prompt prefill for one sequence, after its q/k/v projections ran at M = rows prompt rows:
 * row r sits at position *pos + r (pos: one device int32, the first prompt position; it is not
 * advanced).  Two launches: q and k of every row rotated in place (as otf_rope_kv), k and v
 * written to cache rows *pos .. *pos + rows - 1; then causal attention of row r over cache rows
 * [0, *pos + r], out + r*ldo as otf_attn_decode's layout.  Rows past max_pos write nothing and
 * raise the otf_device_error flag.  No workspace.  Replaces the prompt forward of HF's
 * LlamaAttention that the reference runner keeps around its projections (RoPE, cache update,
 * causal softmax(q k^T / sqrt(d)) v; otf_llm/run_symmetric_2bit.py:150-187), one prompt pass
 * instead of one decode step per prompt token.
 */
OTF_API int otf_attn_prefill(void* q, int64_t ldq, void* k, const void* v, int64_t ldkv, const void* cos_sin,
                             const int32_t* pos, void* k_cache, void* v_cache, void* out, int64_t ldo, float scale,
                             int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_pos, int64_t rows,
                             void* stream);

/*
 * otf_attn_decode without a workspace argument, for callers that cannot allocate device
 * memory (a plugin host that passes only the op's own tensors, an allocator frozen after
 * warm-up, code that must not call cudaMalloc).  No counterpart in the reference.
 * The split-KV scratch is one fixed array of OTF_ATTN_SCRATCH_BYTES that the library keeps on
 * every GPU that loads it until the process exits; otf_attn_workspace_bytes(kv_heads,
 * head_dim, max_pos) must not exceed it (OTF_ERR_UNSUPPORTED otherwise; e.g. 8 KV heads of
 * 128 fit up to max_pos 4032).  Nothing is allocated.  The first call on each device looks up
 * the array's device address: make that call before any stream capture.  All calls share the
 * array, so calls that can run at the same time on one GPU (other streams) race.
 * The address is cached per device and context (a context created again after
 * cudaDeviceReset is looked up afresh); the stream must belong to the current device
 * (OTF_ERR_INVALID otherwise).  A position outside [0, max_pos) writes nothing and raises
 * the otf_device_error flag, as otf_attn_decode does.
 */
#define OTF_ATTN_SCRATCH_BYTES (2 * 1024 * 1024)
OTF_API int otf_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* pos,
                                    void* out, float scale, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                    int64_t max_pos, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OTF_B200_H */
