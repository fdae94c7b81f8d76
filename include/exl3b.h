/*
 * exl3b: the EXL3 inference hot path for NVIDIA B200 (sm_100a), as a C ABI.
 *
 * Plain C: raw device pointers, sizes, a cudaStream_t passed as void*, and an int status.
 *   0  EXL3B_OK
 *   >0 the call was declined (unsupported shape or flags, bad argument, workspace too small);
 *      nothing was launched and no output was touched
 *   <0 -(cudaError_t) from a launch; outputs are unspecified
 * Every call is asynchronous on `stream`, never allocates device memory and never
 * synchronises, so it may be captured into a CUDA graph.  fp16 tensors are passed as
 * uint16_t bit patterns.
 *
 * Each entry point names the reference interface it replaces (reference repository
 * Luke458/qwen38-27b-exl3-rdna4; the pybind extension `exllamav3_ext` is the un-vendored
 * fork CarouselAether/rocm_exl3 @ 311ff5497237a37bea18cf24aa18bc0c573d1d03, whose call
 * sites are in vllm_plugin/exl3rocm/ops.py and tests/test_gpu_parity.py).
 */
#ifndef EXL3B_H
#define EXL3B_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EXL3B_API __attribute__((visibility("default")))
#else
#define EXL3B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3B_OK 0
#define EXL3B_DECLINED 1  /* shape / flags outside what the kernels implement */
#define EXL3B_BAD_ARG 2   /* null or misaligned pointer, bad size */
#define EXL3B_WORKSPACE 3 /* workspace smaller than exl3b_linear_workspace_bytes() */
#define EXL3B_TOO_LARGE 4 /* exl3b_linear_noalloc: the call needs more than its static scratch */

/* codebook ids: the (mcg, mul1) flags of the reference ops map to 0 = 3INST, 1 = MCG, 2 = MUL1
 * (reference tests/test_gpu_parity.py:101) */
#define EXL3B_CB_3INST 0
#define EXL3B_CB_MCG 1
#define EXL3B_CB_MUL1 2
/* or-ed into the codebook argument of the m <= 16 linears: x is bf16 and is rounded to fp16 inside
 * the kernel, exactly as the reference's x.to(float16) at the op boundary (ops.py:72-73) */
#define EXL3B_X_BF16 0x100
/* Epilogue flags (or-ed into `codebook` of exl3b_linear / exl3b_linear_grouped / exl3b_linear_tp;
 * no reference counterpart: the reference runs these as separate vLLM ops, and its own analysis of
 * fusing them is docs/EFFICIENCY_INVESTIGATION.md:36-66).
 *   EXL3B_ACT_SILU_MUL: exl3b_linear_grouped with exactly two groups of equal width (gate, up):
 *     y[0][m][n] = fp16( fp16(silu(gate)) * up ), gate/up being the two groups' fp16 outputs;
 *     the roundings of torch's fp16 F.silu(gate) * up (vLLM SiluAndMul).  y[1] is not written.
 *   EXL3B_Y_ADD: y = fp16(y + result), one fp16 add per element (the residual add); y must hold
 *     the residual before the call.  Not combinable with EXL3B_ACT_SILU_MUL. */
#define EXL3B_ACT_SILU_MUL 0x200
#define EXL3B_Y_ADD 0x400

#define EXL3B_MAX_GROUPS 8
#define EXL3B_GEMV_MAX_ROWS 16

/* Library version, (major << 16) | (minor << 8) | patch. */
EXL3B_API int exl3b_version(void);

/* Human-readable text for a status code (static storage). */
EXL3B_API const char* exl3b_status_string(int status);

/* Decode raw 16-bit trellis states through a codebook to fp32 copies of the fp16 values.
 * Replaces exllamav3_ext.decode(codes, out, mcg, mul1) (reference tests/test_gpu_parity.py:101-109). */
EXL3B_API int exl3b_decode_states(const uint16_t* states, float* out, int64_t count, int codebook, void* stream);

/* Dequantize ("reconstruct") a trellis [k/16][n/16][16K] into fp16 W[k][ldw], output columns
 * n0..n1 of the layer written to W columns 0..n1-n0.  Bit-exact to the reference oracle.
 * Replaces exllamav3_ext.reconstruct(W, B, K, mcg, mul1) and reconstruct_slice(W, B, K, mcg, mul1, n0)
 * (reference vllm_plugin/exl3rocm/ops.py:92-95). Requires n0, n1 multiples of 16, ldw % 8 == 0. */
EXL3B_API int exl3b_dequant(const uint16_t* trellis, int k, int n, int K, int codebook, int n0, int n1,
                  uint16_t* W, int64_t ldw, void* stream);

/* 128-point Hadamard over each 128-column block of a [rows][cols] fp16 matrix:
 *   out = fp16( H128 * fp16(in * pre) * scale / sqrt(128) ) * post     (pre, post optional)
 * in == out is allowed.  Replaces exllamav3_ext.had_r_128(in, out, pre, post, scale)
 * (reference vllm_plugin/exl3rocm/ops.py:88,97). cols % 128 == 0, lds % 4 == 0. */
EXL3B_API int exl3b_had128(const uint16_t* in, int64_t ld_in, uint16_t* out, int64_t ld_out, int64_t rows, int64_t cols,
                 const uint16_t* pre, const uint16_t* post, float scale, void* stream);

/* Workspace for exl3b_linear / exl3b_linear_grouped: m rows, k inputs, `groups` weight groups
 * with n_total (<= 1048576) output columns in all.  The first EXL3B_WS_ZERO_BYTES bytes must be
 * zero before the first call; every call leaves them zero again, so a workspace allocated once
 * with zeros can be reused by calls of any shape issued in stream order.  Calls that may run
 * concurrently need separate workspaces.  After a call that reported a kernel error
 * (exl3b_linear_workspace_error) the workspace must be zeroed again. */
#define EXL3B_WS_ZERO_BYTES (256 + 4 * 8192)
EXL3B_API size_t exl3b_linear_workspace_bytes(int m, int k, int groups, int64_t n_total);

/* 1 when exl3b_linear takes an m x k x n call at K bits in this codebook (EXL3B_X_BF16 / EXL3B_Y_ADD may be
 * or-ed in), else 0: m <= EXL3B_GEMV_MAX_ROWS, k and n multiples of 128, 1 <= K <= 8.  Host-only, no device
 * needed.  Replaces exllamav3_ext.exl3_gemv_mr_supported(m, k, n, K, mcg, mul1) (reference
 * vllm_plugin/exl3rocm/ops.py:83,149; 0002-gemv-multirow.patch:334-338). */
EXL3B_API int exl3b_linear_supported(int m, int k, int n, int K, int codebook);

/* The EXL3 linear for 1 <= m <= 16 (decode / speculative verify):
 *   y[m][n] = had_out( fp16( had_in(x, suh) @ W ), svh )
 * x fp16 [m][k] contiguous, trellis int16 [k/16][n/16][16K], suh fp16 [k], svh fp16 [n],
 * y fp16 rows of stride ldy.  k % 128 == 0, n % 128 == 0, 1 <= K <= 8.  Each output row is
 * bitwise identical to the m = 1 call on that row alone, and repeated calls are bitwise
 * identical.
 * Replaces exllamav3_ext.exl3_gemm (m = 1) and exl3_gemv_mr (m <= 16) with their fused input and
 * output Hadamards (reference vllm_plugin/exl3rocm/ops.py:80-85; multi-row contract
 * vllm_plugin/patches/exl3-fork/0002-gemv-multirow.patch:79-88). */
EXL3B_API int exl3b_linear(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                 const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Up to EXL3B_MAX_GROUPS weight groups that share the input x and the bit width K (gate/up,
 * q/k/v), in one launch.  Group i has its own trellis [k/16][n[i]/16][16K], suh[i], svh[i] and
 * writes y[i] (row stride ldy).  Host arrays of device pointers.  For a fixed set of groups each
 * output row is bitwise identical to the m = 1 call on that row (the work partition spans the
 * groups, so it depends on the group set, not on m).
 * Replaces exllamav3_ext.exl3_mgemm (m = 1) and exl3_gemv_mr_grouped
 * (reference vllm_plugin/exl3rocm/ops.py:134-170, 0002-gemv-multirow.patch:174-182). */
EXL3B_API int exl3b_linear_grouped(const uint16_t* x, int m, int k, int groups, const uint16_t* const* trellis,
                         const int* n, int K, int codebook, const uint16_t* const* suh,
                         const uint16_t* const* svh, uint16_t* const* y, int64_t ldy,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Decode-ceiling microbenchmark of the decode GEMV (no reference counterpart): one CTA per SM runs
 * the GEMV's per-tile work (trellis words from shared memory, window extraction, codebook decode into
 * mma A fragments, one m16n8k16 per 16x16 tile) over one resident stage of 8 k-rows x 64 tiles,
 * `iters` times, with no HBM traffic and no stage hand-offs.  Each launch decodes
 * (*ctas) x 16 warps x iters x 32 tiles; time it with events on `stream`.  trellis: at least
 * 8 x 64 x 32K bytes (16-byte aligned); out: (*ctas) x 512 floats (the accumulators' sums, which
 * keep the work live); *ctas receives the SM count used. */
EXL3B_API int exl3b_decode_ceiling(int K, int codebook, const uint16_t* trellis, int iters, float* out, int* ctas,
                                   void* stream);

/* Workspace of exl3b_gemm: a 256-byte header (error word at offset 0) plus A_had [m][k] fp16. */
EXL3B_API size_t exl3b_gemm_workspace_bytes(int m, int k);

/* The EXL3 linear for any number of rows m >= 1, built for prefill (m in the hundreds and thousands):
 *   y[m][n] = had_out( fp16( had_in(x, suh) @ W ), svh )
 * on the 5th-generation tensor cores: had_in into the workspace, then one persistent kernel whose CTAs
 * decode the trellis tiles of their 256 x 256 output tile into shared memory and feed them to
 * tcgen05.mma (fp32 accumulation in tensor memory); the epilogue rounds to fp16, applies had_out and
 * svh.  W never exists in global memory.  x fp16 [m][k] contiguous (16-byte aligned), trellis
 * [k/16][n/16][16K], suh [k], svh [n], y rows of stride ldy (ldy % 8 == 0, 16-byte aligned).
 * k % 128 == 0, n % 128 == 0, 1 <= K <= 8, codebook 0..2 (EXL3B_X_BF16 is declined: cast x first).
 * Replaces the reference's M > 16 route had_r_128 + reconstruct[_slice] + hgemm_recon
 * (vllm_plugin/exl3rocm/ops.py:86-97), which materialises W and accumulates in fp16. */
EXL3B_API int exl3b_gemm(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                         const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy, void* workspace,
                         size_t workspace_bytes, void* stream);

/* exl3b_linear_grouped with the RMSNorm before it fused in (vLLM rms_norm): the groups run on
 *   h = fp16( fp16(x * rsqrt(mean(x^2) + eps)) * norm_weight )      (mean in fp32, per row)
 * where x [m][k] is the un-normalised input (the residual stream).  norm_weight fp16 [k].  Rows stay
 * independent of m.  No reference counterpart: the reference runs the norm as a separate vLLM op
 * before the EXL3 linear. */
EXL3B_API int exl3b_linear_grouped_rmsnorm(const uint16_t* x, int m, int k, int groups,
                                 const uint16_t* const* trellis, const int* n, int K, int codebook,
                                 const uint16_t* norm_weight, float eps, const uint16_t* const* suh,
                                 const uint16_t* const* svh, uint16_t* const* y, int64_t ldy,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Paged KV cache, head size 128.  Caches are [num_blocks][block_size][num_kv_heads][row] with
 * row = 128 int8 (int8) or 64 bytes of nibbles (int4: element 2i in the low nibble of byte i),
 * and per-(token, head) fp32 scales [num_blocks][block_size][num_kv_heads] (int4: the zero point
 * is stored in the scale's low 4 mantissa bits).  key/value inputs are [tokens][heads][128] with
 * the given strides (elements), dtype 0 = fp16, 1 = bf16.  slot_mapping[t] = block * block_size +
 * offset, negative = skip.
 *
 * Every KV call takes an optional layout (NULL = the dense layout above).  vLLM's per-token-head caches
 * (kv_cache [num_blocks][2][block_size][Hkv][row bytes + 4], the fp32 scale inline after each row, the
 * K and V halves interleaved per block; vllm/v1/attention/backends/triton_attn.py _ensure_scale_caches)
 * are described by their strides: cache strides in bytes (multiples of 4, head stride >= the row bytes)
 * and scale strides in floats.  Rows that all start on 16-byte boundaries are read with 16-byte copies,
 * others with 4-byte ones.
 * ------------------------------------------------------------------------------------------ */
typedef struct {
    int64_t cache_block, cache_slot, cache_head; /* bytes */
    int64_t scale_block, scale_slot, scale_head; /* floats */
} exl3b_kv_layout;

/* int8 per-token-head quantize-on-write: scale = max(absmax/127, 1e-6), q = trunc(clamp(x/scale)).
 * Replaces vLLM's triton_reshape_and_cache_flash_per_token_head_quant, which the reference's
 * int8_per_token_head cache uses (vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:139-238). */
EXL3B_API int exl3b_kv_int8_write(const void* key, const void* value, int dtype, int64_t num_tokens,
                                  int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                                  int64_t v_stride_tok, int64_t v_stride_head, int8_t* key_cache,
                                  int8_t* value_cache, float* k_scale, float* v_scale, const int64_t* slot_mapping,
                                  int block_size, const exl3b_kv_layout* layout, void* stream);

/* exl3b_kv_int8_write fused with the neox rotary embedding of the same tokens (exl3b_rope_neox):
 * row t of qkv (fp16, stride ld) holds num_q_heads q heads, then num_kv_heads k heads, then
 * num_kv_heads v heads of 128.  q is written rotated to q_out (stride ld_q); k is rotated, rounded to
 * fp16 and quantised, v quantised, into the int8 caches, byte-identical to exl3b_rope_neox followed
 * by exl3b_kv_int8_write.  qkv itself is not modified.  No reference counterpart (vLLM runs rotary
 * embedding and the cache write as separate ops). */
EXL3B_API int exl3b_kv_int8_write_rope(const uint16_t* qkv, int64_t ld, uint16_t* q_out, int64_t ld_q,
                             int64_t num_tokens, int num_q_heads, int num_kv_heads, const int64_t* positions,
                             const float* cos_sin, int64_t max_position, int8_t* key_cache, int8_t* value_cache,
                             float* k_scale, float* v_scale, const int64_t* slot_mapping, int block_size,
                             const exl3b_kv_layout* layout, void* stream);

/* int4 quantize-on-write: y = H (x * signs) unnormalised (+ optional rotated-domain bias [heads][128]),
 * 3x3 clip search, asymmetric 4 bit, nibble packing.  With exact_tag != NULL also keeps exact fp16 y
 * rows per request slot: [slots][4 + 128][heads][128] for K (exact_k) and V (exact_v), tags
 * [slots][4 + 128]; position p < 4 -> row p, else row 4 + p % 128, written when p < 4 or p is among
 * the sequence's newest 128 positions.  query_start_loc [num_seqs + 1], seq_lens [num_seqs] (length
 * after this write) and seq_slots [num_seqs] (request slot, < 0 = none) locate each token.
 * Replaces the reference's kv_int4.reshape_and_cache (vllm_plugin/exl3rocm/kv_int4.py:176-213). */
EXL3B_API int exl3b_kv_int4_write(const void* key, const void* value, int dtype, int64_t num_tokens,
                                  int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                                  int64_t v_stride_tok, int64_t v_stride_head, uint8_t* key_cache,
                                  uint8_t* value_cache, float* k_scale, float* v_scale, const int64_t* slot_mapping,
                                  int block_size, const float* rht_signs, const float* bias_k, const float* bias_v,
                                  const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* seq_slots,
                                  int num_seqs, uint16_t* exact_k, uint16_t* exact_v, int32_t* exact_tag,
                                  const exl3b_kv_layout* layout, void* stream);

/* Workspace of the attention calls (split-KV partials; int4 also its rotated q). */
EXL3B_API size_t exl3b_kv_attn_workspace_bytes(int num_tokens, int num_q_heads, int num_seqs, int num_kv_heads,
                                               int max_seq_len);

/* Causal decode / speculative-verify attention over the int8 cache: q [tokens][q_heads][128] fp16,
 * out likewise; query token i of a sequence with q_len = qsl[s+1] - qsl[s] tokens sits at position
 * seq_lens[s] - q_len + i.  max_q_len * (q_heads / kv_heads) <= 32.  block_table [num_seqs][bt_stride]
 * int32, block_size a power of two.  Split-KV with a reduce, as vLLM's 3D unified attention with
 * per-token-head scales (vllm/v1/attention/ops/triton_unified_attention.py:473-545, 646-762). */
EXL3B_API int exl3b_kv_int8_attn(const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                                 int num_kv_heads, int head_size, const int8_t* key_cache, const int8_t* value_cache,
                                 const float* k_scale, const float* v_scale, int block_size,
                                 const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                                 const int32_t* query_start_loc, int num_seqs, int max_q_len, int max_seq_len,
                                 float softmax_scale, void* workspace, size_t workspace_bytes,
                                 const exl3b_kv_layout* layout, void* stream);

/* The same over the int4 cache: q is rotated with the RHT, rows with a matching exact tag (first 4
 * and newest 128 positions of a request slot) are read from the exact fp16 rows, and the output is
 * rotated back: out = fp16(H(rot) * signs / 128 + out_bias[kv head of the query head]).  out_bias
 * (optional, fp32 [num_kv_heads][128]) is the value mean of a cache written with bias_v = -(mean_v @
 * diag(signs) H) (the centering of kv_int4.py:120-158, added back as :563 does).  Replaces the
 * reference's kv_int4.attention (vllm_plugin/exl3rocm/kv_int4.py:345-563). */
EXL3B_API int exl3b_kv_int4_attn(const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                                 int num_kv_heads, int head_size, const uint8_t* key_cache,
                                 const uint8_t* value_cache, const float* k_scale, const float* v_scale,
                                 int block_size, const int32_t* block_table, int64_t bt_stride,
                                 const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                                 int max_q_len, int max_seq_len, float softmax_scale, const float* rht_signs,
                                 const uint16_t* exact_k, const uint16_t* exact_v, const int32_t* exact_tag,
                                 const int32_t* seq_slots, const float* out_bias, void* workspace,
                                 size_t workspace_bytes, const exl3b_kv_layout* layout, void* stream);

/* Prefill over the quantised caches: gather the blocks listed in block_ids (n entries) and dequantise
 * them to fp16 rows out[n][block_size][num_kv_heads][128], for an fp16 attention kernel to read.
 * int8: out = fp16(q * scale).  Replaces gather_dequant (reference vllm_plugin/exl3rocm/kv_dequant.py:42-152). */
EXL3B_API int exl3b_kv_int8_gather(const int8_t* cache, const float* scale, int block_size, int num_kv_heads,
                                   int head_size, const int32_t* block_ids, int64_t n, uint16_t* out,
                                   const exl3b_kv_layout* layout, void* stream);
/* int4: out = fp16((nibble - zp) * scale / sqrt(128)), still rotated but in the orthonormal domain;
 * block_ids lists blocks_per_seq blocks per sequence, and with exact_tag given, positions whose exact row
 * (first 4 / newest 128 of the sequence's request slot) carries a matching tag take that row / sqrt(128).
 * Replaces gather_dequant_int4 + _tail_overlay (reference vllm_plugin/exl3rocm/kv_dequant.py:80-123,
 * kv_int4.py:566-594). */
EXL3B_API int exl3b_kv_int4_gather(const uint8_t* cache, const float* scale, int block_size, int num_kv_heads,
                                   int head_size, const int32_t* block_ids, int64_t n, int blocks_per_seq,
                                   uint16_t* out, const uint16_t* exact, const int32_t* exact_tag,
                                   const int32_t* seq_slots, const int32_t* seq_lens, const exl3b_kv_layout* layout,
                                   void* stream);

/* exl3b_linear without a caller-provided workspace, for callers that cannot allocate device
 * memory: code that runs while a CUDA graph is being captured (cudaMalloc is not allowed there),
 * hosts whose device memory is owned by a pool the caller cannot reach, and latency-critical
 * paths where cudaMalloc's implicit device synchronisation is unacceptable.  This entry point has
 * no counterpart in the reference: the reference always receives its scratch from the torch
 * caching allocator.
 * Same arguments, results and limits as exl3b_linear (each row bitwise equal to exl3b_linear's),
 * but the scratch lives in one static device array of EXL3B_NOALLOC_SCRATCH_BYTES (32 MiB) that
 * every GPU loading this library holds until exit; the call allocates nothing.  A call whose
 * scratch need exceeds the array returns EXL3B_TOO_LARGE before launching anything.  The need is
 * at most 33280 + 4 * m * (1024 * SMs + 2 * n) bytes, so on a B200 (148 SMs) every call with
 * m <= 16 and n <= 131072 fits, at any k, K and codebook (m = 16 at n = 17408 needs 10.8 MB).
 * The first call on a device resolves the array's device address with that device current (a
 * one-time set-up; if it fails, the next call tries again): make it before any stream capture — a
 * first call on a stream that is being captured returns EXL3B_BAD_ARG without touching the stream.
 * Every call clears the array's counter region and error word on `stream` first, and all calls
 * share the array, so calls that can overlap on the GPU (different streams, or graphs replayed
 * concurrently) race: issue them in one stream order. */
#define EXL3B_NOALLOC_SCRATCH_BYTES (32u << 20)
EXL3B_API int exl3b_linear_noalloc(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K,
                                   int codebook, const uint16_t* suh, const uint16_t* svh, uint16_t* y,
                                   int64_t ldy, void* stream);
/* The kernel error word of the last exl3b_linear_noalloc call on the current device (0 = none;
 * otherwise the code of a bounded wait that gave up, after which that call's y is not valid) into
 * *out, synchronising `stream`.  Read it before the next call, which clears it.  No counterpart in
 * the reference (the diagnostic of the static scratch, as exl3b_linear_workspace_error is of a
 * caller's workspace). */
EXL3B_API int exl3b_linear_noalloc_error(int* out, void* stream);

/* ------------------------------------------------------------------------------------------
 * Tensor-parallel row-parallel linear with the all-reduce fused into the kernel.  The reference
 * runs no tensor parallelism (vllm_plugin/exl3rocm/plugin.py:255-257 raises); under vLLM this
 * replaces exl3_gemm on an o_proj / down_proj shard followed by RowParallelLinear's all-reduce.
 *
 * Every rank owns one communication buffer of exl3b_tp_comm_bytes(tp_size, max_blocks, max_rows)
 * bytes, zeroed once, and maps every peer's buffer with CUDA IPC (exl3b_ipc_get_handle /
 * exl3b_ipc_open_handle).  exl3b_linear_tp computes this rank's k-slice of the product, exchanges
 * the fp32 partial sums of each 128-column block with all ranks through the peers' buffers (plain
 * peer stores over NVLink, a flag per block and call, bounded waits), and writes the full output
 * y = had_out(fp16(sum over ranks), svh) on every rank: no further all-reduce is needed.  All ranks
 * must make the same sequence of calls on a buffer, and the calls of one rank on one buffer must
 * be stream-ordered.  Waits that give up after about a second set the workspace error word. */
#define EXL3B_MAX_TP 8
typedef struct {
    int tp_size;                      /* 2 .. EXL3B_MAX_TP */
    int tp_rank;
    int max_blocks;                   /* the buffers hold up to max_blocks 128-column blocks */
    int max_rows;                     /* ... of up to max_rows rows (<= EXL3B_GEMV_MAX_ROWS) */
    void* buffers[EXL3B_MAX_TP];      /* every rank's buffer, mapped into this process (own included) */
} exl3b_tp_comm;

EXL3B_API size_t exl3b_tp_comm_bytes(int tp_size, int max_blocks, int max_rows);
/* A CUDA IPC handle of the allocation holding dev_ptr plus dev_ptr's offset inside it
 * (EXL3B_IPC_HANDLE_BYTES bytes), and the pointer it names, mapped into another process. */
#define EXL3B_IPC_HANDLE_BYTES 72
EXL3B_API int exl3b_ipc_get_handle(const void* dev_ptr, void* handle);
EXL3B_API int exl3b_ipc_open_handle(const void* handle, void** dev_ptr);
EXL3B_API int exl3b_ipc_close(void* dev_ptr);
/* x holds this rank's k/tp_size input features (k here is that local width), trellis / suh its
 * k-slice; n is the full output width (n / 128 <= comm->max_blocks, m <= comm->max_rows). */
EXL3B_API int exl3b_linear_tp(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                              const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy,
                              void* workspace, size_t workspace_bytes, const exl3b_tp_comm* comm, void* stream);

/* Reads the kernel error word of a linear workspace (0 = none; otherwise the code of a wait that
 * gave up) into *out, synchronising `stream`.  Test and diagnostics helper. */
EXL3B_API int exl3b_linear_workspace_error(const void* workspace, int* out, void* stream);

/* ------------------------------------------------------------------------------------------
 * Decoder-layer glue between the linears and the attention.  The reference leaves these steps to
 * vLLM's own kernels (its plugin replaces only the linears and the KV cache); they are here so a
 * decode step runs on this library alone.  fp16 rows with strides in elements.
 * ------------------------------------------------------------------------------------------ */

/* RMSNorm of `rows` rows of `cols` (cols % 8 == 0, <= 16384).  residual != NULL: residual =
 * fp16(x + residual) first, and that sum is normalised (vLLM fused_add_rms_norm); otherwise x is
 * (vLLM rms_norm).  out = fp16( fp16(v * rsqrt(mean(v^2) + eps)) * weight ), mean in fp32. */
EXL3B_API int exl3b_rmsnorm(const uint16_t* x, int64_t ldx, uint16_t* residual, int64_t ldr, const uint16_t* weight,
                            uint16_t* out, int64_t ldo, int rows, int cols, float eps, void* stream);

/* Neox rotary embedding, head size 128 (vLLM get_rope(..., is_neox_style=True)).  Row t of qkv
 * (stride ld) holds num_q_heads q heads then num_k_heads k heads; q is written rotated to q_out
 * (stride ld_q), k is rotated in place.  cos_sin fp32 [max_position][128]: cos of the 64
 * frequencies, then their sin.  positions int64 [tokens]; a position outside [0, max_position)
 * leaves the token's k as it was and writes zeros for its q. */
EXL3B_API int exl3b_rope_neox(uint16_t* qkv, int64_t ld, uint16_t* q_out, int64_t ld_q, int tokens, int num_q_heads,
                              int num_k_heads, const int64_t* positions, const float* cos_sin, int64_t max_position,
                              void* stream);

/* SiluAndMul: out[r][c] = fp16( fp16(silu(in[r][c])) * in[r][n + c] ), n % 8 == 0 (the
 * activation of EXL3B_ACT_SILU_MUL, for rows taken by the dequantise + GEMM route). */
EXL3B_API int exl3b_silu_mul(const uint16_t* in, int64_t ld_in, uint16_t* out, int64_t ld_out, int rows, int n,
                             void* stream);

/* The fp8 input embedding (reference vllm_plugin/exl3rocm/ops.py:183-202, exl3rocm::fp8_embedding):
 * out[t][0..dim) = fp16(table[ids[t]][0..dim)) for a float8_e4m3fn table [rows][dim] (no scale; the
 * checkpoint's table cast as is).  ids int32 (ids_64 = 0) or int64 [n]; an id outside [0, rows) gives a
 * zero row (vLLM masks ids outside a rank's vocab shard before the lookup).  dim % 16 == 0, table and
 * out 16-byte aligned. */
EXL3B_API int exl3b_fp8_embedding(const uint8_t* table, int64_t rows, int64_t dim, const void* ids, int ids_64,
                                  int64_t n, uint16_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXL3B_H */
