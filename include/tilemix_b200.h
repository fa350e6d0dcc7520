/*
 * tilemix_b200 — C ABI of the B200 (sm_100a) TileMix hot path.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t passed as void*, launches asynchronously on that stream and
 * returns an int status (TM_OK or a negative TM_ERR_* code for argument
 * errors found on the host). The library allocates no device memory: the
 * caller owns every buffer, including outputs and the optional device error
 * word. Device-side wait timeouts are reported through that error word.
 *
 * Tensors use the reference's packed varlen layout: token-major
 * [total_tokens, heads, head_dim] with head_dim contiguous, sequences
 * delimited by int32 cu_seqlens[batch + 1].
 */
#ifndef TILEMIX_B200_H_
#define TILEMIX_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TM_OK 0
#define TM_ERR_NULL -1        /* a required pointer is NULL */
#define TM_ERR_SHAPE -2       /* unsupported or inconsistent sizes */
#define TM_ERR_ALIGN -3       /* pointer / stride alignment violated */
#define TM_ERR_UNSUPPORTED -4 /* option outside what the kernels implement */
#define TM_ERR_LAUNCH -5      /* CUDA launch or driver-entry-point failure */
#define TM_ERR_TMAP -6        /* TMA descriptor encoding failed */

/* Routing modes (attention/triton/tilemix.py:159-161). */
#define TM_ROUTE_MIXED 0
#define TM_ROUTE_FP16 1
#define TM_ROUTE_INT8 2

/* Numerics (no reference counterpart: they select which execution of the
 * reference's arithmetic the results reproduce).
 *   TM_NUMERICS_GPU    the reference's Triton kernels as they run on the GPU:
 *                      FP16-route QK^T accumulated in fp16 by the tensor core
 *                      (tl.dot(..., out_dtype=fp16)), fp32 divisions of the
 *                      quantiser and of the final acc / l by the approximate
 *                      PTX div.full.f32 that Triton emits for `/`. The default.
 *   TM_NUMERICS_EXACT  the reference's algorithm in exact arithmetic, as its
 *                      Triton interpreter runs it on the CPU: QK^T accumulated
 *                      in fp32 and rounded once to fp16, IEEE divisions. */
#define TM_NUMERICS_GPU 0
#define TM_NUMERICS_EXACT 1

/*
 * Per-block symmetric INT8 quantisation of a packed fp16 tensor.
 * Replaces quant_per_block_int8_kernel + per_block_int8_single
 * (attention/triton/quant_per_block_varlen.py:6-45 and :48-75).
 *   x            fp16 [tokens, heads, dim]; strides in elements (dim stride 1)
 *   cu_seqlens   int32 [batch+1] token offsets
 *   cu_scale     int32 [batch+1] scale-block offsets (exclusive prefix sum of
 *                ceil(T_b / blk))
 *   out          int8 [tokens, heads, dim]
 *   scale_f32    optional fp32 [sum blocks, heads] (the reference's output)
 *   scale_f16    optional fp16 [sum blocks, heads] (the reference's host cast,
 *                attention/triton/tilemix.py:142-155)
 */
int tm_quant_per_block_int8(const void* x, int64_t x_stride_tok, int64_t x_stride_head,
                            const int32_t* cu_seqlens, const int32_t* cu_scale, int batch, int heads,
                            int dim, int blk, int max_seqlen, float sm_scale, int8_t* out,
                            int64_t out_stride_tok, int64_t out_stride_head, float* scale_f32,
                            void* scale_f16, void* stream);

/* tm_quant_per_block_int8 in the given TM_NUMERICS_* mode (tm_quant_per_block_int8
 * is TM_NUMERICS_GPU): GPU numerics give the codes and scales of the reference's
 * quantiser run on the GPU, exact numerics those of its interpreter run. */
int tm_quant_per_block_int8_ex(const void* x, int64_t x_stride_tok, int64_t x_stride_head,
                               const int32_t* cu_seqlens, const int32_t* cu_scale, int batch, int heads,
                               int dim, int blk, int max_seqlen, float sm_scale, int8_t* out,
                               int64_t out_stride_tok, int64_t out_stride_head, float* scale_f32,
                               void* scale_f16, int numerics, void* stream);

/* tm_quant_per_block_int8_ex with sm_scale 1 that also writes every code as
 * an exact fp16 value to out_f16 ([tokens, heads, dim], 16-byte aligned rows):
 * the V operand of the paired kernel's INT8-V path (tm_attn_params.v8_f16).
 * out (the int8 codes) may be NULL. dim and blk 64 or 128, else
 * TM_ERR_UNSUPPORTED. No reference counterpart: the reference's kernel
 * converts the int8 V tile to fp16 as it loads it (tilemix.py:497). */
int tm_quant_per_block_int8_f16(const void* x, int64_t x_stride_tok, int64_t x_stride_head,
                                const int32_t* cu_seqlens, const int32_t* cu_scale, int batch, int heads,
                                int dim, int blk, int max_seqlen, int8_t* out, int64_t out_stride_tok,
                                int64_t out_stride_head, void* out_f16, int64_t out_f16_stride_tok,
                                int64_t out_f16_stride_head, float* scale_f32, void* scale_f16, int numerics,
                                void* stream);

/* Routing-map patterns of make_precision_bitmask (attention/precision_maps.py:404-636). */
#define TM_MAP_ZERO 0
#define TM_MAP_ONE 1
#define TM_MAP_BAND 2
#define TM_MAP_GLOBAL 3
#define TM_MAP_ROW_RAND 4
#define TM_MAP_ALIGN_SPARSE 5
#define TM_MAP_BIGBIRD 6
#define TM_MAP_SPTRANS 7

/* Arguments of tm_build_precision_map; the names follow the reference's
 * (seq_len, BLOCK_M, BLOCK_N, COMPUTE_BLOCK_N, percentage, pattern_params). */
typedef struct tm_map_params {
  int seq_len;
  int block_m;         /* BLOCK_M: query rows per map row */
  int block_n_mask;    /* BLOCK_N: keys per mask group (map column) */
  int compute_block_n; /* COMPUTE_BLOCK_N: keys per attention tile; divides block_n_mask */
  int pattern;         /* TM_MAP_* */
  double percentage;   /* INT8 share of the causal work, in [0, 1]; read for patterns >= TM_MAP_BAND */
  /* sptrans: stride > 0 (the reference's default is min(128, seq_len / 4)) and
   * c (default min(32, stride / 4)). */
  int stride, c;
  /* global: HOST array of token positions (pattern_params["key_pos"]);
   * NULL = the reference's default 0 .. min(4, seq_len) - 1. */
  const int64_t* key_pos;
  int num_key_pos;
  /* bigbird: >= 0 each (the reference's defaults are 2 and 3). */
  int num_global_block, num_rand_block;
} tm_map_params;

/*
 * Routing map on the GPU: out[r] bit j = 1 routes (query block r, mask group
 * j) to INT8, 0 to FP16. Replaces make_precision_bitmask
 * (attention/precision_maps.py:404-636) for token_mask = None — the path of
 * the model integration (models/tilemix_llama.py:333-364) — bit for bit,
 * including its seeded draws (torch's CPU generator, seed 42: the global
 * generator for row_rand / bigbird, a private one for the weighted retarget).
 *   out         device uint64 [ceil(seq_len / block_m)]
 *   error_flag  optional device int; set to 1 when the weighted retarget ends
 *               farther from its target than one mask-group weight (where the
 *               reference raises RuntimeError, :319-325)
 * Limits: ceil(seq_len / block_n_mask) <= 64 (the reference's own limit,
 * TM_ERR_SHAPE); at most 4096 map rows and 65536 cells (TM_ERR_UNSUPPORTED).
 * One CTA, no device memory besides `out` and `error_flag`.
 */
int tm_build_precision_map(const tm_map_params* params, uint64_t* out, int* error_flag, void* stream);

/*
 * Arguments of the fused mixed-precision attention forward.
 * Mirrors the launch of attn_fwd in launch_prequantized
 * (attention/triton/tilemix.py:1132-1336, kernel signature :503-578).
 */
typedef struct tm_attn_params {
  const void* q; /* fp16 [q_tokens, heads_q, head_dim] */
  const void* k; /* fp16 [k_tokens, heads_k, head_dim] */
  const void* v; /* fp16 [k_tokens, heads_k, head_dim] */
  int64_t q_stride_tok, q_stride_head;
  int64_t k_stride_tok, k_stride_head;
  int64_t v_stride_tok, v_stride_head;
  int64_t q_tokens, k_tokens;
  void* out; /* fp16 [q_tokens, heads_q, head_dim] */
  int64_t o_stride_tok, o_stride_head;

  /* Prequantised Q (launch_prequantized). NULL => Q is quantised inside the
   * kernel with 128-token blocks (requires blkq == 128). */
  const int8_t* q8;
  int64_t q8_stride_tok, q8_stride_head;
  const void* q_scale; /* fp16 [sum ceil(Tq_b/blkq), heads_q] */
  const int32_t* cu_q_scale;
  /* Quantised K (required unless routing_mode == TM_ROUTE_FP16). */
  const int8_t* k8;
  int64_t k8_stride_tok, k8_stride_head;
  const void* k_scale; /* fp16 [sum ceil(Tk_b/blkk), heads_k] */
  const int32_t* cu_k_scale;
  /* Quantised V for the INT8-V PV path (int8_use_fp16_v == 0 with an INT8
   * route): an INT8-routed tile's PV is fp16(p * sv) x fp16(v8)
   * (attention/triton/tilemix.py:449-497). v8 int8 [k_tokens, heads_k,
   * head_dim] (16-byte rows), v_scale fp16 [sum ceil(Tk_b/blkk), heads_k] with
   * int32 block offsets cu_v_scale, blocks of blkk keys as for K. */
  const int8_t* v8;
  int64_t v8_stride_tok, v8_stride_head;
  const void* v_scale;
  const int32_t* cu_v_scale;
  /* Optional exact fp16 copy of the v8 codes ([k_tokens, heads_k, head_dim],
   * 16-byte rows; tm_quant_per_block_int8_f16 writes it beside the codes). With
   * it, INT8-V calls of the paired kernel's shape (head_dim 128, block_m 128,
   * Q quantised in kernel, no bias) run on that kernel, which loads the V
   * operand of INT8-routed tiles from here; v8 may then be NULL. */
  const void* v8_f16;
  int64_t v8_f16_stride_tok, v8_f16_stride_head;

  const int32_t* cu_seqlens_q; /* int32 [batch+1] */
  const int32_t* cu_seqlens_k; /* int32 [batch+1] */
  const uint64_t* precision_bitmask; /* uint64 [heads_k * ceil(max_seqlen_q/block_m)] */
  /* Optional additive fp16 bias, element (z, h, m, n) at bias_stride[0..3]:
   * qk = fp16(qk + fp16(bias * fp16(log2 e))) on the unmasked keys
   * (tilemix.py:264-272, :413-421). As in the reference, the element read is
   * (0, hq, query position, key position): bias_stride[0] is not applied.
   * The caller keeps it covering heads_q x max_seqlen_q x max_seqlen_k. */
  const void* bias;
  int64_t bias_stride[4];

  int batch, heads_q, heads_k, head_dim;
  int max_seqlen_q, max_seqlen_k;
  int block_m, block_n, block_n_mask, blkq, blkk;
  int causal, routing_mode, run_length, scalar_scales, int8_use_fp16_v;
  float sm_scale;
  int* error_flag; /* optional device int, set non-zero on a device-side timeout */
} tm_attn_params;

/*
 * Fused FP16/INT8 tile-routed flash-attention forward (tcgen05 + TMA + TMEM).
 * Replaces attn_fwd (attention/triton/tilemix.py:503-951) as launched by
 * launch_prequantized (:1132-1336). Asynchronous on `stream`. Uses the
 * reference's softmax update rule (rescale_threshold 0) and TM_NUMERICS_GPU.
 */
int tm_attn_fwd(const tm_attn_params* params, void* stream);

/* Optional execution settings of tm_attn_fwd_ex (no reference counterpart:
 * they select between equivalent B200 schedules). */
typedef struct tm_attn_tuning {
  /* log2-domain slack before the running softmax max is moved; 0 = the
   * reference's rule (move on every increase). Larger values trade fp16
   * rounding of P for fewer rescales of the output accumulator. <= 15. */
  float rescale_threshold;
  /* Kernel selection: 0 = automatic (the paired kernel when head_dim is 128,
   * block_m 128, Q is quantised in kernel, there is no bias and INT8 tiles use
   * FP16 V or the fp16 copy of the V codes is given; else the general kernel);
   * 1 = always the general kernel. Other values return TM_ERR_SHAPE. */
  int force_general;
  /* TM_NUMERICS_GPU (0) or TM_NUMERICS_EXACT (1); also the numerics of the
   * in-kernel Q quantisation. */
  int numerics;
} tm_attn_tuning;

/* tm_attn_fwd with explicit tuning (NULL = defaults of tm_attn_fwd: threshold 0,
 * automatic kernel, TM_NUMERICS_GPU). */
int tm_attn_fwd_ex(const tm_attn_params* params, const tm_attn_tuning* tuning, void* stream);

/*
 * tm_attn_fwd_ex for callers that cannot allocate device memory (no
 * counterpart in the reference): a host whose framework owns every device
 * allocation and hands the library only Q/K/V/O, or a plugin hook in which
 * allocating is not allowed. The quantised K operand that tm_attn_fwd takes
 * from caller buffers is produced inside this call (in the numerics of
 * `tuning`) into fixed-size scratch that the library's module holds on each
 * device where it is loaded (loaded at the latest by the first call there):
 * 16 MiB of K codes (k_tokens * heads_k * head_dim <= 16,777,216), 262,144 K
 * scales ((k_tokens / blkk + batch) * heads_k <= 262,144) and batch <= 65,535;
 * blkk must be 64 or 128. Larger problems return TM_ERR_UNSUPPORTED, and every
 * argument is checked before anything is queued. params->k8, k_scale and
 * cu_k_scale must be NULL. FP16-only routing needs no K operand and forwards
 * to tm_attn_fwd_ex. The INT8-V PV path (int8_use_fp16_v == 0 with an INT8
 * route) still reads its V operand (v8, or v8_f16 for the paired kernel's
 * shape) and v_scale / cu_v_scale from the caller: callers that pass only
 * Q/K/V/O set int8_use_fp16_v = 1. The call allocates nothing. Its
 * first call on a device resolves the scratch address (a runtime query, which
 * can fail with TM_ERR_LAUNCH if the module cannot be loaded there), so make a
 * warm-up call at initialisation, before any stream capture. Calls that may
 * overlap on the GPU (several streams or threads) share the scratch and must
 * be serialised by the caller.
 */
int tm_attn_fwd_noalloc(const tm_attn_params* params, const tm_attn_tuning* tuning, void* stream);

/*
 * Llama prefill companions (models/tilemix_llama.py:718-895), fp16.
 *
 * tm_rotary_token_major replaces rotary_token_major / _rotary (:797-822):
 * split-half RoPE of q [batch, heads_q, seq_len, head_dim] and k [batch,
 * heads_k, seq_len, head_dim] (element strides for batch / head / token; the
 * last dim contiguous, rows 16-byte aligned) with cos / sin [1 or batch,
 * seq_len, head_dim] (batch stride 0 when broadcast), into token-major oq
 * [batch, seq_len, heads_q, head_dim] and ok [batch, seq_len, heads_k,
 * head_dim] (contiguous). head_dim 64 or 128.
 * If k8 is non-NULL the same pass also quantises the rotated K for the
 * attention (quant_per_block_varlen.py:6-45, sm_scale 1, blocks of blkk = 64 or
 * 128 tokens per sequence and KV head): k8 int8 [batch * seq_len, heads_k,
 * head_dim], optional k_scale_f16 / k_scale_f32 [batch * ceil(seq_len / blkk),
 * heads_k], bit-identical to tm_quant_per_block_int8_ex run on ok with the
 * same TM_NUMERICS_* mode `numerics`.
 */
int tm_rotary_token_major(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k, int64_t k_sb,
                          int64_t k_sh, int64_t k_st, const void* cos, int64_t cos_sb, int64_t cos_st,
                          const void* sin, int64_t sin_sb, int64_t sin_st, int batch, int heads_q, int heads_k,
                          int seq_len, int head_dim, void* oq, void* ok, int8_t* k8, void* k_scale_f16,
                          float* k_scale_f32, int blkk, int numerics, void* stream);

/* out = fp16(fp16(silu(gate)) * up) elementwise over n fp16 values; replaces
 * silu_mul / _silu_mul (:825-866). */
int tm_silu_mul(const void* gate, const void* up, void* out, int64_t n, void* stream);

/* RMSNorm of `rows` contiguous fp16 rows of `cols` values: var = mean(x^2) in
 * fp32, out = fp16(weight * fp16(x * rsqrt(var + eps))); replaces the
 * squared-mean extension and the tail of PrefillRMSNorm (:718-771). */
int tm_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int cols, float eps, void* stream);

/* Human-readable text for a TM_* status code. */
const char* tm_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* TILEMIX_B200_H_ */
