// C ABI of the attention forward: argument checks, TMA descriptor encoding and
// dispatch between the two sm_100a kernels:
//   * paired  (attn_fwd_paired.cu): head_dim 128, block_m 128, Q quantised in
//     kernel (or FP16-only routing), no bias; INT8-V when the fp16 copy of the
//     V codes is given -- the model / tilemix_attention_with_quant path;
//   * general (attn_fwd_general.cu): everything else the API accepts (block_m 64,
//     head_dim 64, prequantised Q from launch_prequantized, bias, INT8-V from
//     the int8 codes alone).
#include <cudaTypedefs.h>

#include <mutex>

#include "attn_common.cuh"
#include "tilemix_b200.h"

namespace tilemix {

int launch_attn_general(const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v, const CUtensorMap& v8,
                        const AttnArgs& a,
                        int tiles, int heads_q, int batch, cudaStream_t stream);
int launch_attn_paired(const CUtensorMap& q, const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v,
                       const CUtensorMap& vq, const AttnArgs& a, int batch, int max_seqlen_q, cudaStream_t stream);

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over a packed [tokens, heads, dim] tensor: dims {dim, heads, tokens}; box {box_inner, 1, box_rows}.
static int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, int dim, int heads,
                    int64_t tokens, int64_t stride_head, int64_t stride_tok, int box_inner,
                    CUtensorMapSwizzle swz, int box_rows = 64) {
  auto fn = encode_fn();
  if (fn == nullptr) return TM_ERR_LAUNCH;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_head * elem_bytes),
                           static_cast<cuuint64_t>(stride_tok * elem_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), 1u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TM_OK : TM_ERR_TMAP;
}

// 4-D map over a packed fp16 [tokens, heads, 128] tensor that fetches all 128
// dims of `box_rows` tokens in one copy: dims {64 (d low), tokens, 2 (d high),
// heads}, box {64, box_rows, 2, 1}. In shared memory the box lands as two
// [box_rows x 128 B] halves (dims 0-63, then 64-127), the K-major SW128
// operand layout of the tcgen05 kernels.
static int make_map_d128(CUtensorMap* m, const void* base, int heads, int64_t tokens, int64_t stride_head,
                         int64_t stride_tok, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return TM_ERR_LAUNCH;
  cuuint64_t dims[4] = {64u, static_cast<cuuint64_t>(tokens), 2u, static_cast<cuuint64_t>(heads)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(stride_tok * 2), 128u, static_cast<cuuint64_t>(stride_head * 2)};
  cuuint32_t box[4] = {64u, static_cast<cuuint32_t>(box_rows), 2u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TM_OK : TM_ERR_TMAP;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace tilemix

namespace tilemix {

// Whether the call's shape takes the paired kernel (INT8-V additionally needs
// the fp16 copy of the V codes).
static bool paired_shape(const tm_attn_params* p, const tm_attn_tuning* tuning) {
  const bool need_int8 = p->routing_mode != TM_ROUTE_FP16;
  const bool fuse_q = need_int8 && p->q8 == nullptr;
  return !(tuning && tuning->force_general == 1) && p->head_dim == 128 && p->block_m == 128 && (fuse_q || !need_int8) &&
         p->bias == nullptr;
}

// Host-side argument checks of tm_attn_fwd_ex; no CUDA call. TM_OK when the
// call would be launched (or is an empty problem), else the status it returns.
int check_attn_args(const tm_attn_params* p, const tm_attn_tuning* tuning) {
  const float rescale_threshold = tuning ? tuning->rescale_threshold : 0.f;
  const int kernel_choice = tuning ? tuning->force_general : 0;  // 0 auto, 1 general
  const int numerics = tuning ? tuning->numerics : TM_NUMERICS_GPU;
  if (p == nullptr) return TM_ERR_NULL;
  if (p->q == nullptr || p->k == nullptr || p->v == nullptr || p->out == nullptr || p->cu_seqlens_q == nullptr ||
      p->cu_seqlens_k == nullptr)
    return TM_ERR_NULL;
  if (p->batch < 0 || p->heads_q <= 0 || p->heads_k <= 0 || p->heads_q % p->heads_k != 0) return TM_ERR_SHAPE;
  if (p->head_dim != 64 && p->head_dim != 128) return TM_ERR_UNSUPPORTED;
  if (p->block_m != 64 && p->block_m != 128) return TM_ERR_UNSUPPORTED;
  if (p->block_n <= 0 || p->block_n % 64 != 0) return TM_ERR_UNSUPPORTED;
  if (p->block_n_mask <= 0 || p->block_n_mask % p->block_n != 0) return TM_ERR_SHAPE;
  if (p->routing_mode < 0 || p->routing_mode > 2) return TM_ERR_SHAPE;
  if (rescale_threshold < 0.f || rescale_threshold > 15.f) return TM_ERR_SHAPE;
  if (kernel_choice != 0 && kernel_choice != 1) return TM_ERR_SHAPE;
  if (numerics != TM_NUMERICS_GPU && numerics != TM_NUMERICS_EXACT) return TM_ERR_SHAPE;
  if (p->routing_mode == TM_ROUTE_MIXED && p->precision_bitmask == nullptr) return TM_ERR_NULL;
  const bool need_int8 = p->routing_mode != TM_ROUTE_FP16;
  const bool fuse_q = need_int8 && p->q8 == nullptr;
  if (need_int8) {
    if (p->k8 == nullptr || p->k_scale == nullptr || p->cu_k_scale == nullptr) return TM_ERR_NULL;
    if (p->blkk <= 0 || p->blkk % 64 != 0) return TM_ERR_UNSUPPORTED;
    if (fuse_q && p->blkq != 128) return TM_ERR_UNSUPPORTED;
    if (!fuse_q && (p->q_scale == nullptr || p->cu_q_scale == nullptr || p->blkq <= 0)) return TM_ERR_NULL;
  }
  // INT8-V PV path: INT8-routed tiles multiply fp16(p * sv) by fp16(v8) (:449-497).
  const bool v8_path = need_int8 && !p->int8_use_fp16_v;
  if (v8_path && (p->v_scale == nullptr || p->cu_v_scale == nullptr)) return TM_ERR_NULL;
  // The int8 codes feed the general kernel, their fp16 copy the paired one.
  if (v8_path && p->v8 == nullptr && !(p->v8_f16 != nullptr && paired_shape(p, tuning))) return TM_ERR_NULL;
  if (p->bias != nullptr && reinterpret_cast<uintptr_t>(p->bias) % 2 != 0) return TM_ERR_ALIGN;
  if (p->batch == 0 || p->max_seqlen_q == 0) return TM_OK;
  if (p->max_seqlen_k > 0 && (p->max_seqlen_k + p->block_n_mask - 1) / p->block_n_mask > 64) return TM_ERR_SHAPE;
  // Alignment: 16-byte rows for TMA and vector loads/stores.
  const int64_t strides_fp16[] = {p->q_stride_tok, p->q_stride_head, p->k_stride_tok, p->k_stride_head,
                                  p->v_stride_tok, p->v_stride_head, p->o_stride_tok, p->o_stride_head};
  for (int64_t s : strides_fp16)
    if (s % 8 != 0) return TM_ERR_ALIGN;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out)) return TM_ERR_ALIGN;
  if (need_int8) {
    if (!aligned16(p->k8) || p->k8_stride_tok % 16 != 0 || p->k8_stride_head % 16 != 0) return TM_ERR_ALIGN;
    if (!fuse_q && (!aligned16(p->q8) || p->q8_stride_tok % 16 != 0 || p->q8_stride_head % 16 != 0))
      return TM_ERR_ALIGN;
  }
  if (v8_path && p->v8 != nullptr && (!aligned16(p->v8) || p->v8_stride_tok % 16 != 0 || p->v8_stride_head % 16 != 0))
    return TM_ERR_ALIGN;
  if (v8_path && p->v8_f16 != nullptr &&
      (!aligned16(p->v8_f16) || p->v8_f16_stride_tok % 8 != 0 || p->v8_f16_stride_head % 8 != 0))
    return TM_ERR_ALIGN;
  if (p->heads_q > 65535 || p->batch > 65535) return TM_ERR_SHAPE;
  return TM_OK;
}

}  // namespace tilemix

extern "C" int tm_attn_fwd(const tm_attn_params* p, void* stream) { return tm_attn_fwd_ex(p, nullptr, stream); }

extern "C" int tm_attn_fwd_ex(const tm_attn_params* p, const tm_attn_tuning* tuning, void* stream) {
  using namespace tilemix;
  const int rc0 = check_attn_args(p, tuning);
  if (rc0 != TM_OK) return rc0;
  if (p->batch == 0 || p->max_seqlen_q == 0) return TM_OK;
  const float rescale_threshold = tuning ? tuning->rescale_threshold : 0.f;
  const int numerics = tuning ? tuning->numerics : TM_NUMERICS_GPU;
  const bool need_int8 = p->routing_mode != TM_ROUTE_FP16;
  const bool fuse_q = need_int8 && p->q8 == nullptr;
  const bool v8_path = need_int8 && !p->int8_use_fp16_v;
  const int D = p->head_dim;
  CUtensorMap m_k16, m_k8, m_v;
  int rc = make_map(&m_k16, p->k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, p->heads_k, p->k_tokens, p->k_stride_head,
                    p->k_stride_tok, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TM_OK) return rc;
  rc = make_map(&m_v, p->v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, p->heads_k, p->k_tokens, p->v_stride_head,
                p->v_stride_tok, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TM_OK) return rc;
  if (need_int8) {
    rc = make_map(&m_k8, p->k8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, p->heads_k, p->k_tokens, p->k8_stride_head,
                  p->k8_stride_tok, D, D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != TM_OK) return rc;
  } else {
    m_k8 = m_k16;  // never read
  }
  CUtensorMap m_v8 = m_k8;  // read only on the INT8-V path of the general kernel
  const bool paired = paired_shape(p, tuning) && (!v8_path || p->v8_f16 != nullptr);
  if (v8_path && !paired) {
    rc = make_map(&m_v8, p->v8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, p->heads_k, p->k_tokens, p->v8_stride_head,
                  p->v8_stride_tok, D, D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != TM_OK) return rc;
  }

  AttnArgs a;
  a.q = static_cast<const __half*>(p->q);
  a.q_st = p->q_stride_tok;
  a.q_sh = p->q_stride_head;
  a.out = static_cast<__half*>(p->out);
  a.o_st = p->o_stride_tok;
  a.o_sh = p->o_stride_head;
  a.o_vec32 = (reinterpret_cast<uintptr_t>(p->out) % 32 == 0 && p->o_stride_tok % 16 == 0 && p->o_stride_head % 16 == 0) ? 1 : 0;
  a.q8 = p->q8;
  a.q8_st = p->q8_stride_tok;
  a.q8_sh = p->q8_stride_head;
  a.q_scale = static_cast<const __half*>(p->q_scale);
  a.cu_qs = p->cu_q_scale;
  a.k_scale = static_cast<const __half*>(p->k_scale);
  a.cu_ks = p->cu_k_scale;
  a.cu_q = p->cu_seqlens_q;
  a.cu_k = p->cu_seqlens_k;
  a.bitmask = p->precision_bitmask;
  a.HQ = p->heads_q;
  a.HK = p->heads_k;
  a.group = p->heads_q / p->heads_k;
  a.D = D;
  a.block_m = p->block_m;
  a.block_n_mask = p->block_n_mask;
  a.blkq = p->blkq;
  a.blkk = p->blkk;
  a.causal = p->causal;
  a.mode = p->routing_mode;
  a.fuse_q = fuse_q ? 1 : 0;
  // qk_scale = fp32(sm_scale) * fp32(log2 e), as the reference evaluates it (:639).
  a.qk_scale = p->sm_scale * 1.44269502162933349609375f;
  a.rescale_threshold = rescale_threshold;
  a.numerics = numerics == TM_NUMERICS_GPU ? kNumericsGpu : kNumericsExact;
  a.err = p->error_flag;
  a.v8_path = v8_path ? 1 : 0;
  a.v_scale = static_cast<const __half*>(p->v_scale);
  a.cu_vs = p->cu_v_scale;
  a.bias = static_cast<const __half*>(p->bias);
  a.b_sh = p->bias_stride[1];
  a.b_sm = p->bias_stride[2];
  a.b_sn = p->bias_stride[3];

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Bias, prequantised Q and INT8-V from the int8 codes alone run on the general kernel.
  if (paired) {
    // The paired kernel fetches all 128 dims of a tile in one 4-D copy.
    CUtensorMap q4, k4, v4, vq4;
    rc = make_map_d128(&q4, p->q, p->heads_q, p->q_tokens, p->q_stride_head, p->q_stride_tok, 128);
    if (rc != TM_OK) return rc;
    rc = make_map_d128(&k4, p->k, p->heads_k, p->k_tokens, p->k_stride_head, p->k_stride_tok, 64);
    if (rc != TM_OK) return rc;
    rc = make_map_d128(&v4, p->v, p->heads_k, p->k_tokens, p->v_stride_head, p->v_stride_tok, 64);
    if (rc != TM_OK) return rc;
    vq4 = v4;  // read only on the INT8-V path
    if (v8_path) {
      rc = make_map_d128(&vq4, p->v8_f16, p->heads_k, p->k_tokens, p->v8_f16_stride_head, p->v8_f16_stride_tok, 64);
      if (rc != TM_OK) return rc;
    }
    return launch_attn_paired(q4, k4, m_k8, v4, vq4, a, p->batch, p->max_seqlen_q, st);
  }
  const int tiles = (p->max_seqlen_q + 127) / 128;
  return launch_attn_general(m_k16, m_k8, m_v, m_v8, a, tiles, p->heads_q, p->batch, st);
}

extern "C" const char* tm_status_string(int status) {
  switch (status) {
    case TM_OK:
      return "ok";
    case TM_ERR_NULL:
      return "a required pointer is NULL";
    case TM_ERR_SHAPE:
      return "unsupported or inconsistent sizes";
    case TM_ERR_ALIGN:
      return "pointer or stride alignment violated (16-byte rows required)";
    case TM_ERR_UNSUPPORTED:
      return "option not implemented by the sm_100a kernels";
    case TM_ERR_LAUNCH:
      return "CUDA launch failed";
    case TM_ERR_TMAP:
      return "TMA descriptor encoding failed";
    default:
      return "unknown status";
  }
}
