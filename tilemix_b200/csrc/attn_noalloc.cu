// tm_attn_fwd_noalloc: the routed attention forward for callers that cannot
// allocate device memory. The quantised K operand (int8 codes, fp16 block
// scales and their per-sequence block offsets), which tm_attn_fwd takes from
// caller-owned buffers, lives here in fixed-size file-scope device arrays.
// The entry point allocates nothing: no cudaMalloc / cudaFree and no library
// call that allocates.
//
// Scratch capacity (device memory the module holds on every device where it is
// loaded; under CUDA's lazy module loading that happens at the latest when the
// first call on the device resolves the scratch address):
//   K codes   16 MiB  -> k_tokens * heads_k * head_dim <= 16,777,216
//   K scales  512 KiB -> (k_tokens / blkk + batch) * heads_k <= 262,144
//   offsets   256 KiB -> batch + 1 <= 65,536
// Larger problems are rejected with TM_ERR_UNSUPPORTED, and every argument is
// checked (tm_attn_fwd_ex's checks, with the scratch standing in for the K
// operand) before anything is queued on the stream. Every scratch word a call
// reads is written earlier in the same call on the same stream (the offsets by
// prefix_blocks_kernel, codes and scales by the quantiser), so nothing has to
// start at zero. Calls that can be in flight at the same time (other streams,
// other host threads) share the scratch and race.
#include <mutex>

#include "common.cuh"
#include "tilemix_b200.h"

namespace tilemix {

int check_attn_args(const tm_attn_params* p, const tm_attn_tuning* tuning);

namespace noalloc {

constexpr int64_t kMaxK8Bytes = 16ll << 20;
constexpr int64_t kMaxScales = 262144;
constexpr int64_t kMaxOffsets = 65536;

static __device__ __align__(256) int8_t g_k8[kMaxK8Bytes];
static __device__ __align__(256) __half g_k_scale[kMaxScales];
static __device__ __align__(256) int32_t g_cu_k_scale[kMaxOffsets];

struct Scratch {
  int8_t* k8 = nullptr;
  __half* k_scale = nullptr;
  int32_t* cu_k_scale = nullptr;
};

// Exclusive prefix of ceil(T_b / blk) over the batch (one thread; batch is small).
__global__ void prefix_blocks_kernel(const int32_t* __restrict__ cu_seqlens, int batch, int blk,
                                     int32_t* __restrict__ cu_blocks) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int32_t acc = 0;
  cu_blocks[0] = 0;
  for (int b = 0; b < batch; ++b) {
    const int32_t len = cu_seqlens[b + 1] - cu_seqlens[b];
    acc += (len + blk - 1) / blk;
    cu_blocks[b + 1] = acc;
  }
}

// Device addresses of the scratch arrays, resolved once per device (with that
// device current) and cached.
int scratch_for_current_device(Scratch* out) {
  static std::mutex mu;
  static Scratch cache[64];
  static bool ready[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(mu);
  if (!ready[dev]) {
    Scratch s;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.k8), g_k8) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.k_scale), g_k_scale) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.cu_k_scale), g_cu_k_scale) != cudaSuccess)
      return TM_ERR_LAUNCH;
    cache[dev] = s;
    ready[dev] = true;
  }
  *out = cache[dev];
  return TM_OK;
}

}  // namespace noalloc
}  // namespace tilemix

extern "C" int tm_attn_fwd_noalloc(const tm_attn_params* p, const tm_attn_tuning* tuning, void* stream) {
  using namespace tilemix::noalloc;
  if (p == nullptr) return TM_ERR_NULL;
  if (p->routing_mode == TM_ROUTE_FP16) return tm_attn_fwd_ex(p, tuning, stream);  // no K operand needed
  // The K operand comes from the library's scratch.
  if (p->k8 != nullptr || p->k_scale != nullptr || p->cu_k_scale != nullptr) return TM_ERR_UNSUPPORTED;
  if (p->k == nullptr || p->cu_seqlens_k == nullptr) return TM_ERR_NULL;
  if (p->batch < 0 || p->heads_k <= 0 || p->k_tokens < 0 || (p->head_dim != 64 && p->head_dim != 128))
    return TM_ERR_SHAPE;
  if (p->blkk != 64 && p->blkk != 128) return TM_ERR_UNSUPPORTED;
  const int numerics = tuning ? tuning->numerics : TM_NUMERICS_GPU;
  if (numerics != TM_NUMERICS_GPU && numerics != TM_NUMERICS_EXACT) return TM_ERR_SHAPE;
  const int64_t codes = p->k_tokens * p->heads_k * static_cast<int64_t>(p->head_dim);
  const int64_t scale_rows = p->k_tokens / p->blkk + p->batch;  // >= sum_b ceil(T_b / blkk)
  if (codes > kMaxK8Bytes || scale_rows * p->heads_k > kMaxScales || p->batch + 1 > kMaxOffsets)
    return TM_ERR_UNSUPPORTED;

  Scratch s;
  int rc = scratch_for_current_device(&s);
  if (rc != TM_OK) return rc;
  const int64_t k8_st = static_cast<int64_t>(p->heads_k) * p->head_dim;
  tm_attn_params q = *p;
  q.k8 = s.k8;
  q.k8_stride_tok = k8_st;
  q.k8_stride_head = p->head_dim;
  q.k_scale = s.k_scale;
  q.cu_k_scale = s.cu_k_scale;
  rc = tilemix::check_attn_args(&q, tuning);
  if (rc != TM_OK) return rc;
  if (p->batch == 0 || p->max_seqlen_q == 0) return TM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  prefix_blocks_kernel<<<1, 32, 0, st>>>(p->cu_seqlens_k, p->batch, p->blkk, s.cu_k_scale);
  if (cudaGetLastError() != cudaSuccess) return TM_ERR_LAUNCH;
  rc = tm_quant_per_block_int8_ex(p->k, p->k_stride_tok, p->k_stride_head, p->cu_seqlens_k, s.cu_k_scale, p->batch,
                                  p->heads_k, p->head_dim, p->blkk, p->max_seqlen_k, 1.0f, s.k8, k8_st, p->head_dim,
                                  nullptr, s.k_scale, numerics, stream);
  if (rc != TM_OK) return rc;
  return tm_attn_fwd_ex(&q, tuning, stream);
}
