// Per-block symmetric INT8 quantiser over varlen packed [tokens, heads, dim]
// fp16 tensors.
//
// Follows attention/triton/quant_per_block_varlen.py:6-45 (kernel) and
// :48-75 (per_block_int8_single launch): one block = BLK consecutive tokens of
// one sequence and one head; scale = max|x * sm_scale| / 127 (fp32), code =
// trunc(x / scale + 0.5 * sign). Scales are laid out [sum_b ceil(T_b/BLK), H]
// with the per-sequence block offsets in cu_seqlens_scale.
//
// B200 design: HBM-bound. One 128-thread CTA per (block, head); every thread
// keeps its slice of the block in registers between the max pass and the
// quantise pass, so the input is read from HBM exactly once; 16-byte vector
// loads, 8-byte vector stores. The grid is (blocks, heads, batch) like the
// reference's, which gives tens of thousands of CTAs at the BASELINE shapes,
// far more than the 148 SMs x resident CTAs.
#include "common.cuh"
#include "tilemix_b200.h"

namespace tilemix {

constexpr int kQuantThreads = 128;
constexpr int kQuantMaxVec = 16;  // 16-byte vectors held per thread (BLK*D <= 128*8*16)

__device__ __forceinline__ float block_absmax_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) m = fmaxf(m, red[w]);
  return m;
}

template <int kNumerics>
__global__ void __launch_bounds__(kQuantThreads) quant_per_block_int8_kernel(
    const __half* __restrict__ x, int64_t x_stride_tok, int64_t x_stride_head, const int32_t* __restrict__ cu_seqlens,
    const int32_t* __restrict__ cu_scale, int heads, int dim, int blk, float sm_scale, int8_t* __restrict__ out,
    int64_t o_stride_tok, int64_t o_stride_head, float* __restrict__ scale_f32, __half* __restrict__ scale_f16) {
  __shared__ float red[kQuantThreads / 32];
  const int off_blk = blockIdx.x, off_h = blockIdx.y, off_b = blockIdx.z;
  const int start = cu_seqlens[off_b];
  const int len = cu_seqlens[off_b + 1] - start;
  if (off_blk * blk >= len) return;
  const int rows = min(blk, len - off_blk * blk);
  const int vec_per_row = dim >> 3;
  const int nvec = rows * vec_per_row;
  const int64_t tok0 = static_cast<int64_t>(start) + static_cast<int64_t>(off_blk) * blk;
  const __half* xb = x + tok0 * x_stride_tok + static_cast<int64_t>(off_h) * x_stride_head;
  int8_t* ob = out + tok0 * o_stride_tok + static_cast<int64_t>(off_h) * o_stride_head;

  float amax = 0.f;
  const bool in_regs = (blk * vec_per_row) <= kQuantThreads * kQuantMaxVec;
  uint4 regs[kQuantMaxVec];
  if (in_regs) {
#pragma unroll
    for (int i = 0; i < kQuantMaxVec; ++i) {
      const int v = i * kQuantThreads + threadIdx.x;
      regs[i] = make_uint4(0, 0, 0, 0);
      if (v < nvec) {
        const int r = v / vec_per_row, c = (v % vec_per_row) << 3;
        regs[i] = __ldg(reinterpret_cast<const uint4*>(xb + r * x_stride_tok + c));
        const __half2* h = reinterpret_cast<const __half2*>(&regs[i]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __half22float2(h[e]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x * sm_scale), fabsf(f.y * sm_scale)));
        }
      }
    }
  } else {
    for (int v = threadIdx.x; v < nvec; v += kQuantThreads) {
      const int r = v / vec_per_row, c = (v % vec_per_row) << 3;
      uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + r * x_stride_tok + c));
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __half22float2(h[e]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x * sm_scale), fabsf(f.y * sm_scale)));
      }
    }
  }
  amax = block_absmax_reduce(amax, red);
  const float scale = quant_scale<kNumerics>(amax);

  auto quant_vec = [&](const uint4& u) -> uint2 {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __half22float2(h[e]);
      const uint32_t a = static_cast<uint32_t>(quant_code<kNumerics>(f.x * sm_scale, scale)) & 0xFFu;
      const uint32_t b = static_cast<uint32_t>(quant_code<kNumerics>(f.y * sm_scale, scale)) & 0xFFu;
      const uint32_t pair = a | (b << 8);
      if (e < 2)
        lo |= pair << (16 * e);
      else
        hi |= pair << (16 * (e - 2));
    }
    return make_uint2(lo, hi);
  };

  if (in_regs) {
#pragma unroll
    for (int i = 0; i < kQuantMaxVec; ++i) {
      const int v = i * kQuantThreads + threadIdx.x;
      if (v < nvec) {
        const int r = v / vec_per_row, c = (v % vec_per_row) << 3;
        *reinterpret_cast<uint2*>(ob + r * o_stride_tok + c) = quant_vec(regs[i]);
      }
    }
  } else {
    for (int v = threadIdx.x; v < nvec; v += kQuantThreads) {
      const int r = v / vec_per_row, c = (v % vec_per_row) << 3;
      uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + r * x_stride_tok + c));
      *reinterpret_cast<uint2*>(ob + r * o_stride_tok + c) = quant_vec(u);
    }
  }
  if (threadIdx.x == 0) {
    const int64_t sidx = (static_cast<int64_t>(cu_scale[off_b]) + off_blk) * heads + off_h;
    if (scale_f32 != nullptr) scale_f32[sidx] = scale;
    if (scale_f16 != nullptr) scale_f16[sidx] = __float2half_rn(scale);
  }
}

// The same quantisation for sm_scale == 1, head dims 64 / 128 and blocks of
// 64 / 128 tokens: the case of every K (and V) the attention quantises. Sizes
// are compile-time (no per-vector division), the block stays in registers, and
// the codes come from quant_code_pair (the quotient of the numerics, rounded on
// the FMA pipe; exact numerics' Markstein quotient is the IEEE one here because
// every |x| of a block is at most its absmax m, an fp16 value, with scale =
// m / 127, checked against the reference rounding for all such pairs). A block
// whose scale is 0 or not finite quantises to zeros and a NaN value to 0, as in
// the reference.
template <int kNumerics, int DIM, int BLK>
__global__ void __launch_bounds__(kQuantThreads) quant_per_block_int8_unit_kernel(
    const __half* __restrict__ x, int64_t x_stride_tok, int64_t x_stride_head, const int32_t* __restrict__ cu_seqlens,
    const int32_t* __restrict__ cu_scale, int heads, int8_t* __restrict__ out, int64_t o_stride_tok,
    int64_t o_stride_head, float* __restrict__ scale_f32, __half* __restrict__ scale_f16,
    __half* __restrict__ out16 = nullptr, int64_t o16_stride_tok = 0, int64_t o16_stride_head = 0) {
  constexpr int kVecPerRow = DIM / 8;
  constexpr int kVecs = BLK * kVecPerRow / kQuantThreads;  // 16-byte vectors per thread
  __shared__ float red[kQuantThreads / 32];
  const int off_blk = blockIdx.x, off_h = blockIdx.y, off_b = blockIdx.z;
  const int start = cu_seqlens[off_b];
  const int len = cu_seqlens[off_b + 1] - start;
  if (off_blk * BLK >= len) return;
  const int rows = min(BLK, len - off_blk * BLK);
  const int64_t tok0 = static_cast<int64_t>(start) + static_cast<int64_t>(off_blk) * BLK;
  const __half* xb = x + tok0 * x_stride_tok + static_cast<int64_t>(off_h) * x_stride_head;
  int8_t* ob = out == nullptr ? nullptr : out + tok0 * o_stride_tok + static_cast<int64_t>(off_h) * o_stride_head;
  __half* ob16 =
      out16 == nullptr ? nullptr : out16 + tok0 * o16_stride_tok + static_cast<int64_t>(off_h) * o16_stride_head;
  const int c = (threadIdx.x % kVecPerRow) * 8;
  uint4 v[kVecs];
  uint32_t am2 = 0u;
#pragma unroll
  for (int i = 0; i < kVecs; ++i) {
    const int r = i * (kQuantThreads / kVecPerRow) + threadIdx.x / kVecPerRow;
    v[i] = r < rows ? __ldg(reinterpret_cast<const uint4*>(xb + r * x_stride_tok + c)) : make_uint4(0, 0, 0, 0);
    uint32_t a, b;
    asm("max.f16x2 %0, %1, %2;" : "=r"(a) : "r"(v[i].x & 0x7FFF7FFFu), "r"(v[i].y & 0x7FFF7FFFu));
    asm("max.f16x2 %0, %1, %2;" : "=r"(b) : "r"(v[i].z & 0x7FFF7FFFu), "r"(v[i].w & 0x7FFF7FFFu));
    asm("max.f16x2 %0, %1, %2;" : "=r"(a) : "r"(a), "r"(b));
    asm("max.f16x2 %0, %1, %2;" : "=r"(am2) : "r"(am2), "r"(a));
  }
  const float2 amf = __half22float2(*reinterpret_cast<const __half2*>(&am2));
  const float amax = block_absmax_reduce(fmaxf(amf.x, amf.y), red);
  const float scale = quant_scale<kNumerics>(amax);
  const bool finite = scale > 0.f && scale <= 3.4028235e38f;
  QuantDiv qd;
  qd.init(scale);
#pragma unroll
  for (int i = 0; i < kVecs; ++i) {
    const int r = i * (kQuantThreads / kVecPerRow) + threadIdx.x / kVecPerRow;
    if (r >= rows) continue;
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
    uint32_t u[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      if (finite) {
        quant_code_pair<kNumerics>(f.x, f.y, qd, &u[2 * e], &u[2 * e + 1]);
        if (f.x != f.x) u[2 * e] = 0u;  // NaN truncates to 0 in the reference
        if (f.y != f.y) u[2 * e + 1] = 0u;
      } else {
        u[2 * e] = 0u;
        u[2 * e + 1] = 0u;
      }
    }
    const uint32_t lo = __byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410);
    const uint32_t hi = __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410);
    if (ob != nullptr) *reinterpret_cast<uint2*>(ob + r * o_stride_tok + c) = make_uint2(lo, hi);
    if (ob16 != nullptr) {
      // The same codes as exact fp16 values (small integers).
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half2 h2 = __halves2half2(__short2half_rn(static_cast<short>(static_cast<int8_t>(u[2 * e] & 0xFFu))),
                                          __short2half_rn(static_cast<short>(static_cast<int8_t>(u[2 * e + 1] & 0xFFu))));
        w[e] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      *reinterpret_cast<uint4*>(ob16 + r * o16_stride_tok + c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if (threadIdx.x == 0) {
    const int64_t sidx = (static_cast<int64_t>(cu_scale[off_b]) + off_blk) * heads + off_h;
    if (scale_f32 != nullptr) scale_f32[sidx] = scale;
    if (scale_f16 != nullptr) scale_f16[sidx] = __float2half_rn(scale);
  }
}

}  // namespace tilemix

namespace {

template <int kNumerics>
int launch_quant(const void* x, int64_t x_stride_tok, int64_t x_stride_head, const int32_t* cu_seqlens,
                 const int32_t* cu_scale, int heads, int dim, int blk, float sm_scale, int8_t* out,
                 int64_t out_stride_tok, int64_t out_stride_head, float* scale_f32, void* scale_f16, dim3 grid,
                 cudaStream_t st, void* out16 = nullptr, int64_t o16_st = 0, int64_t o16_sh = 0) {
  using namespace tilemix;
  const __half* xh = static_cast<const __half*>(x);
  __half* s16 = static_cast<__half*>(scale_f16);
  if (sm_scale == 1.0f && (dim == 64 || dim == 128) && (blk == 64 || blk == 128)) {
    if (dim == 128 && blk == 64)
      quant_per_block_int8_unit_kernel<kNumerics, 128, 64><<<grid, kQuantThreads, 0, st>>>(
          xh, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, out, out_stride_tok, out_stride_head, scale_f32, s16,
          static_cast<__half*>(out16), o16_st, o16_sh);
    else if (dim == 128)
      quant_per_block_int8_unit_kernel<kNumerics, 128, 128><<<grid, kQuantThreads, 0, st>>>(
          xh, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, out, out_stride_tok, out_stride_head, scale_f32, s16,
          static_cast<__half*>(out16), o16_st, o16_sh);
    else if (blk == 64)
      quant_per_block_int8_unit_kernel<kNumerics, 64, 64><<<grid, kQuantThreads, 0, st>>>(
          xh, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, out, out_stride_tok, out_stride_head, scale_f32, s16,
          static_cast<__half*>(out16), o16_st, o16_sh);
    else
      quant_per_block_int8_unit_kernel<kNumerics, 64, 128><<<grid, kQuantThreads, 0, st>>>(
          xh, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, out, out_stride_tok, out_stride_head, scale_f32, s16,
          static_cast<__half*>(out16), o16_st, o16_sh);
  } else {
    quant_per_block_int8_kernel<kNumerics><<<grid, kQuantThreads, 0, st>>>(
        xh, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, dim, blk, sm_scale, out, out_stride_tok,
        out_stride_head, scale_f32, s16);
  }
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace

extern "C" int tm_quant_per_block_int8_ex(const void* x, int64_t x_stride_tok, int64_t x_stride_head,
                                          const int32_t* cu_seqlens, const int32_t* cu_scale, int batch, int heads,
                                          int dim, int blk, int max_seqlen, float sm_scale, int8_t* out,
                                          int64_t out_stride_tok, int64_t out_stride_head, float* scale_f32,
                                          void* scale_f16, int numerics, void* stream) {
  if (x == nullptr || out == nullptr || cu_seqlens == nullptr || cu_scale == nullptr) return TM_ERR_NULL;
  if (batch < 0 || heads <= 0 || dim <= 0 || blk <= 0 || max_seqlen < 0) return TM_ERR_SHAPE;
  if (numerics != TM_NUMERICS_GPU && numerics != TM_NUMERICS_EXACT) return TM_ERR_SHAPE;
  if ((dim & 7) != 0) return TM_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (x_stride_tok & 7) != 0 || (x_stride_head & 7) != 0)
    return TM_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0 || (out_stride_tok & 7) != 0 || (out_stride_head & 7) != 0)
    return TM_ERR_ALIGN;
  if (batch == 0 || max_seqlen == 0) return TM_OK;
  const int nblk = (max_seqlen + blk - 1) / blk;
  if (heads > 65535 || batch > 65535) return TM_ERR_SHAPE;
  dim3 grid(nblk, heads, batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (numerics == TM_NUMERICS_GPU)
    return launch_quant<tilemix::kNumericsGpu>(x, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, dim, blk,
                                                sm_scale, out, out_stride_tok, out_stride_head, scale_f32, scale_f16,
                                                grid, st);
  return launch_quant<tilemix::kNumericsExact>(x, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, dim, blk,
                                                sm_scale, out, out_stride_tok, out_stride_head, scale_f32, scale_f16,
                                                grid, st);
}

extern "C" int tm_quant_per_block_int8_f16(const void* x, int64_t x_stride_tok, int64_t x_stride_head,
                                           const int32_t* cu_seqlens, const int32_t* cu_scale, int batch, int heads,
                                           int dim, int blk, int max_seqlen, int8_t* out, int64_t out_stride_tok,
                                           int64_t out_stride_head, void* out_f16, int64_t out_f16_stride_tok,
                                           int64_t out_f16_stride_head, float* scale_f32, void* scale_f16,
                                           int numerics, void* stream) {
  if (x == nullptr || out_f16 == nullptr || cu_seqlens == nullptr || cu_scale == nullptr) return TM_ERR_NULL;
  if (batch < 0 || heads <= 0 || max_seqlen < 0) return TM_ERR_SHAPE;
  if (numerics != TM_NUMERICS_GPU && numerics != TM_NUMERICS_EXACT) return TM_ERR_SHAPE;
  if ((dim != 64 && dim != 128) || (blk != 64 && blk != 128)) return TM_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (x_stride_tok & 7) != 0 || (x_stride_head & 7) != 0)
    return TM_ERR_ALIGN;
  if (out != nullptr &&
      ((reinterpret_cast<uintptr_t>(out) & 7u) != 0 || (out_stride_tok & 7) != 0 || (out_stride_head & 7) != 0))
    return TM_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(out_f16) & 15u) != 0 || (out_f16_stride_tok & 7) != 0 ||
      (out_f16_stride_head & 7) != 0)
    return TM_ERR_ALIGN;
  if (heads > 65535 || batch > 65535) return TM_ERR_SHAPE;
  if (batch == 0 || max_seqlen == 0) return TM_OK;
  dim3 grid((max_seqlen + blk - 1) / blk, heads, batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (numerics == TM_NUMERICS_GPU)
    return launch_quant<tilemix::kNumericsGpu>(x, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, dim, blk,
                                                1.0f, out, out_stride_tok, out_stride_head, scale_f32, scale_f16, grid,
                                                st, out_f16, out_f16_stride_tok, out_f16_stride_head);
  return launch_quant<tilemix::kNumericsExact>(x, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, heads, dim, blk,
                                                1.0f, out, out_stride_tok, out_stride_head, scale_f32, scale_f16, grid,
                                                st, out_f16, out_f16_stride_tok, out_f16_stride_head);
}

extern "C" int tm_quant_per_block_int8(const void* x, int64_t x_stride_tok, int64_t x_stride_head,
                                       const int32_t* cu_seqlens, const int32_t* cu_scale, int batch, int heads,
                                       int dim, int blk, int max_seqlen, float sm_scale, int8_t* out,
                                       int64_t out_stride_tok, int64_t out_stride_head, float* scale_f32,
                                       void* scale_f16, void* stream) {
  return tm_quant_per_block_int8_ex(x, x_stride_tok, x_stride_head, cu_seqlens, cu_scale, batch, heads, dim, blk,
                                    max_seqlen, sm_scale, out, out_stride_tok, out_stride_head, scale_f32, scale_f16,
                                    TM_NUMERICS_GPU, stream);
}
