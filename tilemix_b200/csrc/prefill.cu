// Llama prefill companions of the TileMix model integration (sm_100a):
// split-half RoPE with token-major outputs (optionally quantising the rotated
// K for the attention in the same pass), the fused SiLU-multiply of the MLP
// and RMSNorm. Same arithmetic as the reference's prefill path
// (models/tilemix_llama.py:718-895); all three are HBM-bound elementwise /
// row-reduction kernels with 16-byte accesses.
#include <cuda_fp16.h>

#include "common.cuh"
#include "tilemix_b200.h"

namespace tilemix {
namespace prefill {

__device__ __forceinline__ float h2f(unsigned short b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ unsigned short f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// RoPE of 8 rotation pairs (dims [i, i+8) and [i+D/2, i+D/2+8)) of one row:
// out[d] = fp16(fp16(x[d] * c[d]) + fp16(sign(d) * x[(d + D/2) % D] * s[d])),
// sign -1 on the first half, the sum formed in fp32 (:805-822). The fp32
// product of two fp16 values is exact, so each fp16 rounding is the only one.
__device__ __forceinline__ void rope8(const uint4& xl, const uint4& xh, const uint4& cl, const uint4& ch,
                                      const uint4& sl, const uint4& sh, uint4& ol, uint4& oh) {
  const unsigned short* x0 = reinterpret_cast<const unsigned short*>(&xl);
  const unsigned short* x1 = reinterpret_cast<const unsigned short*>(&xh);
  const unsigned short* c0 = reinterpret_cast<const unsigned short*>(&cl);
  const unsigned short* c1 = reinterpret_cast<const unsigned short*>(&ch);
  const unsigned short* s0 = reinterpret_cast<const unsigned short*>(&sl);
  const unsigned short* s1 = reinterpret_cast<const unsigned short*>(&sh);
  unsigned short* o0 = reinterpret_cast<unsigned short*>(&ol);
  unsigned short* o1 = reinterpret_cast<unsigned short*>(&oh);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a0 = h2f(f2h(h2f(x0[e]) * h2f(c0[e])));
    const float b0 = h2f(f2h(-h2f(x1[e]) * h2f(s0[e])));
    o0[e] = f2h(a0 + b0);
    const float a1 = h2f(f2h(h2f(x1[e]) * h2f(c1[e])));
    const float b1 = h2f(f2h(h2f(x0[e]) * h2f(s1[e])));
    o1[e] = f2h(a1 + b1);
  }
}

struct RopeArgs {
  const __half* src;
  int64_t sb, sh, st;  // element strides of [B, H, T, D] (d stride 1)
  const __half* cos;
  const __half* sin;
  int64_t cb, ct, sbb, stt;  // cos / sin strides (batch stride 0 when broadcast)
  __half* dst;               // [B, T, H, D] contiguous
  int B, H, T, D;
};

// One thread per 8 rotation pairs of a row.
__global__ void rope_kernel(const RopeArgs a) {
  const int groups = a.D / 16;
  const int64_t n = static_cast<int64_t>(a.B) * a.T * a.H * groups;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int u = static_cast<int>(i % groups);
  int64_t r = i / groups;  // row index in [B, T, H] order
  const int h = static_cast<int>(r % a.H);
  r /= a.H;
  const int t = static_cast<int>(r % a.T);
  const int b = static_cast<int>(r / a.T);
  const int half = a.D / 2;
  const __half* x = a.src + b * a.sb + h * a.sh + t * a.st + 8 * u;
  const __half* c = a.cos + b * a.cb + t * a.ct + 8 * u;
  const __half* s = a.sin + b * a.sbb + t * a.stt + 8 * u;
  const uint4 xl = *reinterpret_cast<const uint4*>(x), xh = *reinterpret_cast<const uint4*>(x + half);
  const uint4 cl = __ldg(reinterpret_cast<const uint4*>(c)), ch = __ldg(reinterpret_cast<const uint4*>(c + half));
  const uint4 sl = __ldg(reinterpret_cast<const uint4*>(s)), sh = __ldg(reinterpret_cast<const uint4*>(s + half));
  uint4 ol, oh;
  rope8(xl, xh, cl, ch, sl, sh, ol, oh);
  __half* o = a.dst + ((static_cast<int64_t>(b) * a.T + t) * a.H + h) * a.D + 8 * u;
  *reinterpret_cast<uint4*>(o) = ol;
  *reinterpret_cast<uint4*>(o + half) = oh;
}

struct RopeQuantArgs {
  RopeArgs r;
  int8_t* k8;         // [B*T, H, D]
  __half* scale16;    // optional [B * ceil(T/blk), H]
  float* scale32;     // optional, same layout
  int blk;
};

constexpr int kQuantThreads = 256;

// One CTA per (sequence, KV head, block of blk tokens): RoPE of the block's K
// rows, then the block's per-head INT8 quantisation of the rotated values
// (quant_per_block_varlen.py:6-45 with sm_scale 1: scale = absmax / 127 in
// fp32, code = trunc(x / scale + 0.5 * sign), with the division of the
// numerics, common.cuh), so the attention's K quantiser need not read K again.
template <int kNumerics, int D, int BLK>
__global__ void __launch_bounds__(kQuantThreads) rope_quant_kernel(const RopeQuantArgs q) {
  constexpr int kGroups = D / 16;
  constexpr int kUnits = BLK * kGroups / kQuantThreads;  // (row, group) units per thread
  static_assert(BLK * kGroups % kQuantThreads == 0, "units per thread");
  __shared__ float red[kQuantThreads / 32];
  const RopeArgs& a = q.r;
  const int blk_idx = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int half = D / 2;
  uint4 ol[kUnits], oh[kUnits];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < kUnits; ++k) {
    const int unit = threadIdx.x + k * kQuantThreads;
    const int u = unit % kGroups, row = unit / kGroups;
    const int t = blk_idx * BLK + row;
    ol[k] = make_uint4(0, 0, 0, 0);
    oh[k] = make_uint4(0, 0, 0, 0);
    if (t < a.T) {
      const __half* x = a.src + b * a.sb + h * a.sh + t * a.st + 8 * u;
      const __half* c = a.cos + b * a.cb + t * a.ct + 8 * u;
      const __half* s = a.sin + b * a.sbb + t * a.stt + 8 * u;
      rope8(*reinterpret_cast<const uint4*>(x), *reinterpret_cast<const uint4*>(x + half),
            __ldg(reinterpret_cast<const uint4*>(c)), __ldg(reinterpret_cast<const uint4*>(c + half)),
            __ldg(reinterpret_cast<const uint4*>(s)), __ldg(reinterpret_cast<const uint4*>(s + half)), ol[k], oh[k]);
      __half* o = a.dst + ((static_cast<int64_t>(b) * a.T + t) * a.H + h) * D + 8 * u;
      *reinterpret_cast<uint4*>(o) = ol[k];
      *reinterpret_cast<uint4*>(o + half) = oh[k];
      const unsigned short* v0 = reinterpret_cast<const unsigned short*>(&ol[k]);
      const unsigned short* v1 = reinterpret_cast<const unsigned short*>(&oh[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fmaxf(fabsf(h2f(v0[e])), fabsf(h2f(v1[e]))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) m = fmaxf(m, red[w]);
  const float scale = quant_scale<kNumerics>(m);
  const bool finite = scale > 0.f && scale <= 3.4028235e38f;
  QuantDiv qd;
  qd.init(scale);
  const int nblk = (a.T + BLK - 1) / BLK;
  if (threadIdx.x == 0) {
    const int64_t si = (static_cast<int64_t>(b) * nblk + blk_idx) * a.H + h;
    if (q.scale32) q.scale32[si] = scale;
    if (q.scale16) q.scale16[si] = __float2half_rn(scale);
  }
#pragma unroll
  for (int k = 0; k < kUnits; ++k) {
    const int unit = threadIdx.x + k * kQuantThreads;
    const int u = unit % kGroups, row = unit / kGroups;
    const int t = blk_idx * BLK + row;
    if (t >= a.T) continue;
    const unsigned short* v0 = reinterpret_cast<const unsigned short*>(&ol[k]);
    const unsigned short* v1 = reinterpret_cast<const unsigned short*>(&oh[k]);
    uint32_t u0[8], u1[8];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      quant_code_pair<kNumerics>(h2f(v0[e]), h2f(v0[e + 1]), qd, &u0[e], &u0[e + 1]);
      quant_code_pair<kNumerics>(h2f(v1[e]), h2f(v1[e + 1]), qd, &u1[e], &u1[e + 1]);
    }
    uint32_t w0[2], w1[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      w0[i] = finite ? __byte_perm(__byte_perm(u0[4 * i], u0[4 * i + 1], 0x0040),
                                   __byte_perm(u0[4 * i + 2], u0[4 * i + 3], 0x0040), 0x5410)
                     : 0u;
      w1[i] = finite ? __byte_perm(__byte_perm(u1[4 * i], u1[4 * i + 1], 0x0040),
                                   __byte_perm(u1[4 * i + 2], u1[4 * i + 3], 0x0040), 0x5410)
                     : 0u;
    }
    int8_t* k8 = q.k8 + ((static_cast<int64_t>(b) * a.T + t) * a.H + h) * D + 8 * u;
    *reinterpret_cast<uint2*>(k8) = make_uint2(w0[0], w0[1]);
    *reinterpret_cast<uint2*>(k8 + half) = make_uint2(w1[0], w1[1]);
  }
}

// fp16(silu(g)) * up (:851-857): silu with the correctly rounded fp32 division
// of g by 1 + exp(-g), rounded to fp16, times up in fp32, rounded to fp16.
__device__ __forceinline__ unsigned short silu_mul1(unsigned short g16, unsigned short u16) {
  const float g = h2f(g16);
  const float act = h2f(f2h(__fdiv_rn(g, 1.0f + expf(-g))));
  return f2h(act * h2f(u16));
}

__global__ void silu_mul_kernel(const __half* gate, const __half* up, __half* out, int64_t n, int vec) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    if (i * 8 >= n) return;
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(gate) + i), u = __ldg(reinterpret_cast<const uint4*>(up) + i);
    const unsigned short* gs = reinterpret_cast<const unsigned short*>(&g);
    const unsigned short* us = reinterpret_cast<const unsigned short*>(&u);
    uint4 o;
    unsigned short* os = reinterpret_cast<unsigned short*>(&o);
#pragma unroll
    for (int e = 0; e < 8; ++e) os[e] = silu_mul1(gs[e], us[e]);
    reinterpret_cast<uint4*>(out)[i] = o;
  } else {
    if (i >= n) return;
    reinterpret_cast<unsigned short*>(out)[i] =
        silu_mul1(reinterpret_cast<const unsigned short*>(gate)[i], reinterpret_cast<const unsigned short*>(up)[i]);
  }
}

constexpr int kNormThreads = 256;

// RMSNorm of one row per CTA (PrefillRMSNorm, :757-771): var = mean(x^2) in
// fp32, h = fp16(x * rsqrt(var + eps)), out = fp16(weight * h). The fp32 sum's
// order differs from torch's reduction, so var can differ in its last bits.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const __half* x, const __half* w, __half* out,
                                                               int cols, float eps, int vec) {
  __shared__ float red[kNormThreads / 32];
  const __half* xr = x + static_cast<int64_t>(blockIdx.x) * cols;
  __half* orow = out + static_cast<int64_t>(blockIdx.x) * cols;
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(xr);
  float acc = 0.f;
  if (vec) {
    for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
      const unsigned short* vs = reinterpret_cast<const unsigned short*>(&v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = h2f(vs[e]);
        acc = __fadd_rn(acc, __fmul_rn(f, f));
      }
    }
  } else {
    for (int c = threadIdx.x; c < cols; c += kNormThreads) {
      const float f = h2f(xs[c]);
      acc = __fadd_rn(acc, __fmul_rn(f, f));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) sum += red[i];
  // The reference's squared mean adds unfused x*x terms (its extension builds
  // with --fmad=false) and scales the sum by the fp32 factor 1/cols.
  const float r = rsqrtf(__fmul_rn(sum, __frcp_rn(static_cast<float>(cols))) + eps);
  const unsigned short* ws = reinterpret_cast<const unsigned short*>(w);
  unsigned short* os = reinterpret_cast<unsigned short*>(orow);
  if (vec) {
    for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + c));
      const unsigned short* vs = reinterpret_cast<const unsigned short*>(&v);
      const unsigned short* wvs = reinterpret_cast<const unsigned short*>(&wv);
      uint4 o;
      unsigned short* ov = reinterpret_cast<unsigned short*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) ov[e] = f2h(h2f(wvs[e]) * h2f(f2h(h2f(vs[e]) * r)));
      *reinterpret_cast<uint4*>(orow + c) = o;
    }
  } else {
    for (int c = threadIdx.x; c < cols; c += kNormThreads) os[c] = f2h(h2f(ws[c]) * h2f(f2h(h2f(xs[c]) * r)));
  }
}

bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace prefill
}  // namespace tilemix

using namespace tilemix::prefill;

extern "C" int tm_rotary_token_major(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k,
                                     int64_t k_sb, int64_t k_sh, int64_t k_st, const void* cos, int64_t cos_sb,
                                     int64_t cos_st, const void* sin, int64_t sin_sb, int64_t sin_st, int batch,
                                     int heads_q, int heads_k, int seq_len, int head_dim, void* oq, void* ok,
                                     int8_t* k8, void* k_scale_f16, float* k_scale_f32, int blkk, int numerics,
                                     void* stream) {
  if (!q || !k || !cos || !sin || !oq || !ok) return TM_ERR_NULL;
  if (batch < 0 || heads_q <= 0 || heads_k <= 0 || seq_len < 0) return TM_ERR_SHAPE;
  if (head_dim != 64 && head_dim != 128) return TM_ERR_UNSUPPORTED;
  if (batch == 0 || seq_len == 0) return TM_OK;
  if (batch > 65535 || heads_k > 65535) return TM_ERR_SHAPE;
  // 16-byte rows everywhere (each thread moves 8-element chunks).
  const void* ptrs[] = {q, k, cos, sin, oq, ok};
  for (const void* p : ptrs)
    if (!aligned16p(p)) return TM_ERR_ALIGN;
  const int64_t strides[] = {q_sb, q_sh, q_st, k_sb, k_sh, k_st, cos_sb, cos_st, sin_sb, sin_st};
  for (int64_t s : strides)
    if (s % 8 != 0) return TM_ERR_ALIGN;
  if (k8 && blkk != 64 && blkk != 128) return TM_ERR_UNSUPPORTED;
  if (numerics != TM_NUMERICS_GPU && numerics != TM_NUMERICS_EXACT) return TM_ERR_SHAPE;
  if (k8 && !aligned16p(k8)) return TM_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RopeArgs qa{static_cast<const __half*>(q), q_sb, q_sh, q_st, static_cast<const __half*>(cos),
              static_cast<const __half*>(sin), cos_sb, cos_st, sin_sb, sin_st, static_cast<__half*>(oq),
              batch, heads_q, seq_len, head_dim};
  const int64_t nq = static_cast<int64_t>(batch) * seq_len * heads_q * (head_dim / 16);
  rope_kernel<<<static_cast<unsigned>((nq + 255) / 256), 256, 0, st>>>(qa);
  RopeArgs ka = qa;
  ka.src = static_cast<const __half*>(k);
  ka.sb = k_sb;
  ka.sh = k_sh;
  ka.st = k_st;
  ka.dst = static_cast<__half*>(ok);
  ka.H = heads_k;
  if (!k8) {
    const int64_t nk = static_cast<int64_t>(batch) * seq_len * heads_k * (head_dim / 16);
    rope_kernel<<<static_cast<unsigned>((nk + 255) / 256), 256, 0, st>>>(ka);
  } else {
    RopeQuantArgs qq{ka, k8, static_cast<__half*>(k_scale_f16), k_scale_f32, blkk};
    const dim3 grid((seq_len + blkk - 1) / blkk, heads_k, batch);
    using tilemix::kNumericsExact;
    using tilemix::kNumericsGpu;
    const bool gpu = numerics == TM_NUMERICS_GPU;
    if (head_dim == 128 && blkk == 64)
      gpu ? rope_quant_kernel<kNumericsGpu, 128, 64><<<grid, kQuantThreads, 0, st>>>(qq)
          : rope_quant_kernel<kNumericsExact, 128, 64><<<grid, kQuantThreads, 0, st>>>(qq);
    else if (head_dim == 128)
      gpu ? rope_quant_kernel<kNumericsGpu, 128, 128><<<grid, kQuantThreads, 0, st>>>(qq)
          : rope_quant_kernel<kNumericsExact, 128, 128><<<grid, kQuantThreads, 0, st>>>(qq);
    else if (blkk == 64)
      gpu ? rope_quant_kernel<kNumericsGpu, 64, 64><<<grid, kQuantThreads, 0, st>>>(qq)
          : rope_quant_kernel<kNumericsExact, 64, 64><<<grid, kQuantThreads, 0, st>>>(qq);
    else
      gpu ? rope_quant_kernel<kNumericsGpu, 64, 128><<<grid, kQuantThreads, 0, st>>>(qq)
          : rope_quant_kernel<kNumericsExact, 64, 128><<<grid, kQuantThreads, 0, st>>>(qq);
  }
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

extern "C" int tm_silu_mul(const void* gate, const void* up, void* out, int64_t n, void* stream) {
  if (!gate || !up || !out) return TM_ERR_NULL;
  if (n < 0) return TM_ERR_SHAPE;
  if (n == 0) return TM_OK;
  const int vec = (n % 8 == 0 && aligned16p(gate) && aligned16p(up) && aligned16p(out)) ? 1 : 0;
  const int64_t threads = vec ? n / 8 : n;
  silu_mul_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(gate), static_cast<const __half*>(up), static_cast<__half*>(out), n, vec);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

extern "C" int tm_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int cols, float eps,
                           void* stream) {
  if (!x || !weight || !out) return TM_ERR_NULL;
  if (rows < 0 || cols <= 0) return TM_ERR_SHAPE;
  if (rows == 0) return TM_OK;
  if (rows > 0x7FFFFFFF) return TM_ERR_SHAPE;
  const int vec = (cols % 8 == 0 && aligned16p(x) && aligned16p(weight) && aligned16p(out)) ? 1 : 0;
  rms_norm_kernel<<<static_cast<unsigned>(rows), kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), static_cast<const __half*>(weight), static_cast<__half*>(out), cols, eps, vec);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}
