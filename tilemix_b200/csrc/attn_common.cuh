// Pieces shared by the two attention kernels (general and paired).
//
// The per-tile softmax below is the reference's _softmax_prefix_update
// (attention/triton/tilemix.py:179-207) applied to one 64-key score tile held
// in tensor memory, for the one query row owned by the calling thread:
//   qk   = fp16(S)                                (FP16 route, fp32 accumulated S)
//        = fp16(f32(S_i32) * score_scale)         (INT8 route, :401-404)
//   keys at or beyond `lim` are masked to -inf    (causal / length, :256-262)
//   p    = fp16(exp2(f32(qk) - m))                (:195-199)
//   l   += sum exp2(f32(qk) - m)                 (:200, :206; summed before the
//          fp16 rounding of p, a difference below fp16 resolution)
// where m is the row's reference maximum. With threshold 0 it is updated on
// every increase (the reference's rule); with threshold t > 0 it only moves
// when the tile max exceeds it by more than t (log2 units), which bounds
// p by 2^t and makes rescaling of the output accumulator rare.
#pragma once

#include "common.cuh"

namespace tilemix {

constexpr int kKeys = 64;  // keys per hardware score tile

struct AttnArgs {
  const __half* q;
  int64_t q_st, q_sh;
  __half* out;
  int64_t o_st, o_sh;
  const int8_t* q8;
  int64_t q8_st, q8_sh;
  const __half* q_scale;
  const int32_t* cu_qs;
  const __half* k_scale;
  const int32_t* cu_ks;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const uint64_t* bitmask;
  int HQ, HK, group, D;
  int block_m, block_n_mask, blkq, blkk;
  int causal, mode, fuse_q;
  int o_vec32;     // O rows start on 32-byte boundaries (out 32-byte aligned, strides multiples of 16)
  float qk_scale;
  float rescale_threshold;
  int* err;
  // INT8-V PV path (int8_use_fp16_v == 0, general kernel): fp16 V block scales.
  int v8_path;
  const __half* v_scale;
  const int32_t* cu_vs;
  // Additive fp16 bias [., HQ, Tq, Tk] (general kernel); no batch offset, as
  // the reference indexes it (tilemix.py:264-270).
  const __half* bias;
  int64_t b_sh, b_sm, b_sn;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  tmem_st16(taddr, r);
  tmem_st16(taddr + 16, r + 16);
}

// Exact int32 -> fp32 for |x| < 2^22 without the conversion pipe: the bit
// pattern of 1.5*2^23 plus x is the float 1.5*2^23 + x; subtracting 1.5*2^23
// is exact. INT8 scores are bounded by 128 * 127 * 127 < 2^21.
__device__ __forceinline__ float i2f_exact(uint32_t x) { return __uint_as_float(x + 0x4B400000u) - 12582912.0f; }

__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float2 f32x2_unpack(uint64_t v) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(v)), __uint_as_float(static_cast<uint32_t>(v >> 32)));
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ uint64_t f32x2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_add_rm(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// f32(lo or hi half of an fp16 pair) + c, one rounding, on the FMA pipe.
__device__ __forceinline__ float add_f32_f16_lo(uint32_t h2, float c) {
  float r;
  asm("{.reg .f16 l, h;\n\tmov.b32 {l, h}, %1;\n\tadd.rn.f32.f16 %0, l, %2;\n\t}" : "=f"(r) : "r"(h2), "f"(c));
  return r;
}
__device__ __forceinline__ float add_f32_f16_hi(uint32_t h2, float c) {
  float r;
  asm("{.reg .f16 l, h;\n\tmov.b32 {l, h}, %1;\n\tadd.rn.f32.f16 %0, h, %2;\n\t}" : "=f"(r) : "r"(h2), "f"(c));
  return r;
}
__device__ __forceinline__ uint32_t hmax2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// 2^x for a pair of x in [-126, 16) without the MUFU pipe: x = j + f with
// j = floor(x) (an add rounded toward -inf against 1.5 * 2^23 leaves j in the
// low mantissa bits), 2^f on [0, 1) by a degree-5 polynomial in Horner form
// (relative-error minimax fit by the Remez exchange: max relative error
// 1.5e-7 evaluated in fp32, the accuracy class of ex2.approx), and 2^j added to
// the exponent field as an integer. Spreads part of the softmax exponentials
// over the FMA pipe: the MUFU pipe (16 results per clock per SM) is the
// softmax's throughput limit otherwise.
__device__ __forceinline__ void exp2_poly_x2(float x0, float x1, float& e0, float& e1) {
  const uint64_t kMagic = 0x4B4000004B400000ull;  // (1.5 * 2^23, 1.5 * 2^23)
  const uint64_t x = f32x2_pack(x0, x1);
  const uint64_t t = f32x2_add_rm(x, kMagic);    // 1.5 * 2^23 + floor(x), exact
  const uint64_t f = f32x2_add(x, f32x2_sub(kMagic, t));  // x - floor(x) in [0, 1), exact
  uint64_t p = f32x2_fma(0x3AF619053AF61905ull, f, 0x3C1348063C134806ull);
  p = f32x2_fma(p, f, 0x3D64AA233D64AA23ull);
  p = f32x2_fma(p, f, 0x3E75EAD43E75EAD4ull);
  p = f32x2_fma(p, f, 0x3F31727B3F31727Bull);
  p = f32x2_fma(p, f, 0x3F7FFFFF3F7FFFFFull);
  // (1.5 * 2^23 + j) << 23 == j << 23 modulo 2^32.
  e0 = __uint_as_float(static_cast<uint32_t>(p) + (static_cast<uint32_t>(t) << 23));
  e1 = __uint_as_float(static_cast<uint32_t>(p >> 32) + (static_cast<uint32_t>(t >> 32) << 23));
}

// Pairs of a 64-key tile whose exponentials run on the FMA pipe (4 of 32;
// larger shares measured slower: the polynomial costs more issue slots than
// the MUFU pipe it relieves).
__device__ __forceinline__ constexpr bool exp_on_fma(int pair) { return (pair & 7) == 7; }

// One softmax step over a 64-key tile for this thread's row.
//   taddr     TMEM address (lane and first column) of the 64 score columns
//   kind      0: fp32 scores (FP16 route)   1: int32 scores (INT8 route)
//   ss        fp32 value of the fp16 score scale (INT8 route)
//   lim       number of valid keys of this row in the tile (>= 64: none masked)
//   thr       rescale threshold (0 = reference rule)
// Outputs the packed fp16 P row in p[32]; o_scale/need_rescale say whether the
// O accumulator row has to be multiplied by o_scale before this P is added.
// The row maximum is taken over the fp32 values before their fp16 rounding:
// rounding to nearest is monotonic, so fp16(max v) = max fp16(v).
//   brow      optional additive bias of this row and tile (element i at
//             brow[i * bstride]): qk = fp16(qk + fp16(b * fp16(log2 e))) on the
//             valid keys (tilemix.py:264-272, :413-421)
__device__ __forceinline__ void softmax_tile(uint32_t taddr, int kind, float ss, int lim, float thr,
                                             float& m_used, float& l, uint32_t (&p)[32], float& o_scale,
                                             bool& need_rescale, const __half* brow = nullptr,
                                             int64_t bstride = 0) {
  uint32_t s[64];
  tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
  tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
  tmem_wait_ld();
  if (kind != 0) {
    // f32(i) * ss in one rounding: with a = float(i + 0x4B400000) = 1.5*2^23 + i,
    // fma(a, ss, -1.5*2^23*ss) evaluates a*ss - 1.5*2^23*ss = i*ss exactly before
    // its single rounding (-1.5*2^23*ss is exact: ss has an 11-bit significand).
    const float c = -12582912.0f * ss;
    const uint64_t ss2 = f32x2_pack(ss, ss), c2 = f32x2_pack(c, c);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint64_t a2 = f32x2_pack(__uint_as_float(s[2 * i] + 0x4B400000u), __uint_as_float(s[2 * i + 1] + 0x4B400000u));
      const float2 v = f32x2_unpack(f32x2_fma(a2, ss2, c2));
      s[2 * i] = __float_as_uint(v.x);
      s[2 * i + 1] = __float_as_uint(v.y);
    }
  }
  const float kNegInf = -__int_as_float(0x7f800000);
  if (__any_sync(0xffffffffu, lim < kKeys)) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (i >= lim) s[i] = 0xFF800000u;  // -inf
  }
  if (brow != nullptr) {
    // fp16 products and sums, each rounded once: fp32 holds the exact product
    // of two fp16 values, and a sum of two fp16 values rounded to fp32 and then
    // to fp16 is the correctly rounded fp16 sum (24 >= 2 * 11 + 2 bits).
    const float l2e = __half2float(__float2half_rn(1.4426950408889634f));
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      if (i < lim) {
        const float b = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(brow) + i * bstride)));
        const float bb = __half2float(__float2half_rn(b * l2e));
        const float q16 = __half2float(__float2half_rn(__uint_as_float(s[i])));
        s[i] = __float_as_uint(__half2float(__float2half_rn(q16 + bb)));
      }
    }
  }
  // Row maximum: a tree of 3-input maxima (64 -> 22 -> 8 -> 4 -> 2 -> 1).
  float m1[22];
#pragma unroll
  for (int i = 0; i < 21; ++i)
    m1[i] = max3f(__uint_as_float(s[3 * i]), __uint_as_float(s[3 * i + 1]), __uint_as_float(s[3 * i + 2]));
  m1[21] = __uint_as_float(s[63]);
  float m2[8];
#pragma unroll
  for (int i = 0; i < 7; ++i) m2[i] = max3f(m1[3 * i], m1[3 * i + 1], m1[3 * i + 2]);
  m2[7] = m1[21];
  const float m3a = max3f(m2[0], m2[1], m2[2]), m3b = max3f(m2[3], m2[4], m2[5]);
  const float mraw = max3f(m3a, m3b, fmaxf(m2[6], m2[7]));
  const float mx = __half2float(__float2half_rn(mraw));
  const bool has = mx != kNegInf;
  o_scale = 1.f;
  need_rescale = false;
  if (has && mx > m_used + thr) {
    const float alpha = ex2_approx(m_used - mx);  // 0 when m_used == -inf
    need_rescale = (m_used != kNegInf);
    o_scale = alpha;
    l *= alpha;
    m_used = mx;
  }
  if (has) {
    // l accumulates the exponentials before their fp16 rounding (two packed
    // partial sums); the rounding of p stays exactly the reference's.
    const float negm = -m_used;
    // Lower clamp for the FMA-pipe pairs: x >= floor16(m_used - 120) - m_used
    // keeps floor(x) >= -126; every clamped weight is below 2^-120, which is 0
    // in fp16 and below the resolution of l.
    uint32_t lo2;
    {
      const float lo = fmaxf(m_used - 120.f, -65504.f);
      uint16_t lh;
      asm("cvt.rp.f16.f32 %0, %1;" : "=h"(lh) : "f"(lo));
      lo2 = static_cast<uint32_t>(lh) * 0x10001u;
    }
    uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      uint32_t h2 = pack_half2_rn(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]));
      float e0, e1;
      if (exp_on_fma(i)) {
        h2 = hmax2_u32(h2, lo2);
        exp2_poly_x2(add_f32_f16_lo(h2, negm), add_f32_f16_hi(h2, negm), e0, e1);
      } else {
        e0 = ex2_approx(add_f32_f16_lo(h2, negm));
        e1 = ex2_approx(add_f32_f16_hi(h2, negm));
      }
      if (i & 1)
        acc1 = f32x2_add(acc1, f32x2_pack(e0, e1));
      else
        acc0 = f32x2_add(acc0, f32x2_pack(e0, e1));
      p[i] = pack_half2_rn(e0, e1);
    }
    const float2 a0 = f32x2_unpack(acc0), a1 = f32x2_unpack(acc1);
    l += (a0.x + a0.y) + (a1.x + a1.y);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) p[i] = 0u;
  }
}

// Rescale this thread's row of an fp32 O accumulator (D columns) in TMEM, 64
// columns per load / wait round trip (the round trips, not the multiplies, set
// its duration).
template <int D>
__device__ __forceinline__ void rescale_o_row(uint32_t taddr, float scale) {
  const uint64_t s2 = f32x2_pack(scale, scale);
#pragma unroll 1
  for (int c = 0; c < D; c += 64) {
    uint32_t o[64];
    tmem_ld32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
    tmem_ld32(taddr + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      uint64_t v;
      asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(v) : "l"(f32x2_pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]))), "l"(s2));
      o[2 * i] = static_cast<uint32_t>(v);
      o[2 * i + 1] = static_cast<uint32_t>(v >> 32);
    }
    tmem_st32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
    tmem_st32(taddr + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
  }
}

// Normalise this thread's O row (D fp32 columns in TMEM) by l and store it as fp16.
template <int D>
__device__ __forceinline__ void store_o_row(uint32_t taddr, bool have_o, float l, __half* orow, bool store) {
#pragma unroll 1
  for (int c = 0; c < D; c += 32) {
    uint32_t o[32];
    if (have_o) {
      tmem_ld32(taddr + c, o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0u;
    }
    if (store) {
      // acc / l: reciprocal once per row, then per element one residual
      // correction (Markstein's method: q0 = a*r, e = a - q0*l, q = q0 + e*r),
      // which gives the correctly rounded quotient for these normal operands.
      const float rl = __frcp_rn(l);
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float a0 = __uint_as_float(o[2 * i]), a1 = __uint_as_float(o[2 * i + 1]);
        const float q0 = a0 * rl, q1 = a1 * rl;
        w[i] = pack_half2_rn(fmaf(fmaf(-q0, l, a0), rl, q0), fmaf(fmaf(-q1, l, a1), rl, q1));
      }
      uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
      for (int v = 0; v < 4; ++v) dst[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
    }
  }
}

// Route of 64-key tile j of one map row (mode overrides the bitmask).
__device__ __forceinline__ int route_kind(int mode, uint64_t bits, int j, int block_n_mask) {
  if (mode == 1) return 0;  // TM_ROUTE_FP16
  if (mode == 2) return 1;  // TM_ROUTE_INT8
  return static_cast<int>((bits >> ((j * kKeys) / block_n_mask)) & 1ull);
}

// Route of the consecutive 64-key tiles j = 0, 1, 2, ... of one query tile,
// the same as route_kind(mode, bits, j, block_n_mask) but with the mask group
// index j / (block_n_mask / 64) tracked incrementally instead of divided out
// per tile. Call kind() for tile j, then advance() to move to tile j + 1.
struct RouteWalker {
  uint64_t bits;
  int mode, per, grp, sub;
  __device__ __forceinline__ void init(int mode_, uint64_t bits_, int block_n_mask) {
    mode = mode_;
    bits = bits_;
    per = block_n_mask / kKeys;
    grp = 0;
    sub = 0;
  }
  __device__ __forceinline__ int kind() const {
    if (mode == 1) return 0;  // TM_ROUTE_FP16
    if (mode == 2) return 1;  // TM_ROUTE_INT8
    return grp < 64 ? static_cast<int>((bits >> grp) & 1ull) : 0;
  }
  __device__ __forceinline__ void advance() {
    if (++sub == per) {
      sub = 0;
      ++grp;
    }
  }
};

// Number of 64-key tiles the reference visits for the query rows
// [row0, row0 + rows) of a sequence (tilemix.py:603-612), in 64-key units.
__device__ __forceinline__ int visited_key_tiles(int row0, int rows, int seqlen_q, int seqlen_k, int causal) {
  int lim = seqlen_k;
  if (causal) lim = min(seqlen_k, row0 + rows + seqlen_k - seqlen_q);
  return lim <= 0 ? 0 : (lim + kKeys - 1) / kKeys;
}

// fp32 value of the fp16 INT8 score scale fp16(f32(fp16(sq * sk)) * qk_scale) (:380-399).
__device__ __forceinline__ float int8_score_scale(__half sq, __half sk, float qk_scale) {
  return __half2float(__float2half_rn(__half2float(__hmul(sq, sk)) * qk_scale));
}

}  // namespace tilemix
