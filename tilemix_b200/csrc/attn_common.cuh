// Pieces shared by the two attention kernels (general and paired).
//
// The per-tile softmax below is the reference's _softmax_prefix_update
// (attention/triton/tilemix.py:179-207) applied to one 64-key score tile held
// in tensor memory, for the one query row owned by the calling thread:
//   qk   = fp16(S)                                (FP16 route, :254)
//        = fp16(f32(S_i32) * score_scale)         (INT8 route, :401-404)
//   keys at or beyond `lim` are masked to -inf    (causal / length, :256-262)
//   p    = fp16(exp2(f32(qk) - m))                (:195-199)
//   l    = l * alpha + sum f32(p)                 (:200, :206)
// where m is the row's reference maximum. With threshold 0 it is updated on
// every increase (the reference's rule); with threshold t > 0 it only moves
// when the tile max exceeds it by more than t (log2 units), which bounds
// p by 2^t and makes rescaling of the output accumulator rare.
// FP16-route scores arrive in TMEM as the MMA accumulated them: fp16 (one
// value in the low half of each 32-bit column) in GPU numerics, where the
// reference's tl.dot(..., out_dtype=fp16) accumulates in fp16 on the tensor
// core, or fp32 rounded once in exact numerics (common.cuh).
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
  int numerics;    // kNumericsGpu or kNumericsExact (common.cuh)
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

__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
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

// One softmax step over a 64-key tile for this thread's row.
//   taddr     TMEM address (lane and first column) of the 64 score columns
//   kind      0: FP16 route (fp16 or fp32 scores, by kNumerics)   1: INT8 route (int32 scores)
//   ss        fp32 value of the fp16 score scale (INT8 route)
//   lim       number of valid keys of this row in the tile (>= 64: none masked)
//   thr       rescale threshold (0 = reference rule)
// Outputs the packed fp16 P row in p[32]; o_scale/need_rescale say whether the
// O accumulator row has to be multiplied by o_scale before this P is added.
// The scores are rounded to fp16 first (the reference's qk is an fp16 tile)
// and the row maximum is taken over the fp16 pairs. Every exponential runs on
// ex2.approx, as tl.math.exp2 does on the GPU.
//   brow      optional additive bias of this row and tile (element i at
//             brow[i * bstride]): qk = fp16(qk + fp16(b * fp16(log2 e))) on the
//             valid keys (tilemix.py:264-272, :413-421)
template <int kNumerics>
__device__ __forceinline__ void softmax_tile(uint32_t taddr, int kind, float ss, int lim, float thr,
                                             float& m_used, float& l, uint32_t (&p)[32], float& o_scale,
                                             bool& need_rescale, const __half* brow = nullptr,
                                             int64_t bstride = 0) {
  // qk of the row as fp16 pairs: h[i] = (qk[2i], qk[2i+1]).
  uint32_t h[32];
  if (kNumerics == kNumericsGpu && kind == 0) {
    // fp16 accumulator: the load packs the columns' 16-bit values in pairs.
    tmem_ld64_pack16(taddr, h);
    tmem_wait_ld();
  } else {
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
#pragma unroll
    for (int i = 0; i < 32; ++i) h[i] = pack_half2_rn(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]));
  }
  if (__any_sync(0xffffffffu, lim < kKeys)) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (2 * i >= lim)
        h[i] = 0xFC00FC00u;  // (-inf, -inf)
      else if (2 * i + 1 >= lim)
        h[i] = (h[i] & 0xFFFFu) | 0xFC000000u;
    }
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
        const uint32_t hw = h[i >> 1];
        const float q16 = __half2float(__ushort_as_half(static_cast<unsigned short>((i & 1) ? hw >> 16 : hw & 0xFFFFu)));
        const uint32_t r = __half_as_ushort(__float2half_rn(q16 + bb));
        h[i >> 1] = (i & 1) ? ((hw & 0xFFFFu) | (r << 16)) : ((hw & 0xFFFF0000u) | r);
      }
    }
  }
  // Row maximum over the fp16 pairs (a tree of packed maxima), then of the two halves.
  uint32_t m16[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m16[i] = hmax2_u32(h[2 * i], h[2 * i + 1]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) m16[i] = hmax2_u32(m16[i], m16[i + w]);
  }
  const uint32_t mm = hmax2_u32(m16[0], __byte_perm(m16[0], 0u, 0x1032));
  const float kNegInf = -__int_as_float(0x7f800000);
  const float mx = __half2float(__ushort_as_half(static_cast<unsigned short>(mm & 0xFFFFu)));
  const bool has = mx != kNegInf;
  o_scale = 1.f;
  need_rescale = false;
  if (has && mx > m_used + thr) {
    const float alpha = ex2_approx(m_used - mx);  // 0 when m_used == -inf
    need_rescale = (m_used != kNegInf);
    o_scale = alpha;
    m_used = mx;
  }
  if (has) {
    // p = fp16(exp2(f32(qk) - m)), qk - m by the mixed-precision add (one
    // rounding, as fp16 - fp32 promotes to fp32); l sums the rounded p in fp32.
    const float negm = -m_used;
    float la = 0.f, lb = 0.f, lc = 0.f, ld = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float e0 = ex2_approx(add_f32_f16_lo(h[i], negm));
      const float e1 = ex2_approx(add_f32_f16_hi(h[i], negm));
      p[i] = pack_half2_rn(e0, e1);
      if (i & 1) {
        lc = add_f32_f16_lo(p[i], lc);
        ld = add_f32_f16_hi(p[i], ld);
      } else {
        la = add_f32_f16_lo(p[i], la);
        lb = add_f32_f16_hi(p[i], lb);
      }
    }
    // l = l * alpha + l_tile: one FMA on the GPU (the reference's compiler
    // contracts it), a rounded product and a rounded sum in exact numerics.
    const float lt = (la + lb) + (lc + ld);
    l = kNumerics == kNumericsGpu ? fmaf(l, o_scale, lt) : __fadd_rn(__fmul_rn(l, o_scale), lt);
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

// Normalise this thread's O row (D fp32 columns in TMEM) by l and store it as
// fp16 (the division of the numerics, common.cuh normalize_pair).
template <int kNumerics, int D>
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
      const float rl = __frcp_rn(l);
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        w[i] = normalize_pair<kNumerics>(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]), l, rl);
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
