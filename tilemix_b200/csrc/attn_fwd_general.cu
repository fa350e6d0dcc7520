// Fused FP16/INT8 tile-routed flash-attention forward for B200 (sm_100a).
//
// Semantics follow attn_fwd in attention/triton/tilemix.py:503-951:
//   * program -> (query tile, Q head, sequence); KV head = hq / (HQ/HK) (:585-592)
//   * per-sequence lengths from cu_seqlens (:594-601), causal tile bound (:603-612)
//   * q_fp16 = fp16(q * sm_scale*log2e) (:641-649); q8 / per-block Q scale (:651-695)
//   * each key tile is routed by bit (key_start / block_n_mask) of the row word
//     pm[hk * m_blocks + start_m] (:818-933): FP16 QK^T (:210-300) or INT8 QK^T
//     with qk = fp16(f32(i32) * f32(fp16(fp16(sq*sk) * qk_scale))) (:303-404)
//   * shared online softmax, p = fp16(exp2(f32(qk) - m)) (:179-207); PV with
//     FP16 P and V, FP32 accumulation (:284-299, :432-448); out = acc / l (:935-951)
//
// B200 mapping (one CTA = 128 query rows of one head; TMEM lane r = row r):
//   warp 4     TMA producer: K (fp16 and/or int8, only the routed formats) and V
//              tiles of 64 keys into a 3-stage shared-memory ring.
//   warp 5     MMA issuer (one thread): S = Q K^T as tcgen05.mma with Q as the
//              TMEM operand (kind::f16 -> fp32 S, or kind::i8 -> int32 S), and
//              O += P V with P as the TMEM operand (kind::f16, fp32 O in TMEM).
//   warps 0-3  softmax: load Q once (scaled fp16 and int8 codes, quantised in
//              kernel when no prequantised Q is given), then per key tile read S
//              from TMEM, apply the reference rounding chain, write P (fp16) back
//              into TMEM over S, and finally normalise O and store it.
// S/P live in three 64-column TMEM slots so that QK^T of tile j+1 and PV of
// tile j-1 run on the tensor core while the softmax works on tile j.
//
// INT8-V PV path (int8_use_fp16_v == 0, tilemix.py:449-497): an INT8-routed
// tile's PV is fp16(p * sv) x fp16(v8) with sv the V block scale. The producer
// also loads the tile's int8 V; the softmax warps, which see the stage landed
// once its S is complete, write the exact fp16 copy of it into a second fp16
// V buffer of the stage before they publish P. When the two 64-row halves of
// a block_m 64 tile take different routes, P of the FP16 half goes to the
// slot's first 32 columns and P of the INT8 half to the next 32, and the MMA
// warp issues one PV against V and one against the converted V8.
// Additive bias (tilemix.py:264-272): added to the fp16 scores of the valid
// keys before the row maximum, indexed without a batch offset as the
// reference does.
//
// Rescaling of O: with rescale_threshold == 0 the running max is updated on
// every increase exactly as in the reference. With a positive threshold t
// (log2 units) the reference max is only moved when the tile max exceeds it by
// more than t, so P may reach 2^t (fp16-safe for t <= 15) and O is rescaled in
// TMEM only on those rare jumps; the result is the same softmax up to fp16
// rounding of P.
#include "attn_common.cuh"
#include "tilemix_b200.h"

namespace tilemix {
namespace general {

constexpr int kRows = 128;
constexpr int kStages = 3;
constexpr int kSlots = 3;
constexpr int kThreads = 192;

// TMEM columns (32-bit) of the 512 allocated per CTA.
constexpr uint32_t kColO = 0;      // O accumulator, head_dim columns (<=128)
constexpr uint32_t kColS = 128;    // 3 slots x 64 columns (S fp32/int32, then P fp16 in the first 32)
constexpr uint32_t kColX = 320;    // second-format S of a split-route tile (block_m == 64 only)
constexpr uint32_t kColQ16 = 384;  // scaled fp16 Q, head_dim/2 columns
constexpr uint32_t kColQ8 = 448;   // int8 Q codes, head_dim/4 columns
constexpr uint32_t kTmemCols = 512;

// Shared memory (offsets from a 1024-byte aligned base).
constexpr uint32_t kK16Bytes = 64 * 128 * 2;  // one stage of fp16 K (head_dim <= 128)
constexpr uint32_t kK8Bytes = 64 * 128;       // one stage of int8 K
constexpr uint32_t kVBytes = 64 * 128 * 2;    // one stage of fp16 V
constexpr uint32_t kV8Bytes = 64 * 128;       // one stage of int8 V (INT8-V path)
constexpr uint32_t kV8FBytes = 64 * 128 * 2;  // its fp16 copy, in the layout of a V stage
constexpr uint32_t kOffK16 = 0;
constexpr uint32_t kOffV = kOffK16 + kStages * kK16Bytes;
constexpr uint32_t kOffK8 = kOffV + kStages * kVBytes;
constexpr uint32_t kOffV8 = kOffK8 + kStages * kK8Bytes;
constexpr uint32_t kOffV8F = kOffV8 + kStages * kV8Bytes;
constexpr uint32_t kOffBar = kOffV8F + kStages * kV8FBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // barriers + alignment slack


struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t s_full[kSlots];
  uint64_t p_ready[kSlots];
  uint64_t pv_done[kSlots];
  uint64_t q_ready;
  uint64_t mma_done;
  uint32_t tmem_base;
  float red[4];
};

// Per-CTA routing context, identical in every thread.
struct Route {
  uint64_t bits[2];  // map row word per 64-row half (or the single 128-row word)
  int nb[2];         // number of 64-key tiles each half processes
  int halves;        // 1 (block_m 128) or 2 (block_m 64)
  int mode;
  int bnm_shift_div;  // block_n_mask (keys per routing bit)

  __device__ __forceinline__ int kind(int h, int j) const { return route_kind(mode, bits[h], j, bnm_shift_div); }
  __device__ __forceinline__ void needs(int j, bool& n16, bool& n8) const {
    n16 = false;
    n8 = false;
    for (int h = 0; h < halves; ++h) {
      if (j < nb[h]) {
        if (kind(h, j))
          n8 = true;
        else
          n16 = true;
      }
    }
  }
};

__device__ __forceinline__ void named_bar_sync_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Four int8 in a word -> two fp16 pairs, exactly: the byte b + 128 placed in
// the mantissa of 1024.0 gives the fp16 value 1024 + (b + 128); subtracting
// 1152 leaves b.
__device__ __forceinline__ void int8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152.0
  uint32_t a = __byte_perm(x, 0x64646464u, 0x5140), b = __byte_perm(x, 0x64646464u, 0x7362);
  const __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), off);
  const __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), off);
  lo = *reinterpret_cast<const uint32_t*>(&ha);
  hi = *reinterpret_cast<const uint32_t*>(&hb);
}

// The int8 V tile of ring stage s (TMA layout: D bytes per key row, 128- or
// 64-byte swizzle) -> its fp16 copy in the layout of a V stage (64-dim boxes
// of 128-byte rows, 128-byte swizzle). Called by the 128 softmax threads.
template <int D>
__device__ __forceinline__ void convert_v8_stage(uint8_t* smem, int s, int t) {
  const uint8_t* src = smem + kOffV8 + s * kV8Bytes;
  uint8_t* dst = smem + kOffV8F + s * kV8FBytes;
  constexpr int kChunks = D / 16;  // 16-byte int8 chunks per key row
#pragma unroll
  for (int u = t; u < 64 * kChunks; u += 128) {
    const int r = u / kChunks, c = u % kChunks;
    const int pos = (D == 128) ? (c ^ (r & 7)) : (c ^ ((r >> 1) & 3));
    const uint4 w = *reinterpret_cast<const uint4*>(src + r * D + (pos << 4));
    uint32_t h[8];
    int8x4_to_f16x4(w.x, h[0], h[1]);
    int8x4_to_f16x4(w.y, h[2], h[3]);
    int8x4_to_f16x4(w.z, h[4], h[5]);
    int8x4_to_f16x4(w.w, h[6], h[7]);
    // dims 16c .. 16c+15 = 8-dim fp16 chunks cb, cb+1 of 64-dim box (16c)/64
    const int box = (16 * c) / 64, cb = ((16 * c) % 64) / 8;
    uint8_t* row = dst + box * (64 * 64 * 2) + r * 128;
    *reinterpret_cast<uint4*>(row + ((cb ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(row + (((cb + 1) ^ (r & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
  }
}

template <int kNumerics, int D>
__global__ void __launch_bounds__(kThreads, 1)
    tilemix_attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_k16, const __grid_constant__ CUtensorMap tm_k8,
                            const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_v8,
                            const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kOffBar);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
  const int hq = blockIdx.y;
  const int b = blockIdx.z;

  const int q_start = a.cu_q[b];
  const int seqlen_q = a.cu_q[b + 1] - q_start;
  if (tile * kRows >= seqlen_q) return;  // uniform: before any barrier or allocation
  const int k_start = a.cu_k[b];
  const int seqlen_k = a.cu_k[b + 1] - k_start;
  const int hk = hq / a.group;
  const int coff = seqlen_k - seqlen_q;

  Route rt;
  rt.halves = kRows / a.block_m;
  rt.mode = a.mode;
  rt.bnm_shift_div = a.block_n_mask;
  const int m_blocks = (seqlen_q + a.block_m - 1) / a.block_m;
  int n_tiles = 0;
  for (int h = 0; h < 2; ++h) {
    rt.bits[h] = 0;
    rt.nb[h] = 0;
    if (h >= rt.halves) continue;
    const int mrow = tile * rt.halves + h;
    if (mrow * a.block_m >= seqlen_q) continue;
    if (a.mode == TM_ROUTE_MIXED) rt.bits[h] = a.bitmask[static_cast<int64_t>(hk) * m_blocks + mrow];
    int lim = seqlen_k;
    if (a.causal) lim = min(seqlen_k, (mrow + 1) * a.block_m + coff);
    rt.nb[h] = lim <= 0 ? 0 : (lim + kKeys - 1) / kKeys;
    n_tiles = max(n_tiles, rt.nb[h]);
  }

  const uint32_t k16_box_bytes = 64 * 64 * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_ready[s], kRows);
      mbar_init(&bars->pv_done[s], 1);
    }
    mbar_init(&bars->q_ready, kRows);
    mbar_init(&bars->mma_done, 1);
    fence_mbarrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_k16);
      prefetch_tmap(&tm_v);
      if (a.mode != TM_ROUTE_FP16) prefetch_tmap(&tm_k8);
      if (a.v8_path) prefetch_tmap(&tm_v8);
      bool ok = true;
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j % kStages;
        if (j >= kStages) ok = mbar_wait(&bars->empty[s], ((j - kStages) / kStages) & 1, a.err, kErrTimeoutEmpty);
        if (!ok) break;
        bool n16, n8;
        rt.needs(j, n16, n8);
        const bool use_v8 = a.v8_path && n8;     // INT8-routed rows take int8 V
        const bool use_v16 = !a.v8_path || n16;  // the others the fp16 V
        const uint32_t vbytes = static_cast<uint32_t>(D) * 64 * 2;
        const uint32_t bytes = (use_v16 ? vbytes : 0u) + (n16 ? vbytes : 0u) +
                               (n8 ? static_cast<uint32_t>(D) * 64 : 0u) + (use_v8 ? static_cast<uint32_t>(D) * 64 : 0u);
        mbar_arrive_expect_tx(&bars->full[s], bytes);
        const int tok = k_start + j * kKeys;
#pragma unroll
        for (int box = 0; box < D / 64; ++box) {
          if (n16) tma_load_3d(smem + kOffK16 + s * kK16Bytes + box * k16_box_bytes, &tm_k16, &bars->full[s], box * 64, hk, tok);
          if (use_v16) tma_load_3d(smem + kOffV + s * kVBytes + box * k16_box_bytes, &tm_v, &bars->full[s], box * 64, hk, tok);
        }
        if (n8) tma_load_3d(smem + kOffK8 + s * kK8Bytes, &tm_k8, &bars->full[s], 0, hk, tok);
        if (use_v8) tma_load_3d(smem + kOffV8 + s * kV8Bytes, &tm_v8, &bars->full[s], 0, hk, tok);
      }
      // Drain: every issued copy must land before the CTA exits.
      const int first = max(0, n_tiles - kStages);
      for (int j = first; j < n_tiles; ++j) {
        mbar_wait(&bars->full[j % kStages], (j / kStages) & 1, a.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // FP16 scores accumulate in fp16 (GPU numerics) or fp32 (exact numerics).
      const uint32_t idesc_qk16 = make_idesc(kNumerics == kNumericsGpu ? 0 : 1, 0, 0, 0, 128, 64);
      const uint32_t idesc_qk8 = make_idesc(2, 1, 0, 0, 128, 64);
      const uint32_t idesc_pv = make_idesc(1, 0, 0, 1, 128, static_cast<uint32_t>(D));
      const uint32_t k8_layout = (D == 128) ? 2u : 4u;
      const uint32_t k8_sbo = (D == 128) ? 1024u : 512u;
      bool ok = mbar_wait(&bars->q_ready, 0, a.err, kErrTimeoutQ);
      tc_fence_after();
      bool prev_split = false;
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j < n_tiles) {
          const int s = j % kStages;
          const int slot = j % kSlots;
          ok = mbar_wait(&bars->full[s], (j / kStages) & 1, a.err, kErrTimeoutFull);
          if (ok && j >= kSlots) ok = mbar_wait(&bars->pv_done[slot], ((j - kSlots) / kSlots) & 1, a.err, kErrTimeoutPV);
          bool n16, n8;
          rt.needs(j, n16, n8);
          const bool split = n16 && n8;
          if (ok && split && prev_split)
            ok = mbar_wait(&bars->p_ready[(j - 1) % kSlots], ((j - 1) / kSlots) & 1, a.err, kErrTimeoutP);
          if (!ok) break;
          prev_split = split;
          tc_fence_after();
          const uint32_t s_col = kColS + slot * 64;
          if (n16) {
            const uint32_t kbase = smem_u32(smem + kOffK16 + s * kK16Bytes);
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t bdesc = make_sdesc(kbase + (kk >> 2) * k16_box_bytes + (kk & 3) * 32, 16, 1024, 2);
              mma_f16_ts(tbase + s_col, tbase + kColQ16 + kk * 8, bdesc, idesc_qk16, kk > 0 ? 1u : 0u);
            }
          }
          if (n8) {
            const uint32_t dcol = split ? kColX : s_col;
            const uint32_t kbase = smem_u32(smem + kOffK8 + s * kK8Bytes);
            for (int kk = 0; kk < D / 32; ++kk) {
              const uint64_t bdesc = make_sdesc(kbase + kk * 32, 16, k8_sbo, k8_layout);
              mma_i8_ts(tbase + dcol, tbase + kColQ8 + kk * 8, bdesc, idesc_qk8, kk > 0 ? 1u : 0u);
            }
          }
          tc_commit(&bars->s_full[slot]);
        }
        if (j >= 1) {
          const int jj = j - 1;
          const int s = jj % kStages;
          const int slot = jj % kSlots;
          ok = mbar_wait(&bars->p_ready[slot], (jj / kSlots) & 1, a.err, kErrTimeoutP);
          if (!ok) break;
          tc_fence_after();
          const uint32_t p_col = kColS + slot * 64;
          bool pn16, pn8;
          rt.needs(jj, pn16, pn8);
          const bool pv8 = a.v8_path && pn8;
          // PV against V (FP16 rows, or all rows off the INT8-V path), then
          // against the converted int8 V (from P's second 32 columns when the
          // halves of the tile were routed differently).
          const int groups = (pv8 && pn16) ? 2 : 1;
          for (int g = 0; g < groups; ++g) {
            const bool use_v8f = pv8 && (g == 1 || !pn16);
            const uint32_t vbase = smem_u32(smem + (use_v8f ? kOffV8F + s * kV8FBytes : kOffV + s * kVBytes));
            const uint32_t pcol = p_col + (g == 1 ? 32u : 0u);
            for (int kk = 0; kk < kKeys / 16; ++kk) {
              const uint64_t bdesc = make_sdesc(vbase + kk * 16 * 128, k16_box_bytes, 1024, 2);
              mma_f16_ts(tbase + kColO, tbase + pcol + kk * 8, bdesc, idesc_pv, (jj > 0 || kk > 0 || g > 0) ? 1u : 0u);
            }
          }
          tc_commit(&bars->pv_done[slot]);
          tc_commit(&bars->empty[s]);
        }
      }
      // All issued tensor-core work must finish before TMEM is released.
      tc_commit(&bars->mma_done);
      mbar_wait(&bars->mma_done, 0, a.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------------ softmax warps 0-3
    const int t = threadIdx.x;  // row within the CTA tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const int row = tile * kRows + t;
    const bool row_ok = row < seqlen_q;
    const int half = t / a.block_m;  // 0 for block_m 128

    // ---- Q: scaled fp16 codes and int8 codes into TMEM
    const __half* qrow = a.q + (static_cast<int64_t>(q_start) + row) * a.q_st + static_cast<int64_t>(hq) * a.q_sh;
    __half sq16 = __float2half_rn(1.f);
    {
      uint4 raw[D / 8];
#pragma unroll
      for (int c8 = 0; c8 < D / 8; ++c8) raw[c8] = row_ok ? __ldg(reinterpret_cast<const uint4*>(qrow + c8 * 8))
                                                        : make_uint4(0, 0, 0, 0);
      uint32_t packed[D / 2];
      float amax = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < D / 8; ++c8) {
        const __half2* h = reinterpret_cast<const __half2*>(&raw[c8]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h[e]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
          packed[c8 * 4 + e] = pack_half2_rn(f.x * a.qk_scale, f.y * a.qk_scale);
        }
      }
#pragma unroll
      for (int c = 0; c < D / 2; c += 16) tmem_st16(tbase + lane_off + kColQ16 + c, packed + c);
      if (a.mode != TM_ROUTE_FP16) {
        uint32_t codes[D / 4];
        if (a.fuse_q) {
          // Block absmax over the 128 rows of this head = one BLKQ=128 quantisation block.
          float m = amax;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) bars->red[warp] = m;
          named_bar_sync_softmax();
          m = fmaxf(fmaxf(bars->red[0], bars->red[1]), fmaxf(bars->red[2], bars->red[3]));
          const float scale = quant_scale<kNumerics>(m);
          // a zero or non-finite block scale quantises to zeros, as in the reference
          const bool finite = scale > 0.f && scale <= 3.4028235e38f;
          QuantDiv qd;
          qd.init(scale);
          sq16 = __float2half_rn(scale);
#pragma unroll
          for (int c8 = 0; c8 < D / 8; ++c8) {
            const __half2* h = reinterpret_cast<const __half2*>(&raw[c8]);
            uint32_t u[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(h[e]);
              quant_code_pair<kNumerics>(f.x, f.y, qd, &u[2 * e], &u[2 * e + 1]);
              if (!finite) u[2 * e] = u[2 * e + 1] = 0u;
            }
            codes[c8 * 2] = __byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410);
            codes[c8 * 2 + 1] = __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410);
          }
        } else {
          const int8_t* q8row =
              a.q8 + (static_cast<int64_t>(q_start) + row) * a.q8_st + static_cast<int64_t>(hq) * a.q8_sh;
#pragma unroll
          for (int c16 = 0; c16 < D / 16; ++c16) {
            uint4 u = make_uint4(0, 0, 0, 0);
            if (row_ok) u = __ldg(reinterpret_cast<const uint4*>(q8row + c16 * 16));
            codes[c16 * 4 + 0] = u.x;
            codes[c16 * 4 + 1] = u.y;
            codes[c16 * 4 + 2] = u.z;
            codes[c16 * 4 + 3] = u.w;
          }
          const int qs_base = a.cu_qs[b];
          const int qs_end = a.cu_qs[b + 1];
          if (qs_end > qs_base && row_ok) {
            const int idx = min(qs_base + row / a.blkq, qs_end - 1);
            sq16 = a.q_scale[static_cast<int64_t>(idx) * a.HQ + hq];
          }
        }
#pragma unroll
        for (int c = 0; c < D / 4; c += 16) tmem_st16(tbase + lane_off + kColQ8 + c, codes + c);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->q_ready);
    }

    const int ks_base = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[b] : 0;
    const int ks_end = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[b + 1] : 0;
    const int vs_base = a.v8_path ? a.cu_vs[b] : 0;
    const int vs_end = a.v8_path ? a.cu_vs[b + 1] : 0;
    const __half* brow0 = (a.bias != nullptr && row_ok)
                              ? a.bias + static_cast<int64_t>(hq) * a.b_sh + static_cast<int64_t>(row) * a.b_sm
                              : nullptr;
    const float kNegInf = -__int_as_float(0x7f800000);
    float m_used = kNegInf;
    float l = 1.f;
    const int my_nb = rt.nb[half];
    bool ok = true;

    for (int j = 0; j < n_tiles; ++j) {
      const int slot = j % kSlots;
      const bool active = j < my_nb;  // uniform per warp (a warp never straddles halves)
      const int kind = active ? rt.kind(half, j) : 0;
      bool n16, n8;
      rt.needs(j, n16, n8);
      const uint32_t src_col = (kind == 1 && n16 && n8) ? kColX : (kColS + slot * 64);
      float ss = 1.f;
      if (active && kind == 1) {
        __half sk16 = __float2half_rn(1.f);
        if (ks_end > ks_base) {
          const int idx = min(ks_base + (j * kKeys) / a.blkk, ks_end - 1);
          sk16 = a.k_scale[static_cast<int64_t>(idx) * a.HK + hk];
        }
        ss = int8_score_scale(sq16, sk16, a.qk_scale);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[slot], (j / kSlots) & 1, a.err, kErrTimeoutScores));
      if (!ok) break;
      tc_fence_after();

      uint32_t p[32];
      float o_scale = 1.f;
      bool need_rescale = false;
      if (active) {
        int lim = seqlen_k - j * kKeys;
        if (a.causal) lim = min(lim, row + coff + 1 - j * kKeys);
        const __half* brow = brow0 ? brow0 + static_cast<int64_t>(j) * kKeys * a.b_sn : nullptr;
        softmax_tile<kNumerics>(tbase + lane_off + src_col, kind, ss, lim, a.rescale_threshold, m_used, l, p, o_scale,
                     need_rescale, brow, a.b_sn);
        if (kind == 1 && a.v8_path) {
          // p_scaled = fp16(p * sv), sv the V scale of the tile's block (:472-480)
          __half sv = __float2half_rn(1.f);
          if (vs_end > vs_base) sv = a.v_scale[static_cast<int64_t>(min(vs_base + (j * kKeys) / a.blkk, vs_end - 1)) * a.HK + hk];
          const float svf = __half2float(sv);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&p[i]));
            p[i] = pack_half2_rn(f.x * svf, f.y * svf);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) p[i] = 0u;
      }

      if (__any_sync(0xffffffffu, need_rescale)) {
        // O must hold PV(j-1) before it is rescaled; PV(j) waits for our P.
        const int jj = j - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[jj % kSlots], (jj / kSlots) & 1, a.err, kErrTimeoutPV));
        if (!ok) break;
        tc_fence_after();
        rescale_o_row<D>(tbase + lane_off + kColO, o_scale);
      }
      if (a.v8_path && n8) {
        // The int8 V of this tile (landed: its S is complete) as fp16 for the PV.
        convert_v8_stage<D>(smem, j % kStages, t);
        fence_proxy_async_smem();
      }
      if (a.v8_path && n8 && n16) {
        // Split tile: P of FP16-routed rows in columns [0, 32), of INT8-routed
        // rows in [32, 64); the other half of each row is zero.
        const bool int8_row = active && kind == 1;
        uint32_t pa[32], pb[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          pa[i] = int8_row ? 0u : p[i];
          pb[i] = int8_row ? p[i] : 0u;
        }
        tmem_st32(tbase + lane_off + kColS + slot * 64, pa);
        tmem_st32(tbase + lane_off + kColS + slot * 64 + 32, pb);
      } else {
        tmem_st32(tbase + lane_off + kColS + slot * 64, p);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_ready[slot]);
    }

    // ---- epilogue: O / l -> fp16
    __half* orow = a.out + (static_cast<int64_t>(q_start) + row) * a.o_st + static_cast<int64_t>(hq) * a.o_sh;
    if (n_tiles > 0 && ok) {
      const int jj = n_tiles - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[jj % kSlots], (jj / kSlots) & 1, a.err, kErrTimeoutPV));
      tc_fence_after();
    }
    store_o_row<kNumerics, D>(tbase + lane_off + kColO, n_tiles > 0, l, orow, row_ok && ok);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}


}  // namespace general

// Launch the general kernel (any supported block_m, head_dim 64/128, prequantised or fused Q).
int launch_attn_general(const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v, const CUtensorMap& v8,
                        const AttnArgs& a,
                        int tiles, int heads_q, int batch, cudaStream_t stream) {
  using namespace general;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    const int sm = static_cast<int>(kSmemBytes);
    const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    if (cudaFuncSetAttribute(tilemix_attn_fwd_kernel<kNumericsGpu, 64>, attr, sm) != cudaSuccess ||
        cudaFuncSetAttribute(tilemix_attn_fwd_kernel<kNumericsGpu, 128>, attr, sm) != cudaSuccess ||
        cudaFuncSetAttribute(tilemix_attn_fwd_kernel<kNumericsExact, 64>, attr, sm) != cudaSuccess ||
        cudaFuncSetAttribute(tilemix_attn_fwd_kernel<kNumericsExact, 128>, attr, sm) != cudaSuccess)
      return TM_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  dim3 grid(tiles, heads_q, batch);
  const bool gpu = a.numerics == kNumericsGpu;
  if (a.D == 128 && gpu)
    tilemix_attn_fwd_kernel<kNumericsGpu, 128><<<grid, kThreads, kSmemBytes, stream>>>(k16, k8, v, v8, a);
  else if (a.D == 128)
    tilemix_attn_fwd_kernel<kNumericsExact, 128><<<grid, kThreads, kSmemBytes, stream>>>(k16, k8, v, v8, a);
  else if (gpu)
    tilemix_attn_fwd_kernel<kNumericsGpu, 64><<<grid, kThreads, kSmemBytes, stream>>>(k16, k8, v, v8, a);
  else
    tilemix_attn_fwd_kernel<kNumericsExact, 64><<<grid, kThreads, kSmemBytes, stream>>>(k16, k8, v, v8, a);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace tilemix
