// Paired-tile TileMix attention forward with 128-key softmax steps (sm_100a).
//
// Same semantics and CTA work split as the paired kernel (attn_fwd_paired.cu):
// one CTA owns two 128-row query tiles A, B that share a KV head and every K/V
// tile feeds both. The difference is the unit of work of the softmax and MMA
// chains: a *step* of 128 keys (two 64-key routing tiles, each routed FP16 or
// INT8 on its own), so per-step fixed costs — TMEM load/store latency, barrier
// hand-offs, loop overhead — are paid once per 128 keys.
//
// TMEM (512 columns): O_A [0,128), O_B [128,256), one 128-column score slot per
// tile: S_A [256,384), S_B [384,512). P (fp16, 128 keys = 64 columns) is
// written over the first half of its score slot. Per tile X the chain is
//   S_X(j) -> softmax_X(j) -> PV_X(j) -> S_X(j+1) -> ...
// and the tensor core alternates between the two tiles' chains. S_X(j+1) overwrites the
// slot holding P_X(j): it is issued after PV_X(j) by the same thread and
// tcgen05.mma operations from one thread execute in issue order. The commit
// that publishes S_X(j) also covers PV_X(j-1), so the softmax can rescale O
// without another wait.
//
//   warps 0-3 / 4-7   softmax of tile A / B (thread = query row = TMEM lane);
//                     in-kernel Q scaling and INT8 quantisation at start
//   warp 8            TMA producer of K (formats routed by either tile), 64-key
//                     entries of a 3-deep ring, released after the S MMAs
//   warp 10           TMA producer of Q, then V (3-deep ring of 64-key entries,
//                     released after the PV MMAs)
//   warps 9 / 11      MMA issuers of tile A / B (converged warp, elected lane)
#include "attn_common.cuh"
#include "tilemix_b200.h"

namespace tilemix {
namespace paired128 {

constexpr int kD = 128;
constexpr int kRows = 128;
constexpr int kStepKeys = 2 * kKeys;
constexpr int kStages = 3;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;

constexpr uint32_t kQ16Bytes = kRows * kD * 2;  // 32 KB: [dims 0-63][dims 64-127], 128 rows each
constexpr uint32_t kQ8Bytes = kRows * kD;       // 16 KB
constexpr uint32_t kK16Bytes = kKeys * kD * 2;  // 16 KB
constexpr uint32_t kK8Bytes = kKeys * kD;       // 8 KB
constexpr uint32_t kVBytes = kKeys * kD * 2;    // 16 KB
constexpr uint32_t kOffQ16 = 0;
constexpr uint32_t kOffQ8 = kOffQ16 + 2 * kQ16Bytes;
constexpr uint32_t kOffK16 = kOffQ8 + 2 * kQ8Bytes;
constexpr uint32_t kOffV = kOffK16 + kStages * kK16Bytes;
constexpr uint32_t kOffK8 = kOffV + kStages * kVBytes;
constexpr uint32_t kOffBar = kOffK8 + kStages * kK8Bytes;
constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;

struct Barriers {
  uint64_t full_k[kStages];
  uint64_t full_v[kStages];
  uint64_t empty_k[kStages];  // K entry free: both tiles' S of that key tile ran
  uint64_t empty_v[kStages];  // V entry free: both tiles' PV of that key tile ran
  uint64_t q_full[2];
  uint64_t q_ready[2];
  uint64_t s_full[2];
  uint64_t p_ready[2];
  uint64_t pv_done[2];
  uint64_t mma_done[2];
  uint32_t tmem_base;
  float red[2][4];
};

struct QTile {
  uint64_t bits;
  int hq;
  int mtile;
  int nb;  // 64-key tiles visited (0 = tile absent)
};

__device__ __forceinline__ uint32_t col_o(int x) { return static_cast<uint32_t>(x) * 128u; }
__device__ __forceinline__ uint32_t col_s(int x) { return 256u + static_cast<uint32_t>(x) * 128u; }

// One 64-column half of the score slot -> fp16 scores with the reference's
// rounding (FP16 route: fp16(S); INT8 route: fp16(f32(S_i32) * ss), the product
// formed by one FFMA that rounds once).
template <int OFF>
__device__ __forceinline__ void load_half(uint32_t taddr, int kind, float ss, __half2 (&h)[64]) {
  uint32_t s0[32], s1[32];
  tmem_ld32(taddr, s0);
  tmem_ld32(taddr + 32, s1);
  tmem_wait_ld();
  if (kind == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      h[OFF + i] = __floats2half2_rn(__uint_as_float(s0[2 * i]), __uint_as_float(s0[2 * i + 1]));
      h[OFF + 16 + i] = __floats2half2_rn(__uint_as_float(s1[2 * i]), __uint_as_float(s1[2 * i + 1]));
    }
  } else {
    const float c = -12582912.0f * ss;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      h[OFF + i] = __floats2half2_rn(fmaf(__uint_as_float(s0[2 * i] + 0x4B400000u), ss, c),
                                     fmaf(__uint_as_float(s0[2 * i + 1] + 0x4B400000u), ss, c));
      h[OFF + 16 + i] = __floats2half2_rn(fmaf(__uint_as_float(s1[2 * i] + 0x4B400000u), ss, c),
                                          fmaf(__uint_as_float(s1[2 * i + 1] + 0x4B400000u), ss, c));
    }
  }
}

// exp2 of 32 packed pairs h[OFF..OFF+32) relative to m, fp16 P into TMEM at taddr.
template <int OFF>
__device__ __forceinline__ void exp_half(const __half2 (&h)[64], uint64_t negm, uint32_t taddr, uint64_t& acc0,
                                         uint64_t& acc1) {
  uint32_t p[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 f = __half22float2(h[OFF + i]);
    const float2 d = f32x2_unpack(f32x2_add(f32x2_pack(f.x, f.y), negm));
    const float e0 = ex2_approx(d.x), e1 = ex2_approx(d.y);
    const __half2 ph = __floats2half2_rn(e0, e1);
    if (i & 1)
      acc1 = f32x2_add(acc1, f32x2_pack(e0, e1));
    else
      acc0 = f32x2_add(acc0, f32x2_pack(e0, e1));
    p[i] = *reinterpret_cast<const uint32_t*>(&ph);
  }
  tmem_st32(taddr, p);
}

// The reference's softmax update (attention/triton/tilemix.py:179-207) over one
// 128-key step for this thread's row: keys at or beyond `lim` are masked; the
// second half is absent when have1 is false. P goes to the first 64 columns of
// the slot. Returns the factor O must be scaled by (1 = none).
__device__ __forceinline__ float softmax_step(uint32_t tS, int kind0, int kind1, float ss0, float ss1, bool have1,
                                              int lim, float thr, float& m_used, float& l) {
  __half2 h[64];
  load_half<0>(tS, kind0, ss0, h);
  const __half ninf = __ushort_as_half(0xFC00);
  if (have1) {
    load_half<32>(tS + 64, kind1, ss1, h);
  } else {
#pragma unroll
    for (int i = 32; i < 64; ++i) h[i] = __halves2half2(ninf, ninf);
  }
  if (lim < kStepKeys) {
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const __half lo = (2 * i < lim) ? __low2half(h[i]) : ninf;
      const __half hi = (2 * i + 1 < lim) ? __high2half(h[i]) : ninf;
      h[i] = __halves2half2(lo, hi);
    }
  }
  __half2 mt[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) mt[i] = __hmax2(h[i], h[32 + i]);
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) mt[i] = __hmax2(mt[i], mt[i + w]);
  }
  const float kNegInf = -__int_as_float(0x7f800000);
  const float mx = fmaxf(__low2float(mt[0]), __high2float(mt[0]));
  float o_scale = 1.f;
  if (mx != kNegInf && mx > m_used + thr) {
    const float alpha = ex2_approx(m_used - mx);  // 0 when m_used == -inf
    if (m_used != kNegInf) o_scale = alpha;
    l *= alpha;
    m_used = mx;
  }
  uint64_t acc0 = 0, acc1 = 0;
  if (mx != kNegInf) {
    const uint64_t negm = f32x2_pack(-m_used, -m_used);
    exp_half<0>(h, negm, tS, acc0, acc1);
    exp_half<32>(h, negm, tS + 32, acc0, acc1);
    const float2 a0 = f32x2_unpack(acc0), a1 = f32x2_unpack(acc1);
    l += (a0.x + a0.y) + (a1.x + a1.y);
  } else {
    uint32_t z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) z[i] = 0u;
    tmem_st32(tS, z);
    tmem_st32(tS + 32, z);
  }
  return o_scale;
}

__global__ void __launch_bounds__(kThreads, 1)
    tilemix_attn_fwd_paired128_kernel(const __grid_constant__ CUtensorMap tm_q,
                                      const __grid_constant__ CUtensorMap tm_k16,
                                      const __grid_constant__ CUtensorMap tm_k8,
                                      const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kOffBar);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int q_start = a.cu_q[b];
  const int seqlen_q = a.cu_q[b + 1] - q_start;
  const int k_start = a.cu_k[b];
  const int seqlen_k = a.cu_k[b + 1] - k_start;
  const int m_blocks = (seqlen_q + kRows - 1) / kRows;

  QTile tl[2];
  const int rev = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    if (a.pair_heads) {
      tl[x].hq = 2 * static_cast<int>(blockIdx.y) + x;
      tl[x].mtile = rev;
    } else {
      tl[x].hq = blockIdx.y;
      tl[x].mtile = 2 * rev + x;
    }
    const bool valid = tl[x].mtile * kRows < seqlen_q;
    tl[x].nb = valid ? visited_key_tiles(tl[x].mtile * kRows, kRows, seqlen_q, seqlen_k, a.causal) : 0;
    tl[x].bits = 0;
    if (valid && a.mode == TM_ROUTE_MIXED)
      tl[x].bits = a.bitmask[static_cast<int64_t>(tl[x].hq / a.group) * m_blocks + tl[x].mtile];
  }
  if (tl[0].mtile * kRows >= seqlen_q && tl[1].mtile * kRows >= seqlen_q) return;  // uniform, before any barrier
  const int hk = tl[0].hq / a.group;  // both tiles share the KV head
  const int n_iter = max(tl[0].nb, tl[1].nb);
  const int n_steps = (n_iter + 1) / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full_k[s], 1);
      mbar_init(&bars->full_v[s], 1);
      mbar_init(&bars->empty_k[s], 2);  // one release from each MMA warp
      mbar_init(&bars->empty_v[s], 2);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->q_full[x], 1);
      mbar_init(&bars->q_ready[x], kRows);
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->p_ready[x], kRows);
      mbar_init(&bars->pv_done[x], 1);
      mbar_init(&bars->mma_done[x], 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 8 || warp == 10) {
    // ------------------------------------------------------------------ producers (64-key entries)
    const bool is_k = warp == 8;
    if (is_k) {
      prefetch_tmap(&tm_k16);
      if (a.mode != TM_ROUTE_FP16) prefetch_tmap(&tm_k8);
    } else {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_v);
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (tl[x].mtile * kRows >= seqlen_q) continue;
        mbar_arrive_expect_tx_e(&bars->q_full[x], kQ16Bytes);
        tma_load_4d_e(smem + kOffQ16 + x * kQ16Bytes, &tm_q, &bars->q_full[x], 0, q_start + tl[x].mtile * kRows, 0,
                      tl[x].hq);
      }
    }
    bool ok = true;
    RouteWalker rw[2];
#pragma unroll
    for (int x = 0; x < 2; ++x) rw[x].init(a.mode, tl[x].bits, a.block_n_mask);
    for (int j = 0; j < n_iter && ok; ++j) {
      const int s = j % kStages;
      if (j >= kStages)
        ok = __all_sync(0xffffffffu, mbar_wait_spin(is_k ? &bars->empty_k[s] : &bars->empty_v[s],
                                               ((j - kStages) / kStages) & 1, a.err, kErrTimeoutEmpty));
      if (!ok) break;
      const int tok = k_start + j * kKeys;
      if (is_k) {
        bool n16 = false, n8 = false;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (j < tl[x].nb) {
            if (rw[x].kind())
              n8 = true;
            else
              n16 = true;
          }
          rw[x].advance();
        }
        mbar_arrive_expect_tx_e(&bars->full_k[s], (n16 ? kK16Bytes : 0u) + (n8 ? kK8Bytes : 0u));
        if (n16) tma_load_4d_e(smem + kOffK16 + s * kK16Bytes, &tm_k16, &bars->full_k[s], 0, tok, 0, hk);
        if (n8) tma_load_3d_e(smem + kOffK8 + s * kK8Bytes, &tm_k8, &bars->full_k[s], 0, hk, tok);
      } else {
        mbar_arrive_expect_tx_e(&bars->full_v[s], kVBytes);
        tma_load_4d_e(smem + kOffV + s * kVBytes, &tm_v, &bars->full_v[s], 0, tok, 0, hk);
      }
    }
    // Drain: every copy this warp issued has landed before the CTA can exit.
    const int first = max(0, n_iter - kStages);
    for (int j = first; j < n_iter; ++j)
      mbar_wait(is_k ? &bars->full_k[j % kStages] : &bars->full_v[j % kStages], (j / kStages) & 1, a.err,
                kErrTimeoutDrain);
    if (!is_k)
      for (int x = 0; x < 2; ++x)
        if (tl[x].mtile * kRows < seqlen_q) mbar_wait(&bars->q_full[x], 0, a.err, kErrTimeoutDrain);
  } else if (warp == 9 || warp == 11) {
    // ------------------------------------------------------------------ MMA issuers
    // Warp 9 issues tile A's MMAs, warp 11 tile B's, in the order
    //   S_X(j), release K of step j, PV_X(j), release V of step j
    // for every step j of the CTA (a warp releases entries its tile does not use
    // too, after waiting for their data, so a stage's two releases always belong
    // to the same phase).
    const int x = warp == 9 ? 0 : 1;
    const QTile me = tl[x];
    constexpr uint32_t idesc_qk16 = make_idesc(1, 0, 0, 0, 128, 64);
    constexpr uint32_t idesc_qk8 = make_idesc(2, 1, 0, 0, 128, 64);
    constexpr uint32_t idesc_pv = make_idesc(1, 0, 0, 1, 128, kD);
    const uint64_t dq16 = make_sdesc(smem_u32(smem + kOffQ16 + x * kQ16Bytes), 16, 1024, 2);
    const uint64_t dq8 = make_sdesc(smem_u32(smem + kOffQ8 + x * kQ8Bytes), 16, 1024, 2);
    const uint64_t dk16 = make_sdesc(smem_u32(smem + kOffK16), 16, 1024, 2);
    const uint64_t dk8 = make_sdesc(smem_u32(smem + kOffK8), 16, 1024, 2);
    const uint64_t dv = make_sdesc(smem_u32(smem + kOffV), kVBytes / 2, 1024, 2);
    const uint32_t d_o = tbase + col_o(x);
    const uint32_t d_s = tbase + col_s(x);
    bool ok = true;
    if (me.mtile * kRows < seqlen_q)
      ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_ready[x], 0, a.err, kErrTimeoutQ));
    tc_fence_after();
    RouteWalker rw;
    rw.init(a.mode, me.bits, a.block_n_mask);
    for (int j = 0; j < n_steps && ok; ++j) {
      // ---- S_X(j): up to two 64-key routing tiles into the two halves of the slot
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = 2 * j + h;
        if (t >= n_iter) break;
        const int st = t % kStages;
        const int kind = rw.kind();
        rw.advance();
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->full_k[st], (t / kStages) & 1, a.err, kErrTimeoutFull));
        if (!ok) break;
        if (t < me.nb) {
          tc_fence_after();
          const uint32_t d = d_s + 64u * h;
          if (kind == 0) {
            const uint64_t kb = dk16 + ((st * kK16Bytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t off_q = ((kk >> 2) * (kQ16Bytes / 2) + (kk & 3) * 32) >> 4;
              const uint32_t off_k = ((kk >> 2) * (kK16Bytes / 2) + (kk & 3) * 32) >> 4;
              mma_f16_ss_e(d, dq16 + off_q, kb + off_k, idesc_qk16, kk > 0 ? 1u : 0u);
            }
          } else {
            const uint64_t kb = dk8 + ((st * kK8Bytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < kD / 32; ++kk) mma_i8_ss_e(d, dq8 + kk * 2, kb + kk * 2, idesc_qk8, kk > 0 ? 1u : 0u);
          }
        }
      }
      if (!ok) break;
      if (2 * j < me.nb) tc_commit_e(&bars->s_full[x]);
      tc_commit_e(&bars->empty_k[(2 * j) % kStages]);
      if (2 * j + 1 < n_iter) tc_commit_e(&bars->empty_k[(2 * j + 1) % kStages]);

      // ---- PV_X(j) once P_X(j) is in TMEM
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = 2 * j + h;
        if (t >= n_iter) break;
        ok = __all_sync(0xffffffffu,
                        mbar_wait_spin(&bars->full_v[t % kStages], (t / kStages) & 1, a.err, kErrTimeoutFull));
        if (!ok) break;
      }
      if (!ok) break;
      if (2 * j < me.nb) {
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->p_ready[x], j & 1, a.err, kErrTimeoutP));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = 2 * j + h;
          if (t >= me.nb) break;
          const uint64_t vb = dv + (((t % kStages) * kVBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)
            mma_f16_ts_e(d_o, d_s + (4 * h + kk) * 8, vb + ((kk * 16 * 128) >> 4), idesc_pv,
                         (j > 0 || h > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit_e(&bars->pv_done[x]);
      }
      tc_commit_e(&bars->empty_v[(2 * j) % kStages]);
      if (2 * j + 1 < n_iter) tc_commit_e(&bars->empty_v[(2 * j + 1) % kStages]);
    }
    tc_commit_e(&bars->mma_done[x]);
    mbar_wait(&bars->mma_done[x], 0, a.err, kErrTimeoutDrain);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int x = warp >> 2;
    const int t = threadIdx.x & 127;  // row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const QTile me = tl[x];
    if (me.mtile * kRows < seqlen_q) {
      const int row = me.mtile * kRows + t;
      const bool row_ok = row < seqlen_q;
      bool ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_full[x], 0, a.err, kErrTimeoutQ));
      __half sq16 = __float2half_rn(1.f);
      {
        // Scale Q in place (elementwise, so the swizzled layout is irrelevant)
        // and build the INT8 operand of this 128-row block.
        uint8_t* q16 = smem + kOffQ16 + x * kQ16Bytes;
        uint4 raw[16];
        float amax = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4* ptr = reinterpret_cast<uint4*>(q16 + (c >> 3) * (kQ16Bytes / 2) + t * 128 + (((c & 7) ^ (t & 7)) << 4));
          raw[c] = *ptr;
          const __half2* hh = reinterpret_cast<const __half2*>(&raw[c]);
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(hh[e]);
            if (row_ok) amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
            w[e] = pack_half2_rn(f.x * a.qk_scale, f.y * a.qk_scale);
          }
          *ptr = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (a.mode != TM_ROUTE_FP16) {
          float m = amax;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) bars->red[x][warp & 3] = m;
          asm volatile("bar.sync %0, 128;" ::"r"(1 + x) : "memory");
          m = fmaxf(fmaxf(bars->red[x][0], bars->red[x][1]), fmaxf(bars->red[x][2], bars->red[x][3]));
          const float scale = __fdiv_rn(m, 127.f);
          const float rscale = __frcp_rn(scale);
          sq16 = __float2half_rn(scale);
          uint8_t* q8 = smem + kOffQ8 + x * kQ8Bytes;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              const __half2* hh = reinterpret_cast<const __half2*>(&raw[2 * g + hc]);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float2 f0 = __half22float2(hh[2 * e]);
                const float2 f1 = __half22float2(hh[2 * e + 1]);
                w[hc * 2 + e] = (static_cast<uint32_t>(quant_code_rcp(f0.x, scale, rscale)) & 0xFFu) |
                                ((static_cast<uint32_t>(quant_code_rcp(f0.y, scale, rscale)) & 0xFFu) << 8) |
                                ((static_cast<uint32_t>(quant_code_rcp(f1.x, scale, rscale)) & 0xFFu) << 16) |
                                ((static_cast<uint32_t>(quant_code_rcp(f1.y, scale, rscale)) & 0xFFu) << 24);
              }
            }
            *reinterpret_cast<uint4*>(q8 + t * 128 + ((g ^ (t & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->q_ready[x]);
      }

      const int ks_base = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[b] : 0;
      const int ks_end = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[b + 1] : 0;
      const float kNegInf = -__int_as_float(0x7f800000);
      float m_used = kNegInf;
      float l = 1.f;
      const int coff = seqlen_k - seqlen_q;
      const uint32_t tS = tbase + lane_off + col_s(x);
      const uint32_t tO = tbase + lane_off + col_o(x);
      // Routes and K scale rows of consecutive 64-key tiles, tracked incrementally;
      // the scales of a step are loaded one step ahead (unconditional loads of a
      // valid row, selected when used) to keep global loads off the critical path.
      RouteWalker rw;
      rw.init(a.mode, me.bits, a.block_n_mask);
      const int sk_per = a.blkk / kKeys;
      int sk_idx = ks_base, sk_sub = 0;
      const bool have_sk = ks_end > ks_base;
      const __half* sk_col = a.k_scale + hk;
      auto load_next_sk = [&]() -> __half {
        const __half v = have_sk ? sk_col[static_cast<int64_t>(min(sk_idx, ks_end - 1)) * a.HK] : __half();
        if (++sk_sub == sk_per) {
          sk_sub = 0;
          ++sk_idx;
        }
        return v;
      };
      __half skn0 = load_next_sk();
      __half skn1 = load_next_sk();
      const int my_steps = (me.nb + 1) / 2;
      for (int j = 0; ok && j < my_steps; ++j) {
        const bool have1 = 2 * j + 1 < me.nb;
        const int kind0 = rw.kind();
        rw.advance();
        const int kind1 = rw.kind();
        rw.advance();
        const __half sk0 = (have_sk && kind0 == 1) ? skn0 : __float2half_rn(1.f);
        const __half sk1 = (have_sk && kind1 == 1) ? skn1 : __float2half_rn(1.f);
        skn0 = load_next_sk();
        skn1 = load_next_sk();
        const float ss0 = kind0 == 1 ? int8_score_scale(sq16, sk0, a.qk_scale) : 1.f;
        const float ss1 = kind1 == 1 ? int8_score_scale(sq16, sk1, a.qk_scale) : 1.f;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->s_full[x], j & 1, a.err, kErrTimeoutScores));
        if (!ok) break;
        tc_fence_after();
        int lim = seqlen_k - j * kStepKeys;
        if (a.causal) lim = min(lim, row + coff + 1 - j * kStepKeys);
        const float o_scale = softmax_step(tS, kind0, kind1, ss0, ss1, have1, lim, a.rescale_threshold, m_used, l);
        // PV_X(j-1) is complete (the commit that published S_X(j) came after it),
        // so O can be rescaled in place.
        if (__any_sync(0xffffffffu, o_scale != 1.f)) rescale_o_row<kD>(tO, o_scale);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->p_ready[x]);
      }
      __half* orow = a.out + (static_cast<int64_t>(q_start) + row) * a.o_st + static_cast<int64_t>(me.hq) * a.o_sh;
      if (ok && my_steps > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->pv_done[x], (my_steps - 1) & 1, a.err, kErrTimeoutPV));
        tc_fence_after();
      }
      store_o_row<kD>(tO, my_steps > 0, l, orow, row_ok && ok);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace paired128

int launch_attn_paired128(const CUtensorMap& q, const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v,
                          const AttnArgs& a, int batch, int max_seqlen_q, cudaStream_t stream) {
  using namespace paired128;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(tilemix_attn_fwd_paired128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess)
      return TM_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  const int mtiles = (max_seqlen_q + kRows - 1) / kRows;
  dim3 grid;
  if (a.pair_heads)
    grid = dim3(mtiles, a.HQ / 2, batch);
  else
    grid = dim3((mtiles + 1) / 2, a.HQ, batch);
  tilemix_attn_fwd_paired128_kernel<<<grid, kThreads, kSmemBytes, stream>>>(q, k16, k8, v, a);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace tilemix
