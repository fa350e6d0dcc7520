// Paired-tile TileMix attention forward for B200 (sm_100a): the fast path for
// head_dim 128, block_m 128 and in-kernel Q quantisation (BLKQ = 128), which is
// what the model integration and tilemix_attention_with_quant use.
//
// Same semantics as the general kernel (attention/triton/tilemix.py:503-951);
// different mapping. One CTA owns two 128-row query tiles X = A, B that share a
// KV head: either two Q heads of one GQA group at the same query block (their
// routing words are the same map row), or two consecutive query blocks of one
// head. Every K/V tile is loaded once into shared memory and feeds both tiles.
//
//   warps 0-3 / 4-7   softmax warpgroup of tile A / B (thread = query row =
//                     TMEM lane). At start: scale Q in place in shared memory
//                     (fp16(q * sm_scale * log2e)) and quantise it per 128-row
//                     block into the INT8 operand (BLKQ = 128 block = the tile).
//   warp 8            TMA producer of K (only the formats routed by either tile),
//                     64 keys per stage of a 3-stage ring
//   warp 10           TMA producer of the Q tiles, then of V (same ring stages)
//                     Every K16 / V / Q tile arrives in a single 4-D copy (all 128
//                     dims), so each producer issues at most two copies per stage:
//                     a thread's bulk-tensor copies go out one after another, and
//                     splitting K and V over two warps halves that serial chain.
//   warps 9 / 11      MMA issuer of tile A / B: S_X = Q_X K^T (tcgen05 kind::f16
//                     or kind::i8, both operands in shared memory) into a TMEM
//                     score slot of tile X; O_X += P_X V (kind::f16, P from
//                     TMEM, fp32 O). Two issuers halve the serial issue chain.
// TMEM (512 columns): O_A [0,128), O_B [128,256), two 64-column S/P slots per
// tile at [256,384) and [384,512). Each issuer's order per key tile j is
//   S_X(j), PV_X(j-1)
// so S_X(j) runs on the tensor core while the softmax works on tile j-1.
#include "attn_common.cuh"
#include "tilemix_b200.h"

namespace tilemix {
namespace paired {

constexpr int kD = 128;
constexpr int kRows = 128;
constexpr int kStages = 3;
#ifndef TILEMIX_PAIRED_PREFETCH
#define TILEMIX_PAIRED_PREFETCH 0
#endif
constexpr int kPrefetch = TILEMIX_PAIRED_PREFETCH;  // key tiles warmed in L2 ahead of the ring (0 = off)
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;

constexpr uint32_t kQ16Bytes = kRows * kD * 2;  // 32 KB, two 64-column boxes of 16 KB
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
  uint64_t empty_k[kStages];  // K stage free: both tiles' S of that key tile done
  uint64_t empty_v[kStages];  // V stage free: both tiles' PV of that key tile done
  uint64_t q_full[2];
  uint64_t q_ready[2];
  uint64_t s_full[2][2];
  uint64_t p_ready[2][2];
  uint64_t pv_done[2][2];
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
__device__ __forceinline__ uint32_t col_s(int x, int slot) {
  return 256u + static_cast<uint32_t>(x) * 128u + static_cast<uint32_t>(slot) * 64u;
}

__global__ void __launch_bounds__(kThreads, 1)
    tilemix_attn_fwd_paired_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k16,
                                   const __grid_constant__ CUtensorMap tm_k8, const __grid_constant__ CUtensorMap tm_v,
                                   const AttnArgs a) {
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
  const bool valid0 = tl[0].mtile * kRows < seqlen_q;
  const bool valid1 = tl[1].mtile * kRows < seqlen_q;
  if (!valid0 && !valid1) return;  // uniform, before any barrier or allocation
  const int hk = tl[0].hq / a.group;  // both tiles share the KV head
  const int n_iter = max(tl[0].nb, tl[1].nb);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full_k[s], 1);
      mbar_init(&bars->full_v[s], 1);
      mbar_init(&bars->empty_k[s], 2);  // one commit from each MMA warp
      mbar_init(&bars->empty_v[s], 2);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->q_full[x], 1);
      mbar_init(&bars->q_ready[x], kRows);
      for (int s = 0; s < 2; ++s) {
        mbar_init(&bars->s_full[x][s], 1);
        mbar_init(&bars->p_ready[x][s], kRows);
        mbar_init(&bars->pv_done[x][s], 1);
      }
    }
    mbar_init(&bars->mma_done[0], 1);
    mbar_init(&bars->mma_done[1], 1);
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
    // ------------------------------------------------------------------ producers
    // The whole warp runs the loop (warp-uniform control flow); one elected
    // lane issues each copy.
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
      if (kPrefetch > 0 && lane == 0) {
        const int jq = j + kPrefetch;
        if (jq < n_iter) {
          const int ptok = k_start + jq * kKeys;
          if (is_k) {
            tma_prefetch_l2_4d(&tm_k16, 0, ptok, 0, hk);
            if (a.mode != TM_ROUTE_FP16) tma_prefetch_l2_3d(&tm_k8, 0, hk, ptok);
          } else {
            tma_prefetch_l2_4d(&tm_v, 0, ptok, 0, hk);
          }
        }
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
    // One warp per query tile X (warp 9: A, warp 11: B, on different SM
    // sub-partitions), each running converged with one elected lane issuing,
    // in a fixed order per key tile j:
    //   S_X(j), release K(j), PV_X(j-1), release V(j-1)
    // (a stage is free once both warps have committed its release). S_X(j)
    // overwrites TMEM slot j&1, which P_X(j-2) occupied: PV_X(j-2) was issued
    // earlier by the same thread and tcgen05.mma operations from one thread
    // execute in issue order, so it has read P before S_X(j) writes the slot.
    // Descriptors are built once; a byte offset is added as offset >> 4 to the
    // start-address field (all shared-memory offsets here are < 256 KB).
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
    bool ok = true;
    if (me.mtile * kRows < seqlen_q) ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_ready[x], 0, a.err, kErrTimeoutQ));
    tc_fence_after();
    RouteWalker rw;
    rw.init(a.mode, me.bits, a.block_n_mask);
    for (int j = 0; j <= n_iter && ok; ++j) {
      if (j < n_iter) {
        const int st = j % kStages;
        const int kind = rw.kind();
        rw.advance();
        // Wait for K(j) even when this tile does not use it: the release below
        // must not reach the stage's barrier before the other warp's release of
        // the previous use of the stage (the copy of K(j) waited for it), or
        // two releases from this warp could complete one phase.
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->full_k[st], (j / kStages) & 1, a.err, kErrTimeoutFull));
        if (!ok) break;
        if (j < me.nb) {
          tc_fence_after();
          const uint32_t d = tbase + col_s(x, j & 1);
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
          tc_commit_e(&bars->s_full[x][j & 1]);
        }
        tc_commit_e(&bars->empty_k[st]);  // this warp is done with K(j) once its S has run
      }
      if (j >= 1) {
        const int jj = j - 1;
        const int st = jj % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->full_v[st], (jj / kStages) & 1, a.err, kErrTimeoutFull));
        if (!ok) break;
        if (jj < me.nb) {
          ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->p_ready[x][jj & 1], (jj >> 1) & 1, a.err, kErrTimeoutP));
          if (!ok) break;
          tc_fence_after();
          const uint64_t vb = dv + ((st * kVBytes) >> 4);
          const uint32_t pa = tbase + col_s(x, jj & 1);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)
            mma_f16_ts_e(d_o, pa + kk * 8, vb + ((kk * 16 * 128) >> 4), idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          tc_commit_e(&bars->pv_done[x][jj & 1]);
        }
        tc_commit_e(&bars->empty_v[st]);
      }
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
    const bool tile_ok = me.mtile * kRows < seqlen_q;
    if (tile_ok) {
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
          const __half2* h = reinterpret_cast<const __half2*>(&raw[c]);
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h[e]);
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
            // 16 codes of dims [16g, 16g+16) = raw chunks 2g and 2g+1
            uint32_t w[4];
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              const __half2* h = reinterpret_cast<const __half2*>(&raw[2 * g + hc]);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float2 f0 = __half22float2(h[2 * e]);
                const float2 f1 = __half22float2(h[2 * e + 1]);
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
      // K block scale of a tile, loaded one tile ahead to keep the global load
      // off the critical path. Routes and scale blocks of consecutive tiles are
      // tracked incrementally (no per-tile division).
      RouteWalker rw;
      rw.init(a.mode, me.bits, a.block_n_mask);
      const int sk_per = a.blkk / kKeys;  // 64-key tiles per K scale block (blkk % 64 == 0)
      int sk_idx = ks_base, sk_sub = 0;
      // The load is unconditional (clamped to a valid row) and its value is only
      // selected when used, one tile later, so no instruction waits on it early.
      const bool have_sk = ks_end > ks_base;
      const __half* sk_col = a.k_scale + hk;
      auto load_next_sk = [&]() -> __half {  // raw scale of the next tile in order; then step
        const __half v = have_sk ? sk_col[static_cast<int64_t>(min(sk_idx, ks_end - 1)) * a.HK] : __half();
        if (++sk_sub == sk_per) {
          sk_sub = 0;
          ++sk_idx;
        }
        return v;
      };
      __half sk_next = load_next_sk();
      for (int j = 0; ok && j < me.nb; ++j) {
        const int slot = j & 1;
        const int kind = rw.kind();
        rw.advance();
        const __half sk16 = (have_sk && kind == 1) ? sk_next : __float2half_rn(1.f);
        sk_next = load_next_sk();
        const float ss = kind == 1 ? int8_score_scale(sq16, sk16, a.qk_scale) : 1.f;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->s_full[x][slot], (j >> 1) & 1, a.err, kErrTimeoutScores));
        if (!ok) break;
        tc_fence_after();
        int lim = seqlen_k - j * kKeys;
        if (a.causal) lim = min(lim, row + coff + 1 - j * kKeys);
        uint32_t p[32];
        float o_scale;
        bool need_rescale;
        softmax_tile(tbase + lane_off + col_s(x, slot), kind, ss, lim, a.rescale_threshold, m_used, l, p, o_scale,
                     need_rescale);
        if (__any_sync(0xffffffffu, need_rescale)) {
          const int jj = j - 1;
          ok = __all_sync(0xffffffffu,
                          mbar_wait_spin(&bars->pv_done[x][jj & 1], (jj >> 1) & 1, a.err, kErrTimeoutPV));
          if (!ok) break;
          tc_fence_after();
          rescale_o_row<kD>(tbase + lane_off + col_o(x), o_scale);
        }
        tmem_st32(tbase + lane_off + col_s(x, slot), p);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->p_ready[x][slot]);
      }
      __half* orow = a.out + (static_cast<int64_t>(q_start) + row) * a.o_st + static_cast<int64_t>(me.hq) * a.o_sh;
      if (ok && me.nb > 0) {
        const int jj = me.nb - 1;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->pv_done[x][jj & 1], (jj >> 1) & 1, a.err, kErrTimeoutPV));
        tc_fence_after();
      }
      store_o_row<kD>(tbase + lane_off + col_o(x), me.nb > 0, l, orow, row_ok && ok);
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

}  // namespace paired

int launch_attn_paired(const CUtensorMap& q, const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v,
                       const AttnArgs& a, int batch, int max_seqlen_q, cudaStream_t stream) {
  using namespace paired;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(tilemix_attn_fwd_paired_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  tilemix_attn_fwd_paired_kernel<<<grid, kThreads, kSmemBytes, stream>>>(q, k16, k8, v, a);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace tilemix
