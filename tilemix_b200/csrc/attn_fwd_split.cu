// Paired-tile TileMix attention forward with a split-row softmax (sm_100a).
//
// Same CTA work split, memory pipeline and MMA issue as the paired kernel
// (attn_fwd_paired.cu): one CTA owns two 128-row query tiles A, B sharing a KV
// head, 64-key routing tiles, two 64-column TMEM score slots per tile. The
// softmax of each tile runs on 8 warps instead of 4: every query row is shared
// by two threads in different warps of the same TMEM lane quadrant, each
// taking 32 of the tile's 64 key columns. The two exchange their partial row
// maxima through tagged shared-memory words (bounded polls, double-buffered by
// step parity) and keep partial row sums, combined in the epilogue. The aim is
// four softmax warps per SM sub-partition to hide exp / convert latency; on the
// 8 x 4096 causal workload it measures slightly slower than the paired kernel
// (1.22 vs 1.20 ms), so it is an explicit option, not the default.
//
//   warps 0-7 / 8-15  softmax of tile A / B: warps 4h..4h+3 of a tile take key
//                     columns [32h, 32h+32) of rows 32*(warp%4) + lane
//   warp 16           TMA producer of K;  warp 18: TMA producer of Q, then V
//   warps 17 / 19     MMA issuers of tile A / B
#include "attn_common.cuh"
#include "tilemix_b200.h"

namespace tilemix {
namespace split {

constexpr int kD = 128;
constexpr int kRows = 128;
constexpr int kStages = 3;
#ifndef TILEMIX_PAIRED_PREFETCH
#define TILEMIX_PAIRED_PREFETCH 0
#endif
constexpr int kPrefetch = TILEMIX_PAIRED_PREFETCH;  // key tiles warmed in L2 ahead of the ring (0 = off)
constexpr int kThreads = 640;
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
constexpr uint32_t kSmemBytes = kOffBar + 8192 + 512 + 1024;

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
  float red[2][8];                      // Q block absmax per softmax warp
  uint32_t xmax[2][2][2][kRows];        // [tile][step parity][column half][row]: step tag << 16 | fp16 max
  unsigned long long xsum[2][2][kRows]; // [tile][column half][row]: tag << 32 | fp32 partial row sum
};

struct QTile {
  uint64_t bits;
  int hq;
  int mtile;
  int nb;  // 64-key tiles visited (0 = tile absent)
};

// Bounded exchange of one value with the partner thread of a split row: the
// writer publishes (tag, value) in one shared-memory word; the reader polls for
// the tag it expects, giving up after the library's wait timeout.
__device__ __forceinline__ void xchg_put(uint32_t* w, uint32_t tag, uint32_t v16) {
  asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(smem_u32(w)), "r"((tag << 16) | v16) : "memory");
}
__device__ __forceinline__ bool xchg_get(const uint32_t* w, uint32_t tag, uint32_t& v16, int* err, int code) {
  unsigned long long t0 = 0;
  for (uint32_t n = 0;; ++n) {
    uint32_t v;
    asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(w)) : "memory");
    if ((v >> 16) == (tag & 0xFFFFu)) {
      v16 = v & 0xFFFFu;
      return true;
    }
    if (n == 0) t0 = globaltimer_ns();
    if ((n & 1023u) == 1023u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ void xchg_put64(unsigned long long* w, uint32_t v) {
  asm volatile("st.volatile.shared.u64 [%0], %1;" ::"r"(smem_u32(w)), "l"((1ull << 32) | v) : "memory");
}
__device__ __forceinline__ bool xchg_get64(const unsigned long long* w, uint32_t& v, int* err, int code) {
  unsigned long long t0 = 0;
  for (uint32_t n = 0;; ++n) {
    unsigned long long x;
    asm volatile("ld.volatile.shared.u64 %0, [%1];" : "=l"(x) : "r"(smem_u32(w)) : "memory");
    if ((x >> 32) == 1ull) {
      v = static_cast<uint32_t>(x);
      return true;
    }
    if (n == 0) t0 = globaltimer_ns();
    if ((n & 1023u) == 1023u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, code);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t col_o(int x) { return static_cast<uint32_t>(x) * 128u; }
__device__ __forceinline__ uint32_t col_s(int x, int slot) {
  return 256u + static_cast<uint32_t>(x) * 128u + static_cast<uint32_t>(slot) * 64u;
}

__global__ void __launch_bounds__(kThreads, 1)
    tilemix_attn_fwd_split_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k16,
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
      mbar_init(&bars->q_ready[x], 2 * kRows);
      for (int s = 0; s < 2; ++s) {
        mbar_init(&bars->s_full[x][s], 1);
        mbar_init(&bars->p_ready[x][s], 2 * kRows);
        mbar_init(&bars->pv_done[x][s], 1);
      }
    }
    mbar_init(&bars->mma_done[0], 1);
    mbar_init(&bars->mma_done[1], 1);
    fence_mbarrier_init();
  }
  // Exchange words start with tag 0, which no step uses.
  for (int i = threadIdx.x; i < 2 * 2 * 2 * kRows; i += kThreads) (&bars->xmax[0][0][0][0])[i] = 0u;
  for (int i = threadIdx.x; i < 2 * 2 * kRows; i += kThreads) (&bars->xsum[0][0][0])[i] = 0ull;
  if (warp == 17) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 16 || warp == 18) {
    // ------------------------------------------------------------------ producers
    // The whole warp runs the loop (warp-uniform control flow); one elected
    // lane issues each copy.
    const bool is_k = warp == 16;
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
  } else if (warp == 17 || warp == 19) {
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
    const int x = warp == 17 ? 0 : 1;
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
    // ------------------------------------------------------------------ softmax (split rows)
    const int x = warp >> 3;         // tile
    const int hh = (warp >> 2) & 1;  // key-column half of every 64-key tile
    const int quad = warp & 3;       // TMEM lane quadrant
    const int t = quad * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const QTile me = tl[x];
    if (me.mtile * kRows < seqlen_q) {
      const int row = me.mtile * kRows + t;
      const bool row_ok = row < seqlen_q;
      bool ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_full[x], 0, a.err, kErrTimeoutQ));
      __half sq16 = __float2half_rn(1.f);
      {
        // Scale this thread's 64 dims of Q in place and build its half of the
        // INT8 operand of the 128-row block (block absmax over 256 threads).
        uint8_t* q16 = smem + kOffQ16 + x * kQ16Bytes + hh * (kQ16Bytes / 2);
        uint4 raw[8];
        float amax = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4* ptr = reinterpret_cast<uint4*>(q16 + t * 128 + ((c ^ (t & 7)) << 4));
          raw[c] = *ptr;
          const __half2* hq2 = reinterpret_cast<const __half2*>(&raw[c]);
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(hq2[e]);
            if (row_ok) amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
            w[e] = pack_half2_rn(f.x * a.qk_scale, f.y * a.qk_scale);
          }
          *ptr = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (a.mode != TM_ROUTE_FP16) {
          float m = amax;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) bars->red[x][warp & 7] = m;
          asm volatile("bar.sync %0, 256;" ::"r"(1 + x) : "memory");
          m = bars->red[x][0];
#pragma unroll
          for (int i = 1; i < 8; ++i) m = fmaxf(m, bars->red[x][i]);
          const float scale = __fdiv_rn(m, 127.f);
          const float rscale = __frcp_rn(scale);
          sq16 = __float2half_rn(scale);
          uint8_t* q8 = smem + kOffQ8 + x * kQ8Bytes;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            // 16 codes of dims [64hh + 16g, 64hh + 16g + 16) = raw chunks 2g and 2g+1
            uint32_t w[4];
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              const __half2* hq2 = reinterpret_cast<const __half2*>(&raw[2 * g + hc]);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float2 f0 = __half22float2(hq2[2 * e]);
                const float2 f1 = __half22float2(hq2[2 * e + 1]);
                w[hc * 2 + e] = (static_cast<uint32_t>(quant_code_rcp(f0.x, scale, rscale)) & 0xFFu) |
                                ((static_cast<uint32_t>(quant_code_rcp(f0.y, scale, rscale)) & 0xFFu) << 8) |
                                ((static_cast<uint32_t>(quant_code_rcp(f1.x, scale, rscale)) & 0xFFu) << 16) |
                                ((static_cast<uint32_t>(quant_code_rcp(f1.y, scale, rscale)) & 0xFFu) << 24);
              }
            }
            const int gg = 4 * hh + g;
            *reinterpret_cast<uint4*>(q8 + t * 128 + ((gg ^ (t & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->q_ready[x]);
      }

      const int ks_base = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[b] : 0;
      const int ks_end = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[b + 1] : 0;
      const float kNegInf = -__int_as_float(0x7f800000);
      const __half ninf = __ushort_as_half(0xFC00);
      float m_used = kNegInf;
      float l = hh == 0 ? 1.f : 0.f;  // the reference's l starts at 1: carried by one half
      const int coff = seqlen_k - seqlen_q;
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
        const uint32_t tS = tbase + lane_off + col_s(x, slot);
        uint32_t sv[32];
        tmem_ld32(tS + 32 * hh, sv);
        tmem_wait_ld();
        __half2 hv[16];
        if (kind == 0) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            hv[i] = __floats2half2_rn(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
        } else {
          const float c = -12582912.0f * ss;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            hv[i] = __floats2half2_rn(fmaf(__uint_as_float(sv[2 * i] + 0x4B400000u), ss, c),
                                      fmaf(__uint_as_float(sv[2 * i + 1] + 0x4B400000u), ss, c));
        }
        int lim = seqlen_k - j * kKeys;
        if (a.causal) lim = min(lim, row + coff + 1 - j * kKeys);
        lim -= 32 * hh;
        if (lim < 32) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __half lo = (2 * i < lim) ? __low2half(hv[i]) : ninf;
            const __half hi = (2 * i + 1 < lim) ? __high2half(hv[i]) : ninf;
            hv[i] = __halves2half2(lo, hi);
          }
        }
        __half2 mt[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mt[i] = __hmax2(hv[i], hv[8 + i]);
#pragma unroll
        for (int w = 4; w >= 1; w >>= 1) {
#pragma unroll
          for (int i = 0; i < w; ++i) mt[i] = __hmax2(mt[i], mt[i + w]);
        }
        // Partial row max (an fp16 value) to the partner thread, the partner's back.
        const __half pm16 = __hmax(__low2half(mt[0]), __high2half(mt[0]));
        xchg_put(&bars->xmax[x][slot][hh][t], static_cast<uint32_t>(j + 1), __half_as_ushort(pm16));
        uint32_t other16;
        ok = __all_sync(0xffffffffu, xchg_get(&bars->xmax[x][slot][1 - hh][t], static_cast<uint32_t>(j + 1), other16,
                                              a.err, kErrTimeoutExchange));
        if (!ok) break;
        const float mx = fmaxf(__half2float(pm16), __half2float(__ushort_as_half(static_cast<unsigned short>(other16))));
        float o_scale = 1.f;
        if (mx != kNegInf && mx > m_used + a.rescale_threshold) {
          const float alpha = ex2_approx(m_used - mx);  // 0 when m_used == -inf
          if (m_used != kNegInf) o_scale = alpha;
          l *= alpha;
          m_used = mx;
        }
        uint32_t p[16];
        if (mx != kNegInf) {
          const uint64_t negm = f32x2_pack(-m_used, -m_used);
          uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 f = __half22float2(hv[i]);
            const float2 d = f32x2_unpack(f32x2_add(f32x2_pack(f.x, f.y), negm));
            const float e0 = ex2_approx(d.x), e1 = ex2_approx(d.y);
            const __half2 ph = __floats2half2_rn(e0, e1);
            if (i & 1)
              acc1 = f32x2_add(acc1, f32x2_pack(e0, e1));
            else
              acc0 = f32x2_add(acc0, f32x2_pack(e0, e1));
            p[i] = *reinterpret_cast<const uint32_t*>(&ph);
          }
          const float2 a0 = f32x2_unpack(acc0), a1 = f32x2_unpack(acc1);
          l += (a0.x + a0.y) + (a1.x + a1.y);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) p[i] = 0u;
        }
        if (__any_sync(0xffffffffu, o_scale != 1.f)) {
          // O must not move while PV_X(j-1) may still accumulate into it.
          const int jj = j - 1;
          ok = __all_sync(0xffffffffu,
                          mbar_wait_spin(&bars->pv_done[x][jj & 1], (jj >> 1) & 1, a.err, kErrTimeoutPV));
          if (!ok) break;
          tc_fence_after();
          const uint32_t tO = tbase + lane_off + col_o(x) + 64 * hh;
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            uint32_t o[32];
            tmem_ld32(tO + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * o_scale);
            tmem_st32(tO + c, o);
          }
        }
        tmem_st16(tS + 16 * hh, p);  // P: keys [32hh, 32hh+32) -> columns [16hh, 16hh+16)
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->p_ready[x][slot]);
      }
      // Combine the two halves' row sums, then each thread stores its 64 output dims.
      xchg_put64(&bars->xsum[x][hh][t], __float_as_uint(l));
      uint32_t l_other = 0;
      if (ok) ok = __all_sync(0xffffffffu, xchg_get64(&bars->xsum[x][1 - hh][t], l_other, a.err, kErrTimeoutExchange));
      const float l_row = l + __uint_as_float(l_other);
      __half* orow = a.out + (static_cast<int64_t>(q_start) + row) * a.o_st + static_cast<int64_t>(me.hq) * a.o_sh +
                     64 * hh;
      if (ok && me.nb > 0) {
        const int jj = me.nb - 1;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->pv_done[x][jj & 1], (jj >> 1) & 1, a.err, kErrTimeoutPV));
        tc_fence_after();
      }
      store_o_row<64>(tbase + lane_off + col_o(x) + 64 * hh, me.nb > 0, l_row, orow, row_ok && ok);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace split

int launch_attn_split(const CUtensorMap& q, const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v,
                       const AttnArgs& a, int batch, int max_seqlen_q, cudaStream_t stream) {
  using namespace split;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(tilemix_attn_fwd_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  tilemix_attn_fwd_split_kernel<<<grid, kThreads, kSmemBytes, stream>>>(q, k16, k8, v, a);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace tilemix
