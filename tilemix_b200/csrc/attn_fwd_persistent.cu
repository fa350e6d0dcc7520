// Persistent, route-compacted TileMix attention forward for B200 (sm_100a).
// Fast path for head_dim 128, block_m 128 with Q quantised in the kernel
// (BLKQ = 128) or FP16-only routing: the shapes of the model integration and
// of tilemix_attention_with_quant.
//
// Semantics follow attn_fwd (attention/triton/tilemix.py:503-951): the same
// routing of every 64-key tile by its map bit, the same FP16 / INT8 score
// rounding chains, the same masking, online softmax and normalisation. Two
// mechanisms differ and change results only at the level of fp16 rounding of
// P: (1) keys are visited in route order -- the FP16-routed tiles of a row in
// ascending order, then its INT8-routed tiles -- so that two tiles of the same
// route form one 128-key tensor-core step (the reference walks them in key
// order); (2) the optional rescale threshold (see attn_common.cuh).
//
// Work items are (sequence, Q head, 128-row query block), listed grouped by
// (sequence, KV head), longest query blocks first. Each CTA (grid = #SMs) claims
// the next item with a global atomic, so the items in flight at any moment are
// one contiguous window of the list and share K/V in L2.
//
// Roles (16 warps, four warpgroups):
//   WG0 (warps 0-3)   softmax of key tile 0 of every step (S columns 0..63)
//   WG1 (warps 4-7)   softmax of key tile 1 of every step (S columns 64..127);
//                     the two threads of a row exchange their partial maxima
//                     through shared memory so both use one reference max
//   WG2 (warps 8-11)  per item: scale Q in shared memory and quantise it to the
//                     INT8 operand (one BLKQ=128 block); epilogue O / l -> fp16
//   warp 12           TMA producer for K (only in the routed format)
//   warp 13           MMA issuer (event loop): S = Q K^T (kind::f16 / kind::i8,
//                     N = 128 or 64) into one of three TMEM score slots,
//                     O += P V (kind::f16, P read from TMEM)
//   warp 14           TMA producer for V
//   warp 15           TMA producer for Q (two buffers: the next item's Q is
//                     loaded and transformed while the current item runs)
// TMEM: O [0,128), score/P slots [128,256), [256,384), [384,512).
#include "attn_common.cuh"
#include "tilemix_b200.h"

namespace tilemix {
namespace persistent {

constexpr int kD = 128;
constexpr int kRows = 128;
constexpr int kSlots = 3;    // S/P slots in TMEM
constexpr int kKStages = 2;  // K ring (one stage = one step of up to two key tiles)
constexpr int kVStages = 4;  // V ring (one stage = one key tile; two steps deep)
constexpr int kThreads = 512;
// Register split (setmaxnreg): 512 threads launch with 128 each (65536); then
// softmax WGs 144, WG2 128 (unchanged), WG3 96: 2*128*144 + 128*128 + 128*96 = 65536.
constexpr uint32_t kRegSoftmax = 144, kRegWG2 = 128, kRegWG3 = 96;
constexpr uint32_t kTmemCols = 512;
constexpr int kItemRing = 8;  // work-item indices published by the scheduler to the other roles
constexpr int kItemConsumers = 3 + 3 * 128;  // V producer, Q producer, MMA issuer, every WG0/WG1/WG2 thread

constexpr uint32_t kQ16Bytes = kRows * kD * 2;       // 32 KB (two 64-column boxes)
constexpr uint32_t kQ8Bytes = kRows * kD;            // 16 KB
constexpr uint32_t kKStepBytes = 2 * kKeys * kD * 2;  // 32 KB: [t0 d0-63][t1 d0-63][t0 d64-127][t1 d64-127]
constexpr uint32_t kVTileBytes = kKeys * kD * 2;       // 16 KB: [d0-63][d64-127]
// The FP16 Q operand is double-buffered by item; the INT8 Q operand is single:
// an item runs its FP16-routed steps first, so the next item's INT8 operand is
// written while those run.
constexpr uint32_t kOffQ16 = 0;
constexpr uint32_t kOffQ8 = kOffQ16 + 2 * kQ16Bytes;
constexpr uint32_t kOffK = kOffQ8 + kQ8Bytes;
constexpr uint32_t kOffV = kOffK + kKStages * kKStepBytes;
constexpr uint32_t kOffMisc = kOffV + kVStages * kVTileBytes;

struct Misc {
  uint64_t item_full[kItemRing], item_empty[kItemRing];
  int item_q[kItemRing];
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t q_full[2], q_empty[2];  // per FP16 Q buffer (item parity)
  uint64_t q_ready[2];  // per FP16 Q buffer: WG2 -> MMA issuer / softmax (also publishes sq)
  uint64_t q8_empty;    // INT8 Q operand free (last S of an item issued and done)
  uint64_t q8_ready;    // INT8 Q operand of the next item written (WG2 -> MMA issuer)
  uint64_t s_full[kSlots], p_ready[kSlots], pv_done[kSlots];
  uint64_t o_full, o_free;
  uint64_t l_ready[2];  // by item parity: softmax -> WG2 (row sums in lsum)
  uint64_t mma_done;
  uint32_t tmem_base;
  float sq[2];             // fp16 Q block scale (as float) per item parity
  float red[4];            // Q absmax partials of WG2
  float xmax[2][2][kRows]; // [wg][step parity][row] partial tile maxima
  float lsum[2][2][kRows]; // [item parity][wg][row] partial row sums
};
constexpr uint32_t kSmemBytes = kOffMisc + sizeof(Misc) + 1024;

// ---------------------------------------------------------------------------
// Work items and steps
// ---------------------------------------------------------------------------
struct Item {
  int b, hq, hk, mtile;
  int q_start, seqlen_q, k_start, seqlen_k;
  int nb;  // visited 64-key tiles
  uint64_t bits;
  bool valid;  // query block inside the sequence
};

__device__ __forceinline__ Item decode_item(const AttnArgs& a, int idx, int m_tiles) {
  // idx -> (b, hk, mtile desc, head within group)
  Item it;
  const int per_hk = m_tiles * a.group;
  const int per_b = a.HK * per_hk;
  it.b = idx / per_b;
  int r = idx - it.b * per_b;
  it.hk = r / per_hk;
  r -= it.hk * per_hk;
  it.mtile = m_tiles - 1 - r / a.group;
  it.hq = it.hk * a.group + (r % a.group);
  it.q_start = a.cu_q[it.b];
  it.seqlen_q = a.cu_q[it.b + 1] - it.q_start;
  it.k_start = a.cu_k[it.b];
  it.seqlen_k = a.cu_k[it.b + 1] - it.k_start;
  it.valid = it.mtile * kRows < it.seqlen_q;
  it.nb = it.valid ? visited_key_tiles(it.mtile * kRows, kRows, it.seqlen_q, it.seqlen_k, a.causal) : 0;
  it.bits = 0;
  if (it.valid && a.mode == TM_ROUTE_MIXED) {
    const int m_blocks = (it.seqlen_q + kRows - 1) / kRows;
    it.bits = a.bitmask[static_cast<int64_t>(it.hk) * m_blocks + it.mtile];
  }
  return it;
}

// Walks the key tiles of an item in route order: FP16-routed tiles ascending,
// then INT8-routed tiles ascending, two per step.
struct StepIter {
  int cur[2];  // next candidate tile per kind
  int phase;   // 0: FP16 tiles, 1: INT8 tiles, 2: done
  __device__ __forceinline__ int next_of(const AttnArgs& a, const Item& it, int kind, int from) const {
    int j = from;
    while (j < it.nb && route_kind(a.mode, it.bits, j, a.block_n_mask) != kind) ++j;
    return j;
  }
  __device__ __forceinline__ void init(const AttnArgs& a, const Item& it) {
    cur[0] = next_of(a, it, 0, 0);
    cur[1] = next_of(a, it, 1, 0);
    phase = cur[0] < it.nb ? 0 : (cur[1] < it.nb ? 1 : 2);
  }
  // Returns false when the item has no more steps; else kind and tiles (t1 = -1 if single).
  __device__ __forceinline__ bool next(const AttnArgs& a, const Item& it, int& kind, int& t0, int& t1,
                                       bool& last) {
    if (phase == 2) return false;
    kind = phase;
    t0 = cur[kind];
    const int n1 = next_of(a, it, kind, t0 + 1);
    t1 = n1 < it.nb ? n1 : -1;
    cur[kind] = (t1 >= 0) ? next_of(a, it, kind, t1 + 1) : it.nb;
    if (cur[kind] >= it.nb) phase = (kind == 0 && cur[1] < it.nb) ? 1 : 2;
    last = (phase == 2);
    return true;
  }
};

__device__ __forceinline__ uint32_t col_slot(int s) { return 128u + static_cast<uint32_t>(s) * 128u; }

// Scheduler counters used when the caller passes no workspace: [0] next item,
// [1] CTAs finished fetching. The last CTA to finish puts both back to zero.
__device__ int g_sched_counters[2];

// Consumer side of the item ring: the index of the n-th item of this CTA, or -1
// once the work is exhausted (-2 on a timeout).
__device__ __forceinline__ int ring_next(Misc* ms, int& n, int* err) {
  const int e = n % kItemRing;
  if (!mbar_wait(&ms->item_full[e], (n / kItemRing) & 1, err, kErrTimeoutQ)) return -2;
  const int idx = *reinterpret_cast<volatile int*>(&ms->item_q[e]);
  mbar_arrive(&ms->item_empty[e]);
  ++n;
  return idx;
}

// Non-blocking variant for the MMA issuer's event loop: false if the n-th item
// is not published yet.
__device__ __forceinline__ bool ring_try(Misc* ms, int& n, int& idx) {
  const int e = n % kItemRing;
  if (!mbar_test(&ms->item_full[e], (n / kItemRing) & 1)) return false;
  idx = *reinterpret_cast<volatile int*>(&ms->item_q[e]);
  mbar_arrive(&ms->item_empty[e]);
  ++n;
  return true;
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    tilemix_attn_fwd_persistent_kernel(const __grid_constant__ CUtensorMap tm_q,
                                       const __grid_constant__ CUtensorMap tm_k16,
                                       const __grid_constant__ CUtensorMap tm_k8,
                                       const __grid_constant__ CUtensorMap tm_v, const AttnArgs a, int n_items,
                                       int m_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Misc* ms = reinterpret_cast<Misc*>(smem + kOffMisc);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int e = 0; e < kItemRing; ++e) {
      mbar_init(&ms->item_full[e], 1);
      mbar_init(&ms->item_empty[e], kItemConsumers);
    }
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&ms->k_full[s], 1);
      mbar_init(&ms->k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&ms->v_full[s], 1);
      mbar_init(&ms->v_empty[s], 1);
    }
    for (int bq = 0; bq < 2; ++bq) {
      mbar_init(&ms->q_full[bq], 1);
      mbar_init(&ms->q_empty[bq], 1);
    }
    mbar_init(&ms->q8_empty, 1);
    mbar_init(&ms->q8_ready, kRows);
    mbar_init(&ms->q_ready[0], kRows);
    mbar_init(&ms->q_ready[1], kRows);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&ms->s_full[s], 1);
      mbar_init(&ms->p_ready[s], 2 * kRows);
      mbar_init(&ms->pv_done[s], 1);
    }
    mbar_init(&ms->o_full, 1);
    mbar_init(&ms->o_free, kRows);
    mbar_init(&ms->l_ready[0], 2 * kRows);
    mbar_init(&ms->l_ready[1], 2 * kRows);
    mbar_init(&ms->mma_done, 1);
    fence_mbarrier_init();
  }
  if (warp == 13) {
    tmem_alloc(&ms->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ms->tmem_base;

  if (warp >= 12) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegWG3));  // producers + MMA issuer
  if (warp == 12) {
    // ------------------------------------------------------------ Q / K producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k16);
      if (a.mode != TM_ROUTE_FP16) prefetch_tmap(&tm_k8);
      bool ok = true;
      int kq = 0;
      int* ctr = a.sched != nullptr ? a.sched : g_sched_counters;
      int n_f = 0;
      while (ok) {
        // Dynamic scheduler: claim the next item and publish it to the other roles.
        const int e = n_f % kItemRing;
        if (n_f >= kItemRing)
          ok = mbar_wait(&ms->item_empty[e], ((n_f - kItemRing) / kItemRing) & 1, a.err, kErrTimeoutEmpty);
        if (!ok) break;
        int idx = atomicAdd(&ctr[0], 1);
        if (idx >= n_items) idx = -1;
        *reinterpret_cast<volatile int*>(&ms->item_q[e]) = idx;
        mbar_arrive(&ms->item_full[e]);
        ++n_f;
        if (idx < 0) break;
        const Item it = decode_item(a, idx, m_tiles);
        if (it.nb == 0) continue;
        StepIter st;
        st.init(a, it);
        int kind, t0, t1;
        bool last;
        while (st.next(a, it, kind, t0, t1, last)) {
          const int s = kq % kKStages;
          if (kq >= kKStages) ok = mbar_wait(&ms->k_empty[s], ((kq - kKStages) / kKStages) & 1, a.err, kErrTimeoutEmpty);
          if (!ok) break;
          const int ntile = t1 >= 0 ? 2 : 1;
          uint8_t* kst = smem + kOffK + s * kKStepBytes;
          if (kind == 0) {
            mbar_arrive_expect_tx(&ms->k_full[s], ntile * kKeys * kD * 2);
            for (int tt = 0; tt < ntile; ++tt) {
              const int tok = it.k_start + (tt == 0 ? t0 : t1) * kKeys;
              tma_load_3d(kst + tt * 8192, &tm_k16, &ms->k_full[s], 0, it.hk, tok);
              tma_load_3d(kst + 16384 + tt * 8192, &tm_k16, &ms->k_full[s], 64, it.hk, tok);
            }
          } else {
            mbar_arrive_expect_tx(&ms->k_full[s], ntile * kKeys * kD);
            for (int tt = 0; tt < ntile; ++tt) {
              const int tok = it.k_start + (tt == 0 ? t0 : t1) * kKeys;
              tma_load_3d(kst + tt * 8192, &tm_k8, &ms->k_full[s], 0, it.hk, tok);
            }
          }
          ++kq;
        }
      }
      if (ok) {
        __threadfence();
        if (atomicAdd(&ctr[1], 1) == static_cast<int>(gridDim.x) - 1) {
          // every CTA has fetched its last index: leave the counters at zero
          atomicExch(&ctr[0], 0);
          atomicExch(&ctr[1], 0);
        }
      }
    }
  } else if (warp == 14) {
    // ------------------------------------------------------------ V producer
    if (lane == 0) {
      prefetch_tmap(&tm_v);
      bool ok = true;
      int vq = 0, n_c = 0;
      while (ok) {
        const int idx = ring_next(ms, n_c, a.err);
        if (idx < 0) break;
        const Item it = decode_item(a, idx, m_tiles);
        if (it.nb == 0) continue;
        StepIter st;
        st.init(a, it);
        int kind, t0, t1;
        bool last;
        while (st.next(a, it, kind, t0, t1, last)) {
          for (int tt = 0; tt < 2 && ok; ++tt) {
            const int tj = tt == 0 ? t0 : t1;
            if (tj < 0) continue;
            const int s = vq % kVStages;
            if (vq >= kVStages)
              ok = mbar_wait(&ms->v_empty[s], ((vq - kVStages) / kVStages) & 1, a.err, kErrTimeoutEmpty);
            if (!ok) break;
            uint8_t* vst = smem + kOffV + s * kVTileBytes;
            mbar_arrive_expect_tx(&ms->v_full[s], kVTileBytes);
            const int tok = it.k_start + tj * kKeys;
            tma_load_3d(vst, &tm_v, &ms->v_full[s], 0, it.hk, tok);
            tma_load_3d(vst + 8192, &tm_v, &ms->v_full[s], 64, it.hk, tok);
            ++vq;
          }
        }
      }
    }
  } else if (warp == 15) {
    // ------------------------------------------------------------ Q producer (double-buffered)
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      bool ok = true;
      int qi = 0, n_c = 0;
      while (ok) {
        const int idx = ring_next(ms, n_c, a.err);
        if (idx < 0) break;
        const Item it = decode_item(a, idx, m_tiles);
        if (it.nb == 0) continue;
        const int bq = qi & 1;
        if (qi >= 2) ok = mbar_wait(&ms->q_empty[bq], ((qi - 2) >> 1) & 1, a.err, kErrTimeoutEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(&ms->q_full[bq], kQ16Bytes);
        for (int box = 0; box < 2; ++box)
          tma_load_3d(smem + kOffQ16 + bq * kQ16Bytes + box * (kQ16Bytes / 2), &tm_q, &ms->q_full[bq], box * 64,
                      it.hq, it.q_start + it.mtile * kRows);
        ++qi;
      }
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ MMA issuer
    // Fixed software pipeline over the CTA's global step sequence:
    //   S(0), S(1), then for every step g:  PV(g), S(g+2)
    // so the scores of the next step are always ready when the softmax reaches
    // it; every wait blocks on exactly one barrier.
    if (lane == 0) {
      const uint32_t idesc16_n128 = make_idesc(1, 0, 0, 0, 128, 128);
      const uint32_t idesc16_n64 = make_idesc(1, 0, 0, 0, 128, 64);
      const uint32_t idesc8_n128 = make_idesc(2, 1, 0, 0, 128, 128);
      const uint32_t idesc8_n64 = make_idesc(2, 1, 0, 0, 128, 64);
      const uint32_t idesc_pv = make_idesc(1, 0, 0, 1, 128, kD);
      // Descriptor bases; the start-address field is addr >> 4 in the low 14
      // bits, so an operand offset is applied by adding (offset >> 4).
      const uint64_t dq16 = make_sdesc(smem_u32(smem + kOffQ16), 16, 1024, 2);
      const uint64_t dq8 = make_sdesc(smem_u32(smem + kOffQ8), 16, 1024, 2);
      const uint64_t dk = make_sdesc(smem_u32(smem + kOffK), 16, 1024, 2);
      const uint64_t dv = make_sdesc(smem_u32(smem + kOffV), 8192, 1024, 2);
      struct StepRec {
        int kind, t1, qbuf;
        bool first, last;
      };
      StepRec rq[4];
      int rq_head = 0, rq_tail = 0;
      // step generator (consumes the item ring)
      Item gen_it;
      StepIter gen_st;
      bool gen_open = false, gen_end = false, gen_first = false;
      int n_c = 0, qi_gen = 0;
      bool ok = true;
      auto gen_next = [&](StepRec& r) -> bool {
        while (!gen_end) {
          if (!gen_open) {
            const int idx = ring_next(ms, n_c, a.err);
            if (idx < 0) {
              gen_end = true;
              if (idx == -2) ok = false;
              return false;
            }
            gen_it = decode_item(a, idx, m_tiles);
            if (gen_it.nb == 0) continue;
            gen_st.init(a, gen_it);
            gen_open = true;
            gen_first = true;
          }
          int kind, t0, t1;
          bool last;
          if (gen_st.next(a, gen_it, kind, t0, t1, last)) {
            r.kind = kind;
            r.t1 = t1;
            r.qbuf = qi_gen & 1;
            r.first = gen_first;
            r.last = last;
            gen_first = false;
            if (last) {
              gen_open = false;
              ++qi_gen;
            }
            return true;
          }
          gen_open = false;
        }
        return false;
      };
      int g_s = 0, g_p = 0, kq = 0, vq = 0, qi_s = 0, oi = 0;
      auto issue_s = [&](const StepRec& r) {
        const int slot = g_s % kSlots;
        const int ks = kq % kKStages;
        ok = ok && mbar_wait(&ms->k_full[ks], (kq / kKStages) & 1, a.err, kErrTimeoutFull);
        if (ok && g_s >= kSlots)
          ok = mbar_wait(&ms->pv_done[slot], ((g_s - kSlots) / kSlots) & 1, a.err, kErrTimeoutPV);
        if (ok && r.first) ok = mbar_wait(&ms->q_ready[qi_s & 1], (qi_s >> 1) & 1, a.err, kErrTimeoutQ);
        // INT8 steps need the item's INT8 operand; so does every item's last
        // step, which keeps q8_empty from running ahead of WG2's writes.
        if (ok && a.mode != TM_ROUTE_FP16 && (r.kind == 1 || r.last))
          ok = mbar_wait(&ms->q8_ready, qi_s & 1, a.err, kErrTimeoutQ);
        if (!ok) return;
        tc_fence_after();
        const uint32_t d = tbase + col_slot(slot);
        const uint64_t bk = dk + ((ks * kKStepBytes) >> 4);
        const bool two = r.t1 >= 0;
        if (r.kind == 0) {
          const uint64_t aq = dq16 + ((r.qbuf * kQ16Bytes) >> 4);
          const uint32_t idesc = two ? idesc16_n128 : idesc16_n64;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off_a = (kk >> 2) * (kQ16Bytes / 2) + (kk & 3) * 32;
            const uint32_t off_b = (kk >> 2) * 16384 + (kk & 3) * 32;
            mma_f16_ss(d, aq + (off_a >> 4), bk + (off_b >> 4), idesc, kk > 0 ? 1u : 0u);
          }
        } else {
          const uint32_t idesc = two ? idesc8_n128 : idesc8_n64;
#pragma unroll
          for (int kk = 0; kk < kD / 32; ++kk) mma_i8_ss(d, dq8 + (kk * 2), bk + (kk * 2), idesc, kk > 0 ? 1u : 0u);
        }
        tc_commit(&ms->s_full[slot]);
        tc_commit(&ms->k_empty[ks]);
        if (r.last) {
          tc_commit(&ms->q_empty[qi_s & 1]);  // Q buffers reusable once this item's last S is done
          tc_commit(&ms->q8_empty);
          ++qi_s;
        }
        ++kq;
        ++g_s;
      };
      auto issue_pv = [&](const StepRec& r) {
        const int slot = g_p % kSlots;
        const int ntile = r.t1 >= 0 ? 2 : 1;
        ok = ok && mbar_wait(&ms->p_ready[slot], (g_p / kSlots) & 1, a.err, kErrTimeoutP);
        for (int tt = 0; tt < ntile && ok; ++tt)
          ok = mbar_wait(&ms->v_full[(vq + tt) % kVStages], ((vq + tt) / kVStages) & 1, a.err, kErrTimeoutFull);
        if (ok && r.first && oi > 0) ok = mbar_wait(&ms->o_free, (oi - 1) & 1, a.err, kErrTimeoutPV);
        if (!ok) return;
        tc_fence_after();
        const uint32_t pcol = tbase + col_slot(slot);
        for (int tt = 0; tt < ntile; ++tt) {
          const uint64_t bv = dv + ((((vq + tt) % kVStages) * kVTileBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)
            mma_f16_ts(tbase, pcol + tt * 64 + kk * 8, bv + ((kk * 2048) >> 4), idesc_pv,
                       (!r.first || tt > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&ms->pv_done[slot]);
        for (int tt = 0; tt < ntile; ++tt) tc_commit(&ms->v_empty[(vq + tt) % kVStages]);
        if (r.last) {
          tc_commit(&ms->o_full);
          ++oi;
        }
        vq += ntile;
        ++g_p;
      };
      for (int i = 0; i < 2 && ok; ++i) {
        StepRec r;
        if (!gen_next(r)) break;
        issue_s(r);
        rq[rq_tail % 4] = r;
        ++rq_tail;
      }
      // PV(g) before S(g+2): a first step of a new item waits for that item's Q
      // transform, which WG2 does after the epilogue of the item two back; that
      // epilogue needs PV(g) already queued.
      while (ok && rq_head < rq_tail) {
        issue_pv(rq[rq_head % 4]);
        ++rq_head;
        if (!ok) break;
        StepRec r;
        if (gen_next(r) && ok) {
          issue_s(r);
          rq[rq_tail % 4] = r;
          ++rq_tail;
        }
      }
      tc_commit(&ms->mma_done);
      mbar_wait(&ms->mma_done, 0, a.err, kErrTimeoutDrain);
    }
  }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegSoftmax));
    // ------------------------------------------------------------ softmax WG0 / WG1
    const int w = warp >> 2;          // which key tile of the step
    const int t = threadIdx.x & 127;  // row == TMEM lane
    const int q4 = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const float kNegInf = -__int_as_float(0x7f800000);
    bool ok = true;
    int g = 0, ii = 0, n_c = 0;
    while (ok) {
      const int idx = ring_next(ms, n_c, a.err);
      if (idx < 0) break;
      const Item it = decode_item(a, idx, m_tiles);
      if (it.nb == 0) continue;
      const int row = it.mtile * kRows + t;
      const int coff = it.seqlen_k - it.seqlen_q;
      const int ks_base = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[it.b] : 0;
      const int ks_end = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[it.b + 1] : 0;
      ok = __all_sync(0xffffffffu, mbar_wait(&ms->q_ready[ii & 1], (ii >> 1) & 1, a.err, kErrTimeoutQ));
      if (!ok) break;
      const __half sq16 = __float2half_rn(ms->sq[ii & 1]);
      float m_used = kNegInf;
      float l = (w == 0) ? 1.f : 0.f;  // the two partial sums start at the reference's l = 1
      StepIter st;
      st.init(a, it);
      int kind, t0, t1;
      bool last;
      bool first_step = true;
      while (ok && st.next(a, it, kind, t0, t1, last)) {
        const int slot = g % kSlots;
        const int my = (w == 0) ? t0 : t1;  // -1: no tile for this warpgroup in this step
        float ss = 1.f;
        if (my >= 0 && kind == 1) {
          __half sk16 = __float2half_rn(1.f);
          if (ks_end > ks_base) {
            const int idx2 = min(ks_base + (my * kKeys) / a.blkk, ks_end - 1);
            sk16 = a.k_scale[static_cast<int64_t>(idx2) * a.HK + it.hk];
          }
          ss = int8_score_scale(sq16, sk16, a.qk_scale);
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&ms->s_full[slot], (g / kSlots) & 1, a.err, kErrTimeoutScores));
        if (!ok) break;
        tc_fence_after();
        // ---- scores of my tile -> fp16, masked, partial max
        __half2 h[32];
        float mx = kNegInf;
        if (my >= 0) {
          uint32_t s0[32], s1[32];
          const uint32_t taddr = tbase + lane_off + col_slot(slot) + w * 64;
          tmem_ld32(taddr, s0);
          tmem_ld32(taddr + 32, s1);
          tmem_wait_ld();
          if (kind == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              h[i] = __floats2half2_rn(__uint_as_float(s0[2 * i]), __uint_as_float(s0[2 * i + 1]));
              h[16 + i] = __floats2half2_rn(__uint_as_float(s1[2 * i]), __uint_as_float(s1[2 * i + 1]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              h[i] = __floats2half2_rn(i2f_exact(s0[2 * i]) * ss, i2f_exact(s0[2 * i + 1]) * ss);
              h[16 + i] = __floats2half2_rn(i2f_exact(s1[2 * i]) * ss, i2f_exact(s1[2 * i + 1]) * ss);
            }
          }
          int lim = it.seqlen_k - my * kKeys;
          if (a.causal) lim = min(lim, row + coff + 1 - my * kKeys);
          if (lim < kKeys) {
            const __half ninf = __ushort_as_half(0xFC00);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const __half lo = (2 * i < lim) ? __low2half(h[i]) : ninf;
              const __half hi = (2 * i + 1 < lim) ? __high2half(h[i]) : ninf;
              h[i] = __halves2half2(lo, hi);
            }
          }
          __half2 mt[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) mt[i] = __hmax2(h[i], h[16 + i]);
#pragma unroll
          for (int wd = 8; wd >= 1; wd >>= 1) {
#pragma unroll
            for (int i = 0; i < wd; ++i) mt[i] = __hmax2(mt[i], mt[i + wd]);
          }
          mx = fmaxf(__low2float(mt[0]), __high2float(mt[0]));
        }
        // ---- exchange partial maxima with the other warpgroup's thread of this row
        ms->xmax[w][g & 1][t] = mx;
        asm volatile("bar.sync %0, 64;" ::"r"(1 + q4) : "memory");
        const float mx_all = fmaxf(mx, ms->xmax[w ^ 1][g & 1][t]);
        const bool has = mx_all != kNegInf;
        float o_scale = 1.f;
        bool need_rescale = false;
        if (has && mx_all > m_used + a.rescale_threshold) {
          const float alpha = ex2_approx(m_used - mx_all);
          need_rescale = (m_used != kNegInf) && !first_step;
          o_scale = alpha;
          l *= alpha;
          m_used = mx_all;
        }
        uint32_t p[32];
        if (my >= 0 && has) {
          const uint64_t negm = f32x2_pack(-m_used, -m_used);
          uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float2 f = __half22float2(h[i]);
            const float2 dd = f32x2_unpack(f32x2_add(f32x2_pack(f.x, f.y), negm));
            const float e0 = ex2_approx(dd.x), e1 = ex2_approx(dd.y);
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
          for (int i = 0; i < 32; ++i) p[i] = 0u;
        }
        if (__any_sync(0xffffffffu, need_rescale)) {
          // O holds the PVs of this item's earlier steps; wait for the last one.
          const int gp = g - 1;
          ok = __all_sync(0xffffffffu, mbar_wait(&ms->pv_done[gp % kSlots], (gp / kSlots) & 1, a.err, kErrTimeoutPV));
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            uint32_t o[32];
            const uint32_t oaddr = tbase + lane_off + w * 64 + c;
            tmem_ld32(oaddr, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * o_scale);
            tmem_st32(oaddr, o);
          }
        }
        if (my >= 0) tmem_st32(tbase + lane_off + col_slot(slot) + w * 64, p);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&ms->p_ready[slot]);
        first_step = false;
        ++g;
      }
      if (!ok) break;
      ms->lsum[ii & 1][w][t] = l;
      mbar_arrive(&ms->l_ready[ii & 1]);
      ++ii;
    }
  } else {
    // ------------------------------------------------------------ Q transform + epilogue (WG2)
    const int t = threadIdx.x & 127;
    const int q4 = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    bool ok = true;
    int qi = 0, oi = 0;
    Item prev;
    bool have_prev = false;
    auto epilogue = [&](const Item& it, int item_no) -> bool {
      const int row = it.mtile * kRows + t;
      __half* orow = a.out + (static_cast<int64_t>(it.q_start) + row) * a.o_st + static_cast<int64_t>(it.hq) * a.o_sh;
      const bool row_ok = row < it.seqlen_q;
      bool okk = __all_sync(0xffffffffu, mbar_wait(&ms->o_full, oi & 1, a.err, kErrTimeoutPV));
      okk = okk && __all_sync(0xffffffffu,
                              mbar_wait(&ms->l_ready[item_no & 1], (item_no >> 1) & 1, a.err, kErrTimeoutPV));
      tc_fence_after();
      const float l = ms->lsum[item_no & 1][0][t] + ms->lsum[item_no & 1][1][t];
      const float rl = __frcp_rn(l);
      // O / l with one residual correction per element (Markstein's method:
      // q0 = a*r, q = q0 + (a - q0*l)*r gives the correctly rounded quotient).
      uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tbase + lane_off + c * 32, o);
        tmem_wait_ld();
        uint32_t wv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a0 = __uint_as_float(o[2 * i]), a1 = __uint_as_float(o[2 * i + 1]);
          const float q0 = a0 * rl, q1 = a1 * rl;
          wv[i] = pack_half2_rn(fmaf(fmaf(-q0, l, a0), rl, q0), fmaf(fmaf(-q1, l, a1), rl, q1));
        }
        if (row_ok && okk) {
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[c * 4 + v] = make_uint4(wv[4 * v], wv[4 * v + 1], wv[4 * v + 2], wv[4 * v + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&ms->o_free);  // O may now be overwritten by the next item's first PV
      ++oi;
      return okk;
    };
    int n_c = 0;
    while (ok) {
      const int idx = ring_next(ms, n_c, a.err);
      if (idx < 0) break;
      const Item it = decode_item(a, idx, m_tiles);
      if (!it.valid) continue;
      if (it.nb == 0) {
        // no visited keys: the reference writes zeros (acc = 0, l = 1)
        const int row = it.mtile * kRows + t;
        if (row < it.seqlen_q) {
          uint4* dst = reinterpret_cast<uint4*>(a.out + (static_cast<int64_t>(it.q_start) + row) * a.o_st +
                                                static_cast<int64_t>(it.hq) * a.o_sh);
          for (int v = 0; v < kD / 8; ++v) dst[v] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      // ---- Q transform for this item
      ok = __all_sync(0xffffffffu, mbar_wait(&ms->q_full[qi & 1], (qi >> 1) & 1, a.err, kErrTimeoutQ));
      if (!ok) break;
      {
        const int row = it.mtile * kRows + t;
        const bool row_ok = row < it.seqlen_q;
        uint8_t* q16 = smem + kOffQ16 + (qi & 1) * kQ16Bytes;
        auto qchunk = [&](int c) -> uint4* {
          return reinterpret_cast<uint4*>(q16 + (c >> 3) * (kQ16Bytes / 2) + t * 128 + (((c & 7) ^ (t & 7)) << 4));
        };
        // pass 1: absmax of the raw row (the BLKQ=128 block is this item's 128 rows)
        float amax = 0.f;
        if (row_ok) {
#pragma unroll 4
          for (int c = 0; c < 16; ++c) {
            const uint4 u = *qchunk(c);
            const __half2* hh = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(hh[e]);
              amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
            }
          }
        }
        float sqv = 1.f;
        float scale = 1.f;
        if (a.mode != TM_ROUTE_FP16) {
          float m = amax;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) ms->red[q4] = m;
          asm volatile("bar.sync 5, 128;" ::: "memory");
          m = fmaxf(fmaxf(ms->red[0], ms->red[1]), fmaxf(ms->red[2], ms->red[3]));
          asm volatile("bar.sync 5, 128;" ::: "memory");  // red[] may be rewritten next item
          scale = __fdiv_rn(m, 127.f);
          sqv = __half2float(__float2half_rn(scale));
        }
        // pass 2: INT8 codes from the raw values, then fp16(q * qk_scale) in place
        uint32_t codes[32];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4* ptr = qchunk(c);
          const uint4 u = *ptr;
          const __half2* hh = reinterpret_cast<const __half2*>(&u);
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(hh[e]);
            wv[e] = pack_half2_rn(f.x * a.qk_scale, f.y * a.qk_scale);
          }
          if (a.mode != TM_ROUTE_FP16) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float2 f0 = __half22float2(hh[2 * e]);
              const float2 f1 = __half22float2(hh[2 * e + 1]);
              codes[c * 2 + e] = (static_cast<uint32_t>(quant_code(f0.x, scale)) & 0xFFu) |
                                 ((static_cast<uint32_t>(quant_code(f0.y, scale)) & 0xFFu) << 8) |
                                 ((static_cast<uint32_t>(quant_code(f1.x, scale)) & 0xFFu) << 16) |
                                 ((static_cast<uint32_t>(quant_code(f1.y, scale)) & 0xFFu) << 24);
            }
          }
          *ptr = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        if (t == 0) ms->sq[qi & 1] = sqv;
        fence_proxy_async_smem();
        mbar_arrive(&ms->q_ready[qi & 1]);
        if (a.mode != TM_ROUTE_FP16) {
          // INT8 operand: single buffer, free once the previous item's last S is done.
          if (qi > 0) ok = __all_sync(0xffffffffu, mbar_wait(&ms->q8_empty, (qi - 1) & 1, a.err, kErrTimeoutQ));
          if (!ok) break;
          uint8_t* q8 = smem + kOffQ8;
#pragma unroll
          for (int gq = 0; gq < 8; ++gq)
            *reinterpret_cast<uint4*>(q8 + t * 128 + ((gq ^ (t & 7)) << 4)) =
                make_uint4(codes[gq * 4], codes[gq * 4 + 1], codes[gq * 4 + 2], codes[gq * 4 + 3]);
          fence_proxy_async_smem();
          mbar_arrive(&ms->q8_ready);
        }
        ++qi;
      }
      // ---- epilogue of the previous item (overlaps this item's first steps)
      if (have_prev) ok = epilogue(prev, qi - 2);
      prev = it;
      have_prev = true;
    }
    if (ok && have_prev) epilogue(prev, qi - 1);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace persistent

int launch_attn_persistent(const CUtensorMap& q, const CUtensorMap& k16, const CUtensorMap& k8, const CUtensorMap& v,
                           const AttnArgs& a, int batch, int max_seqlen_q, cudaStream_t stream) {
  using namespace persistent;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  static int n_sm[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(tilemix_attn_fwd_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess)
      return TM_ERR_LAUNCH;
    if (cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return TM_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  const int m_tiles = (max_seqlen_q + kRows - 1) / kRows;
  const long long items = static_cast<long long>(batch) * a.HQ * m_tiles;
  if (items > (1ll << 30)) return TM_ERR_SHAPE;
  const int n_items = static_cast<int>(items);
  const int grid = n_items < n_sm[dev] ? n_items : n_sm[dev];
  if (grid <= 0) return TM_OK;
  tilemix_attn_fwd_persistent_kernel<<<grid, kThreads, kSmemBytes, stream>>>(q, k16, k8, v, a, n_items, m_tiles);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace tilemix
