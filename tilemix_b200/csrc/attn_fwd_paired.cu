// Paired-tile TileMix attention forward for B200 (sm_100a): the fast path for
// head_dim 128, block_m 128 and in-kernel Q quantisation (BLKQ = 128), which is
// what the model integration and tilemix_attention_with_quant use.
//
// Same semantics as the general kernel (attention/triton/tilemix.py:503-951);
// different mapping. A work item is two 128-row query tiles X = A, B that share
// a KV head. The tiles of one (sequence, KV head) unit, group x query blocks of
// them, are listed by query block (last first), then Q head, and consecutive
// tiles form the items: two heads of one GQA group at the same query block
// (equal key loops) wherever the group allows, else the last head of a block
// with the first of the next block down (two key tiles apart). Every K/V tile is
// loaded once into shared memory and feeds both tiles.
//
// Persistent: one CTA per SM walks a static list of work items, longest first
// (the last query blocks under causal masking), dealt out in snake order
// (round r gives CTA c item r*G + c, or r*G + G-1-c for odd r). Barrier phases
// run on across items, and the item boundary is overlapped:
//   * the Q producer refills a tile's Q buffers once that tile's own last S
//     MMA of the current item has completed (q_empty), from L2 (it prefetches
//     the next item's Q tiles into L2 when an item starts). Issuing the copy
//     earlier (from the MMA warp right after that S) measured slower: the
//     transform then overlaps the other tile's last softmax steps;
//   * the softmax warpgroup transforms the next item's Q (scale, quantise)
//     while the last PV of the current item runs, then writes the current
//     item's O; meanwhile the MMA warp already runs the next item's first two
//     S tiles. Its first PV waits for o_free (the previous O read out of TMEM).
//
//   warps 0-3 / 4-7   softmax warpgroup of tile A / B (thread = query row =
//                     TMEM lane). Per item: scale Q in place in shared memory
//                     (fp16(q * sm_scale * log2e)) and quantise it per 128-row
//                     block into the INT8 operand (BLKQ = 128 block = the tile).
//   warp 8            TMA producer of K (only the formats routed by either tile),
//                     64 keys per stage of a 3-stage ring (2 stages on the INT8-V
//                     path, whose stages also hold the fp16 V codes)
//   warp 10           TMA producer of the Q tiles, then of V (same ring stages;
//                     on the INT8-V path V and / or the fp16 V codes, as routed)
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
constexpr int kMaxStages = 3;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;

constexpr uint32_t kQ16Bytes = kRows * kD * 2;  // 32 KB, two 64-column boxes of 16 KB
constexpr uint32_t kQ8Bytes = kRows * kD;       // 16 KB
constexpr uint32_t kK16Bytes = kKeys * kD * 2;  // 16 KB
constexpr uint32_t kK8Bytes = kKeys * kD;       // 8 KB
constexpr uint32_t kVBytes = kKeys * kD * 2;    // 16 KB
constexpr uint32_t kOffQ16 = 0;
constexpr uint32_t kOffQ8 = kOffQ16 + 2 * kQ16Bytes;
// Shared-memory rings. FP16-V: three stages of K16, V, K8 (222.7 KB with Q).
// INT8-V: two stages that also hold the fp16 copy of the V codes (a key tile
// that one tile routes FP16 and the other INT8 needs both V operands).
template <bool kV8>
struct Smem {
  static constexpr int kStages = kV8 ? 2 : 3;
  static constexpr uint32_t kOffK16 = kOffQ8 + 2 * kQ8Bytes;
  static constexpr uint32_t kOffV = kOffK16 + kStages * kK16Bytes;
  static constexpr uint32_t kOffK8 = kOffV + kStages * kVBytes;
  static constexpr uint32_t kOffVq = kOffK8 + kStages * kK8Bytes;
  static constexpr uint32_t kOffBar = kOffVq + (kV8 ? kStages * kVBytes : 0u);
  static constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
};
static_assert(Smem<false>::kSmemBytes <= 227 * 1024 && Smem<true>::kSmemBytes <= 227 * 1024, "shared memory");

struct Barriers {
  uint64_t full_k[kMaxStages];
  uint64_t full_v[kMaxStages];
  uint64_t empty_k[kMaxStages];  // K stage free: both tiles' S of that key tile done
  uint64_t empty_v[kMaxStages];  // V stage free: both tiles' PV of that key tile done
  uint64_t q_full[2];         // per item: Q tile landed (or a plain arrive when the tile is absent)
  uint64_t q_ready[2];        // per item: Q transformed by the softmax warpgroup (128 arrivals)
  uint64_t q_empty[2];        // per item: every S of the tile completed, its Q buffers may be refilled
  uint64_t o_free[2];         // per item: O of the tile read out of TMEM (128 arrivals)
  uint64_t s_full[2][2];
  uint64_t p_ready[2][2];
  uint64_t pv_done[2][2];
  uint64_t mma_done[2];
  uint32_t tmem_base;
  float red[2][4];
};
static_assert(sizeof(Barriers) <= 512, "barrier block");

struct QTile {
  uint64_t bits;
  int hq;
  int mtile;
  int nb;  // 64-key tiles visited (0 = tile absent)
};

// One work item, resolved from its index. Items are ordered by level x (0 =
// the first pair of each unit's tile list, the longest under causal masking),
// then sequence, then KV head, in chunks of g.chunk levels: (level chunk, unit,
// level within the chunk). With chunk 1 that is level-major (all units' longest
// items first). Units of many levels (long sequences) use a chunk of one grid's
// worth, so the CTAs of a round work on one unit and stream its K/V through L2
// together, while the chunks still run longest first.
struct Item {
  QTile tl[2];
  int q_start, seqlen_q, k_start, seqlen_k;
  int ks_base, ks_end;  // K scale-block rows of the sequence (INT8 routes)
  int vs_base, vs_end;  // V scale-block rows of the sequence (INT8-V)
  int b, hk, n_iter;
};

struct Grid {
  int nx, ny, nz, n_items;
  int mt;  // query blocks of the longest sequence
  int chunk;  // levels per unit dealt together (1: level-major order)
};

__device__ __forceinline__ Item load_item(int it, const AttnArgs& a, const Grid& g) {
  Item m;
  const int U = g.ny * g.nz;
  const int C = g.chunk;
  const int full = g.nx / C;
  int x, unit;
  if (it < full * C * U) {
    const int k = it / (C * U);
    const int r = it - k * C * U;
    unit = r / C;
    x = k * C + (r - unit * C);
  } else {
    const int Cl = g.nx - full * C;
    const int r = it - full * C * U;
    unit = r / Cl;
    x = full * C + (r - unit * Cl);
  }
  const int z = unit / g.ny;
  const int y = unit - z * g.ny;
  m.b = z;
  m.q_start = a.cu_q[z];
  m.seqlen_q = a.cu_q[z + 1] - m.q_start;
  m.k_start = a.cu_k[z];
  m.seqlen_k = a.cu_k[z + 1] - m.k_start;
  m.ks_base = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[z] : 0;
  m.ks_end = (a.mode != TM_ROUTE_FP16) ? a.cu_ks[z + 1] : 0;
  m.vs_base = a.v8_path ? a.cu_vs[z] : 0;
  m.vs_end = a.v8_path ? a.cu_vs[z + 1] : 0;
  const int m_blocks = (m.seqlen_q + kRows - 1) / kRows;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    // Tile f of the unit's list: query block g.mt-1 - f/group, head f%group of
    // the KV head's group. Past the end of the list (group * g.mt odd) the
    // slot is absent: its block lies beyond every sequence.
    const int f = 2 * x + t;
    const int fb = f / a.group;
    m.tl[t].hq = y * a.group + (f - fb * a.group);
    m.tl[t].mtile = fb < g.mt ? g.mt - 1 - fb : g.mt;
    const bool valid = m.tl[t].mtile * kRows < m.seqlen_q;
    m.tl[t].nb = valid ? visited_key_tiles(m.tl[t].mtile * kRows, kRows, m.seqlen_q, m.seqlen_k, a.causal) : 0;
    m.tl[t].bits = 0;
    if (valid && a.mode == TM_ROUTE_MIXED)
      m.tl[t].bits = a.bitmask[static_cast<int64_t>(m.tl[t].hq / a.group) * m_blocks + m.tl[t].mtile];
  }
  m.hk = y;  // both tiles share the KV head
  m.n_iter = max(m.tl[0].nb, m.tl[1].nb);
  return m;
}

// Item of round r for this CTA (snake order), or -1 past the end.
__device__ __forceinline__ int item_index(int r, const Grid& g) {
  const int G = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  const int it = r * G + ((r & 1) ? G - 1 - c : c);
  return it < g.n_items ? it : -1;
}

// Walks this CTA's items, skipping those without any query row (possible with
// varlen batches). Every role runs the same walk, so all agree on the items.
struct ItemWalk {
  int r = 0;
  __device__ __forceinline__ int next(const AttnArgs& a, const Grid& g, Item& m) {
    for (;;) {
      const int it = item_index(r++, g);
      if (it < 0) return -1;
      m = load_item(it, a, g);
      if (m.tl[0].nb > 0 || m.tl[1].nb > 0) return it;
      // an item whose tiles are both present has nb > 0; both absent: skip
      if (m.tl[0].mtile * kRows < m.seqlen_q || m.tl[1].mtile * kRows < m.seqlen_q) return it;
    }
  }
};

// Tile x of an item, selected by value (x is a runtime value: indexing the
// array would place the item in local memory).
__device__ __forceinline__ QTile tile_of(const Item& m, int x) {
  QTile q;
  q.bits = x ? m.tl[1].bits : m.tl[0].bits;
  q.hq = x ? m.tl[1].hq : m.tl[0].hq;
  q.mtile = x ? m.tl[1].mtile : m.tl[0].mtile;
  q.nb = x ? m.tl[1].nb : m.tl[0].nb;
  return q;
}

__device__ __forceinline__ bool tile_valid(const Item& m, int x) { return tile_of(m, x).mtile * kRows < m.seqlen_q; }

__device__ __forceinline__ uint32_t col_o(int x) { return static_cast<uint32_t>(x) * 128u; }
__device__ __forceinline__ uint32_t col_s(int x, int slot) {
  return 256u + static_cast<uint32_t>(x) * 128u + static_cast<uint32_t>(slot) * 64u;
}

// Scale this thread's Q row in place and build its row of the INT8 operand;
// the block scale is the maximum over the 128 rows (named barrier 1 + x over
// the tile's 128 threads). Two passes over shared memory (absmax, then codes
// and scaling) keep a few registers live instead of the whole row, and the
// codes are rounded with FMA-pipe arithmetic (quant_code_pair), which leaves the
// conversion pipe to the other tile's softmax exponentials. Returns the fp16
// block scale.
template <int kNumerics>
__device__ __forceinline__ __half transform_q(uint8_t* smem, Barriers* bars, const AttnArgs& a, int x, int t,
                                              int warp, int lane, bool row_ok) {
  uint8_t* q16 = smem + kOffQ16 + x * kQ16Bytes;
  // 16-byte chunk c (dims 8c .. 8c+7) of this row in the 128-byte-swizzled tile
  auto chunk = [&](int c) {
    return reinterpret_cast<uint4*>(q16 + (c >> 3) * (kQ16Bytes / 2) + t * 128 + (((c & 7) ^ (t & 7)) << 4));
  };
  const uint64_t qk2 = f32x2_pack(a.qk_scale, a.qk_scale);
  auto scale_f2 = [&](float2 f) {  // fp16(x * qk_scale) of a pair already in fp32
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f32x2_pack(f.x, f.y)), "l"(qk2));
    const float2 v = f32x2_unpack(r);
    return pack_half2_rn(v.x, v.y);
  };
  auto scale_pair = [&](uint32_t h2) {  // fp16(x * qk_scale) of a pair
    return scale_f2(__half22float2(*reinterpret_cast<const __half2*>(&h2)));
  };
  if (a.mode == TM_ROUTE_FP16) {
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      const uint4 r = *chunk(c);
      *chunk(c) = make_uint4(scale_pair(r.x), scale_pair(r.y), scale_pair(r.z), scale_pair(r.w));
    }
    fence_proxy_async_smem();
    return __float2half_rn(1.f);
  }
  // Pass 1: absmax of the row on fp16 pairs (|x| by clearing the sign bits).
  uint32_t am2 = 0u;
  if (row_ok) {
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      const uint4 r = *chunk(c);
      am2 = hmax2_u32(am2, hmax2_u32(r.x & 0x7FFF7FFFu, r.y & 0x7FFF7FFFu));
      am2 = hmax2_u32(am2, hmax2_u32(r.z & 0x7FFF7FFFu, r.w & 0x7FFF7FFFu));
    }
  }
  const float2 amf = __half22float2(*reinterpret_cast<const __half2*>(&am2));
  float m = fmaxf(amf.x, amf.y);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) bars->red[x][warp & 3] = m;
  asm volatile("bar.sync %0, 128;" ::"r"(1 + x) : "memory");
  m = fmaxf(fmaxf(bars->red[x][0], bars->red[x][1]), fmaxf(bars->red[x][2], bars->red[x][3]));
  // The reduction words are reused by the next item: nobody may overwrite
  // them before all four warps have read them.
  asm volatile("bar.sync %0, 128;" ::"r"(1 + x) : "memory");
  const float scale = quant_scale<kNumerics>(m);
  // A zero block (scale 0) or one holding inf (scale inf) quantises to all
  // zeros in the reference (x / scale is 0 or NaN, and NaN truncates to 0).
  const bool finite = scale > 0.f && scale <= 3.4028235e38f;
  QuantDiv qd;
  qd.init(scale);
  uint8_t* q8 = smem + kOffQ8 + x * kQ8Bytes;
#pragma unroll 4
  for (int g = 0; g < 8; ++g) {
    // 16 codes of dims [16g, 16g+16) = chunks 2g and 2g+1
    const uint4 ra = *chunk(2 * g), rb = *chunk(2 * g + 1);
    const uint32_t hw[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
    uint32_t u[16], sc[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      // One conversion of the pair serves the codes and the scaled fp16 copy.
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hw[p]));
      sc[p] = scale_f2(f);
      if (finite) {
        quant_code_pair<kNumerics>(f.x, f.y, qd, &u[2 * p], &u[2 * p + 1]);
      } else {
        u[2 * p] = 0u;
        u[2 * p + 1] = 0u;
      }
    }
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = __byte_perm(__byte_perm(u[4 * i], u[4 * i + 1], 0x0040), __byte_perm(u[4 * i + 2], u[4 * i + 3], 0x0040),
                         0x5410);
    *reinterpret_cast<uint4*>(q8 + t * 128 + ((g ^ (t & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *chunk(2 * g) = make_uint4(sc[0], sc[1], sc[2], sc[3]);
    *chunk(2 * g + 1) = make_uint4(sc[4], sc[5], sc[6], sc[7]);
  }
  fence_proxy_async_smem();
  return __float2half_rn(scale);
}

// Write this thread's O row (128 fp32 columns in TMEM) as fp16 O / l: 32
// columns per TMEM load (four load / wait round trips), stored 16 at a time,
// and release the accumulator (o_free) once all of it has been read. acc / l:
// reciprocal once per row, then per element one residual correction
// (Markstein's method: q0 = a*r, e = a - q0*l, q = q0 + e*r), which gives the
// correctly rounded quotient for these normal operands. Each thread writes its
// own row (rows are a token stride apart), 32 bytes per store where the layout
// allows.
template <int kNumerics>
__device__ __forceinline__ void epilogue_o_row(uint32_t taddr, bool have_o, float l, __half* orow, bool store,
                                               bool vec32, uint64_t* o_free) {
  const float rl = __frcp_rn(l);
  const uint64_t rl2 = f32x2_pack(rl, rl), nl2 = f32x2_pack(-l, -l);
  uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll 1
  for (int c32 = 0; c32 < 4; ++c32) {
    uint32_t o32[32];
    if (have_o) {
      tmem_ld32(taddr + 32 * c32, o32);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o32[i] = 0u;
    }
    if (c32 == 3) {
      tc_fence_before();
      mbar_arrive(o_free);
    }
    if (!store) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = 2 * c32 + h;  // 16-column chunk of the row
      const uint32_t* o = o32 + 16 * h;
      uint32_t w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (kNumerics == kNumericsGpu) {
          w[e] = normalize_pair<kNumerics>(__uint_as_float(o[2 * e]), __uint_as_float(o[2 * e + 1]), l, rl);
        } else {
          const uint64_t a2 = f32x2_pack(__uint_as_float(o[2 * e]), __uint_as_float(o[2 * e + 1]));
          const uint64_t q0 = f32x2_fma(a2, rl2, 0ull);
          const uint64_t r = f32x2_fma(q0, nl2, a2);
          const float2 q = f32x2_unpack(f32x2_fma(r, rl2, q0));
          w[e] = pack_half2_rn(q.x, q.y);
        }
      }
      if (vec32) {
        asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + 2 * c), "r"(w[0]),
                     "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                     : "memory");
      } else {
        dst[2 * c] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[2 * c + 1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
  }
}

// kV8: the INT8-V PV path (int8_use_fp16_v == 0): an INT8-routed tile's PV
// is fp16(p * sv) x fp16(v8) (tilemix.py:449-497), with fp16(v8) loaded from
// the exact fp16 copy of the V codes (tm_vq) and sv the fp16 V block scale.
template <int kNumerics, bool kV8>
__global__ void __launch_bounds__(kThreads, 1)
    tilemix_attn_fwd_paired_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k16,
                                   const __grid_constant__ CUtensorMap tm_k8, const __grid_constant__ CUtensorMap tm_v,
                                   const __grid_constant__ CUtensorMap tm_vq, const AttnArgs a, const Grid grid) {
  using L = Smem<kV8>;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + L::kOffBar);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (item_index(0, grid) < 0) return;  // uniform, before any barrier or allocation

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
      mbar_init(&bars->q_empty[x], 1);
      mbar_init(&bars->o_free[x], kRows);
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
    // The whole warp runs the loops (warp-uniform control flow); one elected
    // lane issues each copy. g counts key tiles over all items (ring position).
    const bool is_k = warp == 8;
    if (is_k) {
      prefetch_tmap(&tm_k16);
      if (a.mode != TM_ROUTE_FP16) prefetch_tmap(&tm_k8);
    } else {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_v);
      if (kV8) prefetch_tmap(&tm_vq);
    }
    bool ok = true;
    uint32_t g = 0;
    int n = 0;  // items done
    ItemWalk walk;
    Item m;
    int it = walk.next(a, grid, m);
    while (it >= 0 && ok) {
      ItemWalk peek = walk;
      Item mn;
      const int it_next = peek.next(a, grid, mn);
      if (!is_k) {
        // Q tiles of this item, each once the previous item's last S of that
        // tile has completed.
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (n > 0)
            ok = ok && __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_empty[x], (n - 1) & 1, a.err, kErrTimeoutQFree));
          if (!ok) break;
          if (tile_valid(m, x)) {
            mbar_arrive_expect_tx_e(&bars->q_full[x], kQ16Bytes);
            tma_load_4d_e(smem + kOffQ16 + x * kQ16Bytes, &tm_q, &bars->q_full[x], 0,
                          m.q_start + tile_of(m, x).mtile * kRows, 0, tile_of(m, x).hq);
          } else if (lane == 0) {
            mbar_arrive(&bars->q_full[x]);
          }
          __syncwarp();
        }
        // Warm L2 with the next item's Q tiles.
        if (ok && it_next >= 0 && lane == 0) {
#pragma unroll
          for (int x = 0; x < 2; ++x)
            if (tile_valid(mn, x)) tma_prefetch_l2_4d(&tm_q, 0, mn.q_start + tile_of(mn, x).mtile * kRows, 0, tile_of(mn, x).hq);
        }
      }
      RouteWalker rw[2];
#pragma unroll
      for (int x = 0; x < 2; ++x) rw[x].init(a.mode, tile_of(m, x).bits, a.block_n_mask);
      for (int j = 0; j < m.n_iter && ok; ++j, ++g) {
        const uint32_t s = g % kStages;
        if (g >= static_cast<uint32_t>(kStages))
          ok = __all_sync(0xffffffffu, mbar_wait_spin(is_k ? &bars->empty_k[s] : &bars->empty_v[s],
                                                      ((g / kStages) + 1) & 1, a.err, kErrTimeoutEmpty));
        if (!ok) break;
        const int tok = m.k_start + j * kKeys;
        if (is_k) {
          bool n16 = false, n8 = false;
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (j < tile_of(m, x).nb) {
              if (rw[x].kind())
                n8 = true;
              else
                n16 = true;
            }
            rw[x].advance();
          }
          mbar_arrive_expect_tx_e(&bars->full_k[s], (n16 ? kK16Bytes : 0u) + (n8 ? kK8Bytes : 0u));
          if (n16) tma_load_4d_e(smem + L::kOffK16 + s * kK16Bytes, &tm_k16, &bars->full_k[s], 0, tok, 0, m.hk);
          if (n8) tma_load_3d_e(smem + L::kOffK8 + s * kK8Bytes, &tm_k8, &bars->full_k[s], 0, m.hk, tok);
        } else {
          // FP16-V: V for every key tile. INT8-V: V for the tiles that route the
          // key tile FP16, the fp16 V codes for those that route it INT8.
          bool v16 = true, vq = false;
          if (kV8) {
            v16 = false;
#pragma unroll
            for (int x = 0; x < 2; ++x) {
              if (j < tile_of(m, x).nb) {
                if (rw[x].kind())
                  vq = true;
                else
                  v16 = true;
              }
              rw[x].advance();
            }
          }
          mbar_arrive_expect_tx_e(&bars->full_v[s], (v16 ? kVBytes : 0u) + (vq ? kVBytes : 0u));
          if (v16) tma_load_4d_e(smem + L::kOffV + s * kVBytes, &tm_v, &bars->full_v[s], 0, tok, 0, m.hk);
          if (kV8 && vq) tma_load_4d_e(smem + L::kOffVq + s * kVBytes, &tm_vq, &bars->full_v[s], 0, tok, 0, m.hk);
        }
      }
      ++n;
      walk = peek;
      m = mn;
      it = it_next;
    }
    // Drain: every copy this warp issued has landed before the CTA can exit.
    const uint32_t first = g > static_cast<uint32_t>(kStages) ? g - kStages : 0u;
    for (uint32_t q = first; q < g; ++q)
      mbar_wait(is_k ? &bars->full_k[q % kStages] : &bars->full_v[q % kStages], (q / kStages) & 1, a.err,
                kErrTimeoutDrain);
  } else if (warp == 9 || warp == 11) {
    // ------------------------------------------------------------------ MMA issuers
    // One warp per query tile X (warp 9: A, warp 11: B, on different SM
    // sub-partitions), each running converged with one elected lane issuing,
    // in a fixed order per key tile j:
    //   S_X(j), release K(j), PV_X(j-1), release V(j-1)
    // (a stage is free once both warps have committed its release). S_X(j)
    // overwrites TMEM slot c&1 (c = step count of tile X over all items), which
    // P_X(c-2) occupied: PV_X(c-2) was issued earlier by the same thread and
    // tcgen05.mma operations from one thread execute in issue order, so it has
    // read P before S_X writes the slot. Descriptors are built once; a byte
    // offset is added as offset >> 4 to the start-address field (all
    // shared-memory offsets here are < 256 KB).
    const int x = warp == 9 ? 0 : 1;
    // FP16 scores accumulate in fp16 (GPU numerics) or fp32 (exact numerics).
    constexpr uint32_t idesc_qk16 = make_idesc(kNumerics == kNumericsGpu ? 0 : 1, 0, 0, 0, 128, 64);
    constexpr uint32_t idesc_qk8 = make_idesc(2, 1, 0, 0, 128, 64);
    constexpr uint32_t idesc_pv = make_idesc(1, 0, 0, 1, 128, kD);
    const uint64_t dq16 = make_sdesc(smem_u32(smem + kOffQ16 + x * kQ16Bytes), 16, 1024, 2);
    const uint64_t dq8 = make_sdesc(smem_u32(smem + kOffQ8 + x * kQ8Bytes), 16, 1024, 2);
    const uint64_t dk16 = make_sdesc(smem_u32(smem + L::kOffK16), 16, 1024, 2);
    const uint64_t dk8 = make_sdesc(smem_u32(smem + L::kOffK8), 16, 1024, 2);
    const uint64_t dv = make_sdesc(smem_u32(smem + L::kOffV), kVBytes / 2, 1024, 2);
    const uint64_t dvq = make_sdesc(smem_u32(smem + L::kOffVq), kVBytes / 2, 1024, 2);
    const uint32_t d_o = tbase + col_o(x);
    bool ok = true;
    uint32_t g = 0;   // key tiles over all items
    uint32_t cx = 0;  // steps of tile X over all items
    int n = 0;
    ItemWalk walk;
    Item m;
    int it = walk.next(a, grid, m);
    while (it >= 0 && ok) {
      ItemWalk peek = walk;
      Item mn;
      const int it_next = peek.next(a, grid, mn);
      const int nb = tile_of(m, x).nb;
      ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_ready[x], n & 1, a.err, kErrTimeoutQ));
      tc_fence_after();
      if (nb == 0) tc_commit_e(&bars->q_empty[x]);
      RouteWalker rw, rw_pv;
      rw.init(a.mode, tile_of(m, x).bits, a.block_n_mask);
      rw_pv.init(a.mode, tile_of(m, x).bits, a.block_n_mask);
      for (int j = 0; j <= m.n_iter && ok; ++j) {
        if (j < m.n_iter) {
          const uint32_t gj = g + j;
          const uint32_t st = gj % kStages;
          const int kind = rw.kind();
          rw.advance();
          // Wait for K(j) even when this tile does not use it: the release below
          // must not reach the stage's barrier before the other warp's release of
          // the previous use of the stage (the copy of K(j) waited for it), or
          // two releases from this warp could complete one phase.
          ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->full_k[st], (gj / kStages) & 1, a.err, kErrTimeoutFull));
          if (!ok) break;
          if (j < nb) {
            tc_fence_after();
            const uint32_t c = cx + j;
            const uint32_t d = tbase + col_s(x, c & 1);
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
              for (int kk = 0; kk < kD / 32; ++kk)
                mma_i8_ss_e(d, dq8 + kk * 2, kb + kk * 2, idesc_qk8, kk > 0 ? 1u : 0u);
            }
            tc_commit_e(&bars->s_full[x][c & 1]);
            // This tile's last S: its Q buffers can be refilled once it completes,
            // while the other tile may still have key tiles to go.
            if (j == nb - 1) tc_commit_e(&bars->q_empty[x]);
          }
          tc_commit_e(&bars->empty_k[st]);  // this warp is done with K(j) once its S has run
        }
        if (j >= 1) {
          const int jj = j - 1;
          const uint32_t gj = g + jj;
          const uint32_t st = gj % kStages;
          const int kind_pv = rw_pv.kind();  // route of key tile jj (INT8-V operand choice)
          rw_pv.advance();
          ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->full_v[st], (gj / kStages) & 1, a.err, kErrTimeoutFull));
          if (!ok) break;
          if (jj < nb) {
            const uint32_t c = cx + jj;
            // Before the last PV's wait for P (about one softmax step away):
            // the last S has completed or is about to.
            ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->p_ready[x][c & 1], (c >> 1) & 1, a.err, kErrTimeoutP));
            if (ok && jj == 0 && n > 0)  // first PV overwrites O: the previous item's O must be read out
              ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->o_free[x], (n - 1) & 1, a.err, kErrTimeoutOFree));
            if (!ok) break;
            tc_fence_after();
            const uint64_t vb = (kV8 && kind_pv == 1 ? dvq : dv) + ((st * kVBytes) >> 4);
            const uint32_t pa = tbase + col_s(x, c & 1);
#pragma unroll
            for (int kk = 0; kk < kKeys / 16; ++kk)
              mma_f16_ts_e(d_o, pa + kk * 8, vb + ((kk * 16 * 128) >> 4), idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
            tc_commit_e(&bars->pv_done[x][c & 1]);
          }
          tc_commit_e(&bars->empty_v[st]);
        }
      }
      g += m.n_iter;
      cx += nb;
      ++n;
      walk = peek;
      m = mn;
      it = it_next;
    }
    tc_commit_e(&bars->mma_done[x]);
    mbar_wait(&bars->mma_done[x], 0, a.err, kErrTimeoutDrain);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int x = warp >> 2;
    const int t = threadIdx.x & 127;  // row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float kNegInf = -__int_as_float(0x7f800000);
    bool ok = true;
    uint32_t cx = 0;  // steps of tile X over all items
    int n = 0;
    ItemWalk walk;
    Item m;
    int it = walk.next(a, grid, m);
    // Q of the first item.
    __half sq16 = __float2half_rn(1.f);
    if (it >= 0) {
      ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_full[x], 0, a.err, kErrTimeoutQ));
      if (tile_valid(m, x)) sq16 = transform_q<kNumerics>(smem, bars, a, x, t, warp, lane, tile_of(m, x).mtile * kRows + t < m.seqlen_q);
      mbar_arrive(&bars->q_ready[x]);
    }
    while (it >= 0 && ok) {
      // Everything the step loop and the epilogue need from the item, so that
      // the item itself is dead during the loop.
      const int nb = tile_of(m, x).nb;
      const int row = tile_of(m, x).mtile * kRows + t;
      const bool store = tile_valid(m, x) && row < m.seqlen_q;
      __half* orow = a.out + (static_cast<int64_t>(m.q_start) + row) * a.o_st + static_cast<int64_t>(tile_of(m, x).hq) * a.o_sh;
      int lim0 = m.seqlen_k;  // keys of this row before tile 0's end is subtracted
      if (a.causal) lim0 = min(lim0, row + (m.seqlen_k - m.seqlen_q) + 1);
      float m_used = kNegInf;
      float l = 1.f;
      const int ks_base = m.ks_base, ks_end = m.ks_end;
      // K block scale of a tile, loaded one tile ahead to keep the global load
      // off the critical path. Routes and scale blocks of consecutive tiles are
      // tracked incrementally (no per-tile division).
      RouteWalker rw;
      rw.init(a.mode, tile_of(m, x).bits, a.block_n_mask);
      const int sk_per = a.blkk / kKeys;  // 64-key tiles per K scale block (blkk % 64 == 0)
      int sk_idx = ks_base, sk_sub = 0;
      // The load is unconditional (clamped to a valid row) and its value is only
      // selected when used, one tile later, so no instruction waits on it early.
      const bool have_sk = ks_end > ks_base;
      const __half* sk_col = a.k_scale + m.hk;
      auto load_next_sk = [&]() -> __half {  // raw scale of the next tile in order; then step
        const __half v = have_sk ? sk_col[static_cast<int64_t>(min(sk_idx, ks_end - 1)) * a.HK] : __half();
        if (++sk_sub == sk_per) {
          sk_sub = 0;
          ++sk_idx;
        }
        return v;
      };
      __half sk_next = load_next_sk();
      // INT8-V: V block scale of a tile, tracked and loaded like the K scale
      // (1 when the sequence has no scale rows, the reference's masked load).
      const int vs_end = m.vs_end;
      const bool have_sv = kV8 && vs_end > m.vs_base;
      const __half* sv_col = a.v_scale + m.hk;
      int sv_idx = m.vs_base, sv_sub = 0;
      auto load_next_sv = [&]() -> __half {
        const __half v = have_sv ? sv_col[static_cast<int64_t>(min(sv_idx, vs_end - 1)) * a.HK] : __half();
        if (++sv_sub == sk_per) {
          sv_sub = 0;
          ++sv_idx;
        }
        return v;
      };
      __half sv_next = kV8 ? load_next_sv() : __half();
      for (int j = 0; ok && j < nb; ++j) {
        const uint32_t c = cx + j;
        const int slot = c & 1;
        const int kind = rw.kind();
        rw.advance();
        const __half sk16 = (have_sk && kind == 1) ? sk_next : __float2half_rn(1.f);
        sk_next = load_next_sk();
        __half sv16 = __float2half_rn(1.f);
        if (kV8) {
          if (have_sv && kind == 1) sv16 = sv_next;
          sv_next = load_next_sv();
        }
        const float ss = kind == 1 ? int8_score_scale(sq16, sk16, a.qk_scale) : 1.f;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->s_full[x][slot], (c >> 1) & 1, a.err, kErrTimeoutScores));
        if (!ok) break;
        tc_fence_after();
        const int lim = lim0 - j * kKeys;
        uint32_t p[32];
        float o_scale;
        bool need_rescale;
        softmax_tile<kNumerics>(tbase + lane_off + col_s(x, slot), kind, ss, lim, a.rescale_threshold, m_used, l, p, o_scale,
                     need_rescale);
        if (kV8 && kind == 1) {
          // p_scaled = fp16(p * sv): the product of two fp16 values rounded once
          // (l above summed the unscaled p, as the reference's l_tile does).
          const __half2 sv2 = __halves2half2(sv16, sv16);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&p[i]), sv2);
            p[i] = *reinterpret_cast<const uint32_t*>(&r);
          }
        }
        // P goes out first; its store overlaps the wait for the previous PV
        // when O has to be rescaled (PV(c-1) must have accumulated into O).
        tmem_st32(tbase + lane_off + col_s(x, slot), p);
        if (__any_sync(0xffffffffu, need_rescale)) {
          const uint32_t cp = c - 1;
          ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->pv_done[x][cp & 1], (cp >> 1) & 1, a.err, kErrTimeoutPV));
          if (!ok) break;
          tc_fence_after();
          rescale_o_row<kD>(tbase + lane_off + col_o(x), o_scale);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->p_ready[x][slot]);
      }
      if (!ok) break;
      cx += nb;
      ItemWalk peek = walk;
      Item mn;
      const int it_next = peek.next(a, grid, mn);
      // The next item's Q (its tile landed after this item's last S of the
      // tile) while the tensor core finishes this item's last PV.
      __half sq16_next = __float2half_rn(1.f);
      if (it_next >= 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->q_full[x], (n + 1) & 1, a.err, kErrTimeoutQ));
        if (!ok) break;
        if (tile_valid(mn, x))
          sq16_next = transform_q<kNumerics>(smem, bars, a, x, t, warp, lane, tile_of(mn, x).mtile * kRows + t < mn.seqlen_q);
        mbar_arrive(&bars->q_ready[x]);
      }
      // This item's O.
      if (nb > 0) {
        const uint32_t cl = cx - 1;
        ok = __all_sync(0xffffffffu, mbar_wait_spin(&bars->pv_done[x][cl & 1], (cl >> 1) & 1, a.err, kErrTimeoutPV));
        tc_fence_after();
      }
      epilogue_o_row<kNumerics>(tbase + lane_off + col_o(x), nb > 0 && ok, l, orow, store && ok, a.o_vec32 != 0,
                     &bars->o_free[x]);
      sq16 = sq16_next;
      ++n;
      walk = peek;
      m = mn;
      it = it_next;
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
                       const CUtensorMap& vq, const AttnArgs& a, int batch, int max_seqlen_q, cudaStream_t stream) {
  using namespace paired;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  static int n_sm[64] = {};
  if (!attr_set[dev]) {
    const int b16 = static_cast<int>(Smem<false>::kSmemBytes), b8 = static_cast<int>(Smem<true>::kSmemBytes);
    if (cudaFuncSetAttribute(tilemix_attn_fwd_paired_kernel<kNumericsGpu, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, b16) != cudaSuccess ||
        cudaFuncSetAttribute(tilemix_attn_fwd_paired_kernel<kNumericsExact, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, b16) != cudaSuccess ||
        cudaFuncSetAttribute(tilemix_attn_fwd_paired_kernel<kNumericsGpu, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, b8) != cudaSuccess ||
        cudaFuncSetAttribute(tilemix_attn_fwd_paired_kernel<kNumericsExact, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, b8) != cudaSuccess)
      return TM_ERR_LAUNCH;
    if (cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm[dev] <= 0)
      return TM_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  const int mtiles = (max_seqlen_q + kRows - 1) / kRows;
  Grid g;
  g.mt = mtiles;
  g.nx = static_cast<int>((static_cast<int64_t>(a.group) * mtiles + 1) / 2);
  g.ny = a.HK;
  g.nz = batch;
  const int64_t items = static_cast<int64_t>(g.nx) * g.ny * g.nz;
  if (items <= 0) return TM_OK;
  if (items > (1ll << 30)) return TM_ERR_SHAPE;
  g.n_items = static_cast<int>(items);
  const int ctas = static_cast<int>(std::min<int64_t>(items, n_sm[dev]));
  // Long units (at least two grids' worth of levels): one unit's levels per round.
  g.chunk = g.nx >= 2 * ctas ? ctas : 1;
  const uint32_t b16 = Smem<false>::kSmemBytes, b8 = Smem<true>::kSmemBytes;
  if (a.v8_path) {
    if (a.numerics == kNumericsGpu)
      tilemix_attn_fwd_paired_kernel<kNumericsGpu, true><<<ctas, kThreads, b8, stream>>>(q, k16, k8, v, vq, a, g);
    else
      tilemix_attn_fwd_paired_kernel<kNumericsExact, true><<<ctas, kThreads, b8, stream>>>(q, k16, k8, v, vq, a, g);
  } else if (a.numerics == kNumericsGpu) {
    tilemix_attn_fwd_paired_kernel<kNumericsGpu, false><<<ctas, kThreads, b16, stream>>>(q, k16, k8, v, vq, a, g);
  } else {
    tilemix_attn_fwd_paired_kernel<kNumericsExact, false><<<ctas, kThreads, b16, stream>>>(q, k16, k8, v, vq, a, g);
  }
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}

}  // namespace tilemix
