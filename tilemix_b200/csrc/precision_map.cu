// Routing-map construction on the GPU: the packed uint64 row words of
// make_precision_bitmask (attention/precision_maps.py:404-636) for the paths
// the model integration uses (token_mask = None): zero, one, and band /
// global / row_rand / align_sparse / bigbird / sptrans at an INT8 percentage.
//
// One CTA builds the whole map (at most 64 mask groups per row, at most
// 65536 cells):
//   * the [num_m x num_n] boolean map lives as one uint64 per row in shared
//     memory (bit j = mask group j routed to INT8); per-row construction runs
//     in parallel, a thread per row;
//   * random draws are MT19937 outputs exactly as torch's CPU generator makes
//     them (seed 42 like the reference). Warp 0 runs the generator: the
//     624-word twist splits into three dependency-free phases of 227, 227 and
//     169 words plus the last word, each a warp-parallel loop;
//   * row permutations (row_rand, bigbird) are torch's CPU randperm
//     (Fisher-Yates, element i swapped with element i + r mod (n - i)); draws
//     for a band of rows are staged in shared memory and every row of the
//     band is shuffled in parallel;
//   * the order-dependent parts — bigbird's top-up flips (:585-601) and the
//     weighted retarget walk (:273-326) — shuffle a uint16 candidate array in
//     shared memory one position at a time, on lane 0 of warp 0, drawing
//     straight from the generator's state, so the walk stops exactly where
//     the reference's does and never generates draws it does not use.
// Causal compute-tile weights (:238-270) are kept as one tile count per row.
// The kernel needs no device memory beyond the output and the error word.
#include "common.cuh"
#include "tilemix_b200.h"

#include <cmath>

namespace tilemix {
namespace pmap {

constexpr int kThreads = 256;
constexpr int kMaxRows = 4096;
constexpr int kMaxCols = 64;
constexpr int kMaxCells = 65536;  // candidate indices row * num_n + col fit in uint16
constexpr int kMtN = 624;
constexpr int kMtM = 397;
constexpr int kPermBytes = kMaxCols * kThreads;                   // randperm scratch, a column per thread
constexpr int kChunkWords = (kMaxCells * 2 - kPermBytes) / 4;    // staged draws per band of rows

enum Pattern : int { kZero = 0, kOne, kBand, kGlobal, kRowRand, kAlignSparse, kBigBird, kSpTrans };

struct MapArgs {
  int seq_len, block_m, block_n_mask, compute_block_n;
  int pattern;
  double percentage;
  int stride, c;                          // sptrans
  uint64_t global_cols;                   // global: FP16 columns, resolved on the host from key_pos
  int num_global_block, num_rand_block;   // bigbird
  uint64_t* out;
  int* err;
};

struct Shared {
  uint64_t bits[kMaxRows];
  int tiles[kMaxRows];  // visited compute tiles of each query block
  int row_off[kMaxRows + 2];
  union {
    uint16_t cand[kMaxCells];
    struct {
      uint8_t perm[kMaxCols][kThreads];
      uint32_t draws[kChunkWords];
    } rows;
  } u;
  uint32_t mt[2][kMtN];
  long long red[kThreads / 32];
};

struct Geo {
  int num_m, num_n, num_compute_n, group;
};

// ---------------------------------------------------------------------------
// Bit helpers and Python arithmetic
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t range_mask(int lo, int hi) {  // bits [lo, hi) of a row word
  lo = max(lo, 0);
  hi = min(hi, kMaxCols);
  if (hi <= lo) return 0ull;
  const uint64_t upto_hi = hi >= 64 ? ~0ull : ((1ull << hi) - 1ull);
  return upto_hi & ~((1ull << lo) - 1ull);
}

// Python's round() of a non-negative double (ties to even), as an integer.
__device__ __forceinline__ long long py_round(double x) { return static_cast<long long>(rint(x)); }

__device__ __forceinline__ long long clamp_ll(long long x, long long lo, long long hi) {
  return x < lo ? lo : (x > hi ? hi : x);
}

// Weight of (row, col) from the row's visited compute-tile count (:253-269).
__device__ __forceinline__ int tile_weight(const Geo& g, int tiles, int col) {
  const int full = tiles / g.group, rem = tiles % g.group;
  if (col < full) return g.group;
  if (col == full && rem != 0 && full < g.num_n) return rem;
  return 0;
}

__device__ __forceinline__ uint64_t visited_cols(const Geo& g, int tiles) {
  const int full = tiles / g.group, rem = tiles % g.group;
  return range_mask(0, full + ((rem != 0 && full < g.num_n) ? 1 : 0));
}

// ---------------------------------------------------------------------------
// MT19937 (Matsumoto & Nishimura 1998), run by one warp. The state of the
// current 624-output block is sh->mt[cur]; idx is the next unread position.
// Every lane of the warp holds the same (cur, idx).
// ---------------------------------------------------------------------------
struct MTStream {
  int cur, idx;
};

__device__ __forceinline__ uint32_t mt_mix(uint32_t cur, uint32_t next, uint32_t far) {
  const uint32_t y = (cur & 0x80000000u) | (next & 0x7fffffffu);
  return far ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
}

__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

__device__ void mt_seed(Shared* sh, MTStream& s, uint32_t seed) {
  if ((threadIdx.x & 31) == 0) {
    uint32_t* st = sh->mt[0];
    st[0] = seed;
    for (int i = 1; i < kMtN; ++i) st[i] = 1812433253u * (st[i - 1] ^ (st[i - 1] >> 30)) + static_cast<uint32_t>(i);
  }
  __syncwarp();
  s.cur = 0;
  s.idx = kMtN;
}

// One twist: new[i] = mix(old[i], old[i+1], x[i+397 mod 624]) with x = old
// below 227 and x = new from there on, so the three ranges below each depend
// only on finished words.
__device__ void mt_refill(Shared* sh, MTStream& s) {
  const int lane = threadIdx.x & 31;
  const uint32_t* old = sh->mt[s.cur];
  uint32_t* nw = sh->mt[s.cur ^ 1];
  constexpr int kSplit = kMtN - kMtM;  // 227
  for (int i = lane; i < kSplit; i += 32) nw[i] = mt_mix(old[i], old[i + 1], old[i + kMtM]);
  __syncwarp();
  for (int i = kSplit + lane; i < 2 * kSplit; i += 32) nw[i] = mt_mix(old[i], old[i + 1], nw[i - kSplit]);
  __syncwarp();
  for (int i = 2 * kSplit + lane; i < kMtN - 1; i += 32) nw[i] = mt_mix(old[i], old[i + 1], nw[i - kSplit]);
  __syncwarp();
  if (lane == 0) nw[kMtN - 1] = mt_mix(old[kMtN - 1], nw[0], nw[kMtM - 1]);
  __syncwarp();
  s.cur ^= 1;
  s.idx = 0;
}

// Appends the next n outputs to dst (shared memory).
__device__ void mt_take(Shared* sh, MTStream& s, uint32_t* dst, int n) {
  const int lane = threadIdx.x & 31;
  for (int done = 0; done < n;) {
    if (s.idx == kMtN) mt_refill(sh, s);
    const int k = min(kMtN - s.idx, n - done);
    const uint32_t* src = sh->mt[s.cur] + s.idx;
    for (int i = lane; i < k; i += 32) dst[done + i] = mt_temper(src[i]);
    s.idx += k;
    done += k;
  }
  __syncwarp();
}

// Visits positions 0 .. steps-1 of torch.randperm(L) applied to cand (so the
// element at position p is cand[perm[p]]), calling visit(cell) on each until
// it returns true. Run by a full warp; lane 0 walks, the warp refills.
template <typename Visit>
__device__ void shuffled_walk(Shared* sh, MTStream& s, uint16_t* cand, int L, int steps, Visit&& visit) {
  const int lane = threadIdx.x & 31;
  int pos = 0;
  int stop = 0;
  while (!stop && pos < steps) {
    const bool drawing = pos < L - 1;  // randperm(L) draws for positions 0 .. L-2 only
    int avail;
    if (drawing) {
      if (s.idx == kMtN) mt_refill(sh, s);
      avail = min(kMtN - s.idx, min(L - 1, steps) - pos);
    } else {
      avail = steps - pos;
    }
    if (lane == 0) {
      const uint32_t* src = sh->mt[s.cur] + s.idx;
      for (int t = 0; t < avail && !stop; ++t) {
        if (drawing) {
          const int z = static_cast<int>(mt_temper(src[t]) % static_cast<uint32_t>(L - pos));
          const uint16_t a = cand[pos];
          cand[pos] = cand[pos + z];
          cand[pos + z] = a;
        }
        stop = visit(static_cast<int>(cand[pos])) ? 1 : 0;
        ++pos;
      }
    }
    __syncwarp();
    if (drawing) s.idx += avail;
    pos = __shfl_sync(0xffffffffu, pos, 0);
    stop = __shfl_sync(0xffffffffu, stop, 0);
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Block-wide helpers
// ---------------------------------------------------------------------------
__device__ long long block_sum(long long v, Shared* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh->red[threadIdx.x >> 5] = v;
  __syncthreads();
  long long total = 0;
  for (int w = 0; w < kThreads / 32; ++w) total += sh->red[w];
  return total;
}

// Row-major list of the cells set in sel(row) into sh->u.cand; returns its length.
template <typename Sel>
__device__ int collect_cells(Shared* sh, const Geo& g, Sel&& sel) {
  for (int r = threadIdx.x; r < g.num_m; r += kThreads) sh->row_off[r] = __popcll(sel(r));
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int r = 0; r < g.num_m; ++r) {
      const int c = sh->row_off[r];
      sh->row_off[r] = acc;
      acc += c;
    }
    sh->row_off[g.num_m] = acc;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < g.num_m; r += kThreads) {
    uint64_t m = sel(r);
    int o = sh->row_off[r];
    while (m) {
      const int col = __ffsll(static_cast<long long>(m)) - 1;
      m &= m - 1;
      sh->u.cand[o++] = static_cast<uint16_t>(r * g.num_n + col);
    }
  }
  __syncthreads();
  return sh->row_off[g.num_m];
}

// First `take` entries of torch.randperm(n) from the n-1 draws at d, as a column mask.
__device__ __forceinline__ uint64_t randperm_prefix(uint8_t (*perm)[kThreads], int n, const uint32_t* d, int take) {
  const int t = threadIdx.x;
  for (int i = 0; i < n; ++i) perm[i][t] = static_cast<uint8_t>(i);
  for (int i = 0; i < n - 1; ++i) {
    const int z = static_cast<int>(d[i] % static_cast<uint32_t>(n - i));
    const uint8_t a = perm[i][t];
    perm[i][t] = perm[i + z][t];
    perm[i + z][t] = a;
  }
  uint64_t m = 0;
  for (int i = 0; i < take && i < n; ++i) m |= 1ull << perm[i][t];
  return m;
}

// Row r of the pattern before any random part (true = INT8).
__device__ uint64_t initial_row(const MapArgs& a, const Geo& g, int r, uint64_t all, int tiles) {
  const double p = a.percentage;
  const int num_n = g.num_n;
  switch (a.pattern) {
    case kZero:
      return 0ull;
    case kOne:
      return visited_cols(g, tiles);
    case kBand: {  // :492-506
      long long tbb = py_round(num_n * (1.0 - p));
      if (tbb % 2 == 0) tbb = max(1ll, tbb - 1);
      tbb = clamp_ll(tbb, 1, num_n);
      const int half = static_cast<int>(tbb / 2);
      return all & ~range_mask(r - half, min(num_n, r + half + 1));
    }
    case kGlobal:  // :507-531
      return all & ~a.global_cols;
    case kRowRand:  // :532-540 (random columns applied per band of rows)
      return all;
    case kAlignSparse: {  // :541-548
      const long long tab = clamp_ll(py_round(num_n * (1.0 - p)), 1, num_n);
      return all & ~range_mask(num_n - static_cast<int>(tab), num_n);
    }
    case kBigBird: {  // :549-579 (band, global rows/columns; random columns later)
      const long long tbr = clamp_ll(py_round(num_n * (1.0 - p) * 0.5), 1, num_n);
      const long long bw = min((tbr % 2 == 0) ? tbr + 1 : tbr, static_cast<long long>(num_n));
      const int center = min(r, num_n - 1);
      const int half = static_cast<int>(bw / 2);
      uint64_t m = all & ~range_mask(center - half, min(num_n, center + half + 1));
      const int ng = min(a.num_global_block, num_n);
      m &= ~range_mask(0, ng);
      return r < ng ? 0ull : m;
    }
    case kSpTrans: {  // :329-376
      uint64_t m = all;
      const int bnm = a.block_n_mask;
      const int qs = r * a.block_m;
      const int qe = min(a.seq_len, (r + 1) * a.block_m);
      for (int qst = qs / a.stride; qst <= (qe - 1) / a.stride; ++qst) {
        const int ss = qst * a.stride;
        const int se = min((qst + 1) * a.stride, qe);
        const int sb = ss / bnm;
        if (sb < num_n) m &= ~range_mask(sb, min(num_n, (se + bnm - 1) / bnm));
        for (int prev = 0; prev < qst; ++prev) {
          const int pe = (prev + 1) * a.stride;
          const int ts = max(prev * a.stride, pe - a.c);
          const int tsb = ts / bnm;
          if (tsb < num_n) m &= ~range_mask(tsb, min(num_n, (pe + bnm - 1) / bnm));
        }
      }
      return m;
    }
    default:
      return 0ull;
  }
}

__global__ void __launch_bounds__(kThreads, 1) build_map_kernel(const MapArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Shared* sh = reinterpret_cast<Shared*>(smem_raw);
  const int tid = threadIdx.x;
  const bool warp0 = tid < 32;
  Geo g;
  g.num_m = (a.seq_len + a.block_m - 1) / a.block_m;
  g.num_n = (a.seq_len + a.block_n_mask - 1) / a.block_n_mask;
  g.num_compute_n = (a.seq_len + a.compute_block_n - 1) / a.compute_block_n;
  g.group = a.block_n_mask / a.compute_block_n;
  const int num_m = g.num_m, num_n = g.num_n;
  const uint64_t all = range_mask(0, num_n);
  const double p = a.percentage;

  for (int r = tid; r < num_m; r += kThreads) {
    const long long reach = static_cast<long long>(r + 1) * a.block_m + a.compute_block_n - 1;
    const int tiles = static_cast<int>(min(static_cast<long long>(g.num_compute_n), reach / a.compute_block_n));
    sh->tiles[r] = tiles;
    sh->bits[r] = initial_row(a, g, r, all, tiles);
  }
  __syncthreads();

  MTStream mts{0, kMtN};
  // ---------------- random columns per row (row_rand, bigbird) ----------------
  if (a.pattern == kRowRand || a.pattern == kBigBird) {
    // torch.manual_seed(42), then randperm(num_n) for every row in order.
    if (warp0) mt_seed(sh, mts, 42u);
    const int take = a.pattern == kRowRand ? static_cast<int>(clamp_ll(py_round(num_n * (1.0 - p)), 1, num_n))
                                           : min(a.num_rand_block, num_n);
    const int per_row = num_n - 1;
    const int band = per_row > 0 ? kChunkWords / per_row : num_m;
    for (int r0 = 0; r0 < num_m; r0 += band) {
      const int r1 = min(num_m, r0 + band);
      if (warp0 && per_row > 0) mt_take(sh, mts, sh->u.rows.draws, (r1 - r0) * per_row);
      __syncthreads();
      for (int r = r0 + tid; r < r1; r += kThreads)
        sh->bits[r] &= ~randperm_prefix(sh->u.rows.perm, num_n, sh->u.rows.draws + (r - r0) * per_row, take);
      __syncthreads();
    }
  }

  // ---------------- bigbird top-up flips (:585-601) ----------------
  if (a.pattern == kBigBird) {
    const long long cells = static_cast<long long>(num_m) * num_n;
    const long long thp = clamp_ll(py_round(static_cast<double>(cells) * (1.0 - p)), 1, cells);
    long long hp = 0;
    for (int r = tid; r < num_m; r += kThreads) hp += __popcll(~sh->bits[r] & all);
    hp = block_sum(hp, sh);
    if (hp != thp) {
      const bool to_fp16 = hp < thp;  // too few FP16 cells: flip INT8 cells, else the reverse
      const int L = collect_cells(sh, g, [&](int r) { return (to_fp16 ? sh->bits[r] : ~sh->bits[r]) & all; });
      if (warp0 && L > 0) {
        const int k = static_cast<int>(min(to_fp16 ? thp - hp : hp - thp, static_cast<long long>(L)));
        // randperm(L) continues the global generator after the row permutations.
        shuffled_walk(sh, mts, sh->u.cand, L, k, [&](int cell) {
          const int rr = cell / num_n, cc = cell % num_n;
          if (to_fp16)
            sh->bits[rr] &= ~(1ull << cc);
          else
            sh->bits[rr] |= 1ull << cc;
          return false;
        });
      }
      __syncthreads();
    }
  }

  // ---------------- weighted retarget (:273-326) ----------------
  if (a.pattern >= kBand) {
    long long tot = 0, cur = 0;
    for (int r = tid; r < num_m; r += kThreads) {
      const int tiles = sh->tiles[r];
      const uint64_t vis = visited_cols(g, tiles);
      const uint64_t b = sh->bits[r] & vis;
      sh->bits[r] = b;
      const int full = tiles / g.group, rem = tiles % g.group;
      const int nfull = min(full, num_n);
      tot += static_cast<long long>(nfull) * g.group + ((rem != 0 && full < num_n) ? rem : 0);
      cur += static_cast<long long>(__popcll(b & range_mask(0, nfull))) * g.group;
      if (rem != 0 && full < num_n && ((b >> full) & 1ull)) cur += rem;
    }
    tot = block_sum(tot, sh);
    cur = block_sum(cur, sh);
    if (tot > 0) {
      const long long target = py_round(static_cast<double>(tot) * p);
      if (cur != target) {
        const bool add = cur < target;
        const int C = collect_cells(sh, g, [&](int r) {
          return (add ? ~sh->bits[r] : sh->bits[r]) & visited_cols(g, sh->tiles[r]);
        });
        if (warp0) {
          // torch.Generator().manual_seed(42) for the candidate order.
          mt_seed(sh, mts, 42u);
          long long current = cur;
          shuffled_walk(sh, mts, sh->u.cand, C, C, [&](int cell) {
            const int rr = cell / num_n, cc = cell % num_n;
            const int w = tile_weight(g, sh->tiles[rr], cc);
            const long long proposed = add ? current + w : current - w;
            if (llabs(target - proposed) <= llabs(target - current)) {
              if (add)
                sh->bits[rr] |= 1ull << cc;
              else
                sh->bits[rr] &= ~(1ull << cc);
              current = proposed;
            }
            return current == target;
          });
          if (tid == 0) {
            // the heaviest cell sits in the last query block, which visits the most tiles
            const int last = sh->tiles[num_m - 1];
            const int max_w = last >= g.group ? g.group : last % g.group;
            if (llabs(current - target) > max_w) record_error(a.err, 1);
          }
        }
      }
    }
  }
  __syncthreads();
  for (int r = tid; r < num_m; r += kThreads) a.out[r] = sh->bits[r];
}

// FP16 columns of the global pattern (:507-526), resolved on the host.
uint64_t global_columns(const tm_map_params* p, int num_n) {
  long long tgc = static_cast<long long>(std::nearbyint(num_n * (1.0 - p->percentage)));
  tgc = tgc < 1 ? 1 : (tgc > num_n ? num_n : tgc);
  bool have[kMaxCols] = {};
  int count = 0;
  auto add_pos = [&](long long pos) {
    if (pos < 0 || pos >= p->seq_len) return;
    const long long col = pos / p->block_n_mask;
    if (col < num_n && !have[col]) {
      have[col] = true;
      ++count;
    }
  };
  if (p->key_pos != nullptr) {
    for (int i = 0; i < p->num_key_pos; ++i) add_pos(p->key_pos[i]);
  } else {
    for (int i = 0; i < 4 && i < p->seq_len; ++i) add_pos(i);
  }
  while (count < tgc && count < num_n) {
    for (int col = 0; col < num_n; ++col) {
      if (!have[col]) {
        have[col] = true;
        ++count;
        break;
      }
    }
  }
  uint64_t m = 0;
  int taken = 0;
  for (int col = 0; col < num_n && taken < tgc; ++col) {
    if (have[col]) {
      m |= 1ull << col;
      ++taken;
    }
  }
  return m;
}

}  // namespace pmap
}  // namespace tilemix

extern "C" int tm_build_precision_map(const tm_map_params* p, uint64_t* out, int* error_flag, void* stream) {
  using namespace tilemix::pmap;
  if (p == nullptr || out == nullptr) return TM_ERR_NULL;
  if (p->seq_len <= 0 || p->block_m <= 0 || p->block_n_mask <= 0 || p->compute_block_n <= 0) return TM_ERR_SHAPE;
  if (p->block_n_mask % p->compute_block_n != 0) return TM_ERR_SHAPE;
  if (p->pattern < TM_MAP_ZERO || p->pattern > TM_MAP_SPTRANS) return TM_ERR_SHAPE;
  const long long num_m = (static_cast<long long>(p->seq_len) + p->block_m - 1) / p->block_m;
  const long long num_n = (static_cast<long long>(p->seq_len) + p->block_n_mask - 1) / p->block_n_mask;
  if (num_n > kMaxCols) return TM_ERR_SHAPE;
  if (num_m > kMaxRows || num_m * num_n > kMaxCells) return TM_ERR_UNSUPPORTED;
  if (p->pattern >= TM_MAP_BAND && !(p->percentage >= 0.0 && p->percentage <= 1.0)) return TM_ERR_SHAPE;
  if (p->pattern == TM_MAP_SPTRANS && p->stride <= 0) return TM_ERR_SHAPE;
  if (p->pattern == TM_MAP_BIGBIRD && (p->num_global_block < 0 || p->num_rand_block < 0)) return TM_ERR_SHAPE;
  if (p->pattern == TM_MAP_GLOBAL && p->num_key_pos > 0 && p->key_pos == nullptr) return TM_ERR_NULL;
  MapArgs a;
  a.seq_len = p->seq_len;
  a.block_m = p->block_m;
  a.block_n_mask = p->block_n_mask;
  a.compute_block_n = p->compute_block_n;
  a.pattern = p->pattern;
  a.percentage = p->percentage;
  a.stride = p->stride;
  a.c = p->c;
  a.global_cols = p->pattern == TM_MAP_GLOBAL ? global_columns(p, static_cast<int>(num_n)) : 0ull;
  a.num_global_block = p->num_global_block;
  a.num_rand_block = p->num_rand_block;
  a.out = out;
  a.err = error_flag;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TM_ERR_LAUNCH;
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(build_map_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(Shared))) != cudaSuccess)
      return TM_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  build_map_kernel<<<1, kThreads, sizeof(Shared), static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_LAUNCH;
}
