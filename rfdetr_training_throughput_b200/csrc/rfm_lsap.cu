// Batched exact rectangular linear assignment with SciPy's semantics.  For
// large batches one warp solves one problem (a CTA holds one to four such
// warps); a batch that runs in one wave of CTAs gets a CTA of four warps per
// problem (two when more than four problems share an SM), which spread each
// scan step over the CTA (MULTI, below).
//
// Replaces lsap_kernel / batch_lap_cuda (kernels_lap.py:88-305) and the device
// unpack of the device_indices patch (patches.py:379-418).
//
// Algorithm: the shortest-augmenting-path method of SciPy's rectangular_lsap
// (SciPy 1.18.1; Crouse, IEEE TAES 2016), which the reference ports at
// kernels_lap.py:127-261.  Unlike that port, this kernel reproduces SciPy's
// result index-for-index, ties included:
//   * float64 duals and path costs on the float32 costs, with the reduced
//     cost evaluated as ((minv + c) - u[i]) - v[j];
//   * SciPy's orientation rule: solved transposed (rows = targets) only when
//     the matrix is tall (num_targets < num_queries);
//   * SciPy's tie rule.  SciPy scans the `remaining` array in order and keeps
//     a strictly smaller path cost, or an equal one whose column is free.  Over
//     a whole scan that selects, among the columns at the minimum, the LAST
//     free one in scan order if any is free, else the FIRST one.  The warp
//     reproduces it as a lexicographic argmin over (cost, key) with
//     key = free ? B-1-pos : B+pos, where pos is the column's position in
//     `remaining`, maintained with SciPy's reverse fill and swap-with-last
//     removal.
//
// Layout.  Lane l owns solver columns l, l+32, ..., l+32(K-1).  Its columns'
// path costs and "still remaining" and "free" bits live in registers; their
// duals v and tie keys too (REGS and EARLY variants) or in shared memory (WIDE,
// for batches of more than 64 problems per SM: fewer registers, more resident
// warps).  The warp argmin is three redux.sync minimum steps over an
// order-preserving integer image of the float64 cost and the key.  Row duals
// (float64), the matching, the path and `remaining` (position -> column) live
// in shared memory as int16.  The dual update needs no cross-lane traffic:
// every visited non-sink column j owns exactly one tree row, row4col[j], so its
// lane applies u[row4col[j]] += minv - spc[j] and v[j] -= minv - spc[j] itself.
//
// One pass over the tile validates it and computes every row's first pick (the
// argmin of its first scan with u = v = 0 and all columns free); a row whose
// pick is still valid at its turn commits it in O(1), which is exact (see the
// comment at the shortcut).  A scan issues all of a lane's loads before the
// first compare; the EARLY variant (problems with 64 or more rows: long
// searches) issues the next scan's row as soon as the argmin names it, before
// the current step's bookkeeping.  The MULTI variants keep as many of a
// problem's rows in shared memory as its CTA's share of the SM holds and run
// each step as a per-thread scan of a few columns, one warp argmin, a
// cross-warp combine through shared memory and one barrier.
//
// Cost source.  Element (q, t) of a problem is read at
// cost[cost_offset + q * stride_q + t * stride_t], so the solver reads either
// the query-major compact matrix or its target-major transpose in place.  The
// problem is used in the solver's orientation (rows = targets when
// transposed).  When every problem's solver rows are contiguous in the source,
// persistent warps (warp w starts on problem w) pull further problems
// (largest first) from a counter in the workspace, claiming the next one before
// the current one's epilogue, and read rows straight from L2/HBM (DIRECT).  Otherwise the host
// packs problems, sorted by tile size, into CTAs of up to four warps under a
// shared-memory budget; a tile within the cap is staged into shared memory
// with cp.async (SHARED), a larger one read in place (DIRECT) or first
// transposed into the caller's workspace (SCRATCH).
//
// Pushed pairs (rfm_lsap_push / rfm_match_push, the sharded sweep's exchange):
// the epilogue also stores each problem's pairs into every destination of a
// push list in device memory (other ranks' gathered buffers, peer memory over
// NVLink), rebuilt from shared memory after the local stores.  The list's
// pointer travels in the argument words only dense batches use, so the
// parameter block, and the code of every kernel that is not pushing, is
// unchanged.
//
// Termination: every inner step removes one column from `remaining`, so each
// augmentation is bounded by num_cols steps (kernels_lap.py:78-84,147-148);
// the path flip is bounded by num_rows + 1 steps.  There are no spin-waits.
#include <math_constants.h>

#include <climits>
#include <mutex>
#include <vector>

#include "rfm_common.cuh"

namespace rfm {
namespace {

constexpr int kSmemPerSm = 228 * 1024;
constexpr int kSmemPerCtaReserved = 1024;
constexpr int kSmemPerBlockMax = 227 * 1024;
constexpr int64_t kTileCapDefault = 16384;  // floats: 64 KB of staged cost per warp
constexpr int kMaxWarpsPerCta = 4;

// Solver variants: REGS keeps column duals and tie keys in registers; WIDE keeps
// them in shared memory (large batches); EARLY is REGS with each scan's row
// requested as soon as the row is known, before the previous step's
// bookkeeping, which pays off when searches run long (batches whose problems
// have at least kEarlyMinRows rows).  COOP is REGS with one problem per CTA
// whose four warps share the load pass (a quarter of the rows each, so a
// problem's rows cost a quarter of the round trips) before warp 0 solves it
// alone: small batches, where every problem is resident at once and the
// step's time is the slowest problem's latency.  MULTI is for batches of long
// problems (searches of many steps) small enough to run in one wave of
// four-warp CTAs: one problem per CTA, whose shared memory is the SM's divided
// by the CTAs the SM holds; the load pass keeps as many of the problem's rows
// there as fit (the rest are read from L2), and every step of a search is spread
// over the four warps.  MULTI_COPY is MULTI for batches whose solver rows are
// not all contiguous in the source: those problems are staged as a transposed
// copy, partly in scratch.
// MULTI_TWO and MULTI_COPY_TWO are the same with two warps per problem, for
// waves of more than kMultiFourPerSm problems per SM.
enum Variant : int {
  kVarRegs = 0,
  kVarWide = 1,
  kVarEarly = 2,
  kVarCoop = 3,
  kVarMulti = 5,
  kVarMultiCopy = 6,
  kVarMultiTwo = 7,
  kVarMultiCopyTwo = 8,
  kVarMultiTwoQueue = 9,      // MULTI_TWO with fewer CTAs than problems, claiming from a counter
  kVarMultiCopyTwoQueue = 10  // the same for MULTI_COPY_TWO (dense batches)
};
__host__ __device__ constexpr bool multi_variant(int v) { return v >= kVarMulti && v <= kVarMultiCopyTwoQueue; }
__host__ __device__ constexpr bool copy_variant(int v) {
  return v == kVarMultiCopy || v == kVarMultiCopyTwo || v == kVarMultiCopyTwoQueue;
}
__host__ __device__ constexpr bool queue_variant(int v) { return v == kVarMultiTwoQueue || v == kVarMultiCopyTwoQueue; }
// Warps that share one problem's searches in a MULTI variant.
__host__ __device__ constexpr int multi_warps(int v) {
  return (v == kVarMultiTwo || v == kVarMultiCopyTwo || queue_variant(v)) ? 2 : 4;
}
// Variants with one problem per CTA; none exists for the 1024-column layout,
// and neither does WIDE.
__host__ __device__ constexpr bool cta_variant(int v) { return v == kVarCoop || multi_variant(v); }
__host__ __device__ constexpr bool narrow_only(int v) { return v == kVarWide || cta_variant(v); }
constexpr int kEarlyMinRows = 64;
// Batches (of up to 320 columns) that run in one wave of MULTI CTAs (their
// shared memory divided among the CTAs an SM holds): four warps per problem up
// to kMultiFourPerSm CTAs per SM, two warps up to kMultiTwoPerSm (or the CTAs
// that fit, registers permitting).  Past four per SM four-warp problems issue
// too much to share an SM well; two warps per problem then run their steps
// faster than one warp does, up to the register file's limit; beyond that
// (kVarMultiTwoQueue) the CTAs that fit claim the remaining problems.  On the
// short problems of the sweep geometry that beat one warp per problem up to
// about 36 problems per SM and lost at 45; larger batches take the one-warp
// layouts.
constexpr int kMultiFourPerSm = 4;
constexpr int kMultiTwoPerSm = 40;
// Batches with more than this many problems per SM use the wide layout.
constexpr int kWideProblemsPerSm = 64;
// Register budget.  The instantiations up to 320 columns run four CTAs of four
// warps per SM (at most 128 registers a thread), or five in the wide layout,
// which keeps the column duals and tie keys in shared memory (at most 102): more
// resident warps for large batches at a longer chain per problem (on the
// 1024-image sweep six wide CTAs per SM ran 1.6 % slower, eight 13 %: the
// tighter budgets lengthen every warp's chain).  The 1024-column one keeps its
// per-lane arrays in registers.  (MULTI compiles to 96 registers, five CTAs per
// SM; capped at 80 or 64 for six or eight CTAs its searches ran 9 % and 22 %
// longer.)
__host__ __device__ constexpr int min_ctas_per_sm(int cols_per_lane, int variant) {
  return cols_per_lane > 10 ? 1 : (variant == kVarWide ? 5 : 4);
}
// Shared-memory budget of one CTA: four CTAs of four warps fill an SM.
constexpr int kCtaBudget = kSmemPerSm / 4 - kSmemPerCtaReserved;
// Tie keys: a free column at position pos gets kKeyBase - 1 - pos, a matched one
// kKeyBase + pos, so the smallest key is SciPy's pick among equal path costs.
constexpr unsigned kKeyBase = 1024u;
constexpr unsigned kNoKey = 0xffffffffu;
// In the search's registers a key is (tie key << kColBits) | column, so the
// warp's argmin names the column without a lookup in `remaining`.
constexpr int kColBits = 10;
constexpr unsigned kColMask = (1u << kColBits) - 1u;
// Persistent launches keep their problem counter at the start of the workspace.
constexpr int64_t kQueueBytes = 256;

enum Mode : int { kModeShared = 0, kModeDirect = 1, kModeScratch = 2 };

struct LsapArgs {
  const float* cost;
  int64_t stride_q, stride_t;
  const rfm_problem* problems;  // pair mode
  const int4* ctas;             // pair mode: {first problem, warps, slot bytes, 0} per CTA
  int num_problems;
  int dense_w;  // dense mode: uniform [P, W, T] problems
  // the two modes' own fields share these 8 bytes (the parameter block keeps its size)
  union {
    struct {
      int t;      // dense mode: tasks per problem
      int warps;  // dense mode: warps per CTA
    } dense;
    const rfm_pair_push* push;  // pair mode: push list in device memory (rfm_pair_push_store), or null
  } mode;
  int slot;              // dense and persistent modes: uniform shared-memory slot per warp
  int* queue;            // persistent mode: next-problem counter (zeroed before the launch)
  int claim_base;        // persistent mode: warps launched; warp w starts on problem w and
                         // claim c of the counter names problem claim_base + c
  int tile_cap;
  int max_rows;
  float* workspace;
  int64_t* q_out;  // pair mode: query indices; dense mode: matching [P, W]
  int64_t* t_out;
  int32_t* status;
};

// The problem in the solver's orientation: nr rows, nc columns, and the
// source strides of one row step (rs) and one column step (cs).
struct Shape {
  bool transposed;
  int nr, nc;
  int64_t rs, cs;
};

__host__ __device__ inline Shape solver_shape(int nq, int nt, int64_t sq, int64_t st) {
  Shape s;
  s.transposed = nt < nq;
  if (s.transposed) {
    s.nr = nt;
    s.nc = nq;
    s.rs = st;
    s.cs = sq;
  } else {
    s.nr = nq;
    s.nc = nt;
    s.rs = sq;
    s.cs = st;
  }
  return s;
}

// SHARED when the tile is within the cap and the warp's slot holds it.
__host__ __device__ inline int choose_mode(const Shape& s, int64_t tile_cap, int64_t slot_floats) {
  const int64_t t = static_cast<int64_t>(s.nr) * s.nc;
  if (t <= tile_cap && t <= slot_floats) return kModeShared;
  if (s.cs == 1) return kModeDirect;
  return kModeScratch;
}

__host__ __device__ inline int64_t fixed_warp_bytes(int cols_cap, int max_rows, bool wide = false) {
  // u and first-pick cost (float64), col4row and first-pick column (int16) per row;
  // the 32 lanes' visited masks; row4col, path, remaining (int16) per column; in
  // the wide layout also the column duals (float64) and tie keys (uint16)
  const int64_t b = static_cast<int64_t>(max_rows) * 20 + 128 + static_cast<int64_t>(cols_cap) * (wide ? 16 : 6);
  return (b + 15) & ~int64_t(15);
}

__host__ __device__ inline int64_t warp_bytes_for(int cols_cap, int max_rows, int64_t tile_floats) {
  return fixed_warp_bytes(cols_cap, max_rows) + ((tile_floats * 4 + 15) & ~int64_t(15));
}

// Order-preserving map of a float64 (NaN excluded) onto uint64; -0 and +0 map
// to the same value (x + 0.0 is +0.0 for either zero), as they compare equal.
__device__ __forceinline__ unsigned long long ordered_bits(double x) {
  const long long b = __double_as_longlong(x + 0.0);
  return b >= 0 ? (static_cast<unsigned long long>(b) | 0x8000000000000000ull)
                : ~static_cast<unsigned long long>(b);
}

__device__ __forceinline__ double from_ordered(unsigned long long o) {
  const unsigned long long b = (o & 0x8000000000000000ull) ? (o & 0x7fffffffffffffffull) : ~o;
  return __longlong_as_double(static_cast<long long>(b));
}

// Lexicographic (value, key) minimum over the warp with three redux.sync steps;
// every lane receives the winner.
__device__ __forceinline__ void warp_argmin(double& v, unsigned& key) {
  const unsigned long long o = ordered_bits(v);
  const unsigned hi = static_cast<unsigned>(o >> 32);
  const unsigned lo = static_cast<unsigned>(o);
  const unsigned mhi = __reduce_min_sync(kFullMask, hi);
  const unsigned mlo = __reduce_min_sync(kFullMask, hi == mhi ? lo : 0xffffffffu);
  key = __reduce_min_sync(kFullMask, (hi == mhi && lo == mlo) ? key : kNoKey);
  v = from_ordered((static_cast<unsigned long long>(mhi) << 32) | mlo);
}

__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

template <int K>
__device__ __forceinline__ void set_key(unsigned (&key)[K], int k_sel, unsigned value) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (k == k_sel) key[k] = value;
  }
}

// Load policies of the scan: shared tile, read-only global, L2-only global.
enum Load : int { kLoadShared = 0, kLoadGlobal = 1, kLoadScratch = 2 };

template <int L>
__device__ __forceinline__ float load_cost(const float* p) {
  if (L == kLoadShared) return *p;
  if (L == kLoadGlobal) return __ldg(p);
  return __ldcg(p);
}

// Issues the loads of one row's costs at the lane's columns in `mask`.
template <int K, int L>
__device__ __forceinline__ void load_row(const float* row, int lane, unsigned mask, float (&cf)[K]) {
#pragma unroll
  for (int k = 0; k < K; ++k) cf[k] = (mask & (1u << k)) ? load_cost<L>(row + lane + 32 * k) : 0.0f;
}

// One scan step of the augmenting-path search over the lane's columns, on a
// row whose costs load_row() requested into cf (all of a lane's loads are in
// flight before the first is used: a row read from memory costs one round
// trip, not one per column).  Column duals and tie keys come from registers,
// or in the wide layout from shared memory (every remaining column's key is
// read, so the (cost, key) comparison compiles to selects, not branches).
//
// The step is branch-free: every column's reduced cost is computed (removed
// columns are masked out afterwards), so the K chains of float64 arithmetic
// overlap, and the lane's lexicographic (path cost, key) minimum is a tree of
// depth log2(K) instead of a chain of K compares.  Keys are unique, so any
// reduction order gives the same minimum.  The key carries the column in its
// low kColBits bits (tie order is decided by the position bits above them).
template <int K, bool kWide>
__device__ __forceinline__ void scan_row(const float (&cf)[K], int lane, int i, double minv, double ui,
                                         const double (&v)[K], const double* v_s, double (&spc)[K],
                                         const unsigned (&key)[K], const uint16_t* key_s, unsigned rem,
                                         int16_t* path_s, double& bv, unsigned& bk) {
  if constexpr (K > 10) {  // 1024 columns: the per-lane arrays leave no registers for the tree
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (rem & (1u << k)) {
        const int j = lane + 32 * k;
        const double r = ((minv + static_cast<double>(cf[k])) - ui) - (kWide ? v_s[j] : v[k]);
        if (r < spc[k]) {
          spc[k] = r;
          path_s[j] = static_cast<int16_t>(i);
        }
        const unsigned kj =
            kWide ? (static_cast<unsigned>(key_s[j]) << kColBits) | static_cast<unsigned>(j) : key[k];
        if (spc[k] < bv || (spc[k] == bv && kj < bk)) {
          bv = spc[k];
          bk = kj;
        }
      }
    }
  } else {
    double rv[K];
    unsigned rk[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int j = lane + 32 * k;
      const bool live = (rem >> k) & 1u;
      const double r = ((minv + static_cast<double>(cf[k])) - ui) - (kWide ? v_s[j] : v[k]);
      const bool better = live && r < spc[k];
      if (better) path_s[j] = static_cast<int16_t>(i);
      spc[k] = better ? r : spc[k];
      rv[k] = live ? spc[k] : CUDART_INF;
      rk[k] = live ? (kWide ? (static_cast<unsigned>(key_s[j]) << kColBits) | static_cast<unsigned>(j) : key[k])
                   : kNoKey;
    }
#pragma unroll
    for (int stride = 1; stride < K; stride *= 2) {
#pragma unroll
      for (int k = 0; k + stride < K; k += 2 * stride) {
        const bool take = rv[k + stride] < rv[k] || (rv[k + stride] == rv[k] && rk[k + stride] < rk[k]);
        rv[k] = take ? rv[k + stride] : rv[k];
        rk[k] = take ? rk[k + stride] : rk[k];
      }
    }
    bv = rv[0];
    bk = rk[0];
  }
}

// Order-preserving map of a float (NaN excluded) onto uint32.
__device__ __forceinline__ unsigned ordered32(float x) {
  const unsigned b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float from_ordered32(unsigned o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// NaN-propagating minimum (PTX min.NaN): a NaN operand makes the result NaN.
__device__ __forceinline__ float min_nan(float x, float y) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(x), "f"(y));
  return r;
}

// NaN-propagating minimum of the lane's entries of one row.
template <int K>
__device__ __forceinline__ float lane_min(const float (&x)[K]) {
  float m = x[0];
#pragma unroll
  for (int k = 1; k < K; ++k) m = min_nan(m, x[k]);
  return m;
}

// First pick of one row when every column is free and v = 0: the smallest
// cost, ties to the smallest column; lane 0 records it (column -1 when the
// row's minimum is +inf, which leaves the row to the full search).  m is
// lane_min(x); entries past the row end hold +inf.  A row holding NaN has
// m = NaN, is flagged by the caller's check (which takes the same m) and is
// never solved, so whatever it records here is unused; without NaN, m is the
// plain minimum.
template <int K>
__device__ __forceinline__ void record_first_pick(const float (&x)[K], float m, int lane, int nc, int row,
                                                  double* pick_m_s, int16_t* pick_w_s) {
  unsigned bj = 0xffffu;
#pragma unroll
  for (int k = K - 1; k >= 0; --k) bj = x[k] == m ? static_cast<unsigned>(lane + 32 * k) : bj;
  const unsigned o = ordered32(m + 0.0f);  // -0 and +0 tie, as the doubles (0 + c) do
  const unsigned mo = __reduce_min_sync(kFullMask, o);
  const unsigned mj = __reduce_min_sync(kFullMask, o == mo ? bj : 0xffffu);
  if (lane == 0) {
    const float mf = from_ordered32(mo);
    pick_m_s[row] = static_cast<double>(mf);
    pick_w_s[row] = static_cast<int16_t>(mf == CUDART_INF_F || mj >= static_cast<unsigned>(nc) ? -1 : static_cast<int>(mj));
  }
}

// Persistent launches: lane 0 claims the warp's next problem.  It is called
// before a problem's epilogue, so the atomic's round trip overlaps the stores.
__device__ __forceinline__ int claim_next(const LsapArgs& a, int lane) {
  return (a.queue != nullptr && lane == 0) ? atomicAdd(a.queue, 1) + a.claim_base : 0;
}

// MULTI: the searches of one problem run on all the warps of its CTA (four, or
// two in the _TWO variants).  Thread t owns columns t, t + 32W, ... (K3 of
// them), so a scan step is K3 columns per thread instead of up to ten per lane;
// each warp reduces its (path cost, key) minimum with redux.sync, the lane
// holding it posts it to a shared slot (double-buffered by step parity, so one
// barrier per step suffices: a warp can only overwrite a slot after every warp
// has passed the next barrier, which it reaches after reading the slot), and
// every thread combines the W posts.
// Every thread then holds the same argmin, so the rest of the step (next row,
// swap-with-last removal of `remaining`, the tie key of the moved column) runs
// without further exchange.  Same arithmetic and tie rule as the one-warp
// search: the result is identical.
struct MultiShared {
  double* u;
  double* pick_m;
  int16_t* col4row;
  int16_t* pick_w;
  int16_t* row4col;
  int16_t* path;
  int16_t* rem;
  unsigned* vis;   // visited-column bitmap of the last search (bit j & 31 of word j >> 5)
  double2* post;  // [2][4] step posts: (path cost, key)
  int* flag;
};
constexpr int kMultiPostBytes = 144;
// [0, 128): the step posts; 128: the flip flag; kMultiClaimOffset: a persistent
// MULTI CTA's next problem.
constexpr int kMultiClaimOffset = 136;
// A MULTI key also carries the column's matched row plus one (0 when free) in
// its low kRowBits bits, so the step's argmin names the next row directly.
// Columns are at most 320 here, and rows at most columns.
constexpr int kRowBits = 9;
constexpr unsigned kRowMask = (1u << kRowBits) - 1u;
constexpr int kTieShift = kColBits + kRowBits;

// A post is (path cost, key) with the key in the low word of .y.
__device__ __forceinline__ double key_as_double(unsigned k) {
  return __longlong_as_double(static_cast<long long>(k));
}

__device__ __forceinline__ bool post_less(const double2& x, const double2& y) {
  const unsigned kx = static_cast<unsigned>(__double_as_longlong(x.y));
  const unsigned ky = static_cast<unsigned>(__double_as_longlong(y.y));
  return x.x < y.x || (x.x == y.x && kx < ky);
}

template <int K3, int kThreads>
__device__ __forceinline__ void multi_row(const float* row, int t, unsigned mask, float (&cf)[K3]) {
#pragma unroll
  for (int k = 0; k < K3; ++k) cf[k] = (mask & (1u << k)) ? row[t + kThreads * k] : 0.0f;
}

// Rows in global memory: the read-only source (kLoadGlobal) or the scratch copy
// this kernel wrote (kLoadScratch, read through L2).
template <int K3, int L, int kThreads>
__device__ __forceinline__ void multi_row_global(const float* row, int t, unsigned mask, float (&cf)[K3]) {
#pragma unroll
  for (int k = 0; k < K3; ++k) cf[k] = (mask & (1u << k)) ? load_cost<L>(row + t + kThreads * k) : 0.0f;
}

// Searches and commits every row of a problem whose costs are staged (rows
// [0, staged) at `tile`, pitch nc) or read from `src` (row pitch rs; kWritten
// when the rows are the scratch copy of this launch).  Called by all
// threads after the load pass; returns the problem's status.
template <int K3, bool kWritten, int kWarps>
__device__ int multi_search(const MultiShared& m, const float* tile, const float* src, int64_t rs, int staged,
                            int nr, int nc, bool bad) {
  constexpr int kMultiWarps = kWarps;
  constexpr int kMultiThreads = 32 * kWarps;
  constexpr int kMultiShift = kWarps == 2 ? 6 : 7;
  static_assert(kWarps == 2 || kWarps == 4, "two or four warps per problem");
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int warp = t >> 5;
  unsigned valid = 0;
#pragma unroll
  for (int k = 0; k < K3; ++k) {
    if (t + kMultiThreads * k < nc) valid |= 1u << k;
  }
  unsigned freem = valid;
  double v[K3];
#pragma unroll
  for (int k = 0; k < K3; ++k) v[k] = 0.0;
  int code = bad ? RFM_STATUS_INVALID : RFM_STATUS_OK;
  int parity = 0;

  for (int cur = 0; cur < nr && code == RFM_STATUS_OK; ++cur) {
    const int w = m.pick_w[cur];
    if (w >= 0 && m.row4col[w] < 0) {  // still valid: commit the trivial augmentation
      const double mv = m.pick_m[cur];
      __syncthreads();  // every thread has read row4col[w] before it changes
      if (t == 0) {
        m.u[cur] += mv;
        m.row4col[w] = static_cast<int16_t>(cur);
        m.col4row[cur] = static_cast<int16_t>(w);
      }
      if ((w & (kMultiThreads - 1)) == t) freem &= ~(1u << (w >> kMultiShift));
      __syncthreads();
      continue;
    }

    double spc[K3];
    unsigned key[K3];
#pragma unroll
    for (int k = 0; k < K3; ++k) {
      const int j = t + kMultiThreads * k;
      const unsigned pos = static_cast<unsigned>(nc - 1 - j);
      spc[k] = CUDART_INF;
      const unsigned kv = (freem & (1u << k)) ? kKeyBase - 1u - pos : kKeyBase + pos;
      const unsigned row1 = j < nc ? static_cast<unsigned>(m.row4col[j] + 1) : 0u;
      key[k] = (kv << kTieShift) | (static_cast<unsigned>(j) << kRowBits) | row1;
      if (j < nc) m.rem[nc - 1 - j] = static_cast<int16_t>(j);
    }
    unsigned rem = valid;
    int i = cur;
    int nrem = nc;
    int sink = -1;
    double minv = 0.0;
    float cf[K3];
    const auto issue_row = [&](int r) {
      if (r < staged) {
        multi_row<K3, kMultiThreads>(tile + r * nc, t, rem, cf);
      } else {
        multi_row_global<K3, kWritten ? kLoadScratch : kLoadGlobal, kMultiThreads>(src + r * rs, t, rem, cf);
      }
    };
    issue_row(cur);
    __syncthreads();  // `remaining` is initialised
    for (int it = 0; it < nc; ++it) {
      const double ui = m.u[i];
      double bv = CUDART_INF;
      unsigned bk = kNoKey;
      {
        double rv[K3];
        unsigned rk[K3];
#pragma unroll
        for (int k = 0; k < K3; ++k) {
          const int j = t + kMultiThreads * k;
          const bool live = (rem >> k) & 1u;
          const double r = ((minv + static_cast<double>(cf[k])) - ui) - v[k];
          const bool better = live && r < spc[k];
          if (better) m.path[j] = static_cast<int16_t>(i);
          spc[k] = better ? r : spc[k];
          rv[k] = live ? spc[k] : CUDART_INF;
          rk[k] = live ? key[k] : kNoKey;
        }
#pragma unroll
        for (int stride = 1; stride < K3; stride *= 2) {
#pragma unroll
          for (int k = 0; k + stride < K3; k += 2 * stride) {
            const bool take = rv[k + stride] < rv[k] || (rv[k + stride] == rv[k] && rk[k + stride] < rk[k]);
            rv[k] = take ? rv[k + stride] : rv[k];
            rk[k] = take ? rk[k + stride] : rk[k];
          }
        }
        bv = rv[0];
        bk = rk[0];
      }
      // the warp's minimum: one redux.sync on the high word of the ordered
      // path cost; only when several lanes share that word do the low word and
      // the key decide (two more).  The lane holding the minimum posts it.
      {
        const unsigned long long o = ordered_bits(bv);
        const unsigned hi = static_cast<unsigned>(o >> 32);
        const unsigned mhi = __reduce_min_sync(kFullMask, hi);
        const unsigned tied = __ballot_sync(kFullMask, hi == mhi);
        bool mine = hi == mhi;
        if (__popc(tied) > 1) {
          const unsigned lo = static_cast<unsigned>(o);
          const unsigned mlo = __reduce_min_sync(kFullMask, mine ? lo : 0xffffffffu);
          mine = mine && lo == mlo;
          const unsigned mk = __reduce_min_sync(kFullMask, mine ? bk : kNoKey);
          mine = mine && bk == mk;
        }
        if (mine) m.post[parity * kMultiWarps + warp] = make_double2(bv, key_as_double(bk));
      }
      __syncthreads();
      {
        // fixed-shape tree over the warps' posts (keys are unique: any order agrees)
        double2 pw[kMultiWarps];
#pragma unroll
        for (int q = 0; q < kMultiWarps; ++q) pw[q] = m.post[parity * kMultiWarps + q];
#pragma unroll
        for (int stride = 1; stride < kMultiWarps; stride *= 2) {
#pragma unroll
          for (int q = 0; q + stride < kMultiWarps; q += 2 * stride) {
            pw[q] = post_less(pw[q + stride], pw[q]) ? pw[q + stride] : pw[q];
          }
        }
        bv = pw[0].x;
        bk = static_cast<unsigned>(__double_as_longlong(pw[0].y));
      }
      parity ^= 1;
      if (bv == CUDART_INF) {
        code = RFM_STATUS_INFEASIBLE;
        break;
      }
      const int js = static_cast<int>((bk >> kRowBits) & kColMask);
      const int rj = static_cast<int>(bk & kRowMask) - 1;
      if (rj >= 0) issue_row(rj);  // the next scan's row, before this step's bookkeeping
      const unsigned tk = bk >> kTieShift;
      const int ps = static_cast<int>(tk < kKeyBase ? kKeyBase - 1u - tk : tk - kKeyBase);
      // swap-with-last removal; the write is read after the next step's barrier
      const int jl = m.rem[nrem - 1];
      if (t == 0) m.rem[ps] = static_cast<int16_t>(jl);
      if ((jl & (kMultiThreads - 1)) == t) {
        const int kl = jl >> kMultiShift;
        const unsigned kv = ((freem >> kl) & 1u) ? kKeyBase - 1u - ps : kKeyBase + ps;
#pragma unroll
        for (int k = 0; k < K3; ++k) {
          if (k == kl) key[k] = (kv << kTieShift) | (key[k] & ((1u << kTieShift) - 1u));
        }
      }
      if ((js & (kMultiThreads - 1)) == t) rem &= ~(1u << (js >> kMultiShift));
      --nrem;
      minv = bv;
      if (rj < 0) {
        sink = js;
        break;
      }
      i = rj;
    }
    if (code != RFM_STATUS_OK) break;
    if (sink < 0) {
      code = RFM_STATUS_NO_SINK;
      break;
    }

    // dual update over the tree: every read of u in the search came before the
    // last step's barrier, and each visited column's row is updated by its owner
    const unsigned visited = valid & ~rem;
    bool raised = false;
#pragma unroll
    for (int k = 0; k < K3; ++k) {
      if (visited & (1u << k)) {
        const int j = t + kMultiThreads * k;
        const double d = minv - spc[k];
        raised |= d < 0.0;
        if (j != sink) m.u[m.row4col[j]] += d;
        v[k] -= d;
      }
    }
    if (t == 0) m.u[cur] += minv;
    raised = __syncthreads_or(raised) != 0;  // also publishes path, u and v

    if (t == 0) {
      int flipped = 0;
      int j = sink;
      for (int step = 0; step <= nr; ++step) {
        const int ii = m.path[j];
        m.row4col[j] = static_cast<int16_t>(ii);
        const int prev = m.col4row[ii];
        m.col4row[ii] = static_cast<int16_t>(j);
        j = prev;
        if (ii == cur) {
          flipped = 1;
          break;
        }
      }
      *m.flag = flipped;
    }
    if ((sink & (kMultiThreads - 1)) == t) freem &= ~(1u << (sink >> kMultiShift));
#pragma unroll
    for (int k = 0; k < K3; ++k) {
      const unsigned b = __ballot_sync(kFullMask, (visited >> k) & 1u);
      if (lane == 0) m.vis[warp + kMultiWarps * k] = raised ? 0xffffffffu : b;
    }
    __syncthreads();
    if (*m.flag == 0) code = RFM_STATUS_NO_SINK;
    // drop the pending picks this search visited (all of them if a dual went down)
    for (int r = cur + 1 + t; r < nr; r += kMultiThreads) {
      const int pw = m.pick_w[r];
      if (pw >= 0 && ((m.vis[pw >> 5] >> (pw & 31)) & 1u)) m.pick_w[r] = -1;
    }
    __syncthreads();
  }
  __syncthreads();
  return code;
}

// Solves problem p with the warp's shared-memory slot at `base` (`slot` bytes).
// Returns, in lane 0, the next problem a persistent warp claimed.
template <int K, bool kDense, int kVariant>
__device__ __forceinline__ int solve_problem(const LsapArgs& a, int p, unsigned char* base, int slot,
                                             int lane) {
  constexpr int kCols = 32 * K;
  constexpr bool kWide = kVariant == kVarWide;
  constexpr bool kCopy = copy_variant(kVariant);
  constexpr bool kMulti = multi_variant(kVariant);
  constexpr int kMultiWarps = multi_warps(kVariant);
  constexpr bool kStage = kMulti;  // rows [0, staged) kept in shared memory
  constexpr bool kEarly = kVariant == kVarEarly || kStage;
  constexpr bool kCoop = kVariant == kVarCoop || kStage;
  constexpr int kLoadWarps = kMulti ? kMultiWarps : (kCoop ? kMaxWarpsPerCta : 1);
  const int warp = kCoop ? static_cast<int>(threadIdx.x >> 5) : 0;
  int64_t cost_off, out_off, scratch_off;
  int nq, nt, qbase;
  if (kDense) {
    nq = a.dense_w;
    nt = a.mode.dense.t;
    cost_off = static_cast<int64_t>(p) * a.dense_w * a.mode.dense.t;
    out_off = static_cast<int64_t>(p) * a.dense_w;
    scratch_off = cost_off;
    qbase = 0;
  } else {
    const rfm_problem d = a.problems[p];
    cost_off = d.cost_offset;
    out_off = d.out_offset;
    scratch_off = d.scratch_offset;
    nq = d.num_queries;
    nt = d.num_targets;
    qbase = d.query_base;
  }
  const Shape s = solver_shape(nq, nt, a.stride_q, a.stride_t);
  const int nr = s.nr;
  const int nc = s.nc;
  int64_t* q_out = a.q_out + out_off;
  int64_t* t_out = kDense ? nullptr : a.t_out + out_off;

  if (nr == 0) {
    grid_dependency_wait();
    const int next = kMulti ? 0 : claim_next(a, lane);  // a MULTI CTA claims in the kernel's loop
    if (kDense) {
      for (int w = lane; w < nq; w += 32) q_out[w] = -1;
    }
    if (a.status != nullptr && lane == 0 && warp == 0) a.status[p] = RFM_STATUS_OK;
    return next;
  }

  double* u_s = reinterpret_cast<double*>(base);
  double* pick_m_s = u_s + a.max_rows;
  double* v_s = pick_m_s + a.max_rows;  // wide layout only
  unsigned* vis_s = reinterpret_cast<unsigned*>(v_s + (kWide ? kCols : 0));
  int16_t* col4row_s = reinterpret_cast<int16_t*>(vis_s + 32);
  int16_t* pick_w_s = col4row_s + a.max_rows;
  int16_t* row4col_s = pick_w_s + a.max_rows;
  int16_t* path_s = row4col_s + kCols;
  int16_t* rem_s = path_s + kCols;
  uint16_t* key_s = reinterpret_cast<uint16_t*>(rem_s + kCols);  // wide layout only
  unsigned valid = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (lane + 32 * k < nc) valid |= 1u << k;
  }
  if (warp == 0) {
    for (int i = lane; i < nr; i += 32) {
      u_s[i] = 0.0;
      col4row_s[i] = -1;
    }
    for (int j = lane; j < nc; j += 32) {
      row4col_s[j] = -1;
      if (kWide) v_s[j] = 0.0;
    }
  }

  // ---- load the cost once: validate it (SciPy rejects NaN and -inf), keep
  // it on chip when it fits, and find every row's first pick ---------------
  // First picks (exact shortcut).  At its turn a row's first scan evaluates
  // ((0 + c) - u) - v[j] with u = 0 over all columns in reverse-fill order.
  // When the pick is a free column the search ends there: u[row] becomes the
  // minimum, v is unchanged (the sink's slack is exactly 0) and only the sink
  // turns matched.  The picks of all rows are therefore computed once, against
  // v = 0 with every column free (SciPy's tie rule then takes the smallest
  // column index; float order equals the order of the exactly promoted
  // doubles), and a row commits its pick in O(1) while it is still valid.  A
  // pick stays the exact argmin until its column is taken or visited by a full
  // search: full searches only lower v on the columns they visit (by
  // minv - spc >= 0), which raises those columns' reduced costs, and columns
  // only ever turn from free to matched, which raises their tie keys.  Should
  // rounding ever make a dual step negative, every pending pick is dropped.
  // a launch with programmatic stream serialization may start while the cost
  // kernel finishes: everything above only touched the descriptor and shared
  // memory, and every counter claim comes after this point
  grid_dependency_wait();
  const float* src = a.cost + cost_off;
  const int64_t fixed = fixed_warp_bytes(kCols, a.max_rows, kWide);
  float* tile = reinterpret_cast<float*>(base + fixed);
  const int mode = choose_mode(s, a.tile_cap, (slot - fixed) / 4);
  // MULTI: solver rows [0, staged) are kept in shared memory (all of them when the tile fits)
  const int staged =
      kStage ? min(nr, static_cast<int>((slot - fixed - (kMulti ? kMultiPostBytes : 0)) / 4 / nc)) : 0;
  bool bad = false;
  const float* rows = src;  // solver row i starts at rows + i * row_pitch
  int64_t row_pitch = s.rs;
  // chk: running NaN-propagating minimum of every entry; NaN or -inf in the
  // tile leaves it below -inf's successor (or NaN), which SciPy rejects
  float chk = CUDART_INF_F;
  if (s.cs == 1) {
    // solver rows are contiguous in the source: one coalesced pass over them,
    // kLoadRows rows per round trip (as many as the variant's register budget
    // holds without spilling: every row's loads are in flight together)
    constexpr int kLoadRows = (kWide || K > 10) ? 2 : (kEarly ? 4 : 6);
    for (int i = warp * kLoadRows; i < nr; i += kLoadWarps * kLoadRows) {
      float x[kLoadRows][K];
#pragma unroll
      for (int r = 0; r < kLoadRows; ++r) {
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int j = lane + 32 * k;
          x[r][k] = (j < nc && i + r < nr) ? __ldg(src + (i + r) * s.rs + j) : CUDART_INF_F;
        }
      }
      float m[kLoadRows];
#pragma unroll
      for (int r = 0; r < kLoadRows; ++r) {
        m[r] = lane_min<K>(x[r]);
        chk = min_nan(chk, m[r]);
      }
      if (kStage || mode == kModeShared) {
        const int keep = kStage ? staged : nr;
#pragma unroll
        for (int r = 0; r < kLoadRows; ++r) {
#pragma unroll
          for (int k = 0; k < K; ++k) {
            const int j = lane + 32 * k;
            if (j < nc && i + r < keep) tile[(i + r) * nc + j] = x[r][k];
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kLoadRows; ++r) {
        if (i + r < nr) record_first_pick<K>(x[r], m[r], lane, nc, i + r, pick_m_s, pick_w_s);
      }
    }
    if (!kStage && mode == kModeShared) {
      rows = tile;
      row_pitch = nc;
    }
  } else if (kCopy) {
    // the source runs along solver rows: the four warps stage a transposed
    // copy, rows [0, staged) in shared memory and the rest in the problem's
    // scratch (the launch only runs MULTI when every tile that does not fit
    // has scratch).  Consecutive lanes read consecutive solver rows, which are
    // consecutive in the source.
    float* scratch = a.workspace + (scratch_off < 0 ? 0 : scratch_off);
    // (the launch never leaves an unstaged tile without scratch; should it, the
    // problem is reported invalid and no memory outside it is touched)
    const bool scratch_ok = staged == nr || (scratch_off >= 0 && a.workspace != nullptr);
    const int copied = scratch_ok ? nr : staged;
    bad = !scratch_ok;
    // Each part is walked as elements e = j * rows + i, every thread striding by
    // the CTA's size; the (i, j) of the next element follow by carrying, without
    // a division.  Rows [0, on_chip) go to the tile by cp.async (every request
    // in flight before one wait); rows [on_chip, copied) go to scratch, four
    // loads in flight per thread.
    constexpr int kStride = 32 * kMultiWarps;
    const int on_chip = staged < copied ? staged : copied;
    if (on_chip > 0) {
      const int di = kStride % on_chip, dj = kStride / on_chip;
      int i = static_cast<int>(threadIdx.x) % on_chip;
      int j = static_cast<int>(threadIdx.x) / on_chip;
      for (; j < nc; i += di, j += dj) {
        if (i >= on_chip) {
          i -= on_chip;
          ++j;
          if (j >= nc) break;
        }
        cp_async4(tile + i * nc + j, src + i * s.rs + j * s.cs);
      }
    }
    const int off_chip = copied - on_chip;
    if (off_chip > 0) {
      const int di = kStride % off_chip, dj = kStride / off_chip;
      int i = static_cast<int>(threadIdx.x) % off_chip;
      int j = static_cast<int>(threadIdx.x) / off_chip;
      while (j < nc) {
        float x[4];
        int64_t at[4];
        int count = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (j < nc) {
            const int r = on_chip + i;
            x[u] = __ldg(src + r * s.rs + j * s.cs);
            at[u] = static_cast<int64_t>(r) * nc + j;
            count = u + 1;
          }
          i += di;
          j += dj;
          if (i >= off_chip) {
            i -= off_chip;
            ++j;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (u < count) scratch[at[u]] = x[u];
        }
      }
    }
    cp_async_wait_all();
    __syncthreads();
    for (int i = warp; i < copied; i += kMultiWarps) {
      float x[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int j = lane + 32 * k;
        x[k] = j >= nc ? CUDART_INF_F : (i < staged ? tile[i * nc + j] : __ldcg(scratch + static_cast<int64_t>(i) * nc + j));
      }
      const float m = lane_min<K>(x);
      chk = min_nan(chk, m);
      record_first_pick<K>(x, m, lane, nc, i, pick_m_s, pick_w_s);
    }
  } else if (warp == 0) {
    // the source runs along solver rows: stage a transposed copy first
    const int total = nr * nc;
    if (mode == kModeShared) {
      for (int e = lane; e < total; e += 32) {
        const int j = e / nr;
        const int i = e - j * nr;
        cp_async4(tile + i * nc + j, src + i * s.rs + j * s.cs);
      }
      cp_async_wait_all();
      __syncwarp();
      rows = tile;
    } else {
      float* scratch = a.workspace + scratch_off;
      for (int e = lane; e < total; e += 32) {
        const int j = e / nr;
        const int i = e - j * nr;
        scratch[static_cast<int64_t>(i) * nc + j] = __ldg(src + i * s.rs + j * s.cs);
      }
      __syncwarp();
      rows = scratch;
    }
    row_pitch = nc;
    for (int i = 0; i < nr; ++i) {
      float x[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int j = lane + 32 * k;
        x[k] = j >= nc ? CUDART_INF_F : (mode == kModeShared ? rows[i * nc + j] : __ldcg(rows + i * nc + j));
      }
      const float m = lane_min<K>(x);
      chk = min_nan(chk, m);
      record_first_pick<K>(x, m, lane, nc, i, pick_m_s, pick_w_s);
    }
  }
  bad = bad || !(chk > -CUDART_INF_F);
  bad = __any_sync(kFullMask, bad);
  if (kCoop) {
    // every warp's first picks and checks are in; warp 0 solves the problem
    // alone (MULTI: all four warps)
    bad = __syncthreads_or(bad) != 0;
    if (!kMulti && warp != 0) return 0;
  }

  unsigned freem = valid;
  int code = bad ? RFM_STATUS_INVALID : RFM_STATUS_OK;
  if constexpr (kMulti) {
    constexpr int K3 = (K + kMultiWarps - 1) / kMultiWarps;
    unsigned char* post = base + slot - kMultiPostBytes;
    const MultiShared ms{u_s, pick_m_s, col4row_s, pick_w_s, row4col_s, path_s, rem_s, vis_s,
                         reinterpret_cast<double2*>(post), reinterpret_cast<int*>(post + 128)};
    if constexpr (kCopy) {
      if (s.cs == 1) {
        code = multi_search<K3, false, kMultiWarps>(ms, tile, src, s.rs, staged, nr, nc, bad);
      } else {
        code = multi_search<K3, true, kMultiWarps>(ms, tile, a.workspace + scratch_off, nc, staged, nr, nc, bad);
      }
    } else {
      code = multi_search<K3, false, kMultiWarps>(ms, tile, src, s.rs, staged, nr, nc, bad);
    }
    if (warp != 0) return 0;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int j = lane + 32 * k;
      if (j < nc && row4col_s[j] >= 0) freem &= ~(1u << k);
    }
  } else {
    double v[K];
#pragma unroll
    for (int k = 0; k < K; ++k) v[k] = 0.0;
    __syncwarp();

    for (int cur = 0; cur < nr && code == RFM_STATUS_OK; ++cur) {
      const int w = pick_w_s[cur];
      if (w >= 0 && row4col_s[w] < 0) {  // still valid: commit the trivial augmentation
        const double m = pick_m_s[cur];
        __syncwarp();
        if (lane == 0) {
          u_s[cur] += m;
          row4col_s[w] = static_cast<int16_t>(cur);
          col4row_s[cur] = static_cast<int16_t>(w);
        }
        if ((w & 31) == lane) freem &= ~(1u << (w >> 5));
        __syncwarp();
        continue;
      }

      // ---- full shortest-augmenting-path search for row `cur` ---------------
      double spc[K];
      unsigned key[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int j = lane + 32 * k;
        const unsigned pos = static_cast<unsigned>(nc - 1 - j);  // remaining[it] = nc-1-it (reverse fill)
        spc[k] = CUDART_INF;
        const unsigned kv = (freem & (1u << k)) ? kKeyBase - 1u - pos : kKeyBase + pos;
        if (!kWide) key[k] = (kv << kColBits) | static_cast<unsigned>(j);
        if (j < nc) {
          if (kWide) key_s[j] = static_cast<uint16_t>(kv);
          rem_s[nc - 1 - j] = static_cast<int16_t>(j);
        }
      }
      unsigned rem = valid;
      int i = cur;
      int nrem = nc;
      int sink = -1;
      double minv = 0.0;
      __syncwarp();

      float cf[K];
      const auto issue_row = [&](int r) {
        const float* row = rows + r * row_pitch;
        if (mode == kModeShared) {
          load_row<K, kLoadShared>(row, lane, rem, cf);
        } else if (mode == kModeDirect) {
          load_row<K, kLoadGlobal>(row, lane, rem, cf);
        } else {
          load_row<K, kLoadScratch>(row, lane, rem, cf);
        }
      };
      if (kEarly) issue_row(cur);
      for (int it = 0; it < nc; ++it) {
        if (!kEarly) issue_row(i);
        const double ui = u_s[i];
        const int last = nrem - 1;
        const int jl = rem_s[last];
        double bv = CUDART_INF;
        unsigned bk = kNoKey;
        scan_row<K, kWide>(cf, lane, i, minv, ui, v, v_s, spc, key, key_s, rem, path_s, bv, bk);
        warp_argmin(bv, bk);
        if (bv == CUDART_INF) {
          code = RFM_STATUS_INFEASIBLE;
          break;
        }
        const int js = static_cast<int>(bk & kColMask);
        const int rj = row4col_s[js];
        if (kEarly && rj >= 0) issue_row(rj);  // the next scan's row, before this step's bookkeeping
        const unsigned tk = bk >> kColBits;
        const int ps = static_cast<int>(tk < kKeyBase ? kKeyBase - 1u - tk : tk - kKeyBase);
        __syncwarp();
        if (lane == 0) rem_s[ps] = static_cast<int16_t>(jl);  // swap-with-last removal
        if ((jl & 31) == lane) {
          const int kl = jl >> 5;
          const unsigned kv = ((freem >> kl) & 1u) ? kKeyBase - 1u - ps : kKeyBase + ps;
          if (kWide) {
            key_s[jl] = static_cast<uint16_t>(kv);
          } else {
            set_key<K>(key, kl, (kv << kColBits) | static_cast<unsigned>(jl));
          }
        }
        if ((js & 31) == lane) rem &= ~(1u << (js >> 5));
        nrem = last;
        minv = bv;
        __syncwarp();
        if (rj < 0) {
          sink = js;
          break;
        }
        i = rj;
      }
      if (code != RFM_STATUS_OK) break;
      if (sink < 0) {
        code = RFM_STATUS_NO_SINK;
        break;
      }

      // ---- dual update over the tree (lane-local, see header comment) -------
      const unsigned visited = valid & ~rem;
      bool raised = false;  // a visited column's v went up: rounding broke minv >= spc
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (visited & (1u << k)) {
          const int j = lane + 32 * k;
          const double d = minv - spc[k];
          raised |= d < 0.0;
          if (j != sink) u_s[row4col_s[j]] += d;
          if (kWide) {
            v_s[j] -= d;
          } else {
            v[k] -= d;
          }
        }
      }
      raised = __any_sync(kFullMask, raised);
      if (lane == 0) u_s[cur] += minv;
      __syncwarp();

      // ---- flip the alternating path ----------------------------------------
      int flipped = 1;
      if (lane == 0) {
        flipped = 0;
        int j = sink;
        for (int step = 0; step <= nr; ++step) {
          const int ii = path_s[j];
          row4col_s[j] = static_cast<int16_t>(ii);
          const int prev = col4row_s[ii];
          col4row_s[ii] = static_cast<int16_t>(j);
          j = prev;
          if (ii == cur) {
            flipped = 1;
            break;
          }
        }
      }
      if ((sink & 31) == lane) freem &= ~(1u << (sink >> 5));
      if (!__shfl_sync(kFullMask, flipped, 0)) code = RFM_STATUS_NO_SINK;

      // ---- drop the pending picks this search visited (all of them if some
      // column's reduced costs went down) ------------------------------------
      vis_s[lane] = raised ? 0xffffffffu : visited;
      __syncwarp();
      for (int r = cur + 1 + lane; r < nr; r += 32) {
        const int pw = pick_w_s[r];
        if (pw >= 0 && ((vis_s[pw & 31] >> (pw >> 5)) & 1u)) pick_w_s[r] = -1;
      }
      __syncwarp();
    }
  }

  // ---- epilogue: write the result in SciPy's order -------------------------
  const int next = kMulti ? 0 : claim_next(a, lane);
  if (kDense) {
    // matching[w] = task of worker w, -1 if none (kernels_lap.py:336-341)
    if (code != RFM_STATUS_OK) {
      for (int w = lane; w < nq; w += 32) q_out[w] = -1;
    } else if (s.transposed) {
      for (int w = lane; w < nc; w += 32) q_out[w] = row4col_s[w];
    } else {
      for (int w = lane; w < nr; w += 32) q_out[w] = col4row_s[w];
    }
  } else if (code != RFM_STATUS_OK) {
    for (int k = lane; k < nr; k += 32) {
      q_out[k] = -1;
      t_out[k] = -1;
    }
  } else if (s.transposed) {
    // rows are targets: emit matched queries (solver columns) in ascending
    // order.  The ballots list the matched columns in shared memory (`remaining`
    // is free by now); the warp then writes the pairs with coalesced stores.
    int16_t* list = rem_s;
    int slot0 = 0;
    const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const bool matched = ((valid & ~freem) >> k) & 1u;
      const unsigned ballot = __ballot_sync(kFullMask, matched);
      if (matched) list[slot0 + __popc(ballot & lt_mask)] = static_cast<int16_t>(lane + 32 * k);
      slot0 += __popc(ballot);
    }
    __syncwarp();
    for (int e = lane; e < slot0; e += 32) {
      const int j = list[e];
      q_out[e] = j + qbase;
      t_out[e] = row4col_s[j];
    }
  } else {
    for (int r = lane; r < nr; r += 32) {
      q_out[r] = r + qbase;
      t_out[r] = col4row_s[r];
    }
  }
  if (!kDense && a.mode.push != nullptr) {
    // the problem's nr pairs also to every push destination (peers' gathered
    // buffers), in the buffer of this step's parity, rebuilt from shared memory
    // as above (the transposed list is still in `remaining`)
    // (the list and the step counter do not change during the launch: read-only loads)
    const rfm_pair_push* pl = a.mode.push;
    const int count = min(__ldg(&pl->count), RFM_MAX_PUSH);  // checked when the list was stored
    const int64_t off = out_off + static_cast<int64_t>(__ldg(pl->epoch) & 1u) * __ldg(&pl->parity_stride);
    for (int d = 0; d < count; ++d) {
      int64_t* const qd = reinterpret_cast<int64_t*>(__ldg(reinterpret_cast<const unsigned long long*>(
                              &pl->query_out[d]))) + off;
      int64_t* const td = reinterpret_cast<int64_t*>(__ldg(reinterpret_cast<const unsigned long long*>(
                              &pl->target_out[d]))) + off;
      for (int k = lane; k < nr; k += 32) {
        int64_t qv = -1, tv = -1;
        if (code == RFM_STATUS_OK) {
          const int j = s.transposed ? rem_s[k] : k;
          qv = j + qbase;
          tv = s.transposed ? row4col_s[j] : col4row_s[k];
        }
        qd[k] = qv;
        td[k] = tv;
      }
    }
  }
  if (a.status != nullptr && lane == 0) a.status[p] = code;
  return next;
}

template <int K, bool kDense, int kVariant>
__global__ void __launch_bounds__(32 * kMaxWarpsPerCta, min_ctas_per_sm(K, kVariant)) lsap_kernel(const LsapArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (queue_variant(kVariant)) {
    // fewer CTAs than problems: CTA c starts on problem c, then claims further
    // problems (sorted largest first) from the counter until none is left.  The
    // claim is passed on in a spare word of the step-post area (static shared
    // memory would not fit beside the SM's shares).
    int* next_problem = reinterpret_cast<int*>(smem_raw + a.slot - kMultiPostBytes + kMultiClaimOffset);
    int p = blockIdx.x;
    while (p < a.num_problems) {
      solve_problem<K, kDense, kVariant>(a, p, smem_raw, a.slot, lane);
      __syncthreads();  // every warp is done with the problem's shared memory
      if (threadIdx.x == 0) *next_problem = atomicAdd(a.queue, 1) + a.claim_base;
      __syncthreads();
      p = *next_problem;
    }
    return;
  }
  if (cta_variant(kVariant)) {
    // one problem per CTA, all its warps in its load pass
    solve_problem<K, kDense, kVariant>(a, blockIdx.x, smem_raw, a.slot, lane);
    return;
  }
  if (kDense) {
    const int p = blockIdx.x * a.mode.dense.warps + warp;
    if (p < a.num_problems) {
      solve_problem<K, kDense, kVariant>(a, p, smem_raw + static_cast<int64_t>(warp) * a.slot, a.slot, lane);
    }
  } else if (a.queue != nullptr) {
    // persistent warps: warp w starts on problem w, then pulls problems (sorted
    // largest first) from the counter until none is left
    unsigned char* base = smem_raw + static_cast<int64_t>(warp) * a.slot;
    int p = blockIdx.x * kMaxWarpsPerCta + warp;
    while (p < a.num_problems) {
      const int next = solve_problem<K, kDense, kVariant>(a, p, base, a.slot, lane);
      p = __shfl_sync(kFullMask, next, 0);
      __syncwarp();
    }
  } else {
    const int4 cta = a.ctas[blockIdx.x];
    if (warp < cta.y) {
      solve_problem<K, kDense, kVariant>(a, cta.x + warp, smem_raw + static_cast<int64_t>(warp) * cta.z, cta.z,
                               lane);
    }
  }
}

int cols_per_lane_for(int max_cols) {
  if (max_cols <= 128) return 4;
  if (max_cols <= 320) return 10;
  if (max_cols <= RFM_MAX_COLS) return 32;
  return -1;
}

// Shared-memory slot of one problem: the fixed arrays plus its tile when staged.
int64_t slot_bytes(const Shape& s, int cols_cap, int max_rows, int64_t tile_cap) {
  const int64_t t = static_cast<int64_t>(s.nr) * s.nc;
  return warp_bytes_for(cols_cap, max_rows, (s.nr > 0 && t <= tile_cap) ? t : 0);
}

// The pair-mode kernel for a column count and variant (the wide and
// cooperative layouts exist for up to 320 columns).
const void* pair_kernel(int cols_per_lane, int variant) {
  switch (cols_per_lane) {
    case 4:
      if (variant == kVarWide) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarWide>);
      if (variant == kVarEarly) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarEarly>);
      if (variant == kVarCoop) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarCoop>);
      if (variant == kVarMulti) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarMulti>);
      if (variant == kVarMultiCopy) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarMultiCopy>);
      if (variant == kVarMultiTwo) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarMultiTwo>);
      if (variant == kVarMultiCopyTwo) return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarMultiCopyTwo>);
      if (variant == kVarMultiTwoQueue) {
        return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarMultiTwoQueue>);
      }
      return reinterpret_cast<const void*>(&lsap_kernel<4, false, kVarRegs>);
    case 10:
      if (variant == kVarWide) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarWide>);
      if (variant == kVarEarly) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarEarly>);
      if (variant == kVarCoop) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarCoop>);
      if (variant == kVarMulti) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarMulti>);
      if (variant == kVarMultiCopy) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarMultiCopy>);
      if (variant == kVarMultiTwo) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarMultiTwo>);
      if (variant == kVarMultiCopyTwo) return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarMultiCopyTwo>);
      if (variant == kVarMultiTwoQueue) {
        return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarMultiTwoQueue>);
      }
      return reinterpret_cast<const void*>(&lsap_kernel<10, false, kVarRegs>);
    case 32:
      if (narrow_only(variant)) return nullptr;
      if (variant == kVarEarly) return reinterpret_cast<const void*>(&lsap_kernel<32, false, kVarEarly>);
      return reinterpret_cast<const void*>(&lsap_kernel<32, false, kVarRegs>);
    default: return nullptr;
  }
}

// Opts a kernel into `smem` bytes of dynamic shared memory once per context
// (the attribute is then left raised): repeated launches, including launches
// being captured into a CUDA graph, make no attribute call.  The attribute
// belongs to the context's copy of the module, so it is cached under the
// context's id: after the context is destroyed and recreated the attribute is
// set again.
struct SmemAttribute {
  unsigned long long context;
  const void* fn;
  int64_t smem;
};
std::mutex g_smem_mutex;
std::vector<SmemAttribute> g_smem_attributes;

bool ensure_dynamic_smem(const void* fn, int64_t smem) {
  if (smem <= 48 * 1024) return true;
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  const unsigned long long ctx = current_context_id();
  if (ctx != 0) {
    for (const SmemAttribute& e : g_smem_attributes) {
      if (e.context == ctx && e.fn == fn && e.smem >= smem) return true;
    }
  }
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess) {
    return false;
  }
  // the call above made the primary context current if it was not yet
  const unsigned long long now = ctx != 0 ? ctx : current_context_id();
  if (now != 0) {
    for (SmemAttribute& e : g_smem_attributes) {
      if (e.context == now && e.fn == fn) {
        e.smem = smem;
        return true;
      }
    }
    g_smem_attributes.push_back({now, fn, smem});
  }
  return true;
}

// CTAs of a solver kernel (CTAs of `threads`) that fit on one SM at this
// shared-memory size.
int query_resident_ctas(const void* fn, int64_t smem, int threads) {
  if (fn == nullptr) return 0;
  if (!ensure_dynamic_smem(fn, smem)) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads,
                                                    static_cast<size_t>(smem)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// query_resident_ctas() memoised per (device, kernel, shared memory): the
// occupancy query and the attribute call cost a few microseconds per launch.
// Occupancy is a property of the device and the kernel, so the memo stays
// valid across contexts; the launch itself raises the attribute per context.
struct OccupancyEntry {
  int device;
  const void* fn;
  int64_t smem;
  int ctas;
};
std::mutex g_occupancy_mutex;
std::vector<OccupancyEntry> g_occupancy;

int resident_ctas(const void* fn, int64_t smem, int threads = 32 * kMaxWarpsPerCta) {
  if (fn == nullptr) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  {
    std::lock_guard<std::mutex> lock(g_occupancy_mutex);
    for (const OccupancyEntry& e : g_occupancy) {
      if (e.device == dev && e.fn == fn && e.smem == smem) {
        return e.ctas;
      }
    }
  }
  const int n = query_resident_ctas(fn, smem, threads);
  if (n > 0) {
    std::lock_guard<std::mutex> lock(g_occupancy_mutex);
    g_occupancy.push_back({dev, fn, smem, n});
  }
  return n;
}

template <bool kDense, int kVariant>
int launch(const LsapArgs& a, int cols_per_lane, int num_ctas, int warps_per_cta, int64_t smem,
           void* stream, bool after_kernel = false) {
  if (smem > kSmemPerBlockMax) return RFM_ERR_UNSUPPORTED;
  const void* fn = nullptr;
  switch (cols_per_lane) {
    case 4: fn = reinterpret_cast<const void*>(&lsap_kernel<4, kDense, kVariant>); break;
    case 10: fn = reinterpret_cast<const void*>(&lsap_kernel<10, kDense, kVariant>); break;
    case 32:
      if (narrow_only(kVariant)) return RFM_ERR_INVALID_ARGUMENT;
      fn = reinterpret_cast<const void*>(&lsap_kernel<32, kDense, narrow_only(kVariant) ? kVarRegs : kVariant>);
      break;
    default: return RFM_ERR_INVALID_ARGUMENT;
  }
  if (!ensure_dynamic_smem(fn, smem)) return launch_status();
  const dim3 grid(static_cast<unsigned>(num_ctas));
  const dim3 block(32 * warps_per_cta);
  if (!kDense && kVariant != kVarEarly && cols_per_lane <= 10 && after_kernel) {
    // programmatic stream serialization, only right after this library's cost
    // kernel (rfm_match): the CTAs may launch while it finishes and wait for it
    // (griddepcontrol.wait) before reading the matrix or the counter.  They
    // read their descriptor before that wait, which is safe because the cost
    // kernel does not write descriptors; after a caller's kernel (standalone
    // rfm_lsap) the launch is an ordinary stream-ordered one.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    constexpr int kV = (kDense || kVariant == kVarEarly) ? kVarRegs : kVariant;
    const cudaError_t e = cols_per_lane == 4 ? cudaLaunchKernelEx(&cfg, lsap_kernel<4, false, kV>, a)
                                             : cudaLaunchKernelEx(&cfg, lsap_kernel<10, false, kV>, a);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) ? RFM_ERR_NO_DEVICE : RFM_ERR_LAUNCH;
    }
    return launch_status();
  }
  switch (cols_per_lane) {
    case 4: lsap_kernel<4, kDense, kVariant><<<grid, block, smem, as_stream(stream)>>>(a); break;
    case 10: lsap_kernel<10, kDense, kVariant><<<grid, block, smem, as_stream(stream)>>>(a); break;
    default:
      lsap_kernel<32, kDense, narrow_only(kVariant) ? kVarRegs : kVariant><<<grid, block, smem, as_stream(stream)>>>(a);
      break;
  }
  return launch_status();
}

}  // namespace
}  // namespace rfm

extern "C" int rfm_lsap_make_plan(rfm_problem* host_problems, int num_problems, int64_t stride_q,
                                  int64_t stride_t, int64_t tile_cap_floats, int32_t* host_ctas,
                                  rfm_lsap_plan* plan) {
  using namespace rfm;
  if (plan == nullptr || num_problems < 0 ||
      (num_problems > 0 && (host_problems == nullptr || host_ctas == nullptr)) || stride_q < 0 ||
      stride_t < 0) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  int64_t cap = tile_cap_floats < 0 ? kTileCapDefault : tile_cap_floats;
  int max_cols = 1, max_rows = 1;
  for (int p = 0; p < num_problems; ++p) {
    const rfm_problem& d = host_problems[p];
    if (d.num_queries < 0 || d.num_targets < 0 || d.cost_offset < 0 || d.out_offset < 0 ||
        d.reserved != 0) {
      return RFM_ERR_INVALID_ARGUMENT;
    }
    const Shape s = solver_shape(d.num_queries, d.num_targets, stride_q, stride_t);
    if (s.nr == 0) continue;
    if (s.nc > max_cols) max_cols = s.nc;
    if (s.nr > max_rows) max_rows = s.nr;
  }
  const int cpl = cols_per_lane_for(max_cols);
  if (cpl < 0) return RFM_ERR_UNSUPPORTED;
  const int cols_cap = 32 * cpl;
  const int64_t fixed = fixed_warp_bytes(cols_cap, max_rows);
  const int64_t hard_cap = (kSmemPerBlockMax - fixed) / 4;
  if (cap > hard_cap) cap = hard_cap;

  // When every problem's solver rows are contiguous in the source, nothing is
  // staged: persistent warps with a uniform slot pull the problems in order.
  bool contiguous = true;
  for (int p = 0; p < num_problems && contiguous; ++p) {
    const rfm_problem& d = host_problems[p];
    const Shape s = solver_shape(d.num_queries, d.num_targets, stride_q, stride_t);
    if (s.nr > 0 && s.cs != 1) contiguous = false;
  }
  if (contiguous) {
    for (int p = 0; p < num_problems; ++p) host_problems[p].scratch_offset = -1;
    plan->cols_per_lane = cpl;
    plan->max_rows = max_rows;
    plan->num_problems = num_problems;
    plan->num_ctas = 0;  // sized at launch from the device's occupancy
    plan->cta_smem_bytes = static_cast<int32_t>(kMaxWarpsPerCta * fixed);
    plan->tile_cap_floats = 0;
    plan->flags = RFM_PLAN_PERSISTENT;
    plan->reserved = 0;
    plan->stride_q = stride_q;
    plan->stride_t = stride_t;
    plan->workspace_bytes = kQueueBytes;
    return RFM_OK;
  }

  // scratch for tiles that are neither staged nor row-contiguous in the source
  int64_t scratch = 0;
  for (int p = 0; p < num_problems; ++p) {
    rfm_problem& d = host_problems[p];
    d.scratch_offset = -1;
    const Shape s = solver_shape(d.num_queries, d.num_targets, stride_q, stride_t);
    if (s.nr == 0) continue;
    const int64_t slot = slot_bytes(s, cols_cap, max_rows, cap);
    if (choose_mode(s, cap, (slot - fixed) / 4) == kModeScratch) {
      d.scratch_offset = scratch;
      scratch += (static_cast<int64_t>(s.nr) * s.nc + 3) & ~int64_t(3);
    }
  }

  // pack consecutive problems into CTAs of up to four warps under the budget;
  // every warp of a CTA gets the CTA's largest slot
  int64_t budget = kCtaBudget;
  for (int p = 0; p < num_problems; ++p) {
    const rfm_problem& d = host_problems[p];
    const int64_t sl = slot_bytes(solver_shape(d.num_queries, d.num_targets, stride_q, stride_t),
                                  cols_cap, max_rows, cap);
    if (sl > budget) budget = sl;
  }
  int num_ctas = 0;
  int64_t cta_smem = 0;
  for (int p = 0; p < num_problems;) {
    const rfm_problem& d0 = host_problems[p];
    int64_t slot = slot_bytes(solver_shape(d0.num_queries, d0.num_targets, stride_q, stride_t),
                              cols_cap, max_rows, cap);
    int count = 1;
    while (count < kMaxWarpsPerCta && p + count < num_problems) {
      const rfm_problem& d = host_problems[p + count];
      const int64_t sl = slot_bytes(solver_shape(d.num_queries, d.num_targets, stride_q, stride_t),
                                    cols_cap, max_rows, cap);
      const int64_t next = sl > slot ? sl : slot;
      if ((count + 1) * next > budget) break;
      slot = next;
      ++count;
    }
    host_ctas[4 * num_ctas + 0] = p;
    host_ctas[4 * num_ctas + 1] = count;
    host_ctas[4 * num_ctas + 2] = static_cast<int32_t>(slot);
    host_ctas[4 * num_ctas + 3] = 0;
    if (count * slot > cta_smem) cta_smem = count * slot;
    ++num_ctas;
    p += count;
  }
  plan->cols_per_lane = cpl;
  plan->max_rows = max_rows;
  plan->num_problems = num_problems;
  plan->num_ctas = num_ctas;
  plan->cta_smem_bytes = static_cast<int32_t>(cta_smem);
  plan->tile_cap_floats = static_cast<int32_t>(cap);
  plan->flags = 0;
  plan->reserved = 0;
  plan->stride_q = stride_q;
  plan->stride_t = stride_t;
  plan->workspace_bytes = scratch * 4;
  return RFM_OK;
}

namespace rfm {
namespace {
// A MULTI launch for a batch of `num_problems` as one wave: ceil(P / SMs) CTAs
// per SM, each taking that share of the SM's shared memory (`slot` bytes),
// with four warps per problem (`fn4`) up to kMultiFourPerSm per SM and two
// (`fn2`) beyond.  `slot` is 0 when the batch is larger than kMultiTwoPerSm per
// SM, when that many CTAs do not fit (registers), or when the share does not
// hold the problem's `fixed` arrays and the step posts.
struct MultiLaunch {
  int slot;
  bool two;
  int ctas;  // the grid: one CTA per problem, or fewer that claim problems from a counter
};

// Shared memory of each of `per_sm` CTAs sharing an SM: whole KB, so that the
// shares plus their reservations fit.
int multi_share(int per_sm) {
  const int smem = (kSmemPerSm / per_sm - kSmemPerCtaReserved) / 1024 * 1024;
  return smem > kSmemPerBlockMax ? kSmemPerBlockMax : smem;
}

// With `fn2_queue` (the claiming two-warp kernel, given when the workspace
// holds a counter: persistent plans, dense batches of 512+ problems), a batch
// of up to kMultiTwoPerSm problems per SM whose CTAs do not all fit at once
// runs as the most such CTAs that do (fewer than the problems, so every CTA
// has its own first problem).
MultiLaunch multi_launch(int num_problems, const void* fn4, const void* fn2, int64_t fixed,
                         const void* fn2_queue = nullptr) {
  const int sms = device_sm_count();
  if (sms < 1 || num_problems < 1 ||
      static_cast<int64_t>(num_problems) > static_cast<int64_t>(kMultiTwoPerSm) * sms) {
    return {0, false, 0};
  }
  const int per_sm = (num_problems + sms - 1) / sms;
  int smem = multi_share(per_sm);
  if (fixed + kMultiPostBytes <= smem) {
    if (per_sm <= kMultiFourPerSm && resident_ctas(fn4, smem, 128) >= per_sm) return {smem, false, num_problems};
    if (resident_ctas(fn2, smem, 64) >= per_sm) return {smem, true, num_problems};
  }
  if (fn2_queue == nullptr) return {0, false, 0};
  for (int n = per_sm - 1; n > kMultiFourPerSm; --n) {
    smem = multi_share(n);
    if (fixed + kMultiPostBytes <= smem && resident_ctas(fn2_queue, smem, 64) >= n) return {smem, true, n * sms};
  }
  return {0, false, 0};
}

const void* dense_queue_kernel(int cols_per_lane) {
  if (cols_per_lane == 4) return reinterpret_cast<const void*>(&lsap_kernel<4, true, kVarMultiCopyTwoQueue>);
  if (cols_per_lane == 10) return reinterpret_cast<const void*>(&lsap_kernel<10, true, kVarMultiCopyTwoQueue>);
  return nullptr;
}

const void* dense_multi_kernel(int cols_per_lane, bool two) {
  if (cols_per_lane == 4) {
    return two ? reinterpret_cast<const void*>(&lsap_kernel<4, true, kVarMultiCopyTwo>)
               : reinterpret_cast<const void*>(&lsap_kernel<4, true, kVarMultiCopy>);
  }
  if (cols_per_lane == 10) {
    return two ? reinterpret_cast<const void*>(&lsap_kernel<10, true, kVarMultiCopyTwo>)
               : reinterpret_cast<const void*>(&lsap_kernel<10, true, kVarMultiCopy>);
  }
  return nullptr;
}

// A push list the solver accepts: none, or 1..RFM_MAX_PUSH destinations with
// both rows and the step counter given.
bool push_valid(const rfm_pair_push* push) {
  if (push->count < 0 || push->count > RFM_MAX_PUSH || push->reserved != 0 || push->parity_stride < 0) {
    return false;
  }
  if (push->count == 0) return true;
  if (push->epoch == nullptr) return false;
  for (int d = 0; d < push->count; ++d) {
    if (push->query_out[d] == nullptr || push->target_out[d] == nullptr) return false;
  }
  return true;
}

// rfm_lsap; with `counter_zeroed` the persistent counter was reset by the cost
// kernel that runs just before on the stream, so there is no memset and the
// persistent launch overlaps that kernel's end.
int lsap_run(const float* cost, const rfm_problem* problems, const int32_t* ctas, const rfm_lsap_plan* plan,
             int64_t* query_out, int64_t* target_out, int32_t* status, void* workspace, void* stream,
             bool counter_zeroed, const rfm_pair_push* device_push) {
  if ((reinterpret_cast<uintptr_t>(device_push) & 15u) != 0) return RFM_ERR_INVALID_ARGUMENT;
  if (plan == nullptr || plan->num_problems < 0 || plan->num_ctas < 0 || plan->max_rows < 1 ||
      plan->workspace_bytes < 0 || plan->stride_q < 0 || plan->stride_t < 0 ||
      plan->tile_cap_floats < 0 || plan->cta_smem_bytes < 0 || plan->cta_smem_bytes > kSmemPerBlockMax ||
      (plan->flags & ~RFM_PLAN_PERSISTENT) != 0 ||
      cols_per_lane_for(32 * plan->cols_per_lane) != plan->cols_per_lane) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  const bool persistent = (plan->flags & RFM_PLAN_PERSISTENT) != 0;
  if (plan->num_problems == 0 || (!persistent && plan->num_ctas == 0)) return RFM_OK;
  if (cost == nullptr || problems == nullptr || (!persistent && ctas == nullptr) ||
      query_out == nullptr || target_out == nullptr ||
      (plan->workspace_bytes > 0 && workspace == nullptr) ||
      (persistent && plan->workspace_bytes < kQueueBytes)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  LsapArgs a;
  a.cost = cost;
  a.stride_q = plan->stride_q;
  a.stride_t = plan->stride_t;
  a.problems = problems;
  a.ctas = reinterpret_cast<const int4*>(ctas);
  a.num_problems = plan->num_problems;
  a.dense_w = 0;
  a.mode.push = device_push;
  a.slot = 0;
  a.queue = nullptr;
  a.claim_base = 0;
  a.tile_cap = plan->tile_cap_floats;
  a.max_rows = plan->max_rows;
  a.workspace = static_cast<float*>(workspace);
  a.q_out = query_out;
  a.t_out = target_out;
  a.status = status;
  const bool early = plan->max_rows >= kEarlyMinRows;
  if (!persistent) {
    const MultiLaunch ml =
        plan->cols_per_lane <= 10
            ? multi_launch(plan->num_problems, pair_kernel(plan->cols_per_lane, kVarMultiCopy),
                           pair_kernel(plan->cols_per_lane, kVarMultiCopyTwo),
                           fixed_warp_bytes(32 * plan->cols_per_lane, plan->max_rows))
            : MultiLaunch{0, false, 0};
    if (ml.slot > 0) {
      // a batch that runs in one wave, some problems not row-contiguous: MULTI_COPY.
      // Every tile above the plan's cap has scratch, so it runs when its shared
      // memory holds that cap.
      const int64_t room =
          (ml.slot - fixed_warp_bytes(32 * plan->cols_per_lane, plan->max_rows) - kMultiPostBytes) / 4;
      if (plan->tile_cap_floats <= room) {
        a.slot = ml.slot;
        a.tile_cap = static_cast<int>(room);
        if (ml.two) {
          return launch<false, kVarMultiCopyTwo>(a, plan->cols_per_lane, plan->num_problems, 2, ml.slot, stream);
        }
        return launch<false, kVarMultiCopy>(a, plan->cols_per_lane, plan->num_problems, 4, ml.slot, stream);
      }
    }
    if (early) {
      return launch<false, kVarEarly>(a, plan->cols_per_lane, plan->num_ctas, kMaxWarpsPerCta,
                                      plan->cta_smem_bytes, stream);
    }
    return launch<false, kVarRegs>(a, plan->cols_per_lane, plan->num_ctas, kMaxWarpsPerCta,
                                   plan->cta_smem_bytes, stream);
  }
  // Persistent warps stage nothing, so each warp's slot is just its fixed arrays;
  // large batches (more problems than 64 per SM) take the wide layout, batches of
  // long problems the early-load variant.
  const int sms = device_sm_count();
  const MultiLaunch ml = plan->cols_per_lane <= 10
                             ? multi_launch(plan->num_problems, pair_kernel(plan->cols_per_lane, kVarMulti),
                                            pair_kernel(plan->cols_per_lane, kVarMultiTwo),
                                            fixed_warp_bytes(32 * plan->cols_per_lane, plan->max_rows),
                                            pair_kernel(plan->cols_per_lane, kVarMultiTwoQueue))
                             : MultiLaunch{0, false, 0};
  if (ml.slot > 0) {
    // MULTI, its rows staged as far as they fit: a batch that runs in one wave,
    // or (fewer CTAs than problems) CTAs that pull problems from the counter
    a.slot = ml.slot;
    a.tile_cap = (a.slot - static_cast<int>(fixed_warp_bytes(32 * plan->cols_per_lane, plan->max_rows))) / 4;
    if (ml.ctas < plan->num_problems) {
      a.queue = static_cast<int*>(workspace);
      a.claim_base = ml.ctas;
      if (!counter_zeroed && cudaMemsetAsync(a.queue, 0, sizeof(int), as_stream(stream)) != cudaSuccess) {
        return launch_status();
      }
      return launch<false, kVarMultiTwoQueue>(a, plan->cols_per_lane, ml.ctas, 2, a.slot, stream, counter_zeroed);
    }
    if (ml.two) {
      return launch<false, kVarMultiTwo>(a, plan->cols_per_lane, ml.ctas, 2, a.slot, stream, counter_zeroed);
    }
    return launch<false, kVarMulti>(a, plan->cols_per_lane, ml.ctas, 4, a.slot, stream, counter_zeroed);
  }
  const bool wide = plan->cols_per_lane <= 10 &&
                    static_cast<int64_t>(plan->num_problems) > static_cast<int64_t>(kWideProblemsPerSm) * sms;
  const int variant = wide ? kVarWide : (early ? kVarEarly : kVarRegs);
  if (!wide && !early && plan->cols_per_lane <= 10) {
    // a small batch whose problems are all resident at once: one problem per
    // CTA, the CTA's four warps sharing its load pass (no counter, no memset)
    const int64_t coop_smem = fixed_warp_bytes(32 * plan->cols_per_lane, plan->max_rows);
    const int coop_ctas = resident_ctas(pair_kernel(plan->cols_per_lane, kVarCoop), coop_smem);
    if (coop_ctas > 0 && static_cast<int64_t>(plan->num_problems) <= static_cast<int64_t>(coop_ctas) * sms) {
      a.slot = static_cast<int>(coop_smem);
      return launch<false, kVarCoop>(a, plan->cols_per_lane, plan->num_problems, kMaxWarpsPerCta, coop_smem,
                                     stream, counter_zeroed);
    }
  }
  const int64_t smem = wide ? kMaxWarpsPerCta * fixed_warp_bytes(32 * plan->cols_per_lane, plan->max_rows, true)
                            : plan->cta_smem_bytes;
  a.queue = static_cast<int*>(workspace);
  a.workspace = reinterpret_cast<float*>(static_cast<char*>(workspace) + kQueueBytes);
  a.slot = static_cast<int>(smem / kMaxWarpsPerCta);
  if (!counter_zeroed && cudaMemsetAsync(a.queue, 0, sizeof(int), as_stream(stream)) != cudaSuccess) {
    return launch_status();
  }
  const int ctas_per_sm = resident_ctas(pair_kernel(plan->cols_per_lane, variant), smem);
  if (ctas_per_sm < 1) return launch_status() != RFM_OK ? RFM_ERR_LAUNCH : RFM_ERR_UNSUPPORTED;
  const int grid = ctas_per_sm * sms;
  const int needed = (plan->num_problems + kMaxWarpsPerCta - 1) / kMaxWarpsPerCta;
  const int num_ctas = grid < needed ? grid : needed;
  a.claim_base = num_ctas * kMaxWarpsPerCta;
  if (variant == kVarWide) {
    return launch<false, kVarWide>(a, plan->cols_per_lane, num_ctas, kMaxWarpsPerCta, smem, stream, counter_zeroed);
  }
  if (variant == kVarEarly) {
    return launch<false, kVarEarly>(a, plan->cols_per_lane, num_ctas, kMaxWarpsPerCta, smem, stream);
  }
  return launch<false, kVarRegs>(a, plan->cols_per_lane, num_ctas, kMaxWarpsPerCta, smem, stream, counter_zeroed);
}
}  // namespace
}  // namespace rfm

extern "C" int rfm_lsap(const float* cost, const rfm_problem* problems, const int32_t* ctas,
                        const rfm_lsap_plan* plan, int64_t* query_out, int64_t* target_out,
                        int32_t* status, void* workspace, void* stream) {
  return rfm::lsap_run(cost, problems, ctas, plan, query_out, target_out, status, workspace, stream, false, nullptr);
}

extern "C" int rfm_lsap_push(const float* cost, const rfm_problem* problems, const int32_t* ctas,
                             const rfm_lsap_plan* plan, int64_t* query_out, int64_t* target_out,
                             int32_t* status, void* workspace, const rfm_pair_push* device_push,
                             void* stream) {
  return rfm::lsap_run(cost, problems, ctas, plan, query_out, target_out, status, workspace, stream, false,
                       device_push);
}

extern "C" int rfm_pair_push_store(const rfm_pair_push* push, void* device_dst) {
  if (push == nullptr || device_dst == nullptr || (reinterpret_cast<uintptr_t>(device_dst) & 15u) != 0 ||
      !rfm::push_valid(push)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (cudaMemcpy(device_dst, push, sizeof(rfm_pair_push), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    return RFM_ERR_LAUNCH;
  }
  return RFM_OK;
}

extern "C" int rfm_match_push(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                              const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
                              int num_queries, int num_classes, int sum_targets, int64_t ld, float cost_class,
                              float cost_bbox, float cost_giou, float focal_alpha, float* cost,
                              const rfm_problem* problems, const int32_t* ctas, const rfm_lsap_plan* plan,
                              int64_t* query_out, int64_t* target_out, int32_t* status, void* workspace,
                              const rfm_pair_push* device_push, void* stream) {
  using namespace rfm;
  if ((reinterpret_cast<uintptr_t>(device_push) & 15u) != 0) return RFM_ERR_INVALID_ARGUMENT;
  // the solver must read the matrix this call writes: target-major, row stride ld
  if (plan == nullptr || plan->stride_q != 1 || plan->stride_t != ld ||
      (plan->num_problems > 0 && sum_targets < 1)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  const bool persistent = (plan->flags & RFM_PLAN_PERSISTENT) != 0;
  // a workspace the solver would reject is rejected before the cost kernel is enqueued
  if (plan->workspace_bytes < 0 || (plan->workspace_bytes > 0 && workspace == nullptr) ||
      (persistent && plan->num_problems > 0 && plan->workspace_bytes < kQueueBytes)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  const bool reset = persistent && plan->num_problems > 0;
  const int rc = cost_run(pred_logits, pred_boxes, tgt_labels, tgt_boxes, tgt_offsets, num_layers, num_images,
                          num_queries, num_classes, sum_targets, ld, RFM_LAYOUT_TARGET_MAJOR, cost_class,
                          cost_bbox, cost_giou, focal_alpha, cost, reset ? static_cast<int*>(workspace) : nullptr,
                          stream);
  if (rc != RFM_OK) return rc;
  return lsap_run(cost, problems, ctas, plan, query_out, target_out, status, workspace, stream, reset,
                  device_push);
}

extern "C" int rfm_match(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                         const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
                         int num_queries, int num_classes, int sum_targets, int64_t ld, float cost_class,
                         float cost_bbox, float cost_giou, float focal_alpha, float* cost,
                         const rfm_problem* problems, const int32_t* ctas, const rfm_lsap_plan* plan,
                         int64_t* query_out, int64_t* target_out, int32_t* status, void* workspace,
                         void* stream) {
  return rfm_match_push(pred_logits, pred_boxes, tgt_labels, tgt_boxes, tgt_offsets, num_layers, num_images,
                        num_queries, num_classes, sum_targets, ld, cost_class, cost_bbox, cost_giou, focal_alpha,
                        cost, problems, ctas, plan, query_out, target_out, status, workspace, nullptr, stream);
}

namespace {
// Dense batches of at least this many problems reserve a claim counter after
// their scratch (kQueueBytes), for the queue layout when one wave does not fit.
constexpr int kDenseQueueMinProblems = 512;

struct DensePlan {
  int cpl, max_rows, warps;
  int64_t slot, tile_cap, scratch_bytes;
  int64_t queue_offset;     // -1: no counter
  int64_t workspace_bytes;  // scratch, then the counter
};

int dense_plan(int num_problems, int num_workers, int num_tasks, DensePlan* out) {
  using namespace rfm;
  if (num_problems < 0 || num_workers < 0 || num_tasks < 0) return RFM_ERR_INVALID_ARGUMENT;
  const Shape s = solver_shape(num_workers, num_tasks, num_tasks, 1);
  out->cpl = cols_per_lane_for(s.nc < 1 ? 1 : s.nc);
  if (out->cpl < 0) return RFM_ERR_UNSUPPORTED;
  out->max_rows = s.nr < 1 ? 1 : s.nr;
  const int64_t fixed = fixed_warp_bytes(32 * out->cpl, out->max_rows);
  out->tile_cap = kTileCapDefault;
  if (out->tile_cap > (kSmemPerBlockMax - fixed) / 4) out->tile_cap = (kSmemPerBlockMax - fixed) / 4;
  out->slot = slot_bytes(s, 32 * out->cpl, out->max_rows, out->tile_cap);
  int w = kMaxWarpsPerCta;
  while (w > 1 && w * out->slot > kCtaBudget) --w;
  out->warps = w;
  out->scratch_bytes = 0;
  if (s.nr > 0 && choose_mode(s, out->tile_cap, (out->slot - fixed) / 4) == kModeScratch) {
    out->scratch_bytes = static_cast<int64_t>(num_problems) * num_workers * num_tasks * 4;
  }
  out->queue_offset = -1;
  out->workspace_bytes = out->scratch_bytes;
  if (num_problems >= kDenseQueueMinProblems && out->cpl <= 10 && s.nr > 0) {
    out->queue_offset = (out->scratch_bytes + 255) & ~int64_t(255);
    out->workspace_bytes = out->queue_offset + kQueueBytes;
  }
  return RFM_OK;
}
}  // namespace

extern "C" int64_t rfm_lsap_dense_workspace_bytes(int num_problems, int num_workers,
                                                  int num_tasks) {
  DensePlan dp;
  const int rc = dense_plan(num_problems, num_workers, num_tasks, &dp);
  if (rc != RFM_OK) return -static_cast<int64_t>(rc);
  return dp.workspace_bytes;
}

extern "C" int rfm_lsap_dense(const float* cost, int num_problems, int num_workers, int num_tasks,
                              int64_t* matching, int32_t* status, void* workspace, void* stream) {
  using namespace rfm;
  DensePlan dp;
  const int rc = dense_plan(num_problems, num_workers, num_tasks, &dp);
  if (rc != RFM_OK) return rc;
  if (num_problems == 0 || num_workers == 0) return RFM_OK;
  if (matching == nullptr || (num_tasks > 0 && cost == nullptr) ||
      (dp.workspace_bytes > 0 && workspace == nullptr)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  LsapArgs a;
  a.cost = cost;
  a.stride_q = num_tasks;
  a.stride_t = 1;
  a.problems = nullptr;
  a.ctas = nullptr;
  a.num_problems = num_problems;
  a.dense_w = num_workers;
  a.mode.dense.t = num_tasks;
  a.mode.dense.warps = dp.warps;
  a.slot = static_cast<int>(dp.slot);
  a.queue = nullptr;
  a.claim_base = 0;
  a.tile_cap = static_cast<int>(dp.tile_cap);
  a.max_rows = dp.max_rows;
  a.workspace = static_cast<float*>(workspace);
  a.q_out = matching;
  a.t_out = nullptr;
  a.status = status;
  if (dp.cpl <= 10) {
    // MULTI_COPY when every tile either fits its CTA's shared memory or has
    // scratch: one wave, or (with the workspace's counter) two-warp CTAs that
    // claim the problems one wave does not hold
    const MultiLaunch ml =
        multi_launch(num_problems, dense_multi_kernel(dp.cpl, false), dense_multi_kernel(dp.cpl, true),
                     fixed_warp_bytes(32 * dp.cpl, dp.max_rows),
                     dp.queue_offset >= 0 ? dense_queue_kernel(dp.cpl) : nullptr);
    const Shape s = solver_shape(num_workers, num_tasks, num_tasks, 1);
    const int64_t room =
        ml.slot > 0 ? (ml.slot - fixed_warp_bytes(32 * dp.cpl, dp.max_rows) - kMultiPostBytes) / 4 : 0;
    // (row-contiguous problems read their unstaged rows from the source)
    if (ml.slot > 0 && (static_cast<int64_t>(s.nr) * s.nc <= room || s.cs == 1 || dp.scratch_bytes > 0)) {
      a.slot = ml.slot;
      a.tile_cap = static_cast<int>(room);
      if (ml.ctas < num_problems) {
        a.queue = reinterpret_cast<int*>(static_cast<char*>(workspace) + dp.queue_offset);
        a.claim_base = ml.ctas;
        if (cudaMemsetAsync(a.queue, 0, sizeof(int), as_stream(stream)) != cudaSuccess) return launch_status();
        return launch<true, kVarMultiCopyTwoQueue>(a, dp.cpl, ml.ctas, 2, ml.slot, stream);
      }
      if (ml.two) return launch<true, kVarMultiCopyTwo>(a, dp.cpl, num_problems, 2, ml.slot, stream);
      return launch<true, kVarMultiCopy>(a, dp.cpl, num_problems, 4, ml.slot, stream);
    }
  }
  const int ctas = (num_problems + dp.warps - 1) / dp.warps;
  if (dp.max_rows >= kEarlyMinRows) return launch<true, kVarEarly>(a, dp.cpl, ctas, dp.warps, dp.warps * dp.slot, stream);
  return launch<true, kVarRegs>(a, dp.cpl, ctas, dp.warps, dp.warps * dp.slot, stream);
}

// ---------------------------------------------------------------------------
// rfm_lsap_dense_noalloc: rfm_lsap_dense with a built-in scratch buffer.
//
// Some callers cannot hand the solver a workspace: hosts that reach the
// library through a C FFI with no device allocator of their own, and training
// loops that run the matcher between kernels where a cudaMalloc/cudaFree
// (which may synchronise the whole device) or a second allocator competing
// with the framework's caching pool is not acceptable.  For them the scratch
// lives in a file-scope __device__ array of RFM_NOALLOC_SCRATCH_BYTES that is
// part of this module, so every GPU that loads the library holds it until the
// process exits.  Host code only ever uses its device address, fetched with
// cudaGetSymbolAddress on the first call made in a CUDA context (once per
// device while its primary context lives) and cached under the context's id:
// a context destroyed and recreated (cudaDeviceReset) reloads the module,
// possibly at another address, and the next call looks it up again.
//
// The solver writes every scratch element before reading it, so nothing has to
// be cleared between calls.  All calls share this one buffer: calls whose work
// overlaps on the GPU (for instance on two streams at once) race on it.
static __device__ __align__(256) float g_noalloc_scratch[RFM_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {
struct NoAllocAddress {
  unsigned long long context;
  void* address;
};
constexpr size_t kNoAllocCacheEntries = 64;
std::mutex g_noalloc_mutex;
std::vector<NoAllocAddress> g_noalloc_addresses;

// Device address of the built-in scratch in the current context.
int noalloc_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return RFM_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  const unsigned long long ctx = rfm::current_context_id();
  if (ctx != 0) {
    for (const NoAllocAddress& e : g_noalloc_addresses) {
      if (e.context == ctx) {
        *out = e.address;
        return RFM_OK;
      }
    }
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) ? RFM_ERR_NO_DEVICE : RFM_ERR_LAUNCH;
  }
  // the lookup made the primary context current if it was not yet
  const unsigned long long now = ctx != 0 ? ctx : rfm::current_context_id();
  if (now != 0) {
    if (g_noalloc_addresses.size() >= kNoAllocCacheEntries) g_noalloc_addresses.erase(g_noalloc_addresses.begin());
    g_noalloc_addresses.push_back({now, p});
  }
  *out = p;
  return RFM_OK;
}
}  // namespace

extern "C" int rfm_lsap_dense_noalloc(const float* cost, int num_problems, int num_workers,
                                      int num_tasks, int64_t* matching, int32_t* status,
                                      void* stream) {
  const int64_t need = rfm_lsap_dense_workspace_bytes(num_problems, num_workers, num_tasks);
  if (need < 0) return static_cast<int>(-need);
  if (need > static_cast<int64_t>(RFM_NOALLOC_SCRATCH_BYTES)) return RFM_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  if (need > 0 && num_problems > 0 && num_workers > 0) {
    const int rc = noalloc_scratch_address(&scratch);
    if (rc != RFM_OK) return rc;
  }
  return rfm_lsap_dense(cost, num_problems, num_workers, num_tasks, matching, status, scratch, stream);
}
