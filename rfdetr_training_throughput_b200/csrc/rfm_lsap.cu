// Batched exact rectangular linear assignment, SciPy semantics, one CTA (one
// warp) per problem.
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
//     reproduces it as an argmin over the key (cost, free ? -(pos+1) : pos),
//     where pos is the column's position in `remaining`, which is maintained
//     with SciPy's reverse fill and swap-with-last removal.
//
// Layout.  Lane l owns columns l, l+32, ..., l+32(K-1).  Its columns' duals
// v, path costs, positions in `remaining`, "still remaining" and "free" bits
// live in registers, so the scan is register work plus one cost load per
// column; the argmin is a 5-step shuffle butterfly.  The row duals, the
// matching and `remaining` (position -> column) live in shared memory.  The
// dual update needs no cross-lane traffic: every visited non-sink column j
// owns exactly one tree row, row4col[j], so its lane applies
// u[row4col[j]] += minv - spc[j] and v[j] -= minv - spc[j] itself.
//
// Cost tile.  The problem's cost is staged once: into shared memory when it
// fits the launch's tile budget (row stride num_targets|1 keeps both access
// orientations bank-conflict free); otherwise a tall problem is transposed
// into the caller's workspace so that each solver row is one coalesced read
// from L2, and a wide or square one is read in place (its solver rows are the
// matrix rows).
//
// Termination: every inner step removes one column from `remaining`, so each
// augmentation is bounded by num_cols steps (kernels_lap.py:78-84,147-148);
// the path flip is bounded by num_rows + 1 steps.
#include <math_constants.h>

#include <climits>

#include "rfm_common.cuh"

namespace rfm {
namespace {

constexpr int kSmemLimitDefault = 227 * 1024;

struct LsapArgs {
  const float* cost;
  int64_t ld;
  const rfm_problem* problems;  // pair mode
  int dense_w, dense_t;         // dense mode: uniform [P, W, T] problems
  int tile_floats;
  int max_rows;
  float* workspace;
  int64_t* q_out;  // pair mode: query indices; dense mode: matching [P, W]
  int64_t* t_out;
  int32_t* status;
};

struct Problem {
  int64_t cost_off, out_off, scratch_off;
  int nq, nt, qbase;
};

enum class Mode { kShared, kDirect, kScratch };

__host__ __device__ inline int64_t tile_need(int nq, int nt) {
  return static_cast<int64_t>(nq) * (nt | 1);
}

__host__ __device__ inline int64_t fixed_smem_bytes(int cols_cap, int max_rows) {
  // u (double) + col4row (int) per row; row4col, path, remaining (int) per column
  const int64_t b = static_cast<int64_t>(max_rows) * 12 + static_cast<int64_t>(cols_cap) * 12;
  return (b + 15) & ~int64_t(15);
}

template <int K>
__device__ __forceinline__ void set_pos(int (&pos)[K], int k_sel, int value) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (k == k_sel) pos[k] = value;
  }
}

// One scan step of the augmenting-path search over the lane's columns.
template <int K, bool kShared>
__device__ __forceinline__ void scan_row(const float* row, int col_stride, int lane, int i,
                                         double minv, double ui, const double (&v)[K],
                                         double (&spc)[K], const int (&pos)[K], unsigned rem,
                                         unsigned freem, int* path_s, double& bv, int& bk) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (rem & (1u << k)) {
      const int j = lane + 32 * k;
      float cf;
      if (kShared) {
        cf = row[j * col_stride];
      } else {
        cf = __ldcg(row + static_cast<int64_t>(j) * col_stride);
      }
      const double r = ((minv + static_cast<double>(cf)) - ui) - v[k];
      if (r < spc[k]) {
        spc[k] = r;
        path_s[j] = i;
      }
      const int key = (freem & (1u << k)) ? -(pos[k] + 1) : pos[k];
      if (spc[k] < bv || (spc[k] == bv && key < bk)) {
        bv = spc[k];
        bk = key;
      }
    }
  }
}

template <int K, bool kDense>
__global__ void __launch_bounds__(32) lsap_kernel(const LsapArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int kCols = 32 * K;
  const int lane = threadIdx.x;
  const int p = blockIdx.x;

  Problem pr;
  if (kDense) {
    pr.nq = a.dense_w;
    pr.nt = a.dense_t;
    pr.cost_off = static_cast<int64_t>(p) * a.dense_w * a.dense_t;
    pr.out_off = static_cast<int64_t>(p) * a.dense_w;
    pr.scratch_off = pr.cost_off;
    pr.qbase = 0;
  } else {
    const rfm_problem d = a.problems[p];
    pr.cost_off = d.cost_offset;
    pr.out_off = d.out_offset;
    pr.scratch_off = d.scratch_offset;
    pr.nq = d.num_queries;
    pr.nt = d.num_targets;
    pr.qbase = d.query_base;
  }
  const int64_t ld = kDense ? a.dense_t : a.ld;
  const bool transposed = pr.nt < pr.nq;
  const int nr = transposed ? pr.nt : pr.nq;
  const int nc = transposed ? pr.nq : pr.nt;
  int64_t* q_out = a.q_out + pr.out_off;
  int64_t* t_out = kDense ? nullptr : a.t_out + pr.out_off;

  if (nr == 0) {
    if (kDense) {
      for (int w = lane; w < pr.nq; w += 32) q_out[w] = -1;
    }
    if (a.status != nullptr && lane == 0) a.status[p] = RFM_STATUS_OK;
    return;
  }

  double* u_s = reinterpret_cast<double*>(smem_raw);
  int* col4row_s = reinterpret_cast<int*>(u_s + a.max_rows);
  int* row4col_s = col4row_s + a.max_rows;
  int* path_s = row4col_s + kCols;
  int* rem_s = path_s + kCols;
  float* tile = reinterpret_cast<float*>(smem_raw + fixed_smem_bytes(kCols, a.max_rows));

  // ---- stage the cost and validate it (SciPy rejects NaN and -inf) --------
  const float* src = a.cost + pr.cost_off;
  const int tp = pr.nt | 1;
  Mode mode;
  bool bad = false;
  float* scratch = nullptr;
  if (tile_need(pr.nq, pr.nt) <= a.tile_floats) {
    mode = Mode::kShared;
    const int total = pr.nq * pr.nt;
    for (int e = lane; e < total; e += 32) {
      const int q = e / pr.nt;
      const int t = e - q * pr.nt;
      const float x = __ldg(src + q * ld + t);
      bad |= (x != x) || (x == -CUDART_INF_F);
      tile[q * tp + t] = x;
    }
  } else if (transposed) {
    mode = Mode::kScratch;
    scratch = a.workspace + pr.scratch_off;
    for (int t = 0; t < pr.nt; ++t) {
      for (int q = lane; q < pr.nq; q += 32) {
        const float x = __ldg(src + q * ld + t);
        bad |= (x != x) || (x == -CUDART_INF_F);
        scratch[static_cast<int64_t>(t) * pr.nq + q] = x;
      }
    }
  } else {
    mode = Mode::kDirect;
    for (int q = 0; q < pr.nq; ++q) {
      for (int t = lane; t < pr.nt; t += 32) {
        const float x = __ldg(src + q * ld + t);
        bad |= (x != x) || (x == -CUDART_INF_F);
      }
    }
  }
  bad = __any_sync(kFullMask, bad);
  for (int i = lane; i < nr; i += 32) {
    u_s[i] = 0.0;
    col4row_s[i] = -1;
  }
  for (int j = lane; j < nc; j += 32) row4col_s[j] = -1;

  unsigned valid = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (lane + 32 * k < nc) valid |= 1u << k;
  }
  unsigned freem = valid;
  double v[K];
#pragma unroll
  for (int k = 0; k < K; ++k) v[k] = 0.0;
  __syncwarp();

  int code = bad ? RFM_STATUS_INVALID : RFM_STATUS_OK;
  for (int cur = 0; cur < nr && code == RFM_STATUS_OK; ++cur) {
    double spc[K];
    int pos[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int j = lane + 32 * k;
      spc[k] = CUDART_INF;
      pos[k] = nc - 1 - j;  // remaining[it] = nc - 1 - it  (reverse fill)
      if (j < nc) rem_s[nc - 1 - j] = j;
    }
    unsigned rem = valid;
    int i = cur;
    int nrem = nc;
    int sink = -1;
    double minv = 0.0;
    __syncwarp();

    for (int it = 0; it < nc; ++it) {
      const double ui = u_s[i];
      double bv = CUDART_INF;
      int bk = INT_MAX;
      if (mode == Mode::kShared) {
        if (transposed) {
          scan_row<K, true>(tile + i, tp, lane, i, minv, ui, v, spc, pos, rem, freem, path_s, bv,
                            bk);
        } else {
          scan_row<K, true>(tile + i * tp, 1, lane, i, minv, ui, v, spc, pos, rem, freem, path_s,
                            bv, bk);
        }
      } else if (mode == Mode::kScratch) {
        scan_row<K, false>(scratch + static_cast<int64_t>(i) * pr.nq, 1, lane, i, minv, ui, v, spc,
                           pos, rem, freem, path_s, bv, bk);
      } else {
        scan_row<K, false>(src + i * ld, 1, lane, i, minv, ui, v, spc, pos, rem, freem, path_s, bv,
                           bk);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const double ov = __shfl_xor_sync(kFullMask, bv, off);
        const int ok = __shfl_xor_sync(kFullMask, bk, off);
        if (ov < bv || (ov == bv && ok < bk)) {
          bv = ov;
          bk = ok;
        }
      }
      if (bv == CUDART_INF) {
        code = RFM_STATUS_INFEASIBLE;
        break;
      }
      const int ps = bk < 0 ? -bk - 1 : bk;
      const int last = nrem - 1;
      const int js = rem_s[ps];
      const int jl = rem_s[last];
      const int rj = row4col_s[js];
      __syncwarp();
      if (lane == 0) rem_s[ps] = jl;  // swap-with-last removal
      if ((jl & 31) == lane) set_pos<K>(pos, jl >> 5, ps);
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
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (visited & (1u << k)) {
        const int j = lane + 32 * k;
        const double d = minv - spc[k];
        if (j != sink) {
          const int r = row4col_s[j];
          u_s[r] += d;
        }
        v[k] -= d;
      }
    }
    if (lane == 0) u_s[cur] += minv;
    __syncwarp();

    // ---- flip the alternating path ----------------------------------------
    int flipped = 1;
    if (lane == 0) {
      flipped = 0;
      int j = sink;
      for (int s = 0; s <= nr; ++s) {
        const int ii = path_s[j];
        row4col_s[j] = ii;
        const int prev = col4row_s[ii];
        col4row_s[ii] = j;
        j = prev;
        if (ii == cur) {
          flipped = 1;
          break;
        }
      }
    }
    if ((sink & 31) == lane) freem &= ~(1u << (sink >> 5));
    if (!__shfl_sync(kFullMask, flipped, 0)) code = RFM_STATUS_NO_SINK;
    __syncwarp();
  }

  // ---- epilogue: write the result in SciPy's order -------------------------
  if (kDense) {
    // matching[w] = task of worker w, -1 if none (kernels_lap.py:336-341)
    if (code != RFM_STATUS_OK) {
      for (int w = lane; w < pr.nq; w += 32) q_out[w] = -1;
    } else if (transposed) {
      for (int w = lane; w < nc; w += 32) q_out[w] = row4col_s[w];
    } else {
      for (int w = lane; w < nr; w += 32) q_out[w] = col4row_s[w];
    }
  } else if (code != RFM_STATUS_OK) {
    for (int k = lane; k < nr; k += 32) {
      q_out[k] = -1;
      t_out[k] = -1;
    }
  } else if (transposed) {
    // rows are targets: emit matched queries (solver columns) in ascending order
    int base = 0;
    const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const bool matched = ((valid & ~freem) >> k) & 1u;
      const unsigned ballot = __ballot_sync(kFullMask, matched);
      if (matched) {
        const int j = lane + 32 * k;
        const int slot = base + __popc(ballot & lt_mask);
        q_out[slot] = j + pr.qbase;
        t_out[slot] = row4col_s[j];
      }
      base += __popc(ballot);
    }
  } else {
    for (int r = lane; r < nr; r += 32) {
      q_out[r] = r + pr.qbase;
      t_out[r] = col4row_s[r];
    }
  }
  if (a.status != nullptr && lane == 0) a.status[p] = code;
}

int smem_limit() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kSmemLimitDefault;
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      v <= 0) {
    return kSmemLimitDefault;
  }
  return v;
}

int cols_per_lane_for(int max_cols) {
  if (max_cols <= 128) return 4;
  if (max_cols <= 320) return 10;
  if (max_cols <= RFM_MAX_COLS) return 32;
  return -1;
}

// Largest on-chip tile (floats) a CTA may stage: the hardware limit, and a
// soft cap that keeps several CTAs resident per SM.
constexpr int64_t kTileSoftCapFloats = 16384;

int64_t tile_budget(int cols_cap, int max_rows, int64_t max_need) {
  const int64_t hard = (static_cast<int64_t>(kSmemLimitDefault) -
                        fixed_smem_bytes(cols_cap, max_rows)) / 4;
  int64_t t = max_need < kTileSoftCapFloats ? max_need : kTileSoftCapFloats;
  if (t > hard) t = hard;
  return t < 0 ? 0 : t;
}

template <bool kDense>
int launch(const LsapArgs& a, int cols_per_lane, int num_problems, void* stream) {
  const int cols_cap = 32 * cols_per_lane;
  const int64_t smem = fixed_smem_bytes(cols_cap, a.max_rows) + static_cast<int64_t>(a.tile_floats) * 4;
  if (smem > smem_limit()) return RFM_ERR_UNSUPPORTED;
  const void* fn = nullptr;
  switch (cols_per_lane) {
    case 4: fn = reinterpret_cast<const void*>(&lsap_kernel<4, kDense>); break;
    case 10: fn = reinterpret_cast<const void*>(&lsap_kernel<10, kDense>); break;
    case 32: fn = reinterpret_cast<const void*>(&lsap_kernel<32, kDense>); break;
    default: return RFM_ERR_INVALID_ARGUMENT;
  }
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
      return launch_status();
    }
  }
  const dim3 grid(static_cast<unsigned>(num_problems));
  const dim3 block(32);
  switch (cols_per_lane) {
    case 4: lsap_kernel<4, kDense><<<grid, block, smem, as_stream(stream)>>>(a); break;
    case 10: lsap_kernel<10, kDense><<<grid, block, smem, as_stream(stream)>>>(a); break;
    default: lsap_kernel<32, kDense><<<grid, block, smem, as_stream(stream)>>>(a); break;
  }
  return launch_status();
}

}  // namespace
}  // namespace rfm

extern "C" int rfm_lsap_make_plan(rfm_problem* host_problems, int num_problems,
                                  rfm_lsap_plan* plan) {
  using namespace rfm;
  if (plan == nullptr || num_problems < 0 || (num_problems > 0 && host_problems == nullptr)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  int max_cols = 1, max_rows = 1;
  int64_t max_need = 0;
  for (int p = 0; p < num_problems; ++p) {
    const rfm_problem& d = host_problems[p];
    if (d.num_queries < 0 || d.num_targets < 0 || d.cost_offset < 0 || d.out_offset < 0 ||
        d.reserved != 0) {
      return RFM_ERR_INVALID_ARGUMENT;
    }
    const int lo = d.num_queries < d.num_targets ? d.num_queries : d.num_targets;
    const int hi = d.num_queries < d.num_targets ? d.num_targets : d.num_queries;
    if (lo == 0) continue;
    if (hi > max_cols) max_cols = hi;
    if (lo > max_rows) max_rows = lo;
    const int64_t need = tile_need(d.num_queries, d.num_targets);
    if (need > max_need) max_need = need;
  }
  const int cpl = cols_per_lane_for(max_cols);
  if (cpl < 0) return RFM_ERR_UNSUPPORTED;
  const int64_t tile = tile_budget(32 * cpl, max_rows, max_need);
  int64_t scratch = 0;
  for (int p = 0; p < num_problems; ++p) {
    rfm_problem& d = host_problems[p];
    d.scratch_offset = -1;
    const int lo = d.num_queries < d.num_targets ? d.num_queries : d.num_targets;
    if (lo == 0) continue;
    if (tile_need(d.num_queries, d.num_targets) > tile && d.num_targets < d.num_queries) {
      d.scratch_offset = scratch;
      scratch += (static_cast<int64_t>(d.num_queries) * d.num_targets + 3) & ~int64_t(3);
    }
  }
  plan->cols_per_lane = cpl;
  plan->tile_floats = static_cast<int32_t>(tile);
  plan->max_rows = max_rows;
  plan->num_problems = num_problems;
  plan->workspace_bytes = scratch * 4;
  return RFM_OK;
}

extern "C" int rfm_lsap(const float* cost, int64_t ld, const rfm_problem* problems,
                        const rfm_lsap_plan* plan, int64_t* query_out, int64_t* target_out,
                        int32_t* status, void* workspace, void* stream) {
  using namespace rfm;
  if (plan == nullptr || plan->num_problems < 0 || plan->tile_floats < 0 || plan->max_rows < 1 ||
      plan->workspace_bytes < 0 || ld < 0) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (plan->num_problems == 0) return RFM_OK;
  if (cost == nullptr || problems == nullptr || query_out == nullptr || target_out == nullptr ||
      (plan->workspace_bytes > 0 && workspace == nullptr)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  LsapArgs a;
  a.cost = cost;
  a.ld = ld;
  a.problems = problems;
  a.dense_w = 0;
  a.dense_t = 0;
  a.tile_floats = plan->tile_floats;
  a.max_rows = plan->max_rows;
  a.workspace = static_cast<float*>(workspace);
  a.q_out = query_out;
  a.t_out = target_out;
  a.status = status;
  return launch<false>(a, plan->cols_per_lane, plan->num_problems, stream);
}

namespace {
struct DensePlan {
  int cpl;
  int64_t tile;
  int max_rows;
  int64_t scratch_bytes;
};

int dense_plan(int num_problems, int num_workers, int num_tasks, DensePlan* out) {
  using namespace rfm;
  if (num_problems < 0 || num_workers < 0 || num_tasks < 0) return RFM_ERR_INVALID_ARGUMENT;
  const int lo = num_workers < num_tasks ? num_workers : num_tasks;
  const int hi = num_workers < num_tasks ? num_tasks : num_workers;
  out->cpl = cols_per_lane_for(hi < 1 ? 1 : hi);
  if (out->cpl < 0) return RFM_ERR_UNSUPPORTED;
  out->max_rows = lo < 1 ? 1 : lo;
  const int64_t need = lo == 0 ? 0 : tile_need(num_workers, num_tasks);
  out->tile = tile_budget(32 * out->cpl, out->max_rows, need);
  out->scratch_bytes = 0;
  if (lo > 0 && need > out->tile && num_tasks < num_workers) {
    out->scratch_bytes = static_cast<int64_t>(num_problems) * num_workers * num_tasks * 4;
  }
  return RFM_OK;
}
}  // namespace

extern "C" int64_t rfm_lsap_dense_workspace_bytes(int num_problems, int num_workers,
                                                  int num_tasks) {
  DensePlan dp;
  const int rc = dense_plan(num_problems, num_workers, num_tasks, &dp);
  if (rc != RFM_OK) return -static_cast<int64_t>(rc);
  return dp.scratch_bytes;
}

extern "C" int rfm_lsap_dense(const float* cost, int num_problems, int num_workers, int num_tasks,
                              int64_t* matching, int32_t* status, void* workspace, void* stream) {
  using namespace rfm;
  DensePlan dp;
  const int rc = dense_plan(num_problems, num_workers, num_tasks, &dp);
  if (rc != RFM_OK) return rc;
  if (num_problems == 0 || num_workers == 0) return RFM_OK;
  if (matching == nullptr || (num_tasks > 0 && cost == nullptr) ||
      (dp.scratch_bytes > 0 && workspace == nullptr)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  LsapArgs a;
  a.cost = cost;
  a.ld = num_tasks;
  a.problems = nullptr;
  a.dense_w = num_workers;
  a.dense_t = num_tasks;
  a.tile_floats = static_cast<int>(dp.tile);
  a.max_rows = dp.max_rows;
  a.workspace = static_cast<float*>(workspace);
  a.q_out = matching;
  a.t_out = nullptr;
  a.status = status;
  return launch<true>(a, dp.cpl, num_problems, stream);
}
