/*
 * oracle/lsap.c - TEST INFRASTRUCTURE ONLY.  CPU restatement of the
 * rectangular linear-sum-assignment algorithm that the reference's CPU path
 * runs: scipy.optimize.linear_sum_assignment (SciPy 1.18.1, the
 * `rectangular_lsap` shortest-augmenting-path solver after Crouse, "On
 * implementing 2D rectangular assignment algorithms", IEEE TAES 2016).
 *
 * The reference calls it per problem at kernels_lap.py:370-379 (its
 * verification oracle) and on a thread pool at patches.py:213-229 (the CPU
 * path it times); SciPy is a third-party dependency that is not vendored in
 * the reference, so this file restates the published algorithm and the test
 * suite pins it index-for-index against the installed SciPy.
 *
 * It is the checker for the CUDA solver and is never linked into the product
 * library.
 *
 * Semantics restated:
 *   - float32 input entries are promoted to float64; all arithmetic is
 *     float64, with the reduced cost evaluated as ((minv + c) - u[i]) - v[j];
 *   - a tall matrix (rows > cols) is solved transposed;
 *   - the column scan visits the `remaining` array in order; `remaining`
 *     starts reverse-filled and loses one column per step by swap-with-last;
 *     a strictly smaller path cost wins, and an equal one wins when its
 *     column is unassigned;
 *   - NaN or -inf entries are rejected; an all-+inf frontier is infeasible;
 *   - results come back ordered by row of the ORIGINAL matrix.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_INFEASIBLE 1
#define ORACLE_INVALID 2

/* Shortest augmenting path from free row `row0`; returns the sink column or -1. */
static int64_t shortest_path(int64_t nr, int64_t nc, const double* c, const double* u,
                             const double* v, int64_t* path, const int64_t* row4col,
                             double* spc, int64_t row0, char* in_row, char* in_col,
                             int64_t* remaining, double* out_min) {
  double minv = 0.0;
  int64_t left = nc;
  for (int64_t k = 0; k < nc; ++k) remaining[k] = nc - 1 - k;
  memset(in_row, 0, (size_t)nr);
  memset(in_col, 0, (size_t)nc);
  for (int64_t j = 0; j < nc; ++j) spc[j] = INFINITY;

  int64_t i = row0;
  int64_t sink = -1;
  while (sink == -1) {
    in_row[i] = 1;
    int64_t best = -1;
    double lowest = INFINITY;
    for (int64_t k = 0; k < left; ++k) {
      const int64_t j = remaining[k];
      const double r = ((minv + c[i * nc + j]) - u[i]) - v[j];
      if (r < spc[j]) {
        path[j] = i;
        spc[j] = r;
      }
      if (spc[j] < lowest || (spc[j] == lowest && row4col[j] == -1)) {
        lowest = spc[j];
        best = k;
      }
    }
    minv = lowest;
    if (minv == INFINITY) return -1;
    const int64_t j = remaining[best];
    if (row4col[j] == -1) {
      sink = j;
    } else {
      i = row4col[j];
    }
    in_col[j] = 1;
    remaining[best] = remaining[--left];
  }
  *out_min = minv;
  return sink;
}

/*
 * Solve one problem.  cost is row-major [nr0 x nc0] float32 with row stride
 * ld.  On success writes min(nr0, nc0) pairs (row, col) of the ORIGINAL
 * orientation into rows_out/cols_out, sorted by row.
 */
int oracle_lsap(int64_t nr0, int64_t nc0, const float* cost, int64_t ld, int64_t* rows_out,
                int64_t* cols_out) {
  if (nr0 < 0 || nc0 < 0 || ld < nc0) return ORACLE_INVALID;
  if (nr0 == 0 || nc0 == 0) return ORACLE_OK;
  const int transpose = nc0 < nr0;
  const int64_t nr = transpose ? nc0 : nr0;
  const int64_t nc = transpose ? nr0 : nc0;

  double* c = (double*)malloc(sizeof(double) * (size_t)(nr * nc));
  for (int64_t a = 0; a < nr0; ++a) {
    for (int64_t b = 0; b < nc0; ++b) {
      const double x = (double)cost[a * ld + b];
      if (x != x || x == -INFINITY) {
        free(c);
        return ORACLE_INVALID;
      }
      if (transpose) {
        c[b * nc + a] = x;
      } else {
        c[a * nc + b] = x;
      }
    }
  }

  double* u = (double*)calloc((size_t)nr, sizeof(double));
  double* v = (double*)calloc((size_t)nc, sizeof(double));
  double* spc = (double*)malloc(sizeof(double) * (size_t)nc);
  int64_t* path = (int64_t*)malloc(sizeof(int64_t) * (size_t)nc);
  int64_t* col4row = (int64_t*)malloc(sizeof(int64_t) * (size_t)nr);
  int64_t* row4col = (int64_t*)malloc(sizeof(int64_t) * (size_t)nc);
  int64_t* remaining = (int64_t*)malloc(sizeof(int64_t) * (size_t)nc);
  char* in_row = (char*)malloc((size_t)nr);
  char* in_col = (char*)malloc((size_t)nc);
  for (int64_t j = 0; j < nc; ++j) {
    path[j] = -1;
    row4col[j] = -1;
  }
  for (int64_t i = 0; i < nr; ++i) col4row[i] = -1;

  int rc = ORACLE_OK;
  for (int64_t row = 0; row < nr; ++row) {
    double minv = 0.0;
    const int64_t sink = shortest_path(nr, nc, c, u, v, path, row4col, spc, row, in_row, in_col,
                                       remaining, &minv);
    if (sink < 0) {
      rc = ORACLE_INFEASIBLE;
      break;
    }
    /* dual update: the tree's rows and columns shift by their slack */
    u[row] += minv;
    for (int64_t i = 0; i < nr; ++i) {
      if (in_row[i] && i != row) u[i] += minv - spc[col4row[i]];
    }
    for (int64_t j = 0; j < nc; ++j) {
      if (in_col[j]) v[j] -= minv - spc[j];
    }
    /* flip the alternating path back from the sink */
    int64_t j = sink;
    for (;;) {
      const int64_t i = path[j];
      row4col[j] = i;
      const int64_t prev = col4row[i];
      col4row[i] = j;
      j = prev;
      if (i == row) break;
    }
  }

  if (rc == ORACLE_OK) {
    if (transpose) {
      /* original rows are the solver's columns: emit in ascending order */
      int64_t k = 0;
      for (int64_t j = 0; j < nc; ++j) {
        if (row4col[j] >= 0) {
          rows_out[k] = j;
          cols_out[k] = row4col[j];
          ++k;
        }
      }
    } else {
      for (int64_t i = 0; i < nr; ++i) {
        rows_out[i] = i;
        cols_out[i] = col4row[i];
      }
    }
  }
  free(c);
  free(u);
  free(v);
  free(spc);
  free(path);
  free(col4row);
  free(row4col);
  free(remaining);
  free(in_row);
  free(in_col);
  return rc;
}

/*
 * Batched form over the same problem descriptors the CUDA solver reads:
 * desc[p] = {cost_offset, out_offset, num_queries, num_targets, query_base}
 * (int64 x 5).  Pairs are written at out_offset with query_base added to
 * the query index; status[p] receives ORACLE_*.  Failed problems get -1.
 */
void oracle_lsap_batch(const float* cost, int64_t ld, const int64_t* desc, int64_t num_problems,
                       int64_t* query_out, int64_t* target_out, int32_t* status) {
  for (int64_t p = 0; p < num_problems; ++p) {
    const int64_t* d = desc + 5 * p;
    const int64_t nq = d[2], nt = d[3];
    const int64_t n = nq < nt ? nq : nt;
    const int rc = oracle_lsap(nq, nt, cost + d[0], ld, query_out + d[1], target_out + d[1]);
    status[p] = rc;
    for (int64_t k = 0; k < n; ++k) {
      if (rc == ORACLE_OK) {
        query_out[d[1] + k] += d[4];
      } else {
        query_out[d[1] + k] = -1;
        target_out[d[1] + k] = -1;
      }
    }
  }
}
