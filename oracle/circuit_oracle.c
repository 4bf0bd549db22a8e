/*
 * circuit oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded CPU restatement of the reference's exact top-k
 * search path, used by tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline as the checker.  Nothing in the product (circuit-rag_b200/) links,
 * loads or calls this code.
 *
 * Every function cites the reference file:line it restates.  Arithmetic is
 * available in two precisions: `f64 = 0` accumulates in float32 in the
 * reference kernels' per-element order (sequential here), `f64 = 1`
 * accumulates in double (the "exact" scores the parity tests compare against).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static double dotv(const float* a, const float* b, int n, int f64) {
  if (f64) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)a[i] * (double)b[i];
    return s;
  }
  float s = 0.f;
  for (int i = 0; i < n; ++i) s = fmaf(a[i], b[i], s);
  return (double)s;
}

/* reference native/kernels/root_bounds.cu:31-54:
 *   dot_r = q.c_r; survive iff dot_r + query_norm * radius_r >= threshold */
int oracle_root_bounds(const float* q, const float* centers, const float* radii, int R, int D, double query_norm,
                       double threshold, int f64, int* mask, double* dots) {
  int n = 0;
  for (int r = 0; r < R; ++r) {
    const double d = dotv(q, centers + (size_t)r * D, D, f64);
    dots[r] = d;
    const double bound = f64 ? d + query_norm * radii[r] : (double)((float)d + (float)query_norm * radii[r]);
    mask[r] = bound >= threshold;
    n += mask[r];
  }
  return n;
}

/* reference native/kernels/parent_projection.cu:34-64:
 *   qP_j = sum_d q[d] B[root, d, j];  perp = sqrt(max(||q||^2 - ||qP||^2, 0)) */
void oracle_project(const float* q, const float* bases, const int* roots, int n_roots, int D, int rank,
                    double query_norm_sq, int f64, double* proj /* [R, rank] */, double* perp /* [R] */) {
  for (int s = 0; s < n_roots; ++s) {
    const int p = roots[s];
    const float* B = bases + (size_t)p * D * rank;
    double n2 = 0.0;
    for (int j = 0; j < rank; ++j) {
      double a;
      if (f64) {
        a = 0.0;
        for (int d = 0; d < D; ++d) a += (double)q[d] * (double)B[(size_t)d * rank + j];
      } else {
        float af = 0.f;
        for (int d = 0; d < D; ++d) af = fmaf(q[d], B[(size_t)d * rank + j], af);
        a = af;
      }
      proj[(size_t)p * rank + j] = a;
      n2 += a * a;
    }
    const double ps = query_norm_sq - n2;
    perp[p] = ps > 0.0 ? sqrt(ps) : 0.0;
  }
}

/* reference native/kernels/child_bounds.cu:30-82:
 *   ub = q.c_P + sum_j max(qP_j l_j, qP_j u_j) + perp_P * rho_c; survive iff
 *   the parent survived and ub >= threshold.  ub_out (optional) gets ub. */
int oracle_child_bounds(const double* proj, const double* perp, const double* dots, const float* L, const float* U,
                        const float* rho, const int* parent, const int* root_mask, int C, int rank,
                        double threshold, int* mask, double* ub_out) {
  int n = 0;
  for (int c = 0; c < C; ++c) {
    const int P = parent[c];
    if (!root_mask[P]) {
      mask[c] = 0;
      if (ub_out) ub_out[c] = -INFINITY;
      continue;
    }
    double box = 0.0;
    for (int j = 0; j < rank; ++j) {
      const double a = proj[(size_t)P * rank + j];
      const double x = a * L[(size_t)c * rank + j], y = a * U[(size_t)c * rank + j];
      box += x > y ? x : y;
    }
    const double ub = dots[P] + box + perp[P] * rho[c];
    if (ub_out) ub_out[c] = ub;
    mask[c] = ub >= threshold;
    n += mask[c];
  }
  return n;
}

/* Top-k of scores[0..n) ordered by (score desc, index asc); partial selection
 * with a k-sized sorted buffer.  Returns min(k, n). */
int oracle_topk(const double* scores, int64_t n, int k, int64_t* out_idx, double* out_scores) {
  int m = 0;
  for (int64_t i = 0; i < n; ++i) {
    const double s = scores[i];
    if (m == k && !(s > out_scores[k - 1])) continue;
    int pos = m < k ? m : k - 1;
    while (pos > 0 && s > out_scores[pos - 1]) {
      out_scores[pos] = out_scores[pos - 1];
      out_idx[pos] = out_idx[pos - 1];
      --pos;
    }
    out_scores[pos] = s;
    out_idx[pos] = i;
    if (m < k) ++m;
  }
  return m;
}

/* Brute force (reference circuit_rag/search.py:58-61 and tests/test_exact.py:26):
 * top-k of X q over all N rows, in double; out_rows are row numbers of X. */
int oracle_brute_topk(const float* X, int64_t N, int D, const float* q, int k, double* out_scores, int64_t* out_rows) {
  double* s = (double*)malloc(sizeof(double) * (size_t)N);
  if (!s) return -1;
  for (int64_t i = 0; i < N; ++i) s[i] = dotv(q, X + (size_t)i * D, D, 1);
  const int m = oracle_topk(s, N, k, out_rows, out_scores);
  free(s);
  return m;
}

/* reference circuit_rag/search.py:26-41 (_seed_threshold): best root by
 * argmax(root_centers @ q) (first index on ties); its children are
 * [best*cpr, (best+1)*cpr) with cpr = C / R; the slice of leaf rows from the
 * smallest offset to the largest offset+size of its non-empty children is
 * scored; T = k-th best - 1e-4, or -1e9 when fewer than k rows. */
double oracle_seed_threshold(const float* q, const float* centers, int R, int D, const int* offsets,
                             const int* sizes, int C, const float* leaf, int k, int f64, int* best_out) {
  int best = 0;
  double bd = -INFINITY;
  for (int r = 0; r < R; ++r) {
    const double d = dotv(q, centers + (size_t)r * D, D, f64);
    if (d > bd) { bd = d; best = r; }
  }
  if (best_out) *best_out = best;
  const int cpr = C / R;
  int64_t start = INT64_MAX, end = -1;
  for (int c = best * cpr; c < (best + 1) * cpr && c < C; ++c) {
    if (sizes[c] <= 0) continue;
    if (offsets[c] < start) start = offsets[c];
    if ((int64_t)offsets[c] + sizes[c] > end) end = (int64_t)offsets[c] + sizes[c];
  }
  if (end < 0 || end - start < k) return -1e9;
  double* s = (double*)malloc(sizeof(double) * (size_t)(end - start));
  int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)k);
  double* top = (double*)malloc(sizeof(double) * (size_t)k);
  if (!s || !idx || !top) { free(s); free(idx); free(top); return -1e9; }
  for (int64_t i = start; i < end; ++i) s[i - start] = dotv(q, leaf + (size_t)i * D, D, f64);
  oracle_topk(s, end - start, k, idx, top);
  const double T = top[k - 1] - 1e-4;
  free(s); free(idx); free(top);
  return T;
}

/* The reference hierarchical pipeline (native/src/dispatch.cu:244-307 driven by
 * circuit_rag/search.py:63-84): seed threshold, root bounds, projection of
 * surviving roots, child bounds, scores of surviving children's rows (others
 * -inf), top-k, ids mapped through original_ids.  Scores in double.  Returns
 * the number of results; *n_scored gets the number of rows scored and
 * child_mask (optional, [C]) the surviving children. */
int oracle_hierarchical_search(const float* q, const float* centers, const float* radii, const float* bases,
                               const float* L, const float* U, const float* rho, const int* parent,
                               const int* offsets, const int* sizes, const float* leaf, const int* original_ids,
                               int R, int C, int64_t N, int D, int rank, int k, double* out_scores, int* out_ids,
                               int64_t* n_scored, int* child_mask) {
  const double T = oracle_seed_threshold(q, centers, R, D, offsets, sizes, C, leaf, k, 1, NULL);
  const double qn = sqrt(dotv(q, q, D, 1));
  int* rmask = (int*)calloc((size_t)R, sizeof(int));
  int* roots = (int*)malloc(sizeof(int) * (size_t)R);
  double* dots = (double*)malloc(sizeof(double) * (size_t)R);
  double* proj = (double*)calloc((size_t)R * rank, sizeof(double));
  double* perp = (double*)calloc((size_t)R, sizeof(double));
  int* cmask = child_mask ? child_mask : (int*)malloc(sizeof(int) * (size_t)C);
  double* s = (double*)malloc(sizeof(double) * (size_t)N);
  int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)k);
  if (!rmask || !roots || !dots || !proj || !perp || !cmask || !s || !idx) return -1;
  oracle_root_bounds(q, centers, radii, R, D, qn, T, 1, rmask, dots);
  int nr = 0;
  for (int r = 0; r < R; ++r)
    if (rmask[r]) roots[nr++] = r;
  oracle_project(q, bases, roots, nr, D, rank, qn * qn, 1, proj, perp);
  oracle_child_bounds(proj, perp, dots, L, U, rho, parent, rmask, C, rank, T, cmask, NULL);
  for (int64_t i = 0; i < N; ++i) s[i] = -INFINITY;
  int64_t scored = 0;
  for (int c = 0; c < C; ++c) {
    if (!cmask[c]) continue;
    for (int64_t v = offsets[c]; v < (int64_t)offsets[c] + sizes[c]; ++v) {
      s[v] = dotv(q, leaf + (size_t)v * D, D, 1);
      ++scored;
    }
  }
  const int m = oracle_topk(s, N, k, idx, out_scores);
  for (int i = 0; i < m; ++i) out_ids[i] = original_ids ? original_ids[idx[i]] : (int)idx[i];
  if (n_scored) *n_scored = scored;
  free(rmask); free(roots); free(dots); free(proj); free(perp); free(s); free(idx);
  if (!child_mask) free(cmask);
  return m;
}
