// TEST INFRASTRUCTURE ONLY.  extern "C" entry points over the reference's own
// per-stage launchers (reference native/include/circuit/dispatch.h:7-139), so
// GPU tests can run the unmodified reference kernels on the same inputs as ours.
// Compiled together with the reference sources by oracle/Makefile into
// oracle/_ref/libcircuit_ref.so; nothing in the product loads it.
#include <cuda_runtime.h>

#include "circuit/dispatch.h"

extern "C" {

int ref_root_bounds(const float* q, const float* centers, const float* radii, float qnorm, float threshold, int R,
                    int D, int* mask, int* idx, int* count, float* dots) {
  cudaMemset(count, 0, sizeof(int));
  circuit::launch_evaluate_root_bounds(q, centers, radii, qnorm, threshold, R, D, mask, idx, count, dots, 0);
  return (int)cudaDeviceSynchronize();
}

int ref_project(const float* q, float qn2, const float* bases, const int* idx, int n, int D, int rank, float* proj,
                float* perp) {
  circuit::launch_parent_projection(q, qn2, bases, idx, n, D, rank, proj, perp, 0);
  return (int)cudaDeviceSynchronize();
}

int ref_child_bounds(const float* proj, const float* perp, const float* dots, const float* L, const float* U,
                     const float* rho, const int* parent, const int* root_mask, float threshold, int C, int rank,
                     int* mask, int* idx, int* count) {
  cudaMemset(count, 0, sizeof(int));
  circuit::launch_evaluate_child_bounds(proj, perp, dots, L, U, rho, parent, root_mask, threshold, C, rank, mask, idx,
                                        count, 0);
  return (int)cudaDeviceSynchronize();
}

int ref_flat_score(const float* q, const float* corpus, int N, int D, float* scores) {
  circuit::launch_flat_exact_score(q, corpus, N, D, scores, 0);
  return (int)cudaDeviceSynchronize();
}

int ref_select_topk(const float* scores, const int* ids, int N, int K, float* out_scores, int* out_ids) {
  circuit::launch_select_topk(scores, ids, N, K, out_scores, out_ids, 0);
  return (int)cudaDeviceSynchronize();
}

}  // extern "C"
