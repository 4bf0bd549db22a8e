// circuit_bench: native latency / throughput bench over a .circuit file.
// Same command line as the reference (reference native/bin/circuit_bench.cpp:11-153):
//     circuit_bench [path.circuit] [k] [num_queries] [batch]
// Host-to-host queries (pinned host buffers, H2D + search + D2H per query) and
// in-VRAM queries, p50/p90/p99/mean latency and QPS, then one JSON line.  With
// a fourth argument B > 0 it also times batches of B queries through
// circuit_search_batch (host buffers; no reference counterpart).
// Differences: dim is read from the index (the reference hard-codes 384), k and
// the query count are optional arguments, errors are reported.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <numeric>
#include <random>
#include <vector>

#include "circuit.h"

static void summarize(const char* name, std::vector<double> lat, double total_ms, double* p50_out, double* qps_out) {
  std::sort(lat.begin(), lat.end());
  const size_t n = lat.size();
  const double p50 = lat[n * 50 / 100], p90 = lat[n * 90 / 100], p99 = lat[std::min(n - 1, n * 99 / 100)];
  const double mean = std::accumulate(lat.begin(), lat.end(), 0.0) / n;
  const double qps = n / total_ms * 1000.0;
  std::printf("%-14s p50 %9.2f us | p90 %9.2f us | p99 %9.2f us | mean %9.2f us | %10.1f q/s\n", name, p50, p90, p99,
              mean, qps);
  *p50_out = p50;
  *qps_out = qps;
}

int main(int argc, char** argv) {
  const char* path = argc > 1 ? argv[1] : "data/scifact_index.circuit";
  const int k = argc > 2 ? std::atoi(argv[2]) : 10;
  const int nq = argc > 3 ? std::atoi(argv[3]) : 500;
  const int nb = argc > 4 ? std::atoi(argv[4]) : 0;
  if (k < 1 || nq < 1 || nb < 0) {
    std::fprintf(stderr, "usage: circuit_bench [path.circuit] [k] [num_queries] [batch]\n");
    return 2;
  }
  auto t0 = std::chrono::steady_clock::now();
  circuit_index_t index = circuit_load_index(path, 0);
  auto t1 = std::chrono::steady_clock::now();
  if (!index) {
    std::fprintf(stderr, "error loading index: %s\n", circuit_last_error());
    return 1;
  }
  int64_t info[8];
  circuit_index_info(index, info);
  const int dim = (int)info[0];
  std::printf("loaded %s: N=%lld dim=%d rank=%lld roots=%lld children=%lld in %.1f ms\n", path, (long long)info[4],
              dim, (long long)info[1], (long long)info[2], (long long)info[3],
              std::chrono::duration<double, std::milli>(t1 - t0).count());

  float* h_query = nullptr;
  float* h_scores = nullptr;
  int* h_ids = nullptr;
  cudaMallocHost(&h_query, dim * sizeof(float));
  cudaMallocHost(&h_scores, k * sizeof(float));
  cudaMallocHost(&h_ids, k * sizeof(int));
  std::mt19937 rng(42);
  std::normal_distribution<float> dist(0.f, 1.f);
  for (int d = 0; d < dim; ++d) h_query[d] = dist(rng);
  circuit_trace_t trace;
  for (int i = 0; i < 20; ++i) {
    if (circuit_search(index, h_query, k, h_scores, h_ids, &trace) != 0) {
      std::fprintf(stderr, "search failed: %s\n", circuit_last_error());
      return 1;
    }
  }
  std::vector<double> lat;
  lat.reserve(nq);
  long long scored = 0;
  auto b0 = std::chrono::steady_clock::now();
  for (int i = 0; i < nq; ++i) {
    for (int d = 0; d < dim; ++d) h_query[d] += dist(rng) * 0.05f;  // drift so no two queries match
    auto q0 = std::chrono::steady_clock::now();
    circuit_search(index, h_query, k, h_scores, h_ids, &trace);
    auto q1 = std::chrono::steady_clock::now();
    lat.push_back(std::chrono::duration<double, std::micro>(q1 - q0).count());
    scored += trace.vectors_scored;
  }
  auto b1 = std::chrono::steady_clock::now();
  double p50_h, qps_h, p50_d, qps_d;
  summarize("host-to-host", lat, std::chrono::duration<double, std::milli>(b1 - b0).count(), &p50_h, &qps_h);

  float* d_query = nullptr;
  float* d_scores = nullptr;
  int* d_ids = nullptr;
  cudaMalloc(&d_query, dim * sizeof(float));
  cudaMalloc(&d_scores, k * sizeof(float));
  cudaMalloc(&d_ids, k * sizeof(int));
  cudaMemcpy(d_query, h_query, dim * sizeof(float), cudaMemcpyHostToDevice);
  lat.clear();
  b0 = std::chrono::steady_clock::now();
  for (int i = 0; i < nq; ++i) {
    auto q0 = std::chrono::steady_clock::now();
    circuit_search_device(index, d_query, k, d_scores, d_ids, &trace);
    auto q1 = std::chrono::steady_clock::now();
    lat.push_back(std::chrono::duration<double, std::micro>(q1 - q0).count());
  }
  b1 = std::chrono::steady_clock::now();
  summarize("in-VRAM", lat, std::chrono::duration<double, std::milli>(b1 - b0).count(), &p50_d, &qps_d);

  double batch_qps = 0.0, batch_ms = 0.0;
  if (nb > 0) {
    std::vector<float> hq((size_t)nb * dim), hs((size_t)nb * k);
    std::vector<int> hi((size_t)nb * k);
    for (auto& v : hq) v = dist(rng);
    if (circuit_search_batch(index, hq.data(), nb, k, hs.data(), hi.data()) != 0) {  // warm-up (workspace)
      std::fprintf(stderr, "batched search failed: %s\n", circuit_last_error());
      return 1;
    }
    const int reps = 3;
    auto c0 = std::chrono::steady_clock::now();
    for (int r = 0; r < reps; ++r) circuit_search_batch(index, hq.data(), nb, k, hs.data(), hi.data());
    auto c1 = std::chrono::steady_clock::now();
    batch_ms = std::chrono::duration<double, std::milli>(c1 - c0).count() / reps;
    batch_qps = nb / batch_ms * 1000.0;
    std::printf("%-14s %9.2f ms per batch of %d | %10.1f q/s\n", "batched", batch_ms, nb, batch_qps);
  }

  std::printf("\nsample top-%d (last host query):\n", k);
  for (int i = 0; i < std::min(k, 10); ++i) std::printf("  rank %2d | id %9d | score %.6f\n", i + 1, h_ids[i], h_scores[i]);
  std::printf("{\"bench\": \"circuit_bench\", \"N\": %lld, \"dim\": %d, \"k\": %d, \"queries\": %d, "
              "\"host_p50_us\": %.3f, \"host_qps\": %.1f, \"vram_p50_us\": %.3f, \"vram_qps\": %.1f, "
              "\"mean_vectors_scored\": %.1f, \"batch\": %d, \"batch_ms\": %.3f, \"batch_qps\": %.1f}\n",
              (long long)info[4], dim, k, nq, p50_h, qps_h, p50_d, qps_d, (double)scored / nq, nb, batch_ms, batch_qps);
  circuit_destroy_index(index);
  cudaFree(d_query);
  cudaFree(d_scores);
  cudaFree(d_ids);
  cudaFreeHost(h_query);
  cudaFreeHost(h_scores);
  cudaFreeHost(h_ids);
  return 0;
}
