// TEST INFRASTRUCTURE ONLY (never part of the product).
//
// Times the reference's native search library (oracle/_ref/libcircuit_ref.so,
// compiled unchanged from reference native/src/gpu_index.cpp + api.cpp and its
// kernels) and this repository's libcircuit.so on the same .circuit file and
// the same queries, in one process on one GPU, and writes both libraries'
// results so a test can check them against each other and against float64
// brute force.  Both libraries export the reference's four C entry points
// (reference native/include/circuit/circuit.h:22-46); each is opened with
// dlopen(RTLD_LOCAL) and called through its own function pointers.
//
// Method (as reference native/bin/circuit_bench.cpp:45-140): host buffers ->
// circuit_search one query at a time, host clock around each call; then device
// buffers -> circuit_search_device.  Each library runs twice, alternating, and
// its better round is reported (clocks and caches warm for both).
//
// usage: native_compare <ours.so> <ref.so> <index.circuit> <queries.f32> <nq> <dim> <k> <out_prefix>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace {

struct Trace {
  float latency_us;
  int vectors_scored;
};
using LoadFn = void* (*)(const char*, int);
using SearchFn = int (*)(void*, const float*, int, float*, int*, Trace*);
using DestroyFn = void (*)(void*);

struct Api {
  std::string name;
  LoadFn load = nullptr;
  SearchFn search = nullptr, search_device = nullptr;
  DestroyFn destroy = nullptr;
};

bool open_api(const char* path, const char* name, Api* api) {
  void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    std::fprintf(stderr, "dlopen %s: %s\n", path, dlerror());
    return false;
  }
  api->name = name;
  api->load = (LoadFn)dlsym(h, "circuit_load_index");
  api->search = (SearchFn)dlsym(h, "circuit_search");
  api->search_device = (SearchFn)dlsym(h, "circuit_search_device");
  api->destroy = (DestroyFn)dlsym(h, "circuit_destroy_index");
  return api->load && api->search && api->search_device && api->destroy;
}

double pct(std::vector<double> v, double q) {
  std::sort(v.begin(), v.end());
  return v[std::min(v.size() - 1, (size_t)(v.size() * q))];
}

struct Round {
  double load_ms, host_p50, host_p99, host_qps, dev_p50, dev_p99, dev_qps;
};

bool run(const Api& api, const char* index_path, const std::vector<float>& Q, int nq, int dim, int k,
         std::vector<float>* scores, std::vector<int>* ids, Round* r) {
  using clk = std::chrono::steady_clock;
  auto t0 = clk::now();
  void* h = api.load(index_path, 0);
  if (!h) {
    std::fprintf(stderr, "%s: load failed\n", api.name.c_str());
    return false;
  }
  r->load_ms = std::chrono::duration<double, std::milli>(clk::now() - t0).count();
  float *hq = nullptr, *hs = nullptr;
  int* hi = nullptr;
  cudaMallocHost(&hq, sizeof(float) * dim);
  cudaMallocHost(&hs, sizeof(float) * k);
  cudaMallocHost(&hi, sizeof(int) * k);
  Trace tr{};
  for (int j = 0; j < 50; ++j) {
    std::copy(Q.begin() + (size_t)(j % nq) * dim, Q.begin() + (size_t)(j % nq + 1) * dim, hq);
    if (api.search(h, hq, k, hs, hi, &tr) != 0) {
      std::fprintf(stderr, "%s: search failed\n", api.name.c_str());
      return false;
    }
  }
  std::vector<double> lat;
  auto b0 = clk::now();
  for (int j = 0; j < nq; ++j) {
    std::copy(Q.begin() + (size_t)j * dim, Q.begin() + (size_t)(j + 1) * dim, hq);
    auto q0 = clk::now();
    api.search(h, hq, k, hs, hi, &tr);
    lat.push_back(std::chrono::duration<double, std::micro>(clk::now() - q0).count());
    std::copy(hs, hs + k, scores->begin() + (size_t)j * k);
    std::copy(hi, hi + k, ids->begin() + (size_t)j * k);
  }
  const double host_ms = std::chrono::duration<double, std::milli>(clk::now() - b0).count();
  r->host_p50 = pct(lat, 0.5);
  r->host_p99 = pct(lat, 0.99);
  r->host_qps = nq / host_ms * 1000.0;
  float *dq = nullptr, *ds = nullptr;
  int* di = nullptr;
  cudaMalloc(&dq, sizeof(float) * dim * (size_t)nq);
  cudaMalloc(&ds, sizeof(float) * k);
  cudaMalloc(&di, sizeof(int) * k);
  cudaMemcpy(dq, Q.data(), sizeof(float) * dim * (size_t)nq, cudaMemcpyHostToDevice);
  for (int j = 0; j < 20; ++j) api.search_device(h, dq + (size_t)(j % nq) * dim, k, ds, di, &tr);
  lat.clear();
  b0 = clk::now();
  for (int j = 0; j < nq; ++j) {
    auto q0 = clk::now();
    api.search_device(h, dq + (size_t)j * dim, k, ds, di, &tr);
    lat.push_back(std::chrono::duration<double, std::micro>(clk::now() - q0).count());
  }
  const double dev_ms = std::chrono::duration<double, std::milli>(clk::now() - b0).count();
  r->dev_p50 = pct(lat, 0.5);
  r->dev_p99 = pct(lat, 0.99);
  r->dev_qps = nq / dev_ms * 1000.0;
  cudaFree(dq);
  cudaFree(ds);
  cudaFree(di);
  cudaFreeHost(hq);
  cudaFreeHost(hs);
  cudaFreeHost(hi);
  api.destroy(h);
  return true;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 9) {
    std::fprintf(stderr, "usage: native_compare <ours.so> <ref.so> <index.circuit> <queries.f32> <nq> <dim> <k> <out>\n");
    return 2;
  }
  cudaSetDeviceFlags(cudaDeviceScheduleSpin);  // as reference native/bin/circuit_bench.cpp:12
  const int nq = std::atoi(argv[5]), dim = std::atoi(argv[6]), k = std::atoi(argv[7]);
  std::vector<float> Q((size_t)nq * dim);
  FILE* f = std::fopen(argv[4], "rb");
  if (!f || std::fread(Q.data(), sizeof(float), Q.size(), f) != Q.size()) {
    std::fprintf(stderr, "cannot read queries\n");
    return 1;
  }
  std::fclose(f);
  Api apis[2];
  if (!open_api(argv[1], "ours", &apis[0]) || !open_api(argv[2], "reference", &apis[1])) return 1;
  std::vector<float> scores[2];
  std::vector<int> ids[2];
  Round best[2]{};
  for (int a = 0; a < 2; ++a) {
    scores[a].resize((size_t)nq * k);
    ids[a].resize((size_t)nq * k);
  }
  for (int round = 0; round < 2; ++round) {
    for (int a = 0; a < 2; ++a) {  // ours, reference, ours, reference
      Round r{};
      if (!run(apis[a], argv[3], Q, nq, dim, k, &scores[a], &ids[a], &r)) return 1;
      if (round == 0 || r.host_p50 < best[a].host_p50) best[a] = r;
    }
  }
  for (int a = 0; a < 2; ++a) {
    const std::string out = std::string(argv[8]) + "." + apis[a].name;
    FILE* o = std::fopen((out + ".scores").c_str(), "wb");
    std::fwrite(scores[a].data(), sizeof(float), scores[a].size(), o);
    std::fclose(o);
    o = std::fopen((out + ".ids").c_str(), "wb");
    std::fwrite(ids[a].data(), sizeof(int), ids[a].size(), o);
    std::fclose(o);
    const Round& b = best[a];
    std::printf("{\"lib\": \"%s\", \"load_ms\": %.2f, \"host_p50_us\": %.2f, \"host_p99_us\": %.2f, "
                "\"host_qps\": %.1f, \"dev_p50_us\": %.2f, \"dev_p99_us\": %.2f, \"dev_qps\": %.1f}\n",
                apis[a].name.c_str(), b.load_ms, b.host_p50, b.host_p99, b.host_qps, b.dev_p50, b.dev_p99, b.dev_qps);
  }
  return 0;
}
