// The object behind circuit_index_t (internal; see include/circuit.h).
// Replaces reference native/include/circuit/gpu_index.hpp:15-67.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <map>
#include <chrono>
#include <vector>

#include "../../include/circuit.h"
#include "engine.h"

namespace cb {
void set_error(const std::string& msg);
const char* get_error();
bool cuda_ok(cudaError_t e, const char* what);
}  // namespace cb

struct circuit_index_opaque {
  int device = -1;
  int D = 0, rank = 0, R = 0, C = 0, N = 0;
  int max_children = 0;

  cb::IndexView view{};
  cb::Workspace ws{};

  // host-pointer search path
  float* dev_query = nullptr;
  float* dev_scores = nullptr;
  int* dev_ids = nullptr;
  void* h_pinned = nullptr;
  float* h_query = nullptr;
  float* h_scores = nullptr;
  int* h_ids = nullptr;
  cb::SearchCtrl* h_ctrl = nullptr;
  void** h_slots = nullptr;         // device-buffer calls: {query, scores, ids}
  volatile uint32_t* h_seq = nullptr;   // mapped: the blocking call's sequence number
  volatile uint32_t* h_done = nullptr;  // mapped: written by the final merge when the results are out
  uint32_t call_counter = 0;
  bool have_host_ctrl = false;
  // device aliases of the mapped staging block (see cb::HostIO)
  void** dev_out_indirect = nullptr;
  cb::HostIO io_host{}, io_device{};
  float* map_scores = nullptr;
  int* map_ids = nullptr;

  cudaStream_t stream = nullptr;
  // CUDA graphs of the blocking search (prologue kernel, search kernels; the
  // final merge writes into the mapped staging block), one per (k, path,
  // host or device buffers); built on the second call with that key, after a
  // direct call has configured the kernels
  std::map<int, cudaGraphExec_t> host_graphs;
  std::map<int, int> host_graph_calls;
  cudaStream_t last_stream = nullptr;
  int last_path = 0;
  int last_k = 0;

  cb::BatchWorkspace bw{};
  bool batch_ready = false;
  std::vector<void*> batch_owned;  // batch buffers, regrown with the batch size

  std::vector<void*> owned;  // device allocations released by release()
  int fd = -1;
  void* map_ptr = nullptr;
  size_t map_size = 0;

  void* dev_alloc(size_t bytes, const char* what);
  void release();
  bool check_dims();
  bool build_host_tables(const int* parent, const int* offsets, const int* sizes, std::vector<int>* ptr,
                         std::vector<int>* list, std::vector<int>* rows);
  bool finish_setup(const int* parent, const int* offsets, const int* sizes);
  bool parse_file(const char* path, void* tensor_info, std::vector<int>* parent, std::vector<int>* offsets,
                  std::vector<int>* sizes);
  void unmap_file();
  bool load_file(const char* path, int dev);
  bool load_shard_file(const char* path, int dev, int rk, int world, double max_imbalance);
  int64_t shard_rows_read = 0;
  bool wrap_device(int dev, int dim, int rnk, int nr, int nc, int64_t n, const float* const* f, const int* const* ints);
  int search_async(const float* dq, int k, int64_t min_hier, float* dscores, int* dids, int64_t* drows,
                   cudaStream_t st, cudaEvent_t e0, cudaEvent_t e1);
  int search_blocking(const float* query, bool host_ptrs, int k, float* out_scores, int* out_ids,
                      circuit_trace_t* trace);
  bool wait_for_results(uint32_t seq);
  int finish_blocking(bool host_ptrs, int k, float* out_scores, int* out_ids, circuit_trace_t* trace,
                      std::chrono::steady_clock::time_point t0);
  void fill_trace(const cb::SearchCtrl& c, circuit_trace_ex_t* t) const;
  int ensure_batch(int B);
  int search_batch_async(const float* dq, int B, int k, float* dscores, int* dids, cudaStream_t st,
                         cudaEvent_t ev_scan_begin = nullptr, cudaEvent_t ev_scan_end = nullptr);
  // Synchronises `st` and reads the last batch's overflow count and device
  // error bits: CIRCUIT_ERR_TIMEOUT when a bounded wait of that batch gave up.
  int batch_status(cudaStream_t st, int* overflow);
  static float key_to_float(uint32_t k);
};
