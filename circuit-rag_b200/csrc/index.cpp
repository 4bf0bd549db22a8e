// Native index object and the C ABI of include/circuit.h.
//
// Replaces the reference's native host library:
//   native/src/api.cpp:7-51          (entry points, NULL / -1 conventions)
//   native/src/gpu_index.cpp:50-141  (mmap + header parse + upload + workspace)
//   native/src/gpu_index.cpp:242-386 (host / device search)
// Differences: every CUDA call is checked; the header is parsed as JSON; the
// file is validated (sizes, offsets, child ranges) before any device work;
// large tensors are uploaded through pinned double-buffered staging; pruning is
// on; k is not clamped to 32.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <new>
#include <string>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/circuit.h"
#include "../../include/circuit_shard.h"
#include "engine.h"
#include "index_internal.h"
#include "json_min.h"

using cb::Workspace;

namespace {

thread_local std::string g_last_error;

}  // namespace

namespace cb {

void set_error(const std::string& msg) { g_last_error = msg; }
const char* get_error() { return g_last_error.c_str(); }

bool cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return false;
}

}  // namespace cb

using cb::cuda_ok;
using cb::set_error;

// ---------------------------------------------------------------- helpers
static const char* kTensorNames[11] = {"root_centers",      "root_radii",       "bases",        "child_intervals_l",
                                       "child_intervals_u", "child_radii",      "child_parent_ids",
                                       "leaf_offsets",      "leaf_sizes",       "leaf_vectors", "original_ids"};

void* circuit_index_opaque::dev_alloc(size_t bytes, const char* what) {
  void* p = nullptr;
  if (bytes == 0) bytes = 16;
  if (!cuda_ok(cudaMalloc(&p, bytes), what)) return nullptr;
  owned.push_back(p);
  return p;
}

void circuit_index_opaque::release() {
  if (device >= 0 && (stream || !owned.empty() || h_pinned)) cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  for (auto& g : host_graphs) cudaGraphExecDestroy(g.second);
  host_graphs.clear();
  for (void* p : owned) cudaFree(p);
  owned.clear();
  for (void* p : batch_owned) cudaFree(p);
  batch_owned.clear();
  if (h_pinned) cudaFreeHost(h_pinned);
  h_pinned = nullptr;
  if (stream) cudaStreamDestroy(stream);
  stream = nullptr;
  if (map_ptr && map_ptr != MAP_FAILED) munmap(map_ptr, map_size);
  map_ptr = nullptr;
  if (fd >= 0) close(fd);
  fd = -1;
}

// Validates the small per-child arrays and builds the per-root CSR of
// non-empty children (sorted by leaf offset) and the per-root row counts.
bool circuit_index_opaque::build_host_tables(const int* parent, const int* offsets, const int* sizes,
                                             std::vector<int>* ptr, std::vector<int>* list, std::vector<int>* rows) {
  ptr->assign(R + 1, 0);
  rows->assign(R, 0);
  std::vector<std::pair<int64_t, int64_t>> spans;
  spans.reserve(C);
  int64_t covered = 0;
  for (int c = 0; c < C; ++c) {
    const int64_t sz = sizes[c], off = offsets[c];
    if (sz < 0) { set_error("leaf_sizes has a negative entry"); return false; }
    if (sz == 0) continue;
    if (parent[c] < 0 || parent[c] >= R) { set_error("child_parent_ids out of range for a non-empty child"); return false; }
    if (off < 0 || off + sz > N) { set_error("leaf_offsets/leaf_sizes reach outside leaf_vectors"); return false; }
    (*ptr)[parent[c] + 1] += 1;
    (*rows)[parent[c]] += (int)sz;
    spans.emplace_back(off, sz);
    covered += sz;
  }
  std::sort(spans.begin(), spans.end());
  for (size_t i = 1; i < spans.size(); ++i)
    if (spans[i - 1].first + spans[i - 1].second > spans[i].first) {
      set_error("child leaf ranges overlap");
      return false;
    }
  if (covered != N) {
    set_error("children do not cover all N leaf rows (" + std::to_string(covered) + " of " + std::to_string(N) + ")");
    return false;
  }
  for (int p = 0; p < R; ++p) (*ptr)[p + 1] += (*ptr)[p];
  list->assign((*ptr)[R], 0);
  std::vector<int> fill(ptr->begin(), ptr->end() - 1);
  for (int c = 0; c < C; ++c)
    if (sizes[c] > 0) (*list)[fill[parent[c]]++] = c;
  for (int p = 0; p < R; ++p)
    std::sort(list->begin() + (*ptr)[p], list->begin() + (*ptr)[p + 1],
              [&](int a, int b) { return offsets[a] < offsets[b]; });
  max_children = 0;
  for (int p = 0; p < R; ++p) max_children = std::max(max_children, (*ptr)[p + 1] - (*ptr)[p]);
  return true;
}

bool circuit_index_opaque::finish_setup(const int* parent, const int* offsets, const int* sizes) {
  std::vector<int> ptr, list, rows;
  if (!build_host_tables(parent, offsets, sizes, &ptr, &list, &rows)) return false;
  int* d_ptr = (int*)dev_alloc(sizeof(int) * ptr.size(), "cudaMalloc(root_child_ptr)");
  int* d_list = (int*)dev_alloc(sizeof(int) * std::max<size_t>(list.size(), 1), "cudaMalloc(root_child_list)");
  int* d_rows = (int*)dev_alloc(sizeof(int) * rows.size(), "cudaMalloc(root_rows)");
  // per CSR entry: the child's leaf offset and where its rows start among its root's rows
  std::vector<int2> span(std::max<size_t>(list.size(), 1), make_int2(0, 0));
  for (int p = 0; p < R; ++p) {
    int v = 0;
    for (int i = ptr[p]; i < ptr[p + 1]; ++i) {
      span[i] = make_int2(offsets[list[i]], v);
      v += sizes[list[i]];
    }
  }
  int2* d_span = (int2*)dev_alloc(sizeof(int2) * span.size(), "cudaMalloc(root_child_span)");
  // the seed sample of every root for k <= 32 (want = min(rows, 128)), with the
  // same arithmetic as the root scan's on-device computation for larger k
  std::vector<int4> tab((size_t)R * cb::SEED_TAB_W, make_int4(0, 0, 0, 0));
  for (int p = 0; p < R; ++p) {
    const int cb0 = ptr[p], nall = ptr[p + 1] - cb0;
    const int nch = std::min(nall, cb::SEED_SAMPLE_MAX);
    if (nch == 0) continue;
    const int vrows = nall > nch ? span[cb0 + nch].y : rows[p];
    const int want = std::min(std::min(vrows, 128), cb::SEED_SAMPLE_MAX);
    const int nb = (want + cb::SEED_BLOCK - 1) / cb::SEED_BLOCK;
    int pos = 0;
    for (int b = 0; b < nb; ++b) {
      const int v = (int)std::floor((double)b * (double)vrows / (double)nb);
      const int v_next = (b + 1 < nb) ? (int)std::floor((double)(b + 1) * (double)vrows / (double)nb) : vrows;
      int lo = 0, hi = nch - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (span[cb0 + mid].y <= v) lo = mid; else hi = mid - 1;
      }
      const int child_end = (lo + 1 < nch) ? span[cb0 + lo + 1].y : vrows;
      const int len = std::min(std::min(cb::SEED_BLOCK, v_next - v), child_end - v);
      tab[(size_t)p * cb::SEED_TAB_W + 1 + b] = make_int4(span[cb0 + lo].x + (v - span[cb0 + lo].y), len, pos, 0);
      pos += len;
    }
    tab[(size_t)p * cb::SEED_TAB_W] = make_int4(nb, pos, 0, 0);
  }
  int4* d_tab = (int4*)dev_alloc(sizeof(int4) * tab.size(), "cudaMalloc(seed_tab)");
  // the hierarchical main scan's static range list: every CSR entry in order,
  // virtual rows numbered along it (children cover all N rows)
  const size_t nnz = list.size();
  std::vector<int4> all(std::max<size_t>(nnz, 1), make_int4(0, 0, 0, -1));
  {
    int v = 0;
    for (size_t i = 0; i < nnz; ++i) {
      const int c = list[i];
      all[i] = make_int4(v, offsets[c], offsets[c] + sizes[c], c);
      v += sizes[c];
    }
  }
  const unsigned long long all_packed = ((unsigned long long)nnz << 32) | (unsigned long long)(uint32_t)N;
  int4* d_all = (int4*)dev_alloc(sizeof(int4) * all.size(), "cudaMalloc(all_ranges)");
  unsigned long long* d_all_packed = (unsigned long long*)dev_alloc(sizeof(unsigned long long), "cudaMalloc(all_packed)");
  double* d_cn = (double*)dev_alloc(sizeof(double) * R, "cudaMalloc(root_cn)");
  double* d_def = (double*)dev_alloc(sizeof(double) * R, "cudaMalloc(root_defect)");
  if (!d_ptr || !d_list || !d_rows || !d_cn || !d_def || !d_span || !d_tab || !d_all || !d_all_packed) return false;
  if (!cuda_ok(cudaMemcpyAsync(d_ptr, ptr.data(), sizeof(int) * ptr.size(), cudaMemcpyHostToDevice, stream), "H2D ptr") ||
      (!list.empty() && !cuda_ok(cudaMemcpyAsync(d_list, list.data(), sizeof(int) * list.size(),
                                                 cudaMemcpyHostToDevice, stream),
                                 "H2D list")) ||
      !cuda_ok(cudaMemcpyAsync(d_rows, rows.data(), sizeof(int) * rows.size(), cudaMemcpyHostToDevice, stream), "H2D rows") ||
      !cuda_ok(cudaMemcpyAsync(d_span, span.data(), sizeof(int2) * span.size(), cudaMemcpyHostToDevice, stream),
               "H2D spans") ||
      !cuda_ok(cudaMemcpyAsync(d_tab, tab.data(), sizeof(int4) * tab.size(), cudaMemcpyHostToDevice, stream),
               "H2D seed table") ||
      !cuda_ok(cudaMemcpyAsync(d_all, all.data(), sizeof(int4) * all.size(), cudaMemcpyHostToDevice, stream),
               "H2D range list") ||
      !cuda_ok(cudaMemcpyAsync(d_all_packed, &all_packed, sizeof(all_packed), cudaMemcpyHostToDevice, stream),
               "H2D range count"))
    return false;
  view.root_child_ptr = d_ptr;
  view.root_child_list = d_list;
  view.root_child_span = d_span;
  view.seed_tab = d_tab;
  view.all_ranges = d_all;
  view.all_packed = d_all_packed;
  view.all_nnz = (int)nnz;
  view.root_rows = d_rows;
  view.root_cn = d_cn;
  view.root_defect = d_def;
  if (!cuda_ok(cb::launch_prepare_roots(view, d_cn, d_def, stream), "prepare_roots")) return false;

  // workspace
  ws.scan_grid = cb::sm_count(device);
  ws.ctrl = (cb::SearchCtrl*)dev_alloc(sizeof(cb::SearchCtrl), "cudaMalloc(ctrl)");
  ws.epoch_counter = (uint32_t*)dev_alloc(sizeof(uint32_t), "cudaMalloc(epoch)");
  ws.sync = (cb::ScanSync*)dev_alloc(sizeof(cb::ScanSync), "cudaMalloc(scan sync)");
  ws.ub_tagged = (unsigned long long*)dev_alloc(sizeof(unsigned long long) * std::max<size_t>(nnz, 1),
                                                "cudaMalloc(ub_tagged)");
  // chunks of the hierarchical main scan: the range holding each chunk's first row
  ws.chunk_rows = cb::overlap_chunk_rows(N, D, ws.scan_grid);
  std::vector<int> first((size_t)(((int64_t)N + ws.chunk_rows - 1) / ws.chunk_rows), 0);
  {
    size_t i = 0;
    for (size_t c = 0; c < first.size(); ++c) {
      const int64_t v = (int64_t)c * ws.chunk_rows;
      while (i + 1 < nnz && all[i + 1].x <= v) ++i;
      first[c] = (int)i;
    }
  }
  int* d_first = (int*)dev_alloc(sizeof(int) * std::max<size_t>(first.size(), 1), "cudaMalloc(chunk table)");
  ws.chunk_first_range = d_first;
  ws.n_chunks = (int)first.size();
  ws.chunk_mark = (uint32_t*)dev_alloc(sizeof(uint32_t) * std::max<size_t>(first.size(), 1), "cudaMalloc(chunk marks)");
  ws.live_list = (int*)dev_alloc(sizeof(int) * std::max<size_t>(first.size(), 1), "cudaMalloc(live list)");
  ws.chunk_taken = (uint32_t*)dev_alloc(sizeof(uint32_t) * std::max<size_t>(first.size(), 1), "cudaMalloc(taken)");
  ws.flat_range = (int4*)dev_alloc(sizeof(int4), "cudaMalloc(flat_range)");
  ws.flat_packed = (unsigned long long*)dev_alloc(sizeof(unsigned long long), "cudaMalloc(flat_packed)");
  ws.ub_root = (float*)dev_alloc(sizeof(float) * R, "cudaMalloc(ub_root)");
  ws.ub_child = (float*)dev_alloc(sizeof(float) * C, "cudaMalloc(ub_child)");
  ws.cta_lists = (unsigned long long*)dev_alloc(sizeof(unsigned long long) * (size_t)(ws.scan_grid + 1) * cb::KMAX,
                                                "cudaMalloc(cta_lists)");
  dev_query = (float*)dev_alloc(sizeof(float) * D, "cudaMalloc(query)");
  dev_scores = (float*)dev_alloc(sizeof(float) * cb::KMAX, "cudaMalloc(scores)");
  dev_ids = (int*)dev_alloc(sizeof(int) * cb::KMAX, "cudaMalloc(ids)");
  dev_out_indirect = (void**)dev_alloc(2 * sizeof(void*), "cudaMalloc(out pointers)");
  if (!ws.ctrl || !ws.sync || !ws.epoch_counter || !ws.ub_tagged || !d_first || !ws.chunk_mark || !ws.live_list ||
      !ws.chunk_taken ||
      !ws.flat_range || !ws.flat_packed ||
      !ws.ub_root || !ws.ub_child ||
      !ws.cta_lists || !dev_query || !dev_scores || !dev_ids || !dev_out_indirect)
    return false;
  const int4 fr = make_int4(0, 0, N, -1);
  const unsigned long long fp = (1ull << 32) | (unsigned long long)(uint32_t)N;
  if (!cuda_ok(cudaMemcpyAsync(ws.flat_range, &fr, sizeof(fr), cudaMemcpyHostToDevice, stream), "H2D flat range") ||
      !cuda_ok(cudaMemcpyAsync(ws.flat_packed, &fp, sizeof(fp), cudaMemcpyHostToDevice, stream), "H2D flat packed") ||
      !cuda_ok(cudaMemsetAsync(ws.ctrl, 0, sizeof(cb::SearchCtrl), stream), "memset ctrl") ||
      !cuda_ok(cudaMemsetAsync(ws.epoch_counter, 0, sizeof(uint32_t), stream), "memset epoch") ||
      !cuda_ok(cudaMemsetAsync(ws.sync, 0, sizeof(cb::ScanSync), stream), "memset scan sync") ||
      !cuda_ok(cudaMemsetAsync(ws.chunk_mark, 0, sizeof(uint32_t) * std::max<size_t>(first.size(), 1), stream),
               "memset chunk marks") ||
      !cuda_ok(cudaMemsetAsync(ws.chunk_taken, 0, sizeof(uint32_t) * std::max<size_t>(first.size(), 1), stream),
               "memset taken") ||
      !cuda_ok(cudaMemsetAsync(ws.ub_tagged, 0, sizeof(unsigned long long) * std::max<size_t>(nnz, 1), stream),
               "memset bounds") ||
      (!first.empty() && !cuda_ok(cudaMemcpyAsync(d_first, first.data(), sizeof(int) * first.size(),
                                                  cudaMemcpyHostToDevice, stream),
                                  "H2D chunk table")))
    return false;
  // pinned, device-mapped host staging for the blocking search: query, scores,
  // ids, ctrl header, call slots.  Graph replays read the query from it and
  // write the results into it from the kernels themselves.
  const size_t pin_bytes = sizeof(float) * D + (sizeof(float) + sizeof(int)) * cb::KMAX + sizeof(cb::SearchCtrl) +
                           4 * sizeof(void*) + 2 * sizeof(uint32_t);
  if (!cuda_ok(cudaHostAlloc(&h_pinned, pin_bytes, cudaHostAllocMapped), "cudaHostAlloc")) return false;
  h_query = (float*)h_pinned;
  h_scores = h_query + D;
  h_ids = (int*)(h_scores + cb::KMAX);
  h_ctrl = (cb::SearchCtrl*)(h_ids + cb::KMAX);
  h_slots = (void**)(h_ctrl + 1);
  h_seq = (volatile uint32_t*)(h_slots + 4);
  h_done = h_seq + 1;
  *h_seq = 0;
  *h_done = 0;
  void* d_pinned = nullptr;
  if (!cuda_ok(cudaHostGetDevicePointer(&d_pinned, h_pinned, 0), "cudaHostGetDevicePointer")) return false;
  const auto alias = [&](const void* h) { return (char*)d_pinned + ((const char*)h - (const char*)h_pinned); };
  io_host = cb::HostIO{(const float*)alias(h_query), nullptr, dev_out_indirect, (cb::SearchCtrl*)alias(h_ctrl),
                       (const uint32_t*)alias((const void*)h_seq), (uint32_t*)alias((const void*)h_done)};
  io_device = cb::HostIO{nullptr, (void* const*)alias(h_slots), dev_out_indirect, (cb::SearchCtrl*)alias(h_ctrl),
                         (const uint32_t*)alias((const void*)h_seq), (uint32_t*)alias((const void*)h_done)};
  map_scores = (float*)alias(h_scores);
  map_ids = (int*)alias(h_ids);
  if (!cuda_ok(cudaStreamSynchronize(stream), "index setup")) return false;
  return true;
}

bool circuit_index_opaque::check_dims() {
  if (D <= 0 || D % 4 != 0 || D > cb::MAX_DIM) {
    set_error("dim must be a positive multiple of 4 and <= " + std::to_string(cb::MAX_DIM));
    return false;
  }
  if (rank <= 0 || rank > cb::MAX_RANK) {
    set_error("rank must be in [1, " + std::to_string(cb::MAX_RANK) + "]");
    return false;
  }
  if (R <= 0 || C <= 0 || N <= 0) { set_error("num_roots, num_total_children and N must be positive"); return false; }
  if (R >= (1 << 30)) { set_error("num_roots too large"); return false; }
  view.D = D;
  view.D4 = D / 4;
  view.rank = rank;
  view.R = R;
  view.C = C;
  view.N = N;
  return true;
}

// ---------------------------------------------------------------- file loading
namespace {
struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t offset = 0, nbytes = 0;
};

// Host -> device copies through two pinned 64 MiB staging buffers: the memcpy
// into one buffer overlaps the DMA out of the other.
class StagedUpload {
 public:
  explicit StagedUpload(cudaStream_t st) : st_(st) {
    ok_ = cuda_ok(cudaMallocHost(&stage_[0], kChunk), "cudaMallocHost(stage)") &&
          cuda_ok(cudaMallocHost(&stage_[1], kChunk), "cudaMallocHost(stage)") &&
          cuda_ok(cudaEventCreateWithFlags(&done_[0], cudaEventDisableTiming), "cudaEventCreate") &&
          cuda_ok(cudaEventCreateWithFlags(&done_[1], cudaEventDisableTiming), "cudaEventCreate");
  }
  ~StagedUpload() {
    for (int i = 0; i < 2; ++i) {
      if (done_[i]) cudaEventDestroy(done_[i]);
      if (stage_[i]) cudaFreeHost(stage_[i]);
    }
  }
  // copies [src, src + bytes) to dst (device)
  bool put(void* dst, const char* src, size_t bytes) {
    size_t pos = 0;
    while (ok_ && pos < bytes) {
      const size_t n = std::min(bytes - pos, kChunk);
      if (used_[slot_]) ok_ = cuda_ok(cudaEventSynchronize(done_[slot_]), "staging wait");
      if (!ok_) break;
      std::memcpy(stage_[slot_], src + pos, n);
      ok_ = cuda_ok(cudaMemcpyAsync((char*)dst + pos, stage_[slot_], n, cudaMemcpyHostToDevice, st_), "H2D") &&
            cuda_ok(cudaEventRecord(done_[slot_], st_), "cudaEventRecord");
      used_[slot_] = true;
      slot_ ^= 1;
      pos += n;
    }
    return ok_;
  }
  bool finish() { return ok_ && cuda_ok(cudaStreamSynchronize(st_), "upload"); }

 private:
  static constexpr size_t kChunk = 64ull << 20;
  cudaStream_t st_;
  void* stage_[2] = {nullptr, nullptr};
  cudaEvent_t done_[2] = {nullptr, nullptr};
  bool used_[2] = {false, false};
  int slot_ = 0;
  bool ok_ = false;
};
}  // namespace

// Maps the file, parses and validates the header and the tensor table, and
// copies out the child tables; sets D, rank, R, C, N.  No device work.
bool circuit_index_opaque::parse_file(const char* path, void* tinfo, std::vector<int>* parent,
                                      std::vector<int>* offsets, std::vector<int>* sizes) {
  TensorInfo* ti = static_cast<TensorInfo*>(tinfo);
  if (!path) { set_error("null path"); return false; }
  fd = open(path, O_RDONLY);
  if (fd < 0) { set_error(std::string("cannot open ") + path); return false; }
  struct stat sb;
  if (fstat(fd, &sb) < 0) { set_error("fstat failed"); return false; }
  map_size = (size_t)sb.st_size;
  if (map_size < 12) { set_error("file too small for a .circuit header"); return false; }
  map_ptr = mmap(nullptr, map_size, PROT_READ, MAP_SHARED, fd, 0);
  if (map_ptr == MAP_FAILED) { map_ptr = nullptr; set_error("mmap failed"); return false; }
  const char* base = static_cast<const char*>(map_ptr);
  if (std::memcmp(base, "CIRCUIT1", 8) != 0) { set_error("invalid magic bytes"); return false; }
  uint32_t header_len = 0;
  std::memcpy(&header_len, base + 8, 4);
  if ((size_t)header_len + 12 > map_size) { set_error("header length exceeds file size"); return false; }
  cb::json::Value meta;
  cb::json::Parser parser(base + 12, header_len);
  if (!parser.parse(&meta) || meta.kind != cb::json::Value::Object) { set_error("header is not valid JSON"); return false; }
  int64_t vals[5];
  const char* keys[5] = {"dim", "rank", "num_roots", "num_total_children", "N"};
  for (int i = 0; i < 5; ++i) {
    const cb::json::Value* v = meta.get(keys[i]);
    if (!v || !v->as_int64(&vals[i])) { set_error(std::string("header lacks integer ") + keys[i]); return false; }
  }
  if (vals[4] >= (int64_t)std::numeric_limits<int>::max()) { set_error("N must be < 2^31"); return false; }
  D = (int)vals[0]; rank = (int)vals[1]; R = (int)vals[2]; C = (int)vals[3]; N = (int)vals[4];
  if (!check_dims()) return false;
  const cb::json::Value* tm = meta.get("tensor_meta");
  if (!tm || tm->kind != cb::json::Value::Object) { set_error("header lacks tensor_meta"); return false; }
  const int64_t expect_numel[11] = {(int64_t)R * D, R, (int64_t)R * D * rank, (int64_t)C * rank, (int64_t)C * rank,
                                    C, C, C, C, (int64_t)N * D, N};
  const bool is_int[11] = {false, false, false, false, false, false, true, true, true, false, true};
  for (int t = 0; t < 11; ++t) {
    const cb::json::Value* e = tm->get(kTensorNames[t]);
    if (!e || e->kind != cb::json::Value::Object) { set_error(std::string("tensor_meta lacks ") + kTensorNames[t]); return false; }
    const cb::json::Value* dt = e->get("dtype");
    const cb::json::Value* sh = e->get("shape");
    const cb::json::Value* off = e->get("offset");
    const cb::json::Value* nb = e->get("nbytes");
    if (!dt || dt->kind != cb::json::Value::String || !sh || sh->kind != cb::json::Value::Array || !off ||
        !off->as_int64(&ti[t].offset) || !nb || !nb->as_int64(&ti[t].nbytes)) {
      set_error(std::string("bad tensor_meta entry for ") + kTensorNames[t]);
      return false;
    }
    ti[t].dtype = dt->str;
    int64_t numel = 1;
    for (const auto& d : sh->arr) {
      int64_t x;
      if (!d.as_int64(&x) || x < 0) { set_error(std::string("bad shape for ") + kTensorNames[t]); return false; }
      ti[t].shape.push_back(x);
      numel *= x;
    }
    if (ti[t].dtype != (is_int[t] ? "int32" : "float32")) { set_error(std::string("unexpected dtype for ") + kTensorNames[t]); return false; }
    if (numel != expect_numel[t] || ti[t].nbytes != numel * 4) {
      set_error(std::string("shape/nbytes mismatch for ") + kTensorNames[t]);
      return false;
    }
    if (ti[t].offset < 12 + (int64_t)header_len || ti[t].offset + ti[t].nbytes > (int64_t)map_size) {
      set_error(std::string("tensor data outside the file for ") + kTensorNames[t]);
      return false;
    }
  }
  // the file only guarantees 4-byte alignment of tensor data (offsets are 12
  // mod 64 with the reference writer), so the small int arrays are copied out
  parent->resize(C);
  offsets->resize(C);
  sizes->resize(C);
  std::memcpy(parent->data(), base + ti[6].offset, 4 * (size_t)C);
  std::memcpy(offsets->data(), base + ti[7].offset, 4 * (size_t)C);
  std::memcpy(sizes->data(), base + ti[8].offset, 4 * (size_t)C);
  return true;
}

void circuit_index_opaque::unmap_file() {
  if (map_ptr) munmap(map_ptr, map_size);
  map_ptr = nullptr;
  if (fd >= 0) close(fd);
  fd = -1;
}

bool circuit_index_opaque::load_file(const char* path, int dev) {
  device = dev;
  TensorInfo ti[11];
  std::vector<int> parent, offsets, sizes;
  if (!parse_file(path, ti, &parent, &offsets, &sizes)) return false;
  {  // validate the child tables on the host before any device work
    std::vector<int> p0, l0, r0;
    if (!build_host_tables(parent.data(), offsets.data(), sizes.data(), &p0, &l0, &r0)) return false;
  }
  const char* base = static_cast<const char*>(map_ptr);
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return false;
  if (!cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
  void* dptr[11];
  for (int t = 0; t < 11; ++t) {
    dptr[t] = dev_alloc((size_t)ti[t].nbytes, "cudaMalloc(index tensor)");
    if (!dptr[t]) return false;
  }
  {
    StagedUpload up(stream);
    for (int t = 0; t < 11; ++t)
      if (!up.put(dptr[t], base + ti[t].offset, (size_t)ti[t].nbytes)) return false;
    if (!up.finish()) return false;
  }
  view.root_centers = (const float*)dptr[0];
  view.root_radii = (const float*)dptr[1];
  view.bases = (const float*)dptr[2];
  view.child_l = (const float*)dptr[3];
  view.child_u = (const float*)dptr[4];
  view.child_radii = (const float*)dptr[5];
  view.child_parent = (const int*)dptr[6];
  view.leaf_offsets = (const int*)dptr[7];
  view.leaf_sizes = (const int*)dptr[8];
  view.leaf = (const float*)dptr[9];
  view.original_ids = (const int*)dptr[10];
  unmap_file();  // everything is on the device
  return finish_setup(parent.data(), offsets.data(), sizes.data());
}

// One rank's shard of a .circuit file: the parts of circuit_plan_shard_parts
// (children of each root in leaf order as atoms) that `rk` of `world` owns.
// Each part becomes a root of this index (the file root's centre, radius and
// basis; a contiguous range of its children); only those byte ranges of the
// file are read.  Original ids stay global.
bool circuit_index_opaque::load_shard_file(const char* path, int dev, int rk, int world, double max_imbalance) {
  device = dev;
  if (world < 1 || rk < 0 || rk >= world || !(max_imbalance >= 1.0)) {
    set_error("load_shard: need 0 <= rank < world and max_imbalance >= 1");
    return false;
  }
  TensorInfo ti[11];
  std::vector<int> parent, offsets, sizes;
  if (!parse_file(path, ti, &parent, &offsets, &sizes)) return false;
  std::vector<int> ptr, list, rows;
  if (!build_host_tables(parent.data(), offsets.data(), sizes.data(), &ptr, &list, &rows)) return false;
  const int R0 = R, C0 = C, N0 = N;
  (void)C0;
  (void)N0;
  // plan over the children of each root (CSR order = leaf order)
  std::vector<int64_t> atom_rows(list.size()), atom_ptr(R0 + 1);
  for (size_t i = 0; i < list.size(); ++i) atom_rows[i] = sizes[list[i]];
  for (int p = 0; p <= R0; ++p) atom_ptr[p] = ptr[p];
  int cap = R0 + 2 * world + 8, np = 0;
  std::vector<int> proot, prank;
  std::vector<int64_t> pa0, pa1;
  for (int attempt = 0; attempt < 2; ++attempt) {
    proot.assign(cap, 0); prank.assign(cap, 0); pa0.assign(cap, 0); pa1.assign(cap, 0);
    const int rc = circuit_plan_shard_parts(atom_rows.data(), atom_ptr.data(), R0, world, max_imbalance, proot.data(),
                                            pa0.data(), pa1.data(), prank.data(), cap, &np, nullptr);
    if (rc == CIRCUIT_OK) break;
    if (np <= cap || attempt == 1) return false;
    cap = np;
  }
  std::vector<int> own;
  for (int i = 0; i < np; ++i)
    if (prank[i] == rk) own.push_back(i);
  if (own.empty()) {
    set_error("load_shard: this rank owns no rows (more ranks than children)");
    return false;
  }
  const int Rs = (int)own.size();
  int cpr = 1;
  int64_t Ns = 0;
  for (int i : own) {
    cpr = std::max(cpr, (int)(pa1[i] - pa0[i]));
    for (int64_t a = pa0[i]; a < pa1[i]; ++a) Ns += atom_rows[a];
  }
  const int Cs = Rs * cpr;
  const char* base = static_cast<const char*>(map_ptr);
  const float* f_centers = reinterpret_cast<const float*>(base + ti[0].offset);
  const float* f_radii = reinterpret_cast<const float*>(base + ti[1].offset);
  const float* f_bases = reinterpret_cast<const float*>(base + ti[2].offset);
  const float* f_l = reinterpret_cast<const float*>(base + ti[3].offset);
  const float* f_u = reinterpret_cast<const float*>(base + ti[4].offset);
  const float* f_crad = reinterpret_cast<const float*>(base + ti[5].offset);
  // the shard's small arrays on the host (memcpy: file data is only 4-byte aligned)
  std::vector<float> centers((size_t)Rs * D), radii(Rs), bases((size_t)Rs * D * rank), cl((size_t)Cs * rank, 0.f),
      cu((size_t)Cs * rank, 0.f), crad(Cs, 0.f);
  std::vector<int> cpar(Cs), coff(Cs, 0), csz(Cs, 0);
  struct Span {
    int64_t src_row, dst_row, n;
  };
  std::vector<Span> spans;
  int64_t cur = 0;
  for (int j = 0; j < Rs; ++j) {
    const int i = own[j], p = proot[i];
    std::memcpy(&centers[(size_t)j * D], f_centers + (size_t)p * D, sizeof(float) * D);
    std::memcpy(&radii[j], f_radii + p, sizeof(float));
    std::memcpy(&bases[(size_t)j * D * rank], f_bases + (size_t)p * D * rank, sizeof(float) * (size_t)D * rank);
    for (int c = 0; c < cpr; ++c) cpar[(size_t)j * cpr + c] = j;
    for (int64_t a = pa0[i]; a < pa1[i]; ++a) {
      const int c = list[a], g = j * cpr + (int)(a - pa0[i]);
      std::memcpy(&cl[(size_t)g * rank], f_l + (size_t)c * rank, sizeof(float) * rank);
      std::memcpy(&cu[(size_t)g * rank], f_u + (size_t)c * rank, sizeof(float) * rank);
      std::memcpy(&crad[g], f_crad + c, sizeof(float));
      coff[g] = (int)cur;
      csz[g] = sizes[c];
      if (!spans.empty() && spans.back().src_row + spans.back().n == offsets[c] &&
          spans.back().dst_row + spans.back().n == cur)
        spans.back().n += sizes[c];  // adjacent in the file and in the shard: one copy
      else
        spans.push_back({offsets[c], cur, sizes[c]});
      cur += sizes[c];
    }
  }
  R = Rs;
  C = Cs;
  N = (int)Ns;
  if (!check_dims()) return false;
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return false;
  if (!cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
  const size_t sz[11] = {centers.size() * 4, radii.size() * 4, bases.size() * 4, cl.size() * 4, cu.size() * 4,
                         crad.size() * 4, cpar.size() * 4, coff.size() * 4, csz.size() * 4,
                         (size_t)Ns * D * 4, (size_t)Ns * 4};
  void* dptr[11];
  for (int t = 0; t < 11; ++t) {
    dptr[t] = dev_alloc(sz[t], "cudaMalloc(shard tensor)");
    if (!dptr[t]) return false;
  }
  {
    StagedUpload up(stream);
    const void* small[9] = {centers.data(), radii.data(), bases.data(), cl.data(), cu.data(),
                            crad.data(), cpar.data(), coff.data(), csz.data()};
    for (int t = 0; t < 9; ++t)
      if (!up.put(dptr[t], static_cast<const char*>(small[t]), sz[t])) return false;
    const char* leaf_src = base + ti[9].offset;
    const char* ids_src = base + ti[10].offset;
    const size_t rb = (size_t)D * 4;
    for (const Span& sp : spans) {
      if (!up.put((char*)dptr[9] + sp.dst_row * rb, leaf_src + sp.src_row * rb, (size_t)sp.n * rb) ||
          !up.put((char*)dptr[10] + sp.dst_row * 4, ids_src + sp.src_row * 4, (size_t)sp.n * 4))
        return false;
    }
    if (!up.finish()) return false;
  }
  view.root_centers = (const float*)dptr[0];
  view.root_radii = (const float*)dptr[1];
  view.bases = (const float*)dptr[2];
  view.child_l = (const float*)dptr[3];
  view.child_u = (const float*)dptr[4];
  view.child_radii = (const float*)dptr[5];
  view.child_parent = (const int*)dptr[6];
  view.leaf_offsets = (const int*)dptr[7];
  view.leaf_sizes = (const int*)dptr[8];
  view.leaf = (const float*)dptr[9];
  view.original_ids = (const int*)dptr[10];
  unmap_file();
  shard_rows_read = Ns;
  return finish_setup(cpar.data(), coff.data(), csz.data());
}

bool circuit_index_opaque::wrap_device(int dev, int dim, int rnk, int nr, int nc, int64_t n, const float* const* f,
                                       const int* const* ints) {
  device = dev;
  if (n <= 0 || n >= (int64_t)std::numeric_limits<int>::max()) { set_error("N must be in [1, 2^31)"); return false; }
  D = dim; rank = rnk; R = nr; C = nc; N = (int)n;
  if (!check_dims()) return false;
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return false;
  for (int i = 0; i < 7; ++i)
    if (!f[i]) { set_error("null float array"); return false; }
  for (int i = 0; i < 4; ++i)
    if (!ints[i]) { set_error("null int array"); return false; }
  if (((uintptr_t)f[6] & 15) || ((uintptr_t)f[0] & 15) || ((uintptr_t)f[2] & 15) || ((uintptr_t)f[3] & 15) ||
      ((uintptr_t)f[4] & 15)) {
    set_error("leaf_vectors, root_centers, bases and child intervals must be 16-byte aligned");
    return false;
  }
  if (!cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
  view.root_centers = f[0];
  view.root_radii = f[1];
  view.bases = f[2];
  view.child_l = f[3];
  view.child_u = f[4];
  view.child_radii = f[5];
  view.leaf = f[6];
  view.child_parent = ints[0];
  view.leaf_offsets = ints[1];
  view.leaf_sizes = ints[2];
  view.original_ids = ints[3];
  std::vector<int> parent(C), offsets(C), sizes(C);
  if (!cuda_ok(cudaMemcpy(parent.data(), ints[0], 4 * (size_t)C, cudaMemcpyDeviceToHost), "D2H child_parent_ids") ||
      !cuda_ok(cudaMemcpy(offsets.data(), ints[1], 4 * (size_t)C, cudaMemcpyDeviceToHost), "D2H leaf_offsets") ||
      !cuda_ok(cudaMemcpy(sizes.data(), ints[2], 4 * (size_t)C, cudaMemcpyDeviceToHost), "D2H leaf_sizes"))
    return false;
  return finish_setup(parent.data(), offsets.data(), sizes.data());
}

// ---------------------------------------------------------------- search
int circuit_index_opaque::search_async(const float* dq, int k, int64_t min_hier, float* dscores, int* dids,
                                       int64_t* drows, cudaStream_t st, cudaEvent_t e0, cudaEvent_t e1) {
  if (k < 1 || k > cb::KMAX) { set_error("k must be in [1, " + std::to_string(cb::KMAX) + "]"); return CIRCUIT_ERR_ARG; }
  if (!dq || !dscores) { set_error("null query or output pointer"); return CIRCUIT_ERR_ARG; }
  if ((uintptr_t)dq & 15) { set_error("query must be 16-byte aligned"); return CIRCUIT_ERR_ARG; }
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  const int hier = ((int64_t)N < min_hier) ? 0 : 1;
  cudaError_t e = cb::launch_search(view, ws, dq, k, hier, dscores, dids, (long long*)drows, st, e0, e1);
  last_stream = st;
  last_path = hier;
  last_k = k;
  if (e != cudaSuccess) { set_error(std::string("search launch: ") + cudaGetErrorString(e)); return CIRCUIT_ERR_CUDA; }
  return CIRCUIT_OK;
}

void circuit_index_opaque::fill_trace(const cb::SearchCtrl& c, circuit_trace_ex_t* t) const {
  std::memset(t, 0, sizeof(*t));
  t->path = last_path;
  t->vectors_total = N;
  t->total_children = C;
  t->device_error = c.error;
  if (last_path) {
    t->vectors_scored = (int64_t)(uint32_t)c.main_packed;
    t->surviving_roots = (int32_t)c.n_surv_roots;
    t->surviving_children = (int32_t)c.n_surv_children;
    t->best_root = c.best_root;
    t->seed_threshold = c.seed_T_key ? key_to_float(c.seed_T_key) : -std::numeric_limits<float>::infinity();
    t->seed_sample_rows = (int32_t)(uint32_t)c.seed_packed;
    t->rows_streamed = (int32_t)c.rows_streamed;
  } else {
    t->vectors_scored = N;
    t->rows_streamed = N;
    t->surviving_roots = R;
    t->surviving_children = -1;
    t->best_root = -1;
    t->seed_threshold = -std::numeric_limits<float>::infinity();
  }
}

float circuit_index_opaque::key_to_float(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

int circuit_index_opaque::search_blocking(const float* query, bool host_ptrs, int k, float* out_scores, int* out_ids,
                                          circuit_trace_t* trace) {
  const auto t0 = std::chrono::steady_clock::now();
  if (!query || !out_scores || !out_ids) { set_error("null query or output pointer"); return CIRCUIT_ERR_ARG; }
  if (k < 1 || k > cb::KMAX) { set_error("k must be in [1, " + std::to_string(cb::KMAX) + "]"); return CIRCUIT_ERR_ARG; }
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  // reference routing: flat scan for N <= 10000 (gpu_index.cpp:151)
  const int64_t min_hier = 10001;
  const int hier = ((int64_t)N < min_hier) ? 0 : 1;
  // Graph replay: one launch of [prologue kernel, search kernels]; the query
  // comes from the mapped staging block (host buffers) or from the caller's
  // device pointer named in its slots, and the final merge writes the results
  // and the control header straight to their destinations.  Device buffers
  // need device (or managed) memory of this device, a 16-byte aligned query
  // (float4 copy) and 4-byte aligned outputs; others take the direct path,
  // whose copies report a bad pointer as an error.
  const auto on_device = [&](const void* p, uintptr_t align) {
    cudaPointerAttributes a{};
    if (((uintptr_t)p & (align - 1)) != 0) return false;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) { cudaGetLastError(); return false; }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == device;
  };
  const bool graph_ok = host_ptrs || (on_device(query, 16) && on_device(out_scores, 4) && on_device(out_ids, 4));
  if (graph_ok) {
    const int key = (k << 2) | (host_ptrs ? 2 : 0) | hier;
    auto g = host_graphs.find(key);
    if (g == host_graphs.end() && ++host_graph_calls[key] >= 2) {
      cudaGraph_t graph = nullptr;
      cudaGraphExec_t exec = nullptr;
      bool built = false;
      if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        const bool ok = cb::launch_search(view, ws, dev_query, k, hier, host_ptrs ? map_scores : nullptr,
                                          host_ptrs ? map_ids : nullptr, nullptr, stream, nullptr, nullptr,
                                          host_ptrs ? &io_host : &io_device) == cudaSuccess;
        const bool ended = cudaStreamEndCapture(stream, &graph) == cudaSuccess;
        built = ok && ended && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
        if (graph) cudaGraphDestroy(graph);
      }
      cudaGetLastError();  // a failed capture falls back to direct launches, for good
      if (built) g = host_graphs.emplace(key, exec).first;
      else host_graph_calls[key] = std::numeric_limits<int>::min();
    }
    if (g != host_graphs.end()) {
      if (host_ptrs) {
        std::memcpy(h_query, query, sizeof(float) * D);
      } else {
        h_slots[0] = const_cast<float*>(query);
        h_slots[1] = out_scores;
        h_slots[2] = out_ids;
      }
      const uint32_t seq = ++call_counter;
      *h_seq = seq;
      if (!cuda_ok(cudaGraphLaunch(g->second, stream), "graph launch") || !wait_for_results(seq))
        return CIRCUIT_ERR_CUDA;
      last_stream = stream;
      last_path = hier;
      last_k = k;
      return finish_blocking(host_ptrs, k, out_scores, out_ids, trace, t0);
    }
  }
  if (host_ptrs) {
    std::memcpy(h_query, query, sizeof(float) * D);
    if (!cuda_ok(cudaMemcpyAsync(dev_query, h_query, sizeof(float) * D, cudaMemcpyHostToDevice, stream), "H2D query"))
      return CIRCUIT_ERR_CUDA;
  } else if (!cuda_ok(cudaMemcpyAsync(dev_query, query, sizeof(float) * D, cudaMemcpyDeviceToDevice, stream), "D2D query")) {
    return CIRCUIT_ERR_CUDA;
  }
  int rc = search_async(dev_query, k, min_hier, dev_scores, dev_ids, nullptr, stream, nullptr, nullptr);
  if (rc != CIRCUIT_OK) return rc;
  const cudaMemcpyKind kind = host_ptrs ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  float* sdst = host_ptrs ? h_scores : out_scores;
  int* idst = host_ptrs ? h_ids : out_ids;
  if (!cuda_ok(cudaMemcpyAsync(sdst, dev_scores, sizeof(float) * k, kind, stream), "copy scores") ||
      !cuda_ok(cudaMemcpyAsync(idst, dev_ids, sizeof(int) * k, kind, stream), "copy ids") ||
      !cuda_ok(cudaMemcpyAsync(h_ctrl, ws.ctrl, cb::CTRL_RESET_BYTES, cudaMemcpyDeviceToHost, stream), "copy ctrl") ||
      !cuda_ok(cudaStreamSynchronize(stream), "search sync"))
    return CIRCUIT_ERR_CUDA;
  return finish_blocking(host_ptrs, k, out_scores, out_ids, trace, t0);
}

// Waits for a graph-replayed blocking search: spins on the completion word the
// final merge writes into the mapped block (its results are out when it appears),
// checking the stream's status every few dozen polls; after kSpinLimitUs it falls
// back to cudaStreamSynchronize, so a long scan does not hold a core for its
// whole duration.  A stream that ends without the word (an error) is synchronised
// to report it.
bool circuit_index_opaque::wait_for_results(uint32_t seq) {
  constexpr double kSpinLimitUs = 200.0;
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t polls = 1;; ++polls) {
    if (*h_done == seq) return true;
    if ((polls & 63) == 0) {
      const cudaError_t q = cudaStreamQuery(stream);
      if (q != cudaErrorNotReady) {
        if (q != cudaSuccess) return cuda_ok(q, "search");
        if (*h_done == seq) return true;
        return cuda_ok(cudaStreamSynchronize(stream), "search sync");
      }
      if (std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count() > kSpinLimitUs)
        return cuda_ok(cudaStreamSynchronize(stream), "search sync");
    }
  }
}

// End of a blocking search once its stream has synchronised: host results leave
// the staging block, a device-side timeout becomes an error, the trace is filled.
int circuit_index_opaque::finish_blocking(bool host_ptrs, int k, float* out_scores, int* out_ids,
                                          circuit_trace_t* trace, std::chrono::steady_clock::time_point t0) {
  if (host_ptrs) {
    std::memcpy(out_scores, h_scores, sizeof(float) * k);
    std::memcpy(out_ids, h_ids, sizeof(int) * k);
  }
  have_host_ctrl = true;
  if (h_ctrl->error) {
    set_error("device-side wait timed out (error bits " + std::to_string(h_ctrl->error) + ")");
    return CIRCUIT_ERR_TIMEOUT;
  }
  if (trace) {
    circuit_trace_ex_t tx;
    fill_trace(*h_ctrl, &tx);
    trace->latency_us = (float)std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
    trace->vectors_scored = (int)std::min<int64_t>(tx.vectors_scored, std::numeric_limits<int>::max());
  }
  return CIRCUIT_OK;
}

// ---------------------------------------------------------------- batched search
int circuit_index_opaque::ensure_batch(int B) {
  if (!batch_ready) {
    if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
    bw.sms = cb::sm_count(device);
    unsigned int* d_key = nullptr;
    if (!cuda_ok(cudaMalloc(&d_key, sizeof(unsigned int)), "cudaMalloc(xmax)")) return CIRCUIT_ERR_CUDA;
    owned.push_back(d_key);
    int* d_err = nullptr;
    if (!cuda_ok(cudaMalloc(&d_err, sizeof(int)), "cudaMalloc(batch err)")) return CIRCUIT_ERR_CUDA;
    owned.push_back(d_err);
    unsigned int key = 0;
    if (!cuda_ok(cb::launch_max_row_norm(view.leaf, N, D, d_key, bw.sms, stream), "max row norm") ||
        !cuda_ok(cudaMemcpyAsync(&key, d_key, sizeof(key), cudaMemcpyDeviceToHost, stream), "D2H xmax") ||
        !cuda_ok(cudaMemsetAsync(d_err, 0, sizeof(int), stream), "memset err") ||
        !cuda_ok(cudaStreamSynchronize(stream), "xmax sync"))
      return CIRCUIT_ERR_CUDA;
    float mx2;
    std::memcpy(&mx2, &key, 4);
    bw.xmax = std::sqrt(mx2) * 1.0001f + 1e-30f;
    bw.err = d_err;
    if (!cb::make_leaf_tensor_map(view.leaf, N, D, bw.tmap)) {
      set_error("cuTensorMapEncodeTiled failed for leaf_vectors");
      return CIRCUIT_ERR_CUDA;
    }
    bw.sample_rows = cb::sample_rows_for(N);
    if (bw.sample_rows > 0 && !cb::make_sample_tensor_map(view.leaf, N, D, bw.smap)) {
      set_error("cuTensorMapEncodeTiled failed for the sampled leaf rows");
      return CIRCUIT_ERR_CUDA;
    }
    batch_ready = true;
  }
  if (B > bw.capacity) {
    if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
    cudaDeviceSynchronize();
    for (void* p : batch_owned) cudaFree(p);
    batch_owned.clear();
    const int cap_B = ((B + 1023) / 1024) * 1024;
    auto grab = [&](size_t bytes, const char* what) -> void* {
      void* p = nullptr;
      if (!cuda_ok(cudaMalloc(&p, bytes), what)) return nullptr;
      batch_owned.push_back(p);
      return p;
    };
    bw.theta = (uint32_t*)grab(sizeof(uint32_t) * cap_B, "cudaMalloc(theta)");
    bw.slots = (uint32_t*)grab(sizeof(uint32_t) * (size_t)cap_B * cb::BATCH_MAX_SLOTS, "cudaMalloc(slots)");
    bw.cand_count = (int*)grab(sizeof(int) * cap_B, "cudaMalloc(cand_count)");
    // the candidate pool holds at least 4,096 queries x 16,384 entries, so a
    // smaller batch gets up to BATCH_CAND_MAX entries per query
    bw.cand_entries = (int64_t)std::max(cap_B, 4096) * bw.cap;
    bw.cand = (unsigned long long*)grab(sizeof(unsigned long long) * (size_t)bw.cand_entries, "cudaMalloc(cand)");
    bw.overflow = (int*)grab(sizeof(int), "cudaMalloc(overflow)");
    bw.unit_counter = (int*)grab(2 * sizeof(int), "cudaMalloc(unit counters)");
    bw.queries = (float*)grab(sizeof(float) * (size_t)cap_B * D, "cudaMalloc(batch queries)");
    bw.qband = (float*)grab(sizeof(float) * (size_t)cap_B, "cudaMalloc(batch bands)");
    // staging for the host-buffer call: any k up to KMAX
    bw.out_scores = (float*)grab(sizeof(float) * (size_t)cap_B * cb::KMAX, "cudaMalloc(batch scores)");
    bw.out_ids = (int*)grab(sizeof(int) * (size_t)cap_B * cb::KMAX, "cudaMalloc(batch ids)");
    if (!bw.theta || !bw.slots || !bw.unit_counter || !bw.cand_count || !bw.cand || !bw.overflow || !bw.queries || !bw.qband || !bw.out_scores ||
        !bw.out_ids) {
      bw.capacity = 0;
      return CIRCUIT_ERR_CUDA;
    }
    bw.capacity = cap_B;
  }
  return CIRCUIT_OK;
}

int circuit_index_opaque::search_batch_async(const float* dq, int B, int k, float* dscores, int* dids,
                                             cudaStream_t st, cudaEvent_t ev0, cudaEvent_t ev1) {
  if (B < 1) { set_error("num_queries must be >= 1"); return CIRCUIT_ERR_ARG; }
  if (k < 1 || k > cb::KMAX) {
    set_error("batched search supports 1 <= k <= " + std::to_string(cb::KMAX));
    return CIRCUIT_ERR_UNSUPPORTED;
  }
  if (D > cb::BATCH_MAX_DIM || D % 4 != 0) {
    set_error("batched search supports dim <= " + std::to_string(cb::BATCH_MAX_DIM) + " with dim % 4 == 0");
    return CIRCUIT_ERR_UNSUPPORTED;
  }
  if (!dq || !dscores || !dids || ((uintptr_t)dq & 15)) {
    set_error("null or misaligned batch pointer");
    return CIRCUIT_ERR_ARG;
  }
  int rc = ensure_batch(B);
  if (rc != CIRCUIT_OK) return rc;
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  cudaError_t e = cb::launch_batch_search(view, bw, dq, B, k, dscores, dids, st, ev0, ev1);
  last_stream = st;
  if (e != cudaSuccess) { set_error(std::string("batch launch: ") + cudaGetErrorString(e)); return CIRCUIT_ERR_CUDA; }
  return CIRCUIT_OK;
}

int circuit_index_opaque::batch_status(cudaStream_t st, int* overflow) {
  *overflow = 0;
  if (!batch_ready || !bw.overflow) return CIRCUIT_OK;
  int err = 0;
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
      !cuda_ok(cudaMemcpyAsync(overflow, bw.overflow, sizeof(int), cudaMemcpyDeviceToHost, st), "D2H overflow") ||
      !cuda_ok(cudaMemcpyAsync(&err, bw.err, sizeof(int), cudaMemcpyDeviceToHost, st), "D2H batch error bits") ||
      !cuda_ok(cudaStreamSynchronize(st), "batch sync"))
    return CIRCUIT_ERR_CUDA;
  if (err) {
    set_error("batched search: a device-side wait timed out (error bits " + std::to_string(err) +
              "); the batch's results are incomplete");
    return CIRCUIT_ERR_TIMEOUT;
  }
  return CIRCUIT_OK;
}

// ---------------------------------------------------------------- C ABI
extern "C" {

int circuit_search_batch_async(circuit_index_t index, const float* dev_queries, int num_queries, int k,
                               float* dev_out_scores, int* dev_out_ids, void* stream, void* ev_scan_begin,
                               void* ev_scan_end) {
  if (!index) return CIRCUIT_ERR_NULL;
  return index->search_batch_async(dev_queries, num_queries, k, dev_out_scores, dev_out_ids, (cudaStream_t)stream,
                                   (cudaEvent_t)ev_scan_begin, (cudaEvent_t)ev_scan_end);
}

int circuit_batch_overflow(circuit_index_t index, int* out_count) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!out_count) { set_error("null out_count"); return CIRCUIT_ERR_ARG; }
  return index->batch_status(index->last_stream, out_count);
}

int circuit_search_batch(circuit_index_t index, const float* host_queries, int num_queries, int k,
                         float* host_scores, int* host_ids) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!host_queries || !host_scores || !host_ids || num_queries < 1) {
    set_error("null batch pointer or num_queries < 1");
    return CIRCUIT_ERR_ARG;
  }
  int rc = index->ensure_batch(num_queries);
  if (rc != CIRCUIT_OK) return rc;
  const size_t qbytes = sizeof(float) * (size_t)num_queries * index->D;
  cudaStream_t st = index->stream;
  if (!cuda_ok(cudaMemcpyAsync(index->bw.queries, host_queries, qbytes, cudaMemcpyHostToDevice, st), "H2D queries"))
    return CIRCUIT_ERR_CUDA;
  rc = index->search_batch_async(index->bw.queries, num_queries, k, index->bw.out_scores, index->bw.out_ids, st);
  if (rc != CIRCUIT_OK) return rc;
  const size_t ob = (size_t)num_queries * k;
  if (!cuda_ok(cudaMemcpyAsync(host_scores, index->bw.out_scores, sizeof(float) * ob, cudaMemcpyDeviceToHost, st),
               "D2H scores") ||
      !cuda_ok(cudaMemcpyAsync(host_ids, index->bw.out_ids, sizeof(int) * ob, cudaMemcpyDeviceToHost, st), "D2H ids"))
    return CIRCUIT_ERR_CUDA;
  int over = 0;
  if ((rc = index->batch_status(st, &over)) != CIRCUIT_OK) return rc;
  // a query whose candidate list overflowed is answered by the single-query search
  for (int q = 0; q < num_queries; ++q) {
    if (host_ids[(size_t)q * k] != -2) continue;
    rc = index->search_blocking(host_queries + (size_t)q * index->D, true, k, host_scores + (size_t)q * k,
                                host_ids + (size_t)q * k, nullptr);
    if (rc != CIRCUIT_OK) return rc;
  }
  return CIRCUIT_OK;
}


int circuit_search_batch_device(circuit_index_t index, const float* dev_queries, int num_queries, int k,
                                float* dev_out_scores, int* dev_out_ids) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!dev_queries || !dev_out_scores || !dev_out_ids || num_queries < 1) {
    set_error("null batch pointer or num_queries < 1");
    return CIRCUIT_ERR_ARG;
  }
  cudaStream_t st = index->stream;
  int rc = index->search_batch_async(dev_queries, num_queries, k, dev_out_scores, dev_out_ids, st);
  if (rc != CIRCUIT_OK) return rc;
  int over = 0;
  if ((rc = index->batch_status(st, &over)) != CIRCUIT_OK) return rc;
  if (over == 0) return CIRCUIT_OK;
  // the first id of each row marks an overflowed query (-2): answer those rows
  // in place with the single-query search, on the same stream
  std::vector<int> first((size_t)num_queries);
  if (!cuda_ok(cudaMemcpy2DAsync(first.data(), sizeof(int), dev_out_ids, sizeof(int) * (size_t)k, sizeof(int),
                                 (size_t)num_queries, cudaMemcpyDeviceToHost, st),
               "D2H first ids") ||
      !cuda_ok(cudaStreamSynchronize(st), "batch sync"))
    return CIRCUIT_ERR_CUDA;
  const int64_t min_hier = 10001;  // the blocking single-query routing
  for (int q = 0; q < num_queries; ++q) {
    if (first[(size_t)q] != -2) continue;
    rc = index->search_async(dev_queries + (size_t)q * index->D, k, min_hier, dev_out_scores + (size_t)q * k,
                             dev_out_ids + (size_t)q * k, nullptr, st, nullptr, nullptr);
    if (rc != CIRCUIT_OK) return rc;
  }
  return cuda_ok(cudaStreamSynchronize(st), "fallback sync") ? CIRCUIT_OK : CIRCUIT_ERR_CUDA;
}

int circuit_selftest_batch_wait_timeout(circuit_index_t index, int* out_error_bits) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!out_error_bits) { set_error("null out_error_bits"); return CIRCUIT_ERR_ARG; }
  int rc = index->ensure_batch(1);
  if (rc != CIRCUIT_OK) return rc;
  cudaStream_t st = index->stream;
  if (!cuda_ok(cudaSetDevice(index->device), "cudaSetDevice") ||
      !cuda_ok(cb::launch_selftest_wait(index->bw.err, st), "selftest launch") ||
      !cuda_ok(cudaMemcpyAsync(out_error_bits, index->bw.err, sizeof(int), cudaMemcpyDeviceToHost, st), "D2H bits") ||
      !cuda_ok(cudaStreamSynchronize(st), "selftest sync"))
    return CIRCUIT_ERR_CUDA;
  index->last_stream = st;
  return CIRCUIT_OK;
}

const char* circuit_last_error(void) { return cb::get_error(); }
int circuit_abi_version(void) { return CIRCUIT_ABI_VERSION; }

circuit_index_t circuit_load_index(const char* filepath, int device_id) {
  auto* idx = new (std::nothrow) circuit_index_opaque();
  if (!idx) { set_error("out of host memory"); return nullptr; }
  if (!idx->load_file(filepath, device_id)) {
    idx->release();
    delete idx;
    return nullptr;
  }
  return idx;
}

circuit_index_t circuit_load_shard(const char* filepath, int rank, int world, int device_id, double max_imbalance) {
  auto* idx = new (std::nothrow) circuit_index_opaque();
  if (!idx) { set_error("out of host memory"); return nullptr; }
  if (!idx->load_shard_file(filepath, device_id, rank, world, max_imbalance)) {
    idx->release();
    delete idx;
    return nullptr;
  }
  return idx;
}

circuit_index_t circuit_index_from_device(int device_id, int dim, int rank, int num_roots, int num_total_children,
                                          int64_t n, const float* root_centers, const float* root_radii,
                                          const float* bases, const float* child_intervals_l,
                                          const float* child_intervals_u, const float* child_radii,
                                          const int* child_parent_ids, const int* leaf_offsets,
                                          const int* leaf_sizes, const float* leaf_vectors,
                                          const int* original_ids) {
  auto* idx = new (std::nothrow) circuit_index_opaque();
  if (!idx) { set_error("out of host memory"); return nullptr; }
  const float* f[7] = {root_centers, root_radii, bases, child_intervals_l, child_intervals_u, child_radii, leaf_vectors};
  const int* ints[4] = {child_parent_ids, leaf_offsets, leaf_sizes, original_ids};
  if (!idx->wrap_device(device_id, dim, rank, num_roots, num_total_children, n, f, ints)) {
    idx->release();
    delete idx;
    return nullptr;
  }
  return idx;
}

int circuit_index_info(circuit_index_t index, int64_t* info) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!info) { set_error("null info"); return CIRCUIT_ERR_ARG; }
  info[0] = index->D; info[1] = index->rank; info[2] = index->R; info[3] = index->C;
  info[4] = index->N; info[5] = index->device; info[6] = index->ws.scan_grid; info[7] = cb::KMAX;
  return CIRCUIT_OK;
}

int circuit_search(circuit_index_t index, const float* query, int k, float* out_scores, int* out_ids,
                   circuit_trace_t* trace) {
  if (!index) return CIRCUIT_ERR_NULL;
  return index->search_blocking(query, true, k, out_scores, out_ids, trace);
}

int circuit_search_device(circuit_index_t index, const float* dev_query, int k, float* dev_out_scores,
                          int* dev_out_ids, circuit_trace_t* trace) {
  if (!index) return CIRCUIT_ERR_NULL;
  return index->search_blocking(dev_query, false, k, dev_out_scores, dev_out_ids, trace);
}

int circuit_search_seed_async(circuit_index_t index, const float* dev_query, int k, float* dev_threshold_out,
                              void* stream) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (k < 1 || k > cb::KMAX) { set_error("k must be in [1, " + std::to_string(cb::KMAX) + "]"); return CIRCUIT_ERR_ARG; }
  if (!dev_query || !dev_threshold_out || ((uintptr_t)dev_query & 15)) {
    set_error("null or misaligned pointer");
    return CIRCUIT_ERR_ARG;
  }
  if (!cuda_ok(cudaSetDevice(index->device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  index->have_host_ctrl = false;
  cudaError_t e = cb::launch_search_seed(index->view, index->ws, dev_query, k, dev_threshold_out, st);
  index->last_stream = st;
  index->last_path = 1;
  index->last_k = k;
  if (e != cudaSuccess) { set_error(std::string("seed launch: ") + cudaGetErrorString(e)); return CIRCUIT_ERR_CUDA; }
  return CIRCUIT_OK;
}

int circuit_search_finish_async(circuit_index_t index, const float* dev_query, int k, const float* dev_threshold_in,
                                float* dev_out_scores, int* dev_out_ids, int64_t* dev_out_rows, void* stream,
                                void* ev_scan_begin, void* ev_scan_end) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (k < 1 || k > cb::KMAX) { set_error("k must be in [1, " + std::to_string(cb::KMAX) + "]"); return CIRCUIT_ERR_ARG; }
  if (!dev_query || !dev_out_scores || ((uintptr_t)dev_query & 15)) {
    set_error("null or misaligned pointer");
    return CIRCUIT_ERR_ARG;
  }
  if (k != index->last_k || index->last_path != 1) {
    set_error("circuit_search_finish_async must follow circuit_search_seed_async with the same k");
    return CIRCUIT_ERR_ARG;
  }
  if (!cuda_ok(cudaSetDevice(index->device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cb::launch_search_finish(index->view, index->ws, dev_query, k, dev_threshold_in, dev_out_scores,
                                           dev_out_ids, (long long*)dev_out_rows, st, (cudaEvent_t)ev_scan_begin,
                                           (cudaEvent_t)ev_scan_end);
  index->last_stream = st;
  if (e != cudaSuccess) { set_error(std::string("finish launch: ") + cudaGetErrorString(e)); return CIRCUIT_ERR_CUDA; }
  return CIRCUIT_OK;
}

int circuit_search_finish_shared_async(circuit_index_t index, const float* dev_query, int k,
                                       const float* dev_threshold_in, unsigned long long* dev_shared_word,
                                       unsigned long long* const* dev_peer_words, int num_peers, uint32_t query_tag,
                                       float* dev_out_scores, int* dev_out_ids, int64_t* dev_out_rows, void* stream,
                                       void* ev_scan_begin, void* ev_scan_end) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (k < 1 || k > cb::KMAX) { set_error("k must be in [1, " + std::to_string(cb::KMAX) + "]"); return CIRCUIT_ERR_ARG; }
  if (!dev_query || !dev_out_scores || ((uintptr_t)dev_query & 15)) {
    set_error("null or misaligned pointer");
    return CIRCUIT_ERR_ARG;
  }
  if (!dev_shared_word || ((uintptr_t)dev_shared_word & 7) || num_peers < 0 || num_peers > 1024 ||
      (num_peers > 0 && (!dev_peer_words || ((uintptr_t)dev_peer_words & 7)))) {
    set_error("shared threshold: null or misaligned word, or a bad peer list");
    return CIRCUIT_ERR_ARG;
  }
  if (k != index->last_k || index->last_path != 1) {
    set_error("circuit_search_finish_shared_async must follow circuit_search_seed_async with the same k");
    return CIRCUIT_ERR_ARG;
  }
  if (!cuda_ok(cudaSetDevice(index->device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  const cb::SharedThreshold sh{dev_shared_word, dev_peer_words, num_peers, query_tag};
  cudaError_t e = cb::launch_search_finish(index->view, index->ws, dev_query, k, dev_threshold_in, dev_out_scores,
                                           dev_out_ids, (long long*)dev_out_rows, st, (cudaEvent_t)ev_scan_begin,
                                           (cudaEvent_t)ev_scan_end, nullptr, &sh);
  index->last_stream = st;
  if (e != cudaSuccess) { set_error(std::string("finish launch: ") + cudaGetErrorString(e)); return CIRCUIT_ERR_CUDA; }
  return CIRCUIT_OK;
}

int circuit_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  if (!dev_ptr || !handle_out) { set_error("null pointer"); return CIRCUIT_ERR_ARG; }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  // the allocation holding dev_ptr (an IPC handle names an allocation's start)
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  if (!range_fn) {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fp, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !fp) {
      set_error("circuit_ipc_export: cuMemGetAddressRange unavailable");
      return CIRCUIT_ERR_CUDA;
    }
    range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fp);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS) {
    set_error("circuit_ipc_export: not device memory");
    return CIRCUIT_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  if (!cuda_ok(cudaIpcGetMemHandle(&h, (void*)base), "cudaIpcGetMemHandle")) return CIRCUIT_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  if (offset_out) *offset_out = (int64_t)((CUdeviceptr)dev_ptr - base);
  return CIRCUIT_OK;
}

int circuit_ipc_import(const void* handle, int device_id, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) { set_error("null pointer"); return CIRCUIT_ERR_ARG; }
  if (!cuda_ok(cudaSetDevice(device_id), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (!cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
    return CIRCUIT_ERR_CUDA;
  *dev_ptr_out = p;
  return CIRCUIT_OK;
}

int circuit_ipc_close(void* dev_ptr) {
  if (!dev_ptr) { set_error("null pointer"); return CIRCUIT_ERR_ARG; }
  return cuda_ok(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle") ? CIRCUIT_OK : CIRCUIT_ERR_CUDA;
}

int circuit_search_async(circuit_index_t index, const float* dev_query, int k, int64_t min_hierarchy_n,
                         float* dev_out_scores, int* dev_out_ids, int64_t* dev_out_rows, void* stream,
                         void* ev_scan_begin, void* ev_scan_end) {
  if (!index) return CIRCUIT_ERR_NULL;
  cudaStream_t st = (cudaStream_t)stream;  // NULL = the legacy default stream, as everywhere in CUDA
  index->have_host_ctrl = false;
  return index->search_async(dev_query, k, min_hierarchy_n, dev_out_scores, dev_out_ids, dev_out_rows, st,
                             (cudaEvent_t)ev_scan_begin, (cudaEvent_t)ev_scan_end);
}

int circuit_last_trace(circuit_index_t index, circuit_trace_ex_t* out) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!out) { set_error("null trace"); return CIRCUIT_ERR_ARG; }
  if (!cuda_ok(cudaSetDevice(index->device), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  if (!index->have_host_ctrl) {
    cudaStream_t st = index->last_stream;
    if (!cuda_ok(cudaMemcpyAsync(index->h_ctrl, index->ws.ctrl, cb::CTRL_RESET_BYTES, cudaMemcpyDeviceToHost, st),
                 "copy ctrl") ||
        !cuda_ok(cudaStreamSynchronize(st), "trace sync"))
      return CIRCUIT_ERR_CUDA;
    index->have_host_ctrl = true;
  }
  index->fill_trace(*index->h_ctrl, out);
  if (index->h_ctrl->error) {
    set_error("device-side wait timed out (error bits " + std::to_string(index->h_ctrl->error) + ")");
    return CIRCUIT_ERR_TIMEOUT;
  }
  return CIRCUIT_OK;
}

int circuit_trace_snapshot_async(circuit_index_t index, void* dst, void* stream) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!dst) { set_error("null snapshot buffer"); return CIRCUIT_ERR_ARG; }
  static_assert(cb::CTRL_RESET_BYTES == CIRCUIT_TRACE_SNAPSHOT_BYTES, "snapshot size");
  cudaStream_t st = (cudaStream_t)stream;
  if (!cuda_ok(cudaSetDevice(index->device), "cudaSetDevice") ||
      !cuda_ok(cudaMemcpyAsync(dst, index->ws.ctrl, cb::CTRL_RESET_BYTES, cudaMemcpyDefault, st),
               "trace snapshot"))
    return CIRCUIT_ERR_CUDA;
  return CIRCUIT_OK;
}

int circuit_trace_decode(circuit_index_t index, const void* snapshot, int path, circuit_trace_ex_t* out) {
  if (!index) return CIRCUIT_ERR_NULL;
  if (!snapshot || !out) { set_error("null snapshot or trace"); return CIRCUIT_ERR_ARG; }
  cb::SearchCtrl c;
  std::memset(&c, 0, sizeof(c));
  std::memcpy(&c, snapshot, cb::CTRL_RESET_BYTES);
  const int saved = index->last_path;
  index->last_path = path ? 1 : 0;
  index->fill_trace(c, out);
  index->last_path = saved;
  if (c.error) {
    set_error("device-side wait timed out (error bits " + std::to_string(c.error) + ")");
    return CIRCUIT_ERR_TIMEOUT;
  }
  return CIRCUIT_OK;
}

void circuit_destroy_index(circuit_index_t index) {
  if (!index) return;
  index->release();
  delete index;
}

}  // extern "C"
