// Batched exact top-k search on the B200 tensor cores.
//
// k_batch_scan  one persistent CTA per SM.  A work unit is (query tile of 128
//               queries, slice of 8,192 leaf rows); units are dealt round-robin
//               in slice-major order so the CTAs in flight read the same slices
//               and the leaf rows come from HBM once, then from L2.
//               - 4 epilogue warps write the 128 query rows (fp32 = tf32 bits)
//                 into TMEM columns [0, D) as the MMA A operand;
//               - a TMA warp streams 64-row leaf tiles (fp32, 128-byte swizzle,
//                 boxes of 32 columns) through a shared-memory ring (2 stages
//                 at D = 384, up to 4 for smaller D);
//               - an MMA warp issues tcgen05.mma kind::tf32 (M=128 queries,
//                 N=64 rows, K=8) into one of two TMEM accumulators
//                 (columns 384-447 / 448-511) and commits to mbarriers;
//               - each epilogue thread owns one query: it reads its 64 scores
//                 with tcgen05.ld, keeps its k best tf32 scores in registers,
//                 and appends every row whose tf32 score is within `band` of
//                 the running k-th best (max of its own and the query's global
//                 atomicMax threshold) to the query's candidate list, with
//                 its tf32 score.
// k_batch_rescore  one CTA per query: drops the candidates below the final
//               threshold minus the band, scores the rest exactly in fp32 (the
//               same arithmetic as the single-query scan, so both paths return
//               identical scores), radix select, original ids.
//
// Exactness: with eps >= |tf32 score - fp32 score| for every row (bound:
// (2^-9 + 2^-20 + 2D 2^-23 + gamma_D) ||q|| max||x||, tf32 truncation of both
// operands plus fp32 accumulation), any row in the fp32 top-k has tf32 score
// >= s_k - eps, and any running k-th best tf32 score is <= s_k + eps, so
// band = 2 eps never drops a top-k row.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <string>

#include "common.cuh"
#include "engine.h"
#include "tcgen05.cuh"
#include "topk.cuh"

namespace cb {

constexpr int BQ = 128;              // queries per tile (UMMA M)
constexpr int BN = 64;               // leaf rows per tile (UMMA N)
constexpr int BATCH_THREADS = 192;   // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int BATCH_MAX_STAGES = 4;
constexpr int SLICE_ROWS = 8192;     // rows per work unit
constexpr int BOX_BYTES = BN * 128;  // one 64 x 32-float box, 128-byte rows
constexpr uint32_t ACC_COL = 384;    // accumulators at columns 384 and 448

struct BatchScanParams {
  const float* Q;        // [B, D]
  int B, D, N, k;
  int kb;                // boxes of 32 columns = ceil(D / 32)
  int stages;            // shared-memory ring depth (<= BATCH_MAX_STAGES)
  int QT, units;         // query tiles, work units
  float band_scale;      // band = band_scale * ||q||
  uint32_t* theta;       // [B] order-preserving keys of the running k-th best
  int* cand_count;       // [B]
  unsigned long long* cand;  // [B * cap]: tf32 score key << 32 | leaf row
  int cap;
  int* err;
};

template <int KB>
__global__ void __launch_bounds__(BATCH_THREADS, 1)
    k_batch_scan(const __grid_constant__ CUtensorMap xmap, BatchScanParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t full[BATCH_MAX_STAGES], empty[BATCH_MAX_STAGES], acc_full[2], acc_empty[2], a_full, a_empty;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stage_bytes = P.kb * BOX_BYTES;
  const int S = P.stages;
  float* stash = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes);  // [BN][BQ] scores

  if (warp == 5) tc::tmem_alloc(&tmem_base, 512);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], BQ);
    }
    mbar_init(&a_full, BQ);
    mbar_init(&a_empty, 1);
    fence_mbar_init();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 4) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < P.units && ok; u += gridDim.x) {
        const int slice = u / P.QT;
        const int r0 = slice * SLICE_ROWS, r1 = min(P.N, r0 + SLICE_ROWS);
        for (int row = r0; row < r1; row += BN, ++it) {
          const int s = it % S, f = it / S;
          if (f > 0 && !mbar_wait(&empty[s], (f - 1) & 1, P.err, ERR_TIMEOUT_EMPTY)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], (uint32_t)stage_bytes);
          unsigned char* dst = smem + (size_t)s * stage_bytes;
          for (int j = 0; j < P.kb; ++j) tc::tma_load_2d(dst + j * BOX_BYTES, &xmap, 32 * j, row, &full[s]);
        }
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_tf32(BQ, BN);
      const uint32_t sbase = smem_u32(smem);
      int it = 0, ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < P.units && ok; u += gridDim.x, ++ui) {
        if (!mbar_wait(&a_full, ui & 1, P.err, ERR_TIMEOUT_FULL)) break;
        tc::fence_after();
        const int slice = u / P.QT;
        const int r0 = slice * SLICE_ROWS, r1 = min(P.N, r0 + SLICE_ROWS);
        for (int row = r0; row < r1; row += BN, ++it) {
          const int s = it % S, f = it / S;
          const int b = it & 1, fb = it >> 1;
          if (!mbar_wait(&full[s], f & 1, P.err, ERR_TIMEOUT_FULL)) { ok = false; break; }
          if (fb > 0 && !mbar_wait(&acc_empty[b], (fb - 1) & 1, P.err, ERR_TIMEOUT_EMPTY)) { ok = false; break; }
          tc::fence_after();
          const uint32_t acc = tmem + ACC_COL + (uint32_t)(b * BN);
          const uint32_t stage = sbase + (uint32_t)(s * stage_bytes);
          for (int j = 0; j < P.kb; ++j) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              tc::mma_tf32_ts(acc, tmem + (uint32_t)(32 * j + 8 * kk),
                              tc::sdesc_k_sw128(stage + (uint32_t)(j * BOX_BYTES + kk * 32)), idesc,
                              (j | kk) ? 1u : 0u);
            }
          }
          tc::commit(&empty[s]);
          tc::commit(&acc_full[b]);
        }
        tc::commit(&a_empty);  // A may be overwritten once every MMA of this unit is done
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue (one query per thread)
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    int it = 0, ui = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < P.units && ok; u += gridDim.x, ++ui) {
      const int qt = u % P.QT, slice = u / P.QT;
      const int q = qt * BQ + 32 * warp + lane;
      const bool qv = q < P.B;
      if (ui > 0 && !mbar_wait(&a_empty, (ui - 1) & 1, P.err, ERR_TIMEOUT_EMPTY)) break;
      tc::fence_after();
      // query row -> TMEM lane, columns [0, 32 kb) (zeros past D and for padding queries)
      float qn2 = 0.f;
      const float* qrow = P.Q + (size_t)(qv ? q : 0) * P.D;
      for (int j = 0; j < P.kb; ++j) {
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = 32 * j + i;
          const float x = (qv && c < P.D) ? __ldg(qrow + c) : 0.f;
          qn2 = fmaf(x, x, qn2);
          v[i] = __float_as_uint(x);
        }
        tc::st_32x32b_x32(tmem + lane_base + (uint32_t)(32 * j), v);
      }
      tc::wait_st();
      tc::fence_before();
      mbar_arrive(&a_full);

      const float band = P.band_scale * sqrtf(qn2) * 1.0001f;
      float top[KB];
#pragma unroll
      for (int i = 0; i < KB; ++i) top[i] = -INFINITY;
      float theta_local = -INFINITY;
      uint32_t g_key = qv ? ld_volatile_u32(P.theta + q) : 0u;
      uint32_t g_pending = g_key;
      float theta = g_key ? key2f(g_key) : -INFINITY;
      uint32_t published = 0;
      const int r0 = slice * SLICE_ROWS, r1 = min(P.N, r0 + SLICE_ROWS);
      int tiles = 0;
      for (int row0 = r0; row0 < r1; row0 += BN, ++it, ++tiles) {
        const int b = it & 1, fb = it >> 1;
        if (!mbar_wait(&acc_full[b], fb & 1, P.err, ERR_TIMEOUT_FULL)) { ok = false; break; }
        tc::fence_after();
        uint32_t sc0[32], sc1[32];
        tc::ld_32x32b_x32(tmem + lane_base + ACC_COL + (uint32_t)(b * BN), sc0);
        tc::ld_32x32b_x32(tmem + lane_base + ACC_COL + (uint32_t)(b * BN + 32), sc1);
        tc::wait_ld();
        tc::fence_before();
        mbar_arrive(&acc_empty[b]);
        if (!qv) continue;
        // global threshold read one tile ahead (its latency overlaps this tile)
        if (g_pending) theta = fmaxf(theta, key2f(g_pending));
        g_pending = ld_volatile_u32(P.theta + q);
        const int nrow = min(BN, r1 - row0);
        // common case, constant register indices: which rows can still matter?
        const float lim = theta - band;
        uint64_t mask = 0ull;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          mask |= (uint64_t)(__uint_as_float(sc0[i]) >= lim) << i;
          mask |= (uint64_t)(__uint_as_float(sc1[i]) >= lim) << (32 + i);
        }
        if (nrow < BN) mask &= (1ull << nrow) - 1ull;
        if (mask) {
          // rare: stage the scores ([row][thread], conflict-free), first raise the
          // k best with them, then append the rows still within the band
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            stash[i * BQ + threadIdx.x] = __uint_as_float(sc0[i]);
            stash[(32 + i) * BQ + threadIdx.x] = __uint_as_float(sc1[i]);
          }
          for (uint64_t m = mask; m; m &= m - 1ull) {
            const int i = __ffsll((long long)m) - 1;
            const float sv = stash[i * BQ + threadIdx.x];
            if (sv > theta_local) {
              float x = sv;
#pragma unroll
              for (int j = 0; j < KB; ++j) {
                const float t = top[j];
                const bool gt = x > t;
                top[j] = gt ? x : t;
                x = gt ? t : x;
              }
              float kth = top[0];
#pragma unroll
              for (int j = 0; j < KB; ++j)
                if (j == P.k - 1) kth = top[j];
              theta_local = kth;
            }
          }
          theta = fmaxf(theta, theta_local);
          const float lim2 = theta - band;
          for (uint64_t m = mask; m; m &= m - 1ull) {
            const int i = __ffsll((long long)m) - 1;
            if (stash[i * BQ + threadIdx.x] >= lim2) {
              const int slot = atomicAdd(P.cand_count + q, 1);
              if (slot < P.cap)
                P.cand[(size_t)q * P.cap + slot] =
                    ((unsigned long long)f2key(stash[i * BQ + threadIdx.x]) << 32) | (uint32_t)(row0 + i);
            }
          }
        }
        if ((tiles & 7) == 7 && theta_local > -INFINITY) {
          const uint32_t key = f2key(theta_local);
          if (key > published) {
            atomicMax(P.theta + q, key);
            published = key;
          }
        }
      }
      if (qv && theta_local > -INFINITY) {
        const uint32_t key = f2key(theta_local);
        if (key > published) atomicMax(P.theta + q, key);
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 5) tc::tmem_dealloc(tmem, 512);
}

// One CTA per query.  The candidate list was appended against running
// thresholds; the query's final threshold (k-th best tf32 score of k rows) is
// tighter, so candidates whose tf32 score is below it minus the band are
// dropped first.  The survivors are scored exactly in fp32 (the single-query
// scan's arithmetic: per-lane float4 FMAs, xor-tree reduction 16..1), then
// selected.
constexpr int RESCORE_SMEM_ROWS = 8192;

template <int VPL>
__global__ void __launch_bounds__(256) k_batch_rescore(const float* __restrict__ Q, const float* __restrict__ leaf,
                                                       const int* __restrict__ original_ids, int D, int k, int cap,
                                                       float band_scale, const uint32_t* __restrict__ theta,
                                                       const int* __restrict__ cand_count,
                                                       const unsigned long long* __restrict__ cand_in,
                                                       float* __restrict__ out_s, int* __restrict__ out_i,
                                                       int* __restrict__ overflow) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);
  unsigned long long* sel = cand + RESCORE_SMEM_ROWS;
  SelectScratch* scratch = reinterpret_cast<SelectScratch*>(sel + 32);
  __shared__ int s_n;
  __shared__ float s_qn2[8];
  const int q = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int total = cand_count[q];
  const int D4 = D >> 2;
  const float4* q4 = reinterpret_cast<const float4*>(Q + (size_t)q * D);
  float4 qv[VPL];
  float qn2 = 0.f;
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int c = lane + 32 * v;
    qv[v] = c < D4 ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    qn2 = fmaf(qv[v].x, qv[v].x, fmaf(qv[v].y, qv[v].y, fmaf(qv[v].z, qv[v].z, fmaf(qv[v].w, qv[v].w, qn2))));
  }
  qn2 = warp_sum(qn2);
  if (threadIdx.x == 0) s_n = 0;
  if (lane == 0) s_qn2[warp] = qn2;
  __syncthreads();
  bool over = total > cap;
  if (!over) {
    const uint32_t tk = theta[q];
    const float lim = tk ? key2f(tk) - band_scale * sqrtf(s_qn2[0]) * 1.0001f : -INFINITY;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const unsigned long long e = cand_in[(size_t)q * cap + i];
      if (key2f((uint32_t)(e >> 32)) >= lim) {
        const int slot = atomicAdd(&s_n, 1);
        if (slot < RESCORE_SMEM_ROWS) cand[slot] = e & 0xFFFFFFFFull;
      }
    }
    __syncthreads();
    over = s_n > RESCORE_SMEM_ROWS;
  }
  if (over) {  // this query must be answered another way
    if (threadIdx.x == 0) atomicAdd(overflow, 1);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      out_s[(size_t)q * k + i] = -INFINITY;
      out_i[(size_t)q * k + i] = -2;
    }
    return;
  }
  const int n = s_n;
  for (int i = warp; i < n; i += nw) {
    const int row = (int)(uint32_t)cand[i];
    const float4* x4 = reinterpret_cast<const float4*>(leaf + (size_t)row * D);
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = lane + 32 * v;
      if (c < D4) {
        const float4 x = __ldg(x4 + c);
        acc = fmaf(x.x, qv[v].x, acc);
        acc = fmaf(x.y, qv[v].y, acc);
        acc = fmaf(x.z, qv[v].z, acc);
        acc = fmaf(x.w, qv[v].w, acc);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL_MASK, acc, o);
    __syncwarp();
    if (lane == 0) cand[i] = pack_cand(f2key(acc), (uint32_t)row);
  }
  __syncthreads();
  int selN = 1;
  while (selN < k) selN <<= 1;
  block_select_topk<false>(cand, n, k, sel, selN, scratch);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long c = sel[i];
    out_s[(size_t)q * k + i] = c ? key2f(cand_key(c)) : -INFINITY;
    out_i[(size_t)q * k + i] = c ? original_ids[cand_row(c)] : -1;
  }
}

// Max row norm (upper bound) of the leaf matrix: one warp per row, grid-stride.
__global__ void k_max_row_norm(const float* __restrict__ leaf, int N, int D, unsigned int* __restrict__ out_key) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  float mx = 0.f;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < N; r += warps) {
    const float* x = leaf + r * D;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s = fmaf(x[d], x[d], s);
    s = warp_sum(s);
    mx = fmaxf(mx, s);
  }
  if (lane == 0) atomicMax(out_key, __float_as_uint(mx));  // non-negative floats order as their bits
}

// ---------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_leaf_tensor_map(const float* leaf, int N, int D, void* out_map) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)N};
  cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)BN};
  cuuint32_t estr[2] = {1, 1};
  return enc(reinterpret_cast<CUtensorMap*>(out_map), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(leaf),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_max_row_norm(const float* leaf, int N, int D, unsigned int* out_key, int sms, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(out_key, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  k_max_row_norm<<<sms * 8, 256, 0, st>>>(leaf, N, D, out_key);
  return cudaGetLastError();
}

// Ring depth from the shared-memory budget; at least 120 KB is requested so that
// one CTA (and one 512-column TMEM allocation) occupies each SM.
static constexpr int BATCH_SMEM_BUDGET = 227 * 1024 - 1024;
static int batch_stages(int kb) {
  const int s = (BATCH_SMEM_BUDGET - BN * BQ * 4 - 1024) / (kb * BOX_BYTES);
  return s < BATCH_MAX_STAGES ? s : BATCH_MAX_STAGES;
}
static int batch_scan_smem(int kb, int stages) {
  const int b = stages * kb * BOX_BYTES + BN * BQ * 4 + 1024;
  return b < 120 * 1024 ? 120 * 1024 : b;
}

template <int KB>
static cudaError_t launch_batch_scan_t(const void* map, const BatchScanParams& P, int grid, cudaStream_t st) {
  const int smem = batch_scan_smem(P.kb, P.stages);
  static int configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(k_batch_scan<KB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  k_batch_scan<KB><<<grid, BATCH_THREADS, smem, st>>>(*reinterpret_cast<const CUtensorMap*>(map), P);
  return cudaGetLastError();
}

template <int VPL>
static cudaError_t launch_rescore_t(const float* Q, const IndexView& ix, const BatchWorkspace& bw, int B, int k,
                                    float band_scale, float* out_s, int* out_i, cudaStream_t st) {
  const size_t smem = (size_t)RESCORE_SMEM_ROWS * 8 + 32 * 8 + sizeof(SelectScratch) + 16;
  static size_t configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(k_batch_rescore<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  k_batch_rescore<VPL><<<B, 256, smem, st>>>(Q, ix.leaf, ix.original_ids, ix.D, k, bw.cap, band_scale, bw.theta,
                                             bw.cand_count, bw.cand, out_s, out_i, bw.overflow);
  return cudaGetLastError();
}

cudaError_t launch_batch_search(const IndexView& ix, const BatchWorkspace& bw, const float* Q, int B, int k,
                                float* out_scores, int* out_ids, cudaStream_t st) {
  cudaError_t e;
  if ((e = cudaMemsetAsync(bw.theta, 0, sizeof(uint32_t) * B, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(bw.cand_count, 0, sizeof(int) * B, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(bw.overflow, 0, sizeof(int), st)) != cudaSuccess) return e;
  BatchScanParams P{};
  P.Q = Q;
  P.B = B;
  P.D = ix.D;
  P.N = ix.N;
  P.k = k;
  P.kb = (ix.D + 31) / 32;
  P.stages = batch_stages(P.kb);
  if (P.stages < 2 || ix.D % 4 != 0 || ix.D > BATCH_MAX_DIM || k < 1 || k > BATCH_MAX_K) return cudaErrorInvalidValue;
  P.QT = (B + BQ - 1) / BQ;
  const int slices = (ix.N + SLICE_ROWS - 1) / SLICE_ROWS;
  P.units = P.QT * slices;
  // eps = (2^-9 + 2^-20 + 2 D 2^-23 + gamma_D) ||q|| max||x||, padded; band = 2 eps
  const double u = 5.9604644775390625e-08;
  const double gD = ix.D * u / (1.0 - ix.D * u);
  const double eps_rel = 1.953125e-3 + 9.5367431640625e-07 + 2.0 * ix.D * 1.1920928955078125e-07 + gD;
  P.band_scale = (float)(2.0 * eps_rel * 1.01 * bw.xmax);
  P.theta = bw.theta;
  P.cand_count = bw.cand_count;
  P.cand = bw.cand;
  P.cap = bw.cap;
  P.err = bw.err;
  const int grid = P.units < bw.sms ? P.units : bw.sms;
  e = (k <= 16) ? launch_batch_scan_t<16>(bw.tmap, P, grid, st) : launch_batch_scan_t<32>(bw.tmap, P, grid, st);
  if (e != cudaSuccess) return e;
  const int vpl = (ix.D / 4 + 31) / 32;
  switch (vpl) {
    case 1: return launch_rescore_t<1>(Q, ix, bw, B, k, P.band_scale, out_scores, out_ids, st);
    case 2: return launch_rescore_t<2>(Q, ix, bw, B, k, P.band_scale, out_scores, out_ids, st);
    default: return launch_rescore_t<3>(Q, ix, bw, B, k, P.band_scale, out_scores, out_ids, st);
  }
}

}  // namespace cb
