// QSA indexer top-k selection on sm_100a: the step in front of the sparse reader.
//
// The reference's QSA layer runs its indexer and receives
// topk_indices_buffer[:num_tokens], int32 [num_tokens, output_width], the
// logical token indices every query token attends to
// (integration/snapshot/qsa.py:537-545, :605-616); the reader masks -1.  The
// indexer module itself is not vendored in the reference, so this file builds
// the selection to that buffer contract: for each row (query token), among the
// scores of positions [0, length) -- its causal context -- the indices of the k
// largest, written in ascending index order; ties at the k-th value go to the
// lowest indices; a context shorter than k yields 0 .. length - 1 and -1 after.
// NaN ranks above every number (torch.topk's order).
//
// One CTA of 512 threads per row, everything in one launch:
//   1. radix select on an order-preserving 32-bit key of each score: three
//      histogram passes over digits of 11, 11 and 10 bits (shared-memory
//      histograms), each narrowing the candidates to the bin that holds the
//      k-th largest key, give that key T exactly and the count of keys above it;
//   2. one ordered collection pass: in rounds of 512 consecutive positions,
//      a position is selected when its key is above T, or equal to T while the
//      tie budget lasts; warp ballots and a block scan place each selected
//      index at its rank, so the output comes out sorted with no sort.
// Reads are coalesced (position = round * 512 + thread); the row's later passes
// are served from L2.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace nvqsa {
namespace {

constexpr int kTopkThreads = 512;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kMaxBins = 2048;

struct TopkParams {
  const float* scores;
  int64_t score_stride;  // elements between rows
  const int32_t* lengths;  // [rows] valid positions per row, or nullptr: all `context`
  int64_t rows, context;
  int32_t k;
  int32_t* out;
  int64_t out_stride;    // elements between rows
};

// Order-preserving key: a larger float gives a larger unsigned key; NaN gets the largest key.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  if ((b & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Exclusive prefix sum over the block of one value per thread; returns the thread's prefix, `total` the sum.
__device__ __forceinline__ int block_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kTopkWarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += y;
    }
    if (lane < kTopkWarps) warp_sums[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  total = warp_sums[kTopkWarps - 1];
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  __syncthreads();  // warp_sums may be reused by the caller's next scan
  return before;
}

__global__ void __launch_bounds__(kTopkThreads) topk_indices_kernel(const TopkParams p) {
  __shared__ int hist[kMaxBins];
  __shared__ int warp_sums[kTopkWarps];
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;       // rank of the k-th key among the candidates of the current pass (1-based)
  __shared__ int s_above;      // keys known to be above every remaining candidate

  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const float* srow = p.scores + row * p.score_stride;
  int32_t* orow = p.out + row * p.out_stride;
  int64_t len = p.lengths ? (int64_t)p.lengths[row] : p.context;
  len = len < 0 ? 0 : (len > p.context ? p.context : len);
  const int k = p.k;

  if (len <= k) {  // everything valid is selected, in order; the rest is padding
    for (int64_t i = tid; i < k; i += kTopkThreads) orow[i] = i < len ? (int32_t)i : -1;
    return;
  }

  // ---------------- 1. radix select: digits of 11, 11 and 10 bits from the top ----------------
  uint32_t prefix = 0, pmask = 0;
  if (tid == 0) {
    s_need = k;
    s_above = 0;
  }
  const int shifts[3] = {21, 10, 0};
  const int widths[3] = {11, 11, 10};
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = shifts[pass], bins = 1 << widths[pass];
    for (int i = tid; i < bins; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    for (int64_t i = tid; i < len; i += kTopkThreads) {
      const uint32_t key = order_key(__ldg(srow + i));
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & (bins - 1)], 1);
    }
    __syncthreads();
    // Counts from the top bin down: thread t owns bins [bins - (t + 1) * per, bins - t * per).
    const int per = bins / kTopkThreads;  // 4 or 2
    int mine = 0;
    for (int j = 0; j < per; ++j) mine += hist[bins - 1 - (tid * per + j)];
    const int need = s_need;  // read before the scan's barriers: the winner below rewrites it
    int total;
    const int before = block_scan(mine, warp_sums, total);  // keys in bins above this thread's range
    if (before < need && before + mine >= need) {
      // the k-th candidate lies in this thread's range: walk it from the top
      int acc = before;
      for (int j = 0; j < per; ++j) {
        const int bin = bins - 1 - (tid * per + j);
        const int c = hist[bin];
        if (acc + c >= need) {
          s_prefix = prefix | ((uint32_t)bin << shift);
          s_need = need - acc;
          s_above += acc;
          break;
        }
        acc += c;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    pmask |= (uint32_t)(bins - 1) << shift;
  }
  const uint32_t T = prefix;     // the k-th largest key
  const int ties = s_need;       // how many keys equal to T are selected (the lowest positions)

  // ---------------- 2. ordered collection ----------------
  const int lane = tid & 31, warp = tid >> 5;
  int base = 0, ties_used = 0;   // block-uniform running counts
#pragma unroll 1
  for (int64_t r0 = 0; r0 < len; r0 += kTopkThreads) {
    const int64_t i = r0 + tid;
    uint32_t key = 0;
    if (i < len) key = order_key(__ldg(srow + i));
    const bool gt = i < len && key > T;
    const bool eq = i < len && key == T;
    // ties in index order: rank among this round's ties, offset by the ties already taken
    const uint32_t eq_b = __ballot_sync(0xffffffffu, eq);
    const uint32_t gt_b = __ballot_sync(0xffffffffu, gt);
    if (lane == 0) {
      hist[warp] = __popc(eq_b);
      hist[kTopkWarps + warp] = __popc(gt_b);
    }
    __syncthreads();
    int eq_before = 0, gt_before = 0, eq_round = 0, gt_round = 0;
    for (int w = 0; w < kTopkWarps; ++w) {
      const int e = hist[w], g = hist[kTopkWarps + w];
      if (w < warp) { eq_before += e; gt_before += g; }
      eq_round += e;
      gt_round += g;
    }
    __syncthreads();  // hist is rewritten by the next round
    const uint32_t below = (1u << lane) - 1u;
    const int my_eq_rank = ties_used + eq_before + __popc(eq_b & below);
    const bool take = gt || (eq && my_eq_rank < ties);
    // selected before this position in this round: all gt before it, ties before it within the budget
    const int eq_taken_before = min(max(ties - ties_used, 0), eq_before + __popc(eq_b & below));
    if (take) orow[base + gt_before + __popc(gt_b & below) + eq_taken_before] = (int32_t)i;
    const int eq_taken_round = min(max(ties - ties_used, 0), eq_round);
    base += gt_round + eq_taken_round;
    ties_used += eq_taken_round;
    if (base >= k) break;
  }
}

}  // namespace
}  // namespace nvqsa

using namespace nvqsa;

extern "C" int nvqsa_topk_indices(const float* scores, int64_t score_stride_row, const int32_t* lengths, int64_t rows,
                                  int64_t context, int32_t k, int32_t* out, int64_t out_stride_row, void* stream) {
  if (rows < 0 || context < 0 || k < 1 || score_stride_row < context || out_stride_row < k)
    return NVQSA_ERR_BAD_SHAPE;
  if (rows == 0) return NVQSA_OK;
  if (!out || (!scores && context > 0)) return NVQSA_ERR_NULL_POINTER;
  if (rows > 0x7fffffffLL) return NVQSA_ERR_BAD_SHAPE;
  TopkParams p;
  p.scores = scores;
  p.score_stride = score_stride_row;
  p.lengths = lengths;
  p.rows = rows;
  p.context = context;
  p.k = k;
  p.out = out;
  p.out_stride = out_stride_row;
  topk_indices_kernel<<<(unsigned)rows, kTopkThreads, 0, as_stream(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}
