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
// NaN ranks above every number (torch.topk's order); -0 equals +0.
//
// One CTA of 32 warps per row; warp w owns the w-th of 32 consecutive
// position ranges of the row (a multiple of 32 positions each), so position
// order is warp order.  On an order-preserving 32-bit key of each score:
//   1. the CTA histograms the top 11 bits (shared atomics into 8
//      sub-histograms, one per four warps) and finds the bin b1 holding the
//      k-th largest key;
//   2. every warp re-reads its range (from L2) and keeps every key at or
//      above b1 with its position in a per-warp list (position order), while
//      the CTA histograms the next 11 bits of the keys inside b1 -> bin b2;
//   3. the listed keys inside (b1, b2) histogram their last 10 bits -> the
//      k-th largest key T exactly, and how many keys equal to T are selected;
//   4. per-warp counts of listed keys above T and equal to T, scanned over the
//      warps, give every warp its output offset and its share of the ties
//      (lowest positions first);
//   5. every warp walks its list in order and writes the selected positions
//      with warp ballots: the output comes out sorted with no sort and no
//      third read of the scores.
// A warp whose list overflows (the top keys concentrated in its range, or many
// equal scores) recomputes steps 3-5 from its range in global memory instead;
// the result is the same.
// Every output store is bounds-checked against k.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace nvqsa {
namespace {

constexpr int kTkThreads = 1024;
constexpr int kTkWarps = kTkThreads / 32;
constexpr int kTkBins = 2048;          // 11-bit digits (the last digit has 10 bits)
constexpr int kTkListPerWarp = 256;    // (key, position) pairs at or above the first pass's bin, per warp
constexpr int kTkUnroll = 8;           // loads in flight per lane
constexpr int kTkSubHists = 8;         // histogram copies (warp w adds into copy w / 4)

struct TopkParams {
  const float* scores;
  int64_t score_stride;    // elements between rows
  const int32_t* lengths;  // [rows] valid positions per row, or nullptr: all `context`
  int64_t rows, context;
  int32_t k;
  int32_t* out;
  int64_t out_stride;      // elements between rows
  int32_t vec;             // every row starts 16-byte aligned: the first pass loads float4
};

struct TopkSmem {
  int hist[kTkSubHists][kTkBins];
  uint32_t lkey[kTkWarps][kTkListPerWarp];
  int32_t lpos[kTkWarps][kTkListPerWarp];
  int warp_sums[kTkWarps];
  int wgt[kTkWarps];   // keys above T, per warp
  int weq[kTkWarps];   // keys equal to T, per warp
  uint32_t s_bin;
  int s_need;
};

// Order-preserving key: a larger float gives a larger unsigned key; NaN gets the largest key; -0 equals +0.
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t b = __float_as_uint(f);
  if ((b & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int m = 16; m; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Exclusive prefix sum over the block of one value per thread; `total` gets the sum.
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
    int w = warp_sums[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += y;
    }
    warp_sums[lane] = w;  // inclusive prefix over the warps
  }
  __syncthreads();
  total = warp_sums[kTkWarps - 1];
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  __syncthreads();  // warp_sums may be reused by the next scan
  return before;
}

// Finds the bin of hist[0, nbins) holding the need-th largest key, counting from the top bin down; returns it
// and leaves the key's rank inside the bin in s_need.
__device__ __forceinline__ uint32_t select_bin(TopkSmem& sm, int nbins, int need) {
  const int tid = threadIdx.x;
  const int per = nbins / kTkThreads;  // 2 or 1: thread t owns bins [nbins - (t + 1) per, nbins - t per)
  int c0 = 0, c1 = 0;
#pragma unroll
  for (int h = 0; h < kTkSubHists; ++h) {
    c0 += sm.hist[h][nbins - 1 - tid * per];
    if (per > 1) c1 += sm.hist[h][nbins - 2 - tid * per];
  }
  int total;
  const int before = block_scan(c0 + c1, sm.warp_sums, total);  // keys in the bins above this thread's
  if (before < need && before + c0 + c1 >= need) {
    if (before + c0 >= need) {
      sm.s_bin = (uint32_t)(nbins - 1 - tid * per);
      sm.s_need = need - before;
    } else {
      sm.s_bin = (uint32_t)(nbins - 2 - tid * per);
      sm.s_need = need - before - c0;
    }
  }
  __syncthreads();
  return sm.s_bin;
}

__global__ void __launch_bounds__(kTkThreads) topk_indices_kernel(const TopkParams p) {
  extern __shared__ __align__(16) uint8_t tk_smem_raw[];
  TopkSmem& sm = *reinterpret_cast<TopkSmem*>(tk_smem_raw);
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const float* srow = p.scores + row * p.score_stride;
  int32_t* orow = p.out + row * p.out_stride;
  int64_t len = p.lengths ? (int64_t)__ldg(p.lengths + row) : p.context;
  len = len < 0 ? 0 : (len > p.context ? p.context : len);
  const int k = p.k;

  if (len <= k) {  // everything valid is selected, in order; the rest is padding
    for (int64_t i = tid; i < k; i += kTkThreads) orow[i] = i < len ? (int32_t)i : -1;
    return;
  }

  // this warp's positions [lo, hi): the warp-th of 32 ranges of a multiple of 32 positions (int32: context
  // < 2^31)
  const int span = (int)((((len + kTkWarps - 1) / kTkWarps) + 31) & ~(int64_t)31);
  const int lo = (int)min(len, (int64_t)warp * span);
  const int hi = (int)min(len, (int64_t)lo + span);
  int* hist = sm.hist[warp / (kTkWarps / kTkSubHists)];

  for (int i = tid; i < kTkSubHists * kTkBins; i += kTkThreads) (&sm.hist[0][0])[i] = 0;
  __syncthreads();

  // ---- 1. top 11 bits ----
  if (p.vec) {  // lane -> 4 consecutive positions (lo is a multiple of 32, the row 16-byte aligned)
    for (int b = lo; b < hi; b += 128 * (kTkUnroll / 2)) {
      float4 v[kTkUnroll / 2];
#pragma unroll
      for (int u = 0; u < kTkUnroll / 2; ++u) {
        const int pos = b + u * 128 + lane * 4;
        if (pos + 3 < hi) {
          v[u] = __ldg(reinterpret_cast<const float4*>(srow + pos));
        } else {
          v[u].x = pos < hi ? __ldg(srow + pos) : 0.0f;
          v[u].y = pos + 1 < hi ? __ldg(srow + pos + 1) : 0.0f;
          v[u].z = pos + 2 < hi ? __ldg(srow + pos + 2) : 0.0f;
          v[u].w = 0.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < kTkUnroll / 2; ++u) {
        const int pos = b + u * 128 + lane * 4;
        if (pos < hi) atomicAdd(&hist[order_key(v[u].x) >> 21], 1);
        if (pos + 1 < hi) atomicAdd(&hist[order_key(v[u].y) >> 21], 1);
        if (pos + 2 < hi) atomicAdd(&hist[order_key(v[u].z) >> 21], 1);
        if (pos + 3 < hi) atomicAdd(&hist[order_key(v[u].w) >> 21], 1);
      }
    }
  } else {
    for (int b = lo; b < hi; b += 32 * kTkUnroll) {
      float v[kTkUnroll];
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const int pos = b + u * 32 + lane;
        v[u] = pos < hi ? __ldg(srow + pos) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u)
        if (b + u * 32 + lane < hi) atomicAdd(&hist[order_key(v[u]) >> 21], 1);
    }
  }
  __syncthreads();
  const uint32_t b1 = select_bin(sm, kTkBins, k);
  const int need1 = sm.s_need;
  for (int i = tid; i < kTkSubHists * kTkBins; i += kTkThreads) (&sm.hist[0][0])[i] = 0;
  __syncthreads();

  // ---- 2. keys at or above b1 kept in the warp's list, in position order; b1's next 11 bits ----
  int nlist = 0;  // warp-uniform
  for (int b = lo; b < hi; b += 32 * kTkUnroll) {
    float v[kTkUnroll];
#pragma unroll
    for (int u = 0; u < kTkUnroll; ++u) {
      const int pos = b + u * 32 + lane;
      v[u] = pos < hi ? __ldg(srow + pos) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kTkUnroll; ++u) {
      const int pos = b + u * 32 + lane;
      const uint32_t key = order_key(v[u]);
      const uint32_t d1 = key >> 21;
      const bool keep = pos < hi && d1 >= b1;
      const uint32_t m = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const int idx = nlist + __popc(m & lt_mask);
        if (idx < kTkListPerWarp) {
          sm.lkey[warp][idx] = key;
          sm.lpos[warp][idx] = pos;
        }
        if (d1 == b1) atomicAdd(&hist[(key >> 10) & (kTkBins - 1)], 1);
      }
      nlist += __popc(m);
    }
  }
  __syncthreads();
  const uint32_t b2 = select_bin(sm, kTkBins, need1);
  const int need2 = sm.s_need;
  for (int i = tid; i < kTkSubHists * kTkBins; i += kTkThreads) (&sm.hist[0][0])[i] = 0;
  __syncthreads();
  const uint32_t prefix22 = (b1 << 11) | b2;
  const bool listed = nlist <= kTkListPerWarp;  // warp-uniform

  // ---- 3. last 10 bits of the keys inside (b1, b2) ----
  if (listed) {
    for (int i = lane; i < nlist; i += 32) {
      const uint32_t key = sm.lkey[warp][i];
      if ((key >> 10) == prefix22) atomicAdd(&hist[key & 1023u], 1);
    }
  } else {
    for (int b = lo; b < hi; b += 32 * kTkUnroll) {
      float v[kTkUnroll];
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const int pos = b + u * 32 + lane;
        v[u] = pos < hi ? __ldg(srow + pos) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const uint32_t key = order_key(v[u]);
        if (b + u * 32 + lane < hi && (key >> 10) == prefix22) atomicAdd(&hist[key & 1023u], 1);
      }
    }
  }
  __syncthreads();
  const uint32_t T = (prefix22 << 10) | select_bin(sm, 1024, need2);
  const int ties = sm.s_need;  // keys equal to T that are selected: the lowest positions

  // ---- 4. per-warp counts above and at T; offsets over the warps ----
  int wg = 0, we = 0;
  if (listed) {
    for (int i = lane; i < nlist; i += 32) {
      const uint32_t key = sm.lkey[warp][i];
      wg += key > T ? 1 : 0;
      we += key == T ? 1 : 0;
    }
  } else {
    for (int b = lo; b < hi; b += 32 * kTkUnroll) {
      float v[kTkUnroll];
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const int pos = b + u * 32 + lane;
        v[u] = pos < hi ? __ldg(srow + pos) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const bool valid = b + u * 32 + lane < hi;
        const uint32_t key = order_key(v[u]);
        wg += (valid && key > T) ? 1 : 0;
        we += (valid && key == T) ? 1 : 0;
      }
    }
  }
  wg = warp_sum(wg);
  we = warp_sum(we);
  if (lane == 0) {
    sm.wgt[warp] = wg;
    sm.weq[warp] = we;
  }
  __syncthreads();
  int gt_before = 0, eq_before = 0;
  for (int w = 0; w < warp; ++w) {
    gt_before += sm.wgt[w];
    eq_before += sm.weq[w];
  }
  const int sel_before = gt_before + min(ties, eq_before);
  const int sel = wg + max(0, min(we, ties - eq_before));

  // ---- 5. selected positions in order: ballots over the list (or over 32 consecutive positions) ----
  int written = 0, eq_seen = eq_before;
  auto emit = [&](uint32_t key, int pos, bool valid) {
    const bool g = valid && key > T, e = valid && key == T;
    const uint32_t em = __ballot_sync(0xffffffffu, e);
    const bool take = g || (e && eq_seen + __popc(em & lt_mask) < ties);
    const uint32_t tm = __ballot_sync(0xffffffffu, take);
    const int oi = sel_before + written + __popc(tm & lt_mask);
    if (take && oi < k) orow[oi] = pos;
    written += __popc(tm);
    eq_seen += __popc(em);
  };
  if (listed) {
    for (int i0 = 0; i0 < nlist && written < sel; i0 += 32) {
      const int i = i0 + lane;
      const bool valid = i < nlist;
      emit(valid ? sm.lkey[warp][i] : 0u, valid ? sm.lpos[warp][i] : 0, valid);
    }
  } else {
    for (int b = lo; b < hi && written < sel; b += 32 * kTkUnroll) {
      float v[kTkUnroll];
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const int pos = b + u * 32 + lane;
        v[u] = pos < hi ? __ldg(srow + pos) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kTkUnroll; ++u) {
        const int pos = b + u * 32 + lane;
        emit(order_key(v[u]), pos, pos < hi);
      }
    }
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
  if (rows > 0x7fffffffLL || context > 0x7fffffffLL) return NVQSA_ERR_BAD_SHAPE;  // grid and int32 positions
  TopkParams p;
  p.scores = scores;
  p.score_stride = score_stride_row;
  p.lengths = lengths;
  p.rows = rows;
  p.context = context;
  p.k = k;
  p.out = out;
  p.out_stride = out_stride_row;
  p.vec = ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0 && (score_stride_row & 3) == 0) ? 1 : 0;
  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVQSA_ERR_CUDA;
  if (!configured[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(topk_indices_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(TopkSmem)) != cudaSuccess)
      return NVQSA_ERR_CUDA;
    configured[dev].store(true, std::memory_order_relaxed);
  }
  topk_indices_kernel<<<(unsigned)rows, kTkThreads, sizeof(TopkSmem), as_stream(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}
