// QSA sparse paged decode attention over an NVFP4 cache, sm_100a.
//
// Replaces the reference's Triton reader (python/nvfp4_qsa/kernels.py:168-403).
// The reference runs one program per (query row, kv head), so a single decode
// row occupies 2 SMs; here the selected tokens of each (row, kv head) are
// split across CTAs (split-KV) and merged with a base-2 log-sum-exp, the
// layout of the reference's split-K sibling (src/qsa_fp8_harness.py:183-208).
//
// One CTA = (row, kv head, split) = 4 warps = 2 warp pairs.
//  * Prologue: the CTA resolves its share of the row's selections through
//    token_to_request / block_table (masking rules of kernels.py:241-257) and
//    compacts the valid ones into a shared list, so masked selections cost
//    nothing (they contribute exp2(-1e20 - m) = 0 in the reference).  The
//    share is every splits-th chunk of 32 index positions (chunks split,
//    split + splits, ...), so a row whose valid selections are bunched in one
//    part of its list -- a sorted list on a device that holds only some of the
//    sequence's pages -- still spreads them evenly over the CTAs.
//  * Gather: for the reference cache layout (one contiguous 288-byte record
//    K data | K scales | V data | V scales per (block, head, token), rows of a
//    [blocks*kv_heads*page, 288] byte matrix) warp 0 fetches each stage of 32
//    records with eight TMA tile::gather4 loads (4 rows each) through a 2D
//    tensor map, into a 4-stage shared-memory ring; an mbarrier per stage
//    tracks the bytes.  Rows past the last valid selection use an
//    out-of-range row coordinate and arrive zero-filled.  Other layouts fall
//    back to one bulk copy per record (contiguous record) or four (split
//    regions).  Within each group of four rows the tokens are permuted
//    ({0,2,1,3}, {5,7,4,6} per 8 tokens) so that both consumer read patterns
//    below are bank-conflict free.  Every mbarrier wait is bounded; a wait
//    that runs out raises a device error flag (nvqsa_read_error_flags) and
//    the CTA returns.
//    Measured on B200: gathers of random 288-byte records top out near
//    4.1 TB/s (gather4 or 64 warps/SM of LDG.128) against 6.5 TB/s for a
//    sequential copy; issuing one bulk copy per record costs the issuing warp
//    ~90 cycles per record, which is why gather4 is used.
//  * Each warp pair takes 16 tokens of a stage; warp h of the pair owns head
//    dimensions [128h, 128h+128).  Dequantisation happens in registers
//    straight into mma.sync fragments: one cvt.rn.f16x2.e2m1x2 per byte and
//    one f16x2 multiply by the E4M3 group scale (both exact: e2m1 * e4m3 has
//    at most 5 significant bits and lies in [2^-10, 2688]).  The head
//    dimension is permuted consistently between Q and K so that each lane's
//    K bytes are one 16-byte chunk; V's nibbles are re-paired across tokens
//    with two LOP3s per word before conversion.
//  * S = Q K^T on m16n8k16 (M = 16 query heads, N = 8 tokens, K = 16 dims);
//    the two warps exchange their half-dimension partial scores through
//    shared memory, run the online softmax in base 2 (masked = -1e20 as in
//    kernels.py:316-331) and accumulate O = P V (M = heads, N = 8 dims,
//    K = 16 tokens) with P converted to f16 in registers.  The running max is
//    only raised when a tile exceeds it by more than 2^8, so the O rescale
//    (64 multiplies per lane) runs a handful of times per CTA instead of
//    every tile; P then stays below 256, well inside f16.
//  * Q is converted bf16 -> f16 after an exact per-head power-of-two
//    pre-scale (amax * 2^e in [2^14, 2^15)), folded back into the score scale.
#include <cuda.h>

#include <algorithm>
#include <cstddef>
#include <atomic>
#include <cstring>
#include <type_traits>

#include "common.cuh"

namespace nvqsa {
namespace {

constexpr int kHeadDim = 256;
constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kTile = 16;                        // tokens per warp tile (one m16n8k16 K-step of P V)
constexpr int kWarpStages = 3;                   // private ring slots per warp
constexpr int kMaxRange = 1024;                  // selections per CTA
constexpr int kChunk = 32;                       // index positions per interleaved chunk (one warp load)
constexpr int kMaxChunks = kMaxRange / kChunk;   // chunks per CTA
constexpr int kCompactIters = kMaxRange / kThreads;
constexpr int kRecordBytes = 288;                // K data + K scales + V data + V scales
constexpr int kStageBytes = kTile * kRecordBytes;
// FP8 sibling reader (gather mode 3): float8_e4m3 K and V rows of 256 bytes from two caches, staged as
// K | V | 16 bytes of skew per token (the skew keeps the per-lane K and V reads bank-conflict free).
constexpr int kGatherFp8 = 3;
constexpr int kGatherBf16 = 4;
// NVFP4 regions whose bases or strides are not 16-byte multiples (the reference takes any strides with a
// contiguous last dim, kernels.py:376-391): records copied with plain loads of copy_width bytes.
constexpr int kGatherPlain = 5;   // BF16 sibling reader: bf16 K and V rows of 512 bytes (sparse_attention_bf16_kernel)
constexpr int kFp8RecordBytes = 528;
constexpr int kFp8Stages = 2;
constexpr float kMaskedScore = -1.0e20f;
constexpr float kRescaleThreshold = 8.0f;        // log2 units: P <= 2^8 between rescales
constexpr uint32_t kSpinLimit = 1u << 22;        // bounded mbarrier waits
constexpr uint32_t kDrainSpinLimit = 1u << 16;   // bounded waits while abandoning a CTA

struct AttnParams {
  CUtensorMap rows_map;          // gather mode 0: [rows, 144] u16 view of the cache records
  const __nv_bfloat16* q;
  int64_t q_stride_row, q_stride_head;
  const uint8_t* region[4];      // key_data, key_scale, value_data, value_scale
  int64_t stride[4][3];          // block, token, head (bytes)
  int64_t num_blocks, page_size;
  int32_t kv_heads, group, query_heads;
  int32_t gather_mode;           // 0: tile::gather4 rows; 1: one bulk copy per record; 2: four per record;
                                 // 5: plain loads of copy_width bytes (unaligned bases or strides)
  int32_t copy_width;            // gather mode 5: 1, 2, 4 or 8 (the largest that divides every base and stride)
  int32_t total_rows;            // gather mode 0: rows of the record matrix (out-of-range row = zero fill)
  float score_scale;             // head_dim^-0.5 * log2(e) / key_global_scale
  float inv_value_scale;         // 1 / value_global_scale
  const int32_t* indices;
  int64_t topk;
  const int32_t* block_table;
  int64_t num_requests, table_width;
  const int32_t* token_to_request;
  int64_t rows;
  int32_t splits;                // CTAs per (row, kv head); CTA s takes chunks s, s + splits, ...
  int32_t mode;                  // 0: bf16 output; 1: fp32 partial (normalised O, lse)
  int32_t cluster;               // > 1: the splits of a (row, kv head) form one thread-block cluster of this size
  int32_t fuse;                  // splits > cluster limit: the last CTA of each (row, kv head) merges the splits
  int32_t final_mode;            // merged result: 0 -> bf16 `out`; 1 -> fp32 final_out / final_lse
  unsigned int* counters;        // [rows * kv_heads] arrival counters (zeroed before the launch)
  float* final_out;              // [rows][query_heads][256]
  float* final_lse;              // [rows][query_heads]
  // Split-KV across GPUs (xworld > 0): this rank's merged (O, lse) goes into slot xrank of every rank's
  // exchange buffer over NVLink, then the unit's final CTA waits for every rank's slot and merges them.
  int32_t xworld, xrank, xparity;
  float* xpeer[8];               // exchange buffer of every rank, as mapped in this process
  int32_t group_rows;            // grouped reader: consecutive rows per group that may share their selections
  int32_t vec_q;                 // 16-byte aligned query rows
  int32_t vec_o;                 // 16-byte aligned output rows
  __nv_bfloat16* out;
  int64_t o_stride_row, o_stride_head;
  float* part_out;               // [splits][rows][query_heads][256]
  float* part_lse;               // [splits][rows][query_heads]
  // Optional timing stamps (nullptr: off), %globaltimer nanoseconds per (row, kv head) unit, kStampSlots each.
  unsigned long long* stamps;
};

template <int REC, int STAGES>
struct __align__(128) SmemT {
  uint8_t rec[kWarps][STAGES][kTile * REC];       // private gather ring of each warp
  uint4 qfrag[16][32];                             // Q A-fragments: [k-step][lane] -> {a0a1,a2a3,a4a5,a6a7}
  int2 sel[kMaxRange];                             // (physical block, token in page) of valid selections
  unsigned long long full_bar[kWarps][STAGES];
  float smul[16];
  int cnt[kCompactIters][kWarps];
  int total;
  int abort;
  int last;
};
using Smem = SmemT<kRecordBytes, kWarpStages>;      // NVFP4 records
using SmemFp8 = SmemT<kFp8RecordBytes, kFp8Stages>;  // FP8 K and V rows

__device__ unsigned int g_error_flags;

// Programmatic dependent launch: let the stream's next reader launch as soon as every CTA of this grid has
// started, and wait (hardware wait, no spin) for the previous grid's completion and memory before touching
// global memory.  Both are no-ops for a launch without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
constexpr unsigned int kErrWaitTimeout = 1u;            // bit 0: an mbarrier wait ran out
// Timing stamps of one (row, kv head) unit (all %globaltimer ns of the GPU that writes them):
//   0 first CTA entry (min)      1 last CTA done with its tiles (max)   2 last part arrived at the unit counter
//   3 local merge done           4 partial pushed to every peer, flags raised
//   5 every peer's flag seen     6 result stored
constexpr int kStampSlots = 8;
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void stamp_min(const AttnParams& p, int64_t unit, int slot) {
  if (p.stamps) atomicMin(p.stamps + unit * kStampSlots + slot, globaltimer_ns());
}
__device__ __forceinline__ void stamp_max(const AttnParams& p, int64_t unit, int slot) {
  if (p.stamps) atomicMax(p.stamps + unit * kStampSlots + slot, globaltimer_ns());
}
__device__ __forceinline__ void stamp_set(const AttnParams& p, int64_t unit, int slot) {
  if (p.stamps) p.stamps[unit * kStampSlots + slot] = globaltimer_ns();
}
constexpr unsigned int kErrPeerTimeout = 2u;            // bit 1: another GPU's split-KV slot never arrived
constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the device error flag raised) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = kSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(&g_error_flags, kErrWaitTimeout);
  return false;
}
// Global -> shared bulk copy into this CTA, completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// TMA tile::gather4: four rows of the record matrix into 4*288 contiguous bytes of this CTA.
__device__ __forceinline__ void gather4_g2s(uint32_t dst, const CUtensorMap* map, int32_t r0, int32_t r1, int32_t r2,
                                            int32_t r3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];\n" ::"r"(dst),
      "l"(map), "r"(0), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(bar)
      : "memory");
}

// Distributed shared memory of a thread-block cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}
__device__ __forceinline__ float4 cluster_ld_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ int cluster_ld_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_st_s32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
// Every thread of every CTA of the cluster arrives; shared-memory writes before it are visible after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t dup_lo(uint32_t x) { return __byte_perm(x, 0, 0x1010); }
__device__ __forceinline__ uint32_t dup_hi(uint32_t x) { return __byte_perm(x, 0, 0x3232); }

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Byte offset of token t (0..15) inside a stage.  Each gather4 writes four
// consecutive 288-byte rows; per 8 tokens the rows hold tokens {0,2,1,3} and
// {5,7,4,6}, which keeps the K (16-byte) and V (8-byte) reads below free of
// shared-memory bank conflicts.
__device__ __forceinline__ int slot_off(int t) {
  const int i = t & 7;
  const int group = ((t >> 3) << 1) | (i >> 2);
  const int row = (i < 4) ? (((i & 1) << 1) | (i >> 1)) : ((((i & 1) ^ 1) << 1) | ((i >> 1) & 1));
  return (group * 4 + row) * kRecordBytes;
}
// Token held by row j (0..3) of gather group g (0..3) of a stage: inverse of slot_off.
__device__ __forceinline__ int group_token(int g, int j) {
  const int i = (g & 1) ? 4 + (((j & 1) << 1) | ((j >> 1) ^ 1)) : (((j & 1) << 1) | (j >> 1));
  return ((g >> 1) << 3) + i;
}

// Head dimensions covered by fragment k-step s (0..15) for mma thread-in-group c:
// k-steps 0..7 walk 16-byte chunk c of the 128 K bytes, 8..15 walk chunk 4+c, so
// each lane's K bytes are two 16-byte loads.  The first of the k-step's 4 dims is
// d = (s < 8) ? 32c + 4s : 128 + 32c + 4(s - 8); a0a1 / b0b1 hold dims d, d+1
// and a4a5 / b2b3 hold d+2, d+3.  Inverse, used to place Q: c = (d % 128) / 32,
// s = (d % 32) / 4 + 8 * (d / 128).

// Log-sum-exp merge of `splits` partials of one (row, query head) by one warp;
// lane L covers dims [8L, 8L + 8).  Split s of the outputs starts at
// part_out + s * out_split_stride ([rows][heads][256] dense), of the lse at
// part_lse + s * lse_split_stride ([rows][heads] dense).  Loads go through L2
// (ld.global.cg): inside the attention kernel the partials were written by
// other CTAs of the same launch.
struct MergeArgs {
  const float* part_out;
  const float* part_lse;
  int splits;
  int64_t out_split_stride, lse_split_stride;
  int mode;                       // 0: bf16 out; 1: fp32 out_f32 + out_lse
  __nv_bfloat16* out;
  int64_t o_stride_row, o_stride_head;
  int vec_o;
  float* out_f32;
  float* out_lse;
};

__device__ __forceinline__ void merge_item(const MergeArgs& a, int64_t row, int head, int64_t w, int lane) {
  // Four splits per round, every load of a round issued before any is used.
  float M = -INFINITY;
  for (int s0 = 0; s0 < a.splits; s0 += 4) {
    float l[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      l[u] = s0 + u < a.splits ? __ldcg(a.part_lse + (int64_t)(s0 + u) * a.lse_split_stride + w) : -INFINITY;
    M = fmaxf(M, fmaxf(fmaxf(l[0], l[1]), fmaxf(l[2], l[3])));
  }
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float den = 0.0f;
  if (M != -INFINITY) {
    for (int s0 = 0; s0 < a.splits; s0 += 4) {
      float l[4];
      float4 x[4], y[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        l[u] = -INFINITY;
        x[u] = y[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s0 + u < a.splits) {
          const int64_t s = s0 + u;
          l[u] = __ldcg(a.part_lse + s * a.lse_split_stride + w);
          const float4* po = reinterpret_cast<const float4*>(a.part_out + s * a.out_split_stride + w * kHeadDim +
                                                             lane * 8);
          x[u] = __ldcg(po);
          y[u] = __ldcg(po + 1);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float wt = l[u] == -INFINITY ? 0.0f : exp2f(l[u] - M);  // empty partials weigh 0
        den += wt;
        acc[0] += wt * x[u].x; acc[1] += wt * x[u].y; acc[2] += wt * x[u].z; acc[3] += wt * x[u].w;
        acc[4] += wt * y[u].x; acc[5] += wt * y[u].y; acc[6] += wt * y[u].z; acc[7] += wt * y[u].w;
      }
    }
  }
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] *= inv;
  if (a.mode == 0) {
    __nv_bfloat16* op = a.out + row * a.o_stride_row + (int64_t)head * a.o_stride_head + lane * 8;
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      u[i] = *reinterpret_cast<uint32_t*>(&b);
    }
    if (a.vec_o) {
      *reinterpret_cast<uint4*>(op) = make_uint4(u[0], u[1], u[2], u[3]);
    } else {
      unsigned short* os = reinterpret_cast<unsigned short*>(op);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        os[2 * i] = (unsigned short)(u[i] & 0xffffu);
        os[2 * i + 1] = (unsigned short)(u[i] >> 16);
      }
    }
  } else {
    float4* op = reinterpret_cast<float4*>(a.out_f32 + w * kHeadDim + lane * 8);
    op[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    op[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (lane == 0) a.out_lse[w] = den > 0.0f ? M + log2f(den) : -INFINITY;
  }
}

// Split-KV beyond one cluster: every part (one per cluster, its rank 0) has written its
// normalised partial and lse to the workspace; the last part to arrive at the unit's
// counter merges all parts into the output.  Called by every thread of the CTA.
// Log-sum-exp merge of `nparts` normalised partials of one (row, kv head) unit, part q at
// part_out + q * rows * heads * 256 and part_lse + q * rows * heads, into the bf16 output
// (out_mode 0) or fp32 f32_out / f32_lse (out_mode 1).  Called by every thread of the CTA;
// `scratch` holds nparts * 16 + 32 floats of shared memory.
__device__ __noinline__ void merge_unit_parts(const AttnParams& p, float* scratch, int64_t row, int kvh, int G, int tid,
                                              const float* part_out, const float* part_lse, int nparts, int out_mode,
                                              float* f32_out, float* f32_lse) {
  {
    // 1. every part's lse of this unit's heads into shared memory (ring space, free now)
    float* wt = scratch;                                      // [nparts][16]: lse, then weights
    float* head_m = wt + nparts * 16;                         // [16]
    float* head_den = head_m + 16;                            // [16]
    const int64_t items = p.rows * p.query_heads;
    const int64_t w0 = row * p.query_heads + (int64_t)kvh * G;
    for (int i = tid; i < nparts * G; i += kThreads) {
      const int part = i / G, j = i - part * G;
      wt[part * 16 + j] = __ldcg(part_lse + (int64_t)part * items + w0 + j);
    }
    __syncthreads();
    // 2. per head: max, weights 2^(lse - max) (0 for empty parts), their sum
    if (tid < G) {
      float M = -INFINITY;
      for (int part = 0; part < nparts; ++part) M = fmaxf(M, wt[part * 16 + tid]);
      float den = 0.0f;
      for (int part = 0; part < nparts; ++part) {
        const float l = wt[part * 16 + tid];
        const float x = (l == -INFINITY) ? 0.0f : exp2f(l - M);
        wt[part * 16 + tid] = x;
        den += x;
      }
      head_m[tid] = M;
      head_den[tid] = den;
    }
    __syncthreads();
    // 3. outputs: item = (head j, 8 dims).  A thread takes up to three items per pass (one pass for
    // G <= 12); each round issues the loads of three parts for all of the pass's items before any is used,
    // so a round costs one L2 round trip and eighteen float4 are in flight per thread.
    constexpr int kItemsPerThread = 3;
    constexpr int kPartsPerRound = 3;
    for (int it0 = 0; it0 < G * 32; it0 += kItemsPerThread * kThreads) {
    float acc[kItemsPerThread][8];
#pragma unroll
    for (int u = 0; u < kItemsPerThread; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.0f;
    for (int q0 = 0; q0 < nparts; q0 += kPartsPerRound) {
      float4 x[kItemsPerThread][kPartsPerRound], y[kItemsPerThread][kPartsPerRound];
#pragma unroll
      for (int u = 0; u < kItemsPerThread; ++u) {
        const int it = it0 + tid + u * kThreads;
        const int j = it >> 5, d8 = it & 31;
        const float* base = part_out + (w0 + (it < G * 32 ? j : 0)) * kHeadDim + d8 * 8;
#pragma unroll
        for (int v = 0; v < kPartsPerRound; ++v) {
          const bool in = q0 + v < nparts && it < G * 32;
          const float4* po = reinterpret_cast<const float4*>(base + (int64_t)(in ? q0 + v : 0) * items * kHeadDim);
          x[u][v] = in ? __ldcg(po) : make_float4(0.f, 0.f, 0.f, 0.f);
          y[u][v] = in ? __ldcg(po + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < kItemsPerThread; ++u) {
        const int it = it0 + tid + u * kThreads;
        const int j = it < G * 32 ? it >> 5 : 0;
#pragma unroll
        for (int v = 0; v < kPartsPerRound; ++v) {
          const float c = q0 + v < nparts ? wt[(q0 + v) * 16 + j] : 0.0f;
          acc[u][0] += c * x[u][v].x; acc[u][1] += c * x[u][v].y; acc[u][2] += c * x[u][v].z;
          acc[u][3] += c * x[u][v].w; acc[u][4] += c * y[u][v].x; acc[u][5] += c * y[u][v].y;
          acc[u][6] += c * y[u][v].z; acc[u][7] += c * y[u][v].w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kItemsPerThread; ++u) {
      const int it = it0 + tid + u * kThreads;
      if (it >= G * 32) continue;
      const int j = it >> 5, d8 = it & 31;
      float (&acc8)[8] = acc[u];
      const float den = head_den[j];
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc8[i] *= inv;
      const int head = kvh * G + j;
      if (out_mode == 0) {
        __nv_bfloat16* op = p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head + d8 * 8;
        uint32_t u4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          __nv_bfloat162 b = __floats2bfloat162_rn(acc8[2 * i], acc8[2 * i + 1]);
          u4[i] = *reinterpret_cast<uint32_t*>(&b);
        }
        if (p.vec_o) {
          *reinterpret_cast<uint4*>(op) = make_uint4(u4[0], u4[1], u4[2], u4[3]);
        } else {
          unsigned short* os = reinterpret_cast<unsigned short*>(op);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            os[2 * i] = (unsigned short)(u4[i] & 0xffffu);
            os[2 * i + 1] = (unsigned short)(u4[i] >> 16);
          }
        }
      } else {
        float4* op = reinterpret_cast<float4*>(f32_out + (w0 + j) * kHeadDim + d8 * 8);
        op[0] = make_float4(acc8[0], acc8[1], acc8[2], acc8[3]);
        op[1] = make_float4(acc8[4], acc8[5], acc8[6], acc8[7]);
        if (d8 == 0) f32_lse[w0 + j] = den > 0.0f ? head_m[j] + log2f(den) : -INFINITY;
      }
    }
    }
  }
}

// Split-KV across GPUs: this rank's merged (O, lse) of the unit sits in slot xrank of its own
// exchange buffer.  Push it into slot xrank of every other rank's buffer (NVLink stores), publish
// a flag per destination (release), wait for every other rank's flag (acquire, bounded by time),
// then merge the ranks' slots into the bf16 output and re-arm the flags of this parity.
__device__ __noinline__ void xrank_exchange(const AttnParams& p, float* scratch, int& status, int64_t row, int kvh,
                                            int G, int tid) {
  const int64_t items = p.rows * p.query_heads;
  const int64_t w0 = row * p.query_heads + (int64_t)kvh * G;
  const int64_t unit = row * p.kv_heads + kvh;
  const int64_t units = p.rows * p.kv_heads;
  const int world = p.xworld, me = p.xrank;
  auto lse_of = [&](float* base) { return base + (int64_t)world * items * kHeadDim; };
  auto flag_of = [&](float* base, int src) {
    return reinterpret_cast<unsigned int*>(lse_of(base) + (int64_t)world * items) +
           ((int64_t)p.xparity * units + unit) * world + src;
  };
  __syncthreads();  // this unit's slot-me stores by the CTA are complete
  float* mine = p.xpeer[me];
  const float4* src_o = reinterpret_cast<const float4*>(mine + ((int64_t)me * items + w0) * kHeadDim);
  const float* src_l = lse_of(mine) + (int64_t)me * items + w0;
  for (int r = 0; r < world; ++r) {
    if (r == me) continue;
    float4* dst_o = reinterpret_cast<float4*>(p.xpeer[r] + ((int64_t)me * items + w0) * kHeadDim);
    for (int i = tid; i < G * (kHeadDim / 4); i += kThreads) dst_o[i] = __ldcg(src_o + i);
    if (tid < G) lse_of(p.xpeer[r])[(int64_t)me * items + w0 + tid] = __ldcg(src_l + tid);
  }
  // Every thread's peer stores precede thread 0's release below in causality order (the barrier), so the
  // system-scope release store of each flag makes them visible to the peer that acquires the flag.
  __syncthreads();
  if (tid == 0) {
    for (int r = 0; r < world; ++r) {
      if (r == me) continue;
      asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(flag_of(p.xpeer[r], me)), "r"(1u) : "memory");
    }
    stamp_set(p, unit, 4);
    // Wait for every other rank's slot: bounded by time, so a rank that never arrives cannot hang the GPU.
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    int ok = 1;
    for (int r = 0; r < world && ok; ++r) {
      if (r == me) continue;
      unsigned int* f = flag_of(mine, r);
      while (true) {
        unsigned int v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(f) : "memory");
        if (v) break;
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > kPeerWaitNs) {
          ok = 0;
          atomicOr(&g_error_flags, kErrPeerTimeout);
          break;
        }
        __nanosleep(200);
      }
    }
    status = ok;
    stamp_set(p, unit, 5);
  }
  __syncthreads();
  if (!status) return;
  merge_unit_parts(p, scratch, row, kvh, G, tid, mine, lse_of(mine), world, 0, nullptr, nullptr);
  __syncthreads();
  if (tid < world) *flag_of(mine, tid) = 0u;  // re-arm this parity for the call after next
  if (tid == 0) stamp_set(p, unit, 6);
}

// Eight fp32 -> bf16 (round to nearest even) at op: one 16-byte store, or eight 2-byte stores.
__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* op, const float (&v)[8], int vec) {
  uint32_t u4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    u4[i] = *reinterpret_cast<uint32_t*>(&b2);
  }
  if (vec) {
    *reinterpret_cast<uint4*>(op) = make_uint4(u4[0], u4[1], u4[2], u4[3]);
  } else {
    unsigned short* os = reinterpret_cast<unsigned short*>(op);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      os[2 * i] = (unsigned short)(u4[i] & 0xffffu);
      os[2 * i + 1] = (unsigned short)(u4[i] >> 16);
    }
  }
}

// Split-KV beyond one cluster, merged by the last cluster: every cluster's ranks have stored their slices of
// the cluster's part (its normalised partial and lse); each fences them, rank 0 counts the cluster's arrival
// at the unit's counter and writes into every rank of its cluster whether it was the last; then each rank of
// the last cluster merges its slice of the unit's (head, 8 dims) items over all `nparts` parts -- one item per
// thread, eight parts' loads in flight -- and stores it, or, across GPUs, exchanges it and merges the GPUs.  Called by every thread of every rank of a
// cluster after the cluster merge (in place of its closing cluster barrier); `scratch` holds nparts * 16 + 32
// floats of shared memory.
__device__ __noinline__ void cluster_last_merge(const AttnParams& p, float* scratch, int* last, int64_t row, int kvh,
                                                int G, int tid, int split) {
  const int C = p.cluster, rank = split % C;
  const int nparts = p.splits / C;
  const int64_t unit = row * p.kv_heads + kvh;
  __threadfence();  // this rank's slice of the part is visible device-wide before the cluster's arrival
  cluster_sync();   // also: every rank keeps its shared memory until all ranks have read it
  if (rank == 0) {
    if (tid == 0) *last = atomicAdd(p.counters + unit, 1u) == (unsigned int)(nparts - 1) ? 1 : 0;
    __syncthreads();
    if (tid < C) cluster_st_s32(cluster_map(smem_u32(last), (uint32_t)tid), *last);
  }
  cluster_sync();  // every rank holds rank 0's verdict in its own shared memory
  if (!*last) return;
  if (rank == 0 && tid == 0) stamp_set(p, unit, 2);
  __threadfence();  // the other parts, counted before ours, are visible
  // every part's lse of this unit's heads, then per head its max, the weights 2^(lse - max) and their sum
  float* wt = scratch;                // [nparts][16]
  float* head_m = wt + nparts * 16;   // [16]
  float* head_den = head_m + 16;      // [16]
  const int64_t items = p.rows * p.query_heads;
  const int64_t w0 = row * p.query_heads + (int64_t)kvh * G;
  for (int i = tid; i < nparts * G; i += kThreads) {
    const int part = i / G, j = i - part * G;
    wt[part * 16 + j] = __ldcg(p.part_lse + (int64_t)part * items + w0 + j);
  }
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int part = 0; part < nparts; ++part) M = fmaxf(M, wt[part * 16 + tid]);
    float den = 0.0f;
    for (int part = 0; part < nparts; ++part) {
      const float l = wt[part * 16 + tid];
      const float x = (l == -INFINITY) ? 0.0f : exp2f(l - M);
      wt[part * 16 + tid] = x;
      den += x;
    }
    head_m[tid] = M;
    head_den[tid] = den;
  }
  __syncthreads();
  const int nitems = G * 32;
  const int it = rank * nitems / C + tid;
  const bool has_item = it < (rank + 1) * nitems / C;
  const int j = has_item ? it >> 5 : 0, d8 = it & 31;
  const int head = kvh * G + j;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float my_lse = -INFINITY;
  if (has_item) {
    const float* base = p.part_out + (w0 + j) * kHeadDim + d8 * 8;
    constexpr int kRound = 8;
    for (int q0 = 0; q0 < nparts; q0 += kRound) {
      float4 x[kRound], y[kRound];
#pragma unroll
      for (int v = 0; v < kRound; ++v) {
        const bool in = q0 + v < nparts;
        const float4* po = reinterpret_cast<const float4*>(base + (int64_t)(in ? q0 + v : 0) * items * kHeadDim);
        x[v] = in ? __ldcg(po) : make_float4(0.f, 0.f, 0.f, 0.f);
        y[v] = in ? __ldcg(po + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int v = 0; v < kRound; ++v) {
        const float cw = q0 + v < nparts ? wt[(q0 + v) * 16 + j] : 0.0f;
        acc[0] += cw * x[v].x; acc[1] += cw * x[v].y; acc[2] += cw * x[v].z; acc[3] += cw * x[v].w;
        acc[4] += cw * y[v].x; acc[5] += cw * y[v].y; acc[6] += cw * y[v].z; acc[7] += cw * y[v].w;
      }
    }
    const float den = head_den[j];
    const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
    my_lse = den > 0.0f ? head_m[j] + log2f(den) : -INFINITY;
  }
  if (p.xworld == 0) {
    if (has_item) {
      if (p.final_mode == 0) {
        __nv_bfloat16* op = p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head + d8 * 8;
        store_bf16x8(op, acc, p.vec_o);
      } else {
        float* op = p.final_out + (row * p.query_heads + head) * kHeadDim + d8 * 8;
        reinterpret_cast<float4*>(op)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        reinterpret_cast<float4*>(op)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        if (d8 == 0) p.final_lse[row * p.query_heads + head] = my_lse;
      }
    }
    if (tid == 0) {
      stamp_max(p, unit, 3);
      stamp_max(p, unit, 6);
    }
    return;
  }

  // ---- across GPUs: every rank of the last cluster pushes its slice of this GPU's merged (O, lse) into slot
  // xrank of every other GPU's exchange buffer; rank 0 publishes a flag per destination (release) and waits
  // for every other GPU's flag (acquire, bounded by time); then each rank merges its slice over the GPUs.
  if (tid == 0) stamp_max(p, unit, 3);
  const int world = p.xworld, me = p.xrank;
  const int64_t units = p.rows * p.kv_heads;
  float* mine = p.xpeer[me];
  auto lse_of = [&](float* b) { return b + (int64_t)world * items * kHeadDim; };
  auto flag_of = [&](float* b, int src) {
    return reinterpret_cast<unsigned int*>(lse_of(b) + (int64_t)world * items) +
           ((int64_t)p.xparity * units + unit) * world + src;
  };
  if (has_item) {
    for (int r = 0; r < world; ++r) {
      if (r == me) continue;
      float4* dst = reinterpret_cast<float4*>(p.xpeer[r] + ((int64_t)me * items + w0 + j) * kHeadDim + d8 * 8);
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      if (d8 == 0) lse_of(p.xpeer[r])[(int64_t)me * items + w0 + j] = my_lse;
    }
  }
  // Every thread's peer stores precede rank 0's system-scope release of the flags in causality order (the
  // cluster barrier), so each flag makes them visible to the GPU that acquires it.
  cluster_sync();
  if (rank == 0) {
    if (tid == 0) {
      for (int r = 0; r < world; ++r) {
        if (r == me) continue;
        asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(flag_of(p.xpeer[r], me)), "r"(1u) : "memory");
      }
      stamp_set(p, unit, 4);
      unsigned long long t0;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
      int ok = 1;
      for (int r = 0; r < world && ok; ++r) {
        if (r == me) continue;
        unsigned int* f = flag_of(mine, r);
        while (true) {
          unsigned int v;
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(f) : "memory");
          if (v) break;
          unsigned long long t;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
          if (t - t0 > kPeerWaitNs) {  // a GPU that never arrives cannot hang this one
            ok = 0;
            atomicOr(&g_error_flags, kErrPeerTimeout);
            break;
          }
          __nanosleep(200);
        }
      }
      *last = ok;
      stamp_set(p, unit, 5);
      for (int r = 0; r < world; ++r) *flag_of(mine, r) = 0u;  // re-arm this parity for the call after next
    }
    __syncthreads();
    if (tid < C) cluster_st_s32(cluster_map(smem_u32(last), (uint32_t)tid), *last);
  }
  cluster_sync();  // every rank holds rank 0's result of the wait, which acquired the other GPUs' slots
  if (!*last) return;
  if (has_item) {
    float lr[8];
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      lr[r] = -INFINITY;
      if (r < world) lr[r] = r == me ? my_lse : __ldcg(lse_of(mine) + (int64_t)r * items + w0 + j);
      M = fmaxf(M, lr[r]);
    }
    float out[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float den = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (r >= world) break;
      const float w = lr[r] == -INFINITY ? 0.0f : exp2f(lr[r] - M);
      den += w;
      if (r == me) {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] += w * acc[i];
      } else {
        const float4* src = reinterpret_cast<const float4*>(mine + ((int64_t)r * items + w0 + j) * kHeadDim + d8 * 8);
        const float4 a = __ldcg(src), b = __ldcg(src + 1);
        out[0] += w * a.x; out[1] += w * a.y; out[2] += w * a.z; out[3] += w * a.w;
        out[4] += w * b.x; out[5] += w * b.y; out[6] += w * b.z; out[7] += w * b.w;
      }
    }
    const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] *= inv;
    store_bf16x8(p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head + d8 * 8, out, p.vec_o);
  }
  if (tid == 0) stamp_max(p, unit, 6);
}

// Split-KV beyond one cluster: every part (one per cluster, its rank 0) has written its
// normalised partial and lse to the workspace; the last part to arrive at the unit's
// counter merges all parts.  Called by every thread of the CTA.
// `arrivals`: CTAs that arrive per unit -- every CTA when each stores a slice of its cluster's part (the
// distributed cluster merge), one per part when a part's rank 0 stores it whole.
__device__ __noinline__ void fused_part_merge(const AttnParams& p, float* scratch, int& last, int64_t row, int kvh,
                                              int G, int tid, int arrivals) {
  const int nparts = p.splits / p.cluster;
  __threadfence();  // this CTA's share of its part is visible device-wide before its arrival is counted
  __syncthreads();
  if (tid == 0) last = atomicAdd(p.counters + (row * p.kv_heads + kvh), 1u) == (unsigned int)(arrivals - 1);
  __syncthreads();
  if (!last) return;
  const int64_t unit = row * p.kv_heads + kvh;
  if (tid == 0) stamp_set(p, unit, 2);
  __threadfence();  // the other parts, counted before ours, are visible
  merge_unit_parts(p, scratch, row, kvh, G, tid, p.part_out, p.part_lse, nparts, p.final_mode, p.final_out,
                   p.final_lse);
  __syncthreads();
  if (tid == 0) stamp_set(p, unit, 3);
  if (p.xworld > 0) xrank_exchange(p, scratch, last, row, kvh, G, tid);
  else if (tid == 0) stamp_set(p, unit, 6);
}

// Split-KV merge inside a thread-block cluster of C CTAs, by threads of every rank.  Each CTA has
// published its (O, m, l) in its own shared memory: accumulator float4 i (NFRAG of them) of slot q
// (SLOTS of them) at comb[i * 64 + q], slot q's (m_r, m_r8, l_r, l_r8) at comb[NFRAG * 64 + q].  Float4
// (i, q) holds, for lane (r, c) = (q & 31) / 4, (q & 31) % 4, dims D = 128 h + 32 c + k and D + 16 of
// heads r and r + 8, where (h, k) = (i / 16, i % 16) when SLOTS = 32 (full-width reader) and (q / 32, i)
// when SLOTS = 64 (warp pairs); so the 16 float4 of one (q, h) run cover 16 consecutive dims.  Work units
// are GE consecutive float4 of a run (GE = 8, 4, 2 for clusters of <= 2, 4, 8), numbered run-fastest so that
// consecutive threads read consecutive slots of a rank; rank r takes the units [128 (r + kC), 128 (r + kC) + 128),
// k = 0, 1, ...; a unit loads its run's (m, l) and its GE float4 from every rank over distributed shared memory (all in
// flight together), weights them by 2^(m_rank - max) and stores the merged, normalised dims as vectors
// (bf16 output, or the fp32 partial and its lse).  Returns false (nothing stored) when a rank aborted.
template <int NFRAG, int SLOTS, int GE>
__device__ __forceinline__ void cluster_merge_units(const AttnParams& p, uint32_t base, int64_t row, int kvh, int G,
                                                    int tid, int split) {
  const int C = p.cluster, rank = split % C;
  constexpr int kGroups = 16 / GE;
  constexpr int kRanks = 16 / GE;       // largest cluster this unit width serves (C <= kRanks)
  constexpr int kUnits = 64 * kGroups;  // (q, h) runs: 32 lanes x 2 halves, or 64 slots
  for (int u = rank * kThreads + tid; u < kUnits; u += C * kThreads) {
    const int run = u % 64, g = u / 64;  // consecutive threads read consecutive slots of a rank
    const int q = SLOTS == 32 ? run >> 1 : run;
    const int h = SLOTS == 32 ? run & 1 : q >> 5;
    const int i0 = (SLOTS == 32 ? 16 * h : 0) + g * GE;
    float4 ml[kRanks], o[kRanks][GE];
#pragma unroll
    for (int rk = 0; rk < kRanks; ++rk) {
      if (rk < C) {
        const uint32_t rb = cluster_map(base, (uint32_t)rk);
        ml[rk] = cluster_ld_f4(rb + (uint32_t)(NFRAG * 64 + q) * 16u);
#pragma unroll
        for (int e = 0; e < GE; ++e) o[rk][e] = cluster_ld_f4(rb + (uint32_t)((i0 + e) * 64 + q) * 16u);
      }
    }
    float Ma = -INFINITY, Mb = -INFINITY;
#pragma unroll
    for (int rk = 0; rk < kRanks; ++rk)
      if (rk < C) { Ma = fmaxf(Ma, ml[rk].x); Mb = fmaxf(Mb, ml[rk].y); }
    float La = 0.f, Lb = 0.f;
    float va[2][GE], vb[2][GE];  // [dim block (D, D + 16)][e] for head r (a) and r + 8 (b)
#pragma unroll
    for (int e = 0; e < GE; ++e) va[0][e] = va[1][e] = vb[0][e] = vb[1][e] = 0.0f;
#pragma unroll
    for (int rk = 0; rk < kRanks; ++rk) {
      if (rk < C) {
        const float wa = ex2(ml[rk].x - Ma), wb = ex2(ml[rk].y - Mb);
        La += wa * ml[rk].z;
        Lb += wb * ml[rk].w;
#pragma unroll
        for (int e = 0; e < GE; ++e) {
          va[0][e] += wa * o[rk][e].x; va[1][e] += wa * o[rk][e].y;
          vb[0][e] += wb * o[rk][e].z; vb[1][e] += wb * o[rk][e].w;
        }
      }
    }
    const int ln = q & 31, r = ln >> 2, c = ln & 3;
    const int D = 128 * h + 32 * c + (i0 & 15);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = r + 8 * hh;
      if (j >= G) continue;
      const float L = hh ? Lb : La, M = hh ? Mb : Ma;
      // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
      const float inv = L > 0.0f ? p.inv_value_scale / fmaxf(L, 1.0e-20f) : 0.0f;
      float(&v)[2][GE] = hh ? vb : va;
      const int head = kvh * G + j;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const int d0 = D + 16 * blk;
        if (p.mode == 0) {
          __nv_bfloat16* op = p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head + d0;
          uint32_t w[GE / 2];
#pragma unroll
          for (int e = 0; e < GE / 2; ++e) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[blk][2 * e] * inv, v[blk][2 * e + 1] * inv);
            w[e] = *reinterpret_cast<uint32_t*>(&b2);
          }
          if (p.vec_o && GE == 8) {
            *reinterpret_cast<uint4*>(op) = make_uint4(w[0], w[1 % (GE / 2)], w[2 % (GE / 2)], w[3 % (GE / 2)]);
          } else if (p.vec_o && GE == 4) {
            *reinterpret_cast<uint2*>(op) = make_uint2(w[0], w[1 % (GE / 2)]);
          } else {
            unsigned short* os = reinterpret_cast<unsigned short*>(op);
#pragma unroll
            for (int e = 0; e < GE / 2; ++e) {
              os[2 * e] = (unsigned short)(w[e] & 0xffffu);
              os[2 * e + 1] = (unsigned short)(w[e] >> 16);
            }
          }
        } else {
          const int64_t slot = ((int64_t)(split / C) * p.rows + row) * p.query_heads + head;
          float* op = p.part_out + slot * kHeadDim + d0;
#pragma unroll
          for (int e = 0; e < GE; e += 2) *reinterpret_cast<float2*>(op + e) = make_float2(v[blk][e] * inv, v[blk][e + 1] * inv);
          if (d0 == 0) p.part_lse[slot] = L > 0.0f ? M + log2f(fmaxf(L, 1.0e-20f)) : -INFINITY;
        }
      }
    }
  }
}

template <int NFRAG, int SLOTS>
__device__ __noinline__ bool cluster_merge_store(const AttnParams& p, const float4* comb, int64_t row, int kvh,
                                                 int G, int tid, int split, const int* abort_flag) {
  const int C = p.cluster;
  // every rank published its abort flag before the caller's cluster barrier: thread rk reads rank rk's, all at once
  const int bad = tid < C ? cluster_ld_s32(cluster_map(smem_u32(abort_flag), (uint32_t)tid)) : 0;
  if (__syncthreads_or(bad)) return false;  // the same for every thread
  const uint32_t base = smem_u32(comb);
  if (C <= 2) cluster_merge_units<NFRAG, SLOTS, 8>(p, base, row, kvh, G, tid, split);
  else if (C <= 4) cluster_merge_units<NFRAG, SLOTS, 4>(p, base, row, kvh, G, tid, split);
  else cluster_merge_units<NFRAG, SLOTS, 2>(p, base, row, kvh, G, tid, split);
  return true;
}

// GMODE: how records reach shared memory (0: tile::gather4 rows; 1: one bulk copy per
// record; 2: four bulk copies per record), fixed per launch so the hot loop carries no
// mode branches.
template <int GMODE>
__global__ void __launch_bounds__(kThreads, 3) sparse_attention_kernel(const __grid_constant__ AttnParams p) {
  pdl_enter();
  constexpr bool kFp8 = GMODE == kGatherFp8;
  constexpr int kStages = kFp8 ? kFp8Stages : kWarpStages;
  constexpr int kAh = kStages - 1;
  using SM = SmemT<kFp8 ? kFp8RecordBytes : kRecordBytes, kStages>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // Tensor copies need 128-byte aligned destinations: align the base explicitly.
  SM& sm = *reinterpret_cast<SM*>(smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u));
  // Byte offset of token t inside a stage: the permuted NVFP4 rows, or plain FP8 slots.
  auto soff = [](int t) { return kFp8 ? t * kFp8RecordBytes : slot_off(t); };

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int r = lane >> 2;  // mma group row
  const int c = lane & 3;   // mma thread-in-group

  int64_t bid = blockIdx.x;
  const int split = (int)(bid % p.splits);
  bid /= p.splits;
  const int kvh = (int)(bid % p.kv_heads);
  const int64_t row = bid / p.kv_heads;
  if (tid == 0) stamp_min(p, row * p.kv_heads + kvh, 0);

  const int64_t chunks = (p.topk + kChunk - 1) / kChunk;
  const int my_chunks = split < chunks ? (int)((chunks - 1 - split) / p.splits + 1) : 0;  // <= kMaxChunks
  const int G = p.group;

  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < kStages; ++b) mbar_init(smem_u32(&sm.full_bar[warp][b]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (tid == 0) sm.abort = 0;

  // ---------------- prologue: all independent global loads first ----------------
  // Selection indices of this CTA's chunks (chunk split + lc * splits, lc = it * kWarps + warp).
  const int32_t req = __ldg(p.token_to_request + row);
  const int32_t* idx_row = p.indices + row * p.topk;
  const int iters = (my_chunks + kWarps - 1) / kWarps;
  int32_t iv[kCompactIters];
#pragma unroll
  for (int it = 0; it < kCompactIters; ++it) {
    const int lc = it * kWarps + warp;
    const int64_t pos = ((int64_t)split + (int64_t)lc * p.splits) * kChunk + lane;
    iv[it] = (lc < my_chunks && pos < p.topk) ? __ldg(idx_row + pos) : -1;
  }
  // Query heads warp, warp + 4, warp + 8, warp + 12 of this kv head; lane L holds dims [8L, 8L + 8).
  uint32_t qw[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = warp + kWarps * i;
    qw[i][0] = qw[i][1] = qw[i][2] = qw[i][3] = 0u;
    if (j < G) {
      const __nv_bfloat16* qrow = p.q + row * p.q_stride_row + (int64_t)(kvh * G + j) * p.q_stride_head + lane * 8;
      if (p.vec_q) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(qrow));
        qw[i][0] = v.x; qw[i][1] = v.y; qw[i][2] = v.z; qw[i][3] = v.w;
      } else {
        const unsigned short* qs = reinterpret_cast<const unsigned short*>(qrow);
#pragma unroll
        for (int t = 0; t < 4; ++t) qw[i][t] = (uint32_t)__ldg(qs + 2 * t) | ((uint32_t)__ldg(qs + 2 * t + 1) << 16);
      }
    }
  }
  // Block-table entries of the selections (kernels.py:236-257 masking).
  const bool req_ok = req >= 0 && (int64_t)req < p.num_requests;
  const int32_t* bt_row = p.block_table + (req_ok ? (int64_t)req * p.table_width : 0);
  // 0 <= idx < 2^31: a 32-bit division (a page larger than that holds every index in page 0)
  const bool huge_page = p.page_size > 0x7fffffffLL;
  int32_t phys[kCompactIters], offs[kCompactIters];
#pragma unroll
  for (int it = 0; it < kCompactIters; ++it) {
    phys[it] = -1;
    offs[it] = 0;
    const int32_t idx = iv[it];
    if (req_ok && idx >= 0) {
      const uint32_t lpage = huge_page ? 0u : (uint32_t)idx / (uint32_t)p.page_size;
      if ((int64_t)lpage < p.table_width) {
        phys[it] = __ldg(bt_row + lpage);
        offs[it] = huge_page ? idx : (int)((uint32_t)idx - lpage * (uint32_t)p.page_size);
      }
    }
  }

  // ---------------- Q: per-head power-of-two pre-scale (exact) into f16 mma fragments ----------------
  // Fragment k-step ks, lane (r, c): a0a1 = Q[r][d, d+1], a2a3 = Q[r+8][d, d+1], a4a5 = Q[r][d+2, d+3],
  // a6a7 = Q[r+8][d+2, d+3] with d the first dim of k-step ks for thread-in-group c; heads >= G stay zero.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = warp + kWarps * i;
    uint32_t amax = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t)
      amax = max(amax, max((qw[i][t] << 16) & 0x7fffffffu, qw[i][t] & 0x7fff0000u));
#pragma unroll
    for (int m = 16; m; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    int e = 0;
    if (amax != 0 && amax < 0x7f800000u) {
      e = 14 - ilogbf(__uint_as_float(amax));
      e = max(-126, min(126, e));
    }
    if (lane == 0) sm.smul[j] = ldexpf(p.score_scale, -e);
    const float mul = ldexpf(1.0f, e);
    const int hh = j >> 3, rr = j & 7;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int d = 8 * lane + 4 * g;
      const int cc = (d & 127) >> 5;
      const int ks = ((d & 31) >> 2) + ((d >> 7) << 3);
      uint32_t* f = reinterpret_cast<uint32_t*>(&sm.qfrag[ks][4 * rr + cc]);
      const uint32_t x0 = qw[i][2 * g], x1 = qw[i][2 * g + 1];
      f[hh] = pack_half2(bf16_lo(x0) * mul, bf16_hi(x0) * mul);
      f[2 + hh] = pack_half2(bf16_lo(x1) * mul, bf16_hi(x1) * mul);
    }
  }

  // ---------------- compact the valid selections ----------------
  uint32_t vmask = 0;
  int pre[kCompactIters];
#pragma unroll
  for (int it = 0; it < kCompactIters; ++it) {
    pre[it] = 0;
    if (it < iters) {
      const bool valid = phys[it] >= 0 && (int64_t)phys[it] < p.num_blocks;
      const uint32_t b = __ballot_sync(0xffffffffu, valid);
      pre[it] = __popc(b & ((1u << lane) - 1u));
      if (valid) vmask |= 1u << it;
      if (lane == 0) sm.cnt[it][warp] = __popc(b);
    }
  }
  __syncthreads();  // exponents, fragments and per-warp counts visible
  {
    int base_all = 0;
#pragma unroll
    for (int it = 0; it < kCompactIters; ++it) {
      if (it < iters) {
        int base = base_all;
        for (int w = 0; w < warp; ++w) base += sm.cnt[it][w];
        if (vmask & (1u << it)) sm.sel[base + pre[it]] = make_int2(phys[it], offs[it]);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) base_all += sm.cnt[it][w];
      }
    }
    if (tid == 0) sm.total = base_all;
  }
  __syncthreads();
  const int n = sm.total;
  const int ntiles = (n + kTile - 1) / kTile;

  // ---------------- per-warp gather pipeline: tiles warp, warp+4, ... ----------------
  const uint8_t* const reg0 = p.region[0];
  const int64_t sb0 = p.stride[0][0], st0 = p.stride[0][1], sh0 = p.stride[0][2];
  auto issue_tile = [&](int k) {  // local tile k of this warp -> ring slot k % kStages
    const int tile = warp + kWarps * k;
    const int slot = k % kStages;
    const uint32_t bar = smem_u32(&sm.full_bar[warp][slot]);
    const int j0 = tile * kTile;
    const int count = min(kTile, n - j0);
    // The slot was last read by this warp's generic loads: order them before the async-proxy writes.
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    if constexpr (GMODE == 0) {
      if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)kStageBytes);
      __syncwarp();
      if (lane < kTile / 4) {
        int32_t rows[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = group_token(lane, j);
          rows[j] = p.total_rows;  // out of range: zero fill
          if (t < count) {
            const int2 e = sm.sel[j0 + t];
            rows[j] = (e.x * p.kv_heads + kvh) * (int32_t)p.page_size + e.y;
          }
        }
        gather4_g2s(smem_u32(&sm.rec[warp][slot][lane * 4 * kRecordBytes]), &p.rows_map, rows[0], rows[1], rows[2],
                    rows[3], bar);
      }
      return;
    }
    if constexpr (GMODE == kGatherPlain) {
      // Synchronous plain loads: the warp copies the tile's records region by region, copy_width bytes per
      // lane and step, then completes the slot's barrier phase with a plain arrive.
      const int w = p.copy_width;
      for (int t = 0; t < count; ++t) {
        const int2 e = sm.sel[j0 + t];
        uint8_t* d = sm.rec[warp][slot] + soff(t);
        const uint32_t dofs[4] = {0, 128, 144, 272};
        const int size[4] = {128, 16, 128, 16};
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint8_t* src = p.region[g] + (int64_t)e.x * p.stride[g][0] + (int64_t)e.y * p.stride[g][1] +
                               (int64_t)kvh * p.stride[g][2];
          for (int b = lane * w; b < size[g]; b += 32 * w) {
            if (w == 8) *reinterpret_cast<uint2*>(d + dofs[g] + b) = __ldg(reinterpret_cast<const uint2*>(src + b));
            else if (w == 4) *reinterpret_cast<uint32_t*>(d + dofs[g] + b) = __ldg(reinterpret_cast<const uint32_t*>(src + b));
            else if (w == 2) *reinterpret_cast<uint16_t*>(d + dofs[g] + b) = __ldg(reinterpret_cast<const uint16_t*>(src + b));
            else d[dofs[g] + b] = __ldg(src + b);
          }
        }
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
      return;
    }
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(count * (kFp8 ? 2 * kHeadDim : kRecordBytes)));
    __syncwarp();
    if (lane < count) {
      const int2 e = sm.sel[j0 + lane];
      const uint32_t dst = smem_u32(&sm.rec[warp][slot][soff(lane)]);
      if constexpr (GMODE == 1) {
        bulk_g2s(dst, reg0 + (int64_t)e.x * sb0 + (int64_t)e.y * st0 + (int64_t)kvh * sh0, kRecordBytes, bar);
      } else if constexpr (kFp8) {  // K row of cache region 0, V row of region 2
        bulk_g2s(dst, reg0 + (int64_t)e.x * sb0 + (int64_t)e.y * st0 + (int64_t)kvh * sh0, kHeadDim, bar);
        bulk_g2s(dst + kHeadDim,
                 p.region[2] + (int64_t)e.x * p.stride[2][0] + (int64_t)e.y * p.stride[2][1] +
                     (int64_t)kvh * p.stride[2][2],
                 kHeadDim, bar);
      } else {
        const uint32_t dofs[4] = {0, 128, 144, 272};
        const uint32_t size[4] = {128, 16, 128, 16};
#pragma unroll
        for (int g = 0; g < 4; ++g)
          bulk_g2s(dst + dofs[g],
                   p.region[g] + (int64_t)e.x * p.stride[g][0] + (int64_t)e.y * p.stride[g][1] +
                       (int64_t)kvh * p.stride[g][2],
                   size[g], bar);
      }
    }
  };
  const int my_tiles = ntiles > warp ? (ntiles - warp + kWarps - 1) / kWarps : 0;
#pragma unroll
  for (int k = 0; k < kAh; ++k)
    if (k < my_tiles) issue_tile(k);

  // Per-lane constants: K bytes of token 8*nt + r (chunks c and 4+c), V tokens {2c, 2c+1, 2c+8, 2c+9}.
  int k_off[2], v_off[4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) k_off[nt] = soff(8 * nt + r);
  {
    const int tt[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
    for (int q = 0; q < 4; ++q) v_off[q] = soff(tt[q]);
  }
  const float smul_r = sm.smul[r];
  const float smul_r8 = sm.smul[r + 8];

  float oacc[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;
  float m_r = kMaskedScore, m_r8 = kMaskedScore;
  float l_r = 0.0f, l_r8 = 0.0f;

  // One tile of 16 tokens at `stage`; TAIL masks tokens at or past n (only a warp's last tile can be short).
  auto tile_body = [&](const uint8_t* stage, const int tok_base, auto tail_tag) {
    constexpr bool TAIL = decltype(tail_tag)::value;

    // ---- S = Q K^T: 16 k-steps over all 256 dims, each on both n-tiles of 8 tokens ----
    float sacc[2][4];
    if constexpr (kFp8) {
      // FP8: one byte per dim; k-step s takes dims d..d+3 of the permuted order (d = 32c + 4s, +128 past
      // s = 7), i.e. word s of the lane's 32 K bytes of its half, converted exactly to f16 pairs (the K
      // scale is folded into the score scale).
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint4 kq[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint8_t* kr = stage + k_off[nt] + 128 * half + 32 * c;
          kq[nt][0] = *reinterpret_cast<const uint4*>(kr);
          kq[nt][1] = *reinterpret_cast<const uint4*>(kr + 16);
        }
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          const uint4 qa = sm.qfrag[8 * half + s2][lane];
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const uint4 v = kq[nt][s2 >> 2];
            const uint32_t word = (s2 & 3) == 0 ? v.x : (s2 & 3) == 1 ? v.y : (s2 & 3) == 2 ? v.z : v.w;
            mma_f16(sacc[nt], qa.x, qa.y, qa.z, qa.w, cvt_e4m3x2_f16x2(word & 0xffffu), cvt_e4m3x2_f16x2(word >> 16));
          }
        }
      }
    } else {
    uint32_t sg[2][4];  // f16x2 group scales {lo, hi} x {chunk c, chunk 4+c}, duplicated per half
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint8_t* rec = stage + k_off[nt];
      const uint32_t sc0 = cvt_e4m3x2_f16x2(*reinterpret_cast<const uint16_t*>(rec + 128 + 2 * c));
      const uint32_t sc1 = cvt_e4m3x2_f16x2(*reinterpret_cast<const uint16_t*>(rec + 136 + 2 * c));
      sg[nt][0] = dup_lo(sc0);
      sg[nt][1] = dup_hi(sc0);
      sg[nt][2] = dup_lo(sc1);
      sg[nt][3] = dup_hi(sc1);
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // k-steps 8*half .. 8*half+7: chunk c (half 0) or 4+c (half 1)
      uint4 kq[2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) kq[nt] = *reinterpret_cast<const uint4*>(stage + k_off[nt] + 64 * half + 16 * c);
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        const int s = 8 * half + s2;
        const uint4 qa = sm.qfrag[s][lane];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint32_t word = (s2 >> 1) == 0 ? kq[nt].x : (s2 >> 1) == 1 ? kq[nt].y : (s2 >> 1) == 2 ? kq[nt].z : kq[nt].w;
          const uint32_t scl = sg[nt][2 * half + (s2 >> 2)];
          uint32_t b0, b1;
          if (s2 & 1) {
            b0 = hmul2_u32(cvt_e2m1x2_f16x2_byte<2>(word), scl);
            b1 = hmul2_u32(cvt_e2m1x2_f16x2_byte<3>(word), scl);
          } else {
            b0 = hmul2_u32(cvt_e2m1x2_f16x2_byte<0>(word), scl);
            b1 = hmul2_u32(cvt_e2m1x2_f16x2_byte<1>(word), scl);
          }
          mma_f16(sacc[nt], qa.x, qa.y, qa.z, qa.w, b0, b1);
        }
      }
    }
    }  // NVFP4 S

    // ---- online softmax (base 2): p = 2^(s * smul - m) with one FFMA ----
    uint32_t pf[4];
    {
      if constexpr (TAIL) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int t0 = tok_base + 8 * nt + 2 * c;
          if (t0 >= n) { sacc[nt][0] = -1.0e30f; sacc[nt][2] = -1.0e30f; }
          if (t0 + 1 >= n) { sacc[nt][1] = -1.0e30f; sacc[nt][3] = -1.0e30f; }
        }
      }
      float mx_r = fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1]));
      float mx_r8 = fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3]));
      mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 1));
      mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 2));
      mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 1));
      mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 2));
      mx_r *= smul_r;  // smul > 0 (global scales are positive): max commutes with the scale
      mx_r8 *= smul_r8;
      const bool up_r = mx_r > m_r + kRescaleThreshold;
      const bool up_r8 = mx_r8 > m_r8 + kRescaleThreshold;
      if (__any_sync(0xffffffffu, up_r || up_r8)) {
        const float mn_r = up_r ? mx_r : m_r, mn_r8 = up_r8 ? mx_r8 : m_r8;
        const float a_r = ex2(m_r - mn_r), a_r8 = ex2(m_r8 - mn_r8);
        m_r = mn_r;
        m_r8 = mn_r8;
        l_r *= a_r;
        l_r8 *= a_r8;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          oacc[i][0] *= a_r; oacc[i][1] *= a_r;
          oacc[i][2] *= a_r8; oacc[i][3] *= a_r8;
        }
      }
      float pv[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pv[nt][0] = ex2(fmaf(sacc[nt][0], smul_r, -m_r));
        pv[nt][1] = ex2(fmaf(sacc[nt][1], smul_r, -m_r));
        pv[nt][2] = ex2(fmaf(sacc[nt][2], smul_r8, -m_r8));
        pv[nt][3] = ex2(fmaf(sacc[nt][3], smul_r8, -m_r8));
      }
      if constexpr (TAIL) {  // masked scores must not count even while the running max is still -1e20
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int t0 = tok_base + 8 * nt + 2 * c;
          if (t0 >= n) { pv[nt][0] = 0.0f; pv[nt][2] = 0.0f; }
          if (t0 + 1 >= n) { pv[nt][1] = 0.0f; pv[nt][3] = 0.0f; }
        }
      }
      l_r += (pv[0][0] + pv[0][1]) + (pv[1][0] + pv[1][1]);
      l_r8 += (pv[0][2] + pv[0][3]) + (pv[1][2] + pv[1][3]);
      pf[0] = pack_half2(pv[0][0], pv[0][1]);
      pf[1] = pack_half2(pv[0][2], pv[0][3]);
      pf[2] = pack_half2(pv[1][0], pv[1][1]);
      pf[3] = pack_half2(pv[1][2], pv[1][3]);
    }

    // ---- O += P V: 32 n-tiles of 8 dims; half h covers dims [128h, 128h+128) ----
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if constexpr (kFp8) {
        // FP8: lane (r, c) takes the 16 V bytes of dims 128h + 16r + [0, 16) of tokens {2c, 2c+1, 2c+8, 2c+9};
        // n-tile 16h + 8kk + 2B + x, column r <-> dim 128h + 16r + 8kk + 2B + x as in the NVFP4 path, so the
        // epilogue stores both alike.  A byte permute pairs the two tokens of each operand.
        uint4 vq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) vq[q] = *reinterpret_cast<const uint4*>(stage + v_off[q] + kHeadDim + 128 * h + 16 * r);
        if constexpr (TAIL) {  // stale slots past the last valid token: zero V so that 0 * V stays 0
          const int tt[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (tok_base + tt[q] >= n) vq[q] = make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
          for (int B = 0; B < 4; ++B) {
            const int wi = 2 * kk + (B >> 1), pb = 2 * (B & 1);
            const uint32_t sel = (uint32_t)(pb | ((pb + 4) << 4) | ((pb + 1) << 8) | ((pb + 5) << 12));
            auto word = [&](const uint4& v) { return wi == 0 ? v.x : wi == 1 ? v.y : wi == 2 ? v.z : v.w; };
            const uint32_t u01 = __byte_perm(word(vq[0]), word(vq[1]), sel);
            const uint32_t u23 = __byte_perm(word(vq[2]), word(vq[3]), sel);
            const int nt = 16 * h + 8 * kk + 2 * B;
            mma_f16(oacc[nt], pf[0], pf[1], pf[2], pf[3], cvt_e4m3x2_f16x2(u01 & 0xffffu),
                    cvt_e4m3x2_f16x2(u23 & 0xffffu));
            mma_f16(oacc[nt + 1], pf[0], pf[1], pf[2], pf[3], cvt_e4m3x2_f16x2(u01 >> 16), cvt_e4m3x2_f16x2(u23 >> 16));
          }
        }
        continue;
      }
      uint2 vw[4];
      uint32_t vsb[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint8_t* rec = stage + v_off[q];
        vw[q] = *reinterpret_cast<const uint2*>(rec + 144 + 64 * h + 8 * r);
        vsb[q] = rec[272 + 8 * h + r];
      }
      if constexpr (TAIL && GMODE != 0) {  // stale slots past the last valid token: zero V so that 0 * V stays 0
        const int tt[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (tok_base + tt[q] >= n) {
            vw[q] = make_uint2(0u, 0u);
            vsb[q] = 0u;
          }
        }
      }
      const uint32_t s01 = cvt_e4m3x2_f16x2(vsb[0] | (vsb[1] << 8));
      const uint32_t s23 = cvt_e4m3x2_f16x2(vsb[2] | (vsb[3] << 8));
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint32_t w0 = kk ? vw[0].y : vw[0].x, w1 = kk ? vw[1].y : vw[1].x;
        const uint32_t w2 = kk ? vw[2].y : vw[2].x, w3 = kk ? vw[3].y : vw[3].x;
        // low nibbles (even dims) of two tokens interleaved into one byte
        const uint32_t x01 = (w0 & 0x0f0f0f0fu) | ((w1 & 0x0f0f0f0fu) << 4);
        const uint32_t y01 = ((w0 >> 4) & 0x0f0f0f0fu) | (w1 & 0xf0f0f0f0u);
        const uint32_t x23 = (w2 & 0x0f0f0f0fu) | ((w3 & 0x0f0f0f0fu) << 4);
        const uint32_t y23 = ((w2 >> 4) & 0x0f0f0f0fu) | (w3 & 0xf0f0f0f0u);
#define NVQSA_PV_BYTE(B)                                                                               \
  {                                                                                                    \
    const int nt = 16 * h + 8 * kk + 2 * (B);                                                          \
    mma_f16(oacc[nt], pf[0], pf[1], pf[2], pf[3], hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(x01), s01),        \
            hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(x23), s23));                                            \
    mma_f16(oacc[nt + 1], pf[0], pf[1], pf[2], pf[3], hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(y01), s01),    \
            hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(y23), s23));                                            \
  }
        NVQSA_PV_BYTE(0)
        NVQSA_PV_BYTE(1)
        NVQSA_PV_BYTE(2)
        NVQSA_PV_BYTE(3)
#undef NVQSA_PV_BYTE
      }
    }
  };

  int k = 0;
  for (; k < my_tiles; ++k) {
    if (k + kAh < my_tiles) issue_tile(k + kAh);  // into the slot tile k-1 used
    const int slot = k % kStages;
    if (!mbar_wait(smem_u32(&sm.full_bar[warp][slot]), (uint32_t)((k / kStages) & 1))) {
      if (lane == 0) sm.abort = 1;
      break;
    }
    const int tok_base = (warp + kWarps * k) * kTile;  // compacted index of the tile's first token
    const uint8_t* stage = sm.rec[warp][slot];
    if (tok_base + kTile <= n)
      tile_body(stage, tok_base, std::false_type{});
    else
      tile_body(stage, tok_base, std::true_type{});
    __syncwarp();  // every lane's reads of this slot precede its refill
  }

  // ---------------- combine the four warps, normalise, store ----------------
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 1);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 2);

  if (k < my_tiles) {
    // This warp gave up: let its copies still in flight land (bounded) before the
    // CTA's shared memory can be released.
    for (int k2 = k + 1; k2 < my_tiles && k2 <= k + kAh; ++k2)
      mbar_wait(smem_u32(&sm.full_bar[warp][k2 % kStages]), (uint32_t)((k2 / kStages) & 1), kDrainSpinLimit);
  }
  __syncthreads();  // every warp left its loop: no bulk copy is in flight, the rings are free
  if (tid == 0) stamp_max(p, row * p.kv_heads + kvh, 1);
  const bool aborted = sm.abort != 0;
  if (aborted && p.cluster <= 1) return;  // a cluster CTA still takes the cluster barriers below

  // Two rounds over shared memory: warps 2,3 -> 0,1, then warp 1 -> 0.  Slot q = sender * 32 + lane;
  // float4 i of slot q at comb[i * 64 + q], so that a warp's stores and loads are contiguous.
  float4* comb = reinterpret_cast<float4*>(&sm.rec[0][0][0]);   // [32][64] float4 + [64] (m, m8, l, l8)
  float4* comb_ml = comb + 32 * 64;
#pragma unroll
  for (int round = 0; round < 2; ++round) {
    if (aborted) break;  // CTA-uniform
    const int senders = round == 0 ? 2 : 1;  // warps [senders, 2*senders) send to warp - senders
    if (warp >= senders && warp < 2 * senders) {
      const int q = (warp - senders) * 32 + lane;
#pragma unroll
      for (int i = 0; i < 32; ++i) comb[i * 64 + q] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
      comb_ml[q] = make_float4(m_r, m_r8, l_r, l_r8);
    }
    __syncthreads();
    if (warp < senders) {
      const int q = warp * 32 + lane;
      const float4 ml = comb_ml[q];
      const float M_r = fmaxf(m_r, ml.x), M_r8 = fmaxf(m_r8, ml.y);
      const float a0 = ex2(m_r - M_r), b0 = ex2(ml.x - M_r);
      const float a1 = ex2(m_r8 - M_r8), b1 = ex2(ml.y - M_r8);
      l_r = l_r * a0 + ml.z * b0;
      l_r8 = l_r8 * a1 + ml.w * b1;
      m_r = M_r;
      m_r8 = M_r8;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float4 v = comb[i * 64 + q];
        oacc[i][0] = oacc[i][0] * a0 + v.x * b0;
        oacc[i][1] = oacc[i][1] * a0 + v.y * b0;
        oacc[i][2] = oacc[i][2] * a1 + v.z * b1;
        oacc[i][3] = oacc[i][3] * a1 + v.w * b1;
      }
    }
    __syncthreads();
  }

  if (p.cluster > 2) {
    // Split-KV inside a thread-block cluster (the CTA's rank is its split): every CTA publishes warp 0's
    // (O, m, l) in its own shared memory; then threads of every rank merge and store one slice each.
    if (warp == 0 && !aborted) {
#pragma unroll
      for (int i = 0; i < 32; ++i) comb[i * 64 + lane] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
      comb_ml[lane] = make_float4(m_r, m_r8, l_r, l_r8);
    }
    cluster_sync();
    const bool ok = cluster_merge_store<32, 32>(p, comb, row, kvh, G, tid, split, &sm.abort);
    if (p.fuse && ok) {  // the last cluster to arrive merges the parts (and exchanges them), a slice per rank
      cluster_last_merge(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), &sm.last, row, kvh, G, tid, split);
      return;
    }
    cluster_sync();  // every rank keeps its shared memory until all ranks have read it; slices are stored
    if (!ok) return;
    if (p.fuse) {
      fused_part_merge(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid, p.splits);
    } else if (p.xworld > 0 && split % p.cluster == 0) {
      xrank_exchange(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid);
    } else if (tid == 0 && split % p.cluster == 0) {
      stamp_set(p, row * p.kv_heads + kvh, 6);
    }
    return;
  }
  if (p.cluster == 2) {
    // A pair of CTAs: warp 0 of rank 0 reads its peer's (O, m, l) over distributed shared memory (one
    // round of loads) and stores the merged result like an unsplit CTA.
    if (warp == 0 && !aborted) {
#pragma unroll
      for (int i = 0; i < 32; ++i) comb[i * 64 + lane] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
      comb_ml[lane] = make_float4(m_r, m_r8, l_r, l_r8);
    }
    cluster_sync();
    bool ok = !aborted && cluster_ld_s32(cluster_map(smem_u32(&sm.abort), 1u ^ (uint32_t)(split & 1))) == 0;
    if ((split & 1) == 0 && warp == 0 && ok) {
      const uint32_t cb = cluster_map(smem_u32(comb), 1u);
      const float4 ml = cluster_ld_f4(cb + (uint32_t)(32 * 64 + lane) * 16u);
      const float M_r = fmaxf(m_r, ml.x), M_r8 = fmaxf(m_r8, ml.y);
      const float a0 = ex2(m_r - M_r), b0 = ex2(ml.x - M_r);
      const float a1 = ex2(m_r8 - M_r8), b1 = ex2(ml.y - M_r8);
      l_r = l_r * a0 + ml.z * b0;
      l_r8 = l_r8 * a1 + ml.w * b1;
      m_r = M_r;
      m_r8 = M_r8;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float4 v = cluster_ld_f4(cb + (uint32_t)(i * 64 + lane) * 16u);
        oacc[i][0] = oacc[i][0] * a0 + v.x * b0;
        oacc[i][1] = oacc[i][1] * a0 + v.y * b0;
        oacc[i][2] = oacc[i][2] * a1 + v.z * b1;
        oacc[i][3] = oacc[i][3] * a1 + v.w * b1;
      }
    }
    cluster_sync();  // rank 1 keeps its shared memory until rank 0 has read it
    if ((split & 1) != 0 || !ok) return;  // rank 0 carries on with the pair's merged (O, m, l)
  }

  if (warp == 0) {
    // lane (r, c) holds dims 128*h + 32c + i (oacc[16h + i][2hh]) and +16 (oacc[16h + i][2hh + 1]).
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = r + 8 * hh;
      if (j >= G) continue;
      const float l = hh ? l_r8 : l_r;
      const float m = hh ? m_r8 : m_r;
      // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
      const float inv = l > 0.0f ? p.inv_value_scale / fmaxf(l, 1.0e-20f) : 0.0f;
      const int head = kvh * G + j;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[i] = oacc[16 * h + i][2 * hh] * inv;
          v[16 + i] = oacc[16 * h + i][2 * hh + 1] * inv;
        }
        const int d0 = 128 * h + 32 * c;
        if (p.mode == 0) {
          __nv_bfloat16* op = p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head + d0;
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&b);
          }
          if (p.vec_o) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              reinterpret_cast<uint4*>(op)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          } else {
            unsigned short* os = reinterpret_cast<unsigned short*>(op);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              os[2 * i] = (unsigned short)(w[i] & 0xffffu);
              os[2 * i + 1] = (unsigned short)(w[i] >> 16);
            }
          }
        } else {
          const int64_t slot = ((int64_t)(split / p.cluster) * p.rows + row) * p.query_heads + head;
          float* op = p.part_out + slot * kHeadDim + d0;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<float4*>(op)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          if (h == 0 && c == 0) p.part_lse[slot] = l > 0.0f ? m + log2f(fmaxf(l, 1.0e-20f)) : -INFINITY;
        }
      }
    }
  }

  // ---------------- split-KV beyond one cluster: the last part to arrive merges all parts ----------------
  if (!p.fuse) {
    if (p.xworld > 0) xrank_exchange(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid);
    return;
  }
  fused_part_merge(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid, p.splits / p.cluster);
}

// One warp per (row, query head): log-sum-exp merge of `splits` partials, split s
// at part_out + s * out_split_stride ([rows][heads][256] dense) and
// part_lse + s * lse_split_stride ([rows][heads] dense).
// mode 0 -> bf16 output; mode 1 -> fp32 normalised output + merged lse.
__global__ void __launch_bounds__(256) merge_kernel(MergeArgs a, int64_t rows, int query_heads) {
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= rows * query_heads) return;
  const int64_t row = w / query_heads;
  merge_item(a, row, (int)(w - row * query_heads), w, lane);
}

#include "sparse_attention_bf16.cuh"
#include "sparse_attention_pair.cuh"
#include "sparse_attention_mtp.cuh"

// ---------------- host-side planning ----------------
// 2D tensor map viewing the cache records as rows [rows, 144] of u16 (288 bytes),
// box 144 x 1 as tile::gather4 requires.  Encoded through the driver entry point
// (no link-time libcuda dependency) and cached per (device, base, rows).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct MapCacheEntry {
  int device;
  const void* base;
  int64_t rows;
  CUtensorMap map;
};
constexpr int kMapCacheSize = 32;
MapCacheEntry g_map_cache[kMapCacheSize];
int g_map_cache_used = 0, g_map_cache_next = 0;

bool record_map(const void* base, int64_t rows, CUtensorMap* out) {
  static EncodeTiledFn encode = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    looked_up = true;
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  if (!encode) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  for (int i = 0; i < g_map_cache_used; ++i)
    if (g_map_cache[i].device == dev && g_map_cache[i].base == base && g_map_cache[i].rows == rows) {
      *out = g_map_cache[i].map;
      return true;
    }
  CUtensorMap map;
  const cuuint64_t dims[2] = {kRecordBytes / 2, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {kRecordBytes};
  const cuuint32_t box[2] = {kRecordBytes / 2, 1};
  const cuuint32_t elem[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  MapCacheEntry& slot = g_map_cache[g_map_cache_next];
  slot = MapCacheEntry{dev, base, rows, map};
  g_map_cache_next = (g_map_cache_next + 1) % kMapCacheSize;
  if (g_map_cache_used < kMapCacheSize) ++g_map_cache_used;
  *out = map;
  return true;
}

constexpr int kMaxDevicesStamps = 64;
constexpr int kReaderCtasPerSm = 3;  // resident CTAs per SM of the full-width reader (registers and shared memory)
constexpr int kBf16CtasPerSm = 2;    // resident CTAs per SM of the BF16 sibling reader (shared memory)

struct Plan {
  int splits;
  bool pair;    // fewer (row, kv head) units than SMs: the warp-pair reader (lower latency per tile)
  int cluster;  // splits of one (row, kv head) merged inside a cluster of this size (1: no cluster)
};
constexpr int kMaxClusterSplits = 8;  // portable thread-block cluster size

// Split plan.  Each CTA pays a fixed prologue (selection resolution, Q
// fragments) and epilogue (warp combine, partial write), so CTAs stay long: a
// batch with at least one (row, kv head) unit per SM keeps the fewest splits
// the 1024-selection CTA limit allows; batches with fewer units than SMs are
// split until every SM has a CTA, down to one 32-position chunk per CTA.
Plan make_plan(int64_t rows, int kv_heads, int64_t topk, int sms, int ctas_per_sm = kReaderCtasPerSm) {
  Plan pl;
  const int64_t units = rows * kv_heads;
  const int64_t chunks = topk > 0 ? (topk + kChunk - 1) / kChunk : 1;
  const int64_t min_splits = (chunks + kMaxChunks - 1) / kMaxChunks;
  int64_t splits = min_splits;
  const int64_t sm_count = sms > 0 ? sms : 148;
  if (units > 0 && units < sm_count) {
    splits = (sm_count + units - 1) / units;
  } else if (units > 0) {
    // Up to as many splits as keep every SM's resident CTAs busy in one wave, rounded down to a power of two:
    // clusters of 3 do not pack onto the GPCs (measured on B200 at 148 units: 3 splits in clusters of 3
    // 71.5 us, 2 splits 46.3 us per 2,048-selection layer).
    int64_t fill = (ctas_per_sm * sm_count) / units;
    while (fill & (fill - 1)) fill &= fill - 1;
    if (fill > splits) splits = fill;
  }
  if (splits > chunks) splits = chunks;
  if (splits < min_splits) splits = min_splits;
  // Beyond one cluster: a multiple of 8 splits in clusters of 8, whose rank-0 parts merge globally
  // (CTAs past the last chunk contribute empty parts).
  if (splits > kMaxClusterSplits) splits = (splits + kMaxClusterSplits - 1) / kMaxClusterSplits * kMaxClusterSplits;
  pl.splits = (int)splits;
  pl.cluster = splits > 1 ? (int)std::min<int64_t>(splits, kMaxClusterSplits) : 1;
  // With at least one unit per SM the grid fills the GPU, and clusters of a size that is not a power of two
  // leave SMs idle (same measurement, 3 splits without a cluster: 51.2 us): merge those parts globally.
  if (units >= sm_count && (pl.cluster & (pl.cluster - 1)) != 0) pl.cluster = 1;
  pl.pair = units > 0 && units < sm_count;
  return pl;
}

// Grouped (MTP) reader plan: groups of rows_per_group consecutive rows, each split into one cluster of
// at most 8 CTAs (each CTA at most 1024 selections); the most splits whose clusters are all resident at
// once (cap[s]: resident clusters of s CTAs on this device, or the SM count when unknown): a group's tiles
// are processed in order by its CTA, so more splits mean shorter chains, but clusters that do not fit on
// the GPCs run as a second wave.
struct MtpPlan {
  bool use;
  int splits;
  int64_t grid;
};
MtpPlan make_mtp_plan(int64_t rows, int kv_heads, int64_t topk, int G, int rows_per_group, int sms,
                      const int* cap) {
  MtpPlan mp{false, 1, 0};
  if (rows_per_group < 2 || rows_per_group * G > kMtpHeads || topk < 1) return mp;
  const int64_t units = (rows + rows_per_group - 1) / rows_per_group * kv_heads;
  const int64_t chunks = (topk + kChunk - 1) / kChunk;
  const int64_t min_splits = (chunks + kMaxChunks - 1) / kMaxChunks;
  if (min_splits > kMtpMaxCluster) return mp;
  const int64_t target = sms > 0 ? sms : 148;
  int64_t splits = min_splits;
  for (int64_t s = min_splits + 1; s <= kMtpMaxCluster && s <= chunks; ++s) {
    const int c = cap ? cap[s] : 0;
    if (c > 0 ? units <= c : units * s <= target) splits = s;
  }
  if (units * splits > 0x7fffffffLL) return mp;
  mp.use = true;
  mp.splits = (int)splits;
  mp.grid = units * splits;
  return mp;
}

// Workspace of a split launch: partial outputs [splits][rows][heads][256] fp32,
// partial lse [splits][rows][heads] fp32 (padded to 256 bytes), then one
// arrival counter per (row, kv head), zeroed on the launch's stream.
struct Workspace {
  size_t lse_offset, counter_offset, bytes;
};
Workspace workspace_layout(const Plan& pl, int64_t rows, int query_heads, int kv_heads) {
  Workspace w{0, 0, 0};
  if (pl.splits <= pl.cluster) return w;  // unsplit, or merged inside one cluster
  const size_t items = (size_t)(pl.splits / pl.cluster) * rows * query_heads;
  w.lse_offset = items * kHeadDim * sizeof(float);
  w.counter_offset = w.lse_offset + ((items * sizeof(float) + 255) / 256) * 256;
  w.bytes = w.counter_offset + (size_t)rows * kv_heads * sizeof(unsigned int);
  return w;
}
size_t workspace_for(const Plan& pl, int64_t rows, int query_heads, int kv_heads) {
  return workspace_layout(pl, rows, query_heads, kv_heads).bytes;
}

// Timing stamp buffer of each device (nvqsa_set_stamp_buffer), handed to every reader launch; nullptr: off.
std::atomic<unsigned long long*> g_stamps[kMaxDevicesStamps] = {};

// Dynamic shared memory above 48 KB is opted into once per device.
constexpr int kMaxDevices = 64;
bool smem_configured[kMaxDevices] = {};

// The reader kernel of a launch (full-width, warp-pair, FP8 or BF16 sibling) with its shared-memory size.
struct ReaderKernel {
  const void* fn;
  size_t smem;  // + slack for the 128-byte alignment of the base
};
ReaderKernel reader_kernel(int gather_mode, bool pair) {
  if (gather_mode == kGatherBf16)
    return {reinterpret_cast<const void*>(sparse_attention_bf16_kernel), sizeof(SmemBf) + 128};
  if (gather_mode == kGatherFp8)
    return {reinterpret_cast<const void*>(sparse_attention_kernel<kGatherFp8>), sizeof(SmemFp8) + 128};
  if (gather_mode == kGatherPlain)
    return {reinterpret_cast<const void*>(sparse_attention_kernel<kGatherPlain>), sizeof(Smem) + 128};
  if (pair) {
    switch (gather_mode) {
      case 0: return {reinterpret_cast<const void*>(sparse_attention_pair_kernel<0>), sizeof(SmemPair<0>) + 128};
      case 1: return {reinterpret_cast<const void*>(sparse_attention_pair_kernel<1>), sizeof(SmemPair<1>) + 128};
      default: return {reinterpret_cast<const void*>(sparse_attention_pair_kernel<2>), sizeof(SmemPair<2>) + 128};
    }
  }
  switch (gather_mode) {
    case 0: return {reinterpret_cast<const void*>(sparse_attention_kernel<0>), sizeof(Smem) + 128};
    case 1: return {reinterpret_cast<const void*>(sparse_attention_kernel<1>), sizeof(Smem) + 128};
    default: return {reinterpret_cast<const void*>(sparse_attention_kernel<2>), sizeof(Smem) + 128};
  }
}

// Dynamic shared memory above 48 KB is opted into once per device and kernel.
int configure_smem() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return NVQSA_ERR_CUDA;
  if (!smem_configured[dev]) {
    for (int k = 0; k < 9; ++k) {
      const ReaderKernel rk = k == 8   ? reader_kernel(kGatherPlain, false)
                              : k == 7 ? reader_kernel(kGatherBf16, false)
                              : k == 6 ? reader_kernel(kGatherFp8, false)
                                       : reader_kernel(k % 3, k >= 3);
      if (cudaFuncSetAttribute(rk.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rk.smem) != cudaSuccess ||
          cudaFuncSetAttribute(rk.fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
        return NVQSA_ERR_CUDA;
    }
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(sparse_attention_mtp_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sizeof(SmemMtp) + 128)) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(sparse_attention_mtp_kernel),
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(sparse_attention_mtp_kernel),
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return NVQSA_ERR_CUDA;
    smem_configured[dev] = true;
  }
  return NVQSA_OK;
}

// Resident clusters of s grouped-reader CTAs (s = 1..8) on each device, queried once; -1 when unknown.
std::atomic<int> g_mtp_capacity[kMaxDevices][kMtpMaxCluster + 1] = {};
int mtp_cluster_capacity(int s) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  int v = g_mtp_capacity[dev][s].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)s, 1, 1);
    cfg.blockDim = dim3(kMtpThreads, 1, 1);
    cfg.dynamicSmemBytes = sizeof(SmemMtp) + 128;
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeClusterDimension;
    a.val.clusterDim.x = (unsigned)s;
    a.val.clusterDim.y = 1;
    a.val.clusterDim.z = 1;
    cfg.attrs = &a;
    cfg.numAttrs = 1;
    if (configure_smem() != NVQSA_OK ||
        cudaOccupancyMaxActiveClusters(&v, reinterpret_cast<const void*>(sparse_attention_mtp_kernel), &cfg) !=
            cudaSuccess ||
        v <= 0) {
      (void)cudaGetLastError();
      v = -1;
    }
    g_mtp_capacity[dev][s].store(v, std::memory_order_relaxed);
  }
  return v;
}

int run_attention(const void* query, int64_t q_stride_row, int64_t q_stride_head, const void* const region[4],
                  const int64_t strides[4][3], int64_t num_blocks, int64_t page_size, int32_t kv_heads,
                  float key_global_scale, float value_global_scale, const int32_t* logical_indices, int64_t topk,
                  const int32_t* block_table, int64_t num_requests, int64_t table_width,
                  const int32_t* token_to_request, void* output, int64_t o_stride_row, int64_t o_stride_head,
                  float* partial_out, float* partial_lse, int64_t rows, int32_t query_heads, int32_t head_dim,
                  void* workspace, size_t workspace_bytes, void* stream, float* const* xpeers = nullptr,
                  int32_t xworld = 0, int32_t xrank = 0, int32_t xparity = 0, int32_t rows_per_group = 1,
                  bool fp8 = false, bool bf16 = false) {
  if (rows < 0 || topk < 0 || kv_heads < 1 || query_heads < 1 || num_blocks < 0 || page_size < 1 ||
      num_requests < 0 || table_width < 0)
    return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  // Global scales must be finite and positive (the reference PackedCache rule, cache.py:16-17).
  if (!(key_global_scale > 0.0f) || !(value_global_scale > 0.0f) || key_global_scale > 3.0e38f ||
      value_global_scale > 3.0e38f)
    return NVQSA_ERR_BAD_SHAPE;
  if (query_heads % kv_heads) return NVQSA_ERR_UNSUPPORTED;
  const int G = query_heads / kv_heads;
  if (G < 1 || G > 16) return NVQSA_ERR_UNSUPPORTED;
  if (rows == 0) return NVQSA_OK;
  const bool partial_mode = partial_out != nullptr;
  if (!query || !token_to_request || (!output && !partial_mode) || (partial_mode && !partial_lse))
    return NVQSA_ERR_NULL_POINTER;
  if (topk > 0 && !logical_indices) return NVQSA_ERR_NULL_POINTER;
  // The widest power of two (<= 16 bytes) dividing every region base and stride: 16 allows TMA and bulk
  // copies; narrower layouts (NVFP4 only) take plain loads of that width.
  int align = 16;
  for (int i = 0; i < 4; ++i) {
    if (!region[i]) return NVQSA_ERR_NULL_POINTER;
    while (align > 1 && !aligned_to(region[i], (uintptr_t)align)) align >>= 1;
    for (int j = 0; j < 3; ++j)
      while (align > 1 && strides[i][j] % align) align >>= 1;
  }
  if (align < 16 && (fp8 || bf16)) return NVQSA_ERR_MISALIGNED;  // the sibling readers keep the 16-byte rule
  if (!aligned_to(query, 2) || (partial_mode ? !aligned_to(partial_out, 16) || !aligned_to(partial_lse, 4)
                                             : !aligned_to(output, 2)))
    return NVQSA_ERR_MISALIGNED;

  const int sms = device_sm_count();
  if (sms <= 0) return NVQSA_ERR_CUDA;
  if (rows_per_group < 1 || rows_per_group > kMtpRows) return NVQSA_ERR_BAD_SHAPE;
  const bool sibling = fp8 || bf16;
  int cap[kMtpMaxCluster + 1] = {};
  if (!sibling && rows_per_group >= 2)
    for (int s = 1; s <= kMtpMaxCluster; ++s) cap[s] = mtp_cluster_capacity(s);
  const MtpPlan mp =
      sibling ? MtpPlan{false, 1, 0} : make_mtp_plan(rows, kv_heads, topk, G, rows_per_group, sms, cap);
  Plan pl = mp.use ? Plan{} : make_plan(rows, kv_heads, topk, sms, bf16 ? kBf16CtasPerSm : kReaderCtasPerSm);
  if (sibling) pl.pair = false;  // the FP8 and BF16 rows run on their full-width readers only
  const Workspace wl = mp.use ? Workspace{0, 0, 0} : workspace_layout(pl, rows, query_heads, kv_heads);
  const size_t need = wl.bytes;
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned_to(workspace, 16))) return NVQSA_ERR_WORKSPACE;
  if (!mp.use && (int64_t)pl.splits * rows * kv_heads > 0x7fffffffLL) return NVQSA_ERR_BAD_SHAPE;
  // The last part's merge keeps one weight per (part, head) in the CTA's ring space.
  if (!mp.use && (size_t)(pl.splits / pl.cluster) * 16 * sizeof(float) + 128 > sizeof(Smem::rec))
    return NVQSA_ERR_UNSUPPORTED;

  AttnParams p;
  p.stamps = nullptr;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevicesStamps)
      p.stamps = g_stamps[dev].load(std::memory_order_relaxed);
  }
  p.q = static_cast<const __nv_bfloat16*>(query);
  p.q_stride_row = q_stride_row;
  p.q_stride_head = q_stride_head;
  for (int i = 0; i < 4; ++i) {
    p.region[i] = static_cast<const uint8_t*>(region[i]);
    for (int j = 0; j < 3; ++j) p.stride[i][j] = strides[i][j];
  }
  p.num_blocks = num_blocks;
  p.page_size = page_size;
  p.kv_heads = kv_heads;
  {
    // The reference layout (cache.py:20-24) stores each (block, head, token) as one
    // contiguous record K data | K scale | V data | V scale.
    const uint8_t* b = p.region[0];
    bool rec = p.region[1] == b + 128 && p.region[2] == b + 144 && p.region[3] == b + 272;
    for (int i = 1; i < 4 && rec; ++i)
      for (int j = 0; j < 3; ++j) rec = rec && p.stride[i][j] == p.stride[0][j];
    p.gather_mode = rec ? 1 : 2;
    p.total_rows = 0;
    p.copy_width = align >= 8 ? 8 : align;
    if (align < 16) p.gather_mode = kGatherPlain;
    // Canonical storage [blocks, kv_heads, page, 288]: records are rows of one matrix.
    const int64_t rows = num_blocks * kv_heads * page_size;
    if (align == 16 && rec && p.stride[0][1] == kRecordBytes && p.stride[0][2] == page_size * kRecordBytes &&
        p.stride[0][0] == kv_heads * page_size * kRecordBytes && rows > 0 && rows < 0x7fffffffLL &&
        record_map(b, rows, &p.rows_map)) {
      p.gather_mode = 0;
      p.total_rows = (int32_t)rows;
    }
  }
  p.group = G;
  p.query_heads = query_heads;
  p.score_scale = (float)(0.0625 * 1.4426950408889634) * (1.0f / key_global_scale);
  p.inv_value_scale = 1.0f / value_global_scale;
  if (fp8) {
    // FP8 sibling reader (src/qsa_fp8_harness.py:101-102, :175): the per-tensor k_scale multiplies the
    // scores, v_scale the normalised output; regions 0 and 2 are the K and V caches.
    p.gather_mode = kGatherFp8;
    p.total_rows = 0;
    p.score_scale = (float)(0.0625 * 1.4426950408889634) * key_global_scale;
    p.inv_value_scale = value_global_scale;
  }
  if (bf16) {
    // BF16 sibling reader (integration/snapshot/qsa.py:352-366): plain bf16 K and V, scale head_dim^-0.5;
    // regions 0 and 2 are the K and V caches.
    p.gather_mode = kGatherBf16;
    p.total_rows = 0;
    p.score_scale = (float)(0.0625 * 1.4426950408889634);
    p.inv_value_scale = 1.0f;
  }
  p.indices = logical_indices;
  p.topk = topk;
  p.block_table = block_table;
  p.num_requests = num_requests;
  p.table_width = table_width;
  p.token_to_request = token_to_request;
  p.rows = rows;
  p.splits = pl.splits;
  p.group_rows = 1;
  p.vec_q = (aligned_to(query, 16) && q_stride_row % 8 == 0 && q_stride_head % 8 == 0) ? 1 : 0;
  p.vec_o = (!partial_mode && aligned_to(output, 16) && o_stride_row % 8 == 0 && o_stride_head % 8 == 0) ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(output);
  p.o_stride_row = o_stride_row;
  p.o_stride_head = o_stride_head;
  p.fuse = 0;
  p.cluster = pl.cluster;
  p.xworld = xworld;
  p.xrank = xrank;
  p.xparity = xparity;
  for (int r = 0; r < 8; ++r) p.xpeer[r] = (xpeers && r < xworld) ? xpeers[r] : nullptr;
  if (xworld > 0) {
    // This rank's merged (O, lse) goes to slot xrank of its own exchange buffer first.
    const int64_t items = rows * query_heads;
    partial_out = p.xpeer[xrank] + (int64_t)xrank * items * kHeadDim;
    partial_lse = p.xpeer[xrank] + (int64_t)xworld * items * kHeadDim + (int64_t)xrank * items;
  }
  const bool to_f32 = partial_mode || xworld > 0;
  p.final_mode = to_f32 ? 1 : 0;
  p.counters = nullptr;
  p.final_out = partial_out;
  p.final_lse = partial_lse;
  if (pl.splits > 1 && pl.splits == pl.cluster) {  // one cluster per unit: its rank 0 stores like an unsplit CTA
    p.mode = to_f32 ? 1 : 0;
    p.part_out = partial_out;
    p.part_lse = partial_lse;
  } else if (pl.splits > 1) {  // several parts per unit (one per cluster) merged by the last to arrive
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    p.mode = 1;
    p.fuse = 1;
    p.part_out = reinterpret_cast<float*>(ws);
    p.part_lse = reinterpret_cast<float*>(ws + wl.lse_offset);
    p.counters = reinterpret_cast<unsigned int*>(ws + wl.counter_offset);
  } else if (to_f32) {
    p.mode = 1;
    p.part_out = partial_out;
    p.part_lse = partial_lse;
  } else {
    p.mode = 0;
    p.part_out = nullptr;
    p.part_lse = nullptr;
  }

  if (const int st = configure_smem()) return st;
  if (mp.use && p.gather_mode == 0 && p.mode == 0 && xworld == 0 && !p.fuse) {
    // grouped reader: the splits of a group form one cluster, merged in shared memory
    p.splits = mp.splits;
    p.cluster = mp.splits;
    p.group_rows = rows_per_group;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)mp.grid, 1, 1);
    cfg.blockDim = dim3(kMtpThreads, 1, 1);
    cfg.dynamicSmemBytes = sizeof(SmemMtp) + 128;
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[2], cluster_attr;
    cluster_attr.id = cudaLaunchAttributeClusterDimension;
    cluster_attr.val.clusterDim.x = (unsigned)mp.splits;
    cluster_attr.val.clusterDim.y = 1;
    cluster_attr.val.clusterDim.z = 1;
    int nattr = 0;
    if (mp.splits > 1) attr[nattr++] = cluster_attr;
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr++].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (unsigned)nattr;
    void* args[1] = {&p};
    if (cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(sparse_attention_mtp_kernel), args) != cudaSuccess)
      return NVQSA_ERR_LAUNCH;
    if (cudaGetLastError() != cudaSuccess) return NVQSA_ERR_LAUNCH;
    return NVQSA_OK;
  }
  if (mp.use) {
    // not eligible after all (layout, output mode): the per-row reader with its own plan
    return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads,
                         key_global_scale, value_global_scale, logical_indices, topk, block_table, num_requests,
                         table_width, token_to_request, output, o_stride_row, o_stride_head, partial_out, partial_lse,
                         rows, query_heads, head_dim, workspace, workspace_bytes, stream, xpeers, xworld, xrank,
                         xparity, 1);
  }
  if (p.gather_mode == kGatherPlain) pl.pair = false;  // plain loads run on the full-width reader only
  const ReaderKernel rk = reader_kernel(p.gather_mode, pl.pair);
  cudaStream_t s = as_stream(stream);
  if (p.fuse && cudaMemsetAsync(p.counters, 0, (size_t)rows * kv_heads * sizeof(unsigned int), s) != cudaSuccess)
    return NVQSA_ERR_LAUNCH;
  const int64_t grid = (int64_t)pl.splits * rows * kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = rk.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2], cluster_attr;
  cluster_attr.id = cudaLaunchAttributeClusterDimension;
  cluster_attr.val.clusterDim.x = (unsigned)pl.cluster;
  cluster_attr.val.clusterDim.y = 1;
  cluster_attr.val.clusterDim.z = 1;
  int nattr = 0;
  if (pl.cluster > 1) attr[nattr++] = cluster_attr;
  if (xworld == 0) {  // the cross-GPU exchange keeps plain stream order
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr++].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = (unsigned)nattr;
  void* args[1] = {&p};
  if (cudaLaunchKernelExC(&cfg, rk.fn, args) != cudaSuccess) return NVQSA_ERR_LAUNCH;
  if (cudaGetLastError() != cudaSuccess) return NVQSA_ERR_LAUNCH;
  return NVQSA_OK;
}

}  // namespace
}  // namespace nvqsa

using namespace nvqsa;

namespace nvqsa {
int write_error_flags(unsigned int* v, bool clear);  // write_cache.cu: the projection writer's flags
}

extern "C" int nvqsa_read_error_flags(uint32_t* flags, int clear) {
  if (!flags) return NVQSA_ERR_NULL_POINTER;
  unsigned int v = 0, wv = 0;
  if (cudaMemcpyFromSymbol(&v, g_error_flags, sizeof(v)) != cudaSuccess) return NVQSA_ERR_CUDA;
  const int ws = nvqsa::write_error_flags(&wv, clear != 0);
  if (ws != NVQSA_OK) return ws;
  *flags = v | wv;
  if (clear && v) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_error_flags, &zero, sizeof(zero)) != cudaSuccess) return NVQSA_ERR_CUDA;
  }
  return NVQSA_OK;
}

extern "C" int nvqsa_set_stamp_buffer(void* stamps) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevicesStamps) return NVQSA_ERR_CUDA;
  if (stamps && !aligned_to(stamps, 8)) return NVQSA_ERR_MISALIGNED;
  g_stamps[dev].store(static_cast<unsigned long long*>(stamps), std::memory_order_relaxed);
  return NVQSA_OK;
}

extern "C" int nvqsa_sparse_attention_workspace_size(int64_t rows, int32_t query_heads, int32_t kv_heads,
                                                     int32_t head_dim, int64_t topk, size_t* workspace_bytes) {
  if (!workspace_bytes) return NVQSA_ERR_NULL_POINTER;
  *workspace_bytes = 0;
  if (rows < 0 || topk < 0 || kv_heads < 1 || query_heads < 1) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  if (rows == 0) return NVQSA_OK;
  const int sms = device_sm_count();
  if (sms <= 0) return NVQSA_ERR_CUDA;
  *workspace_bytes = workspace_for(make_plan(rows, kv_heads, topk, sms), rows, query_heads, kv_heads);
  return NVQSA_OK;
}

extern "C" int nvqsa_sparse_attention(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream) {
  const void* region[4] = {key_data, key_scale, value_data, value_scale};
  const int64_t strides[4][3] = {{kd_stride_block, kd_stride_token, kd_stride_head},
                                 {ks_stride_block, ks_stride_token, ks_stride_head},
                                 {vd_stride_block, vd_stride_token, vd_stride_head},
                                 {vs_stride_block, vs_stride_token, vs_stride_head}};
  return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads,
                       key_global_scale, value_global_scale, logical_indices, topk, block_table, num_requests,
                       table_width, token_to_request, output, o_stride_row, o_stride_head, nullptr, nullptr, rows,
                       query_heads, head_dim, workspace, workspace_bytes, stream);
}

extern "C" int nvqsa_sparse_attention_grouped(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim, int32_t rows_per_group,
    void* workspace, size_t workspace_bytes, void* stream) {
  const void* region[4] = {key_data, key_scale, value_data, value_scale};
  const int64_t strides[4][3] = {{kd_stride_block, kd_stride_token, kd_stride_head},
                                 {ks_stride_block, ks_stride_token, ks_stride_head},
                                 {vd_stride_block, vd_stride_token, vd_stride_head},
                                 {vs_stride_block, vs_stride_token, vs_stride_head}};
  return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads,
                       key_global_scale, value_global_scale, logical_indices, topk, block_table, num_requests,
                       table_width, token_to_request, output, o_stride_row, o_stride_head, nullptr, nullptr, rows,
                       query_heads, head_dim, workspace, workspace_bytes, stream, nullptr, 0, 0, 0, rows_per_group);
}

extern "C" int nvqsa_sparse_attention_fp8(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_cache, int64_t kc_stride_block, int64_t kc_stride_token, int64_t kc_stride_head,
    const void* value_cache, int64_t vc_stride_block, int64_t vc_stride_token, int64_t vc_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads, float k_scale, float v_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream) {
  const void* region[4] = {key_cache, key_cache, value_cache, value_cache};
  const int64_t strides[4][3] = {{kc_stride_block, kc_stride_token, kc_stride_head},
                                 {kc_stride_block, kc_stride_token, kc_stride_head},
                                 {vc_stride_block, vc_stride_token, vc_stride_head},
                                 {vc_stride_block, vc_stride_token, vc_stride_head}};
  return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads, k_scale,
                       v_scale, logical_indices, topk, block_table, num_requests, table_width, token_to_request,
                       output, o_stride_row, o_stride_head, nullptr, nullptr, rows, query_heads, head_dim, workspace,
                       workspace_bytes, stream, nullptr, 0, 0, 0, 1, true);
}

extern "C" int nvqsa_sparse_attention_bf16(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_cache, int64_t kc_stride_block, int64_t kc_stride_token, int64_t kc_stride_head,
    const void* value_cache, int64_t vc_stride_block, int64_t vc_stride_token, int64_t vc_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream) {
  const void* region[4] = {key_cache, key_cache, value_cache, value_cache};
  const int64_t strides[4][3] = {{kc_stride_block, kc_stride_token, kc_stride_head},
                                 {kc_stride_block, kc_stride_token, kc_stride_head},
                                 {vc_stride_block, vc_stride_token, vc_stride_head},
                                 {vc_stride_block, vc_stride_token, vc_stride_head}};
  return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads, 1.0f,
                       1.0f, logical_indices, topk, block_table, num_requests, table_width, token_to_request, output,
                       o_stride_row, o_stride_head, nullptr, nullptr, rows, query_heads, head_dim, workspace,
                       workspace_bytes, stream, nullptr, 0, 0, 0, 1, false, true);
}

extern "C" int nvqsa_sparse_attention_bf16_workspace_size(int64_t rows, int32_t query_heads, int32_t kv_heads,
                                                         int32_t head_dim, int64_t topk, size_t* workspace_bytes) {
  if (!workspace_bytes) return NVQSA_ERR_NULL_POINTER;
  *workspace_bytes = 0;
  if (rows < 0 || topk < 0 || kv_heads < 1 || query_heads < 1 || query_heads % kv_heads) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  if (rows == 0) return NVQSA_OK;
  const int sms = device_sm_count();
  if (sms <= 0) return NVQSA_ERR_CUDA;
  Plan pl = make_plan(rows, kv_heads, topk, sms, kBf16CtasPerSm);
  pl.pair = false;
  *workspace_bytes = workspace_for(pl, rows, query_heads, kv_heads);
  return NVQSA_OK;
}

extern "C" int nvqsa_sparse_attention_partial(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    float* partial_out, float* partial_lse,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream) {
  if (!partial_out || !partial_lse) return NVQSA_ERR_NULL_POINTER;
  const void* region[4] = {key_data, key_scale, value_data, value_scale};
  const int64_t strides[4][3] = {{kd_stride_block, kd_stride_token, kd_stride_head},
                                 {ks_stride_block, ks_stride_token, ks_stride_head},
                                 {vd_stride_block, vd_stride_token, vd_stride_head},
                                 {vs_stride_block, vs_stride_token, vs_stride_head}};
  return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads,
                       key_global_scale, value_global_scale, logical_indices, topk, block_table, num_requests,
                       table_width, token_to_request, nullptr, 0, 0, partial_out, partial_lse, rows, query_heads,
                       head_dim, workspace, workspace_bytes, stream);
}

extern "C" int nvqsa_split_kv_exchange_bytes(int64_t rows, int32_t query_heads, int32_t kv_heads, int32_t world,
                                             size_t* bytes) {
  if (!bytes) return NVQSA_ERR_NULL_POINTER;
  *bytes = 0;
  if (rows < 1 || query_heads < 1 || kv_heads < 1 || world < 1 || world > 8) return NVQSA_ERR_BAD_SHAPE;
  const size_t items = (size_t)rows * query_heads;
  *bytes = (size_t)world * items * (kHeadDim + 1) * sizeof(float) +
           (size_t)2 * rows * kv_heads * world * sizeof(unsigned int);
  return NVQSA_OK;
}

extern "C" int nvqsa_exchange_alloc(size_t bytes, void** ptr) {
  if (!ptr) return NVQSA_ERR_NULL_POINTER;
  *ptr = nullptr;
  if (bytes == 0) return NVQSA_ERR_BAD_SHAPE;
  // A dedicated allocation (its own IPC handle, offset 0), zeroed: every flag starts disarmed.
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return NVQSA_ERR_CUDA;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return NVQSA_ERR_CUDA;
  }
  return NVQSA_OK;
}

extern "C" int nvqsa_exchange_free(void* ptr) {
  if (!ptr) return NVQSA_OK;
  return cudaFree(ptr) == cudaSuccess ? NVQSA_OK : NVQSA_ERR_CUDA;
}

extern "C" int nvqsa_ipc_get_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return NVQSA_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return NVQSA_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return NVQSA_OK;
}

extern "C" int nvqsa_ipc_open_handle(const void* handle, void** ptr) {
  if (!handle || !ptr) return NVQSA_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? NVQSA_OK : NVQSA_ERR_CUDA;
}

extern "C" int nvqsa_ipc_close_handle(void* ptr) {
  if (!ptr) return NVQSA_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? NVQSA_OK : NVQSA_ERR_CUDA;
}

extern "C" int nvqsa_sparse_attention_split_kv(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes,
    void* const* exchange, int32_t world, int32_t rank, int32_t parity, void* stream) {
  if (!exchange || !output) return NVQSA_ERR_NULL_POINTER;
  if (world < 1 || world > 8 || rank < 0 || rank >= world || (parity != 0 && parity != 1)) return NVQSA_ERR_BAD_SHAPE;
  float* peers[8];
  for (int r = 0; r < world; ++r) {
    if (!exchange[r]) return NVQSA_ERR_NULL_POINTER;
    if (!aligned_to(exchange[r], 16)) return NVQSA_ERR_MISALIGNED;
    peers[r] = static_cast<float*>(exchange[r]);
  }
  const void* region[4] = {key_data, key_scale, value_data, value_scale};
  const int64_t strides[4][3] = {{kd_stride_block, kd_stride_token, kd_stride_head},
                                 {ks_stride_block, ks_stride_token, ks_stride_head},
                                 {vd_stride_block, vd_stride_token, vd_stride_head},
                                 {vs_stride_block, vs_stride_token, vs_stride_head}};
  return run_attention(query, q_stride_row, q_stride_head, region, strides, num_blocks, page_size, kv_heads,
                       key_global_scale, value_global_scale, logical_indices, topk, block_table, num_requests,
                       table_width, token_to_request, output, o_stride_row, o_stride_head, nullptr, nullptr, rows,
                       query_heads, head_dim, workspace, workspace_bytes, stream, peers, world, rank, parity);
}

extern "C" int nvqsa_merge_partials_strided(const float* partial_out, int64_t out_split_stride,
                                            const float* partial_lse, int64_t lse_split_stride, int32_t splits,
                                            void* output, int64_t o_stride_row, int64_t o_stride_head, int64_t rows,
                                            int32_t query_heads, int32_t head_dim, void* stream) {
  if (splits < 1 || rows < 0 || query_heads < 1) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  if (rows == 0) return NVQSA_OK;
  if (!partial_out || !partial_lse || !output) return NVQSA_ERR_NULL_POINTER;
  const int64_t items = rows * query_heads;
  if (splits > 1 && (out_split_stride < items * kHeadDim || lse_split_stride < items)) return NVQSA_ERR_BAD_SHAPE;
  if (!aligned_to(partial_out, 16) || out_split_stride % 4 || !aligned_to(partial_lse, 4) || !aligned_to(output, 2))
    return NVQSA_ERR_MISALIGNED;
  const int vec_o = (aligned_to(output, 16) && o_stride_row % 8 == 0 && o_stride_head % 8 == 0) ? 1 : 0;
  const int64_t blocks = (items * 32 + 255) / 256;
  MergeArgs a;
  a.part_out = partial_out;
  a.part_lse = partial_lse;
  a.splits = splits;
  a.out_split_stride = out_split_stride;
  a.lse_split_stride = lse_split_stride;
  a.mode = 0;
  a.out = static_cast<__nv_bfloat16*>(output);
  a.o_stride_row = o_stride_row;
  a.o_stride_head = o_stride_head;
  a.vec_o = vec_o;
  a.out_f32 = nullptr;
  a.out_lse = nullptr;
  merge_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(a, rows, query_heads);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}

extern "C" int nvqsa_merge_partials(const float* partial_out, const float* partial_lse, int32_t splits, void* output,
                                    int64_t o_stride_row, int64_t o_stride_head, int64_t rows, int32_t query_heads,
                                    int32_t head_dim, void* stream) {
  const int64_t items = rows * (int64_t)query_heads;
  return nvqsa_merge_partials_strided(partial_out, items * kHeadDim, partial_lse, items, splits, output, o_stride_row,
                                      o_stride_head, rows, query_heads, head_dim, stream);
}

// ---------------------------------------------------------------------------
// No-allocation entry point.  For callers that may not allocate device memory
// (fixed-buffer hosts, no-allocation serving loops, plugins whose framework
// owns all allocations), the split-KV partials go to this static buffer
// instead of a caller-provided workspace.  Every device that loads the
// library holds the buffer until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[NVQSA_NOALLOC_SCRATCH_BYTES];

namespace {
// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the symbol names a host-side stand-in, never the device memory, so only
// this address may be handed to a kernel.  Atomic entries: host threads that
// make their first call at the same time all store the same address.  A
// cudaDeviceReset of the device invalidates the cached address.
std::atomic<void*> g_noalloc_scratch_ptr[nvqsa::kMaxDevices] = {};

int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= nvqsa::kMaxDevices) return NVQSA_ERR_CUDA;
  void* ptr = g_noalloc_scratch_ptr[dev].load(std::memory_order_relaxed);
  if (!ptr) {
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return NVQSA_ERR_CUDA;
    g_noalloc_scratch_ptr[dev].store(ptr, std::memory_order_relaxed);
  }
  *out = ptr;
  return NVQSA_OK;
}
}  // namespace

extern "C" int nvqsa_sparse_attention_noalloc(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim, void* stream) {
  size_t need = 0;
  if (const int st = nvqsa_sparse_attention_workspace_size(rows, query_heads, kv_heads, head_dim, topk, &need))
    return st;
  if (need > NVQSA_NOALLOC_SCRATCH_BYTES) return NVQSA_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    if (const int st = noalloc_scratch(&scratch)) return st;
  }
  return nvqsa_sparse_attention(query, q_stride_row, q_stride_head, key_data, kd_stride_block, kd_stride_token,
                                kd_stride_head, key_scale, ks_stride_block, ks_stride_token, ks_stride_head,
                                value_data, vd_stride_block, vd_stride_token, vd_stride_head, value_scale,
                                vs_stride_block, vs_stride_token, vs_stride_head, num_blocks, page_size, kv_heads,
                                key_global_scale, value_global_scale, logical_indices, topk, block_table,
                                num_requests, table_width, token_to_request, output, o_stride_row, o_stride_head, rows,
                                query_heads, head_dim, scratch, need, stream);
}
