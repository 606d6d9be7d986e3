// QSA sparse paged decode attention over an NVFP4 cache, sm_100a.
//
// Replaces the reference's Triton reader (python/nvfp4_qsa/kernels.py:168-403).
// The reference runs one program per (query row, kv head), so a single decode
// row occupies 2 SMs; here the selected tokens of each (row, kv head) are
// split across CTAs (split-KV) and merged with a base-2 log-sum-exp, the
// layout of the reference's split-K sibling (src/qsa_fp8_harness.py:183-208).
//
// One CTA = (row, kv head, split) = 4 warps = 2 warp pairs.
//  * Prologue: the CTA resolves its range of selections through
//    token_to_request / block_table (masking rules of kernels.py:241-257) and
//    compacts the valid ones into a shared list, so masked selections cost
//    nothing (they contribute exp2(-1e20 - m) = 0 in the reference).
//  * Records (K data 128 B, K scales 16 B, V data 128 B, V scales 16 B) are
//    gathered into a 4-stage shared-memory ring with 16-byte cp.async,
//    32 tokens per stage, 16-byte chunks XOR-swizzled so that the consumer
//    reads below are bank-conflict free.
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
//    shared memory, run the online softmax (base 2, masked = -1e20 as in
//    kernels.py:316-331), and accumulate O^T-free O = P V (M = heads,
//    N = 8 dims, K = 16 tokens) with P converted to f16 in registers.
//  * Q is converted bf16 -> f16 after an exact per-head power-of-two
//    pre-scale (amax * 2^e in [2^14, 2^15)), folded back into the score scale.
#include "common.cuh"

namespace nvqsa {
namespace {

constexpr int kHeadDim = 256;
constexpr int kThreads = 128;
constexpr int kStageTokens = 32;
constexpr int kStages = 4;
constexpr int kMaxRange = 1024;         // selections per CTA
constexpr int kChunksPerToken = 18;     // 288 bytes / 16
constexpr float kMaskedScore = -1.0e20f;

struct AttnParams {
  const __nv_bfloat16* q;
  int64_t q_stride_row, q_stride_head;
  const uint8_t* region[4];      // key_data, key_scale, value_data, value_scale
  int64_t stride[4][3];          // block, token, head (bytes)
  int64_t num_blocks, page_size;
  int32_t kv_heads, group, query_heads;
  float score_scale;             // head_dim^-0.5 * log2(e) / key_global_scale
  float inv_value_scale;         // 1 / value_global_scale
  const int32_t* indices;
  int64_t topk;
  const int32_t* block_table;
  int64_t num_requests, table_width;
  const int32_t* token_to_request;
  int64_t rows;
  int32_t splits, range;
  int32_t mode;                  // 0: bf16 output; 1: fp32 partial (normalised O, lse)
  int32_t vec_q;                 // 16-byte aligned query rows
  int32_t vec_o;                 // 16-byte aligned output rows
  __nv_bfloat16* out;
  int64_t o_stride_row, o_stride_head;
  float* part_out;               // [splits][rows][query_heads][256]
  float* part_lse;               // [splits][rows][query_heads]
};

struct __align__(16) Smem {
  uint8_t kd[kStages][kStageTokens][128];
  uint8_t vd[kStages][kStageTokens][128];
  uint8_t ks[kStages][kStageTokens][16];
  uint8_t vs[kStages][kStageTokens][16];
  int2 sel[kMaxRange];                       // (physical block, token in page)
  float xchg[2][2][2][32 * 8];               // [pair][parity][half][lane*8]
  float qmul[16];
  float smul[16];
  int cnt[kMaxRange / kThreads][kThreads / 32];
  int total;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void pair_barrier(int pair) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(1 + pair), "r"(64));
}

// 16-byte chunk swizzles (see file header).
__device__ __forceinline__ int swz_k(int chunk, int tok) { return chunk ^ ((tok & 1) << 2); }
__device__ __forceinline__ int swz_v(int chunk, int tok) { return chunk ^ (((tok >> 1) & 3) << 1); }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t dup_lo(uint32_t x) { return __byte_perm(x, 0, 0x1010); }
__device__ __forceinline__ uint32_t dup_hi(uint32_t x) { return __byte_perm(x, 0, 0x3232); }

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__global__ void __launch_bounds__(kThreads, 3) sparse_attention_kernel(const AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int pair = warp >> 1;
  const int half = warp & 1;
  const int r = lane >> 2;  // mma group row
  const int c = lane & 3;   // mma thread-in-group

  int64_t bid = blockIdx.x;
  const int split = (int)(bid % p.splits);
  bid /= p.splits;
  const int kvh = (int)(bid % p.kv_heads);
  const int64_t row = bid / p.kv_heads;

  const int64_t pos0 = (int64_t)split * p.range;
  int64_t pos1 = pos0 + p.range;
  if (pos1 > p.topk) pos1 = p.topk;
  const int len = pos1 > pos0 ? (int)(pos1 - pos0) : 0;

  // ---------------- Q pre-scale exponents ----------------
  const int G = p.group;
  for (int j = warp; j < 16; j += 4) {
    int e = 0;
    if (j < G) {
      const __nv_bfloat16* qrow = p.q + row * p.q_stride_row + (int64_t)(kvh * G + j) * p.q_stride_head;
      uint32_t amax = 0;
      const unsigned short* qs = reinterpret_cast<const unsigned short*>(qrow) + lane * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = max(amax, ((uint32_t)__ldg(qs + i) << 16) & 0x7fffffffu);
#pragma unroll
      for (int m = 16; m; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
      if (amax != 0 && amax < 0x7f800000u) {
        e = 14 - ilogbf(__uint_as_float(amax));
        e = max(-126, min(126, e));
      }
    }
    if (lane == 0) {
      sm.qmul[j] = ldexpf(1.0f, e);
      sm.smul[j] = ldexpf(p.score_scale, -e);
    }
  }

  // ---------------- resolve + compact the CTA's selections ----------------
  const int32_t req = __ldg(p.token_to_request + row);
  const bool req_ok = req >= 0 && (int64_t)req < p.num_requests;
  const int32_t* idx_row = p.indices + row * p.topk + pos0;
  const int32_t* bt_row = p.block_table + (req_ok ? (int64_t)req * p.table_width : 0);
  const int iters = (len + kThreads - 1) / kThreads;
  uint32_t vmask = 0;
  int2 ent[kMaxRange / kThreads];
  int pre[kMaxRange / kThreads];
#pragma unroll
  for (int it = 0; it < kMaxRange / kThreads; ++it) {
    ent[it] = make_int2(0, 0);
    pre[it] = 0;
    if (it < iters) {
      const int pos = it * kThreads + tid;
      bool valid = false;
      if (pos < len && req_ok) {
        const int32_t idx = __ldg(idx_row + pos);
        if (idx >= 0) {
          const int64_t lpage = (int64_t)idx / p.page_size;
          if (lpage < p.table_width) {
            const int32_t phys = __ldg(bt_row + lpage);
            valid = phys >= 0 && (int64_t)phys < p.num_blocks;
            ent[it] = make_int2(phys, (int)((int64_t)idx - lpage * p.page_size));
          }
        }
      }
      const uint32_t b = __ballot_sync(0xffffffffu, valid);
      pre[it] = __popc(b & ((1u << lane) - 1u));
      if (valid) vmask |= 1u << it;
      if (lane == 0) sm.cnt[it][warp] = __popc(b);
    }
  }
  __syncthreads();
  {
    int base_all = 0;
#pragma unroll
    for (int it = 0; it < kMaxRange / kThreads; ++it) {
      if (it < iters) {
        int base = base_all;
        for (int w = 0; w < warp; ++w) base += sm.cnt[it][w];
        if (vmask & (1u << it)) sm.sel[base + pre[it]] = ent[it];
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) base_all += sm.cnt[it][w];
      }
    }
    if (tid == 0) sm.total = base_all;
  }
  __syncthreads();
  const int n = sm.total;
  const int nst = (n + kStageTokens - 1) / kStageTokens;

  // ---------------- gather pipeline ----------------
  auto issue_stage = [&](int st) {
    const int buf = st % kStages;
    for (int ci = tid; ci < kStageTokens * kChunksPerToken; ci += kThreads) {
      const int t = ci / kChunksPerToken;
      const int k = ci - t * kChunksPerToken;
      const int j = st * kStageTokens + t;
      const bool valid = j < n;
      const int2 e = valid ? sm.sel[j] : make_int2(0, 0);
      const uint8_t* base;
      int64_t sb, stt, sh;
      int chunk;
      uint8_t* dst;
      if (k < 8) {
        base = p.region[0]; sb = p.stride[0][0]; stt = p.stride[0][1]; sh = p.stride[0][2]; chunk = k;
        dst = &sm.kd[buf][t][swz_k(chunk, t) * 16];
      } else if (k == 8) {
        base = p.region[1]; sb = p.stride[1][0]; stt = p.stride[1][1]; sh = p.stride[1][2]; chunk = 0;
        dst = &sm.ks[buf][t][0];
      } else if (k < 17) {
        base = p.region[2]; sb = p.stride[2][0]; stt = p.stride[2][1]; sh = p.stride[2][2]; chunk = k - 9;
        dst = &sm.vd[buf][t][swz_v(chunk, t) * 16];
      } else {
        base = p.region[3]; sb = p.stride[3][0]; stt = p.stride[3][1]; sh = p.stride[3][2]; chunk = 0;
        dst = &sm.vs[buf][t][0];
      }
      const uint8_t* src = base;  // zero-fill reads nothing from src
      if (valid) src += (int64_t)e.x * sb + (int64_t)e.y * stt + (int64_t)kvh * sh + chunk * 16;
      cp_async16(dst, src, valid ? 16 : 0);
    }
  };

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < nst) issue_stage(s);
    cp_async_commit();
  }

  // ---------------- Q fragments (registers) ----------------
  // Lane (r, c) of warp half h holds heads r and r+8, head dims
  // 128h + 32c + [0, 32), laid out for 8 k-steps of 16 permuted dims.
  uint32_t qf[8][4];
  {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = r + 8 * hh;
      float qv[32];
      if (j < G) {
        const float mul = sm.qmul[j];
        const __nv_bfloat16* qp =
            p.q + row * p.q_stride_row + (int64_t)(kvh * G + j) * p.q_stride_head + half * 128 + 32 * c;
        if (p.vec_q) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(qp) + v);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              qv[8 * v + 2 * i] = bf16_lo(ww[i]) * mul;
              qv[8 * v + 2 * i + 1] = bf16_hi(ww[i]) * mul;
            }
          }
        } else {
          const unsigned short* qs = reinterpret_cast<const unsigned short*>(qp);
#pragma unroll
          for (int i = 0; i < 32; ++i) qv[i] = __uint_as_float(((uint32_t)__ldg(qs + i)) << 16) * mul;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) qv[i] = 0.0f;
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        qf[s][hh] = pack_half2(qv[4 * s], qv[4 * s + 1]);
        qf[s][2 + hh] = pack_half2(qv[4 * s + 2], qv[4 * s + 3]);
      }
    }
  }
  const float smul_r = sm.smul[r];
  const float smul_r8 = sm.smul[r + 8];

  float oacc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;
  float m_r = kMaskedScore, m_r8 = kMaskedScore;
  float l_r = 0.0f, l_r8 = 0.0f;

  for (int st = 0; st < nst; ++st) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    if (st + kStages - 1 < nst) issue_stage(st + kStages - 1);
    cp_async_commit();

    const int buf = st % kStages;
    const int tok_base = st * kStageTokens + 16 * pair;  // compacted index of this pair's first token
    if (tok_base >= n) continue;                          // pair-uniform: both warps skip together

    // ---- S partial over this warp's 128 dims: 2 n-tiles of 8 tokens ----
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
      const int tk = 16 * pair + 8 * nt + r;
      const uint4 kw = *reinterpret_cast<const uint4*>(&sm.kd[buf][tk][swz_k(4 * half + c, tk) * 16]);
      const uint32_t ksb = *reinterpret_cast<const uint16_t*>(&sm.ks[buf][tk][8 * half + 2 * c]);
      const uint32_t sc = cvt_e4m3x2_f16x2(ksb);
      const uint32_t s_lo = dup_lo(sc), s_hi = dup_hi(sc);
      const uint32_t kwv[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t word = kwv[s >> 1];
        const uint32_t sg = (s < 4) ? s_lo : s_hi;
        uint32_t b0, b1;
        if (s & 1) {
          b0 = hmul2_u32(cvt_e2m1x2_f16x2_byte<2>(word), sg);
          b1 = hmul2_u32(cvt_e2m1x2_f16x2_byte<3>(word), sg);
        } else {
          b0 = hmul2_u32(cvt_e2m1x2_f16x2_byte<0>(word), sg);
          b1 = hmul2_u32(cvt_e2m1x2_f16x2_byte<1>(word), sg);
        }
        mma_f16(sacc[nt], qf[s][0], qf[s][1], qf[s][2], qf[s][3], b0, b1);
      }
    }

    // ---- exchange partial scores with the partner warp ----
    {
      float* mine = &sm.xchg[pair][st & 1][half][lane * 8];
      const float* theirs = &sm.xchg[pair][st & 1][half ^ 1][lane * 8];
      reinterpret_cast<float4*>(mine)[0] = make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]);
      reinterpret_cast<float4*>(mine)[1] = make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]);
      pair_barrier(pair);
      const float4 o0 = reinterpret_cast<const float4*>(theirs)[0];
      const float4 o1 = reinterpret_cast<const float4*>(theirs)[1];
      // Same operand order in both warps (low half first) -> identical sums.
      if (half == 0) {
        sacc[0][0] += o0.x; sacc[0][1] += o0.y; sacc[0][2] += o0.z; sacc[0][3] += o0.w;
        sacc[1][0] += o1.x; sacc[1][1] += o1.y; sacc[1][2] += o1.z; sacc[1][3] += o1.w;
      } else {
        sacc[0][0] = o0.x + sacc[0][0]; sacc[0][1] = o0.y + sacc[0][1];
        sacc[0][2] = o0.z + sacc[0][2]; sacc[0][3] = o0.w + sacc[0][3];
        sacc[1][0] = o1.x + sacc[1][0]; sacc[1][1] = o1.y + sacc[1][1];
        sacc[1][2] = o1.z + sacc[1][2]; sacc[1][3] = o1.w + sacc[1][3];
      }
    }

    // ---- online softmax (base 2) ----
    uint32_t pf[4];
    {
      float x[2][4];
      float mx_r = kMaskedScore, mx_r8 = kMaskedScore;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int t0 = tok_base + 8 * nt + 2 * c;
        const bool v0 = t0 < n, v1 = t0 + 1 < n;
        x[nt][0] = v0 ? sacc[nt][0] * smul_r : kMaskedScore;
        x[nt][1] = v1 ? sacc[nt][1] * smul_r : kMaskedScore;
        x[nt][2] = v0 ? sacc[nt][2] * smul_r8 : kMaskedScore;
        x[nt][3] = v1 ? sacc[nt][3] * smul_r8 : kMaskedScore;
        mx_r = fmaxf(mx_r, fmaxf(x[nt][0], x[nt][1]));
        mx_r8 = fmaxf(mx_r8, fmaxf(x[nt][2], x[nt][3]));
      }
      mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 1));
      mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 2));
      mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 1));
      mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 2));
      const float mn_r = fmaxf(m_r, mx_r), mn_r8 = fmaxf(m_r8, mx_r8);
      const float a_r = exp2f(m_r - mn_r), a_r8 = exp2f(m_r8 - mn_r8);
      m_r = mn_r;
      m_r8 = mn_r8;
      float pv[2][4];
      float sum_r = 0.0f, sum_r8 = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int t0 = tok_base + 8 * nt + 2 * c;
        const bool v0 = t0 < n, v1 = t0 + 1 < n;
        pv[nt][0] = v0 ? exp2f(x[nt][0] - mn_r) : 0.0f;
        pv[nt][1] = v1 ? exp2f(x[nt][1] - mn_r) : 0.0f;
        pv[nt][2] = v0 ? exp2f(x[nt][2] - mn_r8) : 0.0f;
        pv[nt][3] = v1 ? exp2f(x[nt][3] - mn_r8) : 0.0f;
        sum_r += pv[nt][0] + pv[nt][1];
        sum_r8 += pv[nt][2] + pv[nt][3];
      }
      l_r = l_r * a_r + sum_r;
      l_r8 = l_r8 * a_r8 + sum_r8;
      if (__any_sync(0xffffffffu, a_r != 1.0f || a_r8 != 1.0f)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          oacc[i][0] *= a_r; oacc[i][1] *= a_r;
          oacc[i][2] *= a_r8; oacc[i][3] *= a_r8;
        }
      }
      pf[0] = pack_half2(pv[0][0], pv[0][1]);
      pf[1] = pack_half2(pv[0][2], pv[0][3]);
      pf[2] = pack_half2(pv[1][0], pv[1][1]);
      pf[3] = pack_half2(pv[1][2], pv[1][3]);
    }

    // ---- O += P V over this warp's 128 dims: 16 n-tiles of 8 dims ----
    {
      const int t0 = 16 * pair + 2 * c;
      const int tt[4] = {t0, t0 + 1, t0 + 8, t0 + 9};
      const int vchunk = 4 * half + (r >> 1);
      uint2 vw[4];
      uint32_t vsb[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        vw[q] = *reinterpret_cast<const uint2*>(&sm.vd[buf][tt[q]][swz_v(vchunk, tt[q]) * 16 + 8 * (r & 1)]);
        vsb[q] = sm.vs[buf][tt[q]][8 * half + r];
      }
      const uint32_t s01 = cvt_e4m3x2_f16x2(vsb[0] | (vsb[1] << 8));
      const uint32_t s23 = cvt_e4m3x2_f16x2(vsb[2] | (vsb[3] << 8));
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint32_t w0 = k ? vw[0].y : vw[0].x, w1 = k ? vw[1].y : vw[1].x;
        const uint32_t w2 = k ? vw[2].y : vw[2].x, w3 = k ? vw[3].y : vw[3].x;
        // low nibbles (even dims) of two tokens interleaved into one byte
        const uint32_t x01 = (w0 & 0x0f0f0f0fu) | ((w1 & 0x0f0f0f0fu) << 4);
        const uint32_t y01 = ((w0 >> 4) & 0x0f0f0f0fu) | (w1 & 0xf0f0f0f0u);
        const uint32_t x23 = (w2 & 0x0f0f0f0fu) | ((w3 & 0x0f0f0f0fu) << 4);
        const uint32_t y23 = ((w2 >> 4) & 0x0f0f0f0fu) | (w3 & 0xf0f0f0f0u);
#define NVQSA_PV_BYTE(B)                                                                               \
  {                                                                                                    \
    const int nt = 8 * k + 2 * (B);                                                                    \
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
  }

  // ---------------- combine the two pairs, normalise, store ----------------
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 1);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 2);

  cp_async_wait<0>();
  __syncthreads();
  float* comb_o = reinterpret_cast<float*>(&sm.kd[0][0][0]);  // [half][lane][64]
  float* comb_ml = reinterpret_cast<float*>(&sm.vd[0][0][0]); // [half][lane][4]
  if (pair == 1) {
    float* o = comb_o + (half * 32 + lane) * 64;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      reinterpret_cast<float4*>(o)[i] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
    reinterpret_cast<float4*>(comb_ml)[half * 32 + lane] = make_float4(m_r, m_r8, l_r, l_r8);
  }
  __syncthreads();
  if (pair == 1) return;
  {
    const float* o = comb_o + (half * 32 + lane) * 64;
    const float4 ml = reinterpret_cast<const float4*>(comb_ml)[half * 32 + lane];
    const float M_r = fmaxf(m_r, ml.x), M_r8 = fmaxf(m_r8, ml.y);
    const float a0 = exp2f(m_r - M_r), b0 = exp2f(ml.x - M_r);
    const float a1 = exp2f(m_r8 - M_r8), b1 = exp2f(ml.y - M_r8);
    l_r = l_r * a0 + ml.z * b0;
    l_r8 = l_r8 * a1 + ml.w * b1;
    m_r = M_r;
    m_r8 = M_r8;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 v = reinterpret_cast<const float4*>(o)[i];
      oacc[i][0] = oacc[i][0] * a0 + v.x * b0;
      oacc[i][1] = oacc[i][1] * a0 + v.y * b0;
      oacc[i][2] = oacc[i][2] * a1 + v.z * b1;
      oacc[i][3] = oacc[i][3] * a1 + v.w * b1;
    }
  }

#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int j = r + 8 * hh;
    if (j >= G) continue;
    const float l = hh ? l_r8 : l_r;
    const float m = hh ? m_r8 : m_r;
    // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
    const float inv = l > 0.0f ? p.inv_value_scale / fmaxf(l, 1.0e-20f) : 0.0f;
    const int head = kvh * G + j;
    // lane (r, c) holds dims 128*half + 32c + i (from oacc[i][2hh]) and +16 (oacc[i][2hh+1])
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = oacc[i][2 * hh] * inv;
      v[16 + i] = oacc[i][2 * hh + 1] * inv;
    }
    const int d0 = 128 * half + 32 * c;
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
      const int64_t slot = ((int64_t)split * p.rows + row) * p.query_heads + head;
      float* op = p.part_out + slot * kHeadDim + d0;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(op)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      if (half == 0 && c == 0) p.part_lse[slot] = l > 0.0f ? m + log2f(fmaxf(l, 1.0e-20f)) : -INFINITY;
    }
  }
}

// One warp per (row, query head): log-sum-exp merge of `splits` partials.
// mode 0 -> bf16 output; mode 1 -> fp32 normalised output + merged lse.
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ part_out, const float* __restrict__ part_lse,
                                                    int splits, int64_t rows, int query_heads, int mode,
                                                    __nv_bfloat16* out, int64_t o_stride_row, int64_t o_stride_head,
                                                    int vec_o, float* out_f32, float* out_lse) {
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t items = rows * query_heads;
  if (w >= items) return;
  const int64_t row = w / query_heads;
  const int head = (int)(w - row * query_heads);
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, __ldg(part_lse + (int64_t)s * items + w));
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float den = 0.0f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float lse = __ldg(part_lse + (int64_t)s * items + w);
      const float wt = exp2f(lse - M);  // 0 for -inf partials
      if (wt == 0.0f) continue;
      den += wt;
      const float4* po = reinterpret_cast<const float4*>(part_out + ((int64_t)s * items + w) * kHeadDim + lane * 8);
      const float4 a = __ldg(po), b = __ldg(po + 1);
      acc[0] += wt * a.x; acc[1] += wt * a.y; acc[2] += wt * a.z; acc[3] += wt * a.w;
      acc[4] += wt * b.x; acc[5] += wt * b.y; acc[6] += wt * b.z; acc[7] += wt * b.w;
    }
  }
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] *= inv;
  if (mode == 0) {
    __nv_bfloat16* op = out + row * o_stride_row + (int64_t)head * o_stride_head + lane * 8;
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      u[i] = *reinterpret_cast<uint32_t*>(&b);
    }
    if (vec_o) {
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
    float4* op = reinterpret_cast<float4*>(out_f32 + w * kHeadDim + lane * 8);
    op[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    op[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (lane == 0) out_lse[w] = den > 0.0f ? M + log2f(den) : -INFINITY;
  }
}

// ---------------- host-side planning ----------------
struct Plan {
  int splits;
  int range;
};

Plan make_plan(int64_t rows, int kv_heads, int64_t topk, int sms) {
  Plan pl;
  const int64_t units = rows * kv_heads;
  const int64_t target = (int64_t)(sms > 0 ? sms : 148) * 2;
  int64_t splits = units > 0 ? (target + units - 1) / units : 1;
  const int64_t max_splits = topk > 0 ? (topk + kStageTokens - 1) / kStageTokens : 1;
  if (splits > max_splits) splits = max_splits;
  const int64_t min_splits = topk > 0 ? (topk + kMaxRange - 1) / kMaxRange : 1;
  if (splits < min_splits) splits = min_splits;
  if (splits < 1) splits = 1;
  int64_t range = topk > 0 ? (topk + splits - 1) / splits : kStageTokens;
  range = (range + kStageTokens - 1) / kStageTokens * kStageTokens;
  if (range > kMaxRange) range = kMaxRange;
  splits = topk > 0 ? (topk + range - 1) / range : 1;
  pl.splits = (int)splits;
  pl.range = (int)range;
  return pl;
}

size_t workspace_for(const Plan& pl, int64_t rows, int query_heads) {
  if (pl.splits <= 1) return 0;
  const size_t items = (size_t)pl.splits * rows * query_heads;
  return items * kHeadDim * sizeof(float) + ((items * sizeof(float) + 255) / 256) * 256;
}

// Dynamic shared memory above 48 KB is opted into once per device.
constexpr int kMaxDevices = 64;
bool smem_configured[kMaxDevices] = {};

int configure_smem(size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return NVQSA_ERR_CUDA;
  if (!smem_configured[dev]) {
    if (cudaFuncSetAttribute(sparse_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return NVQSA_ERR_CUDA;
    smem_configured[dev] = true;
  }
  return NVQSA_OK;
}

int run_attention(const void* query, int64_t q_stride_row, int64_t q_stride_head, const void* const region[4],
                  const int64_t strides[4][3], int64_t num_blocks, int64_t page_size, int32_t kv_heads,
                  float key_global_scale, float value_global_scale, const int32_t* logical_indices, int64_t topk,
                  const int32_t* block_table, int64_t num_requests, int64_t table_width,
                  const int32_t* token_to_request, void* output, int64_t o_stride_row, int64_t o_stride_head,
                  float* partial_out, float* partial_lse, int64_t rows, int32_t query_heads, int32_t head_dim,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || topk < 0 || kv_heads < 1 || query_heads < 1 || num_blocks < 0 || page_size < 1 ||
      num_requests < 0 || table_width < 0)
    return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  if (query_heads % kv_heads) return NVQSA_ERR_UNSUPPORTED;
  const int G = query_heads / kv_heads;
  if (G < 1 || G > 16) return NVQSA_ERR_UNSUPPORTED;
  if (rows == 0) return NVQSA_OK;
  const bool partial_mode = partial_out != nullptr;
  if (!query || !token_to_request || (!output && !partial_mode) || (partial_mode && !partial_lse))
    return NVQSA_ERR_NULL_POINTER;
  if (topk > 0 && !logical_indices) return NVQSA_ERR_NULL_POINTER;
  for (int i = 0; i < 4; ++i) {
    if (!region[i]) return NVQSA_ERR_NULL_POINTER;
    if (!aligned_to(region[i], 16)) return NVQSA_ERR_MISALIGNED;
    for (int j = 0; j < 3; ++j)
      if (strides[i][j] % 16) return NVQSA_ERR_MISALIGNED;
  }
  if (!aligned_to(query, 2) || (partial_mode ? !aligned_to(partial_out, 16) || !aligned_to(partial_lse, 4)
                                             : !aligned_to(output, 2)))
    return NVQSA_ERR_MISALIGNED;

  const int sms = device_sm_count();
  if (sms <= 0) return NVQSA_ERR_CUDA;
  const Plan pl = make_plan(rows, kv_heads, topk, sms);
  const size_t need = workspace_for(pl, rows, query_heads);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned_to(workspace, 16))) return NVQSA_ERR_WORKSPACE;
  if ((int64_t)pl.splits * rows * kv_heads > 0x7fffffffLL) return NVQSA_ERR_BAD_SHAPE;

  AttnParams p;
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
  p.group = G;
  p.query_heads = query_heads;
  p.score_scale = (float)(0.0625 * 1.4426950408889634) * (1.0f / key_global_scale);
  p.inv_value_scale = 1.0f / value_global_scale;
  p.indices = logical_indices;
  p.topk = topk;
  p.block_table = block_table;
  p.num_requests = num_requests;
  p.table_width = table_width;
  p.token_to_request = token_to_request;
  p.rows = rows;
  p.splits = pl.splits;
  p.range = pl.range;
  p.vec_q = (aligned_to(query, 16) && q_stride_row % 8 == 0 && q_stride_head % 8 == 0) ? 1 : 0;
  p.vec_o = (!partial_mode && aligned_to(output, 16) && o_stride_row % 8 == 0 && o_stride_head % 8 == 0) ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(output);
  p.o_stride_row = o_stride_row;
  p.o_stride_head = o_stride_head;
  float* ws_out = nullptr;
  float* ws_lse = nullptr;
  if (pl.splits > 1) {
    ws_out = static_cast<float*>(workspace);
    ws_lse = ws_out + (size_t)pl.splits * rows * query_heads * kHeadDim;
    p.mode = 1;
    p.part_out = ws_out;
    p.part_lse = ws_lse;
  } else if (partial_mode) {
    p.mode = 1;
    p.part_out = partial_out;
    p.part_lse = partial_lse;
  } else {
    p.mode = 0;
    p.part_out = nullptr;
    p.part_lse = nullptr;
  }

  const size_t smem = sizeof(Smem);
  if (const int st = configure_smem(smem)) return st;
  cudaStream_t s = as_stream(stream);
  const int64_t grid = (int64_t)pl.splits * rows * kv_heads;
  sparse_attention_kernel<<<(unsigned)grid, kThreads, smem, s>>>(p);
  if (cudaGetLastError() != cudaSuccess) return NVQSA_ERR_LAUNCH;
  if (pl.splits > 1) {
    const int64_t items = rows * query_heads;
    const int64_t blocks = (items * 32 + 255) / 256;
    merge_kernel<<<(unsigned)blocks, 256, 0, s>>>(ws_out, ws_lse, pl.splits, rows, query_heads, partial_mode ? 1 : 0,
                                                  p.out, o_stride_row, o_stride_head, p.vec_o, partial_out, partial_lse);
    if (cudaGetLastError() != cudaSuccess) return NVQSA_ERR_LAUNCH;
  }
  return NVQSA_OK;
}

}  // namespace
}  // namespace nvqsa

using namespace nvqsa;

extern "C" int nvqsa_sparse_attention_workspace_size(int64_t rows, int32_t query_heads, int32_t kv_heads,
                                                     int32_t head_dim, int64_t topk, size_t* workspace_bytes) {
  if (!workspace_bytes) return NVQSA_ERR_NULL_POINTER;
  *workspace_bytes = 0;
  if (rows < 0 || topk < 0 || kv_heads < 1 || query_heads < 1) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  if (rows == 0) return NVQSA_OK;
  const int sms = device_sm_count();
  if (sms <= 0) return NVQSA_ERR_CUDA;
  *workspace_bytes = workspace_for(make_plan(rows, kv_heads, topk, sms), rows, query_heads);
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

extern "C" int nvqsa_merge_partials(const float* partial_out, const float* partial_lse, int32_t splits, void* output,
                                    int64_t o_stride_row, int64_t o_stride_head, int64_t rows, int32_t query_heads,
                                    int32_t head_dim, void* stream) {
  if (splits < 1 || rows < 0 || query_heads < 1) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != kHeadDim) return NVQSA_ERR_HEAD_DIM;
  if (rows == 0) return NVQSA_OK;
  if (!partial_out || !partial_lse || !output) return NVQSA_ERR_NULL_POINTER;
  if (!aligned_to(partial_out, 16) || !aligned_to(output, 2)) return NVQSA_ERR_MISALIGNED;
  const int vec_o = (aligned_to(output, 16) && o_stride_row % 8 == 0 && o_stride_head % 8 == 0) ? 1 : 0;
  const int64_t items = rows * query_heads;
  const int64_t blocks = (items * 32 + 255) / 256;
  merge_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(partial_out, partial_lse, splits, rows, query_heads, 0,
                                                                static_cast<__nv_bfloat16*>(output), o_stride_row,
                                                                o_stride_head, vec_o, nullptr, nullptr);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}
