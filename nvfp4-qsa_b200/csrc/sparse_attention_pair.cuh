// QSA sparse decode reader, warp-pair variant: two warps share each 16-token tile.
// Included by sparse_attention.cu inside namespace nvqsa::{anonymous}; uses its
// parameter block, barrier, copy, conversion and merge helpers.
//
// Same CTA decomposition, selection prologue, gather and merges as
// sparse_attention_kernel; the difference is how a tile is shared.  The four
// warps form two pairs, each with its own ring of 16-record tiles (pair p
// takes tiles p, p + 2, ...).  Warp h of a pair owns head dimensions
// [128h, 128h + 128):
//   * S = Q K^T: each warp runs the 8 mma k-steps of its dimensions (K
//     dequantised in registers as in the full-width kernel) and the two
//     partial score tiles are added through shared memory (double-buffered,
//     one 64-thread named barrier per tile), in the same order in both
//     warps, so both hold identical scores, maxima and P;
//   * O += P V: each warp accumulates only its 128 dimensions, 64 fp32
//     registers per lane instead of 128.
// With 128 registers per thread and 54 KB of shared memory four CTAs fit on
// an SM.  Measured on B200 it is the faster reader for batches with fewer
// (row, kv head) units than SMs -- a tile is finished by two warps, so the
// latency-bound single-row decode gets shorter (config 5b: 30 us per layer
// against 37 us) -- and the slower one for large batches (config 5a: 59.7 us
// against 55 us, the duplicated softmax and the per-tile pair barrier cost
// more than the freed registers buy), so the planner picks it only for the
// former.

constexpr int kPairStages = 4;                 // ring slots per pair
constexpr int kPairAhead = kPairStages - 1;    // tiles issued ahead of the one being consumed

template <int GMODE>
struct __align__(128) SmemPair {
  using Sel = typename std::conditional<GMODE == 0, int32_t, int2>::type;
  uint8_t rec[2][kPairStages][kStageBytes];    // gather ring of each pair
  uint4 qfrag[16][32];                          // Q A-fragments [k-step][lane]
  Sel sel[kMaxRange];                           // valid selections: record row (gather4) or (block, offset)
  float4 xch[2][2][2][32][2];                   // partial scores [pair][buffer][warp of pair][lane][2]
  unsigned long long full_bar[2][kPairStages];
  float smul[16];
  int cnt[kCompactIters][kWarps];
  int total;
  int abort;
  int last;
};

// Named barrier of one warp pair (ids 1 and 2; 0 is __syncthreads).
__device__ __forceinline__ void pair_sync(int pair) {
  if (pair == 0)
    asm volatile("bar.sync 1, 64;\n" ::: "memory");
  else
    asm volatile("bar.sync 2, 64;\n" ::: "memory");
}

template <int GMODE>
__global__ void __launch_bounds__(kThreads, 4) sparse_attention_pair_kernel(const __grid_constant__ AttnParams p) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  SmemPair<GMODE>& sm =
      *reinterpret_cast<SmemPair<GMODE>*>(smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u));

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int pair = warp >> 1;
  const int h = warp & 1;   // dimension half of this warp
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

  if (tid == 0) {
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int b = 0; b < kPairStages; ++b) mbar_init(smem_u32(&sm.full_bar[q][b]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    sm.abort = 0;
  }

  // ---------------- prologue: all independent global loads first ----------------
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
  const bool req_ok = req >= 0 && (int64_t)req < p.num_requests;
  const int32_t* bt_row = p.block_table + (req_ok ? (int64_t)req * p.table_width : 0);
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
  // Q: exact per-head power-of-two pre-scale into f16 mma fragments (heads >= G stay zero)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = warp + kWarps * i;
    uint32_t amax = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) amax = max(amax, max((qw[i][t] << 16) & 0x7fffffffu, qw[i][t] & 0x7fff0000u));
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
        if (vmask & (1u << it)) {
          if constexpr (GMODE == 0)
            sm.sel[base + pre[it]] = (phys[it] * p.kv_heads + kvh) * (int32_t)p.page_size + offs[it];
          else
            sm.sel[base + pre[it]] = make_int2(phys[it], offs[it]);
        }
#pragma unroll
        for (int w = 0; w < kWarps; ++w) base_all += sm.cnt[it][w];
      }
    }
    if (tid == 0) sm.total = base_all;
  }
  __syncthreads();
  const int n = sm.total;
  const int ntiles = (n + kTile - 1) / kTile;

  // ---------------- per-pair gather ring: tile pair + 2k lands in slot k % kPairStages ----------------
  const uint8_t* const reg0 = p.region[0];
  const int64_t sb0 = p.stride[0][0], st0 = p.stride[0][1], sh0 = p.stride[0][2];
  auto issue_tile = [&](int k) {  // called by warp h == 0 of the pair
    const int tile = pair + 2 * k;
    const int slot = k % kPairStages;
    const uint32_t bar = smem_u32(&sm.full_bar[pair][slot]);
    const int j0 = tile * kTile;
    const int count = min(kTile, n - j0);
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    if constexpr (GMODE == 0) {
      if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)kStageBytes);
      __syncwarp();
      if (lane < kTile / 4) {
        int32_t rows[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = group_token(lane, j);
          rows[j] = t < count ? sm.sel[j0 + t] : p.total_rows;  // out of range: zero fill
        }
        gather4_g2s(smem_u32(&sm.rec[pair][slot][lane * 4 * kRecordBytes]), &p.rows_map, rows[0], rows[1], rows[2],
                    rows[3], bar);
      }
    } else {
      if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(count * kRecordBytes));
      __syncwarp();
      if (lane < count) {
        const int2 e = sm.sel[j0 + lane];
        const uint32_t dst = smem_u32(&sm.rec[pair][slot][slot_off(lane)]);
        if constexpr (GMODE == 1) {
          bulk_g2s(dst, reg0 + (int64_t)e.x * sb0 + (int64_t)e.y * st0 + (int64_t)kvh * sh0, kRecordBytes, bar);
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
    }
  };
  const int my_tiles = ntiles > pair ? (ntiles - pair + 1) / 2 : 0;
  if (h == 0) {
#pragma unroll
    for (int k = 0; k < kPairAhead; ++k)
      if (k < my_tiles) issue_tile(k);
  }

  int k_off[2], v_off[4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) k_off[nt] = slot_off(8 * nt + r);
  {
    const int tt[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
    for (int q = 0; q < 4; ++q) v_off[q] = slot_off(tt[q]);
  }
  const float smul_r = sm.smul[r];
  const float smul_r8 = sm.smul[r + 8];

  float oacc[16][4];  // this warp's 128 dims: n-tile i = dims 128h + 8i .. + 7
#pragma unroll
  for (int i = 0; i < 16; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;
  float m_r = kMaskedScore, m_r8 = kMaskedScore;
  float l_r = 0.0f, l_r8 = 0.0f;

  // One tile of 16 tokens at `stage`; TAIL masks tokens at or past n.
  auto tile_body = [&](const uint8_t* stage, const int k, const int tok_base, auto tail_tag) {
    constexpr bool TAIL = decltype(tail_tag)::value;
    // ---- partial S over this warp's 128 dims: k-steps 8h .. 8h + 7 on both n-tiles ----
    float sacc[2][4];
    uint32_t sg[2][2];
    uint4 kq[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint8_t* rec = stage + k_off[nt];
      const uint32_t sc = cvt_e4m3x2_f16x2(*reinterpret_cast<const uint16_t*>(rec + 128 + 8 * h + 2 * c));
      sg[nt][0] = dup_lo(sc);
      sg[nt][1] = dup_hi(sc);
      kq[nt] = *reinterpret_cast<const uint4*>(rec + 64 * h + 16 * c);
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
    }
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      const uint4 qa = sm.qfrag[8 * h + s2][lane];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t word =
            (s2 >> 1) == 0 ? kq[nt].x : (s2 >> 1) == 1 ? kq[nt].y : (s2 >> 1) == 2 ? kq[nt].z : kq[nt].w;
        const uint32_t scl = sg[nt][s2 >> 2];
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
    // ---- add the partner's half: S = S(dims 0..127) + S(dims 128..255) in both warps ----
    float4(*xb)[32][2] = sm.xch[pair][k & 1];
    xb[h][lane][0] = make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]);
    xb[h][lane][1] = make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]);
    pair_sync(pair);
    {
      const float4 a0 = xb[0][lane][0], a1 = xb[0][lane][1];
      const float4 b0 = xb[1][lane][0], b1 = xb[1][lane][1];
      sacc[0][0] = a0.x + b0.x; sacc[0][1] = a0.y + b0.y; sacc[0][2] = a0.z + b0.z; sacc[0][3] = a0.w + b0.w;
      sacc[1][0] = a1.x + b1.x; sacc[1][1] = a1.y + b1.y; sacc[1][2] = a1.z + b1.z; sacc[1][3] = a1.w + b1.w;
    }

    // ---- online softmax (base 2), identical in both warps of the pair ----
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
        for (int i = 0; i < 16; ++i) {
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

    // ---- O += P V over this warp's 128 dims ----
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
#define NVQSA_PAIR_PV_BYTE(B)                                                                          \
  {                                                                                                    \
    const int nt = 8 * kk + 2 * (B);                                                                   \
    mma_f16(oacc[nt], pf[0], pf[1], pf[2], pf[3], hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(x01), s01),        \
            hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(x23), s23));                                            \
    mma_f16(oacc[nt + 1], pf[0], pf[1], pf[2], pf[3], hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(y01), s01),    \
            hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(y23), s23));                                            \
  }
      NVQSA_PAIR_PV_BYTE(0)
      NVQSA_PAIR_PV_BYTE(1)
      NVQSA_PAIR_PV_BYTE(2)
      NVQSA_PAIR_PV_BYTE(3)
#undef NVQSA_PAIR_PV_BYTE
    }
  };

  int k = 0;
  for (; k < my_tiles; ++k) {
    const int slot = k % kPairStages;
    if (!mbar_wait(smem_u32(&sm.full_bar[pair][slot]), (uint32_t)((k / kPairStages) & 1))) {
      if (lane == 0) sm.abort = 1;
      break;
    }
    const int tok_base = (pair + 2 * k) * kTile;
    const uint8_t* stage = sm.rec[pair][slot];
    if (tok_base + kTile <= n)
      tile_body(stage, k, tok_base, std::false_type{});
    else
      tile_body(stage, k, tok_base, std::true_type{});
    // Both warps passed this tile's pair barrier, so the slot of tile k - 1 is free.
    if (h == 0 && k + kPairAhead < my_tiles) issue_tile(k + kPairAhead);
    __syncwarp();
  }

  // ---------------- combine the pairs, normalise, store ----------------
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 1);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 2);
  if (k < my_tiles) {
    // This pair gave up: let its copies still in flight land (bounded) before shared memory is released.
    for (int k2 = k + 1; k2 < my_tiles && k2 <= k + kPairAhead; ++k2)
      mbar_wait(smem_u32(&sm.full_bar[pair][k2 % kPairStages]), (uint32_t)((k2 / kPairStages) & 1), kDrainSpinLimit);
  }
  __syncthreads();  // every warp left its loop: no bulk copy is in flight, the rings are free
  if (tid == 0) stamp_max(p, row * p.kv_heads + kvh, 1);
  const bool aborted = sm.abort != 0;
  if (aborted && p.cluster <= 1) return;  // a cluster CTA still takes the cluster barriers below

  // Pair 1 -> pair 0 over shared memory; slot q = h * 32 + lane, float4 i at comb[i * 64 + q].
  float4* comb = reinterpret_cast<float4*>(&sm.rec[0][0][0]);   // [16][64] float4 + [64] (m, m8, l, l8)
  float4* comb_ml = comb + 16 * 64;
  const int q = h * 32 + lane;
  if (!aborted) {
    if (pair == 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) comb[i * 64 + q] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
      comb_ml[q] = make_float4(m_r, m_r8, l_r, l_r8);
    }
    __syncthreads();
    if (pair == 0) {
      const float4 ml = comb_ml[q];
      const float M_r = fmaxf(m_r, ml.x), M_r8 = fmaxf(m_r8, ml.y);
      const float a0 = ex2(m_r - M_r), b0 = ex2(ml.x - M_r);
      const float a1 = ex2(m_r8 - M_r8), b1 = ex2(ml.y - M_r8);
      l_r = l_r * a0 + ml.z * b0;
      l_r8 = l_r8 * a1 + ml.w * b1;
      m_r = M_r;
      m_r8 = M_r8;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 v = comb[i * 64 + q];
        oacc[i][0] = oacc[i][0] * a0 + v.x * b0;
        oacc[i][1] = oacc[i][1] * a0 + v.y * b0;
        oacc[i][2] = oacc[i][2] * a1 + v.z * b1;
        oacc[i][3] = oacc[i][3] * a1 + v.w * b1;
      }
    }
    __syncthreads();
  }

  if (p.cluster > 1) {
    // Split-KV inside a thread-block cluster: pair 0 of every CTA publishes its (O, m, l) halves in its own
    // shared memory; then every thread of every rank merges and stores one slice.
    if (pair == 0 && !aborted) {
#pragma unroll
      for (int i = 0; i < 16; ++i) comb[i * 64 + q] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
      comb_ml[q] = make_float4(m_r, m_r8, l_r, l_r8);
    }
    cluster_sync();
    const bool ok = cluster_merge_store<16, 64>(p, comb, row, kvh, G, tid, split, &sm.abort);
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

  if (pair == 0) {
    // lane (r, c) holds dims 128h + 32c + i (oacc[i][2hh]) and + 16 (oacc[i][2hh + 1]) for heads r, r + 8.
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = r + 8 * hh;
      if (j >= G) continue;
      const float l = hh ? l_r8 : l_r;
      const float m = hh ? m_r8 : m_r;
      // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
      const float inv = l > 0.0f ? p.inv_value_scale / fmaxf(l, 1.0e-20f) : 0.0f;
      const int head = kvh * G + j;
      float v[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = oacc[i][2 * hh] * inv;
        v[16 + i] = oacc[i][2 * hh + 1] * inv;
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
          for (int qq = 0; qq < 4; ++qq)
            reinterpret_cast<uint4*>(op)[qq] = make_uint4(w[4 * qq], w[4 * qq + 1], w[4 * qq + 2], w[4 * qq + 3]);
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
        for (int qq = 0; qq < 8; ++qq)
          reinterpret_cast<float4*>(op)[qq] = make_float4(v[4 * qq], v[4 * qq + 1], v[4 * qq + 2], v[4 * qq + 3]);
        if (h == 0 && c == 0) p.part_lse[slot] = l > 0.0f ? m + log2f(fmaxf(l, 1.0e-20f)) : -INFINITY;
      }
    }
  }

  // ---------------- split-KV beyond one cluster / across GPUs ----------------
  if (!p.fuse) {
    if (p.xworld > 0) xrank_exchange(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid);
    return;
  }
  fused_part_merge(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid, p.splits / p.cluster);
}
