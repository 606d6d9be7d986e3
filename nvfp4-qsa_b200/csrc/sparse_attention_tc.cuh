// QSA sparse decode reader with P.V on the 5th-generation tensor cores (tcgen05).
// Included by sparse_attention.cu inside namespace nvqsa::{anonymous}; uses its
// parameter block, barrier, copy and conversion helpers.
//
// Same CTA decomposition, gather pipeline and merges as sparse_attention_kernel
// (one CTA = (row, kv head, split), 4 warps, TMA tile::gather4 of 288-byte
// records into per-warp rings, clusters for the split merge).  What changes is
// where O lives: instead of 128 fp32 registers per lane, the CTA keeps one
// O^T accumulator (256 dims x 16 query heads, fp32) in 32 columns of tensor
// memory, written by tcgen05.mma.  That frees the registers for the query
// fragments and leaves the CUDA cores only the exact dequantisation, the
// scores and the softmax.
//
// The four warps run in rounds of 64 tokens (one 16-token tile each):
//   1. S = Q K^T on mma.sync (M = 16 heads, N = 8 tokens, K = 16 dims), K
//      dequantised in registers (one cvt.rn.f16x2.e2m1x2 and one f16x2
//      multiply per byte, exact), Q fragments in registers.
//   2. Each warp publishes its tile's per-head maxima; V of its tile is
//      dequantised into a shared V^T tile in the canonical no-swizzle
//      MN-major layout of a tcgen05 A operand (dims x tokens, f16).
//   3. After one CTA barrier every thread derives the same common running
//      max per head (raised only when a tile exceeds it by 2^10, so P stays
//      <= 1024 in f16); on the rare raise each warp rescales its 32 lanes of
//      O^T in tensor memory.
//   4. P = 2^(s * scale - m) goes to a shared P^T tile (tokens x heads, the
//      K-major B operand); after a second barrier one thread issues eight
//      tcgen05.mma (two 128-dim halves x four 16-token steps) into O^T and
//      commits them to an mbarrier that the next round waits on before it
//      overwrites V^T and P^T.
// The epilogue reads O^T back with tcgen05.ld (thread = dim), divides by the
// per-head sum and stores, or merges the cluster's ranks over distributed
// shared memory first.

constexpr int kTcStages = 2;                               // per-warp ring slots
constexpr int kRoundTokens = kWarps * kTile;                // 64 tokens per round
constexpr uint32_t kTcLbo = 128;                            // operand K-group (8 tokens) stride, bytes
constexpr uint32_t kTcSbo = (kRoundTokens / 8) * 128;       // operand M/N-group (8 rows) stride, bytes
constexpr float kTcRescaleThreshold = 10.0f;                // log2 units: P <= 2^10 between raises
constexpr uint32_t kTmemCols = 32;                          // O^T: 2 halves x 16 heads, fp32

template <int GMODE>
struct __align__(128) SmemTc {
  using Sel = typename std::conditional<GMODE == 0, int32_t, int2>::type;
  uint8_t rec[kWarps][kTcStages][kStageBytes];   // gather rings
  uint8_t vt[kHeadDim * kRoundTokens * 2];       // V^T f16, A operand (also Q-fragment scratch in the prologue)
  uint8_t pt[16 * kRoundTokens * 2];             // P^T f16, B operand
  Sel sel[kMaxRange];                            // valid selections: record row (gather4) or (block, offset)
  float tilemax[kWarps][16];
  float smul[16];
  int cnt[kCompactIters][kWarps];
  unsigned long long full_bar[kWarps][kTcStages];
  unsigned long long mma_bar;
  uint32_t tmem_base;
  int total;
  int abort;
  int last;
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
  // no-swizzle canonical layout: start, leading (K-group) and stride (M/N-group) byte offsets, version 1
  return (uint64_t)((addr >> 4) & 0x3fffu) | ((uint64_t)((kTcLbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((kTcSbo >> 4) & 0x3fffu) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptor: D f32, A and B f16, A MN-major, B K-major, N = 16, M = 128.
constexpr uint32_t kTcIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (1u << 15) | (0u << 16) | ((16u >> 3) << 17) |
                              ((128u >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])));
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

template <int GMODE>
__global__ void __launch_bounds__(kThreads, 3) sparse_attention_tc_kernel(const __grid_constant__ AttnParams p) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  SmemTc<GMODE>& sm = *reinterpret_cast<SmemTc<GMODE>*>(smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u));

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
  const int64_t chunks = (p.topk + kChunk - 1) / kChunk;
  const int my_chunks = split < chunks ? (int)((chunks - 1 - split) / p.splits + 1) : 0;  // <= kMaxChunks
  const int G = p.group;

  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < kTcStages; ++b) mbar_init(smem_u32(&sm.full_bar[warp][b]), 1);
    if (warp == 0) mbar_init(smem_u32(&sm.mma_bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (tid == 0) sm.abort = 0;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
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

  // ---------------- Q: exact power-of-two pre-scale into f16 fragments (scratch: the V^T tile) ----------------
  uint4* qscratch = reinterpret_cast<uint4*>(sm.vt);  // [16 k-steps][32 lanes]
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
      uint32_t* f = reinterpret_cast<uint32_t*>(&qscratch[ks * 32 + 4 * rr + cc]);
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
  tc_fence_before();
  __syncthreads();  // exponents, fragments, counts, the tensor-memory address
  tc_fence_after();
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
  uint4 qf[16];
#pragma unroll
  for (int s = 0; s < 16; ++s) qf[s] = qscratch[s * 32 + lane];
  const uint32_t tmem = sm.tmem_base;
  __syncthreads();  // selections and totals visible; the Q scratch is free again
  const int n = sm.total;
  const int ntiles = (n + kTile - 1) / kTile;
  const int rounds = (ntiles + kWarps - 1) / kWarps;

  // ---------------- per-warp gather ring: tile warp + 4k lands in slot k % kTcStages ----------------
  const uint8_t* const reg0 = p.region[0];
  const int64_t sb0 = p.stride[0][0], st0 = p.stride[0][1], sh0 = p.stride[0][2];
  auto issue_tile = [&](int k) {
    const int tile = warp + kWarps * k;
    const int slot = k % kTcStages;
    const uint32_t bar = smem_u32(&sm.full_bar[warp][slot]);
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
        gather4_g2s(smem_u32(&sm.rec[warp][slot][lane * 4 * kRecordBytes]), &p.rows_map, rows[0], rows[1], rows[2],
                    rows[3], bar);
      }
    } else {
      if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(count * kRecordBytes));
      __syncwarp();
      if (lane < count) {
        const int2 e = sm.sel[j0 + lane];
        const uint32_t dst = smem_u32(&sm.rec[warp][slot][slot_off(lane)]);
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
  bool live = true;  // this warp's waits have not run out
  int dead_round = -1;  // round whose wait ran out: its tile and the next may still be in flight
  if (warp < ntiles) issue_tile(0);

  int k_off[2];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) k_off[nt] = slot_off(8 * nt + r);
  const float smul_r = sm.smul[r];
  const float smul_r8 = sm.smul[r + 8];
  float mh = kMaskedScore;  // lanes 0..15: common running max of head `lane` (log2 units)
  float l_r = 0.0f, l_r8 = 0.0f;  // this warp's share of the softmax sums, rows r and r + 8
  const uint32_t tm_lane = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's 32 lanes of O^T

  for (int k = 0; k < rounds; ++k) {
    const int tile = warp + kWarps * k;
    const bool has = tile < ntiles;
    const int slot = k % kTcStages;
    if (live && tile + kWarps < ntiles) issue_tile(k + 1);  // into the slot tile k-1 used
    bool ready = false;
    if (has && live) {
      ready = mbar_wait(smem_u32(&sm.full_bar[warp][slot]), (uint32_t)((k / kTcStages) & 1));
      if (!ready) {
        live = false;
        dead_round = k;
        if (lane == 0) sm.abort = 1;
      }
    }
    const int tok_base = tile * kTile;
    const uint8_t* stage = sm.rec[warp][slot];

    // ---- S = Q K^T for this warp's 16 tokens ----
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = -1.0e30f;
    if (ready) {
      uint32_t sg[2][4];
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
      for (int half = 0; half < 2; ++half) {
        uint4 kq[2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          kq[nt] = *reinterpret_cast<const uint4*>(stage + k_off[nt] + 64 * half + 16 * c);
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          const uint4 qa = qf[8 * half + s2];
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const uint32_t word =
                (s2 >> 1) == 0 ? kq[nt].x : (s2 >> 1) == 1 ? kq[nt].y : (s2 >> 1) == 2 ? kq[nt].z : kq[nt].w;
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
      if (tok_base + kTile > n) {  // the last tile: tokens past n are masked
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int t0 = tok_base + 8 * nt + 2 * c;
          if (t0 >= n) { sacc[nt][0] = -1.0e30f; sacc[nt][2] = -1.0e30f; }
          if (t0 + 1 >= n) { sacc[nt][1] = -1.0e30f; sacc[nt][3] = -1.0e30f; }
        }
      }
    }
    float mx_r = fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1]));
    float mx_r8 = fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3]));
    mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 1));
    mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 2));
    mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 1));
    mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 2));
    if (c == 0) {
      sm.tilemax[warp][r] = mx_r * smul_r;  // smul > 0: max commutes with the scale
      sm.tilemax[warp][r + 8] = mx_r8 * smul_r8;
    }

    // ---- V^T tile: the previous round's P.V must be done before it is overwritten ----
    if (k > 0 && !mbar_wait(smem_u32(&sm.mma_bar), (uint32_t)((k - 1) & 1)) && lane == 0) sm.abort = 1;
    {
      uint8_t* vt = sm.vt;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int t = 8 * (i & 1) + (lane & 7);       // token of the tile
        const int g = (lane >> 3) + 4 * (i >> 1);     // 8-dim chunk: dims 8g .. 8g + 7
        const int kk = warp * kTile + t;              // token of the round
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (ready) {
          const uint8_t* rec = stage + slot_off(t);
          const uint32_t w = *reinterpret_cast<const uint32_t*>(rec + 144 + 4 * g);
          const uint32_t scl = dup_lo(cvt_e4m3x2_f16x2(rec[272 + (g >> 1)]));
          o.x = hmul2_u32(cvt_e2m1x2_f16x2_byte<0>(w), scl);
          o.y = hmul2_u32(cvt_e2m1x2_f16x2_byte<1>(w), scl);
          o.z = hmul2_u32(cvt_e2m1x2_f16x2_byte<2>(w), scl);
          o.w = hmul2_u32(cvt_e2m1x2_f16x2_byte<3>(w), scl);
        }
        *reinterpret_cast<uint4*>(vt + g * kTcSbo + (kk >> 3) * kTcLbo + (kk & 7) * 16) = o;
      }
    }
    __syncthreads();  // tile maxima visible; every warp has read its records of this round

    // ---- common running max (identical in every thread), rare raise ----
    float newm = kMaskedScore, alpha = 1.0f;
    bool up = false;
    if (lane < 16) {
      const float tmax = fmaxf(fmaxf(sm.tilemax[0][lane], sm.tilemax[1][lane]),
                               fmaxf(sm.tilemax[2][lane], sm.tilemax[3][lane]));
      up = tmax > mh + kTcRescaleThreshold;
      newm = up ? tmax : mh;
      alpha = ex2(mh - newm);
      mh = newm;
    }
    const bool raise = __any_sync(0xffffffffu, up);  // same in every warp
    const float m_r = __shfl_sync(0xffffffffu, newm, r);
    const float m_r8 = __shfl_sync(0xffffffffu, newm, r + 8);
    if (raise) {
      l_r *= __shfl_sync(0xffffffffu, alpha, r);
      l_r8 *= __shfl_sync(0xffffffffu, alpha, r + 8);
      if (k > 0) {  // O^T holds rounds 0 .. k-1 (complete: waited above): scale column h by alpha of head h
        float a16[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) a16[h] = __shfl_sync(0xffffffffu, alpha, h);
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float v[16];
          tmem_ld16(tm_lane + 16 * half, v);
#pragma unroll
          for (int h = 0; h < 16; ++h) v[h] *= a16[h];
          tmem_st16(tm_lane + 16 * half, v);
        }
      }
    }

    // ---- P = 2^(s * scale - m) into the P^T tile (f16, P <= 1024) ----
    float pv[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      pv[nt][0] = ex2(fmaf(sacc[nt][0], smul_r, -m_r));
      pv[nt][1] = ex2(fmaf(sacc[nt][1], smul_r, -m_r));
      pv[nt][2] = ex2(fmaf(sacc[nt][2], smul_r8, -m_r8));
      pv[nt][3] = ex2(fmaf(sacc[nt][3], smul_r8, -m_r8));
    }
    if (!ready || tok_base + kTile > n) {  // masked scores never count, even while m is still -1e20
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int t0 = tok_base + 8 * nt + 2 * c;
        if (!ready || t0 >= n) { pv[nt][0] = 0.0f; pv[nt][2] = 0.0f; }
        if (!ready || t0 + 1 >= n) { pv[nt][1] = 0.0f; pv[nt][3] = 0.0f; }
      }
    }
    l_r += (pv[0][0] + pv[0][1]) + (pv[1][0] + pv[1][1]);
    l_r8 += (pv[0][2] + pv[0][3]) + (pv[1][2] + pv[1][3]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int kk = warp * kTile + 8 * nt + 2 * c;  // token of the round (even)
      const uint32_t off = (kk >> 3) * kTcLbo + (kk & 7) * 2;
      *reinterpret_cast<uint32_t*>(sm.pt + off + r * 16) = pack_half2(pv[nt][0], pv[nt][1]);
      *reinterpret_cast<uint32_t*>(sm.pt + kTcSbo + off + r * 16) = pack_half2(pv[nt][2], pv[nt][3]);
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // V^T and P^T -> tensor-core reads
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int j = 0; j < kRoundTokens / 16; ++j) {
          const uint64_t da = umma_desc(smem_u32(sm.vt) + half * 16 * kTcSbo + j * 2 * kTcLbo);
          const uint64_t db = umma_desc(smem_u32(sm.pt) + j * 2 * kTcLbo);
          const uint32_t acc = (k > 0 || j > 0) ? 1u : 0u;
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem + 16 * half),
              "l"(da), "l"(db), "r"(kTcIdesc), "r"(acc)
              : "memory");
        }
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                       smem_u32(&sm.mma_bar))
                   : "memory");
    }
    __syncwarp();
  }

  // ---------------- epilogue ----------------
  if (dead_round >= 0) {  // let this warp's copies still in flight land (bounded) before shared memory is released
    for (int k2 = dead_round; k2 <= dead_round + 1 && warp + kWarps * k2 < ntiles; ++k2)
      mbar_wait(smem_u32(&sm.full_bar[warp][k2 % kTcStages]), (uint32_t)((k2 / kTcStages) & 1), kDrainSpinLimit);
  }
  if (rounds > 0 && !mbar_wait(smem_u32(&sm.mma_bar), (uint32_t)((rounds - 1) & 1)) && lane == 0) sm.abort = 1;
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 1);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 2);
  float* lsum = reinterpret_cast<float*>(sm.pt);  // [kWarps][16]; P^T is free once the last P.V is done
  if (c == 0) {
    lsum[warp * 16 + r] = l_r;
    lsum[warp * 16 + r + 8] = l_r8;
  }
  if (lane < 16) sm.tilemax[0][lane] = mh;  // publish the final running max per head
  tc_fence_after();
  // thread (warp, lane) holds O^T rows of dims d = 32 * warp + lane (columns 0..15) and 128 + d (16..31)
  float o[2][16];
  if (rounds > 0) {
    tmem_ld16(tm_lane, o[0]);
    tmem_ld16(tm_lane + 16, o[1]);
  } else {
#pragma unroll
    for (int h = 0; h < 16; ++h) o[0][h] = o[1][h] = 0.0f;
  }
  tc_fence_before();
  __syncthreads();  // sums, maxima and every tensor-memory read done
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  const bool aborted = sm.abort != 0;
  float mj[16], lj[16];
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    mj[h] = sm.tilemax[0][h];
    lj[h] = (lsum[h] + lsum[16 + h]) + (lsum[32 + h] + lsum[48 + h]);
  }

  if (p.cluster > 1) {
    // Publish (O^T, m, l) in this CTA's shared memory; rank 0 merges the other ranks over
    // distributed shared memory.  Layout: float4 q of thread t at comb[q * 128 + t].
    float4* comb = reinterpret_cast<float4*>(&sm.rec[0][0][0]);   // 8 x 128 float4 = 16 KB
    float* cml = reinterpret_cast<float*>(comb + 8 * 128);        // m[16], l[16]
    __syncthreads();  // every thread has read the per-head sums before the ring space is reused
#pragma unroll
    for (int q = 0; q < 8; ++q)
      comb[q * 128 + tid] = make_float4(o[q >> 2][4 * (q & 3)], o[q >> 2][4 * (q & 3) + 1], o[q >> 2][4 * (q & 3) + 2],
                                        o[q >> 2][4 * (q & 3) + 3]);
    if (tid < 16) {
      cml[tid] = mj[tid];
      cml[16 + tid] = lj[tid];
    }
    cluster_sync();
    bool ok = !aborted;
    if (split % p.cluster == 0 && ok) {
      for (int rk = 1; rk < p.cluster; ++rk) {
        if (cluster_ld_s32(cluster_map(smem_u32(&sm.abort), (uint32_t)rk))) {
          ok = false;
          continue;
        }
        const uint32_t cb = cluster_map(smem_u32(comb), (uint32_t)rk);
        float a[16], b[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float pm = __uint_as_float(cluster_ld_s32(cb + (uint32_t)(8 * 128 * 16 + 4 * h)));
          const float pl = __uint_as_float(cluster_ld_s32(cb + (uint32_t)(8 * 128 * 16 + 64 + 4 * h)));
          const float M = fmaxf(mj[h], pm);
          a[h] = ex2(mj[h] - M);
          b[h] = ex2(pm - M);
          lj[h] = lj[h] * a[h] + pl * b[h];
          mj[h] = M;
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 v = cluster_ld_f4(cb + (uint32_t)(q * 128 + tid) * 16u);
          const int hf = q >> 2, h0 = 4 * (q & 3);
          o[hf][h0] = o[hf][h0] * a[h0] + v.x * b[h0];
          o[hf][h0 + 1] = o[hf][h0 + 1] * a[h0 + 1] + v.y * b[h0 + 1];
          o[hf][h0 + 2] = o[hf][h0 + 2] * a[h0 + 2] + v.z * b[h0 + 2];
          o[hf][h0 + 3] = o[hf][h0 + 3] * a[h0 + 3] + v.w * b[h0 + 3];
        }
      }
    }
    cluster_sync();  // ranks > 0 keep their shared memory until rank 0 has read it
    if (split % p.cluster != 0 || !ok) return;
  } else if (aborted) {
    return;
  }

  // ---------------- store: thread = dims d and 128 + d, every head of this kv head ----------------
  const int d = 32 * warp + lane;
  const int part = split / p.cluster;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j >= G) continue;
    // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
    const float inv = lj[j] > 0.0f ? p.inv_value_scale / fmaxf(lj[j], 1.0e-20f) : 0.0f;
    const int head = kvh * G + j;
    const float v0 = o[0][j] * inv, v1 = o[1][j] * inv;
    if (p.mode == 0) {
      __nv_bfloat16* op = p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head;
      op[d] = __float2bfloat16_rn(v0);
      op[128 + d] = __float2bfloat16_rn(v1);
    } else {
      const int64_t slot = ((int64_t)part * p.rows + row) * p.query_heads + head;
      float* op = p.part_out + slot * kHeadDim;
      op[d] = v0;
      op[128 + d] = v1;
      if (tid == 0) p.part_lse[slot] = lj[j] > 0.0f ? mj[j] + log2f(fmaxf(lj[j], 1.0e-20f)) : -INFINITY;
    }
  }

  // ---------------- split-KV beyond one cluster: the last part to arrive merges all parts ----------------
  if (!p.fuse) {
    if (p.xworld > 0) xrank_exchange(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid);
    return;
  }
  fused_part_merge(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid);
}
