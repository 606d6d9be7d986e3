// BF16 sibling reader: QSA sparse paged decode over a bf16 K/V cache (sm_100a).
// Included by sparse_attention.cu inside namespace nvqsa::{anonymous}; uses its
// parameter block, barrier, copy and merge helpers.
//
// The reference's third forward_qsa branch (integration/snapshot/qsa.py:352-366)
// calls vLLM's BF16 QSA kernel on key/value views [blocks, page, kv_heads, 256]
// of the bf16 main cache; its arithmetic is the FP8 harness kernel's
// (src/qsa_fp8_harness.py:42-208) without the dequantisation: scores
// (Q . K) * d^-0.5 in base 2, masked selections at -1e20, online softmax, P
// cast to bf16 before P . V, output / l (zeros for a row with no valid
// selection).
//
// One CTA = (row, kv head, split) = 4 warps, as the NVFP4 reader, with the
// same prologue (selection resolution and compaction, split chunks).  Each
// warp owns a ring of 8-token tiles; a token's K row and V row (512 bytes
// each) arrive by two bulk copies into a 1,040-byte slot (16 bytes of skew
// keep the ldmatrix row reads conflict-free).  There is nothing to
// dequantise: S = Q K^T runs on bf16 mma.sync m16n8k16 with Q fragments from
// shared memory and K fragments by ldmatrix; P stays in the S accumulator
// registers (bf16 pairs, the m16n8k8 A layout) and O += P V runs on bf16
// m16n8k8 with V fragments by ldmatrix.trans.  The warp combine, cluster
// merge, workspace merge and the split-KV partial format are those of the
// NVFP4 reader.

constexpr int kBfTile = 8;                           // tokens per warp tile (one n-tile of S, one k-step of P V)
constexpr int kBfStages = 2;                         // ring slots per warp
constexpr int kBfRowBytes = 512;                     // 256 bf16
constexpr int kBfSlot = 2 * kBfRowBytes + 16;        // K row | V row | skew
constexpr int kBfStageBytes = kBfTile * kBfSlot;

struct __align__(128) SmemBf {
  uint8_t rec[kWarps][kBfStages][kBfStageBytes];   // private gather rings (epilogue: combine scratch)
  uint4 qfrag[16][32];                             // Q A-fragments: [k-step][lane] -> {a0a1,a2a3,a4a5,a6a7}
  int2 sel[kMaxRange];                             // (physical block, token in page) of valid selections
  unsigned long long full_bar[kWarps][kBfStages];
  int cnt[kCompactIters][kWarps];
  int total;
  int abort;
  int last;
};

__device__ __forceinline__ void mma_bf16_k16(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16_k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

__global__ void __launch_bounds__(kThreads, 2) sparse_attention_bf16_kernel(const __grid_constant__ AttnParams p) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  SmemBf& sm = *reinterpret_cast<SmemBf*>(smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u));

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
    for (int b = 0; b < kBfStages; ++b) mbar_init(smem_u32(&sm.full_bar[warp][b]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (tid == 0) sm.abort = 0;

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

  // ---------------- Q: bf16 A-fragments in natural dim order ----------------
  // k-step s covers dims [16s, 16s + 16).  Lane L holds dims 8L .. 8L + 7 = k-step L / 2, columns 8 (L & 1) + 2t,
  // +1 for word t: thread-in-group t, register a0a1 / a2a3 (rows j, j + 8) for the low 8 columns, a4a5 / a6a7
  // for the high 8.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = warp + kWarps * i;
    const int hh = j >> 3, rr = j & 7;
    const int ks = lane >> 1, hi = lane & 1;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t* f = reinterpret_cast<uint32_t*>(&sm.qfrag[ks][4 * rr + t]);
      f[2 * hi + hh] = qw[i][t];
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
  __syncthreads();
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
  const int ntiles = (n + kBfTile - 1) / kBfTile;

  // ---------------- per-warp gather pipeline: tiles warp, warp + 4, ... ----------------
  auto issue_tile = [&](int k) {
    const int tile = warp + kWarps * k;
    const int slot = k % kBfStages;
    const uint32_t bar = smem_u32(&sm.full_bar[warp][slot]);
    const int j0 = tile * kBfTile;
    const int count = min(kBfTile, n - j0);
    // The slot was last read by this warp's generic loads: order them before the async-proxy writes.
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(count * 2 * kBfRowBytes));
    __syncwarp();
    if (lane < 2 * count) {  // lane 2t: K row of token t, lane 2t + 1: its V row
      const int t = lane >> 1, g = (lane & 1) << 1;
      const int2 e = sm.sel[j0 + t];
      bulk_g2s(smem_u32(&sm.rec[warp][slot][t * kBfSlot + (lane & 1) * kBfRowBytes]),
               p.region[g] + (int64_t)e.x * p.stride[g][0] + (int64_t)e.y * p.stride[g][1] +
                   (int64_t)kvh * p.stride[g][2],
               kBfRowBytes, bar);
    }
  };
  const int my_tiles = ntiles > warp ? (ntiles - warp + kWarps - 1) / kWarps : 0;
#pragma unroll
  for (int k = 0; k < kBfStages - 1; ++k)
    if (k < my_tiles) issue_tile(k);

  // ldmatrix row addresses (byte offsets inside a stage).  K: matrix i of an x4 = k-step half (i & 1) of
  // k-step 2q + (i >> 1); lane L supplies row L & 7 (token) of matrix L >> 3.  V (trans): matrix i = dims
  // 16q + 8i .. +7 of the 8 tokens; lane L supplies token L & 7 of matrix L >> 3.
  const int lrow = lane & 7, lmat = lane >> 3;
  const int k_ld = lrow * kBfSlot + ((lmat >> 1) * 16 + (lmat & 1) * 8) * 2;
  const int v_ld = lrow * kBfSlot + kBfRowBytes + lmat * 16;
  const float smul = p.score_scale;

  float oacc[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;
  float m_r = kMaskedScore, m_r8 = kMaskedScore;
  float l_r = 0.0f, l_r8 = 0.0f;

  int k = 0;
  for (; k < my_tiles; ++k) {
    if (k + kBfStages - 1 < my_tiles) issue_tile(k + kBfStages - 1);
    const int slot = k % kBfStages;
    if (!mbar_wait(smem_u32(&sm.full_bar[warp][slot]), (uint32_t)((k / kBfStages) & 1))) {
      if (lane == 0) sm.abort = 1;
      break;
    }
    const int tok_base = (warp + kWarps * k) * kBfTile;
    const uint32_t stage = smem_u32(&sm.rec[warp][slot][0]);
    const int valid_here = min(kBfTile, n - tok_base);
    if (valid_here < kBfTile) {
      // Slots past the last valid token hold stale bytes: zero their V rows so that 0 * V stays 0.
      uint4* vz = reinterpret_cast<uint4*>(&sm.rec[warp][slot][0]);
      for (int i = lane; i < (kBfTile - valid_here) * (kBfRowBytes / 16); i += 32) {
        const int t = valid_here + i / (kBfRowBytes / 16);
        vz[(t * kBfSlot + kBfRowBytes) / 16 + i % (kBfRowBytes / 16)] = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // ---- S = Q K^T over 16 k-steps (two accumulator chains) ----
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint32_t b00, b01, b10, b11;
      ldmatrix_x4(stage + k_ld + q * 64, b00, b01, b10, b11);
      mma_bf16_k16(s0, sm.qfrag[2 * q][lane], b00, b01);
      mma_bf16_k16(s1, sm.qfrag[2 * q + 1][lane], b10, b11);
    }
    float s[4] = {s0[0] + s1[0], s0[1] + s1[1], s0[2] + s1[2], s0[3] + s1[3]};

    // ---- online softmax (base 2) ----
    {
      const int t0 = tok_base + 2 * c;
      if (t0 >= n) { s[0] = -1.0e30f; s[2] = -1.0e30f; }
      if (t0 + 1 >= n) { s[1] = -1.0e30f; s[3] = -1.0e30f; }
    }
    float mx_r = fmaxf(s[0], s[1]), mx_r8 = fmaxf(s[2], s[3]);
    mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 1));
    mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 2));
    mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 1));
    mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 2));
    mx_r *= smul;
    mx_r8 *= smul;
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
    float pv[4];
    pv[0] = ex2(fmaf(s[0], smul, -m_r));
    pv[1] = ex2(fmaf(s[1], smul, -m_r));
    pv[2] = ex2(fmaf(s[2], smul, -m_r8));
    pv[3] = ex2(fmaf(s[3], smul, -m_r8));
    {
      const int t0 = tok_base + 2 * c;
      if (t0 >= n) { pv[0] = 0.0f; pv[2] = 0.0f; }
      if (t0 + 1 >= n) { pv[1] = 0.0f; pv[3] = 0.0f; }
    }
    // l sums the fp32 p; P is cast to bf16 for P V (the reference's p.to(bfloat16) before tl.dot).
    l_r += pv[0] + pv[1];
    l_r8 += pv[2] + pv[3];
    const uint32_t pa0 = pack_bf162(pv[0], pv[1]);
    const uint32_t pa1 = pack_bf162(pv[2], pv[3]);

    // ---- O += P V: 32 n-tiles of 8 dims, K = the tile's 8 tokens ----
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint32_t v0, v1, v2, v3;
      ldmatrix_x4_trans(stage + v_ld + q * 64, v0, v1, v2, v3);
      mma_bf16_k8(oacc[4 * q], pa0, pa1, v0);
      mma_bf16_k8(oacc[4 * q + 1], pa0, pa1, v1);
      mma_bf16_k8(oacc[4 * q + 2], pa0, pa1, v2);
      mma_bf16_k8(oacc[4 * q + 3], pa0, pa1, v3);
    }
    __syncwarp();  // every lane's reads of this slot precede its refill
  }

  // ---------------- combine the four warps, normalise, store ----------------
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 1);
  l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 2);
  if (k < my_tiles) {
    for (int k2 = k + 1; k2 < my_tiles && k2 <= k + kBfStages - 1; ++k2)
      mbar_wait(smem_u32(&sm.full_bar[warp][k2 % kBfStages]), (uint32_t)((k2 / kBfStages) & 1), kDrainSpinLimit);
  }
  __syncthreads();
  const bool aborted = sm.abort != 0;
  if (aborted && p.cluster <= 1) return;

  float4* comb = reinterpret_cast<float4*>(&sm.rec[0][0][0]);   // [32][64] float4 + [64] (m, m8, l, l8)
  float4* comb_ml = comb + 32 * 64;
#pragma unroll
  for (int round = 0; round < 2; ++round) {
    if (aborted) break;
    const int senders = round == 0 ? 2 : 1;
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

  if (p.cluster > 1) {
    if (warp == 0 && !aborted) {
#pragma unroll
      for (int i = 0; i < 32; ++i) comb[i * 64 + lane] = make_float4(oacc[i][0], oacc[i][1], oacc[i][2], oacc[i][3]);
      comb_ml[lane] = make_float4(m_r, m_r8, l_r, l_r8);
    }
    cluster_sync();
    bool ok = !aborted;
    if (split % p.cluster == 0 && warp == 0 && ok) {
      for (int rk = 1; rk < p.cluster; ++rk) {
        if (cluster_ld_s32(cluster_map(smem_u32(&sm.abort), (uint32_t)rk))) {
          ok = false;
          continue;
        }
        const uint32_t cb = cluster_map(smem_u32(comb), (uint32_t)rk);
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
    }
    cluster_sync();
    if (split % p.cluster != 0 || !ok) return;
  }

  if (warp == 0) {
    // lane (r, c) holds O[head r + 8 hh][dims 8 nt + 2c, 8 nt + 2c + 1] in oacc[nt][2 hh], oacc[nt][2 hh + 1].
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = r + 8 * hh;
      if (j >= G) continue;
      const float l = hh ? l_r8 : l_r;
      const float m = hh ? m_r8 : m_r;
      const float inv = l > 0.0f ? p.inv_value_scale / fmaxf(l, 1.0e-20f) : 0.0f;
      const int head = kvh * G + j;
      if (p.mode == 0) {
        __nv_bfloat16* op = p.out + row * p.o_stride_row + (int64_t)head * p.o_stride_head;
#pragma unroll
        for (int nt = 0; nt < 32; ++nt) {
          const uint32_t w = pack_bf162(oacc[nt][2 * hh] * inv, oacc[nt][2 * hh + 1] * inv);
          if (p.vec_o) {
            *reinterpret_cast<uint32_t*>(op + 8 * nt + 2 * c) = w;
          } else {
            unsigned short* os = reinterpret_cast<unsigned short*>(op + 8 * nt + 2 * c);
            os[0] = (unsigned short)(w & 0xffffu);
            os[1] = (unsigned short)(w >> 16);
          }
        }
      } else {
        const int64_t slot = ((int64_t)(split / p.cluster) * p.rows + row) * p.query_heads + head;
        float* op = p.part_out + slot * kHeadDim;
#pragma unroll
        for (int nt = 0; nt < 32; ++nt)
          *reinterpret_cast<float2*>(op + 8 * nt + 2 * c) =
              make_float2(oacc[nt][2 * hh] * inv, oacc[nt][2 * hh + 1] * inv);
        if (c == 0) p.part_lse[slot] = l > 0.0f ? m + log2f(fmaxf(l, 1.0e-20f)) : -INFINITY;
      }
    }
  }

  if (!p.fuse) {
    if (p.xworld > 0) xrank_exchange(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid);
    return;
  }
  fused_part_merge(p, reinterpret_cast<float*>(&sm.rec[0][0][0]), sm.last, row, kvh, G, tid, p.splits / p.cluster);
}
