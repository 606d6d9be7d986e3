// QSA sparse decode reader for groups of query rows that share one selection
// list: the MTP (multi-token prediction) decode batch, where the draft tokens
// of a sequence attend to the same selected cache tokens (config 4: 12
// sequences x 4 rows, 12 query heads per kv head).  Included by
// sparse_attention.cu inside namespace nvqsa::{anonymous}; uses its parameter
// block, barrier, copy, conversion and cluster helpers.
//
// One CTA of 8 warps = (group of up to 4 consecutive rows, kv head, split),
// one CTA per SM.  Each selected record is gathered ONCE (tile::gather4) into a
// CTA-wide ring of 16 tiles of 16 records that runs up to 6 steps ahead.  A
// step is 32 tokens (two tiles); in iteration i, between two CTA barriers:
//   * warps 0-3 (S warps): warp w computes the scores of row w of the group
//     (its query heads in one m16 tile) over step i's dequantised K tile,
//     runs that row's online softmax and writes P into a shared tile of the
//     group's packed heads (up to 48 = 3 m16 tiles);
//   * warps 4-7 (K warps), at the same time: warp 4 + j dequantises dims
//     [64j, 64j + 64) of step i+1's K into the other half of a double-buffered
//     f16 tile (exact: e2m1 x e4m3), then accumulates O += P V of step i-1
//     over the same dims of every packed head (24 m16n8 fragments, 96 fp32
//     registers), V dequantised in registers from the ring; warp 4 also
//     refills the ring.
// K, P and the rescale factors are double-buffered, so one barrier per step
// orders everything and the scores of a step overlap the P V of the one before.
// The gather and the dequantisation are paid once per record for all rows of
// the group instead of once per row.
//
// Sharing is verified on the device, never assumed: each CTA compares the
// rows' request and the index positions of its chunks against the group's
// first row, and the CTAs of a cluster agree on the result.  A group that does
// not share is processed row by row (one pass per row, one active S warp).
// The ring is filled from the first row's selections before that check
// completes, so the first copies overlap it and the Q preparation.
//
// Splits of a group form one thread-block cluster (up to 8 CTAs): every rank
// publishes its (O, m, l) in shared memory, then every rank merges one slice
// of the output fragments of all ranks over distributed shared memory and
// stores it.

constexpr int kMtpWarps = 8;
constexpr int kMtpThreads = 32 * kMtpWarps;
constexpr int kMtpRing = 16;          // ring stages (tiles of 16 records): 8 steps
constexpr int kMtpStep = 2 * kTile;   // tokens per step: two tiles per CTA barrier
constexpr int kMtpHeads = 48;         // packed query heads of a group (rows x group size)
constexpr int kMtpMTiles = 3;         // m16 tiles of packed heads
constexpr int kKhStride = 264;        // halfs per token row of the dequantised K tile (256 + 8: ldmatrix conflict-free)
constexpr int kPhStride = 40;         // halfs per head row of the P tile (32 + 8: ldmatrix conflict-free)
constexpr int kMtpRows = 4;           // rows per group (one S warp each)
constexpr int kMtpMaxCluster = 8;     // splits of a group: one portable cluster
constexpr int kMtpCompactIters = kMaxRange / kMtpThreads;

struct __align__(128) SmemMtp {
  uint8_t rec[kMtpRing][kStageBytes];     // gather ring; after the last tile it holds the published O
  __half kh[2][kMtpStep][kKhStride];      // dequantised K of a step, double-buffered
  uint4 qf[kMtpRows][16][33];             // Q A-fragments of each row: [row][k-step][lane] (+1: conflict-free stores)
  __half ph[2][kMtpHeads][kPhStride];     // P of a step (packed heads x tokens), double-buffered
  int32_t sel[kMaxRange];                 // record rows (gather4) of the valid selections of the pass
  float alpha[2][kMtpHeads];              // rescale factor of each packed head (read only when its row rescaled)
  int resc[2][kMtpRows];                  // row rescaled its running max in this step
  float smul[kMtpHeads];
  float m_s[kMtpHeads];
  float l_s[kMtpHeads];
  unsigned long long full_bar[kMtpRing];
  int cnt[kMtpCompactIters][kMtpWarps];
  int total;
  int abort;
  int shared_ok;
};
static_assert(sizeof(float4) * kMtpRows * kMtpMTiles * 8 * 32 <= sizeof(SmemMtp::rec), "published O must fit the ring");
static_assert(sizeof(float) * kMtpMaxCluster * kMtpHeads <= sizeof(SmemMtp::ph), "merge weights must fit the P tile");

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& d0, uint32_t& d1, uint32_t& d2, uint32_t& d3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
               : "r"(addr));
}

__global__ void __launch_bounds__(kMtpThreads, 1) sparse_attention_mtp_kernel(const __grid_constant__ AttnParams p) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  SmemMtp& sm = *reinterpret_cast<SmemMtp*>(smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u));

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int r = lane >> 2;  // mma group row
  const int c = lane & 3;   // mma thread-in-group
  const int G = p.group;

  int64_t bid = blockIdx.x;
  const int split = (int)(bid % p.splits);
  bid /= p.splits;
  const int kvh = (int)(bid % p.kv_heads);
  const int64_t grp = bid / p.kv_heads;
  const int64_t row_lo = grp * p.group_rows;
  const int64_t unit = grp * p.kv_heads + kvh;  // timing stamps: 0 entry, 2 prologue done, 1 tiles done, 6 stored
  if (tid == 0) stamp_min(p, unit, 0);
  const int nrows = (int)min((int64_t)p.group_rows, p.rows - row_lo);

  const int64_t chunks = (p.topk + kChunk - 1) / kChunk;
  const int my_chunks = split < chunks ? (int)((chunks - 1 - split) / p.splits + 1) : 0;  // <= kMaxChunks
  const int iters = (my_chunks + kMtpWarps - 1) / kMtpWarps;

  if (tid == 0) {
#pragma unroll
    for (int b = 0; b < kMtpRing; ++b) mbar_init(smem_u32(&sm.full_bar[b]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    sm.abort = 0;
  }

  // Selections of row `prow` for this CTA's chunks -> record rows (gather4), -1 when masked
  // (kernels.py:236-257).
  const bool huge_page = p.page_size > 0x7fffffffLL;
  int32_t rowid[kMtpCompactIters];
  auto load_selections = [&](int64_t prow) {
    const int32_t req = __ldg(p.token_to_request + prow);
    const int32_t* idx_row = p.indices + prow * p.topk;
    int32_t iv[kMtpCompactIters];
#pragma unroll
    for (int it = 0; it < kMtpCompactIters; ++it) {
      const int lc = it * kMtpWarps + warp;
      const int64_t pos = ((int64_t)split + (int64_t)lc * p.splits) * kChunk + lane;
      iv[it] = (lc < my_chunks && pos < p.topk) ? __ldg(idx_row + pos) : -1;
    }
    const bool req_ok = req >= 0 && (int64_t)req < p.num_requests;
    const int32_t* bt_row = p.block_table + (req_ok ? (int64_t)req * p.table_width : 0);
#pragma unroll
    for (int it = 0; it < kMtpCompactIters; ++it) {
      rowid[it] = -1;
      const int32_t idx = iv[it];
      if (req_ok && idx >= 0) {
        const uint32_t lpage = huge_page ? 0u : (uint32_t)idx / (uint32_t)p.page_size;
        if ((int64_t)lpage < p.table_width) {
          const int32_t phys = __ldg(bt_row + lpage);
          const int32_t off = huge_page ? idx : (int)((uint32_t)idx - lpage * (uint32_t)p.page_size);
          if (phys >= 0 && (int64_t)phys < p.num_blocks) rowid[it] = (phys * p.kv_heads + kvh) * (int32_t)p.page_size + off;
        }
      }
    }
  };
  // The valid selections, in chunk order, into sm.sel; returns their count (two CTA barriers).
  auto compact = [&]() -> int {
    uint32_t vmask = 0;
    int pre[kMtpCompactIters];
#pragma unroll
    for (int it = 0; it < kMtpCompactIters; ++it) {
      pre[it] = 0;
      if (it < iters) {
        const bool valid = rowid[it] >= 0;
        const uint32_t b = __ballot_sync(0xffffffffu, valid);
        pre[it] = __popc(b & ((1u << lane) - 1u));
        if (valid) vmask |= 1u << it;
        if (lane == 0) sm.cnt[it][warp] = __popc(b);
      }
    }
    __syncthreads();
    int base_all = 0;
#pragma unroll
    for (int it = 0; it < kMtpCompactIters; ++it) {
      if (it < iters) {
        int base = base_all;
        for (int w = 0; w < warp; ++w) base += sm.cnt[it][w];
        if (vmask & (1u << it)) sm.sel[base + pre[it]] = rowid[it];
#pragma unroll
        for (int w = 0; w < kMtpWarps; ++w) base_all += sm.cnt[it][w];
      }
    }
    __syncthreads();
    return base_all;
  };

  // Ring: tile k of a pass is global tile tiles_done + k, in stage (that) % kMtpRing.  Warp 4 issues.
  int tiles_done = 0;  // tiles consumed in earlier passes: ring stage and phase carry over
  auto issue_tile = [&](int k, int n) {
    const int g = tiles_done + k;
    const int st = g % kMtpRing;
    const uint32_t bar = smem_u32(&sm.full_bar[st]);
    const int j0 = k * kTile;
    const int count = min(kTile, n - j0);
    // the stage was last read by generic loads (ordered before the barrier that let us here)
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)kStageBytes);
    __syncwarp();
    if (lane < kTile / 4) {
      int32_t rw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = group_token(lane, j);
        rw[j] = t < count ? sm.sel[j0 + t] : p.total_rows;  // out of range: zero fill
      }
      gather4_g2s(smem_u32(&sm.rec[st][lane * 4 * kRecordBytes]), &p.rows_map, rw[0], rw[1], rw[2], rw[3], bar);
    }
  };
  auto tile_wait = [&](int k) -> bool {
    const int g = tiles_done + k;
    return mbar_wait(smem_u32(&sm.full_bar[g % kMtpRing]), (uint32_t)((g / kMtpRing) & 1));
  };

  // Q of row `qrow0 + warp` for an S warp: lane L holds dims [8L, 8L + 8) of each head (zero past the active
  // rows and heads).  Pass 0's are loaded first, so their latency overlaps the selection loads.
  uint32_t qw[16][4];
  auto load_q = [&](int64_t qrow0, int act) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      qw[j][0] = qw[j][1] = qw[j][2] = qw[j][3] = 0u;
      if (warp < act && j < G) {
        const __nv_bfloat16* qrow =
            p.q + (qrow0 + warp) * p.q_stride_row + (int64_t)(kvh * G + j) * p.q_stride_head + lane * 8;
        if (p.vec_q) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(qrow));
          qw[j][0] = v.x; qw[j][1] = v.y; qw[j][2] = v.z; qw[j][3] = v.w;
        } else {
          const unsigned short* qs = reinterpret_cast<const unsigned short*>(qrow);
#pragma unroll
          for (int t = 0; t < 4; ++t) qw[j][t] = (uint32_t)__ldg(qs + 2 * t) | ((uint32_t)__ldg(qs + 2 * t + 1) << 16);
        }
      }
    }
  };
  if (warp < kMtpRows) load_q(row_lo, nrows);

  // pass 0 always follows the group's first row: its copies start before the sharing check
  load_selections(row_lo);
  int n = compact();
  if (warp == 4) {
    const int nt = (n + kTile - 1) / kTile;
    for (int k = 0; k < kMtpRing && k < nt; ++k) issue_tile(k, n);
  }

  // ---------- do the group's rows share request and selections? (this CTA's chunks; verdict deferred) ----------
  // Pass 0 runs speculatively as if they did: the ring follows the first row's selections, whose S warp 0
  // result is right either way, and S warps 1-3 score their rows against the same records.  The loads below
  // are compared once the pass's first copies are on their way; the CTA's verdict is taken at the end of the
  // pass and the cluster's at its merge barrier.  A group that does not share keeps only row 0's output of
  // pass 0 and processes its other rows one per pass.
  int32_t shv[kMtpCompactIters][kMtpRows];
  int32_t shr[kMtpRows];
  {
    const int32_t* idx0 = p.indices + row_lo * p.topk;
#pragma unroll
    for (int i = 0; i < kMtpRows; ++i) shr[i] = i < nrows ? __ldg(p.token_to_request + row_lo + i) : 0;
#pragma unroll
    for (int it = 0; it < kMtpCompactIters; ++it) {
      const int lc = it * kMtpWarps + warp;
      const int64_t pos = ((int64_t)split + (int64_t)lc * p.splits) * kChunk + lane;
      const bool in = lc < my_chunks && pos < p.topk;
#pragma unroll
      for (int i = 0; i < kMtpRows; ++i) shv[it][i] = (in && i < nrows) ? __ldg(idx0 + (int64_t)i * p.topk + pos) : 0;
    }
  }
  auto shares = [&]() -> bool {
    bool ok = true;
#pragma unroll
    for (int i = 1; i < kMtpRows; ++i) {
      if (i >= nrows) break;
      ok &= shr[i] == shr[0];
#pragma unroll
      for (int it = 0; it < kMtpCompactIters; ++it) ok &= shv[it][i] == shv[it][0];
    }
    return ok;
  };
  bool same_local = true;  // this thread's share of the check (set during pass 0's prologue)
  bool same = true;        // the cluster's verdict (known at the end of pass 0)
  int passes = nrows;      // 1 once pass 0 finds that the group shares
  bool aborted = false;

  // ldmatrix row addresses: K (tokens x dims) for B of S, P (heads x tokens) for A of P V
  const uint32_t kh_lane = (uint32_t)(((((lane >> 4) << 3) + (lane & 7)) * kKhStride + ((lane >> 3) & 1) * 8) * 2);
  const uint32_t ph_lane = (uint32_t)((((lane & 7) + ((lane >> 3) & 1) * 8) * kPhStride + (lane >> 4) * 8) * 2);
  const int vtok[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
  const bool kwarp = warp >= kMtpRows;

  // K warp 4 + j: dequantise dims [64j, 64j + 64) of tile kk (lane -> token lane/2, dims 64j + 32 (lane % 2) + [0, 32))
  // into rows [16u, 16u + 16) of kh[buf]
  auto dequant_k = [&](int kk, int buf, int u) {
    const int j = warp - kMtpRows;
    const int t = lane >> 1, h = lane & 1;
    const uint8_t* rec = sm.rec[(tiles_done + kk) % kMtpRing] + slot_off(t);
    const uint4 kb = *reinterpret_cast<const uint4*>(rec + 32 * j + 16 * h);
    const uint32_t sc = cvt_e4m3x2_f16x2(*reinterpret_cast<const uint16_t*>(rec + 128 + 4 * j + 2 * h));
    const uint32_t s0 = dup_lo(sc), s1 = dup_hi(sc);
    const uint32_t wd[4] = {kb.x, kb.y, kb.z, kb.w};
    uint32_t o[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t sg = q < 2 ? s0 : s1;
      o[4 * q + 0] = hmul2_u32(cvt_e2m1x2_f16x2_byte<0>(wd[q]), sg);
      o[4 * q + 1] = hmul2_u32(cvt_e2m1x2_f16x2_byte<1>(wd[q]), sg);
      o[4 * q + 2] = hmul2_u32(cvt_e2m1x2_f16x2_byte<2>(wd[q]), sg);
      o[4 * q + 3] = hmul2_u32(cvt_e2m1x2_f16x2_byte<3>(wd[q]), sg);
    }
    uint4* dst = reinterpret_cast<uint4*>(&sm.kh[buf][kTile * u + t][64 * j + 32 * h]);
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
  };

  // Every rank of a cluster takes every pass (their cluster barriers must pair up), aborted or not.
  for (int pass = 0; pass < passes; ++pass) {
    const int64_t prow = row_lo + pass;     // row whose selections the gather follows
    const int act = pass == 0 ? nrows : 1;  // active S warps (rows) of this pass (pass 0: speculatively all)
    const bool live = !aborted;                          // this pass issues copies
    if (pass > 0 && live) {  // a group that does not share: row prow alone, on S warp 0
      load_selections(prow);
      n = compact();
      if (warp == 4) {
        const int nt = (n + kTile - 1) / kTile;
        for (int k = 0; k < kMtpRing && k < nt; ++k) issue_tile(k, n);
      }
    }
    const int ntiles = (n + kTile - 1) / kTile;
    const int nsteps = (ntiles + 1) / 2;

    // ---------------- S warps: Q of their row; K warps: K of step 0 ----------------
    bool ok = true;
    if (!kwarp) {
      if (pass > 0) load_q(prow, act);
      if (warp >= act) {  // pass 0 loaded every row of the group; a row-by-row pass keeps only its own
#pragma unroll
        for (int j = 0; j < 16; ++j) qw[j][0] = qw[j][1] = qw[j][2] = qw[j][3] = 0u;
      }
      // per-head power-of-two pre-scale (exact) into f16 A-fragments of the row's m16 tile (natural dim
      // order: k-step s covers dims [16s, 16s + 16)); heads >= G stay zero
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        uint32_t amax = 0;
#pragma unroll
        for (int t = 0; t < 4; ++t) amax = max(amax, max((qw[j][t] << 16) & 0x7fffffffu, qw[j][t] & 0x7fff0000u));
        amax = __reduce_max_sync(0xffffffffu, amax);
        // scale 2^e brings the head's amax to [2^14, 2^15); |e| <= 100 keeps both products exact
        int e = 0;
        if (amax >= 0x00800000u && amax < 0x7f800000u) e = max(-100, min(100, 14 - ((int)(amax >> 23) - 127)));
        if (lane == 0 && j < G && warp < act) sm.smul[warp * G + j] = p.score_scale * __int_as_float((127 - e) << 23);
        const float mul = __int_as_float((127 + e) << 23);
        // lane L holds dims 8L..8L+7 = k-step L/2, columns 8(L%2)..+7: pairs (2cc, 2cc+1) of half L%2
        const int s = lane >> 1, hi = lane & 1;
        uint32_t* f = reinterpret_cast<uint32_t*>(&sm.qf[warp][s][0]);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint32_t x = qw[j][cc];
          // register 2*hi + (j >= 8) of lane (j % 8) * 4 + cc
          f[((j & 7) * 4 + cc) * 4 + 2 * hi + (j >> 3)] = pack_half2(bf16_lo(x) * mul, bf16_hi(x) * mul);
        }
      }
      if (pass == 0) same_local = shares();
      // P rows of inactive heads stay zero for the whole pass
      for (int i = tid; i < 2 * kMtpHeads * kPhStride / 2; i += 32 * kMtpRows)
        reinterpret_cast<uint32_t*>(&sm.ph[0][0][0])[i] = 0u;
    } else if (ntiles > 0 && live) {
      ok &= tile_wait(0);
      if (ok) dequant_k(0, 0, 0);
      if (ntiles > 1) {
        ok &= tile_wait(1);
        if (ok) dequant_k(1, 0, 1);
      }
    }
    if (kwarp && pass == 0) same_local = shares();
    if (!__syncthreads_and(ok)) {
      aborted = true;
      if (tid == 0) sm.abort = 1;
    }
    if (tid == 0 && pass == 0) stamp_max(p, unit, 2);

    // O accumulators (K warps): dims [64j, 64j + 64) of every packed head, j = warp - 4
    float oacc[kMtpMTiles][8][4];
#pragma unroll
    for (int t = 0; t < kMtpMTiles; ++t)
#pragma unroll
      for (int j = 0; j < 8; ++j) oacc[t][j][0] = oacc[t][j][1] = oacc[t][j][2] = oacc[t][j][3] = 0.0f;
    const bool srow = !kwarp && warp < act;  // this warp runs a row's scores and softmax
    const float smul_r = (srow && r < G) ? sm.smul[warp * G + r] : 1.0f;
    const float smul_r8 = (srow && r + 8 < G) ? sm.smul[warp * G + r + 8] : 1.0f;
    float m_r = kMaskedScore, m_r8 = kMaskedScore;
    float l_r = 0.0f, l_r8 = 0.0f;

    // Iteration i: S warps score step i (tiles 2i, 2i+1) from kh[i & 1] and write P into ph[i & 1]; K warps
    // dequantise step i+1 into kh[(i + 1) & 1] (warp 4 first refills the stages of step i-2, whose last read
    // was P V of step i-2 in the previous iteration) and accumulate P V of step i-1; one CTA barrier.
    int i = 0;
    for (; i <= nsteps && !aborted; ++i) {
      bool okk = true;
      if (kwarp) {
        const int k0 = 2 * i;
        if (warp == 4 && i >= 2) {
          if (k0 + kMtpRing - 4 < ntiles) issue_tile(k0 + kMtpRing - 4, n);
          if (k0 + kMtpRing - 3 < ntiles) issue_tile(k0 + kMtpRing - 3, n);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int kk = k0 + 2 + u;
          if (kk < ntiles) {
            okk &= tile_wait(kk);
            if (okk) dequant_k(kk, (i + 1) & 1, u);
          }
        }
        if (i >= 1 && okk) {
          // ---- O += P V of step i-1 over dims [64j, 64j + 64) of every packed head, one k-step per tile ----
          const int kw = warp - kMtpRows;
          const int pb = (i - 1) & 1;
          const int kp = 2 * (i - 1);
          const bool two = kp + 1 < ntiles;
          const int any = sm.resc[pb][0] | sm.resc[pb][1] | sm.resc[pb][2] | sm.resc[pb][3];
          if (any) {
#pragma unroll
            for (int t = 0; t < kMtpMTiles; ++t) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int head = 16 * t + r + 8 * hh;
                const int hrow = head / G;
                const float a = (head < act * G && sm.resc[pb][hrow]) ? sm.alpha[pb][head] : 1.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  oacc[t][j][2 * hh] *= a;
                  oacc[t][j][2 * hh + 1] *= a;
                }
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (u == 1 && !two) break;  // no stale V enters O
            const uint8_t* stage = sm.rec[(tiles_done + kp + u) % kMtpRing];
            uint32_t pa[kMtpMTiles][4];
            const uint32_t paddr = smem_u32(&sm.ph[pb][0][0]) + ph_lane + (uint32_t)(kTile * 2 * u);
#pragma unroll
            for (int t = 0; t < kMtpMTiles; ++t)
              ldsm_x4(paddr + (uint32_t)(16 * kPhStride * 2 * t), pa[t][0], pa[t][1], pa[t][2], pa[t][3]);
            // lane (r, c): tokens {2c, 2c+1, 2c+8, 2c+9} of the tile, dims 64j + 8r + [0, 8)
            uint32_t vw[4], vsb[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint8_t* rec = stage + slot_off(vtok[q]);
              vw[q] = *reinterpret_cast<const uint32_t*>(rec + 144 + 32 * kw + 4 * r);
              vsb[q] = rec[272 + 4 * kw + (r >> 1)];
            }
            const uint32_t s01 = cvt_e4m3x2_f16x2(vsb[0] | (vsb[1] << 8));
            const uint32_t s23 = cvt_e4m3x2_f16x2(vsb[2] | (vsb[3] << 8));
            // low nibbles (even dims) of two tokens interleaved into one byte; high nibbles (odd dims) likewise
            const uint32_t x01 = (vw[0] & 0x0f0f0f0fu) | ((vw[1] & 0x0f0f0f0fu) << 4);
            const uint32_t y01 = ((vw[0] >> 4) & 0x0f0f0f0fu) | (vw[1] & 0xf0f0f0f0u);
            const uint32_t x23 = (vw[2] & 0x0f0f0f0fu) | ((vw[3] & 0x0f0f0f0fu) << 4);
            const uint32_t y23 = ((vw[2] >> 4) & 0x0f0f0f0fu) | (vw[3] & 0xf0f0f0f0u);
            // n-tile 2B + x, column n <-> dim 64j + 8n + 2B + x
#define NVQSA_MTP_PV_BYTE(B)                                                                     \
  {                                                                                              \
    const uint32_t bx0 = hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(x01), s01);                         \
    const uint32_t bx1 = hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(x23), s23);                         \
    const uint32_t by0 = hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(y01), s01);                         \
    const uint32_t by1 = hmul2_u32(cvt_e2m1x2_f16x2_byte<B>(y23), s23);                         \
    _Pragma("unroll") for (int t = 0; t < kMtpMTiles; ++t) {                                     \
      mma_f16(oacc[t][2 * (B)], pa[t][0], pa[t][1], pa[t][2], pa[t][3], bx0, bx1);               \
      mma_f16(oacc[t][2 * (B) + 1], pa[t][0], pa[t][1], pa[t][2], pa[t][3], by0, by1);           \
    }                                                                                            \
  }
            NVQSA_MTP_PV_BYTE(0)
            NVQSA_MTP_PV_BYTE(1)
            NVQSA_MTP_PV_BYTE(2)
            NVQSA_MTP_PV_BYTE(3)
#undef NVQSA_MTP_PV_BYTE
          }
        }
      } else if (i < nsteps) {
        const int buf = i & 1;
        if (srow) {
          // ---- S = Q K^T for row `warp` over the step's 32 tokens, online softmax, P into the packed tile ----
          // (a missing second tile leaves stale K rows: their scores are masked below)
          float sacc[4][4];
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
          const uint32_t kaddr = smem_u32(&sm.kh[buf][0][0]) + kh_lane;
#pragma unroll
          for (int s = 0; s < 16; ++s) {
            uint32_t b0, b1, b2, b3, b4, b5, b6, b7;
            ldsm_x4(kaddr + 32u * s, b0, b1, b2, b3);
            ldsm_x4(kaddr + (uint32_t)(kTile * kKhStride * 2) + 32u * s, b4, b5, b6, b7);
            const uint4 qa = sm.qf[warp][s][lane];
            mma_f16(sacc[0], qa.x, qa.y, qa.z, qa.w, b0, b1);
            mma_f16(sacc[1], qa.x, qa.y, qa.z, qa.w, b2, b3);
            mma_f16(sacc[2], qa.x, qa.y, qa.z, qa.w, b4, b5);
            mma_f16(sacc[3], qa.x, qa.y, qa.z, qa.w, b6, b7);
          }
          const int tok_base = i * kMtpStep;
          const bool tail = tok_base + kMtpStep > n;
          if (tail) {
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
              const int t0 = tok_base + 8 * nt + 2 * c;
              if (t0 >= n) { sacc[nt][0] = -1.0e30f; sacc[nt][2] = -1.0e30f; }
              if (t0 + 1 >= n) { sacc[nt][1] = -1.0e30f; sacc[nt][3] = -1.0e30f; }
            }
          }
          float mx_r = fmaxf(fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1])),
                             fmaxf(fmaxf(sacc[2][0], sacc[2][1]), fmaxf(sacc[3][0], sacc[3][1])));
          float mx_r8 = fmaxf(fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3])),
                              fmaxf(fmaxf(sacc[2][2], sacc[2][3]), fmaxf(sacc[3][2], sacc[3][3])));
          mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 1));
          mx_r = fmaxf(mx_r, __shfl_xor_sync(0xffffffffu, mx_r, 2));
          mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 1));
          mx_r8 = fmaxf(mx_r8, __shfl_xor_sync(0xffffffffu, mx_r8, 2));
          mx_r *= smul_r;
          mx_r8 *= smul_r8;
          const bool up_r = mx_r > m_r + kRescaleThreshold;
          const bool up_r8 = mx_r8 > m_r8 + kRescaleThreshold;
          const bool up = __any_sync(0xffffffffu, up_r || up_r8);
          if (up) {
            const float mn_r = up_r ? mx_r : m_r, mn_r8 = up_r8 ? mx_r8 : m_r8;
            const float a_r = ex2(m_r - mn_r), a_r8 = ex2(m_r8 - mn_r8);
            m_r = mn_r;
            m_r8 = mn_r8;
            l_r *= a_r;
            l_r8 *= a_r8;
            if (c == 0) {
              if (r < G) sm.alpha[buf][warp * G + r] = a_r;
              if (r + 8 < G) sm.alpha[buf][warp * G + r + 8] = a_r8;
            }
          }
          if (lane == 0) sm.resc[buf][warp] = up ? 1 : 0;
          float pv[4][4];
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            pv[nt][0] = ex2(fmaf(sacc[nt][0], smul_r, -m_r));
            pv[nt][1] = ex2(fmaf(sacc[nt][1], smul_r, -m_r));
            pv[nt][2] = ex2(fmaf(sacc[nt][2], smul_r8, -m_r8));
            pv[nt][3] = ex2(fmaf(sacc[nt][3], smul_r8, -m_r8));
          }
          if (tail) {  // masked scores must not count even while the running max is still -1e20
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
              const int t0 = tok_base + 8 * nt + 2 * c;
              if (t0 >= n) { pv[nt][0] = 0.0f; pv[nt][2] = 0.0f; }
              if (t0 + 1 >= n) { pv[nt][1] = 0.0f; pv[nt][3] = 0.0f; }
            }
          }
          l_r += ((pv[0][0] + pv[0][1]) + (pv[1][0] + pv[1][1])) + ((pv[2][0] + pv[2][1]) + (pv[3][0] + pv[3][1]));
          l_r8 += ((pv[0][2] + pv[0][3]) + (pv[1][2] + pv[1][3])) + ((pv[2][2] + pv[2][3]) + (pv[3][2] + pv[3][3]));
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            if (r < G)
              *reinterpret_cast<uint32_t*>(&sm.ph[buf][warp * G + r][8 * nt + 2 * c]) = pack_half2(pv[nt][0], pv[nt][1]);
            if (r + 8 < G)
              *reinterpret_cast<uint32_t*>(&sm.ph[buf][warp * G + r + 8][8 * nt + 2 * c]) =
                  pack_half2(pv[nt][2], pv[nt][3]);
          }
        } else if (lane == 0) {
          sm.resc[buf][warp] = 0;
        }
      }
      if (!__syncthreads_and(okk)) {  // step i's P and step i+1's K in place; P V of step i-1 done
        if (tid == 0) sm.abort = 1;
        aborted = true;
        break;
      }
    }
    if (aborted && live && warp == 4) {
      // let copies still in flight land (bounded) before the ring is reused or released
      // tiles below 2i were waited for; warp 4 issued up to tile max(16, 2i + 14) - 1
      for (int k2 = 2 * i; k2 < ntiles && k2 < max(kMtpRing, 2 * i + kMtpRing - 2); ++k2) {
        const int g = tiles_done + k2;
        mbar_wait(smem_u32(&sm.full_bar[g % kMtpRing]), (uint32_t)((g / kMtpRing) & 1), kDrainSpinLimit);
      }
    }
    tiles_done += ntiles;

    // ---------------- per-head (m, l) of the active rows ----------------
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
    l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 1);
    l_r8 += __shfl_xor_sync(0xffffffffu, l_r8, 2);
    if (srow && c == 0) {
      if (r < G) { sm.m_s[warp * G + r] = m_r; sm.l_s[warp * G + r] = l_r; }
      if (r + 8 < G) { sm.m_s[warp * G + r + 8] = m_r8; sm.l_s[warp * G + r + 8] = l_r8; }
    }
    // (m, l) visible; no copy in flight, the ring is free; pass 0: this CTA's sharing verdict
    const bool cta_same = __syncthreads_and(pass == 0 ? same_local : true) != 0;
    aborted = sm.abort != 0;
    if (pass == 0 && p.cluster <= 1) {
      same = cta_same;
      passes = same ? 1 : nrows;
    }

    // rows whose output this pass stores (read after the cluster's verdict)
    auto act_out = [&]() { return pass == 0 && !same ? 1 : act; };
    if (tid == 0) stamp_max(p, unit, 1);
    // bf16 output of packed head `head` (< act_out * G)
    auto out_ptr = [&](int head) {
      const int hrow = head / G, j = head - hrow * G;
      return p.out + (prow + hrow) * p.o_stride_row + (int64_t)(kvh * G + j) * p.o_stride_head;
    };
    const int kw = warp - kMtpRows;  // K warp index: its O covers dims [64 kw, 64 kw + 64)
    if (p.cluster > 1) {
      // Every rank publishes its (O, m, l); then every K warp of every rank merges one slice of its O fragments
      // over all ranks (fragment f = 8t + n-tile, slice [24 rank / C, 24 (rank + 1) / C)) through distributed
      // shared memory and stores it, with per-head weights 2^(m_rank - M) / sum.  The sharing verdicts, the
      // abort flags and the per-head (m, l) of every rank are loaded in one round before the CTA barriers that
      // agree on the verdict and publish the weights; then the fragments, two at a time from every rank.
      float4* pub = reinterpret_cast<float4*>(&sm.rec[0][0]);  // [K warp][24][32]
      if (!aborted && kwarp) {
#pragma unroll
        for (int t = 0; t < kMtpMTiles; ++t)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            pub[(kw * 24 + t * 8 + j) * 32 + lane] = make_float4(oacc[t][j][0], oacc[t][j][1], oacc[t][j][2], oacc[t][j][3]);
      }
      if (tid == 0) sm.shared_ok = cta_same ? 1 : 0;
      cluster_sync();
      const int C = p.cluster;
      const int rank = split % C;
      const int f_lo = rank * 24 / C, f_hi = (rank + 1) * 24 / C;
      float4 v[2][kMtpMaxCluster];
#define NVQSA_MTP_LOAD_PAIR(F0)                                                                              \
  _Pragma("unroll") for (int q = 0; q < 2; ++q) {                                                          \
    const uint32_t off = (uint32_t)((kw * 24 + min((F0) + q, f_hi - 1)) * 32 + lane) * 16u;                \
    _Pragma("unroll") for (int rk = 0; rk < kMtpMaxCluster; ++rk) v[q][rk] =                               \
        rk < C ? cluster_ld_f4(cluster_map(smem_u32(pub), (uint32_t)rk) + off) : make_float4(0.f, 0.f, 0.f, 0.f); \
  }
      const int mine = tid < C ? cluster_ld_s32(cluster_map(smem_u32(&sm.shared_ok), (uint32_t)tid)) : 1;
      const int bad_rank = tid < C ? cluster_ld_s32(cluster_map(smem_u32(&sm.abort), (uint32_t)tid)) : 0;
      float mr[kMtpMaxCluster], lr[kMtpMaxCluster];
#pragma unroll
      for (int rk = 0; rk < kMtpMaxCluster; ++rk) {
        mr[rk] = kMaskedScore;
        lr[rk] = 0.0f;
        if (tid < kMtpHeads && rk < C) {
          mr[rk] = __int_as_float(cluster_ld_s32(cluster_map(smem_u32(&sm.m_s[tid]), (uint32_t)rk)));
          lr[rk] = __int_as_float(cluster_ld_s32(cluster_map(smem_u32(&sm.l_s[tid]), (uint32_t)rk)));
        }
      }
      if (pass == 0) {  // the cluster's sharing verdict: every rank takes the same passes
        same = __syncthreads_and(mine) != 0;
        passes = same ? 1 : nrows;
      }
      float* wts = reinterpret_cast<float*>(&sm.ph[0][0][0]);  // [cluster][48] merge weights (P space is free)
      if (tid < kMtpHeads && tid < act_out() * G) {
        float M = kMaskedScore;
#pragma unroll
        for (int rk = 0; rk < kMtpMaxCluster; ++rk) M = fmaxf(M, mr[rk]);
        float L = 0.0f;
#pragma unroll
        for (int rk = 0; rk < kMtpMaxCluster; ++rk) {
          mr[rk] = ex2(mr[rk] - M);
          L += mr[rk] * lr[rk];
        }
        // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
        const float inv = L > 0.0f ? p.inv_value_scale / fmaxf(L, 1.0e-20f) : 0.0f;
#pragma unroll
        for (int rk = 0; rk < kMtpMaxCluster; ++rk)
          if (rk < C) wts[rk * kMtpHeads + tid] = mr[rk] * inv;
      }
      if (!__syncthreads_or(bad_rank) && kwarp) {  // weights in place; no rank gave up
        for (int f0 = f_lo; f0 < f_hi; f0 += 2) {
          NVQSA_MTP_LOAD_PAIR(f0)
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int f = f0 + q;
            if (f >= f_hi) break;
            const int t = f >> 3, jn = f & 7;
            const int h0 = 16 * t + r, h1 = h0 + 8;
            const bool l0 = h0 < act_out() * G, l1 = h1 < act_out() * G;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int rk = 0; rk < kMtpMaxCluster; ++rk) {
              if (rk >= C) break;
              const float w0 = l0 ? wts[rk * kMtpHeads + h0] : 0.0f, w1 = l1 ? wts[rk * kMtpHeads + h1] : 0.0f;
              acc.x += w0 * v[q][rk].x; acc.y += w0 * v[q][rk].y; acc.z += w1 * v[q][rk].z; acc.w += w1 * v[q][rk].w;
            }
            // n-tile jn, columns 2c and 2c+1: dims 64kw + 16c + jn and 64kw + 16c + 8 + jn
            const int d = 64 * kw + 16 * c + jn;
            if (l0) {
              __nv_bfloat16* op = out_ptr(h0);
              op[d] = __float2bfloat16_rn(acc.x);
              op[d + 8] = __float2bfloat16_rn(acc.y);
            }
            if (l1) {
              __nv_bfloat16* op = out_ptr(h1);
              op[d] = __float2bfloat16_rn(acc.z);
              op[d + 8] = __float2bfloat16_rn(acc.w);
            }
          }
        }
      }
#undef NVQSA_MTP_LOAD_PAIR
      cluster_sync();  // every rank keeps its shared memory until all have read it
    } else if (!aborted && kwarp) {
      // one CTA per group: normalise and store every fragment from registers
#pragma unroll
      for (int t = 0; t < kMtpMTiles; ++t) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int head = 16 * t + r + 8 * hh;
          if (head >= act_out() * G) continue;
          const float l = sm.l_s[head];
          // kernels.py:333-337: acc / l when l > 0, else 0; then / value_global_scale
          const float inv = l > 0.0f ? p.inv_value_scale / fmaxf(l, 1.0e-20f) : 0.0f;
          // dims 64kw + 16c + i (n = 2c, n-tile i) and 64kw + 16c + 8 + i (n = 2c + 1)
          uint32_t wv[8];
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            __nv_bfloat162 lo2 = __floats2bfloat162_rn(oacc[t][2 * i2][2 * hh] * inv, oacc[t][2 * i2 + 1][2 * hh] * inv);
            __nv_bfloat162 hi2 =
                __floats2bfloat162_rn(oacc[t][2 * i2][2 * hh + 1] * inv, oacc[t][2 * i2 + 1][2 * hh + 1] * inv);
            wv[i2] = *reinterpret_cast<uint32_t*>(&lo2);
            wv[4 + i2] = *reinterpret_cast<uint32_t*>(&hi2);
          }
          __nv_bfloat16* op = out_ptr(head) + 64 * kw + 16 * c;
          if (p.vec_o) {
            reinterpret_cast<uint4*>(op)[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            reinterpret_cast<uint4*>(op)[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
          } else {
            unsigned short* os = reinterpret_cast<unsigned short*>(op);
#pragma unroll
            for (int i2 = 0; i2 < 8; ++i2) {
              os[2 * i2] = (unsigned short)(wv[i2] & 0xffffu);
              os[2 * i2 + 1] = (unsigned short)(wv[i2] >> 16);
            }
          }
        }
      }
    }
    __syncthreads();  // the next pass rewrites shared memory
  }
  if (tid == 0) stamp_max(p, unit, 6);
}
