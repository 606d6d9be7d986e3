// K/V projection GEMM with the NVFP4 cache writer as its epilogue, on the
// 5th-generation tensor cores.  Included by write_cache.cu inside namespace
// nvqsa::{anonymous}; uses its parameter block, scale table, encoder and slot
// helpers, so the bytes it writes are those of nvqsa_norm_rope_write_cache.
//
// The reference's attention layer computes qkv = hidden @ W_qkv^T (vLLM's
// QKVParallelLinear, bf16 output), splits K and V off it, runs k_norm and the
// rotary embedding on K and only then calls the writer
// (integration/snapshot/qsa.py:658-667 -> :618-640).  Here the K and V
// columns of that GEMM are computed and encoded in one launch, so the bf16 K
// and V never reach HBM unless key_out / value_out ask for them.
//
// One CTA = 128 MH tokens (MH = 1 or 2) x one head (256 columns) of K or of
// V.  The TMA warp streams 64-wide k-slices of the hidden rows (16 KB per 128
// tokens) and of the head's weight rows (32 KB) through a ring of stages with
// TMA (128-byte swizzle); one thread of the MMA warp issues, per 16-wide
// k-step and per 128-token half, a tcgen05.mma (M 128, N 256, K 16, bf16 ->
// fp32) into that half's 128 x 256 fp32 accumulator in tensor memory, and
// releases each stage with tcgen05.commit.  The 8 MH epilogue warps load
// each token's position, slot and cos/sin row during the mainloop; once the
// accumulators are complete two threads per token row (one lane of each of
// two warps on the row's tensor-memory lane) read the row back, round it to
// bf16 as the GEMM output would be, and run the writer's arithmetic on whole
// 16-element groups, 8 groups each: for K the RMS norm (the writer's
// summation order: each thread's partial sums go through shared memory and
// both add all 32 in that order), the rotation (bf16 arithmetic, NeoX halves
// or GPT-J pairs; a NeoX pair of groups stays in one thread), then the group
// scale and E2M1 codes; for V the codes alone.  Each row's 144 record bytes
// are staged in the freed stage buffers and written as 16-byte chunks,
// consecutive threads on consecutive chunks.
//
// Small batches (fewer 128-token tiles than SMs) split each tile's k-blocks
// over a thread-block cluster of up to 8 CTAs; the partial accumulators are
// summed over distributed shared memory in rank order (see the k-split block
// below) before the same epilogue runs on each rank's share of the rows.
constexpr int kPwBN = 256;        // columns per CTA: one head
constexpr int kPwBK = 64;         // k-slice per stage: 128 bytes of bf16 (one swizzle atom row)
constexpr uint32_t kPwStageB = kPwBN * kPwBK * 2;  // 32 KB
// MH halves of 128 tokens per CTA, each its own M = 128 accumulator (256 tensor-memory columns) fed by the
// same weight tile: MH = 2 halves the weight traffic per token.  8 MH epilogue warps (two threads per token
// row, each finishing 8 of its 16 groups), then the TMA and MMA warps.
template <int MH>
struct PwShape {
  static constexpr int kBM = 128 * MH;
  static constexpr int kStages = MH == 1 ? 4 : 3;
  static constexpr int kEpiWarps = 8 * MH;
  static constexpr int kThreads = 32 * (kEpiWarps + 2);
  static constexpr int kTmaWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1;
  static constexpr uint32_t kStageA = (uint32_t)kBM * kPwBK * 2;
  static constexpr uint32_t kTmemCols = 256u * MH;
};
constexpr uint32_t kPwSpinLimit = 1u << 24;        // bounded mbarrier waits (the mainloop is tens of us)
constexpr unsigned int kErrProjWait = 4u;          // bit 2 of the error flags: a projection-writer wait ran out

__device__ unsigned int g_write_error_flags;

template <int MH>
struct __align__(1024) SmemPw {
  uint8_t a[PwShape<MH>::kStages][PwShape<MH>::kStageA];  // hidden rows, swizzled 128-byte rows (1024-byte atoms)
  uint8_t b[PwShape<MH>::kStages][kPwStageB];             // weight rows
  float nw[kPwBN];  // norm weight + offset (fp32); at a multiple of 1024 bytes, read as float2
  unsigned long long full[PwShape<MH>::kStages];
  unsigned long long empty[PwShape<MH>::kStages];
  unsigned long long accum;
  uint32_t tmem;
  float lut[2][256];
  float quot[2][16];
};
constexpr int kPwRecRow = 144;   // staged record bytes per token row: 128 code bytes + 16 scale bytes
constexpr int kPwRedStride = 33;
constexpr int kPwPartStride = 260;  // floats per token row of a k-split partial (16-byte skew per row)  // floats per token row of the norm partials (conflict-free), in the free stages

struct ProjParams {
  CUtensorMap map_x;      // hidden [tokens, hidden] bf16, box 64 x (128 MH)
  CUtensorMap map_w[2];   // K / V weight rows [kv_heads * 256, hidden] bf16, box 64 x 256
  WriteParams w;          // cache regions, slots, scales, norm and rotation (head_dim 256, record layout)
  int32_t kblocks;        // hidden / 64, rounded up (the tail is zero-filled by TMA)
  int32_t ksplit;         // CTAs of a cluster splitting the k-blocks of one tile (1: no split, MH = 1 only)
  int32_t kbs;            // k-blocks per split rank (every rank has at least one)
  __nv_bfloat16* value_out;  // optional bf16 V projection [tokens, kv_heads, 256]
  int64_t value_out_stride_token, value_out_stride_head;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void pw_mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool pw_try_wait(uint32_t bar, uint32_t parity) {
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
__device__ __forceinline__ bool pw_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kPwSpinLimit; ++i)
    if (pw_try_wait(bar, parity)) return true;
  atomicOr(&g_write_error_flags, kErrProjWait);
  return false;
}
__device__ __forceinline__ void pw_tma_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Shared-memory matrix descriptor: K-major operand in 128-byte swizzled rows, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t pw_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3fffu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: D f32, A and B bf16, both K-major, N = 256, M = 128.
constexpr uint32_t kPwIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPwBN >> 3) << 17) |
                              ((uint32_t)(128 >> 4) << 24);

// Every thread of every CTA of the cluster arrives; shared-memory writes before it are visible after it.
__device__ __forceinline__ void pw_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ float4 pw_ld_cluster_f4(uint32_t addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}
__device__ __forceinline__ void pw_tmem_ld16(uint32_t taddr, float (&v)[16]) {
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
__device__ __forceinline__ void pw_tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])));
}

__device__ __forceinline__ void pw_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void pw_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's tensor-memory lane, rounded to bf16 pairs (the GEMM's output).
__device__ __forceinline__ void pw_load_bf16(uint32_t taddr, uint32_t (&w)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
}

// Two groups' columns with both loads in flight before one wait.
__device__ __forceinline__ void pw_load2_bf16(uint32_t ta, uint32_t tb, uint32_t (&wa)[8], uint32_t (&wb)[8]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(ta));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    wa[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    wb[i] = pack_bf16x2(__uint_as_float(r[16 + 2 * i]), __uint_as_float(r[17 + 2 * i]));
  }
}

template <int MH>
__global__ void __launch_bounds__(PwShape<MH>::kThreads, 1) kv_proj_write_kernel(const __grid_constant__ ProjParams p) {
  using S = PwShape<MH>;
  constexpr int kStages = S::kStages;
  extern __shared__ __align__(1024) uint8_t pw_smem_raw[];
  SmemPw<MH>& sm =
      *reinterpret_cast<SmemPw<MH>*>(pw_smem_raw + ((1024u - (smem_u32(pw_smem_raw) & 1023u)) & 1023u));
  const WriteParams& wp = p.w;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = wp.kv_heads;
  const int ks = p.ksplit;                 // CTAs of this tile's cluster, each with its own k-blocks
  const int rank = blockIdx.x % ks;
  const int nt = blockIdx.x / ks;  // 0 .. kvh-1: K head nt; kvh .. 2 kvh-1: V head nt - kvh
  const int kb0 = rank * p.kbs;
  const int r = nt < kvh ? 0 : 1;
  const int head = nt - r * kvh;
  const int64_t m0 = (int64_t)blockIdx.y * S::kBM;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      pw_mbar_init(smem_u32(&sm.full[s]), 1);
      pw_mbar_init(smem_u32(&sm.empty[s]), 1);
    }
    pw_mbar_init(smem_u32(&sm.accum), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == S::kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&sm.tmem)),
                 "r"(S::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  build_out_scale_lut(wp, sm.lut, sm.quot);
  if (wp.norm_weight != nullptr)
    for (int j = tid; j < kPwBN; j += S::kThreads) sm.nw[j] = __fadd_rn(__ldg(wp.norm_weight + j), wp.norm_offset);
  pw_fence_before();
  __syncthreads();
  pw_fence_after();
  const uint32_t tmem = sm.tmem;
  const int kb = min(p.kblocks - kb0, p.kbs);  // this CTA's k-blocks, from kb0

  // ---------------- epilogue rows: two threads per token row ----------------
  // warp w: lane quarter w % 4 of accumulator half (w / 4) % MH, column split c = w / (4 MH); split c
  // finishes the groups g with own(g) == c, keeping each NeoX pair (g, g + half/16) in one thread
  const int q = warp & 3, half_m = (warp >> 2) % MH, c = warp / (4 * MH);
  const int trow = 128 * half_m + 32 * q + lane;  // row inside the tile
  const int64_t row = m0 + trow;
  const bool live = warp < S::kEpiWarps && row < wp.num_tokens && (ks == 1 || trow / ((S::kBM + ks - 1) / ks) == rank);
  const int half = wp.rot_dim >> 1;
  const int P = wp.neox ? (half >> 4) : 0;  // NeoX: groups [0, P) pair with [P, 2P)
  auto own = [&](int g) -> int { return (g < 2 * P) ? (P == 1 ? 0 : (g % P) & 1) : (g & 1); };

  // per-row loads while the mainloop runs: position, slot, and the cos/sin row into L2
  int64_t pos = 0;
  bool pos_ok = live;
  if (live && wp.rot_dim > 0) {
    pos = __ldg(wp.positions + row);
    pos_ok = pos >= 0 && pos < wp.max_position;
    if (!pos_ok) pos = 0;
  }
  int64_t block = 0, offset = 0;
  bool slot_ok = pos_ok && slot_position<true>(wp, __ldg(wp.slots + row), block, offset);
  const __nv_bfloat16* cs = wp.cos_sin + pos * wp.cos_sin_stride;
  // cos/sin of this split's first rotation step (NeoX: 16 of each at 16c; GPT-J: 8 at 8c) into registers,
  // the rest of the row into L2
  uint32_t pre_c[8], pre_s[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) pre_c[i] = pre_s[i] = 0u;
  if (r == 0 && wp.rot_dim > 0 && warp < S::kEpiWarps) {
    if (wp.neox && 16 * c < half) {
      load_bf16_run<16>(cs + 16 * c, pre_c);
      load_bf16_run<16>(cs + half + 16 * c, pre_s);
    } else if (!wp.neox && 16 * c < wp.rot_dim) {
      uint32_t c4[4], s4[4];
      load_bf16_run<8>(cs + 8 * c, c4);
      load_bf16_run<8>(cs + half + 8 * c, s4);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pre_c[i] = c4[i];
        pre_s[i] = s4[i];
      }
    }
    if (c == 0)
      for (int b = 0; b < wp.rot_dim * 2; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(cs + b / 2));
  }

  if (warp == S::kTmaWarp) {
    // ---------------- producer: TMA into the stage ring ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < kb; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !pw_wait(smem_u32(&sm.empty[s]), (uint32_t)(((i / kStages) & 1) ^ 1))) break;
        const uint32_t full = smem_u32(&sm.full[s]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(full),
                     "r"(S::kStageA + kPwStageB)
                     : "memory");
        pw_tma_2d(smem_u32(sm.a[s]), &p.map_x, (kb0 + i) * kPwBK, (int32_t)m0, full);
        pw_tma_2d(smem_u32(sm.b[s]), &p.map_w[r], (kb0 + i) * kPwBK, head * kPwBN, full);
        issued = i + 1;
      }
      // copies still in flight land before the CTA can leave (only a timed-out consumer leaves them)
      for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
        pw_wait(smem_u32(&sm.full[j % kStages]), (uint32_t)((j / kStages) & 1));
    }
    __syncwarp();
  } else if (warp == S::kMmaWarp) {
    // ---------------- MMA issue: one thread ----------------
    if (lane == 0) {
      for (int i = 0; i < kb; ++i) {
        const int s = i % kStages;
        if (!pw_wait(smem_u32(&sm.full[s]), (uint32_t)((i / kStages) & 1))) break;
        pw_fence_after();
        const uint64_t db = pw_desc(smem_u32(sm.b[s]));
#pragma unroll
        for (int k = 0; k < kPwBK / 16; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
#pragma unroll
          for (int h = 0; h < MH; ++h) {
            // half h: A rows [128 h, 128 h + 128) (16 KB further), accumulator columns [256 h, 256 h + 256);
            // advancing the start address by 32 bytes steps 16 elements along K inside the swizzled row
            const uint64_t da = pw_desc(smem_u32(sm.a[s]) + 16384u * h);
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem + 256u * h),
                "l"(da + (uint64_t)(2 * k)), "l"(db + (uint64_t)(2 * k)), "r"(kPwIdesc), "r"(acc)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                         smem_u32(&sm.empty[s]))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                       smem_u32(&sm.accum))
                   : "memory");
    }
    __syncwarp();
  }

  // ---------------- k-split: sum the cluster's partial accumulators (all warps take the cluster barriers) ----------------
  // Each rank parks its fp32 partial in its free stage buffers; rank j then adds, for its rows
  // [j R, j R + R) (R = 128 / ks rounded up), the partials of ranks 0, 1, ..., ks - 1 in that order over
  // distributed shared memory and writes the sums into its own tensor memory, which the epilogue reads.
  if (MH == 1 && ks > 1) {
    float* part = reinterpret_cast<float*>(&sm.a[0][0]);  // [128][kPwPartStride]: stages a and b are contiguous
    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + 128u * c;
    float* prow = part + trow * kPwPartStride + 128 * c;
    if (warp < S::kEpiWarps) {
      pw_wait(smem_u32(&sm.accum), 0u);
      pw_fence_after();
#pragma unroll 1
      for (int j = 0; j < 8; ++j) {
        float v[16];
        pw_tmem_ld16(ta + 16 * j, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<float4*>(prow + 16 * j)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
    pw_fence_before();
    pw_cluster_sync();
    const int rows_per_rank = (S::kBM + ks - 1) / ks;
    const int row0 = rank * rows_per_rank;
    if (warp < S::kEpiWarps) {
      // this rank's rows, 16 bytes per thread at a time (consecutive threads on consecutive chunks): the
      // sum over ranks 0, 1, ..., ks - 1 in that order, written in place (no other rank reads these rows)
      const int nrows = min(rows_per_rank, S::kBM - row0);
      for (int f = tid; f < nrows * (kPwBN / 4); f += 32 * S::kEpiWarps) {
        float* loc = part + (row0 + f / (kPwBN / 4)) * kPwPartStride + 4 * (f % (kPwBN / 4));
        const uint32_t a = smem_u32(loc);
        float4 v[8];
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2)
          if (k2 < ks) v[k2] = pw_ld_cluster_f4(a, (uint32_t)k2);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2)
          if (k2 < ks) {
            acc.x = __fadd_rn(acc.x, v[k2].x);
            acc.y = __fadd_rn(acc.y, v[k2].y);
            acc.z = __fadd_rn(acc.z, v[k2].z);
            acc.w = __fadd_rn(acc.w, v[k2].w);
          }
        *reinterpret_cast<float4*>(loc) = acc;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * S::kEpiWarps) : "memory");  // epilogue warps only
      // the sums into this thread's tensor-memory row half (rows of other ranks get zeros; the epilogue
      // skips them)
      const bool owned = trow / rows_per_rank == rank;
#pragma unroll 1
      for (int j = 0; j < 8; ++j) {
        float acc[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 v = owned ? reinterpret_cast<const float4*>(prow + 16 * j)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
          acc[4 * i] = v.x;
          acc[4 * i + 1] = v.y;
          acc[4 * i + 2] = v.z;
          acc[4 * i + 3] = v.w;
        }
        pw_tmem_st16(ta + 16 * j, acc);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
    }
    pw_fence_before();
    pw_cluster_sync();  // every remote read is done (the stage buffers may be reused) and the sums are in place
    pw_fence_after();
  }

  if (warp < S::kEpiWarps) {
    const bool ready = pw_wait(smem_u32(&sm.accum), 0u);
    pw_fence_after();
    slot_ok = slot_ok && ready;
    uint8_t* rec = wp.data[0] + ((int64_t)(int32_t)block * wp.rec_block32 +
                                 (int32_t)((int32_t)offset * wp.rec_token32 + head * wp.rec_head32));
    uint8_t* drow = rec + (r == 0 ? 0 : wp.off_vd);
    uint8_t* srow = rec + (r == 0 ? wp.off_ks : wp.off_vs);
    const uint32_t taddr = tmem + 256u * half_m + ((uint32_t)(32 * q) << 16);
    const float gs = wp.global_scale[r];
    // the row's record bytes are staged in the free stage buffers and written out row by row (coalesced)
    uint8_t* stage_base = &sm.a[0][0];
    uint8_t* stage = stage_base + trow * kPwRecRow;
    uint8_t** rowptr = reinterpret_cast<uint8_t**>(stage_base + S::kBM * kPwRecRow);
    if (c == 0) rowptr[trow] = slot_ok ? drow : nullptr;

    // encode one finished 16-element group (bf16 pairs) and store its 8 code bytes and scale byte
    auto put_group = [&](int g, const uint32_t (&x)[8]) {
      bool exact;
      const uint32_t amax = group_amax_bits<16>(x);
      const float ga = __fmul_rn(gs, __uint_as_float(amax));
      uint32_t sb = cvt_e4m3(div6_fast(ga, exact));
      const bool slow = __any_sync(0xffffffffu, !wp.plain || !exact);
      uint32_t packed[2];
      if (slow) {
        sb = cvt_e4m3(__fdiv_rn(ga, 6.0f));
        encode_row<16, true>(x, sm.lut[r][sb], wp.zero, packed);
      } else {
        encode_row<16, false>(x, sm.lut[r][sb], wp.zero, packed);
      }
      *reinterpret_cast<uint2*>(stage + 8 * g) = make_uint2(packed[0], packed[1]);
      stage[128 + g] = (uint8_t)sb;
    };
    auto put_bf16 = [&](__nv_bfloat16* out, int g, const uint32_t (&x)[8]) {
      uint4* o = reinterpret_cast<uint4*>(out + 16 * g);
      o[0] = make_uint4(x[0], x[1], x[2], x[3]);
      o[1] = make_uint4(x[4], x[5], x[6], x[7]);
    };

    if (r == 1) {
      __nv_bfloat16* vo = (p.value_out && live && ready)
                              ? p.value_out + row * p.value_out_stride_token + head * p.value_out_stride_head
                              : nullptr;
#pragma unroll 1
      for (int g = c; g < 16; g += 4) {  // groups g and g + 2 of this thread's 8
        uint32_t x0[8], x1[8];
        pw_load2_bf16(taddr + 16 * g, taddr + 16 * (g + 2), x0, x1);
        if (vo) {
          put_bf16(vo, g, x0);
          put_bf16(vo, g + 2, x1);
        }
        put_group(g, x0);
        put_group(g + 2, x1);
      }
    } else {
      __nv_bfloat16* ko = (wp.key_out && pos_ok && ready)
                              ? wp.key_out + row * wp.key_out_stride_token + head * wp.key_out_stride_head
                              : nullptr;
      const bool norm = wp.norm_weight != nullptr;
      float rr = 1.0f;
      if (norm) {
        // the writer's order: partial l = (even squares of [8l, 8l+8)) + (odd squares), then pairwise at
        // distances 16, 8, 4, 2, 1; each thread computes its groups' partials, both read all 32
        float* red = reinterpret_cast<float*>(&sm.b[0][0]) + trow * kPwRedStride;  // stages are free now
        auto partials = [&](int g, const uint32_t (&x)[8]) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = make_float2(bf_lo(x[4 * h + i]), bf_hi(x[4 * h + i]));
              a = __ffma2_rn(f, f, a);
            }
            red[2 * g + h] = __fadd_rn(a.x, a.y);
          }
        };
#pragma unroll 1
        for (int g = c; g < 16; g += 4) {  // this split's partials: groups g and g + 2
          uint32_t x0[8], x1[8];
          pw_load2_bf16(taddr + 16 * g, taddr + 16 * (g + 2), x0, x1);
          partials(g, x0);
          partials(g + 2, x1);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(32 * S::kEpiWarps) : "memory");  // epilogue warps only
        float part[32];
#pragma unroll
        for (int l = 0; l < 32; ++l) part[l] = red[l];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
          for (int l = 0; l < m; ++l) part[l] = __fadd_rn(part[l], part[l + m]);
        rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(part[0], wp.inv_head_dim), wp.norm_eps)));
      }
      const float2 rr2 = make_float2(rr, rr);
      // group g (read back and rounded) normed: y = bf16((x * r) * (w + offset))
      auto normed = [&](int g, uint32_t (&x)[8]) {
        if (norm) {
          const float2* wv = reinterpret_cast<const float2*>(sm.nw + 16 * g);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 y = __fmul2_rn(__fmul2_rn(make_float2(bf_lo(x[i]), bf_hi(x[i])), rr2), wv[i]);
            x[i] = pack_bf16x2(y.x, y.y);
          }
        }
      };
      auto finish = [&](int g, const uint32_t (&x)[8]) {
        if (ko) put_bf16(ko, g, x);
        put_group(g, x);
      };
      const int rot_groups = wp.rot_dim >> 4;  // groups of 16 inside the rotated dims
      if (wp.rot_dim > 0 && wp.neox) {
#pragma unroll 1
        for (int ga = 0; ga < P; ++ga) {
          if (own(ga) != c) continue;
          uint32_t x1[8], x2[8], cw[8], sw[8];
          if (ga == c) {  // the first pair of this split: cos/sin loaded during the mainloop
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              cw[i] = pre_c[i];
              sw[i] = pre_s[i];
            }
          } else {
            load_bf16_run<16>(cs + 16 * ga, cw);
            load_bf16_run<16>(cs + half + 16 * ga, sw);
          }
          pw_load2_bf16(taddr + 16 * ga, taddr + 16 * (ga + P), x1, x2);
          normed(ga, x1);
          normed(ga + P, x2);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t a = x1[i], b = x2[i];
            x1[i] = bf16x2_add(bf16x2_mul(a, cw[i]), bf16x2_mul(b, sw[i]) ^ 0x80008000u);
            x2[i] = bf16x2_add(bf16x2_mul(b, cw[i]), bf16x2_mul(a, sw[i]));
          }
          finish(ga, x1);
          finish(ga + P, x2);
        }
      } else if (wp.rot_dim > 0) {
        // GPT-J: word i of group g = elements (16g + 2i, 16g + 2i + 1), cos/sin index 8g + i
#pragma unroll 1
        for (int g = c; g < rot_groups; g += 2) {
          uint32_t x[8], cw[4], sw[4];
          if (g == c) {  // the first rotated group of this split: cos/sin loaded during the mainloop
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              cw[i] = pre_c[i];
              sw[i] = pre_s[i];
            }
          } else {
            load_bf16_run<8>(cs + 8 * g, cw);
            load_bf16_run<8>(cs + half + 8 * g, sw);
          }
          pw_load_bf16(taddr + 16 * g, x);
          normed(g, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t sel = (i & 1) ? 0x3232u : 0x1010u;
            const uint32_t cc = __byte_perm(cw[i >> 1], 0u, sel), ss = __byte_perm(sw[i >> 1], 0u, sel);
            x[i] = bf16x2_add(bf16x2_mul(x[i], cc), bf16x2_mul(__byte_perm(x[i], 0u, 0x1032u), ss) ^ 0x00008000u);
          }
          finish(g, x);
        }
      }
      // dims past the rotation pass through: this split's groups g = c (mod 2) from there, two at a time
      int g = wp.rot_dim > 0 ? rot_groups : 0;
      if ((g & 1) != c) ++g;
#pragma unroll 1
      for (; g < 16; g += 4) {
        uint32_t x0[8], x1[8];
        if (g + 2 < 16) {
          pw_load2_bf16(taddr + 16 * g, taddr + 16 * (g + 2), x0, x1);
          normed(g, x0);
          finish(g, x0);
          normed(g + 2, x1);
          finish(g + 2, x1);
        } else {
          pw_load_bf16(taddr + 16 * g, x0);
          normed(g, x0);
          finish(g, x0);
        }
      }
    }
    // write the staged records: 9 chunks of 16 bytes per row (8 of codes, 1 of scales), consecutive threads
    // on consecutive chunks
    asm volatile("bar.sync 1, %0;" ::"r"(32 * S::kEpiWarps) : "memory");  // epilogue warps only
    const int64_t sdelta = srow - drow;
    for (int idx = tid; idx < S::kBM * 9; idx += 32 * S::kEpiWarps) {
      const int rr = idx / 9, j = idx - 9 * rr;
      uint8_t* d = rowptr[rr];
      if (d) {
        const uint4 v = *reinterpret_cast<const uint4*>(stage_base + rr * kPwRecRow + 16 * j);
        *reinterpret_cast<uint4*>(j < 8 ? d + 16 * j : d + sdelta) = v;
      }
    }
  }

  pw_fence_before();
  __syncthreads();
  if (warp == S::kMmaWarp) {
    __syncwarp();
    pw_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(S::kTmemCols));
  }
}
