// NVFP4 paged KV-cache writer for sm_100a.
//
// Replaces the reference's Triton writer (python/nvfp4_qsa/kernels.py:46-165),
// which launches one 4-warp program per (token, kv head) and runs twice, once
// for K and once for V.  Here ONE launch writes K and V: a warp owns a token
// and two kv heads, each lane loads head_dim/32 contiguous bf16 values of the
// four rows (K and V of both heads) with one vector load each, the group
// amax is a warp shuffle over the 16 / (head_dim/32) lanes that share a
// 16-element group, the E4M3 scale
// and the E2M1 codes come from the sm_100a cvt instructions, and each lane
// stores its packed bytes so that a warp writes each 128-byte data row with a
// single coalesced store instruction.
//
// Bit-exactness with the codec oracle (python/nvfp4_qsa/oracle.py:47-69):
//   amax      : max |x| per group, NaN-propagating (integer max of |x| bits)
//   scale     = e4m3_rn(min(g * amax / 6, 448))                    oracle.py:54-56
//   out_scale = g / max(float(scale), 1e-30)                        oracle.py:57
//   y         = x * out_scale, clamp +-6, RNE to E2M1, sign = y<0   oracle.py:58-63
// The reference Triton kernel (kernels.py:94-96) instead substitutes 1e30 for
// a zero scale, so it writes code 0 where the oracle saturates to +-6 for
// groups whose scale rounds to zero; this kernel follows the oracle.
#include <cuda.h>

#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace nvqsa {
namespace {

struct WriteParams {
  const __nv_bfloat16* src[2];  // K, V
  int64_t src_stride_token[2];  // elements
  int64_t src_stride_head[2];
  uint8_t* data[2];
  int64_t data_stride[2][3];  // block, token, head (bytes)
  uint8_t* scale[2];
  int64_t scale_stride[2][3];
  const int64_t* slots;
  int64_t num_tokens;
  int64_t num_blocks;
  int64_t page_size;
  int64_t num_slots;    // num_blocks * page_size (record layout only)
  uint64_t page_magic;  // slot / page_size = (slot * page_magic) >> page_shift for slot < 2^31
  int32_t page_shift;
  float global_scale[2];
  int32_t kv_heads;
  int32_t vec_src;  // 1: 16-byte aligned source rows -> vector loads
  // Record layout (set when `record` is 1): the four regions are views of one
  // [blocks, kv_heads, page, record] storage (same strides, region bases at
  // small offsets from K data), K and V share their strides, and every slot,
  // token index and per-block offset fits 31 bits (see nvqsa_write_cache).
  int32_t record;
  int32_t src_token32, src_head32;            // K/V source strides (elements)
  int32_t rec_block32, rec_token32, rec_head32;  // record strides (bytes)
  int32_t off_ks, off_vd, off_vs;             // region bases minus the K data base (bytes)
  // +0.0f, read at run time: the encoder's x * s + 0 must keep its add, which
  // the compiler drops when the addend is a literal zero feeding the E2M1
  // conversion (that conversion writes code 8 for -0).
  float zero;
  // 1: both global scales in [2^-6, 2^28] (see the encoder's fast path)
  int32_t plain;
  int32_t lut_by_scaling;  // 1: scale table by power-of-two scaling of g / k (see build_out_scale_lut)
  int32_t byte_store;      // 1: packed data rows not aligned to the lane's store width: store bytes one by one
  // K-norm and RoPE ahead of the encoder (nvqsa_norm_rope_write_cache only).
  const int64_t* positions;      // [num_tokens]
  const __nv_bfloat16* cos_sin;  // [max_position, >= rot_dim]: cos in [0, rot/2), sin in [rot/2, rot)
  int64_t cos_sin_stride;        // elements
  int64_t max_position;
  const float* norm_weight;      // [head_dim] or null (no norm)
  float norm_offset;             // added to every weight in fp32 (1 for GemmaRMSNorm)
  float norm_eps;
  float inv_head_dim;
  int32_t rot_dim;               // 0: no rotation
  int32_t neox;                  // 1: rotate halves (x[i], x[i + rot/2]); 0: GPT-J pairs (x[2i], x[2i+1])
  __nv_bfloat16* key_out;        // optional normed, rotated bf16 K [num_tokens, kv_heads, head_dim]
  int64_t key_out_stride_token, key_out_stride_head;
  int32_t group_path;  // head_dim 256, record layout, vector rows, 8-byte aligned records: write_cache_group_kernel
};

template <int EPL>
struct Vec;  // EPL bf16 values loaded per lane
template <>
struct Vec<2> { using T = uint32_t; };
template <>
struct Vec<4> { using T = uint2; };
template <>
struct Vec<8> { using T = uint4; };

// The EPL bf16 values of one lane as EPL/2 raw words (element 2i in the low half of word i).
template <int EPL, bool VEC>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, uint32_t (&w)[EPL / 2]) {
  if constexpr (VEC && EPL <= 8) {
    typename Vec<EPL>::T v = __ldg(reinterpret_cast<const typename Vec<EPL>::T*>(p));
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) w[i] = u[i];
  } else if constexpr (VEC) {
#pragma unroll
    for (int q = 0; q < EPL / 8; ++q) {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + q);
      w[4 * q] = v.x;
      w[4 * q + 1] = v.y;
      w[4 * q + 2] = v.z;
      w[4 * q + 3] = v.w;
    }
  } else {
    const unsigned short* s = reinterpret_cast<const unsigned short*>(p);
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) w[i] = (uint32_t)__ldg(s + 2 * i) | ((uint32_t)__ldg(s + 2 * i + 1) << 16);
  }
}

// NaN-propagating max |x| of the lane's values as fp32 bits: for |x| bit
// patterns integer order == float order and NaN sorts above +inf, so the max
// runs on the raw bf16 halves (16x2 SIMD), then over the LPG lanes of the group.
template <int EPL>
__device__ __forceinline__ uint32_t group_amax_bits(const uint32_t (&w)[EPL / 2]) {
  constexpr int LPG = 16 / EPL;
  uint32_t m2 = w[0] & 0x7fff7fffu;
#pragma unroll
  for (int i = 1; i < EPL / 2; ++i) m2 = __vmaxu2(m2, w[i] & 0x7fff7fffu);
  uint32_t a = max(m2 & 0xffffu, m2 >> 16) << 16;
#pragma unroll
  for (int m = 1; m < LPG; m <<= 1) a = max(a, __shfl_xor_sync(0xffffffffu, a, m));
  return a;
}

// E2M1 codes of the lane's values scaled by out_scale (oracle.py:58-63),
// EPL/2 bytes with element 2i in the low nibble of byte i.  The oracle rounds
// y = x * s and takes sign = y < 0, so an exact -0 (a -0 input, or a negative
// product that underflows) must give code 0 while a tiny negative y that
// rounds to a nonzero value keeps code 8; the hardware conversion keeps the
// sign of -0, hence y = x * s + 0 with +0 from a kernel parameter (see
// WriteParams::zero).  In the slow path the product (f32x2) and the add are
// rounded separately -- a packed multiply followed by a packed add was
// contracted into one FMA, which keeps the sign of an underflowing product --
// and NaN maps to code 0 (every threshold test of the oracle is false for
// NaN; the hardware conversion would saturate it).
template <int EPL, bool SLOW>
__device__ __forceinline__ void encode_row(const uint32_t (&w)[EPL / 2], float s, float zero,
                                           uint32_t (&packed)[(EPL + 7) / 8]) {
  const float2 s2 = make_float2(s, s);
  float y[EPL];
  if constexpr (!SLOW) {
    // Fast path (plain global scales, no NaN or inf in the group): no product
    // of a nonzero bf16 value underflows to zero (|x| >= 2^-133 and
    // |s| >= 2^-6 / 448), so one rounding of x * s + 0 equals the two, and an
    // exact zero product gives +0.
    const float2 z2 = make_float2(zero, zero);
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      const float2 y2 =
          __ffma2_rn(make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u)), s2, z2);
      y[2 * i] = y2.x;
      y[2 * i + 1] = y2.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      const float2 m2 = __fmul2_rn(make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u)), s2);
      y[2 * i] = __fadd_rn(m2.x, zero);
      y[2 * i + 1] = __fadd_rn(m2.y, zero);
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) y[i] = (y[i] != y[i]) ? 0.0f : y[i];
  }
  if constexpr (EPL >= 8) {
#pragma unroll
    for (int j = 0; j < EPL / 8; ++j) {
      float y8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y8[i] = y[8 * j + i];
      packed[j] = cvt_e2m1x8(y8);
    }
  } else {
    packed[0] = 0;
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) packed[0] |= cvt_e2m1x2(y[2 * i + 1], y[2 * i]) << (8 * i);
  }
}

template <int EPL>
__device__ __forceinline__ void store_lane_bytes(uint8_t* row, int lane, const uint32_t (&packed)[(EPL + 7) / 8]) {
#pragma unroll
  for (int j = 0; j < EPL / 2; ++j) row[lane * (EPL / 2) + j] = (uint8_t)(packed[j >> 2] >> (8 * (j & 3)));
}

template <int EPL>
__device__ __forceinline__ void store_lane(uint8_t* row, int lane, const uint32_t (&packed)[(EPL + 7) / 8]) {
  if constexpr (EPL == 2) {
    row[lane] = (uint8_t)packed[0];
  } else if constexpr (EPL == 4) {
    reinterpret_cast<uint16_t*>(row)[lane] = (uint16_t)packed[0];
  } else if constexpr (EPL == 8) {
    reinterpret_cast<uint32_t*>(row)[lane] = packed[0];
  } else {
    reinterpret_cast<uint2*>(row)[lane] = make_uint2(packed[0], packed[1]);
  }
}

// out_scale_lut[r][b] = g_r / max(e4m3(b), 1e-30) for every scale byte b
// (oracle.py:57), the per-group divide of the encoder as a table read.  When
// the host has set lut_by_scaling (both global scales finite with
// 2^-117 <= |g| <= 2^100) the table comes from 32 divisions: a normal E4M3
// value is (8+m) * 2^(e-10) and a subnormal one m * 2^-9, so
// g / e4m3(b) = (g / k) * 2^j with k in 1..15, and with every entry a normal
// float the power-of-two scaling is exact and equals the IEEE division
// entry for entry.  Otherwise each entry is divided directly.
__device__ __forceinline__ void build_out_scale_lut(const WriteParams& p, float (*lut)[256], float (*quot)[16]) {
  if (p.lut_by_scaling) {
    if (threadIdx.x < 32) {
      const int r = threadIdx.x >> 4, k = threadIdx.x & 15;  // quot[r][0] = g / 1e-30, quot[r][k] = g / k
      quot[r][k] = __fdiv_rn(p.global_scale[r], k == 0 ? 1e-30f : (float)k);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 512; i += blockDim.x) {
      const int r = i >> 8, b = i & 255, e = (b >> 3) & 15, m = b & 7;
      // -0, a negative scale or zero: max(den, 1e-30) = 1e-30, entry g / 1e-30 unscaled;
      // subnormal m * 2^-9: (g / m) * 2^9; normal (8+m) * 2^(e-10): (g / (8+m)) * 2^(10-e)
      const bool clamp = b >= 0x80 || b == 0;
      const int k = clamp ? 0 : (e == 0 ? m : 8 + m);
      const int j = clamp ? 0 : (e == 0 ? 9 : 10 - e);
      const float v = __fmul_rn(quot[r][k], __int_as_float((127 + j) << 23));
      lut[r][b] = ((b & 0x7f) == 0x7f) ? __int_as_float(0x7fffffff) : v;  // g / NaN
    }
  } else {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) {
      const float bs = e4m3_to_f32((uint32_t)(i & 255));
      const float den = (bs < 1e-30f) ? 1e-30f : bs;  // clamp_min; NaN stays NaN
      lut[i >> 8][i & 255] = __fdiv_rn(p.global_scale[i >> 8], den);
    }
  }
}

// slot -> (block, offset); false for a slot that is negative or past the
// cache, which the writer skips (kernels.py:71-77).
template <bool RECORD>
__device__ __forceinline__ bool slot_position(const WriteParams& p, int64_t slot, int64_t& block, int64_t& offset) {
  if (slot < 0) return false;
  if constexpr (RECORD) {  // slot < num_blocks * page_size < 2^31: multiply-shift division
    if (slot >= p.num_slots) return false;
    const uint32_t b32 = (uint32_t)(((uint64_t)(uint32_t)slot * p.page_magic) >> p.page_shift);
    block = b32;
    offset = (int64_t)((uint32_t)slot - b32 * (uint32_t)p.page_size);
  } else {
    block = slot / p.page_size;
    if (block >= p.num_blocks) return false;
    offset = slot - block * p.page_size;
  }
  return true;
}

// Encode and store one item: the K and V rows of kv heads h0 and h0 + 1
// (x = K h0, V h0, K h1, V h1; the h1 rows are ignored when h0 is the last
// head) into the slot's records.
template <int EPL, bool RECORD>
__device__ __forceinline__ void write_item(const WriteParams& p, const float (*out_scale_lut)[256], int lane,
                                           int64_t block, int64_t offset, int h0, const uint32_t (&x)[4][EPL / 2]) {
  constexpr int LPG = 16 / EPL;
  const bool two = h0 + 1 < p.kv_heads;
  // Group scales of the four rows (oracle.py:54-57).  With plain global
  // scales every table entry a finite non-negative g * amax / 6 can reach is
  // finite, so the fast division is the only check: it fails for NaN / inf
  // inputs and tiny or huge g * amax.  Otherwise (one warp vote), or when the
  // scales are not plain, every row is redone with the IEEE division and
  // encoded on the slow path.  The satfinite E4M3 conversion clamps to +-448
  // as the oracle's clamp does.
  uint32_t amax_bits[4], sb[4];
  float os[4];
  bool rare = !p.plain;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    bool exact;
    amax_bits[q] = group_amax_bits<EPL>(x[q]);
    const float bs = div6_fast(__fmul_rn(p.global_scale[q & 1], __uint_as_float(amax_bits[q])), exact);
    sb[q] = cvt_e4m3(bs);
    os[q] = out_scale_lut[q & 1][sb[q]];
    rare |= !exact;
  }
  const bool slow = __any_sync(0xffffffffu, rare);
  if (slow) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      sb[q] = cvt_e4m3(__fdiv_rn(__fmul_rn(p.global_scale[q & 1], __uint_as_float(amax_bits[q])), 6.0f));
      os[q] = out_scale_lut[q & 1][sb[q]];
    }
  }
  uint8_t* drow[2];
  uint8_t* srow[2];
  if constexpr (RECORD) {
    uint8_t* rec = p.data[0] + ((int64_t)(int32_t)block * p.rec_block32 +
                                (int32_t)((int32_t)offset * p.rec_token32 + h0 * p.rec_head32));
    drow[0] = rec;
    srow[0] = rec + p.off_ks;
    drow[1] = rec + p.off_vd;
    srow[1] = rec + p.off_vs;
  } else {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      drow[r] = p.data[r] + block * p.data_stride[r][0] + offset * p.data_stride[r][1] + h0 * p.data_stride[r][2];
      srow[r] = p.scale[r] + block * p.scale_stride[r][0] + offset * p.scale_stride[r][1] + h0 * p.scale_stride[r][2];
    }
  }
  // the fast / slow choice is warp-uniform: one branch for the four rows
  auto encode_store = [&](auto slow_tag) {
    constexpr bool SLOW = decltype(slow_tag)::value;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      if (hh == 1 && !two) break;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int q = 2 * hh + r;
        uint32_t packed[(EPL + 7) / 8];
        encode_row<EPL, SLOW>(x[q], os[q], p.zero, packed);
        const int64_t hstep_d = RECORD ? (int64_t)p.rec_head32 : p.data_stride[r][2];
        const int64_t hstep_s = RECORD ? (int64_t)p.rec_head32 : p.scale_stride[r][2];
        if (p.byte_store)
          store_lane_bytes<EPL>(drow[r] + (hh ? hstep_d : 0), lane, packed);
        else
          store_lane<EPL>(drow[r] + (hh ? hstep_d : 0), lane, packed);
        if ((lane % LPG) == 0) (srow[r] + (hh ? hstep_s : 0))[lane / LPG] = (uint8_t)sb[q];
      }
    }
  };
  if (slow)
    encode_store(std::true_type{});
  else
    encode_store(std::false_type{});
}

// ---------------------------------------------------------------------------
// K-norm + RoPE ahead of the encoder (nvqsa_norm_rope_write_cache).
//
// The caller of the reference writer (integration/snapshot/qsa.py:618-667)
// takes K from the QKV projection through vLLM's GemmaRMSNorm k_norm and its
// rotary embedding, both in bf16, and hands the result to
// qsa_write_cache_nvfp4.  Here the same two steps run on the rows already in
// registers, so K makes one trip from HBM instead of three.
//   norm : ss = sum x^2 (fp32; per lane, the squares of its even and of its
//          odd elements are summed in element order by FMA and then added;
//          the 32 lane sums are added pairwise at distances 16, 8, 4, 2, 1),
//          r = 1 / sqrt(ss / head_dim + eps) (IEEE sqrt, IEEE divide),
//          y = bf16_rn((x * r) * (w + offset))      vLLM ir rms_norm order
//   rope : cos/sin rows of the bf16 cache at the token's position,
//          o1 = bf16(bf16(x1 c) - bf16(x2 s)), o2 = bf16(bf16(x2 c) + bf16(x1 s))
//          -- torch's bf16 elementwise arithmetic of vLLM's native rotary
//          embedding: each product and sum rounds to bf16 (here on packed
//          bf16x2 words, which round identically; see bf16x2_mul).
// ---------------------------------------------------------------------------

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// N consecutive bf16 values (N even) from p into N/2 words with vector loads (p aligned to 2N bytes).
template <int N>
__device__ __forceinline__ void load_bf16_run(const __nv_bfloat16* p, uint32_t (&w)[N / 2]) {
  if constexpr (N == 2) {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else if constexpr (N == 4) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x;
    w[1] = v.y;
  } else {
#pragma unroll
    for (int q = 0; q < N / 8; ++q) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + q);
      w[4 * q] = v.x;
      w[4 * q + 1] = v.y;
      w[4 * q + 2] = v.z;
      w[4 * q + 3] = v.w;
    }
  }
}

// Lane roles in the rotation: a lane holds elements [lane*EPL, lane*EPL + EPL).
// NeoX: a lane below rot/2 holds x1 (its partner lane + rot/(2 EPL) holds x2),
// a lane in [rot/2, rot) holds x2; both read cos/sin at element index mod rot/2.
// GPT-J: (x[2i], x[2i+1]) lie in one word, cos/sin index i.
struct RopeLane {
  bool active;  // lane holds rotated elements
  bool first;   // NeoX: lane holds x1
  int partner;  // NeoX: lane holding the other half
  int cs0;      // first cos/sin index of the lane
};

template <int EPL>
__device__ __forceinline__ RopeLane rope_lane(const WriteParams& p, int lane) {
  RopeLane r;
  const int e0 = lane * EPL, half = p.rot_dim >> 1;
  r.active = e0 < p.rot_dim;
  r.first = e0 < half;
  const int shift = half / EPL;
  r.partner = p.neox ? (r.first ? lane + shift : lane - shift) : lane;
  if (!r.active) r.partner = lane;
  r.cs0 = p.neox ? (r.first ? e0 : e0 - half) : (e0 >> 1);
  return r;
}

// cos/sin values of one lane for the token at `pos` (EPL each for NeoX, EPL/2 for GPT-J).
template <int EPL>
__device__ __forceinline__ void load_cos_sin(const WriteParams& p, const RopeLane& rl, int64_t pos,
                                             uint32_t (&cw)[EPL / 2], uint32_t (&sw)[EPL / 2]) {
  const __nv_bfloat16* row = p.cos_sin + pos * p.cos_sin_stride + rl.cs0;
  const int half = p.rot_dim >> 1;
  if (p.neox) {
    load_bf16_run<EPL>(row, cw);
    load_bf16_run<EPL>(row + half, sw);
  } else if constexpr (EPL >= 4) {
    uint32_t c2[EPL / 4], s2[EPL / 4];
    load_bf16_run<EPL / 2>(row, c2);
    load_bf16_run<EPL / 2>(row + half, s2);
#pragma unroll
    for (int i = 0; i < EPL / 4; ++i) {
      cw[i] = c2[i];
      sw[i] = s2[i];
    }
  } else {  // EPL == 2: one GPT-J pair per lane
    cw[0] = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(row));
    sw[0] = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(row + half));
  }
}

// Packed bf16 arithmetic (sm_90+ PTX).  For bf16 operands these equal
// torch's bf16 elementwise ops (fp32 result, then round to bf16): a product
// of two bf16 values is exact in fp32 except below 2^-126, where the fp32
// rounding can only land on the bf16 tie at 2^-134 from below, which both
// routes round to zero; a sum of two bf16 values is exact in fp32 unless
// their exponents differ by more than 16, and then the fp32 rounding cannot
// create a bf16 tie.  NaN results are the canonical 0x7fff in both.
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// k-norm + rotation of the K rows of both heads of an item (k1 is a copy of
// k0's head when the item has one head).  The two rows share one reduction:
// lanes 0-15 finish head h0's sum and lanes 16-31 head h1's, then one square
// root and divide serve both.  Per lane the squares of the even and of the odd
// elements are summed separately in element order (one f32x2 FMA per word)
// and then added; the 32 lane sums are added pairwise at distances 16, 8, 4,
// 2, 1.
template <int EPL>
__device__ __forceinline__ void norm_rope_pair(const WriteParams& p, int lane, const RopeLane& rl,
                                               const float2 (&wp)[EPL / 2], const uint32_t (&cw)[EPL / 2],
                                               const uint32_t (&sw)[EPL / 2], uint32_t (&k0)[EPL / 2],
                                               uint32_t (&k1)[EPL / 2]) {
  constexpr int NW = EPL / 2;
  if (p.norm_weight != nullptr) {
    float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const float2 f0 = make_float2(bf_lo(k0[i]), bf_hi(k0[i]));
      const float2 f1 = make_float2(bf_lo(k1[i]), bf_hi(k1[i]));
      a0 = __ffma2_rn(f0, f0, a0);
      a1 = __ffma2_rn(f1, f1, a1);
    }
    const float s0 = __fadd_rn(a0.x, a0.y), s1 = __fadd_rn(a1.x, a1.y);
    const bool low = lane < 16;
    float t = low ? s0 : s1;
    t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, low ? s1 : s0, 16));
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, m));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(t, p.inv_head_dim), p.norm_eps)));
    const float r0 = __shfl_sync(0xffffffffu, r, 0), r1 = __shfl_sync(0xffffffffu, r, 16);
    const float2 r02 = make_float2(r0, r0), r12 = make_float2(r1, r1);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const float2 y0 = __fmul2_rn(__fmul2_rn(make_float2(bf_lo(k0[i]), bf_hi(k0[i])), r02), wp[i]);
      const float2 y1 = __fmul2_rn(__fmul2_rn(make_float2(bf_lo(k1[i]), bf_hi(k1[i])), r12), wp[i]);
      k0[i] = pack_bf16x2(y0.x, y0.y);
      k1[i] = pack_bf16x2(y1.x, y1.y);
    }
  }
  if (p.rot_dim > 0) {
    if (p.neox) {
      // first half: own = x1, partner = x2 -> x1 c - x2 s; second half: own = x2, partner = x1 -> x2 c + x1 s
      uint32_t o0[NW], o1[NW];
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        o0[i] = __shfl_sync(0xffffffffu, k0[i], rl.partner);
        o1[i] = __shfl_sync(0xffffffffu, k1[i], rl.partner);
      }
      if (rl.active) {
        const uint32_t neg = rl.first ? 0x80008000u : 0u;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
          k0[i] = bf16x2_add(bf16x2_mul(k0[i], cw[i]), bf16x2_mul(o0[i], sw[i]) ^ neg);
          k1[i] = bf16x2_add(bf16x2_mul(k1[i], cw[i]), bf16x2_mul(o1[i], sw[i]) ^ neg);
        }
      }
    } else if (rl.active) {
      // word i = (x1, x2) = elements (2k, 2k+1), k = cs0 + i: (x1 c - x2 s, x2 c + x1 s)
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        const uint32_t sel = (i & 1) ? 0x3232u : 0x1010u;
        const uint32_t cc = __byte_perm(cw[i >> 1], 0u, sel), ss = __byte_perm(sw[i >> 1], 0u, sel);
        k0[i] = bf16x2_add(bf16x2_mul(k0[i], cc), bf16x2_mul(__byte_perm(k0[i], 0u, 0x1032u), ss) ^ 0x00008000u);
        k1[i] = bf16x2_add(bf16x2_mul(k1[i], cc), bf16x2_mul(__byte_perm(k1[i], 0u, 0x1032u), ss) ^ 0x00008000u);
      }
    }
  }
}

// The EPL bf16 values of one lane with vector stores (p aligned to min(2 EPL, 16) bytes).
template <int EPL>
__device__ __forceinline__ void store_bf16_row(__nv_bfloat16* p, const uint32_t (&w)[EPL / 2]) {
  if constexpr (EPL == 2) {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  } else if constexpr (EPL == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int q = 0; q < EPL / 8; ++q)
      reinterpret_cast<uint4*>(p)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
}

// Item w -> (token, first kv head of its pair).
template <bool RECORD>
__device__ __forceinline__ void item_token(int64_t w, int head_pairs, int64_t& token, int& h0) {
  if constexpr (RECORD) {
    token = head_pairs == 1 ? w : (int64_t)((uint32_t)w / (uint32_t)head_pairs);
  } else {
    token = head_pairs == 1 ? w : w / head_pairs;
  }
  h0 = 2 * (int)(w - token * head_pairs);
}

// One warp per item (token, pair of kv heads), grid-stride over all items,
// rows loaded into registers.  Any head_dim and layout.  A warp issues every
// global load of its first item (the slot and the K and V rows of both heads)
// before the CTA builds its scale table, so the table is built while the
// loads are in flight.  FUSE: the K rows pass through the k-norm and the
// rotary embedding first (nvqsa_norm_rope_write_cache); an item whose position
// is outside [0, max_position) is skipped entirely.
template <int HEAD_DIM, bool VEC, bool RECORD, bool FUSE>
__global__ void __launch_bounds__(256, HEAD_DIM >= 512 ? 2 : 4) write_cache_kernel(const WriteParams p) {
  constexpr int EPL = HEAD_DIM / 32;
  constexpr int NW = EPL / 2;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int head_pairs = (p.kv_heads + 1) >> 1;
  const int64_t items = p.num_tokens * head_pairs;
  const int64_t w0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  __shared__ float out_scale_lut[2][256];
  __shared__ float quot[2][16];

  int64_t token = 0, slot = -1;
  int h0 = 0;
  uint32_t x[4][NW];  // K h0, V h0, K h1, V h1
  // FUSE state: the lane's norm weights (+ offset), rotation role, the item's position and cos/sin
  __shared__ __align__(16) float wsm[FUSE ? HEAD_DIM : 1];
  uint32_t cw[FUSE ? NW : 1], sw[FUSE ? NW : 1];
  RopeLane rl{};
  bool pos_ok = true;
  if constexpr (FUSE) {
    rl = rope_lane<EPL>(p, lane);
    if (p.norm_weight != nullptr)
      for (int j = threadIdx.x; j < HEAD_DIM; j += blockDim.x) wsm[j] = __fadd_rn(__ldg(p.norm_weight + j), p.norm_offset);
  }
  auto load_item = [&](int64_t w) {
    item_token<RECORD>(w, head_pairs, token, h0);
    slot = __ldg(p.slots + token);
    if constexpr (FUSE) {
      if (p.rot_dim > 0) {
        const int64_t pos = __ldg(p.positions + token);
        pos_ok = pos >= 0 && pos < p.max_position;
        if (pos_ok && rl.active) load_cos_sin<EPL>(p, rl, pos, cw, sw);
      }
    }
    const bool two = h0 + 1 < p.kv_heads;
    if constexpr (RECORD) {
      // one source offset for K and V: token * stride + head * stride + lane * EPL
      const int64_t off = (int64_t)(int32_t)token * p.src_token32 + (h0 * p.src_head32 + lane * EPL);
      const int h1 = two ? p.src_head32 : 0;
      load_row<EPL, VEC>(p.src[0] + off, x[0]);
      load_row<EPL, VEC>(p.src[1] + off, x[1]);
      load_row<EPL, VEC>(p.src[0] + off + h1, x[2]);
      load_row<EPL, VEC>(p.src[1] + off + h1, x[3]);
    } else {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int head = two ? h0 + hh : h0;
#pragma unroll
        for (int r = 0; r < 2; ++r)
          load_row<EPL, VEC>(p.src[r] + token * p.src_stride_token[r] + head * p.src_stride_head[r] + lane * EPL,
                             x[2 * hh + r]);
      }
    }
  };

  if (w0 < items) load_item(w0);
  build_out_scale_lut(p, out_scale_lut, quot);
  __syncthreads();
  for (int64_t w = w0; w < items; w += warps) {
    if (w != w0) load_item(w);
    if constexpr (FUSE) {
      if (!pos_ok) continue;  // warp-uniform: one position per item
      const bool two = h0 + 1 < p.kv_heads;
      float2 wp[EPL / 2];
#pragma unroll
      for (int j = 0; j < EPL / 2; ++j) wp[j] = reinterpret_cast<const float2*>(wsm + lane * EPL)[j];
      norm_rope_pair<EPL>(p, lane, rl, wp, cw, sw, x[0], x[2]);
      if (p.key_out != nullptr) {
        __nv_bfloat16* ko = p.key_out + token * p.key_out_stride_token + h0 * p.key_out_stride_head + lane * EPL;
        store_bf16_row<EPL>(ko, x[0]);
        if (two) store_bf16_row<EPL>(ko + p.key_out_stride_head, x[2]);
      }
    }
    int64_t block, offset;
    if (slot_position<RECORD>(p, slot, block, offset))
      write_item<EPL, RECORD>(p, out_scale_lut, lane, block, offset, h0, x);
  }
}

// head_dim 256, record layout, 16-byte aligned source rows, no norm or rotation: a lane owns one whole
// 16-element group of one head (lanes 0-15 head h0, lanes 16-31 head h0 + 1) of the K and the V row, so
// the group amax needs no shuffle, each group's scale is computed once, and a lane stores 8 data bytes
// and its scale byte per row.  Same arithmetic and bytes as write_cache_kernel.
__global__ void __launch_bounds__(256, 4) write_cache_group_kernel(const WriteParams p) {
  const int lane = threadIdx.x & 31;
  const int hh = lane >> 4, g = lane & 15;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int head_pairs = (p.kv_heads + 1) >> 1;
  const int64_t items = p.num_tokens * head_pairs;
  const int64_t w0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  __shared__ float out_scale_lut[2][256];
  __shared__ float quot[2][16];

  int64_t token = 0, slot = -1;
  int h0 = 0;
  uint32_t x[2][8];  // K, V: the lane's 16 bf16 values of its head
  auto load_item = [&](int64_t w) {
    item_token<true>(w, head_pairs, token, h0);
    slot = __ldg(p.slots + token);
    const int h = (h0 + 1 < p.kv_heads) ? h0 + hh : h0;
    const int64_t off = (int64_t)(int32_t)token * p.src_token32 + (h * p.src_head32 + 16 * g);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(p.src[r] + off));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(p.src[r] + off) + 1);
      x[r][0] = a.x; x[r][1] = a.y; x[r][2] = a.z; x[r][3] = a.w;
      x[r][4] = b.x; x[r][5] = b.y; x[r][6] = b.z; x[r][7] = b.w;
    }
  };

  if (w0 < items) load_item(w0);
  build_out_scale_lut(p, out_scale_lut, quot);
  __syncthreads();
  for (int64_t w = w0; w < items; w += warps) {
    if (w != w0) load_item(w);
    int64_t block, offset;
    if (!slot_position<true>(p, slot, block, offset)) continue;
    const bool mine = hh == 0 || h0 + 1 < p.kv_heads;
    uint32_t amax_bits[2], sb[2];
    float os[2];
    bool rare = !p.plain;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      bool exact;
      amax_bits[r] = group_amax_bits<16>(x[r]);
      const float bs = div6_fast(__fmul_rn(p.global_scale[r], __uint_as_float(amax_bits[r])), exact);
      sb[r] = cvt_e4m3(bs);
      os[r] = out_scale_lut[r][sb[r]];
      rare |= !exact;
    }
    const bool slow = __any_sync(0xffffffffu, rare);
    if (slow) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        sb[r] = cvt_e4m3(__fdiv_rn(__fmul_rn(p.global_scale[r], __uint_as_float(amax_bits[r])), 6.0f));
        os[r] = out_scale_lut[r][sb[r]];
      }
    }
    uint8_t* rec = p.data[0] + ((int64_t)(int32_t)block * p.rec_block32 +
                                (int32_t)((int32_t)offset * p.rec_token32 + (h0 + hh) * p.rec_head32));
    uint8_t* drow[2] = {rec, rec + p.off_vd};
    uint8_t* srow[2] = {rec + p.off_ks, rec + p.off_vs};
    auto encode_store = [&](auto slow_tag) {
      constexpr bool SLOW = decltype(slow_tag)::value;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        uint32_t packed[2];
        encode_row<16, SLOW>(x[r], os[r], p.zero, packed);
        if (mine) {
          *reinterpret_cast<uint2*>(drow[r] + 8 * g) = make_uint2(packed[0], packed[1]);
          srow[r][g] = (uint8_t)sb[r];
        }
      }
    };
    if (slow)
      encode_store(std::true_type{});
    else
      encode_store(std::false_type{});
  }
}

template <int HD, bool VEC, bool RECORD, bool FUSE>
cudaError_t launch_write_impl(const WriteParams& p, cudaStream_t stream) {
  const int64_t items = p.num_tokens * ((p.kv_heads + 1) / 2);
  const int threads = 256;
  const int warps_per_block = threads / 32;
  int64_t blocks = (items + warps_per_block - 1) / warps_per_block;
  // One resident wave (occupancy of this instantiation on this device); grid-stride beyond.
  static OccupancyCache occ;
  const int per_sm = occ.get(write_cache_kernel<HD, VEC, RECORD, FUSE>, threads);
  const int sms = device_sm_count();
  const int64_t cap = (int64_t)(sms > 0 ? sms : 148) * per_sm;
  if (blocks > cap) blocks = cap;
  write_cache_kernel<HD, VEC, RECORD, FUSE><<<(unsigned)blocks, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int HD, bool FUSE>
cudaError_t launch_write(const WriteParams& p, cudaStream_t stream) {
  if constexpr (HD == 256 && !FUSE) {
    if (p.group_path) {
      const int64_t items = p.num_tokens * ((p.kv_heads + 1) / 2);
      int64_t blocks = (items + 7) / 8;
      static OccupancyCache occ;
      const int per_sm = occ.get(write_cache_group_kernel, 256);
      const int sms = device_sm_count();
      const int64_t cap = (int64_t)(sms > 0 ? sms : 148) * per_sm;
      if (blocks > cap) blocks = cap;
      write_cache_group_kernel<<<(unsigned)blocks, 256, 0, stream>>>(p);
      return cudaGetLastError();
    }
  }
  if (p.record)
    return p.vec_src ? launch_write_impl<HD, true, true, FUSE>(p, stream)
                     : launch_write_impl<HD, false, true, FUSE>(p, stream);
  return p.vec_src ? launch_write_impl<HD, true, false, FUSE>(p, stream)
                   : launch_write_impl<HD, false, false, FUSE>(p, stream);
}

template <bool FUSE>
cudaError_t launch_write_any(const WriteParams& p, int head_dim, cudaStream_t s) {
  switch (head_dim) {
    case 64: return launch_write<64, FUSE>(p, s);
    case 128: return launch_write<128, FUSE>(p, s);
    case 256: return launch_write<256, FUSE>(p, s);
    default: return launch_write<512, FUSE>(p, s);
  }
}

#include "kv_proj_write.cuh"

}  // namespace

// Error flags of this file's kernels (bit 2: a projection-writer wait ran out), for nvqsa_read_error_flags.
int write_error_flags(unsigned int* v, bool clear) {
  if (cudaMemcpyFromSymbol(v, g_write_error_flags, sizeof(*v)) != cudaSuccess) return NVQSA_ERR_CUDA;
  if (clear && *v) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_write_error_flags, &zero, sizeof(zero)) != cudaSuccess) return NVQSA_ERR_CUDA;
  }
  return NVQSA_OK;
}

}  // namespace nvqsa

using namespace nvqsa;

// Shared host checks and parameter setup of both writer entries.  Returns
// NVQSA_OK with `go` set when there is work to launch.
static int prepare_write(
    WriteParams& p, bool& go,
    const void* key, int64_t key_stride_token, int64_t key_stride_head,
    const void* value, int64_t value_stride_token, int64_t value_stride_head,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int64_t num_tokens, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size, float key_global_scale, float value_global_scale) {
  go = false;
  if (num_tokens < 0 || kv_heads < 0 || num_blocks < 0 || page_size < 1) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512) return NVQSA_ERR_HEAD_DIM;
  if (num_tokens == 0 || kv_heads == 0 || num_blocks == 0) return NVQSA_OK;
  if (!key || !value || !key_data || !key_scale || !value_data || !value_scale || !slot_mapping)
    return NVQSA_ERR_NULL_POINTER;

  p = WriteParams{};
  p.src[0] = static_cast<const __nv_bfloat16*>(key);
  p.src[1] = static_cast<const __nv_bfloat16*>(value);
  p.src_stride_token[0] = key_stride_token;
  p.src_stride_head[0] = key_stride_head;
  p.src_stride_token[1] = value_stride_token;
  p.src_stride_head[1] = value_stride_head;
  p.data[0] = static_cast<uint8_t*>(key_data);
  p.data[1] = static_cast<uint8_t*>(value_data);
  p.scale[0] = static_cast<uint8_t*>(key_scale);
  p.scale[1] = static_cast<uint8_t*>(value_scale);
  const int64_t ds[2][3] = {{kd_stride_block, kd_stride_token, kd_stride_head}, {vd_stride_block, vd_stride_token, vd_stride_head}};
  const int64_t ss[2][3] = {{ks_stride_block, ks_stride_token, ks_stride_head}, {vs_stride_block, vs_stride_token, vs_stride_head}};
  for (int r = 0; r < 2; ++r)
    for (int i = 0; i < 3; ++i) {
      p.data_stride[r][i] = ds[r][i];
      p.scale_stride[r][i] = ss[r][i];
    }
  p.slots = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_blocks = num_blocks;
  p.page_size = page_size;
  p.global_scale[0] = key_global_scale;
  p.global_scale[1] = value_global_scale;
  p.kv_heads = kv_heads;
  // Record layout: the four regions share one set of strides and lie within
  // 2^31 bytes of K data, K and V share their strides, and slots, token
  // indices and per-block offsets fit 31 bits; then one record base per item
  // addresses all four stores and one offset both source rows.
  const int64_t i31 = 0x7fffffffLL;
  auto fits = [&](int64_t v) { return v >= -i31 && v <= i31; };
  auto gap = [&](const void* a, const void* b) {
    return (int64_t)(reinterpret_cast<uintptr_t>(a) - reinterpret_cast<uintptr_t>(b));
  };
  bool record = num_blocks <= i31 / page_size && num_tokens <= i31 / ((kv_heads + 1) / 2);
  record = record && p.src_stride_token[0] == p.src_stride_token[1] && p.src_stride_head[0] == p.src_stride_head[1] &&
           fits(p.src_stride_token[0]) && fits(p.src_stride_head[0]) &&
           std::llabs(p.src_stride_head[0]) <= (i31 - head_dim) / (kv_heads + 1);
  for (int i = 0; i < 3; ++i)
    record = record && p.data_stride[1][i] == p.data_stride[0][i] && p.scale_stride[0][i] == p.data_stride[0][i] &&
             p.scale_stride[1][i] == p.data_stride[0][i] && fits(p.data_stride[0][i]);
  record = record && std::llabs(p.data_stride[0][1]) <= i31 / (2 * page_size) &&
           std::llabs(p.data_stride[0][2]) <= i31 / (2 * (kv_heads + 1)) && fits(gap(p.scale[0], p.data[0])) &&
           fits(gap(p.data[1], p.data[0])) && fits(gap(p.scale[1], p.data[0]));
  p.record = record ? 1 : 0;
  if (record) {
    p.src_token32 = (int32_t)p.src_stride_token[0];
    p.src_head32 = (int32_t)p.src_stride_head[0];
    p.rec_block32 = (int32_t)p.data_stride[0][0];
    p.rec_token32 = (int32_t)p.data_stride[0][1];
    p.rec_head32 = (int32_t)p.data_stride[0][2];
    p.off_ks = (int32_t)gap(p.scale[0], p.data[0]);
    p.off_vd = (int32_t)gap(p.data[1], p.data[0]);
    p.off_vs = (int32_t)gap(p.scale[1], p.data[0]);
  }
  p.num_slots = record ? num_blocks * page_size : 0;
  // Division by the invariant page size (Granlund & Montgomery, "Division by
  // invariant integers using multiplication", PLDI 1994): with L = ceil(log2 d),
  // s = 31 + L and m = ceil(2^s / d) < 2^32, floor(n * m / 2^s) = floor(n / d)
  // for every 0 <= n < 2^31.
  {
    int L = 0;
    while ((1LL << L) < page_size) ++L;
    p.page_shift = 31 + L;
    p.page_magic = record ? (((uint64_t)1 << p.page_shift) + (uint64_t)page_size - 1) / (uint64_t)page_size : 0;
  }
  // Scale table by exact power-of-two scaling of g / k when both global scales are in range.
  auto scalable = [](float g) { return std::isfinite(g) && std::fabs(g) >= 0x1p-117f && std::fabs(g) <= 0x1p100f; };
  p.zero = 0.0f;
  auto plain = [](float g) { return g >= 0x1p-6f && g <= 0x1p28f; };
  p.plain = (plain(key_global_scale) && plain(value_global_scale)) ? 1 : 0;
  p.lut_by_scaling = (scalable(key_global_scale) && scalable(value_global_scale)) ? 1 : 0;

  // Packed-row stores are (head_dim/64)-byte words when rows and strides are aligned to that width; any
  // other layout (the reference takes any strides with a contiguous last dim) stores bytes.
  const int store_bytes = head_dim / 64;
  p.byte_store = 0;
  for (int r = 0; r < 2; ++r) {
    if (!aligned_to(p.data[r], store_bytes)) p.byte_store = 1;
    for (int i = 0; i < 3; ++i)
      if (p.data_stride[r][i] % store_bytes) p.byte_store = 1;
  }
  // Source rows: 2-byte aligned always (bf16); vector loads when 16-byte aligned.
  const int vec_bytes = head_dim >= 256 ? 16 : head_dim / 16;  // bytes per lane load
  bool vec = true;
  for (int r = 0; r < 2; ++r) {
    if (!aligned_to(p.src[r], 2)) return NVQSA_ERR_MISALIGNED;
    if (!aligned_to(p.src[r], vec_bytes) || (p.src_stride_token[r] * 2) % vec_bytes ||
        (p.src_stride_head[r] * 2) % vec_bytes)
      vec = false;
  }
  p.vec_src = vec ? 1 : 0;
  p.group_path = (head_dim == 256 && record && vec && aligned_to(p.data[0], 8) && p.off_ks % 8 == 0 &&
                  p.off_vd % 8 == 0 && p.rec_block32 % 8 == 0 && p.rec_token32 % 8 == 0 && p.rec_head32 % 8 == 0)
                     ? 1
                     : 0;
  go = true;
  return NVQSA_OK;
}

extern "C" int nvqsa_write_cache(
    const void* key, int64_t key_stride_token, int64_t key_stride_head,
    const void* value, int64_t value_stride_token, int64_t value_stride_head,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int64_t num_tokens, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size,
    float key_global_scale, float value_global_scale, void* stream) {
  WriteParams p;
  bool go = false;
  const int st = prepare_write(p, go, key, key_stride_token, key_stride_head, value, value_stride_token,
                               value_stride_head, key_data, kd_stride_block, kd_stride_token, kd_stride_head,
                               key_scale, ks_stride_block, ks_stride_token, ks_stride_head, value_data,
                               vd_stride_block, vd_stride_token, vd_stride_head, value_scale, vs_stride_block,
                               vs_stride_token, vs_stride_head, slot_mapping, num_tokens, kv_heads, head_dim,
                               num_blocks, page_size, key_global_scale, value_global_scale);
  if (st != NVQSA_OK || !go) return st;
  const cudaError_t err = launch_write_any<false>(p, head_dim, as_stream(stream));
  return err == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}

extern "C" int nvqsa_norm_rope_write_cache(
    const void* key, int64_t key_stride_token, int64_t key_stride_head,
    const void* value, int64_t value_stride_token, int64_t value_stride_head,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int64_t num_tokens, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size, float key_global_scale, float value_global_scale,
    const float* norm_weight, float norm_weight_offset, float eps,
    const int64_t* positions, const void* cos_sin_cache, int64_t cos_sin_stride, int64_t max_position,
    int32_t rotary_dim, int32_t is_neox_style,
    void* key_out, int64_t key_out_stride_token, int64_t key_out_stride_head, void* stream) {
  // Rotation and norm arguments first, so that bad ones are reported even for an empty batch.
  if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512) return NVQSA_ERR_HEAD_DIM;
  const int epl = head_dim / 32;
  if (rotary_dim < 0 || rotary_dim > head_dim || rotary_dim % (2 * epl) != 0) return NVQSA_ERR_BAD_SHAPE;
  if (rotary_dim > 0) {
    if (!positions || !cos_sin_cache) return NVQSA_ERR_NULL_POINTER;
    if (max_position < 1 || cos_sin_stride < rotary_dim) return NVQSA_ERR_BAD_SHAPE;
    if (!aligned_to(cos_sin_cache, 2)) return NVQSA_ERR_MISALIGNED;
  }
  if (!(eps >= 0.0f) || !std::isfinite(eps) || !std::isfinite(norm_weight_offset)) return NVQSA_ERR_BAD_SHAPE;
  if (norm_weight && !aligned_to(norm_weight, 4)) return NVQSA_ERR_MISALIGNED;

  WriteParams p;
  bool go = false;
  const int st = prepare_write(p, go, key, key_stride_token, key_stride_head, value, value_stride_token,
                               value_stride_head, key_data, kd_stride_block, kd_stride_token, kd_stride_head,
                               key_scale, ks_stride_block, ks_stride_token, ks_stride_head, value_data,
                               vd_stride_block, vd_stride_token, vd_stride_head, value_scale, vs_stride_block,
                               vs_stride_token, vs_stride_head, slot_mapping, num_tokens, kv_heads, head_dim,
                               num_blocks, page_size, key_global_scale, value_global_scale);
  if (st != NVQSA_OK || !go) return st;
  p.norm_weight = norm_weight;
  p.norm_offset = norm_weight_offset;
  p.norm_eps = eps;
  p.inv_head_dim = 1.0f / (float)head_dim;  // a power of two: exact
  p.rot_dim = rotary_dim;
  p.neox = is_neox_style ? 1 : 0;
  p.positions = positions;
  p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin_cache);
  p.cos_sin_stride = cos_sin_stride;
  p.max_position = max_position;
  // A lane reads head_dim/32 (NeoX) or head_dim/64 (GPT-J) consecutive cos and sin values starting at a
  // multiple of that count, with one vector load each: the table base and row stride must keep that
  // alignment (a contiguous table always does, since rotary_dim is a multiple of head_dim/16).
  if (rotary_dim > 0) {
    const int run_bytes = 2 * (is_neox_style ? epl : (epl / 2 > 0 ? epl / 2 : 1));
    if (!aligned_to(cos_sin_cache, run_bytes) || (cos_sin_stride * 2) % run_bytes != 0) return NVQSA_ERR_MISALIGNED;
  }
  p.key_out = static_cast<__nv_bfloat16*>(key_out);
  p.key_out_stride_token = key_out_stride_token;
  p.key_out_stride_head = key_out_stride_head;
  // key_out rows take one vector store per lane: base and strides aligned to min(head_dim/16, 16) bytes
  const int ko_bytes = 2 * epl > 16 ? 16 : 2 * epl;
  if (key_out && (!aligned_to(key_out, ko_bytes) || (key_out_stride_token * 2) % ko_bytes != 0 ||
                  (key_out_stride_head * 2) % ko_bytes != 0))
    return NVQSA_ERR_MISALIGNED;
  const cudaError_t err = launch_write_any<true>(p, head_dim, as_stream(stream));
  return err == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}

// ---------------- K/V projection fused with the writer ----------------
namespace {

using PwEncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// bf16 matrix [rows, cols] with a row stride in elements, read in boxes of 64 columns x box_rows rows
// swizzled in 128-byte rows; rows and columns past the end read as zero.
bool pw_encode(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int64_t row_stride,
               uint32_t box_rows) {
  static std::atomic<PwEncodeTiledFn> encode{nullptr};
  PwEncodeTiledFn fn = encode.load(std::memory_order_acquire);
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !f)
      return false;
    fn = reinterpret_cast<PwEncodeTiledFn>(f);
    encode.store(fn, std::memory_order_release);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kPwBK, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kPwMaxDevices = 64;
std::atomic<int> g_pw_smem_set[kPwMaxDevices][2];

}  // namespace

extern "C" int nvqsa_kv_proj_write_cache(
    const void* hidden, int64_t hidden_stride_token, int64_t num_tokens, int32_t hidden_size,
    const void* key_weight, const void* value_weight, int64_t weight_stride_row,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size, float key_global_scale, float value_global_scale,
    const float* norm_weight, float norm_weight_offset, float eps,
    const int64_t* positions, const void* cos_sin_cache, int64_t cos_sin_stride, int64_t max_position,
    int32_t rotary_dim, int32_t is_neox_style,
    void* key_out, int64_t key_out_stride_token, int64_t key_out_stride_head,
    void* value_out, int64_t value_out_stride_token, int64_t value_out_stride_head, void* stream) {
  if (head_dim != kPwBN) return NVQSA_ERR_HEAD_DIM;
  if (num_tokens < 0 || kv_heads < 1 || hidden_size < 1 || num_blocks < 0 || page_size < 1)
    return NVQSA_ERR_BAD_SHAPE;
  if (hidden_stride_token < hidden_size || weight_stride_row < hidden_size) return NVQSA_ERR_BAD_SHAPE;
  if ((num_tokens + 127) / 128 > 65535 || kv_heads > 32767) return NVQSA_ERR_BAD_SHAPE;
  const bool neox = is_neox_style != 0;
  if (rotary_dim < 0 || rotary_dim > head_dim || rotary_dim % (neox ? 32 : 16) != 0) return NVQSA_ERR_BAD_SHAPE;
  if (rotary_dim > 0) {
    if (!positions || !cos_sin_cache) return NVQSA_ERR_NULL_POINTER;
    if (max_position < 1 || cos_sin_stride < rotary_dim) return NVQSA_ERR_BAD_SHAPE;
    if (!aligned_to(cos_sin_cache, 16) || (cos_sin_stride * 2) % 16 != 0) return NVQSA_ERR_MISALIGNED;
  }
  if (!(eps >= 0.0f) || !std::isfinite(eps) || !std::isfinite(norm_weight_offset)) return NVQSA_ERR_BAD_SHAPE;
  if (norm_weight && !aligned_to(norm_weight, 16)) return NVQSA_ERR_MISALIGNED;
  if (!hidden || !key_weight || !value_weight) return NVQSA_ERR_NULL_POINTER;
  if (!aligned_to(hidden, 16) || !aligned_to(key_weight, 16) || !aligned_to(value_weight, 16) ||
      (hidden_stride_token * 2) % 16 != 0 || (weight_stride_row * 2) % 16 != 0)
    return NVQSA_ERR_MISALIGNED;
  auto out_ok = [](const void* o, int64_t st, int64_t sh) {
    return !o || (aligned_to(o, 16) && (st * 2) % 16 == 0 && (sh * 2) % 16 == 0);
  };
  if (!out_ok(key_out, key_out_stride_token, key_out_stride_head) ||
      !out_ok(value_out, value_out_stride_token, value_out_stride_head))
    return NVQSA_ERR_MISALIGNED;

  WriteParams w;
  bool go = false;
  const int st = prepare_write(w, go, hidden, 0, 0, hidden, 0, 0, key_data, kd_stride_block, kd_stride_token,
                               kd_stride_head, key_scale, ks_stride_block, ks_stride_token, ks_stride_head, value_data,
                               vd_stride_block, vd_stride_token, vd_stride_head, value_scale, vs_stride_block,
                               vs_stride_token, vs_stride_head, slot_mapping, num_tokens, kv_heads, head_dim,
                               num_blocks, page_size, key_global_scale, value_global_scale);
  if (st != NVQSA_OK || !go) return st;
  // the epilogue addresses a token's four regions from one record base and writes them in 16-byte chunks
  if (!w.record || !aligned_to(w.data[0], 16) || w.off_ks % 16 != 0 || w.off_vd % 16 != 0 || w.off_vs % 16 != 0 ||
      w.rec_block32 % 16 != 0 || w.rec_token32 % 16 != 0 || w.rec_head32 % 16 != 0)
    return NVQSA_ERR_MISALIGNED;
  w.norm_weight = norm_weight;
  w.norm_offset = norm_weight_offset;
  w.norm_eps = eps;
  w.inv_head_dim = 1.0f / (float)head_dim;
  w.rot_dim = rotary_dim;
  w.neox = neox ? 1 : 0;
  w.positions = positions;
  w.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin_cache);
  w.cos_sin_stride = cos_sin_stride;
  w.max_position = max_position;
  w.key_out = static_cast<__nv_bfloat16*>(key_out);
  w.key_out_stride_token = key_out_stride_token;
  w.key_out_stride_head = key_out_stride_head;

  ProjParams pp;
  pp.w = w;
  pp.kblocks = (hidden_size + kPwBK - 1) / kPwBK;
  pp.ksplit = 1;
  pp.kbs = pp.kblocks;
  pp.value_out = static_cast<__nv_bfloat16*>(value_out);
  pp.value_out_stride_token = value_out_stride_token;
  pp.value_out_stride_head = value_out_stride_head;
  const int64_t wrows = (int64_t)kv_heads * head_dim;
  // 256-token CTAs (two accumulators sharing each weight tile) once 128-token CTAs would take more than one
  // wave: half the weight traffic per token and one epilogue per 256 tokens
  const int sms = device_sm_count();
  const int64_t ctas128 = (num_tokens + 127) / 128 * 2 * kv_heads;
  const int mh = ctas128 > (sms > 0 ? sms : 148) ? 2 : 1;
  const int bm = 128 * mh;
  if (!pw_encode(&pp.map_x, hidden, hidden_size, num_tokens, hidden_stride_token, (uint32_t)bm) ||
      !pw_encode(&pp.map_w[0], key_weight, hidden_size, wrows, weight_stride_row, kPwBN) ||
      !pw_encode(&pp.map_w[1], value_weight, hidden_size, wrows, weight_stride_row, kPwBN))
    return NVQSA_ERR_CUDA;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kPwMaxDevices) return NVQSA_ERR_CUDA;
  const void* fn = mh == 2 ? reinterpret_cast<const void*>(kv_proj_write_kernel<2>)
                           : reinterpret_cast<const void*>(kv_proj_write_kernel<1>);
  const size_t smem = (mh == 2 ? sizeof(SmemPw<2>) : sizeof(SmemPw<1>)) + 1024;
  if (!g_pw_smem_set[dev][mh - 1].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return NVQSA_ERR_CUDA;
    g_pw_smem_set[dev][mh - 1].store(1, std::memory_order_release);
  }
  const unsigned mtiles = (unsigned)((num_tokens + bm - 1) / bm);
  if (mh == 1) {
    // few tiles (decode batches): split each tile's k-blocks over a cluster of up to 8 CTAs so that the
    // weights are read by that many more SMs; every rank keeps at least one k-block
    const int64_t tiles = (int64_t)mtiles * 2 * kv_heads;
    const int fill = (int)std::min<int64_t>(8, (sms > 0 ? sms : 148) / std::max<int64_t>(tiles, 1));
    const int cand = std::min(fill, pp.kblocks);
    if (cand >= 2) {
      pp.kbs = (pp.kblocks + cand - 1) / cand;
      pp.ksplit = (pp.kblocks + pp.kbs - 1) / pp.kbs;
    }
    if (pp.ksplit > 1) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(2 * kv_heads * pp.ksplit), mtiles);
      cfg.blockDim = dim3(PwShape<1>::kThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = as_stream(stream);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)pp.ksplit;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, kv_proj_write_kernel<1>, pp) == cudaSuccess) return NVQSA_OK;
      (void)cudaGetLastError();  // clusters of this size not schedulable here: run unsplit
      pp.ksplit = 1;
      pp.kbs = pp.kblocks;
    }
  }
  const dim3 grid((unsigned)(2 * kv_heads), mtiles);
  if (mh == 2)
    kv_proj_write_kernel<2><<<grid, PwShape<2>::kThreads, smem, as_stream(stream)>>>(pp);
  else
    kv_proj_write_kernel<1><<<grid, PwShape<1>::kThreads, smem, as_stream(stream)>>>(pp);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}
