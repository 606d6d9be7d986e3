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
// loads are in flight.
template <int HEAD_DIM, bool VEC, bool RECORD>
__global__ void __launch_bounds__(256, HEAD_DIM >= 512 ? 2 : 4) write_cache_kernel(const WriteParams p) {
  constexpr int EPL = HEAD_DIM / 32;
  constexpr int NW = EPL / 2;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int head_pairs = (p.kv_heads + 1) >> 1;
  const int64_t items = p.num_tokens * head_pairs;
  __shared__ float out_scale_lut[2][256];
  __shared__ float quot[2][16];

  int64_t token = 0, slot = -1;
  int h0 = 0;
  uint32_t x[4][NW];  // K h0, V h0, K h1, V h1
  auto load_item = [&](int64_t w) {
    item_token<RECORD>(w, head_pairs, token, h0);
    slot = __ldg(p.slots + token);
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

  const int64_t w0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w0 < items) load_item(w0);
  build_out_scale_lut(p, out_scale_lut, quot);
  __syncthreads();
  for (int64_t w = w0; w < items; w += warps) {
    if (w != w0) load_item(w);
    int64_t block, offset;
    if (slot_position<RECORD>(p, slot, block, offset))
      write_item<EPL, RECORD>(p, out_scale_lut, lane, block, offset, h0, x);
  }
}

template <int HD, bool VEC, bool RECORD>
cudaError_t launch_write_impl(const WriteParams& p, cudaStream_t stream) {
  const int64_t items = p.num_tokens * ((p.kv_heads + 1) / 2);
  const int threads = 256;
  const int warps_per_block = threads / 32;
  int64_t blocks = (items + warps_per_block - 1) / warps_per_block;
  // One resident wave (occupancy of this instantiation on this device); grid-stride beyond.
  static int per_sm = 0;
  if (per_sm <= 0 &&
      (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, write_cache_kernel<HD, VEC, RECORD>, threads, 0) !=
           cudaSuccess ||
       per_sm <= 0))
    per_sm = 2;
  const int sms = device_sm_count();
  const int64_t cap = (int64_t)(sms > 0 ? sms : 148) * per_sm;
  if (blocks > cap) blocks = cap;
  write_cache_kernel<HD, VEC, RECORD><<<(unsigned)blocks, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_write(const WriteParams& p, cudaStream_t stream) {
  if (p.record)
    return p.vec_src ? launch_write_impl<HD, true, true>(p, stream) : launch_write_impl<HD, false, true>(p, stream);
  return p.vec_src ? launch_write_impl<HD, true, false>(p, stream) : launch_write_impl<HD, false, false>(p, stream);
}

}  // namespace
}  // namespace nvqsa

using namespace nvqsa;

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
  if (num_tokens < 0 || kv_heads < 0 || num_blocks < 0 || page_size < 1) return NVQSA_ERR_BAD_SHAPE;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512) return NVQSA_ERR_HEAD_DIM;
  if (num_tokens == 0 || kv_heads == 0 || num_blocks == 0) return NVQSA_OK;
  if (!key || !value || !key_data || !key_scale || !value_data || !value_scale || !slot_mapping)
    return NVQSA_ERR_NULL_POINTER;

  WriteParams p;
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

  // Packed-row stores are (head_dim/64)-byte words: rows and strides must be
  // aligned to that width.
  const int store_bytes = head_dim / 64;
  for (int r = 0; r < 2; ++r) {
    if (!aligned_to(p.data[r], store_bytes)) return NVQSA_ERR_MISALIGNED;
    for (int i = 0; i < 3; ++i)
      if (p.data_stride[r][i] % store_bytes) return NVQSA_ERR_MISALIGNED;
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

  cudaError_t err;
  cudaStream_t s = as_stream(stream);
  switch (head_dim) {
    case 64: err = launch_write<64>(p, s); break;
    case 128: err = launch_write<128>(p, s); break;
    case 256: err = launch_write<256>(p, s); break;
    default: err = launch_write<512>(p, s); break;
  }
  return err == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}
