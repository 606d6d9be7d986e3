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
  float global_scale[2];
  int32_t kv_heads;
  int32_t vec_src;      // 1: 16-byte aligned source rows -> vector loads
  int32_t small_slots;  // 1: num_blocks * page_size < 2^31
};

template <int EPL>
struct Vec;  // EPL bf16 values loaded per lane
template <>
struct Vec<2> { using T = uint32_t; };
template <>
struct Vec<4> { using T = uint2; };
template <>
struct Vec<8> { using T = uint4; };

template <int EPL, bool VEC>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&x)[EPL]) {
  if constexpr (VEC && EPL <= 8) {
    typename Vec<EPL>::T v = __ldg(reinterpret_cast<const typename Vec<EPL>::T*>(p));
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else if constexpr (VEC) {
#pragma unroll
    for (int q = 0; q < EPL / 8; ++q) {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + q);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[8 * q + 2 * i] = __uint_as_float(w[i] << 16);
        x[8 * q + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
  } else {
    const unsigned short* s = reinterpret_cast<const unsigned short*>(p);
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = __uint_as_float(((uint32_t)__ldg(s + i)) << 16);
  }
}

// Encode the EPL values this lane holds; returns the packed codes
// (EPL/2 bytes, element 2j in the low nibble of byte j) and the group's
// E4M3 scale byte (identical on every lane of the group).  out_scale_lut[b]
// holds g / max(e4m3(b), 1e-30) for every scale byte b, computed with the
// same IEEE division (oracle.py:57), so the per-group divide is a table read.
template <int EPL>
__device__ __forceinline__ void encode_lane(const float (&x)[EPL], float g, const float* out_scale_lut,
                                            uint32_t (&packed)[(EPL + 7) / 8], uint32_t& scale_byte) {
  constexpr int LPG = 16 / EPL;  // lanes sharing one 16-element group
  // NaN-propagating amax: for |x| bit patterns integer order == float order,
  // and NaN patterns sort above +inf.
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < EPL; ++i) amax_bits = max(amax_bits, __float_as_uint(x[i]) & 0x7fffffffu);
#pragma unroll
  for (int m = 1; m < LPG; m <<= 1) amax_bits = max(amax_bits, __shfl_xor_sync(0xffffffffu, amax_bits, m));
  const float amax = __uint_as_float(amax_bits);

  float bs = __fdiv_rn(__fmul_rn(g, amax), 6.0f);
  bs = (bs > 448.0f) ? 448.0f : bs;  // NaN stays NaN -> 0x7f below
  scale_byte = cvt_e4m3(bs);
  const float out_scale = out_scale_lut[scale_byte];

#pragma unroll
  for (int j = 0; j < (EPL + 7) / 8; ++j) packed[j] = 0;
  // y = x * out_scale is NaN only when the group holds a NaN / inf input or
  // out_scale is NaN or zero; only then is the per-element NaN -> 0 rule
  // (oracle.py:42: every threshold test is false for NaN) needed.
  const bool nan_possible = !(amax_bits < 0x7f800000u && out_scale > 0.0f);
  const bool slow = __any_sync(0xffffffffu, nan_possible);
  if constexpr (EPL >= 8) {
#pragma unroll
    for (int j = 0; j < EPL / 8; ++j) {
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // -0 + 0 = +0: the oracle's sign is y < 0, hardware keeps the sign of -0
        y[i] = __fadd_rn(__fmul_rn(x[8 * j + i], out_scale), 0.0f);
        if (slow) y[i] = (y[i] != y[i]) ? 0.0f : y[i];
      }
      packed[j] = cvt_e2m1x8(y);
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      const float lo = e2m1_prepare(__fmul_rn(x[2 * i], out_scale));
      const float hi = e2m1_prepare(__fmul_rn(x[2 * i + 1], out_scale));
      packed[i / 4] |= cvt_e2m1x2(hi, lo) << (8 * (i % 4));
    }
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

// One warp per (token, pair of kv heads); grid-stride over all items.  Every
// global load of an item (the slot and the K and V rows of both heads) is
// issued before the first use, so a warp waits for memory once per item.
template <int HEAD_DIM, bool VEC>
__global__ void __launch_bounds__(256) write_cache_kernel(const WriteParams p) {
  constexpr int EPL = HEAD_DIM / 32;
  constexpr int LPG = 16 / EPL;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int head_pairs = (p.kv_heads + 1) >> 1;
  // g / max(scale, 1e-30) for every E4M3 scale byte, K and V (oracle.py:57).
  __shared__ float out_scale_lut[2][256];
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const float bs = e4m3_to_f32((uint32_t)(i & 255));
    const float den = (bs < 1e-30f) ? 1e-30f : bs;  // clamp_min; NaN stays NaN
    out_scale_lut[i >> 8][i & 255] = __fdiv_rn(p.global_scale[i >> 8], den);
  }
  __syncthreads();
  const int64_t items = p.num_tokens * head_pairs;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < items; w += warps) {
    const int64_t token = head_pairs == 1 ? w : w / head_pairs;
    const int h0 = 2 * (int)(w - token * head_pairs);
    const bool two = h0 + 1 < p.kv_heads;
    const int64_t slot = __ldg(p.slots + token);
    float x[4][EPL];  // K h0, V h0, K h1, V h1
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int head = two ? h0 + hh : h0;
#pragma unroll
      for (int r = 0; r < 2; ++r)
        load_row<EPL, VEC>(p.src[r] + token * p.src_stride_token[r] + head * p.src_stride_head[r] + lane * EPL,
                           x[2 * hh + r]);
    }
    if (slot < 0) continue;  // kernels.py:71-77: negative slots are skipped
    int64_t block, offset;
    if (p.small_slots) {  // every valid slot fits in 32 bits: 32-bit division
      if (slot >= p.num_blocks * p.page_size) continue;
      const uint32_t b32 = (uint32_t)slot / (uint32_t)p.page_size;
      block = b32;
      offset = (int64_t)((uint32_t)slot - b32 * (uint32_t)p.page_size);
    } else {
      block = slot / p.page_size;
      if (block >= p.num_blocks) continue;
      offset = slot - block * p.page_size;
    }
    // Row bases of this token's slot, computed once per item.
    uint8_t* drow[2];
    uint8_t* srow[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      drow[r] = p.data[r] + block * p.data_stride[r][0] + offset * p.data_stride[r][1] + h0 * p.data_stride[r][2];
      srow[r] = p.scale[r] + block * p.scale_stride[r][0] + offset * p.scale_stride[r][1] + h0 * p.scale_stride[r][2];
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      if (hh == 1 && !two) break;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        uint32_t packed[(EPL + 7) / 8];
        uint32_t sbyte;
        encode_lane<EPL>(x[2 * hh + r], p.global_scale[r], out_scale_lut[r], packed, sbyte);
        store_lane<EPL>(drow[r] + hh * p.data_stride[r][2], lane, packed);
        if ((lane % LPG) == 0) (srow[r] + hh * p.scale_stride[r][2])[lane / LPG] = (uint8_t)sbyte;
      }
    }
  }
}

template <int HD, bool VEC>
cudaError_t launch_write_impl(const WriteParams& p, cudaStream_t stream) {
  const int64_t items = p.num_tokens * ((p.kv_heads + 1) / 2);
  const int threads = 256;
  const int warps_per_block = threads / 32;
  int64_t blocks = (items + warps_per_block - 1) / warps_per_block;
  // One resident wave (occupancy of this instantiation on this device); grid-stride beyond.
  static int per_sm = 0;
  if (per_sm <= 0 &&
      (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, write_cache_kernel<HD, VEC>, threads, 0) !=
           cudaSuccess ||
       per_sm <= 0))
    per_sm = 2;
  const int sms = device_sm_count();
  const int64_t cap = (int64_t)(sms > 0 ? sms : 148) * per_sm;
  if (blocks > cap) blocks = cap;
  write_cache_kernel<HD, VEC><<<(unsigned)blocks, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_write(const WriteParams& p, cudaStream_t stream) {
  return p.vec_src ? launch_write_impl<HD, true>(p, stream) : launch_write_impl<HD, false>(p, stream);
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
  p.small_slots = (num_blocks <= 0x7fffffffLL / page_size) ? 1 : 0;

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
