// Flat NVFP4 codec on device rows: the GPU form of the reference package's
// encode()/decode() (python/nvfp4_qsa/oracle.py:47-85), used by the
// nvfp4_qsa.encode / nvfp4_qsa.decode host API.  Not the serving hot path
// (the paged writer in write_cache.cu is); kept simple: one thread per group
// for encode, one thread per packed byte for decode.
#include "common.cuh"

namespace nvqsa {
namespace {

__global__ void encode_rows_kernel(const float* __restrict__ x, int64_t groups, int block_size,
                                   const float* __restrict__ gptr, uint8_t* __restrict__ nibbles,
                                   uint8_t* __restrict__ packed, uint8_t* __restrict__ scales,
                                   int64_t* __restrict__ counts, float zero) {
  const float g = __ldg(gptr);
  unsigned long long clip = 0, sat = 0;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const float* xp = x + gi * block_size;
    uint32_t amax_bits = 0;  // NaN-propagating |x| max (oracle.py:53 amax)
    for (int i = 0; i < block_size; ++i) amax_bits = max(amax_bits, __float_as_uint(__ldg(xp + i)) & 0x7fffffffu);
    float bs = __fdiv_rn(__fmul_rn(g, __uint_as_float(amax_bits)), 6.0f);  // oracle.py:54
    bs = (bs > 448.0f) ? 448.0f : bs;
    if (fabsf(bs) >= 447.999f) ++sat;  // oracle.py:64 blockscale_sat_rate
    const uint32_t sbyte = cvt_e4m3(bs);
    const float bs_f32 = e4m3_to_f32(sbyte);
    const float den = (bs_f32 < 1e-30f) ? 1e-30f : bs_f32;
    const float out_scale = __fdiv_rn(g, den);  // oracle.py:57
    scales[gi] = (uint8_t)sbyte;
    for (int i = 0; i < block_size; i += 2) {
      const float y0 = __fmul_rn(__ldg(xp + i), out_scale);
      const float y1 = __fmul_rn(__ldg(xp + i + 1), out_scale);
      clip += (fabsf(y0) > 6.0f) + (fabsf(y1) > 6.0f);  // oracle.py:59 clip6_rate
      const uint32_t byte = cvt_e2m1x2(e2m1_prepare(y1, zero), e2m1_prepare(y0, zero));
      packed[(gi * block_size + i) >> 1] = (uint8_t)byte;
      if (nibbles) {
        nibbles[gi * block_size + i] = (uint8_t)(byte & 0xfu);
        nibbles[gi * block_size + i + 1] = (uint8_t)(byte >> 4);
      }
    }
  }
  if (counts) {
    if (clip) atomicAdd(reinterpret_cast<unsigned long long*>(counts), clip);
    if (sat) atomicAdd(reinterpret_cast<unsigned long long*>(counts) + 1, sat);
  }
}

__device__ __constant__ float kE2m1Grid[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

__global__ void decode_rows_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                   int64_t nbytes, int block_size, const float* __restrict__ gptr,
                                   float* __restrict__ out) {
  const float g = __ldg(gptr);
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nbytes; b += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t byte = __ldg(packed + b);
    const int64_t elem = 2 * b;
    const float f = __fdiv_rn(e4m3_to_f32(__ldg(scales + elem / block_size)), g);  // bs / g (oracle.py:85)
    const uint32_t lo = byte & 0xfu, hi = byte >> 4;
    float v0 = kE2m1Grid[lo & 7u], v1 = kE2m1Grid[hi & 7u];
    v0 = (lo & 8u) ? -v0 : v0;  // sign * magnitude (oracle.py:80-82)
    v1 = (hi & 8u) ? -v1 : v1;
    out[elem] = __fmul_rn(v0, f);
    out[elem + 1] = __fmul_rn(v1, f);
  }
}

unsigned grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  const int sms = device_sm_count();
  const int64_t cap = (int64_t)(sms > 0 ? sms : 148) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

}  // namespace
}  // namespace nvqsa

using namespace nvqsa;

extern "C" int nvqsa_encode_rows(const float* x, int64_t m, int64_t n, int32_t block_size, const float* global_scale,
                                 uint8_t* nibbles, uint8_t* packed, uint8_t* scales, int64_t* counts, void* stream) {
  if (m < 0 || n < 0 || block_size < 2 || (block_size & 1) || (n % block_size)) return NVQSA_ERR_BAD_SHAPE;
  if (m == 0 || n == 0) return NVQSA_OK;
  if (!x || !global_scale || !packed || !scales) return NVQSA_ERR_NULL_POINTER;
  const int64_t groups = m * (n / block_size);
  encode_rows_kernel<<<grid_for(groups, 128), 128, 0, as_stream(stream)>>>(x, groups, block_size, global_scale,
                                                                            nibbles, packed, scales, counts,
                                                                            0.0f);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}

extern "C" int nvqsa_decode_rows(const uint8_t* packed, const uint8_t* scales, int64_t m, int64_t n, int32_t block_size,
                                 const float* global_scale, float* out, void* stream) {
  if (m < 0 || n < 0 || block_size < 2 || (block_size & 1) || (n % block_size)) return NVQSA_ERR_BAD_SHAPE;
  if (m == 0 || n == 0) return NVQSA_OK;
  if (!packed || !scales || !global_scale || !out) return NVQSA_ERR_NULL_POINTER;
  const int64_t nbytes = m * n / 2;
  decode_rows_kernel<<<grid_for(nbytes, 256), 256, 0, as_stream(stream)>>>(packed, scales, nbytes, block_size,
                                                                            global_scale, out);
  return cudaGetLastError() == cudaSuccess ? NVQSA_OK : NVQSA_ERR_LAUNCH;
}

extern "C" const char* nvqsa_status_string(int status) {
  switch (status) {
    case NVQSA_OK: return "ok";
    case NVQSA_ERR_NULL_POINTER: return "a required pointer is NULL";
    case NVQSA_ERR_BAD_SHAPE: return "invalid or inconsistent sizes";
    case NVQSA_ERR_HEAD_DIM: return "head_dim not supported by this build";
    case NVQSA_ERR_MISALIGNED: return "pointer or stride breaks the alignment contract";
    case NVQSA_ERR_WORKSPACE: return "workspace missing or too small";
    case NVQSA_ERR_UNSUPPORTED: return "head grouping or block size not supported by this build";
    case NVQSA_ERR_LAUNCH: return "CUDA kernel launch failed";
    case NVQSA_ERR_CUDA: return "CUDA runtime query failed";
    case NVQSA_ERR_SCRATCH_LIMIT: return "problem needs more scratch than the built-in no-allocation buffer holds";
    default: return "unknown status";
  }
}

extern "C" int nvqsa_abi_version(void) { return 1; }
