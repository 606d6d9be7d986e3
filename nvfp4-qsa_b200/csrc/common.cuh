// Shared device helpers for the NVFP4 QSA kernels (sm_100a).
//
// Numeric contract: every helper here is exact or IEEE round-to-nearest-even
// and is written with explicit __f*_rn intrinsics so that nvcc cannot contract
// a multiply and an add into an FMA; the writer's bytes must equal the
// reference codec (python/nvfp4_qsa/oracle.py:47-69) bit for bit.
#pragma once

#include <atomic>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "nvfp4_qsa.h"

namespace nvqsa {

// ---------------------------------------------------------------------------
// Conversions (PTX cvt forms introduced for sm_100a).
// ---------------------------------------------------------------------------

// Two fp32 -> one byte of two E2M1 codes, round-to-nearest-even, saturating
// to +-6.  `hi` lands in bits 7:4, `lo` in bits 3:0.  Measured on B200 to agree
// with the reference's threshold rounding (oracle.py:30-44) for every finite
// fp32 once -0 is mapped to +0 and NaN to 0 (see e2m1_prepare).
__device__ __forceinline__ uint32_t cvt_e2m1x2(float hi, float lo) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\t"
      "mov.b32 %0, {b, 0, 0, 0};\n\t}"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out & 0xffu;
}

// Eight fp32 -> one word of eight E2M1 codes (element 2j in the low nibble of
// byte j), same rounding as cvt_e2m1x2.
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float (&y)[8]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(y[0]), "f"(y[1]), "f"(y[2]), "f"(y[3]), "f"(y[4]), "f"(y[5]), "f"(y[6]), "f"(y[7]));
  return out;
}

// The reference takes sign = (y < 0) and maps NaN to code 0 (all its threshold
// comparisons are false).  Hardware cvt keeps the sign of -0 and saturates NaN,
// so normalise first: -0 + 0 = +0 under round-to-nearest, NaN -> 0.  `zero`
// must be a +0.0f the compiler cannot see (a kernel parameter): an add of a
// literal zero whose only use is the E2M1 conversion is dropped, and -0 then
// converts to code 8.
__device__ __forceinline__ float e2m1_prepare(float y, float zero) {
  float z = __fadd_rn(y, zero);
  return (z != z) ? 0.0f : z;
}

// fp32 -> E4M3 byte (round-to-nearest-even, saturate to 448, NaN -> 0x7f).
__device__ __forceinline__ uint32_t cvt_e4m3(float x) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(0.0f), "f"(x));
  return out & 0xffu;
}

// Two E4M3 bytes (lo in bits 7:0) -> f16x2, exact.
__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t two_bytes) {
  uint32_t out;
  uint16_t v = (uint16_t)two_bytes;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(v));
  return out;
}

// E4M3 byte -> fp32, exact.
__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  uint32_t h2 = cvt_e4m3x2_f16x2(byte & 0xffu);
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu)));
}

// One byte holding two E2M1 codes -> f16x2 (low nibble -> low half), exact.
// The byte is taken from bits 7:0 of `w`.
__device__ __forceinline__ uint32_t cvt_e2m1x2_f16x2(uint32_t w) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
      : "=r"(out)
      : "r"(w));
  return out;
}

// Byte k (0..3) of w -> f16x2.
template <int K>
__device__ __forceinline__ uint32_t cvt_e2m1x2_f16x2_byte(uint32_t w) {
  uint32_t out;
  if constexpr (K == 0) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}" : "=r"(out) : "r"(w));
  } else if constexpr (K == 1) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b1;\n\t}" : "=r"(out) : "r"(w));
  } else if constexpr (K == 2) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b2;\n\t}" : "=r"(out) : "r"(w));
  } else {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b3;\n\t}" : "=r"(out) : "r"(w));
  }
  return out;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 x = *reinterpret_cast<__half2*>(&a);
  __half2 y = *reinterpret_cast<__half2*>(&b);
  __half2 r = __hmul2(x, y);
  return *reinterpret_cast<uint32_t*>(&r);
}

// x / 6 rounded to nearest even, bit-identical to the IEEE division of the
// codec oracle (oracle.py:54).  For 2^-100 <= |x| < 2^127 it is Markstein's
// correction of the product with the rounded reciprocal: q = x * RN(1/6) is
// within one ulp of x/6, the remainder r = x - 6q is exact under FMA, and
// q + r * RN(1/6) rounds to the correctly rounded quotient (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990; the same one-FMA correction of a
// product with a rounded constant is analysed by N. Brisebarre and J.-M.
// Muller, "Correctly rounded multiplication by arbitrary precision
// constants", IEEE Trans. Computers 57(2), 2008).  Zeros keep their sign.
// div6_fast returns that quotient and clears `exact` for NaN, infinities and
// |x| outside [2^-100, 2^127), which take the IEEE division (div6_rn does it
// per value; the writer does it once per warp when any lane needs it).
// Checked against the IEEE division for all 2^32 inputs by the GPU tests.
__device__ __forceinline__ float div6_fast(float x, bool& exact) {
  const uint32_t b = __float_as_uint(x) & 0x7fffffffu;
  const float c = 0x1.555556p-3f;  // RN(1/6)
  const float q = __fmul_rn(x, c);
  const float r = __fmaf_rn(-q, 6.0f, x);
  const float q1 = __fmaf_rn(r, c, q);
  exact = (b - 0x0d800000u < 0x7f000000u - 0x0d800000u) || b == 0u;
  return b == 0u ? x : q1;
}

__device__ __forceinline__ float div6_rn(float x) {
  bool exact;
  const float q = div6_fast(x, exact);
  return exact ? q : __fdiv_rn(x, 6.0f);
}

// ---------------------------------------------------------------------------
// Launch helpers.
// ---------------------------------------------------------------------------
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return sms;
}

inline bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Resident blocks per SM of one kernel instantiation, looked up once per device (devices of different kinds
// in one process keep their own figure).  Atomic entries: concurrent first calls store the same value.
struct OccupancyCache {
  static constexpr int kDevices = 64;
  std::atomic<int> per_sm[kDevices] = {};
  template <typename Kernel>
  int get(Kernel kernel, int threads) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevices) return 2;
    int v = per_sm[dev].load(std::memory_order_relaxed);
    if (v <= 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, threads, 0) != cudaSuccess || v <= 0) v = 2;
      per_sm[dev].store(v, std::memory_order_relaxed);
    }
    return v;
  }
};

}  // namespace nvqsa
