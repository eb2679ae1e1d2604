// Shared helpers of libod_b200: status codes, the per-thread error message, dtype conversions with the exact
// rounding points of PyTorch's bf16/fp16 elementwise ops (compute in fp32, round to nearest even once per op).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdarg.h>

#include "../../include/od_b200.h"

namespace od {

// Records a printf-style message as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the last error and returns OD_OK.
int ok();
// Device address of the library's device-side error word on the current device (set by bounded waits).
int32_t* device_error_word();

#define OD_CUDA_TRY(call)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return ::od::fail(OD_ECUDA, "%s failed: %s (%s:%d)", #call,      \
                                             cudaGetErrorString(e_), __FILE__, __LINE__);   \
  } while (0)

#define OD_REQUIRE(cond, ...)                                                               \
  do {                                                                                      \
    if (!(cond)) return ::od::fail(OD_EINVAL, __VA_ARGS__);                                 \
  } while (0)

// After a launch: report configuration errors synchronously (no device sync).
#define OD_LAUNCH_CHECK()                                                                   \
  do {                                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess) return ::od::fail(OD_ECUDA, "kernel launch failed: %s (%s:%d)",  \
                                             cudaGetErrorString(e_), __FILE__, __LINE__);   \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// ------------------------------------------------------------------------------------------------ element types
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// Round through a storage dtype: the value PyTorch holds after one op on that dtype.
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float rhf(float v) { return __half2float(__float2half_rn(v)); }

// Int8Tensor.quantize's scale from a row's absmax: max(amax, 1e-8) / 127 in IEEE fp32.
__device__ __forceinline__ float quant_scale(float amax) { return __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f); }

// RN(1 / s), computed once per row for quant_val.
__device__ __forceinline__ float quant_recip(float s) { return __frcp_rn(s); }

// Int8Tensor.quantize's value: clamp(round_half_even(x / s), -127, 127) with x / s the IEEE fp32 quotient, bit for
// bit, given r = RN(1 / s) and |x / s| <= 128 (x is an element of the row whose absmax gave s). y = RN(x * r) lies
// within 2.3e-5 of RN(x / s) (two roundings of relative size 2^-24 on a value of at most 128), so the two round to
// the same integer unless y is within 1e-4 of a half-integer; only then is the quotient formed. Rounding to
// nearest-even is the addition of 1.5 * 2^23 (exact for |y| < 2^22), whose low mantissa bits are the integer.
__device__ __forceinline__ int quant_int(float x, float s, float r) {
  constexpr float kMagic = 12582912.0f;       // 1.5 * 2^23, bit pattern 0x4B400000
  const float y = __fmul_rn(x, r);
  float t = __fadd_rn(y, kMagic);
  if (fabsf(__fsub_rn(y, __fsub_rn(t, kMagic))) > 0.4999f) t = __fadd_rn(__fdiv_rn(x, s), kMagic);
  return min(max(__float_as_int(t) - 0x4B400000, -127), 127);
}
__device__ __forceinline__ int8_t quant_val(float x, float s, float r) {
  return static_cast<int8_t>(quant_int(x, s, r));
}
// four quantised values packed little-endian into one word
__device__ __forceinline__ uint32_t quant4(float a, float b, float c, float d, float s, float r) {
  return (static_cast<uint32_t>(quant_int(a, s, r)) & 0xFFu) | ((static_cast<uint32_t>(quant_int(b, s, r)) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(quant_int(c, s, r)) & 0xFFu) << 16) | (static_cast<uint32_t>(quant_int(d, s, r)) << 24);
}

// ---- bf16 pairs (two bf16 in one 32-bit word, lower element in the low half)
// RN of the exact product / sum of two bf16 values: equal to rounding the fp32 result to bf16 (a product of two 8-bit
// significands is exact in fp32; a sum is exact unless the exponents differ by more than 16, and then both forms round
// to the larger operand).
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// elementwise max of |a| and |b| (exact; NaN operands are ignored as fmaxf does)
__device__ __forceinline__ uint32_t babsmax2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a & 0x7FFF7FFFu), "r"(b & 0x7FFF7FFFu));
  return d;
}
__device__ __forceinline__ float bmax_halves(uint32_t a) {
  return fmaxf(__uint_as_float(a << 16), __uint_as_float(a & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
__device__ __forceinline__ void unpack8(const uint4& w, float (&v)[8]) {
  const float2 a = unpack2(w.x), b = unpack2(w.y), c = unpack2(w.z), d = unpack2(w.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ uint32_t babsmax4(const uint4& w, uint32_t acc) {
  return babsmax2(acc, babsmax2(babsmax2(w.x, w.y), babsmax2(w.z, w.w)));
}

// Four int8 (one 32-bit word) -> two bf16 pairs of RN(x * s), s a bf16 pair; equal to rounding float(x) * s to bf16,
// since the product of two 8-bit significands is exact. Integer path without the conversion pipe: the byte
// (x ^ 0x80) = x + 128 placed under the exponent of 2^23 gives the float 2^23 + x + 128 exactly; subtracting
// 2^23 + 128 leaves x, whose upper 16 bits are its exact bf16 (|x| <= 128 has at most 8 significant bits).
__device__ __forceinline__ void dequant4_bf16(uint32_t w, uint32_t s2, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float2 off = make_float2(-8388736.f, -8388736.f);
  const float2 f01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651))), off);
  const float2 f23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653))), off);
  const uint32_t x01 = __byte_perm(__float_as_uint(f01.x), __float_as_uint(f01.y), 0x7632);
  const uint32_t x23 = __byte_perm(__float_as_uint(f23.x), __float_as_uint(f23.y), 0x7632);
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(lo) : "r"(x01), "r"(s2));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(hi) : "r"(x23), "r"(s2));
}

// Eight quantised values of a row (quant_int's rounding, two pairs at a time), packed little-endian in two words.
// The byte of round(y) is the low byte of the bits of y + 1.5 * 2^23. No clamp: every element x of the row whose
// absmax gave s has |x / s| <= 127 * (1 + 2^-23), which rounds into [-127, 127].
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float s, float r) {
  constexpr float kMagic = 12582912.0f;
  const float2 r2 = make_float2(r, r), m2 = make_float2(kMagic, kMagic), nm2 = make_float2(-kMagic, -kMagic);
  uint32_t b[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 y = __fmul2_rn(make_float2(v[2 * i], v[2 * i + 1]), r2);
    float2 t = __fadd2_rn(y, m2);
    const float2 n = __fadd2_rn(t, nm2);
    const float2 d = __fadd2_rn(y, make_float2(-n.x, -n.y));
    if (fmaxf(fabsf(d.x), fabsf(d.y)) > 0.4999f) {     // rare: one of the pair is near a half-integer
      if (fabsf(d.x) > 0.4999f) t.x = __fadd_rn(__fdiv_rn(v[2 * i], s), kMagic);
      if (fabsf(d.y) > 0.4999f) t.y = __fadd_rn(__fdiv_rn(v[2 * i + 1], s), kMagic);
    }
    b[2 * i] = __float_as_uint(t.x);
    b[2 * i + 1] = __float_as_uint(t.y);
  }
  return make_uint2(__byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410),
                    __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Store a scale in the requested dtype.
__device__ __forceinline__ void store_scale(void* p, int64_t i, float s, int dtype) {
  if (dtype == OD_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(s);
  else if (dtype == OD_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(s);
  else reinterpret_cast<float*>(p)[i] = s;
}
__device__ __forceinline__ float load_scale(const void* p, int64_t i, int dtype) {
  if (dtype == OD_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == OD_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

}  // namespace od
