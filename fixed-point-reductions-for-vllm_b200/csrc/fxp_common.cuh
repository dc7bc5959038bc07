// Shared device helpers of the FxPR B200 kernels: dtype loads/stores, the
// Q-format casts (F2X / X2F) with the reference's exact semantics, the
// "magic constant" round-to-nearest-even fast path, and the fp32 primitives
// whose rounding the reference leaves to the GPU compiler.
//
// Build with --fmad=false: every multiply-add below is spelled out, so the
// compiler may not contract separate roundings of the reference into FMAs.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/fxpr_b200.h"

namespace fxpr {

// ---------------------------------------------------------------------------
// error reporting (host)
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int check_launch(const char* what);
int num_sms();  // SM count of the current device (cached per device)

// ---------------------------------------------------------------------------
// loads / stores of the supported element types as fp32
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// runtime-dtype load of element i as fp32 (F16/BF16/F32; F64 rounded RN)
__device__ __forceinline__ float load_f32(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case FXPR_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case FXPR_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case FXPR_F64: return __double2float_rn(reinterpret_cast<const double*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

__device__ __forceinline__ void store_f32(void* p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case FXPR_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case FXPR_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case FXPR_F64: reinterpret_cast<double*>(p)[i] = (double)v; break;
    default: reinterpret_cast<float*>(p)[i] = v;
  }
}

// ---------------------------------------------------------------------------
// Q-format constants (fixed_point.py:41-48)
// ---------------------------------------------------------------------------
// mant = mantissa bits + 1 of the input float type: fp16 11, fp32 24, fp64 53
__host__ __device__ constexpr int safe_shift(int bits, int mant) {
  return bits <= mant ? 0 : bits - mant;
}
__host__ __device__ inline double qmax_of(int bits, int mant) {
  return ldexp(1.0, bits - 1) - ldexp(1.0, safe_shift(bits, mant));
}
__host__ __device__ inline double qmin_of(int bits) { return -ldexp(1.0, bits - 1); }

// fp32 clamp bounds for accumulator width BITS
template <int BITS> struct F32Bounds;
template <> struct F32Bounds<16> {
  static constexpr float qmin = -32768.0f, qmax = 32767.0f;
};
template <> struct F32Bounds<32> {
  static constexpr float qmin = -2147483648.0f, qmax = 2147483392.0f;  // 2^31 - 2^8
};
template <> struct F32Bounds<64> {
  static constexpr float qmin = -9223372036854775808.0f;
  static constexpr float qmax = 9223370937343148032.0f;  // 2^63 - 2^40
};

// Accumulator register type: int16 accumulation is carried in int32 (the low
// 16 bits of a mod-2^32 sum equal the mod-2^16 sum).
template <int BITS> struct Acc { using T = int32_t; };
template <> struct Acc<64> { using T = long long; };

// F2X of an already-scaled fp32 value: maxnum/minnum clamp (NaN -> qmin),
// RNE conversion (fixed_point.py:50-53).
template <int BITS>
__device__ __forceinline__ typename Acc<BITS>::T f2x_scaled(float s) {
  const float c = fminf(fmaxf(s, F32Bounds<BITS>::qmin), F32Bounds<BITS>::qmax);
  if constexpr (BITS == 64) {
    return __float2ll_rn(c);
  } else {
    return __float2int_rn(c);
  }
}

// F2X of an fp32 value (fixed_point.py:48-53); `scale` = 2^f as fp32.
template <int BITS>
__device__ __forceinline__ typename Acc<BITS>::T f2x_f32(float x, float scale) {
  return f2x_scaled<BITS>(__fmul_rn(x, scale));
}

// Wrap an accumulator to its reference width (int16: sign-extend low 16 bits)
template <int BITS>
__device__ __forceinline__ typename Acc<BITS>::T wrap_acc(typename Acc<BITS>::T v) {
  if constexpr (BITS == 16) {
    return (int32_t)(int16_t)(v & 0xFFFF);
  } else {
    return v;
  }
}

// X2F into fp32 (fixed_point.py:68-69): RNE int->float, times 2^-f
template <int BITS>
__device__ __forceinline__ float x2f_f32(typename Acc<BITS>::T v, float inv_scale) {
  if constexpr (BITS == 64) {
    return __fmul_rn(__ll2float_rn(v), inv_scale);
  } else {
    return __fmul_rn(__int2float_rn(v), inv_scale);
  }
}

// ---------------------------------------------------------------------------
// "Magic constant" round-to-nearest-even.
// For an fp32 value |v| <= 2^22, C + v with C = 1.5 * 2^23 lands in
// [2^23, 2^24] where the fp32 spacing is 1, so the single RN rounding of the
// add is RNE(v) (C is even, so ties resolve with v's own parity), and
// bits(C + v) - bits(C) == RNE(v) as an integer. With an exact product
// (bf16/fp16 operands) fmaf(a, b, C) rounds a*b directly.
// ---------------------------------------------------------------------------
constexpr float kMagic = 12582912.0f;       // 1.5 * 2^23
constexpr int32_t kMagicBits = 0x4B400000;  // bits of kMagic

// ---------------------------------------------------------------------------
// fp32 primitives the reference leaves to the compiler. Triton 3.6 lowers
// `tl.math.exp2` to the hardware base-2 exponential, `/` to its fast divide
// and `tl.sqrt` to its fast square root (documented as "fast" ops in
// triton/language/math.py); these wrappers issue the corresponding documented
// PTX instructions. The GPU tests pin each against Triton on the same device.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float prim_exp2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float prim_div(float a, float b) {
  float y;
  asm("div.full.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
  return y;
}
__device__ __forceinline__ float prim_sqrt(float x) {
  float y;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float prim_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ float prim_exp(float x) { return __expf(x); }
__device__ __forceinline__ float prim_log(float x) { return logf(x); }

// ---------------------------------------------------------------------------
// packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction, two lanes)
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
  return *reinterpret_cast<unsigned long long*>(&v);
}
__device__ __forceinline__ float2 bits_f2(unsigned long long v) {
  return *reinterpret_cast<float2*>(&v);
}
#ifndef FXPR_ASM_F32X2
// compiler builtins for the packed ops (correctly rounded, never contracted),
// so register pairs are allocated by the compiler rather than through
// 64-bit asm operands
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
#else
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
#endif
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}

// ---------------------------------------------------------------------------
// async copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes));
}
// same, with an L2 prefetch of the surrounding 256-byte segment
__device__ __forceinline__ void cp_async16_l2pf(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// |x| < 2^E from the maximum absolute fp32 bit pattern of a set of values
// (for non-negative floats the integer order of the patterns is the numeric
// order, so an integer max gives the exact max magnitude); 1000 for inf/NaN.
__device__ __forceinline__ int exp_bound_f32(uint32_t m) {
  const int e = (m >> 23) & 0xFF;
  return e == 0xFF ? 1000 : (e == 0 ? -126 : e - 126);
}

// max |x| over the elements packed in a 32-bit word, as an fp32 bit pattern
// with the same power-of-two bound
template <typename T> __device__ __forceinline__ uint32_t abs_max_as_f32(uint32_t w);
template <> __device__ __forceinline__ uint32_t abs_max_as_f32<float>(uint32_t w) {
  return w & 0x7FFFFFFFu;
}
template <> __device__ __forceinline__ uint32_t abs_max_as_f32<__nv_bfloat16>(uint32_t w) {
  return max(w & 0x7FFFu, (w >> 16) & 0x7FFFu) << 16;
}
template <> __device__ __forceinline__ uint32_t abs_max_as_f32<__half>(uint32_t w) {
  const uint32_t h = max(w & 0x7FFFu, (w >> 16) & 0x7FFFu);
  const uint32_t e = (h >> 10) & 0x1F;
  if (e == 0x1F) return 0x7F800000u;
  if (e == 0) return h ? (uint32_t)(127 - 14) << 23 : 0u;  // subnormal: < 2^-14
  return ((e - 15 + 127) << 23) | 0x7FFFFFu;
}

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool valid_bits(int b) { return b == 16 || b == 32 || b == 64; }
inline bool is_float_dtype(int d) {
  return d == FXPR_F16 || d == FXPR_BF16 || d == FXPR_F32 || d == FXPR_F64;
}
inline int elem_size(int d) {
  switch (d) {
    case FXPR_F16: case FXPR_BF16: case FXPR_I16: return 2;
    case FXPR_F32: case FXPR_I32: return 4;
    case FXPR_F64: case FXPR_I64: return 8;
  }
  return 0;
}

}  // namespace fxpr
