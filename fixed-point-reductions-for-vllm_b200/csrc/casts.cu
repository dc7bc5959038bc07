// Elementwise Q-format casts, the fixed-point row sum, the row-parallel
// linear epilogue, the fixed-point log-softmax and the primitive probe.
// All HBM-bound and simple: grid-stride loops / one CTA per row.
#include "fxp_common.cuh"

namespace fxpr {

// ---------------------------------------------------------------------------
// F2X for every input float type (fixed_point.py:25-53). The scale and the
// clamp constants are converted to the input's own type, as Triton does with
// the Python constants; the final conversion saturates (PTX cvt), which only
// matters for fp16 where the clamp constants overflow to inf.
// ---------------------------------------------------------------------------
template <int BITS>
__device__ __forceinline__ long long f2x_any(const void* p, int dtype, int64_t i, int frac) {
  if (dtype == FXPR_F64) {
    const double x = reinterpret_cast<const double*>(p)[i];
    const double s = __dmul_rn(x, ldexp(1.0, frac));
    // the clamp constants are fp32 values (Triton materialises Python floats
    // as fp32); out-of-range results saturate in the conversion
    const double c = fmin(fmax(s, (double)(float)qmin_of(BITS)), (double)(float)qmax_of(BITS, 53));
    if (BITS == 64) return __double2ll_rn(c);
    return __double2int_rn(c);
  }
  if (dtype == FXPR_F16) {
    const __half x = reinterpret_cast<const __half*>(p)[i];
    const __half s = __hmul(x, __float2half_rn(ldexpf(1.0f, frac)));
    const __half c = __hmin(__hmax(s, __float2half_rn((float)qmin_of(BITS))),
                            __float2half_rn((float)qmax_of(BITS, 11)));
    if (BITS == 64) return __half2ll_rn(c);
    if (BITS == 16) return __half2short_rn(c);
    return __half2int_rn(c);
  }
  const float x = (dtype == FXPR_BF16)
                      ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                      : reinterpret_cast<const float*>(p)[i];
  return (long long)f2x_f32<BITS>(x, ldexpf(1.0f, frac));
}

template <int BITS>
__global__ void f2x_kernel(const void* __restrict__ x, int dtype, void* __restrict__ q, int64_t n,
                           int frac) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const long long v = f2x_any<BITS>(x, dtype, i, frac);
    if (BITS == 16) reinterpret_cast<int16_t*>(q)[i] = (int16_t)v;
    else if (BITS == 32) reinterpret_cast<int32_t*>(q)[i] = (int32_t)v;
    else reinterpret_cast<long long*>(q)[i] = v;
  }
}

__device__ __forceinline__ long long load_int(const void* p, int bits, int64_t i) {
  if (bits == 16) return reinterpret_cast<const int16_t*>(p)[i];
  if (bits == 32) return reinterpret_cast<const int32_t*>(p)[i];
  return reinterpret_cast<const long long*>(p)[i];
}

__global__ void x2f_kernel(const void* __restrict__ q, int bits, void* __restrict__ y, int dtype,
                           int64_t n, int frac) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const long long v = load_int(q, bits, i);
    if (dtype == FXPR_F64) {
      reinterpret_cast<double*>(y)[i] = __dmul_rn(__ll2double_rn(v), ldexp(1.0, -frac));
    } else if (dtype == FXPR_F16) {
      const __half h = (bits == 64) ? __ll2half_rn(v) : __int2half_rn((int)v);
      reinterpret_cast<__half*>(y)[i] = __hmul(h, __double2half(ldexp(1.0, -frac)));
    } else {
      const float f = (bits == 64) ? __ll2float_rn(v) : __int2float_rn((int)v);
      reinterpret_cast<float*>(y)[i] = __fmul_rn(f, ldexpf(1.0f, -frac));
    }
  }
}

static int grid_for(int64_t n, int threads) {
  int64_t g = cdiv(n, threads);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

// ---------------------------------------------------------------------------
// fixed-point row sum (tests/test_sum.py:13-29): F2X per element in int_b,
// exact int64 sum, saturating clamp to the int_b range, X2F to fp32.
// ---------------------------------------------------------------------------
template <int BITS, int VEC, typename T>
__global__ void __launch_bounds__(256) fxp_sum_kernel(const T* __restrict__ x, int64_t cols,
                                                      int64_t stride, float* __restrict__ out,
                                                      int frac, int dtype) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * stride;
  long long acc = 0;
  if constexpr (VEC > 1) {
    struct alignas(16) V { T v[VEC]; };
    const V* xv = reinterpret_cast<const V*>(xr);
    const int64_t nv = cols / VEC;
    int64_t i = threadIdx.x;
    // four 16-byte loads in flight per thread before any is consumed
    for (; i + 3 * (int64_t)blockDim.x < nv; i += 4 * (int64_t)blockDim.x) {
      V t[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) t[k] = xv[i + k * blockDim.x];
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc += f2x_any<BITS>(t[k].v, dtype, e, frac);
    }
    for (; i < nv; i += blockDim.x) {
      const V t = xv[i];
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc += f2x_any<BITS>(t.v, dtype, e, frac);
    }
    for (int64_t i = nv * VEC + threadIdx.x; i < cols; i += blockDim.x)
      acc += f2x_any<BITS>(xr, dtype, i, frac);
  } else {
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) acc += f2x_any<BITS>(xr, dtype, i, frac);
  }
  // integer block reduction (exact, order-free)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ long long red[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    acc = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      if (BITS < 64) {
        const long long hi = (1LL << (BITS - 1)) - 1, lo = -(1LL << (BITS - 1));
        acc = acc > hi ? hi : (acc < lo ? lo : acc);
      }
      out[row] = __fmul_rn(__ll2float_rn(acc), ldexpf(1.0f, -frac));
    }
  }
}

// Vectorised bf16 / fp32 variant: one warp per row (grid-stride over rows),
// 16-byte loads eight deep per lane, F2X by the magic-constant rounding (two
// elements per packed FMA; x * 2^f is exact, so one rounding = RNE), integer
// sums of the bit patterns, warp-shuffle reduction. A lane whose elements all
// satisfy |x| * 2^f < 2^22 (int16: < 32767.5, inside the clamp range) is
// exact on the fast path; a lane with a larger, inf or NaN element recomputes
// its own elements with the clamp-and-convert path. Same bits either way.
template <int BITS, typename T>
__global__ void __launch_bounds__(256) fxp_sum_magic_kernel(const T* __restrict__ x, int64_t rows,
                                                            int64_t cols, int64_t stride,
                                                            float* __restrict__ out, int frac,
                                                            float thr) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int DEPTH = 8;  // 16-byte loads in flight per lane
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const float scale = ldexpf(1.0f, frac);
  const float2 S2 = make_float2(scale, scale), C2 = make_float2(kMagic, kMagic);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const T* xr = x + row * stride;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    const int64_t nv = cols / VEC;
    long long acc = 0;
    uint32_t m_u = 0, m_s = 0x80008000u;  // |x| bound of 16-bit elements (raw halves)
    uint32_t m32 = 0;                     // |x| bound of fp32 elements (bit patterns)
    auto take = [&](uint4 w) {
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      uint32_t part = 0;
      if constexpr (sizeof(T) == 2) {
        m_u = __vimax3_u16x2(m_u, w.x, w.y);
        m_u = __vimax3_u16x2(m_u, w.z, w.w);
        m_s = (uint32_t)__vimax3_s16x2((int)m_s, (int)w.x, (int)w.y);
        m_s = (uint32_t)__vimax3_s16x2((int)m_s, (int)w.z, (int)w.w);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = make_float2(__uint_as_float(ws[k] << 16), __uint_as_float(ws[k] & 0xFFFF0000u));
          const float2 r = fma2(f, S2, C2);
          part += __float_as_uint(r.x) + __float_as_uint(r.y);
        }
        part -= (uint32_t)8 * (uint32_t)kMagicBits;
      } else {
        m32 = max(max(m32, ws[0] & 0x7FFFFFFFu), ws[1] & 0x7FFFFFFFu);
        m32 = max(max(m32, ws[2] & 0x7FFFFFFFu), ws[3] & 0x7FFFFFFFu);
#pragma unroll
        for (int k = 0; k < 4; k += 2) {
          const float2 r = fma2(make_float2(__uint_as_float(ws[k]), __uint_as_float(ws[k + 1])), S2, C2);
          part += __float_as_uint(r.x) + __float_as_uint(r.y);
        }
        part -= (uint32_t)4 * (uint32_t)kMagicBits;
      }
      acc += (long long)(int32_t)part;  // |part| <= 8 * 2^22
    };
    int64_t i = lane;
    for (; i + (DEPTH - 1) * 32 < nv; i += DEPTH * 32) {
      uint4 t[DEPTH];
#pragma unroll
      for (int k = 0; k < DEPTH; ++k) t[k] = __ldcs(xv + i + k * 32);
#pragma unroll
      for (int k = 0; k < DEPTH; ++k) take(t[k]);
    }
    for (; i < nv; i += 32) take(__ldcs(xv + i));
    float mx;
    if constexpr (sizeof(T) == 2) {
      const uint32_t pk = __vmaxu2(m_u & 0x7FFF7FFFu, m_s & 0x7FFF7FFFu);
      mx = __uint_as_float(max(pk & 0xFFFFu, pk >> 16) << 16);
    } else {
      mx = __uint_as_float(m32);
    }
    if (!(mx < thr)) {  // this lane's vectors again, each element clamped alone
      acc = 0;
      for (int64_t v = lane; v < nv; v += 32)
        for (int e = 0; e < VEC; ++e) acc += (long long)f2x_f32<BITS>(to_f32(xr[v * VEC + e]), scale);
    }
    for (int64_t k = nv * VEC + lane; k < cols; k += 32)
      acc += (long long)f2x_f32<BITS>(to_f32(xr[k]), scale);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      if (BITS < 64) {
        const long long hi = (1LL << (BITS - 1)) - 1, lo = -(1LL << (BITS - 1));
        acc = acc > hi ? hi : (acc < lo ? lo : acc);
      }
      out[row] = __fmul_rn(__ll2float_rn(acc), ldexpf(1.0f, -frac));
    }
  }
}

template <int BITS>
static int launch_fxp_sum(const void* x, int dtype, int64_t rows, int64_t cols, int64_t stride,
                          float* out, int frac, cudaStream_t st) {
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((stride * elem_size(dtype)) % 16 == 0);
  // about four 16-byte loads per thread: short rows get small CTAs, so that
  // many rows are resident per SM
  const int64_t nvec = cols * elem_size(dtype) / 16;
  int threads = (int)(((nvec + 4 * 32 - 1) / (4 * 32)) * 32);
  threads = threads < 64 ? 64 : (threads > 256 ? 256 : threads);
  const dim3 grid((unsigned)rows), block(threads);
  // |x| bound of the magic-constant path: |x| * 2^f below 2^22 (int16: inside
  // the clamp range), as an fp32 threshold on |x|
  const float thr = (float)ldexp(BITS == 16 ? 32767.5 : 4194304.0, -frac);
  if (aligned && frac <= 100 && (dtype == FXPR_BF16 || dtype == FXPR_F32)) {
    // 8 rows (warps) per CTA, at most 16 CTAs per SM's worth of rows in one wave
    int64_t g = cdiv(rows, 8);
    const int64_t cap = (int64_t)num_sms() * 8;
    if (g > cap) g = cap;
    if (dtype == FXPR_BF16)
      fxp_sum_magic_kernel<BITS, __nv_bfloat16><<<(unsigned)g, 256, 0, st>>>(
          (const __nv_bfloat16*)x, rows, cols, stride, out, frac, thr);
    else
      fxp_sum_magic_kernel<BITS, float><<<(unsigned)g, 256, 0, st>>>((const float*)x, rows, cols,
                                                                      stride, out, frac, thr);
    return check_launch("fxpr_fxp_sum");
  }
  switch (dtype) {
    case FXPR_BF16:
      if (aligned)
        fxp_sum_kernel<BITS, 8><<<grid, block, 0, st>>>((const __nv_bfloat16*)x, cols, stride, out, frac, dtype);
      else
        fxp_sum_kernel<BITS, 1><<<grid, block, 0, st>>>((const __nv_bfloat16*)x, cols, stride, out, frac, dtype);
      break;
    case FXPR_F16:
      if (aligned)
        fxp_sum_kernel<BITS, 8><<<grid, block, 0, st>>>((const __half*)x, cols, stride, out, frac, dtype);
      else
        fxp_sum_kernel<BITS, 1><<<grid, block, 0, st>>>((const __half*)x, cols, stride, out, frac, dtype);
      break;
    case FXPR_F32:
      if (aligned)
        fxp_sum_kernel<BITS, 4><<<grid, block, 0, st>>>((const float*)x, cols, stride, out, frac, dtype);
      else
        fxp_sum_kernel<BITS, 1><<<grid, block, 0, st>>>((const float*)x, cols, stride, out, frac, dtype);
      break;
    default:
      fxp_sum_kernel<BITS, 1><<<grid, block, 0, st>>>((const double*)x, cols, stride, out, frac, dtype);
  }
  return check_launch("fxpr_fxp_sum");
}

// ---------------------------------------------------------------------------
// row-parallel linear epilogue: out = cast(X2F(acc) + fp32(bias))
// (quantisation_config.py:181-187)
// ---------------------------------------------------------------------------
__global__ void x2f_bias_kernel(const void* __restrict__ acc, int bits, int64_t M, int64_t N,
                                int64_t acc_stride, const void* __restrict__ bias, int bias_dtype,
                                void* __restrict__ out, int out_dtype, int64_t out_stride,
                                int frac) {
  const int64_t total = M * N;
  const float inv = ldexpf(1.0f, -frac);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float v;
    if (bits == 64) {
      v = __fmul_rn(__ll2float_rn(reinterpret_cast<const long long*>(acc)[m * acc_stride + n]), inv);
    } else {
      int32_t a = reinterpret_cast<const int32_t*>(acc)[m * acc_stride + n];
      if (bits == 16) a = (int16_t)(a & 0xFFFF);
      v = __fmul_rn(__int2float_rn(a), inv);
    }
    if (bias) v = __fadd_rn(v, load_f32(bias, bias_dtype, n));
    store_f32(out, out_dtype, m * out_stride + n, v);
  }
}

// ---------------------------------------------------------------------------
// log-softmax with a fixed-point exp-sum (softmax.py:8-52): logits rounded to
// fp16 before the max and the exp, exp-sum as an integer, log of its X2F.
// ---------------------------------------------------------------------------
template <int BITS>
__global__ void __launch_bounds__(256) log_softmax_kernel(const float* __restrict__ x,
                                                          int64_t xs, float* __restrict__ y,
                                                          int64_t ys, int64_t n, int frac) {
  const int64_t row = blockIdx.x;
  const float* xr = x + row * xs;
  float* yr = y + row * ys;
  __shared__ float redf[32];
  __shared__ unsigned long long redi[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
    m = fmaxf(m, __half2float(__float2half_rn(xr[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) redf[warp] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < nw; ++w) m = fmaxf(m, redf[w]);
  const float scale = ldexpf(1.0f, frac);
  unsigned long long acc = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = prim_exp(__fsub_rn(__half2float(__float2half_rn(xr[i])), m));
    acc += (unsigned long long)(long long)f2x_f32<BITS>(e, scale);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) redi[warp] = acc;
  __syncthreads();
  acc = 0;
  for (int w = 0; w < nw; ++w) acc += redi[w];
  const float sum_f = (BITS == 64) ? __ll2float_rn((long long)acc)
                                   : __int2float_rn((int32_t)(uint32_t)acc);  // int32 wrap
  const float ls = prim_log(__fmul_rn(sum_f, ldexpf(1.0f, -frac)));
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __half2float(__float2half_rn(xr[i]));
    yr[i] = __fsub_rn(__fsub_rn(v, m), ls);
  }
}

// ---------------------------------------------------------------------------
// primitive probe (test hook)
// ---------------------------------------------------------------------------
__global__ void probe_kernel(int op, const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = a[i];
    float r;
    switch (op) {
      case 0: r = prim_exp2(x); break;
      case 1: r = prim_div(x, b[i]); break;
      case 2: r = prim_sqrt(x); break;
      case 3: r = prim_tanh(x); break;
      case 4: r = prim_exp(x); break;
      default: r = prim_log(x); break;
    }
    out[i] = r;
  }
}

}  // namespace fxpr

using namespace fxpr;

extern "C" int fxpr_float_to_fixed(const void* x, int x_dtype, void* q, int int_bits, int64_t n,
                                   int frac_bits, void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  if (x_dtype != FXPR_F16 && x_dtype != FXPR_F32 && x_dtype != FXPR_F64) {
    set_error("float_to_fixed: x must be float16/float32/float64");
    return FXPR_ERR_INVALID;
  }
  if (frac_bits < 0 || frac_bits >= 127) {
    set_error("float_to_fixed: frac_bits out of range: %d", frac_bits);
    return FXPR_ERR_INVALID;
  }
  if (n <= 0) return FXPR_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  const int g = grid_for(n, 256);
  if (int_bits == 16) f2x_kernel<16><<<g, 256, 0, st>>>(x, x_dtype, q, n, frac_bits);
  else if (int_bits == 32) f2x_kernel<32><<<g, 256, 0, st>>>(x, x_dtype, q, n, frac_bits);
  else f2x_kernel<64><<<g, 256, 0, st>>>(x, x_dtype, q, n, frac_bits);
  return check_launch("fxpr_float_to_fixed");
}

extern "C" int fxpr_fixed_to_float(const void* q, int int_bits, void* y, int y_dtype, int64_t n,
                                   int frac_bits, void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  if (y_dtype != FXPR_F16 && y_dtype != FXPR_F32 && y_dtype != FXPR_F64) {
    set_error("fixed_to_float: output must be float16/float32/float64");
    return FXPR_ERR_INVALID;
  }
  if (n <= 0) return FXPR_OK;
  x2f_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(q, int_bits, y, y_dtype, n,
                                                                 frac_bits);
  return check_launch("fxpr_fixed_to_float");
}

extern "C" int fxpr_fxp_sum(const void* x, int x_dtype, int64_t rows, int64_t cols,
                            int64_t row_stride, float* out, int frac_bits, int int_bits,
                            void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  if (!is_float_dtype(x_dtype)) {
    set_error("fxp_sum: x must be a float tensor");
    return FXPR_ERR_INVALID;
  }
  if (rows <= 0) return FXPR_OK;
  if (rows > 0x7fffffffLL) {
    set_error("fxp_sum: too many rows");
    return FXPR_ERR_INVALID;
  }
  const cudaStream_t st = (cudaStream_t)stream;
  if (int_bits == 16) return launch_fxp_sum<16>(x, x_dtype, rows, cols, row_stride, out, frac_bits, st);
  if (int_bits == 32) return launch_fxp_sum<32>(x, x_dtype, rows, cols, row_stride, out, frac_bits, st);
  return launch_fxp_sum<64>(x, x_dtype, rows, cols, row_stride, out, frac_bits, st);
}

extern "C" int fxpr_fixed_to_float_bias(const void* acc, int int_bits, int64_t M, int64_t N,
                                        int64_t acc_row_stride, const void* bias, int bias_dtype,
                                        void* out, int out_dtype, int64_t out_row_stride,
                                        int frac_bits, void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  if (M * N <= 0) return FXPR_OK;
  x2f_bias_kernel<<<grid_for(M * N, 256), 256, 0, (cudaStream_t)stream>>>(
      acc, int_bits, M, N, acc_row_stride, bias, bias_dtype, out, out_dtype, out_row_stride,
      frac_bits);
  return check_launch("fxpr_fixed_to_float_bias");
}

extern "C" int fxpr_log_softmax_fxp(const float* x, int64_t xs, float* y, int64_t ys, int64_t rows,
                                    int64_t n, int frac_bits, int int_bits, void* stream) {
  if (int_bits != 32 && int_bits != 64) {
    set_error("log_softmax_fxp supports 32/64-bit accumulators, got %d", int_bits);
    return int_bits == 16 ? FXPR_ERR_UNSUPPORTED : FXPR_ERR_INVALID;
  }
  if (rows <= 0) return FXPR_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  if (int_bits == 32) log_softmax_kernel<32><<<(unsigned)rows, 256, 0, st>>>(x, xs, y, ys, n, frac_bits);
  else log_softmax_kernel<64><<<(unsigned)rows, 256, 0, st>>>(x, xs, y, ys, n, frac_bits);
  return check_launch("fxpr_log_softmax_fxp");
}

extern "C" int fxpr_probe_prims(int op, const float* a, const float* b, float* out, int64_t n,
                                void* stream) {
  if (n <= 0) return FXPR_OK;
  probe_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(op, a, b, out, n);
  return check_launch("fxpr_probe_prims");
}
