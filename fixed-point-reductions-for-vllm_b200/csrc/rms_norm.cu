// Fixed-point RMSNorm (rms_norm.py:10-60), optional fused residual add.
// One CTA per row: 16-byte vector loads of x, the fp32 row (x + residual) is
// kept in shared memory between the integer squared-sum and the scaling
// pass, so x is read from HBM once and y written once.
#include "fxp_common.cuh"

namespace fxpr {

template <typename T> constexpr int x_dtype_of() {
  return std::is_same<T, __nv_bfloat16>::value ? FXPR_BF16
         : (std::is_same<T, __half>::value ? FXPR_F16 : FXPR_F32);
}

template <int BITS, typename XT, int VEC>
__global__ void __launch_bounds__(256) rms_norm_kernel(
    const XT* __restrict__ x, int64_t xs, const void* __restrict__ w, int w_dtype,
    void* __restrict__ y, int y_dtype, int64_t ys, void* __restrict__ res, int res_dtype,
    int64_t rs, int64_t hidden, float eps, int frac) {
  extern __shared__ float row_s[];
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  const int64_t row = blockIdx.x;
  const XT* xr = x + row * xs;
  const float scale = ldexpf(1.0f, frac);
  UAcc acc = 0;

  auto visit = [&](int64_t i, float v) {
    if (res) {
      v = __fadd_rn(v, load_f32(res, res_dtype, row * rs + i));  // rms_norm.py:43
      store_f32(res, res_dtype, row * rs + i, v);                // rms_norm.py:44
    }
    row_s[i] = v;
    acc += (UAcc)f2x_f32<BITS>(__fmul_rn(v, v), scale);         // rms_norm.py:46-51
  };

  if constexpr (VEC > 1) {
    struct alignas(16) V { XT v[VEC]; };
    const V* xv = reinterpret_cast<const V*>(xr);
    const int64_t nv = hidden / VEC;
    for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
      const V t = xv[j];
#pragma unroll
      for (int e = 0; e < VEC; ++e) visit(j * VEC + e, to_f32(t.v[e]));
    }
    for (int64_t i = nv * VEC + threadIdx.x; i < hidden; i += blockDim.x) visit(i, to_f32(xr[i]));
  } else {
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) visit(i, to_f32(xr[i]));
  }

  // exact integer block reduction (wraps like the reference's int32/int64 sum)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ UAcc red[32];
  __shared__ float rrms_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    acc = (lane < (int)(blockDim.x >> 5)) ? red[lane] : (UAcc)0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      // tl.sum of int16 F2X values accumulates in int32 (no 16-bit wrap)
      float sum_f;
      if constexpr (BITS == 64) {
        sum_f = x2f_f32<64>((long long)acc, ldexpf(1.0f, -frac));
      } else {
        sum_f = x2f_f32<32>((int32_t)acc, ldexpf(1.0f, -frac));
      }
      const float mean = fmaxf(prim_div(sum_f, (float)hidden), 0.0f);  // rms_norm.py:56
      rrms_s = prim_div(1.0f, prim_sqrt(__fadd_rn(mean, eps)));       // rms_norm.py:57
    }
  }
  __syncthreads();
  const float rrms = rrms_s;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(row_s[i], load_f32(w, w_dtype, i)), rrms);  // rms_norm.py:59
    store_f32(y, y_dtype, row * ys + i, v);
  }
}

// Register-resident variant for aligned rows of up to THREADS * MAXV * VEC
// elements: every 16-byte load of x (and of the residual) is issued before
// any is consumed, so a CTA keeps the whole row in flight; no shared-memory
// staging of the row.
template <int BITS, typename XT, int MAXV, bool RES>
__global__ void __launch_bounds__(256) rms_norm_vec_kernel(
    const XT* __restrict__ x, int64_t xs, const void* __restrict__ w, int w_dtype,
    void* __restrict__ y, int y_dtype, int64_t ys, XT* __restrict__ res, int64_t rs,
    int64_t hidden, float eps, int frac) {
  constexpr int VEC = 16 / sizeof(XT);
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  struct alignas(16) V { XT v[VEC]; };
  const int64_t row = blockIdx.x;
  const int nv = (int)(hidden / VEC);
  const V* xr = reinterpret_cast<const V*>(x + row * xs);
  V* rr = RES ? reinterpret_cast<V*>(res + row * rs) : nullptr;
  const float scale = ldexpf(1.0f, frac);
  V xv[MAXV], rv[MAXV];
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j < nv) {
      xv[k] = xr[j];
      if (RES) rv[k] = rr[j];
    }
  }
  float xf[MAXV][VEC];
  UAcc acc = 0;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j < nv) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        float v = to_f32(xv[k].v[e]);
        if (RES) {
          v = __fadd_rn(v, to_f32(rv[k].v[e]));  // rms_norm.py:43
          rv[k].v[e] = from_f32<XT>(v);
        }
        xf[k][e] = v;
        acc += (UAcc)f2x_f32<BITS>(__fmul_rn(v, v), scale);  // rms_norm.py:46-51
      }
      if (RES) rr[j] = rv[k];  // rms_norm.py:44
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ UAcc red[8];
  __shared__ float rrms_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    UAcc tot = 0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += red[k];
    float sum_f;
    if constexpr (BITS == 64) {
      sum_f = x2f_f32<64>((long long)tot, ldexpf(1.0f, -frac));
    } else {
      sum_f = x2f_f32<32>((int32_t)tot, ldexpf(1.0f, -frac));  // int16 squares sum in int32
    }
    const float mean = fmaxf(prim_div(sum_f, (float)hidden), 0.0f);  // rms_norm.py:56
    rrms_s = prim_div(1.0f, prim_sqrt(__fadd_rn(mean, eps)));       // rms_norm.py:57
  }
  __syncthreads();
  const float rrms = rrms_s;
  const bool wy_vec = (w_dtype == FXPR_BF16 && y_dtype == FXPR_BF16 && std::is_same<XT, __nv_bfloat16>::value);
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j < nv) {
      if (wy_vec) {
        const V wv = reinterpret_cast<const V*>(w)[j];
        V out;
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          out.v[e] = from_f32<XT>(__fmul_rn(__fmul_rn(xf[k][e], to_f32(wv.v[e])), rrms));  // rms_norm.py:59
        reinterpret_cast<V*>(reinterpret_cast<XT*>(y) + row * ys)[j] = out;
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const int64_t i = (int64_t)j * VEC + e;
          store_f32(y, y_dtype, row * ys + i, __fmul_rn(__fmul_rn(xf[k][e], load_f32(w, w_dtype, i)), rrms));
        }
      }
    }
  }
}

template <int BITS, typename XT>
static int launch_rms(const void* x, int64_t xs, const void* w, int w_dtype, void* y, int y_dtype,
                      int64_t ys, void* res, int res_dtype, int64_t rs, int64_t rows, int64_t hidden,
                      float eps, int frac, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(XT);
  const size_t smem = (size_t)hidden * sizeof(float);
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((xs * (int64_t)sizeof(XT)) % 16 == 0);
  const bool res_ok = !res || (res_dtype == x_dtype_of<XT>() && (uintptr_t)res % 16 == 0 &&
                               (rs * (int64_t)sizeof(XT)) % 16 == 0);
  const bool y_ok = (uintptr_t)y % 16 == 0 && (ys * elem_size(y_dtype)) % 16 == 0 &&
                    (uintptr_t)w % 16 == 0;
  if (aligned && res_ok && y_ok && hidden % VEC == 0 && hidden <= 256 * 4 * VEC) {
    // enough threads for four 16-byte loads each (more rows resident per SM)
    const int nvec = (int)(hidden / VEC);
    const int threads = ((nvec + 4 * 32 - 1) / (4 * 32)) * 32;
    if (res)
      rms_norm_vec_kernel<BITS, XT, 4, true><<<(unsigned)rows, threads, 0, st>>>(
          (const XT*)x, xs, w, w_dtype, y, y_dtype, ys, (XT*)res, rs, hidden, eps, frac);
    else
      rms_norm_vec_kernel<BITS, XT, 4, false><<<(unsigned)rows, threads, 0, st>>>(
          (const XT*)x, xs, w, w_dtype, y, y_dtype, ys, nullptr, 0, hidden, eps, frac);
    return check_launch("fxpr_rms_norm_fxp");
  }
  auto k = aligned ? rms_norm_kernel<BITS, XT, VEC> : rms_norm_kernel<BITS, XT, 1>;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
      set_error("rms_norm_fxp: hidden size %lld too large", (long long)hidden);
      return FXPR_ERR_INVALID;
    }
  }
  k<<<(unsigned)rows, 256, smem, st>>>((const XT*)x, xs, w, w_dtype, y, y_dtype, ys, res, res_dtype,
                                       rs, hidden, eps, frac);
  return check_launch("fxpr_rms_norm_fxp");
}

// ---------------------------------------------------------------------------
// Fused row-parallel epilogue + residual RMSNorm: the raw integer accumulator
// of a row-parallel linear layer (after the integer allreduce) goes through
// X2F + bias and the cast to the activation dtype -- exactly the linear
// method's output -- then the fp32 residual add (written back to residual)
// and the fixed-point RMSNorm of the fp32 sum, in one pass over the row.
// Same bits as fxpr_fixed_to_float_bias followed by fxpr_rms_norm_fxp with a
// residual (quantisation_config.py:181-187, then rms_norm.py:36-59).
// ---------------------------------------------------------------------------
template <int BITS, typename XT>
__global__ void __launch_bounds__(256) x2f_add_rms_norm_kernel(
    const void* __restrict__ acc_in, int64_t as, const void* __restrict__ bias, int bias_dtype,
    XT* __restrict__ res, int64_t rs, const void* __restrict__ w, int w_dtype, XT* __restrict__ y,
    int64_t ys, int64_t hidden, float eps, int frac) {
  extern __shared__ float row_s[];
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  const int64_t row = blockIdx.x;
  const float scale = ldexpf(1.0f, frac), inv = ldexpf(1.0f, -frac);
  UAcc acc = 0;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    float h;
    if constexpr (BITS == 64) {
      h = __fmul_rn(__ll2float_rn(reinterpret_cast<const long long*>(acc_in)[row * as + i]), inv);
    } else {
      int32_t a = reinterpret_cast<const int32_t*>(acc_in)[row * as + i];
      if (BITS == 16) a = (int16_t)(a & 0xFFFF);
      h = __fmul_rn(__int2float_rn(a), inv);
    }
    if (bias) h = __fadd_rn(h, load_f32(bias, bias_dtype, i));
    const float x = to_f32(from_f32<XT>(h));                  // the linear layer's output dtype
    const float v = __fadd_rn(x, to_f32(res[row * rs + i]));  // rms_norm.py:43
    res[row * rs + i] = from_f32<XT>(v);                      // rms_norm.py:44
    row_s[i] = v;
    acc += (UAcc)f2x_f32<BITS>(__fmul_rn(v, v), scale);       // rms_norm.py:46-51
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ UAcc red[8];
  __shared__ float rrms_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    UAcc tot = 0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += red[k];
    float sum_f;
    if constexpr (BITS == 64) {
      sum_f = x2f_f32<64>((long long)tot, inv);
    } else {
      sum_f = x2f_f32<32>((int32_t)tot, inv);  // int16 squares sum in int32
    }
    const float mean = fmaxf(prim_div(sum_f, (float)hidden), 0.0f);  // rms_norm.py:56
    rrms_s = prim_div(1.0f, prim_sqrt(__fadd_rn(mean, eps)));       // rms_norm.py:57
  }
  __syncthreads();
  const float rrms = rrms_s;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x)
    y[row * ys + i] = from_f32<XT>(__fmul_rn(__fmul_rn(row_s[i], load_f32(w, w_dtype, i)), rrms));  // rms_norm.py:59
}

template <int BITS, typename XT>
static int launch_x2f_rms(const void* acc, int64_t as, const void* bias, int bias_dtype, void* res,
                          int64_t rs, const void* w, int w_dtype, void* y, int64_t ys, int64_t rows,
                          int64_t hidden, float eps, int frac, cudaStream_t st) {
  auto k = x2f_add_rms_norm_kernel<BITS, XT>;
  const size_t smem = (size_t)hidden * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    set_error("fixed_to_float_add_rms_norm: hidden size %lld too large", (long long)hidden);
    return FXPR_ERR_INVALID;
  }
  k<<<(unsigned)rows, 256, smem, st>>>(acc, as, bias, bias_dtype, (XT*)res, rs, w, w_dtype, (XT*)y,
                                       ys, hidden, eps, frac);
  return check_launch("fxpr_fixed_to_float_add_rms_norm");
}

template <int BITS>
static int dispatch_x2f_rms(const void* acc, int64_t as, const void* bias, int bias_dtype, void* res,
                            int act_dtype, int64_t rs, const void* w, int w_dtype, void* y, int64_t ys,
                            int64_t rows, int64_t hidden, float eps, int frac, cudaStream_t st) {
  switch (act_dtype) {
    case FXPR_BF16:
      return launch_x2f_rms<BITS, __nv_bfloat16>(acc, as, bias, bias_dtype, res, rs, w, w_dtype, y,
                                                 ys, rows, hidden, eps, frac, st);
    case FXPR_F16:
      return launch_x2f_rms<BITS, __half>(acc, as, bias, bias_dtype, res, rs, w, w_dtype, y, ys,
                                          rows, hidden, eps, frac, st);
    default:
      return launch_x2f_rms<BITS, float>(acc, as, bias, bias_dtype, res, rs, w, w_dtype, y, ys, rows,
                                         hidden, eps, frac, st);
  }
}

template <int BITS>
static int dispatch_rms(const void* x, int x_dtype, int64_t xs, const void* w, int w_dtype, void* y,
                        int y_dtype, int64_t ys, void* res, int res_dtype, int64_t rs, int64_t rows,
                        int64_t hidden, float eps, int frac, cudaStream_t st) {
  switch (x_dtype) {
    case FXPR_BF16:
      return launch_rms<BITS, __nv_bfloat16>(x, xs, w, w_dtype, y, y_dtype, ys, res, res_dtype, rs,
                                             rows, hidden, eps, frac, st);
    case FXPR_F16:
      return launch_rms<BITS, __half>(x, xs, w, w_dtype, y, y_dtype, ys, res, res_dtype, rs, rows,
                                      hidden, eps, frac, st);
    default:
      return launch_rms<BITS, float>(x, xs, w, w_dtype, y, y_dtype, ys, res, res_dtype, rs, rows,
                                     hidden, eps, frac, st);
  }
}

}  // namespace fxpr

using namespace fxpr;

extern "C" int fxpr_rms_norm_fxp(const void* x, int x_dtype, int64_t x_row_stride, const void* w,
                                 int w_dtype, void* y, int y_dtype, int64_t y_row_stride,
                                 void* residual, int res_dtype, int64_t res_row_stride, int64_t rows,
                                 int64_t hidden, float eps, int frac_bits, int int_bits,
                                 void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  auto ok_f = [](int d) { return d == FXPR_F16 || d == FXPR_BF16 || d == FXPR_F32; };
  if (!ok_f(x_dtype) || !ok_f(w_dtype) || !ok_f(y_dtype) || (residual && !ok_f(res_dtype))) {
    set_error("rms_norm_fxp: tensors must be float16/bfloat16/float32");
    return FXPR_ERR_INVALID;
  }
  if (rows <= 0 || hidden <= 0) return FXPR_OK;
  if (rows > 0x7fffffffLL || hidden * 4 > 200 * 1024) {
    set_error("rms_norm_fxp: shape too large (rows < 2^31, hidden <= 51200)");
    return FXPR_ERR_INVALID;
  }
  const cudaStream_t st = (cudaStream_t)stream;
  if (int_bits == 16)
    return dispatch_rms<16>(x, x_dtype, x_row_stride, w, w_dtype, y, y_dtype, y_row_stride, residual,
                            res_dtype, res_row_stride, rows, hidden, eps, frac_bits, st);
  if (int_bits == 32)
    return dispatch_rms<32>(x, x_dtype, x_row_stride, w, w_dtype, y, y_dtype, y_row_stride, residual,
                            res_dtype, res_row_stride, rows, hidden, eps, frac_bits, st);
  return dispatch_rms<64>(x, x_dtype, x_row_stride, w, w_dtype, y, y_dtype, y_row_stride, residual,
                          res_dtype, res_row_stride, rows, hidden, eps, frac_bits, st);
}

extern "C" int fxpr_fixed_to_float_add_rms_norm(const void* acc, int int_bits, int64_t acc_row_stride,
                                                const void* bias, int bias_dtype, void* residual,
                                                int act_dtype, int64_t res_row_stride, const void* w,
                                                int w_dtype, void* y, int64_t y_row_stride,
                                                int64_t rows, int64_t hidden, float eps,
                                                int frac_bits, void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  auto ok_f = [](int d) { return d == FXPR_F16 || d == FXPR_BF16 || d == FXPR_F32; };
  if (!ok_f(act_dtype) || !ok_f(w_dtype) || (bias && !ok_f(bias_dtype))) {
    set_error("fixed_to_float_add_rms_norm: activations, weight and bias must be float16/bfloat16/float32");
    return FXPR_ERR_UNSUPPORTED;
  }
  if (!residual || !acc || !y || !w) {
    set_error("fixed_to_float_add_rms_norm: null pointer");
    return FXPR_ERR_INVALID;
  }
  if (rows <= 0 || hidden <= 0) return FXPR_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  if (int_bits == 16)
    return dispatch_x2f_rms<16>(acc, acc_row_stride, bias, bias_dtype, residual, act_dtype,
                                res_row_stride, w, w_dtype, y, y_row_stride, rows, hidden, eps,
                                frac_bits, st);
  if (int_bits == 32)
    return dispatch_x2f_rms<32>(acc, acc_row_stride, bias, bias_dtype, residual, act_dtype,
                                res_row_stride, w, w_dtype, y, y_row_stride, rows, hidden, eps,
                                frac_bits, st);
  return dispatch_x2f_rms<64>(acc, acc_row_stride, bias, bias_dtype, residual, act_dtype,
                              res_row_stride, w, w_dtype, y, y_row_stride, rows, hidden, eps,
                              frac_bits, st);
}
