// Shared pieces of the paged attention kernels: launch parameters, 16-byte
// chunk unpacking and the magnitude guards of the magic-constant fast path.
#pragma once

#include "fxp_common.cuh"

namespace fxpr {
namespace attn {

constexpr int THREADS = 256;
constexpr int KT = 64;    // keys per tile
#ifndef FXPR_ATTN_NBUF
#define FXPR_ATTN_NBUF 3
#endif
constexpr int NBUF = FXPR_ATTN_NBUF;  // K/V tile buffers (NBUF - 1 tiles in flight)
constexpr int MAX_SPLITS = 8;
#ifndef FXPR_ATTN_CHUNK
#define FXPR_ATTN_CHUNK 512
#endif
constexpr int CHUNK = FXPR_ATTN_CHUNK;  // keys per work unit of the chunked path

struct Params {
  const void* q;
  int q_dtype;
  int64_t q_st, q_sh;
  const void* k;
  const void* v;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  void* o;
  int o_dtype;
  int64_t o_st, o_sh;
  const int32_t* qsl;
  const int32_t* seq_lens;
  const int32_t* bt;
  int64_t bt_stride;
  const float* alibi;
  int num_heads, num_kv_heads, group, gs, head_slices, qt, page;
  int causal, window;
  float scale_log2, softcap_log2;
  float softcap_rcp;  // RN(1 / softcap_log2): Triton folds the division by the constant cap
  int frac;
  int exact_qk;  // q and K are 16-bit floats: products are exact in fp32
  int cap;       // score capacity (keys) per CTA
  int splits;
  int qtiles;
  int page_shift;  // log2(page) when page is a power of two, else -1
  float one;      // 1.0f, opaque to the compiler (magic add as an FMA)
  // chunked path: caller workspace (no state between calls)
  uint32_t* ws_cnt;            // [items] chunks finished
  unsigned long long* ws_acc;  // [items][RP][D] integer PV partial sums
  unsigned long long* ws_den;  // [items][RP] integer normaliser partial sums
  float* ws_m;                 // [items][nchunk_max][RP] chunk row maxima
  float* ws_s;                 // [items][nchunk_max][RP][CHUNK] scores
  int nchunk_max;
};

// 16-byte chunk of KV elements -> fp32 pairs
template <typename T> struct Chunk;
template <> struct Chunk<__nv_bfloat16> {
  static constexpr int E = 8;
  __device__ static __forceinline__ void unpack(uint4 w, float2 (&out)[4]) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      out[i] = make_float2(__uint_as_float(ws[i] << 16), __uint_as_float(ws[i] & 0xFFFF0000u));
  }
};
template <> struct Chunk<__half> {
  static constexpr int E = 8;
  __device__ static __forceinline__ void unpack(uint4 w, float2 (&out)[4]) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = __half22float2(*reinterpret_cast<const __half2*>(&ws[i]));
  }
};
template <> struct Chunk<float> {
  static constexpr int E = 4;
  __device__ static __forceinline__ void unpack(uint4 w, float2 (&out)[2]) {
    out[0] = make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
    out[1] = make_float2(__uint_as_float(w.z), __uint_as_float(w.w));
  }
};

template <typename T> __device__ __forceinline__ uint32_t chunk_abs_max(uint4 w) {
  return max(max(abs_max_as_f32<T>(w.x), abs_max_as_f32<T>(w.y)),
             max(abs_max_as_f32<T>(w.z), abs_max_as_f32<T>(w.w)));
}

// two V values -> fp32 after the reference's cast to fp16 (attention.py:245-249)
template <typename T> __device__ __forceinline__ float2 v_pair_f16(const unsigned char* p);
template <> __device__ __forceinline__ float2 v_pair_f16<__nv_bfloat16>(const unsigned char* p) {
  const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
  const float a = __uint_as_float(w << 16), b = __uint_as_float(w & 0xFFFF0000u);
  return __half22float2(__floats2half2_rn(a, b));
}
template <> __device__ __forceinline__ float2 v_pair_f16<__half>(const unsigned char* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <> __device__ __forceinline__ float2 v_pair_f16<float>(const unsigned char* p) {
  const float2 f = *reinterpret_cast<const float2*>(p);
  return __half22float2(__floats2half2_rn(f.x, f.y));
}

// Running max of |x| over raw 16-byte chunks / element pairs, kept as packed
// 16-bit halves (bf16, fp16: one SIMD max per word) or as an fp32 pattern.
// (16-bit: NaN-propagating packed max of |x|, so NaN keeps the halves NaN and
// fails the guard)
template <typename T> __device__ __forceinline__ void absmax_word(uint32_t& m, uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&m);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w);
    a = __hmax2_nan(a, __habs2(b));
    m = *reinterpret_cast<uint32_t*>(&a);
  } else if constexpr (std::is_same<T, __half>::value) {
    __half2 a = *reinterpret_cast<__half2*>(&m);
    const __half2 b = *reinterpret_cast<const __half2*>(&w);
    a = __hmax2_nan(a, __habs2(b));
    m = *reinterpret_cast<uint32_t*>(&a);
  } else {
    m = max(m, w & 0x7FFFFFFFu);
  }
}
// the running max as an fp32 value bounding |x| (inf/NaN stay non-finite)
template <typename T> __device__ __forceinline__ float absmax_value(uint32_t m) {
  if constexpr (sizeof(T) == 2) {
    const uint32_t h = max(m & 0xFFFFu, m >> 16);
    return __uint_as_float(abs_max_as_f32<T>(h));
  } else {
    return __uint_as_float(m);
  }
}

// decode path for grouped-query batches (attention_decode.cu)
bool decode_supported(const fxpr_attention_params* a, int G);
int64_t decode_workspace_bytes(int items, int kmax, int D);
int launch_decode(const fxpr_attention_params* a, int kmax, void* workspace, cudaStream_t st);

// chunked two-kernel path (attention_chunked.cu)
bool chunked_supported(int D, int rp, int kv_dtype);
int launch_chunked(const Params& p, int D, int rp, int bits, int kv_dtype, int req, int ys,
                   cudaStream_t st);

}  // namespace attn
}  // namespace fxpr
