// Fixed-point GEMM on CUDA cores (gemm.py:7-46, 97-196; library_ops.py:14-45).
//
// C[m,n] = X2F( sum_k F2X(fp32(a[m,k]) * fp32(b[k,n])) ), integer accumulator
// wrapping at the reference width. Every product is rounded to the 2^-f grid
// before the add, which is non-linear per product, so no tensor-core MMA can
// reproduce it: the kernel runs on the FP32/INT pipes.
//
// Fast path (per K chunk, chosen CTA-wide by an exponent guard): the A tile is
// staged in shared memory pre-scaled by 2^f, so one packed FMA
// (fma.rn.f32x2) gives C + RNE(a*b*2^f) for two products at once (exact
// products for 16-bit operands; fp32 operands use an RN multiply then the
// magic add, which is again exact RNE of the rounded product), and IADD3s
// fold the bit patterns into the int32 accumulator. The magic constant is
// subtracted once per chunk. The guard |a|*|b|*2^f < 2^22 (2^14 for int16)
// rules out saturation and keeps the magic add exact; a chunk that fails it
// (large values, inf, NaN) runs the exact clamp+convert path instead.
//
// Work split: tiles of BM x 128 outputs; split-K over CTAs when the tile
// count is below the resident CTA count. Split partials are added with
// integer atomics (exact and order-free) into a self-cleaning workspace; the
// last CTA of a tile (ticket counter) converts and stores the tile and zeroes
// the workspace and the counter again.
#include <atomic>
#include "fxp_common.cuh"

namespace fxpr {
namespace gemm {

constexpr int BN = 128;
constexpr int BK = 32;
constexpr int TN = 4;
constexpr int THREADS = 256;
constexpr int STAGES = 3;
constexpr int A_LD = BK + 4;  // fp32 row pitch of the staged A tile
#ifndef FXPR_GEMM_KK_UNROLL
#define FXPR_GEMM_KK_UNROLL 2
#endif
constexpr int KK_UNROLL = FXPR_GEMM_KK_UNROLL;  // unroll of the fast k loop

// B tile staging layouts
enum { B_NCONTIG = 0, B_KCONTIG = 1, B_GENERIC = 2 };

template <typename T> struct BLay {
  static constexpr int nrow_bytes = BN * (int)sizeof(T);       // [k][n]
  static constexpr int krow_bytes = BK * (int)sizeof(T) + 16;  // [n][k] + 16 B pad
  static constexpr int stage_bytes_n = BK * nrow_bytes;
  static constexpr int stage_bytes_k = BN * krow_bytes;
  static constexpr int stage_bytes =
      stage_bytes_n > stage_bytes_k ? stage_bytes_n : stage_bytes_k;
};

template <typename T> __device__ __forceinline__ float2 pair_f32(T lo, T hi) {
  return make_float2(to_f32(lo), to_f32(hi));
}

struct Params {
  const void* a;
  int a_dtype;
  int64_t sam, sak;
  const void* b;
  int64_t sbk, sbn;
  void* c;
  int out_kind;
  int64_t scm, scn;
  int64_t M, N, K;
  int frac;
  int splits;
  int64_t tiles_n;
  void* ws;       // int32/int64 partial tiles
  int* counters;  // per-tile tickets
  float one;      // 1.0f, opaque to the compiler (see the magic add below)
  float2 cf2;     // (Cf, Cf), Cf = 1.5 * 2^(23 - frac): the scale-absorbing magic constant
};

template <int BITS> struct MinBlocks { static constexpr int v = 2; };
template <> struct MinBlocks<64> { static constexpr int v = 1; };

template <int BM, int BITS, typename BT, int LAYOUT, bool EXACT>
__global__ void __launch_bounds__(THREADS, MinBlocks<BITS>::v) gemm_kernel(Params p) {
  constexpr int TM = BM / 8;
  constexpr int APT = BM * BK / THREADS;  // A elements staged per thread per chunk
  constexpr int SB = BLay<BT>::stage_bytes;
  constexpr int NRB = BLay<BT>::nrow_bytes;
  constexpr int KRB = BLay<BT>::krow_bytes;
  constexpr int EPC = 16 / (int)sizeof(BT);  // elements per 16-byte chunk
  constexpr double LIMV = (BITS == 16) ? 32767.5 : 4194304.0;

  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* bstage = smem;
  float* As = reinterpret_cast<float*>(smem + STAGES * SB);
  __shared__ uint32_t gor[3][2];  // per-chunk max |A| and |B| bit patterns
  __shared__ int s_last;

  const int t = threadIdx.x, tx = t & 31, ty = t >> 5;
  const int64_t tile = blockIdx.x;
  const int split = blockIdx.y;
  const int64_t m0 = (tile / p.tiles_n) * BM, n0 = (tile % p.tiles_n) * BN;
  const int64_t nchunks = cdiv(p.K, BK);
  const int64_t c0 = nchunks * split / p.splits, c1 = nchunks * (split + 1) / p.splits;
  const float scale = ldexpf(1.0f, p.frac);
  const double scale_d = ldexp(1.0, p.frac);
  const BT* B = reinterpret_cast<const BT*>(p.b);

  if (t < 6) (&gor[0][0])[t] = 0u;

  // ---- B tile staging (cp.async for the two aligned layouts) ----
  auto issue_b = [&](int64_t c, int s) {
    unsigned char* dst = bstage + s * SB;
    const int64_t k0 = c * BK;
    if constexpr (LAYOUT == B_NCONTIG) {
      constexpr int CPR = BN / EPC;
      for (int q = t; q < BK * CPR; q += THREADS) {
        const int kr = q / CPR, cc = q % CPR;
        const int64_t k = k0 + kr, n = n0 + cc * EPC;
        int bytes = 0;
        const BT* src = B;
        if (k < p.K && n < p.N) {
          bytes = (int)((p.N - n < EPC ? p.N - n : EPC) * sizeof(BT));
          src = B + k * p.sbk + n;
        }
        cp_async16(dst + kr * NRB + cc * 16, src, bytes);
      }
    } else if constexpr (LAYOUT == B_KCONTIG) {
      constexpr int CPR = BK / EPC;
      for (int q = t; q < BN * CPR; q += THREADS) {
        const int nr = q / CPR, cc = q % CPR;
        const int64_t k = k0 + cc * EPC, n = n0 + nr;
        int bytes = 0;
        const BT* src = B;
        if (k < p.K && n < p.N) {
          bytes = (int)((p.K - k < EPC ? p.K - k : EPC) * sizeof(BT));
          src = B + n * p.sbn + k;
        }
        cp_async16(dst + nr * KRB + cc * 16, src, bytes);
      }
    } else {
      for (int q = t; q < BK * BN; q += THREADS) {
        const int kr = q / BN, nn = q % BN;
        const int64_t k = k0 + kr, n = n0 + nn;
        BT v = from_f32<BT>(0.0f);
        if (k < p.K && n < p.N) v = B[k * p.sbk + n * p.sbn];
        reinterpret_cast<BT*>(dst + kr * NRB)[nn] = v;
      }
    }
  };
  // max |b| (as fp32 patterns) over the B elements this thread staged: its
  // own copies are visible to it after cp.async.wait_group
  auto own_b_or = [&](int s) -> uint32_t {
    const unsigned char* src = bstage + s * SB;
    uint32_t o = 0;
    if constexpr (LAYOUT == B_GENERIC) {
      for (int q = t; q < BK * BN; q += THREADS) {
        const int kr = q / BN, nn = q % BN;
        o = max(o, __float_as_uint(to_f32(reinterpret_cast<const BT*>(src + kr * NRB)[nn])) & 0x7FFFFFFFu);
      }
    } else {
      constexpr int CPR = (LAYOUT == B_NCONTIG) ? BN / EPC : BK / EPC;
      constexpr int NCH = (LAYOUT == B_NCONTIG) ? BK * CPR : BN * CPR;
      constexpr int RB = (LAYOUT == B_NCONTIG) ? NRB : KRB;
      for (int q = t; q < NCH; q += THREADS) {
        const int r = q / CPR, cc = q % CPR;
        const uint4 v = *reinterpret_cast<const uint4*>(src + r * RB + cc * 16);
        o = max(o, max(max(abs_max_as_f32<BT>(v.x), abs_max_as_f32<BT>(v.y)),
                     max(abs_max_as_f32<BT>(v.z), abs_max_as_f32<BT>(v.w))));
      }
    }
    return o;
  };

  // ---- A staging through registers (converted to fp32, scaled by 2^f) ----
  float areg[APT];
  // A elements of thread t: row (t*APT)/BK, k offset (t*APT)%BK .. +APT-1
  const bool a_vec = (p.sak == 1) && (p.a_dtype == FXPR_BF16 || p.a_dtype == FXPR_F16) &&
                     ((reinterpret_cast<uintptr_t>(p.a) & 15) == 0) && ((p.sam & 7) == 0);
  auto load_a = [&](int64_t c) {
    const int e0 = t * APT;
    const int64_t m = m0 + e0 / BK, k0 = c * BK + e0 % BK;
    if constexpr (APT == 8) {
      if (a_vec && m < p.M && k0 + 8 <= p.K) {
        const uint4 w = *reinterpret_cast<const uint4*>(
            reinterpret_cast<const char*>(p.a) + (m * p.sam + k0) * 2);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (p.a_dtype == FXPR_BF16) {
            areg[2 * h] = __uint_as_float(ws[h] << 16);
            areg[2 * h + 1] = __uint_as_float(ws[h] & 0xFFFF0000u);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[h]));
            areg[2 * h] = f.x;
            areg[2 * h + 1] = f.y;
          }
        }
        return;
      }
    }
#pragma unroll
    for (int r = 0; r < APT; ++r) {
      const int64_t k = k0 + r;
      areg[r] = (m < p.M && k < p.K) ? load_f32(p.a, p.a_dtype, m * p.sam + k * p.sak) : 0.0f;
    }
  };
  auto store_a = [&](int buf) -> uint32_t {
    float* dst = As + buf * BM * A_LD;
    uint32_t o = 0;
#pragma unroll
    for (int r = 0; r < APT; ++r) {
      const int e = t * APT + r;
      dst[(e / BK) * A_LD + (e % BK)] = __fmul_rn(areg[r], scale);
      o = max(o, __float_as_uint(areg[r]) & 0x7FFFFFFFu);
    }
    return o;
  };

  // ---- B fragments: TN columns x 4 k values as two k-pairs ----
  auto b_frag = [&](const unsigned char* Bb, int kk, float2 (&bp)[TN][2]) {
    if constexpr (LAYOUT == B_KCONTIG) {
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const BT* row = reinterpret_cast<const BT*>(Bb + (tx + 32 * j) * KRB) + kk;
        if constexpr (sizeof(BT) == 2) {
          const uint2 w = *reinterpret_cast<const uint2*>(row);
          const BT* e = reinterpret_cast<const BT*>(&w);
          bp[j][0] = pair_f32(e[0], e[1]);
          bp[j][1] = pair_f32(e[2], e[3]);
        } else {
          const float4 w = *reinterpret_cast<const float4*>(row);
          bp[j][0] = make_float2(w.x, w.y);
          bp[j][1] = make_float2(w.z, w.w);
        }
      }
    } else {
      BT rows[4][TN];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const BT* src = reinterpret_cast<const BT*>(Bb + (kk + r) * NRB) + tx * TN;
        if constexpr (sizeof(BT) == 2) {
          *reinterpret_cast<uint2*>(rows[r]) = *reinterpret_cast<const uint2*>(src);
        } else {
          *reinterpret_cast<float4*>(rows[r]) = *reinterpret_cast<const float4*>(src);
        }
      }
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        bp[j][0] = pair_f32(rows[0][j], rows[1][j]);
        bp[j][1] = pair_f32(rows[2][j], rows[3][j]);
      }
    }
  };
  auto b_val = [&](const unsigned char* Bb, int kk, int j) -> float {
    if constexpr (LAYOUT == B_KCONTIG) {
      return to_f32(reinterpret_cast<const BT*>(Bb + (tx + 32 * j) * KRB)[kk]);
    } else {
      return to_f32(reinterpret_cast<const BT*>(Bb + kk * NRB)[tx * TN + j]);
    }
  };
  auto n_local = [&](int j) -> int { return LAYOUT == B_KCONTIG ? tx + 32 * j : tx * TN + j; };

  uint32_t acc[TM][TN];
  unsigned long long acc64[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      acc[i][j] = 0u;
      acc64[i][j] = 0ull;
    }

  // ---- main pipeline ----
  const int64_t nloc = c1 - c0;
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nloc) issue_b(c0 + s, s);
    cp_async_commit();
  }
  if (nloc > 0) load_a(c0);
  __syncthreads();  // gor zeroed

  for (int64_t it = 0; it < nloc; ++it) {
    const int64_t c = c0 + it;
    const int slot = (int)(it % 3);
    const int buf = (int)(it & 1);
    const int s = (int)(it % STAGES);
    uint32_t aor = store_a(buf);
    cp_async_wait<STAGES - 2>();
    uint32_t bor = own_b_or(s);
    aor = __reduce_max_sync(0xffffffffu, aor);
    bor = __reduce_max_sync(0xffffffffu, bor);
    if (tx == 0) {
      atomicMax(&gor[slot][0], aor);
      atomicMax(&gor[slot][1], bor);
    }
    __syncthreads();
    // fast path iff max|a| * max|b| * 2^f < 2^22 (32767.5 for int16): no
    // saturation and an exact magic-constant rounding; NaN/inf compare false
    const double ma = (double)__uint_as_float(gor[slot][0]);
    const double mb = (double)__uint_as_float(gor[slot][1]);
    const bool fast = (ma * mb * scale_d < LIMV) && (ma * scale_d < 3.0e38);
    if (t == 0) {
      // slot read two iterations ago; every thread has passed this barrier
      const int z = (int)((it + 2) % 3);
      gor[z][0] = 0u;
      gor[z][1] = 0u;
    }
    // refill the stage consumed in the previous iteration
    if (it + STAGES - 1 < nloc) issue_b(c + STAGES - 1, (int)((it + STAGES - 1) % STAGES));
    cp_async_commit();
    if (it + 1 < nloc) load_a(c + 1);

    const float* Ab = As + buf * BM * A_LD;
    const unsigned char* Bb = bstage + s * SB;
    if (fast) {
      const float2 C2 = make_float2(kMagic, kMagic);
      const float2 ONE2 = make_float2(p.one, p.one);
#pragma unroll KK_UNROLL
      for (int kk = 0; kk < BK; kk += 4) {
        float2 bp[TN][2];
        b_frag(Bb, kk, bp);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float4 v = *reinterpret_cast<const float4*>(Ab + (ty * TM + i) * A_LD + kk);
          const float2 a0 = make_float2(v.x, v.y), a1 = make_float2(v.z, v.w);
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            float2 r0, r1;
            if constexpr (EXACT) {
              r0 = fma2(a0, bp[j][0], C2);
              r1 = fma2(a1, bp[j][1], C2);
            } else {
              // RN product, then the magic add as an FMA by a runtime 1.0:
              // a plain add could be fused with the multiply into one rounding
              r0 = fma2(mul2(a0, bp[j][0]), ONE2, C2);
              r1 = fma2(mul2(a1, bp[j][1]), ONE2, C2);
            }
            acc[i][j] += __float_as_uint(r0.x) + __float_as_uint(r0.y);
            acc[i][j] += __float_as_uint(r1.x) + __float_as_uint(r1.y);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          acc[i][j] -= (uint32_t)BK * (uint32_t)kMagicBits;
          if constexpr (BITS == 64) {
            acc64[i][j] += (unsigned long long)(long long)(int32_t)acc[i][j];
            acc[i][j] = 0u;
          }
        }
    } else {
      // exact reference path: fp32 product, x 2^f, clamp, RNE convert
      for (int kk = 0; kk < BK; ++kk) {
        const int64_t k = c * BK + kk;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const int64_t m = m0 + ty * TM + i;
          const float a = (m < p.M && k < p.K) ? load_f32(p.a, p.a_dtype, m * p.sam + k * p.sak) : 0.0f;
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            const auto v = f2x_f32<BITS>(__fmul_rn(a, b_val(Bb, kk, j)), scale);
            if constexpr (BITS == 64) {
              acc64[i][j] += (unsigned long long)v;
            } else {
              acc[i][j] += (uint32_t)v;
            }
          }
        }
      }
    }
  }
  cp_async_wait<0>();

  // ---- epilogue ----
  const float inv = ldexpf(1.0f, -p.frac);
  auto final_store = [&](int64_t m, int64_t n, unsigned long long v) {
    if (p.out_kind == 0) {
      float f;
      if constexpr (BITS == 64) {
        f = x2f_f32<64>((long long)v, inv);
      } else {
        f = x2f_f32<BITS>(wrap_acc<BITS>((int32_t)(uint32_t)v), inv);
      }
      reinterpret_cast<float*>(p.c)[m * p.scm + n * p.scn] = f;
    } else if constexpr (BITS == 64) {
      reinterpret_cast<long long*>(p.c)[m * p.scm + n * p.scn] = (long long)v;
    } else {
      reinterpret_cast<int32_t*>(p.c)[m * p.scm + n * p.scn] = (int32_t)(uint32_t)v;
    }
  };
  auto value = [&](int i, int j) -> unsigned long long {
    if constexpr (BITS == 64) return acc64[i][j];
    else return (unsigned long long)acc[i][j];
  };
  if (p.splits == 1) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t m = m0 + ty * TM + i, n = n0 + n_local(j);
        if (m < p.M && n < p.N) final_store(m, n, value(i, j));
      }
    return;
  }
  const int64_t wbase = tile * (int64_t)BM * BN;
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int ml = ty * TM + i, nl = n_local(j);
      if (m0 + ml < p.M && n0 + nl < p.N) {
        if constexpr (BITS == 64) {
          atomicAdd(reinterpret_cast<unsigned long long*>(p.ws) + wbase + ml * BN + nl, acc64[i][j]);
        } else {
          atomicAdd(reinterpret_cast<unsigned int*>(p.ws) + wbase + ml * BN + nl, acc[i][j]);
        }
      }
    }
  __threadfence();
  __syncthreads();
  if (t == 0) s_last = (atomicAdd(p.counters + tile, 1) == p.splits - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int ml = ty * TM + i, nl = n_local(j);
      const int64_t m = m0 + ml, n = n0 + nl;
      if (m < p.M && n < p.N) {
        unsigned long long v;
        if constexpr (BITS == 64) {
          v = atomicExch(reinterpret_cast<unsigned long long*>(p.ws) + wbase + ml * BN + nl, 0ull);
        } else {
          v = atomicExch(reinterpret_cast<unsigned int*>(p.ws) + wbase + ml * BN + nl, 0u);
        }
        final_store(m, n, v);
      }
    }
  if (t == 0) p.counters[tile] = 0;
}

// ---------------------------------------------------------------------------
// K-contiguous 16-bit operands (the linear-layer layout: activations [M, K],
// weight [N, K] read as its transpose), the serving hot path.
//
// Both tiles are staged through registers (16-byte loads of chunk c+1 while
// chunk c is computed) and converted once per CTA to fp32 in shared memory,
// [rows][BK + 4] with k contiguous, so the inner loop reads k-pairs of both
// operands with 16-byte loads (A: warp broadcast; B: four lanes a bank
// group apart) and spends one packed FMA and one IADD3 per two products.
//
// The magic constant absorbs the 2^f scale: with Cf = 1.5 * 2^(23 - f), fp32
// values in [2^(23 - f), 2^(24 - f)) are spaced 2^-f apart and Cf is an even
// multiple of 2^-f, so RN(a * b + Cf) = Cf + RNE(a * b * 2^f) * 2^-f for an
// exact product |a * b * 2^f| <= 2^22, and bits(r) - bits(Cf) is that
// integer. No operand is scaled.
// ---------------------------------------------------------------------------
constexpr int KC_LD = BK + 4;  // fp32 row pitch of the staged tiles

template <int BM, int BITS, typename T>
__global__ void __launch_bounds__(THREADS, BM == 16 ? 4 : 2) gemm_kc_kernel(Params p) {
  constexpr int TM = BM / 8;
  constexpr int A_LOADS = BM * BK / 8 / THREADS;  // 16-byte loads of A per thread per chunk (BM 64: 1)
  constexpr int A_THREADS = BM * BK / 8;          // threads that load A (BM 16: 64)
  constexpr int B_LOADS = BN * BK / 8 / THREADS;  // 2
  constexpr double LIMV = (BITS == 16) ? 32767.5 : 4194304.0;
  static_assert(BK == 32 && BN == 128, "tile shape");

  extern __shared__ __align__(16) unsigned char smem[];
  float* As = reinterpret_cast<float*>(smem);                  // [2][BM][KC_LD]
  float* Bs = As + 2 * BM * KC_LD;                             // [2][BN][KC_LD]
  __shared__ uint32_t gmax[3][2];  // per chunk: max |a|, max |b| as fp32 patterns
  __shared__ int s_last;

  const int t = threadIdx.x, tx = t & 31, ty = t >> 5;
  const int64_t tile = blockIdx.x;
  const int split = blockIdx.y;
  const int64_t m0 = (tile / p.tiles_n) * BM, n0 = (tile % p.tiles_n) * BN;
  const int64_t nchunks = cdiv(p.K, BK);
  const int64_t c0 = nchunks * split / p.splits, c1 = nchunks * (split + 1) / p.splits;
  const int64_t nloc = c1 - c0;
  const float scale = ldexpf(1.0f, p.frac);
  const uint32_t cf_bits = __float_as_uint(p.cf2.x);
  const T* A = reinterpret_cast<const T*>(p.a);
  const T* B = reinterpret_cast<const T*>(p.b);
  if (t < 6) (&gmax[0][0])[t] = 0u;

  // this thread's 16-byte pieces: A row/k of load u, B column/k of load u
  uint4 ra[A_LOADS > 0 ? A_LOADS : 1], rb[B_LOADS];
  auto load_chunk = [&](int64_t c) {
    const int64_t k0 = c * BK;
#pragma unroll
    for (int u = 0; u < (A_LOADS > 0 ? A_LOADS : 1); ++u) {
      const int q = t + u * THREADS;
      const int64_t m = m0 + q / (BK / 8), k = k0 + (q % (BK / 8)) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (q < A_THREADS && m < p.M && k < p.K) v = *reinterpret_cast<const uint4*>(A + m * p.sam + k);
      ra[u] = v;
    }
#pragma unroll
    for (int u = 0; u < B_LOADS; ++u) {
      const int q = t + u * THREADS;
      const int64_t n = n0 + q / (BK / 8), k = k0 + (q % (BK / 8)) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (n < p.N && k < p.K) v = __ldcs(reinterpret_cast<const uint4*>(B + n * p.sbn + k));
      rb[u] = v;
    }
  };
  // convert the staged pieces into buffer `buf` and fold their |x| into gmax[slot]
  auto store_chunk = [&](int buf, int slot) {
    uint32_t mu_a = 0, ms_a = 0x80008000u, mu_b = 0, ms_b = 0x80008000u;
    float* Ad = As + buf * BM * KC_LD;
    float* Bd = Bs + buf * BN * KC_LD;
    auto put = [&](float* dst, uint4 v) {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      float f[8];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          f[2 * h] = __uint_as_float(w[h] << 16);
          f[2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
        } else {
          const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&w[h]));
          f[2 * h] = g.x;
          f[2 * h + 1] = g.y;
        }
      }
      *reinterpret_cast<float4*>(dst) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
    };
#pragma unroll
    for (int u = 0; u < (A_LOADS > 0 ? A_LOADS : 1); ++u) {
      const int q = t + u * THREADS;
      if (q < A_THREADS) {
        put(Ad + (q / (BK / 8)) * KC_LD + (q % (BK / 8)) * 8, ra[u]);
        mu_a = __vimax3_u16x2(mu_a, ra[u].x, ra[u].y);
        mu_a = __vimax3_u16x2(mu_a, ra[u].z, ra[u].w);
        ms_a = (uint32_t)__vimax3_s16x2((int)ms_a, (int)ra[u].x, (int)ra[u].y);
        ms_a = (uint32_t)__vimax3_s16x2((int)ms_a, (int)ra[u].z, (int)ra[u].w);
      }
    }
#pragma unroll
    for (int u = 0; u < B_LOADS; ++u) {
      const int q = t + u * THREADS;
      put(Bd + (q / (BK / 8)) * KC_LD + (q % (BK / 8)) * 8, rb[u]);
      mu_b = __vimax3_u16x2(mu_b, rb[u].x, rb[u].y);
      mu_b = __vimax3_u16x2(mu_b, rb[u].z, rb[u].w);
      ms_b = (uint32_t)__vimax3_s16x2((int)ms_b, (int)rb[u].x, (int)rb[u].y);
      ms_b = (uint32_t)__vimax3_s16x2((int)ms_b, (int)rb[u].z, (int)rb[u].w);
    }
    // |x| bounds as fp32 patterns (16-bit halves -> max magnitude -> fp32)
    auto bound = [](uint32_t mu, uint32_t ms) -> uint32_t {
      const uint32_t pk = __vmaxu2(mu & 0x7FFF7FFFu, ms & 0x7FFF7FFFu);
      return abs_max_as_f32<T>(max(pk & 0xFFFFu, pk >> 16));
    };
    const uint32_t ba = __reduce_max_sync(0xffffffffu, bound(mu_a, ms_a));
    const uint32_t bb = __reduce_max_sync(0xffffffffu, bound(mu_b, ms_b));
    if (tx == 0) {
      atomicMax(&gmax[slot][0], ba);
      atomicMax(&gmax[slot][1], bb);
    }
  };

  uint32_t acc[TM][TN];
  unsigned long long acc64[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      acc[i][j] = 0u;
      acc64[i][j] = 0ull;
    }

  if (nloc > 0) load_chunk(c0);
  __syncthreads();  // gmax zeroed
  if (nloc > 0) store_chunk(0, 0);
  if (nloc > 1) load_chunk(c0 + 1);
  __syncthreads();

  const float2 CF2 = p.cf2;  // a kernel parameter: the packed FMA reads it from the constant bank
  for (int64_t it = 0; it < nloc; ++it) {
    const int buf = (int)(it & 1), slot = (int)(it % 3);
    const float ma = __uint_as_float(gmax[slot][0]), mb = __uint_as_float(gmax[slot][1]);
    // fast iff max|a| * max|b| * 2^f < 2^22 (int16: < 32767.5); NaN/inf fail
    const bool fast = (double)__fmul_ru(ma, mb) * (double)scale < LIMV;
    if (t == 0) {  // the slot read two chunks ago is free again
      const int z = (int)((it + 2) % 3);
      gmax[z][0] = 0u;
      gmax[z][1] = 0u;
    }
    const float* Ab = As + buf * BM * KC_LD + (ty * TM) * KC_LD;
    const float* Bb = Bs + buf * BN * KC_LD + tx * KC_LD;
    if (fast) {
#pragma unroll
      for (int kk = 0; kk < BK; kk += 4) {
        float4 bv[TN];
#pragma unroll
        for (int j = 0; j < TN; ++j) bv[j] = *reinterpret_cast<const float4*>(Bb + j * 32 * KC_LD + kk);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float4 av = *reinterpret_cast<const float4*>(Ab + i * KC_LD + kk);
          const float2 a0 = make_float2(av.x, av.y), a1 = make_float2(av.z, av.w);
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            const float2 r0 = fma2(a0, make_float2(bv[j].x, bv[j].y), CF2);
            const float2 r1 = fma2(a1, make_float2(bv[j].z, bv[j].w), CF2);
            acc[i][j] += __float_as_uint(r0.x) + __float_as_uint(r0.y);
            acc[i][j] += __float_as_uint(r1.x) + __float_as_uint(r1.y);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          acc[i][j] -= (uint32_t)BK * cf_bits;
          if constexpr (BITS == 64) {
            acc64[i][j] += (unsigned long long)(long long)(int32_t)acc[i][j];
            acc[i][j] = 0u;
          }
        }
    } else {
      // exact reference path on the staged (exact) fp32 values
#pragma unroll 1
      for (int kk = 0; kk < BK; ++kk) {
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float a = Ab[i * KC_LD + kk];
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            const auto v = f2x_f32<BITS>(__fmul_rn(a, Bb[j * 32 * KC_LD + kk]), scale);
            if constexpr (BITS == 64) {
              acc64[i][j] += (unsigned long long)v;
            } else {
              acc[i][j] += (uint32_t)v;
            }
          }
        }
      }
    }
    if (it + 1 < nloc) store_chunk(buf ^ 1, (int)((it + 1) % 3));
    if (it + 2 < nloc) load_chunk(c0 + it + 2);
    __syncthreads();
  }

  // ---- epilogue (as gemm_kernel: direct store, or split-K integer atomics) ----
  const float inv = ldexpf(1.0f, -p.frac);
  auto final_store = [&](int64_t m, int64_t n, unsigned long long v) {
    if (p.out_kind == 0) {
      float f;
      if constexpr (BITS == 64) {
        f = x2f_f32<64>((long long)v, inv);
      } else {
        f = x2f_f32<BITS>(wrap_acc<BITS>((int32_t)(uint32_t)v), inv);
      }
      reinterpret_cast<float*>(p.c)[m * p.scm + n * p.scn] = f;
    } else if constexpr (BITS == 64) {
      reinterpret_cast<long long*>(p.c)[m * p.scm + n * p.scn] = (long long)v;
    } else {
      reinterpret_cast<int32_t*>(p.c)[m * p.scm + n * p.scn] = (int32_t)(uint32_t)v;
    }
  };
  auto value = [&](int i, int j) -> unsigned long long {
    if constexpr (BITS == 64) return acc64[i][j];
    else return (unsigned long long)acc[i][j];
  };
  if (p.splits == 1) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t m = m0 + ty * TM + i, n = n0 + tx + 32 * j;
        if (m < p.M && n < p.N) final_store(m, n, value(i, j));
      }
    return;
  }
  const int64_t wbase = tile * (int64_t)BM * BN;
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int ml = ty * TM + i, nl = tx + 32 * j;
      if (m0 + ml < p.M && n0 + nl < p.N) {
        if constexpr (BITS == 64) {
          atomicAdd(reinterpret_cast<unsigned long long*>(p.ws) + wbase + ml * BN + nl, acc64[i][j]);
        } else {
          atomicAdd(reinterpret_cast<unsigned int*>(p.ws) + wbase + ml * BN + nl, acc[i][j]);
        }
      }
    }
  __threadfence();
  __syncthreads();
  if (t == 0) s_last = (atomicAdd(p.counters + tile, 1) == p.splits - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int ml = ty * TM + i, nl = tx + 32 * j;
      const int64_t m = m0 + ml, n = n0 + nl;
      if (m < p.M && n < p.N) {
        unsigned long long v;
        if constexpr (BITS == 64) {
          v = atomicExch(reinterpret_cast<unsigned long long*>(p.ws) + wbase + ml * BN + nl, 0ull);
        } else {
          v = atomicExch(reinterpret_cast<unsigned int*>(p.ws) + wbase + ml * BN + nl, 0u);
        }
        final_store(m, n, v);
      }
    }
  if (t == 0) p.counters[tile] = 0;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Plan {
  int bm;
  int64_t tiles, tiles_n;
  int splits;
};

// Tile height: 16 rows for M <= 16, 32 for M <= 32 (and with 64-bit
// accumulators, whose extra int64 registers would not fit 64 rows), else 64
static Plan make_plan(int64_t M, int64_t N, int64_t K, int bits) {
  Plan pl;
  pl.bm = M <= 16 ? 16 : ((M <= 32 || bits == 64) ? 32 : 64);
  pl.tiles_n = cdiv(N, BN);
  pl.tiles = cdiv(M, pl.bm) * pl.tiles_n;
  // resident CTAs per SM: 16-row tiles are small enough for four
  const int64_t target = (int64_t)num_sms() * (pl.bm == 16 ? 4 : 2);
  const int64_t nchunks = cdiv(K, BK);
  int64_t s = pl.tiles >= target ? 1 : target / pl.tiles;
  const int64_t smax = nchunks / 2 > 1 ? nchunks / 2 : 1;  // >= 2 chunks per split
  if (s > smax) s = smax;
  if (s > 64) s = 64;
  if (s < 1) s = 1;
  pl.splits = (int)s;
  return pl;
}

static int64_t ws_bytes(const Plan& pl, int bits) {
  if (pl.splits == 1) return 0;
  const int64_t elem = bits == 64 ? 8 : 4;
  return pl.tiles * pl.bm * BN * elem + pl.tiles * (int64_t)sizeof(int);
}

template <int BM, int BITS, typename BT, int LAYOUT, bool EXACT>
static int launch(const Params& p, int64_t tiles, cudaStream_t st) {
  auto k = gemm_kernel<BM, BITS, BT, LAYOUT, EXACT>;
  const int smem = STAGES * BLay<BT>::stage_bytes + 2 * BM * A_LD * (int)sizeof(float);
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      set_error("gemm_fxp: cannot configure %d bytes of shared memory", smem);
      return FXPR_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const dim3 grid((unsigned)tiles, (unsigned)p.splits);
  k<<<grid, THREADS, smem, st>>>(p);
  return check_launch("fxpr_gemm_fxp");
}

template <int BM, int BITS, typename BT>
static int pick_layout(const Params& p, int64_t tiles, bool exact, cudaStream_t st) {
  const int es = (int)sizeof(BT);
  const bool al = ((uintptr_t)p.b % 16) == 0;
  const bool ncontig = al && p.sbn == 1 && (p.sbk * es) % 16 == 0;
  const bool kcontig = al && p.sbk == 1 && (p.sbn * es) % 16 == 0;
  if constexpr (std::is_same<BT, __nv_bfloat16>::value) {
    if (exact && ncontig) return launch<BM, BITS, BT, B_NCONTIG, true>(p, tiles, st);
    if (exact && kcontig) return launch<BM, BITS, BT, B_KCONTIG, true>(p, tiles, st);
  }
  if (ncontig) return launch<BM, BITS, BT, B_NCONTIG, false>(p, tiles, st);
  if (kcontig) return launch<BM, BITS, BT, B_KCONTIG, false>(p, tiles, st);
  return launch<BM, BITS, BT, B_GENERIC, false>(p, tiles, st);
}

template <int BM, int BITS, typename T>
static int launch_kc(const Params& p, int64_t tiles, cudaStream_t st) {
  auto k = gemm_kc_kernel<BM, BITS, T>;
  const int smem = 2 * (BM + BN) * KC_LD * (int)sizeof(float);
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      set_error("gemm_fxp: cannot configure %d bytes of shared memory", smem);
      return FXPR_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const dim3 grid((unsigned)tiles, (unsigned)p.splits);
  k<<<grid, THREADS, smem, st>>>(p);
  return check_launch("fxpr_gemm_fxp");
}

// both operands 16-bit of one type, k contiguous, 16-byte aligned rows
static bool kc_ok(const Params& p, int b_dtype) {
  if (p.a_dtype != b_dtype || (b_dtype != FXPR_BF16 && b_dtype != FXPR_F16)) return false;
  if (p.sak != 1 || p.sbk != 1 || p.K % 8 != 0) return false;
  if ((uintptr_t)p.a % 16 != 0 || (uintptr_t)p.b % 16 != 0) return false;
  if (p.sam % 8 != 0 || p.sbn % 8 != 0) return false;
  return p.frac >= 0 && p.frac <= 100;
}

template <int BM, int BITS>
static int pick_btype(const Params& p, int b_dtype, int64_t tiles, cudaStream_t st) {
  if (kc_ok(p, b_dtype))
    return b_dtype == FXPR_BF16 ? launch_kc<BM, BITS, __nv_bfloat16>(p, tiles, st)
                                : launch_kc<BM, BITS, __half>(p, tiles, st);
  const bool a16 = p.a_dtype == FXPR_BF16 || p.a_dtype == FXPR_F16;
  switch (b_dtype) {
    case FXPR_BF16: return pick_layout<BM, BITS, __nv_bfloat16>(p, tiles, a16, st);
    case FXPR_F16: return pick_layout<BM, BITS, __half>(p, tiles, a16, st);
    default: return pick_layout<BM, BITS, float>(p, tiles, false, st);
  }
}

}  // namespace gemm
}  // namespace fxpr

using namespace fxpr;

extern "C" int64_t fxpr_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int int_bits) {
  if (M <= 0 || N <= 0) return 0;
  return gemm::ws_bytes(gemm::make_plan(M, N, K, int_bits), int_bits);
}

extern "C" int fxpr_gemm_fxp(const void* a, int a_dtype, int64_t sam, int64_t sak, const void* b,
                             int b_dtype, int64_t sbk, int64_t sbn, void* c, int out_kind,
                             int64_t scm, int64_t scn, int64_t M, int64_t N, int64_t K,
                             int frac_bits, int int_bits, void* workspace, int64_t workspace_bytes,
                             void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  auto okd = [](int d) { return d == FXPR_F16 || d == FXPR_BF16 || d == FXPR_F32; };
  if (!okd(a_dtype) || !okd(b_dtype)) {
    set_error("gemm_fxp: a and b must be float16/bfloat16/float32");
    return FXPR_ERR_UNSUPPORTED;
  }
  if (frac_bits < 0 || frac_bits > 100) {
    set_error("gemm_fxp: frac_bits must be in [0, 100], got %d", frac_bits);
    return FXPR_ERR_INVALID;
  }
  if (out_kind != 0 && out_kind != 1) {
    set_error("gemm_fxp: bad out_kind %d", out_kind);
    return FXPR_ERR_INVALID;
  }
  if (M < 0 || N < 0 || K < 0) {
    set_error("gemm_fxp: negative shape");
    return FXPR_ERR_INVALID;
  }
  if (M == 0 || N == 0) return FXPR_OK;
  const gemm::Plan pl = gemm::make_plan(M, N, K, int_bits);
  if (pl.tiles > 0x7fffffffLL) {
    set_error("gemm_fxp: problem too large");
    return FXPR_ERR_INVALID;
  }
  const int64_t need = gemm::ws_bytes(pl, int_bits);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) {
    set_error("gemm_fxp: workspace of %lld bytes required", (long long)need);
    return FXPR_ERR_INVALID;
  }
  gemm::Params p;
  p.a = a; p.a_dtype = a_dtype; p.sam = sam; p.sak = sak;
  p.b = b; p.sbk = sbk; p.sbn = sbn;
  p.c = c; p.out_kind = out_kind; p.scm = scm; p.scn = scn;
  p.M = M; p.N = N; p.K = K; p.frac = frac_bits; p.one = 1.0f;
  p.cf2 = make_float2(ldexpf(1.5f, 23 - frac_bits), ldexpf(1.5f, 23 - frac_bits));
  p.splits = pl.splits; p.tiles_n = pl.tiles_n;
  p.ws = workspace;
  p.counters = need > 0 ? reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + need -
                                                 pl.tiles * (int64_t)sizeof(int))
                        : nullptr;
  const cudaStream_t st = (cudaStream_t)stream;
  if (pl.bm == 16) {
    if (int_bits == 16) return gemm::pick_btype<16, 16>(p, b_dtype, pl.tiles, st);
    if (int_bits == 32) return gemm::pick_btype<16, 32>(p, b_dtype, pl.tiles, st);
    return gemm::pick_btype<16, 64>(p, b_dtype, pl.tiles, st);
  }
  if (pl.bm == 32) {
    if (int_bits == 16) return gemm::pick_btype<32, 16>(p, b_dtype, pl.tiles, st);
    if (int_bits == 32) return gemm::pick_btype<32, 32>(p, b_dtype, pl.tiles, st);
    return gemm::pick_btype<32, 64>(p, b_dtype, pl.tiles, st);
  }
  if (int_bits == 16) return gemm::pick_btype<64, 16>(p, b_dtype, pl.tiles, st);
  return gemm::pick_btype<64, 32>(p, b_dtype, pl.tiles, st);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of fxpr_gemm_fxp.
//
// Some callers cannot allocate device memory at the moment they run a GEMM:
// for example an engine that plans every device buffer up front and forbids
// allocation while serving, or a host binding (FFI from another language)
// that has no device allocator of its own to hand a workspace to us. For
// them the split-K workspace lives in a fixed array in this library's device
// image instead of a caller-supplied buffer.
//
// The array is a host-side stand-in in host code, never a device address:
// the device address is looked up once per device with cudaGetSymbolAddress
// (with that device current) on the first call made on it, so that first call
// should happen before any stream capture. Every call shares the one array,
// so calls that overlap on the GPU (different streams, or several host
// threads) race on it; serialise them. Each call zeroes the part it needs
// before the launch.
// ---------------------------------------------------------------------------
namespace fxpr {
namespace gemm {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Per-device address cache. Host threads may race on the first lookup; each
// stores the same address, and the atomics make the race benign.
static void* noalloc_scratch_ptr(int* rc) {
  static std::atomic<void*> ptrs[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("gemm_fxp_noalloc: no current CUDA device");
    *rc = FXPR_ERR_CUDA;
    return nullptr;
  }
  void* cached = ptrs[dev].load(std::memory_order_acquire);
  if (cached == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("gemm_fxp_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      *rc = FXPR_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev].store(p, std::memory_order_release);
    cached = p;
  }
  *rc = FXPR_OK;
  return cached;
}

}  // namespace gemm
}  // namespace fxpr

extern "C" int fxpr_gemm_fxp_noalloc(const void* a, int a_dtype, int64_t sam, int64_t sak,
                                     const void* b, int b_dtype, int64_t sbk, int64_t sbn, void* c,
                                     int out_kind, int64_t scm, int64_t scn, int64_t M, int64_t N,
                                     int64_t K, int frac_bits, int int_bits, void* stream) {
  if (!valid_bits(int_bits)) {
    set_error("fxp_int_bits must be 16/32/64, got %d", int_bits);
    return FXPR_ERR_INVALID;
  }
  if (M <= 0 || N <= 0) return fxpr_gemm_fxp(a, a_dtype, sam, sak, b, b_dtype, sbk, sbn, c, out_kind,
                                             scm, scn, M, N, K, frac_bits, int_bits, nullptr, 0,
                                             stream);
  const int64_t need = fxpr_gemm_workspace_bytes(M, N, K, int_bits);
  if (need > gemm::kNoAllocScratchBytes) {
    set_error("gemm_fxp_noalloc: this shape needs %lld bytes of split-K scratch, above the "
              "fixed %lld-byte maximum; use fxpr_gemm_fxp with a caller workspace",
              (long long)need, (long long)gemm::kNoAllocScratchBytes);
    return FXPR_ERR_INVALID;
  }
  void* ws = nullptr;
  if (need > 0) {
    int rc = FXPR_OK;
    ws = gemm::noalloc_scratch_ptr(&rc);
    if (rc != FXPR_OK) return rc;
    const cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)need, (cudaStream_t)stream);
    if (e != cudaSuccess) {
      set_error("gemm_fxp_noalloc: clearing the scratch failed: %s", cudaGetErrorString(e));
      return FXPR_ERR_CUDA;
    }
  }
  return fxpr_gemm_fxp(a, a_dtype, sam, sak, b, b_dtype, sbk, sbn, c, out_kind, scm, scn, M, N, K,
                       frac_bits, int_bits, ws, need, stream);
}
