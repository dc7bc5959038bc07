// Paged decode attention for grouped-query batches (one query row per
// request, 4 query heads per KV head), the serving hot path of
// attention.py:18-489, as two persistent kernels whose warps are
// independent workers fed by TMA.
//
// Work decomposition. A request's context is cut into pages of 16 keys; the
// pages of all (request, KV head) items are concatenated in one sequence and
// every warp of the grid takes an equal contiguous slice of it (to one
// page). There is no CTA-wide barrier after the prologue: each warp runs
// its own ring of STAGES page buffers, and lane 0 issues one TMA box per
// page (16 keys x head_dim of one KV head) on the buffer's mbarrier.
//
//   scores  q.k in integers (every product rounded to Q-format, exact
//           integer sum), X2F, scale, mask -> fp32 scores of the page and
//           its row maxima, written to the workspace. The warp that owns an
//           item's first page clears the item's integer accumulators.
//   pv      row max of the item = max over its pages' maxima (the
//           reference's whole-context pass-1 max), p = exp2(s - max), the
//           integer normaliser and integer PV sums over the warp's pages of
//           the item; a warp that holds a whole item finalises it from
//           registers, otherwise it adds its integer partials to the item's
//           accumulators and the warp completing the item's page count
//           divides and stores (integer addition: exact, order-free).
//
// Results are bit-identical to the two other device paths and to the
// oracle; only the schedule differs.
#include "attention_common.cuh"
#include "tma.cuh"

namespace fxpr {
namespace attn {
namespace dq {

#ifndef FXPR_DQ_WARPS
#define FXPR_DQ_WARPS 4
#endif
#ifndef FXPR_DQ_MINB1
#define FXPR_DQ_MINB1 4
#endif
#ifndef FXPR_DQ_MINB2
#define FXPR_DQ_MINB2 4
#endif
constexpr int W = FXPR_DQ_WARPS;  // warps (workers) per CTA
constexpr int PG = 16;     // keys per page tile
constexpr int RP = 4;      // query rows per item (the GQA group)
constexpr int TPK = 8;     // lanes sharing one key in the scores kernel
#ifndef FXPR_DQ_STAGES
#define FXPR_DQ_STAGES 2
#endif
constexpr int S = FXPR_DQ_STAGES;  // page buffers per warp
constexpr int MAX_REQ = 4096;
constexpr int kRedGroup = 72;             // words per key group in the transpose buffer
constexpr int kRedWords = 4 * kRedGroup;  // per warp

// error bits written to the workspace's first word
constexpr uint32_t kErrContextCut = 1u;  // a context longer than max_seq_len was cut
constexpr uint32_t kErrWaitTimeout = 2u; // a page copy did not land in time

struct DqParams {
  const void* q;
  int64_t q_st, q_sh;
  void* o;
  int o_dtype;
  int64_t o_st, o_sh;
  const int32_t* qsl;
  const int32_t* seq_lens;
  const int32_t* bt;
  int64_t bt_stride;
  int R, KVH, page, page_shift, kmax;
  float scale_log2;
  int frac;
  float one;
  int v_exact16;  // bf16 V and frac <= 16: bf16 -> fp16 -> fp32 is the identity here
  uint32_t* err;
  uint32_t* cnt;             // [items] pages finished (pv)
  unsigned long long* den;   // [items][RP]
  unsigned long long* acc;   // [items][RP][D]
  float* m;                  // [pages][RP] page row maxima
  float* s;                  // [pages][RP][PG] scores
};

template <int D> struct Geo {
  static constexpr int ROWB = D * 2;          // bytes of one key row (16-bit elements)
  static constexpr int PAGEB = PG * ROWB;     // one TMA box
  static constexpr int CQ = D / 64;           // 16-byte chunks per lane per key (scores)
  static constexpr int DPT = CQ * 8;          // dims per lane per key (scores)
  static constexpr int DPL = D / 32;          // dims per lane (pv)
};

// pages of every item of request r (0 without a query row); kend = keys
__device__ __forceinline__ int pages_of(const DqParams& p, int r, int* kend) {
  const int qlen = p.qsl[r + 1] - p.qsl[r];
  const int sl = p.seq_lens[r];
  const int ke = min(sl, p.kmax);
  if (kend) *kend = ke;
  if (qlen < 1) return 0;
  return max(1, (ke + PG - 1) / PG);
}

// pre[r] = first page of request r's items in the sequence; pre[R] = total.
// Called by the whole CTA (contains __syncthreads).
__device__ void build_prefix(const DqParams& p, int* pre) {
  const int t = threadIdx.x, lane = t & 31;
  for (int r = t; r < p.R; r += blockDim.x) pre[r + 1] = pages_of(p, r, nullptr) * p.KVH;
  __syncthreads();
  if (t < 32) {
    int carry = 0;
    for (int base = 0; base < p.R; base += 32) {
      const int r = base + lane;
      int v = r < p.R ? pre[r + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (r < p.R) pre[r + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) pre[0] = 0;
  }
  __syncthreads();
}

// where page G of the sequence lives: item (request * KVH + kv head) and
// page within the item
__device__ __forceinline__ void locate(const DqParams& p, const int* pre, int G, int* item, int* pg,
                                       int* np_out) {
  int lo = 0, hi = p.R;  // pre[lo] <= G < pre[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pre[mid] <= G) lo = mid;
    else hi = mid;
  }
  const int np = (pre[lo + 1] - pre[lo]) / p.KVH;
  const int rem = G - pre[lo];
  const int kvh = rem / np;
  *item = lo * p.KVH + kvh;
  *pg = rem - kvh * np;
  *np_out = np;
}

// one lane's view of page (base + lane) of the warp's slice: item, page in
// the item, and the TMA coordinates of its box (cache block; kv head and
// first slot packed as kvh | slot0 << 16)
struct Slot {
  int item, pg, blk, kc;
};

__device__ __forceinline__ Slot resolve(const DqParams& p, const int* pre, int base, int G1) {
  Slot s{-1, 0, 0, 0};
  const int G = base + (int)(threadIdx.x & 31);
  if (G < G1) {
    int np;
    locate(p, pre, G, &s.item, &s.pg, &np);
    const int r = s.item / p.KVH;
    const int kvh = s.item - r * p.KVH;
    const int key0 = s.pg * PG;
    const int col = p.page_shift >= 0 ? (key0 >> p.page_shift) : key0 / p.page;
    const int slot0 = key0 - col * p.page;
    s.kc = kvh | (slot0 << 16);
    s.blk = __ldg(p.bt + (int64_t)r * p.bt_stride + col);
  }
  return s;
}

// 32-bit shared-memory loads and stores
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void sts64f(uint32_t a, float x, float y) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(x), "f"(y) : "memory");
}

// Running |x| bound over raw 16-bit element pairs without unpacking: the
// unsigned max of the raw halves is the largest negative magnitude (sign bit
// set) when any is negative, else the largest positive one; the signed max
// is the largest positive magnitude when any is non-negative. Together
// (|.| of both) they bound every |x|, NaN and inf included.
struct AbsMax16 {
  uint32_t u = 0, s = 0x80008000u;
  __device__ __forceinline__ void add2(uint32_t a, uint32_t b) {
    u = __vimax3_u16x2(u, a, b);
    s = (uint32_t)__vimax3_s16x2((int)s, (int)a, (int)b);
  }
  // the bound as the running max of |x| patterns packed in two halves
  __device__ __forceinline__ uint32_t packed() const {
    return __vmaxu2(u & 0x7FFF7FFFu, s & 0x7FFF7FFFu);
  }
};

template <typename T>
__device__ __forceinline__ float absmax_f32(const AbsMax16& m) {
  return absmax_value<T>(m.packed());
}

// 8 elements of a 16-byte chunk as 4 fp32 pairs (exact)
template <typename T>
__device__ __forceinline__ void unpack8(uint4 w, float2 (&out)[4]) {
  Chunk<T>::unpack(w, out);
}

template <int N>
__device__ __forceinline__ void reduce_scatter8_u32(uint32_t (&v)[N], int kq) {
  static_assert(N == 8, "8 values over 8 lanes");
#pragma unroll
  for (int s = 4, n = 8; s >= 1; s >>= 1, n >>= 1) {
    const bool hi = (kq & s) != 0;
#pragma unroll
    for (int k = 0; k < n / 2; ++k) {
      const uint32_t send = hi ? v[k] : v[k + n / 2];
      const uint32_t keep = hi ? v[k + n / 2] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
}
__device__ __forceinline__ void reduce_scatter8_u64(unsigned long long (&v)[8], int kq) {
#pragma unroll
  for (int s = 4, n = 8; s >= 1; s >>= 1, n >>= 1) {
    const bool hi = (kq & s) != 0;
#pragma unroll
    for (int k = 0; k < n / 2; ++k) {
      const unsigned long long send = hi ? v[k] : v[k + n / 2];
      const unsigned long long keep = hi ? v[k + n / 2] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
}

// After a wait gave up at page i: bounded waits for the pages issued after
// it, so no copy is left in flight into this warp's buffers.
__device__ __forceinline__ void drain(uint64_t* bars, int i, int n) {
  for (int k = i + 1; k < n && k < i + S; ++k) (void)tma::mbar_wait(&bars[k % S], (uint32_t)((k / S) & 1));
}

// Per-warp page pipeline: the slice's page list in two 32-page batches of
// lane-held slots (A: current, B: next, resolved 32 pages ahead so their
// block-table reads land early), and the TMA issue of page i into buffer
// i % S.
struct Pipe {
  Slot A, B;
  int a_idx;
  __device__ __forceinline__ void advance(const DqParams& p, const int* pre, int G0, int G1) {
    A = B;
    ++a_idx;
    B = resolve(p, pre, G0 + (a_idx + 1) * 32, G1);
  }
  // (item, pg) of page i (in batch A)
  __device__ __forceinline__ int2 item_pg(int i) const {
    return make_int2(__shfl_sync(0xffffffffu, A.item, i & 31), __shfl_sync(0xffffffffu, A.pg, i & 31));
  }
  // coordinates of page i: (kv head | slot0 << 16, block)
  __device__ __forceinline__ int2 coords(int i) const {
    const bool b = (i >> 5) != a_idx;
    return make_int2(__shfl_sync(0xffffffffu, b ? B.kc : A.kc, i & 31),
                     __shfl_sync(0xffffffffu, b ? B.blk : A.blk, i & 31));
  }
};

// ---------------------------------------------------------------------------
// kernel 1: scores and page row maxima
// ---------------------------------------------------------------------------
// exact q.k partial dots of one lane (keys kA and kA + 4, its dims), every
// product clamped and rounded on its own; the rare path for values the
// magic-constant rounding cannot take (large, inf, NaN)
struct Dots8 {
  unsigned long long v[8];
};
template <int D, int BITS, typename T>
__device__ __forceinline__ Dots8 exact_dots(const T* qbase, int64_t q_sh, uint32_t kt, int kA, int kq,
                                         float scale) {
  using GE = Geo<D>;
  Dots8 r;
#pragma unroll
  for (int v = 0; v < 8; ++v) r.v[v] = 0ull;
#pragma unroll 1
  for (int h = 0; h < GE::CQ; ++h) {
    const int c = kq + TPK * h;
#pragma unroll 1
    for (int e = 0; e < 8; ++e) {
      float qf[RP];
#pragma unroll
      for (int row = 0; row < RP; ++row) qf[row] = to_f32(qbase[row * q_sh + c * 8 + e]);
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
        const uint32_t w = lds32(kt + (kA + 4 * mm) * GE::ROWB + c * 16 + (e >> 1) * 4);
        const uint16_t bitsk = (uint16_t)(w >> (16 * (e & 1)));
        const float kf = to_f32(*reinterpret_cast<const T*>(&bitsk));
#pragma unroll
        for (int row = 0; row < RP; ++row)
          r.v[mm * RP + row] += (unsigned long long)(long long)f2x_f32<BITS>(__fmul_rn(qf[row], kf), scale);
      }
    }
  }
  return r;
}

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(W * 32, FXPR_DQ_MINB1)
dq_scores_kernel(const __grid_constant__ CUtensorMap kmap, const DqParams p) {
  using GE = Geo<D>;
  constexpr int ROWB = GE::ROWB, PAGEB = GE::PAGEB, CQ = GE::CQ, DPT = GE::DPT;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* stage0 = smem + warp * (S * PAGEB);
  const uint32_t stage0_a = tma::smem_addr(stage0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + W * S * PAGEB) + warp * S;
  // per warp: the partial-dot transpose buffer, [key group][value][lane] with
  // a 72-word group pitch (conflict-free writes), then the page prefix
  uint32_t* red = reinterpret_cast<uint32_t*>(smem + W * S * PAGEB + W * S * 8) + warp * kRedWords;
  int* pre = reinterpret_cast<int*>(smem + W * S * PAGEB + W * S * 8 + W * kRedWords * 4);

  build_prefix(p, pre);
  const int64_t T_ = pre[p.R];
  const int64_t nw = (int64_t)gridDim.x * W, g = (int64_t)blockIdx.x * W + warp;
  const int G0 = (int)(T_ * g / nw), G1 = (int)(T_ * (g + 1) / nw);
  const int n = G1 - G0;
  if (n <= 0) return;
  if (lane == 0) {
    for (int s = 0; s < S; ++s) tma::mbar_init(&bars[s], 1);
    tma::mbar_init_fence();
  }
  __syncwarp();
  const uint64_t pol = tma::policy_evict_first();

  Pipe pp;
  pp.A = resolve(p, pre, G0, G1);
  pp.B = resolve(p, pre, G0 + 32, G1);
  pp.a_idx = 0;
  auto issue = [&](int i) {
    const int2 c = pp.coords(i);
    if (lane == 0) {
      uint64_t* bar = &bars[i % S];
      tma::fence_proxy_async();
      tma::mbar_expect_tx(bar, PAGEB);
      tma::load_4d(stage0 + (i % S) * PAGEB, &kmap, 0, c.x & 0xFFFF, c.x >> 16, c.y, bar, pol);
    }
  };
  for (int i = 0; i < S - 1 && i < n; ++i) issue(i);

  const int kg = lane >> 3, kq = lane & (TPK - 1);
  const int my_row = kq & 3, my_key = kg + 4 * (kq >> 2);  // after the reduce-scatter
  const uint32_t lane_off = kg * ROWB + kq * 16;
  const float scale = ldexpf(1.0f, p.frac), inv_scale = ldexpf(1.0f, -p.frac);
  const float2 C2 = make_float2(kMagic, kMagic);
  int cur_item = -1, kend = 0;
  const T* qbase = nullptr;
  float kthr = 0.0f;
  float2 qr[RP][CQ][4];  // this lane's q dims (pre-scaled by 2^f), fp32 pairs

  for (int i = 0; i < n; ++i) {
    if ((i >> 5) != pp.a_idx) pp.advance(p, pre, G0, G1);
    if (i + S - 1 < n) issue(i + S - 1);
    const int2 ip = pp.item_pg(i);
    if (ip.x != cur_item) {
      cur_item = ip.x;
      const int r = ip.x / p.KVH;
      const int kvh = ip.x - r * p.KVH;
      const int sl_r = p.seq_lens[r];
      kend = min(sl_r, p.kmax);
      if (sl_r > p.kmax && lane == 0) atomicOr(p.err, kErrContextCut);
      qbase = reinterpret_cast<const T*>(p.q) + (int64_t)p.qsl[r] * p.q_st + (int64_t)(kvh * RP) * p.q_sh;
      uint32_t qo = 0;
#pragma unroll
      for (int row = 0; row < RP; ++row)
#pragma unroll
        for (int h = 0; h < CQ; ++h) {
          const uint4 w = *reinterpret_cast<const uint4*>(qbase + row * p.q_sh + (kq + TPK * h) * 8);
          float2 f[4];
          unpack8<T>(w, f);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            qo = max(qo, max(__float_as_uint(f[e].x) & 0x7FFFFFFFu, __float_as_uint(f[e].y) & 0x7FFFFFFFu));
            qr[row][h][e] = make_float2(__fmul_rn(f[e].x, scale), __fmul_rn(f[e].y, scale));
          }
        }
      qo = max(qo, __shfl_xor_sync(0xffffffffu, qo, 1));
      qo = max(qo, __shfl_xor_sync(0xffffffffu, qo, 2));
      qo = max(qo, __shfl_xor_sync(0xffffffffu, qo, 4));
      const double mq = (double)__uint_as_float(qo) * (double)ldexp(1.0, p.frac);
      kthr = mq < 3.0e38 ? __double2float_rd(4194304.0 / mq) : 0.0f;  // NaN: 0
    }
    if (ip.y == 0) {  // first page of the item: clear its pv accumulators
      unsigned long long* a = p.acc + (int64_t)ip.x * (RP * D);
      for (int e = lane; e < RP * D; e += 32) a[e] = 0ull;
      if (lane < RP) p.den[(int64_t)ip.x * RP + lane] = 0ull;
      if (lane == 0) p.cnt[ip.x] = 0u;
    }
    if (!tma::mbar_wait(&bars[i % S], (uint32_t)((i / S) & 1))) {
      if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
      drain(bars, i, n);
      break;
    }
    const uint32_t kt = stage0_a + (i % S) * PAGEB;
    float* srow = p.s + ((int64_t)G0 + i) * (RP * PG) + my_row * PG;
    const int jbase = ip.y * PG;
    float rmax = -INFINITY;
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      uint4 w[2][CQ];
#pragma unroll
      for (int mm = 0; mm < 2; ++mm)
#pragma unroll
        for (int h = 0; h < CQ; ++h) w[mm][h] = lds128(kt + lane_off + (st * 8 + 4 * mm) * ROWB + h * TPK * 16);
      AbsMax16 km;
      uint32_t acc[2][RP];
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
#pragma unroll
        for (int row = 0; row < RP; ++row) acc[mm][row] = 0u;
#pragma unroll
        for (int h = 0; h < CQ; ++h) {
          km.add2(w[mm][h].x, w[mm][h].y);
          km.add2(w[mm][h].z, w[mm][h].w);
          float2 kp[4];
          unpack8<T>(w[mm][h], kp);
#pragma unroll
          for (int row = 0; row < RP; ++row)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 r2 = fma2(qr[row][h][e], kp[e], C2);
              acc[mm][row] += __float_as_uint(r2.x) + __float_as_uint(r2.y);
            }
        }
      }
      const bool fast = absmax_f32<T>(km) < kthr;
      long long dot;
      if (__all_sync(0xffffffffu, fast)) {
        uint32_t v[8];
#pragma unroll
        for (int mm = 0; mm < 2; ++mm)
#pragma unroll
          for (int row = 0; row < RP; ++row)
            v[mm * RP + row] = acc[mm][row] - (uint32_t)DPT * (uint32_t)kMagicBits;
        // sum over the 8 lanes of the key group, value kq to lane kq: each
        // lane stores its 8 partials as [value][lane] and reads its value's 8
        const uint32_t wbase = tma::smem_addr(red) + (kg * kRedGroup) * 4;
#pragma unroll
        for (int k = 0; k < 8; ++k) sts32(wbase + (k * 8 + kq) * 4, v[k]);
        __syncwarp();
        const uint4 a = lds128(wbase + (kq * 8) * 4), b = lds128(wbase + (kq * 8 + 4) * 4);
        __syncwarp();  // the buffer is rewritten by the next step
        dot = (long long)(int32_t)((a.x + a.y + a.z) + (a.w + b.x + b.y) + (b.z + b.w));  // |dot| < 2^29
      } else {
        Dots8 ex = exact_dots<D, BITS, T>(qbase, p.q_sh, kt, st * 8 + kg, kq, scale);
        reduce_scatter8_u64(ex.v, kq);
        dot = (BITS == 64) ? (long long)ex.v[0] : (long long)(int32_t)(uint32_t)ex.v[0];
      }
      // lane kq now holds (key st * 8 + my_key, row my_row)
      const int key = st * 8 + my_key;
      float qk = (BITS == 64) ? __ll2float_rn(dot) : __int2float_rn((int)dot);
      qk = __fmul_rn(__fmul_rn(qk, inv_scale), p.scale_log2);
      const float sc = jbase + key < kend ? qk : -INFINITY;
      srow[key] = sc;
      rmax = fmaxf(rmax, sc);
    }
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 4));
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 8));
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 16));
    if (lane < RP) p.m[((int64_t)G0 + i) * RP + lane] = rmax;
    __syncwarp();  // every lane is done with this page's buffer
  }
}

// ---------------------------------------------------------------------------
// kernel 2: normaliser, PV and the integer combine
// ---------------------------------------------------------------------------
// DPL V elements of a key row as fp32 after the reference's cast to fp16
// (attention.py:245-249); E16: the bf16 -> fp16 step is exact, skip it
template <typename T, int DPL, bool E16, typename R>
__device__ __forceinline__ void v_to_f32(R r, float* f) {
  uint32_t w[DPL / 2];
  if constexpr (DPL == 4) {
    w[0] = r.x;
    w[1] = r.y;
  } else {
    w[0] = r;
  }
#pragma unroll
  for (int k = 0; k < DPL / 2; ++k) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value && E16) {
      f[2 * k] = __uint_as_float(w[k] << 16);
      f[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    } else {
      const float2 t2 = v_pair_f16<T>(reinterpret_cast<const unsigned char*>(&w[k]));
      f[2 * k] = t2.x;
      f[2 * k + 1] = t2.y;
    }
  }
}

template <int DPL> struct VLoad;
template <> struct VLoad<4> {
  using R = uint2;
  __device__ static __forceinline__ R ld(uint32_t a) { return lds64(a); }
};
template <> struct VLoad<2> {
  using R = uint32_t;
  __device__ static __forceinline__ R ld(uint32_t a) { return lds32(a); }
};

// exact PV partial sums of one lane over the page's keys inside the context
// (fp16-rounded V, every product clamped and rounded on its own)
template <int D> struct PvPart {
  unsigned long long v[RP][D / 32];
};
template <int D, int BITS, typename T>
__device__ __forceinline__ PvPart<D> exact_pv(uint32_t vt, uint32_t ps, int nvalid, int d0) {
  constexpr int DPL = D / 32;
  PvPart<D> r;
#pragma unroll
  for (int row = 0; row < RP; ++row)
#pragma unroll
    for (int d = 0; d < DPL; ++d) r.v[row][d] = 0ull;
#pragma unroll 1
  for (int k = 0; k < nvalid && k < PG; ++k) {
    float vv[DPL];
    v_to_f32<T, DPL, false>(VLoad<DPL>::ld(vt + k * D * 2 + d0 * 2), vv);
#pragma unroll
    for (int row = 0; row < RP; ++row) {
      const float pv = __uint_as_float(lds32(ps + (row * PG + k) * 4));
#pragma unroll
      for (int d = 0; d < DPL; ++d)
        r.v[row][d] += (unsigned long long)(long long)f2x_scaled<BITS>(__fmul_rn(pv, vv[d]));
    }
  }
  return r;
}

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(W * 32, FXPR_DQ_MINB2)
dq_pv_kernel(const __grid_constant__ CUtensorMap vmap, const DqParams p) {
  using GE = Geo<D>;
  constexpr int ROWB = GE::ROWB, PAGEB = GE::PAGEB, DPL = GE::DPL;
  constexpr int STB = PAGEB + RP * PG * 4;  // V page + its scores
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* stage0 = smem + warp * (S * STB);
  const uint32_t stage0_a = tma::smem_addr(stage0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + W * S * STB) + warp * S;
  int* pre = reinterpret_cast<int*>(smem + W * S * STB + W * S * 8);

  build_prefix(p, pre);
  const int64_t T_ = pre[p.R];
  const int64_t nw = (int64_t)gridDim.x * W, g = (int64_t)blockIdx.x * W + warp;
  const int G0 = (int)(T_ * g / nw), G1 = (int)(T_ * (g + 1) / nw);
  const int n = G1 - G0;
  if (n <= 0) return;
  if (lane == 0) {
    for (int s = 0; s < S; ++s) tma::mbar_init(&bars[s], 1);
    tma::mbar_init_fence();
  }
  __syncwarp();
  const uint64_t pol = tma::policy_evict_first();

  Pipe pp;
  pp.A = resolve(p, pre, G0, G1);
  pp.B = resolve(p, pre, G0 + 32, G1);
  pp.a_idx = 0;
  auto issue = [&](int i) {
    const int2 c = pp.coords(i);
    if (lane == 0) {
      uint64_t* bar = &bars[i % S];
      unsigned char* dst = stage0 + (i % S) * STB;
      tma::fence_proxy_async();
      tma::mbar_expect_tx(bar, STB);
      tma::load_4d(dst, &vmap, 0, c.x & 0xFFFF, c.x >> 16, c.y, bar, pol);
      tma::load_bulk(dst + PAGEB, p.s + ((int64_t)G0 + i) * (RP * PG), RP * PG * 4, bar);
    }
  };
  for (int i = 0; i < S - 1 && i < n; ++i) issue(i);

  const float scale = ldexpf(1.0f, p.frac), inv_scale = ldexpf(1.0f, -p.frac);
  const float2 C2 = make_float2(kMagic, kMagic);
  const float2 ONE2 = make_float2(p.one, p.one);
  const double scale_d = ldexp(1.0, p.frac);
  // PV fast path iff max|v| <= 65504 and max|v| * (1 + 2^-10) * 2^f < 2^22
  const float vthr = __double2float_rd(fmin(65504.5, 4194304.0 / (scale_d * (1.0 + 1.0 / 1024))));
  const int pr = lane >> 3, pk = (lane & 7) * 2;  // p-phase: row and key pair of this lane
  const int d0 = lane * DPL;                      // pv-phase: dims of this lane

  int cur_item = -1, kend = 0, tok = 0, kvh = 0, np = 0, run = 0;
  float g_row = -INFINITY;  // max of row pr over the item
  UAcc acc[RP][DPL];
  UAcc den = 0;  // this lane's share of row pr

  // add the warp's partial sums of the current item to the output (whole
  // item) or to the item's accumulators (the last contributor finalises)
  auto flush = [&]() {
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    UAcc dn[RP];
    if (run != np) {
      unsigned long long* ga = p.acc + (int64_t)cur_item * (RP * D);
#pragma unroll
      for (int row = 0; row < RP; ++row)
#pragma unroll
        for (int d = 0; d < DPL; ++d)
          if (acc[row][d]) atomicAdd(ga + row * D + d0 + d, (unsigned long long)acc[row][d]);
      if ((lane & 7) == 0 && den) atomicAdd(p.den + (int64_t)cur_item * RP + pr, (unsigned long long)den);
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) last = (atomicAdd(p.cnt + cur_item, (unsigned)run) + (unsigned)run == (unsigned)np);
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) return;
      __threadfence();
#pragma unroll
      for (int row = 0; row < RP; ++row) {
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[row][d] = (UAcc)__ldcg(ga + row * D + d0 + d);
        dn[row] = (UAcc)__ldcg(p.den + (int64_t)cur_item * RP + row);
      }
    } else {
#pragma unroll
      for (int row = 0; row < RP; ++row) dn[row] = __shfl_sync(0xffffffffu, den, row * 8);
    }
#pragma unroll
    for (int row = 0; row < RP; ++row) {
      float df;
      if constexpr (BITS == 64) df = __fmul_rn(__ll2float_rn((long long)dn[row]), inv_scale);
      else df = __fmul_rn(__int2float_rn((int32_t)dn[row]), inv_scale);
      const float dsafe = fmaxf(df, 1.0e-6f);
      const int64_t ob = (int64_t)tok * p.o_st + (int64_t)(kvh * RP + row) * p.o_sh + d0;
#pragma unroll
      for (int d = 0; d < DPL; ++d) {
        float af;
        if constexpr (BITS == 64) af = __fmul_rn(__ll2float_rn((long long)acc[row][d]), inv_scale);
        else af = __fmul_rn(__int2float_rn((int32_t)acc[row][d]), inv_scale);
        store_f32(p.o, p.o_dtype, ob + d, prim_div(af, dsafe));
      }
    }
  };

  for (int i = 0; i < n; ++i) {
    if ((i >> 5) != pp.a_idx) pp.advance(p, pre, G0, G1);
    if (i + S - 1 < n) issue(i + S - 1);
    const int2 ip = pp.item_pg(i);
    if (ip.x != cur_item) {
      if (cur_item >= 0) flush();
      cur_item = ip.x;
      const int r = ip.x / p.KVH;
      kvh = ip.x - r * p.KVH;
      tok = p.qsl[r];
      kend = min(p.seq_lens[r], p.kmax);
      np = (pre[r + 1] - pre[r]) / p.KVH;
      run = 0;
      den = 0;
#pragma unroll
      for (int row = 0; row < RP; ++row)
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[row][d] = 0;
      // the item's row maxima: max over its pages
      const int64_t P0 = (int64_t)pre[r] + (int64_t)kvh * np;
      float gm[RP] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      for (int k = lane; k < np; k += 32) {
        const float4 mx = *reinterpret_cast<const float4*>(p.m + (P0 + k) * RP);
        gm[0] = fmaxf(gm[0], mx.x);
        gm[1] = fmaxf(gm[1], mx.y);
        gm[2] = fmaxf(gm[2], mx.z);
        gm[3] = fmaxf(gm[3], mx.w);
      }
#pragma unroll
      for (int row = 0; row < RP; ++row)
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) gm[row] = fmaxf(gm[row], __shfl_xor_sync(0xffffffffu, gm[row], o));
      g_row = pr == 0 ? gm[0] : pr == 1 ? gm[1] : pr == 2 ? gm[2] : gm[3];
    }
    if (!tma::mbar_wait(&bars[i % S], (uint32_t)((i / S) & 1))) {
      if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
      drain(bars, i, n);
      cur_item = -1;  // no output for a page that never landed
      break;
    }
    ++run;
    const uint32_t vt = stage0_a + (i % S) * STB;
    const uint32_t ps = vt + PAGEB;  // [RP][PG] score -> p * 2^f
    const int jbase = ip.y * PG;
    // ---- p = exp2(score - max) for keys inside the context (attention.py:237-243) ----
    {
      const uint32_t a = ps + (pr * PG + pk) * 4;
      const uint2 sc = lds64(a);
      const int j = jbase + pk;
      const float p0 = j < kend ? prim_exp2(__fsub_rn(__uint_as_float(sc.x), g_row)) : 0.0f;
      const float p1 = j + 1 < kend ? prim_exp2(__fsub_rn(__uint_as_float(sc.y), g_row)) : 0.0f;
      den += (UAcc)f2x_f32<BITS>(p0, scale) + (UAcc)f2x_f32<BITS>(p1, scale);
      sts64f(a, __fmul_rn(p0, scale), __fmul_rn(p1, scale));
    }
    __syncwarp();
    // ---- PV (attention.py:245-255): acc[row][d] += F2X(p * fp16(v)) ----
    uint32_t tv[RP][DPL];
#pragma unroll
    for (int row = 0; row < RP; ++row)
#pragma unroll
      for (int d = 0; d < DPL; ++d) tv[row][d] = 0u;
    AbsMax16 vm;
    const uint32_t vlane = vt + d0 * 2;
    auto pv_page = [&](auto e16) {
#pragma unroll
      for (int k4 = 0; k4 < PG; k4 += 4) {
        float4 p4[RP];
#pragma unroll
        for (int row = 0; row < RP; ++row) p4[row] = lds128f(ps + (row * PG + k4) * 4);
#pragma unroll
        for (int h2 = 0; h2 < 4; h2 += 2) {
          const auto ra = VLoad<DPL>::ld(vlane + (k4 + h2) * ROWB);
          const auto rb = VLoad<DPL>::ld(vlane + (k4 + h2 + 1) * ROWB);
          if constexpr (DPL == 4) {
            vm.add2(ra.x, ra.y);
            vm.add2(rb.x, rb.y);
          } else {
            vm.add2(ra, rb);
          }
          float va[DPL], vb[DPL];
          v_to_f32<T, DPL, decltype(e16)::value>(ra, va);
          v_to_f32<T, DPL, decltype(e16)::value>(rb, vb);
#pragma unroll
          for (int row = 0; row < RP; ++row) {
            const float2 pq = h2 == 0 ? make_float2(p4[row].x, p4[row].y) : make_float2(p4[row].z, p4[row].w);
#pragma unroll
            for (int d = 0; d < DPL; ++d) {
              const float2 r2 = fma2(mul2(pq, make_float2(va[d], vb[d])), ONE2, C2);
              tv[row][d] += __float_as_uint(r2.x) + __float_as_uint(r2.y);
            }
          }
        }
      }
    };
    if (p.v_exact16) pv_page(std::true_type{});
    else pv_page(std::false_type{});
    const bool fast = absmax_f32<T>(vm) < vthr;
    if (__all_sync(0xffffffffu, fast)) {
#pragma unroll
      for (int row = 0; row < RP; ++row)
#pragma unroll
        for (int d = 0; d < DPL; ++d)
          acc[row][d] += (UAcc)(long long)(int32_t)(tv[row][d] - (uint32_t)PG * (uint32_t)kMagicBits);
    } else {
      const PvPart<D> ex = exact_pv<D, BITS, T>(vt, ps, kend - jbase, d0);
#pragma unroll
      for (int row = 0; row < RP; ++row)
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[row][d] += (UAcc)ex.v[row][d];
    }
    __syncwarp();  // every lane is done with this page's buffer
  }
  if (cur_item >= 0) flush();
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int D>
static size_t smem1(int R) {
  return (size_t)W * S * Geo<D>::PAGEB + W * S * 8 + (size_t)W * kRedWords * 4 + (size_t)(R + 1) * 4;
}
template <int D>
static size_t smem2(int R) {
  return (size_t)W * S * (Geo<D>::PAGEB + RP * PG * 4) + W * S * 8 + (size_t)(R + 1) * 4;
}

struct KernelCfg {
  bool configured[64];
  int ctas_per_sm[64];
};

template <typename K>
static int persistent_grid(K kernel, size_t smem, KernelCfg& cfg, int* grid) {
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cache = dev >= 0 && dev < 64;
  if (!cache || !cfg.configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
        cudaSuccess) {
      set_error("unified_attention_fxp: cannot configure shared memory (decode path)");
      return FXPR_ERR_CUDA;
    }
    if (cache) cfg.configured[dev] = true;
  }
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, W * 32, smem) != cudaSuccess ||
      per < 1)
    per = 1;
  *grid = num_sms() * per;
  return FXPR_OK;
}

template <int D, int BITS, typename T>
static int launch_t(const DqParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                    cudaStream_t st) {
  static KernelCfg c1 = {}, c2 = {};
  auto k1 = dq_scores_kernel<D, BITS, T>;
  auto k2 = dq_pv_kernel<D, BITS, T>;
  const size_t s1 = smem1<D>(p.R), s2 = smem2<D>(p.R);
  int g1 = 0, g2 = 0;
  int rc = persistent_grid(k1, s1, c1, &g1);
  if (rc != FXPR_OK) return rc;
  rc = persistent_grid(k2, s2, c2, &g2);
  if (rc != FXPR_OK) return rc;
  k1<<<g1, W * 32, s1, st>>>(kmap, p);
  rc = check_launch("fxpr_unified_attention_fxp (decode scores)");
  if (rc != FXPR_OK) return rc;
  k2<<<g2, W * 32, s2, st>>>(vmap, p);
  return check_launch("fxpr_unified_attention_fxp (decode pv)");
}

}  // namespace dq

int64_t decode_workspace_bytes(int items, int kmax, int D) {
  const int64_t pages = (int64_t)items * ((kmax + dq::PG - 1) / dq::PG);
  auto a256 = [](int64_t x) { return (x + 255) / 256 * 256; };
  int64_t off = 256;                                   // error word
  off = a256(off + (int64_t)items * 4);                // cnt
  off = a256(off + (int64_t)items * dq::RP * 8);       // den
  off = a256(off + (int64_t)items * dq::RP * D * 8);   // acc
  off = a256(off + pages * dq::RP * 4);                // m
  off = a256(off + pages * dq::RP * dq::PG * 4);       // s
  return off;
}

bool decode_supported(const fxpr_attention_params* a, int G) {
  if (a->max_query_len != 1 || G != dq::RP) return false;
  if (a->head_dim != 64 && a->head_dim != 128) return false;
  if (a->kv_dtype != FXPR_BF16 && a->kv_dtype != FXPR_F16) return false;
  if (a->q_dtype != a->kv_dtype) return false;
  if (a->num_blocks <= 0 || a->page_size % dq::PG != 0) return false;
  if (a->logits_soft_cap > 0.0f || a->alibi_slopes != nullptr || a->window_size > 0) return false;
  if (a->num_requests > dq::MAX_REQ) return false;
  if ((uintptr_t)a->q % 16 != 0 || a->q_stride_tok % 8 != 0 || a->q_stride_head % 8 != 0) return false;
  return true;
}

int launch_decode(const fxpr_attention_params* a, int kmax, void* workspace, cudaStream_t st) {
  using namespace dq;
  const int D = a->head_dim;
  const int items = a->num_requests * a->num_kv_heads;
  const int64_t pages = (int64_t)items * ((kmax + PG - 1) / PG);
  if (pages > 0x7fffffffLL) {
    set_error("unified_attention_fxp: too many pages for the decode path");
    return FXPR_ERR_UNSUPPORTED;
  }
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  auto a256 = [](int64_t x) { return (x + 255) / 256 * 256; };
  DqParams p = {};
  int64_t off = 256;
  p.err = reinterpret_cast<uint32_t*>(ws);
  p.cnt = reinterpret_cast<uint32_t*>(ws + off);
  off = a256(off + (int64_t)items * 4);
  p.den = reinterpret_cast<unsigned long long*>(ws + off);
  off = a256(off + (int64_t)items * RP * 8);
  p.acc = reinterpret_cast<unsigned long long*>(ws + off);
  off = a256(off + (int64_t)items * RP * D * 8);
  p.m = reinterpret_cast<float*>(ws + off);
  off = a256(off + pages * RP * 4);
  p.s = reinterpret_cast<float*>(ws + off);
  p.q = a->q; p.q_st = a->q_stride_tok; p.q_sh = a->q_stride_head;
  p.o = a->o; p.o_dtype = a->o_dtype; p.o_st = a->o_stride_tok; p.o_sh = a->o_stride_head;
  p.qsl = a->query_start_loc; p.seq_lens = a->seq_lens; p.bt = a->block_table;
  p.bt_stride = a->bt_stride;
  p.R = a->num_requests; p.KVH = a->num_kv_heads; p.page = a->page_size;
  p.page_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1 << sh) == a->page_size) p.page_shift = sh;
  p.kmax = kmax;
  p.scale_log2 = a->scale_log2;
  p.frac = a->frac_bits;
  p.one = 1.0f;
  p.v_exact16 = (a->kv_dtype == FXPR_BF16 && a->frac_bits <= 16) ? 1 : 0;

  // tensor maps: (head_dim, kv head, slot, block) over each cache, one page box
  CUtensorMap kmap, vmap;
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a->num_kv_heads, (uint64_t)a->page_size,
                            (uint64_t)a->num_blocks};
  const uint32_t box[4] = {(uint32_t)D, 1u, (uint32_t)PG, 1u};
  const uint64_t ks[3] = {(uint64_t)a->k_stride_head * 2, (uint64_t)a->k_stride_slot * 2,
                          (uint64_t)a->k_stride_blk * 2};
  const uint64_t vs[3] = {(uint64_t)a->v_stride_head * 2, (uint64_t)a->v_stride_slot * 2,
                          (uint64_t)a->v_stride_blk * 2};
  if (!tma::encode_4d_u16(&kmap, a->k_cache, dims, ks, box) ||
      !tma::encode_4d_u16(&vmap, a->v_cache, dims, vs, box))
    return FXPR_ERR_CUDA;
  if (cudaMemsetAsync(ws, 0, 4, st) != cudaSuccess) {
    set_error("unified_attention_fxp: clearing the error word failed");
    return FXPR_ERR_CUDA;
  }
  const bool bf = a->kv_dtype == FXPR_BF16;
  if (D == 128) {
    if (a->int_bits == 32) return bf ? launch_t<128, 32, __nv_bfloat16>(p, kmap, vmap, st)
                                     : launch_t<128, 32, __half>(p, kmap, vmap, st);
    return bf ? launch_t<128, 64, __nv_bfloat16>(p, kmap, vmap, st)
              : launch_t<128, 64, __half>(p, kmap, vmap, st);
  }
  if (a->int_bits == 32) return bf ? launch_t<64, 32, __nv_bfloat16>(p, kmap, vmap, st)
                                   : launch_t<64, 32, __half>(p, kmap, vmap, st);
  return bf ? launch_t<64, 64, __nv_bfloat16>(p, kmap, vmap, st)
            : launch_t<64, 64, __half>(p, kmap, vmap, st);
}

}  // namespace attn
}  // namespace fxpr
