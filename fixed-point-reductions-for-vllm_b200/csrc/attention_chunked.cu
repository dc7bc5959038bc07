// Paged unified attention with fixed-point softmax (attention.py:18-489) as
// two streaming kernels over fixed chunks of CHUNK keys.
//
// Work unit = (chunk of keys, KV head (slice of its query-head group),
// request, tile of queries); rows are the (query, head) pairs of the unit
// that share one KV head. Every unit has the same size, so the grid balances
// over the SMs whatever the spread of context lengths, and a unit is short
// enough that several are resident per SM and hide each other's start-up.
//
//   scores  K tiles -> integer q.k -> fp32 score (X2F, scale, softcap,
//           alibi, masks), written to a scratch [rows][CHUNK], and the
//           unit's row maxima.
//   pv      global row max = max over the item's chunk maxima (the
//           reference's whole-context pass-1 max); p = exp2(score - max),
//           integer normaliser and integer PV partial sums over V tiles,
//           added into per-item integer accumulators (exact, order-free).
//           The last unit of an item (ticket counter) converts, divides and
//           stores. The scores kernel's first unit of an item clears them.
// Scores add 2 x 4 bytes per (row, key) of traffic to the 2 x D x 2 bytes
// of K and V per key (about 3% for D = 128 bf16, 4 rows).
#include "attention_common.cuh"

namespace fxpr {
namespace attn {

// tile buffers of the two kernels (NBS - 1, NBP - 1 tiles in flight per CTA)
#ifndef FXPR_ACH_NBS
#define FXPR_ACH_NBS 3
#endif
#ifndef FXPR_ACH_NBP
#define FXPR_ACH_NBP 3
#endif
constexpr int NBS = FXPR_ACH_NBS;
constexpr int NBP = FXPR_ACH_NBP;

// keys per tile of the decode scores kernel (the PV kernel and the general
// scores kernel use KT)
#ifndef FXPR_ACH_KT
#define FXPR_ACH_KT 128
#endif
constexpr int KTC = FXPR_ACH_KT;
static_assert(CHUNK % KTC == 0 && CHUNK % KT == 0, "chunk of whole tiles");

template <int D, typename KVT, int NK = KT>
struct Tile {
  static constexpr int ROWB = D * (int)sizeof(KVT);  // bytes of one key row
  static constexpr int NC = ROWB / 16;               // 16-byte chunks per key row
  static constexpr int SWZ = (NC < 8 ? NC : 8) - 1;  // chunk swizzle mask
  static constexpr int TILEB = NK * ROWB;
  static constexpr int TPK = THREADS / NK;  // threads per key row in the copies
  static constexpr int CPT = NC / TPK;      // 16-byte chunks copied per thread
};

template <int D, int RP, typename KVT, int NK = KT>
struct ScoreSmem {
  static constexpr size_t off_q = 0;
  static constexpr size_t off_qraw = off_q + (size_t)RP * D * 4;
  static constexpr size_t off_kv = off_qraw + (size_t)RP * D * 4;
  static constexpr size_t bytes = off_kv + (size_t)NBS * Tile<D, KVT, NK>::TILEB;
};
template <int D, int RP, typename KVT>
struct PvSmem {
  static constexpr size_t off_p = 0;  // [RP][CHUNK] scores, then p * 2^f
  static constexpr size_t off_kv = off_p + (size_t)RP * CHUNK * 4;
  static constexpr size_t bytes = off_kv + (size_t)NBP * Tile<D, KVT>::TILEB;
};

// Rows of a unit (attention.py:319-353). Returns the key limit over its rows
// (the reference walks keys to the end of its 64-row query block), or -1 if
// the query tile is empty.
template <int RP>
__device__ __forceinline__ int unit_rows(const Params& p, int req, int qtile, int kvh, int hslice,
                                         int* row_tok, int* row_head, int* row_pos, int* row_kend) {
  const int t = threadIdx.x;
  const int q_start = p.qsl[req], q_end = p.qsl[req + 1];
  const int qlen = q_end - q_start;
  if (qtile * p.qt >= qlen) return -1;
  const int seq_len = p.seq_lens[req];
  const int ctx = seq_len - qlen;
  if (t < RP) {
    const int qi = t / p.gs, gh = t % p.gs;
    const int qoff = qtile * p.qt + qi;
    const int hg = hslice * p.gs + gh;
    int tok = -1, kend = 0, pos = 0, head = 0;
    if (qi < p.qt && qoff < qlen && hg < p.group) {
      tok = q_start + qoff;
      head = kvh * p.group + hg;
      pos = ctx + qoff;
      kend = p.causal ? min(seq_len, ctx + (qoff / 64 + 1) * 64) : seq_len;
    }
    row_tok[t] = tok;
    row_head[t] = head;
    row_pos[t] = pos;
    row_kend[t] = kend;
  }
  __syncthreads();
  int kr_hi = 0;
#pragma unroll
  for (int i = 0; i < RP; ++i) kr_hi = max(kr_hi, row_kend[i]);
  return kr_hi;
}

// Copies of one K or V tile: each thread copies CPT consecutive 16-byte
// chunks of one key row, XOR-swizzled in shared memory.
template <int D, typename KVT, int NK = KT>
struct TileCopier {
  using TL = Tile<D, KVT, NK>;
  const Params& p;
  int64_t bt_row;
  int kb, ke, kvh, my_jl, c0;
  __device__ TileCopier(const Params& p_, int req, int kb_, int ke_, int kvh_)
      : p(p_), bt_row((int64_t)req * p_.bt_stride), kb(kb_), ke(ke_), kvh(kvh_) {
    my_jl = threadIdx.x / TL::TPK;
    c0 = (threadIdx.x % TL::TPK) * TL::CPT;
  }
  __device__ __forceinline__ int block_of(int ti) const {
    const int j = kb + ti * NK + my_jl;
    if (j >= ke) return -1;
    const int bi = p.page_shift >= 0 ? (j >> p.page_shift) : j / p.page;
    return p.bt[bt_row + bi];
  }
  __device__ __forceinline__ void issue(const void* base, int64_t sb, int64_t ss, int64_t sh,
                                        int ti, unsigned char* dst_tile, int blk) const {
    const int j = kb + ti * NK + my_jl;
    unsigned char* dst = dst_tile + my_jl * TL::ROWB;
    const unsigned char* src = reinterpret_cast<const unsigned char*>(base);
    int bytes = 0;
    if (blk >= 0) {
      const int slot = p.page_shift >= 0 ? (j & (p.page - 1)) : j % p.page;
      src += ((int64_t)blk * sb + (int64_t)slot * ss + (int64_t)kvh * sh) * (int64_t)sizeof(KVT);
      bytes = 16;
    }
#pragma unroll
    for (int u = 0; u < TL::CPT; ++u) {
      const int c = c0 + u;
      cp_async16(dst + ((c ^ (my_jl & TL::SWZ)) * 16), src + c * 16, bytes);
    }
  }
};

// The PV kernel (next on the stream) combines an item of several chunks in
// global integer accumulators: the item's chunk-0 scores unit clears them,
// so the workspace needs no state between calls.
template <int RP, int D>
__device__ __forceinline__ void clear_item(const Params& p, int64_t item, int chunk, int kr_hi) {
  if (chunk != 0 || kr_hi <= CHUNK) return;
  const int t = threadIdx.x;
  for (int e = t; e < RP * D; e += THREADS) p.ws_acc[item * (RP * D) + e] = 0ull;
  if (t < RP) p.ws_den[item * RP + t] = 0ull;
  if (t == 0) p.ws_cnt[item] = 0u;
}

// q of the rows (pre-scaled by 2^f and raw) into shared memory; max |q| into
// *q_or. Returns the K magnitude threshold of the fast path:
// max|q| * max|k| * 2^f < 2^22 (strict, rounded down).
template <int RP, int D>
__device__ __forceinline__ float stage_q(const Params& p, const int* row_tok, const int* row_head,
                                         float* q_s, float* q_raw, uint32_t* q_or, float scale) {
  const int t = threadIdx.x;
  uint32_t qo = 0;
  for (int e = t; e < RP * D; e += THREADS) {
    const int i = e / D, d = e % D;
    float v = 0.0f;
    if (row_tok[i] >= 0)
      v = load_f32(p.q, p.q_dtype, (int64_t)row_tok[i] * p.q_st + (int64_t)row_head[i] * p.q_sh + d);
    q_raw[e] = v;
    q_s[e] = __fmul_rn(v, scale);
    qo = max(qo, __float_as_uint(v) & 0x7FFFFFFFu);
  }
  qo = __reduce_max_sync(0xffffffffu, qo);
  if ((t & 31) == 0) atomicMax(q_or, qo);
  __syncthreads();
  const double scale_d = ldexp(1.0, p.frac);
  const double mq = (double)__uint_as_float(*q_or);
  const bool q_ok = mq * scale_d < 3.0e38;  // q * 2^f finite (NaN: false)
  return q_ok ? __double2float_rd(4194304.0 / (mq * scale_d)) : 0.0f;
}

// fp32 score of (row i, key j) from the integer dot (attention.py:119-148);
// -inf when masked. PL: no softcap, ALiBi or sliding window (checked by the
// host), so those steps are compiled out.
template <int BITS, bool PL>
__device__ __forceinline__ float score_of(const Params& p, long long di, int j, int kend, int pos,
                                          int head, float inv_scale) {
  float qk = (BITS == 64) ? __ll2float_rn(di) : __int2float_rn((int)di);
  qk = __fmul_rn(__fmul_rn(qk, inv_scale), p.scale_log2);
  bool ok = j < kend;
  if constexpr (!PL) {
    if (p.softcap_log2 > 0.0f) qk = __fmul_rn(p.softcap_log2, prim_tanh(__fmul_rn(qk, p.softcap_rcp)));
    if (p.alibi) qk = __fmaf_rn(p.alibi[head], __fsub_rn((float)j, (float)pos), qk);  // contracted, as Triton lowers it
    if (p.window > 0) ok = ok && (j > pos - p.window);
  }
  if (p.causal) ok = ok && (pos >= j);
  return ok ? qk : -INFINITY;
}

// ---------------------------------------------------------------------------
// kernel 1 (general shapes): scores and chunk row maxima. Four threads share
// a key (each a quarter of its dims), q read from shared memory.
// ---------------------------------------------------------------------------
template <int D, int RP, int BITS, typename KVT, bool PL>
__global__ void __launch_bounds__(THREADS) chunk_scores_kernel(Params p) {
  using TL = Tile<D, KVT>;
  using SM = ScoreSmem<D, RP, KVT>;
  constexpr int ROWB = TL::ROWB, NC = TL::NC, SWZ = TL::SWZ, TILEB = TL::TILEB;
  constexpr int CE = Chunk<KVT>::E;
  constexpr int RPT = RP / 4;
  constexpr int RG = RP < 4 ? RP : 4;
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  static_assert(NC % 4 == 0 && NC % TL::TPK == 0, "head_dim too small for the chunk mapping");

  extern __shared__ __align__(16) unsigned char smem[];
  float* q_s = reinterpret_cast<float*>(smem + SM::off_q);
  float* q_raw = reinterpret_cast<float*>(smem + SM::off_qraw);
  unsigned char* kvbuf = smem + SM::off_kv;
  __shared__ int row_tok[RP], row_head[RP], row_pos[RP], row_kend[RP];
  __shared__ uint32_t q_or;
  __shared__ float wmax[THREADS / 32][RP];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int chunk = blockIdx.x;
  const int kvh = blockIdx.y / p.head_slices, hslice = blockIdx.y % p.head_slices;
  const int req = blockIdx.z / p.qtiles, qtile = blockIdx.z % p.qtiles;
  if (t == 0) q_or = 0u;
  const int kr_hi = unit_rows<RP>(p, req, qtile, kvh, hslice, row_tok, row_head, row_pos, row_kend);
  const int kb = chunk * CHUNK;
  if (kr_hi < 0 || (chunk > 0 && kb >= kr_hi)) return;  // uniform over the CTA
  const int ke = min(kb + CHUNK, kr_hi);
  const int ntiles = (ke - kb + KT - 1) / KT;
  const int64_t item = (int64_t)blockIdx.z * gridDim.y + blockIdx.y;
  const int64_t unit = item * p.nchunk_max + chunk;
  const float scale = ldexpf(1.0f, p.frac);
  const float inv_scale = ldexpf(1.0f, -p.frac);

  TileCopier<D, KVT> cp(p, req, kb, ke, kvh);
#pragma unroll
  for (int s0 = 0; s0 < NBS - 1; ++s0) {
    if (s0 < ntiles)
      cp.issue(p.k, p.k_sb, p.k_ss, p.k_sh, s0, kvbuf + s0 * TILEB, cp.block_of(s0));
    cp_async_commit();
  }
  int next_blk = (NBS - 1 < ntiles) ? cp.block_of(NBS - 1) : -1;
  clear_item<RP, D>(p, item, chunk, kr_hi);
  const float kthr = stage_q<RP, D>(p, row_tok, row_head, q_s, q_raw, &q_or, scale);

  float* sdst = p.ws_s + unit * (RP * CHUNK);
  float rmax[RPT];
#pragma unroll
  for (int u = 0; u < RPT; ++u) rmax[u] = -INFINITY;
  const float2 C2 = make_float2(kMagic, kMagic);
  const float2 ONE2 = make_float2(p.one, p.one);
  const int jl = t >> 2, dq = t & 3;

  for (int ti = 0; ti < ntiles; ++ti) {
    cp_async_wait<NBS - 2>();
    __syncthreads();  // tile ti visible to all; buffer (ti+NBS-1)%NBS free
    if (ti + NBS - 1 < ntiles) {
      cp.issue(p.k, p.k_sb, p.k_ss, p.k_sh, ti + NBS - 1,
               kvbuf + ((ti + NBS - 1) % NBS) * TILEB, next_blk);
      next_blk = (ti + NBS < ntiles) ? cp.block_of(ti + NBS) : -1;
    }
    cp_async_commit();

    // ---- integer q.k of this thread's quarter of key jl (attention.py:80-118) ----
    const unsigned char* kt = kvbuf + (ti % NBS) * TILEB;
    const int j = kb + ti * KT + jl;
    uint32_t acc[RP];
#pragma unroll
    for (int i = 0; i < RP; ++i) acc[i] = 0u;
    uint32_t km = 0;
    auto body = [&](auto exact) {
#pragma unroll
      for (int rr = 0; rr < NC / 4; ++rr) {
        const int c = rr * 4 + dq;
        const uint4 w = *reinterpret_cast<const uint4*>(kt + jl * ROWB + ((c ^ (jl & SWZ)) * 16));
        absmax_word<KVT>(km, w.x);
        absmax_word<KVT>(km, w.y);
        absmax_word<KVT>(km, w.z);
        absmax_word<KVT>(km, w.w);
        float2 kp[CE / 2];
        Chunk<KVT>::unpack(w, kp);
#pragma unroll
        for (int ig = 0; ig < RP; ig += RG) {
          float4 qv[RG][CE / 4];
#pragma unroll
          for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int e = 0; e < CE / 4; ++e)
              qv[r][e] = *reinterpret_cast<const float4*>(q_s + (ig + r) * D + c * CE + 4 * e);
#pragma unroll
          for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int e = 0; e < CE / 4; ++e) {
              float2 r0, r1;
              if constexpr (decltype(exact)::value) {
                r0 = fma2(make_float2(qv[r][e].x, qv[r][e].y), kp[2 * e], C2);
                r1 = fma2(make_float2(qv[r][e].z, qv[r][e].w), kp[2 * e + 1], C2);
              } else {
                r0 = fma2(mul2(make_float2(qv[r][e].x, qv[r][e].y), kp[2 * e]), ONE2, C2);
                r1 = fma2(mul2(make_float2(qv[r][e].z, qv[r][e].w), kp[2 * e + 1]), ONE2, C2);
              }
              acc[ig + r] += __float_as_uint(r0.x) + __float_as_uint(r0.y);
              acc[ig + r] += __float_as_uint(r1.x) + __float_as_uint(r1.y);
            }
        }
      }
    };
    if (p.exact_qk) body(std::true_type{});
    else body(std::false_type{});
    long long dot[RP];
    if (absmax_value<KVT>(km) < kthr) {
#pragma unroll
      for (int i = 0; i < RP; ++i) {
        acc[i] -= (uint32_t)(D / 4) * (uint32_t)kMagicBits;
        dot[i] = (BITS == 64) ? (long long)(int32_t)acc[i] : (long long)acc[i];
      }
    } else {
      // values the magic constant cannot round exactly: the exact path
      UAcc ex[RP];
#pragma unroll
      for (int i = 0; i < RP; ++i) ex[i] = 0;
      for (int rr = 0; rr < NC / 4; ++rr) {
        const int c = rr * 4 + dq;
        const KVT* kv = reinterpret_cast<const KVT*>(kt + jl * ROWB + ((c ^ (jl & SWZ)) * 16));
        for (int e = 0; e < CE; ++e) {
          const float kf = to_f32(kv[e]);
#pragma unroll
          for (int i = 0; i < RP; ++i)
            ex[i] += (UAcc)f2x_f32<BITS>(__fmul_rn(q_raw[i * D + c * CE + e], kf), scale);
        }
      }
#pragma unroll
      for (int i = 0; i < RP; ++i) dot[i] = (long long)ex[i];
    }
#pragma unroll
    for (int i = 0; i < RP; ++i) {
      if constexpr (BITS == 64) {
        dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], 1);
        dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], 2);
      } else {
        uint32_t v = (uint32_t)dot[i];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        dot[i] = (long long)(int32_t)v;
      }
    }
    if (j < ke) {
#pragma unroll
      for (int u = 0; u < RPT; ++u) {
        const int i = dq + 4 * u;
        long long di = dot[4 * u];  // dot[i] without runtime register indexing
#pragma unroll
        for (int w = 1; w < 4; ++w)
          if (dq == w) di = dot[4 * u + w];
        const float s = score_of<BITS, PL>(p, di, j, row_kend[i], row_pos[i], row_head[i], inv_scale);
        sdst[i * CHUNK + (j - kb)] = s;
        rmax[u] = fmaxf(rmax[u], s);
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int u = 0; u < RPT; ++u) {
    float m = rmax[u];
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    if (lane < 4) wmax[warp][lane + 4 * u] = m;
  }
  __syncthreads();
  if (t < RP) {
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) m = fmaxf(m, wmax[w][t]);
    p.ws_m[unit * RP + t] = m;
  }
}

// ---------------------------------------------------------------------------
// kernel 1, decode shapes (4 rows, head_dim 64/128): q held in registers.
// 8 threads share a key, each owning D/8 of its dims (chunks kq, kq+8, ...),
// and take 2 keys per tile, so every K element is read from shared memory
// once and q never is; the 8 partial dots of (2 keys x 4 rows) are
// reduce-scattered over the 8 lanes, one score per lane.
// ---------------------------------------------------------------------------
template <int D, int BITS, typename KVT, bool PL>
__global__ void __launch_bounds__(THREADS, 2) chunk_scores_rq_kernel(Params p) {
  constexpr int RP = 4;
  using TL = Tile<D, KVT, KTC>;
  using SM = ScoreSmem<D, RP, KVT, KTC>;
  constexpr int ROWB = TL::ROWB, NC = TL::NC, SWZ = TL::SWZ, TILEB = TL::TILEB;
  constexpr int CE = Chunk<KVT>::E;
  constexpr int TPQ = 8;                // threads per key
  constexpr int KSTEP = THREADS / TPQ;  // keys per step (32)
  constexpr int KM = KTC / KSTEP;       // keys per thread per tile
  constexpr int CQ = NC / TPQ;          // 16-byte chunks per thread per key
  constexpr int DPT = CQ * CE;          // dims per thread
  constexpr int NV = KM * RP;           // partial dots per lane
  constexpr int VPL = NV / TPQ;         // scores per lane after the reduce-scatter
  static_assert(NC % TPQ == 0 && NV % TPQ == 0 && RP % VPL == 0, "rq mapping");

  extern __shared__ __align__(16) unsigned char smem[];
  float* q_s = reinterpret_cast<float*>(smem + SM::off_q);
  float* q_raw = reinterpret_cast<float*>(smem + SM::off_qraw);
  unsigned char* kvbuf = smem + SM::off_kv;
  __shared__ int row_tok[RP], row_head[RP], row_pos[RP], row_kend[RP];
  __shared__ uint32_t q_or;
  __shared__ float wmax[THREADS / 32][RP];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int kq = t & (TPQ - 1), kl = t / TPQ;
  const int chunk = blockIdx.x;
  const int kvh = blockIdx.y / p.head_slices, hslice = blockIdx.y % p.head_slices;
  const int req = blockIdx.z / p.qtiles, qtile = blockIdx.z % p.qtiles;
  if (t == 0) q_or = 0u;
  const int kr_hi = unit_rows<RP>(p, req, qtile, kvh, hslice, row_tok, row_head, row_pos, row_kend);
  const int kb = chunk * CHUNK;
  if (kr_hi < 0 || (chunk > 0 && kb >= kr_hi)) return;  // uniform over the CTA
  const int ke = min(kb + CHUNK, kr_hi);
  const int ntiles = (ke - kb + KTC - 1) / KTC;
  const int64_t item = (int64_t)blockIdx.z * gridDim.y + blockIdx.y;
  const int64_t unit = item * p.nchunk_max + chunk;
  const float scale = ldexpf(1.0f, p.frac);
  const float inv_scale = ldexpf(1.0f, -p.frac);

  TileCopier<D, KVT, KTC> cp(p, req, kb, ke, kvh);
#pragma unroll
  for (int s0 = 0; s0 < NBS - 1; ++s0) {
    if (s0 < ntiles)
      cp.issue(p.k, p.k_sb, p.k_ss, p.k_sh, s0, kvbuf + s0 * TILEB, cp.block_of(s0));
    cp_async_commit();
  }
  int next_blk = (NBS - 1 < ntiles) ? cp.block_of(NBS - 1) : -1;
  clear_item<RP, D>(p, item, chunk, kr_hi);
  const float kthr = stage_q<RP, D>(p, row_tok, row_head, q_s, q_raw, &q_or, scale);

  // this thread's q (pre-scaled), as fp32 pairs
  float2 qr[RP][DPT / 2];
#pragma unroll
  for (int i = 0; i < RP; ++i)
#pragma unroll
    for (int h = 0; h < CQ; ++h)
#pragma unroll
      for (int e = 0; e < CE; e += 2)
        qr[i][(h * CE + e) / 2] =
            *reinterpret_cast<const float2*>(q_s + i * D + (kq + TPQ * h) * CE + e);

  float* sdst = p.ws_s + unit * (RP * CHUNK);
  // after the reduce-scatter lane kq holds partial-dot indices VPL*kq + e,
  // index = m * RP + i: one key step my_m, rows my_i0 + e
  const int my_m = (VPL * kq) / RP, my_i0 = (VPL * kq) % RP;
  float rmax[VPL];
#pragma unroll
  for (int e = 0; e < VPL; ++e) rmax[e] = -INFINITY;
  const float2 C2 = make_float2(kMagic, kMagic);
  const float2 ONE2 = make_float2(p.one, p.one);

  for (int ti = 0; ti < ntiles; ++ti) {
    cp_async_wait<NBS - 2>();
    __syncthreads();  // tile ti visible to all; buffer (ti+NBS-1)%NBS free
    if (ti + NBS - 1 < ntiles) {
      cp.issue(p.k, p.k_sb, p.k_ss, p.k_sh, ti + NBS - 1,
               kvbuf + ((ti + NBS - 1) % NBS) * TILEB, next_blk);
      next_blk = (ti + NBS < ntiles) ? cp.block_of(ti + NBS) : -1;
    }
    cp_async_commit();

    const unsigned char* kt = kvbuf + (ti % NBS) * TILEB;
    uint4 w[KM][CQ];
#pragma unroll
    for (int m = 0; m < KM; ++m) {
      const int jl = kl + KSTEP * m;
#pragma unroll
      for (int h = 0; h < CQ; ++h)
        w[m][h] = *reinterpret_cast<const uint4*>(kt + jl * ROWB + (((kq + TPQ * h) ^ (jl & SWZ)) * 16));
    }
    uint32_t km = 0;
    uint32_t acc[KM][RP];
#pragma unroll
    for (int m = 0; m < KM; ++m)
#pragma unroll
      for (int i = 0; i < RP; ++i) acc[m][i] = 0u;
    auto body = [&](auto exact) {
#pragma unroll
      for (int m = 0; m < KM; ++m)
#pragma unroll
        for (int h = 0; h < CQ; ++h) {
          absmax_word<KVT>(km, w[m][h].x);
          absmax_word<KVT>(km, w[m][h].y);
          absmax_word<KVT>(km, w[m][h].z);
          absmax_word<KVT>(km, w[m][h].w);
          float2 kp[CE / 2];
          Chunk<KVT>::unpack(w[m][h], kp);
#pragma unroll
          for (int i = 0; i < RP; ++i)
#pragma unroll
            for (int e = 0; e < CE / 2; ++e) {
              float2 r;
              if constexpr (decltype(exact)::value) {
                r = fma2(qr[i][h * CE / 2 + e], kp[e], C2);
              } else {
                r = fma2(mul2(qr[i][h * CE / 2 + e], kp[e]), ONE2, C2);
              }
              acc[m][i] += __float_as_uint(r.x) + __float_as_uint(r.y);
            }
        }
    };
    if (p.exact_qk) body(std::true_type{});
    else body(std::false_type{});
    const bool fast = absmax_value<KVT>(km) < kthr;
    // 8 partial dots per lane, value index v = m * 4 + i; the reduce-scatter
    // over the 8 lanes of the key group leaves value kq on lane kq
    long long val[VPL];
    if (BITS == 32 || __all_sync(0xffffffffu, fast)) {
      uint32_t v[NV];
#pragma unroll
      for (int m = 0; m < KM; ++m)
#pragma unroll
        for (int i = 0; i < RP; ++i) v[m * RP + i] = acc[m][i] - (uint32_t)DPT * (uint32_t)kMagicBits;
      if (!__all_sync(0xffffffffu, fast) && !fast) {  // BITS == 32 here: exact path, wrapping sums
#pragma unroll
        for (int m = 0; m < KM; ++m) {
          const int jl = kl + KSTEP * m;
          uint32_t ex[RP];
#pragma unroll
          for (int i = 0; i < RP; ++i) ex[i] = 0u;
          for (int h = 0; h < CQ; ++h) {
            const int c = kq + TPQ * h;
            const KVT* kv = reinterpret_cast<const KVT*>(kt + jl * ROWB + ((c ^ (jl & SWZ)) * 16));
            for (int e = 0; e < CE; ++e) {
              const float kf = to_f32(kv[e]);
#pragma unroll
              for (int i = 0; i < RP; ++i)
                ex[i] += (uint32_t)f2x_f32<BITS>(__fmul_rn(q_raw[i * D + c * CE + e], kf), scale);
            }
          }
#pragma unroll
          for (int i = 0; i < RP; ++i) v[m * RP + i] = ex[i];
        }
      }
#pragma unroll
      for (int s = TPQ / 2, n = NV; s >= 1; s >>= 1, n >>= 1) {
        const bool hi = (kq & s) != 0;
#pragma unroll
        for (int k = 0; k < n / 2; ++k) {
          const uint32_t send = hi ? v[k] : v[k + n / 2];
          const uint32_t keep = hi ? v[k + n / 2] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
      }
      // fast-path dots of 64-bit runs stay below 2^31 in magnitude
#pragma unroll
      for (int e = 0; e < VPL; ++e) val[e] = (BITS == 64) ? (long long)(int32_t)v[e] : (long long)v[e];
    } else {
      // 64-bit accumulators with a lane on the exact path somewhere in the warp
      long long v[NV];
#pragma unroll
      for (int m = 0; m < KM; ++m)
#pragma unroll
        for (int i = 0; i < RP; ++i)
          v[m * RP + i] = (long long)(int32_t)(acc[m][i] - (uint32_t)DPT * (uint32_t)kMagicBits);
      if (!fast) {
#pragma unroll
        for (int m = 0; m < KM; ++m) {
          const int jl = kl + KSTEP * m;
          unsigned long long ex[RP];
#pragma unroll
          for (int i = 0; i < RP; ++i) ex[i] = 0ull;
          for (int h = 0; h < CQ; ++h) {
            const int c = kq + TPQ * h;
            const KVT* kv = reinterpret_cast<const KVT*>(kt + jl * ROWB + ((c ^ (jl & SWZ)) * 16));
            for (int e = 0; e < CE; ++e) {
              const float kf = to_f32(kv[e]);
#pragma unroll
              for (int i = 0; i < RP; ++i)
                ex[i] += (unsigned long long)f2x_f32<64>(__fmul_rn(q_raw[i * D + c * CE + e], kf), scale);
            }
          }
#pragma unroll
          for (int i = 0; i < RP; ++i) v[m * RP + i] = (long long)ex[i];
        }
      }
#pragma unroll
      for (int s = TPQ / 2, n = NV; s >= 1; s >>= 1, n >>= 1) {
        const bool hi = (kq & s) != 0;
#pragma unroll
        for (int k = 0; k < n / 2; ++k) {
          const long long send = hi ? v[k] : v[k + n / 2];
          const long long keep = hi ? v[k + n / 2] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
      }
#pragma unroll
      for (int e = 0; e < VPL; ++e) val[e] = v[e];
    }

    const int j = kb + ti * KTC + kl + KSTEP * my_m;
    if (j < ke) {
#pragma unroll
      for (int e = 0; e < VPL; ++e) {
        const int i = my_i0 + e;
        const float s = score_of<BITS, PL>(p, val[e], j, row_kend[i], row_pos[i], row_head[i], inv_scale);
        sdst[i * CHUNK + (j - kb)] = s;
        rmax[e] = fmaxf(rmax[e], s);
      }
    }
  }
  cp_async_wait<0>();
  // lanes holding the same rows differ in the bits from RP / VPL up
#pragma unroll
  for (int e = 0; e < VPL; ++e) {
#pragma unroll
    for (int o = RP / VPL; o < 32; o <<= 1) rmax[e] = fmaxf(rmax[e], __shfl_xor_sync(0xffffffffu, rmax[e], o));
    if (lane < RP / VPL) wmax[warp][lane * VPL + e] = rmax[e];
  }
  __syncthreads();
  if (t < RP) {
    float m = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < THREADS / 32; ++w2) m = fmaxf(m, wmax[w2][t]);
    p.ws_m[unit * RP + t] = m;
  }
}

// ---------------------------------------------------------------------------
// kernel 2: normaliser, PV and the integer combine
// ---------------------------------------------------------------------------
template <int D, int RP, int BITS, typename KVT>
__global__ void __launch_bounds__(THREADS) chunk_pv_kernel(Params p) {
  using TL = Tile<D, KVT>;
  using SM = PvSmem<D, RP, KVT>;
  constexpr int ROWB = TL::ROWB, SWZ = TL::SWZ, TILEB = TL::TILEB;
  constexpr int CE = Chunk<KVT>::E;
  constexpr int KG = 512 / D;   // PV key groups
  constexpr int KPT = KT / KG;  // PV keys per thread per tile (contiguous)
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  static_assert(KPT % 4 == 0 && KPT >= 4, "PV key quads");
  static_assert((size_t)RP * D * 8 <= (size_t)NBP * TILEB, "partials reuse the tile buffers");

  extern __shared__ __align__(16) unsigned char smem[];
  float* P_all = reinterpret_cast<float*>(smem + SM::off_p);  // [RP][CHUNK]: score, then p * 2^f
  unsigned char* kvbuf = smem + SM::off_kv;
  __shared__ int row_tok[RP], row_head[RP], row_pos[RP], row_kend[RP];
  __shared__ float gmax_s[RP];
  __shared__ unsigned long long den_s[RP];
  __shared__ int last_s;

  const int t = threadIdx.x, lane = t & 31;
  const int chunk = blockIdx.x;
  const int kvh = blockIdx.y / p.head_slices, hslice = blockIdx.y % p.head_slices;
  const int req = blockIdx.z / p.qtiles, qtile = blockIdx.z % p.qtiles;
  const int kr_hi = unit_rows<RP>(p, req, qtile, kvh, hslice, row_tok, row_head, row_pos, row_kend);
  const int kb = chunk * CHUNK;
  if (kr_hi < 0 || (chunk > 0 && kb >= kr_hi)) return;  // uniform over the CTA
  const int ke = min(kb + CHUNK, kr_hi);
  const int ntiles = (ke - kb + KT - 1) / KT;
  const int nk = ntiles * KT;
  // units of this item; a context beyond the caller's max_seq_len hint is cut
  // at the workspace's capacity (nchunk_max units) instead of overrunning it
  const int nch = min(p.nchunk_max, max(1, (kr_hi + CHUNK - 1) / CHUNK));
  const int64_t item = (int64_t)blockIdx.z * gridDim.y + blockIdx.y;
  const int64_t unit = item * p.nchunk_max + chunk;
  const float scale = ldexpf(1.0f, p.frac);
  const float inv_scale = ldexpf(1.0f, -p.frac);

  // the unit's scores (written by kernel 1) ride with the first V tile
  {
    const float* src = p.ws_s + unit * (RP * CHUNK);
    const int per_row = nk / 4;  // 16-byte pieces per row
    for (int e = t; e < RP * per_row; e += THREADS) {
      const int i = e / per_row, c = e % per_row;
      cp_async16(P_all + i * CHUNK + 4 * c, src + i * CHUNK + 4 * c, 16);
    }
  }
  TileCopier<D, KVT> cp(p, req, kb, ke, kvh);
#pragma unroll
  for (int s0 = 0; s0 < NBP - 1; ++s0) {
    if (s0 < ntiles)
      cp.issue(p.v, p.v_sb, p.v_ss, p.v_sh, s0, kvbuf + s0 * TILEB, cp.block_of(s0));
    cp_async_commit();
  }
  int next_blk = (NBP - 1 < ntiles) ? cp.block_of(NBP - 1) : -1;

  if (t < RP) {
    den_s[t] = 0ull;
    float m = -INFINITY;
    const float* mrow = p.ws_m + item * p.nchunk_max * RP + t;
    for (int c = 0; c < nch; ++c) m = fmaxf(m, mrow[c * RP]);
    gmax_s[t] = m;  // == the reference's pass-1 max over the whole context
  }
  cp_async_wait<NBP - 2>();  // scores and V tile 0
  __syncthreads();

  // ---- p = exp2(score - max) (attention.py:237), normaliser (238-243) ----
  // in place; a warp's 32 elements lie in one row (nk is a multiple of 64)
  for (int e = t; e < RP * nk; e += THREADS) {
    const int i = e / nk, k = e % nk;
    const int j = kb + k;
    float pv = 0.0f;
    UAcc den = 0;
    if (j < ke) {
      pv = prim_exp2(__fsub_rn(P_all[i * CHUNK + k], gmax_s[i]));
      if (j < row_kend[i]) den = (UAcc)f2x_f32<BITS>(pv, scale);
    }
    P_all[i * CHUNK + k] = __fmul_rn(pv, scale);
    if constexpr (BITS == 64) {
#pragma unroll
      for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    } else {
      den = __reduce_add_sync(0xffffffffu, den);
    }
    if (lane == 0 && den) atomicAdd(&den_s[i], (unsigned long long)den);
  }

  // ---- PV (attention.py:245-255): acc[row][d] += F2X(p * fp16(v)) ----
  const int dp = t % (D / 2), kg = t / (D / 2);
  const int vchunk = (2 * dp) / CE, vin = ((2 * dp) % CE) * (int)sizeof(KVT);
  uint32_t accv[RP][2];
  unsigned long long accv64[RP][2];
#pragma unroll
  for (int i = 0; i < RP; ++i) {
    accv[i][0] = accv[i][1] = 0u;
    accv64[i][0] = accv64[i][1] = 0ull;
  }
  const float2 C2 = make_float2(kMagic, kMagic);
  const float2 ONE2 = make_float2(p.one, p.one);
  // PV fast path iff max|v| <= 65504 and max|v| * (1 + 2^-10) * 2^f < 2^22
  const double scale_d = ldexp(1.0, p.frac);
  const float vthr = __double2float_rd(fmin(65504.5, 4194304.0 / (scale_d * (1.0 + 1.0 / 1024))));
  // bf16 -> fp16 is exact for 2^-17 <= |v| <= 65504 (7 mantissa bits fit);
  // smaller |v| give |p * v * 2^f| < 1/2 -> 0 either way when f <= 16
  const bool v_exact16 = std::is_same<KVT, __nv_bfloat16>::value && p.frac <= 16;
  using VRaw = typename std::conditional<sizeof(KVT) == 2, uint32_t, uint2>::type;
  auto v_raw = [&](const unsigned char* vt, int jl) -> VRaw {
    return *reinterpret_cast<const VRaw*>(vt + jl * ROWB + ((vchunk ^ (jl & SWZ)) * 16) + vin);
  };
  // fp32(fp16(v)) as the reference computes it; E16: the bf16 -> fp16 step is exact
  auto v_f32 = [&](VRaw r, auto e16) -> float2 {
    if constexpr (sizeof(KVT) == 2 && std::is_same<KVT, __nv_bfloat16>::value && decltype(e16)::value) {
      const uint32_t w = reinterpret_cast<const uint32_t&>(r);
      return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    } else {
      return v_pair_f16<KVT>(reinterpret_cast<const unsigned char*>(&r));
    }
  };

  for (int ti = 0; ti < ntiles; ++ti) {
    if (ti > 0) cp_async_wait<NBP - 2>();
    __syncthreads();  // V tile ti (and, first time, p) visible; buffer (ti+NBP-1)%NBP free
    if (ti + NBP - 1 < ntiles) {
      cp.issue(p.v, p.v_sb, p.v_ss, p.v_sh, ti + NBP - 1,
               kvbuf + ((ti + NBP - 1) % NBP) * TILEB, next_blk);
      next_blk = (ti + NBP < ntiles) ? cp.block_of(ti + NBP) : -1;
    }
    cp_async_commit();

    const unsigned char* vt = kvbuf + (ti % NBP) * TILEB;
    const float* Pk = P_all + ti * KT + kg * KPT;  // this thread's keys: kg * KPT + u
    uint32_t tv[RP][2];
#pragma unroll
    for (int i = 0; i < RP; ++i) tv[i][0] = tv[i][1] = 0u;
    uint32_t vm = 0;
    auto pv_tile = [&](auto e16) {
#pragma unroll
    for (int u = 0; u < KPT; u += 4) {
      float4 pr[RP];
#pragma unroll
      for (int i = 0; i < RP; ++i) pr[i] = *reinterpret_cast<const float4*>(Pk + i * CHUNK + u);
#pragma unroll
      for (int h2 = 0; h2 < 4; h2 += 2) {
        const int ja = kg * KPT + u + h2, jb = ja + 1;
        const VRaw ra_ = v_raw(vt, ja), rb_ = v_raw(vt, jb);
        if constexpr (sizeof(KVT) == 2) {
          absmax_word<KVT>(vm, ra_);
          absmax_word<KVT>(vm, rb_);
        } else {
          absmax_word<KVT>(vm, ra_.x);
          absmax_word<KVT>(vm, ra_.y);
          absmax_word<KVT>(vm, rb_.x);
          absmax_word<KVT>(vm, rb_.y);
        }
        const float2 va = v_f32(ra_, e16), vb = v_f32(rb_, e16);
        const float2 v0 = make_float2(va.x, vb.x), v1 = make_float2(va.y, vb.y);
#pragma unroll
        for (int i = 0; i < RP; ++i) {
          const float2 pp = h2 == 0 ? make_float2(pr[i].x, pr[i].y) : make_float2(pr[i].z, pr[i].w);
          const float2 r0 = fma2(mul2(pp, v0), ONE2, C2);
          const float2 r1 = fma2(mul2(pp, v1), ONE2, C2);
          tv[i][0] += __float_as_uint(r0.x) + __float_as_uint(r0.y);
          tv[i][1] += __float_as_uint(r1.x) + __float_as_uint(r1.y);
        }
      }
    }
    };
    if (v_exact16) pv_tile(std::true_type{});
    else pv_tile(std::false_type{});
    if (absmax_value<KVT>(vm) < vthr) {
#pragma unroll
      for (int i = 0; i < RP; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t v = tv[i][h] - (uint32_t)KPT * (uint32_t)kMagicBits;
          if constexpr (BITS == 64) {
            accv64[i][h] += (unsigned long long)(long long)(int32_t)v;
          } else {
            accv[i][h] += v;
          }
        }
    } else {
      for (int u = 0; u < KPT; ++u) {
        const int jl = kg * KPT + u;
        const int j = kb + ti * KT + jl;
        if (j >= ke) continue;
        const float2 vv = v_pair_f16<KVT>(vt + jl * ROWB + ((vchunk ^ (jl & SWZ)) * 16) + vin);
#pragma unroll
        for (int i = 0; i < RP; ++i) {
          if (j >= row_kend[i]) continue;
          const float ps = Pk[i * CHUNK + u];
          const auto x0 = f2x_scaled<BITS>(__fmul_rn(ps, vv.x));
          const auto x1 = f2x_scaled<BITS>(__fmul_rn(ps, vv.y));
          if constexpr (BITS == 64) {
            accv64[i][0] += (unsigned long long)x0;
            accv64[i][1] += (unsigned long long)x1;
          } else {
            accv[i][0] += (uint32_t)x0;
            accv[i][1] += (uint32_t)x1;
          }
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every tile consumed: the tile buffers hold the unit partials
  unsigned long long* acc_s = reinterpret_cast<unsigned long long*>(kvbuf);
  for (int e = t; e < RP * D; e += THREADS) acc_s[e] = 0ull;
  __syncthreads();

  // ---- unit partials (integer, exact) ----
#pragma unroll
  for (int i = 0; i < RP; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const unsigned long long v = (BITS == 64) ? accv64[i][h] : (unsigned long long)accv[i][h];
      if (v) atomicAdd(&acc_s[i * D + 2 * dp + h], v);
    }
  __syncthreads();

  // ---- combine over the item's units, finalize (attention.py:257-279) ----
  auto finalize = [&](int e, unsigned long long a, unsigned long long dn) {
    const int i = e / D, d = e % D;
    float af, df;
    if constexpr (BITS == 64) {
      af = __fmul_rn(__ll2float_rn((long long)a), inv_scale);
      df = __fmul_rn(__ll2float_rn((long long)dn), inv_scale);
    } else {
      af = __fmul_rn(__int2float_rn((int32_t)(uint32_t)a), inv_scale);
      df = __fmul_rn(__int2float_rn((int32_t)(uint32_t)dn), inv_scale);
    }
    const float out = prim_div(af, fmaxf(df, 1.0e-6f));
    store_f32(p.o, p.o_dtype, (int64_t)row_tok[i] * p.o_st + (int64_t)row_head[i] * p.o_sh + d, out);
  };
  if (nch == 1) {  // the unit is the whole item
    for (int e = t; e < RP * D; e += THREADS)
      if (row_tok[e / D] >= 0) finalize(e, acc_s[e], den_s[e / D]);
    return;
  }
  unsigned long long* gacc = p.ws_acc + item * (RP * D);
  unsigned long long* gden = p.ws_den + item * RP;
  for (int e = t; e < RP * D; e += THREADS)
    if (row_tok[e / D] >= 0 && acc_s[e]) atomicAdd(&gacc[e], acc_s[e]);
  if (t < RP && row_tok[t] >= 0 && den_s[t]) atomicAdd(&gden[t], den_s[t]);
  __threadfence();
  __syncthreads();
  if (t == 0) last_s = (atomicAdd(&p.ws_cnt[item], 1u) == (unsigned)(nch - 1));
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  for (int e = t; e < RP * D; e += THREADS)
    if (row_tok[e / D] >= 0) finalize(e, __ldcg(&gacc[e]), __ldcg(&gden[e / D]));
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr size_t kChunkSmemMax = 200 * 1024;

template <int D, int RP, typename KVT>
static bool chunk_fits() {
  return ScoreSmem<D, RP, KVT>::bytes <= kChunkSmemMax && ScoreSmem<D, RP, KVT, KTC>::bytes <= kChunkSmemMax &&
         PvSmem<D, RP, KVT>::bytes <= kChunkSmemMax;
}

static int configure(const void* k, size_t smem, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return FXPR_OK;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    set_error("unified_attention_fxp: cannot configure shared memory");
    return FXPR_ERR_CUDA;
  }
  if (dev >= 0 && dev < 64) done[dev] = true;
  return FXPR_OK;
}

template <int D, int RP, int BITS, typename KVT>
static int launch_chunked_t(const Params& p, int req, int ys, cudaStream_t st) {
  if (!chunk_fits<D, RP, KVT>()) {
    set_error("unified_attention_fxp: chunked path does not fit shared memory");
    return FXPR_ERR_UNSUPPORTED;
  }
  constexpr bool rq = RP == 4 && (D == 64 || D == 128);
  const size_t s1 = rq ? ScoreSmem<D, RP, KVT, KTC>::bytes : ScoreSmem<D, RP, KVT>::bytes;
  const size_t s2 = PvSmem<D, RP, KVT>::bytes;
  const bool plain = !(p.softcap_log2 > 0.0f) && p.alibi == nullptr && p.window <= 0;
  void (*k1)(Params);
  if constexpr (rq) {  // decode: q in registers
    k1 = plain ? chunk_scores_rq_kernel<D, BITS, KVT, true> : chunk_scores_rq_kernel<D, BITS, KVT, false>;
  } else {
    k1 = plain ? chunk_scores_kernel<D, RP, BITS, KVT, true> : chunk_scores_kernel<D, RP, BITS, KVT, false>;
  }
  void (*k2)(Params) = chunk_pv_kernel<D, RP, BITS, KVT>;
  static bool done1[2][64] = {{false}}, done2[64] = {false};
  int rc = configure((const void*)k1, s1, done1[plain ? 1 : 0]);
  if (rc != FXPR_OK) return rc;
  rc = configure((const void*)k2, s2, done2);
  if (rc != FXPR_OK) return rc;
  const dim3 grid((unsigned)p.nchunk_max, (unsigned)ys, (unsigned)((int64_t)req * p.qtiles));
  k1<<<grid, THREADS, s1, st>>>(p);
  rc = check_launch("fxpr_unified_attention_fxp (scores)");
  if (rc != FXPR_OK) return rc;
  k2<<<grid, THREADS, s2, st>>>(p);
  return check_launch("fxpr_unified_attention_fxp (pv)");
}

template <int D, int RP>
static bool fits_kv(int kv_dtype) {
  switch (kv_dtype) {
    case FXPR_BF16: return chunk_fits<D, RP, __nv_bfloat16>();
    case FXPR_F16: return chunk_fits<D, RP, __half>();
    default:
      if constexpr (D <= 128) return chunk_fits<D, RP, float>();
      return false;
  }
}

bool chunked_supported(int D, int rp, int kv_dtype) {
  switch (D) {
    case 32: return rp == 4 ? fits_kv<32, 4>(kv_dtype) : fits_kv<32, 16>(kv_dtype);
    case 64: return rp == 4 ? fits_kv<64, 4>(kv_dtype) : fits_kv<64, 16>(kv_dtype);
    case 128: return rp == 4 ? fits_kv<128, 4>(kv_dtype) : fits_kv<128, 16>(kv_dtype);
    case 256: return rp == 4 ? fits_kv<256, 4>(kv_dtype) : fits_kv<256, 16>(kv_dtype);
  }
  return false;
}

template <int D, int RP, int BITS>
static int pick_kv_chunked(const Params& p, int kv_dtype, int req, int ys, cudaStream_t st) {
  switch (kv_dtype) {
    case FXPR_BF16: return launch_chunked_t<D, RP, BITS, __nv_bfloat16>(p, req, ys, st);
    case FXPR_F16: return launch_chunked_t<D, RP, BITS, __half>(p, req, ys, st);
    default:
      if constexpr (D <= 128) {
        return launch_chunked_t<D, RP, BITS, float>(p, req, ys, st);
      } else {
        set_error("unified_attention_fxp: float32 KV cache supports head_dim <= 128");
        return FXPR_ERR_UNSUPPORTED;
      }
  }
}

template <int D>
static int pick_rp_chunked(const Params& p, int rp, int bits, int kv_dtype, int req, int ys,
                           cudaStream_t st) {
  if (rp == 4) {
    if (bits == 32) return pick_kv_chunked<D, 4, 32>(p, kv_dtype, req, ys, st);
    return pick_kv_chunked<D, 4, 64>(p, kv_dtype, req, ys, st);
  }
  if (bits == 32) return pick_kv_chunked<D, 16, 32>(p, kv_dtype, req, ys, st);
  return pick_kv_chunked<D, 16, 64>(p, kv_dtype, req, ys, st);
}

int launch_chunked(const Params& p, int D, int rp, int bits, int kv_dtype, int req, int ys,
                   cudaStream_t st) {
  switch (D) {
    case 32: return pick_rp_chunked<32>(p, rp, bits, kv_dtype, req, ys, st);
    case 64: return pick_rp_chunked<64>(p, rp, bits, kv_dtype, req, ys, st);
    case 128: return pick_rp_chunked<128>(p, rp, bits, kv_dtype, req, ys, st);
    default: return pick_rp_chunked<256>(p, rp, bits, kv_dtype, req, ys, st);
  }
}

}  // namespace attn
}  // namespace fxpr
