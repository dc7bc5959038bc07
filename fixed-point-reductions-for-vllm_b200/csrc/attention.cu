// Paged unified attention with fixed-point softmax (attention.py:18-489),
// split-KV across a thread-block cluster with an exact integer combine.
//
// One CTA = (KV split s, KV head (slice of its query-head group), request,
// tile of queries). Its rows are (query, head) pairs that share one KV head,
// so every K/V element loaded from HBM is used by all rows of the group.
//
//   pass 1  K tiles (cp.async, 3 buffers) -> integer q.k per (row, key)
//           -> fp32 score (X2F, scale, softcap, alibi, masks) kept in shared
//           memory, row max over the split.
//   DSMEM   row maxima exchanged across the cluster: global max per row,
//           identical to the reference's whole-context pass 1.
//   pass 2  V tiles -> p = exp2(score - max), integer normaliser and integer
//           PV accumulation.
//   DSMEM   integer partials summed across the cluster (exact, order-free),
//           X2F, divide, store.
// The result is bitwise independent of the split count and of the tiling.
//
// Products use the magic-constant RNE path when an exponent guard proves
// |product * 2^f| < 2^22 for the whole tile; otherwise the exact
// clamp-and-convert path of the reference runs for that tile.
#include <cooperative_groups.h>

#include "attention_common.cuh"

namespace cg = cooperative_groups;

namespace fxpr {
namespace attn {

template <int D, int RP, typename KVT>
struct Smem {
  static constexpr int ROWB = D * (int)sizeof(KVT);  // bytes of one key row
  static constexpr int NC = ROWB / 16;               // 16-byte chunks per key row
  static constexpr int SWZ = (NC < 8 ? NC : 8) - 1;  // chunk swizzle mask
  static constexpr int TILEB = KT * ROWB;
  static constexpr size_t off_q = 0;
  static constexpr size_t off_qraw = off_q + (size_t)RP * D * 4;
  static constexpr size_t off_kv = off_qraw + (size_t)RP * D * 4;
  static constexpr size_t off_p = off_kv + (size_t)NBUF * TILEB;
  static constexpr size_t off_acc = off_p + (size_t)KT * RP * 4;
  static constexpr size_t off_den = off_acc + (size_t)RP * D * 8;
  static constexpr size_t off_stmp = off_den + (size_t)RP * 8;
  static constexpr size_t off_s = off_stmp + (size_t)RP * KT * 4;
  // scores [RP][cap + 8] floats, then the block indices of the first cap keys
  static size_t bytes(int cap) { return off_s + (size_t)RP * (cap + 8) * 4 + (size_t)cap * 4; }
};

}  // namespace attn
}  // namespace fxpr

namespace fxpr {
namespace attn {

template <int D, int RP, int BITS, typename KVT>
__global__ void __launch_bounds__(THREADS) attn_kernel(Params p) {
  using SM = Smem<D, RP, KVT>;
  constexpr int ROWB = SM::ROWB, NC = SM::NC, SWZ = SM::SWZ, TILEB = SM::TILEB;
  constexpr int CE = Chunk<KVT>::E;  // elements per 16-byte chunk
  constexpr int KG = 512 / D;         // PV key groups
  constexpr int KPT = KT / KG;        // PV keys per thread per tile
  constexpr int RPT = RP / 4;         // score rows finalised per thread
  constexpr int TPK = THREADS / KT;   // threads per key row in the copies
  constexpr int CPT = NC / TPK;       // 16-byte chunks copied per thread
  constexpr int RG = RP < 4 ? RP : 4; // rows per q-register group in the score loop
  using UAcc = typename std::conditional<BITS == 64, unsigned long long, uint32_t>::type;
  static_assert(NC % 4 == 0 && NC % TPK == 0, "head_dim too small for the chunk mapping");
  static_assert(KPT % 4 == 0 && KPT >= 4, "PV key quads");

  extern __shared__ __align__(16) unsigned char smem[];
  float* q_s = reinterpret_cast<float*>(smem + SM::off_q);
  float* q_raw = reinterpret_cast<float*>(smem + SM::off_qraw);
  unsigned char* kvbuf = smem + SM::off_kv;
  float* P = reinterpret_cast<float*>(smem + SM::off_p);  // [row][key slot], p * 2^f
  unsigned long long* acc_s = reinterpret_cast<unsigned long long*>(smem + SM::off_acc);
  unsigned long long* den_s = reinterpret_cast<unsigned long long*>(smem + SM::off_den);
  float* S_tmp = reinterpret_cast<float*>(smem + SM::off_stmp);
  float* S = reinterpret_cast<float*>(smem + SM::off_s);
  int* blk_cache = reinterpret_cast<int*>(S + RP * (p.cap + 8));  // [cap] physical blocks

  __shared__ int row_tok[RP], row_head[RP], row_pos[RP], row_kend[RP];
  __shared__ uint32_t q_or;
  __shared__ float wmax[THREADS / 32][RP];
  __shared__ float rmax_s[RP], gmax_s[RP];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int nsplit = p.splits;

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int kvh = blockIdx.y / p.head_slices, hslice = blockIdx.y % p.head_slices;
  const int req = blockIdx.z / p.qtiles, qtile = blockIdx.z % p.qtiles;
  const int q_start = p.qsl[req], q_end = p.qsl[req + 1];
  const int qlen = q_end - q_start;
  const int seq_len = p.seq_lens[req];
  const int ctx = seq_len - qlen;
  if (qtile * p.qt >= qlen) return;  // uniform over the cluster (same y, z)
  const float scale = ldexpf(1.0f, p.frac);
  const float inv_scale = ldexpf(1.0f, -p.frac);

  // ---- rows: (query, head) pairs of this CTA (attention.py:319-353) ----
  if (t < RP) {
    const int qi = t / p.gs, gh = t % p.gs;
    const int qoff = qtile * p.qt + qi;
    const int hg = hslice * p.gs + gh;
    int tok = -1, kend = 0, pos = 0, head = 0;
    if (qi < p.qt && qoff < qlen && hg < p.group) {
      tok = q_start + qoff;
      head = kvh * p.group + hg;
      pos = ctx + qoff;
      // the reference walks keys up to the end of its 64-row query block
      kend = p.causal ? min(seq_len, ctx + (qoff / 64 + 1) * 64) : seq_len;
    }
    row_tok[t] = tok;
    row_head[t] = head;
    row_pos[t] = pos;
    row_kend[t] = kend;
  }
  if (t == 0) q_or = 0u;
  __syncthreads();
  {
    uint32_t qo = 0;
    for (int e = t; e < RP * D; e += THREADS) {
      const int i = e / D, d = e % D;
      float v = 0.0f;
      if (row_tok[i] >= 0)
        v = load_f32(p.q, p.q_dtype, (int64_t)row_tok[i] * p.q_st + (int64_t)row_head[i] * p.q_sh + d);
      q_raw[e] = v;
      q_s[e] = __fmul_rn(v, scale);
      qo = max(qo, __float_as_uint(v) & 0x7FFFFFFFu);
      acc_s[e] = 0ull;
    }
    if (t < RP) den_s[t] = 0ull;
    qo = __reduce_max_sync(0xffffffffu, qo);
    if (lane == 0) atomicMax(&q_or, qo);
  }
  __syncthreads();

  int kr_hi = 0;
#pragma unroll
  for (int i = 0; i < RP; ++i) kr_hi = max(kr_hi, row_kend[i]);
  const int chunk = ((kr_hi + nsplit - 1) / nsplit + 15) & ~15;
  const int kb = min(rank * chunk, kr_hi);
  const int ke = min(kb + chunk, kr_hi);
  const int ntiles = (ke - kb + KT - 1) / KT;
  const int64_t bt_row = (int64_t)req * p.bt_stride;

  // Per-thread fast-path thresholds (strict): a score product is exact through
  // the magic constant iff max|q| * max|k| * 2^f < 2^22; a PV product iff
  // max|v| <= 65504 (fp16 finite) and max|v| * (1 + 2^-10) * 2^f < 2^22.
  // Rounded down to fp32 so the float compare is conservative.
  const double scale_d = ldexp(1.0, p.frac);
  const double mq = (double)__uint_as_float(q_or);
  const bool q_ok = mq * scale_d < 3.0e38;  // q * 2^f finite (NaN: false)
  const float kthr = q_ok ? __double2float_rd(4194304.0 / (mq * scale_d)) : 0.0f;
  const float vthr = __double2float_rd(fmin(65504.5, 4194304.0 / (scale_d * (1.0 + 1.0 / 1024))));

  // ---- tile copies: each thread copies CPT consecutive 16-byte chunks of
  // one key row, XOR-swizzled in shared memory. The physical block of the
  // row comes from `blk` (looked up ahead of time, see below) ----
  const int my_jl = t / TPK;
  auto block_of = [&](int ti) -> int {  // physical block of this thread's key in tile ti
    const int j = kb + ti * KT + my_jl;
    if (j >= ke) return -1;
    const int bi = p.page_shift >= 0 ? (j >> p.page_shift) : j / p.page;
    return p.bt[bt_row + bi];
  };
  auto issue = [&](const void* base, int64_t sb, int64_t ss, int64_t sh, int ti, int b, int blk) {
    const int c0 = (t % TPK) * CPT;
    const int j = kb + ti * KT + my_jl;
    unsigned char* dst = kvbuf + b * TILEB + my_jl * ROWB;
    const unsigned char* src = reinterpret_cast<const unsigned char*>(base);
    int bytes = 0;
    if (blk >= 0) {
      const int slot = p.page_shift >= 0 ? (j & (p.page - 1)) : j % p.page;
      src += ((int64_t)blk * sb + (int64_t)slot * ss + (int64_t)kvh * sh) * (int64_t)sizeof(KVT);
      bytes = 16;
    }
#pragma unroll
    for (int u = 0; u < CPT; ++u) {
      const int c = c0 + u;
#if FXPR_ATTN_L2PF
      cp_async16_l2pf(dst + ((c ^ (my_jl & SWZ)) * 16), src + c * 16, bytes);
#else
      cp_async16(dst + ((c ^ (my_jl & SWZ)) * 16), src + c * 16, bytes);
#endif
    }
  };
  // block of tile ti: from the shared-memory cache filled in pass 1 when the
  // tile lies within the score capacity, else from the block table
  auto cached_block = [&](int ti) -> int {
    if ((ti + 1) * KT <= p.cap) return blk_cache[ti * KT + my_jl];
    return block_of(ti);
  };

  // ---- scores of one K tile (attention.py:80-148) ----
  // dst == nullptr: only the row max is updated (keys beyond the capacity)
  float rmax[RPT];
#pragma unroll
  for (int u = 0; u < RPT; ++u) rmax[u] = -INFINITY;

  auto qk_tile = [&](int ti, int b, float* dst, int pitch, int col0, bool upd_max) {
    const unsigned char* kt = kvbuf + b * TILEB;
    const int jl = t >> 2, dq = t & 3;
    const int j = kb + ti * KT + jl;
    long long dot[RP];
    uint32_t acc[RP];
#pragma unroll
    for (int i = 0; i < RP; ++i) acc[i] = 0u;
    uint32_t km = 0;
    const float2 C2 = make_float2(kMagic, kMagic);
    const float2 ONE2 = make_float2(p.one, p.one);
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
          float4 qv[RG][CE / 4];  // q of RG rows for this chunk, loaded ahead of the math
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
    if (absmax_value<KVT>(km) < kthr) {
#pragma unroll
      for (int i = 0; i < RP; ++i) {
        acc[i] -= (uint32_t)(D / 4) * (uint32_t)kMagicBits;
        dot[i] = (BITS == 64) ? (long long)(int32_t)acc[i] : (long long)acc[i];
      }
    } else {
      // this thread's keys hold values the magic constant cannot round
      // exactly: redo its products on the exact reference path
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
    // reduce over the 4 lanes that share the key
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
    if (j >= ke) return;
#pragma unroll
    for (int u = 0; u < RPT; ++u) {
      const int i = dq + 4 * u;
      long long di = dot[4 * u];  // select dot[i] without runtime register indexing
#pragma unroll
      for (int w = 1; w < 4; ++w)
        if (dq == w) di = dot[4 * u + w];
      float s = -INFINITY;
      if (j < row_kend[i]) {
        float qk = (BITS == 64) ? __ll2float_rn(di) : __int2float_rn((int)di);
        qk = __fmul_rn(__fmul_rn(qk, inv_scale), p.scale_log2);
        if (p.softcap_log2 > 0.0f)
          qk = __fmul_rn(p.softcap_log2, prim_tanh(__fmul_rn(qk, p.softcap_rcp)));
        const int pos = row_pos[i];
        if (p.alibi)
          qk = __fmaf_rn(p.alibi[row_head[i]], __fsub_rn((float)j, (float)pos), qk);  // contracted, as Triton lowers it
        bool ok = true;
        if (p.causal) ok = ok && (pos >= j);
        if (p.window > 0) ok = ok && (j > pos - p.window);
        s = ok ? qk : -INFINITY;
      }
      if (dst) dst[i * pitch + col0 + jl] = s;
      if (upd_max) rmax[u] = fmaxf(rmax[u], s);
    }
  };

  // ================= pass 1: scores and row max =================
  auto remember = [&](int ti, int blk) {
    if ((t % TPK) == 0 && (ti + 1) * KT <= p.cap) blk_cache[ti * KT + my_jl] = blk;
  };
#pragma unroll
  for (int s0 = 0; s0 < NBUF - 1; ++s0) {
    if (s0 < ntiles) {
      const int blk = block_of(s0);
      remember(s0, blk);
      issue(p.k, p.k_sb, p.k_ss, p.k_sh, s0, s0, blk);
    }
    cp_async_commit();
  }
  // the block-table entry of the next tile to issue is loaded one iteration
  // early, so no global round trip sits in front of a copy
  int next_blk = (NBUF - 1 < ntiles) ? block_of(NBUF - 1) : -1;
  for (int ti = 0; ti < ntiles; ++ti) {
    const int b = ti % NBUF;
    cp_async_wait<NBUF - 2>();
    __syncthreads();  // tile ti visible to all; buffer (ti+NBUF-1)%NBUF free
    if (ti + NBUF - 1 < ntiles) {
      remember(ti + NBUF - 1, next_blk);
      issue(p.k, p.k_sb, p.k_ss, p.k_sh, ti + NBUF - 1, (ti + NBUF - 1) % NBUF, next_blk);
      next_blk = (ti + NBUF < ntiles) ? block_of(ti + NBUF) : -1;
    }
    cp_async_commit();
    const bool store = (ti + 1) * KT <= p.cap;
    qk_tile(ti, b, store ? S : nullptr, p.cap + 8, ti * KT, true);
  }
  // row max over this split
#pragma unroll
  for (int u = 0; u < RPT; ++u) {
    float m = rmax[u];
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    if (lane < 4) wmax[warp][lane + 4 * u] = m;
  }
  __syncthreads();  // also: every thread is done with the K buffers
  if (t < RP) {
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) m = fmaxf(m, wmax[w][t]);
    rmax_s[t] = m;
  }
  // start streaming V while the maxima are exchanged
  __syncthreads();  // block cache complete
#pragma unroll
  for (int s0 = 0; s0 < NBUF - 1; ++s0) {
    if (s0 < ntiles) issue(p.v, p.v_sb, p.v_ss, p.v_sh, s0, s0, cached_block(s0));
    cp_async_commit();
  }
  cluster.sync();
  if (t < RP) {
    float m = -INFINITY;
    for (int q = 0; q < nsplit; ++q) m = fmaxf(m, *cluster.map_shared_rank(&rmax_s[t], q));
    gmax_s[t] = m;  // == the reference's pass-1 max over the whole context
  }
  __syncthreads();

  // ================= pass 2: normaliser and PV =================
  const int prow = t % RP;  // p-phase row of this thread
  UAcc den_acc = 0;
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
  // bf16 -> fp16 is exact for 2^-17 <= |v| <= 65504 (7 mantissa bits fit);
  // smaller |v| give |p * v * 2^f| < 1/2 -> 0 either way when f <= 16
  const bool v_exact16 = std::is_same<KVT, __nv_bfloat16>::value && p.frac <= 16;

  // raw V pair of key jl at this thread's two dims
  using VRaw = typename std::conditional<sizeof(KVT) == 2, uint32_t, uint2>::type;
  auto v_raw = [&](const unsigned char* vt, int jl) -> VRaw {
    return *reinterpret_cast<const VRaw*>(vt + jl * ROWB + ((vchunk ^ (jl & SWZ)) * 16) + vin);
  };
  auto v_f32 = [&](VRaw r) -> float2 {  // fp32(fp16(v)) as the reference computes it
    if constexpr (sizeof(KVT) == 2) {
      if (v_exact16) return make_float2(__uint_as_float(r << 16), __uint_as_float(r & 0xFFFF0000u));
      return v_pair_f16<KVT>(reinterpret_cast<const unsigned char*>(&r));
    } else {
      return v_pair_f16<KVT>(reinterpret_cast<const unsigned char*>(&r));
    }
  };

  for (int ti = 0; ti < ntiles; ++ti) {
    const int b = ti % NBUF;
    cp_async_wait<NBUF - 2>();
    __syncthreads();  // V tile ti visible; previous P consumed; buffer (ti+NBUF-1)%NBUF free
    const bool recompute = (ti + 1) * KT > p.cap;
    if (recompute) {
      // scores beyond the capacity: reload this K tile into the free buffer
      const int kbuf = (ti + NBUF - 1) % NBUF;
      issue(p.k, p.k_sb, p.k_ss, p.k_sh, ti, kbuf, block_of(ti));
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
      qk_tile(ti, kbuf, S_tmp, KT, 0, false);
      __syncthreads();
    }
    if (ti + NBUF - 1 < ntiles)
      issue(p.v, p.v_sb, p.v_ss, p.v_sh, ti + NBUF - 1, (ti + NBUF - 1) % NBUF,
            cached_block(ti + NBUF - 1));
    cp_async_commit();

    // p = exp2(score - max) (attention.py:237), normaliser (238-243)
    const float gm = gmax_s[prow];
    const int kend_p = row_kend[prow];
    for (int jl = t / RP; jl < KT; jl += THREADS / RP) {
      const int j = kb + ti * KT + jl;
      float pv = 0.0f;
      if (j < ke) {
        const float sc = recompute ? S_tmp[prow * KT + jl] : S[prow * (p.cap + 8) + ti * KT + jl];
        pv = prim_exp2(__fsub_rn(sc, gm));
        if (j < kend_p) den_acc += (UAcc)f2x_f32<BITS>(pv, scale);
      }
      // key slot: the KPT keys of PV thread group kg are contiguous
      P[prow * KT + (jl % KG) * KPT + jl / KG] = __fmul_rn(pv, scale);
    }
    __syncthreads();

    // PV (attention.py:245-255): acc[row][d] += F2X(p * fp16(v)); optimistic
    // magic-constant path, per-thread exact redo if its V values are too large
    const unsigned char* vt = kvbuf + b * TILEB;
    uint32_t tv[RP][2];
#pragma unroll
    for (int i = 0; i < RP; ++i) tv[i][0] = tv[i][1] = 0u;
    uint32_t vm = 0;
    const float* Pk = P + kg * KPT;
#pragma unroll
    for (int u = 0; u < KPT; u += 4) {
      // p of keys u..u+3 of this thread for every row: one 16-byte load per row
      float4 pr[RP];
#pragma unroll
      for (int i = 0; i < RP; ++i) pr[i] = *reinterpret_cast<const float4*>(Pk + i * KT + u);
#pragma unroll
      for (int h2 = 0; h2 < 4; h2 += 2) {
        const int ja = kg + KG * (u + h2), jb = kg + KG * (u + h2 + 1);
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
        const float2 va = v_f32(ra_), vb = v_f32(rb_);
        // (key a, key b) pairs at dim 0 and at dim 1
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
        const int jl = kg + KG * u;
        const int j = kb + ti * KT + jl;
        if (j >= ke) continue;
        const float2 vv = v_pair_f16<KVT>(vt + jl * ROWB + ((vchunk ^ (jl & SWZ)) * 16) + vin);
#pragma unroll
        for (int i = 0; i < RP; ++i) {
          if (j >= row_kend[i]) continue;
          const float ps = P[i * KT + kg * KPT + u];
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

  // ---- CTA partials (integer, exact) ----
#pragma unroll
  for (int i = 0; i < RP; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const unsigned long long v = (BITS == 64) ? accv64[i][h] : (unsigned long long)accv[i][h];
      if (v) atomicAdd(&acc_s[i * D + 2 * dp + h], v);
    }
  if (den_acc) atomicAdd(&den_s[prow], (unsigned long long)den_acc);
  __syncthreads();
  cluster.sync();

  // ---- split combine across the cluster, finalize (attention.py:257-279) ----
  for (int e = t; e < RP * D; e += THREADS) {
    if (e % nsplit != rank) continue;
    const int i = e / D, d = e % D;
    if (row_tok[i] < 0) continue;
    unsigned long long a = 0, dn = 0;
    for (int q = 0; q < nsplit; ++q) {
      a += *cluster.map_shared_rank(&acc_s[e], q);
      dn += *cluster.map_shared_rank(&den_s[i], q);
    }
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
  }
  cluster.sync();
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr size_t kSmemBudget = 113 * 1024;  // two CTAs per SM

template <int D, int RP, int BITS, typename KVT>
static int launch(const Params& base, int max_keys, int splits, int req, int ys, cudaStream_t st) {
  using SM = Smem<D, RP, KVT>;
  Params p = base;
  if (SM::off_s > kSmemBudget) {
    set_error("unified_attention_fxp: head_dim/dtype combination exceeds shared memory");
    return FXPR_ERR_UNSUPPORTED;
  }
  // score capacity: one split's keys when they fit the budget; keys beyond
  // the capacity are rescored in pass 2
  const int need = ((max_keys + splits - 1) / splits + 15) / 16 * 16 + 16;
  int cap_max = (int)((kSmemBudget - SM::off_s) / (RP * 4 + 4) - 8) / KT * KT;
  int cap = (need + KT - 1) / KT * KT;
  if (cap > cap_max) cap = cap_max;
  p.cap = cap;
  p.splits = splits;
  const size_t smem = SM::bytes(cap);
  auto k = attn_kernel<D, RP, BITS, KVT>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget) !=
        cudaSuccess) {
      set_error("unified_attention_fxp: cannot configure shared memory");
      return FXPR_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int64_t gz = (int64_t)req * p.qtiles;
  if (gz > 65535) {
    set_error("unified_attention_fxp: too many (request, query tile) pairs: %lld", (long long)gz);
    return FXPR_ERR_UNSUPPORTED;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)splits, (unsigned)ys, (unsigned)gz);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k, p);
  if (e != cudaSuccess) {
    set_error("unified_attention_fxp: launch failed: %s", cudaGetErrorString(e));
    return FXPR_ERR_CUDA;
  }
  return check_launch("fxpr_unified_attention_fxp");
}

template <int D, int RP, int BITS>
static int pick_kv(const Params& p, int kv_dtype, int max_keys, int splits, int req, int ys,
                   cudaStream_t st) {
  switch (kv_dtype) {
    case FXPR_BF16: return launch<D, RP, BITS, __nv_bfloat16>(p, max_keys, splits, req, ys, st);
    case FXPR_F16: return launch<D, RP, BITS, __half>(p, max_keys, splits, req, ys, st);
    default:
      if constexpr (D <= 128) {
        return launch<D, RP, BITS, float>(p, max_keys, splits, req, ys, st);
      } else {
        set_error("unified_attention_fxp: float32 KV cache supports head_dim <= 128");
        return FXPR_ERR_UNSUPPORTED;
      }
  }
}

template <int D>
static int pick_rp(const Params& p, int rp, int bits, int kv_dtype, int max_keys, int splits,
                   int req, int ys, cudaStream_t st) {
  if (rp == 4) {
    if (bits == 32) return pick_kv<D, 4, 32>(p, kv_dtype, max_keys, splits, req, ys, st);
    return pick_kv<D, 4, 64>(p, kv_dtype, max_keys, splits, req, ys, st);
  }
  if (bits == 32) return pick_kv<D, 16, 32>(p, kv_dtype, max_keys, splits, req, ys, st);
  return pick_kv<D, 16, 64>(p, kv_dtype, max_keys, splits, req, ys, st);
}

}  // namespace attn
}  // namespace fxpr

using namespace fxpr;

namespace {

// Shape decisions shared by the launch and the workspace query.
struct Plan {
  int G, rp, gs, head_slices, qt, qtiles, ys, max_keys, nchunk_max;
  int decode_kmax;  // > 0: the decode path runs, keys per context capped here
  int64_t items;
  // chunked-path workspace layout (bytes); total 0 = path not applicable
  int64_t off_acc, off_den, off_m, off_s, total;
};

constexpr int64_t kChunkWsLimit = 1ll << 30;

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

int validate(const fxpr_attention_params* a) {
  if (!a) {
    set_error("unified_attention_fxp: null params");
    return FXPR_ERR_INVALID;
  }
  if (a->int_bits == 16) {
    set_error("unified_attention_fxp: int16 accumulators are not supported");
    return FXPR_ERR_UNSUPPORTED;
  }
  if (a->int_bits != 32 && a->int_bits != 64) {
    set_error("fxp_int_bits must be 16/32/64, got %d", a->int_bits);
    return FXPR_ERR_INVALID;
  }
  const int D = a->head_dim;
  if (D != 32 && D != 64 && D != 128 && D != 256) {
    set_error("unified_attention_fxp: head_dim %d not supported (32/64/128/256)", D);
    return FXPR_ERR_UNSUPPORTED;
  }
  auto okf = [](int d) { return d == FXPR_F16 || d == FXPR_BF16 || d == FXPR_F32; };
  if (!okf(a->q_dtype) || !okf(a->kv_dtype) || !okf(a->o_dtype)) {
    set_error("unified_attention_fxp: q/kv/o must be float16/bfloat16/float32");
    return FXPR_ERR_UNSUPPORTED;
  }
  if (a->num_kv_heads <= 0 || a->num_heads % a->num_kv_heads != 0 || a->page_size <= 0) {
    set_error("unified_attention_fxp: bad head counts or page size");
    return FXPR_ERR_INVALID;
  }
  return FXPR_OK;
}

Plan plan_of(const fxpr_attention_params* a) {
  Plan pl = {};
  pl.G = a->num_heads / a->num_kv_heads;
  pl.rp = (a->max_query_len == 1 && pl.G <= 4) ? 4 : 16;
  pl.gs = pl.G < pl.rp ? pl.G : pl.rp;
  pl.head_slices = (pl.G + pl.gs - 1) / pl.gs;
  pl.qt = pl.rp / pl.gs;
  pl.qtiles = (a->max_query_len + pl.qt - 1) / pl.qt;
  pl.ys = a->num_kv_heads * pl.head_slices;
  const int max_keys = a->max_seq_len > 0 ? a->max_seq_len : a->block_table_cols * a->page_size;
  pl.max_keys = max_keys < 1 ? 1 : max_keys;
  pl.nchunk_max = (pl.max_keys + attn::CHUNK - 1) / attn::CHUNK;
  pl.items = (int64_t)(a->num_requests > 0 ? a->num_requests : 0) * pl.qtiles * pl.ys;
  pl.decode_kmax = 0;
  if (a->num_requests > 0 && attn::decode_supported(a, pl.G)) {
    const int64_t cap = (int64_t)a->block_table_cols * a->page_size;
    const int kmax = (int)(pl.max_keys < cap ? pl.max_keys : cap);
    const int64_t need = attn::decode_workspace_bytes(a->num_requests * a->num_kv_heads, kmax, a->head_dim);
    if (kmax > 0 && need <= kChunkWsLimit) {
      pl.decode_kmax = kmax;
      pl.total = need;
      return pl;
    }
  }
  if (!attn::chunked_supported(a->head_dim, pl.rp, a->kv_dtype) || pl.items <= 0 ||
      (int64_t)a->num_requests * pl.qtiles > 65535 || pl.nchunk_max > 65535)
    return pl;
  const int64_t rows = pl.items * pl.rp;
  pl.off_acc = align256(pl.items * 4);
  pl.off_den = align256(pl.off_acc + rows * a->head_dim * 8);
  pl.off_m = align256(pl.off_den + rows * 8);
  pl.off_s = align256(pl.off_m + rows * pl.nchunk_max * 4);
  const int64_t total = pl.off_s + rows * pl.nchunk_max * attn::CHUNK * 4;
  if (total <= kChunkWsLimit) pl.total = total;
  return pl;
}

}  // namespace

extern "C" int64_t fxpr_attention_workspace_bytes(const fxpr_attention_params* a) {
  if (validate(a) != FXPR_OK) return 0;
  if (a->num_requests <= 0 || a->max_query_len <= 0) return 0;
  return plan_of(a).total;
}

extern "C" int fxpr_unified_attention_fxp(const fxpr_attention_params* a, void* stream) {
  const int rc = validate(a);
  if (rc != FXPR_OK) return rc;
  const int D = a->head_dim;
  const int es = elem_size(a->kv_dtype);
  const bool aligned = ((uintptr_t)a->k_cache % 16 == 0) && ((uintptr_t)a->v_cache % 16 == 0) &&
                       ((a->k_stride_blk * es) % 16 == 0) && ((a->k_stride_slot * es) % 16 == 0) &&
                       ((a->k_stride_head * es) % 16 == 0) && ((a->v_stride_blk * es) % 16 == 0) &&
                       ((a->v_stride_slot * es) % 16 == 0) && ((a->v_stride_head * es) % 16 == 0);
  if (!aligned) {
    set_error("unified_attention_fxp: KV cache rows must be 16-byte aligned");
    return FXPR_ERR_INVALID;
  }
  if (a->num_requests <= 0 || a->max_query_len <= 0) return FXPR_OK;
  const Plan pl = plan_of(a);
  attn::Params p = {};
  p.q = a->q; p.q_dtype = a->q_dtype; p.q_st = a->q_stride_tok; p.q_sh = a->q_stride_head;
  p.k = a->k_cache; p.v = a->v_cache;
  p.k_sb = a->k_stride_blk; p.k_ss = a->k_stride_slot; p.k_sh = a->k_stride_head;
  p.v_sb = a->v_stride_blk; p.v_ss = a->v_stride_slot; p.v_sh = a->v_stride_head;
  p.o = a->o; p.o_dtype = a->o_dtype; p.o_st = a->o_stride_tok; p.o_sh = a->o_stride_head;
  p.qsl = a->query_start_loc; p.seq_lens = a->seq_lens; p.bt = a->block_table;
  p.bt_stride = a->bt_stride; p.alibi = a->alibi_slopes;
  p.num_heads = a->num_heads; p.num_kv_heads = a->num_kv_heads; p.group = pl.G; p.gs = pl.gs;
  p.head_slices = pl.head_slices; p.qt = pl.qt; p.page = a->page_size;
  p.causal = a->is_causal; p.window = a->window_size;
  p.scale_log2 = a->scale_log2; p.softcap_log2 = a->logits_soft_cap;
  p.softcap_rcp = a->logits_soft_cap > 0.0f ? 1.0f / a->logits_soft_cap : 0.0f;
  p.frac = a->frac_bits;
  p.exact_qk = (a->q_dtype != FXPR_F32) && (a->kv_dtype != FXPR_F32);
  p.qtiles = pl.qtiles;
  p.one = 1.0f;
  p.page_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1 << sh) == a->page_size) p.page_shift = sh;
  const cudaStream_t st = (cudaStream_t)stream;
  const int R = a->num_requests;

  if (a->workspace && pl.total > 0 && a->workspace_bytes >= pl.total) {
    if ((uintptr_t)a->workspace % 256 != 0) {
      set_error("unified_attention_fxp: workspace must be 256-byte aligned");
      return FXPR_ERR_INVALID;
    }
    if (pl.decode_kmax > 0) return attn::launch_decode(a, pl.decode_kmax, a->workspace, st);
    unsigned char* ws = reinterpret_cast<unsigned char*>(a->workspace);
    p.ws_cnt = reinterpret_cast<uint32_t*>(ws);
    p.ws_acc = reinterpret_cast<unsigned long long*>(ws + pl.off_acc);
    p.ws_den = reinterpret_cast<unsigned long long*>(ws + pl.off_den);
    p.ws_m = reinterpret_cast<float*>(ws + pl.off_m);
    p.ws_s = reinterpret_cast<float*>(ws + pl.off_s);
    p.nchunk_max = pl.nchunk_max;
    return attn::launch_chunked(p, D, pl.rp, a->int_bits, a->kv_dtype, R, pl.ys, st);
  }

  const int max_keys = pl.max_keys;
  const int rp = pl.rp;
  int splits = a->num_kv_splits < 1 ? 1 : a->num_kv_splits;
  if (splits > attn::MAX_SPLITS) splits = attn::MAX_SPLITS;
  const int max_useful = (max_keys + attn::KT - 1) / attn::KT;  // no split shorter than a tile
  if (splits > max_useful) splits = max_useful < 1 ? 1 : max_useful;
  const int ys = pl.ys;
  // The split count only changes the schedule, never the result. Use the
  // knob as an upper bound: once the (request, head, query tile) work items
  // alone fill about two waves of resident CTAs, extra splits only add
  // per-CTA fixed cost (metadata loads, q staging, the cluster combine).
  {
    const int64_t items = (int64_t)a->num_requests * ys * p.qtiles;
    const int64_t resident = (int64_t)num_sms() * 3;
    int64_t want = (2 * resident + items - 1) / items;
    if (want < 1) want = 1;
    if (splits > want) splits = (int)want;
  }
  switch (D) {
    case 32: return attn::pick_rp<32>(p, rp, a->int_bits, a->kv_dtype, max_keys, splits, R, ys, st);
    case 64: return attn::pick_rp<64>(p, rp, a->int_bits, a->kv_dtype, max_keys, splits, R, ys, st);
    case 128: return attn::pick_rp<128>(p, rp, a->int_bits, a->kv_dtype, max_keys, splits, R, ys, st);
    default: return attn::pick_rp<256>(p, rp, a->int_bits, a->kv_dtype, max_keys, splits, R, ys, st);
  }
}
