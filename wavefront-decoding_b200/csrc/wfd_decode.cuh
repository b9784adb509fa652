// K1 — wavefront decode attention on CUDA cores (sm_100a).
//
// One persistent grid covers the flattened work space
//     (segment, query group, kv head, key)
// with an equal key share per CTA ("stream-K" split): every CTA streams the same
// number of K/V bytes, so a ragged wave (slot lengths staggered by loop depth)
// finishes in one pass without a tail.  A unit (segment, query group, kv head)
// that straddles CTAs is finished by the last CTA to reach it (atomic arrival
// counter, no spinning), which merges the partial softmax states.
//
// Per CTA: 4 warps, each with a private STAGES-deep ring in shared memory: the
// warp's lanes stage its K/V rows with the TMA bulk-copy engine (cp.async.bulk,
// one row per copy, mbarrier completion) and consume them without any CTA-wide
// barrier inside the key loop.  Each key row is read by LANES = Dh/VEC lanes
// holding 16 contiguous bytes each; the NQ query vectors of one kv head (GQA
// group x window rows) live in registers, so every K/V byte is read from HBM
// once for all query heads that share it.  Scores of TK keys x NQ queries are
// reduced with a butterfly reduce-scatter (one score per lane), the online
// softmax runs in the log2 domain in fp32, and the probabilities are all-gathered
// back for the P.V FMAs (packed fp32x2 FMA).
#pragma once

#include "wfd_common.cuh"

namespace wfd {

struct DecodeParams {
  const void* q;
  const void* k;      // key buffer rows (cache or packed)
  const void* v;
  const void* k_new;  // window rows (slot mode) or null; already appended to k / v by the plan kernel
  const void* v_new;
  void* out;
  const Seg* segs;
  const long long* prefix;
  int n_segs;
  int Hq, Hkv, G;
  float scale_log2;   // softmax scale * log2(e)
  int causal;
  long long k_row_offset;  // added to every segment's k_row0 (layer offset in slot mode)
  float* ws_part;          // 2 * gridDim.x partial slots
  int* ws_cnt;             // gridDim.x arrival counters (zero between launches)
  int* err;
};

__host__ __device__ constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x >> 1); }
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }

template <typename T, int DH, int NQ>
struct DecodeCfg {
  static constexpr int VEC = Elem<T>::kVec;
  static constexpr int LANES = DH / VEC;         // lanes per key row
  static constexpr int GROUPS = 32 / LANES;      // key groups per warp
  static constexpr int TK = cmin(LANES / NQ, 8); // keys per group per step
  static constexpr int P = TK * NQ;              // partial scores per lane
  static constexpr int LOGP = ilog2(P);
  static constexpr int LOGL = ilog2(LANES);
  static constexpr int NWARPS = 4;
  static constexpr int THREADS = NWARPS * 32;
  static constexpr int KPW = GROUPS * TK;        // keys per warp per stage
  static constexpr int KPS = NWARPS * KPW;       // keys per CTA-wide stage (warps interleave)
  static constexpr int ROWB = DH * (int)sizeof(T);
  // every warp owns a private ring of STAGES buffers (KPW K rows, then KPW V
  // rows) with its own mbarriers, so no CTA barrier sits inside the key loop
  static constexpr int WSTAGE_BYTES = KPW * ROWB * 2;
  static constexpr int STAGES = cmax(2, cmin(8, 16384 / WSTAGE_BYTES));
  static constexpr int WARP_BYTES = STAGES * WSTAGE_BYTES;
  static constexpr int NG = NWARPS * GROUPS;     // independent softmax states per CTA
  static constexpr int MERGE_BYTES = NG * NQ * (DH + 2) * 4;
  static constexpr int SMEM = cmax(NWARPS * WARP_BYTES, MERGE_BYTES);
  static_assert(KPW <= 32, "one lane issues one row copy pair");
  static constexpr int PART_FLOATS = NQ * (DH + 2);  // one partial slot
  static_assert(LANES >= 8 && LANES <= 32 && (LANES & (LANES - 1)) == 0, "lanes per row");
  static_assert(NQ >= 1 && NQ <= LANES && (NQ & (NQ - 1)) == 0, "NQ must be a power of two <= LANES");
  static_assert(P <= LANES, "partials per lane");
};

__device__ __forceinline__ int bitrev(int x, int bits) {
  return bits == 0 ? 0 : (int)(__brev((unsigned)x) >> (32 - bits));
}

// Butterfly reduce-scatter of P partial sums over the P lanes that differ in
// lane bits 0..log2(P)-1.  Returns this lane's fully reduced element, whose
// original index is bitrev(lane & (P-1)).
template <int P>
__device__ __forceinline__ float reduce_scatter(float (&v)[P], int lig) {
#pragma unroll
  for (int l = 0; (P >> l) > 1; ++l) {
    const int H = (P >> l) >> 1;
    const bool up = (lig >> l) & 1;
#pragma unroll
    for (int i = 0; i < (P >> 1); ++i) {
      if (i < H) {
        const float send = up ? v[i] : v[i + H];
        const float keep = up ? v[i + H] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1 << l);
      }
    }
  }
  return v[0];
}

// Inverse of reduce_scatter's index map: every lane ends with all P values in
// original index order.
template <int P>
__device__ __forceinline__ void all_gather(float x, float (&o)[P], int lig) {
  constexpr int LOGP = ilog2(P);
  o[0] = x;
#pragma unroll
  for (int k = 0; k < LOGP; ++k) {
    const int S = 1 << k;
    const int l = LOGP - 1 - k;
    const bool up = (lig >> l) & 1;
#pragma unroll
    for (int i = 0; i < (P >> 1); ++i) {
      if (i < S) {
        const float mine = o[i];
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1 << l);
        o[i] = up ? other : mine;
        o[i + S] = up ? mine : other;
      }
    }
  }
}

template <typename T, int DH, int NQ>
__device__ __forceinline__ void issue_stage(const DecodeParams& p, const Seg& S, int h, int r_base, int cnt,
                                            unsigned char* stage, uint64_t* bar, int lane) {
  using C = DecodeCfg<T, DH, NQ>;
  if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(cnt * C::ROWB * 2));
  __syncwarp();
  const int win0 = S.k_len - S.q_len;  // first window key (appended rows)
  if (lane < cnt) {
    const int k = lane;
    const int r = r_base + k;
    const T* ksrc;
    const T* vsrc;
    if (S.new_row0 >= 0 && r >= win0) {
      const long long row = (long long)S.new_row0 + (r - win0);
      ksrc = static_cast<const T*>(p.k_new) + (row * p.Hkv + h) * DH;
      vsrc = static_cast<const T*>(p.v_new) + (row * p.Hkv + h) * DH;
    } else {
      const long long row = S.k_row0 + p.k_row_offset + r;
      ksrc = static_cast<const T*>(p.k) + (row * p.Hkv + h) * DH;
      vsrc = static_cast<const T*>(p.v) + (row * p.Hkv + h) * DH;
    }
    bulk_g2s(stage + k * C::ROWB, ksrc, C::ROWB, bar);
    bulk_g2s(stage + C::KPW * C::ROWB + k * C::ROWB, vsrc, C::ROWB, bar);
  }
}

template <typename T, int DH, int NQ>
__global__ void __launch_bounds__(128) wave_decode_kernel(const DecodeParams p) {
  using C = DecodeCfg<T, DH, NQ>;
  constexpr int VEC = C::VEC;
  constexpr int P = C::P;
  constexpr int TK = C::TK;
  constexpr int LANES = C::LANES;
  const float NEG_INF = -__int_as_float(0x7f800000);

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full_bar[C::NWARPS][C::STAGES];
  __shared__ int s_flag;
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane / LANES, lig = lane % LANES;
  const int gbase = grp * LANES;

  if (tid == 0) {
    for (int w = 0; w < C::NWARPS; ++w)
      for (int s = 0; s < C::STAGES; ++s) mbar_init(&full_bar[w][s], 1);
    fence_mbar_init();
    s_abort = 0;
  }
  griddep_wait();  // plan outputs (segs, prefix) and the workspace
  __syncthreads();
  unsigned char* const wbase = smem + warp * C::WARP_BYTES;  // this warp's stage ring
  uint64_t* const wbar = full_bar[warp];

  const long long total = (long long)p.Hkv * p.prefix[p.n_segs];
  if (total <= 0) return;
  const long long share = (total + gridDim.x - 1) / gridDim.x;
  const long long a = (long long)blockIdx.x * share;
  if (a >= total) return;
  const long long b = (a + share < total) ? a + share : total;

  // this lane's (key, query) pair after the reduce-scatter
  const int jp = bitrev(lig & (P - 1), C::LOGP);
  const int t_j = jp / NQ, nq_j = jp % NQ;
  const bool pair_writer = (t_j == 0) && (lig < P);

  // last segment whose flattened start is <= a
  int seg;
  {
    int lo = 0, hi = p.n_segs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((long long)p.Hkv * p.prefix[mid] <= a) lo = mid;
      else hi = mid - 1;
    }
    seg = lo;
  }

  uint32_t gs = 0;  // this warp's stages consumed so far (mbarrier phase bookkeeping)
  long long pos = a;
  while (pos < b) {
    while (seg + 1 <= p.n_segs - 1 && (long long)p.Hkv * p.prefix[seg + 1] <= pos) ++seg;
    const Seg S = p.segs[seg];
    const long long seg_base = (long long)p.Hkv * p.prefix[seg];
    const long long o = pos - seg_base;
    const int u = (int)(o / S.k_len);
    const int r_lo = (int)(o - (long long)u * S.k_len);
    const long long unit_start = seg_base + (long long)u * S.k_len;
    const long long unit_end = unit_start + S.k_len;
    const int r_hi = (int)(((unit_end < b) ? unit_end : b) - unit_start);
    const int qg = u / p.Hkv, h = u % p.Hkv;
    pos = unit_start + r_hi;

    // ---- query vectors of this unit (pre-scaled into the log2 domain) ----
    float2 qv[NQ][VEC / 2];
    int lim_j = -1;
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq) {
      const int vq = qg * NQ + nq;
      const bool valid = vq < S.q_len * p.G;
      const int row = valid ? vq / p.G : 0;
      const int g = valid ? vq % p.G : 0;
      float f[VEC];
      if (valid) {
        const T* src = static_cast<const T*>(p.q) + ((long long)(S.q_row0 + row) * p.Hq + h * p.G + g) * DH + lig * VEC;
        Elem<T>::unpack(ld_nc_v4(src), f);
      } else {
#pragma unroll
        for (int d = 0; d < VEC; ++d) f[d] = 0.f;
      }
#pragma unroll
      for (int d = 0; d < VEC / 2; ++d) qv[nq][d] = make_float2(f[2 * d] * p.scale_log2, f[2 * d + 1] * p.scale_log2);
      const int lim = !valid ? -1 : (p.causal ? S.k_len - S.q_len + row : S.k_len - 1);
      if (nq == nq_j) lim_j = lim;
    }

    // ---- online softmax state ----
    float m_run = NEG_INF, l_run = 0.f;
    float2 ov[NQ][VEC / 2];
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
      for (int d = 0; d < VEC / 2; ++d) ov[nq][d] = make_float2(0.f, 0.f);

    const int n_keys = r_hi - r_lo;
    // warp w takes keys [n*KPS + w*KPW, +KPW) of every CTA-wide stage n
    const int wk0 = warp * C::KPW;
    const int n_st = (n_keys > wk0) ? (n_keys - wk0 + C::KPS - 1) / C::KPS : 0;

    // ring prologue (the previous unit's merge used the same smem: order the
    // generic-proxy writes before the bulk copies)
    __syncthreads();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int n = 0; n < n_st && n < C::STAGES; ++n) {
      const int buf = (int)((gs + n) % C::STAGES);
      const int cnt = cmin(C::KPW, n_keys - (n * C::KPS + wk0));
      issue_stage<T, DH, NQ>(p, S, h, r_lo + n * C::KPS + wk0, cnt, wbase + buf * C::WSTAGE_BYTES, &wbar[buf], lane);
    }

    const int kb = grp * TK;  // my first key inside this warp's stage
    int n_stop = n_st;        // first stage not consumed (abort bookkeeping)
    bool abort_w = false;
    for (int n = 0; n < n_st; ++n) {
      const int buf = (int)((gs + n) % C::STAGES);
      const uint32_t par = ((gs + n) / C::STAGES) & 1u;
      const int cnt = cmin(C::KPW, n_keys - (n * C::KPS + wk0));
      const int rb = r_lo + n * C::KPS + wk0;
      abort_w = __any_sync(0xffffffffu, !mbar_wait_bounded(&wbar[buf], par));
      const unsigned char* kst = wbase + buf * C::WSTAGE_BYTES;
      const unsigned char* vst = kst + C::KPW * C::ROWB;

      // scores
      float part[P];
#pragma unroll
      for (int t = 0; t < TK; ++t) {
        const int kidx = kb + t;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (kidx < cnt) raw = *reinterpret_cast<const uint4*>(kst + kidx * C::ROWB + lig * 16);
        float kf[VEC];
        Elem<T>::unpack(raw, kf);
#pragma unroll
        for (int nq = 0; nq < NQ; ++nq) {
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int d = 0; d < VEC / 2; ++d) acc = __ffma2_rn(qv[nq][d], make_float2(kf[2 * d], kf[2 * d + 1]), acc);
          part[t * NQ + nq] = acc.x + acc.y;
        }
      }
      float s = reduce_scatter<P>(part, lig);
#pragma unroll
      for (int l = C::LOGP; l < C::LOGL; ++l) s += __shfl_xor_sync(0xffffffffu, s, 1 << l);
      {
        const int kj = kb + t_j;
        const bool ok = (kj < cnt) && (rb + kj <= lim_j);
        s = ok ? s : NEG_INF;
      }
      float tmax = s;
#pragma unroll
      for (int msk = 1; msk < TK; msk <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, msk));
      const float m_new = fmaxf(m_run, tmax);
      const float alpha = (m_new == NEG_INF) ? 1.f : fast_exp2(m_run - m_new);
      const float pj = (s == NEG_INF) ? 0.f : fast_exp2(s - m_new);
      l_run = l_run * alpha + pj;
      m_run = m_new;

      float pall[P];
      all_gather<P>(pj, pall, lig);

      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int nq = 0; nq < NQ; ++nq) {
          const float an = __shfl_sync(0xffffffffu, alpha, gbase + bitrev(nq, C::LOGP));
          const float2 a2 = make_float2(an, an);
#pragma unroll
          for (int d = 0; d < VEC / 2; ++d) ov[nq][d] = __fmul2_rn(ov[nq][d], a2);
        }
      }
#pragma unroll
      for (int t = 0; t < TK; ++t) {
        const int kidx = kb + t;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (kidx < cnt) raw = *reinterpret_cast<const uint4*>(vst + kidx * C::ROWB + lig * 16);
        float vf[VEC];
        Elem<T>::unpack(raw, vf);
#pragma unroll
        for (int nq = 0; nq < NQ; ++nq) {
          const float pv = pall[t * NQ + nq];
          const float2 p2 = make_float2(pv, pv);
#pragma unroll
          for (int d = 0; d < VEC / 2; ++d) ov[nq][d] = __ffma2_rn(p2, make_float2(vf[2 * d], vf[2 * d + 1]), ov[nq][d]);
        }
      }

      __syncwarp();  // every lane of this warp is done with the buffer
      if (abort_w) {
        n_stop = n;
        break;
      }
      if (n + C::STAGES < n_st) {
        const int n2 = n + C::STAGES;
        const int cnt2 = cmin(C::KPW, n_keys - (n2 * C::KPS + wk0));
        issue_stage<T, DH, NQ>(p, S, h, r_lo + n2 * C::KPS + wk0, cnt2, wbase + buf * C::WSTAGE_BYTES, &wbar[buf],
                               lane);
      }
    }
    if (abort_w) {
      // a bounded wait gave up: drain this warp's copies that can still be in
      // flight (stages n_stop .. n_stop+STAGES-1), then leave with the CTA
      if (lane == 0) {
        set_error(p.err, kErrTimeout);
        for (int n = n_stop; n < n_st && n < n_stop + C::STAGES; ++n)
          mbar_wait_bounded(&wbar[(gs + n) % C::STAGES], ((gs + n) / C::STAGES) & 1u);
        s_abort = 1;
      }
    }
    gs += (uint32_t)n_st;
    float l_sum = l_run;
#pragma unroll
    for (int msk = 1; msk < TK; msk <<= 1) l_sum += __shfl_xor_sync(0xffffffffu, l_sum, msk);
    __syncthreads();  // all warps done with their rings: smem becomes the merge buffer
    if (s_abort) return;

    // ---- merge the NG softmax states of this CTA ----
    float* m_s = reinterpret_cast<float*>(smem);
    float* l_s = m_s + C::NG * NQ;
    float* o_s = l_s + C::NG * NQ;
    const int gg = warp * C::GROUPS + grp;
    if (pair_writer) {
      m_s[gg * NQ + nq_j] = m_run;
      l_s[gg * NQ + nq_j] = l_sum;
    }
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq) {
      float* dst = o_s + ((size_t)gg * NQ + nq) * DH + lig * VEC;
#pragma unroll
      for (int d = 0; d < VEC / 2; ++d) *reinterpret_cast<float2*>(dst + 2 * d) = ov[nq][d];
    }
    __syncthreads();

    const int c_first = (int)(unit_start / share);
    const int c_last = (int)((unit_end - 1) / share);
    const int n_contrib = c_last - c_first + 1;
    constexpr int VPR = DH / VEC;
    float* part_base = nullptr;
    if (n_contrib > 1) {
      const int slot = (unit_start < a) ? 2 * (int)blockIdx.x : 2 * (int)blockIdx.x + 1;
      part_base = p.ws_part + (size_t)slot * C::PART_FLOATS;
    }
    for (int c = tid; c < NQ * VPR; c += C::THREADS) {
      const int nq = c / VPR, d0 = (c % VPR) * VEC;
      float M = NEG_INF;
#pragma unroll
      for (int g2 = 0; g2 < C::NG; ++g2) M = fmaxf(M, m_s[g2 * NQ + nq]);
      float L = 0.f, acc[VEC];
#pragma unroll
      for (int d = 0; d < VEC; ++d) acc[d] = 0.f;
#pragma unroll
      for (int g2 = 0; g2 < C::NG; ++g2) {
        const float mg = m_s[g2 * NQ + nq];
        const float w = (mg == NEG_INF) ? 0.f : fast_exp2(mg - M);
        L += w * l_s[g2 * NQ + nq];
        const float* src = o_s + ((size_t)g2 * NQ + nq) * DH + d0;
#pragma unroll
        for (int d = 0; d < VEC; ++d) acc[d] += w * src[d];
      }
      if (n_contrib == 1) {
        const int vq = qg * NQ + nq;
        if (vq < S.q_len * p.G) {
          const int row = vq / p.G, g = vq % p.G;
          const float inv = (L > 0.f) ? 1.f / L : 0.f;
          float r[VEC];
#pragma unroll
          for (int d = 0; d < VEC; ++d) r[d] = acc[d] * inv;
          T* dst = static_cast<T*>(p.out) + ((long long)(S.q_row0 + row) * p.Hq + h * p.G + g) * DH + d0;
          *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(r);
        }
      } else {
        if (d0 == 0) {
          part_base[nq] = M;
          part_base[NQ + nq] = L;
        }
        float* dst = part_base + 2 * NQ + nq * DH + d0;
#pragma unroll
        for (int d = 0; d < VEC; ++d) dst[d] = acc[d];
      }
    }

    if (n_contrib > 1) {
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const int prev = atomicAdd(p.ws_cnt + c_first, 1);
        s_flag = (prev == n_contrib - 1) ? 1 : 0;
      }
      __syncthreads();
      if (s_flag) {
        __threadfence();
        for (int c = tid; c < NQ * VPR; c += C::THREADS) {
          const int nq = c / VPR, d0 = (c % VPR) * VEC;
          float M = NEG_INF;
          for (int k = 0; k < n_contrib; ++k) {
            const int cc = c_first + k;
            const int slot = (k == 0) ? 2 * cc + 1 : 2 * cc;
            M = fmaxf(M, ld_cg_f32(p.ws_part + (size_t)slot * C::PART_FLOATS + nq));
          }
          float L = 0.f, acc[VEC];
#pragma unroll
          for (int d = 0; d < VEC; ++d) acc[d] = 0.f;
          for (int k = 0; k < n_contrib; ++k) {
            const int cc = c_first + k;
            const int slot = (k == 0) ? 2 * cc + 1 : 2 * cc;
            const float* base = p.ws_part + (size_t)slot * C::PART_FLOATS;
            const float mk = ld_cg_f32(base + nq);
            const float w = (mk == NEG_INF) ? 0.f : fast_exp2(mk - M);
            L += w * ld_cg_f32(base + NQ + nq);
            const float* src = base + 2 * NQ + nq * DH + d0;
#pragma unroll
            for (int d = 0; d < VEC; ++d) acc[d] += w * ld_cg_f32(src + d);
          }
          const int vq = qg * NQ + nq;
          if (vq < S.q_len * p.G) {
            const int row = vq / p.G, g = vq % p.G;
            const float inv = (L > 0.f) ? 1.f / L : 0.f;
            float r[VEC];
#pragma unroll
            for (int d = 0; d < VEC; ++d) r[d] = acc[d] * inv;
            T* dst = static_cast<T*>(p.out) + ((long long)(S.q_row0 + row) * p.Hq + h * p.G + g) * DH + d0;
            *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(r);
          }
        }
        if (tid == 0) p.ws_cnt[c_first] = 0;  // leave the counter zeroed for the next launch
      }
    }
  }
}

}  // namespace wfd
