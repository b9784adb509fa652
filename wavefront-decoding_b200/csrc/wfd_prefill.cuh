// K7 — dense prompt (prefill) attention on the tcgen05 tensor cores, bf16,
// head_dim 64 or 128: the causal attention over (B, L) that the prompt pass of
// every layer runs (reference: write_prefill + attn_dense, ouro_blocks_batch.py:123-144,
// fa4_attention.py:191-232), for B segments of Lq query rows over Lk key rows
// (bottom-right causal: row i sees keys j <= i + Lk - Lq).
//
// Unlike the decode / verify kernel (K2, swap-AB with a few query columns), a
// prompt has many query rows per head, so the MMAs run query-major:
//     S[128 q x 128 keys]  = Q[128 x Dh] . K_tile^T          (A = Q, B = K, both K-major)
//     O_t[128 q x Dh]      = P[128 x 128 keys] . V_tile       (A = P K-major, B = V MN-major)
// with S (double-buffered) and O_t in TMEM.  Each softmax thread owns one query
// row (its TMEM lane): row max and sum need no cross-thread reduction; it reads
// its S row twice from TMEM (max, then probabilities), writes its P row (bf16)
// to shared memory for the P.V MMA, and accumulates O_t into registers with
// the online-softmax rescale.
//
// Persistent grid: tiles (segment, query head, 128-row query block) are taken
// heaviest first (the causal key range grows with the query block) round-robin
// over the CTAs.  Warp 0 streams Q (two buffers) and the K/V tiles (a ring) by
// TMA, warp 1 issues the MMAs, warps 2..5 run the softmax.  Every wait is
// bounded; on an abort the CTA drains its copies and MMAs, frees TMEM and
// returns, with the error word set.
#pragma once

#include "wfd_verify.cuh"

namespace wfd {

struct PrefillParams {
  void* out;  // (B * Lq, Hq, Dh) bf16
  int n_seqs, Lq, Lk, Hq, Hkv, G;
  int causal;
  int n_qb;  // query blocks per segment
  float scale_log2;
  int* err;
};

template <int DH>
struct PfCfg {
  static constexpr int KB = DH / 64;              // 64-dim boxes of a Q / K / V tile
  static constexpr int BOX = 128 * 128;           // 128 rows x 128 B (64 bf16), SWIZZLE_128B
  static constexpr int Q_BYTES = KB * BOX;
  static constexpr int KV_STAGE = 2 * KB * BOX;   // K boxes, then V boxes
  static constexpr int STAGES = DH == 64 ? 3 : 2;
  static constexpr int P_BYTES = 2 * BOX;         // 128 q rows x 128 keys bf16: keys 0-63, 64-127
  static constexpr int SMEM = 2 * Q_BYTES + STAGES * KV_STAGE + P_BYTES + 1024;
  static constexpr int TMEM_COLS = 512;           // S x 2 (128 columns each), O_t (DH)
  static constexpr int O_COL = 256;
  static_assert(DH == 64 || DH == 128, "head dim");
  static_assert(SMEM + 2048 <= 232448, "shared memory per CTA (dynamic + the kernel's static arrays)");
};

constexpr int kPfThreads = 320;  // TMA warp, MMA warp, 8 softmax warps

// 2^x with the MUFU approximation (ex2.approx.ftz.f32): the probabilities are
// rounded to bf16 for the P.V MMA, far coarser than its error.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void pf_tile(const PrefillParams& p, int t, int& b, int& hq, int& qb, int& nk, int& d) {
  const int per_qb = p.n_seqs * p.Hq;
  qb = p.n_qb - 1 - t / per_qb;  // heaviest query blocks first
  const int rem = t % per_qb;
  b = rem / p.Hq;
  hq = rem % p.Hq;
  d = p.Lk - p.Lq;
  const int nkb = (p.Lk + 127) / 128;
  int last = nkb - 1;
  if (p.causal) {
    const long long lim = (long long)qb * 128 + 127 + d;  // largest key the block's last row sees
    if (lim < 0) {
      last = -1;
    } else if (lim / 128 < last) {
      last = (int)(lim / 128);
    }
  }
  nk = last + 1;
}

template <int DH>
__global__ void __launch_bounds__(kPfThreads)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using C = PfCfg<DH>;
  constexpr int STAGES = C::STAGES;
  constexpr int KB = C::KB;
  const float NEG_INF = -__int_as_float(0x7f800000);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qs = smem;                          // 2 x Q tile
  unsigned char* kvs = qs + 2 * C::Q_BYTES;          // STAGES x (K boxes, V boxes)
  unsigned char* ps = kvs + STAGES * C::KV_STAGE;    // P tile (A operand, K-major, SW128)

  __shared__ __align__(8) uint64_t bar_full[STAGES];
  __shared__ __align__(8) uint64_t bar_empty[STAGES];
  __shared__ __align__(8) uint64_t bar_qfull[2];
  __shared__ __align__(8) uint64_t bar_qfree[2];
  __shared__ __align__(8) uint64_t bar_sfull[2];
  __shared__ __align__(8) uint64_t bar_sfree[2];
  __shared__ __align__(8) uint64_t bar_pfull;
  __shared__ __align__(8) uint64_t bar_ofull;
  __shared__ __align__(8) uint64_t bar_ofree;
  __shared__ __align__(8) uint64_t bar_drain;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ float s_xch[256];  // per row and key half: the tile's maximum, at the end the sum

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_q)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_k)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_v)) : "memory");
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_qfull[s], 1);
      mbar_init(&bar_qfree[s], 1);
      mbar_init(&bar_sfull[s], 1);
      mbar_init(&bar_sfree[s], 8);
    }
    mbar_init(&bar_pfull, 8);
    mbar_init(&bar_ofull, 1);
    mbar_init(&bar_ofree, 8);
    mbar_init(&bar_drain, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  griddep_wait();  // q / k / v come from the predecessor
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int n_tiles = p.n_seqs * p.Hq * p.n_qb;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    uint32_t it = 0, n_iss = 0, ti = 0, q_iss = 0;  // issued K/V tiles and Q tiles form prefixes (issue stops at an abort)
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++ti) {
      int b, hq, qb, nk, d;
      pf_tile(p, t, b, hq, qb, nk, d);
      const int hk = hq / p.G;
      const int qbuf = (int)(ti & 1u);
      const bool qgo = ti >= 2 ? tc_wait(&bar_qfree[qbuf], ((ti >> 1) - 1) & 1u, &s_abort, p.err) : !s_abort;
      if (qgo && lane == 0) {
        mbar_arrive_expect_tx(&bar_qfull[qbuf], (uint32_t)C::Q_BYTES);
#pragma unroll
        for (int bx = 0; bx < KB; ++bx)
          tma_load_3d(qs + qbuf * C::Q_BYTES + bx * C::BOX, &tm_q, 64 * bx, hq, b * p.Lq + qb * 128, &bar_qfull[qbuf]);
        q_iss = ti + 1;
      }
      __syncwarp();
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int stage = (int)(it % STAGES);
        const bool go = it >= (uint32_t)STAGES ? tc_wait(&bar_empty[stage], ((it / STAGES) - 1) & 1u, &s_abort, p.err)
                                               : !s_abort;
        if (go && lane == 0) {
          unsigned char* dst = kvs + stage * C::KV_STAGE;
          mbar_arrive_expect_tx(&bar_full[stage], (uint32_t)C::KV_STAGE);
#pragma unroll
          for (int bx = 0; bx < KB; ++bx) {
            tma_load_3d(dst + bx * C::BOX, &tm_k, 64 * bx, hk, b * p.Lk + kb * 128, &bar_full[stage]);
            tma_load_3d(dst + (KB + bx) * C::BOX, &tm_v, 64 * bx, hk, b * p.Lk + kb * 128, &bar_full[stage]);
          }
          n_iss = it + 1;
        }
        __syncwarp();
      }
    }
    // copies in flight land before the CTA exits (also after an abort): the last
    // phase of every stage filled, and the Q buffers
    if (lane == 0) {
      for (uint32_t j = (n_iss > (uint32_t)STAGES ? n_iss - STAGES : 0); j < n_iss; ++j)
        if (!mbar_wait_bounded(&bar_full[j % STAGES], (j / STAGES) & 1u)) set_error(p.err, kErrTimeout);
      for (uint32_t k = (q_iss > 2 ? q_iss - 2 : 0); k < q_iss; ++k)
        if (!mbar_wait_bounded(&bar_qfull[k & 1u], (k >> 1) & 1u)) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC_S = umma_idesc(128, false, false);
    constexpr uint32_t IDESC_PV = umma_idesc(DH, false, true);
    uint32_t it = 0, pv = 0, ti = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++ti) {
      int b, hq, qb, nk, d;
      pf_tile(p, t, b, hq, qb, nk, d);
      const int qbuf = (int)(ti & 1u);
      const uint32_t qa = smem_u32(qs + qbuf * C::Q_BYTES);
      tc_wait(&bar_qfull[qbuf], (ti >> 1) & 1u, &s_abort, p.err);
      tc_fence_after();
      if (nk == 0) {  // no key visible: release the Q buffer at once
        if (lane == 0) umma_commit(&bar_qfree[qbuf]);
        __syncwarp();
        continue;
      }
      for (int kb = 0; kb <= nk; ++kb) {
        if (kb < nk) {
          const uint32_t ik = it + kb;
          const int stage = (int)(ik % STAGES);
          const int sb = (int)(ik & 1u);
          bool go = tc_wait(&bar_full[stage], (ik / STAGES) & 1u, &s_abort, p.err);
          if (ik >= 2) go = tc_wait(&bar_sfree[sb], ((ik >> 1) - 1) & 1u, &s_abort, p.err) && go;
          tc_fence_after();
          if (go && lane == 0) {
            const uint32_t k_addr = smem_u32(kvs + stage * C::KV_STAGE);
#pragma unroll
            for (int j = 0; j < DH / 16; ++j) {
              const uint32_t off = (uint32_t)((j >> 2) * C::BOX + (j & 3) * 32);
              umma_f16(tmem + (uint32_t)(sb * 128), umma_desc(qa + off, 16, 1024, 2), umma_desc(k_addr + off, 16, 1024, 2),
                       IDESC_S, j > 0 ? 1u : 0u);
            }
            umma_commit(&bar_sfull[sb]);
            if (kb == nk - 1) umma_commit(&bar_qfree[qbuf]);
          }
          __syncwarp();
        }
        if (kb >= 1) {
          bool go = tc_wait(&bar_pfull, pv & 1u, &s_abort, p.err);
          if (pv >= 1) go = tc_wait(&bar_ofree, (pv - 1) & 1u, &s_abort, p.err) && go;
          tc_fence_after();
          const int stage = (int)((it + kb - 1) % STAGES);
          if (go && lane == 0) {
            const uint32_t v_addr = smem_u32(kvs + stage * C::KV_STAGE + KB * C::BOX);
            const uint32_t p_addr = smem_u32(ps);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // keys 16j .. 16j + 15: P bytes 32 (j % 4) of box j / 4; V rows 16j.. (2048 B per 16 rows)
              umma_f16(tmem + (uint32_t)C::O_COL, umma_desc(p_addr + (j >> 2) * C::BOX + (j & 3) * 32, 16, 1024, 2),
                       umma_desc(v_addr + j * 2048, C::BOX, 1024, 2), IDESC_PV, j > 0 ? 1u : 0u);
            }
            umma_commit(&bar_ofull);
            umma_commit(&bar_empty[stage]);
          }
          __syncwarp();
          ++pv;
        }
      }
      it += nk;
    }
    if (lane == 0) {
      umma_commit(&bar_drain);
      if (!mbar_wait_bounded(&bar_drain, 0)) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    // 8 warps: warp w reads TMEM lane quadrant w % 4 (32 query rows) and key
    // half h = (w - 2) / 4 of every S tile (64 keys), writes that half of the
    // rows' P and accumulates half of their O columns; the two halves of a row
    // exchange their maxima (and, at the end, their sums) through shared memory.
    const int qd = warp & 3;
    const int row = qd * 32 + lane;                 // query row of the tile == TMEM lane
    const int h = (warp - 2) >> 2;                  // key half / O-column half
    constexpr int OH = DH / 2;                      // O columns per thread
    const uint32_t tq = tmem + ((uint32_t)(qd * 32) << 16);
    const float c2 = p.scale_log2;
    uint32_t it = 0, pv = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      int b, hq, qb, nk, d;
      pf_tile(p, t, b, hq, qb, nk, d);
      const int grow = qb * 128 + row;              // query row within its segment
      const int klim = grow + d;                    // causal: last visible key
      const int tile_klim = qb * 128 + d;           // the smallest limit of the tile's rows
      float m = NEG_INF, l = 0.f, a_pend = 1.f;
      float oacc[OH];
#pragma unroll
      for (int e = 0; e < OH; ++e) oacc[e] = 0.f;
      for (int kb = 0; kb < nk; ++kb) {
        const uint32_t ik = it + kb;
        const int sb = (int)(ik & 1u);
        tc_wait(&bar_sfull[sb], (ik >> 1) & 1u, &s_abort, p.err);
        tc_fence_after();
        const int key0 = kb * 128 + h * 64;
        // keys past the segment or the causal limit: only the tile's boundary blocks have any
        const bool edge = kb * 128 + 127 >= p.Lk || (p.causal && kb * 128 + 127 > tile_klim);
        // this thread's 64 scores of the tile, in NV loads of 64 / NV columns (head_dim 128
        // keeps 32 at a time in registers and reads them twice)
        constexpr int NV = DH == 64 ? 1 : 2;
        constexpr int VW = 64 / NV;
        float v[VW];
        auto load_scores = [&](int part) {
#pragma unroll
          for (int c = 0; c < VW / 32; ++c)
            tmem_ld<32>(tq + (uint32_t)(sb * 128 + h * 64 + part * VW + c * 32),
                        *reinterpret_cast<float(*)[32]>(v + c * 32));
          tc_wait_ld();
          if (edge) {
#pragma unroll
            for (int e = 0; e < VW; ++e) {
              const int key = key0 + part * VW + e;
              if (!(key < p.Lk && (!p.causal || key <= klim))) v[e] = NEG_INF;
            }
          }
        };
        float mx0 = NEG_INF, mx1 = NEG_INF, mx2 = NEG_INF, mx3 = NEG_INF;
#pragma unroll
        for (int part = 0; part < NV; ++part) {
          if (NV > 1 || part == 0) load_scores(part);
#pragma unroll
          for (int e = 0; e < VW; e += 4) {
            mx0 = fmaxf(mx0, v[e]);
            mx1 = fmaxf(mx1, v[e + 1]);
            mx2 = fmaxf(mx2, v[e + 2]);
            mx3 = fmaxf(mx3, v[e + 3]);
          }
        }
        s_xch[h * 128 + row] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        softmax_bar<256>();
        const float mx = fmaxf(s_xch[row], s_xch[128 + row]);
        softmax_bar<256>();  // both halves have read: s_xch may be rewritten
        const float mn = (mx == NEG_INF) ? m : fmaxf(m, mx * c2);
        const float alpha = (m == NEG_INF || mn == NEG_INF) ? 1.f : ex2_approx(m - mn);
        // the previous tile's P.V: its MMA is done with P once o_full fires
        if (kb >= 1) {
          tc_wait(&bar_ofull, pv & 1u, &s_abort, p.err);
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < OH / 32; ++c) {
            float o[32];
            tmem_ld<32>(tq + (uint32_t)(C::O_COL + h * OH + c * 32), o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) oacc[c * 32 + e] = fmaf(oacc[c * 32 + e], a_pend, o[e]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_ofree);
          ++pv;
        }
        // probabilities (bf16) into this half of the row of P (box h), and their sum
        const float nm = (mn == NEG_INF) ? 0.f : -mn;
        float sum = 0.f;
        unsigned char* prow = ps + h * C::BOX + row * 128;
#pragma unroll
        for (int part = 0; part < NV; ++part) {
          if (NV > 1) load_scores(part);  // one part: the scores are still in registers
#pragma unroll
          for (int cq = 0; cq < VW / 8; ++cq) {
            const int ch = part * (VW / 8) + cq;  // 16-byte chunk (8 keys) of the row in box h
            uint32_t w[4];
#pragma unroll
            for (int e2 = 0; e2 < 4; ++e2) {
              const float p0 = ex2_approx(fmaf(v[cq * 8 + 2 * e2], c2, nm));
              const float p1 = ex2_approx(fmaf(v[cq * 8 + 2 * e2 + 1], c2, nm));
              sum += p0 + p1;
              __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
              w[e2] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        l = l * alpha + sum;
        m = mn;
        a_pend = alpha;
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bar_sfree[sb]);
          mbar_arrive(&bar_pfull);
        }
      }
      if (nk > 0) {
        tc_wait(&bar_ofull, pv & 1u, &s_abort, p.err);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < OH / 32; ++c) {
          float o[32];
          tmem_ld<32>(tq + (uint32_t)(C::O_COL + h * OH + c * 32), o);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) oacc[c * 32 + e] = fmaf(oacc[c * 32 + e], a_pend, o[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_ofree);
        ++pv;
      }
      it += nk;
      // the row's sum: both halves
      s_xch[h * 128 + row] = l;
      softmax_bar<256>();
      const float lt = s_xch[row] + s_xch[128 + row];
      softmax_bar<256>();                            // s_xch is rewritten by the next tile
      if (grow < p.Lq) {
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        __nv_bfloat16* orow =
            static_cast<__nv_bfloat16*>(p.out) + ((long long)(b * p.Lq + grow) * p.Hq + hq) * DH + h * OH;
#pragma unroll
        for (int c = 0; c < OH / 8; ++c) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = oacc[c * 8 + e] * inv;
          reinterpret_cast<uint4*>(orow)[c] = Elem<__nv_bfloat16>::pack(f);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
}

}  // namespace wfd
