// K8 — the skinny linear layers of a looped-LM block on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA, sm_100a), bf16, for unions of at most a few dozen
// rows, with the block's element-wise work fused around them.
//
// Swap-AB: per 128-feature tile of W (K x F, row-major, features contiguous)
//     Y^T[128 features x NP rows] += W_tile^T[128 x 128 k] . X^T      (A = W, MN-major; B = X, K-major)
// so the output features fill the MMA's M = 128 and the few rows are its N (16,
// 32 or 64).  A CTA owns one feature tile and one range of 128-row k stages;
// the k ranges of a tile (the split, at most 8) form one thread-block cluster.
// Row r of the tile is finished by cluster CTA r % split: as soon as its MMAs are
// done, each CTA stores its partial sums of a row into the owner's receive area
// (st.shared::cluster; the area is used once per launch and never initialised,
// so a store may land before the owner runs), and after one cluster barrier the
// owner adds them in rank order (deterministic; the order does not depend on the
// row count, so a row's result does not depend on the other rows of the launch).
//
// The block's element-wise work rides on the same launch:
//   row norm   RMSNorm folded in: the norm weight is pre-multiplied into W's rows
//              and each CTA sums x^2 over its k range; the merge scales row r by
//              rsqrt(sum / K + eps)
//   plain      y (n, F) bf16 (the lm_head)
//   residual   out (n, F) += y, in place (o_proj, SwiGLU down projection)
//   swiglu     W's columns interleave gate and up per 64 (tile j = gate features
//              64j.., then up features 64j..): out (n, F/2) = silu(g) * u
//   rope       RoPE at each row's position and the split into q / k / v of the
//              fused QKV projection (pairs (i, i + Dh/2) or (2i, 2i + 1) of a head
//              lie in one tile)
// Each output is rounded to bf16 where the unfused chain stores bf16 (the GEMM
// output before RoPE / SwiGLU), so the results follow that chain's arithmetic.
//
// Warp roles (192 threads): warp 0 TMA producer (W tiles, then X tiles), warp 1
// TMEM allocator + MMA issuer, warps 2..5 epilogue (warp w reads TMEM lane
// quadrant w % 4 = features 32 (w % 4) ..).  Launched with programmatic stream
// serialization: the producer issues the W loads of its first stages before
// griddep_wait(), so the weights stream while the previous kernel finishes;
// X (the MMAs' B operand, also the row norms' input) and every output are
// touched only after it.
// Every mbarrier wait is bounded; the cluster barrier is reached by every thread
// of every CTA whatever happens (a thread-block cluster's CTAs are resident
// together, so a peer's shared memory exists from the start).  No multicast.
#pragma once

#include <cuda.h>

#include "wfd_verify.cuh"

namespace wfd {

enum LinearMode { kLinPlain = 0, kLinResidual = 1, kLinSwiglu = 2, kLinRope = 3 };

struct LinearParams {
  int n_rows, K, F;        // W is (K, F) row-major
  int n_k;                 // 128-row k stages: ceil(K / 128)
  int n_tiles;             // 128-feature tiles: ceil(F / 128)
  int split;               // CTAs per feature tile (contiguous k-stage ranges) = the cluster size, <= 8
  int mode, row_norm;
  float eps;
  __nv_bfloat16* out;      // plain: (n, F); residual: (n, F) in place; swiglu: (n, F / 2)
  int ldo;
  __nv_bfloat16 *q, *k, *v;  // rope: q (n, H, Dh), k / v (n, Hkv, Dh), contiguous
  int H, Hkv, Dh, style;
  const float *cosb, *sinb;  // (max_pos, Dh / 2) fp32
  const int32_t* pos;        // row r at pos[r * pos_stride]; null: r % pos_period
  int pos_stride, pos_period, max_pos;
  int* err;
};

constexpr int kLinThreads = 192;
constexpr int kLinTile = 128;

template <int NP>
struct LinCfg {
  static constexpr int STAGES = 2;                 // W ring (a CTA holds 1-6 k stages)
  static constexpr int A_BOX = kLinTile * 128;     // 128 k rows x 64 features (128 B)
  static constexpr int A_BYTES = 2 * A_BOX;        // 128 features
  static constexpr int B_BOX = NP * 128;           // NP rows x 64 k
  static constexpr int B_BYTES = 2 * B_BOX;        // 128 k
  static constexpr int XR = 4;                     // rows per merge batch
  static constexpr int XBUF = XR * kLinTile * 4;   // feature exchange of one batch
  // accumulator chains (k steps alternate between them; summed in the epilogue):
  // the same for every NP, so a row's sum order does not depend on the row count
  static constexpr int CH = 2;
  static constexpr int TMEM_COLS = CH * NP <= 32 ? 32 : (CH * NP <= 64 ? 64 : 128);
  // receive area: from each of the (at most 8) CTAs of the cluster, partial sums
  // [rows][128] of the rows this CTA owns (ceil(NP / split)), then their row sums
  static constexpr int RECV_BYTES = (NP + 8) * kLinTile * 4 + 8 * NP * 4;
  static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + RECV_BYTES + XBUF + 1024;
  static_assert(NP == 16 || NP == 32 || NP == 64, "N of the swap-AB MMA");
  // up to 32 rows two CTAs share an SM (a CTA of the next launch can stream its
  // weights beside one of this launch); 64-row CTAs take an SM each
  static_assert(NP == 64 || 2 * (SMEM + 1024 + 1024) <= 233472, "shared memory");
  static_assert(SMEM + 2048 <= 232448, "shared memory");
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared-memory variable in cluster CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int NP>
__global__ void __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     const LinearParams p) {
  using C = LinCfg<NP>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ unsigned char lin_smem_raw[];
  unsigned char* sm =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(lin_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* as = sm;                                 // STAGES x W tile
  unsigned char* bs = sm + STAGES * C::A_BYTES;           // STAGES x X tile
  float* recv = reinterpret_cast<float*>(bs + STAGES * C::B_BYTES);   // [split][RL][128]
  float* recv_ss = recv + (NP + 8) * kLinTile;                           // [split][RL]
  float* xbuf = reinterpret_cast<float*>(bs + STAGES * C::B_BYTES + C::RECV_BYTES);

  __shared__ __align__(8) uint64_t bar_full[STAGES];
  __shared__ __align__(8) uint64_t bar_empty[STAGES];
  __shared__ __align__(8) uint64_t bar_done;   // every MMA of the CTA complete: accumulators readable
  __shared__ __align__(8) uint64_t bar_drain;  // the MMA warp's own completion check before exit
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ float s_ss[NP];  // this CTA's k range: sum of x^2 per row (read by the cluster's merge)
  __shared__ int s_pos[NP];   // rope: each row's position (checked), loaded during the main loop

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x / p.split, ks = blockIdx.x - tile * p.split;
  const int f0 = tile * kLinTile;
  const int k_lo = (int)(((long long)ks * p.n_k) / p.split);
  const int k_hi = (int)(((long long)(ks + 1) * p.n_k) / p.split);
  const int n_st = k_hi - k_lo;
  const int row0 = blockIdx.y * NP;

  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      // released by the MMA commit, and with the row norm by the 4 epilogue warps too
      mbar_init(&bar_empty[s], p.row_norm ? 5 : 1);
    }
    mbar_init(&bar_done, 1);
    mbar_init(&bar_drain, 1);
    fence_mbar_init();
    s_abort = 0;
    // the W tiles of the first stages go out at once: they do not depend on the
    // previous kernel, and they are the bulk of the bytes
    const int pre = n_st < STAGES ? n_st : STAGES;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&bar_full[i], (uint32_t)(C::A_BYTES + C::B_BYTES));
      const int kr = (k_lo + i) * kLinTile;
      tma_load_2d(as + i * C::A_BYTES, &tm_w, f0, kr, &bar_full[i]);
      tma_load_2d(as + i * C::A_BYTES + C::A_BOX, &tm_w, f0 + 64, kr, &bar_full[i]);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int split = p.split;
  const int rank = (int)cluster_rank();
  const int RL = (NP + split - 1) / split;  // rows each CTA of the cluster owns
  const int rows_here = min(NP, p.n_rows - row0);
  const int n_own = rank < rows_here ? (rows_here - rank + split - 1) / split : 0;
  // the next launch may start its own set-up and weight loads beside this CTA
  griddep_launch_dependents();

  float pacc[NP];  // epilogue warps: this CTA's partial sums, thread t = feature t
  // epilogue warps: feature t of the tile; per batch of owned rows the residual
  // rows and rotation angles, loaded ahead of the sums
  const int t = (warp & 3) * 32 + lane;
  const int f = f0 + t;
  const int half = p.Dh >> 1;
  const int hh = p.mode == kLinRope ? f / p.Dh : 0, ii = p.mode == kLinRope ? f - hh * p.Dh : 0;
  const bool first = p.style ? (ii & 1) == 0 : ii < half;
  const int pi = p.style ? (ii >> 1) : (ii < half ? ii : ii - half);  // rope: frequency index
  const bool rotate = p.mode == kLinRope && hh < p.H + p.Hkv;
  float base[C::XR], cs[C::XR], sn[C::XR];
  auto load_side = [&](int lb) {
#pragma unroll
    for (int i = 0; i < C::XR; ++i) {
      const int r = min(rank + (lb + i) * split, rows_here - 1);  // clamped: loads stay in range
      base[i] = 0.f;
      cs[i] = 1.f;
      sn[i] = 0.f;
      if (p.mode == kLinResidual && f < p.F) base[i] = __bfloat162float(p.out[(long long)(row0 + r) * p.ldo + f]);
      if (rotate) {
        const long long a = (long long)s_pos[r] * half + pi;
        cs[i] = p.cosb[a];
        sn[i] = p.sinb[a];
      }
    }
  };
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    const int pre = n_st < STAGES ? n_st : STAGES;  // W of these stages is already on its way
    griddep_wait();  // X is the previous kernel's output
    uint32_t n_iss = 0;
    if (lane == 0) {
      for (int i = 0; i < pre; ++i) {
        const int kr = (k_lo + i) * kLinTile;
        tma_load_2d(bs + i * C::B_BYTES, &tm_x, kr, row0, &bar_full[i]);
        tma_load_2d(bs + i * C::B_BYTES + C::B_BOX, &tm_x, kr + 64, row0, &bar_full[i]);
      }
      n_iss = (uint32_t)pre;
    }
    for (int i = pre; i < n_st; ++i) {
      const int stage = i % STAGES;
      const bool go = tc_wait(&bar_empty[stage], (uint32_t)((i / STAGES) - 1) & 1u, &s_abort, p.err);
      if (!go) break;
      if (lane == 0) {
        const int kr = (k_lo + i) * kLinTile;
        mbar_arrive_expect_tx(&bar_full[stage], (uint32_t)(C::A_BYTES + C::B_BYTES));
        tma_load_2d(as + stage * C::A_BYTES, &tm_w, f0, kr, &bar_full[stage]);
        tma_load_2d(as + stage * C::A_BYTES + C::A_BOX, &tm_w, f0 + 64, kr, &bar_full[stage]);
        tma_load_2d(bs + stage * C::B_BYTES, &tm_x, kr, row0, &bar_full[stage]);
        tma_load_2d(bs + stage * C::B_BYTES + C::B_BOX, &tm_x, kr + 64, row0, &bar_full[stage]);
        n_iss = (uint32_t)i + 1;
      }
      __syncwarp();
    }
    // copies in flight land before the CTA exits, also after an abort: the last
    // phase of every stage this lane filled (earlier phases completed before the
    // stage was refilled)
    if (lane == 0) {
      for (uint32_t j = (n_iss > (uint32_t)STAGES ? n_iss - STAGES : 0); j < n_iss; ++j)
        if (!mbar_wait_bounded(&bar_full[j % STAGES], (j / STAGES) & 1u)) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = umma_idesc(NP, true, false);
    for (int i = 0; i < n_st; ++i) {
      const int stage = i % STAGES;
      const bool go = tc_wait(&bar_full[stage], (uint32_t)(i / STAGES) & 1u, &s_abort, p.err);
      tc_fence_after();
      if (go && lane == 0) {
        const uint32_t a_addr = smem_u32(as + stage * C::A_BYTES);
        const uint32_t b_addr = smem_u32(bs + stage * C::B_BYTES);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // k step j: W rows 16j..16j+15 (two 8-row groups of both feature boxes);
          // X dims 16j.. = box j / 4, byte 32 (j % 4) inside the 128-byte row
          const int g = i * 8 + j;
          umma_f16(tmem + (uint32_t)((g % C::CH) * NP), umma_desc(a_addr + j * 2048, C::A_BOX, 1024, 2),
                   umma_desc(b_addr + (j >> 2) * C::B_BOX + (j & 3) * 32, 16, 1024, 2), IDESC,
                   g >= C::CH ? 1u : 0u);
        }
        umma_commit(&bar_empty[stage]);
      }
      __syncwarp();
      if (!go) break;
    }
    if (lane == 0) {
      umma_commit(&bar_done);
      // every MMA this lane issued is complete before TMEM is freed
      umma_commit(&bar_drain);
      if (!mbar_wait_bounded(&bar_drain, 0)) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int qd = warp & 3;              // TMEM lane quadrant (feature t = 32 qd + lane)
    const int ew = warp - 2;              // 0..3
    griddep_wait();                       // the outputs (and what the previous kernel wrote)
    if (p.mode == kLinRope) {
      for (int r = t; r < NP; r += 128) {
        const int gr = row0 + r;
        int ps = 0;
        if (gr < p.n_rows) {
          ps = p.pos ? p.pos[(long long)gr * p.pos_stride] : (gr % p.pos_period);
          if (ps < 0 || ps >= p.max_pos) {
            set_error(p.err, kErrBadPos);
            ps = 0;
          }
        }
        s_pos[r] = ps;
      }
    }
    if (p.row_norm) {
      // sum of x^2 over this CTA's k range, from the X tiles the MMAs read: each
      // stage is released to the producer only after these warps have read it
      // (bar_empty counts their arrivals).  Warp ew takes rows ew + 8i (lanes
      // 0..15) and ew + 4 + 8i (lanes 16..31); a lane reads one 16-byte chunk of
      // the row's 128-byte line in each of the two 64-k boxes.  A swizzled line
      // holds exactly its own row's chunks, so the order of the sum depends on
      // the row index only.
      constexpr int RPW = NP / 8;  // rows per half-warp
      float ssl[RPW];
#pragma unroll
      for (int i = 0; i < RPW; ++i) ssl[i] = 0.f;
      const int hl = lane & 15, sub = lane >> 4;
      for (int it = 0; it < n_st; ++it) {
        const int stage = it % STAGES;
        tc_wait(&bar_full[stage], (uint32_t)(it / STAGES) & 1u, &s_abort, p.err);
        const unsigned char* xb = bs + stage * C::B_BYTES + (hl >> 3) * C::B_BOX + (hl & 7) * 16;
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
          const int r = ew + 4 * sub + 8 * i;
          float f[8];
          Elem<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(xb + r * 128), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ssl[i] = fmaf(f[e], f[e], ssl[i]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_empty[stage]);
      }
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        float v = ssl[i];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (hl == 0) s_ss[ew + 4 * sub + 8 * i] = v;
      }
    }
    epi_bar();  // s_pos
    if (n_own > 0) load_side(0);

    tc_wait(&bar_done, 0, &s_abort, p.err);
    tc_fence_after();
    // this CTA's partial sums, in registers (thread t: feature t, every row)
    const uint32_t tq = tmem + ((uint32_t)(qd * 32) << 16);
#pragma unroll
    for (int c0 = 0; c0 < NP; c0 += 16) {
      float a[16], b[16];
      tmem_ld<16>(tq + (uint32_t)c0, a);
      tmem_ld<16>(tq + (uint32_t)(NP + c0), b);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) pacc[c0 + j] = a[j] + b[j];
    }
  }

  if (warp >= 2) {
    // push: row r's partial sums go to their owner, CTA r % split, slot (rank, r / split)
    const uint32_t recv_s = smem_u32(recv), rss_s = smem_u32(recv_ss);
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      if (r < rows_here) {
        const int o = r % split, rl = r / split;
        st_dsmem(peer_addr(recv_s + (uint32_t)(((rank * RL + rl) * kLinTile + t) * 4), (uint32_t)o), pacc[r]);
      }
    }
    if (p.row_norm) {
      for (int r = t; r < rows_here; r += 128)
        st_dsmem(peer_addr(rss_s + (uint32_t)((rank * RL + r / split) * 4), (uint32_t)(r % split)), s_ss[r]);
    }
  }

  // every partial of the cluster has landed in its owner's shared memory
  cluster_sync_all();

  if (warp >= 2) {
    // ------------------------------------------------------------ merge + output
#pragma unroll 1
    for (int lb = 0; lb < n_own; lb += C::XR) {
      if (lb > 0) load_side(lb);
      float y[C::XR];
#pragma unroll
      for (int i = 0; i < C::XR; ++i) {
        const int rl = min(lb + i, RL - 1);
        float acc = 0.f, ssum = 0.f;
        for (int c = 0; c < split; ++c) {  // rank order
          acc += recv[(c * RL + rl) * kLinTile + t];
          if (p.row_norm) ssum += recv_ss[c * RL + rl];
        }
        y[i] = p.row_norm ? acc * rsqrtf(ssum / (float)p.K + p.eps) : acc;
      }
      const int rb = rank + lb * split;  // block row of local row lb; local row lb + i is rb + i * split
      if (p.mode == kLinPlain || p.mode == kLinResidual) {
        if (f < p.F) {
#pragma unroll
          for (int i = 0; i < C::XR; ++i) {
            const int r = rb + i * split;
            if (r < rows_here) {
              p.out[(long long)(row0 + r) * p.ldo + f] = __float2bfloat16_rn(base[i] + y[i]);
            }
          }
        }
      } else if (p.mode == kLinSwiglu) {
        // features t >= 64 of the tile are the up projections of features t - 64
        if (t >= 64) {
#pragma unroll
          for (int i = 0; i < C::XR; ++i) xbuf[i * kLinTile + t] = bf16_round(y[i]);
        }
        epi_bar();
        const int fo = tile * 64 + t;
        if (t < 64 && fo < p.F / 2) {
#pragma unroll
          for (int i = 0; i < C::XR; ++i) {
            const int r = rb + i * split;
            if (r < rows_here) {
              const float g = bf16_round(y[i]), u = xbuf[i * kLinTile + t + 64];
              p.out[(long long)(row0 + r) * p.ldo + fo] = __float2bfloat16_rn(g / (1.f + expf(-g)) * u);
            }
          }
        }
        epi_bar();  // xbuf is rewritten by the next batch
      } else {
        // RoPE + split: the rotation partner of feature t lies in this tile
#pragma unroll
        for (int i = 0; i < C::XR; ++i) xbuf[i * kLinTile + t] = bf16_round(y[i]);
        epi_bar();
        const int tp = p.style ? (t ^ 1) : (first ? t + half : t - half);  // partner feature
        if (f < p.F) {
#pragma unroll
          for (int i = 0; i < C::XR; ++i) {
            const int r = rb + i * split;
            if (r >= rows_here) continue;
            const int gr = row0 + r;
            const float yv = xbuf[i * kLinTile + t];
            float o = yv;
            if (rotate) {
              const float yp = xbuf[i * kLinTile + tp];
              // pair (a, b) = (first, second): a' = a c - b s, b' = b c + a s
              o = first ? yv * cs[i] - yp * sn[i] : yv * cs[i] + yp * sn[i];
            }
            __nv_bfloat16* dst;
            if (hh < p.H)
              dst = p.q + ((long long)gr * p.H + hh) * p.Dh + ii;
            else if (hh < p.H + p.Hkv)
              dst = p.k + ((long long)gr * p.Hkv + (hh - p.H)) * p.Dh + ii;
            else
              dst = p.v + ((long long)gr * p.Hkv + (hh - p.H - p.Hkv)) * p.Dh + ii;
            *dst = __float2bfloat16_rn(o);
          }
        }
        epi_bar();
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
