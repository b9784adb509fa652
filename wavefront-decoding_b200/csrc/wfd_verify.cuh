// K2 — wavefront verify / decode attention on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA, sm_100a), bf16 inputs, Dh = 128 or 64.
//
// Swap-AB formulation: per 128-key tile of one (segment, query group, kv head)
// unit
//     S^T[128 keys x N]  = K_tile[128 x Dh] . Q^T            (A = K, K-major)
//     O^T[128 dims x N] += V_tile^T[128 x 128 keys] . P^T     (A = V, MN-major)
// For Dh = 64 the P.V MMA keeps M = 128: its upper 64 rows read the shared memory
// after the tile (the next stage, or a guard region after the last one) and land
// in TMEM lanes that are never read back; a stage is then half as large, so the
// ring holds twice as many.
// where N = NQP (16 or 32) >= the unit's query vectors (window rows x GQA
// group): the tensor core's M = 128 dimension runs over keys (then over head
// dims), so a handful of query rows still fill the instruction.  Accumulators
// live in TMEM; each of the four softmax warps owns one 32-lane TMEM quadrant
// (= 32 keys of S^T, then 32 head dims of O^T).
//
// Warp roles (one CTA per SM; 192 threads, 320 for 32 query columns):
//   warp 0      TMA producer: K and V tiles (2 boxes of 64 dims each, 128B
//               swizzle) into a STAGES-deep ring, mbarrier complete_tx; and
//               each unit's Q^T operand into one of two buffers ahead of the
//               MMA warp (a unit boundary then waits on no global load)
//   warp 1      TMEM allocator + tcgen05.mma issuer (one lane issues)
//   warps 2..   softmax / correction, 4 warps per slice of 16 query columns
//               (warp w reads TMEM lane quadrant w % 4): S^T from TMEM, column
//               maxima across the 128 keys, exp2, P^T (bf16) to shared memory,
//               O^T accumulated in registers with the online-softmax rescale
// The persistent grid splits the flattened (segment, query group, kv head,
// key) space into equal key shares exactly like the CUDA-core kernel; units
// that straddle CTAs are merged by the last CTA to arrive.  A CTA starts from
// its 64-byte start record (first segment, its bounds, its Seg), written by the
// plan kernel, and every role keeps the current segment in registers.  Every
// wait is bounded and reports through the error word; no multicast, no cluster
// launch.
//
// Head pairs (head_dim 64): with `pair` set, a unit is two consecutive kv heads
// of a head_dim-64 cache read as one 128-dim head (the two 64-dim boxes are the
// two heads).  Q^T is block-diagonal: query column n of head e (e = 0, 1) holds
// its 64 dims in half e and zeros in the other, so S^T = K.Q^T gives each column
// its own head's scores, and O^T rows [64e, 64e + 64) of column n are its output
// (the other half is discarded).  The MMA count per byte is then that of
// head_dim 128: the tensor-core issue rate, not the HBM, bounds a 64-dim tile.
//
// Window keys are read from the KV cache: the window rows are appended by the
// plan kernel's extra blocks in the launch before this one.  Launched with
// programmatic stream serialization: barrier set-up and the TMEM allocation
// overlap the previous kernel; griddep_wait() precedes every read of its outputs.
#pragma once

#include <cuda.h>

#include "wfd_common.cuh"

namespace wfd {

constexpr int kVerifyMaxRows = 32;  // query vectors per unit (larger windows -> query groups)
constexpr int kSelfPlanMax = 256;  // item tables up to this size are planned by the attention CTAs themselves
#ifndef WFD_MMA_CHAINS
#define WFD_MMA_CHAINS 2
#endif
constexpr int kTcTile = 128;        // keys per tile == MMA M
// threads: TMA warp + MMA warp + 4 softmax warps per 16 query columns
__host__ __device__ constexpr int tc_threads(int nqp) { return nqp == 32 ? 320 : 192; }

// Tensor maps of the tail pieces of a K / V tile: boxes of 64, 32, 16 and 8 rows.
struct TailMaps {
  CUtensorMap k[4];
  CUtensorMap v[4];
};

struct VerifyParams {
  const void* q;
  void* out;
  const Seg* segs;
  const long long* prefix;
  const CtaStart* start;  // start record of each CTA, from the plan kernel (null: search here)
  int n_segs;
  int Hq, Hkv, G;
  float scale_log2;
  int causal;
  long long k_row_offset;
  int pair;  // 1: units are pairs of head_dim-64 kv heads (Hkv counts pairs, DH == 128)
  // 1: batch-invariant split: every unit is processed whole by the CTA whose share
  // contains its first key (no split, no merge), so a row's result depends on its
  // own unit only, not on the other work items of the launch
  int invariant;
  float* ws_part;
  int* ws_cnt;
  int* err;
  // Self-planned start (slot-table calls with at most kSelfPlanMax items, else
  // null): every CTA computes its share's first segment from the item table
  // itself, before the plan kernel has finished, and streams the key tiles the
  // window append cannot touch before it waits for that kernel.
  const wfd_item* items;
  int n_slots, n_seqs, max_seq, n_rows;  // the plan kernel's item checks
  int Gv, NQ;                            // query vectors per kv (pair) head, per unit
  // optional per-row positions of slot-table windows (gapped windows): row j of
  // a segment sits at row_pos[(q_row0 + j) * row_pos_stride] and sees keys up to
  // that position; null: rows sit at k_len - q_len + j (bottom-right causal)
  const int32_t* row_pos;
  int row_pos_stride;
  // 1 (a test hook): the CTA gives up as a wait that ran out of its bound does
  // (timeout bit, abort flag) right after its first K/V copies are issued.
  // Checked once per CTA, not in the waits: the wait loops stay as lean as
  // possible (a runtime trip count in them cost 8 us a config-2 step).
  int fail_waits;
};

template <int NQP, int DH>
struct TcCfg {
  static constexpr int KB = DH / 64;                       // 64-dim boxes per K (and per V) tile
  static constexpr int STAGES = DH == 128 ? 3 : (NQP == 32 ? 5 : 6);
  static constexpr int BOX_BYTES = kTcTile * 128;          // 128 rows x 64 bf16
  static constexpr int KV_STAGE = 2 * KB * BOX_BYTES;      // K boxes, then V boxes
  static constexpr int GUARD = DH == 128 ? 0 : BOX_BYTES;  // read by the M = 128 P.V MMA of the last stage
  static constexpr int Q_BYTES = NQP * DH * 2;             // KB boxes of NQP rows x 128 B (one of two buffers)
  static constexpr int P_ROWB = NQP * 2;                   // one key row of P^T
  static constexpr int P_BYTES = kTcTile * P_ROWB;
  static constexpr int P_SWZ_BITS = NQP == 16 ? 1 : 2;     // Swizzle<1,4,3> (32B) / <2,4,3> (64B)
  static constexpr uint64_t P_LAYOUT = NQP == 16 ? 6 : 4;  // UMMA layout SWIZZLE_32B / SWIZZLE_64B
  static constexpr int P_ATOM = 8 * P_ROWB;                // 8 key rows
  static constexpr int RED_FLOATS = 2 * 4 * NQP;           // double-buffered per-warp column values
  static constexpr int SMEM =
      STAGES * KV_STAGE + GUARD + 2 * Q_BYTES + P_BYTES + 2 * RED_FLOATS * 4 + (3 * NQP + 4) * 4 + 1024;
  // Each accumulation (S^T of a tile: CHS, O^T of a tile: CHO) is split over
  // independent TMEM accumulators (k-steps j with j % CH == c go to chain c,
  // summed by the softmax warps): consecutive MMAs into one accumulator wait
  // for each other, so CH chains keep CH MMAs in flight.
  // With 32 columns the softmax warps bound the tile period: a second S chain
  // doubles their TMEM reads (config 3: 1829 vs 1912 us a step with one chain)
  // and a second O chain measured 1.6 % slower; with 16 columns the chains let
  // the MMA warp keep two MMAs in flight.
  static constexpr int CHS = NQP == 32 ? 1 : WFD_MMA_CHAINS;
  static constexpr int CHO = NQP == 32 ? 1 : WFD_MMA_CHAINS;
  static constexpr int S_COL = 0;                          // S^T buffer sb, chain c: (sb * CHS + c) * NQP
  static constexpr int O_COL = 2 * CHS * NQP;              // O^T chain c: O_COL + c * NQP
  static constexpr int TMEM_USED = (2 * CHS + CHO) * NQP;
  static constexpr int TMEM_COLS = TMEM_USED <= 32 ? 32 : TMEM_USED <= 64 ? 64 : TMEM_USED <= 128 ? 128 : 256;
  static constexpr int PART_FLOATS = NQP * (DH + 2);
  static_assert(NQP == 16 || NQP == 32, "N of the swap-AB MMA");
  static_assert(DH == 64 || DH == 128, "head dim");
  static_assert(SMEM + 3072 <= 232448, "shared memory per CTA (dynamic + the kernel's static arrays)");
};

// Any window size runs on the tensor cores: more than kVerifyMaxRows query
// vectors per kv head are split into query groups (K/V re-read per group).
inline bool verify_supported(int dtype, int dh, int G, int max_q) {
  (void)G;
  (void)max_q;
  return dtype == WFD_DTYPE_BF16 && (dh == 128 || dh == 64);
}
inline int verify_rows(int G, int max_q) { return (long long)G * max_q <= 16 ? 16 : 32; }

// ---------------------------------------------------------------------------
// tcgen05 / TMA primitives (inline PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor (sm_100 UMMA): start, leading / stride byte
// offsets (16-byte units), descriptor version 1, swizzle layout code.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint64_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= layout << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc(int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory"); }

// 32 TMEM lanes x 32-bit, N consecutive columns -> N registers per thread
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]);

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded mbarrier wait by every lane of a warp, with a warp-uniform result.
// It gives up at the spin limit (setting the error word and the CTA abort
// flag) or as soon as another role has aborted.  After an abort the roles keep
// their control flow (same loop trips, same named barriers) but issue no more
// TMA or MMA work, so nothing in the CTA can block without a bound.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  // The first probe (non-blocking, so an aborted role never suspends on it) and
  // the abort flag's load are independent: a wait whose phase has completed
  // costs one shared-memory round trip, not two.  These waits sit on the tile
  // loops' critical paths (config 3: 1622 -> 1577 us a step).
  bool ok = mbar_test_wait(bar, parity);
  const bool aborted = *abort_flag;
  if (aborted) {
    ok = false;
  } else if (!ok) {
    for (uint32_t i = 1; i < kSpinLimit; ++i) {
      if (mbar_try_wait(bar, parity)) {
        ok = true;
        break;
      }
      if ((i & 255u) == 255u && *abort_flag) break;
    }
    if (!ok && !*abort_flag) {
      set_error(err, kErrTimeout);
      *abort_flag = 1;
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// Column sums of the N values each of the 32 lanes holds: butterfly
// reduce-scatter; lane l ends with column bitrev(l mod N) summed over all 32
// lanes, in an order fixed by the lane pattern.  Destroys w.  (Column maxima
// take one redux.sync per column instead: warp_max_f32.)
template <int N>
__device__ __forceinline__ float warp_col_sum(float (&w)[N], int lane) {
#pragma unroll
  for (int l = 0; (N >> l) > 1; ++l) {
    const int H = (N >> l) >> 1;
    const bool up = (lane >> l) & 1;
#pragma unroll
    for (int i = 0; i < (N >> 1); ++i) {
      if (i < H) {
        const float send = up ? w[i] : w[i + H];
        const float keep = up ? w[i + H] : w[i];
        const float got = __shfl_xor_sync(0xffffffffu, send, 1 << l);
        w[i] = keep + got;
      }
    }
  }
  float r = w[0];
  constexpr int LOGN = N == 1 ? 0 : N == 2 ? 1 : N == 4 ? 2 : N == 8 ? 3 : N == 16 ? 4 : 5;
#pragma unroll
  for (int l = LOGN; l < 5; ++l) {
    const float got = __shfl_xor_sync(0xffffffffu, r, 1 << l);
    r = r + got;
  }
  return r;
}

// Maximum of v over the 32 lanes of the warp, in every lane (the f32 form of
// redux.sync is sm_100a).  NaN inputs are ignored, as by fmaxf.
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

template <int N>
__device__ __forceinline__ int reduced_col(int lane) {
  constexpr int LOGN = N == 1 ? 0 : N == 2 ? 1 : N == 4 ? 2 : N == 8 ? 3 : N == 16 ? 4 : 5;
  if constexpr (LOGN == 0) {
    return 0;
  } else {
    return (int)(__brev((unsigned)(lane & (N - 1))) >> (32 - LOGN));
  }
}

// Segment i of a slot-mode item table exactly as the plan kernel builds it
// (invalid items get no work); returns its work in unit-keys per kv head.
__device__ __forceinline__ long long slot_segment(const VerifyParams& p, const wfd_item& it, Seg& s) {
  s.k_row0 = 0;
  s.k_len = 0;
  s.q_row0 = 0;
  s.q_len = 0;
  s.new_row0 = -1;
  s.lens_idx = -1;
  s.n_qg = 0;
  int last = 0;
  if (check_slot_item(it, p.n_slots, p.n_seqs, p.max_seq, p.n_rows, p.row_pos, p.row_pos_stride, last) != 0) return 0;
  s.k_row0 = ((long long)it.slot * p.n_seqs + it.seq) * (long long)p.max_seq;
  s.k_len = last + 1;
  s.q_row0 = it.q_row0;
  s.q_len = it.q_len;
  s.new_row0 = it.q_row0;
  s.lens_idx = it.slot * p.n_seqs + it.seq;
  const long long qv = (long long)it.q_len * p.Gv;
  s.n_qg = qv == 0 ? 0 : (int)((qv + p.NQ - 1) / p.NQ);
  return (long long)s.n_qg * s.k_len;
}

// The (segment, unit, key range) pieces of one CTA's share, in order; every
// role walks the same sequence.  The current segment (its Seg, its first and
// the next segment's first work index) stays in registers, so moving to the
// next unit of the same segment reads no global memory.
struct UnitIter {
  long long pos, b;
  int seg;
  bool have = false;
  Seg S{};
  long long base = 0, nbase = 0;
  bool waited = true;  // false: griddep_wait() not yet executed by this thread (self-planned start)
  __device__ __forceinline__ long long seg_base(const VerifyParams& p, int i) const {
    return i <= p.n_segs - 1 ? (long long)p.Hkv * p.prefix[i] : 0x7fffffffffffffffll;
  }
  __device__ __forceinline__ bool next(const VerifyParams& p, Seg& Sout, int& u, int& r_lo, int& r_hi,
                                       long long& unit_start) {
    for (;;) {
      if (pos >= b) return false;
      if (!have || pos >= nbase) {
        if (!waited) {  // the segment table and prefix are the plan kernel's outputs
          griddep_wait();
          waited = true;
        }
        if (!have) {
          base = seg_base(p, seg);
          nbase = seg_base(p, seg + 1);
        }
        while (pos >= nbase) {  // largest seg with Hkv * prefix[seg] <= pos
          ++seg;
          base = nbase;
          nbase = seg_base(p, seg + 1);
        }
        S = p.segs[seg];
        have = true;
      }
      Sout = S;
      const long long o = pos - base;
      u = (int)(o / S.k_len);
      unit_start = base + (long long)u * S.k_len;
      const long long unit_end = unit_start + S.k_len;
      if (p.invariant) {
        if (unit_start < pos) {  // began in the previous CTA's share: that CTA processes it
          pos = unit_end;
          continue;
        }
        r_lo = 0;
        r_hi = S.k_len;  // whole unit, possibly past b
        pos = unit_end;
        return true;
      }
      r_lo = (int)(o - (long long)u * S.k_len);
      r_hi = (int)(((unit_end < b) ? unit_end : b) - unit_start);
      pos = unit_start + r_hi;
      return true;
    }
  }
};

// NA = query columns the softmax works on (the MMA always computes NQP): 1 for
// MHA decode rows, 4 for GQA-4 decode rows, else NQP.  Every unit has at most NA
// query vectors; P^T columns >= NA are zeroed once and never written again.
template <int NQP, int DH, int NA>
__global__ void __launch_bounds__(tc_threads(NQP), 1)
    wave_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                   const __grid_constant__ TailMaps tails, const VerifyParams p) {
  using C = TcCfg<NQP, DH>;
  constexpr int STAGES = C::STAGES;
  constexpr int KB = C::KB;
  static_assert(NA == 1 || NA == 4 || NA == 16 || NA == 32, "active query columns");
  static_assert(NA <= NQP, "active query columns");
  constexpr int THREADS = tc_threads(NQP);
  constexpr int H2 = NQP == 32 ? 2 : 1;  // column slices of the softmax (4 warps each)
  constexpr int NL = NA / H2;            // active query columns per softmax thread
  constexpr int LW = NQP / H2;           // TMEM columns one tcgen05.ld reads per slice
  constexpr int SMT = 128 * H2;          // softmax threads
  static_assert(THREADS == 64 + SMT, "warp roles");
  const float NEG_INF = -__int_as_float(0x7f800000);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* kvs = smem;                               // STAGES x (K0 K1 V0 V1)
  unsigned char* qs = kvs + STAGES * C::KV_STAGE + C::GUARD;  // 2 x Q^T operand (K-major, SW128)
  unsigned char* ps = qs + 2 * C::Q_BYTES;                 // P^T operand (MN-major)
  float* red = reinterpret_cast<float*>(ps + C::P_BYTES);  // [2][4][NQP] column maxima
  float* lred = red + C::RED_FLOATS;                       // [2][4][NQP] column sums
  float* mst = lred + C::RED_FLOATS;                       // [NQP] running column max (log2-scaled)
  float* ast = mst + NQP;                                  // [NQP] this tile's rescale factors
  float* msf = ast + NQP;                                  // [NQP] mst with -inf as 0 (exp2 of masked scores)
  int* rflag = reinterpret_cast<int*>(msf + NQP);          // [H2] any factor != 1 this tile

  __shared__ __align__(8) uint64_t bar_full[STAGES];
  __shared__ __align__(8) uint64_t bar_empty[STAGES];
  __shared__ __align__(8) uint64_t bar_sfull[2];
  __shared__ __align__(8) uint64_t bar_sfree[2];
  __shared__ __align__(8) uint64_t bar_pfull;
  __shared__ __align__(8) uint64_t bar_ofull;
  __shared__ __align__(8) uint64_t bar_ofree;
  __shared__ __align__(8) uint64_t bar_qready[2];  // unit's Q^T written (producer)
  __shared__ __align__(8) uint64_t bar_qfree[2];   // unit's S MMAs done with its Q^T (MMA commit)
  __shared__ __align__(8) uint64_t bar_drain;      // every MMA of the CTA complete (final MMA commit)
  __shared__ uint32_t s_tmem;
  __shared__ int s_rp[NQP];  // gapped windows: each query column's row position (softmax warps)
  __shared__ volatile int s_abort;
  __shared__ int s_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // Self-planned start: the item table comes from the plan kernel's
  // predecessor, which had completed before the plan kernel let this grid start,
  // so it is read before griddep_wait(); everything the plan kernel writes
  // (segment table, prefix, appended window rows) is read only after it.  The
  // loads go out first, under the barrier and TMEM set-up; thread t holds items
  // [t * IPT, t * IPT + IPT).
  const bool self = p.items != nullptr;
  constexpr int IPT = (kSelfPlanMax + THREADS - 1) / THREADS;
  wfd_item my[IPT];
  if (self) {
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const int i = tid * IPT + k;
      if (i < p.n_segs) my[k] = p.items[i];
    }
  }
  // the tensor maps' descriptors are fetched while the CTA sets up
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_k)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_v)) : "memory");

  }

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_sfull[s], 1);
      mbar_init(&bar_sfree[s], 4 * H2);
    }
    mbar_init(&bar_pfull, 1);
    mbar_init(&bar_ofull, 1);
    mbar_init(&bar_ofree, 4 * H2);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_qready[s], 1);
      mbar_init(&bar_qfree[s], 1);
    }
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
  __shared__ long long s_wtot[THREADS / 32];  // self-planned: work of each warp's items
  __shared__ Seg s_S0;                         // self-planned: the share's first segment
  __shared__ long long s_base0, s_nbase0;
  __shared__ int s_seg0, s_slot0, s_seq0, s_minpos;
  if (!self) griddep_wait();  // plan outputs, appended window rows and the workspace
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  CtaStart cs{};
  long long total;
  long long w[IPT];
  long long excl = 0;
  if (self) {
    // per-item work (the plan kernel's rule; invalid items have none), then an
    // exclusive prefix over the CTA: warp shuffles, one barrier
    long long tsum = 0;
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      Seg sg;
      w[k] = (tid * IPT + k < p.n_segs) ? slot_segment(p, my[k], sg) : 0;
      tsum += w[k];
    }
    long long incl = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wtot[warp] = incl;
    if (tid == 0) s_minpos = 0x7fffffff;
    __syncthreads();
    long long before = 0, all = 0;
#pragma unroll
    for (int k = 0; k < THREADS / 32; ++k) {
      before += (k < warp) ? s_wtot[k] : 0;
      all += s_wtot[k];
    }
    excl = before + incl - tsum;
    total = (long long)p.Hkv * all;
  } else {
    // independent loads in flight together: this CTA's start record (from the
    // plan kernel) and the total work
    if (p.start != nullptr) cs = p.start[blockIdx.x];
    total = (long long)p.Hkv * p.prefix[p.n_segs];
  }
  long long share = 1, a = 0, b = 0;
  if (total > 0) {
    share = (total + gridDim.x - 1) / gridDim.x;
    a = (long long)blockIdx.x * share;
    b = (a + share < total) ? a + share : total;
  }
  // first segment of this CTA's share: the largest i with Hkv * prefix[i] <= a
  // (prefix is non-decreasing).  A CTA-wide k-ary search: every round the 192
  // threads probe 192 pivots of [lo, hi] at once, so up to 192 segments take
  // one round of loads instead of a chain of dependent ones.
  int seg0 = 0;
  int minpos = 0;  // self-planned: keys of the first segment below this are never written by the append
  if (self) {
    // the item whose work holds a (the largest i with Hkv * prefix[i] <= a has
    // work: a < total) is found by its owner thread
    if (a < b) {
      long long pf = excl;
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        const int i = tid * IPT + k;
        if (w[k] > 0 && (long long)p.Hkv * pf <= a && a < (long long)p.Hkv * (pf + w[k])) {
          slot_segment(p, my[k], s_S0);
          s_base0 = (long long)p.Hkv * pf;
          s_nbase0 = i + 1 <= p.n_segs - 1 ? (long long)p.Hkv * (pf + w[k]) : 0x7fffffffffffffffll;
          s_seg0 = i;
          s_slot0 = my[k].slot;
          s_seq0 = my[k].seq;
        }
        pf += w[k];
      }
    }
    __syncthreads();
    if (a < b) {
      // the lowest window position any item appends to the first segment's
      // (slot, sequence): items of one call may share a slot
      const int sl0 = s_slot0, sq0 = s_seq0;
      int mp = 0x7fffffff;
#pragma unroll
      for (int k = 0; k < IPT; ++k)
        if (w[k] > 0 && my[k].slot == sl0 && my[k].seq == sq0 && my[k].pos0 < mp) mp = my[k].pos0;
      if (mp != 0x7fffffff) atomicMin(&s_minpos, mp);
    }
    __syncthreads();
    if (a < b) {
      seg0 = s_seg0;
      cs.S = s_S0;
      cs.base = s_base0;
      cs.nbase = s_nbase0;
      cs.seg = seg0;
    }
    minpos = s_minpos;
  } else if (a < b && p.start != nullptr) {
    seg0 = cs.seg;
  } else if (a < b) {
    int lo = 0, hi = p.n_segs - 1;
    while (lo < hi) {
      const int span = hi - lo;
      int piv = -1;
      if (span <= THREADS) {
        if (tid < span) piv = lo + 1 + tid;
      } else {
        piv = lo + (int)(((long long)(tid + 1) * span) / (THREADS + 1));
      }
      const int c = __syncthreads_count(piv >= 0 && (long long)p.Hkv * p.prefix[piv] <= a);
      if (span <= THREADS) {
        lo = hi = lo + c;
      } else {
        const int nlo = c == 0 ? lo : lo + (int)(((long long)c * span) / (THREADS + 1));
        const int nhi = c == THREADS ? hi : lo + (int)(((long long)(c + 1) * span) / (THREADS + 1)) - 1;
        lo = nlo;
        hi = nhi;
      }
    }
    seg0 = lo;
  }
  // every role walks the same units; with a start record the first segment is
  // already in registers
  auto make_iter = [&]() {
    UnitIter r{a, b, seg0};
    if (a < b && (p.start != nullptr || self)) {
      r.have = true;
      r.S = cs.S;
      r.base = cs.base;
      r.nbase = cs.nbase;
    }
    r.waited = !self;
    return r;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    UnitIter itr = make_iter();
    Seg S;
    int u, r_lo, r_hi;
    long long ustart;
    uint32_t it = 0, units = 0;
    uint32_t n_iss = 0;  // tiles whose TMA loads were issued (a prefix of the sequence: issue stops at an abort)
    while (itr.next(p, S, u, r_lo, r_hi, ustart)) {
      const int h = u % p.Hkv, qg = u / p.Hkv;
      const int n_t = (r_hi - r_lo + kTcTile - 1) / kTcTile;
      const long long row0 = S.k_row0 + p.k_row_offset + r_lo;

      for (int t = 0; t < n_t; ++t, ++it) {
        const int stage = (int)(it % STAGES);
        if (!itr.waited && (itr.seg != seg0 || r_lo + (t + 1) * kTcTile > minpos)) {
          // this tile may hold rows the plan kernel's append writes
          griddep_wait();
          itr.waited = true;
        }
        const bool go = (it >= (uint32_t)STAGES) ? tc_wait(&bar_empty[stage], ((it / STAGES) - 1) & 1u, &s_abort, p.err)
                                                 : !s_abort;
        if (go && lane == 0) {
          unsigned char* dst = kvs + stage * C::KV_STAGE;
          const int row = (int)(row0 + (long long)t * kTcTile);
          // A tail tile with at most 96 rows of this range loads only those rows,
          // rounded up to 8: pieces of 64 / 32 / 16 / 8 rows (1 KB-aligned in the
          // 128B-swizzled stage, so the layout is that of a full box).  The stage's
          // other rows keep older data, masked like every key past the range
          // (scores -inf, V rows zeroed by the softmax).  Longer tails take the
          // full box: the few rows saved do not pay for the extra copies.
          const int rows_left = r_hi - r_lo - t * kTcTile;
          const int nr = rows_left > 96 ? kTcTile : ((rows_left + 7) & ~7);
          mbar_arrive_expect_tx(&bar_full[stage], (uint32_t)(nr * 128 * 2 * KB));
#pragma unroll
          for (int bx = 0; bx < KB; ++bx) {
            // box bx: dims 64bx.. of head h, or (pair) head 2h + bx
            const int cx = p.pair ? 0 : 64 * bx, ch = p.pair ? 2 * h + bx : h;
            if (nr == kTcTile) {
              tma_load_3d(dst + bx * C::BOX_BYTES, &tm_k, cx, ch, row, &bar_full[stage]);
              tma_load_3d(dst + (KB + bx) * C::BOX_BYTES, &tm_v, cx, ch, row, &bar_full[stage]);
            } else {
              int off = 0;
#pragma unroll
              for (int pc = 0; pc < 4; ++pc) {
                const int pr = 64 >> pc;  // piece rows
                if (nr & pr) {
                  tma_load_3d(dst + bx * C::BOX_BYTES + off * 128, &tails.k[pc], cx, ch, row + off, &bar_full[stage]);
                  tma_load_3d(dst + (KB + bx) * C::BOX_BYTES + off * 128, &tails.v[pc], cx, ch, row + off,
                              &bar_full[stage]);
                  off += pr;
                }
              }
            }
          }
          n_iss = it + 1;
          if (p.fail_waits && n_iss == 1) {  // test hook: give up with this tile's copies in flight
            set_error(p.err, kErrTimeout);
            s_abort = 1;
          }
        }
        __syncwarp();
        if (t == 0) {
          // ---- once the unit's first K / V tile is on its way: its Q^T operand
          // into buffer units & 1, after the S MMAs of unit units - 2 are done
          // with it.  Row n = query vector qg*NQP + n (pair: n < nvh head 2h,
          // else 2h + 1); rows past the unit's vectors are zero.  This warp runs
          // ahead of the MMA warp, so the load is off its path.
          {
            const int qb = (int)(units & 1u);
            const bool qgo =
                units >= 2 ? tc_wait(&bar_qfree[qb], ((units >> 1) - 1) & 1u, &s_abort, p.err) : !s_abort;
            if (qgo) {
              const int nvh = S.q_len * p.G;
              const int nvec = (p.pair ? 2 * nvh : nvh) - qg * NQP;
              unsigned char* qd = qs + qb * C::Q_BYTES;
              for (int c = lane; c < NQP * (DH / 8); c += 32) {
                const int n = c / (DH / 8), ch = c % (DH / 8);
                uint4 val = make_uint4(0, 0, 0, 0);
                if (n < nvec) {
                  if (p.pair) {
                    const int e = n >= nvh ? 1 : 0, v = n - e * nvh;
                    const int row = v / p.G, g = v % p.G;
                    if ((ch >> 3) == e)
                      val = ld_nc_v4(static_cast<const __nv_bfloat16*>(p.q) +
                                     ((long long)(S.q_row0 + row) * p.Hq + (2 * h + e) * p.G + g) * 64 + (ch & 7) * 8);
                  } else {
                    const int v = qg * NQP + n;
                    const int row = v / p.G, g = v % p.G;
                    val = ld_nc_v4(static_cast<const __nv_bfloat16*>(p.q) +
                                   ((long long)(S.q_row0 + row) * p.Hq + h * p.G + g) * DH + ch * 8);
                  }
                }
                const int box = ch >> 3, cc = ch & 7;
                const uint32_t off = (uint32_t)(box * NQP * 128 + n * 128 + ((cc ^ (n & 7)) << 4));
                *reinterpret_cast<uint4*>(qd + off) = val;
              }
              fence_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_qready[qb]);
            ++units;
          }
        }
      }
    }
    // the MMA warp's last commits arrive on these barriers: see them land
    // before this CTA may exit
    for (uint32_t k = (units > 2 ? units - 2 : 0); k < units; ++k)
      tc_wait(&bar_qfree[k & 1u], (k >> 1) & 1u, &s_abort, p.err);
    const uint32_t n_used = it;
    for (uint32_t j = (n_used > (uint32_t)STAGES ? n_used - STAGES : 0); j < n_used; ++j)
      tc_wait(&bar_empty[j % STAGES], (j / STAGES) & 1u, &s_abort, p.err);
    // Copies in flight must land before the CTA exits, also after an abort (which
    // skips the waits above): wait, with the fixed bound and whatever the abort
    // flag says, for the last phase of every stage this lane filled.  Earlier
    // phases of a stage completed before it was refilled.
    if (lane == 0) {
      for (uint32_t j = (n_iss > (uint32_t)STAGES ? n_iss - STAGES : 0); j < n_iss; ++j)
        if (!mbar_wait_bounded(&bar_full[j % STAGES], (j / STAGES) & 1u)) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    UnitIter itr = make_iter();
    Seg S;
    int u, r_lo, r_hi;
    long long ustart;
    uint32_t it = 0, pv = 0, units = 0;
    constexpr uint32_t IDESC_S = umma_idesc(NQP, false, false);
    constexpr uint32_t IDESC_PV = umma_idesc(NQP, true, true);
    const uint32_t q_addr = smem_u32(qs);
    const uint32_t p_addr = smem_u32(ps);
    while (itr.next(p, S, u, r_lo, r_hi, ustart)) {
      const int n_t = (r_hi - r_lo + kTcTile - 1) / kTcTile;
      const int qb = (int)(units & 1u);
      const uint32_t qa = q_addr + (uint32_t)(qb * C::Q_BYTES);
      tc_wait(&bar_qready[qb], (units >> 1) & 1u, &s_abort, p.err);
      tc_fence_after();
      for (int t = 0; t <= n_t; ++t) {
        if (t < n_t) {
          const uint32_t ti = it + t;
          const int stage = (int)(ti % STAGES);
          const int sb = (int)(ti & 1u);
          bool go = tc_wait(&bar_full[stage], (ti / STAGES) & 1u, &s_abort, p.err);
          if (ti >= 2) go = tc_wait(&bar_sfree[sb], ((ti >> 1) - 1) & 1u, &s_abort, p.err) && go;
          tc_fence_after();
          if (go && lane == 0) {
            const uint32_t k_addr = smem_u32(kvs + stage * C::KV_STAGE);
#pragma unroll
            for (int j = 0; j < DH / 16; ++j) {
              // K step j: dims 16j..16j+15 = box j/4, byte 32*(j%4) inside the 128B row
              const uint32_t koff = (uint32_t)((j >> 2) * C::BOX_BYTES + (j & 3) * 32);
              const uint32_t qoff = (uint32_t)((j >> 2) * (NQP * 128) + (j & 3) * 32);
              umma_f16(tmem + (uint32_t)((sb * C::CHS + j % C::CHS) * NQP), umma_desc(k_addr + koff, 16, 1024, 2),
                       umma_desc(qa + qoff, 16, 1024, 2), IDESC_S, j >= C::CHS ? 1u : 0u);
            }
            umma_commit(&bar_sfull[sb]);
            if (t == n_t - 1) umma_commit(&bar_qfree[qb]);  // the unit's Q^T buffer may be rewritten
          }
          __syncwarp();
        }
        if (t >= 1) {
          bool go = tc_wait(&bar_pfull, pv & 1u, &s_abort, p.err);
          if (pv >= 1) go = tc_wait(&bar_ofree, (pv - 1) & 1u, &s_abort, p.err) && go;
          tc_fence_after();
          const uint32_t tp = it + t - 1;
          const int stage = (int)(tp % STAGES);
          if (go && lane == 0) {
            const uint32_t v_addr = smem_u32(kvs + stage * C::KV_STAGE + KB * C::BOX_BYTES);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // K step j: keys 16j..16j+15 = two 8-row groups of both V boxes / of P^T
              umma_f16(tmem + (uint32_t)(C::O_COL + (j % C::CHO) * NQP), umma_desc(v_addr + j * 2048, C::BOX_BYTES, 1024, 2),
                       umma_desc(p_addr + j * 2 * C::P_ATOM, 16, C::P_ATOM, C::P_LAYOUT), IDESC_PV,
                       j >= C::CHO ? 1u : 0u);
            }
            umma_commit(&bar_ofull);
            umma_commit(&bar_empty[stage]);
          }
          __syncwarp();
          ++pv;
        }
      }
      it += n_t;
      ++units;
    }
    // Every MMA this lane issued must be complete before TMEM is freed and the
    // CTA exits, also after an abort (whose consumers stop waiting for them):
    // one last commit tracks all of them.
    if (lane == 0) {
      umma_commit(&bar_drain);
      if (!mbar_wait_bounded(&bar_drain, 0)) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    // 4 * H2 warps: warp w reads TMEM lane quadrant w % 4 (32 keys of S^T, then 32
    // head dims of O^T) and query columns [col0, col0 + NL) of the tile.
    const int sw = warp - 2;            // 0 .. 4 * H2 - 1
    const int sq = sw & 3;              // quadrant warp within its column slice
    const int col0 = (sw >> 2) * NL;    // first query column of this thread
    const int qd = warp & 3;            // TMEM lane quadrant this warp may access
    const int stid = tid - 64;          // 0 .. SMT - 1 within the softmax group
    const int my_row = qd * 32 + lane;  // key row of S^T, then head dim of O^T, this thread owns
    const uint32_t tq = tmem + ((uint32_t)(qd * 32) << 16);
    UnitIter itr = make_iter();
    Seg S;
    int u, r_lo, r_hi;
    long long ustart;
    uint32_t it = 0, pv = 0, units = 0;
    constexpr int PCHL = (NL + 7) / 8;  // 16-byte chunks of a P^T row this thread writes
    for (int c = stid; c < C::P_BYTES / 16; c += SMT) reinterpret_cast<uint4*>(ps)[c] = make_uint4(0, 0, 0, 0);
    fence_async_smem();
    while (itr.next(p, S, u, r_lo, r_hi, ustart)) {
      const int h = u % p.Hkv, qg = u / p.Hkv;
      const int n_t = (r_hi - r_lo + kTcTile - 1) / kTcTile;
      const int nvh = S.q_len * p.G;                                   // query vectors per kv head
      const int nvec = (p.pair ? 2 * nvh : nvh) - qg * NQP;  // of this unit / group (may exceed NQP)

      // gapped windows: the position of each column's row, in shared memory (not
      // registers: the 32-column variant is at its register limit); the barrier at
      // the end of the previous unit keeps it from being rewritten early
      if (p.row_pos != nullptr) {
        if (sq == 0 && lane < NL) {
          const int n = col0 + lane;
          const int vn = (p.pair && n >= nvh) ? n - nvh : n;
          const int row = (p.pair ? vn : qg * NQP + n) / p.G;
          s_rp[n] = n < nvec ? p.row_pos[(long long)(S.q_row0 + row) * p.row_pos_stride] : -1;
        }
        softmax_bar<SMT>();
      }
      // the CTAs whose shares hold keys of this unit; if the others have all
      // published their partials by the time this CTA gets to the unit (the usual
      // case for a CTA's last unit: the next CTA began with the rest of it), this
      // CTA merges without publishing its own.  Read now, used after the tiles.
      const int c_first = (int)(ustart / share);
      const int c_last = (int)((ustart + S.k_len - 1) / share);
      const int n_contrib = p.invariant ? 1 : c_last - c_first + 1;
      int arrived = 0;
      if (n_contrib > 1 && stid == 0) arrived = ld_relaxed_gpu(p.ws_cnt + c_first);
      // running column maxima live in shared memory (mst, log2-scaled), owned
      // by lanes 0..NL-1 of the first warp of each column slice
      if (sq == 0 && lane < NL) mst[col0 + lane] = NEG_INF;
      float lp[NL], oacc[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        lp[j] = 0.f;
        oacc[j] = 0.f;
      }
      const float c2 = p.scale_log2;
      for (int t = 0; t < n_t; ++t) {
        const uint32_t ti = it + t;
        const int sb = (int)(ti & 1u);
        tc_wait(&bar_sfull[sb], (ti >> 1) & 1u, &s_abort, p.err);
        tc_fence_after();
        float s[LW];
        tmem_ld<LW>(tq + (uint32_t)(sb * C::CHS * NQP + col0), s);
        if constexpr (C::CHS == 2) {
          float s1[LW];
          tmem_ld<LW>(tq + (uint32_t)((sb * C::CHS + 1) * NQP + col0), s1);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < LW; ++j) s[j] += s1[j];
        }
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_sfree[sb]);

        // key `key` (unit index) is visible to query vector v = qg*NQP + n iff
        // key <= k_len - q_len + v / G, i.e. n >= (key - (k_len - q_len)) * G - qg*NQP
        const int key = r_lo + t * kTcTile + my_row;
        const bool kvalid = key < r_hi;
        const int thr = p.causal ? (key - (S.k_len - S.q_len)) * p.G - qg * NQP : -(1 << 30);
        const int nlim = kvalid ? nvec : 0;
        // a tile whose keys all lie in the unit and below the causal frontier of
        // the window's first row, for real query columns only, masks nothing
        // (warp-uniform)
        const int tile_last = r_lo + t * kTcTile + kTcTile - 1;
        const bool interior = tile_last < r_hi && col0 + NL <= nvec && p.row_pos == nullptr &&
                              (!p.causal || tile_last <= S.k_len - S.q_len);
        if (interior) {
          // every score stands
        } else if (p.row_pos != nullptr && p.causal) {
#pragma unroll
          for (int j = 0; j < NL; ++j) {
            const int n = col0 + j;
            s[j] = (n < nlim && key <= s_rp[n]) ? s[j] : NEG_INF;  // the row sees keys up to its position
          }
        } else {
#pragma unroll
          for (int j = 0; j < NL; ++j) {
            const int n = col0 + j;
            const int vn = (p.pair && n >= nvh) ? n - nvh : n;  // vector index within its head
            s[j] = (n < nlim && vn >= thr) ? s[j] : NEG_INF;    // raw (unscaled) scores
          }
        }
        // column maxima over the tile's 128 keys: this warp's 32 by redux, the
        // quadrants' by the column owner below
        float* rb = red + (ti & 1u) * (4 * NQP);
        {
          float r[NL];
#pragma unroll
          for (int j = 0; j < NL; ++j) r[j] = warp_max_f32(s[j]);
          if (lane == 0) {
            float* rw = rb + sq * NQP + col0;
            if constexpr (NL % 4 == 0) {
#pragma unroll
              for (int j = 0; j < NL; j += 4) *reinterpret_cast<float4*>(rw + j) = make_float4(r[j], r[j + 1], r[j + 2], r[j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < NL; ++j) rw[j] = r[j];
            }
          }
        }
        softmax_bar<SMT>();
        // column owner: new running max (moved only when the tile exceeds it by
        // more than 8 in log2 units; O and l share the stale max, so the result
        // is exact) and the rescale factor alpha
        if (sq == 0) {
          float alpha = 1.f;
          if (lane < NL) {
            const int cl = col0 + lane;
            const float tmax = fmaxf(fmaxf(rb[cl], rb[NQP + cl]), fmaxf(rb[2 * NQP + cl], rb[3 * NQP + cl]));
            const float mo = mst[cl];
            float mn = mo;
            if (tmax != NEG_INF) {
              const float ts = tmax * c2;
              if (mo == NEG_INF) {
                mn = ts;
              } else if (ts > mo + 8.f) {
                alpha = fast_exp2(mo - ts);
                mn = ts;
              }
            }
            if (mn != mo) mst[cl] = mn;
            // a column with no visible key yet has only -inf scores: exp2(-inf - 0) = 0
            msf[cl] = mn == NEG_INF ? 0.f : mn;
            ast[cl] = alpha;
          }
          const bool any = __any_sync(0xffffffffu, alpha != 1.f);
          if (lane == 0) rflag[sw >> 2] = any ? 1 : 0;
        }
        softmax_bar<SMT>();
        const int stage = (int)(ti % STAGES);
        if (!kvalid && col0 == 0) {
          // rows past the unit may hold anything (even NaN): zero this key's V row
          unsigned char* vrow = kvs + stage * C::KV_STAGE + KB * C::BOX_BYTES + my_row * 128;
#pragma unroll
          for (int bx = 0; bx < KB; ++bx)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(vrow + bx * C::BOX_BYTES + c * 16) = make_uint4(0, 0, 0, 0);
        }
        // the previous tile's P.V: its MMA is done once o_full fires, which also
        // frees the P^T buffer.  oacc holds O_{t-2} already rescaled to m_{t-1}.
        if (t >= 1) {
          tc_wait(&bar_ofull, pv & 1u, &s_abort, p.err);
          tc_fence_after();
          float o[LW];
          tmem_ld<LW>(tq + (uint32_t)(C::O_COL + col0), o);
          if constexpr (C::CHO == 2) {
            float o1[LW];
            tmem_ld<LW>(tq + (uint32_t)(C::O_COL + NQP + col0), o1);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < LW; ++j) o[j] += o1[j];
          }
          tc_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_ofree);
          ++pv;
#pragma unroll
          for (int j = 0; j < NL; ++j) oacc[j] += o[j];
        }
        // rescale the running sums when some column's max moved
        if (rflag[sw >> 2]) {
          if constexpr (NL >= 4) {
#pragma unroll
            for (int n4 = 0; n4 < NL / 4; ++n4) {
              const float4 a4 = reinterpret_cast<const float4*>(ast + col0)[n4];
              const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                lp[n4 * 4 + e] *= av[e];
                oacc[n4 * 4 + e] *= av[e];
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < NL; ++j) {
              lp[j] *= ast[col0 + j];
              oacc[j] *= ast[col0 + j];
            }
          }
        }
        // probabilities of this key; P^T row (bf16, swizzled MN-major), this thread's chunks
#pragma unroll
        for (int c = 0; c < PCHL; ++c) {
          float mv[8];
          if constexpr (NL >= 8) {
            const float4 m0 = reinterpret_cast<const float4*>(msf + col0)[2 * c];
            const float4 m1 = reinterpret_cast<const float4*>(msf + col0)[2 * c + 1];
            mv[0] = m0.x; mv[1] = m0.y; mv[2] = m0.z; mv[3] = m0.w;
            mv[4] = m1.x; mv[5] = m1.y; mv[6] = m1.z; mv[7] = m1.w;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) mv[e] = e < NL ? msf[col0 + e] : 0.f;
          }
          uint32_t w4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float pr2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int j = c * 8 + 2 * i + e;
              if (j < NL) {
                pr2[e] = fast_exp2(fmaf(s[j], c2, -mv[2 * i + e]));  // masked: exp2(-inf) = 0
                lp[j] += pr2[e];
              } else {
                pr2[e] = 0.f;
              }
            }
            __nv_bfloat162 h2 = __floats2bfloat162_rn(pr2[0], pr2[1]);
            w4[i] = *reinterpret_cast<uint32_t*>(&h2);
          }
          uint32_t off = (uint32_t)(my_row * C::P_ROWB + (col0 / 8 + c) * 16);
          off ^= ((off >> 7) & ((1u << C::P_SWZ_BITS) - 1u)) << 4;
          *reinterpret_cast<uint4*>(ps + off) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
        fence_async_smem();
        softmax_bar<SMT>();
        if (stid == 0) mbar_arrive(&bar_pfull);
      }
      {
        tc_wait(&bar_ofull, pv & 1u, &s_abort, p.err);
        tc_fence_after();
        float o[LW];
        tmem_ld<LW>(tq + (uint32_t)(C::O_COL + col0), o);
        if constexpr (C::CHO == 2) {
          float o1[LW];
          tmem_ld<LW>(tq + (uint32_t)(C::O_COL + NQP + col0), o1);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < LW; ++j) o[j] += o1[j];
        }
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_ofree);
        ++pv;
#pragma unroll
        for (int j = 0; j < NL; ++j) oacc[j] += o[j];
      }
      it += n_t;
      ++units;

      // ---- column sums of the unnormalised probabilities over the tile's 128 key rows
      float* lb = lred + (units & 1u) * (4 * NQP);
      {
        float w[NL];
#pragma unroll
        for (int j = 0; j < NL; ++j) w[j] = lp[j];
        const float r = warp_col_sum<NL>(w, lane);
        if (lane < NL) lb[sq * NQP + col0 + reduced_col<NL>(lane)] = r;
      }
      softmax_bar<SMT>();
      auto lsum = [&](int n) { return lb[n] + lb[NQP + n] + lb[2 * NQP + n] + lb[3 * NQP + n]; };

      const int dim = my_row;  // O^T TMEM lane == head dim (lanes >= DH hold nothing)
      const bool dim_ok = dim < DH;
      // output element of query column n held by this thread's O^T row, or -1
      auto out_at = [&](int n) -> long long {
        if (p.pair) {
          const int e = n >= nvh ? 1 : 0;
          if ((dim >> 6) != e) return -1;
          const int v = n - e * nvh;
          const int row = v / p.G, g = v % p.G;
          return ((long long)(S.q_row0 + row) * p.Hq + (2 * h + e) * p.G + g) * 64 + (dim & 63);
        }
        const int v = qg * NQP + n;
        const int row = v / p.G, g = v % p.G;
        return ((long long)(S.q_row0 + row) * p.Hq + h * p.G + g) * DH + dim;
      };
      if (n_contrib == 1) {
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const int n = col0 + j;
          if (n < nvec && dim_ok) {
            const float L = lsum(n);
            const long long oi = out_at(n);
            if (oi >= 0) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(L > 0.f ? oacc[j] / L : 0.f);
          }
        }
      } else {
        // 2: every other contributor had published when this CTA began the unit
        // (relaxed read, made an acquire by the fence), so this CTA merges now
        if (stid == 0) {
          s_flag = (arrived == n_contrib - 1) ? 2 : 0;
          if (s_flag == 2) fence_acq_rel_gpu();
        }
        softmax_bar<SMT>();
        if (s_flag != 2) {
          const int slot = (ustart < a) ? 2 * (int)blockIdx.x : 2 * (int)blockIdx.x + 1;
          float* pb = p.ws_part + (size_t)slot * C::PART_FLOATS;
          // every thread holds the same m[]; thread n publishes column n's (m, l);
          // O^T only for the unit's query columns (the merge reads no others)
          if (stid < NA) {
            pb[stid] = mst[stid];
            pb[NQP + stid] = lsum(stid);
          }
#pragma unroll
          for (int j = 0; j < NL; ++j)
            if (col0 + j < nvec && dim_ok) pb[2 * NQP + (col0 + j) * DH + dim] = oacc[j];
          __threadfence();
          softmax_bar<SMT>();
          if (stid == 0) {
            const int prev = atomicAdd(p.ws_cnt + c_first, 1);
            s_flag = (prev == n_contrib - 1) ? 1 : 0;
          }
          softmax_bar<SMT>();
        }
        if (s_flag && dim_ok) {
          __threadfence();
          // Online merge, this thread's columns in chunks of MCH, contributors in
          // key order (the result does not depend on which CTA arrives last): this
          // CTA's own (m, l, O) come from shared memory and registers; for every
          // other contributor all loads of a chunk are independent (one round trip).
          constexpr int MCH = NL < 16 ? NL : 16;
          const int k_own = (int)blockIdx.x - c_first;
#pragma unroll
          for (int j0 = 0; j0 < NL; j0 += MCH) {
            const int c0 = col0 + j0;
            if (c0 < nvec) {
              float M[MCH], Ls[MCH], acc[MCH];
#pragma unroll
              for (int j = 0; j < MCH; ++j) {
                M[j] = NEG_INF;
                Ls[j] = 0.f;
                acc[j] = 0.f;
              }
              for (int k = 0; k < n_contrib; ++k) {
                float mk[MCH], lk[MCH], ok[MCH];
                if (k == k_own) {
#pragma unroll
                  for (int j = 0; j < MCH; ++j) {
                    mk[j] = mst[c0 + j];
                    lk[j] = lsum(c0 + j);
                    ok[j] = oacc[j0 + j];
                  }
                } else {
                  const int cc = c_first + k;
                  const int sl = (k == 0) ? 2 * cc + 1 : 2 * cc;
                  const float* base = p.ws_part + (size_t)sl * C::PART_FLOATS;
#pragma unroll
                  for (int j = 0; j < MCH; ++j) {
                    mk[j] = ld_cg_f32(base + c0 + j);
                    lk[j] = ld_cg_f32(base + NQP + c0 + j);
                    ok[j] = (c0 + j < nvec) ? ld_cg_f32(base + 2 * NQP + (c0 + j) * DH + dim) : 0.f;
                  }
                }
#pragma unroll
                for (int j = 0; j < MCH; ++j) {
                  const float nm = fmaxf(M[j], mk[j]);
                  if (nm != NEG_INF) {
                    const float wa = (M[j] == NEG_INF) ? 0.f : fast_exp2(M[j] - nm);
                    const float wb = (mk[j] == NEG_INF) ? 0.f : fast_exp2(mk[j] - nm);
                    Ls[j] = Ls[j] * wa + lk[j] * wb;
                    acc[j] = acc[j] * wa + ok[j] * wb;
                    M[j] = nm;
                  }
                }
              }
#pragma unroll
              for (int j = 0; j < MCH; ++j) {
                const int n = c0 + j;
                if (n < nvec) {
                  const long long oi = out_at(n);
                  if (oi >= 0)
                    static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(Ls[j] > 0.f ? acc[j] / Ls[j] : 0.f);
                }
              }
            }
          }
        }
        if (s_flag && stid == 0) p.ws_cnt[c_first] = 0;
        softmax_bar<SMT>();  // s_flag is re-written by the next unit
      }
    }
  }

  // a self-planned CTA may not have needed the plan kernel's outputs; it still
  // completes only after that kernel, so stream order holds for what follows
  if (self) griddep_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
}

}  // namespace wfd
