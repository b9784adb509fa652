// K0 — segment planner.
//
// Turns one of the three caller-facing work descriptions into the normalised
// segment table (wfd::Seg) plus an exclusive prefix over per-segment work, which
// the attention kernels use to split the flattened (segment, query-group,
// kv-head, key) space evenly over a persistent grid.  One CTA; runs before every
// attention launch so that lengths can live in device memory (CUDA-graph replay
// with changing positions, as the reference's graph engine requires,
// graph_blocks.py:5-11).
#pragma once

#include "wfd_common.cuh"

namespace wfd {

enum PlanMode : int { kPlanSlots = 0, kPlanCu = 1, kPlanSegs = 2 };

struct PlanParams {
  int mode;
  int n;  // items / segments
  // kPlanSlots
  const wfd_item* items;
  int n_slots, n_seqs, max_seq, n_rows;
  // kPlanCu
  const int32_t* cu_q;
  const int32_t* cu_k;
  int total_q, total_k;
  // kPlanSegs
  const int32_t* s_q_row0;
  const int32_t* s_q_len;
  const int32_t* s_k_row0;
  const int32_t* s_k_len;
  // common
  int G, NQ;         // GQA group size, query vectors per decode unit
  int qg_split;      // 1: split rows into ceil(q_len*G/NQ) query groups; 0: one group
  // outputs
  Seg* segs;
  long long* prefix;  // n + 1 entries, per-kv-head work units
  // optional: the start record (first segment and its bounds) of each CTA of a
  // persistent grid of seg_grid CTAs that splits seg_units * prefix[n] into
  // equal shares (tcgen05 kernel)
  CtaStart* start;
  int seg_grid, seg_units;
  // zero-fill of query rows that see no keys (k_len == 0)
  void* out;
  int Hq, Dh, elem_bytes;
  int* err;
  // optional window append (slot mode, blocks 1..gridDim.x-1): rows
  // k_new[q_row0 + j] of every valid item go to key row
  // (slot * n_seqs + seq) * max_seq + k_row_offset + pos0 + j of k_app / v_app,
  // and the slot length lens[slot * n_seqs + seq + lens_offset] rises to pos0 + q_len
  const char* k_new;
  const char* v_new;
  char* k_app;
  char* v_app;
  long long row_bytes, k_row_offset;
  int32_t* lens;
  int lens_offset;
  // optional per-row positions of slot-table windows (gapped windows): row j of
  // an item sits at row_pos[(q_row0 + j) * row_pos_stride]
  const int32_t* row_pos;
  int row_pos_stride;
};

constexpr int kPlanThreads = 1024;
// Up to this many segments the prefix sums are also kept in shared memory, so
// the per-CTA start-record searches run on shared memory instead of making a
// chain of dependent global loads each.
constexpr int kPlanStaged = 4095;

__device__ __forceinline__ long long block_excl_scan(long long x, long long* warp_tot, long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    long long w = (lane < (blockDim.x >> 5)) ? warp_tot[lane] : 0;
    long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    warp_tot[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  long long r = warp_tot[warp] + incl - x;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const PlanParams p) {
  griddep_wait();  // launched with programmatic stream serialization (items come from the predecessor)
  griddep_launch_dependents();  // the attention kernel may run its prologue meanwhile
  if (blockIdx.x > 0) {
    // ---- window append: the tensor-core kernel reads every key through TMA, so
    // the window rows go to the cache before it starts (it waits for this grid).
    // Items are checked as below; invalid ones are skipped (block 0 reports them).
    const long long nvec = p.row_bytes / 16;
    for (int i = blockIdx.x - 1; i < p.n; i += gridDim.x - 1) {
      const wfd_item it = p.items[i];
      int last = 0;
      if (it.q_len <= 0 ||
          check_slot_item(it, p.n_slots, p.n_seqs, p.max_seq, p.n_rows, p.row_pos, p.row_pos_stride, last) != 0)
        continue;
      const long long row0 = ((long long)it.slot * p.n_seqs + it.seq) * p.max_seq + p.k_row_offset;
      for (long long e = threadIdx.x; e < (long long)it.q_len * nvec; e += blockDim.x) {
        const long long j = e / nvec, c = e % nvec;
        const int pos = p.row_pos != nullptr ? p.row_pos[(it.q_row0 + j) * p.row_pos_stride] : it.pos0 + (int)j;
        if (pos < it.pos0 || pos > last) {  // a gapped window's middle row out of order: skipped, reported
          if (c == 0) set_error(p.err, kErrBadPos);
          continue;
        }
        const long long src = (it.q_row0 + j) * p.row_bytes + c * 16;
        const long long dst = (row0 + pos) * p.row_bytes + c * 16;
        *reinterpret_cast<uint4*>(p.k_app + dst) = ld_nc_v4(p.k_new + src);
        *reinterpret_cast<uint4*>(p.v_app + dst) = ld_nc_v4(p.v_new + src);
      }
      if (threadIdx.x == 0 && p.lens != nullptr)
        atomicMax(p.lens + it.slot * p.n_seqs + it.seq + p.lens_offset, last + 1);
    }
    return;
  }
  __shared__ long long warp_tot[32];
  __shared__ long long s_total;
  __shared__ long long s_prefix[kPlanStaged + 1];
  const bool staged = p.n <= kPlanStaged;
  long long carry = 0;
  for (int base = 0; base < p.n; base += kPlanThreads) {
    const int i = base + threadIdx.x;
    long long work = 0;
    if (i < p.n) {
      Seg s;
      s.k_row0 = 0;
      s.k_len = 0;
      s.q_row0 = 0;
      s.q_len = 0;
      s.new_row0 = -1;
      s.lens_idx = -1;
      bool ok = true;
      if (p.mode == kPlanSlots) {
        const wfd_item it = p.items[i];
        int last = 0;
        const int bad = check_slot_item(it, p.n_slots, p.n_seqs, p.max_seq, p.n_rows, p.row_pos, p.row_pos_stride, last);
        if (bad) {
          set_error(p.err, bad);
          ok = false;
        }
        if (ok) {
          s.k_row0 = ((long long)it.slot * p.n_seqs + it.seq) * (long long)p.max_seq;
          s.k_len = last + 1;
          s.q_row0 = it.q_row0;
          s.q_len = it.q_len;
          s.new_row0 = it.q_row0;
          s.lens_idx = it.slot * p.n_seqs + it.seq;
        }
      } else if (p.mode == kPlanCu) {
        const int q0 = p.cu_q[i], q1 = p.cu_q[i + 1];
        const int k0 = p.cu_k[i], k1 = p.cu_k[i + 1];
        if (q0 < 0 || q1 < q0 || q1 > p.total_q || k0 < 0 || k1 < k0 || k1 > p.total_k) {
          set_error(p.err, kErrBadSegs);
          ok = false;
        } else {
          s.k_row0 = k0;
          s.k_len = k1 - k0;
          s.q_row0 = q0;
          s.q_len = q1 - q0;
        }
      } else {
        const int q0 = p.s_q_row0[i], ql = p.s_q_len[i];
        const int k0 = p.s_k_row0[i], kl = p.s_k_len[i];
        if (q0 < 0 || ql < 0 || (long long)q0 + ql > p.total_q || k0 < 0 || kl < 0 ||
            (long long)k0 + kl > p.total_k) {
          set_error(p.err, kErrBadSegs);
          ok = false;
        } else {
          s.k_row0 = k0;
          s.k_len = kl;
          s.q_row0 = q0;
          s.q_len = ql;
        }
      }
      if (!ok) {
        s.k_len = 0;
        s.q_len = 0;
      }
      const long long qv = (long long)s.q_len * p.G;
      s.n_qg = (qv == 0) ? 0 : (p.qg_split ? (int)((qv + p.NQ - 1) / p.NQ) : 1);
      work = (long long)s.n_qg * s.k_len;
      p.segs[i] = s;
      // Query rows with no key to attend produce zeros (written here; no
      // attention CTA visits a zero-work segment).
      if (ok && s.q_len > 0 && s.k_len == 0 && p.out != nullptr) {
        const long long row_bytes = (long long)p.Hq * p.Dh * p.elem_bytes;
        uint4* o = reinterpret_cast<uint4*>(static_cast<char*>(p.out) + (long long)s.q_row0 * row_bytes);
        const long long nvec = (long long)s.q_len * row_bytes / 16;
        for (long long v = 0; v < nvec; ++v) o[v] = make_uint4(0, 0, 0, 0);
      }
    }
    const long long excl = block_excl_scan(work, warp_tot, &s_total);
    if (i < p.n) {
      p.prefix[i] = carry + excl;
      if (staged) s_prefix[i] = carry + excl;
    }
    carry += s_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    p.prefix[p.n] = carry;
    if (staged) s_prefix[p.n] = carry;
  }
  if (p.start != nullptr) {
    __syncthreads();  // the prefix above is complete and visible to the block
    const long long total = (long long)p.seg_units * carry;
    const long long share = total > 0 ? (total + p.seg_grid - 1) / p.seg_grid : 1;
    const long long* pf = staged ? s_prefix : p.prefix;
    for (int c = threadIdx.x; c < p.seg_grid; c += blockDim.x) {
      const long long a = (long long)c * share;
      int lo = 0, hi = p.n - 1;  // largest i with seg_units * prefix[i] <= a
      if (total <= 0 || a >= total) {
        lo = 0;
      } else {
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if ((long long)p.seg_units * pf[mid] <= a) lo = mid;
          else hi = mid - 1;
        }
      }
      CtaStart cs;
      cs.S = p.segs[lo];
      cs.base = (long long)p.seg_units * pf[lo];
      cs.nbase = lo + 1 <= p.n - 1 ? (long long)p.seg_units * pf[lo + 1] : 0x7fffffffffffffffll;
      cs.seg = lo;
      cs.pad[0] = cs.pad[1] = cs.pad[2] = 0;
      p.start[c] = cs;
    }
  }
}

}  // namespace wfd
