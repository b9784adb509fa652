// Device-side wavefront scheduling: the per-tick route and settle of the batch
// scheduler (scheduler_batch.py:268-360 of the reference) as three small
// kernels, so a whole tick (P union -> R union -> route -> C union -> settle)
// is one CUDA graph and the host only checks a done flag every few ticks.
//
// Token slots: every sequence b owns W fixed slots; slot j of b is pool row
// b * W + j of the engine's state pool.  A slot is free (state 0), queued for
// the prelude (1) or in the recurrent wave (2).  In lossless wavefront
// decoding every live token of a sequence has a distinct step, so per tick and
// sequence at most one token reaches the commit point (verify) and at most one
// the draft point, and settle queues at most one new token: the P union has one
// row per sequence, the C union two (2b verify, 2b + 1 draft), the R union is
// the compacted list of live tokens.  Counters follow the host scheduler
// field by field.
//
// Union tables use the engine's int32 row layout: 0 pool row, 1 position,
// 2 token id, 3 cache sequence, 4 slot base (step * n_core), 5 live,
// 6.. first cache row of the row's (prelude / coda slot, sequence).
#pragma once

#include "wfd_common.cuh"

namespace wfd {

constexpr int kSchedThreads = 1024;
constexpr int kSchedMaxW = 32;
enum : int { kCtP = 0, kCtR = 1, kCtC = 2, kCtProp = 3, kCtAcc = 4, kCtRej = 5, kCtRoll = 6, kSeqCounters = 8 };
enum : int { kBtTicks = 0, kBtP = 1, kBtC = 2, kBtRTotal = 3, kBtRMax = 4, kBatchCounters = 8 };

struct SchedParams {
  // token slots (B * W)
  int32_t* alive;
  int32_t* state;
  int32_t* tok;
  int32_t* pos;
  int32_t* step;
  // sequences
  int32_t* n_commit;   // (B)
  int32_t* done;       // (B)
  int32_t* committed;  // (B, max_new)
  int32_t* seq_ct;     // (B, kSeqCounters)
  const uint8_t* emu;  // (B, emu_len) accept draws, or null = greedy gold == draft
  int32_t* emu_ctr;    // (B)
  int32_t* batch_ct;   // (kBatchCounters)
  unsigned long long* keys;  // (3) sum of k_len = position + 1 over live P / R / C rows (K/V read accounting)
  int32_t* c_slot;     // (2B) token slot of C row, -1 = none
  int32_t* lens;       // KV lengths (n_kv_slots, lens_stride)
  int32_t* err;
  // union tables
  int32_t* p_tab;      // (B, p_cols)
  int32_t* r_tab;      // (r_cap, 6)
  int32_t* c_tab;      // (2B, c_cols)
  const int32_t* c_out;  // (2B) greedy ids of the C union
  int B, W, T_total, T_draft, max_new, emu_len;
  int n_core, n_kv_slots, lens_stride, max_seq;
  int p_cols, c_cols, r_cap;
  int scratch_row, scratch_seq;
  int p_slot0, n_prelude, c_slot0, n_coda;  // first KV slot and count of the prelude / coda layers
  int depth_slots;                           // core depth slots (KV sharing: depth r -> slot r % depth_slots)
  int gap_windows;                           // 1: a sequence's tokens on one depth slot form one window, gaps included
};

__device__ __forceinline__ void sched_pad_row(int32_t* row, int cols, const SchedParams& p, int seg_slot0) {
  row[0] = p.scratch_row;
  row[1] = 0;
  row[2] = 0;
  row[3] = p.scratch_seq;
  row[4] = 0;
  row[5] = 0;
  for (int j = 6; j < cols; ++j) row[j] = ((seg_slot0 + (j - 6)) * p.lens_stride + p.scratch_seq) * p.max_seq;
}

__device__ __forceinline__ void sched_fill_row(int32_t* row, int cols, const SchedParams& p, int seg_slot0, int b,
                                               int slot, int base) {
  row[0] = slot;  // pool row == token slot
  row[1] = p.pos[slot];
  row[2] = p.tok[slot];
  row[3] = b;
  row[4] = base;
  row[5] = 1;
  for (int j = 6; j < cols; ++j) row[j] = ((seg_slot0 + (j - 6)) * p.lens_stride + b) * p.max_seq;
}

// P table (one row per sequence: its queued token, now entering the wave at
// step 0) and the compacted R table of every live token.  One block.
__global__ void __launch_bounds__(kSchedThreads) sched_pre_tick_kernel(const SchedParams p) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  __shared__ int s_cnt[kSchedThreads];
  __shared__ int s_any_p;
  __shared__ unsigned long long s_keys[2];
  const int b = threadIdx.x;
  if (b == 0) {
    s_any_p = 0;
    s_keys[0] = s_keys[1] = 0ull;
  }
  __syncthreads();
  // This sequence's token slots are read once, all loads independent: bit j of
  // `live` = slot j in the wave, of `queued` = slot j queued for the prelude.
  int cnt = 0;
  uint32_t live = 0;
  if (b < p.B) {
    int32_t* prow = p.p_tab + (long long)b * p.p_cols;
    int pj = -1;
    if (!p.done[b]) {
      uint32_t queued = 0;
#pragma unroll 4
      for (int j = 0; j < p.W; ++j) {
        const int s = b * p.W + j;
        const int a = p.alive[s], st = p.state[s];
        if (a && st == 2) live |= 1u << j;
        if (a && st == 1) queued |= 1u << j;
      }
      if (__popc(queued) > 1) set_error(p.err, kErrSched);
      if (queued) pj = b * p.W + (31 - __clz(queued));  // the last queued slot
    }
    if (pj >= 0) {
      p.state[pj] = 2;
      p.step[pj] = 0;
      sched_fill_row(prow, p.p_cols, p, p.p_slot0, b, pj, 0);
      s_any_p = 1;
      atomicAdd(&s_keys[0], (unsigned long long)(p.pos[pj] + 1));
      live |= 1u << (pj - b * p.W);
    } else {
      sched_pad_row(prow, p.p_cols, p, p.p_slot0);
    }
    cnt = __popc(live);
    if (cnt > 0) p.seq_ct[b * kSeqCounters + kCtR] += 1;
  }
  s_cnt[b] = cnt;
  __syncthreads();
  // inclusive scan of the per-sequence counts (Hillis-Steele, blockDim entries)
  for (int off = 1; off < kSchedThreads; off <<= 1) {
    const int v = b >= off ? s_cnt[b - off] : 0;
    __syncthreads();
    s_cnt[b] += v;
    __syncthreads();
  }
  const int total = s_cnt[kSchedThreads - 1];
  if (b < p.B && cnt > 0) {
    // This sequence's live tokens in (depth slot, position) order.  A run of
    // consecutive positions on one depth slot (KV sharing) becomes one window:
    // its first row carries the run length in column 5 (the item's q_len), the
    // other rows 0, so the shared slot prefix is read once per run
    // (ouro_blocks_batch.py:184-205).  With gap_windows every token of the
    // sequence on one depth slot joins one window whatever the gaps between their
    // positions (the attention reads each row's position from column 1).
    // Without sharing the live tokens of a sequence have distinct steps, so
    // every run is one token and the rows keep token-slot order.
    const bool shared = p.depth_slots > 0 && p.depth_slots < p.T_total;
    int ord[kSchedMaxW], dsl[kSchedMaxW], psn[kSchedMaxW];
    int m = 0;
    for (uint32_t bits = live; bits; bits &= bits - 1) {
      const int s = b * p.W + (__ffs(bits) - 1);
      const int d = shared ? p.step[s] % p.depth_slots : p.step[s];
      const int ps = p.pos[s];
      int k = m++;
      while (shared && k > 0 && (dsl[k - 1] > d || (dsl[k - 1] == d && psn[k - 1] > ps))) {
        ord[k] = ord[k - 1];
        dsl[k] = dsl[k - 1];
        psn[k] = psn[k - 1];
        --k;
      }
      ord[k] = s;
      dsl[k] = d;
      psn[k] = ps;
    }
    int r = s_cnt[b] - cnt;
    unsigned long long kk = 0;
    for (int i = 0; i < m;) {
      int e = i + 1;
      while (shared && e < m && dsl[e] == dsl[i] && (p.gap_windows || psn[e] == psn[e - 1] + 1)) ++e;
      for (int k = i; k < e; ++k, ++r) {
        if (r < p.r_cap) {
          int32_t* row = p.r_tab + (long long)r * 6;
          sched_fill_row(row, 6, p, 0, b, ord[k], dsl[k] * p.n_core);
          row[5] = k == i ? e - i : 0;
        }
      }
      kk += (unsigned long long)(psn[e - 1] + 1);  // the run's window reads its slot prefix once
      i = e;
    }
    atomicAdd(&s_keys[1], kk);
  }
  if (total > p.r_cap && b == 0) set_error(p.err, kErrSched);
  for (int r = total + b; r < p.r_cap; r += kSchedThreads) sched_pad_row(p.r_tab + (long long)r * 6, 6, p, 0);
  __syncthreads();
  if (b == 0) {
    p.keys[0] += s_keys[0];
    p.keys[1] += s_keys[1];
    if (s_any_p) p.batch_ct[kBtP] += 1;
    if (total > 0) {
      p.batch_ct[kBtTicks] += 1;
      p.batch_ct[kBtRTotal] += total;
      if (total > p.batch_ct[kBtRMax]) p.batch_ct[kBtRMax] = total;
    }
  }
}

// After the R union: every live token advanced one step.  Route commit points
// (step == T_total, C row 2b) and draft points (step == T_draft, C row 2b + 1).
__global__ void __launch_bounds__(kSchedThreads) sched_route_kernel(const SchedParams p) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  __shared__ int s_any_c;
  __shared__ unsigned long long s_keys;
  const int b = threadIdx.x;
  if (b == 0) {
    s_any_c = 0;
    s_keys = 0ull;
  }
  __syncthreads();
  if (b < p.B) {
    int vs = -1, ds = -1;
    if (!p.done[b]) {
      // the sequence's slots in the wave, read once (independent loads)
      uint32_t wave = 0;
#pragma unroll 4
      for (int j = 0; j < p.W; ++j) {
        const int s = b * p.W + j;
        const int a = p.alive[s], st = p.state[s];
        if (a && st == 2) wave |= 1u << j;
      }
      for (uint32_t bits = wave; bits; bits &= bits - 1) {
        const int s = b * p.W + (__ffs(bits) - 1);
        const int st = ++p.step[s];
        if (st == p.T_total) {
          if (vs >= 0) set_error(p.err, kErrSched);
          vs = s;
        } else if (st == p.T_draft) {
          if (ds >= 0) set_error(p.err, kErrSched);
          ds = s;
        }
      }
    }
    p.c_slot[2 * b] = vs;
    p.c_slot[2 * b + 1] = ds;
    int32_t* r0 = p.c_tab + (long long)(2 * b) * p.c_cols;
    int32_t* r1 = r0 + p.c_cols;
    if (vs >= 0) sched_fill_row(r0, p.c_cols, p, p.c_slot0, b, vs, 0);
    else sched_pad_row(r0, p.c_cols, p, p.c_slot0);
    if (ds >= 0) sched_fill_row(r1, p.c_cols, p, p.c_slot0, b, ds, 0);
    else sched_pad_row(r1, p.c_cols, p, p.c_slot0);
    if (vs >= 0 || ds >= 0) {
      p.seq_ct[b * kSeqCounters + kCtC] += 1;
      s_any_c = 1;
      atomicAdd(&s_keys, (unsigned long long)((vs >= 0 ? p.pos[vs] + 1 : 0) + (ds >= 0 ? p.pos[ds] + 1 : 0)));
    }
  }
  __syncthreads();
  if (b == 0) {
    if (s_any_c) p.batch_ct[kBtC] += 1;
    p.keys[2] += s_keys;
  }
}

__device__ __forceinline__ void sched_commit(const SchedParams& p, int b, int token) {
  const int n = p.n_commit[b];
  if (n < p.max_new) p.committed[(long long)b * p.max_new + n] = token;
  p.n_commit[b] = n + 1;
  if (n + 1 >= p.max_new) p.done[b] = 1;
}

// Settle: accept / reject the commit point's successor, cascade rollback, queue
// the next token and the new leading-edge draft.  One thread per sequence; the
// sequence's token slots are read once and updated in registers.
__global__ void __launch_bounds__(kSchedThreads) sched_settle_kernel(const SchedParams p) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= p.B || p.done[b]) return;
  const int vs = p.c_slot[2 * b], ds = p.c_slot[2 * b + 1];
  int32_t* ct = p.seq_ct + b * kSeqCounters;
  const int base = b * p.W;
  uint32_t alive = 0, wave = 0;  // bit j: slot j alive / alive and in the wave
  int pos[kSchedMaxW];
#pragma unroll 4
  for (int j = 0; j < p.W; ++j) {
    const int a = p.alive[base + j], st = p.state[base + j];
    pos[j] = p.pos[base + j];
    if (a) alive |= 1u << j;
    if (a && st == 2) wave |= 1u << j;
  }
  const uint32_t all = p.W >= 32 ? 0xffffffffu : ((1u << p.W) - 1u);
  auto drop = [&](int j) {
    p.alive[base + j] = 0;
    p.state[base + j] = 0;
    alive &= ~(1u << j);
    wave &= ~(1u << j);
  };
  // queue a token for the prelude in the first free slot (sched order of the host)
  auto queue = [&](int token, int position) {
    const uint32_t free_slots = ~alive & all;
    if (!free_slots) {
      set_error(p.err, kErrSched);
      return;
    }
    const int j = __ffs(free_slots) - 1, s = base + j;
    p.alive[s] = 1;
    p.state[s] = 1;
    p.tok[s] = token;
    p.pos[s] = position;
    p.step[s] = 0;
    alive |= 1u << j;
    pos[j] = position;
    ct[kCtP] += 1;
  };
  bool rejected = false;
  if (vs >= 0) {
    const int gold = p.c_out[2 * b];
    const int next_pos = pos[vs - base] + 1;
    drop(vs - base);
    int nxt = -1;
    for (uint32_t bits = wave; bits; bits &= bits - 1) {
      const int j = __ffs(bits) - 1;
      if (pos[j] == next_pos) nxt = base + j;
    }
    if (nxt < 0) {  // boundary: nothing speculated at next_pos
      sched_commit(p, b, gold);
      if (!p.done[b]) queue(gold, next_pos);
      else ct[kCtP] += 1;  // the host queues it before noticing the sequence is done
    } else {
      bool accept;
      if (p.emu != nullptr) {
        const int k = p.emu_ctr[b]++;
        accept = k < p.emu_len ? p.emu[(long long)b * p.emu_len + k] != 0 : false;
        if (k >= p.emu_len) set_error(p.err, kErrSched);
      } else {
        accept = gold == p.tok[nxt];
      }
      ct[kCtProp] += 1;
      if (accept) {
        ct[kCtAcc] += 1;
        sched_commit(p, b, p.tok[nxt]);
      } else {
        ct[kCtRej] += 1;
        ct[kCtRoll] += 1;
        rejected = true;
        sched_commit(p, b, gold);
        for (uint32_t bits = alive; bits; bits &= bits - 1) {  // rollback: every token at or after next_pos
          const int j = __ffs(bits) - 1;
          if (pos[j] >= next_pos) drop(j);
        }
        for (int k = 0; k < p.n_kv_slots; ++k) {
          int32_t* l = p.lens + (long long)k * p.lens_stride + b;
          if (*l > next_pos) *l = next_pos;
        }
        if (!p.done[b]) queue(gold, next_pos);
        else ct[kCtP] += 1;
      }
    }
  }
  if (p.done[b]) {  // finished: drop the working state (clear_working_state)
    for (int j = 0; j < p.W; ++j) {
      p.alive[base + j] = 0;
      p.state[base + j] = 0;
    }
    return;
  }
  if (!rejected && ds >= 0) queue(p.c_out[2 * b + 1], pos[ds - base] + 1);
}

}  // namespace wfd
