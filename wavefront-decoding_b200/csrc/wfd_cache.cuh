// K3 / K4 — KV-slot cache kernels: append, prefill write, rollback and accept
// commits, packed gather.  All are byte movers (HBM-bound at best, launch-bound
// at decode sizes): 16-byte vector accesses, one warp per K/V row, no smem.
#pragma once

#include "wfd_common.cuh"

namespace wfd {

struct CacheGeom {
  int n_slots, n_seqs, max_seq, Hkv, Dh, elem_bytes;
  __host__ __device__ long long row_bytes() const { return (long long)Hkv * Dh * elem_bytes; }
  __host__ __device__ long long row_index(int slot, int seq, int pos) const {
    return ((long long)slot * n_seqs + seq) * (long long)max_seq + pos;
  }
};

__device__ __forceinline__ void copy_row(char* dst, const char* src, long long bytes, int lane) {
  for (long long o = (long long)lane * 16; o < bytes; o += 32 * 16) {
    *reinterpret_cast<uint4*>(dst + o) = ld_nc_v4(src + o);
  }
}

// write_tokens: one warp per new row.
__global__ void append_kernel(const char* k_new, const char* v_new, char* kc, char* vc, int32_t* lens,
                              const int32_t* slots, const int32_t* seqs, const int32_t* positions, int n,
                              int slot_offset, CacheGeom g, int* err) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const int slot = slots[warp] + slot_offset, seq = seqs[warp], pos = positions[warp];
  if (slot < 0 || slot >= g.n_slots || seq < 0 || seq >= g.n_seqs) {
    if (lane == 0) set_error(err, kErrBadSlot);
    return;
  }
  if (pos < 0 || pos >= g.max_seq) {
    if (lane == 0) set_error(err, kErrBadPos);
    return;
  }
  const long long rb = g.row_bytes();
  const long long dst = g.row_index(slot, seq, pos) * rb;
  copy_row(kc + dst, k_new + (long long)warp * rb, rb, lane);
  copy_row(vc + dst, v_new + (long long)warp * rb, rb, lane);
  if (lane == 0 && lens != nullptr) atomicMax(lens + slot * g.n_seqs + seq, pos + 1);
}

// write_prefill: k, v (n_seqs, L, Hkv, Dh) -> positions [0, L) of `slot`.
__global__ void prefill_kernel(const char* k, const char* v, char* kc, char* vc, int32_t* lens, int slot, int L,
                               CacheGeom g) {
  const long long rb = g.row_bytes();
  const long long n_rows = (long long)g.n_seqs * L;
  const long long nvec = rb / 16;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n_rows * nvec;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / nvec, c = e % nvec;
    const int seq = (int)(row / L), pos = (int)(row % L);
    const long long dst = g.row_index(slot, seq, pos) * rb + c * 16;
    *reinterpret_cast<uint4*>(kc + dst) = ld_nc_v4(k + row * rb + c * 16);
    *reinterpret_cast<uint4*>(vc + dst) = ld_nc_v4(v + row * rb + c * 16);
  }
  if (blockIdx.x == 0 && lens != nullptr) {
    for (int s = threadIdx.x; s < g.n_seqs; s += blockDim.x) atomicMax(lens + slot * g.n_seqs + s, L);
  }
}

// drop_positions_at_and_after for every sequence with drop_pos[b] >= 0.
__global__ void commit_drop_kernel(int32_t* lens, const int32_t* drop_pos, int n_slots, int n_seqs) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n_slots * n_seqs) return;
  const int b = (int)(i % n_seqs);
  const int d = drop_pos[b];
  if (d >= 0 && lens[i] > d) lens[i] = d;
}

// Accept commit: one CTA per item.  Accepted rows move (in order) to positions
// pos0, pos0+1, ...; a row moves only to a position <= its own, and rows are
// moved one at a time with a CTA barrier between them, so no accepted row is
// overwritten before it has been copied.
constexpr int kCommitThreads = 256;

__global__ void __launch_bounds__(kCommitThreads)
    commit_window_kernel(char* kc, char* vc, int32_t* lens, const wfd_item* items, int n_items,
                         const int32_t* accept_len, const uint8_t* accept_mask, int32_t* acc_rows, int32_t* acc_count,
                         int n_rows, int slot_offset, CacheGeom g, int* err) {
  const int it_idx = blockIdx.x;
  if (it_idx >= n_items) return;
  const wfd_item it = items[it_idx];
  const int slot = it.slot + slot_offset;
  const bool ok_slot = slot >= 0 && slot < g.n_slots && it.seq >= 0 && it.seq < g.n_seqs;
  const bool ok_pos = it.pos0 >= 0 && it.q_len >= 0 && (long long)it.pos0 + it.q_len <= g.max_seq;
  if (!ok_slot || !ok_pos) {
    if (threadIdx.x == 0) set_error(err, ok_slot ? kErrBadPos : kErrBadSlot);
    return;
  }
  // the window's q rows index accept_mask and acc_rows (n_rows entries)
  if (it.q_row0 < 0 || (long long)it.q_row0 + it.q_len > n_rows) {
    if (threadIdx.x == 0) set_error(err, kErrBadRows);
    return;
  }
  __shared__ int s_rank[1024];
  __shared__ int s_n;
  if (it.q_len > 1024) {
    if (threadIdx.x == 0) set_error(err, kErrBadRows);
    return;
  }
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < it.q_len; ++j) {
      bool acc;
      if (accept_len != nullptr) {
        acc = j < accept_len[it_idx];
      } else {
        acc = accept_mask[it.q_row0 + j] != 0;
      }
      s_rank[j] = acc ? n++ : -1;
    }
    s_n = n;
    if (acc_count != nullptr) acc_count[it_idx] = n;
    lens[slot * g.n_seqs + it.seq] = it.pos0 + n;
  }
  __syncthreads();
  const int n_acc = s_n;
  if (acc_rows != nullptr) {
    for (int j = threadIdx.x; j < it.q_len; j += blockDim.x) {
      const int rk = s_rank[j];
      if (rk >= 0) acc_rows[it.q_row0 + rk] = it.q_row0 + j;
    }
  }
  const long long rb = g.row_bytes();
  for (int j = 0; j < it.q_len; ++j) {
    const int rk = s_rank[j];
    if (rk >= 0 && rk != j) {
      const long long src = g.row_index(slot, it.seq, it.pos0 + j) * rb;
      const long long dst = g.row_index(slot, it.seq, it.pos0 + rk) * rb;
      for (long long o = (long long)threadIdx.x * 16; o < rb; o += (long long)blockDim.x * 16) {
        const uint4 kv = ld_cg_v4(kc + src + o);
        const uint4 vv = ld_cg_v4(vc + src + o);
        *reinterpret_cast<uint4*>(kc + dst + o) = kv;
        *reinterpret_cast<uint4*>(vc + dst + o) = vv;
      }
      __syncthreads();
    }
  }
  (void)n_acc;
}

// gather_pack: segment i copies positions [0, cu_k[i+1]-cu_k[i]) of (slot, seq).
__global__ void gather_pack_kernel(const char* kc, const char* vc, char* kp, char* vp, const int32_t* slots,
                                   const int32_t* seqs, const int32_t* cu_k, int n, CacheGeom g, int* err) {
  const int i = blockIdx.y;
  if (i >= n) return;
  const int slot = slots[i], seq = seqs[i];
  const int k0 = cu_k[i], k1 = cu_k[i + 1];
  const int len = k1 - k0;
  if (slot < 0 || slot >= g.n_slots || seq < 0 || seq >= g.n_seqs) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_error(err, kErrBadSlot);
    return;
  }
  if (len < 0 || len > g.max_seq || k0 < 0) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_error(err, kErrBadPos);
    return;
  }
  const long long rb = g.row_bytes();
  const long long nvec = rb / 16;
  const long long src0 = g.row_index(slot, seq, 0) * rb;
  const long long dst0 = (long long)k0 * rb;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < (long long)len * nvec;
       e += (long long)gridDim.x * blockDim.x) {
    *reinterpret_cast<uint4*>(kp + dst0 + e * 16) = ld_nc_v4(kc + src0 + e * 16);
    *reinterpret_cast<uint4*>(vp + dst0 + e * 16) = ld_nc_v4(vc + src0 + e * 16);
  }
}

}  // namespace wfd
