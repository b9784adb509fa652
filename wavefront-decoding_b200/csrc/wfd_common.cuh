// Shared device helpers for the wavefront attention / KV-slot kernels (sm_100a).
//
// Everything here is plain CUDA + inline PTX for Blackwell: mbarrier-tracked bulk
// copies (the TMA engine's non-tensor path), bounded waits that report through an
// error word instead of trapping, and the segment table the planner produces.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/wfd_b200.h"

namespace wfd {

// One attention segment after planning.  A segment is a run of q_len query rows
// that all read the same key rows [k_row0, k_row0 + k_len) of one key buffer; the
// last q_len keys are the rows those queries appended (bottom-right causal window,
// exactly the FA2/SDPA varlen convention used by the reference's attn_varlen).
struct Seg {
  long long k_row0;   // first key row, in rows of (Hkv * Dh) elements
  int k_len;          // number of keys the last query row sees
  int q_row0;         // first query row in q / out
  int q_len;          // query rows in the segment
  int new_row0;       // >= 0: keys [k_len - q_len, k_len) come from k_new rows new_row0.. and
                      //       are appended to the key buffer; < 0: all keys already in place
  int n_qg;           // query groups (ceil(q_len * G / NQ)) the decode kernel splits the rows into
  int lens_idx;       // slot * n_seqs + seq of the slot length to raise (slot mode), else -1
};
static_assert(sizeof(Seg) == 32, "Seg must stay 32 bytes");

// Where one CTA of the persistent tensor-core grid starts (written by the plan
// kernel): its first segment, that segment's first work index and the next
// segment's (in unit-keys), and the segment itself.  One 64-byte load replaces
// the dependent prefix / segment loads a CTA would otherwise make at start.
struct CtaStart {
  Seg S;
  long long base, nbase;  // nbase: LLONG_MAX for the last segment
  int seg;
  int pad[3];
};
static_assert(sizeof(CtaStart) == 64, "CtaStart must stay 64 bytes");

// Error bits written into the caller's device error word (atomicOr).  The host
// turns them into WFD_ERR_* status codes; no kernel ever traps.
enum : int {
  kErrTimeout = 1 << 0,      // a bounded mbarrier / flag wait gave up
  kErrBadSlot = 1 << 1,      // slot / sequence index out of range
  kErrBadPos = 1 << 2,       // position or length outside the slot capacity
  kErrBadRows = 1 << 3,      // query / new-row index outside the given tensors
  kErrBadSegs = 1 << 4,      // cu_seqlens not monotone / out of range
  kErrSched = 1 << 7,        // device-scheduler invariant (slot overflow, two commit points in a tick)
};

__device__ __forceinline__ void set_error(int* err, int bits) {
  if (err) atomicOr(err, bits);
}

// Checks of a slot-table work item (wfd_item) and the position of its last row:
// row j sits at pos0 + j, or, with per-row positions (gapped windows), at
// row_pos[(q_row0 + j) * rp_stride], increasing, the first one pos0.  Returns
// the error bit (0: valid).
__device__ __forceinline__ int check_slot_item(const wfd_item& it, int n_slots, int n_seqs, int max_seq, int n_rows,
                                               const int32_t* row_pos, int rp_stride, int& last) {
  if (it.slot < 0 || it.slot >= n_slots || it.seq < 0 || it.seq >= n_seqs) return kErrBadSlot;
  if (it.q_row0 < 0 || it.q_len < 0 || (long long)it.q_row0 + it.q_len > n_rows) return kErrBadRows;
  if (it.pos0 < 0) return kErrBadPos;
  last = it.pos0 + it.q_len - 1;
  if (row_pos != nullptr && it.q_len > 0) {
    if (row_pos[(long long)it.q_row0 * rp_stride] != it.pos0) return kErrBadPos;
    last = row_pos[(long long)(it.q_row0 + it.q_len - 1) * rp_stride];
    if (last < it.pos0) return kErrBadPos;
  }
  if ((long long)last + 1 > max_seq) return kErrBadPos;
  return 0;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk copy (PTX ISA 8.x, sm_90+; used here on sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch (sm_90+): a kernel launched with programmatic
// stream serialization may start while its predecessor still runs; it must
// execute griddep_wait() before it touches anything the predecessor writes (or
// reads and this kernel overwrites).  griddep_launch_dependents() lets the next
// such kernel start early.  Both are no-ops without a programmatic dependency.
// Every kernel of this library is launched that way and waits first; only the
// plan -> append -> attention chain inside one call triggers early, because a
// kernel's successor outside the call may be a library kernel that reads our
// output before it waits (seen on B200 as run-to-run differences when an early
// trigger preceded a cuBLAS GEMM).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of the phase (test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: try_wait already suspends for a hardware time slice, so the spin
// limit below is a multi-second ceiling, never reached by a healthy pipeline.
constexpr uint32_t kSpinLimit = 1u << 20;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completion tracked as tx bytes
// on `bar`.  Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// element helpers
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;  // elements per 16-byte vector
  // unpack 8 bf16 (one uint4) into 8 floats: a bf16 is the high half of an fp32.
  __device__ __forceinline__ static void unpack(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <>
struct Elem<float> {
  static constexpr int kVec = 4;
  __device__ __forceinline__ static void unpack(const uint4& u, float (&f)[4]) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float r;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
  // exp2 of a log2-domain score; -inf -> 0.
  return exp2f(x);
}

}  // namespace wfd
