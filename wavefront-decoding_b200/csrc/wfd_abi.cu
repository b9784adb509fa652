// extern "C" entry points of libwfd_b200.so (declared in include/wfd_b200.h).
//
// Host side only: argument checks, workspace carving, kernel-variant selection
// and launches.  Every launch goes to the caller's stream; nothing here
// allocates device memory or synchronises (except wfd_read_error, whose job is
// to read the device error word).
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <utility>
#include <mutex>

#include "wfd_cache.cuh"
#include "wfd_common.cuh"
#include "wfd_decode.cuh"
#include "wfd_linear.cuh"
#include "wfd_model.cuh"
#include "wfd_sched.cuh"
#include "wfd_plan.cuh"
#include "wfd_prefill.cuh"
#include "wfd_verify.cuh"

using namespace wfd;

namespace {

constexpr int kMaxDevices = 64;

// Batch-invariant attention (wfd_set_batch_invariant): read when a launch is
// built, so a captured CUDA graph keeps the mode it was captured with.
std::atomic<int> g_batch_invariant{0};
// Test hook (wfd_test_fail_waits): every bounded wait of the tensor-core kernel
// gives up at once.  Read when a launch is built.
std::atomic<int> g_fail_waits{0};
constexpr int kGridPerSm = 4;  // upper bound on resident decode CTAs per SM used for sizing

struct DevInfo {
  int sms = 0;
  bool init = false;
};
DevInfo g_dev[kMaxDevices];
std::mutex g_mu;

int current_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev[dev].init) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_dev[dev].sms = sms;
    g_dev[dev].init = true;
  }
  return g_dev[dev].sms;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int elem_bytes(int dtype) { return dtype == WFD_DTYPE_BF16 ? 2 : 4; }
inline int pow2ceil(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}
constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Largest NQ the CUDA-core kernel is built for: query vectors per unit are
// register-resident (q and the output accumulator), so 16-byte-vector bf16 rows
// stop at 8 vectors and fp32 rows at 16.
inline int nq_cap(int dtype, int dh) { return dtype == WFD_DTYPE_BF16 ? 8 : 16; }

// Workspace layout, all regions 256-byte aligned.  The arrival counters come
// first, at an offset that depends on nothing but the device: they must stay
// zero between launches, so every call has to find them at the same place
// whatever its item count or head_dim.
struct WsLayout {
  size_t cnt, part, segs, prefix, start, total;
};

constexpr size_t ws_part_floats(bool tc_only, int head_dim, size_t sms) {
  // decode: NQ <= 16 query vectors per partial slot, kGridPerSm CTAs per SM;
  // tensor cores: kVerifyMaxRows vectors per slot, one CTA per SM.
  return tc_only ? 2 * sms * kVerifyMaxRows * (size_t)(head_dim + 2)
                 : (2 * sms * kGridPerSm * (size_t)16 * (head_dim + 2) > 2 * sms * kVerifyMaxRows * (size_t)(head_dim + 2)
                        ? 2 * sms * kGridPerSm * (size_t)16 * (head_dim + 2)
                        : 2 * sms * kVerifyMaxRows * (size_t)(head_dim + 2));
}

WsLayout ws_layout(int max_items, int head_dim, int sms, bool tc_only = false) {
  WsLayout w;
  const size_t n_ctas = (size_t)sms * kGridPerSm;
  w.cnt = 0;
  w.part = align256(w.cnt + n_ctas * sizeof(int));
  w.segs = align256(w.part + ws_part_floats(tc_only, head_dim, (size_t)sms) * sizeof(float));
  w.prefix = align256(w.segs + (size_t)max_items * sizeof(Seg));
  w.start = align256(w.prefix + (size_t)(max_items + 1) * sizeof(long long));
  w.total = align256(w.start + (size_t)sms * sizeof(CtaStart));
  return w;
}

// Launch with programmatic stream serialization (the kernel calls
// griddep_wait() before reading its predecessor's outputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename T, int DH, int NQ>
int launch_decode_t(const DecodeParams& p, int sms, cudaStream_t st) {
  using C = DecodeCfg<T, DH, NQ>;
  static bool attr_set[kMaxDevices] = {};
  static int occ_cache[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(wave_decode_kernel<T, DH, NQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return WFD_ERR_CUDA;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, wave_decode_kernel<T, DH, NQ>, C::THREADS, C::SMEM) !=
        cudaSuccess)
      return WFD_ERR_CUDA;
    occ_cache[dev] = occ < 1 ? 1 : (occ > kGridPerSm ? kGridPerSm : occ);
    attr_set[dev] = true;
  }
  const int grid = sms * occ_cache[dev];
  if (launch_pdl(wave_decode_kernel<T, DH, NQ>, dim3(grid), dim3(C::THREADS), C::SMEM, st, p) != cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

template <typename T, int DH>
int launch_decode_dh(int nq, const DecodeParams& p, int sms, cudaStream_t st) {
  switch (nq) {
    case 1: return launch_decode_t<T, DH, 1>(p, sms, st);
    case 2: return launch_decode_t<T, DH, 2>(p, sms, st);
    case 4: return launch_decode_t<T, DH, 4>(p, sms, st);
    case 8: return launch_decode_t<T, DH, 8>(p, sms, st);
    default: break;
  }
  if constexpr (Elem<T>::kVec == 4) {
    if (nq == 16) return launch_decode_t<T, DH, 16>(p, sms, st);
  }
  return WFD_ERR_UNSUPPORTED;
}

int launch_decode(int dtype, int dh, int nq, const DecodeParams& p, int sms, cudaStream_t st) {
  if (dtype == WFD_DTYPE_BF16) {
    if (dh == 128) return launch_decode_dh<__nv_bfloat16, 128>(nq, p, sms, st);
    if (dh == 64) return launch_decode_dh<__nv_bfloat16, 64>(nq, p, sms, st);
  } else {
    if (dh == 128) return launch_decode_dh<float, 128>(nq, p, sms, st);
    if (dh == 64) return launch_decode_dh<float, 64>(nq, p, sms, st);
  }
  return WFD_ERR_UNSUPPORTED;
}

// ---- tensor maps for the tcgen05 kernel (driver entry point, no -lcuda) ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// (Dh, Hkv, rows) bf16 key / value buffer (Dh 64 or 128); box = 64 dims x 1 head x
// 128 rows, 128-byte swizzle (the UMMA SWIZZLE_128B layout); rows past the end read as 0.
bool make_kv_map(CUtensorMap* m, const void* base, long long rows, int Hkv, int Dh, int box_rows = kTcTile) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)Dh, (cuuint64_t)Hkv, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)Dh * 2, (cuuint64_t)Hkv * Dh * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NQP, int DH, int NA>
int launch_tc(const VerifyParams& vp, const CUtensorMap& tk, const CUtensorMap& tv, const TailMaps& tails, int sms,
              cudaStream_t st) {
  using C = TcCfg<NQP, DH>;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(wave_tc_kernel<NQP, DH, NA>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return WFD_ERR_CUDA;
    attr_set[dev] = true;
  }
  if (launch_pdl(wave_tc_kernel<NQP, DH, NA>, dim3(sms), dim3(tc_threads(NQP)), C::SMEM, st, tk, tv, tails, vp) !=
      cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

// active query columns of the softmax: every unit has at most G * max_q vectors
int verify_active(int nqp, int G, int max_q) {
  if (nqp == 32) return 32;
  const long long nv = (long long)G * max_q;
  return nv <= 1 ? 1 : nv <= 4 ? 4 : 16;
}

template <int DH>
int launch_tc_dh(int nqp, int na, const VerifyParams& vp, const CUtensorMap& tk, const CUtensorMap& tv,
                 const TailMaps& tails, int sms, cudaStream_t st) {
  if (nqp == 32) return launch_tc<32, DH, 32>(vp, tk, tv, tails, sms, st);
  if (na == 1) return launch_tc<16, DH, 1>(vp, tk, tv, tails, sms, st);
  if (na == 4) return launch_tc<16, DH, 4>(vp, tk, tv, tails, sms, st);
  return launch_tc<16, DH, 16>(vp, tk, tv, tails, sms, st);
}

// Dh: the cache's head dim (tensor maps); kdh: the kernel's (128 for head pairs).
int launch_verify(int nqp, int na, const VerifyParams& vp, const void* k, const void* v, long long rows, int Hkv,
                  int Dh, int kdh, int sms, cudaStream_t st) {
  if (rows <= 0 || rows >= (1ll << 31)) return WFD_ERR_UNSUPPORTED;  // TMA row coordinates are int32
  if ((Dh != 64 && Dh != 128) || (kdh != Dh && !(Dh == 64 && kdh == 128 && vp.pair))) return WFD_ERR_UNSUPPORTED;
  // full (128-row) boxes, and the tail pieces (64, 32, 16, 8 rows)
  CUtensorMap tk, tv;
  TailMaps tails;
  if (!make_kv_map(&tk, k, rows, Hkv, Dh) || !make_kv_map(&tv, v, rows, Hkv, Dh)) return WFD_ERR_CUDA;
  for (int pc = 0; pc < 4; ++pc)
    if (!make_kv_map(&tails.k[pc], k, rows, Hkv, Dh, 64 >> pc) || !make_kv_map(&tails.v[pc], v, rows, Hkv, Dh, 64 >> pc))
      return WFD_ERR_CUDA;
  return kdh == 128 ? launch_tc_dh<128>(nqp, na, vp, tk, tv, tails, sms, st)
                    : launch_tc_dh<64>(nqp, na, vp, tk, tv, tails, sms, st);
}

// Common core of every attention entry point: plan, then attend.
struct AttnArgs {
  int mode;
  // plan inputs
  const wfd_item* items;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t *s_q_row0, *s_q_len, *s_k_row0, *s_k_len;
  int n, max_q;
  int n_slots, n_seqs, max_seq, n_rows, total_q, total_k;
  int slot_offset;
  // tensors
  const void *q, *k, *v, *k_new, *v_new;
  void *k_app, *v_app, *out;
  int32_t* lens;
  int Hq, Hkv, Dh, dtype, causal;
  float scale;
  void* ws;
  size_t ws_bytes;
  int* err;
  int which;           // -1 auto, 0 decode kernel, 1 verify kernel
  long long key_rows;  // rows of (Hkv * Dh) elements in k / v (tensor-map extent)
  const int32_t* row_pos;  // slot mode, optional: per-row positions (gapped windows)
  int row_pos_stride;
};

int run_attention(const AttnArgs& A, cudaStream_t st) {
  if (A.n < 0 || A.Hq <= 0 || A.Hkv <= 0 || A.Hq % A.Hkv != 0) return WFD_ERR_INVALID_ARG;
  if (A.n == 0) return WFD_OK;
  if (A.dtype != WFD_DTYPE_BF16 && A.dtype != WFD_DTYPE_F32) return WFD_ERR_UNSUPPORTED;
  if (A.Dh != 64 && A.Dh != 128) return WFD_ERR_UNSUPPORTED;
  if (!A.q || !A.k || !A.v || !A.out || !A.ws) return WFD_ERR_INVALID_ARG;
  if (!aligned16(A.q) || !aligned16(A.k) || !aligned16(A.v) || !aligned16(A.out)) return WFD_ERR_ALIGNMENT;
  if ((A.k_new && !aligned16(A.k_new)) || (A.v_new && !aligned16(A.v_new))) return WFD_ERR_ALIGNMENT;
  const int G = A.Hq / A.Hkv;
  const int sms = current_sms();
  if (sms <= 0) return WFD_ERR_CUDA;

  const int max_q = A.max_q < 1 ? 1 : A.max_q;
  int which = A.which;
  const bool tc_ok = verify_supported(A.dtype, A.Dh, G, max_q) && A.key_rows > 0 && A.key_rows < (1ll << 31);
  // bf16 runs on the tensor cores, decode rows included: measured on B200, config
  // 2 (GQA 4, Dh 128): CUDA-core kernel 54 % of HBM peak (issue-bound), tcgen05
  // kernel 81 %.  Head_dim 64 with an even kv-head count runs as pairs of heads
  // on the 128-dim kernel (the 64-dim tile is bound by the tensor-core issue
  // rate, not HBM); single-row MHA at head_dim 64 with an odd kv-head count stays
  // on the CUDA cores (54 % vs 52 %), as does fp32 (tcgen05 would take it as tf32).
  const bool pair_ok = A.Dh == 64 && A.Hkv % 2 == 0 && 2ll * G * max_q <= kVerifyMaxRows;
  const bool odd_mha_d64_decode = A.Dh == 64 && !pair_ok && (long long)G * max_q == 1;
  const bool invariant = g_batch_invariant.load(std::memory_order_relaxed) != 0;
  if (which < 0) which = (tc_ok && (invariant || !odd_mha_d64_decode || A.row_pos != nullptr)) ? 1 : 0;
  if (which == 1 && !tc_ok) return WFD_ERR_UNSUPPORTED;
  // gapped windows (per-row positions) are read by the tensor-core kernel only
  if (A.row_pos != nullptr && (which != 1 || A.mode != kPlanSlots || A.row_pos_stride < 1)) return WFD_ERR_UNSUPPORTED;
  const bool pair = which == 1 && pair_ok;
  const int Gv = pair ? 2 * G : G;  // query vectors per unit and kv (pair) head

  const WsLayout L = ws_layout(A.n, pair ? 128 : A.Dh, sms, which == 1);
  if (A.ws_bytes < L.total || !aligned16(A.ws)) return WFD_ERR_WORKSPACE;
  char* ws = static_cast<char*>(A.ws);

  int NQ;
  if (which == 0) {
    NQ = pow2ceil(max_q * G);
    const int cap = nq_cap(A.dtype, A.Dh);
    if (NQ > cap) NQ = cap;
  } else {
    NQ = verify_rows(Gv, max_q);
  }

  PlanParams pp;
  memset(&pp, 0, sizeof(pp));
  pp.mode = A.mode;
  pp.n = A.n;
  pp.items = A.items;
  pp.n_slots = A.n_slots;
  pp.n_seqs = A.n_seqs;
  pp.max_seq = A.max_seq;
  pp.n_rows = A.n_rows;
  pp.cu_q = A.cu_q;
  pp.cu_k = A.cu_k;
  pp.total_q = A.total_q;
  pp.total_k = A.total_k;
  pp.s_q_row0 = A.s_q_row0;
  pp.s_q_len = A.s_q_len;
  pp.s_k_row0 = A.s_k_row0;
  pp.s_k_len = A.s_k_len;
  pp.G = which == 1 ? Gv : G;
  pp.NQ = NQ;
  pp.qg_split = 1;
  pp.segs = reinterpret_cast<Seg*>(ws + L.segs);
  pp.prefix = reinterpret_cast<long long*>(ws + L.prefix);
  // Small slot tables: the tcgen05 CTAs plan their own start from the items
  // (and start streaming before the plan kernel ends); otherwise the plan
  // kernel writes one start record per CTA.
  const bool self_plan = which == 1 && A.mode == kPlanSlots && A.n <= kSelfPlanMax;
  if (which == 1 && !self_plan) {  // the tcgen05 grid: one CTA per SM over (pair) kv-head units
    pp.start = reinterpret_cast<CtaStart*>(ws + L.start);
    pp.seg_grid = sms;
    pp.seg_units = pair ? A.Hkv / 2 : A.Hkv;
  }
  pp.row_pos = A.row_pos;
  pp.row_pos_stride = A.row_pos_stride;
  pp.out = A.out;
  pp.Hq = A.Hq;
  pp.Dh = A.Dh;
  pp.elem_bytes = elem_bytes(A.dtype);
  pp.err = A.err;
  // The window rows are appended to the cache before the attention starts, by
  // extra blocks of the plan kernel: the tensor-core kernel reads every key
  // through TMA, and with KV sharing (several items of one launch on the same
  // slot and sequence) an item reads rows another item appends.
  int plan_blocks = 1;
  if (A.k_new != nullptr && A.k_app != nullptr) {
    if (A.mode != kPlanSlots) return WFD_ERR_INVALID_ARG;
    pp.k_new = static_cast<const char*>(A.k_new);
    pp.v_new = static_cast<const char*>(A.v_new);
    pp.k_app = static_cast<char*>(A.k_app);
    pp.v_app = static_cast<char*>(A.v_app);
    pp.row_bytes = (long long)A.Hkv * A.Dh * elem_bytes(A.dtype);
    pp.k_row_offset = (long long)A.slot_offset * A.n_seqs * (long long)A.max_seq;
    pp.lens = A.lens;
    pp.lens_offset = A.slot_offset * A.n_seqs;
    plan_blocks = 1 + (A.n < 4 * sms ? A.n : 4 * sms);
  }
  if (launch_pdl(plan_kernel, dim3(plan_blocks), dim3(kPlanThreads), 0, st, pp) != cudaSuccess)
    return WFD_ERR_CUDA;

  const float scale = A.scale > 0.f ? A.scale : 1.0f / std::sqrt((float)A.Dh);
  const float log2e = 1.4426950408889634f;

  if (which == 1) {
    const long long k_row_offset = (long long)A.slot_offset * A.n_seqs * (long long)A.max_seq;
    VerifyParams vp;
    memset(&vp, 0, sizeof(vp));
    vp.q = A.q;
    vp.out = A.out;
    vp.segs = pp.segs;
    vp.prefix = pp.prefix;
    vp.start = pp.start;
    vp.n_segs = A.n;
    vp.Hq = A.Hq;
    vp.Hkv = pair ? A.Hkv / 2 : A.Hkv;
    vp.G = G;
    vp.pair = pair ? 1 : 0;
    vp.invariant = invariant ? 1 : 0;
    vp.scale_log2 = scale * log2e;
    vp.causal = A.causal;
    vp.k_row_offset = k_row_offset;
    vp.ws_part = reinterpret_cast<float*>(ws + L.part);
    vp.ws_cnt = reinterpret_cast<int*>(ws + L.cnt);
    vp.err = A.err;
    vp.fail_waits = g_fail_waits.load(std::memory_order_relaxed);
    vp.row_pos = A.row_pos;
    vp.row_pos_stride = A.row_pos_stride;
    if (self_plan) {
      vp.items = A.items;
      vp.n_slots = A.n_slots;
      vp.n_seqs = A.n_seqs;
      vp.max_seq = A.max_seq;
      vp.n_rows = A.n_rows;
      vp.Gv = Gv;
      vp.NQ = NQ;
    }
    return launch_verify(NQ, verify_active(NQ, Gv, max_q), vp, A.k, A.v, A.key_rows, A.Hkv, A.Dh, pair ? 128 : A.Dh,
                         sms, st);
  }

  DecodeParams dp;
  memset(&dp, 0, sizeof(dp));
  dp.q = A.q;
  dp.k = A.k;
  dp.v = A.v;
  dp.k_new = A.k_new;
  dp.v_new = A.v_new;
  dp.out = A.out;
  dp.segs = pp.segs;
  dp.prefix = pp.prefix;
  dp.n_segs = A.n;
  dp.Hq = A.Hq;
  dp.Hkv = A.Hkv;
  dp.G = G;
  dp.scale_log2 = scale * log2e;
  dp.causal = A.causal;
  dp.k_row_offset = (long long)A.slot_offset * A.n_seqs * (long long)A.max_seq;
  dp.ws_part = reinterpret_cast<float*>(ws + L.part);
  dp.ws_cnt = reinterpret_cast<int*>(ws + L.cnt);
  dp.err = A.err;
  return launch_decode(A.dtype, A.Dh, NQ, dp, sms, st);
}

// Host-side checks of a slot-table call that need no device data (the ones
// run_attention would otherwise make after the plan has been queued).
int wave_validate(const void* q, const void* k_new, const void* v_new, const void* k_cache, const void* v_cache,
                  const void* out, const wfd_item* items, int32_t n_items, int32_t slot_offset, int32_t n_rows,
                  int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_heads, int32_t n_kv_heads) {
  if (!items || !k_new || !v_new || !k_cache || !v_cache || !q || !out || n_items < 0) return WFD_ERR_INVALID_ARG;
  if (n_slots <= 0 || n_seqs <= 0 || max_seq <= 0 || n_rows < 0) return WFD_ERR_INVALID_ARG;
  if (slot_offset < 0 || slot_offset >= n_slots) return WFD_ERR_INVALID_ARG;
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0) return WFD_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(out) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(k_new) ||
      !aligned16(v_new))
    return WFD_ERR_ALIGNMENT;
  return WFD_OK;
}

int wave_common(int which, const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                void* out, int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q,
                int32_t slot_offset, int32_t n_rows, int32_t n_slots, int32_t n_seqs, int32_t max_seq,
                int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                void* workspace, size_t workspace_bytes, int32_t* d_err, void* stream,
                const int32_t* row_pos = nullptr, int32_t row_pos_stride = 1) {
  if (n_items == 0) return WFD_OK;  // empty tick: nothing to append or attend
  const int rc = wave_validate(q, k_new, v_new, k_cache, v_cache, out, items, n_items, slot_offset, n_rows, n_slots,
                               n_seqs, max_seq, n_heads, n_kv_heads);
  if (rc != WFD_OK) return rc;
  AttnArgs A;
  memset(&A, 0, sizeof(A));
  A.mode = kPlanSlots;
  A.items = items;
  A.n = n_items;
  A.max_q = max_q;
  // items are checked against the slots the table can address at this offset
  A.n_slots = n_slots - slot_offset;
  A.n_seqs = n_seqs;
  A.max_seq = max_seq;
  A.n_rows = n_rows;
  A.slot_offset = slot_offset;
  A.q = q;
  A.k = k_cache;
  A.v = v_cache;
  A.k_new = k_new;
  A.v_new = v_new;
  A.k_app = k_cache;
  A.v_app = v_cache;
  A.out = out;
  A.lens = lens;
  A.Hq = n_heads;
  A.Hkv = n_kv_heads;
  A.Dh = head_dim;
  A.dtype = dtype;
  A.causal = 1;
  A.scale = scale;
  A.ws = workspace;
  A.ws_bytes = workspace_bytes;
  A.err = d_err;
  A.which = which;
  A.key_rows = (long long)n_slots * n_seqs * (long long)max_seq;
  A.row_pos = row_pos;
  A.row_pos_stride = row_pos_stride;
  return run_attention(A, static_cast<cudaStream_t>(stream));
}

CacheGeom geom(int n_slots, int n_seqs, int max_seq, int Hkv, int Dh, int dtype) {
  CacheGeom g;
  g.n_slots = n_slots;
  g.n_seqs = n_seqs;
  g.max_seq = max_seq;
  g.Hkv = Hkv;
  g.Dh = Dh;
  g.elem_bytes = elem_bytes(dtype);
  return g;
}

bool geom_ok(int n_slots, int n_seqs, int max_seq, int Hkv, int Dh, int dtype) {
  if (n_slots <= 0 || n_seqs <= 0 || max_seq <= 0 || Hkv <= 0 || Dh <= 0) return false;
  if (dtype != WFD_DTYPE_BF16 && dtype != WFD_DTYPE_F32) return false;
  return ((long long)Hkv * Dh * elem_bytes(dtype)) % 16 == 0;
}

// ---- fixed workspace for wfd_wave_attn_static (no device allocation) ----
// Sized for the tensor-core path (bf16, head_dim 128) with up to
// kStaticMaxItems work items on a device with up to kStaticMaxSms SMs.
constexpr int kStaticMaxItems = 4096;
constexpr int kStaticMaxSms = 160;

constexpr size_t static_ws_bytes() {
  return align256(align256(align256(align256(align256((size_t)kStaticMaxSms * kGridPerSm * sizeof(int)) +
                                             ws_part_floats(true, 128, kStaticMaxSms) * sizeof(float)) +
                                    (size_t)kStaticMaxItems * sizeof(Seg)) +
                           (size_t)(kStaticMaxItems + 1) * sizeof(long long)) +
                  (size_t)kStaticMaxSms * sizeof(CtaStart));
}
constexpr size_t kStaticWsBytes = static_ws_bytes();

}  // namespace

// One copy per device that loads the library, kept until the process exits.
// Host code must not use this name as a device address: the device address
// comes from cudaGetSymbolAddress (static_ws_device_ptr below).
static __device__ __align__(256) unsigned char g_wfd_static_ws[kStaticWsBytes];

namespace {

void* g_static_ptr[kMaxDevices] = {};

// Resolve the array's device address once per device, with that device current.
void* static_ws_device_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_wfd_static_ws) != cudaSuccess) return nullptr;
    g_static_ptr[dev] = p;
  }
  return g_static_ptr[dev];
}

}  // namespace

extern "C" {

int wfd_wave_attn_static(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                         void* out, int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q,
                         int32_t slot_offset, int32_t n_rows, int32_t n_slots, int32_t n_seqs, int32_t max_seq,
                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                         int32_t* d_err, void* stream) {
  // first, whatever the arguments: the array's device address on this device,
  // so that a first call of any shape (an empty one included) does the lookup
  void* ws = static_ws_device_ptr();
  if (ws == nullptr) return WFD_ERR_CUDA;
  if (dtype != WFD_DTYPE_BF16 || head_dim != 128) return WFD_ERR_UNSUPPORTED;
  if (n_items < 0 || n_items > kStaticMaxItems) return WFD_ERR_WORKSPACE;
  const int sms = current_sms();
  if (sms <= 0) return WFD_ERR_CUDA;
  if (sms > kStaticMaxSms) return WFD_ERR_WORKSPACE;
  if (n_items == 0) return WFD_OK;
  // every host-side check before the first thing is queued on the stream: a
  // rejected call leaves the stream untouched
  const int rc = wave_validate(q, k_new, v_new, k_cache, v_cache, out, items, n_items, slot_offset, n_rows, n_slots,
                               n_seqs, max_seq, n_heads, n_kv_heads);
  if (rc != WFD_OK) return rc;
  if ((long long)n_slots * n_seqs * (long long)max_seq >= (1ll << 31)) return WFD_ERR_UNSUPPORTED;
  const WsLayout L = ws_layout(n_items, head_dim, sms, true);
  if (L.total > kStaticWsBytes) return WFD_ERR_WORKSPACE;
  // the split-K arrival counters must start at zero; the array keeps whatever
  // the previous call (possibly an aborted one) left there
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(ws, 0, L.part, st) != cudaSuccess) return WFD_ERR_CUDA;
  return wave_common(1, q, k_new, v_new, k_cache, v_cache, out, lens, items, n_items, max_q, slot_offset, n_rows,
                     n_slots, n_seqs, max_seq, n_heads, n_kv_heads, head_dim, dtype, scale, ws, kStaticWsBytes,
                     d_err, stream);
}

int wfd_abi_version(void) { return WFD_ABI_VERSION; }

const char* wfd_status_string(int status) {
  switch (status) {
    case WFD_OK: return "ok";
    case WFD_ERR_INVALID_ARG: return "invalid argument";
    case WFD_ERR_UNSUPPORTED: return "unsupported dtype / head_dim / shape";
    case WFD_ERR_WORKSPACE: return "workspace missing or too small";
    case WFD_ERR_CUDA: return "CUDA runtime error";
    case WFD_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case WFD_ERR_DEVICE_TIMEOUT: return "device: bounded wait gave up";
    case WFD_ERR_DEVICE_BOUNDS: return "device: index or length out of range";
    default: return "unknown status";
  }
}

int wfd_set_batch_invariant(int32_t on) {
  g_batch_invariant.store(on ? 1 : 0);
  return WFD_OK;
}

int wfd_get_batch_invariant(void) { return g_batch_invariant.load(); }

int wfd_test_fail_waits(int32_t on) {
  g_fail_waits.store(on ? 1 : 0);
  return WFD_OK;
}

int wfd_read_error(int32_t* d_err, int32_t* h_err, void* stream) {
  if (!d_err || !h_err) return WFD_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess) return WFD_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return WFD_ERR_CUDA;
  *h_err = v;
  if (v == 0) return WFD_OK;
  if (cudaMemsetAsync(d_err, 0, sizeof(int32_t), st) != cudaSuccess) return WFD_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return WFD_ERR_CUDA;
  return (v & kErrTimeout) ? WFD_ERR_DEVICE_TIMEOUT : WFD_ERR_DEVICE_BOUNDS;
}

size_t wfd_workspace_bytes(int32_t max_items, int32_t head_dim, int32_t dtype) {
  (void)dtype;
  const int sms = current_sms();
  if (sms <= 0 || max_items < 0) return 0;
  return ws_layout(max_items, head_dim, sms).total;
}

int wfd_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (!workspace) return WFD_ERR_INVALID_ARG;
  return cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess ? WFD_OK
                                                                                                  : WFD_ERR_CUDA;
}

int wfd_wave_attn(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache, void* out,
                  int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q, int32_t slot_offset,
                  int32_t n_rows, int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_heads,
                  int32_t n_kv_heads, int32_t head_dim, int32_t dtype, float scale, void* workspace,
                  size_t workspace_bytes, int32_t* d_err, void* stream) {
  return wave_common(-1, q, k_new, v_new, k_cache, v_cache, out, lens, items, n_items, max_q, slot_offset, n_rows,
                     n_slots, n_seqs, max_seq, n_heads, n_kv_heads, head_dim, dtype, scale, workspace,
                     workspace_bytes, d_err, stream);
}

int wfd_wave_attn_kernel(int32_t which, const void* q, const void* k_new, const void* v_new, void* k_cache,
                         void* v_cache, void* out, int32_t* lens, const wfd_item* items, int32_t n_items,
                         int32_t max_q, int32_t slot_offset, int32_t n_rows, int32_t n_slots, int32_t n_seqs,
                         int32_t max_seq, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype,
                         float scale, void* workspace, size_t workspace_bytes, int32_t* d_err, void* stream) {
  if (which != 0 && which != 1) return WFD_ERR_INVALID_ARG;
  return wave_common(which, q, k_new, v_new, k_cache, v_cache, out, lens, items, n_items, max_q, slot_offset,
                     n_rows, n_slots, n_seqs, max_seq, n_heads, n_kv_heads, head_dim, dtype, scale, workspace,
                     workspace_bytes, d_err, stream);
}

int wfd_wave_attn_rows(int32_t which, const void* q, const void* k_new, const void* v_new, void* k_cache,
                       void* v_cache, void* out, int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q,
                       const int32_t* row_pos, int32_t row_pos_stride, int32_t slot_offset, int32_t n_rows,
                       int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_heads, int32_t n_kv_heads,
                       int32_t head_dim, int32_t dtype, float scale, void* workspace, size_t workspace_bytes,
                       int32_t* d_err, void* stream) {
  if (which < -1 || which > 1) return WFD_ERR_INVALID_ARG;
  if (row_pos != nullptr && row_pos_stride < 1) return WFD_ERR_INVALID_ARG;
  return wave_common(which, q, k_new, v_new, k_cache, v_cache, out, lens, items, n_items, max_q, slot_offset, n_rows,
                     n_slots, n_seqs, max_seq, n_heads, n_kv_heads, head_dim, dtype, scale, workspace,
                     workspace_bytes, d_err, stream, row_pos, row_pos_stride);
}

int wfd_attn_varlen(const void* q, const void* k, const void* v, void* out, const int32_t* cu_q, const int32_t* cu_k,
                    int32_t n_seg, int32_t max_q, int32_t total_q, int32_t total_k, int32_t n_heads,
                    int32_t n_kv_heads, int32_t head_dim, int32_t dtype, int32_t causal, float scale,
                    void* workspace, size_t workspace_bytes, int32_t* d_err, void* stream) {
  if (!cu_q || !cu_k || total_q < 0 || total_k < 0) return WFD_ERR_INVALID_ARG;
  AttnArgs A;
  memset(&A, 0, sizeof(A));
  A.mode = kPlanCu;
  A.cu_q = cu_q;
  A.cu_k = cu_k;
  A.n = n_seg;
  A.max_q = max_q;
  A.total_q = total_q;
  A.total_k = total_k;
  A.q = q;
  A.k = k;
  A.v = v;
  A.out = out;
  A.Hq = n_heads;
  A.Hkv = n_kv_heads;
  A.Dh = head_dim;
  A.dtype = dtype;
  A.causal = causal ? 1 : 0;
  A.scale = scale;
  A.ws = workspace;
  A.ws_bytes = workspace_bytes;
  A.err = d_err;
  A.which = -1;
  A.key_rows = total_k;
  return run_attention(A, static_cast<cudaStream_t>(stream));
}

int wfd_attn_segments(const void* q, const void* k, const void* v, void* out, const int32_t* q_row0,
                      const int32_t* q_len, const int32_t* k_row0, const int32_t* k_len, int32_t n_seg,
                      int32_t max_q, int32_t total_q, int32_t total_k, int32_t n_heads, int32_t n_kv_heads,
                      int32_t head_dim, int32_t dtype, int32_t causal, float scale, void* workspace,
                      size_t workspace_bytes, int32_t* d_err, void* stream) {
  if (!q_row0 || !q_len || !k_row0 || !k_len || total_q < 0 || total_k < 0) return WFD_ERR_INVALID_ARG;
  AttnArgs A;
  memset(&A, 0, sizeof(A));
  A.mode = kPlanSegs;
  A.s_q_row0 = q_row0;
  A.s_q_len = q_len;
  A.s_k_row0 = k_row0;
  A.s_k_len = k_len;
  A.n = n_seg;
  A.max_q = max_q;
  A.total_q = total_q;
  A.total_k = total_k;
  A.q = q;
  A.k = k;
  A.v = v;
  A.out = out;
  A.Hq = n_heads;
  A.Hkv = n_kv_heads;
  A.Dh = head_dim;
  A.dtype = dtype;
  A.causal = causal ? 1 : 0;
  A.scale = scale;
  A.ws = workspace;
  A.ws_bytes = workspace_bytes;
  A.err = d_err;
  A.which = -1;
  A.key_rows = total_k;
  return run_attention(A, static_cast<cudaStream_t>(stream));
}

int wfd_attn_prefill(const void* q, const void* k, const void* v, void* out, int32_t n_seqs, int32_t q_len,
                     int32_t k_len, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype,
                     int32_t causal, float scale, int32_t* d_err, void* stream) {
  if (dtype != WFD_DTYPE_BF16 || (head_dim != 64 && head_dim != 128)) return WFD_ERR_UNSUPPORTED;
  if (n_seqs < 0 || q_len < 0 || k_len < 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0)
    return WFD_ERR_INVALID_ARG;
  if (n_seqs == 0 || q_len == 0) return WFD_OK;
  if (!q || !k || !v || !out) return WFD_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return WFD_ERR_ALIGNMENT;
  const long long q_rows = (long long)n_seqs * q_len, k_rows = (long long)n_seqs * k_len;
  if (k_len == 0 || q_rows >= (1ll << 31) || k_rows >= (1ll << 31)) return WFD_ERR_UNSUPPORTED;
  const int sms = current_sms();
  if (sms <= 0) return WFD_ERR_CUDA;
  CUtensorMap tq, tk, tv;
  if (!make_kv_map(&tq, q, q_rows, n_heads, head_dim) || !make_kv_map(&tk, k, k_rows, n_kv_heads, head_dim) ||
      !make_kv_map(&tv, v, k_rows, n_kv_heads, head_dim))
    return WFD_ERR_CUDA;
  PrefillParams pp;
  memset(&pp, 0, sizeof(pp));
  pp.out = out;
  pp.n_seqs = n_seqs;
  pp.Lq = q_len;
  pp.Lk = k_len;
  pp.Hq = n_heads;
  pp.Hkv = n_kv_heads;
  pp.G = n_heads / n_kv_heads;
  pp.causal = causal ? 1 : 0;
  pp.n_qb = (q_len + 127) / 128;
  pp.scale_log2 = (scale > 0.f ? scale : 1.0f / std::sqrt((float)head_dim)) * 1.4426950408889634f;
  pp.err = d_err;
  const long long tiles = (long long)n_seqs * n_heads * pp.n_qb;
  if (tiles >= (1ll << 31)) return WFD_ERR_UNSUPPORTED;
  const int grid = (int)(tiles < sms ? tiles : sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr64[kMaxDevices] = {}, attr128[kMaxDevices] = {};
  cudaError_t e;
  if (head_dim == 64) {
    if (!attr64[dev]) {
      if (cudaFuncSetAttribute(prefill_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, PfCfg<64>::SMEM) !=
          cudaSuccess)
        return WFD_ERR_CUDA;
      attr64[dev] = true;
    }
    e = launch_pdl(prefill_tc_kernel<64>, dim3(grid), dim3(kPfThreads), PfCfg<64>::SMEM, st, tq, tk, tv, pp);
  } else {
    if (!attr128[dev]) {
      if (cudaFuncSetAttribute(prefill_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               PfCfg<128>::SMEM) != cudaSuccess)
        return WFD_ERR_CUDA;
      attr128[dev] = true;
    }
    e = launch_pdl(prefill_tc_kernel<128>, dim3(grid), dim3(kPfThreads), PfCfg<128>::SMEM, st, tq, tk, tv, pp);
  }
  if (e != cudaSuccess) return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

int wfd_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache, int32_t* lens,
               const int32_t* slots, const int32_t* seqs, const int32_t* positions, int32_t n, int32_t slot_offset,
               int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_kv_heads, int32_t head_dim,
               int32_t dtype, int32_t* d_err, void* stream) {
  if (!geom_ok(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype)) return WFD_ERR_INVALID_ARG;
  if (n < 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!k_new || !v_new || !k_cache || !v_cache || !slots || !seqs || !positions) return WFD_ERR_INVALID_ARG;
  if (!aligned16(k_new) || !aligned16(v_new) || !aligned16(k_cache) || !aligned16(v_cache)) return WFD_ERR_ALIGNMENT;
  const int threads = 256;
  const int blocks = (int)(((long long)n * 32 + threads - 1) / threads);
  if (launch_pdl(append_kernel, dim3(blocks), dim3(threads), 0, static_cast<cudaStream_t>(stream),
                 static_cast<const char*>(k_new), static_cast<const char*>(v_new), static_cast<char*>(k_cache),
                 static_cast<char*>(v_cache), lens, slots, seqs, positions, n, slot_offset,
                 geom(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype), d_err) != cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

int wfd_write_prefill(const void* k, const void* v, void* k_cache, void* v_cache, int32_t* lens, int32_t slot,
                      int32_t L, int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_kv_heads,
                      int32_t head_dim, int32_t dtype, void* stream) {
  if (!geom_ok(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype)) return WFD_ERR_INVALID_ARG;
  if (slot < 0 || slot >= n_slots || L < 0 || L > max_seq) return WFD_ERR_INVALID_ARG;
  if (L == 0) return WFD_OK;
  if (!k || !v || !k_cache || !v_cache) return WFD_ERR_INVALID_ARG;
  if (!aligned16(k) || !aligned16(v) || !aligned16(k_cache) || !aligned16(v_cache)) return WFD_ERR_ALIGNMENT;
  const int sms = current_sms();
  prefill_kernel<<<sms > 0 ? sms * 4 : 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(k), static_cast<const char*>(v), static_cast<char*>(k_cache),
      static_cast<char*>(v_cache), lens, slot, L, geom(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype));
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

int wfd_commit_drop(int32_t* lens, const int32_t* drop_pos, int32_t n_slots, int32_t n_seqs, void* stream) {
  if (!lens || !drop_pos || n_slots <= 0 || n_seqs <= 0) return WFD_ERR_INVALID_ARG;
  const long long n = (long long)n_slots * n_seqs;
  const int threads = 256;
  commit_drop_kernel<<<(int)((n + threads - 1) / threads), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      lens, drop_pos, n_slots, n_seqs);
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

int wfd_commit_window(void* k_cache, void* v_cache, int32_t* lens, const wfd_item* items, int32_t n_items,
                      const int32_t* accept_len, const uint8_t* accept_mask, int32_t* acc_rows, int32_t* acc_count,
                      int32_t n_rows, int32_t slot_offset, int32_t n_slots, int32_t n_seqs, int32_t max_seq,
                      int32_t n_kv_heads, int32_t head_dim, int32_t dtype, int32_t* d_err, void* stream) {
  if (!geom_ok(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype)) return WFD_ERR_INVALID_ARG;
  if (n_items < 0 || n_rows < 0 || !lens || !items || !k_cache || !v_cache) return WFD_ERR_INVALID_ARG;
  if ((accept_len == nullptr) == (accept_mask == nullptr)) return WFD_ERR_INVALID_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache)) return WFD_ERR_ALIGNMENT;
  if (n_items == 0) return WFD_OK;
  commit_window_kernel<<<n_items, kCommitThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<char*>(k_cache), static_cast<char*>(v_cache), lens, items, n_items, accept_len, accept_mask,
      acc_rows, acc_count, n_rows, slot_offset, geom(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype), d_err);
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

int wfd_gather_pack(const void* k_cache, const void* v_cache, void* k_pack, void* v_pack, const int32_t* slots,
                    const int32_t* seqs, const int32_t* cu_k, int32_t n, int32_t n_slots, int32_t n_seqs,
                    int32_t max_seq, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, int32_t* d_err,
                    void* stream) {
  if (!geom_ok(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype)) return WFD_ERR_INVALID_ARG;
  if (n < 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!k_cache || !v_cache || !k_pack || !v_pack || !slots || !seqs || !cu_k) return WFD_ERR_INVALID_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(k_pack) || !aligned16(v_pack))
    return WFD_ERR_ALIGNMENT;
  dim3 grid(8, n);
  gather_pack_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(k_cache), static_cast<const char*>(v_cache), static_cast<char*>(k_pack),
      static_cast<char*>(v_pack), slots, seqs, cu_k, n, geom(n_slots, n_seqs, max_seq, n_kv_heads, head_dim, dtype),
      d_err);
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// looped-LM block helpers
// ---------------------------------------------------------------------------
namespace {
int model_grid(long long work) {
  const int sms = current_sms();
  long long g = (work + kModelThreads - 1) / kModelThreads;
  const long long cap = (long long)(sms > 0 ? sms : 148) * 8;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}
}  // namespace

extern "C" int wfd_rmsnorm(const void* x, const void* w, void* y, int32_t n, int32_t d, float eps, int32_t dtype,
                           void* stream) {
  if (n < 0 || d <= 0 || d % 8 != 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!x || !w || !y) return WFD_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return WFD_ERR_ALIGNMENT;
  const int grid = (n + kModelThreads / 32 - 1) / (kModelThreads / 32);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3(grid), dim3(kModelThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
                   static_cast<__nv_bfloat16*>(y), n, d, eps) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(rmsnorm_kernel<float>, dim3(grid), dim3(kModelThreads), 0, st, static_cast<const float*>(x),
                   static_cast<const float*>(w), static_cast<float*>(y), n, d, eps) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_rope_split(const void* qkv, const float* cos_tab, const float* sin_tab, const int32_t* pos,
                              int32_t pos_stride, int32_t pos_period, int32_t max_pos, void* q, void* k, void* v,
                              int32_t n, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t style,
                              int32_t dtype, int32_t* d_err, void* stream) {
  if (n < 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 || max_pos <= 0)
    return WFD_ERR_INVALID_ARG;
  if (style != 0 && style != 1) return WFD_ERR_INVALID_ARG;
  if (!pos && pos_period <= 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!qkv || !cos_tab || !sin_tab || !q || !k || !v || !d_err) return WFD_ERR_INVALID_ARG;
  const long long work = (long long)n * (n_heads + 2 * n_kv_heads) * (head_dim / 2);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = model_grid(work);
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(rope_split_kernel<__nv_bfloat16>, dim3(grid), dim3(kModelThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(qkv), cos_tab, sin_tab, pos, pos_stride, pos_period,
                   static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v),
                   n, n_heads, n_kv_heads, head_dim, style, max_pos, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(rope_split_kernel<float>, dim3(grid), dim3(kModelThreads), 0, st, static_cast<const float*>(qkv),
                   cos_tab, sin_tab, pos, pos_stride, pos_period, static_cast<float*>(q), static_cast<float*>(k),
                   static_cast<float*>(v), n, n_heads, n_kv_heads, head_dim, style, max_pos, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

namespace {
// (rows, chunks per row) of a row-scaled kernel: about two CTAs per SM, at least
// one element group per thread of a chunk
dim3 norm_grid(int n, long long per_row_groups) {
  const int sms = current_sms() > 0 ? current_sms() : 148;
  long long gy = (2ll * sms + n - 1) / n;
  const long long cap = (per_row_groups + kNormThreads - 1) / kNormThreads;
  if (gy > cap) gy = cap;
  if (gy < 1) gy = 1;
  if (gy > 65535) gy = 65535;
  return dim3((unsigned)n, (unsigned)gy);
}
bool norm_args_ok(const void* x, int32_t ldx, int32_t d, float eps) {
  return x && d > 0 && d % 8 == 0 && ldx >= d && ldx % 8 == 0 && eps >= 0.f && aligned16(x);
}
}  // namespace

extern "C" int wfd_rope_split_norm(const void* qkv, const void* x, int32_t ldx, int32_t d, float eps,
                                   const float* cos_tab, const float* sin_tab, const int32_t* pos, int32_t pos_stride,
                                   int32_t pos_period, int32_t max_pos, void* q, void* k, void* v, int32_t n,
                                   int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t style, int32_t dtype,
                                   int32_t* d_err, void* stream) {
  if (n < 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 || max_pos <= 0)
    return WFD_ERR_INVALID_ARG;
  if (style != 0 && style != 1) return WFD_ERR_INVALID_ARG;
  if (!pos && pos_period <= 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!qkv || !cos_tab || !sin_tab || !q || !k || !v || !d_err) return WFD_ERR_INVALID_ARG;
  if (!norm_args_ok(x, ldx, d, eps)) return x && !aligned16(x) ? WFD_ERR_ALIGNMENT : WFD_ERR_INVALID_ARG;
  const dim3 grid = norm_grid(n, (long long)(n_heads + 2 * n_kv_heads) * (head_dim / 2));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(rope_split_norm_kernel<__nv_bfloat16>, grid, dim3(kNormThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(x), ldx, d, eps, cos_tab,
                   sin_tab, pos, pos_stride, pos_period, static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k),
                   static_cast<__nv_bfloat16*>(v), n_heads, n_kv_heads, head_dim, style, max_pos, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(rope_split_norm_kernel<float>, grid, dim3(kNormThreads), 0, st, static_cast<const float*>(qkv),
                   static_cast<const float*>(x), ldx, d, eps, cos_tab, sin_tab, pos, pos_stride, pos_period,
                   static_cast<float*>(q), static_cast<float*>(k), static_cast<float*>(v), n_heads, n_kv_heads,
                   head_dim, style, max_pos, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_silu_mul_norm(const void* gu, const void* x, int32_t ldx, int32_t d, float eps, void* out,
                                 int32_t n, int32_t dff, int32_t dtype, void* stream) {
  if (n < 0 || dff <= 0 || dff % 8 != 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!gu || !out) return WFD_ERR_INVALID_ARG;
  if (!aligned16(gu) || !aligned16(out)) return WFD_ERR_ALIGNMENT;
  if (!norm_args_ok(x, ldx, d, eps)) return x && !aligned16(x) ? WFD_ERR_ALIGNMENT : WFD_ERR_INVALID_ARG;
  const dim3 grid = norm_grid(n, dff / 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(silu_mul_norm_kernel<__nv_bfloat16>, grid, dim3(kNormThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(gu), static_cast<const __nv_bfloat16*>(x), ldx, d, eps,
                   static_cast<__nv_bfloat16*>(out), dff) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(silu_mul_norm_kernel<float>, grid, dim3(kNormThreads), 0, st, static_cast<const float*>(gu),
                   static_cast<const float*>(x), ldx, d, eps, static_cast<float*>(out), dff) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_silu_mul(const void* gu, void* out, int32_t n, int32_t dff, int32_t dtype, void* stream) {
  if (n < 0 || dff <= 0 || dff % 8 != 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!gu || !out) return WFD_ERR_INVALID_ARG;
  if (!aligned16(gu) || !aligned16(out)) return WFD_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = model_grid((long long)n * (dff / 8));
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(silu_mul_kernel<__nv_bfloat16>, dim3(grid), dim3(kModelThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), n, dff) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(silu_mul_kernel<float>, dim3(grid), dim3(kModelThreads), 0, st, static_cast<const float*>(gu),
                   static_cast<float*>(out), n, dff) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

// ---- K8: skinny linear layers (wfd_linear) ----
namespace {

// (K, F) bf16 weights: box = 64 features x 128 k rows, 128-byte swizzle (the
// MN-major A operand); features or k rows past the end read as 0.
bool make_w_map(CUtensorMap* m, const void* base, int K, int F) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)F, (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)F * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)kLinTile};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// (n_rows, K) bf16 rows of stride ldx: box = 64 k x np rows, 128-byte swizzle (the
// K-major B operand); rows past n_rows read as 0.
bool make_x_map(CUtensorMap* m, const void* base, int n_rows, int K, int ldx, int np) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)n_rows};
  cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)np};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// k ranges per feature tile (= the cluster size): the largest of 1, 2, 4, 8 with
// at least one 128-row k stage per CTA and at most 7/4 CTAs per SM, so the
// clusters of a launch are resident at once when two CTAs fit an SM (up to 32
// rows per block; whole clusters must fit a GPC).  Depends on F, K and the SM
// count only, never on the row count: the merge order of a row stays the same.
constexpr int kLinMaxSplit = 8;
int linear_split(int n_tiles, int n_k, int sms) {
  int s = 1;
  while (2 * s <= kLinMaxSplit && 2 * s <= n_k && (long long)n_tiles * 2 * s * 4 <= 7ll * sms) s *= 2;
  return s;
}

template <int NP>
int launch_linear(const LinearParams& lp, const CUtensorMap& tw, const CUtensorMap& tx, dim3 grid, int split,
                  cudaStream_t st) {
  using C = LinCfg<NP>;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(linear_tc_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return WFD_ERR_CUDA;
    attr_set[dev] = true;
  }
  // programmatic stream serialization + one cluster per feature tile (its k ranges)
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kLinThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)split;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, linear_tc_kernel<NP>, tw, tx, lp) != cudaSuccess) return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

}  // namespace

extern "C" size_t wfd_linear_params_bytes(void) { return sizeof(wfd_linear_params); }

extern "C" int wfd_linear(const wfd_linear_params* a, void* stream) {
  if (!a) return WFD_ERR_INVALID_ARG;
  const int n = a->n_rows, K = a->K, F = a->F;
  if (n < 0 || K <= 0 || F <= 0 || K % 8 != 0 || F % 8 != 0 || a->ldx < K || a->ldx % 8 != 0)
    return WFD_ERR_INVALID_ARG;
  if (a->mode < WFD_LINEAR_PLAIN || a->mode > WFD_LINEAR_ROPE) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!a->x || !a->w || !a->err) return WFD_ERR_INVALID_ARG;
  if (!aligned16(a->x) || !aligned16(a->w)) return WFD_ERR_ALIGNMENT;
  if (a->mode == WFD_LINEAR_ROPE) {
    if (a->Dh != 64 && a->Dh != 128) return WFD_ERR_UNSUPPORTED;
    if (a->H <= 0 || a->Hkv <= 0 || (long long)(a->H + 2 * a->Hkv) * a->Dh != F || F % kLinTile != 0)
      return WFD_ERR_INVALID_ARG;
    if (a->rope_style != 0 && a->rope_style != 1) return WFD_ERR_INVALID_ARG;
    if (!a->q || !a->k || !a->v || !a->cos_tab || !a->sin_tab || a->max_pos <= 0) return WFD_ERR_INVALID_ARG;
    if (a->pos ? a->pos_stride < 1 : a->pos_period < 1) return WFD_ERR_INVALID_ARG;
  } else {
    if (!a->out) return WFD_ERR_INVALID_ARG;
    const int width = a->mode == WFD_LINEAR_SWIGLU ? F / 2 : F;
    if (a->mode == WFD_LINEAR_SWIGLU && F % kLinTile != 0) return WFD_ERR_INVALID_ARG;
    if (a->ldo < width) return WFD_ERR_INVALID_ARG;
  }
  const int sms = current_sms();
  if (sms <= 0) return WFD_ERR_CUDA;
  const int np = n <= 16 ? 16 : (n <= 32 ? 32 : 64);
  const int rb = (n + np - 1) / np;
  const int n_tiles = (F + kLinTile - 1) / kLinTile;
  const int n_k = (K + kLinTile - 1) / kLinTile;
  const int split = linear_split(n_tiles, n_k, sms);
  if ((long long)n_tiles * split >= (1ll << 31) || rb > 65535) return WFD_ERR_UNSUPPORTED;

  LinearParams lp;
  memset(&lp, 0, sizeof(lp));
  lp.n_rows = n;
  lp.K = K;
  lp.F = F;
  lp.n_k = n_k;
  lp.n_tiles = n_tiles;
  lp.split = split;
  lp.mode = a->mode;
  lp.row_norm = a->row_norm ? 1 : 0;
  lp.eps = a->eps;
  lp.out = static_cast<__nv_bfloat16*>(a->out);
  lp.ldo = a->ldo;
  lp.q = static_cast<__nv_bfloat16*>(a->q);
  lp.k = static_cast<__nv_bfloat16*>(a->k);
  lp.v = static_cast<__nv_bfloat16*>(a->v);
  lp.H = a->H;
  lp.Hkv = a->Hkv;
  lp.Dh = a->Dh;
  lp.style = a->rope_style;
  lp.cosb = a->cos_tab;
  lp.sinb = a->sin_tab;
  lp.pos = a->pos;
  lp.pos_stride = a->pos_stride;
  lp.pos_period = a->pos_period;
  lp.max_pos = a->max_pos;
  lp.err = a->err;

  CUtensorMap tw, tx;
  if (!make_w_map(&tw, a->w, K, F) || !make_x_map(&tx, a->x, n, K, a->ldx, np)) return WFD_ERR_CUDA;
  const dim3 grid((unsigned)(n_tiles * split), (unsigned)rb);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (np == 16) return launch_linear<16>(lp, tw, tx, grid, split, st);
  if (np == 32) return launch_linear<32>(lp, tw, tx, grid, split, st);
  return launch_linear<64>(lp, tw, tx, grid, split, st);
}

extern "C" int wfd_gather_rows(const void* a, const void* b, const int32_t* idx, int32_t idx_stride, void* out,
                               int32_t n, int32_t d, int32_t n_src, int32_t dtype, int32_t* d_err, void* stream) {
  if (n < 0 || d <= 0 || d % 8 != 0 || n_src <= 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!a || !idx || !out || !d_err) return WFD_ERR_INVALID_ARG;
  if (!aligned16(a) || (b && !aligned16(b)) || !aligned16(out)) return WFD_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = model_grid((long long)n * (d / 8));
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(gather_rows_kernel<__nv_bfloat16>, dim3(grid), dim3(kModelThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), idx, idx_stride,
                   static_cast<__nv_bfloat16*>(out), n, d, n_src, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(gather_rows_kernel<float>, dim3(grid), dim3(kModelThreads), 0, st, static_cast<const float*>(a),
                   static_cast<const float*>(b), idx, idx_stride, static_cast<float*>(out), n, d, n_src,
                   d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_scatter_rows(const void* src, const int32_t* idx, int32_t idx_stride, void* dst, void* zero,
                                int32_t n, int32_t d, int32_t n_dst, int32_t dtype, int32_t* d_err, void* stream) {
  if (n < 0 || d <= 0 || d % 8 != 0 || n_dst <= 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!src || !idx || !dst || !d_err) return WFD_ERR_INVALID_ARG;
  if (!aligned16(src) || !aligned16(dst) || (zero && !aligned16(zero))) return WFD_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = model_grid((long long)n * (d / 8));
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(scatter_rows_kernel<__nv_bfloat16>, dim3(grid), dim3(kModelThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(src), idx, idx_stride, static_cast<__nv_bfloat16*>(dst),
                   static_cast<__nv_bfloat16*>(zero), n, d, n_dst, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(scatter_rows_kernel<float>, dim3(grid), dim3(kModelThreads), 0, st,
                   static_cast<const float*>(src), idx, idx_stride, static_cast<float*>(dst),
                   static_cast<float*>(zero), n, d, n_dst, d_err) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_items_from_table(const int32_t* tab, int32_t cols, int32_t c_slot, int32_t c_seq, int32_t c_pos,
                                    int32_t c_qlen, wfd_item* items, int32_t n, void* stream) {
  if (n < 0 || cols <= 0) return WFD_ERR_INVALID_ARG;
  if (c_slot < 0 || c_slot >= cols || c_seq < 0 || c_seq >= cols || c_pos < 0 || c_pos >= cols || c_qlen < 0 ||
      c_qlen >= cols)
    return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!tab || !items) return WFD_ERR_INVALID_ARG;
  if (launch_pdl(items_from_table_kernel, dim3((n + 255) / 256), dim3(256), 0, static_cast<cudaStream_t>(stream),
                 tab, cols, c_slot, c_seq, c_pos, c_qlen, reinterpret_cast<int32_t*>(items), n) != cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_argmax_rows(const void* x, int32_t* out, int32_t n, int32_t V, int32_t dtype, void* stream) {
  if (n < 0 || V <= 0) return WFD_ERR_INVALID_ARG;
  if (n == 0) return WFD_OK;
  if (!x || !out) return WFD_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vec = (V % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
  if (dtype == WFD_DTYPE_BF16) {
    if (launch_pdl(argmax_rows_kernel<__nv_bfloat16>, dim3(n), dim3(kArgmaxThreads), 0, st,
                   static_cast<const __nv_bfloat16*>(x), out, V, vec) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else if (dtype == WFD_DTYPE_F32) {
    if (launch_pdl(argmax_rows_kernel<float>, dim3(n), dim3(kArgmaxThreads), 0, st, static_cast<const float*>(x),
                   out, V, vec) != cudaSuccess)
      return WFD_ERR_CUDA;
  } else
    return WFD_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// device-side wavefront scheduling
// ---------------------------------------------------------------------------
static_assert(sizeof(wfd_sched_params) == sizeof(wfd::SchedParams), "wfd_sched_params layout");
static_assert(offsetof(wfd_sched_params, c_out) == offsetof(wfd::SchedParams, c_out), "wfd_sched_params layout");
static_assert(offsetof(wfd_sched_params, n_coda) == offsetof(wfd::SchedParams, n_coda), "wfd_sched_params layout");
static_assert(offsetof(wfd_sched_params, depth_slots) == offsetof(wfd::SchedParams, depth_slots),
              "wfd_sched_params layout");
static_assert(offsetof(wfd_sched_params, gap_windows) == offsetof(wfd::SchedParams, gap_windows),
              "wfd_sched_params layout");

extern "C" size_t wfd_sched_params_bytes(void) { return sizeof(wfd_sched_params); }

namespace {
int sched_check(const wfd_sched_params* p) {
  if (!p) return WFD_ERR_INVALID_ARG;
  if (p->B <= 0 || p->B > kSchedThreads || p->W <= 0 || p->W > kSchedMaxW) return WFD_ERR_UNSUPPORTED;
  if (p->T_draft < 1 || p->T_total < p->T_draft || p->max_new < 1 || p->r_cap < 1) return WFD_ERR_INVALID_ARG;
  if (p->p_cols < 6 || p->c_cols < 6 || p->emu_len < 0) return WFD_ERR_INVALID_ARG;
  if (!p->alive || !p->state || !p->tok || !p->pos || !p->step || !p->n_commit || !p->done || !p->committed ||
      !p->seq_ct || !p->emu_ctr || !p->batch_ct || !p->keys || !p->c_slot || !p->lens || !p->err || !p->p_tab ||
      !p->r_tab || !p->c_tab || !p->c_out)
    return WFD_ERR_INVALID_ARG;
  return WFD_OK;
}
}  // namespace

extern "C" int wfd_sched_pre_tick(const wfd_sched_params* p, void* stream) {
  const int rc = sched_check(p);
  if (rc != WFD_OK) return rc;
  if (launch_pdl(sched_pre_tick_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream),
                 *reinterpret_cast<const SchedParams*>(p)) != cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_sched_route(const wfd_sched_params* p, void* stream) {
  const int rc = sched_check(p);
  if (rc != WFD_OK) return rc;
  if (launch_pdl(sched_route_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream),
                 *reinterpret_cast<const SchedParams*>(p)) != cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

extern "C" int wfd_sched_settle(const wfd_sched_params* p, void* stream) {
  const int rc = sched_check(p);
  if (rc != WFD_OK) return rc;
  if (launch_pdl(sched_settle_kernel, dim3((p->B + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream),
                 *reinterpret_cast<const SchedParams*>(p)) != cudaSuccess)
    return WFD_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WFD_OK : WFD_ERR_CUDA;
}

