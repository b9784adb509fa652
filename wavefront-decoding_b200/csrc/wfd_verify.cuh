// K2 — wavefront verify attention on tcgen05 tensor cores (sm_100a).
// (Interface only in this revision; the kernel body lands with the tcgen05 path.)
#pragma once

#include "wfd_common.cuh"

namespace wfd {

constexpr int kVerifyMinRows = 8;   // window rows from which the tensor-core kernel is preferred
constexpr int kVerifyMaxRows = 64;  // query vectors (window rows x GQA group) per unit

struct VerifyParams {
  const void* q;
  const void* k;
  const void* v;
  const void* k_new;
  const void* v_new;
  void* k_app;
  void* v_app;
  void* out;
  int32_t* lens;
  const Seg* segs;
  const long long* prefix;
  int n_segs;
  int Hq, Hkv, G;
  float scale_log2;
  int causal;
  long long k_row_offset;
  int lens_offset;
  float* ws_part;
  int* ws_cnt;
  int* err;
};

inline bool verify_supported(int dtype, int dh, int G, int max_q) {
  (void)dtype; (void)dh; (void)G; (void)max_q;
  return false;
}
inline int verify_rows(int G, int max_q) { return G * max_q; }
inline int launch_verify(int, int, int, const VerifyParams&, int, cudaStream_t) { return WFD_ERR_UNSUPPORTED; }

}  // namespace wfd
