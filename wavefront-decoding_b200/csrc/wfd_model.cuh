// Fused element-wise kernels of the looped-LM blocks that surround the
// wavefront attention in the engine: RMSNorm, the RoPE + split of a fused QKV
// projection, and the SwiGLU gate.  Each replaces a chain of framework
// element-wise launches (fp32 up-cast, pow / mean / rsqrt / mul, slicing,
// concatenation, down-cast) by one launch that reads its input once and writes
// its output once; all arithmetic is fp32 whatever the storage type.
#pragma once

#include "wfd_common.cuh"

namespace wfd {

constexpr int kModelThreads = 256;

template <typename T>
struct Vec8;  // 8 elements in one 16-byte (bf16) or two 16-byte (f32) accesses

template <>
struct Vec8<__nv_bfloat16> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};

template <>
struct Vec8<float> {
  __device__ __forceinline__ static void load(const float* p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ __forceinline__ static void store(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w, one warp per row, d % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(kModelThreads) rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                 T* __restrict__ y, int n, int d, float eps) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int row = blockIdx.x * (kModelThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const T* xr = x + (long long)row * d;
  T* yr = y + (long long)row * d;
  float ss = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    float v[8];
    Vec8<T>::load(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / (float)d + eps);
  for (int c = lane * 8; c < d; c += 256) {
    float v[8], g[8];
    Vec8<T>::load(xr + c, v);
    Vec8<T>::load(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * g[i];
    Vec8<T>::store(yr + c, v);
  }
}

// qkv (n, (H + 2 Hkv) * Dh) -> q (n, H, Dh) and k (n, Hkv, Dh) rotated by RoPE at
// each row's position, v (n, Hkv, Dh) copied.  The rotation pairs dims (i, i + Dh/2)
// (style 0) or (2i, 2i + 1) (style 1) by the angle of frequency i; cos / sin are
// (positions, Dh/2) fp32 tables.  Row r's position is pos[r * pos_stride], or
// r % pos_period when pos is null (a prompt of pos_period tokens per sequence).
template <typename T>
__global__ void __launch_bounds__(kModelThreads)
    rope_split_kernel(const T* __restrict__ qkv, const float* __restrict__ cosb, const float* __restrict__ sinb,
                      const int32_t* __restrict__ pos, int pos_stride, int pos_period, T* __restrict__ q,
                      T* __restrict__ k, T* __restrict__ v, int n, int H, int Hkv, int Dh, int style, int max_pos,
                      int* err) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int half = Dh >> 1;
  const int heads = H + 2 * Hkv;
  const long long per_row = (long long)heads * half;  // element pairs per row
  const long long total = (long long)n * per_row;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / per_row);
    const int rem = (int)(e - (long long)r * per_row);
    const int hh = rem / half, i = rem - hh * half;
    const T* src = qkv + (long long)r * heads * Dh + (long long)hh * Dh;
    const int i0 = style ? 2 * i : i, i1 = style ? 2 * i + 1 : i + half;
    const float a = to_f(src[i0]), b = to_f(src[i1]);
    if (hh >= H + Hkv) {  // v: plain copy
      T* dst = v + ((long long)r * Hkv + (hh - H - Hkv)) * Dh;
      dst[i0] = src[i0];
      dst[i1] = src[i1];
      continue;
    }
    int p = pos ? pos[(long long)r * pos_stride] : (r % pos_period);
    if (p < 0 || p >= max_pos) {
      set_error(err, kErrBadPos);
      p = 0;
    }
    const float c = cosb[(long long)p * half + i], s = sinb[(long long)p * half + i];
    T* dst = hh < H ? q + ((long long)r * H + hh) * Dh : k + ((long long)r * Hkv + (hh - H)) * Dh;
    dst[i0] = from_f<T>(a * c - b * s);
    dst[i1] = from_f<T>(b * c + a * s);
  }
}

// out (n, dff) = silu(g) * u for gu (n, 2 dff) = [g | u] per row, dff % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(kModelThreads) silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out,
                                                                  int n, int dff) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int vpr = dff / 8;
  const long long total = (long long)n * vpr;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / vpr), c = (int)(e - (long long)r * vpr) * 8;
    float g[8], u[8];
    Vec8<T>::load(gu + (long long)r * 2 * dff + c, g);
    Vec8<T>::load(gu + (long long)r * 2 * dff + dff + c, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = g[i] / (1.f + expf(-g[i])) * u[i];
    Vec8<T>::store(out + (long long)r * dff + c, g);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm folded into the next linear layer: with W' = diag(norm weight) W, the
// layer's output for row r is s_r * (x_r . W') with s_r = rsqrt(mean(x_r^2) + eps),
// so the GEMM takes x itself and the scale rides on the kernel after it.  These
// variants of the RoPE split and the SwiGLU gate compute s_r from x (one CTA per
// row and chunk of the row; every CTA of a row sums x_r^2 in the same order) and
// apply it to the GEMM output before their own arithmetic.  Each row is
// processed independently of the others.
// ---------------------------------------------------------------------------
constexpr int kNormThreads = 256;

// s_r for row `row` of x (d elements, d % 8 == 0), for every thread of the CTA
template <typename T>
__device__ __forceinline__ float row_scale(const T* __restrict__ x, long long ldx, int row, int d, float eps) {
  __shared__ float s_part[kNormThreads / 32];
  const T* xr = x + (long long)row * ldx;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < d; c += kNormThreads * 8) {
    float v[8];
    Vec8<T>::load(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += s_part[w];
  return rsqrtf(tot / (float)d + eps);
}

// rope_split_kernel with the row scale: CTA (row, chunk) handles element pairs
// [chunk * per, (chunk + 1) * per) of the row; v is s_r * its GEMM output.
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    rope_split_norm_kernel(const T* __restrict__ qkv, const T* __restrict__ x, int ldx, int d, float eps,
                           const float* __restrict__ cosb, const float* __restrict__ sinb,
                           const int32_t* __restrict__ pos, int pos_stride, int pos_period, T* __restrict__ q,
                           T* __restrict__ k, T* __restrict__ v, int H, int Hkv, int Dh, int style, int max_pos,
                           int* err) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int r = blockIdx.x;
  const float sc = row_scale(x, ldx, r, d, eps);
  const int half = Dh >> 1;
  const int heads = H + 2 * Hkv;
  const int per_row = heads * half;
  const int per = (per_row + gridDim.y - 1) / gridDim.y;
  const int e0 = blockIdx.y * per, e1 = min(per_row, e0 + per);
  int ps = pos ? pos[(long long)r * pos_stride] : (r % pos_period);
  if (ps < 0 || ps >= max_pos) {
    if (threadIdx.x == 0 && blockIdx.y == 0) set_error(err, kErrBadPos);
    ps = 0;
  }
  const T* src_row = qkv + (long long)r * heads * Dh;
  for (int e = e0 + threadIdx.x; e < e1; e += kNormThreads) {
    const int hh = e / half, i = e - hh * half;
    const T* src = src_row + (long long)hh * Dh;
    const int i0 = style ? 2 * i : i, i1 = style ? 2 * i + 1 : i + half;
    const float a = to_f(src[i0]) * sc, b = to_f(src[i1]) * sc;
    if (hh >= H + Hkv) {
      T* dst = v + ((long long)r * Hkv + (hh - H - Hkv)) * Dh;
      dst[i0] = from_f<T>(a);
      dst[i1] = from_f<T>(b);
      continue;
    }
    const float c = cosb[(long long)ps * half + i], s = sinb[(long long)ps * half + i];
    T* dst = hh < H ? q + ((long long)r * H + hh) * Dh : k + ((long long)r * Hkv + (hh - H)) * Dh;
    dst[i0] = from_f<T>(a * c - b * s);
    dst[i1] = from_f<T>(b * c + a * s);
  }
}

// silu_mul_kernel with the row scale: out = silu(s_r g) * (s_r u), CTA (row, chunk)
// handles 8-element vectors [chunk * per, (chunk + 1) * per) of the row.
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    silu_mul_norm_kernel(const T* __restrict__ gu, const T* __restrict__ x, int ldx, int d, float eps,
                         T* __restrict__ out, int dff) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int r = blockIdx.x;
  const float sc = row_scale(x, ldx, r, d, eps);
  const int vpr = dff / 8;
  const int per = (vpr + gridDim.y - 1) / gridDim.y;
  const int v0 = blockIdx.y * per, v1 = min(vpr, v0 + per);
  for (int vi = v0 + threadIdx.x; vi < v1; vi += kNormThreads) {
    const int c = vi * 8;
    float g[8], u[8];
    Vec8<T>::load(gu + (long long)r * 2 * dff + c, g);
    Vec8<T>::load(gu + (long long)r * 2 * dff + dff + c, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gs = g[i] * sc;
      g[i] = gs / (1.f + expf(-gs)) * (u[i] * sc);
    }
    Vec8<T>::store(out + (long long)r * dff + c, g);
  }
}

}  // namespace wfd

namespace wfd {

// ---------------------------------------------------------------------------
// Engine row plumbing: gathers / scatters of state-pool rows by int32 indices
// (a strided column of the union table), the wave item table built from the
// union table, and the greedy id of each logits row.
// ---------------------------------------------------------------------------

// out[i] = a[idx[i * s]] (+ b[idx[i * s]] when b is given), rows of d elements
template <typename T>
__global__ void __launch_bounds__(kModelThreads)
    gather_rows_kernel(const T* __restrict__ a, const T* __restrict__ b, const int32_t* __restrict__ idx, int stride,
                       T* __restrict__ out, int n, int d, int n_src, int* err) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int vpr = d / 8;
  const long long total = (long long)n * vpr;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(e / vpr), c = (int)(e - (long long)i * vpr) * 8;
    int r = idx[(long long)i * stride];
    if (r < 0 || r >= n_src) {
      set_error(err, kErrBadRows);
      r = 0;
    }
    float v[8];
    Vec8<T>::load(a + (long long)r * d + c, v);
    if (b != nullptr) {
      float w[8];
      Vec8<T>::load(b + (long long)r * d + c, w);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] += w[k];
    }
    Vec8<T>::store(out + (long long)i * d + c, v);
  }
}

// dst[idx[i * s]] = src[i] (and zero[idx[i * s]] = 0 when zero is given)
template <typename T>
__global__ void __launch_bounds__(kModelThreads)
    scatter_rows_kernel(const T* __restrict__ src, const int32_t* __restrict__ idx, int stride, T* __restrict__ dst,
                        T* __restrict__ zero, int n, int d, int n_dst, int* err) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const int vpr = d / 8;
  const long long total = (long long)n * vpr;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(e / vpr), c = (int)(e - (long long)i * vpr) * 8;
    const int r = idx[(long long)i * stride];
    if (r < 0 || r >= n_dst) {
      set_error(err, kErrBadRows);
      continue;
    }
    float v[8];
    Vec8<T>::load(src + (long long)i * d + c, v);
    Vec8<T>::store(dst + (long long)r * d + c, v);
    if (zero != nullptr) {
      float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      Vec8<T>::store(zero + (long long)r * d + c, z);
    }
  }
}

// items[i] = {tab[i][c_slot], tab[i][c_seq], tab[i][c_pos], tab[i][c_qlen], i}
__global__ void items_from_table_kernel(const int32_t* __restrict__ tab, int cols, int c_slot, int c_seq, int c_pos,
                                        int c_qlen, int32_t* __restrict__ items, int n) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int32_t* r = tab + (long long)i * cols;
    int32_t* it = items + (long long)i * 5;
    it[0] = r[c_slot];
    it[1] = r[c_seq];
    it[2] = r[c_pos];
    it[3] = r[c_qlen];
    it[4] = i;
  }
}

// out[r] = argmax over the V logits of row r (the first index of the maximum,
// as torch.argmax), one CTA of kArgmaxThreads per row.  A row of the lm_head
// output is ~100 KB and the launch has only a few rows, so each CTA keeps
// several 16-byte loads in flight per thread (`vec` != 0: V % 8 == 0 and x
// 16-byte aligned) instead of one scalar load at a time.  The comparison is a
// total order on (value, -index), so the result does not depend on which
// thread sees which element.
constexpr int kArgmaxThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const T* __restrict__ x, int32_t* __restrict__ out,
                                                                      int V, int vec) {
  griddep_wait();  // launched with programmatic stream serialization (no early trigger)
  const T* row = x + (long long)blockIdx.x * V;
  float best = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  auto take = [&](float v, int j) {
    if (v > best || (v == best && j < bi)) {
      best = v;
      bi = j;
    }
  };
  if (vec) {
    constexpr int U = 4;  // 16-byte loads in flight per thread
    const int nv = V >> 3;
    int c = threadIdx.x;
    for (; c + (U - 1) * kArgmaxThreads < nv; c += U * kArgmaxThreads) {
      float a[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u) Vec8<T>::load(row + 8 * (c + u * kArgmaxThreads), a[u]);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) take(a[u][i], 8 * (c + u * kArgmaxThreads) + i);
    }
    for (; c < nv; c += kArgmaxThreads) {
      float a[8];
      Vec8<T>::load(row + 8 * c, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) take(a[i], 8 * c + i);
    }
  } else {
    for (int j = threadIdx.x; j < V; j += kArgmaxThreads) take(to_f(row[j]), j);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  __shared__ float sb[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kArgmaxThreads / 32; ++k)
      if (sb[k] > best || (sb[k] == best && si[k] < bi)) {
        best = sb[k];
        bi = si[k];
      }
    out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace wfd
