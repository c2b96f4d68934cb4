// Shared device helpers for libcacheslide_sm100: dtype conversion, status
// reporting and paged-slot addressing.  Built for sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cacheslide_b200.h"

#define CS_HOST_CHECK(cond)        \
  do {                             \
    if (!(cond)) return CS_ERR_INVALID; \
  } while (0)

#define CS_LAUNCH_CHECK()                                  \
  do {                                                     \
    if (cudaPeekAtLastError() != cudaSuccess) {            \
      (void)cudaGetLastError();                            \
      return CS_ERR_CUDA;                                  \
    }                                                      \
  } while (0)

namespace cs {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__host__ __device__ inline int dtype_size(int32_t dt) {
  switch (dt) {
    case CS_F32: return 4;
    case CS_F16: return 2;
    case CS_BF16: return 2;
    case CS_F64: return 8;
    default: return 0;
  }
}

__device__ __forceinline__ void report(int32_t* status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---- element conversion ---------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ double to_d(float x) { return (double)x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
  static __device__ __forceinline__ float from_d(double x) { return (float)x; }
};
template <> struct Elem<double> {
  static __device__ __forceinline__ float to_f(double x) { return (float)x; }
  static __device__ __forceinline__ double to_d(double x) { return x; }
  static __device__ __forceinline__ double from_f(float x) { return (double)x; }
  static __device__ __forceinline__ double from_d(double x) { return x; }
};
// float64 -> half/bfloat16 goes through float32 (two roundings), which is how
// torch's `.to(dtype)` converts and therefore what the reference's WCA blend
// produces (wca.py:339-344).
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ double to_d(__half x) { return (double)__half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ __half from_d(double x) {
    return __float2half_rn(__double2float_rn(x));
  }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ double to_d(__nv_bfloat16 x) {
    return (double)__bfloat162float(x);
  }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_d(double x) {
    return __float2bfloat16_rn(__double2float_rn(x));
  }
};

// generic "to accumulation type" helper
template <typename A, typename T>
__device__ __forceinline__ A to_acc(T x) {
  if constexpr (sizeof(A) == 8) return Elem<T>::to_d(x);
  else return Elem<T>::to_f(x);
}
template <typename T, typename A>
__device__ __forceinline__ T from_acc(A x) {
  if constexpr (sizeof(A) == 8) return Elem<T>::from_d(x);
  else return Elem<T>::from_f(x);
}

// ---- paged KV addressing ----------------------------------------------------
// Slot s < native_total lives at cache[s / bs, h, s % bs, e]; otherwise in the
// sidecar row s - native_total.  `e` runs over [0, 2*D): K first, then V.
struct PagedView {
  char* cache;
  char* side_k;
  char* side_v;
  int64_t native_total, side_capacity, bs, head_dim, kv_heads;
  int64_t sb, sh, so, se;      // byte strides of the native view
  int64_t ssr, ssh, sse;       // byte strides of the sidecar
  int esize;

  __host__ static PagedView make(const cs_paged_kv& kv) {
    PagedView p;
    p.esize = dtype_size(kv.dtype);
    p.cache = static_cast<char*>(kv.cache);
    p.side_k = static_cast<char*>(kv.side_k);
    p.side_v = static_cast<char*>(kv.side_v);
    p.native_total = kv.num_blocks * kv.block_size;
    p.side_capacity = (kv.side_k && kv.side_v) ? kv.side_capacity : 0;
    p.bs = kv.block_size;
    p.head_dim = kv.head_dim;
    p.kv_heads = kv.kv_heads;
    p.sb = kv.stride_block * p.esize;
    p.sh = kv.stride_head * p.esize;
    p.so = kv.stride_offset * p.esize;
    p.se = kv.stride_elem * p.esize;
    p.ssr = kv.side_stride_row * p.esize;
    p.ssh = kv.side_stride_head * p.esize;
    p.sse = kv.side_stride_elem * p.esize;
    return p;
  }

  __device__ __forceinline__ bool valid(int64_t s) const {
    return s >= 0 && s < native_total + side_capacity;
  }
  // byte address of element e (0 <= e < 2D) of (slot, head); slot must be valid
  __device__ __forceinline__ char* addr(int64_t s, int64_t h, int64_t e) const {
    if (s < native_total) {
      int64_t b = s / bs, o = s - b * bs;
      return cache + b * sb + h * sh + o * so + e * se;
    }
    int64_t r = s - native_total;
    if (e < head_dim) return side_k + r * ssr + h * ssh + e * sse;
    return side_v + r * ssr + h * ssh + (e - head_dim) * sse;
  }
  // the K and V halves of slot s's records (head 0, element 0) and the
  // byte stride between heads: element e of head h of the K half is at
  // k + h * hstride + e * (element stride); slot must be valid
  __device__ __forceinline__ void record(int64_t s, char*& k, char*& v, int64_t& hstride) const {
    if (s < native_total) {
      const int64_t b = s / bs, o = s - b * bs;
      k = cache + b * sb + o * so;
      v = k + head_dim * se;
      hstride = sh;
    } else {
      const int64_t r = s - native_total;
      k = side_k + r * ssr;
      v = side_v + r * ssr;
      hstride = ssh;
    }
  }
  // whether records can move as aligned 16-byte vectors
  __host__ bool vec16() const {
    if (se != esize) return false;
    if ((head_dim * esize) % 16) return false;
    auto al = [](int64_t x) { return (x % 16) == 0; };
    if (!al(reinterpret_cast<uintptr_t>(cache)) || !al(sb) || !al(sh) || !al(so)) return false;
    if (side_capacity > 0) {
      if (sse != esize) return false;
      if (!al(reinterpret_cast<uintptr_t>(side_k)) || !al(reinterpret_cast<uintptr_t>(side_v)) ||
          !al(ssr) || !al(ssh))
        return false;
    }
    return true;
  }
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ double warp_sum(double x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
template <typename A>
__device__ __forceinline__ A warp_max(A x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    A y = __shfl_xor_sync(0xffffffffu, x, o);
    x = y > x ? y : x;
  }
  return x;
}

// Batched launches: up to kBatchItems requests per launch, request i owning
// the global rows [start[i], start[i + 1]).  The request of global row r is
// the largest i with start[i] <= r (binary search; warp-uniform when a warp
// owns a row).  Requests with no rows are never found.
constexpr int kBatchItems = 64;

__device__ __forceinline__ int batch_item(const int64_t* start, int count, int64_t r) {
  int lo = 0, hi = count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= r) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace cs
