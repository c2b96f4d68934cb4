// Standalone CoPE building blocks on device tensors [head, query, key]:
//   cs_cope_positions      CoPE.contextual_positions   (position.py:295-307)
//   cs_cope_bias           CoPE.positional_bias        (position.py:309-344)
//   cs_cope_validate_path  validate_contextual_path    (position.py:28-114)
//   cs_cope_chunk_offsets  CCPEProfile tables -> per-chunk carried counts
// One warp per (head, query) row; keys are walked newest-first in tiles of 32
// with a warp-shuffle suffix scan and a carried count.
#include <math.h>

#include "common.cuh"

namespace cs {
namespace {

template <typename A> struct Lim;
template <> struct Lim<float> {
  static __device__ __forceinline__ float eps() { return 1.1920928955078125e-07f; }
};
template <> struct Lim<double> {
  static __device__ __forceinline__ double eps() { return 2.220446049250313e-16; }
};

__device__ __forceinline__ float sig(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ double sig(double x) { return 1.0 / (1.0 + exp(-x)); }

template <typename A>
__global__ void positions_kernel(const A* __restrict__ logits, int64_t ls_h, int64_t ls_q,
                                 const uint8_t* __restrict__ allowed, int64_t as_h, int64_t as_q,
                                 int H, int64_t nq, int64_t nk, int npos, A* out, int64_t os_h,
                                 int64_t os_q, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)H * nq;
  const A top = (A)(npos - 1);
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t h = row / nq, q = row - h * nq;
    A carry = A(0);
    int32_t bits = 0;
    for (int64_t t_end = nk; t_end > 0; t_end -= 32) {
      const int64_t j = t_end - 32 + lane;
      A g = A(0);
      if (j >= 0 && allowed[h * as_h + q * as_q + j]) {
        const A x = logits[h * ls_h + q * ls_q + j];
        if (!isfinite(x)) bits |= CS_ST_LOGIT_NONFINITE;
        g = sig(x);
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        A t = __shfl_down_sync(0xffffffffu, g, o);
        if (lane + o < 32) g += t;
      }
      const A r = g + carry;
      carry = __shfl_sync(0xffffffffu, r, 0);
      if (j >= 0) out[h * os_h + q * os_q + j] = r < A(0) ? A(0) : (r > top ? top : r);
    }
    bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
    if (lane == 0 && bits) report(status, bits);
  }
}

// bias[h, q, k] for q rows [nq, H, D] (dtype T) and positions (dtype A)
template <typename T, typename A>
__global__ void bias_kernel(const T* __restrict__ query, int64_t qs_t, int64_t qs_h,
                            const A* __restrict__ E, int64_t es_d, int64_t es_p, int d, int npos,
                            const A* __restrict__ pos, int64_t ps_h, int64_t ps_q, int H,
                            int64_t nq, int64_t nk, A* out, int64_t os_h, int64_t os_q,
                            int32_t* status) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  A* tab = reinterpret_cast<A*>(smem) + (size_t)warp * npos;
  const int64_t rows = (int64_t)H * nq;
  const A top = (A)(npos - 1);
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + warp; row < rows;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t h = row / nq, q = row - h * nq;
    const T* qv = query + q * qs_t + h * qs_h;
    for (int pp = lane; pp < npos; pp += 32) {
      A acc = A(0);
      for (int e = 0; e < d; ++e) acc += to_acc<A>(qv[e]) * E[e * es_d + pp * es_p];
      tab[pp] = acc;
    }
    __syncwarp();
    int32_t bits = 0;
    for (int64_t j = lane; j < nk; j += 32) {
      A p = pos[h * ps_h + q * ps_q + j];
      if (!(p >= A(0) && p <= top)) {
        bits |= CS_ST_POS_RANGE;
        p = p >= A(0) ? (p <= top ? p : top) : A(0);
      }
      const int lo = (int)floor(p);
      const int hi = lo + 1 < npos ? lo + 1 : npos - 1;
      const A f = p - (A)lo;
      out[h * os_h + q * os_q + j] = tab[lo] + f * (tab[hi] - tab[lo]);
    }
    bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
    if (lane == 0 && bits) report(status, bits);
    __syncwarp();
  }
}

template <typename A>
__global__ void validate_kernel(const A* __restrict__ pos, int64_t ps_h, int64_t ps_q,
                                const int64_t* __restrict__ qpos, const int64_t* __restrict__ kpos,
                                const uint8_t* __restrict__ mask, int64_t ms_h, int64_t ms_q,
                                int H, int64_t nq, int64_t nk, A atol, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)H * nq;
  const A eps = Lim<A>::eps();
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t h = row / nq, q = row - h * nq;
    const int64_t qp = qpos[q];
    int32_t bits = 0;
    for (int64_t j = lane; j < nk; j += 32) {
      const A p = pos[h * ps_h + q * ps_q + j];
      if (!isfinite(p)) bits |= CS_ST_POS_RANGE;
      const int64_t kp = kpos[j];
      const bool valid = kp <= qp && (mask == nullptr || mask[h * ms_h + q * ms_q + j]);
      if (!valid) continue;
      const A rnd = eps * fabs(p);
      if (p < -(atol + rnd)) bits |= CS_ST_PATH_NEG;
      A avail = (A)(qp - kp);
      avail = (avail < A(-1) ? A(-1) : avail) + A(1);
      if (p > avail + atol + rnd) bits |= CS_ST_PATH_AVAIL;
      if (j + 1 < nk) {
        const int64_t kn = kpos[j + 1];
        const bool vn = kn <= qp && (mask == nullptr || mask[h * ms_h + q * ms_q + j + 1]);
        if (vn) {
          const A pn = pos[h * ps_h + q * ps_q + j + 1];
          const A diff = p - pn;
          const A ptol = atol + rnd + eps * fabs(pn);
          if (diff < -ptol) bits |= CS_ST_PATH_INCR;
          if (diff > (A)(kn - kp) + ptol) bits |= CS_ST_PATH_GAP;
        }
      }
    }
    bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
    if (lane == 0 && bits) report(status, bits);
  }
}

int rows_grid(int64_t rows, int warps_per_block) {
  int64_t b = (rows + warps_per_block - 1) / warps_per_block;
  int64_t cap = (int64_t)num_sms() * 16;
  if (b > cap) b = cap;
  return b < 1 ? 1 : (int)b;
}

// One warp per (head, query row): the row's offsets are first set to -1
// (carry the running count), then, for a fixed query, every fixed chunk older
// than the query's segment gets the canonical position of its last key minus
// that key's own gate sigmoid(q . k / sqrt(d)) (fp32 logits, as position.py's
// _logits accumulates bf16 / fp16 / fp32 inputs).
template <typename T>
__global__ void chunk_offsets_kernel(const T* __restrict__ q, int64_t qs_t, int64_t qs_h, int nq,
                                     int hq, int d, const int64_t* __restrict__ qpos,
                                     const int32_t* __restrict__ q_ord,
                                     const int32_t* __restrict__ q_seg, const T* __restrict__ k,
                                     int64_t ks_t, int64_t ks_h, int hkv,
                                     const int64_t* __restrict__ last_key,
                                     const int32_t* __restrict__ last_ord,
                                     const int32_t* __restrict__ seg_of_chunk, int nfc,
                                     const float* __restrict__ table, int64_t tb_h, int64_t tb_r,
                                     int64_t tb_c, int tb_rows, int tb_cols, float* offsets,
                                     int64_t of_h, int64_t of_t, int nseg, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)hq * nq;
  const int group = hq / hkv;
  const float inv = 1.f / sqrtf((float)d);
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int h = (int)(row / nq), r = (int)(row - (int64_t)h * nq);
    float* out = offsets + h * of_h + qpos[r] * of_t;
    for (int c = lane; c < nseg; c += 32) out[c] = -1.f;
    __syncwarp();
    const int qo = q_ord[r], qs = q_seg[r];
    if (qo < 0) continue;  // a dynamic query: contextual counts
    if (qo >= tb_rows) {
      if (lane == 0) report(status, CS_ST_POS_RANGE);
      continue;
    }
    const T* qr = q + r * qs_t + h * qs_h;
    for (int f = 0; f < nfc; ++f) {
      const int seg = seg_of_chunk[f];
      if (seg >= qs) continue;  // the query's own chunk and newer: no reset
      const int ko = last_ord[f];
      const T* kr = k + last_key[f] * ks_t + (h / group) * ks_h;
      float dot = 0.f;
      for (int e = lane; e < d; e += 32) dot += Elem<T>::to_f(qr[e]) * Elem<T>::to_f(kr[e]);
      dot = warp_sum(dot);
      if (lane == 0) {
        if (ko < 0 || ko >= tb_cols || seg < 0 || seg >= nseg) {
          report(status, CS_ST_POS_RANGE);
        } else {
          const float gate = 1.f / (1.f + expf(-(dot * inv)));
          out[seg] = table[h * tb_h + (int64_t)qo * tb_r + (int64_t)ko * tb_c] - gate;
        }
      }
    }
  }
}

}  // namespace
}  // namespace cs

using namespace cs;

// logits/out dtype: CS_F32 or CS_F64 (accumulation dtypes); allowed: uint8
extern "C" CS_API int cs_cope_positions(const void* logits, int64_t ls_h, int64_t ls_q,
                                        const uint8_t* allowed, int64_t as_h, int64_t as_q,
                                        int32_t heads, int64_t nq, int64_t nk, int32_t npos,
                                        int32_t dtype, void* out, int64_t os_h, int64_t os_q,
                                        int32_t* status, void* stream) {
  CS_HOST_CHECK(heads > 0 && nq >= 0 && nk >= 0 && npos >= 2);
  if (nq == 0 || nk == 0) return CS_OK;
  CS_HOST_CHECK(logits && allowed && out);
  const int threads = 256;
  auto s = as_stream(stream);
  int g = rows_grid((int64_t)heads * nq, threads / 32);
  if (dtype == CS_F64)
    positions_kernel<double><<<g, threads, 0, s>>>((const double*)logits, ls_h, ls_q, allowed,
                                                   as_h, as_q, heads, nq, nk, npos, (double*)out,
                                                   os_h, os_q, status);
  else if (dtype == CS_F32)
    positions_kernel<float><<<g, threads, 0, s>>>((const float*)logits, ls_h, ls_q, allowed, as_h,
                                                  as_q, heads, nq, nk, npos, (float*)out, os_h,
                                                  os_q, status);
  else
    return CS_ERR_INVALID;
  CS_LAUNCH_CHECK();
  return CS_OK;
}

// query dtype `in_dtype`; E, positions and out in the accumulation dtype
extern "C" CS_API int cs_cope_bias(const void* query, int64_t qs_t, int64_t qs_h, const void* E,
                                   int64_t es_d, int64_t es_p, int32_t d, int32_t npos,
                                   const void* positions, int64_t ps_h, int64_t ps_q,
                                   int32_t heads, int64_t nq, int64_t nk, int32_t in_dtype,
                                   void* out, int64_t os_h, int64_t os_q, int32_t* status,
                                   void* stream) {
  CS_HOST_CHECK(heads > 0 && nq >= 0 && nk >= 0 && npos >= 2 && d > 0);
  if (nq == 0 || nk == 0) return CS_OK;
  CS_HOST_CHECK(query && E && positions && out);
  const int threads = 128;
  auto s = as_stream(stream);
  int g = rows_grid((int64_t)heads * nq, threads / 32);
  size_t acc = in_dtype == CS_F64 ? 8 : 4;
  size_t smem = (threads / 32) * npos * acc;
  if (smem > 48 * 1024) return CS_ERR_UNSUPPORTED;
#define CS_BIAS(T, A)                                                                       \
  bias_kernel<T, A><<<g, threads, smem, s>>>((const T*)query, qs_t, qs_h, (const A*)E, es_d, \
                                             es_p, d, npos, (const A*)positions, ps_h, ps_q,  \
                                             heads, nq, nk, (A*)out, os_h, os_q, status)
  switch (in_dtype) {
    case CS_F64: CS_BIAS(double, double); break;
    case CS_F32: CS_BIAS(float, float); break;
    case CS_F16: CS_BIAS(__half, float); break;
    case CS_BF16: CS_BIAS(__nv_bfloat16, float); break;
    default: return CS_ERR_INVALID;
  }
#undef CS_BIAS
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" CS_API int cs_cope_validate_path(const void* positions, int64_t ps_h, int64_t ps_q,
                                            const int64_t* qpos, const int64_t* kpos,
                                            const uint8_t* mask, int64_t ms_h, int64_t ms_q,
                                            int32_t heads, int64_t nq, int64_t nk, double atol,
                                            int32_t dtype, int32_t* status, void* stream) {
  CS_HOST_CHECK(heads > 0 && nq >= 0 && nk >= 0 && status);
  if (nq == 0 || nk == 0) return CS_OK;
  CS_HOST_CHECK(positions && qpos && kpos);
  const int threads = 256;
  auto s = as_stream(stream);
  int g = rows_grid((int64_t)heads * nq, threads / 32);
  if (dtype == CS_F64)
    validate_kernel<double><<<g, threads, 0, s>>>((const double*)positions, ps_h, ps_q, qpos,
                                                  kpos, mask, ms_h, ms_q, heads, nq, nk, atol,
                                                  status);
  else if (dtype == CS_F32)
    validate_kernel<float><<<g, threads, 0, s>>>((const float*)positions, ps_h, ps_q, qpos, kpos,
                                                 mask, ms_h, ms_q, heads, nq, nk, (float)atol,
                                                 status);
  else
    return CS_ERR_INVALID;
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" CS_API int cs_cope_chunk_offsets(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head, int32_t nq, int32_t hq,
    int32_t d, const int64_t* qpos, const int32_t* q_ord, const int32_t* q_seg, const void* k,
    int64_t k_stride_tok, int64_t k_stride_head, int32_t hkv, const int64_t* last_key,
    const int32_t* last_ord, const int32_t* seg_of_chunk, int32_t nfixed_chunks,
    const float* table, int64_t tb_stride_h, int64_t tb_stride_r, int64_t tb_stride_c,
    int32_t tb_rows, int32_t tb_cols, int32_t dtype, float* offsets, int64_t off_stride_h,
    int64_t off_stride_t, int32_t nseg, int32_t* status, void* stream) {
  CS_HOST_CHECK(nq >= 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && d > 0 && nseg > 0 &&
                nfixed_chunks >= 0 && tb_rows >= 0 && tb_cols >= 0);
  if (nq == 0) return CS_OK;
  CS_HOST_CHECK(q && qpos && q_ord && q_seg && offsets);
  CS_HOST_CHECK(nfixed_chunks == 0 || (k && last_key && last_ord && seg_of_chunk && table));
  const int threads = 256;
  int64_t blocks = ((int64_t)hq * nq * 32 + threads - 1) / threads;
  if (blocks > (int64_t)num_sms() * 16) blocks = (int64_t)num_sms() * 16;
  auto s = as_stream(stream);
  auto go = [&](auto tag) {
    using T = decltype(tag);
    chunk_offsets_kernel<T><<<(int)blocks, threads, 0, s>>>(
        static_cast<const T*>(q), q_stride_tok, q_stride_head, nq, hq, d, qpos, q_ord, q_seg,
        static_cast<const T*>(k), k_stride_tok, k_stride_head, hkv, last_key, last_ord,
        seg_of_chunk, nfixed_chunks, table, tb_stride_h, tb_stride_r, tb_stride_c, tb_rows,
        tb_cols, offsets, off_stride_h, off_stride_t, nseg, status);
  };
  switch (dtype) {
    case CS_F32: go(float{}); break;
    case CS_F16: go(__half{}); break;
    case CS_BF16: go(__nv_bfloat16{}); break;
    default: return CS_ERR_INVALID;
  }
  CS_LAUNCH_CHECK();
  return CS_OK;
}
