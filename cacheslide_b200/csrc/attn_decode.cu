// Split-key CoPE decode: a few query rows over a long paged context, for up
// to kMaxBatch requests per launch.
//
// The contextual position of key j is the sum of the gates of all newer keys,
// so a key split cannot finish on its own: it needs the gate total of every
// newer split.  On the tensor-core path (128-element 16-bit heads) one
// kernel does it in a single pass over the token records: each split
// publishes its gate totals and takes the count carried from the newer
// splits by a decoupled look-back, then finishes the interpolated bias, a
// partial softmax and its PV, and the last split of each (row, KV head) to
// finish merges the partials (decode_onepass_tc).  Other shapes run two
// CUDA-core phases and a combine kernel: phase 1 writes every split's logits
// and gate totals (reading K once), phase 2 gives each split the carried
// count and its partial softmax and PV (reading V once).  K and V cross HBM
// once; logits and partials stay in L2.  All requests of a batch share the
// launches.
//
// Modes: contextual positions, plain causal (the decode row of a CacheSlide
// request is a dynamic token: no canonical substitution, no association
// restriction).  Everything else reports CS_ERR_UNSUPPORTED.
#include <math.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace cs {

int validate_attn_params(const cs_attn_params* p);

namespace {

constexpr int kSplit = 128;  // keys per split == threads per CTA
constexpr int kMaxG = 8;     // query heads per KV head handled by one CTA
constexpr int kMaxD = 256;
constexpr int kMaxBatch = 8;

// one request of a batch (compact, so a batch fits the kernel parameters)
struct DecodeReq {
  const char* q;
  int64_t q_st, q_sh;
  const int64_t* qpos;
  const int64_t* kpos;
  const int64_t* slots;
  const char* k;
  const char* v;
  int64_t k_st, k_sh, v_st, v_sh;
  PagedView pv;
  const float* E;
  int64_t e_sd, e_sp;
  char* out;
  int64_t o_st, o_sh;
  int32_t* status;
  float* logits;  // [nq][hq][nk_pad]
  float* gsum;    // [nq][hq][nsplit]
  float* table;   // [nq][hq][npos]
  float* po;      // [nq][hq][nsplit][dv]
  float* pm;      // [nq][hq][nsplit]
  float* pl;      // [nq][hq][nsplit]
  int* cnt;       // [nq][hkv] finished splits (one-pass path)
  uint64_t* lb;   // [nq][hq][nsplit] split state words (one-pass path)
  uint32_t* tstat;  // [nq][hkv] q.E tables published (one-pass path)
  int nq, nk, nsplit, nk_pad, row0;
};

struct DecodeBatch {
  int count, hq, hkv, d, dv, npos, G, out_dtype, rows;
  float inv_scale;
  DecodeReq r[kMaxBatch];
};

__device__ __forceinline__ const DecodeReq& request_of(const DecodeBatch& b, int z, int64_t& i) {
  int k = 0;
  while (k + 1 < b.count && z >= b.r[k + 1].row0) ++k;
  i = z - b.r[k].row0;
  return b.r[k];
}

__device__ __forceinline__ int64_t causal_limit(const DecodeReq& r, int64_t qp) {
  if (r.kpos == nullptr) return qp + 1 < r.nk ? qp + 1 : r.nk;
  int64_t lo = 0, hi = r.nk;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (r.kpos[mid] <= qp) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// K (v false) or V row of key j, head g; `slot` is slots[j] on the paged path
template <typename T>
__device__ __forceinline__ const char* kv_row_at(const DecodeReq& r, int64_t slot, int64_t j,
                                                 int g, bool v, bool& ok, int d) {
  if (r.slots) {
    ok = r.pv.valid(slot);
    if (!ok) return nullptr;
    return r.pv.addr(slot, g, v ? r.pv.head_dim : 0);
  }
  ok = true;
  return (v ? r.v : r.k) +
         (j * (v ? r.v_st : r.k_st) + (int64_t)g * (v ? r.v_sh : r.k_sh)) * (int64_t)sizeof(T);
}

template <typename T>
__device__ __forceinline__ const char* kv_row(const DecodeReq& r, int64_t j, int g, bool v,
                                              bool& ok, int d) {
  return kv_row_at<T>(r, r.slots ? r.slots[j] : 0, j, g, v, ok, d);
}

// phase 1: logits of this split's keys for the G heads of KV head g, gate
// totals, and (split 0) the q.E tables
template <typename T>
__global__ void __launch_bounds__(kSplit) decode_phase1(const __grid_constant__ DecodeBatch b) {
  const int s = blockIdx.x, g = blockIdx.y;
  int64_t i;
  const DecodeReq& r = request_of(b, blockIdx.z, i);
  if (s >= r.nsplit) return;
  const int tid = threadIdx.x, G = b.G, d = b.d;
  __shared__ float qs[kMaxG * kMaxD];
  __shared__ float red[kMaxG][kSplit / 32];
  const int64_t qp = r.qpos[i];
  const int64_t nlim = causal_limit(r, qp);
  for (int e = tid; e < G * d; e += kSplit) {
    const int hh = e / d, x = e - hh * d;
    const T* qrow = reinterpret_cast<const T*>(
        r.q + (i * r.q_st + (int64_t)(g * G + hh) * r.q_sh) * (int64_t)sizeof(T));
    qs[e] = Elem<T>::to_f(qrow[x]);
  }
  __syncthreads();
  const int64_t j = (int64_t)s * kSplit + tid;
  float gate[kMaxG];
  int32_t bits = 0;
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) gate[hh] = 0.f;
  if (j < nlim) {
    bool ok;
    const char* kr = kv_row<T>(r, j, g, false, ok, d);
    if (!ok) {
      bits |= CS_ST_SLOT_RANGE;
    } else {
      float acc[kMaxG];
#pragma unroll
      for (int hh = 0; hh < kMaxG; ++hh) acc[hh] = 0.f;
      constexpr int V = 16 / sizeof(T);
      const int64_t se = r.slots ? r.pv.se : (int64_t)sizeof(T);
      if (se == (int64_t)sizeof(T) && (reinterpret_cast<uintptr_t>(kr) & 15) == 0 && d % V == 0) {
        for (int e0 = 0; e0 < d; e0 += V) {
          uint4 raw = *reinterpret_cast<const uint4*>(kr + e0 * sizeof(T));
          const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int u = 0; u < V; ++u) {
            const float kv = Elem<T>::to_f(x[u]);
#pragma unroll
            for (int hh = 0; hh < kMaxG; ++hh)
              if (hh < G) acc[hh] = fmaf(qs[hh * d + e0 + u], kv, acc[hh]);
          }
        }
      } else {
        for (int e = 0; e < d; ++e) {
          const float kv = Elem<T>::to_f(*reinterpret_cast<const T*>(kr + e * se));
#pragma unroll
          for (int hh = 0; hh < kMaxG; ++hh)
            if (hh < G) acc[hh] = fmaf(qs[hh * d + e], kv, acc[hh]);
        }
      }
#pragma unroll
      for (int hh = 0; hh < kMaxG; ++hh) {
        if (hh >= G) break;
        const float l = acc[hh] * b.inv_scale;
        if (!isfinite(l)) bits |= CS_ST_LOGIT_NONFINITE;
        r.logits[(i * b.hq + g * G + hh) * r.nk_pad + j] = l;
        gate[hh] = 1.f / (1.f + expf(-l));
      }
    }
  }
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    if (hh >= G) break;
    const float v = warp_sum(gate[hh]);
    if (lane == 0) red[hh][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float tot = 0.f;
    for (int w = kSplit / 32 - 1; w >= 0; --w) tot += red[tid][w];
    r.gsum[(i * b.hq + g * G + tid) * r.nsplit + s] = tot;
  }
  if (s == 0) {
    for (int e = tid; e < G * b.npos; e += kSplit) {
      const int hh = e / b.npos, pp = e - hh * b.npos;
      float t = 0.f;
      for (int x = 0; x < d; ++x) t = fmaf(qs[hh * d + x], r.E[x * r.e_sd + pp * r.e_sp], t);
      r.table[(i * b.hq + g * G + hh) * b.npos + pp] = t;
    }
  }
  bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
  if (lane == 0 && bits) report(r.status, bits);
}

// phase 2: carried count, reverse scan, bias, partial softmax and PV
template <typename T>
__global__ void __launch_bounds__(kSplit) decode_phase2(const __grid_constant__ DecodeBatch b) {
  const int s = blockIdx.x, g = blockIdx.y;
  int64_t i;
  const DecodeReq& r = request_of(b, blockIdx.z, i);
  if (s >= r.nsplit) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = b.G;
  const int npos = b.npos, dv = b.dv;
  extern __shared__ __align__(16) float dyn[];
  float* tab = dyn;             // [G][npos]
  float* wts = tab + G * npos;  // [G][kSplit]
  __shared__ float wtot[kMaxG][kSplit / 32];
  __shared__ float carry0[kMaxG];
  __shared__ float red[kMaxG][kSplit / 32];
  __shared__ float mmax[kMaxG];
  __shared__ const char* vrows[kSplit];
  const int64_t qp = r.qpos[i];
  const int64_t nlim = causal_limit(r, qp);
  const int64_t base = (int64_t)s * kSplit;
  const int64_t rowh0 = i * b.hq + (int64_t)g * G;
  if (base >= nlim) {  // split entirely in the future: empty partial
    if (tid < G) {
      r.pm[(rowh0 + tid) * r.nsplit + s] = -INFINITY;
      r.pl[(rowh0 + tid) * r.nsplit + s] = 0.f;
    }
    return;
  }
  const int last = (int)((nlim - 1) / kSplit);
  // count carried from the newer splits: a warp per head, lanes over splits
  for (int hh = warp; hh < G; hh += kSplit / 32) {
    float c = 0.f;
    for (int t = s + 1 + lane; t <= last; t += 32) c += r.gsum[(rowh0 + hh) * r.nsplit + t];
    c = warp_sum(c);
    if (lane == 0) carry0[hh] = c;
  }
  for (int e = tid; e < G * npos; e += kSplit) tab[e] = r.table[rowh0 * npos + e];
  const int64_t j = base + tid;
  const bool live = j < nlim;
  int32_t bits = 0;
  {
    bool ok = false;
    const char* vr = live ? kv_row<T>(r, j, g, true, ok, b.d) : nullptr;
    if (live && !ok) bits |= CS_ST_SLOT_RANGE;
    vrows[tid] = ok ? vr : nullptr;
  }
  float lg[kMaxG], gt[kMaxG];
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    lg[hh] = 0.f;
    gt[hh] = 0.f;
    if (hh < G && live) {
      lg[hh] = r.logits[(rowh0 + hh) * r.nk_pad + j];
      gt[hh] = 1.f / (1.f + expf(-lg[hh]));
    }
  }
  // reverse inclusive scan within each warp (lane l sums lanes l..31)
  float suf[kMaxG];
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    float v = gt[hh];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += t;
    }
    suf[hh] = v;
    if (lane == 0 && hh < G) wtot[hh][warp] = v;
  }
  __syncthreads();
  const float top = (float)(npos - 1);
  float score[kMaxG];
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    score[hh] = -INFINITY;
    if (hh >= G) continue;
    float c = carry0[hh];
    for (int w = kSplit / 32 - 1; w > warp; --w) c += wtot[hh][w];
    const float R = suf[hh] + c;
    const float pos = R < 0.f ? 0.f : (R > top ? top : R);
    const int lo = (int)floorf(pos);
    const int hi = lo + 1 < npos ? lo + 1 : npos - 1;
    const float f = pos - (float)lo;
    const float tlo = tab[hh * npos + lo];
    if (live) score[hh] = lg[hh] + (tlo + f * (tab[hh * npos + hi] - tlo));
  }
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    if (hh >= G) break;
    const float v = warp_max(score[hh]);
    if (lane == 0) red[hh][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float m = -INFINITY;
    for (int w = 0; w < kSplit / 32; ++w) m = fmaxf(m, red[tid][w]);
    mmax[tid] = m;
  }
  __syncthreads();
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    if (hh >= G) break;
    const float w = live ? expf(score[hh] - mmax[hh]) : 0.f;
    wts[hh * kSplit + tid] = w;
    const float v = warp_sum(w);
    __syncwarp();
    if (lane == 0) wtot[hh][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float l = 0.f;
    for (int w = 0; w < kSplit / 32; ++w) l += wtot[tid][w];
    r.pm[(rowh0 + tid) * r.nsplit + s] = mmax[tid];
    r.pl[(rowh0 + tid) * r.nsplit + s] = l;
  }
  // PV: thread <-> output dimension, keys broadcast from shared memory
  const int nkeys = (int)((nlim - base) < kSplit ? (nlim - base) : kSplit);
  const int64_t se = r.slots ? r.pv.se : (int64_t)sizeof(T);
  for (int x = tid; x < dv; x += kSplit) {
    float acc[kMaxG];
#pragma unroll
    for (int hh = 0; hh < kMaxG; ++hh) acc[hh] = 0.f;
    for (int kk = 0; kk < nkeys; ++kk) {
      const char* vr = vrows[kk];
      if (vr == nullptr) continue;
      const float vv = Elem<T>::to_f(*reinterpret_cast<const T*>(vr + x * se));
#pragma unroll
      for (int hh = 0; hh < kMaxG; ++hh)
        if (hh < G) acc[hh] = fmaf(wts[hh * kSplit + kk], vv, acc[hh]);
    }
#pragma unroll
    for (int hh = 0; hh < kMaxG; ++hh)
      if (hh < G) r.po[((rowh0 + hh) * r.nsplit + s) * dv + x] = acc[hh];
  }
  if (bits) report(r.status, bits);
}

// combine split partials: one CTA per (query row, head).  The split weights
// e^(m_s - M) are formed once per split, cooperatively, into shared memory
// (chunks of kCombChunk splits), and each thread owns up to two output
// dimensions.
constexpr int kCombThreads = 128;
constexpr int kCombChunk = 1024;
static_assert(kMaxD <= 2 * kCombThreads, "two output dimensions per thread");

__global__ void __launch_bounds__(kCombThreads) decode_combine(const __grid_constant__ DecodeBatch b) {
  int64_t i;
  const DecodeReq& r = request_of(b, blockIdx.x, i);
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nw = kCombThreads / 32;
  const int64_t rowh = i * b.hq + h;
  const int64_t nlim = causal_limit(r, r.qpos[i]);
  const int nsp = nlim > 0 ? (int)((nlim - 1) / kSplit) + 1 : 0;
  const float* pm = r.pm + rowh * r.nsplit;
  const float* pl = r.pl + rowh * r.nsplit;
  const float* po = r.po + rowh * r.nsplit * (int64_t)b.dv;
  __shared__ float wsp[kCombChunk];
  __shared__ float red[nw];
  float m = -INFINITY;
  for (int s = tid; s < nsp; s += kCombThreads) m = fmaxf(m, pm[s]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < nw; ++w) M = fmaxf(M, red[w]);
  const int x0 = tid, x1 = tid + kCombThreads;
  float l = 0.f, acc0 = 0.f, acc1 = 0.f;
  for (int c0 = 0; c0 < nsp; c0 += kCombChunk) {
    const int cn = nsp - c0 < kCombChunk ? nsp - c0 : kCombChunk;
    __syncthreads();  // previous chunk's weights consumed (and red[] read)
    for (int s = tid; s < cn; s += kCombThreads) {
      const float ms = pm[c0 + s];
      const float w = ms > -INFINITY ? expf(ms - M) : 0.f;
      wsp[s] = w;
      l = fmaf(w, pl[c0 + s], l);
    }
    __syncthreads();
    if (x0 < b.dv) {
#pragma unroll 8
      for (int s = 0; s < cn; ++s) acc0 = fmaf(wsp[s], po[(int64_t)(c0 + s) * b.dv + x0], acc0);
    }
    if (x1 < b.dv) {
#pragma unroll 8
      for (int s = 0; s < cn; ++s) acc1 = fmaf(wsp[s], po[(int64_t)(c0 + s) * b.dv + x1], acc1);
    }
  }
  l = warp_sum(l);
  __syncthreads();
  if (lane == 0) red[warp] = l;
  __syncthreads();
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < nw; ++w) L += red[w];
  const float inv = L > 0.f ? 1.f / L : 0.f;
  char* orow = r.out + (i * r.o_st + (int64_t)h * r.o_sh) * dtype_size(b.out_dtype);
  int32_t bits = 0;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int x = u ? x1 : x0;
    if (x >= b.dv) continue;
    const float val = (u ? acc1 : acc0) * inv;
    if (!isfinite(val)) bits |= CS_ST_LOGIT_NONFINITE;
    switch (b.out_dtype) {
      case CS_F32: reinterpret_cast<float*>(orow)[x] = val; break;
      case CS_F16: reinterpret_cast<__half*>(orow)[x] = __float2half_rn(val); break;
      default: reinterpret_cast<__nv_bfloat16*>(orow)[x] = __float2bfloat16_rn(val); break;
    }
  }
  if (bits) report(r.status, bits);
}

// ------------------------------------------------- tensor-core path: D = DV = 128
// 16-bit K/V rows with 16-byte aligned 128-element records.  A CTA takes one
// split (128 keys) of one KV head for one query row.  Thread t resolves the
// slot of key t; the warps copy the 128 key rows, later the 128 value rows
// (two 256-byte rows per warp instruction, cp.async), into one 128-byte
// swizzled tile, and two tcgen05.mma chains compute the split:
//   S[key][h]  = K_split (M = 128 keys) x q^T (N = 16 heads, G used)
//   O^T[x][h]  = V_split^T (M = 128 dims, MN-major) x P^T (N = 16)
// with the accumulator in 32 TMEM columns, read back one lane (key or
// dimension) per thread.  Gates use the hardware 2^x and reciprocal.
constexpr int kFastD = 128;
constexpr int kTcN = 16;            // MMA N: the G query heads, zero-padded
constexpr uint32_t kTcCols = 32;    // TMEM columns per CTA (allocation unit)
constexpr uint32_t kTileB = 32768;  // 128 rows x 256 B
constexpr uint32_t kSmallB = kTcN * 256;
constexpr size_t kOnepassSmem = 1024 + kTileB + kSmallB;  // the K / V tile and the q / P tile

// e^x = 2^(x log2 e) on the hardware 2^x (exp_fast(-inf) = 0)
__device__ __forceinline__ float exp_fast(float x) { return ex2(x * 1.4426950408889634f); }

__device__ __forceinline__ float fast_gate(float logit) {  // 1 / (1 + e^-logit)
  return rcp_approx(1.f + ex2(-logit * 1.4426950408889634f));
}

// rows 0..127 of the split (thread t resolved key t: `row`) into the swizzled
// tile at `dst`; warp w copies its keys 32w..32w+31 two at a time.  Rows of
// dead keys (null) are zero-filled from `dummy`, a valid global address.  The
// rows are read once: they go through L2 as first to be evicted, so the
// split partials written meanwhile stay there for the merge.
__device__ __forceinline__ void copy_split_rows(uint32_t dst, const char* row, const char* dummy) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t pol = l2_evict_first_policy();
#pragma unroll
  for (int it = 0; it < 16; ++it) {
    const int kl = 2 * it + (lane >> 4);
    const char* src = reinterpret_cast<const char*>(
        __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(row), kl));
    const int c = lane & 15;
    cp_async16_hint(dst + sw128(warp * 32 + kl, c, 128), src ? src + c * 16 : dummy,
                    src != nullptr, pol);
  }
}

// bounded wait of every thread on the CTA's MMA barrier (phase `parity`)
__device__ __forceinline__ bool wait_mma(uint32_t bar, uint32_t parity = 0) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

template <typename T>
constexpr int umma_fmt() {
  return std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
}

// q.E tables of the G heads of (row i, KV head g): T[h][p] = sum_x q[h][x]
// E[x][p] into r.table, q from the swizzled q tile `gQ`.  `part` is 16 KB of
// free shared memory (the vectorised path's per-group partials).  Called by
// all threads of the CTA.
template <typename T, int G>
__device__ void qe_table(const DecodeBatch& b, const DecodeReq& r, int64_t rowh0,
                         const unsigned char* gQ, float* part) {
  const int tid = threadIdx.x;
  const int npos = b.npos, p4 = npos / 4;
  const bool vec = r.e_sp == 1 && (npos & 3) == 0 && (r.e_sd & 3) == 0 && p4 <= kSplit &&
                   kSplit % p4 == 0 && kFastD % (kSplit / p4) == 0 &&
                   (reinterpret_cast<uintptr_t>(r.E) & 15) == 0;
  auto qx = [&](int hh, int x) {  // q[hh][x] from the swizzled q tile
    return Elem<T>::to_f(*reinterpret_cast<const T*>(gQ + sw128(hh, x >> 3, kTcN) + (x & 7) * 2));
  };
  if (vec) {
    // thread t: positions 4(t % p4) .. +3 over a group of dimensions (one
    // float4 load per dimension, all issued together); the groups'
    // partials meet in `part` as [ng][G][npos]
    const int ng = kSplit / p4, dpg = kFastD / ng;
    const int p0 = (tid % p4) * 4, grp = tid / p4, x0 = grp * dpg;
    float acc[G][4];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) acc[hh][0] = acc[hh][1] = acc[hh][2] = acc[hh][3] = 0.f;
    constexpr int UB = G >= 8 ? 4 : 8;  // float4 loads in flight (registers)
    for (int x = x0; x < x0 + dpg; x += UB) {
      float4 ev[UB];
#pragma unroll
      for (int u = 0; u < UB; ++u)
        ev[u] = x + u < x0 + dpg
                    ? __ldg(reinterpret_cast<const float4*>(r.E + (int64_t)(x + u) * r.e_sd + p0))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < UB; ++u) {
        if (x + u >= x0 + dpg) break;
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
          const float qv = qx(hh, x + u);
          acc[hh][0] = fmaf(qv, ev[u].x, acc[hh][0]);
          acc[hh][1] = fmaf(qv, ev[u].y, acc[hh][1]);
          acc[hh][2] = fmaf(qv, ev[u].z, acc[hh][2]);
          acc[hh][3] = fmaf(qv, ev[u].w, acc[hh][3]);
        }
      }
    }
#pragma unroll
    for (int hh = 0; hh < G; ++hh)
      *reinterpret_cast<float4*>(part + (grp * G + hh) * npos + p0) =
          make_float4(acc[hh][0], acc[hh][1], acc[hh][2], acc[hh][3]);
    __syncthreads();
    for (int e = tid; e < G * npos; e += kSplit) {
      float t = 0.f;
      for (int k = 0; k < ng; ++k) t += part[k * G * npos + e];
      r.table[rowh0 * npos + e] = t;
    }
  } else {  // a thread per (h, p)
    for (int e = tid; e < G * npos; e += kSplit) {
      const int hh = e / npos, pp = e - hh * npos;
      const float* ep = r.E + pp * r.e_sp;
      float t0 = 0.f, t1 = 0.f;
#pragma unroll 8
      for (int x = 0; x < kFastD; x += 2) {
        t0 = fmaf(qx(hh, x), ep[x * r.e_sd], t0);
        t1 = fmaf(qx(hh, x + 1), ep[(x + 1) * r.e_sd], t1);
      }
      r.table[rowh0 * npos + e] = t0 + t1;
    }
  }
}

// Merge the split partials of the G heads of (row i, KV head g) into the
// output rows in one online pass.  A warp takes up to four heads (G = 8: two
// warps share a split, four heads each) and every NS-th split, lane x
// dimensions 4x..4x+3; a batch of U = ROWS / 4 splits is loaded at once
// (ROWS float4 partial rows), and the warp's running maximum per head
// rescales its sums
// when a batch raises it.  The warps' (maximum, sum, accumulator) per head
// are then merged through `buf` (G * NS * 130 floats of shared memory).
// Partials written by other CTAs are read through L2.
template <int G, int ROWS>
__device__ void combine_heads(const DecodeBatch& b, const DecodeReq& r, int64_t i, int g,
                              int nsp, float* buf, int32_t& bits) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nw = kSplit / 32;
  constexpr int GH = G > 4 ? 4 : G;  // heads per warp
  constexpr int NS = nw / (G / GH);  // warps per head, each taking every NS-th split
  constexpr int U = ROWS / GH;       // splits per batch: ROWS partial rows in flight
  static_assert(G * NS * (kFastD + 2) * 4 <= (int)kTileB, "the merge buffer fits the V tile");
  const int h0 = (warp / NS) * GH, sw = warp % NS;
  const int64_t rowh0 = i * b.hq + (int64_t)g * G + h0;
  float m[GH], l[GH];
  float4 acc[GH];
#pragma unroll
  for (int hh = 0; hh < GH; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
    acc[hh] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int s0 = sw; s0 < nsp; s0 += NS * U) {
    float ms[U][GH], ls[U][GH];
    float4 o[U][GH];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int s = s0 + u * NS;
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
        const int64_t rs = (rowh0 + hh) * r.nsplit + s;
        if (s < nsp) {
          ms[u][hh] = __ldcg(r.pm + rs);
          ls[u][hh] = __ldcg(r.pl + rs);
          o[u][hh] = __ldcg(reinterpret_cast<const float4*>(r.po + rs * kFastD) + lane);
        } else {
          ms[u][hh] = -INFINITY;
          ls[u][hh] = 0.f;
          o[u][hh] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
#pragma unroll
    for (int hh = 0; hh < GH; ++hh) {
      float mb = m[hh];
#pragma unroll
      for (int u = 0; u < U; ++u) mb = fmaxf(mb, ms[u][hh]);
      if (mb > m[hh]) {  // uniform over the warp: its lanes read the same split maxima
        const float c = exp_fast(m[hh] - mb);  // 0 while nothing was accumulated
        acc[hh].x *= c;
        acc[hh].y *= c;
        acc[hh].z *= c;
        acc[hh].w *= c;
        l[hh] *= c;
        m[hh] = mb;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float w = ms[u][hh] > -INFINITY ? exp_fast(ms[u][hh] - m[hh]) : 0.f;
        acc[hh].x = fmaf(w, o[u][hh].x, acc[hh].x);
        acc[hh].y = fmaf(w, o[u][hh].y, acc[hh].y);
        acc[hh].z = fmaf(w, o[u][hh].z, acc[hh].z);
        acc[hh].w = fmaf(w, o[u][hh].w, acc[hh].w);
        l[hh] = fmaf(w, ls[u][hh], l[hh]);
      }
    }
  }
  // buf: [G][NS][128] accumulators, then [G][NS] maxima and [G][NS] sums
  float* wm = buf + G * NS * kFastD;
  float* wl = wm + G * NS;
#pragma unroll
  for (int hh = 0; hh < GH; ++hh) {
    const int e = (h0 + hh) * NS + sw;
    reinterpret_cast<float4*>(buf + e * kFastD)[lane] = acc[hh];
    if (lane == 0) {
      wm[e] = m[hh];
      wl[e] = l[hh];
    }
  }
  __syncthreads();
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NS; ++w) M = fmaxf(M, wm[hh * NS + w]);
    float L = 0.f, v = 0.f;
#pragma unroll
    for (int w = 0; w < NS; ++w) {
      const float mw = wm[hh * NS + w];
      const float c = mw > -INFINITY ? exp_fast(mw - M) : 0.f;
      L = fmaf(c, wl[hh * NS + w], L);
      v = fmaf(c, buf[(hh * NS + w) * kFastD + tid], v);
    }
    const float val = v * (L > 0.f ? 1.f / L : 0.f);
    if (!isfinite(val)) bits |= CS_ST_LOGIT_NONFINITE;
    char* orow = r.out + (i * r.o_st + (int64_t)(g * G + hh) * r.o_sh) * dtype_size(b.out_dtype);
    switch (b.out_dtype) {
      case CS_F32: reinterpret_cast<float*>(orow)[tid] = val; break;
      case CS_F16: reinterpret_cast<__half*>(orow)[tid] = __float2half_rn(val); break;
      default: reinterpret_cast<__nv_bfloat16*>(orow)[tid] = __float2bfloat16_rn(val); break;
    }
  }
}

// ----------------------------------------------------------- one-pass decode
// Split state words for the count carried between splits: bits 32..33 hold
// the state (0 not yet published, 1 the split's own gate total, 2 the total
// of this split and every newer one), bits 0..31 the float value.
constexpr uint64_t kAggregate = 1ull << 32, kInclusive = 2ull << 32;

__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Count carried into split s from splits s+1..last of one head (`words`:
// that head's state words), called by a whole warp: the look-back of a
// single-pass scan (Merrill and Garland, "Single-pass Parallel Prefix Scan
// with Decoupled Look-back", 2016).  Lane l reads split t0 + l; a window
// ends at its first split that holds an inclusive total, the splits before
// it add their own totals.  Splits past `last` have no keys (inclusive 0).
// Waits are bounded and record CS_ST_TIMEOUT on expiry.
__device__ float look_back(const uint64_t* words, int s, int last, int32_t& bits) {
  const int lane = threadIdx.x & 31;
  float carry = 0.f;
  for (int t0 = s + 1; t0 <= last; t0 += 32) {
    const int t = t0 + lane;
    uint64_t w = t <= last ? ld_relaxed_u64(words + t) : kInclusive;
    const long long c0 = clock64();
    while (__any_sync(0xffffffffu, (w >> 32) == 0)) {
      if ((w >> 32) == 0) {
        w = ld_relaxed_u64(words + t);
        if ((w >> 32) == 0 && clock64() - c0 > kWaitCycles) {
          bits |= CS_ST_TIMEOUT;
          w = kInclusive;
        }
      }
    }
    const unsigned incl = __ballot_sync(0xffffffffu, (w >> 32) == 2);
    const int first = incl ? __ffs(incl) - 1 : 32;
    carry += warp_sum(lane <= first ? __uint_as_float((uint32_t)w) : 0.f);
    if (incl) break;
  }
  return carry;
}

// Sum (or maximum) over the warp of G values per lane, all G at once: a
// transposed butterfly halves the values each lane holds per exchange (lanes
// with the offset bit set keep the upper half), then reduces the one left,
// (G - 1) + (5 - log2 G) shuffles in all instead of 5 G.  Every lane gets the
// total of value `head`; the lanes with lane % (32 / G) == 0 hold heads
// 0..G-1 once each.
template <int G, bool MAX>
__device__ __forceinline__ float warp_reduce_g(const float (&v)[G], int& head) {
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "G is a power of two up to 8");
  const int lane = threadIdx.x & 31;
  float w[G];
#pragma unroll
  for (int j = 0; j < G; ++j) w[j] = v[j];
  head = 0;
  int o = 16;
#pragma unroll
  for (int W = G; W > 1; W >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < W / 2; ++j) {
      const float send = up ? w[j] : w[j + W / 2];
      const float keep = up ? w[j + W / 2] : w[j];
      const float got = __shfl_xor_sync(0xffffffffu, send, o);
      w[j] = MAX ? fmaxf(keep, got) : keep + got;
    }
    if (up) head += W / 2;
  }
#pragma unroll
  for (; o >= 1; o >>= 1) {
    const float got = __shfl_xor_sync(0xffffffffu, w[0], o);
    w[0] = MAX ? fmaxf(w[0], got) : w[0] + got;
  }
  return w[0];
}

// Zeroes the one-pass flags (the first n16 16-byte words of the batch
// workspace) and lets the dependent decode grid start at once.  When the
// caller allows it (CS_LAUNCH_OVERLAP_PREV) it is itself launched as a
// programmatic dependent of the preceding grid (which starts it early only
// if that grid signals so, as the paged-cache scatter does) and waits for
// that grid before it exits, so its completion implies the preceding grid's:
// the decode grid's griddepcontrol.wait covers both.  Its stores come before
// that wait, so a preceding grid that uses the same workspace (an earlier
// decode) must not signal early: decode_onepass_tc never executes
// griddepcontrol.launch_dependents, and must not, or the flags of a decode
// still running could be cleared under it.
__global__ void __launch_bounds__(256) decode_zero_flags(uint4* p, int64_t n16) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x; e < n16; e += (int64_t)gridDim.x * 256)
    p[e] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// One-pass decode for the tensor-core shapes: a CTA takes one 128-key split
// of one (row, KV head).  Its K rows land in the tile, S = K q^T runs on the
// tensor cores and stays in registers, and the V rows are then copied into
// the same tile while the CTA publishes the split's gate totals, takes the
// count carried from the newer splits by a look-back over their state
// words, and computes the interpolated bias and a partial softmax; O^T =
// V^T P^T follows, and the last split of (row, KV head) to finish merges the
// partials.  One 32 KB tile keeps five CTAs on an SM.
//
// Block k takes split nsplit - 1 - k / groups of group k % groups, so the
// newest splits of every group come first and a CTA only waits on blocks of
// lower index, which the hardware dispatches no later than its own (the
// order single-pass scans rely on); every wait is bounded all the same.
// The group's newest split with visible keys computes the q.E tables and
// publishes them with a flag; a split whose carried count already reaches
// the last position for every head needs only T[h][npos - 1], which it
// computes itself from the last column of E.  The state words, table flags
// and arrival counters are zeroed by decode_zero_flags, the grid before
// this one; this grid is its programmatic dependent: a CTA reads the slots,
// query position and E column at once, and waits (griddepcontrol.wait, which
// also covers the grid before the zeroing one) before it reads any K / V row
// or flag or writes any output.
template <typename T, int G>
__global__ void __launch_bounds__(kSplit, 5) decode_onepass_tc(const __grid_constant__ DecodeBatch b) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ int last_split;
  __shared__ float wtot[G][kSplit / 32];
  __shared__ float red[G][kSplit / 32];
  __shared__ float tsp[G][kSplit / 32];
  __shared__ float carry0[G];
  const int groups = b.rows * b.hkv;
  const int si = (int)(blockIdx.x / groups), grp = (int)(blockIdx.x - si * groups);
  const int g = grp % b.hkv;
  int64_t i;
  const DecodeReq& r = request_of(b, grp / b.hkv, i);
  if (si >= r.nsplit) return;
  const int s = r.nsplit - 1 - si;
  const int npos = b.npos;
  const int64_t j = (int64_t)s * kSplit + tid;
  // the key's slot, loaded beside the query position it is masked by
  const int64_t slot = r.slots != nullptr && j < r.nk ? __ldg(r.slots + j) : 0;
  const int64_t qp = r.qpos[i];
  const int64_t nlim = causal_limit(r, qp);
  const int64_t base = (int64_t)s * kSplit;
  const int64_t rowh0 = i * b.hq + (int64_t)g * G;
  const int64_t gl = i * b.hkv + g;
  if (base >= nlim) {  // split entirely in the future: nothing to publish
    if (s == 0) {      // no visible key at all: zero output rows
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int e = tid; e < G * kFastD; e += kSplit) {
        char* orow = r.out + (i * r.o_st + (int64_t)(g * G + e / kFastD) * r.o_sh) *
                                 dtype_size(b.out_dtype);
        const int x = e % kFastD;
        switch (b.out_dtype) {
          case CS_F32: reinterpret_cast<float*>(orow)[x] = 0.f; break;
          case CS_F16: reinterpret_cast<__half*>(orow)[x] = __float2half_rn(0.f); break;
          default: reinterpret_cast<__nv_bfloat16*>(orow)[x] = __float2bfloat16_rn(0.f); break;
        }
      }
    }
    return;
  }
  const int last = (int)((nlim - 1) / kSplit);  // newest split with visible keys
  const uint32_t sraw = smem_u32(dsm);
  const uint32_t sT = (sraw + 1023u) & ~1023u, sQ = sT + kTileB;  // K, then V; q, then P
  unsigned char* gQ = dsm + (sQ - sraw);
  float* tile = reinterpret_cast<float*>(dsm + (sT - sraw));
  const uint32_t mb = smem_u32(&bar);
  if (warp == 0) tmem_alloc(smem_u32(&tslot), kTcCols);
  if (tid == 0) {
    mbar_init(mb, 1);
    mbar_init_fence();
  }
  const bool live = j < nlim;
  int32_t bits = 0;
  // E[tid][npos - 1], for T[h][npos - 1] of saturated splits
  const float elast = __ldg(r.E + (int64_t)tid * r.e_sd + (int64_t)(npos - 1) * r.e_sp);
  const char* krow = nullptr;
  const char* vrow = nullptr;
  if (live) {
    bool okk, okv;
    krow = kv_row_at<T>(r, slot, j, g, false, okk, kFastD);
    vrow = kv_row_at<T>(r, slot, j, g, true, okv, kFastD);
    if (!okk || !okv) bits |= CS_ST_SLOT_RANGE;
  }
  const char* q0 = r.q + (i * r.q_st + (int64_t)g * G * r.q_sh) * (int64_t)sizeof(T);
  // the preceding grids (flag zeroing, and the one before it, e.g. the write
  // of the newest rows) are complete and visible from here on
  asm volatile("griddepcontrol.wait;" ::: "memory");
  copy_split_rows(sT, krow, q0);
  for (int e = tid; e < kTcN * 16; e += kSplit) {  // q rows (heads), zero beyond G
    const int hh = e >> 4, c = e & 15;
    const char* src = q0 + (int64_t)hh * r.q_sh * (int64_t)sizeof(T) + c * 16;
    cp_async16(sQ + sw128(hh, c, kTcN), hh < G ? src : q0, hh < G);
  }
  cp_async_wait_all();
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (tid == 0) {
    const uint32_t idesc = umma_idesc(128, kTcN, umma_fmt<T>(), 0, 0);
#pragma unroll
    for (int kk = 0; kk < kFastD / 16; ++kk) {
      const uint32_t ko = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
      const uint32_t qo = (kk >> 2) * (kTcN * 128) + (kk & 3) * 32;
      tc_mma(tmem, umma_desc(sT + ko, 16, 1024), umma_desc(sQ + qo, 16, 1024), idesc,
             kk ? 1u : 0u);
    }
    tc_commit(mb);
  }
  // partial sums of T[h][npos - 1] = q[h] . E[:, npos - 1] while S runs
  {
    float pq[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh)
      pq[hh] = elast * Elem<T>::to_f(*reinterpret_cast<const T*>(
                           gQ + sw128(hh, tid >> 3, kTcN) + (tid & 7) * 2));
    int hw;
    const float v = warp_reduce_g<G, false>(pq, hw);
    if ((lane & (32 / G - 1)) == 0) tsp[hw][warp] = v;
  }
  const bool done1 = wait_mma(mb, 0);  // S complete: the tile's K rows are read
  tc_fence_after();
  uint32_t acc[16];
  CS_TMEM_LD16(tmem + ((uint32_t)(warp * 32) << 16), acc);
  tmem_wait_ld();
  if (!done1) bits |= CS_ST_TIMEOUT;
  // V rows into the tile, in flight until the PV product (the newest split
  // first uses the tile for its q.E tables, after publishing its totals)
  if (s != last) copy_split_rows(sT, vrow, q0);
  // logits, gates and the reverse scan of the gates within each warp
  float lg[G], suf[G];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    float l = 0.f, v = 0.f;
    if (live && done1) {
      l = __uint_as_float(acc[hh]) * b.inv_scale;
      if (!isfinite(l)) bits |= CS_ST_LOGIT_NONFINITE;
      v = fast_gate(l);
    }
    lg[hh] = l;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += t;
    }
    suf[hh] = v;
    if (lane == 0) wtot[hh][warp] = v;
  }
  tc_fence_before();
  __syncthreads();
  // publish the split's gate totals (warp h, head h), take the per-warp
  // maxima of the logits while the newer splits publish theirs, then look
  // back for the carried count (a warp per head)
  if (s < last && lane == 0) {
    for (int hh = warp; hh < G; hh += kSplit / 32) {
      float agg = 0.f;
#pragma unroll
      for (int w = 0; w < kSplit / 32; ++w) agg += wtot[hh][w];
      st_relaxed_u64(r.lb + (rowh0 + hh) * r.nsplit + s, kAggregate | __float_as_uint(agg));
    }
  }
  {
    float lv[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) lv[hh] = live ? lg[hh] : -INFINITY;
    int hw;
    const float v = warp_reduce_g<G, true>(lv, hw);
    if ((lane & (32 / G - 1)) == 0) red[hw][warp] = v;
  }
  for (int hh = warp; hh < G; hh += kSplit / 32) {
    float agg = 0.f;
#pragma unroll
    for (int w = 0; w < kSplit / 32; ++w) agg += wtot[hh][w];
    uint64_t* words = r.lb + (rowh0 + hh) * r.nsplit;
    const float carry = s < last ? look_back(words, s, last, bits) : 0.f;
    if (lane == 0) {
      st_relaxed_u64(words + s, kInclusive | __float_as_uint(carry + agg));
      carry0[hh] = carry;
    }
  }
  if (s == last) {  // q.E tables, with the tile as scratch before V arrives
    qe_table<T, G>(b, r, rowh0, gQ, tile);
    __threadfence();
    __syncthreads();
    copy_split_rows(sT, vrow, q0);
  }
  __syncthreads();
  // the q.E tables are read by the splits whose counts stay below the last
  // position for some head
  const float top = (float)(npos - 1);
  bool saturated = s != last;
#pragma unroll
  for (int hh = 0; hh < G; ++hh) saturated = saturated && carry0[hh] >= top;
  if (!saturated) {
    if (tid == 0) {
      if (s == last) {
        st_release_u32(r.tstat + gl, 1u);
      } else {
        const long long c0 = clock64();
        while (ld_acquire_u32(r.tstat + gl) == 0u) {
          if (clock64() - c0 > kWaitCycles) {
            bits |= CS_ST_TIMEOUT;
            break;
          }
        }
      }
    }
    __syncthreads();
  }
  // counts, bias and the split's softmax maximum
  float score[G], m[G];
  if (saturated) {
    // every count >= carry >= npos - 1: the last table entry, the same for
    // all keys of the head, so the maximum is the logits' maximum plus it
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float tb = 0.f, mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kSplit / 32; ++w) {
        tb += tsp[hh][w];
        mx = fmaxf(mx, red[hh][w]);
      }
      score[hh] = lg[hh] + tb;  // every key of a saturated split is visible
      m[hh] = mx + tb;
    }
  } else {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float c = carry0[hh];
      for (int w = kSplit / 32 - 1; w > warp; --w) c += wtot[hh][w];
      const float R = suf[hh] + c;
      const float pos = R < 0.f ? 0.f : (R > top ? top : R);
      const int lo = (int)floorf(pos);
      const int hi = lo + 1 < npos ? lo + 1 : npos - 1;
      const float f = pos - (float)lo;
      const float* trow = r.table + (rowh0 + hh) * npos;
      const float tlo = __ldcg(trow + lo);
      score[hh] = live ? lg[hh] + (tlo + f * (__ldcg(trow + hi) - tlo)) : -INFINITY;
      const float v = warp_max(score[hh]);
      if (lane == 0) red[hh][warp] = v;  // the logit maxima are not read on this path
    }
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      m[hh] = -INFINITY;
#pragma unroll
      for (int w = 0; w < kSplit / 32; ++w) m[hh] = fmaxf(m[hh], red[hh][w]);
    }
  }
  // P^T over the q tile (free after S; its rows beyond G stay zero)
  float pw[G];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    const T wq = Elem<T>::from_f(live ? exp_fast(score[hh] - m[hh]) : 0.f);
    *reinterpret_cast<T*>(gQ + sw128(hh, tid >> 3, kTcN) + (tid & 7) * 2) = wq;
    pw[hh] = Elem<T>::to_f(wq);
  }
  cp_async_wait_all();  // V
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    const uint32_t idesc = umma_idesc(128, kTcN, umma_fmt<T>(), 1, 0);  // A = V^T, MN-major
#pragma unroll
    for (int kk = 0; kk < kSplit / 16; ++kk) {
      const uint32_t po = (kk >> 2) * (kTcN * 128) + (kk & 3) * 32;
      tc_mma(tmem, umma_desc(sT + kk * 2048, 16384, 1024), umma_desc(sQ + po, 16, 1024), idesc,
             kk ? 1u : 0u);
    }
    tc_commit(mb);
  }
  // row sums of the rounded weights while the product runs
  {
    int hw;
    const float v = warp_reduce_g<G, false>(pw, hw);
    if ((lane & (32 / G - 1)) == 0) wtot[hw][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float l = 0.f, mt = m[0];
    for (int w = 0; w < kSplit / 32; ++w) l += wtot[tid][w];
#pragma unroll
    for (int hh = 1; hh < G; ++hh)
      if (hh == tid) mt = m[hh];
    r.pm[(rowh0 + tid) * r.nsplit + s] = mt;
    r.pl[(rowh0 + tid) * r.nsplit + s] = l;
  }
  const bool done2 = wait_mma(mb, 1);
  tc_fence_after();
  CS_TMEM_LD16(tmem + ((uint32_t)(warp * 32) << 16), acc);
  tmem_wait_ld();
  if (!done2) bits |= CS_ST_TIMEOUT;
#pragma unroll
  for (int hh = 0; hh < G; ++hh)
    r.po[((rowh0 + hh) * r.nsplit + s) * kFastD + tid] = __uint_as_float(acc[hh]);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    if (!done2) wait_mma(mb, 1);  // drain before the columns are released
    tmem_dealloc(tmem, kTcCols);
  }
  if (tid == 0) {
    // the CTA's partial (ordered before this thread by the barrier) is
    // visible before its arrival is counted
    __threadfence();
    last_split = atomicAdd(&r.cnt[gl], 1) == last;
    if (last_split) __threadfence();
  }
  __syncthreads();
  if (last_split)  // the tile is idle: this CTA's product was read back above
    combine_heads<G, 8>(b, r, i, g, last + 1, tile, bits);
  bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
  if (lane == 0 && bits) report(r.status, bits);
}

// whether the tensor-core kernels take this request: 128-element 16-bit
// records whose rows start on 16-byte boundaries (cp.async), G in {1,2,4,8}
bool fast_decode_ok(const cs_attn_params* p) {
  if (p->d != kFastD || p->dv != kFastD) return false;
  const int G = p->hq / p->hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return false;
  const int64_t es = 2;
  auto al16 = [](int64_t x) { return (x % 16) == 0; };
  if (!al16(reinterpret_cast<uintptr_t>(p->q)) || !al16(p->q_stride_tok * es) ||
      !al16(p->q_stride_head * es))
    return false;
  if (p->kv_slots) {
    const PagedView pv = PagedView::make(p->paged);
    if (pv.se != es || !al16(reinterpret_cast<uintptr_t>(pv.cache)) || !al16(pv.sb) ||
        !al16(pv.sh) || !al16(pv.so) || !al16(pv.head_dim * es))
      return false;
    if (pv.side_capacity > 0 &&
        (pv.sse != es || !al16(reinterpret_cast<uintptr_t>(pv.side_k)) ||
         !al16(reinterpret_cast<uintptr_t>(pv.side_v)) || !al16(pv.ssr) || !al16(pv.ssh)))
      return false;
  } else if (!al16(reinterpret_cast<uintptr_t>(p->k)) || !al16(reinterpret_cast<uintptr_t>(p->v)) ||
             !al16(p->k_stride_tok * es) || !al16(p->k_stride_head * es) ||
             !al16(p->v_stride_tok * es) || !al16(p->v_stride_head * es)) {
    return false;
  }
  return true;
}

bool decode_supported(const cs_attn_params* p) {
  if (p->nq_dev != nullptr) return false;  // a device row count is a prefill option
  if (p->in_dtype != CS_BF16 && p->in_dtype != CS_F16) return false;
  if (p->out_dtype != CS_BF16 && p->out_dtype != CS_F16 && p->out_dtype != CS_F32) return false;
  if (p->pos_mode != CS_POS_CONTEXTUAL) return false;
  if (p->gate_mask || p->vis_mask || p->q_selected || p->out_positions || p->positions_only ||
      p->strict)
    return false;
  const int G = p->hq / p->hkv;
  if (G > kMaxG || p->d > kMaxD || p->dv > kMaxD) return false;
  if (p->npos > 1024) return false;
  return true;
}

// Workspace of one request, in floats.  The first `zero` floats are zeroed
// before each one-pass launch (split state words, table flags, arrival
// counters); a batch places the zeroed parts of all its requests first, then
// their data parts.
struct Layout {
  int nsplit, nk_pad;
  int64_t lb, tstat, cnt, zero;                   // offsets in the zeroed part
  int64_t logits, gsum, table, po, pm, pl, data;  // offsets in the data part
  int64_t total;
};

Layout layout_of(const cs_attn_params* p) {
  Layout L;
  L.nsplit = (p->nk + kSplit - 1) / kSplit;
  L.nk_pad = L.nsplit * kSplit;
  const int64_t rows = (int64_t)p->nq * p->hq;
  int64_t off = 0;
  auto take = [&](int64_t n) {
    const int64_t o = off;
    off += (n + 63) / 64 * 64;  // 256-byte aligned sections
    return o;
  };
  L.lb = take(rows * L.nsplit * 2);  // 64-bit words
  L.tstat = take((int64_t)p->nq * p->hkv);
  L.cnt = take((int64_t)p->nq * p->hkv);
  L.zero = off;
  off = 0;
  L.logits = take(rows * L.nk_pad);
  L.gsum = take(rows * L.nsplit);
  L.table = take(rows * p->npos);
  L.po = take(rows * L.nsplit * p->dv);
  L.pm = take(rows * L.nsplit);
  L.pl = take(rows * L.nsplit);
  L.data = off;
  L.total = L.zero + L.data;
  return L;
}

bool same_shape(const cs_attn_params* a, const cs_attn_params* b) {
  return a->hq == b->hq && a->hkv == b->hkv && a->d == b->d && a->dv == b->dv &&
         a->npos == b->npos && a->in_dtype == b->in_dtype && a->out_dtype == b->out_dtype &&
         a->scale == b->scale;
}

void fill_request(DecodeReq& q, const cs_attn_params* p, float* zs, float* ws, const Layout& L,
                  int row0) {
  q.q = static_cast<const char*>(p->q);
  q.q_st = p->q_stride_tok;
  q.q_sh = p->q_stride_head;
  q.qpos = p->qpos;
  q.kpos = p->kpos;
  q.slots = p->kv_slots;
  q.k = static_cast<const char*>(p->k);
  q.v = static_cast<const char*>(p->v);
  q.k_st = p->k_stride_tok;
  q.k_sh = p->k_stride_head;
  q.v_st = p->v_stride_tok;
  q.v_sh = p->v_stride_head;
  q.pv = p->kv_slots ? PagedView::make(p->paged) : PagedView{};
  q.E = static_cast<const float*>(p->E);
  q.e_sd = p->e_stride_d;
  q.e_sp = p->e_stride_p;
  q.out = static_cast<char*>(p->out);
  q.o_st = p->o_stride_tok;
  q.o_sh = p->o_stride_head;
  q.status = p->status;
  q.logits = ws + L.logits;
  q.gsum = ws + L.gsum;
  q.table = ws + L.table;
  q.po = ws + L.po;
  q.pm = ws + L.pm;
  q.pl = ws + L.pl;
  q.cnt = reinterpret_cast<int*>(zs + L.cnt);
  q.lb = reinterpret_cast<uint64_t*>(zs + L.lb);
  q.tstat = reinterpret_cast<uint32_t*>(zs + L.tstat);
  q.nq = p->nq;
  q.nk = p->nk;
  q.nsplit = L.nsplit;
  q.nk_pad = L.nk_pad;
  q.row0 = row0;
}

// Raises the dynamic shared memory limit of `kern` on the current device,
// once per device and kernel.  The cache is keyed by the kernel's template
// arguments (Tag), not by the function pointer type: every instantiation of
// a kernel template shares that type.
template <typename T, int G>
struct OnepassTag {};
template <typename Tag, typename K>
bool smem_configured(K kern, int bytes) {
  static std::atomic<uint64_t> done{0};  // bit d: device d configured
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return false;
  done.fetch_or(bit, std::memory_order_release);
  return true;
}

int launch_batch(const cs_attn_params* ps, int count, char* workspace, cudaStream_t stream) {
  DecodeBatch b{};
  const cs_attn_params* p0 = &ps[0];
  b.count = 0;
  b.hq = p0->hq;
  b.hkv = p0->hkv;
  b.d = p0->d;
  b.dv = p0->dv;
  b.npos = p0->npos;
  b.G = p0->hq / p0->hkv;
  b.out_dtype = p0->out_dtype;
  b.inv_scale = (float)(1.0 / p0->scale);
  Layout L[kMaxBatch];
  int64_t zero = 0, data = 0;  // floats
  for (int k = 0; k < count; ++k) {
    L[k] = layout_of(&ps[k]);
    zero += L[k].zero;
  }
  float* ws = reinterpret_cast<float*>(workspace);
  int rows = 0, nsplit_max = 0;
  int64_t zoff = 0;
  for (int k = 0; k < count; ++k) {
    const cs_attn_params* p = &ps[k];
    float* zs = ws + zoff;
    float* ds = ws + zero + data;
    zoff += L[k].zero;
    data += L[k].data;
    if (p->nq == 0) continue;
    fill_request(b.r[b.count], p, zs, ds, L[k], rows);
    rows += p->nq;
    nsplit_max = L[k].nsplit > nsplit_max ? L[k].nsplit : nsplit_max;
    ++b.count;
  }
  if (b.count == 0) return CS_OK;
  b.rows = rows;
  bool fast = true;
  for (int k = 0; k < count; ++k) fast = fast && (ps[k].nq == 0 || fast_decode_ok(&ps[k]));
  if (fast) {
    const int64_t n16 = zero / 4;  // zero is a multiple of 64 floats
    // the decode grid is always a programmatic dependent of the zeroing
    // grid (which writes only the flags).  The zeroing grid is one of the
    // preceding grid only when the caller says that grid writes none of the
    // inputs the decode CTAs read before their griddepcontrol.wait (slots,
    // query positions, E), e.g. cs_slide_scatter of the newest records;
    // otherwise it starts in plain stream order, after that grid completes.
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t zcfg{};
    zcfg.gridDim = dim3((unsigned)std::min<int64_t>((n16 + 255) / 256, 148));
    zcfg.blockDim = dim3(256);
    zcfg.stream = stream;
    zcfg.attrs = pdl;
    zcfg.numAttrs = (p0->launch_flags & CS_LAUNCH_OVERLAP_PREV) ? 1 : 0;
    if (cudaLaunchKernelEx(&zcfg, decode_zero_flags, reinterpret_cast<uint4*>(workspace), n16) !=
        cudaSuccess)
      return CS_ERR_CUDA;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((int64_t)rows * b.hkv * nsplit_max));
    cfg.blockDim = dim3(kSplit);
    cfg.dynamicSmemBytes = kOnepassSmem;
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    int rc = CS_OK;
    auto go = [&](auto tag, auto gtag) {
      using T = decltype(tag);
      constexpr int G = decltype(gtag)::value;
      auto kern = decode_onepass_tc<T, G>;
      if (!smem_configured<OnepassTag<T, G>>(kern, (int)kOnepassSmem)) {
        rc = CS_ERR_CUDA;
        return;
      }
      if (cudaLaunchKernelEx(&cfg, kern, b) != cudaSuccess) rc = CS_ERR_CUDA;
    };
    auto by_g = [&](auto tag) {
      switch (b.G) {
        case 1: go(tag, std::integral_constant<int, 1>{}); break;
        case 2: go(tag, std::integral_constant<int, 2>{}); break;
        case 4: go(tag, std::integral_constant<int, 4>{}); break;
        default: go(tag, std::integral_constant<int, 8>{}); break;
      }
    };
    if (p0->in_dtype == CS_BF16) by_g(__nv_bfloat16{});
    else by_g(__half{});
    if (rc != CS_OK) return rc;
  } else {
    const dim3 grid(nsplit_max, b.hkv, rows);
    const size_t smem2 = (size_t)(b.G * b.npos + b.G * kSplit) * sizeof(float);
    if (smem2 > 48 * 1024) return CS_ERR_UNSUPPORTED;
    if (p0->in_dtype == CS_BF16) {
      decode_phase1<__nv_bfloat16><<<grid, kSplit, 0, stream>>>(b);
      decode_phase2<__nv_bfloat16><<<grid, kSplit, smem2, stream>>>(b);
    } else {
      decode_phase1<__half><<<grid, kSplit, 0, stream>>>(b);
      decode_phase2<__half><<<grid, kSplit, smem2, stream>>>(b);
    }
    decode_combine<<<dim3(rows, b.hq), kCombThreads, 0, stream>>>(b);
  }
  CS_LAUNCH_CHECK();
  return CS_OK;
}

int check_batch(const cs_attn_params* ps, int count) {
  if (!ps || count < 1) return CS_ERR_INVALID;
  for (int k = 0; k < count; ++k) {
    const int rc = validate_attn_params(&ps[k]);
    if (rc != CS_OK) return rc;
    if (!decode_supported(&ps[k]) || !same_shape(&ps[0], &ps[k])) return CS_ERR_UNSUPPORTED;
  }
  return CS_OK;
}

}  // namespace

// shared with the no-allocation variant
int64_t decode_workspace_bytes(const cs_attn_params* p) {
  if (validate_attn_params(p) != CS_OK || !decode_supported(p)) return 0;
  return layout_of(p).total * (int64_t)sizeof(float);
}

int launch_decode(const cs_attn_params* p, void* workspace, cudaStream_t stream) {
  const int rc = check_batch(p, 1);
  if (rc != CS_OK) return rc;
  if (p->nq == 0) return CS_OK;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255)) return CS_ERR_INVALID;
  return launch_batch(p, 1, static_cast<char*>(workspace), stream);
}

}  // namespace cs

using namespace cs;

extern "C" int64_t cs_cope_attn_decode_workspace(const cs_attn_params* p) {
  return decode_workspace_bytes(p);
}

extern "C" int cs_cope_attn_decode(const cs_attn_params* p, void* workspace, void* stream) {
  return launch_decode(p, workspace, as_stream(stream));
}

extern "C" int64_t cs_cope_attn_decode_batch_workspace(const cs_attn_params* params,
                                                       int32_t count) {
  if (check_batch(params, count) != CS_OK) return 0;
  int64_t total = 0;
  for (int k = 0; k < count; ++k) total += layout_of(&params[k]).total * (int64_t)sizeof(float);
  return total;
}

extern "C" int cs_cope_attn_decode_batch(const cs_attn_params* params, int32_t count,
                                         void* workspace, void* stream) {
  const int rc = check_batch(params, count);
  if (rc != CS_OK) return rc;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255)) return CS_ERR_INVALID;
  char* ws = static_cast<char*>(workspace);
  for (int first = 0; first < count; first += kMaxBatch) {
    const int n = count - first < kMaxBatch ? count - first : kMaxBatch;
    const int r = launch_batch(params + first, n, ws, as_stream(stream));
    if (r != CS_OK) return r;
    for (int k = first; k < first + n; ++k) ws += layout_of(&params[k]).total * sizeof(float);
  }
  return CS_OK;
}
