// Split-key CoPE decode: a few query rows over a long paged context.
//
// The contextual position of key j is the sum of the gates of all newer keys,
// so a key split cannot finish on its own: phase 1 computes every split's
// logits and gate totals (reading K once), phase 2 gives each split the count
// carried from the newer splits, finishes the reverse scan, the interpolated
// bias and a partial softmax with its PV (reading V once), and a combine
// kernel merges the split partials.  K and V each cross HBM once; the logits
// and partials (a few hundred KB) stay in L2.
//
// Modes: contextual positions, plain causal (the decode row of a CacheSlide
// request is a dynamic token: no canonical substitution, no association
// restriction).  Everything else reports CS_ERR_UNSUPPORTED.
#include <math.h>

#include "common.cuh"

namespace cs {

int validate_attn_params(const cs_attn_params* p);

namespace {

constexpr int kSplit = 128;    // keys per split == threads per CTA
constexpr int kMaxG = 8;       // query heads per KV head handled by one CTA
constexpr int kMaxD = 256;

struct DecodeArgs {
  cs_attn_params p;
  PagedView pv;
  int G, nsplit, nk_pad;
  // workspace sections (floats), per query row
  float* logits;  // [nq][hq][nk_pad]
  float* gsum;    // [nq][hq][nsplit]
  float* table;   // [nq][hq][npos]
  float* po;      // [nq][hq][nsplit][dv]
  float* pm;      // [nq][hq][nsplit]
  float* pl;      // [nq][hq][nsplit]
};

__device__ __forceinline__ int64_t causal_limit(const cs_attn_params& p, int64_t qp) {
  if (p.kpos == nullptr) return qp + 1 < p.nk ? qp + 1 : p.nk;
  int64_t lo = 0, hi = p.nk;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (p.kpos[mid] <= qp) lo = mid + 1; else hi = mid;
  }
  return lo;
}

template <typename T>
__device__ __forceinline__ const char* key_row(const DecodeArgs& a, int64_t j, int g, bool v,
                                               bool& ok) {
  const cs_attn_params& p = a.p;
  if (p.kv_slots) {
    int64_t s = p.kv_slots[j];
    ok = a.pv.valid(s);
    if (!ok) return nullptr;
    return a.pv.addr(s, g, v ? a.pv.head_dim : 0);
  }
  ok = true;
  const char* base = static_cast<const char*>(v ? p.v : p.k);
  int64_t st = v ? p.v_stride_tok : p.k_stride_tok, sh = v ? p.v_stride_head : p.k_stride_head;
  return base + (j * st + (int64_t)g * sh) * (int64_t)sizeof(T);
}

// phase 1: logits of this split's keys for the G heads of KV head g, gate
// totals, and (split 0) the q.E tables
template <typename T>
__global__ void __launch_bounds__(kSplit) decode_phase1(DecodeArgs a) {
  const cs_attn_params& p = a.p;
  const int s = blockIdx.x, g = blockIdx.y;
  const int64_t i = blockIdx.z;
  const int tid = threadIdx.x, G = a.G, d = p.d;
  __shared__ float qs[kMaxG * kMaxD];
  __shared__ float red[kMaxG][kSplit / 32];
  const int64_t qp = p.qpos[i];
  const int64_t nlim = causal_limit(p, qp);
  for (int e = tid; e < G * d; e += kSplit) {
    int hh = e / d, x = e - hh * d;
    const T* qrow = reinterpret_cast<const T*>(
        static_cast<const char*>(p.q) +
        (i * p.q_stride_tok + (int64_t)(g * G + hh) * p.q_stride_head) * (int64_t)sizeof(T));
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
    const char* kr = key_row<T>(a, j, g, false, ok);
    if (!ok) {
      bits |= CS_ST_SLOT_RANGE;
    } else {
      float acc[kMaxG];
#pragma unroll
      for (int hh = 0; hh < kMaxG; ++hh) acc[hh] = 0.f;
      constexpr int V = 16 / sizeof(T);
      const int64_t se = p.kv_slots ? a.pv.se : (int64_t)sizeof(T);
      if (se == (int64_t)sizeof(T) && (reinterpret_cast<uintptr_t>(kr) & 15) == 0 && d % V == 0) {
        for (int e0 = 0; e0 < d; e0 += V) {
          uint4 raw = *reinterpret_cast<const uint4*>(kr + e0 * sizeof(T));
          const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int u = 0; u < V; ++u) {
            float kv = Elem<T>::to_f(x[u]);
#pragma unroll
            for (int hh = 0; hh < kMaxG; ++hh)
              if (hh < G) acc[hh] = fmaf(qs[hh * d + e0 + u], kv, acc[hh]);
          }
        }
      } else {
        for (int e = 0; e < d; ++e) {
          float kv = Elem<T>::to_f(*reinterpret_cast<const T*>(kr + e * se));
#pragma unroll
          for (int hh = 0; hh < kMaxG; ++hh)
            if (hh < G) acc[hh] = fmaf(qs[hh * d + e], kv, acc[hh]);
        }
      }
#pragma unroll
      for (int hh = 0; hh < kMaxG; ++hh) {
        if (hh >= G) break;
        float l = acc[hh] / (float)p.scale;
        if (!isfinite(l)) bits |= CS_ST_LOGIT_NONFINITE;
        a.logits[(i * p.hq + g * G + hh) * a.nk_pad + j] = l;
        gate[hh] = 1.f / (1.f + expf(-l));
      }
    }
  }
  // gate totals of this split, per head
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    if (hh >= G) break;
    float v = warp_sum(gate[hh]);
    if (lane == 0) red[hh][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float tot = 0.f;
    for (int w = kSplit / 32 - 1; w >= 0; --w) tot += red[tid][w];
    a.gsum[(i * p.hq + g * G + tid) * a.nsplit + s] = tot;
  }
  if (s == 0) {
    const float* E = static_cast<const float*>(p.E);
    for (int e = tid; e < G * p.npos; e += kSplit) {
      int hh = e / p.npos, pp = e - hh * p.npos;
      float t = 0.f;
      for (int x = 0; x < d; ++x) t = fmaf(qs[hh * d + x], E[x * p.e_stride_d + pp * p.e_stride_p], t);
      a.table[(i * p.hq + g * G + hh) * p.npos + pp] = t;
    }
  }
  bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
  if (lane == 0 && bits) report(p.status, bits);
}

// phase 2: carried count, reverse scan, bias, partial softmax and PV
template <typename T>
__global__ void __launch_bounds__(kSplit) decode_phase2(DecodeArgs a) {
  const cs_attn_params& p = a.p;
  const int s = blockIdx.x, g = blockIdx.y;
  const int64_t i = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = a.G;
  const int npos = p.npos, dv = p.dv;
  extern __shared__ __align__(16) float dyn[];
  float* tab = dyn;                      // [G][npos]
  float* wts = tab + G * npos;           // [G][kSplit]
  __shared__ float wtot[kMaxG][kSplit / 32];
  __shared__ float carry0[kMaxG];
  __shared__ float red[kMaxG][kSplit / 32];
  __shared__ float mmax[kMaxG];
  __shared__ const char* vrows[kSplit];
  const int64_t qp = p.qpos[i];
  const int64_t nlim = causal_limit(p, qp);
  const int64_t base = (int64_t)s * kSplit;
  const int64_t rowh0 = i * p.hq + (int64_t)g * G;
  if (base >= nlim) {  // split entirely in the future: empty partial
    if (tid < G) {
      a.pm[(rowh0 + tid) * a.nsplit + s] = -INFINITY;
      a.pl[(rowh0 + tid) * a.nsplit + s] = 0.f;
    }
    return;
  }
  const int last = (int)((nlim - 1) / kSplit);
  if (tid < G) {
    float c = 0.f;
    for (int t = last; t > s; --t) c += a.gsum[(rowh0 + tid) * a.nsplit + t];
    carry0[tid] = c;
  }
  for (int e = tid; e < G * npos; e += kSplit) tab[e] = a.table[rowh0 * npos + e];
  const int64_t j = base + tid;
  const bool live = j < nlim;
  int32_t bits = 0;
  {
    bool ok = false;
    const char* vr = live ? key_row<T>(a, j, g, true, ok) : nullptr;
    if (live && !ok) bits |= CS_ST_SLOT_RANGE;
    vrows[tid] = ok ? vr : nullptr;
  }
  float lg[kMaxG], gt[kMaxG];
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    lg[hh] = 0.f;
    gt[hh] = 0.f;
    if (hh < G && live) {
      lg[hh] = a.logits[(rowh0 + hh) * a.nk_pad + j];
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
      float t = __shfl_down_sync(0xffffffffu, v, o);
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
    float R = suf[hh] + c;
    float pos = R < 0.f ? 0.f : (R > top ? top : R);
    int lo = (int)floorf(pos);
    int hi = lo + 1 < npos ? lo + 1 : npos - 1;
    float f = pos - (float)lo;
    float tlo = tab[hh * npos + lo];
    if (live) score[hh] = lg[hh] + (tlo + f * (tab[hh * npos + hi] - tlo));
  }
  // split max and weights
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    if (hh >= G) break;
    float v = warp_max(score[hh]);
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
    float w = live ? expf(score[hh] - mmax[hh]) : 0.f;
    wts[hh * kSplit + tid] = w;
    float v = warp_sum(w);
    __syncwarp();
    if (lane == 0) wtot[hh][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float l = 0.f;
    for (int w = 0; w < kSplit / 32; ++w) l += wtot[tid][w];
    a.pm[(rowh0 + tid) * a.nsplit + s] = mmax[tid];
    a.pl[(rowh0 + tid) * a.nsplit + s] = l;
  }
  // PV: thread <-> output dimension, keys broadcast from shared memory
  const int nkeys = (int)((nlim - base) < kSplit ? (nlim - base) : kSplit);
  const int64_t se = p.kv_slots ? a.pv.se : (int64_t)sizeof(T);
  for (int x = tid; x < dv; x += kSplit) {
    float acc[kMaxG];
#pragma unroll
    for (int hh = 0; hh < kMaxG; ++hh) acc[hh] = 0.f;
    for (int kk = 0; kk < nkeys; ++kk) {
      const char* vr = vrows[kk];
      if (vr == nullptr) continue;
      float vv = Elem<T>::to_f(*reinterpret_cast<const T*>(vr + x * se));
#pragma unroll
      for (int hh = 0; hh < kMaxG; ++hh)
        if (hh < G) acc[hh] = fmaf(wts[hh * kSplit + kk], vv, acc[hh]);
    }
#pragma unroll
    for (int hh = 0; hh < kMaxG; ++hh)
      if (hh < G) a.po[((rowh0 + hh) * a.nsplit + s) * dv + x] = acc[hh];
  }
  if (bits) report(p.status, bits);
}

// combine split partials: one CTA per (query row, head)
__global__ void decode_combine(DecodeArgs a) {
  const cs_attn_params& p = a.p;
  const int64_t i = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t rowh = i * p.hq + h;
  const int64_t nlim = causal_limit(p, p.qpos[i]);
  const int nsp = nlim > 0 ? (int)((nlim - 1) / kSplit) + 1 : 0;
  float M = -INFINITY;
  for (int s = 0; s < nsp; ++s) M = fmaxf(M, a.pm[rowh * a.nsplit + s]);
  float L = 0.f;
  for (int s = 0; s < nsp; ++s) {
    float m = a.pm[rowh * a.nsplit + s];
    if (m > -INFINITY) L += expf(m - M) * a.pl[rowh * a.nsplit + s];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  char* orow = static_cast<char*>(p.out) +
               (i * p.o_stride_tok + (int64_t)h * p.o_stride_head) * dtype_size(p.out_dtype);
  int32_t bits = 0;
  for (int x = threadIdx.x; x < p.dv; x += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsp; ++s) {
      float m = a.pm[rowh * a.nsplit + s];
      if (m > -INFINITY) acc += expf(m - M) * a.po[(rowh * a.nsplit + s) * p.dv + x];
    }
    float val = acc * inv;
    if (!isfinite(val)) bits |= CS_ST_LOGIT_NONFINITE;
    switch (p.out_dtype) {
      case CS_F32: reinterpret_cast<float*>(orow)[x] = val; break;
      case CS_F16: reinterpret_cast<__half*>(orow)[x] = __float2half_rn(val); break;
      default: reinterpret_cast<__nv_bfloat16*>(orow)[x] = __float2bfloat16_rn(val); break;
    }
  }
  if (bits) report(p.status, bits);
}

bool decode_supported(const cs_attn_params* p) {
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

struct Layout {
  int G, nsplit, nk_pad;
  int64_t logits, gsum, table, po, pm, pl, total;  // float offsets / count
};

Layout layout_of(const cs_attn_params* p) {
  Layout L;
  L.G = p->hq / p->hkv;
  L.nsplit = (p->nk + kSplit - 1) / kSplit;
  L.nk_pad = L.nsplit * kSplit;
  const int64_t rows = (int64_t)p->nq * p->hq;
  int64_t off = 0;
  auto take = [&](int64_t n) {
    int64_t o = off;
    off += (n + 63) / 64 * 64;  // 256-byte aligned sections
    return o;
  };
  L.logits = take(rows * L.nk_pad);
  L.gsum = take(rows * L.nsplit);
  L.table = take(rows * p->npos);
  L.po = take(rows * L.nsplit * p->dv);
  L.pm = take(rows * L.nsplit);
  L.pl = take(rows * L.nsplit);
  L.total = off;
  return L;
}

}  // namespace

// shared with the no-allocation variant
int64_t decode_workspace_bytes(const cs_attn_params* p) {
  if (validate_attn_params(p) != CS_OK || !decode_supported(p)) return 0;
  return layout_of(p).total * (int64_t)sizeof(float);
}

int launch_decode(const cs_attn_params* p, void* workspace, cudaStream_t stream) {
  int rc = validate_attn_params(p);
  if (rc != CS_OK) return rc;
  if (!decode_supported(p)) return CS_ERR_UNSUPPORTED;
  if (p->nq == 0) return CS_OK;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255)) return CS_ERR_INVALID;
  Layout L = layout_of(p);
  DecodeArgs a;
  a.p = *p;
  a.pv = p->kv_slots ? PagedView::make(p->paged) : PagedView{};
  a.G = L.G;
  a.nsplit = L.nsplit;
  a.nk_pad = L.nk_pad;
  float* ws = static_cast<float*>(workspace);
  a.logits = ws + L.logits;
  a.gsum = ws + L.gsum;
  a.table = ws + L.table;
  a.po = ws + L.po;
  a.pm = ws + L.pm;
  a.pl = ws + L.pl;
  dim3 grid(L.nsplit, p->hkv, p->nq);
  size_t smem2 = (size_t)(L.G * p->npos + L.G * kSplit) * sizeof(float);
  if (smem2 > 48 * 1024) return CS_ERR_UNSUPPORTED;
  if (p->in_dtype == CS_BF16) {
    decode_phase1<__nv_bfloat16><<<grid, kSplit, 0, stream>>>(a);
    decode_phase2<__nv_bfloat16><<<grid, kSplit, smem2, stream>>>(a);
  } else {
    decode_phase1<__half><<<grid, kSplit, 0, stream>>>(a);
    decode_phase2<__half><<<grid, kSplit, smem2, stream>>>(a);
  }
  decode_combine<<<dim3(p->nq, p->hq), 128, 0, stream>>>(a);
  CS_LAUNCH_CHECK();
  return CS_OK;
}

}  // namespace cs

using namespace cs;

extern "C" int64_t cs_cope_attn_decode_workspace(const cs_attn_params* p) {
  return decode_workspace_bytes(p);
}

extern "C" int cs_cope_attn_decode(const cs_attn_params* p, void* workspace, void* stream) {
  return launch_decode(p, workspace, as_stream(stream));
}
