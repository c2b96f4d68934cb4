// Generic CoPE / CCPE attention (cope_attention, position.py:404-560).
//
// One warp owns one (query row, KV head, group of up to 4 query heads) and
// walks the causal keys from the newest one backwards in tiles of 32 keys,
// one key per lane.  Per tile it
//   1. computes the logits of the lane's key for every head of the group,
//   2. turns them into gates and runs a segmented reverse scan across the
//      lanes, combined with the count carried from the newer tiles
//      (contextual positions, position.py:295-307; a chunk boundary whose
//      offset is >= 0 restarts the count: the compressed CCPE positions),
//   3. substitutes fixed/table positions, validates the path (strict mode,
//      position.py:28-114) and interpolates the learned bias from the q.E table
//      kept in shared memory (position.py:309-344),
//   4. applies visibility (masks, SelectedAssociationPolicy) and folds the
//      tile into an online softmax and the PV accumulator (each lane owns
//      dv/32 output dimensions).
// Every mode of the reference operator runs here, with float64 accumulation for
// float64 inputs and float32 otherwise.  It is the decode / small-shape path and
// the parity workhorse; the tensor-core kernel covers large bf16/fp16 prefill.
#include <math.h>

#include "common.cuh"

namespace cs {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxDvPerLane = 8;  // dv <= 256

template <typename A> __device__ __forceinline__ A a_exp(A x);
template <> __device__ __forceinline__ float a_exp<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double a_exp<double>(double x) { return exp(x); }
template <typename A> __device__ __forceinline__ A a_sigmoid(A x) {
  return A(1) / (A(1) + a_exp<A>(-x));
}
template <typename A> __device__ __forceinline__ A a_inf();
template <> __device__ __forceinline__ float a_inf<float>() { return __int_as_float(0x7f800000); }
template <> __device__ __forceinline__ double a_inf<double>() {
  return __longlong_as_double(0x7ff0000000000000ll);
}
template <typename A> __device__ __forceinline__ A a_eps();
template <> __device__ __forceinline__ float a_eps<float>() { return 1.1920928955078125e-07f; }
template <> __device__ __forceinline__ double a_eps<double>() { return 2.220446049250313e-16; }

struct Launch {
  cs_attn_params p;
  PagedView pv;
  int group;   // query heads per KV head
  int hb;      // heads per warp
  int nhc;     // head chunks per KV head
  int dvl;     // output dims per lane
};

template <typename T, typename A, int HB>
__device__ __forceinline__ void row_dot(const char* row, int64_t se, const A* __restrict__ qs,
                                        int d, A out[HB]) {
#pragma unroll
  for (int h = 0; h < HB; ++h) out[h] = A(0);
  if (se == (int64_t)sizeof(T) && (reinterpret_cast<uintptr_t>(row) % 16) == 0 &&
      (d * (int)sizeof(T)) % 16 == 0) {
    constexpr int V = 16 / sizeof(T);
    const uint4* vp = reinterpret_cast<const uint4*>(row);
    for (int e0 = 0; e0 < d; e0 += V) {
      uint4 raw = vp[e0 / V];
      const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < V; ++u) {
        A kv = to_acc<A>(x[u]);
#pragma unroll
        for (int h = 0; h < HB; ++h) out[h] += qs[h * d + e0 + u] * kv;
      }
    }
  } else {
    for (int e = 0; e < d; ++e) {
      A kv = to_acc<A>(*reinterpret_cast<const T*>(row + e * se));
#pragma unroll
      for (int h = 0; h < HB; ++h) out[h] += qs[h * d + e] * kv;
    }
  }
}

template <typename T, typename A, int HB>
__global__ void __launch_bounds__(kWarps * 32) cope_generic_kernel(Launch L) {
  const cs_attn_params& p = L.p;
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int d = p.d, npos = p.npos, dvl = L.dvl;
  A* qs = reinterpret_cast<A*>(smem) + (size_t)warp * HB * (d + npos);
  A* ts = qs + HB * d;
  const A atol = (A)p.atol;
  const A top = (A)(npos - 1);
  const bool paged = p.kv_slots != nullptr;
  const char* kbase = static_cast<const char*>(p.k);
  const char* vbase = static_cast<const char*>(p.v);
  const int64_t items = (int64_t)p.nq * p.hkv * L.nhc;

  for (int64_t item = (int64_t)blockIdx.x * kWarps + warp; item < items;
       item += (int64_t)gridDim.x * kWarps) {
    const int64_t i = item / (p.hkv * L.nhc);
    const int rem = (int)(item - i * p.hkv * L.nhc);
    const int g = rem / L.nhc;
    const int h0 = g * L.group + (rem % L.nhc) * HB;  // first query head
    const int64_t qp = p.qpos[i];

    // ---- stage q rows and the q.E tables (position.py:335-338)
    for (int hh = 0; hh < HB; ++hh) {
      const T* qrow = reinterpret_cast<const T*>(static_cast<const char*>(p.q) +
                                                 (i * p.q_stride_tok + (int64_t)(h0 + hh) *
                                                                           p.q_stride_head) *
                                                     (int64_t)sizeof(T));
      for (int e = lane; e < d; e += 32) qs[hh * d + e] = to_acc<A>(qrow[e]);
    }
    __syncwarp();
    for (int pp = lane; pp < npos; pp += 32) {
      A t[HB];
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) t[hh] = A(0);
      const A* ecol = static_cast<const A*>(p.E) + pp * p.e_stride_p;
      for (int e = 0; e < d; ++e) {
        A ev = ecol[e * p.e_stride_d];
#pragma unroll
        for (int hh = 0; hh < HB; ++hh) t[hh] += qs[hh * d + e] * ev;
      }
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) ts[hh * npos + pp] = t[hh];
    }
    __syncwarp();

    // ---- causal limit: keys with coordinate <= qp form a prefix
    int64_t nlim;
    if (p.kpos == nullptr) {
      nlim = qp + 1 < p.nk ? qp + 1 : p.nk;
    } else {
      int64_t lo = 0, hi = p.nk;
      if (lane == 0) {
        while (lo < hi) {
          int64_t mid = (lo + hi) >> 1;
          if (p.kpos[mid] <= qp) lo = mid + 1; else hi = mid;
        }
      }
      nlim = __shfl_sync(0xffffffffu, lo, 0);
    }
    const int qchunk = (p.pos_mode == CS_POS_CHUNK && nlim > 0) ? p.key_chunk[nlim - 1] : -1;
    const int32_t qrow_t = (p.pos_mode == CS_POS_TABLE) ? p.q_row[i] : -1;
    const bool qsel = p.q_selected != nullptr && p.q_selected[i] != 0;

    A carry[HB], m[HB], lsum[HB], acc[HB][kMaxDvPerLane], prev_p[HB];
    bool prev_valid[HB];
#pragma unroll
    for (int hh = 0; hh < HB; ++hh) {
      carry[hh] = A(0);
      m[hh] = -a_inf<A>();
      lsum[hh] = A(0);
      prev_p[hh] = A(0);
      prev_valid[hh] = false;
#pragma unroll
      for (int x = 0; x < kMaxDvPerLane; ++x) acc[hh][x] = A(0);
    }
    int32_t bits = 0;

    for (int64_t t_end = nlim; t_end > 0; t_end -= 32) {
      const int64_t j = t_end - 32 + lane;
      const bool active = j >= 0;
      A lg[HB];
      const char* vrow = nullptr;
      bool kv_ok = active;
      if (active) {
        const char* krow;
        if (paged) {
          int64_t s = p.kv_slots[j];
          if (!L.pv.valid(s)) {
            kv_ok = false;
            bits |= CS_ST_SLOT_RANGE;
          } else {
            krow = L.pv.addr(s, g, 0);
            vrow = L.pv.addr(s, g, L.pv.head_dim);
          }
        } else {
          krow = kbase + (j * p.k_stride_tok + (int64_t)g * p.k_stride_head) * (int64_t)sizeof(T);
          vrow = vbase + (j * p.v_stride_tok + (int64_t)g * p.v_stride_head) * (int64_t)sizeof(T);
        }
        if (kv_ok) {
          row_dot<T, A, HB>(krow, paged ? L.pv.se : (int64_t)sizeof(T), qs, d, lg);
#pragma unroll
          for (int hh = 0; hh < HB; ++hh) lg[hh] = lg[hh] / (A)p.scale;
        }
      }
      if (!kv_ok) {
#pragma unroll
        for (int hh = 0; hh < HB; ++hh) lg[hh] = A(0);
      }
      const int64_t kp = active ? (p.kpos ? p.kpos[j] : j) : 0;
      const bool kfix = active && p.k_fixed != nullptr && p.k_fixed[j] != 0;
      int kc = -1;
      bool boundary = false;
      if (p.pos_mode == CS_POS_CHUNK && active) {
        kc = p.key_chunk[j];
        boundary = (j + 1 < p.nk) && p.key_chunk[j + 1] != kc && kc < qchunk;
      }
      const int32_t kord = (p.pos_mode == CS_POS_TABLE && active) ? p.k_ord[j] : -1;

#pragma unroll
      for (int hh = 0; hh < HB; ++hh) {
        const int h = h0 + hh;
        bool gate_ok = active && kv_ok;
        if (gate_ok && p.gate_mask)
          gate_ok = p.gate_mask[h * p.gm_stride_h + i * p.gm_stride_q + j] != 0;
        const A gv = gate_ok ? a_sigmoid<A>(lg[hh]) : A(0);
        // affine element of the reverse recurrence R_j = a_j * R_{j+1} + b_j
        A ea = A(1), eb = gv;
        if (boundary) {
          float off = p.chunk_off[h * p.co_stride_h + i * p.co_stride_q + kc];
          if (off >= 0.f) {
            ea = A(0);
            eb = gv + (A)off;
          }
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          A a2 = __shfl_down_sync(0xffffffffu, ea, o);
          A b2 = __shfl_down_sync(0xffffffffu, eb, o);
          if (lane + o < 32) {
            eb = eb + ea * b2;
            ea = ea * a2;
          }
        }
        const A R = eb + ea * carry[hh];
        carry[hh] = __shfl_sync(0xffffffffu, R, 0);
        A pos = R < A(0) ? A(0) : (R > top ? top : R);
        bool subst = false;
        if (p.pos_mode == CS_POS_FIXED && active) {
          pos = *reinterpret_cast<const A*>(static_cast<const char*>(p.fixed_pos) +
                                            (h * p.fp_stride_h + i * p.fp_stride_q +
                                             j * p.fp_stride_k) * (int64_t)sizeof(A));
          subst = true;
        } else if (p.pos_mode == CS_POS_TABLE && qrow_t >= 0 && kord >= 0) {
          pos = *reinterpret_cast<const A*>(static_cast<const char*>(p.table) +
                                            (h * p.tb_stride_h + (int64_t)qrow_t * p.tb_stride_r +
                                             (int64_t)kord * p.tb_stride_c) * (int64_t)sizeof(A));
          subst = true;
        }
        if (subst && !(pos >= A(0) && pos <= top)) {
          bits |= CS_ST_POS_RANGE;
          pos = (pos >= A(0)) ? (pos <= top ? pos : top) : A(0);
        }
        if (p.strict) {
          // validate_contextual_path on causal (& attention_mask) cells
          const A rnd = a_eps<A>() * fabs(pos);
          if (gate_ok) {
            if (pos < -(atol + rnd)) bits |= CS_ST_PATH_NEG;
            A avail = (A)(qp - kp);
            avail = (avail < A(-1) ? A(-1) : avail) + A(1);
            if (pos > avail + atol + rnd) bits |= CS_ST_PATH_AVAIL;
          }
          A pn = __shfl_down_sync(0xffffffffu, pos, 1);
          bool vn = __shfl_down_sync(0xffffffffu, (int)gate_ok, 1) != 0;
          int64_t kn = __shfl_down_sync(0xffffffffu, kp, 1);
          if (lane == 31) {
            pn = prev_p[hh];
            vn = prev_valid[hh];
            kn = (j + 1 < p.nk) ? (p.kpos ? p.kpos[j + 1] : j + 1) : kp;
          }
          if (gate_ok && vn) {
            const A diff = pos - pn;
            const A ptol = atol + rnd + a_eps<A>() * fabs(pn);
            if (diff < -ptol) bits |= CS_ST_PATH_INCR;
            if (diff > (A)(kn - kp) + ptol) bits |= CS_ST_PATH_GAP;
          }
          prev_p[hh] = __shfl_sync(0xffffffffu, pos, 0);
          prev_valid[hh] = __shfl_sync(0xffffffffu, (int)gate_ok, 0) != 0;
        }
        if (p.out_positions && active) {
          *reinterpret_cast<A*>(static_cast<char*>(p.out_positions) +
                                (h * p.op_stride_h + i * p.op_stride_q + j) * (int64_t)sizeof(A)) =
              pos;
        }
        if (p.positions_only) continue;
        // interpolated learned bias (floor / floor+1, position.py:339-344)
        const int lo = (int)floor(pos);
        const int hi = lo + 1 < npos ? lo + 1 : npos - 1;
        const A frac = pos - (A)lo;
        const A tlo = ts[hh * npos + lo];
        const A score = lg[hh] + (tlo + frac * (ts[hh * npos + hi] - tlo));
        if (gate_ok && !isfinite(score)) bits |= CS_ST_LOGIT_NONFINITE;
        bool vis = gate_ok;
        if (vis && p.vis_mask) vis = p.vis_mask[h * p.vm_stride_h + i * p.vm_stride_q + j] != 0;
        if (vis && p.q_selected) vis = !qsel || !kfix || kp == qp;
        const A smax = warp_max<A>(vis ? score : -a_inf<A>());
        if (!(smax > -a_inf<A>())) {
          lg[hh] = A(0);  // weight of this head in this tile
          continue;
        }
        const A mnew = smax > m[hh] ? smax : m[hh];
        const A corr = a_exp<A>(m[hh] - mnew);
        m[hh] = mnew;
        lsum[hh] *= corr;
#pragma unroll
        for (int x = 0; x < kMaxDvPerLane; ++x) acc[hh][x] *= corr;
        const A w = vis ? a_exp<A>(score - mnew) : A(0);
        lsum[hh] += w;
        lg[hh] = w;  // reuse the register for this tile's weight
      }
      if (p.positions_only) continue;
      // PV: lanes own output dims; keys are broadcast one at a time
      for (int kk = 0; kk < 32; ++kk) {
        A wk[HB];
        bool any = false;
#pragma unroll
        for (int hh = 0; hh < HB; ++hh) {
          wk[hh] = __shfl_sync(0xffffffffu, lg[hh], kk);
          any |= wk[hh] != A(0);
        }
        const char* vr = reinterpret_cast<const char*>(__shfl_sync(
            0xffffffffu, (unsigned long long)reinterpret_cast<uintptr_t>(vrow), kk));
        if (!any || vr == nullptr) continue;
        const int64_t ve = paged ? L.pv.se : (int64_t)sizeof(T);
#pragma unroll
        for (int x = 0; x < kMaxDvPerLane; ++x) {
          if (x >= dvl) break;
          const int e = lane + 32 * x;
          if (e < p.dv) {
            A val = to_acc<A>(*reinterpret_cast<const T*>(vr + e * ve));
#pragma unroll
            for (int hh = 0; hh < HB; ++hh) acc[hh][x] += wk[hh] * val;
          }
        }
      }
    }

    // ---- positions of the non-causal cells, when a trace is requested
    if (p.out_positions) {
      for (int64_t j = nlim + lane; j < p.nk; j += 32) {
        for (int hh = 0; hh < HB; ++hh) {
          const int h = h0 + hh;
          A pos = A(0);
          if (p.pos_mode == CS_POS_FIXED) {
            pos = *reinterpret_cast<const A*>(static_cast<const char*>(p.fixed_pos) +
                                              (h * p.fp_stride_h + i * p.fp_stride_q +
                                               j * p.fp_stride_k) * (int64_t)sizeof(A));
          } else if (p.pos_mode == CS_POS_TABLE && qrow_t >= 0 && p.k_ord[j] >= 0) {
            pos = *reinterpret_cast<const A*>(static_cast<const char*>(p.table) +
                                              (h * p.tb_stride_h + (int64_t)qrow_t * p.tb_stride_r +
                                               (int64_t)p.k_ord[j] * p.tb_stride_c) *
                                                  (int64_t)sizeof(A));
          }
          *reinterpret_cast<A*>(static_cast<char*>(p.out_positions) +
                                (h * p.op_stride_h + i * p.op_stride_q + j) * (int64_t)sizeof(A)) =
              pos;
        }
      }
    }
    bits = (int32_t)__reduce_or_sync(0xffffffffu, (unsigned)bits);
    if (lane == 0 && bits) report(p.status, bits);
    if (!p.positions_only) {
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) {
        const A total = warp_sum(lsum[hh]);
        const A inv = total > A(0) ? A(1) / total : A(0);
        char* orow = static_cast<char*>(p.out) +
                     (i * p.o_stride_tok + (int64_t)(h0 + hh) * p.o_stride_head) *
                         (int64_t)dtype_size(p.out_dtype);
        for (int x = 0; x < dvl; ++x) {
          const int e = lane + 32 * x;
          if (e >= p.dv) break;
          const A val = acc[hh][x] * inv;
          switch (p.out_dtype) {
            case CS_F32: reinterpret_cast<float*>(orow)[e] = (float)val; break;
            case CS_F64: reinterpret_cast<double*>(orow)[e] = (double)val; break;
            case CS_F16: reinterpret_cast<__half*>(orow)[e] = from_acc<__half>(val); break;
            default: reinterpret_cast<__nv_bfloat16*>(orow)[e] = from_acc<__nv_bfloat16>(val); break;
          }
        }
      }
    }
    __syncwarp();
  }
}

template <typename T, typename A, int HB>
int launch_generic(const Launch& L, cudaStream_t stream) {
  size_t smem = (size_t)kWarps * HB * (L.p.d + L.p.npos) * sizeof(A);
  auto kern = cope_generic_kernel<T, A, HB>;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return CS_ERR_UNSUPPORTED;
  }
  int64_t items = (int64_t)L.p.nq * L.p.hkv * L.nhc;
  int64_t blocks = (items + kWarps - 1) / kWarps;
  int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  kern<<<(int)blocks, kWarps * 32, smem, stream>>>(L);
  CS_LAUNCH_CHECK();
  return CS_OK;
}

template <typename T, typename A>
int dispatch_hb(const Launch& L, cudaStream_t s) {
  switch (L.hb) {
    case 4: return launch_generic<T, A, 4>(L, s);
    case 2: return launch_generic<T, A, 2>(L, s);
    default: return launch_generic<T, A, 1>(L, s);
  }
}

}  // namespace

// shared with the other attention translation units
int validate_attn_params(const cs_attn_params* p) {
  if (!p) return CS_ERR_INVALID;
  if (p->nq < 0 || p->hq <= 0 || p->hkv <= 0 || p->d <= 0 || p->dv <= 0 || p->nk <= 0)
    return CS_ERR_INVALID;
  if (p->hq % p->hkv) return CS_ERR_INVALID;
  if (p->npos < 2 || p->npos > 4096) return CS_ERR_INVALID;
  if (!(p->scale > 0)) return CS_ERR_INVALID;
  if (p->nq > 0 && (!p->q || !p->qpos || !p->E)) return CS_ERR_INVALID;
  if (!p->positions_only && p->nq > 0 && !p->out) return CS_ERR_INVALID;
  if (dtype_size(p->in_dtype) == 0 || dtype_size(p->out_dtype) == 0) return CS_ERR_INVALID;
  if (p->kv_slots) {
    const cs_paged_kv& kv = p->paged;
    if (!kv.cache || kv.dtype != p->in_dtype || kv.kv_heads != p->hkv || kv.head_dim != p->d ||
        p->dv != p->d || kv.block_size <= 0 || kv.num_blocks <= 0)
      return CS_ERR_INVALID;
  } else if (!p->k || !p->v) {
    return CS_ERR_INVALID;
  }
  switch (p->pos_mode) {
    case CS_POS_CONTEXTUAL: break;
    case CS_POS_FIXED: if (!p->fixed_pos) return CS_ERR_INVALID; break;
    case CS_POS_TABLE: if (!p->table || !p->q_row || !p->k_ord) return CS_ERR_INVALID; break;
    case CS_POS_CHUNK:
      if (!p->key_chunk || !p->chunk_off || p->nchunks <= 0) return CS_ERR_INVALID;
      break;
    default: return CS_ERR_INVALID;
  }
  if ((p->q_selected == nullptr) != (p->k_fixed == nullptr)) return CS_ERR_INVALID;
  return CS_OK;
}

}  // namespace cs

using namespace cs;

extern "C" int cs_cope_attn(const cs_attn_params* p, void* stream) {
  if (p != nullptr && p->nq_dev != nullptr) return CS_ERR_UNSUPPORTED;  // prefill only
  int rc = validate_attn_params(p);
  if (rc != CS_OK) return rc;
  if (p->nq == 0) return CS_OK;
  if (p->dv > 32 * kMaxDvPerLane || p->d > 1024) return CS_ERR_UNSUPPORTED;
  Launch L;
  L.p = *p;
  L.pv = p->kv_slots ? PagedView::make(p->paged) : PagedView{};
  L.group = p->hq / p->hkv;
  L.hb = (L.group % 4 == 0) ? 4 : (L.group % 2 == 0 ? 2 : 1);
  L.nhc = L.group / L.hb;
  L.dvl = (p->dv + 31) / 32;
  cudaStream_t s = as_stream(stream);
  switch (p->in_dtype) {
    case CS_F64: return dispatch_hb<double, double>(L, s);
    case CS_F32: return dispatch_hb<float, float>(L, s);
    case CS_F16: return dispatch_hb<__half, float>(L, s);
    case CS_BF16: return dispatch_hb<__nv_bfloat16, float>(L, s);
    default: return CS_ERR_INVALID;
  }
}
