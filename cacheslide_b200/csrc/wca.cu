// Weighted Correction Attention kernels: float64 deviation/weight reductions,
// mean-head cosine, block radix top-k with stable tie-break, the fused
// blend (+ paged scatter) update and the selection commit.
//
// All reductions accumulate in float64 like the reference (wca.py:55-112).
// Each token row is owned by one warp; rows are [heads, dim] with arbitrary
// row/head strides and a contiguous innermost dimension.
#include <initializer_list>
#include <type_traits>

#include "common.cuh"

namespace cs {
namespace {

constexpr int kSelectThreads = 1024;
constexpr int kSelectMaxChosen = 16384;  // ordered picks staged in shared memory

// --------------------------------------------------------------- row access
template <typename T>
struct Rows {
  const char* base;
  int64_t srow, shead;  // byte strides
  __device__ __forceinline__ const T* ptr(int64_t r, int64_t h) const {
    return reinterpret_cast<const T*>(base + r * srow + h * shead);
  }
};

// Order-preserving map from float64 to uint64 (larger key -> larger code).
__device__ __forceinline__ uint64_t order_code(double x) {
  uint64_t b = __double_as_longlong(x);
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

// inclusive block scan of an int over blockDim.x threads (multiple of 32)
__device__ int block_inclusive_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int nw = blockDim.x >> 5;
    int w = lane < nw ? warp_tot[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < nw) warp_tot[lane] = w;
  }
  __syncthreads();
  int add = warp > 0 ? warp_tot[warp - 1] : 0;
  __syncthreads();
  return v + add;
}

__device__ int block_sum(int v, int* warp_tot) {
  int inc = block_inclusive_scan(v, warp_tot);
  __shared__ int total;
  if (threadIdx.x == blockDim.x - 1) total = inc;
  __syncthreads();
  int t = total;
  __syncthreads();
  return t;
}

// Shared-memory workspace of the block selection.
struct SelectSmem {
  int hist[256];
  int warp_tot[32];
  uint64_t prefix, mask;
  int remaining;
  int whole_bin;  // the k-th pick's bin is taken whole: no finer digits needed
  int chosen_count;
  int eq_taken;
};

// Select the `slots` largest keys among available tokens, ties to the lower
// index (the order of a stable descending argsort, wca.py:282-285), for n
// beyond what shared memory stages.  Must be called by every thread of one
// block of kSelectThreads threads.  `avail` is a functor (int64 i) -> bool
// evaluated against the current state.  The order codes stay in global
// memory (L2): one pass counts the available keys and finds the first byte
// where their codes differ; MSB-first 8-bit radix passes from that byte
// (per-warp histogram copies) find the k-th code and stop once its bin is
// taken whole; an ordered compaction stages the picks (code, index) in
// shared memory, and a bitonic sort there puts them in rank order.
template <typename Avail>
__device__ int64_t block_select_topk(const double* __restrict__ keys, Avail avail, int64_t n,
                                     int64_t slots, uint8_t* __restrict__ selected,
                                     int64_t* __restrict__ chosen_out, SelectSmem& sm,
                                     double* stage_key, int* stage_idx, int32_t* status) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned full = 0xffffffffu;
  __shared__ int hist4[4][256];
  __shared__ uint64_t wlo[32], whi[32];
  // how many are available, and the range of their codes
  int local = 0;
  uint64_t lo = ~0ull, hi = 0ull;
  for (int64_t i = tid; i < n; i += blockDim.x) {
    if (!avail(i)) continue;
    ++local;
    const uint64_t c = order_code(keys[i]);
    lo = c < lo ? c : lo;
    hi = c > hi ? c : hi;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t l2 = __shfl_xor_sync(full, lo, o), h2 = __shfl_xor_sync(full, hi, o);
    lo = l2 < lo ? l2 : lo;
    hi = h2 > hi ? h2 : hi;
  }
  if (lane == 0) {
    wlo[warp] = lo;
    whi[warp] = hi;
  }
  const int64_t total = block_sum(local, sm.warp_tot);  // also orders wlo / whi
  const int64_t want = slots < total ? slots : total;
  if (want <= 0) return 0;
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    lo = lane < nw ? wlo[lane] : ~0ull;
    hi = lane < nw ? whi[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t l2 = __shfl_xor_sync(full, lo, o), h2 = __shfl_xor_sync(full, hi, o);
      lo = l2 < lo ? l2 : lo;
      hi = h2 > hi ? h2 : hi;
    }
    if (lane == 0) {
      sm.mask = lo ^ hi;
      sm.prefix = hi;
    }
  }
  __syncthreads();
  const uint64_t diff = sm.mask;
  int top = 56;  // first byte (from the top) where the available codes differ
  while (top > 0 && ((diff >> top) & 255ull) == 0ull) top -= 8;
  uint64_t mask = top < 56 ? (~0ull << (top + 8)) : 0ull;
  uint64_t prefix = sm.prefix & mask;
  int remaining = (int)want;
  int* mine = hist4[warp & 3];
  __syncthreads();
  for (int shift = top; shift >= 0; shift -= 8) {
    for (int b = tid; b < 4 * 256; b += blockDim.x) hist4[b >> 8][b & 255] = 0;
    __syncthreads();
    for (int64_t i = tid; i < n; i += blockDim.x) {
      if (!avail(i)) continue;
      const uint64_t c = order_code(keys[i]);
      if ((c & mask) == prefix) atomicAdd(&mine[(c >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending)
      int cnt[8], sum = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int b = 255 - 8 * lane - q;
        cnt[q] = hist4[0][b] + hist4[1][b] + hist4[2][b] + hist4[3][b];
        sum += cnt[q];
      }
      int inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(full, inc, o);
        if (lane >= o) inc += t;
      }
      const unsigned hit = __ballot_sync(full, inc >= remaining);
      const int owner = __ffs(hit) - 1;
      if (lane == owner) {
        int above = inc - sum, bsel = 0, inbin = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (above + cnt[q] >= remaining) {
            bsel = 255 - 8 * lane - q;
            inbin = cnt[q];
            break;
          }
          above += cnt[q];
        }
        sm.prefix = prefix | ((uint64_t)bsel << shift);
        sm.remaining = remaining - above;
        sm.whole_bin = remaining - above == inbin;
      }
    }
    __syncthreads();
    prefix = sm.prefix;
    remaining = sm.remaining;
    mask |= 255ull << shift;
    const bool whole = sm.whole_bin != 0;
    __syncthreads();
    if (whole) break;  // every code with these leading bytes is a pick
  }
  // ordered compaction: code above the k-th's leading bytes, or equal to them
  // among the first `remaining` by index
  if (tid == 0) {
    sm.chosen_count = 0;
    sm.eq_taken = 0;
  }
  __syncthreads();
  const bool stage = chosen_out != nullptr && want <= kSelectMaxChosen;
  uint64_t* scode = reinterpret_cast<uint64_t*>(stage_key);
  for (int64_t base = 0; base < n; base += blockDim.x) {
    const int64_t i = base + tid;
    const bool av = i < n && avail(i);
    const uint64_t c = av ? order_code(keys[i]) : 0ull;
    const int gt = (av && (c & mask) > prefix) ? 1 : 0;
    const int eq = (av && (c & mask) == prefix) ? 1 : 0;
    const int inc = block_inclusive_scan(gt | (eq << 16), sm.warp_tot);
    const int gt_before = (inc & 0xFFFF) - gt + sm.chosen_count;
    const int eq_before = (inc >> 16) - eq + sm.eq_taken;
    const bool pick = gt || (eq && eq_before < remaining);
    if (pick) {
      selected[i] = 1;
      if (stage) {
        const int slot = gt_before + (eq_before < remaining ? eq_before : remaining);
        scode[slot] = c;
        stage_idx[slot] = (int)i;
      }
    }
    __syncthreads();
    if (tid == blockDim.x - 1) {
      sm.chosen_count = gt_before + gt;
      sm.eq_taken = eq_before + eq;
    }
    __syncthreads();
  }
  const int k = (int)want;
  if (chosen_out != nullptr) {
    if (!stage) {
      if (tid == 0) report(status, CS_ST_SLOT_RANGE);
      return k;
    }
    // bitonic sort of the picks by (code descending, index ascending) over
    // the next power of two, padding after every pick
    int m = 1;
    while (m < k) m <<= 1;
    for (int a = k + tid; a < m; a += blockDim.x) {
      scode[a] = 0ull;
      stage_idx[a] = 0x7FFFFFFF;
    }
    __syncthreads();
    for (int w = 2; w <= m; w <<= 1) {
      for (int j = w >> 1; j > 0; j >>= 1) {
        for (int t = tid; t < (m >> 1); t += blockDim.x) {
          const int lo2 = 2 * t - (t & (j - 1)), hi2 = lo2 + j;
          const uint64_t cl = scode[lo2], ch = scode[hi2];
          const int il = stage_idx[lo2], ih = stage_idx[hi2];
          const bool hi_first = ch > cl || (ch == cl && ih < il);
          const bool lo_first = cl > ch || (cl == ch && il < ih);
          if ((lo2 & w) == 0 ? hi_first : lo_first) {
            scode[lo2] = ch;
            scode[hi2] = cl;
            stage_idx[lo2] = ih;
            stage_idx[hi2] = il;
          }
        }
        __syncthreads();
      }
    }
    for (int a = tid; a < k; a += blockDim.x) chosen_out[a] = stage_idx[a];
  }
  __syncthreads();
  return k;
}

// Top-k by a block-wide bitonic sort in shared memory (n <= kSortMax): every
// token gets the order code of its key (0 when unavailable) and its index;
// sorting by (code descending, index ascending) gives the stable descending
// order of wca.py:282-285 directly, so the first `want` entries are the picks
// in rank order.  `dyn` holds kSortMax codes and kSortMax indices.
constexpr int kSortMax = 16384;

template <typename Avail>
__device__ int64_t block_sort_topk(const double* __restrict__ keys, Avail avail, int64_t n,
                                   int64_t slots, uint8_t* __restrict__ selected,
                                   int64_t* __restrict__ chosen_out, SelectSmem& sm,
                                   unsigned char* dyn) {
  uint64_t* code = reinterpret_cast<uint64_t*>(dyn);
  uint32_t* idx = reinterpret_cast<uint32_t*>(dyn + sizeof(uint64_t) * kSortMax);
  const int tid = threadIdx.x;
  int m = 1;
  while (m < n) m <<= 1;
  int local = 0;
  for (int i = tid; i < m; i += blockDim.x) {
    const bool av = i < n && avail(i);
    local += av ? 1 : 0;
    code[i] = av ? order_code(keys[i]) : 0ull;
    // unavailable tokens after every available one with the same code;
    // padding last of all
    idx[i] = i < n ? ((uint32_t)i | (av ? 0u : 0x80000000u)) : 0xFFFFFFFFu;
  }
  const int64_t total = block_sum(local, sm.warp_tot);  // also orders the writes above
  const int64_t want = slots < total ? slots : total;
  if (want <= 0) return 0;
  for (int k = 2; k <= m; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < (m >> 1); i += blockDim.x) {
        const int lo = 2 * i - (i & (j - 1)), hi = lo + j;
        const uint64_t cl = code[lo], ch = code[hi];
        const uint32_t il = idx[lo], ih = idx[hi];
        const bool hi_first = ch > cl || (ch == cl && ih < il);
        const bool lo_first = cl > ch || (cl == ch && il < ih);
        if ((lo & k) == 0 ? hi_first : lo_first) {
          code[lo] = ch;
          code[hi] = cl;
          idx[lo] = ih;
          idx[hi] = il;
        }
      }
      __syncthreads();
    }
  }
  for (int64_t rk = tid; rk < want; rk += blockDim.x) {
    const int i = (int)(idx[rk] & 0x7FFFFFFFu);
    selected[i] = 1;
    if (chosen_out) chosen_out[rk] = i;
  }
  __syncthreads();
  return want;
}

// Top-k for n <= kSortMax and at most kFastPicks picks: the order codes of
// all tokens are staged in shared memory once; an MSB-first 8-bit radix
// select finds the code of the k-th pick (warp-aggregated histogram, bin
// search by one warp); an ordered compaction takes the picks, ties to the
// lower index; only the picks are then sorted by (code descending, index
// ascending), one per thread in registers (shuffles for partners within a
// warp, shared memory beyond).  Larger pick counts use block_sort_topk.
constexpr int kFastPicks = 1024;  // == kSelectThreads

template <typename Avail>
__device__ int64_t block_topk_staged(const double* __restrict__ keys, Avail avail, int64_t n,
                                     int64_t slots, uint8_t* __restrict__ selected,
                                     int64_t* __restrict__ chosen_out, SelectSmem& sm,
                                     unsigned char* dyn) {
  uint64_t* code = reinterpret_cast<uint64_t*>(dyn);  // [kSortMax], 0: unavailable
  uint64_t* pcode = code + kSortMax;                   // [kFastPicks] picks, then exchange
  uint32_t* pidx = reinterpret_cast<uint32_t*>(pcode + kFastPicks);
  int* whist = reinterpret_cast<int*>(pidx + kFastPicks);  // [32 warps][256] private histograms
  __shared__ int hist[256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned full = 0xffffffffu;
  int local = 0;
#pragma unroll 4
  for (int64_t i = tid; i < n; i += blockDim.x) {
    const bool av = avail(i);
    local += av ? 1 : 0;
    code[i] = av ? order_code(keys[i]) : 0ull;
  }
  const int64_t total = block_sum(local, sm.warp_tot);  // also orders the writes above
  const int64_t want = slots < total ? slots : total;
  if (want <= 0) return 0;
  if (want > kFastPicks)
    return block_sort_topk(keys, avail, n, slots, selected, chosen_out, sm, dyn);
  // the leading bytes shared by the smallest and largest available code are
  // those of every available code: the radix passes start below them
  uint64_t lo = ~0ull, hi = 0ull;
  for (int64_t i = tid; i < n; i += blockDim.x) {
    const uint64_t c = code[i];
    if (c != 0ull) {
      lo = c < lo ? c : lo;
      hi = c > hi ? c : hi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t l2 = __shfl_xor_sync(full, lo, o), h2 = __shfl_xor_sync(full, hi, o);
    lo = l2 < lo ? l2 : lo;
    hi = h2 > hi ? h2 : hi;
  }
  uint64_t* wmin = reinterpret_cast<uint64_t*>(whist);  // [32] lo, [32] hi, scratch
  if (lane == 0) {
    wmin[warp] = lo;
    wmin[32 + warp] = hi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    lo = lane < nw ? wmin[lane] : ~0ull;
    hi = lane < nw ? wmin[32 + lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t l2 = __shfl_xor_sync(full, lo, o), h2 = __shfl_xor_sync(full, hi, o);
      lo = l2 < lo ? l2 : lo;
      hi = h2 > hi ? h2 : hi;
    }
    if (lane == 0) sm.mask = lo ^ hi;  // differing bits
  }
  __syncthreads();
  const uint64_t diff = sm.mask;
  int top = 56;  // first byte (from the top) where the codes differ
  while (top > 0 && ((diff >> top) & 255ull) == 0ull) top -= 8;
  // radix select: prefix / mask of the k-th code, `remaining` of its ties
  uint64_t mask = top < 56 ? (~0ull << (top + 8)) : 0ull;
  uint64_t prefix = hi & mask;
  int remaining = (int)want;
  // four histogram copies, shared by warps w, w+4, ...: few enough to sum
  // quickly, enough to spread the atomics of equal digits
  int* mine = whist + (warp & 3) * 256;
  __syncthreads();  // wmin (aliasing whist) read by all before the histograms
  for (int b = tid; b < 4 * 256; b += blockDim.x) whist[b] = 0;
  __syncthreads();
  for (int shift = top; shift >= 0; shift -= 8) {
    for (int64_t base = 0; base < n; base += blockDim.x) {
      const int64_t i = base + tid;
      const uint64_t c = i < n ? code[i] : 0ull;
      if (c != 0ull && (c & mask) == prefix) atomicAdd(&mine[(c >> shift) & 255], 1);
    }
    __syncthreads();
    for (int b = tid; b < 256; b += blockDim.x) {
      hist[b] = whist[b] + whist[256 + b] + whist[512 + b] + whist[768 + b];
      whist[b] = whist[256 + b] = whist[512 + b] = whist[768 + b] = 0;  // for the next pass
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending)
      int cnt[8], sum = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cnt[q] = hist[255 - 8 * lane - q];
        sum += cnt[q];
      }
      int inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(full, inc, o);
        if (lane >= o) inc += t;
      }
      const int need = sm.remaining = remaining;  // every lane reads the same value
      const unsigned hit = __ballot_sync(full, inc >= need);
      const int owner = __ffs(hit) - 1;
      if (lane == owner) {
        int above = inc - sum, b = 0, inbin = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (above + cnt[q] >= need) {
            b = 255 - 8 * lane - q;
            inbin = cnt[q];
            break;
          }
          above += cnt[q];
        }
        sm.prefix = prefix | ((uint64_t)b << shift);
        sm.remaining = need - above;
        sm.whole_bin = need - above == inbin;
      }
    }
    __syncthreads();
    prefix = sm.prefix;
    remaining = sm.remaining;
    mask |= 255ull << shift;
    const bool whole = sm.whole_bin != 0;
    __syncthreads();
    // every code whose leading bytes equal the prefix is a pick: the
    // compaction below compares leading bytes only
    if (whole) break;
  }
  // ordered compaction of the picks: code above the k-th, or equal to it
  // among the first `remaining` by index
  if (tid == 0) {
    sm.chosen_count = 0;
    sm.eq_taken = 0;
  }
  __syncthreads();
  // one scan per step over (greater, equal) counts packed in 16-bit halves:
  // a pick's slot is #greater before it + min(#equal before it, remaining)
  for (int64_t base = 0; base < n; base += blockDim.x) {
    const int64_t i = base + tid;
    const uint64_t c = i < n ? code[i] : 0ull;
    const int gt = (c != 0ull && (c & mask) > prefix) ? 1 : 0;
    const int eq = (c != 0ull && (c & mask) == prefix) ? 1 : 0;
    const int inc = block_inclusive_scan(gt | (eq << 16), sm.warp_tot);
    const int gt_before = (inc & 0xFFFF) - gt + sm.chosen_count;  // greater ones so far
    const int eq_before = (inc >> 16) - eq + sm.eq_taken;
    const bool pick = gt || (eq && eq_before < remaining);
    if (pick) {
      const int slot = gt_before + (eq_before < remaining ? eq_before : remaining);
      pcode[slot] = c;
      pidx[slot] = (uint32_t)i;
    }
    __syncthreads();
    if (tid == blockDim.x - 1) {
      sm.chosen_count = gt_before + gt;
      sm.eq_taken = eq_before + eq;
    }
    __syncthreads();
  }
  // sort of the picks by (code descending, index ascending), a strict total
  // order (the padding entries get distinct indices too): each warp sorts 32
  // entries with a shuffle bitonic network, then rounds of pairwise merges,
  // where an entry's place in the merged run is its place in its own run plus
  // the number of entries of the partner run before it (binary search).
  int P = 32;
  while (P < want) P <<= 1;
  const bool part = tid < P;  // warp-uniform (P is a multiple of 32)
  auto before = [](uint64_t ca, uint32_t ia, uint64_t cb, uint32_t ib) {
    return ca > cb || (ca == cb && ia < ib);
  };
  uint64_t c = (tid < want) ? pcode[tid] : 0ull;
  uint32_t id = (tid < want) ? pidx[tid] : 0xFFFFFFFFu - (uint32_t)tid;
  if (part) {
    for (int k = 2; k <= 32; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        const uint64_t pc = __shfl_xor_sync(full, c, j);
        const uint32_t pi = __shfl_xor_sync(full, id, j);
        const bool partner_first = before(pc, pi, c, id);
        // lane, not tid: every warp's run ends up in the same (ascending) order
        const bool keep_first = ((lane & j) == 0) == ((lane & k) == 0);
        if (keep_first == partner_first) {
          c = pc;
          id = pi;
        }
      }
    }
  }
  uint64_t* scode = reinterpret_cast<uint64_t*>(whist);  // merge buffer (histograms done)
  uint32_t* sidx = reinterpret_cast<uint32_t*>(scode + kFastPicks);
  for (int w = 32; w < P; w <<= 1) {
    __syncthreads();  // previous readers of the runs are done
    if (part) {
      scode[tid] = c;
      sidx[tid] = id;
    }
    __syncthreads();
    if (part) {
      const int run = tid & ~(w - 1), pos = tid - run;
      const int other = run ^ w;  // partner run [other, other + w)
      int lo = 0, hi = w;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (before(scode[other + mid], sidx[other + mid], c, id)) lo = mid + 1;
        else hi = mid;
      }
      const int dst = (run & ~(2 * w - 1)) + pos + lo;
      pcode[dst] = c;
      pidx[dst] = id;
    }
    __syncthreads();
    if (part) {
      c = pcode[tid];
      id = pidx[tid];
    }
  }
  if (tid < want) {
    selected[id] = 1;
    if (chosen_out) chosen_out[tid] = id;
  }
  __syncthreads();
  return want;
}

// ------------------------------------------------------------ row reductions
// one warp per row: dev = sum (f - c)^2, nrm = sum c^2 (float64)
// returns true (in every lane) when all inputs of the row pair are finite
template <typename T>
__device__ __forceinline__ bool row_dev_nrm(Rows<T> c, int64_t crow, Rows<T> f, int64_t frow,
                                            int64_t heads, int64_t dim, double& dev,
                                            double& nrm) {
  const int lane = threadIdx.x & 31;
  double d_acc = 0.0, n_acc = 0.0;
  bool ok = true;
  for (int64_t h = 0; h < heads; ++h) {
    const T* cp = c.ptr(crow, h);
    const T* fp = f.ptr(frow, h);
    for (int64_t e = lane; e < dim; e += 32) {
      double cv = Elem<T>::to_d(cp[e]);
      double fv = Elem<T>::to_d(fp[e]);
      ok &= isfinite(cv) && isfinite(fv);
      double df = __dsub_rn(fv, cv);
      d_acc = __dadd_rn(d_acc, __dmul_rn(df, df));
      n_acc = __dadd_rn(n_acc, __dmul_rn(cv, cv));
    }
  }
  dev = warp_sum(d_acc);
  nrm = warp_sum(n_acc);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ bool finite(double x) { return isfinite(x); }

// cosine of one head from its dot product and squared norms: the
// reference's amax-scaled unit vectors (wca.py:96-112) reduce to
// dot / (|a| |b|); a zero vector gives 0 there and here
__device__ __forceinline__ double head_cos(double dot, double aa, double bb) {
  if (!(aa > 0.0) || !(bb > 0.0)) return 0.0;
  return fmin(fmax(dot / (sqrt(aa) * sqrt(bb)), -1.0), 1.0);
}

// mean-head cosine of one row pair, result valid in every lane
template <typename T>
__device__ double row_cosine(Rows<T> a, int64_t arow, Rows<T> b, int64_t brow, int64_t heads,
                             int64_t dim) {
  const int lane = threadIdx.x & 31;
  double acc = 0.0;
  for (int64_t h = 0; h < heads; ++h) {
    const T* ap = a.ptr(arow, h);
    const T* bp = b.ptr(brow, h);
    double dot = 0.0, aa = 0.0, bb = 0.0;
    for (int64_t e = lane; e < dim; e += 32) {
      const double x = Elem<T>::to_d(ap[e]), y = Elem<T>::to_d(bp[e]);
      dot = __dadd_rn(dot, __dmul_rn(x, y));
      aa = __dadd_rn(aa, __dmul_rn(x, x));
      bb = __dadd_rn(bb, __dmul_rn(y, y));
    }
    acc += head_cos(warp_sum(dot), warp_sum(aa), warp_sum(bb));
  }
  return acc / (double)heads;
}

// ------------------------------------------------------ 16-byte row vectors
// Rows of 16-bit elements with 16-byte aligned heads: a warp reads a row as
// heads x G8 vectors of 8 elements (G8 = dim / 8 divides 32), lane l taking
// vectors l, l + 32, ...; in every step each aligned group of G8 lanes holds
// one head.
//
// Finiteness of 16-bit inputs is read off the row sums: a sum of squares of
// finite 16-bit values (or of their differences) cannot overflow float64,
// and any infinity or NaN among them makes the sum infinite or NaN.
template <typename T>
__device__ __forceinline__ void widen8(const uint4& u, double (&x)[8]) {
  const T* el = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int k = 0; k < 8; ++k) x[k] = Elem<T>::to_d(el[k]);
}

// whether a 16-bit float's bits hold an infinity or a NaN
template <typename T>
__device__ __forceinline__ bool nonfinite_bits(T y) {
  if constexpr (sizeof(T) == 2) {
    constexpr uint32_t kExp = std::is_same<T, __nv_bfloat16>::value ? 0x7F80u : 0x7C00u;
    return (*reinterpret_cast<const uint16_t*>(&y) & kExp) == kExp;
  } else {
    return !isfinite(Elem<T>::to_d(y));
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, double (&x)[8]) {
  widen8<T>(*reinterpret_cast<const uint4*>(p), x);
}

template <typename T, int G8>
__device__ __forceinline__ bool row_dev_nrm_vec(Rows<T> c, int64_t crow, Rows<T> f, int64_t frow,
                                                int64_t heads, double& dev, double& nrm) {
  const int lane = threadIdx.x & 31;
  double d_acc = 0.0, n_acc = 0.0;
  const int64_t groups = heads * G8;
#pragma unroll 4
  for (int64_t g = lane; g < groups; g += 32) {
    const int64_t h = g / G8;
    const int e = (int)(g % G8) * 8;
    double cv[8], fv[8];
    load8(c.ptr(crow, h) + e, cv);
    load8(f.ptr(frow, h) + e, fv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const double df = __dsub_rn(fv[k], cv[k]);
      d_acc = __dadd_rn(d_acc, __dmul_rn(df, df));
      n_acc = __dadd_rn(n_acc, __dmul_rn(cv[k], cv[k]));
    }
  }
  dev = warp_sum(d_acc);
  nrm = warp_sum(n_acc);
  return isfinite(dev) && isfinite(nrm);  // 16-bit rows: the inputs' finiteness
}

// A row held in registers: IT = heads * G8 / 32 vectors per lane (vector
// g = it * 32 + lane: head g / G8, elements (g % G8) * 8 ..), every load of
// the row issued before any arithmetic, so a warp keeps whole rows in flight.
template <typename T, int G8, int IT>
__device__ __forceinline__ void load_row(Rows<T> x, int64_t row, uint4 (&v)[IT]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int g = it * 32 + lane;
    v[it] = *reinterpret_cast<const uint4*>(x.ptr(row, g / G8) + (g % G8) * 8);
  }
}

// pairwise sum of per-vector partial sums (IT a power of two)
template <int IT>
__device__ __forceinline__ double tree_sum(const double (&p)[IT]) {
  if constexpr (IT == 1) {
    return p[0];
  } else {
    double h[IT / 2];
#pragma unroll
    for (int i = 0; i < IT / 2; ++i) h[i] = __dadd_rn(p[2 * i], p[2 * i + 1]);
    return tree_sum<IT / 2>(h);
  }
}

// dev / nrm of a register-resident row pair: one partial sum per vector (so
// the dependent float64 chains are 8 long), pairwise over the vectors, then
// the butterfly over the lanes (any summation order is within the
// tolerance of the reference's own float64 reduction); true when both sums
// are finite, i.e. all inputs are (16-bit rows)
template <typename T, int IT>
__device__ __forceinline__ bool dev_nrm_regs(const uint4 (&c)[IT], const uint4 (&f)[IT],
                                             double& dev, double& nrm) {
  double dp[IT], np[IT];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    double cv[8], fv[8];
    widen8<T>(c[it], cv);
    widen8<T>(f[it], fv);
    dp[it] = np[it] = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const double df = __dsub_rn(fv[k], cv[k]);
      dp[it] = __dadd_rn(dp[it], __dmul_rn(df, df));
      np[it] = __dadd_rn(np[it], __dmul_rn(cv[k], cv[k]));
    }
  }
  dev = warp_sum(tree_sum<IT>(dp));
  nrm = warp_sum(tree_sum<IT>(np));
  return isfinite(dev) && isfinite(nrm);
}

// the deviation / norm of one row pair on the widest path the layout allows
template <typename T, int G8, int IT>
__device__ __forceinline__ bool row_dev(Rows<T> c, int64_t crow, Rows<T> f, int64_t frow,
                                        int64_t heads, int64_t dim, double& dev, double& nrm) {
  if constexpr (IT > 0) {
    uint4 cv[IT], fv[IT];
    load_row<T, G8, IT>(c, crow, cv);
    load_row<T, G8, IT>(f, frow, fv);
    return dev_nrm_regs<T, IT>(cv, fv, dev, nrm);
  } else if constexpr (G8 > 0) {
    return row_dev_nrm_vec<T, G8>(c, crow, f, frow, heads, dev, nrm);
  } else {
    return row_dev_nrm(c, crow, f, frow, heads, dim, dev, nrm);
  }
}

// per-head dot / squared norms of the G8-lane group, summed into lanes with
// lane % G8 == 0
template <int G8>
__device__ __forceinline__ void group_sum3(double& x, double& y, double& z) {
#pragma unroll
  for (int o = G8 / 2; o > 0; o >>= 1) {
    x += __shfl_xor_sync(0xffffffffu, x, o);
    y += __shfl_xor_sync(0xffffffffu, y, o);
    z += __shfl_xor_sync(0xffffffffu, z, o);
  }
}

template <typename T, int G8>
__device__ double row_cosine_vec(Rows<T> a, int64_t arow, Rows<T> b, int64_t brow,
                                 int64_t heads) {
  const int lane = threadIdx.x & 31;
  double acc = 0.0;
  const int64_t groups = heads * G8;
  for (int64_t g0 = 0; g0 < groups; g0 += 32) {
    const int64_t g = g0 + lane;
    double dot = 0.0, aa = 0.0, bb = 0.0;
    if (g < groups) {
      const int64_t h = g / G8;
      const int e = (int)(g % G8) * 8;
      double x[8], y[8];
      load8(a.ptr(arow, h) + e, x);
      load8(b.ptr(brow, h) + e, y);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        dot = __dadd_rn(dot, __dmul_rn(x[k], y[k]));
        aa = __dadd_rn(aa, __dmul_rn(x[k], x[k]));
        bb = __dadd_rn(bb, __dmul_rn(y[k], y[k]));
      }
    }
    group_sum3<G8>(dot, aa, bb);
    if (g < groups && (lane % G8) == 0) acc += head_cos(dot, aa, bb);
  }
  return warp_sum(acc) / (double)heads;
}

// lane 0 of a row's warp: weight, status bits, outputs; returns the row's
// reused (bit 0) and candidate (bit 1) flags for the counts
__device__ __forceinline__ int dev_epilogue(int64_t r, double dev, double nrm, bool in_ok,
                                            double eps, int clamp, double* dev_out,
                                            double* alpha_out, const uint8_t* reused,
                                            uint8_t* candidate, int32_t* status) {
  const double den = nrm + eps;
  double a = dev / den;
  if (!in_ok) report(status, CS_ST_INPUT_NONFINITE);
  if (!finite(dev) || !finite(den) || !finite(a)) report(status, CS_ST_NONFINITE);
  if (clamp) a = fmin(fmax(a, 0.0), 1.0);
  if (dev_out) dev_out[r] = dev;
  if (alpha_out) alpha_out[r] = a;
  if (!candidate) return 0;
  const bool ru = reused[r] != 0;
  const bool cand = ru && dev > 0.0;
  candidate[r] = cand ? 1 : 0;
  return (ru ? 1 : 0) | (cand ? 2 : 0);
}

// one warp per row; G8 > 0 selects the 16-byte vector path, IT > 0 the
// register-resident rows.  The reused / candidate counts are gathered per
// block and added once per block.
template <typename T, int G8, int IT>
__global__ void __launch_bounds__(256, IT > 0 ? 3 : 1) deviation_kernel(Rows<T> c, const int64_t* __restrict__ crows, Rows<T> f,
                                 int64_t n, int64_t heads, int64_t dim, double eps, int clamp,
                                 double* dev_out, double* alpha_out,
                                 const uint8_t* __restrict__ reused, uint8_t* candidate,
                                 unsigned long long* counts, int32_t* status) {
  __shared__ unsigned long long cnt[2];
  if (threadIdx.x == 0) cnt[0] = cnt[1] = 0ull;
  __syncthreads();
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    double dev, nrm;
    const int64_t crow = crows ? crows[r] : r;
    const bool in_ok = row_dev<T, G8, IT>(c, crow, f, r, heads, dim, dev, nrm);
    if ((threadIdx.x & 31) == 0) {
      const int fl = dev_epilogue(r, dev, nrm, in_ok, eps, clamp, dev_out, alpha_out, reused,
                                  candidate, status);
      if (fl & 1) atomicAdd(&cnt[0], 1ull);
      if (fl & 2) atomicAdd(&cnt[1], 1ull);
    }
  }
  if (candidate) {
    __syncthreads();
    if (threadIdx.x == 0) {
      if (cnt[0]) atomicAdd(&counts[0], cnt[0]);
      if (cnt[1]) atomicAdd(&counts[1], cnt[1]);
    }
  }
}

template <typename T, int G8>
__global__ void cosine_kernel(Rows<T> a, Rows<T> b, const int64_t* __restrict__ brows, int64_t n,
                              int64_t heads, int64_t dim, double* out) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    const int64_t br = brows ? brows[r] : r;
    double c;
    if constexpr (G8 > 0)
      c = row_cosine_vec<T, G8>(a, r, b, br, heads);
    else
      c = row_cosine(a, r, b, br, heads, dim);
    if ((threadIdx.x & 31) == 0) out[r] = c;
  }
}

// Per-row partial sums for a rank that holds `heads` of `heads_total` KV
// heads (KV-head tensor parallelism): dev = sum over its heads and dims of
// (f - c)^2, nrm = sum of c^2, cos = sum over its heads of the head cosine /
// heads_total.  Summed over the ranks these are the squared deviation, the
// norm and the head-mean cosine of all heads (wca.py:55-112).
template <typename T, int G8, int IT>
__global__ void row_sums_kernel(Rows<T> c, const int64_t* __restrict__ crows, Rows<T> f, int64_t n,
                                int64_t heads, int64_t dim, int64_t heads_total, double* dev_out,
                                double* nrm_out, double* cos_out, int32_t* status) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    const int64_t crow = crows ? crows[r] : r;
    double dev = 0.0, nrm = 0.0, cs = 0.0;
    bool in_ok = true;
    if (dev_out || nrm_out)  // the summation of deviation_kernel / update_kernel
      in_ok = row_dev<T, G8, IT>(c, crow, f, r, heads, dim, dev, nrm);
    if (cos_out) {
      if constexpr (G8 > 0)
        cs = row_cosine_vec<T, G8>(f, r, c, crow, heads);
      else
        cs = row_cosine(f, r, c, crow, heads, dim);
      cs = cs * (double)heads / (double)heads_total;
    }
    if ((threadIdx.x & 31) == 0) {
      if (!in_ok) report(status, CS_ST_INPUT_NONFINITE);
      if (!finite(dev) || !finite(nrm)) report(status, CS_ST_NONFINITE);
      if (dev_out) dev_out[r] = dev;
      if (nrm_out) nrm_out[r] = nrm;
      if (cos_out) cos_out[r] = cs;
    }
  }
}

// adaptation weights (and, with `reused`, candidates and their counts) from
// complete row sums: alpha = dev / (nrm + eps), optionally clamped to [0, 1]
// (wca.py:65-93); candidate = reused and dev > 0 (wca.py:152-200)
__global__ void weights_kernel(const double* __restrict__ dev, const double* __restrict__ nrm,
                               int64_t n, double eps, int clamp, const uint8_t* __restrict__ reused,
                               double* alpha_out, uint8_t* candidate, unsigned long long* counts,
                               int32_t* status) {
  __shared__ unsigned long long cnt[2];
  if (threadIdx.x == 0) cnt[0] = cnt[1] = 0ull;
  __syncthreads();
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n;
       r += (int64_t)gridDim.x * blockDim.x) {
    const double den = nrm[r] + eps;
    double a = dev[r] / den;
    if (!finite(dev[r]) || !finite(den) || !finite(a)) report(status, CS_ST_NONFINITE);
    if (clamp) a = fmin(fmax(a, 0.0), 1.0);
    if (alpha_out) alpha_out[r] = a;
    if (candidate) {
      const bool ru = reused[r] != 0;
      const bool cand = ru && dev[r] > 0.0;
      candidate[r] = cand ? 1 : 0;
      if (ru) atomicAdd(&cnt[0], 1ull);
      if (cand) atomicAdd(&cnt[1], 1ull);
    }
  }
  if (candidate) {
    __syncthreads();
    if (threadIdx.x == 0) {
      if (cnt[0]) atomicAdd(&counts[0], cnt[0]);
      if (cnt[1]) atomicAdd(&counts[1], cnt[1]);
    }
  }
}

// 128 threads per update block, three blocks per SM for the
// register-resident rows (their four rows' raw vectors stay live across the
// deviation pass)
constexpr int kUpdThreads = 128;

// fused update of one active row r (cached row indices[r]): weight, blend
// (float64, no contraction), cast, write dense and/or paged records,
// optional cosine.  G8 > 0 selects the 16-byte vector path, IT > 0 the
// register-resident rows: the four rows are loaded once, before any
// arithmetic, and -- when the blend weight is the stored one (previous_layer
// mode) -- the deviation, the blend and the cosine share one pass over them.
template <typename T, int G8, int IT>
__device__ __forceinline__ void update_row(
    Rows<T> ck, Rows<T> cv, Rows<T> fk, Rows<T> fv, int64_t idx, int64_t r, int64_t heads,
    int64_t dim, const double* __restrict__ alpha, const uint8_t* __restrict__ mandatory,
    int same_layer, double eps, int clamp, T* fused_k, T* fused_v, double* next_alpha_out,
    double* used_out, double* cos_out, PagedView pv, int use_paged, int64_t slot,
    int32_t* status) {
  const int lane = threadIdx.x & 31;
  const bool slot_ok = !use_paged || pv.valid(slot);
  if (use_paged && !slot_ok && lane == 0) report(status, CS_ST_SLOT_RANGE);
  const bool man = mandatory[idx] != 0;
  double dev, nrm, w, cs = 0.0;
  bool bad = false;
  // the weight from this row's deviation / norm (wca.py:65-93)
  auto next_weight = [&]() {
    double nx = dev / (nrm + eps);
    if (clamp) nx = fmin(fmax(nx, 0.0), 1.0);
    return nx;
  };
  if constexpr (IT > 0) {  // heads * G8 == 32 * IT: every lane holds IT vectors
    uint4 okr[IT], fkr[IT], ovr[IT], fvr[IT];
    load_row<T, G8, IT>(ck, idx, okr);
    load_row<T, G8, IT>(fk, r, fkr);
    load_row<T, G8, IT>(cv, idx, ovr);
    load_row<T, G8, IT>(fv, r, fvr);
    // the pool has unit element strides on the vector path (vec16): head h
    // element e of a record half is at base + h * hstride + e * sizeof(T)
    char *pk = nullptr, *pvv = nullptr;
    int64_t hstride = 0;
    if (use_paged && slot_ok) pv.record(slot, pk, pvv, hstride);
    double dp[IT], np[IT], cacc = 0.0;  // per-vector partial sums of dev / nrm
    // vector `it` of the four rows: the K blend with its cosine partials (and
    // the deviation sums when `acc`), then the V blend; V's inputs are
    // checked through the fused values
    auto vec = [&](int it, double wv, bool acc) {
      const int g = it * 32 + lane;
      const int64_t h = g / G8;
      const int e = (g % G8) * 8;
      const double wo = __dsub_rn(1.0, wv);
      double dot = 0.0, aa = 0.0, bb = 0.0;
      alignas(16) T y[8];
      if (acc) dp[it] = np[it] = 0.0;
      {
        double o8[8], f8[8];
        widen8<T>(okr[it], o8);
        widen8<T>(fkr[it], f8);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (acc) {
            const double df = __dsub_rn(f8[k], o8[k]);
            dp[it] = __dadd_rn(dp[it], __dmul_rn(df, df));
            np[it] = __dadd_rn(np[it], __dmul_rn(o8[k], o8[k]));
          }
          y[k] = Elem<T>::from_d(__dadd_rn(__dmul_rn(wv, f8[k]), __dmul_rn(wo, o8[k])));
          bad |= nonfinite_bits(y[k]);
          dot = __dadd_rn(dot, __dmul_rn(f8[k], o8[k]));
          aa = __dadd_rn(aa, __dmul_rn(f8[k], f8[k]));
          bb = __dadd_rn(bb, __dmul_rn(o8[k], o8[k]));
        }
        const uint4 uk = *reinterpret_cast<const uint4*>(y);
        if (fused_k) *reinterpret_cast<uint4*>(fused_k + (r * heads + h) * dim + e) = uk;
        if (pk) *reinterpret_cast<uint4*>(pk + h * hstride + e * (int64_t)sizeof(T)) = uk;
      }
      {
        double o8[8], f8[8];
        widen8<T>(ovr[it], o8);
        widen8<T>(fvr[it], f8);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          y[k] = Elem<T>::from_d(__dadd_rn(__dmul_rn(wv, f8[k]), __dmul_rn(wo, o8[k])));
          bad |= nonfinite_bits(y[k]);
        }
        const uint4 uv = *reinterpret_cast<const uint4*>(y);
        if (fused_v) *reinterpret_cast<uint4*>(fused_v + (r * heads + h) * dim + e) = uv;
        if (pvv) *reinterpret_cast<uint4*>(pvv + h * hstride + e * (int64_t)sizeof(T)) = uv;
      }
      if (cos_out) {
        group_sum3<G8>(dot, aa, bb);
        if ((lane % G8) == 0) cacc += head_cos(dot, aa, bb);
      }
    };
    if (!same_layer) {  // the stored weight: one pass
      w = man ? 1.0 : alpha[idx];
#pragma unroll
      for (int it = 0; it < IT; ++it) vec(it, w, true);
      dev = warp_sum(tree_sum<IT>(dp));
      nrm = warp_sum(tree_sum<IT>(np));
    } else {  // this layer's weight: the deviation first
      bad |= !dev_nrm_regs<T, IT>(okr, fkr, dev, nrm);
      w = man ? 1.0 : next_weight();
#pragma unroll
      for (int it = 0; it < IT; ++it) vec(it, w, false);
    }
    bad |= !isfinite(dev) || !isfinite(nrm);  // 16-bit rows: the inputs' finiteness
    if (cos_out) cs = warp_sum(cacc) / (double)heads;
  } else {
    if constexpr (G8 > 0)
      bad = !row_dev_nrm_vec<T, G8>(ck, idx, fk, r, heads, dev, nrm);
    else
      bad = !row_dev_nrm(ck, idx, fk, r, heads, dim, dev, nrm);
    w = man ? 1.0 : (same_layer ? next_weight() : alpha[idx]);
    const double wo = __dsub_rn(1.0, w);
    if constexpr (G8 > 0) {
      // blend K and V, K cosine of fresh vs cached, from one read of the rows
      double cacc = 0.0;
      const int64_t groups = heads * G8;
      for (int64_t g0 = 0; g0 < groups; g0 += 32) {
        const int64_t g = g0 + lane;
        double dot = 0.0, aa = 0.0, bb = 0.0;
        if (g < groups) {
          const int64_t h = g / G8;
          const int e = (int)(g % G8) * 8;
          double ok8[8], fk8[8], ov8[8], fv8[8];
          load8(ck.ptr(idx, h) + e, ok8);
          load8(fk.ptr(r, h) + e, fk8);
          load8(cv.ptr(idx, h) + e, ov8);
          load8(fv.ptr(r, h) + e, fv8);
          alignas(16) T yk[8];
          alignas(16) T yv[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            yk[k] = Elem<T>::from_d(__dadd_rn(__dmul_rn(w, fk8[k]), __dmul_rn(wo, ok8[k])));
            yv[k] = Elem<T>::from_d(__dadd_rn(__dmul_rn(w, fv8[k]), __dmul_rn(wo, ov8[k])));
            bad |= nonfinite_bits(yk[k]) || nonfinite_bits(yv[k]);
            dot = __dadd_rn(dot, __dmul_rn(fk8[k], ok8[k]));
            aa = __dadd_rn(aa, __dmul_rn(fk8[k], fk8[k]));
            bb = __dadd_rn(bb, __dmul_rn(ok8[k], ok8[k]));
          }
          const uint4 uk = *reinterpret_cast<const uint4*>(yk);
          const uint4 uv = *reinterpret_cast<const uint4*>(yv);
          if (fused_k) {
            *reinterpret_cast<uint4*>(fused_k + (r * heads + h) * dim + e) = uk;
            *reinterpret_cast<uint4*>(fused_v + (r * heads + h) * dim + e) = uv;
          }
          if (use_paged && slot_ok) {
            *reinterpret_cast<uint4*>(pv.addr(slot, h, e)) = uk;
            *reinterpret_cast<uint4*>(pv.addr(slot, h, dim + e)) = uv;
          }
        }
        if (cos_out) {
          group_sum3<G8>(dot, aa, bb);
          if (g < groups && (lane % G8) == 0) cacc += head_cos(dot, aa, bb);
        }
      }
      if (cos_out) cs = warp_sum(cacc) / (double)heads;
    } else {
      for (int half = 0; half < 2; ++half) {
        Rows<T> o = half ? cv : ck;
        Rows<T> f = half ? fv : fk;
        T* dst = half ? fused_v : fused_k;
        for (int64_t h = 0; h < heads; ++h) {
          const T* op = o.ptr(idx, h);
          const T* fp = f.ptr(r, h);
          for (int64_t e = lane; e < dim; e += 32) {
            double x = __dadd_rn(__dmul_rn(w, Elem<T>::to_d(fp[e])),
                                 __dmul_rn(wo, Elem<T>::to_d(op[e])));
            T y = Elem<T>::from_d(x);
            bad |= nonfinite_bits(y);
            if (dst) dst[(r * heads + h) * dim + e] = y;
            if (use_paged && slot_ok)
              *reinterpret_cast<T*>(pv.addr(slot, h, half * dim + e)) = y;
          }
        }
      }
      if (cos_out) cs = row_cosine(fk, r, ck, idx, heads, dim);
    }
  }
  const double den = nrm + eps;
  const double nxt = next_weight();
  bad |= !finite(dev) || !finite(den) || !finite(dev / den);
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    if (bad) report(status, CS_ST_NONFINITE);
    if (next_alpha_out) next_alpha_out[r] = nxt;
    if (used_out) used_out[r] = w;
    if (cos_out) cos_out[r] = cs;
  }
}

template <typename T, int G8, int IT>
__global__ void __launch_bounds__(kUpdThreads, IT > 0 ? 2 : 1) update_kernel(Rows<T> ck, Rows<T> cv, Rows<T> fk, Rows<T> fv,
                              const int64_t* __restrict__ indices, int64_t a, int64_t heads,
                              int64_t dim, const double* __restrict__ alpha,
                              const uint8_t* __restrict__ mandatory, int same_layer, double eps,
                              int clamp, T* fused_k, T* fused_v, double* next_alpha_out,
                              double* used_out, double* cos_out, PagedView pv, int use_paged,
                              const int64_t* __restrict__ slots, int32_t* status) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < a;
       r += warps) {
    update_row<T, G8, IT>(ck, cv, fk, fv, indices[r], r, heads, dim, alpha, mandatory,
                          same_layer, eps, clamp, fused_k, fused_v, next_alpha_out, used_out,
                          cos_out, pv, use_paged, use_paged ? slots[r] : 0, status);
  }
}

// ------------------------------------------------------------- select kernels
__global__ void __launch_bounds__(kSelectThreads)
    select_kernel(const double* __restrict__ keys, const uint8_t* __restrict__ available, int64_t n,
                  int64_t slots, uint8_t* selected, int64_t* chosen_out, int64_t* count_out,
                  int32_t* status) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ SelectSmem sm;
  double* stage_key = reinterpret_cast<double*>(dyn);
  int* stage_idx = reinterpret_cast<int*>(dyn + sizeof(double) * kSelectMaxChosen);
  auto avail = [&](int64_t i) { return available[i] != 0; };
  int64_t k = n <= kSortMax
                  ? block_topk_staged(keys, avail, n, slots, selected, chosen_out, sm, dyn)
                  : block_select_topk(keys, avail, n, slots, selected, chosen_out, sm, stage_key,
                                      stage_idx, status);
  if (threadIdx.x == 0 && count_out) *count_out = k;
}

// the commit of one request by the whole block (kSelectThreads threads)
__device__ __forceinline__ void commit_block(
    const int64_t* __restrict__ indices, int64_t a, const double* __restrict__ next_alpha,
    const double* __restrict__ cosv, double thr, int distance_mode, int64_t n, int64_t budget,
    const double* __restrict__ initial, double* alpha, uint8_t* candidate, uint8_t* selected,
    uint8_t* removed, int64_t* removed_out, int64_t* promoted_out, int64_t* counts_out,
    int32_t* status) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ SelectSmem sm;
  __shared__ int removed_count;
  double* stage_key = reinterpret_cast<double*>(dyn);
  int* stage_idx = reinterpret_cast<int*>(dyn + sizeof(double) * kSelectMaxChosen);
  const int tid = threadIdx.x;
  if (tid == 0) removed_count = 0;
  __syncthreads();
  // removal decisions use the selection state before this commit; the
  // indices are sorted, so an ordered compaction lists removals ascending
  for (int64_t base = 0; base < a; base += blockDim.x) {
    int64_t r = base + tid;
    int rm = 0;
    int64_t idx = 0;
    if (r < a) {
      idx = indices[r];
      if (cosv) {
        double m = distance_mode ? 1.0 - cosv[r] : cosv[r];
        rm = (selected[idx] && m < thr) ? 1 : 0;
      }
    }
    int pos = block_inclusive_scan(rm, sm.warp_tot) - rm + removed_count;
    __syncthreads();
    if (r < a) {
      alpha[idx] = next_alpha[r];
      if (rm) {
        selected[idx] = 0;
        candidate[idx] = 0;
        removed[idx] = 1;
        if (removed_out) removed_out[pos] = idx;
      }
    }
    __syncthreads();
    if (tid == blockDim.x - 1) removed_count = pos + rm;
    __syncthreads();
  }
  int local = 0;
  for (int64_t i = tid; i < n; i += blockDim.x) local += selected[i] ? 1 : 0;
  int64_t nsel = block_sum(local, sm.warp_tot);
  int64_t slots = budget - nsel;
  if (slots < 0) slots = 0;
  auto avail = [&](int64_t i) { return candidate[i] && !selected[i] && !removed[i]; };
  // `selected` changes only after the radix passes finish counting
  int64_t k = n <= kSortMax
                  ? block_topk_staged(initial, avail, n, slots, selected, promoted_out, sm, dyn)
                  : block_select_topk(initial, avail, n, slots, selected, promoted_out, sm,
                                      stage_key, stage_idx, status);
  if (tid == 0 && counts_out) {
    counts_out[0] = removed_count;
    counts_out[1] = k;
  }
}

__global__ void __launch_bounds__(kSelectThreads)
    commit_kernel(const int64_t* __restrict__ indices, int64_t a,
                  const double* __restrict__ next_alpha, const double* __restrict__ cosv,
                  double thr, int distance_mode, int64_t n, int64_t budget,
                  const double* __restrict__ initial, double* alpha, uint8_t* candidate,
                  uint8_t* selected, uint8_t* removed, int64_t* removed_out,
                  int64_t* promoted_out, int64_t* counts_out, int32_t* status) {
  commit_block(indices, a, next_alpha, cosv, thr, distance_mode, n, budget, initial, alpha,
               candidate, selected, removed, removed_out, promoted_out, counts_out, status);
}

// ------------------------------------------------------------ batched kernels
// Several requests per launch (the calls of one step): each item holds one
// request's arguments, rows are numbered across the requests (batch_item).
constexpr int kBatch = kBatchItems;

template <typename T>
struct InitItem {
  Rows<T> c, f;
  const uint8_t* reused;
  double* dev;
  double* alpha;
  uint8_t* candidate;
  uint8_t* selected;
  uint8_t* removed;
  unsigned long long* counts;
  int32_t* status;
};

template <typename T>
struct InitBatch {
  InitItem<T> it[kBatch];
  int64_t start[kBatch + 1];
  int count;
};

struct CountsBatch {
  unsigned long long* counts[kBatch];
  int count;
};

__global__ void zero_counts_kernel(const __grid_constant__ CountsBatch b) {
  const int i = threadIdx.x;
  if (i < b.count) b.counts[i][0] = b.counts[i][1] = 0ull;
}

// cs_wca_initialize of every item: one warp per row, the counts gathered
// per block and request
template <typename T, int G8, int IT>
__global__ void __launch_bounds__(256, IT > 0 ? 3 : 1)
    initialize_batch_kernel(const __grid_constant__ InitBatch<T> b, int64_t heads, int64_t dim,
                            double eps, int clamp) {
  __shared__ unsigned long long cnt[kBatch][2];
  for (int i = threadIdx.x; i < 2 * kBatch; i += blockDim.x) cnt[i >> 1][i & 1] = 0ull;
  __syncthreads();
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = b.start[b.count];
  for (int64_t g = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); g < total;
       g += warps) {
    const int i = batch_item(b.start, b.count, g);
    const InitItem<T>& q = b.it[i];
    const int64_t r = g - b.start[i];
    double dev, nrm;
    const bool in_ok = row_dev<T, G8, IT>(q.c, r, q.f, r, heads, dim, dev, nrm);
    if ((threadIdx.x & 31) == 0) {
      if (q.selected) q.selected[r] = 0;
      if (q.removed) q.removed[r] = 0;
      const int fl = dev_epilogue(r, dev, nrm, in_ok, eps, clamp, q.dev, q.alpha, q.reused,
                                  q.candidate, q.status);
      if (fl & 1) atomicAdd(&cnt[i][0], 1ull);
      if (fl & 2) atomicAdd(&cnt[i][1], 1ull);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * b.count; i += blockDim.x) {
    const unsigned long long v = cnt[i >> 1][i & 1];
    if (v) atomicAdd(&b.it[i >> 1].counts[i & 1], v);
  }
}

template <typename T>
struct UpdItem {
  Rows<T> ck, cv, fk, fv;
  const int64_t* indices;
  const double* alpha;
  const uint8_t* mandatory;
  T* fused_k;
  T* fused_v;
  double* next_alpha;
  double* used;
  double* cos;
  const int64_t* slots;
  int32_t* status;
  const int64_t* a_dev;  // or NULL: rows r >= *a_dev are skipped
};

template <typename T>
struct UpdBatch {
  UpdItem<T> it[kBatch];
  int64_t start[kBatch + 1];
  int count;
};
static_assert(sizeof(UpdBatch<double>) <= 32000, "batched update arguments exceed the parameter space");

template <typename T, int G8, int IT>
__global__ void __launch_bounds__(kUpdThreads, IT > 0 ? 3 : 1)
    update_batch_kernel(const __grid_constant__ UpdBatch<T> b, int64_t heads, int64_t dim,
                        int same_layer, double eps, int clamp, PagedView pv, int use_paged) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = b.start[b.count];
  for (int64_t g = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); g < total;
       g += warps) {
    const int i = batch_item(b.start, b.count, g);
    const UpdItem<T>& q = b.it[i];
    const int64_t r = g - b.start[i];
    if (q.a_dev != nullptr && r >= __ldg(q.a_dev)) continue;  // past the device row count
    update_row<T, G8, IT>(q.ck, q.cv, q.fk, q.fv, q.indices[r], r, heads, dim, q.alpha,
                          q.mandatory, same_layer, eps, clamp, q.fused_k, q.fused_v,
                          q.next_alpha, q.used, q.cos, pv, use_paged,
                          use_paged ? q.slots[r] : 0, q.status);
  }
}

struct CommitBatch {
  cs_wca_commit_item it[kBatch];
  int count;
};

// one block per request
__global__ void __launch_bounds__(kSelectThreads)
    commit_batch_kernel(const __grid_constant__ CommitBatch b, double thr, int distance_mode) {
  const cs_wca_commit_item& q = b.it[blockIdx.x];
  int64_t a = q.a;
  if (q.a_dev != nullptr) {  // a row count in device memory, at most a
    const int64_t c = __ldg(q.a_dev);
    a = c < 0 ? 0 : (c < a ? c : a);
  }
  commit_block(q.indices, a, q.next_alpha, q.cos, thr, distance_mode, q.n, q.budget,
               q.initial_dev, q.alpha, q.candidate, q.selected, q.removed, q.removed_out,
               q.promoted_out, q.counts_out, q.status);
}

constexpr size_t kSelectDynSmem = (sizeof(double) + sizeof(int)) * kSelectMaxChosen;

bool select_smem_ready() {
  static bool done = false;
  if (!done) {
    if (cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSelectDynSmem) != cudaSuccess)
      return false;
    if (cudaFuncSetAttribute(commit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSelectDynSmem) != cudaSuccess)
      return false;
    if (cudaFuncSetAttribute(commit_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSelectDynSmem) != cudaSuccess)
      return false;
    done = true;
  }
  return true;
}

int row_grid(int64_t rows, int warps_per_block) {
  int64_t blocks = (rows + warps_per_block - 1) / warps_per_block;
  int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

// vector width of the row kernels: G8 = dim / 8 when the rows are 16-bit
// elements in 16-byte aligned heads (every base and byte stride a multiple
// of 16) and G8 divides 32 with at least 4 lanes per head; 0 otherwise
template <typename T>
int vec_groups(int64_t dim, std::initializer_list<const void*> bases,
               std::initializer_list<int64_t> elem_strides) {
  if (sizeof(T) != 2 || dim % 8) return 0;
  const int64_t g8 = dim / 8;
  if (g8 != 4 && g8 != 8 && g8 != 16 && g8 != 32) return 0;
  for (const void* b : bases)
    if (b != nullptr && (reinterpret_cast<uintptr_t>(b) & 15)) return 0;
  for (int64_t st : elem_strides)
    if ((st * (int64_t)sizeof(T)) % 16) return 0;
  return (int)g8;
}

// call f with std::integral_constant<int, G8> (0 = scalar path)
template <typename T, typename F>
void with_g8(int g8, F&& f) {
  if constexpr (sizeof(T) == 2) {
    switch (g8) {
      case 4: f(std::integral_constant<int, 4>{}); return;
      case 8: f(std::integral_constant<int, 8>{}); return;
      case 16: f(std::integral_constant<int, 16>{}); return;
      case 32: f(std::integral_constant<int, 32>{}); return;
      default: break;
    }
  }
  f(std::integral_constant<int, 0>{});
}

// vectors per lane of a register-resident row: IT = heads * G8 / 32 when it
// is exact and small (1, 2 or 4) and G8 is 8 or 16; 0 otherwise
inline int row_iters(int g8, int64_t heads) {
  if (g8 != 8 && g8 != 16) return 0;
  const int64_t groups = heads * g8;
  if (groups % 32) return 0;
  const int64_t it = groups / 32;
  return (it == 1 || it == 2 || it == 4) ? (int)it : 0;
}

// call f(G8, IT) with std::integral_constant arguments (0, 0: scalar path)
template <typename T, typename F>
void with_vec(int g8, int it, F&& f) {
  using std::integral_constant;
  if constexpr (sizeof(T) == 2) {
    switch (g8 * 8 + it) {
      case 4 * 8: f(integral_constant<int, 4>{}, integral_constant<int, 0>{}); return;
      case 8 * 8: f(integral_constant<int, 8>{}, integral_constant<int, 0>{}); return;
      case 8 * 8 + 1: f(integral_constant<int, 8>{}, integral_constant<int, 1>{}); return;
      case 8 * 8 + 2: f(integral_constant<int, 8>{}, integral_constant<int, 2>{}); return;
      case 8 * 8 + 4: f(integral_constant<int, 8>{}, integral_constant<int, 4>{}); return;
      case 16 * 8: f(integral_constant<int, 16>{}, integral_constant<int, 0>{}); return;
      case 16 * 8 + 1: f(integral_constant<int, 16>{}, integral_constant<int, 1>{}); return;
      case 16 * 8 + 2: f(integral_constant<int, 16>{}, integral_constant<int, 2>{}); return;
      case 16 * 8 + 4: f(integral_constant<int, 16>{}, integral_constant<int, 4>{}); return;
      case 32 * 8: f(integral_constant<int, 32>{}, integral_constant<int, 0>{}); return;
      default: break;
    }
  }
  f(integral_constant<int, 0>{}, integral_constant<int, 0>{});
}

template <typename T>
Rows<T> rows_of(const void* p, int64_t srow, int64_t shead) {
  return Rows<T>{static_cast<const char*>(p), srow * (int64_t)sizeof(T),
                 shead * (int64_t)sizeof(T)};
}

}  // namespace
}  // namespace cs

using namespace cs;

#define CS_DISPATCH_FLOAT(dt, T, ...)                       \
  switch (dt) {                                             \
    case CS_F32: { using T = float; __VA_ARGS__; break; }   \
    case CS_F16: { using T = __half; __VA_ARGS__; break; }  \
    case CS_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; } \
    case CS_F64: { using T = double; __VA_ARGS__; break; }  \
    default: return CS_ERR_INVALID;                         \
  }

extern "C" int cs_wca_deviation(const void* cached, int64_t c_stride_row, int64_t c_stride_head,
                                const int64_t* cached_rows, const void* fresh,
                                int64_t f_stride_row, int64_t f_stride_head, int64_t n,
                                int64_t heads, int64_t dim, int32_t dtype, double epsilon,
                                int32_t clamp, double* dev_out, double* alpha_out,
                                int32_t* status, void* stream) {
  CS_HOST_CHECK(n >= 0 && heads > 0 && dim > 0);
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(cached && fresh);
  const int threads = 256;
  CS_DISPATCH_FLOAT(dtype, T, {
    const int g8 = vec_groups<T>(dim, {cached, fresh},
                                 {c_stride_row, c_stride_head, f_stride_row, f_stride_head});
    with_vec<T>(g8, row_iters(g8, heads), [&](auto G, auto I) {
      deviation_kernel<T, decltype(G)::value, decltype(I)::value>
          <<<row_grid(n, threads / 32), threads, 0, as_stream(stream)>>>(
              rows_of<T>(cached, c_stride_row, c_stride_head), cached_rows,
              rows_of<T>(fresh, f_stride_row, f_stride_head), n, heads, dim, epsilon, clamp,
              dev_out, alpha_out, nullptr, nullptr, nullptr, status);
    });
  });
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_initialize(const void* cached, int64_t c_stride_row, int64_t c_stride_head,
                                 const void* fresh, int64_t f_stride_row, int64_t f_stride_head,
                                 int64_t n, int64_t heads, int64_t dim, int32_t dtype,
                                 const uint8_t* reused, double epsilon, int32_t clamp,
                                 double* dev_out, double* alpha_out, uint8_t* candidate,
                                 uint8_t* selected, uint8_t* removed, int64_t* counts_out,
                                 int32_t* status, void* stream) {
  CS_HOST_CHECK(n >= 0 && heads > 0 && dim > 0 && counts_out && candidate && reused);
  auto s = as_stream(stream);
  if (cudaMemsetAsync(counts_out, 0, 2 * sizeof(int64_t), s) != cudaSuccess) return CS_ERR_CUDA;
  if (selected && n > 0 && cudaMemsetAsync(selected, 0, n, s) != cudaSuccess) return CS_ERR_CUDA;
  if (removed && n > 0 && cudaMemsetAsync(removed, 0, n, s) != cudaSuccess) return CS_ERR_CUDA;
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(cached && fresh);
  const int threads = 256;
  CS_DISPATCH_FLOAT(dtype, T, {
    const int g8 = vec_groups<T>(dim, {cached, fresh},
                                 {c_stride_row, c_stride_head, f_stride_row, f_stride_head});
    with_vec<T>(g8, row_iters(g8, heads), [&](auto G, auto I) {
      deviation_kernel<T, decltype(G)::value, decltype(I)::value>
          <<<row_grid(n, threads / 32), threads, 0, s>>>(
          rows_of<T>(cached, c_stride_row, c_stride_head), nullptr,
          rows_of<T>(fresh, f_stride_row, f_stride_head), n, heads, dim, epsilon, clamp,
          dev_out, alpha_out, reused, candidate,
          reinterpret_cast<unsigned long long*>(counts_out), status);
    });
  });
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_cosine(const void* a, int64_t a_stride_row, int64_t a_stride_head,
                             const void* b, int64_t b_stride_row, int64_t b_stride_head,
                             const int64_t* b_rows, int64_t n, int64_t heads, int64_t dim,
                             int32_t dtype, double epsilon, double* cos_out, int32_t* status,
                             void* stream) {
  (void)status;
  CS_HOST_CHECK(n >= 0 && heads > 0 && dim > 0);
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(a && b && cos_out);
  const int threads = 256;
  (void)epsilon;  // scale-invariant: the reference's max clamp does not change the result
  CS_DISPATCH_FLOAT(dtype, T, {
    const int g8 = vec_groups<T>(dim, {a, b},
                                 {a_stride_row, a_stride_head, b_stride_row, b_stride_head});
    with_g8<T>(g8, [&](auto G) {
      cosine_kernel<T, decltype(G)::value>
          <<<row_grid(n, threads / 32), threads, 0, as_stream(stream)>>>(
              rows_of<T>(a, a_stride_row, a_stride_head),
              rows_of<T>(b, b_stride_row, b_stride_head), b_rows, n, heads, dim, cos_out);
    });
  });
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_row_sums(const void* cached, int64_t c_stride_row, int64_t c_stride_head,
                               const int64_t* cached_rows, const void* fresh,
                               int64_t f_stride_row, int64_t f_stride_head, int64_t n,
                               int64_t heads, int64_t dim, int32_t dtype, int64_t heads_total,
                               double* dev_out, double* nrm_out, double* cos_out,
                               int32_t* status, void* stream) {
  CS_HOST_CHECK(n >= 0 && heads > 0 && dim > 0 && heads_total >= heads);
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(cached && fresh);
  const int threads = 256;
  CS_DISPATCH_FLOAT(dtype, T, {
    const int g8 = vec_groups<T>(dim, {cached, fresh},
                                 {c_stride_row, c_stride_head, f_stride_row, f_stride_head});
    with_vec<T>(g8, row_iters(g8, heads), [&](auto G, auto I) {
      row_sums_kernel<T, decltype(G)::value, decltype(I)::value>
          <<<row_grid(n, threads / 32), threads, 0, as_stream(stream)>>>(
              rows_of<T>(cached, c_stride_row, c_stride_head), cached_rows,
              rows_of<T>(fresh, f_stride_row, f_stride_head), n, heads, dim, heads_total,
              dev_out, nrm_out, cos_out, status);
    });
  });
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_weights(const double* dev, const double* nrm, int64_t n, double epsilon,
                              int32_t clamp, const uint8_t* reused, double* alpha_out,
                              uint8_t* candidate, int64_t* counts_out, int32_t* status,
                              void* stream) {
  CS_HOST_CHECK(n >= 0 && (candidate == nullptr || (reused && counts_out)));
  auto s = as_stream(stream);
  if (candidate && cudaMemsetAsync(counts_out, 0, 2 * sizeof(int64_t), s) != cudaSuccess)
    return CS_ERR_CUDA;
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(dev && nrm);
  const int threads = 256;
  int blocks = (int)((n + threads - 1) / threads);
  blocks = blocks > 1184 ? 1184 : blocks;
  weights_kernel<<<blocks, threads, 0, s>>>(dev, nrm, n, epsilon, clamp, reused, alpha_out,
                                            candidate,
                                            reinterpret_cast<unsigned long long*>(counts_out),
                                            status);
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_select_topk(const double* keys, const uint8_t* available, int64_t n,
                                  int64_t slots, uint8_t* selected, int64_t* chosen_out,
                                  int64_t* count_out, int32_t* status, void* stream) {
  CS_HOST_CHECK(n >= 0 && slots >= 0);
  if (chosen_out != nullptr && (slots < n ? slots : n) > kSelectMaxChosen)
    return CS_ERR_UNSUPPORTED;
  auto s = as_stream(stream);
  if (n == 0) {
    if (count_out && cudaMemsetAsync(count_out, 0, sizeof(int64_t), s) != cudaSuccess)
      return CS_ERR_CUDA;
    return CS_OK;
  }
  CS_HOST_CHECK(keys && available && selected);
  if (!select_smem_ready()) return CS_ERR_CUDA;
  select_kernel<<<1, kSelectThreads, kSelectDynSmem, s>>>(keys, available, n, slots, selected,
                                                          chosen_out, count_out, status);
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_update(const void* cached_k, const void* cached_v, int64_t c_stride_row,
                             int64_t c_stride_head, const void* fresh_k, const void* fresh_v,
                             int64_t f_stride_row, int64_t f_stride_head, const int64_t* indices,
                             int64_t a, int64_t heads, int64_t dim, int32_t dtype,
                             const double* alpha, const uint8_t* mandatory, int32_t same_layer,
                             double epsilon, int32_t clamp, void* fused_k, void* fused_v,
                             double* next_alpha_out, double* used_alpha_out, double* cos_out,
                             const cs_paged_kv* kv, const int64_t* slots, int32_t* status,
                             void* stream) {
  CS_HOST_CHECK(a >= 0 && heads > 0 && dim > 0);
  if (a == 0) return CS_OK;
  CS_HOST_CHECK(cached_k && cached_v && fresh_k && fresh_v && indices && alpha && mandatory);
  CS_HOST_CHECK((fused_k == nullptr) == (fused_v == nullptr));
  PagedView pv{};
  int use_paged = 0;
  if (kv != nullptr) {
    CS_HOST_CHECK(slots && kv->cache && kv->dtype == dtype && kv->head_dim == dim &&
                  kv->kv_heads == heads && kv->block_size > 0);
    pv = PagedView::make(*kv);
    use_paged = 1;
  }
  CS_DISPATCH_FLOAT(dtype, T, {
    int g8 = vec_groups<T>(dim, {cached_k, cached_v, fresh_k, fresh_v, fused_k, fused_v},
                           {c_stride_row, c_stride_head, f_stride_row, f_stride_head});
    if (use_paged && !pv.vec16()) g8 = 0;
    with_vec<T>(g8, row_iters(g8, heads), [&](auto G, auto I) {
      update_kernel<T, decltype(G)::value, decltype(I)::value>
          <<<row_grid(a, kUpdThreads / 32), kUpdThreads, 0, as_stream(stream)>>>(
              rows_of<T>(cached_k, c_stride_row, c_stride_head),
              rows_of<T>(cached_v, c_stride_row, c_stride_head),
              rows_of<T>(fresh_k, f_stride_row, f_stride_head),
              rows_of<T>(fresh_v, f_stride_row, f_stride_head), indices, a, heads, dim, alpha,
              mandatory, same_layer, epsilon, clamp, static_cast<T*>(fused_k),
              static_cast<T*>(fused_v), next_alpha_out, used_alpha_out, cos_out, pv, use_paged,
              slots, status);
    });
  });
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_wca_commit(const int64_t* indices, int64_t a, const double* next_alpha,
                             const double* cos, double threshold, int32_t distance_mode,
                             int64_t n, int64_t budget, const double* initial_dev, double* alpha,
                             uint8_t* candidate, uint8_t* selected, uint8_t* removed,
                             int64_t* removed_out, int64_t* promoted_out, int64_t* counts_out,
                             int32_t* status, void* stream) {
  CS_HOST_CHECK(a >= 0 && n >= 0 && budget >= 0 && counts_out);
  CS_HOST_CHECK(n == 0 || (initial_dev && alpha && candidate && selected && removed));
  CS_HOST_CHECK(a == 0 || (indices && next_alpha));
  if (promoted_out != nullptr && (budget < n ? budget : n) > kSelectMaxChosen)
    return CS_ERR_UNSUPPORTED;
  if (!select_smem_ready()) return CS_ERR_CUDA;
  commit_kernel<<<1, kSelectThreads, kSelectDynSmem, as_stream(stream)>>>(
      indices, a, next_alpha, cos, threshold, distance_mode, n, budget, initial_dev, alpha,
      candidate, selected, removed, removed_out, promoted_out, counts_out, status);
  CS_LAUNCH_CHECK();
  return CS_OK;
}

// ------------------------------------------------------------ batched calls
extern "C" int cs_wca_initialize_batch(const cs_wca_initialize_item* items, int32_t count,
                                       int64_t heads, int64_t dim, int32_t dtype, double epsilon,
                                       int32_t clamp, void* stream) {
  CS_HOST_CHECK(count >= 0 && (count == 0 || items) && heads > 0 && dim > 0);
  for (int32_t i = 0; i < count; ++i) {
    const cs_wca_initialize_item& q = items[i];
    CS_HOST_CHECK(q.n >= 0 && q.counts_out && q.candidate && q.reused);
    CS_HOST_CHECK(q.n == 0 || (q.cached && q.fresh));
  }
  auto s = as_stream(stream);
  CS_DISPATCH_FLOAT(dtype, T, {
    for (int32_t first = 0; first < count; first += kBatch) {
      const int m = count - first < kBatch ? count - first : kBatch;
      CountsBatch z{};
      z.count = m;
      InitBatch<T> b{};  // copied into the kernel's parameter space by the launch
      b.count = m;
      b.start[0] = 0;
      int g8 = -1;
      for (int j = 0; j < m; ++j) {
        const cs_wca_initialize_item& q = items[first + j];
        z.counts[j] = reinterpret_cast<unsigned long long*>(q.counts_out);
        b.it[j] = InitItem<T>{rows_of<T>(q.cached, q.c_stride_row, q.c_stride_head),
                              rows_of<T>(q.fresh, q.f_stride_row, q.f_stride_head),
                              q.reused, q.dev_out, q.alpha_out, q.candidate, q.selected,
                              q.removed, z.counts[j], q.status};
        b.start[j + 1] = b.start[j] + q.n;
        if (q.n == 0) continue;
        const int gj = vec_groups<T>(dim, {q.cached, q.fresh},
                                     {q.c_stride_row, q.c_stride_head, q.f_stride_row,
                                      q.f_stride_head});
        g8 = g8 < 0 ? gj : (g8 == gj ? g8 : 0);
      }
      zero_counts_kernel<<<1, kBatch, 0, s>>>(z);
      CS_LAUNCH_CHECK();
      const int64_t total = b.start[m];
      if (total == 0) continue;
      const int threads = 256;
      with_vec<T>(g8 < 0 ? 0 : g8, row_iters(g8 < 0 ? 0 : g8, heads), [&](auto G, auto I) {
        initialize_batch_kernel<T, decltype(G)::value, decltype(I)::value>
            <<<row_grid(total, threads / 32), threads, 0, s>>>(b, heads, dim, epsilon, clamp);
      });
      CS_LAUNCH_CHECK();
    }
  });
  return CS_OK;
}

extern "C" int cs_wca_update_batch(const cs_wca_update_item* items, int32_t count, int64_t heads,
                                   int64_t dim, int32_t dtype, int32_t same_layer, double epsilon,
                                   int32_t clamp, const cs_paged_kv* kv, void* stream) {
  CS_HOST_CHECK(count >= 0 && (count == 0 || items) && heads > 0 && dim > 0);
  PagedView pv{};
  int use_paged = 0;
  if (kv != nullptr) {
    CS_HOST_CHECK(kv->cache && kv->dtype == dtype && kv->head_dim == dim &&
                  kv->kv_heads == heads && kv->block_size > 0);
    pv = PagedView::make(*kv);
    use_paged = 1;
  }
  for (int32_t i = 0; i < count; ++i) {
    const cs_wca_update_item& q = items[i];
    CS_HOST_CHECK(q.a >= 0);
    if (q.a == 0) continue;
    CS_HOST_CHECK(q.cached_k && q.cached_v && q.fresh_k && q.fresh_v && q.indices && q.alpha &&
                  q.mandatory);
    CS_HOST_CHECK((q.fused_k == nullptr) == (q.fused_v == nullptr));
    CS_HOST_CHECK(!use_paged || q.slots);
  }
  auto s = as_stream(stream);
  CS_DISPATCH_FLOAT(dtype, T, {
    for (int32_t first = 0; first < count; first += kBatch) {
      const int m = count - first < kBatch ? count - first : kBatch;
      UpdBatch<T> b{};  // copied into the kernel's parameter space by the launch
      b.count = m;
      b.start[0] = 0;
      int g8 = -1;
      for (int j = 0; j < m; ++j) {
        const cs_wca_update_item& q = items[first + j];
        b.it[j] = UpdItem<T>{rows_of<T>(q.cached_k, q.c_stride_row, q.c_stride_head),
                             rows_of<T>(q.cached_v, q.c_stride_row, q.c_stride_head),
                             rows_of<T>(q.fresh_k, q.f_stride_row, q.f_stride_head),
                             rows_of<T>(q.fresh_v, q.f_stride_row, q.f_stride_head),
                             q.indices, q.alpha, q.mandatory, static_cast<T*>(q.fused_k),
                             static_cast<T*>(q.fused_v), q.next_alpha_out, q.used_alpha_out,
                             q.cos_out, q.slots, q.status, q.a_dev};
        b.start[j + 1] = b.start[j] + q.a;
        if (q.a == 0) continue;
        int gj = vec_groups<T>(dim, {q.cached_k, q.cached_v, q.fresh_k, q.fresh_v, q.fused_k,
                                     q.fused_v},
                               {q.c_stride_row, q.c_stride_head, q.f_stride_row,
                                q.f_stride_head});
        g8 = g8 < 0 ? gj : (g8 == gj ? g8 : 0);
      }
      const int64_t total = b.start[m];
      if (total == 0) continue;
      if (g8 < 0 || (use_paged && !pv.vec16())) g8 = 0;
      with_vec<T>(g8, row_iters(g8, heads), [&](auto G, auto I) {
        update_batch_kernel<T, decltype(G)::value, decltype(I)::value>
            <<<row_grid(total, kUpdThreads / 32), kUpdThreads, 0, s>>>(
                b, heads, dim, same_layer, epsilon, clamp, pv, use_paged);
      });
      CS_LAUNCH_CHECK();
    }
  });
  return CS_OK;
}

extern "C" int cs_wca_commit_batch(const cs_wca_commit_item* items, int32_t count,
                                   double threshold, int32_t distance_mode, void* stream) {
  CS_HOST_CHECK(count >= 0 && (count == 0 || items));
  for (int32_t i = 0; i < count; ++i) {
    const cs_wca_commit_item& q = items[i];
    CS_HOST_CHECK(q.a >= 0 && q.n >= 0 && q.budget >= 0 && q.counts_out);
    CS_HOST_CHECK(q.n == 0 || (q.initial_dev && q.alpha && q.candidate && q.selected &&
                               q.removed));
    CS_HOST_CHECK(q.a == 0 || (q.indices && q.next_alpha));
    if (q.promoted_out != nullptr && (q.budget < q.n ? q.budget : q.n) > kSelectMaxChosen)
      return CS_ERR_UNSUPPORTED;
  }
  if (count == 0) return CS_OK;
  if (!select_smem_ready()) return CS_ERR_CUDA;
  auto s = as_stream(stream);
  for (int32_t first = 0; first < count; first += kBatch) {
    CommitBatch b{};
    b.count = count - first < kBatch ? count - first : kBatch;
    for (int j = 0; j < b.count; ++j) b.it[j] = items[first + j];
    commit_batch_kernel<<<b.count, kSelectThreads, kSelectDynSmem, s>>>(b, threshold,
                                                                        distance_mode);
    CS_LAUNCH_CHECK();
  }
  return CS_OK;
}

// ------------------------------------------------------------ active rows
// The layer's active rows (WCAState.active_indices, wca.py:194-196:
// nonzero(selected | mandatory), ascending) and, per active row, the
// association flag of runtime.py:448-454 (selected and not mandatory), written
// on the device with the count, so that the next launches of the layer need
// no host read.  One block: a pass takes 1024 rows, a block-wide exclusive
// scan of the active flags gives each row its output index.
namespace cs {
namespace {
constexpr int kActThreads = 1024;
__global__ void __launch_bounds__(kActThreads)
    active_rows_kernel(const uint8_t* __restrict__ selected, const uint8_t* __restrict__ mandatory,
                       int64_t n, int64_t capacity, int64_t* __restrict__ rows_out,
                       uint8_t* __restrict__ sel_out, int64_t* __restrict__ count_out,
                       int32_t* status) {
  __shared__ int wcount[kActThreads / 32];
  __shared__ int woff[kActThreads / 32];
  __shared__ int64_t base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) base = 0;
  __syncthreads();
  for (int64_t j0 = 0; j0 < n; j0 += kActThreads) {
    const int64_t j = j0 + tid;
    const bool sel = j < n && selected[j] != 0;
    const bool man = j < n && mandatory[j] != 0;
    const bool act = sel || man;
    const unsigned bal = __ballot_sync(0xffffffffu, act);
    if (lane == 0) wcount[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the 32 warp counts
      const int c = wcount[lane];
      int x = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      woff[lane] = x - c;
    }
    __syncthreads();
    const int64_t pos = base + woff[warp] + __popc(bal & ((1u << lane) - 1u));
    if (act && pos < capacity) {
      rows_out[pos] = j;
      sel_out[pos] = (sel && !man) ? 1 : 0;
    }
    __syncthreads();
    if (tid == kActThreads - 1) base += woff[warp] + __popc(bal);
    __syncthreads();
  }
  const int64_t total = base;
  const int64_t cnt = total < capacity ? total : capacity;
  for (int64_t q = cnt + tid; q < capacity; q += kActThreads) {  // rows past the count
    rows_out[q] = -1;
    sel_out[q] = 0;
  }
  if (tid == 0) {
    *count_out = cnt;
    if (total > capacity) report(status, CS_ST_SLOT_RANGE);
  }
}
}  // namespace
}  // namespace cs

extern "C" int cs_wca_active_rows(const uint8_t* selected, const uint8_t* mandatory, int64_t n,
                                  int64_t capacity, int64_t* rows_out, uint8_t* sel_out,
                                  int64_t* count_out, int32_t* status, void* stream) {
  if (n < 0 || capacity < 0 || count_out == nullptr) return CS_ERR_INVALID;
  if (n > 0 && (selected == nullptr || mandatory == nullptr)) return CS_ERR_INVALID;
  if (capacity > 0 && (rows_out == nullptr || sel_out == nullptr)) return CS_ERR_INVALID;
  cs::active_rows_kernel<<<1, cs::kActThreads, 0, cs::as_stream(stream)>>>(selected, mandatory, n, capacity,
                                                                rows_out, sel_out, count_out,
                                                                status);
  CS_LAUNCH_CHECK();
  return CS_OK;
}
