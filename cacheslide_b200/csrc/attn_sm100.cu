// Tensor-core CoPE / CCPE prefill for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA computes two 128-row query tiles ("a" and "b"): each is R = 128 / G
// query rows x the G query heads of one KV head (GQA packing: every row of
// both tiles reads the same K/V tiles).  The two tiles alternate on the
// tensor cores: while the softmax warps of one tile work on its scores, the
// MMA warp runs the other tile's PV and next QK.
// Warp roles (416 threads):
//   warps 0-7   softmax, one thread per S row (TMEM lane r of its tile's
//               columns): warps 0-3 tile a, 4-7 tile b.  Per key tile: gates
//               sigmoid(q.k / sqrt(d)), the reverse cumulative count of
//               position.py:295-307 (restarted at chunk boundaries in the
//               chunk-reset mode), the q.E bias interpolated from a per-row
//               table in shared memory, causal / association masks, the tile
//               max, then P = 2^(s - m) packed to 16-bit pairs back into TMEM
//               over the tile's own S columns.  Once a row's count is >=
//               npos-1 all older keys share one bias: only logit, max and
//               exponential remain (saturated tiles, one pass).
//   warps 8-11  producer: both Q tiles, the E table split into bf16 hi + lo,
//               the key metadata of every key tile (fixed keys, chunk
//               boundaries), and the K tile (one stage) and V tiles (two
//               stages) read through the per-key slot table: TMA 64 x 16 tile
//               loads for runs of 16 keys in consecutive rows, tile::gather4
//               for groups of 4 keys, cp.async for the rest, all into the
//               128-byte swizzled UMMA layout.
//   warp 12     MMA issuer (one thread) and TMEM owner: T = Q E (hi + lo) of
//               both tiles, then per key tile QK(a), QK(b), PV(a) once P(a)
//               is ready, QK(a) of the next key tile, PV(b), QK(b) of the
//               next; completions are tracked with tcgen05.commit.
// TMEM (512 columns): S(a) [0,128), S(b) [128,256) (P over their first 64
// columns; T = Q E over their first NP columns at start), O(a) [256,384), O(b)
// [384,512).  Every mbarrier wait is bounded; on expiry the CTA raises
// CS_ST_TIMEOUT, drains its copies and MMAs, frees its TMEM and returns.
#include <cuda.h>
#include <math.h>

#include <cstdlib>
#include <cstring>
#include <numeric>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace cs {

int validate_attn_params(const cs_attn_params* p);

namespace {

constexpr int kThreads = 416;  // 8 softmax + 4 producer + 1 MMA warps
// registers a thread: at launch (13 warps, four on one SM sub-partition:
// 128), then after the split the producer warpgroup gives 64 of them back
// and the two softmax warpgroups take 32 more each; the MMA warp keeps 128
constexpr int kLaunchRegs = 128, kSoftRegs = 160, kProdRegs = 64;
static_assert(256 * kSoftRegs + 128 * kProdRegs + 32 * kLaunchRegs <= kThreads * kLaunchRegs,
              "register split exceeds the CTA's launch allocation");
constexpr int kTileN = 128;  // keys per tile
constexpr int kD = 128;      // head dim of this kernel
// npos up to 64: a float q.E table per row; up to 128: a half table per row
// (the same 32 KB a tile; fp16 keeps 11 significant bits of the log2-domain
// bias, below the bf16 rounding of P that the PV MMA already applies)
constexpr int kMaxNpos = 128;

// Two query tiles per CTA ("a" = 0, "b" = 1), 128 S rows each, one softmax
// thread per row.  Shared memory map (bytes from the 1024-aligned base):
constexpr uint32_t kQ = 0;          // 2 x 32 KB Q tiles   [tile][2 cb][128 rows][128 B]
constexpr uint32_t kK0 = 65536;     // 32 KB  K tile (one stage: freed when both QKs are done)
constexpr uint32_t kV0 = 98304;     // 2 x 32 KB V tiles
constexpr uint32_t kP = 163840;     // 32 / 64 KB  E hi/lo staging for T = Q E at start (NP 64 / 128)
constexpr uint32_t kTab = 163840;   // 2 x 32 KB q.E tables [tile][128 rows][NP] float / half, after T
constexpr uint32_t kMeta = 229376;  // barriers, flags, key metadata

// metadata block (offsets from kMeta)
constexpr uint32_t kBarQ = 0;       // producer + softmax -> MMA: Q tiles + E staged
constexpr uint32_t kBarT = 8;       // MMA -> softmax: both T = Q E done
// A tcgen05.commit tracks the MMAs issued since the thread's previous
// commit, so every barrier below is committed right after the MMAs it stands
// for, and a consumer of several MMA groups waits on each group's barrier.
constexpr uint32_t kBarK = 16;      // producer -> MMA: K tile
constexpr uint32_t kBarV = 32;      // [2 stages] producer -> MMA: V tile
constexpr uint32_t kBarS = 48;      // [2 tiles] MMA -> softmax / producer: QK done
constexpr uint32_t kBarP = 64;      // [2 tiles] softmax -> MMA: P in TMEM (128 arrivals)
constexpr uint32_t kBarTab = 80;    // [2 tiles] softmax -> MMA: table read, S columns free
constexpr uint32_t kBarPV = 96;     // [2 tiles][2 V stages] MMA -> softmax / producer: PV done
constexpr uint32_t kBarEnd = 128;   // MMA drain
constexpr uint32_t kBarMeta = 136;  // [4] producer -> softmax: key metadata of slot it % 4
constexpr uint32_t kTmemSlot = 168; // TMEM base address
constexpr uint32_t kAbort = 172;    // abort flag
constexpr uint32_t kFixMask = 176;  // [4 slots][4 words] key is fixed
constexpr uint32_t kBndMask = 240;  // [4 slots][4 words] key is the last of its chunk
constexpr uint32_t kBndKc = 304;    // [4 slots][4 chunks] int: chunk id of the newest boundary
constexpr uint32_t kRedN = 368;     // [8] int64: per-warp key needs of the CTA's rows
// Key tiles a CTA can skip.  When every row of the CTA is a selected row of
// the association policy (it sees only non-fixed keys and itself), a key tile
// is needed only if it holds a key some row sees, or a gate that feeds the
// count of such a key; the others are neither loaded nor computed.
constexpr uint32_t kAllSel = 432;   // [8] int: per warp, every valid query row is selected
constexpr int kMaxMapTiles = 512;   // tile map bound (64K keys); more keys: no skipping
constexpr int kMapWords = kMaxMapTiles / 32;
constexpr uint32_t kNeed = 464;     // [16] words: key tile t is needed (bit t)
constexpr uint32_t kNfTile = 528;   // [16] words: key tile t holds a non-fixed key
constexpr uint32_t kChunkFl = 592;  // [0] chunk ids unusable (out of range / decreasing),
                                    // [1..2] 64-bit mask: chunk holds a non-fixed key
constexpr int kMaxMapChunks = 64;
constexpr uint32_t kChunkS = 608;   // [64] int: first key of chunk c
constexpr uint32_t kChunkE = 864;   // [64] int: last key of chunk c
constexpr uint32_t kSlotTile = 1120; // [4 slots] int: key tile of the slot's step
constexpr uint32_t kChunkF = 1136;  // [64] int: first non-fixed key of chunk c
constexpr uint32_t kMetaBytes = kChunkF + 4 * kMaxMapChunks;
constexpr uint32_t kSmemBytes = kMeta + kMetaBytes;  // 230,768 B (limit 232,448)

// TMEM columns: S of each tile (P packed over its first 64 columns), O of
// each tile; T = Q E lands in the first NP S columns of its tile at start
constexpr uint32_t kColS = 0, kColO = 256;  // + 128 * tile
// named barrier 1: the 128 producer threads
// tile::gather4: rows r0..r3 of a 2-D tensor map, 64 elements from column x,
// into 4 consecutive 128-byte rows at dst (the map's 128-byte swizzle applies)
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int x, int r0,
                                            int r1, int r2, int r3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(bar)
      : "memory");
}
// barrier that also ANDs a flag over its participants: every participant
// leaves with the same answer, so exits from loops stay collective and no
// partner is left waiting at a later barrier
__device__ __forceinline__ bool named_and(uint32_t id, uint32_t count, bool v) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)v), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}
// floor of a nonnegative float below 2^22 with plain FP adds (round-down
// add of 1.5 * 2^23 leaves the integer part in the low mantissa bits)
__device__ __forceinline__ float floor_pos(float x, int& i) {
  const float t = __fadd_rd(x, 12582912.0f);
  i = __float_as_int(t) - 0x4B400000;
  return t - 12582912.0f;
}

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct Pack2<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
// packed pair -> (lo, hi)
__device__ __forceinline__ float2 unpack2(uint32_t w, __nv_bfloat16) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 unpack2(uint32_t w, __half) {
  return make_float2(__half2float(__ushort_as_half((unsigned short)(w & 0xffffu))),
                     __half2float(__ushort_as_half((unsigned short)(w >> 16))));
}

struct Args {
  // K/V row maps of the TMA path (2-D: row x element, 128-byte swizzle):
  // [0] primary K, [1] primary V, [2] sidecar K, [3] sidecar V with 64 x 1
  // boxes for tile::gather4, and [4..7] the same maps with 64 x 16 boxes for
  // runs of 16 keys in consecutive rows.  The primary maps are the paged cache
  // (K and V in one row, V from element vx0) or the dense K and V tensors.
  CUtensorMap tm[8];
  cs_attn_params p;
  PagedView pv;
  int G, R, fmt;  // heads per KV head, rows per tile, 0 = f16 / 1 = bf16
  int pairs_per_head;  // query-tile pairs (one CTA each) per KV head
  int bs_shift;   // log2(block size) when it is a power of two, else -1
  int tma;        // 1: K/V tiles by TMA gather4 (per-row cp.async otherwise)
  int vx0;        // first V element of a primary V map row
  int64_t nrb, nrh, nro;       // paged slot (b, o), head g -> map row b*nrb + g*nrh + o*nro
  int64_t srr, srh;            // sidecar row r, head g -> map row r*srr + g*srh
  int64_t krt, krh, vrt, vrh;  // dense key j, head g -> K row j*krt + g*krh, V row j*vrt + g*vrh
};

// K row address of key j for KV head g (0 = no row: zero fill); bit 0 tags a
// sidecar row, whose V lives at the same offset in side_v.  rk / rv receive the
// row indices of the key's K and V in the tensor maps of the TMA path.
template <typename T>
__device__ __forceinline__ uint64_t key_src(const Args& a, int64_t j, int g, int32_t& rk,
                                            int32_t& rv) {
  const cs_attn_params& p = a.p;
  rk = rv = 0;
  if (j >= p.nk) return 0;
  if (p.kv_slots) {
    const int64_t s = p.kv_slots[j];
    const PagedView& pv = a.pv;
    if (!pv.valid(s)) return 0;
    if (s < pv.native_total) {
      int64_t b, o;
      if (a.bs_shift >= 0) {
        b = s >> a.bs_shift;
        o = s - (b << a.bs_shift);
      } else {
        b = s / pv.bs;
        o = s - b * pv.bs;
      }
      rk = rv = (int32_t)(b * a.nrb + g * a.nrh + o * a.nro);
      return reinterpret_cast<uint64_t>(pv.cache + b * pv.sb + g * pv.sh + o * pv.so);
    }
    const int64_t r = s - pv.native_total;
    rk = rv = (int32_t)(r * a.srr + g * a.srh);
    return reinterpret_cast<uint64_t>(pv.side_k + r * pv.ssr + g * pv.ssh) | 1ull;
  }
  rk = (int32_t)(j * a.krt + g * a.krh);
  rv = (int32_t)(j * a.vrt + g * a.vrh);
  return reinterpret_cast<uint64_t>(static_cast<const char*>(p.k) +
                                    (j * p.k_stride_tok + (int64_t)g * p.k_stride_head) *
                                        (int64_t)sizeof(T));
}

template <typename T>
__device__ __forceinline__ const char* value_row_addr(const Args& a, uint64_t kaddr, int64_t j,
                                                      int g) {
  const cs_attn_params& p = a.p;
  if (p.kv_slots) {
    if (kaddr & 1ull) return a.pv.side_v + ((kaddr & ~1ull) - reinterpret_cast<uint64_t>(a.pv.side_k));
    return reinterpret_cast<const char*>(kaddr) + kD * a.pv.se;
  }
  return static_cast<const char*>(p.v) +
         (j * p.v_stride_tok + (int64_t)g * p.v_stride_head) * (int64_t)sizeof(T);
}

// E^T split into bf16/f16 hi + lo in the swizzled B-operand layout of
// T = Q E (row = position p, K = dimension), shared by the 384 producer and
// softmax threads (`t` = 0..383).  When E's positions are contiguous and
// 16-byte aligned a thread takes 4 positions x 8 dimensions: eight float4
// loads, then one 16-byte shared store per position for hi and for lo.
// Otherwise one element per step, all of a thread's loads issued before its
// stores (the stores could alias the loads as far as the compiler knows).
template <typename T, int NP>
__device__ __forceinline__ void stage_e_split(uint8_t* smem, const cs_attn_params& p, int t) {
  const float* E = static_cast<const float*>(p.E);
  constexpr uint32_t kLo = NP * 256;  // lo half after the NP rows x 256 B of hi
  const bool vec = p.e_stride_p == 1 && p.npos % 4 == 0 && p.e_stride_d % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(E) & 15) == 0;
  if (vec) {
    constexpr int kUnits = (NP / 4) * (kD / 8);  // 256 or 512 units of 4 x 8
#pragma unroll 1
    for (int u = t; u < kUnits; u += 384) {
      const int p0 = (u % (NP / 4)) * 4, d0 = (u / (NP / 4)) * 8;
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = p0 < p.npos
                   ? __ldg(reinterpret_cast<const float4*>(E + (int64_t)(d0 + j) * p.e_stride_d + p0))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          const float e0 = q == 0 ? v[j].x : q == 1 ? v[j].y : q == 2 ? v[j].z : v[j].w;
          const float e1 = q == 0 ? v[j + 1].x : q == 1 ? v[j + 1].y : q == 2 ? v[j + 1].z : v[j + 1].w;
          const float h0 = Elem<T>::to_f(Elem<T>::from_f(e0)), h1 = Elem<T>::to_f(Elem<T>::from_f(e1));
          hw[j / 2] = Pack2<T>::pack(h0, h1);
          lw[j / 2] = Pack2<T>::pack(e0 - h0, e1 - h1);
        }
        const uint32_t off = sw128(p0 + q, d0 >> 3, NP);
        *reinterpret_cast<uint4*>(smem + kP + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(smem + kP + kLo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }
    return;
  }
  // general strides: groups of 8 elements a thread, loads before stores
  constexpr int kN = NP * kD, kThr = 384;
#pragma unroll 1
  for (int base = 0; base < kN; base += 8 * kThr) {
    float ev[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = base + u * kThr + t;
      const int dd = idx / NP, pp = idx - dd * NP;  // consecutive threads: consecutive p
      ev[u] = idx < kN && pp < p.npos
                  ? __ldg(E + (int64_t)dd * p.e_stride_d + (int64_t)pp * p.e_stride_p)
                  : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = base + u * kThr + t;
      if (idx >= kN) break;
      const int dd = idx / NP, pp = idx - dd * NP;
      const T hi = Elem<T>::from_f(ev[u]);
      const T lo = Elem<T>::from_f(ev[u] - Elem<T>::to_f(hi));
      const uint32_t off = sw128(pp, dd >> 3, NP) + (dd & 7) * 2;
      *reinterpret_cast<T*>(smem + kP + off) = hi;
      *reinterpret_cast<T*>(smem + kP + kLo + off) = lo;
    }
  }
}

// Requests of one batched launch (cs_cope_attn_prefill_batch): same head
// layout and dtype, each with its own inputs, positions, slots and maps.
constexpr int kMaxPrefillBatch = 8;
struct BatchArgs {
  Args r[kMaxPrefillBatch];
  int count, hkv, max_pairs;
};
static_assert(sizeof(BatchArgs) <= 32000, "batched prefill arguments exceed the parameter space");

// one CTA: query-tile pair `pair` of KV head g of request a; NP = 64 or 128
// bounds npos (the q.E table's width)
template <typename T, int NP, bool TBL>
__device__ __forceinline__ void prefill_cta(const Args& a, int g, int pair);

template <typename T, int NP, bool TBL>
__global__ void __launch_bounds__(kThreads, 1) cope_prefill_sm100(const __grid_constant__ Args a) {
  // the heaviest (latest) pairs of all KV heads are launched first, so the
  // light ones fill the tail of the grid
  prefill_cta<T, NP, TBL>(a, blockIdx.x % a.p.hkv, a.pairs_per_head - 1 - blockIdx.x / a.p.hkv);
}

// all requests of a step in one grid, heaviest pairs of every request first
// (pair rank j from the top, then request, then KV head); a request with
// fewer pairs leaves its CTAs of the lowest ranks empty
template <typename T, int NP, bool TBL>
__global__ void __launch_bounds__(kThreads, 1)
    cope_prefill_sm100_batch(const __grid_constant__ BatchArgs b) {
  const int per_rank = b.count * b.hkv;
  const int j = blockIdx.x / per_rank, ri = (blockIdx.x / b.hkv) % b.count;
  const Args& a = b.r[ri];
  const int pair = a.pairs_per_head - 1 - j;
  if (pair < 0) return;
  prefill_cta<T, NP, TBL>(a, blockIdx.x % b.hkv, pair);
}

// TBL: the canonical-table mode (CanonicalPositionPolicy, attention.py:
// 32-57): a row with a table row (q_row >= 0) takes, at every key with a
// table column (k_ord >= 0), the table's position instead of its count, and
// with `strict` checks the combined path (validate_contextual_path,
// position.py:28-114); such rows always take the contextual path.
template <typename T, int NP, bool TBL>
__device__ __forceinline__ void prefill_cta(const Args& a, const int g, const int pair) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const cs_attn_params& p = a.p;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (sbase & 1023) {  // the UMMA swizzle atoms need a 1024-byte aligned base
    if (tid == 0) report(p.status, CS_ST_TIMEOUT);
    return;
  }
  uint8_t* meta = smem + kMeta;
  volatile int* abort = reinterpret_cast<volatile int*>(meta + kAbort);
  const uint32_t mb = sbase + kMeta;

  // the CTA's two query tiles: query rows i0 .. i0 + 2R - 1 of KV head g (R
  // rows x G heads per tile)
  const int G = a.G, R = a.R;
  const int64_t i0 = (int64_t)pair * 2 * R;
  const float top = (float)(p.npos - 1);
  // live query rows: nq, or a count in device memory (at most nq); a CTA
  // whose rows all lie past it leaves at once (every thread reads the same
  // value, so the exit is uniform and comes before any barrier or TMEM use)
  int64_t nq = p.nq;
  if (p.nq_dev != nullptr) {
    const int64_t c = __ldg(p.nq_dev);
    nq = c < 0 ? 0 : (c < nq ? c : nq);
  }
  if (i0 >= nq) return;

  if (tid == 0) {
    mbar_init(mb + kBarQ, 384);  // Q copies (producer) + E split (producer and softmax)
    mbar_init(mb + kBarT, 1);
    mbar_init(mb + kBarK, 128);  // one copy-completion arrival per producer thread
    for (int s = 0; s < 2; ++s) {
      mbar_init(mb + kBarV + 8 * s, 128);
      mbar_init(mb + kBarS + 8 * s, 1);
      mbar_init(mb + kBarP + 8 * s, 128);  // the 128 rows of the tile
      mbar_init(mb + kBarTab + 8 * s, 128);
      mbar_init(mb + kBarPV + 16 * s, 1);
      mbar_init(mb + kBarPV + 16 * s + 8, 1);
    }
    for (int s = 0; s < 4; ++s) mbar_init(mb + kBarMeta + 8 * s, 128);
    mbar_init(mb + kBarEnd, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp < 8) {  // keys needed by the furthest row of the two tiles: one row per thread
    int64_t n = 0;
    bool sel = true;
    if (tid < 2 * R && i0 + tid < nq) {
      const int64_t qp = p.qpos[i0 + tid];
      n = qp + 1 < p.nk ? qp + 1 : p.nk;
      sel = p.q_selected != nullptr && p.q_selected[i0 + tid] != 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int64_t m = __shfl_xor_sync(0xffffffffu, n, o);
      n = m > n ? m : n;
    }
    sel = __all_sync(0xffffffffu, sel);
    if (lane == 0) {
      reinterpret_cast<int64_t*>(meta + kRedN)[warp] = n;
      reinterpret_cast<int*>(meta + kAllSel)[warp] = sel ? 1 : 0;
    }
  } else if (warp == 12) {  // empty tile and chunk maps (filled after the first barrier)
    uint32_t* w = reinterpret_cast<uint32_t*>(meta + kNeed);
    w[lane] = 0u;  // kNeed and kNfTile: 32 consecutive words
    if (lane < 4) reinterpret_cast<uint32_t*>(meta + kChunkFl)[lane] = 0u;
    int* cs = reinterpret_cast<int*>(meta + kChunkS);
    int* ce = reinterpret_cast<int*>(meta + kChunkE);
    int* cf = reinterpret_cast<int*>(meta + kChunkF);
    cs[lane] = cs[32 + lane] = 0x7fffffff;
    cf[lane] = cf[32 + lane] = 0x7fffffff;
    ce[lane] = ce[32 + lane] = -1;
  }
  // the Q tiles and the E table need nothing from the set-up above: their
  // copies start before the first barrier (the arrivals on kBarQ come after
  // it, once the barrier is initialised)
  if (warp >= 8 && warp < 12) {
    // Q: S row r of tile qt = query row i0 + qt R + r / G, head g G + r % G
    // (the G heads of a query row are adjacent, so a warp's 32 rows span
    // 32 / G query positions: the rows of a warp saturate their counts at
    // nearby keys); lane l of warp w resolves rows 32(w-8) + l of both
    // tiles, then the warp copies its 2 x 32 rows two at a time (16 lanes x
    // 16 bytes per row)
    const int pt = tid - 256;
    const char* qrow[2];
#pragma unroll
    for (int qt = 0; qt < 2; ++qt) {
      const int64_t i = i0 + qt * R + pt / G;
      const int h = g * G + pt % G;
      qrow[qt] = i < nq ? static_cast<const char*>(p.q) +
                                (i * p.q_stride_tok + (int64_t)h * p.q_stride_head) *
                                    (int64_t)sizeof(T)
                          : nullptr;
    }
#pragma unroll
    for (int qt = 0; qt < 2; ++qt) {
#pragma unroll
      for (int it = 0; it < 16; ++it) {
        const int rl = 2 * it + (lane >> 4), c16 = lane & 15;
        const char* src = reinterpret_cast<const char*>(
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(qrow[qt]), rl));
        cp_async16(sbase + kQ + qt * 32768 + sw128((warp - 8) * 32 + rl, c16, 128),
                   src ? src + c16 * 16 : static_cast<const char*>(p.q), src != nullptr);
      }
    }
  }
  if (warp < 12) stage_e_split<T, NP>(smem, p, tid);
  if (warp == 12) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     mb + kTmemSlot),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(meta + kTmemSlot);
  int64_t nneed = 0;
  for (int w = 0; w < 8; ++w) {
    const int64_t n = reinterpret_cast<const volatile int64_t*>(meta + kRedN)[w];
    nneed = n > nneed ? n : nneed;
  }
  const int ntile = (int)((nneed + kTileN - 1) / kTileN);
  // ---------------------------------------------------------- key tile map
  // Only when every query row of the CTA is a selected row (association
  // policy, attention.py:61-72): such a row sees the non-fixed keys and its
  // own key.  The count of a seen key j (position.py:295-307) sums the gates
  // of keys j .. qp; in the chunk-reset mode it restarts at the end of the
  // first chunk at or after j's that carries an offset for the row.  A key
  // tile is needed when it holds a seen key or such a gate; the others are
  // hidden from every row and change no count a row uses.  (Strict path
  // validation checks every causal key, so it keeps every tile.)
  bool use_map = false;
  // per S row (softmax threads): the newest key whose gate feeds the count of
  // a key the row sees other than its own; above it (the row's own key
  // aside) no gate matters to the row (set for rows of a tile-map CTA)
  int64_t chain_hi = INT64_MAX;
  {
    bool allsel = p.q_selected != nullptr && p.k_fixed != nullptr && !(TBL && p.strict != 0);
    for (int w = 0; w < 8; ++w) allsel = allsel && reinterpret_cast<const volatile int*>(meta + kAllSel)[w] != 0;
    use_map = allsel && ntile > 0 && ntile <= kMaxMapTiles;
  }
  if (use_map) {
    uint32_t* need = reinterpret_cast<uint32_t*>(meta + kNeed);
    uint32_t* nft = reinterpret_cast<uint32_t*>(meta + kNfTile);
    uint32_t* cfl = reinterpret_cast<uint32_t*>(meta + kChunkFl);
    int* cs = reinterpret_cast<int*>(meta + kChunkS);
    int* ce = reinterpret_cast<int*>(meta + kChunkE);
    int* cf = reinterpret_cast<int*>(meta + kChunkF);
    const bool chunked = p.pos_mode == CS_POS_CHUNK;
    // keys 0 .. nneed-1: tiles and chunks holding a non-fixed key, chunk
    // ranges.  A thread takes 16 consecutive keys a pass (one 16-byte load of
    // the fixed flags, four of the chunk ids when aligned), so the loads of
    // its keys are in flight together
    const bool vfix = (reinterpret_cast<uintptr_t>(p.k_fixed) & 15) == 0;
    const bool vkc = chunked && (reinterpret_cast<uintptr_t>(p.key_chunk) & 15) == 0;
#pragma unroll 1
    for (int64_t j0 = (int64_t)tid * 16; j0 < nneed; j0 += (int64_t)kThreads * 16) {
      const bool whole = j0 + 16 <= nneed;
      uint32_t fw[4];  // fixed flags, 4 keys a word
      int kc[16];
      if (whole && vfix) {
        const uint4 f4 = __ldg(reinterpret_cast<const uint4*>(p.k_fixed + j0));
        fw[0] = f4.x, fw[1] = f4.y, fw[2] = f4.z, fw[3] = f4.w;
      } else {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          uint32_t x = 0u;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int64_t j = j0 + 4 * w + b;
            x |= (uint32_t)(j < nneed ? p.k_fixed[j] : 1) << (8 * b);
          }
          fw[w] = x;
        }
      }
      int kprev = -1, knext = -1;
      if (chunked) {
        if (whole && vkc) {
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int4 c4 = __ldg(reinterpret_cast<const int4*>(p.key_chunk + j0) + w);
            kc[4 * w] = c4.x, kc[4 * w + 1] = c4.y, kc[4 * w + 2] = c4.z, kc[4 * w + 3] = c4.w;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) kc[k] = j0 + k < nneed ? p.key_chunk[j0 + k] : -1;
        }
        kprev = j0 > 0 ? p.key_chunk[j0 - 1] : -1;
        knext = j0 + 16 < nneed ? p.key_chunk[j0 + 16] : -1;
      }
      bool anynf = false;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int64_t j = j0 + k;
        if (j >= nneed) break;
        const bool nf = ((fw[k >> 2] >> (8 * (k & 3))) & 0xffu) == 0u;
        anynf |= nf;
        if (!chunked) continue;
        const int c = kc[k];
        if (c < 0 || c >= kMaxMapChunks) {
          cfl[0] = 1u;
          continue;
        }
        const int kp = k > 0 ? kc[k - 1] : kprev;
        const int kn = k < 15 ? (j + 1 < nneed ? kc[k + 1] : -1) : knext;
        if (kp > c) cfl[0] = 1u;
        if (kp != c) cs[c] = (int)j;
        if (kn != c) ce[c] = (int)j;
        if (nf) {
          atomicOr(&cfl[1 + (c >> 5)], 1u << (c & 31));
          atomicMin(&cf[c], (int)j);
        }
      }
      // the 16 keys lie in one key tile
      if (anynf) atomicOr(&nft[(int)(j0 >> 12)], 1u << (int)((j0 >> 7) & 31));
    }
    __syncthreads();
    if (warp < 8) {  // one S row per thread, as in the softmax role below
      const int r = (warp & 3) * 32 + lane;
      const int64_t i = i0 + (warp >> 2) * R + r / G;
      const int h = g * G + r % G;
      if (i < nq) {
        const int64_t qp = p.qpos[i];
        const int64_t nl = qp + 1 < p.nk ? qp + 1 : p.nk;
        auto mark = [&](int t0, int t1) {  // tiles t0 .. t1
          for (int w = t0 >> 5; w <= (t1 >> 5); ++w) {
            const int lo = w * 32 > t0 ? 0 : t0 - w * 32;
            const int hi = w * 32 + 31 < t1 ? 31 : t1 - w * 32;
            const uint32_t bits = (hi == 31 ? ~0u : ((2u << hi) - 1u)) & ~((1u << lo) - 1u);
            atomicOr(&need[w], bits);
          }
        };
        if (nl > 0) {
          const int tq = (int)((nl - 1) >> 7);
          mark(tq, tq);  // the row's own key
          if (chunked && cfl[0] == 0u) {
            const int qc = p.key_chunk[nl - 1];
            const float* off = p.chunk_off + (int64_t)h * p.co_stride_h + i * p.co_stride_q;
            const uint64_t nfc = (uint64_t)cfl[1] | ((uint64_t)cfl[2] << 32);
            bool live = false, stop = false;
            int64_t hi = -1;
            // the row's offsets eight chunks at a time (loads in flight together)
            for (int c8 = 0; !stop && c8 <= qc && c8 < kMaxMapChunks; c8 += 8) {
              float o8[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) o8[k] = c8 + k < qc ? off[c8 + k] : -1.f;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const int c = c8 + k;
                if (c > qc || c >= kMaxMapChunks) break;
                if (ce[c] < 0) continue;  // no key of chunk c below nneed
                if (cs[c] >= nl) {
                  stop = true;
                  break;
                }
                // a gate chain coming up from an older chunk needs all of chunk
                // c; one that starts here needs it from its first seen key on
                const bool from_first = !live && ((nfc >> c) & 1ull) && cf[c] < nl;
                if (live || from_first) {
                  const int64_t e = ce[c] < nl - 1 ? ce[c] : nl - 1;
                  mark((live ? cs[c] : cf[c]) >> 7, (int)(e >> 7));
                  live = true;
                  hi = e > hi ? e : hi;
                }
                if (c < qc && o8[k] >= 0.f) live = false;
              }
            }
            chain_hi = hi;
          } else {
            int first = -1;
            for (int w = 0; w < kMapWords && first < 0; ++w)
              if (nft[w]) first = w * 32 + __ffs(nft[w]) - 1;
            if (first >= 0 && first < tq) mark(first, tq);
          }
        }
      }
    }
    __syncthreads();
  }
  // steps: the needed key tiles, newest first
  const uint32_t* needmap = reinterpret_cast<const uint32_t*>(meta + kNeed);
  int nlist = ntile;
  if (use_map) {
    nlist = 0;
    for (int w = 0; w < kMapWords; ++w) nlist += __popc(needmap[w]);
  }


  if (warp >= 8 && warp < 12) {
    // ================================================================ producer
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProdRegs));
    const int pt = tid - 256;  // 0..127
    cp_async_wait_all();
    fence_async_smem();
    mbar_arrive(mb + kBarQ);

    const bool tma = a.tma != 0;
    const unsigned kAll = 0xffffffffu;
    const int wrow0 = 32 * (warp - 8);  // first tile row (key) of this warp
    // source and metadata of key key0 + pt, read one tile ahead so that their
    // global loads overlap the stage waits
    uint64_t ka = 0;
    int32_t rk = 0, rv = 0;
    bool fixed = false, bnd = false;
    int kcj = -1;
    bool slot_bad = false;  // a key some row sees has no valid slot (read as zeros)
    const int64_t nmax = nneed;
    // key tile of the step load_key prepares (newest first, needed tiles only)
    int ktile = ntile;
    auto load_key = [&]() {
      if (use_map) {
        int w = (ktile - 1) >> 5;
        const int b = (ktile - 1) & 31;
        uint32_t m = needmap[w] & (b == 31 ? ~0u : ((2u << b) - 1u));
        while (m == 0u && w > 0) m = needmap[--w];
        ktile = w * 32 + 31 - __clz(m);  // nlist bounds the steps: a bit is left
      } else {
        --ktile;
      }
      const int64_t j = (int64_t)ktile * kTileN + pt;

      const bool in = j < p.nk;
      // keys past the end: zero rows by cp.async; the TMA path repeats the
      // last key's row (finite data, and its P column is zero)
      ka = key_src<T>(a, tma && !in ? p.nk - 1 : j, g, rk, rv);
      slot_bad |= j < nmax && ka == 0;
      fixed = in && p.k_fixed != nullptr && p.k_fixed[j] != 0;
      kcj = in && p.pos_mode == CS_POS_CHUNK ? p.key_chunk[j] : -1;
      bnd = kcj >= 0 && (j + 1 < p.nk) && p.key_chunk[j + 1] != kcj;
    };
    // what the V copy of a tile needs from its K step
    struct VSrc {
      uint64_t ka;
      int64_t key0;
      int rv, v1, v2, v3, grp, run;
      uint32_t tx;
    };
    // publish the key metadata of tile it2 (slot it2 % 4) and start its K copy
    auto issue_k = [&](int it2, VSrc& vs) {
      const int slot = it2 & 3;
      const int64_t key0 = (int64_t)ktile * kTileN;
      {
        const unsigned fm = __ballot_sync(kAll, fixed);
        const unsigned bm = __ballot_sync(kAll, bnd);
        // chunk id of the newest boundary of these 32 keys (-1: none)
        const int kc_top = __shfl_sync(kAll, kcj, bm ? 31 - __clz(bm) : 0);
        if (pt == 0) reinterpret_cast<int*>(meta + kSlotTile)[slot] = (int)(key0 / kTileN);
        if (lane == 0) {
          reinterpret_cast<unsigned*>(meta + kFixMask)[slot * 4 + (warp - 8)] = fm;
          reinterpret_cast<unsigned*>(meta + kBndMask)[slot * 4 + (warp - 8)] = bm;
          reinterpret_cast<int*>(meta + kBndKc)[slot * 4 + (warp - 8)] = bm ? kc_top : -1;
        }
      }
      mbar_arrive(mb + kBarMeta + 8 * slot);  // metadata published (release)
      vs.ka = ka;
      vs.key0 = key0;
      vs.rv = rv;
      vs.grp = vs.run = 0;
      vs.tx = 0;
      const uint32_t kdst = sbase + kK0;
      if (tma) {
        // 16 keys (a half warp) in consecutive rows of one map are one 64 x 16
        // tile load per operand and 64-column half (run 1: primary map, 2:
        // sidecar); otherwise a group of 4 keys (lanes 4q..4q+3) whose rows
        // all live in one map (grp 1 / 2) takes tile::gather4 loads, issued by
        // the group's first lane; other groups copy their own rows by cp.async
        const int cls = ka == 0 ? 0 : ((ka & 1ull) ? 2 : 1);
        const int h0 = lane & ~15;
        const int c0 = __shfl_sync(kAll, cls, h0);
        const int r0k = __shfl_sync(kAll, rk, h0), r0v = __shfl_sync(kAll, rv, h0);
        const unsigned bseq = __ballot_sync(
            kAll, cls != 0 && cls == c0 && rk == r0k + (lane & 15) && rv == r0v + (lane & 15));
        vs.run = ((bseq >> h0) & 0xFFFFu) == 0xFFFFu ? c0 : 0;
        const unsigned b1 = __ballot_sync(kAll, cls == 1), b2 = __ballot_sync(kAll, cls == 2);
        const int sh = lane & ~3;
        vs.grp = vs.run ? 0
                        : (((b1 >> sh) & 0xFu) == 0xFu ? 1 : (((b2 >> sh) & 0xFu) == 0xFu ? 2 : 0));
        vs.tx = __popc(__ballot_sync(kAll, vs.run != 0 && (lane & 15) == 0)) * 4096u +
                __popc(__ballot_sync(kAll, vs.grp != 0 && (lane & 3) == 0)) * 1024u;
        const int k1 = __shfl_down_sync(kAll, rk, 1);
        const int k2 = __shfl_down_sync(kAll, rk, 2);
        const int k3 = __shfl_down_sync(kAll, rk, 3);
        vs.v1 = __shfl_down_sync(kAll, rv, 1);
        vs.v2 = __shfl_down_sync(kAll, rv, 2);
        vs.v3 = __shfl_down_sync(kAll, rv, 3);
        if (lane == 0 && vs.tx) mbar_expect_tx(mb + kBarK, vs.tx);
        if (vs.run && (lane & 15) == 0) {
          const CUtensorMap* m = vs.run == 1 ? &a.tm[4] : &a.tm[6];
          for (int cb = 0; cb < 2; ++cb)
            tma_tile2d(kdst + cb * 16384 + pt * 128, m, cb * 64, rk, mb + kBarK);
        }
        if (vs.grp && (lane & 3) == 0) {
          const CUtensorMap* m = vs.grp == 1 ? &a.tm[0] : &a.tm[2];
          for (int cb = 0; cb < 2; ++cb)
            tma_gather4(kdst + cb * 16384 + pt * 128, m, cb * 64, rk, k1, k2, k3, mb + kBarK);
        }
        if (!vs.run && !vs.grp) {
          for (int c16 = 0; c16 < 16; ++c16) {
            const char* src = ka ? reinterpret_cast<const char*>(ka & ~1ull) + c16 * 16
                                 : static_cast<const char*>(p.q);
            cp_async16(kdst + sw128(pt, c16, 128), src, ka != 0);
          }
        }
      } else {
        // per-row cp.async: each warp copies its own 32 rows, two 256-byte
        // rows per instruction (row addresses from the owning lanes)
        const int c16 = lane & 15;
#pragma unroll 4
        for (int m = 0; m < 16; ++m) {
          const int src_lane = (lane >> 4) + 2 * m;
          const uint64_t ra = __shfl_sync(kAll, ka, src_lane);
          const char* src = ra ? reinterpret_cast<const char*>(ra & ~1ull) + c16 * 16
                               : static_cast<const char*>(p.q);
          cp_async16(kdst + sw128(wrow0 + src_lane, c16, 128), src, ra != 0);
        }
      }
      cp_async_arrive_noinc(mb + kBarK);
    };
    auto issue_v = [&](int it2, const VSrc& vs) {
      const int st = it2 & 1;
      if (tma) {
        if (lane == 0 && vs.tx) mbar_expect_tx(mb + kBarV + 8 * st, vs.tx);
        if (vs.run && (lane & 15) == 0) {
          const CUtensorMap* m = vs.run == 1 ? &a.tm[5] : &a.tm[7];
          const int x0 = vs.run == 1 ? a.vx0 : 0;
          for (int cb = 0; cb < 2; ++cb)
            tma_tile2d(sbase + kV0 + st * 32768 + cb * 16384 + pt * 128, m, x0 + cb * 64, vs.rv,
                       mb + kBarV + 8 * st);
        }
        if (vs.grp && (lane & 3) == 0) {
          const CUtensorMap* m = vs.grp == 1 ? &a.tm[1] : &a.tm[3];
          const int x0 = vs.grp == 1 ? a.vx0 : 0;
          for (int cb = 0; cb < 2; ++cb)
            tma_gather4(sbase + kV0 + st * 32768 + cb * 16384 + pt * 128, m, x0 + cb * 64, vs.rv,
                        vs.v1, vs.v2, vs.v3, mb + kBarV + 8 * st);
        }
        if (!vs.run && !vs.grp) {
          const int64_t jr = vs.key0 + pt < p.nk ? vs.key0 + pt : p.nk - 1;
          const char* vrow =
              vs.ka ? value_row_addr<T>(a, vs.ka, jr, g) : static_cast<const char*>(p.q);
          for (int c16 = 0; c16 < 16; ++c16)
            cp_async16(sbase + kV0 + st * 32768 + sw128(pt, c16, 128), vrow + c16 * 16,
                       vs.ka != 0);
        }
      } else {
        const int c16 = lane & 15;
#pragma unroll 4
        for (int m = 0; m < 16; ++m) {
          const int src_lane = (lane >> 4) + 2 * m;
          const uint64_t ra = __shfl_sync(kAll, vs.ka, src_lane);
          const int row = wrow0 + src_lane;
          const char* src = ra ? value_row_addr<T>(a, ra, vs.key0 + row, g) + c16 * 16
                               : static_cast<const char*>(p.q);
          cp_async16(sbase + kV0 + st * 32768 + sw128(row, c16, 128), src, ra != 0);
        }
      }
      cp_async_arrive_noinc(mb + kBarV + 8 * st);
    };
    // K has one stage, free once both tiles' QK of key tile it are done.  V
    // has two: stage (it+1)&1 held V(it-1), free once both PVs of tile it-1
    // are done; the PV barriers are per tile and V stage, so their next
    // phase needs the V copy issued here and cannot be missed.
    VSrc vs{};
    if (nlist > 0) {
      load_key();
      issue_k(0, vs);
      issue_v(0, vs);
      if (nlist > 1) load_key();
    }
    for (int it = 0; it + 1 < nlist; ++it) {
      bool ok = mbar_wait(mb + kBarS, it & 1, abort) && mbar_wait(mb + kBarS + 8, it & 1, abort);
      if (!named_and(1, 128, ok)) break;
      issue_k(it + 1, vs);
      const uint32_t pst = 8 * ((it + 1) & 1), pph = ((it - 1) >> 1) & 1;
      ok = it < 1 || (mbar_wait(mb + kBarPV + pst, pph, abort) &&
                      mbar_wait(mb + kBarPV + 16 + pst, pph, abort));
      if (!named_and(1, 128, ok)) break;
      issue_v(it + 1, vs);
      if (it + 2 < nlist) load_key();
    }
    if (use_map && p.kv_slots) {  // skipped tiles: their keys' slots are checked all the same
#pragma unroll 1
      for (int t = 0; t < ntile; ++t) {
        if ((needmap[t >> 5] >> (t & 31)) & 1u) continue;
        const int64_t j = (int64_t)t * kTileN + pt;
        int32_t r1, r2;
        if (j < nmax && key_src<T>(a, j, g, r1, r2) == 0) slot_bad = true;
      }
    }
    if (slot_bad) report(p.status, CS_ST_SLOT_RANGE);

  } else if (warp == 12) {
    // ================================================================== MMA
    if (lane == 0) {
      const uint32_t id_s = umma_idesc(128, 128, a.fmt, 0, 0);  // S = Q K^T
      const uint32_t id_t = umma_idesc(128, NP, a.fmt, 0, 0);   // T = Q E
      const uint32_t id_o = umma_idesc(128, 128, a.fmt, 0, 1);  // O += P V (V MN-major)
      bool ok = mbar_wait(mb + kBarQ, 0, abort);
      if (ok) {
        tc_fence_after();
        for (int qt = 0; qt < 2; ++qt) {
          for (int half = 0; half < 2; ++half) {
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t aoff = qt * 32768 + (kk >> 2) * 16384 + (kk & 3) * 32;
              const uint32_t boff = half * (NP * 256) + (kk >> 2) * (NP * 128) + (kk & 3) * 32;
              tc_mma(tmem + kColS + 128 * qt, umma_desc(sbase + kQ + aoff, 16, 1024),
                     umma_desc(sbase + kP + boff, 16, 1024), id_t, (half | kk) ? 1u : 0u);
            }
          }
        }
        tc_commit(mb + kBarT);
      }
      auto issue_qk = [&](int qt) {
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          tc_mma(tmem + kColS + 128 * qt, umma_desc(sbase + kQ + qt * 32768 + off, 16, 1024),
                 umma_desc(sbase + kK0 + off, 16, 1024), id_s, kk ? 1u : 0u);
        }
        tc_commit(mb + kBarS + 8 * qt);
      };
      if (ok && nlist > 0) {
        ok = mbar_wait(mb + kBarK, 0, abort);
        for (int qt = 0; ok && qt < 2; ++qt) {
          // the tile's S columns hold T until its softmax has read the table
          if (!(ok = mbar_wait(mb + kBarTab + 8 * qt, 0, abort))) break;
          fence_async_smem();
          tc_fence_after();
          issue_qk(qt);
        }
      }
      int lastpv[2] = {-1, -1};  // last key tile whose PV was issued, per tile
      for (int it = 0; ok && it < nlist; ++it) {
        const int st = it & 1;
        for (int qt = 0; ok && qt < 2; ++qt) {
          if (!(ok = mbar_wait(mb + kBarP + 8 * qt, it & 1, abort))) break;
          if (!(ok = mbar_wait(mb + kBarV + 8 * st, (it >> 1) & 1, abort))) break;
          fence_async_smem();
          tc_fence_after();
          for (int kk = 0; kk < kTileN / 16; ++kk) {
            // P of keys 16kk..16kk+15 (packed pairs over the tile's S columns)
            const uint32_t pcol = kColS + 128 * qt + kk * 8;
            const uint32_t boff = kk * 2048;  // V: MN-major
            tc_mma_ts(tmem + kColO + 128 * qt, tmem + pcol,
                      umma_desc(sbase + kV0 + st * 32768 + boff, 16384, 1024), id_o,
                      (it | kk) ? 1u : 0u);
          }
          tc_commit(mb + kBarPV + 16 * qt + 8 * st);
          lastpv[qt] = it;
          if (it + 1 < nlist) {
            // S(it+1) of this tile overwrites the TMEM columns where P(it)
            // lives: PV(it) must be done
            if (!(ok = mbar_wait(mb + kBarPV + 16 * qt + 8 * st, (it >> 1) & 1, abort))) break;
            if (qt == 0 && !(ok = mbar_wait(mb + kBarK, (it + 1) & 1, abort))) break;
            fence_async_smem();
            tc_fence_after();
            issue_qk(qt);
          }
        }
      }
      // drain before TMEM is released: the last PVs (and a commit of
      // anything still uncommitted after an early exit)
      tc_commit(mb + kBarEnd);
      long long t0 = clock64();
      while (!mbar_try(mb + kBarEnd, 0) && clock64() - t0 < kWaitCycles) {
      }
      for (int qt = 0; qt < 2; ++qt) {
        const int last = lastpv[qt];
        if (last < 0) continue;
        const uint32_t bar = mb + kBarPV + 16 * qt + 8 * (last & 1);
        t0 = clock64();
        while (!mbar_try(bar, (last >> 1) & 1) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
    __syncwarp();
  } else {
    // ================================================================ softmax
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftRegs));
    // One thread per S row: warps 0-3 hold tile a, warps 4-7 tile b; warp w
    // addresses TMEM lanes 32(w%4)..32(w%4)+31 of its tile's columns.  A row
    // is never shared, so no barrier joins the softmax warps: every wait
    // result is made warp-uniform (the TMEM loads are warp-collective) and
    // the loop exits on any expired wait.
    const int qt = warp >> 2, q4 = warp & 3;
    const int r = q4 * 32 + lane;  // TMEM lane == tile row
    const int64_t i = i0 + qt * R + r / G;
    const int h = g * G + r % G;
    const bool row_ok = i < nq;
    const int64_t qp = row_ok ? p.qpos[i] : -1;
    const int64_t nlim = row_ok ? (qp + 1 < p.nk ? qp + 1 : p.nk) : 0;
    const bool qsel = row_ok && p.q_selected != nullptr && p.q_selected[i] != 0;
    const bool chunked = p.pos_mode == CS_POS_CHUNK;
    const int qchunk = (row_ok && chunked && nlim > 0) ? p.key_chunk[nlim - 1] : -1;
    const float* offrow =
        (row_ok && chunked) ? p.chunk_off + (int64_t)h * p.co_stride_h + i * p.co_stride_q
                            : nullptr;
    // canonical-table mode: this row's table row (float32 positions) or -1
    const int32_t qrow = (TBL && row_ok) ? p.q_row[i] : -1;
    const float* tabrow =
        qrow >= 0 ? static_cast<const float*>(p.table) + (int64_t)h * p.tb_stride_h +
                        (int64_t)qrow * p.tb_stride_r
                  : nullptr;
    const bool warp_tbl = TBL && __any_sync(0xffffffffu, qrow >= 0);
    const bool strict = TBL && p.strict != 0;
    const float atol = (float)p.atol;
    float prevp = 0.f;  // strict: the position of the next newer causal key
    bool prevv = false;
    int32_t sbits = 0;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const uint32_t sc = tmem + lane_base + kColS + 128 * qt;  // this row's S columns
    const uint32_t oc = tmem + lane_base + kColO + 128 * qt;  // this row's O columns
    // q.E table of row r: T[p] (log2 domain) at index p ^ tsw -- float with
    // tsw = r & 31 (NP = 64), half with tsw = 2 (r & 31) (NP = 128) -- so
    // that the 32 rows of a warp reading the same entry hit distinct banks;
    // a row's table is written and read by its own thread only
    using TabT = typename std::conditional<NP == 64, float, __half>::type;
    TabT* Tab = reinterpret_cast<TabT*>(smem + kTab + qt * 32768) + r * NP;
    const int tsw = NP == 64 ? (r & 31) : 2 * (r & 31);
    auto tab_get = [&](int idx) -> float {
      if constexpr (NP == 64) return Tab[idx ^ tsw];
      else return __half2float(Tab[idx ^ tsw]);
    };
    const float inv_sqrt_d = (float)(1.0 / p.scale);
    const float LOG2E = 1.4426950408889634f;
    const float scale2 = inv_sqrt_d * LOG2E;
    const float half_scale = 0.5f * inv_sqrt_d;

    fence_async_smem();  // this thread's share of the E table (staged before the barrier)
    mbar_arrive(mb + kBarQ);
    bool ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarT, 0, abort));
    tc_fence_after();
    {
      uint32_t v[32];
#pragma unroll
      for (int hb = 0; hb < NP / 32; ++hb) {
        CS_TMEM_LD32(sc + 32 * hb, v);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float tv = __uint_as_float(v[c]) * LOG2E;
          if constexpr (NP == 64) Tab[(32 * hb + c) ^ tsw] = tv;
          else Tab[(32 * hb + c) ^ tsw] = __float2half_rn(tv);
        }
      }
    }
    tc_fence_before();
    mbar_arrive(mb + kBarTab + 8 * qt);  // the S columns are free for QK
    const float tsat2 = tab_get(p.npos - 1);  // saturated bias (log2 domain)
    // interpolated bias at position pos in [0, npos - 1] (position.py:339-344)
    auto bias_at = [&](float pos) {
      int lo;
      const float fl = floor_pos(pos, lo);
      const int hi = lo + 1 < p.npos ? lo + 1 : p.npos - 1;
      const float t0 = tab_get(lo);
      return fmaf(pos - fl, tab_get(hi) - t0, t0);
    };

    float carry = 0.f;       // running count entering the newer edge of the tile
    float mref = -INFINITY;  // softmax reference max (log2 domain)
    float lsum = 0.f;        // the row sum
    // count restart at the chunk boundary ending at key j, or -1 for none
    auto restart_at = [&](int64_t j) -> float {
      const int kc = p.key_chunk[j];
      return kc < qchunk ? offrow[kc] : -1.f;
    };
    // O row times f (after PV of the previous tile)
    auto rescale_o = [&](float f) {
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t o[32];
        CS_TMEM_LD32(oc + 32 * cc, o);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
        CS_TMEM_ST32(oc + 32 * cc, o);
      }
      tmem_wait_st();
    };
    for (int it = 0; ok && it < nlist; ++it) {
      const int slot = it & 3;
      // key metadata of slot it % 4 (the step's key tile among them): the
      // producer publishes it ahead of S(it), and the slot is not reused
      // before P(it) of both tiles.  Masks, chunk restarts and the fast /
      // contextual decision are settled while QK(it) may still be running,
      // so their latency hides behind it.
      ok = mbar_wait(mb + kBarMeta + 8 * slot, (it >> 2) & 1, abort);
      const int kt = ok ? reinterpret_cast<const volatile int*>(meta + kSlotTile)[slot] : 0;
      const int64_t key0 = (int64_t)kt * kTileN;
      const unsigned* fixm = reinterpret_cast<const unsigned*>(meta + kFixMask) + slot * 4;
      const unsigned* bndm = reinterpret_cast<const unsigned*>(meta + kBndMask) + slot * 4;
      const int* bndkc = reinterpret_cast<const int*>(meta + kBndKc) + slot * 4;
      const int nvalid =
          (int)(nlim - key0 < 0 ? 0 : (nlim - key0 > kTileN ? kTileN : nlim - key0));
      // columns hidden from the row, bit c of word cc (key 32 cc + c): past
      // the causal / key limit, or fixed keys seen by a selected row (its own
      // key stays visible)
      unsigned hide0, hide1, hide2, hide3;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int lim = nvalid - cc * 32;
        unsigned m = lim >= 32 ? 0u : (lim <= 0 ? ~0u : (~0u << lim));
        if (qsel) {
          unsigned fx = fixm[cc];
          const int64_t self = qp - key0 - cc * 32;
          if (self >= 0 && self < 32) fx &= ~(1u << (int)self);
          m |= fx;
        }
        (cc == 0 ? hide0 : cc == 1 ? hide1 : cc == 2 ? hide2 : hide3) = m;
      }
      // (selects, not an indexed array: the chunk loops below are not unrolled)
      auto hide_of = [&](int cc) {
        return cc == 0 ? hide0 : cc == 1 ? hide1 : cc == 2 ? hide2 : hide3;
      };
      const bool anyb = chunked && ok && (bndm[0] | bndm[1] | bndm[2] | bndm[3]) != 0u;
      // the row is saturated for this tile when its count is already >= npos-1
      // and no live chunk boundary of the tile restarts it below that value
      // (a table row never is: its positions come from the table)
      bool sat = carry >= top && qrow < 0;
      if (anyb && sat) {
#pragma unroll 1
        for (int cc = 0; cc < 4 && sat; ++cc) {
          const int lim = nvalid - cc * 32;
          unsigned bits = bndm[cc] & (lim >= 32 ? ~0u : (lim <= 0 ? 0u : ((1u << lim) - 1u)));
          while (bits && sat) {
            const int c = 31 - __clz(bits);
            bits &= ~(1u << c);
            const float off = restart_at(key0 + cc * 32 + c);
            if (off >= 0.f && off < top) sat = false;
          }
        }
      }
      const bool fast = __all_sync(0xffffffffu, sat || nvalid == 0);
      // S(it) of this tile from the MMA warp
      ok = ok && mbar_wait(mb + kBarS + 8 * qt, it & 1, abort);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      if (fast && __all_sync(0xffffffffu, mref > -INFINITY || nvalid == 0)) {
        // Saturated tile after the first: one pass, chunk by chunk in
        // increasing key order (P of chunk cc goes to S columns 16cc..16cc+15,
        // already read).  Every visible score is x = S * scale2 + tsat2 -
        // mref.  A chunk whose sum passes 2^8 (some x above the lazy-rescale
        // limit; NaN counts too) is rare: it is redone against its own
        // maximum cm (sh = cm), and after the four chunks the reference moves
        // to the largest cm: O and the row sum are rescaled (after PV of the
        // previous tile), and so is each chunk's P (2^(sh - trel)).
        carry = sat ? fmaxf(carry, top) : carry;
        const float fb = tsat2 - mref;
        float pk = 0.f, trel = -INFINITY;
        float sh0 = 0.f, sh1 = 0.f, sh2 = 0.f, sh3 = 0.f;  // per-chunk shifts (rare path)
        // chunk cc of the row from v (its raw S, loaded): P into v[0..15],
        // stored over S columns 16cc..16cc+15; returns the chunk's sum
        auto one_chunk = [&](uint32_t(&v)[32], int cc) -> float {
          const unsigned hm = hide_of(cc);
          if (__all_sync(0xffffffffu, hm == ~0u)) {
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] = 0u;
          } else if (__all_sync(0xffffffffu, hm == 0u)) {  // every column visible (common)
#pragma unroll
            for (int c = 0; c < 32; ++c)
              v[c] = __float_as_uint(ex2(fmaf(__uint_as_float(v[c]), scale2, fb)));
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              v[c] = __float_as_uint(
                  (hm >> c) & 1u ? 0.f : ex2(fmaf(__uint_as_float(v[c]), scale2, fb)));
          }
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const float e0 = __uint_as_float(v[2 * u]), e1 = __uint_as_float(v[2 * u + 1]);
            s0 += e0;
            s1 += e1;
            v[u] = Pack2<T>::pack(e0, e1);  // in place: keys 2u, 2u+1 already read
          }
          float pc = s0 + s1;
          if (__any_sync(0xffffffffu, !(pc <= 256.f))) {  // rare; the whole warp redoes
            CS_TMEM_LD32(sc + 32 * cc, v);
            tmem_wait_ld();
            float cm = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float x = (hm >> c) & 1u ? -INFINITY : fmaf(__uint_as_float(v[c]), scale2, fb);
              v[c] = __float_as_uint(x);
              cm = fmaxf(cm, x);
            }
            const float shc = cm > 8.f ? cm : 0.f;
            sh0 = cc == 0 ? shc : sh0;
            sh1 = cc == 1 ? shc : sh1;
            sh2 = cc == 2 ? shc : sh2;
            sh3 = cc == 3 ? shc : sh3;
            trel = fmaxf(trel, cm);
            float r0 = 0.f, r1 = 0.f;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const float e0 = ex2(__uint_as_float(v[2 * u]) - shc);
              const float e1 = ex2(__uint_as_float(v[2 * u + 1]) - shc);
              r0 += e0;
              r1 += e1;
              v[u] = Pack2<T>::pack(e0, e1);
            }
            pc = r0 + r1;
          }
          CS_TMEM_ST16(sc + 16 * cc, v);
          return pc;
        };
        // two register buffers: the TMEM load of the next chunk is in flight
        // while the current one is computed (a wait covers every earlier load
        // of the thread, so it is placed after that computation)
        uint32_t va[32], vb[32];
        CS_TMEM_LD32(sc, va);
        tmem_wait_ld();
#pragma unroll 1
        for (int cp = 0; cp < 2; ++cp) {
          CS_TMEM_LD32(sc + 32 * (2 * cp + 1), vb);
          pk += one_chunk(va, 2 * cp);
          tmem_wait_ld();
          if (cp == 0) CS_TMEM_LD32(sc + 64, va);
          pk += one_chunk(vb, 2 * cp + 1);
          if (cp == 0) tmem_wait_ld();
        }
        if (__any_sync(0xffffffffu, trel > 8.f)) {  // rare: move the reference
          const bool mv = trel > 8.f;
          tmem_wait_st();
          if (it > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarPV + 16 * qt + 8 * ((it - 1) & 1),
                                                   ((it - 1) >> 1) & 1, abort));
            if (!ok) break;
            tc_fence_after();
          }
          const float f = mv ? ex2(-trel) : 1.f;
          lsum *= f;
          rescale_o(f);
          pk = 0.f;
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {  // each chunk's P: 2^(sh - trel)
            const float shc = cc == 0 ? sh0 : cc == 1 ? sh1 : cc == 2 ? sh2 : sh3;
            const float fk = mv ? ex2(shc - trel) : 1.f;
            uint32_t w[16];
            CS_TMEM_LD16(sc + 16 * cc, w);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const float2 e = unpack2(w[u], T{});
              pk += e.x * fk + e.y * fk;
              w[u] = Pack2<T>::pack(e.x * fk, e.y * fk);
            }
            CS_TMEM_ST16(sc + 16 * cc, w);
          }
          mref = mv ? mref + trel : mref;
        }
        lsum += pk;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(mb + kBarP + 8 * qt);
        continue;
      }
      float tmax = -INFINITY;
      // contextual chunks that took the own-key-only path (bit cc) and their
      // one score per row
      unsigned somask = 0u;
      float xs0 = -INFINITY, xs1 = -INFINITY, xs2 = -INFINITY, xs3 = -INFINITY;
      if (fast) {
        // saturated, the row's first visible tile: every visible score is
        // S * scale2 + tsat2, a monotone map of the raw S, so the tile max
        // comes from the raw scores (which stay in TMEM for the P pass)
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          const unsigned hm = hide_of(cc);
          if (__all_sync(0xffffffffu, hm == ~0u)) continue;
          uint32_t v[32];
          CS_TMEM_LD32(sc + 32 * cc, v);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            m0 = (hm >> c) & 1u ? m0 : fmaxf(m0, __uint_as_float(v[c]));
            m1 = (hm >> (c + 1)) & 1u ? m1 : fmaxf(m1, __uint_as_float(v[c + 1]));
          }
        }
        const float mraw = fmaxf(m0, m1);
        tmax = mraw > -INFINITY ? fmaf(mraw, scale2, tsat2) : -INFINITY;
        carry = sat ? fmaxf(carry, top) : carry;
      } else {
        // contextual: chunks newest first; per chunk the gates and the
        // reverse count (restarted at chunk boundaries), then positions,
        // interpolated bias and masks; the scores (log2 domain) go back
        // over S for the P pass
        float Rc = carry;
        float t0 = -INFINITY, t1 = -INFINITY;
#pragma unroll 1
        for (int cc = 3; cc >= 0; --cc) {
          const unsigned hm = hide_of(cc);
          const int lim = nvalid - cc * 32;
          uint32_t s[32], v[32];
          CS_TMEM_LD32(sc + 32 * cc, s);
          tmem_wait_ld();
          const unsigned bdc = cc == 0 ? bndm[0] : cc == 1 ? bndm[1] : cc == 2 ? bndm[2] : bndm[3];
          // chunk saturated for the whole warp: no boundary restarts a count
          // and every row either reaches it with a count >= npos - 1 or has
          // no causal key in it: one bias (tsat2) for every visible column,
          // and the gates change no position
          if (!warp_tbl && __all_sync(0xffffffffu, bdc == 0u && (lim <= 0 || Rc >= top))) {
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float x0 =
                  (hm >> c) & 1u ? -INFINITY : fmaf(__uint_as_float(s[c]), scale2, tsat2);
              const float x1 =
                  (hm >> (c + 1)) & 1u ? -INFINITY : fmaf(__uint_as_float(s[c + 1]), scale2, tsat2);
              s[c] = __float_as_uint(x0);
              s[c + 1] = __float_as_uint(x1);
              t0 = fmaxf(t0, x0);
              t1 = fmaxf(t1, x1);
            }
            CS_TMEM_ST32(sc + 32 * cc, s);
            if (lim > 0) Rc = fmaxf(Rc, top);
            continue;
          }
          // every column a row sees in the chunk is its own key, and the chunk
          // lies above every gate chain of the row's other seen keys: the own
          // key's count is its gate (it is the newest causal key, so the
          // count entering it is Rc) and no other gate of the chunk matters.
          // One gate and one interpolation a row; the P pass takes the one
          // score from xs (the scores are not stored back).
          {
            const int64_t selfc = qp - (key0 + cc * 32);
            const unsigned selfbit = (selfc >= 0 && selfc < 32) ? (1u << (int)selfc) : 0u;
            if (!warp_tbl &&
                __all_sync(0xffffffffu, key0 + cc * 32 > chain_hi && (~hm & ~selfbit) == 0u)) {
              float zs = 0.f;
#pragma unroll
              for (int c = 0; c < 32; ++c) zs = (selfbit >> c) & 1u ? __uint_as_float(s[c]) : zs;
              float xs = -INFINITY;
              if ((~hm & selfbit) != 0u) {
                Rc = Rc + fmaf(0.5f, tanh_approx(zs * half_scale), 0.5f);
                xs = fmaf(zs, scale2, bias_at(fminf(Rc, top)));
              }
              t0 = fmaxf(t0, xs);
              xs0 = cc == 0 ? xs : xs0;
              xs1 = cc == 1 ? xs : xs1;
              xs2 = cc == 2 ? xs : xs2;
              xs3 = cc == 3 ? xs : xs3;
              somask |= 1u << cc;
              continue;
            }
          }
#pragma unroll
          for (int c = 0; c < 32; ++c)  // gate = sigmoid(z) = (1 + tanh(z / 2)) / 2: one MUFU op
            v[c] = __float_as_uint(fmaf(0.5f, tanh_approx(__uint_as_float(s[c]) * half_scale), 0.5f));
          const unsigned bd = bndm[cc];
          if (bd == 0u) {  // warp-uniform: no chunk boundary, a plain suffix sum
#pragma unroll
            for (int c = 31; c >= 0; --c) {
              Rc = c < lim ? Rc + __uint_as_float(v[c]) : Rc;
              v[c] = __float_as_uint(Rc);
            }
          } else {
            const int cf = 31 - __clz(bd);
            const int kcf = bndkc[cc];
            const float rf = (kcf >= 0 && kcf < qchunk) ? offrow[kcf] : -1.f;
#pragma unroll
            for (int c = 31; c >= 0; --c) {
              float base = Rc;
              if ((bd >> c) & 1u) {  // warp-uniform: last key of a chunk
                const float off = c == cf ? rf : restart_at(key0 + cc * 32 + c);
                if (off >= 0.f) base = off;
              }
              Rc = c < lim ? base + __uint_as_float(v[c]) : Rc;
              v[c] = __float_as_uint(Rc);
            }
          }
          if constexpr (TBL) {
            if (qrow >= 0) {
              // table positions at keys with a table column, then (strict)
              // the path checks of validate_contextual_path on the causal
              // keys, newest first so each pair is (key, next newer key)
              const int64_t j0 = key0 + cc * 32;
#pragma unroll
              for (int c = 31; c >= 0; --c) {
                if (c >= lim) continue;
                float pos = fminf(__uint_as_float(v[c]), top);
                const int32_t ko = __ldg(p.k_ord + j0 + c);
                if (ko >= 0) {
                  float t = __ldg(tabrow + (int64_t)ko * p.tb_stride_c);
                  if (!(t >= 0.f && t <= top)) {
                    sbits |= CS_ST_POS_RANGE;
                    t = t >= 0.f ? fminf(t, top) : 0.f;
                  }
                  pos = t;
                }
                if (strict) {
                  const float rnd = 1.1920928955078125e-07f * fabsf(pos);
                  if (pos < -(atol + rnd)) sbits |= CS_ST_PATH_NEG;
                  const float avail = (float)(qp - (j0 + c)) + 1.f;
                  if (pos > avail + atol + rnd) sbits |= CS_ST_PATH_AVAIL;
                  if (prevv) {
                    const float diff = pos - prevp;
                    const float ptol = atol + rnd + 1.1920928955078125e-07f * fabsf(prevp);
                    if (diff < -ptol) sbits |= CS_ST_PATH_INCR;
                    if (diff > 1.f + ptol) sbits |= CS_ST_PATH_GAP;
                  }
                  prevp = pos;
                  prevv = true;
                }
                v[c] = __float_as_uint(pos);
              }
            }
          }
          // interpolated bias and score, eight columns at a time: the
          // positions first, then all sixteen table reads, then the
          // arithmetic, so the shared-memory loads are in flight together
          // (each column's arithmetic is that of bias_at)
#pragma unroll
          for (int c0 = 0; c0 < 32; c0 += 8) {
            float fr[8];
            int lo[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const float pos = fminf(__uint_as_float(v[c0 + u]), top);
              const float fl = floor_pos(pos, lo[u]);
              fr[u] = pos - fl;
            }
            float tl[8], th[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              tl[u] = tab_get(lo[u]);
              th[u] = tab_get(lo[u] + 1 < p.npos ? lo[u] + 1 : p.npos - 1);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int c = c0 + u;
              const float x = (hm >> c) & 1u
                                  ? -INFINITY
                                  : fmaf(__uint_as_float(s[c]), scale2,
                                         fmaf(fr[u], th[u] - tl[u], tl[u]));
              s[c] = __float_as_uint(x);
              if (u & 1) t1 = fmaxf(t1, x);
              else t0 = fmaxf(t0, x);
            }
          }
          CS_TMEM_ST32(sc + 32 * cc, s);
        }
        tmem_wait_st();
        tmax = fmaxf(t0, t1);
        carry = Rc;
      }
      float mnew = mref;
      bool rescale = false;
      if (tmax > mref + 8.f) {  // lazy rescaling: keep a stale max unless it lags by 2^8
        mnew = tmax;
        rescale = mref > -INFINITY;
      }
      if (it > 0 && __any_sync(0xffffffffu, rescale)) {
        ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarPV + 16 * qt + 8 * ((it - 1) & 1),
                                               ((it - 1) >> 1) & 1, abort));
        if (!ok) break;
        tc_fence_after();
        const float f = rescale ? ex2(mref - mnew) : 1.f;
        lsum *= f;
        rescale_o(f);
      }
      mref = mnew;
      // P = 2^(s - mref) as packed 16-bit pairs over the tile's S columns,
      // chunks in increasing order so no score is overwritten before it is
      // read; PV takes P from TMEM.  A saturated tile forms s - mref =
      // S * scale2 + (tsat2 - mref) from the raw S.
      const float mcur = mref > -INFINITY ? mref : 0.f;
      const float fb = tsat2 - mcur;
      float part0 = 0.f, part1 = 0.f;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const unsigned hm = hide_of(cc);
        uint32_t v[32];
        if ((fast || !((somask >> cc) & 1u)) && __all_sync(0xffffffffu, hm == ~0u)) {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = 0u;
        } else if ((somask >> cc) & 1u) {  // own key only: one exponential a row
          const int64_t selfc = qp - (key0 + cc * 32);
          const float xs = cc == 0 ? xs0 : cc == 1 ? xs1 : cc == 2 ? xs2 : xs3;
          const float es = ex2(xs - mcur);
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __float_as_uint(selfc == c ? es : 0.f);
        } else {
          CS_TMEM_LD32(sc + 32 * cc, v);
          tmem_wait_ld();
          if (fast) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              v[c] = __float_as_uint(
                  (hm >> c) & 1u ? 0.f : ex2(fmaf(__uint_as_float(v[c]), scale2, fb)));
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] = __float_as_uint(ex2(__uint_as_float(v[c]) - mcur));
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float e0 = __uint_as_float(v[2 * u]), e1 = __uint_as_float(v[2 * u + 1]);
          part0 += e0;
          part1 += e1;
          v[u] = Pack2<T>::pack(e0, e1);
        }
        CS_TMEM_ST16(sc + 16 * cc, v);
      }
      lsum += part0 + part1;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(mb + kBarP + 8 * qt);
    }
    // epilogue: O / l
    if (ok && nlist > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarPV + 16 * qt + 8 * ((nlist - 1) & 1),
                                             ((nlist - 1) >> 1) & 1, abort));
      tc_fence_after();
    }
    int32_t bits = sbits;  // table-mode range / strict path bits
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    char* orow = row_ok ? static_cast<char*>(p.out) + (i * p.o_stride_tok +
                                                       (int64_t)h * p.o_stride_head) *
                                                          dtype_size(p.out_dtype)
                        : nullptr;
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      const int col0 = cc * 32;
      uint32_t v[32];
      if (nlist > 0 && ok) {
        CS_TMEM_LD32(oc + col0, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = 0u;
      }
      if (row_ok && ok) {
        if (p.out_dtype == CS_F32) {
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            float4 x = make_float4(__uint_as_float(v[c]) * inv, __uint_as_float(v[c + 1]) * inv,
                                   __uint_as_float(v[c + 2]) * inv,
                                   __uint_as_float(v[c + 3]) * inv);
            if (!isfinite(x.x + x.y + x.z + x.w)) bits |= CS_ST_LOGIT_NONFINITE;
            reinterpret_cast<float4*>(orow)[(col0 + c) / 4] = x;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint32_t w[4];
            float chk = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float x0 = __uint_as_float(v[c + 2 * u]) * inv;
              const float x1 = __uint_as_float(v[c + 2 * u + 1]) * inv;
              chk += x0 + x1;
              w[u] = Pack2<T>::pack(x0, x1);
            }
            if (!isfinite(chk)) bits |= CS_ST_LOGIT_NONFINITE;
            reinterpret_cast<uint4*>(orow)[(col0 + c) / 8] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
    if (bits) report(p.status, bits);
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort) report(p.status, CS_ST_TIMEOUT);
  if (warp == 12) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

bool prefill_supported(const cs_attn_params* p) {
  if (p->in_dtype != CS_BF16 && p->in_dtype != CS_F16) return false;
  if (p->out_dtype != p->in_dtype && p->out_dtype != CS_F32) return false;
  if (p->d != kD || p->dv != kD) return false;
  if (p->npos > kMaxNpos) return false;
  const int G = p->hq / p->hkv;
  if (G < 1 || G > 128 || 128 % G) return false;
  if (p->pos_mode != CS_POS_CONTEXTUAL && p->pos_mode != CS_POS_CHUNK &&
      p->pos_mode != CS_POS_TABLE)
    return false;
  if (p->pos_mode == CS_POS_TABLE && (!p->table || !p->q_row || !p->k_ord)) return false;
  // strict: checked for table rows; a contextual path is valid by construction
  if (p->strict && p->pos_mode == CS_POS_CHUNK) return false;
  if (p->gate_mask || p->vis_mask || p->out_positions || p->positions_only) return false;
  if (p->kpos != nullptr) return false;
  const int es = 2;
  auto al = [](int64_t x) { return (x % 16) == 0; };
  if (!al(reinterpret_cast<uintptr_t>(p->q)) || !al(p->q_stride_tok * es) ||
      !al(p->q_stride_head * es))
    return false;
  if (!al(reinterpret_cast<uintptr_t>(p->out)) || !al(p->o_stride_tok * dtype_size(p->out_dtype)) ||
      !al(p->o_stride_head * dtype_size(p->out_dtype)))
    return false;
  if (p->kv_slots) {
    PagedView pv = PagedView::make(p->paged);
    if (!pv.vec16()) return false;
  } else {
    if (!al(reinterpret_cast<uintptr_t>(p->k)) || !al(reinterpret_cast<uintptr_t>(p->v)) ||
        !al(p->k_stride_tok * es) || !al(p->k_stride_head * es) || !al(p->v_stride_tok * es) ||
        !al(p->v_stride_head * es))
      return false;
  }
  return true;
}

// cuTensorMapEncodeTiled from the driver, resolved at first use through the
// runtime (the library does not link libcuda, so it loads on hosts without a GPU)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static const EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// 2-D row map over `rows` rows of `inner` 16-bit elements, `unit` bytes apart,
// read in 64 x box_rows boxes with the 128-byte swizzle of the UMMA operand tiles
bool encode_rows(CUtensorMap* m, const void* base, bool bf16, int64_t inner, int64_t rows,
                 int64_t unit, uint32_t box_rows) {
  if (base == nullptr || reinterpret_cast<uintptr_t>(base) % 16 || unit % 16 ||
      unit < inner * 2 || rows < 1 || rows > INT32_MAX || inner < 128)
    return false;
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)unit};
  const cuuint32_t box[2] = {64, box_rows}, es[2] = {1, 1};
  const EncodeTiledFn encode = encode_tiled();
  if (encode == nullptr) return false;
  return encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row structure of the K/V storage for the TMA path: every row the kernel
// reads must be base + row * unit, with unit the gcd of the byte strides.
// Returns false (per-row cp.async path) when a stride is negative or the
// layout does not fit the rules of encode_rows.
bool setup_tma(Args& a) {
  const cs_attn_params& p = a.p;
  const bool bf16 = p.in_dtype == CS_BF16;
  const int64_t es = 2;
  // map i with 64 x 1 boxes (gather4) and map i + 4 with 64 x 16 boxes (runs)
  auto encode = [&](int i, const void* base, int64_t inner, int64_t rows, int64_t unit) {
    return encode_rows(&a.tm[i], base, bf16, inner, rows, unit, 1) &&
           encode_rows(&a.tm[i + 4], base, bf16, inner, rows, unit, 16);
  };
  auto gcd3 = [](int64_t x, int64_t y, int64_t z) { return std::gcd(std::gcd(x, y), z); };
  if (p.kv_slots) {
    const PagedView& pv = a.pv;
    if (pv.sb < 0 || pv.sh < 0 || pv.so < 0 || pv.se != es) return false;
    const int64_t unit = gcd3(pv.sb, pv.sh, pv.so);
    if (unit <= 0) return false;
    const int64_t nb = pv.native_total / pv.bs;
    const int64_t rows = ((nb - 1) * pv.sb + (pv.kv_heads - 1) * pv.sh + (pv.bs - 1) * pv.so) /
                             unit + 1;
    if (!encode(0, pv.cache, 2 * pv.head_dim, rows, unit)) return false;
    a.tm[1] = a.tm[0];
    a.tm[5] = a.tm[4];
    a.vx0 = (int)pv.head_dim;
    a.nrb = pv.sb / unit;
    a.nrh = pv.sh / unit;
    a.nro = pv.so / unit;
    if (pv.side_capacity > 0) {
      if (pv.ssr < 0 || pv.ssh < 0 || pv.sse != es) return false;
      const int64_t su = std::gcd(pv.ssr, pv.ssh);
      if (su <= 0) return false;
      const int64_t srows = ((pv.side_capacity - 1) * pv.ssr + (pv.kv_heads - 1) * pv.ssh) / su + 1;
      if (!encode(2, pv.side_k, pv.head_dim, srows, su) ||
          !encode(3, pv.side_v, pv.head_dim, srows, su))
        return false;
      a.srr = pv.ssr / su;
      a.srh = pv.ssh / su;
    } else {  // never addressed: no slot reaches the sidecar
      a.tm[2] = a.tm[3] = a.tm[0];
      a.tm[6] = a.tm[7] = a.tm[4];
    }
    return true;
  }
  const int64_t kt = p.k_stride_tok * es, kh = p.k_stride_head * es;
  const int64_t vt = p.v_stride_tok * es, vh = p.v_stride_head * es;
  if (kt < 0 || kh < 0 || vt < 0 || vh < 0) return false;
  const int64_t ku = std::gcd(kt, kh), vu = std::gcd(vt, vh);
  if (ku <= 0 || vu <= 0) return false;
  const int64_t krows = ((int64_t)(p.nk - 1) * kt + (int64_t)(p.hkv - 1) * kh) / ku + 1;
  const int64_t vrows = ((int64_t)(p.nk - 1) * vt + (int64_t)(p.hkv - 1) * vh) / vu + 1;
  if (!encode(0, p.k, p.d, krows, ku) || !encode(1, p.v, p.dv, vrows, vu)) return false;
  a.tm[2] = a.tm[0];
  a.tm[3] = a.tm[1];
  a.tm[6] = a.tm[4];
  a.tm[7] = a.tm[5];
  a.vx0 = 0;
  a.krt = kt / ku;
  a.krh = kh / ku;
  a.vrt = vt / vu;
  a.vrh = vh / vu;
  return true;
}

// CACHESLIDE_PREFILL_COPY=cpasync selects the per-row cp.async K/V path
// (the path taken anyway when the storage has no row structure for TMA)
bool tma_enabled() {
  const char* e = std::getenv("CACHESLIDE_PREFILL_COPY");
  return !(e != nullptr && std::strcmp(e, "cpasync") == 0);
}

// host-side argument block of one request (false: unsupported)
bool make_args(const cs_attn_params* p, Args& a) {
  memset(&a, 0, sizeof(a));
  a.p = *p;
  a.pv = p->kv_slots ? PagedView::make(p->paged) : PagedView{};
  a.G = p->hq / p->hkv;
  a.R = 128 / a.G;
  a.fmt = p->in_dtype == CS_BF16 ? 1 : 0;
  a.pairs_per_head = (p->nq + 2 * a.R - 1) / (2 * a.R);
  a.bs_shift = -1;
  if (p->kv_slots) {
    const int64_t bs = p->paged.block_size;
    if ((bs & (bs - 1)) == 0) {
      int s = 0;
      while ((1ll << s) < bs) ++s;
      a.bs_shift = s;
    }
  }
  a.tma = (p->nk > 0 && tma_enabled() && setup_tma(a)) ? 1 : 0;
  return true;
}

// once per kernel: the register split inside the kernel (setmaxnreg) is
// sized for a launch at exactly kLaunchRegs registers a thread; any other
// count could leave a warpgroup waiting for registers, so it is refused
template <typename K>
int configure(K kern, bool& done) {
  if (done) return CS_OK;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return CS_ERR_CUDA;
  if (fa.numRegs != kLaunchRegs) return CS_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSmemBytes) != cudaSuccess)
    return CS_ERR_CUDA;
  done = true;
  return CS_OK;
}

bool same_prefill_shape(const cs_attn_params* a, const cs_attn_params* b) {
  return a->hq == b->hq && a->hkv == b->hkv && a->in_dtype == b->in_dtype &&
         (a->npos > 64) == (b->npos > 64) &&
         (a->pos_mode == CS_POS_TABLE) == (b->pos_mode == CS_POS_TABLE);
}

}  // namespace
}  // namespace cs

using namespace cs;

extern "C" int cs_cope_attn_prefill(const cs_attn_params* p, void* stream) {
  int rc = validate_attn_params(p);
  if (rc != CS_OK) return rc;
  if (!prefill_supported(p)) return CS_ERR_UNSUPPORTED;
  if (p->nq == 0) return CS_OK;
  Args a;
  make_args(p, a);
  const int blocks = a.pairs_per_head * p->hkv;
  static bool configured[8] = {false, false, false, false, false, false, false, false};
  auto launch = [&](auto kern, int which) -> int {
    const int c = configure(kern, configured[which]);
    if (c != CS_OK) return c;
    kern<<<blocks, kThreads, kSmemBytes, as_stream(stream)>>>(a);
    CS_LAUNCH_CHECK();
    return CS_OK;
  };
  const bool bf = p->in_dtype == CS_BF16, wide = p->npos > 64;
  if (p->pos_mode == CS_POS_TABLE) {
    if (wide)
      return bf ? launch(cope_prefill_sm100<__nv_bfloat16, 128, true>, 7)
                : launch(cope_prefill_sm100<__half, 128, true>, 6);
    return bf ? launch(cope_prefill_sm100<__nv_bfloat16, 64, true>, 5)
              : launch(cope_prefill_sm100<__half, 64, true>, 4);
  }
  if (wide)
    return bf ? launch(cope_prefill_sm100<__nv_bfloat16, 128, false>, 3)
              : launch(cope_prefill_sm100<__half, 128, false>, 2);
  return bf ? launch(cope_prefill_sm100<__nv_bfloat16, 64, false>, 1)
            : launch(cope_prefill_sm100<__half, 64, false>, 0);
}

extern "C" int cs_cope_attn_prefill_batch(const cs_attn_params* params, int32_t count,
                                          void* stream) {
  if (params == nullptr || count < 1) return CS_ERR_INVALID;
  for (int k = 0; k < count; ++k) {
    const int rc = validate_attn_params(&params[k]);
    if (rc != CS_OK) return rc;
    if (!prefill_supported(&params[k]) || !same_prefill_shape(&params[0], &params[k]))
      return CS_ERR_UNSUPPORTED;
  }
  static bool configured[8] = {false, false, false, false, false, false, false, false};
  for (int first = 0; first < count; first += kMaxPrefillBatch) {
    const int n = count - first < kMaxPrefillBatch ? count - first : kMaxPrefillBatch;
    BatchArgs b;  // the launch copies it into the kernel's parameter space
    memset(&b, 0, sizeof(b));
    b.hkv = params[first].hkv;
    for (int k = 0; k < n; ++k) {
      const cs_attn_params* p = &params[first + k];
      if (p->nq == 0) continue;
      make_args(p, b.r[b.count]);
      b.max_pairs = b.r[b.count].pairs_per_head > b.max_pairs ? b.r[b.count].pairs_per_head
                                                               : b.max_pairs;
      ++b.count;
    }
    if (b.count == 0) continue;
    const int blocks = b.max_pairs * b.count * b.hkv;
    auto launch = [&](auto kern, int which) -> int {
      const int c = configure(kern, configured[which]);
      if (c != CS_OK) return c;
      kern<<<blocks, kThreads, kSmemBytes, as_stream(stream)>>>(b);
      CS_LAUNCH_CHECK();
      return CS_OK;
    };
    const bool wide = params[first].npos > 64;
    const bool bf = params[first].in_dtype == CS_BF16;
    const bool tbl = params[first].pos_mode == CS_POS_TABLE;
    int rc;
    if (tbl)
      rc = wide ? (bf ? launch(cope_prefill_sm100_batch<__nv_bfloat16, 128, true>, 7)
                      : launch(cope_prefill_sm100_batch<__half, 128, true>, 6))
                : (bf ? launch(cope_prefill_sm100_batch<__nv_bfloat16, 64, true>, 5)
                      : launch(cope_prefill_sm100_batch<__half, 64, true>, 4));
    else
      rc = wide ? (bf ? launch(cope_prefill_sm100_batch<__nv_bfloat16, 128, false>, 3)
                      : launch(cope_prefill_sm100_batch<__half, 128, false>, 2))
                : (bf ? launch(cope_prefill_sm100_batch<__nv_bfloat16, 64, false>, 1)
                      : launch(cope_prefill_sm100_batch<__half, 64, false>, 0));
    if (rc != CS_OK) return rc;
  }
  return CS_OK;
}
