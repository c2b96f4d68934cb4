// SLIDE paged KV data movement: gather, scatter and paged-to-paged relocate.
//
// Each (slot, kv_head) record is 2*D elements (K then V).  With the native
// layout [block, kv_head, offset, 2*D] and a contiguous innermost dimension a
// record is 2*D*esize contiguous bytes (512 for D=128 bf16); one warp moves a
// whole token row (every KV head) as aligned 16-byte vectors, several in
// flight per lane: fully coalesced, bit-exact.
// Views whose innermost stride is not 1 (or whose rows are not 16-byte
// aligned) take an element-wise path with the same semantics.
#include "common.cuh"

namespace cs {
namespace {

// 16-byte vector count per K or V half of a record
struct Geometry {
  int64_t n, heads, head_dim;
  int esize;
};

template <typename V>
__device__ __forceinline__ void move(char* dst, const char* src) {
  *reinterpret_cast<V*>(dst) = *reinterpret_cast<const V*>(src);
}

// gather: out[r] = record(slots[r]); unit = bytes moved per thread step
template <typename V>
__global__ void gather_kernel(PagedView pv, const int64_t* __restrict__ slots, int64_t n,
                              char* __restrict__ out_k, char* __restrict__ out_v,
                              int64_t o_row, int64_t o_head, int32_t* status) {
  const int64_t per_half = pv.head_dim * pv.esize / (int64_t)sizeof(V);
  const int64_t per_rec = 2 * per_half;
  const int64_t total = n * pv.kv_heads * per_rec;
  const int64_t elems_per_unit = (int64_t)sizeof(V) / pv.esize;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t rec = t / per_rec, u = t - rec * per_rec;
    int64_t r = rec / pv.kv_heads, h = rec - r * pv.kv_heads;
    int64_t s = slots[r];
    if (!pv.valid(s)) {
      if (u == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    int half = u >= per_half;
    int64_t within = (u - half * per_half) * elems_per_unit;
    const char* src = pv.addr(s, h, half * pv.head_dim + within);
    char* dst = (half ? out_v : out_k) + r * o_row + h * o_head + within * pv.esize;
    move<V>(dst, src);
  }
}

template <typename V>
__global__ void scatter_kernel(PagedView pv, const int64_t* __restrict__ slots,
                               const int64_t* __restrict__ rows, int64_t n,
                               const char* __restrict__ in_k, const char* __restrict__ in_v,
                               int64_t i_row, int64_t i_head, int32_t* status) {
  // a grid launched after this one as its programmatic dependent (the
  // decode's flag-zeroing grid) may start now; it waits for this grid's
  // completion before anything reads the rows written here
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t per_half = pv.head_dim * pv.esize / (int64_t)sizeof(V);
  const int64_t per_rec = 2 * per_half;
  const int64_t total = n * pv.kv_heads * per_rec;
  const int64_t elems_per_unit = (int64_t)sizeof(V) / pv.esize;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t rec = t / per_rec, u = t - rec * per_rec;
    int64_t r = rec / pv.kv_heads, h = rec - r * pv.kv_heads;
    int64_t s = slots[r];
    if (!pv.valid(s)) {
      if (u == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    int64_t src_row = rows ? rows[r] : r;
    int half = u >= per_half;
    int64_t within = (u - half * per_half) * elems_per_unit;
    const char* src = (half ? in_v : in_k) + src_row * i_row + h * i_head + within * pv.esize;
    move<V>(pv.addr(s, h, half * pv.head_dim + within), src);
  }
}

template <typename V>
__global__ void relocate_kernel(PagedView pv, const int64_t* __restrict__ src_slots,
                                const int64_t* __restrict__ dst_slots, int64_t n,
                                int32_t* status) {
  const int64_t per_half = pv.head_dim * pv.esize / (int64_t)sizeof(V);
  const int64_t per_rec = 2 * per_half;
  const int64_t total = n * pv.kv_heads * per_rec;
  const int64_t elems_per_unit = (int64_t)sizeof(V) / pv.esize;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t rec = t / per_rec, u = t - rec * per_rec;
    int64_t r = rec / pv.kv_heads, h = rec - r * pv.kv_heads;
    int64_t s = src_slots[r], d = dst_slots[r];
    if (!pv.valid(s) || !pv.valid(d)) {
      if (u == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    int64_t e = u * elems_per_unit;  // 0 .. 2D, never straddles the K|V split
    move<V>(pv.addr(d, h, e), pv.addr(s, h, e));
  }
}

// Row-per-warp paths for the common layout: a token row (all KV heads) is
// moved by one warp as 16-byte vectors, every lane holding UPL vectors of the
// K half and UPL of the V half in flight before it stores any; the slot is
// resolved once per row.  Used when a head's half-record is a power-of-two
// number of 16-byte vectors (UH) and the row's K half is 32 * UPL of them.
// Unit q of a row half: head q >> log2(UH), vector q & (UH - 1) of that head.
struct RowGeom {
  int uh_shift;  // log2(16-byte vectors per head half)
  int upl;       // vectors per lane per half: heads * UH / 32
};

__host__ bool row_geom(const PagedView& pv, RowGeom& g) {
  const int64_t uh = pv.head_dim * pv.esize / 16;
  if (uh < 1 || (uh & (uh - 1))) return false;
  const int64_t units = pv.kv_heads * uh;
  if (units % 32) return false;
  const int64_t upl = units / 32;
  if (upl != 1 && upl != 2 && upl != 4 && upl != 8) return false;
  int sh = 0;
  while ((1ll << sh) < uh) ++sh;
  g.uh_shift = sh;
  g.upl = (int)upl;
  return true;
}

// record of slots[r] = rows ? in[rows[r]] : in[r]
template <int UPL>
__global__ void __launch_bounds__(256) scatter_rows_kernel(
    PagedView pv, const int64_t* __restrict__ slots, const int64_t* __restrict__ rows, int64_t n,
    const char* __restrict__ in_k, const char* __restrict__ in_v, int64_t i_row, int64_t i_head,
    int uh_shift, int32_t* status) {
  // a grid launched after this one as its programmatic dependent (the
  // decode's flag-zeroing grid) may start now; it waits for this grid's
  // completion before anything reads the rows written here
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int uh_mask = (1 << uh_shift) - 1;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    const int64_t s = slots[r];
    if (!pv.valid(s)) {
      if (lane == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    const int64_t src = rows ? rows[r] : r;
    uint4 kx[UPL], vx[UPL];
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int q = lane + 32 * k;
      const int64_t off = src * i_row + (int64_t)(q >> uh_shift) * i_head + (q & uh_mask) * 16;
      kx[k] = *reinterpret_cast<const uint4*>(in_k + off);
      vx[k] = *reinterpret_cast<const uint4*>(in_v + off);
    }
    char *dk, *dv;
    int64_t hs;
    pv.record(s, dk, dv, hs);  // one block / sidecar lookup per row
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int q = lane + 32 * k;
      const int64_t off = (int64_t)(q >> uh_shift) * hs + (q & uh_mask) * 16;
      *reinterpret_cast<uint4*>(dk + off) = kx[k];
      *reinterpret_cast<uint4*>(dv + off) = vx[k];
    }
  }
}

// out[r] = record of slots[r]
template <int UPL>
__global__ void __launch_bounds__(256) gather_rows_kernel(
    PagedView pv, const int64_t* __restrict__ slots, int64_t n, char* __restrict__ out_k,
    char* __restrict__ out_v, int64_t o_row, int64_t o_head, int uh_shift, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int uh_mask = (1 << uh_shift) - 1;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    const int64_t s = slots[r];
    if (!pv.valid(s)) {
      if (lane == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    char *sk, *sv;
    int64_t hs;
    pv.record(s, sk, sv, hs);  // one block / sidecar lookup per row
    uint4 kx[UPL], vx[UPL];
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int q = lane + 32 * k;
      const int64_t off = (int64_t)(q >> uh_shift) * hs + (q & uh_mask) * 16;
      kx[k] = *reinterpret_cast<const uint4*>(sk + off);
      vx[k] = *reinterpret_cast<const uint4*>(sv + off);
    }
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int q = lane + 32 * k;
      const int64_t off = r * o_row + (int64_t)(q >> uh_shift) * o_head + (q & uh_mask) * 16;
      *reinterpret_cast<uint4*>(out_k + off) = kx[k];
      *reinterpret_cast<uint4*>(out_v + off) = vx[k];
    }
  }
}

// record of dst_slots[r] = record of src_slots[r]
template <int UPL>
__global__ void __launch_bounds__(256) relocate_rows_kernel(
    PagedView pv, const int64_t* __restrict__ src_slots, const int64_t* __restrict__ dst_slots,
    int64_t n, int uh_shift, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int uh_mask = (1 << uh_shift) - 1;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    const int64_t s = src_slots[r], d = dst_slots[r];
    if (!pv.valid(s) || !pv.valid(d)) {
      if (lane == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    char *sk, *sv, *dk, *dv;
    int64_t shs, dhs;
    pv.record(s, sk, sv, shs);  // one block / sidecar lookup per row and side
    pv.record(d, dk, dv, dhs);
    uint4 kx[UPL], vx[UPL];
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int q = lane + 32 * k;
      const int64_t off = (int64_t)(q >> uh_shift) * shs + (q & uh_mask) * 16;
      kx[k] = *reinterpret_cast<const uint4*>(sk + off);
      vx[k] = *reinterpret_cast<const uint4*>(sv + off);
    }
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int q = lane + 32 * k;
      const int64_t off = (int64_t)(q >> uh_shift) * dhs + (q & uh_mask) * 16;
      *reinterpret_cast<uint4*>(dk + off) = kx[k];
      *reinterpret_cast<uint4*>(dv + off) = vx[k];
    }
  }
}

// Several requests' scatters in one launch: request i owns the global rows
// [start[i], start[i + 1]); a warp finds its request by binary search over
// the prefix (uniform across the warp, read from the parameter space).
constexpr int kBatch = kBatchItems;

struct ScatterRows {
  const int64_t* slots;
  const int64_t* rows;
  const char* k;
  const char* v;
  int64_t irow, ihead;  // byte strides
  int32_t* status;
};

struct ScatterBatch {
  ScatterRows it[kBatch];
  int64_t start[kBatch + 1];
  int count;
};

template <int UPL>
__global__ void __launch_bounds__(256) scatter_rows_batch_kernel(
    PagedView pv, const __grid_constant__ ScatterBatch b, int uh_shift) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int uh_mask = (1 << uh_shift) - 1;
  const int64_t total = b.start[b.count];
  for (int64_t g = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); g < total;
       g += warps) {
    const int i = batch_item(b.start, b.count, g);
    const ScatterRows& q = b.it[i];
    const int64_t r = g - b.start[i];
    const int64_t s = q.slots[r];
    if (!pv.valid(s)) {
      if (lane == 0) report(q.status, CS_ST_SLOT_RANGE);
      continue;
    }
    const int64_t src = q.rows ? q.rows[r] : r;
    uint4 kx[UPL], vx[UPL];
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int u = lane + 32 * k;
      const int64_t off = src * q.irow + (int64_t)(u >> uh_shift) * q.ihead + (u & uh_mask) * 16;
      kx[k] = *reinterpret_cast<const uint4*>(q.k + off);
      vx[k] = *reinterpret_cast<const uint4*>(q.v + off);
    }
    char *dk, *dv;
    int64_t hs;
    pv.record(s, dk, dv, hs);  // one block / sidecar lookup per row
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int u = lane + 32 * k;
      const int64_t off = (int64_t)(u >> uh_shift) * hs + (u & uh_mask) * 16;
      *reinterpret_cast<uint4*>(dk + off) = kx[k];
      *reinterpret_cast<uint4*>(dv + off) = vx[k];
    }
  }
}

// Page images for spill / reload: page q of the list is the block_size
// consecutive slots pages[q] * bs .. + bs - 1 (a native block, or sidecar
// rows), laid out as one native block [kv_head][offset][2D] in `img` (the
// record format of the cache itself).  One warp per slot row; pack copies
// records into the image, unpack writes them back.
template <int UPL, bool kPack>
__global__ void __launch_bounds__(256) page_image_kernel(
    PagedView pv, const int64_t* __restrict__ pages, int64_t count, char* img, int uh_shift,
    int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int uh_mask = (1 << uh_shift) - 1;
  const int64_t rows = count * pv.bs;
  const int64_t half = pv.head_dim * pv.esize;                 // bytes of a K or V half
  const int64_t img_head = pv.bs * 2 * half, img_page = pv.kv_heads * img_head;
  for (int64_t g = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); g < rows;
       g += warps) {
    const int64_t q = g / pv.bs, o = g - q * pv.bs;
    const int64_t first = pages[q] * pv.bs, s = first + o;
    if (pages[q] < 0 || !pv.valid(first)) {  // the page is not in the arena
      if (lane == 0 && o == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    char* base = img + q * img_page + o * 2 * half;
    if (!pv.valid(s)) {  // past the end of a partial sidecar page: zeros in the image
      if constexpr (kPack) {
        for (int64_t h = 0; h < pv.kv_heads; ++h)
          for (int64_t b = lane * 16; b < 2 * half; b += 32 * 16)
            *reinterpret_cast<uint4*>(base + h * img_head + b) = make_uint4(0, 0, 0, 0);
      }
      continue;
    }
    char *rk, *rv;
    int64_t hs;
    pv.record(s, rk, rv, hs);
    uint4 kx[UPL], vx[UPL];
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int u = lane + 32 * k;
      const int64_t h = u >> uh_shift, off = (int64_t)(u & uh_mask) * 16;
      if constexpr (kPack) {
        kx[k] = *reinterpret_cast<const uint4*>(rk + h * hs + off);
        vx[k] = *reinterpret_cast<const uint4*>(rv + h * hs + off);
      } else {
        kx[k] = *reinterpret_cast<const uint4*>(base + h * img_head + off);
        vx[k] = *reinterpret_cast<const uint4*>(base + h * img_head + half + off);
      }
    }
#pragma unroll
    for (int k = 0; k < UPL; ++k) {
      const int u = lane + 32 * k;
      const int64_t h = u >> uh_shift, off = (int64_t)(u & uh_mask) * 16;
      if constexpr (kPack) {
        *reinterpret_cast<uint4*>(base + h * img_head + off) = kx[k];
        *reinterpret_cast<uint4*>(base + h * img_head + half + off) = vx[k];
      } else {
        *reinterpret_cast<uint4*>(rk + h * hs + off) = kx[k];
        *reinterpret_cast<uint4*>(rv + h * hs + off) = vx[k];
      }
    }
  }
}

// the same page images for any view: one thread per element
template <typename V, bool kPack>
__global__ void page_image_elem_kernel(PagedView pv, const int64_t* __restrict__ pages,
                                       int64_t count, char* img, int32_t* status) {
  const int64_t d2 = 2 * pv.head_dim;
  const int64_t total = count * pv.kv_heads * pv.bs * d2;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    // image element t = ((q * kv_heads + h) * bs + o) * 2D + e
    const int64_t e = t % d2, rest = t / d2;
    const int64_t o = rest % pv.bs, qh = rest / pv.bs;
    const int64_t h = qh % pv.kv_heads, q = qh / pv.kv_heads;
    const int64_t first = pages[q] * pv.bs, s = first + o;
    V* dst = reinterpret_cast<V*>(img) + t;
    if (pages[q] < 0 || !pv.valid(first)) {
      if (e == 0 && o == 0 && h == 0) report(status, CS_ST_SLOT_RANGE);
      continue;
    }
    if (!pv.valid(s)) {
      if constexpr (kPack) *dst = V(0);
      continue;
    }
    V* rec = reinterpret_cast<V*>(pv.addr(s, h, e));
    if constexpr (kPack) *dst = *rec;
    else *rec = *dst;
  }
}

// warps for n rows: one row per warp up to 16 CTAs of 8 warps per SM
int row_grid_for(int64_t n) {
  int64_t blocks = (n + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

int grid_for(int64_t units, int threads) {
  int64_t blocks = (units + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

bool aligned16(const void* p, int64_t a, int64_t b) {
  return (reinterpret_cast<uintptr_t>(p) % 16 == 0) && (a % 16 == 0) && (b % 16 == 0);
}

bool check_view(const cs_paged_kv* kv) {
  return kv && kv->cache && kv->num_blocks > 0 && kv->kv_heads > 0 && kv->block_size > 0 &&
         kv->head_dim > 0 && dtype_size(kv->dtype) > 0;
}

}  // namespace
}  // namespace cs

using namespace cs;

extern "C" int cs_slide_gather(const cs_paged_kv* kv, const int64_t* slots, int64_t n,
                               void* out_k, void* out_v, int64_t out_stride_row,
                               int64_t out_stride_head, int32_t* status, void* stream) {
  CS_HOST_CHECK(check_view(kv) && n >= 0);
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(slots && out_k && out_v);
  PagedView pv = PagedView::make(*kv);
  const int64_t orow = out_stride_row * pv.esize, ohead = out_stride_head * pv.esize;
  const int threads = 256;
  RowGeom rg{};
  if (pv.vec16() && aligned16(out_k, orow, ohead) && aligned16(out_v, orow, ohead) &&
      row_geom(pv, rg)) {
    auto go = [&](auto kern) {
      kern<<<row_grid_for(n), 256, 0, as_stream(stream)>>>(pv, slots, n, (char*)out_k,
                                                           (char*)out_v, orow, ohead,
                                                           rg.uh_shift, status);
    };
    switch (rg.upl) {
      case 1: go(gather_rows_kernel<1>); break;
      case 2: go(gather_rows_kernel<2>); break;
      case 4: go(gather_rows_kernel<4>); break;
      default: go(gather_rows_kernel<8>); break;
    }
  } else if (pv.vec16() && aligned16(out_k, orow, ohead) && aligned16(out_v, orow, ohead)) {
    int64_t units = n * pv.kv_heads * 2 * (pv.head_dim * pv.esize / 16);
    gather_kernel<uint4><<<grid_for(units, threads), threads, 0, as_stream(stream)>>>(
        pv, slots, n, (char*)out_k, (char*)out_v, orow, ohead, status);
  } else {
    int64_t units = n * pv.kv_heads * 2 * pv.head_dim;
    int g = grid_for(units, threads);
    auto s = as_stream(stream);
    switch (pv.esize) {
      case 2: gather_kernel<uint16_t><<<g, threads, 0, s>>>(pv, slots, n, (char*)out_k, (char*)out_v, orow, ohead, status); break;
      case 4: gather_kernel<uint32_t><<<g, threads, 0, s>>>(pv, slots, n, (char*)out_k, (char*)out_v, orow, ohead, status); break;
      default: gather_kernel<uint64_t><<<g, threads, 0, s>>>(pv, slots, n, (char*)out_k, (char*)out_v, orow, ohead, status); break;
    }
  }
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_slide_scatter(const cs_paged_kv* kv, const int64_t* slots, const int64_t* rows,
                                int64_t n, const void* k, const void* v, int64_t in_stride_row,
                                int64_t in_stride_head, int32_t* status, void* stream) {
  CS_HOST_CHECK(check_view(kv) && n >= 0);
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(slots && k && v);
  PagedView pv = PagedView::make(*kv);
  const int64_t irow = in_stride_row * pv.esize, ihead = in_stride_head * pv.esize;
  const int threads = 256;
  auto s = as_stream(stream);
  RowGeom rg{};
  if (pv.vec16() && aligned16(k, irow, ihead) && aligned16(v, irow, ihead) && row_geom(pv, rg)) {
    auto go = [&](auto kern) {
      kern<<<row_grid_for(n), 256, 0, s>>>(pv, slots, rows, n, (const char*)k, (const char*)v,
                                           irow, ihead, rg.uh_shift, status);
    };
    switch (rg.upl) {
      case 1: go(scatter_rows_kernel<1>); break;
      case 2: go(scatter_rows_kernel<2>); break;
      case 4: go(scatter_rows_kernel<4>); break;
      default: go(scatter_rows_kernel<8>); break;
    }
  } else if (pv.vec16() && aligned16(k, irow, ihead) && aligned16(v, irow, ihead)) {
    int64_t units = n * pv.kv_heads * 2 * (pv.head_dim * pv.esize / 16);
    scatter_kernel<uint4><<<grid_for(units, threads), threads, 0, s>>>(
        pv, slots, rows, n, (const char*)k, (const char*)v, irow, ihead, status);
  } else {
    int64_t units = n * pv.kv_heads * 2 * pv.head_dim;
    int g = grid_for(units, threads);
    switch (pv.esize) {
      case 2: scatter_kernel<uint16_t><<<g, threads, 0, s>>>(pv, slots, rows, n, (const char*)k, (const char*)v, irow, ihead, status); break;
      case 4: scatter_kernel<uint32_t><<<g, threads, 0, s>>>(pv, slots, rows, n, (const char*)k, (const char*)v, irow, ihead, status); break;
      default: scatter_kernel<uint64_t><<<g, threads, 0, s>>>(pv, slots, rows, n, (const char*)k, (const char*)v, irow, ihead, status); break;
    }
  }
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_slide_relocate(const cs_paged_kv* kv, const int64_t* src_slots,
                                 const int64_t* dst_slots, int64_t n, int32_t* status,
                                 void* stream) {
  CS_HOST_CHECK(check_view(kv) && n >= 0);
  if (n == 0) return CS_OK;
  CS_HOST_CHECK(src_slots && dst_slots);
  PagedView pv = PagedView::make(*kv);
  const int threads = 256;
  auto s = as_stream(stream);
  RowGeom rg{};
  if (pv.vec16() && row_geom(pv, rg)) {
    auto go = [&](auto kern) {
      kern<<<row_grid_for(n), 256, 0, s>>>(pv, src_slots, dst_slots, n, rg.uh_shift, status);
    };
    switch (rg.upl) {
      case 1: go(relocate_rows_kernel<1>); break;
      case 2: go(relocate_rows_kernel<2>); break;
      case 4: go(relocate_rows_kernel<4>); break;
      default: go(relocate_rows_kernel<8>); break;
    }
  } else if (pv.vec16()) {
    int64_t units = n * pv.kv_heads * 2 * (pv.head_dim * pv.esize / 16);
    relocate_kernel<uint4><<<grid_for(units, threads), threads, 0, s>>>(pv, src_slots, dst_slots, n,
                                                                         status);
  } else {
    int64_t units = n * pv.kv_heads * 2 * pv.head_dim;
    int g = grid_for(units, threads);
    switch (pv.esize) {
      case 2: relocate_kernel<uint16_t><<<g, threads, 0, s>>>(pv, src_slots, dst_slots, n, status); break;
      case 4: relocate_kernel<uint32_t><<<g, threads, 0, s>>>(pv, src_slots, dst_slots, n, status); break;
      default: relocate_kernel<uint64_t><<<g, threads, 0, s>>>(pv, src_slots, dst_slots, n, status); break;
    }
  }
  CS_LAUNCH_CHECK();
  return CS_OK;
}

extern "C" int cs_slide_scatter_batch(const cs_paged_kv* kv, const cs_slide_scatter_item* items,
                                      int32_t count, void* stream) {
  CS_HOST_CHECK(check_view(kv) && count >= 0 && (count == 0 || items));
  PagedView pv = PagedView::make(*kv);
  RowGeom rg{};
  bool rows_path = pv.vec16() && row_geom(pv, rg);
  for (int32_t i = 0; i < count; ++i) {
    const cs_slide_scatter_item& it = items[i];
    CS_HOST_CHECK(it.n >= 0 && (it.n == 0 || (it.slots && it.k && it.v)));
    const int64_t irow = it.in_stride_row * pv.esize, ihead = it.in_stride_head * pv.esize;
    if (it.n > 0 && !(aligned16(it.k, irow, ihead) && aligned16(it.v, irow, ihead)))
      rows_path = false;
  }
  if (!rows_path) {  // the general layouts: one launch per request
    for (int32_t i = 0; i < count; ++i) {
      const cs_slide_scatter_item& it = items[i];
      const int rc = cs_slide_scatter(kv, it.slots, it.rows, it.n, it.k, it.v, it.in_stride_row,
                                      it.in_stride_head, it.status, stream);
      if (rc != CS_OK) return rc;
    }
    return CS_OK;
  }
  auto s = as_stream(stream);
  for (int32_t first = 0; first < count; first += kBatch) {
    ScatterBatch b{};  // copied into the kernel's parameter space by the launch
    b.count = count - first < kBatch ? count - first : kBatch;
    b.start[0] = 0;
    for (int j = 0; j < b.count; ++j) {
      const cs_slide_scatter_item& it = items[first + j];
      b.it[j] = ScatterRows{it.slots, it.rows, static_cast<const char*>(it.k),
                            static_cast<const char*>(it.v), it.in_stride_row * pv.esize,
                            it.in_stride_head * pv.esize, it.status};
      b.start[j + 1] = b.start[j] + it.n;
    }
    const int64_t total = b.start[b.count];
    if (total == 0) continue;
    auto go = [&](auto kern) { kern<<<row_grid_for(total), 256, 0, s>>>(pv, b, rg.uh_shift); };
    switch (rg.upl) {
      case 1: go(scatter_rows_batch_kernel<1>); break;
      case 2: go(scatter_rows_batch_kernel<2>); break;
      case 4: go(scatter_rows_batch_kernel<4>); break;
      default: go(scatter_rows_batch_kernel<8>); break;
    }
    CS_LAUNCH_CHECK();
  }
  return CS_OK;
}

namespace {
int page_images(const cs_paged_kv* kv, const int64_t* pages, int64_t count, void* image,
                int32_t* status, void* stream, bool pack) {
  CS_HOST_CHECK(check_view(kv) && count >= 0);
  if (count == 0) return CS_OK;
  CS_HOST_CHECK(pages && image);
  PagedView pv = PagedView::make(*kv);
  RowGeom rg{};
  auto s = as_stream(stream);
  if (!pv.vec16() || !row_geom(pv, rg) || (reinterpret_cast<uintptr_t>(image) & 15)) {
    const int64_t units = count * pv.kv_heads * pv.bs * 2 * pv.head_dim;
    const int g = grid_for(units, 256);
    char* img = static_cast<char*>(image);
    switch (pv.esize) {
      case 2: pack ? page_image_elem_kernel<uint16_t, true><<<g, 256, 0, s>>>(pv, pages, count, img, status)
                   : page_image_elem_kernel<uint16_t, false><<<g, 256, 0, s>>>(pv, pages, count, img, status); break;
      case 4: pack ? page_image_elem_kernel<uint32_t, true><<<g, 256, 0, s>>>(pv, pages, count, img, status)
                   : page_image_elem_kernel<uint32_t, false><<<g, 256, 0, s>>>(pv, pages, count, img, status); break;
      default: pack ? page_image_elem_kernel<uint64_t, true><<<g, 256, 0, s>>>(pv, pages, count, img, status)
                    : page_image_elem_kernel<uint64_t, false><<<g, 256, 0, s>>>(pv, pages, count, img, status); break;
    }
    CS_LAUNCH_CHECK();
    return CS_OK;
  }
  const int64_t rows = count * pv.bs;
  auto go = [&](auto kern) {
    kern<<<row_grid_for(rows), 256, 0, s>>>(pv, pages, count, static_cast<char*>(image),
                                            rg.uh_shift, status);
  };
  switch (rg.upl) {
    case 1: pack ? go(page_image_kernel<1, true>) : go(page_image_kernel<1, false>); break;
    case 2: pack ? go(page_image_kernel<2, true>) : go(page_image_kernel<2, false>); break;
    case 4: pack ? go(page_image_kernel<4, true>) : go(page_image_kernel<4, false>); break;
    default: pack ? go(page_image_kernel<8, true>) : go(page_image_kernel<8, false>); break;
  }
  CS_LAUNCH_CHECK();
  return CS_OK;
}
}  // namespace

extern "C" int cs_slide_pack_pages(const cs_paged_kv* kv, const int64_t* pages, int64_t count,
                                   void* image, int32_t* status, void* stream) {
  return page_images(kv, pages, count, image, status, stream, true);
}

extern "C" int cs_slide_unpack_pages(const cs_paged_kv* kv, const int64_t* pages, int64_t count,
                                     const void* image, int32_t* status, void* stream) {
  return page_images(kv, pages, count, const_cast<void*>(image), status, stream, false);
}
