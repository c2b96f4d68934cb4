// Selective layer loop on the tensor cores (sm_100a): the QKV projection of
// a layer's active rows only, with the rows gathered on the fly and the LoRA
// delta in the same accumulator (runtime.py:409-460, artifacts.py:189-193):
//
//   out[r] = x_r W^T + bf16(x_r A^T) B^T,   x_r = src_{row_src[r]}[row_idx[r]]
//
// where src0 is the previous layer's output (rows that continue) and src1
// the layer's input snapshot (rows newly selected, restored).  The reference
// first builds the gathered hidden states with index copies, then runs the
// projection and the two LoRA linears separately.
//
// One CTA computes a 128 x 256 tile of `out` (128 active rows x 256 output
// features); the K loop runs over the hidden size in blocks of 64 through a
// four-stage shared-memory ring:
//   warps 0-3  producer: each thread copies one gathered row of the A block
//              (its source row resolved once), two rows of the W block and a
//              share of the LoRA-A block with cp.async into the 128-byte
//              swizzled K-major UMMA layout; one cp.async-completion arrival
//              per thread fills a stage.  After the K loop the same warps
//              are the epilogue (TMEM lane = tile row).
//   warp 4     MMA issuer (one thread) and TMEM owner: per stage four
//              K = 16 steps of D += A W^T (M = 128, N = 256) and, with LoRA,
//              of T += A A_lora^T (N = 16 or 32); each stage's MMAs are
//              committed to the stage's "empty" barrier.
// Then the epilogue warps read T, round it to 16 bits into shared memory
// (the A operand of one more MMA chain against the B_lora block), the MMA
// thread adds T B_lora^T into D, and the epilogue writes D as 16-bit rows.
// TMEM: D in columns [0, 256), T in [256, 256 + TR).  Every wait is bounded;
// on expiry the CTA sets CS_ST_TIMEOUT and returns after draining.
#include "common.cuh"
#include "sm100.cuh"

namespace cs {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kThreads = 5 * 32;  // 4 producer / epilogue warps + 1 MMA warp
constexpr uint32_t kStageA = kBM * 128;   // 16 KB: 128 rows x 64 elements
constexpr uint32_t kStageB = kBN * 128;   // 32 KB: 256 rows x 64 elements
constexpr uint32_t kStageL = 32 * 128;    // 4 KB: up to 32 LoRA-A rows
constexpr uint32_t kA = 0;
constexpr uint32_t kB = kA + kStages * kStageA;   // 65536
constexpr uint32_t kL = kB + kStages * kStageB;   // 196608
constexpr uint32_t kMeta = kL + kStages * kStageL;  // 212992
constexpr uint32_t kFull = 0, kEmpty = 32, kTReady = 64, kLoraDone = 72, kSlot = 80,
                   kAbortFlag = 84, kMetaBytes = 128;
constexpr uint32_t kSmem = kMeta + kMetaBytes + 1024;  // + alignment slack

template <typename T> struct Pk;
template <> struct Pk<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct Pk<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    qkv_gather_lora_kernel(const __grid_constant__ cs_qkv_params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint8_t* meta = smem + kMeta;
  const uint32_t mb = sbase + kMeta;
  volatile int* abort = reinterpret_cast<volatile int*>(meta + kAbortFlag);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.x * kBM, n0 = (int64_t)blockIdx.y * kBN;
  // rows: a, or a count in device memory (at most a); a CTA whose rows all
  // lie past it leaves before any barrier or TMEM use (a uniform exit)
  int64_t arows = p.a;
  if (p.a_dev != nullptr) {
    const int64_t c = __ldg(p.a_dev);
    arows = c < 0 ? 0 : (c < arows ? c : arows);
  }
  if (m0 >= arows) return;
  const int nk = (int)(p.hidden / kBK);
  const int TR = p.rank > 16 ? 32 : 16;  // LoRA columns of T (padded)
  const bool lora = p.rank > 0;
  const int fmt = p.dtype == CS_BF16 ? 1 : 0;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(mb + kFull + 8 * s, 128);
      mbar_init(mb + kEmpty + 8 * s, 1);
    }
    mbar_init(mb + kTReady, 128);
    mbar_init(mb + kLoraDone, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == 4) tmem_alloc(mb + kSlot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(meta + kSlot);

  if (warp < 4) {
    // ============================================================ producer
    const int r = tid;  // the A row this thread copies
    const int64_t row = m0 + r;
    const char* arow = nullptr;
    if (row < arows) {
      const int src = p.row_src[row];
      const int64_t idx = p.row_idx[row];
      const bool ok = src == 0 ? (idx >= 0 && idx < p.src0_rows) : (idx >= 0 && idx < p.src1_rows);
      if (ok) {
        arow = static_cast<const char*>(src == 0 ? p.src0 : p.src1) +
               idx * (src == 0 ? p.src0_stride : p.src1_stride) * (int64_t)sizeof(T);
      } else if (p.status) {
        report(p.status, CS_ST_SLOT_RANGE);
      }
    }
    const char* w = static_cast<const char*>(p.w);
    const char* la = static_cast<const char*>(p.lora_a);
    bool ok = true;
    for (int kt = 0; kt < nk && ok; ++kt) {
      const int s = kt % kStages;
      if (kt >= kStages) ok = mbar_wait(mb + kEmpty + 8 * s, ((kt / kStages) - 1) & 1, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      const int64_t kb = (int64_t)kt * kBK * (int64_t)sizeof(T);  // byte offset in a row
      const uint32_t sa = sbase + kA + s * kStageA, sb = sbase + kB + s * kStageB;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        cp_async16(sa + sw128(r, c, kBM), arow ? arow + kb + c * 16 : p.w, arow != nullptr);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int br = r + 128 * h;
        const char* wrow = w + (n0 + br) * p.hidden * (int64_t)sizeof(T) + kb;
#pragma unroll
        for (int c = 0; c < 8; ++c) cp_async16(sb + sw128(br, c, kBN), wrow + c * 16, true);
      }
      if (lora) {
        const uint32_t sl = sbase + kL + s * kStageL;
        for (int u = r; u < TR * 8; u += 128) {
          const int lr = u >> 3, c = u & 7;
          const bool v = lr < p.rank;
          cp_async16(sl + sw128(lr, c, TR),
                     v ? la + (int64_t)lr * p.hidden * (int64_t)sizeof(T) + kb + c * 16 : p.w, v);
        }
      }
      cp_async_arrive_noinc(mb + kFull + 8 * s);
    }
    cp_async_wait_all();
    // ============================================================ epilogue
    const int last = nk - 1;
    ok = ok && mbar_wait(mb + kEmpty + 8 * (last % kStages), (last / kStages) & 1, abort);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (ok && lora) {
      // T row -> 16-bit A operand (stage 0's A block, free once every MMA
      // has completed); B_lora block -> stage 0's B block
      uint32_t v[32];
      if (TR == 16) {
        CS_TMEM_LD16(tmem + lane_base + kBN, v);
      } else {
        CS_TMEM_LD32(tmem + lane_base + kBN, v);
      }
      tmem_wait_ld();
      uint8_t* ta = smem + kA;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c >= TR / 8) break;
        uint32_t w4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w4[j] = Pk<T>::pack(__uint_as_float(v[8 * c + 2 * j]), __uint_as_float(v[8 * c + 2 * j + 1]));
        *reinterpret_cast<uint4*>(ta + sw128(r, c, kBM)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      uint8_t* tb = smem + kB;
      const char* lb = static_cast<const char*>(p.lora_b);
      for (int h = 0; h < 2; ++h) {
        const int br = r + 128 * h;
        const char* brow = lb + (n0 + br) * (int64_t)p.rank * (int64_t)sizeof(T);
        for (int c = 0; c < TR / 8; ++c) {
          uint4 x = make_uint4(0, 0, 0, 0);
          if (c * 8 < p.rank) x = *reinterpret_cast<const uint4*>(brow + c * 16);
          *reinterpret_cast<uint4*>(tb + sw128(br, c, kBN)) = x;
        }
      }
      fence_async_smem();  // the generic-proxy stores, visible to the MMA
      tc_fence_before();
      mbar_arrive(mb + kTReady);
      ok = __all_sync(0xffffffffu, mbar_wait(mb + kLoraDone, 0, abort));
      tc_fence_after();
    }
    if (ok) {
      const int64_t orow = m0 + r;
      char* out = static_cast<char*>(p.out) + orow * p.out_stride * (int64_t)sizeof(T) +
                  n0 * (int64_t)sizeof(T);
#pragma unroll 1
      for (int cc = 0; cc < kBN / 32; ++cc) {
        uint32_t v[32];
        CS_TMEM_LD32(tmem + lane_base + 32 * cc, v);
        tmem_wait_ld();
        if (orow < arows) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              w4[j] = Pk<T>::pack(__uint_as_float(v[8 * q + 2 * j]),
                                  __uint_as_float(v[8 * q + 2 * j + 1]));
            *reinterpret_cast<uint4*>(out + (cc * 32 + q * 8) * (int64_t)sizeof(T)) =
                make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
    }
  } else {
    if (lane == 0) {
    // ================================================================= MMA
    const uint32_t id_d = umma_idesc(kBM, kBN, fmt, 0, 0);
    const uint32_t id_t = umma_idesc(kBM, TR, fmt, 0, 0);
    bool ok = true;
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % kStages;
      if (!(ok = mbar_wait(mb + kFull + 8 * s, (kt / kStages) & 1, abort))) break;
      tc_fence_after();
      const uint32_t sa = sbase + kA + s * kStageA, sb = sbase + kB + s * kStageB;
      const uint32_t sl = sbase + kL + s * kStageL;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        tc_mma(tmem, umma_desc(sa + kk * 32, 16, 1024), umma_desc(sb + kk * 32, 16, 1024), id_d,
               (kt | kk) ? 1u : 0u);
        if (lora)
          tc_mma(tmem + kBN, umma_desc(sa + kk * 32, 16, 1024),
                 umma_desc(sl + kk * 32, 16, 1024), id_t, (kt | kk) ? 1u : 0u);
      }
      tc_commit(mb + kEmpty + 8 * s);
    }
    if (ok && lora && (ok = mbar_wait(mb + kTReady, 0, abort))) {
      tc_fence_after();
      for (int kk = 0; kk < TR / 16; ++kk)
        tc_mma(tmem, umma_desc(sbase + kA + kk * 32, 16, 1024),
               umma_desc(sbase + kB + kk * 32, 16, 1024), id_d, 1u);
      tc_commit(mb + kLoraDone);
    }
    // drain before TMEM is released: every issued MMA has completed once
    // its group's barrier has (MMAs of one thread complete in order)
    if (!ok) {
      tc_commit(mb + kLoraDone);
      const long long t0 = clock64();
      while (!mbar_try(mb + kLoraDone, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
    }
    __syncwarp();
  }
  if (*abort && tid == 0 && p.status) report(p.status, CS_ST_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace cs

using namespace cs;

extern "C" int cs_qkv_gather_lora(const cs_qkv_params* p, void* stream) {
  CS_HOST_CHECK(p && p->a >= 0 && p->hidden > 0 && p->n_out > 0 && p->rank >= 0);
  CS_HOST_CHECK(p->dtype == CS_BF16 || p->dtype == CS_F16);
  if (p->hidden % 64 || p->n_out % 256 || p->rank > 32 || p->rank % 8) return CS_ERR_UNSUPPORTED;
  if (p->a == 0) return CS_OK;
  CS_HOST_CHECK(p->src0 || p->src1);
  CS_HOST_CHECK(p->row_src && p->row_idx && p->w && p->out);
  CS_HOST_CHECK(p->rank == 0 || (p->lora_a && p->lora_b));
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al(p->src0) || !al(p->src1) || !al(p->w) || !al(p->out) || !al(p->lora_a) ||
      !al(p->lora_b) || p->src0_stride % 8 || p->src1_stride % 8 || p->out_stride % 8)
    return CS_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)((p->a + kBM - 1) / kBM), (unsigned)(p->n_out / kBN));
  auto s = as_stream(stream);
  auto go = [&](auto kern) -> int {
    static bool ready[2] = {false, false};
    const int which = p->dtype == CS_BF16;
    if (!ready[which]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
          cudaSuccess)
        return CS_ERR_CUDA;
      ready[which] = true;
    }
    kern<<<grid, kThreads, kSmem, s>>>(*p);
    CS_LAUNCH_CHECK();
    return CS_OK;
  };
  return p->dtype == CS_BF16 ? go(qkv_gather_lora_kernel<__nv_bfloat16>)
                             : go(qkv_gather_lora_kernel<__half>);
}
