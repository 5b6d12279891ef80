// Row GEMM of the general route on tcgen05 tensor cores:
//   C[rows, n] (fp32, row-major, ldc) = A[rows, k] (row-major, lda) * B^T + beta C,
// with element (j, kk) of B at Bm[j * ldbn + kk * ldbk].  These are the
// general route's stem projection, drive projection and synthesis: tall and
// skinny (rows = B T tokens, n and k <= 128), so the whole B operand stays in
// shared memory for the life of a persistent CTA and the CTA walks 128-row
// tiles of A.
//
// Precision:
//   * A and B bf16: one bf16 x bf16 MMA per K step, fp32 accumulation (the
//     products are exact);
//   * A and B fp32: each operand is split x = hi + lo with hi, lo in bf16 and
//     every K step issues hi*hi + hi*lo + lo*hi into the fp32 accumulator: the
//     dropped lo*lo term and the split residual are ~2^-16 relative, fp32-level
//     accuracy on bf16 tensor cores (the fp32 parity gate is 1e-4).
//
// Per tile: 256 threads load the A tile (zero past `rows` and past k), convert
// or split it into K-major no-swizzle slabs (element (r, kk) at
// ((kk / 8) * 128 + r) * 8 + kk % 8), one thread issues the MMAs, every thread
// waits on an mbarrier (bounded) and the epilogue moves the accumulator out in
// 32-column chunks through a shared-memory staging tile (TMEM loads at
// 16-column-aligned offsets), adding beta C, with coalesced row-segment stores.  The next
// tile's A rows are loaded into registers while the MMAs run.
#pragma once

#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace lnet {

constexpr int kRgRows = 128, kRgThreads = 256;
// Shapes served: n, k <= 128.  This kernel carries one tile at a time per SM; it
// serves the operands the warp-specialised kernel below cannot address by TMA
// (unaligned bases, row pitches that are not multiples of 16 bytes).
constexpr int kRgMaxN = 128, kRgMaxK = 128;
constexpr int kRgSmemLimit = 227 * 1024;
constexpr int kRgStagePitch = 36;  // floats per staged row of a 32-column chunk (bank spread)
constexpr int kRgStageBytes = kRgRows * kRgStagePitch * 4;

__host__ __device__ constexpr int rg_pad16(int v) { return (v + 15) / 16 * 16; }

struct RowGemmShape {
  int n_pad, k_pad, parts;  // parts = 1 (bf16) or 2 (hi, lo)
  int b_bytes() const { return parts * n_pad * k_pad * 2; }
  int a_bytes() const { return parts * kRgRows * k_pad * 2; }
  int smem() const { return b_bytes() + a_bytes() + kRgStageBytes + 64; }
};

// (hi, lo) bf16 split of a float.
__device__ __forceinline__ void rg_split(float x, __nv_bfloat16 &hi, __nv_bfloat16 &lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

template <bool SPLIT>
__global__ void __launch_bounds__(kRgThreads, 1) rowgemm_kernel(
    const void *__restrict__ A, int64_t lda, const void *__restrict__ Bm, int64_t ldbn,
    int64_t ldbk, float *__restrict__ C, int64_t ldc, int64_t rows, int n, int k, float beta,
    int n_pad, int k_pad, uint32_t *__restrict__ status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int P = SPLIT ? 2 : 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b_part = n_pad * k_pad * 2, a_part = kRgRows * k_pad * 2;
  uint8_t *b_s = smem, *a_s = smem + P * b_part;
  float *stage = reinterpret_cast<float *>(a_s + P * a_part);
  uint64_t *mbar = reinterpret_cast<uint64_t *>(a_s + P * a_part + kRgStageBytes);
  uint32_t *tslot = reinterpret_cast<uint32_t *>(a_s + P * a_part + kRgStageBytes + 8);
  if (tid == 0) {
    sm100::mbar_init(mbar, 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 256);
    sm100::tmem_relinquish();
  }
  // B once: element (j, kk) of part p at p * b_part + (((kk / 8) * n_pad + j) * 8 + kk % 8) * 2
  for (int e = tid; e < n_pad * k_pad; e += kRgThreads) {
    const int j = e / k_pad, kk = e - j * k_pad;
    float v = 0.f;
    if (j < n && kk < k) {
      const int64_t off = (int64_t)j * ldbn + (int64_t)kk * ldbk;
      v = SPLIT ? reinterpret_cast<const float *>(Bm)[off]
                : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(Bm)[off]);
    }
    __nv_bfloat16 hi, lo;
    rg_split(v, hi, lo);
    const int idx = (((kk >> 3) * n_pad + j) << 3) + (kk & 7);
    reinterpret_cast<__nv_bfloat16 *>(b_s)[idx] = hi;
    if (SPLIT) reinterpret_cast<__nv_bfloat16 *>(b_s + b_part)[idx] = lo;
  }
  sm100::fence_proxy_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tslot;
  const int64_t tiles = (rows + kRgRows - 1) / kRgRows;
  // A tile loads: 8 consecutive k per thread-chunk (one 16-byte core-row piece)
  const int chunks = kRgRows * (k_pad / 8);  // per tile
  constexpr int kMaxPer = kRgRows * (kRgMaxK / 8) / kRgThreads;  // 8
  const int per = (chunks + kRgThreads - 1) / kRgThreads;
  float av[kMaxPer][8];
  // 16-byte vector loads of A rows when the rows are 16-byte aligned
  const bool vec_a = (reinterpret_cast<uintptr_t>(A) % 16 == 0) &&
                     ((lda * (SPLIT ? 4 : 2)) % 16 == 0);
  const bool vec_c = (reinterpret_cast<uintptr_t>(C) % 16 == 0) && (ldc % 4 == 0);
  auto fetch = [&](int64_t tile) {
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      if (i >= per) break;
      const int c = tid + i * kRgThreads;
      const int r = c / (k_pad / 8), kc = c - r * (k_pad / 8);
      const int64_t row = tile * kRgRows + r;
#pragma unroll
      for (int q = 0; q < 8; ++q) av[i][q] = 0.f;
      if (c < chunks && row < rows) {
        const int k0 = kc * 8;
        if (SPLIT) {
          const float *src = reinterpret_cast<const float *>(A) + row * lda + k0;
          if (vec_a && k0 + 8 <= k) {
            const float4 u0 = __ldg(reinterpret_cast<const float4 *>(src));
            const float4 u1 = __ldg(reinterpret_cast<const float4 *>(src) + 1);
            av[i][0] = u0.x; av[i][1] = u0.y; av[i][2] = u0.z; av[i][3] = u0.w;
            av[i][4] = u1.x; av[i][5] = u1.y; av[i][6] = u1.z; av[i][7] = u1.w;
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (k0 + q < k) av[i][q] = __ldg(src + q);
          }
        } else {
          const __nv_bfloat16 *src = reinterpret_cast<const __nv_bfloat16 *>(A) + row * lda + k0;
          if (vec_a && k0 + 8 <= k) {
            const uint4 u = __ldg(reinterpret_cast<const uint4 *>(src));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              av[i][2 * q] = __uint_as_float(w[q] << 16);
              av[i][2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
            }
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (k0 + q < k) av[i][q] = __bfloat162float(src[q]);
          }
        }
      }
    }
  };
  const int qd = warp & 3, half = warp >> 2;
  const int rloc = 32 * qd + lane;
  const uint32_t lane_addr = tbase + ((uint32_t)(32 * qd) << 16);
  uint32_t phase = 0;
  bool timed_out = false;
  int64_t tile = blockIdx.x;
  if (tile < tiles) fetch(tile);
  for (; tile < tiles; tile += gridDim.x) {
    // A tile -> slabs
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      if (i >= per) break;
      const int c = tid + i * kRgThreads;
      if (c >= chunks) break;
      const int r = c / (k_pad / 8), kc = c - r * (k_pad / 8);
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __nv_bfloat16 h0, l0, h1, l1;
        rg_split(av[i][2 * q], h0, l0);
        rg_split(av[i][2 * q + 1], h1, l1);
        hw[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        lw[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
      }
      const int off = (kc * kRgRows + r) * 16;
      *reinterpret_cast<uint4 *>(a_s + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      if (SPLIT) *reinterpret_cast<uint4 *>(a_s + a_part + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      sm100::tc_fence_after();
      const uint32_t idesc = sm100::idesc_bf16_f32(kRgRows, n_pad);
      const uint32_t ah = sm100::smem_u32(a_s), al = ah + a_part;
      const uint32_t bh = sm100::smem_u32(b_s), bl = bh + b_part;
      const int sa = kRgRows * 16, sb = n_pad * 16;
      for (int kk = 0; kk < k_pad / 16; ++kk) {
        const uint64_t dah = sm100::make_desc(ah + 2 * kk * sa, sa, 128);
        const uint64_t dbh = sm100::make_desc(bh + 2 * kk * sb, sb, 128);
        sm100::mma_bf16(tbase, dah, dbh, idesc, kk > 0 ? 1u : 0u);
        if (SPLIT) {
          const uint64_t dal = sm100::make_desc(al + 2 * kk * sa, sa, 128);
          const uint64_t dbl = sm100::make_desc(bl + 2 * kk * sb, sb, 128);
          sm100::mma_bf16(tbase, dah, dbl, idesc, 1u);
          sm100::mma_bf16(tbase, dal, dbh, idesc, 1u);
        }
      }
      sm100::mma_commit(mbar);
    }
    const int64_t next = tile + gridDim.x;
    if (next < tiles) fetch(next);  // overlaps the MMAs
    if (!sm100::mbar_wait_bounded(mbar, phase, 1u << 20)) timed_out = true;
    phase ^= 1u;
    sm100::tc_fence_after();
    // epilogue, 32 columns at a time: TMEM -> staging tile (warp w: rows of lane
    // quarter w % 4, 16-column half w / 4 of the chunk), then coalesced stores
    // of whole row segments (plus beta C) from the staging tile
    for (int c0 = 0; c0 < n_pad; c0 += 32) {
      if (c0 + 16 * half < n_pad) {  // warp-uniform
        float v[16];
        sm100::tmem_ld16(lane_addr + c0 + 16 * half, v);
        sm100::tmem_ld_wait();
        if (timed_out) {  // the accumulator is not trustworthy: poison the tile
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = __int_as_float(0x7fc00000);
        }
        float *dst = stage + rloc * kRgStagePitch + 16 * half;
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4 *>(dst + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < kRgRows * 8 / kRgThreads; ++i) {
        const int idx = tid + i * kRgThreads;
        const int r = idx >> 3, c4 = idx & 7;
        const int col = c0 + 4 * c4;
        const int64_t row = tile * kRgRows + r;
        if (row >= rows || col >= n) continue;
        const float4 o = *reinterpret_cast<const float4 *>(stage + r * kRgStagePitch + 4 * c4);
        float *dst = C + row * ldc + col;
        if (vec_c && col + 4 <= n) {
          float4 w = o;
          if (beta != 0.f) {
            const float4 c4v = *reinterpret_cast<const float4 *>(dst);
            w.x = fmaf(beta, c4v.x, w.x);
            w.y = fmaf(beta, c4v.y, w.y);
            w.z = fmaf(beta, c4v.z, w.z);
            w.w = fmaf(beta, c4v.w, w.w);
          }
          *reinterpret_cast<float4 *>(dst) = w;
        } else {
          const float e[4] = {o.x, o.y, o.z, o.w};
          for (int q = 0; q < 4 && col + q < n; ++q)
            dst[q] = beta != 0.f ? fmaf(beta, dst[q], e[q]) : e[q];
        }
      }
      __syncthreads();
    }
    sm100::tc_fence_before();
    __syncthreads();  // TMEM and the A slabs free for the next tile
  }
  if (timed_out && status) atomicOr(status, 1u << 9);
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, 256);
  }
}

// ---------------------------------------------------------------- warp-specialised row GEMM
// The same product for operands the TMA can address (A and C 16-byte aligned,
// row pitches multiples of 16 bytes), as a warp-specialised pipeline per
// persistent CTA:
//   * warp 0 (one thread): TMA loads of A into a ring of shared-memory stages,
//     one 128-row x 128-byte box per stage (64 bf16 or 32 fp32 columns) with
//     128-byte swizzle, zero fill past the tensor; bf16 stages are the MMA's A
//     operand as they land.  The first ring's worth is issued before the B
//     operand is staged, so those loads overlap it;
//   * warps 8..11 (fp32 A only): split each landed fp32 stage in place into
//     bf16 hi and lo slabs (all reads of the stage finish before the writes);
//   * warp 1 (one thread): the tcgen05 MMAs of each stage into one of two TMEM
//     accumulators, committing every stage back to the ring and every finished
//     tile to the epilogue;
//   * warps 4..7: the epilogue.  Warp w drains TMEM lane quarter w % 4 (tile
//     rows 32 (w % 4) ..) 32 columns at a time into its own 128-byte swizzled
//     32 x 32 staging boxes (two buffers) and stores each box by its own TMA
//     tensor store -- or TMA reduce-add for beta = 1 (C += A B^T) -- so four
//     store streams per SM run without a cross-warp barrier.  The copy engine
//     clips rows past `rows` and columns past n.
// Every wait is bounded; a give-up sets a flag that ends every role's waits,
// poisons the remaining output with NaN and reports bit 9 of the status word.
constexpr int kWsThreads = 384;
constexpr int kWsKsBf16 = 64, kWsKsF32 = 32;  // K per stage
constexpr int kWsStageBytes = kRgRows * 64 * 2;  // 16 KB: one bf16 or fp32 stage
constexpr int kWsMaxStages = 8;
constexpr int kWsMaxN = 256;
constexpr int kWsBMax = 128 * 1024;      // B operand (all parts) in shared memory
constexpr int kWsBox = 32 * 32 * 4;      // one epilogue box: 32 rows x 32 fp32 columns
constexpr int kWsOutBuf = 2;             // staging boxes per epilogue warp
constexpr int kWsStaging = 4 * kWsOutBuf * kWsBox;
constexpr uint32_t kWsSpin = 1u << 20;

__host__ __device__ constexpr int ws_pad(int v, int m) { return (v + m - 1) / m * m; }

struct RowWsShape {
  int n_pad, k_pad, parts, stages;
  static RowWsShape make(int n, int k, bool split) {
    // K padded to the 64-element swizzle atom of B (a multiple of both stage widths)
    RowWsShape s{ws_pad(n, 16), ws_pad(k, 64), split ? 2 : 1, 0};
    const int fixed = ws_pad(s.b_bytes(), 1024) + kWsStaging + 2048;
    s.stages = std::min(kWsMaxStages, (kRgSmemLimit - fixed) / kWsStageBytes);
    return s;
  }
  int b_bytes() const { return parts * n_pad * k_pad * 2; }
  int smem() const {
    return ws_pad(b_bytes(), 1024) + stages * kWsStageBytes + kWsStaging + 1024 + 1024;
  }
  int tmem_cols() const { return n_pad <= 64 ? 128 : (n_pad <= 128 ? 256 : 512); }
  bool ok() const { return stages >= 2 && b_bytes() <= kWsBMax && smem() <= kRgSmemLimit; }
};

struct WsBars {
  uint64_t full[kWsMaxStages];   // stage landed (TMA)
  uint64_t split[kWsMaxStages];  // fp32 stage split into bf16 slabs (fp32 A)
  uint64_t empty[kWsMaxStages];  // stage free (MMA commit)
  uint64_t acc_full[2], acc_free[2];
  uint32_t tmem, err;
};

template <int PENDING>
__device__ __forceinline__ void ws_bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(PENDING) : "memory");
}

template <bool SPLIT>
__global__ void __launch_bounds__(kWsThreads, 1) rowgemm_ws_kernel(
    const __grid_constant__ CUtensorMap amap, const void *__restrict__ Bm, int64_t ldbn,
    int64_t ldbk, const __grid_constant__ CUtensorMap cmap, int64_t rows, int n, int k,
    int reduce_add, int n_pad, int k_pad, int stages, int tmem_cols,
    uint32_t *__restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int P = SPLIT ? 2 : 1;
  constexpr int KS = SPLIT ? kWsKsF32 : kWsKsBf16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b_part = n_pad * k_pad * 2;
  uint8_t *b_s = smem;
  uint8_t *ring = smem + ws_pad(P * b_part, 1024);
  uint8_t *stage_out = ring + stages * kWsStageBytes;  // 1024-aligned
  WsBars *bars = reinterpret_cast<WsBars *>(stage_out + kWsStaging);
  volatile uint32_t *err = &bars->err;
  const int64_t tiles = (rows + kRgRows - 1) / kRgRows;
  const int kst = k_pad / KS;
  const int64_t my_tiles =
      (int64_t)blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t fills = my_tiles * kst;  // ring fills of this CTA
  auto fill = [&](int64_t f) {           // fill f: local tile f / kst, K stage f % kst
    const int s = (int)(f % stages);
    const int64_t tile = blockIdx.x + (f / kst) * (int64_t)gridDim.x;
    const int ks = (int)(f % kst);
    sm100::mbar_arrive_expect_tx(&bars->full[s], kWsStageBytes);
    sm100::tma_load_2d(sm100::smem_u32(ring + s * kWsStageBytes), &amap, &bars->full[s], ks * KS,
                       (int)(tile * kRgRows));
  };
  if (tid == 0) {
    for (int i = 0; i < stages; ++i) {
      sm100::mbar_init(&bars->full[i], 1);
      sm100::mbar_init(&bars->split[i], 1);
      sm100::mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&bars->acc_full[i], 1);
      sm100::mbar_init(&bars->acc_free[i], 4);
    }
    bars->err = 0;
    sm100::fence_barrier_init();
    // the first ring's worth of A, in flight while B is staged
    for (int64_t f = 0; f < fills && f < stages; ++f) fill(f);
  }
  if (warp == 0) {
    sm100::tmem_alloc(&bars->tmem, (uint32_t)tmem_cols);
    sm100::tmem_relinquish();
  }
  // B once (every thread) as the MMA's K-major operand in the 128-byte swizzled
  // layout: 8 columns j x 64 K elements per 1024-byte atom, atom (j / 8, kg / 8)
  // at ((kg / 8) * (n_pad / 8) + j / 8) * 1024, 16-byte row piece (j, kg) at
  // (j % 8) * 128 + ((kg % 8) ^ (j % 8)) * 16 inside it.  Work item = one piece
  // (eight K elements of column j).  Consecutive threads take consecutive K
  // groups of one column where B's K stride is 1 (coalesced rows), else
  // consecutive columns of one K group (coalesced along B's unit stride); the
  // swizzle keeps both write patterns free of bank conflicts.  Each CTA starts
  // at a different item (whole warps' worth apart): all CTAs read B at once, and
  // rotated starts spread their requests over different L2 lines.
  {
    const int kgs = k_pad / 8;
    const int items = n_pad * kgs;
    const int es = SPLIT ? 4 : 2;
    const bool kk_inner = ldbk == 1;
    const bool vec = kk_inner && ldbn % 8 == 0 && reinterpret_cast<uintptr_t>(Bm) % (8 * es) == 0;
    constexpr int U = 4;
    const int rot = (int)((blockIdx.x * 37u * 32u) % (uint32_t)items);
    auto item = [&](int i) { const int c = i + rot; return c >= items ? c - items : c; };
    for (int base = 0; base < items; base += U * kWsThreads) {
      float v[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * kWsThreads + tid;
        const int c = item(i < items ? i : 0);
        const int jj = kk_inner ? c / kgs : c % n_pad;
        const int kg = kk_inner ? c - jj * kgs : c / n_pad;
        const int k0 = 8 * kg;
#pragma unroll
        for (int w = 0; w < 8; ++w) v[u][w] = 0.f;
        if (i < items && jj < n && k0 < k) {
          const int64_t row = (int64_t)jj * ldbn;
          if (vec && k0 + 8 <= k) {
            if (SPLIT) {
              const float4 *p4 = reinterpret_cast<const float4 *>(
                  reinterpret_cast<const float *>(Bm) + row + k0);
              const float4 a4 = __ldg(p4), b4 = __ldg(p4 + 1);
              v[u][0] = a4.x; v[u][1] = a4.y; v[u][2] = a4.z; v[u][3] = a4.w;
              v[u][4] = b4.x; v[u][5] = b4.y; v[u][6] = b4.z; v[u][7] = b4.w;
            } else {
              const uint4 b8 = __ldg(reinterpret_cast<const uint4 *>(
                  reinterpret_cast<const __nv_bfloat16 *>(Bm) + row + k0));
              const uint32_t wv[4] = {b8.x, b8.y, b8.z, b8.w};
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                v[u][2 * w] = __uint_as_float(wv[w] << 16);
                v[u][2 * w + 1] = __uint_as_float(wv[w] & 0xFFFF0000u);
              }
            }
          } else {
#pragma unroll
            for (int w = 0; w < 8; ++w) {
              if (k0 + w < k) {
                const int64_t off = row + (int64_t)(k0 + w) * ldbk;
                v[u][w] = SPLIT ? __ldg(reinterpret_cast<const float *>(Bm) + off)
                                : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(Bm)[off]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * kWsThreads + tid;
        if (i < items) {
          const int c = item(i);
          const int jj = kk_inner ? c / kgs : c % n_pad;
          const int kg = kk_inner ? c - jj * kgs : c / n_pad;
          const int off = ((kg >> 3) * (n_pad >> 3) + (jj >> 3)) * 1024 + (jj & 7) * 128 +
                          (((kg & 7) ^ (jj & 7)) << 4);
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __nv_bfloat16 h0, l0, h1, l1;
            rg_split(v[u][2 * q], h0, l0);
            rg_split(v[u][2 * q + 1], h1, l1);
            hw[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
            lw[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
          }
          *reinterpret_cast<uint4 *>(b_s + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          if (SPLIT)
            *reinterpret_cast<uint4 *>(b_s + b_part + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
    }
  }
  sm100::fence_proxy_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = bars->tmem;
  const uint32_t acc_stride = (uint32_t)tmem_cols / 2;
  // bounded wait that gives up at once after any role has given up
  auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
    if (*err) return false;
    if (sm100::mbar_wait_bounded(bar, parity, kWsSpin)) return true;
    *err = 1u;
    return false;
  };

  if (warp == 0) {
    // ---- TMA producer: fill f reuses slot f % stages once fill f - stages is consumed
    if (lane == 0) {
      for (int64_t f = stages; f < fills; ++f) {
        wait(&bars->empty[f % stages], (uint32_t)(((f / stages) - 1) & 1));
        fill(f);
      }
      // this thread's copies have landed before the CTA may exit: the last fill of
      // every slot (fill f has parity (f / stages) & 1); bounded, also after a give-up
      for (int x = 0; x < stages && x < fills; ++x) {
        const int64_t f = x + (fills - 1 - x) / stages * stages;
        sm100::mbar_wait_bounded(&bars->full[x], (uint32_t)((f / stages) & 1), kWsSpin);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, aph = 0, a = 0;
      const uint32_t idesc = sm100::idesc_bf16_f32(kRgRows, n_pad);
      const uint32_t bh = sm100::smem_u32(b_s), bl = bh + b_part;
      const uint32_t b_atom_col = (uint32_t)(n_pad / 8) * 1024;  // B bytes per 64 K elements
      constexpr int SA = kRgRows * 16;  // A slab stride (8 columns x 128 rows)
      for (int64_t lt = 0; lt < my_tiles; ++lt) {
        wait(&bars->acc_free[a], aph ^ 1u);
        sm100::tc_fence_after();
        const uint32_t d = tbase + a * acc_stride;
        for (int ks = 0; ks < kst; ++ks) {
          wait(SPLIT ? &bars->split[s] : &bars->full[s], ph);
          sm100::tc_fence_after();
          const uint32_t ah = sm100::smem_u32(ring + s * kWsStageBytes);
          const uint32_t al = ah + kWsStageBytes / 2;  // split: lo slabs after the hi slabs
#pragma unroll
          for (int kk = 0; kk < KS / 16; ++kk) {
            const int t = ks * KS / 16 + kk;  // K=16 step: B atom column t / 4, 32 bytes per step
            const uint32_t boff = (uint32_t)(t >> 2) * b_atom_col + (uint32_t)(t & 3) * 32;
            // bf16: the landed 128-byte swizzled stage; split: no-swizzle slabs
            const uint64_t dah = SPLIT ? sm100::make_desc(ah + 2 * kk * SA, SA, 128)
                                       : sm100::make_desc_sw128(ah + 32 * kk);
            const uint64_t dbh = sm100::make_desc_sw128(bh + boff);
            const uint32_t acc = (ks > 0 || kk > 0) ? 1u : 0u;
            sm100::mma_bf16(d, dah, dbh, idesc, acc);
            if (SPLIT) {
              const uint64_t dal = sm100::make_desc(al + 2 * kk * SA, SA, 128);
              const uint64_t dbl = sm100::make_desc_sw128(bl + boff);
              sm100::mma_bf16(d, dah, dbl, idesc, 1u);
              sm100::mma_bf16(d, dal, dbh, idesc, 1u);
            }
          }
          sm100::mma_commit(&bars->empty[s]);
          if (++s == stages) { s = 0; ph ^= 1u; }
        }
        sm100::mma_commit(&bars->acc_full[a]);
        a ^= 1u;
        if (a == 0) aph ^= 1u;
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---- epilogue: warp w drains TMEM lane quarter w % 4 = tile rows 32 (w % 4) ..
    const int qd = warp & 3;
    uint8_t *boxes = stage_out + qd * kWsOutBuf * kWsBox;
    const uint32_t boxes_u32 = sm100::smem_u32(boxes);
    uint32_t a = 0, aph = 0, chunk_no = 0;
    for (int64_t lt = 0; lt < my_tiles; ++lt) {
      const int64_t tile = blockIdx.x + lt * (int64_t)gridDim.x;
      wait(&bars->acc_full[a], aph);
      sm100::tc_fence_after();
      const uint32_t lane_addr = tbase + a * acc_stride + ((uint32_t)(32 * qd) << 16);
      for (int c0 = 0; c0 < n_pad; c0 += 32, ++chunk_no) {
        const int b = (int)(chunk_no % kWsOutBuf);
        // the copy that last read this box has finished reading it
        if (lane == 0) ws_bulk_wait_read<kWsOutBuf - 1>();
        __syncwarp();
        float v[32];
        if (c0 + 32 <= n_pad) {
          sm100::tmem_ld32(lane_addr + c0, v);
        } else {  // a 16-column tail (n_pad % 32 == 16)
          sm100::tmem_ld16(lane_addr + c0, v);
#pragma unroll
          for (int q = 16; q < 32; ++q) v[q] = 0.f;
        }
        sm100::tmem_ld_wait();
        if (*err) {  // a wait gave up somewhere: the accumulator is not trustworthy
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __int_as_float(0x7fc00000);
        }
        uint8_t *box = boxes + b * kWsBox;
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // 16-byte chunk q of row `lane`, swizzled with the row
          const int jq = q ^ (lane & 7);
          *reinterpret_cast<float4 *>(box + lane * 128 + jq * 16) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t src = boxes_u32 + b * kWsBox;
          const int r0 = (int)(tile * kRgRows) + 32 * qd;
          if (reduce_add)
            sm100::tma_reduce_add_2d(&cmap, src, c0, r0);
          else
            sm100::tma_store_2d(&cmap, src, c0, r0);
          sm100::bulk_commit();
        }
      }
      // this warp's TMEM reads are complete: the accumulator may be overwritten
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&bars->acc_free[a]);
      a ^= 1u;
      if (a == 0) aph ^= 1u;
    }
    if (lane == 0) sm100::bulk_wait_all();  // this warp's output copies are complete
  } else if (SPLIT && warp >= 8) {
    // ---- fp32 split, in place: thread ct owns tile row ct of every stage
    const int ct = tid - 256;
    int s = 0;
    uint32_t ph = 0;
    for (int64_t f = 0; f < fills; ++f) {
      wait(&bars->full[s], ph);
      uint8_t *st = ring + s * kWsStageBytes;
      float x[KS];  // row ct: 128 bytes at ct * 128, 16-byte chunk q at q ^ (ct % 8)
#pragma unroll
      for (int q = 0; q < KS / 4; ++q) {
        const float4 f4 = *reinterpret_cast<const float4 *>(st + ct * 128 + ((q ^ (ct & 7)) * 16));
        x[4 * q] = f4.x; x[4 * q + 1] = f4.y; x[4 * q + 2] = f4.z; x[4 * q + 3] = f4.w;
      }
      sm100::named_sync(2, 128);  // every read of the stage precedes the first write
#pragma unroll
      for (int g = 0; g < KS / 8; ++g) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __nv_bfloat16 h0, l0, h1, l1;
          rg_split(x[8 * g + 2 * q], h0, l0);
          rg_split(x[8 * g + 2 * q + 1], h1, l1);
          hw[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
          lw[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        *reinterpret_cast<uint4 *>(st + (g * kRgRows + ct) * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(st + kWsStageBytes / 2 + (g * kRgRows + ct) * 16) =
            make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      sm100::fence_proxy_async_smem();
      sm100::named_sync(2, 128);
      if (ct == 0) sm100::mbar_arrive(&bars->split[s]);
      if (++s == stages) { s = 0; ph ^= 1u; }
    }
  }
  __syncthreads();
  if (tid == 0 && *err && status) atomicOr(status, 1u << 9);
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, (uint32_t)tmem_cols);
  }
}

int sm_count();

// Whether rowgemm serves this call (types, sizes, shared memory).
inline bool rowgemm_supported(cudaDataType ta, cudaDataType tb, int n, int k) {
  const bool bf = ta == CUDA_R_16BF && tb == CUDA_R_16BF;
  const bool f32 = ta == CUDA_R_32F && tb == CUDA_R_32F;
  if (!bf && !f32) return false;
  if (n < 1 || k < 1 || n > kRgMaxN || k > kRgMaxK) return false;
  RowGemmShape s{rg_pad16(n), rg_pad16(k), f32 ? 2 : 1};
  return s.smem() <= kRgSmemLimit;
}

// `status`: device error word (bit 9: an MMA wait gave up) or NULL.
inline int rowgemm(cudaStream_t st, const void *A, cudaDataType ta, int64_t lda, const void *Bm,
                   int64_t ldbn, int64_t ldbk, float *C, int64_t ldc, int64_t rows, int n, int k,
                   float beta, uint32_t *status, const char *what) {
  const bool split = ta == CUDA_R_32F;
  RowGemmShape s{rg_pad16(n), rg_pad16(k), split ? 2 : 1};
  const int64_t tiles = cdiv(rows, kRgRows);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, sm_count());
  if (split) {
    LNET_TRY(cuda_check(cudaFuncSetAttribute(rowgemm_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kRgSmemLimit),
                        "cudaFuncSetAttribute(rowgemm_kernel)"));
    rowgemm_kernel<true><<<grid, kRgThreads, s.smem(), st>>>(A, lda, Bm, ldbn, ldbk, C, ldc,
                                                             rows, n, k, beta, s.n_pad, s.k_pad,
                                                             status);
  } else {
    LNET_TRY(cuda_check(cudaFuncSetAttribute(rowgemm_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kRgSmemLimit),
                        "cudaFuncSetAttribute(rowgemm_kernel)"));
    rowgemm_kernel<false><<<grid, kRgThreads, s.smem(), st>>>(A, lda, Bm, ldbn, ldbk, C, ldc,
                                                              rows, n, k, beta, s.n_pad,
                                                              s.k_pad, status);
  }
  return after_launch(what);
}

// Whether the warp-specialised row GEMM serves this call: types, sizes, shared
// memory, and operands the TMA can address.
inline bool rowgemm_ws_supported(const void *A, cudaDataType ta, cudaDataType tb, int64_t lda,
                                 int n, int k, const float *C, int64_t ldc) {
  const bool bf = ta == CUDA_R_16BF && tb == CUDA_R_16BF;
  const bool f32 = ta == CUDA_R_32F && tb == CUDA_R_32F;
  if (!bf && !f32) return false;
  if (n < 1 || k < 1 || n > kWsMaxN) return false;
  const int es = f32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(A) % 16 != 0 || (lda * es) % 16 != 0 || lda < k) return false;
  if (reinterpret_cast<uintptr_t>(C) % 16 != 0 || ldc % 4 != 0 || ldc < n) return false;
  return RowWsShape::make(n, k, f32).ok();
}

// 2-D map of a row-major [rows][cols] matrix (row pitch `ld` elements), box
// box_cols x box_rows.
inline int encode_rows_map(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int es,
                           int64_t ld, int64_t rows, int cols, int box_cols, int box_rows,
                           CUtensorMapSwizzle swz) {
  PFN_cuTensorMapEncodeTiled_v12000 encode;
  LNET_TRY(tensor_map_encoder(&encode));
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * es};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult res = encode(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(LNET_ERR_CUDA, "cuTensorMapEncodeTiled (row GEMM) failed (%d)", (int)res);
  return LNET_OK;
}

// beta is 0 (C = A B^T) or 1 (C += A B^T).
inline int rowgemm_ws(cudaStream_t st, const void *A, cudaDataType ta, int64_t lda,
                      const void *Bm, int64_t ldbn, int64_t ldbk, float *C, int64_t ldc,
                      int64_t rows, int n, int k, float beta, uint32_t *status, const char *what) {
  if (beta != 0.f && beta != 1.f)
    return fail(LNET_ERR_INVALID_ARGUMENT, "%s: beta %g (row GEMM takes 0 or 1)", what, beta);
  const bool split = ta == CUDA_R_32F;
  const RowWsShape s = RowWsShape::make(n, k, split);
  CUtensorMap amap, cmap;
  if (split)
    LNET_TRY(encode_rows_map(&amap, A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, lda, rows, k, kWsKsF32,
                             kRgRows, CU_TENSOR_MAP_SWIZZLE_128B));
  else
    LNET_TRY(encode_rows_map(&amap, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, lda, rows, k,
                             kWsKsBf16, kRgRows, CU_TENSOR_MAP_SWIZZLE_128B));
  LNET_TRY(encode_rows_map(&cmap, C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ldc, rows, n, 32, 32,
                           CU_TENSOR_MAP_SWIZZLE_128B));
  const int64_t tiles = cdiv(rows, kRgRows);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, sm_count());
  const int red = beta != 0.f ? 1 : 0;
  if (split) {
    LNET_TRY(cuda_check(cudaFuncSetAttribute(rowgemm_ws_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kRgSmemLimit),
                        "cudaFuncSetAttribute(rowgemm_ws_kernel)"));
    rowgemm_ws_kernel<true><<<grid, kWsThreads, s.smem(), st>>>(
        amap, Bm, ldbn, ldbk, cmap, rows, n, k, red, s.n_pad, s.k_pad, s.stages, s.tmem_cols(),
        status);
  } else {
    LNET_TRY(cuda_check(cudaFuncSetAttribute(rowgemm_ws_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kRgSmemLimit),
                        "cudaFuncSetAttribute(rowgemm_ws_kernel)"));
    rowgemm_ws_kernel<false><<<grid, kWsThreads, s.smem(), st>>>(
        amap, Bm, ldbn, ldbk, cmap, rows, n, k, red, s.n_pad, s.k_pad, s.stages, s.tmem_cols(),
        status);
  }
  return after_launch(what);
}

}  // namespace lnet
