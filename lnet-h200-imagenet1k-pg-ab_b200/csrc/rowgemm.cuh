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

namespace lnet {

constexpr int kRgRows = 128, kRgThreads = 256;
// Shapes served: n, k <= 128 (BASELINE configs 2 and 3 and every small general-route
// request).  This kernel carries one tile at a time per SM; at n = k = 256 (config 5)
// it measured slower than cuBLAS's pipelined bf16 GEMMs, which keep those shapes.
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

}  // namespace lnet
