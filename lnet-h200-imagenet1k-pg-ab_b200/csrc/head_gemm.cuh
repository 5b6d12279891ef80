// Affine readout logits = F G^T + bias on tcgen05 tensor cores.
//
// F [B, W] are the radial-log features (W = 14 M), G [K, W] the classifier
// weights, both fp32.  Each operand is split as x = hi + lo with hi, lo in
// bf16, and every K=16 step issues hi*hi + hi*lo + lo*hi into one fp32 TMEM
// accumulator, which keeps the readout at fp32-level accuracy (the dropped
// lo*lo term and the split residual are ~2^-16 relative).
// One CTA (4 warps) owns a 128-row x 64-class tile and walks W in blocks of
// 64: threads split their rows/classes into shared-memory slabs, one thread
// issues the 12 MMAs, all wait on an mbarrier (bounded), then the next block.
#pragma once

#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace lnet {

constexpr int kHeadRows = 128, kHeadN = 64, kHeadKB = 64, kHeadThreads = 128;
constexpr int kHeadSlabA = kHeadRows * 16, kHeadSlabB = kHeadN * 16;
constexpr int kHeadABytes = (kHeadKB / 8) * kHeadSlabA;  // one of hi / lo
constexpr int kHeadBBytes = (kHeadKB / 8) * kHeadSlabB;
constexpr int kHeadSmem = 2 * kHeadABytes + 2 * kHeadBBytes + 64;

__device__ __forceinline__ void split_bf16x8(const float *v, uint4 &hi, uint4 &lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat16 a = __float2bfloat16_rn(v[2 * i]), b = __float2bfloat16_rn(v[2 * i + 1]);
    __nv_bfloat16 c = __float2bfloat16_rn(v[2 * i] - __bfloat162float(a));
    __nv_bfloat16 d = __float2bfloat16_rn(v[2 * i + 1] - __bfloat162float(b));
    h[i] = (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
    l[i] = (uint32_t)__bfloat16_as_ushort(c) | ((uint32_t)__bfloat16_as_ushort(d) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Loads 8 consecutive fp32 values of `row` starting at column k (zero past `width`).
__device__ __forceinline__ void load8(const float *row, int k, int width, float *v) {
  if (k + 8 <= width && (width & 3) == 0) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(row + k));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(row + k + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = k + i < width ? __ldg(row + k + i) : 0.f;
  }
}

// Split-K: CTA z covers K blocks [z * bpc, (z + 1) * bpc) and writes its partial
// tile to partial[z][B][K].
__global__ void __launch_bounds__(kHeadThreads) head_gemm_kernel(
    const float *__restrict__ F, int64_t B, int width, const float *__restrict__ G,
    float *__restrict__ partial, int K, int blocks_per_cta) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *a_hi = smem, *a_lo = smem + kHeadABytes;
  uint8_t *b_hi = smem + 2 * kHeadABytes, *b_lo = b_hi + kHeadBBytes;
  uint64_t *mbar = reinterpret_cast<uint64_t *>(b_lo + kHeadBBytes);
  uint32_t *tslot = reinterpret_cast<uint32_t *>(b_lo + kHeadBBytes + 8);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t r0 = (int64_t)blockIdx.x * kHeadRows;
  const int n0 = blockIdx.y * kHeadN;
  if (tid == 0) {
    sm100::mbar_init(mbar, 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, kHeadN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tslot;
  const int64_t row = r0 + tid;
  const float *frow = row < B ? F + row * width : nullptr;
  const int brow = tid & (kHeadN - 1), bhalf = tid >> 6;  // class row, K half of the block
  const int cls = n0 + brow;
  const float *grow = cls < K ? G + (int64_t)cls * width : nullptr;
  uint32_t phase = 0;
  bool timed_out = false;
  const int total_blk = (width + kHeadKB - 1) / kHeadKB;
  const int kb_begin = blockIdx.z * blocks_per_cta;
  const int nblk = max(0, min(blocks_per_cta, total_blk - kb_begin));
  // operands of block kb are loaded into registers one block ahead, so their
  // global latency overlaps the previous block's MMAs
  float av[kHeadKB], bv[kHeadKB / 2];
  auto fetch = [&](int kb) {
    const int k0 = (kb_begin + kb) * kHeadKB;
#pragma unroll
    for (int c = 0; c < kHeadKB / 8; ++c) {
      if (frow) {
        load8(frow, k0 + 8 * c, width, av + 8 * c);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) av[8 * c + i] = 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < kHeadKB / 16; ++c) {
      const int cc = bhalf * (kHeadKB / 16) + c;
      if (grow) {
        load8(grow, k0 + 8 * cc, width, bv + 8 * c);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) bv[8 * c + i] = 0.f;
      }
    }
  };
  fetch(0);
  for (int kb = 0; kb < nblk; ++kb) {
    if (kb > 0) {  // MMAs of block kb - 1 still read the slabs
      if (!sm100::mbar_wait_bounded(mbar, phase, 1u << 20)) timed_out = true;
      phase ^= 1u;
      sm100::tc_fence_after();
    }
#pragma unroll
    for (int c = 0; c < kHeadKB / 8; ++c) {
      uint4 hi, lo;
      split_bf16x8(av + 8 * c, hi, lo);
      *reinterpret_cast<uint4 *>(a_hi + c * kHeadSlabA + tid * 16) = hi;
      *reinterpret_cast<uint4 *>(a_lo + c * kHeadSlabA + tid * 16) = lo;
    }
#pragma unroll
    for (int c = 0; c < kHeadKB / 16; ++c) {
      const int cc = bhalf * (kHeadKB / 16) + c;
      uint4 hi, lo;
      split_bf16x8(bv + 8 * c, hi, lo);
      *reinterpret_cast<uint4 *>(b_hi + cc * kHeadSlabB + brow * 16) = hi;
      *reinterpret_cast<uint4 *>(b_lo + cc * kHeadSlabB + brow * 16) = lo;
    }
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      sm100::tc_fence_after();
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(kHeadRows, kHeadN);
      const uint32_t ah = sm100::smem_u32(a_hi), al = sm100::smem_u32(a_lo);
      const uint32_t bh = sm100::smem_u32(b_hi), bl = sm100::smem_u32(b_lo);
      for (int kk = 0; kk < kHeadKB / 16; ++kk) {
        const uint64_t dah = sm100::make_desc(ah + 2 * kk * kHeadSlabA, kHeadSlabA, 128);
        const uint64_t dal = sm100::make_desc(al + 2 * kk * kHeadSlabA, kHeadSlabA, 128);
        const uint64_t dbh = sm100::make_desc(bh + 2 * kk * kHeadSlabB, kHeadSlabB, 128);
        const uint64_t dbl = sm100::make_desc(bl + 2 * kk * kHeadSlabB, kHeadSlabB, 128);
        sm100::mma_bf16(tbase, dah, dbh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        sm100::mma_bf16(tbase, dah, dbl, idesc, 1u);
        sm100::mma_bf16(tbase, dal, dbh, idesc, 1u);
      }
      sm100::mma_commit(mbar);
    }
    if (kb + 1 < nblk) fetch(kb + 1);
  }
  if (nblk > 0 && !sm100::mbar_wait_bounded(mbar, phase, 1u << 20)) timed_out = true;
  sm100::tc_fence_after();
  // epilogue: thread tid owns row r0 + tid (TMEM lane tid)
  float acc[kHeadN];
#pragma unroll
  for (int j = 0; j < kHeadN / 16; ++j)
    sm100::tmem_ld16(tbase + ((uint32_t)(32 * warp) << 16) + 16 * j, acc + 16 * j);
  sm100::tmem_ld_wait();
  if (row < B) {
    float *dst = partial + ((int64_t)blockIdx.z * B + row) * K;
#pragma unroll
    for (int j = 0; j < kHeadN; ++j) {
      const int c = n0 + j;
      if (c < K) dst[c] = timed_out ? __int_as_float(0x7fc00000) : (nblk > 0 ? acc[j] : 0.f);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, kHeadN);
  }
}

// logits[b, k] = bias[k] + sum_z partial[z][b][k], summed in a fixed order.
__global__ void head_reduce_kernel(const float *__restrict__ partial, const float *__restrict__ bias,
                                   float *__restrict__ logits, int64_t n, int K, int splits) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = __ldg(bias + (int)(i % K));
    for (int z = 0; z < splits; ++z) acc += partial[z * n + i];
    logits[i] = acc;
  }
}

constexpr int kHeadSplits = 4;  // measured best at B=256, K=1000 (6 and 11 are slower)

inline size_t head_partial_floats(int64_t B, int K) { return (size_t)kHeadSplits * B * K; }

// logits [B, K] from features [B, width]; `partial` holds head_partial_floats(B, K)
// floats.  A wait that gives up writes NaN logits.
inline int head_gemm(const float *feats, int64_t B, int width, const float *G, const float *bias,
                     float *logits, int K, float *partial, cudaStream_t st) {
  LNET_TRY(cuda_check(cudaFuncSetAttribute(head_gemm_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmem),
                      "cudaFuncSetAttribute(head_gemm_kernel)"));
  const int total_blk = (width + kHeadKB - 1) / kHeadKB;
  const int bpc = (total_blk + kHeadSplits - 1) / kHeadSplits;
  dim3 grid((unsigned)cdiv(B, kHeadRows), (unsigned)cdiv(K, kHeadN), kHeadSplits);
  head_gemm_kernel<<<grid, kHeadThreads, kHeadSmem, st>>>(feats, B, width, G, partial, K, bpc);
  LNET_TRY(after_launch("head_gemm_kernel"));
  const int64_t n = B * K;
  const int blocks = (int)std::min<int64_t>(cdiv(n, 256), 148 * 8);
  head_reduce_kernel<<<blocks, 256, 0, st>>>(partial, bias, logits, n, K, kHeadSplits);
  return after_launch("head_reduce_kernel");
}

}  // namespace lnet
