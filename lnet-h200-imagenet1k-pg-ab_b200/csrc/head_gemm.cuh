// Affine readout logits = F G^T + bias on tcgen05 tensor cores.
//
// F [B, W] are the radial-log features (W = 14 M), G [K, W] the classifier
// weights, both fp32.  Each operand is split as x = hi + lo with hi, lo in
// bf16, and every K=16 step issues hi*hi + hi*lo + lo*hi into one fp32 TMEM
// accumulator, which keeps the readout at fp32-level accuracy (the dropped
// lo*lo term and the split residual are ~2^-16 relative).
// One CTA (8 warps) owns a 128-row x 64-class tile and a range of W (split-K)
// walked in blocks of 64: the operand tiles are read with coalesced float4
// loads (16 threads per 256-byte row, the next block prefetched into
// registers), split into padded shared-memory slabs, one thread issues the 12
// MMAs and all wait on an mbarrier (bounded).  The partial tile leaves through
// a padded shared-memory transpose as coalesced float4 stores.
#pragma once

#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace lnet {

constexpr int kHeadRows = 128, kHeadN = 64, kHeadKB = 64, kHeadThreads = 256;
// K-chunk slab strides padded by 16 bytes: the eight 8-column chunks a row's
// float4 loads spread over fall in distinct bank groups
constexpr int kHeadSlabA = kHeadRows * 16 + 16, kHeadSlabB = kHeadN * 16 + 16;
constexpr int kHeadABytes = (kHeadKB / 8) * kHeadSlabA;  // one of hi / lo
constexpr int kHeadBBytes = (kHeadKB / 8) * kHeadSlabB;
constexpr int kHeadOutPitch = kHeadN + 4;  // floats per row of the epilogue transpose
constexpr int kHeadOperandBytes = 2 * kHeadABytes + 2 * kHeadBBytes;
constexpr int kHeadSmem =
    std::max(kHeadOperandBytes, kHeadRows * kHeadOutPitch * 4) + 64;
constexpr int kHeadA4 = kHeadRows * kHeadKB / 4 / kHeadThreads;  // float4 of A per thread
constexpr int kHeadB4 = kHeadN * kHeadKB / 4 / kHeadThreads;     // float4 of B per thread

// (hi, lo) bf16 pairs of four floats, packed as two 8-byte words each
__device__ __forceinline__ void split_bf16x4(const float4 &v, uint2 &hi, uint2 &lo) {
  const float x[4] = {v.x, v.y, v.z, v.w};
  uint32_t h[2], l[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    __nv_bfloat16 a = __float2bfloat16_rn(x[2 * i]), b = __float2bfloat16_rn(x[2 * i + 1]);
    __nv_bfloat16 c = __float2bfloat16_rn(x[2 * i] - __bfloat162float(a));
    __nv_bfloat16 d = __float2bfloat16_rn(x[2 * i + 1] - __bfloat162float(b));
    h[i] = (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
    l[i] = (uint32_t)__bfloat16_as_ushort(c) | ((uint32_t)__bfloat16_as_ushort(d) << 16);
  }
  hi = make_uint2(h[0], h[1]);
  lo = make_uint2(l[0], l[1]);
}

// Four consecutive fp32 of `row` from column k (zero past `width` or a NULL row).
__device__ __forceinline__ float4 load4(const float *row, int k, int width) {
  if (!row) return make_float4(0.f, 0.f, 0.f, 0.f);
  if (k + 4 <= width && (width & 3) == 0) return __ldg(reinterpret_cast<const float4 *>(row + k));
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = k + i < width ? __ldg(row + k + i) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Split-K: CTA z covers K blocks [z * bpc, (z + 1) * bpc) and writes its partial
// tile to partial[z][B][K].
__global__ void __launch_bounds__(kHeadThreads) head_gemm_kernel(
    const float *__restrict__ F, int64_t B, int width, const float *__restrict__ G,
    float *__restrict__ partial, int K, int blocks_per_cta) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *a_hi = smem, *a_lo = smem + kHeadABytes;
  uint8_t *b_hi = smem + 2 * kHeadABytes, *b_lo = b_hi + kHeadBBytes;
  uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + kHeadSmem - 64);
  uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + kHeadSmem - 56);
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
  uint32_t phase = 0;
  bool timed_out = false;
  const int total_blk = (width + kHeadKB - 1) / kHeadKB;
  const int kb_begin = blockIdx.z * blocks_per_cta;
  const int nblk = max(0, min(blocks_per_cta, total_blk - kb_begin));
  const int c4 = tid & 15;  // float4 column of the 64-wide block
  // operands of block kb, loaded one block ahead (coalesced: 16 threads per row)
  float4 av[kHeadA4], bv[kHeadB4];
  auto fetch = [&](int kb) {
    const int k0 = (kb_begin + kb) * kHeadKB + 4 * c4;
#pragma unroll
    for (int i = 0; i < kHeadA4; ++i) {
      const int64_t row = r0 + (tid >> 4) + 16 * i;
      av[i] = load4(row < B ? F + row * width : nullptr, k0, width);
    }
#pragma unroll
    for (int i = 0; i < kHeadB4; ++i) {
      const int cls = n0 + (tid >> 4) + 16 * i;
      bv[i] = load4(cls < K ? G + (int64_t)cls * width : nullptr, k0, width);
    }
  };
  if (nblk > 0) fetch(0);
  for (int kb = 0; kb < nblk; ++kb) {
    if (kb > 0) {  // MMAs of block kb - 1 still read the slabs
      if (!sm100::mbar_wait_bounded(mbar, phase, 1u << 20)) timed_out = true;
      phase ^= 1u;
      sm100::tc_fence_after();
    }
    // element (r, k) of a slab operand at (k / 8) * slab + r * 16 + (k % 8) * 2
    const int kc = c4 >> 1, half = (c4 & 1) * 8;
#pragma unroll
    for (int i = 0; i < kHeadA4; ++i) {
      const int r = (tid >> 4) + 16 * i;
      uint2 hi, lo;
      split_bf16x4(av[i], hi, lo);
      *reinterpret_cast<uint2 *>(a_hi + kc * kHeadSlabA + r * 16 + half) = hi;
      *reinterpret_cast<uint2 *>(a_lo + kc * kHeadSlabA + r * 16 + half) = lo;
    }
#pragma unroll
    for (int i = 0; i < kHeadB4; ++i) {
      const int r = (tid >> 4) + 16 * i;
      uint2 hi, lo;
      split_bf16x4(bv[i], hi, lo);
      *reinterpret_cast<uint2 *>(b_hi + kc * kHeadSlabB + r * 16 + half) = hi;
      *reinterpret_cast<uint2 *>(b_lo + kc * kHeadSlabB + r * 16 + half) = lo;
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
  // epilogue: warp w reads TMEM lanes 32 (w % 4).. (rows) and 32 of the 64 columns
  float *stage = reinterpret_cast<float *>(smem);  // [128][kHeadOutPitch], the slabs are dead
  {
    const int row = 32 * (warp & 3) + (tid & 31), col0 = 32 * (warp >> 2);
    float acc[32];
    sm100::tmem_ld16(tbase + ((uint32_t)(32 * (warp & 3)) << 16) + col0, acc);
    sm100::tmem_ld16(tbase + ((uint32_t)(32 * (warp & 3)) << 16) + col0 + 16, acc + 16);
    sm100::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4 *>(stage + row * kHeadOutPitch + col0 + j) =
          make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
  }
  __syncthreads();
  const float nanv = __int_as_float(0x7fc00000);
  for (int i = tid; i < kHeadRows * kHeadN / 4; i += kHeadThreads) {
    const int r = i >> 4, c = (i & 15) * 4;
    const int64_t row = r0 + r;
    if (row >= B) continue;
    float4 v = *reinterpret_cast<const float4 *>(stage + r * kHeadOutPitch + c);
    if (nblk == 0) v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (timed_out) v = make_float4(nanv, nanv, nanv, nanv);
    float *dst = partial + ((int64_t)blockIdx.z * B + row) * K + n0 + c;
    if (n0 + c + 4 <= K && (K & 3) == 0) {
      *reinterpret_cast<float4 *>(dst) = v;
    } else {
      const float e[4] = {v.x, v.y, v.z, v.w};
      for (int j = 0; j < 4; ++j)
        if (n0 + c + j < K) dst[j] = e[j];
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
// `status` (may be NULL): the forward's device error word; when any bounded
// wait of the forward gave up (a look-back, a tile or an MMA completion), the
// moments behind the logits are not trustworthy and every logit is NaN.
__global__ void head_reduce_kernel(const float *__restrict__ partial, const float *__restrict__ bias,
                                   float *__restrict__ logits, int64_t n, int K, int splits,
                                   const uint32_t *__restrict__ status) {
  const bool poisoned = status && __ldcg(status) != 0u;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = __ldg(bias + (int)(i % K));
    for (int z = 0; z < splits; ++z) acc += partial[z * n + i];
    logits[i] = poisoned ? __int_as_float(0x7fc00000) : acc;
  }
}

constexpr int kHeadSplits = 4;  // measured best at B=256, K=1000 (6 and 11 are slower)

inline size_t head_partial_floats(int64_t B, int K) { return (size_t)kHeadSplits * B * K; }

// logits [B, K] from features [B, width]; `partial` holds head_partial_floats(B, K)
// floats.  A wait that gives up (here, or earlier in the forward: a nonzero
// `status` word) writes NaN logits.
inline int head_gemm(const float *feats, int64_t B, int width, const float *G, const float *bias,
                     float *logits, int K, float *partial, cudaStream_t st,
                     const uint32_t *status = nullptr) {
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
  head_reduce_kernel<<<blocks, 256, 0, st>>>(partial, bias, logits, n, K, kHeadSplits, status);
  return after_launch("head_reduce_kernel");
}

}  // namespace lnet
