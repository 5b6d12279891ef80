// Unit-grid fused route of the ALPHABET forward (placeholder until the fused
// kernels land) and the scratch-free head kernel.
#pragma once

#include "common.cuh"
#include "generic_kernels.cuh"

namespace lnet {

struct FusedWorkspace {
  float *moments = nullptr;  // [2][B][7M]
};

inline void plan_fused(Arena &ar, FusedWorkspace &w, const lnet_b200_alphabet_params *p,
                       const lnet_b200_alphabet_request *r) {
  w.moments = ar.take<float>((size_t)2 * r->batch * 7 * p->modes);
}

inline bool fused_supported(const lnet_b200_alphabet_params *, const lnet_b200_alphabet_request *) {
  return false;
}

inline int fused_forward(const lnet_b200_alphabet_params *, const lnet_b200_alphabet_request *,
                         FusedWorkspace &, float *, float *, cudaStream_t) {
  return fail(LNET_ERR_UNSUPPORTED, "fused route not built");
}

// Head without scratch: every block rebuilds the radial-log features of its
// row in shared memory, then each warp produces logits for its classes.
constexpr int kHeadClassesPerBlock = 64;
__global__ void __launch_bounds__(256) head_kernel(const float *__restrict__ wm,
                                                   const float *__restrict__ rm,
                                                   const float *__restrict__ G,
                                                   const float *__restrict__ bias,
                                                   float *__restrict__ logits, int modes,
                                                   int classes) {
  extern __shared__ float feats[];
  const int64_t b = blockIdx.y;
  const int width = 14 * modes;
  for (int j = threadIdx.x; j < width; j += blockDim.x) {
    const float *src = j < 7 * modes ? wm + b * 7 * modes : rm + b * 7 * modes;
    feats[j] = radial_feature(src, modes, j < 7 * modes ? j : j - 7 * modes);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.x * kHeadClassesPerBlock;
  for (int k = k0 + warp; k < min(classes, k0 + kHeadClassesPerBlock); k += blockDim.x >> 5) {
    const float *g = G + (int64_t)k * width;
    float acc = 0.f;
    for (int j = lane; j < width; j += 32) acc = fmaf(feats[j], g[j], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) logits[b * classes + k] = acc + bias[k];
  }
}

inline int fused_head(const lnet_b200_alphabet_params *p, int64_t B, const float *wm,
                      const float *rm, float *logits, cudaStream_t st) {
  const int M = p->modes, K = p->output_dim;
  size_t smem = (size_t)14 * M * sizeof(float);
  if (smem > 48 * 1024) {
    LNET_TRY(cuda_check(cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "cudaFuncSetAttribute(head_kernel)"));
  }
  dim3 g((unsigned)cdiv(K, kHeadClassesPerBlock), (unsigned)B);
  head_kernel<<<g, 256, smem, st>>>(wm, rm, p->head_weight, p->head_bias, logits, M, K);
  return after_launch("head_kernel");
}

}  // namespace lnet
