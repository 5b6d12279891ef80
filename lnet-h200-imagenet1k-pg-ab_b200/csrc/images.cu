// Input pipeline of the image configuration: uint8 images [B, H, W, 3] ->
// normalised, patchified tokens [B, (H/p)(W/p), 3 p^2] (bf16 or fp32).
//
// Per element (the transform of scripts/train_alphabet2d_imagenet100.py:292-310,
// ConvertImageDtype(float32) then Normalize(mean, std), fp32 throughout):
//   v = (u / 255 - mean[ch]) / std[ch]     (IEEE divisions, as torch computes it)
// and the token layout of the harness patchify
//   x[b, pr * (W/p) + pc, (i * p + j) * 3 + ch] = v(b, pr * p + i, pc * p + j, ch),
// so the tokens are bit-identical to the harness computing the same transform
// in PyTorch.  HBM-bound: one thread per (token, pixel row of its patch) reads
// the 3p contiguous bytes of that row and writes 3p contiguous tokens channels.
#include <cuda_bf16.h>

#include "common.cuh"
#include "lnet_b200.h"

namespace lnet {

struct Normalise {
  float mean[3], std[3];
};

__device__ __forceinline__ float normalise(uint32_t u, int ch, const Normalise &nz) {
  return ((float)u / 255.0f - nz.mean[ch]) / nz.std[ch];
}

__device__ __forceinline__ void put(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void put(float *p, float v) { *p = v; }

// Generic patch size.
template <typename T>
__global__ void patchify_kernel(const uint8_t *__restrict__ img, int64_t batch, int H, int W,
                                int p, Normalise nz, T *__restrict__ out) {
  const int PW = W / p, PH = H / p;
  const int64_t tokens = (int64_t)PH * PW;
  const int64_t n = batch * tokens * p;
  const int C = 3 * p * p;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bt = idx / p;
    const int i = (int)(idx - bt * p);
    const int64_t b = bt / tokens;
    const int t = (int)(bt - b * tokens);
    const int pr = t / PW, pc = t - (t / PW) * PW;
    const uint8_t *src = img + ((b * H + (int64_t)pr * p + i) * W + (int64_t)pc * p) * 3;
    T *dst = out + bt * C + (int64_t)i * p * 3;
    for (int e = 0; e < 3 * p; ++e) put(dst + e, normalise(src[e], e % 3, nz));
  }
}

// p = 4: a patch row is 12 bytes (three aligned 32-bit words, since every
// row offset is a multiple of 12) and 12 bf16 out (three 8-byte stores).
__global__ void patchify4_bf16_kernel(const uint8_t *__restrict__ img, int64_t batch, int H, int W,
                                      Normalise nz, __nv_bfloat16 *__restrict__ out) {
  const int PW = W / 4, PH = H / 4;
  const int64_t tokens = (int64_t)PH * PW;
  const int64_t n = batch * tokens * 4;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bt = idx >> 2;
    const int i = (int)(idx & 3);
    const int64_t b = bt / tokens;
    const int t = (int)(bt - b * tokens);
    const int pr = t / PW, pc = t - (t / PW) * PW;
    const uint32_t *src = reinterpret_cast<const uint32_t *>(
        img + ((b * H + (int64_t)pr * 4 + i) * W + (int64_t)pc * 4) * 3);
    const uint32_t w[3] = {__ldg(src), __ldg(src + 1), __ldg(src + 2)};
    uint32_t packed[6];
#pragma unroll
    for (int e = 0; e < 12; e += 2) {
      const uint32_t u0 = (w[e / 4] >> (8 * (e % 4))) & 0xFFu;
      const uint32_t u1 = (w[(e + 1) / 4] >> (8 * ((e + 1) % 4))) & 0xFFu;
      __nv_bfloat162 h =
          __floats2bfloat162_rn(normalise(u0, e % 3, nz), normalise(u1, (e + 1) % 3, nz));
      packed[e / 2] = *reinterpret_cast<uint32_t *>(&h);
    }
    uint2 *dst = reinterpret_cast<uint2 *>(out + bt * 48 + i * 12);
    dst[0] = make_uint2(packed[0], packed[1]);
    dst[1] = make_uint2(packed[2], packed[3]);
    dst[2] = make_uint2(packed[4], packed[5]);
  }
}

}  // namespace lnet

using namespace lnet;

extern "C" int lnet_b200_patchify_images(const uint8_t *images, int64_t batch, int32_t height,
                                         int32_t width, int32_t patch, const float *mean,
                                         const float *std, void *tokens, int32_t tokens_dtype,
                                         lnet_stream_t stream) {
  reset_launches();
  begin_entry((cudaStream_t)stream);
  if (batch < 0 || height < 1 || width < 1 || patch < 1)
    return fail(LNET_ERR_INVALID_ARGUMENT, "patchify: invalid shape");
  if (height % patch != 0 || width % patch != 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "patchify: image %dx%d is not divisible by patch %d",
                height, width, patch);
  if (!images || !tokens || !mean || !std)
    return fail(LNET_ERR_INVALID_ARGUMENT, "patchify: NULL pointer");
  if (tokens_dtype != LNET_BF16 && tokens_dtype != LNET_F32)
    return fail(LNET_ERR_UNSUPPORTED, "patchify: tokens must be bf16 or fp32");
  if (batch == 0) return LNET_OK;
  Normalise nz;
  for (int c = 0; c < 3; ++c) {
    if (!(std[c] != 0.f)) return fail(LNET_ERR_INVALID_ARGUMENT, "patchify: std must be nonzero");
    nz.mean[c] = mean[c];
    nz.std[c] = std[c];
  }
  const int64_t n = batch * (int64_t)(height / patch) * (width / patch) * patch;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n, 256), 148 * 32);
  cudaStream_t st = (cudaStream_t)stream;
  if (patch == 4 && tokens_dtype == LNET_BF16 && reinterpret_cast<uintptr_t>(images) % 4 == 0 &&
      reinterpret_cast<uintptr_t>(tokens) % 8 == 0) {
    patchify4_bf16_kernel<<<grid, 256, 0, st>>>(images, batch, height, width, nz,
                                                (__nv_bfloat16 *)tokens);
    return after_launch("patchify4_bf16_kernel");
  }
  if (tokens_dtype == LNET_BF16)
    patchify_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(images, batch, height, width, patch, nz,
                                                         (__nv_bfloat16 *)tokens);
  else
    patchify_kernel<float><<<grid, 256, 0, st>>>(images, batch, height, width, patch, nz,
                                                 (float *)tokens);
  return after_launch("patchify_kernel");
}
