// Stage kernels of the general ALPHABET path (every metadata combination).
//
// Each kernel is one bandwidth-bound pass over [B, T, *] fp32 tensors (the
// projections are library GEMMs, blas.cuh); the fused route (fused_path.cuh)
// replaces them for the compiled shapes without metadata.
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace lnet {

// ---------------------------------------------------------------- fp32 -> bf16 copy
__global__ void to_bf16_kernel(const float *__restrict__ src, __nv_bfloat16 *__restrict__ dst,
                               int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// ---------------------------------------------------------------- stem input mask
// xm[b,t,c] = x[b,t,c] * obs[b,t,c|0] * valid[b,t]
template <typename TX>
__global__ void mask_inputs_kernel(const TX *__restrict__ x, const float *__restrict__ obs,
                                   int obs_channels, const float *__restrict__ valid,
                                   float *__restrict__ xm, int64_t tokens, int channels) {
  // block-stride over tokens, threads over channels (no per-element division)
  for (int64_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
    for (int c = threadIdx.x; c < channels; c += blockDim.x) {
      const int64_t i = tok * channels + c;
      float v = load_f(x, i);
      if (obs) v *= obs[tok * obs_channels + (obs_channels == 1 ? 0 : c)];
      if (valid) v *= valid[tok];
      xm[i] = v;
    }
  }
}

// ---------------------------------------------------------------- unit-grid depthwise conv
constexpr int kDwTile = 16;  // steps per block
// out[b,t,d] = post[b,t] * SiLU(bias[d] + sum_k w[d,k] * pre[b,t] in[b, t + k*dil - pad, d])
template <typename TI>
__global__ void dwconv_unit_kernel(const TI *__restrict__ in, const float *__restrict__ w,
                                   const float *__restrict__ bias,
                                   const float *__restrict__ in_mask,
                                   const float *__restrict__ out_mask, float *__restrict__ out,
                                   int64_t batch, int64_t steps, int dim, int taps,
                                   int dilation) {
  // block (step tile, row): kDwTile consecutive steps of one row, threads over
  // channels (the taps of neighbouring steps overlap and hit L1; no division)
  const int pad = dilation * (taps - 1) / 2;
  const unsigned tiles = (unsigned)((steps + kDwTile - 1) / kDwTile);
  const int64_t b = blockIdx.x / tiles;  // grid = rows x tiles, flattened
  const int64_t t_begin = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kDwTile;
  const int64_t t_end = min(steps, t_begin + kDwTile);
  const TI *row_in = in + b * steps * dim;
  float *row_out = out + b * steps * dim;
  const float *im = in_mask ? in_mask + b * steps : nullptr;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    const float bd = bias[d];
    for (int64_t t = t_begin; t < t_end; ++t) {
      float acc = 0.f;
      for (int k = 0; k < taps; ++k) {
        const int64_t s = t + (int64_t)k * dilation - pad;
        if (s < 0 || s >= steps) continue;
        float v = load_f(row_in, s * dim + d);
        if (im) v *= im[s];
        acc = fmaf(w[d * taps + k], v, acc);
      }
      float y = silu_f(acc + bd);
      if (out_mask) y *= out_mask[b * steps + t];
      row_out[t * dim + d] = y;
    }
  }
}

// Shared-memory tile form of the same conv for the canonical geometry (TAPS
// taps, dilation DIL, fp32, dim % 4 == 0, 16-byte aligned rows).  Block =
// (row, kDwTileSteps steps, kDwTileChans channels): the block stages the
// kDwTileSteps + 2 PAD input steps of its channels with independent float4 loads
// (every load in flight at once), then each thread produces outputs of one
// channel quad from shared memory.  Same arithmetic as dwconv_unit_kernel, term
// for term: taps outside the sequence read 0 and fmaf(w, 0, acc) == acc.
constexpr int kDwTileSteps = 32, kDwTileChans = 64, kDwTileThreads = 128;
template <int TAPS, int DIL>
__global__ void __launch_bounds__(kDwTileThreads) dwconv_tile_kernel(
    const float *__restrict__ in, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ in_mask, const float *__restrict__ out_mask,
    float *__restrict__ out, int64_t steps, int dim) {
  constexpr int PAD = DIL * (TAPS - 1) / 2;
  constexpr int ROWS = kDwTileSteps + 2 * PAD;
  constexpr int Q = kDwTileChans / 4;
  __shared__ float4 tile[ROWS][Q];
  const int quads = dim >> 2;
  const int qbase = blockIdx.y * Q;
  const int nq = min(Q, quads - qbase);
  const unsigned tiles = (unsigned)((steps + kDwTileSteps - 1) / kDwTileSteps);
  const int64_t b = blockIdx.x / tiles;
  const int64_t t0 = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kDwTileSteps;
  const float4 *row = reinterpret_cast<const float4 *>(in + b * steps * dim) + qbase;
  for (int i = threadIdx.x; i < ROWS * Q; i += kDwTileThreads) {
    const int r = i / Q, qq = i - (i / Q) * Q;
    const int64_t s = t0 - PAD + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qq < nq && s >= 0 && s < steps) {
      v = __ldg(row + s * quads + qq);
      if (in_mask) {
        const float mk = in_mask[b * steps + s];
        v.x *= mk; v.y *= mk; v.z *= mk; v.w *= mk;
      }
    }
    tile[r][qq] = v;
  }
  __syncthreads();
  const int q = threadIdx.x % Q, g = threadIdx.x / Q;
  if (q >= nq) return;
  const int c = 4 * (qbase + q);
  float wk[4][TAPS];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int k = 0; k < TAPS; ++k) wk[j][k] = w[(c + j) * TAPS + k];
  const float4 bd = reinterpret_cast<const float4 *>(bias)[qbase + q];
  float4 *orow = reinterpret_cast<float4 *>(out + b * steps * dim) + qbase + q;
#pragma unroll 2
  for (int i = g; i < kDwTileSteps; i += kDwTileThreads / Q) {
    const int64_t t = t0 + i;
    if (t >= steps) break;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int k = 0; k < TAPS; ++k) {
      const float4 v = tile[i + k * DIL][q];
      a0 = fmaf(wk[0][k], v.x, a0);
      a1 = fmaf(wk[1][k], v.y, a1);
      a2 = fmaf(wk[2][k], v.z, a2);
      a3 = fmaf(wk[3][k], v.w, a3);
    }
    float4 y = make_float4(silu_f(a0 + bd.x), silu_f(a1 + bd.y), silu_f(a2 + bd.z),
                           silu_f(a3 + bd.w));
    if (out_mask) {
      const float mk = out_mask[b * steps + t];
      y.x *= mk; y.y *= mk; y.z *= mk; y.w *= mk;
    }
    orow[t * quads] = y;
  }
}

// Depthwise conv + SiLU + RMSNorm in one pass (canonical geometry, dim % 4 == 0,
// dim <= 256) over tiles of kDnSteps steps x all channels of one row: the
// per-step sum of squares reduced through shared memory (each quad's four
// squares, strided partial sums, a shuffle tree), xhat = y rs g written
// directly, the conv output y itself only when `y_out` is given.  With `base`,
// also writes the writer's residual base y + ls (ds xhat) (the synthesis GEMM
// adds ls (s W^T) on top).
//
// A tile's input steps [t0 - PAD, t0 + kDnSteps + PAD) are one contiguous span
// of memory, brought into shared memory by one bulk TMA copy on an mbarrier.
// Persistent blocks walk the tiles with two buffers: the copy of the next tile
// is in flight while the current one is computed.  Thread 0 waits (bounded) and
// tells the block through shared memory; on timeout it sets kErrBulk in
// `status`, waits once more for the copies still in flight, and the block
// returns.  Shared memory: two input tiles [kDnSteps + 2 PAD][dim],
// [kDnSteps][dim / 4] squares, [kDnSteps] scales, two mbarriers, a flag.
constexpr int kDnSteps = 32, kDnThreads = 256, kDnMaxPer = 8, kDnParts = kDnThreads / kDnSteps;
constexpr int kDnBlocksPerSM = 2;
constexpr uint32_t kErrBulk = 1u << 8;
constexpr uint32_t kBulkSpinLimit = 1u << 20;
__host__ __device__ constexpr size_t dwconv_norm_smem(int rows, int quads, int elem_bytes) {
  return 2 * (size_t)rows * quads * 4 * elem_bytes + (size_t)kDnSteps * quads * 4 +
         kDnSteps * 4 + 32;
}
// Four consecutive channels of T as one shared-memory / global element.
template <typename T> struct Quad4;
template <> struct Quad4<float> {
  using V = float4;
  __device__ static float4 get(V v) { return v; }
  __device__ static V put(float4 f) { return f; }
};
template <> struct Quad4<__nv_bfloat16> {
  using V = uint2;
  __device__ static float4 get(V v) {
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
  }
  __device__ static V put(float4 f) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(f.x, f.y), hi = __floats2bfloat162_rn(f.z, f.w);
    return make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                      *reinterpret_cast<const uint32_t *>(&hi));
  }
};
template <int TAPS, int DIL, typename TIN, typename TXH>
__global__ void __launch_bounds__(kDnThreads, kDnBlocksPerSM) dwconv_norm_kernel(
    const TIN *__restrict__ in, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ in_mask, const float *__restrict__ out_mask,
    const float *__restrict__ g, const float *__restrict__ ls, const float *__restrict__ ds,
    TXH *__restrict__ xhat, float *__restrict__ base, float *__restrict__ y_out, int64_t batch,
    int64_t steps, int dim, uint32_t *__restrict__ status) {
  constexpr int PAD = DIL * (TAPS - 1) / 2;
  constexpr int ROWS = kDnSteps + 2 * PAD;
  using QI = Quad4<TIN>;
  using VI = typename QI::V;
  extern __shared__ float4 dn_smem[];
  const int quads = dim >> 2;
  const int groups = kDnThreads / quads;
  VI *tiles = reinterpret_cast<VI *>(dn_smem);                       // [2][ROWS][quads]
  float *sq = reinterpret_cast<float *>(tiles + 2 * ROWS * quads);   // [kDnSteps][quads]
  float *rs_s = sq + kDnSteps * quads;                               // [kDnSteps]
  uint64_t *bars = reinterpret_cast<uint64_t *>(rs_s + kDnSteps);    // [2]
  volatile uint32_t *fail_flag = reinterpret_cast<uint32_t *>(bars + 2);
  const int64_t per_row = (steps + kDnSteps - 1) / kDnSteps;
  const int64_t total = batch * per_row;
  const int q = threadIdx.x % quads, grp = threadIdx.x / quads;
  const bool active = grp < groups;

  auto issue = [&](int64_t id, int buf) {
    const int64_t b = id / per_row, first = (id - b * per_row) * kDnSteps - PAD;
    const int64_t lo = max((int64_t)0, first), hi = min(steps, first + ROWS);
    const uint32_t bytes = (uint32_t)((hi - lo) * dim * (int64_t)sizeof(TIN));
    sm100::mbar_arrive_expect_tx(&bars[buf], bytes);
    sm100::bulk_load(sm100::smem_u32(tiles + buf * ROWS * quads + (lo - first) * quads),
                     in + (b * steps + lo) * dim, bytes, &bars[buf]);
  };
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::fence_barrier_init();
    *fail_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0 && (int64_t)blockIdx.x < total) issue(blockIdx.x, 0);

  // per-thread constants
  float wk[4][TAPS];
  float4 bd = make_float4(0.f, 0.f, 0.f, 0.f), gq = bd, lq = bd, dq = bd;
  if (active) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int k = 0; k < TAPS; ++k) wk[j][k] = w[(4 * q + j) * TAPS + k];
    bd = reinterpret_cast<const float4 *>(bias)[q];
    gq = reinterpret_cast<const float4 *>(g)[q];
    if (base) {
      lq = reinterpret_cast<const float4 *>(ls)[q];
      dq = reinterpret_cast<const float4 *>(ds)[q];
    }
  }

  int k = 0;
  for (int64_t id = blockIdx.x; id < total; id += gridDim.x, ++k) {
    const int cur = k & 1;
    const int64_t nxt = id + gridDim.x;
    if (threadIdx.x == 0) {
      if (nxt < total) {
        sm100::fence_proxy_async_smem();  // this buffer's last generic writes before the copy
        issue(nxt, cur ^ 1);
      }
      if (!sm100::mbar_wait_bounded(&bars[cur], (k >> 1) & 1, kBulkSpinLimit)) {
        atomicOr(status, kErrBulk);
        sm100::mbar_wait_bounded(&bars[cur], (k >> 1) & 1, kBulkSpinLimit);
        if (nxt < total) sm100::mbar_wait_bounded(&bars[cur ^ 1], ((k + 1) >> 1) & 1, kBulkSpinLimit);
        *fail_flag = 1;
      }
    }
    __syncthreads();
    if (*fail_flag) return;
    const int64_t b = id / per_row, t0 = (id - b * per_row) * kDnSteps, first = t0 - PAD;
    const int64_t lo = max((int64_t)0, first), hi = min(steps, first + ROWS);
    VI *tile = tiles + cur * ROWS * quads;
    if (lo > first || hi < first + ROWS || in_mask) {
      for (int i = threadIdx.x; i < ROWS * quads; i += kDnThreads) {
        const int64_t s = first + i / quads;
        if (s < lo || s >= hi) {
          tile[i] = QI::put(make_float4(0.f, 0.f, 0.f, 0.f));
        } else if (in_mask) {  // (re-rounded for bf16 input)
          const float mk = in_mask[b * steps + s];
          float4 v = QI::get(tile[i]);
          v.x *= mk; v.y *= mk; v.z *= mk; v.w *= mk;
          tile[i] = QI::put(v);
        }
      }
      __syncthreads();
    }
    float4 y[kDnMaxPer];
    if (active) {
#pragma unroll
      for (int n = 0; n < kDnMaxPer; ++n) {
        const int i = grp + n * groups;
        if (i >= kDnSteps) break;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int kk = 0; kk < TAPS; ++kk) {
          const float4 v = QI::get(tile[(i + kk * DIL) * quads + q]);
          a0 = fmaf(wk[0][kk], v.x, a0);
          a1 = fmaf(wk[1][kk], v.y, a1);
          a2 = fmaf(wk[2][kk], v.z, a2);
          a3 = fmaf(wk[3][kk], v.w, a3);
        }
        float4 yy = make_float4(silu_f(a0 + bd.x), silu_f(a1 + bd.y), silu_f(a2 + bd.z),
                                silu_f(a3 + bd.w));
        if (out_mask) {
          const float mk = t0 + i < steps ? out_mask[b * steps + t0 + i] : 0.f;
          yy.x *= mk; yy.y *= mk; yy.z *= mk; yy.w *= mk;
        }
        y[n] = yy;
        sq[i * quads + q] = fmaf(yy.w, yy.w, fmaf(yy.z, yy.z, fmaf(yy.y, yy.y, yy.x * yy.x)));
      }
    }
    __syncthreads();
    {  // per step: kDnParts threads sum strided quads, then a shuffle tree
      const int i = threadIdx.x / kDnParts, part = threadIdx.x % kDnParts;
      float ss = 0.f;
      for (int qq = part; qq < quads; qq += kDnParts) ss += sq[i * quads + qq];
#pragma unroll
      for (int o = kDnParts / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (part == 0) rs_s[i] = rsqrtf(ss / (float)dim + kFp32Eps);
    }
    __syncthreads();
    if (active) {
      const int64_t tile_off = (b * steps + t0) * quads + q;
      auto *xo = reinterpret_cast<typename Quad4<TXH>::V *>(xhat) + tile_off;
      float4 *yo = y_out ? reinterpret_cast<float4 *>(y_out) + tile_off : nullptr;
      float4 *bo = base ? reinterpret_cast<float4 *>(base) + tile_off : nullptr;
      const int n_steps = (int)min((int64_t)kDnSteps, steps - t0);
#pragma unroll
      for (int n = 0; n < kDnMaxPer; ++n) {
        const int i = grp + n * groups;
        if (i >= n_steps) break;
        const int off = i * quads;
        const float r = rs_s[i];
        const float4 yy = y[n];
        const float4 xh = make_float4(yy.x * r * gq.x, yy.y * r * gq.y, yy.z * r * gq.z,
                                      yy.w * r * gq.w);
        xo[off] = Quad4<TXH>::put(xh);
        if (yo) yo[off] = yy;
        if (bo)
          bo[off] = make_float4(yy.x + lq.x * (dq.x * xh.x), yy.y + lq.y * (dq.y * xh.y),
                                yy.z + lq.z * (dq.z * xh.z), yy.w + lq.w * (dq.w * xh.w));
      }
    }
    __syncthreads();  // the tile, squares and scales are reused next iteration
  }
}

// The writer's residual base v = x + ls (ds xhat) (dwconv_norm_kernel's `base`
// formula), for the slice entry points.
__global__ void residual_base_kernel(const float *__restrict__ x, const float *__restrict__ xhat,
                                     const float *__restrict__ ds, const float *__restrict__ ls,
                                     float *__restrict__ v, int64_t tokens, int dim) {
  const int64_t n = tokens * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % dim);
    v[i] = x[i] + ls[d] * (ds[d] * xhat[i]);
  }
}

// out[d, j] = scale[d] * frame[d, j] for a [dim, n] row-major frame.
__global__ void scale_rows_kernel(const float *__restrict__ frame, const float *__restrict__ scale,
                                  float *__restrict__ out, int dim, int n) {
  const int64_t total = (int64_t)dim * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = scale[i / n] * frame[i];
}

// ---------------------------------------------------------------- physical-time depthwise conv
// Restates _physical_time_depthwise_conv (src/lnet/alphabet_backbone.py:80-160).
// One block per (token); threads over channels.  The sample positions are
// shared by all channels and computed once per token by thread 0..taps-1.
template <typename TI>
__global__ void dwconv_physical_kernel(const TI *__restrict__ in, const float *__restrict__ w,
                                       const float *__restrict__ bias,
                                       const float *__restrict__ in_mask,
                                       const float *__restrict__ ts,
                                       const float *__restrict__ valid,
                                       float *__restrict__ out, int64_t steps, int dim,
                                       int taps, int dilation) {
  __shared__ int64_t s_lo[16], s_hi[16];
  __shared__ float s_w[16];
  __shared__ int s_on[16];
  const int64_t tok = blockIdx.x;
  const int64_t b = tok / steps;
  const int64_t t = tok - b * steps;
  const float *row = ts + b * steps;
  if (threadIdx.x < taps) {
    int k = threadIdx.x;
    float offset = (float)(k * dilation - dilation * (taps - 1) / 2);
    float q = row[t] + offset;
    int64_t up_u = lower_bound_f(row, steps, q);
    int64_t up = up_u < steps - 1 ? up_u : steps - 1;
    int64_t lo = up_u - 1;
    lo = lo < 0 ? 0 : (lo > steps - 1 ? steps - 1 : lo);
    float lt = row[lo], ut = row[up];
    float dur = ut - lt;
    float interp = dur > 0.f ? (q - lt) / fmaxf(dur, kFp32Tiny) : 0.f;
    interp = fminf(fmaxf(interp, 0.f), 1.f);
    bool on = (q >= row[0]) && (q <= row[steps - 1]);
    if (valid) {
      float lv = valid[b * steps + lo], uv = valid[b * steps + up];
      const float eps8 = 8.0f * kFp32Eps;
      float support = interp <= eps8 ? lv : (interp >= 1.0f - eps8 ? uv : lv * uv);
      on = on && (support > 0.f);
    }
    s_lo[k] = b * steps + lo;
    s_hi[k] = b * steps + up;
    s_w[k] = interp;
    s_on[k] = on;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float acc = 0.f;
    for (int k = 0; k < taps; ++k) {
      float a = load_f(in, s_lo[k] * dim + d);
      float c = load_f(in, s_hi[k] * dim + d);
      if (in_mask) {
        a *= in_mask[s_lo[k]];
        c *= in_mask[s_hi[k]];
      }
      float v = s_on[k] ? lerp_torch(a, c, s_w[k]) : 0.f;
      acc = fmaf(v, w[d * taps + k], acc);
    }
    float y = silu_f(acc + bias[d]);
    if (valid) y *= valid[tok];
    out[tok * dim + d] = y;
  }
}

// Tiled form of the same conv for fp32 rows with 4 | dim and 16-byte aligned
// rows: one block per (row, 32-token tile).  The sample positions, weights and
// support of every (token, tap) of the tile are resolved once into shared
// memory (binary search over the row's timestamps); then threads take
// (token, 4-channel quad) pairs with 16-byte loads of the two interpolation
// rows.  The per-element arithmetic is the per-token kernel's, in the same order.
constexpr int kPtTile = 32, kPtMaxTaps = 8, kPtThreads = 256;
__global__ void __launch_bounds__(kPtThreads) dwconv_physical_tile_kernel(
    const float *__restrict__ in, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ in_mask, const float *__restrict__ ts,
    const float *__restrict__ valid, float *__restrict__ out, int64_t steps, int dim, int taps,
    int dilation) {
  __shared__ int s_lo[kPtTile][kPtMaxTaps], s_hi[kPtTile][kPtMaxTaps];
  __shared__ float s_w[kPtTile][kPtMaxTaps], s_mlo[kPtTile][kPtMaxTaps], s_mhi[kPtTile][kPtMaxTaps];
  __shared__ int s_on[kPtTile][kPtMaxTaps];
  extern __shared__ float s_wt[];  // [taps][dim] weights, then [dim] bias
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.x * kPtTile;
  const int n_tok = (int)min((int64_t)kPtTile, steps - t0);
  const float *row = ts + b * steps;
  const float first = row[0], last = row[steps - 1];
  for (int i = threadIdx.x; i < taps * dim; i += blockDim.x) {
    const int k = i / dim, d = i - k * dim;
    s_wt[i] = w[d * taps + k];
  }
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s_wt[taps * dim + i] = bias[i];
  for (int i = threadIdx.x; i < n_tok * taps; i += blockDim.x) {
    const int j = i / taps, k = i - j * taps;
    const int64_t t = t0 + j;
    const float offset = (float)(k * dilation - dilation * (taps - 1) / 2);
    const float q = row[t] + offset;
    const int64_t up_u = lower_bound_f(row, steps, q);
    const int64_t up = up_u < steps - 1 ? up_u : steps - 1;
    int64_t lo = up_u - 1;
    lo = lo < 0 ? 0 : (lo > steps - 1 ? steps - 1 : lo);
    const float lt = row[lo], ut = row[up];
    const float dur = ut - lt;
    float interp = dur > 0.f ? (q - lt) / fmaxf(dur, kFp32Tiny) : 0.f;
    interp = fminf(fmaxf(interp, 0.f), 1.f);
    bool on = (q >= first) && (q <= last);
    if (valid) {
      const float lv = valid[b * steps + lo], uv = valid[b * steps + up];
      const float eps8 = 8.0f * kFp32Eps;
      const float support = interp <= eps8 ? lv : (interp >= 1.0f - eps8 ? uv : lv * uv);
      on = on && (support > 0.f);
    }
    s_lo[j][k] = (int)lo;
    s_hi[j][k] = (int)up;
    s_w[j][k] = interp;
    s_on[j][k] = on;
    s_mlo[j][k] = in_mask ? in_mask[b * steps + lo] : 1.f;
    s_mhi[j][k] = in_mask ? in_mask[b * steps + up] : 1.f;
  }
  __syncthreads();
  const int quads = dim / 4;
  const float *in_row = in + b * steps * dim;
  for (int i = threadIdx.x; i < n_tok * quads; i += blockDim.x) {
    const int j = i / quads, qd = i - j * quads, d0 = 4 * qd;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < taps; ++k) {
      const float4 a4 = *reinterpret_cast<const float4 *>(in_row + (int64_t)s_lo[j][k] * dim + d0);
      const float4 c4 = *reinterpret_cast<const float4 *>(in_row + (int64_t)s_hi[j][k] * dim + d0);
      const float av[4] = {a4.x, a4.y, a4.z, a4.w}, cv[4] = {c4.x, c4.y, c4.z, c4.w};
      const float wk = s_w[j][k], ml = s_mlo[j][k], mh = s_mhi[j][k];
      const bool on = s_on[j][k] != 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a = av[e], c = cv[e];
        if (in_mask) {
          a *= ml;
          c *= mh;
        }
        const float v = on ? lerp_torch(a, c, wk) : 0.f;
        acc[e] = fmaf(v, s_wt[k * dim + d0 + e], acc[e]);
      }
    }
    const int64_t tok = b * steps + t0 + j;
    const float vt = valid ? valid[tok] : 1.f;
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      y[e] = silu_f(acc[e] + s_wt[taps * dim + d0 + e]);
      if (valid) y[e] *= vt;
    }
    *reinterpret_cast<float4 *>(out + tok * dim + d0) = make_float4(y[0], y[1], y[2], y[3]);
  }
}

// ts[b, t] = fp32(sum_{s<=t} double(dt[b, s])) as a block scan in double, one
// block per row: each thread sums eight consecutive steps, the block scans the
// thread sums, and a running carry joins the 2048-step segments.  (A parallel
// cumsum, as a GPU cumsum is; for step sizes whose partial sums are exact in
// double -- every clipped Exponential(1) grid -- it equals the sequential sum.)
constexpr int kTsThreads = 256;
__global__ void __launch_bounds__(kTsThreads) timestamps_scan_kernel(const float *__restrict__ dt,
                                                                    float *__restrict__ ts,
                                                                    int64_t steps) {
  __shared__ double s_warp[kTsThreads / 32];
  const int64_t b = blockIdx.x;
  const float *src = dt + b * steps;
  float *dst = ts + b * steps;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  double carry = 0.0;
  for (int64_t seg = 0; seg < steps; seg += 8 * kTsThreads) {
    const int64_t t0 = seg + 8 * threadIdx.x;
    double v[8], sum = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[e] = t0 + e < steps ? (double)src[t0 + e] : 0.0;
      sum += v[e];
    }
    double incl = sum;  // inclusive scan of the thread sums: warp, then across warps
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) s_warp[wid] = incl;
    __syncthreads();
    double before = 0.0, total = 0.0;
    for (int q = 0; q < kTsThreads / 32; ++q) {
      if (q < wid) before += s_warp[q];
      total += s_warp[q];
    }
    double run = carry + before + (incl - sum);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      run += v[e];
      if (t0 + e < steps) dst[t0 + e] = (float)run;
    }
    carry += total;
    __syncthreads();
  }
}

// ---------------------------------------------------------------- RMSNorm
// One warp per token: out = x * rsqrt(mean(x^2) + eps) * g
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ g,
                               float *__restrict__ out, int64_t tokens, int dim) {
  int64_t tok = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (tok >= tokens) return;
  const float *row = x + tok * dim;
  float ss = 0.f;
  for (int d = lane; d < dim; d += 32) ss = fmaf(row[d], row[d], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  float rs = rsqrtf(ss / (float)dim + kFp32Eps);
  for (int d = lane; d < dim; d += 32) out[tok * dim + d] = row[d] * rs * g[d];
}

// The same RMSNorm over float4 quads (dim % 4 == 0, 16-byte aligned rows):
// `width` lanes per token -- dim / 4 when that is a power of two below 32, so
// 32 / width tokens share a warp and short rows (D = 64: 16 quads) still fill
// it; else 32 lanes striding over the quads.
__global__ void rmsnorm4_kernel(const float4 *__restrict__ x, const float4 *__restrict__ g,
                                float4 *__restrict__ out, int64_t tokens, int quads) {
  const int lane = threadIdx.x & 31;
  const int width = quads < 32 && (quads & (quads - 1)) == 0 ? quads : 32;
  const int per_warp = 32 / width;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t tok = warp * per_warp + lane / width;
  const int sl = lane & (width - 1);
  const bool on = tok < tokens;
  const float4 *row = x + tok * quads;
  float ss = 0.f;
  if (on)
    for (int q = sl; q < quads; q += width) {
      const float4 v = row[q];
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
  for (int o = width >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!on) return;
  const float rs = rsqrtf(ss / (float)(4 * quads) + kFp32Eps);
  for (int q = sl; q < quads; q += width) {
    const float4 v = row[q], w = g[q];
    out[tok * quads + q] = make_float4(v.x * rs * w.x, v.y * rs * w.y, v.z * rs * w.z,
                                       v.w * rs * w.w);
  }
}

// ---------------------------------------------------------------- drive (gamma (x) e * mask)
// e[tok, 0:M] / e[tok, M:2M] -> u in place; gamma from the per-mode table or per step.
// Without dt the gains are the per-mode table g_tab_re/im (zoh_kernel); with dt
// they are evaluated per (step, mode) in fp32 (zoh_eval_f32), and `step_a`
// (when given) receives the step's transition a = exp(p dt) as
// [tok][re M | im M] for the scans.  A block takes kDriveTokens tokens: the
// event masks (amax over the raw channels) are reduced once per token by a warp
// into shared memory, the mode poles once per block, and then one thread per
// (token, mode) pair, consecutive modes on consecutive lanes (block x).
constexpr int kDriveTokens = 32;
constexpr int kDriveMaxModes = 256;
__global__ void __launch_bounds__(256) drive_kernel(
    float *__restrict__ e, const float *__restrict__ raw_decay, const float *__restrict__ raw_freq,
    const float *__restrict__ dt, const float *__restrict__ g_tab_re,
    const float *__restrict__ g_tab_im, const float *__restrict__ event_mask, int obs_channels,
    int64_t tokens, int modes, float *__restrict__ step_a) {
  // per mode: (damping, frequency) with dt, the gain table (re, im) without
  __shared__ float s_pa[kDriveMaxModes], s_pb[kDriveMaxModes], s_mask[kDriveTokens];
  const int64_t tok0 = (int64_t)blockIdx.x * kDriveTokens;
  const int ntok = (int)(tokens - tok0 < kDriveTokens ? tokens - tok0 : kDriveTokens);
  // (modes past kDriveMaxModes are looked up per pair instead)
  auto mode_consts = [&](int m, float &pa, float &pb) {
    if (dt) {
      double damping, frequency;
      mode_pole(raw_decay[m], raw_freq[m], damping, frequency);
      pa = (float)damping;
      pb = (float)frequency;
    } else {
      pa = g_tab_re[m];
      pb = g_tab_im[m];
    }
  };
  const int tid = threadIdx.y * blockDim.x + threadIdx.x, nthreads = blockDim.x * blockDim.y;
  for (int m = tid; m < min(modes, kDriveMaxModes); m += nthreads)
    mode_consts(m, s_pa[m], s_pb[m]);
  if (event_mask) {
    // event mask = amax over raw channels (src/lnet/alphabet_backbone.py:568)
    const int warp = tid >> 5, lane = tid & 31;
    for (int t = warp; t < ntok; t += nthreads >> 5) {
      const float *om = event_mask + (tok0 + t) * obs_channels;
      float mx = -INFINITY;
      for (int c = lane; c < obs_channels; c += 32) mx = fmaxf(mx, om[c]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) s_mask[t] = mx;
    }
  }
  __syncthreads();
  // 2-D block: x over modes, y over the block's tokens (no index division)
  for (int t = threadIdx.y; t < ntok; t += blockDim.y)
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    const int64_t tok = tok0 + t;
    float pa, pb;
    if (m < kDriveMaxModes) {
      pa = s_pa[m];
      pb = s_pb[m];
    } else {
      mode_consts(m, pa, pb);
    }
    float gr, gi;
    if (dt) {
      const Zoh z = zoh_eval_f32(pa, pb, dt[tok]);
      gr = z.g_re;
      gi = z.g_im;
      if (step_a) {
        step_a[tok * 2 * modes + m] = z.a_re;
        step_a[tok * 2 * modes + modes + m] = z.a_im;
      }
    } else {
      gr = pa;
      gi = pb;
    }
    float *row = e + tok * 2 * modes;
    const float er = row[m], ei = row[modes + m];
    float ur = gr * er - gi * ei;
    float ui = gr * ei + gi * er;
    if (event_mask) {
      ur *= s_mask[t];
      ui *= s_mask[t];
    }
    row[m] = ur;
    row[modes + m] = ui;
  }
}

// ---------------------------------------------------------------- chunked scan
// s_t = a_t s_{t-1} + u_t per (row, mode); three passes over chunks of `chunk` steps:
//   local: chunk end state from zero + chunk transition product,
//   carry: sequential combine over chunks,
//   apply: rescan each chunk from its true carry-in (states overwrite u).
// `step_a`: the per-step transitions written by drive_kernel (or NULL: evaluate).
__device__ __forceinline__ void step_coeff(const float *raw_decay, const float *raw_freq,
                                           const float *a_tab_re, const float *a_tab_im,
                                           const float *dt, const float *step_a, int modes,
                                           int64_t tok, int m, float &ar, float &ai) {
  if (dt && step_a) {
    ar = step_a[tok * 2 * modes + m];
    ai = step_a[tok * 2 * modes + modes + m];
  } else if (dt) {
    double damping, frequency;
    mode_pole(raw_decay[m], raw_freq[m], damping, frequency);
    Zoh z = zoh_eval_f32((float)damping, (float)frequency, dt[tok]);
    ar = z.a_re;
    ai = z.a_im;
  } else {
    ar = a_tab_re[m];
    ai = a_tab_im[m];
  }
}

// Loads (transitions and inputs) of `n` <= kScanGroup consecutive steps from
// token `tok0` for mode m, all issued before the caller's dependent steps.
constexpr int kScanGroup = 8;
__device__ __forceinline__ void scan_group_load(const float *raw_decay, const float *raw_freq,
                                                const float *a_tab_re, const float *a_tab_im,
                                                const float *dt, const float *step_a,
                                                const float *u, int modes, int64_t tok0, int n,
                                                int m, float *ar, float *ai, float *xr,
                                                float *xi) {
#pragma unroll
  for (int k = 0; k < kScanGroup; ++k) {
    if (k < n) {
      step_coeff(raw_decay, raw_freq, a_tab_re, a_tab_im, dt, step_a, modes, tok0 + k, m, ar[k],
                 ai[k]);
      const float *row = u + (tok0 + k) * 2 * modes;
      xr[k] = row[m];
      xi[k] = row[modes + m];
    } else {
      ar[k] = ai[k] = xr[k] = xi[k] = 0.f;
    }
  }
}

// Per-chunk scan records [B, nchunk, kRecFloats, M]: E re/im (the chunk's map
// s -> P s + E; the carry pass rewrites E with the chunk's carry-in), P re/im,
// then the last four zero-start ("local") states of the chunk, re/im each, in
// step order (slots 4..11).
constexpr int kRecFloats = 12;
__global__ void scan_local_kernel(const float *__restrict__ u, const float *__restrict__ raw_decay,
                                  const float *__restrict__ raw_freq,
                                  const float *__restrict__ a_re_tab,
                                  const float *__restrict__ a_im_tab,
                                  const float *__restrict__ dt, const float *__restrict__ step_a,
                                  float *__restrict__ carries, int64_t steps, int modes, int chunk,
                                  int64_t n_chunks) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * chunk;
  const int64_t t1 = min(steps, t0 + chunk);
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    float sr = 0.f, si = 0.f, pr = 1.f, pi = 0.f;
    float *rec = carries + (b * n_chunks + c) * kRecFloats * modes;
    const int64_t t_tail = max(t0, t1 - 4);
    auto step = [&](int64_t t) {
      int64_t tok = b * steps + t;
      float ar, ai;
      step_coeff(raw_decay, raw_freq, a_re_tab, a_im_tab, dt, step_a, modes, tok, m, ar, ai);
      const float *row = u + tok * 2 * modes;
      float nr = ar * sr - ai * si + row[m];
      float ni = ai * sr + ar * si + row[modes + m];
      sr = nr;
      si = ni;
      float qr = ar * pr - ai * pi;
      float qi = ai * pr + ar * pi;
      pr = qr;
      pi = qi;
    };
    for (int64_t t = t0; t < t_tail; ++t) step(t);
    for (int64_t t = t_tail; t < t1; ++t) {  // local tail states (slot 0 = fourth-to-last step)
      step(t);
      const int slot = (int)(t - (t1 - 4));
      rec[(4 + 2 * slot) * modes + m] = sr;
      rec[(5 + 2 * slot) * modes + m] = si;
    }
    rec[m] = sr;
    rec[modes + m] = si;
    rec[2 * modes + m] = pr;
    rec[3 * modes + m] = pi;
  }
}

// Carry pass over the per-chunk records (kRecFloats; chunk c maps its entry
// state s to P s + E): rewrites E with the carry-in of each chunk.  `init` (optional, [B, 2M] re | im): the state before step 0 (a
// time slice's carry-in); zero when NULL.
//
// Block (32 modes, kCarryParts ranges of chunks), grid (mode groups, rows).
// Three phases instead of one serial pass over all chunks: each thread composes
// the maps of its range; one thread per mode chains the kCarryParts composed
// maps; each thread re-walks its range from its carry-in.  The chain length
// drops from nchunk to 2 nchunk / kCarryParts + kCarryParts dependent steps.
constexpr int kCarryParts = 32;
__global__ void __launch_bounds__(32 * kCarryParts) scan_carry_kernel(
    float *__restrict__ carries, int64_t batch, int modes, int64_t n_chunks,
    const float *__restrict__ init) {
  __shared__ float sm[4][kCarryParts][33];
  const int lane = threadIdx.x & 31, part = threadIdx.x >> 5;
  const int m = blockIdx.x * 32 + lane;
  const int64_t b = blockIdx.y;
  const bool on = m < modes;
  const int64_t per = (n_chunks + kCarryParts - 1) / kCarryParts;
  const int64_t c0 = min(n_chunks, part * per), c1 = min(n_chunks, c0 + per);
  float *base = carries + b * n_chunks * kRecFloats * modes;
  float Pr = 1.f, Pi = 0.f, Er = 0.f, Ei = 0.f;
  if (on) {
    for (int64_t c = c0; c < c1; ++c) {
      const float *rec = base + c * kRecFloats * modes;
      const float er = rec[m], ei = rec[modes + m], pr = rec[2 * modes + m],
                  pi = rec[3 * modes + m];
      const float nPr = pr * Pr - pi * Pi, nPi = pi * Pr + pr * Pi;
      const float nEr = pr * Er - pi * Ei + er, nEi = pi * Er + pr * Ei + ei;
      Pr = nPr; Pi = nPi; Er = nEr; Ei = nEi;
    }
  }
  sm[0][part][lane] = Pr;
  sm[1][part][lane] = Pi;
  sm[2][part][lane] = Er;
  sm[3][part][lane] = Ei;
  __syncthreads();
  if (part == 0 && on) {
    float sr = init ? init[b * 2 * modes + m] : 0.f;
    float si = init ? init[b * 2 * modes + modes + m] : 0.f;
    for (int k = 0; k < kCarryParts; ++k) {
      const float pr = sm[0][k][lane], pi = sm[1][k][lane], er = sm[2][k][lane],
                  ei = sm[3][k][lane];
      sm[2][k][lane] = sr;  // carry-in of range k
      sm[3][k][lane] = si;
      const float nr = pr * sr - pi * si + er, ni = pi * sr + pr * si + ei;
      sr = nr;
      si = ni;
    }
  }
  __syncthreads();
  if (!on) return;
  float sr = sm[2][part][lane], si = sm[3][part][lane];
  for (int64_t c = c0; c < c1; ++c) {
    float *rec = base + c * kRecFloats * modes;
    const float er = rec[m], ei = rec[modes + m], pr = rec[2 * modes + m],
                pi = rec[3 * modes + m];
    rec[m] = sr;  // carry-in of chunk c
    rec[modes + m] = si;
    const float nr = pr * sr - pi * si + er, ni = pi * sr + pr * si + ei;
    sr = nr;
    si = ni;
  }
}

__global__ void scan_apply_kernel(float *__restrict__ u, const float *__restrict__ raw_decay,
                                  const float *__restrict__ raw_freq,
                                  const float *__restrict__ a_re_tab,
                                  const float *__restrict__ a_im_tab,
                                  const float *__restrict__ dt, const float *__restrict__ step_a,
                                  const float *__restrict__ carries, int64_t steps, int modes,
                                  int chunk, int64_t n_chunks) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * chunk;
  const int64_t t1 = min(steps, t0 + chunk);
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    const float *rec = carries + (b * n_chunks + c) * kRecFloats * modes;
    float sr = rec[m], si = rec[modes + m];
    for (int64_t tg = t0; tg < t1; tg += kScanGroup) {
      float ar[kScanGroup], ai[kScanGroup], xr[kScanGroup], xi[kScanGroup];
      scan_group_load(raw_decay, raw_freq, a_re_tab, a_im_tab, dt, step_a, u, modes,
                      b * steps + tg, (int)(t1 - tg < kScanGroup ? t1 - tg : kScanGroup), m, ar, ai, xr, xi);
#pragma unroll
      for (int k = 0; k < kScanGroup; ++k) {
        if (tg + k < t1) {
          const float nr = ar[k] * sr - ai[k] * si + xr[k];
          const float ni = ai[k] * sr + ar[k] * si + xi[k];
          sr = nr;
          si = ni;
          float *row = u + (b * steps + tg + k) * 2 * modes;
          row[m] = sr;
          row[modes + m] = si;
        }
      }
    }
  }
}

// ---------------------------------------------------------------- unit-grid moments
// Partial sums over a chunk of steps of E, C1, C2, C4 (re, im), optionally
// valid-weighted (_modal_moments / _masked_modal_moments,
// src/lnet/pac_tight_frame_models.py:1632-1702).  partial layout [B, nchunk, 7M].
// `hist` (optional, [B, 4, 2M]): the states at steps -1 .. -4 of a time slice,
// so lag products across the slice start are counted; without it they are
// skipped (sequence start).
__global__ void moments_partial_kernel(const float *__restrict__ s,
                                       const float *__restrict__ valid,
                                       float *__restrict__ partial, int64_t steps, int modes,
                                       int chunk, int64_t n_chunks,
                                       const float *__restrict__ hist) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * chunk;
  const int64_t t1 = min(steps, t0 + chunk);
  const int lags[3] = {1, 2, 4};
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    float acc[7] = {0, 0, 0, 0, 0, 0, 0};
    for (int64_t t = t0; t < t1; ++t) {
      int64_t tok = b * steps + t;
      const float *row = s + tok * 2 * modes;
      float cr = row[m], ci = row[modes + m];
      float wt = valid ? valid[tok] : 1.f;
      acc[0] += (cr * cr + ci * ci) * wt;
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const float *prow;
        if (t >= lags[l]) {
          prow = row - (int64_t)lags[l] * 2 * modes;
        } else if (hist) {
          prow = hist + (b * 4 + (lags[l] - t - 1)) * 2 * modes;
        } else {
          continue;
        }
        float pr = prow[m], pi = prow[modes + m];
        float w = valid ? wt * valid[tok - lags[l]] : 1.f;
        acc[1 + 2 * l] += (cr * pr + ci * pi) * w;
        acc[2 + 2 * l] += (ci * pr - cr * pi) * w;
      }
    }
    float *out = partial + (b * n_chunks + c) * 7 * modes;
#pragma unroll
    for (int j = 0; j < 7; ++j) out[j * modes + m] = acc[j];
  }
}

// Raw (unnormalised) moment sums of each row, the chunk partials added in
// order in double: sums [B, 7M] (time-split ranks all-reduce these).
__global__ void moment_sums_kernel(const float *__restrict__ partial, double *__restrict__ sums,
                                   int64_t batch, int modes, int64_t n_chunks) {
  const int64_t n = batch * 7 * modes;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / (7 * modes);
    const int j = (int)(i - b * 7 * modes);
    double acc = 0.0;
    for (int64_t c = 0; c < n_chunks; ++c) acc += (double)partial[(b * n_chunks + c) * 7 * modes + j];
    sums[i] = acc;
  }
}

// Scan apply pass with the moments accumulated on the fly (static poles): per
// (chunk, row) block, each thread walks one mode through the chunk from its
// carry-in, optionally writes the states in place over u (WRITE_STATES; the
// writer's synthesis GEMM reads them, the reader needs moments only), and sums
// E and the lag-1/2/4 products (valid-weighted when `valid`), holding the last
// four states in registers.  A chunk c > 0 starts that history from the true
// states of the previous chunk's last four steps, rebuilt from its record:
// local tail state + a^(L - k) x its carry-in (L = chunk, every chunk but the
// last is full), so the pairs straddling the chunk start are counted here.
// u is read eight steps ahead of the recurrence.  partial layout [B, nchunk,
// 7M]; products as in moments_partial_kernel.
template <bool WRITE_STATES>
__global__ void scan_apply_moments_kernel(float *__restrict__ u, const float *__restrict__ a_re_tab,
                                          const float *__restrict__ a_im_tab,
                                          const float *__restrict__ carries,
                                          const float *__restrict__ valid,
                                          float *__restrict__ partial, int64_t steps, int modes,
                                          int chunk, int64_t n_chunks) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * chunk;
  const int len = (int)min((int64_t)chunk, steps - t0);
  const int64_t M2 = 2 * modes;
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    const float ar = a_re_tab[m], ai = a_im_tab[m];
    const float *rec = carries + (b * n_chunks + c) * kRecFloats * modes;
    float sr = rec[m], si = rec[modes + m];
    // h0 = state at t - 1, h1 at t - 2, h2 at t - 3, h3 at t - 4
    float hr0 = 0.f, hi0 = 0.f, hr1 = 0.f, hi1 = 0.f, hr2 = 0.f, hi2 = 0.f, hr3 = 0.f, hi3 = 0.f;
    if (c > 0) {
      const float *prv = carries + (b * n_chunks + c - 1) * kRecFloats * modes;
      const float cr = prv[m], ci = prv[modes + m];  // carry-in of chunk c - 1
      float pr = 1.f, pi = 0.f;                       // a^j, j = 1 .. chunk
      for (int j = 1; j <= chunk - 4; ++j) {
        const float qr = ar * pr - ai * pi, qi = ai * pr + ar * pi;
        pr = qr;
        pi = qi;
      }
      float tr[4], ti[4];
#pragma unroll
      for (int slot = 0; slot < 4; ++slot) {  // local step chunk - 4 + slot: a^(chunk - 3 + slot)
        const float qr = ar * pr - ai * pi, qi = ai * pr + ar * pi;
        pr = qr;
        pi = qi;
        const float lr = prv[(4 + 2 * slot) * modes + m], li = prv[(5 + 2 * slot) * modes + m];
        tr[slot] = lr + (pr * cr - pi * ci);
        ti[slot] = li + (pi * cr + pr * ci);
      }
      hr0 = tr[3]; hi0 = ti[3]; hr1 = tr[2]; hi1 = ti[2];
      hr2 = tr[1]; hi2 = ti[1]; hr3 = tr[0]; hi3 = ti[0];
    }
    float e0 = 0.f, c1r = 0.f, c1i = 0.f, c2r = 0.f, c2i = 0.f, c4r = 0.f, c4i = 0.f;
    float *row = u + (b * steps + t0) * M2;
    const float *vrow = valid ? valid + b * steps + t0 : nullptr;
    const int reach = c > 0 ? 4 : 0;  // history steps available before the chunk
    for (int i0 = 0; i0 < len; i0 += 8) {
      float ur[8], ui[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        ur[k] = i0 + k < len ? row[(i0 + k) * M2 + m] : 0.f;
        ui[k] = i0 + k < len ? row[(i0 + k) * M2 + modes + m] : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k;
        if (i >= len) break;
        const float nr = ar * sr - ai * si + ur[k];
        const float ni = ai * sr + ar * si + ui[k];
        sr = nr;
        si = ni;
        if (WRITE_STATES) {
          row[i * M2 + m] = sr;
          row[i * M2 + modes + m] = si;
        }
        const float wt = vrow ? vrow[i] : 1.f;
        e0 += (sr * sr + si * si) * wt;
        if (i + reach >= 1) {
          const float w = vrow ? wt * vrow[i - 1] : 1.f;
          c1r += (sr * hr0 + si * hi0) * w;
          c1i += (si * hr0 - sr * hi0) * w;
        }
        if (i + reach >= 2) {
          const float w = vrow ? wt * vrow[i - 2] : 1.f;
          c2r += (sr * hr1 + si * hi1) * w;
          c2i += (si * hr1 - sr * hi1) * w;
        }
        if (i + reach >= 4) {
          const float w = vrow ? wt * vrow[i - 4] : 1.f;
          c4r += (sr * hr3 + si * hi3) * w;
          c4i += (si * hr3 - sr * hi3) * w;
        }
        hr3 = hr2; hi3 = hi2; hr2 = hr1; hi2 = hi1; hr1 = hr0; hi1 = hi0; hr0 = sr; hi0 = si;
      }
    }
    float *out = partial + (b * n_chunks + c) * 7 * modes;
    out[m] = e0;
    out[modes + m] = c1r;
    out[2 * modes + m] = c1i;
    out[3 * modes + m] = c2r;
    out[4 * modes + m] = c2i;
    out[5 * modes + m] = c4r;
    out[6 * modes + m] = c4i;
  }
}

// Normalised moments [B, 7M] from the chunk partials;
// valid counts clamped at one (_masked_modal_moments, sum(...).clamp_min(1.0)),
// else divided by the pair count.  Grid (ceil(7M / 32), B); block = 32 features
// x kFinalParts chunk ranges summed in double, combined in range order.
constexpr int kFinalParts = 32;
__global__ void __launch_bounds__(32 * kFinalParts) moments_finalize_kernel(
    const float *__restrict__ partial, const float *__restrict__ valid,
    float *__restrict__ moments, int64_t steps, int modes, int64_t n_chunks) {
  const int64_t b = blockIdx.y;
  const int lane = threadIdx.x & 31, part = threadIdx.x >> 5;
  __shared__ double s_cnt[4];
  __shared__ double red[kFinalParts][33];
  const int lags[3] = {1, 2, 4};
  if (valid) {
    double cnt[4] = {0, 0, 0, 0};
    for (int64_t t = threadIdx.x; t < steps; t += blockDim.x) {
      const double v = valid[b * steps + t];
      cnt[0] += v;
      for (int l = 0; l < 3; ++l)
        if (t >= lags[l]) cnt[1 + l] += v * (double)valid[b * steps + t - lags[l]];
    }
    for (int k = 0; k < 4; ++k) {
      double v = cnt[k];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[part][k] = v;
    }
    __syncthreads();
    if (threadIdx.x < 4) {
      double v = 0;
      for (int w = 0; w < kFinalParts; ++w) v += red[w][threadIdx.x];
      s_cnt[threadIdx.x] = v;
    }
    __syncthreads();
  }
  const int j = blockIdx.x * 32 + lane;
  const bool on = j < 7 * modes;
  const int64_t per = (n_chunks + kFinalParts - 1) / kFinalParts;
  const int64_t c0 = min(n_chunks, part * per), c1 = min(n_chunks, c0 + per);
  double acc = 0.0;
  if (on)
    for (int64_t c = c0; c < c1; ++c) acc += (double)partial[(b * n_chunks + c) * 7 * modes + j];
  __syncthreads();
  red[part][lane] = acc;
  __syncthreads();
  if (part != 0 || !on) return;
  double total = 0.0;
  for (int w = 0; w < kFinalParts; ++w) total += red[w][lane];
  const int kind = j / modes;  // 0 = E, 1..6 = lag pairs (re, im)
  const int lag_idx = kind == 0 ? -1 : (kind - 1) / 2;
  float outv;
  if (lag_idx >= 0 && steps <= lags[lag_idx]) {
    outv = 0.f;
  } else if (valid) {
    const float cntf = (float)s_cnt[lag_idx + 1];
    outv = (float)total / fmaxf(cntf, 1.0f);
  } else {
    const int64_t n = lag_idx < 0 ? steps : steps - lags[lag_idx];
    outv = (float)(total / (double)n);
  }
  moments[b * 7 * modes + j] = outv;
}

// Gains folded into the drive frame (static poles, no event mask):
// out[:, m] = g_re W_re - g_im W_im, out[:, M + m] = g_re W_im + g_im W_re, so
// the drive GEMM yields u = g (x^ W) directly (frame [D, 2M] row-major).
// `out_bf16` (optional): the same frame rounded to bf16, for a bf16 drive GEMM.
__global__ void fold_gain_kernel(const float *__restrict__ frame, const float *__restrict__ g_re,
                                 const float *__restrict__ g_im, float *__restrict__ out,
                                 __nv_bfloat16 *__restrict__ out_bf16, int dim, int modes) {
  const int64_t n = (int64_t)dim * modes;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = i / modes;
    const int m = (int)(i - d * modes);
    const float *w = frame + d * 2 * modes;
    const float wr = w[m], wi = w[modes + m];
    const float fr = g_re[m] * wr - g_im[m] * wi, fi = g_re[m] * wi + g_im[m] * wr;
    out[d * 2 * modes + m] = fr;
    out[d * 2 * modes + modes + m] = fi;
    if (out_bf16) {
      out_bf16[d * 2 * modes + m] = __float2bfloat16_rn(fr);
      out_bf16[d * 2 * modes + modes + m] = __float2bfloat16_rn(fi);
    }
  }
}

// ---------------------------------------------------------------- physical-time moments
// Restates _physical_time_modal_moments / _interpolate_modal_state
// (src/lnet/pac_tight_frame_models.py:1705-1833).  Per chunk of steps:
// sample positions of the three lag queries are computed once per token,
// then every mode accumulates.  partial layout per (b, chunk):
// [8 * M mode sums (E_duration, E_event, C1r, C1i, C2r, C2i, C4r, C4i)] + [5 scalars:
//  sum(dt*valid), sum(valid), pair weights of lags 1, 2, 4].
constexpr int kPtChunk = 64;
constexpr int kPtRedFloats = 8 * 256;  // step-group partial sums (256 threads)
__global__ void pt_moments_partial_kernel(const float *__restrict__ s,
                                          const float *__restrict__ ts,
                                          const float *__restrict__ dt,
                                          const float *__restrict__ valid,
                                          float *__restrict__ partial, int64_t steps,
                                          int modes, int64_t n_chunks) {
  __shared__ int64_t s_lo[3][kPtChunk], s_hi[3][kPtChunk];
  __shared__ float s_ip[3][kPtChunk], s_pw[3][kPtChunk];
  __shared__ float s_dw[kPtChunk], s_v[kPtChunk];
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * kPtChunk;
  const int n = (int)min((int64_t)kPtChunk, steps - t0);
  const float *row = ts + b * steps;
  const int rec = 8 * modes + 5;
  for (int j = threadIdx.x; j < n * 3; j += blockDim.x) {
    int i = j / 3, l = j - (j / 3) * 3;
    int lag = l == 0 ? 1 : (l == 1 ? 2 : 4);
    int64_t t = t0 + i;
    int64_t tok = b * steps + t;
    float q = row[t] - (float)lag;
    int64_t up_u = lower_bound_f(row, steps, q);
    int64_t up = up_u < steps - 1 ? up_u : steps - 1;
    int64_t lo = up_u - 1;
    lo = lo < 0 ? 0 : (lo > steps - 1 ? steps - 1 : lo);
    float lt = row[lo], ut = row[up];
    float span = ut - lt;
    float ip = span > 0.f ? (q - lt) / fmaxf(span, kFp32Tiny) : 0.f;
    ip = fminf(fmaxf(ip, 0.f), 1.f);
    float lv = valid ? valid[b * steps + lo] : 1.f;
    float uv = valid ? valid[b * steps + up] : 1.f;
    const float eps8 = 8.0f * kFp32Eps;
    float support = ip <= eps8 ? lv : (ip >= 1.0f - eps8 ? uv : lv * uv);
    bool in_bounds = (q >= row[0]) && (q <= row[steps - 1]);
    support = support * (in_bounds ? 1.f : 0.f);
    float vt = valid ? valid[tok] : 1.f;
    s_lo[l][i] = b * steps + lo;
    s_hi[l][i] = b * steps + up;
    s_ip[l][i] = ip;
    s_pw[l][i] = dt[tok] * vt * support;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int64_t tok = b * steps + t0 + i;
    float vt = valid ? valid[tok] : 1.f;
    s_dw[i] = dt[tok] * vt;
    s_v[i] = vt;
  }
  __syncthreads();
  float *out = partial + (b * n_chunks + c) * rec;
  // threads = (step group g, mode m): with modes <= blockDim / 2 the chunk's steps
  // are split over `groups` interleaved groups whose sums meet in shared memory
  __shared__ float s_red[kPtRedFloats];
  const int groups = modes * 2 <= (int)blockDim.x && 8 * (int)blockDim.x <= kPtRedFloats
                         ? (int)blockDim.x / modes : 1;
  const int g = groups > 1 ? (int)threadIdx.x / modes : 0;
  const int m0 = groups > 1 ? (int)threadIdx.x - g * modes : (int)threadIdx.x;
  const int m_step = groups > 1 ? modes : (int)blockDim.x;
  for (int m = m0; m < modes && g < groups; m += m_step) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = g; i < n; i += groups) {
      int64_t tok = b * steps + t0 + i;
      const float *cur = s + tok * 2 * modes;
      float cr = cur[m], ci = cur[modes + m];
      float e = cr * cr + ci * ci;
      acc[0] += e * s_dw[i];
      acc[1] += e * s_v[i];
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const float *lo = s + s_lo[l][i] * 2 * modes;
        const float *hi = s + s_hi[l][i] * 2 * modes;
        float pr = lerp_torch(lo[m], hi[m], s_ip[l][i]);
        float pi = lerp_torch(lo[modes + m], hi[modes + m], s_ip[l][i]);
        float w = s_pw[l][i];
        acc[2 + 2 * l] += (cr * pr + ci * pi) * w;
        acc[3 + 2 * l] += (ci * pr - cr * pi) * w;
      }
    }
    if (groups > 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) s_red[(g * 8 + j) * modes + m] = acc[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j * modes + m] = acc[j];
    }
  }
  if (groups > 1) {
    __syncthreads();
    for (int e = threadIdx.x; e < 8 * modes; e += blockDim.x) {
      float v = 0.f;
      for (int q = 0; q < groups; ++q) v += s_red[q * 8 * modes + e];
      out[e] = v;
    }
  }
  if (threadIdx.x < 5) {
    float acc = 0.f;
    for (int i = 0; i < n; ++i) {
      if (threadIdx.x == 0) acc += s_dw[i];
      else if (threadIdx.x == 1) acc += s_v[i];
      else acc += s_pw[threadIdx.x - 2][i];
    }
    out[8 * modes + threadIdx.x] = acc;
  }
}

// Grid (ceil(M / 32), B); block = 32 modes x kPtFinalParts chunk ranges summed
// in double and combined in range order (the five per-row scalars likewise).
constexpr int kPtFinalParts = 8;
__global__ void __launch_bounds__(32 * kPtFinalParts) pt_moments_finalize_kernel(
    const float *__restrict__ partial, float *__restrict__ moments, int modes, int64_t n_chunks) {
  const int64_t b = blockIdx.y;
  const int lane = threadIdx.x & 31, part = threadIdx.x >> 5;
  const int m = blockIdx.x * 32 + lane;
  const int rec = 8 * modes + 5;
  __shared__ double red[kPtFinalParts][8][33];
  __shared__ double sc_part[kPtFinalParts][5];
  __shared__ double sc[5];
  const int64_t per = (n_chunks + kPtFinalParts - 1) / kPtFinalParts;
  const int64_t c0 = min(n_chunks, part * per), c1 = min(n_chunks, c0 + per);
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  double sa = 0.0;
  for (int64_t c = c0; c < c1; ++c) {
    const float *p = partial + (b * n_chunks + c) * rec;
    if (m < modes) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += (double)p[j * modes + m];
    }
    if (lane < 5) sa += (double)p[8 * modes + lane];
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[part][j][lane] = acc[j];
  if (lane < 5) sc_part[part][lane] = sa;
  __syncthreads();
  if (threadIdx.x < 5) {
    double a = 0.0;
    for (int w = 0; w < kPtFinalParts; ++w) a += sc_part[w][threadIdx.x];
    sc[threadIdx.x] = a;
  }
  __syncthreads();
  if (part != 0 || m >= modes) return;
  double tot[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    double a = 0.0;
    for (int w = 0; w < kPtFinalParts; ++w) a += red[w][j][lane];
    tot[j] = a;
  }
  const bool use_duration = sc[0] > 0.0;
  float *o = moments + b * 7 * modes;
  const float ecount = fmaxf((float)(use_duration ? sc[0] : sc[1]), 1.0f);
  o[m] = (float)(use_duration ? tot[0] : tot[1]) / ecount;
  for (int l = 0; l < 3; ++l) {
    const float pc = fmaxf((float)sc[2 + l], 1.0f);
    o[(1 + 2 * l) * modes + m] = (float)tot[2 + 2 * l] / pc;
    o[(2 + 2 * l) * modes + m] = (float)tot[3 + 2 * l] / pc;
  }
}

// ---------------------------------------------------------------- writer residual
// v = x + ls * (modal + ds * xhat)
__global__ void residual_kernel(const float *__restrict__ x, const float *__restrict__ xhat,
                                const float *__restrict__ modal, const float *__restrict__ ds,
                                const float *__restrict__ ls, float *__restrict__ v,
                                int64_t tokens, int dim) {
  for (int64_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
      const int64_t i = tok * dim + d;
      v[i] = x[i] + ls[d] * (modal[i] + ds[d] * xhat[i]);
    }
  }
}

// ---------------------------------------------------------------- head features
// Radial-log feature j of one row's moments (src/lnet/alphabet.py:29-46); the
// affine head itself is head_gemm.cuh.
__device__ __forceinline__ float radial_feature(const float *mom, int modes, int j) {
  if (j < modes) return log1pf(fmaxf(mom[j], 0.f));
  int pair = (j - modes) / (2 * modes);
  int within = (j - modes) - pair * 2 * modes;
  int base = modes + pair * 2 * modes;
  int mm = within % modes;
  float re = mom[base + mm], im = mom[base + modes + mm];
  float r = sqrtf(fmaxf(re * re + im * im, kFp32Tiny));
  float scale = log1pf(r) / r;
  return scale * (within < modes ? re : im);
}

__global__ void head_features_kernel(const float *__restrict__ wm, const float *__restrict__ rm,
                                     float *__restrict__ feats, int64_t batch, int modes) {
  int64_t n = batch * 14 * modes;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = i / (14 * modes);
    int j = (int)(i - b * 14 * modes);
    const float *src = j < 7 * modes ? wm + b * 7 * modes : rm + b * 7 * modes;
    feats[i] = radial_feature(src, modes, j < 7 * modes ? j : j - 7 * modes);
  }
}


// ---------------------------------------------------------------- ZOH table
__global__ void zoh_kernel(const float *__restrict__ raw_decay, const float *__restrict__ raw_freq,
                           int modes, const float *__restrict__ dt, int64_t steps,
                           float *__restrict__ a_re, float *__restrict__ a_im,
                           float *__restrict__ g_re, float *__restrict__ g_im) {
  int64_t rows = dt ? steps : 1;
  int64_t n = rows * modes;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / modes;
    int m = (int)(i - r * modes);
    double damping, frequency;
    mode_pole(raw_decay[m], raw_freq[m], damping, frequency);
    Zoh z = zoh_eval(damping, frequency, dt ? (double)dt[r] : 1.0);
    a_re[i] = z.a_re;
    a_im[i] = z.a_im;
    if (g_re) g_re[i] = z.g_re;
    if (g_im) g_im[i] = z.g_im;
  }
}

}  // namespace lnet
