// Training path of the general route: a forward that keeps its activations
// and the backward pass (VJP) of every stage, for every metadata combination
// (time_delta, observation and valid masks), all in fp32.
//
// Forward (lnet_b200_alphabet_train_forward): the general-route stages with
// separate buffers per block, full-fp32 GEMMs.  Kept in the workspace:
// stem input x32 [BT, C], proj / y1 / xhat1 / modal / v / y2 / xhat2 [BT, D],
// writer and reader states s1 / s2 [BT, 2M], moments, features, per-mode
// a / g tables.
//
// Backward (lnet_b200_alphabet_backward), the adjoint of each stage in reverse
// order (the same restatement as the numpy backward oracle):
//   head GEMMs -> radial-log VJP -> moments VJP (per-step state gradient)
//   -> reverse chunked scan lambda_t = dS_t + conj(a) lambda_{t+1}, with the
//      drive gradient de = conj(g) lambda and the per-mode sums for da, dg
//   -> pole chain rule (ZOH a = exp(p), g = (a - 1) / p, p = -damping + i freq)
//   -> drive GEMMs (dxhat = de F^T, dF += xhat^T de) -> RMSNorm VJP
//   -> conv + SiLU VJP (recomputing the pre-activation) -> ...
// The writer's synthesis + residual adds ls (dv F) to its state gradient and
// ls (dv^T s1) to its frame gradient.  Every reduction over tokens is
// deterministic: per-part partial sums then an ordered final sum in double.
#pragma once

namespace lnet {

// ---------------------------------------------------------------- plan
struct TrainPlan {
  float *x32, *proj, *y1, *xh1, *s1, *modal, *v, *y2, *xh2, *s2;
  float *m1, *m2, *feats, *a_tab;  // a_tab: [8][M] as in the general route
  // scratch
  float *carries, *partial, *wfold, *head_partial, *ts, *ptcounts;
  float *dS, *dX, *dY, *dV, *rs, *dfeats, *dm, *counts, *colpart, *polepart, *polesum, *wls;
};

constexpr int kColParts = 148 * 8;  // row parts of a column reduction (at most)
constexpr int kBwdTile = 16;        // steps per block of the token-wise backward kernels
constexpr int kWgTile = 128;        // steps per block of the conv weight-gradient partials
constexpr int kMbTile = 64;         // steps per block of the moments VJP
constexpr int kCbTile = 32;         // steps per block of the fused conv VJP

static void plan_train(Arena &ar, TrainPlan &tp, const lnet_b200_alphabet_params *p,
                       const lnet_b200_alphabet_request *r) {
  const int64_t B = r->batch, bt = B * r->steps;
  const int C = p->raw_input_dim, D = p->model_dim, M = p->modes, K = p->output_dim;
  const int64_t n_scan = cdiv(std::max<int64_t>(r->steps, 1), kScanChunk);
  auto f = [&](size_t n) { return ar.take<float>(n); };
  tp.x32 = f((size_t)bt * C);
  tp.proj = f((size_t)bt * D);
  tp.y1 = f((size_t)bt * D);
  tp.xh1 = f((size_t)bt * D);
  tp.s1 = f((size_t)bt * 2 * M);
  tp.modal = f((size_t)bt * D);
  tp.v = f((size_t)bt * D);
  tp.y2 = f((size_t)bt * D);
  tp.xh2 = f((size_t)bt * D);
  tp.s2 = f((size_t)bt * 2 * M);
  tp.m1 = f((size_t)B * 7 * M);
  tp.m2 = f((size_t)B * 7 * M);
  tp.feats = f((size_t)B * 14 * M);
  tp.a_tab = f((size_t)8 * M);
  tp.carries = f((size_t)B * n_scan * kRecFloats * M);
  tp.partial = f((size_t)B * n_scan * (8 * M + 5));  // physical-time partials are widest
  tp.ts = f((size_t)bt);
  tp.ptcounts = f((size_t)B * 8);
  tp.wfold = f((size_t)D * 2 * M);
  tp.head_partial = f(head_partial_floats(B, K));
  tp.dS = f((size_t)bt * 2 * M);
  tp.dX = f((size_t)bt * D);
  tp.dY = f((size_t)bt * D);
  tp.dV = f((size_t)bt * D);
  tp.rs = f((size_t)bt);
  tp.dfeats = f((size_t)B * 14 * M);
  tp.dm = f((size_t)2 * B * 7 * M);
  tp.counts = f((size_t)B * 4);
  const int64_t wg_parts = B * cdiv(std::max<int64_t>(r->steps, 1), kCbTile);
  // widest column reduction: 4M pole sums, D * taps conv weights (generic
  // kernels), 14M / K / C / D otherwise; or the fused conv VJP's partials
  const int64_t widest = std::max<int64_t>({(int64_t)D * (p->conv_kernel + 1), 14 * M, 4 * M, C, K});
  tp.colpart = f((size_t)std::max<int64_t>((int64_t)kColParts * widest,
                                           wg_parts * D * (p->conv_kernel + 1)));
  tp.polepart = f((size_t)B * n_scan * 4 * M);
  tp.polesum = f((size_t)std::max(4 * M, D * (p->conv_kernel + 1)));
  tp.wls = f((size_t)D * 2 * M);
}

static bool train_supported(const lnet_b200_alphabet_request *) { return true; }

// A Plan view of the training buffers for block_scan_moments.
static Plan block_view(const TrainPlan &tp, float *xhat, float *states) {
  Plan pl;
  pl.ts = tp.ts;
  pl.xhat = xhat;
  pl.drive = states;
  pl.carries = tp.carries;
  pl.partial = tp.partial;
  pl.wfold = tp.wfold;
  return pl;
}

// ---------------------------------------------------------------- forward
template <typename TX>
static int train_forward_impl(const lnet_b200_alphabet_params *p,
                              const lnet_b200_alphabet_request *r, TrainPlan &tp, float *logits,
                              cudaStream_t st) {
  const int64_t B = r->batch, T = r->steps, bt = B * T;
  const int C = p->raw_input_dim, D = p->model_dim, M = p->modes;
  // GEMM precision as in the inference route: exact fp32 for fp32 requests,
  // TF32 tensor cores for bf16 requests
  const bool tf32 = r->act_dtype == LNET_BF16;
  const lnet_b200_alphabet_request rq = *r;
  mask_inputs_kernel<TX><<<token_grid(bt), token_block(C), 0, st>>>(
      (const TX *)r->x, r->observation_mask, r->obs_channels, r->valid_mask, tp.x32, bt, C);
  LNET_TRY(after_launch("mask_inputs_kernel"));
  LNET_TRY(gemm_rows(st, tp.x32, CUDA_R_32F, C, p->stem_projection, CUDA_R_32F, C, 1, tp.proj, D,
                     bt, D, C, tf32, "gemm(stem)"));
  if (r->time_delta) {  // physical-time convs and moments
    LNET_TRY(timestamps(r->time_delta, tp.ts, B, T, st));
    LNET_TRY(physical_conv(tp.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr, tp.ts,
                           r->valid_mask, tp.y1, B, T, D, p->conv_kernel, p->conv_dilation, st,
                           "dwconv_physical(stem)"));
  } else {
    LNET_TRY(depthwise_conv(tp.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr,
                            r->valid_mask, tp.y1, B, T, D, p->conv_kernel, p->conv_dilation, st,
                            "depthwise_conv(stem)"));
  }
  Plan pw = block_view(tp, tp.xh1, tp.s1);
  LNET_TRY(block_scan_moments(tp.y1, p->writer_norm, p->writer_frame, p->writer_raw_decay,
                              p->writer_raw_frequency, tp.a_tab, tp.a_tab + M, tp.a_tab + 4 * M,
                              tp.a_tab + 5 * M, r->observation_mask, r->obs_channels, &rq, D, M,
                              pw, tp.m1, /*write_states=*/true, st));
  LNET_TRY(gemm_rows(st, tp.s1, CUDA_R_32F, 2 * M, p->writer_frame, CUDA_R_32F, 2 * M, 1,
                     tp.modal, D, bt, D, 2 * M, tf32, "gemm(synthesis)"));
  residual_kernel<<<token_grid(bt), token_block(D), 0, st>>>(
      tp.y1, tp.xh1, tp.modal, p->writer_direct_scale, p->writer_layer_scale, tp.v, bt, D);
  LNET_TRY(after_launch("residual_kernel"));
  if (r->time_delta) {
    LNET_TRY(physical_conv(tp.v, p->reader_conv_weight, p->reader_conv_bias, r->valid_mask,
                           tp.ts, r->valid_mask, tp.y2, B, T, D, p->conv_kernel, p->conv_dilation,
                           st, "dwconv_physical(reader)"));
  } else {
    LNET_TRY(depthwise_conv(tp.v, p->reader_conv_weight, p->reader_conv_bias, r->valid_mask,
                            r->valid_mask, tp.y2, B, T, D, p->conv_kernel, p->conv_dilation, st,
                            "depthwise_conv(reader)"));
  }
  Plan pr = block_view(tp, tp.xh2, tp.s2);
  LNET_TRY(block_scan_moments(tp.y2, p->reader_norm, p->reader_frame, p->reader_raw_decay,
                              p->reader_raw_frequency, tp.a_tab + 2 * M, tp.a_tab + 3 * M,
                              tp.a_tab + 6 * M, tp.a_tab + 7 * M, nullptr, 1, &rq, D, M, pr,
                              tp.m2, /*write_states=*/true, st));
  return head_run(p, B, tp.m1, tp.m2, tp.feats, tp.head_partial, logits, st, nullptr);
}

// ---------------------------------------------------------------- backward kernels
// Column sums of value(row, col) over rows: partial[part][col] over a row
// range per part, then colsum_final_kernel adds the parts in order (double).
struct ColPlain {
  const float *a;
  int width;
  __device__ float operator()(int64_t row, int col) const { return a[row * width + col]; }
};
struct ColProd {  // a * b (* c[col]) (+ d e[col]) style products of the synthesis scales
  const float *dv, *modal, *xh, *ls, *ds;
  int width, which;  // 0: dv (modal + ds xh), 1: dv ls xh
  __device__ float operator()(int64_t row, int col) const {
    const int64_t i = row * width + col;
    return which == 0 ? dv[i] * (modal[i] + ds[col] * xh[i]) : dv[i] * ls[col] * xh[i];
  }
};
struct ColRmsGamma {  // dxhat * y * rs
  const float *dxh, *y, *rs;
  int width;
  __device__ float operator()(int64_t row, int col) const {
    const int64_t i = row * width + col;
    return dxh[i] * y[i] * rs[row];
  }
};
struct ColConvW {  // dz[t, d] * xin[t + k dil - pad, d] (masked input), col = d * taps + k
  const float *dz, *xin, *in_mask;
  int64_t steps;
  int dim, taps, dil;
  __device__ float operator()(int64_t row, int col) const {
    const int d = col / taps, k = col - (col / taps) * taps;
    const int64_t b = row / steps, t = row - b * steps;
    const int64_t s = t + (int64_t)k * dil - (int64_t)dil * (taps - 1) / 2;
    if (s < 0 || s >= steps) return 0.f;
    float x = xin[(b * steps + s) * dim + d];
    if (in_mask) x *= in_mask[b * steps + s];
    return dz[row * dim + d] * x;
  }
};

// Block = 32 columns x 8 row lanes; each lane sums every 8th row of its part,
// then the 8 lanes are added in order through shared memory.
template <typename F>
__global__ void __launch_bounds__(256) colsum_partial_kernel(F f, int64_t rows, int width,
                                                             float *__restrict__ partial) {
  __shared__ float red[8][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  const int lane_row = threadIdx.y;
  const int part = blockIdx.y;
  const int64_t per = (rows + gridDim.y - 1) / gridDim.y;
  const int64_t r0 = min(rows, part * per), r1 = min(rows, r0 + per);
  float a0 = 0.f, a1 = 0.f;
  if (col < width) {
    int64_t row = r0 + lane_row;
    for (; row + 8 < r1; row += 16) {
      a0 += f(row, col);
      a1 += f(row + 8, col);
    }
    if (row < r1) a0 += f(row, col);
  }
  red[lane_row][threadIdx.x] = a0 + a1;
  __syncthreads();
  if (lane_row == 0 && col < width) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += red[k][threadIdx.x];
    partial[(int64_t)part * width + col] = acc;
  }
}

// Block = 32 columns x 32 lanes; lane j sums parts j, j + 32, ... in double,
// the lanes are then added in order.
__global__ void __launch_bounds__(1024) colsum_final_kernel(const float *__restrict__ partial,
                                                            int parts, int width,
                                                            float *__restrict__ out) {
  __shared__ double red[32][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  double acc = 0.0;
  if (col < width)
    for (int q = threadIdx.y; q < parts; q += 32) acc += (double)partial[(int64_t)q * width + col];
  red[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && col < width) {
    double total = 0.0;
    for (int k = 0; k < 32; ++k) total += red[k][threadIdx.x];
    out[col] = (float)total;
  }
}

template <typename F>
static int colsum(F f, int64_t rows, int width, float *partial, float *out, cudaStream_t st,
                  const char *what) {
  const int parts = (int)std::max<int64_t>(1, std::min<int64_t>(kColParts, cdiv(rows, 128)));
  const dim3 grid((unsigned)cdiv(width, 32), (unsigned)parts);
  colsum_partial_kernel<F><<<grid, dim3(32, 8), 0, st>>>(f, rows, width, partial);
  LNET_TRY(after_launch(what));
  colsum_final_kernel<<<(unsigned)cdiv(width, 32), dim3(32, 32), 0, st>>>(partial, parts, width,
                                                                          out);
  return after_launch("colsum_final_kernel");
}

// The same final reduction for partials written by other kernels.
static int colsum_finish(const float *partial, int parts, int width, float *out, cudaStream_t st) {
  colsum_final_kernel<<<(unsigned)cdiv(width, 32), dim3(32, 32), 0, st>>>(partial, parts, width,
                                                                          out);
  return after_launch("colsum_final_kernel");
}

// VJP of radial_feature for both blocks: dm [2][B][7M] from dfeats [B][14M].
__global__ void radial_backward_kernel(const float *__restrict__ m1, const float *__restrict__ m2,
                                       const float *__restrict__ dfeats, float *__restrict__ dm,
                                       int64_t batch, int modes) {
  const int64_t n = 2 * batch * 7 * modes;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t blk = i / (batch * 7 * modes);
    const int64_t rem = i - blk * batch * 7 * modes;
    const int64_t b = rem / (7 * modes);
    const int j = (int)(rem - b * 7 * modes);
    const float *mom = (blk == 0 ? m1 : m2) + b * 7 * modes;
    const float *df = dfeats + b * 14 * modes + blk * 7 * modes;
    float out;
    if (j < modes) {
      const float e = mom[j];
      out = e > 0.f ? df[j] / (1.0f + e) : 0.f;
    } else {
      const int pair = (j - modes) / (2 * modes);
      const int within = (j - modes) - pair * 2 * modes;
      const int base = modes + pair * 2 * modes;
      const int mm = within % modes;
      const float re = mom[base + mm], im = mom[base + modes + mm];
      const float gre = df[base + mm], gim = df[base + modes + mm];
      const float q = re * re + im * im;
      const float r = sqrtf(fmaxf(q, kFp32Tiny));
      const float sc = log1pf(r) / r;
      const float kk = q > kFp32Tiny ? (r / (1.0f + r) - log1pf(r)) / (r * r * r) : 0.f;
      out = within < modes ? gre * (sc + re * re * kk) + gim * (im * re * kk)
                           : gre * (re * im * kk) + gim * (sc + im * im * kk);
    }
    dm[i] = out;
  }
}

// Per-row pair counts for the masked moments: [B][4] = max(sum v, 1) and
// max(sum v_t v_{t-l}, 1) for l = 1, 2, 4 (T and T - l without a mask).
__global__ void moment_counts_kernel(const float *__restrict__ valid, int64_t steps,
                                     float *__restrict__ counts) {
  const int64_t b = blockIdx.x;
  const int lags[3] = {1, 2, 4};
  __shared__ double red[4][32];
  double c[4] = {0, 0, 0, 0};
  for (int64_t t = threadIdx.x; t < steps; t += blockDim.x) {
    const double v = valid[b * steps + t];
    c[0] += v;
    for (int l = 0; l < 3; ++l)
      if (t >= lags[l]) c[1 + l] += v * (double)valid[b * steps + t - lags[l]];
  }
  for (int k = 0; k < 4; ++k) {
    double x = c[k];
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if ((threadIdx.x & 31) == 0) red[k][threadIdx.x >> 5] = x;
  }
  __syncthreads();
  if (threadIdx.x < 4) {
    double x = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) x += red[threadIdx.x][w];
    counts[b * 4 + threadIdx.x] = fmaxf((float)x, 1.0f);
  }
}

// State gradient of the (masked) moments, one thread per (token, mode):
// dS_t += 2 s_t dE w_t / c0 + sum_l [pairs with t as the current state and as
// the earlier one] (w = v_t v_{t-l}).  `accumulate`: add to dS.
__global__ void moments_backward_kernel(const float *__restrict__ s, const float *__restrict__ dm,
                                        const float *__restrict__ valid,
                                        const float *__restrict__ counts,
                                        float *__restrict__ dS, int64_t batch, int64_t steps,
                                        int modes, int accumulate) {
  // block = (row, kMbTile steps), threads over modes; each thread streams its
  // mode through the tile with states t-4 .. t+8 in registers (w[4] = step
  // t), so every state is loaded once per tile (+ 12 halo steps).
  const int64_t M2 = 2 * modes;
  const unsigned tiles = (unsigned)((steps + kMbTile - 1) / kMbTile);
  const int64_t b = blockIdx.x / tiles;
  const int64_t t_begin = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kMbTile;
  const int64_t t_end = min(steps, t_begin + kMbTile);
  const float *g = dm + b * 7 * modes;
  const float *vrow = valid ? valid + b * steps : nullptr;
  const float c0 = valid ? counts[b * 4] : (float)steps;
  float cl[3];
  const int lags[3] = {1, 2, 4};
#pragma unroll
  for (int l = 0; l < 3; ++l)
    cl[l] = valid ? counts[b * 4 + 1 + l] : (float)(steps - lags[l]);
  const float *srow = s + b * steps * M2;
  float *orow = dS + b * steps * M2;
  // the count normalisations folded into the per-mode cotangents (no division
  // per step)
  const float ic0 = 1.f / c0;
  float icl[3];
#pragma unroll
  for (int l = 0; l < 3; ++l) icl[l] = 1.f / cl[l];
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    const float ge2 = 2.f * g[m] * ic0;
    float dr[3], di[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      dr[l] = g[(1 + 2 * l) * modes + m] * icl[l];
      di[l] = g[(2 + 2 * l) * modes + m] * icl[l];
    }
    // w[0..8] = steps t-4 .. t+4; w[9..12] = t+5 .. t+8, loaded four steps
    // before they enter the window
    float wr[13], wi[13];
#pragma unroll
    for (int j = 0; j < 12; ++j) {  // steps t_begin - 4 .. t_begin + 7
      const int64_t t = t_begin - 4 + j;
      const bool in = t >= 0 && t < steps;
      wr[j] = in ? srow[t * M2 + m] : 0.f;
      wi[j] = in ? srow[t * M2 + modes + m] : 0.f;
    }
    for (int64_t t = t_begin; t < t_end; ++t) {
      const int64_t tn = t + 8;
      const bool in = tn < steps;
      wr[12] = in ? srow[tn * M2 + m] : 0.f;
      wi[12] = in ? srow[tn * M2 + modes + m] : 0.f;
      const float cr = wr[4], ci = wi[4];
      const float vt = vrow ? vrow[t] : 1.f;
      float gr = cr * ge2 * vt, gi = ci * ge2 * vt;
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const int lag = lags[l];
        if (steps <= lag) continue;
        if (t >= lag) {  // t as the current state, s_{t-lag} as the earlier one
          const float pr = wr[4 - lag], pi = wi[4 - lag];
          const float w = vrow ? vt * vrow[t - lag] : 1.f;
          gr += (dr[l] * pr - di[l] * pi) * w;
          gi += (dr[l] * pi + di[l] * pr) * w;
        }
        if (t + lag < steps) {  // t as the earlier state of s_{t+lag}
          const float nr = wr[4 + lag], ni = wi[4 + lag];
          const float w = vrow ? vt * vrow[t + lag] : 1.f;
          gr += (dr[l] * nr + di[l] * ni) * w;
          gi += (dr[l] * ni - di[l] * nr) * w;
        }
      }
      float *out = orow + t * M2;
      if (accumulate) {
        out[m] += gr;
        out[modes + m] += gi;
      } else {
        out[m] = gr;
        out[modes + m] = gi;
      }
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        wr[j] = wr[j + 1];
        wi[j] = wi[j + 1];
      }
    }
  }
}

// Reverse scan, local pass: per (chunk, row), lambda from a zero state after
// the chunk walked backwards (lambda_t = dS_t + conj(a_{t+1}) lambda_{t+1};
// a per mode, or per step from dt); records at the reversed chunk index so
// that scan_carry_kernel (forward composition order) yields each chunk's
// lambda entering from the later steps.  Record: E = local lambda at the
// chunk start, P = the product of the conj(a_{t+1}) of the chunk.
// Pole coefficients of step `tok` for mode m: the per-mode tables, or the ZOH
// of that step's dt (double, rounded once).
__device__ __forceinline__ Zoh step_zoh(const float *a_re, const float *a_im, const float *g_re,
                                        const float *g_im, const float *raw_decay,
                                        const float *raw_freq, const float *dt, int64_t tok,
                                        int m) {
  if (!dt) return Zoh{a_re[m], a_im[m], g_re ? g_re[m] : 0.f, g_im ? g_im[m] : 0.f};
  double damping, frequency;
  mode_pole(raw_decay[m], raw_freq[m], damping, frequency);
  return zoh_eval(damping, frequency, (double)dt[tok]);
}

__global__ void rscan_local_kernel(const float *__restrict__ dS, const float *__restrict__ a_re,
                                   const float *__restrict__ a_im,
                                   const float *__restrict__ raw_decay,
                                   const float *__restrict__ raw_freq,
                                   const float *__restrict__ dt, float *__restrict__ rec_all,
                                   int64_t steps, int modes, int chunk, int64_t n_chunks) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * chunk, t1 = min(steps, t0 + chunk);
  const int64_t M2 = 2 * modes;
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    // (nar, nai) = a_{t+1}, the coefficient that carries lambda_{t+1} back to t
    float nar = 0.f, nai = 0.f;
    if (t1 < steps) {
      const Zoh z = step_zoh(a_re, a_im, nullptr, nullptr, raw_decay, raw_freq, dt,
                             b * steps + t1, m);
      nar = z.a_re;
      nai = z.a_im;
    }
    float lr = 0.f, li = 0.f, pr = 1.f, pi = 0.f;
    for (int64_t t = t1 - 1; t >= t0; --t) {
      const float *row = dS + (b * steps + t) * M2;
      const float nr = row[m] + nar * lr + nai * li;
      const float ni = row[modes + m] + nar * li - nai * lr;
      lr = nr;
      li = ni;
      const float qr = nar * pr + nai * pi, qi = nar * pi - nai * pr;  // conj(a_{t+1}) P
      pr = qr;
      pi = qi;
      const Zoh z = step_zoh(a_re, a_im, nullptr, nullptr, raw_decay, raw_freq, dt,
                             b * steps + t, m);
      nar = z.a_re;
      nai = z.a_im;
    }
    float *rec = rec_all + (b * n_chunks + (n_chunks - 1 - c)) * kRecFloats * modes;
    rec[m] = lr;
    rec[modes + m] = li;
    rec[2 * modes + m] = pr;
    rec[3 * modes + m] = pi;
  }
}

// Reverse scan, apply pass: walks each chunk backwards from the lambda that
// enters it, writes de = conj(g_t) lambda (times the writer's event mask) over
// dS, and sums per (row, chunk, mode) da = lambda x s_{t-1} and dg = lambda x
// u_t / g_t (real-pair form; u_t = s_t - a_t s_{t-1}, the masked drive) into
// polepart [B, nchunk, 4, M].  With per-step coefficients (dt) it sums dL/dp
// directly instead (slots 0, 1), the derivatives of a and g depending on dt.
__global__ void rscan_apply_kernel(float *__restrict__ dS, const float *__restrict__ s,
                                   const float *__restrict__ a_re, const float *__restrict__ a_im,
                                   const float *__restrict__ g_re, const float *__restrict__ g_im,
                                   const float *__restrict__ raw_decay,
                                   const float *__restrict__ raw_freq,
                                   const float *__restrict__ dt, const float *__restrict__ rec_all,
                                   float *__restrict__ polepart, int64_t steps, int modes,
                                   int chunk, int64_t n_chunks,
                                   const float *__restrict__ event_mask, int obs_channels) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * chunk, t1 = min(steps, t0 + chunk);
  const int64_t M2 = 2 * modes;
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    double pdr = 0.0, pdi = 0.0;  // dL/dp (dt) or the da, dg sums (static)
    double pr_ = 0.0, pi_ = 0.0;  // the pole p (dt)
    if (dt) {
      double damping, frequency;
      mode_pole(raw_decay[m], raw_freq[m], damping, frequency);
      pr_ = -damping;
      pi_ = frequency;
    }
    const float *rec = rec_all + (b * n_chunks + (n_chunks - 1 - c)) * kRecFloats * modes;
    float lr = rec[m], li = rec[modes + m];  // lambda_{t1}
    float nar = 0.f, nai = 0.f;                // a_{t+1}
    if (t1 < steps) {
      const Zoh z = step_zoh(a_re, a_im, g_re, g_im, raw_decay, raw_freq, dt, b * steps + t1, m);
      nar = z.a_re;
      nai = z.a_im;
    }
    float dar = 0.f, dai = 0.f, dgr = 0.f, dgi = 0.f;
    // groups of up to 8 steps (descending): the group's dS and state loads (and
    // the state one step before it) are issued before its dependent steps
    for (int64_t tg = t1 - 1; tg >= t0; tg -= 8) {
      const int n = (int)(tg - t0 + 1 < 8 ? tg - t0 + 1 : 8);
      float xr[8], xi[8], svr[9], svi[9];
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const int64_t t = tg - k;
        const bool ld = k <= n && t >= 0;
        const int64_t tok = b * steps + t;
        svr[k] = ld ? s[tok * M2 + m] : 0.f;
        svi[k] = ld ? s[tok * M2 + modes + m] : 0.f;
        if (k < 8) {
          xr[k] = k < n ? dS[tok * M2 + m] : 0.f;
          xi[k] = k < n ? dS[tok * M2 + modes + m] : 0.f;
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k >= n) break;
        const int64_t t = tg - k;
        const int64_t tok = b * steps + t;
        float *row = dS + tok * M2;
        const float nr = xr[k] + nar * lr + nai * li;
        const float ni = xi[k] + nar * li - nai * lr;
        lr = nr;
        li = ni;
        const Zoh z = step_zoh(a_re, a_im, g_re, g_im, raw_decay, raw_freq, dt, tok, m);
        const float ar = z.a_re, ai = z.a_im, gr = z.g_re, gi = z.g_im;
        const float sr = svr[k], si = svi[k];
        const float pr = svr[k + 1], pi = svi[k + 1];  // zero before step 0
        const float ddr = lr * pr + li * pi, ddi = -lr * pi + li * pr;  // da at this step
        const float ur = sr - (ar * pr - ai * pi), ui = si - (ai * pr + ar * pi);
        const float igden = 1.f / (gr * gr + gi * gi);
        const float er = (ur * gr + ui * gi) * igden, ei = (ui * gr - ur * gi) * igden;
        const float dgr_ = lr * er + li * ei, dgi_ = -lr * ei + li * er;  // dg at this step
        if (dt) {
          // dL/dp += Re/Im pairs with a'(p) = dt a and g'(p) = (dt a p - (a - 1)) / p^2
          const double h = (double)dt[tok];
          const double far = h * ar, fai = h * ai;
          double fgr = 0.0, fgi = 0.0;
          if (sqrt(pr_ * pr_ + pi_ * pi_) * h >= 1.0e-6) {
            const double apr = ar * pr_ - ai * pi_, api = ar * pi_ + ai * pr_;
            const double nr2 = h * apr - (ar - 1.0), ni2 = h * api - ai;
            const double p2r = pr_ * pr_ - pi_ * pi_, p2i = 2.0 * pr_ * pi_;
            const double den = p2r * p2r + p2i * p2i;
            fgr = (nr2 * p2r + ni2 * p2i) / den;
            fgi = (ni2 * p2r - nr2 * p2i) / den;
          }
          pdr += ddr * far + ddi * fai + dgr_ * fgr + dgi_ * fgi;
          pdi += -ddr * fai + ddi * far - dgr_ * fgi + dgi_ * fgr;
        } else {
          dar += ddr;
          dai += ddi;
          dgr += dgr_;
          dgi += dgi_;
        }
        float ev = 1.f;  // u = event g e: de carries the event mask (amax over channels)
        if (event_mask) {
          const float *om = event_mask + tok * obs_channels;
          ev = om[0];
          for (int c2 = 1; c2 < obs_channels; ++c2) ev = fmaxf(ev, om[c2]);
        }
        row[m] = (lr * gr + li * gi) * ev;  // de = conj(g) lambda
        row[modes + m] = (-lr * gi + li * gr) * ev;
        nar = ar;
        nai = ai;
      }
    }
    float *pp = polepart + (b * n_chunks + c) * 4 * modes;
    if (dt) {
      pp[m] = (float)pdr;
      pp[modes + m] = (float)pdi;
      pp[2 * modes + m] = 0.f;
      pp[3 * modes + m] = 0.f;
    } else {
      pp[m] = dar;
      pp[modes + m] = dai;
      pp[2 * modes + m] = dgr;
      pp[3 * modes + m] = dgi;
    }
  }
}

// d raw_decay, d raw_frequency from the summed da, dg of every (row, chunk):
// dL/dp by the Cauchy-Riemann form of a'(p) = a and g'(p) = (a p - (a - 1)) / p^2
// (dt = 1), then damping = dmin + (dmax - dmin) sigmoid(raw), freq = pi tanh(raw).
// `sums` [4][M]: da re, da im, dg re, dg im summed over every (row, chunk).
// `per_step`: sums hold dL/dp (re, im) already (time_delta requests).
__global__ void pole_backward_kernel(const float *__restrict__ sums, int modes,
                                     const float *__restrict__ raw_decay,
                                     const float *__restrict__ raw_freq,
                                     float *__restrict__ d_decay, float *__restrict__ d_freq,
                                     int per_step) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= modes) return;
  double s[4];
  for (int k = 0; k < 4; ++k) s[k] = (double)sums[k * modes + m];
  if (per_step) {
    const double sig = 1.0 / (1.0 + exp(-(double)raw_decay[m]));
    const double th = tanh((double)raw_freq[m]);
    d_decay[m] = (float)(-s[0] * (kDampingMax - kDampingMin) * sig * (1.0 - sig));
    d_freq[m] = (float)(s[1] * kPi * (1.0 - th * th));
    return;
  }
  const double sig = 1.0 / (1.0 + exp(-(double)raw_decay[m]));
  const double damping = kDampingMin + (kDampingMax - kDampingMin) * sig;
  const double th = tanh((double)raw_freq[m]);
  const double pr = -damping, pi = kPi * th;
  const double ea = exp(pr);
  const double ar = ea * cos(pi), ai = ea * sin(pi);
  // fg = (a p - (a - 1)) / p^2
  const double apr = ar * pr - ai * pi, api = ar * pi + ai * pr;
  const double nr = apr - (ar - 1.0), ni = api - ai;
  const double p2r = pr * pr - pi * pi, p2i = 2.0 * pr * pi;
  const double den = p2r * p2r + p2i * p2i;
  const double fgr = (nr * p2r + ni * p2i) / den, fgi = (ni * p2r - nr * p2i) / den;
  const double dpr = s[0] * ar + s[1] * ai + s[2] * fgr + s[3] * fgi;
  const double dpi = -s[0] * ai + s[1] * ar - s[2] * fgi + s[3] * fgr;
  d_decay[m] = (float)(-dpr * (kDampingMax - kDampingMin) * sig * (1.0 - sig));
  d_freq[m] = (float)(dpi * kPi * (1.0 - th * th));
}

// RMSNorm VJP, one warp per token: dy = rs g dxh - y rs^3 sum(g dxh y) / D
// (+ add); also stores rs for the gain's column sum.
__global__ void rms_backward_kernel(const float *__restrict__ y, const float *__restrict__ dxh,
                                    const float *__restrict__ g, const float *__restrict__ add,
                                    float *__restrict__ dy, float *__restrict__ rs_out,
                                    int64_t tokens, int dim) {
  const int64_t tok = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (tok >= tokens) return;
  const float *yr = y + tok * dim, *dr = dxh + tok * dim;
  float ss = 0.f, dot = 0.f;
  for (int d = lane; d < dim; d += 32) {
    ss = fmaf(yr[d], yr[d], ss);
    dot = fmaf(dr[d] * g[d], yr[d], dot);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    dot += __shfl_xor_sync(0xffffffffu, dot, o);
  }
  const float rs = rsqrtf(ss / (float)dim + kFp32Eps);
  const float k = rs * rs * rs * dot / (float)dim;
  for (int d = lane; d < dim; d += 32) {
    float v = rs * g[d] * dr[d] - yr[d] * k;
    if (add) v += add[tok * dim + d];
    dy[tok * dim + d] = v;
  }
  if (lane == 0) rs_out[tok] = rs;
}

// The same VJP over float4 quads (dim % 4 == 0, 16-byte aligned rows), with the
// lane layout of rmsnorm4_kernel: `width` lanes per token.
__global__ void rms_backward4_kernel(const float4 *__restrict__ y, const float4 *__restrict__ dxh,
                                     const float4 *__restrict__ g, const float4 *__restrict__ add,
                                     float4 *__restrict__ dy, float *__restrict__ rs_out,
                                     int64_t tokens, int quads) {
  const int lane = threadIdx.x & 31;
  const int width = quads < 32 && (quads & (quads - 1)) == 0 ? quads : 32;
  const int per_warp = 32 / width;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t tok = warp * per_warp + lane / width;
  const int sl = lane & (width - 1);
  const bool on = tok < tokens;
  const float4 *yr = y + tok * quads, *dr = dxh + tok * quads;
  float ss = 0.f, dot = 0.f;
  if (on)
    for (int q = sl; q < quads; q += width) {
      const float4 v = yr[q], d = dr[q], w = g[q];
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      dot = fmaf(d.x * w.x, v.x, fmaf(d.y * w.y, v.y, fmaf(d.z * w.z, v.z, fmaf(d.w * w.w, v.w, dot))));
    }
  for (int o = width >> 1; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    dot += __shfl_xor_sync(0xffffffffu, dot, o);
  }
  if (!on) return;
  const float rs = rsqrtf(ss / (float)(4 * quads) + kFp32Eps);
  const float k = rs * rs * rs * dot / (float)(4 * quads);
  for (int q = sl; q < quads; q += width) {
    const float4 v = yr[q], d = dr[q], w = g[q];
    float4 o = make_float4(rs * w.x * d.x - v.x * k, rs * w.y * d.y - v.y * k,
                           rs * w.z * d.z - v.z * k, rs * w.w * d.w - v.w * k);
    if (add) {
      const float4 a = add[tok * quads + q];
      o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
    }
    dy[tok * quads + q] = o;
  }
  if (sl == 0) rs_out[tok] = rs;
}

// rms_backward_kernel or, where the rows allow it, rms_backward4_kernel.
static int rms_backward(const float *y, const float *dxh, const float *g, const float *add,
                        float *dy, float *rs, int64_t tokens, int D, cudaStream_t st) {
  auto al = [](const void *q) { return q == nullptr || reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  const int quads = D / 4;
  if (D % 4 == 0 && quads > 0 && al(y) && al(dxh) && al(g) && al(add) && al(dy)) {
    const bool pow2 = (quads & (quads - 1)) == 0;
    const int per_warp = quads < 32 && pow2 ? 32 / quads : 1;
    rms_backward4_kernel<<<(unsigned)cdiv(tokens, 8 * per_warp), 256, 0, st>>>(
        reinterpret_cast<const float4 *>(y), reinterpret_cast<const float4 *>(dxh),
        reinterpret_cast<const float4 *>(g), reinterpret_cast<const float4 *>(add),
        reinterpret_cast<float4 *>(dy), rs, tokens, quads);
  } else {
    rms_backward_kernel<<<(unsigned)cdiv(tokens, 8), 256, 0, st>>>(y, dxh, g, add, dy, rs,
                                                                  tokens, D);
  }
  return after_launch("rms_backward_kernel");
}

// Conv + SiLU VJP, pre-activation gradient: dz = dy * out_mask * silu'(z),
// z = bias + sum_k w_k in[t + k dil - pad] * in_mask (recomputed).
__global__ void conv_dz_kernel(const float *__restrict__ in, const float *__restrict__ w,
                               const float *__restrict__ bias, const float *__restrict__ in_mask,
                               const float *__restrict__ out_mask, const float *__restrict__ dy,
                               float *__restrict__ dz, int64_t batch, int64_t steps, int dim,
                               int taps, int dil) {
  // block = (row, kBwdTile steps), threads over channels
  const int pad = dil * (taps - 1) / 2;
  const unsigned tiles = (unsigned)((steps + kBwdTile - 1) / kBwdTile);
  const int64_t b = blockIdx.x / tiles;
  const int64_t t_begin = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kBwdTile;
  const int64_t t_end = min(steps, t_begin + kBwdTile);
  const float *rin = in + b * steps * dim;
  const float *im = in_mask ? in_mask + b * steps : nullptr;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    const float bd = bias[d];
    for (int64_t t = t_begin; t < t_end; ++t) {
      float z = 0.f;
      for (int k = 0; k < taps; ++k) {
        const int64_t sidx = t + (int64_t)k * dil - pad;
        if (sidx < 0 || sidx >= steps) continue;
        float v = rin[sidx * dim + d];
        if (im) v *= im[sidx];
        z = fmaf(w[d * taps + k], v, z);
      }
      z += bd;
      const float sg = 1.0f / (1.0f + expf(-z));
      const int64_t i = (b * steps + t) * dim + d;
      float gz = dy[i] * sg * (1.0f + z * (1.0f - sg));
      if (out_mask) gz *= out_mask[b * steps + t];
      dz[i] = gz;
    }
  }
}

// Input gradient of the depthwise conv: dx[s] = in_mask[s] sum_k w_k dz[s - k dil + pad].
__global__ void conv_dx_kernel(const float *__restrict__ dz, const float *__restrict__ w,
                               const float *__restrict__ in_mask, float *__restrict__ dx,
                               int64_t batch, int64_t steps, int dim, int taps, int dil) {
  const int pad = dil * (taps - 1) / 2;
  const unsigned tiles = (unsigned)((steps + kBwdTile - 1) / kBwdTile);
  const int64_t b = blockIdx.x / tiles;
  const int64_t s_begin = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kBwdTile;
  const int64_t s_end = min(steps, s_begin + kBwdTile);
  const float *rz = dz + b * steps * dim;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    for (int64_t si = s_begin; si < s_end; ++si) {
      float acc = 0.f;
      for (int k = 0; k < taps; ++k) {
        const int64_t t = si - (int64_t)k * dil + pad;
        if (t < 0 || t >= steps) continue;
        acc = fmaf(w[d * taps + k], rz[t * dim + d], acc);
      }
      if (in_mask) acc *= in_mask[b * steps + si];
      dx[(b * steps + si) * dim + d] = acc;
    }
  }
}

// Conv weight and bias gradient partials: block = (row, kWgTile steps),
// threads over channels; each thread accumulates, over its tile, dz[t] x
// xin[t + k dil - pad] (masked input) for every tap and dz[t] for the bias,
// and writes partial[part][d * (taps + 1) + j] (j = taps: the bias).
template <int TAPS>
__global__ void conv_wgrad_kernel(const float *__restrict__ dz, const float *__restrict__ xin,
                                  const float *__restrict__ in_mask, float *__restrict__ partial,
                                  int64_t steps, int dim, int dil) {
  constexpr int taps = TAPS;
  const int pad = dil * (taps - 1) / 2;
  const unsigned tiles = (unsigned)((steps + kWgTile - 1) / kWgTile);
  const int64_t b = blockIdx.x / tiles;
  const int64_t t_begin = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kWgTile;
  const int64_t t_end = min(steps, t_begin + kWgTile);
  const float *rz = dz + b * steps * dim;
  const float *rx = xin + b * steps * dim;
  const float *im = in_mask ? in_mask + b * steps : nullptr;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float acc[TAPS + 1];
#pragma unroll
    for (int k = 0; k <= TAPS; ++k) acc[k] = 0.f;
    for (int64_t t = t_begin; t < t_end; ++t) {
      const float g = rz[t * dim + d];
      acc[taps] += g;
#pragma unroll
      for (int k = 0; k < taps; ++k) {
        const int64_t sidx = t + (int64_t)k * dil - pad;
        if (sidx < 0 || sidx >= steps) continue;
        float x = rx[sidx * dim + d];
        if (im) x *= im[sidx];
        acc[k] = fmaf(g, x, acc[k]);
      }
    }
    float *out = partial + (int64_t)blockIdx.x * dim * (taps + 1) + d * (taps + 1);
#pragma unroll
    for (int k = 0; k <= taps; ++k) out[k] = acc[k];
  }
}

// 16-byte asynchronous global -> shared copy (zero-filled when `bytes` is 0);
// completion is awaited with cp.async.wait_group (a hardware wait).
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sm100::smem_u32(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// The conv + SiLU VJP in one pass for a row's kCbTile steps (TAPS taps,
// 4 | dim <= 256): stage the input of steps [s0 - 2 pad, s0 + kCbTile + 2 pad)
// and dy of [s0 - pad, s0 + kCbTile + pad) in shared memory with 16-byte
// asynchronous copies (zero outside the sequence), form dz = dy out_mask
// silu'(z) in place (z recomputed from the masked input), then per channel the
// input gradient of the core steps and the weight / bias partial sums over
// them (partial[block][d (TAPS + 1) + j]).
template <int TAPS>
__global__ void __launch_bounds__(256) conv_backward_kernel(
    const float *__restrict__ in, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ in_mask, const float *__restrict__ out_mask,
    const float *__restrict__ dy, float *__restrict__ dx, float *__restrict__ partial,
    int64_t steps, int dim, int dil) {
  extern __shared__ float4 cb_smem4[];
  float *cb_smem = reinterpret_cast<float *>(cb_smem4);
  const int pad = dil * (TAPS - 1) / 2;
  const int xrows = kCbTile + 4 * pad, zrows = kCbTile + 2 * pad;
  const int quads = dim >> 2;
  float *sx = cb_smem;          // [xrows][dim] masked input
  float *sz = sx + xrows * dim; // [zrows][dim] dy, then dz
  const unsigned tiles = (unsigned)((steps + kCbTile - 1) / kCbTile);
  const int64_t b = blockIdx.x / tiles;
  const int64_t s0 = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kCbTile;
  const float *rin = in + b * steps * dim;
  const float *rdy = dy + b * steps * dim;
  const float *im = in_mask ? in_mask + b * steps : nullptr;
  const float *om = out_mask ? out_mask + b * steps : nullptr;
  // thread -> (row group, 16-byte column quad) for the copies and (row group,
  // channel) for the arithmetic: no per-element index division
  const int qgroups = max(1, (int)blockDim.x / quads);
  const int qg = (int)threadIdx.x / quads, q = (int)threadIdx.x - qg * quads;
  if (qg < qgroups) {
    for (int r = qg; r < xrows; r += qgroups) {
      const int64_t t = s0 - 2 * pad + r;
      const bool live = t >= 0 && t < steps;
      cp_async16(sx + r * dim + 4 * q, rin + (live ? t : 0) * dim + 4 * q, live ? 16 : 0);
    }
    for (int r = qg; r < zrows; r += qgroups) {
      const int64_t t = s0 - pad + r;
      const bool live = t >= 0 && t < steps;
      cp_async16(sz + r * dim + 4 * q, rdy + (live ? t : 0) * dim + 4 * q, live ? 16 : 0);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const int groups = max(1, (int)blockDim.x / dim);
  const int gid = (int)threadIdx.x / dim, d = (int)threadIdx.x - gid * dim;
  if (im) {
    if (gid < groups)
      for (int r = gid; r < xrows; r += groups) {
        const int64_t t = s0 - 2 * pad + r;
        if (t >= 0 && t < steps) sx[r * dim + d] *= im[t];
      }
    __syncthreads();
  }
  if (gid < groups) {
    float wk[TAPS];
#pragma unroll
    for (int k = 0; k < TAPS; ++k) wk[k] = w[d * TAPS + k];
    const float bd = bias[d];
    for (int r = gid; r < zrows; r += groups) {
      const int64_t t = s0 - pad + r;
      float gz = 0.f;
      if (t >= 0 && t < steps) {
        float z = 0.f;
#pragma unroll
        for (int k = 0; k < TAPS; ++k) z = fmaf(wk[k], sx[(r + k * dil) * dim + d], z);
        z += bd;
        const float sg = __fdividef(1.0f, 1.0f + __expf(-z));
        gz = sz[r * dim + d] * sg * (1.0f + z * (1.0f - sg));
        if (om) gz *= om[t];
      }
      sz[r * dim + d] = gz;
    }
  }
  __syncthreads();
  const int n_core = (int)min((int64_t)kCbTile, steps - s0);
  // the core steps are dealt round-robin to the `groups` thread groups of each
  // channel; their weight / bias sums meet in shared memory (the input tile's
  // space, free once every thread has passed the barrier below)
  float aw[TAPS + 1];
#pragma unroll
  for (int k = 0; k <= TAPS; ++k) aw[k] = 0.f;
  if (gid < groups) {
    float wk[TAPS];
#pragma unroll
    for (int k = 0; k < TAPS; ++k) wk[k] = w[d * TAPS + k];
    for (int r = gid; r < n_core; r += groups) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < TAPS; ++k) acc = fmaf(wk[k], sz[(r - k * dil + 2 * pad) * dim + d], acc);
      if (im) acc *= im[s0 + r];
      dx[(b * steps + s0 + r) * dim + d] = acc;
      const float g = sz[(r + pad) * dim + d];
      aw[TAPS] += g;
#pragma unroll
      for (int k = 0; k < TAPS; ++k) aw[k] = fmaf(g, sx[(r + pad + k * dil) * dim + d], aw[k]);
    }
  }
  __syncthreads();
  float *red = sx;  // [groups][dim][TAPS + 1]
  if (gid < groups) {
#pragma unroll
    for (int k = 0; k <= TAPS; ++k) red[(gid * dim + d) * (TAPS + 1) + k] = aw[k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim * (TAPS + 1); i += blockDim.x) {
    float v = 0.f;
    for (int q = 0; q < groups; ++q) v += red[q * dim * (TAPS + 1) + i];
    partial[(int64_t)blockIdx.x * dim * (TAPS + 1) + i] = v;
  }
}

// Spread [D][taps + 1] sums into the weight [D, taps] and bias [D] gradients.
__global__ void conv_wgrad_split_kernel(const float *__restrict__ sums, float *__restrict__ dw,
                                        float *__restrict__ db, int dim, int taps) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dim * (taps + 1)) return;
  const int d = i / (taps + 1), k = i - d * (taps + 1);
  if (k < taps)
    dw[d * taps + k] = sums[i];
  else
    db[d] = sums[i];
}

// dxh_res = dv ls ds (the residual's xhat path).
__global__ void residual_dxh_kernel(const float *__restrict__ dv, const float *__restrict__ ls,
                                    const float *__restrict__ ds, float *__restrict__ dxh,
                                    int64_t tokens, int dim) {
  const int64_t n = tokens * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % dim);
    dxh[i] = dv[i] * ls[d] * ds[d];
  }
}

// ---------------------------------------------------------------- physical time (time_delta)
// Sample position of a physical-time lookup at `q` in one row's timestamps:
// lower / upper index, interpolation weight and whether q lies inside the row
// (the arithmetic of dwconv_physical_kernel and pt_moments_partial_kernel).
struct PtPos {
  int64_t lo, hi;
  float w;
  bool in;
};
__device__ __forceinline__ PtPos pt_position(const float *row, int64_t steps, float q) {
  const int64_t up_u = lower_bound_f(row, steps, q);
  PtPos r;
  r.hi = up_u < steps - 1 ? up_u : steps - 1;
  int64_t lo = up_u - 1;
  r.lo = lo < 0 ? 0 : (lo > steps - 1 ? steps - 1 : lo);
  const float lt = row[r.lo], ut = row[r.hi];
  const float span = ut - lt;
  const float ip = span > 0.f ? (q - lt) / fmaxf(span, kFp32Tiny) : 0.f;
  r.w = fminf(fmaxf(ip, 0.f), 1.f);
  r.in = (q >= row[0]) && (q <= row[steps - 1]);
  return r;
}
__device__ __forceinline__ float pt_support(const float *vrow, const PtPos &p) {
  if (!vrow) return 1.f;
  const float lv = vrow[p.lo], uv = vrow[p.hi];
  const float eps8 = 8.0f * kFp32Eps;
  return p.w <= eps8 ? lv : (p.w >= 1.0f - eps8 ? uv : lv * uv);
}

// Per-row normalisers of the physical-time moments: counts[b] = {energy count
// ec, use-duration flag, pair weights pc_1, pc_2, pc_4} (as
// pt_moments_finalize_kernel forms them).  One block per row.
__global__ void pt_counts_kernel(const float *__restrict__ ts, const float *__restrict__ dt,
                                 const float *__restrict__ valid, int64_t steps,
                                 float *__restrict__ counts) {
  const int64_t b = blockIdx.x;
  const float *row = ts + b * steps;
  const float *vrow = valid ? valid + b * steps : nullptr;
  const int lags[3] = {1, 2, 4};
  __shared__ double red[5][32];
  double c[5] = {0, 0, 0, 0, 0};
  for (int64_t t = threadIdx.x; t < steps; t += blockDim.x) {
    const float vt = vrow ? vrow[t] : 1.f;
    c[0] += (double)(dt[b * steps + t] * vt);
    c[1] += (double)vt;
    for (int l = 0; l < 3; ++l) {
      const PtPos pp = pt_position(row, steps, row[t] - (float)lags[l]);
      const float sup = pt_support(vrow, pp) * (pp.in ? 1.f : 0.f);
      c[2 + l] += (double)(dt[b * steps + t] * vt * sup);
    }
  }
  for (int k = 0; k < 5; ++k) {
    double x = c[k];
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if ((threadIdx.x & 31) == 0) red[k][threadIdx.x >> 5] = x;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot[5] = {0, 0, 0, 0, 0};
    for (int k = 0; k < 5; ++k)
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot[k] += red[k][w];
    const bool use_d = tot[0] > 0.0;
    counts[b * 8 + 0] = fmaxf((float)(use_d ? tot[0] : tot[1]), 1.0f);
    counts[b * 8 + 1] = use_d ? 1.f : 0.f;
    for (int l = 0; l < 3; ++l) counts[b * 8 + 2 + l] = fmaxf((float)tot[2 + l], 1.0f);
  }
}

// State gradient of the physical-time moments, added with atomics into a zeroed
// dS: per (row, chunk) block with threads over modes; for each step the energy
// term (duration-weighted when the row's durations sum above zero), and for
// each lag the pair with the state interpolated at t - lag: the current-state
// term at t and the interpolated-state term scattered onto its lower / upper
// samples with weights 1 - w and w.
__global__ void pt_moments_backward_kernel(const float *__restrict__ s, const float *__restrict__ ts,
                                           const float *__restrict__ dt,
                                           const float *__restrict__ valid,
                                           const float *__restrict__ counts,
                                           const float *__restrict__ dm, float *__restrict__ dS,
                                           int64_t steps, int modes) {
  __shared__ int64_t s_lo[3][kPtChunk], s_hi[3][kPtChunk];
  __shared__ float s_ip[3][kPtChunk], s_pw[3][kPtChunk], s_ew[kPtChunk];
  const int64_t c = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = c * kPtChunk;
  const int n = (int)min((int64_t)kPtChunk, steps - t0);
  const float *row = ts + b * steps;
  const float *vrow = valid ? valid + b * steps : nullptr;
  const float *cnt = counts + b * 8;
  const int lags[3] = {1, 2, 4};
  for (int j = threadIdx.x; j < n * 3; j += blockDim.x) {
    const int i = j / 3, l = j - (j / 3) * 3;
    const int64_t t = t0 + i;
    const PtPos pp = pt_position(row, steps, row[t] - (float)lags[l]);
    const float vt = vrow ? vrow[t] : 1.f;
    s_lo[l][i] = b * steps + pp.lo;
    s_hi[l][i] = b * steps + pp.hi;
    s_ip[l][i] = pp.w;
    s_pw[l][i] = dt[b * steps + t] * vt * pt_support(vrow, pp) * (pp.in ? 1.f : 0.f) / cnt[2 + l];
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float vt = vrow ? vrow[t0 + i] : 1.f;
    s_ew[i] = (cnt[1] > 0.f ? dt[b * steps + t0 + i] * vt : vt) / cnt[0];
  }
  __syncthreads();
  const int64_t M2 = 2 * modes;
  const float *g = dm + b * 7 * modes;
  for (int m = threadIdx.x; m < modes; m += blockDim.x) {
    const float ge = g[m];
    float dr[3], di[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      dr[l] = g[(1 + 2 * l) * modes + m];
      di[l] = g[(2 + 2 * l) * modes + m];
    }
    for (int i = 0; i < n; ++i) {
      const int64_t tok = b * steps + t0 + i;
      const float cr = s[tok * M2 + m], ci = s[tok * M2 + modes + m];
      float gr = 2.f * cr * ge * s_ew[i], gi = 2.f * ci * ge * s_ew[i];
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const float pw = s_pw[l][i];
        if (pw == 0.f) continue;
        const float *lo = s + s_lo[l][i] * M2, *hi = s + s_hi[l][i] * M2;
        const float w = s_ip[l][i];
        const float pr = lerp_torch(lo[m], hi[m], w), pi = lerp_torch(lo[modes + m], hi[modes + m], w);
        gr += (dr[l] * pr - di[l] * pi) * pw;
        gi += (dr[l] * pi + di[l] * pr) * pw;
        const float hr = (dr[l] * cr + di[l] * ci) * pw, hi_ = (dr[l] * ci - di[l] * cr) * pw;
        atomicAdd(dS + s_lo[l][i] * M2 + m, (1.f - w) * hr);
        atomicAdd(dS + s_lo[l][i] * M2 + modes + m, (1.f - w) * hi_);
        atomicAdd(dS + s_hi[l][i] * M2 + m, w * hr);
        atomicAdd(dS + s_hi[l][i] * M2 + modes + m, w * hi_);
      }
      atomicAdd(dS + tok * M2 + m, gr);
      atomicAdd(dS + tok * M2 + modes + m, gi);
    }
  }
}

// The physical-time conv + SiLU VJP for a row's kCbTile steps (threads over
// channels): sample positions of every (step, tap) in shared memory, the
// pre-activation recomputed on the masked input, dz = dy out_mask silu'(z),
// the input gradient scattered onto the lower / upper samples with atomics
// (times the input mask there), and weight / bias partial sums
// (partial[block][d (taps + 1) + j]).
constexpr int kPcTaps = 8;
__global__ void pconv_backward_kernel(const float *__restrict__ in, const float *__restrict__ w,
                                      const float *__restrict__ bias,
                                      const float *__restrict__ in_mask,
                                      const float *__restrict__ ts,
                                      const float *__restrict__ valid,
                                      const float *__restrict__ out_mask,
                                      const float *__restrict__ dy, float *__restrict__ dx,
                                      float *__restrict__ partial, int64_t steps, int dim,
                                      int taps, int dil) {
  __shared__ int64_t s_lo[kCbTile][kPcTaps], s_hi[kCbTile][kPcTaps];
  __shared__ float s_w[kCbTile][kPcTaps], s_on[kCbTile][kPcTaps];
  const unsigned tiles = (unsigned)((steps + kCbTile - 1) / kCbTile);
  const int64_t b = blockIdx.x / tiles;
  const int64_t t0 = (int64_t)(blockIdx.x - (unsigned)b * tiles) * kCbTile;
  const int n = (int)min((int64_t)kCbTile, steps - t0);
  const float *row = ts + b * steps;
  const float *vrow = valid ? valid + b * steps : nullptr;
  const int left = dil * (taps - 1) / 2;
  for (int j = threadIdx.x; j < n * taps; j += blockDim.x) {
    const int i = j / taps, k = j - (j / taps) * taps;
    const PtPos pp = pt_position(row, steps, row[t0 + i] + (float)(k * dil - left));
    bool on = pp.in;
    if (vrow) on = on && (pt_support(vrow, pp) > 0.f);
    s_lo[i][k] = b * steps + pp.lo;
    s_hi[i][k] = b * steps + pp.hi;
    s_w[i][k] = pp.w;
    s_on[i][k] = on ? 1.f : 0.f;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float aw[kPcTaps];
    for (int k = 0; k < taps; ++k) aw[k] = 0.f;
    float ab = 0.f;
    for (int i = 0; i < n; ++i) {
      const int64_t tok = b * steps + t0 + i;
      float samp[kPcTaps];
      for (int k = 0; k < taps; ++k) {
        float a = in[s_lo[i][k] * dim + d], c2 = in[s_hi[i][k] * dim + d];
        if (in_mask) {
          a *= in_mask[s_lo[i][k]];
          c2 *= in_mask[s_hi[i][k]];
        }
        samp[k] = s_on[i][k] > 0.f ? lerp_torch(a, c2, s_w[i][k]) : 0.f;
      }
      float zf = 0.f;  // the forward's order: taps 0..K-1, then the bias
      for (int k = 0; k < taps; ++k) zf = fmaf(samp[k], w[d * taps + k], zf);
      zf += bias[d];
      const float sg = 1.0f / (1.0f + expf(-zf));
      float gz = dy[tok * dim + d] * sg * (1.0f + zf * (1.0f - sg));
      if (out_mask) gz *= out_mask[tok];
      ab += gz;
      for (int k = 0; k < taps; ++k) {
        aw[k] = fmaf(gz, samp[k], aw[k]);
        const float g = gz * w[d * taps + k] * s_on[i][k];
        if (g == 0.f) continue;
        const float wl = s_w[i][k];
        const float ml = in_mask ? in_mask[s_lo[i][k]] : 1.f;
        const float mh = in_mask ? in_mask[s_hi[i][k]] : 1.f;
        atomicAdd(dx + s_lo[i][k] * dim + d, (1.f - wl) * g * ml);
        atomicAdd(dx + s_hi[i][k] * dim + d, wl * g * mh);
      }
    }
    float *out = partial + (int64_t)blockIdx.x * dim * (taps + 1) + d * (taps + 1);
    for (int k = 0; k < taps; ++k) out[k] = aw[k];
    out[taps] = ab;
  }
}

// ---------------------------------------------------------------- backward orchestration
// C[n1, n2] (row-major) = sum_r A[r, n1] Bm[r, n2] (+ beta C): the weight
// gradients (A [R, n1], Bm [R, n2] row-major).
static int gemm_wgrad(cudaStream_t st, const float *A, int64_t n1, const float *Bm, int64_t n2,
                      float *C, int64_t R, float beta, bool tf32, const char *what) {
  if (R == 0 || n1 == 0 || n2 == 0) return LNET_OK;
  if (R > INT32_MAX) return fail(LNET_ERR_UNSUPPORTED, "%s: %lld rows", what, (long long)R);
  cublasHandle_t h;
  LNET_TRY(blas_handle(&h));
  if (cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS)
    return fail(LNET_ERR_CUDA, "cublasSetStream failed");
  // column-major: C^T [n2 x n1] = Bm_cm [n2 x R] * (A_cm [n1 x R])^T
  const float alpha = 1.f;
  const cublasStatus_t s = cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_T, (int)n2, (int)n1, (int)R,
                                        &alpha, Bm, CUDA_R_32F, (int)n2, A, CUDA_R_32F, (int)n1,
                                        &beta, C, CUDA_R_32F, (int)n2,
                                        tf32 ? CUBLAS_COMPUTE_32F_FAST_TF32 : CUBLAS_COMPUTE_32F,
                                        CUBLAS_GEMM_DEFAULT);
  if (s != CUBLAS_STATUS_SUCCESS) return fail(LNET_ERR_CUDA, "%s: cublasGemmEx status %d", what, (int)s);
  return after_library(what);
}

// One block's backward from its state gradient in tp.dS (already holding the
// moments' and, for the writer, the synthesis' contributions): reverse scan,
// pole gradients, drive GEMMs.  dxh receives de F^T (+ beta dxh); dframe
// receives xhat^T de (+ beta_frame dframe).
static int block_backward(const TrainPlan &tp, const float *states, const float *xh,
                          const float *frame, const float *raw_decay, const float *raw_freq,
                          const float *a_re, const float *a_im, const float *g_re,
                          const float *g_im, float *dxh, float dxh_beta, float *dframe,
                          float frame_beta, float *d_decay, float *d_freq, int64_t B, int64_t T,
                          int D, int M, bool tf32, const float *event_mask, int obs_channels,
                          const float *dt, cudaStream_t st) {
  const int64_t n_scan = cdiv(T, kScanChunk);
  const int threads = std::min(128, (int)cdiv(M, 32) * 32);
  const dim3 gs((unsigned)n_scan, (unsigned)B);
  rscan_local_kernel<<<gs, threads, 0, st>>>(tp.dS, a_re, a_im, raw_decay, raw_freq, dt,
                                             tp.carries, T, M, kScanChunk, n_scan);
  LNET_TRY(after_launch("rscan_local_kernel"));
  scan_carry_kernel<<<dim3((unsigned)cdiv(M, 32), (unsigned)B), 32 * kCarryParts, 0, st>>>(
      tp.carries, B, M, n_scan, nullptr);
  LNET_TRY(after_launch("scan_carry_kernel"));
  rscan_apply_kernel<<<gs, threads, 0, st>>>(tp.dS, states, a_re, a_im, g_re, g_im, raw_decay,
                                             raw_freq, dt, tp.carries, tp.polepart, T, M,
                                             kScanChunk, n_scan, event_mask, obs_channels);
  LNET_TRY(after_launch("rscan_apply_kernel"));
  LNET_TRY(colsum(ColPlain{tp.polepart, 4 * M}, B * n_scan, 4 * M, tp.colpart, tp.polesum, st,
                  "colsum(pole)"));
  pole_backward_kernel<<<(unsigned)cdiv(M, 64), 64, 0, st>>>(tp.polesum, M, raw_decay, raw_freq,
                                                             d_decay, d_freq, dt ? 1 : 0);
  LNET_TRY(after_launch("pole_backward_kernel"));
  const int64_t bt = B * T;
  LNET_TRY(gemm_rows(st, tp.dS, CUDA_R_32F, 2 * M, frame, CUDA_R_32F, 2 * M, 1, dxh, D, bt, D,
                     2 * M, tf32, "gemm(d xhat)", dxh_beta));
  return gemm_wgrad(st, xh, D, tp.dS, 2 * M, dframe, bt, frame_beta, tf32, "gemm(d frame)");
}

static int conv_backward(const TrainPlan &tp, const float *in, const float *w, const float *bias,
                         const float *in_mask, const float *out_mask, const float *dy, float *dx,
                         float *dw, float *db, int64_t B, int64_t T, int D, int taps, int dil,
                         cudaStream_t st) {
  const int64_t bt = B * T;
  if (taps == 5 && D <= 256 && D % 4 == 0) {  // one fused pass
    const int pad = dil * (taps - 1) / 2;
    const size_t smem = (size_t)(2 * kCbTile + 6 * pad) * D * sizeof(float);
    if (smem > 227 * 1024) return fail(LNET_ERR_UNSUPPORTED, "conv backward: dilation too large");
    LNET_TRY(cuda_check(cudaFuncSetAttribute(conv_backward_kernel<5>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "cudaFuncSetAttribute(conv_backward_kernel)"));
    const unsigned cb_grid = (unsigned)(B * cdiv(T, kCbTile));
    const unsigned cb_threads = 256;  // D <= 256: every channel has at least one thread
    conv_backward_kernel<5><<<cb_grid, cb_threads, smem, st>>>(in, w, bias, in_mask, out_mask,
                                                                dy, dx, tp.colpart, T, D, dil);
    LNET_TRY(after_launch("conv_backward_kernel"));
    LNET_TRY(colsum_finish(tp.colpart, (int)cb_grid, D * (taps + 1), tp.polesum, st));
    conv_wgrad_split_kernel<<<(unsigned)cdiv(D * (taps + 1), 256), 256, 0, st>>>(tp.polesum, dw,
                                                                                db, D, taps);
    return after_launch("conv_wgrad_split_kernel");
  }
  float *dz = tp.dY;  // dy is consumed element-wise in place
  const unsigned grid = (unsigned)(B * cdiv(T, kBwdTile));
  const unsigned threads = (unsigned)std::min(256, (int)cdiv(D, 32) * 32);
  conv_dz_kernel<<<grid, threads, 0, st>>>(in, w, bias, in_mask, out_mask, dy, dz, B, T, D, taps,
                                           dil);
  LNET_TRY(after_launch("conv_dz_kernel"));
  conv_dx_kernel<<<grid, threads, 0, st>>>(dz, w, in_mask, dx, B, T, D, taps, dil);
  LNET_TRY(after_launch("conv_dx_kernel"));
  if (taps != 5) {  // other kernel sizes: the generic column sums
    LNET_TRY(colsum(ColConvW{dz, in, in_mask, T, D, taps, dil}, bt, D * taps, tp.colpart, dw, st,
                    "colsum(conv w)"));
    return colsum(ColPlain{dz, D}, bt, D, tp.colpart, db, st, "colsum(conv b)");
  }
  const unsigned wg_grid = (unsigned)(B * cdiv(T, kWgTile));
  conv_wgrad_kernel<5><<<wg_grid, threads, 0, st>>>(dz, in, in_mask, tp.colpart, T, D, dil);
  LNET_TRY(after_launch("conv_wgrad_kernel"));
  LNET_TRY(colsum_finish(tp.colpart, (int)wg_grid, D * (taps + 1), tp.polesum, st));
  conv_wgrad_split_kernel<<<(unsigned)cdiv(D * (taps + 1), 256), 256, 0, st>>>(tp.polesum, dw, db,
                                                                              D, taps);
  return after_launch("conv_wgrad_split_kernel");
}

// The state gradient of one block's moments into tp.dS (overwritten).
static int moments_vjp(const TrainPlan &tp, const lnet_b200_alphabet_request *r,
                       const float *states, const float *dm, int64_t B, int64_t T, int M,
                       cudaStream_t st) {
  if (r->time_delta) {
    LNET_TRY(cuda_check(cudaMemsetAsync(tp.dS, 0, (size_t)B * T * 2 * M * sizeof(float), st),
                        "cudaMemsetAsync(dS)"));
    const int threads = std::min(128, (int)cdiv(M, 32) * 32);
    pt_moments_backward_kernel<<<dim3((unsigned)cdiv(T, kPtChunk), (unsigned)B), threads, 0,
                                 st>>>(states, tp.ts, r->time_delta, r->valid_mask, tp.ptcounts,
                                       dm, tp.dS, T, M);
    return after_launch("pt_moments_backward_kernel");
  }
  const unsigned mb_grid = (unsigned)(B * cdiv(T, kMbTile));
  const unsigned mb_threads = (unsigned)std::min(128, (int)cdiv(M, 32) * 32);
  moments_backward_kernel<<<mb_grid, mb_threads, 0, st>>>(states, dm, r->valid_mask, tp.counts,
                                                          tp.dS, B, T, M, 0);
  return after_launch("moments_backward_kernel");
}

// The conv + SiLU VJP of one block (physical-time when the request has dt).
static int conv_vjp(const TrainPlan &tp, const lnet_b200_alphabet_request *r, const float *in,
                    const float *w, const float *bias, const float *in_mask,
                    const float *out_mask, const float *dy, float *dx, float *dw, float *db,
                    int64_t B, int64_t T, int D, int taps, int dil, cudaStream_t st) {
  if (!r->time_delta)
    return conv_backward(tp, in, w, bias, in_mask, out_mask, dy, dx, dw, db, B, T, D, taps, dil,
                         st);
  if (taps > kPcTaps) return fail(LNET_ERR_UNSUPPORTED, "physical-time conv: more than 8 taps");
  LNET_TRY(cuda_check(cudaMemsetAsync(dx, 0, (size_t)B * T * D * sizeof(float), st),
                      "cudaMemsetAsync(dx)"));
  const unsigned grid = (unsigned)(B * cdiv(T, kCbTile));
  const unsigned threads = (unsigned)std::min(256, (int)cdiv(D, 32) * 32);
  pconv_backward_kernel<<<grid, threads, 0, st>>>(in, w, bias, in_mask, tp.ts, r->valid_mask,
                                                  out_mask, dy, dx, tp.colpart, T, D, taps, dil);
  LNET_TRY(after_launch("pconv_backward_kernel"));
  LNET_TRY(colsum_finish(tp.colpart, (int)grid, D * (taps + 1), tp.polesum, st));
  conv_wgrad_split_kernel<<<(unsigned)cdiv(D * (taps + 1), 256), 256, 0, st>>>(tp.polesum, dw, db,
                                                                              D, taps);
  return after_launch("conv_wgrad_split_kernel");
}

static int train_backward_impl(const lnet_b200_alphabet_params *p,
                               const lnet_b200_alphabet_request *r, TrainPlan &tp,
                               const float *dlogits, const lnet_b200_alphabet_grads *gd,
                               cudaStream_t st) {
  const int64_t B = r->batch, T = r->steps, bt = B * T;
  const int C = p->raw_input_dim, D = p->model_dim, M = p->modes, K = p->output_dim;
  const int taps = p->conv_kernel, dil = p->conv_dilation;
  const float *valid = r->valid_mask;
  const bool tf32 = r->act_dtype == LNET_BF16;  // as the training forward
  // head
  LNET_TRY(gemm_wgrad(st, dlogits, K, tp.feats, 14 * M, gd->head_weight, B, 0.f, false,
                      "gemm(d head)"));
  LNET_TRY(colsum(ColPlain{dlogits, K}, B, K, tp.colpart, gd->head_bias, st, "colsum(head b)"));
  LNET_TRY(gemm_rows(st, dlogits, CUDA_R_32F, K, p->head_weight, CUDA_R_32F, 1, 14 * M, tp.dfeats,
                     14 * M, B, 14 * M, K, false, "gemm(d feats)"));
  radial_backward_kernel<<<grid_for(2 * B * 7 * M), 256, 0, st>>>(tp.m1, tp.m2, tp.dfeats, tp.dm,
                                                                  B, M);
  LNET_TRY(after_launch("radial_backward_kernel"));
  if (r->time_delta) {
    pt_counts_kernel<<<(unsigned)B, 256, 0, st>>>(tp.ts, r->time_delta, valid, T, tp.ptcounts);
    LNET_TRY(after_launch("pt_counts_kernel"));
  } else if (valid) {
    moment_counts_kernel<<<(unsigned)B, 256, 0, st>>>(valid, T, tp.counts);
    LNET_TRY(after_launch("moment_counts_kernel"));
  }
  const float *dm1 = tp.dm, *dm2 = tp.dm + B * 7 * M;
  // reader block
  LNET_TRY(moments_vjp(tp, r, tp.s2, dm2, B, T, M, st));
  LNET_TRY(block_backward(tp, tp.s2, tp.xh2, p->reader_frame, p->reader_raw_decay,
                          p->reader_raw_frequency, tp.a_tab + 2 * M, tp.a_tab + 3 * M,
                          tp.a_tab + 6 * M, tp.a_tab + 7 * M, tp.dX, 0.f, gd->reader_frame, 0.f,
                          gd->reader_raw_decay, gd->reader_raw_frequency, B, T, D, M, tf32,
                          nullptr, 1, r->time_delta, st));
  LNET_TRY(rms_backward(tp.y2, tp.dX, p->reader_norm, nullptr, tp.dY, tp.rs, bt, D, st));
  LNET_TRY(colsum(ColRmsGamma{tp.dX, tp.y2, tp.rs, D}, bt, D, tp.colpart, gd->reader_norm, st,
                  "colsum(reader norm)"));
  // reader conv: input v (masked), dv out
  LNET_TRY(conv_vjp(tp, r, tp.v, p->reader_conv_weight, p->reader_conv_bias, valid, valid,
                    tp.dY, tp.dV, gd->reader_conv_weight, gd->reader_conv_bias, B, T, D, taps,
                    dil, st));
  // writer synthesis + residual: v = y1 + ls (s1 F^T + ds xh1)
  const float *ls = p->writer_layer_scale, *ds = p->writer_direct_scale;
  LNET_TRY(colsum(ColProd{tp.dV, tp.modal, tp.xh1, ls, ds, D, 0}, bt, D, tp.colpart,
                  gd->writer_layer_scale, st, "colsum(layer scale)"));
  LNET_TRY(colsum(ColProd{tp.dV, tp.modal, tp.xh1, ls, ds, D, 1}, bt, D, tp.colpart,
                  gd->writer_direct_scale, st, "colsum(direct scale)"));
  scale_rows_kernel<<<grid_for((int64_t)D * 2 * M), 256, 0, st>>>(p->writer_frame, ls, tp.wls, D,
                                                                   2 * M);
  LNET_TRY(after_launch("scale_rows_kernel"));
  // dS1 = moments VJP + dv (ls F) (the GEMM accumulates, beta = 1)
  LNET_TRY(moments_vjp(tp, r, tp.s1, dm1, B, T, M, st));
  LNET_TRY(gemm_rows(st, tp.dV, CUDA_R_32F, D, tp.wls, CUDA_R_32F, 1, 2 * M, tp.dS, 2 * M, bt,
                     2 * M, D, tf32, "gemm(d states synth)", /*beta=*/1.f));
  // dF1 = ls (dv^T s1) (+ the drive part below)
  LNET_TRY(gemm_wgrad(st, tp.dV, D, tp.s1, 2 * M, gd->writer_frame, bt, 0.f, tf32,
                      "gemm(d frame synth)"));
  scale_rows_kernel<<<grid_for((int64_t)D * 2 * M), 256, 0, st>>>(gd->writer_frame, ls,
                                                                   gd->writer_frame, D, 2 * M);
  LNET_TRY(after_launch("scale_rows_kernel"));
  residual_dxh_kernel<<<grid_for(bt * D), 256, 0, st>>>(tp.dV, ls, ds, tp.dX, bt, D);
  LNET_TRY(after_launch("residual_dxh_kernel"));
  LNET_TRY(block_backward(tp, tp.s1, tp.xh1, p->writer_frame, p->writer_raw_decay,
                          p->writer_raw_frequency, tp.a_tab, tp.a_tab + M, tp.a_tab + 4 * M,
                          tp.a_tab + 5 * M, tp.dX, 1.f, gd->writer_frame, 1.f,
                          gd->writer_raw_decay, gd->writer_raw_frequency, B, T, D, M, tf32,
                          r->observation_mask, r->obs_channels, r->time_delta, st));
  // writer RMSNorm: dy1 = rms VJP + dv (residual identity)
  LNET_TRY(rms_backward(tp.y1, tp.dX, p->writer_norm, tp.dV, tp.dY, tp.rs, bt, D, st));
  LNET_TRY(colsum(ColRmsGamma{tp.dX, tp.y1, tp.rs, D}, bt, D, tp.colpart, gd->writer_norm, st,
                  "colsum(writer norm)"));
  // stem conv: input proj (no input mask), output mask valid; dproj -> tp.dV
  LNET_TRY(conv_vjp(tp, r, tp.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr, valid,
                    tp.dY, tp.dV, gd->stem_conv_weight, gd->stem_conv_bias, B, T, D, taps, dil,
                    st));
  return gemm_wgrad(st, tp.dV, D, tp.x32, C, gd->stem_projection, bt, 0.f, tf32,
                    "gemm(d projection)");
}

static int train_entry(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                       void *ws, size_t ws_bytes, TrainPlan &tp) {
  LNET_TRY(check_params(p));
  LNET_TRY(check_request(p, r));
  if (!train_supported(r))
    return fail(LNET_ERR_UNSUPPORTED, "training path: time_delta is not supported");
  Arena ar(ws, ws_bytes);
  plan_train(ar, tp, p, r);
  if (!ws || !ar.ok())
    return fail(LNET_ERR_WORKSPACE, "training workspace of %zu bytes < required %zu", ws_bytes,
                ar.used);
  return LNET_OK;
}

}  // namespace lnet

extern "C" int lnet_b200_alphabet_train_workspace_size(const lnet_b200_alphabet_params *params,
                                                       const lnet_b200_alphabet_request *req,
                                                       size_t *bytes) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (!bytes) return fail(LNET_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  Arena a(nullptr, 0);
  TrainPlan tp;
  plan_train(a, tp, params, req);
  *bytes = a.used;
  return LNET_OK;
}

extern "C" int lnet_b200_alphabet_train_forward(const lnet_b200_alphabet_params *params,
                                                const lnet_b200_alphabet_request *req,
                                                void *workspace, size_t workspace_bytes,
                                                float *logits, lnet_stream_t stream) {
  reset_launches();
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  TrainPlan tp;
  LNET_TRY(train_entry(params, req, workspace, workspace_bytes, tp));
  if (!logits) return fail(LNET_ERR_INVALID_ARGUMENT, "logits must not be NULL");
  if (req->batch == 0 || req->steps == 0) return LNET_OK;
  if (req->x_dtype == LNET_BF16)
    return train_forward_impl<__nv_bfloat16>(params, req, tp, logits, st);
  return train_forward_impl<float>(params, req, tp, logits, st);
}

extern "C" int lnet_b200_alphabet_backward(const lnet_b200_alphabet_params *params,
                                           const lnet_b200_alphabet_request *req,
                                           void *workspace, size_t workspace_bytes,
                                           const float *dlogits,
                                           const lnet_b200_alphabet_grads *grads,
                                           lnet_stream_t stream) {
  reset_launches();
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  TrainPlan tp;
  LNET_TRY(train_entry(params, req, workspace, workspace_bytes, tp));
  if (!dlogits || !grads) return fail(LNET_ERR_INVALID_ARGUMENT, "NULL dlogits or grads");
  const float *const need[] = {grads->stem_projection, grads->stem_conv_weight,
                               grads->stem_conv_bias, grads->writer_norm, grads->writer_frame,
                               grads->writer_raw_decay, grads->writer_raw_frequency,
                               grads->writer_direct_scale, grads->writer_layer_scale,
                               grads->reader_conv_weight, grads->reader_conv_bias,
                               grads->reader_norm, grads->reader_frame, grads->reader_raw_decay,
                               grads->reader_raw_frequency, grads->head_weight, grads->head_bias};
  for (const float *q : need)
    if (!q) return fail(LNET_ERR_INVALID_ARGUMENT, "a gradient pointer is NULL");
  if (req->batch == 0 || req->steps == 0) return LNET_OK;
  return train_backward_impl(params, req, tp, dlogits, grads, st);
}
