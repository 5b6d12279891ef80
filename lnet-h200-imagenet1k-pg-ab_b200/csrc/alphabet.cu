// Orchestration of the ALPHABET forward path behind the lnet_b200 C ABI.
//
// Two routes share one workspace plan:
//   * the general route (generic_kernels.cuh): one stage kernel per
//     reference operation, used whenever time_delta is present and for the
//     stage-level entry points;
//   * the fused unit-grid route (fused_path.cuh): stem+writer and reader as
//     single chunked-scan kernels, used by lnet_b200_alphabet_forward when no
//     time_delta is given and the shape fits the fused kernels.
#include <algorithm>
#include <atomic>
#include <chrono>

#include <type_traits>

#include "blas.cuh"
#include "common.cuh"
#include "fused_path.cuh"
#include "generic_kernels.cuh"

namespace lnet {

constexpr int kScanChunk = 64;

// Host part of the look-back record tags (record_tag): one time-derived,
// nonzero value per process, mixed into every tag so that words left in reused
// device memory by another process or by other data do not read as records.
// The per-call part is the workspace's device counter, which only increases.
uint32_t process_tag_seed() {
  static const uint32_t seed = [] {
    const uint32_t s =
        (uint32_t)std::chrono::steady_clock::now().time_since_epoch().count() * 0x9E3779B1u;
    return s == 0u ? 0x2545F491u : s;
  }();
  return seed;
}

// One-shot test hook (lnet_b200_debug_inject_lookback_miss): the next fused
// forward's look-backs expect a tag no record carries and give up after a
// short bounded wait, which sets the look-back error bit.
static std::atomic<int> g_inject_miss{0};
int take_lookback_injection() { return g_inject_miss.exchange(0); }

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
    return 148;
  return n;
}
constexpr int kMomChunk = 64;
static_assert(kMomChunk == kScanChunk, "fused scan + moments partials share the chunking");

static int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), 148 * 32)); }
// Token-major elementwise kernels: blocks stride over tokens, threads over the
// channels of a token.
static unsigned token_grid(int64_t tokens) {
  // capped: one block per token measured slower (block scheduling) at 2^20 tokens
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(tokens, 148 * 64));
}
static unsigned dw_grid(int64_t batch, int64_t steps) {
  return (unsigned)(batch * cdiv(steps, kDwTile));  // rows x step tiles
}
static unsigned token_block(int width) { return (unsigned)std::min(256, std::max(32, (width + 31) / 32 * 32)); }

static dim3 carry_grid(int64_t batch, int modes) {
  return dim3((unsigned)cdiv(modes, 32), (unsigned)batch);
}

// Depthwise conv + SiLU over [B, T, D] fp32 (see dwconv_unit_kernel); the
// shared-memory tile kernel for the canonical K5 d4 geometry on aligned rows.
static int depthwise_conv(const float *in, const float *w, const float *bias,
                          const float *in_mask, const float *out_mask, float *out, int64_t B,
                          int64_t T, int D, int taps, int dilation, cudaStream_t st,
                          const char *what) {
  const bool quad = taps == 5 && dilation == 4 && D % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(bias) % 16 == 0;
  if (quad) {
    const dim3 grid((unsigned)(B * cdiv(T, kDwTileSteps)), (unsigned)cdiv(D, kDwTileChans));
    dwconv_tile_kernel<5, 4><<<grid, kDwTileThreads, 0, st>>>(in, w, bias, in_mask, out_mask, out,
                                                             T, D);
  } else {
    dwconv_unit_kernel<float><<<dw_grid(B, T), token_block(D), 0, st>>>(
        in, w, bias, in_mask, out_mask, out, B, T, D, taps, dilation);
  }
  return after_launch(what);
}


// ---------------------------------------------------------------- validation
static int check_params(const lnet_b200_alphabet_params *p) {
  if (!p) return fail(LNET_ERR_INVALID_ARGUMENT, "params must not be NULL");
  if (p->raw_input_dim < 1 || p->model_dim < 1 || p->modes < 1 || p->output_dim < 1)
    return fail(LNET_ERR_INVALID_ARGUMENT, "dimensions must be positive (C=%d D=%d M=%d K=%d)",
                p->raw_input_dim, p->model_dim, p->modes, p->output_dim);
  if (p->conv_kernel < 1 || p->conv_kernel > 16 || p->conv_dilation < 1)
    return fail(LNET_ERR_UNSUPPORTED, "conv kernel %d / dilation %d unsupported", p->conv_kernel,
                p->conv_dilation);
  if ((p->conv_dilation * (p->conv_kernel - 1)) % 2 != 0)
    return fail(LNET_ERR_UNSUPPORTED, "odd receptive span (same padding) is not supported");
  const void *need[] = {p->stem_projection, p->stem_conv_weight, p->stem_conv_bias,
                        p->writer_norm, p->writer_frame, p->writer_raw_decay,
                        p->writer_raw_frequency, p->writer_direct_scale, p->writer_layer_scale,
                        p->reader_conv_weight, p->reader_conv_bias, p->reader_norm,
                        p->reader_frame, p->reader_raw_decay, p->reader_raw_frequency,
                        p->head_weight, p->head_bias};
  for (const void *q : need)
    if (!q) return fail(LNET_ERR_INVALID_ARGUMENT, "a parameter pointer is NULL");
  return LNET_OK;
}

static int check_request(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r) {
  if (!r) return fail(LNET_ERR_INVALID_ARGUMENT, "request must not be NULL");
  if (r->batch < 0 || r->steps < 0) return fail(LNET_ERR_INVALID_ARGUMENT, "negative batch/steps");
  if (r->batch > 65535) return fail(LNET_ERR_UNSUPPORTED, "batch > 65535 per call");
  if (r->x_dtype != LNET_F32 && r->x_dtype != LNET_BF16)
    return fail(LNET_ERR_UNSUPPORTED, "x dtype must be float32 or bfloat16");
  if (r->act_dtype != LNET_F32 && r->act_dtype != LNET_BF16)
    return fail(LNET_ERR_UNSUPPORTED, "activation dtype must be float32 or bfloat16");
  if (r->batch > 0 && r->steps > 0 && !r->x) return fail(LNET_ERR_INVALID_ARGUMENT, "x is NULL");
  if (r->observation_mask && r->obs_channels != 1 && r->obs_channels != p->raw_input_dim)
    return fail(LNET_ERR_INVALID_ARGUMENT, "observation_mask channels must be 1 or C");
  return LNET_OK;
}

// ---------------------------------------------------------------- workspace plan
struct Plan {
  float *xm = nullptr;        // [BT, C]   masked raw input
  float *proj = nullptr;      // [BT, D]   projection / reader encoded
  float *first_local = nullptr;  // [BT, D]
  float *xhat = nullptr;      // [BT, D]
  float *drive = nullptr;     // [BT, 2M]  drive, then states
  float *stream = nullptr;    // [BT, D]   writer stream
  float *modal = nullptr;     // [BT, D]
  float *ts = nullptr;        // [BT]
  float *step_a = nullptr;    // [BT, 2M] per-step transitions (physical time only)
  float *carries = nullptr;   // [B, nchunk, kRecFloats, M] scan records
  float *partial = nullptr;   // moment partials
  float *wfold = nullptr;     // [D, 2M] drive frame with the ZOH gains folded in
  __nv_bfloat16 *wfold_bf16 = nullptr;  // the same in bf16 (bf16 drive GEMM)
  uint32_t *status = nullptr; // general-route device error bits (zeroed per forward)
  float *a_tab = nullptr;     // [8][M] a_re, a_im (writer, reader), then g_re, g_im (writer, reader)
  __nv_bfloat16 *w_bf16 = nullptr;  // [D, C] stem projection in bf16 (bf16 inputs)
  float *moments = nullptr;   // [2][B][7M]
  float *feats = nullptr;     // [B, 14M]
  float *head_partial = nullptr;  // split-K partial logits
  FusedWorkspace fused;       // fused-route scratch
};

static void plan_generic(Arena &ar, Plan &pl, const lnet_b200_alphabet_params *p,
                         const lnet_b200_alphabet_request *r) {
  const int64_t bt = r->batch * r->steps;
  const int D = p->model_dim, M = p->modes, C = p->raw_input_dim;
  const int64_t n_scan = cdiv(std::max<int64_t>(r->steps, 1), kScanChunk);
  const int64_t n_mom = cdiv(std::max<int64_t>(r->steps, 1), kMomChunk);
  pl.xm = ar.take<float>((size_t)bt * C);
  pl.proj = ar.take<float>((size_t)bt * D);
  pl.first_local = ar.take<float>((size_t)bt * D);
  pl.xhat = ar.take<float>((size_t)bt * D);
  pl.drive = ar.take<float>((size_t)bt * 2 * M);
  pl.stream = ar.take<float>((size_t)bt * D);
  pl.modal = ar.take<float>((size_t)bt * D);
  pl.ts = ar.take<float>((size_t)bt);
  if (r->time_delta) pl.step_a = ar.take<float>((size_t)bt * 2 * M);
  pl.carries = ar.take<float>((size_t)r->batch * n_scan * kRecFloats * M);
  pl.partial = ar.take<float>((size_t)r->batch * n_mom * (8 * M + 5));
  pl.wfold = ar.take<float>((size_t)D * 2 * M);
  pl.wfold_bf16 = ar.take<__nv_bfloat16>((size_t)D * 2 * M);
  pl.status = ar.take<uint32_t>(4);
  pl.a_tab = ar.take<float>((size_t)8 * M);
  pl.w_bf16 = ar.take<__nv_bfloat16>((size_t)D * C);
  pl.moments = ar.take<float>((size_t)2 * r->batch * 7 * M);
  pl.feats = ar.take<float>((size_t)r->batch * 14 * M);
  pl.head_partial = ar.take<float>(head_partial_floats(r->batch, p->output_dim));
}

// ---------------------------------------------------------------- general-route stages
// Stem projection x W^T -> pl.proj (inputs masked first when metadata asks).
// The shapes the conv + RMSNorm forward (forward_generic_normed) serves:
// step-indexed requests, canonical K5 d4 conv, 4 | D <= 256.  The slice entry
// points follow the same arithmetic for them.
static bool normed_route(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r) {
  const int D = p->model_dim;
  return !r->time_delta && p->conv_kernel == 5 && p->conv_dilation == 4 && D % 4 == 0 &&
         D <= 256;
}

// bf16 drive operands (xhat and the gain-folded frame in bf16) for bf16
// requests on that route without an event mask.
static bool half_drive(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r) {
  return normed_route(p, r) && r->act_dtype == LNET_BF16 && p->model_dim % 8 == 0 &&
         !r->observation_mask;
}

template <typename TX>
static int stem_projection(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                           Plan &pl, cudaStream_t st) {
  const int64_t bt = r->batch * r->steps;
  const int C = p->raw_input_dim, D = p->model_dim;
  const TX *x = (const TX *)r->x;
  const bool tf32 = r->act_dtype == LNET_BF16;
  if (r->observation_mask || r->valid_mask) {
    mask_inputs_kernel<TX><<<token_grid(bt), token_block(C), 0, st>>>(
        x, r->observation_mask, r->obs_channels, r->valid_mask, pl.xm, bt, C);
    LNET_TRY(after_launch("mask_inputs_kernel"));
    LNET_TRY(gemm_rows(st, pl.xm, CUDA_R_32F, C, p->stem_projection, CUDA_R_32F, C, 1, pl.proj, D,
                       bt, D, C, tf32, "gemm(stem)"));
  } else if (std::is_same<TX, float>::value) {
    LNET_TRY(gemm_rows(st, x, CUDA_R_32F, C, p->stem_projection, CUDA_R_32F, C, 1, pl.proj, D, bt,
                       D, C, tf32, "gemm(stem)"));
  } else {  // bf16 x: bf16 x bf16 -> fp32 (the weights rounded to bf16, as under autocast)
    to_bf16_kernel<<<grid_for((int64_t)D * C), 256, 0, st>>>(p->stem_projection, pl.w_bf16,
                                                             (int64_t)D * C);
    LNET_TRY(after_launch("to_bf16_kernel"));
    LNET_TRY(gemm_rows(st, x, CUDA_R_16BF, C, pl.w_bf16, CUDA_R_16BF, C, 1, pl.proj, D, bt, D, C,
                       false, "gemm(stem)"));
  }
  return LNET_OK;
}

// Physical-time depthwise conv of fp32 rows: the tiled kernel where the rows
// allow it (4 | dim, 16-byte aligned, at most kPtMaxTaps taps), else the
// per-token kernel.
static int physical_conv(const float *in, const float *w, const float *bias, const float *in_mask,
                         const float *ts, const float *valid, float *out, int64_t B, int64_t T,
                         int D, int taps, int dilation, cudaStream_t st, const char *what) {
  auto al = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (D % 4 == 0 && al(in) && al(out) && taps <= kPtMaxTaps && T <= INT32_MAX) {
    const dim3 grid((unsigned)cdiv(T, kPtTile), (unsigned)B);
    const size_t sm = (size_t)(taps + 1) * D * sizeof(float);
    dwconv_physical_tile_kernel<<<grid, kPtThreads, sm, st>>>(in, w, bias, in_mask, ts, valid, out,
                                                             T, D, taps, dilation);
    return after_launch(what);
  }
  dwconv_physical_kernel<float><<<(unsigned)(B * T), token_block(D), 0, st>>>(
      in, w, bias, in_mask, ts, valid, out, T, D, taps, dilation);
  return after_launch(what);
}

static int timestamps(const float *dt, float *ts, int64_t B, int64_t T, cudaStream_t st) {
  timestamps_scan_kernel<<<(unsigned)B, kTsThreads, 0, st>>>(dt, ts, T);
  return after_launch("timestamps_scan_kernel");
}

template <typename TX>
static int stem_generic(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                        Plan &pl, float *first_local, cudaStream_t st) {
  const int64_t B = r->batch, T = r->steps, bt = B * T;
  const int D = p->model_dim;
  LNET_TRY(stem_projection<TX>(p, r, pl, st));
  if (r->time_delta) {
    LNET_TRY(timestamps(r->time_delta, pl.ts, B, T, st));
    return physical_conv(pl.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr, pl.ts,
                         r->valid_mask, first_local, B, T, D, p->conv_kernel, p->conv_dilation,
                         st, "dwconv_physical(stem)");
  }
  return depthwise_conv(pl.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr, r->valid_mask,
                        first_local, B, T, D, p->conv_kernel, p->conv_dilation, st,
                        "depthwise_conv(stem)");
}

// RMSNorm of [tokens, D] fp32 rows: the float4 kernel where the rows allow it.
static int rmsnorm(const float *in, const float *g, float *out, int64_t tokens, int D,
                   cudaStream_t st) {
  auto al = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  const int quads = D / 4;
  const bool pow2 = quads > 0 && (quads & (quads - 1)) == 0;
  if (D % 4 == 0 && quads > 0 && al(in) && al(g) && al(out)) {
    const int per_warp = quads < 32 && pow2 ? 32 / quads : 1;
    rmsnorm4_kernel<<<(unsigned)cdiv(tokens, 8 * per_warp), 256, 0, st>>>(
        reinterpret_cast<const float4 *>(in), reinterpret_cast<const float4 *>(g),
        reinterpret_cast<float4 *>(out), tokens, quads);
    return after_launch("rmsnorm_kernel");
  }
  rmsnorm_kernel<<<(unsigned)cdiv(tokens, 8), 256, 0, st>>>(in, g, out, tokens, D);
  return after_launch("rmsnorm_kernel");
}

// Block body shared by writer and reader: RMSNorm -> drive -> ZOH gamma -> scan -> moments.
// `write_states`: leave the states in pl.drive (the writer's synthesis reads them).
// `normed`: pl.xhat already holds RMSNorm(in); `xhat_bf16`: in bf16 (static
// poles and no event mask only: the drive GEMM then runs bf16 x bf16).
static int block_scan_moments(const float *in, const float *norm, const float *frame,
                              const float *raw_decay, const float *raw_freq, float *a_re,
                              float *a_im, float *g_re, float *g_im, const float *event_mask,
                              int obs_channels,
                              const lnet_b200_alphabet_request *r, int D, int M, Plan &pl,
                              float *moments, bool write_states, cudaStream_t st,
                              bool normed = false, bool xhat_bf16 = false) {
  const int64_t B = r->batch, T = r->steps, bt = B * T;
  const bool tf32 = r->act_dtype == LNET_BF16;
  if (!normed) {  // else pl.xhat holds RMSNorm(in) already (conv_norm)
    LNET_TRY(rmsnorm(in, norm, pl.xhat, bt, D, st));
  }
  if (!r->time_delta) {  // per-mode a and gamma tables (static poles)
    zoh_kernel<<<1, 128, 0, st>>>(raw_decay, raw_freq, M, nullptr, 1, a_re, a_im, g_re, g_im);
    LNET_TRY(after_launch("zoh_kernel"));
  }
  if (!r->time_delta && !event_mask) {
    // u = g (x^ W) in one GEMM over the gain-folded frame
    fold_gain_kernel<<<grid_for((int64_t)D * M), 256, 0, st>>>(
        frame, g_re, g_im, pl.wfold, xhat_bf16 ? pl.wfold_bf16 : nullptr, D, M);
    LNET_TRY(after_launch("fold_gain_kernel"));
    if (xhat_bf16)  // bf16 x bf16 tensor-core GEMM, fp32 accumulation
      LNET_TRY(gemm_rows(st, pl.xhat, CUDA_R_16BF, D, pl.wfold_bf16, CUDA_R_16BF, 1, 2 * M,
                         pl.drive, 2 * M, bt, 2 * M, D, false, "gemm(drive)"));
    else
      LNET_TRY(gemm_rows(st, pl.xhat, CUDA_R_32F, D, pl.wfold, CUDA_R_32F, 1, 2 * M, pl.drive,
                         2 * M, bt, 2 * M, D, tf32, "gemm(drive)"));
  } else {
    LNET_TRY(gemm_rows(st, pl.xhat, CUDA_R_32F, D, frame, CUDA_R_32F, 1, 2 * M, pl.drive, 2 * M,
                       bt, 2 * M, D, tf32, "gemm(drive)"));
    const unsigned mx = (unsigned)std::min(256, (int)cdiv(M, 32) * 32);
    drive_kernel<<<(unsigned)cdiv(bt, kDriveTokens), dim3(mx, 256 / mx), 0, st>>>(pl.drive, raw_decay, raw_freq,
                                                            r->time_delta, g_re, g_im, event_mask,
                                                            obs_channels, bt, M, pl.step_a);
    LNET_TRY(after_launch("drive_kernel"));
  }
  const int64_t n_scan = cdiv(T, kScanChunk);
  const int threads = std::min(128, (int)cdiv(M, 32) * 32);
  dim3 gs((unsigned)n_scan, (unsigned)B);
  scan_local_kernel<<<gs, threads, 0, st>>>(pl.drive, raw_decay, raw_freq, a_re, a_im,
                                            r->time_delta, pl.step_a, pl.carries, T, M, kScanChunk, n_scan);
  LNET_TRY(after_launch("scan_local_kernel"));
  scan_carry_kernel<<<carry_grid(B, M), 32 * kCarryParts, 0, st>>>(pl.carries, B, M, n_scan,
                                                                nullptr);
  LNET_TRY(after_launch("scan_carry_kernel"));
  if (!r->time_delta) {
    if (write_states)
      scan_apply_moments_kernel<true><<<gs, threads, 0, st>>>(
          pl.drive, a_re, a_im, pl.carries, r->valid_mask, pl.partial, T, M, kScanChunk, n_scan);
    else
      scan_apply_moments_kernel<false><<<gs, threads, 0, st>>>(
          pl.drive, a_re, a_im, pl.carries, r->valid_mask, pl.partial, T, M, kScanChunk, n_scan);
    LNET_TRY(after_launch("scan_apply_moments_kernel"));
    const dim3 gf((unsigned)cdiv(7 * M, 32), (unsigned)B);
    moments_finalize_kernel<<<gf, 32 * kFinalParts, 0, st>>>(pl.partial, r->valid_mask, moments,
                                                            T, M, n_scan);
    return after_launch("moments_finalize_kernel");
  }
  scan_apply_kernel<<<gs, threads, 0, st>>>(pl.drive, raw_decay, raw_freq, a_re, a_im,
                                            r->time_delta, pl.step_a, pl.carries, T, M, kScanChunk, n_scan);
  LNET_TRY(after_launch("scan_apply_kernel"));
  const int64_t n_mom = cdiv(T, kMomChunk);
  dim3 gm((unsigned)n_mom, (unsigned)B);
  pt_moments_partial_kernel<<<gm, 256, 0, st>>>(pl.drive, pl.ts, r->time_delta,
                                                    r->valid_mask, pl.partial, T, M, n_mom);
  LNET_TRY(after_launch("pt_moments_partial_kernel"));
  pt_moments_finalize_kernel<<<dim3((unsigned)cdiv(M, 32), (unsigned)B), 32 * kPtFinalParts, 0,
                               st>>>(pl.partial, moments, M, n_mom);
  return after_launch("pt_moments_finalize_kernel");
}

// Whether the conv + RMSNorm kernel applies (canonical K5 d4 conv on aligned
// fp32 rows, 4 | D <= 256, step-indexed convs).
static bool conv_norm_ok(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                         const Plan &pl) {
  auto al = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  return normed_route(p, r) && al(pl.proj) && al(pl.stream) && al(pl.xhat) &&
         al(p->stem_conv_bias) && al(p->reader_conv_bias) && al(p->writer_norm) &&
         al(p->reader_norm) && al(p->writer_layer_scale) && al(p->writer_direct_scale);
}

template <typename TIN, typename TXH>
static int conv_norm(const TIN *in, const float *w, const float *bias, const float *in_mask,
                     const float *out_mask, const float *g, const float *ls, const float *ds,
                     TXH *xhat, float *base, uint32_t *status, int64_t B, int64_t T, int D,
                     cudaStream_t st, const char *what) {
  constexpr int rows = kDnSteps + 16;
  static_assert(kDnParts <= 32 && kDnSteps * kDnParts == kDnThreads, "reduction layout");
  const size_t smem = dwconv_norm_smem(rows, D / 4, sizeof(TIN));
  auto kernel = dwconv_norm_kernel<5, 4, TIN, TXH>;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device, per instantiation
  int dev = 0;
  LNET_TRY(cuda_check(cudaGetDevice(&dev), "cudaGetDevice"));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    LNET_TRY(cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)dwconv_norm_smem(rows, 64, sizeof(TIN))),
                        "cudaFuncSetAttribute(dwconv_norm_kernel)"));
    attr_set.fetch_or(bit);
  }
  const int64_t tiles = B * cdiv(T, kDnSteps);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, (int64_t)sm_count() * kDnBlocksPerSM);
  kernel<<<grid, kDnThreads, smem, st>>>(in, w, bias, in_mask, out_mask, g, ls, ds, xhat, base,
                                         nullptr, B, T, D, status);
  return after_launch(what);
}

// The whole general route with the conv + RMSNorm kernel (conv_norm_ok): the
// stem conv writes xhat and the writer's residual base straight into the
// stream buffer, the synthesis GEMM accumulates ls (s W^T) onto it (beta = 1,
// ls folded into the frame rows), and the reader conv writes its xhat only.
template <typename TX>
static int forward_generic_normed(const lnet_b200_alphabet_params *p,
                                  const lnet_b200_alphabet_request *r, Plan &pl, float *wm,
                                  float *rm, cudaStream_t st) {
  const int64_t B = r->batch, T = r->steps, bt = B * T;
  const int D = p->model_dim, M = p->modes;
  const bool tf32 = r->act_dtype == LNET_BF16;
  // bf16 requests: xhat in bf16 and the drive GEMMs bf16 x bf16 with fp32
  // accumulation (the operand precision of the fused route); the projection,
  // the stream and the states stay fp32 (the time-split pieces compute the
  // same arithmetic: lnet_b200_block_drive rounds xhat the same way).
  const bool half = half_drive(p, r);
  LNET_TRY(stem_projection<TX>(p, r, pl, st));
  const float *ls = p->writer_layer_scale, *ds = p->writer_direct_scale;
  __nv_bfloat16 *xh16 = reinterpret_cast<__nv_bfloat16 *>(pl.xhat);
  if (half)
    LNET_TRY(conv_norm((const float *)pl.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr,
                       r->valid_mask, p->writer_norm, ls, ds, xh16, pl.stream, pl.status, B, T,
                       D, st, "conv_norm(stem)"));
  else
    LNET_TRY(conv_norm((const float *)pl.proj, p->stem_conv_weight, p->stem_conv_bias, nullptr,
                       r->valid_mask, p->writer_norm, ls, ds, pl.xhat, pl.stream, pl.status, B,
                       T, D, st, "conv_norm(stem)"));
  LNET_TRY(block_scan_moments(nullptr, p->writer_norm, p->writer_frame, p->writer_raw_decay,
                              p->writer_raw_frequency, pl.a_tab, pl.a_tab + M,
                              pl.a_tab + 4 * M, pl.a_tab + 5 * M, r->observation_mask,
                              r->obs_channels, r, D, M, pl, wm, /*write_states=*/true, st,
                              /*normed=*/true, /*xhat_bf16=*/half));
  scale_rows_kernel<<<grid_for((int64_t)D * 2 * M), 256, 0, st>>>(
      p->writer_frame, p->writer_layer_scale, pl.wfold, D, 2 * M);
  LNET_TRY(after_launch("scale_rows_kernel"));
  LNET_TRY(gemm_rows(st, pl.drive, CUDA_R_32F, 2 * M, pl.wfold, CUDA_R_32F, 2 * M, 1, pl.stream,
                     D, bt, D, 2 * M, tf32, "gemm(synthesis)", /*beta=*/1.f));
  if (half)
    LNET_TRY(conv_norm((const float *)pl.stream, p->reader_conv_weight, p->reader_conv_bias,
                       r->valid_mask, r->valid_mask, p->reader_norm, nullptr, nullptr, xh16,
                       nullptr, pl.status, B, T, D, st, "conv_norm(reader)"));
  else
    LNET_TRY(conv_norm((const float *)pl.stream, p->reader_conv_weight, p->reader_conv_bias,
                       r->valid_mask, r->valid_mask, p->reader_norm, nullptr, nullptr, pl.xhat,
                       nullptr, pl.status, B, T, D, st, "conv_norm(reader)"));
  return block_scan_moments(nullptr, p->reader_norm, p->reader_frame, p->reader_raw_decay,
                            p->reader_raw_frequency, pl.a_tab + 2 * M, pl.a_tab + 3 * M,
                            pl.a_tab + 6 * M, pl.a_tab + 7 * M, nullptr, 1, r, D, M, pl, rm,
                            /*write_states=*/false, st, /*normed=*/true, /*xhat_bf16=*/half);
}

static int writer_generic(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                          const float *first_local, Plan &pl, float *stream_out, float *moments,
                          cudaStream_t st) {
  const int64_t bt = r->batch * r->steps;
  const int D = p->model_dim, M = p->modes;
  LNET_TRY(block_scan_moments(first_local, p->writer_norm, p->writer_frame, p->writer_raw_decay,
                              p->writer_raw_frequency, pl.a_tab, pl.a_tab + M,
                              pl.a_tab + 4 * M, pl.a_tab + 5 * M,
                              r->observation_mask, r->obs_channels, r, D, M, pl, moments,
                              /*write_states=*/true, st));
  LNET_TRY(gemm_rows(st, pl.drive, CUDA_R_32F, 2 * M, p->writer_frame, CUDA_R_32F, 2 * M, 1,
                     pl.modal, D, bt, D, 2 * M, r->act_dtype == LNET_BF16, "gemm(synthesis)"));
  residual_kernel<<<token_grid(bt), token_block(D), 0, st>>>(first_local, pl.xhat, pl.modal,
                                                     p->writer_direct_scale,
                                                     p->writer_layer_scale, stream_out, bt, D);
  return after_launch("residual_kernel");
}

// `ts_ready`: pl.ts already holds this request's timestamps (whole forward).
static int reader_generic(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                          const float *first_stream, Plan &pl, float *moments, cudaStream_t st,
                          bool ts_ready = false) {
  const int64_t B = r->batch, T = r->steps, bt = B * T;
  const int D = p->model_dim, M = p->modes;
  if (r->time_delta) {
    if (!pl.ts) return fail(LNET_ERR_INVALID_ARGUMENT, "timestamps missing");
    if (!ts_ready) LNET_TRY(timestamps(r->time_delta, pl.ts, B, T, st));
    LNET_TRY(physical_conv(first_stream, p->reader_conv_weight, p->reader_conv_bias,
                           r->valid_mask, pl.ts, r->valid_mask, pl.proj, B, T, D, p->conv_kernel,
                           p->conv_dilation, st, "dwconv_physical(reader)"));
  } else {
    LNET_TRY(depthwise_conv(first_stream, p->reader_conv_weight, p->reader_conv_bias,
                            r->valid_mask, r->valid_mask, pl.proj, B, T, D, p->conv_kernel,
                            p->conv_dilation, st, "depthwise_conv(reader)"));
  }
  // the reader block sees no observation mask (src/lnet/alphabet.py:384-389)
  return block_scan_moments(pl.proj, p->reader_norm, p->reader_frame, p->reader_raw_decay,
                            p->reader_raw_frequency, pl.a_tab + 2 * M, pl.a_tab + 3 * M,
                            pl.a_tab + 6 * M, pl.a_tab + 7 * M, nullptr,
                            1, r, D, M, pl, moments, /*write_states=*/false, st);
}

static int head_run(const lnet_b200_alphabet_params *p, int64_t B, const float *wm,
                    const float *rm, float *feats, float *partial, float *logits,
                    cudaStream_t st, const uint32_t *status) {
  const int M = p->modes;
  head_features_kernel<<<grid_for(B * 14 * M), 256, 0, st>>>(wm, rm, feats, B, M);
  LNET_TRY(after_launch("head_features_kernel"));
  return head_gemm(feats, B, 14 * M, p->head_weight, p->head_bias, logits, p->output_dim, partial,
                   st, status);
}

static int plan_all(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                    void *ws, size_t ws_bytes, Plan &pl, bool fused) {
  Arena measure(nullptr, 0);
  Plan dummy;
  if (fused)
    plan_fused(measure, dummy.fused, p, r);
  else
    plan_generic(measure, dummy, p, r);
  if (ws_bytes < measure.used || !ws)
    return fail(LNET_ERR_WORKSPACE, "workspace of %zu bytes < required %zu", ws_bytes,
                measure.used);
  Arena ar(ws, ws_bytes);
  if (fused)
    plan_fused(ar, pl.fused, p, r);
  else
    plan_generic(ar, pl, p, r);
  return LNET_OK;
}

static int g_route = 0;  // 0 = automatic, 1 = general route only

static bool use_fused(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r) {
  return g_route == 0 && !r->time_delta && fused_supported(p, r);
}

}  // namespace lnet

using namespace lnet;

extern "C" int lnet_b200_debug_inject_lookback_miss(void) {
  g_inject_miss.store(1);
  return LNET_OK;
}

extern "C" int lnet_b200_set_gemm_backend(int backend) {
  if (backend != 0 && backend != 1)
    return fail(LNET_ERR_INVALID_ARGUMENT, "gemm backend must be 0 or 1");
  rowgemm_enabled() = backend == 0;
  return LNET_OK;
}

extern "C" int lnet_b200_set_route(int route) {
  if (route != 0 && route != 1) return fail(LNET_ERR_INVALID_ARGUMENT, "route must be 0 or 1");
  g_route = route;
  return LNET_OK;
}

extern "C" int lnet_b200_alphabet_route(const lnet_b200_alphabet_params *params,
                                        const lnet_b200_alphabet_request *req) {
  if (check_params(params) != LNET_OK || check_request(params, req) != LNET_OK) return -1;
  return use_fused(params, req) ? 0 : 1;
}

extern "C" int lnet_b200_alphabet_device_status(const lnet_b200_alphabet_params *params,
                                                const lnet_b200_alphabet_request *req,
                                                const void *workspace, size_t workspace_bytes,
                                                uint32_t *status) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (!status) return fail(LNET_ERR_INVALID_ARGUMENT, "status must not be NULL");
  *status = 0;
  if (req->batch == 0 || req->steps == 0) return LNET_OK;
  const bool fused = use_fused(params, req);
  Plan pl;
  LNET_TRY(plan_all(params, req, const_cast<void *>(workspace), workspace_bytes, pl, fused));
  const uint32_t *err = fused ? pl.fused.flags + 2 : pl.status;
  return cuda_check(cudaMemcpy(status, err, sizeof(uint32_t), cudaMemcpyDeviceToHost),
                    "cudaMemcpy(device status)");
}

extern "C" int lnet_b200_alphabet_workspace_size(const lnet_b200_alphabet_params *params,
                                                 const lnet_b200_alphabet_request *req,
                                                 size_t *bytes) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (!bytes) return fail(LNET_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  Arena a(nullptr, 0), b(nullptr, 0);
  Plan pa, pb;
  plan_generic(a, pa, params, req);
  size_t need = a.used;
  if (use_fused(params, req)) {
    plan_fused(b, pb.fused, params, req);
    need = std::max(need, b.used);
  }
  *bytes = need;
  return LNET_OK;
}

static int alphabet_forward_impl(const lnet_b200_alphabet_params *params,
                                 const lnet_b200_alphabet_request *req, void *workspace,
                                 size_t workspace_bytes, float *logits, float *writer_moments,
                                 float *reader_moments, bool prepared, lnet_stream_t stream,
                                 const int64_t *lengths = nullptr,
                                 const ImageInput *img = nullptr) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (req->batch == 0) return LNET_OK;
  if (req->steps == 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "sequences must contain at least one step");
  if (!logits) return fail(LNET_ERR_INVALID_ARGUMENT, "logits is NULL");
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  const int64_t B = req->batch;
  const int M = params->modes;
  Plan pl;
  if (use_fused(params, req)) {
    LNET_TRY(plan_all(params, req, workspace, workspace_bytes, pl, true));
    float *wm = writer_moments ? writer_moments : pl.fused.moments;
    float *rm = reader_moments ? reader_moments : pl.fused.moments + B * 7 * M;
    LNET_TRY(fused_forward(params, req, pl.fused, wm, rm, prepared, lengths, st, img));
    return head_gemm(pl.fused.feats, B, 14 * M, params->head_weight, params->head_bias, logits,
                     params->output_dim, pl.fused.head_partial, st, pl.fused.flags + 2);
  }
  if (img) return fail(LNET_ERR_UNSUPPORTED, "image input is served by the fused route only");
  LNET_TRY(plan_all(params, req, workspace, workspace_bytes, pl, false));
  float *wm = writer_moments ? writer_moments : pl.moments;
  float *rm = reader_moments ? reader_moments : pl.moments + B * 7 * M;
  LNET_TRY(cuda_check(cudaMemsetAsync(pl.status, 0, sizeof(uint32_t), st), "cudaMemsetAsync"));
  if (conv_norm_ok(params, req, pl)) {
    if (req->x_dtype == LNET_BF16)
      LNET_TRY(forward_generic_normed<__nv_bfloat16>(params, req, pl, wm, rm, st));
    else
      LNET_TRY(forward_generic_normed<float>(params, req, pl, wm, rm, st));
    return head_run(params, B, wm, rm, pl.feats, pl.head_partial, logits, st, pl.status);
  }
  if (req->x_dtype == LNET_BF16)
    LNET_TRY(stem_generic<__nv_bfloat16>(params, req, pl, pl.first_local, st));
  else
    LNET_TRY(stem_generic<float>(params, req, pl, pl.first_local, st));
  LNET_TRY(writer_generic(params, req, pl.first_local, pl, pl.stream, wm, st));
  LNET_TRY(reader_generic(params, req, pl.stream, pl, rm, st, /*ts_ready=*/true));
  return head_run(params, B, wm, rm, pl.feats, pl.head_partial, logits, st, pl.status);
}

extern "C" int lnet_b200_alphabet_forward(const lnet_b200_alphabet_params *params,
                                          const lnet_b200_alphabet_request *req, void *workspace,
                                          size_t workspace_bytes, float *logits,
                                          float *writer_moments, float *reader_moments,
                                          lnet_stream_t stream) {
  return alphabet_forward_impl(params, req, workspace, workspace_bytes, logits, writer_moments,
                               reader_moments, false, stream);
}

extern "C" int lnet_b200_alphabet_forward_lengths(const lnet_b200_alphabet_params *params,
                                                  const lnet_b200_alphabet_request *req,
                                                  const int64_t *lengths, int32_t prepared,
                                                  void *workspace, size_t workspace_bytes,
                                                  float *logits, float *writer_moments,
                                                  float *reader_moments, lnet_stream_t stream) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (!lengths) return fail(LNET_ERR_INVALID_ARGUMENT, "lengths is NULL");
  if (req->time_delta || req->valid_mask)
    return fail(LNET_ERR_INVALID_ARGUMENT,
                "forward_lengths: the lengths replace the valid mask; pass no time_delta");
  if (req->batch > 0 && req->steps > 0 && !use_fused(params, req))
    return fail(LNET_ERR_UNSUPPORTED,
                "forward_lengths: this request does not take the fused route; pass the valid "
                "mask to lnet_b200_alphabet_forward");
  return alphabet_forward_impl(params, req, workspace, workspace_bytes, logits, writer_moments,
                               reader_moments, prepared != 0, stream, lengths);
}

// The request an image forward stands for: tokens [B, (H/4)(W/4), 48] in bf16.
static lnet_b200_alphabet_request image_request(const uint8_t *images, int64_t batch,
                                                int32_t height, int32_t width) {
  lnet_b200_alphabet_request r{};
  r.batch = batch;
  r.steps = (int64_t)(height / 4) * (width / 4);
  r.x_dtype = LNET_BF16;
  r.act_dtype = LNET_BF16;
  r.x = images;
  return r;
}

extern "C" int lnet_b200_alphabet_images_workspace_size(const lnet_b200_alphabet_params *params,
                                                        int64_t batch, int32_t height,
                                                        int32_t width, size_t *bytes) {
  if (batch < 0 || height < 4 || width < 4 || height % 4 != 0 || width % 4 != 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "images_workspace_size: invalid image shape");
  // any aligned non-null pointer stands for the images
  const lnet_b200_alphabet_request rq =
      image_request(reinterpret_cast<const uint8_t *>(uintptr_t(256)), batch, height, width);
  return lnet_b200_alphabet_workspace_size(params, &rq, bytes);
}

extern "C" int lnet_b200_alphabet_forward_images(
    const lnet_b200_alphabet_params *params, const uint8_t *images, int64_t batch,
    int32_t height, int32_t width, const float *mean, const float *std, int32_t prepared,
    void *workspace, size_t workspace_bytes, float *logits, float *writer_moments,
    float *reader_moments, lnet_stream_t stream) {
  reset_launches();
  LNET_TRY(check_params(params));
  if (batch < 0 || height < 4 || width < 4 || height % 4 != 0 || width % 4 != 0)
    return fail(LNET_ERR_INVALID_ARGUMENT,
                "forward_images: images must be [B, H, W, 3] with H, W positive multiples of 4 "
                "(got B=%lld, H=%d, W=%d)", (long long)batch, height, width);
  if (!images || !mean || !std) return fail(LNET_ERR_INVALID_ARGUMENT, "forward_images: NULL pointer");
  if (reinterpret_cast<uintptr_t>(images) % 16 != 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "forward_images: images must be 16-byte aligned");
  ImageInput img{images, height, width, {}, {}};
  for (int c = 0; c < 3; ++c) {
    if (!(std[c] != 0.f)) return fail(LNET_ERR_INVALID_ARGUMENT, "forward_images: std must be nonzero");
    img.mean[c] = mean[c];
    img.std[c] = std[c];
  }
  const lnet_b200_alphabet_request r = image_request(images, batch, height, width);
  LNET_TRY(check_request(params, &r));
  if (batch > 0 && !use_fused(params, &r))
    return fail(LNET_ERR_UNSUPPORTED,
                "forward_images: these parameters do not take the fused route (48 raw channels "
                "and a compiled shape are needed); patchify with lnet_b200_patchify_images and "
                "call lnet_b200_alphabet_forward");
  return alphabet_forward_impl(params, &r, workspace, workspace_bytes, logits, writer_moments,
                               reader_moments, prepared != 0, stream, nullptr, &img);
}

extern "C" int lnet_b200_alphabet_prepare(const lnet_b200_alphabet_params *params,
                                          const lnet_b200_alphabet_request *req, void *workspace,
                                          size_t workspace_bytes, lnet_stream_t stream) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  if (req->batch == 0 || req->steps == 0 || !use_fused(params, req)) return LNET_OK;
  Plan pl;
  LNET_TRY(plan_all(params, req, workspace, workspace_bytes, pl, true));
  return fused_prepare(params, pl.fused, st);
}

extern "C" int lnet_b200_alphabet_forward_prepared(const lnet_b200_alphabet_params *params,
                                                   const lnet_b200_alphabet_request *req,
                                                   void *workspace, size_t workspace_bytes,
                                                   float *logits, float *writer_moments,
                                                   float *reader_moments, lnet_stream_t stream) {
  return alphabet_forward_impl(params, req, workspace, workspace_bytes, logits, writer_moments,
                               reader_moments, true, stream);
}

extern "C" int lnet_b200_stem(const lnet_b200_alphabet_params *params,
                              const lnet_b200_alphabet_request *req, void *workspace,
                              size_t workspace_bytes, float *first_local, lnet_stream_t stream) {
  reset_launches();
  begin_entry((cudaStream_t)stream);
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (req->batch == 0 || req->steps == 0) return LNET_OK;
  Plan pl;
  LNET_TRY(plan_all(params, req, workspace, workspace_bytes, pl, false));
  if (req->x_dtype == LNET_BF16)
    return stem_generic<__nv_bfloat16>(params, req, pl, first_local, (cudaStream_t)stream);
  return stem_generic<float>(params, req, pl, first_local, (cudaStream_t)stream);
}

extern "C" int lnet_b200_writer(const lnet_b200_alphabet_params *params,
                                const lnet_b200_alphabet_request *req, const float *first_local,
                                void *workspace, size_t workspace_bytes, float *stream_out,
                                float *moments, lnet_stream_t stream) {
  reset_launches();
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (req->batch == 0 || req->steps == 0) return LNET_OK;
  Plan pl;
  LNET_TRY(plan_all(params, req, workspace, workspace_bytes, pl, false));
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  if (req->time_delta) {
    LNET_TRY(timestamps(req->time_delta, pl.ts, req->batch, req->steps, st));
  }
  return writer_generic(params, req, first_local, pl, stream_out, moments, st);
}

extern "C" int lnet_b200_reader(const lnet_b200_alphabet_params *params,
                                const lnet_b200_alphabet_request *req, const float *first_stream,
                                void *workspace, size_t workspace_bytes, float *moments,
                                lnet_stream_t stream) {
  reset_launches();
  begin_entry((cudaStream_t)stream);
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (req->batch == 0 || req->steps == 0) return LNET_OK;
  Plan pl;
  LNET_TRY(plan_all(params, req, workspace, workspace_bytes, pl, false));
  return reader_generic(params, req, first_stream, pl, moments, (cudaStream_t)stream);
}

extern "C" int lnet_b200_head(const lnet_b200_alphabet_params *params, int64_t batch,
                              const float *writer_moments, const float *reader_moments,
                              float *logits, lnet_stream_t stream) {
  reset_launches();
  begin_entry((cudaStream_t)stream);
  LNET_TRY(check_params(params));
  if (batch <= 0) return LNET_OK;
  if (!writer_moments || !reader_moments || !logits)
    return fail(LNET_ERR_INVALID_ARGUMENT, "head: NULL tensor pointer");
  return fused_head(params, batch, writer_moments, reader_moments, logits, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- time-split pieces
// One rank's slice of steps of every row (lnet_b200.timesplit): the pieces of
// the general route with the slice's carry-in and lag history exposed.  No
// metadata (static poles); tensors are fp32 [B, Ts, *] for req->batch rows of
// req->steps = Ts steps; `workspace` is sized by lnet_b200_alphabet_workspace_size
// for the same request.
static int slice_entry(const lnet_b200_alphabet_params *params,
                       const lnet_b200_alphabet_request *req, void *workspace,
                       size_t workspace_bytes, Plan &pl, cudaStream_t st) {
  reset_launches();
  begin_entry(st);
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (req->time_delta || req->observation_mask || req->valid_mask)
    return fail(LNET_ERR_UNSUPPORTED, "time-split pieces take no metadata");
  return plan_all(params, req, workspace, workspace_bytes, pl, false);
}

struct BlockParams {
  const float *norm, *frame, *decay, *freq;
};
static BlockParams block_params(const lnet_b200_alphabet_params *p, int block) {
  return block == 0 ? BlockParams{p->writer_norm, p->writer_frame, p->writer_raw_decay,
                                  p->writer_raw_frequency}
                    : BlockParams{p->reader_norm, p->reader_frame, p->reader_raw_decay,
                                  p->reader_raw_frequency};
}

extern "C" int lnet_b200_block_drive(const lnet_b200_alphabet_params *params,
                                     const lnet_b200_alphabet_request *req, int32_t block,
                                     const float *in, void *workspace, size_t workspace_bytes,
                                     float *u_out, float *xhat_out, lnet_stream_t stream) {
  auto st = (cudaStream_t)stream;
  Plan pl;
  LNET_TRY(slice_entry(params, req, workspace, workspace_bytes, pl, st));
  if (block != 0 && block != 1) return fail(LNET_ERR_INVALID_ARGUMENT, "block must be 0 or 1");
  if (!in || !u_out) return fail(LNET_ERR_INVALID_ARGUMENT, "block_drive: NULL tensor pointer");
  const int64_t bt = req->batch * req->steps;
  if (bt == 0) return LNET_OK;
  const int D = params->model_dim, M = params->modes;
  const BlockParams bp = block_params(params, block);
  float *xhat = xhat_out ? xhat_out : pl.xhat;
  LNET_TRY(rmsnorm(in, bp.norm, xhat, bt, D, st));
  // the same arithmetic as the unsplit forward: one GEMM over the gain-folded
  // frame, bf16 operands for bf16 requests (half_drive)
  float *a_re = pl.a_tab, *a_im = pl.a_tab + M, *g_re = pl.a_tab + 4 * M, *g_im = pl.a_tab + 5 * M;
  zoh_kernel<<<1, 128, 0, st>>>(bp.decay, bp.freq, M, nullptr, 1, a_re, a_im, g_re, g_im);
  LNET_TRY(after_launch("zoh_kernel"));
  const bool half = half_drive(params, req);
  fold_gain_kernel<<<grid_for((int64_t)D * M), 256, 0, st>>>(
      bp.frame, g_re, g_im, pl.wfold, half ? pl.wfold_bf16 : nullptr, D, M);
  LNET_TRY(after_launch("fold_gain_kernel"));
  if (half) {
    __nv_bfloat16 *xh16 = reinterpret_cast<__nv_bfloat16 *>(pl.proj);
    to_bf16_kernel<<<grid_for(bt * D), 256, 0, st>>>(xhat, xh16, bt * D);
    LNET_TRY(after_launch("to_bf16_kernel"));
    return gemm_rows(st, xh16, CUDA_R_16BF, D, pl.wfold_bf16, CUDA_R_16BF, 1, 2 * M, u_out, 2 * M,
                     bt, 2 * M, D, false, "gemm(drive)");
  }
  return gemm_rows(st, xhat, CUDA_R_32F, D, pl.wfold, CUDA_R_32F, 1, 2 * M, u_out, 2 * M, bt,
                   2 * M, D, req->act_dtype == LNET_BF16, "gemm(drive)");
}

extern "C" int lnet_b200_block_scan(const lnet_b200_alphabet_params *params,
                                    const lnet_b200_alphabet_request *req, int32_t block,
                                    float *u_states, const float *init, void *workspace,
                                    size_t workspace_bytes, lnet_stream_t stream) {
  auto st = (cudaStream_t)stream;
  Plan pl;
  LNET_TRY(slice_entry(params, req, workspace, workspace_bytes, pl, st));
  if (block != 0 && block != 1) return fail(LNET_ERR_INVALID_ARGUMENT, "block must be 0 or 1");
  if (!u_states) return fail(LNET_ERR_INVALID_ARGUMENT, "block_scan: NULL tensor pointer");
  const int64_t B = req->batch, T = req->steps;
  if (B * T == 0) return LNET_OK;
  const int M = params->modes;
  const BlockParams bp = block_params(params, block);
  float *a_re = pl.a_tab, *a_im = pl.a_tab + M;
  zoh_kernel<<<1, 128, 0, st>>>(bp.decay, bp.freq, M, nullptr, 1, a_re, a_im, nullptr, nullptr);
  LNET_TRY(after_launch("zoh_kernel"));
  const int64_t n_scan = cdiv(T, kScanChunk);
  const int threads = std::min(128, (int)cdiv(M, 32) * 32);
  dim3 gs((unsigned)n_scan, (unsigned)B);
  scan_local_kernel<<<gs, threads, 0, st>>>(u_states, bp.decay, bp.freq, a_re, a_im, nullptr,
                                            nullptr, pl.carries, T, M, kScanChunk, n_scan);
  LNET_TRY(after_launch("scan_local_kernel"));
  scan_carry_kernel<<<carry_grid(B, M), 32 * kCarryParts, 0, st>>>(pl.carries, B, M, n_scan, init);
  LNET_TRY(after_launch("scan_carry_kernel"));
  scan_apply_kernel<<<gs, threads, 0, st>>>(u_states, bp.decay, bp.freq, a_re, a_im, nullptr,
                                            nullptr, pl.carries, T, M, kScanChunk, n_scan);
  return after_launch("scan_apply_kernel");
}

extern "C" int lnet_b200_block_moment_sums(const lnet_b200_alphabet_params *params,
                                           const lnet_b200_alphabet_request *req,
                                           const float *states, const float *history,
                                           void *workspace, size_t workspace_bytes, double *sums,
                                           lnet_stream_t stream) {
  auto st = (cudaStream_t)stream;
  Plan pl;
  LNET_TRY(slice_entry(params, req, workspace, workspace_bytes, pl, st));
  if (!states || !sums) return fail(LNET_ERR_INVALID_ARGUMENT, "moment_sums: NULL tensor pointer");
  const int64_t B = req->batch, T = req->steps;
  if (B * T == 0) return LNET_OK;
  const int M = params->modes;
  const int64_t n_mom = cdiv(T, kMomChunk);
  const int threads = std::min(128, (int)cdiv(M, 32) * 32);
  dim3 gm((unsigned)n_mom, (unsigned)B);
  moments_partial_kernel<<<gm, threads, 0, st>>>(states, nullptr, pl.partial, T, M, kMomChunk,
                                                 n_mom, history);
  LNET_TRY(after_launch("moments_partial_kernel"));
  moment_sums_kernel<<<grid_for(B * 7 * M), 256, 0, st>>>(pl.partial, sums, B, M, n_mom);
  return after_launch("moment_sums_kernel");
}

extern "C" int lnet_b200_writer_output(const lnet_b200_alphabet_params *params,
                                       const lnet_b200_alphabet_request *req, const float *states,
                                       const float *xhat, const float *first_local,
                                       void *workspace, size_t workspace_bytes, float *stream_out,
                                       lnet_stream_t stream) {
  auto st = (cudaStream_t)stream;
  Plan pl;
  LNET_TRY(slice_entry(params, req, workspace, workspace_bytes, pl, st));
  if (!states || !xhat || !first_local || !stream_out)
    return fail(LNET_ERR_INVALID_ARGUMENT, "writer_output: NULL tensor pointer");
  const int64_t bt = req->batch * req->steps;
  if (bt == 0) return LNET_OK;
  const int D = params->model_dim, M = params->modes;
  const bool tf32 = req->act_dtype == LNET_BF16;
  if (normed_route(params, req)) {  // the unsplit forward's arithmetic (forward_generic_normed)
    residual_base_kernel<<<grid_for(bt * D), 256, 0, st>>>(first_local, xhat,
                                                           params->writer_direct_scale,
                                                           params->writer_layer_scale, stream_out,
                                                           bt, D);
    LNET_TRY(after_launch("residual_base_kernel"));
    scale_rows_kernel<<<grid_for((int64_t)D * 2 * M), 256, 0, st>>>(
        params->writer_frame, params->writer_layer_scale, pl.wfold, D, 2 * M);
    LNET_TRY(after_launch("scale_rows_kernel"));
    return gemm_rows(st, states, CUDA_R_32F, 2 * M, pl.wfold, CUDA_R_32F, 2 * M, 1, stream_out,
                     D, bt, D, 2 * M, tf32, "gemm(synthesis)", /*beta=*/1.f);
  }
  LNET_TRY(gemm_rows(st, states, CUDA_R_32F, 2 * M, params->writer_frame, CUDA_R_32F, 2 * M, 1,
                     pl.modal, D, bt, D, 2 * M, tf32, "gemm(synthesis)"));
  residual_kernel<<<token_grid(bt), token_block(D), 0, st>>>(
      first_local, xhat, pl.modal, params->writer_direct_scale, params->writer_layer_scale,
      stream_out, bt, D);
  return after_launch("residual_kernel");
}

extern "C" int lnet_b200_depthwise_conv_silu(const lnet_b200_alphabet_params *params,
                                             const lnet_b200_alphabet_request *req, int32_t which,
                                             const float *in, float *out, lnet_stream_t stream) {
  reset_launches();
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  LNET_TRY(check_params(params));
  LNET_TRY(check_request(params, req));
  if (which != 0 && which != 1) return fail(LNET_ERR_INVALID_ARGUMENT, "which must be 0 or 1");
  if (!in || !out) return fail(LNET_ERR_INVALID_ARGUMENT, "conv: NULL tensor pointer");
  const int64_t B = req->batch, T = req->steps;
  if (B * T == 0) return LNET_OK;
  const int D = params->model_dim;
  return depthwise_conv(in, which == 0 ? params->stem_conv_weight : params->reader_conv_weight,
                        which == 0 ? params->stem_conv_bias : params->reader_conv_bias, nullptr,
                        nullptr, out, B, T, D, params->conv_kernel, params->conv_dilation, st,
                        "depthwise_conv");
}

extern "C" int lnet_b200_zoh(const float *raw_decay, const float *raw_frequency, int32_t modes,
                             const float *dt, int64_t steps, float *a_re, float *a_im,
                             float *g_re, float *g_im, lnet_stream_t stream) {
  reset_launches();
  begin_entry((cudaStream_t)stream);
  if (modes < 1) return fail(LNET_ERR_INVALID_ARGUMENT, "modes must be positive");
  if (!raw_decay || !raw_frequency || !a_re || !a_im)
    return fail(LNET_ERR_INVALID_ARGUMENT, "zoh: NULL tensor pointer");
  if (dt && steps < 1) return LNET_OK;
  int64_t n = (dt ? steps : 1) * modes;
  zoh_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(raw_decay, raw_frequency, modes, dt,
                                                            steps, a_re, a_im, g_re, g_im);
  return after_launch("zoh_kernel");
}

// ---------------------------------------------------------------- training path
#include "train_path.cuh"
