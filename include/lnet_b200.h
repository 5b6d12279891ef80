/*
 * lnet_b200 — C ABI of the B200-native ALPHABET forward path and the
 * pole-residue Laplace layer.
 *
 * Conventions (all entry points):
 *   - every tensor is a caller-owned, contiguous, row-major DEVICE buffer on
 *     the current CUDA device; the library allocates nothing per call;
 *   - work is enqueued on `stream` with no host synchronisation;
 *   - the return value is LNET_OK or an error code; the message of the last
 *     error on the calling thread is returned by lnet_b200_last_error();
 *   - optional metadata pointers may be NULL (= absent);
 *   - complex per-mode quantities are packed as [..., 2M] = [re(M) | im(M)].
 *
 * Reference interfaces each entry point replaces are cited as
 * path:line relative to the reference project root (daehwa00/lnet-h200-imagenet1k-pg-ab).
 */
#ifndef LNET_B200_H
#define LNET_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *lnet_stream_t; /* == cudaStream_t */

enum lnet_b200_status {
  LNET_OK = 0,
  LNET_ERR_INVALID_ARGUMENT = 1, /* maps to ValueError on the Python side */
  LNET_ERR_UNSUPPORTED = 2,      /* shape/dtype outside what the kernels handle (TypeError) */
  LNET_ERR_WORKSPACE = 3,        /* workspace too small */
  LNET_ERR_CUDA = 4,             /* a CUDA launch or runtime call failed */
};

enum lnet_b200_dtype {
  LNET_F32 = 0,
  LNET_BF16 = 1,
  LNET_F64 = 2,
};

/* Effective ALPHABET parameters, all fp32 device pointers.  Frames are the
 * materialised constrained frames `block.frame.weight` ([D, 2M]).
 * Names follow the reference state_dict (src/lnet/alphabet.py:66-125,
 * src/lnet/pac_tight_frame_models.py:320-443,
 * src/lnet/pac_laplace_native_input.py:98-138). */
typedef struct lnet_b200_alphabet_params {
  int32_t raw_input_dim; /* C   */
  int32_t model_dim;     /* D   */
  int32_t modes;         /* M   (frame is [D, 2M]) */
  int32_t output_dim;    /* K   classes */
  int32_t conv_kernel;   /* 5 */
  int32_t conv_dilation; /* 4 */
  const float *stem_projection;  /* [D, C]  stem.projection.weight */
  const float *stem_conv_weight; /* [D, K5] stem.local.weight */
  const float *stem_conv_bias;   /* [D]     stem.local.bias */
  const float *writer_norm;      /* [D]     forward_block.norm.weight */
  const float *writer_frame;     /* [D, 2M] forward_block.frame.weight */
  const float *writer_raw_decay; /* [M] */
  const float *writer_raw_frequency; /* [M] */
  const float *writer_direct_scale;  /* [D] */
  const float *writer_layer_scale;   /* [D] */
  const float *reader_conv_weight;   /* [D, K5] second_local.weight */
  const float *reader_conv_bias;     /* [D]     second_local.bias */
  const float *reader_norm;          /* [D]     backward_block.norm.weight */
  const float *reader_frame;         /* [D, 2M] backward_block.frame.weight */
  const float *reader_raw_decay;     /* [M] */
  const float *reader_raw_frequency; /* [M] */
  const float *head_weight;          /* [K, 14M] head.classifier.weight */
  const float *head_bias;            /* [K]      head.classifier.bias */
} lnet_b200_alphabet_params;

/* One forward request.  x is [B, T, C] in `x_dtype`; metadata are fp32:
 *   time_delta [B, T] (finite, >= 0), observation_mask [B, T, obs_channels]
 *   with obs_channels in {1, C}, valid_mask [B, T] (values in [0, 1]).
 * `act_dtype` selects the storage type of the [B, T, D] activations that
 * cross HBM between kernels (LNET_F32 or LNET_BF16); state, moments and all
 * arithmetic are fp32. */
typedef struct lnet_b200_alphabet_request {
  int64_t batch;
  int64_t steps;
  int32_t x_dtype;
  int32_t act_dtype;
  const void *x;
  const float *time_delta;
  const float *observation_mask;
  int32_t obs_channels;
  const float *valid_mask;
} lnet_b200_alphabet_request;

/* Bytes of device workspace lnet_b200_alphabet_forward needs for `req`. */
int lnet_b200_alphabet_workspace_size(const lnet_b200_alphabet_params *params,
                                      const lnet_b200_alphabet_request *req,
                                      size_t *bytes);

/* Full `Alphabet.forward(inputs, time_delta=, observation_mask=, valid_mask=)`
 * -> logits [B, K] fp32.  Replaces the eager/Triton dispatch of
 * src/lnet/alphabet.py:350-416 (Alphabet.forward) and everything below it.
 * Optional outputs (NULL = not wanted): writer_moments / reader_moments
 * [B, 7M] raw (pre radial-log) moments. Workspace must be 256-byte aligned. */
int lnet_b200_alphabet_forward(const lnet_b200_alphabet_params *params,
                               const lnet_b200_alphabet_request *req, void *workspace,
                               size_t workspace_bytes, float *logits, float *writer_moments,
                               float *reader_moments, lnet_stream_t stream);

/* Test hook, one shot: the next fused-route forward in this process looks for
 * look-back records under a tag that no record carries, so every look-back
 * gives up after a short bounded wait (64 polls), sets the look-back error bit
 * and the call writes NaN logits.  Used by the tests that check that a
 * give-up surfaces; no reference counterpart. */
int lnet_b200_debug_inject_lookback_miss(void);

/* GEMM backend of the general route (process-wide): 0 = this library's tcgen05
 * row GEMMs wherever the shape fits them (bf16 x bf16 for bf16 operands,
 * split-bf16 x3 for fp32 operands; n <= 256 with TMA-addressable operands, or
 * n, k <= 128 otherwise), cuBLAS for any other shape (default); 1 = cuBLAS for
 * every GEMM (used by the tests to compare the two).  No reference
 * counterpart: replaces the reference's torch matmuls on this path. */
int lnet_b200_set_gemm_backend(int backend);

/* Route selection for lnet_b200_alphabet_forward (process-wide):
 * 0 = automatic (the fused unit-grid kernels when the request has no
 * time_delta or valid mask (observation masks are served: the writer masks its
 * input tiles and drive), bf16 activations and a compiled shape; the general
 * route otherwise), 1 = general route only.  No reference counterpart: replaces the
 * reference's per-instance fused-inference gates (src/lnet/alphabet.py:190-223,
 * 257-348). */
int lnet_b200_set_route(int route);
/* Route the current setting picks for (params, req): 0 fused, 1 general, -1 invalid. */
int lnet_b200_alphabet_route(const lnet_b200_alphabet_params *params,
                             const lnet_b200_alphabet_request *req);

/* Prepared static inference (replaces Alphabet.prepare_for_inference_,
 * src/lnet/alphabet.py:190-222): lnet_b200_alphabet_prepare writes the fused
 * route's prepared operands (bf16 GEMM operand slabs with the ZOH gains folded
 * in, pole constants) for `params` into `workspace`; they sit at the start of
 * the workspace at offsets that depend on (C, D, M) only.
 * lnet_b200_alphabet_forward_prepared is lnet_b200_alphabet_forward without
 * rebuilding them: valid while the parameters are unchanged and for every
 * request whose workspace size (lnet_b200_alphabet_workspace_size) fits in
 * `workspace_bytes`.  Requests that take the general route ignore the
 * preparation.  Calls sharing a workspace must be ordered (one stream). */
int lnet_b200_alphabet_prepare(const lnet_b200_alphabet_params *params,
                               const lnet_b200_alphabet_request *req, void *workspace,
                               size_t workspace_bytes, lnet_stream_t stream);
int lnet_b200_alphabet_forward_prepared(const lnet_b200_alphabet_params *params,
                                        const lnet_b200_alphabet_request *req, void *workspace,
                                        size_t workspace_bytes, float *logits,
                                        float *writer_moments, float *reader_moments,
                                        lnet_stream_t stream);

/* lnet_b200_alphabet_forward (prepared = 0) or ..._forward_prepared (prepared =
 * 1) for a right-padded request: `lengths` (int64 [B], device) holds each row's
 * valid length L_b, meaning valid_mask[b, t] = 1 for t < L_b and 0 after, and
 * req carries no valid mask or time_delta (an observation mask is allowed).  The result equals the forward with that valid mask
 * (src/lnet/pac_tight_frame_models.py:1660-1702 masked moments,
 * src/lnet/alphabet_backbone.py:649-676 / :872-992 stem and reader masking): a
 * right-padded row computes exactly as an unpadded row of L_b steps, so the
 * fused route serves it, skipping the padded chunks.  Fails with
 * LNET_ERR_UNSUPPORTED when the request does not take the fused route (then
 * pass the mask to lnet_b200_alphabet_forward).  The module
 * (B200Alphabet.forward) detects right-padded masks and calls this. */
int lnet_b200_alphabet_forward_lengths(const lnet_b200_alphabet_params *params,
                                       const lnet_b200_alphabet_request *req,
                                       const int64_t *lengths, int32_t prepared,
                                       void *workspace, size_t workspace_bytes, float *logits,
                                       float *writer_moments, float *reader_moments,
                                       lnet_stream_t stream);

/* Device-side status of the last lnet_b200_alphabet_forward in `workspace`
 * for this request's route (synchronises the device).  Every wait inside the
 * kernels is bounded; a wait that gave up sets a bit: 1 << 0..3 and 1 << 9 MMA
 * completion (writer stem, writer drive, writer synthesis, reader drive; reader
 * conv), 1 << 4 / 1 << 5
 * look-back (writer / reader), 1 << 6 / 1 << 7 tile loads (writer / reader) on
 * the fused route; 1 << 8 a bulk input copy of the general route's conv +
 * RMSNorm kernel.  Nonzero means the results of that call are invalid, and
 * that call wrote NaN to every logit (the head reads this word before writing
 * them), so a give-up never yields finite logits.  No reference counterpart
 * (the reference has no device-side waits). */
int lnet_b200_alphabet_device_status(const lnet_b200_alphabet_params *params,
                                     const lnet_b200_alphabet_request *req,
                                     const void *workspace, size_t workspace_bytes,
                                     uint32_t *status);

/* Stage entry points (same request/params conventions; intermediate tensors
 * fp32 [B, T, D] unless noted). */

/* ZOH coefficients a = exp(p dt), gamma = (a - 1)/p with p = -damping + i freq,
 * damping = 1e-3 + (2 - 1e-3) sigmoid(raw_decay), freq = pi tanh(raw_frequency).
 * dt == NULL -> unit grid, outputs [M]; else dt is [steps] and outputs are
 * [steps, M].  Replaces src/lnet/pac_real2d_math.py:20-53 and
 * src/lnet/pac_tight_frame_models.py:458-459,487-491. */
int lnet_b200_zoh(const float *raw_decay, const float *raw_frequency, int32_t modes,
                  const float *dt, int64_t steps, float *a_re, float *a_im, float *g_re,
                  float *g_im, lnet_stream_t stream);

/* Raw stem: first_local = valid * SiLU(DWConv(P (x * obs * valid))) (or the
 * physical-time conv when time_delta is given).  Replaces
 * AlphabetBackbone._edge_stem (src/lnet/alphabet_backbone.py:593-676). */
int lnet_b200_stem(const lnet_b200_alphabet_params *params,
                   const lnet_b200_alphabet_request *req, void *workspace,
                   size_t workspace_bytes, float *first_local, lnet_stream_t stream);

/* Tied writer block: stream v [B, T, D] and raw moments [B, 7M].  Replaces
 * _TightFrameBlock.forward (src/lnet/pac_tight_frame_models.py:717-1507) as
 * called by AlphabetBackbone._writer (src/lnet/alphabet_backbone.py:704-718). */
int lnet_b200_writer(const lnet_b200_alphabet_params *params,
                     const lnet_b200_alphabet_request *req, const float *first_local,
                     void *workspace, size_t workspace_bytes, float *stream_out,
                     float *moments, lnet_stream_t stream);

/* Terminal reader: local conv of the masked writer stream, SiLU, mask,
 * moments-only reader block -> raw moments [B, 7M].  Replaces
 * AlphabetBackbone._terminal_reader (src/lnet/alphabet_backbone.py:872-992). */
int lnet_b200_reader(const lnet_b200_alphabet_params *params,
                     const lnet_b200_alphabet_request *req, const float *first_stream,
                     void *workspace, size_t workspace_bytes, float *moments,
                     lnet_stream_t stream);

/* Head: radial-log of both moment banks, concatenation, affine readout.
 * Replaces radial_log_lag124_moments + _ModalAffineHead
 * (src/lnet/alphabet.py:29-63) and modal_affine_readout_inference
 * (src/lnet/pac_triton_modal_affine_readout_inference.py:73-111). */
int lnet_b200_head(const lnet_b200_alphabet_params *params, int64_t batch,
                   const float *writer_moments, const float *reader_moments, float *logits,
                   lnet_stream_t stream);

/* The image configuration's whole forward from uint8 images [B, H, W, 3]
 * (device, 16-byte aligned; H, W multiples of 4): the normalise + 4x4 patchify
 * of lnet_b200_patchify_images (same arithmetic, so the same bf16 tokens) runs
 * inside the fused writer, which builds each 144-token x tile from the image
 * bytes instead of loading a token tensor, then the forward of
 * lnet_b200_alphabet_forward (prepared = 0) or ..._forward_prepared (1) on
 * those tokens.  No token tensor is written or read.  Replaces the harness
 * transform (scripts/train_alphabet2d_imagenet100.py:292-310), its patchify
 * reshape and Alphabet.forward (src/lnet/alphabet.py:350-416).  `mean`, `std`
 * are HOST arrays of 3 floats.  Needs the fused route: raw_input_dim 48 and a
 * compiled (C, D, M) shape, else LNET_ERR_UNSUPPORTED (then patchify and call
 * lnet_b200_alphabet_forward).  Workspace size from
 * lnet_b200_alphabet_images_workspace_size. */
int lnet_b200_alphabet_images_workspace_size(const lnet_b200_alphabet_params *params,
                                             int64_t batch, int32_t height, int32_t width,
                                             size_t *bytes);
int lnet_b200_alphabet_forward_images(const lnet_b200_alphabet_params *params,
                                      const uint8_t *images, int64_t batch, int32_t height,
                                      int32_t width, const float *mean, const float *std,
                                      int32_t prepared, void *workspace, size_t workspace_bytes,
                                      float *logits, float *writer_moments,
                                      float *reader_moments, lnet_stream_t stream);

/* Input pipeline of the image configuration: uint8 images [B, H, W, 3]
 * (device) -> tokens [B, (H/p)(W/p), 3 p^2] (`tokens_dtype` LNET_BF16 or
 * LNET_F32), per element v = (u / 255 - mean[ch]) / std[ch] in fp32 (IEEE
 * divisions) and token channel (i * p + j) * 3 + ch for pixel (i, j) of the
 * patch.  `mean` and `std` are HOST arrays of 3 floats.  Replaces the
 * harness transform ConvertImageDtype(float32) + Normalize(mean, std)
 * (scripts/train_alphabet2d_imagenet100.py:292-310) followed by the 4x4
 * patchify reshape, so that a caller can copy uint8 images (half the bytes of
 * bf16 tokens) to the device. */
int lnet_b200_patchify_images(const uint8_t *images, int64_t batch, int32_t height,
                              int32_t width, int32_t patch, const float *mean, const float *std,
                              void *tokens, int32_t tokens_dtype, lnet_stream_t stream);

/* Time-split pieces (the sequence split over ranks of lnet_b200.timesplit).
 * Each works on one rank's slice of steps of every row: req->batch rows of
 * req->steps = Ts steps, no metadata (static poles), fp32 tensors; workspace
 * sized by lnet_b200_alphabet_workspace_size for the same request.  GEMMs use
 * TF32 when req->act_dtype is LNET_BF16.  Together with lnet_b200_stem and
 * lnet_b200_head they restate lnet_b200_alphabet_forward on a slice with the
 * carry-in and lag history of the preceding steps supplied by the caller.
 *
 * block_drive: u [B,Ts,2M] = gamma (x) (RMSNorm_block(in) frame_block) and
 *   optionally x-hat [B,Ts,D] (block 0 writer, 1 reader);
 *   (src/lnet/pac_tight_frame_models.py:1038-1039,1145-1149).
 * block_scan: in place, u -> states s_t = a s_{t-1} + u_t starting from
 *   `init` [B,2M] (the state before the slice; NULL = zero)
 *   (src/lnet/pac_recurrence.py:191-212).
 * block_moment_sums: raw sums [B,7M] (fp64) of E, C1, C2, C4 over the slice,
 *   lag products reaching before the slice taken from `history` [B,4,2M]
 *   (states at steps -1..-4; NULL = sequence start); dividing the all-rank
 *   sums by T and T - lag gives the raw moments
 *   (src/lnet/pac_tight_frame_models.py:1632-1657).
 * writer_output: stream [B,Ts,D] = x + ls (s frame^T + ds x-hat)
 *   (src/lnet/pac_tight_frame_models.py:1480,1490,1503-1507).
 * depthwise_conv_silu: SiLU(bias + K5/d4 depthwise conv) of in [B,Ts,D], zero
 *   padding at the slice edges (callers pass a slice with a +-8-step halo);
 *   which 0 = stem.local, 1 = second_local (src/lnet/alphabet_backbone.py:872-992). */
int lnet_b200_block_drive(const lnet_b200_alphabet_params *params,
                          const lnet_b200_alphabet_request *req, int32_t block, const float *in,
                          void *workspace, size_t workspace_bytes, float *u_out, float *xhat_out,
                          lnet_stream_t stream);
int lnet_b200_block_scan(const lnet_b200_alphabet_params *params,
                         const lnet_b200_alphabet_request *req, int32_t block, float *u_states,
                         const float *init, void *workspace, size_t workspace_bytes,
                         lnet_stream_t stream);
int lnet_b200_block_moment_sums(const lnet_b200_alphabet_params *params,
                                const lnet_b200_alphabet_request *req, const float *states,
                                const float *history, void *workspace, size_t workspace_bytes,
                                double *sums, lnet_stream_t stream);
int lnet_b200_writer_output(const lnet_b200_alphabet_params *params,
                            const lnet_b200_alphabet_request *req, const float *states,
                            const float *xhat, const float *first_local, void *workspace,
                            size_t workspace_bytes, float *stream_out, lnet_stream_t stream);
int lnet_b200_depthwise_conv_silu(const lnet_b200_alphabet_params *params,
                                  const lnet_b200_alphabet_request *req, int32_t which,
                                  const float *in, float *out, lnet_stream_t stream);

/* Pole-residue Laplace layer in float64:
 *   y_t = sum_{m,i} R[o, m, i] s_t[m, i] + D x_t + bias,
 *   s_t[m, i] = exp(p_m dt) s_{t-1}[m, i] + dt phi1(p_m dt) x_t[i],
 *   p_m = -(softplus(raw_decay_m) + min_decay).
 * x and y are [B, T, Dm] in `x_dtype` (LNET_F32 or LNET_F64); parameters are
 * float64: raw_decay [M], residues [Dm, M, Dm], direct [Dm, Dm], bias [Dm].
 * Replaces PoleResidueTemporalMixing.forward (src/lnet/laplace.py:126-159). */
int lnet_b200_laplace_workspace_size(int64_t batch, int64_t steps, int32_t model_dim,
                                     int32_t modes, size_t *bytes);
int lnet_b200_laplace_forward(const double *raw_decay, const double *residues,
                              const double *direct, const double *bias, int32_t model_dim,
                              int32_t modes, double dt, double min_decay, int32_t x_dtype,
                              const void *x, int64_t batch, int64_t steps, void *y,
                              void *workspace, size_t workspace_bytes, lnet_stream_t stream);

/* The same layer when its residues are diagonal in channels (R[o, m, i] = 0
 * for i != o, e.g. M real poles per channel): given, per output channel o, the
 * indices mode_index[o, j] (int32 [Dm, K]) of the modes with a nonzero
 * residue and those residues residue[o, j] = R[o, mode_index[o, j], o]
 * (float64 [Dm, K]; unused slots: any valid index with residue 0), computes
 * the same y with K state updates per channel instead of a dense [Dm, M Dm]
 * contraction.  K <= 16; no workspace.  The caller (B200PoleResidueTemporalMixing)
 * detects the structure from the dense residues.  A specialisation of
 * PoleResidueTemporalMixing.forward (src/lnet/laplace.py:126-159) for the
 * per-channel pole layout. */
int lnet_b200_laplace_forward_channelwise(const double *raw_decay, const int32_t *mode_index,
                                          const double *residue, const double *direct,
                                          const double *bias, int32_t model_dim, int32_t modes,
                                          int32_t modes_per_channel, double dt,
                                          double min_decay, int32_t x_dtype, const void *x,
                                          int64_t batch, int64_t steps, void *y,
                                          lnet_stream_t stream);

/* Allocation-free variant of lnet_b200_laplace_forward for callers that may
 * not allocate device memory (foreign memory pools, plugin hosts that forbid
 * cudaMalloc, real-time loops).  Same arguments minus the workspace: the
 * scratch lives in a fixed array inside the library (see
 * lnet_b200_laplace_noalloc_max_scratch_bytes; every GPU that loads the
 * library holds it until exit).  Shapes needing more scratch than that
 * (lnet_b200_laplace_workspace_size) fail with LNET_ERR_WORKSPACE.  The first
 * call on a device looks up the array's device address; make that first call
 * before any stream capture.  The address is kept for the life of the
 * process: do not use this entry point on a device after cudaDeviceReset of
 * that device.  All calls share the array: calls that overlap on the GPU
 * race.  No counterpart in the reference. */
size_t lnet_b200_laplace_noalloc_max_scratch_bytes(void);
int lnet_b200_laplace_forward_noalloc(const double *raw_decay, const double *residues,
                                      const double *direct, const double *bias,
                                      int32_t model_dim, int32_t modes, double dt,
                                      double min_decay, int32_t x_dtype, const void *x,
                                      int64_t batch, int64_t steps, void *y,
                                      lnet_stream_t stream);

/* Number of kernel launches the most recent successful lnet_b200_* call on
 * this thread enqueued. */
int lnet_b200_last_launch_count(void);

/* Optional per-launch device timing (diagnostics; off by default).
 * lnet_b200_profile_enable(1) clears old records and makes every following
 * launch record a CUDA event on its stream; lnet_b200_profile_read
 * synchronises those events and writes, per distinct kernel name, the total
 * milliseconds and launch count (names '\n'-separated in names_buf).  Returns
 * the number of kernels written.  No reference counterpart: replaces the
 * torch.profiler usage of the reference's launch tuning scripts. */
void lnet_b200_profile_enable(int on);
int lnet_b200_profile_read(char *names_buf, int names_bytes, float *total_ms, int *launches,
                           int max_entries);

/* Per-phase cycle tracing of the fused kernels (off by default).  Counters
 * are the clock64 cycles thread 0 of every CTA spends per phase, summed over
 * CTAs; slots (writer row 0, reader row 1): 0 claim, 1 tile load, 2 first GEMM
 * wait, 3 token epilogue, 4 drive GEMM wait, 5 scan, 6 synthesis wait,
 * 7 residual epilogue, 10 scan pass 1, 11 look-back, 12 scan pass 2,
 * 15 items.  No reference counterpart (the reference profiles with
 * torch.profiler, src/lnet/pac_launch_tuning.py). */
int lnet_b200_trace_enable(int on);
int lnet_b200_trace_read(unsigned long long *out /* [2][16] */);
/* Same, ordered on `stream` only (out must be pinned host memory): observes the
 * counters of fused kernels still running on another stream. */
int lnet_b200_trace_read_async(unsigned long long *out, lnet_stream_t stream);

/* ---------------------------------------------------------------- training
 * Backward pass of the ALPHABET forward (the reference trains through torch
 * autograd over its custom ops: register_autograd in
 * src/lnet/pac_triton_recurrence_op.py:603-684 and the VJP kernels of
 * src/lnet/pac_triton_parallel_static_recurrence_lag124_training.py:488-876).
 * Static-pole requests without observation masks (valid masks allowed);
 * fp32 throughout.  lnet_b200_alphabet_train_forward computes the logits and
 * keeps every activation the backward needs in `workspace` (sized by
 * lnet_b200_alphabet_train_workspace_size); lnet_b200_alphabet_backward then
 * writes dL/dparameter for dL/dlogits [B, K] into caller buffers shaped like
 * the parameters (frames: the gradient at the materialised [D, 2M] weight).
 * The workspace must not be reused between the two calls. */
typedef struct lnet_b200_alphabet_grads {
  float *stem_projection;
  float *stem_conv_weight;
  float *stem_conv_bias;
  float *writer_norm;
  float *writer_frame;
  float *writer_raw_decay;
  float *writer_raw_frequency;
  float *writer_direct_scale;
  float *writer_layer_scale;
  float *reader_conv_weight;
  float *reader_conv_bias;
  float *reader_norm;
  float *reader_frame;
  float *reader_raw_decay;
  float *reader_raw_frequency;
  float *head_weight;
  float *head_bias;
} lnet_b200_alphabet_grads;

int lnet_b200_alphabet_train_workspace_size(const lnet_b200_alphabet_params *params,
                                            const lnet_b200_alphabet_request *req,
                                            size_t *bytes);
int lnet_b200_alphabet_train_forward(const lnet_b200_alphabet_params *params,
                                     const lnet_b200_alphabet_request *req, void *workspace,
                                     size_t workspace_bytes, float *logits,
                                     lnet_stream_t stream);
int lnet_b200_alphabet_backward(const lnet_b200_alphabet_params *params,
                                const lnet_b200_alphabet_request *req, void *workspace,
                                size_t workspace_bytes, const float *dlogits,
                                const lnet_b200_alphabet_grads *grads, lnet_stream_t stream);

/* Message of the last error on the calling thread ("" if none). */
const char *lnet_b200_last_error(void);

/* Library version string. */
const char *lnet_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LNET_B200_H */
