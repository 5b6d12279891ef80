// Fused unit-grid route of the ALPHABET forward on sm_100a.
//
// Work item = one chunk of kChunk (=128) consecutive steps of one batch row.
// Items are claimed from an atomic counter in chunk-major order
// (item = chunk * B + row), one item ahead, so the predecessor (row, chunk - 1)
// of every item was claimed earlier by a running CTA: the decoupled look-back
// below always makes progress.
//
// fused_writer_kernel (persistent, one CTA of 512 threads per SM = two
// independent item streams of 256 threads sharing the weight operands):
//   1. x rows [t0 - 8, t0 + 136) by TMA (3-D tensor map, one 8-channel box per
//      no-swizzle K-major slab, zero fill outside [0, T)), fetched one item
//      ahead into the tile region;
//   2. stem projection + dilated depthwise conv as ONE tcgen05 GEMM:
//        acc[t, d] = sum_k sum_c x[t + 4k - 8, c] * (w[d, k] P[d, c]),
//      the five taps are five row-shifted descriptors over the same tile;
//   3. +bias, SiLU, RMSNorm (thread per step, two threads per row), xhat ->
//      bf16 slab; the bf16 stem output waits in the output rows (L2);
//   4. drive GEMM in mode-major orientation: the A operand repeats the mode
//      rows every 64 lanes, so every TMEM lane quarter holds the complex drive
//      u_m(t) of 32 modes over all 128 steps (gamma is folded into the frame)
//      and every warp can scan without a transpose;
//   5. scan: each mode's 128 steps are cut into four sub-chunks of 32 scanned
//      by four threads; sub-chunk end states combine in shared memory into the
//      chunk aggregate, which the last sub-chunk's threads publish and then
//      resolve against their predecessors (decoupled look-back over tagged
//      records, the predecessor's inclusive record prefetched); a second pass
//      from the true carries accumulates E, C1, C2, C4 and writes the states
//      (bf16) as the A operand of
//   6. the synthesis GEMM (token-major), during which the chunk's moments are
//      added to the row's fp64 sums, and the residual epilogue
//      v = x + ls (s W^T + ds xhat), stored as bf16.
// fused_reader_kernel (two CTAs of 256 threads per SM): the same skeleton on
//   the writer stream: TMA tile, conv on CUDA cores, SiLU, RMSNorm, drive
//   GEMM, scan, moments.
// fused_finalize_kernel: moments and radial-log features from the row sums.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "generic_kernels.cuh"
#include "head_gemm.cuh"
#include "sm100.cuh"

namespace lnet {

constexpr int kChunk = 128;
constexpr int kHalo = 8;
constexpr int kTaps = 5;
constexpr int kXRows = kChunk + 2 * kHalo;
constexpr int kFusedThreads = 256;
constexpr uint32_t kSpinLimit = 1u << 20;
// Device error bits (first error word of the fused route's flag block):
// bit 0..3: an MMA completion wait gave up (writer stem, writer drive, writer
// synthesis, reader drive); bit 4 / 5: a look-back wait gave up (writer / reader);
// bit 6 / 7: a tile (TMA) wait gave up (writer / reader).
constexpr uint32_t kErrTile = 1u << 6;
constexpr uint32_t kErrLookback = 1u << 4;

// Per-block pole constants (floats, M entries each), SUB = steps per scan
// sub-chunk of the block (64 writer, 32 reader):
//   [0] a_re, [1] a_im, [2 + 2i] / [3 + 2i]  re/im of a^(128 - i),
//   [10 + 2i] / [11 + 2i] re/im of a^(SUB - i)  (i = 0..3), [18]/[19] a^(2 SUB),
//   [20]/[21] a^(3 SUB).
constexpr int kConsts = 22;
constexpr int KC_AL = 2, KC_AS = 10, KC_A2S = 18, KC_A3S = 20;
constexpr int kWriterSub = 32, kReaderSub = 32;
constexpr int kWriterNSub = 4;
constexpr int kWriterDriveRows = 128, kReaderDriveRows = 128;
// Thread (of an item stream) that issues the next tile's TMA copies: not
// thread 0, whose async-unit instructions queue behind its MMAs.
constexpr int kTileIssuer = 32;

template <int NSUB>
struct ScanLayout {
  static constexpr int SUB = kChunk / NSUB;
  static constexpr int END = 0;                   // [NSUB][2][64]
  static constexpr int LAST = NSUB * 128;         // [NSUB][8][64]
  static constexpr int CARRY = LAST + NSUB * 512; // [8][64]
  static constexpr int MOM = CARRY + 512;         // [NSUB][7][64]
  static constexpr int FLOATS = MOM + NSUB * 448;
};


constexpr int cmax(int a, int b) { return a > b ? a : b; }

// ---------------------------------------------------------------- workspace
struct FusedWorkspace {
  float *moments = nullptr;            // [2][B][7M]
  float *feats = nullptr;              // [B][14M] radial-log features
  float *head_partial = nullptr;       // split-K partial logits
  __nv_bfloat16 *q = nullptr;          // stem B operand   [5][C/8][D][8]
  __nv_bfloat16 *wdrive = nullptr;     // writer drive A   [2][D/8][64][8]
  __nv_bfloat16 *rdrive = nullptr;     // reader drive A   [2][D/8][128][8]
  __nv_bfloat16 *wsyn = nullptr;       // synthesis B      [2M/8][D][8]
  float *consts = nullptr;             // [2][kConsts * M]
  __nv_bfloat16 *stream = nullptr;     // [B, T, D]
  // per-row moment sums [2 (writer, reader)][B][7M]: every item adds its
  // chunk's partial moments (fp64 atomics: the sum of a row's ~T/128 fp32
  // partials is exact in double for any realistic spread, so the result does
  // not depend on the order of the additions)
  double *rowsum = nullptr;
  int64_t rowsum_len = 0;
  // look-back records [B * nch][2 (aggregate, inclusive)][4 states][2 (re, im)][M];
  // each entry = (state bits) | (epoch << 32), single-copy atomic 8-byte words
  unsigned long long *wrec = nullptr;
  unsigned long long *rrec = nullptr;
  uint32_t *flags = nullptr;           // counters[2] + error[2]
  size_t flag_words = 0;
  // Replay counter of the look-back tags, kept in the workspace and advanced
  // on the device at the end of every call (fused_finalize_kernel), so that
  // replays of a captured CUDA graph (same host arguments) still tag their
  // records differently (record_tag).
  uint32_t *epoch_word = nullptr;
};

inline int64_t fused_chunks(int64_t steps) { return cdiv(steps, kChunk); }

inline void plan_fused(Arena &ar, FusedWorkspace &w, const lnet_b200_alphabet_params *p,
                       const lnet_b200_alphabet_request *r) {
  const int C = p->raw_input_dim, D = p->model_dim, M = p->modes;
  const int64_t B = r->batch, nch = fused_chunks(std::max<int64_t>(r->steps, 1));
  // prepared operands first: their offsets depend on (C, D, M) only, so a
  // workspace prepared once serves every batch and length it is large enough for
  w.q = ar.take<__nv_bfloat16>((size_t)kTaps * C * D);
  w.wdrive = ar.take<__nv_bfloat16>((size_t)2 * D * kWriterDriveRows);
  w.rdrive = ar.take<__nv_bfloat16>((size_t)2 * D * 128);
  w.wsyn = ar.take<__nv_bfloat16>((size_t)2 * M * D);
  w.consts = ar.take<float>((size_t)2 * kConsts * M);
  w.moments = ar.take<float>((size_t)2 * B * 7 * M);
  w.feats = ar.take<float>((size_t)B * 14 * M);
  w.head_partial = ar.take<float>(head_partial_floats(B, p->output_dim));
  w.stream = ar.take<__nv_bfloat16>((size_t)B * r->steps * D);
  w.wrec = ar.take<unsigned long long>((size_t)B * nch * 16 * M);
  w.rrec = ar.take<unsigned long long>((size_t)B * nch * 16 * M);
  w.rowsum_len = 2 * B * 7 * M;  // zeroed with the flags by one memset per call
  w.rowsum = ar.take<double>((size_t)w.rowsum_len);
  w.flag_words = 4;
  w.flags = ar.take<uint32_t>(w.flag_words);
  w.epoch_word = ar.take<uint32_t>(1);
}

// ---------------------------------------------------------------- operand preparation
// Writes every bf16 operand in its shared-memory slab layout
// (element (row, k) of an R-row K-major operand at ((k / 8) * R + row) * 8 + k % 8)
// and the per-mode pole constants, all in double before one rounding.
__device__ __forceinline__ void cmul_d(double ar, double ai, double br, double bi, double &cr,
                                       double &ci) {
  cr = ar * br - ai * bi;
  ci = ar * bi + ai * br;
}

__global__ void fused_prepare_kernel(lnet_b200_alphabet_params p, FusedWorkspace w) {
  const int C = p.raw_input_dim, D = p.model_dim, M = p.modes, K5 = p.conv_kernel;
  // per-mode ZOH input gains of both blocks, once per CTA (M <= 64)
  __shared__ float zg[2][2][64];  // [block][re | im][mode]
  for (int i = threadIdx.x; i < 2 * M; i += blockDim.x) {
    const int blk = i / M, m = i - (i / M) * M;
    double damping, frequency;
    mode_pole(blk == 0 ? p.writer_raw_decay[m] : p.reader_raw_decay[m],
              blk == 0 ? p.writer_raw_frequency[m] : p.reader_raw_frequency[m], damping,
              frequency);
    const Zoh z = zoh_eval(damping, frequency, 1.0);
    zg[blk][0][m] = z.g_re;
    zg[blk][1][m] = z.g_im;
  }
  __syncthreads();
  // every index below 2^31 (operand sizes of one block): 32-bit arithmetic
  const int n_q = kTaps * C * D;
  // drive A rows per block: 128 (modes repeated every 64 lanes)
  const int n_wdrive = 2 * D * kWriterDriveRows;
  const int n_rdrive = 2 * D * kReaderDriveRows;
  const int n_syn = 2 * M * D;
  const int total = n_q + n_wdrive + n_rdrive + n_syn + 2 * M;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    if (i < n_q) {  // Q_k[d][c] = w[d][k] * P[d][c]
      const int k = i / (C * D);
      const int rem = i - k * C * D;
      int d = rem / C, c = rem - d * C;
      double v = (double)p.stem_conv_weight[d * K5 + k] * (double)p.stem_projection[d * C + c];
      w.q[k * C * D + ((c / 8) * D + d) * 8 + (c % 8)] = __float2bfloat16_rn((float)v);
      continue;
    }
    int j = i - n_q;
    if (j < n_wdrive + n_rdrive) {  // drive A: lane r holds mode r % 64 (zero if >= M), K = d
      const int blk = j < n_wdrive ? 0 : 1;
      const int R = blk == 0 ? kWriterDriveRows : kReaderDriveRows;
      const int rem = blk == 0 ? j : j - n_wdrive;
      const int part = rem / (D * R);
      const int rem2 = rem - part * D * R;
      int d = rem2 / R, r = rem2 - d * R;
      int m = r % 64;
      float out = 0.f;
      if (m < M) {
        const float *frame = blk == 0 ? p.writer_frame : p.reader_frame;
        const double gr = zg[blk][0][m], gi = zg[blk][1][m];
        double fr = frame[d * 2 * M + m], fi = frame[d * 2 * M + M + m];
        out = (float)(part == 0 ? gr * fr - gi * fi : gr * fi + gi * fr);
      }
      __nv_bfloat16 *dst = blk == 0 ? w.wdrive : w.rdrive;
      dst[part * D * R + ((d / 8) * R + r) * 8 + (d % 8)] = __float2bfloat16_rn(out);
      continue;
    }
    j -= n_wdrive + n_rdrive;
    if (j < n_syn) {  // synthesis B rows = d, K = 2M
      const int d = j / (2 * M), jj = j - d * 2 * M;
      w.wsyn[((jj / 8) * D + d) * 8 + (jj % 8)] = __float2bfloat16_rn(p.writer_frame[d * 2 * M + jj]);
      continue;
    }
    j -= n_syn;  // per-mode constants of both blocks
    const int blk = j / M, m = j - blk * M;
    double damping, frequency;
    mode_pole(blk == 0 ? p.writer_raw_decay[m] : p.reader_raw_decay[m],
              blk == 0 ? p.writer_raw_frequency[m] : p.reader_raw_frequency[m], damping,
              frequency);
    Zoh z = zoh_eval(damping, frequency, 1.0);
    // Powers of the fp32 coefficient the scan multiplies by, accumulated in
    // double so that carries match step-by-step propagation.
    const double ar = (double)z.a_re, ai = (double)z.a_im;
    double pr = 1.0, pi = 0.0;
    float *k = w.consts + blk * kConsts * M;
    for (int step = 1; step <= kChunk; ++step) {
      double nr, ni;
      cmul_d(pr, pi, ar, ai, nr, ni);
      pr = nr;
      pi = ni;
      const int sub = blk == 0 ? kWriterSub : kReaderSub;
      int slots[4] = {-1, -1, -1, -1};
      if (step >= kChunk - 3) slots[0] = KC_AL + 2 * (kChunk - step);
      if (step >= sub - 3 && step <= sub) slots[1] = KC_AS + 2 * (sub - step);
      if (step == 2 * sub) slots[2] = KC_A2S;
      if (step == 3 * sub) slots[3] = KC_A3S;
      for (int s = 0; s < 4; ++s) {
        if (slots[s] < 0) continue;
        k[slots[s] * M + m] = (float)pr;
        k[(slots[s] + 1) * M + m] = (float)pi;
      }
    }
    k[m] = z.a_re;
    k[M + m] = z.a_im;
  }
}

// ---------------------------------------------------------------- shared-memory plans
template <int D, int M>
struct ReaderPlan {
  static_assert(D % 32 == 0 && M % 8 == 0 && M <= 64 && D <= 256, "shape");
  static constexpr int SLAB_AD = 128 * 16;
  static constexpr int AD_BYTES = 2 * (D / 8) * SLAB_AD;
  static constexpr int SLAB_V = kXRows * 16;  // stream tile: K-major slabs of 8 channels (one TMA box)
  static constexpr int V_BYTES = (D / 8) * SLAB_V;  // (the next item's after the conv)
  static constexpr int SLAB_XH = kChunk * 16;
  // xhat slab, then (once the drive GEMM has read it) the scan scratch
  static constexpr int XH_BYTES = cmax((D / 8) * SLAB_XH, ScanLayout<4>::FLOATS * 4);
  static constexpr int OFF_AD = 0;
  static constexpr int OFF_V = OFF_AD + AD_BYTES;
  static constexpr int OFF_XH = OFF_V + V_BYTES;
  static constexpr int OFF_PAR = OFF_XH + XH_BYTES;               // float [7][D]: w(5), bias, g
  static constexpr int OFF_K = OFF_PAR + 7 * D * 4;
  static constexpr int OFF_RED = OFF_K + kConsts * M * 4;
  static constexpr int OFF_MISC = OFF_RED + 2 * kChunk * 4;
  static constexpr int BYTES = OFF_MISC + 64;
  // at most two CTAs per SM so that two 256-column TMEM allocations always fit
  static constexpr int LAUNCH_BYTES = cmax(BYTES, 100 * 1024);
  static constexpr int TMEM_COLS = 256;  // [0,128) u re, [128,256) u im
  static_assert(2 * (LAUNCH_BYTES + 1024) <= 228 * 1024, "two reader CTAs must fit one SM");
  static_assert(OFF_V % 128 == 0 && SLAB_V % 128 == 0, "TMA destinations must be 128-byte aligned");
};

struct FusedArgs {
  CUtensorMap tmap;         // 3-D map of `in` ([B][T][W] bf16), box 8 x 144 x 1
  const __nv_bfloat16 *in;  // writer: x [B,T,C]; reader: stream [B,T,D]
  int64_t B, T;
  int64_t n_chunks;
  const __nv_bfloat16 *q, *drive, *syn;
  const float *consts;      // kConsts * M floats of this block
  const float *conv_w, *conv_b, *norm, *ds, *ls;
  __nv_bfloat16 *out;       // writer stream
  double *rowsum;           // this block's per-row moment sums [B][7M]
  unsigned long long *rec;  // [B * nch][2][4][2][M] tagged look-back records
  uint32_t epoch;           // host part of this call's record tag (per-process seed)
  const uint32_t *epoch_word;  // device part (per-call counter, see record_tag)
  uint32_t read_xor;        // 0; nonzero only under the look-back miss test hook
  uint32_t spin_limit;      // polls before a look-back wait gives up
  uint32_t *counter;
  uint32_t *error;
  int trace;       // 1: accumulate per-phase cycles of CTA thread 0 into g_fused_trace
  int kernel_id;   // 0 writer, 1 reader
};

// Per-phase cycle totals of thread 0 of every CTA (tracing; off by default).
// Slots: 0 claim, 1 tile load, 2 first GEMM wait, 3 token epilogue, 4 drive GEMM
// wait, 5 scan (whole), 6 synthesis wait, 7 residual epilogue, 8 look-backs
// resolved by the prefetched record, 9 look-backs (chunk > 0), 10 scan pass 1,
// 11 look-back, 12 scan pass 2, 15 items processed.
static __device__ unsigned long long g_fused_trace[2][16];

#define LNET_TRACE(slot)                                                        \
  do {                                                                          \
    if (a.trace && threadIdx.x == 0) {                                          \
      unsigned long long _now = clock64();                                      \
      atomicAdd(&g_fused_trace[a.kernel_id][slot], _now - t_last);              \
      t_last = _now;                                                            \
    }                                                                           \
  } while (0)

// 16-byte copy of prepared operands into shared memory.
__device__ __forceinline__ void copy_smem(void *dst, const void *src, int bytes) {
  const uint4 *s = reinterpret_cast<const uint4 *>(src);
  uint4 *d = reinterpret_cast<uint4 *>(dst);
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = __ldg(s + i);
}
__device__ __forceinline__ void copy_floats(float *dst, const float *src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldg(src + i);
}

// Eight bf16 (one 16-byte vector) -> float, exactly: a bf16 is the upper half
// of the float with the same value, so the widening is a shift or a mask on
// the integer pipe instead of a conversion instruction.
__device__ __forceinline__ void bf16x8_to_float(const uint4 &v, float *f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Two floats -> packed bf16x2 (a in the low half), round to nearest even.
// (An integer-arithmetic rounding measured slower: the conversion pipe is not
// the limit here.)
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}


// SiLU for the bf16 route: v/2 + (v/2) tanh(v/2) with one tanh.approx, i.e.
// one multi-function-unit operation per element instead of an exponential and
// a reciprocal (the epilogues are bound by that unit: 9 % faster end to end).
// Absolute error ~|v| 2^-11, below the bf16 rounding of the stored activation.
// LNET_SILU_EXP2 selects the exponential form (relative error ~1e-6).
__device__ __forceinline__ float silu_fast(float v) {
#if defined(LNET_SILU_EXP2)
  return __fdividef(v, 1.0f + __expf(-v));
#else
  const float h = 0.5f * v;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
#endif
}

__device__ __forceinline__ void cmac(float ar, float ai, float br, float bi, float &cr,
                                     float &ci) {  // c += a * b
  cr = fmaf(ar, br, fmaf(-ai, bi, cr));
  ci = fmaf(ar, bi, fmaf(ai, br, ci));
}

// Tag of one call's look-back records: the workspace's call counter (advanced
// on the device at the end of every call, so eager calls and replays of a
// captured graph alike never reuse a tag within a workspace's lifetime, until
// the 32-bit counter wraps) XOR a per-process seed (so that data that other
// uses of the memory left behind does not read as records).  Never 0:
// zero-filled memory must not read as a published record.
__device__ __forceinline__ uint32_t record_tag(uint32_t host_seed, const uint32_t *epoch_word) {
  const uint32_t t = host_seed ^ __ldcg(epoch_word);
  return t == 0u ? 0x5BD1E995u : t;
}

// Tagged look-back words: (fp32 bits) | (epoch << 32), written and read as one
// 64-bit access (single-copy atomic), so a reader that sees this call's epoch
// also sees the value written with it -- no flags and no fences are needed.
__device__ __forceinline__ void st_tag(unsigned long long *p, float v, uint32_t epoch) {
  __stcg(p, ((unsigned long long)epoch << 32) | __float_as_uint(v));
}
__device__ __forceinline__ bool ld_tag(const unsigned long long *p, uint32_t epoch, float &v) {
  const unsigned long long x = __ldcg(p);
  v = __uint_as_float((uint32_t)x);
  return (uint32_t)(x >> 32) == epoch;
}

// ---------------------------------------------------------------- scan + look-back
// Executed by the 256 threads of one item stream (local thread id `ltid`).
// NSUB = 4 (writer and reader): the drive operand repeats the mode rows every
//   64 lanes, so local warp w reads lane quarter w % 4 = modes 32 * (w % 2) +
//   lane of sub-chunk q = (w % 4) / 2 + 2 * (w / 4): all four SM sub-partitions
//   scan.
// NSUB = 2 (drive rows in lanes 0..63 only): local warps with w % 4 < 2 scan
//   modes 32 * (w % 4) + lane of sub-chunk q = w / 4; the others only join the
//   barriers.
// Sub-chunk q covers steps [SUB q, SUB q + SUB), SUB = 128 / NSUB.  u_re / u_im
// live in TMEM columns [col_re, col_re + 128) / [col_im, ...).  Writes the chunk's
// moment partial sums [7][M] to the row's sums `rowsum` (or leaves the
// per-sub-chunk sums in `mom_out` for the caller to add with reduce_moments).

// Named barrier over one 256-thread item stream.  The non-aligned form counts
// threads, so it stays correct when a warp reaches it diverged (e.g. after a
// single-lane MMA issue); the aligned `bar.sync` would count each divergent
// part of a warp as a separate warp arrival.
__device__ __forceinline__ void group_sync(int id) {
  asm volatile("barrier.sync %0, 256;" ::"r"(id) : "memory");
}

// The previous chunk's inclusive record, loaded by the publishing threads
// before the scan starts (its producer has usually finished by then), so the
// look-back costs no memory round trip when the tags already match.
struct LookbackPrefetch {
  unsigned long long w[8];  // [state k][re | im] of the inclusive record
};

template <int M, int NSUB>
__device__ __forceinline__ void lookback_prefetch(int ltid, const unsigned long long *rec,
                                                  int64_t row, int64_t chunk, int64_t n_chunks,
                                                  LookbackPrefetch &p) {
  const int lwarp = ltid >> 5, lane = ltid & 31, Q = lwarp & 3;
  int q, m;
  bool scanner;
  if constexpr (NSUB == 4) {
    q = (Q >> 1) + 2 * (lwarp >> 2);
    m = 32 * (Q & 1) + lane;
    scanner = true;
  } else {
    q = lwarp >> 2;
    m = 32 * Q + lane;
    scanner = Q < 2;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) p.w[k] = 0ull;
  if (scanner && q == NSUB - 1 && m < M && chunk > 0) {
    const unsigned long long *pv = rec + (row * n_chunks + chunk - 1) * 16 * M + 8 * M + m;
    // volatile: issued here, not sunk to the first use behind the scan's barriers
#pragma unroll
    for (int k = 0; k < 8; ++k)
      asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(p.w[k]) : "l"(pv + k * M));
  }
}

template <int M, bool WRITE_STATES, int NSUB>
__device__ __forceinline__ void chunk_scan(int ltid, int bar_group, int bar_lb, uint32_t tbase,
                                           int col_re, int col_im, int n, int64_t row,
                                           int64_t chunk, int64_t n_chunks, const float *K,
                                           unsigned long long *rec, uint32_t host_epoch,
                                           const uint32_t *epoch_word, uint32_t read_xor,
                                           uint32_t spin, uint32_t *error,
                                           uint8_t *s_slab, int slab_s, float *sc,
                                           double *rowsum, int trace, int kid,
                                           const LookbackPrefetch &pre,
                                           float *mom_out = nullptr) {
  using L = ScanLayout<NSUB>;
  constexpr int SUB = L::SUB;
  unsigned long long t_scan = trace ? clock64() : 0;
  auto mark = [&](int slot) {
    if (trace && threadIdx.x == 0) {
      unsigned long long now = clock64();
      atomicAdd(&g_fused_trace[kid][slot], now - t_scan);
      t_scan = now;
    }
  };
  const int lwarp = ltid >> 5, lane = ltid & 31;
  const int Q = lwarp & 3;
  int q, m;
  bool scanner;
  if constexpr (NSUB == 4) {
    q = (Q >> 1) + 2 * (lwarp >> 2);
    m = 32 * (Q & 1) + lane;
    scanner = true;
  } else {
    q = lwarp >> 2;
    m = 32 * Q + lane;
    scanner = Q < 2;
  }
  const bool live = scanner && m < M;
  const int mk = live ? m : 0;
  const bool publisher_group = scanner && q == NSUB - 1;
  const uint32_t lane_addr = tbase + ((uint32_t)(32 * Q) << 16);
  const int s0 = SUB * q;
  const int len = scanner ? max(0, min(SUB, n - s0)) : 0;
  const float ar = K[mk], ai = K[M + mk];

  // ---- pass 1: sub-chunk local scan from zero (32-step pieces: 4 TMEM loads, one wait)
  float sr = 0.f, si = 0.f;
  float l_r[4] = {0, 0, 0, 0}, l_i[4] = {0, 0, 0, 0};  // l[0] = last state
  for (int c0 = 0; c0 < len; c0 += 32) {
    float ur[32], ui[32];
    sm100::tmem_ld16(lane_addr + col_re + s0 + c0, ur);
    sm100::tmem_ld16(lane_addr + col_re + s0 + c0 + 16, ur + 16);
    sm100::tmem_ld16(lane_addr + col_im + s0 + c0, ui);
    sm100::tmem_ld16(lane_addr + col_im + s0 + c0 + 16, ui + 16);
    sm100::tmem_ld_wait();
    if (c0 + 32 <= len) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float nr = fmaf(ar, sr, fmaf(-ai, si, ur[i]));
        float ni = fmaf(ai, sr, fmaf(ar, si, ui[i]));
        sr = nr;
        si = ni;
        if (i >= 28) {
          l_r[31 - i] = sr;
          l_i[31 - i] = si;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (c0 + i < len) {
          float nr = fmaf(ar, sr, fmaf(-ai, si, ur[i]));
          float ni = fmaf(ai, sr, fmaf(ar, si, ui[i]));
          sr = nr;
          si = ni;
          l_r[3] = l_r[2]; l_i[3] = l_i[2];
          l_r[2] = l_r[1]; l_i[2] = l_i[1];
          l_r[1] = l_r[0]; l_i[1] = l_i[0];
          l_r[0] = sr; l_i[0] = si;
        }
      }
    }
  }
  if (live) {
    sc[L::END + (2 * q) * 64 + m] = sr;
    sc[L::END + (2 * q + 1) * 64 + m] = si;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sc[L::LAST + (8 * q + 2 * k) * 64 + m] = l_r[k];
      sc[L::LAST + (8 * q + 2 * k + 1) * 64 + m] = l_i[k];
    }
  }
  group_sync(bar_group);
  mark(10);
  // chunk-local state before sub-chunk j: c_0 = 0, c_{j+1} = a^SUB c_j + e_j
  // (all end states loaded at once, then the short dependent chain)
  const float asr = K[KC_AS * M + mk], asi = K[(KC_AS + 1) * M + mk];
  float cr = 0.f, ci = 0.f, cpr = 0.f, cpi = 0.f;  // c_q and c_{q-1}
  float e_r[NSUB - 1], e_i[NSUB - 1];
#pragma unroll
  for (int j = 0; j < NSUB - 1; ++j) {
    e_r[j] = j < q ? sc[L::END + (2 * j) * 64 + mk] : 0.f;
    e_i[j] = j < q ? sc[L::END + (2 * j + 1) * 64 + mk] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < NSUB - 1; ++j) {
    if (j < q) {
      cpr = cr;
      cpi = ci;
      float nr = e_r[j], ni = e_i[j];
      cmac(asr, asi, cr, ci, nr, ni);
      cr = nr;
      ci = ni;
    }
  }

  // ---- aggregate, look-back and inclusive record: threads of the last sub-chunk.
  // Record layout per item: [agg | incl][state k = 0..3][re | im][M]; state 0 is
  // the chunk's last state.
  if (publisher_group && live) {
    const uint32_t epoch = record_tag(host_epoch, epoch_word);  // this call's record tag
    const uint32_t rtag = epoch ^ read_xor;  // the tag looked for (== epoch outside tests)
    const int64_t item = row * n_chunks + chunk;  // record index (row-major)
    unsigned long long *my = rec + item * 16 * M;
    float g_r[4], g_i[4];  // chunk-local last four states
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      g_r[k] = l_r[k];
      g_i[k] = l_i[k];
      cmac(K[(KC_AS + 2 * k) * M + m], K[(KC_AS + 2 * k + 1) * M + m], cr, ci, g_r[k], g_i[k]);
      st_tag(my + (2 * k) * M + m, g_r[k], epoch);
      st_tag(my + (2 * k + 1) * M + m, g_i[k], epoch);
    }
    float p_r[4] = {0, 0, 0, 0}, p_i[4] = {0, 0, 0, 0};
    if (chunk > 0) {
      const unsigned long long *pv = rec + (item - 1) * 16 * M;
      const float aLr = K[KC_AL * M + m], aLi = K[(KC_AL + 1) * M + m];
      bool done = true;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const unsigned long long xr = pre.w[2 * k], xi = pre.w[2 * k + 1];
        done &= (uint32_t)(xr >> 32) == rtag && (uint32_t)(xi >> 32) == rtag;
        p_r[k] = __uint_as_float((uint32_t)xr);
        p_i[k] = __uint_as_float((uint32_t)xi);
      }
      if (trace && m == 0) {
        atomicAdd(&g_fused_trace[kid][9], 1ull);
        if (done) atomicAdd(&g_fused_trace[kid][8], 1ull);
      }
      for (uint32_t it = 0; it < spin && !done; ++it) {
        bool ok = true;  // inclusive record of the previous chunk
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          ok &= ld_tag(pv + 8 * M + (2 * k) * M + m, rtag, p_r[k]);
          ok &= ld_tag(pv + 8 * M + (2 * k + 1) * M + m, rtag, p_i[k]);
        }
        if (ok) {
          done = true;
          break;
        }
        ok = true;  // its aggregate, completed by the true end X of chunk - 2
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          ok &= ld_tag(pv + (2 * k) * M + m, rtag, p_r[k]);
          ok &= ld_tag(pv + (2 * k + 1) * M + m, rtag, p_i[k]);
        }
        if (!ok) {
          __nanosleep(32);
          continue;
        }
        float xr = 0.f, xi = 0.f, mr = 1.f, mi = 0.f;
        bool walk_ok = true;
        for (int64_t qq = chunk - 2; qq >= 0 && walk_ok; --qq) {
          const unsigned long long *qv = rec + (row * n_chunks + qq) * 16 * M;
          bool found = false;
          for (uint32_t jt = 0; jt < spin; ++jt) {
            float er, ei;
            if (ld_tag(qv + 8 * M + m, rtag, er) && ld_tag(qv + 9 * M + m, rtag, ei)) {
              cmac(mr, mi, er, ei, xr, xi);
              qq = -1;  // inclusive: the walk ends here
              found = true;
              break;
            }
            if (ld_tag(qv + m, rtag, er) && ld_tag(qv + M + m, rtag, ei)) {
              cmac(mr, mi, er, ei, xr, xi);
              float nr = mr * aLr - mi * aLi, ni = mr * aLi + mi * aLr;
              mr = nr;
              mi = ni;
              found = true;
              break;
            }
            __nanosleep(32);
          }
          if (!found) walk_ok = false;
        }
        if (!walk_ok) break;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          cmac(K[(KC_AL + 2 * k) * M + m], K[(KC_AL + 2 * k + 1) * M + m], xr, xi, p_r[k],
               p_i[k]);
        done = true;
      }
      if (!done) {
        atomicOr(error, kErrLookback << kid);
#pragma unroll
        for (int k = 0; k < 4; ++k) p_r[k] = p_i[k] = 0.f;
      }
    }
    // inclusive record (only consumed when the chunk is full)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float vr = g_r[k], vi = g_i[k];
      cmac(K[(KC_AL + 2 * k) * M + m], K[(KC_AL + 2 * k + 1) * M + m], p_r[0], p_i[0], vr, vi);
      st_tag(my + 8 * M + (2 * k) * M + m, vr, epoch);
      st_tag(my + 8 * M + (2 * k + 1) * M + m, vi, epoch);
      sc[L::CARRY + (2 * k) * 64 + m] = p_r[k];
      sc[L::CARRY + (2 * k + 1) * 64 + m] = p_i[k];
    }
  }
  group_sync(bar_group);
  mark(11);

  // ---- pass 2 from the true state before this sub-chunk
  const float car = sc[L::CARRY + mk], cai = sc[L::CARRY + 64 + mk];
  // a^(SUB q) and a^(SUB (q - 1))
  float pqr = 1.f, pqi = 0.f, pq1r = 1.f, pq1i = 0.f;
  if (q == 1) { pqr = asr; pqi = asi; }
  if (q == 2) { pqr = K[KC_A2S * M + mk]; pqi = K[(KC_A2S + 1) * M + mk]; pq1r = asr; pq1i = asi; }
  if (q == 3) {
    pqr = K[KC_A3S * M + mk]; pqi = K[(KC_A3S + 1) * M + mk];
    pq1r = K[KC_A2S * M + mk]; pq1i = K[(KC_A2S + 1) * M + mk];
  }
  float h_r[4], h_i[4];  // true states at the four steps before this sub-chunk
  if (q == 0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h_r[k] = sc[L::CARRY + (2 * k) * 64 + mk];
      h_i[k] = sc[L::CARRY + (2 * k + 1) * 64 + mk];
    }
  } else {
    float ipr = cpr, ipi = cpi;  // true state before sub-chunk q - 1
    cmac(pq1r, pq1i, car, cai, ipr, ipi);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h_r[k] = sc[L::LAST + (8 * (q - 1) + 2 * k) * 64 + mk];
      h_i[k] = sc[L::LAST + (8 * (q - 1) + 2 * k + 1) * 64 + mk];
      cmac(K[(KC_AS + 2 * k) * M + mk], K[(KC_AS + 2 * k + 1) * M + mk], ipr, ipi, h_r[k],
           h_i[k]);
    }
  }
  sr = cr;
  si = ci;
  cmac(pqr, pqi, car, cai, sr, si);
  // History before the sequence start is exactly zero (the carry of chunk 0 is
  // zero), so lag products that reach before step 0 contribute nothing and
  // need no guard; the counts T - lag are applied when the moments are finalised.
  float h1r = h_r[0], h1i = h_i[0], h2r = h_r[1], h2i = h_i[1];
  float h3r = h_r[2], h3i = h_i[2], h4r = h_r[3], h4i = h_i[3];
  float e = 0.f, c1r = 0.f, c1i = 0.f, c2r = 0.f, c2i = 0.f, c4r = 0.f, c4i = 0.f;
  auto step2 = [&](float u_re, float u_im) {
    float nr = fmaf(ar, sr, fmaf(-ai, si, u_re));
    float ni = fmaf(ai, sr, fmaf(ar, si, u_im));
    sr = nr;
    si = ni;
    e = fmaf(sr, sr, fmaf(si, si, e));
    c1r = fmaf(sr, h1r, fmaf(si, h1i, c1r));
    c1i = fmaf(si, h1r, fmaf(-sr, h1i, c1i));
    c2r = fmaf(sr, h2r, fmaf(si, h2i, c2r));
    c2i = fmaf(si, h2r, fmaf(-sr, h2i, c2i));
    c4r = fmaf(sr, h4r, fmaf(si, h4i, c4r));
    c4i = fmaf(si, h4r, fmaf(-sr, h4i, c4i));
    h4r = h3r; h4i = h3i;
    h3r = h2r; h3i = h2i;
    h2r = h1r; h2i = h1i;
    h1r = sr; h1i = si;
  };
  // State slab for the synthesis GEMM, M-major (steps contiguous): element
  // (t, j) at (j / 8) * slab_s + (t / 8) * 128 + (j % 8) * 16 + (t % 8) * 2.
  auto s_addr = [&](int t, int j) {
    return s_slab + (j / 8) * slab_s + (t / 8) * 128 + (j % 8) * 16 + (t % 8) * 2;
  };
  for (int c0 = 0; c0 < len; c0 += 32) {
    float ur[32], ui[32];
    sm100::tmem_ld16(lane_addr + col_re + s0 + c0, ur);
    sm100::tmem_ld16(lane_addr + col_re + s0 + c0 + 16, ur + 16);
    sm100::tmem_ld16(lane_addr + col_im + s0 + c0, ui);
    sm100::tmem_ld16(lane_addr + col_im + s0 + c0 + 16, ui + 16);
    sm100::tmem_ld_wait();
    if (c0 + 32 <= len) {
#pragma unroll
      for (int g8 = 0; g8 < 4; ++g8) {
        float br[8], bi[8];
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) {
          step2(ur[8 * g8 + i8], ui[8 * g8 + i8]);
          br[i8] = sr;
          bi[i8] = si;
        }
        if constexpr (WRITE_STATES) {
          if (live) {
            const int t = s0 + c0 + 8 * g8;
            uint4 vr, vi;
            vr.x = pack_bf16x2(br[0], br[1]); vr.y = pack_bf16x2(br[2], br[3]);
            vr.z = pack_bf16x2(br[4], br[5]); vr.w = pack_bf16x2(br[6], br[7]);
            vi.x = pack_bf16x2(bi[0], bi[1]); vi.y = pack_bf16x2(bi[2], bi[3]);
            vi.z = pack_bf16x2(bi[4], bi[5]); vi.w = pack_bf16x2(bi[6], bi[7]);
            *reinterpret_cast<uint4 *>(s_addr(t, m)) = vr;
            *reinterpret_cast<uint4 *>(s_addr(t, M + m)) = vi;
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (c0 + i < len) {
          step2(ur[i], ui[i]);
          if constexpr (WRITE_STATES) {
            if (live) {
              const int t = s0 + c0 + i;
              *reinterpret_cast<__nv_bfloat16 *>(s_addr(t, m)) = __float2bfloat16_rn(sr);
              *reinterpret_cast<__nv_bfloat16 *>(s_addr(t, M + m)) = __float2bfloat16_rn(si);
            }
          }
        }
      }
    }
  }
  mark(12);
  // moment partials per sub-chunk: [NSUB][7][64], reduced below, or by the
  // caller from `mom_out` after its own barrier (no extra barrier here)
  if (live) {
    float *mo = (mom_out ? mom_out : sc + L::MOM) + q * 7 * 64 + m;
    mo[0] = e;
    mo[64] = c1r;
    mo[128] = c1i;
    mo[192] = c2r;
    mo[256] = c2i;
    mo[320] = c4r;
    mo[384] = c4i;
  }
  if (mom_out) return;
  group_sync(bar_group);
  for (int j = ltid; j < 7 * M; j += 256) {
    const int k = j / M, mm = j - (j / M) * M;
    const float *mo = sc + L::MOM + k * 64 + mm;
    float acc = 0.f;
#pragma unroll
    for (int qq = 0; qq < NSUB; ++qq) acc += mo[qq * 7 * 64];
    atomicAdd(rowsum + j, (double)acc);
  }
}

// Adds the per-sub-chunk moment partials [NSUB][7][64] of one chunk to the
// row's sums rowsum[7][M].
template <int M, int NSUB>
__device__ __forceinline__ void reduce_moments(int ltid, const float *mom, double *rowsum) {
  for (int j = ltid; j < 7 * M; j += kFusedThreads) {
    const int k = j / M, mm = j - (j / M) * M;
    float acc = 0.f;
#pragma unroll
    for (int qq = 0; qq < NSUB; ++qq) acc += mom[qq * 7 * 64 + k * 64 + mm];
    atomicAdd(rowsum + j, (double)acc);
  }
}

// Issues one GEMM: `ksteps` K=16 steps of D[tmem] (+)= A * B^T.
__device__ __forceinline__ void issue_gemm(uint32_t d_tmem, uint32_t a_addr, int a_slab,
                                           uint32_t b_addr, int b_slab, int ksteps,
                                           uint32_t idesc, bool accumulate_first) {
  for (int kk = 0; kk < ksteps; ++kk) {
    uint64_t ad = sm100::make_desc(a_addr + 2 * kk * a_slab, a_slab, 128);
    uint64_t bd = sm100::make_desc(b_addr + 2 * kk * b_slab, b_slab, 128);
    sm100::mma_bf16(d_tmem, ad, bd, idesc, (accumulate_first || kk > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ void wait_mma(uint64_t *mbar, uint32_t &phase, uint32_t *error,
                                         uint32_t site) {
  if (!sm100::mbar_wait_bounded(mbar, phase, kSpinLimit)) {
    if (threadIdx.x % 256 == 0) atomicOr(error, 1u << site);
  }
  phase ^= 1u;
  sm100::tc_fence_after();
}

// ---------------------------------------------------------------- writer kernel
// One CTA of 512 threads per SM runs two independent item streams (threads
// [0, 256) and [256, 512)).  The streams share the weight operands in shared
// memory; each owns half of the TMEM columns, an mbarrier, named barriers and
// its tile buffers, so one stream's GEMM waits, look-back and global-memory
// latencies overlap the other stream's arithmetic.
constexpr int kWriterStreams = 2;

template <int C, int D, int M>
struct WriterPlan {
  static_assert(C % 16 == 0 && D % 32 == 0 && M % 8 == 0 && M <= 64 && D <= 256, "shape");
  // shared by both streams
  static constexpr int SLAB_AD = 128 * 16;  // drive A rows: modes repeated every 64 lanes
  static constexpr int AD_BYTES = 2 * (D / 8) * SLAB_AD;
  static constexpr int SLAB_Q = D * 16;
  static constexpr int Q_BYTES = kTaps * (C / 8) * SLAB_Q;
  static constexpr int SLAB_WS = D * 16;
  static constexpr int WS_BYTES = (2 * M / 8) * SLAB_WS;
  static constexpr int OFF_AD = 0;
  static constexpr int OFF_Q = OFF_AD + AD_BYTES;
  static constexpr int OFF_WS = OFF_Q + Q_BYTES;
  static constexpr int OFF_PAR = OFF_WS + WS_BYTES;            // float [4][D]: bias, g, ds, ls
  static constexpr int OFF_K = OFF_PAR + 4 * D * 4;            // float [kConsts * M]
  static constexpr int SHARED_END = (OFF_K + kConsts * M * 4 + 127) / 128 * 128;
  // per stream
  static constexpr int SLAB_X = kXRows * 16;  // one TMA box; 128-byte multiple
  static constexpr int X_BYTES = cmax((C / 8) * SLAB_X, ScanLayout<kWriterNSub>::FLOATS * 4);
  static constexpr int SLAB_XH = kChunk * 16;
  static constexpr int SLAB_S = kChunk * 16;  // state slab: one 8-column K group, M-major
  static constexpr int XS_BYTES = cmax((D / 8) * SLAB_XH, (2 * M / 8) * SLAB_S);
  static constexpr int G_X = 0;                       // x tile, scan scratch, next x tile
  static constexpr int G_XS = G_X + X_BYTES;          // xhat slab, then state slab
  static constexpr int G_RED = G_XS + XS_BYTES;       // float [2][128]
  static constexpr int G_RS = G_RED + 2 * kChunk * 4; // float [128]
  static constexpr int G_MOM = G_RS + kChunk * 4;     // float [NSUB][7][64] moment partials
  static constexpr int G_MISC = G_MOM + kWriterNSub * 7 * 64 * 4;  // mbar, item
  static constexpr int G_BYTES = (G_MISC + 64 + 127) / 128 * 128;
  static constexpr int OFF_TMEM_SLOT = SHARED_END + kWriterStreams * G_BYTES;
  static constexpr int BYTES = OFF_TMEM_SLOT + 16;
  static constexpr int TMEM_COLS = 512;  // 256 per stream: u re [0,128), u im [128,256);
                                         // stem and synthesis accumulators reuse [0, D)
  static_assert(BYTES <= 232448, "writer shared memory exceeds 227 KB");
  static_assert(SLAB_X % 128 == 0 && SHARED_END % 128 == 0 && G_BYTES % 128 == 0,
                "TMA destinations must be 128-byte aligned");
};

template <int C, int D, int M>
__global__ void __launch_bounds__(kFusedThreads * kWriterStreams, 1)
    fused_writer_kernel(const __grid_constant__ FusedArgs a) {
  using P = WriterPlan<C, D, M>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int g = tid / kFusedThreads, ltid = tid % kFusedThreads;
  const int lwarp = ltid >> 5, lane = ltid & 31;
  uint8_t *gs = smem + P::SHARED_END + g * P::G_BYTES;
  uint64_t *mbar = reinterpret_cast<uint64_t *>(gs + P::G_MISC);
  int64_t *item_slot = reinterpret_cast<int64_t *>(gs + P::G_MISC + 8);  // [2]
  uint64_t *tbar = reinterpret_cast<uint64_t *>(gs + P::G_MISC + 24);     // x tile arrival
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + P::OFF_TMEM_SLOT);
  float *red = reinterpret_cast<float *>(gs + P::G_RED);
  float *rs_s = reinterpret_cast<float *>(gs + P::G_RS);
  float *s_mom = reinterpret_cast<float *>(gs + P::G_MOM);
  float *par = reinterpret_cast<float *>(smem + P::OFF_PAR);
  const float *s_bias = par, *s_norm = par + D, *s_ds = par + 2 * D, *s_ls = par + 3 * D;
  float *s_k = reinterpret_cast<float *>(smem + P::OFF_K);
  float *s_scan = reinterpret_cast<float *>(gs + P::G_X);  // x tile is dead during the scan
  const uint32_t s_base = sm100::smem_u32(smem);
  const uint32_t g_base = sm100::smem_u32(gs);
  const int bar_group = 1 + g, bar_lb = 3 + g;

  if (ltid == 0) {
    sm100::mbar_init(mbar, 1);
    sm100::mbar_init(tbar, 1);
    sm100::fence_barrier_init();
  }
  if (tid < 32) {
    sm100::tmem_alloc(tmem_slot, P::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  copy_smem(smem + P::OFF_AD, a.drive, P::AD_BYTES);
  copy_smem(smem + P::OFF_Q, a.q, P::Q_BYTES);
  copy_smem(smem + P::OFF_WS, a.syn, P::WS_BYTES);
  copy_floats(par, a.conv_b, D);
  copy_floats(par + D, a.norm, D);
  copy_floats(par + 2 * D, a.ds, D);
  copy_floats(par + 3 * D, a.ls, D);
  copy_floats(s_k, a.consts, kConsts * M);
  sm100::fence_proxy_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tmem_slot + 256u * g;
  uint32_t phase = 0;
  const int row = 32 * (lwarp & 3) + lane;  // step within the chunk (TMEM lane)
  const int half = lwarp >> 2;              // column half of the token-major epilogues
  constexpr int HD = D / 2;
  const uint32_t lane_addr = tbase + ((uint32_t)(32 * (lwarp & 3)) << 16);
  const int64_t total = a.B * a.n_chunks;
  if (a.trace && ltid == 0) atomicAdd(&g_fused_trace[a.kernel_id][13], 1ull);

  unsigned long long t_last = clock64();
  // Items are claimed one ahead (alternating slots): iteration k processes
  // item_slot[k & 1] and claims the next into item_slot[(k + 1) & 1].
  // The x tile of an item is fetched one item ahead by TMA (one 8-channel box
  // of rows [t0 - 8, t0 + 136) per K slab, zero outside [0, T)) into the x
  // region, free once the previous item's scan has finished.  Thread 0 only.
  uint32_t tphase = 0;
  auto issue_tile = [&](int64_t it) {
    const int64_t ch = (uint32_t)it / (uint32_t)a.B, bb = it - ch * a.B;  // items < 2^31
    sm100::mbar_arrive_expect_tx(tbar, (C / 8) * kXRows * 16);
#pragma unroll
    for (int kc = 0; kc < C / 8; ++kc)
      sm100::tma_load_3d(g_base + P::G_X + kc * P::SLAB_X, &a.tmap, tbar, kc * 8,
                         (int)(ch * kChunk - kHalo), (int)bb);
  };
  if (ltid == 0) item_slot[0] = (int64_t)atomicAdd(a.counter, 1u);
  group_sync(bar_group);
  if (ltid == 0 && item_slot[0] < total) issue_tile(item_slot[0]);
  for (int iter = 0;; ++iter) {
    const int64_t item = item_slot[iter & 1];
    if (item >= total) break;
    LNET_TRACE(0);
    const int64_t chunk = (uint32_t)item / (uint32_t)a.B, b = item - chunk * a.B;
    const int64_t t0 = chunk * kChunk;
    const int n = (int)min((int64_t)kChunk, a.T - t0);
    __nv_bfloat16 *out_row = a.out + ((b * a.T + t0 + row) * D + half * HD);

    LNET_TRACE(1);
    // 1-2. x tile (TMA, issued one item ahead), then the stem GEMM: five
    // row-shifted views of the tile
    if (ltid == 0) {
      if (!sm100::mbar_wait_bounded(tbar, tphase, kSpinLimit)) atomicOr(a.error, kErrTile);
      tphase ^= 1u;
      sm100::tc_fence_after();
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(128, D);
      for (int k = 0; k < kTaps; ++k)
        issue_gemm(tbase, g_base + P::G_X + 4 * k * 16, P::SLAB_X,
                   s_base + P::OFF_Q + k * (C / 8) * P::SLAB_Q, P::SLAB_Q, C / 16, idesc, k > 0);
      sm100::mma_commit(mbar);
    }
    wait_mma(mbar, phase, a.error, 0);
    LNET_TRACE(2);
    // 3. bias + SiLU + RMSNorm (thread per step, two column halves)
    {
      float f[HD];
#pragma unroll
      for (int j = 0; j < HD / 16; ++j)
        sm100::tmem_ld16(lane_addr + half * HD + 16 * j, f + 16 * j);
      sm100::tmem_ld_wait();
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < HD; ++i) {
        f[i] = silu_fast(f[i] + s_bias[half * HD + i]);
        ss = fmaf(f[i], f[i], ss);
      }
      red[half * kChunk + row] = ss;
      group_sync(bar_group);
      const float rs = rsqrtf((red[row] + red[kChunk + row]) / (float)D + kFp32Eps);
      if (half == 0) rs_s[row] = rs;
#pragma unroll
      for (int gq = 0; gq < HD / 8; ++gq) {
        const int d0 = half * HD + 8 * gq;
        uint4 xh, fl;
        float h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = f[8 * gq + i] * rs * s_norm[d0 + i];
        xh.x = pack_bf16x2(h[0], h[1]);
        xh.y = pack_bf16x2(h[2], h[3]);
        xh.z = pack_bf16x2(h[4], h[5]);
        xh.w = pack_bf16x2(h[6], h[7]);
        fl.x = pack_bf16x2(f[8 * gq + 0], f[8 * gq + 1]);
        fl.y = pack_bf16x2(f[8 * gq + 2], f[8 * gq + 3]);
        fl.z = pack_bf16x2(f[8 * gq + 4], f[8 * gq + 5]);
        fl.w = pack_bf16x2(f[8 * gq + 6], f[8 * gq + 7]);
        *reinterpret_cast<uint4 *>(gs + P::G_XS + (d0 / 8) * P::SLAB_XH + row * 16) = xh;
        // the stem output waits in the output rows (L2) for the residual epilogue
        if (row < n) *reinterpret_cast<uint4 *>(out_row + 8 * gq) = fl;
      }
    }
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    group_sync(bar_group);
    LNET_TRACE(3);
    // 4. drive GEMM, mode-major: lanes = modes, columns = steps (overwrites the stem acc)
    if (ltid == 0) {
      sm100::tc_fence_after();
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(128, 128);
      for (int part = 0; part < 2; ++part)
        issue_gemm(tbase + part * 128, s_base + P::OFF_AD + part * (D / 8) * P::SLAB_AD,
                   P::SLAB_AD, g_base + P::G_XS, P::SLAB_XH, D / 16, idesc, false);
      sm100::mma_commit(mbar);
    }
    // the last thread claims the next item while the drive GEMM runs (off the
    // MMA-issuing thread, whose barrier arrival gates the stream)
    if (ltid == kFusedThreads - 1) item_slot[(iter + 1) & 1] = (int64_t)atomicAdd(a.counter, 1u);
    LookbackPrefetch pre;
    lookback_prefetch<M, kWriterNSub>(ltid, a.rec, b, chunk, a.n_chunks, pre);
    wait_mma(mbar, phase, a.error, 1);
    LNET_TRACE(4);
    // 5. scan + look-back + moments; states -> synthesis A operand (aliases xhat)
    chunk_scan<M, true, kWriterNSub>(ltid, bar_group, bar_lb, tbase, 0, 128, n, b, chunk,
                                     a.n_chunks, s_k, a.rec, a.epoch, a.epoch_word, a.read_xor,
                                     a.spin_limit, a.error,
                                     gs + P::G_XS,
                                     P::SLAB_S, s_scan,
                                     a.rowsum + b * 7 * M, a.trace,
                                     a.kernel_id, pre, s_mom);
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    group_sync(bar_group);
    LNET_TRACE(5);
    // 6. synthesis GEMM (token-major) into columns [0, D); meanwhile the next
    // item's x tile and this row's stem output are fetched
    if (ltid == 0) {
      sm100::tc_fence_after();
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(128, D, /*a_mn_major=*/true);
      issue_gemm(tbase, g_base + P::G_XS, P::SLAB_S, s_base + P::OFF_WS, P::SLAB_WS, 2 * M / 16,
                 idesc, false);
      sm100::mma_commit(mbar);
    }
    if (ltid == kTileIssuer) {
      const int64_t next = item_slot[(iter + 1) & 1];
      if (next < total) issue_tile(next);
    }
    uint4 flv[HD / 8];
    if (row < n) {
#pragma unroll
      for (int gq = 0; gq < HD / 8; ++gq) flv[gq] = *reinterpret_cast<const uint4 *>(out_row + 8 * gq);
    }
    reduce_moments<M, kWriterNSub>(ltid, s_mom, a.rowsum + b * 7 * M);
    wait_mma(mbar, phase, a.error, 2);
    LNET_TRACE(6);
    // 7. residual epilogue: v = fl + ls * (modal + ds * xhat), xhat = fl * rs * g
    {
      float modal[HD];
#pragma unroll
      for (int j = 0; j < HD / 16; ++j)
        sm100::tmem_ld16(lane_addr + half * HD + 16 * j, modal + 16 * j);
      sm100::tmem_ld_wait();
      const float rsr = rs_s[row];
      if (row < n) {
#pragma unroll
        for (int gq = 0; gq < HD / 8; ++gq) {
          const int d0 = half * HD + 8 * gq;
          float fv[8];
          bf16x8_to_float(flv[gq], fv);
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int d = d0 + i;
            const float x = fv[i];
            const float xh = x * rsr * s_norm[d];
            o[i] = x + s_ls[d] * (modal[8 * gq + i] + s_ds[d] * xh);
          }
          uint4 ov;
          ov.x = pack_bf16x2(o[0], o[1]);
          ov.y = pack_bf16x2(o[2], o[3]);
          ov.z = pack_bf16x2(o[4], o[5]);
          ov.w = pack_bf16x2(o[6], o[7]);
          *reinterpret_cast<uint4 *>(out_row + 8 * gq) = ov;
        }
      }
    }
    sm100::tc_fence_before();
    group_sync(bar_group);
    LNET_TRACE(7);
    if (a.trace && tid == 0) atomicAdd(&g_fused_trace[a.kernel_id][15], 1ull);
  }
  if (a.trace && ltid == 0) atomicAdd(&g_fused_trace[a.kernel_id][14], 1ull);
  __syncthreads();
  if (tid < 32) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(*tmem_slot, P::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- reader kernel
template <int D, int M>
__global__ void __launch_bounds__(kFusedThreads, 2)
    fused_reader_kernel(const __grid_constant__ FusedArgs a) {
  using P = ReaderPlan<D, M>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + P::OFF_MISC);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + P::OFF_MISC + 8);
  int64_t *item_slot = reinterpret_cast<int64_t *>(smem + P::OFF_MISC + 16);  // [2]
  uint64_t *tbar = reinterpret_cast<uint64_t *>(smem + P::OFF_MISC + 32);      // tile arrival
  float *red = reinterpret_cast<float *>(smem + P::OFF_RED);
  float *par = reinterpret_cast<float *>(smem + P::OFF_PAR);
  const float *s_w = par, *s_bias = par + kTaps * D, *s_norm = par + (kTaps + 1) * D;
  float *s_k = reinterpret_cast<float *>(smem + P::OFF_K);
  float *s_scan = reinterpret_cast<float *>(smem + P::OFF_XH);  // xhat is dead during the scan
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t s_base = sm100::smem_u32(smem);

  if (tid == 0) {
    sm100::mbar_init(mbar, 1);
    sm100::mbar_init(tbar, 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, P::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  copy_smem(smem + P::OFF_AD, a.drive, P::AD_BYTES);
  // conv weights transposed to [tap][channel]
  for (int i = tid; i < kTaps * D; i += kFusedThreads) {
    const int k = i / D, d = i - (i / D) * D;
    par[i] = __ldg(a.conv_w + d * kTaps + k);
  }
  copy_floats(par + kTaps * D, a.conv_b, D);
  copy_floats(par + (kTaps + 1) * D, a.norm, D);
  copy_floats(s_k, a.consts, kConsts * M);
  sm100::fence_proxy_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  uint32_t phase = 0;
  const int row = 32 * (warp & 3) + lane;
  const int half = warp >> 2;
  constexpr int HD = D / 2;
  const int64_t total = a.B * a.n_chunks;
  if (a.trace && tid == 0) atomicAdd(&g_fused_trace[a.kernel_id][13], 1ull);

  unsigned long long t_last = clock64();
  // Stream tiles are fetched one item ahead by TMA (thread 0; one 8-channel
  // box per K slab), issued as soon as the conv of the current item has read
  // the tile region.
  uint32_t tphase = 0;
  auto issue_tile = [&](int64_t it) {
    const int64_t ch = (uint32_t)it / (uint32_t)a.B, bb = it - ch * a.B;  // items < 2^31
    sm100::mbar_arrive_expect_tx(tbar, (D / 8) * kXRows * 16);
#pragma unroll
    for (int kc = 0; kc < D / 8; ++kc)
      sm100::tma_load_3d(s_base + P::OFF_V + kc * P::SLAB_V, &a.tmap, tbar, kc * 8,
                         (int)(ch * kChunk - kHalo), (int)bb);
  };
  if (tid == 0) item_slot[0] = (int64_t)atomicAdd(a.counter, 1u);
  __syncthreads();
  if (tid == 0 && item_slot[0] < total) issue_tile(item_slot[0]);
  for (int iter = 0;; ++iter) {
    const int64_t item = item_slot[iter & 1];
    if (item >= total) break;
    LNET_TRACE(0);
    const int64_t chunk = (uint32_t)item / (uint32_t)a.B, b = item - chunk * a.B;
    const int64_t t0 = chunk * kChunk;
    const int n = (int)min((int64_t)kChunk, a.T - t0);

    // 1. stream tile rows [t0 - 8, t0 + 136), zero outside [0, T), issued one item ahead
    if (!sm100::mbar_wait_bounded(tbar, tphase, kSpinLimit) && tid == 0)
      atomicOr(a.error, kErrTile << 1);
    tphase ^= 1u;
    // the last thread claims the next item (its latency overlaps the conv)
    if (tid == kFusedThreads - 1) item_slot[(iter + 1) & 1] = (int64_t)atomicAdd(a.counter, 1u);
    LNET_TRACE(1);
    // 2. depthwise conv (K5, dilation 4) + bias + SiLU + RMSNorm
    float f[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) f[i] = s_bias[half * HD + i];
#pragma unroll
    for (int k = 0; k < kTaps; ++k) {
      const uint8_t *src = smem + P::OFF_V + (half * HD / 8) * P::SLAB_V + (row + 4 * k) * 16;
      const float *wk = s_w + k * D + half * HD;
#pragma unroll
      for (int g = 0; g < HD / 8; ++g) {
        const uint4 v = *reinterpret_cast<const uint4 *>(src + g * P::SLAB_V);
        float vv[8];
        bf16x8_to_float(v, vv);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[8 * g + i] = fmaf(wk[8 * g + i], vv[i], f[8 * g + i]);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < HD; ++i) {
      f[i] = silu_fast(f[i]);
      ss = fmaf(f[i], f[i], ss);
    }
    red[half * kChunk + row] = ss;
    __syncthreads();
    if (tid == kTileIssuer) {  // every thread has read the tile: fetch the next item's
      const int64_t next = item_slot[(iter + 1) & 1];
      if (next < total) issue_tile(next);
    }
    const float rs = rsqrtf((red[row] + red[kChunk + row]) / (float)D + kFp32Eps);
#pragma unroll
    for (int g = 0; g < HD / 8; ++g) {
      const int d0 = half * HD + 8 * g;
      float h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = f[8 * g + i] * rs * s_norm[d0 + i];
      uint4 xh;
      xh.x = pack_bf16x2(h[0], h[1]);
      xh.y = pack_bf16x2(h[2], h[3]);
      xh.z = pack_bf16x2(h[4], h[5]);
      xh.w = pack_bf16x2(h[6], h[7]);
      *reinterpret_cast<uint4 *>(smem + P::OFF_XH + (d0 / 8) * P::SLAB_XH + row * 16) = xh;
    }
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    LNET_TRACE(3);
    // 3. drive GEMM (mode-major)
    if (tid == 0) {
      sm100::tc_fence_after();
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(128, 128);
      for (int part = 0; part < 2; ++part)
        issue_gemm(tbase + part * 128, s_base + P::OFF_AD + part * (D / 8) * P::SLAB_AD,
                   P::SLAB_AD, s_base + P::OFF_XH, P::SLAB_XH, D / 16, idesc, false);
      sm100::mma_commit(mbar);
    }
    LookbackPrefetch pre;
    lookback_prefetch<M, 4>(tid, a.rec, b, chunk, a.n_chunks, pre);
    wait_mma(mbar, phase, a.error, 3);
    LNET_TRACE(4);
    // 4. scan + look-back + moments
    chunk_scan<M, false, 4>(tid, 0, 1, tbase, 0, 128, n, b, chunk, a.n_chunks, s_k, a.rec,
                            a.epoch, a.epoch_word, a.read_xor, a.spin_limit, a.error, nullptr,
                            0, s_scan,
                            a.rowsum + b * 7 * M, a.trace, a.kernel_id,
                            pre);
    sm100::tc_fence_before();
    __syncthreads();
    LNET_TRACE(5);
    if (a.trace && tid == 0) atomicAdd(&g_fused_trace[a.kernel_id][15], 1ull);
  }
  if (a.trace && tid == 0) atomicAdd(&g_fused_trace[a.kernel_id][14], 1ull);
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, P::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- moments finalize
// Moment k of the row sums divided by its count (T, or T - lag; 0 if T <= lag).
__device__ __forceinline__ float finalize_moment(const double *rs, int modes, int j,
                                                 int64_t steps) {
  const int k = j / modes;
  if (k == 0) return (float)(rs[j] / (double)steps);
  const int lag = k <= 2 ? 1 : (k <= 4 ? 2 : 4);
  return steps <= lag ? 0.f : (float)(rs[j] / (double)(steps - lag));
}

// One thread per (row, feature): raw moments [b][k*M + m] of both blocks and
// the radial-log features of src/lnet/alphabet.py:29-46 (the arithmetic of
// radial_feature) into feats[b][blk * 7M + j].
// Also advances the workspace's look-back call counter for the next call.
__global__ void fused_finalize_kernel(const double *__restrict__ rowsum, float *__restrict__ wm,
                                      float *__restrict__ rm, float *__restrict__ feats,
                                      int64_t batch, int64_t steps, int modes,
                                      uint32_t *__restrict__ epoch_word) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *epoch_word = *epoch_word + 1u;
  }
  const int W = 7 * modes;
  const int64_t n = batch * 2 * W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / (2 * W);
    const int jj = (int)(i - b * 2 * W), blk = jj >= W ? 1 : 0, j = jj - blk * W;
    const double *rs = rowsum + (blk * batch + b) * W;
    const float v = finalize_moment(rs, modes, j, steps);
    (blk == 0 ? wm : rm)[b * W + j] = v;
    float f;
    if (j < modes) {
      f = log1pf(fmaxf(v, 0.f));
    } else {
      const int pair = (j - modes) / (2 * modes);
      const int within = (j - modes) - pair * 2 * modes;
      const int base = modes + pair * 2 * modes, mm = within % modes;
      const float re = finalize_moment(rs, modes, base + mm, steps);
      const float im = finalize_moment(rs, modes, base + modes + mm, steps);
      const float r = sqrtf(fmaxf(re * re + im * im, kFp32Tiny));
      const float scale = log1pf(r) / r;
      f = scale * (within < modes ? re : im);
    }
    feats[b * 2 * W + jj] = f;
  }
}

// ---------------------------------------------------------------- dispatch
struct FusedShapeKey {
  int C, D, M;
};
constexpr FusedShapeKey kFusedShapes[] = {{48, 96, 48}};

inline bool fused_supported(const lnet_b200_alphabet_params *p,
                            const lnet_b200_alphabet_request *r) {
  if (r->time_delta || r->observation_mask || r->valid_mask) return false;
  if (r->x_dtype != LNET_BF16 || r->act_dtype != LNET_BF16) return false;
  if (p->conv_kernel != kTaps || p->conv_dilation != 4) return false;
  if (r->steps < 1 || r->batch < 1) return false;
  if (reinterpret_cast<uintptr_t>(r->x) % 16 != 0) return false;  // TMA source
  if (r->batch * fused_chunks(r->steps) >= (int64_t)1 << 31) return false;
  if (r->batch * 14 * p->modes >= (int64_t)1 << 31) return false;
  for (const auto &s : kFusedShapes)
    if (s.C == p->raw_input_dim && s.D == p->model_dim && s.M == p->modes) return true;
  return false;
}

int sm_count();
uint32_t process_tag_seed();
int take_lookback_injection();
int fused_trace_enabled();

// Tiled 3-D tensor map of a [B][T][W] bf16 tensor with an 8 x 144 x 1 box
// (one K slab of a tile), zero fill outside the tensor.  The driver entry
// point is resolved once through the runtime.
inline int encode_tile_map(CUtensorMap *map, const void *base, int64_t B, int64_t T, int W) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!encode) return fail(LNET_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)W * 2, (cuuint64_t)T * W * 2};
  const cuuint32_t box[3] = {8, (cuuint32_t)kXRows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return fail(LNET_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)res);
  return LNET_OK;
}

// Writes the prepared operands (bf16 slabs, pole constants) of `p` into `w`.
inline int fused_prepare(const lnet_b200_alphabet_params *p, FusedWorkspace &w, cudaStream_t st) {
  fused_prepare_kernel<<<sm_count(), 256, 0, st>>>(*p, w);
  return after_launch("fused_prepare_kernel");
}

// `prepared`: the operands in `w` were written by fused_prepare for these
// parameters (lnet_b200_alphabet_prepare) and are not rebuilt.
template <int C, int D, int M>
int fused_forward_shape(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                        FusedWorkspace &w, float *wm, float *rm, bool prepared, cudaStream_t st) {
  using WP = WriterPlan<C, D, M>;
  using RP = ReaderPlan<D, M>;
  const int64_t B = r->batch, T = r->steps, nch = fused_chunks(T);
  const int sms = sm_count();
  if (!prepared) LNET_TRY(fused_prepare(p, w, st));
  // per-call state: the row moment sums and, right behind them, counters and error words
  LNET_TRY(cuda_check(cudaMemsetAsync(w.rowsum, 0,
                                      reinterpret_cast<char *>(w.flags + w.flag_words) -
                                          reinterpret_cast<char *>(w.rowsum),
                                      st),
                      "cudaMemsetAsync(row sums, flags)"));
  uint32_t *counters = w.flags;
  FusedArgs wa{};
  wa.in = (const __nv_bfloat16 *)r->x;
  LNET_TRY(encode_tile_map(&wa.tmap, r->x, B, T, C));
  wa.B = B;
  wa.T = T;
  wa.n_chunks = nch;
  wa.q = w.q;
  wa.drive = w.wdrive;
  wa.syn = w.wsyn;
  wa.consts = w.consts;
  wa.conv_b = p->stem_conv_bias;
  wa.norm = p->writer_norm;
  wa.ds = p->writer_direct_scale;
  wa.ls = p->writer_layer_scale;
  wa.out = w.stream;
  wa.rowsum = w.rowsum;
  wa.rec = w.wrec;
  wa.epoch = process_tag_seed();
  wa.read_xor = 0;
  wa.spin_limit = kSpinLimit;
  if (take_lookback_injection()) {  // test hook: every look-back misses and gives up early
    wa.read_xor = 0x80000000u;
    wa.spin_limit = 64;
  }
  wa.epoch_word = w.epoch_word;
  wa.counter = counters;
  wa.error = counters + 2;
  wa.trace = fused_trace_enabled();
  wa.kernel_id = 0;
  LNET_TRY(cuda_check(cudaFuncSetAttribute(fused_writer_kernel<C, D, M>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, WP::BYTES),
                      "cudaFuncSetAttribute(fused_writer_kernel)"));
  const int64_t items = B * nch;
  fused_writer_kernel<C, D, M><<<(unsigned)std::min<int64_t>(cdiv(items, kWriterStreams), sms),
                                 kFusedThreads * kWriterStreams, WP::BYTES, st>>>(wa);
  LNET_TRY(after_launch("fused_writer_kernel"));
  FusedArgs ra = wa;
  ra.in = w.stream;
  if (reinterpret_cast<uintptr_t>(w.stream) % 16 != 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  LNET_TRY(encode_tile_map(&ra.tmap, w.stream, B, T, D));
  ra.drive = w.rdrive;
  ra.syn = nullptr;
  ra.consts = w.consts + kConsts * M;
  ra.conv_w = p->reader_conv_weight;
  ra.conv_b = p->reader_conv_bias;
  ra.norm = p->reader_norm;
  ra.out = nullptr;
  ra.rowsum = w.rowsum + B * 7 * M;
  ra.rec = w.rrec;
  ra.counter = counters + 1;
  ra.kernel_id = 1;
  LNET_TRY(cuda_check(cudaFuncSetAttribute(fused_reader_kernel<D, M>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           RP::LAUNCH_BYTES),
                      "cudaFuncSetAttribute(fused_reader_kernel)"));
  fused_reader_kernel<D, M><<<(unsigned)std::min<int64_t>(items, 2 * (int64_t)sms),
                              kFusedThreads, RP::LAUNCH_BYTES, st>>>(ra);
  LNET_TRY(after_launch("fused_reader_kernel"));
  fused_finalize_kernel<<<(unsigned)std::min<int64_t>(cdiv(B * 14 * M, 256), 8 * sms), 256, 0,
                          st>>>(w.rowsum, wm, rm, w.feats, B, T, M, w.epoch_word);
  return after_launch("fused_finalize_kernel");
}

inline int fused_forward(const lnet_b200_alphabet_params *p, const lnet_b200_alphabet_request *r,
                         FusedWorkspace &w, float *wm, float *rm, bool prepared, cudaStream_t st) {
  if (p->raw_input_dim == 48 && p->model_dim == 96 && p->modes == 48)
    return fused_forward_shape<48, 96, 48>(p, r, w, wm, rm, prepared, st);
  return fail(LNET_ERR_UNSUPPORTED, "no fused kernel instance for C=%d D=%d M=%d",
              p->raw_input_dim, p->model_dim, p->modes);
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

namespace lnet {
static int g_trace_on = 0;
static unsigned long long *g_trace_dev = nullptr;
int fused_trace_enabled() { return g_trace_on; }
}  // namespace lnet

// Enable (1) / disable (0) per-phase cycle tracing of the fused kernels; enabling clears
// the counters of the current device.
extern "C" int lnet_b200_trace_enable(int on) {
  lnet::g_trace_on = on != 0;
  if (on) {
    void *p = nullptr;
    LNET_TRY(lnet::cuda_check(cudaGetSymbolAddress(&p, lnet::g_fused_trace),
                              "cudaGetSymbolAddress(g_fused_trace)"));
    lnet::g_trace_dev = static_cast<unsigned long long *>(p);
    unsigned long long zero[32] = {};
    return lnet::cuda_check(cudaMemcpyToSymbol(lnet::g_fused_trace, zero, sizeof(zero)),
                            "cudaMemcpyToSymbol(g_fused_trace)");
  }
  return LNET_OK;
}

// Copies the 2 x 16 phase counters (writer, reader) of the current device to `out`
// (synchronises the device).
extern "C" int lnet_b200_trace_read(unsigned long long *out) {
  if (!out) return lnet::fail(LNET_ERR_INVALID_ARGUMENT, "out is NULL");
  return lnet::cuda_check(
      cudaMemcpyFromSymbol(out, lnet::g_fused_trace, 32 * sizeof(unsigned long long)),
      "cudaMemcpyFromSymbol(g_fused_trace)");
}

// Same as lnet_b200_trace_read, ordered on `stream` only (pinned `out`), so it can
// observe the counters of kernels still running on another stream.  Call
// lnet_b200_trace_enable(1) first (it resolves the counters' device address).
extern "C" int lnet_b200_trace_read_async(unsigned long long *out, lnet_stream_t stream) {
  if (!out) return lnet::fail(LNET_ERR_INVALID_ARGUMENT, "out is NULL");
  if (!lnet::g_trace_dev) return lnet::fail(LNET_ERR_INVALID_ARGUMENT, "tracing not enabled");
  cudaStream_t st = (cudaStream_t)stream;
  LNET_TRY(lnet::cuda_check(cudaMemcpyAsync(out, lnet::g_trace_dev, 32 * sizeof(unsigned long long),
                                            cudaMemcpyDeviceToHost, st),
                            "cudaMemcpyAsync(trace)"));
  return lnet::cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
}
