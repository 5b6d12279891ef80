// Pole-residue Laplace layer (PoleResidueTemporalMixing, src/lnet/laplace.py:55-159) in float64.
//
// Work split: the (mode, channel) state vector of one row is cut into
// slices of kSlice entries; one CTA owns one (slice, row), runs its states
// sequentially over T and contracts them with the matching residue slice
// into a per-slice partial output [T, D].  A second kernel sums the slices in
// a fixed order and adds the direct term and the bias, so the result is
// deterministic.  No state ever reaches HBM.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace lnet {

constexpr int kSlice = 256;  // state entries per CTA (= threads)
constexpr int kStepTile = 32;
constexpr int kOutTile = 16;
static_assert(kSlice == 256 && kStepTile == 32 && kOutTile == 16,
              "the contraction maps 8 warps x 4 steps and 4 output quads x 8 K parts");
// Row pitch of the state and residue tiles in shared memory: an odd number of
// doubles, so the 16 residue rows (and 2 state rows) one warp reads for one
// entry e fall in distinct banks (a pitch of kSlice put them all in one).
constexpr int kPitch = kSlice + 1;

__device__ __forceinline__ double softplus_d(double x) {
  return x > 20.0 ? x : log1p(exp(x));
}

// dt * phi1(p dt) with the series branch of _phi1 (src/lnet/laplace.py:37-42)
__device__ __forceinline__ void laplace_zoh(double raw_decay, double dt, double min_decay,
                                            double &a, double &b) {
  double pole = -(softplus_d(raw_decay) + min_decay);
  double z = pole * dt;
  double phi = fabs(z) < 1.0e-4 ? 1.0 + z / 2.0 + z * z / 6.0 : expm1(z) / z;
  a = exp(z);
  b = dt * phi;
}

template <typename TX>
__global__ void __launch_bounds__(kSlice) laplace_slice_kernel(
    const TX *__restrict__ x, const double *__restrict__ raw_decay,
    const double *__restrict__ residues, int dim, int modes, double dt, double min_decay,
    int64_t steps, double *__restrict__ partial) {
  extern __shared__ double smem[];
  double *s_state = smem;                        // [kStepTile][kPitch]
  double *s_res = smem + kStepTile * kPitch;     // [kOutTile][kPitch]
  double *s_x = s_res + kOutTile * kPitch;       // [kStepTile][dim] input tile
  const int slice = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int64_t md = (int64_t)modes * dim;
  const int j = threadIdx.x;
  const int64_t k = (int64_t)slice * kSlice + j;
  const bool live = k < md;
  const int m = live ? (int)(k / dim) : 0;
  const int i = live ? (int)(k - (int64_t)m * dim) : 0;
  double a = 0.0, bcoef = 0.0;
  if (live) laplace_zoh(raw_decay[m], dt, min_decay, a, bcoef);
  double state = 0.0;
  double *out_row = partial + ((int64_t)slice * gridDim.y + b) * steps * dim;
  for (int64_t t0 = 0; t0 < steps; t0 += kStepTile) {
    const int nt = (int)min((int64_t)kStepTile, steps - t0);
    // the input tile, loaded by all threads at once (no load on the recurrence chain)
    for (int e = j; e < nt * dim; e += kSlice)
      s_x[e] = (double)load_f(x, (b * steps + t0) * dim + e);
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
      const double xv = live ? s_x[tt * dim + i] : 0.0;
      state = a * state + bcoef * xv;
      s_state[tt * kPitch + j] = live ? state : 0.0;
    }
    for (int o0 = 0; o0 < dim; o0 += kOutTile) {
      const int no = min(kOutTile, dim - o0);
      __syncthreads();
      for (int r = 0; r < no; ++r)
        s_res[r * kPitch + j] = live ? residues[(int64_t)(o0 + r) * md + k] : 0.0;
      __syncthreads();
      // Register-blocked contraction: warp w owns steps 4w..4w+3; lane = (output
      // quad os, K part kp); each thread accumulates a 4 x 4 block over the
      // entries e = kp mod 8 (consecutive kp read consecutive doubles), then
      // the 8 K parts are summed by a shuffle tree.  Four FMAs per two shared
      // loads instead of one per two.
      {
        const int warp = j >> 5, lane = j & 31;
        const int os = lane & 3, kp = lane >> 2;
        const int tb = warp * 4;
        double acc[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) acc[u][v] = 0.0;
#pragma unroll 4
        for (int e = kp; e < kSlice; e += 8) {
          double sv[4], rv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) sv[u] = s_state[(tb + u) * kPitch + e];
#pragma unroll
          for (int v = 0; v < 4; ++v) rv[v] = s_res[(os * 4 + v) * kPitch + e];
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[u][v] = fma(rv[v], sv[u], acc[u][v]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v)
#pragma unroll
            for (int o = 4; o < 32; o <<= 1)
              acc[u][v] += __shfl_xor_sync(0xffffffffu, acc[u][v], o);
        if (kp == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int tt = tb + u, r = os * 4 + v;
              if (tt < nt && r < no) out_row[(t0 + tt) * dim + o0 + r] = acc[u][v];
            }
        }
      }
    }
    __syncthreads();
  }
}

template <typename TX>
__global__ void laplace_reduce_kernel(const TX *__restrict__ x, const double *__restrict__ partial,
                                      const double *__restrict__ direct,
                                      const double *__restrict__ bias, int dim, int n_slices,
                                      int64_t tokens, TX *__restrict__ y) {
  int64_t n = tokens * dim;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t tok = idx / dim;
    int o = (int)(idx - tok * dim);
    double acc = 0.0;
    for (int s = 0; s < n_slices; ++s) acc += partial[(int64_t)s * n + idx];
    double dsum = 0.0;
    for (int i = 0; i < dim; ++i) dsum = fma((double)load_f(x, tok * dim + i), direct[o * dim + i], dsum);
    double v = acc + dsum + bias[o];
    if constexpr (sizeof(TX) == 8)
      y[idx] = v;
    else
      y[idx] = (TX)(float)v;
  }
}

// Scratch bytes of one call (per-slice partial outputs), or false when the
// product does not fit in 64 bits (the shape is refused before any launch).
static bool laplace_partial_bytes(int64_t batch, int64_t steps, int dim, int modes,
                                  size_t *bytes) {
  const uint64_t n_slices = (uint64_t)cdiv((int64_t)modes * dim, kSlice);
  uint64_t v = n_slices;
  if (__builtin_mul_overflow(v, (uint64_t)batch, &v) ||
      __builtin_mul_overflow(v, (uint64_t)steps, &v) ||
      __builtin_mul_overflow(v, (uint64_t)dim, &v) ||
      __builtin_mul_overflow(v, (uint64_t)sizeof(double), &v))
    return false;
  *bytes = (size_t)v;
  return true;
}

template <typename TX>
static int laplace_run(const double *raw_decay, const double *residues, const double *direct,
                       const double *bias, int dim, int modes, double dt, double min_decay,
                       const TX *x, int64_t batch, int64_t steps, TX *y, double *partial,
                       cudaStream_t stream) {
  int n_slices = (int)cdiv((int64_t)modes * dim, kSlice);
  const size_t smem =
      ((size_t)(kStepTile + kOutTile) * kPitch + (size_t)kStepTile * dim) * sizeof(double);
  if (smem > 232448)
    return fail(LNET_ERR_UNSUPPORTED, "laplace: model_dim %d too large for the input tile", dim);
  LNET_TRY(cuda_check(cudaFuncSetAttribute(laplace_slice_kernel<TX>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem),
                      "cudaFuncSetAttribute(laplace_slice_kernel)"));
  dim3 grid(n_slices, (unsigned)batch);
  laplace_slice_kernel<TX><<<grid, kSlice, smem, stream>>>(x, raw_decay, residues, dim, modes,
                                                           dt, min_decay, steps, partial);
  LNET_TRY(after_launch("laplace_slice_kernel"));
  int64_t n = batch * steps * dim;
  int blocks = (int)std::min<int64_t>(cdiv(n, 256), 148 * 16);
  laplace_reduce_kernel<TX><<<blocks, 256, 0, stream>>>(x, partial, direct, bias, dim, n_slices,
                                                        batch * steps, y);
  return after_launch("laplace_reduce_kernel");
}

}  // namespace lnet

using namespace lnet;

extern "C" int lnet_b200_laplace_workspace_size(int64_t batch, int64_t steps, int32_t model_dim,
                                                int32_t modes, size_t *bytes) {
  reset_launches();
  if (!bytes) return fail(LNET_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  if (batch < 0 || steps < 0 || model_dim < 1 || modes < 1)
    return fail(LNET_ERR_INVALID_ARGUMENT, "invalid laplace shape");
  if (!laplace_partial_bytes(batch, steps, model_dim, modes, bytes))
    return fail(LNET_ERR_INVALID_ARGUMENT, "laplace: workspace size overflows (B=%lld, T=%lld)",
                (long long)batch, (long long)steps);
  return LNET_OK;
}

extern "C" int lnet_b200_laplace_forward(const double *raw_decay, const double *residues,
                                         const double *direct, const double *bias,
                                         int32_t model_dim, int32_t modes, double dt,
                                         double min_decay, int32_t x_dtype, const void *x,
                                         int64_t batch, int64_t steps, void *y, void *workspace,
                                         size_t workspace_bytes, lnet_stream_t stream) {
  reset_launches();
  if (model_dim < 1 || modes < 1 || batch < 0 || steps < 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "invalid laplace shape (D=%d, M=%d, B=%lld, T=%lld)",
                model_dim, modes, (long long)batch, (long long)steps);
  if (batch == 0 || steps == 0) return LNET_OK;
  if (!raw_decay || !residues || !direct || !bias || !x || !y)
    return fail(LNET_ERR_INVALID_ARGUMENT, "laplace: NULL tensor pointer");
  if (batch > 65535) return fail(LNET_ERR_UNSUPPORTED, "laplace: batch > 65535");
  size_t need = 0;
  if (!laplace_partial_bytes(batch, steps, model_dim, modes, &need))
    return fail(LNET_ERR_INVALID_ARGUMENT, "laplace: workspace size overflows (B=%lld, T=%lld)",
                (long long)batch, (long long)steps);
  if (!workspace || workspace_bytes < need)
    return fail(LNET_ERR_WORKSPACE, "laplace: workspace of %zu bytes < required %zu",
                workspace_bytes, need);
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  if (x_dtype == LNET_F64)
    return laplace_run<double>(raw_decay, residues, direct, bias, model_dim, modes, dt, min_decay,
                               (const double *)x, batch, steps, (double *)y, (double *)workspace,
                               st);
  if (x_dtype == LNET_F32)
    return laplace_run<float>(raw_decay, residues, direct, bias, model_dim, modes, dt, min_decay,
                              (const float *)x, batch, steps, (float *)y, (double *)workspace, st);
  return fail(LNET_ERR_UNSUPPORTED, "laplace: x dtype must be float32 or float64");
}

namespace lnet {

// ---------------------------------------------------------------- channel-diagonal residues
// When R[o, m, i] = 0 for every i != o (each output reads only the states of its
// own input channel -- the per-channel pole layout), the readout collapses to
//   y_t[o] = sum_j r[o, j] s_t[m_j, o] + (D x_t)[o] + bias[o],
// with only the K modes m_j = mode_index[o, j] whose residue is nonzero.  One
// thread owns (row, channel, time chunk) with its K states in registers: a
// local scan of its chunk from zero, the chunk carries combined in shared
// memory (each chunk's true initial state = sum over earlier chunks of
// a^(steps between) * their local end states), then a second scan from the true
// carry that writes y.  The CTA first stages its row's input [T, D] in shared
// memory (as double) when it fits, so the scans read no global memory.  No
// scratch in global memory.
constexpr int kDiagChunks = 32;   // time chunks per (row, channel)
constexpr int kDiagChans = 8;     // channels per CTA
// the row's input [T, D] as double in shared memory when it fits (else read from global)
constexpr size_t kDiagStageBytes = 160 * 1024;
constexpr int kDiagMaxModes = 16; // K bound (registers per thread)

// DIMC: the model width when it is a compile-time 16 (the direct-term row of D
// then lives in registers), else 0 (read per step).  Staged rows are stored
// per chunk with one double of padding between chunks, so the four chunks a
// warp spans read different shared-memory banks.
template <typename TX, int K, bool STAGED, int DIMC>
__global__ void __launch_bounds__(kDiagChunks * kDiagChans) laplace_diag_kernel(
    const TX *__restrict__ x, const double *__restrict__ raw_decay,
    const int32_t *__restrict__ mode_index, const double *__restrict__ residue,
    const double *__restrict__ direct, const double *__restrict__ bias, int dim, int kmodes,
    double dt, double min_decay, int64_t steps, TX *__restrict__ y) {
  __shared__ double s_end[kDiagChunks][kDiagChans][K];
  const int o_loc = threadIdx.x % kDiagChans, c = threadIdx.x / kDiagChans;
  const int o = blockIdx.x * kDiagChans + o_loc;
  const int64_t b = blockIdx.y;
  const bool live = o < dim;
  const int64_t L = (steps + kDiagChunks - 1) / kDiagChunks;
  const int64_t t_begin = c * L, t_end = min(steps, t_begin + L);
  // the pole coefficients of the CTA's (channel, mode) pairs, evaluated once per
  // CTA (not once per chunk thread): a, the input gain g and a^L (L = chunk length)
  __shared__ double s_coef[3][kDiagChans][K];
  for (int p = threadIdx.x; p < kDiagChans * K; p += blockDim.x) {
    const int ol = p / K, j = p - ol * K, oo = blockIdx.x * kDiagChans + ol;
    double ca = 0.0, cg = 0.0, caL = 1.0;
    if (oo < dim && j < kmodes) {
      laplace_zoh(raw_decay[mode_index[oo * kmodes + j]], dt, min_decay, ca, cg);
      for (int64_t k = 0; k < L; ++k) caL *= ca;
    }
    s_coef[0][ol][j] = ca;
    s_coef[1][ol][j] = cg;
    s_coef[2][ol][j] = caL;
  }
  __syncthreads();
  double a[K], g[K], r[K], s[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    a[j] = s_coef[0][o_loc][j];
    g[j] = s_coef[1][o_loc][j];
    r[j] = live && j < kmodes ? residue[o * kmodes + j] : 0.0;
    s[j] = 0.0;
  }
  const TX *xr = x + b * steps * dim;
  extern __shared__ double s_x[];  // [T][D] when STAGED
  if constexpr (STAGED) {
    // eight independent loads in flight per thread per round
    const int64_t n = steps * dim;
    for (int64_t e0 = threadIdx.x; e0 < n; e0 += 8 * (int64_t)blockDim.x) {
      double v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t e = e0 + u * (int64_t)blockDim.x;
        v[u] = e < n ? (double)load_f(xr, e) : 0.0;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t e = e0 + u * (int64_t)blockDim.x;
        if (e < n) s_x[e + (e / dim) / L] = v[u];  // + one double per earlier chunk
      }
    }
    __syncthreads();
  }
  const double *s_xc = s_x + c;  // this chunk's padded rows (STAGED)
  auto xin = [&](int64_t e) -> double {
    if constexpr (STAGED)
      return s_xc[e];
    else
      return (double)load_f(xr, e);
  };
  double drow[DIMC > 0 ? DIMC : 1];
  if constexpr (DIMC > 0) {
#pragma unroll
    for (int i = 0; i < DIMC; ++i) drow[i] = live ? direct[o * DIMC + i] : 0.0;
  }
  // ---- pass 1: local scan from zero
  for (int64_t t = t_begin; t < t_end; ++t) {
    const double xv = live ? xin(t * dim + o) : 0.0;
#pragma unroll
    for (int j = 0; j < K; ++j) s[j] = fma(a[j], s[j], g[j] * xv);
  }
#pragma unroll
  for (int j = 0; j < K; ++j) s_end[c][o_loc][j] = s[j];
  __syncthreads();
  // ---- carry: the state before this chunk, from the earlier chunks' local ends
  // (every earlier chunk is full, L steps)
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const double aL = s_coef[2][o_loc][j];
    double carry = 0.0;
    for (int cc = 0; cc < c; ++cc) carry = fma(aL, carry, s_end[cc][o_loc][j]);
    s[j] = carry;
  }
  // ---- pass 2: from the true carry, the readout
  const double bo = live ? bias[o] : 0.0;
  for (int64_t t = t_begin; t < t_end; ++t) {
    const double xv = live ? xin(t * dim + o) : 0.0;
    double acc = 0.0;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      s[j] = fma(a[j], s[j], g[j] * xv);
      acc = fma(r[j], s[j], acc);
    }
    if (live) {
      double dsum = 0.0;
      if constexpr (DIMC > 0) {
#pragma unroll
        for (int i = 0; i < DIMC; ++i) dsum = fma(xin(t * DIMC + i), drow[i], dsum);
      } else {
        for (int i = 0; i < dim; ++i) dsum = fma(xin(t * dim + i), direct[o * dim + i], dsum);
      }
      const double v = acc + dsum + bo;
      if constexpr (sizeof(TX) == 8)
        y[(b * steps + t) * dim + o] = v;
      else
        y[(b * steps + t) * dim + o] = (TX)(float)v;
    }
  }
}

template <typename TX>
static int laplace_diag_run(const double *raw_decay, const int32_t *mode_index,
                            const double *residue, const double *direct, const double *bias,
                            int dim, int kmodes, double dt, double min_decay, const TX *x,
                            int64_t batch, int64_t steps, TX *y, cudaStream_t st) {
  const dim3 grid((unsigned)cdiv(dim, kDiagChans), (unsigned)batch);
  const int threads = kDiagChunks * kDiagChans;
  const size_t stage = ((size_t)steps * dim + kDiagChunks) * sizeof(double);  // + chunk pads
  const bool staged = stage <= kDiagStageBytes;
#define LNET_DIAG_LAUNCH(KK, DC)                                                              \
  if (staged) {                                                                               \
    auto kern = laplace_diag_kernel<TX, KK, true, DC>;                                        \
    LNET_TRY(cuda_check(cudaFuncSetAttribute(kern,                                            \
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                                             (int)kDiagStageBytes),                           \
                        "cudaFuncSetAttribute(laplace_diag_kernel)"));                        \
    kern<<<grid, threads, stage, st>>>(x, raw_decay, mode_index, residue, direct, bias, dim,   \
                                       kmodes, dt, min_decay, steps, y);                      \
  } else {                                                                                    \
    laplace_diag_kernel<TX, KK, false, DC><<<grid, threads, 0, st>>>(                         \
        x, raw_decay, mode_index, residue, direct, bias, dim, kmodes, dt, min_decay, steps,   \
        y);                                                                                   \
  }
#define LNET_DIAG_CASE(KK)                                                                    \
  if (kmodes <= KK) {                                                                         \
    if (dim == 16) {                                                                          \
      LNET_DIAG_LAUNCH(KK, 16)                                                                \
    } else {                                                                                  \
      LNET_DIAG_LAUNCH(KK, 0)                                                                 \
    }                                                                                         \
    return after_launch("laplace_diag_kernel");                                               \
  }
  LNET_DIAG_CASE(4)
  LNET_DIAG_CASE(8)
  LNET_DIAG_CASE(16)
#undef LNET_DIAG_CASE
#undef LNET_DIAG_LAUNCH
  return fail(LNET_ERR_UNSUPPORTED, "laplace (channel-diagonal): %d modes per channel > %d",
              kmodes, kDiagMaxModes);
}

}  // namespace lnet

extern "C" int lnet_b200_laplace_forward_channelwise(
    const double *raw_decay, const int32_t *mode_index, const double *residue,
    const double *direct, const double *bias, int32_t model_dim, int32_t modes,
    int32_t modes_per_channel, double dt, double min_decay, int32_t x_dtype, const void *x,
    int64_t batch, int64_t steps, void *y, lnet_stream_t stream) {
  reset_launches();
  if (model_dim < 1 || modes < 1 || batch < 0 || steps < 0 || modes_per_channel < 1)
    return fail(LNET_ERR_INVALID_ARGUMENT,
                "invalid laplace shape (D=%d, M=%d, K=%d, B=%lld, T=%lld)", model_dim, modes,
                modes_per_channel, (long long)batch, (long long)steps);
  if (modes_per_channel > kDiagMaxModes)
    return fail(LNET_ERR_UNSUPPORTED, "laplace (channel-diagonal): %d modes per channel > %d",
                modes_per_channel, kDiagMaxModes);
  if (batch == 0 || steps == 0) return LNET_OK;
  if (!raw_decay || !mode_index || !residue || !direct || !bias || !x || !y)
    return fail(LNET_ERR_INVALID_ARGUMENT, "laplace: NULL tensor pointer");
  if (batch > 65535) return fail(LNET_ERR_UNSUPPORTED, "laplace: batch > 65535");
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  if (x_dtype == LNET_F64)
    return laplace_diag_run<double>(raw_decay, mode_index, residue, direct, bias, model_dim,
                                    modes_per_channel, dt, min_decay, (const double *)x, batch,
                                    steps, (double *)y, st);
  if (x_dtype == LNET_F32)
    return laplace_diag_run<float>(raw_decay, mode_index, residue, direct, bias, model_dim,
                                   modes_per_channel, dt, min_decay, (const float *)x, batch,
                                   steps, (float *)y, st);
  return fail(LNET_ERR_UNSUPPORTED, "laplace: x dtype must be float32 or float64");
}

// ---------------------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory at all: code running inside a
// memory pool it does not own, plugins whose host framework forbids
// cudaMalloc on the calling thread, or tight real-time loops where an
// allocation (and its implicit synchronisation) is not allowed.  For them,
// lnet_b200_laplace_forward_noalloc keeps the per-slice partial outputs in
// the fixed array below instead of a caller workspace.
//
// The array lives in the library image: every GPU that loads the library
// holds kNoAllocScratchBytes of it until the process exits.  Every call on a
// device shares it; calls whose kernels overlap on the GPU (different
// streams, or different host threads without ordering) race on it.  The
// slice kernel writes every partial it later reads, so nothing has to be
// cleared between calls; the array keeps the last call's contents.
namespace lnet {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) double g_noalloc_scratch[kNoAllocScratchBytes / sizeof(double)];

// Device address of g_noalloc_scratch per device.  In host code the symbol
// name is only a host-side stand-in, so the address is looked up once per
// device (with that device current, by the first call on that device) and
// reused for the life of the process.  cudaDeviceReset ends the context that
// address belongs to: do not call this entry point on a device after a
// cudaDeviceReset of it.
constexpr int kMaxDevices = 64;
static double *g_noalloc_ptr[kMaxDevices] = {};
static std::mutex g_noalloc_mutex;

static int noalloc_scratch(double **out) {
  int dev = 0;
  LNET_TRY(cuda_check(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev < 0 || dev >= kMaxDevices) return fail(LNET_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    LNET_TRY(cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                        "cudaGetSymbolAddress(g_noalloc_scratch)"));
    g_noalloc_ptr[dev] = static_cast<double *>(p);
  }
  *out = g_noalloc_ptr[dev];
  return LNET_OK;
}

}  // namespace lnet

extern "C" size_t lnet_b200_laplace_noalloc_max_scratch_bytes(void) {
  return lnet::kNoAllocScratchBytes;
}

extern "C" int lnet_b200_laplace_forward_noalloc(const double *raw_decay, const double *residues,
                                                 const double *direct, const double *bias,
                                                 int32_t model_dim, int32_t modes, double dt,
                                                 double min_decay, int32_t x_dtype,
                                                 const void *x, int64_t batch, int64_t steps,
                                                 void *y, lnet_stream_t stream) {
  reset_launches();
  if (model_dim < 1 || modes < 1 || batch < 0 || steps < 0)
    return fail(LNET_ERR_INVALID_ARGUMENT, "invalid laplace shape (D=%d, M=%d, B=%lld, T=%lld)",
                model_dim, modes, (long long)batch, (long long)steps);
  if (batch == 0 || steps == 0) return LNET_OK;
  if (!raw_decay || !residues || !direct || !bias || !x || !y)
    return fail(LNET_ERR_INVALID_ARGUMENT, "laplace: NULL tensor pointer");
  if (batch > 65535) return fail(LNET_ERR_UNSUPPORTED, "laplace: batch > 65535");
  if (x_dtype != LNET_F64 && x_dtype != LNET_F32)
    return fail(LNET_ERR_UNSUPPORTED, "laplace: x dtype must be float32 or float64");
  size_t need = 0;
  if (!laplace_partial_bytes(batch, steps, model_dim, modes, &need))
    return fail(LNET_ERR_INVALID_ARGUMENT, "laplace: scratch size overflows (B=%lld, T=%lld)",
                (long long)batch, (long long)steps);
  if (need > kNoAllocScratchBytes)
    return fail(LNET_ERR_WORKSPACE,
                "laplace (no-alloc): this shape needs %zu bytes of scratch but the built-in "
                "array holds %zu; use lnet_b200_laplace_forward with a caller workspace",
                need, kNoAllocScratchBytes);
  double *scratch = nullptr;
  LNET_TRY(noalloc_scratch(&scratch));
  auto st = (cudaStream_t)stream;
  begin_entry(st);
  if (x_dtype == LNET_F64)
    return laplace_run<double>(raw_decay, residues, direct, bias, model_dim, modes, dt, min_decay,
                               (const double *)x, batch, steps, (double *)y, scratch, st);
  return laplace_run<float>(raw_decay, residues, direct, bias, model_dim, modes, dt, min_decay,
                            (const float *)x, batch, steps, (float *)y, scratch, st);
}
