// Shared device helpers, error plumbing and launch accounting for lnet_b200.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "lnet_b200.h"

namespace lnet {

constexpr float kFp32Eps = 1.1920928955078125e-07f;   // torch.finfo(float32).eps
constexpr float kFp32Tiny = 1.1754943508222875e-38f;  // torch.finfo(float32).tiny
constexpr double kDampingMin = 1.0e-3;
constexpr double kDampingMax = 2.0;
constexpr double kPi = 3.14159265358979323846;

// ---------------------------------------------------------------- errors
int fail(int code, const char *fmt, ...);
int cuda_check(cudaError_t err, const char *what);
void reset_launches();
// Marks the start of an entry point's launches on `stream` (for profiling).
void begin_entry(cudaStream_t stream);
void count_launch(int n = 1);
int launch_count();
// Checks the most recent launch on this thread and counts it.
int after_launch(const char *what);
// After a library call (cuBLAS): profiling record only, not counted as a launch
// of this library's kernels.
int after_library(const char *what);

#define LNET_TRY(expr)              \
  do {                              \
    int _st = (expr);               \
    if (_st != LNET_OK) return _st; \
  } while (0)

// ---------------------------------------------------------------- loads
__device__ __forceinline__ float load_f(const float *p, int64_t i) { return p[i]; }
__device__ __forceinline__ float load_f(const __nv_bfloat16 *p, int64_t i) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(p[i]) << 16);  // exact widening
}
__device__ __forceinline__ double load_f(const double *p, int64_t i) { return p[i]; }
__device__ __forceinline__ void store_f(float *p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void store_f(__nv_bfloat16 *p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// SiLU v / (1 + e^-v) of the fp32 general route, with the documented fast
// intrinsics __expf and __fdividef (each within a few ulp over the range that
// matters; relative error of the result ~1e-6, far below the fp32 parity
// bound).  Large negative v: e^-v overflows to inf (or exceeds 2^126) and the
// quotient is -0 / 0, the limit of SiLU.
__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// torch.lerp: a + w (b - a) if |w| < 0.5 else b - (b - a)(1 - w)
__device__ __forceinline__ float lerp_torch(float a, float b, float w) {
  return fabsf(w) < 0.5f ? a + w * (b - a) : b - (b - a) * (1.0f - w);
}

// First index in ts[0..n) with ts[i] >= q (torch.searchsorted(right=False)).
__device__ __forceinline__ int64_t lower_bound_f(const float *ts, int64_t n, float q) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (ts[mid] < q)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Damping / frequency of one mode (src/lnet/pac_tight_frame_models.py:458-459,487-491),
// evaluated in double.
__device__ __forceinline__ void mode_pole(float raw_decay, float raw_frequency, double &damping,
                                          double &frequency) {
  double r = (double)raw_decay;
  damping = kDampingMin + (kDampingMax - kDampingMin) / (1.0 + exp(-r));
  frequency = kPi * tanh((double)raw_frequency);
}

// Zero-order hold a = exp(p dt), gamma = (a - 1)/p, gamma = dt when |p dt| < 1e-6
// (src/lnet/pac_real2d_math.py:20-53), evaluated in double and rounded once.
struct Zoh {
  float a_re, a_im, g_re, g_im;
};
__device__ __forceinline__ Zoh zoh_eval(double damping, double frequency, double step) {
  double scaled = exp(-damping * step);
  double s, c;
  sincos(frequency * step, &s, &c);
  double ar = scaled * c, ai = scaled * s;
  double shr = ar - 1.0, shi = ai;
  double pr = -damping, pi = frequency;
  double den = pr * pr + pi * pi;
  double gr = (shr * pr + shi * pi) / den;
  double gi = (shi * pr - shr * pi) / den;
  if (sqrt((pr * step) * (pr * step) + (pi * step) * (pi * step)) < 1.0e-6) {
    gr = step;
    gi = 0.0;
  }
  return Zoh{(float)ar, (float)ai, (float)gr, (float)gi};
}

// The same zero-order hold in fp32 for per-step evaluation (one (step, mode)
// pair per call, where the double form's exp and sincos dominated the drive
// pass).  a - 1 is formed without cancellation: with x = -damping dt and
// phi = frequency dt, a - 1 = expm1(x) cos(phi) - 2 sin^2(phi / 2)
// + i exp(x) sin(phi), and cos(phi), sin(phi) come from sincos(phi / 2).  Every
// term is then a product of correctly rounded library results, a few fp32 ulp
// from the double evaluation; gamma is one complex division by p.
__device__ __forceinline__ Zoh zoh_eval_f32(float damping, float frequency, float step) {
  const float x = -damping * step, ph = frequency * step;
  const float em1 = expm1f(x), e = expf(x);
  float s2, c2;
  sincosf(0.5f * ph, &s2, &c2);
  const float sn = 2.f * s2 * c2;
  const float cs = fmaf(-2.f * s2, s2, 1.f);
  const float ar = e * cs, ai = e * sn;
  const float shr = fmaf(em1, cs, -2.f * s2 * s2), shi = ai;
  const float pr = -damping, pi = frequency;
  const float den = fmaf(pr, pr, pi * pi);
  float gr = fmaf(shr, pr, shi * pi) / den;
  float gi = fmaf(shi, pr, -shr * pi) / den;
  if (sqrtf(fmaf(x, x, ph * ph)) < 1.0e-6f) {
    gr = step;
    gi = 0.f;
  }
  return Zoh{ar, ai, gr, gi};
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace.
struct Arena {
  char *base;
  size_t size;
  size_t used = 0;
  bool measure_only;
  Arena(void *b, size_t s) : base((char *)b), size(s), measure_only(b == nullptr) {}
  template <typename T>
  T *take(size_t count) {
    size_t off = align_up(used, 256);
    used = off + align_up(count * sizeof(T), 256);
    if (measure_only) return nullptr;
    return (T *)(base + off);
  }
  bool ok() const { return measure_only || used <= size; }
};

}  // namespace lnet
