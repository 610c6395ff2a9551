// tfx_math.h -- the exact-erf GELU arithmetic of the reference, for device
// kernels and (compiled by a host C++ compiler with -ffp-contract=off) for the
// CPU-side exhaustive check against the oracle.
//
// The reference's f32 erf is the MLX Metal erff sequence as written in
// crates/cpu-kernels/src/lib.rs:449-505 (erf_f32 + mlx_expm1f). erf_mlx()
// below evaluates the same IEEE operations in the same order for every input
// that reaches them, so its results are bit-identical to the reference; it
// only leaves out work that is dead for erf's arguments:
//
//   * erf calls expm1 only with r = poly(t), t = |x| > 0.9277344, and there
//     r <= -1.66, so in mlx_expm1f j = rint(r * log2 e) <= -2: the a == 0,
//     j == 0 and j == 1 cases never fire;
//   * for r <= -20 mlx_expm1f returns exactly -1 (its own |a - 1| > 88
//     override included), so clamping r at -20 changes no result and keeps
//     j in [-29, -2], where 0.5 * 2^j (Rust powi) is the normal number with
//     exponent field j + 126 and can be built from the bits of the magic sum.
//
// Both facts are verified over all 2^32 inputs by the CPU test suite, which
// compiles this header with the host compiler and compares with the oracle's
// literal restatement bit for bit.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define TFX_HD __host__ __device__ __forceinline__
#else
#define TFX_HD static inline
#endif

namespace tfx {
namespace math {

TFX_HD float fma_rn(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return fmaf(a, b, c);
#endif
}
TFX_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
TFX_HD float add_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
TFX_HD float sub_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
TFX_HD int32_t f2bits(float v) {
#if defined(__CUDA_ARCH__)
  return __float_as_int(v);
#else
  int32_t i;
  memcpy(&i, &v, 4);
  return i;
#endif
}
TFX_HD float bits2f(int32_t i) {
#if defined(__CUDA_ARCH__)
  return __int_as_float(i);
#else
  float v;
  memcpy(&v, &i, 4);
  return v;
#endif
}

// Coefficients of the reference's erf (crates/cpu-kernels/src/lib.rs:449-471)
// and expm1 (:474-505); see the file comment.
constexpr float kErfBranch = 0.9277344f;
constexpr float kS0 = -5.967617e-4f, kS1 = 4.9911942e-3f, kS2 = -2.6768135e-2f,
                kS3 = 1.1281992e-1f, kS4 = -3.7612534e-1f, kS5 = 1.2837917e-1f;
constexpr float kL0 = -1.7285347e-5f, kL1 = 3.8319713e-4f, kL2 = -3.8839644e-3f,
                kL3 = 2.4254622e-2f, kL4 = -1.0677788e-1f, kL5 = -6.3484669e-1f,
                kL6 = -1.2871751e-1f;
constexpr float kLog2e = 1.442695f, kMagic = 12582912.0f, kLn2Hi = -0.693145752f;
constexpr float kE0 = 1.9735098e-4f, kE1 = 1.3930907e-3f, kE2 = 8.33344e-3f,
                kE3 = 4.1666802e-2f, kE4 = 1.6666672e-1f, kE5 = 4.9999997e-1f;
constexpr float kClamp = -20.0f;
constexpr int32_t kMagicBits = 0x4B400000;  // bit pattern of kMagic
constexpr float kFrac1Sqrt2 = 0.70710678118654752440f;

// mlx_expm1f for the arguments erf gives it (a <= -1.66); bit-identical there.
TFX_HD float expm1_erf_domain(float a) {
  a = fmaxf(a, kClamp);
  const float big = fma_rn(kLog2e, a, kMagic);
  const float j = sub_rn(big, kMagic);
  const float f = fma_rn(j, kLn2Hi, a);
  const float s = mul_rn(f, f);
  float r = fma_rn(kE0, f, kE1);
  r = fma_rn(r, f, kE2);
  r = fma_rn(r, f, kE3);
  r = fma_rn(r, f, kE4);
  r = fma_rn(r, f, kE5);
  const float v = fma_rn(r, s, f);
  const float t = bits2f((f2bits(big) - kMagicBits + 126) << 23);  // 0.5 * 2^j
  const float y = sub_rn(t, 0.5f);
  const float x = sub_rn(sub_rn(t, y), 0.5f);
  r = add_rn(fma_rn(v, t, x), y);
  return add_rn(r, r);
}

// erf_f32 of crates/cpu-kernels/src/lib.rs:449-471, branch-free.
TFX_HD float erf_mlx(float a) {
  const float t = fabsf(a);
  const float s = mul_rn(a, a);
  float q = fma_rn(kS0, s, kS1);
  q = fma_rn(q, s, kS2);
  q = fma_rn(q, s, kS3);
  q = fma_rn(q, s, kS4);
  q = fma_rn(q, s, kS5);
  const float small = fma_rn(q, a, a);
  float r = fma_rn(kL0, t, kL1);
  const float u = fma_rn(kL2, t, kL3);
  r = fma_rn(r, s, u);
  r = fma_rn(r, t, kL4);
  r = fma_rn(r, t, kL5);
  r = fma_rn(r, t, kL6);
  r = fma_rn(r, t, -t);
  const float large = copysignf(-expm1_erf_domain(r), a);
  return t > kErfBranch ? large : small;
}

// gelu_erf_f32 of crates/cpu-kernels/src/lib.rs:509-511: (0.5 x)(1 + erf(x/sqrt2)).
TFX_HD float gelu_mlx(float x) {
  return mul_rn(mul_rn(0.5f, x), add_rn(1.0f, erf_mlx(mul_rn(x, kFrac1Sqrt2))));
}

#if defined(__CUDACC__)
// The same two functions on a pair of values, using sm_100's paired f32
// FMA/MUL/ADD (per component identical to __fmaf_rn / __fmul_rn / __fadd_rn).
// Device-only; declared in nvcc's host pass too so device lambdas parse.
__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }

__device__ __forceinline__ float2 expm1_erf_domain2(float2 a) {
  a = make_float2(fmaxf(a.x, kClamp), fmaxf(a.y, kClamp));
  const float2 big = __ffma2_rn(splat(kLog2e), a, splat(kMagic));
  const float2 j = __fadd2_rn(big, splat(-kMagic));
  const float2 f = __ffma2_rn(j, splat(kLn2Hi), a);
  const float2 s = __fmul2_rn(f, f);
  float2 r = __ffma2_rn(splat(kE0), f, splat(kE1));
  r = __ffma2_rn(r, f, splat(kE2));
  r = __ffma2_rn(r, f, splat(kE3));
  r = __ffma2_rn(r, f, splat(kE4));
  r = __ffma2_rn(r, f, splat(kE5));
  const float2 v = __ffma2_rn(r, s, f);
  const float2 t = make_float2(__int_as_float((__float_as_int(big.x) - kMagicBits + 126) << 23),
                               __int_as_float((__float_as_int(big.y) - kMagicBits + 126) << 23));
  const float2 y = __fadd2_rn(t, splat(-0.5f));
  const float2 x = __fadd2_rn(__fadd2_rn(t, make_float2(-y.x, -y.y)), splat(-0.5f));
  r = __fadd2_rn(__ffma2_rn(v, t, x), y);
  return __fadd2_rn(r, r);
}

__device__ __forceinline__ float2 erf_mlx2(float2 a) {
  const float2 t = make_float2(fabsf(a.x), fabsf(a.y));
  const float2 s = __fmul2_rn(a, a);
  float2 q = __ffma2_rn(splat(kS0), s, splat(kS1));
  q = __ffma2_rn(q, s, splat(kS2));
  q = __ffma2_rn(q, s, splat(kS3));
  q = __ffma2_rn(q, s, splat(kS4));
  q = __ffma2_rn(q, s, splat(kS5));
  const float2 small = __ffma2_rn(q, a, a);
  float2 r = __ffma2_rn(splat(kL0), t, splat(kL1));
  const float2 u = __ffma2_rn(splat(kL2), t, splat(kL3));
  r = __ffma2_rn(r, s, u);
  r = __ffma2_rn(r, t, splat(kL4));
  r = __ffma2_rn(r, t, splat(kL5));
  r = __ffma2_rn(r, t, splat(kL6));
  r = __ffma2_rn(r, t, make_float2(-t.x, -t.y));
  const float2 e = expm1_erf_domain2(r);
  const float2 large = make_float2(copysignf(-e.x, a.x), copysignf(-e.y, a.y));
  return make_float2(t.x > kErfBranch ? large.x : small.x, t.y > kErfBranch ? large.y : small.y);
}

__device__ __forceinline__ float2 gelu_mlx2(float2 x) {
  const float2 e = erf_mlx2(__fmul2_rn(x, splat(kFrac1Sqrt2)));
  return __fmul2_rn(__fmul2_rn(splat(0.5f), x), __fadd2_rn(splat(1.0f), e));
}
#endif

}  // namespace math
}  // namespace tfx
