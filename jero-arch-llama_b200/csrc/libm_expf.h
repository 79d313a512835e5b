// expf with the reference's rounding, for host and device.
//
// The reference's f32::exp calls the platform libm's expf (glibc on Linux),
// and so does the oracle.  glibc computes expf (since 2.27; the method of
// Arm's optimized-routines) as
//   z = x * (N / ln 2) in double, N = 32; k = nearest integer to z (the
//   1.5 * 2^52 shift); r = z - k (both from the unrounded product, i.e.
//   fused multiply-adds);
//   s = 2^(k / N) = 2^(k div N) * 2^((k mod N) / N), read from a table of
//   2^(i / 32) whose exponent field is offset by i << 47 so that adding
//   k << 47 to the bits scales by 2^(k div N);
//   y = (C0 r + C1) r^2 + (C2 r + 1), a degree-3 polynomial for
//   2^(r / N) in which the fused multiply-adds of FMA-capable x86-64 hosts
//   (the library's FMA variant) are used;
//   expf(x) = (float)(y * s).
// Its result is not always the correctly rounded exp (it differs on about
// 6e-4 of arguments), so parity with the reference needs this very
// evaluation.  The table holds the correctly rounded doubles of 2^(i/32)
// (minus i << 47), computed from the definition; the polynomial
// coefficients are those of the published method.  It equals the host's
// glibc expf on every float with |x| <= 110 (2,243,428,356 arguments, checked
// exhaustively; a CPU test repeats the check on a sample).
#pragma once

#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define JAL_HD __host__ __device__ __forceinline__
#else
#define JAL_HD inline
#endif

namespace jal {
namespace libm {

// bits(2^(i/32)) - (i << 47), i < 32: the correctly rounded doubles of
// 2^(i/32) (computed from the definition in 60-digit decimal arithmetic).
#define JAL_EXP2_32_TABLE \
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull, \
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, \
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull, \
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull, \
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull, \
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull, \
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull, \
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull, \

#ifdef __CUDACC__
// One copy per translation unit in global memory: lanes of a warp index it
// with different i, which L1-cached loads serve in one or two transactions.
static __device__ const uint64_t kExp2Tab32Dev[32] = {JAL_EXP2_32_TABLE};
#endif
static const uint64_t kExp2Tab32Host[32] = {JAL_EXP2_32_TABLE};

JAL_HD uint64_t exp2_32_table(int i) {
#ifdef __CUDA_ARCH__
  return __ldg(&kExp2Tab32Dev[i]);
#else
  return kExp2Tab32Host[i];
#endif
}

JAL_HD double bits_to_d(uint64_t u) {
  double d;
  memcpy(&d, &u, 8);
  return d;
}
JAL_HD uint64_t d_to_bits(double d) {
  uint64_t u;
  memcpy(&u, &d, 8);
  return u;
}

// Multiply-add with one rounding, and the unfused forms, for host and device.
JAL_HD double fma_d(double a, double b, double c) {
#ifdef __CUDA_ARCH__
  return __fma_rn(a, b, c);
#else
  return __builtin_fma(a, b, c);
#endif
}
JAL_HD double mul_d(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dmul_rn(a, b);
#else
  volatile double p = a * b;  // no contraction into a neighbouring add
  return p;
#endif
}
JAL_HD double add_d(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dadd_rn(a, b);
#else
  return a + b;
#endif
}

JAL_HD float expf_ref(float x) {
  uint32_t ux;
  memcpy(&ux, &x, 4);
  const uint32_t abstop = (ux >> 20) & 0x7ffu;
  if (abstop >= 0x42bu) {                   // |x| >= 88 or not finite
    if (ux == 0xff800000u) return 0.0f;     // -inf
    if (abstop >= 0x7f8u) return x + x;     // +inf, NaN
    if (x > 88.72283172607421875f) return __builtin_inff();  // overflow
    if (x < -103.972076416015625f) return 0.0f;               // underflow
  }
  const double InvLn2N = bits_to_d(0x3ff71547652b82feull) * 32.0;
  const double Shift = 6755399441055744.0;  // 1.5 * 2^52
  const double C0 = bits_to_d(0x3fac6af84b912394ull) / 32768.0;  // (~ln2^3 / 6) / N^3
  const double C1 = bits_to_d(0x3fcebfce50fac4f3ull) / 1024.0;   // (~ln2^2 / 2) / N^2
  const double C2 = bits_to_d(0x3fe62e42ff0c52d6ull) / 32.0;     // (~ln2) / N
  const double xd = (double)x;
  double kd = fma_d(InvLn2N, xd, Shift);  // z + Shift with z = x * N / ln 2 unrounded
  const uint64_t ki = d_to_bits(kd);
  kd = add_d(kd, -Shift);
  const double r = fma_d(InvLn2N, xd, -kd);  // z - k
  const uint64_t t = exp2_32_table((int)(ki % 32)) + (ki << 47);
  const double s = bits_to_d(t);
  const double zz = fma_d(C0, r, C1);
  const double r2 = mul_d(r, r);
  double y = fma_d(C2, r, 1.0);
  y = fma_d(zz, r2, y);
  y = mul_d(y, s);
  return (float)y;
}

}  // namespace libm
}  // namespace jal
