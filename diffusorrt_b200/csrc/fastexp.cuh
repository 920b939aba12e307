// exp(x) for x <= 0 in double precision, table-driven (P. T. P. Tang, "Table-driven implementation
// of the exponential function in IEEE floating-point arithmetic", ACM TOMS 15(2), 1989):
//   x = (32 k + j) ln2 / 32 + r,  |r| <= ln2 / 64,  j in [0, 32)
//   exp(x) = 2^k * 2^(j/32) * exp(r),  exp(r) - 1 = r q(r) with q the degree-5 Taylor polynomial of
//   (exp(r) - 1) / r (truncation below 2^-59 relative on |r| <= ln2 / 64).
// The reduction uses ln2 / 32 split into a 21-bit head (n * head exact for |n| < 2^32) and a tail.
// The 32 table entries 2^(j/32) and the constants were rounded to double from 60-digit decimal
// values. The selector's softmax terms all have x <= 0; below -708 (subnormal results) the CUDA
// exp() takes over. Accuracy is checked against CUDA's exp() by the GPU tests (|error| <= 2 ulp).
#pragma once
#include <cuda_runtime.h>

namespace drt {

// In global memory, read through L1 (lanes index it divergently; the constant cache would
// serialise those reads).
__device__ const double kExp2Table32[32] = {
    0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,
    0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,
    0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,
    0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,
    0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,
    0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,
    0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,
    0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0};

__device__ __forceinline__ double exp_nonpos(double x) {
  if (!(x >= -708.0)) return exp(x);  // subnormal or zero results, -inf, NaN
  constexpr double kInvL = 0x1.71547652b82fep+5;   // 32 / ln2
  constexpr double kL1 = 0x1.62e4200000000p-6;     // ln2 / 32, head
  constexpr double kL2 = 0x1.fdf473de6af28p-27;    // ln2 / 32 - head
  const double n = rint(x * kInvL);
  const double r = fma(-n, kL2, fma(-n, kL1, x));
  const int ni = static_cast<int>(n);
  const int j = ni & 31;
  const int k = ni >> 5;  // floor(ni / 32)
  double q = 1.0 / 720.0;
  q = fma(q, r, 1.0 / 120.0);
  q = fma(q, r, 1.0 / 24.0);
  q = fma(q, r, 1.0 / 6.0);
  q = fma(q, r, 0.5);
  q = fma(q, r, 1.0);
  const double t = __ldg(&kExp2Table32[j]);
  const double m = fma(t, r * q, t);
  return m * __longlong_as_double(static_cast<long long>(k + 1023) << 52);
}

}  // namespace drt
