// rk_detmath.cuh — the reference's deterministic float64 functions on the
// device: num.Log (internal/num/num.go:128-163), num.Exp (num.go:101-123)
// and num.Sincos (num.go:244-297), every operation an explicitly rounded
// IEEE double operation, so that they return the CPU's bits.
#pragma once
#include "rk_common.cuh"

namespace rk {

RK_DEV uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// num.Log for positive normal x (num.go:128-163), every operation rounded.
RK_DEV double log_det(double x) {
  const double ln2Hi = 6.93147180369123816490e-01, ln2Lo = 1.90821492927058770002e-10;
  const double l1 = 6.666666666666735130e-01, l2 = 3.999999999940941908e-01, l3 = 2.857142874366239149e-01,
               l4 = 2.222219843214978396e-01, l5 = 1.818357216161805012e-01, l6 = 1.531383769920937332e-01,
               l7 = 1.479819860511658591e-01;
  const unsigned long long b = __double_as_longlong(x);
  int ki = int((b >> 52) & 0x7ff) - 1022;
  double f1 = __longlong_as_double((long long)((b & 0x000fffffffffffffull) | (1022ull << 52)));  // [0.5, 1)
  if (f1 < 0x1.6a09e667f3bcdp-1) {
    f1 = __dmul_rn(f1, 2.0);
    ki--;
  }
  const double f = __dsub_rn(f1, 1.0);
  const double k = double(ki);
  const double s = __ddiv_rn(f, __dadd_rn(2.0, f));
  const double s2 = __dmul_rn(s, s);
  const double s4 = __dmul_rn(s2, s2);
  const double t1 =
      __dmul_rn(s2, __dadd_rn(l1, __dmul_rn(s4, __dadd_rn(l3, __dmul_rn(s4, __dadd_rn(l5, __dmul_rn(s4, l7)))))));
  const double t2 = __dmul_rn(s4, __dadd_rn(l2, __dmul_rn(s4, __dadd_rn(l4, __dmul_rn(s4, l6)))));
  const double r = __dadd_rn(t1, t2);
  const double hfsq = __dmul_rn(__dmul_rn(0.5, f), f);
  return __dsub_rn(__dmul_rn(k, ln2Hi),
                   __dsub_rn(__dsub_rn(hfsq, __dadd_rn(__dmul_rn(s, __dadd_rn(hfsq, r)), __dmul_rn(k, ln2Lo))), f));
}

// num.Sincos (num.go:244-297).
RK_DEV void sincos_det(double x, double &sn, double &cs) {
  const double pio2a = 1.57079632673412561417e+00, pio2b = 6.07710050630396597660e-11,
               pio2c = 2.02226624879595063154e-21;
  const double sc[6] = {1.58962301576546568060e-10, -2.50507477628578072866e-8, 2.75573136213857245213e-6,
                        -1.98412698295895385996e-4, 8.33333333332211858878e-3,  -1.66666666666666307295e-1};
  const double cc[6] = {-1.13585365213876817300e-11, 2.08757008419747316778e-9, -2.75573141792967388112e-7,
                        2.48015872888517045348e-5,  -1.38888888888730564116e-3, 4.16666666666665929218e-2};
  const double k = rint(__dmul_rn(x, 0x1.45f306dc9c883p-1));
  double r = __dsub_rn(x, __dmul_rn(k, pio2a));
  r = __dsub_rn(r, __dmul_rn(k, pio2b));
  r = __dsub_rn(r, __dmul_rn(k, pio2c));
  const double z = __dmul_rn(r, r);
  double ps = sc[0], pc = cc[0];
#pragma unroll
  for (int i = 1; i < 6; i++) {
    ps = __dadd_rn(__dmul_rn(ps, z), sc[i]);
    pc = __dadd_rn(__dmul_rn(pc, z), cc[i]);
  }
  const double s = __dadd_rn(r, __dmul_rn(__dmul_rn(r, z), ps));
  const double c = __dadd_rn(__dsub_rn(1.0, __dmul_rn(0.5, z)), __dmul_rn(__dmul_rn(z, z), pc));
  switch (((long long)k) & 3) {
    case 0: sn = s; cs = c; break;
    case 1: sn = c; cs = -s; break;
    case 2: sn = -s; cs = -c; break;
    default: sn = -c; cs = s; break;
  }
}

// num.Exp (num.go:101-123) for |x| within float64's normal range of e^x.
RK_DEV double exp_det(double x) {
  if (x != x) return x;
  if (x > 709.78) return __longlong_as_double(0x7ff0000000000000ll);
  if (x < -745.13) return 0.0;
  const double ln2Hi = 6.93147180369123816490e-01, ln2Lo = 1.90821492927058770002e-10;
  const double n = rint(__dmul_rn(x, 1.4426950408889634));
  double r = __dsub_rn(x, __dmul_rn(n, ln2Hi));
  r = __dsub_rn(r, __dmul_rn(n, ln2Lo));
  double p = 0x1.6124613a86d09p-33;  // 1.0/6227020800
  double fact[13];
  fact[0] = 1.0;
  for (int k = 1; k <= 12; k++) fact[k] = __dmul_rn(fact[k - 1], double(k < 2 ? 1 : k));
  for (int k = 12; k >= 0; k--) p = __dadd_rn(__dmul_rn(p, r), __ddiv_rn(1.0, fact[k]));
  const int ni = int(n);
  // p·2^n, exact while the result is a normal double (the callers' range).
  return __dmul_rn(p, __longlong_as_double((long long)(ni + 1023) << 52));
}

}  // namespace rk
