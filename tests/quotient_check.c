/* Exhaustive check of the quotient used by the packed int8 row quantizer (quant_rows16_kernel in
 * mac-kernels-public_b200/csrc/qlin_aux.cu).
 *
 * The kernel forms x / s as Markstein's correction (P. Markstein, IBM J. Res. Dev. 34(1), 1990):
 *   y = RN(1/s),  q0 = RN(x*y),  r = fma(q0, -s, x),  q = fma(r, y, q0)
 * where the reference divides, q = RN(x/s), and then maps the quotient to the code
 * sat8(rint(RN_dtype(q))).  For one input dtype (fp16 or bf16, argv[1]) this program takes every
 * finite x and every s the quantizer can meet: s = RN_dtype(max(amax / 127, 1e-30)), so every
 * positive finite fp16 value (the smallest normal replaces a zero), or every bf16 value from
 * RN_bf16(1e-30) up; the kernel divides when s > 1e37.  It counts the pairs whose Markstein
 * quotient differs from the IEEE quotient (+0 and -0 compare equal) with |x/s| >= 1/16, and the
 * pairs whose codes differ; both must be zero.  (Below 1/16 the residual r of the smallest bf16 s
 * can fall among the subnormals and the quotient can be off by one unit in the last place; such
 * quotients round to code 0 either way, which the code count confirms.)  Pairs outside 2^-30 s <= |x| <= 256 s are not
 * evaluated: the row's values satisfy |x| <= amax, and amax / s <= 191 (fp16 s rounded down to the
 * smallest subnormal at worst; bf16 at most 127.3), so larger quotients do not occur; below 2^-30
 * both quotients lie under 2^-29 and the code is 0.  The arithmetic is the host's IEEE single
 * precision (round to nearest even, subnormals kept), the same operations the kernel issues.
 * Output: "<dtype> pairs <n> quotient mismatches <a> code mismatches <b>"; exit status 1 unless
 * both are zero.
 *
 * Build: gcc -O2 -mfma -ffp-contract=off quotient_check.c -o quotient_check -lm
 * (-DPLANT_UNCORRECTED builds a planted mistake, q = q0 without the correction, which must fail.)
 * The scan stops after 1000 mismatches of either kind.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint32_t to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* fp16 bit pattern -> float (exact), from the format's definition: 1 sign, 5 exponent (bias 15),
 * 10 fraction bits; exponent 0 subnormal, 31 infinity / NaN. */
static float f16_value(uint16_t h) {
  const int sign = h >> 15, e = (h >> 10) & 31, f = h & 1023;
  float v;
  if (e == 0) v = ldexpf((float)f, -24);
  else if (e == 31) v = f ? NAN : INFINITY;
  else v = ldexpf((float)(1024 + f), e - 25);
  return sign ? -v : v;
}

static float bf16_value(uint16_t h) { return from_bits((uint32_t)h << 16); }

/* Round to the nearest fp16 / bf16 value, ties to even (overflow to infinity). */
static float round_dtype(float q, int bf16) {
  const float a = fabsf(q);
  if (a == 0.f || !isfinite(q)) return q;
  int e;
  frexpf(a, &e); /* a in [2^(e-1), 2^e) */
  int lsb = e - (bf16 ? 8 : 11);
  if (!bf16 && lsb < -24) lsb = -24; /* fp16 subnormal spacing */
  const float r = ldexpf(nearbyintf(ldexpf(a, -lsb)), lsb);
  if (!bf16 && r >= 65520.f) return copysignf(INFINITY, q);
  return copysignf(r, q);
}

static int code_of(float q, int bf16) {
  float h = round_dtype(q, bf16);
  h = fminf(fmaxf(h, -128.f), 127.f);
  return (int)nearbyintf(h);
}

int main(int argc, char** argv) {
  const int bf16 = argc > 1 && strcmp(argv[1], "bf16") == 0;
  const float s_min = bf16 ? bf16_value((uint16_t)(to_bits(1e-30f) >> 16)) : 0.f;
  float* xs = malloc(sizeof(float) * 65536);
  float* ss = malloc(sizeof(float) * 65536);
  int nx = 0, ns = 0;
  for (uint32_t h = 0; h < 65536; ++h) {
    const float v = bf16 ? bf16_value((uint16_t)h) : f16_value((uint16_t)h);
    if (!isfinite(v)) continue;
    xs[nx++] = v;
    if (v > 0.f && v >= s_min && v <= 1e37f) ss[ns++] = v;
  }
  long long pairs = 0, bad_q = 0, bad_code = 0;
  for (int i = 0; i < ns; ++i) {
    const float s = ss[i];
    const float y = 1.0f / s, nsv = -s, lo = ldexpf(s, -30), hi = 256.f * s;
    for (int j = 0; j < nx; ++j) {
      const float x = xs[j];
      if (fabsf(x) < lo || fabsf(x) > hi) continue;
      ++pairs;
      const float q0 = x * y;
      const float r = fmaf(q0, nsv, x);
#ifdef PLANT_UNCORRECTED
      const float q = q0 + 0.f * r;
#else
      const float q = fmaf(r, y, q0);
#endif
      const float d = x / s;
      if (q == d) continue;
      if (fabsf(d) >= 0x1p-4f) {
        if (bad_q < 8) fprintf(stderr, "x = %a, s = %a: %a != %a\n", x, s, q, d);
        ++bad_q;
      }
      bad_code += code_of(q, bf16) != code_of(d, bf16);
    }
    if (bad_q >= 1000 || bad_code >= 1000) break;
  }
  printf("%s pairs %lld quotient mismatches %lld code mismatches %lld\n", bf16 ? "bf16" : "fp16", pairs, bad_q,
         bad_code);
  free(xs);
  free(ss);
  return bad_q != 0 || bad_code != 0;
}
