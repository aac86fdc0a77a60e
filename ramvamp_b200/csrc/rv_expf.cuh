// rv_expf.cuh -- the SiLU exponential, bit-identical to the host libm expf.
//
// The reference's SiLU is v / (1 + (-v).exp()) in f32
// (kernels/primitives/activation.rs:14-16) and Rust's f32::exp is glibc's
// expf, which is not correctly rounded.  expf_ref(x) reproduces it: exp is
// evaluated in double and rounded to float, which is the correctly rounded
// result except within ~2^-28 ulp of a rounding midpoint; only when the
// double result lies within 2^-9 ulp of a midpoint (about 0.4% of inputs) is
// x looked up in an open-addressing table of the inputs where the host expf
// differs from that (gen_expf_exceptions.c builds the list at build time
// from the host libm: 170,648 misrounded inputs, all within 0.0017 ulp of a
// midpoint, plus 50 inputs within 2^-24 ulp of one).
#pragma once
#include "rv_internal.cuh"

#define RV_EXPF_TABLE_BITS 19
#define RV_EXPF_TABLE_SIZE (1u << RV_EXPF_TABLE_BITS)
#define RV_EXPF_EMPTY 0xFFFFFFFFu

// key = input bits, value = host expf bits; EMPTY keys are NaN patterns.
__device__ uint2 g_expf_table[RV_EXPF_TABLE_SIZE];
__constant__ int g_expf_max_probe;

__host__ __device__ inline uint32_t rv_expf_hash(uint32_t key) {
  return (key * 2654435761u) >> (32 - RV_EXPF_TABLE_BITS);
}

RV_DEVFN bool expf_near_midpoint(double yd, float f) {
  if (isnan(f)) return false;
  if (isinf(f)) return true;  // overflow boundary: always consult the table
  const float up = nextafterf(f, INFINITY), dn = nextafterf(f, -INFINITY);
  if (isinf(up)) return true;
  const double df = (double)f, dup = (double)up, ddn = (double)dn;
  const double mh = 0.5 * (df + dup), ml = 0.5 * (df + ddn);  // exact in double
  return (mh - yd) <= (dup - df) * 0x1p-9 || (yd - ml) <= (df - ddn) * 0x1p-9;
}

RV_DEVFN float expf_ref(float x) {
  const double yd = exp((double)x);
  const float f = __double2float_rn(yd);
  if (!expf_near_midpoint(yd, f)) return f;
  const uint32_t key = __float_as_uint(x);
  uint32_t h = rv_expf_hash(key);
  const int probes = g_expf_max_probe;
  for (int p = 0; p <= probes; p++) {
    const uint2 e = g_expf_table[(h + (uint32_t)p) & (RV_EXPF_TABLE_SIZE - 1)];
    if (e.x == key) return __uint_as_float(e.y);
    if (e.x == RV_EXPF_EMPTY) break;
  }
  return f;
}

// silu(g) * u exactly as activation.rs:14-16, 161-163 evaluates it.
RV_DEVFN float swiglu_ref(float g, float u) {
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf_ref(-g)));
  return __fmul_rn(s, u);
}
