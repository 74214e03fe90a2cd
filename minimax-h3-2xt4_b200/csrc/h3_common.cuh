// Shared device helpers for the B200 tensor-parallel W8A8 INT8 linear path.
//
// Every floating-point step that the reference writes as an explicitly rounded
// intrinsic (__fadd_rn, __fmul_rn, __fdiv_rn, __fmaf_rn in the TileLang sources of
// patches/tilelang_*.py) is written the same way here, so the compiler can neither
// contract nor reorder it.  The library is also built with --fmad=false.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/h3b200.h"

#define H3_DEV __device__ __forceinline__

namespace h3 {

// ---------------------------------------------------------------------------
// Bit-pattern float constants (exactly the float32 values the reference uses).
// ---------------------------------------------------------------------------
H3_DEV float f32_bits(uint32_t b) { return __uint_as_float(b); }

// float32(1/127): tilelang_row_quant.py:38, tilelang_swiglu_quant.py:58
#define H3_INV127_BITS 0x3c010204u
// float32(1e-30): the scale floor of the same lines
#define H3_SCALE_FLOOR_BITS 0x0da24260u

// ---------------------------------------------------------------------------
// h3_expf: exp(x) for the SwiGLU denominator.
//
// The reference calls CUDA's expf (tilelang_swiglu_quant.py:22).  A CPU oracle
// cannot reproduce that bit for bit, so the path uses its own exponential, written
// from the Cody-Waite argument reduction (Cody & Waite, "Software Manual for the
// Elementary Functions", 1980) with a two-part ln2 whose rounding error is carried
// along, the degree-8 Taylor polynomial of exp(r) - 1 - r on |r| <= ln2/2, and a
// Fast2Sum (Dekker 1971) of 1 + r so only the final addition rounds at full weight.
// Every step is an explicit IEEE RN operation; the CPU oracle restates the same steps
// and is bit-identical.  Measured on the CPU: <= 0.61 ulp, correctly rounded for
// 99.3% of the fp16 inputs the SwiGLU sees.  The disagreement against CUDA expf is
// measured on the GPU by tests/test_gpu_kernels.py.
// ---------------------------------------------------------------------------
// Shared core: for xc in [-104, 89], n = rint(xc / ln2) and y = exp(xc - n ln2) in
// [0.7, 1.42], such that exp(xc) = y * 2^n.
H3_DEV void exp_core(float xc, float& y, int& ni) {
  const float l2e = f32_bits(0x3fb8aa3bu);       // float32(1/ln 2)
  const float ln2_hi = f32_bits(0x3f317200u);    // 16 significant bits
  const float ln2_lo = f32_bits(0x35bfbe8eu);    // float32(ln2 - ln2_hi)
  // n = rint(xc / ln2) by the 1.5 * 2^23 addition (|xc / ln2| < 2^22), integer from
  // the low mantissa bits
  const float big = __fadd_rn(__fmul_rn(xc, l2e), 12582912.0f);
  const float n = __fadd_rn(big, -12582912.0f);
  const float r1 = __fmaf_rn(-n, ln2_hi, xc);                // exact
  const float r = __fmaf_rn(-n, ln2_lo, r1);                 // rounded reduced argument
  const float corr = __fmaf_rn(-n, ln2_lo, __fadd_rn(r1, -r));  // its rounding error
  float t = __fmaf_rn(r, f32_bits(0x37d00d01u), f32_bits(0x39500d01u));  // 1/40320, 1/5040
  t = __fmaf_rn(t, r, f32_bits(0x3ab60b61u));                             // 1/720
  t = __fmaf_rn(t, r, f32_bits(0x3c088889u));                             // 1/120
  t = __fmaf_rn(t, r, f32_bits(0x3d2aaaabu));                             // 1/24
  t = __fmaf_rn(t, r, f32_bits(0x3e2aaaabu));                             // 1/6
  t = __fmaf_rn(t, r, 0.5f);
  const float s = __fmaf_rn(t, __fmul_rn(r, r), corr);
  const float hi = __fadd_rn(1.0f, r);
  const float lo = __fadd_rn(r, -__fadd_rn(hi, -1.0f));      // exact error of 1 + r
  y = __fadd_rn(hi, __fadd_rn(lo, s));
  ni = __float_as_int(big) - 0x4B400000;
}

H3_DEV float h3_expf(float x) {
  // Branch-free: the reduction runs on x clamped to [-104, 89] and the special
  // results (overflow to +inf, underflow to 0, NaN) are selected at the end, which is
  // the same value the early-return form gives for every input.
  const float xc = fminf(fmaxf(x, -104.0f), 89.0f);
  float y;
  int ni;
  exp_core(xc, y, ni);
  const int h = ni >> 1;                         // floor(ni / 2)
  const float s1 = __uint_as_float((uint32_t)(h + 127) << 23);
  const float s2 = __uint_as_float((uint32_t)(ni - h + 127) << 23);
  float res = __fmul_rn(__fmul_rn(y, s1), s2);
  res = (x > 89.0f) ? __uint_as_float(0x7f800000u) : res;
  res = (x < -104.0f) ? 0.0f : res;
  return (x != x) ? __fadd_rn(x, x) : res;
}

// 1 +rn h3_expf(-g), for every non-NaN float g, at lower cost.  Outside
// -g in [-17, 88.9] the sum is already decided: for -g < -17, exp(-g) < 2^-24 and
// 1 + exp(-g) rounds to 1, which exp(-17) gives too; for -g > 88.9 both overflow to
// +inf.  Inside, n >= -25, so y * 2^(n-1) is an exact normal product and the final
// doubling is exact or overflows exactly where (y * 2^h) * 2^(n-h) does.  A NaN g
// yields 1 here (instead of NaN), which still makes g / den NaN.
H3_DEV float silu_den(float g) {
  const float x = fminf(fmaxf(-g, -17.0f), 88.9f);
  float y;
  int ni;
  exp_core(x, y, ni);
  const float s = __uint_as_float((uint32_t)(ni - 1 + 127) << 23);
  return __fadd_rn(1.0f, __fmul_rn(__fmul_rn(y, s), 2.0f));
}

// silu(g) = g /rn (1 +rn exp(-g)), the activation half of the reference's SwiGLU
// (tilelang_swiglu_quant.py:22-23), reference form.
H3_DEV float silu_ieee(float g) {
  return __fdiv_rn(g, __fadd_rn(1.0f, h3_expf(-g)));
}

// The same value as silu_ieee for every gate that is an fp16 value (the only gates the
// path has: the reference rounds them to fp16 first, tilelang_swiglu_quant.py:21),
// branch-free and without the IEEE division's slow path.  Both operands are scaled,
// exactly, by 2^-64 (|g| >= 2^-24 or g = 0, den in [1, FLT_MAX]), so the reciprocal
// and every intermediate below stay normal.  The quotient is computed by division of
// our own: y = rcp.approx(den'), then the quotient correction of P. Markstein (IBM J.
// Res. Dev. 34(1), 1990): q0 = g' y, r = g' - q0 den' (exact), q = q0 + r y; on
// sm_100 this is correctly rounded for every denominator the fp16 gates produce
// (checked exhaustively, below).  Infinite and NaN quotients keep q0 (the
// IEEE result for g = +-inf or NaN), an infinite denominator (g < -88.7) gives g * 0
// (-0 for a finite g, NaN for -inf, as g / inf does), and a zero quotient takes the
// sign of g.  Verified bit-identical to silu_ieee on all 65536 fp16 gate values
// (tests/test_gpu_kernels.py).
H3_DEV float silu_fast(float g) {
  const float den = silu_den(g);
  const float a = __fmul_rn(g, 5.421010862427522e-20f);      // 2^-64
  const float nb = __fmul_rn(den, -5.421010862427522e-20f);  // -den * 2^-64
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(-nb));
  const float q0 = __fmul_rn(a, y);
  float q = __fmaf_rn(__fmaf_rn(q0, nb, a), y, q0);
  const float inf = __uint_as_float(0x7f800000u);
  q = fabsf(q0) < inf ? q : q0;
  q = den == inf ? __fmul_rn(g, 0.0f) : q;
  return __uint_as_float((__float_as_uint(q) & 0x7fffffffu) | (__float_as_uint(g) & 0x80000000u));
}

// FP32 SwiGLU of one (gate, up) pair, in the order of tilelang_swiglu_quant.py:21-24:
//   a = (gate /rn (1 +rn exp(-gate))) *rn up
H3_DEV float swiglu_f32(float gate, float up) { return __fmul_rn(silu_fast(gate), up); }

// ---------------------------------------------------------------------------
// Packed FP32 pairs.  sm_100's add / sub / mul / fma .rn.f32x2 instructions work on two
// floats held in one 64-bit register pair and round each lane exactly as the scalar
// .rn instruction does, so two independent computations written with them give the
// same bits as the scalar form at half the instruction issue.  One caution, measured:
// a mul.rn.f32x2 whose result feeds an add.rn.f32x2 can be contracted into a fused
// multiply-add by the assembler, so a product that feeds an addition is written with
// the scalar __fmul_rn / __fadd_rn (never contracted) or as an explicit fma.
// ---------------------------------------------------------------------------
typedef uint64_t f32x2;

H3_DEV f32x2 pk2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
H3_DEV f32x2 dup2(float v) { return pk2(v, v); }
H3_DEV float lo2(f32x2 v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  (void)b;
  return a;
}
H3_DEV float hi2(f32x2 v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  (void)a;
  return b;
}
H3_DEV f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
H3_DEV f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
H3_DEV f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
H3_DEV f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// ---------------------------------------------------------------------------
// The SwiGLU of two independent (gate, up) pairs on packed lanes: exp_core, silu_den,
// silu_fast and swiglu_f32 above, operation for operation, with every add / sub / mul
// / fma that can run on f32x2 doing so.  Rewrites that keep the bits: -n * c is
// written n * (-c) (the same product), a + (-b) as a - b, and 1 + (y s) 2 as one fma
// of the exactly doubled product.  The products that feed an addition stay scalar
// (xc * log2(e)) or feed only a multiplicand, so no contraction can change a rounding.
// Checked bit-identical to the scalar form on every fp16 gate by h3_silu_compare.
// ---------------------------------------------------------------------------
H3_DEV void exp_core2(float x0, float x1, f32x2& y, int& n0, int& n1) {
  const float l2e = f32_bits(0x3fb8aa3bu);
  const float big0 = __fadd_rn(__fmul_rn(x0, l2e), 12582912.0f);
  const float big1 = __fadd_rn(__fmul_rn(x1, l2e), 12582912.0f);
  const f32x2 n = add2(pk2(big0, big1), dup2(-12582912.0f));
  const f32x2 r1 = fma2(n, dup2(-f32_bits(0x3f317200u)), pk2(x0, x1));
  const f32x2 m_lo = dup2(-f32_bits(0x35bfbe8eu));
  const f32x2 r = fma2(n, m_lo, r1);
  const f32x2 corr = fma2(n, m_lo, sub2(r1, r));
  f32x2 t = fma2(r, dup2(f32_bits(0x37d00d01u)), dup2(f32_bits(0x39500d01u)));
  t = fma2(t, r, dup2(f32_bits(0x3ab60b61u)));
  t = fma2(t, r, dup2(f32_bits(0x3c088889u)));
  t = fma2(t, r, dup2(f32_bits(0x3d2aaaabu)));
  t = fma2(t, r, dup2(f32_bits(0x3e2aaaabu)));
  t = fma2(t, r, dup2(0.5f));
  const f32x2 sp = fma2(t, mul2(r, r), corr);
  const f32x2 one = dup2(1.0f);
  const f32x2 hi = add2(one, r);
  const f32x2 lo = sub2(r, sub2(hi, one));
  y = add2(hi, add2(lo, sp));
  n0 = __float_as_int(big0) - 0x4B400000;
  n1 = __float_as_int(big1) - 0x4B400000;
}

H3_DEV f32x2 silu_den2(float g0, float g1) {
  f32x2 y;
  int n0, n1;
  exp_core2(fminf(fmaxf(-g0, -17.0f), 88.9f), fminf(fmaxf(-g1, -17.0f), 88.9f), y, n0, n1);
  const f32x2 s = pk2(__uint_as_float((uint32_t)(n0 + 126) << 23),
                      __uint_as_float((uint32_t)(n1 + 126) << 23));
  return fma2(mul2(y, s), dup2(2.0f), dup2(1.0f));
}

H3_DEV float silu_fix(float g, float den, float q0, float q) {
  const float inf = __uint_as_float(0x7f800000u);
  q = fabsf(q0) < inf ? q : q0;
  q = den == inf ? __fmul_rn(g, 0.0f) : q;
  return __uint_as_float((__float_as_uint(q) & 0x7fffffffu) | (__float_as_uint(g) & 0x80000000u));
}

H3_DEV f32x2 silu_fast2(float g0, float g1) {
  const f32x2 den = silu_den2(g0, g1);
  const f32x2 a = mul2(pk2(g0, g1), dup2(5.421010862427522e-20f));   // 2^-64
  const f32x2 nb = mul2(den, dup2(-5.421010862427522e-20f));
  float y0, y1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(-lo2(nb)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y1) : "f"(-hi2(nb)));
  const f32x2 y = pk2(y0, y1);
  const f32x2 q0 = mul2(a, y);
  const f32x2 q = fma2(fma2(q0, nb, a), y, q0);
  return pk2(silu_fix(g0, lo2(den), lo2(q0), lo2(q)), silu_fix(g1, hi2(den), hi2(q0), hi2(q)));
}

// swiglu_f32 of two (gate, up) pairs.  The final products are the scalar __fmul_rn,
// which is never contracted: a caller may add the result (the ConvRot butterfly does),
// and a mul.rn.f32x2 feeding an add.rn.f32x2 can become a fused multiply-add.
H3_DEV f32x2 swiglu_f32x2(float g0, float g1, float u0, float u1) {
  const f32x2 s = silu_fast2(g0, g1);
  return pk2(__fmul_rn(lo2(s), u0), __fmul_rn(hi2(s), u1));
}

// Row scale of the production row quantizer (tilelang_row_quant.py:37-38):
//   scale = fmaxf(fminf(max, FLT_MAX) *rn float32(1/127), 1e-30)
H3_DEV float row_scale_from_max(float m) {
  const float mm = fminf(m, 3.4028234663852886e38f);
  return fmaxf(__fmul_rn(mm, f32_bits(H3_INV127_BITS)), f32_bits(H3_SCALE_FLOOR_BITS));
}

// One INT8 code (tilelang_row_quant.py:40-44).  division: 0 = IEEE (__fdiv_rn),
// 1 = the reference's production '__fdividef' fast division.
H3_DEV int8_t quantize_code(float x, float scale, int division) {
  const float scaled = division ? __fdividef(x, scale) : __fdiv_rn(x, scale);
  const float rounded = rintf(scaled);
  const float clipped = fminf(127.0f, fmaxf(-128.0f, rounded));
  return (int8_t)(int)clipped;
}

// x / scale, correctly rounded, from inv = RN(1 / scale) (computed once per row): the
// quotient correction step of P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990 - with a correctly
// rounded reciprocal and a first quotient within one ulp, RN(q0 + (x - q0*scale)*inv)
// is RN(x / scale); the remainder is exact in one FMA.  Infinite and NaN quotients
// take q0, which is then the IEEE result (scale is finite and >= 1e-30).
H3_DEV float div_by_scale(float x, float scale, float inv) {
  const float q0 = __fmul_rn(x, inv);
  const float r = __fmaf_rn(-q0, scale, x);
  const float q1 = __fmaf_rn(r, inv, q0);
  return fabsf(q0) < __uint_as_float(0x7f800000u) ? q1 : q0;
}

// The same code as quantize_code(x, scale, 0) without conversion-unit work: clamping
// before rounding gives the same integer (rint is monotone and the bounds are
// integers), and adding 1.5 * 2^23 rounds |t| <= 128 to the nearest integer, ties to
// even, leaving it in the low mantissa bits.
H3_DEV int8_t quantize_code_rn(float x, float scale, float inv) {
  const float t = fminf(127.0f, fmaxf(-128.0f, div_by_scale(x, scale, inv)));
  return (int8_t)(__float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000);
}

H3_DEV int8_t quantize_code_mode(float x, float scale, float inv, int division) {
  return division ? quantize_code(x, scale, 1) : quantize_code_rn(x, scale, inv);
}

// ---------------------------------------------------------------------------
// Regular ConvRot256 butterfly (tilelang_swiglu_quant.py:26-36,46) on two 256-value
// groups at once: lane 0 of every f32x2 pair holds one group's value, lane 1 the
// other's.  One radix-4 stage over a 16-value register block, stride S in {1, 4};
// output digit d of each 4-point set (a, b, c, d) is
//   d=0: ((a+b)+c)-d   d=1: ((a+b)-c)+d   d=2: ((a-b)+c)+d   d=3: ((b-a)+c)+d
// which is B[i] = ((p+q)+r)+s with the reference's negations; every addition is the
// f32x2 form of the IEEE RN one (x + (-y) and x - y are the same operation).
// ---------------------------------------------------------------------------
template <int S>
H3_DEV void radix4_stage2(f32x2 (&v)[16]) {
#pragma unroll
  for (int base = 0; base < 16; ++base) {
    if ((base / S) % 4 != 0) continue;
    const f32x2 a = v[base], b = v[base + S], c = v[base + 2 * S], d = v[base + 3 * S];
    const f32x2 ab = add2(a, b);
    v[base]         = sub2(add2(ab, c), d);
    v[base + S]     = add2(sub2(ab, c), d);
    v[base + 2 * S] = add2(add2(sub2(a, b), c), d);
    v[base + 3 * S] = add2(add2(sub2(b, a), c), d);
  }
}

// Full 256-point rotation of two groups held by 16 consecutive lanes of a warp (lane
// % 16 == block index b, v[j] = element 16*b + j of each group on entry).  Stages 0-1
// run on the lane's own block, a transpose through shared memory hands every lane the
// 16 values {16*t + r}, stages 2-3 run on those, and a second transpose restores
// v[j] = rotated element 16*b + j, multiplied by 1/16.  tile: 16 x 17 pairs of shared
// memory private to this half warp.
H3_DEV void convrot256_halfwarp2(f32x2 (&v)[16], f32x2* tile, int b) {
  radix4_stage2<1>(v);
  radix4_stage2<4>(v);
#pragma unroll
  for (int j = 0; j < 16; ++j) tile[b * 17 + j] = v[j];
  __syncwarp();
#pragma unroll
  for (int t = 0; t < 16; ++t) v[t] = tile[t * 17 + b];
  __syncwarp();
  radix4_stage2<1>(v);
  radix4_stage2<4>(v);
  const f32x2 sixteenth = dup2(0.0625f);
#pragma unroll
  for (int t = 0; t < 16; ++t) tile[t * 17 + b] = mul2(v[t], sixteenth);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = tile[b * 17 + j];
  __syncwarp();
}

// max(m, |a|, |b|), NaN if any operand is NaN (three-input max of sm_100).
H3_DEV float max_abs2_nan(float m, float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return r;
}

// Codes of 16 pairs for a row whose maximum m (over the very values quantised) is
// finite: then |x / scale| <= 127 * (1 + 2^-23), so the clamp of quantize_code_rn never
// changes its input and the quotient is never infinite, and the code is the low byte
// of RN(div_by_scale(x) + 1.5 * 2^23).  c0 receives lane 0's codes, c1 lane 1's.
H3_DEV void quantize_pairs_finite(const f32x2 (&v)[16], float scale, float inv, uint4& c0,
                                  uint4& c1) {
  const f32x2 i2 = dup2(inv), ns = dup2(-scale), magic = dup2(12582912.0f);
  uint32_t w0[4], w1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const f32x2 x = v[4 * k + e];
      const f32x2 q0 = mul2(x, i2);
      const f32x2 t = add2(fma2(fma2(q0, ns, x), i2, q0), magic);
      lo[e] = __float_as_uint(lo2(t));
      hi[e] = __float_as_uint(hi2(t));
    }
    w0[k] = __byte_perm(__byte_perm(lo[0], lo[1], 0x0040), __byte_perm(lo[2], lo[3], 0x0040), 0x5410);
    w1[k] = __byte_perm(__byte_perm(hi[0], hi[1], 0x0040), __byte_perm(hi[2], hi[3], 0x0040), 0x5410);
  }
  c0 = make_uint4(w0[0], w0[1], w0[2], w0[3]);
  c1 = make_uint4(w1[0], w1[1], w1[2], w1[3]);
}

// ---------------------------------------------------------------------------
// Vector load/store helpers.
// ---------------------------------------------------------------------------
H3_DEV void load_half16_as_float(const __half* p, float (&v)[16]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  uint4 u0 = __ldg(q), u1 = __ldg(q + 1);
  const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
  const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f0 = __half22float2(h0[i]);
    float2 f1 = __half22float2(h1[i]);
    v[2 * i] = f0.x; v[2 * i + 1] = f0.y;
    v[8 + 2 * i] = f1.x; v[8 + 2 * i + 1] = f1.y;
  }
}

H3_DEV void load_float16(const float* p, float (&v)[16]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 f = __ldg(q + i);
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
}

H3_DEV void store_float16(float* p, const float (&v)[16]) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

H3_DEV void store_int8x16(int8_t* p, const int8_t (&c)[16]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = (uint32_t)(uint8_t)c[4 * i] | ((uint32_t)(uint8_t)c[4 * i + 1] << 8) |
           ((uint32_t)(uint8_t)c[4 * i + 2] << 16) | ((uint32_t)(uint8_t)c[4 * i + 3] << 24);
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

H3_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Records an error code in the library's error word.  The word sits in host-mapped
// pinned memory (the no-allocation entry keeps its own in static device memory), so
// this is a plain system-scope store rather than an atomic: any non-zero code means a
// failure, and the host can read it while kernels are still running.
H3_DEV void report_error(int* err, int code) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(err), "r"(code) : "memory");
}

// ---------------------------------------------------------------------------
// Output stage shared by the row epilogues.
//   y: FP32 dequantised row output of one element
// ---------------------------------------------------------------------------
struct RowOut {
  int kind;
  void* out;
  __half* residual;
  const float* gate;
  int64_t gate_rows;
  const int32_t* labels;
  int* err;
};

H3_DEV float gate_value(const RowOut& o, int64_t r, int64_t c, int64_t width) {
  if (o.gate == nullptr) return 1.0f;
  int64_t lab = o.labels ? (int64_t)__ldg(o.labels + r) : 0;
  if (lab < 0 || lab >= o.gate_rows) {
    report_error(o.err, H3_ERR_INVALID);
    lab = 0;
  }
  return __ldg(o.gate + lab * width + c);
}

// Applies the out_kind of one element (tilelang_dit_fusion.py:68-75 for RESIDUAL).
H3_DEV void row_store(const RowOut& o, int64_t r, int64_t c, int64_t width, float y) {
  const int64_t idx = r * width + c;
  if (o.kind == H3_OUT_F32) {
    reinterpret_cast<float*>(o.out)[idx] = y;
  } else if (o.kind == H3_OUT_F16) {
    reinterpret_cast<__half*>(o.out)[idx] = __float2half_rn(y);
  } else {
    const float branch = __half2float(__float2half_rn(y));
    const float g = gate_value(o, r, c, width);
    const float x = __half2float(o.residual[idx]);
    o.residual[idx] = __float2half_rn(__fmaf_rn(branch, g, x));
  }
}

}  // namespace h3

// ---------------------------------------------------------------------------
// Host-side helpers shared by the entry points.
// ---------------------------------------------------------------------------
namespace h3host {

// Makes a device current for the lifetime of the object and, when it goes out of
// scope, makes the caller's previous device current again: an entry point never leaves
// the calling thread on another GPU.
class DeviceScope {
 public:
  DeviceScope() = default;
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
  ~DeviceScope();
  int bind(const void* ptr, int* device);  // the device owning ptr (host pointers: INVALID)
  int bind_index(int device);              // a device by ordinal

 private:
  int prev_ = -1;
};
int sm_count(int device);
int* error_word(int device);       // device view of the lazily created mapped error word
int* error_word_host(int device);  // host view of it (nullptr before its first use)
int check_launch();                                  // maps cudaGetLastError to a status
// Tensor map of `rows` rows of `row_bytes` bytes each (row pitch = row_bytes) viewed as
// uint8 [rows][row_bytes / 128][128], copied in boxes of box_lines 128-byte lines of
// one row with the 128-byte swizzle (row staging of the activation producers).
bool encode_row_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                    int box_lines);

inline bool aligned(const void* p, unsigned a) { return ((uintptr_t)p % a) == 0; }

}  // namespace h3host
