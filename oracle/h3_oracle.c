/*
 * ORACLE - TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's arithmetic for the tensor-parallel W8A8 INT8
 * linear path (chinokikiss/minimax-h3-2xt4, patches/).  Only tests/, the smoke
 * check of __graft_entry__.py and the cpu_baseline leg of bench.py load this
 * library, and only as the checker.  The product (libh3b200.so and the h3tp package)
 * never links, loads or calls it.
 *
 * Built with -ffp-contract=off and without -ffast-math, so every float expression
 * below is evaluated as written: one IEEE round-to-nearest-even operation per
 * operator, in source order, exactly as the reference's explicit __fadd_rn /
 * __fmul_rn / __fdiv_rn intrinsics do.  fmaf() is used only where the reference (or
 * the documented exponential) performs a fused multiply-add.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <float.h>

#define EXPORT __attribute__((visibility("default")))

static inline float bits2f(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t f2bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* ------------------------------------------------------------------------
 * IEEE binary16 <-> binary32 (round to nearest even, overflow to infinity)
 * --------------------------------------------------------------------- */
EXPORT float h3o_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t mant = h & 0x3ffu;
  if (exp == 0x1fu) return bits2f(sign | 0x7f800000u | (mant << 13));
  if (exp == 0) {
    const float v = (float)mant * bits2f(0x33800000u); /* mant * 2^-24, exact */
    return sign ? -v : v;
  }
  return bits2f(sign | ((exp - 15u + 127u) << 23) | (mant << 13));
}

EXPORT uint16_t h3o_float_to_half(float f) {
  const uint32_t x = f2bits(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    return (uint16_t)(sign | 0x7c00u);
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (ax >= 0x38800000u) {                                  /* normal binary16 */
    const uint32_t mant = ax & 0x7fffffu;
    const uint32_t exp = (ax >> 23) - 127u + 15u;
    uint32_t h = (exp << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
  }
  if (ax <= 0x33000000u) return sign; /* <= 2^-25: rounds to (signed) zero */
  {
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    const int e = (int)(ax >> 23);
    const int shift = 126 - e; /* 14..24 */
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
  }
}

static inline float f16r(float v) { return h3o_half_to_float(h3o_float_to_half(v)); }

/* ------------------------------------------------------------------------
 * Exponential of the SwiGLU denominator: Cody-Waite reduction with a two-part
 * ln 2 (keeping the reduction's rounding error), the degree-8 Taylor polynomial of
 * exp(r) - 1 - r on |r| <= ln2/2, and a Fast2Sum of 1 + r so only the last addition
 * rounds at full weight.  This is the
 * path's documented replacement for CUDA expf (tilelang_swiglu_quant.py:22).
 * --------------------------------------------------------------------- */
EXPORT float h3o_expf(float x) {
  if (x != x) return x + x;
  if (x > 89.0f) return bits2f(0x7f800000u);
  if (x < -104.0f) return 0.0f;
  const float l2e = bits2f(0x3fb8aa3bu);
  const float ln2_hi = bits2f(0x3f317200u);
  const float ln2_lo = bits2f(0x35bfbe8eu);
  const float n = rintf(x * l2e);
  const float r1 = fmaf(-n, ln2_hi, x);     /* exact */
  const float r = fmaf(-n, ln2_lo, r1);     /* reduced argument, rounded */
  const float corr = fmaf(-n, ln2_lo, r1 - r); /* its rounding error */
  float t = fmaf(r, bits2f(0x37d00d01u), bits2f(0x39500d01u)); /* 1/40320, 1/5040 */
  t = fmaf(t, r, bits2f(0x3ab60b61u));     /* 1/720 */
  t = fmaf(t, r, bits2f(0x3c088889u));     /* 1/120 */
  t = fmaf(t, r, bits2f(0x3d2aaaabu));     /* 1/24 */
  t = fmaf(t, r, bits2f(0x3e2aaaabu));     /* 1/6 */
  t = fmaf(t, r, 0.5f);
  const float s = fmaf(t, r * r, corr);    /* exp(r) - 1 - r, plus the correction */
  const float hi = 1.0f + r;
  const float lo = r - (hi - 1.0f);        /* exact error of 1 + r (Fast2Sum) */
  const float y = hi + (lo + s);
  const int ni = (int)n;
  const int h = ni >> 1;
  const float s1 = bits2f((uint32_t)(h + 127) << 23);
  const float s2 = bits2f((uint32_t)(ni - h + 127) << 23);
  return (y * s1) * s2;
}

/* tilelang_swiglu_quant.py:21-24:
 *   activated = gate /rn (1 +rn expf(-gate)); A = activated *rn up */
EXPORT float h3o_swiglu(float gate, float up) {
  const float den = 1.0f + h3o_expf(-gate);
  const float act = gate / den;
  return act * up;
}

/* tilelang_swiglu_quant.py:26-36,46: four radix-4 stages with strides 1, 4, 16, 64;
 * B[i] = ((p+q)+r)+s, then each value times float32(1/16). */
EXPORT void h3o_convrot256(float* A) {
  float B[256];
  for (int stage = 0; stage < 4; ++stage) {
    const int stride = 1 << (2 * stage);
    for (int i = 0; i < 256; ++i) {
      const int digit = (i / stride) % 4;
      const int base = i - digit * stride;
      const float a = A[base], b = A[base + stride], c = A[base + 2 * stride],
                  d = A[base + 3 * stride];
      const float p = digit == 3 ? -a : a;
      const float q = digit == 2 ? -b : b;
      const float r = digit == 1 ? -c : c;
      const float s = digit == 0 ? -d : d;
      B[i] = ((p + q) + r) + s;
    }
    memcpy(A, B, sizeof(B));
  }
  for (int i = 0; i < 256; ++i) A[i] = A[i] * (1.0f / 16.0f);
}

/* Row scale and one code of the row quantizer (tilelang_row_quant.py:37-44),
 * division 'rn' (IEEE). */
static inline float row_scale(float m) {
  const float mm = fminf(m, FLT_MAX);
  return fmaxf(mm * bits2f(0x3c010204u), bits2f(0x0da24260u));
}
static inline int8_t code(float x, float scale) {
  const float scaled = x / scale;
  const float rounded = nearbyintf(scaled);
  const float clipped = fminf(127.0f, fmaxf(-128.0f, rounded));
  return (int8_t)(int)clipped;
}

/* FC2 producer, phase 'stored' (tilelang_swiglu_quant.py:37-51) plus the row
 * maximum of prepare (:86).  kind 0: fp16 [rows, 2*width] = [gate | up];
 * kind 1: fp32 [rows, width] activation; kind 2: fp16 [rows, width] activation. */
EXPORT void h3o_fc2_rotate(const void* x, int kind, int64_t rows, int64_t width, float* R,
                           float* rowmax) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float m = 0.0f;
    for (int64_t g = 0; g < width / 256; ++g) {
      float A[256];
      for (int i = 0; i < 256; ++i) {
        const int64_t c = g * 256 + i;
        if (kind == 0) {
          const uint16_t* xh = (const uint16_t*)x + r * 2 * width;
          A[i] = h3o_swiglu(h3o_half_to_float(xh[c]), h3o_half_to_float(xh[width + c]));
        } else if (kind == 1) {
          A[i] = ((const float*)x)[r * width + c];
        } else {
          A[i] = h3o_half_to_float(((const uint16_t*)x)[r * width + c]);
        }
      }
      h3o_convrot256(A);
      for (int i = 0; i < 256; ++i) {
        R[r * width + g * 256 + i] = A[i];
        m = fmaxf(m, fabsf(A[i]));
      }
    }
    rowmax[r] = m;
  }
}

/* Row quantizer with an external maximum (tilelang_row_quant.py:27-46, 'rn'). */
EXPORT void h3o_row_quantize(const float* X, int64_t rows, int64_t width, int64_t stride,
                             int64_t start, const float* rowmax, int8_t* q, float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float s = row_scale(rowmax[r]);
    for (int64_t c = 0; c < width; ++c) q[r * width + c] = code(X[r * stride + start + c], s);
    scale[r] = s;
  }
}

/* Column activation preparation (dit_column_linear.py:13-21) as this path defines it
 * where the Kitchen source is absent: rotated = f16(H256 x) in the butterfly order
 * above, then the row quantizer with the row's own maximum. */
EXPORT void h3o_column_quantize(const uint16_t* x, int64_t rows, int64_t k, int convrot,
                                int8_t* q, float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float m = 0.0f;
    float A[256];
    /* first pass: maximum */
    for (int64_t g = 0; g < (convrot ? k / 256 : 1); ++g) {
      if (convrot) {
        for (int i = 0; i < 256; ++i) A[i] = h3o_half_to_float(x[r * k + g * 256 + i]);
        h3o_convrot256(A);
        for (int i = 0; i < 256; ++i) m = fmaxf(m, fabsf(f16r(A[i])));
      } else {
        for (int64_t c = 0; c < k; ++c) m = fmaxf(m, fabsf(h3o_half_to_float(x[r * k + c])));
      }
    }
    const float s = row_scale(m);
    for (int64_t g = 0; g < (convrot ? k / 256 : 1); ++g) {
      if (convrot) {
        for (int i = 0; i < 256; ++i) A[i] = h3o_half_to_float(x[r * k + g * 256 + i]);
        h3o_convrot256(A);
        for (int i = 0; i < 256; ++i) q[r * k + g * 256 + i] = code(f16r(A[i]), s);
      } else {
        for (int64_t c = 0; c < k; ++c) q[r * k + c] = code(h3o_half_to_float(x[r * k + c]), s);
      }
    }
    scale[r] = s;
  }
}

/* Exact INT32 GEMM: C[m, n] = sum_k A[m, k] * W[n, k] (torch._int_mm semantics). */
EXPORT void h3o_int8_gemm(const int8_t* A, const int8_t* W, int64_t M, int64_t N, int64_t K,
                          int32_t* C) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    const int8_t* a = A + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const int8_t* w = W + n * K;
      int32_t acc = 0;
      for (int64_t k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)w[k];
      C[m * N + n] = acc;
    }
  }
}

/* Ordered column epilogue (tilelang_column_epilogue.py:11-27), optional bias added
 * after the product: y = f16((f32(C) * (A[m] * W[n])) + bias[n]). */
EXPORT void h3o_column_epilogue(const int32_t* C, int64_t M, int64_t N, const float* A,
                                const float* W, int64_t wlen, const float* bias, uint16_t* Y) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      const float s = A[m] * W[wlen == 1 ? 0 : n];
      float v = (float)C[m * N + n] * s;
      if (bias) v = v + bias[n];
      Y[m * N + n] = h3o_float_to_half(v);
    }
}

/* FC1 column output followed by the FC2 producer's SwiGLU, in one place:
 * C is [M, 2*Nh] = [gate | up] accumulators; y = swiglu(f16(col(gate)), f16(col(up))).
 * out_kind 0 stores fp32, 1 stores fp16. */
EXPORT void h3o_swiglu_epilogue(const int32_t* C, int64_t M, int64_t Nh, const float* A,
                                const float* W, const float* bias, int out_kind, void* out) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < Nh; ++n) {
      float vg = (float)C[m * 2 * Nh + n] * (A[m] * W[n]);
      float vu = (float)C[m * 2 * Nh + Nh + n] * (A[m] * W[Nh + n]);
      if (bias) {
        vg = vg + bias[n];
        vu = vu + bias[Nh + n];
      }
      const float y = h3o_swiglu(f16r(vg), f16r(vu));
      if (out_kind == 0)
        ((float*)out)[m * Nh + n] = y;
      else
        ((uint16_t*)out)[m * Nh + n] = h3o_float_to_half(y);
    }
}

/* Scaled-FP16 codec (tilelang_transport_tradeoffs.py:26-39). */
EXPORT void h3o_fp16_encode(const int32_t* P, int64_t n, int shift, uint16_t* Y) {
  const float f = ldexpf(1.0f, -shift);
  for (int64_t i = 0; i < n; ++i) Y[i] = h3o_float_to_half((float)P[i] * f);
}

static inline int32_t trunc_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return (int32_t)v; /* C conversion truncates toward zero */
}

EXPORT void h3o_fp16_decode(const uint16_t* Y, int64_t n, int shift, int32_t* P) {
  const float f = ldexpf(1.0f, shift);
  for (int64_t i = 0; i < n; ++i) P[i] = trunc_i32(h3o_half_to_float(Y[i]) * f);
}

/* Gated residual of tilelang_dit_fusion.py:68-75 for one element. */
static inline uint16_t gated(float y, float g, uint16_t x) {
  const float branch = f16r(y);
  return h3o_float_to_half(fmaf(branch, g, h3o_half_to_float(x)));
}

static void row_out(int out_kind, void* out, uint16_t* residual, const float* gate,
                    const int32_t* labels, int64_t r, int64_t c, int64_t width, float y) {
  const int64_t idx = r * width + c;
  if (out_kind == 0) {
    ((float*)out)[idx] = y;
  } else if (out_kind == 1) {
    ((uint16_t*)out)[idx] = h3o_float_to_half(y);
  } else {
    const float g = gate ? gate[(labels ? (int64_t)labels[r] : 0) * width + c] : 1.0f;
    residual[idx] = gated(y, g, residual[idx]);
  }
}

/* Partial reduction in rank order (fp32 sum, one fp16 rounding), then the reference's
 * fused epilogue (tilelang_transport_p2.py:15-47 / tilelang_dit_fusion.py:57-77). */
EXPORT void h3o_row_reduce_finish(const uint16_t* parts, int world, int64_t part_stride,
                                  int64_t rows, int64_t width, int shift, const float* A,
                                  const float* W, int out_kind, void* out, uint16_t* residual,
                                  const float* gate, const int32_t* labels) {
  const float up = ldexpf(1.0f, shift);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < width; ++c) {
      float t = h3o_half_to_float(parts[r * width + c]);
      for (int w = 1; w < world; ++w) t = t + h3o_half_to_float(parts[w * part_stride + r * width + c]);
      const float reduced = f16r(t);
      const int32_t restored = trunc_i32(reduced * up);
      const float value = (float)restored * A[r];
      const float y = value * W[c];
      row_out(out_kind, out, residual, gate, labels, r, c, width, y);
    }
}

/* parallel_int8.dequantize CPU branch (parallel_int8.py:66-69):
 * y = ((f32(acc) * a) * w) [+ bias], then cast. out_kind 0 fp32, 1 fp16,
 * 2 gated residual update (tilelang_dit_fusion.py gate order). */
EXPORT void h3o_dequantize_i32(const int32_t* acc, int64_t rows, int64_t width, const float* A,
                               const float* W, int64_t wlen, const float* bias, int out_kind,
                               void* out, uint16_t* residual, const float* gate,
                               const int32_t* labels) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < width; ++c) {
      float y = (float)acc[r * width + c] * A[r];
      y = y * W[wlen == 1 ? 0 : c];
      if (bias) y = y + bias[c];
      row_out(out_kind, out, residual, gate, labels, r, c, width, y);
    }
}

/* gated_add of h3_tensor_flow.py:145-152 (gate_kernel, tilelang_dit_fusion.py:39-53)
 * with an fp32 branch rounded to fp16 first: X = f16(fma(f16(y), G[label], X)). */
EXPORT void h3o_gated_add(const float* y, int64_t rows, int64_t width, uint16_t* residual,
                          const float* gate, const int32_t* labels) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < width; ++c)
      row_out(2, NULL, residual, gate, labels, r, c, width, y[r * width + c]);
}

/* ---------------------------------------------------------------------------
 * Packed INT8 transport ('int8_gather'): tilelang_transport_tradeoffs.py:40-62 (pack),
 * tilelang_transport_p2.py:28-42 (reconstruction inside the epilogue), and its torch
 * statement in benchmarks/tp2_tradeoffs.py:73-78.
 * Wire format per row: for each 128-column group, 128 code bytes (two's complement)
 * then the 4 bytes of the fp32 scale (little endian); row pitch = groups * 132.
 * ------------------------------------------------------------------------- */
static inline int32_t rint_i32(float v) {
  if (v != v) return 0;
  const float r = rintf(v); /* round half to even */
  if (r >= 2147483648.0f) return INT32_MAX;
  if (r <= -2147483648.0f) return INT32_MIN;
  return (int32_t)r;
}

/* scale = max(max_i |f32(P_i)| *rn f32(1/127), f32(1e-8));
 * q_i = clamp(rint(f32(P_i) /rn scale), -127, 127). */
EXPORT void h3o_pack8(const int32_t* P, int64_t rows, int64_t width, uint8_t* out) {
  const int64_t groups = width / 128, pitch = groups * 132;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t g = 0; g < groups; ++g) {
      const int32_t* p = P + r * width + g * 128;
      uint8_t* o = out + r * pitch + g * 132;
      float m = 0.0f;
      for (int i = 0; i < 128; ++i) m = fmaxf(m, fabsf((float)p[i]));
      const float s = fmaxf(m * bits2f(0x3c010204u), bits2f(0x322bcc77u));
      for (int i = 0; i < 128; ++i) {
        const float q = fminf(127.0f, fmaxf(-127.0f, rintf((float)p[i] / s)));
        o[i] = (uint8_t)(int8_t)(int)q;
      }
      memcpy(o + 128, &s, 4);
    }
}

/* restored = rint( sum_w f32(q_w) *rn s_w ), the sum in rank order with RN additions
 * (the reference's two-rank form: x0 +rn x1). parts: world payloads, part_stride bytes
 * apart. */
EXPORT void h3o_unpack8_restore(const uint8_t* parts, int world, int64_t part_stride,
                                int64_t rows, int64_t width, int32_t* out) {
  const int64_t groups = width / 128, pitch = groups * 132;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < width; ++c) {
      const int64_t g = c / 128, i = c % 128;
      float total = 0.0f;
      for (int w = 0; w < world; ++w) {
        const uint8_t* o = parts + w * part_stride + r * pitch + g * 132;
        float s;
        memcpy(&s, o + 128, 4);
        const float x = (float)(int8_t)o[i] * s;
        total = w == 0 ? x : total + x;
      }
      out[r * width + c] = rint_i32(total);
    }
}

/* ---------------------------------------------------------------------------
 * Modulated RMSNorm (tilelang_dit_fusion.py:11-37, h3_tensor_flow.py:134-143) as the
 * fused column producer computes it:
 *   ss = sum_i f32(x_i) *rn f32(x_i)            (the kernel's fixed order, below)
 *   mean = ss *rn f32(1/width);  inv = RN(1/sqrt(mean +rn f32(eps)))
 *   h_i = f16( (((f32(x_i) *rn inv) *rn W_i) *rn (1 +rn Scale[l][i])) +rn Shift[l][i] )
 * The reference's rsqrtf is CUDA's approximation and its sum order TileLang's; here the
 * reciprocal square root is correctly rounded and the order is fixed.
 * ------------------------------------------------------------------------- */

/* RN(1/sqrt(v)) for a positive finite float v, exactly: the double estimate is within
 * one float ulp, and the final choice compares v against the squared midpoints in
 * 128-bit integer arithmetic. */
static float rsqrt_rn(float v) {
  if (!(v > 0.0f)) return v == 0.0f ? INFINITY : NAN;
  if (isinf(v)) return 0.0f;
  float y = (float)(1.0 / sqrt((double)v));
  int ev;
  const double fv = frexp((double)v, &ev);               /* v = fv * 2^ev, fv in [0.5,1) */
  const unsigned __int128 V = (unsigned __int128)(uint64_t)ldexp(fv, 24); /* 24 bits */
  const int ve = ev - 24;
  for (int it = 0; it < 3; ++it) {
    /* candidate is correct iff lo_mid < 1/sqrt(v) < hi_mid, i.e. lo_mid^2 * v < 1 < hi_mid^2 * v */
    const float up = nextafterf(y, INFINITY), dn = nextafterf(y, 0.0f);
    int moved = 0;
    for (int side = 0; side < 2; ++side) {
      const double mid = 0.5 * ((double)y + (double)(side ? up : dn)); /* exact in double */
      int em;
      const double fm = frexp(mid, &em);                  /* mid = fm * 2^em */
      const unsigned __int128 Mq = (unsigned __int128)(uint64_t)ldexp(fm, 26); /* 26 bits */
      const unsigned __int128 prod = Mq * Mq * V;         /* mid^2 * v = prod * 2^e2 */
      const int e2 = 2 * (em - 26) + ve;
      /* compare prod * 2^e2 with 1 */
      int cmp;
      if (e2 >= 0) cmp = 1;                               /* prod >= 1, so > 1 unless prod==1 && e2==0 */
      else if (-e2 >= 127) cmp = -1;
      else {
        const unsigned __int128 one = (unsigned __int128)1 << (-e2);
        cmp = prod > one ? 1 : (prod < one ? -1 : 0);
      }
      if (e2 == 0 && prod == 1) cmp = 0;
      if (side == 1 && cmp <= 0) { y = up; moved = 1; break; }    /* 1/sqrt(v) >= hi_mid */
      if (side == 0 && cmp >= 0) { y = dn; moved = 1; break; }    /* 1/sqrt(v) <= lo_mid */
    }
    if (!moved) break;
  }
  return y;
}

/* The kernel's thread layout for a row of `width` values: 16-value blocks, T threads,
 * each holding NP pairs of blocks (tid + (2p) T, tid + (2p + 1) T). */
static void row_team(int64_t width, int* T, int* NP) {
  const int64_t blocks = width / 16;
  int t = (int)((blocks + 1) / 2 < 512 ? (blocks + 1) / 2 : 512);
  t = (t + 31) / 32 * 32;
  if (t < 32) t = 32;
  *T = t;
  *NP = (int)((blocks + 2 * t - 1) / (2 * t));
}

/* Sum of squares in the kernel's order: per thread, per pair p, the two blocks' squares
 * summed separately over i = 0..15, then (lane 0 + lane 1), pairs accumulated in
 * order; per warp an xor butterfly (offsets 16, 8, 4, 2, 1); warps summed in order. */
static float sum_squares(const uint16_t* x, int64_t width) {
  int T, NP;
  row_team(width, &T, &NP);
  const int64_t blocks = width / 16;
  float tsum[512];
  for (int tid = 0; tid < T; ++tid) {
    float t = 0.0f;
    for (int p = 0; p < NP; ++p) {
      float s[2] = {0.0f, 0.0f};
      for (int e = 0; e < 2; ++e) {
        const int64_t blk = tid + (int64_t)(2 * p + e) * T;
        for (int i = 0; i < 16; ++i) {
          const float v = blk < blocks ? h3o_half_to_float(x[blk * 16 + i]) : 0.0f;
          const float sq = v * v;
          s[e] = i == 0 ? sq : s[e] + sq;
        }
      }
      const float tp = s[0] + s[1];
      t = p == 0 ? tp : t + tp;
    }
    tsum[tid] = t;
  }
  float total = 0.0f;
  for (int w = 0; w < T / 32; ++w) {
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = tsum[32 * w + l];
    for (int o = 16; o > 0; o >>= 1) {
      float n[32];
      for (int l = 0; l < 32; ++l) n[l] = v[l] + v[l ^ o];
      memcpy(v, n, sizeof(v));
    }
    total = total + v[0];
  }
  return total;
}

EXPORT void h3o_modulated_norm(const uint16_t* x, int64_t rows, int64_t width, const float* W,
                               float eps, const float* shift, const float* scale,
                               const int32_t* labels, uint16_t* h) {
  const float inv_width = (float)(1.0 / (double)width);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * width;
    const float mean = sum_squares(xr, width) * inv_width;
    const float inv = rsqrt_rn(mean + eps);
    const int64_t l = labels ? labels[r] : 0;
    for (int64_t i = 0; i < width; ++i) {
      const float value = h3o_half_to_float(xr[i]) * inv;
      const float gain = value * W[i];
      const float factor = 1.0f + scale[l * width + i];
      const float scaled = gain * factor;
      h[r * width + i] = h3o_float_to_half(scaled + shift[l * width + i]);
    }
  }
}

EXPORT float h3o_rsqrt_rn(float v) { return rsqrt_rn(v); }

/* shift_for of tilelang_transport_tradeoffs.py:20-22 on the full reduction length. */
EXPORT int h3o_transport_shift(int64_t full_k) {
  if (full_k <= 0) return 0;
  const double v = (double)full_k * 127.0 * 127.0 / 60000.0;
  const int s = (int)ceil(log2(v));
  return s > 0 ? s : 0;
}
