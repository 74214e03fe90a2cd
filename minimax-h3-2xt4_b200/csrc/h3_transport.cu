// Row-parallel transport and epilogue kernels: the scaled-FP16 codec, the
// fixed-order partial reduction fused with decode + dequant (+ gated residual), and
// the standalone column / INT32 dequant epilogues.  All HBM-bound elementwise work,
// 8 columns (16 bytes of fp16) per thread.

#include "h3_common.cuh"

namespace h3 {

// ---------------------------------------------------------------------------
// Scaled-FP16 codec (tilelang_transport_tradeoffs.py:26-39)
// ---------------------------------------------------------------------------
__global__ void fp16_encode_kernel(const int32_t* __restrict__ p, int64_t n, float factor,
                                   __half* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(__fmul_rn(__int2float_rn(__ldg(p + i)), factor));
}

__global__ void fp16_decode_kernel(const __half* __restrict__ y, int64_t n, float factor,
                                   int32_t* __restrict__ p) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = __float2int_rz(__fmul_rn(__half2float(y[i]), factor));
}

// ---------------------------------------------------------------------------
// Fixed-order reduction of `world` fp16 partials + decode + dequant + store.
// ---------------------------------------------------------------------------
template <int VEC>
__global__ void row_reduce_finish_kernel(const __half* __restrict__ parts, int world,
                                         int64_t part_stride, int64_t rows, int64_t width,
                                         float up_factor, const float* __restrict__ row_scale,
                                         const float* __restrict__ weight_scale, RowOut o) {
  const int64_t chunks = width / VEC;
  const int64_t total = rows * chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / chunks;
    const int64_t c0 = (i - r * chunks) * VEC;
    const int64_t base = r * width + c0;
    float t[VEC];
    if (VEC == 8) {
      for (int w = 0; w < world; ++w) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(parts + w * part_stride + base));
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h[j]);
          if (w == 0) {
            t[2 * j] = f.x; t[2 * j + 1] = f.y;
          } else {
            t[2 * j] = __fadd_rn(t[2 * j], f.x);
            t[2 * j + 1] = __fadd_rn(t[2 * j + 1], f.y);
          }
        }
      }
    } else {
      for (int w = 0; w < world; ++w) {
        const float f = __half2float(parts[w * part_stride + base]);
        t[0] = (w == 0) ? f : __fadd_rn(t[0], f);
      }
    }
    const float a = __ldg(row_scale + r);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float reduced = __half2float(__float2half_rn(t[j]));
      const int32_t restored = __float2int_rz(__fmul_rn(reduced, up_factor));
      const float value = __fmul_rn(__int2float_rn(restored), a);
      const float y = __fmul_rn(value, __ldg(weight_scale + c0 + j));
      row_store(o, r, c0 + j, width, y);
    }
  }
}

// ---------------------------------------------------------------------------
// Standalone ordered column epilogue (tilelang_column_epilogue.py:11-27)
// ---------------------------------------------------------------------------
__global__ void column_dequantize_kernel(const int32_t* __restrict__ acc, int64_t rows,
                                         int64_t width, const float* __restrict__ row_scale,
                                         const float* __restrict__ weight_scale, int scalar,
                                         __half* __restrict__ y) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    const float s = __fmul_rn(__ldg(row_scale + r), __ldg(weight_scale + (scalar ? 0 : c)));
    y[i] = __float2half_rn(__fmul_rn(__int2float_rn(__ldg(acc + i)), s));
  }
}

// parallel_int8.dequantize CPU order: ((acc * a) * w) + bias
__global__ void dequantize_i32_kernel(const int32_t* __restrict__ acc, int64_t rows,
                                      int64_t width, const float* __restrict__ row_scale,
                                      const float* __restrict__ weight_scale, int scalar,
                                      const float* __restrict__ bias, int out_kind,
                                      void* __restrict__ out) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    float v = __fmul_rn(__int2float_rn(__ldg(acc + i)), __ldg(row_scale + r));
    v = __fmul_rn(v, __ldg(weight_scale + (scalar ? 0 : c)));
    if (bias != nullptr) v = __fadd_rn(v, __ldg(bias + c));
    if (out_kind == H3_OUT_F32)
      reinterpret_cast<float*>(out)[i] = v;
    else
      reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
  }
}

// gate_kernel of tilelang_dit_fusion.py:39-53 with an fp32 or fp16 branch.
__global__ void gated_add_kernel(const void* __restrict__ branch, int branch_kind, int64_t rows,
                                 int64_t width, RowOut o) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    const float y = branch_kind == H3_OUT_F32 ? reinterpret_cast<const float*>(branch)[i]
                                              : __half2float(reinterpret_cast<const __half*>(branch)[i]);
    row_store(o, r, c, width, y);
  }
}

// ---------------------------------------------------------------------------
// Packed INT8 transport ('int8_gather', tilelang_transport_tradeoffs.py:40-62 and
// tilelang_transport_p2.py:28-42).  Wire format per row: for each 128-column group,
// 128 code bytes then the 4 bytes of the fp32 scale; row pitch groups * 132 bytes.
// ---------------------------------------------------------------------------
// One warp per (row, group): lane l owns columns 4l..4l+3.
__global__ void pack8_kernel(const int32_t* __restrict__ p, int64_t rows, int64_t width,
                             uint8_t* __restrict__ out) {
  const int64_t groups = width / 128, pitch = groups * 132;
  const int lane = threadIdx.x & 31;
  const int64_t total = rows * groups;
  for (int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; t < total;
       t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t r = t / groups, g = t - r * groups;
    const int4 v = __ldg(reinterpret_cast<const int4*>(p + r * width + g * 128) + lane);
    const float x[4] = {__int2float_rn(v.x), __int2float_rn(v.y), __int2float_rn(v.z),
                        __int2float_rn(v.w)};
    float m = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    m = warp_max(m);
    const float scale = fmaxf(__fmul_rn(m, f32_bits(H3_INV127_BITS)), f32_bits(0x322bcc77u));
    const float inv = __fdiv_rn(1.0f, scale);
    uint32_t b[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float q = fminf(127.0f, fmaxf(-127.0f, div_by_scale(x[e], scale, inv)));
      b[e] = __float_as_uint(__fadd_rn(q, 12582912.0f));
    }
    uint8_t* o = out + r * pitch + g * 132;
    reinterpret_cast<uint32_t*>(o)[lane] =
        __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
    if (lane == 0) *reinterpret_cast<float*>(o + 128) = scale;
  }
}

// restored = rint(sum_w f32(q_w) *rn s_w) in rank order, then the row epilogue; 4 columns
// (one 32-bit word of codes per rank) per thread.
__global__ void unpack8_finish_kernel(const uint8_t* __restrict__ parts, int world,
                                      int64_t part_stride, int64_t rows, int64_t width,
                                      const float* __restrict__ row_scale,
                                      const float* __restrict__ weight_scale, RowOut o) {
  const int64_t groups = width / 128, pitch = groups * 132;
  const int64_t quads = width / 4;
  const int64_t total = rows * quads;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / quads;
    const int64_t c0 = (i - r * quads) * 4;
    const int64_t g = c0 / 128, off = r * pitch + g * 132;
    float t[4];
    for (int w = 0; w < world; ++w) {
      const uint8_t* b = parts + w * part_stride + off;
      const float s = __ldg(reinterpret_cast<const float*>(b + 128));
      const uint32_t q = __ldg(reinterpret_cast<const uint32_t*>(b + (c0 - g * 128)));
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x = __fmul_rn((float)(int8_t)(q >> (8 * e)), s);
        t[e] = w == 0 ? x : __fadd_rn(t[e], x);
      }
    }
    if (o.kind == H3_OUT_I32) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        reinterpret_cast<int32_t*>(o.out)[r * width + c0 + e] = __float2int_rn(t[e]);
      continue;
    }
    const float a = __ldg(row_scale + r);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int32_t restored = __float2int_rn(t[e]);
      row_store(o, r, c0 + e, width,
                __fmul_rn(__fmul_rn(__int2float_rn(restored), a), __ldg(weight_scale + c0 + e)));
    }
  }
}

static int elementwise_grid(int64_t total, int dev) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256,
                                                     (int64_t)h3host::sm_count(dev) * 32));
}

}  // namespace h3

using namespace h3;

extern "C" int h3_transport_shift(int64_t full_k) {
  if (full_k <= 0) return 0;
  // smallest s >= 0 with full_k * 127^2 / 60000 <= 2^s, in exact integer arithmetic
  const int64_t num = full_k * 127 * 127;
  int s = 0;
  while ((int64_t)60000 << s < num) ++s;
  return s;
}

extern "C" int h3_fp16_encode(const int32_t* partial, int64_t n, int shift, void* out_f16,
                              void* stream) {
  if (partial == nullptr || out_f16 == nullptr || n < 0 || shift < 0 || shift > 60)
    return H3_ERR_INVALID;
  if (n == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(partial, &dev)) return s;
  const float factor = ldexpf(1.0f, -shift);
  fp16_encode_kernel<<<elementwise_grid(n, dev), 256, 0, (cudaStream_t)stream>>>(
      partial, n, factor, reinterpret_cast<__half*>(out_f16));
  return h3host::check_launch();
}

extern "C" int h3_fp16_decode(const void* payload_f16, int64_t n, int shift, int32_t* out,
                              void* stream) {
  if (payload_f16 == nullptr || out == nullptr || n < 0 || shift < 0 || shift > 60)
    return H3_ERR_INVALID;
  if (n == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(payload_f16, &dev)) return s;
  const float factor = ldexpf(1.0f, shift);
  fp16_decode_kernel<<<elementwise_grid(n, dev), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __half*>(payload_f16), n, factor, out);
  return h3host::check_launch();
}

extern "C" int h3_row_reduce_finish(const void* parts_f16, int world, int64_t part_stride,
                                    int64_t rows, int64_t width, int shift,
                                    const float* row_scale, const float* weight_scale,
                                    int out_kind, void* out, void* residual_f16,
                                    const float* gate, int64_t gate_rows,
                                    const int32_t* labels, void* stream) {
  if (parts_f16 == nullptr || row_scale == nullptr || weight_scale == nullptr || world < 1 ||
      world > 64 || rows < 0 || width <= 0 || shift < 0 || shift > 60)
    return H3_ERR_INVALID;
  if (world > 1 && part_stride < rows * width) return H3_ERR_INVALID;
  if (out_kind == H3_OUT_RESIDUAL) {
    if (residual_f16 == nullptr) return H3_ERR_INVALID;
    if (gate != nullptr && (gate_rows < 1 || (labels == nullptr && gate_rows != 1)))
      return H3_ERR_INVALID;
  } else if (out_kind == H3_OUT_F32 || out_kind == H3_OUT_F16) {
    if (out == nullptr) return H3_ERR_INVALID;
  } else {
    return H3_ERR_INVALID;
  }
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(parts_f16, &dev)) return s;
  RowOut o{out_kind, out, reinterpret_cast<__half*>(residual_f16), gate, gate_rows, labels,
           h3host::error_word(dev)};
  if (o.err == nullptr) return H3_ERR_CUDA;
  const float up = ldexpf(1.0f, shift);
  const __half* parts = reinterpret_cast<const __half*>(parts_f16);
  const bool vec = width % 8 == 0 && h3host::aligned(parts_f16, 16) && part_stride % 8 == 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (vec) {
    row_reduce_finish_kernel<8><<<elementwise_grid(rows * width / 8, dev), 256, 0, st>>>(
        parts, world, part_stride, rows, width, up, row_scale, weight_scale, o);
  } else {
    row_reduce_finish_kernel<1><<<elementwise_grid(rows * width, dev), 256, 0, st>>>(
        parts, world, part_stride, rows, width, up, row_scale, weight_scale, o);
  }
  return h3host::check_launch();
}

extern "C" int h3_column_dequantize(const int32_t* acc, int64_t rows, int64_t width,
                                    const float* row_scale, const float* weight_scale,
                                    int64_t weight_scale_len, void* out_f16, void* stream) {
  if (acc == nullptr || row_scale == nullptr || weight_scale == nullptr ||
      out_f16 == nullptr || rows < 0 || width <= 0 ||
      (weight_scale_len != 1 && weight_scale_len != width))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(acc, &dev)) return s;
  column_dequantize_kernel<<<elementwise_grid(rows * width, dev), 256, 0,
                             (cudaStream_t)stream>>>(acc, rows, width, row_scale, weight_scale,
                                                     weight_scale_len == 1,
                                                     reinterpret_cast<__half*>(out_f16));
  return h3host::check_launch();
}

extern "C" int h3_dequantize_i32(const int32_t* acc, int64_t rows, int64_t width,
                                 const float* row_scale, const float* weight_scale,
                                 int64_t weight_scale_len, const float* bias, int out_kind,
                                 void* out, void* stream) {
  if (acc == nullptr || row_scale == nullptr || weight_scale == nullptr || out == nullptr ||
      rows < 0 || width <= 0 || (weight_scale_len != 1 && weight_scale_len != width) ||
      (out_kind != H3_OUT_F32 && out_kind != H3_OUT_F16))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(acc, &dev)) return s;
  dequantize_i32_kernel<<<elementwise_grid(rows * width, dev), 256, 0, (cudaStream_t)stream>>>(
      acc, rows, width, row_scale, weight_scale, weight_scale_len == 1, bias, out_kind, out);
  return h3host::check_launch();
}

extern "C" int h3_gated_add(const void* branch, int branch_kind, int64_t rows, int64_t width,
                            void* residual_f16, const float* gate, int64_t gate_rows,
                            const int32_t* labels, void* stream) {
  if (branch == nullptr || residual_f16 == nullptr || rows < 0 || width <= 0 ||
      (branch_kind != H3_OUT_F32 && branch_kind != H3_OUT_F16))
    return H3_ERR_INVALID;
  if (gate != nullptr && (gate_rows < 1 || (labels == nullptr && gate_rows != 1)))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(branch, &dev)) return s;
  RowOut o{H3_OUT_RESIDUAL, nullptr, reinterpret_cast<__half*>(residual_f16), gate, gate_rows,
           labels, h3host::error_word(dev)};
  if (o.err == nullptr) return H3_ERR_CUDA;
  gated_add_kernel<<<elementwise_grid(rows * width, dev), 256, 0, (cudaStream_t)stream>>>(
      branch, branch_kind, rows, width, o);
  return h3host::check_launch();
}

extern "C" int h3_pack8(const int32_t* partial, int64_t rows, int64_t width, void* out_u8,
                        void* stream) {
  if (partial == nullptr || out_u8 == nullptr || rows < 0 || width <= 0 || width % 128 != 0 ||
      !h3host::aligned(partial, 16) || !h3host::aligned(out_u8, 4))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(partial, &dev)) return s;
  pack8_kernel<<<elementwise_grid(rows * (width / 128) * 32, dev), 256, 0, (cudaStream_t)stream>>>(
      partial, rows, width, reinterpret_cast<uint8_t*>(out_u8));
  return h3host::check_launch();
}

extern "C" int h3_unpack8_finish(const void* parts_u8, int world, int64_t part_stride,
                                 int64_t rows, int64_t width, const float* row_scale,
                                 const float* weight_scale, int out_kind, void* out,
                                 void* residual_f16, const float* gate, int64_t gate_rows,
                                 const int32_t* labels, void* stream) {
  if (parts_u8 == nullptr || world < 1 || world > 64 || rows < 0 || width <= 0 ||
      width % 128 != 0 || !h3host::aligned(parts_u8, 4) || part_stride % 4 != 0)
    return H3_ERR_INVALID;
  if (world > 1 && part_stride < rows * (width / 128) * 132) return H3_ERR_INVALID;
  if (out_kind != H3_OUT_I32 && (row_scale == nullptr || weight_scale == nullptr))
    return H3_ERR_INVALID;
  if (out_kind == H3_OUT_I32) {
    if (out == nullptr || !h3host::aligned(out, 4)) return H3_ERR_INVALID;
  } else if (out_kind == H3_OUT_RESIDUAL) {
    if (residual_f16 == nullptr) return H3_ERR_INVALID;
    if (gate != nullptr && (gate_rows < 1 || (labels == nullptr && gate_rows != 1)))
      return H3_ERR_INVALID;
  } else if (out_kind == H3_OUT_F32 || out_kind == H3_OUT_F16) {
    if (out == nullptr) return H3_ERR_INVALID;
  } else {
    return H3_ERR_INVALID;
  }
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(parts_u8, &dev)) return s;
  RowOut o{out_kind, out, reinterpret_cast<__half*>(residual_f16), gate, gate_rows, labels,
           h3host::error_word(dev)};
  if (o.err == nullptr) return H3_ERR_CUDA;
  unpack8_finish_kernel<<<elementwise_grid(rows * width / 4, dev), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(parts_u8), world, part_stride, rows, width, row_scale,
      weight_scale, o);
  return h3host::check_launch();
}
