// Activation producers of the INT8 linear path: FP32 SwiGLU, regular ConvRot256
// rotation, row maxima and per-row INT8 quantisation.
//
// All of these are HBM-bound: one read of the activation, one write of the codes
// (plus, for the two-pass TP>1 form, one more read).  A CTA owns a whole row, so the
// row maximum that the quantiser needs is a CTA reduction, and at TP=1 the row is
// rotated, reduced and quantised from registers in a single pass.
//
// Thread layout: a row of `width` values is split into 16-value blocks; 16 lanes
// (a half warp) own the 16 blocks of one 256-value ConvRot group.  Each lane loads
// its block with 128-bit loads, the group is rotated by convrot256_halfwarp, and
// each lane stores its 16 results with 128-bit stores.

#include "h3_common.cuh"

namespace h3 {

enum ProducerMode { MODE_MAX = 0, MODE_QUANT = 1, MODE_LOCAL = 2 };

struct RowTeam {
  int threads;  // CTA size, multiple of 32
  int nb;       // 16-value blocks per thread
};

static RowTeam row_team(int64_t width) {
  const int64_t blocks = width / 16;
  int threads = (int)std::min<int64_t>(blocks, 512);
  threads = std::max(32, (threads + 31) / 32 * 32);
  int nb = (int)((blocks + threads - 1) / threads);
  return {threads, nb};
}

// Load the 16 activation values of block `blk` in row `row` (before rotation).
template <int KIND>
H3_DEV void load_activation(const void* x, int64_t row, int64_t width, int64_t blk,
                            float (&v)[16]) {
  const int64_t e = blk * 16;
  if (KIND == H3_IN_GATEUP_F16) {
    const __half* xr = reinterpret_cast<const __half*>(x) + row * 2 * width;
    float g[16], u[16];
    load_half16_as_float(xr + e, g);
    load_half16_as_float(xr + width + e, u);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = swiglu_f32(g[j], u[j]);
  } else if (KIND == H3_IN_ACT_F32) {
    load_float16(reinterpret_cast<const float*>(x) + row * width + e, v);
  } else {
    load_half16_as_float(reinterpret_cast<const __half*>(x) + row * width + e, v);
  }
}

H3_DEV float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

// FC2 producer.  One CTA per row (grid-stride over rows).
template <int KIND, int MODE, int NB>
__global__ void __launch_bounds__(512) swiglu_rotate_kernel(
    const void* __restrict__ x, int64_t rows, int64_t width, float* __restrict__ rotated,
    float* __restrict__ row_max, const float* __restrict__ row_max_in, int division,
    int8_t* __restrict__ q, float* __restrict__ scale_out) {
  extern __shared__ float smem[];
  const int tid = threadIdx.x;
  const int half = tid >> 4, b = tid & 15;
  float* tile = smem + half * (16 * 17);
  float* red = smem + (blockDim.x / 16) * (16 * 17);
  const int64_t blocks = width / 16;

  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[NB][16];
    float local_max = 0.0f;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const int64_t blk = tid + (int64_t)j * blockDim.x;
      const bool valid = blk < blocks;  // uniform across each half warp
      if (valid) {
        load_activation<KIND>(x, row, width, blk, v[j]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[j][i] = 0.0f;
      }
      convrot256_halfwarp(v[j], tile, b);
      if (valid) {
#pragma unroll
        for (int i = 0; i < 16; ++i) local_max = fmaxf(local_max, fabsf(v[j][i]));
        if (MODE == MODE_MAX && rotated != nullptr)
          store_float16(rotated + row * width + blk * 16, v[j]);
      }
    }
    float scale = 0.0f;
    if (MODE == MODE_MAX || MODE == MODE_LOCAL) {
      const float m = block_reduce_max(local_max, red);
      if (tid == 0) row_max[row] = m;
      scale = row_scale_from_max(m);
    } else {
      scale = row_scale_from_max(__ldg(row_max_in + row));
    }
    if (MODE == MODE_QUANT || MODE == MODE_LOCAL) {
      const float inv = __fdiv_rn(1.0f, scale);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int64_t blk = tid + (int64_t)j * blockDim.x;
        if (blk < blocks) {
          int8_t c[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) c[i] = quantize_code_mode(v[j][i], scale, inv, division);
          store_int8x16(q + row * width + blk * 16, c);
        }
      }
      if (tid == 0) scale_out[row] = scale;
    }
  }
}

// Column activation preparation (QKV / FC1 input): optional ConvRot256 with an fp16
// rounding of the rotated value, then the row quantiser.  One CTA per row.
template <int NB, bool ROTATE>
__global__ void __launch_bounds__(512) column_quantize_kernel(
    const __half* __restrict__ x, int64_t rows, int64_t k, int8_t* __restrict__ q,
    float* __restrict__ scale_out) {
  extern __shared__ float smem[];
  const int tid = threadIdx.x;
  const int half = tid >> 4, b = tid & 15;
  float* tile = smem + half * (16 * 17);
  float* red = smem + (blockDim.x / 16) * (16 * 17);
  const int64_t blocks = k / 16;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[NB][16];
    float local_max = 0.0f;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const int64_t blk = tid + (int64_t)j * blockDim.x;
      const bool valid = blk < blocks;
      if (valid) {
        load_half16_as_float(x + row * k + blk * 16, v[j]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[j][i] = 0.0f;
      }
      if (ROTATE) {
        convrot256_halfwarp(v[j], tile, b);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[j][i] = __half2float(__float2half_rn(v[j][i]));
      }
      if (valid) {
#pragma unroll
        for (int i = 0; i < 16; ++i) local_max = fmaxf(local_max, fabsf(v[j][i]));
      }
    }
    const float m = block_reduce_max(local_max, red);
    const float scale = row_scale_from_max(m);
    const float inv = __fdiv_rn(1.0f, scale);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const int64_t blk = tid + (int64_t)j * blockDim.x;
      if (blk < blocks) {
        int8_t c[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) c[i] = quantize_code_rn(v[j][i], scale, inv);
        store_int8x16(q + row * k + blk * 16, c);
      }
    }
    if (tid == 0) scale_out[row] = scale;
  }
}

// Row quantiser with an external maximum (tilelang_row_quant.py:27-46).
__global__ void row_quantize_kernel(const float* __restrict__ x, int64_t rows, int64_t width,
                                    int64_t stride, int64_t start,
                                    const float* __restrict__ row_max, int division,
                                    int8_t* __restrict__ q, float* __restrict__ scale_out) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    const float scale = row_scale_from_max(__ldg(row_max + r));
    const float inv = __fdiv_rn(1.0f, scale);
    q[i] = quantize_code_mode(__ldg(x + r * stride + start + c), scale, inv, division);
    if (c == 0) scale_out[r] = scale;
  }
}

__global__ void expf_compare_kernel(const float* __restrict__ x, int64_t n,
                                    float* __restrict__ ours, float* __restrict__ ref) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    ours[i] = h3_expf(x[i]);
    ref[i] = expf(x[i]);
  }
}

__global__ void silu_compare_kernel(const float* __restrict__ g, int64_t n,
                                    float* __restrict__ fast, float* __restrict__ ieee,
                                    float* __restrict__ cuda) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    fast[i] = silu_fast(g[i]);
    ieee[i] = silu_ieee(g[i]);
    if (cuda != nullptr) cuda[i] = __fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i])));
  }
}

__global__ void quant_compare_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                     int64_t n, int8_t* __restrict__ fast, int8_t* __restrict__ ieee) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float s = scale[i];
    fast[i] = quantize_code_rn(x[i], s, __fdiv_rn(1.0f, s));
    ieee[i] = quantize_code(x[i], s, H3_DIV_RN);
  }
}

// ---------------------------------------------------------------------------
// Launch helpers
// ---------------------------------------------------------------------------
template <int KIND, int MODE>
static int launch_producer(const void* x, int64_t rows, int64_t width, float* rotated,
                           float* row_max, const float* row_max_in, int division, int8_t* q,
                           float* scale, cudaStream_t stream) {
  const RowTeam t = row_team(width);
  const size_t smem = (size_t)(t.threads / 16) * 16 * 17 * 4 + 32 * 4;
  const int64_t grid64 = std::min<int64_t>(rows, 1 << 20);
  const int grid = (int)grid64;
#define H3_LAUNCH_NB(NBV)                                                                  \
  swiglu_rotate_kernel<KIND, MODE, NBV><<<grid, t.threads, smem, stream>>>(               \
      x, rows, width, rotated, row_max, row_max_in, division, q, scale)
  switch (t.nb) {
    case 1: H3_LAUNCH_NB(1); break;
    case 2: H3_LAUNCH_NB(2); break;
    case 3: case 4: H3_LAUNCH_NB(4); break;
    default: return H3_ERR_INVALID;
  }
#undef H3_LAUNCH_NB
  return h3host::check_launch();
}

template <int MODE>
static int dispatch_kind(int kind, const void* x, int64_t rows, int64_t width, float* rotated,
                         float* row_max, const float* row_max_in, int division, int8_t* q,
                         float* scale, cudaStream_t stream) {
  switch (kind) {
    case H3_IN_GATEUP_F16:
      return launch_producer<H3_IN_GATEUP_F16, MODE>(x, rows, width, rotated, row_max,
                                                     row_max_in, division, q, scale, stream);
    case H3_IN_ACT_F32:
      return launch_producer<H3_IN_ACT_F32, MODE>(x, rows, width, rotated, row_max,
                                                  row_max_in, division, q, scale, stream);
    case H3_IN_ACT_F16:
      return launch_producer<H3_IN_ACT_F16, MODE>(x, rows, width, rotated, row_max,
                                                  row_max_in, division, q, scale, stream);
    default:
      return H3_ERR_INVALID;
  }
}

static bool producer_geometry_ok(const void* x, int kind, int64_t rows, int64_t width) {
  if (x == nullptr || rows < 0 || width <= 0 || width % 256 != 0) return false;
  if (width > 4 * 512 * 16) return false;  // up to 32768 values per row
  if (kind < H3_IN_GATEUP_F16 || kind > H3_IN_ACT_F16) return false;
  return h3host::aligned(x, 16);
}

}  // namespace h3

using namespace h3;

extern "C" int h3_swiglu_rotate_max(const void* x, int input_kind, int64_t rows,
                                    int64_t width, float* rotated, float* row_max,
                                    void* stream) {
  if (!producer_geometry_ok(x, input_kind, rows, width) || row_max == nullptr)
    return H3_ERR_INVALID;
  if (rotated != nullptr && !h3host::aligned(rotated, 16)) return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(x, &dev)) return s;
  return dispatch_kind<MODE_MAX>(input_kind, x, rows, width, rotated, row_max, nullptr, 0,
                                 nullptr, nullptr, (cudaStream_t)stream);
}

extern "C" int h3_swiglu_rotate_quantize(const void* x, int input_kind, int64_t rows,
                                         int64_t width, const float* row_max, int division,
                                         int8_t* q, float* scale, void* stream) {
  if (!producer_geometry_ok(x, input_kind, rows, width) || row_max == nullptr ||
      q == nullptr || scale == nullptr || !h3host::aligned(q, 16) ||
      (division != H3_DIV_RN && division != H3_DIV_FAST))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(x, &dev)) return s;
  return dispatch_kind<MODE_QUANT>(input_kind, x, rows, width, nullptr, nullptr, row_max,
                                   division, q, scale, (cudaStream_t)stream);
}

extern "C" int h3_swiglu_rotate_quantize_local(const void* x, int input_kind, int64_t rows,
                                               int64_t width, int division, int8_t* q,
                                               float* scale, float* row_max, void* stream) {
  if (!producer_geometry_ok(x, input_kind, rows, width) || row_max == nullptr ||
      q == nullptr || scale == nullptr || !h3host::aligned(q, 16) ||
      (division != H3_DIV_RN && division != H3_DIV_FAST))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(x, &dev)) return s;
  return dispatch_kind<MODE_LOCAL>(input_kind, x, rows, width, nullptr, row_max, nullptr,
                                   division, q, scale, (cudaStream_t)stream);
}

extern "C" int h3_column_quantize(const void* x_f16, int64_t rows, int64_t k, int convrot,
                                  int8_t* q, float* scale, void* stream) {
  if (x_f16 == nullptr || q == nullptr || scale == nullptr || rows < 0 || k <= 0)
    return H3_ERR_INVALID;
  if (convrot ? (k % 256 != 0) : (k % 16 != 0)) return H3_ERR_INVALID;
  if (k > 4 * 512 * 16) return H3_ERR_INVALID;
  if (!h3host::aligned(x_f16, 16) || !h3host::aligned(q, 16)) return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(x_f16, &dev)) return s;
  const RowTeam t = row_team(k);
  const size_t smem = (size_t)(t.threads / 16) * 16 * 17 * 4 + 32 * 4;
  const int grid = (int)std::min<int64_t>(rows, 1 << 20);
  cudaStream_t st = (cudaStream_t)stream;
  const __half* xh = reinterpret_cast<const __half*>(x_f16);
#define H3_COLQ(NBV, ROT) \
  column_quantize_kernel<NBV, ROT><<<grid, t.threads, smem, st>>>(xh, rows, k, q, scale)
  if (convrot) {
    switch (t.nb) {
      case 1: H3_COLQ(1, true); break;
      case 2: H3_COLQ(2, true); break;
      case 3: case 4: H3_COLQ(4, true); break;
      default: return H3_ERR_INVALID;
    }
  } else {
    switch (t.nb) {
      case 1: H3_COLQ(1, false); break;
      case 2: H3_COLQ(2, false); break;
      case 3: case 4: H3_COLQ(4, false); break;
      default: return H3_ERR_INVALID;
    }
  }
#undef H3_COLQ
  return h3host::check_launch();
}

extern "C" int h3_row_quantize(const float* rotated, int64_t rows, int64_t width,
                               int64_t stride, int64_t start, const float* row_max,
                               int division, int8_t* q, float* scale, void* stream) {
  if (rotated == nullptr || row_max == nullptr || q == nullptr || scale == nullptr ||
      rows < 0 || width <= 0 || start < 0 || start + width > stride ||
      (division != H3_DIV_RN && division != H3_DIV_FAST))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(rotated, &dev)) return s;
  const int64_t total = rows * width;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)h3host::sm_count(dev) * 16);
  row_quantize_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(rotated, rows, width, stride,
                                                             start, row_max, division, q, scale);
  return h3host::check_launch();
}

extern "C" int h3_expf_compare(const float* x, int64_t n, float* ours, float* cuda,
                               void* stream) {
  if (x == nullptr || ours == nullptr || cuda == nullptr || n < 0) return H3_ERR_INVALID;
  if (n == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(x, &dev)) return s;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 4096);
  expf_compare_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, n, ours, cuda);
  return h3host::check_launch();
}

extern "C" int h3_silu_compare(const float* g, int64_t n, float* fast, float* ieee,
                               float* cuda, void* stream) {
  if (g == nullptr || fast == nullptr || ieee == nullptr || n < 0) return H3_ERR_INVALID;
  if (n == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(g, &dev)) return s;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 4096);
  silu_compare_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(g, n, fast, ieee, cuda);
  return h3host::check_launch();
}

extern "C" int h3_quant_compare(const float* x, const float* scale, int64_t n, int8_t* fast,
                                int8_t* ieee, void* stream) {
  if (x == nullptr || scale == nullptr || fast == nullptr || ieee == nullptr || n < 0)
    return H3_ERR_INVALID;
  if (n == 0) return H3_OK;
  int dev;
  if (int s = h3host::bind_device_of(x, &dev)) return s;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)h3host::sm_count(dev) * 16);
  quant_compare_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, scale, n, fast, ieee);
  return h3host::check_launch();
}
