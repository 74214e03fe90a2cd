// Activation producers of the INT8 linear path: FP32 SwiGLU, regular ConvRot256
// rotation, row maxima and per-row INT8 quantisation.
//
// All of these are HBM-bound: one read of the activation, one write of the codes
// (plus, for the two-pass TP>1 form, one more read).  A CTA owns a whole row, so the
// row maximum that the quantiser needs is a CTA reduction, and at TP=1 the row is
// rotated, reduced and quantised from registers in a single pass.
//
// Thread layout: a row of `width` values is split into 16-value blocks; 16 lanes
// (a half warp) own the 16 blocks of one 256-value ConvRot group, and every lane holds
// two blocks of two different groups as packed f32x2 pairs.  Each lane loads its
// blocks with 128-bit loads, the two groups are rotated together by
// convrot256_halfwarp2 (f32x2 arithmetic, per-lane IEEE rounding), and the codes are
// stored 16 bytes at a time.

#include "h3_common.cuh"

namespace h3 {

enum ProducerMode { MODE_MAX = 0, MODE_QUANT = 1, MODE_LOCAL = 2 };

// Row-maximum exchange over NVLink peer memory, for the TP>1 producer in one pass
// (it replaces the NCCL MAX all-reduce between the two passes of the reference,
// tilelang_swiglu_quant.py:86-87).  bases[w] is rank w's workspace buffer; at slots_off
// each holds u64 slots [rows][world] = (epoch << 32) | max bits.  Value and tag share
// one aligned 64-bit word, so relaxed system-scope accesses suffice: nothing else is
// ordered by a slot.
struct PeerMax {
  uint64_t bases[8];
  int64_t slots_off;
  int world, rank;
  uint32_t epoch;
  int* err;
};

constexpr unsigned long long PEER_TIMEOUT_NS = 2000000000ull;

// This rank's maximum of `row` into slot [row][rank] of every rank (threads < world).
H3_DEV void peer_publish(const PeerMax& pm, int64_t row, float m) {
  const int tid = threadIdx.x;
  if (tid < pm.world) {
    const unsigned long long v = ((unsigned long long)pm.epoch << 32) | __float_as_uint(m);
    unsigned long long* slot =
        reinterpret_cast<unsigned long long*>(pm.bases[tid] + pm.slots_off) + row * pm.world +
        pm.rank;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(slot), "l"(v) : "memory");
  }
}

// Maximum over ranks of `row`, read from this rank's slots (called by every thread).
// `deadline` bounds the waiting of the whole CTA: it is set at the first slot that is
// not ready; once it has passed, every later wait gives up after one look, the rank's
// own maximum `m` stands in for the missing ones and H3_ERR_TIMEOUT is recorded.  A
// slot is rewritten with the next epoch only after every rank has finished this
// launch, since the row reduce that follows it waits for all ranks.
H3_DEV float peer_wait(const PeerMax& pm, int64_t row, float m, float* red,
                       uint64_t& deadline) {
  const int tid = threadIdx.x;
  if (tid < pm.world) {
    const unsigned long long* mine =
        reinterpret_cast<const unsigned long long*>(pm.bases[pm.rank] + pm.slots_off) +
        row * pm.world + tid;
    float got = m;
    while (true) {
      unsigned long long w;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(mine) : "memory");
      if ((uint32_t)(w >> 32) == pm.epoch) {
        got = __uint_as_float((uint32_t)w);
        break;
      }
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (deadline == 0) deadline = now + PEER_TIMEOUT_NS;
      if (now > deadline) {
        report_error(pm.err, H3_ERR_TIMEOUT);
        break;
      }
      __nanosleep(32);
    }
    red[tid] = got;
  }
  __syncthreads();
  float g = red[0];
  for (int w = 1; w < pm.world; ++w) g = fmaxf(g, red[w]);
  __syncthreads();
  return g;
}

struct RowTeam {
  int threads;  // CTA size, multiple of 32
  int nb;       // packed pairs of 16-value blocks per thread
};

// Pairs of 16-value blocks per thread (nb = pairs) and CTA size for a row of `width`.
static RowTeam row_team(int64_t width) {
  const int64_t blocks = width / 16;
  int threads = (int)std::min<int64_t>((blocks + 1) / 2, 512);
  threads = std::max(32, (threads + 31) / 32 * 32);
  int pairs = (int)((blocks + 2 * threads - 1) / (2 * threads));
  return {threads, pairs};
}

// Dynamic shared memory of a producer CTA: one 16 x 17 tile of pairs per half warp and
// the 32-float reduction buffer.
__host__ __device__ inline size_t producer_smem(int threads) {
  return (size_t)(threads / 16) * 16 * 17 * sizeof(unsigned long long) + 32 * sizeof(float);
}

// Activation values of blocks blk0 (lane 0) and blk1 (lane 1) of row `row`, before
// rotation; a block that is not valid reads as zeros.
template <int KIND>
H3_DEV void load_activation2(const void* x, int64_t row, int64_t width, int64_t blk0,
                             int64_t blk1, bool ok0, bool ok1, f32x2 (&p)[16]) {
  float a[16], b[16];
  if (KIND == H3_IN_GATEUP_F16) {
    const __half* xr = reinterpret_cast<const __half*>(x) + row * 2 * width;
    float g0[16], g1[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) g0[j] = g1[j] = a[j] = b[j] = 0.0f;
    if (ok0) {
      load_half16_as_float(xr + blk0 * 16, g0);
      load_half16_as_float(xr + width + blk0 * 16, a);
    }
    if (ok1) {
      load_half16_as_float(xr + blk1 * 16, g1);
      load_half16_as_float(xr + width + blk1 * 16, b);
    }
    // two (gate, up) pairs on packed lanes: the same bits as swiglu_f32 of each
#pragma unroll
    for (int j = 0; j < 16; ++j) p[j] = swiglu_f32x2(g0[j], g1[j], a[j], b[j]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) a[j] = b[j] = 0.0f;
  if (KIND == H3_IN_ACT_F32) {
    if (ok0) load_float16(reinterpret_cast<const float*>(x) + row * width + blk0 * 16, a);
    if (ok1) load_float16(reinterpret_cast<const float*>(x) + row * width + blk1 * 16, b);
  } else {
    if (ok0) load_half16_as_float(reinterpret_cast<const __half*>(x) + row * width + blk0 * 16, a);
    if (ok1) load_half16_as_float(reinterpret_cast<const __half*>(x) + row * width + blk1 * 16, b);
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) p[j] = pk2(a[j], b[j]);
}

// L2 prefetch of this thread's blocks of row `row` (the CTA's next row): the loads that
// follow one iteration later then find the row in L2, with no register held meanwhile.
template <int KIND>
H3_DEV void prefetch_activation2(const void* x, int64_t row, int64_t width, int64_t blk0,
                                 int64_t blk1, bool ok0, bool ok1) {
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    if (!(e == 0 ? ok0 : ok1)) continue;
    const int64_t blk = e == 0 ? blk0 : blk1;
    const char* p;
    if (KIND == H3_IN_ACT_F32)
      p = reinterpret_cast<const char*>(reinterpret_cast<const float*>(x) + row * width + blk * 16);
    else if (KIND == H3_IN_ACT_F16)
      p = reinterpret_cast<const char*>(reinterpret_cast<const __half*>(x) + row * width + blk * 16);
    else
      p = reinterpret_cast<const char*>(reinterpret_cast<const __half*>(x) + row * 2 * width + blk * 16);
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    if (KIND == H3_IN_GATEUP_F16)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + width * 2));
  }
}

// ---------------------------------------------------------------------------
// Row staging (the persistent producers).  A CTA keeps ROW_STAGES rows of its input in
// flight: each row is copied global -> shared memory by TMA (cp.async.bulk.tensor,
// boxes of 128-byte lines with the 128-byte swizzle, completing on the stage's
// mbarrier) while the CTA rotates and quantises an earlier row.  With the swizzle,
// 16-byte chunk c of line l sits at chunk position c ^ (l & 7) of the line, so the
// 16-byte reads of the lanes' 32- or 64-byte blocks fall on eight different bank
// groups in every quarter warp.  The copies read this GPU's own memory (no multicast).
// ---------------------------------------------------------------------------
constexpr int ROW_STAGES = 2;
constexpr unsigned long long STAGE_TIMEOUT_NS = 2000000000ull;

struct RowStage {
  int row_bytes;    // bytes of one input row (a multiple of 128)
  int stage_bytes;  // row_bytes rounded up to 1024
  int box_lines;    // 128-byte lines per TMA box (<= 256, divides row_bytes / 128)
  int boxes;        // boxes per row
  int* err;
};

H3_DEV uint32_t stage_su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Thread 0: the copy of `row` into one stage, completing on its barrier.
H3_DEV void stage_issue(const CUtensorMap* map, const RowStage& st, uint8_t* buf, uint64_t* bar,
                        int64_t row) {
  const uint32_t b = stage_su32(bar);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b),
               "r"((uint32_t)st.row_bytes)
               : "memory");
  for (int k = 0; k < st.boxes; ++k)
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(stage_su32(buf + k * st.box_lines * 128)),
        "l"(map), "r"(0), "r"(k * st.box_lines), "r"((int)row), "r"(b)
        : "memory");
}

// Bounded wait for a stage's copy (2 s of %globaltimer).
H3_DEV bool stage_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t b = stage_su32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    if (ok) return true;
    uint64_t now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (it == 0)
      t0 = now;
    else if (now - t0 > STAGE_TIMEOUT_NS)
      return false;
  }
}

// The 16-byte chunk at byte `off` of a staged (swizzled) row.
H3_DEV uint4 stage_chunk(const uint8_t* stage, int64_t off) {
  const int64_t line = off >> 7;
  const int c = (int)((off >> 4) & 7) ^ (int)(line & 7);
  return *reinterpret_cast<const uint4*>(stage + (line << 7) + (c << 4));
}

H3_DEV void stage_half16(const uint8_t* stage, int64_t off, float (&v)[16]) {
  const uint4 u[2] = {stage_chunk(stage, off), stage_chunk(stage, off + 16)};
  const __half2* h = reinterpret_cast<const __half2*>(u);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

H3_DEV void stage_float16(const uint8_t* stage, int64_t off, float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 u = stage_chunk(stage, off + 16 * j);
    v[4 * j] = __uint_as_float(u.x);
    v[4 * j + 1] = __uint_as_float(u.y);
    v[4 * j + 2] = __uint_as_float(u.z);
    v[4 * j + 3] = __uint_as_float(u.w);
  }
}

// load_activation2 from a staged row (byte offsets of the row as laid out in HBM).
template <int KIND>
H3_DEV void stage_activation2(const uint8_t* stage, int64_t width, int64_t blk0, int64_t blk1,
                              bool ok0, bool ok1, f32x2 (&p)[16]) {
  float a[16], b[16];
  if (KIND == H3_IN_GATEUP_F16) {
    float g0[16], g1[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) g0[j] = g1[j] = a[j] = b[j] = 0.0f;
    if (ok0) {
      stage_half16(stage, blk0 * 32, g0);
      stage_half16(stage, 2 * width + blk0 * 32, a);
    }
    if (ok1) {
      stage_half16(stage, blk1 * 32, g1);
      stage_half16(stage, 2 * width + blk1 * 32, b);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) p[j] = pk2(swiglu_f32(g0[j], a[j]), swiglu_f32(g1[j], b[j]));
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) a[j] = b[j] = 0.0f;
  if (KIND == H3_IN_ACT_F32) {
    if (ok0) stage_float16(stage, blk0 * 64, a);
    if (ok1) stage_float16(stage, blk1 * 64, b);
  } else {
    if (ok0) stage_half16(stage, blk0 * 32, a);
    if (ok1) stage_half16(stage, blk1 * 32, b);
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) p[j] = pk2(a[j], b[j]);
}

// Shared memory of a staged producer CTA: the 1024-aligned stages, then the rotation
// tiles and reduction buffer of producer_smem, then the stage barriers.
static size_t staged_smem(int threads, const RowStage& st) {
  return 1024 + (size_t)ROW_STAGES * st.stage_bytes + producer_smem(threads) + ROW_STAGES * 8;
}


// The staged prologue: barriers initialised and the CTA's first ROW_STAGES rows in
// flight.  Returns the stage area; *bars_out receives the barriers.
H3_DEV uint8_t* stage_begin(uint8_t* smem_raw, const CUtensorMap* map, const RowStage& st,
                            int64_t rows, uint8_t*& rest, uint64_t*& bars) {
  uint8_t* stages = smem_raw + ((1024u - (stage_su32(smem_raw) & 1023u)) & 1023u);
  rest = stages + ROW_STAGES * st.stage_bytes;
  bars = reinterpret_cast<uint64_t*>(rest + producer_smem(blockDim.x));
  if (threadIdx.x == 0) {
    for (int k = 0; k < ROW_STAGES; ++k)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(stage_su32(bars + k)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int k = 0; k < ROW_STAGES; ++k) {
      const int64_t r = blockIdx.x + (int64_t)k * gridDim.x;
      if (r < rows) stage_issue(map, st, stages + k * st.stage_bytes, bars + k, r);
    }
  }
  __syncthreads();
  return stages;
}

// Waits for the stage of loop iteration `it` (row `row`).  On a timeout (which would
// mean the copy engine failed) every thread learns it together; thread 0 records
// H3_ERR_TIMEOUT and waits, bounded, for the copies still in flight, and the caller
// returns.
H3_DEV bool stage_ready(const RowStage& st, uint64_t* bars, int it, int64_t row, int64_t rows) {
  const bool ok = stage_wait(bars + it % ROW_STAGES, (uint32_t)(it / ROW_STAGES) & 1u);
  if (!__syncthreads_or(!ok)) return true;
  if (threadIdx.x == 0) {
    report_error(st.err, H3_ERR_TIMEOUT);
    for (int k = 0; k < ROW_STAGES; ++k) {
      const int j = it + k;
      if (row + (int64_t)k * gridDim.x < rows)
        stage_wait(bars + j % ROW_STAGES, (uint32_t)(j / ROW_STAGES) & 1u);
    }
  }
  return false;
}

// After every lane has read the stage of iteration `it`: refill it with the row
// ROW_STAGES iterations ahead.
H3_DEV void stage_next(const CUtensorMap* map, const RowStage& st, uint8_t* stages,
                       uint64_t* bars, int it, int64_t row, int64_t rows) {
  __syncthreads();
  const int64_t next = row + (int64_t)ROW_STAGES * gridDim.x;
  if (threadIdx.x == 0 && next < rows)
    stage_issue(map, st, stages + (it % ROW_STAGES) * st.stage_bytes, bars + it % ROW_STAGES, next);
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

// CTA maximum with NaN propagation (a NaN anywhere gives NaN).
H3_DEV float block_reduce_max_nan(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    asm("max.NaN.f32 %0, %0, %1;" : "+f"(v) : "f"(w));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) asm("max.NaN.f32 %0, %0, %1;" : "+f"(m) : "f"(red[w]));
  __syncthreads();
  return m;
}

// Maximum of |v| over the valid values of this thread, ignoring NaN (fmaxf), as the
// reference's row maximum does; only rows that hold a NaN or an infinity need it.
template <int NP>
H3_DEV float local_max_ignoring_nan(const f32x2 (&v)[NP][16], const bool (&ok)[NP][2]) {
  float m = 0.0f;
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (ok[p][0]) m = fmaxf(m, fabsf(lo2(v[p][i])));
      if (ok[p][1]) m = fmaxf(m, fabsf(hi2(v[p][i])));
    }
  return m;
}

// Codes of the valid blocks of this thread.  finite: the row maximum (over exactly
// these values) is finite, so the packed form applies; otherwise each code goes
// through the clamped scalar quantiser.
template <int NP>
H3_DEV void quantize_store(const f32x2 (&v)[NP][16], const bool (&ok)[NP][2],
                           const int64_t (&blk)[NP][2], bool finite, float scale, float inv,
                           int division, int8_t* qrow) {
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    if (finite && division == H3_DIV_RN) {
      uint4 c0, c1;
      quantize_pairs_finite(v[p], scale, inv, c0, c1);
      if (ok[p][0]) *reinterpret_cast<uint4*>(qrow + blk[p][0] * 16) = c0;
      if (ok[p][1]) *reinterpret_cast<uint4*>(qrow + blk[p][1] * 16) = c1;
    } else {
      int8_t c0[16], c1[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        c0[i] = quantize_code_mode(lo2(v[p][i]), scale, inv, division);
        c1[i] = quantize_code_mode(hi2(v[p][i]), scale, inv, division);
      }
      if (ok[p][0]) store_int8x16(qrow + blk[p][0] * 16, c0);
      if (ok[p][1]) store_int8x16(qrow + blk[p][1] * 16, c1);
    }
  }
}

// FC2 producer.  One CTA per row (grid-stride over rows); each thread owns NB = 2 * NP
// 16-value blocks, processed as NP packed pairs of blocks that lie in different
// ConvRot groups (blocks tid + (2p) * T and tid + (2p + 1) * T for T threads).
template <int KIND, int MODE, int NP, bool STAGED>
__global__ void __launch_bounds__(512) swiglu_rotate_kernel(
    const void* __restrict__ x, int64_t rows, int64_t width, float* __restrict__ rotated,
    float* __restrict__ row_max, const float* __restrict__ row_max_in, int division,
    int8_t* __restrict__ q, float* __restrict__ scale_out, const __grid_constant__ CUtensorMap map,
    const RowStage st) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* rest = smem_raw;
  uint8_t* stages = nullptr;
  uint64_t* bars = nullptr;
  if (STAGED) stages = stage_begin(smem_raw, &map, st, rows, rest, bars);
  f32x2* smem2 = reinterpret_cast<f32x2*>(rest);
  const int tid = threadIdx.x;
  const int half = tid >> 4, b = tid & 15;
  f32x2* tile = smem2 + half * (16 * 17);
  float* red = reinterpret_cast<float*>(smem2 + (blockDim.x / 16) * (16 * 17));
  const int64_t blocks = width / 16;
  int64_t blk[NP][2];
  bool ok[NP][2];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      blk[p][e] = tid + (int64_t)(2 * p + e) * blockDim.x;
      ok[p][e] = blk[p][e] < blocks;  // uniform across each half warp
    }

  int it = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    f32x2 v[NP][16];
    if (STAGED) {
      if (!stage_ready(st, bars, it, row, rows)) return;
      const uint8_t* stg = stages + (it % ROW_STAGES) * st.stage_bytes;
#pragma unroll
      for (int p = 0; p < NP; ++p)
        stage_activation2<KIND>(stg, width, blk[p][0], blk[p][1], ok[p][0], ok[p][1], v[p]);
      stage_next(&map, st, stages, bars, it, row, rows);
    }
    if (!STAGED && row + gridDim.x < rows) {
#pragma unroll
      for (int p = 0; p < NP; ++p)
        prefetch_activation2<KIND>(x, row + gridDim.x, width, blk[p][0], blk[p][1], ok[p][0],
                                   ok[p][1]);
    }
    float m_nan = 0.0f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      if (!STAGED)
        load_activation2<KIND>(x, row, width, blk[p][0], blk[p][1], ok[p][0], ok[p][1], v[p]);
      convrot256_halfwarp2(v[p], tile, b);
      // invalid blocks rotate zeros, which leave the maximum unchanged
#pragma unroll
      for (int i = 0; i < 16; ++i) m_nan = max_abs2_nan(m_nan, lo2(v[p][i]), hi2(v[p][i]));
      if (MODE == MODE_MAX && rotated != nullptr) {
        float r0[16], r1[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          r0[i] = lo2(v[p][i]);
          r1[i] = hi2(v[p][i]);
        }
        if (ok[p][0]) store_float16(rotated + row * width + blk[p][0] * 16, r0);
        if (ok[p][1]) store_float16(rotated + row * width + blk[p][1] * 16, r1);
      }
    }
    float scale = 0.0f;
    bool finite = false;
    if (MODE == MODE_MAX || MODE == MODE_LOCAL) {
      float m = block_reduce_max_nan(m_nan, red);
      finite = m < __uint_as_float(0x7f800000u);  // false for +inf and NaN
      if (!finite) m = block_reduce_max(local_max_ignoring_nan<NP>(v, ok), red);
      if (tid == 0) row_max[row] = m;
      scale = row_scale_from_max(m);
    } else {
      scale = row_scale_from_max(__ldg(row_max_in + row));
    }
    if (MODE == MODE_QUANT || MODE == MODE_LOCAL) {
      const float inv = __fdiv_rn(1.0f, scale);
      // MODE_QUANT's maximum comes from outside and may be below |x|: scalar path
      quantize_store<NP>(v, ok, blk, MODE == MODE_LOCAL && finite, scale, inv, division,
                         q + row * width);
      if (tid == 0) scale_out[row] = scale;
    }
  }
}

// FC2 producer at TP>1 in one pass.  The row loop is pipelined by one row: a CTA
// rotates row i into registers and publishes its local maximum to every rank, then
// waits for the global maximum of its previous row, quantises that row from the shared-
// memory stash, and only then moves row i from its registers into the stash, so the
// NVLink round trip of a maximum overlaps the next row's loads and rotation.  Each
// thread reads back only what it stashed, and reads row i-1 before it overwrites it
// with row i, so one stash buffer suffices and needs no barrier.  Launched as a
// persistent grid (every CTA resident), so a CTA waiting for a peer's row never waits
// for a CTA that cannot run.
template <int KIND, int NP>
__global__ void __launch_bounds__(512) swiglu_rotate_peer_kernel(
    const void* __restrict__ x, int64_t rows, int64_t width, float* __restrict__ row_max,
    int division, int8_t* __restrict__ q, float* __restrict__ scale_out, const PeerMax pm) {
  extern __shared__ f32x2 smem2[];
  const int tid = threadIdx.x;
  const int T = blockDim.x;
  const int half = tid >> 4, b = tid & 15;
  f32x2* tile = smem2 + half * (16 * 17);
  float* red = reinterpret_cast<float*>(smem2 + (T / 16) * (16 * 17));
  f32x2* stash = reinterpret_cast<f32x2*>(red + 32);  // [NP * 16][T]
  const int64_t blocks = width / 16;
  int64_t blk[NP][2];
  bool ok[NP][2];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      blk[p][e] = tid + (int64_t)(2 * p + e) * T;
      ok[p][e] = blk[p][e] < blocks;
    }
  uint64_t deadline = 0;
  int64_t prev = -1;
  bool prev_finite = false;
  float prev_local = 0.0f;

  for (int64_t row = blockIdx.x;; row += gridDim.x) {
    const bool have = row < rows;
    bool finite = false;
    float m = 0.0f;
    f32x2 v[NP][16];
    if (have) {
      if (row + gridDim.x < rows) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
          prefetch_activation2<KIND>(x, row + gridDim.x, width, blk[p][0], blk[p][1], ok[p][0],
                                     ok[p][1]);
      }
      float m_nan = 0.0f;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        load_activation2<KIND>(x, row, width, blk[p][0], blk[p][1], ok[p][0], ok[p][1], v[p]);
        convrot256_halfwarp2(v[p], tile, b);
#pragma unroll
        for (int i = 0; i < 16; ++i) m_nan = max_abs2_nan(m_nan, lo2(v[p][i]), hi2(v[p][i]));
      }
      m = block_reduce_max_nan(m_nan, red);
      finite = m < __uint_as_float(0x7f800000u);  // false for +inf and NaN
      if (!finite) m = block_reduce_max(local_max_ignoring_nan<NP>(v, ok), red);
      peer_publish(pm, row, m);
    }
    if (prev >= 0) {
      const float g = peer_wait(pm, prev, prev_local, red, deadline);
      // g >= every local |x|: a finite local row keeps the packed quantiser exact when
      // the global maximum is finite too
      const bool fin = prev_finite && g < __uint_as_float(0x7f800000u);
      const float scale = row_scale_from_max(g);
      const float inv = __fdiv_rn(1.0f, scale);
      f32x2 w[NP][16];
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int i = 0; i < 16; ++i) w[p][i] = stash[(p * 16 + i) * T + tid];
      quantize_store<NP>(w, ok, blk, fin, scale, inv, division, q + prev * width);
      if (tid == 0) {
        scale_out[prev] = scale;
        if (row_max != nullptr) row_max[prev] = g;
      }
    }
    if (!have) break;
    // row i-1 is read (above, by this same thread): row i takes its place
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int i = 0; i < 16; ++i) stash[(p * 16 + i) * T + tid] = v[p][i];
    prev = row;
    prev_finite = finite;
    prev_local = m;
  }
}

// Modulated RMSNorm in front of the column quantiser (tilelang_dit_fusion.py:11-37):
// the activation tables and the per-row result.  Unused unless NORM.
struct NormArgs {
  const float* weight;  // [width]
  const float* shift;   // [mod_rows, width]
  const float* scale;   // [mod_rows, width]
  const int32_t* labels;
  int64_t mod_rows;
  float eps, inv_width;
  __half* h;  // optional fp16 output of the norm
  int* err;
};

// CTA sum with the order the oracle restates: a warp xor butterfly, then the warps in
// order.
H3_DEV float block_reduce_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) m = __fadd_rn(m, red[w]);
  __syncthreads();
  return m;
}

// h = f16( (((x *rn inv) *rn W) *rn (1 +rn Scale[l])) +rn Shift[l] ) for the pairs of
// blocks of this thread, in place; the sum of squares runs in the order of
// oracle/h3_oracle.c (per block over i, then the two lanes, then the pairs).
template <int NP>
H3_DEV void modulated_norm_pairs(f32x2 (&v)[NP][16], const int64_t (&blk)[NP][2],
                                 const bool (&ok)[NP][2], int64_t row, int64_t width,
                                 const NormArgs& na, float* red) {
  // A product feeding an addition is written with the scalar __fmul_rn / __fadd_rn,
  // which are never contracted into a fused multiply-add; pure products use f32x2.
  float t = 0.0f;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    float s0 = __fmul_rn(lo2(v[p][0]), lo2(v[p][0]));
    float s1 = __fmul_rn(hi2(v[p][0]), hi2(v[p][0]));
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      s0 = __fadd_rn(s0, __fmul_rn(lo2(v[p][i]), lo2(v[p][i])));
      s1 = __fadd_rn(s1, __fmul_rn(hi2(v[p][i]), hi2(v[p][i])));
    }
    const float tp = __fadd_rn(s0, s1);
    t = p == 0 ? tp : __fadd_rn(t, tp);
  }
  const float total = block_reduce_sum(t, red);
  const float inv = __frsqrt_rn(__fadd_rn(__fmul_rn(total, na.inv_width), na.eps));
  int64_t lab = na.labels ? (int64_t)__ldg(na.labels + row) : 0;
  if (lab < 0 || lab >= na.mod_rows) {
    report_error(na.err, H3_ERR_INVALID);
    lab = 0;
  }
  const float* sh = na.shift + lab * width;
  const float* sc = na.scale + lab * width;
  const f32x2 inv2 = dup2(inv), one = dup2(1.0f);
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    float w[2][16], f[2][16], d[2][16];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t c = (ok[p][e] ? blk[p][e] : 0) * 16;
      load_float16(na.weight + c, w[e]);
      load_float16(sc + c, f[e]);
      load_float16(sh + c, d[e]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const f32x2 scaled = mul2(mul2(mul2(v[p][i], inv2), pk2(w[0][i], w[1][i])),
                                add2(one, pk2(f[0][i], f[1][i])));
      const float y0 = __fadd_rn(lo2(scaled), d[0][i]), y1 = __fadd_rn(hi2(scaled), d[1][i]);
      const float2 hf = __half22float2(__floats2half2_rn(y0, y1));
      v[p][i] = pk2(ok[p][0] ? hf.x : 0.0f, ok[p][1] ? hf.y : 0.0f);
    }
    if (na.h != nullptr) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (!ok[p][e]) continue;
        __half2 hv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          hv[j] = e == 0 ? __floats2half2_rn(lo2(v[p][2 * j]), lo2(v[p][2 * j + 1]))
                         : __floats2half2_rn(hi2(v[p][2 * j]), hi2(v[p][2 * j + 1]));
        uint4* dst = reinterpret_cast<uint4*>(na.h + row * width + blk[p][e] * 16);
        dst[0] = *reinterpret_cast<uint4*>(&hv[0]);
        dst[1] = *reinterpret_cast<uint4*>(&hv[4]);
      }
    }
  }
}

// Column activation preparation (QKV / FC1 input): optional modulated RMSNorm
// (NORM), optional ConvRot256 with an fp16 rounding of the rotated value, then the row
// quantiser.  One CTA per row, packed pairs of blocks as in swiglu_rotate_kernel.
// QUANT = false stops after the norm (its fp16 output only).
template <int NP, bool ROTATE, bool NORM, bool QUANT, bool STAGED>
__global__ void __launch_bounds__(512) column_quantize_kernel(
    const __half* __restrict__ x, int64_t rows, int64_t k, int8_t* __restrict__ q,
    float* __restrict__ scale_out, const NormArgs na, const __grid_constant__ CUtensorMap map,
    const RowStage st) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* rest = smem_raw;
  uint8_t* stages = nullptr;
  uint64_t* bars = nullptr;
  if (STAGED) stages = stage_begin(smem_raw, &map, st, rows, rest, bars);
  f32x2* smem2 = reinterpret_cast<f32x2*>(rest);
  const int tid = threadIdx.x;
  const int half = tid >> 4, b = tid & 15;
  f32x2* tile = smem2 + half * (16 * 17);
  float* red = reinterpret_cast<float*>(smem2 + (blockDim.x / 16) * (16 * 17));
  const int64_t blocks = k / 16;
  int64_t blk[NP][2];
  bool ok[NP][2];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      blk[p][e] = tid + (int64_t)(2 * p + e) * blockDim.x;
      ok[p][e] = blk[p][e] < blocks;
    }
  int it = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    f32x2 v[NP][16];
    if (STAGED) {
      if (!stage_ready(st, bars, it, row, rows)) return;
      const uint8_t* stg = stages + (it % ROW_STAGES) * st.stage_bytes;
#pragma unroll
      for (int p = 0; p < NP; ++p)
        stage_activation2<H3_IN_ACT_F16>(stg, k, blk[p][0], blk[p][1], ok[p][0], ok[p][1], v[p]);
      stage_next(&map, st, stages, bars, it, row, rows);
    } else {
      // the modulated-norm form spends long enough on a row for an L2 prefetch of the
      // next one to pay (measured 3-4% faster); the plain quantiser measured 5% slower
      if (NORM && row + gridDim.x < rows) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
          prefetch_activation2<H3_IN_ACT_F16>(x, row + gridDim.x, k, blk[p][0], blk[p][1],
                                              ok[p][0], ok[p][1]);
      }
#pragma unroll
      for (int p = 0; p < NP; ++p)
        load_activation2<H3_IN_ACT_F16>(x, row, k, blk[p][0], blk[p][1], ok[p][0], ok[p][1], v[p]);
    }
    if (NORM) modulated_norm_pairs<NP>(v, blk, ok, row, k, na, red);
    if (!QUANT) continue;
    float m_nan = 0.0f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      if (ROTATE) {
        convrot256_halfwarp2(v[p], tile, b);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 f = __half22float2(__floats2half2_rn(lo2(v[p][i]), hi2(v[p][i])));
          v[p][i] = pk2(f.x, f.y);
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) m_nan = max_abs2_nan(m_nan, lo2(v[p][i]), hi2(v[p][i]));
    }
    float m = block_reduce_max_nan(m_nan, red);
    const bool finite = m < __uint_as_float(0x7f800000u);
    if (!finite) m = block_reduce_max(local_max_ignoring_nan<NP>(v, ok), red);
    const float scale = row_scale_from_max(m);
    const float inv = __fdiv_rn(1.0f, scale);
    quantize_store<NP>(v, ok, blk, finite, scale, inv, H3_DIV_RN, q + row * k);
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
    // the scalar form, checked against the packed-pair form on both of its lanes
    const float scalar = silu_fast(g[i]);
    const int64_t other = (i & 1) ? i - 1 : (i + 1 < n ? i + 1 : i);
    const f32x2 pair = (i & 1) ? silu_fast2(g[other], g[i]) : silu_fast2(g[i], g[other]);
    const float packed = (i & 1) ? hi2(pair) : lo2(pair);
    const bool same = __float_as_uint(packed) == __float_as_uint(scalar) ||
                      (packed != packed && scalar != scalar);
    fast[i] = same ? scalar : 3.4028234663852886e38f;  // FLT_MAX: the forms disagree
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
// Opts a kernel into more than 48 KB of dynamic shared memory (once per kernel).
template <typename K>
static bool allow_smem(K kernel, size_t smem, bool& done) {
  if (smem <= 48 * 1024 || done) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return false;
  done = true;
  return true;
}

// Whether the producers stage their rows through TMA or load them straight into
// registers (the default).  Staging is opt-in, H3_ROW_STAGING=1 in the environment: on
// one B200 at M = 32768 it measured slower (column quantiser 0.127 ms against 0.107,
// TP1 FC2 producer 0.361 against 0.320) - the persistent grid with two row stages per
// CTA halves the resident warps, and the rows' compute, not their loads, sets the pace.
// Both give the same bits.
static bool row_staging_enabled() {
  static const bool on = [] {
    const char* v = getenv("H3_ROW_STAGING");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}

// Row staging geometry and tensor map for `rows` rows of `row_bytes` bytes at x; false
// when the rows cannot be staged (then the kernels load straight from HBM).
static bool plan_row_stage(const void* x, int64_t rows, int64_t row_bytes, int threads,
                           CUtensorMap* map, RowStage* st) {
  if (!row_staging_enabled() || rows <= 0 || rows >= ((int64_t)1 << 31) || row_bytes % 128)
    return false;
  const int64_t lines = row_bytes / 128;
  const int box = lines <= 256 ? (int)lines : 256;
  if (lines % box) return false;
  st->row_bytes = (int)row_bytes;
  st->stage_bytes = (int)((row_bytes + 1023) / 1024 * 1024);
  st->box_lines = box;
  st->boxes = (int)(lines / box);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  st->err = h3host::error_word(dev);
  if (st->err == nullptr || staged_smem(threads, *st) > 227 * 1024) return false;
  return h3host::encode_row_map(map, x, rows, row_bytes, box);
}

// A persistent grid for a staged kernel: resident CTAs per SM times the SMs, at most one
// CTA per row.
template <typename K>
static int staged_grid(K kernel, int threads, size_t smem, int64_t rows) {
  int per_sm = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    return 0;
  return (int)std::min<int64_t>(rows, (int64_t)per_sm * h3host::sm_count(dev));
}

// Bytes of one producer input row as it lies in HBM.
static int64_t producer_row_bytes(int kind, int64_t width) {
  return kind == H3_IN_GATEUP_F16 ? 4 * width : kind == H3_IN_ACT_F32 ? 4 * width : 2 * width;
}

template <int KIND, int MODE, int NP>
static int launch_producer_np(const void* x, int64_t rows, int64_t width, float* rotated,
                              float* row_max, const float* row_max_in, int division, int8_t* q,
                              float* scale, int threads, cudaStream_t stream) {
  CUtensorMap map;
  RowStage st{};
  if (plan_row_stage(x, rows, producer_row_bytes(KIND, width), threads, &map, &st)) {
    static bool smem_set = false;
    const size_t smem = staged_smem(threads, st);
    if (!allow_smem(swiglu_rotate_kernel<KIND, MODE, NP, true>, smem, smem_set)) return H3_ERR_CUDA;
    const int grid = staged_grid(swiglu_rotate_kernel<KIND, MODE, NP, true>, threads, smem, rows);
    if (grid > 0) {
      swiglu_rotate_kernel<KIND, MODE, NP, true><<<grid, threads, smem, stream>>>(
          x, rows, width, rotated, row_max, row_max_in, division, q, scale, map, st);
      return h3host::check_launch();
    }
  }
  static bool smem_set = false;
  const size_t smem = producer_smem(threads);
  if (!allow_smem(swiglu_rotate_kernel<KIND, MODE, NP, false>, smem, smem_set)) return H3_ERR_CUDA;
  const int grid = (int)std::min<int64_t>(rows, 1 << 20);
  memset(&map, 0, sizeof(map));
  swiglu_rotate_kernel<KIND, MODE, NP, false><<<grid, threads, smem, stream>>>(
      x, rows, width, rotated, row_max, row_max_in, division, q, scale, map, RowStage{});
  return h3host::check_launch();
}

template <int KIND, int MODE>
static int launch_producer(const void* x, int64_t rows, int64_t width, float* rotated,
                           float* row_max, const float* row_max_in, int division, int8_t* q,
                           float* scale, cudaStream_t stream) {
  const RowTeam t = row_team(width);
  if (t.nb == 1)
    return launch_producer_np<KIND, MODE, 1>(x, rows, width, rotated, row_max, row_max_in,
                                             division, q, scale, t.threads, stream);
  if (t.nb == 2)
    return launch_producer_np<KIND, MODE, 2>(x, rows, width, rotated, row_max, row_max_in,
                                             division, q, scale, t.threads, stream);
  return H3_ERR_INVALID;
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

// The peer producer's shared memory: the producer's plus the stash of one row.
static size_t peer_producer_smem(int threads, int np) {
  return producer_smem(threads) + (size_t)np * 16 * threads * sizeof(unsigned long long);
}

template <int KIND, int NP>
static int launch_peer_np(const void* x, int64_t rows, int64_t width, float* row_max,
                          int division, int8_t* q, float* scale, int threads,
                          const PeerMax& pm, cudaStream_t stream) {
  static bool smem_set = false;
  const size_t smem = peer_producer_smem(threads, NP);
  if (!allow_smem(swiglu_rotate_peer_kernel<KIND, NP>, smem, smem_set)) return H3_ERR_CUDA;
  int per_sm = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &per_sm, swiglu_rotate_peer_kernel<KIND, NP>, threads, smem) != cudaSuccess ||
      per_sm < 1)
    return H3_ERR_CUDA;
  const int grid = (int)std::min<int64_t>(rows, (int64_t)per_sm * h3host::sm_count(dev));
  swiglu_rotate_peer_kernel<KIND, NP><<<grid, threads, smem, stream>>>(
      x, rows, width, row_max, division, q, scale, pm);
  return h3host::check_launch();
}

template <int KIND>
static int launch_peer(const void* x, int64_t rows, int64_t width, float* row_max,
                       int division, int8_t* q, float* scale, const PeerMax& pm,
                       cudaStream_t stream) {
  const RowTeam t = row_team(width);
  if (t.nb != 1 || peer_producer_smem(t.threads, 1) > 227 * 1024) return H3_ERR_INVALID;
  return launch_peer_np<KIND, 1>(x, rows, width, row_max, division, q, scale, t.threads, pm,
                                 stream);
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(x, &dev)) return s;
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(x, &dev)) return s;
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(x, &dev)) return s;
  return dispatch_kind<MODE_LOCAL>(input_kind, x, rows, width, nullptr, row_max, nullptr,
                                   division, q, scale, (cudaStream_t)stream);
}

extern "C" int h3_swiglu_rotate_quantize_peer(const void* x, int input_kind, int64_t rows,
                                              int64_t width, const void* const* bases, int world,
                                              int rank, int64_t slots_off, uint32_t epoch,
                                              int division, int8_t* q, float* scale,
                                              float* row_max, void* stream) {
  if (!producer_geometry_ok(x, input_kind, rows, width) || width > H3_PEER_PRODUCER_MAX_WIDTH ||
      q == nullptr || scale == nullptr || !h3host::aligned(q, 16) ||
      (division != H3_DIV_RN && division != H3_DIV_FAST) || bases == nullptr ||
      (world != 2 && world != 4 && world != 8) || rank < 0 || rank >= world || slots_off < 0 ||
      slots_off % 8 != 0 || epoch == 0)
    return H3_ERR_INVALID;
  PeerMax pm{};
  for (int w = 0; w < world; ++w) {
    if (bases[w] == nullptr || !h3host::aligned(bases[w], 16)) return H3_ERR_INVALID;
    pm.bases[w] = reinterpret_cast<uint64_t>(bases[w]);
  }
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(x, &dev)) return s;
  pm.slots_off = slots_off;
  pm.world = world;
  pm.rank = rank;
  pm.epoch = epoch;
  pm.err = h3host::error_word(dev);
  if (pm.err == nullptr) return H3_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  switch (input_kind) {
    case H3_IN_GATEUP_F16:
      return launch_peer<H3_IN_GATEUP_F16>(x, rows, width, row_max, division, q, scale, pm, st);
    case H3_IN_ACT_F32:
      return launch_peer<H3_IN_ACT_F32>(x, rows, width, row_max, division, q, scale, pm, st);
    default:
      return launch_peer<H3_IN_ACT_F16>(x, rows, width, row_max, division, q, scale, pm, st);
  }
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(x_f16, &dev)) return s;
  const RowTeam t = row_team(k);
  const size_t smem = producer_smem(t.threads);
  const int grid = (int)std::min<int64_t>(rows, 1 << 20);
  cudaStream_t st = (cudaStream_t)stream;
  const __half* xh = reinterpret_cast<const __half*>(x_f16);
  static bool smem_set[2][2][2] = {};
  CUtensorMap map;
  RowStage rs{};
  const bool staged = plan_row_stage(x_f16, rows, 2 * k, t.threads, &map, &rs);
  if (!staged) memset(&map, 0, sizeof(map));
#define H3_COLQ(NPV, ROT)                                                                  \
  do {                                                                                     \
    if (staged) {                                                                          \
      auto kern = column_quantize_kernel<NPV, ROT, false, true, true>;                     \
      const size_t ssm = staged_smem(t.threads, rs);                                       \
      if (!allow_smem(kern, ssm, smem_set[NPV - 1][ROT][1])) return H3_ERR_CUDA;           \
      const int g = staged_grid(kern, t.threads, ssm, rows);                               \
      if (g > 0) {                                                                         \
        kern<<<g, t.threads, ssm, st>>>(xh, rows, k, q, scale, NormArgs{}, map, rs);       \
        break;                                                                             \
      }                                                                                    \
      memset(&map, 0, sizeof(map));                                                        \
    }                                                                                      \
    if (!allow_smem(column_quantize_kernel<NPV, ROT, false, true, false>, smem,            \
                    smem_set[NPV - 1][ROT][0]))                                            \
      return H3_ERR_CUDA;                                                                  \
    column_quantize_kernel<NPV, ROT, false, true, false>                                   \
        <<<grid, t.threads, smem, st>>>(xh, rows, k, q, scale, NormArgs{}, map, RowStage{}); \
  } while (0)
  if (t.nb == 1) {
    if (convrot) H3_COLQ(1, true); else H3_COLQ(1, false);
  } else if (t.nb == 2) {
    if (convrot) H3_COLQ(2, true); else H3_COLQ(2, false);
  } else {
    return H3_ERR_INVALID;
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(rotated, &dev)) return s;
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(x, &dev)) return s;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 4096);
  expf_compare_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, n, ours, cuda);
  return h3host::check_launch();
}

extern "C" int h3_silu_compare(const float* g, int64_t n, float* fast, float* ieee,
                               float* cuda, void* stream) {
  if (g == nullptr || fast == nullptr || ieee == nullptr || n < 0) return H3_ERR_INVALID;
  if (n == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(g, &dev)) return s;
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
  h3host::DeviceScope scope;
  if (int s = scope.bind(x, &dev)) return s;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)h3host::sm_count(dev) * 16);
  quant_compare_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, scale, n, fast, ieee);
  return h3host::check_launch();
}

extern "C" int h3_modulated_norm_quantize(const void* x_f16, int64_t rows, int64_t width,
                                          const float* norm_weight, float eps,
                                          const float* shift, const float* scale,
                                          int64_t mod_rows, const int32_t* labels, int convrot,
                                          int8_t* q, float* row_scale, void* h_f16,
                                          void* stream) {
  const bool quant = q != nullptr || row_scale != nullptr;
  if (x_f16 == nullptr || norm_weight == nullptr || shift == nullptr || scale == nullptr ||
      rows < 0 || width <= 0 || width % 16 != 0 || width > 4 * 512 * 16 || mod_rows < 1 ||
      (labels == nullptr && mod_rows != 1) || (quant && (q == nullptr || row_scale == nullptr)) ||
      (!quant && h_f16 == nullptr) || (quant && convrot && width % 256 != 0))
    return H3_ERR_INVALID;
  if (!h3host::aligned(x_f16, 16) || !h3host::aligned(norm_weight, 16) ||
      !h3host::aligned(shift, 16) || !h3host::aligned(scale, 16) ||
      (q != nullptr && !h3host::aligned(q, 16)) || (h_f16 != nullptr && !h3host::aligned(h_f16, 16)))
    return H3_ERR_INVALID;
  if (rows == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(x_f16, &dev)) return s;
  NormArgs na{norm_weight, shift, scale, labels, mod_rows, eps,
              (float)(1.0 / (double)width), reinterpret_cast<__half*>(h_f16),
              h3host::error_word(dev)};
  if (na.err == nullptr) return H3_ERR_CUDA;
  const RowTeam t = row_team(width);
  const size_t smem = producer_smem(t.threads);
  const int grid = (int)std::min<int64_t>(rows, 1 << 20);
  cudaStream_t st = (cudaStream_t)stream;
  const __half* xh = reinterpret_cast<const __half*>(x_f16);
  static bool smem_set[2][3][2] = {};
  CUtensorMap map;
  RowStage rs{};
  const bool staged = plan_row_stage(x_f16, rows, 2 * width, t.threads, &map, &rs);
  if (!staged) memset(&map, 0, sizeof(map));
#define H3_NORMQ(NPV, ROT, QU, SLOT)                                                       \
  do {                                                                                     \
    if (staged) {                                                                          \
      auto kern = column_quantize_kernel<NPV, ROT, true, QU, true>;                        \
      const size_t ssm = staged_smem(t.threads, rs);                                       \
      if (!allow_smem(kern, ssm, smem_set[NPV - 1][SLOT][1])) return H3_ERR_CUDA;          \
      const int g = staged_grid(kern, t.threads, ssm, rows);                               \
      if (g > 0) {                                                                         \
        kern<<<g, t.threads, ssm, st>>>(xh, rows, width, q, row_scale, na, map, rs);       \
        break;                                                                             \
      }                                                                                    \
      memset(&map, 0, sizeof(map));                                                        \
    }                                                                                      \
    if (!allow_smem(column_quantize_kernel<NPV, ROT, true, QU, false>, smem,               \
                    smem_set[NPV - 1][SLOT][0]))                                           \
      return H3_ERR_CUDA;                                                                  \
    column_quantize_kernel<NPV, ROT, true, QU, false>                                      \
        <<<grid, t.threads, smem, st>>>(xh, rows, width, q, row_scale, na, map, RowStage{}); \
  } while (0)
  if (t.nb == 1) {
    if (!quant) H3_NORMQ(1, false, false, 0);
    else if (convrot) H3_NORMQ(1, true, true, 1);
    else H3_NORMQ(1, false, true, 2);
  } else if (t.nb == 2) {
    if (!quant) H3_NORMQ(2, false, false, 0);
    else if (convrot) H3_NORMQ(2, true, true, 1);
    else H3_NORMQ(2, false, true, 2);
  } else {
    return H3_ERR_INVALID;
  }
#undef H3_NORMQ
  return h3host::check_launch();
}
