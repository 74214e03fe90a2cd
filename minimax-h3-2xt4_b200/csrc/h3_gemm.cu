// tcgen05 kind::i8 GEMM for sm_100a with fused epilogues.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]      A: int8 [M, K] activations (K-major)
//                                          B: int8 [N, K] weights     (K-major)
//
// Design (one CTA per SM, persistent over output tiles):
//   - tile 128 x 256 x 128 (BM x BN x BK, BK in bytes); A and B tiles are moved
//     global -> shared by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast)
//     into a 4-stage ring guarded by mbarriers;
//   - warp 0 lane 0 issues the TMA loads; warp 1 lane 0 issues tcgen05.mma
//     (cta_group::1, kind::i8, M=128, N=256, K=32 per instruction) into an INT32
//     accumulator in tensor memory (TMEM); two 256-column accumulators are
//     double-buffered so the epilogue of tile i overlaps the MMAs of tile i+1;
//   - warps 2-17 (four per 32-lane TMEM quadrant, each owning a quarter of the
//     tile's columns) read the accumulator with tcgen05.ld, apply the fused epilogue and
//     store to global memory with 128-bit accesses.
//
// Every mbarrier wait is bounded (2 s of %globaltimer); a wait that gives up sets the
// library's device error word (H3_ERR_TIMEOUT), raises a CTA-wide abort flag, and
// every role then leaves its loop, waits (bounded) for its own TMA copies and MMAs in
// flight, and the CTA frees its TMEM and returns.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "h3_common.cuh"

namespace h3 {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes == int8 elements; one 128-byte swizzle atom row
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;  // 16 KiB
constexpr int B_STAGE = BN * BK;  // 32 KiB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int EPI_WARPS = 16;                // four warps per 32-lane TMEM quadrant
constexpr int EPI_PARTS = EPI_WARPS / 4;     // column slices of a tile, one per warp
constexpr int THREADS = 64 + 32 * EPI_WARPS;  // warp 0 TMA, warp 1 MMA, warps 2.. epilogue
constexpr int TMEM_COLS = 512;
// per epilogue warp: 64 floats of staged weight scales (EPI_SWIGLU)
constexpr int EPI_SMEM = EPI_WARPS * 64 * 4;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + EPI_SMEM;
constexpr unsigned long long TIMEOUT_NS = 2000000000ull;

// 2-SM (cta_group::2) variant: a CTA pair computes a 256 x 256 tile; each CTA stages
// its 128 rows of A and 128 rows (one N half) of B, and holds 128 x 256 of the INT32
// accumulator in its own TMEM.
constexpr int BM2 = 256;
constexpr int B_HALF = (BN / 2) * BK;          // 16 KiB
constexpr int STAGES2 = 6;
constexpr int STAGE2_BYTES = A_STAGE + B_HALF;  // 32 KiB per CTA
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + 1024 + 256 + EPI_SMEM;

// Instruction descriptor, kind::i8: D = S32 (bits 4-5 = 2), A = B = signed 8-bit
// (bits 7-9 and 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

constexpr uint32_t IDESC2 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM2 >> 4) << 24);

enum Epi {
  EPI_I32 = 0,
  EPI_COLUMN = 1,
  EPI_SWIGLU = 2,
  EPI_ROW_ENCODE = 3,
  EPI_ROW_DEQUANT = 4,
  EPI_ROW_PACK8 = 5
};

// Owner-routed encode output (EPI_ROW_ENCODE with world > 0): row r of this rank's
// partial belongs to rank o = r / per, and is stored into o's peer-mapped workspace at
// bases[o] + partial_off, slot row rank * per + (r - o * per) - the reduce-scatter of
// the partials fused into the GEMM's epilogue.
struct PushOut {
  uint64_t bases[8];
  int64_t partial_off;
  int64_t per;
  int world, rank;
};

struct Args {
  int64_t M;          // rows of A / output rows
  int64_t N;          // output columns (SWIGLU: gate rows = n_packed / 2)
  int64_t K;
  int tiles_m, tiles_n, num_kb;
  int group_m, group_n;  // tile raster (tile_coords)
  void* out;
  int out_kind;
  const float* row_scale;
  const float* weight_scale;
  int scalar_w;
  const float* bias;
  float enc_factor;
  RowOut row;
  int res_vec;    // residual / gate rows may use 128-bit accesses
  int scale_vec;  // weight scales / bias may use 128-bit loads
  int out_wide;   // output rows may use 256-bit stores (32-byte base, N % 16 == 0)
  int res_wide;   // residual rows may use 256-bit loads and stores (same conditions)
  PushOut push;   // EPI_ROW_ENCODE: owner-routed output when push.world > 0
  int m_rotate;   // M-blocks the tile order is rotated by (owner-routed output)
  int* err;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
H3_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

H3_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

H3_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

H3_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (and raises the abort flag) on timeout, or when another
// role has already aborted and honour_abort is set.
H3_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                      bool honour_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 63u) == 0) {
      if (honour_abort && *abort_flag) return false;
      if (globaltimer() - t0 > TIMEOUT_NS) {
        *abort_flag = 1;
        report_error(err, H3_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

H3_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

H3_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

H3_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                        uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

H3_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
H3_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

H3_DEV void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

H3_DEV void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

H3_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of `saddr` (a shared::cta address) in CTA `rank` of the cluster
H3_DEV uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

H3_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

H3_DEV void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// TMA load into this CTA's shared memory that completes its bytes on the pair
// leader's mbarrier (no multicast).
H3_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                             uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(cluster_bar)
      : "memory");
}

H3_DEV void tc_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_bar)
               : "memory");
}

H3_DEV void tc_mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core groups 1024 B
// apart (SBO), descriptor version 1, base offset 0 (stage buffers are 1024-aligned).
H3_DEV uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1u << 46;             // version
  d |= (uint64_t)2u << 61;             // SWIZZLE_128B
  return d;
}

H3_DEV void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

H3_DEV void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

H3_DEV void tmem_ld8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// tcgen05.wait::ld with the 16 destination registers of the loads it completes passed
// through it: the loads write those registers asynchronously, and the operands keep the
// compiler from moving any use of them above the wait.
H3_DEV void tmem_wait_ld(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

H3_DEV void tmem_wait_ld(uint32_t (&a)[8], uint32_t (&b)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]),
                 "+r"(a[6]), "+r"(a[7]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]),
                 "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])
               :
               : "memory");
}

// Tile order.  group_n > 0: groups of group_n N-blocks (a weight slab that stays in
// L2) sweep all M-blocks, N fastest, so A is read from HBM once per group; otherwise
// groups of group_m M-blocks (16 when unset) sweep all N-blocks, M fastest, so B is
// read once per group.  The host picks the form with less HBM traffic.
H3_DEV void rotate_m(const Args& a, int& mb) {
  mb += a.m_rotate;
  if (mb >= a.tiles_m) mb -= a.tiles_m;
}

H3_DEV void tile_coords(int tile, const Args& a, int& mb, int& nb) {
  if (a.group_n > 0) {
    const int group = a.group_n * a.tiles_m;
    const int g = tile / group;
    const int first_n = g * a.group_n;
    const int gn = min(a.tiles_n - first_n, a.group_n);
    const int local = tile - g * group;
    nb = first_n + local % gn;
    mb = local / gn;
    rotate_m(a, mb);
    return;
  }
  const int G = a.group_m > 0 ? a.group_m : 16;
  const int group = G * a.tiles_n;
  const int g = tile / group;
  const int first_m = g * G;
  const int gm = min(a.tiles_m - first_m, G);
  const int local = tile - g * group;
  mb = first_m + local % gm;
  nb = local / gm;
  rotate_m(a, mb);
}

// ---------------------------------------------------------------------------
// Epilogue helpers: one thread owns one output row and 32 consecutive columns.
//
// A warp's store writes 32 different rows, one segment of each.  sm_100's 256-bit
// accesses (ld / st .v8.b32) make that segment a whole 32-byte sector per lane and
// instruction instead of two 16-byte halves: half the store instructions and memory
// requests, no partially written sectors.  Measured on the FC1-shaped INT32 GEMM
// (M = 32768, N = 16384, K = 3072): 1.71 ms with 128-bit stores, 1.17 ms with 256-bit.
// ---------------------------------------------------------------------------
H3_DEV void st_v8(void* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]),
               "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// the same for output that is not read again soon: no L1 line, L2 evict-first
H3_DEV void st_v8_stream(void* p, const uint32_t (&w)[8]) {
  asm volatile(
      "st.global.L1::no_allocate.L2::evict_first.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p),
      "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
      : "memory");
}

H3_DEV void ld_v8(const void* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                 "=r"(w[6]), "=r"(w[7])
               : "l"(p)
               : "memory");
}

template <int C>
H3_DEV void store_f16_chunk(__half* dst, int64_t n0, int64_t N, const float (&v)[C], bool vec,
                            bool wide = false) {
  if (C % 16 == 0 && wide && n0 + C <= N) {
#pragma unroll
    for (int i = 0; i < C / 16; ++i) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half2 h = __floats2half2_rn(v[16 * i + 2 * j], v[16 * i + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      st_v8(dst + 16 * i, w);
    }
  } else if (vec && n0 + C <= N) {
    uint4* p = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      __half2 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
      p[i] = *reinterpret_cast<uint4*>(h);
    }
  } else {
#pragma unroll
    for (int j = 0; j < C; ++j)
      if (n0 + j < N) dst[j] = __float2half_rn(v[j]);
  }
}

// stream: evict-first stores (__stcs) for outputs that are not read again soon
template <int C>
H3_DEV void store_f32_chunk(float* dst, int64_t n0, int64_t N, const float (&v)[C], bool vec,
                            bool stream = false, bool wide = false) {
  if (C % 8 == 0 && wide && n0 + C <= N) {
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = __float_as_uint(v[8 * i + j]);
      if (stream)
        st_v8_stream(dst + 8 * i, w);
      else
        st_v8(dst + 8 * i, w);
    }
  } else if (vec && n0 + C <= N) {
    float4* p = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < C / 4; ++i) {
      const float4 f = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      if (stream)
        __stcs(p + i, f);
      else
        p[i] = f;
    }
  } else {
#pragma unroll
    for (int j = 0; j < C; ++j)
      if (n0 + j < N) dst[j] = v[j];
  }
}

// Gated residual update of C consecutive columns of one row
// (tilelang_dit_fusion.py:68-75): X = f16(fma(f32(f16(y)), G[lab], f32(X))).
template <int C>
H3_DEV void residual_chunk(const RowOut& o, int64_t row, int64_t n0, int64_t N, int64_t lab,
                           const float (&y)[C], bool vec, bool wide = false) {
  if (C % 16 == 0 && wide && n0 + C <= N) {
    __half* p = o.residual + row * N + n0;
    const float4* g4 = o.gate ? reinterpret_cast<const float4*>(o.gate + lab * N + n0) : nullptr;
#pragma unroll
    for (int i = 0; i < C / 16; ++i) {
      uint32_t u[8];
      ld_v8(p + 16 * i, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float g0 = 1.0f, g1 = 1.0f;
        if (g4 != nullptr) {
          const float4 gq = __ldg(g4 + 4 * i + j / 2);
          g0 = (j & 1) ? gq.z : gq.x;
          g1 = (j & 1) ? gq.w : gq.y;
        }
        __half2 h = *reinterpret_cast<const __half2*>(&u[j]);
        const float2 x = __half22float2(h);
        const float b0 = __half2float(__float2half_rn(y[16 * i + 2 * j]));
        const float b1 = __half2float(__float2half_rn(y[16 * i + 2 * j + 1]));
        h = __floats2half2_rn(__fmaf_rn(b0, g0, x.x), __fmaf_rn(b1, g1, x.y));
        u[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      st_v8(p + 16 * i, u);
    }
  } else if (vec && n0 + C <= N) {
    uint4* p = reinterpret_cast<uint4*>(o.residual + row * N + n0);
    const float4* g4 = o.gate ? reinterpret_cast<const float4*>(o.gate + lab * N + n0) : nullptr;
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      uint4 u = p[i];
      __half2* h = reinterpret_cast<__half2*>(&u);
      float g[8];
      if (g4 != nullptr) {
        const float4 ga = __ldg(g4 + 2 * i), gb = __ldg(g4 + 2 * i + 1);
        g[0] = ga.x; g[1] = ga.y; g[2] = ga.z; g[3] = ga.w;
        g[4] = gb.x; g[5] = gb.y; g[6] = gb.z; g[7] = gb.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = 1.0f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = __half22float2(h[j]);
        const float b0 = __half2float(__float2half_rn(y[8 * i + 2 * j]));
        const float b1 = __half2float(__float2half_rn(y[8 * i + 2 * j + 1]));
        h[j] = __floats2half2_rn(__fmaf_rn(b0, g[2 * j], x.x), __fmaf_rn(b1, g[2 * j + 1], x.y));
      }
      p[i] = u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < C; ++j)
      if (n0 + j < N) row_store(o, row, n0 + j, N, y[j]);
  }
}

template <int C>
H3_DEV void load_scales(const float* w, int64_t n0, int64_t N, int scalar, float (&s)[C],
                        bool vec = false) {
  if (vec && !scalar && n0 + C <= N) {
    const float4* p = reinterpret_cast<const float4*>(w + n0);
#pragma unroll
    for (int i = 0; i < C / 4; ++i) {
      const float4 f = __ldg(p + i);
      s[4 * i] = f.x; s[4 * i + 1] = f.y; s[4 * i + 2] = f.z; s[4 * i + 3] = f.w;
    }
  } else if (scalar) {
    const float v = __ldg(w);
#pragma unroll
    for (int j = 0; j < C; ++j) s[j] = v;
  } else {
#pragma unroll
    for (int j = 0; j < C; ++j) s[j] = (n0 + j < N) ? __ldg(w + n0 + j) : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// Epilogue of one output tile: this warp's 32 TMEM lanes (`row` is the lane's output
// row) and one EPI_PARTS-th of the tile's 256 accumulator columns.
// ---------------------------------------------------------------------------
template <int EPI>
H3_DEV void epilogue_tile(const Args& args, uint32_t tbase, int64_t row, bool row_ok, int nb,
                          int part, float* wsm) {
  const int64_t N = args.N;
  if (EPI == EPI_SWIGLU) {
    // accumulator columns [0,128) = gate rows, [128,256) = up rows of this tile
    constexpr int GCOLS = (BN / 2) / EPI_PARTS;  // gate columns of this warp
    const int64_t n_base = (int64_t)nb * (BN / 2) + part * GCOLS;
    const float a = row_ok ? __ldg(args.row_scale + row) : 0.0f;
    const bool vec4 = args.scale_vec != 0;
    constexpr int SW = 8;  // columns per step: keeps the SwiGLU epilogue within 96 registers
    // This warp's 32 gate and 32 up weight scales, staged in shared memory once per
    // tile (one coalesced load per lane) and read back as broadcasts.
    const int lane = threadIdx.x & 31;
    __syncwarp();
    {
      const int64_t nl = n_base + lane;
      wsm[lane] = nl < N ? __ldg(args.weight_scale + nl) : 0.0f;
      wsm[32 + lane] = nl < N ? __ldg(args.weight_scale + N + nl) : 0.0f;
    }
    __syncwarp();
#pragma unroll 1
    for (int c = 0; c < GCOLS / SW; ++c) {
      const int64_t n0 = n_base + c * SW;
      if (n0 >= N) break;  // warp-uniform
      uint32_t rg[SW], ru[SW];
      tmem_ld8_nowait(tbase + part * GCOLS + c * SW, rg);
      tmem_ld8_nowait(tbase + BN / 2 + part * GCOLS + c * SW, ru);
      float wg[SW], wu[SW];
#pragma unroll
      for (int i = 0; i < SW / 4; ++i) {
        const float4 g4 = reinterpret_cast<const float4*>(wsm + c * SW)[i];
        const float4 u4 = reinterpret_cast<const float4*>(wsm + 32 + c * SW)[i];
        wg[4 * i] = g4.x; wg[4 * i + 1] = g4.y; wg[4 * i + 2] = g4.z; wg[4 * i + 3] = g4.w;
        wu[4 * i] = u4.x; wu[4 * i + 1] = u4.y; wu[4 * i + 2] = u4.z; wu[4 * i + 3] = u4.w;
      }
      float bg[SW], bu[SW];
      if (args.bias != nullptr) {
        load_scales<SW>(args.bias, n0, N, 0, bg, vec4);
        load_scales<SW>(args.bias + N, n0, N, 0, bu, vec4);
      }
      tmem_wait_ld(rg, ru);
      float y[SW];
      if (args.bias == nullptr) {
        // two columns per step on packed f32x2 lanes (the same bits, half the issue)
        const f32x2 a2 = dup2(a);
#pragma unroll
        for (int j = 0; j < SW; j += 2) {
          const f32x2 vg = mul2(pk2(__int2float_rn((int32_t)rg[j]), __int2float_rn((int32_t)rg[j + 1])),
                                mul2(a2, pk2(wg[j], wg[j + 1])));
          const f32x2 vu = mul2(pk2(__int2float_rn((int32_t)ru[j]), __int2float_rn((int32_t)ru[j + 1])),
                                mul2(a2, pk2(wu[j], wu[j + 1])));
          const f32x2 o = swiglu_f32x2(__half2float(__float2half_rn(lo2(vg))),
                                       __half2float(__float2half_rn(hi2(vg))),
                                       __half2float(__float2half_rn(lo2(vu))),
                                       __half2float(__float2half_rn(hi2(vu))));
          y[j] = lo2(o);
          y[j + 1] = hi2(o);
        }
      } else {
#pragma unroll
        for (int j = 0; j < SW; ++j) {
          float vg = __fmul_rn(__int2float_rn((int32_t)rg[j]), __fmul_rn(a, wg[j]));
          float vu = __fmul_rn(__int2float_rn((int32_t)ru[j]), __fmul_rn(a, wu[j]));
          vg = __fadd_rn(vg, bg[j]);
          vu = __fadd_rn(vu, bu[j]);
          const float g = __half2float(__float2half_rn(vg));
          const float u = __half2float(__float2half_rn(vu));
          y[j] = swiglu_f32(g, u);
        }
      }
      if (row_ok) {
        if (args.out_kind == H3_OUT_F32)
          store_f32_chunk<SW>(reinterpret_cast<float*>(args.out) + row * N + n0, n0, N, y,
                              (N & 3) == 0, true, args.out_wide != 0);
        else
          store_f16_chunk<SW>(reinterpret_cast<__half*>(args.out) + row * N + n0, n0, N, y,
                              (N & 7) == 0);
      }
    }
  } else if (EPI == EPI_ROW_PACK8) {
    // Packed INT8 transport payload (tilelang_transport_tradeoffs.py:40-62): per row and
    // 128-column group, scale = max(max|f32(P)| *rn f32(1/127), 1e-8) and
    // q = clamp(rint(f32(P) /rn scale), -127, 127).  A group is the columns of two warps
    // of the same TMEM lane quadrant (parts 2g', 2g'+1); each warp reads the whole group
    // from TMEM for the maximum (no exchange between warps) and codes its own 64.
    constexpr int COLS = BN / EPI_PARTS;  // 64
    const int gl = part >> 1;             // group within the tile
    const int64_t g = (int64_t)nb * (BN / 128) + gl;
    if (g * 128 >= N) return;  // warp-uniform: the whole group is past the last column
    float m = 0.0f;
#pragma unroll 1
    for (int c = 0; c < 128 / 16; ++c) {
      uint32_t r[16];
      tmem_ld16_nowait(tbase + gl * 128 + c * 16, r);
      tmem_wait_ld(r);
#pragma unroll
      for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(__int2float_rn((int32_t)r[j])));
    }
    const float scale = fmaxf(__fmul_rn(m, f32_bits(H3_INV127_BITS)), f32_bits(0x322bcc77u));
    const float inv = __fdiv_rn(1.0f, scale);
    uint8_t* dst = reinterpret_cast<uint8_t*>(args.out) + row * ((N / 128) * 132) + g * 132;
#pragma unroll 1
    for (int c = 0; c < COLS / 16; ++c) {
      uint32_t r[16];
      tmem_ld16_nowait(tbase + part * COLS + c * 16, r);
      tmem_wait_ld(r);
      if (!row_ok) continue;
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t b[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // |x / scale| <= 127 (1 + 2^-23): the clamp is kept for form's sake, the code
          // is the low byte of RN(q + 1.5 * 2^23)
          const float q = fminf(127.0f, fmaxf(-127.0f, div_by_scale(
                                                             __int2float_rn((int32_t)r[4 * k + e]),
                                                             scale, inv)));
          b[e] = __float_as_uint(__fadd_rn(q, 12582912.0f));
        }
        w[k] = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
      }
      uint32_t* d = reinterpret_cast<uint32_t*>(dst + (part & 1) * COLS + c * 16);
#pragma unroll
      for (int k = 0; k < 4; ++k) d[k] = w[k];
    }
    if (row_ok && (part & 1) == 0) *reinterpret_cast<float*>(dst + 128) = scale;
  } else {
    constexpr int COLS = BN / EPI_PARTS;  // accumulator columns of this warp
    const int64_t n_base = (int64_t)nb * BN + part * COLS;
    const float a = (row_ok && args.row_scale != nullptr) ? __ldg(args.row_scale + row) : 0.0f;
    int64_t lab = 0;
    if (EPI == EPI_ROW_DEQUANT && args.row.kind == H3_OUT_RESIDUAL && row_ok &&
        args.row.gate != nullptr && args.row.labels != nullptr) {
      lab = __ldg(args.row.labels + row);
      if (lab < 0 || lab >= args.row.gate_rows) {
        report_error(args.row.err, H3_ERR_INVALID);
        lab = 0;
      }
    }
#pragma unroll 1
    for (int c = 0; c < COLS / 16; ++c) {
      const int64_t n0 = n_base + c * 16;
      if (n0 >= N) break;  // warp-uniform
      uint32_t r[16];
      tmem_ld16_nowait(tbase + part * COLS + c * 16, r);
      float w[16];
      if (EPI == EPI_COLUMN || EPI == EPI_ROW_DEQUANT)
        load_scales<16>(args.weight_scale, n0, N, EPI == EPI_COLUMN ? args.scalar_w : 0, w,
                        args.scale_vec != 0);
      tmem_wait_ld(r);
      if (!row_ok) continue;
      if (EPI == EPI_I32) {
        int32_t* dst = reinterpret_cast<int32_t*>(args.out) + row * N + n0;
        if (args.out_wide && n0 + 16 <= N) {
          uint32_t w0[8], w1[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            w0[j] = r[j];
            w1[j] = r[8 + j];
          }
          st_v8(dst, w0);
          st_v8(dst + 8, w1);
        } else if (n0 + 16 <= N && (N & 3) == 0) {
          int4* p = reinterpret_cast<int4*>(dst);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            p[i] = make_int4((int)r[4 * i], (int)r[4 * i + 1], (int)r[4 * i + 2], (int)r[4 * i + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (n0 + j < N) dst[j] = (int32_t)r[j];
        }
      } else if (EPI == EPI_COLUMN) {
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          y[j] = __fmul_rn(__int2float_rn((int32_t)r[j]), __fmul_rn(a, w[j]));
          if (args.bias != nullptr && n0 + j < N) y[j] = __fadd_rn(y[j], __ldg(args.bias + n0 + j));
        }
        store_f16_chunk<16>(reinterpret_cast<__half*>(args.out) + row * N + n0, n0, N, y,
                            (N & 7) == 0, args.out_wide != 0);
      } else if (EPI == EPI_ROW_ENCODE) {
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = __fmul_rn(__int2float_rn((int32_t)r[j]), args.enc_factor);
        __half* dst;
        if (args.push.world > 0) {
          // the owner's slot row for this rank, selected without indexing the
          // parameter array by a register
          const int64_t owner = row / args.push.per;
          uint64_t base = args.push.bases[0];
#pragma unroll
          for (int o = 1; o < 8; ++o)
            if (owner == o) base = args.push.bases[o];
          const int64_t slot = (int64_t)args.push.rank * args.push.per + (row - owner * args.push.per);
          dst = reinterpret_cast<__half*>(base + args.push.partial_off) + slot * N + n0;
        } else {
          dst = reinterpret_cast<__half*>(args.out) + row * N + n0;
        }
        store_f16_chunk<16>(dst, n0, N, y, (N & 7) == 0, args.out_wide != 0);
      } else {  // EPI_ROW_DEQUANT
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          y[j] = __fmul_rn(__fmul_rn(__int2float_rn((int32_t)r[j]), a), w[j]);
        if (args.row.kind == H3_OUT_F32) {
          store_f32_chunk<16>(reinterpret_cast<float*>(args.row.out) + row * N + n0, n0, N, y,
                              (N & 3) == 0, false, args.out_wide != 0);
        } else if (args.row.kind == H3_OUT_F16) {
          store_f16_chunk<16>(reinterpret_cast<__half*>(args.row.out) + row * N + n0, n0, N, y,
                              (N & 7) == 0, args.out_wide != 0);
        } else {
          residual_chunk<16>(args.row, row, n0, N, lab, y, args.res_vec != 0,
                             args.res_wide != 0);
        }
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmB2, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* wsm = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256) +
               (threadIdx.x / 32 >= 2 ? (threadIdx.x / 32 - 2) * 64 : 0);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(tfull + a), 1);
      mbar_init(smem_u32(tempty + a), 32 * EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = args.tiles_m * args.tiles_n;
  const int num_kb = args.num_kb;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, args, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full + stage);
          mbar_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(smem_u32(sA + stage * A_STAGE), &tmA, kb * BK, mb * BM, fb);
          if (EPI == EPI_SWIGLU) {
            tma_load_2d(smem_u32(sB + stage * B_STAGE), &tmB, kb * BK, nb * (BN / 2), fb);
            tma_load_2d(smem_u32(sB + stage * B_STAGE + (BN / 2) * BK), &tmB2, kb * BK,
                        nb * (BN / 2), fb);
          } else {
            tma_load_2d(smem_u32(sB + stage * B_STAGE), &tmB, kb * BK, nb * BN, fb);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every TMA copy this thread issued must have landed before the CTA exits.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          mbar_wait(smem_u32(full + s), (issued_parity >> s) & 1u, abort_flag, args.err, false);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer --------------------------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(smem_u32(tempty + acc), acc_phase ^ 1u, abort_flag, args.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_STAGE);
          const uint32_t b0 = smem_u32(sB + stage * B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            tc_mma_i8(d_tmem, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), IDESC,
                      (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(empty + stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(tfull + acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // All MMAs issued by this thread complete before TMEM is released.
      tc_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, abort_flag, args.err, false);
    }
  } else {
    // ------------------------------ epilogue ------------------------------------
    const int quad = warp & 3;          // TMEM lanes [32*quad, 32*quad + 32)
    const int part = (warp - 2) >> 2;   // which column slice of the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, args, mb, nb);
      if (!mbar_wait(smem_u32(tfull + acc), acc_phase, abort_flag, args.err)) break;
      tc_fence_after();
      const int64_t row = (int64_t)mb * BM + quad * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      epilogue_tile<EPI>(args, tbase, row, row < args.M, nb, part, wsm);
      tc_fence_before();
      mbar_arrive(smem_u32(tempty + acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // owner-routed rows went to other GPUs: performed before the kernel completes
    if (EPI == EPI_ROW_ENCODE && args.push.world > 0) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}


// ---------------------------------------------------------------------------
// 2-SM kernel: clusters of two CTAs; CTA rank 0 (the leader) issues the M=256 MMAs.
//   full[s]   leader only: one arrive.expect_tx (both CTAs' bytes) + the TMA bytes of
//             both CTAs (each CTA's loads complete on the leader's barrier)
//   empty[s]  each CTA: released by the leader's commit after the MMAs read stage s
//   tfull[a]  each CTA: released by the leader's commit when accumulator a is final
//   tempty[a] leader only: one arrive per epilogue warp of both CTAs
// ---------------------------------------------------------------------------
template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmB2, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES2 * A_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES2;
  uint64_t* tfull = bars + 2 * STAGES2;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* wsm = reinterpret_cast<float*>(smem + STAGES2 * STAGE2_BYTES + 256) +
               (threadIdx.x / 32 >= 2 ? (threadIdx.x / 32 - 2) * 64 : 0);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(tfull + a), 1);
      mbar_init(smem_u32(tempty + a), 2 * EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = args.tiles_m * args.tiles_n;
  const int num_kb = args.num_kb;
  const int cluster_id = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------- TMA producer (both CTAs) ----------------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < total_tiles && ok; tile += clusters) {
        int mb, nb;
        tile_coords(tile, args, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full + stage);
          if (leader) mbar_expect_tx(fb, 2 * STAGE2_BYTES);
          const uint32_t fb_leader = cluster_addr(fb, 0);
          tma_load_2d_pair(smem_u32(sA + stage * A_STAGE), &tmA, kb * BK,
                           mb * BM2 + (int)rank * BM, fb_leader);
          if (EPI == EPI_SWIGLU) {
            // rank 0 stages the 128 gate rows, rank 1 the 128 up rows of this tile
            tma_load_2d_pair(smem_u32(sB + stage * B_HALF), rank == 0 ? &tmB : &tmB2, kb * BK,
                             nb * (BN / 2), fb_leader);
          } else {
            tma_load_2d_pair(smem_u32(sB + stage * B_HALF), &tmB, kb * BK,
                             nb * BN + (int)rank * (BN / 2), fb_leader);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader's full barriers complete only when both CTAs' copies landed.
      if (leader)
        for (int s = 0; s < STAGES2; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(smem_u32(full + s), (issued_parity >> s) & 1u, abort_flag, args.err, false);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------------------- MMA issuer (leader) ---------------------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < total_tiles && ok; tile += clusters) {
        if (!mbar_wait(smem_u32(tempty + acc), acc_phase ^ 1u, abort_flag, args.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_STAGE);
          const uint32_t b0 = smem_u32(sB + stage * B_HALF);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            tc_mma_i8_pair(d_tmem, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), IDESC2,
                           (kb | k) != 0 ? 1u : 0u);
          }
          const uint32_t eb = smem_u32(empty + stage);
          tc_commit_pair(cluster_addr(eb, 0));
          tc_commit_pair(cluster_addr(eb, 1));
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t tb = smem_u32(tfull + acc);
        tc_commit_pair(cluster_addr(tb, 0));
        tc_commit_pair(cluster_addr(tb, 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // All MMAs complete before either CTA releases its TMEM.
      tc_commit_pair(cluster_addr(smem_u32(drain), 0));
      mbar_wait(smem_u32(drain), 0, abort_flag, args.err, false);
    }
  } else {
    // ---------------------------- epilogue (both CTAs) ----------------------------
    const int quad = warp & 3;
    const int part = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cluster_id; tile < total_tiles; tile += clusters) {
      int mb, nb;
      tile_coords(tile, args, mb, nb);
      if (!mbar_wait(smem_u32(tfull + acc), acc_phase, abort_flag, args.err)) break;
      tc_fence_after();
      const int64_t row = (int64_t)mb * BM2 + (int64_t)rank * BM + quad * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      epilogue_tile<EPI>(args, tbase, row, row < args.M, nb, part, wsm);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(cluster_addr(smem_u32(tempty + acc), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (EPI == EPI_ROW_ENCODE && args.push.world > 0) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair still reads its smem or TMEM
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major int8 [rows, k] with a (box_rows x 128-byte) box and 128-byte swizzle.
static bool make_map(CUtensorMap* map, const int8_t* base, int64_t rows, int64_t k, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool device_is_sm100(int dev) {
  static int cache[64] = {0};  // 0 unknown, 1 yes, 2 no
  if (dev < 0 || dev >= 64) return false;
  if (cache[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cache[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return cache[dev] == 1;
}

// Chooses the tile raster: keep a slab of A (group_m M-blocks) or of B (group_n
// N-blocks) of about 32 MB resident in the 126 MB L2 while the other operand streams,
// whichever reads fewer bytes from HBM: A + B * ceil(tiles_m / group_m) against
// B + A * ceil(tiles_n / group_n).
static void set_raster(Args& a, int64_t a_block_bytes, int64_t b_block_bytes) {
  const int64_t budget = 32ll << 20;
  const int64_t gm = std::max<int64_t>(1, std::min<int64_t>(a.tiles_m, budget / a_block_bytes));
  const int64_t gn = std::max<int64_t>(1, std::min<int64_t>(a.tiles_n, budget / b_block_bytes));
  const int64_t A = a_block_bytes * a.tiles_m, B = b_block_bytes * a.tiles_n;
  const int64_t m_cost = A + B * ((a.tiles_m + gm - 1) / gm);
  const int64_t n_cost = B + A * ((a.tiles_n + gn - 1) / gn);
  a.group_m = n_cost < m_cost ? 0 : (int)gm;
  a.group_n = n_cost < m_cost ? (int)gn : 0;
}

// Geometry every GEMM launch accepts: K a multiple of 16, M < 2^31, N <= 2^24,
// K <= 2^20, 16-byte aligned operands and a tile count that fits an int.
template <int EPI>
static bool gemm_geometry_ok(const int8_t* q, const int8_t* w, int64_t M, int64_t N, int64_t K) {
  if (q == nullptr || w == nullptr || M < 0 || N <= 0 || K <= 0 || K % 16 != 0) return false;
  if (!h3host::aligned(q, 16) || !h3host::aligned(w, 16)) return false;
  if (M > (int64_t)1 << 31 || N > (int64_t)1 << 24 || K > (int64_t)1 << 20) return false;
  const bool pair = M > BM;
  const int64_t tile_m = pair ? BM2 : BM, tile_n = EPI == EPI_SWIGLU ? BN / 2 : BN;
  return ((M + tile_m - 1) / tile_m) * ((N + tile_n - 1) / tile_n) <= INT32_MAX;
}

// Enqueues one GEMM.  args.err, when the caller set it, replaces the library's device
// error word (the no-allocation entry keeps its own in static memory).
template <int EPI>
static int launch(const int8_t* q, const int8_t* w, int64_t M, int64_t N, int64_t K, Args args,
                  cudaStream_t stream) {
  if (!gemm_geometry_ok<EPI>(q, w, M, N, K)) return H3_ERR_INVALID;
  if (M == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(q, &dev)) return s;
  if (!device_is_sm100(dev)) return H3_ERR_UNSUPPORTED;
  // CTA pairs (256-row tiles) once there is more than one 128-row block; a single
  // CTA per tile below that.
  const bool pair = M > BM;
  const int bn_rows = EPI == EPI_SWIGLU ? BN / 2 : (pair ? BN / 2 : BN);
  CUtensorMap tA, tB, tB2;
  if (!make_map(&tA, q, M, K, BM)) return H3_ERR_INVALID;
  if (EPI == EPI_SWIGLU) {
    if (!make_map(&tB, w, N, K, bn_rows)) return H3_ERR_INVALID;
    if (!make_map(&tB2, w + N * K, N, K, bn_rows)) return H3_ERR_INVALID;
  } else {
    if (!make_map(&tB, w, N, K, bn_rows)) return H3_ERR_INVALID;
    tB2 = tB;
  }
  const int tile_n = EPI == EPI_SWIGLU ? BN / 2 : BN;
  args.M = M;
  args.N = N;
  args.K = K;
  args.tiles_m = (int)((M + (pair ? BM2 : BM) - 1) / (pair ? BM2 : BM));
  args.tiles_n = (int)((N + tile_n - 1) / tile_n);
  args.num_kb = (int)((K + BK - 1) / BK);
  set_raster(args, (pair ? BM2 : BM) * K, (EPI == EPI_SWIGLU ? 2 * tile_n : tile_n) * K);
  {
    const void* o = EPI == EPI_ROW_DEQUANT ? args.row.out : args.out;
    bool wide = o != nullptr && h3host::aligned(o, 32);
    if (args.push.world > 0) {
      wide = args.push.partial_off % 32 == 0;
      for (int w = 0; w < args.push.world; ++w)
        wide = wide && args.push.bases[w] % 32 == 0;
    }
    args.out_wide = wide && N % 16 == 0;
    // Owner-routed rows: every rank starts on its own row block and walks the blocks
    // from there, so that at any time the ranks store into different owners instead of
    // all into the owner of the same rows (an incast on one GPU's links).
    args.m_rotate = 0;
    if (args.push.world > 0) {
      const int64_t tm = (M + (pair ? BM2 : BM) - 1) / (pair ? BM2 : BM);
      args.m_rotate = (int)(((int64_t)args.push.rank * args.push.per / (pair ? BM2 : BM)) % tm);
    }
    args.res_wide = EPI == EPI_ROW_DEQUANT && args.row.residual != nullptr &&
                    h3host::aligned(args.row.residual, 32) && N % 16 == 0 &&
                    (args.row.gate == nullptr || h3host::aligned(args.row.gate, 16));
  }
  if (args.err == nullptr) args.err = h3host::error_word(dev);
  if (args.err == nullptr) return H3_ERR_CUDA;
  if (args.row.err == nullptr) args.row.err = args.err;
  const int64_t tiles = (int64_t)args.tiles_m * args.tiles_n;
  const int sms = h3host::sm_count(dev);
  static bool attr_set[64][2] = {{false}};
  if (pair) {
    if (!attr_set[dev][1]) {
      if (cudaFuncSetAttribute(gemm_i8_pair_kernel<EPI>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES) != cudaSuccess)
        return H3_ERR_CUDA;
      attr_set[dev][1] = true;
    }
    const int grid = 2 * (int)std::min<int64_t>(tiles, sms / 2);
    gemm_i8_pair_kernel<EPI><<<grid, THREADS, SMEM2_BYTES, stream>>>(tA, tB, tB2, args);
  } else {
    if (!attr_set[dev][0]) {
      if (cudaFuncSetAttribute(gemm_i8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               SMEM_BYTES) != cudaSuccess)
        return H3_ERR_CUDA;
      attr_set[dev][0] = true;
    }
    const int grid = (int)std::min<int64_t>(tiles, sms);
    gemm_i8_kernel<EPI><<<grid, THREADS, SMEM_BYTES, stream>>>(tA, tB, tB2, args);
  }
  return h3host::check_launch();
}

static Args blank_args() {
  Args a;
  memset(&a, 0, sizeof(a));
  a.row.kind = H3_OUT_F32;
  return a;
}

}  // namespace gemm
}  // namespace h3

using namespace h3;
using namespace h3::gemm;

extern "C" int h3_int8_gemm_i32(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                                int64_t k, int32_t* out, void* stream) {
  if (out == nullptr || !h3host::aligned(out, 16)) return H3_ERR_INVALID;
  Args a = blank_args();
  a.out = out;
  return launch<EPI_I32>(q, w, m, n, k, a, (cudaStream_t)stream);
}

extern "C" int h3_int8_gemm_column(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                                   int64_t k, const float* row_scale, const float* weight_scale,
                                   int64_t weight_scale_len, const float* bias, void* out_f16,
                                   void* stream) {
  if (out_f16 == nullptr || row_scale == nullptr || weight_scale == nullptr ||
      (weight_scale_len != 1 && weight_scale_len != n) || !h3host::aligned(out_f16, 16))
    return H3_ERR_INVALID;
  Args a = blank_args();
  a.out = out_f16;
  a.row_scale = row_scale;
  a.weight_scale = weight_scale;
  a.scalar_w = weight_scale_len == 1;
  a.bias = bias;
  a.scale_vec = n % 4 == 0 && h3host::aligned(weight_scale, 16);
  return launch<EPI_COLUMN>(q, w, m, n, k, a, (cudaStream_t)stream);
}

extern "C" int h3_int8_gemm_swiglu(const int8_t* q, const int8_t* w, int64_t m,
                                   int64_t n_packed, int64_t k, const float* row_scale,
                                   const float* weight_scale, const float* bias, int out_kind,
                                   void* out, void* stream) {
  if (out == nullptr || row_scale == nullptr || weight_scale == nullptr || n_packed <= 0 ||
      n_packed % 2 != 0 || (out_kind != H3_OUT_F32 && out_kind != H3_OUT_F16) ||
      !h3host::aligned(out, 16) || k % 16 != 0)
    return H3_ERR_INVALID;
  Args a = blank_args();
  a.out = out;
  a.out_kind = out_kind;
  a.row_scale = row_scale;
  a.weight_scale = weight_scale;
  a.bias = bias;
  a.scale_vec = (n_packed / 2) % 4 == 0 && h3host::aligned(weight_scale, 16) &&
                (bias == nullptr || h3host::aligned(bias, 16));
  return launch<EPI_SWIGLU>(q, w, m, n_packed / 2, k, a, (cudaStream_t)stream);
}

extern "C" int h3_int8_gemm_row_encode(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                                       int64_t k, int shift, void* out_f16, void* stream) {
  if (out_f16 == nullptr || shift < 0 || shift > 60 || !h3host::aligned(out_f16, 16))
    return H3_ERR_INVALID;
  Args a = blank_args();
  a.out = out_f16;
  a.enc_factor = ldexpf(1.0f, -shift);
  return launch<EPI_ROW_ENCODE>(q, w, m, n, k, a, (cudaStream_t)stream);
}

extern "C" int h3_int8_gemm_row_encode_push(const int8_t* q, const int8_t* w, int64_t m,
                                            int64_t n, int64_t k, int shift,
                                            const void* const* bases, int world, int rank,
                                            int64_t partial_off, void* stream) {
  if (shift < 0 || shift > 60 || bases == nullptr || (world != 2 && world != 4 && world != 8) ||
      rank < 0 || rank >= world || partial_off < 0 || partial_off % 16 != 0 || n % 8 != 0)
    return H3_ERR_INVALID;
  Args a = blank_args();
  for (int r = 0; r < world; ++r) {
    if (bases[r] == nullptr || !h3host::aligned(bases[r], 16)) return H3_ERR_INVALID;
    a.push.bases[r] = reinterpret_cast<uint64_t>(bases[r]);
  }
  a.push.world = world;
  a.push.rank = rank;
  a.push.partial_off = partial_off;
  a.push.per = m > 0 ? (m + world - 1) / world : 1;
  a.out = const_cast<void*>(bases[rank]);
  a.enc_factor = ldexpf(1.0f, -shift);
  return launch<EPI_ROW_ENCODE>(q, w, m, n, k, a, (cudaStream_t)stream);
}

extern "C" int h3_int8_gemm_row_pack8(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                                      int64_t k, void* out_u8, void* stream) {
  if (out_u8 == nullptr || n % 128 != 0 || !h3host::aligned(out_u8, 16)) return H3_ERR_INVALID;
  Args a = blank_args();
  a.out = out_u8;
  return launch<EPI_ROW_PACK8>(q, w, m, n, k, a, (cudaStream_t)stream);
}

extern "C" int h3_int8_gemm_row_dequant(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                                        int64_t k, const float* row_scale,
                                        const float* weight_scale, int out_kind, void* out,
                                        void* residual_f16, const float* gate, int64_t gate_rows,
                                        const int32_t* labels, void* stream) {
  if (row_scale == nullptr || weight_scale == nullptr) return H3_ERR_INVALID;
  if (out_kind == H3_OUT_RESIDUAL) {
    if (residual_f16 == nullptr) return H3_ERR_INVALID;
    if (gate != nullptr && (gate_rows < 1 || (labels == nullptr && gate_rows != 1)))
      return H3_ERR_INVALID;
  } else if (out_kind == H3_OUT_F32 || out_kind == H3_OUT_F16) {
    if (out == nullptr || !h3host::aligned(out, 16)) return H3_ERR_INVALID;
  } else {
    return H3_ERR_INVALID;
  }
  Args a = blank_args();
  a.row_scale = row_scale;
  a.weight_scale = weight_scale;
  a.row = RowOut{out_kind, out, reinterpret_cast<__half*>(residual_f16), gate, gate_rows, labels,
                 nullptr};
  a.scale_vec = n % 4 == 0 && h3host::aligned(weight_scale, 16);
  a.res_vec = (n % 8 == 0) && h3host::aligned(residual_f16, 16) &&
              (gate == nullptr || h3host::aligned(gate, 16));
  return launch<EPI_ROW_DEQUANT>(q, w, m, n, k, a, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Column linear that allocates nothing.
//
// For callers that must not allocate device memory: runtimes that account for every
// byte of device memory through their own pool (the ComfyUI rank worker budgets
// weights and activations; an allocation behind its back defeats that budget), and
// latency-critical paths where cudaMalloc's implicit synchronisation is unacceptable.  The activation codes, the
// row scales and the device error word live in one file-scope static __device__
// array of H3_NOALLOC_SCRATCH_BYTES, held by every GPU that loads this library until
// the process exits.  Every call on a device shares that array and leaves its
// contents behind, so calls whose GPU work overlaps (different streams, or several
// host threads) race with each other.
// ---------------------------------------------------------------------------
namespace h3 {
namespace noalloc {

static __device__ __align__(256) uint8_t g_scratch[H3_NOALLOC_SCRATCH_BYTES];

// Device address of g_scratch for each device, looked up once with that device
// current.  In host code g_scratch names a host-side shadow, not device memory, so
// only the address returned by cudaGetSymbolAddress may be handed to a kernel.
static uint8_t* scratch_ptr(int dev) {
  static uint8_t* cache[64] = {nullptr};
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cache[dev] = static_cast<uint8_t*>(p);
  }
  return cache[dev];
}

static int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

}  // namespace noalloc
}  // namespace h3

extern "C" int h3_column_linear_noalloc(const void* x_f16, int64_t m, int64_t k, int convrot,
                                        const int8_t* w, int64_t n, const float* weight_scale,
                                        int64_t weight_scale_len, const float* bias,
                                        void* out_f16, void* stream) {
  using namespace h3::noalloc;
  // layout: [error word | row scales | codes], each 256-byte aligned
  const int64_t scale_off = 256;
  const int64_t code_off = m >= 0 ? scale_off + align256(m * 4) : 0;
  // Everything the two launches below would refuse is refused here, before either runs:
  // the GEMM's geometry (checked on the codes' future address), the quantiser's width
  // rules, and the size of the static scratch.
  if (x_f16 == nullptr || w == nullptr || weight_scale == nullptr || out_f16 == nullptr ||
      m < 0 || m > ((int64_t)1 << 31) || (weight_scale_len != 1 && weight_scale_len != n) ||
      !h3host::aligned(x_f16, 16) || !h3host::aligned(out_f16, 16) ||
      !gemm_geometry_ok<EPI_COLUMN>(reinterpret_cast<const int8_t*>(256), w, m, n, k) ||
      (convrot ? k % 256 != 0 : k % 16 != 0) || k > 4 * 512 * 16)
    return H3_ERR_INVALID;
  if (code_off + m * k > (int64_t)H3_NOALLOC_SCRATCH_BYTES)
    return H3_ERR_INVALID;  // beyond the static scratch: use h3_column_quantize + h3_int8_gemm_column
  if (m == 0) return H3_OK;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(x_f16, &dev)) return s;
  if (!device_is_sm100(dev)) return H3_ERR_UNSUPPORTED;
  uint8_t* base = scratch_ptr(dev);
  if (base == nullptr) return H3_ERR_CUDA;
  int* err = reinterpret_cast<int*>(base);
  float* row_scale = reinterpret_cast<float*>(base + scale_off);
  int8_t* q = reinterpret_cast<int8_t*>(base + code_off);
  cudaStream_t st = (cudaStream_t)stream;
  // the error word is the only scratch that must start at zero; codes and scales are
  // rewritten in full below
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return H3_ERR_CUDA;
  if (int s = h3_column_quantize(x_f16, m, k, convrot, q, row_scale, stream)) return s;

  // GEMM + ordered column epilogue, as h3_int8_gemm_column with the static error word
  Args args = blank_args();
  args.out = out_f16;
  args.row_scale = row_scale;
  args.weight_scale = weight_scale;
  args.scalar_w = weight_scale_len == 1;
  args.bias = bias;
  args.scale_vec = n % 4 == 0 && h3host::aligned(weight_scale, 16);
  args.err = err;
  return launch<EPI_COLUMN>(q, w, m, n, k, args, st);
}

extern "C" int h3_column_linear_noalloc_error(int device, int* code) {
  if (code == nullptr) return H3_ERR_INVALID;
  *code = 0;
  h3host::DeviceScope scope;
  if (int s = scope.bind_index(device)) return s;
  uint8_t* base = h3::noalloc::scratch_ptr(device);
  if (base == nullptr) return H3_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return H3_ERR_CUDA;
  return cudaMemcpy(code, base, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess ? H3_OK
                                                                                    : H3_ERR_CUDA;
}
