// Row transport over NVLink peer memory: the scaled-FP16 partial SUM of the row
// parallel linear (tilelang_transport_p2.py:57-58, NCCL fp16 SUM) fused with its
// epilogue (decode, FP32 dequant, gated residual; tilelang_dit_fusion.py:57-77).
//
// Every rank owns one buffer of the same layout, mapped into every other rank's
// address space (torch symmetric memory); `bases[w]` is rank w's buffer as seen from
// this process.  Rank r owns rows [r * per, min(rows, (r + 1) * per)) of the output.
//
//   [flags_off]    ready[64] u32 | done[64] u32 | counter u32   (zeroed once at set-up)
//   [partial_off]  fp16 [rows][width]: this rank's encoded partial (written by the row
//                  GEMM's encode epilogue)
//   [final_off]    fp16 [rows][width]: the other ranks' finished rows, stored there by
//                  their reduce kernels
//
// One call with epoch e (the same on every rank, increasing by one per call):
//   reduce kernel  each CTA stores e into ready[rank] of every rank (release, system
//                  scope), waits until its own ready[w] >= e for every w, then loads
//                  the rows it owns from every rank's partial (bulk copies into shared
//                  memory, reduce_bulk_kernel; or coalesced 16-byte loads per lane,
//                  reduce_kernel), sums them in rank order 0..world-1 (fp32, one fp16 rounding
//                  at the end, the bits of an NCCL fp16 SUM at world 2), decodes,
//                  dequantises and applies the gated residual to those rows of the
//                  local residual, and stores the finished rows into every peer's final
//                  area (coalesced NVLink stores, in the other direction of the links).
//                  The last CTA to finish stores e into done[rank] of every rank.
//   gather kernel  waits until done[w] >= e for every peer w and copies the peers'
//                  finished rows from its own final area into the residual (local).
//
// The NVLS form of the reduce kernel (h3_peer_reduce_nvls) takes the multicast address
// of the same buffers (an NVLink SHARP / NVLS multicast object bound to every rank's
// allocation): each 16-byte chunk of the owned rows is read with one
// multimem.ld_reduce, which makes the NVSwitch fetch the chunk from every rank and
// return the lane-wise sum (fp32 accumulation, one fp16 rounding), and each finished
// chunk is written with one multimem.st, which the switch replicates into every rank's
// final area.  Per rank the links then carry about 2*rows*width bytes each way instead
// of 2 * (world-1)/world * 2*rows*width.  At world 2 the switch's sum of two fp16
// values is the single RN addition (the fp32 sum of two fp16 values rounds once to
// fp16 correctly); at world 4 and 8 the switch's summation order is its own, so the
// result can differ from the rank-order sum in the last fp16 bit where the fp32
// partial sums are inexact.  Flags, waits and buffer reuse are those of the p2p form.
//
// Reuse across calls is ordered by the flags: a rank rewrites its partial only in its
// next row GEMM, after its gather of this call, which waited for every peer's done
// (so every peer has finished loading it); and a rank stores into a peer's final area
// only after that peer signalled ready for the new call (so the peer's previous
// gather has finished).  All waits are bounded (2 s of %globaltimer); a wait that
// gives up records H3_ERR_TIMEOUT in the library's device error word, and a reduce
// that timed out publishes no done flag, so the peers' gathers time out too rather
// than read unfinished rows.

#include "h3_common.cuh"

namespace h3 {
namespace peer {

constexpr int MAX_WORLD = 8;
constexpr int64_t READY = 0, DONE = 256, COUNTER = 512;
constexpr unsigned long long TIMEOUT_NS = 2000000000ull;
// 128 threads a CTA: with up to 64 registers a thread, one CTA fits on an SM beside a
// GEMM CTA (576 threads, <= 96 registers), so a reduce issued on another stream runs
// while the tensor cores work (the pipelined TP forward relies on it).
constexpr int THREADS = 128;

struct Args {
  uint64_t bases[MAX_WORLD];
  uint64_t mc;  // multicast (NVLS) address of the same buffer, 0 when unused
  int64_t flags_off, partial_off, final_off;
  int world, rank;
  int64_t rows, width, row_begin, row_end, per;
  float up;
  const float* row_scale;
  const float* weight_scale;
  __half* residual;
  const float* gate;
  int64_t gate_rows;
  const int32_t* labels;
  uint32_t epoch;
  int64_t own_off;  // FP16_PUSHED: this rank's own rows of its block (slot `rank`)
  int final_local;  // finished rows into this rank's own final area (the peers pull them)
  int* err;
};

H3_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

H3_DEV uint32_t* flag(const Args& a, int owner, int64_t region, int slot) {
  return reinterpret_cast<uint32_t*>(a.bases[owner] + a.flags_off + region) + slot;
}

H3_DEV void store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

H3_DEV uint32_t load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..world-1 each wait for one rank's flag in `region` of this rank's buffer;
// returns (to every thread of the CTA) whether all of them arrived in time.
H3_DEV bool wait_all(const Args& a, int64_t region, bool skip_self) {
  bool ok = true;
  if ((int)threadIdx.x < a.world && !(skip_self && (int)threadIdx.x == a.rank)) {
    const uint32_t* f = flag(a, a.rank, region, threadIdx.x);
    const uint64_t t0 = globaltimer();
    while ((int32_t)(load_acquire(f) - a.epoch) < 0) {
      if (globaltimer() - t0 > TIMEOUT_NS) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  ok = __syncthreads_and(ok);
  if (ok) asm volatile("fence.acq_rel.sys;" ::: "memory");
  return ok;
}

// Reads data another GPU stored into this GPU's memory (through L2, not L1).
H3_DEV uint4 load_received(uint64_t base, int64_t off) {
  return __ldcg(reinterpret_cast<const uint4*>(base + off));
}

// Reads another GPU's memory over NVLink (not cached).
H3_DEV uint4 load_peer(uint64_t base, int64_t off) {
  return __ldcv(reinterpret_cast<const uint4*>(base + off));
}

// In-switch reduction (NVLS): the NVSwitch loads this 16-byte chunk from every rank's
// buffer and returns their sum, accumulated in fp32 and rounded once to fp16 per lane.
H3_DEV uint4 load_reduce_nvls(uint64_t mc, int64_t off) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc + off)
               : "memory");
  return v;
}

// One store through the multicast address: the switch writes the chunk into every
// rank's buffer.
H3_DEV void store_all_nvls(uint64_t mc, int64_t off, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + off),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Decode of an already reduced fp16 chunk: restored = (int32) trunc(f32(t) *rn 2^s).
H3_DEV void restore_reduced(const Args& a, uint4 u, int32_t (&q)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    q[2 * j] = __float2int_rz(__fmul_rn(f.x, a.up));
    q[2 * j + 1] = __float2int_rz(__fmul_rn(f.y, a.up));
  }
}

// fp16 payloads (scaled-FP16 scheme): rank-order fp32 sum of the W partial chunks, one
// fp16 rounding, truncating decode (tilelang_transport_p2.py:15-47).
template <int W>
H3_DEV void restore_fp16(const Args& a, const uint4 (&u)[W], int32_t (&q)[8]) {
  float t[8];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const __half2* h = reinterpret_cast<const __half2*>(&u[w]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      if (w == 0) {
        t[2 * j] = f.x;
        t[2 * j + 1] = f.y;
      } else {
        t[2 * j] = __fadd_rn(t[2 * j], f.x);
        t[2 * j + 1] = __fadd_rn(t[2 * j + 1], f.y);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k)
    q[k] = __float2int_rz(__fmul_rn(__half2float(__float2half_rn(t[k])), a.up));
}

// Packed INT8 payloads ('int8_gather', tilelang_transport_tradeoffs.py:40-62 and
// tilelang_transport_p2.py:28-42): rows of groups * 132 bytes, per 128-column group 128
// codes then the fp32 scale.  restored = rint(sum_w f32(q_w) *rn s_w), rank order.
template <int W>
H3_DEV void load_restore_int8(const Args& a, int64_t r, int64_t c0, int32_t (&q)[8]) {
  const int64_t g = c0 >> 7;
  const int64_t row = a.partial_off + r * ((a.width >> 7) * 132) + g * 132;
  const int64_t off = row + (c0 - (g << 7));
  uint32_t w0[W], w1[W];
  float sc[W];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const uint64_t base = a.bases[w];
    if (w == a.rank) {
      w0[w] = __ldcg(reinterpret_cast<const unsigned int*>(base + off));
      w1[w] = __ldcg(reinterpret_cast<const unsigned int*>(base + off + 4));
      sc[w] = __ldcg(reinterpret_cast<const float*>(base + row + 128));
    } else {
      w0[w] = __ldcv(reinterpret_cast<const unsigned int*>(base + off));
      w1[w] = __ldcv(reinterpret_cast<const unsigned int*>(base + off + 4));
      sc[w] = __ldcv(reinterpret_cast<const float*>(base + row + 128));
    }
  }
  float t[8];
#pragma unroll
  for (int w = 0; w < W; ++w)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t word = k < 4 ? w0[w] : w1[w];
      const float x = __fmul_rn((float)(int8_t)(word >> (8 * (k & 3))), sc[w]);
      t[k] = w == 0 ? x : __fadd_rn(t[k], x);
    }
#pragma unroll
  for (int k = 0; k < 8; ++k) q[k] = __float2int_rn(t[k]);
}

// The shared epilogue of one 8-column chunk from its restored INT32 sums: dequant
// y = (f32(q) *rn A[r]) *rn W[c], then X = f16(fma(f32(f16(y)), G[lab], f32(X))).
H3_DEV uint4 epilogue_chunk(const Args& a, const int32_t (&q)[8], int64_t r, int64_t c0,
                            uint4 x) {
  const float s = __ldg(a.row_scale + r);
  const float4 w0 = __ldg(reinterpret_cast<const float4*>(a.weight_scale + c0));
  const float4 w1 = __ldg(reinterpret_cast<const float4*>(a.weight_scale + c0) + 1);
  const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  float g[8];
  if (a.gate != nullptr) {
    int64_t lab = a.labels ? (int64_t)__ldg(a.labels + r) : 0;
    if (lab < 0 || lab >= a.gate_rows) {
      report_error(a.err, H3_ERR_INVALID);
      lab = 0;
    }
    const float4* gp = reinterpret_cast<const float4*>(a.gate + lab * a.width + c0);
    const float4 g0 = __ldg(gp), g1 = __ldg(gp + 1);
    g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
    g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = 1.0f;
  }
  __half2* xh = reinterpret_cast<__half2*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float b[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int k = 2 * j + e;
      const float y = __fmul_rn(__fmul_rn(__int2float_rn(q[k]), s), ws[k]);
      b[e] = __half2float(__float2half_rn(y));
    }
    const float2 xf = __half22float2(xh[j]);
    xh[j] = __floats2half2_rn(__fmaf_rn(b[0], g[2 * j], xf.x), __fmaf_rn(b[1], g[2 * j + 1], xf.y));
  }
  return x;
}

// FP16_PUSHED: the row GEMM already stored every rank's partial of this rank's block
// into this rank's buffer (slot w = rank w's rows, h3_int8_gemm_row_encode_push), so
// the reduce reads only local memory.
enum Payload { FP16_P2P = 0, INT8_P2P = 1, FP16_NVLS = 2, FP16_PUSHED = 3 };

template <int W, int PAYLOAD>
__global__ void __launch_bounds__(THREADS) reduce_kernel(const Args a) {
  // Phase 0: this rank's partial is complete (stream order after the row GEMM);
  // announce it to every rank.
  if ((int)threadIdx.x < W) {
    __threadfence_system();
    store_release(flag(a, threadIdx.x, READY, a.rank), a.epoch);
  }
  const bool ok = wait_all(a, READY, false);
  if (ok) {
    const int64_t chunks = a.width >> 3;
    const int64_t total = (a.row_end - a.row_begin) * chunks;
    const int64_t first = a.row_begin * chunks;  // uint4 index of the block's first chunk
    const int64_t stride = (int64_t)gridDim.x * THREADS;
    uint4* res = reinterpret_cast<uint4*>(a.residual);
    uint64_t own = a.bases[0];  // this rank's buffer, without indexing by a register
#pragma unroll
    for (int w = 1; w < W; ++w)
      if (w == a.rank) own = a.bases[w];
    // U chunks per thread and iteration, all their loads issued before any is used: the
    // NVLink (or switch) round trip is paid once per U chunks.  U keeps the loaded
    // words within the register budget that lets a CTA sit beside a GEMM CTA.
    constexpr int U = PAYLOAD == FP16_NVLS ? 4
                      : ((PAYLOAD == FP16_P2P || PAYLOAD == FP16_PUSHED) && W == 2) ? 2 : 1;
    constexpr int L = (PAYLOAD == FP16_P2P || PAYLOAD == FP16_PUSHED) ? W : 1;  // words a chunk
    for (int64_t i0 = blockIdx.x * (int64_t)THREADS + threadIdx.x; i0 < total; i0 += stride * U) {
      uint4 u[U][L], x[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int64_t i = i0 + k * stride;
        if (i >= total || PAYLOAD == INT8_P2P) continue;
        const int64_t e = first + i;  // uint4 index of the chunk in [rows][width]
        if (PAYLOAD == FP16_NVLS) {
          u[k][0] = load_reduce_nvls(a.mc, a.partial_off + e * 16);
        } else if (PAYLOAD == FP16_PUSHED) {
          // chunk i of slot w (rank w's rows of this block) in this rank's own buffer
#pragma unroll
          for (int w = 0; w < L; ++w)
            u[k][w] = load_received(own, w == a.rank ? a.own_off + i * 16
                                                     : a.partial_off + (w * a.per * chunks + i) * 16);
        } else {
#pragma unroll
          for (int w = 0; w < L; ++w)
            u[k][w] = w == a.rank ? load_received(a.bases[w], a.partial_off + e * 16)
                                  : load_peer(a.bases[w], a.partial_off + e * 16);
        }
        x[k] = res[e];
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int64_t i = i0 + k * stride;
        if (i >= total) break;
        const int64_t e = first + i;
        const int64_t r = e / chunks;
        const int64_t c0 = (e - r * chunks) << 3;
        int32_t q[8];
        if (PAYLOAD == FP16_NVLS) {
          restore_reduced(a, u[k][0], q);
        } else if (PAYLOAD == INT8_P2P) {
          load_restore_int8<W>(a, r, c0, q);
          x[k] = res[e];
        } else {
          uint4 uw[W];
#pragma unroll
          for (int w = 0; w < W; ++w) uw[w] = u[k][w < L ? w : 0];
          restore_fp16<W>(a, uw, q);
        }
        const uint4 y = epilogue_chunk(a, q, r, c0, x[k]);
        res[e] = y;
        if (PAYLOAD == FP16_NVLS) {
          store_all_nvls(a.mc, a.final_off + e * 16, y);
        } else if (a.final_local) {
          reinterpret_cast<uint4*>(own + a.final_off)[e] = y;
        } else {
#pragma unroll
          for (int w = 0; w < W; ++w)
            if (w != a.rank) reinterpret_cast<uint4*>(a.bases[w] + a.final_off)[e] = y;
        }
      }
    }
  } else if (threadIdx.x == 0) {
    report_error(a.err, H3_ERR_TIMEOUT);
  }
  // Every thread fences its stores to the peers; then count this CTA (failures in the
  // high half-word); the last one resets the counter and, when every CTA succeeded,
  // publishes done to every rank.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* counter =
        reinterpret_cast<unsigned int*>(a.bases[a.rank] + a.flags_off + COUNTER);
    const unsigned int old = atomicAdd(counter, ok ? 1u : 0x10000u);
    const unsigned int seen = (old & 0xffffu) + (old >> 16);
    if (seen == gridDim.x - 1) {
      const bool all_ok = ok && (old >> 16) == 0;
      *reinterpret_cast<volatile unsigned int*>(counter) = 0;
      __threadfence_system();
      if (all_ok)
        for (int w = 0; w < W; ++w) store_release(flag(a, w, DONE, a.rank), a.epoch);
    }
  }
}

// ---------------------------------------------------------------------------
// Pull reduce with bulk copies (the default p2p form).  The owned rows of every rank's
// partial reach shared memory through cp.async.bulk - the SM's bulk-copy unit, one
// 2-8 KB request per rank and tile, completing on the stage's mbarrier - instead of one
// 16-byte load per lane: NVLink then carries a few large reads instead of many small
// ones, and no thread holds a register while they are in flight.  The copies read the
// peers' memory directly and carry no multicast.  BULK_STAGES tiles of BULK_STAGE bytes
// (the W ranks' slices of BULK_STAGE / 16 / W chunks) are in flight per CTA; the sum,
// decode, epilogue and final-row stores are those of reduce_kernel.  Every wait is
// bounded; a CTA that gives up records H3_ERR_TIMEOUT, waits (bounded again) for the
// copies it issued to land before it leaves, and publishes no done flag.
// ---------------------------------------------------------------------------
constexpr int BULK_THREADS = 128;
constexpr int BULK_STAGES = 4;
constexpr int BULK_STAGE = 16384;

H3_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

H3_DEV bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for a stage barrier; `deadline` is set at the first wait that has to
// spin and bounds all later ones of the same caller.
H3_DEV bool bulk_wait(uint32_t bar, uint32_t parity, uint64_t& deadline) {
  while (!mbar_try(bar, parity)) {
    const uint64_t now = globaltimer();
    if (deadline == 0) deadline = now + TIMEOUT_NS;
    if (now > deadline) return false;
  }
  return true;
}

// Thread 0: tile t of the owned block (chunks [t * TC, ...)) from every rank into stage s.
template <int W>
H3_DEV void bulk_issue(const Args& a, uint8_t* stages, uint64_t* bars, int64_t t, int s,
                       int64_t total, uint64_t block_off) {
  constexpr int TC = BULK_STAGE / 16 / W;
  const int64_t c0 = t * TC;
  const uint32_t bytes = (uint32_t)(min((int64_t)TC, total - c0) * 16);
  const uint32_t bar = smem_u32(bars + s);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes * W)
               : "memory");
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const uint32_t dst = smem_u32(stages + ((int64_t)s * W + w) * TC * 16);
    const uint64_t src = a.bases[w] + block_off + (uint64_t)c0 * 16;
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
  }
}

template <int W>
__global__ void __launch_bounds__(BULK_THREADS) reduce_bulk_kernel(const Args a) {
  extern __shared__ __align__(128) uint8_t stages[];
  __shared__ __align__(8) uint64_t bars[BULK_STAGES];
  constexpr int TC = BULK_STAGE / 16 / W;
  if (threadIdx.x == 0) {
    for (int s = 0; s < BULK_STAGES; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bars + s)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // Phase 0: this rank's partial is complete (stream order after the row GEMM).
  if ((int)threadIdx.x < W) {
    __threadfence_system();
    store_release(flag(a, threadIdx.x, READY, a.rank), a.epoch);
  }
  bool ok = wait_all(a, READY, false);  // also orders the barrier initialisation
  const int64_t chunks = a.width >> 3;
  const int64_t total = (a.row_end - a.row_begin) * chunks;
  const int64_t first = a.row_begin * chunks;
  const uint64_t block_off = (uint64_t)a.partial_off + (uint64_t)first * 16;
  const int64_t tiles = (total + TC - 1) / TC;
  const int64_t mine = (ok && blockIdx.x < tiles) ? (tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (threadIdx.x == 0)
    for (int64_t k = 0; k < mine && k < BULK_STAGES; ++k)
      bulk_issue<W>(a, stages, bars, blockIdx.x + k * gridDim.x, (int)k, total, block_off);
  uint4* res = reinterpret_cast<uint4*>(a.residual);
  uint64_t deadline = 0;
  int64_t k = 0;
  for (; k < mine; ++k) {
    const int s = (int)(k % BULK_STAGES);
    const bool landed = bulk_wait(smem_u32(bars + s), (uint32_t)((k / BULK_STAGES) & 1), deadline);
    if (!__syncthreads_and(landed)) {
      ok = false;
      break;
    }
    const int64_t c0 = (blockIdx.x + k * gridDim.x) * TC;
    const int n = (int)min((int64_t)TC, total - c0);
    const uint4* st = reinterpret_cast<const uint4*>(stages + (int64_t)s * W * TC * 16);
    for (int j = threadIdx.x; j < n; j += BULK_THREADS) {
      uint4 u[W];
#pragma unroll
      for (int w = 0; w < W; ++w) u[w] = st[w * TC + j];
      const int64_t e = first + c0 + j;  // uint4 index of the chunk in [rows][width]
      const int64_t r = e / chunks;
      const int64_t cc = (e - r * chunks) << 3;
      int32_t q[8];
      restore_fp16<W>(a, u, q);
      const uint4 y = epilogue_chunk(a, q, r, cc, res[e]);
      res[e] = y;
#pragma unroll
      for (int w = 0; w < W; ++w)
        if (w != a.rank) reinterpret_cast<uint4*>(a.bases[w] + a.final_off)[e] = y;
    }
    __syncthreads();  // stage s has been read by every thread
    if (threadIdx.x == 0 && k + BULK_STAGES < mine)
      bulk_issue<W>(a, stages, bars, blockIdx.x + (k + BULK_STAGES) * gridDim.x, s, total,
                    block_off);
  }
  if (!ok && threadIdx.x == 0) {
    report_error(a.err, H3_ERR_TIMEOUT);
    // the copies this CTA issued land in its shared memory: wait for them (bounded)
    uint64_t drain = 0;
    for (int64_t kk = k; kk < mine && kk < k + BULK_STAGES; ++kk)
      bulk_wait(smem_u32(bars + kk % BULK_STAGES), (uint32_t)((kk / BULK_STAGES) & 1), drain);
  }
  // done publication as in reduce_kernel
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* counter =
        reinterpret_cast<unsigned int*>(a.bases[a.rank] + a.flags_off + COUNTER);
    const unsigned int old = atomicAdd(counter, ok ? 1u : 0x10000u);
    const unsigned int seen = (old & 0xffffu) + (old >> 16);
    if (seen == gridDim.x - 1) {
      const bool all_ok = ok && (old >> 16) == 0;
      *reinterpret_cast<volatile unsigned int*>(counter) = 0;
      __threadfence_system();
      if (all_ok)
        for (int w = 0; w < W; ++w) store_release(flag(a, w, DONE, a.rank), a.epoch);
    }
  }
}

template <int W>
__global__ void __launch_bounds__(THREADS) gather_kernel(const Args a) {
  if (!wait_all(a, DONE, true)) {
    if (threadIdx.x == 0) report_error(a.err, H3_ERR_TIMEOUT);
    return;
  }
  const int64_t chunks = a.width >> 3;
  const int64_t own = a.row_end - a.row_begin;
  const int64_t total = (a.rows - own) * chunks;
  const uint64_t fin = a.bases[a.rank] + a.final_off;
  uint4* res = reinterpret_cast<uint4*>(a.residual);
  for (int64_t i = blockIdx.x * (int64_t)THREADS + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * THREADS) {
    int64_t r = i / chunks;
    if (r >= a.row_begin) r += own;
    const int64_t e = r * chunks + i % chunks;
    res[e] = load_received(fin, e * 16);
  }
}

// The bulk-copy pull reduce is the p2p default; H3_PEER_BULK=0 selects the lane-load
// reduce_kernel (the same bits), read once per process.
static bool bulk_pull() {
  static const bool on = [] {
    const char* e = getenv("H3_PEER_BULK");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

template <int W>
cudaError_t launch_bulk(const Args& a, int dev, cudaStream_t st) {
  constexpr int TC = BULK_STAGE / 16 / W;
  const size_t smem = (size_t)BULK_STAGES * BULK_STAGE;
  static bool attr[64] = {false};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(reduce_bulk_kernel<W>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  const int64_t total = (a.row_end - a.row_begin) * (a.width >> 3);
  const int64_t tiles = (total + TC - 1) / TC;
  // three CTAs an SM (64 KB of stages each): 48 tiles of 16 KB in flight per SM
  const int blocks = (int)std::max<int64_t>(
      1, std::min<int64_t>(tiles, (int64_t)h3host::sm_count(dev) * 3));
  reduce_bulk_kernel<W><<<blocks, BULK_THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

template <int W>
cudaError_t launch(const Args& a, int blocks, bool gather, int payload, int dev,
                   cudaStream_t st) {
  if (gather)
    gather_kernel<W><<<blocks, THREADS, 0, st>>>(a);
  else if (payload == FP16_P2P && bulk_pull())
    return launch_bulk<W>(a, dev, st);
  else if (payload == INT8_P2P)
    reduce_kernel<W, INT8_P2P><<<blocks, THREADS, 0, st>>>(a);
  else if (payload == FP16_NVLS)
    reduce_kernel<W, FP16_NVLS><<<blocks, THREADS, 0, st>>>(a);
  else if (payload == FP16_PUSHED)
    reduce_kernel<W, FP16_PUSHED><<<blocks, THREADS, 0, st>>>(a);
  else
    reduce_kernel<W, FP16_P2P><<<blocks, THREADS, 0, st>>>(a);
  return cudaGetLastError();
}

int run(const void* const* bases, const void* mc, int world, int rank, int64_t flags_off,
        int64_t partial_off, int64_t final_off, int64_t rows, int64_t width, int shift,
        const float* row_scale, const float* weight_scale, void* residual_f16, const float* gate,
        int64_t gate_rows, const int32_t* labels, uint32_t epoch, bool gather, int payload,
        void* stream, int64_t own_off = -1, bool final_local = false) {
  const bool packed = payload == INT8_P2P;
  if (payload == FP16_NVLS && (mc == nullptr || !h3host::aligned(mc, 16))) return H3_ERR_INVALID;
  if (bases == nullptr || residual_f16 == nullptr || (world != 2 && world != 4 && world != 8) ||
      rank < 0 || rank >= world || rows < 0 || width <= 0 || width % 8 || epoch == 0 ||
      flags_off < 0 || partial_off < 0 || final_off < 0 || flags_off % 16 ||
      partial_off % 16 || final_off % 16 || !h3host::aligned(residual_f16, 16))
    return H3_ERR_INVALID;
  if (!gather) {
    if (row_scale == nullptr || weight_scale == nullptr || shift < 0 || shift > 60 ||
        !h3host::aligned(weight_scale, 16))
      return H3_ERR_INVALID;
    if (gate != nullptr &&
        (gate_rows < 1 || (labels == nullptr && gate_rows != 1) || !h3host::aligned(gate, 16)))
      return H3_ERR_INVALID;
    if (packed && width % 128 != 0) return H3_ERR_INVALID;
  }
  Args a{};
  a.mc = reinterpret_cast<uint64_t>(mc);
  for (int w = 0; w < world; ++w) {
    if (bases[w] == nullptr || !h3host::aligned(bases[w], 16)) return H3_ERR_INVALID;
    a.bases[w] = reinterpret_cast<uint64_t>(bases[w]);
  }
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(residual_f16, &dev)) return s;
  a.flags_off = flags_off;
  a.partial_off = partial_off;
  a.final_off = final_off;
  a.world = world;
  a.rank = rank;
  a.rows = rows;
  a.width = width;
  a.per = rows ? (rows + world - 1) / world : 1;
  a.row_begin = std::min<int64_t>(rows, rank * a.per);
  a.row_end = std::min<int64_t>(rows, (rank + 1) * a.per);
  a.up = ldexpf(1.0f, shift);
  a.row_scale = row_scale;
  a.weight_scale = weight_scale;
  a.residual = reinterpret_cast<__half*>(residual_f16);
  a.gate = gate;
  a.gate_rows = gate_rows;
  a.labels = labels;
  a.epoch = epoch;
  // own rows: slot `rank` of the owner-routed layout unless given
  a.own_off = own_off >= 0 ? own_off : partial_off + rank * a.per * (width / 8) * 16;
  a.final_local = final_local ? 1 : 0;
  if (own_off >= 0 && own_off % 16 != 0) return H3_ERR_INVALID;
  a.err = h3host::error_word(dev);
  if (a.err == nullptr) return H3_ERR_CUDA;
  // Enough CTAs to keep every SM's load slots busy; the flags make any grid size safe
  // (no CTA waits for another CTA of the same launch).
  const int64_t items = (gather ? rows - (a.row_end - a.row_begin) : a.row_end - a.row_begin) *
                        (width / 8);
  const int blocks = (int)std::max<int64_t>(
      1, std::min<int64_t>((items + THREADS - 1) / THREADS, (int64_t)h3host::sm_count(dev) * 16));
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = world == 2 ? launch<2>(a, blocks, gather, payload, dev, st)
                  : world == 4 ? launch<4>(a, blocks, gather, payload, dev, st)
                               : launch<8>(a, blocks, gather, payload, dev, st);
  return e == cudaSuccess ? H3_OK : H3_ERR_CUDA;
}

}  // namespace peer
}  // namespace h3

namespace h3 {
namespace peer {
// One warp: optionally stores `epoch` into flag `region`[rank] of every rank, then waits
// (bounded) until this rank's flags region[w] >= epoch for every other rank w.  Orders
// the copy-engine pulls of the dma exchange after the peers' matching kernels.
__global__ void signal_kernel(const Args a, int64_t region, int publish) {
  if (publish && (int)threadIdx.x < a.world) {
    __threadfence_system();
    store_release(flag(a, threadIdx.x, region, a.rank), a.epoch);
  }
  if (!wait_all(a, region, true) && threadIdx.x == 0) report_error(a.err, H3_ERR_TIMEOUT);
}
}  // namespace peer
}  // namespace h3

extern "C" int h3_peer_signal(const void* const* bases, int world, int rank, int64_t flags_off,
                              int which, uint32_t epoch, int publish, void* stream) {
  if (bases == nullptr || (world != 2 && world != 4 && world != 8) || rank < 0 ||
      rank >= world || epoch == 0 || flags_off < 0 || flags_off % 16 || (which != 0 && which != 1))
    return H3_ERR_INVALID;
  h3::peer::Args a{};
  for (int w = 0; w < world; ++w) {
    if (bases[w] == nullptr || !h3host::aligned(bases[w], 16)) return H3_ERR_INVALID;
    a.bases[w] = reinterpret_cast<uint64_t>(bases[w]);
  }
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(bases[rank], &dev)) return s;
  a.flags_off = flags_off;
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  a.err = h3host::error_word(dev);
  if (a.err == nullptr) return H3_ERR_CUDA;
  h3::peer::signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a, which ? h3::peer::DONE : h3::peer::READY,
                                                             publish);
  return h3host::check_launch();
}

extern "C" int h3_peer_reduce_staged(const void* const* bases, int world, int rank,
                                     int64_t flags_off, int64_t stage_off, int64_t own_off,
                                     int64_t final_off, int64_t rows, int64_t width, int shift,
                                     const float* row_scale, const float* weight_scale,
                                     void* residual_f16, const float* gate, int64_t gate_rows,
                                     const int32_t* labels, uint32_t epoch, void* stream) {
  if (own_off < 0) return H3_ERR_INVALID;
  return h3::peer::run(bases, nullptr, world, rank, flags_off, stage_off, final_off, rows, width,
                       shift, row_scale, weight_scale, residual_f16, gate, gate_rows, labels,
                       epoch, false, h3::peer::FP16_PUSHED, stream, own_off, true);
}

extern "C" int h3_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (dst == nullptr || src == nullptr || bytes < 0) return H3_ERR_INVALID;
  if (bytes == 0) return H3_OK;
  return cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice,
                         (cudaStream_t)stream) == cudaSuccess ? H3_OK : H3_ERR_CUDA;
}

extern "C" int h3_peer_reduce(const void* const* bases, int world, int rank, int64_t flags_off,
                              int64_t partial_off, int64_t final_off, int64_t rows,
                              int64_t width, int shift, const float* row_scale,
                              const float* weight_scale, void* residual_f16, const float* gate,
                              int64_t gate_rows, const int32_t* labels, uint32_t epoch,
                              void* stream) {
  return h3::peer::run(bases, nullptr, world, rank, flags_off, partial_off, final_off, rows,
                       width, shift, row_scale, weight_scale, residual_f16, gate, gate_rows,
                       labels, epoch, false, h3::peer::FP16_P2P, stream);
}

extern "C" int h3_peer_reduce_pushed(const void* const* bases, int world, int rank,
                                     int64_t flags_off, int64_t partial_off, int64_t final_off,
                                     int64_t rows, int64_t width, int shift,
                                     const float* row_scale, const float* weight_scale,
                                     void* residual_f16, const float* gate, int64_t gate_rows,
                                     const int32_t* labels, uint32_t epoch, void* stream) {
  return h3::peer::run(bases, nullptr, world, rank, flags_off, partial_off, final_off, rows,
                       width, shift, row_scale, weight_scale, residual_f16, gate, gate_rows,
                       labels, epoch, false, h3::peer::FP16_PUSHED, stream);
}

extern "C" int h3_peer_reduce_nvls(const void* const* bases, const void* multicast, int world,
                                   int rank, int64_t flags_off, int64_t partial_off,
                                   int64_t final_off, int64_t rows, int64_t width, int shift,
                                   const float* row_scale, const float* weight_scale,
                                   void* residual_f16, const float* gate, int64_t gate_rows,
                                   const int32_t* labels, uint32_t epoch, void* stream) {
  return h3::peer::run(bases, multicast, world, rank, flags_off, partial_off, final_off, rows,
                       width, shift, row_scale, weight_scale, residual_f16, gate, gate_rows,
                       labels, epoch, false, h3::peer::FP16_NVLS, stream);
}

extern "C" int h3_peer_reduce_int8(const void* const* bases, int world, int rank,
                                   int64_t flags_off, int64_t partial_off, int64_t final_off,
                                   int64_t rows, int64_t width, const float* row_scale,
                                   const float* weight_scale, void* residual_f16,
                                   const float* gate, int64_t gate_rows, const int32_t* labels,
                                   uint32_t epoch, void* stream) {
  return h3::peer::run(bases, nullptr, world, rank, flags_off, partial_off, final_off, rows,
                       width, 0, row_scale, weight_scale, residual_f16, gate, gate_rows, labels,
                       epoch, false, h3::peer::INT8_P2P, stream);
}

extern "C" int h3_peer_gather(const void* const* bases, int world, int rank, int64_t flags_off,
                              int64_t final_off, int64_t rows, int64_t width, void* residual_f16,
                              uint32_t epoch, void* stream) {
  return h3::peer::run(bases, nullptr, world, rank, flags_off, 0, final_off, rows, width, 0,
                       nullptr, nullptr, residual_f16, nullptr, 0, nullptr, epoch, true,
                       h3::peer::FP16_P2P, stream);
}
