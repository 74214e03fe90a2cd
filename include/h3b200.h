/*
 * h3b200.h - C ABI of the B200-native (sm_100a) tensor-parallel W8A8 INT8 linear path.
 *
 * Every entry point takes raw device pointers, element counts and a cudaStream_t
 * (passed as void*), enqueues its kernels on that stream and returns an int status
 * (H3_OK or an H3_ERR_* code).  It runs on the device that owns its first device
 * pointer and leaves the calling thread's current device as it found it.  Nothing
 * here allocates the caller's tensors: outputs are written into caller-provided
 * device buffers, the way the reference's
 * native extension (comfy_kitchen._C.cublas_gemm_int8 / dequantize_int8_linear,
 * called from patches/optimized_tp.py:34-43 and patches/parallel_int8.py:53-65)
 * receives DLPack tensors plus a raw stream.  Geometry is checked before any launch
 * and rejected with H3_ERR_INVALID, the way the reference raises ValueError before
 * either rank enters a collective (patches/tilelang_swiglu_quant.py:95-105).
 *
 * Conventions
 *   - fp16 buffers are IEEE binary16 (torch.float16), passed as void*.
 *   - Matrices are row-major and contiguous unless a stride argument says otherwise.
 *   - int8 weight matrices are [N, K] (output channel major), as in the pre-baked
 *     rank shards of patches/rank_local_int8.py:62-80.
 *   - K (the reduction length) must be a multiple of 16 for the GEMMs, and widths
 *     fed to the ConvRot256 kernels a multiple of 256.
 */
#ifndef H3B200_H
#define H3B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  H3_OK = 0,
  H3_ERR_INVALID = 1,     /* unsupported geometry, null or misaligned pointer       */
  H3_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed                    */
  H3_ERR_TIMEOUT = 3,     /* a bounded device-side wait gave up (see h3_device_error) */
  H3_ERR_UNSUPPORTED = 4  /* the device is not an sm_100 part                         */
};

/* FC2 producer input layouts */
enum {
  H3_IN_GATEUP_F16 = 0, /* fp16 [rows, 2*width] = [gate_r | up_r] (FC1 column output) */
  H3_IN_ACT_F32 = 1,    /* fp32 [rows, width] = silu(f16 gate) * f16 up, pre-computed  */
  H3_IN_ACT_F16 = 2     /* fp16 [rows, width] post-SwiGLU activation                    */
};

/* Quantizer division (patches/tilelang_row_quant.py:27,40) */
enum { H3_DIV_RN = 0, H3_DIV_FAST = 1 };

/* Output kinds */
enum {
  H3_OUT_F32 = 0,      /* fp32 store                                                   */
  H3_OUT_F16 = 1,      /* fp16 store (round to nearest even)                           */
  H3_OUT_RESIDUAL = 2, /* gated residual update in place: X = f16(fma(f16(y), G, X))    */
  H3_OUT_I32 = 3       /* h3_unpack8_finish only: the restored INT32 sum, no dequant    */
};

/* ----------------------------------------------------------------------------
 * Library / device status
 * ------------------------------------------------------------------------- */
int h3_abi_version(void);
const char* h3_status_string(int status);
/* Reads, then clears, the device-side error word that bounded waits set when
 * they give up.  Synchronises the device (not during stream capture).  *code = 0
 * when nothing failed. */
int h3_device_error(int device, int* code);
/* The same word as it stands, without synchronising or clearing: the word lives in
 * host-mapped page-locked memory that kernels write with a system-scope store, so the
 * host can poll it once per operator call at no device cost.  *code = 0 when nothing
 * has failed (or nothing has run yet on that device). */
int h3_device_error_peek(int device, int* code);
/* Measurement aid (no reference counterpart): one 32-thread CTA that sleeps for `ns`
 * nanoseconds (<= 10 s) and writes out[0] = elapsed ns of %globaltimer, out[1] = SM
 * cycles of %clock64 over the same interval (out: 2 x u64 in device memory).  Launched
 * on a second stream beside other kernels, out[1] / out[0] is the SM clock they ran at. */
int h3_sm_clock_probe(unsigned long long ns, unsigned long long* out, void* stream);

/* ----------------------------------------------------------------------------
 * Column path (QKV / FC1): ColumnParallelLinearINT8.forward, tp_dit.py:69-96
 * ------------------------------------------------------------------------- */

/* Activation preparation of column_linear: optional regular ConvRot256 rotation
 * (rotated = f16(H256 x)), then per-row INT8 quantisation with
 * scale = max(amax * f32(1/127), 1e-30), q = clamp(rint(x / scale), -128, 127).
 * Replaces dit_column_linear.py:13-21 (_prepare_activation: Kitchen eager
 * _rotate_activation + quantize_int8_rowwise).
 *   x_f16 [rows, k], q [rows, k], scale [rows].  convrot: 1 = rotate, 0 = none. */
int h3_column_quantize(const void* x_f16, int64_t rows, int64_t k, int convrot,
                       int8_t* q, float* scale, void* stream);

/* The column input producer with the modulated RMSNorm in front (fused version of
 * tilelang_dit_fusion.py:11-37 -> h3_column_quantize; h3_tensor_flow.py:134-143):
 *   ss = sum_i f32(x_i)^2 (fixed order), inv = RN(1/sqrt(ss *rn f32(1/width) +rn eps)),
 *   h_i = f16( (((f32(x_i) *rn inv) *rn W_i) *rn (1 +rn scale[l][i])) +rn shift[l][i] ),
 * l = labels[row] (labels may be NULL when mod_rows == 1); then h goes through the
 * column quantiser (ConvRot256 when convrot, f16 rounding, row scale, codes) without
 * being stored.  q / row_scale may both be NULL to produce only h; h_f16 (fp16
 * [rows, width]) may be NULL when quantising.  The reference's own kernel calls the
 * approximate rsqrtf; this one is correctly rounded. */
int h3_modulated_norm_quantize(const void* x_f16, int64_t rows, int64_t width,
                               const float* norm_weight, float eps, const float* shift,
                               const float* scale, int64_t mod_rows, const int32_t* labels,
                               int convrot, int8_t* q, float* row_scale, void* h_f16,
                               void* stream);

/* Direct INT8 GEMM, INT32 out: out[m, n] = sum_k q[m, k] * w[n, k], exact.
 * Replaces optimized_tp.py:34-43 (native_int_mm) and parallel_int8.py:46-50. */
int h3_int8_gemm_i32(const int8_t* q, const int8_t* w, int64_t m, int64_t n, int64_t k,
                     int32_t* out, void* stream);

/* INT8 GEMM with the ordered column dequant epilogue fused:
 *   y[m, n] = f16( (f32(acc) *rn (row_scale[m] *rn weight_scale[n])) [+rn bias[n]] )
 * Replaces dit_column_linear.py:138-149 (native_int_mm followed by
 * tilelang_column_epilogue.py:11-40).  weight_scale_len is 1 (scalar) or n.
 * bias may be NULL. */
int h3_int8_gemm_column(const int8_t* q, const int8_t* w, int64_t m, int64_t n, int64_t k,
                        const float* row_scale, const float* weight_scale,
                        int64_t weight_scale_len, const float* bias, void* out_f16,
                        void* stream);

/* FC1 with the FP32 SwiGLU epilogue fused.  w is the component-packed rank shard
 * [gate_r | up_r] of n_packed rows (patches/rank_local_int8.py:66-75); the output
 * has n_packed/2 columns:
 *   g = f16(col_dequant(gate)), u = f16(col_dequant(up)),
 *   y = (g /rn (1 +rn exp(-g))) *rn u    (tilelang_swiglu_quant.py:21-24)
 * out_kind H3_OUT_F32 stores y (same bytes as the fp16 [gate|up] store it
 * replaces, tp_dit.py:356); H3_OUT_F16 stores f16(y).  bias ([n_packed]) may be NULL. */
int h3_int8_gemm_swiglu(const int8_t* q, const int8_t* w, int64_t m, int64_t n_packed,
                        int64_t k, const float* row_scale, const float* weight_scale,
                        const float* bias, int out_kind, void* out, void* stream);

/* Standalone ordered column epilogue (tilelang_column_epilogue.py:11-40):
 *   y = f16(f32(acc) *rn (row_scale[m] *rn weight_scale[n])) */
int h3_column_dequantize(const int32_t* acc, int64_t rows, int64_t width,
                         const float* row_scale, const float* weight_scale,
                         int64_t weight_scale_len, void* out_f16, void* stream);

/* ----------------------------------------------------------------------------
 * FC2 `fused_stored` producer: tilelang_swiglu_quant.py:12-92
 * ------------------------------------------------------------------------- */

/* Phase 'stored' (rotated != NULL) or 'maximum' (rotated == NULL) of fused_kernel
 * (tilelang_swiglu_quant.py:37-51) with the group maxima already reduced to one
 * maximum per row (prepare, :86).  x per input_kind; rotated fp32 [rows, width];
 * row_max [rows] = max |rotated| over the local row. */
int h3_swiglu_rotate_max(const void* x, int input_kind, int64_t rows, int64_t width,
                         float* rotated, float* row_max, void* stream);

/* Phase 'recompute' (tilelang_swiglu_quant.py:52-64): recompute the rotated values
 * from x and quantise them with the (globally reduced) row_max using the quantizer
 * of tilelang_row_quant.py:27-46.  q [rows, width], scale [rows]. */
int h3_swiglu_rotate_quantize(const void* x, int input_kind, int64_t rows, int64_t width,
                              const float* row_max, int division, int8_t* q, float* scale,
                              void* stream);

/* TP=1 single pass: rotation, row maximum and quantisation of a whole row in one
 * kernel (no collective in between).  Writes q, scale and row_max. */
int h3_swiglu_rotate_quantize_local(const void* x, int input_kind, int64_t rows,
                                    int64_t width, int division, int8_t* q, float* scale,
                                    float* row_max, void* stream);

/* Row quantizer with an external (reduced) maximum: tilelang_row_quant.py:27-46.
 * Reads rotated[r, start + c] for c < width, row pitch `stride` floats. */
int h3_row_quantize(const float* rotated, int64_t rows, int64_t width, int64_t stride,
                    int64_t start, const float* row_max, int division, int8_t* q,
                    float* scale, void* stream);

/* ----------------------------------------------------------------------------
 * Row path (O / FC2): RowParallelLinearINT8.forward, tp_dit.py:141-162
 * ------------------------------------------------------------------------- */

/* Power-of-two transport shift for a full (all-rank) reduction length full_k:
 * max(0, ceil(log2(full_k * 127 * 127 / 60000))).  Equals the reference's
 * shift_for(local_k) (tilelang_transport_tradeoffs.py:20-22) at TP2, where
 * full_k = 2 * local_k. */
int h3_transport_shift(int64_t full_k);

/* INT8 GEMM with the scaled-FP16 encode fused (parallel_int8.int_mm followed by
 * tilelang_transport_tradeoffs.py:26-39 encode):  y = f16(f32(acc) *rn 2^-shift) */
int h3_int8_gemm_row_encode(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                            int64_t k, int shift, void* out_f16, void* stream);

/* TP=1 row GEMM with the dequant fused (exact INT32, no transport):
 *   y = (f32(acc) *rn row_scale[m]) *rn weight_scale[n]   (parallel_int8.py:66)
 * out_kind F32/F16 store y into out; H3_OUT_RESIDUAL updates residual_f16 in place
 * with X = f16(fma(f32(f16(y)), G[labels[m], n], f32(X))) (tilelang_dit_fusion.py:
 * 57-77); gate == NULL means G = 1.  labels may be NULL when gate_rows == 1. */
int h3_int8_gemm_row_dequant(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                             int64_t k, const float* row_scale, const float* weight_scale,
                             int out_kind, void* out, void* residual_f16, const float* gate,
                             int64_t gate_rows, const int32_t* labels, void* stream);

/* Scaled-FP16 codec (tilelang_transport_tradeoffs.py:26-39):
 *   encode y = f16(f32(p) *rn 2^-shift);   decode p = (int32)(f32(y) *rn 2^shift) */
int h3_fp16_encode(const int32_t* partial, int64_t n, int shift, void* out_f16,
                   void* stream);
int h3_fp16_decode(const void* payload_f16, int64_t n, int shift, int32_t* out,
                   void* stream);

/* Fixed-order partial reduction + fused epilogue (tilelang_transport_p2.py:15-47 and
 * tilelang_dit_fusion.py:57-77), for the rows this rank owns:
 *   t = f16( f32(P_0) + f32(P_1) + ... + f32(P_{world-1}) )   (fp32 sum, rank order)
 *   restored = (int32) trunc(f32(t) *rn 2^shift)
 *   y = (f32(restored) *rn row_scale[m]) *rn weight_scale[n]
 * then stored per out_kind as in h3_int8_gemm_row_dequant.  parts_f16 holds `world`
 * fp16 [rows, width] blocks, part_stride elements apart.  At world == 2 the sum is
 * the single RN fp16 addition of NCCL's fp16 SUM; world == 1 is the reference's
 * epilogue / row_gate_kernel applied to an already reduced payload. */
int h3_row_reduce_finish(const void* parts_f16, int world, int64_t part_stride,
                         int64_t rows, int64_t width, int shift, const float* row_scale,
                         const float* weight_scale, int out_kind, void* out,
                         void* residual_f16, const float* gate, int64_t gate_rows,
                         const int32_t* labels, void* stream);

/* INT32 dequantisation of parallel_int8.dequantize (parallel_int8.py:53-69):
 *   y = ((f32(acc) *rn row_scale[m]) *rn weight_scale[n]) [+rn bias[n]]
 * stored as out_kind F32 or F16. */
int h3_dequantize_i32(const int32_t* acc, int64_t rows, int64_t width,
                      const float* row_scale, const float* weight_scale,
                      int64_t weight_scale_len, const float* bias, int out_kind, void* out,
                      void* stream);

/* Gated residual add (tilelang_dit_fusion.py:39-53, the gate_kernel of gated_add):
 *   X[m, n] = f16( fma(f32(f16(branch[m, n])), G[labels[m], n], f32(X[m, n])) )
 * branch is fp32 (branch_kind H3_OUT_F32, rounded to fp16 first, as the row output's
 * .to(fp16) does) or fp16 (H3_OUT_F16).  gate == NULL means G = 1 (plain fp16
 * residual add); labels may be NULL when gate_rows == 1. */
int h3_gated_add(const void* branch, int branch_kind, int64_t rows, int64_t width,
                 void* residual_f16, const float* gate, int64_t gate_rows,
                 const int32_t* labels, void* stream);

/* ----------------------------------------------------------------------------
 * Packed INT8 transport, the reference's 'int8_gather' scheme
 * (tilelang_transport_tradeoffs.py:40-88, tilelang_transport_p2.py:28-42, torch
 * statement benchmarks/tp2_tradeoffs.py:73-78).  Payload of a [rows, width] INT32
 * partial (width % 128 == 0): uint8 [rows, width/128 * 132]; per 128-column group
 * 128 codes then the 4 bytes of the fp32 scale:
 *   scale = max(max|f32(P)| *rn f32(1/127), f32(1e-8)),
 *   q = clamp(rint(f32(P) /rn scale), -127, 127)
 * Reconstruction over `world` payloads, in rank order:
 *   restored = rint( f32(q_0) *rn s_0 +rn f32(q_1) *rn s_1 +rn ... )
 * ------------------------------------------------------------------------- */

/* INT8 GEMM with the pack fused into the epilogue (int_mm + pack_int8). */
int h3_int8_gemm_row_pack8(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                           int64_t k, void* out_u8, void* stream);
/* Standalone pack of an INT32 partial (pack_int8). */
int h3_pack8(const int32_t* partial, int64_t rows, int64_t width, void* out_u8, void* stream);
/* Reconstruction of `world` payloads (part_stride bytes apart) + the row epilogue
 * y = (f32(restored) *rn row_scale[m]) *rn weight_scale[n], stored per out_kind as in
 * h3_row_reduce_finish; out_kind H3_OUT_I32 stores the restored INT32 (unpack_int8). */
int h3_unpack8_finish(const void* parts_u8, int world, int64_t part_stride, int64_t rows,
                      int64_t width, const float* row_scale, const float* weight_scale,
                      int out_kind, void* out, void* residual_f16, const float* gate,
                      int64_t gate_rows, const int32_t* labels, void* stream);

/* ----------------------------------------------------------------------------
 * Row transport over NVLink peer memory.  Replaces, for the residual form of the
 * row output, the reference's NCCL fp16 SUM of the encoded partials
 * (tilelang_transport_p2.py:57-58, tilelang_swiglu_quant.py:116-127) and the fused
 * row-gate epilogue that follows it (tilelang_dit_fusion.py:57-77, 146-151), with the
 * same arithmetic as h3_row_reduce_finish(out_kind = H3_OUT_RESIDUAL).
 *
 * bases[w] (w < world, world in {2, 4, 8}) is rank w's workspace buffer mapped into
 * this process (every rank's buffer has the same layout; the caller maps them, e.g.
 * with torch symmetric memory).  Rank r owns rows [r*per, min(rows, (r+1)*per)),
 * per = ceil(rows / world).  Layout of each buffer:
 *   flags_off    1024 bytes of u32 flags, zeroed on every rank before the first call
 *   partial_off  fp16 [rows][width]: that rank's partial (h3_int8_gemm_row_encode)
 *   final_off    fp16 [rows][width]: the other ranks' finished rows
 * One call, on one stream, the same `epoch` (1, 2, 3, ... per call) on every rank:
 *   h3_peer_reduce  loads the owned rows of every rank's partial (NVLink loads), fixed
 *       rank-order reduction, decode, dequant and gated residual update of those rows
 *       of residual_f16, also stored into every peer's final area (NVLink stores);
 *   h3_peer_gather  copies the peers' finished rows into residual_f16.
 * Waits for peers are bounded (2 s); a wait that gives up leaves H3_ERR_TIMEOUT in
 * h3_device_error and the workspace must be re-created.  width % 8 == 0; pointers
 * 16-byte aligned. */
int h3_peer_reduce(const void* const* bases, int world, int rank, int64_t flags_off,
                   int64_t partial_off, int64_t final_off, int64_t rows, int64_t width,
                   int shift, const float* row_scale, const float* weight_scale,
                   void* residual_f16, const float* gate, int64_t gate_rows,
                   const int32_t* labels, uint32_t epoch, void* stream);
/* h3_peer_reduce with the reduction done in the NVSwitch (NVLS): `multicast` is the
 * multicast address of the same workspace buffers (an NVLS multicast object bound to
 * every rank's buffer, e.g. torch symmetric memory's multicast_ptr).  Each 16-byte
 * chunk of the owned rows is read with one multimem.ld_reduce (the switch sums the
 * `world` fp16 partials, fp32 accumulation, one fp16 rounding) and each finished chunk is
 * stored into every rank's final area with one multimem.st; the epilogue, flags and
 * h3_peer_gather are those of h3_peer_reduce.  Bit-identical to h3_peer_reduce at
 * world 2; at world 4 and 8 the switch's summation order is its own (rare last-bit
 * differences of the fp16 sum where the fp32 partial sums are inexact). */
/* The reduce-scatter fused into the row GEMM: h3_int8_gemm_row_encode whose output row
 * r (owner o = r / per) is stored straight into rank o's buffer (NVLink stores from the
 * GEMM epilogue, overlapping its tensor work) at partial_off, slot row rank * per +
 * (r - o * per), so that each owner's partial area holds [world][per][n]: every rank's
 * rows of its block.  The area must hold world * per rows.  bases / world / rank as for
 * h3_peer_reduce; n % 8 == 0. */
int h3_int8_gemm_row_encode_push(const int8_t* q, const int8_t* w, int64_t m, int64_t n,
                                 int64_t k, int shift, const void* const* bases, int world,
                                 int rank, int64_t partial_off, void* stream);
/* h3_peer_reduce after h3_int8_gemm_row_encode_push: the owned rows' partials are
 * already in this rank's buffer (slot w = rank w), so the reduce reads local memory
 * only; the same rank-order sum, epilogue, final-row stores into every peer, flags and
 * h3_peer_gather.  Same bits as h3_peer_reduce. */
int h3_peer_reduce_pushed(const void* const* bases, int world, int rank, int64_t flags_off,
                          int64_t partial_off, int64_t final_off, int64_t rows, int64_t width,
                          int shift, const float* row_scale, const float* weight_scale,
                          void* residual_f16, const float* gate, int64_t gate_rows,
                          const int32_t* labels, uint32_t epoch, void* stream);
/* The copy-engine ("dma") form of the exchange, four steps on one stream per rank:
 *   1. h3_peer_signal(which = 0, publish = 1): this rank's partial (h3_int8_gemm_row_encode
 *      at partial_off) is complete; wait (bounded) until every rank's is;
 *   2. h3_copy_async per peer w: rank w's rows of this rank's block, from w's partial area,
 *      into slot w of this rank's staging area at stage_off ([world][per][width] fp16);
 *   3. h3_peer_reduce_staged: the rank-order reduce + epilogue of the block from the
 *      staging slots (this rank's own rows read in place at own_off), the finished rows
 *      stored into this rank's own final area, then done published to every rank;
 *   4. h3_peer_signal(which = 1, publish = 0): wait (bounded) for every peer's done, then
 *      h3_copy_async per peer: its finished rows from its final area into residual_f16.
 * Copies between GPUs go through the copy engines (cudaMemcpyAsync), which carry NVLink
 * traffic faster than loads and stores issued by the SMs.  Same bits as h3_peer_reduce.
 * A wait that gives up records H3_ERR_TIMEOUT; the copies that follow it then move
 * whatever the buffers hold, and the error word says so. */
int h3_peer_signal(const void* const* bases, int world, int rank, int64_t flags_off, int which,
                   uint32_t epoch, int publish, void* stream);
int h3_peer_reduce_staged(const void* const* bases, int world, int rank, int64_t flags_off,
                          int64_t stage_off, int64_t own_off, int64_t final_off, int64_t rows,
                          int64_t width, int shift, const float* row_scale,
                          const float* weight_scale, void* residual_f16, const float* gate,
                          int64_t gate_rows, const int32_t* labels, uint32_t epoch,
                          void* stream);
/* cudaMemcpyAsync device to device (either side may be a peer's mapped buffer). */
int h3_copy_async(void* dst, const void* src, int64_t bytes, void* stream);
int h3_peer_reduce_nvls(const void* const* bases, const void* multicast, int world, int rank,
                        int64_t flags_off, int64_t partial_off, int64_t final_off, int64_t rows,
                        int64_t width, int shift, const float* row_scale,
                        const float* weight_scale, void* residual_f16, const float* gate,
                        int64_t gate_rows, const int32_t* labels, uint32_t epoch, void* stream);
/* h3_peer_reduce for packed INT8 payloads (h3_int8_gemm_row_pack8 output at
 * partial_off): restored = rint(rank-order sum of f32(q_w) *rn s_w), then the same
 * epilogue, final-row stores and flags.  width % 128 == 0. */
int h3_peer_reduce_int8(const void* const* bases, int world, int rank, int64_t flags_off,
                        int64_t partial_off, int64_t final_off, int64_t rows, int64_t width,
                        const float* row_scale, const float* weight_scale, void* residual_f16,
                        const float* gate, int64_t gate_rows, const int32_t* labels,
                        uint32_t epoch, void* stream);
int h3_peer_gather(const void* const* bases, int world, int rank, int64_t flags_off,
                   int64_t final_off, int64_t rows, int64_t width, void* residual_f16,
                   uint32_t epoch, void* stream);

/* TP>1 producer in one pass: h3_swiglu_rotate_max + the NCCL MAX all-reduce of the row
 * maxima (tilelang_swiglu_quant.py:86-87) + h3_swiglu_rotate_quantize, with the row
 * maxima exchanged over peer memory inside the kernel.  bases/world/rank as above;
 * at slots_off every buffer holds u64 slots [rows][world] (zeroed before the first
 * call, a region of their own: not the partial or final area); epoch (1, 2, 3, ...
 * per call, the same on every rank) tags each slot.  The kernel runs a persistent
 * grid; every rank must launch it for the same rows and width, and no kernel that
 * waits for other ranks (a collective of another communicator) may run beside it on
 * any rank: its CTAs could keep one of ours from becoming resident, the rule NCCL
 * states for concurrent communicators.  Waits are bounded (2 s per CTA in total); a
 * wait that gives up uses the local maximum and leaves H3_ERR_TIMEOUT in
 * h3_device_error.  row_max (optional) receives the global maxima.  width up to
 * H3_PEER_PRODUCER_MAX_WIDTH (a row of each CTA is staged in shared memory). */
#define H3_PEER_PRODUCER_MAX_WIDTH 16384
int h3_swiglu_rotate_quantize_peer(const void* x, int input_kind, int64_t rows,
                                   int64_t width, const void* const* bases, int world,
                                   int rank, int64_t slots_off, uint32_t epoch, int division,
                                   int8_t* q, float* scale, float* row_max, void* stream);

/* ----------------------------------------------------------------------------
 * Column linear without allocation.  No counterpart in the reference: added for
 * callers that may not allocate device memory (runtimes that budget all device
 * memory through their own pool, paths that cannot afford cudaMalloc's implicit
 * device synchronisation).
 * ------------------------------------------------------------------------- */

/* Bytes of the file-scope static __device__ scratch array that every GPU loading
 * this library holds until the process exits. */
#define H3_NOALLOC_SCRATCH_BYTES (32u << 20)

/* The column path of h3_column_quantize followed by h3_int8_gemm_column in one call
 * that allocates nothing: the INT8 codes, the row scales and the error word live in
 * the static scratch array.  Requires 256 + roundup256(4*m) + m*k <=
 * H3_NOALLOC_SCRATCH_BYTES (e.g. m*k up to ~32 MiB) and returns H3_ERR_INVALID,
 * launching nothing, beyond that.  The first call on a device looks the array's
 * device address up (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls on a device share the array: calls whose GPU work overlaps race
 * and must be serialised by the caller (one stream, or events).
 * h3_column_linear_noalloc_error reads (without clearing) the error word of the last
 * call; the next call clears it.  It synchronises the device, so it must not be called
 * while a stream of that device is being captured. */
int h3_column_linear_noalloc(const void* x_f16, int64_t m, int64_t k, int convrot,
                             const int8_t* w, int64_t n, const float* weight_scale,
                             int64_t weight_scale_len, const float* bias, void* out_f16,
                             void* stream);
int h3_column_linear_noalloc_error(int device, int* code);

/* ----------------------------------------------------------------------------
 * Diagnostics
 * ------------------------------------------------------------------------- */

/* Evaluates the library's exponential (h3_expf) and CUDA's expf on n inputs:
 * ours[i] = h3_expf(x[i]), cuda[i] = expf(x[i]).  Used to measure how often the
 * oracle-pinned exponential differs from the one the reference calls. */
int h3_expf_compare(const float* x, int64_t n, float* ours, float* cuda, void* stream);

/* Evaluates silu(g) = g / (1 + exp(-g)) three ways: fast[i] as the kernels compute it
 * (h3_expf and a branch-free division of the library's own: reciprocal and
 * Markstein's quotient correction; FLT_MAX where its scalar form and its packed-pair
 * form, the one the FC1 epilogue runs, disagree), ieee[i] with h3_expf and the IEEE
 * division (the two must agree bit for bit on every fp16 g), and cuda[i] (may be
 * NULL) with CUDA's expf, the reference's form (tilelang_swiglu_quant.py:22-23). */
int h3_silu_compare(const float* g, int64_t n, float* fast, float* ieee, float* cuda,
                    void* stream);

/* INT8 codes of x[i] / scale[i] two ways: fast[i] as the kernels compute them
 * (one correctly rounded reciprocal per scale, a Markstein quotient correction and
 * magic-number rounding), ieee[i] with IEEE division, rintf and a float-to-int
 * conversion (tilelang_row_quant.py:40-44, division 'rn').  They must agree. */
int h3_quant_compare(const float* x, const float* scale, int64_t n, int8_t* fast,
                     int8_t* ieee, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B200_H */
