/*
 * iron_b200.h -- C ABI of libiron_b200.so, the B200 (sm_100a) kernels behind the
 * IRON operator classes.
 *
 * Conventions (every entry point):
 *   - Returns an int status: IRON_OK (0) or a negative iron_status_t. Never throws,
 *     never aborts, never prints. iron_strerror() names a status.
 *   - All tensors are device pointers owned by the caller. bf16 values travel as
 *     uint16_t bit patterns. Shapes are element counts; strides are element counts.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy default
 *     stream. Work is enqueued asynchronously; the call returns after launch.
 *   - Arguments are validated on the host before any launch (null pointers,
 *     shapes, 16-byte alignment where the kernel uses vector loads). A CUDA launch
 *     failure is reported as IRON_ERR_CUDA; iron_last_cuda_error() gives the code.
 *   - The library keeps no state beyond a per-device attribute cache; distinct
 *     streams may be used from distinct threads.
 *   - `flags` bit IRON_FLAG_PDL launches the kernel with programmatic dependent
 *     launch: it may start before the previous kernel on the stream finishes and
 *     streams its weights before waiting for that kernel. Use it only when the
 *     weights are not written by the preceding kernel (inference graphs).
 *
 * Each entry point names the IRON (reference) interface it replaces as
 * file:line within the reference project.
 */
#ifndef IRON_B200_H
#define IRON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  IRON_OK = 0,
  IRON_ERR_NULL = -1,          /* a required pointer is NULL */
  IRON_ERR_SHAPE = -2,         /* a size is <= 0, or sizes are inconsistent */
  IRON_ERR_ALIGN = -3,         /* a pointer or leading dimension is misaligned */
  IRON_ERR_UNSUPPORTED = -4,   /* a valid request this build does not implement */
  IRON_ERR_CUDA = -5,          /* a CUDA runtime call failed */
  IRON_ERR_WORKSPACE = -6,     /* the caller's workspace is too small */
  IRON_ERR_TIMEOUT = -7,       /* a bounded device-side wait gave up */
  IRON_ERR_ARG = -8            /* any other invalid argument */
} iron_status_t;

#define IRON_FLAG_PDL 0x1u
/* iron_gemv_int4g32: SwiGLU epilogue. Each 16-row tile holds 8 gate rows then the
 * 8 matching up rows; y gets N/2 columns: bf16(silu(gate)) * up, IRON's
 * SwiGLUDecode rounding (iron/operators/swiglu_decode/reference.py:49-53). */
#define IRON_FLAG_SWIGLU 0x2u
/* GEMVs (int4 and bf16): x is written by no kernel that can still run while this one does, so
 * it may be read through the read-only (non-coherent) path. Without the flag x is read
 * with L2-coherent loads. With programmatic dependent launch a kernel starts before
 * its predecessors end, so the flag is only for callers that bound their windows: a
 * GEMV that adds a residual lets its dependents launch only after its own wait, and
 * every activation buffer is rewritten only in a later window than its last reader
 * (the Llama decode step and tensor-parallel block: o_proj and down_proj bound each
 * layer's two windows). */
#define IRON_FLAG_X_READONLY 0x4u

/* GEMV epilogues (applied in fp32 to each output before the bf16 store). */
#define IRON_EPI_NONE 0
#define IRON_EPI_GELU 1     /* tanh-approximation GELU */

/* ---- library ------------------------------------------------------------ */

/* Human-readable name of a status code. Never NULL. */
const char *iron_strerror(int status);
/* The cudaError_t of the last IRON_ERR_CUDA on this thread (0 if none). */
int iron_last_cuda_error(void);
/* ABI version: (major << 16) | minor. */
int iron_abi_version(void);

/* ---- GEMV (bf16 weights) --------------------------------------------------
 * Replaces GEMV(M, K, num_batches, epilogue) -- iron/operators/gemv/op.py:22-159,
 * golden iron/operators/gemv/reference.py:9-11 (C = A @ B).
 *   For b in [0, num_batches), v in [0, n_vec):
 *     y[b*y_bstride + v*M + m] = epi( sum_k W[b*w_bstride + m*ldw + k] * x[b*x_bstride + v*K + k] )
 *                                + (residual ? residual[b*y_bstride + v*M + m] : 0)
 *   fp32 accumulation, one bf16 rounding per output. num_batches > 1 is IRON's batched
 *   GEMV (independent matrices); n_vec > 1 is a decode batch sharing one matrix.
 *   W, x rows must start on 16-byte boundaries (ldw, K multiples of 8).
 */
int iron_gemv_bf16(const uint16_t *W, const uint16_t *x, uint16_t *y,
                   int M, int K, int64_t ldw,
                   int num_batches, int64_t w_bstride, int64_t x_bstride,
                   int64_t y_bstride, int n_vec,
                   const uint16_t *residual, int epilogue, unsigned flags,
                   void *stream);

/* ---- int4 group-32 GEMV ---------------------------------------------------
 * The fused Dequant+GEMV of the north star (no single reference op; composes
 * iron/operators/dequant/op.py:20-81 with iron/operators/gemv/op.py:22-159).
 * Logical weights: signed two's-complement int4 q[n,k] in [-8, 7] and one bf16
 * scale per 32 consecutive k of a row; the value is q * scale.
 *
 * Natural layout (what a checkpoint holds):
 *   codes:  uint8 [N, K/2]; element k of row n is nibble (k&1) of byte n*K/2 + k/2
 *           (low nibble = even k).
 *   scales: bf16 [N, K/32].
 * iron_pack_int4g32 repacks both into the GEMV's streaming layout (done once,
 * like IRON's flm.GEMM pack_B, iron/operators/flm/gemm/op.py:455-473):
 * (N/16)*(K/128) units of 1152 bytes, unit (t, c) = rows 16t..16t+15, k 128c..128c+127.
 */
int iron_pack_int4g32(const uint8_t *codes, const uint16_t *scales, uint8_t *packed,
                      int N, int K, void *stream);
/*   y[v, n] = sum_k bf16(q[n,k] * scale[n,k/32]) * x[v,k]  (fp32 accumulate; one
 *             bf16 rounding) + residual[v, n] if residual != NULL -- the dequantized
 *   weights are exactly IRON Dequant's. x: bf16 [n_vec, K]; y: bf16 [n_vec, N]
 *   (N/2 with IRON_FLAG_SWIGLU); K % 128 == 0, N % 16 == 0, 1 <= n_vec <= 64.
 *   Needs no workspace. From 33 vectors on (N % 128 == 0, no fused RMSNorm) the
 *   product runs on the tcgen05 tensor cores (the same dequantized weights, fp32
 *   accumulate, K split over a thread-block cluster and summed in a fixed order); a
 *   bounded wait that runs out there is reported by iron_gemm_status.
 */
/* iron_unpack_int4g32: the packed layout back to bf16 rows out [N, K], each weight
 * bf16(q * scale) exactly (bit-identical to iron_dequant_s4g32_rows on the natural
 * codes); the prefill GEMMs read int4 weights through it. */
int iron_unpack_int4g32(const uint8_t *packed, uint16_t *out, int N, int K, void *stream);
/* iron_gemv_int4g32_ex: iron_gemv_int4g32 plus a fused RMSNorm of x (norm_weight
 * [K], eps; n_vec <= 8, K <= 2048; rmsnorm_kernel's arithmetic, replacing the RMSNorm step
 * before IRON's projections, llama_npu.py:459-480) and a fused greedy argmax
 * (argmax_keys [n_vec * 32] 64-bit keys, zero before the call; iron_argmax_finalize
 * turns them into tokens and re-zeroes them, replacing the argmax sampling of
 * llama_inference_harness.py:146-169). */
int iron_gemv_int4g32_ex(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                         const uint16_t *residual, const uint16_t *norm_weight, float eps,
                         unsigned long long *argmax_keys, unsigned flags, void *stream);
/* iron_l2_prefetch (no reference counterpart): requests [ptr, ptr + bytes) into L2
 * (cp.async.bulk.prefetch.L2 in 64 KB pieces; ptr 16-byte aligned) and returns once
 * the requests are issued. The decode engine runs it on a side branch of its graph so
 * later GEMVs' weights stream in while the chain is latency-bound. */
int iron_l2_prefetch(const void *ptr, size_t bytes, unsigned flags, void *stream);
int iron_argmax_finalize(unsigned long long *keys, int32_t *tokens, int32_t *pos, int B, unsigned flags,
                         void *stream);
/* q4 weights: IRON's asymmetric int4 q4nx values (min + scale * code per group of 32
 * along K, unsigned codes; format of iron/operators/flm/dequant/README.md, values of
 * iron/operators/flm/dequant/reference.py:40-77), replacing flm.DequantBFP followed by
 * the GEMV. iron_pack_q4g32: natural codes [N, K/2] (even k low nibble), bf16 scales and
 * mins [N, K/32] -> 1280-byte streaming units (N % 16 == 0, K % 128 == 0). The GEMV
 * (n_vec <= 8, optional residual as iron_gemv_int4g32) multiplies bf16(min + scale *
 * code) -- IRON's fp32 value rounded once -- with fp32 accumulate; iron_unpack_q4g32
 * writes those bf16 weights [N, K] (for checks). */
int iron_pack_q4g32(const uint8_t *codes, const uint16_t *scales, const uint16_t *mins, uint8_t *packed, int N,
                    int K, void *stream);
int iron_unpack_q4g32(const uint8_t *packed, uint16_t *out, int N, int K, void *stream);
int iron_gemv_q4g32(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                    const uint16_t *residual, unsigned flags, void *stream);
/* iron_gemv_int4g32_chain (no reference counterpart as one call: it folds the weighted
 * RMSNorm steps of IRON's decode runlist, iron/applications/llama_3.2_1b/llama_npu.py:
 * 463-470 and :536, into the GEMVs around them). The int4 GEMV of iron_gemv_int4g32
 * (n_vec <= 8) with the decode chain's extras, all optional (NULL / 0: off):
 *   - residual [n_vec, N]: y = bf16(bf16(W x) + residual) (as iron_gemv_int4g32);
 *   - ss_in [n_vec, K / 16] fp32 with eps (K 2048 or 4096): x holds bf16(h * w) for some
 *     rows h whose per-16-element sums of squares are ss_in; the output is scaled by
 *     inv = 1 / sqrt(sum(ss_in[v]) / K + eps) before rounding (and before SwiGLU), i.e.
 *     y = W . rmsnorm(h) * w up to the rounding of x -- the RMSNorm without its kernel;
 *   - ss_out [n_vec, N / 16], y_weighted [n_vec, N], weight [N] (all three or none): the
 *     producer side -- y_weighted = bf16(y * weight) and the per-16-row sums of squares
 *     of the stored y, the next chained GEMV's x and ss_in;
 *   - argmax_keys [n_vec * 32]: the greedy argmax epilogue (as iron_gemv_int4g32_ex).
 * IRON_FLAG_SWIGLU excludes residual, argmax and the producer side. The partial sums are
 * combined in a fixed order, so results are bitwise reproducible. */
typedef struct {
  const uint16_t *residual;
  const float *ss_in;
  float eps;
  float *ss_out;
  uint16_t *y_weighted;
  const uint16_t *weight;
  unsigned long long *argmax_keys;
} iron_gemv_chain;
int iron_gemv_int4g32_chain(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                            const iron_gemv_chain *c, unsigned flags, void *stream);
/* iron_embed_chain (no reference counterpart as one call: IRON embeds on the CPU,
 * llama_npu.py:1177-1183, and normalises in the runlist): x[b] = table[tokens[b]] (a
 * zero row for a token outside [0, V)), xw[b] = bf16(x[b] * weight) and ss[b, E / 16]
 * the per-16-element sums of squares of x[b] -- the first layer's chained RMSNorm input
 * for iron_gemv_int4g32_chain. E % 16 == 0. */
int iron_embed_chain(const int32_t *tokens, const uint16_t *table, uint16_t *x, uint16_t *xw, const uint16_t *weight,
                     float *ss, int B, int E, int V, unsigned flags, void *stream);
/* iron_gemv_int4g32_allreduce (no reference counterpart as one call: it replaces a
 * row-parallel projection followed by the NCCL all-reduce of the tensor-parallel
 * block): the int4 GEMV of this rank's input columns (n_vec <= 8), whose output tiles
 * are all-reduced over the ranks inside the kernel -- each finished 16-row tile's
 * fp32 partial goes into every rank's receive buffer over NVLink as 8-byte
 * (value, flag) stores and every rank sums them in rank order -- then rounded to bf16
 * and, with `residual`, y = bf16(bf16(sum) + residual) on every rank. `peers` points to
 * an iron_allreduce_peers in host memory; recv[r] is rank r's buffer ([world, N, n_vec]
 * 8-byte slots, zero before first use and left zero), mapped into this process with
 * iron_ipc_open for r != rank. All ranks launch it for the same shape; a wait for a peer's tile gives up after
 * wait_us microseconds (0: one second), sets *status and goes on with the values it has
 * (later waits of the same launch give up at once). iron_ipc_alloc / iron_ipc_free give these buffers their own zero-filled
 * allocations (an IPC handle maps the start of an allocation); iron_ipc_handle /
 * iron_ipc_open / iron_ipc_close wrap CUDA IPC (64-byte handles). */
typedef struct {
  int world, rank;
  float *recv[8];
  unsigned *status;
  unsigned wait_us;
} iron_allreduce_peers;
int iron_gemv_int4g32_allreduce(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                                const uint16_t *residual, const void *peers, unsigned flags, void *stream);
int iron_ipc_alloc(size_t bytes, void **dev_ptr_out);
int iron_ipc_free(void *dev_ptr);
int iron_ipc_handle(const void *dev_ptr, void *handle_out);
int iron_ipc_open(const void *handle, void **dev_ptr_out);
int iron_ipc_close(void *dev_ptr);
int iron_gemv_int4g32(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K,
                      int n_vec, const uint16_t *residual, unsigned flags, void *stream);

/* Dequantize natural-layout int4g32 weights to bf16 [N, K], bit-exact:
 * out[n,k] = bf16(q[n,k] * scale[n,k/32]) (the fp32 product rounded once). */
int iron_dequant_s4g32_rows(const uint8_t *codes, const uint16_t *scales,
                            uint16_t *out, int N, int K, void *stream);

/* ---- Dequant (uint4 tiles) ------------------------------------------------
 * Replaces Dequant(size, ..., tile_size, group_size) -- iron/operators/dequant/op.py:20-81,
 * golden iron/operators/dequant/reference.py:8-18; payload layout from the packer
 * iron/operators/dequant/reference.py:68-92.
 *   payload: per tile of tile_size elements, tile_size/2 code bytes (element 2k = low
 *   nibble of byte k, unsigned 0..15), then tile_size/group_size bf16 scales (LE).
 *   out[i] = bf16(code_i * scale_{i/group_size}); size a multiple of tile_size,
 *   tile_size a multiple of group_size, group_size even.
 */
int iron_dequant_u4(const uint8_t *payload, uint16_t *out, int64_t size,
                    int tile_size, int group_size, void *stream);


/* ---- RMSNorm ----------------------------------------------------------------
 * Replaces RMSNorm(size, ..., tile_size, weighted, epsilon) -- iron/operators/rms_norm/op.py:19-122,
 * golden iron/operators/rms_norm/reference.py:7-16.
 *   y[r, :] = x[r, :] / sqrt(mean(x[r, :]^2) + eps) * (weight ? weight : 1), fp32 statistics.
 *   residual != NULL: x := bf16(x + residual) first (stored to x_out if != NULL) --
 *   the decode block's residual add fused with the following norm.
 */
int iron_rmsnorm(const uint16_t *x, const uint16_t *residual, uint16_t *x_out,
                 const uint16_t *weight, uint16_t *y, int rows, int cols, float eps,
                 unsigned flags, void *stream);

/* ---- RoPE -------------------------------------------------------------------
 * Replaces RoPE(rows, cols, angle_rows, method_type) -- iron/operators/rope/op.py:18-92,
 * golden iron/operators/rope/reference.py:69-102. angles: [*, cols] interleaved
 * cos/sin (bf16 `angles` or fp32 `angles_f32`, one of them). Row r of x uses angle
 * row r / (rows / angle_rows), or pos[r / (rows / angle_rows)] when pos != NULL.
 * method 0: two halves (HF); 1: interleaved pairs. fp32 math, one rounding.
 */
int iron_rope(const uint16_t *x, const uint16_t *angles, const float *angles_f32, uint16_t *y,
              int rows, int cols, int angle_rows, const int32_t *pos, int method,
              unsigned flags, void *stream);

/* ---- Softmax ----------------------------------------------------------------
 * Replaces Softmax(rows, cols, ..., vector_size_parameter) -- iron/operators/softmax/op.py:21-97,
 * golden iron/operators/softmax/reference.py:9-11, mask iron/operators/softmax/design.py:85-91.
 * Row softmax over the first `valid` columns (valid_dev, if set, is read on the
 * device at run time); columns >= valid are 0. fp32 math.
 */
int iron_softmax(const uint16_t *x, uint16_t *y, int rows, int cols, int valid,
                 const int32_t *valid_dev, unsigned flags, void *stream);

/* ---- element-wise -------------------------------------------------------------
 * Replaces SiLU (iron/operators/silu/op.py:12-26), ElementwiseMul
 * (iron/operators/elementwise_mul/op.py:12-24), ElementwiseAdd
 * (iron/operators/elementwise_add/op.py:12-24) and SwiGLUDecode's SiLU+Mul pair
 * (iron/operators/swiglu_decode/op.py:56-62). op: 0 silu(a), 1 a*b, 2 a+b, 3 silu(a)*b.
 */
int iron_eltwise(const uint16_t *a, const uint16_t *b, uint16_t *y, int64_t n, int op,
                 unsigned flags, void *stream);

/* ---- StridedCopy ------------------------------------------------------------
 * Replaces StridedCopy -- iron/operators/strided_copy/op.py:18-100, golden
 * iron/operators/strided_copy/reference.py:37-75 (the decode KV-cache append).
 * Each access pattern (<= 4 dims, element strides) is padded to 4-D; the innermost
 * dimension is split into `channels` parts; element j of channel c moves from the
 * input pattern (+ *in_addend_dev) to the output pattern (+ *out_addend_dev).
 * Addends are element counts read on the device (runtime parameters). Elements
 * whose source or destination falls outside [0, in_size) / [0, out_size) are skipped.
 */
int iron_strided_copy(const void *in, void *out, int elem_size, int ndim_in,
                      const int64_t *in_sizes, const int64_t *in_strides, int64_t in_offset,
                      int ndim_out, const int64_t *out_sizes, const int64_t *out_strides,
                      int64_t out_offset, int channels, const int32_t *in_addend_dev,
                      const int32_t *out_addend_dev, int64_t in_size, int64_t out_size,
                      unsigned flags, void *stream);

/* ---- Repeat / Transpose -------------------------------------------------------
 * Replace Repeat (iron/operators/repeat/op.py:17-69; repeat_interleave along dim 0 of
 * rows x row_bytes) and Transpose (iron/operators/transpose/op.py:18-120; `batches`
 * independent M x N -> N x M, elem_size 2 or 4).
 */
int iron_repeat_interleave(const void *in, void *out, int64_t rows, int64_t row_bytes,
                           int repeat, unsigned flags, void *stream);
int iron_transpose(const void *in, void *out, int M, int N, int batches, int elem_size,
                   unsigned flags, void *stream);

/* ---- GQA decode attention (split-KV) -------------------------------------------
 * Replaces the decode attention steps of IRON's Llama pipeline (Repeat x2, scores
 * GEMV, scale, masked Softmax, per-head Transpose, context GEMV:
 * iron/applications/llama_3.2_1b/llama_npu.py:495-529; CPU truth
 * iron/applications/llama_3.2_1b/llama_cpu.py:118-140).
 *   q: bf16 [B, Hq, D]; caches: element (b, h, t, d) at b*kv_batch_stride +
 *   h*kv_head_stride + t*D + d; lens: int32 [B] valid tokens (device).
 *   out[b, hq] = softmax(scale * q K_{hq/(Hq/Hkv)}^T over t < lens[b]) V, fp32 softmax.
 *   D == 64 (Llama-3.2-1B) or 128 (Llama-3-8B); Hq % Hkv == 0, Hq/Hkv <= 16. Long
 *   caches are split over CTAs; then `workspace` (>= iron_attn_decode_workspace_bytes_d,
 *   or iron_attn_decode_workspace_bytes for D == 64) holds the partials (no zeroing
 *   needed; calls sharing a workspace must not overlap on the GPU).
 */
size_t iron_attn_decode_workspace_bytes(int B, int Hq, int Hkv, int Lmax);
size_t iron_attn_decode_workspace_bytes_d(int B, int Hq, int Hkv, int Lmax, int D);
int iron_attn_decode(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                     const int32_t *lens, uint16_t *out, int B, int Hq, int Hkv, int D, int Lmax,
                     int64_t kv_batch_stride, int64_t kv_head_stride, float scale,
                     void *workspace, size_t workspace_bytes, unsigned flags, void *stream);

/* Decode attention without a caller-provided workspace. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory -- code
 * whose device memory is owned by another allocator (a serving engine that
 * reserves the GPU's memory up front and hands out nothing more) and code on a
 * latency-critical path where cudaMalloc's implicit device synchronisation is
 * not acceptable. Same arguments and results as iron_attn_decode minus the
 * workspace: the split partials go to a fixed 1 MiB array inside the library
 * (per device, held until the process exits). At head_dim 64 with 32 query / 8 kv
 * heads on a 148-SM B200 that holds the partials of every batch up to 32768 tokens; at
 * head_dim 128 some batches do not fit (at 32768 tokens: 1, 2, 4, 8, 9, 16-18 and
 * 32-36). Where the usual split count's partials would not fit it, the extra splits
 * that long caches get (at most 4096 tokens per CTA) are dropped, down to the count
 * that fills two waves of the SMs; requests whose partials exceed 1 MiB even then
 * return IRON_ERR_WORKSPACE (after the same argument checks as iron_attn_decode). The
 * first call on a device looks up the array's device address (with that device
 * current) and caches it with the CUDA context it belongs to, so make that first call
 * before any stream capture; after cudaDeviceReset the next call looks it up again.
 * Nothing is allocated: no cudaMalloc or cudaFree. Every call uses the same
 * array, so calls that overlap on the GPU (other streams, other threads) race;
 * each call writes every partial it reads, so no clearing is needed.
 */
int iron_attn_decode_noalloc(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                             const int32_t *lens, uint16_t *out, int B, int Hq, int Hkv, int D,
                             int Lmax, int64_t kv_batch_stride, int64_t kv_head_stride,
                             float scale, unsigned flags, void *stream);

/* Fused decode attention (no reference counterpart as one call: it replaces the decode
 * RoPE, the two KV-cache StridedCopy appends and the attention runlist steps of
 * iron/applications/llama_3.2_1b/llama_npu.py:481-529). qkv bf16 [B, (Hq + 2 Hkv) * D]
 * (q heads, k heads, v heads) un-rotated; pos int32 [B] tokens already cached; lut fp32
 * [ctx, D] interleaved cos/sin. Rotates q and the new k at pos[b], appends k / v to the
 * caches at slot pos[b] and attends over 0..pos[b] (split partials in `workspace`,
 * >= iron_attn_decode_qkv_workspace_bytes, merged by a second kernel as in
 * iron_attn_decode).
 */
size_t iron_attn_decode_qkv_workspace_bytes(int B, int Hq, int Hkv, int Lmax, int D);
/* iron_attn_decode_kernels: launches one decode-attention call makes (1, or 2 when a
 * split-combine kernel follows). With GQA groups of <= 4 query heads, when all of them
 * fit in one wave of the SMs and no CTA gets more than 512 of the Lmax tokens, the
 * splits of a (sequence, kv head) run as one cluster of
 * 16 or 8 CTAs that merge through distributed shared memory (one launch, no workspace
 * use); otherwise the partials go through `workspace` and a combine kernel. */
int iron_attn_decode_kernels(int B, int Hq, int Hkv, int Lmax);
int iron_attn_decode_qkv(const uint16_t *qkv, const int32_t *pos, const float *lut, uint16_t *k_cache,
                         uint16_t *v_cache, uint16_t *out, int B, int Hq, int Hkv, int D, int Lmax,
                         int64_t kv_batch_stride, int64_t kv_head_stride, float scale, void *workspace,
                         size_t workspace_bytes, unsigned flags, void *stream);

/* ---- decode-step glue ----------------------------------------------------------
 * iron_rope_kv_append replaces the decode RoPE of q and k plus the two StridedCopy
 * KV-cache writes at the runtime cache_offset (iron/applications/llama_3.2_1b/
 * llama_npu.py:481-495, :1161-1169): qkv bf16 [B, (Hq + 2 Hkv) * D] (q heads, then k,
 * then v), pos int32 [B] (tokens already cached), lut fp32 [ctx, D] interleaved
 * cos/sin. Writes q_out bf16 [B, Hq, D] (two-halves RoPE), k/v into cache slot
 * pos[b] (same strides as iron_attn_decode) and lens[b] = pos[b] + 1 (if lens).
 * iron_embed: x[b] = table[tokens[b]] (bf16 rows of E; table has V rows, and a token
 * outside [0, V) gives a zero row instead of a read past the table). iron_argmax: first index
 * of each row's maximum into out[b]; if pos != NULL, pos[b] += 1 afterwards (so a
 * replayed decode graph feeds its own output to the next step).
 */
int iron_rope_kv_append(const uint16_t *qkv, const int32_t *pos, const float *lut,
                        uint16_t *q_out, uint16_t *k_cache, uint16_t *v_cache, int32_t *lens,
                        int B, int Hq, int Hkv, int D, int64_t kv_batch_stride,
                        int64_t kv_head_stride, unsigned flags, void *stream);
int iron_embed(const int32_t *tokens, const uint16_t *table, uint16_t *x, int B, int E, int V,
               unsigned flags, void *stream);
int iron_argmax(const uint16_t *logits, int32_t *out, int B, int V, int32_t *pos, unsigned flags,
                void *stream);

/* Next-token sampling on the device, replacing the per-token logits read-back and the
 * CPU sampling of IRON's generate_token (iron/applications/llama_3.2_1b/
 * llama_inference_harness.py:146-169; its decode loop reads the logits at
 * iron/common/sequence.py:721-730). For each of the B rows of logits (bf16 [B, V]):
 * divide by `temperature` (> 0; 0 leaves the logits as they are, as the harness
 * does), keep the logits >= the top_k-th largest (ties kept; top_k <= 0 or >= V keeps
 * all), softmax, and draw one index with probability proportional to its weight.
 * The uniform draw is a function of (seed, row b, pos[b]) (SplitMix64), so the result
 * is bitwise reproducible and a replayed decode graph draws afresh as positions
 * advance. tokens[b] gets the index; with `pos`, pos[b] += 1 afterwards (pos NULL:
 * position 0 for every row). */
int iron_sample_topk(const uint16_t *logits, int B, int V, float temperature, int top_k,
                     unsigned long long seed, int32_t *tokens, int32_t *pos, unsigned flags, void *stream);

/* ---- prefill attention ------------------------------------------------------------
 * Causal (or full) grouped-query attention over a sequence, replacing IRON's MHA
 * operator (iron/operators/mha/op.py:21-135, golden mha/reference.py:27-94) and the
 * CPU attention of its Llama prefill. D = 64; H a multiple of Hkv (query head h
 * reads kv head h / (H / Hkv)). Element (b, h, t, d) of q / out lives at
 * b*s[0] + h*s[1] + t*s[2] + d for the strides s = q_strides / out_strides (3
 * int64 each, multiples of 8), and likewise for k and v with kv_strides. Queries
 * t < S attend to keys j < S_kv (and j <= t if causal); output rows S <= t < S_pad
 * are written as zeros. S_pad must be a multiple of 64. scale multiplies the logits.
 */
int iron_attn_prefill(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out, int B, int H,
                      int Hkv, int D, int S, int S_pad, int S_kv, const int64_t *q_strides,
                      const int64_t *kv_strides, const int64_t *out_strides, float scale, int causal,
                      unsigned flags, void *stream);

/* ---- tensor-core GEMM (prefill projections) -------------------------------------
 * C = epilogue(A . B^T) on tcgen05 tensor cores with TMEM accumulators: A bf16
 * [M, K] (row pitch lda), B bf16 [N, K] K-major (row pitch ldb), C bf16 [M, N]
 * (row pitch ldc), fp32 accumulation. Replaces the NPU GEMMs of
 * iron/operators/gemm/op.py:21-231 (b_col_maj=True layout; the Python operator
 * transposes a row-major B first) and iron/operators/flm/gemm/op.py:64-499, whose
 * epilogue it fuses: the accumulator is rounded to bf16, then `epilogue` (bits 0-7:
 * 0 none, 1 gelu as x*sigmoid(1.702x), 2 silu, 3 sigmoid) and, if `clamp`, a clamp
 * to [clamp_lo, clamp_hi] (flm/gemm/reference.py:8-57); bit 8 of `epilogue`
 * (IRON_GEMM_ROUND_FLOOR) rounds every fp32 -> bf16 conversion toward -inf
 * (flm Rounding.FLOOR) instead of to nearest even. If `residual` (bf16 [M, N], row pitch
 * ldr) is given, C = bf16(bf16(epilogue(acc)) + residual), the residual add of a
 * decoder block. Epilogue 4 (IRON_GEMM_EPI_SWIGLU) is the SwiGLU of an interleaved
 * gate/up projection: B's rows come in groups of 16 (8 gate rows, then the 8 matching
 * up rows) and C [M, N/2] gets bf16(bf16(silu(bf16(gate))) * bf16(up)) per pair
 * (no residual, clamp or floor rounding with it; N a multiple of 16). K, N, lda, ldb, ldc multiples
 * of 8; pointers 16-byte aligned. block_n = 0 picks the tile width (64/128/192/256).
 * iron_gemm_status returns IRON_ERR_TIMEOUT if any GEMM since the last reset hit
 * its bounded-wait deadline (reset != 0 clears it); it synchronises the device.
 */
#define IRON_GEMM_ROUND_FLOOR 0x100
#define IRON_GEMM_EPI_SWIGLU 4

int iron_gemm_bf16(const uint16_t *A, const uint16_t *B, uint16_t *C, int M, int N, int K,
                   int64_t lda, int64_t ldb, int64_t ldc, const uint16_t *residual, int64_t ldr,
                   int epilogue, int clamp, float clamp_lo, float clamp_hi, int block_n, unsigned flags,
                   void *stream);
int iron_gemm_status(int reset);

#ifdef __cplusplus
}
#endif

#endif /* IRON_B200_H */
