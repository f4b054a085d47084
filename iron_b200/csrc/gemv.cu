// bf16 GEMV kernel, and the exact dequantization of the int4 group-32 format.
//
// Both are HBM-bound streams over the weight matrix. A warp owns a 16-row tile
// and a slice of K; it loads 16-byte pieces of two rows per lane straight into
// registers (ld.global.nc, no L1 allocation) and uses the m16n8k16 bf16 MMA only
// as a warp-wide dot-product reducer with fp32 accumulation: the 8 MMA columns
// carry up to 8 decode vectors, so batches of 1..8 cost the same weight traffic.
// The logical k order inside one MMA is free as long as A and B agree, which lets
// every lane feed its own contiguous 16 bytes without shuffles.
//
// K is split over the 4 warps of a CTA and, for matrices with few row tiles, over
// the CTAs of a thread-block cluster (partials reduced through distributed shared
// memory), so that every launch puts >= 2 CTAs on each of the 148 SMs.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace iron {

constexpr int kGemvWarps = 4;       // warps per CTA, each a K slice
constexpr int kGemvThreads = 32 * kGemvWarps;

__device__ __forceinline__ uint4 zero4() { return make_uint4(0u, 0u, 0u, 0u); }


__device__ __forceinline__ uint16_t ld_stream_u16(const uint16_t *p) {
  uint16_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

// (a & b) ^ c in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Signed int4 pair -> exactly dequantized bf16x2.
// `w_shifted` holds nibble i of the low 16 bits in bits 0-3 and nibble i of the
// high 16 bits in bits 16-19. OR-ing (nib ^ 8) into the mantissa of bf16 128.0
// (0x4300) gives 136 + q exactly, q = signed value in [-8, 7]; subtracting 136
// (0x4308) is exact; the scale multiply rounds the exact product once, i.e.
// bf16(q * s), the dequantized weight bit for bit.
__device__ __forceinline__ uint32_t s4x2_dequant(uint32_t w_shifted, uint32_t scale2) {
  uint32_t biased = lop3_and_xor(w_shifted, 0x000f000fu, 0x43084308u);
  return bf16x2_mul(bf16x2_sub(biased, 0x43084308u), scale2);
}

// ---------------------------------------------------------------------------
// Cross-warp / cross-CTA reduction of the 16x(8*NT) partial tile, epilogue, store.
// Each lane of each warp holds acc[t][4] in the m16n8 C-fragment layout:
//   c0,c1 -> row gid,   cols 2*tid, 2*tid+1;  c2,c3 -> row gid+8, same cols.
template <int NT, int CS>
__device__ __forceinline__ void gemv_reduce_store(float (&acc)[NT][4], float *red,
                                                  int row0, int M, int n_vec,
                                                  uint16_t *__restrict__ y,
                                                  const uint16_t *__restrict__ residual,
                                                  int epilogue) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // red: [kGemvWarps][NT][4][32] floats, lane-contiguous to avoid bank conflicts.
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[((warp * NT + t) * 4 + e) * 32 + lane] = acc[t][e];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) s += red[((w * NT + t) * 4 + e) * 32 + lane];
        acc[t][e] = s;
      }
  }
  if constexpr (CS > 1) {
    // Ranks 1..CS-1 deposit their CTA partial into rank 0's shared memory.
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    float *slot0 = red + kGemvWarps * NT * 4 * 32;  // [CS][NT][4][32]
    if (warp == 0 && rank > 0) {
      float *remote = cluster.map_shared_rank(slot0, 0);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) remote[((rank * NT + t) * 4 + e) * 32 + lane] = acc[t][e];
    }
    cluster.sync();
    if (rank != 0) return;
    if (warp == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float s = acc[t][e];
#pragma unroll
          for (int r = 1; r < CS; ++r) s += slot0[((r * NT + t) * 4 + e) * 32 + lane];
          acc[t][e] = s;
        }
    }
  }
  if (warp != 0) return;
  const int gid = lane >> 2, tid = lane & 3;
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = row0 + gid + ((e >> 1) << 3);
      const int v = t * 8 + tid * 2 + (e & 1);
      if (row < M && v < n_vec) {
        float r = acc[t][e];
        if (epilogue == IRON_EPI_GELU) r = gelu_tanh(r);
        const int64_t o = static_cast<int64_t>(v) * M + row;
        if (residual) r = __bfloat162float(__float2bfloat16_rn(r)) + bf16_bits_to_float(ld_act_u16(residual + o));
        y[o] = float_to_bf16_bits(r);
      }
    }
}

// ---------------------------------------------------------------------------
// bf16 GEMV. Chunk = 32 k of a 16-row tile: lane (gid, tid) loads elements
// [32c + 8 tid, +8) of rows gid and gid+8 (two 16-byte loads) and feeds them as
// two k16 MMA steps; B is the matching 16 bytes of each vector, unpermuted.
// kRO: x through the read-only path (IRON_FLAG_X_READONLY), else L2-coherent loads.
template <int NT, int CS, int U, bool kRO>
__global__ void __launch_bounds__(kGemvThreads)
gemv_bf16_kernel(const uint16_t *__restrict__ W, const uint16_t *__restrict__ x,
                 uint16_t *__restrict__ y, int M, int K, int64_t ldw, int64_t w_bstride,
                 int64_t x_bstride, int64_t y_bstride, int n_vec,
                 const uint16_t *__restrict__ residual, int epilogue) {
  __shared__ float red[(kGemvWarps + CS) * NT * 4 * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid = lane & 3;
  const int rank = (CS > 1) ? static_cast<int>(blockIdx.x % CS) : 0;
  const int row0 = blockIdx.y * 16;
  const int b = blockIdx.z;
  W += b * w_bstride;
  x += b * x_bstride;
  y += b * y_bstride;
  if (residual) residual += b * y_bstride;

  const int chunks = (K + 31) / 32;
  const int slices = kGemvWarps * CS;
  const int per = (chunks + slices - 1) / slices;
  const int slice = rank * kGemvWarps + warp;
  const int c_begin = min(chunks, slice * per);
  const int c_end = min(chunks, c_begin + per);

  const int row_lo = row0 + gid, row_hi = row_lo + 8;
  const uint16_t *w_lo = W + static_cast<int64_t>(min(row_lo, M - 1)) * ldw + tid * 8;
  const uint16_t *w_hi = W + static_cast<int64_t>(min(row_hi, M - 1)) * ldw + tid * 8;
  const bool lo_ok = row_lo < M, hi_ok = row_hi < M;

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

  uint4 a_lo[U], a_hi[U];
  auto load = [&](int c0) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      const int k = c * 32 + tid * 8;
      const bool ok = c < c_end && k < K;
      a_lo[u] = (ok && lo_ok) ? ld_stream_v4(w_lo + c * 32) : zero4();
      a_hi[u] = (ok && hi_ok) ? ld_stream_v4(w_hi + c * 32) : zero4();
    }
  };
  load(c_begin);
  pdl_wait();  // weights may be streamed early; activations may not
  for (int c0 = c_begin; c0 < c_end; c0 += U) {
    uint4 n_lo[U], n_hi[U];
#pragma unroll
    for (int u = 0; u < U; ++u) { n_lo[u] = a_lo[u]; n_hi[u] = a_hi[u]; }
    if (c0 + U < c_end) load(c0 + U);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      const int k = c * 32 + tid * 8;
      const bool ok = c < c_end && k < K;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int v = t * 8 + gid;
        const uint4 xb = (ok && v < n_vec)
                             ? (kRO ? __ldg(reinterpret_cast<const uint4 *>(x + static_cast<int64_t>(v) * K + k))
                                    : ld_act_v4(x + static_cast<int64_t>(v) * K + k))
                             : zero4();
        const uint32_t A0[4] = {n_lo[u].x, n_hi[u].x, n_lo[u].y, n_hi[u].y};
        mma_bf16_16816(acc[t], A0, xb.x, xb.y);
        const uint32_t A1[4] = {n_lo[u].z, n_hi[u].z, n_lo[u].w, n_hi[u].w};
        mma_bf16_16816(acc[t], A1, xb.z, xb.w);
      }
    }
  }
  pdl_launch_dependents();
  gemv_reduce_store<NT, CS>(acc, red, row0, M, n_vec, y, residual, epilogue);
}

// ---------------------------------------------------------------------------
// Exact dequantization of the int4g32 GEMV format to bf16 rows (parity check).
__global__ void dequant_s4g32_rows_kernel(const uint8_t *__restrict__ Wq,
                                          const uint16_t *__restrict__ scales,
                                          uint16_t *__restrict__ out, int64_t total_bytes,
                                          int K) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total_bytes) return;
  const int64_t half = K / 2;
  const int64_t n = i / half, kb = i % half;
  const uint8_t byte = Wq[i];
  const float s = bf16_bits_to_float(scales[n * (K / 32) + (2 * kb) / 32]);
  const int q0 = static_cast<int>(byte & 0xF) - ((byte & 0x8) ? 16 : 0);
  const int q1 = static_cast<int>(byte >> 4) - ((byte & 0x80) ? 16 : 0);
  const uint32_t pair = static_cast<uint32_t>(float_to_bf16_bits(static_cast<float>(q0) * s)) |
                        (static_cast<uint32_t>(float_to_bf16_bits(static_cast<float>(q1) * s)) << 16);
  reinterpret_cast<uint32_t *>(out)[i] = pair;
}

// ---------------------------------------------------------------------------
template <int NT, int CS>
static int launch_bf16(const uint16_t *W, const uint16_t *x, uint16_t *y, int M, int K,
                       int64_t ldw, int nb, int64_t wb, int64_t xb, int64_t yb, int n_vec,
                       const uint16_t *res, int epi, bool pdl, bool ro, cudaStream_t s) {
  dim3 grid(CS, (M + 15) / 16, nb);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemvThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (CS > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = CS;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = ro ? cudaLaunchKernelEx(&cfg, gemv_bf16_kernel<NT, CS, 4, true>, W, x, y, M, K, ldw, wb, xb, yb,
                                          n_vec, res, epi)
                     : cudaLaunchKernelEx(&cfg, gemv_bf16_kernel<NT, CS, 4, false>, W, x, y, M, K, ldw, wb, xb, yb,
                                          n_vec, res, epi);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}

// Smallest cluster split that gives >= 2 CTAs per SM without slicing K below
// two chunks per warp.
static int pick_split(int64_t tiles, int chunks) {
  const int64_t want = 2LL * sm_count();
  int cs = 1;
  while (cs < 8 && tiles * cs < want && chunks >= 2 * kGemvWarps * cs * 2) cs *= 2;
  return cs;
}

#define IRON_DISPATCH_NT(n_vec, CALL)                  \
  do {                                                 \
    if ((n_vec) <= 8) { constexpr int NT = 1; CALL; }  \
    else if ((n_vec) <= 16) { constexpr int NT = 2; CALL; } \
    else if ((n_vec) <= 32) { constexpr int NT = 4; CALL; } \
    else { constexpr int NT = 8; CALL; }               \
  } while (0)

#define IRON_DISPATCH_CS(cs, CALL)                     \
  do {                                                 \
    switch (cs) {                                      \
      case 1: { constexpr int CS = 1; CALL; } break;   \
      case 2: { constexpr int CS = 2; CALL; } break;   \
      case 4: { constexpr int CS = 4; CALL; } break;   \
      default: { constexpr int CS = 8; CALL; } break;  \
    }                                                  \
  } while (0)

}  // namespace iron

using namespace iron;

extern "C" int iron_gemv_bf16(const uint16_t *W, const uint16_t *x, uint16_t *y, int M, int K,
                              int64_t ldw, int num_batches, int64_t w_bstride,
                              int64_t x_bstride, int64_t y_bstride, int n_vec,
                              const uint16_t *residual, int epilogue, unsigned flags,
                              void *stream) {
  if (!W || !x || !y) return IRON_ERR_NULL;
  if (M <= 0 || K <= 0 || num_batches <= 0 || n_vec <= 0 || n_vec > 64 || ldw < K)
    return IRON_ERR_SHAPE;
  if (num_batches > 65535 || (M + 15) / 16 > 65535) return IRON_ERR_SHAPE;
  if (K % 8 || ldw % 8 || !aligned16(W) || !aligned16(x)) return IRON_ERR_ALIGN;
  if (num_batches > 1 && (w_bstride % 8 || x_bstride % 8)) return IRON_ERR_ALIGN;
  if (epilogue != IRON_EPI_NONE && epilogue != IRON_EPI_GELU) return IRON_ERR_ARG;
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t tiles = static_cast<int64_t>((M + 15) / 16) * num_batches;
  const int cs = pick_split(tiles, (K + 31) / 32);
  int st = IRON_OK;
  IRON_DISPATCH_NT(n_vec, IRON_DISPATCH_CS(cs, st = (launch_bf16<NT, CS>(
                                               W, x, y, M, K, ldw, num_batches, w_bstride,
                                               x_bstride, y_bstride, n_vec, residual,
                                               epilogue, pdl, (flags & IRON_FLAG_X_READONLY) != 0, s))));
  return st;
}

extern "C" int iron_dequant_s4g32_rows(const uint8_t *Wq, const uint16_t *scales, uint16_t *out,
                                       int N, int K, void *stream) {
  if (!Wq || !scales || !out) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || K % 32) return IRON_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(out) & 3u) return IRON_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(N) * (K / 2);
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return IRON_ERR_SHAPE;
  dequant_s4g32_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                              static_cast<cudaStream_t>(stream)>>>(Wq, scales, out, total, K);
  return launch_status();
}
