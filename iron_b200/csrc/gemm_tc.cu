// bf16 GEMM on the 5th-generation tensor cores: C = epilogue(A . B^T).
//
// Replaces the prefill projections of IRON's GEMM operators
// (iron/operators/gemm/op.py:21-231, iron/operators/flm/gemm/op.py:64-499;
// goldens gemm/reference.py:7-18 and flm/gemm/reference.py:8-57): A [M, K] and
// B [N, K] are K-major bf16 in HBM, C [M, N] bf16 row-major, fp32 accumulation.
// The flm epilogue (activation after the bf16 conversion, then an optional
// clamp) is fused into the TMEM drain.
//
// Persistent and warp-specialised: one CTA per SM walks 128 x BN output tiles
// with a ring of shared-memory stages (TMA loads of 64-wide k-blocks, 128-byte
// swizzle) and two TMEM accumulators, so the drain of one tile overlaps the
// mainloop of the next. The drain stages each warp's 32 x 32 output block in
// shared memory (swizzled, conflict-free) and writes it with one TMA bulk store.
// Every mbarrier wait gives up after 2 s without progress; a timeout sets the
// status word and the CTA leaves after freeing its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include <cooperative_groups.h>

#include "common.cuh"
#include "s4.cuh"
#include "tc.cuh"

namespace iron {
namespace gemm {

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint64_t kDeadlineNs = 2000000000ull;

__device__ unsigned g_gemm_status;  // 0 = ok, else the first failing role's code

struct Epi {
  int mode;   // 0 none, 1 gelu (x * sigmoid(1.702 x)), 2 silu, 3 sigmoid, 4 swiglu (interleaved 8 + 8)
  int floor;  // round fp32 -> bf16 toward -inf instead of to nearest even
  int clamp;
  float lo, hi;
};

__device__ __forceinline__ float to_bf16(float c, int floor) {
  return __bfloat162float(floor ? __float2bfloat16_rd(c) : __float2bfloat16_rn(c));
}

// The activation sees the bf16-rounded accumulator (flm/gemm/reference.py:34-57);
// the result is rounded to bf16 again on the way out.
__device__ __forceinline__ float apply_epi(float c, const Epi &e) {
  c = to_bf16(c, e.floor);
  if (e.mode == 1) c = c / (1.0f + __expf(-1.702f * c));
  else if (e.mode == 2) c = c / (1.0f + __expf(-c));
  else if (e.mode == 3) c = 1.0f / (1.0f + __expf(-c));
  if (e.clamp) c = fminf(fmaxf(c, e.lo), e.hi);
  return to_bf16(c, e.floor);
}

// Gate/up pair of the interleaved SwiGLU layout: bf16(bf16(silu(bf16(g))) * bf16(u)).
__device__ __forceinline__ float swiglu_pair(float g, float u) {
  g = __bfloat162float(__float2bfloat16_rn(g));
  u = __bfloat162float(__float2bfloat16_rn(u));
  const float sw = __bfloat162float(__float2bfloat16_rn(g / (1.0f + __expf(-g))));
  return sw * u;
}

__device__ __forceinline__ uint32_t add_res2(uint32_t packed, uint32_t res) {
  // bf16(projection) + bf16(residual), rounded once more
  return pack_bf16x2(bf16_lo(packed) + bf16_lo(res), bf16_hi(packed) + bf16_hi(res));
}

// Output staging: per epilogue warp two buffers of 32 rows x 32 columns of bf16 (64-byte
// rows; the SwiGLU form's 16 output columns use 32-byte rows of the same buffers),
// written in the TMA store's swizzled order (64B / 32B swizzle) so that the 32 lanes'
// 16-byte stores are free of bank conflicts.
constexpr int kStgBytes = 32 * 64;

template <int BN>
struct Cfg {
  static constexpr int kStageA = BM * BK * 2;
  static constexpr int kStageB = BN * BK * 2;
  static constexpr int kStage = kStageA + kStageB;
  static constexpr int kStages = (192 * 1024) / kStage;
  static constexpr int kBars = 1024;  // mbarriers and the TMEM slot
  static constexpr int kSmem = 1024 + kStages * kStage + kBars + kEpiWarps * 2 * kStgBytes;
};

// Byte offset of 16-byte chunk g of row r in a staging buffer (TMA 64B / 32B swizzle:
// chunk bits 4-5 (4) XORed with address bits 7-8 (7)).
__device__ __forceinline__ uint32_t stg64(int r, int g) { return r * 64 + ((g ^ ((r >> 1) & 3)) << 4); }
__device__ __forceinline__ uint32_t stg32(int r, int g) { return r * 32 + ((g ^ ((r >> 2) & 1)) << 4); }

// Persistent, warp-specialised kernel. Each CTA walks the output tiles
// blockIdx.x, blockIdx.x + gridDim.x, ... with two TMEM accumulators, so the
// epilogue of one tile overlaps the mainloop of the next:
//   warp 0, one thread : TMA producer (A and B k-blocks into the stage ring);
//   warp 1, one thread : MMA issuer (accumulator i % 2 of the CTA's i-th tile);
//   warp 2            : allocates / frees the two accumulators' TMEM columns;
//   warps 2..5        : epilogue, warp w draining TMEM lanes 32 (w % 4) ..
//                       32 (w % 4) + 31 (the lane quarter that warp may access).
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
                   const uint16_t *__restrict__ R, int64_t ldr, Epi epi) {
  using G = Cfg<BN>;
  constexpr int S = G::kStages;
  // two accumulators of BN columns; TMEM is allocated in powers of two (BN = 192: 512)
  constexpr uint32_t kCols = 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 128-byte swizzle atoms need 1024-B alignment
  const uint32_t stage0 = base;
  const uint32_t bars = base + S * G::kStage;
  const uint32_t full0 = bars, empty0 = bars + 8 * S;
  const uint32_t tfull0 = bars + 16 * S, tempty0 = tfull0 + 16;  // [2] each
  const uint32_t tslot = tempty0 + 16;
  uint32_t *tslot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tslot - raw));
  const uint32_t stg0 = bars + G::kBars;  // 1024-byte aligned

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_count = (K + BK - 1) / BK;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;

  if (threadIdx.x == 0) {
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
    tc::prefetch_tmap(&tmC);
    for (int s = 0; s < S; ++s) {
      tc::mbar_init_u32(full0 + 8 * s, 1);
      tc::mbar_init_u32(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init_u32(tfull0 + 8 * a, 1);
      tc::mbar_init_u32(tempty0 + 8 * a, kEpiWarps);
    }
    mbar_init_fence();
  }
  if (warp == 2) tc::tmem_alloc(tslot, kCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot_ptr;
  pdl_wait();  // A is the previous kernel's output; the prologue above overlapped it
  constexpr uint64_t deadline = kDeadlineNs;  // per wait

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer ----
      bool ok = true;
      int it = 0, issued = 0;  // it: k-blocks issued by this CTA over all its tiles
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN;
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % S;
          if (!tc::wait_until(empty0 + 8 * s, ((it / S) & 1) ^ 1, deadline)) {
            ok = false;
            break;
          }
          const uint32_t sa = stage0 + s * G::kStage, sb = sa + G::kStageA;
          tc::expect_tx(full0 + 8 * s, G::kStage);
          tc::tma_load_2d(sa, &tmA, kb * BK, m0, full0 + 8 * s);
          tc::tma_load_2d(sb, &tmB, kb * BK, n0, full0 + 8 * s);
          issued = it + 1;
        }
      }
      if (!ok) {
        atomicCAS(&g_gemm_status, 0u, 1u);
        // let copies already in flight land before the CTA's shared memory goes away
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
          tc::wait_until(full0 + 8 * (j % S), (j / S) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
      bool ok = true;
      int it = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int acc = i & 1;
        const uint32_t d = tmem + acc * BN;
        if (!tc::wait_until(tempty0 + 8 * acc, ((i >> 1) & 1) ^ 1, deadline)) {  // epilogue drained it
          ok = false;
          break;
        }
        tc::fence_after_sync();
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % S;
          if (!tc::wait_until(full0 + 8 * s, (it / S) & 1, deadline)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = stage0 + s * G::kStage, sb = sa + G::kStageA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc::mma_bf16(d, tc::sdesc_kmajor_sw128(sa + 32 * k), tc::sdesc_kmajor_sw128(sb + 32 * k), idesc,
                         (kb | k) != 0);
          tc::mma_commit(empty0 + 8 * s);  // stage free once these MMAs have read it
        }
        tc::mma_commit(tfull0 + 8 * acc);  // accumulator ready (partial on error)
      }
      if (!ok) atomicCAS(&g_gemm_status, 0u, 2u);
    }
  } else {
    // ---- epilogue: TMEM -> registers -> bf16 -> shared staging -> TMA store ----
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t stg = stg0 + q * 2 * kStgBytes;
    uint8_t *stg_ptr = smem_raw + (stg - raw);
    const int out_cols = epi.mode == 4 ? N / 2 : N;
    // no activation, clamp or floor rounding: the drain is a plain conversion. (Per-value
    // option branches made the drain instruction-bound: 25 us per 128 x 256 tile on
    // B200, twice a K = 2048 tile's mainloop.)
    const bool plain = epi.mode == 0 && !epi.floor && !epi.clamp;
    int i = 0, nb = 0;  // nb: blocks this warp has stored (buffer nb & 1)
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int acc = i & 1;
      const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN;
      const bool have = __all_sync(0xffffffffu, tc::wait_until(tfull0 + 8 * acc, (i >> 1) & 1, deadline));
      if (!have) {
        if (lane == 0) atomicCAS(&g_gemm_status, 0u, 3u);
        break;
      }
      tc::fence_after_sync();
      const int row = m0 + q * 32 + lane;
      const uint32_t trow = tmem + acc * BN + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32, ++nb) {
        uint32_t r[32];
        tc::tmem_ld32(trow + c, r);
        const uint32_t buf = (nb & 1) * kStgBytes;
        if (lane == 0) tc::bulk_wait_read<1>();  // this buffer's store (two blocks ago) has read it
        __syncwarp();
        if (epi.mode == 4) {
          // two 16-column groups: 8 gate then 8 up columns -> 8 outputs each
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const uint32_t *rg = r + 16 * g;
            uint4 v;
            v.x = pack_bf16x2(swiglu_pair(__uint_as_float(rg[0]), __uint_as_float(rg[8])),
                              swiglu_pair(__uint_as_float(rg[1]), __uint_as_float(rg[9])));
            v.y = pack_bf16x2(swiglu_pair(__uint_as_float(rg[2]), __uint_as_float(rg[10])),
                              swiglu_pair(__uint_as_float(rg[3]), __uint_as_float(rg[11])));
            v.z = pack_bf16x2(swiglu_pair(__uint_as_float(rg[4]), __uint_as_float(rg[12])),
                              swiglu_pair(__uint_as_float(rg[5]), __uint_as_float(rg[13])));
            v.w = pack_bf16x2(swiglu_pair(__uint_as_float(rg[6]), __uint_as_float(rg[14])),
                              swiglu_pair(__uint_as_float(rg[7]), __uint_as_float(rg[15])));
            *reinterpret_cast<uint4 *>(stg_ptr + buf + stg32(lane, g)) = v;
          }
        } else {
          const uint16_t *res = (R && row < M) ? R + static_cast<int64_t>(row) * ldr + n0 + c : nullptr;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 v;
            if (plain) {  // one rounding per value, two values per conversion
              v.x = pack_bf16x2(__uint_as_float(r[8 * g + 0]), __uint_as_float(r[8 * g + 1]));
              v.y = pack_bf16x2(__uint_as_float(r[8 * g + 2]), __uint_as_float(r[8 * g + 3]));
              v.z = pack_bf16x2(__uint_as_float(r[8 * g + 4]), __uint_as_float(r[8 * g + 5]));
              v.w = pack_bf16x2(__uint_as_float(r[8 * g + 6]), __uint_as_float(r[8 * g + 7]));
            } else {
              v.x = pack_bf16x2(apply_epi(__uint_as_float(r[8 * g + 0]), epi), apply_epi(__uint_as_float(r[8 * g + 1]), epi));
              v.y = pack_bf16x2(apply_epi(__uint_as_float(r[8 * g + 2]), epi), apply_epi(__uint_as_float(r[8 * g + 3]), epi));
              v.z = pack_bf16x2(apply_epi(__uint_as_float(r[8 * g + 4]), epi), apply_epi(__uint_as_float(r[8 * g + 5]), epi));
              v.w = pack_bf16x2(apply_epi(__uint_as_float(r[8 * g + 6]), epi), apply_epi(__uint_as_float(r[8 * g + 7]), epi));
            }
            if (res && n0 + c + 8 * g + 8 <= N) {
              const uint4 rv = ld_act_v4(res + 8 * g);
              v.x = add_res2(v.x, rv.x);
              v.y = add_res2(v.y, rv.y);
              v.z = add_res2(v.z, rv.z);
              v.w = add_res2(v.w, rv.w);
            }
            *reinterpret_cast<uint4 *>(stg_ptr + buf + stg64(lane, g)) = v;
          }
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        // rows past M and columns past the output's width are clipped by the store
        const int x = epi.mode == 4 ? (n0 + c) / 2 : n0 + c;
        if (lane == 0 && m0 + q * 32 < M && x < out_cols) {
          tc::tma_store_2d(&tmC, stg + buf, x, m0 + q * 32);
          tc::bulk_commit();
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tempty0 + 8 * acc) : "memory");
    }
    if (lane == 0) tc::bulk_wait_all();  // the stores have written C (and read the staging)
  }
  __syncwarp();
  pdl_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 2) tc::tmem_free(tmem, kCols);
}

// ---- int4 g32 weights x a batch of vectors on the tensor cores -----------------------
//
// The int4 GEMV of iron_gemv_int4g32 for 33..64 vectors (decode batches), where the
// mma.sync dot-product engine becomes compute-bound (B200, batch 64: 41-107 TFLOP/s).
// A CTA owns a 128-row tile of the weights and a slice of K (a cluster of up to 8
// CTAs splits K). Per 128-k stage:
//   - eight dequantising warps read their 16-row unit of the packed weights (the same
//     1152-byte units as the GEMV, requested one stage ahead) and write the exact bf16
//     values bf16(q * s) into shared memory in the 128-byte-swizzled K-major layout
//     (streaming the units into a shared ring by bulk copies instead, which left room
//     for 3 stages rather than 4, measured 2.04 against 1.82 ms per B200 batch-64
//     decode step);
//   - one thread loads the stage's activations [vectors, 128 k] by TMA;
//   - one thread issues tcgen05.mma (M = 128 weight rows, N = vectors rounded up to 16)
//     into a TMEM accumulator.
// The weights never depend on the previous kernel, so the dequantising warps fill the
// ring before the activations arrive; only the activation loads wait
// (griddepcontrol.wait). The epilogue parks each CTA's fp32 partial tile in shared
// memory; after a cluster barrier CTA r sums rows [r * 128 / CS, (r + 1) * 128 / CS) of
// every rank's tile in rank order (bitwise deterministic) and applies the GEMV's
// epilogue: plain, + residual, interleaved SwiGLU, or the greedy argmax keys.
namespace s4tc {

namespace cg = cooperative_groups;

constexpr int kRows = 128;                        // weight rows per tile (MMA M)
constexpr int kKB = 128;                          // k per stage: one packed unit
constexpr int kStages = 4;
constexpr int kDqWarps = 8;                       // a 16-row unit each; also the TMEM drain
constexpr int kDrainWarps = 8;
constexpr int kThreads = 32 * (2 + kDqWarps);     // warp 0: activation TMA, warp 1: MMA + TMEM
constexpr int kMaxVec = 64;
constexpr int kStageA = kRows * kKB * 2;          // two 64-k swizzle blocks of 16 KB
constexpr int kStageB = kMaxVec * kKB * 2;        // two 64-k blocks of up to 8 KB
constexpr int kStage = kStageA + kStageB;
constexpr int kSmem = 1024 + kStages * kStage + 1024;
constexpr int kUnitBytes = 1152;

struct Args {
  const uint8_t *packed;
  uint16_t *y;
  const uint16_t *residual;
  unsigned long long *amax;
  int N, K, n_vec, swiglu;
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (v != v) u = 0u;  // NaN never wins
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned>(~row);
}

// Eight rows of a unit for this lane: rows row0 + gid, k 32 j + 8 tid + 0..7 of each
// 32-k group j (words w, this row's group scales s01 = groups 0-1, s23 = groups 2-3), as
// bf16(q * s) -- the GEMV's exact dequantisation -- stored at the rows' 16-byte chunks of
// the stage's two swizzled 64-k blocks.
__device__ __forceinline__ void dequant_rows(uint32_t stage_a, int row0, const uint4 &wv, uint32_t s01,
                                             uint32_t s23) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tid = lane & 3;
  const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
  const uint32_t sp[2] = {s01, s23};
  const int r = row0 + gid;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t s2 = prmt_(sp[j >> 1], sp[j >> 1], (j & 1) ? 0x3232u : 0x1010u);
    uint32_t p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = s4x2_dequant_(wd[j] >> (4 * q), s2);
    const uint32_t blk = stage_a + (j >> 1) * (kRows * 128);
    const int c16 = ((j & 1) << 2) | tid;  // 16-byte chunk of the 128-byte row
    st_shared_v4(blk + r * 128 + ((c16 ^ (r & 7)) << 4), p[0], p[1], p[2], p[3]);
  }
}

template <int CS>
__global__ void __launch_bounds__(kThreads, 1)
    s4tc_kernel(const __grid_constant__ CUtensorMap tmX, Args a, int nmma) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 128-byte swizzle atoms: 1024-B aligned
  const uint32_t bars = base + kStages * kStage;
  const uint32_t full0 = bars, empty0 = bars + 8 * kStages, accf = bars + 16 * kStages;
  const uint32_t tslot = accf + 8;
  uint32_t *tslot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tslot - raw));
  float *P = reinterpret_cast<float *>(smem_raw + (base - raw));  // fp32 partial tile, after the mainloop
  const int pstride = nmma + 1;                                   // [128][nmma + 1]: conflict-free columns

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = CS > 1 ? static_cast<int>(blockIdx.x % CS) : 0;
  const int tile = blockIdx.x / CS;
  const int cpt = a.K / kKB;
  const int c0 = rank * cpt / CS, nkb = (rank + 1) * cpt / CS - c0;  // this CTA's k-blocks
  const uint32_t cols = nmma <= 32 ? 32u : 64u;
  constexpr uint64_t deadline = kDeadlineNs;

  if (threadIdx.x == 0) {
    tc::prefetch_tmap(&tmX);
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init_u32(full0 + 8 * s, kDqWarps + 1);  // the dequantising warps + the activation load
      tc::mbar_init_u32(empty0 + 8 * s, 1);
    }
    tc::mbar_init_u32(accf, 1);
    mbar_init_fence();
  }
  if (warp == 1) tc::tmem_alloc(tslot, cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---- activations: [vectors, 128 k] per stage, two 64-k boxes of nmma rows ----
      pdl_wait();  // x is the previous kernel's output
      bool ok = true;
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (!tc::wait_until(empty0 + 8 * s, ((kb / kStages) & 1) ^ 1, deadline)) {
          ok = false;
          break;
        }
        const uint32_t sb = base + s * kStage + kStageA;
        tc::expect_tx(full0 + 8 * s, static_cast<uint32_t>(nmma) * kKB * 2);
        tc::tma_load_2d(sb, &tmX, (c0 + kb) * kKB, 0, full0 + 8 * s);
        tc::tma_load_2d(sb + kStageB / 2, &tmX, (c0 + kb) * kKB + 64, 0, full0 + 8 * s);
        issued = kb + 1;
      }
      if (!ok) {
        atomicCAS(&g_gemm_status, 0u, 5u);
        for (int j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)  // copies in flight land
          tc::wait_until(full0 + 8 * (j % kStages), (j / kStages) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA: D[128 rows, nmma vectors] += W[128, 16] . X[nmma, 16]^T per 16 k ----
      const uint32_t idesc = tc::idesc_bf16_f32(kRows, nmma);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % kStages;
        if (!tc::wait_until(full0 + 8 * s, (kb / kStages) & 1, deadline)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t sa = base + s * kStage, sb = sa + kStageA;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_bf16(tmem, tc::sdesc_kmajor_sw128(sa + h * (kRows * 128) + 32 * k),
                         tc::sdesc_kmajor_sw128(sb + h * (kStageB / 2) + 32 * k), idesc, (kb | h | k) != 0);
        tc::mma_commit(empty0 + 8 * s);  // the stage is free once these MMAs have read it
      }
      if (!ok) atomicCAS(&g_gemm_status, 0u, 6u);
      tc::mma_commit(accf);  // accumulator ready (partial on error)
    }
  } else {
    // ---- dequantising warps: unit u (rows 16 u .. 16 u + 15) of each k-block (16
    // warps on 8-row halves measured slower) ----
    const int u = warp - 2, gid = lane >> 2;
    const uint8_t *ub = a.packed + (static_cast<int64_t>(tile) * 8 + u) * cpt * kUnitBytes;
    auto load = [&](int kb, uint4 &lo, uint4 &hi, uint4 &sc) {
      const uint8_t *p = ub + static_cast<int64_t>(c0 + kb) * kUnitBytes;
      lo = ld_stream_v4(p + lane * 16);
      hi = ld_stream_v4(p + 512 + lane * 16);
      sc = ld_stream_v4(p + 1024 + gid * 16);
    };
    bool ok = true;
    auto put = [&](int kb, const uint4 &lo, const uint4 &hi, const uint4 &sc) {
      const int s = kb % kStages;
      if (ok && !tc::wait_until(empty0 + 8 * s, ((kb / kStages) & 1) ^ 1, deadline)) ok = false;
      if (ok) {
        dequant_rows(base + s * kStage, u * 16, lo, sc.x, sc.y);
        dequant_rows(base + s * kStage, u * 16 + 8, hi, sc.z, sc.w);
      }
      tc::fence_proxy_async_smem();  // the tensor core reads these stores through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + 8 * s);
    };
    // three register sets: two units in flight while one is dequantised
    uint4 l0 = {}, h0 = {}, s0 = {}, l1 = {}, h1 = {}, s1 = {}, l2 = {}, h2 = {}, s2 = {};
    if (nkb > 0) load(0, l0, h0, s0);
    if (nkb > 1) load(1, l1, h1, s1);
    for (int kb = 0; kb < nkb; kb += 3) {
      if (kb + 2 < nkb) load(kb + 2, l2, h2, s2);
      put(kb, l0, h0, s0);
      if (kb + 1 >= nkb) break;
      if (kb + 3 < nkb) load(kb + 3, l0, h0, s0);
      put(kb + 1, l1, h1, s1);
      if (kb + 2 >= nkb) break;
      if (kb + 4 < nkb) load(kb + 4, l1, h1, s1);
      put(kb + 2, l2, h2, s2);
    }
    if (!ok && lane == 0) atomicCAS(&g_gemm_status, 0u, 7u);
  }

  // ---- epilogue ----
  pdl_wait();  // every thread: the previous kernel's outputs (the residual) are visible
  pdl_launch_dependents();
  if (warp >= 2 && warp < 2 + kDrainWarps) {
    // TMEM lane quarter (warp % 4) = rows 32 q .. 32 q + 31; two warps per quarter split the columns
    const bool have = __all_sync(0xffffffffu, tc::wait_until(accf, 0, deadline));
    if (!have && lane == 0) atomicCAS(&g_gemm_status, 0u, 8u);
    tc::fence_after_sync();
    const int q = warp & 3, part = (warp - 2) >> 2, nh = nmma / 2;
    const int row = q * 32 + lane;
    for (int c = part * nh; c < (part + 1) * nh; c += 8) {
      uint32_t r[8];
      tc::tmem_ld8(tmem + (static_cast<uint32_t>(q * 32) << 16) + c, r);
#pragma unroll
      for (int e = 0; e < 8; ++e) P[row * pstride + c + e] = __uint_as_float(r[e]);
    }
  }
  tc::fence_before_sync();
  if constexpr (CS > 1) cg::this_cluster().sync();
  else __syncthreads();
  // rows [r0, r0 + rows_r) of the tile: every rank's partial, summed in rank order
  const int rows_r = kRows / CS, r0 = rank * rows_r;
  const int row_base = tile * kRows + r0;
  if (threadIdx.x < 256) {
    const float *parts[CS];
#pragma unroll
    for (int qq = 0; qq < CS; ++qq) {
      if constexpr (CS > 1) parts[qq] = cg::this_cluster().map_shared_rank(P, qq);
      else parts[qq] = P;
    }
    // a thread owns 8 consecutive rows of one vector: 16-byte stores and residual loads
    if (a.swiglu) {
      // per 16-row group: rows 0-7 gate, 8-15 up -> 8 outputs
      const int H = a.N / 2, groups = rows_r / 16, items = a.n_vec * groups;
      for (int it = threadIdx.x; it < items; it += 256) {
        const int t = it / groups, gi = it % groups, rg = r0 + gi * 16;
        float g[8], u[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = u[e] = 0.f;
#pragma unroll
        for (int qq = 0; qq < CS; ++qq)
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            g[e] += parts[qq][(rg + e) * pstride + t];
            u[e] += parts[qq][(rg + 8 + e) * pstride + t];
          }
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float sv[2];
#pragma unroll
          for (int f = 0; f < 2; ++f) {
            const float gte = __bfloat162float(__float2bfloat16_rn(g[e + f]));
            const float up = __bfloat162float(__float2bfloat16_rn(u[e + f]));
            sv[f] = __bfloat162float(__float2bfloat16_rn(gte / (1.f + __expf(-gte)))) * up;
          }
          o[e / 2] = pack_bf16x2(sv[0], sv[1]);
        }
        *reinterpret_cast<uint4 *>(a.y + static_cast<int64_t>(t) * H + (row_base + gi * 16) / 2) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
    } else {
      // 8 rows a thread (4 in 8-CTA clusters, to occupy all 256 threads, measured slower)
      constexpr int kR = 8;
      const int groups = rows_r / kR, items = a.n_vec * groups;  // groups: 2..16, divides 32
      for (int b0 = 0; b0 < items; b0 += 256) {
        const int it = b0 + threadIdx.x;
        const bool valid = it < items;
        const int t = valid ? it / groups : 0, i0 = valid ? (it % groups) * kR : 0;
        const int grow0 = row_base + i0;
        unsigned long long key = 0ull;
        if (valid) {
          float v[kR];
#pragma unroll
          for (int e = 0; e < kR; ++e) v[e] = 0.f;
#pragma unroll
          for (int qq = 0; qq < CS; ++qq)
#pragma unroll
            for (int e = 0; e < kR; ++e) v[e] += parts[qq][(r0 + i0 + e) * pstride + t];
          const int64_t o = static_cast<int64_t>(t) * a.N + grow0;
          uint32_t rw[kR / 2];
          if (a.residual) {
            // the residual is added to the bf16-rounded projection (IRON adds two bf16 buffers)
            const uint4 rv = ld_act_v4(a.residual + o);
            rw[0] = rv.x, rw[1] = rv.y, rw[2] = rv.z, rw[3] = rv.w;
#pragma unroll
            for (int e = 0; e < kR; e += 2) {
              v[e] = __bfloat162float(__float2bfloat16_rn(v[e])) + bf16_lo(rw[e / 2]);
              v[e + 1] = __bfloat162float(__float2bfloat16_rn(v[e + 1])) + bf16_hi(rw[e / 2]);
            }
          }
          uint32_t w[kR / 2];
#pragma unroll
          for (int e = 0; e < kR; e += 2) w[e / 2] = pack_bf16x2(v[e], v[e + 1]);
          *reinterpret_cast<uint4 *>(a.y + o) = make_uint4(w[0], w[1], w[2], w[3]);
          if (a.amax) {
#pragma unroll
            for (int e = 0; e < kR; ++e) {
              const unsigned long long k = argmax_key((e & 1) ? bf16_hi(w[e / 2]) : bf16_lo(w[e / 2]), grow0 + e);
              key = k > key ? k : key;
            }
          }
        }
        if (a.amax) {  // the vector's best over the CTA's rows: one atomic per vector and slice
          for (int x = 1; x < groups; x <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, x);
            key = other > key ? other : key;
          }
          if (valid && (lane % groups) == 0) atomicMax(a.amax + t * 32 + ((grow0 >> 7) & 31), key);
        }
      }
    }
  }
  if constexpr (CS > 1) cg::this_cluster().sync();  // the other ranks have read this CTA's partial
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_free(tmem, cols);
}

}  // namespace s4tc

// ---- host side ---------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// K-major bf16 matrix [rows, K] with row pitch ld (elements): boxes of 64 x box_rows,
// 128-byte swizzle.
int make_tmap(CUtensorMap *m, const void *ptr, int rows, int K, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return IRON_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? IRON_OK : IRON_ERR_ARG;
}

// The output C [rows, cols] (row pitch ld elements) as the epilogue's TMA store sees
// it: boxes of 32 rows x box_cols columns, 64B swizzle for 32-column boxes (SwiGLU's
// 16-column boxes: 32B), matching stg64 / stg32.
int make_store_tmap(CUtensorMap *m, void *ptr, int rows, int cols, int64_t ld, int box_cols) {
  auto fn = encode_fn();
  if (!fn) return IRON_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), 32u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? IRON_OK : IRON_ERR_ARG;
}

// Pick the tile width: whole waves of 128 x BN tiles over the SMs, discounted for
// the shared-memory operand traffic of narrow tiles (a 128 x 128 MMA reads its
// operands from shared memory at the rate the SM supplies them; measured on B200 at
// M = 2048, K = 2048, N = 2048 / 3072 / 8192: per wave-slot 192-wide tiles run about
// 0.8 of the 256-wide tile's rate, 128-wide 0.59-0.69, 64-wide about 0.35; 192 wins
// where it fills the waves better, e.g. N = 3072: 970 against 917 TFLOP/s).
int pick_bn(int M, int N, int sms) {
  const int cand[4] = {256, 192, 128, 64};
  const double smem_eff[4] = {1.0, 0.8, 0.62, 0.35};
  int best = 64;
  double best_e = -1;
  for (int i = 0; i < 4; ++i) {
    const int bn = cand[i];
    if (N < bn && bn != 64) continue;
    const int64_t tiles = static_cast<int64_t>((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double e = static_cast<double>(tiles) / (waves * sms) * smem_eff[i] *
                     (static_cast<double>(N) / (((N + bn - 1) / bn) * bn));
    if (e > best_e + 1e-9) {
      best_e = e;
      best = bn;
    }
  }
  return best;
}

template <int BN>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tc, int M, int N, int K,
                const uint16_t *R, int64_t ldr, Epi epi, cudaStream_t s, bool pdl) {
  using G = Cfg<BN>;
  static PerDeviceOnce attr_set;  // per instantiation and device: the shared memory opt-in
  const int ast = attr_set.run([]() {
    return call_status(cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem));
  });
  if (ast != IRON_OK) return ast;
  const int64_t tiles = static_cast<int64_t>((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  dim3 grid(static_cast<unsigned>(tiles < sm_count() ? tiles : sm_count()));
  return launch(gemm_tc_kernel<BN>, grid, dim3(kThreads), G::kSmem, s, pdl, ta, tb, tc, M, N, K, R, ldr, epi);
}

namespace s4tc {
template <int CS>
static int launch_cs(const CUtensorMap &tx, const Args &a, int nmma, int tiles, bool pdl, cudaStream_t s) {
  static PerDeviceOnce attr_set;  // per instantiation and device: the shared memory opt-in
  const int ast = attr_set.run([]() {
    return call_status(cudaFuncSetAttribute(s4tc_kernel<CS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  });
  if (ast != IRON_OK) return ast;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles * CS));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, s4tc_kernel<CS>, tx, a, nmma);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}
}  // namespace s4tc
}  // namespace gemm

// The tensor-core form of the int4 g32 GEMV for 33..64 vectors (declared in s4.cuh).
// IRON_ERR_UNSUPPORTED: not this form's shape (N % 128, vector count); the caller then
// runs the mma.sync GEMV.
int launch_s4_tc(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                 const uint16_t *residual, int swiglu, unsigned long long *amax, bool pdl, cudaStream_t s) {
  using namespace gemm::s4tc;
  // from 33 vectors on (B200 decode, ms per step with / without this form: 64 vectors
  // 2.29 / 2.93; 32: 1.66 / 1.54; 16: 1.28 / 0.95)
  if (n_vec <= 32 || n_vec > kMaxVec || N % kRows || K % kKB) return IRON_ERR_UNSUPPORTED;
  if (!aligned16(y) || (residual && !aligned16(residual))) return IRON_ERR_UNSUPPORTED;
  const int nmma = (n_vec + 15) / 16 * 16;
  CUtensorMap tx;
  const int st = gemm::make_tmap(&tx, x, n_vec, K, K, nmma);
  if (st != IRON_OK) return st;
  const Args a{packed, y, residual, amax, N, K, n_vec, swiglu};
  const int tiles = N / kRows, cpt = K / kKB;
  // split K over a cluster while the doubled grid still fits one wave (and every CTA
  // keeps at least two k-blocks)
  int cs = 1;
  while (cs < 8 && tiles * cs * 2 <= sm_count() && cpt >= cs * 4) cs *= 2;
  switch (cs) {
    case 1: return gemm::s4tc::launch_cs<1>(tx, a, nmma, tiles, pdl, s);
    case 2: return gemm::s4tc::launch_cs<2>(tx, a, nmma, tiles, pdl, s);
    case 4: return gemm::s4tc::launch_cs<4>(tx, a, nmma, tiles, pdl, s);
    default: return gemm::s4tc::launch_cs<8>(tx, a, nmma, tiles, pdl, s);
  }
}

}  // namespace iron

using namespace iron;
using namespace iron::gemm;

extern "C" int iron_gemm_bf16(const uint16_t *A, const uint16_t *B, uint16_t *C, int M, int N, int K,
                              int64_t lda, int64_t ldb, int64_t ldc, const uint16_t *residual, int64_t ldr,
                              int epilogue, int clamp, float clamp_lo, float clamp_hi, int block_n, unsigned flags,
                              void *stream) {
  if (!A || !B || !C) return IRON_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return IRON_ERR_SHAPE;
  const int act = epilogue & 0xff, floor_rnd = (epilogue >> 8) & 1;
  if (act > 4 || (epilogue & ~0x1ff) || (clamp && !(clamp_lo <= clamp_hi))) return IRON_ERR_ARG;
  if (act == 4 && (residual || clamp || floor_rnd || N % 16)) return IRON_ERR_ARG;
  const int64_t out_cols = act == 4 ? N / 2 : N;
  if (K % 8 || N % 8 || lda < K || ldb < K || ldc < out_cols) return IRON_ERR_SHAPE;
  if (residual && ldr < N) return IRON_ERR_SHAPE;
  if (lda % 8 || ldb % 8 || ldc % 8 || !aligned16(A) || !aligned16(B) || !aligned16(C)) return IRON_ERR_ALIGN;
  if (residual && (ldr % 8 || !aligned16(residual))) return IRON_ERR_ALIGN;
  int bn = block_n ? block_n : pick_bn(M, N, sm_count());
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256) return IRON_ERR_ARG;
  CUtensorMap ta, tb, tc;
  int st = make_tmap(&ta, A, M, K, lda, BM);
  if (st == IRON_OK) st = make_tmap(&tb, B, N, K, ldb, bn);
  if (st == IRON_OK) st = make_store_tmap(&tc, C, M, static_cast<int>(out_cols), ldc, act == 4 ? 16 : 32);
  if (st != IRON_OK) return st;
  Epi epi{act, floor_rnd, clamp, clamp_lo, clamp_hi};
  auto s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  switch (bn) {
    case 256: return launch_gemm<256>(ta, tb, tc, M, N, K, residual, ldr, epi, s, pdl);
    case 192: return launch_gemm<192>(ta, tb, tc, M, N, K, residual, ldr, epi, s, pdl);
    case 128: return launch_gemm<128>(ta, tb, tc, M, N, K, residual, ldr, epi, s, pdl);
    default: return launch_gemm<64>(ta, tb, tc, M, N, K, residual, ldr, epi, s, pdl);
  }
}

extern "C" int iron_gemm_status(int reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v)) != cudaSuccess) return launch_status();
  if (reset) {
    unsigned z = 0;
    if (cudaMemcpyToSymbol(g_gemm_status, &z, sizeof(z)) != cudaSuccess) return launch_status();
  }
  return v ? IRON_ERR_TIMEOUT : IRON_OK;
}
