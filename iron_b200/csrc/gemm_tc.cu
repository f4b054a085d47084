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

#include "common.cuh"
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

}  // namespace gemm
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
