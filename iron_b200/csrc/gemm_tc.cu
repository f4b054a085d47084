// bf16 GEMM on the 5th-generation tensor cores: C = epilogue(A . B^T).
//
// Replaces the prefill projections of IRON's GEMM operators
// (iron/operators/gemm/op.py:21-231, iron/operators/flm/gemm/op.py:64-499;
// goldens gemm/reference.py:7-18 and flm/gemm/reference.py:8-57): A [M, K] and
// B [N, K] are K-major bf16 in HBM, C [M, N] bf16 row-major, fp32 accumulation.
// The flm epilogue (activation after the bf16 conversion, then an optional
// clamp) is fused into the TMEM drain.
//
// One CTA computes one 128 x BN output tile with four warps:
//   warp 0, one thread : TMA producer -- A and B k-blocks (64 wide, 128-byte
//                        swizzle) into a ring of shared-memory stages;
//   warp 1, one thread : MMA issuer -- four tcgen05.mma (K = 16) per stage into
//                        a 128 x BN fp32 accumulator in TMEM, a commit per
//                        stage releasing it to the producer, a final commit;
//   warp 2            : allocates / frees the TMEM columns;
//   all four warps    : epilogue -- each warp drains its 32 TMEM lanes (rows),
//                        32 columns at a time, converts, applies the
//                        activation and writes 64 contiguous bytes per row.
// Every mbarrier wait is bounded by a 2-second deadline; a timeout sets the
// status word and the CTA leaves after freeing its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace iron {
namespace gemm {

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 128;
constexpr uint64_t kDeadlineNs = 2000000000ull;

__device__ unsigned g_gemm_status;  // 0 = ok, else the first failing role's code

struct Epi {
  int mode;   // 0 none, 1 gelu (x * sigmoid(1.702 x)), 2 silu, 3 sigmoid
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

template <int BN>
struct Cfg {
  static constexpr int kStageA = BM * BK * 2;
  static constexpr int kStageB = BN * BK * 2;
  static constexpr int kStage = kStageA + kStageB;
  static constexpr int kStages = (192 * 1024) / kStage;
  static constexpr int kSmem = 1024 + kStages * kStage + 256;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   uint16_t *__restrict__ C, int M, int N, int K, int64_t ldc, Epi epi) {
  using G = Cfg<BN>;
  constexpr int S = G::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 128-byte swizzle atoms need 1024-B alignment
  const uint32_t stage0 = base;
  const uint32_t bars = base + S * G::kStage;  // full[S], empty[S], accum
  const uint32_t full0 = bars, empty0 = bars + 8 * S, accum = bars + 16 * S;
  const uint32_t tslot = accum + 8;
  uint32_t *tslot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tslot - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int kb_count = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
    for (int s = 0; s < S; ++s) {
      tc::mbar_init_u32(full0 + 8 * s, 1);
      tc::mbar_init_u32(empty0 + 8 * s, 1);
    }
    tc::mbar_init_u32(accum, 1);
    mbar_init_fence();
  }
  if (warp == 2) tc::tmem_alloc(tslot, BN);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot_ptr;
  pdl_wait();  // A is the previous kernel's output; the prologue above overlapped it
  const uint64_t deadline = tc::globaltimer_ns() + kDeadlineNs;

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // ---- producer ----
    int issued = 0;
    for (int kb = 0; kb < kb_count; ++kb) {
      const int s = kb % S;
      const uint32_t par = ((kb / S) & 1) ^ 1;
      if (!tc::wait_until(empty0 + 8 * s, par, deadline)) {
        ok = false;
        break;
      }
      const uint32_t sa = stage0 + s * G::kStage, sb = sa + G::kStageA;
      tc::expect_tx(full0 + 8 * s, G::kStage);
      tc::tma_load_2d(sa, &tmA, kb * BK, m0, full0 + 8 * s);
      tc::tma_load_2d(sb, &tmB, kb * BK, n0, full0 + 8 * s);
      issued = kb + 1;
    }
    if (!ok) {
      atomicCAS(&g_gemm_status, 0u, 1u);
      // let copies already in flight land before the CTA's shared memory goes away
      for (int kb = (issued > S ? issued - S : 0); kb < issued; ++kb)
        tc::wait_until(full0 + 8 * (kb % S), (kb / S) & 1, tc::globaltimer_ns() + 100000000ull);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
    for (int kb = 0; kb < kb_count; ++kb) {
      const int s = kb % S;
      if (!tc::wait_until(full0 + 8 * s, (kb / S) & 1, deadline)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t sa = stage0 + s * G::kStage, sb = sa + G::kStageA;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        tc::mma_bf16(tmem, tc::sdesc_kmajor_sw128(sa + 32 * k), tc::sdesc_kmajor_sw128(sb + 32 * k), idesc,
                     (kb | k) != 0);
      }
      tc::mma_commit(empty0 + 8 * s);  // stage free once these MMAs have read it
    }
    if (!ok) atomicCAS(&g_gemm_status, 0u, 2u);
    tc::mma_commit(accum);  // accumulator complete (or the MMAs issued so far, on error)
  }
  __syncwarp();
  pdl_launch_dependents();

  // ---- epilogue: TMEM -> registers -> bf16 -> HBM ----
  // warp-uniform verdict: the TMEM loads below are .sync.aligned
  const bool have = __all_sync(0xffffffffu, tc::wait_until(accum, 0, deadline));
  tc::fence_after_sync();
  if (!have) {
    if (lane == 0) atomicCAS(&g_gemm_status, 0u, 3u);
  } else {
    const int row = m0 + warp * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tc::tmem_ld32(trow + c, r);
      if (row < M) {
        uint16_t *dst = C + static_cast<int64_t>(row) * ldc + n0 + c;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (n0 + c + 8 * q + 8 <= N) {
            uint4 v;
            v.x = pack_bf16x2(apply_epi(__uint_as_float(r[8 * q + 0]), epi), apply_epi(__uint_as_float(r[8 * q + 1]), epi));
            v.y = pack_bf16x2(apply_epi(__uint_as_float(r[8 * q + 2]), epi), apply_epi(__uint_as_float(r[8 * q + 3]), epi));
            v.z = pack_bf16x2(apply_epi(__uint_as_float(r[8 * q + 4]), epi), apply_epi(__uint_as_float(r[8 * q + 5]), epi));
            v.w = pack_bf16x2(apply_epi(__uint_as_float(r[8 * q + 6]), epi), apply_epi(__uint_as_float(r[8 * q + 7]), epi));
            *reinterpret_cast<uint4 *>(dst + 8 * q) = v;
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 2) tc::tmem_free(tmem, BN);
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

// Pick the tile width: whole waves of 128 x BN tiles over the SMs, discounted for
// the shared-memory operand traffic of narrow tiles.
int pick_bn(int M, int N, int sms) {
  const int cand[3] = {256, 128, 64};
  const double smem_eff[3] = {1.0, 0.95, 0.66};
  int best = 64;
  double best_e = -1;
  for (int i = 0; i < 3; ++i) {
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
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, uint16_t *C, int M, int N, int K, int64_t ldc,
                Epi epi, cudaStream_t s, bool pdl) {
  using G = Cfg<BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem) !=
        cudaSuccess)
      return launch_status();
    attr_set[dev] = true;
  }
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  return launch(gemm_tc_kernel<BN>, grid, dim3(kThreads), G::kSmem, s, pdl, ta, tb, C, M, N, K, ldc, epi);
}

}  // namespace gemm
}  // namespace iron

using namespace iron;
using namespace iron::gemm;

extern "C" int iron_gemm_bf16(const uint16_t *A, const uint16_t *B, uint16_t *C, int M, int N, int K,
                              int64_t lda, int64_t ldb, int64_t ldc, int epilogue, int clamp, float clamp_lo,
                              float clamp_hi, int block_n, unsigned flags, void *stream) {
  if (!A || !B || !C) return IRON_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return IRON_ERR_SHAPE;
  if (K % 8 || N % 8 || lda < K || ldb < K || ldc < N) return IRON_ERR_SHAPE;
  if (lda % 8 || ldb % 8 || ldc % 8 || !aligned16(A) || !aligned16(B) || !aligned16(C)) return IRON_ERR_ALIGN;
  const int act = epilogue & 0xff, floor_rnd = (epilogue >> 8) & 1;
  if (act > 3 || (epilogue & ~0x1ff) || (clamp && !(clamp_lo <= clamp_hi))) return IRON_ERR_ARG;
  int bn = block_n ? block_n : pick_bn(M, N, sm_count());
  if (bn != 64 && bn != 128 && bn != 256) return IRON_ERR_ARG;
  CUtensorMap ta, tb;
  int st = make_tmap(&ta, A, M, K, lda, BM);
  if (st == IRON_OK) st = make_tmap(&tb, B, N, K, ldb, bn);
  if (st != IRON_OK) return st;
  Epi epi{act, floor_rnd, clamp, clamp_lo, clamp_hi};
  auto s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  switch (bn) {
    case 256: return launch_gemm<256>(ta, tb, C, M, N, K, ldc, epi, s, pdl);
    case 128: return launch_gemm<128>(ta, tb, C, M, N, K, ldc, epi, s, pdl);
    default: return launch_gemm<64>(ta, tb, C, M, N, K, ldc, epi, s, pdl);
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
