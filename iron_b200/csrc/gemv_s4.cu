// int4 group-32 GEMV (the fused Dequant + GEMV).
//
// Weights are first repacked (iron_pack_int4g32) into units of one 16-row tile x
// 128 k (4 groups): 1024 code bytes in the order the MMA fragments want them
// (lane-major, so every warp load is 512 contiguous bytes; within a 32-bit word the
// nibbles of k 2q and 2q+1 sit at bits 4q and 16+4q) followed by the tile's
// 16 x 4 bf16 scales (128 B). A unit is 1152 bytes; units are stored tile-major.
//
// One CTA of four warps per 16-row tile; its warps split the tile's units (and a
// thread-block cluster splits K further when the matrix has too few tiles to put
// two CTAs on every SM). Every warp issues the loads of its units straight into
// registers, launches its dependents and only then waits for the previous kernel
// (griddepcontrol.wait): the weights never depend on it, so consecutive GEMVs of
// an inference graph stream their weights while their predecessor finishes.
//
// Codes are unpacked with a LOP3 bf16 "magic number" into the exact dequantized
// weights bf16(q * scale) -- the values IRON's Dequant produces -- and reduced
// against the activations with bf16 MMAs, fp32 accumulate, used as a warp-wide
// dot-product engine. Warp partials are summed in a fixed order through shared
// memory (and distributed shared memory across a cluster), so results are
// bitwise deterministic.
#include <cooperative_groups.h>
#include <cstring>

#include "common.cuh"
#include "s4.cuh"

namespace cg = cooperative_groups;

namespace iron {

constexpr int kS4UnitBytes = 1152;
// q4 (asymmetric) units append 128 bytes of group mins, laid out as the scales: 1280 B.
constexpr int kQ4UnitBytes = 1280;
constexpr int kS4CodeBytes = 1024;

struct S4Range {
  int b, e;
};
// Part i of `parts` near-equal contiguous parts of [b, e).
__device__ __forceinline__ S4Range s4_split(int b, int e, int parts, int i) {
  const int n = e - b;
  return {b + i * n / parts, b + (i + 1) * n / parts};
}

constexpr int kS4ArgmaxSlots = 32;  // argmax key slots per vector

// Tensor-parallel all-reduce fused into the GEMV epilogue (row-parallel layers):
// every rank pushes its fp32 partial of each finished 16-row tile into every rank's
// receive buffer over NVLink (peer stores of value + flag), waits for all sources'
// values of the tile in its own buffer and sums them in source order -- so every rank
// holds the bitwise-identical sum without a separate collective. recv[r]: rank r's
// buffer (peer-mapped for r != rank).
constexpr int kS4MaxWorld = 8;
struct S4AllReduce {
  int world, rank;
  float *recv[kS4MaxWorld];       // [world (source), N, n_vec] x (fp32 value, flag) 8-byte slots, zero between uses
  unsigned *status;               // non-zero: a wait for a peer's tile gave up
  unsigned wait_us;               // give-up time of a wait for a peer's value (0: 1 s)
};

struct S4Epi {
  const uint16_t *residual;
  int swiglu;
  const uint16_t *norm_w;
  float eps;
  unsigned long long *amax;
  S4AllReduce ar;  // ar.world > 1: all-reduce the output over the ranks first
  int x_ro;        // IRON_FLAG_X_READONLY: x through the read-only path, else L2-coherent loads
  // RMSNorm folded into the decode chain (single-tile kernels, n_vec <= 8):
  const float *ss_in;    // [n_vec, K/16] partial sums of squares of the unweighted input rows
  float *ss_out;         // [n_vec, N/16] partial sums of squares of y (per 16-row tile)
  uint16_t *yw;          // [n_vec, N] bf16(y * yw_w): the next GEMV's input
  const uint16_t *yw_w;  // [N] the next RMSNorm's weights
  int asym;              // q4 units (min + scale * code, 1280 B) instead of int4 g32
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned r;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}
__device__ __forceinline__ uint64_t s4_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Warp 0 of the CTA finishing `tile`: exchange the tile's partial (v, rows gid / gid + 8,
// vectors 2 tid + e) with the other ranks and return the sum over ranks in v. Every value
// travels as one 8-byte store of (fp32 bits, flag 1) into the receiver's slot [source,
// row, vector] -- a single NVLink transaction, so the receiver sees the value whenever it
// sees the flag and no memory fence is needed; the receiver clears the slot after use
// (the next write to it comes one all-reduce site later, after this rank has passed it).
__device__ __forceinline__ void st_pair_sys(unsigned long long *p, float v) {
  const unsigned long long w = (1ull << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_pair_sys(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

__device__ __forceinline__ void s4_allreduce_tile(float (&v)[4], int tile, int N, int n_vec, const S4AllReduce &ar) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tid = lane & 3;
  // static indices into ar.recv (a runtime index would copy the parameter to local memory)
  float *own = ar.recv[0];
#pragma unroll
  for (int dst = 0; dst < kS4MaxWorld; ++dst) {
    if (dst >= ar.world) break;
    if (dst == ar.rank) own = ar.recv[dst];
    unsigned long long *rb = reinterpret_cast<unsigned long long *>(ar.recv[dst]) +
                             static_cast<int64_t>(ar.rank) * N * n_vec;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = tile * 16 + gid + ((e >> 1) << 3), vv = tid * 2 + (e & 1);
      if (vv < n_vec) st_pair_sys(rb + static_cast<int64_t>(row) * n_vec + vv, v[e]);
    }
  }
  unsigned long long *mine = reinterpret_cast<unsigned long long *>(own);
  const uint64_t limit_ns = ar.wait_us ? static_cast<uint64_t>(ar.wait_us) * 1000ull : 1000000000ull;
  bool gave_up = false;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int row = tile * 16 + gid + ((e >> 1) << 3), vv = tid * 2 + (e & 1);
    float sum = 0.f;
    if (vv < n_vec) {
      for (int src = 0; src < ar.world; ++src) {
        unsigned long long *slot = mine + (static_cast<int64_t>(src) * N + row) * n_vec + vv;
        unsigned long long w = ld_pair_sys(slot);
        uint64_t start = 0;
        for (uint32_t i = 0; (w >> 32) == 0ull && !gave_up; ++i) {
          if ((i & 63u) == 0u) {
            if (ld_acquire_sys(ar.status) != 0u) gave_up = true;  // an earlier wait gave up: fail fast
            const uint64_t t = s4_now_ns();
            if (start == 0) start = t;
            else if (t - start > limit_ns) {  // no value from the peer within the limit
              atomicOr(ar.status, 1u);
              gave_up = true;
            }
          }
          w = ld_pair_sys(slot);
        }
        sum += __uint_as_float(static_cast<unsigned>(w & 0xffffffffull));
        *slot = 0ull;
      }
    }
    v[e] = sum;
  }
}

__device__ __forceinline__ unsigned long long s4_argmax_key(float v, int row) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (v != v) u = 0u;  // NaN never wins
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned>(~row);
}

// Store a finished 16-row tile (C-fragment layout v). swiglu == 0: rows as they
// are, plus the residual. swiglu == 1: the tile's rows 0-7 are gate rows and
// 8-15 the matching up rows of output rows 8*tile..8*tile+7 (y has N/2 columns):
// y = bf16(bf16(silu(bf16(gate))) * bf16(up)), the rounding sequence of IRON's
// SwiGLUDecode (iron/operators/swiglu_decode/reference.py:49-53).
// What a GEMV does around the dot products: an RMSNorm of x first (norm_w != null),
// a residual add or the SwiGLU of interleaved gate/up rows on the output, and the
// greedy argmax of each output vector (amax != null: 64-bit keys, larger value then
// lower row wins).
// The residual a tile's store adds, res_s[v * 16 + r] = residual[v, 16 tile + r]:
// every thread requests its share right after griddepcontrol.wait (it was written
// before the wait returned). Up to 16 vectors (one value per thread) it stays in a
// register until the thread's dot products are done, so nothing waits on it early;
// wider tiles park it at once (8 values per thread would spill).
template <int NT, int kThreads>
struct S4Residual {
  static constexpr int kPer = (16 * 8 * NT + kThreads - 1) / kThreads;
  static constexpr bool kHold = NT <= 2;
  float r[kHold ? kPer : 1];
  __device__ __forceinline__ void load(float *res_s, int tile, int N, int n_vec, const uint16_t *residual) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + k * kThreads;
      const float v = i < 16 * n_vec
                          ? bf16_bits_to_float(ld_act_u16(residual + static_cast<int64_t>(i >> 4) * N + tile * 16 + (i & 15)))
                          : 0.f;
      if constexpr (kHold) r[k] = v;
      else if (i < 16 * n_vec) res_s[i] = v;
    }
  }
  __device__ __forceinline__ void park(float *res_s, int n_vec) const {
    if constexpr (kHold) {
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int i = threadIdx.x + k * kThreads;
        if (i < 16 * n_vec) res_s[i] = r[k];
      }
    }
  }
};

// The chain writer (yw != null): y2 = bf16(y * w[row]) into yw and, per vector, the sum
// of squares of the tile's 16 stored (bf16) y values into ss_out[v, tile] -- summed over
// the rows in a fixed order (shuffles), so the RMSNorm scale built from them downstream
// is bitwise reproducible. w_lo / w_hi: w of rows gid / gid + 8.
template <int NT>
__device__ __forceinline__ void s4_store(const float (&v)[NT][4], int tile, int N, int n_vec,
                                         uint16_t *__restrict__ y, const float *res_s, int swiglu,
                                         unsigned long long *amax = nullptr, uint16_t *yw = nullptr,
                                         float *ss_out = nullptr, float w_lo = 0.f, float w_hi = 0.f) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tid = lane & 3;
  const int row0 = tile * 16;
  if (swiglu) {
    const int H = N / 2;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int vv = t * 8 + tid * 2 + e;
        if (vv < n_vec) {
          const float gte = __bfloat162float(__float2bfloat16_rn(v[t][e]));
          const float up = __bfloat162float(__float2bfloat16_rn(v[t][e + 2]));
          const float sw = __bfloat162float(__float2bfloat16_rn(gte / (1.f + __expf(-gte))));
          y[static_cast<int64_t>(vv) * H + tile * 8 + gid] = float_to_bf16_bits(sw * up);
        }
      }
    return;
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    unsigned long long best[2] = {0ull, 0ull};  // per vector 2tid + (e & 1)
    float sq[2] = {0.f, 0.f};                   // per vector 2tid + (e & 1): chain writer
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = row0 + gid + ((e >> 1) << 3);
      const int vv = t * 8 + tid * 2 + (e & 1);
      if (vv < n_vec) {
        const int64_t o = static_cast<int64_t>(vv) * N + row;
        float r = v[t][e];
        // the residual is added to the bf16-rounded projection, as IRON adds two
        // bf16 buffers (iron/operators/elementwise_add/reference.py:7-9)
        if (res_s) r = __bfloat162float(__float2bfloat16_rn(r)) + res_s[vv * 16 + (row - row0)];
        const uint16_t yb = float_to_bf16_bits(r);
        y[o] = yb;
        if (yw) {
          const float yf = bf16_bits_to_float(yb);
          yw[o] = float_to_bf16_bits(yf * ((e >> 1) ? w_hi : w_lo));
          sq[e & 1] += yf * yf;
        }
        if (amax) {
          const unsigned long long k = s4_argmax_key(bf16_bits_to_float(yb), row);
          best[e & 1] = k > best[e & 1] ? k : best[e & 1];
        }
      }
    }
    if (yw) {
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int x = 4; x <= 16; x <<= 1) sq[q] += __shfl_xor_sync(0xffffffffu, sq[q], x);
      if (gid == 0)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int vv = t * 8 + tid * 2 + q;
          if (vv < n_vec) ss_out[static_cast<int64_t>(vv) * (N / 16) + tile] = sq[q];
        }
    }
    if (amax) {
      // best (value, then lowest row) of the tile's 16 rows per vector: reduce over the
      // 8 lanes of each tid, then one atomic per tile and vector, into one of
      // kS4ArgmaxSlots slots (spreads the contention of 8016 tiles over L2 lines)
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int x = 4; x <= 16; x <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[q], x);
          best[q] = other > best[q] ? other : best[q];
        }
      if (gid == 0)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int vv = t * 8 + tid * 2 + q;
          if (vv < n_vec) atomicMax(amax + vv * kS4ArgmaxSlots + (tile & (kS4ArgmaxSlots - 1)), best[q]);
        }
    }
  }
}

// One 16-row x 128-k unit against the activations: per 32-k group the codes become the
// exact dequantized weights bf16(q * s) -- IRON's Dequant values -- as bf16x2 pairs (LOP3
// magic number, exact subtract, one rounding multiply by the group scale) and two MMAs
// accumulate them against x in fp32. The B fragments are x's 16-byte loads as they sit
// in memory (this lane's 8 consecutive k of a group); lanes of vectors past n_vec read
// the last vector (their columns are never stored), so up to 8 vectors no load is
// predicated. (Applying
// the group scale to the MMA's fp32 group sums instead measured no faster on B200 and
// would change the results from IRON's dequantize-then-GEMV by up to ~1e-2.)
// kAsym: the q4 (min + scale * code) weights: codes unsigned, mn the row pair's bf16
// group mins laid out as sc (q4x2_dequant_: bf16(min + scale * code), one rounding).
template <int NT, bool kShared = false, bool kRO = false, bool kAsym = false>
__device__ __forceinline__ void s4_unit_gx(float (&acc)[2][NT][4], const uint4 &clo, const uint4 &chi,
                                           const uint4 &sc, const uint16_t *__restrict__ x, int K,
                                           int n_vec, int kbase, int ldx = -1, int xoff = 0,
                                           const uint4 &mn = make_uint4(0u, 0u, 0u, 0u)) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tid = lane & 3;
  const uint32_t wl[4] = {clo.x, clo.y, clo.z, clo.w};
  const uint32_t wh[4] = {chi.x, chi.y, chi.z, chi.w};
  const uint32_t sl2[2] = {sc.x, sc.y}, sh2[2] = {sc.z, sc.w};
  uint4 xr[4][NT];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      // single-tile form: every lane loads (lanes past n_vec the last vector); wider
      // tiles predicate (their register budget has no room for the extra addresses)
      const int vv = NT == 1 ? min(gid, n_vec - 1) : t * 8 + gid;
      if (NT == 1 || vv < n_vec) {
        if constexpr (kShared)
          xr[j][t] = *reinterpret_cast<const uint4 *>(x + vv * ldx + kbase - xoff + j * 32 + tid * 8);
        else {
          const uint16_t *px = x + static_cast<int64_t>(vv) * K + kbase + j * 32 + tid * 8;
          if constexpr (kRO) xr[j][t] = __ldg(reinterpret_cast<const uint4 *>(px));
          else xr[j][t] = ld_act_v4(px);
        }
      } else {
        xr[j][t] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sel = (j & 1) ? 0x3232u : 0x1010u;
    const uint32_t s2_lo = prmt_(sl2[j >> 1], sl2[j >> 1], sel);
    const uint32_t s2_hi = prmt_(sh2[j >> 1], sh2[j >> 1], sel);
    uint32_t pl[4], ph[4];
    if constexpr (kAsym) {
      const uint32_t ml2[2] = {mn.x, mn.y}, mh2[2] = {mn.z, mn.w};
      const uint32_t m2_lo = prmt_(ml2[j >> 1], ml2[j >> 1], sel);
      const uint32_t m2_hi = prmt_(mh2[j >> 1], mh2[j >> 1], sel);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        pl[q] = q4x2_dequant_(wl[j] >> (4 * q), s2_lo, m2_lo);
        ph[q] = q4x2_dequant_(wh[j] >> (4 * q), s2_hi, m2_hi);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        pl[q] = s4x2_dequant_(wl[j] >> (4 * q), s2_lo);
        ph[q] = s4x2_dequant_(wh[j] >> (4 * q), s2_hi);
      }
    }
    const uint32_t A0[4] = {pl[0], ph[0], pl[1], ph[1]};
    const uint32_t A1[4] = {pl[2], ph[2], pl[3], ph[3]};
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint4 e = xr[j][t];
      mma_bf16_16816(acc[j & 1][t], A0, e.x, e.y);  // k (0,1) / (2,3) of this lane's 8
      mma_bf16_16816(acc[j & 1][t], A1, e.z, e.w);  // k (4,5) / (6,7)
    }
  }
}

// Tile kernel: one CTA of four warps per 16-row tile (or per K-slice of a tile
// when a cluster splits K), every warp loading all of its units straight into
// registers before griddepcontrol.wait; partials reduced through shared memory
// and, across a cluster, distributed shared memory.
// Warps per CTA and units each warp loads per round (all at once). Up to 16 vectors:
// 8 warps x 2 units (a 16-unit K = 2048 tile entirely in flight, 59 registers --
// measured on B200: 3.76 us per config-2 launch against 5.3 us at 4 x 4); more
// vectors keep 4 x 4 (the reduction buffer and the wider accumulators).
template <int NT>
constexpr int s4_warps() { return NT <= 2 ? 8 : 4; }
// CTAs per SM the register budget must allow: single-tile (<= 8 vector) kernels keep
// four 8-warp CTAs per SM (<= 64 registers a thread; at 66 registers the occupancy cliff
// to 3 CTAs per SM put config 2's 512 CTAs into two waves: 5.8 against 3.5 us per
// launch); the wider tiles (and the fused-norm and q4 forms) keep the compiler's own choice (0).
template <int NT, bool kNorm>
constexpr int s4_min_ctas() { return (NT == 1 && !kNorm) ? 4 : 0; }
template <int NT>
constexpr int s4_units() { return NT <= 2 ? 2 : 4; }
// kW (single-tile kernels; 0: the defaults above). kW = 4: CTAs of 4 warps, 8 per SM, for matrices with more tiles
// than one wave of 8-warp CTAs holds (the gate / up projection, the lm-head): the
// smaller CTAs all fit in one wave or retire in finer steps (B200, 1 vector: gate / up
// 5.67 against 6.17 us, lm-head 35.3 against 38.0 us per launch).
// kW = 16: CTAs of 16 warps, 2 per SM, in place of a 2-CTA cluster splitting K (the QKV and
// O projections: one CTA per tile) -- the same warps per tile without the cluster barrier,
// which with the skew between the two CTAs' SMs cost 0.6-1 us of a B200 decode GEMV
// (decode step 0.4215 -> 0.4075 ms).
template <int NT, int kW>
constexpr int s4_cta_warps() { return (kW && NT == 1) ? kW : s4_warps<NT>(); }
template <int NT, bool kNorm, int kW>
constexpr int s4_cta_min() { return (kW == 4 && NT == 1) ? 8 : (kW == 16 && NT == 1) ? 2 : s4_min_ctas<NT, kNorm>(); }

// kNorm: the RMSNorm prologue (n_vec <= 8) -- x normalised into shared memory first.
// (Staging a plain x the same way measured slower on B200: 4.16 against 3.77 us per
// config-2 launch; the per-unit L1 reads overlap better than one synchronised copy.)
// kChain (NT == 1): the decode chain's folded RMSNorm (S4Epi ss_in / ss_out / yw); a
// separate instantiation, so the plain GEMV carries none of its shared memory or code.
template <int NT, int CS, bool kNorm = false, bool kAR = false, bool kRO = false, bool kChain = false,
          bool kAsym = false, int kW = 0>
__global__ void __launch_bounds__(32 * s4_cta_warps<NT, kW>(), s4_cta_min<NT, kNorm || kAsym, kW>())
gemv_s4g32_tile_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ x,
                       uint16_t *__restrict__ y, int N, int K, int n_vec, S4Epi epi) {
  constexpr int kT4Warps = s4_cta_warps<NT, kW>();
  constexpr int kT4Units = s4_units<NT>();
  __shared__ float red[(kT4Warps + CS) * NT * 128];
  extern __shared__ __align__(16) uint16_t xs_norm[];  // [n_vec, this CTA's k range] when staged
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid = lane & 3;
  const int rank = (CS > 1) ? static_cast<int>(blockIdx.x % CS) : 0;
  const int tile = blockIdx.x / CS;
  const int cpt = K / 128;
  const S4Range kr = s4_split(0, cpt, CS * kT4Warps, rank * kT4Warps + warp);  // my chunks
  constexpr int kUnit = kAsym ? kQ4UnitBytes : kS4UnitBytes;
  const uint8_t *base = packed + (static_cast<int64_t>(tile) * cpt) * kUnit;

  float acc[2][NT][4];  // two accumulator sets (even / odd groups): two independent MMA chains
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[a][t][0] = acc[a][t][1] = acc[a][t][2] = acc[a][t][3] = 0.f;

  uint4 lo[kT4Units], hi[kT4Units], sc[kT4Units], mn[kAsym ? kT4Units : 1];
  auto load = [&](int c0) {
#pragma unroll
    for (int u = 0; u < kT4Units; ++u) {
      if (c0 + u < kr.e) {
        const uint8_t *p = base + static_cast<int64_t>(c0 + u) * kUnit;
        lo[u] = ld_stream_v4(p + lane * 16);
        hi[u] = ld_stream_v4(p + 512 + lane * 16);
        sc[u] = ld_stream_v4(p + kS4CodeBytes + gid * 16);
        if constexpr (kAsym) mn[u] = ld_stream_v4(p + kS4UnitBytes + gid * 16);
      }
    }
  };
  load(kr.b);
  constexpr bool norm = kNorm && NT == 1;
  const S4Range cr = s4_split(0, cpt, CS, rank);  // this CTA's units (all its warps')
  const int kc0 = cr.b * 128, klen = (cr.e - cr.b) * 128;
  constexpr int kThr = 32 * kT4Warps;
  uint4 wreg[2];  // the norm weights of this thread's positions (klen <= 2048): never depend on the previous kernel
  if constexpr (norm) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int k = threadIdx.x * 8 + j * kThr * 8;
      if (k < klen) wreg[j] = __ldg(reinterpret_cast<const uint4 *>(epi.norm_w + kc0 + k));
    }
  }
  // the chain's small inputs land in shared memory by asynchronous copies (no registers
  // held across the main loop): the writer's RMSNorm weights of this tile's 16 rows
  // (before the wait: they never depend on the previous kernel) and, after the wait,
  // warp v's vector-v partial sums of squares (K / 16 floats)
  constexpr bool chain = kChain && NT == 1;
  __shared__ __align__(16) uint16_t w_s[chain ? 16 : 8];
  __shared__ __align__(16) float pss_s[chain ? 8 * 256 : 4];
  if (chain && epi.yw && warp == 0 && rank == 0 && lane < 2) cp_async16(w_s + lane * 8, epi.yw_w + tile * 16 + lane * 8);
  // a GEMV that adds a residual (a decoder block's o_proj and down_proj) bounds a
  // window (see ld_act_v4): its dependents launch only after its wait
  const bool bound = epi.residual != nullptr;
  if (!bound) pdl_launch_dependents();
  pdl_wait();
  if (bound) pdl_launch_dependents();
  // chain prologue: warp w requests the partial sums of squares of vectors w, w + warps,
  // ... now and sums them after its units (K / 16 partials: K / 2048 16-byte pieces per lane)
  __shared__ float inv_s[8];
  const bool ss_warp = chain && epi.ss_in != nullptr && rank == 0 && warp < n_vec;
  if (ss_warp) {
    for (int vv = warp; vv < n_vec; vv += kT4Warps) {
      const float *ps = epi.ss_in + static_cast<int64_t>(vv) * (K / 16) + lane * 4;
      float *pd = pss_s + vv * 256 + lane * 4;
      cp_async16(pd, ps);
      if (K == 4096) cp_async16(pd + 128, ps + 128);
    }
  }
  if constexpr (chain) cp_async_commit();
  __shared__ float res_s[16 * 8 * NT];
  const bool has_res = epi.residual != nullptr && rank == 0;
  S4Residual<NT, 32 * kT4Warps> rres;
  if (has_res) rres.load(res_s, tile, N, n_vec, epi.residual);
  if constexpr (norm) {
    // RMSNorm (rmsnorm_kernel's arithmetic): one pass over the whole x for the sums of
    // squares that also parks this CTA's k range in shared memory, then the range
    // normalised in place (x * inv * w, rounded to bf16)
    float ss[8];
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      ss[v] = 0.f;
      if (v < n_vec)
        for (int k = threadIdx.x * 8; k < K; k += kThr * 8) {
          const uint4 r = ld_act_v4(x + static_cast<int64_t>(v) * K + k);
          const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) ss[v] += bf16_lo(w4[i]) * bf16_lo(w4[i]) + bf16_hi(w4[i]) * bf16_hi(w4[i]);
          if (k >= kc0 && k < kc0 + klen) *reinterpret_cast<uint4 *>(xs_norm + v * klen + k - kc0) = r;
        }
      ss[v] = warp_sum(ss[v]);
    }
    if (lane == 0)
#pragma unroll
      for (int v = 0; v < 8; ++v) red[warp * 8 + v] = ss[v];
    __syncthreads();
    for (int v = 0; v < n_vec; ++v) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < kT4Warps; ++q) t += red[q * 8 + v];
      const float iv = rsqrtf(t / K + epi.eps);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = threadIdx.x * 8 + j * kThr * 8;
        if (k < klen) {
          uint4 *px = reinterpret_cast<uint4 *>(xs_norm + v * klen + k);
          const uint4 r = *px, w = wreg[j];
          uint4 o;
          o.x = pack_bf16x2(bf16_lo(r.x) * iv * bf16_lo(w.x), bf16_hi(r.x) * iv * bf16_hi(w.x));
          o.y = pack_bf16x2(bf16_lo(r.y) * iv * bf16_lo(w.y), bf16_hi(r.y) * iv * bf16_hi(w.y));
          o.z = pack_bf16x2(bf16_lo(r.z) * iv * bf16_lo(w.z), bf16_hi(r.z) * iv * bf16_hi(w.z));
          o.w = pack_bf16x2(bf16_lo(r.w) * iv * bf16_lo(w.w), bf16_hi(r.w) * iv * bf16_hi(w.w));
          *px = o;
        }
      }
    }
    __syncthreads();  // the normalised slice complete; `red` free again
  }
  for (int c0 = kr.b; c0 < kr.e; c0 += kT4Units) {
#pragma unroll
    for (int u = 0; u < kT4Units; ++u) {
      const int c = c0 + u;
      if (c < kr.e) {
        // B fragments straight from the activations (L1-cached) or the normalised
        // slice: this lane's 8 consecutive k of chunk j are k 0-7 of its code word
        if constexpr (norm) s4_unit_gx<NT, true>(acc, lo[u], hi[u], sc[u], xs_norm, K, n_vec, c * 128, klen, kc0);
        else if constexpr (kAsym) s4_unit_gx<NT, false, kRO, true>(acc, lo[u], hi[u], sc[u], x, K, n_vec, c * 128, -1, 0, mn[u]);
        else s4_unit_gx<NT, false, kRO>(acc, lo[u], hi[u], sc[u], x, K, n_vec, c * 128);
      }
    }
    if (c0 + kT4Units < kr.e) load(c0 + kT4Units);
  }
  if (has_res) rres.park(res_s, n_vec);
  if constexpr (chain) cp_async_wait_all();  // this thread's chain copies (if any) have landed
  if (ss_warp) {  // inv_s[v] = 1 / sqrt(mean(x_v^2) + eps), the partials summed in a fixed order
    for (int vv = warp; vv < n_vec; vv += kT4Warps) {
      const float4 a = *reinterpret_cast<const float4 *>(pss_s + vv * 256 + lane * 4);
      float t = (a.x + a.y) + (a.z + a.w);
      if (K == 4096) {
        const float4 c = *reinterpret_cast<const float4 *>(pss_s + vv * 256 + 128 + lane * 4);
        t += (c.x + c.y) + (c.z + c.w);
      }
      t = warp_sum(t);
      if (lane == 0) inv_s[vv] = rsqrtf(t / K + epi.eps);
    }
  }
  // reduce over warps (and cluster ranks) in fixed order
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[((warp * NT + t) * 4 + e) * 32 + lane] = acc[0][t][e] + acc[1][t][e];
  __syncthreads();
  float v[NT][4];
  if (warp == 0) {
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < kT4Warps; ++q) sum += red[((q * NT + t) * 4 + e) * 32 + lane];
        v[t][e] = sum;
      }
  }
  if constexpr (CS > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    float *slot0 = red + kT4Warps * NT * 128;
    if (warp == 0 && rank > 0) {
      float *remote = cluster.map_shared_rank(slot0, 0);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) remote[((rank * NT + t) * 4 + e) * 32 + lane] = v[t][e];
    }
    cluster.sync();
    if (rank != 0) return;
    if (warp == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
          for (int r = 1; r < CS; ++r) v[t][e] += slot0[((r * NT + t) * 4 + e) * 32 + lane];
    }
  }
  if constexpr (kAR && NT == 1) {
    if (warp == 0) s4_allreduce_tile(v[0], tile, N, n_vec, epi.ar);
  }
  if constexpr (chain) {
    if (epi.ss_in && warp == 0) {  // the folded RMSNorm: y = inv * (W . (x * w))
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int vv = tid * 2 + (e & 1);
        if (vv < n_vec) v[0][e] *= inv_s[vv];
      }
    }
  }
  if (warp == 0) {
    float w_lo = 0.f, w_hi = 0.f;  // (w_s landed before the block barrier above)
    if (chain && epi.yw) {
      w_lo = bf16_bits_to_float(w_s[gid]);
      w_hi = bf16_bits_to_float(w_s[gid + 8]);
    }
    s4_store<NT>(v, tile, N, n_vec, y, epi.residual ? res_s : nullptr, epi.swiglu, epi.amax, chain ? epi.yw : nullptr,
                 epi.ss_out, w_lo, w_hi);
  }
}

// Repack natural-layout codes [N, K/2] + scales [N, K/32] into GEMV units.
// One thread per 16-byte piece of a unit (72 pieces per unit).
// (kAsym: q4 units, the group mins in pieces 72..79 laid out as the scales)
template <bool kAsym = false>
__global__ void pack_s4g32_kernel(const uint8_t *__restrict__ codes,
                                  const uint16_t *__restrict__ scales, uint8_t *__restrict__ out,
                                  int N, int K, int64_t pieces, const uint16_t *__restrict__ mins = nullptr) {
  constexpr int kPieces = kAsym ? 80 : 72;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= pieces) return;
  const int cpt = K / 128;
  const int64_t unit = p / kPieces;
  const int piece = static_cast<int>(p % kPieces);
  const int64_t tile = unit / cpt;
  const int c = static_cast<int>(unit % cpt);
  uint32_t words[4];
  if (piece < 64) {
    const int h = piece >> 5, lane = piece & 31;
    const int gid = lane >> 2, tid = lane & 3;
    const int64_t row = tile * 16 + gid + 8 * h;
    const uint8_t *src = codes + row * (K / 2);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint8_t *g = src + (c * 4 + j) * 16 + tid * 4;
      words[j] = s4_word_pack(static_cast<uint32_t>(g[0]) | (static_cast<uint32_t>(g[1]) << 8) |
                              (static_cast<uint32_t>(g[2]) << 16) | (static_cast<uint32_t>(g[3]) << 24));
    }
  } else {
    const int gid = (piece - 64) & 7;
    const int64_t rlo = tile * 16 + gid, rhi = rlo + 8;
    const uint16_t *src = (kAsym && piece >= 72) ? mins : scales;
    const uint16_t *slo = src + rlo * (K / 32) + c * 4;
    const uint16_t *shi = src + rhi * (K / 32) + c * 4;
    words[0] = slo[0] | (static_cast<uint32_t>(slo[1]) << 16);
    words[1] = slo[2] | (static_cast<uint32_t>(slo[3]) << 16);
    words[2] = shi[0] | (static_cast<uint32_t>(shi[1]) << 16);
    words[3] = shi[2] | (static_cast<uint32_t>(shi[3]) << 16);
  }
  reinterpret_cast<uint4 *>(out)[p] = make_uint4(words[0], words[1], words[2], words[3]);
}

template <int NT, int CS, int kW = 0>
static int launch_s4_tile(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K,
                          int n_vec, const S4Epi &epi, bool pdl, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((N / 16) * CS));
  cfg.blockDim = dim3(32 * s4_cta_warps<NT, kW>());
  cfg.stream = s;
  if (epi.norm_w) {
    // the CTA's normalised k range of every vector (<= 8 x 2048 bf16 = 32 KB)
    const int klen_max = (((K / 128) + CS - 1) / CS) * 128;
    cfg.dynamicSmemBytes = static_cast<size_t>(n_vec) * klen_max * 2;
  }
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
  cudaError_t e;
  if (epi.asym) {
    if constexpr (NT != 1) return IRON_ERR_SHAPE;
    e = epi.x_ro ? cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<1, CS, false, false, true, false, true>, packed, x, y, N, K, n_vec, epi)
                 : cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<1, CS, false, false, false, false, true>, packed, x, y, N, K, n_vec, epi);
  } else if (epi.ar.world > 1) {
    if constexpr (NT != 1) return IRON_ERR_SHAPE;
    e = epi.x_ro ? cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<1, CS, false, true, true>, packed, x, y, N, K, n_vec, epi)
                 : cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<1, CS, false, true, false>, packed, x, y, N, K, n_vec, epi);
  } else if (epi.ss_in || epi.yw) {
    if constexpr (NT != 1) return IRON_ERR_SHAPE;
    e = epi.x_ro ? cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<1, CS, false, false, true, true, false, kW>, packed, x, y, N, K, n_vec, epi)
                 : cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<1, CS, false, false, false, true, false, kW>, packed, x, y, N, K, n_vec, epi);
  } else if (epi.norm_w) {
    e = cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<NT, CS, true>, packed, x, y, N, K, n_vec, epi);
  } else {
    e = epi.x_ro ? cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<NT, CS, false, false, true, false, false, kW>, packed, x, y, N, K, n_vec, epi)
                 : cudaLaunchKernelEx(&cfg, gemv_s4g32_tile_kernel<NT, CS, false, false, false, false, false, kW>, packed, x, y, N, K, n_vec, epi);
  }
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}

template <int NT>
static int launch_s4_tile_cs(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K,
                             int n_vec, const S4Epi &res, bool pdl, cudaStream_t s) {
  // split K over a cluster until every SM holds >= 2 CTAs (and each warp >= 1 chunk)
  // (64-vector tiles stop at clusters of 4: their reduction slots and residual fill
  // the static shared memory)
  constexpr int kMaxCS = NT >= 8 ? 4 : 8;
  const int tiles = N / 16, cpt = K / 128;
  int cs = 1;
  while (cs < kMaxCS && tiles * cs < 2 * sm_count() && cpt >= s4_warps<NT>() * cs * 2) cs *= 2;
  // more tiles than one wave of four 8-warp CTAs per SM: the half-width CTAs (plain and
  // chain single-tile forms)
  if constexpr (NT == 1) {
    if (cs == 1 && tiles > 4 * sm_count() && !res.norm_w && !res.asym && res.ar.world <= 1)
      return launch_s4_tile<1, 1, 4>(packed, x, y, N, K, n_vec, res, pdl, s);
    // a 2-CTA cluster splitting K: one 16-warp CTA per tile instead (each warp keeps >= 1
    // unit). Clusters of 4 (the down projection) stay: halving them to 2 x 16 warps measured
    // 404.5 against 402.8 us per B200 decode step.
    if (cs == 2 && cpt >= 16 && !res.norm_w && !res.asym && res.ar.world <= 1)
      return launch_s4_tile<1, 1, 16>(packed, x, y, N, K, n_vec, res, pdl, s);
  }
  switch (cs) {
    case 1: return launch_s4_tile<NT, 1>(packed, x, y, N, K, n_vec, res, pdl, s);
    case 2: return launch_s4_tile<NT, 2>(packed, x, y, N, K, n_vec, res, pdl, s);
    case 4: return launch_s4_tile<NT, 4>(packed, x, y, N, K, n_vec, res, pdl, s);
    default:
      if constexpr (kMaxCS == 8) return launch_s4_tile<NT, 8>(packed, x, y, N, K, n_vec, res, pdl, s);
      else return launch_s4_tile<NT, 4>(packed, x, y, N, K, n_vec, res, pdl, s);
  }
}

// Inverse of pack_s4g32_kernel: one thread per 16-byte code piece writes its
// row's 4 x 8 dequantized weights, bf16(q * s) exactly (the products of a 4-bit
// integer and a bf16 scale are exact in fp32, so one rounding gives the
// Dequant golden's value).
template <bool kAsym = false>
__global__ void unpack_s4g32_kernel(const uint8_t *__restrict__ packed, uint16_t *__restrict__ out, int K,
                                    int64_t pieces) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= pieces) return;
  const int cpt = K / 128;
  const int64_t unit = p / 64;
  const int piece = static_cast<int>(p % 64);
  const int64_t tile = unit / cpt;
  const int c = static_cast<int>(unit % cpt);
  const int h = piece >> 5, lane = piece & 31, gid = lane >> 2, tid = lane & 3;
  const uint4 *u = reinterpret_cast<const uint4 *>(packed) + unit * (kAsym ? 80 : 72);
  const uint4 cw = u[piece];
  const uint4 sw = u[64 + gid];
  const uint4 mw = kAsym ? u[72 + gid] : make_uint4(0u, 0u, 0u, 0u);
  const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
  const uint32_t sc[2] = {h ? sw.z : sw.x, h ? sw.w : sw.y};  // groups (0,1), (2,3) of the row
  const uint32_t mc[2] = {h ? mw.z : mw.x, h ? mw.w : mw.y};
  const int64_t row = tile * 16 + gid + 8 * h;
  uint16_t *dst = out + row * K + c * 128 + tid * 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float scale = (j & 1) ? bf16_hi(sc[j >> 1]) : bf16_lo(sc[j >> 1]);
    const float mn = (j & 1) ? bf16_hi(mc[j >> 1]) : bf16_lo(mc[j >> 1]);
    uint32_t o[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      if constexpr (kAsym) {  // min + scale * code (exact in fp32), rounded once
        const float lo = fmaf(static_cast<float>(s4_word_nibble(words[j], 2 * b)), scale, mn);
        const float hi = fmaf(static_cast<float>(s4_word_nibble(words[j], 2 * b + 1)), scale, mn);
        o[b] = pack_bf16x2(lo, hi);
      } else {
        const float lo = static_cast<float>(static_cast<int>(s4_word_nibble(words[j], 2 * b) ^ 8u) - 8) * scale;
        const float hi = static_cast<float>(static_cast<int>(s4_word_nibble(words[j], 2 * b + 1) ^ 8u) - 8) * scale;
        o[b] = pack_bf16x2(lo, hi);
      }
    }
    *reinterpret_cast<uint4 *>(dst + j * 32) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace iron

using namespace iron;

extern "C" int iron_pack_int4g32(const uint8_t *codes, const uint16_t *scales, uint8_t *packed,
                                 int N, int K, void *stream) {
  if (!codes || !scales || !packed) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || N % 16 || K % 128) return IRON_ERR_SHAPE;
  if (!aligned16(packed)) return IRON_ERR_ALIGN;
  const int64_t pieces = static_cast<int64_t>(N / 16) * (K / 128) * 72;
  const int threads = 256;
  pack_s4g32_kernel<false><<<static_cast<unsigned>((pieces + threads - 1) / threads), threads, 0,
                      static_cast<cudaStream_t>(stream)>>>(codes, scales, packed, N, K, pieces);
  return launch_status();
}

extern "C" int iron_unpack_int4g32(const uint8_t *packed, uint16_t *out, int N, int K, void *stream) {
  if (!packed || !out) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || N % 16 || K % 128) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(out)) return IRON_ERR_ALIGN;
  const int64_t pieces = static_cast<int64_t>(N / 16) * (K / 128) * 64;
  const int threads = 256;
  unpack_s4g32_kernel<false><<<static_cast<unsigned>((pieces + threads - 1) / threads), threads, 0,
                        static_cast<cudaStream_t>(stream)>>>(packed, out, K, pieces);
  return launch_status();
}

// q4 weights (asymmetric int4: min + scale * code per 32-k group, IRON's q4nx values).
extern "C" int iron_pack_q4g32(const uint8_t *codes, const uint16_t *scales, const uint16_t *mins, uint8_t *packed,
                               int N, int K, void *stream) {
  if (!codes || !scales || !mins || !packed) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || N % 16 || K % 128) return IRON_ERR_SHAPE;
  if (!aligned16(packed)) return IRON_ERR_ALIGN;
  const int64_t pieces = static_cast<int64_t>(N / 16) * (K / 128) * 80;
  const int threads = 256;
  pack_s4g32_kernel<true><<<static_cast<unsigned>((pieces + threads - 1) / threads), threads, 0,
                            static_cast<cudaStream_t>(stream)>>>(codes, scales, packed, N, K, pieces, mins);
  return launch_status();
}

extern "C" int iron_unpack_q4g32(const uint8_t *packed, uint16_t *out, int N, int K, void *stream) {
  if (!packed || !out) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || N % 16 || K % 128) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(out)) return IRON_ERR_ALIGN;
  const int64_t pieces = static_cast<int64_t>(N / 16) * (K / 128) * 64;
  const int threads = 256;
  unpack_s4g32_kernel<true><<<static_cast<unsigned>((pieces + threads - 1) / threads), threads, 0,
                              static_cast<cudaStream_t>(stream)>>>(packed, out, K, pieces);
  return launch_status();
}

extern "C" int iron_gemv_q4g32(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                               const uint16_t *residual, unsigned flags, void *stream) {
  if (!packed || !x || !y) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || n_vec <= 0 || n_vec > 8 || K % 128 || N % 16) return IRON_ERR_SHAPE;
  if (static_cast<int64_t>(N / 16) * (K / 128) > 0x7fffffffLL) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(x)) return IRON_ERR_ALIGN;
  if (flags & IRON_FLAG_SWIGLU) return IRON_ERR_ARG;
  S4Epi epi{residual, 0, nullptr, 0.f, nullptr, {}, (flags & IRON_FLAG_X_READONLY) ? 1 : 0};
  epi.ar.world = 1;
  epi.asym = 1;
  return launch_s4_tile_cs<1>(packed, x, y, N, K, n_vec, epi, (flags & IRON_FLAG_PDL) != 0,
                              static_cast<cudaStream_t>(stream));
}

extern "C" int iron_gemv_int4g32_ex(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K,
                                    int n_vec, const uint16_t *residual, const uint16_t *norm_weight,
                                    float eps, unsigned long long *argmax_keys, unsigned flags,
                                    void *stream) {
  if (!packed || !x || !y) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || n_vec <= 0 || n_vec > 64) return IRON_ERR_SHAPE;
  if (K % 128 || N % 16) return IRON_ERR_SHAPE;
  if (static_cast<int64_t>(N / 16) * (K / 128) > 0x7fffffffLL) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(x)) return IRON_ERR_ALIGN;
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  const int swiglu = (flags & IRON_FLAG_SWIGLU) ? 1 : 0;
  if (swiglu && (residual || argmax_keys)) return IRON_ERR_ARG;
  if (norm_weight) {
    if (n_vec > 8 || K > 2048) return IRON_ERR_SHAPE;  // the fused prologue's shared slice and registers
    if (!aligned16(norm_weight)) return IRON_ERR_ALIGN;
  }
  S4Epi epi{residual, swiglu, norm_weight, eps, argmax_keys, {}, (flags & IRON_FLAG_X_READONLY) ? 1 : 0};
  epi.ar.world = 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_vec <= 8) return launch_s4_tile_cs<1>(packed, x, y, N, K, n_vec, epi, pdl, s);
  if (!norm_weight) {  // 33..64 vectors: the tensor-core form where it takes the shape
    const int st = launch_s4_tc(packed, x, y, N, K, n_vec, residual, swiglu, argmax_keys, pdl, s);
    if (st != IRON_ERR_UNSUPPORTED) return st;
  }
#ifdef IRON_S4_ONLY_NT1
  return IRON_ERR_SHAPE;
#else
  if (n_vec <= 16) return launch_s4_tile_cs<2>(packed, x, y, N, K, n_vec, epi, pdl, s);
  if (n_vec <= 32) return launch_s4_tile_cs<4>(packed, x, y, N, K, n_vec, epi, pdl, s);
  return launch_s4_tile_cs<8>(packed, x, y, N, K, n_vec, epi, pdl, s);
#endif
}

extern "C" int iron_gemv_int4g32_chain(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                                       const iron_gemv_chain *c, unsigned flags, void *stream) {
  if (!packed || !x || !y || !c) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || n_vec <= 0 || n_vec > 8 || K % 128 || N % 16) return IRON_ERR_SHAPE;
  if (static_cast<int64_t>(N / 16) * (K / 128) > 0x7fffffffLL) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(x)) return IRON_ERR_ALIGN;
  const int swiglu = (flags & IRON_FLAG_SWIGLU) ? 1 : 0;
  const bool writer = c->ss_out || c->y_weighted || c->weight;
  if (writer && !(c->ss_out && c->y_weighted && c->weight)) return IRON_ERR_NULL;
  if (swiglu && (c->residual || c->argmax_keys || writer)) return IRON_ERR_ARG;
  if (c->ss_in) {
    if (K != 2048 && K != 4096) return IRON_ERR_SHAPE;  // K / 16 partials: one or two float4 per lane
    if (!aligned16(c->ss_in)) return IRON_ERR_ALIGN;
    if (!(c->eps >= 0.f)) return IRON_ERR_ARG;
  }
  S4Epi epi{c->residual, swiglu, nullptr, c->eps, c->argmax_keys, {}, (flags & IRON_FLAG_X_READONLY) ? 1 : 0};
  epi.ar.world = 1;
  epi.ss_in = c->ss_in;
  epi.ss_out = c->ss_out;
  epi.yw = c->y_weighted;
  epi.yw_w = c->weight;
  return launch_s4_tile_cs<1>(packed, x, y, N, K, n_vec, epi, (flags & IRON_FLAG_PDL) != 0,
                              static_cast<cudaStream_t>(stream));
}

extern "C" int iron_gemv_int4g32_allreduce(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K,
                                           int n_vec, const uint16_t *residual, const void *peers,
                                           unsigned flags, void *stream) {
  if (!packed || !x || !y || !peers) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || n_vec <= 0 || n_vec > 8 || K % 128 || N % 16) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(x)) return IRON_ERR_ALIGN;
  if (flags & IRON_FLAG_SWIGLU) return IRON_ERR_ARG;
  S4Epi epi{residual, 0, nullptr, 0.f, nullptr, {}, (flags & IRON_FLAG_X_READONLY) ? 1 : 0};
  std::memcpy(&epi.ar, peers, sizeof(S4AllReduce));
  if (epi.ar.world < 1 || epi.ar.world > kS4MaxWorld || epi.ar.rank < 0 || epi.ar.rank >= epi.ar.world ||
      !epi.ar.status)
    return IRON_ERR_ARG;
  for (int r = 0; r < epi.ar.world; ++r)
    if (!epi.ar.recv[r]) return IRON_ERR_NULL;
  return launch_s4_tile_cs<1>(packed, x, y, N, K, n_vec, epi, (flags & IRON_FLAG_PDL) != 0,
                              static_cast<cudaStream_t>(stream));
}

// CUDA IPC plumbing for the peer buffers of the fused all-reduce. A handle maps the
// START of a cudaMalloc allocation, so the buffers come from iron_ipc_alloc (their own
// zero-filled allocation), not from a caching allocator's pool.
extern "C" int iron_ipc_alloc(size_t bytes, void **dev_ptr_out) {
  if (!dev_ptr_out) return IRON_ERR_NULL;
  if (bytes == 0) return IRON_ERR_SHAPE;
  if (cudaMalloc(dev_ptr_out, bytes) != cudaSuccess) return launch_status();
  if (cudaMemset(*dev_ptr_out, 0, bytes) != cudaSuccess) return launch_status();
  return IRON_OK;
}

extern "C" int iron_ipc_free(void *dev_ptr) {
  if (!dev_ptr) return IRON_ERR_NULL;
  if (cudaFree(dev_ptr) != cudaSuccess) return launch_status();
  return IRON_OK;
}

extern "C" int iron_ipc_handle(const void *dev_ptr, void *handle_out) {
  if (!dev_ptr || !handle_out) return IRON_ERR_NULL;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)) != cudaSuccess) return launch_status();
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  return IRON_OK;
}

extern "C" int iron_ipc_open(const void *handle, void **dev_ptr_out) {
  if (!handle || !dev_ptr_out) return IRON_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return launch_status();
  return IRON_OK;
}

extern "C" int iron_ipc_close(void *dev_ptr) {
  if (!dev_ptr) return IRON_ERR_NULL;
  if (cudaIpcCloseMemHandle(dev_ptr) != cudaSuccess) return launch_status();
  return IRON_OK;
}

extern "C" int iron_gemv_int4g32(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N,
                                 int K, int n_vec, const uint16_t *residual, unsigned flags,
                                 void *stream) {
  return iron_gemv_int4g32_ex(packed, x, y, N, K, n_vec, residual, nullptr, 0.f, nullptr, flags, stream);
}

// Greedy next token from the argmax keys an lm-head GEMV left: tokens[b], pos[b] += 1
// (if pos), and the keys reset for the next step.
__global__ void argmax_finalize_kernel(unsigned long long *keys, int *tokens, int *pos, int B) {
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int b = blockIdx.x, lane = threadIdx.x;  // one warp per vector, a lane per slot
  unsigned long long k = ld_act(keys + b * kS4ArgmaxSlots + lane);  // the lm-head GEMV's atomics
  keys[b * kS4ArgmaxSlots + lane] = 0ull;
#pragma unroll
  for (int x = 16; x > 0; x >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, x);
    k = o > k ? o : k;
  }
  if (lane == 0) {
    tokens[b] = static_cast<int>(~static_cast<unsigned>(k & 0xffffffffull));
    if (pos) pos[b] += 1;
  }
}

// Bring [ptr, ptr + bytes) into L2 ahead of its readers: each CTA's thread 0 issues
// cp.async.bulk.prefetch.L2 for one 64 KB piece (fire and forget: the kernel ends
// when the requests are issued). Meant for a side branch of a decode graph, so the
// weights of a later GEMV stream in while the main chain is latency-bound.
constexpr uint32_t kL2PrefetchPiece = 64 * 1024;
__global__ void l2_prefetch_kernel(const uint8_t *__restrict__ p, size_t bytes) {
  const size_t off = static_cast<size_t>(blockIdx.x) * kL2PrefetchPiece;
  if (threadIdx.x != 0 || off >= bytes) return;
  const size_t left = bytes - off;
  const uint32_t n = static_cast<uint32_t>(left < kL2PrefetchPiece ? left : kL2PrefetchPiece) & ~15u;
  if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(n) : "memory");
}

extern "C" int iron_l2_prefetch(const void *ptr, size_t bytes, unsigned flags, void *stream) {
  if (!ptr) return IRON_ERR_NULL;
  if (bytes == 0) return IRON_OK;
  if (!aligned16(ptr)) return IRON_ERR_ALIGN;
  const size_t pieces = (bytes + kL2PrefetchPiece - 1) / kL2PrefetchPiece;
  if (pieces > 0x7fffffffu) return IRON_ERR_SHAPE;
  return launch(l2_prefetch_kernel, dim3(static_cast<unsigned>(pieces)), dim3(32), 0,
                static_cast<cudaStream_t>(stream), (flags & IRON_FLAG_PDL) != 0,
                static_cast<const uint8_t *>(ptr), bytes);
}

extern "C" int iron_argmax_finalize(unsigned long long *keys, int32_t *tokens, int32_t *pos, int B, unsigned flags,
                                    void *stream) {
  if (!keys || !tokens) return IRON_ERR_NULL;
  if (B <= 0 || B > 65535) return IRON_ERR_SHAPE;
  return launch(argmax_finalize_kernel, dim3(B), dim3(kS4ArgmaxSlots), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, keys, tokens, pos, B);
}
