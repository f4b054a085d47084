// Persistent Llama-3.2-1B decode step: the whole step in ONE kernel.
//
// The graph path (decode.cu + gemv_s4.cu + attention.cu, 148 launches per step)
// pays, per launch, the grid-dependency latency and the spread of 500+ CTAs
// starting; at batch 1 that, not HBM, sets the step time. Here one CTA per SM
// (a cooperative launch, so every CTA is resident) runs the step's phases in
// order and a bounded grid barrier separates them:
//
//   per layer:  QKV    RMSNorm(x) into shared memory (every CTA, redundantly),
//                      int4 GEMV work items, last-arriver tile finalisation
//               ATTN   RoPE of q and the new k, KV-cache append, 64-token chunks
//                      of GQA attention per warp, last-arriver merge per head
//               O      GEMV on the attention output, + residual -> h
//               GU     RMSNorm(h) into shared memory, gate/up GEMV, SwiGLU -> act
//               D      GEMV on act, + residual -> x
//   then:       LM     RMSNorm(x), lm-head GEMV, argmax by 64-bit atomicMax
//               NEXT   token and position update (one CTA)
//
// A GEMV phase splits each 16-row tile's K into P parts (work items of whole
// 128-k units); a warp takes items round-robin, writes its fp32 partial, and the
// warp that arrives last at a tile's counter sums the P partials in part order
// (bitwise deterministic) and applies the epilogue. Every warp issues the weight
// loads of its first item BEFORE the barrier that precedes the phase -- weights
// never depend on the previous phase -- so HBM streams while the grid syncs.
// The arithmetic of every step is that of the graph path's kernels (exact int4
// dequantization, bf16 rounding points of IRON's pipeline).
//
// Every wait (grid barrier) gives up after 1 s without progress, sets the status
// word and makes every CTA leave; activations written by other CTAs are read
// through L2 (ld.global.cg), never through the non-coherent L1 path.
#include <cooperative_groups.h>

#include "common.cuh"
#include "s4.cuh"

namespace iron {
namespace mk {

constexpr int kWarps = 8;  // 8 warps x 255 registers: the attention and GEMV code need no spills
constexpr int kThreads = 32 * kWarps;
constexpr int kE = 2048, kHq = 32, kHkv = 8, kD = 64, kG = 4, kQKV = 3072, kHid = 8192;
constexpr int kMaxB = 8;
constexpr int kChunk = 64;          // tokens per attention work item
constexpr int kUnitBytes = 1152;
constexpr int kVStride = 72;        // padded V tile row (elements)
constexpr uint64_t kTimeoutNs = 1000000000ull;

struct Layer {
  const uint8_t *qkv, *o, *gu, *d;  // packed int4 g32 (iron_pack_int4g32 layout)
  const uint16_t *n1, *n2;          // RMSNorm weights
  uint16_t *kc, *vc;                // this layer's caches [B, Hkv, L, 64]
};

struct Args {
  const Layer *layers;
  int n_layers;
  const uint16_t *embed;  // [V, E] bf16
  const uint16_t *nf;
  const uint8_t *lm;      // packed [V, E]
  int V;
  const float *lut;       // [L, 64] fp32 cos/sin interleaved
  int *tokens, *pos;      // [B]
  uint16_t *x, *h, *qkv, *attn, *act, *logits;  // logits may be null
  float *part;            // GEMV partials
  unsigned *cnt;          // per-tile arrival counters (zero at launch, left zero)
  float *apart;           // attention partials [B, Hkv, chunks, 4, 66]
  unsigned *hcnt;         // per-(sequence, kv head) arrival counters
  unsigned long long *amax;  // [B] argmax keys (zero at launch, left zero)
  unsigned *bar;          // grid barrier {arrivals, generation}
  unsigned *status;       // 0 ok; bit 0: a barrier timed out; bit 1: a position / token out of range
  int B, L, max_chunks;
  int64_t kv_b, kv_h;     // cache strides (elements)
  float eps, scale_log2;
};

// ---- memory helpers ----------------------------------------------------------------
__device__ __forceinline__ uint4 ld_cg4(const void *p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float ld_cg_f(const float *p) {
  float r;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint16_t ld_cg_u16(const uint16_t *p) {
  uint16_t r;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned r;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid barrier over gridDim.x resident CTAs (sense by generation counter).
// Returns false (and sets the status word) when a wait ran out.
__device__ bool grid_sync(const Args &a) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned g = ld_acquire(a.bar + 1);
    __threadfence();
    const unsigned arrived = atomicAdd(a.bar, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(a.bar, 0u);
      __threadfence();
      atomicAdd(a.bar + 1, 1u);
    } else {
      uint64_t start = 0;
      for (uint32_t i = 0;; ++i) {
        if (ld_acquire(a.bar + 1) != g) break;
        if ((i & 127u) == 0u) {
          if (ld_acquire(a.status) != 0u) {  // another CTA gave up: do not wait for it
            ok = 0;
            break;
          }
          const uint64_t t = now_ns();
          if (start == 0) start = t;
          else if (t - start > kTimeoutNs) {
            atomicOr(a.status, 1u);
            ok = 0;
            break;
          }
        }
      }
    }
    __threadfence();
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// ---- RMSNorm of B rows of E into shared memory (same arithmetic as rmsnorm_kernel) ----
// src rows: `x` (stride E) or, if emb_tokens, embedding rows table[tokens[b]].
__device__ void rmsnorm_to_smem(const uint16_t *x, const int *emb_tokens, const uint16_t *w, uint16_t *xs,
                                int B, float eps, float *red) {
  for (int b = 0; b < B; ++b) {
    const uint16_t *xr = emb_tokens ? x + static_cast<int64_t>(emb_tokens[b]) * kE : x + b * kE;
    // E elements over the CTA's threads: kPer contiguous elements per thread, 4 per 8-byte load
    constexpr int kPer = kE / kThreads;
    const int c0 = threadIdx.x * kPer;
    float v[kPer];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; i += 4) {
      uint2 raw;
      if (emb_tokens) raw = __ldg(reinterpret_cast<const uint2 *>(xr + c0 + i));
      else asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(raw.x), "=r"(raw.y) : "l"(xr + c0 + i));
      v[i] = bf16_lo(raw.x);
      v[i + 1] = bf16_hi(raw.x);
      v[i + 2] = bf16_lo(raw.y);
      v[i + 3] = bf16_hi(raw.y);
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += v[i + j] * v[i + j];
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += red[i];
    const float inv = rsqrtf(tot / kE + eps);
#pragma unroll
    for (int i = 0; i < kPer; i += 4) {
      const uint2 wr = __ldg(reinterpret_cast<const uint2 *>(w + c0 + i));
      uint2 o;
      o.x = pack_bf16x2(v[i] * inv * bf16_lo(wr.x), v[i + 1] * inv * bf16_hi(wr.x));
      o.y = pack_bf16x2(v[i + 2] * inv * bf16_lo(wr.y), v[i + 3] * inv * bf16_hi(wr.y));
      *reinterpret_cast<uint2 *>(xs + b * kE + c0 + i) = o;
    }
    __syncthreads();  // `red` reused by the next row
  }
}

// ---- int4 GEMV work items ------------------------------------------------------------
struct Gemv {
  const uint8_t *w;  // packed matrix
  int N, K;          // rows, inputs
  int P;             // parts per tile
  int cpt, upp;      // units per tile, units per part
  int items;         // tiles * P
};
__device__ __forceinline__ Gemv make_gemv(const uint8_t *w, int N, int K, int P) {
  Gemv g;
  g.w = w;
  g.N = N;
  g.K = K;
  g.P = P;
  g.cpt = K / 128;
  g.upp = g.cpt / P;
  g.items = (N / 16) * P;
  return g;
}

constexpr int kPre = 2;  // units per load group (the first group is loaded before the barrier)

struct UnitRegs {
  uint4 lo, hi, sc;
};
__device__ __forceinline__ void load_unit(UnitRegs &r, const uint8_t *p, int lane) {
  r.lo = ld_stream_v4(p + lane * 16);
  r.hi = ld_stream_v4(p + 512 + lane * 16);
  r.sc = ld_stream_v4(p + 1024 + (lane >> 2) * 16);
}

// One unit (16 rows x 128 k) against the B vectors: B fragments from `xsrc`
// ([B, K] bf16, shared memory or global through L2).
template <bool kSmem>
__device__ __forceinline__ void unit_mma(float (&d)[2][4], const UnitRegs &u, const uint16_t *xsrc, int K, int B,
                                         int kbase, int lane) {
  const int gid = lane >> 2, tid = lane & 3;
  const uint32_t wl[4] = {u.lo.x, u.lo.y, u.lo.z, u.lo.w};
  const uint32_t wh[4] = {u.hi.x, u.hi.y, u.hi.z, u.hi.w};
  const uint32_t sl2[2] = {u.sc.x, u.sc.y}, sh2[2] = {u.sc.z, u.sc.w};
  uint4 xr[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    xr[j] = make_uint4(0u, 0u, 0u, 0u);
    if (gid < B) {
      const uint16_t *p = xsrc + static_cast<int64_t>(gid) * K + kbase + j * 32 + tid * 8;
      xr[j] = kSmem ? *reinterpret_cast<const uint4 *>(p) : ld_cg4(p);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sel = (j & 1) ? 0x3232u : 0x1010u;
    const uint32_t s2_lo = prmt_(sl2[j >> 1], sl2[j >> 1], sel);
    const uint32_t s2_hi = prmt_(sh2[j >> 1], sh2[j >> 1], sel);
    uint32_t pl[4], ph[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      pl[q] = s4x2_dequant_(wl[j] >> (4 * q), s2_lo);
      ph[q] = s4x2_dequant_(wh[j] >> (4 * q), s2_hi);
    }
    const uint32_t A0[4] = {pl[0], ph[0], pl[1], ph[1]};
    const uint32_t A1[4] = {pl[2], ph[2], pl[3], ph[3]};
    const uint4 e = xr[j];
    mma_bf16_16816(d[j & 1], A0, e.x, e.y);  // packed nibble order: consecutive k pairs
    mma_bf16_16816(d[j & 1], A1, e.z, e.w);
  }
}

// Prefetch the first units of this warp's first item (before the barrier).
__device__ __forceinline__ int gemv_prefetch(const Gemv &g, UnitRegs (&pre)[kPre], int wg, int lane) {
  if (wg >= g.items) return 0;
  const int tile = wg / g.P, part = wg % g.P;
  const int u0 = part * g.upp;
  const int n = g.upp < kPre ? g.upp : kPre;
#pragma unroll
  for (int i = 0; i < kPre; ++i)
    if (i < n) load_unit(pre[i], g.w + (static_cast<int64_t>(tile) * g.cpt + u0 + i) * kUnitBytes, lane);
  return n;
}

// Run this warp's items; `fin(tile, v)` finalises a tile (v = the summed C fragment).
// Units stream in groups of kPre, double-buffered: the next group's loads (possibly
// of the next item) are in flight while the current group computes.
template <bool kSmem, class Fin>
__device__ void gemv_run(const Gemv &g, const UnitRegs (&pre)[kPre], int npre, const uint16_t *xsrc, int B,
                         float *part, unsigned *cnt, int wg, int W, int lane, Fin &&fin) {
  if (wg >= g.items) return;
  const int groups = (g.upp + kPre - 1) / kPre;
  UnitRegs cur[kPre], nxt[kPre];
#pragma unroll
  for (int i = 0; i < kPre; ++i) cur[i] = pre[i];
  (void)npre;  // the first group of the first item was loaded by gemv_prefetch
  int item = wg, gi = 0;
  float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  while (true) {
    const int tile = item / g.P, p = item % g.P;
    const int u0 = p * g.upp + gi * kPre;
    const int n = (g.upp - gi * kPre) < kPre ? (g.upp - gi * kPre) : kPre;
    // next group: the rest of this item, else the first group of the next item
    int nitem = item, ngi = gi + 1;
    if (ngi >= groups) {
      nitem = item + W;
      ngi = 0;
    }
    if (nitem < g.items) {
      const int nt = nitem / g.P, np = nitem % g.P;
      const int nu0 = np * g.upp + ngi * kPre;
      const int nn = (g.upp - ngi * kPre) < kPre ? (g.upp - ngi * kPre) : kPre;
      const uint8_t *nb = g.w + (static_cast<int64_t>(nt) * g.cpt + nu0) * kUnitBytes;
#pragma unroll
      for (int i = 0; i < kPre; ++i)
        if (i < nn) load_unit(nxt[i], nb + static_cast<int64_t>(i) * kUnitBytes, lane);
    }
#pragma unroll
    for (int i = 0; i < kPre; ++i)
      if (i < n) unit_mma<kSmem>(d, cur[i], xsrc, g.K, B, (u0 + i) * 128, lane);
    if (gi == groups - 1) {
      float v[4] = {d[0][0] + d[1][0], d[0][1] + d[1][1], d[0][2] + d[1][2], d[0][3] + d[1][3]};
#pragma unroll
      for (int e = 0; e < 4; ++e) d[0][e] = d[1][e] = 0.f;
      if (g.P == 1) {
        fin(tile, v);
      } else {
        float *slot = part + (static_cast<int64_t>(tile) * g.P + p) * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e) slot[e * 32 + lane] = v[e];
        __threadfence();
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(cnt + tile, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == static_cast<unsigned>(g.P - 1)) {
          __threadfence();
          float sm[4] = {0.f, 0.f, 0.f, 0.f};
          const float *t0 = part + static_cast<int64_t>(tile) * g.P * 128;
          for (int q = 0; q < g.P; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) sm[e] += ld_cg_f(t0 + q * 128 + e * 32 + lane);
          if (lane == 0) cnt[tile] = 0u;  // reused by a later phase, after a grid barrier
          fin(tile, sm);
        }
      }
    }
    if (nitem >= g.items) break;
    item = nitem;
    gi = ngi;
#pragma unroll
    for (int i = 0; i < kPre; ++i) cur[i] = nxt[i];
  }
}

// ---- L2 prefetch of a later phase's inputs ------------------------------------------------
__device__ __forceinline__ void l2_prefetch(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Issue (from lane 0) the L2 prefetches of this warp's share of a GEMV phase, at most
// `max_items` items.
__device__ __forceinline__ void prefetch_gemv(const Gemv &g, int wg, int W, int lane, int max_items) {
  if (lane != 0) return;
  int k = 0;
  for (int item = wg; item < g.items && k < max_items; item += W, ++k) {
    const int tile = item / g.P, p = item % g.P;
    l2_prefetch(g.w + (static_cast<int64_t>(tile) * g.cpt + p * g.upp) * kUnitBytes,
                static_cast<uint32_t>(g.upp * kUnitBytes));
  }
}

// Ordered key of a bf16 logit for atomicMax: larger value wins, then the lower row.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (v != v) u = 0u;  // NaN never wins
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned>(~row);
}

// ---- attention work items --------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// Items (b, kv head, chunk) enumerated sequence by sequence.
__device__ __forceinline__ bool attn_item(const Args &a, const int *posv, int item, int &b, int &h, int &c) {
  for (b = 0; b < a.B; ++b) {
    const int nch = (posv[b] + 1 + kChunk - 1) / kChunk;
    if (item < nch * kHkv) {
      h = item / nch;
      c = item % nch;
      return true;
    }
    item -= nch * kHkv;
  }
  return false;
}

__device__ void attn_phase(const Args &a, const Layer &ly, const int *posv, int wg, int W, int lane,
                           uint16_t *qs, uint16_t *vs) {
  const int gid = lane >> 2, tid = lane & 3;
  for (int item = wg;; item += W) {
    int b, h, c;
    if (!attn_item(a, posv, item, b, h, c)) break;
    const int p = posv[b];
    const int nch = (p + 1 + kChunk - 1) / kChunk;
    const float *ang = a.lut + static_cast<int64_t>(p) * kD;
    const uint16_t *src = a.qkv + static_cast<int64_t>(b) * kQKV;
    // RoPE of the group's 4 query heads into the warp's q buffer (two-halves rotation,
    // fp32, rounded once: rope_kv_append_kernel's arithmetic)
    {
      const float cs = ang[2 * lane], sn = ang[2 * lane + 1];
#pragma unroll
      for (int r = 0; r < kG; ++r) {
        const uint16_t *xq = src + (h * kG + r) * kD;
        const float x1 = bf16_bits_to_float(ld_cg_u16(xq + lane)), x2 = bf16_bits_to_float(ld_cg_u16(xq + lane + 32));
        qs[r * kD + lane] = float_to_bf16_bits(x1 * cs - x2 * sn);
        qs[r * kD + lane + 32] = float_to_bf16_bits(x1 * sn + x2 * cs);
      }
      if (c == nch - 1) {
        // the chunk holding position p appends the new k (roped) and v to the cache
        const uint16_t *xk = src + (kHq + h) * kD, *xv = src + (kHq + kHkv + h) * kD;
        const float x1 = bf16_bits_to_float(ld_cg_u16(xk + lane)), x2 = bf16_bits_to_float(ld_cg_u16(xk + lane + 32));
        uint16_t *kd = ly.kc + b * a.kv_b + h * a.kv_h + static_cast<int64_t>(p) * kD;
        uint16_t *vd = ly.vc + b * a.kv_b + h * a.kv_h + static_cast<int64_t>(p) * kD;
        kd[lane] = float_to_bf16_bits(x1 * cs - x2 * sn);
        kd[lane + 32] = float_to_bf16_bits(x1 * sn + x2 * cs);
        vd[lane] = ld_cg_u16(xv + lane);
        vd[lane + 32] = ld_cg_u16(xv + lane + 32);
        __threadfence_block();
      }
    }
    __syncwarp();
    // Q fragments (rows = the group's heads, rows >= 4 zero), permuted k order
    uint32_t qa[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int d = 32 * (ks >> 1) + 8 * tid + 4 * (ks & 1);
      const uint32_t *q0 = reinterpret_cast<const uint32_t *>(qs + gid * kD + d);
      qa[ks][0] = gid < kG ? q0[0] : 0u;
      qa[ks][1] = 0u;
      qa[ks][2] = gid < kG ? q0[1] : 0u;
      qa[ks][3] = 0u;
    }
    const uint16_t *kb = ly.kc + b * a.kv_b + h * a.kv_h;
    const uint16_t *vb = ly.vc + b * a.kv_b + h * a.kv_h;
    const int t_begin = c * kChunk, t_end = min(p + 1, t_begin + kChunk);
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_lo = -INFINITY, l_lo = 0.f;
    for (int blk = t_begin; blk < t_end; blk += 16) {
      uint4 kr[2][2], vr[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int t = blk + nt * 8 + gid;
#pragma unroll
        for (int db = 0; db < 2; ++db)
          kr[nt][db] = t < t_end ? ld_cg4(kb + static_cast<int64_t>(t) * kD + db * 32 + tid * 8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = i * 32 + lane, row = idx >> 3, c16 = idx & 7;
        const int t = blk + row;
        vr[i] = t < t_end ? ld_cg4(vb + static_cast<int64_t>(t) * kD + c16 * 8) : make_uint4(0, 0, 0, 0);
      }
      __syncwarp();  // previous block's V tile reads done
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = i * 32 + lane, row = idx >> 3, c16 = idx & 7;
        *reinterpret_cast<uint4 *>(vs + row * kVStride + c16 * 8) = vr[i];
      }
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint4 &w = kr[nt][ks >> 1];
          mma_bf16_16816(s[nt], qa[ks], (ks & 1) ? w.z : w.x, (ks & 1) ? w.w : w.y);
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = blk + nt * 8 + 2 * tid + e;
          s[nt][e] = t < t_end ? s[nt][e] * a.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[nt][e]);
        }
#pragma unroll
      for (int x = 1; x <= 2; x <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
      const float mn = fmaxf(m_lo, mx);
      const float al = mn == -INFINITY ? 1.f : exp2f(m_lo - mn);
      m_lo = mn;
      float ps = 0.f;
      float pr[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          pr[nt][e] = mn == -INFINITY ? 0.f : exp2f(s[nt][e] - mn);
          ps += pr[nt][e];
        }
      l_lo = l_lo * al + ps;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j][0] *= al;
        o[j][1] *= al;
      }
      const uint32_t pa[4] = {pack_bf16x2(pr[0][0], pr[0][1]), 0u, pack_bf16x2(pr[1][0], pr[1][1]), 0u};
      __syncwarp();  // V tile visible to ldmatrix
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = jp * 16 + (lane >> 4) * 8;
        uint32_t vb4[4];
        ldsm_x4_t(vb4, vs + row * kVStride + col);
        mma_bf16_16816(o[2 * jp], pa, vb4[0], vb4[1]);
        mma_bf16_16816(o[2 * jp + 1], pa, vb4[2], vb4[3]);
      }
    }
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) l_lo += __shfl_xor_sync(0xffffffffu, l_lo, x);
    // partial (m, l, o) of rows 0..3 (heads of the group)
    float *pp = a.apart + ((static_cast<int64_t>(b) * kHkv + h) * a.max_chunks + c) * (kG * 66);
    if (gid < kG) {
      if (tid == 0) {
        pp[gid * 66] = m_lo;
        pp[gid * 66 + 1] = l_lo;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        pp[gid * 66 + 2 + 8 * j + 2 * tid] = o[j][0];
        pp[gid * 66 + 2 + 8 * j + 2 * tid + 1] = o[j][1];
      }
    }
    __threadfence();
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = atomicAdd(a.hcnt + b * kHkv + h, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == static_cast<unsigned>(nch - 1)) {
      // last chunk of this (sequence, kv head): merge the chunks in order
      __threadfence();
      const float *p0 = a.apart + (static_cast<int64_t>(b) * kHkv + h) * a.max_chunks * (kG * 66);
#pragma unroll
      for (int r = 0; r < kG; ++r) {
        float M = -INFINITY;
        for (int q = 0; q < nch; ++q) M = fmaxf(M, ld_cg_f(p0 + q * (kG * 66) + r * 66));
        float Lsum = 0.f, O0 = 0.f, O1 = 0.f;
        if (M != -INFINITY) {
          for (int q = 0; q < nch; ++q) {
            const float *pq = p0 + q * (kG * 66) + r * 66;
            const float f = exp2f(ld_cg_f(pq) - M);
            Lsum += ld_cg_f(pq + 1) * f;
            O0 += ld_cg_f(pq + 2 + lane) * f;
            O1 += ld_cg_f(pq + 2 + 32 + lane) * f;
          }
        }
        const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
        uint16_t *dst = a.attn + static_cast<int64_t>(b) * kE + (h * kG + r) * kD;
        dst[lane] = float_to_bf16_bits(O0 * inv);
        dst[lane + 32] = float_to_bf16_bits(O1 * inv);
      }
      if (lane == 0) a.hcnt[b * kHkv + h] = 0u;
    }
  }
}

// L2 prefetch of phase `ph` (5 per layer: QKV, ATTN, O, GU, D; then LM): the weights
// of this warp's work items, or for ATTN the cached K/V rows of its chunks. Issued
// two phases ahead, so HBM streams while the grid computes and syncs.
__device__ void prefetch_phase(const Args &a, int ph, const int *posv, int wg, int W, int lane) {
  if (ph > 5 * a.n_layers) return;
  if (ph == 5 * a.n_layers) {
    prefetch_gemv(make_gemv(a.lm, a.V, kE, 1), wg, W, lane, 3);  // the head of the 263 MB lm-head share
    return;
  }
  const Layer &ly = a.layers[ph / 5];
  switch (ph % 5) {
    case 0: prefetch_gemv(make_gemv(ly.qkv, kQKV, kE, 8), wg, W, lane, 1 << 30); break;
    case 2: prefetch_gemv(make_gemv(ly.o, kE, kE, 16), wg, W, lane, 1 << 30); break;
    case 3: prefetch_gemv(make_gemv(ly.gu, 2 * kHid, kE, 2), wg, W, lane, 1 << 30); break;
    case 4: prefetch_gemv(make_gemv(ly.d, kE, kHid, 16), wg, W, lane, 1 << 30); break;
    default: {
      if (lane != 0) return;
      for (int item = wg;; item += W) {
        int b, h, c;
        if (!attn_item(a, posv, item, b, h, c)) break;
        const int t0 = c * kChunk, t1 = min(posv[b], t0 + kChunk);  // rows already cached
        if (t1 <= t0) continue;
        const int64_t off = b * a.kv_b + h * a.kv_h + static_cast<int64_t>(t0) * kD;
        l2_prefetch(ly.kc + off, static_cast<uint32_t>((t1 - t0) * kD * 2));
        l2_prefetch(ly.vc + off, static_cast<uint32_t>((t1 - t0) * kD * 2));
      }
    }
  }
}

// ---- the kernel ----------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(Args a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem);                    // [B, E] normalised input
  float *red = reinterpret_cast<float *>(smem + kMaxB * kE * 2);         // [kWarps]
  uint8_t *warp_area = smem + kMaxB * kE * 2 + 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint16_t *qs = reinterpret_cast<uint16_t *>(warp_area + warp * (kG * kD * 2 + 16 * kVStride * 2));
  uint16_t *vs = qs + kG * kD;
  const int wg = blockIdx.x * kWarps + warp, W = gridDim.x * kWarps;
  __shared__ int posv[kMaxB];
  __shared__ int tokv[kMaxB];
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  if (threadIdx.x < a.B) {
    const int p = a.pos[threadIdx.x], t = a.tokens[threadIdx.x];
    posv[threadIdx.x] = p;
    tokv[threadIdx.x] = t;
    if (p < 0 || p >= a.L || t < 0 || t >= a.V) bad = 1;  // would index past the cache / table
  }
  __syncthreads();
  if (bad) {  // every CTA sees the same inputs and leaves before any barrier
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.status, 2u);
    return;
  }

  const int B = a.B;
  UnitRegs pre[kPre];
  bool ok = true;
  prefetch_phase(a, 0, posv, wg, W, lane);
  prefetch_phase(a, 1, posv, wg, W, lane);
  for (int l = 0; l < a.n_layers && ok; ++l) {
    const Layer ly = a.layers[l];
    // QKV: x (the embedding rows for layer 0) -> RMSNorm -> GEMV
    const Gemv gq = make_gemv(ly.qkv, kQKV, kE, 8);
    int npre = gemv_prefetch(gq, pre, wg, lane);
    if (l > 0) ok = grid_sync(a);  // x from the previous layer's D phase
    if (!ok) break;
    prefetch_phase(a, 5 * l + 2, posv, wg, W, lane);
    rmsnorm_to_smem(l == 0 ? a.embed : a.x, l == 0 ? tokv : nullptr, ly.n1, xs, B, a.eps, red);
    if (l == 0 && blockIdx.x == 0) {  // the residual stream starts as the embedding rows
      for (int i = threadIdx.x; i < B * kE / 8; i += kThreads) {
        const int b = i / (kE / 8), c = (i % (kE / 8)) * 8;
        *reinterpret_cast<uint4 *>(a.x + b * kE + c) =
            __ldg(reinterpret_cast<const uint4 *>(a.embed + static_cast<int64_t>(tokv[b]) * kE + c));
      }
    }
    gemv_run<true>(gq, pre, npre, xs, B, a.part, a.cnt, wg, W, lane, [&](int tile, const float (&v)[4]) {
      const int gid = lane >> 2, tid = lane & 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = tile * 16 + gid + ((e >> 1) << 3), vv = 2 * tid + (e & 1);
        if (vv < B) a.qkv[static_cast<int64_t>(vv) * kQKV + row] = float_to_bf16_bits(v[e]);
      }
    });
    ok = grid_sync(a);
    if (!ok) break;
    // ATTN
    prefetch_phase(a, 5 * l + 3, posv, wg, W, lane);
    attn_phase(a, ly, posv, wg, W, lane, qs, vs);
    // O: prefetch, barrier, GEMV on attn (+ x residual) -> h
    const Gemv go = make_gemv(ly.o, kE, kE, 16);
    npre = gemv_prefetch(go, pre, wg, lane);
    ok = grid_sync(a);
    if (!ok) break;
    prefetch_phase(a, 5 * l + 4, posv, wg, W, lane);
    gemv_run<false>(go, pre, npre, a.attn, B, a.part, a.cnt, wg, W, lane, [&](int tile, const float (&v)[4]) {
      const int gid = lane >> 2, tid = lane & 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = tile * 16 + gid + ((e >> 1) << 3), vv = 2 * tid + (e & 1);
        if (vv < B) {
          const int64_t o = static_cast<int64_t>(vv) * kE + row;
          a.h[o] = float_to_bf16_bits(__bfloat162float(__float2bfloat16_rn(v[e])) + bf16_bits_to_float(ld_cg_u16(a.x + o)));
        }
      }
    });
    // GU: prefetch, barrier, RMSNorm(h), GEMV, SwiGLU -> act
    const Gemv gg = make_gemv(ly.gu, 2 * kHid, kE, 2);
    npre = gemv_prefetch(gg, pre, wg, lane);
    ok = grid_sync(a);
    if (!ok) break;
    prefetch_phase(a, 5 * l + 5, posv, wg, W, lane);
    rmsnorm_to_smem(a.h, nullptr, ly.n2, xs, B, a.eps, red);
    gemv_run<true>(gg, pre, npre, xs, B, a.part, a.cnt, wg, W, lane, [&](int tile, const float (&v)[4]) {
      const int gid = lane >> 2, tid = lane & 3;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int vv = 2 * tid + e;
        if (vv < B) {
          const float gte = __bfloat162float(__float2bfloat16_rn(v[e]));
          const float up = __bfloat162float(__float2bfloat16_rn(v[e + 2]));
          const float sw = __bfloat162float(__float2bfloat16_rn(gte / (1.f + __expf(-gte))));
          a.act[static_cast<int64_t>(vv) * kHid + tile * 8 + gid] = float_to_bf16_bits(sw * up);
        }
      }
    });
    // D: prefetch, barrier, GEMV on act (+ h residual) -> x
    const Gemv gd = make_gemv(ly.d, kE, kHid, 16);
    npre = gemv_prefetch(gd, pre, wg, lane);
    ok = grid_sync(a);
    if (!ok) break;
    prefetch_phase(a, 5 * l + 6, posv, wg, W, lane);
    gemv_run<false>(gd, pre, npre, a.act, B, a.part, a.cnt, wg, W, lane, [&](int tile, const float (&v)[4]) {
      const int gid = lane >> 2, tid = lane & 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = tile * 16 + gid + ((e >> 1) << 3), vv = 2 * tid + (e & 1);
        if (vv < B) {
          const int64_t o = static_cast<int64_t>(vv) * kE + row;
          a.x[o] = float_to_bf16_bits(__bfloat162float(__float2bfloat16_rn(v[e])) + bf16_bits_to_float(ld_cg_u16(a.h + o)));
        }
      }
    });
  }
  if (ok) {
    // LM: RMSNorm(x), lm-head GEMV (whole tiles), argmax keys
    const Gemv gl = make_gemv(a.lm, a.V, kE, 1);
    const int npre = gemv_prefetch(gl, pre, wg, lane);
    ok = grid_sync(a);
    if (ok) {
      rmsnorm_to_smem(a.x, nullptr, a.nf, xs, B, a.eps, red);
      gemv_run<true>(gl, pre, npre, xs, B, a.part, a.cnt, wg, W, lane, [&](int tile, const float (&v)[4]) {
        const int gid = lane >> 2, tid = lane & 3;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = tile * 16 + gid + ((e >> 1) << 3), vv = 2 * tid + (e & 1);
          if (vv < B) {
            const uint16_t lb = float_to_bf16_bits(v[e]);
            if (a.logits) a.logits[static_cast<int64_t>(vv) * a.V + row] = lb;
            atomicMax(a.amax + vv, argmax_key(bf16_bits_to_float(lb), row));
          }
        }
      });
      ok = grid_sync(a);
      if (ok && blockIdx.x == 0 && threadIdx.x < B) {
        const unsigned long long k = atomicExch(a.amax + threadIdx.x, 0ull);
        a.tokens[threadIdx.x] = static_cast<int>(~static_cast<unsigned>(k & 0xffffffffull));
        a.pos[threadIdx.x] = posv[threadIdx.x] + 1;
      }
    }
  }
}

}  // namespace mk
}  // namespace iron

using namespace iron;

extern "C" size_t iron_llama_decode_persistent_scratch_bytes(int B, int max_seq) {
  if (B <= 0 || B > mk::kMaxB || max_seq <= 0) return 0;
  const size_t part = static_cast<size_t>(1024) * 2 * 128 * sizeof(float);  // largest T * P * 128 floats
  const size_t chunks = (max_seq + mk::kChunk - 1) / mk::kChunk;
  const size_t apart = static_cast<size_t>(B) * mk::kHkv * chunks * mk::kG * 66 * sizeof(float);
  const size_t cnt = 8192 * sizeof(unsigned);
  const size_t hcnt = mk::kMaxB * mk::kHkv * sizeof(unsigned);
  return part + apart + cnt + hcnt + 64 * 8 + 256;
}

extern "C" int iron_llama_decode_persistent(const void *layers, int n_layers, const uint16_t *embed,
                                            const uint16_t *final_norm, const uint8_t *lm_head, int vocab,
                                            const float *rope_lut, int32_t *tokens, int32_t *pos,
                                            uint16_t *x, uint16_t *h, uint16_t *qkv, uint16_t *attn,
                                            uint16_t *act, uint16_t *logits, int B, int max_seq,
                                            int64_t kv_batch_stride, int64_t kv_head_stride, float eps,
                                            void *scratch, size_t scratch_bytes, unsigned *status,
                                            unsigned flags, void *stream) {
  if (!layers || !embed || !final_norm || !lm_head || !rope_lut || !tokens || !pos || !x || !h || !qkv ||
      !attn || !act || !scratch || !status)
    return IRON_ERR_NULL;
  if (B <= 0 || B > mk::kMaxB || n_layers <= 0 || vocab <= 0 || vocab % 16 || max_seq <= 0) return IRON_ERR_SHAPE;
  if (scratch_bytes < iron_llama_decode_persistent_scratch_bytes(B, max_seq)) return IRON_ERR_WORKSPACE;
  if (!aligned16(scratch) || !aligned16(x) || !aligned16(h) || !aligned16(act) || !aligned16(embed))
    return IRON_ERR_ALIGN;
  mk::Args a;
  a.layers = static_cast<const mk::Layer *>(layers);
  a.n_layers = n_layers;
  a.embed = embed;
  a.nf = final_norm;
  a.lm = lm_head;
  a.V = vocab;
  a.lut = rope_lut;
  a.tokens = tokens;
  a.pos = pos;
  a.x = x;
  a.h = h;
  a.qkv = qkv;
  a.attn = attn;
  a.act = act;
  a.logits = logits;
  uint8_t *s = static_cast<uint8_t *>(scratch);
  a.part = reinterpret_cast<float *>(s);
  s += static_cast<size_t>(1024) * 2 * 128 * sizeof(float);
  a.max_chunks = (max_seq + mk::kChunk - 1) / mk::kChunk;
  a.apart = reinterpret_cast<float *>(s);
  s += static_cast<size_t>(B) * mk::kHkv * a.max_chunks * mk::kG * 66 * sizeof(float);
  a.cnt = reinterpret_cast<unsigned *>(s);
  s += 8192 * sizeof(unsigned);
  a.hcnt = reinterpret_cast<unsigned *>(s);
  s += mk::kMaxB * mk::kHkv * sizeof(unsigned);
  s = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(s) + 63) & ~static_cast<uintptr_t>(63));
  a.amax = reinterpret_cast<unsigned long long *>(s);
  s += mk::kMaxB * 8;
  a.bar = reinterpret_cast<unsigned *>(s);
  a.status = status;
  a.B = B;
  a.L = max_seq;
  a.kv_b = kv_batch_stride;
  a.kv_h = kv_head_stride;
  a.eps = eps;
  a.scale_log2 = 0.125f * 1.4426950408889634f;  // 1 / sqrt(64)
  const size_t smem = mk::kMaxB * mk::kE * 2 + 128 + mk::kWarps * (mk::kG * mk::kD * 2 + 16 * mk::kVStride * 2);
  static PerDeviceOnce attr_set;  // per device: the shared memory opt-in
  const int ast = attr_set.run([&]() {
    return call_status(cudaFuncSetAttribute(mk::decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)));
  });
  if (ast != IRON_OK) return ast;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(mk::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  // cooperative: every CTA resident (the grid barrier needs it). No programmatic
  // dependent launch: the step reads what the previous launch wrote.
  (void)flags;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, mk::decode_step_kernel, a);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}
