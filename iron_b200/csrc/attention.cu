// GQA decode attention with split-KV (flash-decoding) and the combine pass.
//
// Replaces the decode attention of IRON's Llama pipeline -- the Repeat x2,
// score GEMV, scale, masked Softmax, 32x Transpose and context GEMV of
// iron/applications/llama_3.2_1b/llama_npu.py:495-529 (CPU truth
// iron/applications/llama_3.2_1b/llama_cpu.py:118-140) -- which copy the whole
// padded cache several times per token, by one pass over each sequence's valid
// K/V rows.
//
// One CTA = (split, kv head, sequence); its four warps take 16-token blocks in
// turn. The query heads sharing the kv head (the GQA group, <= 16) are the rows
// of m16n8k16 bf16 MMAs: S = Q K^T reads K fragments straight from the cache rows
// (the logical k order inside an MMA is free as long as A and B agree, so each
// lane feeds its own 16 contiguous bytes), the online softmax runs in fp32 in
// exp2 space, and O += P V takes P from the S accumulators and V through a
// padded shared-memory tile read with ldmatrix.trans. Partial (max, sum, O) of
// each split go to the workspace; a second kernel merges the splits.
// Memory-bound: each cache row is read once per kv head, not once per q head.
#include <mutex>

#include <cooperative_groups.h>

#include "common.cuh"

namespace iron {

namespace cg = cooperative_groups;

// Head dims: 64 (Llama-3.2-1B; IRON's MHA supports d = 64 only, mha/op.py:39-41) and
// 128 (the Llama-3-8B block).
constexpr int kAWarps = 4;
// warps per CTA in the cluster form at head_dim 64: one 16-token block per warp, so a
// split of up to 128 tokens (2048 per sequence in 16 CTAs) is requested entirely before
// the wait (B200, batch 1 at 2048 tokens: the 4-warp CTA walked 3 blocks per warp, two of
// them after the wait -- 2.6 us of a 5.7 us attention). Two such CTAs must fit an SM
// (launch bound 2): at 12 warps a CTA held most of an SM's registers, and 16-CTA
// clusters that need 16 free SMs of one GPC went out in two waves (measured: a tenth
// of the CTAs started 4.7 us late). head_dim 128 keeps 4 warps (registers and shared
// memory).
constexpr int kAClusterWarps = 8;
template <int kAD>
constexpr int attn_cluster_warps() { return kAD == 64 ? kAClusterWarps : kAWarps; }
template <int kAD, int kCS>
constexpr int attn_min_ctas() { return (kCS > 1 && kAD == 64) ? 2 : 0; }
constexpr int kABlk = 16;     // tokens per warp step
constexpr int kAMinChunk = 64;   // tokens per split at least
constexpr int kAMaxSplits = 64;  // splits per sequence at most (the combine holds one value per split)
// tokens per CTA at most (while splits are left): one CTA streams about one 16-token
// block per warp per memory round trip, so in a ragged batch the CTA of the longest
// sequence would otherwise set the time (B200, batch 64 at up to 32768 tokens)
constexpr int kAMaxChunk = 4096;
// tokens per CTA at most in the cluster form (16 or 8 CTAs per (sequence, kv head)):
// beyond it the few clusters cannot keep enough rows in flight
constexpr int kAClusterMaxChunk = 512;

struct AttnArgs {
  const uint16_t *q;    // [B, Hq, D]
  const uint16_t *k;    // cache, element (b, h, t, d) at b*bstride + h*hstride + t*D + d
  const uint16_t *v;
  const int *lens;      // [B] valid tokens per sequence
  uint16_t *out;        // [B, Hq, D]
  float *ws;            // [B, Hq, splits, 2 + D] partial (max, sum, o)
  int64_t bstride, hstride;
  int Hq, Hkv, splits, chunk;
  int maxlen;           // cache rows per (sequence, kv head): lengths / positions beyond it do nothing
  int l2_prefetch;      // fused form: request the split's cached rows into L2 before the wait
  float scale_log2;     // softmax scale * log2(e)
  // fused decode form: q, the new k and v come from the QKV projection `qkv`
  // [B, (Hq + 2 Hkv) D] at position pos[b] (RoPE from `lut`, the new rows appended to
  // the cache)
  const uint16_t *qkv;
  const int *pos;
  const float *lut;
};

// cache rows: written by earlier steps, or (row p) by the RoPE + append kernel that
// precedes this one and lets it launch only at its end -- constant while this runs
__device__ __forceinline__ uint4 ldg16(const uint16_t *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// kCS > 1: the splits of one (sequence, kv head) are a thread-block cluster of kCS
// CTAs (gridDim.x == kCS); each CTA writes its (max, sum, output) rows into rank 0's
// shared memory and rank 0 merges them in rank order after one cluster barrier -- no
// workspace, no second kernel.
template <int kAD, bool kFused = false, int kCS = 1>
__global__ void __launch_bounds__(32 * ((kCS > 1 && kAD == 64) ? kAClusterWarps : kAWarps), attn_min_ctas<kAD, kCS>())
attn_decode_kernel(AttnArgs a) {
  constexpr int kW = (kCS > 1 && kAD == 64) ? kAClusterWarps : kAWarps;  // warps of this CTA
  constexpr int kG = kCS > 1 ? 4 : 16;                    // query-head rows kept per warp (the cluster form: g <= 4)
  constexpr int kAVStride = kAD + 8;  // padded V tile row: an odd number of 16-byte chunks
  constexpr int kVBytes = kW * kABlk * kAVStride * 2;
  constexpr int kOBytes = kW * kG * kAD * 4;
  // the V tiles (loop) and the warp-merge buffer (after it) share the storage
  __shared__ __align__(16) uint8_t smem[kVBytes > kOBytes ? kVBytes : kOBytes];
  __shared__ float red_m[kW][16], red_l[kW][16];
  extern __shared__ __align__(16) float cbuf[];  // kCS > 1 (rank 0): [kCS][g][2 + kAD]
  uint16_t (*vtile)[kABlk * kAVStride] = reinterpret_cast<uint16_t (*)[kABlk * kAVStride]>(smem);
  float (*red_o)[kG][kAD] = reinterpret_cast<float (*)[kG][kAD]>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid = lane & 3;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = a.Hq / a.Hkv;      // query heads per kv head (MMA rows used)
  const int hq0 = h * g;

  // fused form: the group's roped q rows and the new k / v row, staged here
  __shared__ __align__(16) uint16_t qbuf[kFused ? 16 * kAD : 8];
  __shared__ __align__(16) uint16_t knew[kFused ? kAD : 8], vnew[kFused ? kAD : 8];

  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  int len, p = -1;
  bool valid = true;
  if constexpr (kFused) {
    // pos is final before this launch (written by the previous step, which the step's
    // first kernel waits for), so it and the cached rows below it are read before the
    // wait for the QKV projection
    p = ld_act_i32(a.pos + b);
    valid = p >= 0 && p < a.maxlen;
    if (!valid) p = 0;
    len = valid ? p + 1 : 0;
  } else {
    pdl_wait();
    len = min(max(ld_act_i32(a.lens + b), 0), a.maxlen);
  }
  const int t_begin = split * a.chunk;
  const int t_end = min(len, t_begin + a.chunk);

  const uint16_t *kb = a.k + b * a.bstride + h * a.hstride;
  const uint16_t *vb = a.v + b * a.bstride + h * a.hstride;

  // register prefetch of one block: K rows (token gid of each 8-token half, 16 B x 2)
  // and this lane's four 16-byte pieces of the V tile
  constexpr int kDB = kAD / 32;  // 16-byte K pieces per token per lane
  constexpr int kVR = kAD / 16;  // 16-byte V pieces per lane per block
  // (fused form: the new token's row comes from the staged knew / vnew once `staged`)
  auto load_block = [&](int blk, uint4 (&kr)[2][kDB], uint4 (&vr)[kVR], bool staged) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int t = blk + nt * 8 + gid;
#pragma unroll
      for (int db = 0; db < kDB; ++db)
        kr[nt][db] = t >= t_end ? make_uint4(0u, 0u, 0u, 0u)
                     : (kFused && t == p) ? (staged ? *reinterpret_cast<const uint4 *>(knew + db * 32 + tid * 8)
                                                   : make_uint4(0u, 0u, 0u, 0u))
                                          : ldg16(kb + static_cast<int64_t>(t) * kAD + db * 32 + tid * 8);
    }
#pragma unroll
    for (int i = 0; i < kVR; ++i) {
      const int idx = i * 32 + lane, row = idx / (kAD / 8), c16 = idx % (kAD / 8);
      const int t = blk + row;
      vr[i] = t >= t_end ? make_uint4(0u, 0u, 0u, 0u)
              : (kFused && t == p) ? (staged ? *reinterpret_cast<const uint4 *>(vnew + c16 * 8)
                                             : make_uint4(0u, 0u, 0u, 0u))
                                   : ldg16(vb + static_cast<int64_t>(t) * kAD + c16 * 8);
    }
  };

  uint4 kr[2][kDB], vr[kVR];
  int blk = t_begin + warp * kABlk;
  // the first block's cache rows are requested before anything else (they do not
  // depend on the QKV projection; the fused form's new row p comes later)
  if (blk < t_end) load_block(blk, kr, vr, false);
  if constexpr (kFused) {
    // the split's further cached rows into L2, then wait for the QKV projection
    const int r0 = t_begin + kW * kABlk, r1 = min(t_end, p);
    if (a.l2_prefetch && threadIdx.x == 0 && r1 > r0) {
      const uint32_t bytes = static_cast<uint32_t>(r1 - r0) * kAD * 2;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kb + static_cast<int64_t>(r0) * kAD), "r"(bytes)
                   : "memory");
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vb + static_cast<int64_t>(r0) * kAD), "r"(bytes)
                   : "memory");
    }
    pdl_wait();
  }

  const uint16_t *qrow = a.q;
  int64_t qstride = kAD;
  if constexpr (kFused) {
    // RoPE (two halves, fp32, rounded once: rope_kv_append_kernel's arithmetic) of the
    // group's q heads and of the new k; the split that holds position p appends k, v
    const int half = kAD / 2;
    const uint16_t *src = a.qkv + static_cast<int64_t>(b) * (a.Hq + 2 * a.Hkv) * kAD;
    const float *ang = a.lut + static_cast<int64_t>(p) * kAD;
    const bool owner = valid && t_begin <= p && p < t_begin + a.chunk;
    // zero rows g..15 of the q tile (no loads)
    for (int i = g * kAD + threadIdx.x * 8; i < 16 * kAD; i += 32 * kW * 8)
      *reinterpret_cast<uint4 *>(qbuf + i) = make_uint4(0u, 0u, 0u, 0u);
    // one pass: every thread issues the loads of its q pair and (the first `half`
    // threads) of its new k / v pair before using any of them -- one L2 round trip
    for (int i0 = 0; i0 < g * half || i0 < half; i0 += 32 * kW) {
      const int i = i0 + threadIdx.x;
      const bool hq_ = i < g * half, hk_ = i < half;
      const int r = hq_ ? i / half : 0, jq = hq_ ? i % half : 0;
      const uint16_t *xq = src + (hq0 + r) * kAD;
      const uint16_t *xk = src + (a.Hq + h) * kAD, *xv = src + (a.Hq + a.Hkv + h) * kAD;
      uint16_t q1 = 0, q2 = 0, k1r = 0, k2r = 0, v1 = 0, v2 = 0;
      float cq = 0.f, sq = 0.f, ck = 0.f, sk = 0.f;
      if (hq_) {
        q1 = ld_act_u16(xq + jq);
        q2 = ld_act_u16(xq + jq + half);
        cq = ang[2 * jq];
        sq = ang[2 * jq + 1];
      }
      if (hk_) {
        k1r = ld_act_u16(xk + i);
        k2r = ld_act_u16(xk + i + half);
        v1 = ld_act_u16(xv + i);
        v2 = ld_act_u16(xv + i + half);
        ck = ang[2 * i];
        sk = ang[2 * i + 1];
      }
      if (hq_) {
        const float x1 = bf16_bits_to_float(q1), x2 = bf16_bits_to_float(q2);
        qbuf[r * kAD + jq] = float_to_bf16_bits(x1 * cq - x2 * sq);
        qbuf[r * kAD + jq + half] = float_to_bf16_bits(x1 * sq + x2 * cq);
      }
      if (hk_) {
        const float x1 = bf16_bits_to_float(k1r), x2 = bf16_bits_to_float(k2r);
        const uint16_t k1 = float_to_bf16_bits(x1 * ck - x2 * sk), k2 = float_to_bf16_bits(x1 * sk + x2 * ck);
        knew[i] = k1;
        knew[i + half] = k2;
        vnew[i] = v1;
        vnew[i + half] = v2;
        if (owner) {
          // the fused entry passes writable caches
          uint16_t *kd = const_cast<uint16_t *>(a.k) + b * a.bstride + h * a.hstride + static_cast<int64_t>(p) * kAD;
          uint16_t *vd = const_cast<uint16_t *>(a.v) + b * a.bstride + h * a.hstride + static_cast<int64_t>(p) * kAD;
          kd[i] = k1;
          kd[i + half] = k2;
          vd[i] = v1;
          vd[i + half] = v2;
        }
      }
    }
    __syncthreads();
    qrow = qbuf;
    if (blk < t_end && blk <= p && p < blk + kABlk) load_block(blk, kr, vr, true);
  }

  // Q fragments (rows = heads of the group; rows >= g are zero). k-step ks covers
  // physical d = 32*(ks/2) + 8*tid + 4*(ks%2) + {0,1 | 2,3} for logical {2tid | 2tid+8}.
  uint32_t qa[kAD / 16][4];
#pragma unroll
  for (int ks = 0; ks < kAD / 16; ++ks) {
    const int d = 32 * (ks >> 1) + 8 * tid + 4 * (ks & 1);
    const uint16_t *qr0 = kFused ? qrow + gid * kAD : qrow + (static_cast<int64_t>(b) * a.Hq + hq0 + gid) * qstride;
    const uint16_t *qr8 = kFused ? qrow + (gid + 8) * kAD : qrow + (static_cast<int64_t>(b) * a.Hq + hq0 + gid + 8) * qstride;
    const uint32_t *q0 = reinterpret_cast<const uint32_t *>(qr0 + d);
    const uint32_t *q8 = reinterpret_cast<const uint32_t *>(qr8 + d);
    // fused: the staged q tile in shared memory; else q from the RoPE kernel's output
    qa[ks][0] = gid < g ? (kFused ? q0[0] : ld_act_u32(q0)) : 0u;
    qa[ks][1] = gid + 8 < g ? (kFused ? q8[0] : ld_act_u32(q8)) : 0u;
    qa[ks][2] = gid < g ? (kFused ? q0[1] : ld_act_u32(q0 + 1)) : 0u;
    qa[ks][3] = gid + 8 < g ? (kFused ? q8[1] : ld_act_u32(q8 + 1)) : 0u;
  }

  float o[kAD / 8][4];
#pragma unroll
  for (int j = 0; j < kAD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY;  // running max of rows gid / gid+8 (log2 units)
  float l_lo = 0.f, l_hi = 0.f;              // this lane's share of the running sums
  uint16_t *vs = vtile[warp];

  for (; blk < t_end; blk += kW * kABlk) {
    // stage V, then prefetch the next block while this one computes
#pragma unroll
    for (int i = 0; i < kVR; ++i) {
      const int idx = i * 32 + lane, row = idx / (kAD / 8), c16 = idx % (kAD / 8);
      *reinterpret_cast<uint4 *>(vs + row * kAVStride + c16 * 8) = vr[i];
    }
    uint4 kc[2][kDB];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int db = 0; db < kDB; ++db) kc[nt][db] = kr[nt][db];
    const int nxt = blk + kW * kABlk;
    if (nxt < t_end) load_block(nxt, kr, vr, true);
    // the stand-alone form (long, ragged caches): the block after the next one goes to L2
    // now, so each warp has one block in registers and one in flight from DRAM without
    // more registers (B200, config 4: 5.93 -> 6.46 TB/s, 353 -> 323 us; in the fused
    // decode step it measured slightly slower: batch 64 1.815 against 1.806 ms per step)
    if (!kFused && lane == 0) {
      const int pf = nxt + kW * kABlk;
      if (pf < t_end) {
        const uint32_t bytes = static_cast<uint32_t>(min(kABlk, t_end - pf)) * kAD * 2;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kb + static_cast<int64_t>(pf) * kAD), "r"(bytes)
                     : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vb + static_cast<int64_t>(pf) * kAD), "r"(bytes)
                     : "memory");
      }
    }

    // S = Q K^T for the two 8-token halves
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < kAD / 16; ++ks) {
        const uint4 &w = kc[nt][ks >> 1];
        const uint32_t b0 = (ks & 1) ? w.z : w.x, b1 = (ks & 1) ? w.w : w.y;
        mma_bf16_16816(s[nt], qa[ks], b0, b1);
      }
    }
    // scale, mask (only the cache's ragged last block has tokens past t_end), block max
    // per row
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
    if (blk + kABlk <= t_end) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[nt][e] *= a.scale_log2;
          if (e < 2) mx_lo = fmaxf(mx_lo, s[nt][e]); else mx_hi = fmaxf(mx_hi, s[nt][e]);
        }
    } else {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = blk + nt * 8 + 2 * tid + (e & 1);
          s[nt][e] = t < t_end ? s[nt][e] * a.scale_log2 : -INFINITY;
          if (e < 2) mx_lo = fmaxf(mx_lo, s[nt][e]); else mx_hi = fmaxf(mx_hi, s[nt][e]);
        }
    }
#pragma unroll
    for (int o_ = 1; o_ <= 2; o_ <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, o_));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, o_));
    }
    // token blk is inside the cache, so both rows' maxima are finite from the first
    // block on: the first rescale is ex2(-inf) = 0 and masked tokens give ex2(-inf) = 0,
    // with no guards
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float al_lo = ex2_approx(m_lo - mn_lo);
    const float al_hi = ex2_approx(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float p[2][4];
    float ps_lo = 0.f, ps_hi = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[nt][e] = ex2_approx(s[nt][e] - ((e < 2) ? mn_lo : mn_hi));
        if (e < 2) ps_lo += p[nt][e]; else ps_hi += p[nt][e];
      }
    l_lo = l_lo * al_lo + ps_lo;
    l_hi = l_hi * al_hi + ps_hi;
#pragma unroll
    for (int j = 0; j < kAD / 8; ++j) {
      o[j][0] *= al_lo; o[j][1] *= al_lo;
      o[j][2] *= al_hi; o[j][3] *= al_hi;
    }
    // P as the A operand (rows = heads, k = the 16 tokens)
    const uint32_t pa[4] = {pack_bf16x2(p[0][0], p[0][1]), pack_bf16x2(p[0][2], p[0][3]),
                            pack_bf16x2(p[1][0], p[1][1]), pack_bf16x2(p[1][2], p[1][3])};
    __syncwarp();  // V tile stores visible to ldmatrix
#pragma unroll
    for (int jp = 0; jp < kAD / 16; ++jp) {
      const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int col = jp * 16 + (lane >> 4) * 8;
      uint32_t vb4[4];
      ldsm_x4_trans(vb4, vs + row * kAVStride + col);
      mma_bf16_16816(o[2 * jp], pa, vb4[0], vb4[1]);
      mma_bf16_16816(o[2 * jp + 1], pa, vb4[2], vb4[3]);
    }
    __syncwarp();  // done reading the V tile before the next block overwrites it
  }
  // full row sums across the four lanes of each row
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, o_);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, o_);
  }
  // merge the warps (red_o reuses the V tiles: every warp must be done with them)
  __syncthreads();
  if (tid == 0) {
    red_m[warp][gid] = m_lo; red_m[warp][gid + 8] = m_hi;
    red_l[warp][gid] = l_lo; red_l[warp][gid + 8] = l_hi;
  }
#pragma unroll
  for (int j = 0; j < kAD / 8; ++j) {
    if (gid < kG) {
      red_o[warp][gid][8 * j + 2 * tid] = o[j][0];
      red_o[warp][gid][8 * j + 2 * tid + 1] = o[j][1];
    }
    if (gid + 8 < kG) {
      red_o[warp][gid + 8 < kG ? gid + 8 : 0][8 * j + 2 * tid] = o[j][2];
      red_o[warp][gid + 8 < kG ? gid + 8 : 0][8 * j + 2 * tid + 1] = o[j][3];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * kAD; idx += blockDim.x) {
    const int r = idx / kAD, d = idx % kAD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kW; ++w) M = fmaxf(M, red_m[w][r]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kW; ++w) {
        const float f = exp2f(red_m[w][r] - M);
        L += red_l[w][r] * f;
        O += red_o[w][r][d] * f;
      }
    }
    const int64_t hq = static_cast<int64_t>(b) * a.Hq + hq0 + r;
    if constexpr (kCS > 1) {
      float *dst = cg::this_cluster().map_shared_rank(cbuf, 0) + (split * g + r) * (2 + kAD);
      if (d == 0) {
        dst[0] = M;
        dst[1] = L;
      }
      dst[2 + d] = O;
    } else if (a.splits == 1) {
      a.out[hq * kAD + d] = float_to_bf16_bits(L > 0.f ? O / L : 0.f);
    } else {
      float *pw = a.ws + (hq * a.splits + split) * (2 + kAD);
      if (d == 0) {
        pw[0] = M;
        pw[1] = L;
      }
      pw[2 + d] = O;
    }
  }
  if constexpr (kCS > 1) {
    // out = sum_q O_q 2^(m_q - M) / sum_q L_q 2^(m_q - M) over the cluster's ranks
    cg::this_cluster().sync();
    if (split != 0) return;
    for (int idx = threadIdx.x; idx < g * kAD; idx += blockDim.x) {
      const int r = idx / kAD, d = idx % kAD;
      float M = -INFINITY;
#pragma unroll
      for (int q = 0; q < kCS; ++q) M = fmaxf(M, cbuf[(q * g + r) * (2 + kAD)]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int q = 0; q < kCS; ++q) {
          const float *c = cbuf + (q * g + r) * (2 + kAD);
          const float f = exp2f(c[0] - M);
          L += c[1] * f;
          O += c[2 + d] * f;
        }
      }
      a.out[(static_cast<int64_t>(b) * a.Hq + hq0 + r) * kAD + d] = float_to_bf16_bits(L > 0.f ? O / L : 0.f);
    }
  }
}

// Merge the splits of each (sequence, q head): out = sum_s O_s 2^(m_s - M) / sum_s L_s 2^(m_s - M).
// Every load is issued before any is used -- this thread's output column of every
// split into registers, one split's (m, l) per thread into shared memory -- so the
// merge costs one L2 round trip whatever the split count (<= kAMaxSplits). The sums
// run in split order, as before.
template <int kAD>
__global__ void attn_combine_kernel(const float *__restrict__ ws, uint16_t *__restrict__ out, int splits) {
  static_assert(kAD >= kAMaxSplits, "one (m, l) pair per thread");
  __shared__ float sm_m[kAMaxSplits], sm_l[kAMaxSplits];
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int64_t hq = blockIdx.x;
  const int d = threadIdx.x;
  const float *p = ws + hq * splits * (2 + kAD);
  float ov[kAMaxSplits];
#pragma unroll
  for (int s = 0; s < kAMaxSplits; ++s) ov[s] = s < splits ? ld_act_f32(p + s * (2 + kAD) + 2 + d) : 0.f;
  if (d < splits) {
    sm_m[d] = ld_act_f32(p + d * (2 + kAD));
    sm_l[d] = ld_act_f32(p + d * (2 + kAD) + 1);
  }
  __syncthreads();
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, sm_m[s]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
#pragma unroll
    for (int s = 0; s < kAMaxSplits; ++s) {
      if (s < splits) {
        const float f = exp2f(sm_m[s] - M);
        L += sm_l[s] * f;
        O += ov[s] * f;
      }
    }
  }
  out[hq * kAD + d] = float_to_bf16_bits(L > 0.f ? O / L : 0.f);
}

// Split count: enough CTAs for two waves of the SMs and chunks of at most `max_chunk`
// tokens, with chunks of >= kAMinChunk tokens and at most `limit` (<= kAMaxSplits) splits.
__host__ __device__ inline int attn_splits(int B, int Hkv, int Lmax, int sms, int limit = kAMaxSplits,
                                           int max_chunk = kAMaxChunk) {
  int max_splits = (Lmax + kAMinChunk - 1) / kAMinChunk;
  if (max_splits > limit) max_splits = limit;
  if (max_splits < 1) max_splits = 1;
  int s = 1;
  while (s < max_splits && (static_cast<int64_t>(B) * Hkv * s < 2LL * sms || (Lmax + s - 1) / s > max_chunk))
    s *= 2;
  return s < max_splits ? s : max_splits;
}

// ---------------------------------------------------------------------------
// Fixed scratch for iron_attn_decode_noalloc: the split partials of callers that
// cannot allocate device memory. 1 MiB per device (room for the partials of the
// Llama shapes up to 32 K tokens), held by every GPU that loads the library
// until the process exits.
constexpr size_t kAttnScratchBytes = static_cast<size_t>(1) << 20;
static __device__ __align__(256) float g_attn_scratch[kAttnScratchBytes / sizeof(float)];

// Device address of g_attn_scratch on the current device. In host code the
// symbol names a host-side stand-in, not device memory, so the address is looked up
// with the device current (cudaGetSymbolAddress) at the first call on each device and
// cached together with the CUDA context it belongs to: after cudaDeviceReset (or any
// teardown of the device's primary context) the module is loaded again, the current
// context differs, and the address is looked up again instead of reusing a stale one.
typedef int (*CtxGetCurrentFn)(void **);  // cuCtxGetCurrent (CUresult, CUcontext *)
static CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

static float *attn_scratch_address(int *status) {
  static std::mutex mu;
  static float *cache[64] = {nullptr};
  static void *cache_ctx[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_cuda_error(e);
    *status = IRON_ERR_CUDA;
    return nullptr;
  }
  // the context current on this thread; null before the runtime has made the device's
  // primary context current here (the lookup below does that)
  const CtxGetCurrentFn get_ctx = ctx_get_current();
  void *ctx = nullptr;
  if (get_ctx && get_ctx(&ctx) != 0) ctx = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev] || !ctx || cache_ctx[dev] != ctx) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) {
      set_last_cuda_error(e);
      (void)cudaGetLastError();
      *status = IRON_ERR_CUDA;
      return nullptr;
    }
    if (get_ctx && get_ctx(&ctx) != 0) ctx = nullptr;
    cache[dev] = static_cast<float *>(p);
    cache_ctx[dev] = ctx;
  }
  *status = IRON_OK;
  return cache[dev];
}

}  // namespace iron

using namespace iron;

// Cluster form: the splits of a (sequence, kv head) as one cluster of 16 or 8 CTAs
// that merge through distributed shared memory. It serves GQA groups of <= 4 query
// heads (rank 0 holds cluster x 4 rows of partials) when the sequence would be split
// and all clusters fit in one wave of the SMs: the largest such size (B200, batch 1:
// 16 -> 484 us per step, 8 -> 499, no cluster 516; batch 2: 8 -> 522, none 542; batch
// 8, 64 clusters of 8: 42 us slower than independent splits and a combine kernel), as
// long as a CTA's share stays within kAClusterMaxChunk tokens (batch 1 at 32768 tokens:
// 19.1 us with 64 independent splits against 30.4 us in clusters of 16).
static int attn_cluster_size(int B, int Hq, int Hkv, int Lmax) {
  const int sms = sm_count();
  if (Hq / Hkv > 4 || attn_splits(B, Hkv, Lmax, sms) <= 1) return 0;
  for (int cs = 16; cs >= 8; cs /= 2)
    if (static_cast<int64_t>(B) * Hkv * cs <= sms) return (Lmax + cs - 1) / cs <= kAClusterMaxChunk ? cs : 0;
  return 0;
}

static bool attn_use_cluster(int B, int Hq, int Hkv, int Lmax) { return attn_cluster_size(B, Hq, Hkv, Lmax) > 0; }

template <int kAD, bool kFused, int kCS>
static int launch_attn_cluster_cs(AttnArgs a, int B, int Hkv, int Lmax, bool pdl, cudaStream_t s) {
  auto kern = attn_decode_kernel<kAD, kFused, kCS>;
  constexpr size_t kMaxSmem = static_cast<size_t>(kCS) * 4 * (2 + kAD) * sizeof(float);
  static PerDeviceOnce configured;  // per instantiation and device: cluster / shared memory opt-ins
  const int cst = configured.run([&]() {
    cudaError_t e = cudaSuccess;
    if (kCS > 8) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kMaxSmem));
    return call_status(e);
  });
  if (cst != IRON_OK) return cst;
  a.splits = kCS;
  a.chunk = ((Lmax + kCS - 1) / kCS + kABlk - 1) / kABlk * kABlk;  // whole 16-token blocks
  a.ws = nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCS, Hkv, B);
  cfg.blockDim = dim3(32 * attn_cluster_warps<kAD>());
  cfg.dynamicSmemBytes = static_cast<size_t>(kCS) * (a.Hq / a.Hkv) * (2 + kAD) * sizeof(float);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = kCS;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}

template <int kAD, bool kFused>
static int launch_attn_cluster(AttnArgs a, int B, int Hq, int Hkv, int Lmax, bool pdl, cudaStream_t s) {
  return attn_cluster_size(B, Hq, Hkv, Lmax) == 16 ? launch_attn_cluster_cs<kAD, kFused, 16>(a, B, Hkv, Lmax, pdl, s)
                                                   : launch_attn_cluster_cs<kAD, kFused, 8>(a, B, Hkv, Lmax, pdl, s);
}

static size_t attn_ws_bytes(int B, int Hq, int Hkv, int Lmax, int D, int limit = kAMaxSplits) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0) return 0;
  const int s = attn_splits(B, Hkv, Lmax, sm_count(), limit);
  if (s == 1) return 0;
  return static_cast<size_t>(B) * Hq * s * (2 + D) * sizeof(float);
}

extern "C" size_t iron_attn_decode_workspace_bytes(int B, int Hq, int Hkv, int Lmax) {
  return attn_ws_bytes(B, Hq, Hkv, Lmax, 64);
}

extern "C" size_t iron_attn_decode_workspace_bytes_d(int B, int Hq, int Hkv, int Lmax, int D) {
  return (D == 64 || D == 128) ? attn_ws_bytes(B, Hq, Hkv, Lmax, D) : 0;
}

// Argument checks of iron_attn_decode and iron_attn_decode_noalloc (same order, same
// statuses): pointers, shape, head size, GQA grouping, alignment.
static int attn_decode_check(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                             const int32_t *lens, const uint16_t *out, int B, int Hq, int Hkv, int D, int Lmax,
                             int64_t kv_batch_stride, int64_t kv_head_stride) {
  if (!q || !k_cache || !v_cache || !lens || !out) return IRON_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0 || B > 65535 || Hkv > 65535) return IRON_ERR_SHAPE;
  if (D != 64 && D != 128) return IRON_ERR_UNSUPPORTED;
  if (Hq % Hkv || Hq / Hkv > 16) return IRON_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (kv_batch_stride % 8) ||
      (kv_head_stride % 8))
    return IRON_ERR_ALIGN;
  return IRON_OK;
}

// iron_attn_decode with at most `limit` splits per sequence
static int attn_decode_impl(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                            const int32_t *lens, uint16_t *out, int B, int Hq, int Hkv, int D, int Lmax,
                            int64_t kv_batch_stride, int64_t kv_head_stride, float scale, void *workspace,
                            size_t workspace_bytes, unsigned flags, void *stream, int limit) {
  const int chk = attn_decode_check(q, k_cache, v_cache, lens, out, B, Hq, Hkv, D, Lmax, kv_batch_stride,
                                    kv_head_stride);
  if (chk != IRON_OK) return chk;
  AttnArgs a;
  a.q = q;
  a.k = k_cache;
  a.v = v_cache;
  a.lens = lens;
  a.out = out;
  a.bstride = kv_batch_stride;
  a.hstride = kv_head_stride;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.splits = attn_splits(B, Hkv, Lmax, sm_count(), limit);
  a.chunk = ((Lmax + a.splits - 1) / a.splits + kAWarps * kABlk - 1) / (kAWarps * kABlk) * (kAWarps * kABlk);
  a.maxlen = Lmax;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.ws = static_cast<float *>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  if (attn_use_cluster(B, Hq, Hkv, Lmax))
    return D == 64 ? launch_attn_cluster<64, false>(a, B, Hq, Hkv, Lmax, pdl, s)
                   : launch_attn_cluster<128, false>(a, B, Hq, Hkv, Lmax, pdl, s);
  if (a.splits > 1) {
    if (!workspace) return IRON_ERR_NULL;
    if (workspace_bytes < attn_ws_bytes(B, Hq, Hkv, Lmax, D, limit)) return IRON_ERR_WORKSPACE;
  }
  int st = D == 64 ? launch(attn_decode_kernel<64>, dim3(a.splits, Hkv, B), dim3(32 * kAWarps), 0, s, pdl, a)
                   : launch(attn_decode_kernel<128>, dim3(a.splits, Hkv, B), dim3(32 * kAWarps), 0, s, pdl, a);
  if (st != IRON_OK || a.splits == 1) return st;
  return D == 64 ? launch(attn_combine_kernel<64>, dim3(B * Hq), dim3(64), 0, s, pdl,
                          static_cast<const float *>(a.ws), out, a.splits)
                 : launch(attn_combine_kernel<128>, dim3(B * Hq), dim3(128), 0, s, pdl,
                          static_cast<const float *>(a.ws), out, a.splits);
}

extern "C" int iron_attn_decode(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                const int32_t *lens, uint16_t *out, int B, int Hq, int Hkv, int D,
                                int Lmax, int64_t kv_batch_stride, int64_t kv_head_stride,
                                float scale, void *workspace, size_t workspace_bytes,
                                unsigned flags, void *stream) {
  return attn_decode_impl(q, k_cache, v_cache, lens, out, B, Hq, Hkv, D, Lmax, kv_batch_stride, kv_head_stride,
                          scale, workspace, workspace_bytes, flags, stream, kAMaxSplits);
}

// Same computation as iron_attn_decode, for callers that cannot allocate the
// workspace: the split partials go to the library's fixed per-device array (with
// fewer splits where the usual count's partials would not fit it).
extern "C" int iron_attn_decode_noalloc(const uint16_t *q, const uint16_t *k_cache,
                                        const uint16_t *v_cache, const int32_t *lens, uint16_t *out,
                                        int B, int Hq, int Hkv, int D, int Lmax,
                                        int64_t kv_batch_stride, int64_t kv_head_stride, float scale,
                                        unsigned flags, void *stream) {
  const int chk = attn_decode_check(q, k_cache, v_cache, lens, out, B, Hq, Hkv, D, Lmax, kv_batch_stride,
                                    kv_head_stride);
  if (chk != IRON_OK) return chk;
  if (attn_use_cluster(B, Hq, Hkv, Lmax))  // merges in the cluster: no partials
    return iron_attn_decode(q, k_cache, v_cache, lens, out, B, Hq, Hkv, D, Lmax, kv_batch_stride, kv_head_stride,
                            scale, nullptr, 0, flags, stream);
  // the splits that the chunk cap adds come off where their partials would not fit the
  // array (down to the two-wave count, whose partials must fit)
  const int waves = attn_splits(B, Hkv, Lmax, sm_count(), kAMaxSplits, 0x7fffffff);
  int limit = kAMaxSplits;
  while (limit / 2 >= waves && attn_ws_bytes(B, Hq, Hkv, Lmax, D, limit) > kAttnScratchBytes) limit /= 2;
  const size_t need = attn_ws_bytes(B, Hq, Hkv, Lmax, D, limit);
  if (need > kAttnScratchBytes) return IRON_ERR_WORKSPACE;  // beyond the fixed array
  void *ws = nullptr;
  if (need > 0) {
    int st = IRON_OK;
    ws = attn_scratch_address(&st);
    if (st != IRON_OK) return st;
  }
  return attn_decode_impl(q, k_cache, v_cache, lens, out, B, Hq, Hkv, D, Lmax, kv_batch_stride, kv_head_stride,
                          scale, ws, need, flags, stream, limit);
}

// Fused decode attention: q, k, v of the new token from the QKV projection, RoPE at
// pos[b], the new k / v appended to the cache, lens = pos + 1 -- no separate RoPE /
// append launches; the split merge follows as the combine kernel.
extern "C" int iron_attn_decode_qkv(const uint16_t *qkv, const int32_t *pos, const float *lut,
                                    uint16_t *k_cache, uint16_t *v_cache, uint16_t *out, int B, int Hq, int Hkv,
                                    int D, int Lmax, int64_t kv_batch_stride, int64_t kv_head_stride, float scale,
                                    void *workspace, size_t workspace_bytes, unsigned flags, void *stream) {
  if (!qkv || !pos || !lut || !k_cache || !v_cache || !out) return IRON_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0 || B > 65535 || Hkv > 65535) return IRON_ERR_SHAPE;
  if (D != 64 && D != 128) return IRON_ERR_UNSUPPORTED;
  if (Hq % Hkv || Hq / Hkv > 16) return IRON_ERR_SHAPE;
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache) || (kv_batch_stride % 8) ||
      (kv_head_stride % 8))
    return IRON_ERR_ALIGN;
  AttnArgs a = {};
  a.k = k_cache;
  a.v = v_cache;
  a.out = out;
  a.bstride = kv_batch_stride;
  a.hstride = kv_head_stride;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.splits = attn_splits(B, Hkv, Lmax, sm_count());
  a.chunk = ((Lmax + a.splits - 1) / a.splits + kAWarps * kABlk - 1) / (kAWarps * kABlk) * (kAWarps * kABlk);
  a.maxlen = Lmax;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.qkv = qkv;
  a.pos = pos;
  a.lut = lut;
  // the cached rows go to L2 ahead of the loop while the whole K / V working set fits in
  // half of L2 (B200: batch 1 and 8 gain 28 / 16 us per step; batch 64 -- 300 MB per
  // layer -- loses 88 us to the thrash)
  a.l2_prefetch = static_cast<int64_t>(B) * Hkv * Lmax * D * 4 <= (64LL << 20) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  if (attn_use_cluster(B, Hq, Hkv, Lmax))
    return D == 64 ? launch_attn_cluster<64, true>(a, B, Hq, Hkv, Lmax, pdl, s)
                   : launch_attn_cluster<128, true>(a, B, Hq, Hkv, Lmax, pdl, s);
  if (a.splits > 1) {
    if (!workspace) return IRON_ERR_NULL;
    if (workspace_bytes < attn_ws_bytes(B, Hq, Hkv, Lmax, D)) return IRON_ERR_WORKSPACE;
    a.ws = static_cast<float *>(workspace);
  }
  // the splits merge in the combine kernel, which PDL overlaps with this one's tail
  // (measured faster on B200 than merging in the last split CTA)
  int st = D == 64 ? launch(attn_decode_kernel<64, true>, dim3(a.splits, Hkv, B), dim3(32 * kAWarps), 0, s, pdl, a)
                   : launch(attn_decode_kernel<128, true>, dim3(a.splits, Hkv, B), dim3(32 * kAWarps), 0, s, pdl, a);
  if (st != IRON_OK || a.splits == 1) return st;
  return D == 64 ? launch(attn_combine_kernel<64>, dim3(B * Hq), dim3(64), 0, s, pdl, static_cast<const float *>(a.ws),
                          out, a.splits)
                 : launch(attn_combine_kernel<128>, dim3(B * Hq), dim3(128), 0, s, pdl,
                          static_cast<const float *>(a.ws), out, a.splits);
}

extern "C" int iron_attn_decode_kernels(int B, int Hq, int Hkv, int Lmax) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0 || Hq % Hkv) return 0;
  if (attn_use_cluster(B, Hq, Hkv, Lmax)) return 1;
  return attn_splits(B, Hkv, Lmax, sm_count()) > 1 ? 2 : 1;
}

extern "C" size_t iron_attn_decode_qkv_workspace_bytes(int B, int Hq, int Hkv, int Lmax, int D) {
  return (D == 64 || D == 128) ? attn_ws_bytes(B, Hq, Hkv, Lmax, D) : 0;
}
