// Causal GQA attention for prefill (flash-attention style, one pass over K/V).
//
// Replaces IRON's MHA operator (iron/operators/mha/op.py:21-135; golden
// mha/reference.py:27-94: SDPA with is_causal, scale 1/sqrt(d), K/V heads shared
// by heads/kv_heads query heads) and the CPU attention of IRON's Llama prefill
// (iron/applications/llama_3.2_1b/llama_npu.py:854-992).
//
// One CTA = 64 query rows of one (sequence, query head); its four warps own 16
// rows each. K and V blocks of 64 keys are staged in shared memory (double
// buffered, the next block prefetched into registers while the current one
// computes); S = Q K^T uses m16n8k16 bf16 MMAs with K fragments from ldmatrix,
// the online softmax runs in fp32 in exp2 space, O += P V takes P from the S
// accumulators and V through ldmatrix.trans. Only blocks on or below the
// diagonal are visited. Rows at or past the valid length are written as zeros
// (IRON's padded output rows).
#include "common.cuh"

namespace iron {

namespace {
constexpr int kPD = 64;       // head dim
constexpr int kPBlk = 64;     // queries per CTA and keys per block
constexpr int kPStride = 72;  // padded smem row (elements): conflict-free ldmatrix
constexpr int kPThreads = 128;

struct PrefillArgs {
  const uint16_t *q, *k, *v;
  uint16_t *out;
  int64_t qb, qh, qs;  // element strides of q / out: batch, head, token
  int64_t ob, oh, os;
  int64_t kb, kh, ks;  // element strides of k and v
  int H, Hkv, S, S_kv, q_blocks;
  int causal;
  float scale_log2;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
}  // namespace

__global__ void __launch_bounds__(kPThreads) attn_prefill_kernel(PrefillArgs a) {
  __shared__ __align__(16) uint16_t ks_[2][kPBlk * kPStride];
  __shared__ __align__(16) uint16_t vs_[2][kPBlk * kPStride];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid = lane & 3;
  // heavy (late) query blocks first
  const int qt = a.q_blocks - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hkv);
  const int q0 = qt * kPBlk + warp * 16;

  pdl_wait();
  const uint16_t *qp = a.q + b * a.qb + h * a.qh;
  const uint16_t *kp = a.k + b * a.kb + hk * a.kh;
  const uint16_t *vp = a.v + b * a.kb + hk * a.kh;

  // Q fragments of the warp's 16 rows (rows past S read as zero)
  uint32_t qa[4][4];
  {
    const int r0 = q0 + gid, r1 = r0 + 8;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int d = kk * 16 + 2 * tid;
      const uint32_t *p0 = reinterpret_cast<const uint32_t *>(qp + r0 * a.qs + d);
      const uint32_t *p1 = reinterpret_cast<const uint32_t *>(qp + r1 * a.qs + d);
      qa[kk][0] = r0 < a.S ? ld_act_u32(p0) : 0u;
      qa[kk][1] = r1 < a.S ? ld_act_u32(p1) : 0u;
      qa[kk][2] = r0 < a.S ? ld_act_u32(p0 + 4) : 0u;
      qa[kk][3] = r1 < a.S ? ld_act_u32(p1 + 4) : 0u;
    }
  }

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

  const int q_last = min(qt * kPBlk + kPBlk, a.S) - 1;  // last valid query row of the CTA
  const int kv_end = a.causal ? min(a.S_kv, q_last + 1) : a.S_kv;
  const int nblk = q_last < qt * kPBlk ? 0 : (kv_end + kPBlk - 1) / kPBlk;

  // each thread moves 4 x 16 B of K and 4 x 16 B of V per block
  uint4 kr[4], vr[4];
  auto fetch = [&](int blk) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = i * kPThreads + threadIdx.x, row = idx >> 3, c = (idx & 7) * 8;
      const int t = blk * kPBlk + row;
      const bool in = t < a.S_kv;
      kr[i] = in ? ld_act_v4(kp + t * a.ks + c) : make_uint4(0, 0, 0, 0);
      vr[i] = in ? ld_act_v4(vp + t * a.ks + c) : make_uint4(0, 0, 0, 0);
    }
  };
  if (nblk > 0) fetch(0);

  for (int blk = 0; blk < nblk; ++blk) {
    const int buf = blk & 1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = i * kPThreads + threadIdx.x, row = idx >> 3, c = (idx & 7) * 8;
      *reinterpret_cast<uint4 *>(&ks_[buf][row * kPStride + c]) = kr[i];
      *reinterpret_cast<uint4 *>(&vs_[buf][row * kPStride + c]) = vr[i];
    }
    __syncthreads();
    if (blk + 1 < nblk) fetch(blk + 1);

    // S = Q K^T: 8 key n-tiles of 8
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t kb4[4];
        ldsm_x4(kb4, &ks_[buf][(nt * 8 + (lane & 7)) * kPStride + half * 32 + (lane >> 3) * 8]);
        mma_bf16_16816(s[nt], qa[2 * half], kb4[0], kb4[1]);
        mma_bf16_16816(s[nt], qa[2 * half + 1], kb4[2], kb4[3]);
      }
    }
    // running max of the raw scores (the scale is positive: max(s) * c = max(s * c));
    // blocks wholly inside the valid, causal region skip the mask
    const int key0 = blk * kPBlk;
    const float c = a.scale_log2;
    const bool full = key0 + kPBlk <= a.S_kv && (!a.causal || key0 + kPBlk - 1 <= q0);
    if (!full) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + nt * 8 + 2 * tid + (e & 1);
          const int row = q0 + gid + ((e >> 1) << 3);
          if (!(key < a.S_kv && (!a.causal || key <= row))) s[nt][e] = -INFINITY;
        }
    }
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx_lo = fmaxf(mx_lo, fmaxf(s[nt][0], s[nt][1]));
      mx_hi = fmaxf(mx_hi, fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, x));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, x));
    }
    const float mn_lo = fmaxf(m_lo, mx_lo * c), mn_hi = fmaxf(m_hi, mx_hi * c);
    const float al_lo = mn_lo == -INFINITY ? 1.f : exp2f(m_lo - mn_lo);
    const float al_hi = mn_hi == -INFINITY ? 1.f : exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    // p = 2^(s c - m), one rounding (a fully masked row of a partial block: 0)
    float ps_lo = 0.f, ps_hi = 0.f;
    if (full) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[nt][e] = ex2_approx(fmaf(s[nt][e], c, -(e < 2 ? mn_lo : mn_hi)));
          if (e < 2) ps_lo += s[nt][e];
          else ps_hi += s[nt][e];
        }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mr = e < 2 ? mn_lo : mn_hi;
          s[nt][e] = mr == -INFINITY ? 0.f : ex2_approx(fmaf(s[nt][e], c, -mr));
          if (e < 2) ps_lo += s[nt][e];
          else ps_hi += s[nt][e];
        }
    }
    l_lo = l_lo * al_lo + ps_lo;
    l_hi = l_hi * al_hi + ps_hi;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= al_lo;
      o[j][1] *= al_lo;
      o[j][2] *= al_hi;
      o[j][3] *= al_hi;
    }
    // O += P V over the block's four 16-key steps
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pack_bf16x2(s[2 * kk][0], s[2 * kk][1]), pack_bf16x2(s[2 * kk][2], s[2 * kk][3]),
                              pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                              pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t vb4[4];
        const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm_x4_t(vb4, &vs_[buf][row * kPStride + jp * 16 + (lane >> 4) * 8]);
        mma_bf16_16816(o[2 * jp], pa, vb4[0], vb4[1]);
        mma_bf16_16816(o[2 * jp + 1], pa, vb4[2], vb4[3]);
      }
    }
  }
  pdl_launch_dependents();
#pragma unroll
  for (int x = 1; x <= 2; x <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, x);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, x);
  }
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  const int r0 = q0 + gid, r1 = r0 + 8;
  uint16_t *op = a.out + b * a.ob + h * a.oh;
  const bool v0 = r0 < a.S, v1 = r1 < a.S;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int d = j * 8 + 2 * tid;
    *reinterpret_cast<uint32_t *>(op + r0 * a.os + d) = v0 ? pack_bf16x2(o[j][0] * inv_lo, o[j][1] * inv_lo) : 0u;
    *reinterpret_cast<uint32_t *>(op + r1 * a.os + d) = v1 ? pack_bf16x2(o[j][2] * inv_hi, o[j][3] * inv_hi) : 0u;
  }
}

}  // namespace iron

using namespace iron;

extern "C" int iron_attn_prefill(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out, int B,
                                 int H, int Hkv, int D, int S, int S_pad, int S_kv, const int64_t *q_strides,
                                 const int64_t *kv_strides, const int64_t *out_strides, float scale, int causal,
                                 unsigned flags, void *stream) {
  if (!q || !k || !v || !out || !q_strides || !kv_strides || !out_strides) return IRON_ERR_NULL;
  if (B <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || S_kv <= 0 || S_pad < S) return IRON_ERR_SHAPE;
  if (D != kPD || H % Hkv) return IRON_ERR_UNSUPPORTED;
  if (S_pad % kPBlk) return IRON_ERR_SHAPE;
  for (int i = 0; i < 3; ++i)
    if (q_strides[i] % 8 || kv_strides[i] % 8 || out_strides[i] % 8) return IRON_ERR_ALIGN;
  if (q_strides[2] < D || kv_strides[2] < D || out_strides[2] < D) return IRON_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return IRON_ERR_ALIGN;
  PrefillArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.qb = q_strides[0];
  a.qh = q_strides[1];
  a.qs = q_strides[2];
  a.kb = kv_strides[0];
  a.kh = kv_strides[1];
  a.ks = kv_strides[2];
  a.ob = out_strides[0];
  a.oh = out_strides[1];
  a.os = out_strides[2];
  a.H = H;
  a.Hkv = Hkv;
  a.S = S;
  a.S_kv = S_kv;
  a.q_blocks = S_pad / kPBlk;
  a.causal = causal;
  a.scale_log2 = scale * 1.4426950408889634f;
  return launch(attn_prefill_kernel, dim3(a.q_blocks, H, B), dim3(kPThreads), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, a);
}
