// Decode-step glue kernels of the Llama pipeline: fused RoPE + KV-cache append,
// token embedding gather and greedy argmax.
//
// rope_kv_append replaces, per decode step, IRON's RoPE on queries and keys and
// the two StridedCopy KV-cache writes with the runtime cache_offset
// (iron/applications/llama_3.2_1b/llama_npu.py:481-495, :1161-1169): one kernel
// reads the fused QKV projection, rotates q and k (two-halves RoPE,
// iron/applications/llama_3.2_1b/llama_cpu.py:17-38) from an fp32 cos/sin table at
// each sequence's own position, writes k and v into cache slot pos[b] and sets
// lens[b] = pos[b] + 1 for the attention that follows.
#include "common.cuh"

namespace iron {

__global__ void rope_kv_append_kernel(const uint16_t *__restrict__ qkv, const int *__restrict__ pos,
                                      const float *__restrict__ lut, uint16_t *__restrict__ q_out,
                                      uint16_t *__restrict__ k_cache, uint16_t *__restrict__ v_cache,
                                      int *__restrict__ lens, int Hq, int Hkv, int D,
                                      int64_t kv_bstride, int64_t kv_hstride) {
  pdl_wait();
  pdl_launch_dependents();  // after the wait: bounds a window (the attention reads the new rows as cache rows)
  const int b = blockIdx.x;
  const int p = ld_act_i32(pos + b);
  const int half = D / 2;
  const int rows = Hq + 2 * Hkv;  // q heads, k heads, v heads
  const uint16_t *src = qkv + static_cast<int64_t>(b) * rows * D;
  const float *ang = lut + static_cast<int64_t>(p) * D;
  for (int i = threadIdx.x; i < rows * half; i += blockDim.x) {
    const int r = i / half, j = i % half;
    const uint16_t *x = src + r * D;
    if (r < Hq + Hkv) {
      const float c = ang[2 * j], sn = ang[2 * j + 1];
      const float x1 = bf16_bits_to_float(ld_act_u16(x + j)), x2 = bf16_bits_to_float(ld_act_u16(x + j + half));
      const uint16_t y1 = float_to_bf16_bits(x1 * c - x2 * sn);
      const uint16_t y2 = float_to_bf16_bits(x1 * sn + x2 * c);
      if (r < Hq) {
        uint16_t *qo = q_out + (static_cast<int64_t>(b) * Hq + r) * D;
        qo[j] = y1;
        qo[j + half] = y2;
      } else {
        uint16_t *kc = k_cache + b * kv_bstride + (r - Hq) * kv_hstride + static_cast<int64_t>(p) * D;
        kc[j] = y1;
        kc[j + half] = y2;
      }
    } else {
      uint16_t *vc = v_cache + b * kv_bstride + (r - Hq - Hkv) * kv_hstride + static_cast<int64_t>(p) * D;
      vc[j] = ld_act_u16(x + j);
      vc[j + half] = ld_act_u16(x + j + half);
    }
  }
  if (threadIdx.x == 0 && lens) lens[b] = p + 1;
}

// A token outside [0, V) (-1 is what iron_argmax_finalize gives when no logit was
// written) reads nothing: its row becomes zeros.
__global__ void embed_kernel(const int *__restrict__ tokens, const uint4 *__restrict__ table,
                             uint4 *__restrict__ x, int row_vecs, int V) {
  // The first kernel of a decode step: it lets the step's kernels launch only after the
  // previous step finished (its token / position update), because some of them read the
  // positions before their own wait.
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int64_t t = ld_act_i32(tokens + b);
  const bool ok = t >= 0 && t < V;
  for (int i = threadIdx.x; i < row_vecs; i += blockDim.x)
    x[static_cast<int64_t>(b) * row_vecs + i] = ok ? table[t * row_vecs + i] : make_uint4(0u, 0u, 0u, 0u);
}

// The embedding gather plus the first layer's chained RMSNorm input: xw = bf16(x * w)
// and per 16 elements the sum of squares of x (two threads' 8 elements each, summed
// through one shuffle: a fixed order).
__global__ void embed_chain_kernel(const int *__restrict__ tokens, const uint4 *__restrict__ table,
                                   uint4 *__restrict__ x, uint4 *__restrict__ xw, const uint4 *__restrict__ w,
                                   float *__restrict__ ss, int row_vecs, int V) {
  pdl_wait();  // as embed_kernel: the step's first kernel waits for the previous step
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int64_t t = ld_act_i32(tokens + b);
  const bool ok = t >= 0 && t < V;
  for (int i0 = 0; i0 < row_vecs; i0 += blockDim.x) {  // uniform trip count (the shuffle)
    const int i = i0 + threadIdx.x;
    float q = 0.f;
    if (i < row_vecs) {
      const uint4 r = ok ? table[t * row_vecs + i] : make_uint4(0u, 0u, 0u, 0u);
      const uint4 wv = __ldg(w + i);
      x[static_cast<int64_t>(b) * row_vecs + i] = r;
      const uint32_t a[4] = {r.x, r.y, r.z, r.w}, c[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float lo = bf16_lo(a[k]), hi = bf16_hi(a[k]);
        q += lo * lo + hi * hi;
        o[k] = pack_bf16x2(lo * bf16_lo(c[k]), hi * bf16_hi(c[k]));
      }
      xw[static_cast<int64_t>(b) * row_vecs + i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    q += __shfl_xor_sync(0xffffffffu, q, 1);
    if (i < row_vecs && (i & 1) == 0) ss[static_cast<int64_t>(b) * (row_vecs / 2) + i / 2] = q;
  }
}

// First index of the maximum of each row (NaN never wins).
__global__ void argmax_kernel(const uint16_t *__restrict__ logits, int *__restrict__ out, int V,
                              int *__restrict__ pos) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int64_t b = blockIdx.x;
  const uint16_t *row = logits + b * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = bf16_bits_to_float(ld_act_u16(row + i));
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out[b] = bi == 0x7fffffff ? 0 : bi;
      if (pos) pos[b] += 1;  // the next decode step writes the next cache slot
    }
  }
}

}  // namespace iron

using namespace iron;

extern "C" int iron_rope_kv_append(const uint16_t *qkv, const int32_t *pos, const float *lut,
                                   uint16_t *q_out, uint16_t *k_cache, uint16_t *v_cache,
                                   int32_t *lens, int B, int Hq, int Hkv, int D,
                                   int64_t kv_batch_stride, int64_t kv_head_stride, unsigned flags,
                                   void *stream) {
  if (!qkv || !pos || !lut || !q_out || !k_cache || !v_cache) return IRON_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 2) return IRON_ERR_SHAPE;
  return launch(rope_kv_append_kernel, dim3(B), dim3(256), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, qkv, pos, lut, q_out, k_cache, v_cache, lens, Hq, Hkv,
                D, kv_batch_stride, kv_head_stride);
}

extern "C" int iron_embed(const int32_t *tokens, const uint16_t *table, uint16_t *x, int B, int E, int V,
                          unsigned flags, void *stream) {
  if (!tokens || !table || !x) return IRON_ERR_NULL;
  if (B <= 0 || E <= 0 || V <= 0) return IRON_ERR_SHAPE;
  if (E % 8 || !aligned16(table) || !aligned16(x)) return IRON_ERR_ALIGN;
  return launch(embed_kernel, dim3(B), dim3(256), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, tokens, reinterpret_cast<const uint4 *>(table),
                reinterpret_cast<uint4 *>(x), E / 8, V);
}

extern "C" int iron_embed_chain(const int32_t *tokens, const uint16_t *table, uint16_t *x, uint16_t *xw,
                                const uint16_t *weight, float *ss, int B, int E, int V, unsigned flags,
                                void *stream) {
  if (!tokens || !table || !x || !xw || !weight || !ss) return IRON_ERR_NULL;
  if (B <= 0 || E <= 0 || V <= 0 || B > 65535) return IRON_ERR_SHAPE;
  if (E % 16) return IRON_ERR_SHAPE;
  if (!aligned16(table) || !aligned16(x) || !aligned16(xw) || !aligned16(weight)) return IRON_ERR_ALIGN;
  return launch(embed_chain_kernel, dim3(B), dim3(256), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, tokens, reinterpret_cast<const uint4 *>(table),
                reinterpret_cast<uint4 *>(x), reinterpret_cast<uint4 *>(xw), reinterpret_cast<const uint4 *>(weight),
                ss, E / 8, V);
}

extern "C" int iron_argmax(const uint16_t *logits, int32_t *out, int B, int V, int32_t *pos,
                           unsigned flags, void *stream) {
  if (!logits || !out) return IRON_ERR_NULL;
  if (B <= 0 || V <= 0) return IRON_ERR_SHAPE;
  return launch(argmax_kernel, dim3(B), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, logits, out, V, pos);
}
