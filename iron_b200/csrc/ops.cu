// Row-wise and element-wise operators of the decode path: RMSNorm, RoPE, masked
// softmax, SiLU / multiply / add / SwiGLU activation, IRON's StridedCopy (the
// KV-cache append), repeat-interleave and batched transpose.
//
// All are HBM- or latency-bound. Rows are processed by one CTA (or one warp for
// short rows) with 16-byte vector loads where the row length allows, statistics
// in fp32, one bf16 rounding per output. Runtime parameters that a captured CUDA
// graph must be able to change (softmax valid length, copy offsets) can be read
// from device memory.
#include "common.cuh"

namespace iron {

// ---------------------------------------------------------------------------
// Block reduction helper (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < nw ? scratch[lane] : 0.f;
  return warp_sum(r);
}
__device__ __forceinline__ float block_max(float v, float *scratch) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < nw ? scratch[lane] : -INFINITY;
  return warp_max(r);
}

__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
  f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x); f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
  f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z); f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// ---------------------------------------------------------------------------
// RMSNorm: y = x / sqrt(mean(x^2) + eps) [* w]   (iron/operators/rms_norm/reference.py:7-16)
// One CTA per row; optional residual input r: x := x + r first, written back to
// `x_out` (the decode block's "h = x + attn" fused with the second norm).
__global__ void rmsnorm_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ r,
                               uint16_t *__restrict__ x_out, const uint16_t *__restrict__ w,
                               uint16_t *__restrict__ y, int cols, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const uint16_t *xr = x + row * cols;
  const uint16_t *rr = r ? r + row * cols : nullptr;
  uint16_t *yr = y + row * cols;
  uint16_t *xo = x_out ? x_out + row * cols : nullptr;
  const int stride = blockDim.x * 8;
  // vector path: each thread keeps up to 4 chunks of 8 in registers (cols <= 8192 at 256 thr)
  const bool vec = (cols & 7) == 0 && cols <= 4 * stride;
  // the weights never depend on the previous kernel: requested before waiting for it
  uint4 wv[4];
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int c = threadIdx.x * 8 + n * stride;
    wv[n] = (vec && w && c < cols) ? *reinterpret_cast<const uint4 *>(w + c) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_launch_dependents();  // at entry: the next kernel may start its weight loads
  pdl_wait();
  float ss = 0.f;
  if (vec) {
    float v[4][8];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int c = threadIdx.x * 8 + n * stride;
      if (c < cols) {
        unpack8(ld_act_v4(xr + c), v[n]);
        if (rr) {
          float q[8];
          unpack8(ld_act_v4(rr + c), q);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[n][i] = __bfloat162float(__float2bfloat16_rn(v[n][i] + q[i]));
          if (xo) *reinterpret_cast<uint4 *>(xo + c) = pack8(v[n]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[n][i] * v[n][i];
      }
    }
    const float inv = rsqrtf(block_sum(ss, scratch) / cols + eps);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int c = threadIdx.x * 8 + n * stride;
      if (c < cols) {
        float o[8];
        if (w) {
          float ww[8];
          unpack8(wv[n], ww);
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = v[n][i] * inv * ww[i];
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = v[n][i] * inv;
        }
        *reinterpret_cast<uint4 *>(yr + c) = pack8(o);
      }
    }
    return;
  }
  // scalar path: odd widths, or rows longer than the register cache
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float a = bf16_bits_to_float(ld_act_u16(xr + c));
    if (rr) {
      a = __bfloat162float(__float2bfloat16_rn(a + bf16_bits_to_float(ld_act_u16(rr + c))));
      if (xo) xo[c] = float_to_bf16_bits(a);
    }
    ss += a * a;
  }
  const float inv = rsqrtf(block_sum(ss, scratch) / cols + eps);
  __syncthreads();  // x_out writes visible before re-reading them
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float a = rr ? bf16_bits_to_float(xo ? xo[c]
                                         : float_to_bf16_bits(bf16_bits_to_float(ld_act_u16(xr + c)) +
                                                              bf16_bits_to_float(ld_act_u16(rr + c))))
                 : bf16_bits_to_float(ld_act_u16(xr + c));
    float o = a * inv;
    if (w) o *= bf16_bits_to_float(w[c]);
    yr[c] = float_to_bf16_bits(o);
  }
}

// ---------------------------------------------------------------------------
// RoPE (iron/operators/rope/reference.py:69-102): angles row a holds interleaved
// [cos, sin, cos, sin, ...]; row r of x uses angle row r / (rows / angle_rows).
// method 0: two halves; 1: interleaved pairs. fp32, one rounding.
// With `pos` != NULL the angle row of x row r is pos[r / rows_per_pos] (a LUT
// indexed by each sequence's position: the batched decode form).
__global__ void rope_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ angles,
                            const float *__restrict__ angles_f32, uint16_t *__restrict__ y,
                            int rows, int cols, int rows_per_angle, const int *__restrict__ pos,
                            int method) {
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int half = cols / 2;
  const int64_t total = static_cast<int64_t>(rows) * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / half), j = static_cast<int>(i % half);
    int arow = r / rows_per_angle;
    if (pos) arow = ld_act_i32(pos + arow);
    float c, s;
    if (angles_f32) {
      c = angles_f32[static_cast<int64_t>(arow) * cols + 2 * j];
      s = angles_f32[static_cast<int64_t>(arow) * cols + 2 * j + 1];
    } else {
      c = bf16_bits_to_float(angles[static_cast<int64_t>(arow) * cols + 2 * j]);
      s = bf16_bits_to_float(angles[static_cast<int64_t>(arow) * cols + 2 * j + 1]);
    }
    const uint16_t *xr = x + static_cast<int64_t>(r) * cols;
    uint16_t *yr = y + static_cast<int64_t>(r) * cols;
    if (method == 0) {
      const float x1 = bf16_bits_to_float(ld_act_u16(xr + j)), x2 = bf16_bits_to_float(ld_act_u16(xr + j + half));
      yr[j] = float_to_bf16_bits(x1 * c - x2 * s);
      yr[j + half] = float_to_bf16_bits(x2 * c + x1 * s);
    } else {
      const float xe = bf16_bits_to_float(ld_act_u16(xr + 2 * j)), xo = bf16_bits_to_float(ld_act_u16(xr + 2 * j + 1));
      yr[2 * j] = float_to_bf16_bits(xe * c - xo * s);
      yr[2 * j + 1] = float_to_bf16_bits(xe * s + xo * c);
    }
  }
}

// ---------------------------------------------------------------------------
// Softmax over each row's first `valid` columns (iron/operators/softmax/reference.py:9-11
// with the device mask of iron/operators/softmax/design.py:85-91); masked columns
// are 0. `valid_dev` (if set) overrides `valid` at run time.
__global__ void softmax_kernel(const uint16_t *__restrict__ x, uint16_t *__restrict__ y, int cols,
                               int valid, const int *__restrict__ valid_dev) {
  __shared__ float scratch[32];
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  if (valid_dev) valid = ld_act_i32(valid_dev);
  valid = max(0, min(valid, cols));
  const int64_t row = blockIdx.x;
  const uint16_t *xr = x + row * cols;
  uint16_t *yr = y + row * cols;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < valid; c += blockDim.x) m = fmaxf(m, bf16_bits_to_float(ld_act_u16(xr + c)));
  m = block_max(m, scratch);
  float s = 0.f;
  for (int c = threadIdx.x; c < valid; c += blockDim.x) s += __expf(bf16_bits_to_float(ld_act_u16(xr + c)) - m);
  s = block_sum(s, scratch);
  const float inv = 1.f / s;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    yr[c] = float_to_bf16_bits(c < valid ? __expf(bf16_bits_to_float(ld_act_u16(xr + c)) - m) * inv : 0.f);
}

// ---------------------------------------------------------------------------
// Element-wise (iron/operators/{silu,elementwise_mul,elementwise_add}/reference.py):
// op 0: silu(a); 1: a * b; 2: a + b; 3: silu(a) * b (SwiGLU's SiLU + Mul fused).
__device__ __forceinline__ float silu_f(float v) { return v / (1.f + __expf(-v)); }

__global__ void eltwise_kernel(const uint16_t *__restrict__ a, const uint16_t *__restrict__ b,
                               uint16_t *__restrict__ y, int64_t n, int op) {
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int64_t n8 = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    float fa[8], fb[8] = {0, 0, 0, 0, 0, 0, 0, 0}, o[8];
    unpack8(ld_act_v4(a + 8 * i), fa);
    if (op != 0) unpack8(ld_act_v4(b + 8 * i), fb);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      o[k] = op == 0 ? silu_f(fa[k]) : op == 1 ? fa[k] * fb[k] : op == 2 ? fa[k] + fb[k]
                                                                        : silu_f(fa[k]) * fb[k];
    reinterpret_cast<uint4 *>(y)[i] = pack8(o);
  }
  for (int64_t i = n8 * 8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const float fa = bf16_bits_to_float(ld_act_u16(a + i));
    const float fb = op != 0 ? bf16_bits_to_float(ld_act_u16(b + i)) : 0.f;
    const float o = op == 0 ? silu_f(fa) : op == 1 ? fa * fb : op == 2 ? fa + fb : silu_f(fa) * fb;
    y[i] = float_to_bf16_bits(o);
  }
}

// ---------------------------------------------------------------------------
// StridedCopy (iron/operators/strided_copy/reference.py:37-75): access patterns are
// padded to 4-D; the innermost dimension is split into `channels` equal parts and
// element j of channel c moves from the input pattern to the output pattern.
struct Tap4 {
  int64_t size[4], stride[4];
  int64_t offset;
};

__device__ __forceinline__ int64_t tap_offset(const Tap4 &t, int64_t split3, int c, int64_t j) {
  // j is the row-major index within (size0, size1, size2, split3)
  const int64_t i3 = j % split3;
  int64_t q = j / split3;
  const int64_t i2 = q % t.size[2];
  q /= t.size[2];
  const int64_t i1 = q % t.size[1];
  const int64_t i0 = q / t.size[1];
  return t.offset + static_cast<int64_t>(c) * split3 * t.stride[3] + i0 * t.stride[0] +
         i1 * t.stride[1] + i2 * t.stride[2] + i3 * t.stride[3];
}

template <typename T>
__global__ void strided_copy_kernel(const T *__restrict__ in, T *__restrict__ out, Tap4 src, Tap4 dst,
                                    int channels, int64_t src_split3, int64_t dst_split3,
                                    int64_t per_channel, const int *__restrict__ in_add,
                                    const int *__restrict__ out_add, int64_t in_size,
                                    int64_t out_size) {
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int64_t ia = in_add ? ld_act_i32(in_add) : 0, oa = out_add ? ld_act_i32(out_add) : 0;
  const int64_t total = per_channel * channels;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i / per_channel);
    const int64_t j = i - c * per_channel;
    const int64_t so = tap_offset(src, src_split3, c, j) + ia;
    const int64_t d = tap_offset(dst, dst_split3, c, j) + oa;
    if (so >= 0 && so < in_size && d >= 0 && d < out_size) out[d] = ld_act(in + so);
  }
}

// ---------------------------------------------------------------------------
// repeat_interleave along dim 0 (iron/operators/repeat/reference.py:7-9), 16-byte vectors.
__global__ void repeat_kernel(const uint4 *__restrict__ in, uint4 *__restrict__ out, int64_t rows,
                              int64_t row_vecs, int repeat) {
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int64_t total = rows * repeat * row_vecs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t orow = i / row_vecs, v = i - orow * row_vecs;
    out[i] = ld_act(in + (orow / repeat) * row_vecs + v);
  }
}

// Batched transpose (iron/operators/transpose/reference.py:7-10) through a 32x33 tile.
template <typename T>
__global__ void transpose_kernel(const T *__restrict__ in, T *__restrict__ out, int M, int N) {
  __shared__ T tile[32][33];
  pdl_launch_dependents();  // at entry: the next kernel may start its weight / cache loads
  pdl_wait();
  const int64_t b = blockIdx.z;
  const T *src = in + b * static_cast<int64_t>(M) * N;
  T *dst = out + b * static_cast<int64_t>(M) * N;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < M && c < N) tile[i][threadIdx.x] = ld_act(src + static_cast<int64_t>(r) * N + c);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;  // out row c, col r
    if (r < M && c < N) dst[static_cast<int64_t>(c) * M + r] = tile[threadIdx.x][i];
  }
}

// The same RMSNorm with one warp per row (cols % 256 == 0, cols <= 2048: each lane keeps
// its cols / 256 chunks of 8 in registers, the sum of squares reduced by shuffles). The
// CTA-per-row kernel pays a block-wide barrier per row (B200: the 2048-token prefill
// 6.59 -> 6.44 ms with this form for its 33 norms).
constexpr int kNormWarpChunks = 8;
__global__ void __launch_bounds__(256) rmsnorm_warp_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ r,
                                                           uint16_t *__restrict__ x_out, const uint16_t *__restrict__ w,
                                                           uint16_t *__restrict__ y, int rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int nch = cols >> 8;
  // the weights never depend on the previous kernel: requested before waiting for it
  uint4 wv[kNormWarpChunks];
#pragma unroll
  for (int n = 0; n < kNormWarpChunks; ++n)
    wv[n] = (w && n < nch) ? *reinterpret_cast<const uint4 *>(w + n * 256 + lane * 8) : make_uint4(0u, 0u, 0u, 0u);
  pdl_launch_dependents();
  pdl_wait();
  if (row >= rows) return;
  const uint16_t *xr = x + row * cols;
  const uint16_t *rr = r ? r + row * cols : nullptr;
  uint16_t *xo = x_out ? x_out + row * cols : nullptr;
  uint16_t *yr = y + row * cols;
  float v[kNormWarpChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int n = 0; n < kNormWarpChunks; ++n) {
    if (n < nch) {
      const int c = n * 256 + lane * 8;
      unpack8(ld_act_v4(xr + c), v[n]);
      if (rr) {
        float q[8];
        unpack8(ld_act_v4(rr + c), q);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[n][i] = __bfloat162float(__float2bfloat16_rn(v[n][i] + q[i]));
        if (xo) *reinterpret_cast<uint4 *>(xo + c) = pack8(v[n]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[n][i] * v[n][i];
    }
  }
  const float inv = rsqrtf(warp_sum(ss) / cols + eps);
#pragma unroll
  for (int n = 0; n < kNormWarpChunks; ++n) {
    if (n < nch) {
      float o[8];
      if (w) {
        float ww[8];
        unpack8(wv[n], ww);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[n][i] * inv * ww[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[n][i] * inv;
      }
      *reinterpret_cast<uint4 *>(yr + n * 256 + lane * 8) = pack8(o);
    }
  }
}

static unsigned grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<unsigned>(g);
}

}  // namespace iron

using namespace iron;

extern "C" int iron_rmsnorm(const uint16_t *x, const uint16_t *residual, uint16_t *x_out,
                            const uint16_t *weight, uint16_t *y, int rows, int cols, float eps,
                            unsigned flags, void *stream) {
  if (!x || !y) return IRON_ERR_NULL;
  if (rows <= 0 || cols <= 0 || rows > 0x7fffffff) return IRON_ERR_SHAPE;
  if ((cols & 7) == 0 && (!aligned16(x) || !aligned16(y) || (weight && !aligned16(weight)) ||
                          (residual && !aligned16(residual)) || (x_out && !aligned16(x_out))))
    return IRON_ERR_ALIGN;
  // one warp per row for many rows (a prefill's tokens); a decode batch's few rows keep a
  // CTA each, spread over more SMs
  if (rows >= 256 && cols % 256 == 0 && cols <= 256 * kNormWarpChunks)
    return launch(rmsnorm_warp_kernel, dim3(static_cast<unsigned>((static_cast<int64_t>(rows) + 7) / 8)), dim3(256), 0,
                  static_cast<cudaStream_t>(stream), (flags & IRON_FLAG_PDL) != 0, x, residual, x_out, weight, y,
                  rows, cols, eps);
  const int threads = cols >= 2048 ? 256 : 128;
  return launch(rmsnorm_kernel, dim3(rows), dim3(threads), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, x, residual, x_out, weight, y, cols, eps);
}

extern "C" int iron_rope(const uint16_t *x, const uint16_t *angles, const float *angles_f32,
                         uint16_t *y, int rows, int cols, int angle_rows, const int32_t *pos,
                         int method, unsigned flags, void *stream) {
  if (!x || !y || (!angles && !angles_f32)) return IRON_ERR_NULL;
  if (rows <= 0 || cols <= 0 || cols % 2 || angle_rows <= 0 || rows % angle_rows) return IRON_ERR_SHAPE;
  if (method != 0 && method != 1) return IRON_ERR_ARG;
  const int64_t work = static_cast<int64_t>(rows) * (cols / 2);
  return launch(rope_kernel, dim3(grid_for(work, 256)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), (flags & IRON_FLAG_PDL) != 0, x, angles,
                angles_f32, y, rows, cols, rows / angle_rows, pos, method);
}

extern "C" int iron_softmax(const uint16_t *x, uint16_t *y, int rows, int cols, int valid,
                            const int32_t *valid_dev, unsigned flags, void *stream) {
  if (!x || !y) return IRON_ERR_NULL;
  if (rows <= 0 || cols <= 0) return IRON_ERR_SHAPE;
  const int threads = cols >= 1024 ? 256 : 128;
  return launch(softmax_kernel, dim3(rows), dim3(threads), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, x, y, cols, valid, valid_dev);
}

extern "C" int iron_eltwise(const uint16_t *a, const uint16_t *b, uint16_t *y, int64_t n, int op,
                            unsigned flags, void *stream) {
  if (!a || !y || (op != 0 && !b)) return IRON_ERR_NULL;
  if (n <= 0) return IRON_ERR_SHAPE;
  if (op < 0 || op > 3) return IRON_ERR_ARG;
  if ((n & 7) == 0 && (!aligned16(a) || !aligned16(y) || (b && !aligned16(b)))) return IRON_ERR_ALIGN;
  if ((n & 7) != 0 && (reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(y) |
                       reinterpret_cast<uintptr_t>(b)) & 1)
    return IRON_ERR_ALIGN;
  return launch(eltwise_kernel, dim3(grid_for(n / 8 + 1, 256)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), (flags & IRON_FLAG_PDL) != 0, a, b, y, n, op);
}

extern "C" int iron_strided_copy(const void *in, void *out, int elem_size, int ndim_in,
                                 const int64_t *in_sizes, const int64_t *in_strides,
                                 int64_t in_offset, int ndim_out, const int64_t *out_sizes,
                                 const int64_t *out_strides, int64_t out_offset, int channels,
                                 const int32_t *in_addend_dev, const int32_t *out_addend_dev,
                                 int64_t in_size, int64_t out_size, unsigned flags, void *stream) {
  if (!in || !out || !in_sizes || !in_strides || !out_sizes || !out_strides) return IRON_ERR_NULL;
  if (ndim_in < 1 || ndim_in > 4 || ndim_out < 1 || ndim_out > 4 || channels < 1) return IRON_ERR_SHAPE;
  Tap4 s, d;
  for (int i = 0; i < 4; ++i) {
    const int si = i - (4 - ndim_in), di = i - (4 - ndim_out);
    s.size[i] = si >= 0 ? in_sizes[si] : 1;
    s.stride[i] = si >= 0 ? in_strides[si] : 0;
    d.size[i] = di >= 0 ? out_sizes[di] : 1;
    d.stride[i] = di >= 0 ? out_strides[di] : 0;
    if (s.size[i] < 0 || d.size[i] < 0) return IRON_ERR_SHAPE;
  }
  s.offset = in_offset;
  d.offset = out_offset;
  // every dimension is >= 1 after padding, so the channel split is on the innermost one
  const int64_t s3 = s.size[3] / channels, d3 = d.size[3] / channels;
  const int64_t s_per = s.size[0] * s.size[1] * s.size[2] * s3;
  const int64_t d_per = d.size[0] * d.size[1] * d.size[2] * d3;
  if (s_per != d_per) return IRON_ERR_SHAPE;  // the two patterns must move as many elements
  if (s_per == 0) return IRON_OK;
  const unsigned grid = grid_for(s_per * channels, 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  switch (elem_size) {
    case 1: return launch(strided_copy_kernel<uint8_t>, dim3(grid), dim3(256), 0, st, pdl,
                          static_cast<const uint8_t *>(in), static_cast<uint8_t *>(out), s, d, channels,
                          s3, d3, s_per, in_addend_dev, out_addend_dev, in_size, out_size);
    case 2: return launch(strided_copy_kernel<uint16_t>, dim3(grid), dim3(256), 0, st, pdl,
                          static_cast<const uint16_t *>(in), static_cast<uint16_t *>(out), s, d,
                          channels, s3, d3, s_per, in_addend_dev, out_addend_dev, in_size, out_size);
    case 4: return launch(strided_copy_kernel<uint32_t>, dim3(grid), dim3(256), 0, st, pdl,
                          static_cast<const uint32_t *>(in), static_cast<uint32_t *>(out), s, d,
                          channels, s3, d3, s_per, in_addend_dev, out_addend_dev, in_size, out_size);
    case 8: return launch(strided_copy_kernel<uint64_t>, dim3(grid), dim3(256), 0, st, pdl,
                          static_cast<const uint64_t *>(in), static_cast<uint64_t *>(out), s, d,
                          channels, s3, d3, s_per, in_addend_dev, out_addend_dev, in_size, out_size);
    default: return IRON_ERR_ARG;
  }
}

extern "C" int iron_repeat_interleave(const void *in, void *out, int64_t rows, int64_t row_bytes,
                                      int repeat, unsigned flags, void *stream) {
  if (!in || !out) return IRON_ERR_NULL;
  if (rows <= 0 || row_bytes <= 0 || repeat <= 0) return IRON_ERR_SHAPE;
  if (row_bytes % 16 || !aligned16(in) || !aligned16(out)) return IRON_ERR_ALIGN;
  const int64_t vecs = row_bytes / 16;
  return launch(repeat_kernel, dim3(grid_for(rows * repeat * vecs, 256)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), (flags & IRON_FLAG_PDL) != 0,
                static_cast<const uint4 *>(in), static_cast<uint4 *>(out), rows, vecs, repeat);
}

extern "C" int iron_transpose(const void *in, void *out, int M, int N, int batches, int elem_size,
                              unsigned flags, void *stream) {
  if (!in || !out) return IRON_ERR_NULL;
  if (M <= 0 || N <= 0 || batches <= 0 || batches > 65535) return IRON_ERR_SHAPE;
  dim3 grid((N + 31) / 32, (M + 31) / 32, batches), block(32, 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  if (grid.y > 65535) return IRON_ERR_SHAPE;
  switch (elem_size) {
    case 2: return launch(transpose_kernel<uint16_t>, grid, block, 0, st, pdl,
                          static_cast<const uint16_t *>(in), static_cast<uint16_t *>(out), M, N);
    case 4: return launch(transpose_kernel<uint32_t>, grid, block, 0, st, pdl,
                          static_cast<const uint32_t *>(in), static_cast<uint32_t *>(out), M, N);
    default: return IRON_ERR_ARG;
  }
}
