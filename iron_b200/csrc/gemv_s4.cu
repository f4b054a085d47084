// int4 group-32 GEMV, streamed through a bulk-copy shared-memory ring.
//
// Weights are first repacked (iron_pack_int4g32) into units of one 16-row tile x
// 128 k (4 groups): 1024 code bytes in the order the MMA fragments want them
// (lane-major, so every warp reads 512 contiguous bytes) followed by the tile's
// 16 x 4 bf16 scales (128 B). A unit is 1152 bytes; the units of a matrix are
// stored tile-major, so any contiguous range of units is one contiguous block.
//
// One CTA per SM takes an equal share of the units (ranges may split a tile
// between neighbouring CTAs). A producer warp streams the share into a ring of
// shared-memory stages with cp.async.bulk + mbarriers; the first stages are
// issued before griddepcontrol.wait, so under programmatic dependent launch a
// GEMV streams its weights while the previous kernel is still running. Eight
// consumer warps unpack the codes with a LOP3 bf16 "magic number" (exact values
// 136 + q), reduce each 32-k group with two bf16 MMAs (plus two MMAs with a
// constant -136 operand that cancel the bias) and apply the group scale in fp32
// to the MMA result. Tiles split between CTAs are combined by the last CTA to
// arrive (per-tile counter), summing the partials in CTA order, so the result is
// bitwise deterministic.
#include "pipeline.cuh"

namespace iron {

constexpr int kS4UnitBytes = 1152;
constexpr int kS4CodeBytes = 1024;
constexpr int kS4StepUnits = 16;   // units per pipeline stage
constexpr int kS4Stages = 4;
constexpr int kS4Consumers = 8;    // consumer warps
constexpr int kS4Threads = 32 * (kS4Consumers + 1);
constexpr int kS4MaxCtas = 256;    // bound used for the workspace size

struct S4Work {
  int64_t U;   // total units
  int cpt;     // units (chunks of 128 k) per tile
  int G;       // CTAs
};

__device__ __forceinline__ int64_t s4_unit_begin(int64_t c, const S4Work &w) {
  return c * w.U / w.G;
}
// CTA owning unit u: the largest c with floor(c*U/G) <= u.
__device__ __forceinline__ int s4_owner(int64_t u, const S4Work &w) {
  return static_cast<int>(((u + 1) * w.G - 1) / w.U);
}

__device__ __forceinline__ uint32_t lop3_and_xor_(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t prmt_(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ void mma_zero(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// ws layout: [int err, pad to 16][int counters[tiles], pad to 16][float slots[G][2][NT*512/4]]
__host__ __device__ inline int64_t s4_counters_off() { return 16; }
__host__ __device__ inline int64_t s4_slots_off(int64_t tiles) {
  return 16 + ((tiles * 4 + 15) / 16) * 16;
}

template <int NT>
__global__ void __launch_bounds__(kS4Threads, (NT == 1) ? 2 : 1)
gemv_s4g32_stream_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ x,
                         uint16_t *__restrict__ y, int N, int K, int n_vec,
                         const uint16_t *__restrict__ residual, uint8_t *__restrict__ ws,
                         S4Work w) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kS4Stages];
  __shared__ __align__(8) uint64_t empty_bar[kS4Stages];
  uint8_t *stages = smem;
  float *red = reinterpret_cast<float *>(smem + kS4Stages * kS4StepUnits * kS4UnitBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int64_t u0 = s4_unit_begin(cta, w), u1 = s4_unit_begin(cta + 1, w);
  int *err = ws ? reinterpret_cast<int *>(ws) : nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS4Stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kS4Consumers);
    }
    mbar_init_fence();
  }
  __syncthreads();
  // The next kernel of the stream may launch now: it can only stream its own
  // weights until it reaches griddepcontrol.wait, which waits for this grid.
  pdl_launch_dependents();

  // ---------------- producer warp ----------------
  if (warp == kS4Consumers) {
    if (lane == 0) {
      int64_t pos = u0;
      int step = 0;
      bool ok = true;
      while (pos < u1) {
        const int64_t tile_end = (pos / w.cpt + 1) * w.cpt;
        const int64_t end = min(min(u1, tile_end), pos + kS4StepUnits);
        const int s = step % kS4Stages;
        if (step >= kS4Stages) {
          if (!mbar_wait(&empty_bar[s], ((step / kS4Stages) - 1) & 1)) {
            raise_error(err, IRON_ERR_TIMEOUT);
            ok = false;
            break;
          }
        }
        const uint32_t bytes = static_cast<uint32_t>((end - pos) * kS4UnitBytes);
        mbar_arrive_expect_tx(&full_bar[s], bytes);
        bulk_g2s(stages + s * kS4StepUnits * kS4UnitBytes, packed + pos * kS4UnitBytes, bytes,
                 &full_bar[s]);
        pos = end;
        ++step;
      }
      // Do not leave with copies in flight: wait (bounded) for the last stages.
      if (ok) {
        for (int k = max(0, step - kS4Stages); k < step; ++k)
          (void)mbar_wait(&full_bar[k % kS4Stages], (k / kS4Stages) & 1);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  pdl_wait();  // activations and outputs belong to the preceding kernel's world
  const int gid = lane >> 2, tid = lane & 3;
  const uint32_t kBias[4] = {0xC308C308u, 0xC308C308u, 0xC308C308u, 0xC308C308u};  // -136
  float acc[NT][4];
  int64_t pos = u0;
  int step = 0;
  int tile_count = 0;
  bool failed = false;  // after a timed-out wait: skip work, keep barrier participation
  while (pos < u1) {
    const int64_t tile = pos / w.cpt;
    const int64_t tile_begin = tile * w.cpt, tile_end = tile_begin + w.cpt;
    if (pos == u0 || pos == tile_begin) {
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
    }
    const int64_t end = min(min(u1, tile_end), pos + kS4StepUnits);
    const int s = step % kS4Stages;
    if (!failed && !mbar_wait(&full_bar[s], (step / kS4Stages) & 1)) {
      raise_error(err, IRON_ERR_TIMEOUT);
      failed = true;
    }
    const uint8_t *stage = stages + s * kS4StepUnits * kS4UnitBytes;
#pragma unroll 1
    for (int64_t u = pos + warp; !failed && u < end; u += kS4Consumers) {
      const uint8_t *unit = stage + (u - pos) * kS4UnitBytes;
      const uint4 clo = *reinterpret_cast<const uint4 *>(unit + lane * 16);
      const uint4 chi = *reinterpret_cast<const uint4 *>(unit + 512 + lane * 16);
      const uint4 sc = *reinterpret_cast<const uint4 *>(unit + kS4CodeBytes + gid * 16);
      const int c = static_cast<int>(u - tile_begin);  // chunk within the row
      const uint32_t wl[4] = {clo.x, clo.y, clo.z, clo.w};
      const uint32_t wh[4] = {chi.x, chi.y, chi.z, chi.w};
      const uint32_t sl2[2] = {sc.x, sc.y}, sh2[2] = {sc.z, sc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t pl[4], ph[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pl[i] = lop3_and_xor_(wl[j] >> (4 * i), 0x000f000fu, 0x43084308u);
          ph[i] = lop3_and_xor_(wh[j] >> (4 * i), 0x000f000fu, 0x43084308u);
        }
        const float s_lo = (j & 1) ? bf16_hi(sl2[j >> 1]) : bf16_lo(sl2[j >> 1]);
        const float s_hi = (j & 1) ? bf16_hi(sh2[j >> 1]) : bf16_lo(sh2[j >> 1]);
        const uint32_t A0[4] = {pl[0], ph[0], pl[1], ph[1]};
        const uint32_t A1[4] = {pl[2], ph[2], pl[3], ph[3]};
        const int kx = (c * 4 + j) * 32 + tid * 8;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int v = t * 8 + gid;
          uint4 xb = make_uint4(0u, 0u, 0u, 0u);
          if (v < n_vec) xb = __ldg(reinterpret_cast<const uint4 *>(x + static_cast<int64_t>(v) * K + kx));
          const uint32_t b0 = prmt_(xb.x, xb.z, 0x5410u), b1 = prmt_(xb.x, xb.z, 0x7632u);
          const uint32_t b2 = prmt_(xb.y, xb.w, 0x5410u), b3 = prmt_(xb.y, xb.w, 0x7632u);
          float d[4];
          mma_zero(d, A0, b0, b1);
          mma_bf16_16816(d, kBias, b0, b1);
          mma_bf16_16816(d, A1, b2, b3);
          mma_bf16_16816(d, kBias, b2, b3);
          acc[t][0] = fmaf(s_lo, d[0], acc[t][0]);
          acc[t][1] = fmaf(s_lo, d[1], acc[t][1]);
          acc[t][2] = fmaf(s_hi, d[2], acc[t][2]);
          acc[t][3] = fmaf(s_hi, d[3], acc[t][3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);

    const bool tile_done = (end == tile_end) || (end == u1);
    if (tile_done) {
      float *rb = red + (tile_count & 1) * (kS4Consumers * NT * 128);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) rb[((warp * NT + t) * 4 + e) * 32 + lane] = acc[t][e];
      named_sync(1, 32 * kS4Consumers);
      if (warp == 0) {
        float v[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float sum = 0.f;
#pragma unroll
            for (int q = 0; q < kS4Consumers; ++q) sum += rb[((q * NT + t) * 4 + e) * 32 + lane];
            v[t][e] = sum;
          }
        const bool whole = tile_begin >= u0 && tile_end <= u1;
        bool store = whole && !failed;
        if (!whole && !failed) {
          // Publish this CTA's partial; the last contributor combines in CTA order.
          const int side = (tile == u0 / w.cpt) ? 0 : 1;
          float *slots = reinterpret_cast<float *>(ws + s4_slots_off(static_cast<int64_t>(w.U / w.cpt)));
          float *mine = slots + (static_cast<int64_t>(cta) * 2 + side) * (NT * 128);
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) mine[(t * 4 + e) * 32 + lane] = v[t][e];
          __threadfence();
          __syncwarp();
          int *counter = reinterpret_cast<int *>(ws + s4_counters_off()) + tile;
          const int c_first = s4_owner(tile_begin, w), c_last = s4_owner(tile_end - 1, w);
          int prev = 0;
          if (lane == 0) prev = atomicAdd(counter, 1);
          prev = __shfl_sync(0xffffffffu, prev, 0);
          if (prev == c_last - c_first) {
            __threadfence();
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) v[t][e] = 0.f;
            for (int cc = c_first; cc <= c_last; ++cc) {
              const int sd = (tile == s4_unit_begin(cc, w) / w.cpt) ? 0 : 1;
              const float *theirs = slots + (static_cast<int64_t>(cc) * 2 + sd) * (NT * 128);
#pragma unroll
              for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) v[t][e] += __ldcg(theirs + (t * 4 + e) * 32 + lane);
            }
            if (lane == 0) *counter = 0;  // leave the workspace zeroed for the next call
            store = true;
          }
        }
        if (store) {
          const int row0 = static_cast<int>(tile) * 16;
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int row = row0 + gid + ((e >> 1) << 3);
              const int vv = t * 8 + tid * 2 + (e & 1);
              if (vv < n_vec) {
                const int64_t o = static_cast<int64_t>(vv) * N + row;
                float r = v[t][e];
                if (residual) r += bf16_bits_to_float(residual[o]);
                y[o] = float_to_bf16_bits(r);
              }
            }
        }
      }
      ++tile_count;
    }
    pos = end;
    ++step;
  }
}

// Repack natural-layout codes [N, K/2] + scales [N, K/32] into GEMV units.
// One thread per 16-byte piece of a unit (72 pieces per unit).
__global__ void pack_s4g32_kernel(const uint8_t *__restrict__ codes,
                                  const uint16_t *__restrict__ scales, uint8_t *__restrict__ out,
                                  int N, int K, int64_t pieces) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= pieces) return;
  const int cpt = K / 128;
  const int64_t unit = p / 72;
  const int piece = static_cast<int>(p % 72);
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
      words[j] = static_cast<uint32_t>(g[0]) | (static_cast<uint32_t>(g[1]) << 8) |
                 (static_cast<uint32_t>(g[2]) << 16) | (static_cast<uint32_t>(g[3]) << 24);
    }
  } else {
    const int gid = piece - 64;
    const int64_t rlo = tile * 16 + gid, rhi = rlo + 8;
    const uint16_t *slo = scales + rlo * (K / 32) + c * 4;
    const uint16_t *shi = scales + rhi * (K / 32) + c * 4;
    words[0] = slo[0] | (static_cast<uint32_t>(slo[1]) << 16);
    words[1] = slo[2] | (static_cast<uint32_t>(slo[3]) << 16);
    words[2] = shi[0] | (static_cast<uint32_t>(shi[1]) << 16);
    words[3] = shi[2] | (static_cast<uint32_t>(shi[3]) << 16);
  }
  reinterpret_cast<uint4 *>(out)[p] = make_uint4(words[0], words[1], words[2], words[3]);
}

static int s4_grid(int64_t units) {
  const int64_t g = sm_count();
  return static_cast<int>(units < g ? units : g);
}

template <int NT>
static int launch_s4_stream(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K,
                            int n_vec, const uint16_t *res, uint8_t *ws, bool pdl,
                            cudaStream_t s) {
  S4Work w;
  w.cpt = K / 128;
  w.U = static_cast<int64_t>(N / 16) * w.cpt;
  w.G = s4_grid(w.U);
  const size_t smem = static_cast<size_t>(kS4Stages) * kS4StepUnits * kS4UnitBytes +
                      2 * kS4Consumers * NT * 128 * sizeof(float);
  static bool attr_set[9] = {false};
  if (!attr_set[NT]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_s4g32_stream_kernel<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return IRON_ERR_CUDA;
    }
    attr_set[NT] = true;
  }
  return launch(gemv_s4g32_stream_kernel<NT>, dim3(w.G), dim3(kS4Threads), smem, s, pdl, packed, x,
                y, N, K, n_vec, res, ws, w);
}

}  // namespace iron

using namespace iron;

extern "C" size_t iron_gemv_int4g32_workspace_bytes(int N, int K, int n_vec) {
  if (N <= 0 || K <= 0 || n_vec <= 0) return 0;
  const int nt = n_vec <= 8 ? 1 : n_vec <= 16 ? 2 : n_vec <= 32 ? 4 : 8;
  const int64_t tiles = N / 16;
  return static_cast<size_t>(s4_slots_off(tiles) +
                             static_cast<int64_t>(kS4MaxCtas) * 2 * nt * 128 * sizeof(float));
}

extern "C" int iron_pack_int4g32(const uint8_t *codes, const uint16_t *scales, uint8_t *packed,
                                 int N, int K, void *stream) {
  if (!codes || !scales || !packed) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || N % 16 || K % 128) return IRON_ERR_SHAPE;
  if (!aligned16(packed)) return IRON_ERR_ALIGN;
  const int64_t pieces = static_cast<int64_t>(N / 16) * (K / 128) * 72;
  const int threads = 256;
  pack_s4g32_kernel<<<static_cast<unsigned>((pieces + threads - 1) / threads), threads, 0,
                      static_cast<cudaStream_t>(stream)>>>(codes, scales, packed, N, K, pieces);
  return launch_status();
}

extern "C" int iron_gemv_int4g32(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N,
                                 int K, int n_vec, const uint16_t *residual, void *workspace,
                                 size_t workspace_bytes, unsigned flags, void *stream) {
  if (!packed || !x || !y || !workspace) return IRON_ERR_NULL;
  if (N <= 0 || K <= 0 || n_vec <= 0 || n_vec > 64) return IRON_ERR_SHAPE;
  if (K % 128 || N % 16) return IRON_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(x) || !aligned16(workspace)) return IRON_ERR_ALIGN;
  if (workspace_bytes < iron_gemv_int4g32_workspace_bytes(N, K, n_vec)) return IRON_ERR_WORKSPACE;
  if (sm_count() > kS4MaxCtas) return IRON_ERR_UNSUPPORTED;
  const bool pdl = (flags & IRON_FLAG_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  if (n_vec <= 8) return launch_s4_stream<1>(packed, x, y, N, K, n_vec, residual, ws, pdl, s);
  if (n_vec <= 16) return launch_s4_stream<2>(packed, x, y, N, K, n_vec, residual, ws, pdl, s);
  if (n_vec <= 32) return launch_s4_stream<4>(packed, x, y, N, K, n_vec, residual, ws, pdl, s);
  return launch_s4_stream<8>(packed, x, y, N, K, n_vec, residual, ws, pdl, s);
}
