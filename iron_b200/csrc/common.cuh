// Shared helpers for the sm_100a kernels of libiron_b200.so.
#pragma once

#include <atomic>
#include <cstring>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/iron_b200.h"

namespace iron {

// Records the CUDA error of the last failed launch on this thread.
void set_last_cuda_error(cudaError_t e);

// Maps a CUDA error after a launch to a status; records it for iron_last_cuda_error().
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Status of a CUDA runtime call that is not a launch: records a failure for
// iron_last_cuda_error() and clears it from the runtime.
inline int call_status(cudaError_t e) {
  if (e == cudaSuccess) return IRON_OK;
  set_last_cuda_error(e);
  (void)cudaGetLastError();
  return IRON_ERR_CUDA;
}

// Number of SMs of the current device, cached per device.
int sm_count();

// One-time setup per device (function attributes apply to the current device), safe
// under concurrent callers: two threads may both run the setup, which is idempotent.
struct PerDeviceOnce {
  std::atomic<bool> done[64];
  template <typename F>
  int run(F &&setup) {  // setup() -> status; recorded as done only when it succeeds
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    const bool cached = dev >= 0 && dev < 64;
    if (cached && done[dev].load(std::memory_order_acquire)) return IRON_OK;
    const int st = setup();
    if (st == IRON_OK && cached) done[dev].store(true, std::memory_order_release);
    return st;
  }
};

// Launch `kernel` on `stream`, optionally allowing programmatic dependent launch.
template <typename... KArgs, typename... Args>
inline int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return IRON_ERR_CUDA;
  }
  return IRON_OK;
}

// ---- device helpers ---------------------------------------------------------

// Wait for the preceding kernel of the stream (no-op when launched without PDL).
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next kernel of the stream to start launching.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float bf16_bits_to_float(uint16_t v) {
  return __uint_as_float(static_cast<uint32_t>(v) << 16);
}
// Round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet).
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Loads of data that another kernel of the stream produces (activations, positions,
// partials). Kernels trigger their dependents early (programmatic dependent launch),
// so a kernel can start -- and its SM's L1 be refilled by other kernels still running
// there -- before the data it reads after griddepcontrol.wait is written. Two rules
// keep every read fresh:
//  - kernels that bound a window trigger their dependents only after their own wait:
//    the int4 GEMVs that add a residual (o_proj and down_proj, two per decoder layer),
//    RoPE + KV append and the embedding gather that starts a step. Between two bounds
//    every activation buffer is written once, and every reader of its previous
//    contents sits before the earlier bound, so it has finished before any kernel
//    that reads the new contents is launched;
//  - small kernels read such data with these loads (ld.global.cg: cached in L2 only;
//    the wait's memory clobber keeps them after it), while the bandwidth-heavy GEMV
//    activations and cache rows, written in the same window before their readers'
//    wait, use the read-only path where the caller keeps these windows.
__device__ __forceinline__ uint4 ld_act_v4(const void *p) { return __ldcg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ uint2 ld_act_v2(const void *p) { return __ldcg(reinterpret_cast<const uint2 *>(p)); }
__device__ __forceinline__ uint32_t ld_act_u32(const void *p) { return __ldcg(reinterpret_cast<const unsigned *>(p)); }
__device__ __forceinline__ uint16_t ld_act_u16(const void *p) {
  return __ldcg(reinterpret_cast<const unsigned short *>(p));
}
__device__ __forceinline__ float ld_act_f32(const float *p) { return __ldcg(p); }
__device__ __forceinline__ int ld_act_i32(const int *p) { return __ldcg(p); }
template <typename T>
__device__ __forceinline__ T ld_act(const T *p) {
  static_assert(sizeof(T) == 1 || sizeof(T) == 2 || sizeof(T) == 4 || sizeof(T) == 8 || sizeof(T) == 16,
                "1/2/4/8/16-byte elements");
  T r;
  if constexpr (sizeof(T) == 1) {
    const unsigned char b = __ldcg(reinterpret_cast<const unsigned char *>(p));
    memcpy(&r, &b, 1);
  } else if constexpr (sizeof(T) == 2) {
    const uint16_t v = ld_act_u16(p);
    memcpy(&r, &v, 2);
  } else if constexpr (sizeof(T) == 4) {
    const uint32_t v = ld_act_u32(p);
    memcpy(&r, &v, 4);
  } else if constexpr (sizeof(T) == 8) {
    const uint2 v = ld_act_v2(p);
    memcpy(&r, &v, 8);
  } else {
    const uint4 v = ld_act_v4(p);
    memcpy(&r, &v, 16);
  }
  return r;
}

// Asynchronous 16-byte global -> shared copy (both addresses 16-byte aligned), L2 only;
// completes for the issuing thread at cp_async_wait_all() after cp_async_commit().
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// 16-byte streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 2^x by the hardware approximation (ex2.approx.ftz.f32). The softmax loops call it
// with x <= 0 (results in [0, 1], ex2(-inf) = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// tanh-approximation GELU: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;
  float inner = k0 * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

// m16n8k16 bf16 MMA with fp32 accumulate: D = A * B + D.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace iron
