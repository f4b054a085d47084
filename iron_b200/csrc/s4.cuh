// int4 group-32 weight helpers of the GEMV kernels:
// exact dequantization of a signed nibble pair to bf16x2 (bf16(q * s), the value
// IRON's Dequant produces) and the byte-permute / LOP3 primitives it uses.
#pragma once

#include "common.cuh"

namespace iron {

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
// Signed int4 pair -> the exactly dequantized bf16x2 (IRON's Dequant then GEMV).
// `w` holds the wanted nibble at bits 0-3 and 16-19. OR-ing (nib ^ 8) into the
// mantissa of bf16 128.0 gives 136 + q exactly (q in [-8, 7]); subtracting 136 is
// exact; the scale multiply rounds the exact product once: bf16(q * s).
__device__ __forceinline__ uint32_t s4x2_dequant_(uint32_t w, uint32_t scale2) {
  uint32_t biased = lop3_and_xor_(w, 0x000f000fu, 0x43084308u), q, r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(biased), "r"(0x43084308u));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(q), "r"(scale2));
  return r;
}

// Unsigned int4 pair -> bf16x2 of min + scale * code, rounded once (fma): OR-ing the
// nibble into the mantissa of bf16 128.0 gives 128 + code exactly, subtracting 128 is
// exact, and the fma rounds the exact min + scale * code to bf16.
__device__ __forceinline__ uint32_t q4x2_dequant_(uint32_t w, uint32_t scale2, uint32_t min2) {
  uint32_t biased, q, r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(biased) : "r"(w), "r"(0x000f000fu), "r"(0x43004300u));
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(biased), "r"(0x43004300u));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(q), "r"(scale2), "r"(min2));
  return r;
}

// Nibble order of a packed 32-bit code word. Natural order (4 code bytes of one row,
// element 2b in the low nibble of byte b) holds k_i at bits 4i; the packed word holds
// k_2q at bits 4q and k_2q+1 at bits 16 + 4q, so that s4x2_dequant_(w >> 4q) is the
// bf16x2 pair (k_2q, k_2q+1): two consecutive k, which is how the activations sit in
// memory -- their 16-byte loads are the MMA B fragments without any permute.
__host__ __device__ __forceinline__ uint32_t s4_word_pack(uint32_t natural) {
  uint32_t r = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    r |= ((natural >> (8 * q)) & 0xfu) << (4 * q);             // k_2q
    r |= ((natural >> (8 * q + 4)) & 0xfu) << (16 + 4 * q);    // k_2q+1
  }
  return r;
}
// Nibble of element k_i (i in 0..7) of a packed word.
__device__ __forceinline__ uint32_t s4_word_nibble(uint32_t packed, int i) {
  return (packed >> ((i & 1) ? 16 + 4 * (i >> 1) : 4 * (i >> 1))) & 0xfu;
}

// The tensor-core form of the int4 g32 GEMV for 33..64 vectors (gemm_tc.cu): the same
// packed units and epilogues (residual, interleaved SwiGLU, argmax keys). Returns
// IRON_ERR_UNSUPPORTED for shapes it does not take (N % 128, 32 vectors or fewer).
int launch_s4_tc(const uint8_t *packed, const uint16_t *x, uint16_t *y, int N, int K, int n_vec,
                 const uint16_t *residual, int swiglu, unsigned long long *amax, bool pdl, cudaStream_t s);

}  // namespace iron
