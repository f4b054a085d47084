// uint4 tile dequantization: IRON's Dequant payload -> bf16.
//
// Per tile of T elements the payload holds T/2 code bytes (element 2k is the low
// nibble of byte k, unsigned 0..15) and then T/G little-endian bf16 scales. Each
// output is bf16(code * scale), the exact fp32 product rounded once. The kernel
// is write-bound (2 B out per 0.56 B in): one thread turns one code byte into a
// bf16x2 store, so warps write 128 contiguous bytes per instruction.
#include "common.cuh"

namespace iron {

__global__ void dequant_u4_kernel(const uint8_t *__restrict__ payload, uint32_t *__restrict__ out,
                                  int64_t total_pairs, int tile, int group) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= total_pairs) return;
  const int pairs_per_tile = tile / 2;
  const int64_t t = p / pairs_per_tile;
  const int j = static_cast<int>(p - t * pairs_per_tile);  // code byte within the tile
  const int64_t tile_bytes = tile / 2 + 2 * (tile / group);
  const uint8_t *base = payload + t * tile_bytes;
  const uint8_t code = base[j];
  const int g = (2 * j) / group;  // both elements of a byte share a group (group even)
  const uint8_t *sp = base + tile / 2 + 2 * g;
  const uint16_t sbits = static_cast<uint16_t>(sp[0]) | (static_cast<uint16_t>(sp[1]) << 8);
  const float s = bf16_bits_to_float(sbits);
  const float lo = static_cast<float>(code & 0xF) * s;
  const float hi = static_cast<float>(code >> 4) * s;
  out[p] = static_cast<uint32_t>(float_to_bf16_bits(lo)) |
           (static_cast<uint32_t>(float_to_bf16_bits(hi)) << 16);
}

}  // namespace iron

extern "C" int iron_dequant_u4(const uint8_t *payload, uint16_t *out, int64_t size, int tile_size,
                               int group_size, void *stream) {
  if (!payload || !out) return IRON_ERR_NULL;
  if (size <= 0 || tile_size <= 0 || group_size <= 0) return IRON_ERR_SHAPE;
  if (group_size % 2 || tile_size % group_size || size % tile_size) return IRON_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(out) & 3u) return IRON_ERR_ALIGN;
  const int64_t pairs = size / 2;
  const int threads = 256;
  const int64_t blocks = (pairs + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return IRON_ERR_SHAPE;
  iron::dequant_u4_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                            static_cast<cudaStream_t>(stream)>>>(
      payload, reinterpret_cast<uint32_t *>(out), pairs, tile_size, group_size);
  return iron::launch_status();
}
