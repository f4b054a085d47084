// On-device next-token sampling: temperature, top-k and a multinomial draw, the steps
// of IRON's generate_token (iron/applications/llama_3.2_1b/llama_inference_harness.py:
// 146-169) on the logits the lm-head GEMV left in HBM, so no logits row crosses to the
// host per token.
//
// One CTA of 1024 threads per sequence. Top-k keeps every logit >= the k-th largest
// (ties kept, as torch.topk + `logits < min_val -> -inf` keeps them); the k-th
// largest is found exactly by a two-pass radix select over order-preserving 16-bit
// keys of the bf16 logits (a 256-bin histogram of the high byte, then of the low
// byte among the chosen high byte). The kept logits are scaled by 1/temperature and
// exponentiated against their maximum in fp32; a counter-based uniform u picks the
// first index whose running sum of weights exceeds u times their total. Each thread
// owns a contiguous chunk of the vocabulary and the running sums are combined in a
// fixed order, so the draw is bitwise reproducible for a given seed and position.
//
// The uniform comes from SplitMix64 (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) applied to (seed, sequence,
// position): each decode step draws afresh as positions advance, and a graph replay
// needs no host-side RNG state.
#include "common.cuh"

namespace iron {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint32_t logit_key(uint16_t bits) {
  // order-preserving: larger bf16 value -> larger key; NaN sorts below everything
  if ((bits & 0x7fffu) > 0x7f80u) return 0u;
  return (bits & 0x8000u) ? (~bits & 0xffffu) : (bits | 0x8000u);
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Uniform in [0, 1) with 24 random bits, a function of (seed, sequence, position).
__device__ __forceinline__ float sample_uniform(uint64_t seed, int b, int pos) {
  const uint64_t z = splitmix64(seed ^ splitmix64((static_cast<uint64_t>(static_cast<uint32_t>(pos)) << 32) |
                                                  static_cast<uint32_t>(b)));
  return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

// In a 256-bin histogram (shared), the bin holding the k-th largest key and how many
// keys lie above that bin. Executed by warp 0; results in *bin_out / *above_out.
__device__ __forceinline__ void select_bin(const unsigned *hist, int k, int *bin_out, int *above_out) {
  const int lane = threadIdx.x & 31;
  // lane l owns bins 255 - 8l .. 248 - 8l (descending); suffix counts from the top
  unsigned own = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) own += hist[255 - 8 * lane - i];
  unsigned incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const unsigned excl = incl - own;  // keys in the bins above this lane's eight
  const bool here = excl < static_cast<unsigned>(k) && incl >= static_cast<unsigned>(k);
  if (here) {
    unsigned above = excl;
    int bin = 255 - 8 * lane;
    for (int i = 0; i < 8; ++i) {
      const int bb = 255 - 8 * lane - i;
      if (above + hist[bb] >= static_cast<unsigned>(k)) {
        bin = bb;
        break;
      }
      above += hist[bb];
    }
    *bin_out = bin;
    *above_out = static_cast<int>(above);
  }
}

// Histogram of 8 key bits (the high byte, or the low byte of keys whose high byte is
// `hi_match`) over the row: warp-private bins (lanes with equal bins aggregated by
// __match_any_sync, so no two lanes of a warp add to one bin at once), summed into
// hist[256] at the end.
__device__ __forceinline__ void key_histogram(const uint16_t *row, int V, bool low, uint32_t hi_match,
                                              unsigned (*wh)[256], unsigned *hist) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int i = lane; i < 256; i += 32) wh[warp][i] = 0u;
  __syncwarp();
  const int rounds = (V + kSampleThreads - 1) / kSampleThreads;  // uniform trip count per warp
  for (int j = 0; j < rounds; ++j) {
    const int i = j * kSampleThreads + t;
    uint32_t bin = 256u;  // no bin
    if (i < V) {
      const uint32_t key = logit_key(ld_act_u16(row + i));
      if (!low) bin = key >> 8;
      else if ((key >> 8) == hi_match) bin = key & 0xffu;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, bin);
    if (bin < 256u && lane == __ffs(peers) - 1) wh[warp][bin] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int b = t; b < 256; b += kSampleThreads) {
    unsigned sum = 0u;
    for (int w = 0; w < kSampleThreads / 32; ++w) sum += wh[w][b];
    hist[b] = sum;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSampleThreads)
sample_topk_kernel(const uint16_t *__restrict__ logits, int V, float inv_temp, int top_k, uint64_t seed,
                   int *__restrict__ tokens, int *__restrict__ pos) {
  pdl_wait();
  pdl_launch_dependents();  // after the wait: the next step reads the token this writes
  __shared__ unsigned wh[kSampleThreads / 32][256];
  __shared__ unsigned hist[256];
  __shared__ int sel_bin, sel_above, max_key;
  __shared__ float warp_sums[32];
  __shared__ int claimed;
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint16_t *row = logits + static_cast<int64_t>(b) * V;
  const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int c0 = min(V, t * chunk), c1 = min(V, c0 + chunk);
  const int p = pos ? ld_act_i32(pos + b) : 0;
  if (t == 0) {
    max_key = 0;
    claimed = -1;
  }
  __syncthreads();

  // ---- threshold key: the k-th largest (0 keeps everything) ----------------------
  uint32_t thresh = 0u;
  if (top_k > 0 && top_k < V) {
    key_histogram(row, V, false, 0u, wh, hist);
    if (warp == 0) select_bin(hist, top_k, &sel_bin, &sel_above);
    __syncthreads();
    const uint32_t hi = static_cast<uint32_t>(sel_bin);
    const int k2 = top_k - sel_above;
    key_histogram(row, V, true, hi, wh, hist);
    if (warp == 0) select_bin(hist, k2, &sel_bin, &sel_above);
    __syncthreads();
    thresh = (hi << 8) | static_cast<uint32_t>(sel_bin);
  }
  // ---- the largest kept logit --------------------------------------------------------
  int mk = 0;
  for (int i = t; i < V; i += kSampleThreads) mk = max(mk, static_cast<int>(logit_key(ld_act_u16(row + i))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mk = max(mk, __shfl_xor_sync(0xffffffffu, mk, o));
  if (lane == 0) atomicMax(&max_key, mk);
  __syncthreads();
  const uint32_t mkey = static_cast<uint32_t>(max_key);
  const uint16_t mbits = (mkey & 0x8000u) ? static_cast<uint16_t>(mkey & 0x7fffu) : static_cast<uint16_t>(~mkey);
  const float mx = bf16_bits_to_float(mbits) * inv_temp;

  // ---- weights exp((l - max) / T) of the kept logits: chunk sums, fixed-order scan -----
  float own = 0.f;
  for (int i = c0; i < c1; ++i) {
    const uint16_t v = ld_act_u16(row + i);
    if (logit_key(v) >= thresh && logit_key(v) > 0u) own += __expf(bf16_bits_to_float(v) * inv_temp - mx);
  }
  float incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  float wbase = 0.f, total = 0.f;
  for (int w = 0; w < kSampleThreads / 32; ++w) {
    if (w < warp) wbase += warp_sums[w];
    total += warp_sums[w];
  }
  const float before = wbase + incl - own;  // weights of all chunks before this thread's
  const float r = sample_uniform(seed, b, p) * total;
  if (own > 0.f && before <= r && r < before + own) {
    float acc = before;
    int pick = -1, last = -1;
    for (int i = c0; i < c1; ++i) {
      const uint16_t v = ld_act_u16(row + i);
      if (logit_key(v) >= thresh && logit_key(v) > 0u) {
        last = i;
        acc += __expf(bf16_bits_to_float(v) * inv_temp - mx);
        if (acc > r) {
          pick = i;
          break;
        }
      }
    }
    atomicMax(&claimed, pick >= 0 ? pick : last);
  }
  __syncthreads();
  if (t == 0) {
    int tok = claimed;
    if (tok < 0) {  // r fell past the rounded total: the last kept logit
      for (int i = V - 1; i >= 0; --i)
        if (logit_key(ld_act_u16(row + i)) >= thresh && logit_key(ld_act_u16(row + i)) > 0u) {
          tok = i;
          break;
        }
    }
    tokens[b] = tok;
    if (pos) pos[b] = p + 1;
  }
}

}  // namespace iron

using namespace iron;

extern "C" int iron_sample_topk(const uint16_t *logits, int B, int V, float temperature, int top_k,
                                unsigned long long seed, int32_t *tokens, int32_t *pos, unsigned flags,
                                void *stream) {
  if (!logits || !tokens) return IRON_ERR_NULL;
  if (B <= 0 || B > 65535 || V <= 0) return IRON_ERR_SHAPE;
  if (!(temperature >= 0.f) || temperature != temperature) return IRON_ERR_ARG;
  const float inv_temp = temperature > 0.f ? 1.0f / temperature : 1.0f;
  return launch(sample_topk_kernel, dim3(B), dim3(kSampleThreads), 0, static_cast<cudaStream_t>(stream),
                (flags & IRON_FLAG_PDL) != 0, logits, V, inv_temp, top_k, static_cast<uint64_t>(seed), tokens,
                pos);
}
