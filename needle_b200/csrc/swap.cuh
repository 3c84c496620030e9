// Batched KV block swap between the device cache and a pinned host cache.
//
// needle copies swapped blocks one `.to()` per block per layer
// (needle/model/runner.py:175-192).  Here one launch moves every (layer,
// block) pair: the host cache is pinned memory, which the GPU addresses
// directly through unified virtual addressing, so the kernel reads and
// writes it over PCIe/C2C with 16-byte accesses, coalesced along each block.
// A block of one layer is two contiguous runs (its K half and its V half) of
// block_bytes each, at offsets blk * block_bytes and (N + blk) * block_bytes
// of that layer's [2, N, kv_heads, block_size, head_dim] cache.
#pragma once
#include "nb_common.cuh"

namespace nb {

constexpr int kSwapMaxLayers = 192;

struct SwapLayers {
  const uint8_t* src[kSwapMaxLayers];
  uint8_t* dst[kSwapMaxLayers];
};

__global__ void __launch_bounds__(256)
    swap_blocks_kernel(const __grid_constant__ SwapLayers L, int num_layers,
                       const int32_t* __restrict__ pairs, int num_pairs, int64_t src_blocks,
                       int64_t dst_blocks, int64_t block_bytes) {
  const int64_t vec_per_half = block_bytes / 16;
  const int64_t per_layer = (int64_t)num_pairs * 2 * vec_per_half;
  const int64_t total = per_layer * num_layers;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int layer = (int)(g / per_layer);
    int64_t r = g - layer * per_layer;
    const int64_t vec = r % vec_per_half;
    r /= vec_per_half;
    const int half = (int)(r & 1);
    const int pair = (int)(r >> 1);
    const int s = __ldg(pairs + 2 * pair), d = __ldg(pairs + 2 * pair + 1);
    if (s < 0 || s >= src_blocks || d < 0 || d >= dst_blocks) {
      if (vec == 0 && half == 0) set_error(kErrBlockId);
      continue;
    }
    const uint4* from = reinterpret_cast<const uint4*>(
        L.src[layer] + ((int64_t)half * src_blocks + s) * block_bytes) + vec;
    uint4* to = reinterpret_cast<uint4*>(L.dst[layer] + ((int64_t)half * dst_blocks + d) * block_bytes) + vec;
    *to = *from;
  }
}

}  // namespace nb

extern "C" {

int nb_swap_kv_blocks(const void* const* src_caches, void* const* dst_caches, int num_layers,
                      const int32_t* block_pairs, int num_pairs, int64_t src_num_blocks,
                      int64_t dst_num_blocks, int64_t block_bytes, void* stream) {
  using namespace nbh;
  if (!src_caches || !dst_caches || !block_pairs)
    return fail(NB_ERR_INVALID_ARG, "null pointer argument");
  if (num_layers <= 0 || num_layers > nb::kSwapMaxLayers)
    return fail(NB_ERR_INVALID_ARG, "num_layers must be in [1, %d]", nb::kSwapMaxLayers);
  if (num_pairs < 0 || src_num_blocks <= 0 || dst_num_blocks <= 0 || block_bytes <= 0 ||
      block_bytes % 16)
    return fail(NB_ERR_INVALID_ARG, "bad sizes (block_bytes must be a positive multiple of 16)");
  if (num_pairs == 0) return NB_OK;
  nb::SwapLayers L;
  for (int i = 0; i < num_layers; ++i) {
    if (!src_caches[i] || !dst_caches[i] || (uintptr_t)src_caches[i] % 16 ||
        (uintptr_t)dst_caches[i] % 16)
      return fail(NB_ERR_INVALID_ARG, "layer %d: null or unaligned cache pointer", i);
    L.src[i] = (const uint8_t*)src_caches[i];
    L.dst[i] = (uint8_t*)dst_caches[i];
  }
  const int64_t total = (int64_t)num_layers * num_pairs * 2 * (block_bytes / 16);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = 8ll * num_sms() * 8;  // grid-stride beyond a few waves
  if (blocks > cap) blocks = cap;
  nb::swap_blocks_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      L, num_layers, block_pairs, num_pairs, src_num_blocks, dst_num_blocks, block_bytes);
  return check_launch("swap_kv_blocks");
}

}  // extern "C"
