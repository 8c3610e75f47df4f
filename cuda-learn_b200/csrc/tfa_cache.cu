// Paged KV-cache write (the kernel form of ToyFlashAttentionImpl.do_kv_cache_update,
// flash_attention_backend/toy_flash_attn/impl.py:121-144): scatter each new token's K and
// V rows into cache slot slot_mapping[i] = block * block_size + offset; slots < 0 are
// padding and skipped. Pure data movement: one warp per (token, kv head), 16-byte copies.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/tfa.h"

namespace tfa {
namespace {

__global__ void __launch_bounds__(256) kv_cache_update_kernel(
    const uint4* __restrict__ key, int64_t ks0, int64_t ks1, const uint4* __restrict__ value, int64_t vs0,
    int64_t vs1, uint4* __restrict__ k_cache, int64_t kc0, int64_t kc1, int64_t kc2, uint4* __restrict__ v_cache,
    int64_t vc0, int64_t vc1, int64_t vc2, const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int hkv,
    int vec_per_head, int64_t block_size, int64_t num_slots, int* err) {
  // strides are in 16-byte units here
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t tok = warp_global / hkv;
  const int h = (int)(warp_global % hkv);
  if (tok >= num_tokens) return;
  const int64_t slot = slot_mapping[tok];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (lane == 0 && err) atomicCAS(err, 0, 111);
    return;
  }
  const int64_t blk = slot / block_size, off = slot % block_size;
  for (int u = lane; u < vec_per_head; u += 32) {
    k_cache[blk * kc0 + off * kc1 + h * kc2 + u] = key[tok * ks0 + h * ks1 + u];
    v_cache[blk * vc0 + off * vc1 + h * vc2 + u] = value[tok * vs0 + h * vs1 + u];
  }
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace tfa

extern "C" int tfa_kv_cache_update(const void* key, const int64_t key_stride[2], const void* value,
                                   const int64_t value_stride[2], void* k_cache, const int64_t k_cache_stride[3],
                                   void* v_cache, const int64_t v_cache_stride[3], const int64_t* slot_mapping,
                                   int64_t num_tokens, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                                   int64_t num_blocks, void* workspace, void* stream) {
  using namespace tfa;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0) return TFA_ERR_SHAPE;
  if (num_tokens == 0) return TFA_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping || !key_stride || !value_stride || !k_cache_stride ||
      !v_cache_stride)
    return TFA_ERR_NULL_POINTER;
  // 16-byte units: head_dim * 2 bytes and every stride must be multiples of 8 elements
  if ((head_dim % 8) != 0) return TFA_ERR_LAYOUT;
  for (int i = 0; i < 2; ++i)
    if (key_stride[i] % 8 || value_stride[i] % 8) return TFA_ERR_LAYOUT;
  for (int i = 0; i < 3; ++i)
    if (k_cache_stride[i] % 8 || v_cache_stride[i] % 8) return TFA_ERR_LAYOUT;
  if (!a16(key) || !a16(value) || !a16(k_cache) || !a16(v_cache)) return TFA_ERR_LAYOUT;
  const int64_t warps = num_tokens * num_kv_heads;
  const int64_t threads = warps * 32;
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > INT32_MAX) return TFA_ERR_SHAPE;
  int* err = workspace ? reinterpret_cast<int*>(workspace) + 2 : nullptr;
  kv_cache_update_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(key), key_stride[0] / 8, key_stride[1] / 8, reinterpret_cast<const uint4*>(value),
      value_stride[0] / 8, value_stride[1] / 8, reinterpret_cast<uint4*>(k_cache), k_cache_stride[0] / 8,
      k_cache_stride[1] / 8, k_cache_stride[2] / 8, reinterpret_cast<uint4*>(v_cache), v_cache_stride[0] / 8,
      v_cache_stride[1] / 8, v_cache_stride[2] / 8, slot_mapping, num_tokens, (int)num_kv_heads, (int)(head_dim / 8),
      block_size, num_blocks * block_size, err);
  return cudaGetLastError() == cudaSuccess ? TFA_OK : TFA_ERR_CUDA;
}
