// Host-side creation of TMA tensor maps for the paged KV cache.
//
// The KV cache of one tensor (K or V) is [num_blocks, block_size, num_kv_heads, head_dim]
// bf16 with an arbitrary element stride per dimension and a contiguous head_dim. The map
// is 4-D with the dimensions listed innermost first: (head_dim, kv_head, slot, block).
// A box is (64 columns, 1 head, rows slots, 1 block) and lands in shared memory as
// rows x 128 bytes with the 128-byte swizzle, which is the K-major / MN-major SW128
// operand layout the tcgen05 MMAs read.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

namespace tfa {

inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// strides_elems: element strides of (block, slot, kv_head) -- head_dim stride must be 1.
// Returns 0 on success, a non-zero CUresult (or -1 if the driver entry is missing).
inline int encode_kv_map(CUtensorMap* map, const void* base, int64_t num_blocks, int64_t block_size,
                         int64_t num_kv_heads, int64_t head_dim, const int64_t strides_elems[3],
                         uint32_t box_rows) {
  auto fn = get_encode_tiled();
  if (!fn) return -1;
  cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)num_kv_heads, (cuuint64_t)block_size,
                        (cuuint64_t)num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)strides_elems[2] * 2, (cuuint64_t)strides_elems[1] * 2,
                           (cuuint64_t)strides_elems[0] * 2};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  // L2 promotion: a head_dim-64 row of one kv head is 128 bytes, and promoting it to a
  // 256-byte L2 fill also fetches the next head's row from DRAM (measured on B200 with the
  // paged gather alone, 8 kv heads: 26 GB/s per SM with 256-byte promotion, 35 GB/s with
  // 128-byte). A head_dim-128 row is 256 bytes, read as two adjacent 128-byte panels.
  const CUtensorMapL2promotion prom =
      head_dim == 64 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, prom, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

// Whole pages for the page decode kernel: the same cache, with the dimensions listed as
// (head_dim, slot, kv_head, block) so that a box of (64 columns, all slots, all kv heads,
// 1 block) lands head-major (row = kv_head * block_size + slot) as rows of 128 bytes with
// the 128-byte swizzle. A full page is one box per 64-column panel.
inline int encode_page_map(CUtensorMap* map, const void* base, int64_t num_blocks, int64_t block_size,
                           int64_t num_kv_heads, int64_t head_dim, const int64_t strides_elems[3]) {
  auto fn = get_encode_tiled();
  if (!fn) return -1;
  cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)block_size, (cuuint64_t)num_kv_heads,
                        (cuuint64_t)num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)strides_elems[1] * 2, (cuuint64_t)strides_elems[2] * 2,
                           (cuuint64_t)strides_elems[0] * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)block_size, (cuuint32_t)num_kv_heads, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

// Query rows for the decode kernel: q is [total_q, num_q_heads, head_dim] bf16 with
// element strides (token, head) and a contiguous head_dim. The map is 3-D, innermost
// first (head_dim, q_head, token); a box is (64 columns, group heads, tokens) and lands
// as group * tokens rows of 128 bytes (row = token * group + head, the packed-row order)
// with the 128-byte swizzle, the K-major SW128 operand layout of the MMA. Tokens past
// total_q are zero-filled.
inline int encode_q_map(CUtensorMap* map, const void* base, int64_t total_q, int64_t num_q_heads, int64_t head_dim,
                        int64_t token_stride, int64_t head_stride, uint32_t group, uint32_t tokens) {
  auto fn = get_encode_tiled();
  if (!fn) return -1;
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)num_q_heads, (cuuint64_t)total_q};
  cuuint64_t strides[2] = {(cuuint64_t)head_stride * 2, (cuuint64_t)token_stride * 2};
  cuuint32_t box[3] = {64, group, tokens};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

}  // namespace tfa
