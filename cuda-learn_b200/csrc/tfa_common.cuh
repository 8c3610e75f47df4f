// Shared device code of the paged attention forward: kernel parameters, the work-item
// decomposition (sequence x kv head x q tile x kv split), the mask rule and the paged
// K/V producer (TMA gather through block_table).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100.cuh"

namespace tfa {

constexpr int kBN = 128;           // kv tokens per tile
constexpr float kLn2 = 0.69314718055994530942f;

// Error codes written by kernels into params.err (first one wins).
enum DeviceError : int {
  kDevErrTimeoutProducer = 101,
  kDevErrTimeoutMma = 102,
  kDevErrTimeoutSoftmax = 103,
  kDevErrBadBlockId = 110,
};

struct FwdParams {
  const __nv_bfloat16* q;  // [total_q, Hq, D], row strides in elements
  int64_t q_s0, q_s1;
  __nv_bfloat16* out;      // [total_q, Hq, D]
  int64_t o_s0, o_s1;
  float* lse;              // optional [total_q, Hq] natural-log LSE (contiguous)
  const int* cu_seqlens_q; // [batch + 1]
  const int* seqused_k;    // [batch]
  const int* block_table;  // [batch, bt_s0...] (inner stride 1)
  int64_t bt_s0;
  int batch, total_q, hq, hkv, group;
  int block_size, box_rows, num_blocks;
  int causal, wl, wr;      // window sides, -1 = unbounded
  float scale_log2;        // softmax_scale * log2(e)
  int rows_per_tile;       // packed (token, q head) rows per item: 16 (decode) or 128 (prefill)
  int q_tiles;             // q tiles per (sequence, kv head)
  int max_splits;          // S_max: split slots per (sequence, kv head, q tile)
  int split_cap;           // max kv tiles per split
  int num_items;           // max_splits * q_tiles * batch * hkv
  float* split_o;          // [max_splits, total_q, Hq, D] fp32 (normalised partial outputs)
  float* split_lse;        // [max_splits, total_q, Hq] fp32 (log2 domain, scaled)
  int* sched;              // [2]: next-item counter, finished-CTA counter (self-resetting)
  int* err;                // first device error code, 0 if none
  int seq_filter;          // 0: every sequence; 1: only q_len * group <= 16 (decode-shaped);
                           // 2: only q_len * group > 16 (a call split across both kernels)
  int debug_stall;         // test hook: the MMA warp waits on a barrier nobody arrives on
  const int* item_list;    // decode kernel: existing items (g * max_splits + split), longest
                           // first, built on the device for the call (NULL: slot order)
  const int* item_count;   // number of entries of item_list
  int max_seqlen_k_pages;   // block-table entries a sequence may use (prefetch bound)
  int* group_cnt;          // decode kernel instance that merges in-kernel: per work group, splits
                           // finished so far (self-resetting); the last one merges the group
};

// One unit of work: the packed q rows [row0, row0 + nrows) of kv head h of sequence b,
// against kv tiles [tile_begin, tile_end).
struct Work {
  int g;  // work group (q tile slot, sequence, kv head): the item index with split 0
  int b, h, split, nsplits;
  int q0, q_len, kv_len;
  int row0, nrows;
  int tile_begin, tile_end;
  bool exists;  // false: split slot unused by this sequence (nothing to do, nothing to write)
};

__device__ __forceinline__ int imin(int a, int b) { return a < b ? a : b; }
__device__ __forceinline__ int imax(int a, int b) { return a > b ? a : b; }

// Visible kv range [lo, hi] of query token i (0-based within its sequence).
// Restates the rule of flash_attention_func.py:367-376 with q/kv tail alignment.
__device__ __forceinline__ void visible_range(const FwdParams& p, int i, int q_len, int kv_len, int& lo, int& hi) {
  const int off = kv_len - q_len;
  lo = p.wl < 0 ? 0 : imax(0, i + off - p.wl);
  int h = (p.causal || p.wr >= 0) ? (i + off + (p.causal ? 0 : p.wr)) : (kv_len - 1);
  hi = imin(kv_len - 1, h);
}

// Number of kv tiles (and the first tile) touched by a q tile, before splitting.
__device__ __forceinline__ void tile_span(const FwdParams& p, int q_len, int kv_len, int row0, int nrows, int& t_lo,
                                          int& n_tiles) {
  n_tiles = 0;
  t_lo = 0;
  if (nrows <= 0 || kv_len <= 0) return;
  int lo_a, hi_a, lo_b, hi_b;
  visible_range(p, row0 / p.group, q_len, kv_len, lo_a, hi_a);
  visible_range(p, (row0 + nrows - 1) / p.group, q_len, kv_len, lo_b, hi_b);
  const int lo = imax(0, lo_a);
  const int hi = imin(kv_len - 1, hi_b);
  if (hi < lo) return;
  t_lo = lo / kBN;
  n_tiles = hi / kBN - t_lo + 1;
}

__device__ __forceinline__ int splits_for(const FwdParams& p, int n_tiles) {
  if (n_tiles <= 0) return 1;
  return imin(p.max_splits, (n_tiles + p.split_cap - 1) / p.split_cap);
}

// Item order: split slot slowest, then q tile (longest first for causal prefill),
// then sequence, then kv head.
__device__ __forceinline__ Work get_work(const FwdParams& p, int idx) {
  Work w;
  w.g = idx % (p.q_tiles * p.batch * p.hkv);
  w.h = idx % p.hkv;
  idx /= p.hkv;
  w.b = idx % p.batch;
  idx /= p.batch;
  const int qt = p.q_tiles - 1 - (idx % p.q_tiles);
  w.split = idx / p.q_tiles;
  w.q0 = p.cu_seqlens_q[w.b];
  w.q_len = p.cu_seqlens_q[w.b + 1] - w.q0;
  w.kv_len = p.seqused_k[w.b];
  w.row0 = qt * p.rows_per_tile;
  w.nrows = imax(0, imin(p.rows_per_tile, w.q_len * p.group - w.row0));
  // a sequence the other kernel of a mixed call handles has no rows here
  if (p.seq_filter != 0 && ((p.seq_filter == 1) != (w.q_len * p.group <= 16))) w.nrows = 0;
  int t_lo, n;
  tile_span(p, w.q_len, w.kv_len, w.row0, w.nrows, t_lo, n);
  w.nsplits = splits_for(p, n);
  w.exists = w.nrows > 0 && w.split < w.nsplits;
  w.tile_begin = t_lo + (int)(((long long)n * w.split) / w.nsplits);
  w.tile_end = t_lo + (int)(((long long)n * (w.split + 1)) / w.nsplits);
  if (!w.exists) w.tile_end = w.tile_begin;
  return w;
}

// Work item of group g (= q tile slot, sequence, kv head: the get_work order with
// split 0) and split slot `split`.
__device__ __forceinline__ Work work_of(const FwdParams& p, int g, int split) {
  const int groups = p.q_tiles * p.batch * p.hkv;
  return get_work(p, split * groups + g);
}

// Item idx of the device-built list (only compiled into the decode kernel instance that
// runs with a list, so no load through the list pointer exists where it is null).
__device__ __forceinline__ Work get_work_from_list(const FwdParams& p, int idx) {
  const int e = p.item_list[idx];
  return work_of(p, e / p.max_splits, e % p.max_splits);
}

// Called once per CTA by the producer's lane 0 after its final (out-of-range) claim: no
// claim can follow it from this CTA, so when every CTA has passed here the last one
// resets the scheduler counters for the next launch on the same stream. Done by the
// producer as soon as it stops claiming, off the consumers' critical path.
__device__ __forceinline__ void scheduler_finish(const FwdParams& p) {
  __threadfence();
  if (atomicAdd(&p.sched[1], 1) == (int)gridDim.x - 1) {
    atomicExch(&p.sched[0], 0);
    atomicExch(&p.sched[1], 0);
    __threadfence();
  }
}

// Programmatic dependent launch: lets the next kernel on the stream (the split-KV combine
// after an attention kernel, the decode kernel after the item-list kernel) be scheduled
// before this grid finishes; the dependent waits with grid_dependency_wait().
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Paged K/V gather: a producer warp fetches the 128-token tile of kv head h of sequence b
// page group by page group (one TMA box per 16-slot group and 64 columns). One tile of one
// tensor is kPanels panels of 128 rows x 128 B (64 head-dim columns, 128-byte swizzle);
// the gather debug kernel stages V and K of a tile together as [V panels][K panels]. Rows
// at or past kv_len are zero-filled by out-of-range TMA coordinates, so stale or NaN cache
// slots never reach an MMA.
// ---------------------------------------------------------------------------
template <int D>
struct KvStage {
  static constexpr int kPanels = D / 64;
  static constexpr int kPanelBytes = kBN * 128;            // 16 KB
  static constexpr int kTensorBytes = kPanels * kPanelBytes;
  static constexpr int kBytes = 2 * kTensorBytes;          // V then K (gather debug kernel)
};

struct KvMaps {
  CUtensorMap k_box, k_row, v_box, v_row;
  // whole pages, rows head-major (dims head_dim, slot, kv head, block): the page decode
  // kernel's boxes (encoded only for calls that use it)
  CUtensorMap k_page, v_page;
};

// Page and row count of 16-slot group g (box_rows slots when block_size < 16) of a tile.
// The block-table load is only issued here; its value is first used in issue_group, so
// callers can overlap its latency with a pipeline wait.
struct GroupSrc {
  int page;   // physical block (or out of range -> zero fill)
  int slot;   // first slot inside the block
  int valid;  // rows < kv_len in this group
};

__device__ __forceinline__ GroupSrc resolve_group(const FwdParams& p, const Work& w, int tile, int g) {
  const int R = p.box_rows;
  const int pos = tile * kBN + g * R;
  GroupSrc s;
  int valid = w.kv_len - pos;
  s.valid = valid < 0 ? 0 : (valid > R ? R : valid);
  s.slot = pos % p.block_size;
  s.page = p.num_blocks;
  if (s.valid > 0) s.page = __ldg(p.block_table + (int64_t)w.b * p.bt_s0 + pos / p.block_size);
  return s;
}

// Issues the TMA boxes of one group of one tensor (K or V) into `dst` (the group's first
// row inside a 128-row panel set).
template <int D>
__device__ __forceinline__ void issue_group_tensor(const FwdParams& p, const CUtensorMap* box, const CUtensorMap* row,
                                                   const Work& w, GroupSrc src, uint32_t dst, uint64_t* full_bar,
                                                   uint64_t policy) {
  const int R = p.box_rows;
  int valid = src.valid, page = src.page;
  if (valid > 0 && (page < 0 || page >= p.num_blocks)) {
    atomicCAS(p.err, 0, (int)kDevErrBadBlockId);
    page = p.num_blocks;
    valid = R;  // whole box out of range -> zeros
  }
#pragma unroll
  for (int ch = 0; ch < KvStage<D>::kPanels; ++ch) {
    const uint32_t off = dst + ch * KvStage<D>::kPanelBytes;
    if (valid == R) {
      tma_load_4d(off, box, ch * 64, w.h, src.slot, page, full_bar, policy);
    } else if (valid == 0) {
      tma_load_4d(off, box, ch * 64, w.h, 0, p.num_blocks, full_bar, policy);
    } else {
      for (int r = 0; r < R; ++r) {
        const int sl = r < valid ? src.slot + r : p.block_size;  // slot index block_size is out of range -> zeros
        tma_load_4d(off + r * 128, row, ch * 64, w.h, sl, page, full_bar, policy);
      }
    }
  }
}

template <int D>
__device__ __forceinline__ void issue_group(const FwdParams& p, const KvMaps& maps, const Work& w, int g, GroupSrc src,
                                            uint8_t* stage, uint64_t* full_bar, uint64_t policy) {
  const int R = p.box_rows;
  int valid = src.valid, page = src.page;
  if (valid > 0 && (page < 0 || page >= p.num_blocks)) {
    atomicCAS(p.err, 0, (int)kDevErrBadBlockId);
    page = p.num_blocks;
    valid = R;  // whole box out of range -> zeros
  }
  const uint32_t v_dst = smem_u32(stage) + g * R * 128;
  const uint32_t k_dst = v_dst + KvStage<D>::kTensorBytes;
  if (valid == R) {
    // Full group: all K boxes (its 64-column panels are adjacent in memory), then all V
    // boxes. With one lane per group the warp issues each box for every group in turn.
#pragma unroll
    for (int ch = 0; ch < KvStage<D>::kPanels; ++ch)
      tma_load_4d(k_dst + ch * KvStage<D>::kPanelBytes, &maps.k_box, ch * 64, w.h, src.slot, page, full_bar, policy);
#pragma unroll
    for (int ch = 0; ch < KvStage<D>::kPanels; ++ch)
      tma_load_4d(v_dst + ch * KvStage<D>::kPanelBytes, &maps.v_box, ch * 64, w.h, src.slot, page, full_bar, policy);
    return;
  }
#pragma unroll
  for (int ch = 0; ch < KvStage<D>::kPanels; ++ch) {
    const uint32_t off = ch * KvStage<D>::kPanelBytes;
    if (valid == 0) {
      tma_load_4d(k_dst + off, &maps.k_box, ch * 64, w.h, 0, p.num_blocks, full_bar, policy);
      tma_load_4d(v_dst + off, &maps.v_box, ch * 64, w.h, 0, p.num_blocks, full_bar, policy);
    } else {
      for (int r = 0; r < R; ++r) {
        const int sl = r < valid ? src.slot + r : p.block_size;  // slot index block_size is out of range -> zeros
        tma_load_4d(k_dst + off + r * 128, &maps.k_row, ch * 64, w.h, sl, page, full_bar, policy);
        tma_load_4d(v_dst + off + r * 128, &maps.v_row, ch * 64, w.h, sl, page, full_bar, policy);
      }
    }
  }
}

// Boxes of one group of one tensor (tensor 1 = K, 0 = V) into `half`, one tile of that
// tensor (kPanels panels of 128 rows).
template <int D>
__device__ __forceinline__ void issue_group_one(const FwdParams& p, const KvMaps& maps, const Work& w, int g,
                                                GroupSrc src, int tensor, uint8_t* half, uint64_t* full_bar,
                                                uint64_t policy) {
  const uint32_t dst = smem_u32(half) + g * p.box_rows * 128;
  const CUtensorMap* box = tensor ? &maps.k_box : &maps.v_box;
  if (src.valid == p.box_rows && src.page >= 0 && src.page < p.num_blocks) {
#pragma unroll
    for (int ch = 0; ch < KvStage<D>::kPanels; ++ch)
      tma_load_4d(dst + ch * KvStage<D>::kPanelBytes, box, ch * 64, w.h, src.slot, src.page, full_bar, policy);
    return;
  }
  issue_group_tensor<D>(p, box, tensor ? &maps.k_row : &maps.v_row, w, src, dst, full_bar, policy);
}

// Gathers one whole tile (all groups) into `stage`; used where no prefetch is possible.
template <int D>
__device__ __forceinline__ void produce_tile(const FwdParams& p, const KvMaps& maps, const Work& w, int tile,
                                             uint8_t* stage, uint64_t* full_bar, int lane, uint64_t policy) {
  if (lane == 0) mbar_arrive_expect_tx(full_bar, KvStage<D>::kBytes);
  __syncwarp();
  const int groups = kBN / p.box_rows;
  for (int g = lane; g < groups; g += 32)
    issue_group<D>(p, maps, w, g, resolve_group(p, w, tile, g), stage, full_bar, policy);
}

#ifdef TFA_PROFILE
__device__ void decode_stamp_hook(int i);
__device__ void decode_tile_hook(int c, int i);
#endif

// Producer warp main loop of the decode kernel. Fetches work items dynamically,
// publishes each (index, descriptor, and its Q rows loaded by TMA) into the two-slot item
// queue, so the consumers start an item without global loads, and streams the K tiles of
// its items into the K ring. When a tile has at most 32 groups (block_size >= 4), lane g
// owns group g and the block-table entries of tile t+1 are requested before the wait for
// tile t's free slot, so the table latency hides behind the pipeline; the next item is
// claimed while the last tile of the current one waits for its slot. The first item of CTA i is item i; later items
// come from the shared counter offset by the grid size, so start-up has no atomic.
template <int D, int STAGES, bool kList>
__device__ __forceinline__ void producer_loop(const FwdParams& p, const KvMaps& maps, uint8_t* ring,
                                              uint64_t* full, uint64_t* empty, uint64_t* item_full,
                                              uint64_t* item_empty, int* item_slot, Work* item_work,
                                              const CUtensorMap* q_map, uint8_t* q_bufs, int q_buf_bytes,
                                              uint64_t* q_full, volatile int* abort_flag, int lane) {
  const uint64_t policy = l2_policy_evict_first();
  const int groups = kBN / p.box_rows;
  const bool lane_per_group = groups <= 32;
  const int q_tokens = 16 / p.group;  // tokens per Q box (G heads each)
  const uint32_t q_tx = (uint32_t)(KvStage<D>::kPanels * p.group * q_tokens * 128);
  int c = 0;
  // item indices handed out: the device-built list's length, or every slot
  int bound = p.num_items;
  if constexpr (kList) {
    // This instance is launched as a programmatic dependent of the list kernel: its set-up
    // overlapped that kernel; the list and its length are read only after it completed.
    grid_dependency_wait();
    bound = *reinterpret_cast<const volatile int*>(p.item_count);
  }
  int claimed = (lane == 0) ? (int)blockIdx.x : 0;  // next item index (lane 0)
  auto claim = [&]() {
    if (lane == 0) claimed = atomicAdd(&p.sched[0], 1) + (int)gridDim.x;
  };
  for (int k = 0;; ++k) {
    const int slot = k & 1;
    if (!mbar_wait(&item_empty[slot], ((k >> 1) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
    int idx = __shfl_sync(0xffffffffu, claimed, 0);
    Work w;
    // Skip split slots a sequence does not use without bothering the consumers.
    while (idx < bound) {
      if constexpr (kList) w = get_work_from_list(p, idx);
      else w = get_work(p, idx);
      if (w.exists) break;
      claim();
      idx = __shfl_sync(0xffffffffu, claimed, 0);
    }
    if (lane == 0) {
      item_slot[slot] = idx < bound ? idx : p.num_items;  // the consumers stop at num_items
      if (idx < bound) {
        // The item's descriptor and Q rows (all heads of the group, its tokens, packed-row
        // order) go into this slot's buffers. The slot's previous item has finished: its
        // consumers arrived on item_empty only after its last MMA completed.
        item_work[slot] = w;
        mbar_arrive_expect_tx(&q_full[slot], q_tx);
        const uint32_t qdst = smem_u32(q_bufs + slot * q_buf_bytes);
#pragma unroll
        for (int ch = 0; ch < KvStage<D>::kPanels; ++ch)
          tma_load_3d(qdst + ch * (16 * 128), q_map, ch * 64, w.h * p.group, w.q0 + w.row0 / p.group, &q_full[slot]);
      }
      mbar_arrive(&item_full[slot]);
    }
    if (idx >= bound) {
      if (lane == 0) scheduler_finish(p);
      return;
    }
#ifdef TFA_PROFILE
    if (lane == 0 && k == 0 && blockIdx.x == 0 && p.rows_per_tile == 16) decode_stamp_hook(2);
#endif
    if (w.tile_end == w.tile_begin) claim();
    if (lane_per_group) {
      GroupSrc cur{}, nxt{};
      if (lane < groups) cur = resolve_group(p, w, w.tile_begin, lane);
      for (int t = w.tile_begin; t < w.tile_end; ++t, ++c) {
        if (t + 1 < w.tile_end) {
          if (lane < groups) nxt = resolve_group(p, w, t + 1, lane);
        } else {
          claim();
        }
        const int st = c % STAGES;
        if (!mbar_wait(&empty[st], ((c / STAGES) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
        if (lane == 0) mbar_arrive_expect_tx(&full[st], KvStage<D>::kTensorBytes);
        __syncwarp();
        if (lane < groups) issue_group_one<D>(p, maps, w, lane, cur, 1, ring + st * KvStage<D>::kTensorBytes, &full[st], policy);
#ifdef TFA_PROFILE
        if (lane == 0 && p.rows_per_tile == 16) decode_tile_hook(c, 0);
#endif
        cur = nxt;
      }
    } else {
      for (int t = w.tile_begin; t < w.tile_end; ++t, ++c) {
        if (t + 1 == w.tile_end) claim();
        const int st = c % STAGES;
        if (!mbar_wait(&empty[st], ((c / STAGES) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
        if (lane == 0) mbar_arrive_expect_tx(&full[st], KvStage<D>::kTensorBytes);
        __syncwarp();
        for (int g = lane; g < groups; g += 32)
          issue_group_one<D>(p, maps, w, g, resolve_group(p, w, t, g), 1, ring + st * KvStage<D>::kTensorBytes, &full[st],
                             policy);
      }
    }
  }
}

// Second producer warp of the decode kernel: follows the item queue like a consumer and
// fills the ring of V tiles (the first producer fills the ring of K tiles), so the two
// warps' barrier waits and loop overhead overlap each other's TMA issue. The rings have
// their own barriers: a K slot is free again once QK has read it, a V slot after P.V.
template <int D, int STAGES>
__device__ __forceinline__ void producer_follow_v(const FwdParams& p, const KvMaps& maps, uint8_t* ring,
                                                  uint64_t* full, uint64_t* empty, uint64_t* item_full,
                                                  uint64_t* item_empty, const int* item_slot,
                                                  const Work* item_work, volatile int* abort_flag, int lane) {
  const uint64_t policy = l2_policy_evict_first();
  const int groups = kBN / p.box_rows;
  const bool lane_per_group = groups <= 32;
  int c = 0;
  for (int k = 0;; ++k) {
    const int slot = k & 1;
    if (!mbar_wait(&item_full[slot], (k >> 1) & 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
    const int idx = item_slot[slot];
    if (idx >= p.num_items) return;
    const Work w = item_work[slot];
    GroupSrc cur{}, nxt{};
    if (lane_per_group && lane < groups && w.tile_begin < w.tile_end) cur = resolve_group(p, w, w.tile_begin, lane);
    for (int t = w.tile_begin; t < w.tile_end; ++t, ++c) {
      if (lane_per_group && lane < groups && t + 1 < w.tile_end) nxt = resolve_group(p, w, t + 1, lane);
      const GroupSrc src = cur;
      cur = nxt;
      const int st = c % STAGES;
      if (!mbar_wait(&empty[st], ((c / STAGES) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
      if (lane == 0) mbar_arrive_expect_tx(&full[st], KvStage<D>::kTensorBytes);
      __syncwarp();
      if (lane_per_group) {
        if (lane < groups) issue_group_one<D>(p, maps, w, lane, src, 0, ring + st * KvStage<D>::kTensorBytes, &full[st], policy);
#ifdef TFA_PROFILE
        if (lane == 0) decode_tile_hook(c, 1);
#endif
      } else {
        for (int g = lane; g < groups; g += 32)
          issue_group_one<D>(p, maps, w, g, resolve_group(p, w, t, g), 0, ring + st * KvStage<D>::kTensorBytes, &full[st],
                             policy);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[slot]);
  }
}

// Producer variant with separate K and V slots: tile t's K goes to slot (2u) % NSLOTS and
// its V to slot (2u + 1) % NSLOTS, u counting tiles, each slot KvStage<D>::kTensorBytes.
// Used by the prefill kernel, which keeps K_t and V_t alive for different lengths of time.
template <int D, int NSLOTS, bool kKOnly = false>
__device__ __forceinline__ void producer_loop_kv_slots(const FwdParams& p, const KvMaps& maps, uint8_t* slots,
                                                       uint64_t* full, uint64_t* empty, uint64_t* item_full,
                                                       uint64_t* item_empty, int* item_slot,
                                                       volatile int* abort_flag, int lane) {
  constexpr int kSlotBytes = KvStage<D>::kTensorBytes;
  const uint64_t policy = l2_policy_evict_first();
  const int groups = kBN / p.box_rows;
  int c = 0;  // slot loads issued
  int claimed = (lane == 0) ? (int)blockIdx.x : 0;
  auto claim = [&]() {
    if (lane == 0) claimed = atomicAdd(&p.sched[0], 1) + (int)gridDim.x;
  };
  for (int k = 0;; ++k) {
    const int slot = k & 1;
    if (!mbar_wait(&item_empty[slot], ((k >> 1) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
    int idx = __shfl_sync(0xffffffffu, claimed, 0);
    Work w;
    while (idx < p.num_items) {
      w = get_work(p, idx);
      if (w.exists) break;
      claim();
      idx = __shfl_sync(0xffffffffu, claimed, 0);
    }
    if (lane == 0) {
      item_slot[slot] = idx;
      mbar_arrive(&item_full[slot]);
    }
    if (idx >= p.num_items) {
      if (lane == 0) scheduler_finish(p);
      return;
    }
    if (w.tile_end == w.tile_begin) claim();
    for (int t = w.tile_begin; t < w.tile_end; ++t) {
      if (t + 1 == w.tile_end) claim();
#pragma unroll 1
      for (int which = 0; which < 2; ++which, ++c) {
        if (kKOnly && which == 1) continue;  // the follower warp loads V into the odd slots
        const int st = c % NSLOTS;
        if (!mbar_wait(&empty[st], ((c / NSLOTS) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
        if (lane == 0) mbar_arrive_expect_tx(&full[st], kSlotBytes);
        __syncwarp();
        const uint32_t base = smem_u32(slots + st * kSlotBytes);
        for (int g = lane; g < groups; g += 32) {
          const GroupSrc src = resolve_group(p, w, t, g);
          if (which == 0)
            issue_group_tensor<D>(p, &maps.k_box, &maps.k_row, w, src, base + g * p.box_rows * 128, &full[st], policy);
          else
            issue_group_tensor<D>(p, &maps.v_box, &maps.v_row, w, src, base + g * p.box_rows * 128, &full[st], policy);
        }
      }
    }
  }
}

// Second producer warp of the prefill kernel: follows the item queue like a consumer and
// issues the V loads of every kv tile (slot 2u + 1 for tile u) while producer_loop_kv_slots
// (with kKOnly) issues the K loads, so two warps share the TMA issue work of a tile.
template <int D, int NSLOTS>
__device__ __forceinline__ void producer_follow_kv_slots(const FwdParams& p, const KvMaps& maps, uint8_t* slots,
                                                         uint64_t* full, uint64_t* empty, uint64_t* item_full,
                                                         uint64_t* item_empty, const int* item_slot,
                                                         volatile int* abort_flag, int lane) {
  constexpr int kSlotBytes = KvStage<D>::kTensorBytes;
  const uint64_t policy = l2_policy_evict_first();
  const int groups = kBN / p.box_rows;
  int c = 1;  // slot load index of the next V
  for (int k = 0;; ++k) {
    const int slot = k & 1;
    if (!mbar_wait(&item_full[slot], (k >> 1) & 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
    const int idx = item_slot[slot];
    if (idx >= p.num_items) return;
    const Work w = get_work(p, idx);
    for (int t = w.tile_begin; t < w.tile_end; ++t, c += 2) {
      const int st = c % NSLOTS;
      if (!mbar_wait(&empty[st], ((c / NSLOTS) & 1) ^ 1, abort_flag, p.err, kDevErrTimeoutProducer)) return;
      if (lane == 0) mbar_arrive_expect_tx(&full[st], kSlotBytes);
      __syncwarp();
      const uint32_t base = smem_u32(slots + st * kSlotBytes);
      for (int g = lane; g < groups; g += 32)
        issue_group_tensor<D>(p, &maps.v_box, &maps.v_row, w, resolve_group(p, w, t, g), base + g * p.box_rows * 128,
                              &full[st], policy);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[slot]);
  }
}


__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Reduces 16 per-lane columns over the 32 lanes of a warp with a transposing butterfly
// (8 + 4 + 2 + 1 + 1 shuffles instead of 16 x 5). On return, lane L holds the total of
// column col16_of_lane(L); v is clobbered.
template <bool kMax>
__device__ __forceinline__ float col16_reduce(float (&v)[16], int lane) {
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int m = 16 >> step;    // lane mask of this step
    const int half = 8 >> step;  // columns kept after it
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = hi ? v[i] : v[i + half];
      const float keep = hi ? v[i + half] : v[i];
      v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, m));
    }
  }
  return op(v[0], __shfl_xor_sync(0xffffffffu, v[0], 1));
}
__device__ __forceinline__ int col16_of_lane(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Device-side launch helpers live in the per-kernel .cu files.
template <int D>
cudaError_t launch_decode(const FwdParams& p, const KvMaps& maps, const CUtensorMap& q_map, int grid, cudaStream_t s,
                          int mode);
template <int D>
cudaError_t launch_prefill(const FwdParams& p, const KvMaps& maps, int grid, cudaStream_t s);
template <int D>
cudaError_t launch_combine(const FwdParams& p, int max_rows, cudaStream_t s);
// Page decode kernel (8 kv heads, 16-slot pages, one q token per sequence): whether a
// shape is supported, its MMA N (q heads per token, padded), and the launch.
bool page_decode_supported(int head_dim, int num_kv_heads, int block_size, int group);
int page_decode_cols(int group);
cudaError_t launch_decode_pages(int head_dim, int group, const FwdParams& p, const KvMaps& maps,
                                const CUtensorMap& q_map, int grid, cudaStream_t s);
cudaError_t launch_item_list(const FwdParams& p, int* list, int* count, cudaStream_t s);
template <int D>
cudaError_t launch_gather(const FwdParams& p, const KvMaps& maps, int max_tiles, const int64_t* kv_offsets,
                          void* k_out, void* v_out, cudaStream_t s);
template <int D>
int decode_smem_bytes();
template <int D>
int prefill_smem_bytes();

}  // namespace tfa
