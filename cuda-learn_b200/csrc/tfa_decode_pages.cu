// Decode over whole pages (one q token per sequence, 8 kv heads, 16-slot pages).
//
// With 8 kv heads and 16 slots a page holds 128 rows of head_dim values, laid out
// [slot][kv head][head_dim] and contiguous in HBM. The per-head decode kernel reads such a
// page as eight 16-row boxes, one per kv head, each from a different CTA: every box is a
// strided 2 KB read, which caps the whole GPU near 4.8-5 TB/s at head_dim 64 (random
// pages). This kernel's work item is (sequence, kv split) over ALL kv heads, and its kv
// tile is one page, fetched as one 16 KB box per 64-column panel through a tensor map
// whose dimensions run (head_dim, slot, kv head, block): the 128 rows land head-major
// (row = head * 16 + slot) in the 128-byte-swizzled layout the MMAs read.
//
//   S^T[128 rows x N] = Kpage[128 x D] . Q^T   (Q: the token's hq heads, N = hq padded to 16)
//   O^T[D x N]        = Vpage^T[D x 128] . P^T (P zero wherever row head != column head)
//
// Softmax thread t owns row t = (head t / 16, slot t % 16). Only its head's G columns
// (the q heads of that kv head) are live, and a column's max and sum reduce over the 16
// lanes of one head inside one warp. P^T is written to shared memory; its cross-head
// entries are zeroed once per launch and never written, so the P.V MMA over all 128 rows
// adds exactly each head's own rows. The un-normalised O^T of each tile is folded into
// registers (thread = head-dim lane, all N columns) with each column's rescale factor,
// broadcast through shared memory (three buffers: a fast warp writing tile j + 1's factors
// cannot overwrite the ones a slow warp still reads for tile j - 1).
//
// Splits use the per-head kernel's split rule per (sequence, head) work group, so the
// split partials are those the combine kernel expects. Rows of a page past kv_len are
// zero-filled (per-row loads on a sequence's partial last page), as in the per-head kernel.
//
// Warp roles (224 threads): 0 = K producer, item scheduler and Q loader, 6 = V producer,
// 1 = MMA issuer and TMEM owner, 2-5 = softmax / epilogue.
#include <cmath>
#include <mutex>

#include "tfa_common.cuh"

namespace tfa {

namespace {

constexpr int kPageRows = 128;  // 16 slots x 8 kv heads
constexpr int kHeadLanes = 16;  // rows (and softmax lanes) per kv head
constexpr int kPageHeads = 8;

template <int D, int G>
struct PageCfg {
  static constexpr int N = (8 * G) < 16 ? 16 : 8 * G;   // MMA N: the token's q heads, padded
  static constexpr int kPanels = D / 64;
  static constexpr int kTileBytes = kPanels * kPageRows * 128;  // one K or V page
  static constexpr int kKSlots = D == 128 ? 3 : 6;
  static constexpr int kVSlots = D == 128 ? 3 : 6;
  // V ring first: at D = 64 the P.V MMA spans M = 128 head-dim rows and its upper 64 rows
  // read the 16 KB after a V tile, which then stays inside this CTA's shared memory.
  static constexpr int kVOff = 0;
  static constexpr int kKOff = kVSlots * kTileBytes;
  static constexpr int kQBytes = kPanels * N * 128;       // Q: N rows x D, K-major SW128
  static constexpr int kPBytes = 2 * N * 128;             // P^T: N rows x 128 page rows
  static constexpr int kQOff = kKOff + kKSlots * kTileBytes;
  static constexpr int kPOff = kQOff + 2 * kQBytes;
  static constexpr int kDynBytes = kPOff + 2 * kPBytes + 1024;
  static constexpr uint32_t kTmemCols = 4 * N <= 64 ? 64 : (4 * N <= 128 ? 128 : 256);  // S^T x2, O^T x2
  static_assert(kDynBytes <= 227 * 1024 - 2048, "shared memory");
};

// Work item idx of the page kernel: split idx / batch of sequence idx % batch. Its page
// range is the split's part of the visible kv range, using the per-head kernel's split of
// work group (sequence, kv head 0); every kv head of a sequence has the same range.
struct PageWork {
  Work w;       // the per-head kernel's item for kv head 0 (kv range, splits, q token)
  int lo, hi;   // visible kv positions of the q token
  int pg_begin, pg_end;  // page tiles of this item
};

__device__ __forceinline__ PageWork page_work(const FwdParams& p, int idx) {
  PageWork pw;
  const int b = idx % p.batch;
  const int split = idx / p.batch;
  pw.w = get_work(p, split * (p.batch * p.hkv) + b * p.hkv);
  pw.lo = 1;
  pw.hi = 0;
  pw.pg_begin = pw.pg_end = 0;
  if (pw.w.exists) {
    visible_range(p, 0, pw.w.q_len, pw.w.kv_len, pw.lo, pw.hi);
    const int t0 = imax(pw.w.tile_begin * kBN, pw.lo);
    const int t1 = imin(pw.w.tile_end * kBN, pw.hi + 1);
    if (t1 > t0) {
      pw.pg_begin = t0 / kHeadLanes;
      pw.pg_end = (t1 + kHeadLanes - 1) / kHeadLanes;
    }
  }
  return pw;
}

// Loads page tile pg of item pw (K or V) into `dst`: one box per panel when the page is
// full, else one row box per (head, slot) with slots past kv_len zero-filled.
template <int D>
__device__ __forceinline__ void load_page(const FwdParams& p, const CUtensorMap* page_map, const CUtensorMap* row_map,
                                          const PageWork& pw, int pg, uint32_t dst, uint64_t* full_bar, int lane,
                                          uint64_t policy) {
  constexpr int kPanels = D / 64;
  int page = __ldg(p.block_table + (int64_t)pw.w.b * p.bt_s0 + pg);
  const int valid = imin(kHeadLanes, pw.w.kv_len - pg * kHeadLanes);
  if (page < 0 || page >= p.num_blocks) {
    if (lane == 0) atomicCAS(p.err, 0, (int)kDevErrBadBlockId);
    page = p.num_blocks;  // whole page out of range -> zeros
  }
  if (valid == kHeadLanes || page == p.num_blocks) {
    if (lane == 0) {
#pragma unroll
      for (int ch = 0; ch < kPanels; ++ch)
        tma_load_4d(dst + ch * (kPageRows * 128), page_map, ch * 64, 0, 0, page, full_bar, policy);
    }
    return;
  }
  // partial page: row (head h, slot s) from the per-row map; slot index 16 is out of range
  for (int rr = lane; rr < kPageRows; rr += 32) {
    const int h = rr / kHeadLanes, s = rr % kHeadLanes;
    const int sl = s < valid ? s : kHeadLanes;
#pragma unroll
    for (int ch = 0; ch < kPanels; ++ch)
      tma_load_4d(dst + ch * (kPageRows * 128) + rr * 128, row_map, ch * 64, h, sl, page, full_bar, policy);
  }
}

template <int D, int G>
__global__ void __launch_bounds__(224, 1)
    decode_page_kernel(const __grid_constant__ FwdParams p, const __grid_constant__ KvMaps maps,
                       const __grid_constant__ CUtensorMap q_map) {
  using Cfg = PageCfg<D, G>;
  constexpr int N = Cfg::N;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* k_ring = smem + Cfg::kKOff;
  uint8_t* v_ring = smem + Cfg::kVOff;
  uint8_t* q_smem = smem + Cfg::kQOff;
  uint8_t* p_smem = smem + Cfg::kPOff;

  __shared__ uint64_t full_k[Cfg::kKSlots], empty_k[Cfg::kKSlots], full_v[Cfg::kVSlots], empty_v[Cfg::kVSlots];
  __shared__ uint64_t s_full[2], s_free[2], p_full[2], o_full[2], o_free[2];
  __shared__ uint64_t item_full[2], item_empty[2], q_full[2], red_bar;
  __shared__ int item_slot[2];
  __shared__ PageWork item_work[2];  // the item's descriptor, published by the K producer
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ uint64_t stall_bar;  // never arrived on: the time-limit test hook waits here
  __shared__ float alpha_sm[3][N];  // per-column rescale factor of a tile (three tiles in flight)
  __shared__ float lsum_sm[2][N], lse_sm[2][N];  // per item parity: column sums and LSEs

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < Cfg::kKSlots; ++i) {
      mbar_init(&full_k[i], 1);
      mbar_init(&empty_k[i], 1);
    }
    for (int i = 0; i < Cfg::kVSlots; ++i) {
      mbar_init(&full_v[i], 1);
      mbar_init(&empty_v[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 6);  // MMA warp, 4 softmax warps, V producer
      mbar_init(&q_full[i], 1);
    }
    mbar_init(&red_bar, 4);
    abort_flag = 0;
    mbar_init(&stall_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.k_page);
    tma_prefetch_desc(&maps.v_page);
    tma_prefetch_desc(&q_map);
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, Cfg::kTmemCols);
  if (warp >= 2 && warp <= 5) {
    // P^T buffers start zeroed: the cross-head and padding entries are never written
    for (int i = tid - 64; i < 2 * Cfg::kPBytes / 16; i += 128)
      reinterpret_cast<uint4*>(p_smem)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid - 64; i < 3 * N; i += 128) alpha_sm[i / N][i % N] = 1.f;  // padding columns stay 1
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  if (tid == 0) allow_dependent_launch();

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------------ producers
    const uint64_t policy = l2_policy_evict_first();
    const bool is_k = warp == 0;
    uint8_t* ring = is_k ? k_ring : v_ring;
    uint64_t* full = is_k ? full_k : full_v;
    uint64_t* empty = is_k ? empty_k : empty_v;
    const int stages = is_k ? Cfg::kKSlots : Cfg::kVSlots;
    const CUtensorMap* pmap = is_k ? &maps.k_page : &maps.v_page;
    const CUtensorMap* rmap = is_k ? &maps.k_row : &maps.v_row;
    int c = 0;
    int claimed = (int)blockIdx.x;  // warp 0: next item index
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      int idx;
      if (is_k) {
        if (!mbar_wait(&item_empty[slot], ((k >> 1) & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutProducer)) break;
        idx = claimed;
        PageWork pw{};
        while (idx < p.num_items) {
          pw = page_work(p, idx);
          if (pw.w.exists) break;
          if (lane == 0) claimed = atomicAdd(&p.sched[0], 1) + (int)gridDim.x;
          idx = __shfl_sync(0xffffffffu, claimed, 0);
        }
        if (lane == 0) {
          item_slot[slot] = idx < p.num_items ? idx : p.num_items;
          if (idx < p.num_items) {
            item_work[slot] = pw;
            mbar_arrive_expect_tx(&q_full[slot], (uint32_t)Cfg::kQBytes);
            const uint32_t qdst = smem_u32(q_smem + slot * Cfg::kQBytes);
#pragma unroll
            for (int ch = 0; ch < Cfg::kPanels; ++ch)
              tma_load_3d(qdst + ch * (N * 128), &q_map, ch * 64, 0, pw.w.q0, &q_full[slot]);
          }
          mbar_arrive(&item_full[slot]);
        }
        if (idx >= p.num_items) {
          if (lane == 0) scheduler_finish(p);
          break;
        }
        // the next item is claimed while the last page of this one waits for its slot
        auto claim = [&]() {
          if (lane == 0) claimed = atomicAdd(&p.sched[0], 1) + (int)gridDim.x;
          claimed = __shfl_sync(0xffffffffu, claimed, 0);
        };
        if (pw.pg_end == pw.pg_begin) claim();
        for (int pg = pw.pg_begin; pg < pw.pg_end; ++pg, ++c) {
          if (pg + 1 == pw.pg_end) claim();
          const int st = c % stages;
          if (!mbar_wait(&empty[st], ((c / stages) & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutProducer)) goto done;
          if (lane == 0) mbar_arrive_expect_tx(&full[st], (uint32_t)Cfg::kTileBytes);
          __syncwarp();
          load_page<D>(p, pmap, rmap, pw, pg, smem_u32(ring + st * Cfg::kTileBytes), &full[st], lane, policy);
        }
      } else {
        if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutProducer)) break;
        idx = item_slot[slot];
        if (idx >= p.num_items) break;
        const PageWork pw = item_work[slot];
        for (int pg = pw.pg_begin; pg < pw.pg_end; ++pg, ++c) {
          const int st = c % stages;
          if (!mbar_wait(&empty[st], ((c / stages) & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutProducer)) goto done;
          if (lane == 0) mbar_arrive_expect_tx(&full[st], (uint32_t)Cfg::kTileBytes);
          __syncwarp();
          load_page<D>(p, pmap, rmap, pw, pg, smem_u32(ring + st * Cfg::kTileBytes), &full[st], lane, policy);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[slot]);
      }
    }
  done:;
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_qk = make_idesc_bf16_f32(128, N, false, false);
    const uint32_t idesc_pv = make_idesc_bf16_f32(128, N, true, false);
    int c = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      const int idx = item_slot[slot];
      if (idx >= p.num_items) break;
      const PageWork pw = item_work[slot];
      if (p.debug_stall && k == 0 && !mbar_wait(&stall_bar, 0, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      const int n = pw.pg_end - pw.pg_begin;
      const uint32_t q_addr = smem_u32(q_smem + slot * Cfg::kQBytes);
      if (!mbar_wait(&q_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      if (lane == 0 && n > 0) {
        auto issue_qk = [&](int cc) {
          const int st = cc % Cfg::kKSlots;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(k_ring + st * Cfg::kTileBytes);
          const uint32_t d_tmem = tmem + (cc & 1) * N;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kPageRows * 128) + (kk & 3) * 32;
            const uint32_t qoff = (kk >> 2) * (N * 128) + (kk & 3) * 32;
            umma_bf16_ss(d_tmem, make_sdesc_sw128(k_addr + off, 16, 1024), make_sdesc_sw128(q_addr + qoff, 16, 1024),
                         idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty_k[st]);
          umma_commit(&s_full[cc & 1]);
        };
        auto issue_pv = [&](int cj) {
          tc_fence_after();
          const int st = cj % Cfg::kVSlots;
          const uint32_t v_addr = smem_u32(v_ring + st * Cfg::kTileBytes);
          const uint32_t pb = smem_u32(p_smem + (cj & 1) * Cfg::kPBytes);
          const uint32_t d_tmem = tmem + 2 * N + (cj & 1) * N;
#pragma unroll
          for (int kk = 0; kk < kPageRows / 16; ++kk) {
            const uint32_t voff = kk * 2048;
            const uint32_t poff = (kk >> 2) * (N * 128) + (kk & 3) * 32;
            umma_bf16_ss(d_tmem, make_sdesc_sw128(v_addr + voff, kPageRows * 128, 1024),
                         make_sdesc_sw128(pb + poff, 16, 1024), idesc_pv, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty_v[st]);
          umma_commit(&o_full[cj & 1]);
        };
        // QK of tile jq and P.V of tile jp as soon as each one's inputs are ready; QK runs
        // at most two tiles ahead (two S buffers).
        int jq = 0, jp = 0;
        uint32_t idle = 0;
        uint64_t t0 = 0;
        while (jp < n) {
          bool progress = false;
          if (jq < n && jq < jp + 2) {
            const int cq = c + jq;
            if (mbar_test(&full_k[cq % Cfg::kKSlots], (cq / Cfg::kKSlots) & 1) &&
                mbar_test(&s_free[cq & 1], ((cq >> 1) & 1) ^ 1)) {
              issue_qk(cq);
              ++jq;
              progress = true;
            }
          }
          if (jp < jq) {
            const int cp = c + jp;
            if (mbar_test(&p_full[cp & 1], (cp >> 1) & 1) && mbar_test(&o_free[cp & 1], ((cp >> 1) & 1) ^ 1) &&
                mbar_test(&full_v[cp % Cfg::kVSlots], (cp / Cfg::kVSlots) & 1)) {
              issue_pv(cp);
              ++jp;
              progress = true;
            }
          }
          if (progress) {
            idle = 0;
            continue;
          }
          if (idle++ == 0) {
            t0 = global_timer_ns();
          } else if ((idle & 63u) == 0) {
            if (abort_flag) {
              ok = false;
              break;
            }
            if (global_timer_ns() - t0 > kWaitLimitNs) {
              abort_flag = 1;
              atomicCAS(p.err, 0, kDevErrTimeoutMma);
              ok = false;
              break;
            }
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      c += n;
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int quad = warp & 3;           // TMEM lane quadrant
    const int tl = quad * 32 + lane;     // page row (softmax) and head-dim lane (epilogue)
    const int hh = tl / kHeadLanes;      // kv head of this row
    const int s_in_page = tl % kHeadLanes;
    const int hi_half = lane >> 4;       // the warp's second kv head
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const int col_w = (quad * 2) * G;    // the warp's first live column
    int c = 0, bp = 0, at = 0;
    auto sm_sync = [&]() -> bool {  // the four softmax warps (bounded)
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_bar);
      const bool r = mbar_wait(&red_bar, bp & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax);
      ++bp;
      return r;
    };
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) break;
      const int idx = item_slot[slot];
      if (idx >= p.num_items) break;
      const PageWork pw = item_work[slot];
      const int n = pw.pg_end - pw.pg_begin;
      const int tok = pw.w.q0;
      float m[G], l[G], a_prev[N], o[N];
#pragma unroll
      for (int q = 0; q < G; ++q) {
        m[q] = -INFINITY;
        l[q] = 0.f;
      }
#pragma unroll
      for (int q = 0; q < N; ++q) {
        o[q] = 0.f;
        a_prev[q] = 1.f;
      }
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        const int cj = c + j;
        if (!mbar_wait(&s_full[cj & 1], (cj >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[16];
        tmem_ld16(lane_base + (cj & 1) * N + col_w, sv);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[cj & 1]);
        const int pos = (pw.pg_begin + j) * kHeadLanes + s_in_page;
        const bool vis = pos >= pw.lo && pos <= pw.hi;
        float a[G];
        uint8_t* pb = p_smem + (cj & 1) * Cfg::kPBytes + (tl >> 6) * (N * 128);
        const int cu = (tl & 63) >> 3, ce = (tl & 7) * 2;
#pragma unroll
        for (int q = 0; q < G; ++q) {
          const float v = hi_half ? sv[G + q] : sv[q];
          const float sc = vis ? v * p.scale_log2 : -INFINITY;
          float mx = sc;
#pragma unroll
          for (int o2 = 1; o2 < kHeadLanes; o2 <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
          const float mn = fmaxf(m[q], mx);
          a[q] = (m[q] == -INFINITY) ? 1.f : ex2_approx(m[q] - mn);
          const float pv = ex2_approx(sc - ((mn == -INFINITY) ? 0.f : mn));
          l[q] = l[q] * a[q] + pv;
          m[q] = mn;
          // P^T row n = hh * G + q (its q head), column tl (page row), K-major SW128
          const int nrow = hh * G + q;
          *reinterpret_cast<__nv_bfloat16*>(pb + nrow * 128 + ((cu ^ (nrow & 7)) << 4) + ce) = __float2bfloat16(pv);
          if (s_in_page == 0) alpha_sm[at][nrow] = a[q];
        }
        fence_proxy_async_smem();
        if (!sm_sync()) {  // factors of this tile published; P of all four warps written
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive(&p_full[cj & 1]);
        // fold the previous tile's P.V (thread = head-dim lane, every column)
        if (j > 0) {
          const int cp = cj - 1;
          if (!mbar_wait(&o_full[cp & 1], (cp >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
          float ot[N];
          if constexpr (N == 16) {
            tmem_ld16(lane_base + 2 * N + (cp & 1) * N, ot);
          } else {
#pragma unroll
            for (int h32 = 0; h32 < N / 32; ++h32) {
              float t32[32];
              tmem_ld32(lane_base + 2 * N + (cp & 1) * N + h32 * 32, t32);
#pragma unroll
              for (int i = 0; i < 32; ++i) ot[h32 * 32 + i] = t32[i];
            }
          }
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[cp & 1]);
#pragma unroll
          for (int q = 0; q < N; ++q) o[q] = o[q] * a_prev[q] + ot[q];
        }
#pragma unroll
        for (int q = 0; q < N; ++q) a_prev[q] = alpha_sm[at][q];
        at = at == 2 ? 0 : at + 1;
      }
      if (ok && n > 0) {
        const int cl = c + n - 1;
        if (!mbar_wait(&o_full[cl & 1], (cl >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
          ok = false;
        } else {
          tc_fence_after();
          float ot[N];
          if constexpr (N == 16) {
            tmem_ld16(lane_base + 2 * N + (cl & 1) * N, ot);
          } else {
#pragma unroll
            for (int h32 = 0; h32 < N / 32; ++h32) {
              float t32[32];
              tmem_ld32(lane_base + 2 * N + (cl & 1) * N + h32 * 32, t32);
#pragma unroll
              for (int i = 0; i < 32; ++i) ot[h32 * 32 + i] = t32[i];
            }
          }
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[cl & 1]);
#pragma unroll
          for (int q = 0; q < N; ++q) o[q] = o[q] * a_prev[q] + ot[q];
        }
      }
      if (!ok) break;
      c += n;
      // column sums over the head's 16 lanes; slot-0 lanes publish sum and LSE (log2)
#pragma unroll
      for (int q = 0; q < G; ++q) {
        float sm = l[q];
#pragma unroll
        for (int o2 = 1; o2 < kHeadLanes; o2 <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o2);
        if (s_in_page == 0) {
          lsum_sm[k & 1][hh * G + q] = sm;
          lse_sm[k & 1][hh * G + q] = sm > 0.f ? m[q] + lg2_approx(sm) : -INFINITY;
        }
      }
      if (!sm_sync()) break;
      const bool direct = (pw.w.nsplits == 1);
      if (tl < D) {
#pragma unroll
        for (int q = 0; q < N; ++q) {
          if (q >= p.hq) break;
          const float ls = lsum_sm[k & 1][q];
          const float inv = ls > 0.f ? __frcp_rn(ls) : 0.f;
          if (direct) {
            p.out[(int64_t)tok * p.o_s0 + (int64_t)q * p.o_s1 + tl] = __float2bfloat16(o[q] * inv);
          } else {
            p.split_o[(((int64_t)pw.w.split * p.total_q + tok) * p.hq + q) * D + tl] = o[q] * inv;
          }
        }
      }
      if (tl < p.hq) {
        if (direct) {
          if (p.lse) p.lse[(int64_t)tok * p.hq + tl] = lse_sm[k & 1][tl] * kLn2;
        } else {
          p.split_lse[((int64_t)pw.w.split * p.total_q + tok) * p.hq + tl] = lse_sm[k & 1][tl];
        }
      }
      // buffers of item parity k & 1 are written again only by item k + 2, after the
      // epilogue sm_sync of item k + 1, which every thread reaches after this epilogue
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
    }
  }

  if (abort_flag && (warp == 0 || warp == 6)) {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int D, int G>
cudaError_t launch_one(const FwdParams& p, const KvMaps& maps, const CUtensorMap& q_map, int grid, cudaStream_t s) {
  static bool configured[128] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(decode_page_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, PageCfg<D, G>::kDynBytes);
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
  }
  decode_page_kernel<D, G><<<grid, 224, PageCfg<D, G>::kDynBytes, s>>>(p, maps, q_map);
  return cudaGetLastError();
}

}  // namespace

bool page_decode_supported(int head_dim, int num_kv_heads, int block_size, int group) {
  if (num_kv_heads != kPageHeads || block_size != kHeadLanes) return false;
  return (group == 1 || group == 2 || group == 4) && (head_dim == 64 || head_dim == 128);
}

int page_decode_cols(int group) { return 8 * group < 16 ? 16 : 8 * group; }

cudaError_t launch_decode_pages(int head_dim, int group, const FwdParams& p, const KvMaps& maps,
                                const CUtensorMap& q_map, int grid, cudaStream_t s) {
  if (head_dim == 64) {
    switch (group) {
      case 1: return launch_one<64, 1>(p, maps, q_map, grid, s);
      case 2: return launch_one<64, 2>(p, maps, q_map, grid, s);
      case 4: return launch_one<64, 4>(p, maps, q_map, grid, s);
    }
  } else if (head_dim == 128) {
    switch (group) {
      case 1: return launch_one<128, 1>(p, maps, q_map, grid, s);
      case 2: return launch_one<128, 2>(p, maps, q_map, grid, s);
      case 4: return launch_one<128, 4>(p, maps, q_map, grid, s);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace tfa
