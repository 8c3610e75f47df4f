// Decode-shaped paged attention (q_len * group <= 16 packed rows per kv head).
//
// One work item = (sequence b, kv head h, kv split). All q heads of the GQA group (and
// all q tokens of the sequence, for short speculative chunks) are packed into N <= 16
// columns, so every K/V byte is read from HBM once per kv head. The contractions run on
// tcgen05 with the kv tile on the M axis:
//   S^T[128 tok x 16] = K[128 tok x D] . Q^T            (A = K tile, K-major; B = Q, K-major)
//   O^T[D x 16]      = V^T[D x 128 tok] . P^T           (A = V tile, MN-major; B = P, K-major)
// Both accumulate in TMEM. Softmax threads own one kv token (TMEM lane) each, reduce the
// per-column max across the 128 tokens with warp shuffles plus a 4-warp exchange, and
// write P^T back to shared memory for the second MMA. The un-normalised output of each
// tile is folded into registers (thread = head-dim lane) with the running rescale.
//
// Warp roles (224 threads): warp 0 = TMA producer of K (and the item scheduler), warp 6 =
// TMA producer of V, warp 1 = MMA issuer + TMEM owner, warps 2-5 = softmax / epilogue.
// Producer warp 0 also publishes each item's descriptor in shared memory and loads its Q
// rows by TMA into a per-item-slot buffer, ahead of time: an item boundary then costs no
// global-memory round trip on the consumer side.
#include <cmath>
#include <mutex>

#include "tfa_common.cuh"

#ifndef TFA_DECODE_KSLOTS
#define TFA_DECODE_KSLOTS 3
#endif
#ifndef TFA_DECODE_VSLOTS
#define TFA_DECODE_VSLOTS 3
#endif

namespace tfa {

namespace {

constexpr int kNP = 16;  // packed q rows (MMA N)

#ifdef TFA_PROFILE
__device__ unsigned long long g_decode_stamp[32];
__device__ unsigned long long g_decode_tile[16][12];
__device__ unsigned long long g_decode_end[512];
__device__ unsigned long long g_decode_begin[512];
__device__ int g_decode_ntiles[512];
#define STAMP(i) do { if (blockIdx.x == 0) g_decode_stamp[i] = global_timer_ns(); } while (0)
#define PH(cj, i) do { if (blockIdx.x == 0 && (cj) < 16) g_decode_tile[cj][i] = global_timer_ns(); } while (0)
}  // namespace
__device__ void decode_stamp_hook(int i) { g_decode_stamp[i] = global_timer_ns(); }
__device__ void decode_tile_hook(int c, int i) { if (blockIdx.x == 0 && c < 16) g_decode_tile[c][i] = global_timer_ns(); }
namespace {
#else
#define STAMP(i) do {} while (0)
#define PH(cj, i) do {} while (0)
#endif

template <int D>
struct DecodeCfg {
  static constexpr int kPanels = D / 64;
  // K and V tiles live in separate rings: a K slot is released as soon as QK has read
  // it, a V slot only after the tile's softmax and P.V, so the V ring holds its tiles longer
  static constexpr int kKSlots = (D == 128) ? TFA_DECODE_KSLOTS : 6;
  static constexpr int kVSlots = (D == 128) ? TFA_DECODE_VSLOTS : 6;
  static constexpr int kTileBytes = KvStage<D>::kTensorBytes;  // one K or V tile
  // V ring first: the P.V MMA always spans M = 128 head-dim rows, so for D = 64 its upper
  // 64 rows read the 16 KB after the V tile (their output rows are never used). With the
  // V ring first that read stays inside this CTA's shared memory (next V slot / K ring).
  static constexpr int kVOff = 0;
  static constexpr int kKOff = kVSlots * kTileBytes;
  static constexpr int kQBytes = kPanels * kNP * 128;  // Q: kNP rows x D, K-major SW128 panels
  static constexpr int kPBytes = 2 * kNP * 128;        // P^T: kNP rows x 128 tokens (2 panels)
  static constexpr int kQOff = kKOff + kKSlots * kTileBytes;  // two Q buffers (one per item slot)
  static constexpr int kPOff = kQOff + 2 * kQBytes;      // two P buffers
  static constexpr int kDynBytes = kPOff + 2 * kPBytes + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = 64;              // S^T x2 (16 cols), O^T x2 (16 cols)
};

// Merges the split partials of work group w (all of its splits have finished and
// published their rows) into `out` and the LSE: out = sum_s 2^(lse_s - M) o_s / sum_s
// 2^(lse_s - M), M = max_s lse_s (the LSE merge of v8/flash_attn_func.cu:701-777, in an
// online form over chunks of eight splits). Run by the 128 softmax threads of the CTA
// whose split finished last: D / 4 threads per row, four columns each, so a pass covers
// 512 / D rows; every load of a chunk is issued before any is used (one L2 round trip
// per chunk). Partials are read with L1-bypassing loads (other CTAs wrote them).
template <int D>
__device__ __forceinline__ void merge_splits(const FwdParams& p, const Work& w, int tq) {
  constexpr int kTpr = D / 4;        // threads per row
  constexpr int kRpp = 128 / kTpr;   // rows per pass
  constexpr int kChunk = 8;
  const int64_t stride = (int64_t)p.total_q * p.hq;
  const int c4 = (tq % kTpr) * 4;
  const int ns = w.nsplits;
  for (int r = tq / kTpr; r < w.nrows; r += kRpp) {
    const int R = w.row0 + r;
    const int tok = w.q0 + R / p.group;
    const int qh = w.h * p.group + R % p.group;
    const int64_t pair = (int64_t)tok * p.hq + qh;
    float mx = -INFINITY, wsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < ns; s0 += kChunk) {
      float ls[kChunk];
      float4 ov[kChunk];
#pragma unroll
      for (int i = 0; i < kChunk; ++i) {
        const int s = s0 + i;
        if (s < ns) {
          ls[i] = __ldcg(p.split_lse + s * stride + pair);
          ov[i] = __ldcg(reinterpret_cast<const float4*>(p.split_o + (s * stride + pair) * D + c4));
        } else {
          ls[i] = -INFINITY;
          ov[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float cm = mx;
#pragma unroll
      for (int i = 0; i < kChunk; ++i) cm = fmaxf(cm, ls[i]);
      if (cm == -INFINITY) continue;
      const float sc = (mx == -INFINITY) ? 0.f : ex2_approx(mx - cm);
      wsum *= sc;
      acc.x *= sc;
      acc.y *= sc;
      acc.z *= sc;
      acc.w *= sc;
#pragma unroll
      for (int i = 0; i < kChunk; ++i) {
        const float wl = (ls[i] == -INFINITY) ? 0.f : ex2_approx(ls[i] - cm);
        wsum += wl;
        acc.x += wl * ov[i].x;
        acc.y += wl * ov[i].y;
        acc.z += wl * ov[i].z;
        acc.w += wl * ov[i].w;
      }
      mx = cm;
    }
    const float inv = (mx == -INFINITY) ? 0.f : 1.f / wsum;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p.out + (int64_t)tok * p.o_s0 + (int64_t)qh * p.o_s1 + c4) = packed;
    if (c4 == 0 && p.lse) p.lse[pair] = (mx == -INFINITY) ? -INFINITY : (mx + lg2_approx(wsum)) * kLn2;
  }
}

// kMode: 0 = items in slot order, split partials (if any) merged by the combine kernel;
// 1 = items from the device-built list (the only instance that reads it), combine kernel;
// 2 = items in slot order, split partials merged inside this kernel by the last split of
// each group (the only instance that touches the per-group counters).
template <int D, int kMode>
__global__ void __launch_bounds__(224, 1)
    decode_kernel(const __grid_constant__ FwdParams p, const __grid_constant__ KvMaps maps,
                  const __grid_constant__ CUtensorMap q_map) {
  using Cfg = DecodeCfg<D>;
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
  __shared__ Work item_work[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ uint64_t stall_bar;  // never arrived on: the time-limit test hook waits here
  __shared__ __align__(16) float red_max[2][4][kNP];
  __shared__ __align__(16) float red_sum[2][4][kNP];
  __shared__ int merge_flag[2];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (tid == 0) STAMP(0);
#ifdef TFA_PROFILE
  const unsigned long long t_begin_prof = global_timer_ns();
#endif
  if constexpr (kMode != 1) {
    // The first item of this CTA is item blockIdx.x: bring its sequence's lengths and the
    // start of its block-table row into L2 while the CTA sets up (the producer's first
    // loads then hit L2 instead of waiting a DRAM round trip after the prologue).
    if (warp == 0 && lane < 3) {
      const int b = (int)((blockIdx.x / (unsigned)p.hkv) % (unsigned)p.batch);
      const void* a = lane == 0 ? (const void*)(p.cu_seqlens_q + b)
                    : lane == 1 ? (const void*)(p.seqused_k + b) : (const void*)(p.block_table + (int64_t)b * p.bt_s0);
      prefetch_l2(a);
    }
    // warp 6 (the V producer, idle until the first item is published) brings the rest of
    // that sequence's block-table row into L2: a split's or a window's first page lies
    // anywhere in it
    if (warp == 6) {
      const int b = (int)((blockIdx.x / (unsigned)p.hkv) % (unsigned)p.batch);
      const int64_t pages = p.max_seqlen_k_pages;
      for (int64_t i = 32 * (1 + lane); i < pages && i < 32 * 64; i += 32 * 32)
        prefetch_l2(p.block_table + (int64_t)b * p.bt_s0 + i);
    }
  }

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
      mbar_init(&item_empty[i], 6);
      mbar_init(&q_full[i], 1);
    }
    mbar_init(&red_bar, 4);
    abort_flag = 0;
    mbar_init(&stall_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.k_box);
    tma_prefetch_desc(&maps.v_box);
    tma_prefetch_desc(&q_map);
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  if (tid == 0) allow_dependent_launch();
  if (tid == 0) STAMP(1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    producer_loop<D, Cfg::kKSlots, kMode == 1>(p, maps, k_ring, full_k, empty_k, item_full, item_empty, item_slot, item_work, &q_map,
                                   q_smem, Cfg::kQBytes, q_full, &abort_flag, lane);
  } else if (warp == 6) {
    producer_follow_v<D, Cfg::kVSlots>(p, maps, v_ring, full_v, empty_v, item_full, item_empty, item_slot, item_work,
                                       &abort_flag, lane);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_qk = make_idesc_bf16_f32(128, kNP, false, false);
    const uint32_t idesc_pv = make_idesc_bf16_f32(128, kNP, true, false);
    int c = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      const int idx = item_slot[slot];
      if (idx >= p.num_items) break;
      const Work w = item_work[slot];
      // Test hook (FwdParams::debug_stall): wait for a phase that never completes, so the
      // time limit expires, the error word is set and every warp of the CTA unwinds.
      if (p.debug_stall && k == 0 && !mbar_wait(&stall_bar, 0, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      const int n = w.tile_end - w.tile_begin;
      const uint32_t q_addr = smem_u32(q_smem + slot * Cfg::kQBytes);
      if (!mbar_wait(&q_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      if (lane == 0 && k == 0) STAMP(4);
      if (lane == 0 && n > 0) {
        auto issue_qk = [&](int cc) {
          const int st = cc % Cfg::kKSlots;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(k_ring + st * Cfg::kTileBytes);
          const uint32_t d_tmem = tmem + (cc & 1) * kNP;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * KvStage<D>::kPanelBytes + (kk & 3) * 32;
            const uint32_t qoff = (kk >> 2) * (kNP * 128) + (kk & 3) * 32;
            umma_bf16_ss(d_tmem, make_sdesc_sw128(k_addr + off, 16, 1024), make_sdesc_sw128(q_addr + qoff, 16, 1024),
                         idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty_k[st]);  // frees the K slot once QK has read it
          umma_commit(&s_full[cc & 1]);
          PH(cc, 2);
        };
        auto issue_pv = [&](int cj) {
          tc_fence_after();
          const int st = cj % Cfg::kVSlots;
          const uint32_t v_addr = smem_u32(v_ring + st * Cfg::kTileBytes);
          const uint32_t pb = smem_u32(p_smem + (cj & 1) * Cfg::kPBytes);
          const uint32_t d_tmem = tmem + 32 + (cj & 1) * kNP;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint32_t voff = kk * 2048;
            const uint32_t poff = (kk >> 2) * (kNP * 128) + (kk & 3) * 32;
            umma_bf16_ss(d_tmem, make_sdesc_sw128(v_addr + voff, KvStage<D>::kPanelBytes, 1024),
                         make_sdesc_sw128(pb + poff, 16, 1024), idesc_pv, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty_v[st]);  // frees the V slot once this P.V has read it
          umma_commit(&o_full[cj & 1]);
          PH(cj, 3);
        };
        // QK of tile jq and P.V of tile jp are issued as soon as each one's inputs are
        // ready, in whichever order that happens: a P.V (which frees its stage) never
        // waits behind the next tile's K/V arrival, so all stages stay in flight while
        // the kernel is bound by HBM. QK runs at most two tiles ahead (two S buffers).
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
          // bounded: same wall-clock limit and abort protocol as mbar_wait
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
    const int sw = warp - 2;                // 0..3 among the softmax warps
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int tl = quad * 32 + lane;        // TMEM lane: kv token within tile / head-dim index
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const int tq = sw * 32 + lane;          // 0..127 softmax thread index
    int c = 0, bp = 0;
    // Exchange barrier among the four softmax warps (bounded, unlike bar.sync).
    auto sm_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_bar);
      const bool r = mbar_wait(&red_bar, bp & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax);
      ++bp;
      return r;
    };
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) break;
      if (warp == 2 && lane == 0 && k == 0) STAMP(6);
      const int idx = item_slot[slot];
      if (idx >= p.num_items) break;
      const Work w = item_work[slot];
      const int n = w.tile_end - w.tile_begin;

      // Per-row constants, computed by lane r for row r and broadcast: visible kv range,
      // and where the row's output goes.
      int lo_l = 1, hi_l = 0, tok_l = 0, qh_l = 0;
      if (lane < w.nrows) {
        const int R = w.row0 + lane;
        tok_l = R / p.group;
        qh_l = w.h * p.group + (R - tok_l * p.group);
        visible_range(p, tok_l, w.q_len, w.kv_len, lo_l, hi_l);
        tok_l += w.q0;
      }
      int lo[kNP], hi[kNP];
#pragma unroll
      for (int r = 0; r < kNP; ++r) {
        lo[r] = __shfl_sync(0xffffffffu, lo_l, r);
        hi[r] = __shfl_sync(0xffffffffu, hi_l, r);
      }
      float m[kNP], l[kNP], o[kNP], a_prev[kNP];
#pragma unroll
      for (int r = 0; r < kNP; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
        o[r] = 0.f;
        a_prev[r] = 1.f;
      }
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        const int cj = c + j;
        if (!mbar_wait(&s_full[cj & 1], (cj >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (warp == 2 && lane == 0 && cj == 0) STAMP(8);
        if (warp == 2 && lane == 0) PH(cj, 4);
        float s[kNP];
        tmem_ld16(lane_base + (cj & 1) * kNP, s);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[cj & 1]);
        if (warp == 2 && lane == 0) PH(cj, 5);

        const int pos = (w.tile_begin + j) * kBN + tl;
        float a[kNP];
#pragma unroll
        for (int r = 0; r < kNP; ++r) s[r] = (pos >= lo[r] && pos <= hi[r]) ? s[r] * p.scale_log2 : -INFINITY;
        {
          float t[kNP];
#pragma unroll
          for (int r = 0; r < kNP; ++r) t[r] = s[r];
          const float wm = col16_reduce<true>(t, lane);
          if ((lane & 1) == 0) red_max[cj & 1][sw][col16_of_lane(lane)] = wm;
        }
        if (warp == 2 && lane == 0) PH(cj, 6);
        if (!sm_sync()) {
          ok = false;
          break;
        }
        if (warp == 2 && lane == 0) PH(cj, 7);
        float cmax[kNP];
#pragma unroll
        for (int q4 = 0; q4 < kNP / 4; ++q4) {
          float4 a0 = *reinterpret_cast<const float4*>(&red_max[cj & 1][0][q4 * 4]);
          float4 a1 = *reinterpret_cast<const float4*>(&red_max[cj & 1][1][q4 * 4]);
          float4 a2 = *reinterpret_cast<const float4*>(&red_max[cj & 1][2][q4 * 4]);
          float4 a3 = *reinterpret_cast<const float4*>(&red_max[cj & 1][3][q4 * 4]);
          cmax[q4 * 4 + 0] = fmaxf(fmaxf(a0.x, a1.x), fmaxf(a2.x, a3.x));
          cmax[q4 * 4 + 1] = fmaxf(fmaxf(a0.y, a1.y), fmaxf(a2.y, a3.y));
          cmax[q4 * 4 + 2] = fmaxf(fmaxf(a0.z, a1.z), fmaxf(a2.z, a3.z));
          cmax[q4 * 4 + 3] = fmaxf(fmaxf(a0.w, a1.w), fmaxf(a2.w, a3.w));
        }
#pragma unroll
        for (int r = 0; r < kNP; ++r) {
          const float tmax = cmax[r];
          const float mn = fmaxf(m[r], tmax);
          a[r] = (m[r] == -INFINITY) ? 1.f : ex2_approx(m[r] - mn);
          const float ms = (mn == -INFINITY) ? 0.f : mn;
          s[r] = ex2_approx(s[r] - ms);
          l[r] = l[r] * a[r] + s[r];
          m[r] = mn;
        }
        if (warp == 2 && lane == 0) PH(cj, 8);
        // fold the previous tile's P.V into the register accumulator
        if (j > 0) {
          const int cp = cj - 1;
          if (!mbar_wait(&o_full[cp & 1], (cp >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
            ok = false;
            break;
          }
          if (warp == 2 && lane == 0) PH(cj, 9);
          tc_fence_after();
          float ot[kNP];
          tmem_ld16(lane_base + 32 + (cp & 1) * kNP, ot);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[cp & 1]);
#pragma unroll
          for (int r = 0; r < kNP; ++r) o[r] = o[r] * a_prev[r] + ot[r];
        }
        if (warp == 2 && lane == 0) PH(cj, 10);
#pragma unroll
        for (int r = 0; r < kNP; ++r) a_prev[r] = a[r];
        // P^T -> shared memory: row r (q row), column tl (kv token), K-major SW128.
        uint8_t* pb = p_smem + (cj & 1) * Cfg::kPBytes + (tl >> 6) * (kNP * 128);
        const int cu = (tl & 63) >> 3, ce = (tl & 7) * 2;
#pragma unroll
        for (int r = 0; r < kNP; ++r)
          *reinterpret_cast<__nv_bfloat16*>(pb + r * 128 + ((cu ^ (r & 7)) << 4) + ce) = __float2bfloat16(s[r]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[cj & 1]);
        if (warp == 2 && lane == 0 && cj == 0) STAMP(9);
        if (warp == 2 && lane == 0) PH(cj, 11);
      }
      if (ok && n > 0) {
        const int cl = c + n - 1;
        if (!mbar_wait(&o_full[cl & 1], (cl >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
          ok = false;
        } else {
          tc_fence_after();
          float ot[kNP];
          tmem_ld16(lane_base + 32 + (cl & 1) * kNP, ot);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[cl & 1]);
#pragma unroll
          for (int r = 0; r < kNP; ++r) o[r] = o[r] * a_prev[r] + ot[r];
        }
      }
      if (!ok) break;
      if (warp == 2 && lane == 0 && k == 0) STAMP(10);
      c += n;

      // column sums of the per-token partial denominators
      {
        float t[kNP];
#pragma unroll
        for (int r = 0; r < kNP; ++r) t[r] = l[r];
        const float ws = col16_reduce<false>(t, lane);
        if ((lane & 1) == 0) red_sum[k & 1][sw][col16_of_lane(lane)] = ws;
      }
      if (warp == 2 && lane == 0 && k == 0) STAMP(15);
      if (!sm_sync()) break;
      if (warp == 2 && lane == 0 && k == 0) STAMP(16);
      const bool direct = (w.nsplits == 1);
      // lane r: normaliser, LSE and destination of row r
      float inv_l = 0.f;
      int64_t dst_l = 0;
      if (lane < w.nrows) {
        const float lsum = red_sum[k & 1][0][lane] + red_sum[k & 1][1][lane] + red_sum[k & 1][2][lane] +
                           red_sum[k & 1][3][lane];
        inv_l = lsum > 0.f ? __frcp_rn(lsum) : 0.f;
        dst_l = direct ? (int64_t)tok_l * p.o_s0 + (int64_t)qh_l * p.o_s1
                       : (((int64_t)w.split * p.total_q + tok_l) * p.hq + qh_l);
        if (sw == 0) {
          // m[] is replicated in every thread; this lane needs m[lane]
          float ml = -INFINITY;
#pragma unroll
          for (int r = 0; r < kNP; ++r) ml = (r == lane) ? m[r] : ml;
          const float lse2 = lsum > 0.f ? ml + lg2_approx(lsum) : -INFINITY;
          if (direct) {
            if (p.lse) p.lse[(int64_t)tok_l * p.hq + qh_l] = lse2 * kLn2;
          } else {
            p.split_lse[dst_l] = lse2;
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kNP; ++r) {
        if (r >= w.nrows) break;
        const float inv = __shfl_sync(0xffffffffu, inv_l, r);
        const int64_t dst = __shfl_sync(0xffffffffu, dst_l, r);
        if (tl < D) {
          if (direct) p.out[dst + tl] = __float2bfloat16(o[r] * inv);
          else p.split_o[dst * D + tl] = o[r] * inv;
        }
        if (warp == 2 && lane == 0 && k == 0 && r == 0) STAMP(17);
      }
      if (kMode == 2 && !direct) {
        // Split combine inside the kernel: every split publishes its rows, then counts
        // itself done for the group; the split that completes the count merges them all
        // (and resets the count for the next launch).
        __threadfence();
        if (!sm_sync()) break;
        if (sw == 0 && lane == 0) {
          const int done = atomicAdd(&p.group_cnt[w.g], 1);
          const int last = done == w.nsplits - 1 ? 1 : 0;
          if (last) {
            atomicExch(&p.group_cnt[w.g], 0);
            __threadfence();
          }
          merge_flag[k & 1] = last;
        }
        if (!sm_sync()) break;
        if (merge_flag[k & 1]) merge_splits<D>(p, w, tq);
      }
      __syncwarp();
      if (warp == 2 && lane == 0 && k == 0) STAMP(11);
      if (lane == 0) mbar_arrive(&item_empty[slot]);
    }
    if (warp == 2 && lane == 0) STAMP(12);
#ifdef TFA_PROFILE
    if (warp == 2 && lane == 0 && blockIdx.x < 512) g_decode_ntiles[blockIdx.x] = c;
#endif
  }

  if (abort_flag && (warp == 0 || warp == 6)) {
    // Let TMA copies that may still be in flight land before the CTA's shared memory
    // is released (bounded: 100 us).
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) STAMP(13);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (tid == 0) STAMP(14);
#ifdef TFA_PROFILE
  if (tid == 0 && blockIdx.x < 512) g_decode_end[blockIdx.x] = global_timer_ns();
  if (tid == 0 && blockIdx.x < 512) g_decode_begin[blockIdx.x] = t_begin_prof;
#endif
}

}  // namespace

template <int D>
int decode_smem_bytes() {
  return DecodeCfg<D>::kDynBytes;
}

template <int D>
cudaError_t launch_decode(const FwdParams& p, const KvMaps& maps, const CUtensorMap& q_map, int grid, cudaStream_t s,
                          int mode) {
  static bool configured[128][3] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128 || mode < 0 || mode > 2) return cudaErrorInvalidValue;
  auto kernel = mode == 0 ? decode_kernel<D, 0> : mode == 1 ? decode_kernel<D, 1> : decode_kernel<D, 2>;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev][mode]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeCfg<D>::kDynBytes);
      if (e != cudaSuccess) return e;
      configured[dev][mode] = true;
    }
  }
  if (mode == 1) {
    // after the item-list kernel, as its programmatic dependent (the list is read only after
    // griddepcontrol.wait in the producer)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(224);
    cfg.dynamicSmemBytes = DecodeCfg<D>::kDynBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p, maps, q_map);
  }
  kernel<<<grid, 224, DecodeCfg<D>::kDynBytes, s>>>(p, maps, q_map);
  return cudaGetLastError();
}

#ifdef TFA_PROFILE
extern "C" __attribute__((visibility("default"))) int tfa_decode_stamps_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, g_decode_stamp, sizeof(g_decode_stamp));
}
extern "C" __attribute__((visibility("default"))) int tfa_decode_tiles_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, g_decode_tile, sizeof(g_decode_tile));
}
extern "C" __attribute__((visibility("default"))) int tfa_decode_cta_read(unsigned long long* b, unsigned long long* e, int* n) {
  cudaMemcpyFromSymbol(b, g_decode_begin, sizeof(g_decode_begin));
  cudaMemcpyFromSymbol(n, g_decode_ntiles, sizeof(g_decode_ntiles));
  return (int)cudaMemcpyFromSymbol(e, g_decode_end, sizeof(g_decode_end));
}
extern "C" __attribute__((visibility("default"))) int tfa_decode_ends_read(unsigned long long* host) {
  cudaError_t e = cudaMemcpyFromSymbol(host, g_decode_end, sizeof(g_decode_end));
  return (int)e;
}
#endif

template int decode_smem_bytes<64>();
template int decode_smem_bytes<128>();
template cudaError_t launch_decode<64>(const FwdParams&, const KvMaps&, const CUtensorMap&, int, cudaStream_t, int);
template cudaError_t launch_decode<128>(const FwdParams&, const KvMaps&, const CUtensorMap&, int, cudaStream_t,
                                        int);

}  // namespace tfa
