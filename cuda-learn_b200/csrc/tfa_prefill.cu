// Prefill-shaped paged attention (any q length; used when q_len * group > 16).
//
// One work item = (sequence b, kv head h, q tile pair of 2 x 128 packed rows, kv split).
// A packed row is one (q token, q head of the GQA group) pair, so all rows of an item
// share the kv head and every K/V tile is read once for the whole group. The two 128-row
// tiles A and B each have their own softmax warpgroup; at D = 64 they also have their own
// MMA warp, so the two chains QK(j+1) -> softmax(j+1) -> P.V(j+1) run independently, and at
// D = 128 one MMA warp interleaves them (PV_A QK_A PV_B QK_B ...). Either way one tile's
// softmax overlaps the other tile's tensor-core work.
//
// Per kv tile and q tile:
//   S[128 x 128] = Q[128 x D] . K^T   (tcgen05, A = Q K-major, B = K K-major), S in TMEM
//   O[128 x D]  += P[128 x 128] . V   (tcgen05, A = P from TMEM, B = V MN-major), O in TMEM
// Softmax threads own one row each (TMEM lane = row) and hold its 128 scores in
// registers (one TMEM load per tile); P is stored back to TMEM as bf16 pairs and read from
// there by the P.V MMA, so P never touches shared memory (whose bandwidth the MMAs' smem
// operands and the TMA fills already use). At D = 128 P overwrites the first 64 columns of
// the tile's S region; at D = 64 it has columns of its own, so the next QK may start as
// soon as S has been loaded. O is rescaled in TMEM only when a row's max grows by more
// than 2^8 over the max its P values are referenced to (values of P stay <= 256, far inside
// bf16/fp32 range), so most tiles need no O round trip.
//
// Warps (384 threads, three warpgroups): 0 = TMA producer of K and item scheduler, 3 = TMA
// producer of V (K and V tiles in separate, alternating slots), 1 = MMA issuer of tile A
// (of both tiles at D = 128) and TMEM owner, 2 = MMA issuer of tile B at D = 64 (idle at
// D = 128), 4-7 = softmax/epilogue of tile A, 8-11 = softmax/epilogue of tile B. The first
// warpgroup gives up registers (setmaxnreg) so that each softmax thread can hold its
// 128-score row without spilling: 384 threads launch with 168 registers each (a
// sub-partition holds 3 warps x 32 x 168 of its 16 K registers), then 72 for the
// producer/MMA warpgroup and 216 for the softmax ones.
#include <cmath>
#include <mutex>

#include "tfa_common.cuh"

namespace tfa {

namespace {

#ifdef TFA_PROFILE
__device__ unsigned long long g_prefill_tl[2][16][12];
#define TL(x, j, e) do { if (blockIdx.x == 0 && (j) < 16) g_prefill_tl[x][j][e] = global_timer_ns(); } while (0)
#else
#define TL(x, j, e) do {} while (0)
#endif
#ifdef TFA_PROFILE
__device__ unsigned long long g_prefill_prof[1024 * 16];
#define PROF_WAIT(cat, expr) ([&]() { const long long _t0 = clock64(); const bool _r = (expr); prof[cat] += clock64() - _t0; return _r; }())
#else
#define PROF_WAIT(cat, expr) (expr)
#endif

constexpr int kRows = 128;                // rows per q tile
constexpr float kRescaleThreshold = 8.f;  // log2 units

template <int D>
struct PrefillCfg {
  static constexpr int kPanels = D / 64;
  static constexpr int kSlotBytes = KvStage<D>::kTensorBytes;  // one K or V tile
  static constexpr int kSlots = (D == 128) ? 5 : 10;
  static constexpr int kQBytes = kPanels * kRows * 128;        // per q tile
  static constexpr int kQOff = kSlots * kSlotBytes;
  static constexpr int kDynBytes = kQOff + 2 * kQBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;                   // S_A, S_B, O_A, O_B (+ P_A, P_B at D = 64)
  // D = 64 leaves TMEM room for P of its own (O needs 64 columns per tile): QK(j+1) may then
  // overwrite S as soon as the softmax has loaded S(j), overlapping the softmax's exponent
  // phase. At D = 128 (2 x 128 S + 2 x 128 O = 512 columns) P aliases the first 64 S columns.
  static constexpr bool kSeparateP = (D == 64);
  // MMA warps: one per q tile at D = 64 (each tile's chain then waits only on its own
  // softmax: P2 265 -> 229 us per call), one for both tiles at D = 128.
  static constexpr int kMmaWarps = (D == 64) ? 2 : 1;
};

__device__ __forceinline__ uint32_t s_col_of(int x) { return x == 0 ? 0u : 128u; }
__device__ __forceinline__ uint32_t o_col_of(int x) { return x == 0 ? 256u : 384u; }
template <int D>
__device__ __forceinline__ uint32_t p_col_of(int x) {
  return D == 64 ? (x == 0 ? 320u : 448u) : s_col_of(x);  // D = 64: after O's 64 columns
}

constexpr int kThreads = 384;
constexpr uint32_t kRegsLaunch = 168;   // per thread at launch
constexpr uint32_t kRegsControl = 72;   // producer / MMA warpgroup after the split
constexpr uint32_t kRegsSoftmax = 216;  // each softmax warpgroup after the split
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch,
              "register split exceeds the launch's registers");

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ FwdParams p, const __grid_constant__ KvMaps maps) {
  using Cfg = PrefillCfg<D>;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* slots = smem;
  uint8_t* q_smem = smem + Cfg::kQOff;

  __shared__ uint64_t full[Cfg::kSlots], empty[Cfg::kSlots];
  __shared__ uint64_t s_full[2], s_free[2], p_full[2], o_full[2], o_free[2];
  __shared__ uint64_t item_full[2], item_empty[2], q_full[2];
  __shared__ int item_slot[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ uint64_t stall_bar;  // never arrived on: the time-limit test hook waits here

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
#ifdef TFA_PROFILE
  unsigned long long prof[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const long long prof_start = clock64();
#endif

  if (tid == 0) {
    for (int i = 0; i < Cfg::kSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], Cfg::kMmaWarps);  // released by every MMA warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);  // D = 64: the softmax warpgroup has loaded S
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 9 + Cfg::kMmaWarps);  // MMA warps, 8 softmax warps, the V producer
      mbar_init(&q_full[i], 8);
    }
    abort_flag = 0;
    mbar_init(&stall_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.k_box);
    tma_prefetch_desc(&maps.v_box);
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  if (tid == 0) allow_dependent_launch();

  if (warp < 4) {
    // producer / MMA warpgroup: every warp gives up registers first
    warpgroup_reg_release<kRegsControl>();
    if (warp == 0) {
      producer_loop_kv_slots<D, Cfg::kSlots, true>(p, maps, slots, full, empty, item_full, item_empty, item_slot,
                                                   &abort_flag, lane);
    } else if (warp == 3) {
      producer_follow_kv_slots<D, Cfg::kSlots>(p, maps, slots, full, empty, item_full, item_empty, item_slot,
                                               &abort_flag, lane);
    } else if (warp == 1 || (warp == 2 && Cfg::kMmaWarps == 2)) {
      if constexpr (Cfg::kMmaWarps == 2) {
        // ------------------------------------------------------------ MMA issuers
        // One MMA warp per q tile (warp 1: tile A, warp 2: tile B), so each tile's chain
        // QK(j+1) -> softmax -> P.V(j) waits only on its own softmax: a group of MMAs holds its
        // issuing thread for about its execution time, and one warp serving both tiles in a
        // fixed order made each tile's P.V wait behind the other tile's QK and P.V. A K/V slot
        // is released once both warps are done with it (empty barriers count two).
        const int x = warp - 1;
        const uint32_t idesc_qk = make_idesc_bf16_f32(128, 128, false, false);
        const uint32_t idesc_pv = make_idesc_bf16_f32(128, D, false, true);
        const uint32_t qx = smem_u32(q_smem) + x * Cfg::kQBytes;
        int c = 0;   // slot loads consumed (2 per kv tile)
        int ts = 0;  // kv tiles processed by this q tile (phase counter)
        int oi = 0;  // items with rows in this q tile
        bool ok = true;
        auto slot_wait = [&](int cc) -> bool {
          return PROF_WAIT(0, mbar_wait(&full[cc % Cfg::kSlots], (cc / Cfg::kSlots) & 1, &abort_flag, p.err, kDevErrTimeoutMma));
        };
        auto issue_qk = [&](int kslot) {
          TL(x, ts, 0);
          const uint32_t k_addr = smem_u32(slots + kslot * Cfg::kSlotBytes);
  #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * KvStage<D>::kPanelBytes + (kk & 3) * 32;
            umma_bf16_ss(tmem + s_col_of(x), make_sdesc_sw128(qx + off, 16, 1024),
                         make_sdesc_sw128(k_addr + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[x]);
          TL(x, ts, 1);
        };
        auto issue_pv = [&](int vslot, bool first) {
          TL(x, ts, 2);
          const uint32_t v_addr = smem_u32(slots + vslot * Cfg::kSlotBytes);
          const uint32_t p_tmem = tmem + p_col_of<D>(x);  // P as bf16 pairs (over S's first 64 columns at D = 128)
  #pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            umma_bf16_ts(tmem + o_col_of(x), p_tmem + kk * 8,
                         make_sdesc_sw128(v_addr + kk * 2048, KvStage<D>::kPanelBytes, 1024), idesc_pv,
                         (!first || kk > 0) ? 1u : 0u);
          }
          umma_commit(&o_full[x]);
          TL(x, ts, 3);
        };
        // A slot this q tile does not read (an item without rows in it): released once filled.
        auto pass_slot = [&](int cc) -> bool {
          if (!slot_wait(cc)) return false;
          mbar_arrive(&empty[cc % Cfg::kSlots]);
          return true;
        };
        for (int k = 0; ok; ++k) {
          const int slot = k & 1;
          if (!PROF_WAIT(3, mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma))) break;
          const int idx = item_slot[slot];
          if (idx >= p.num_items) break;
          const Work w = get_work(p, idx);
          // Test hook (FwdParams::debug_stall): wait for a phase that never completes, so the
          // time limit expires, the error word is set and every warp of the CTA unwinds.
          if (p.debug_stall && k == 0 && !mbar_wait(&stall_bar, 0, &abort_flag, p.err, kDevErrTimeoutMma)) break;
          const int n = w.tile_end - w.tile_begin;
          const bool active = (x == 0) || (w.nrows > kRows);  // this q tile has rows
          if (!PROF_WAIT(3, mbar_wait(&q_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma))) break;
          if (lane == 0 && n > 0) {
            if (!active) {
              for (int j = 0; ok && j < 2 * n; ++j) ok = pass_slot(c + j);
            } else {
              ok = slot_wait(c);  // K_0
              if (ok) {
                tc_fence_after();
                issue_qk(c % Cfg::kSlots);
                umma_commit(&empty[c % Cfg::kSlots]);
              }
              for (int j = 0; ok && j < n; ++j) {
                const int kc = c + 2 * j;  // slot load index of K_j; V_j is kc + 1
                const bool more = j + 1 < n;
                if constexpr (Cfg::kSeparateP) {
                  // QK(j+1) as soon as the softmax has loaded S(j) (P lives elsewhere), then P.V(j)
                  if (more) {
                    if (!slot_wait(kc + 2) ||
                        !PROF_WAIT(2, mbar_wait(&s_free[x], ts & 1, &abort_flag, p.err, kDevErrTimeoutMma))) {
                      ok = false;
                      break;
                    }
                    tc_fence_after();
                    issue_qk((kc + 2) % Cfg::kSlots);
                    umma_commit(&empty[(kc + 2) % Cfg::kSlots]);  // K_{j+1} consumed
                  }
                  if (!slot_wait(kc + 1) ||  // V_j
                      !PROF_WAIT(1, mbar_wait(&p_full[x], ts & 1, &abort_flag, p.err, kDevErrTimeoutMma)) ||
                      (j == 0 && !PROF_WAIT(2, mbar_wait(&o_free[x], (oi & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutMma)))) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  issue_pv((kc + 1) % Cfg::kSlots, j == 0);
                  umma_commit(&empty[(kc + 1) % Cfg::kSlots]);  // V_j consumed
                  ++ts;
                } else {
                  // P(j) overwrites the first columns of S(j): QK(j+1) waits until P.V(j) has read it
                  if (!slot_wait(kc + 1) ||  // V_j
                      !PROF_WAIT(1, mbar_wait(&p_full[x], ts & 1, &abort_flag, p.err, kDevErrTimeoutMma)) ||
                      (j == 0 && !PROF_WAIT(2, mbar_wait(&o_free[x], (oi & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutMma)))) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  issue_pv((kc + 1) % Cfg::kSlots, j == 0);
                  umma_commit(&empty[(kc + 1) % Cfg::kSlots]);  // V_j consumed
                  ++ts;
                  if (more) {
                    if (!mbar_wait(&o_full[x], (ts - 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma) || !slot_wait(kc + 2)) {
                      ok = false;
                      break;
                    }
                    tc_fence_after();
                    issue_qk((kc + 2) % Cfg::kSlots);
                    umma_commit(&empty[(kc + 2) % Cfg::kSlots]);  // K_{j+1} consumed
                  }
                }
              }
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          ts = __shfl_sync(0xffffffffu, ts, 0);
          if (n > 0 && active) ++oi;
          c += 2 * n;
          __syncwarp();
          if (lane == 0) mbar_arrive(&item_empty[slot]);
        }
      } else {
        // ------------------------------------------------------------ MMA issuer (both tiles)
        // At D = 128 one warp issues for both tiles in the order PV_A(j) QK_A(j+1) PV_B(j)
        // QK_B(j+1): the tiles' large MMA groups then alternate on the tensor pipe instead
        // of colliding (two MMA warps measured 17 % slower on P1).
        // ------------------------------------------------------------ MMA issuer
        const uint32_t idesc_qk = make_idesc_bf16_f32(128, 128, false, false);
        const uint32_t idesc_pv = make_idesc_bf16_f32(128, D, false, true);
        const uint32_t q_addr = smem_u32(q_smem);
        int c = 0;           // slot loads consumed (2 per kv tile)
        int ts0 = 0, ts1 = 0;  // kv tiles processed per q tile (phase counters)
        int oi0 = 0, oi1 = 0;  // non-empty items per q tile
        bool ok = true;
        auto slot_wait = [&](int cc) -> bool {
          return PROF_WAIT(0, mbar_wait(&full[cc % Cfg::kSlots], (cc / Cfg::kSlots) & 1, &abort_flag, p.err, kDevErrTimeoutMma));
        };
        auto issue_qk = [&](int x, int kslot) {
          const uint32_t k_addr = smem_u32(slots + kslot * Cfg::kSlotBytes);
          const uint32_t qx = q_addr + x * Cfg::kQBytes;
    #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * KvStage<D>::kPanelBytes + (kk & 3) * 32;
            umma_bf16_ss(tmem + s_col_of(x), make_sdesc_sw128(qx + off, 16, 1024),
                         make_sdesc_sw128(k_addr + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[x]);
        };
        auto issue_pv = [&](int x, int vslot, bool first) {
          const uint32_t v_addr = smem_u32(slots + vslot * Cfg::kSlotBytes);
          const uint32_t p_tmem = tmem + p_col_of<D>(x);  // P as bf16 pairs (over S's first 64 columns at D = 128)
    #pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            umma_bf16_ts(tmem + o_col_of(x), p_tmem + kk * 8,
                         make_sdesc_sw128(v_addr + kk * 2048, KvStage<D>::kPanelBytes, 1024), idesc_pv,
                         (!first || kk > 0) ? 1u : 0u);
          }
          umma_commit(&o_full[x]);
        };
        for (int k = 0; ok; ++k) {
          const int slot = k & 1;
          if (!PROF_WAIT(3, mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma))) break;
          const int idx = item_slot[slot];
          if (idx >= p.num_items) break;
          const Work w = get_work(p, idx);
          // Test hook (FwdParams::debug_stall): wait for a phase that never completes, so the
          // time limit expires, the error word is set and every warp of the CTA unwinds.
          if (p.debug_stall && k == 0 && !mbar_wait(&stall_bar, 0, &abort_flag, p.err, kDevErrTimeoutMma)) break;
          const int n = w.tile_end - w.tile_begin;
          const int nx = w.nrows > kRows ? 2 : 1;  // q tiles with rows
          if (!PROF_WAIT(3, mbar_wait(&q_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma))) break;
          if (lane == 0 && n > 0) {
            // QK of the first kv tile for both q tiles
            ok = slot_wait(c);
            if (ok) {
              tc_fence_after();
              for (int x = 0; x < nx; ++x) issue_qk(x, c % Cfg::kSlots);
              umma_commit(&empty[c % Cfg::kSlots]);  // K_0 consumed
            }
            for (int j = 0; ok && j < n; ++j) {
              const int kc = c + 2 * j;  // slot load index of K_j; V_j is kc + 1
              const bool more = j + 1 < n;
              if constexpr (Cfg::kSeparateP) {
                // QK(j+1) as soon as the softmax has loaded S(j) (P lives elsewhere), then P.V(j)
                if (more) {
                  if (!slot_wait(kc + 2)) {  // K_{j+1}
                    ok = false;
                    break;
                  }
                  for (int x = 0; x < nx; ++x) {
                    if (!PROF_WAIT(2, mbar_wait(&s_free[x], (x ? ts1 : ts0) & 1, &abort_flag, p.err, kDevErrTimeoutMma))) {
                      ok = false;
                      break;
                    }
                    tc_fence_after();
                    issue_qk(x, (kc + 2) % Cfg::kSlots);
                  }
                  if (!ok) break;
                  umma_commit(&empty[(kc + 2) % Cfg::kSlots]);  // K_{j+1} consumed
                }
                if (!slot_wait(kc + 1)) {  // V_j
                  ok = false;
                  break;
                }
                for (int x = 0; x < nx; ++x) {
                  const int tsx = x ? ts1 : ts0, oix = x ? oi1 : oi0;
                  if (!PROF_WAIT(1, mbar_wait(&p_full[x], tsx & 1, &abort_flag, p.err, kDevErrTimeoutMma)) ||
                      (j == 0 && !PROF_WAIT(2, mbar_wait(&o_free[x], (oix & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutMma)))) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  issue_pv(x, (kc + 1) % Cfg::kSlots, j == 0);
                  if (x) ++ts1; else ++ts0;
                }
                if (!ok) break;
                umma_commit(&empty[(kc + 1) % Cfg::kSlots]);  // V_j consumed
                continue;
              }
              if (!slot_wait(kc + 1)) {  // V_j
                ok = false;
                break;
              }
              for (int x = 0; x < nx; ++x) {
                const int tsx = x ? ts1 : ts0, oix = x ? oi1 : oi0;
                if (!PROF_WAIT(1, mbar_wait(&p_full[x], tsx & 1, &abort_flag, p.err, kDevErrTimeoutMma)) ||
                    (j == 0 && !PROF_WAIT(2, mbar_wait(&o_free[x], (oix & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutMma)))) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                issue_pv(x, (kc + 1) % Cfg::kSlots, j == 0);
                if (x) ++ts1; else ++ts0;
                if (more) {
                  // QK(j+1) overwrites S, whose first columns hold the P this P.V reads:
                  // wait for the P.V to finish. K_{j+1} is awaited only now, so its load
                  // overlaps the softmax of tile A.
                  if (!mbar_wait(&o_full[x], ((x ? ts1 : ts0) - 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma) ||
                      (x == 0 && !slot_wait(kc + 2))) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  issue_qk(x, (kc + 2) % Cfg::kSlots);
                }
              }
              if (!ok) break;
              umma_commit(&empty[(kc + 1) % Cfg::kSlots]);            // V_j consumed
              if (more) umma_commit(&empty[(kc + 2) % Cfg::kSlots]);  // K_{j+1} consumed
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          ts0 = __shfl_sync(0xffffffffu, ts0, 0);
          ts1 = __shfl_sync(0xffffffffu, ts1, 0);
          if (n > 0) {
            ++oi0;
            if (nx == 2) ++oi1;
          }
          c += 2 * n;
          __syncwarp();
          if (lane == 0) mbar_arrive(&item_empty[slot]);
        }
      }
    }
  } else {
    warpgroup_reg_claim<kRegsSoftmax>();
      // ------------------------------------------------------------ softmax / epilogue
      const int x = (warp - 4) >> 2;   // q tile of this warpgroup
      const int quad = warp & 3;       // TMEM lane quadrant this warp may access
      const int r = quad * 32 + lane;  // row of the q tile == TMEM lane
      const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
      const uint32_t s_col = lane_base + s_col_of(x);
      const uint32_t o_col = lane_base + o_col_of(x);
      const uint32_t p_col = lane_base + p_col_of<D>(x);
      uint8_t* q_tile = q_smem + x * Cfg::kQBytes;
      int ts = 0;  // kv tiles processed by this q tile (phase counter)
      for (int k = 0;; ++k) {
        const int slot = k & 1;
        if (!PROF_WAIT(3, mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax))) break;
        const int idx = item_slot[slot];
        if (idx >= p.num_items) break;
        const Work w = get_work(p, idx);
        const int n = w.tile_end - w.tile_begin;
        const bool tile_active = (x == 0) || (w.nrows > kRows);
        const int R = w.row0 + x * kRows + r;
        const bool row_valid = (x * kRows + r) < w.nrows;
        const int tok = w.q0 + (row_valid ? R / p.group : 0);
        const int qh = w.h * p.group + R % p.group;

        // Q row -> shared memory (K-major, 128-byte swizzle), zero for padding rows.
        {
          const __nv_bfloat16* src = p.q + (int64_t)tok * p.q_s0 + (int64_t)qh * p.q_s1;
  #pragma unroll
          for (int u = 0; u < D / 8; ++u) {
            uint4 val = make_uint4(0, 0, 0, 0);
            if (row_valid) val = __ldg(reinterpret_cast<const uint4*>(src + u * 8));
            const int ch = u >> 3, uu = u & 7;
            *reinterpret_cast<uint4*>(q_tile + ch * (kRows * 128) + r * 128 + ((uu ^ (r & 7)) << 4)) = val;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&q_full[slot]);
        }
        if (!tile_active) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&item_empty[slot]);
          continue;
        }
        int lo = 1, hi = 0;
        if (row_valid) visible_range(p, R / p.group, w.q_len, w.kv_len, lo, hi);

        float m_ref = -INFINITY;  // max the P values and O are referenced to (scaled log2 domain)
        float l = 0.f;
        bool ok = true;
        for (int j = 0; j < n; ++j) {
          if (!PROF_WAIT(0, mbar_wait(&s_full[x], ts & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax))) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (quad == 0 && lane == 0) TL(x, ts, 4);
          const int base = (w.tile_begin + j) * kBN;
          const bool full_tile = __all_sync(0xffffffffu, (base >= lo) && (base + kBN - 1 <= hi));
          // the whole 128-score row in registers, one TMEM load
          float sv[128];
          tmem_ld128_sync(s_col, sv);
          if (quad == 0 && lane == 0) TL(x, ts, 5);
          if constexpr (Cfg::kSeparateP) {  // S(j) is in registers: QK(j+1) may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[x]);
          }
          // row max over 8 independent partial maxima, three-input max (short chains)
          float m8[8];
  #pragma unroll
          for (int e = 0; e < 8; ++e) m8[e] = -INFINITY;
          if (!full_tile) {
  #pragma unroll
            for (int i = 0; i < 128; ++i) sv[i] = (base + i >= lo && base + i <= hi) ? sv[i] : -INFINITY;
          }
  #pragma unroll
          for (int i = 0; i < 64; ++i) m8[i & 7] = fmax3(m8[i & 7], sv[2 * i], sv[2 * i + 1]);
          float tmax = fmaxf(fmax3(m8[0], m8[1], m8[2]), fmax3(fmax3(m8[3], m8[4], m8[5]), m8[6], m8[7]));
          tmax *= p.scale_log2;
          if (quad == 0 && lane == 0) TL(x, ts, 6);
          // reference max: moves only when the new max exceeds it by the threshold
          float alpha = 1.f;
          bool rescale = false;
          if (tmax > m_ref + kRescaleThreshold || (m_ref == -INFINITY && tmax > -INFINITY)) {
            if (m_ref != -INFINITY) {
              alpha = ex2_approx(m_ref - tmax);
              rescale = true;
            }
            m_ref = tmax;
          }
          // Rescaling O needs the previous P.V of this q tile complete. At D = 128 writing P
          // needs no wait: P(j) overwrites only S(j), and the MMA warp issued QK(j) after
          // P.V(j-1), which read P(j-1) from those columns, had completed. At D = 64 P has
          // columns of its own, which P.V(j-1) reads: that wait comes just before the first
          // P store, so the exponentials overlap it.
          const bool rescale_any = j > 0 && __any_sync(0xffffffffu, rescale);
          bool p_wait = Cfg::kSeparateP && j > 0 && !rescale_any;
          if (rescale_any) {
            if (!PROF_WAIT(1, mbar_wait(&o_full[x], (ts - 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax))) {
              ok = false;
              break;
            }
            tc_fence_after();
            {
  #pragma unroll 1
              for (int cc = 0; cc < D / 32; ++cc) {
                float t[32];
                tmem_ld32(o_col + cc * 32, t);
                tmem_wait_ld();
  #pragma unroll
                for (int i = 0; i < 32; ++i) t[i] *= alpha;
                tmem_st32(o_col + cc * 32, t);
              }
              tmem_wait_st();
            }
          }
          l *= alpha;
          // P = 2^(s*scale - m_ref) -> bf16 pairs -> TMEM (P's columns), row sum
          const float ms = (m_ref == -INFINITY) ? 0.f : m_ref;
          const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
          const uint64_t neg_ms2 = f2_pack(-ms, -ms);
          uint64_t rs2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};  // packed partial row sums
  #pragma unroll
          for (int h = 0; h < 2; ++h) {
            float pk[32];
  #pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int i0 = h * 64 + 2 * c;
              float a, b;
              f2_unpack(f2_fma(f2_pack(sv[i0], sv[i0 + 1]), scale2, neg_ms2), a, b);
              const float p0 = ex2_approx(a), p1 = ex2_approx(b);
              rs2[c & 1] = f2_add(rs2[c & 1], f2_pack(p0, p1));
              __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
              pk[c] = __uint_as_float(*reinterpret_cast<uint32_t*>(&h2));
            }
            if (h == 0 && p_wait) {
              if (quad == 0 && lane == 0) TL(x, ts, 7);
              if (!mbar_wait(&o_full[x], (ts - 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) ok = false;
              tc_fence_after();
              p_wait = false;
              if (quad == 0 && lane == 0) TL(x, ts, 8);
            }
            tmem_st32(p_col + h * 32, pk);
          }
          tmem_wait_st();
          if (!ok) break;
          float r0, r1, r2, r3;
          f2_unpack(rs2[0], r0, r1);
          f2_unpack(rs2[1], r2, r3);
          l += (r0 + r1) + (r2 + r3);
          if (quad == 0 && lane == 0) TL(x, ts, 9);
          ++ts;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[x]);
        }
        if (!ok) break;
        if (n > 0) {
          if (!PROF_WAIT(2, mbar_wait(&o_full[x], (ts - 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax))) break;
          tc_fence_after();
        }

        // epilogue: O / l -> out (single split) or the fp32 partial buffers
        const bool direct = (w.nsplits == 1);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const float lse2 = l > 0.f ? m_ref + lg2_approx(l) : -INFINITY;
        const int64_t prow_idx = ((int64_t)w.split * p.total_q + tok) * p.hq + qh;
  #pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          float t[32];
          if (n > 0) {
            tmem_ld32(o_col + cc * 32, t);
            tmem_wait_ld();
          } else {
  #pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = 0.f;
          }
          if (row_valid) {
            if (direct) {
              __nv_bfloat16* dst = p.out + (int64_t)tok * p.o_s0 + (int64_t)qh * p.o_s1 + cc * 32;
  #pragma unroll
              for (int v4 = 0; v4 < 4; ++v4) {
                uint32_t pk[4];
  #pragma unroll
                for (int e = 0; e < 4; ++e) {
                  __nv_bfloat162 h2 = __floats2bfloat162_rn(t[v4 * 8 + 2 * e] * inv, t[v4 * 8 + 2 * e + 1] * inv);
                  pk[e] = *reinterpret_cast<uint32_t*>(&h2);
                }
                *reinterpret_cast<uint4*>(dst + v4 * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            } else {
              float* dst = p.split_o + prow_idx * D + cc * 32;
  #pragma unroll
              for (int v4 = 0; v4 < 8; ++v4)
                *reinterpret_cast<float4*>(dst + v4 * 4) =
                    make_float4(t[v4 * 4] * inv, t[v4 * 4 + 1] * inv, t[v4 * 4 + 2] * inv, t[v4 * 4 + 3] * inv);
            }
          }
        }
        if (row_valid) {
          if (direct) {
            if (p.lse) p.lse[(int64_t)tok * p.hq + qh] = lse2 * kLn2;
          } else {
            p.split_lse[prow_idx] = lse2;
          }
        }
        if (n > 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[x]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[slot]);
      }
  }

#ifdef TFA_PROFILE
  prof[4] = clock64() - prof_start;
  if (lane == 0 && (warp == 1 || warp == 4 || warp == 8) && blockIdx.x < 1024) {
    const int base_idx = blockIdx.x * 16 + (warp == 1 ? 0 : (warp == 4 ? 5 : 10));
    for (int i = 0; i < 5; ++i) g_prefill_prof[base_idx + i] = prof[i];
  }
#endif
  if (abort_flag && (warp == 0 || warp == 3)) {
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

}  // namespace

template <int D>
int prefill_smem_bytes() {
  return PrefillCfg<D>::kDynBytes;
}

template <int D>
cudaError_t launch_prefill(const FwdParams& p, const KvMaps& maps, int grid, cudaStream_t s) {
  static bool configured[128] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, PrefillCfg<D>::kDynBytes);
      if (e != cudaSuccess) return e;
      // The in-kernel register split only fits if the kernel launches with the registers it
      // was designed for; a smaller launch budget would make the softmax warpgroups' claim
      // wait forever, so such a build refuses to launch.
      cudaFuncAttributes fa;
      if ((e = cudaFuncGetAttributes(&fa, prefill_kernel<D>)) != cudaSuccess) return e;
      if ((uint32_t)fa.numRegs * kThreads < 128 * kRegsControl + 256 * kRegsSoftmax) return cudaErrorInvalidKernelImage;
      configured[dev] = true;
    }
  }
  prefill_kernel<D><<<grid, kThreads, PrefillCfg<D>::kDynBytes, s>>>(p, maps);
  return cudaGetLastError();
}

#ifdef TFA_PROFILE
extern "C" __attribute__((visibility("default"))) int tfa_prefill_tl_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, g_prefill_tl, sizeof(g_prefill_tl));
}
extern "C" __attribute__((visibility("default"))) int tfa_prefill_prof_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, g_prefill_prof, sizeof(g_prefill_prof));
}
#endif

template int prefill_smem_bytes<64>();
template int prefill_smem_bytes<128>();
template cudaError_t launch_prefill<64>(const FwdParams&, const KvMaps&, int, cudaStream_t);
template cudaError_t launch_prefill<128>(const FwdParams&, const KvMaps&, int, cudaStream_t);

}  // namespace tfa
