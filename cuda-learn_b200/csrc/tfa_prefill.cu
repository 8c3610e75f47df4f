// Prefill-shaped paged attention (any q length; used when q_len * group > 16).
//
// One work item = (sequence b, kv head h, q tile of 128 packed rows, kv split). A packed
// row is one (q token, q head of the GQA group) pair, so the rows of a tile share the
// kv head and every K/V tile is read once for the whole group. Per kv tile:
//   S[128 x 128] = Q[128 x D] . K^T        (tcgen05, A = Q K-major, B = K tile K-major)
//   O[128 x D]  += P[128 x 128] . V        (tcgen05, A = P K-major,  B = V tile MN-major)
// S is double-buffered in TMEM so the QK^T of tile j+1 overlaps the softmax of tile j.
// Softmax threads own one row each (TMEM lane = row): the row max and sum need no
// cross-thread exchange. O stays in TMEM; when a warp's running max moves, that warp
// rescales its O rows in TMEM before the next P.V is issued.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = MMA issuer + TMEM owner,
// warps 2-5 = softmax / epilogue.
#include <cmath>

#include "tfa_common.cuh"

namespace tfa {

namespace {

constexpr int kRows = 128;

template <int D>
struct PrefillCfg {
  static constexpr int kPanels = D / 64;
  static constexpr int kStages = (D == 128) ? 2 : 4;
  static constexpr int kStageBytes = KvStage<D>::kBytes;
  static constexpr int kQBytes = kPanels * kRows * 128;  // 16 KB per 64 columns
  static constexpr int kPBytes = 2 * kRows * 128;        // 128 rows x 128 tokens bf16
  static constexpr int kQOff = kStages * kStageBytes;
  static constexpr int kPOff = kQOff + kQBytes;
  static constexpr int kDynBytes = kPOff + kPBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;             // S x2 (256 cols) + O (D cols)
  static constexpr uint32_t kOCol = 256;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    prefill_kernel(const __grid_constant__ FwdParams p, const __grid_constant__ KvMaps maps) {
  using Cfg = PrefillCfg<D>;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* q_smem = smem + Cfg::kQOff;
  uint8_t* p_smem = smem + Cfg::kPOff;

  __shared__ uint64_t full[Cfg::kStages], empty[Cfg::kStages];
  __shared__ uint64_t s_full[2], s_free[2];
  __shared__ uint64_t p_full, o_full, o_free, q_full[2];
  __shared__ uint64_t item_full[2], item_empty[2];
  __shared__ int item_slot[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < Cfg::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 5);
      mbar_init(&q_full[i], 4);
    }
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
    mbar_init(&o_free, 4);
    abort_flag = 0;
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

  if (warp == 0) {
    producer_loop<D, Cfg::kStages>(p, maps, stages, full, empty, item_full, item_empty, item_slot, &abort_flag,
                                   lane);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_qk = make_idesc_bf16_f32(128, 128, false, false);
    const uint32_t idesc_pv = make_idesc_bf16_f32(128, D, false, true);
    const uint32_t q_addr = smem_u32(q_smem);
    const uint32_t p_addr = smem_u32(p_smem);
    int c = 0, oi = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      const int idx = item_slot[slot];
      if (idx >= p.num_items) break;
      const Work w = get_work(p, idx);
      const int n = w.tile_end - w.tile_begin;
      if (!mbar_wait(&q_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) break;
      if (lane == 0 && n > 0) {
        auto issue_qk = [&](int cc) -> bool {
          const int st = cc % Cfg::kStages;
          if (!mbar_wait(&full[st], (cc / Cfg::kStages) & 1, &abort_flag, p.err, kDevErrTimeoutMma)) return false;
          if (!mbar_wait(&s_free[cc & 1], ((cc >> 1) & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutMma)) return false;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(stages + st * Cfg::kStageBytes) + KvStage<D>::kTensorBytes;
          const uint32_t d_tmem = tmem + (cc & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * KvStage<D>::kPanelBytes + (kk & 3) * 32;
            umma_bf16_ss(d_tmem, make_sdesc_sw128(q_addr + off, 16, 1024), make_sdesc_sw128(k_addr + off, 16, 1024),
                         idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[cc & 1]);
          return true;
        };
        ok = issue_qk(c);
        for (int j = 0; ok && j < n; ++j) {
          const int cj = c + j;
          if (j + 1 < n && !(ok = issue_qk(cj + 1))) break;
          if (!mbar_wait(&p_full, cj & 1, &abort_flag, p.err, kDevErrTimeoutMma)) {
            ok = false;
            break;
          }
          if (j == 0 && !mbar_wait(&o_free, (oi & 1) ^ 1, &abort_flag, p.err, kDevErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int st = cj % Cfg::kStages;
          const uint32_t v_addr = smem_u32(stages + st * Cfg::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint32_t poff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
            umma_bf16_ss(tmem + Cfg::kOCol, make_sdesc_sw128(p_addr + poff, 16, 1024),
                         make_sdesc_sw128(v_addr + kk * 2048, KvStage<D>::kPanelBytes, 1024), idesc_pv,
                         (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[st]);
          umma_commit(&o_full);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (n > 0) ++oi;
      c += n;
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // packed row of the tile == TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    int c = 0;
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      if (!mbar_wait(&item_full[slot], (k >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) break;
      const int idx = item_slot[slot];
      if (idx >= p.num_items) break;
      const Work w = get_work(p, idx);
      const int n = w.tile_end - w.tile_begin;
      const bool row_valid = r < w.nrows;
      const int R = w.row0 + r;
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
          *reinterpret_cast<uint4*>(q_smem + ch * (kRows * 128) + r * 128 + ((uu ^ (r & 7)) << 4)) = val;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[slot]);
      }
      int lo = 1, hi = 0;
      if (row_valid) visible_range(p, R / p.group, w.q_len, w.kv_len, lo, hi);

      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        const int cj = c + j;
        if (!mbar_wait(&s_full[cj & 1], (cj >> 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[128];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float t[32];
          tmem_ld32(lane_base + (cj & 1) * 128 + q4 * 32, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[q4 * 32 + i] = t[i];
        }
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[cj & 1]);

        const int base = (w.tile_begin + j) * kBN;
        float tmax = -INFINITY;
        const bool full_tile = (base >= lo) && (base + kBN - 1 <= hi);
        if (__all_sync(0xffffffffu, full_tile)) {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            s[i] *= p.scale_log2;
            tmax = fmaxf(tmax, s[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            const int pos = base + i;
            s[i] = (pos >= lo && pos <= hi) ? s[i] * p.scale_log2 : -INFINITY;
            tmax = fmaxf(tmax, s[i]);
          }
        }
        const float mn = fmaxf(m, tmax);
        const float alpha = (m == -INFINITY) ? 1.f : ex2_approx(m - mn);
        // previous P.V must be complete before O is rescaled or P is overwritten
        if (j > 0) {
          if (!mbar_wait(&o_full, (cj - 1) & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const bool need = alpha != 1.f;
          if (__any_sync(0xffffffffu, need)) {
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc) {
              float t[32];
              tmem_ld32(lane_base + Cfg::kOCol + cc * 32, t);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) t[i] *= alpha;
              tmem_st32(lane_base + Cfg::kOCol + cc * 32, t);
            }
            tmem_wait_st();
          }
        }
        const float ms = (mn == -INFINITY) ? 0.f : mn;
        float rs = 0.f;
        uint8_t* prow = p_smem + r * 128;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = ex2_approx(s[u * 8 + 2 * e] - ms);
            const float p1 = ex2_approx(s[u * 8 + 2 * e + 1] - ms);
            rs += p0 + p1;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            pk[e] = *reinterpret_cast<uint32_t*>(&h2);
          }
          const int ch = u >> 3, uu = u & 7;
          *reinterpret_cast<uint4*>(prow + ch * (kRows * 128) + ((uu ^ (r & 7)) << 4)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        l = l * alpha + rs;
        m = mn;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full);
      }
      if (!ok) break;
      if (n > 0) {
        const int cl = c + n - 1;
        if (!mbar_wait(&o_full, cl & 1, &abort_flag, p.err, kDevErrTimeoutSoftmax)) break;
        tc_fence_after();
      }
      c += n;

      // epilogue: O / l -> out (single split) or the fp32 partial buffers
      const bool direct = (w.nsplits == 1);
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const float lse2 = l > 0.f ? m + lg2_approx(l) : -INFINITY;
      const int64_t prow_idx = ((int64_t)w.split * p.total_q + tok) * p.hq + qh;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        float t[32];
        if (n > 0) {
          tmem_ld32(lane_base + Cfg::kOCol + cc * 32, t);
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
        if (lane == 0) mbar_arrive(&o_free);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
    }
  }

  if (abort_flag && warp == 0) {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (tid == 0) scheduler_finish(p);
}

}  // namespace

template <int D>
int prefill_smem_bytes() {
  return PrefillCfg<D>::kDynBytes;
}

template <int D>
cudaError_t launch_prefill(const FwdParams& p, const KvMaps& maps, int grid, cudaStream_t s) {
  static bool configured[128] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PrefillCfg<D>::kDynBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  prefill_kernel<D><<<grid, 192, PrefillCfg<D>::kDynBytes, s>>>(p, maps);
  return cudaGetLastError();
}

template int prefill_smem_bytes<64>();
template int prefill_smem_bytes<128>();
template cudaError_t launch_prefill<64>(const FwdParams&, const KvMaps&, int, cudaStream_t);
template cudaError_t launch_prefill<128>(const FwdParams&, const KvMaps&, int, cudaStream_t);

}  // namespace tfa
