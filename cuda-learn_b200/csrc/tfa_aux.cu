// LSE combine of split-KV partial outputs, and the gather debug kernel.
#include <cmath>
#include <mutex>

#include "tfa_common.cuh"

namespace tfa {

namespace {

// Merges the split partials of one (q token, q head) row into `out` (and the LSE).
template <int D, int EPL>
__device__ __forceinline__ void combine_row(const FwdParams& p, int64_t pair, int tok, int qh, int ns, int lane) {
  const int64_t stride = (int64_t)p.total_q * p.hq;
  __nv_bfloat16* dst = p.out + (int64_t)tok * p.o_s0 + (int64_t)qh * p.o_s1 + lane * EPL;
  float acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
  float mx = -INFINITY, wsum = 0.f;
  // All split LSEs are loaded at once (lane s holds split s), then every partial row is
  // requested independently of the others so their latencies overlap.
  for (int s0 = 0; s0 < ns; s0 += 32) {
    const int s = s0 + lane;
    const float ls = s < ns ? p.split_lse[s * stride + pair] : -INFINITY;
    const float cmx = warp_max(ls);
    const float nmx = fmaxf(mx, cmx);
    if (nmx == -INFINITY) continue;
    const float scale_old = (mx == -INFINITY) ? 0.f : ex2_approx(mx - nmx);
    wsum *= scale_old;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] *= scale_old;
    mx = nmx;
    const float wl = (ls == -INFINITY) ? 0.f : ex2_approx(ls - mx);
    wsum += warp_sum(wl);
    const int cnt = ns - s0 < 32 ? ns - s0 : 32;
#pragma unroll 4
    for (int i = 0; i < cnt; ++i) {
      const float wgt = __shfl_sync(0xffffffffu, wl, i);
      const float* src = p.split_o + ((s0 + i) * stride + pair) * D + lane * EPL;
      if constexpr (EPL == 4) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        acc[0] += wgt * v.x;
        acc[1] += wgt * v.y;
        acc[2] += wgt * v.z;
        acc[3] += wgt * v.w;
      } else {
        const float2 v = *reinterpret_cast<const float2*>(src);
        acc[0] += wgt * v.x;
        acc[1] += wgt * v.y;
      }
    }
  }
  if (mx == -INFINITY) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = __float2bfloat16(0.f);
    if (lane == 0 && p.lse) p.lse[pair] = -INFINITY;
    return;
  }
  const float inv = 1.f / wsum;
#pragma unroll
  for (int e = 0; e < EPL; ++e) dst[e] = __float2bfloat16(acc[e] * inv);
  if (lane == 0 && p.lse) p.lse[pair] = (mx + lg2_approx(wsum)) * kLn2;
}

// Restates the merge of v8's splitkv_combine_kernel (v8/flash_attn_func.cu:701-777):
// out = sum_s 2^(lse_s - M) * o_s / sum_s 2^(lse_s - M), M = max_s lse_s, all in the
// log2 domain of the scaled scores. One CTA per work group (q tile slot, sequence, kv
// head; the attention kernels' item order with split 0), one warp per packed row of it
// (up to 16 warps, looping over larger groups);
// partial outputs are already normalised per split. Groups that were not split were
// written directly by the attention kernel and return at once. The group's geometry only
// depends on the call's inputs, so it is computed before the wait for the attention
// kernel (programmatic dependent launch), overlapping that kernel's tail.
template <int D>
__global__ void __launch_bounds__(512) combine_kernel(const __grid_constant__ FwdParams p) {
  constexpr int EPL = D / 32;  // elements per lane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Work w = get_work(p, (int)blockIdx.x);
  const int ns = w.nsplits;
  if (ns <= 1 || w.nrows <= 0) return;
  grid_dependency_wait();  // partials of the attention kernel are complete and visible
  const int nwarps = (int)(blockDim.x >> 5);
  for (int r = warp; r < w.nrows; r += nwarps) {
    const int R = w.row0 + r;
    const int tok = w.q0 + R / p.group;
    const int qh = w.h * p.group + R % p.group;
    const int64_t pair = (int64_t)tok * p.hq + qh;
    combine_row<D, EPL>(p, pair, tok, qh, ns, lane);
  }
}

// Builds the decode kernel's item list for one call: every existing (group, split) item,
// ordered by kv tiles per split, longest first, so the persistent grid hands out the long
// items early and the short ones (whole short sequences) last, which shortens its tail.
// One CTA; a counting sort over the tiles-per-split key (splits hold at most 64 tiles).
// Entry = g * max_splits + split; the number of entries goes to *count.
__global__ void __launch_bounds__(1024) item_list_kernel(const __grid_constant__ FwdParams p, int* list, int* count) {
  constexpr int kKeys = 65;
  __shared__ int hist[kKeys];
  __shared__ int base[kKeys];
  if (threadIdx.x == 0) allow_dependent_launch();  // the decode kernel's set-up overlaps this kernel
  const int groups = p.q_tiles * p.batch * p.hkv;
  for (int i = threadIdx.x; i < kKeys; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  auto key_of = [&](int g, int& ns) {
    const Work w = work_of(p, g, 0);
    ns = w.exists ? w.nsplits : 0;
    return kKeys - 1 - imin(kKeys - 1, w.tile_end - w.tile_begin);
  };
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    int ns;
    const int key = key_of(g, ns);
    if (ns) atomicAdd(&hist[key], ns);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < kKeys; ++i) {
      base[i] = acc;
      acc += hist[i];
    }
    *count = acc;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    int ns;
    const int key = key_of(g, ns);
    if (!ns) continue;
    const int pos = atomicAdd(&base[key], ns);
    for (int sp = 0; sp < ns; ++sp) list[pos + sp] = g * p.max_splits + sp;
  }
}

// One CTA per (kv tile, sequence, kv head): the producer warp stages the tile with the
// attention kernels' TMA gather (produce_tile), then all threads copy the valid rows out.
template <int D>
__global__ void __launch_bounds__(128) gather_kernel(const __grid_constant__ FwdParams p,
                                                     const __grid_constant__ KvMaps maps, const int64_t* kv_offsets,
                                                     __nv_bfloat16* k_out, __nv_bfloat16* v_out) {
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* stage = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full;
  __shared__ volatile int abort_flag;
  const int t = blockIdx.x, b = blockIdx.y, h = blockIdx.z;
  const int kv_len = p.seqused_k[b];
  if (t * kBN >= kv_len) return;
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  Work w{};
  w.b = b;
  w.h = h;
  w.kv_len = kv_len;
  if (threadIdx.x < 32) produce_tile<D>(p, maps, w, t, stage, &full, threadIdx.x, l2_policy_evict_first());
  if (!mbar_wait(&full, 0, &abort_flag, p.err, kDevErrTimeoutProducer)) return;
  const int rows = imin(kBN, kv_len - t * kBN);
  const int64_t base = kv_offsets[b] + (int64_t)t * kBN;
  for (int i = threadIdx.x; i < rows * D; i += blockDim.x) {
    const int r = i / D, c = i % D;
    const uint32_t off = sw128_offset(r, c, kBN);
    const int64_t o = ((base + r) * p.hkv + h) * D + c;
    v_out[o] = *reinterpret_cast<const __nv_bfloat16*>(stage + off);
    k_out[o] = *reinterpret_cast<const __nv_bfloat16*>(stage + KvStage<D>::kTensorBytes + off);
  }
}

}  // namespace

template <int D>
cudaError_t launch_combine(const FwdParams& p, int max_rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)p.q_tiles * p.batch * p.hkv;  // one CTA per work group
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  // one warp per packed row of a group, up to 16
  const int warps = max_rows < 1 ? 1 : (max_rows > 16 ? 16 : max_rows);
  cfg.blockDim = dim3(32 * warps);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_kernel<D>, p);
}

template <int D>
cudaError_t launch_gather(const FwdParams& p, const KvMaps& maps, int max_tiles, const int64_t* kv_offsets,
                          void* k_out, void* v_out, cudaStream_t s) {
  const int smem = KvStage<D>::kBytes + 1024;
  static bool configured[128] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gather_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
  }
  dim3 grid(max_tiles, p.batch, p.hkv);
  gather_kernel<D><<<grid, 128, smem, s>>>(p, maps, kv_offsets, reinterpret_cast<__nv_bfloat16*>(k_out),
                                           reinterpret_cast<__nv_bfloat16*>(v_out));
  return cudaGetLastError();
}

cudaError_t launch_item_list(const FwdParams& p, int* list, int* count, cudaStream_t s) {
  item_list_kernel<<<1, 1024, 0, s>>>(p, list, count);
  return cudaGetLastError();
}

template cudaError_t launch_combine<64>(const FwdParams&, int, cudaStream_t);
template cudaError_t launch_combine<128>(const FwdParams&, int, cudaStream_t);
template cudaError_t launch_gather<64>(const FwdParams&, const KvMaps&, int, const int64_t*, void*, void*,
                                       cudaStream_t);
template cudaError_t launch_gather<128>(const FwdParams&, const KvMaps&, int, const int64_t*, void*, void*,
                                        cudaStream_t);

}  // namespace tfa
