// Router kernels: gate logits, warp-shuffle top-k + softmax, and the stable
// token->expert permutation (a counting sort that is stable by construction).
//
// Reference behaviour restated: the mlx_lm MoE block's gate -> softmax ->
// argpartition top-k (bigrig_engine/stream.py:1436-1439, adapter.py:74-92) and the
// host-side np.argsort(kind="stable") permutation with its inverse
// (bigrig_engine/stream.py:1246-1250, 1275-1276, 1527-1531).
#include "common.cuh"
#include "launch.h"
#include "routing.cuh"

namespace bigrig {

// ---------------------------------------------------------------- logits
// One warp per (token, expert): fp32 dot of a bf16 x row and a bf16 gate row,
// 8 bf16 per lane per 128-bit load.  Blocks of 8 warps share one token's x row
// through L1.  H must be a multiple of 8.
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w,
                                                            const float* __restrict__ bias,
                                                            float* __restrict__ logits, int T,
                                                            int H, int E) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  const int t = blockIdx.y;
  if (e >= E || t >= T) return;
  const uint16_t* xr = x + static_cast<size_t>(t) * H;
  const uint16_t* wr = w + static_cast<size_t>(e) * H;
  float acc = 0.f;
  for (int c = lane * 8; c < H; c += 32 * 8) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
    uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc = fmaf(__uint_as_float(xs[i] << 16), __uint_as_float(ws[i] << 16), acc);
      acc = fmaf(__uint_as_float(xs[i] & 0xffff0000u), __uint_as_float(ws[i] & 0xffff0000u), acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) logits[static_cast<size_t>(t) * E + e] = acc + (bias ? bias[e] : 0.f);
}

// ---------------------------------------------------------------- top-k
// One warp per token over logits[T, E] (fp32 or bf16), E <= 256.
template <int PER_LANE>
__global__ void __launch_bounds__(256) router_topk_kernel(const void* __restrict__ logits,
                                                          int dtype, int T, int E, int k,
                                                          int mode, int norm_topk,
                                                          int32_t* __restrict__ indices,
                                                          float* __restrict__ scores) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const size_t row = static_cast<size_t>(t) * E;
  auto load = [&](int e) {
    return dtype == BIGRIG_F32 ? static_cast<const float*>(logits)[row + e]
                               : bf16_bits_to_f32(static_cast<const uint16_t*>(logits)[row + e]);
  };
  topk_warp<PER_LANE>(load, E, k, mode, norm_topk, indices + static_cast<size_t>(t) * k,
                      scores + static_cast<size_t>(t) * k);
}

// ---------------------------------------------------------------- permutation
// One CTA of 1024 threads.  Pass 1 counts pairs per expert, a serial scan turns
// counts into offsets, pass 2 places pairs chunk by chunk (1024 per chunk, in
// order): inside a warp __match_any_sync ranks equal experts by lane, per-warp
// counts are prefix-summed across warps per expert, and a running offset per
// expert carries across chunks.  Equal experts therefore keep their input order,
// which is exactly np.argsort(kind="stable").
constexpr int kPermThreads = 1024;

__global__ void __launch_bounds__(kPermThreads) permute_kernel(
    const int32_t* __restrict__ idx, int P, int E, int32_t* __restrict__ order,
    int32_t* __restrict__ inv, int32_t* __restrict__ offsets, int32_t* __restrict__ seg_expert,
    int32_t* __restrict__ seg_start, int32_t* __restrict__ num_seg, int32_t* __restrict__ err) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int run[kMaxExperts];
  __shared__ int tot[kMaxExperts];
  __shared__ int wcnt[32][kMaxExperts];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E; e += kPermThreads) cnt[e] = 0;
  __syncthreads();
  int bad = 0;
  for (int i = tid; i < P; i += kPermThreads) {
    const int e = idx[i];
    if (e < 0) continue;                 // padding row (expert-parallel dispatch), skipped
    if (e >= E) { ++bad; continue; }
    atomicAdd(&cnt[e], 1);
  }
  if (bad && err) atomicAdd(err, bad);
  __syncthreads();
  if (tid == 0) {
    int acc = 0, ns = 0;
    for (int e = 0; e < E; ++e) {
      const int c = cnt[e];
      offsets[e] = acc;
      run[e] = acc;
      if (c > 0) { seg_expert[ns] = e; seg_start[ns] = acc; ++ns; }
      acc += c;
    }
    offsets[E] = acc;
    seg_start[ns] = acc;
    *num_seg = ns;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int base = 0; base < P; base += kPermThreads) {
    const int i = base + tid;
    int e = (i < P) ? idx[i] : -1;
    if (e >= E) e = -1;
    for (int j = tid; j < 32 * E; j += kPermThreads) wcnt[j / E][j % E] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int in_warp = __popc(same & lt_mask);
    if (e >= 0 && in_warp == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    for (int x = tid; x < E; x += kPermThreads) {
      int s = 0;
      for (int w = 0; w < 32; ++w) { const int c = wcnt[w][x]; wcnt[w][x] = s; s += c; }
      tot[x] = s;
    }
    __syncthreads();
    if (e >= 0) {
      const int dest = run[e] + wcnt[warp][e] + in_warp;
      order[dest] = i;
      inv[i] = dest;
    }
    __syncthreads();
    for (int x = tid; x < E; x += kPermThreads) run[x] += tot[x];
    __syncthreads();
  }
}

// Decode-sized permutation (P <= 32 pairs): one warp (see permute_warp).
__global__ void __launch_bounds__(32) permute_warp_kernel(
    const int32_t* __restrict__ idx, int P, int E, int32_t* __restrict__ order,
    int32_t* __restrict__ inv, int32_t* __restrict__ offsets, int32_t* __restrict__ seg_expert,
    int32_t* __restrict__ seg_start, int32_t* __restrict__ num_seg, int32_t* __restrict__ err) {
  pdl_wait();
  permute_warp(idx, P, E, order, inv, offsets, seg_expert, seg_start, num_seg, err);
}

// ---------------------------------------------------------------- launchers
int launch_router_logits(const void* x, const void* w, const float* bias, float* logits, int T,
                         int H, int E, cudaStream_t s) {
  dim3 grid((E + 7) / 8, T);
  TimedLaunch tl(BIGRIG_K_ROUTER_LOGITS, s);
  router_logits_kernel<<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(x),
                                            static_cast<const uint16_t*>(w), bias, logits, T, H, E);
  return check_launch("router_logits_kernel");
}

int launch_router_topk(const void* logits, int dtype, int T, int E, int k, int mode, int norm,
                       int32_t* indices, float* scores, cudaStream_t s) {
  const dim3 grid((T + 7) / 8);
  const int per = (E + 31) / 32;
  TimedLaunch tl(BIGRIG_K_ROUTER_TOPK, s);
#define BIGRIG_TOPK(N)                                                                      \
  case N:                                                                                   \
    router_topk_kernel<N><<<grid, 256, 0, s>>>(logits, dtype, T, E, k, mode, norm, indices, \
                                               scores);                                     \
    break;
  switch (per) {
    BIGRIG_TOPK(1)
    BIGRIG_TOPK(2)
    BIGRIG_TOPK(3)
    BIGRIG_TOPK(4)
    BIGRIG_TOPK(5)
    BIGRIG_TOPK(6)
    BIGRIG_TOPK(7)
    BIGRIG_TOPK(8)
    default:
      return set_error(BIGRIG_ERR_UNSUPPORTED, "router_topk: n_experts must be <= 256");
  }
#undef BIGRIG_TOPK
  return check_launch("router_topk_kernel");
}

int launch_permute(const int32_t* indices, int P, int E, int32_t* order, int32_t* inv,
                   int32_t* offsets, int32_t* seg_expert, int32_t* seg_start, int32_t* num_seg,
                   int32_t* err, cudaStream_t s) {
  TimedLaunch tl(BIGRIG_K_PERMUTE, s);
  if (P <= 32) {
    permute_warp_kernel<<<1, 32, 0, s>>>(indices, P, E, order, inv, offsets, seg_expert, seg_start,
                                         num_seg, err);
    return check_launch("permute_warp_kernel");
  }
  permute_kernel<<<1, kPermThreads, 0, s>>>(indices, P, E, order, inv, offsets, seg_expert,
                                            seg_start, num_seg, err);
  return check_launch("permute_kernel");
}

}  // namespace bigrig
