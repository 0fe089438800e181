// Warp-level routing helpers shared by the router kernels and the fused decode route.
#pragma once

#include "common.cuh"

namespace bigrig {

// Top-k of one token's E logits (E <= 32 * PER_LANE) by one warp: k rounds of a warp
// arg-max in which a candidate beats another when its logit is larger, or equal with a
// lower expert id -- the stable descending order.  Lane r < k writes rank r's expert to
// idx[r] and its score to sc[r] (softmax over E then top-k, optionally renormalised;
// or top-k then softmax over the k).  `load(e)` returns logit e as fp32.
template <int PER_LANE, typename Load>
__device__ __forceinline__ void topk_warp(Load load, int E, int k, int mode, int norm_topk,
                                          int32_t* idx, float* sc) {
  const int lane = threadIdx.x & 31;
  float v[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? load(e) : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) mx = fmaxf(mx, v[i]);
  mx = warp_max(mx);
  float denom = 0.f;
  if (mode == BIGRIG_SOFTMAX_TOPK) {
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i)
      if (i * 32 + lane < E) denom += expf(v[i] - mx);
    denom = warp_sum(denom);
  }
  uint32_t taken = 0;
  float first_logit = 0.f, my_logit = 0.f;
  int my_idx = -1;
  for (int r = 0; r < k; ++r) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !(taken & (1u << i))) {
        if (v[i] > best || (v[i] == best && e < best_e)) { best = v[i]; best_e = e; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) { best = ob; best_e = oe; }
    }
    if ((best_e & 31) == lane) taken |= 1u << (best_e >> 5);
    if (lane == r) { my_idx = best_e; my_logit = best; }
    if (r == 0) first_logit = best;
  }
  float s = 0.f;
  if (mode == BIGRIG_SOFTMAX_TOPK) {
    s = (lane < k) ? expf(my_logit - mx) / denom : 0.f;
    if (norm_topk) s = s / warp_sum(s);
  } else {
    const float ex = (lane < k) ? expf(my_logit - first_logit) : 0.f;
    s = ex / warp_sum(ex);
  }
  if (lane < k) {
    idx[lane] = my_idx;
    sc[lane] = s;
  }
}

// topk_warp's result for one token whose E logits sit in shared memory, without its k
// dependent arg-max rounds: every candidate's rank in the (logit descending, expert id
// ascending) order is counted directly against all E logits, the k best are scattered to
// their ranks, and the scores come from the same formulas and reductions as topk_warp, so
// indices and scores are bit-identical to it.  NaN logits are never selected (as in
// topk_warp); a rank no finite logit fills keeps idx -1.  `lg` is 16-byte aligned shared
// memory with room for a multiple of 4 entries; `rank_lg` is 32 floats of shared scratch.
template <int PER_LANE>
__device__ __forceinline__ void topk_rank_warp(const float* lg, int E, int k, int mode,
                                               int norm_topk, int32_t* idx, float* sc,
                                               float* rank_lg) {
  const int lane = threadIdx.x & 31;
  if (lane < k) idx[lane] = -1;
  float v[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? lg[e] : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) mx = fmaxf(mx, v[i]);
  mx = warp_max(mx);
  float denom = 0.f;
  if (mode == BIGRIG_SOFTMAX_TOPK) {
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i)
      if (i * 32 + lane < E) denom += expf(v[i] - mx);
    denom = warp_sum(denom);
  }
  __syncwarp();
  // ranks: every candidate against all E logits, four per shared-memory load (lg is
  // 16-byte aligned; the tail past E is skipped by index)
  int rank[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) rank[i] = 0;
#pragma unroll 2
  for (int u0 = 0; u0 < E; u0 += 4) {
    const float4 w4 = *reinterpret_cast<const float4*>(lg + u0);
    const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int u = u0 + q;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int e = i * 32 + lane;
        rank[i] += u < E && ((w[q] > v[i]) || (w[q] == v[i] && u < e));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = i * 32 + lane;
    if (e < E && v[i] == v[i] && rank[i] < k) {
      idx[rank[i]] = e;
      rank_lg[rank[i]] = v[i];
    }
  }
  __syncwarp();
  const int my_idx = lane < k ? idx[lane] : -1;
  const float my_logit = (lane < k && my_idx >= 0) ? rank_lg[lane] : -INFINITY;
  const float first_logit = idx[0] >= 0 ? rank_lg[0] : -INFINITY;
  float s = 0.f;
  if (mode == BIGRIG_SOFTMAX_TOPK) {
    s = (lane < k) ? expf(my_logit - mx) / denom : 0.f;
    if (norm_topk) s = s / warp_sum(s);
  } else {
    const float ex = (lane < k) ? expf(my_logit - first_logit) : 0.f;
    s = ex / warp_sum(ex);
  }
  if (lane < k) sc[lane] = s;
  __syncwarp();
}

// Stable expert-sorted permutation of P <= 32 pairs by one warp.  Lane i holds pair i;
// its sorted position is the number of pairs (e_j, j) lexicographically below (e_i, i).
// Runs of equal experts become the segments; offsets[x] counts the pairs with expert < x.
// Negative ids mark padding rows and ids >= E are errors (counted in err); both sort
// last and are left out of the segments.
__device__ __forceinline__ void permute_warp(const int32_t* idx, int P, int E, int32_t* order,
                                             int32_t* inv, int32_t* offsets, int32_t* seg_expert,
                                             int32_t* seg_start, int32_t* num_seg, int32_t* err) {
  const int lane = threadIdx.x & 31;
  int e = lane < P ? idx[lane] : 0x7fffffff;
  const bool bad = lane < P && e >= E;
  const bool pad = lane < P && e < 0;       // padding row (expert-parallel dispatch)
  if (bad || pad) e = 0x7ffffffe;
  const unsigned nbad = __popc(__ballot_sync(0xffffffffu, bad));
  const unsigned nskip = __popc(__ballot_sync(0xffffffffu, bad || pad));
  if (lane == 0 && nbad && err) atomicAdd(err, static_cast<int>(nbad));
  int rank = 0;
  for (int j = 0; j < 32; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e, j);
    rank += (ej < e) || (ej == e && j < lane);
  }
  if (lane < P) {
    order[rank] = lane;
    inv[lane] = rank;
  }
  int se = 0x7fffffff;
  for (int j = 0; j < 32; ++j) {
    const int rj = __shfl_sync(0xffffffffu, rank, j);
    const int ej = __shfl_sync(0xffffffffu, e, j);
    if (rj == lane) se = ej;
  }
  const int prev = __shfl_up_sync(0xffffffffu, se, 1);
  const bool first = lane < P && se < E && (lane == 0 || prev != se);
  const unsigned firsts = __ballot_sync(0xffffffffu, first);
  if (first) {
    const int si = __popc(firsts & ((1u << lane) - 1u));
    seg_expert[si] = se;
    seg_start[si] = lane;
  }
  if (lane == 0) {
    *num_seg = __popc(firsts);
    seg_start[__popc(firsts)] = P - static_cast<int>(nskip);
  }
  for (int x0 = 0; x0 <= E; x0 += 32) {          // uniform trip count: every lane shuffles
    const int x = x0 + lane;
    int below = 0;
    for (int j = 0; j < P; ++j) below += __shfl_sync(0xffffffffu, e, j) < x;
    if (x <= E) offsets[x] = below;
  }
}

// Programmatic dependent launch: wait for the preceding kernel's results (a no-op when
// the kernel was launched without the attribute), and let the next kernel be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

}  // namespace bigrig
