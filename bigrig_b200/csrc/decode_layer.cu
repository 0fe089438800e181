// One decode token through one MoE layer in ONE persistent cooperative kernel.
//
// Replaces, for a single token, the launch chain route -> gate_up -> down+combine
// (decode.cu, gemv.cu), and with it the mlx_lm block's router, the per-expert
// quantized_matmul calls of _forward_views_one (bigrig_engine/stream.py:1278-1318) and
// the caller's weighted sum (stream.py:1523-1525).  An OLMoE decode layer moves ~28 MB,
// ~4 us of HBM time.  One CTA per SM runs the whole layer with 16 consumer warps and
// one producer warp:
//
//   logits   CTA c < ceil(E/4) computes the logits of experts 4c..4c+3 (one warp each,
//            router rows bulk-copied as the kernel starts) and publishes each as a
//            64-bit (value, tag) word, the tag naming this launch -- no fence, no counter
//   routing  the producer warp of every CTA polls the E tagged words, ranks them
//            (topk_rank_warp: the chain's indices and scores bit for bit) and reads the
//            slots from a copy of g2s staged at start
//   gate/up  items of (routed expert, 8 features), dealt round-robin to CTAs and
//            streamed by the producer through a ring of tensor-map (or bulk) copies with
//            full / empty mbarriers.  As an item lands, 8 or 16 consumer warps take their
//            slices of its hidden dimension (with 8, the two halves of the consumers take
//            alternate items), on the tensor cores: warp-level bf16 MMAs (m16n8k16)
//            whose 16 rows are the item's 8 gate and 8 up rows, A converted in registers
//            from the codes to exact bf16 integers q, B the token; after the last item
//            the partials of every row are added in warp order and h written.
//   barrier  grid-wide, consumer threads only (the producer is already streaming the
//            down-projection weights into the ring)
//   down     items of (16 hidden features, a group of routed experts), a pair of warps
//            per expert of an item (each half of the intermediate dimension), the same
//            MMAs with h as B; then the combine in rank order plus the residual
//
// Group affine.  w = s q + b per group of 64 inputs, so sum_k w_k x_k = s sum(q x) +
// b sum(x) per group.  The MMA's 8 output columns keep 8 groups apart: B's column c
// holds the token's values for the group whose window position is c and zeros
// elsewhere, so column c of the accumulator is that group's sum(q x); every 8 groups
// the accumulator is scaled by s in fp32, b sum(x) is added and the columns restart.
// Products q x are exact, sums fp32: the precision of the fp32 GEMV in a different
// summation order.  Rounding points are the chain's: gate/up fp32, h bf16, each
// expert's y bf16, the combine fp32 in rank order.
//
// Every wait -- mbarriers, tagged logits, the grid barrier -- is bounded; a timeout
// counts in the error words and the kernel carries on to its end.
#include <cuda.h>

#include <atomic>
#include <cstring>

#include "gemv_common.cuh"
#include "routing.cuh"

// Phase-boundary hooks (DL_STAMP: thread 0 of each CTA; DL_WSTAMP: lane 0 of each warp);
// empty in the library, defined by instrumented builds that record timestamps.
#ifndef DL_STAMP
#define DL_STAMP(i)
#endif
#ifndef DL_WSTAMP
#define DL_WSTAMP(i)
#endif

namespace bigrig {

constexpr int kDlFeat = 8;               // features of a gate/up item (x2: its gate and up rows)
constexpr int kDlFeatDown = 16;          // hidden features of a down tile (the MMA's 16 rows)
constexpr int kDlRouterPerCta = 4;       // experts whose logits one CTA computes
constexpr int kDlMaxStages = 12;
constexpr int kDlCW = 16;                // consumer warps
constexpr int kDlGroup = 64;             // quantisation group size the kernel is built for
// Polls of a flag or of the grid barrier before a wait gives up (error word 1): ~0.5 s.
constexpr uint32_t kDlSpinLimit = 1u << 20;

struct DecodeLayerArgs {
  const uint16_t* x;          // [H] bf16
  const uint16_t* gate_w;     // [E, H] bf16
  const float* gate_b;        // [E] or null
  const int32_t* g2s;         // [E] or null
  const uint8_t* slab;
  bigrig_expert_layout L;
  const uint16_t* residual;   // [H] or null
  uint16_t* out;              // [H]
  int32_t* idx_out;           // [k]
  float* sc_out;              // [k]
  const int32_t* pre_idx;     // [k] routing computed before the launch, or null: route here
  const float* pre_sc;        // [k] its scores
  uint16_t* h;                // [k, I] scratch, rank-ordered rows
  unsigned long long* tagged; // [E] logit bits | tag << 32
  unsigned long long* arrivals;  // grid-barrier arrivals over all launches
  int32_t* err;
  int E, k, mode, norm;
  int stage_bytes, nstages, seg_per_item, max_tiles, max_items, ksplit;
  int seg_stride;             // bytes between a down item's expert segments in a stage
  int wpi;                    // consumer warps per gate/up item (8 or 16)
  int maps;                   // kDlMapGateUp | kDlMapDown: which copies go through tensor maps
  uint32_t spin_limit;        // polls before a flag or barrier wait gives up
  uint32_t phantom;           // CTAs the grid barrier waits for beyond the grid (tests only)
};

// The copy engine takes one copy at a time, at a cost per copy that the small scale and
// bias rows do not amortise.  Tensor maps over the slab fetch what the bulk path needs six
// copies for in two (an item's gate and up codes in one box; its gate and up scales and
// biases in another) and a down segment's scales and biases in one.
constexpr int kDlMapGateUp = 1;
constexpr int kDlMapDown = 2;

__device__ __forceinline__ void tma4_g2s_hint(void* dst, const CUtensorMap* m, int c0, int c1, int c2,
                                              int c3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma5_g2s_hint(void* dst, const CUtensorMap* m, int c0, int c1, int c2,
                                              int c3, int c4, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Wait for a ring stage; after a timeout, wait once more (bounded) so that the stage's
// copies are not still landing when the kernel moves on.
__device__ __forceinline__ bool stage_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (bar_wait(bar, parity, err)) return true;
  bar_wait(bar, parity, nullptr);
  return false;
}

// ------------------------------------------------------------------ MMA building blocks
// D[16x8] += A[16x16] B[16x8], bf16 inputs, fp32 accumulators.  Lane (g = lane/4,
// t = lane%4) holds A rows g and g+8 at k-slots {2t, 2t+1} (a0 / a1) and {2t+8, 2t+9}
// (a2 / a3), B column g at k-slots {2t, 2t+1} (b0) and {2t+8, 2t+9} (b1), and D rows g
// and g+8 at columns {2t, 2t+1}.  The lower half of a register is the lower k-slot.
__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two 4-bit fields -- bits 0-3 and 16-19 of v -- as an exact bf16x2 pair: OR-ed into the
// mantissa of 128.0 they read 128 + q, and subtracting 128 leaves q.
__device__ __forceinline__ uint32_t nibble_pair(uint32_t v) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(r) : "r"(v));
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(r), "r"(0x43004300u));
  return r;
}

// Code layout of a k-block (the K a lane's 16-byte chunk of a row covers, times 4 lanes):
//   4-bit: 128 K (2 groups), 8 k-steps; lane t owns words 4t..4t+3 = K [32t, 32t+32);
//          k-step s uses word s/2: slots {2t,2t+1} <- codes (j, j+4), {2t+8,2t+9} <-
//          codes (j+1, j+5) of the word, j = 2 (s%2)
//   8-bit: 64 K (1 group), 4 k-steps; lane t owns K [16t, 16t+16); k-step s uses word s:
//          slots {2t,2t+1} <- codes (0, 2), {2t+8,2t+9} <- codes (1, 3), low nibbles in
//          one MMA and high nibbles in another (whose sum counts 16x)
template <int BITS>
struct KBlock {
  static constexpr int K = BITS == 4 ? 128 : 64;
  static constexpr int STEPS = BITS == 4 ? 8 : 4;
  static constexpr int GROUPS = K / kDlGroup;
  static constexpr int BYTES = K * BITS / 8;   // bytes of one row in one k-block
};

// The K indices (within the k-block) of the lower and upper halves of a lane's k-slot
// pair: pair 0 is slots {2t, 2t+1}, pair 1 is {2t+8, 2t+9}.
template <int BITS>
__device__ __forceinline__ void slot_k(int t, int s, int pair, int& k_lo, int& k_hi) {
  if constexpr (BITS == 4) {
    const int base = 32 * t + 8 * (s >> 1) + 2 * (s & 1) + pair;
    k_lo = base;
    k_hi = base + 4;
  } else {
    const int base = 16 * t + 4 * s + pair;
    k_lo = base;
    k_hi = base + 2;
  }
}

// Most k-blocks of the hidden dimension one consumer warp owns in the gate/up phase (its
// B fragments live in registers): 16 warps x this covers H = 4096.
template <int BITS>
constexpr int kDlMaxSliceBlocks = BITS == 4 ? 2 : 4;

// One k-block of 16 rows against B fragments held in registers: gate rows g from wg,
// up rows g+8 from wu (the lane's 16-byte chunk of each).
template <int BITS>
__device__ __forceinline__ void mma_block(float* d, float* dh, const uint4 wg, const uint4 wu,
                                          const uint2* b) {
  using KB = KBlock<BITS>;
  const uint32_t gw[4] = {wg.x, wg.y, wg.z, wg.w};
  const uint32_t uw[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
  for (int s = 0; s < KB::STEPS; ++s) {
    if constexpr (BITS == 4) {
      const uint32_t G = gw[s >> 1], U = uw[s >> 1];
      const int sh = 8 * (s & 1);
      // even and odd k-steps in two accumulators: two dependent MMA chains of half the
      // length (the caller adds them)
      mma_bf16_16816((s & 1) ? dh : d, nibble_pair(G >> sh), nibble_pair(U >> sh),
                     nibble_pair(G >> (sh + 4)), nibble_pair(U >> (sh + 4)), b[s].x, b[s].y);
    } else {
      const uint32_t G = gw[s], U = uw[s];
      mma_bf16_16816(d, nibble_pair(G), nibble_pair(U), nibble_pair(G >> 8), nibble_pair(U >> 8),
                     b[s].x, b[s].y);
      mma_bf16_16816(dh, nibble_pair(G >> 4), nibble_pair(U >> 4), nibble_pair(G >> 12),
                     nibble_pair(U >> 12), b[s].x, b[s].y);
    }
  }
}

// nr rows of length K (row r at src + r * K) re-laid as B fragments: row r's (b0, b1) of
// k-step s of k-block blk for lane t at perm[r * rstride + (blk * STEPS + s) * 4 + t], plus
// the fp32 sum of each group of 64 at gsum[r * (K / 64) + group] (eight lanes per group,
// a fixed shuffle tree).  Threads tid < nthr (whole warps) take part.
template <int BITS>
__device__ __forceinline__ void build_bperm(const uint16_t* __restrict__ src, int K, int nr,
                                            uint2* __restrict__ perm, int rstride,
                                            float* __restrict__ gsum, int tid, int nthr) {
  using KB = KBlock<BITS>;
  const int nblk = (K + KB::K - 1) / KB::K;
  const int per_row = nblk * KB::STEPS * 4;
  for (int i = tid; i < nr * per_row; i += nthr) {
    const int r = i / per_row, j = i - r * per_row;
    const int t = j & 3, s = (j >> 2) % KB::STEPS, blk = (j >> 2) / KB::STEPS;
    const uint16_t* row = src + static_cast<size_t>(r) * K;
    uint32_t b[2];
#pragma unroll
    for (int pair = 0; pair < 2; ++pair) {
      int klo, khi;
      slot_k<BITS>(t, s, pair, klo, khi);
      klo += blk * KB::K;
      khi += blk * KB::K;
      const uint32_t lo = klo < K ? row[klo] : 0u;
      const uint32_t hi = khi < K ? row[khi] : 0u;
      b[pair] = lo | (hi << 16);
    }
    perm[static_cast<size_t>(r) * rstride + j] = make_uint2(b[0], b[1]);
  }
  // group sums: lane l of an 8-lane team adds elements 8l..8l+7 of its group
  const int ng = K / kDlGroup;
  const int total = nr * ng * 8;
  for (int base = 0; base < total; base += nthr) {
    const int i = base + tid;
    float v = 0.f;
    if (i < total) {
      const int grp = i >> 3, l = i & 7;
      const uint4 raw = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(grp) * kDlGroup + 8 * l);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        v += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xffff0000u);
    }
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    if (i < total && (i & 7) == 0) gsum[i >> 3] = v;
  }
}

// One warp's share of an MMA GEMV over k-blocks [blk0, blk1) of 16 rows whose codes start
// at rows_g (rows g) and rows_u (rows g+8).  Scales / biases of row r, group G at
// sc[r * ng + G] / bi[r * ng + G] (rows g: sc_g / bi_g, rows g+8: sc_u / bi_u).  Returns
// the lane's fp32 partial sums of rows g (x) and g+8 (y) over its groups; the caller adds
// the four lanes of a row.  Not inlined: the gate/up and the down phase run the same
// instructions, so the second finds them in the instruction cache.
template <int BITS, int SDT>
__device__ __noinline__ float2 mma_rows(const uint8_t* rows_g, const uint8_t* rows_u, int pitch,
                                        const uint16_t* sc_g, const uint16_t* bi_g,
                                        const uint16_t* sc_u, const uint16_t* bi_u, int ng,
                                        const uint2* __restrict__ bperm,
                                        const float* __restrict__ gsum, int blk0, int blk1) {
  constexpr bool TWO = true;
  using KB = KBlock<BITS>;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint8_t* rg = rows_g + g * pitch + 16 * t;
  const uint8_t* ru = TWO ? rows_u + g * pitch + 16 * t : nullptr;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  float dh[4] = {0.f, 0.f, 0.f, 0.f};            // 8-bit: high-nibble sums; 4-bit: odd k-steps
  int wstart = blk0 * KB::GROUPS;                // first group of the open column window
  float pg = 0.f, pu = 0.f;
  auto flush = [&](int wend) {
    // columns 2t, 2t+1 of the window [wstart, wend)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int G = wstart + 2 * t + c;
      if (G < wend) {
        const float vg = BITS == 4 ? d[c] + dh[c] : fmaf(16.f, dh[c], d[c]);
        const float vu = BITS == 4 ? d[2 + c] + dh[2 + c] : fmaf(16.f, dh[2 + c], d[2 + c]);
        const float xs = gsum[G];
        pg = fmaf(half_to_f32<SDT>(sc_g[g * ng + G]), vg, fmaf(half_to_f32<SDT>(bi_g[g * ng + G]), xs, pg));
        if (TWO)
          pu = fmaf(half_to_f32<SDT>(sc_u[g * ng + G]), vu, fmaf(half_to_f32<SDT>(bi_u[g * ng + G]), xs, pu));
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = dh[i] = 0.f;
    wstart = wend;
  };
  for (int blk = blk0; blk < blk1; ++blk) {
    const int g_lane = blk * KB::GROUPS + (BITS == 4 ? (t >> 1) : 0);   // group of this lane's K
    const bool live = g_lane < ng;
    uint4 wg = make_uint4(0, 0, 0, 0), wu = make_uint4(0, 0, 0, 0);
    if (live) {
      wg = *reinterpret_cast<const uint4*>(rg + blk * KB::BYTES);
      if (TWO) wu = *reinterpret_cast<const uint4*>(ru + blk * KB::BYTES);
    }
    const int col = g_lane - wstart;             // this lane's B column in the window
    const uint32_t gw[4] = {wg.x, wg.y, wg.z, wg.w};
    const uint32_t uw[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
    for (int s = 0; s < KB::STEPS; ++s) {
      uint2 b = make_uint2(0u, 0u);
      if (live && g == col) b = bperm[(blk * KB::STEPS + s) * 4 + t];
      if constexpr (BITS == 4) {
        const uint32_t G = gw[s >> 1], U = uw[s >> 1];
        const int sh = 8 * (s & 1);
        const uint32_t a0 = nibble_pair(G >> sh), a2 = nibble_pair(G >> (sh + 4));
        const uint32_t a1 = TWO ? nibble_pair(U >> sh) : 0u, a3 = TWO ? nibble_pair(U >> (sh + 4)) : 0u;
        mma_bf16_16816((s & 1) ? dh : d, a0, a1, a2, a3, b.x, b.y);   // two chains, as mma_block
      } else {
        const uint32_t G = gw[s], U = uw[s];
        const uint32_t l0 = nibble_pair(G), l2 = nibble_pair(G >> 8);
        const uint32_t h0 = nibble_pair(G >> 4), h2 = nibble_pair(G >> 12);
        const uint32_t l1 = TWO ? nibble_pair(U) : 0u, l3 = TWO ? nibble_pair(U >> 8) : 0u;
        const uint32_t h1 = TWO ? nibble_pair(U >> 4) : 0u, h3 = TWO ? nibble_pair(U >> 12) : 0u;
        mma_bf16_16816(d, l0, l1, l2, l3, b.x, b.y);
        mma_bf16_16816(dh, h0, h1, h2, h3, b.x, b.y);
      }
    }
    const int gnext = (blk + 1) * KB::GROUPS;
    if (gnext - wstart >= 8 || blk + 1 == blk1) flush(min(gnext, ng));
  }
  return make_float2(pg, pu);
}

template <int BITS, int SDT>
__global__ void __launch_bounds__((kDlCW + 1) * 32, 1) decode_layer_kernel(
    DecodeLayerArgs a, const __grid_constant__ CUtensorMap tm_code,
    const __grid_constant__ CUtensorMap tm_gsb, const __grid_constant__ CUtensorMap tm_dsb) {
  using KB = KBlock<BITS>;
  constexpr int NF = kDlFeat;
  constexpr int ND = kDlFeatDown;
  constexpr int CW = kDlCW;
  constexpr int CT = CW * 32;              // consumer threads
  constexpr int MAXNB = kDlMaxSliceBlocks<BITS>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(16) float s_lg[kMaxExperts];
  __shared__ int32_t s_g2s[kMaxExperts];
  __shared__ int32_t s_idx[32], s_slot[32];
  __shared__ float s_sc[32], s_rank_lg[32];
  __shared__ unsigned long long s_epoch;
  __shared__ float s_resid[2 * kDlFeatDown];     // the combine's residual values
  const bigrig_expert_layout& L = a.L;
  const int H = L.hidden, I = L.inter, E = a.E, k = a.k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool producer = warp == CW;
  const int G = gridDim.x, cta = blockIdx.x;
  const int pitch_h = H * BITS / 8, pitch_i = I * BITS / 8;
  const int gh = H / kDlGroup, gi = I / kDlGroup;
  const int nblk_h = (gh + KB::GROUPS - 1) / KB::GROUPS, nblk_i = (gi + KB::GROUPS - 1) / KB::GROUPS;
  const int nst = a.nstages, stage_bytes = a.stage_bytes;
  const int ksplit = a.ksplit;                   // warps per routed expert in the down phase

  const int tiles_g = I / NF;
  const int n_items = k * tiles_g;
  const int my_items = cta < n_items ? (n_items - 1 - cta) / G + 1 : 0;
  const int tiles_d = H / ND;
  const int my_tiles = cta < tiles_d ? (tiles_d - 1 - cta) / G + 1 : 0;
  const int spi = a.seg_per_item;
  const int ipt = (k + spi - 1) / spi;           // down items per tile
  const int n_down = my_tiles * ipt;
  const int item_bytes = 2 * NF * pitch_h + 4 * NF * gh * 2;
  const int seg_bytes = ND * pitch_i + 2 * ND * gi * 2;
  const int seg_stride = a.seg_stride;

  // tensor-map copies land at 128-byte aligned addresses: every carved buffer, the stage
  // size and the segment stride are multiples of 128
  SmemCarve sc(smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u));
  uint64_t* bars = sc.take<uint64_t>((2 * kDlMaxStages + 4) * 8);
  uint16_t* xraw = sc.take<uint16_t>(static_cast<size_t>(H) * 2);
  uint2* xperm = sc.take<uint2>(static_cast<size_t>(nblk_h) * KB::STEPS * 4 * 8);
  float* xgs = sc.take<float>(static_cast<size_t>(gh) * 4);
  uint16_t* hraw = sc.take<uint16_t>(static_cast<size_t>(k) * I * 2);
  uint2* hperm = sc.take<uint2>(static_cast<size_t>(k) * nblk_i * KB::STEPS * 4 * 8);
  float* hgs = sc.take<float>(static_cast<size_t>(k) * gi * 4);
  float2* gpart = sc.take<float2>(static_cast<size_t>(a.max_items) * CW * NF * 8);
  float2* dpart = sc.take<float2>(static_cast<size_t>(a.max_tiles) * k * ksplit * 8 * 8);
  uint8_t* ring = sc.take<uint8_t>(static_cast<size_t>(nst) * stage_bytes);
  uint16_t* wr = reinterpret_cast<uint16_t*>(ring);     // router rows, before any item
  uint64_t* full = bars;
  uint64_t* empty = bars + kDlMaxStages;
  uint64_t* bar_x = bars + 2 * kDlMaxStages;
  uint64_t* bar_r = bar_x + 1;
  uint64_t* bar_h = bar_x + 2;
  uint64_t* bar_s = bar_x + 3;                   // scores written (for the combine)
  DL_STAMP(0);

  // ---------------------------------------------------------------- start
  const bool routed = a.pre_idx != nullptr;      // routing given: no logits, no ranking
  const int n_mine = routed ? 0 : max(0, min(kDlRouterPerCta, E - cta * kDlRouterPerCta));
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      bar_init(full + i, 1);
      bar_init(empty + i, CW);
    }
    bar_init(bar_x, 1);
    bar_init(bar_r, 1);
    bar_init(bar_h, 1);
    bar_init(bar_s, 1);
    bar_expect_tx(bar_x, H * 2);
    bulk_g2s(xraw, a.x, H * 2, bar_x);
    if (n_mine > 0) {
      // router rows are read every step: keep them in L2 against the streamed experts
      bar_expect_tx(bar_r, static_cast<uint32_t>(n_mine) * H * 2);
      bulk_g2s_hint(wr, a.gate_w + static_cast<size_t>(cta) * kDlRouterPerCta * H, n_mine * H * 2,
                    bar_r, l2_evict_last());
    }
  }
  if (producer) {
    // this launch's index: the barrier arrivals of all earlier launches over G (arrivals
    // of this launch that are already in add fewer than G)
    if (lane == 0) s_epoch = ld_acquire_u64(a.arrivals) / static_cast<unsigned long long>(G);
    if (lane == 1 && (a.maps & kDlMapGateUp)) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_code)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_gsb)) : "memory");
    }
    if (lane == 2 && (a.maps & kDlMapDown))
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_dsb)) : "memory");
    for (int e = lane; e < E; e += 32) s_g2s[e] = a.g2s ? a.g2s[e] : e;
  }
  if (threadIdx.x < 32) s_idx[threadIdx.x] = -1;
  __syncthreads();
  const unsigned long long epoch = s_epoch;
  const unsigned long long tag = ((epoch + 1ull) & 0xffffffffull) << 32;

  bool xok = true;
  if (routed) {
    // ------------------------------------------------------------ routing given
    // the producer reads it and starts streaming at once; the consumers meanwhile take x
    // into B fragments and pick up the routing from an mbarrier the producer arrives on
    if (producer) {
      if (lane < k) {
        const int e = a.pre_idx[lane];
        const int ev = (e >= 0 && e < E) ? e : -1;
        s_idx[lane] = ev;
        s_slot[lane] = ev >= 0 ? s_g2s[ev] : -1;
      }
      __syncwarp();
      if (lane == 0) bar_arrive(bar_r);
    } else {
      xok = stage_wait(bar_x, 0, a.err);
      build_bperm<BITS>(xraw, H, 1, xperm, 0, xgs, threadIdx.x, CT);
      named_sync(1, CT);
      stage_wait(bar_r, 0, a.err);
    }
    DL_STAMP(1);
  } else {                                       // routing computed here, from x
  // ---------------------------------------------------------------- router logits
  if (!producer) {
    xok = stage_wait(bar_x, 0, a.err);
    if (warp < n_mine) {
      const bool rok = stage_wait(bar_r, 0, a.err);
      const uint16_t* w = wr + static_cast<size_t>(warp) * H;
      float acc = 0.f;
      for (int c = lane * 8; c < H; c += 32 * 8) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xraw + c);
        const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
        const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w};
        const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc = fmaf(__uint_as_float(xa[i] << 16), __uint_as_float(wa[i] << 16), acc);
          acc = fmaf(__uint_as_float(xa[i] & 0xffff0000u), __uint_as_float(wa[i] & 0xffff0000u), acc);
        }
      }
      acc = warp_sum(acc);
      const int e = cta * kDlRouterPerCta + warp;
      // a logit that could not be computed is published as NaN: never selected
      const float v = (xok && rok) ? acc + (a.gate_b ? a.gate_b[e] : 0.f) : __int_as_float(0x7fc00000);
      if (lane == 0) st_relaxed_u64(a.tagged + e, tag | __float_as_uint(v));
    }
  }
  __syncthreads();                               // router rows read: the ring is free
  DL_STAMP(1);

  // ---------------------------------------------------------------- routing
  // the producer collects the E tagged logits; every consumer thread then ranks (logit
  // descending, expert id ascending -- topk_warp's order) a share of them: 8 threads per
  // candidate, each counting the candidates above it among E/8 others
  if (producer) {
    uint32_t need = 0;
    for (int e = lane, i = 0; e < E; e += 32, ++i) need |= 1u << i;
    for (uint32_t n = 0; need; ++n) {
#pragma unroll
      for (int i = 0; i < kMaxExperts / 32; ++i) {
        if (need & (1u << i)) {
          const int e = lane + 32 * i;
          const unsigned long long v = ld_relaxed_u64(a.tagged + e);
          if ((v & 0xffffffff00000000ull) == tag) {
            s_lg[e] = __uint_as_float(static_cast<uint32_t>(v));
            need &= ~(1u << i);
          }
        }
      }
      if (n > a.spin_limit) {
        if (lane == 0) atomicAdd(a.err + 1, 1);
        for (int i = 0; i < kMaxExperts / 32; ++i)
          if (need & (1u << i)) s_lg[lane + 32 * i] = __int_as_float(0x7fc00000);
        break;
      }
    }
    __syncwarp();
    DL_STAMP(8);
  } else {
    build_bperm<BITS>(xraw, H, 1, xperm, 0, xgs, threadIdx.x, CT);
  }
  __syncthreads();                               // logits in s_lg
  if (!producer) {
    const int per_cand = (E + 7) / 8;
    for (int c0 = 0; c0 < E; c0 += CT / 8) {
      const int c = c0 + (threadIdx.x >> 3), part = threadIdx.x & 7;
      int r = 0;
      float v = 0.f;
      if (c < E) {
        v = s_lg[c];
        const int u0 = part * per_cand, u1 = min(E, u0 + per_cand);
        for (int u = u0; u < u1; ++u) {
          const float w = s_lg[u];
          r += (w > v) || (w == v && u < c);
        }
      }
      r += __shfl_xor_sync(0xffffffffu, r, 1);
      r += __shfl_xor_sync(0xffffffffu, r, 2);
      r += __shfl_xor_sync(0xffffffffu, r, 4);
      if (c < E && part == 0 && v == v && r < k) {   // NaN logits are never selected
        s_idx[r] = c;
        s_rank_lg[r] = v;
      }
    }
  }
  __syncthreads();                               // ranks in s_idx / s_rank_lg
  if (producer) {
    DL_STAMP(9);
    if (lane < k) {
      const int e = s_idx[lane];
      s_slot[lane] = (e >= 0 && e < E) ? s_g2s[e] : -1;
    }
    __syncwarp();
  }
  }                                              // end of the routing computed here

  if (producer) {
    // ------------------------------------------------------------ stream the ring
    // the first stages go out at once; then the scores (needed only by the combine);
    // then the rest as stages free up
    const int total = my_items + n_down;
    const int first = min(nst, total);
    const uint64_t once = l2_evict_first();     // expert weights: read once per token
    // one ring stage: lane 0 arms the barrier, then the stage's copies go out in one warp
    // instruction per kind, a lane per copy (a gate/up item is two tensor-map boxes or six
    // bulk copies: codes, scales, biases of gate and up; a down item per routed expert
    // its codes plus one box or two bulk copies of scales and biases)
    auto issue = [&](int q) {
      const int b = q % nst;
      if (q >= nst) stage_wait(empty + b, ((q / nst) - 1) & 1, a.err);
      if (q < 16) DL_WSTAMP(16 + q);
      uint8_t* dst = ring + static_cast<size_t>(b) * stage_bytes;
      if (q < my_items) {
        const int it = cta + q * G;
        const int s = it / tiles_g, f0 = (it - s * tiles_g) * NF;
        const int slot = s_slot[s];
        if (lane == 0) bar_expect_tx(full + b, slot >= 0 ? static_cast<uint32_t>(item_bytes) : 0u);
        __syncwarp();
        if (slot >= 0 && (a.maps & kDlMapGateUp)) {
          // [proj][row][code bytes] and [proj][scales, biases][8-row block] boxes
          if (lane == 0) tma4_g2s_hint(dst, &tm_code, 0, f0, 0, slot, full + b, once);
          if (lane == 1)
            tma5_g2s_hint(dst + 2 * NF * pitch_h, &tm_gsb, 0, f0 / NF, 0, 0, slot, full + b, once);
        } else if (slot >= 0 && lane < 6) {
          const uint8_t* base = a.slab + static_cast<int64_t>(slot) * L.slot_stride;
          const int m = lane / 3, part = lane % 3;   // projection; codes / scales / biases
          const uint8_t* src;
          uint8_t* d;
          uint32_t bytes;
          if (part == 0) {
            src = base + L.weight_off[m] + static_cast<int64_t>(f0) * pitch_h;
            d = dst + m * NF * pitch_h;
            bytes = NF * pitch_h;
          } else {
            const int64_t off = part == 1 ? L.scales_off[m] : L.biases_off[m];
            src = base + off + static_cast<int64_t>(f0) * gh * 2;
            d = dst + 2 * NF * pitch_h + (2 * m + part - 1) * NF * gh * 2;
            bytes = NF * gh * 2;
          }
          bulk_g2s_hint(d, src, bytes, full + b, once);
        }
      } else {
        const int d = q - my_items;
        const int f0 = (cta + (d / ipt) * G) * ND;
        const int s0 = (d % ipt) * spi, s1 = min(k, s0 + spi);
        uint32_t bytes = 0;
        for (int s = s0; s < s1; ++s) bytes += s_slot[s] >= 0 ? seg_bytes : 0;
        if (lane == 0) bar_expect_tx(full + b, bytes);
        __syncwarp();
        const int per = (a.maps & kDlMapDown) ? 2 : 3;   // copies per routed expert
        for (int c = lane; c < per * (s1 - s0); c += 32) {
          const int s = s0 + c / per, part = c % per;
          const int slot = s_slot[s];
          if (slot < 0) continue;
          const uint8_t* base = a.slab + static_cast<int64_t>(slot) * L.slot_stride;
          uint8_t* dd = dst + static_cast<size_t>(s - s0) * seg_stride;
          if (part == 0)
            bulk_g2s_hint(dd, base + L.weight_off[2] + static_cast<int64_t>(f0) * pitch_i,
                          ND * pitch_i, full + b, once);
          else if (per == 2)                           // [scales, biases][16-row block]
            tma4_g2s_hint(dd + ND * pitch_i, &tm_dsb, 0, f0 / ND, 0, slot, full + b, once);
          else
            bulk_g2s_hint(dd + ND * pitch_i + (part - 1) * ND * gi * 2,
                          base + (part == 1 ? L.scales_off[2] : L.biases_off[2]) +
                              static_cast<int64_t>(f0) * gi * 2,
                          ND * gi * 2, full + b, once);
        }
      }
      __syncwarp();
    };
    for (int q = 0; q < first; ++q) issue(q);
    DL_STAMP(2);
    // scores: given, or topk_warp's formulas and reductions over the same values in the
    // same lanes
    if (routed) {
      if (lane < k) {
        s_sc[lane] = a.pre_sc[lane];
        if (cta == 0) {
          if (a.idx_out != a.pre_idx) a.idx_out[lane] = s_idx[lane];
          if (a.sc_out != a.pre_sc) a.sc_out[lane] = s_sc[lane];
          if (s_slot[lane] < 0) atomicAdd(a.err, 1);
        }
      }
      __syncwarp();
      if (lane == 0) bar_arrive(bar_s);
    } else {
      const int per = (E + 31) / 32;
      float mx = -INFINITY;
      for (int i = 0; i < per; ++i)
        if (i * 32 + lane < E) mx = fmaxf(mx, s_lg[i * 32 + lane]);
      mx = warp_max(mx);
      const int my_idx = lane < k ? s_idx[lane] : -1;
      const float my_logit = (lane < k && my_idx >= 0) ? s_rank_lg[lane] : -INFINITY;
      const float first_logit = s_idx[0] >= 0 ? s_rank_lg[0] : -INFINITY;
      float sv = 0.f;
      if (a.mode == BIGRIG_SOFTMAX_TOPK) {
        float denom = 0.f;
        for (int i = 0; i < per; ++i)
          if (i * 32 + lane < E) denom += expf(s_lg[i * 32 + lane] - mx);
        denom = warp_sum(denom);
        sv = (lane < k) ? expf(my_logit - mx) / denom : 0.f;
        if (a.norm) sv = sv / warp_sum(sv);
      } else {
        const float ex = (lane < k) ? expf(my_logit - first_logit) : 0.f;
        sv = ex / warp_sum(ex);
      }
      if (lane < k) {
        s_sc[lane] = sv;
        if (cta == 0) {
          a.idx_out[lane] = my_idx;
          a.sc_out[lane] = sv;
          if (s_slot[lane] < 0) atomicAdd(a.err, 1);
        }
      }
      __syncwarp();
      if (lane == 0) bar_arrive(bar_s);
    }
    for (int q = first; q < total; ++q) issue(q);
    DL_STAMP(13);
    return;                                      // consumers wait for every stage it filled
  }

  // the combine's residual, fetched now (into shared memory, so the load completes
  // here) so that its latency hides behind the layer
  if (a.residual && threadIdx.x < my_tiles * ND) {
    const int tl = threadIdx.x / ND, f = threadIdx.x % ND;
    s_resid[threadIdx.x] = bf16_bits_to_f32(a.residual[(cta + tl * G) * ND + f]);
  }

  // ---------------------------------------------------------------- gate/up
  // consumer warp w owns k-blocks [kb0, kb1) of the hidden dimension in every item; its B
  // fragments (the token) stay in registers for all items.  Per item it leaves the partial
  // sums of the 8 gate and 8 up rows over its blocks; they are added after the last item.
  // with 8 warps per item (when a warp's share of the hidden dimension fits its registers)
  // the two halves of the consumers take alternate items: each warp runs twice the MMAs
  // per item for half the items, half the per-item waits and reductions
  const int wpi = a.wpi, ngrp = CW / wpi;
  const int wl = warp % wpi, grp = warp / wpi;
  const int kb0 = wl * nblk_h / wpi, kb1 = (wl + 1) * nblk_h / wpi;
  const int nb = kb1 - kb0;
  uint2 breg[MAXNB][KB::STEPS];
#pragma unroll
  for (int bi = 0; bi < MAXNB; ++bi) {
    const int blk = kb0 + bi;
    const int g_lane = blk * KB::GROUPS + (BITS == 4 ? (t >> 1) : 0);
    const bool use = bi < nb && g_lane < gh && g == g_lane - kb0 * KB::GROUPS;
#pragma unroll
    for (int s = 0; s < KB::STEPS; ++s)
      breg[bi][s] = use ? xperm[(blk * KB::STEPS + s) * 4 + t] : make_uint2(0u, 0u);
  }
  // the lane's two accumulator columns: groups kb0*GROUPS + 2t + {0, 1}
  const int gend = min(kb1 * KB::GROUPS, gh);
  int gcol[2];
  float xg[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    gcol[c] = kb0 * KB::GROUPS + 2 * t + c;
    xg[c] = gcol[c] < gend ? xgs[gcol[c]] : 0.f;
  }
  const uint8_t* goff = nullptr;                 // this lane's code bytes in a stage
  for (int j = 0; j < my_items; ++j) {
    const int b = j % nst;
    const bool landed = stage_wait(full + b, (j / nst) & 1, a.err);
    if (j == 0) DL_STAMP(3);
    if (j == 0) DL_WSTAMP(0);
    if (j % ngrp != grp) {                       // the other half's item: free the stage
      __syncwarp();
      if (lane == 0) bar_arrive(empty + b);
      continue;
    }
    const int it = cta + j * G;
    const int s = it / tiles_g;
    const bool have = s_slot[s] >= 0 && landed && xok;
    const uint8_t* st = ring + static_cast<size_t>(b) * stage_bytes;
    goff = st + g * pitch_h + 16 * t + kb0 * KB::BYTES;
    const uint16_t* sb = reinterpret_cast<const uint16_t*>(st + 2 * NF * pitch_h);
    float pg = 0.f, pu = 0.f;
    if (have && nb > 0) {
      float d[4] = {0.f, 0.f, 0.f, 0.f}, dh[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int bi = 0; bi < MAXNB; ++bi) {
        if (bi < nb) {
          const uint4 wg = *reinterpret_cast<const uint4*>(goff + bi * KB::BYTES);
          const uint4 wu = *reinterpret_cast<const uint4*>(goff + NF * pitch_h + bi * KB::BYTES);
          mma_block<BITS>(d, dh, wg, wu, breg[bi]);
        }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (gcol[c] < gend) {
          const int G0 = gcol[c];
          const float vg = BITS == 4 ? d[c] + dh[c] : fmaf(16.f, dh[c], d[c]);
          const float vu = BITS == 4 ? d[2 + c] + dh[2 + c] : fmaf(16.f, dh[2 + c], d[2 + c]);
          pg = fmaf(half_to_f32<SDT>(sb[(0 * NF + g) * gh + G0]), vg,
                    fmaf(half_to_f32<SDT>(sb[(1 * NF + g) * gh + G0]), xg[c], pg));
          pu = fmaf(half_to_f32<SDT>(sb[(2 * NF + g) * gh + G0]), vu,
                    fmaf(half_to_f32<SDT>(sb[(3 * NF + g) * gh + G0]), xg[c], pu));
        }
      }
    }
    pg += __shfl_xor_sync(0xffffffffu, pg, 1);
    pu += __shfl_xor_sync(0xffffffffu, pu, 1);
    pg += __shfl_xor_sync(0xffffffffu, pg, 2);
    pu += __shfl_xor_sync(0xffffffffu, pu, 2);
    if (t == 0) gpart[(j * wpi + wl) * NF + g] = make_float2(pg, pu);
    __syncwarp();
    if (lane == 0) bar_arrive(empty + b);        // stage b read by this warp
  }
  DL_STAMP(4);
  DL_WSTAMP(1);
  named_sync(1, CT);
  // h = bf16(silu(gate) * up), the wpi partials of each row added in warp order
  for (int i = threadIdx.x; i < my_items * NF; i += CT) {
    const int j = i / NF, f = i - j * NF;
    const int it = cta + j * G;
    const int s = it / tiles_g, f0 = (it - s * tiles_g) * NF;
    float gv = 0.f, uv = 0.f;
    for (int w = 0; w < wpi; ++w) {
      const float2 o = gpart[(j * wpi + w) * NF + f];
      gv += o.x;
      uv += o.y;
    }
    a.h[static_cast<size_t>(s) * I + f0 + f] = s_slot[s] >= 0 ? f32_to_bf16_bits(silu_f32(gv) * uv) : 0;
  }
  DL_STAMP(10);

  // ---------------------------------------------------------------- grid barrier
  named_sync(1, CT);
  if (threadIdx.x == 0) {
    // one-way release add (the CTA's h stores, ordered before it by the named barrier,
    // become visible with it), then acquire polls without a back-off
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(a.arrivals) : "memory");
    const unsigned long long target = (epoch + 1ull) * static_cast<unsigned long long>(G) + a.phantom;
    uint32_t n = 0;
    while (static_cast<long long>(ld_acquire_u64(a.arrivals) - target) < 0) {
      if (++n > a.spin_limit) {
        atomicAdd(a.err + 1, 1);
        break;
      }
    }
    fence_proxy_async_global();                  // h, written by other CTAs, is read by bulk copy
    if (n_down > 0) {
      bar_expect_tx(bar_h, static_cast<uint32_t>(k) * I * 2);
      bulk_g2s(hraw, a.h, k * I * 2, bar_h);
    }
  }
  // lanes 1-31 of warp 0 must not spin on bar_h beside lane 0's barrier spin: a warp
  // can run one side of a divergent spin for its whole bound before the other
  __syncwarp();
  DL_STAMP(5);
  if (n_down == 0) return;

  // ---------------------------------------------------------------- down + combine
  const bool hok = stage_wait(bar_h, 0, a.err);
  const int hstride = nblk_i * KB::STEPS * 4;
  build_bperm<BITS>(hraw, I, k, hperm, hstride, hgs, threadIdx.x, CT);
  named_sync(1, CT);
  DL_STAMP(6);
  // warp w takes routed expert s = w / ksplit (and s + CW / ksplit, ...) over k-blocks
  // [ks * nblk_i / ksplit, ...) of the intermediate dimension, ks = w % ksplit, in every
  // down tile of the CTA
  const int ks = warp % ksplit;
  const int db0 = ks * nblk_i / ksplit, db1 = (ks + 1) * nblk_i / ksplit;
  // When no down item refills a stage (n_down <= nst) nobody waits for the down stages to
  // be released: a warp waits only on the stages holding its experts, so all warps start
  // at once instead of walking the stages in order.  Otherwise every warp releases every
  // down stage in order (the producer refills them).
  const bool direct = n_down <= nst;
  for (int d = 0; d < n_down; ++d) {
    const int tl = d / ipt;
    const int s0 = (d % ipt) * spi, s1 = min(k, s0 + spi);
    if (direct) {
      bool mine = false;
      for (int s = warp / ksplit; s < k; s += CW / ksplit) mine |= s >= s0 && s < s1;
      if (!mine) continue;
    }
    const int q = my_items + d;
    const int b = q % nst;
    const bool landed = stage_wait(full + b, (q / nst) & 1, a.err) && hok;
    if (d == n_down - 1) DL_STAMP(14);
    if (d < 8) DL_WSTAMP(8 + d);
    for (int s = warp / ksplit; s < k; s += CW / ksplit) {
      if (s < s0 || s >= s1) continue;
      const bool have = s_slot[s] >= 0 && landed && db0 < db1;
      const uint8_t* wc = ring + static_cast<size_t>(b) * stage_bytes + static_cast<size_t>(s - s0) * seg_stride;
      const uint16_t* sb = reinterpret_cast<const uint16_t*>(wc + ND * pitch_i);
      float2 p = make_float2(0.f, 0.f);
      DL_WSTAMP(2);
      if (have)
        p = mma_rows<BITS, SDT>(wc, wc + 8 * pitch_i, pitch_i, sb, sb + ND * gi, sb + 8 * gi,
                                sb + ND * gi + 8 * gi, gi, hperm + static_cast<size_t>(s) * hstride,
                                hgs + s * gi, db0, db1);
      p.x += __shfl_xor_sync(0xffffffffu, p.x, 1);
      p.y += __shfl_xor_sync(0xffffffffu, p.y, 1);
      p.x += __shfl_xor_sync(0xffffffffu, p.x, 2);
      p.y += __shfl_xor_sync(0xffffffffu, p.y, 2);
      if (t == 0) dpart[((tl * k + s) * ksplit + ks) * 8 + g] = p;   // features g and g + 8
      DL_WSTAMP(3);
    }
    __syncwarp();
    if (!direct && lane == 0) bar_arrive(empty + b);
  }
  DL_STAMP(11);
  DL_WSTAMP(4);
  named_sync(1, CT);
  DL_STAMP(12);
  // combine in rank order, plus the residual; y of a routed expert is its k-split
  // partials added in order and rounded to bf16
  const bool scores = stage_wait(bar_s, 0, a.err);
  if (threadIdx.x < my_tiles * ND) {
    const int tl = threadIdx.x / ND, f = threadIdx.x % ND;
    const int o = (cta + tl * G) * ND + f;
    float acc = 0.f;
    for (int r = 0; r < k; ++r) {
      float y = 0.f;
      for (int q = 0; q < ksplit; ++q) {
        const float2 pp = dpart[((tl * k + r) * ksplit + q) * 8 + (f & 7)];
        y += f < 8 ? pp.x : pp.y;
      }
      y = s_slot[r] >= 0 ? bf16_round(y) : 0.f;
      acc = acc + (scores ? s_sc[r] : 0.f) * y;
    }
    if (a.residual) acc = s_resid[threadIdx.x] + bf16_round(acc);
    a.out[o] = f32_to_bf16_bits(acc);
  }
  DL_STAMP(7);
}

// ------------------------------------------------------------------ launcher
namespace {

// dynamic shared memory: the 227 KB a block may hold, less the kernel's static arrays
// (routing state) and a margin
constexpr size_t kDlSmemLimit = 222 * 1024;

int sm_count_dl() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms = n;
  }
  return sms;
}

struct DlPlan {
  int stage_bytes, nstages, seg_per_item, max_tiles, max_items, ksplit, seg_stride, wpi;
  size_t smem;
};

// The persistent kernel's plan for a layer, or false when it cannot run it: more than
// 32 routed experts, a quantisation group other than 64, a hidden dimension wider than
// 16 warps' register-held slices, a layer whose fixed shared memory leaves no room for a
// ring of two stages.
bool decode_layer_plan(const bigrig_expert_layout& L, int k, int E, int G, DlPlan* p) {
  if (G <= 0 || k > 32 || E > kMaxExperts || L.group_size != kDlGroup) return false;
  if (L.flags != 0) return false;   // gated SwiGLU without projection biases only: the
                                    // other shapes take the three-kernel chain
  if (L.hidden % kDlGroup || L.inter % kDlGroup || L.hidden % kDlFeatDown) return false;
  const int kb_k = L.bits == 4 ? 128 : 64, steps = L.bits == 4 ? 8 : 4;
  const int max_slice = L.bits == 4 ? kDlMaxSliceBlocks<4> : kDlMaxSliceBlocks<8>;
  const size_t gh = L.hidden / kDlGroup, gi = L.inter / kDlGroup;
  const size_t nblk_h = (L.hidden + kb_k - 1) / kb_k, nblk_i = (L.inter + kb_k - 1) / kb_k;
  if (nblk_h > static_cast<size_t>(kDlCW) * max_slice) return false;
  p->wpi = nblk_h <= static_cast<size_t>(kDlCW / 2) * max_slice ? kDlCW / 2 : kDlCW;
  const size_t ph = static_cast<size_t>(L.hidden) * L.bits / 8;
  const size_t pi = static_cast<size_t>(L.inter) * L.bits / 8;
  const size_t item = 2 * kDlFeat * ph + 4 * kDlFeat * gh * 2;
  const size_t seg = round128(kDlFeatDown * pi + 2 * kDlFeatDown * gi * 2);
  const size_t stage = round128(item > seg ? item : seg);
  int spi = static_cast<int>(stage / seg);
  if (spi > k) spi = k;
  int ksplit = 1;
  while (ksplit * 2 * k <= kDlCW) ksplit *= 2;   // warps per routed expert in the down phase
  const int tiles_d = L.hidden / kDlFeatDown;
  const int n_items = k * (L.inter / kDlFeat);
  p->max_tiles = (tiles_d + G - 1) / G;
  p->max_items = (n_items + G - 1) / G;
  p->ksplit = ksplit;
  // (the first 128 bytes: room to align the carve)
  const size_t fixed = 128 + round128((2 * kDlMaxStages + 4) * 8) + round128(L.hidden * 2) +
                       round128(nblk_h * steps * 4 * 8) + round128(gh * 4) +
                       round128(static_cast<size_t>(k) * L.inter * 2) +
                       round128(static_cast<size_t>(k) * nblk_i * steps * 4 * 8) +
                       round128(static_cast<size_t>(k) * gi * 4) +
                       round128(static_cast<size_t>(p->max_items) * kDlCW * kDlFeat * 8) +
                       round128(static_cast<size_t>(p->max_tiles) * k * ksplit * 8 * 8);
  if (fixed >= kDlSmemLimit) return false;
  size_t nst = (kDlSmemLimit - fixed) / stage;
  if (nst > static_cast<size_t>(kDlMaxStages)) nst = kDlMaxStages;
  if (nst < 2 || nst * stage < static_cast<size_t>(kDlRouterPerCta) * L.hidden * 2) return false;
  p->stage_bytes = static_cast<int>(stage);
  p->nstages = static_cast<int>(nst);
  p->seg_per_item = spi;
  p->seg_stride = static_cast<int>(seg);
  p->smem = fixed + nst * stage;
  return true;
}

using DlEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

DlEncodeFn dl_encode_fn() {
  static DlEncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<DlEncodeFn>(p);
  }
  return fn;
}

// Slots a map may address: the slab's extent is not passed in, and a box only touches the
// slot whose index it is given.
constexpr cuuint64_t kDlMapSlots = 1u << 16;

// A map of 8-byte elements over the slab, no swizzle, no fill.  False when the layout breaks
// a rule of tiled maps (16-byte aligned base and strides, at most 256 elements per box side)
// or the encoder refuses it.
bool dl_encode(CUtensorMap* m, int rank, const uint8_t* base, const cuuint64_t* dims,
               const cuuint64_t* strides, const cuuint32_t* box) {
  DlEncodeFn fn = dl_encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  for (int i = 0; i < rank; ++i)
    if (box[i] < 1 || box[i] > 256 || dims[i] < box[i]) return false;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] == 0 || (strides[i] & 15)) return false;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, static_cast<cuuint32_t>(rank), const_cast<uint8_t*>(base),
            dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The maps of a layer's slab (kDlMapGateUp / kDlMapDown of those it could build).
//   code  [8-byte words of a row][row][gate, up][slot], box: an item's 8 rows of both
//   gsb   [words of an 8-row block's scales][block][scales, biases][gate, up][slot]
//   dsb   [words of a 16-row block of down scales][block][scales, biases][slot]
// The slab keeps gate, up (and each projection's scales and biases) at fixed distances,
// which is what lets one box span them.
int dl_maps(const uint8_t* slab, const bigrig_expert_layout& L, CUtensorMap* code, CUtensorMap* gsb,
            CUtensorMap* dsb) {
  const int64_t ph = static_cast<int64_t>(L.hidden) * L.bits / 8;
  const int64_t gh = L.hidden / L.group_size, gi = L.inter / L.group_size;
  const int64_t pst = L.weight_off[1] - L.weight_off[0];
  const int64_t kst = L.biases_off[0] - L.scales_off[0];
  const int64_t dkst = L.biases_off[2] - L.scales_off[2];
  int maps = 0;
  if (ph % 8 == 0 && pst > 0 && kst > 0 && L.scales_off[1] - L.scales_off[0] == pst &&
      L.biases_off[1] - L.biases_off[0] == pst && L.weight_off[0] % 16 == 0 &&
      L.scales_off[0] % 16 == 0 && L.inter % kDlFeat == 0) {
    const cuuint64_t cd[4] = {static_cast<cuuint64_t>(ph / 8), static_cast<cuuint64_t>(L.inter), 2, kDlMapSlots};
    const cuuint64_t cs[3] = {static_cast<cuuint64_t>(ph), static_cast<cuuint64_t>(pst),
                              static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t cb[4] = {static_cast<cuuint32_t>(ph / 8), kDlFeat, 2, 1};
    const int64_t blk = kDlFeat * gh * 2;            // an 8-row block's scales, bytes
    const cuuint64_t sd[5] = {static_cast<cuuint64_t>(blk / 8), static_cast<cuuint64_t>(L.inter / kDlFeat), 2, 2,
                              kDlMapSlots};
    const cuuint64_t ss[4] = {static_cast<cuuint64_t>(blk), static_cast<cuuint64_t>(kst),
                              static_cast<cuuint64_t>(pst), static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t sb[5] = {static_cast<cuuint32_t>(blk / 8), 1, 2, 2, 1};
    if (dl_encode(code, 4, slab + L.weight_off[0], cd, cs, cb) &&
        dl_encode(gsb, 5, slab + L.scales_off[0], sd, ss, sb))
      maps |= kDlMapGateUp;
  }
  if (dkst > 0 && L.scales_off[2] % 16 == 0 && L.hidden % kDlFeatDown == 0) {
    const int64_t blk = kDlFeatDown * gi * 2;        // a 16-row block's scales, bytes
    const cuuint64_t dd[4] = {static_cast<cuuint64_t>(blk / 8), static_cast<cuuint64_t>(L.hidden / kDlFeatDown), 2,
                              kDlMapSlots};
    const cuuint64_t ds[3] = {static_cast<cuuint64_t>(blk), static_cast<cuuint64_t>(dkst),
                              static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t db[4] = {static_cast<cuuint32_t>(blk / 8), 1, 2, 1};
    if (dl_encode(dsb, 4, slab + L.scales_off[2], dd, ds, db)) maps |= kDlMapDown;
  }
  return maps;
}

template <int BITS, int SDT>
int dl_launch(const DecodeLayerArgs& args, const CUtensorMap& tm_code, const CUtensorMap& tm_gsb,
              const CUtensorMap& tm_dsb, size_t smem, int G, cudaStream_t s) {
  auto kern = decode_layer_kernel<BITS, SDT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "decode_layer: cannot reserve %zu bytes of smem", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3((kDlCW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TimedLaunch tl(BIGRIG_K_DECODE_LAYER, s);
  cudaLaunchKernelEx(&cfg, kern, args, tm_code, tm_gsb, tm_dsb);
  return check_launch("decode_layer_kernel");
}

}  // namespace

namespace {
std::atomic<uint32_t> g_dl_phantom{0};
std::atomic<uint32_t> g_dl_spin{kDlSpinLimit};
}  // namespace

void dl_wait_test(uint32_t* phantom, uint32_t* spin_limit) {
  *phantom = g_dl_phantom.load();
  *spin_limit = g_dl_spin.load();
}

void set_dl_wait_test(uint32_t phantom, uint32_t spin_limit) {
  g_dl_phantom.store(phantom);
  g_dl_spin.store(spin_limit ? spin_limit : kDlSpinLimit);
}

bool decode_layer_fits(const bigrig_expert_layout& L, int k, int E) {
  DlPlan p;
  return decode_layer_plan(L, k, E, sm_count_dl(), &p);
}

int launch_decode_layer(const void* x, const void* gate_w, const float* gate_b, int E, int k,
                        int mode, int norm, const int32_t* g2s, const void* slab,
                        const bigrig_expert_layout& L, const void* residual, void* out,
                        int32_t* idx_out, float* sc_out, void* h, void* tagged, void* arrivals,
                        int32_t* err, cudaStream_t s, const int32_t* pre_idx, const float* pre_sc) {
  const int G = sm_count_dl();
  DlPlan p;
  if (!decode_layer_plan(L, k, E, G, &p))
    return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_layer: layer does not fit one CTA");
  DecodeLayerArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.gate_w = static_cast<const uint16_t*>(gate_w);
  a.gate_b = gate_b;
  a.g2s = g2s;
  a.slab = static_cast<const uint8_t*>(slab);
  a.L = L;
  a.residual = static_cast<const uint16_t*>(residual);
  a.out = static_cast<uint16_t*>(out);
  a.idx_out = idx_out;
  a.sc_out = sc_out;
  a.pre_idx = pre_idx;
  a.pre_sc = pre_sc;
  a.h = static_cast<uint16_t*>(h);
  a.tagged = static_cast<unsigned long long*>(tagged);
  a.arrivals = static_cast<unsigned long long*>(arrivals);
  a.err = err;
  a.E = E;
  a.k = k;
  a.mode = mode;
  a.norm = norm;
  a.stage_bytes = p.stage_bytes;
  a.nstages = p.nstages;
  a.seg_per_item = p.seg_per_item;
  a.max_tiles = p.max_tiles;
  a.max_items = p.max_items;
  a.ksplit = p.ksplit;
  a.seg_stride = p.seg_stride;
  a.wpi = p.wpi;
  CUtensorMap tm_code, tm_gsb, tm_dsb;
  memset(&tm_code, 0, sizeof(tm_code));
  memset(&tm_gsb, 0, sizeof(tm_gsb));
  memset(&tm_dsb, 0, sizeof(tm_dsb));
  a.maps = dl_maps(a.slab, L, &tm_code, &tm_gsb, &tm_dsb);
  dl_wait_test(&a.phantom, &a.spin_limit);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16)
    return dl_launch<4, BIGRIG_F16>(a, tm_code, tm_gsb, tm_dsb, p.smem, G, s);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16)
    return dl_launch<4, BIGRIG_BF16>(a, tm_code, tm_gsb, tm_dsb, p.smem, G, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16)
    return dl_launch<8, BIGRIG_F16>(a, tm_code, tm_gsb, tm_dsb, p.smem, G, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16)
    return dl_launch<8, BIGRIG_BF16>(a, tm_code, tm_gsb, tm_dsb, p.smem, G, s);
  return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_layer: bits=%d scale_dtype=%d", L.bits, L.scale_dtype);
}

}  // namespace bigrig
