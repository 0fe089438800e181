// One decode token through one MoE layer, split by (routed expert, 64-feature group).
//
// Replaces, for a single token, the mlx_lm block's router, the per-expert
// quantized_matmul calls of _forward_views_one (bigrig_engine/stream.py:1278-1318) and
// the caller's weighted sum (stream.py:1523-1525), like decode_layer.cu, with a work
// split that needs no exchange between gate/up and down.  Work unit u = (rank j, group g)
// owns intermediate features [64 g, 64 g + 64) of routed expert j:
//
//   gate/up  the 64 gate and 64 up rows over the whole hidden dimension, streamed by the
//            producer warp as 8 tiles of 16 rows (TMA, 128-byte swizzle) through a ring
//            of full / empty mbarrier stages; 16 consumer warps each own every 16th
//            block of the hidden dimension, so h[64 g .. 64 g + 63] is complete inside
//            the CTA once the tiles are done (partials added in warp order)
//   down     the same 64 columns of the down projection for all H rows -- exactly one
//            quantisation group per row, so one scale and bias per row -- giving the
//            unit's partial y[H], stored to ypart[u][H]
//   combine  after one grid barrier each CTA sums, for its rows, the partials of every
//            routed expert over g in order, rounds y to bf16, and adds the experts in
//            rank order plus the residual (the chain's rounding points and order)
//
// Dot products on the integer tensor cores.  mma.sync m16n8k32 u8 x s8 -> s32 (full rate
// on sm_100a, twice the bf16 MAC rate): A is the weight codes as bytes -- 4-bit words are
// split into their even and odd nibbles with one mask each, a K permutation that B
// follows -- and B holds the activation as three signed byte planes of a 23-bit fixed
// point copy, X = round(x 2^(22-e)) = d0 + 256 d1 + 65536 d2 (balanced digits), one plane
// per B column, two quantisation groups side by side in columns 0-5.  Products and
// sums are exact integers per group; per group the accumulator columns are combined in
// fp32 and scaled: sum_k w x = s (2^(e-22) sum q X) + b sum x.  Activations within 2^15
// of the vector's largest magnitude are represented exactly, smaller ones to 2^(e-23).
//
// Every wait -- mbarriers, tagged logits, the grid barrier -- is bounded; a timeout
// counts in the error words and the kernel carries on to its end.
#include <cuda.h>

#include <map>
#include <mutex>
#include <tuple>

#include "gemv_common.cuh"
#include "routing.cuh"

// Phase-boundary hook, called by one thread: empty in the library, defined by instrumented
// builds that record timestamps.
#ifndef DS_STAMP
#define DS_STAMP(i)
#endif

namespace bigrig {

void dl_wait_test(uint32_t* phantom, uint32_t* spin_limit);   // decode_layer.cu test hook

namespace {

constexpr int kDsCW = 16;                 // consumer warps
constexpr int kDsCT = kDsCW * 32;
constexpr int kDsRows = 32;               // rows of a gate/up tile: two MMA row groups
constexpr int kDsM = 16;                  // the MMA's M
constexpr int kDsFeat = 64;               // features of a unit (one quantisation group)
constexpr int kDsTiles = 2 * kDsFeat / kDsRows;   // gate/up tiles of a unit (4)
constexpr int kDsWarpsPerRows = kDsCW / (kDsRows / kDsM);   // warps sharing a row group (8)
constexpr int kDsMaxWin = 4;              // most windows of the hidden dimension a warp owns
constexpr int kDsDownRows = 256;          // down-stage rows come in multiples of this
constexpr int kDsMaxStages = 12;
constexpr int kDsRouterPerCta = 4;
// dynamic shared memory of a CTA: 227 KB less the kernel's static arrays (~3 KB)
constexpr size_t kDsSmemLimit = 223 * 1024;
constexpr uint32_t kDsSpinLimit = 1u << 20;

struct SplitArgs {
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
  const float* pre_sc;
  float* ypart;               // [k * I / 64, H] unit partials
  unsigned long long* tagged; // [E] logit bits | tag << 32
  unsigned long long* arrivals;
  int32_t* err;
  int E, k, mode, norm;
  int stage_bytes, nstages, nch;   // ring; K chunks of a gate/up tile
  int down_rows;                   // rows of a down stage
  uint32_t spin_limit, phantom;
};

// ------------------------------------------------------------------ small PTX helpers
__device__ __forceinline__ unsigned long long ds_ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ds_ld_relaxed(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void ds_st_relaxed(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void ds_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void ds_named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ bool ds_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (bar_wait(bar, parity, err)) return true;
  bar_wait(bar, parity, nullptr);          // let the stage's copies land before moving on
  return false;
}

// D[16x8] += A[16x32] (u8) B[32x8] (s8), int32 accumulators.  Lane (g, t): A rows g (a0,
// a2) and g + 8 (a1, a3) at k-slots 4t..4t+3 (a0, a1) and 16+4t..16+4t+3 (a2, a3); B column
// g at the same k-slots (b0, b1); D rows g (d0, d1) and g + 8 (d2, d3), columns 2t, 2t+1.
__device__ __forceinline__ void mma_u8s8(int* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The even / odd nibbles of a word of 4-bit codes as four bytes each.
__device__ __forceinline__ uint32_t lo_nibbles(uint32_t w) { return w & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t hi_nibbles(uint32_t w) { return (w >> 4) & 0x0F0F0F0Fu; }

// Balanced base-256 digits of a fixed-point value |X| <= 2^22: X = d0 + 256 d1 + 65536 d2,
// d0 and d1 in [-128, 127], d2 in [-65, 65].
__device__ __forceinline__ int digit(int X, int p) {
  const int d0 = static_cast<int>(static_cast<int8_t>(X & 0xFF));
  if (p == 0) return d0;
  const int X1 = (X - d0) >> 8;
  const int d1 = static_cast<int>(static_cast<int8_t>(X1 & 0xFF));
  return p == 1 ? d1 : (X1 - d1) >> 8;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// The fixed-point scale of a group whose largest magnitude is amax: X = round(v * up) with
// |X| <= 2^22; v = X * back.  0 for an all-zero group.
constexpr float kDsFix = 4194304.0f;       // 2^22
__device__ __forceinline__ void fix_scale(float amax, float& up, float& back) {
  up = amax > 0.f ? kDsFix / amax : 0.f;
  back = amax / kDsFix;
}

// B fragments (the activation's three digit planes) of one window of the hidden dimension:
// two quantisation groups, 4 MMAs, column 3c + p = plane p of the window's group c.
//   4-bit: one 64-byte block; MMA m takes word 4t + m from lane t -- even nibbles at
//     k-slots 4t.., odd nibbles at 16 + 4t.. -- so lanes t < 2 carry group 0, t >= 2 group 1
//   8-bit: two 64-byte blocks, one group each; MMA m takes words 4t + 2 (m % 2) (k-slots
//     4t..) and 4t + 2 (m % 2) + 1 (16 + 4t..) of block m / 2
// X: the fixed-point activation; k0: the window's first element; ng: its groups that exist.
template <int BITS>
__device__ __forceinline__ void b_window(const int* X, int k0, int ng, int g, int t, uint32_t* b) {
  const int col_grp = g / 3, p = g % 3;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint32_t b0 = 0, b1 = 0;
    if constexpr (BITS == 4) {
      const int grp = t >> 1;
      if (g < 6 && grp == col_grp && grp < ng) {
        const int* e = X + k0 + 8 * (4 * t + m);
        b0 = pack4(digit(e[0], p), digit(e[2], p), digit(e[4], p), digit(e[6], p));
        b1 = pack4(digit(e[1], p), digit(e[3], p), digit(e[5], p), digit(e[7], p));
      }
    } else {
      const int blk = m >> 1;
      if (g < 6 && blk == col_grp && blk < ng) {
        const int* e = X + k0 + 64 * blk + 4 * (4 * t + 2 * (m & 1));
        b0 = pack4(digit(e[0], p), digit(e[1], p), digit(e[2], p), digit(e[3], p));
        b1 = pack4(digit(e[4], p), digit(e[5], p), digit(e[6], p), digit(e[7], p));
      }
    }
    b[2 * m] = b0;
    b[2 * m + 1] = b1;
  }
}

// B fragments of the down slice (64 elements of h, one group, 2 MMAs, columns 0-2 = planes).
// 4-bit: lane t takes words 2t, 2t + 1 of a row's 8; MMA m word 2t + m, even / odd nibbles.
// 8-bit: lane t takes words 4t..4t+3 of a row's 16; MMA m words 4t + 2m and 4t + 2m + 1.
template <int BITS>
__device__ __forceinline__ void b_down(const int* hX, int g, int t, uint32_t* b) {
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    uint32_t b0 = 0, b1 = 0;
    if (g < 3) {
      if constexpr (BITS == 4) {
        const int* e = hX + 8 * (2 * t + m);
        b0 = pack4(digit(e[0], g), digit(e[2], g), digit(e[4], g), digit(e[6], g));
        b1 = pack4(digit(e[1], g), digit(e[3], g), digit(e[5], g), digit(e[7], g));
      } else {
        const int* e = hX + 4 * (4 * t + 2 * m);
        b0 = pack4(digit(e[0], g), digit(e[1], g), digit(e[2], g), digit(e[3], g));
        b1 = pack4(digit(e[4], g), digit(e[5], g), digit(e[6], g), digit(e[7], g));
      }
    }
    b[2 * m] = b0;
    b[2 * m + 1] = b1;
  }
}

__device__ __forceinline__ void ds_tma4(void* dst, const CUtensorMap* m, int c0, int c1, int c2,
                                        int c3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar)),
      "l"(policy)
      : "memory");
}

// 16 bytes global -> shared through the load/store unit (L1 bypassed), and the mbarrier
// arrive that fires once all of this thread's earlier such copies have landed (the
// pending count is raised first, so the phase also waits for them).
__device__ __forceinline__ void ds_cp16(void* dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)),
               "l"(src), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void ds_cp4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void ds_cp_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ uint4 ds_lds128(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// tm_gu: the gate/up codes as [8-byte words of a row][row][gate, up][slot], box of one
// tile's 32 rows x a chunk of each row (whole rows up to 2 KB): a stage is [32 rows][chunk].
// The down slices -- 32 or 64 bytes of every row -- go by 16-byte cp.async copies.
// One CTA of 17 warps per SM: five of them share one of the SM's four 16K-register
// sub-partitions, so at most 96 registers a thread.  MW: windows a warp owns (2 while
// H <= 2048, else 4).
template <int BITS, int SDT, int MW>
__global__ void __launch_bounds__((kDsCW + 1) * 32, 1) decode_split_kernel(
    SplitArgs a, const __grid_constant__ CUtensorMap tm_gu) {
  constexpr int GBYTES = 64 * BITS / 8;          // bytes of one group of a row
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ float s_lg[kMaxExperts];
  __shared__ int32_t s_g2s[kMaxExperts];
  __shared__ int32_t s_idx[32], s_slot[32];
  __shared__ float s_sc[32], s_rank_lg[32];
  __shared__ float s_red[kDsCW];
  __shared__ unsigned long long s_epoch;
  __shared__ float s_hscale, s_hsum;
  const bigrig_expert_layout& L = a.L;
  const int H = L.hidden, I = L.inter, E = a.E, k = a.k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool producer = warp == kDsCW;
  const int G = gridDim.x, cta = blockIdx.x;
  const int gh = H / 64, gi = I / 64;
  const int pitch_h = H * BITS / 8, pitch_i = I * BITS / 8;
  const int nch = a.nch, cbytes = pitch_h / nch;
  const int U = k * gi;
  const int my_units = cta < U ? (U - 1 - cta) / G + 1 : 0;
  const int rd = a.down_rows;
  const int nd = (H + rd - 1) / rd;
  const int n_gu = kDsTiles * nch;
  const int gu_code = kDsRows * cbytes;
  const int sc_bytes = kDsRows * gh * 2;
  const int nst = a.nstages, stage_bytes = a.stage_bytes;

  // the ring first (1024-byte aligned), then the CTA's other buffers
  uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = base;
  SmemCarve sc(ring + static_cast<size_t>(nst) * stage_bytes);
  uint64_t* full = sc.take<uint64_t>(kDsMaxStages * 8);
  uint64_t* empty = sc.take<uint64_t>(kDsMaxStages * 8);
  uint64_t* bar_x = sc.take<uint64_t>(4 * 8);
  uint64_t* bar_r = bar_x + 1;
  uint64_t* bar_s = bar_x + 2;
  uint16_t* xraw = sc.take<uint16_t>(static_cast<size_t>(H) * 2);
  int* X = sc.take<int>(static_cast<size_t>(H) * 4);
  float* xsum = sc.take<float>(static_cast<size_t>(gh) * 4);
  float* xsg = sc.take<float>(static_cast<size_t>(gh) * 4);   // 2^(e_group - 14)
  float* part = sc.take<float>(2 * kDsFeat * kDsCW * 4);
  uint32_t* dsc = sc.take<uint32_t>(static_cast<size_t>(H) * 4);   // down scale, bias: the
  uint32_t* dbi = sc.take<uint32_t>(static_cast<size_t>(H) * 4);   // aligned word holding each
  float* yp = sc.take<float>(static_cast<size_t>(H) * 4);
  float* hv = sc.take<float>(kDsFeat * 4);
  int* hX = sc.take<int>(kDsFeat * 4);
  uint16_t* wr = reinterpret_cast<uint16_t*>(ring);     // router rows, before any stage

  const bool routed = a.pre_idx != nullptr;
  const int n_mine = routed ? 0 : max(0, min(kDsRouterPerCta, E - cta * kDsRouterPerCta));
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      bar_init(full + i, 1);
      bar_init(empty + i, kDsCW);
    }
    bar_init(bar_x, 1);
    bar_init(bar_r, 1);
    bar_init(bar_s, 1);
    bar_expect_tx(bar_x, H * 2);
    bulk_g2s(xraw, a.x, H * 2, bar_x);
    if (n_mine > 0) {
      bar_expect_tx(bar_r, static_cast<uint32_t>(n_mine) * H * 2);
      bulk_g2s_hint(wr, a.gate_w + static_cast<size_t>(cta) * kDsRouterPerCta * H, n_mine * H * 2,
                    bar_r, l2_evict_last());
    }
  }
  if (producer) {
    if (lane == 0) s_epoch = ds_ld_acquire(a.arrivals) / static_cast<unsigned long long>(G);
    if (lane == 1)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_gu)) : "memory");
    for (int e = lane; e < E; e += 32) s_g2s[e] = a.g2s ? a.g2s[e] : e;
  }
  if (threadIdx.x < 32) s_idx[threadIdx.x] = -1;
  __syncthreads();
  const unsigned long long epoch = s_epoch;
  const unsigned long long tag = ((epoch + 1ull) & 0xffffffffull) << 32;
  if (threadIdx.x == 0) DS_STAMP(0);

  // ---------------------------------------------------------------- x, router logits
  bool xok = true;
  if (!producer) {
    xok = ds_wait(bar_x, 0, a.err);
    if (warp < n_mine) {
      const bool rok = ds_wait(bar_r, 0, a.err);
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
      const int e = cta * kDsRouterPerCta + warp;
      const float v = (xok && rok) ? acc + (a.gate_b ? a.gate_b[e] : 0.f) : __int_as_float(0x7fc00000);
      if (lane == 0) ds_st_relaxed(a.tagged + e, tag | __float_as_uint(v));
    }
    if (threadIdx.x == 0) DS_STAMP(1);
    // the fixed-point copy of x, one exponent per quantisation group: one warp per group,
    // two elements a lane; its sum by a fixed shuffle tree
    for (int grp = warp; grp < gh; grp += kDsCW) {
      const float v0 = bf16_bits_to_f32(xraw[grp * 64 + lane]);
      const float v1 = bf16_bits_to_f32(xraw[grp * 64 + 32 + lane]);
      float up, back;
      fix_scale(warp_max(fmaxf(fabsf(v0), fabsf(v1))), up, back);
      X[grp * 64 + lane] = __float2int_rn(v0 * up);
      X[grp * 64 + 32 + lane] = __float2int_rn(v1 * up);
      const float v = warp_sum(v0 + v1);
      if (lane == 0) {
        xsum[grp] = v;
        xsg[grp] = back;
      }
    }
  }
  __syncthreads();                               // router rows read: the ring is free


  // ---------------------------------------------------------------- routing
  if (routed) {
    if (producer) {
      if (lane < k) {
        const int e = a.pre_idx[lane];
        const int ev = (e >= 0 && e < E) ? e : -1;
        s_idx[lane] = ev;
        s_slot[lane] = ev >= 0 ? s_g2s[ev] : -1;
        s_sc[lane] = a.pre_sc[lane];
      }
      __syncwarp();
    }
    __syncthreads();
  } else {
    // the producer collects the E tagged logits; the consumers then rank them (logit
    // descending, id ascending: the warp top-k's order), 8 threads per candidate
    if (producer) {
      uint32_t need = 0;
      for (int e = lane, i = 0; e < E; e += 32, ++i) need |= 1u << i;
      for (uint32_t n = 0; need; ++n) {
#pragma unroll
        for (int i = 0; i < kMaxExperts / 32; ++i) {
          if (need & (1u << i)) {
            const int e = lane + 32 * i;
            const unsigned long long v = ds_ld_relaxed(a.tagged + e);
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
    }
    __syncthreads();                             // logits in s_lg
    if (!producer) {
      const int per_cand = (E + 7) / 8;
      for (int c0 = 0; c0 < E; c0 += kDsCT / 8) {
        const int c = c0 + (threadIdx.x >> 3), part_id = threadIdx.x & 7;
        int r = 0;
        float v = 0.f;
        if (c < E) {
          v = s_lg[c];
          const int u0 = part_id * per_cand, u1 = min(E, u0 + per_cand);
          for (int u = u0; u < u1; ++u) {
            const float w = s_lg[u];
            r += (w > v) || (w == v && u < c);
          }
        }
        r += __shfl_xor_sync(0xffffffffu, r, 1);
        r += __shfl_xor_sync(0xffffffffu, r, 2);
        r += __shfl_xor_sync(0xffffffffu, r, 4);
        if (c < E && part_id == 0 && v == v && r < k) {   // NaN logits are never selected
          s_idx[r] = c;
          s_rank_lg[r] = v;
        }
      }
    }
    __syncthreads();                             // ranks in s_idx / s_rank_lg
    if (producer) {
      if (lane < k) {
        const int e = s_idx[lane];
        s_slot[lane] = (e >= 0 && e < E) ? s_g2s[e] : -1;
      }
      // scores: the warp top-k's formulas and reductions over the same values and lanes
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
      if (lane < k) s_sc[lane] = sv;
      __syncwarp();
    }
  }
  if (threadIdx.x == 0) DS_STAMP(2);
  if (producer) {
    if (lane < k && cta == 0) {
      if (a.idx_out && a.idx_out != a.pre_idx) a.idx_out[lane] = s_idx[lane];
      if (a.sc_out && a.sc_out != a.pre_sc) a.sc_out[lane] = s_sc[lane];
      if (s_slot[lane] < 0) atomicAdd(a.err, 1);
    }
    __syncwarp();
    if (lane == 0) ds_arrive(bar_s);             // scores and slots visible to the combine

    // ------------------------------------------------------------ stream the ring
    const uint64_t once = l2_evict_first();
    int q = 0;
    for (int iu = 0; iu < my_units; ++iu) {
      const int u = cta + iu * G, j = u / gi, grp = u - j * gi;
      const int slot = s_slot[j];
      if (slot < 0) continue;                    // the consumers skip it too
      const uint8_t* ebase = a.slab + static_cast<int64_t>(slot) * L.slot_stride;
      for (int st = 0; st < n_gu + nd; ++st, ++q) {
        const int b = q % nst;
        if (q >= nst) ds_wait(empty + b, ((q / nst) - 1) & 1, a.err);
        uint8_t* dst = ring + static_cast<size_t>(b) * stage_bytes;
        if (st < n_gu) {
          const int r = st / nch, ch = st - r * nch;
          const int proj = r < kDsTiles / 2 ? 0 : 1;
          const int row0 = grp * kDsFeat + (r % (kDsTiles / 2)) * kDsRows;
          // the stage's barrier is armed before any of its copies is issued
          if (lane == 0) bar_expect_tx(full + b, static_cast<uint32_t>(gu_code + 2 * sc_bytes));
          __syncwarp();
          if (lane == 0) {
            ds_tma4(dst, &tm_gu, ch * (cbytes / 8), row0, proj, slot, full + b, once);
          } else if (lane == 1) {
            bulk_g2s_hint(dst + gu_code, ebase + L.scales_off[proj] + static_cast<int64_t>(row0) * gh * 2,
                          sc_bytes, full + b, once);
          } else if (lane == 2) {
            bulk_g2s_hint(dst + gu_code + sc_bytes,
                          ebase + L.biases_off[proj] + static_cast<int64_t>(row0) * gh * 2, sc_bytes,
                          full + b, once);
          }
        } else {
          // rows [d rd, d rd + rd) of the down slice: 16-byte granules, a lane every 32nd
          const int row0 = (st - n_gu) * rd;
          constexpr int GPR = GBYTES / 16;         // granules of a row
          const uint8_t* src = ebase + L.weight_off[2] + static_cast<int64_t>(grp) * GBYTES;
          for (int gi16 = lane; gi16 < rd * GPR; gi16 += 32) {
            const int rr = gi16 / GPR, part = gi16 - rr * GPR;
            if (row0 + rr < H)
              ds_cp16(dst + gi16 * 16, src + static_cast<int64_t>(row0 + rr) * pitch_i + part * 16, once);
          }
          ds_cp_arrive(full + b);
          __syncwarp();
          if (lane == 0) ds_arrive(full + b);
        }
        __syncwarp();
      }
    }
    if (lane == 0) DS_STAMP(11);
    return;                                      // the consumers wait for every stage it filled
  }


  // ---------------------------------------------------------------- consumers
  // a tile's 32 rows are two MMA row groups: warps 0-7 take rows 0-15, warps 8-15 rows
  // 16-31; within a row group warp w8 owns windows w8, w8 + 8, ... of the hidden dimension
  // (two quantisation groups each); its B fragments (the token's digit planes) stay in
  // registers for the whole layer
  const int w8 = warp % kDsWarpsPerRows, rgrp = warp / kDsWarpsPerRows;
  const int nwin = (gh + 1) / 2;
  uint32_t breg[MW][8];
#pragma unroll
  for (int wi = 0; wi < MW; ++wi) {
    const int win = w8 + kDsWarpsPerRows * wi;
    if (win < nwin) {
      b_window<BITS>(X, win * 128, min(2, gh - 2 * win), g, t, breg[wi]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) breg[wi][i] = 0u;
    }
  }
  const int rl = rgrp * kDsM + g, rh = rl + 8;   // this lane's two rows of a tile
  // this lane's two accumulator columns 2t, 2t + 1: (group, plane) = (c / 3, c % 3); lane 3
  // holds none.  Plane weights 1, 256, 65536; the bias term goes with each group's plane 0.
  const int ca = 2 * t, cb = 2 * t + 1;
  const int ga = ca / 3, gb = cb / 3;
  const float wa = ca % 3 == 0 ? 1.f : ca % 3 == 1 ? 256.f : 65536.f;
  const float wb = cb % 3 == 0 ? 1.f : cb % 3 == 1 ? 256.f : 65536.f;
  const bool bias_a = ca % 3 == 0, bias_b = cb % 3 == 0;
  int q = 0;
  for (int iu = 0; iu < my_units; ++iu) {
    const int u = cta + iu * G, j = u / gi, grp = u - j * gi;
    const int slot = s_slot[j];
    float* ydst = a.ypart + static_cast<size_t>(u) * H;
    if (slot < 0 || !xok) {
      for (int i = threadIdx.x * 4; i < H; i += kDsCT * 4)
        *reinterpret_cast<float4*>(ydst + i) = make_float4(0.f, 0.f, 0.f, 0.f);
      if (slot >= 0) q += n_gu + nd;             // the producer filled its stages: drain them
      if (slot >= 0)
        for (int st = 0; st < n_gu + nd; ++st) {
          const int qq = q - n_gu - nd + st, b = qq % nst;
          ds_wait(full + b, (qq / nst) & 1, a.err);
          __syncwarp();
          if (lane == 0) ds_arrive(empty + b);
        }
      continue;
    }
    const uint8_t* ebase = a.slab + static_cast<int64_t>(slot) * L.slot_stride;
    // this unit's down scales and biases (one of each per row): each 2-byte element is
    // copied as the aligned 4-byte word that holds it, now, and waited for before the down
    // phase, so that the copies land behind the gate/up tiles
    {
      const uint8_t* sp = ebase + L.scales_off[2];
      const uint8_t* bp = ebase + L.biases_off[2];
      for (int r = threadIdx.x; r < H; r += kDsCT) {
        const int64_t w = (static_cast<int64_t>(r) * gi + grp) >> 1;
        ds_cp4(dsc + r, sp + 4 * w);
        ds_cp4(dbi + r, bp + 4 * w);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // ---- gate/up: 4 tiles of 32 rows (2 gate, then 2 up), each in nch K chunks
    for (int r = 0; r < kDsTiles; ++r) {
      float p_lo = 0.f, p_hi = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++q) {
        const int b = q % nst;
        const bool landed = ds_wait(full + b, (q / nst) & 1, a.err);
        if (iu == 0 && ch == 0 && threadIdx.x == 0) {
          if (r == 0) DS_STAMP(3);
          if (r == 1) DS_STAMP(12);
          if (r == 2) DS_STAMP(13);
          if (r == kDsTiles - 1) DS_STAMP(14);
        }
        const uint8_t* st = ring + static_cast<size_t>(b) * stage_bytes;
        const uint16_t* ssc = reinterpret_cast<const uint16_t*>(st + gu_code);
        const uint16_t* sbi = ssc + kDsRows * gh;
        if (landed) {
#pragma unroll
          for (int wi = 0; wi < MW; ++wi) {
            const int win = w8 + kDsWarpsPerRows * wi;
            const int wb0 = win * (BITS == 4 ? 64 : 128);       // the window's first byte
            if (win >= nwin || wb0 < ch * cbytes || wb0 >= (ch + 1) * cbytes) continue;
            const int ng = min(2, gh - 2 * win);
            const uint8_t* al = st + rl * cbytes + (wb0 - ch * cbytes) + 16 * t;
            const uint8_t* ah = al + 8 * cbytes;
            int d[4] = {0, 0, 0, 0};
            if constexpr (BITS == 4) {
              uint4 ul = ds_lds128(al), uh = ds_lds128(ah);
              if ((t >> 1) >= ng) ul = uh = make_uint4(0u, 0u, 0u, 0u);
              const uint32_t wl[4] = {ul.x, ul.y, ul.z, ul.w}, wh[4] = {uh.x, uh.y, uh.z, uh.w};
#pragma unroll
              for (int m = 0; m < 4; ++m)
                mma_u8s8(d, lo_nibbles(wl[m]), lo_nibbles(wh[m]), hi_nibbles(wl[m]), hi_nibbles(wh[m]),
                         breg[wi][2 * m], breg[wi][2 * m + 1]);
            } else {
#pragma unroll
              for (int blk = 0; blk < 2; ++blk) {
                uint4 ul = ds_lds128(al + 64 * blk), uh = ds_lds128(ah + 64 * blk);
                if (blk >= ng) ul = uh = make_uint4(0u, 0u, 0u, 0u);
                mma_u8s8(d, ul.x, uh.x, ul.y, uh.y, breg[wi][4 * blk], breg[wi][4 * blk + 1]);
                mma_u8s8(d, ul.z, uh.z, ul.w, uh.w, breg[wi][4 * blk + 2], breg[wi][4 * blk + 3]);
              }
            }
            // column a (d0 row rl, d2 row rh) and column b (d1, d3) of this lane
            const int G0 = 2 * win;
            if (ca < 6 && ga < ng) {
              const int G = G0 + ga;
              const float f = xsg[G] * wa;
              p_lo = fmaf(half_to_f32<SDT>(ssc[rl * gh + G]) * f, static_cast<float>(d[0]), p_lo);
              p_hi = fmaf(half_to_f32<SDT>(ssc[rh * gh + G]) * f, static_cast<float>(d[2]), p_hi);
              if (bias_a) {
                p_lo = fmaf(half_to_f32<SDT>(sbi[rl * gh + G]), xsum[G], p_lo);
                p_hi = fmaf(half_to_f32<SDT>(sbi[rh * gh + G]), xsum[G], p_hi);
              }
            }
            if (cb < 6 && gb < ng) {
              const int G = G0 + gb;
              const float f = xsg[G] * wb;
              p_lo = fmaf(half_to_f32<SDT>(ssc[rl * gh + G]) * f, static_cast<float>(d[1]), p_lo);
              p_hi = fmaf(half_to_f32<SDT>(ssc[rh * gh + G]) * f, static_cast<float>(d[3]), p_hi);
              if (bias_b) {
                p_lo = fmaf(half_to_f32<SDT>(sbi[rl * gh + G]), xsum[G], p_lo);
                p_hi = fmaf(half_to_f32<SDT>(sbi[rh * gh + G]), xsum[G], p_hi);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) ds_arrive(empty + b);
      }
      p_lo += __shfl_xor_sync(0xffffffffu, p_lo, 1);
      p_hi += __shfl_xor_sync(0xffffffffu, p_hi, 1);
      p_lo += __shfl_xor_sync(0xffffffffu, p_lo, 2);
      p_hi += __shfl_xor_sync(0xffffffffu, p_hi, 2);
      if (t == 0) {
        part[(r * kDsRows + rl) * kDsWarpsPerRows + w8] = p_lo;
        part[(r * kDsRows + rh) * kDsWarpsPerRows + w8] = p_hi;
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // this thread's scale words
    ds_named_sync(1, kDsCT);
    if (iu == 0 && threadIdx.x == 0) DS_STAMP(4);
    // ---- h = bf16(silu(gate) * up) for the unit's 64 features; the partials of each row
    // added in warp order
    if (threadIdx.x < kDsFeat) {
      const int f = threadIdx.x;
      float gv = 0.f, uv = 0.f;
      for (int w = 0; w < kDsWarpsPerRows; ++w) {
        gv += part[f * kDsWarpsPerRows + w];
        uv += part[(kDsFeat + f) * kDsWarpsPerRows + w];
      }
      const float h = bf16_round(silu_f32(gv) * uv);
      hv[f] = h;
      const float m = warp_max(fabsf(h));
      if (lane == 0) s_red[warp] = m;
    }
    ds_named_sync(1, kDsCT);
    if (iu == 0 && threadIdx.x == 0) DS_STAMP(17);
    if (threadIdx.x < kDsFeat) {
      float up, back;
      fix_scale(fmaxf(s_red[0], s_red[1]), up, back);
      hX[threadIdx.x] = __float2int_rn(hv[threadIdx.x] * up);
      if (threadIdx.x == 0) s_hscale = back;
      if (warp == 0) {
        const float v = warp_sum(hv[lane] + hv[lane + 32]);
        if (lane == 0) s_hsum = v;
      }
    }
    ds_named_sync(1, kDsCT);
    uint32_t bd[4];
    b_down<BITS>(hX, g, t, bd);
    const float hs = s_hscale, hsum = s_hsum;
    if (iu == 0 && threadIdx.x == 0) DS_STAMP(5);
    // ---- down: this unit's 64 columns of all H rows, 256 rows a stage, 16 a warp
    for (int dd = 0; dd < nd; ++dd, ++q) {
      const int b = q % nst;
      // warp-uniform (the tile loop below shuffles)
      const bool landed = __all_sync(0xffffffffu, ds_wait(full + b, (q / nst) & 1, a.err));
      if (iu == 0 && threadIdx.x == 0) {
        if (dd == 0) DS_STAMP(15);
        if (dd == nd - 1) DS_STAMP(16);
      }
      const uint8_t* st = ring + static_cast<size_t>(b) * stage_bytes;
      for (int tl = warp; landed && tl * kDsM < rd; tl += kDsCW) {
        const int row_lo = dd * rd + tl * kDsM + g, row_hi = row_lo + 8;
        const uint8_t* al = st + (tl * kDsM + g) * GBYTES;
        const uint8_t* ah = al + 8 * GBYTES;
        int d[4] = {0, 0, 0, 0};
        if constexpr (BITS == 4) {
          const uint2 wl = *reinterpret_cast<const uint2*>(al + 8 * t);
          const uint2 wh = *reinterpret_cast<const uint2*>(ah + 8 * t);
          mma_u8s8(d, lo_nibbles(wl.x), lo_nibbles(wh.x), hi_nibbles(wl.x), hi_nibbles(wh.x), bd[0], bd[1]);
          mma_u8s8(d, lo_nibbles(wl.y), lo_nibbles(wh.y), hi_nibbles(wl.y), hi_nibbles(wh.y), bd[2], bd[3]);
        } else {
          const uint4 wl = ds_lds128(al + 16 * t);
          const uint4 wh = ds_lds128(ah + 16 * t);
          mma_u8s8(d, wl.x, wh.x, wl.y, wh.y, bd[0], bd[1]);
          mma_u8s8(d, wl.z, wh.z, wl.w, wh.w, bd[2], bd[3]);
        }
        // columns 0-2 hold the three planes: lane t = 0 planes 0 and 1, lane t = 1 plane 2
        // (d0 of rows row_lo, d2 of row_hi); added in that order, then scaled
        float v_lo = t == 0 ? fmaf(256.f, static_cast<float>(d[1]), static_cast<float>(d[0]))
                            : 65536.f * static_cast<float>(d[0]);
        float v_hi = t == 0 ? fmaf(256.f, static_cast<float>(d[3]), static_cast<float>(d[2]))
                            : 65536.f * static_cast<float>(d[2]);
        v_lo += __shfl_down_sync(0xffffffffu, v_lo, 1);
        v_hi += __shfl_down_sync(0xffffffffu, v_hi, 1);
        if (t == 0) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int row = h2 ? row_hi : row_lo;
            if (row < H) {
              // the element's half of its aligned word
              const int sh = static_cast<int>((static_cast<int64_t>(row) * gi + grp) & 1) * 16;
              const float sv = half_to_f32<SDT>(static_cast<uint16_t>(dsc[row] >> sh));
              const float bv = half_to_f32<SDT>(static_cast<uint16_t>(dbi[row] >> sh));
              yp[row] = fmaf(sv * hs, h2 ? v_hi : v_lo, bv * hsum);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) ds_arrive(empty + b);
    }
    ds_named_sync(1, kDsCT);
    if (iu == 0 && threadIdx.x == 0) DS_STAMP(6);
    for (int i = threadIdx.x * 4; i < H; i += kDsCT * 4)
      *reinterpret_cast<float4*>(ydst + i) = *reinterpret_cast<const float4*>(yp + i);
  }
  if (threadIdx.x == 0) DS_STAMP(7);


  // ---------------------------------------------------------------- grid barrier
  ds_named_sync(1, kDsCT);
  if (threadIdx.x == 0) {
    // one-way release add (the CTA's partial stores, ordered before it by the named
    // barrier, become visible with it), then acquire polls
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(a.arrivals) : "memory");
    const unsigned long long target = (epoch + 1ull) * static_cast<unsigned long long>(G) + a.phantom;
    uint32_t n = 0;
    while (static_cast<long long>(ds_ld_acquire(a.arrivals) - target) < 0) {
      if (++n > a.spin_limit) {
        atomicAdd(a.err + 1, 1);
        break;
      }
    }
  }
  ds_named_sync(1, kDsCT);
  if (threadIdx.x == 0) DS_STAMP(8);

  // ---------------------------------------------------------------- combine
  // rows [cta R, cta R + R): y of each routed expert is its units' partials added in group
  // order and rounded to bf16; the experts are added in rank order, then the residual
  const int R = (H + G - 1) / G;
  const int row0 = cta * R;
  if (row0 >= H) return;
  const bool scores = ds_wait(bar_s, 0, a.err);
  // every thread loads: (expert, row) pairs x S interleaved subsets of the groups, each
  // subset added in group order, then the S subset sums of a pair in subset order
  float* ysm = part;                            // [k * R]
  float* ysub = part + 1024;                    // [k * R * S]
  const int pairs = k * R;
  const int S = max(1, min(gi, kDsCT / pairs));
  for (int idx = threadIdx.x; idx < pairs * S; idx += kDsCT) {
    const int pr = idx / S, sub = idx - pr * S;
    const int j = pr / R, r = pr - j * R, row = row0 + r;
    float y = 0.f;
    if (row < H && s_slot[j] >= 0) {
      // up to eight L2 loads in flight at once (guarded, not a dependent chain), then their
      // adds in group order
      const float* src = a.ypart + static_cast<size_t>(j) * gi * H + row;
      for (int gg = sub; gg < gi; gg += 8 * S) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = gg + i * S < gi ? __ldcg(src + static_cast<size_t>(gg + i * S) * H) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) y += v[i];
      }
    }
    ysub[idx] = y;
  }
  ds_named_sync(1, kDsCT);
  for (int pr = threadIdx.x; pr < pairs; pr += kDsCT) {
    float y = 0.f;
    for (int sub = 0; sub < S; ++sub) y += ysub[pr * S + sub];
    ysm[pr] = bf16_round(y);
  }
  ds_named_sync(1, kDsCT);
  for (int r = threadIdx.x; r < R && row0 + r < H; r += kDsCT) {
    const int row = row0 + r;
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc = acc + (scores ? s_sc[j] : 0.f) * ysm[j * R + r];
    if (a.residual) acc = bf16_bits_to_f32(a.residual[row]) + bf16_round(acc);
    a.out[row] = f32_to_bf16_bits(acc);
  }
  if (threadIdx.x == 0) DS_STAMP(9);
}

}  // namespace
}  // namespace bigrig

namespace bigrig {
namespace {

struct SplitPlan {
  int stage_bytes, nstages, nch, down_rows;
  size_t smem;
};

int ds_sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

inline size_t r128(size_t n) { return (n + 127) / 128 * 128; }

// Whether one CTA of the kernel for these codes fits an SM with `smem` bytes of dynamic
// shared memory (the cooperative launch needs every CTA resident); remembered per
// (bits, scale dtype, smem).
template <int MW>
const void* ds_kernel(int bits, int sdt) {
  if (bits == 4) return sdt == BIGRIG_F16 ? reinterpret_cast<const void*>(&decode_split_kernel<4, BIGRIG_F16, MW>)
                                         : reinterpret_cast<const void*>(&decode_split_kernel<4, BIGRIG_BF16, MW>);
  return sdt == BIGRIG_F16 ? reinterpret_cast<const void*>(&decode_split_kernel<8, BIGRIG_F16, MW>)
                           : reinterpret_cast<const void*>(&decode_split_kernel<8, BIGRIG_BF16, MW>);
}

// the windows a warp owns for a hidden dimension of gh groups (four groups a window, eight
// warps a row group)
inline int ds_mw(int gh) { return (gh + 1) / 2 <= 2 * kDsWarpsPerRows ? 2 : 4; }

bool ds_resident(int bits, int sdt, int mw, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, bool> seen;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(bits, sdt * 4 + mw, smem);
  auto it = seen.find(key);
  if (it != seen.end()) return it->second;
  const void* fn = mw == 2 ? ds_kernel<2>(bits, sdt) : ds_kernel<4>(bits, sdt);
  int n = 0;
  const bool ok = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)) == cudaSuccess &&
                  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, (kDsCW + 1) * 32, smem) ==
                      cudaSuccess &&
                  n >= 1;
  cudaGetLastError();                      // a refusal here is an answer, not an error
  seen[key] = ok;
  return ok;
}

// The split kernel's plan for a layer, or false when it cannot run it: the gated SwiGLU
// expert without projection biases, 4- or 8-bit codes in groups of 64, a hidden
// dimension of at most 4096 (16 warps x 4 blocks; down scales held 8 a thread), at most
// 32 routed experts, and a ring of at least two stages beside the fixed buffers.
bool decode_split_plan(const bigrig_expert_layout& L, int k, int E, int G, SplitPlan* p) {
  if (G <= 0 || k < 1 || k > 32 || E < 1 || E > kMaxExperts) return false;
  if (L.group_size != 64 || L.flags != 0 || (L.bits != 4 && L.bits != 8)) return false;
  const int H = L.hidden, I = L.inter;
  if (H % 64 || I % 64 || H > 4096 || H < 64) return false;
  const int gh = H / 64;
  if ((gh + 1) / 2 > kDsWarpsPerRows * kDsMaxWin) return false;   // windows of two groups
  // a tile's rows in nch chunks of at most 2 KB (one box line: 256 eight-byte words) and a
  // stage of at most 48 KB of codes; with more than one chunk each is a whole number of
  // windows (a single chunk may end in a partial window)
  const int pitch = H * L.bits / 8, wbytes = L.bits == 4 ? 64 : 128;
  int nch = 1;
  while (pitch / nch > 2048 || kDsRows * (pitch / nch) > 49152 || (nch > 1 && pitch % (wbytes * nch))) {
    if (++nch > 16) return false;
  }
  const size_t gu = static_cast<size_t>(kDsRows) * (pitch / nch) + 2 * kDsRows * gh * 2;
  // a down stage: as many 256-row blocks as a gate/up stage's room holds (the whole slice
  // when it fits), so that few down stages wait for ring slots
  const size_t grow = 64 * L.bits / 8;                  // bytes of one row's group
  const size_t stage = ((gu > kDsDownRows * grow ? gu : kDsDownRows * grow) + 1023) / 1024 * 1024;
  const int hr = (H + kDsDownRows - 1) / kDsDownRows * kDsDownRows;
  int rd = static_cast<int>(stage / grow) / kDsDownRows * kDsDownRows;
  if (rd > hr) rd = hr;
  const size_t fixed = 1024 + r128(kDsMaxStages * 8) * 2 + r128(4 * 8) + r128(H * 2) + r128(H * 4) +
                       r128(gh * 4) * 2 + r128(2 * kDsFeat * kDsCW * 4) + r128(H * 4) * 3 +
                       r128(kDsFeat * 4) * 2;
  if (fixed >= kDsSmemLimit) return false;
  size_t nst = (kDsSmemLimit - fixed) / stage;
  if (nst > static_cast<size_t>(kDsMaxStages)) nst = kDsMaxStages;
  if (nst < 2 || nst * stage < static_cast<size_t>(kDsRouterPerCta) * H * 2) return false;
  if (static_cast<size_t>(k) * ((H + G - 1) / G) > static_cast<size_t>(kDsFeat * kDsCW))   // combine scratch
    return false;
  (void)I;
  p->stage_bytes = static_cast<int>(stage);
  p->nstages = static_cast<int>(nst);
  p->nch = nch;
  p->down_rows = rd;
  p->smem = fixed + nst * stage;
  return ds_resident(L.bits, L.scale_dtype, ds_mw(gh), p->smem);
}

using DsEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

DsEncodeFn ds_encode_fn() {
  static DsEncodeFn fn = nullptr;
  if (!fn) {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<DsEncodeFn>(q);
  }
  return fn;
}

constexpr cuuint64_t kDsMapSlots = 1u << 16;

// A map of 8-byte words over the slab, no swizzle; false when the layout breaks a rule of tiled maps (16-byte
// aligned base and strides, 1..256 elements per box side) or the encoder refuses it.
bool ds_encode(CUtensorMap* m, int rank, const uint8_t* base, const cuuint64_t* dims,
               const cuuint64_t* strides, const cuuint32_t* box) {
  DsEncodeFn fn = ds_encode_fn();
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

template <int BITS, int SDT, int MW>
int ds_launch(const SplitArgs& args, const CUtensorMap& gu, size_t smem, int G, cudaStream_t s) {
  auto kern = decode_split_kernel<BITS, SDT, MW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "decode_split: cannot reserve %zu bytes of smem", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3((kDsCW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TimedLaunch tl(BIGRIG_K_DECODE_SPLIT, s);
  cudaLaunchKernelEx(&cfg, kern, args, gu);
  return check_launch("decode_split_kernel");
}

}  // namespace

bool decode_split_fits(const bigrig_expert_layout& L, int k, int E) {
  SplitPlan p;
  return decode_split_plan(L, k, E, ds_sm_count(), &p);
}

// Measured on B200 (one-token layers, eager launches): the split kernel is faster than the
// feature-tiled one once its units fill at least two waves of CTAs (Mixtral shape, 448
// units: 206 vs 236 us); with one partial wave (OLMoE 128, Qwen3 96 units) or a second wave
// mostly idle (gpt-oss 180) the tiled kernel is faster (25 vs 27-29 us, 41 vs 60 us).
bool decode_split_preferred(const bigrig_expert_layout& L, int k, int E) {
  return k * (L.inter / 64) >= 2 * ds_sm_count() && decode_split_fits(L, k, E);
}

size_t decode_split_scratch(const bigrig_expert_layout& L, int k) {
  return static_cast<size_t>(k) * (L.inter / 64) * L.hidden * sizeof(float);
}

int launch_decode_split(const void* x, const void* gate_w, const float* gate_b, int E, int k,
                        int mode, int norm, const int32_t* g2s, const void* slab,
                        const bigrig_expert_layout& L, const void* residual, void* out,
                        int32_t* idx_out, float* sc_out, float* ypart, void* tagged,
                        void* arrivals, int32_t* err, cudaStream_t s, const int32_t* pre_idx,
                        const float* pre_sc) {
  const int G = ds_sm_count();
  SplitPlan p;
  if (!decode_split_plan(L, k, E, G, &p))
    return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_split: layer does not fit the kernel");
  const uint8_t* sl = static_cast<const uint8_t*>(slab);
  const int64_t pitch = static_cast<int64_t>(L.hidden) * L.bits / 8;
  CUtensorMap gu;
  {
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(pitch / 8), static_cast<cuuint64_t>(L.inter), 2,
                                kDsMapSlots};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(pitch),
                                   static_cast<cuuint64_t>(L.weight_off[1] - L.weight_off[0]),
                                   static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(pitch / 8 / p.nch), static_cast<cuuint32_t>(kDsRows),
                               1, 1};
    if (L.weight_off[1] <= L.weight_off[0] ||
        !ds_encode(&gu, 4, sl + L.weight_off[0], dims, strides, box))
      return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_split: cannot map the gate/up codes");
  }
  SplitArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.gate_w = static_cast<const uint16_t*>(gate_w);
  a.gate_b = gate_b;
  a.g2s = g2s;
  a.slab = sl;
  a.L = L;
  a.residual = static_cast<const uint16_t*>(residual);
  a.out = static_cast<uint16_t*>(out);
  a.idx_out = idx_out;
  a.sc_out = sc_out;
  a.pre_idx = pre_idx;
  a.pre_sc = pre_sc;
  a.ypart = ypart;
  a.tagged = static_cast<unsigned long long*>(tagged);
  a.arrivals = static_cast<unsigned long long*>(arrivals);
  a.err = err;
  a.E = E;
  a.k = k;
  a.mode = mode;
  a.norm = norm;
  a.stage_bytes = p.stage_bytes;
  a.nstages = p.nstages;
  a.nch = p.nch;
  a.down_rows = p.down_rows;
  dl_wait_test(&a.phantom, &a.spin_limit);
  if (a.spin_limit == 0) a.spin_limit = kDsSpinLimit;
#define BIGRIG_DS(B, S)                                                                    \
  if (L.bits == B && L.scale_dtype == S)                                                   \
    return ds_mw(L.hidden / 64) == 2 ? ds_launch<B, S, 2>(a, gu, p.smem, G, s)            \
                                     : ds_launch<B, S, 4>(a, gu, p.smem, G, s);
  BIGRIG_DS(4, BIGRIG_F16)
  BIGRIG_DS(4, BIGRIG_BF16)
  BIGRIG_DS(8, BIGRIG_F16)
  BIGRIG_DS(8, BIGRIG_BF16)
#undef BIGRIG_DS
  return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_split: bits=%d scale_dtype=%d", L.bits,
                   L.scale_dtype);
}

}  // namespace bigrig
