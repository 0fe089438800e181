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

#include "gemv_common.cuh"
#include "routing.cuh"

namespace bigrig {

void dl_wait_test(uint32_t* phantom, uint32_t* spin_limit);   // decode_layer.cu test hook

namespace {

constexpr int kDsCW = 16;                 // consumer warps
constexpr int kDsCT = kDsCW * 32;
constexpr int kDsRows = 16;               // rows of a gate/up tile (the MMA's M)
constexpr int kDsFeat = 64;               // features of a unit (one quantisation group)
constexpr int kDsTiles = 2 * kDsFeat / kDsRows;   // gate/up tiles of a unit (8)
constexpr int kDsDownRows = 256;          // rows of a down stage (one TMA box)
constexpr int kDsMaxStages = 12;
constexpr int kDsMaxBlocks = 4;           // blocks of the hidden dimension a warp owns
constexpr int kDsRouterPerCta = 4;
constexpr size_t kDsSmemLimit = 227 * 1024;
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

// Balanced base-256 digit p (0, 1, 2) of a fixed-point value |X| < 2^22, as a signed byte.
__device__ __forceinline__ int digit(int X, int p) {
  const int d0 = static_cast<int>(static_cast<int8_t>(X & 0xFF));
  if (p == 0) return d0;
  const int X1 = (X - d0) >> 8;
  const int d1 = static_cast<int>(static_cast<int8_t>(X1 & 0xFF));
  if (p == 1) return d1;
  return (X1 - d1) >> 8;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// Exponent e with max|v| < 2^e (v finite), so that |round(v 2^(22-e))| < 2^22; 0 for 0.
__device__ __forceinline__ int fixed_exp(float amax) {
  if (!(amax > 0.f)) return 0;
  int e;
  frexpf(amax, &e);                        // amax = m 2^e, m in [0.5, 1)
  return e;
}


// MMA row g of a gate/up tile reads tile row kRowOf[g] (and kRowOf[g] + 8): with the
// 128-byte swizzle (16-byte chunk c of tile row r at c ^ (r & 7)) the eight lanes of a
// load phase -- rows g = 2q, 2q + 1 -- then hit eight different bank groups.
__device__ __forceinline__ int row_of(int g) { return (g >> 1) | ((g & 1) << 2); }

// Byte offset of 16-byte chunk c (0..7 within a 128-byte piece) of tile row r, piece p, in a
// swizzled stage laid out [piece][16 rows][128 bytes].
__device__ __forceinline__ int swz(int p, int r, int c) {
  return ((p * kDsRows + r) << 7) + ((c ^ (r & 7)) << 4);
}

// B fragments (the activation's digit planes) of one block of the hidden dimension.
//   4-bit block: 128 codes = two groups, 4 MMAs; MMA m takes word 4t + m of the block from
//     lane t: even nibbles at k-slots 4t.., odd nibbles at 16 + 4t..; columns 0-2 are the
//     planes of the block's first group (lanes t = 0, 1 carry it), 3-5 of the second
//   8-bit block: 64 codes = one group, 2 MMAs; MMA m takes words 4t + 2m (k-slots 4t..)
//     and 4t + 2m + 1 (16 + 4t..); columns 0-2 the planes
// X: the fixed-point activation in shared memory; k0: the block's first element; ng:
// groups of the block that exist (1 for the half block at the end of a 4-bit row).
template <int BITS>
__device__ __forceinline__ void b_block(const int* X, int k0, int ng, int g, int t, uint32_t* b) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t b0 = 0, b1 = 0;
      if (g < 3 * ng && (t >> 1) == g / 3) {
        const int p = g % 3;
        const int* e = X + k0 + 8 * (4 * t + m);
        b0 = pack4(digit(e[0], p), digit(e[2], p), digit(e[4], p), digit(e[6], p));
        b1 = pack4(digit(e[1], p), digit(e[3], p), digit(e[5], p), digit(e[7], p));
      }
      b[2 * m] = b0;
      b[2 * m + 1] = b1;
    }
  } else {
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      uint32_t b0 = 0, b1 = 0;
      if (g < 3) {
        const int* e = X + k0 + 4 * (4 * t + 2 * m);
        b0 = pack4(digit(e[0], g), digit(e[1], g), digit(e[2], g), digit(e[3], g));
        b1 = pack4(digit(e[4], g), digit(e[5], g), digit(e[6], g), digit(e[7], g));
      }
      b[2 * m] = b0;
      b[2 * m + 1] = b1;
    }
  }
}

// B fragments of the down slice (64 elements of h, one group, 2 MMAs).  4-bit: lane t takes
// words 2t, 2t + 1 of a row's 8; MMA m word 2t + m, even / odd nibbles.  8-bit: as b_block.
template <int BITS>
__device__ __forceinline__ void b_down(const int* hX, int g, int t, uint32_t* b) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      uint32_t b0 = 0, b1 = 0;
      if (g < 3) {
        const int* e = hX + 8 * (2 * t + m);
        b0 = pack4(digit(e[0], g), digit(e[2], g), digit(e[4], g), digit(e[6], g));
        b1 = pack4(digit(e[1], g), digit(e[3], g), digit(e[5], g), digit(e[7], g));
      }
      b[2 * m] = b0;
      b[2 * m + 1] = b1;
    }
  } else {
    b_block<8>(hX, 0, 1, g, t, b);
  }
}

// The lane's share of two rows' dot product over one block, from its int32 accumulator
// columns 2t, 2t+1 (column c = plane c % 3 of the block's group c / 3): per group
// s * 256^plane * d, plus b * sum(x) of the group from the lane holding its plane 0.
// sc / bi: the two rows' scales and biases of group G0 and G0 + 1 (fp32); xs: group sums.
__device__ __forceinline__ void flush2(const int* d, int t, int ng, const float* s_lo,
                                       const float* s_hi, const float* b_lo, const float* b_hi,
                                       const float* xsum, float& p_lo, float& p_hi) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int col = 2 * t + c;
    const int grp = col / 3, pl = col % 3;
    if (col < 3 * ng) {
      const float w = pl == 0 ? 1.f : pl == 1 ? 256.f : 65536.f;
      p_lo = fmaf(s_lo[grp] * w, static_cast<float>(d[c]), p_lo);
      p_hi = fmaf(s_hi[grp] * w, static_cast<float>(d[2 + c]), p_hi);
      if (pl == 0) {
        p_lo = fmaf(b_lo[grp], xsum[grp], p_lo);
        p_hi = fmaf(b_hi[grp], xsum[grp], p_hi);
      }
    }
  }
}


__device__ __forceinline__ void ds_tma5(void* dst, const CUtensorMap* m, int c0, int c1, int c2,
                                        int c3, int c4, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void ds_tma3(void* dst, const CUtensorMap* m, int c0, int c1, int c2,
                                        uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint4 ds_lds128(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// tm_gu: the gate/up codes as [128-byte piece bytes][row][piece][gate, up][slot], box of
// one tile's 16 rows x a chunk of pieces, 128-byte swizzle.  tm_dn: the down codes as
// [row bytes][row][slot], box of one group's bytes x 256 rows.
template <int BITS, int SDT>
__global__ void __launch_bounds__((kDsCW + 1) * 32, 1) decode_split_kernel(
    SplitArgs a, const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dn) {
  constexpr int GB = BITS == 4 ? 2 : 1;          // quantisation groups of a 64-byte block
  constexpr int MPB = BITS == 4 ? 4 : 2;         // MMAs of a block
  constexpr int GBYTES = 64 * BITS / 8;          // bytes of one group of a row
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ float s_lg[kMaxExperts];
  __shared__ int32_t s_g2s[kMaxExperts];
  __shared__ int32_t s_idx[32], s_slot[32];
  __shared__ float s_sc[32], s_rank_lg[32];
  __shared__ float s_red[kDsCW];
  __shared__ unsigned long long s_epoch;
  __shared__ float s_hscale, s_hsum, s_xs;
  const bigrig_expert_layout& L = a.L;
  const int H = L.hidden, I = L.inter, E = a.E, k = a.k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool producer = warp == kDsCW;
  const int G = gridDim.x, cta = blockIdx.x;
  const int gh = H / 64, gi = I / 64;
  const int nblk = (gh + GB - 1) / GB;
  const int pitch_h = H * BITS / 8;
  const int pieces = (pitch_h + 127) / 128;
  const int nch = a.nch, cpieces = pieces / nch, cblk = 2 * cpieces;
  const int U = k * gi;
  const int my_units = cta < U ? (U - 1 - cta) / G + 1 : 0;
  const int rd = H < kDsDownRows ? H : kDsDownRows;
  const int nd = (H + rd - 1) / rd;
  const int n_gu = kDsTiles * nch;
  const int gu_code = kDsRows * cpieces * 128;
  const int sc_bytes = kDsRows * gh * 2;
  const int nst = a.nstages, stage_bytes = a.stage_bytes;

  // the ring first (1024-byte aligned for the swizzle), then the CTA's other buffers
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
  float* part = sc.take<float>(2 * kDsFeat * kDsCW * 4);
  uint32_t* dsb = sc.take<uint32_t>(static_cast<size_t>(H) * 4);
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
    if (lane == 1) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_gu)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_dn)) : "memory");
    }
    for (int e = lane; e < E; e += 32) s_g2s[e] = a.g2s ? a.g2s[e] : e;
  }
  if (threadIdx.x < 32) s_idx[threadIdx.x] = -1;
  __syncthreads();
  const unsigned long long epoch = s_epoch;
  const unsigned long long tag = ((epoch + 1ull) & 0xffffffffull) << 32;

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
    // the fixed-point copy of x: its largest magnitude first
    float m = 0.f;
    for (int i = threadIdx.x; i < H; i += kDsCT) m = fmaxf(m, fabsf(bf16_bits_to_f32(xraw[i])));
    m = warp_max(m);
    if (lane == 0) s_red[warp] = m;
  }
  __syncthreads();                               // router rows read: the ring is free
  if (!producer) {
    float m = 0.f;
    for (int w = 0; w < kDsCW; ++w) m = fmaxf(m, s_red[w]);
    const int e = fixed_exp(m);
    const float up = ldexpf(1.f, 22 - e);
    for (int i = threadIdx.x; i < H; i += kDsCT)
      X[i] = __float2int_rn(bf16_bits_to_f32(xraw[i]) * up);
    // group sums of x: one warp per group, two elements a lane, a fixed shuffle tree
    for (int grp = warp; grp < gh; grp += kDsCW) {
      float v = bf16_bits_to_f32(xraw[grp * 64 + lane]) + bf16_bits_to_f32(xraw[grp * 64 + 32 + lane]);
      v = warp_sum(v);
      if (lane == 0) xsum[grp] = v;
    }
    if (threadIdx.x == 0) s_xs = ldexpf(1.f, e - 22);
  }


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
            ds_tma5(dst, &tm_gu, 0, row0, ch * cpieces, proj, slot, full + b, once);
          } else if (lane == 1) {
            bulk_g2s_hint(dst + gu_code, ebase + L.scales_off[proj] + static_cast<int64_t>(row0) * gh * 2,
                          sc_bytes, full + b, once);
          } else if (lane == 2) {
            bulk_g2s_hint(dst + gu_code + sc_bytes,
                          ebase + L.biases_off[proj] + static_cast<int64_t>(row0) * gh * 2, sc_bytes,
                          full + b, once);
          }
        } else {
          const int d = st - n_gu;
          if (lane == 0) {
            bar_expect_tx(full + b, static_cast<uint32_t>(rd * GBYTES));
            ds_tma3(dst, &tm_dn, grp * GBYTES, d * rd, slot, full + b, once);
          }
        }
        __syncwarp();
      }
    }
    return;                                      // the consumers wait for every stage it filled
  }


  // ---------------------------------------------------------------- consumers
  // warp w owns blocks w, w + 16, ... of the hidden dimension in every tile; its B
  // fragments (the token's digit planes) stay in registers for the whole layer
  const float xs = s_xs;
  uint32_t breg[kDsMaxBlocks][2 * MPB];
#pragma unroll
  for (int bi = 0; bi < kDsMaxBlocks; ++bi) {
    const int blk = warp + kDsCW * bi;
    if (blk < nblk) {
      b_block<BITS>(X, blk * 64 * GB, min(GB, gh - blk * GB), g, t, breg[bi]);
    } else {
#pragma unroll
      for (int i = 0; i < 2 * MPB; ++i) breg[bi][i] = 0u;
    }
  }
  const int rl = row_of(g), rh = rl + 8;
  const int n_drows = (H + kDsCT - 1) / kDsCT;   // down rows whose scales a thread loads
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
    // this unit's down scales and biases (one of each per row), loaded now and stored after
    // the gate/up tiles so that their latency hides behind them
    uint32_t dsr[4096 / kDsCT];
    {
      const uint16_t* sp = reinterpret_cast<const uint16_t*>(ebase + L.scales_off[2]) + grp;
      const uint16_t* bp = reinterpret_cast<const uint16_t*>(ebase + L.biases_off[2]) + grp;
#pragma unroll
      for (int i = 0; i < 4096 / kDsCT; ++i) {
        const int r = threadIdx.x + i * kDsCT;
        dsr[i] = 0u;
        if (i < n_drows && r < H)
          dsr[i] = static_cast<uint32_t>(ld_nc_u16(sp + static_cast<size_t>(r) * gi)) |
                   (static_cast<uint32_t>(ld_nc_u16(bp + static_cast<size_t>(r) * gi)) << 16);
      }
    }
    // ---- gate/up: 8 tiles of 16 rows (4 gate, then 4 up), each in nch K chunks
    for (int r = 0; r < kDsTiles; ++r) {
      float p_lo = 0.f, p_hi = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++q) {
        const int b = q % nst;
        const bool landed = ds_wait(full + b, (q / nst) & 1, a.err);
        const uint8_t* st = ring + static_cast<size_t>(b) * stage_bytes;
        const uint16_t* ssc = reinterpret_cast<const uint16_t*>(st + gu_code);
        const uint16_t* sbi = ssc + kDsRows * gh;
        if (landed) {
#pragma unroll
          for (int bi = 0; bi < kDsMaxBlocks; ++bi) {
            const int blk = warp + kDsCW * bi;
            if (blk >= nblk || blk < ch * cblk || blk >= (ch + 1) * cblk) continue;
            const int lb = blk - ch * cblk;
            const int ng = min(GB, gh - blk * GB);
            const int c16 = 4 * (lb & 1) + t;
            uint4 wl = ds_lds128(st + swz(lb >> 1, rl, c16));
            uint4 wh = ds_lds128(st + swz(lb >> 1, rh, c16));
            if (BITS == 4 && ng == 1 && t >= 2) wl = wh = make_uint4(0u, 0u, 0u, 0u);
            const uint32_t ul[4] = {wl.x, wl.y, wl.z, wl.w};
            const uint32_t uh[4] = {wh.x, wh.y, wh.z, wh.w};
            int d[4] = {0, 0, 0, 0};
#pragma unroll
            for (int m = 0; m < MPB; ++m) {
              if constexpr (BITS == 4)
                mma_u8s8(d, lo_nibbles(ul[m]), lo_nibbles(uh[m]), hi_nibbles(ul[m]), hi_nibbles(uh[m]),
                         breg[bi][2 * m], breg[bi][2 * m + 1]);
              else
                mma_u8s8(d, ul[2 * m], uh[2 * m], ul[2 * m + 1], uh[2 * m + 1], breg[bi][2 * m],
                         breg[bi][2 * m + 1]);
            }
            const int G0 = blk * GB;
            float s_lo[2], s_hi[2], b_lo[2], b_hi[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int gg = G0 + (i < ng ? i : 0);
              s_lo[i] = half_to_f32<SDT>(ssc[rl * gh + gg]) * xs;
              s_hi[i] = half_to_f32<SDT>(ssc[rh * gh + gg]) * xs;
              b_lo[i] = half_to_f32<SDT>(sbi[rl * gh + gg]);
              b_hi[i] = half_to_f32<SDT>(sbi[rh * gh + gg]);
            }
            flush2(d, t, ng, s_lo, s_hi, b_lo, b_hi, xsum + G0, p_lo, p_hi);
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
        part[(r * kDsRows + rl) * kDsCW + warp] = p_lo;
        part[(r * kDsRows + rh) * kDsCW + warp] = p_hi;
      }
    }
#pragma unroll
    for (int i = 0; i < 4096 / kDsCT; ++i) {
      const int r = threadIdx.x + i * kDsCT;
      if (i < n_drows && r < H) dsb[r] = dsr[i];
    }
    ds_named_sync(1, kDsCT);
    // ---- h = bf16(silu(gate) * up) for the unit's 64 features; the partials of each row
    // added in warp order
    if (threadIdx.x < kDsFeat) {
      const int f = threadIdx.x;
      float gv = 0.f, uv = 0.f;
      for (int w = 0; w < kDsCW; ++w) {
        gv += part[f * kDsCW + w];
        uv += part[(kDsFeat + f) * kDsCW + w];
      }
      const float h = bf16_round(silu_f32(gv) * uv);
      hv[f] = h;
      const float m = warp_max(fabsf(h));
      if (lane == 0) s_red[warp] = m;
    }
    ds_named_sync(1, kDsCT);
    if (threadIdx.x < kDsFeat) {
      const int e = fixed_exp(fmaxf(s_red[0], s_red[1]));
      hX[threadIdx.x] = __float2int_rn(hv[threadIdx.x] * ldexpf(1.f, 22 - e));
      if (threadIdx.x == 0) s_hscale = ldexpf(1.f, e - 22);
      if (warp == 0) {
        const float v = warp_sum(hv[lane] + hv[lane + 32]);
        if (lane == 0) s_hsum = v;
      }
    }
    ds_named_sync(1, kDsCT);
    uint32_t bd[4];
    b_down<BITS>(hX, g, t, bd);
    const float hs = s_hscale, hsum = s_hsum;
    // ---- down: this unit's 64 columns of all H rows, 256 rows a stage, 16 a warp
    for (int dd = 0; dd < nd; ++dd, ++q) {
      const int b = q % nst;
      const bool landed = ds_wait(full + b, (q / nst) & 1, a.err);
      const uint8_t* st = ring + static_cast<size_t>(b) * stage_bytes;
      if (landed && warp * kDsRows < rd) {
        const int row_lo = dd * rd + warp * kDsRows + g, row_hi = row_lo + 8;
        const uint8_t* al = st + (warp * kDsRows + g) * GBYTES;
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
        const uint32_t vl = row_lo < H ? dsb[row_lo] : 0u, vh = row_hi < H ? dsb[row_hi] : 0u;
        const float s_lo = half_to_f32<SDT>(static_cast<uint16_t>(vl)) * hs;
        const float s_hi = half_to_f32<SDT>(static_cast<uint16_t>(vh)) * hs;
        const float b_lo = half_to_f32<SDT>(static_cast<uint16_t>(vl >> 16));
        const float b_hi = half_to_f32<SDT>(static_cast<uint16_t>(vh >> 16));
        float y_lo = 0.f, y_hi = 0.f;
        flush2(d, t, 1, &s_lo, &s_hi, &b_lo, &b_hi, &hsum, y_lo, y_hi);
        y_lo += __shfl_xor_sync(0xffffffffu, y_lo, 1);
        y_hi += __shfl_xor_sync(0xffffffffu, y_hi, 1);
        y_lo += __shfl_xor_sync(0xffffffffu, y_lo, 2);
        y_hi += __shfl_xor_sync(0xffffffffu, y_hi, 2);
        if (t == 0) {
          if (row_lo < H) yp[row_lo] = y_lo;
          if (row_hi < H) yp[row_hi] = y_hi;
        }
      }
      __syncwarp();
      if (lane == 0) ds_arrive(empty + b);
    }
    ds_named_sync(1, kDsCT);
    for (int i = threadIdx.x * 4; i < H; i += kDsCT * 4)
      *reinterpret_cast<float4*>(ydst + i) = *reinterpret_cast<const float4*>(yp + i);
  }


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

  // ---------------------------------------------------------------- combine
  // rows [cta R, cta R + R): y of each routed expert is its units' partials added in group
  // order and rounded to bf16; the experts are added in rank order, then the residual
  const int R = (H + G - 1) / G;
  const int row0 = cta * R;
  if (row0 >= H) return;
  const bool scores = ds_wait(bar_s, 0, a.err);
  float* ysm = part;
  for (int idx = threadIdx.x; idx < k * R; idx += kDsCT) {
    const int j = idx / R, r = idx - j * R, row = row0 + r;
    float y = 0.f;
    if (row < H && s_slot[j] >= 0) {
      const float* src = a.ypart + static_cast<size_t>(j) * gi * H + row;
      for (int gg = 0; gg < gi; ++gg) {
        float v;
        asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(src + static_cast<size_t>(gg) * H));
        y += v;
      }
    }
    ysm[idx] = bf16_round(y);
  }
  ds_named_sync(1, kDsCT);
  for (int r = threadIdx.x; r < R && row0 + r < H; r += kDsCT) {
    const int row = row0 + r;
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc = acc + (scores ? s_sc[j] : 0.f) * ysm[j * R + r];
    if (a.residual) acc = bf16_bits_to_f32(a.residual[row]) + bf16_round(acc);
    a.out[row] = f32_to_bf16_bits(acc);
  }
}

}  // namespace
}  // namespace bigrig

namespace bigrig {
namespace {

struct SplitPlan {
  int stage_bytes, nstages, nch;
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

// The split kernel's plan for a layer, or false when it cannot run it: the gated SwiGLU
// expert without projection biases, 4- or 8-bit codes in groups of 64, a hidden
// dimension of at most 4096 (16 warps x 4 blocks; down scales held 8 a thread), at most
// 32 routed experts, and a ring of at least two stages beside the fixed buffers.
bool decode_split_plan(const bigrig_expert_layout& L, int k, int E, int G, SplitPlan* p) {
  if (G <= 0 || k < 1 || k > 32 || E < 1 || E > kMaxExperts) return false;
  if (L.group_size != 64 || L.flags != 0 || (L.bits != 4 && L.bits != 8)) return false;
  const int H = L.hidden, I = L.inter;
  if (H % 64 || I % 64 || H > 4096 || H < 64) return false;
  const int gh = H / 64, GB = L.bits == 4 ? 2 : 1;
  if ((gh + GB - 1) / GB > kDsCW * kDsMaxBlocks) return false;
  const int pitch = H * L.bits / 8, pieces = (pitch + 127) / 128;
  int nch = 1;
  while (kDsRows * (pieces / nch) * 128 > 32768 && pieces % (2 * nch) == 0) nch *= 2;
  const size_t gu = static_cast<size_t>(kDsRows) * (pieces / nch) * 128 + 2 * kDsRows * gh * 2;
  const int rd = H < kDsDownRows ? H : kDsDownRows;
  const size_t dn = static_cast<size_t>(rd) * (64 * L.bits / 8);
  const size_t stage = ((gu > dn ? gu : dn) + 1023) / 1024 * 1024;
  const size_t fixed = 1024 + r128(kDsMaxStages * 8) * 2 + r128(4 * 8) + r128(H * 2) + r128(H * 4) +
                       r128(gh * 4) + r128(2 * kDsFeat * kDsCW * 4) + r128(H * 4) + r128(H * 4) +
                       r128(kDsFeat * 4) * 2;
  if (fixed >= kDsSmemLimit) return false;
  size_t nst = (kDsSmemLimit - fixed) / stage;
  if (nst > static_cast<size_t>(kDsMaxStages)) nst = kDsMaxStages;
  if (nst < 2 || nst * stage < static_cast<size_t>(kDsRouterPerCta) * H * 2) return false;
  if (static_cast<size_t>(k) * ((H + G - 1) / G) > static_cast<size_t>(2 * kDsFeat * kDsCW))
    return false;
  (void)I;
  p->stage_bytes = static_cast<int>(stage);
  p->nstages = static_cast<int>(nst);
  p->nch = nch;
  p->smem = fixed + nst * stage;
  return true;
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

// A byte map over the slab; false when the layout breaks a rule of tiled maps (16-byte
// aligned base and strides, 1..256 elements per box side) or the encoder refuses it.
bool ds_encode(CUtensorMap* m, int rank, const uint8_t* base, const cuuint64_t* dims,
               const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz) {
  DsEncodeFn fn = ds_encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  for (int i = 0; i < rank; ++i)
    if (box[i] < 1 || box[i] > 256 || dims[i] < box[i]) return false;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] == 0 || (strides[i] & 15)) return false;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, static_cast<cuuint32_t>(rank), const_cast<uint8_t*>(base),
            dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BITS, int SDT>
int ds_launch(const SplitArgs& args, const CUtensorMap& gu, const CUtensorMap& dn, size_t smem,
              int G, cudaStream_t s) {
  auto kern = decode_split_kernel<BITS, SDT>;
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
  cudaLaunchKernelEx(&cfg, kern, args, gu, dn);
  return check_launch("decode_split_kernel");
}

}  // namespace

bool decode_split_fits(const bigrig_expert_layout& L, int k, int E) {
  SplitPlan p;
  return decode_split_plan(L, k, E, ds_sm_count(), &p);
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
  const int64_t pitch_i = static_cast<int64_t>(L.inter) * L.bits / 8;
  const int pieces = static_cast<int>((pitch + 127) / 128);
  CUtensorMap gu, dn;
  {
    const cuuint64_t dims[5] = {128, static_cast<cuuint64_t>(L.inter), static_cast<cuuint64_t>(pieces), 2,
                                kDsMapSlots};
    const cuuint64_t strides[4] = {static_cast<cuuint64_t>(pitch), 128,
                                   static_cast<cuuint64_t>(L.weight_off[1] - L.weight_off[0]),
                                   static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t box[5] = {128, static_cast<cuuint32_t>(kDsRows),
                               static_cast<cuuint32_t>(pieces / p.nch), 1, 1};
    if (L.weight_off[1] <= L.weight_off[0] ||
        !ds_encode(&gu, 5, sl + L.weight_off[0], dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_split: cannot map the gate/up codes");
  }
  {
    const int rd = L.hidden < kDsDownRows ? L.hidden : kDsDownRows;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(pitch_i), static_cast<cuuint64_t>(L.hidden),
                                kDsMapSlots};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(pitch_i), static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(64 * L.bits / 8), static_cast<cuuint32_t>(rd), 1};
    if (!ds_encode(&dn, 3, sl + L.weight_off[2], dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_split: cannot map the down codes");
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
  dl_wait_test(&a.phantom, &a.spin_limit);
  if (a.spin_limit == 0) a.spin_limit = kDsSpinLimit;
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16) return ds_launch<4, BIGRIG_F16>(a, gu, dn, p.smem, G, s);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16) return ds_launch<4, BIGRIG_BF16>(a, gu, dn, p.smem, G, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16) return ds_launch<8, BIGRIG_F16>(a, gu, dn, p.smem, G, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16) return ds_launch<8, BIGRIG_BF16>(a, gu, dn, p.smem, G, s);
  return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_split: bits=%d scale_dtype=%d", L.bits,
                   L.scale_dtype);
}

}  // namespace bigrig
