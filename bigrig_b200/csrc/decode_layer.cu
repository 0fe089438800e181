// One decode token through one MoE layer in ONE persistent cooperative kernel.
//
// Replaces, for a single token, the launch chain route -> gate_up -> down+combine
// (decode.cu, gemv.cu), and with it the mlx_lm block's router, the per-expert
// quantized_matmul calls of _forward_views_one (bigrig_engine/stream.py:1278-1318) and
// the caller's weighted sum (stream.py:1523-1525).  An OLMoE decode layer moves ~28 MB,
// ~4 us of HBM time; as a chain of kernels every step also paid launches and dependent
// global round trips.  Here one CTA per SM runs the whole layer with CW consumer warps
// and one producer warp:
//
//   logits   CTA c < ceil(E/4) computes the logits of experts 4c..4c+3 (one warp each,
//            router rows bulk-copied as the kernel starts) and publishes each as a
//            64-bit (value, tag) word, the tag naming this launch -- no fence, no counter
//   routing  the producer warp of every CTA polls the E tagged words, ranks them
//            (topk_rank_warp: the same indices and scores as the chain's top-k) and
//            reads the slots from a copy of g2s staged at start
//   gate/up  items of (routed expert, 8 features), dealt round-robin to CTAs; the
//            producer streams a CTA's items through a ring of bulk copies with full /
//            empty mbarriers; consumer warp w computes feature w % 8 of every item of
//            its group with x held in registers, no block-wide barrier per item; h rows
//            go to global
//   barrier  grid-wide, consumer threads only (the producer is already streaming the
//            down-projection weights into the ring)
//   down     items of (8 hidden features, a group of routed experts); a warp per expert
//            of an item; then the combine in rank order plus the residual
//
// Per-feature arithmetic is the chain's (same chunk order per lane, same fp32x2 dot,
// same group affine, same warp sums, same combine), so the output is bit-identical to
// it.  Every wait -- mbarriers, tagged logits, the grid barrier -- is bounded; a timeout
// counts in the error words and the kernel carries on to its end.
#include "gemv_common.cuh"
#include "routing.cuh"

// Phase-boundary hook (thread 0 of each CTA); empty in the library, defined by
// instrumented builds that record per-CTA timestamps.
#ifndef DL_STAMP
#define DL_STAMP(i)
#endif

namespace bigrig {

constexpr int kDlFeat = 8;               // features of a gate/up item and of a down tile
constexpr int kDlRouterPerCta = 4;       // experts whose logits one CTA computes
constexpr int kDlMaxStages = 12;
constexpr uint32_t kDlSpinLimit = 1u << 22;

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
  uint16_t* h;                // [k, I] scratch, rank-ordered rows
  unsigned long long* tagged; // [E] logit bits | tag << 32
  uint32_t* sync;             // [3]: barrier count, barrier generation, launch epoch
  int32_t* err;
  int E, k, mode, norm;
  int stage_bytes, nstages, seg_per_item, max_tiles;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
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

template <int BITS, int SDT, int NCH, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) decode_layer_kernel(DecodeLayerArgs a) {
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  constexpr int NF = kDlFeat;
  constexpr int NGRP = CW / NF;            // consumer groups sharing the gate/up items
  constexpr int CT = CW * 32;              // consumer threads
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_lg[kMaxExperts];
  __shared__ int32_t s_g2s[kMaxExperts];
  __shared__ int32_t s_idx[32], s_slot[32];
  __shared__ float s_sc[32], s_rank_lg[32];
  __shared__ uint32_t s_epoch;
  const bigrig_expert_layout& L = a.L;
  const int H = L.hidden, I = L.inter, E = a.E, k = a.k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool producer = warp == CW;
  const int G = gridDim.x, cta = blockIdx.x;
  const int pitch_h = H * BITS / 8, pitch_i = I * BITS / 8;
  const int gh = H / L.group_size, gi = I / L.group_size;
  const int nch_h = H / CPL, nch_i = I / CPL;
  const int nst = a.nstages, stage_bytes = a.stage_bytes;
  uint32_t* bar_count = a.sync;
  uint32_t* bar_gen = a.sync + 1;
  uint32_t* epoch = a.sync + 2;

  SmemCarve sc(smem);
  uint64_t* bars = sc.take<uint64_t>((2 * kDlMaxStages + 3) * 8);
  uint16_t* xraw = sc.take<uint16_t>(static_cast<size_t>(H) * 2);
  float* xs = sc.take<float>(static_cast<size_t>(H) * 4);
  float* xcs = sc.take<float>(static_cast<size_t>(nch_h) * 4);
  uint16_t* hraw = sc.take<uint16_t>(static_cast<size_t>(k) * I * 2);
  float* hs = sc.take<float>(static_cast<size_t>(k) * I * 4);
  float* hcs = sc.take<float>(static_cast<size_t>(k) * nch_i * 4);
  float* ybuf = sc.take<float>(static_cast<size_t>(a.max_tiles) * k * NF * 4);
  uint8_t* ring = sc.take<uint8_t>(static_cast<size_t>(nst) * stage_bytes);
  uint16_t* wr = reinterpret_cast<uint16_t*>(ring);     // router rows, before any item
  uint64_t* full = bars;
  uint64_t* empty = bars + kDlMaxStages;
  uint64_t* bar_x = bars + 2 * kDlMaxStages;
  uint64_t* bar_r = bar_x + 1;
  uint64_t* bar_h = bar_x + 2;
  DL_STAMP(0);

  // ---------------------------------------------------------------- start
  const int n_mine = max(0, min(kDlRouterPerCta, E - cta * kDlRouterPerCta));
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      bar_init(full + i, 1);
      bar_init(empty + i, CW);
    }
    bar_init(bar_x, 1);
    bar_init(bar_r, 1);
    bar_init(bar_h, 1);
    bar_expect_tx(bar_x, H * 2);
    bulk_g2s(xraw, a.x, H * 2, bar_x);
    if (n_mine > 0) {
      bar_expect_tx(bar_r, static_cast<uint32_t>(n_mine) * H * 2);
      bulk_g2s(wr, a.gate_w + static_cast<size_t>(cta) * kDlRouterPerCta * H, n_mine * H * 2,
               bar_r);
    }
  }
  if (producer) {
    if (lane == 0) s_epoch = ld_acquire_u32(epoch);
    for (int e = lane; e < E; e += 32) s_g2s[e] = a.g2s ? a.g2s[e] : e;
  }
  __syncthreads();
  const unsigned long long tag = static_cast<unsigned long long>(s_epoch + 1u) << 32;

  // ---------------------------------------------------------------- router logits
  bool xok = true;
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

  const int tiles_g = I / NF;
  const int n_items = k * tiles_g;
  const int my_items = cta < n_items ? (n_items - 1 - cta) / G + 1 : 0;
  const int tiles_d = H / NF;
  const int my_tiles = cta < tiles_d ? (tiles_d - 1 - cta) / G + 1 : 0;
  const int spi = a.seg_per_item;
  const int ipt = (k + spi - 1) / spi;           // down items per tile
  const int n_down = my_tiles * ipt;
  const int seg_bytes = NF * pitch_i + 2 * NF * gi * 2;

  if (producer) {
    // ------------------------------------------------------------ routing
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
      if (n > kDlSpinLimit) {
        if (lane == 0) atomicAdd(a.err + 1, 1);
        for (int i = 0; i < kMaxExperts / 32; ++i)
          if (need & (1u << i)) s_lg[lane + 32 * i] = __int_as_float(0x7fc00000);
        break;
      }
    }
    __syncwarp();
    const int per = (E + 31) / 32;
#define BIGRIG_TK(N) \
  if (per == N) topk_rank_warp<N>(s_lg, E, k, a.mode, a.norm, s_idx, s_sc, s_rank_lg);
    BIGRIG_TK(1) BIGRIG_TK(2) BIGRIG_TK(3) BIGRIG_TK(4)
    BIGRIG_TK(5) BIGRIG_TK(6) BIGRIG_TK(7) BIGRIG_TK(8)
#undef BIGRIG_TK
    if (lane < k) {
      const int e = s_idx[lane];
      const int slot = (e >= 0 && e < E) ? s_g2s[e] : -1;
      s_slot[lane] = slot;
      if (cta == 0) {
        a.idx_out[lane] = e;
        a.sc_out[lane] = s_sc[lane];
        if (slot < 0) atomicAdd(a.err, 1);
      }
    }
    __syncwarp();
    DL_STAMP(2);
    // ------------------------------------------------------------ stream the ring
    if (lane == 0) {
      const uint32_t item_bytes = static_cast<uint32_t>(2 * NF * pitch_h + 4 * NF * gh * 2);
      for (int q = 0; q < my_items + n_down; ++q) {
        const int b = q % nst;
        if (q >= nst) stage_wait(empty + b, ((q / nst) - 1) & 1, a.err);
        uint8_t* dst = ring + static_cast<size_t>(b) * stage_bytes;
        if (q < my_items) {
          const int it = cta + q * G;
          const int s = it / tiles_g, f0 = (it - s * tiles_g) * NF;
          const int slot = s_slot[s];
          bar_expect_tx(full + b, slot >= 0 ? item_bytes : 0u);
          if (slot < 0) continue;
          const uint8_t* base = a.slab + static_cast<int64_t>(slot) * L.slot_stride;
          uint16_t* sb = reinterpret_cast<uint16_t*>(dst + 2 * NF * pitch_h);
          for (int m = 0; m < 2; ++m) {
            bulk_g2s(dst + m * NF * pitch_h, base + L.weight_off[m] + static_cast<int64_t>(f0) * pitch_h,
                     NF * pitch_h, full + b);
            bulk_g2s(sb + (2 * m) * NF * gh, base + L.scales_off[m] + static_cast<int64_t>(f0) * gh * 2,
                     NF * gh * 2, full + b);
            bulk_g2s(sb + (2 * m + 1) * NF * gh,
                     base + L.biases_off[m] + static_cast<int64_t>(f0) * gh * 2, NF * gh * 2, full + b);
          }
        } else {
          const int d = q - my_items;
          const int f0 = (cta + (d / ipt) * G) * NF;
          const int s0 = (d % ipt) * spi, s1 = min(k, s0 + spi);
          uint32_t bytes = 0;
          for (int s = s0; s < s1; ++s) bytes += s_slot[s] >= 0 ? seg_bytes : 0;
          bar_expect_tx(full + b, bytes);
          for (int s = s0; s < s1; ++s) {
            if (s_slot[s] < 0) continue;
            const uint8_t* base = a.slab + static_cast<int64_t>(s_slot[s]) * L.slot_stride;
            uint8_t* dd = dst + static_cast<size_t>(s - s0) * seg_bytes;
            uint16_t* sb = reinterpret_cast<uint16_t*>(dd + NF * pitch_i);
            bulk_g2s(dd, base + L.weight_off[2] + static_cast<int64_t>(f0) * pitch_i, NF * pitch_i,
                     full + b);
            bulk_g2s(sb, base + L.scales_off[2] + static_cast<int64_t>(f0) * gi * 2, NF * gi * 2,
                     full + b);
            bulk_g2s(sb + NF * gi, base + L.biases_off[2] + static_cast<int64_t>(f0) * gi * 2,
                     NF * gi * 2, full + b);
          }
        }
      }
    }
    return;                                      // consumers wait for every stage it filled
  }

  // ---------------------------------------------------------------- consumers: x in registers
  relayout_rows<BITS>(xs, xcs, xraw, H, 1, threadIdx.x, CT);
  named_sync(1, CT);
  ChunkX<BITS> cx[NCH];
  float xc[NCH];
  {
    const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch_h) {
        load_chunk_x<BITS>(cx[i], x4 + c, nch_h);
        xc[i] = xcs[c];
      } else {
        xc[i] = 0.f;
#pragma unroll
        for (int q = 0; q < CPL / 2; ++q) cx[i].v[q] = make_float2(0.f, 0.f);
      }
    }
  }

  // ---------------------------------------------------------------- gate/up
  const int grp = warp / NF, fl = warp % NF;
  for (int j = 0; j < my_items; ++j) {
    const int b = j % nst;
    const bool landed = stage_wait(full + b, (j / nst) & 1, a.err);
    if (j == 0) DL_STAMP(3);
    if (j % NGRP == grp) {
      const int it = cta + j * G;
      const int s = it / tiles_g, f0 = (it - s * tiles_g) * NF;
      const bool have = s_slot[s] >= 0 && landed && xok;
      const uint8_t* st = ring + static_cast<size_t>(b) * stage_bytes;
      const uint16_t* sb = reinterpret_cast<const uint16_t*>(st + 2 * NF * pitch_h);
      float ag = 0.f, au = 0.f;
      if (have) {
        const uint8_t* wg = st + fl * pitch_h;
        const uint8_t* wu = st + (NF + fl) * pitch_h;
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
          const int c = lane + 32 * i;
          if (c < nch_h) {
            const int g = (c * CPL) / L.group_size;
            const uint4 cg = *reinterpret_cast<const uint4*>(wg + c * 16);
            const uint4 cu = *reinterpret_cast<const uint4*>(wu + c * 16);
            const float dg = chunk_dot2<BITS>(cg, cx[i]);
            const float du = chunk_dot2<BITS>(cu, cx[i]);
            ag = fmaf(half_to_f32<SDT>(sb[(0 * NF + fl) * gh + g]), dg,
                      fmaf(half_to_f32<SDT>(sb[(1 * NF + fl) * gh + g]), xc[i], ag));
            au = fmaf(half_to_f32<SDT>(sb[(2 * NF + fl) * gh + g]), du,
                      fmaf(half_to_f32<SDT>(sb[(3 * NF + fl) * gh + g]), xc[i], au));
          }
        }
      }
      const float gv = warp_sum(ag);
      const float uv = warp_sum(au);
      if (lane == 0)
        a.h[static_cast<size_t>(s) * I + f0 + fl] = have ? f32_to_bf16_bits(silu_f32(gv) * uv) : 0;
    }
    __syncwarp();
    if (lane == 0) bar_arrive(empty + b);
  }
  DL_STAMP(4);

  // ---------------------------------------------------------------- grid barrier
  __threadfence();
  named_sync(1, CT);
  if (threadIdx.x == 0) {
    const uint32_t gen = ld_acquire_u32(bar_gen);
    if (atomicAdd(bar_count, 1u) == static_cast<uint32_t>(G) - 1) {
      // every CTA read this launch's epoch at its start: advance it for the next launch
      atomicExch(bar_count, 0u);
      atomicAdd(epoch, 1u);
      __threadfence();
      atomicAdd(bar_gen, 1u);
    } else {
      uint32_t n = 0;
      while (ld_acquire_u32(bar_gen) == gen) {
        if (++n > kDlSpinLimit) {
          atomicAdd(a.err + 1, 1);
          break;
        }
        __nanosleep(20);
      }
    }
    __threadfence();
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
  relayout_rows<BITS>(hs, hcs, hraw, I, k, threadIdx.x, CT);
  named_sync(1, CT);
  DL_STAMP(6);
  const float4* h4 = reinterpret_cast<const float4*>(hs);
  const int dgroups = CW / spi;                  // down items in flight at once
  const int dgrp = warp / spi, dseg = warp % spi;
  for (int d = 0; d < n_down; ++d) {
    const int q = my_items + d;
    const int b = q % nst;
    const bool landed = stage_wait(full + b, (q / nst) & 1, a.err) && hok;
    if (dgrp < dgroups && d % dgroups == dgrp) {
      const int tl = d / ipt;
      const int s0 = (d % ipt) * spi;
      const int s = s0 + dseg;
      if (s < k) {
        const bool have = s_slot[s] >= 0 && landed;
        const uint8_t* wc = ring + static_cast<size_t>(b) * stage_bytes + static_cast<size_t>(dseg) * seg_bytes;
        const uint16_t* sb = reinterpret_cast<const uint16_t*>(wc + NF * pitch_i);
        float acc[NF];
#pragma unroll
        for (int f = 0; f < NF; ++f) acc[f] = 0.f;
        if (have) {
          for (int c = lane; c < nch_i; c += 32) {
            const int g = (c * CPL) / L.group_size;
            ChunkX<BITS> ch;
            load_chunk_x<BITS>(ch, h4 + static_cast<size_t>(s) * Q * nch_i + c, nch_i);
            const float csum = hcs[s * nch_i + c];
#pragma unroll
            for (int f = 0; f < NF; ++f) {
              const uint4 cw = *reinterpret_cast<const uint4*>(wc + f * pitch_i + c * 16);
              const float dv = chunk_dot2<BITS>(cw, ch);
              acc[f] = fmaf(half_to_f32<SDT>(sb[f * gi + g]), dv,
                            fmaf(half_to_f32<SDT>(sb[(NF + f) * gi + g]), csum, acc[f]));
            }
          }
        }
#pragma unroll
        for (int f = 0; f < NF; ++f) {
          const float v = warp_sum(acc[f]);
          if (lane == 0) ybuf[(tl * k + s) * NF + f] = have ? bf16_round(v) : 0.f;
        }
      }
    }
    __syncwarp();
    if (lane == 0) bar_arrive(empty + b);
  }
  named_sync(1, CT);
  // combine in rank order, plus the residual
  if (threadIdx.x < my_tiles * NF) {
    const int tl = threadIdx.x / NF, f = threadIdx.x % NF;
    const int o = (cta + tl * G) * NF + f;
    float acc = 0.f;
    for (int r = 0; r < k; ++r) acc = acc + s_sc[r] * ybuf[(tl * k + r) * NF + f];
    if (a.residual) acc = bf16_bits_to_f32(a.residual[o]) + bf16_round(acc);
    a.out[o] = f32_to_bf16_bits(acc);
  }
  DL_STAMP(7);
}

// ------------------------------------------------------------------ launcher
namespace {

constexpr size_t kDlSmemLimit = 220 * 1024;

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
  int nch;          // 16-byte code chunks per lane of a hidden row (register-resident x)
  int cw;           // consumer warps
  int stage_bytes, nstages, seg_per_item, max_tiles;
  size_t smem;
};

// The persistent kernel's plan for a layer, or false when it cannot run it: more than
// 32 routed experts, a hidden row too wide to keep in registers, a layer whose fixed
// shared memory leaves no room for a ring of two stages.
bool decode_layer_plan(const bigrig_expert_layout& L, int k, int E, int G, DlPlan* p) {
  if (G <= 0 || k > 32 || E > kMaxExperts || L.hidden % kDlFeat || L.inter % kDlFeat) return false;
  const int cpl = 128 / L.bits;
  const int nch_h = L.hidden / cpl, nch_i = L.inter / cpl;
  const int nch = (nch_h + 31) / 32;
  if (nch > 4) return false;
  p->nch = nch <= 2 ? 2 : 4;
  p->cw = p->nch == 2 ? 16 : 8;
  const size_t ph = static_cast<size_t>(L.hidden) * L.bits / 8;
  const size_t pi = static_cast<size_t>(L.inter) * L.bits / 8;
  const size_t gh = L.hidden / L.group_size, gi = L.inter / L.group_size;
  const size_t item = 2 * kDlFeat * ph + 4 * kDlFeat * gh * 2;
  const size_t seg = kDlFeat * pi + 2 * kDlFeat * gi * 2;
  const size_t stage = item > seg ? item : seg;
  int spi = static_cast<int>(stage / seg);
  if (spi > k) spi = k;
  if (spi > p->cw) spi = p->cw;
  const int tiles_d = L.hidden / kDlFeat;
  p->max_tiles = (tiles_d + G - 1) / G;
  const size_t fixed = round128((2 * kDlMaxStages + 3) * 8) + round128(L.hidden * 2) +
                       round128(L.hidden * 4) + round128(nch_h * 4) +
                       round128(static_cast<size_t>(k) * L.inter * 2) +
                       round128(static_cast<size_t>(k) * L.inter * 4) +
                       round128(static_cast<size_t>(k) * nch_i * 4) +
                       round128(static_cast<size_t>(p->max_tiles) * k * kDlFeat * 4);
  if (fixed >= kDlSmemLimit) return false;
  size_t nst = (kDlSmemLimit - fixed) / stage;
  if (nst > static_cast<size_t>(kDlMaxStages)) nst = kDlMaxStages;
  if (nst < 2 || nst * stage < static_cast<size_t>(kDlRouterPerCta) * L.hidden * 2) return false;
  p->stage_bytes = static_cast<int>(stage);
  p->nstages = static_cast<int>(nst);
  p->seg_per_item = spi;
  p->smem = fixed + nst * stage;
  return true;
}

template <int BITS, int SDT, int NCH, int CW>
int dl_launch(const DecodeLayerArgs& args, size_t smem, int G, cudaStream_t s) {
  auto kern = decode_layer_kernel<BITS, SDT, NCH, CW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "decode_layer: cannot reserve %zu bytes of smem", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3((CW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TimedLaunch tl(BIGRIG_K_DECODE_LAYER, s);
  cudaLaunchKernelEx(&cfg, kern, args);
  return check_launch("decode_layer_kernel");
}

template <int BITS, int SDT>
int dl_shape(const DecodeLayerArgs& args, const DlPlan& p, int G, cudaStream_t s) {
  if (p.nch == 2) return dl_launch<BITS, SDT, 2, 16>(args, p.smem, G, s);
  return dl_launch<BITS, SDT, 4, 8>(args, p.smem, G, s);
}

}  // namespace

bool decode_layer_fits(const bigrig_expert_layout& L, int k, int E) {
  DlPlan p;
  return decode_layer_plan(L, k, E, sm_count_dl(), &p);
}

int launch_decode_layer(const void* x, const void* gate_w, const float* gate_b, int E, int k,
                        int mode, int norm, const int32_t* g2s, const void* slab,
                        const bigrig_expert_layout& L, const void* residual, void* out,
                        int32_t* idx_out, float* sc_out, void* h, void* tagged, uint32_t* sync,
                        int32_t* err, cudaStream_t s) {
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
  a.h = static_cast<uint16_t*>(h);
  a.tagged = static_cast<unsigned long long*>(tagged);
  a.sync = sync;
  a.err = err;
  a.E = E;
  a.k = k;
  a.mode = mode;
  a.norm = norm;
  a.stage_bytes = p.stage_bytes;
  a.nstages = p.nstages;
  a.seg_per_item = p.seg_per_item;
  a.max_tiles = p.max_tiles;
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16) return dl_shape<4, BIGRIG_F16>(a, p, G, s);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16) return dl_shape<4, BIGRIG_BF16>(a, p, G, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16) return dl_shape<8, BIGRIG_F16>(a, p, G, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16) return dl_shape<8, BIGRIG_BF16>(a, p, G, s);
  return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_layer: bits=%d scale_dtype=%d", L.bits, L.scale_dtype);
}

}  // namespace bigrig
