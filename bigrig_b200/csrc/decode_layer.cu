// One decode token through one MoE layer in ONE persistent cooperative kernel.
//
// Replaces, for a single token, the launch chain route -> gate_up -> down+combine
// (decode.cu, gemv.cu), and with it the mlx_lm block's router, the per-expert
// quantized_matmul calls of _forward_views_one (bigrig_engine/stream.py:1278-1318) and
// the caller's weighted sum (stream.py:1523-1525).  An OLMoE decode layer moves ~28 MB,
// ~4 us of HBM time; as a chain of kernels every step also paid launches and dependent
// global round trips.  Here one CTA per SM runs the whole layer:
//
//   phase 1  router logits: CTA c owns experts 8c..8c+7, one warp each, the router rows
//            bulk-copied into shared memory as the kernel starts
//   flag     the router CTAs bump a counter; every CTA waits for all of them
//   phase 2  every CTA derives the top-k, the scores and the expert-sorted order itself
//            (the same values in every CTA), then the slab slot of each routed expert
//   phase 3  gate/up: items of (routed expert, 8 features) dealt round-robin to CTAs,
//            a CTA's items all requested at once through a ring of bulk copies; warp w
//            computes feature w of an item with x held in registers; h to global
//            -> the CTA's down-projection tiles are requested before the barrier
//   barrier  grid-wide
//   phase 4  down for the CTA's 8-feature tiles over all routed experts, then the
//            combine in rank order plus the residual
//
// Per-feature arithmetic is the chain's (same chunk order per lane, same fp32x2 dot,
// same group affine, same warp sums, same combine), so the result is bit-identical to
// it.  Every wait -- mbarriers, the router flag, the grid barrier -- is bounded; a
// timeout counts in the error words and the kernel carries on to its end.
#include "gemv_common.cuh"
#include "routing.cuh"

// Phase-boundary hook (thread 0 of each CTA); empty in the library, defined by
// instrumented builds that record per-CTA timestamps.
#ifndef DL_STAMP
#define DL_STAMP(i)
#endif

namespace bigrig {

constexpr int kDlWarps = 8;              // also the features of one gate/up item
constexpr int kDlThreads = kDlWarps * 32;
constexpr int kDlFeatDown = 8;           // hidden features of one down tile
constexpr int kDlMaxStages = 8;
constexpr uint32_t kGridSpinLimit = 1u << 22;

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
  uint16_t* h;                // [k, I] scratch, expert-sorted rows
  float* logits;              // [E] scratch
  uint32_t* sync;             // [3]: router count, barrier count, barrier generation
  int32_t* err;
  int E, k, mode, norm;
  int ring_bytes;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Wait (bounded) until *p >= target.
__device__ __forceinline__ void spin_until(const uint32_t* p, uint32_t target, int32_t* err) {
  uint32_t n = 0;
  while (ld_acquire_u32(p) < target) {
    if (++n > kGridSpinLimit) {
      atomicAdd(err + 1, 1);
      return;
    }
    __nanosleep(20);
  }
}

template <int BITS, int SDT, int NCH>
__global__ void __launch_bounds__(kDlThreads, 1) decode_layer_kernel(DecodeLayerArgs a) {
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  constexpr int NFD = kDlFeatDown;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int32_t s_idx[32], s_inv[32], s_slot[32];
  __shared__ float s_sc[32];
  const bigrig_expert_layout& L = a.L;
  const int H = L.hidden, I = L.inter, E = a.E, k = a.k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int pitch_h = H * BITS / 8, pitch_i = I * BITS / 8;
  const int gh = H / L.group_size, gi = I / L.group_size;
  const int nch_h = H / CPL, nch_i = I / CPL;
  uint32_t* router_count = a.sync;
  uint32_t* bar_count = a.sync + 1;
  uint32_t* bar_gen = a.sync + 2;

  SmemCarve sc(smem);
  uint64_t* bars = sc.take<uint64_t>((3 + kDlMaxStages) * 8);
  uint16_t* xraw = sc.take<uint16_t>(static_cast<size_t>(H) * 2);
  float* xs = sc.take<float>(static_cast<size_t>(H) * 4);
  float* xcs = sc.take<float>(static_cast<size_t>(nch_h) * 4);
  uint16_t* hraw = sc.take<uint16_t>(static_cast<size_t>(k) * I * 2);
  float* hs = sc.take<float>(static_cast<size_t>(k) * I * 4);
  float* hcs = sc.take<float>(static_cast<size_t>(k) * nch_i * 4);
  float* ybuf = sc.take<float>(static_cast<size_t>(k) * NFD * 4);
  uint8_t* ring = sc.take<uint8_t>(a.ring_bytes);
  uint16_t* wr = reinterpret_cast<uint16_t*>(ring);     // router rows, phase 1 only
  uint64_t* bar_r = bars + 0;
  uint64_t* bar_x = bars + 1;
  uint64_t* bar_h = bars + 2;
  uint64_t* stage_bar = bars + 3;
  DL_STAMP(0);

  // ---------------------------------------------------------------- phase 1: logits
  const int n_router = (E + kDlWarps - 1) / kDlWarps;
  const int n_mine = max(0, min(kDlWarps, E - cta * kDlWarps));
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3 + kDlMaxStages; ++i) bar_init(bars + i, 1);
    if (n_mine > 0) {
      bar_expect_tx(bar_r, static_cast<uint32_t>(n_mine) * H * 2);
      bulk_g2s(wr, a.gate_w + static_cast<size_t>(cta) * kDlWarps * H, n_mine * H * 2, bar_r);
    }
    bar_expect_tx(bar_x, H * 2);
    bulk_g2s(xraw, a.x, H * 2, bar_x);
  }
  __syncthreads();
  bool ok = bar_wait(bar_x, 0, a.err);
  if (!ok) bar_wait(bar_x, 0, nullptr);
  if (n_mine > 0) {
    const bool okr = bar_wait(bar_r, 0, a.err);
    if (!okr) bar_wait(bar_r, 0, nullptr);
    ok = ok && okr;
  }
  DL_STAMP(1);
  if (warp < n_mine && ok) {
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
    const int e = cta * kDlWarps + warp;
    if (lane == 0) a.logits[e] = acc + (a.gate_b ? a.gate_b[e] : 0.f);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (n_mine > 0) atomicAdd(router_count, 1u);
    spin_until(router_count, static_cast<uint32_t>(n_router), a.err);
    __threadfence();
  }
  DL_STAMP(2);
  // x re-laid as pre-scaled fp32 while thread 0 waits
  relayout_rows<BITS>(xs, xcs, xraw, H, 1);
  __syncthreads();

  // ---------------------------------------------------------------- phase 2: routing
  if (warp == 0) {
    s_slot[lane] = -1;
    auto load = [&](int e) -> float { return __ldcg(a.logits + e); };
    const int per = (E + 31) / 32;
#define BIGRIG_TK(N) if (per == N) topk_warp<N>(load, E, k, a.mode, a.norm, s_idx, s_sc);
    BIGRIG_TK(1) BIGRIG_TK(2) BIGRIG_TK(3) BIGRIG_TK(4)
    BIGRIG_TK(5) BIGRIG_TK(6) BIGRIG_TK(7) BIGRIG_TK(8)
#undef BIGRIG_TK
    __syncwarp();
    // stable expert-sorted position of rank r (one token: the k experts are distinct)
    const int e = lane < k ? s_idx[lane] : 0x7fffffff;
    int pos = 0;
    for (int j = 0; j < k; ++j) {
      const int ej = __shfl_sync(0xffffffffu, e, j);
      pos += (ej < e) || (ej == e && j < lane);
    }
    const bool valid = e >= 0 && e < E;
    const int slot = valid ? (a.g2s ? a.g2s[e] : e) : -1;
    __syncwarp();
    if (lane < k) {
      s_inv[lane] = pos;
      s_slot[pos] = slot;
      if (cta == 0) {
        a.idx_out[lane] = e;
        a.sc_out[lane] = s_sc[lane];
        if (slot < 0 && a.err) atomicAdd(a.err, 1);
      }
    }
  }
  // x in registers for all of phase 3: chunk lane + 32 i of the row
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
  __syncthreads();
  DL_STAMP(3);
  const int nseg = k;

  // ---------------------------------------------------------------- phase 3: gate/up
  const int tiles_g = I / kDlWarps;
  const int n_items = nseg * tiles_g;
  const int item_bytes = 2 * kDlWarps * pitch_h + 4 * kDlWarps * gh * 2;
  const int nb3 = min(kDlMaxStages, a.ring_bytes / item_bytes);
  uint32_t phase_bits = 0;
  auto issue_item = [&](int it, int b) {
    const int s = it / tiles_g, f0 = (it - s * tiles_g) * kDlWarps;
    const int slot = s_slot[s];
    uint8_t* dst = ring + static_cast<size_t>(b) * item_bytes;
    bar_expect_tx(stage_bar + b, slot >= 0 ? static_cast<uint32_t>(item_bytes) : 0u);
    if (slot < 0) return;
    const uint8_t* base = a.slab + static_cast<int64_t>(slot) * L.slot_stride;
    uint16_t* sb = reinterpret_cast<uint16_t*>(dst + 2 * kDlWarps * pitch_h);
    for (int m = 0; m < 2; ++m) {
      bulk_g2s(dst + m * kDlWarps * pitch_h, base + L.weight_off[m] + static_cast<int64_t>(f0) * pitch_h,
               kDlWarps * pitch_h, stage_bar + b);
      bulk_g2s(sb + (2 * m) * kDlWarps * gh, base + L.scales_off[m] + static_cast<int64_t>(f0) * gh * 2,
               kDlWarps * gh * 2, stage_bar + b);
      bulk_g2s(sb + (2 * m + 1) * kDlWarps * gh,
               base + L.biases_off[m] + static_cast<int64_t>(f0) * gh * 2, kDlWarps * gh * 2,
               stage_bar + b);
    }
  };
  const int my_items = cta < n_items ? (n_items - 1 - cta) / G + 1 : 0;
  if (threadIdx.x == 0)
    for (int j = 0; j < min(nb3, my_items); ++j) issue_item(cta + j * G, j);
  for (int j = 0; j < my_items; ++j) {
    const int b = j % nb3;
    const int it = cta + j * G;
    const int s = it / tiles_g, f0 = (it - s * tiles_g) * kDlWarps;
    const bool have = s_slot[s] >= 0;
    const uint32_t par = (phase_bits >> b) & 1u;
    const bool landed = bar_wait(stage_bar + b, par, a.err);
    if (!landed) bar_wait(stage_bar + b, par, nullptr);
    phase_bits ^= 1u << b;
    if (j == 0) DL_STAMP(4);
    const uint8_t* st = ring + static_cast<size_t>(b) * item_bytes;
    const uint16_t* sb = reinterpret_cast<const uint16_t*>(st + 2 * kDlWarps * pitch_h);
    float ag = 0.f, au = 0.f;
    if (have && landed) {
      const uint8_t* wg = st + warp * pitch_h;
      const uint8_t* wu = st + (kDlWarps + warp) * pitch_h;
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        const int c = lane + 32 * i;
        if (c < nch_h) {
          const int grp = (c * CPL) / L.group_size;
          const uint4 cg = *reinterpret_cast<const uint4*>(wg + c * 16);
          const uint4 cu = *reinterpret_cast<const uint4*>(wu + c * 16);
          const float dg = chunk_dot2<BITS>(cg, cx[i]);
          const float du = chunk_dot2<BITS>(cu, cx[i]);
          ag = fmaf(half_to_f32<SDT>(sb[(0 * kDlWarps + warp) * gh + grp]), dg,
                    fmaf(half_to_f32<SDT>(sb[(1 * kDlWarps + warp) * gh + grp]), xc[i], ag));
          au = fmaf(half_to_f32<SDT>(sb[(2 * kDlWarps + warp) * gh + grp]), du,
                    fmaf(half_to_f32<SDT>(sb[(3 * kDlWarps + warp) * gh + grp]), xc[i], au));
        }
      }
    }
    const float g = warp_sum(ag);
    const float u = warp_sum(au);
    if (lane == 0)
      a.h[static_cast<size_t>(s) * I + f0 + warp] = have && landed ? f32_to_bf16_bits(silu_f32(g) * u) : 0;
    __syncthreads();                              // stage b consumed
    if (threadIdx.x == 0 && j + nb3 < my_items) issue_item(cta + (j + nb3) * G, b);
  }

  // ---------------------------------------------------------------- down prefetch
  const int tiles_d = H / NFD;
  const int seg_bytes = NFD * pitch_i + 2 * NFD * gi * 2;
  const int tile_bytes = nseg * seg_bytes;
  const int nb4 = min(kDlMaxStages, a.ring_bytes / tile_bytes);
  int n_have = 0;
  for (int s = 0; s < nseg; ++s) n_have += s_slot[s] >= 0;
  auto issue_tile = [&](int t, int b) {
    const int f0 = t * NFD;
    uint8_t* dst = ring + static_cast<size_t>(b) * tile_bytes;
    bar_expect_tx(stage_bar + b, static_cast<uint32_t>(n_have) * seg_bytes);
    for (int s = 0; s < nseg; ++s) {
      if (s_slot[s] < 0) continue;
      const uint8_t* base = a.slab + static_cast<int64_t>(s_slot[s]) * L.slot_stride;
      uint8_t* d = dst + static_cast<size_t>(s) * seg_bytes;
      uint16_t* sb = reinterpret_cast<uint16_t*>(d + NFD * pitch_i);
      bulk_g2s(d, base + L.weight_off[2] + static_cast<int64_t>(f0) * pitch_i, NFD * pitch_i,
               stage_bar + b);
      bulk_g2s(sb, base + L.scales_off[2] + static_cast<int64_t>(f0) * gi * 2, NFD * gi * 2,
               stage_bar + b);
      bulk_g2s(sb + NFD * gi, base + L.biases_off[2] + static_cast<int64_t>(f0) * gi * 2,
               NFD * gi * 2, stage_bar + b);
    }
  };
  const int my_tiles = cta < tiles_d ? (tiles_d - 1 - cta) / G + 1 : 0;
  // every gate/up stage was waited for and consumed (the loop ends in a barrier)
  if (threadIdx.x == 0)
    for (int j = 0; j < min(nb4, my_tiles); ++j) issue_tile(cta + j * G, j);

  DL_STAMP(5);
  // ---------------------------------------------------------------- grid barrier
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t gen = ld_acquire_u32(bar_gen);
    __threadfence();
    if (atomicAdd(bar_count, 1u) == static_cast<uint32_t>(G) - 1) {
      // every CTA is past the router wait: both counters back to zero for the next call
      atomicExch(router_count, 0u);
      atomicExch(bar_count, 0u);
      __threadfence();
      atomicAdd(bar_gen, 1u);
    } else {
      uint32_t n = 0;
      while (ld_acquire_u32(bar_gen) == gen) {
        if (++n > kGridSpinLimit) {
          atomicAdd(a.err + 1, 1);
          break;
        }
        __nanosleep(20);
      }
    }
    __threadfence();
    fence_proxy_async_global();                   // h, written above, is read by bulk copy
  }
  __syncthreads();
  DL_STAMP(6);

  // ---------------------------------------------------------------- phase 4: down + combine
  if (my_tiles > 0) {
    if (threadIdx.x == 0) {
      bar_expect_tx(bar_h, static_cast<uint32_t>(nseg) * I * 2);
      bulk_g2s(hraw, a.h, nseg * I * 2, bar_h);
    }
    const bool hok = bar_wait(bar_h, 0, a.err);
    if (!hok) bar_wait(bar_h, 0, nullptr);
    relayout_rows<BITS>(hs, hcs, hraw, I, nseg);
    __syncthreads();
    DL_STAMP(7);
    const float4* h4 = reinterpret_cast<const float4*>(hs);
    // warp units: (segment, slice of the tile's features); fewer segments, finer slices
    const int fs = nseg >= kDlWarps ? 1 : (nseg * 2 >= kDlWarps ? 2 : (nseg * 4 >= kDlWarps ? 4 : 8));
    const int nfu = NFD / fs;
    for (int j = 0; j < my_tiles; ++j) {
      const int b = j % nb4;
      const int t = cta + j * G, f0 = t * NFD;
      const uint32_t par = (phase_bits >> b) & 1u;
      bool landed = bar_wait(stage_bar + b, par, a.err);
      if (!landed) bar_wait(stage_bar + b, par, nullptr);
      phase_bits ^= 1u << b;
      landed = landed && hok;
      const uint8_t* st = ring + static_cast<size_t>(b) * tile_bytes;
      for (int u = warp; u < nseg * fs; u += kDlWarps) {
        const int s = u / fs, fl0 = (u - s * fs) * nfu;
        const bool have = s_slot[s] >= 0 && landed;
        const uint8_t* wc = st + static_cast<size_t>(s) * seg_bytes;
        const uint16_t* sb = reinterpret_cast<const uint16_t*>(wc + NFD * pitch_i);
        float acc[NFD];
#pragma unroll
        for (int q = 0; q < NFD; ++q) acc[q] = 0.f;
        if (have) {
          for (int c = lane; c < nch_i; c += 32) {
            const int grp = (c * CPL) / L.group_size;
            ChunkX<BITS> ch;
            load_chunk_x<BITS>(ch, h4 + static_cast<size_t>(s) * Q * nch_i + c, nch_i);
            const float csum = hcs[s * nch_i + c];
#pragma unroll
            for (int q = 0; q < NFD; ++q) {
              if (q < nfu) {
                const int fl = fl0 + q;
                const uint4 cw = *reinterpret_cast<const uint4*>(wc + fl * pitch_i + c * 16);
                const float d = chunk_dot2<BITS>(cw, ch);
                acc[q] = fmaf(half_to_f32<SDT>(sb[fl * gi + grp]), d,
                              fmaf(half_to_f32<SDT>(sb[(NFD + fl) * gi + grp]), csum, acc[q]));
              }
            }
          }
        }
#pragma unroll
        for (int q = 0; q < NFD; ++q) {
          if (q < nfu) {
            const float v = warp_sum(acc[q]);
            if (lane == 0) ybuf[s * NFD + fl0 + q] = have ? bf16_round(v) : 0.f;
          }
        }
      }
      __syncthreads();
      // combine in rank order, plus the residual
      if (threadIdx.x < NFD) {
        const int fl = threadIdx.x, f = f0 + fl;
        float acc = 0.f;
        for (int r = 0; r < k; ++r) acc = acc + s_sc[r] * ybuf[s_inv[r] * NFD + fl];
        if (a.residual) acc = bf16_bits_to_f32(a.residual[f]) + bf16_round(acc);
        a.out[f] = f32_to_bf16_bits(acc);
      }
      __syncthreads();
      if (threadIdx.x == 0 && j + nb4 < my_tiles) issue_tile(cta + (j + nb4) * G, b);
    }
  }
  DL_STAMP(8);
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
  size_t smem;
  int ring;
};

// The persistent kernel's plan for a layer, or false when it cannot run it: more than
// 32 routed experts, a hidden row too wide to keep in registers, a layer whose fixed
// shared memory leaves no room for a two-stage ring.
bool decode_layer_plan(const bigrig_expert_layout& L, int k, int E, DlPlan* p) {
  if (k > 32 || E > kMaxExperts || L.hidden % kDlFeatDown || L.inter % kDlWarps) return false;
  const int cpl = 128 / L.bits;
  const int nch_h = L.hidden / cpl, nch_i = L.inter / cpl;
  const int nch = (nch_h + 31) / 32;
  if (nch > 4) return false;
  const size_t ph = static_cast<size_t>(L.hidden) * L.bits / 8;
  const size_t pi = static_cast<size_t>(L.inter) * L.bits / 8;
  const size_t gh = L.hidden / L.group_size, gi = L.inter / L.group_size;
  const size_t item = 2 * kDlWarps * ph + 4 * kDlWarps * gh * 2;
  const size_t tile = static_cast<size_t>(k) * (kDlFeatDown * pi + 2 * kDlFeatDown * gi * 2);
  const size_t fixed = round128((3 + kDlMaxStages) * 8) + round128(L.hidden * 2) +
                       round128(L.hidden * 4) + round128(nch_h * 4) +
                       round128(static_cast<size_t>(k) * L.inter * 2) +
                       round128(static_cast<size_t>(k) * L.inter * 4) +
                       round128(static_cast<size_t>(k) * nch_i * 4) +
                       round128(static_cast<size_t>(k) * kDlFeatDown * 4);
  if (fixed >= kDlSmemLimit) return false;
  size_t ring = (kDlSmemLimit - fixed) / 128 * 128;
  const size_t cap = kDlMaxStages * (item > tile ? item : tile);
  if (ring > cap) ring = cap;
  if (ring < 2 * item || ring < 2 * tile || ring < static_cast<size_t>(kDlWarps) * L.hidden * 2)
    return false;
  p->nch = nch <= 2 ? 2 : 4;
  p->ring = static_cast<int>(ring);
  p->smem = fixed + ring;
  return true;
}

template <int BITS, int SDT, int NCH>
int dl_launch(const DecodeLayerArgs& args, size_t smem, cudaStream_t s) {
  auto kern = decode_layer_kernel<BITS, SDT, NCH>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "decode_layer: cannot reserve %zu bytes of smem", smem);
  const int sms = sm_count_dl();
  if (sms <= 0) return set_error(BIGRIG_ERR_CUDA, "decode_layer: no device");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kDlThreads);
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
int dl_nch(const DecodeLayerArgs& args, const DlPlan& p, cudaStream_t s) {
  if (p.nch == 2) return dl_launch<BITS, SDT, 2>(args, p.smem, s);
  return dl_launch<BITS, SDT, 4>(args, p.smem, s);
}

}  // namespace

bool decode_layer_fits(const bigrig_expert_layout& L, int k, int E) {
  DlPlan p;
  return decode_layer_plan(L, k, E, &p);
}

int launch_decode_layer(const void* x, const void* gate_w, const float* gate_b, int E, int k,
                        int mode, int norm, const int32_t* g2s, const void* slab,
                        const bigrig_expert_layout& L, const void* residual, void* out,
                        int32_t* idx_out, float* sc_out, void* h, float* logits, uint32_t* sync,
                        int32_t* err, cudaStream_t s) {
  DlPlan p;
  if (!decode_layer_plan(L, k, E, &p))
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
  a.logits = logits;
  a.sync = sync;
  a.err = err;
  a.E = E;
  a.k = k;
  a.mode = mode;
  a.norm = norm;
  a.ring_bytes = p.ring;
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16) return dl_nch<4, BIGRIG_F16>(a, p, s);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16) return dl_nch<4, BIGRIG_BF16>(a, p, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16) return dl_nch<8, BIGRIG_F16>(a, p, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16) return dl_nch<8, BIGRIG_BF16>(a, p, s);
  return set_error(BIGRIG_ERR_UNSUPPORTED, "decode_layer: bits=%d scale_dtype=%d", L.bits, L.scale_dtype);
}

}  // namespace bigrig
