// Fused decode-step MoE layer: three launches chained by programmatic dependent
// launch instead of seven.
//
//   route_kernel        router logits x . W^T (+ bias) spread over ceil(E/8) CTAs; the
//                       last CTA to finish (a ticket counter, no waiting) runs the
//                       warp-shuffle top-k of every token and the stable permutation
//   gemv_gate_up_kernel (gemv.cu) h = bf16(silu(x.Wg^T) * (x.Wu^T)) per routed pair
//   down_combine_kernel each CTA owns a slice of the hidden features for ALL routed
//                       experts: the down projection of every pair, then
//                       out[t] = residual[t] + sum_j score[t, j] * bf16(y[t, j]) in rank
//                       order, exactly the standalone combine's arithmetic
//
// Replaces, for decode-sized calls (T * k <= 32), the mlx_lm block's gate / softmax /
// argpartition, the host routing readback of a sync-free layer and the per-expert
// quantized_matmul sequence of _forward_views_one (bigrig_engine/stream.py:1278-1318),
// plus the caller's weighted sum (stream.py:1523-1525).
#include "gemv_common.cuh"
#include "routing.cuh"

namespace bigrig {

constexpr int kRouteWarps = 8;

template <int PER_LANE>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ gate_w,
    const float* __restrict__ gate_b, const void* __restrict__ logits_in, int logits_dtype, int T,
    int H, int E, int k, int mode, int norm_topk, float* __restrict__ logits_ws,
    int32_t* __restrict__ ticket, int32_t* __restrict__ idx_out, float* __restrict__ sc_out,
    RouteOut ro, int local_first, int local_n, int32_t* __restrict__ idx_local) {
  __shared__ int s_last;
  __shared__ int32_t s_idx[32];
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (logits_in == nullptr) {
    const int e = blockIdx.x * kRouteWarps + warp;
    if (e < E) {
      const uint16_t* wr = gate_w + static_cast<size_t>(e) * H;
      for (int t = 0; t < T; ++t) {
        const uint16_t* xr = x + static_cast<size_t>(t) * H;
        float acc = 0.f;
        for (int c = lane * 8; c < H; c += 32 * 8) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
          const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
          const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
          const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc = fmaf(__uint_as_float(xs[i] << 16), __uint_as_float(ws[i] << 16), acc);
            acc = fmaf(__uint_as_float(xs[i] & 0xffff0000u), __uint_as_float(ws[i] & 0xffff0000u), acc);
          }
        }
        acc = warp_sum(acc);
        if (lane == 0) logits_ws[static_cast<size_t>(t) * E + e] = acc + (gate_b ? gate_b[e] : 0.f);
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) *ticket = 0;              // ready for the next call
  }
  pdl_trigger();
  // top-k of every token, one warp per token
  for (int t = warp; t < T; t += kRouteWarps) {
    const size_t row = static_cast<size_t>(t) * E;
    auto load = [&](int e) -> float {
      if (logits_in == nullptr) return __ldcg(logits_ws + row + e);
      return logits_dtype == BIGRIG_F32 ? static_cast<const float*>(logits_in)[row + e]
                                        : bf16_bits_to_f32(static_cast<const uint16_t*>(logits_in)[row + e]);
    };
    topk_warp<PER_LANE>(load, E, k, mode, norm_topk, idx_out + static_cast<size_t>(t) * k,
                        sc_out + static_cast<size_t>(t) * k);
  }
  __threadfence_block();
  __syncthreads();
  if (warp == 0) {
    const int P = T * k;
    int e = lane < P ? idx_out[lane] : 0;
    if (local_n > 0) {
      // expert parallelism: the pairs of this rank's experts in its own numbering, the
      // others padding (-1), which the permutation leaves out of the segments
      e = (e >= local_first && e < local_first + local_n) ? e - local_first : -1;
      if (lane < P) idx_local[lane] = e;
    }
    s_idx[lane] = e;
    __syncwarp();
    permute_warp(s_idx, P, local_n > 0 ? local_n : E, ro.order, ro.inv, ro.offsets, ro.seg_expert,
                 ro.seg_start, ro.num_seg, ro.err);
  }
}

// ------------------------------------------------------------------ down + combine
constexpr int kDcMaxSeg = 32;      // decode calls: at most 32 pairs, so at most 32 experts

size_t down_combine_smem(int P, const bigrig_expert_layout& L, int nf) {
  const size_t pitch = static_cast<size_t>(L.inter) * L.bits / 8;
  const size_t G = L.inter / L.group_size;
  const size_t nchunk = L.inter / (128 / L.bits);
  const size_t S = P < kDcMaxSeg ? P : kDcMaxSeg;
  return 128 + round128(S * nf * pitch) + round128(S * 2 * nf * G * 2) +
         round128(static_cast<size_t>(P) * L.inter * 2) +
         round128(static_cast<size_t>(P) * L.inter * 4) + round128(P * nchunk * 4) +
         round128(static_cast<size_t>(P) * nf * 4);
}

size_t down_combine_smem(int P, const bigrig_expert_layout& L) { return down_combine_smem(P, L, 8); }

// Each CTA owns NF hidden features for every routed expert of the call: the experts'
// down-projection rows for those features and every pair's h row arrive by bulk copy,
// each warp computes NR features for all pairs, and the CTA combines its features.
template <int BITS, int SDT, int NR, int ROWS>
__global__ void __launch_bounds__(kGemvWarps * 32) down_combine_kernel(
    const uint16_t* __restrict__ h, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, const float* __restrict__ scores, const uint16_t* __restrict__ residual,
    uint16_t* __restrict__ out, uint16_t* __restrict__ y_out, int T) {
  constexpr int NF = kGemvWarps * NR;
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int seg_slot[kDcMaxSeg];
  __shared__ int seg_row0[kDcMaxSeg + 1];
  __shared__ int s_nvalid, abort_flag;
  pdl_wait();
  pdl_trigger();
  const int H = L.hidden, I = L.inter;
  const int P = rv.P;
  const int nseg = min(min(*rv.num_seg, rv.s_max), kDcMaxSeg);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * NF;
  const int64_t pitch = static_cast<int64_t>(I) * BITS / 8;
  const int G = I / L.group_size;
  const int nchunk = I / CPL;
  const int S = P < kDcMaxSeg ? P : kDcMaxSeg;
  SmemCarve sc(smem);
  uint64_t* bar = sc.take<uint64_t>(8);
  uint8_t* wc = sc.take<uint8_t>(static_cast<size_t>(S) * NF * pitch);
  uint16_t* wsb = sc.take<uint16_t>(static_cast<size_t>(S) * 2 * NF * G * 2);
  uint16_t* hraw = sc.take<uint16_t>(static_cast<size_t>(P) * I * 2);
  float* hs = sc.take<float>(static_cast<size_t>(P) * I * 4);
  float* cs = sc.take<float>(static_cast<size_t>(P) * nchunk * 4);
  float* ybuf = sc.take<float>(static_cast<size_t>(P) * NF * 4);
  const float4* h4 = reinterpret_cast<const float4*>(hs);
  if (threadIdx.x == 0) {
    bar_init(bar, 1);
    abort_flag = 0;
    // validate every segment and issue all copies of the CTA at once
    uint32_t bytes = 0;
    int nvalid = 0;
    for (int s = 0; s < nseg; ++s) {
      int row0, R;
      const int slot = segment_slot(rv, s, row0, R);
      seg_slot[s] = slot;
      seg_row0[s] = row0;
      seg_row0[s + 1] = row0 + R;
      if (R > 0) nvalid = row0 + R;
      if (slot >= 0) bytes += static_cast<uint32_t>(NF * pitch + 2 * NF * G * 2);
      else if (R > 0) atomicAdd(rv.err, 1);
    }
    s_nvalid = nvalid;
    bytes += static_cast<uint32_t>(nvalid) * I * 2;
    bar_expect_tx(bar, bytes);
    for (int s = 0; s < nseg; ++s) {
      if (seg_slot[s] < 0) continue;
      const uint8_t* base = slab + static_cast<int64_t>(seg_slot[s]) * L.slot_stride;
      bulk_g2s(wc + static_cast<size_t>(s) * NF * pitch, base + L.weight_off[2] + f0 * pitch,
               NF * pitch, bar);
      bulk_g2s(wsb + static_cast<size_t>(s) * 2 * NF * G,
               base + L.scales_off[2] + static_cast<int64_t>(f0) * G * 2, NF * G * 2, bar);
      bulk_g2s(wsb + (static_cast<size_t>(s) * 2 + 1) * NF * G,
               base + L.biases_off[2] + static_cast<int64_t>(f0) * G * 2, NF * G * 2, bar);
    }
    if (nvalid > 0) bulk_g2s(hraw, h, nvalid * I * 2, bar);
  }
  for (int i = threadIdx.x; i < P * NF; i += blockDim.x) ybuf[i] = 0.f;
  __syncthreads();
  if (!bar_wait(bar, 0, rv.err)) {
    abort_flag = 1;
    bar_wait(bar, 0, nullptr);         // let this CTA's own copies land before it exits
  }
  __syncthreads();
  if (!abort_flag) {
    relayout_rows<BITS>(hs, cs, hraw, I, s_nvalid);
    __syncthreads();
    for (int s = 0; s < nseg; ++s) {
      if (seg_slot[s] < 0) continue;
      const uint8_t* ws = wc + static_cast<size_t>(s) * NF * pitch;
      const uint16_t* sbs = wsb + static_cast<size_t>(s) * 2 * NF * G;
      const int ra = seg_row0[s], rb = seg_row0[s + 1];
      for (int r0 = ra; r0 < rb; r0 += ROWS) {
        float acc[NR][ROWS];
#pragma unroll
        for (int i = 0; i < NR; ++i)
#pragma unroll
          for (int rr = 0; rr < ROWS; ++rr) acc[i][rr] = 0.f;
        for (int c = lane; c < nchunk; c += 32) {
          const int grp = (c * CPL) / L.group_size;
          uint4 cw[NR];
          float sw[NR], bw[NR];
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            const int fl = warp * NR + i;
            cw[i] = *reinterpret_cast<const uint4*>(ws + fl * pitch + c * 16);
            sw[i] = half_to_f32<SDT>(sbs[fl * G + grp]);
            bw[i] = half_to_f32<SDT>(sbs[(NF + fl) * G + grp]);
          }
#pragma unroll
          for (int rr = 0; rr < ROWS; ++rr) {
            if (r0 + rr < rb) {
              ChunkX<BITS> cx;
              load_chunk_x<BITS>(cx, h4 + static_cast<size_t>(r0 + rr) * Q * nchunk + c, nchunk);
              const float csum = cs[(r0 + rr) * nchunk + c];
#pragma unroll
              for (int i = 0; i < NR; ++i) {
                const float d = chunk_dot2<BITS>(cw[i], cx);
                acc[i][rr] = fmaf(sw[i], d, fmaf(bw[i], csum, acc[i][rr]));
              }
            }
          }
        }
        const uint8_t* sbase = slab + static_cast<int64_t>(seg_slot[s]) * L.slot_stride;
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          const float bd = proj_bias(sbase, L, 2, f0 + warp * NR + i);
#pragma unroll
          for (int rr = 0; rr < ROWS; ++rr) {
            if (r0 + rr < rb) {
              const float v = warp_sum(acc[i][rr]) + bd;
              if (lane == 0) ybuf[(r0 + rr) * NF + warp * NR + i] = bf16_round(v);
            }
          }
        }
      }
    }
  }
  __syncthreads();
  // combine in rank order (the standalone combine's arithmetic), plus the residual
  const int k = rv.k;
  for (int idx = threadIdx.x; idx < T * NF; idx += blockDim.x) {
    const int t = idx / NF, fl = idx - t * NF;
    const int f = f0 + fl;
    float a = 0.f;
    for (int j = 0; j < k; ++j) {
      const int pos = rv.inv[t * k + j];
      const float yv = (pos >= 0 && pos < P) ? ybuf[pos * NF + fl] : 0.f;
      a = a + scores[t * k + j] * yv;
      if (y_out) y_out[(static_cast<size_t>(t) * k + j) * H + f] = f32_to_bf16_bits(yv);
    }
    if (residual) a = bf16_bits_to_f32(residual[static_cast<size_t>(t) * H + f]) + bf16_round(a);
    out[static_cast<size_t>(t) * H + f] = f32_to_bf16_bits(a);
  }
}

// ------------------------------------------------------------------ launchers
template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      const char* name, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) != cudaSuccess)
    return check_launch(name);
  return check_launch(name);
}

int launch_route(const void* x, const void* gate_w, const float* gate_b, const void* logits_in,
                 int logits_dtype, int T, int H, int E, int k, int mode, int norm, float* logits_ws,
                 int32_t* ticket, int32_t* idx_out, float* sc_out, const RouteOut& ro,
                 cudaStream_t s, int local_first, int local_n, int32_t* idx_local) {
  const int per = (E + 31) / 32;
  const dim3 grid(logits_in ? 1 : (E + kRouteWarps - 1) / kRouteWarps);
  TimedLaunch tl(BIGRIG_K_ROUTE, s);
#define BIGRIG_ROUTE(N)                                                                         \
  case N:                                                                                       \
    return launch_pdl(route_kernel<N>, grid, dim3(kRouteWarps * 32), 0, s, "route_kernel",      \
                      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(gate_w),    \
                      gate_b, logits_in, logits_dtype, T, H, E, k, mode, norm, logits_ws, ticket, \
                      idx_out, sc_out, ro, local_first, local_n, idx_local);
  switch (per) {
    BIGRIG_ROUTE(1)
    BIGRIG_ROUTE(2)
    BIGRIG_ROUTE(3)
    BIGRIG_ROUTE(4)
    BIGRIG_ROUTE(5)
    BIGRIG_ROUTE(6)
    BIGRIG_ROUTE(7)
    BIGRIG_ROUTE(8)
  }
#undef BIGRIG_ROUTE
  return set_error(BIGRIG_ERR_UNSUPPORTED, "route: n_experts must be <= 256");
}

template <int BITS, int SDT, int ROWS>
static int dc_launch(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, const float* scores, const void* residual,
                     void* out, void* y_out, int T, cudaStream_t s) {
  constexpr int NR = 2;          // 8 features per CTA: 256 CTAs for a 2048-wide hidden
  const size_t smem = down_combine_smem(rv.P, L, kGemvWarps * NR);
  auto kern = down_combine_kernel<BITS, SDT, NR, ROWS>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "down_combine: cannot reserve %zu bytes of smem", smem);
  const dim3 grid(L.hidden / (kGemvWarps * NR));
  TimedLaunch tl(BIGRIG_K_DOWN_COMBINE, s);
  return launch_pdl(kern, grid, dim3(kGemvWarps * 32), smem, s, "down_combine_kernel",
                    static_cast<const uint16_t*>(h), rv, static_cast<const uint8_t*>(slab), L,
                    scores, static_cast<const uint16_t*>(residual), static_cast<uint16_t*>(out),
                    static_cast<uint16_t*>(y_out), T);
}

template <int BITS, int SDT>
static int dc_rows(const void* h, const RouteView& rv, const void* slab,
                   const bigrig_expert_layout& L, const float* scores, const void* residual,
                   void* out, void* y_out, int T, cudaStream_t s) {
  if (rv.max_rows <= 1) return dc_launch<BITS, SDT, 1>(h, rv, slab, L, scores, residual, out, y_out, T, s);
  return dc_launch<BITS, SDT, 4>(h, rv, slab, L, scores, residual, out, y_out, T, s);
}

int launch_down_combine(const void* h, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, const float* scores, const void* residual,
                        void* out, void* y_out, int T, cudaStream_t s) {
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16) return dc_rows<4, BIGRIG_F16>(h, rv, slab, L, scores, residual, out, y_out, T, s);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16) return dc_rows<4, BIGRIG_BF16>(h, rv, slab, L, scores, residual, out, y_out, T, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16) return dc_rows<8, BIGRIG_F16>(h, rv, slab, L, scores, residual, out, y_out, T, s);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16) return dc_rows<8, BIGRIG_BF16>(h, rv, slab, L, scores, residual, out, y_out, T, s);
  return set_error(BIGRIG_ERR_UNSUPPORTED, "down_combine: bits=%d scale_dtype=%d", L.bits, L.scale_dtype);
}

}  // namespace bigrig
