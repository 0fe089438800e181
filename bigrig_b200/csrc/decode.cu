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
    RouteOut ro) {
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
    s_idx[lane] = lane < P ? idx_out[lane] : 0;
    __syncwarp();
    permute_warp(s_idx, P, E, ro.order, ro.inv, ro.offsets, ro.seg_expert, ro.seg_start,
                 ro.num_seg, ro.err);
  }
}

// ------------------------------------------------------------------ down + combine
constexpr int kDcWarps = 4;
constexpr int kDcFeatures = 8;     // hidden features per CTA
constexpr int kDcBatch = 4;        // (expert, feature) items a warp keeps in flight

template <int BITS, int SDT, int ROWS>
__global__ void __launch_bounds__(kDcWarps * 32) down_combine_kernel(
    const uint16_t* __restrict__ h, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, const float* __restrict__ scores, const uint16_t* __restrict__ residual,
    uint16_t* __restrict__ out, uint16_t* __restrict__ y_out, int T) {
  extern __shared__ __align__(16) float smem[];
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  pdl_wait();
  pdl_trigger();
  const int H = L.hidden, I = L.inter;
  const int P = rv.P;
  const int nseg = *rv.num_seg;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * kDcFeatures;
  const int nchunk = I / CPL;
  // every routed pair's h row, pre-scaled, then a [P][kDcFeatures] buffer of y values
  stage_rows<BITS>(smem, h, I, P, P, [](int rr) { return rr; });
  float* ybuf = smem + static_cast<size_t>(P) * (I + nchunk);
  for (int i = threadIdx.x; i < P * kDcFeatures; i += blockDim.x) ybuf[i] = 0.f;
  __syncthreads();
  const float4* xs = reinterpret_cast<const float4*>(smem);
  const float* cs = smem + static_cast<size_t>(P) * I;
  const int items = nseg * kDcFeatures;
  for (int it0 = warp * kDcBatch; it0 < items; it0 += kDcWarps * kDcBatch) {
    uint4 w[kDcBatch];
    float sc[kDcBatch], bi[kDcBatch];
    int row0[kDcBatch], nrow[kDcBatch], fl[kDcBatch];
    bool ok[kDcBatch];
#pragma unroll
    for (int b = 0; b < kDcBatch; ++b) {
      const int it = it0 + b;
      ok[b] = it < items;
      const int s = ok[b] ? it / kDcFeatures : 0;
      fl[b] = it - s * kDcFeatures;
      const int f = min(f0 + fl[b], H - 1);
      const int e = rv.seg_expert[s];
      int slot = rv.g2s ? rv.g2s[e] : e;
      row0[b] = rv.seg_start[s];
      nrow[b] = rv.seg_start[s + 1] - row0[b];
      if (slot < 0) { ok[b] = false; slot = 0; }
      const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
      const int64_t pitch = static_cast<int64_t>(I) * BITS / 8;
      const int gp = I / L.group_size;
      w[b] = make_uint4(0, 0, 0, 0);
      sc[b] = bi[b] = 0.f;
      if (ok[b] && lane < nchunk) {
        w[b] = ld_stream_v4(base + L.weight_off[2] + f * pitch + lane * 16);
        const int grp = (lane * CPL) / L.group_size;
        sc[b] = half_to_f32<SDT>(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + L.scales_off[2]) + static_cast<int64_t>(f) * gp + grp));
        bi[b] = half_to_f32<SDT>(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + L.biases_off[2]) + static_cast<int64_t>(f) * gp + grp));
      }
    }
#pragma unroll
    for (int b = 0; b < kDcBatch; ++b) {
      if (it0 + b >= items) break;
      for (int r0 = 0; r0 < nrow[b]; r0 += ROWS) {
        float acc[ROWS];
#pragma unroll
        for (int rr = 0; rr < ROWS; ++rr) acc[rr] = 0.f;
        // lane < nchunk holds this feature's first chunk; further chunks stream here
        for (int c = lane; c < nchunk; c += 32) {
          uint4 wc = w[b];
          float s_ = sc[b], b_ = bi[b];
          if (c != lane) {
            if (ok[b]) {
              const int f = min(f0 + fl[b], H - 1);
              const int s = (it0 + b) / kDcFeatures;
              const int e = rv.seg_expert[s];
              const int slot = rv.g2s ? rv.g2s[e] : e;
              const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
              const int64_t pitch = static_cast<int64_t>(I) * BITS / 8;
              const int gp = I / L.group_size;
              const int grp = (c * CPL) / L.group_size;
              wc = ld_stream_v4(base + L.weight_off[2] + f * pitch + c * 16);
              s_ = half_to_f32<SDT>(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + L.scales_off[2]) + static_cast<int64_t>(f) * gp + grp));
              b_ = half_to_f32<SDT>(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + L.biases_off[2]) + static_cast<int64_t>(f) * gp + grp));
            } else {
              wc = make_uint4(0, 0, 0, 0);
              s_ = b_ = 0.f;
            }
          }
#pragma unroll
          for (int rr = 0; rr < ROWS; ++rr) {
            if (r0 + rr < nrow[b]) {
              const int row = row0[b] + r0 + rr;
              const float4* xq = xs + static_cast<size_t>(row) * Q * nchunk + c;
              const float d = chunk_dot<BITS>(wc, xq, nchunk);
              acc[rr] = fmaf(s_, d, fmaf(b_, cs[row * nchunk + c], acc[rr]));
            }
          }
        }
#pragma unroll
        for (int rr = 0; rr < ROWS; ++rr) {
          if (r0 + rr < nrow[b]) {
            const float v = warp_sum(acc[rr]);
            if (lane == 0) ybuf[(row0[b] + r0 + rr) * kDcFeatures + fl[b]] = ok[b] ? bf16_round(v) : 0.f;
          }
        }
      }
    }
  }
  __syncthreads();
  // combine in rank order (the standalone combine's arithmetic), plus the residual
  const int k = rv.k;
  for (int idx = threadIdx.x; idx < T * kDcFeatures; idx += blockDim.x) {
    const int t = idx / kDcFeatures, fl = idx - t * kDcFeatures;
    const int f = f0 + fl;
    if (f >= H) continue;
    float a = 0.f;
    for (int j = 0; j < k; ++j) {
      const float yv = ybuf[rv.inv[t * k + j] * kDcFeatures + fl];
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
                 cudaStream_t s) {
  const int per = (E + 31) / 32;
  const dim3 grid(logits_in ? 1 : (E + kRouteWarps - 1) / kRouteWarps);
  TimedLaunch tl(BIGRIG_K_ROUTE, s);
#define BIGRIG_ROUTE(N)                                                                         \
  case N:                                                                                       \
    return launch_pdl(route_kernel<N>, grid, dim3(kRouteWarps * 32), 0, s, "route_kernel",      \
                      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(gate_w),    \
                      gate_b, logits_in, logits_dtype, T, H, E, k, mode, norm, logits_ws, ticket, \
                      idx_out, sc_out, ro);
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

size_t down_combine_smem(int P, const bigrig_expert_layout& L) {
  const int nchunk = L.inter / (128 / L.bits);
  return static_cast<size_t>(P) * (L.inter + nchunk) * sizeof(float) +
         static_cast<size_t>(P) * kDcFeatures * sizeof(float);
}

template <int BITS, int SDT, int ROWS>
static int dc_launch(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, const float* scores, const void* residual,
                     void* out, void* y_out, int T, cudaStream_t s) {
  const size_t smem = down_combine_smem(rv.P, L);
  auto kern = down_combine_kernel<BITS, SDT, ROWS>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "down_combine: cannot reserve %zu bytes of smem", smem);
  const dim3 grid((L.hidden + kDcFeatures - 1) / kDcFeatures);
  TimedLaunch tl(BIGRIG_K_DOWN_COMBINE, s);
  return launch_pdl(kern, grid, dim3(kDcWarps * 32), smem, s, "down_combine_kernel",
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
