// Grouped dequantising GEMV for decode-sized MoE calls (a few rows per expert).
//
// Replaces the reference's per-expert mx.quantized_matmul calls of
// _forward_views_one / _forward_views (bigrig_engine/stream.py:1237-1318) with two
// kernels over the expert-sorted pairs:
//   gate_up: h[p, :] = bf16(silu(x.Wg^T) * (x.Wu^T)) for every pair p (gate/up in fp32)
//   down:    y[pair, :] = bf16(h[p, :] . Wd^T), written at the pair's unpermuted
//            (token, k) position, so no separate unpermute pass exists.
// A CTA owns NF output features of one expert: its weight rows arrive once by bulk
// copy and serve every pass over the expert's rows (see gemv_common.cuh).
#include "gemv_common.cuh"
#include "routing.cuh"

namespace bigrig {

// Gate/up (fc1 of a plain expert: one matrix) staging for nf features and `rows` rows.
size_t gemv_gate_up_smem(const bigrig_expert_layout& L, int nf, int rows) {
  const size_t nm = (L.flags & BIGRIG_LAYOUT_PLAIN) ? 1 : 2;
  const size_t pitch = static_cast<size_t>(L.hidden) * L.bits / 8;
  const size_t G = L.hidden / L.group_size;
  const size_t nchunk = L.hidden / (128 / L.bits);
  return 128 + round128(nm * nf * pitch) + round128(2 * nm * nf * G * 2) +
         round128(static_cast<size_t>(rows) * L.hidden * 2) +
         round128(static_cast<size_t>(rows) * L.hidden * 4) + round128(rows * nchunk * 4);
}

size_t gemv_down_smem(const bigrig_expert_layout& L, int nf, int rows) {
  const size_t pitch = static_cast<size_t>(L.inter) * L.bits / 8;
  const size_t G = L.inter / L.group_size;
  const size_t nchunk = L.inter / (128 / L.bits);
  return 128 + round128(nf * pitch) + round128(2 * nf * G * 2) +
         round128(static_cast<size_t>(rows) * L.inter * 2) +
         round128(static_cast<size_t>(rows) * L.inter * 4) + round128(rows * nchunk * 4);
}

// ------------------------------------------------------------------ gate/up
// GATED: gate and up rows, h = act(gate, up); else the plain expert's fc1, h = act(fc1).
// Projection biases (BIGRIG_LAYOUT_BIAS) are added to the fp32 outputs first.
template <int BITS, int SDT, int NR, int ROWS, bool GATED>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_gate_up_kernel(
    const uint16_t* __restrict__ x, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, uint16_t* __restrict__ h, int rows_cap) {
  constexpr int NF = kGemvWarps * NR;
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int abort_flag;
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.y;
  if (s >= min(*rv.num_seg, rv.s_max)) return;
  const int H = L.hidden, I = L.inter;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * NF;
  int row0, R;
  const int slot = segment_slot(rv, s, row0, R);
  if (slot < 0) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(rv.err, 1);
    for (int i = threadIdx.x; i < R * NF; i += blockDim.x)
      h[static_cast<size_t>(row0 + i / NF) * I + f0 + i % NF] = 0;
    return;
  }
  constexpr int NM = GATED ? 2 : 1;           // weight matrices
  const int64_t pitch = static_cast<int64_t>(H) * BITS / 8;
  const int G = H / L.group_size;
  const int nchunk = H / CPL;
  SmemCarve sc(smem);
  uint64_t* bar = sc.take<uint64_t>(8);
  uint8_t* wc = sc.take<uint8_t>(NM * NF * pitch);
  uint16_t* wsb = sc.take<uint16_t>(2 * NM * NF * G * 2);
  uint16_t* xraw = sc.take<uint16_t>(static_cast<size_t>(rows_cap) * H * 2);
  float* xs = sc.take<float>(static_cast<size_t>(rows_cap) * H * 4);
  float* cs = sc.take<float>(static_cast<size_t>(rows_cap) * nchunk * 4);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
  if (threadIdx.x == 0) {
    bar_init(bar, 1);
    abort_flag = 0;
  }
  __syncthreads();
  uint32_t phase = 0;
  for (int r0 = 0; r0 < R; r0 += rows_cap) {
    const int nr = min(rows_cap, R - r0);
    if (threadIdx.x == 0) {
      uint32_t bytes = static_cast<uint32_t>(nr) * H * 2;
      if (r0 == 0) bytes += static_cast<uint32_t>(NM * NF * pitch + 2 * NM * NF * G * 2);
      bar_expect_tx(bar, bytes);
      if (r0 == 0) {
        for (int m = 0; m < NM; ++m) {
          bulk_g2s(wc + m * NF * pitch, base + L.weight_off[m] + f0 * pitch, NF * pitch, bar);
          bulk_g2s(wsb + (2 * m) * NF * G, base + L.scales_off[m] + static_cast<int64_t>(f0) * G * 2,
                   NF * G * 2, bar);
          bulk_g2s(wsb + (2 * m + 1) * NF * G,
                   base + L.biases_off[m] + static_cast<int64_t>(f0) * G * 2, NF * G * 2, bar);
        }
      }
      for (int rr = 0; rr < nr; ++rr) {
        const int tok = rv.order[row0 + r0 + rr] / rv.k;
        bulk_g2s(xraw + static_cast<size_t>(rr) * H, x + static_cast<int64_t>(tok) * H, H * 2, bar);
      }
    }
    if (!bar_wait(bar, phase, rv.err)) {
      abort_flag = 1;
      bar_wait(bar, phase, nullptr);   // let this CTA's own copies land before it exits
    }
    phase ^= 1;
    __syncthreads();
    if (abort_flag) break;
    relayout_rows<BITS>(xs, cs, xraw, H, nr);
    __syncthreads();
    float acc[2][NR][ROWS];
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) acc[0][i][rr] = acc[1][i][rr] = 0.f;
    for (int c = lane; c < nchunk; c += 32) {
      const int grp = (c * CPL) / L.group_size;
      uint4 cg[NR], cu[NR];
      float sg[NR], bg[NR], su[NR], bu[NR];
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const int fl = warp * NR + i;
        cg[i] = *reinterpret_cast<const uint4*>(wc + fl * pitch + c * 16);
        sg[i] = half_to_f32<SDT>(wsb[(0 * NF + fl) * G + grp]);
        bg[i] = half_to_f32<SDT>(wsb[(1 * NF + fl) * G + grp]);
        if constexpr (GATED) {
          cu[i] = *reinterpret_cast<const uint4*>(wc + (NF + fl) * pitch + c * 16);
          su[i] = half_to_f32<SDT>(wsb[(2 * NF + fl) * G + grp]);
          bu[i] = half_to_f32<SDT>(wsb[(3 * NF + fl) * G + grp]);
        }
      }
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          ChunkX<BITS> cx;
          load_chunk_x<BITS>(cx, x4 + static_cast<size_t>(rr) * Q * nchunk + c, nchunk);
          const float csum = cs[rr * nchunk + c];
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            const float dg = chunk_dot2<BITS>(cg[i], cx);
            acc[0][i][rr] = fmaf(sg[i], dg, fmaf(bg[i], csum, acc[0][i][rr]));
            if constexpr (GATED) {
              const float du = chunk_dot2<BITS>(cu[i], cx);
              acc[1][i][rr] = fmaf(su[i], du, fmaf(bu[i], csum, acc[1][i][rr]));
            }
          }
        }
      }
    }
    const int act = BIGRIG_LAYOUT_ACT(L.flags);
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int f = f0 + warp * NR + i;
      const float bgate = proj_bias(base, L, 0, f);
      const float bup = GATED ? proj_bias(base, L, 1, f) : 0.f;
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          const float g = warp_sum(acc[0][i][rr]) + bgate;
          const float u = GATED ? warp_sum(acc[1][i][rr]) + bup : 0.f;
          if (lane == 0)
            h[static_cast<size_t>(row0 + r0 + rr) * I + f] =
                f32_to_bf16_bits(GATED ? act_gated(g, u, act) : act_plain(g, act));
        }
      }
    }
    __syncthreads();      // the next pass overwrites xraw / xs
  }
}

// ------------------------------------------------------------------ down
template <int BITS, int SDT, int NR, int ROWS>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_down_kernel(
    const uint16_t* __restrict__ h, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, uint16_t* __restrict__ y, int rows_cap) {
  constexpr int NF = kGemvWarps * NR;
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int abort_flag;
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.y;
  if (s >= min(*rv.num_seg, rv.s_max)) return;
  const int H = L.hidden, I = L.inter;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * NF;
  int row0, R;
  const int slot = segment_slot(rv, s, row0, R);
  if (slot < 0) {
    for (int i = threadIdx.x; i < R * NF; i += blockDim.x)
      y[static_cast<size_t>(rv.order[row0 + i / NF]) * H + f0 + i % NF] = 0;
    return;
  }
  const int64_t pitch = static_cast<int64_t>(I) * BITS / 8;
  const int G = I / L.group_size;
  const int nchunk = I / CPL;
  SmemCarve sc(smem);
  uint64_t* bar = sc.take<uint64_t>(8);
  uint8_t* wc = sc.take<uint8_t>(NF * pitch);
  uint16_t* wsb = sc.take<uint16_t>(2 * NF * G * 2);
  uint16_t* hraw = sc.take<uint16_t>(static_cast<size_t>(rows_cap) * I * 2);
  float* hs = sc.take<float>(static_cast<size_t>(rows_cap) * I * 4);
  float* cs = sc.take<float>(static_cast<size_t>(rows_cap) * nchunk * 4);
  const float4* h4 = reinterpret_cast<const float4*>(hs);
  const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
  if (threadIdx.x == 0) {
    bar_init(bar, 1);
    abort_flag = 0;
  }
  __syncthreads();
  uint32_t phase = 0;
  for (int r0 = 0; r0 < R; r0 += rows_cap) {
    const int nr = min(rows_cap, R - r0);
    if (threadIdx.x == 0) {
      uint32_t bytes = static_cast<uint32_t>(nr) * I * 2;
      if (r0 == 0) bytes += static_cast<uint32_t>(NF * pitch + 2 * NF * G * 2);
      bar_expect_tx(bar, bytes);
      if (r0 == 0) {
        bulk_g2s(wc, base + L.weight_off[2] + f0 * pitch, NF * pitch, bar);
        bulk_g2s(wsb, base + L.scales_off[2] + static_cast<int64_t>(f0) * G * 2, NF * G * 2, bar);
        bulk_g2s(wsb + NF * G, base + L.biases_off[2] + static_cast<int64_t>(f0) * G * 2,
                 NF * G * 2, bar);
      }
      bulk_g2s(hraw, h + static_cast<int64_t>(row0 + r0) * I, nr * I * 2, bar);
    }
    if (!bar_wait(bar, phase, rv.err)) {
      abort_flag = 1;
      bar_wait(bar, phase, nullptr);   // let this CTA's own copies land before it exits
    }
    phase ^= 1;
    __syncthreads();
    if (abort_flag) break;
    relayout_rows<BITS>(hs, cs, hraw, I, nr);
    __syncthreads();
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
        cw[i] = *reinterpret_cast<const uint4*>(wc + fl * pitch + c * 16);
        sw[i] = half_to_f32<SDT>(wsb[fl * G + grp]);
        bw[i] = half_to_f32<SDT>(wsb[(NF + fl) * G + grp]);
      }
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          ChunkX<BITS> cx;
          load_chunk_x<BITS>(cx, h4 + static_cast<size_t>(rr) * Q * nchunk + c, nchunk);
          const float csum = cs[rr * nchunk + c];
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            const float d = chunk_dot2<BITS>(cw[i], cx);
            acc[i][rr] = fmaf(sw[i], d, fmaf(bw[i], csum, acc[i][rr]));
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const float bd = proj_bias(base, L, 2, f0 + warp * NR + i);
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          const float v = warp_sum(acc[i][rr]) + bd;
          if (lane == 0)
            y[static_cast<size_t>(rv.order[row0 + r0 + rr]) * H + f0 + warp * NR + i] =
                f32_to_bf16_bits(v);
        }
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ combine
// out[t, f] = bf16(sum_j score[t, j] * y[t, j, f]), fp32 accumulation in j order;
// with a residual: out = bf16(residual + bf16(sum)), the decoder's h + moe(h).
__global__ void combine_kernel(const uint16_t* __restrict__ y, const float* __restrict__ scores,
                               int T, int k, int H, uint16_t* __restrict__ out,
                               const uint16_t* __restrict__ residual) {
  pdl_wait();
  const int t = blockIdx.y;
  const int f = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (t >= T || f >= H) return;
  float a0 = 0.f, a1 = 0.f;
  for (int j = 0; j < k; ++j) {
    const float sc = scores[static_cast<size_t>(t) * k + j];
    const uint32_t v = *reinterpret_cast<const uint32_t*>(y + (static_cast<size_t>(t) * k + j) * H + f);
    a0 = a0 + sc * __uint_as_float(v << 16);
    a1 = a1 + sc * __uint_as_float(v & 0xffff0000u);
  }
  if (residual) {
    const uint32_t r = *reinterpret_cast<const uint32_t*>(residual + static_cast<size_t>(t) * H + f);
    a0 = __uint_as_float(r << 16) + bf16_round(a0);
    a1 = __uint_as_float(r & 0xffff0000u) + bf16_round(a1);
  }
  const uint32_t packed = static_cast<uint32_t>(f32_to_bf16_bits(a0)) |
                          (static_cast<uint32_t>(f32_to_bf16_bits(a1)) << 16);
  *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(t) * H + f) = packed;
}

// ------------------------------------------------------------------ launchers
constexpr size_t kGemvSmemBudget = 220 * 1024;

// Features per CTA and rows per pass: the most features (16, 8, else 4) and rows (<= 4,
// <= the rows one expert can get) whose staging fits the shared-memory budget.  A tile's
// scale/bias block (features x groups x 2 bytes) must be a multiple of 16 bytes.
template <typename SmemFn>
static bool pick_tile(SmemFn fn, int max_rows, int groups, int* nf, int* rows) {
  for (int f : {16, 8, 4}) {
    if ((f * groups) % 8) continue;
    for (int r = max_rows < kGemvRows ? max_rows : kGemvRows; r >= 1; --r) {
      if (fn(f, r) <= kGemvSmemBudget) {
        *nf = f;
        *rows = r;
        return true;
      }
    }
  }
  return false;
}

template <typename Kern>
static int launch_gemv(Kern kern, dim3 grid, size_t smem, cudaStream_t s, const char* name,
                       const void* act, const RouteView& rv, const void* slab,
                       const bigrig_expert_layout& L, void* out, int rows) {
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "%s: cannot reserve %zu bytes of smem", name, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, static_cast<const uint16_t*>(act), rv,
                     static_cast<const uint8_t*>(slab), L, static_cast<uint16_t*>(out), rows);
  return check_launch(name);
}

template <int BITS, int SDT>
static int gate_up_impl(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, cudaStream_t s) {
  int nf = 0, rows = 0;
  if (!pick_tile([&](int f, int r) { return gemv_gate_up_smem(L, f, r); }, rv.max_rows,
                 L.hidden / L.group_size, &nf, &rows))
    return set_error(BIGRIG_ERR_UNSUPPORTED, "gemv gate_up: hidden=%d does not fit shared memory",
                     L.hidden);
  const size_t smem = gemv_gate_up_smem(L, nf, rows);
  const dim3 grid(L.inter / nf, rv.s_max);
  TimedLaunch tl(BIGRIG_K_GATE_UP, s);
  const char* n = "gemv_gate_up_kernel";
#define BIGRIG_GU(NR, RW)                                                                   \
  return (L.flags & BIGRIG_LAYOUT_PLAIN)                                                    \
             ? launch_gemv(gemv_gate_up_kernel<BITS, SDT, NR, RW, false>, grid, smem, s, n, x, \
                           rv, slab, L, h, rows)                                            \
             : launch_gemv(gemv_gate_up_kernel<BITS, SDT, NR, RW, true>, grid, smem, s, n, x,  \
                           rv, slab, L, h, rows)
  if (nf == 16) {
    if (rows == 1) BIGRIG_GU(4, 1);
    if (rows == 2) BIGRIG_GU(4, 2);
    BIGRIG_GU(4, 4);
  }
  if (nf == 8) {
    if (rows == 1) BIGRIG_GU(2, 1);
    if (rows == 2) BIGRIG_GU(2, 2);
    BIGRIG_GU(2, 4);
  }
  if (rows == 1) BIGRIG_GU(1, 1);
  if (rows == 2) BIGRIG_GU(1, 2);
  BIGRIG_GU(1, 4);
#undef BIGRIG_GU
}

template <int BITS, int SDT>
static int down_impl(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, cudaStream_t s) {
  int nf = 0, rows = 0;
  if (!pick_tile([&](int f, int r) { return gemv_down_smem(L, f, r); }, rv.max_rows,
                 L.inter / L.group_size, &nf, &rows))
    return set_error(BIGRIG_ERR_UNSUPPORTED, "gemv down: inter=%d does not fit shared memory",
                     L.inter);
  const size_t smem = gemv_down_smem(L, nf, rows);
  const dim3 grid(L.hidden / nf, rv.s_max);
  TimedLaunch tl(BIGRIG_K_DOWN, s);
  const char* n = "gemv_down_kernel";
#define BIGRIG_DN(NR, RW) \
  return launch_gemv(gemv_down_kernel<BITS, SDT, NR, RW>, grid, smem, s, n, h, rv, slab, L, y, rows)
  if (nf == 16) {
    if (rows == 1) BIGRIG_DN(4, 1);
    if (rows == 2) BIGRIG_DN(4, 2);
    BIGRIG_DN(4, 4);
  }
  if (nf == 8) {
    if (rows == 1) BIGRIG_DN(2, 1);
    if (rows == 2) BIGRIG_DN(2, 2);
    BIGRIG_DN(2, 4);
  }
  if (rows == 1) BIGRIG_DN(1, 1);
  if (rows == 2) BIGRIG_DN(1, 2);
  BIGRIG_DN(1, 4);
#undef BIGRIG_DN
}

#define BIGRIG_DISPATCH_FMT(FN, ...)                                                  \
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16) return FN<4, BIGRIG_F16>(__VA_ARGS__);   \
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16) return FN<4, BIGRIG_BF16>(__VA_ARGS__); \
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16) return FN<8, BIGRIG_F16>(__VA_ARGS__);   \
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16) return FN<8, BIGRIG_BF16>(__VA_ARGS__); \
  return set_error(BIGRIG_ERR_UNSUPPORTED, "bits=%d scale_dtype=%d not built", L.bits,    \
                   L.scale_dtype);

int launch_gemv_gate_up(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, cudaStream_t s) {
  BIGRIG_DISPATCH_FMT(gate_up_impl, x, rv, slab, L, h, s)
}

int launch_gemv_down(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, cudaStream_t s) {
  BIGRIG_DISPATCH_FMT(down_impl, h, rv, slab, L, y, s)
}

int launch_combine(const void* y, const float* scores, int T, int k, int H, void* out,
                   cudaStream_t s, const void* residual) {
  const int threads = 128;
  const dim3 grid((H / 2 + threads - 1) / threads, T);
  TimedLaunch tl(BIGRIG_K_COMBINE, s);
  combine_kernel<<<grid, threads, 0, s>>>(static_cast<const uint16_t*>(y), scores, T, k, H,
                                          static_cast<uint16_t*>(out),
                                          static_cast<const uint16_t*>(residual));
  return check_launch("combine_kernel");
}

}  // namespace bigrig
