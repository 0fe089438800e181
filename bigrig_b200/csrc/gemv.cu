// Grouped dequantising GEMV for decode-sized MoE calls (a few rows per expert).
//
// Replaces the reference's per-expert mx.quantized_matmul calls of
// _forward_views_one / _forward_views (bigrig_engine/stream.py:1237-1318) with two
// kernels over the expert-sorted pairs:
//   gate_up: h[p, :] = bf16(silu(x.Wg^T) * (x.Wu^T)) for every pair p (gate/up in fp32)
//   down:    y[pair, :] = bf16(h[p, :] . Wd^T), written at the pair's unpermuted
//            (token, k) position, so no separate unpermute pass exists.
//
// Weights stream once from HBM as 128-bit non-allocating loads, 16 bytes of codes
// per lane per step, coalesced along the row.  Codes become floats without integer
// conversions: OR-ing a code field into the mantissa of 2^23 and subtracting 2^23
// yields q * 16^j (4-bit) or q * 256^j (8-bit) for the field's position j inside a
// half-word, and the activation is pre-scaled by 16^-j (or 256^-j) once in shared
// memory, so each code costs one LOP3, one FADD and one FFMA.  The group affine is
// applied once per 16-byte chunk: sum (s q + b) x = s sum(q x) + b sum(x).
#include "gemv_common.cuh"
#include "routing.cuh"

namespace bigrig {

// ------------------------------------------------------------------ gate/up
template <int BITS, int SDT, int NR, int ROWS>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_gate_up_kernel(
    const uint16_t* __restrict__ x, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, uint16_t* __restrict__ h, int rows_cap) {
  extern __shared__ __align__(16) float smem[];
  __shared__ int row_tok[kGemvRows];
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.y;
  if (s >= *rv.num_seg) return;
  const int H = L.hidden, I = L.inter;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = rv.seg_expert[s];
  const int slot = rv.g2s ? rv.g2s[e] : e;
  const int row0 = rv.seg_start[s], R = rv.seg_start[s + 1] - row0;
  const int fbase = blockIdx.x * (kGemvWarps * NR) + warp * NR;
  if (slot < 0) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(rv.err, 1);
    for (int idx = threadIdx.x; idx < R * kGemvWarps * NR; idx += blockDim.x) {
      const int rr = idx / (kGemvWarps * NR), f = blockIdx.x * (kGemvWarps * NR) + idx % (kGemvWarps * NR);
      if (f < I) h[static_cast<size_t>(row0 + rr) * I + f] = 0;
    }
    return;
  }
  const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
  const ProjView pg = proj_view(base, L, 0, H), pu = proj_view(base, L, 1, H);
  const int nchunk = H / CPL;
  const float4* xs = reinterpret_cast<const float4*>(smem);
  const float* cs = smem + static_cast<size_t>(rows_cap) * H;

  for (int r0 = 0; r0 < R; r0 += rows_cap) {
    const int nr = min(rows_cap, R - r0);
    __syncthreads();
    if (threadIdx.x < nr) row_tok[threadIdx.x] = rv.order[row0 + r0 + threadIdx.x] / rv.k;
    __syncthreads();
    stage_rows<BITS>(smem, x, H, nr, rows_cap, [&](int rr) { return row_tok[rr]; });
    __syncthreads();
    float acc[2][NR][ROWS];
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) acc[0][i][rr] = acc[1][i][rr] = 0.f;

    for (int c = lane; c < nchunk; c += 32) {
      uint4 wg[NR], wu[NR];
      float sg[NR], bg[NR], su[NR], bu[NR];
      const int grp = (c * CPL) / L.group_size;
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const int f = min(fbase + i, I - 1);
        wg[i] = ld_stream_v4(pg.codes + f * pg.code_pitch + c * 16);
        wu[i] = ld_stream_v4(pu.codes + f * pu.code_pitch + c * 16);
      }
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const int f = min(fbase + i, I - 1);
        sg[i] = half_to_f32<SDT>(ld_nc_u16(pg.scales + f * pg.group_pitch + grp));
        bg[i] = half_to_f32<SDT>(ld_nc_u16(pg.biases + f * pg.group_pitch + grp));
        su[i] = half_to_f32<SDT>(ld_nc_u16(pu.scales + f * pu.group_pitch + grp));
        bu[i] = half_to_f32<SDT>(ld_nc_u16(pu.biases + f * pu.group_pitch + grp));
      }
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          const float4* xq = xs + static_cast<size_t>(rr) * Q * nchunk + c;
          const float csum = cs[rr * nchunk + c];
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            const float dg = chunk_dot<BITS>(wg[i], xq, nchunk);
            const float du = chunk_dot<BITS>(wu[i], xq, nchunk);
            acc[0][i][rr] = fmaf(sg[i], dg, fmaf(bg[i], csum, acc[0][i][rr]));
            acc[1][i][rr] = fmaf(su[i], du, fmaf(bu[i], csum, acc[1][i][rr]));
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          const float g = warp_sum(acc[0][i][rr]);
          const float u = warp_sum(acc[1][i][rr]);
          const int f = fbase + i;
          if (lane == 0 && f < I)
            h[static_cast<size_t>(row0 + r0 + rr) * I + f] = f32_to_bf16_bits(silu_f32(g) * u);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ down
template <int BITS, int SDT, int NR, int ROWS>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_down_kernel(
    const uint16_t* __restrict__ h, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, uint16_t* __restrict__ y, int rows_cap) {
  extern __shared__ __align__(16) float smem[];
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.y;
  if (s >= *rv.num_seg) return;
  const int H = L.hidden, I = L.inter;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = rv.seg_expert[s];
  const int slot = rv.g2s ? rv.g2s[e] : e;
  const int row0 = rv.seg_start[s], R = rv.seg_start[s + 1] - row0;
  const int fbase = blockIdx.x * (kGemvWarps * NR) + warp * NR;
  if (slot < 0) {
    for (int idx = threadIdx.x; idx < R * kGemvWarps * NR; idx += blockDim.x) {
      const int rr = idx / (kGemvWarps * NR), f = blockIdx.x * (kGemvWarps * NR) + idx % (kGemvWarps * NR);
      if (f < H) y[static_cast<size_t>(rv.order[row0 + rr]) * H + f] = 0;
    }
    return;
  }
  const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
  const ProjView pd = proj_view(base, L, 2, I);
  const int nchunk = I / CPL;
  const float4* xs = reinterpret_cast<const float4*>(smem);
  const float* cs = smem + static_cast<size_t>(rows_cap) * I;

  for (int r0 = 0; r0 < R; r0 += rows_cap) {
    const int nr = min(rows_cap, R - r0);
    __syncthreads();
    stage_rows<BITS>(smem, h, I, nr, rows_cap, [&](int rr) { return row0 + r0 + rr; });
    __syncthreads();
    float acc[NR][ROWS];
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) acc[i][rr] = 0.f;

    for (int c = lane; c < nchunk; c += 32) {
      uint4 wd[NR];
      float sd[NR], bd[NR];
      const int grp = (c * CPL) / L.group_size;
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const int f = min(fbase + i, H - 1);
        wd[i] = ld_stream_v4(pd.codes + f * pd.code_pitch + c * 16);
      }
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const int f = min(fbase + i, H - 1);
        sd[i] = half_to_f32<SDT>(ld_nc_u16(pd.scales + f * pd.group_pitch + grp));
        bd[i] = half_to_f32<SDT>(ld_nc_u16(pd.biases + f * pd.group_pitch + grp));
      }
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          const float4* xq = xs + static_cast<size_t>(rr) * Q * nchunk + c;
          const float csum = cs[rr * nchunk + c];
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            const float d = chunk_dot<BITS>(wd[i], xq, nchunk);
            acc[i][rr] = fmaf(sd[i], d, fmaf(bd[i], csum, acc[i][rr]));
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        if (rr < nr) {
          const float v = warp_sum(acc[i][rr]);
          const int f = fbase + i;
          if (lane == 0 && f < H) {
            const int pair = rv.order[row0 + r0 + rr];
            y[static_cast<size_t>(pair) * H + f] = f32_to_bf16_bits(v);
          }
        }
      }
    }
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
// Rows staged per pass: at most kGemvRows, at most the largest number of rows one
// expert can receive (an expert appears once per token, so <= T), and within a
// 200 KB shared-memory budget (Mixtral's 14336-wide down projection fits 3).
static int gemv_rows_cap(int K, int bits, int max_rows) {
  const size_t per_row = static_cast<size_t>(K) * sizeof(float) + (K / (128 / bits)) * sizeof(float);
  int cap = static_cast<int>((200u * 1024u) / per_row);
  cap = cap < kGemvRows ? cap : kGemvRows;
  cap = cap < max_rows ? cap : max_rows;
  return cap < 1 ? 1 : cap;
}

static size_t gemv_smem(int K, int bits, int rows_cap) {
  return static_cast<size_t>(rows_cap) * (static_cast<size_t>(K) + K / (128 / bits)) * sizeof(float);
}

template <typename Kern>
static int prepare(Kern kern, size_t smem) {
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return set_error(BIGRIG_ERR_CUDA, "cudaFuncSetAttribute(smem=%zu) failed", smem);
  }
  return 0;
}

template <int BITS, int SDT, int ROWS>
static int gate_up_rows(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, int cap, cudaStream_t s) {
  constexpr int NR = 4;
  const size_t smem = gemv_smem(L.hidden, BITS, cap);
  auto kern = gemv_gate_up_kernel<BITS, SDT, NR, ROWS>;
  if (int rc = prepare(kern, smem)) return rc;
  const dim3 grid((L.inter + kGemvWarps * NR - 1) / (kGemvWarps * NR), rv.s_max);
  TimedLaunch tl(BIGRIG_K_GATE_UP, s);
  kern<<<grid, kGemvWarps * 32, smem, s>>>(static_cast<const uint16_t*>(x), rv,
                                           static_cast<const uint8_t*>(slab), L,
                                           static_cast<uint16_t*>(h), cap);
  return check_launch("gemv_gate_up_kernel");
}

template <int BITS, int SDT, int ROWS>
static int down_rows(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, int cap, cudaStream_t s) {
  constexpr int NR = 8;
  const size_t smem = gemv_smem(L.inter, BITS, cap);
  auto kern = gemv_down_kernel<BITS, SDT, NR, ROWS>;
  if (int rc = prepare(kern, smem)) return rc;
  const dim3 grid((L.hidden + kGemvWarps * NR - 1) / (kGemvWarps * NR), rv.s_max);
  TimedLaunch tl(BIGRIG_K_DOWN, s);
  kern<<<grid, kGemvWarps * 32, smem, s>>>(static_cast<const uint16_t*>(h), rv,
                                           static_cast<const uint8_t*>(slab), L,
                                           static_cast<uint16_t*>(y), cap);
  return check_launch("gemv_down_kernel");
}

// Accumulator rows are a template parameter (1, 2 or 4) so a one-token decode keeps
// its register footprint, and with it the occupancy that hides HBM latency.
template <int BITS, int SDT>
static int gate_up_impl(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, cudaStream_t s) {
  const int cap = gemv_rows_cap(L.hidden, BITS, rv.max_rows);
  if (cap == 1) return gate_up_rows<BITS, SDT, 1>(x, rv, slab, L, h, 1, s);
  if (cap == 2) return gate_up_rows<BITS, SDT, 2>(x, rv, slab, L, h, 2, s);
  return gate_up_rows<BITS, SDT, 4>(x, rv, slab, L, h, cap, s);
}

template <int BITS, int SDT>
static int down_impl(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, cudaStream_t s) {
  const int cap = gemv_rows_cap(L.inter, BITS, rv.max_rows);
  if (cap == 1) return down_rows<BITS, SDT, 1>(h, rv, slab, L, y, 1, s);
  if (cap == 2) return down_rows<BITS, SDT, 2>(h, rv, slab, L, y, 2, s);
  return down_rows<BITS, SDT, 4>(h, rv, slab, L, y, cap, s);
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
