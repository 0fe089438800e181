// Helpers of the dequantising GEMV kernels: code-to-float conversion, the per-chunk
// dot product and the activation staging (see gemv.cu for the scheme).
#pragma once

#include "common.cuh"
#include "launch.h"

namespace bigrig {

constexpr int kGemvWarps = 4;
constexpr int kGemvRows = 4;  // token rows per pass (rows of one expert <= tokens)

template <int BITS>
__device__ __forceinline__ float prescale(int kk) {
  if constexpr (BITS == 4) return __uint_as_float((127u - 4u * static_cast<uint32_t>(kk & 3)) << 23);
  else return __uint_as_float((127u - 8u * static_cast<uint32_t>(kk & 1)) << 23);
}

// Partial dot of one 16-byte code chunk with its CPL pre-scaled activations.
template <int BITS>
__device__ __forceinline__ float chunk_dot(const uint4 w, const float4* __restrict__ xq,
                                           int qstride) {
  constexpr float M = 8388608.f;
  constexpr uint32_t E23 = 0x4B000000u;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  float a0 = 0.f, a1 = 0.f;
  if constexpr (BITS == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = ws[i], hi = ws[i] >> 16;
      const float4 xa = xq[(2 * i) * qstride];
      const float4 xb = xq[(2 * i + 1) * qstride];
      a0 = fmaf(__uint_as_float((lo & 0x000Fu) | E23) - M, xa.x, a0);
      a1 = fmaf(__uint_as_float((lo & 0x00F0u) | E23) - M, xa.y, a1);
      a0 = fmaf(__uint_as_float((lo & 0x0F00u) | E23) - M, xa.z, a0);
      a1 = fmaf(__uint_as_float((lo & 0xF000u) | E23) - M, xa.w, a1);
      a0 = fmaf(__uint_as_float((hi & 0x000Fu) | E23) - M, xb.x, a0);
      a1 = fmaf(__uint_as_float((hi & 0x00F0u) | E23) - M, xb.y, a1);
      a0 = fmaf(__uint_as_float((hi & 0x0F00u) | E23) - M, xb.z, a0);
      a1 = fmaf(__uint_as_float((hi & 0xF000u) | E23) - M, xb.w, a1);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = ws[i], hi = ws[i] >> 16;
      const float4 xa = xq[i * qstride];
      a0 = fmaf(__uint_as_float((lo & 0x00FFu) | E23) - M, xa.x, a0);
      a1 = fmaf(__uint_as_float((lo & 0xFF00u) | E23) - M, xa.y, a1);
      a0 = fmaf(__uint_as_float((hi & 0x00FFu) | E23) - M, xa.z, a0);
      a1 = fmaf(__uint_as_float((hi & 0xFF00u) | E23) - M, xa.w, a1);
    }
  }
  return a0 + a1;
}

// Stage `nr` activation rows (bf16, gathered through `row_of`) into shared memory
// as pre-scaled fp32 in a [row][CPL/4][chunk] float4 layout, so that lanes reading
// consecutive chunks hit consecutive banks; plus the plain fp32 sum of each chunk.
// Rows are read as 128-bit vectors; the lanes holding one chunk's vectors are
// adjacent, so a chunk's sum is a two- or four-lane shuffle reduction.
template <int BITS, typename RowOf>
__device__ __forceinline__ void stage_rows(float* __restrict__ smem, const uint16_t* __restrict__ src,
                                           int K, int nr, int rows_cap, RowOf row_of) {
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  constexpr int VPC = CPL / 8;             // 8-element vectors per chunk (4 or 2)
  const int nchunk = K / CPL;
  const int nvec = K / 8;
  float4* xs = reinterpret_cast<float4*>(smem);
  float* cs = smem + static_cast<size_t>(rows_cap) * K;
  const int total = nr * nvec;
  for (int base = 0; base < total; base += blockDim.x) {
    const int idx = base + threadIdx.x;
    const bool active = idx < total;
    float part = 0.f;
    int rr = 0, v = 0;
    if (active) {
      rr = idx / nvec;
      v = idx - rr * nvec;
      const uint4 raw = *reinterpret_cast<const uint4*>(src + row_of(rr) * static_cast<size_t>(K) + v * 8);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      float f[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) part += f[i];
      const int kk0 = v * 8;
      const int c = kk0 / CPL, q0 = (kk0 - c * CPL) >> 2;
      xs[(static_cast<size_t>(rr) * Q + q0) * nchunk + c] =
          make_float4(f[0] * prescale<BITS>(kk0), f[1] * prescale<BITS>(kk0 + 1),
                      f[2] * prescale<BITS>(kk0 + 2), f[3] * prescale<BITS>(kk0 + 3));
      xs[(static_cast<size_t>(rr) * Q + q0 + 1) * nchunk + c] =
          make_float4(f[4] * prescale<BITS>(kk0 + 4), f[5] * prescale<BITS>(kk0 + 5),
                      f[6] * prescale<BITS>(kk0 + 6), f[7] * prescale<BITS>(kk0 + 7));
    }
    // the VPC vectors of a chunk sit in adjacent lanes (nvec is a multiple of VPC)
#pragma unroll
    for (int o = 1; o < VPC; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (active && (v % VPC) == 0) cs[rr * nchunk + v / VPC] = part;
  }
}

struct ProjView {
  const uint8_t* codes;     // row 0 of the projection
  const uint16_t* scales;
  const uint16_t* biases;
  int64_t code_pitch;       // bytes per output row
  int group_pitch;          // half entries per output row
};

__device__ __forceinline__ ProjView proj_view(const uint8_t* base, const bigrig_expert_layout& L,
                                              int proj, int K) {
  ProjView v;
  v.codes = base + L.weight_off[proj];
  v.scales = reinterpret_cast<const uint16_t*>(base + L.scales_off[proj]);
  v.biases = reinterpret_cast<const uint16_t*>(base + L.biases_off[proj]);
  v.code_pitch = static_cast<int64_t>(K) * L.bits / 8;
  v.group_pitch = K / L.group_size;
  return v;
}

}  // namespace bigrig
