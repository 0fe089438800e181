// Building blocks of the dequantising GEMV kernels (gemv.cu, decode.cu).
//
// Scheme.  A CTA owns a few output features of one expert (or of every routed expert,
// for the fused down+combine).  One thread moves the CTA's weight rows -- codes, scales,
// biases -- and the routed activation rows from global memory into shared memory with
// bulk asynchronous copies completed on an mbarrier, so every byte a CTA needs is in
// flight at once; the activation rows are then re-laid as pre-scaled fp32.  Each warp
// computes its features from shared memory, a lane owning one 16-byte code chunk
// (32 four-bit or 16 eight-bit codes) per step.  Codes become floats without integer
// conversions: a code field OR-ed into the mantissa of 2^23, minus 2^23, is q * 16^j
// (4-bit) or q * 256^j (8-bit) for the field's position j in its half-word, and the
// activation is pre-scaled by 16^-j (or 256^-j) once.  Pairs of codes go through
// Blackwell's packed fp32x2 subtract and fused multiply-add.  The group affine is
// applied once per chunk: sum (s q + b) x = s sum(q x) + b sum(x).
#pragma once

#include "common.cuh"
#include "launch.h"

namespace bigrig {

constexpr int kGemvWarps = 4;
constexpr int kGemvRows = 4;  // activation rows per pass (rows of one expert <= tokens)

template <int BITS>
__device__ __forceinline__ float prescale(int kk) {
  if constexpr (BITS == 4) return __uint_as_float((127u - 4u * static_cast<uint32_t>(kk & 3)) << 23);
  else return __uint_as_float((127u - 8u * static_cast<uint32_t>(kk & 1)) << 23);
}

// The CPL pre-scaled activations of one chunk, as float2 pairs in code order.
template <int BITS>
struct ChunkX {
  float2 v[128 / BITS / 2];
};

template <int BITS>
__device__ __forceinline__ void load_chunk_x(ChunkX<BITS>& cx, const float4* __restrict__ xq,
                                             int qstride) {
  constexpr int Q = 128 / BITS / 4;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 f = xq[q * qstride];
    cx.v[2 * q] = make_float2(f.x, f.y);
    cx.v[2 * q + 1] = make_float2(f.z, f.w);
  }
}

// sum over the chunk of q_j * x_j (pre-scaled activations), packed fp32x2 arithmetic.
template <int BITS>
__device__ __forceinline__ float chunk_dot2(const uint4 w, const ChunkX<BITS>& cx) {
  const float2 NM2 = make_float2(-8388608.f, -8388608.f);
  constexpr uint32_t E23 = 0x4B000000u;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
  if constexpr (BITS == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = ws[i], hi = ws[i] >> 16;
      const float2 q01 = __fadd2_rn(make_float2(__uint_as_float((lo & 0x000Fu) | E23),
                                                __uint_as_float((lo & 0x00F0u) | E23)), NM2);
      const float2 q23 = __fadd2_rn(make_float2(__uint_as_float((lo & 0x0F00u) | E23),
                                                __uint_as_float((lo & 0xF000u) | E23)), NM2);
      const float2 q45 = __fadd2_rn(make_float2(__uint_as_float((hi & 0x000Fu) | E23),
                                                __uint_as_float((hi & 0x00F0u) | E23)), NM2);
      const float2 q67 = __fadd2_rn(make_float2(__uint_as_float((hi & 0x0F00u) | E23),
                                                __uint_as_float((hi & 0xF000u) | E23)), NM2);
      a = __ffma2_rn(q01, cx.v[4 * i + 0], a);
      b = __ffma2_rn(q23, cx.v[4 * i + 1], b);
      a = __ffma2_rn(q45, cx.v[4 * i + 2], a);
      b = __ffma2_rn(q67, cx.v[4 * i + 3], b);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = ws[i], hi = ws[i] >> 16;
      const float2 q01 = __fadd2_rn(make_float2(__uint_as_float((lo & 0x00FFu) | E23),
                                                __uint_as_float((lo & 0xFF00u) | E23)), NM2);
      const float2 q23 = __fadd2_rn(make_float2(__uint_as_float((hi & 0x00FFu) | E23),
                                                __uint_as_float((hi & 0xFF00u) | E23)), NM2);
      a = __ffma2_rn(q01, cx.v[2 * i + 0], a);
      b = __ffma2_rn(q23, cx.v[2 * i + 1], b);
    }
  }
  return (a.x + a.y) + (b.x + b.y);
}

// Re-lay `nr` bf16 rows (row r at src + r * K, in shared memory) as pre-scaled fp32 in a
// [row][CPL/4][chunk] float4 layout -- lanes reading consecutive chunks hit consecutive
// banks -- plus the fp32 sum of every chunk at cs[row * nchunk + chunk].
// Threads tid < nthreads (whole warps) take part.
template <int BITS>
__device__ __forceinline__ void relayout_rows(float* __restrict__ xs, float* __restrict__ cs,
                                              const uint16_t* __restrict__ src, int K, int nr,
                                              int tid, int nthreads) {
  constexpr int CPL = 128 / BITS;
  constexpr int Q = CPL / 4;
  constexpr int VPC = CPL / 8;             // 8-element vectors per chunk (4 or 2)
  const int nchunk = K / CPL;
  const int nvec = K / 8;
  float4* x4 = reinterpret_cast<float4*>(xs);
  const int total = nr * nvec;
  for (int base = 0; base < total; base += nthreads) {
    const int idx = base + tid;
    const bool active = idx < total;
    float part = 0.f;
    int rr = 0, v = 0;
    if (active) {
      rr = idx / nvec;
      v = idx - rr * nvec;
      const uint4 raw = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(rr) * K + v * 8);
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
      x4[(static_cast<size_t>(rr) * Q + q0) * nchunk + c] =
          make_float4(f[0] * prescale<BITS>(kk0), f[1] * prescale<BITS>(kk0 + 1),
                      f[2] * prescale<BITS>(kk0 + 2), f[3] * prescale<BITS>(kk0 + 3));
      x4[(static_cast<size_t>(rr) * Q + q0 + 1) * nchunk + c] =
          make_float4(f[4] * prescale<BITS>(kk0 + 4), f[5] * prescale<BITS>(kk0 + 5),
                      f[6] * prescale<BITS>(kk0 + 6), f[7] * prescale<BITS>(kk0 + 7));
    }
    // the VPC vectors of a chunk sit in adjacent lanes (nvec is a multiple of VPC)
#pragma unroll
    for (int o = 1; o < VPC; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (active && (v % VPC) == 0) cs[rr * nchunk + v / VPC] = part;
  }
}

template <int BITS>
__device__ __forceinline__ void relayout_rows(float* __restrict__ xs, float* __restrict__ cs,
                                              const uint16_t* __restrict__ src, int K, int nr) {
  relayout_rows<BITS>(xs, cs, src, K, nr, threadIdx.x, blockDim.x);
}

// Validate one segment's routing metadata; the slot to read, or -1 (R = 0 when the
// metadata itself is inconsistent, so nothing is written for it).
__device__ __forceinline__ int segment_slot(const RouteView& rv, int s, int& row0, int& R) {
  const int e = rv.seg_expert[s];
  row0 = rv.seg_start[s];
  R = rv.seg_start[s + 1] - row0;
  const bool ok = e >= 0 && e < rv.n_experts && row0 >= 0 && R > 0 && row0 + R <= rv.P;
  if (!ok) {
    R = 0;
    row0 = 0;
    return -1;
  }
  return rv.g2s ? rv.g2s[e] : e;
}

// Shared-memory carve helper: 128-byte aligned bump allocation.
struct SmemCarve {
  uint8_t* p;
  __device__ explicit SmemCarve(uint8_t* base) : p(base) {}
  template <typename T>
  __device__ T* take(size_t bytes) {
    T* r = reinterpret_cast<T*>(p);
    p += (bytes + 127) / 128 * 128;
    return r;
  }
};

__host__ __device__ inline size_t round128(size_t n) { return (n + 127) / 128 * 128; }

}  // namespace bigrig
