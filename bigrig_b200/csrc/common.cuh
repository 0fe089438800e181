// Shared device helpers for the B200 MoE expert path (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "bigrig_b200.h"

namespace bigrig {

constexpr int kWarp = 32;
constexpr int kMaxExperts = 256;  // router / permutation kernels keep per-expert state in smem

// Round-to-nearest-even fp32 -> bf16 bits; NaN -> 0x7FC0 (matches the numpy restatement).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ float bf16_round(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

// fp16 bits <-> fp32 with the hardware converters (round to nearest even).
__device__ __forceinline__ float f16_bits_to_f32(uint16_t b) {
  float f;
  asm("{ .reg .b16 h; mov.b16 h, %1; cvt.f32.f16 %0, h; }" : "=f"(f) : "h"(b));
  return f;
}

__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
  uint16_t b;
  asm("{ .reg .b16 h; cvt.rn.f16.f32 h, %1; mov.b16 %0, h; }" : "=h"(b) : "f"(f));
  return b;
}

template <int SDT>
__device__ __forceinline__ float half_to_f32(uint16_t b) {
  if constexpr (SDT == BIGRIG_F16) return f16_bits_to_f32(b);
  else return bf16_bits_to_f32(b);
}

template <int SDT>
__device__ __forceinline__ uint16_t f32_to_half(float f) {
  if constexpr (SDT == BIGRIG_F16) return f32_to_f16_bits(f);
  else return f32_to_bf16_bits(f);
}

// Streaming 128-bit load of data read exactly once (expert codes): bypass L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

// The activation of a gated expert (BIGRIG_LAYOUT_ACT of the layout's flags) from its
// fp32 gate and up outputs: SwiGLU, or gpt-oss's clamped form
// g' = min(g, 7), u' = clamp(u, -7, 7), g' sigmoid(1.702 g') (u' + 1).
__device__ __forceinline__ float act_gated(float g, float u, int act) {
  if (act == BIGRIG_ACT_GPT_OSS) {
    g = fminf(g, 7.0f);
    u = fminf(fmaxf(u, -7.0f), 7.0f);
    return g / (1.0f + expf(-1.702f * g)) * (u + 1.0f);
  }
  return silu_f32(g) * u;
}

// The activation of a plain fc1/fc2 expert from its fp32 fc1 output.
__device__ __forceinline__ float act_plain(float h, int act) {
  if (act == BIGRIG_ACT_RELU2) {
    h = fmaxf(h, 0.0f);
    return h * h;
  }
  return silu_f32(h);
}

// Element f of projection p's affine bias in the expert at `base` (BIGRIG_LAYOUT_BIAS),
// as fp32; 0 when the layout carries none.
__device__ __forceinline__ float proj_bias(const uint8_t* base, const bigrig_expert_layout& L,
                                           int p, int f) {
  if (!(L.flags & BIGRIG_LAYOUT_BIAS)) return 0.0f;
  const uint8_t* b = base + L.bias_off[p];
  switch (BIGRIG_LAYOUT_BIAS_DTYPE(L.flags)) {
    case BIGRIG_F16: return f16_bits_to_f32(reinterpret_cast<const uint16_t*>(b)[f]);
    case BIGRIG_BF16: return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(b)[f]);
    default: return reinterpret_cast<const float*>(b)[f];
  }
}

// ------------------------------------------------------------------ mbarrier + bulk copy
// Non-tensor bulk copies (cp.async.bulk, no multicast) from global into this CTA's shared
// memory, completed through an mbarrier's transaction count.  Every wait is bounded.
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(
                   smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool bar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity`; false (after recording in err[1]) when it never came.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  for (uint32_t n = 0; n < kWaitLimit; ++n)
    if (bar_try_wait(bar, parity)) return true;
  if (err) atomicAdd(err + 1, 1);
  return false;
}

// L2 eviction policies for bulk copies: weights read once per token stream through L2
// (evict first), small tables every step reads stay (evict last).
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 cache policy from l2_evict_first / l2_evict_last
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// bytes and both addresses must be multiples of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace bigrig
