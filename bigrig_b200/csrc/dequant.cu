// Dequantise one expert projection from its MLX affine codes into the scale dtype.
//
// Replaces mx.dequantize (bigrig_engine/tune.py:64-70, precision.py:186-189) for
// the test and oracle comparisons: out = round(f32(scale) * q + f32(bias)) with a
// single fp32 rounding of the add (scale * q is exact in fp32), then one
// round-to-nearest-even into fp16/bf16.  One thread per uint32 code word.
#include "common.cuh"
#include "launch.h"

namespace bigrig {

template <int BITS, int SDT>
__global__ void dequant_kernel(const uint32_t* __restrict__ codes, const uint16_t* __restrict__ scales,
                               const uint16_t* __restrict__ biases, int rows, int cols, int group,
                               uint16_t* __restrict__ out) {
  constexpr int PER = 32 / BITS;
  const int words_per_row = cols / PER;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (wid >= static_cast<int64_t>(rows) * words_per_row) return;
  const int r = static_cast<int>(wid / words_per_row);
  const int wc = static_cast<int>(wid - static_cast<int64_t>(r) * words_per_row);
  const int col0 = wc * PER;
  const int g = col0 / group;
  const int groups = cols / group;
  const float s = half_to_f32<SDT>(scales[static_cast<int64_t>(r) * groups + g]);
  const float b = half_to_f32<SDT>(biases[static_cast<int64_t>(r) * groups + g]);
  const uint32_t w = codes[wid];
  uint16_t* o = out + static_cast<int64_t>(r) * cols + col0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const float q = static_cast<float>((w >> (j * BITS)) & ((1u << BITS) - 1u));
    o[j] = f32_to_half<SDT>(__fadd_rn(__fmul_rn(s, q), b));
  }
}

int launch_dequant(const void* slab, const bigrig_expert_layout& L, int slot, int proj, void* out,
                   cudaStream_t st) {
  const uint8_t* base = static_cast<const uint8_t*>(slab) + static_cast<int64_t>(slot) * L.slot_stride;
  const int rows = proj == 2 ? L.hidden : L.inter;
  const int cols = proj == 2 ? L.inter : L.hidden;
  const auto* codes = reinterpret_cast<const uint32_t*>(base + L.weight_off[proj]);
  const auto* sc = reinterpret_cast<const uint16_t*>(base + L.scales_off[proj]);
  const auto* bi = reinterpret_cast<const uint16_t*>(base + L.biases_off[proj]);
  const int64_t words = static_cast<int64_t>(rows) * cols / (32 / L.bits);
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((words + threads - 1) / threads);
  auto* o = static_cast<uint16_t*>(out);
  TimedLaunch tl(BIGRIG_K_DEQUANT, st);
#define BIGRIG_DQ(B, S)                                                                       \
  if (L.bits == B && L.scale_dtype == S) {                                                    \
    dequant_kernel<B, S><<<blocks, threads, 0, st>>>(codes, sc, bi, rows, cols, L.group_size, o); \
    return check_launch("dequant_kernel");                                                    \
  }
  BIGRIG_DQ(4, BIGRIG_F16)
  BIGRIG_DQ(4, BIGRIG_BF16)
  BIGRIG_DQ(8, BIGRIG_F16)
  BIGRIG_DQ(8, BIGRIG_BF16)
#undef BIGRIG_DQ
  return set_error(BIGRIG_ERR_UNSUPPORTED, "dequant: bits=%d scale_dtype=%d not built", L.bits,
                   L.scale_dtype);
}

}  // namespace bigrig
