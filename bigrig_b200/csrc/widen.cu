// Admission of 3-bit experts: their codes widened to the 4-bit layout the kernels read.
//
// MLX affine 3-bit codes (bigrig_engine/stream.py:144-151 quant block; the shipped
// Qwen3-30B-A3B-3bit manifest gives gate_proj weight [768, 192] for in = 2048) are one
// little-endian bit stream per row, so a code can straddle two 32-bit words.  A code q in
// [0, 7] is also a valid 4-bit code with the same scale and bias, so the widened expert
// dequantises to exactly the same weights: every expert kernel (persistent decode, GEMV,
// tcgen05 GEMM) serves a 3-bit model unchanged.  The price is 4/3 of the code bytes in
// HBM and per decode step; host DRAM and PCIe keep carrying the 3-bit bytes.
//
// One thread per 32 codes of a row: 3 source words in, 4 packed words out (coalesced
// enough for a copy that runs once per admitted expert).
#include "common.cuh"
#include "launch.h"

namespace bigrig {

__global__ void widen3to4_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                 int64_t n_blocks) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_blocks) return;
  uint32_t w[4];
  w[0] = src[3 * i];
  w[1] = src[3 * i + 1];
  w[2] = src[3 * i + 2];
  w[3] = 0u;
  uint32_t out[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const int bit = 3 * c, word = bit >> 5, sh = bit & 31;
    uint32_t v = w[word] >> sh;
    if (sh > 29) v |= w[word + 1] << (32 - sh);
    out[c >> 3] |= (v & 7u) << (4 * (c & 7));
  }
  dst[4 * i] = out[0];
  dst[4 * i + 1] = out[1];
  dst[4 * i + 2] = out[2];
  dst[4 * i + 3] = out[3];
}

int launch_widen_expert(const void* src, void* dst, const bigrig_expert_layout& L, cudaStream_t s) {
  // the 3-bit expert lies out as the 4-bit one does -- per projection weight, scales,
  // biases in gate, up, down order -- with 3/4 of the code bytes
  const auto* in = static_cast<const uint8_t*>(src);
  auto* out = static_cast<uint8_t*>(dst);
  int64_t pos = 0;
  for (int p = 0; p < 3; ++p) {
    const int64_t rows = p == 2 ? L.hidden : L.inter, cols = p == 2 ? L.inter : L.hidden;
    const int64_t n_blocks = rows * cols / 32;              // 32 codes each
    const int64_t code3 = n_blocks * 3 * 4;
    const int64_t sb = 2 * rows * (cols / L.group_size) * 2;  // scales then biases
    if (L.weight_off[p] % 16 || L.biases_off[p] != L.scales_off[p] + sb / 2 ||
        L.scales_off[p] != L.weight_off[p] + n_blocks * 16)
      return set_error(BIGRIG_ERR_UNSUPPORTED, "widen_expert: projection %d is not laid out as "
                       "weight, scales, biases", p);
    const unsigned threads = 256;
    const unsigned blocks = static_cast<unsigned>((n_blocks + threads - 1) / threads);
    widen3to4_kernel<<<blocks, threads, 0, s>>>(reinterpret_cast<const uint32_t*>(in + pos),
                                                reinterpret_cast<uint32_t*>(out + L.weight_off[p]),
                                                n_blocks);
    if (int rc = check_launch("widen3to4_kernel")) return rc;
    if (cudaMemcpyAsync(out + L.scales_off[p], in + pos + code3, sb, cudaMemcpyDeviceToDevice, s) !=
        cudaSuccess)
      return set_error(BIGRIG_ERR_CUDA, "widen_expert: %s", cudaGetErrorString(cudaGetLastError()));
    pos += code3 + sb;
  }
  return BIGRIG_OK;
}

}  // namespace bigrig
