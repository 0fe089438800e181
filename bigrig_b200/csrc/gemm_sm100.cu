// Expert-grouped GEMM for prefill-sized MoE calls on the 5th-generation tensor
// cores (tcgen05, accumulators in TMEM), with the MLX affine dequantisation fused
// into the operand staging.
//
// Replaces the reference's per-expert mx.quantized_matmul / gather_qmm over the
// expert-sorted (token, k) pairs (bigrig_engine/stream.py:1237-1276, 1320-1336,
// 1605-1631).  Two passes over the pairs grouped by expert:
//   gate_up: h[p, f] = bf16(silu(x.Wg^T) * (x.Wu^T))   (two fp32 accumulators)
//   down:    y[pair, f] = bf16(h[p, :] . Wd^T), scattered to (token, k) order
//
// Swap-AB: D[feature, token] = W[feature, K] . X[token, K]^T, so the expert's
// output features fill the 128-row M of the MMA and the few tokens an expert gets
// are the N dimension (a multiple of 16 up to 256).  The weight operand A is
// dequantised into tensor memory (one row per TMEM lane); the token operand B is a
// K-major tile of 64 K-elements in 128-byte-swizzled shared memory, so each of the
// four K=16 MMAs of an iteration starts 32 bytes further into the swizzle atom.
//
// Warp roles in a CTA of 576 threads, persistent over (expert, feature tile, token
// slice) work items:
//   warp 17    loader: one lane issues every copy -- a tile's scale and bias blocks
//              (one bulk copy each, they are contiguous), the codes as TMA boxes of
//              128 rows x 128 bytes (four 4-bit or two 8-bit iterations per box) and
//              the token rows as one TMA box per iteration -- each completing on its
//              ring slot's mbarrier by transaction count.
//   warps 0-7  producers: dequantise their row's codes from the swizzled box into
//              registers (w = OT(s * q + b), OT the operand type) and write them to
//              the A slot in TMEM with tcgen05.st; warp 0 also waits for the slot's
//              token rows; all arrive on the slot's hardware named barrier.
//   warp 16    MMA issuer: syncs on the slot's named barrier, one lane issues
//              tcgen05.mma (A from TMEM, B from shared memory) and commits the slot
//              back to its empty barrier and a finished tile to its accumulator
//              barrier.
//   warps 8-15 epilogue: TMEM accumulators -> silu(gate) * up (h, expert-sorted
//              rows) or the down output scattered to (token, k) order.
// Every mbarrier wait is bounded: past the limit the CTA records an error, raises
// a shared abort flag so every other wait returns at once, drains the MMAs it
// issued and the copies in flight, frees its TMEM and returns.
#include <cuda.h>

#include "gemv_common.cuh"

namespace bigrig {
namespace sm100 {

constexpr int kProducerWarps = 8;
constexpr int kProducerThreads = kProducerWarps * 32;
static_assert(kProducerThreads == 256, "one producer thread per A-tile row and matrix");
constexpr int kEpilogueWarps = 8;          // two per TMEM lane quarter
constexpr int kMmaWarp = kProducerWarps + kEpilogueWarps;
constexpr int kLoaderWarp = kMmaWarp + 1;
constexpr int kThreads = (kLoaderWarp + 1) * 32;
// A-slot handoff producers -> MMA warp: hardware named barrier kReadyBar0 + slot, which
// the producer warps arrive on and the MMA warp syncs on (the issuing warp touches no
// shared memory to learn that a slot is ready; every shared-memory access it makes holds
// up its next tcgen05.mma by hundreds of cycles under tensor load)
constexpr int kReadyBar0 = 1;
constexpr int kReadyCount = (kProducerWarps + 1) * 32;
constexpr int kBlockM = 128;
constexpr int kBlockK = 64;                 // one 128-byte swizzle atom of bf16 per row
constexpr uint32_t kSpinLimit = 1u << 22;   // a few seconds of polling before giving up

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the hardware suspend the thread for up to ~1 us while the phase is
// incomplete (it returns as soon as the phase completes): waiting warps stop competing
// for issue slots with the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity`.  Returns false when the CTA is aborting.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* err, int where) {
  uint32_t n = 0;
  while (!mbar_try_wait_sleep(bar, parity)) {
    if (*abort_flag) return false;
    if (++n > kSpinLimit) {
      *abort_flag = 1;
      if (err) atomicAdd(err + 1, 1);
      if (err) atomicExch(err + 2, where);
      return false;
    }
  }
  return true;
}

// mbar_wait with the reason it returned: 0 the phase completed, 1 the CTA is aborting
// (another role raised the flag), 2 this wait ran out (it raised the flag).
__device__ __forceinline__ int mbar_wait_why(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             int32_t* err, int where) {
  uint32_t n = 0;
  while (!mbar_try_wait_sleep(bar, parity)) {
    if (*abort_flag) return 1;
    if (++n > kSpinLimit) {
      *abort_flag = 1;
      if (err) atomicAdd(err + 1, 1);
      if (err) atomicExch(err + 2, where);
      return 2;
    }
  }
  return 0;
}

// Bounded wait that does not give up on the abort flag (catch-up arrivals after an abort).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t n = 0; n < kSpinLimit; ++n)
    if (mbar_try_wait_sleep(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);          // start address
  d |= static_cast<uint64_t>(1) << 16;                        // leading byte offset (unused)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;                // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                        // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                        // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: f16 x f16 or bf16 x bf16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N, int ot = BIGRIG_BF16) {
  const uint32_t fmt = ot == BIGRIG_F16 ? 0u : 1u;  // 0 f16, 1 bf16 (A and B alike)
  return (1u << 4)                                   // D format f32
         | (fmt << 7)                                // A format
         | (fmt << 10)                               // B format
         | (static_cast<uint32_t>(N >> 3) << 17)     // N
         | (static_cast<uint32_t>(M >> 4) << 24);    // M
}

// A from tensor memory (128 lanes = rows, K in 32-bit columns of operand pairs), B from
// a shared-memory descriptor.
__device__ __forceinline__ void mma_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t db,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void nb_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void nb_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 32 lanes x 16 columns of 32 bits from TMEM (this warp's lane quarter), not waited for.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// fp32 -> bf16 bits, round to nearest even (the hardware conversion).
__device__ __forceinline__ uint16_t bf16_rn(float f) {
  uint16_t b;
  asm("{ .reg .b16 h; cvt.rn.bf16.f32 h, %1; mov.b16 %0, h; }" : "=h"(b) : "f"(f));
  return b;
}

// silu(g) = g / (1 + e^-g) with the fast exponential and division: h is rounded to a
// 16-bit type right after, far above their error.
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// 32 lanes x 8 columns of fp32 from TMEM (this warp's lane quarter).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Byte offset of 16-byte chunk `j` (0..7) of row `r` in a 128B-swizzled K-major tile.
__device__ __forceinline__ uint32_t swz(int r, int j) {
  return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
}

// ------------------------------------------------------------------ dequantisation
// One 16-byte code chunk of a row -> bf16 in the A tile.  4-bit: 32 codes -> 64 bytes
// (tile chunks jbase..jbase+3); 8-bit: 16 codes -> 32 bytes (jbase, jbase+1).
// w = bf16(fma(s, q, b)) with q recovered exactly through the 2^23 mantissa trick and
// the scale pre-divided by the code field's power of 16 (or 256), which is exact.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Packed-pair arithmetic in the operand type OT (BIGRIG_F16 or BIGRIG_BF16), one rounding.
template <int OT>
__device__ __forceinline__ uint32_t x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (OT == BIGRIG_F16) asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <int OT>
__device__ __forceinline__ uint32_t x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  if constexpr (OT == BIGRIG_F16) asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Tensor-core operand type of a format: the 4-bit path computes in the scale dtype (as
// the reference's fp16 and bf16 models do); the 8-bit path in bf16.
__host__ __device__ constexpr int operand_type(int bits, int sdt) {
  return bits == 4 && sdt == BIGRIG_F16 ? BIGRIG_F16 : BIGRIG_BF16;
}

// K order inside every 8-element block of the 4-bit path's operands: slot 2i holds
// element i and slot 2i+1 element i+4, so that one mask of a 32-bit code word yields
// the pair of codes (i, i+4).  A dot product over K is unchanged when both operands
// carry the same order; the token operand is permuted to match.
__host__ __device__ constexpr int k8_slot(int i) { return i < 4 ? 2 * i : 2 * (i - 4) + 1; }

// 4-bit: one 16-byte chunk (32 codes) of a row -> 16 words of OT pairs (o[0..15], K
// order as k8_slot says).  The pair 0x6400 | n (fp16) or 0x4300 | n (bf16) is the value
// 1024 + n or 128 + n exactly; subtracting the base leaves q exactly, and one packed fma
// gives w = OT(s * q + b) with a single rounding, s and b being the format's own scale
// and bias (exact in OT).
//
// fp16 takes the odd nibbles without a shift: 0x6400 | (n << 4) is 1024 + 16 n, and
// fma(v, 1/16, -64) = n exactly (fp16 has the mantissa bits to hold 16 n; bf16 does not).
template <int OT>
__device__ __forceinline__ void dequant_chunk4(uint4 w, uint32_t s2, uint32_t b2, uint32_t* o) {
  constexpr uint32_t base = OT == BIGRIG_F16 ? 0x64006400u : 0x43004300u, m = 0x000F000Fu;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {            // word i: codes 8i..8i+7 -> words 4i..4i+3
    const uint32_t c = ws[i];
    if constexpr (OT == BIGRIG_F16) {
      constexpr uint32_t m_hi = 0x00F000F0u, sixteenth = 0x2C002C00u, neg64 = 0xD400D400u;
      const uint32_t c8 = c >> 8;
      o[4 * i + 0] = x2_fma<OT>(x2_sub<OT>((c & m) | base, base), s2, b2);
      o[4 * i + 1] = x2_fma<OT>(x2_fma<OT>((c & m_hi) | base, sixteenth, neg64), s2, b2);
      o[4 * i + 2] = x2_fma<OT>(x2_sub<OT>((c8 & m) | base, base), s2, b2);
      o[4 * i + 3] = x2_fma<OT>(x2_fma<OT>((c8 & m_hi) | base, sixteenth, neg64), s2, b2);
    } else {
      o[4 * i + 0] = x2_fma<OT>(x2_sub<OT>((c & m) | base, base), s2, b2);
      o[4 * i + 1] = x2_fma<OT>(x2_sub<OT>(((c >> 4) & m) | base, base), s2, b2);
      o[4 * i + 2] = x2_fma<OT>(x2_sub<OT>(((c >> 8) & m) | base, base), s2, b2);
      o[4 * i + 3] = x2_fma<OT>(x2_sub<OT>(((c >> 12) & m) | base, base), s2, b2);
    }
  }
}

// 8-bit: one 16-byte chunk (16 codes) -> 8 words of bf16 pairs, natural K order.
// w = bf16(fma(s, q, b)) in fp32, q recovered exactly through the 2^23 mantissa trick
// with the scale pre-divided by 256 for the high byte (exact).
__device__ __forceinline__ void dequant_chunk8(uint4 w, float s, float b, uint32_t* o) {
  constexpr float M = 8388608.f;
  constexpr uint32_t E23 = 0x4B000000u;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  const float s1 = s * 0.00390625f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {            // word i: codes 4i..4i+3 -> words 2i, 2i+1
    const uint32_t a = ws[i];
    o[2 * i] = pack_bf16x2(fmaf(s, __uint_as_float((a & 0x00FFu) | E23) - M, b),
                           fmaf(s1, __uint_as_float((a & 0xFF00u) | E23) - M, b));
    o[2 * i + 1] = pack_bf16x2(fmaf(s, __uint_as_float(((a >> 16) & 0x00FFu) | E23) - M, b),
                               fmaf(s1, __uint_as_float(((a >> 16) & 0xFF00u) | E23) - M, b));
  }
}

// 32 lanes x N 32-bit columns into TMEM (this warp's lane quarter), N = 16 or 32.
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t* v) {
  if constexpr (N == 16) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
  } else {
    static_assert(N == 32, "tmem_st: 16 or 32 columns");
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
        "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
        "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
  }
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// fp32 pair -> fp16 pair, saturating at the largest finite fp16 (no infinities).
__device__ __forceinline__ uint32_t pack_f16x2_sat(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// xs[p] = x[order[p] / k] for the P expert-sorted pairs: the gate/up token operand as
// contiguous rows for its TMA boxes.  The 4-bit path also takes it to the operand type
// OT (bf16 -> fp16 is exact inside the fp16 range and saturates outside it) and to the
// k8_slot order inside every 8-element block.
template <int OT, bool K8>
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ order,
                                   int k, int P, int chunks_per_row, uint4* __restrict__ xs) {
  const int64_t n = static_cast<int64_t>(P) * chunks_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(i / chunks_per_row), c = static_cast<int>(i % chunks_per_row);
    uint4 v = x[static_cast<int64_t>(order[p] / k) * chunks_per_row + c];
    if constexpr (OT == BIGRIG_F16) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = pack_f16x2_sat(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xFFFF0000u));
    }
    if constexpr (K8) {
      uint4 o;
      o.x = __byte_perm(v.x, v.z, 0x5410);   // (e0, e4)
      o.y = __byte_perm(v.x, v.z, 0x7632);   // (e1, e5)
      o.z = __byte_perm(v.y, v.w, 0x5410);   // (e2, e6)
      o.w = __byte_perm(v.y, v.w, 0x7632);   // (e3, e7)
      v = o;
    }
    xs[i] = v;
  }
}

// ------------------------------------------------------------------ TMA
// Tiled tensor loads (no multicast) into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, int x, int y, int z,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ uint32_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
  return v;
}

// ------------------------------------------------------------------ pipeline shape
// Rings (shared memory unless noted):
//   codes : RS slots of NMAT TMA boxes, 128 rows x 128 bytes each (F iterations of
//           one row's codes), 128-byte swizzled
//   B     : SA slots of BN token rows x 64 operands, 128-byte swizzled (one iteration)
//   scales: NSB per-tile buffers of the tile's scale and bias blocks (NMAT x 2 x 128
//           rows x K / group_size)
//   A     : (TMEM) SA slots of NMAT dequantised 128 x 64 tiles, one row per TMEM lane,
//           written by the producers with tcgen05.st and read by the MMA from tensor
//           memory, so the weights never make a round trip through shared memory
// An A slot and the B slot of the same index form one ring slot: one MMA commit per
// iteration frees both.  The accumulators take the TMEM columns after the A slots.  RS
// and NSB are chosen at launch (the scale buffer's size depends on K).
//
// Producer thread mapping: warp w owns TMEM lane quarter w % 4, i.e. rows
// 32 (w % 4) + lane of the tile; gate/up warps 0-3 take the gate rows and 4-7 the up
// rows (every code chunk of the row), down warps 0-3 the first and 4-7 the second half
// of each row's code chunks of an iteration.
template <int MODE, int BN, int BITS>
struct GemmShape {
  static constexpr int NMAT = MODE == 0 ? 2 : 1;
  // K-steps of 64 per iteration (one slot, one handoff, one commit): the down pass has
  // one matrix, so it takes two steps to give each handoff eight MMAs like gate/up
  static constexpr int KS = MODE == 0 ? 1 : 2;
  static constexpr int ROW_BYTES = kBlockK * BITS / 8;            // one row's codes per step
  static constexpr int F = 128 / ROW_BYTES;                       // steps per code box
  static constexpr int IPB = F / KS;                              // iterations per code box
  static constexpr int CPI = ROW_BYTES / 16;                      // 16-byte chunks per step
  static constexpr int JT = CPI;                                  // chunks per thread and step
  static constexpr int WPC = 64 / BITS;                           // A words per code chunk
  static constexpr int AW = JT * WPC;                             // A words per thread (32)
  static constexpr int SLOT_COLS = NMAT * KS * 32;                // TMEM columns of an A slot
  static constexpr int CODE_BOX = kBlockM * 128;
  static constexpr int CODE_SLOT = NMAT * CODE_BOX;
  static constexpr int B_BOX = BN * kBlockK * 2;                  // one step's token rows
  static constexpr int B_BYTES = KS * B_BOX;                      // one token-row slot
  // TMEM: SA A slots, then NBUF accumulators of NMAT x BN columns.  Two accumulators (the
  // epilogue drains one while the MMA fills the other) with as many A slots as fit (up
  // to 4, at least 2), else one accumulator and 3 slots.
  static constexpr int ACC_COLS = NMAT * BN;
  static constexpr int SA = 4 * SLOT_COLS + 2 * ACC_COLS <= 512 ? 4
                          : 3 * SLOT_COLS + 2 * ACC_COLS <= 512 ? 3
                          : 2 * SLOT_COLS + 2 * ACC_COLS <= 512 ? 2 : 3;
  static constexpr int A_COLS = SA * SLOT_COLS;
  static constexpr int NBUF = A_COLS + 2 * ACC_COLS <= 512 ? 2 : 1;  // accumulator buffers
  static constexpr int TMEM_COLS = 512;
  static constexpr int kMeta = 2048;                              // barriers, flags, tile prefix
  static constexpr int kLimit = 227 * 1024;
  static constexpr size_t smem(int rs, int sb, int nsb, int sc_bytes) {
    return 1024 + static_cast<size_t>(rs) * CODE_SLOT + static_cast<size_t>(sb) * B_BYTES +
           static_cast<size_t>(nsb) * sc_bytes + kMeta;
  }
  // Token-row slots: the A slots' ring (one commit frees both) once a step carries enough
  // MMA work to cover a TMA load's latency; small tiles (a few rows per expert, decode
  // batches) get their own deeper ring of small slots and a second commit per step.
  static constexpr int SB = BN <= 32 ? 12 : BN <= 64 ? 8 : SA;
  static constexpr bool SPLIT_B = SB != SA;
  static_assert(A_COLS + NBUF * ACC_COLS <= TMEM_COLS, "grouped_gemm: TMEM columns");
  static_assert(AW == 32 && F % KS == 0, "grouped_gemm: mapping");
};

struct GemmRings {
  int rs, sb, nsb, sc_bytes;
};

// A work item: one 128-feature tile of one expert against one slice of its rows.  A
// segment of R rows is cut into ceil(R / BN) equal slices (multiples of 16), so a
// segment just over BN rows gets two half-size MMAs instead of a full and a sliver.
struct GemmTile {
  int slot, row0, m0, n0, rows, local;
};

// A CTA's work items come in increasing order, so each role walks the segments forward
// instead of searching the tile prefix for every item.
struct TileWalker {
  int seg = 0;
  __device__ __forceinline__ GemmTile at(const RouteView& rv, const int* tile_start, int nseg,
                                         int m_tiles, int BN, int tile) {
    while (seg + 1 < nseg && tile_start[seg + 1] <= tile) ++seg;
    GemmTile t;
    int R;
    t.local = tile - tile_start[seg];
    t.slot = segment_slot(rv, seg, t.row0, R);
    const int nt = (R + BN - 1) / BN;
    const int rpt = (((R + nt - 1) / nt) + 15) & ~15;
    const int mt = t.local / nt, ni = t.local - mt * nt;
    t.m0 = mt * kBlockM;
    t.n0 = ni * rpt;
    t.rows = min(rpt, R - t.n0);
    return t;
  }
};

// Ring cursor: slot index and the parity of its current use.
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++slot == n) { slot = 0; phase ^= 1u; }
  }
};

// ------------------------------------------------------------------ phase timing
// Tuning builds only (-DBIGRIG_GEMM_PROFILE): one producer lane, one epilogue lane,
// the MMA lane and the loader lane add clock64 spans per phase into g_gemm_prof (read
// and cleared through bigrig_gemm_prof_read).  A normal build compiles none of it.
#ifdef BIGRIG_GEMM_PROFILE
__device__ unsigned long long g_gemm_prof[64];      // [MODE][32]
#define GG_T(v) const long long v = clock64()
#define GG_ADD(i, v) (prof[i] += clock64() - (v))
#define GG_INC(i) (prof[i] += 1)
#else
#define GG_T(v)
#define GG_ADD(i, v)
#define GG_INC(i)
#endif

// ------------------------------------------------------------------ the kernel
// MODE 0: gate/up (two weight matrices, output h); MODE 1: down (one matrix, output y);
// MODE 2: a plain expert's fc1 (one matrix over the hidden dimension, output h).
// tm_code0/1: the codes of projection gate/up (MODE 0) or down (tm_code0, MODE 1) over
// the slab as [slot][row][byte]; tm_act: the token operand [P rows][K] (expert-sorted).
template <int MODE, int BN, int BITS, int SDT>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(
    const __grid_constant__ CUtensorMap tm_code0, const __grid_constant__ CUtensorMap tm_code1,
    const __grid_constant__ CUtensorMap tm_act, RouteView rv, const uint8_t* __restrict__ slab,
    bigrig_expert_layout L, GemmRings rg,
    uint16_t* __restrict__ out) {       // MODE 0: h [P, I]; MODE 1: y [P, H] ((token, k) order)
  using G = GemmShape<MODE, BN, BITS>;
  constexpr int NMAT = G::NMAT, JT = G::JT, NBUF = G::NBUF, WPC = G::WPC, F = G::F, CPI = G::CPI;
  constexpr int KS = G::KS, IPB = G::IPB;
  constexpr int S = G::SA;               // slots: an A slot in TMEM and a B slot in smem
  constexpr int OT = operand_type(BITS, SDT);
  const int RS = rg.rs, NSB = rg.nsb;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned by an offset from the shared array itself, so that every pointer
  // below stays in the shared address space (plain LDS/STS, no generic addressing)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* code_ring = smem;
  uint8_t* b_ring = code_ring + RS * G::CODE_SLOT;
  const int SB = G::SPLIT_B ? rg.sb : S;  // token-row slots (split rings: chosen at launch)
  uint8_t* sc_ring = b_ring + SB * G::B_BYTES;
  uint64_t* code_full = reinterpret_cast<uint64_t*>(sc_ring + NSB * rg.sc_bytes);
  uint64_t* code_empty = code_full + RS;
  uint64_t* b_full = code_empty + RS;    // [G::SB]
  uint64_t* s_empty = b_full + G::SB;    // A slot (and, unsplit, its B slot) free again
  uint64_t* b_empty = s_empty + S;       // split rings only: token-row slot free again
  uint64_t* sc_full = b_empty + G::SB;
  uint64_t* sc_empty = sc_full + 2;
  uint64_t* acc_full = sc_empty + 2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  int* tile_rows = reinterpret_cast<int*>(drain_bar + 1);  // [8] token columns of tile j at j % 8
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(tile_rows + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);
  int* tile_start = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_base_s + 2));  // [nseg+1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = MODE != 1 ? L.hidden : L.inter;        // reduction length
  const int NF = MODE != 1 ? L.inter : L.hidden;       // output features
  const int m_tiles = (NF + kBlockM - 1) / kBlockM;
  const int k_steps = K / kBlockK;                     // 64-element K steps
  const int k_iters = (k_steps + KS - 1) / KS;         // iterations (slots) per tile
  const int gpitch = K / L.group_size;
  const int nseg = min(min(*rv.num_seg, rv.s_max), kMaxExperts);

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; ++i) {
      mbar_init(&code_full[i], 1);
      mbar_init(&code_empty[i], kProducerWarps);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < S; ++i) mbar_init(&s_empty[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], kProducerWarps);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpilogueWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // tile prefix over segments: segment s owns m_tiles * ceil(R_s / BN) work items
  if (warp == 0 && lane == 0) {
    int acc = 0;
    for (int s = 0; s < nseg; ++s) {
      tile_start[s] = acc;
      int row0, R;
      segment_slot(rv, s, row0, R);        // R = 0 for inconsistent metadata: no tiles
      acc += m_tiles * ((R + BN - 1) / BN);
    }
    tile_start[nseg] = acc;
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_base_s, G::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  const uint32_t tmem_acc = tmem + G::A_COLS;          // accumulators after the A slots
  const int total = tile_start[nseg];
  const int my_tiles = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int sc_half = kBlockM * gpitch * 2;            // one (mat, scale|bias) block in bytes
#ifdef BIGRIG_GEMM_PROFILE
  long long prof[32] = {};
  GG_T(t_kernel);
#endif

  if (warp < kProducerWarps) {
    // ---------------------------------------------------------------- producers
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;                      // tile row = TMEM lane
    const int mat = MODE == 0 ? half : 0;                   // gate/up: the matrix
    const int ts = MODE == 0 ? 0 : half;                    // down: the step of the iteration
    const uint32_t code_base = smem_u32(code_ring) + mat * G::CODE_BOX + r * 128;
    const uint32_t sc_base = smem_u32(sc_ring) + (mat * 2) * sc_half + r * gpitch * 2;
    // this thread's A columns: slot s at s * SLOT_COLS + mat * KS * 32 + ts * 32, lane r
    const uint32_t a_taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + mat * KS * 32 + ts * 32;
    // a row's scales start 16-byte aligned when K / group_size is a multiple of 8: then
    // eight groups come in one 16-byte read (lanes are rows gpitch * 2 bytes apart, so
    // per-group 2-byte reads would pile onto two banks)
    const bool s_vec = (gpitch & 7) == 0;
    const int ipg = L.group_size / kBlockK;                 // iterations per scale group
    Ring cr, ar, br;                          // br: token-row slots (split rings only)
    bool ok = true;
    // Every iteration of a tile gets exactly one arrival on its slot's named barrier from
    // every producer warp, on the way out too.  The MMA warp checks the abort flag once
    // per tile, so a warp that gives up (a bounded wait ran out, or another role aborted:
    // the flag is set either way) keeps arriving to the end of its tile, each arrival
    // after the slot's previous use completed -- never two on one barrier phase.  If a
    // slot wait itself ran out, the MMAs are stuck: one last arrival, unthrottled (the MMA
    // warp already took the slot's previous phase), and no more.
    auto bail = [&](int kit, bool throttle_first) {
      for (int q = kit; q < k_iters; ++q) {
        if ((q > kit || throttle_first) &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(&s_empty[ar.slot], ar.phase ^ 1)))
          break;
        __syncwarp();
        nb_arrive(kReadyBar0 + ar.slot, kReadyCount);
        ar.next(S);
        if (!throttle_first && q == kit) break;
      }
      ok = false;
    };
    for (int j = 0; j < my_tiles && ok; ++j) {
      const int sb = j % NSB;
      GG_T(t7);
      if (!__all_sync(0xffffffffu, mbar_wait(&sc_full[sb], (j / NSB) & 1, abort_flag, rv.err, 1))) {
        bail(0, true);
        break;
      }
      GG_ADD(7, t7);
      const uint32_t s_addr = sc_base + sb * rg.sc_bytes, b_addr = s_addr + sc_half;
      uint4 s8 = make_uint4(0, 0, 0, 0), b8 = s8;
      int cur8 = -1;                          // block of 8 groups held in s8 / b8
      for (int kit0 = 0; kit0 < k_steps && ok; kit0 += F) {
        // this thread's codes of its steps of the box's IPB iterations, read at once;
        // the box is handed back to the loader right away
        GG_T(t0);
        if (!__all_sync(0xffffffffu, mbar_wait(&code_full[cr.slot], cr.phase, abort_flag, rv.err, 2))) {
          bail(kit0 / KS, true);
          break;
        }
        GG_ADD(0, t0);
        const uint32_t cb = code_base + cr.slot * G::CODE_SLOT;
        uint4 wb[IPB][JT];
        uint32_t landed = 0;
#pragma unroll
        for (int ib = 0; ib < IPB; ++ib)
#pragma unroll
          for (int c = 0; c < JT; ++c) {
            wb[ib][c] = lds128(cb + ((((ib * KS + ts) * CPI + c) ^ (r & 7)) << 4));
            landed ^= wb[ib][c].w;
          }
        // the loads must have returned before the box goes back to the loader (its next
        // TMA box overwrites it): an instruction reading every load's result makes the
        // warp wait for all of them
        asm volatile("" ::"r"(landed));
        __syncwarp();
        if (lane == 0) mbar_arrive(&code_empty[cr.slot]);
        cr.next(RS);
#pragma unroll
        for (int ib = 0; ib < IPB; ++ib) {
          const int it_step = kit0 + ib * KS;       // first step of this iteration
          if (it_step >= k_steps || !ok) break;
          const int kstep = it_step + ts;           // this thread's step
          const bool have = kstep < k_steps;        // (an odd last step has no partner)
          GG_T(t2);
          uint32_t av[G::AW];
          if (have) {
            const int grp = ipg == 1 ? kstep : kstep / ipg;
            uint32_t sh, bh;
            if (s_vec) {
              if ((grp >> 3) != cur8) {
                cur8 = grp >> 3;
                s8 = lds128(s_addr + cur8 * 16);
                b8 = lds128(b_addr + cur8 * 16);
              }
              const int wi = (grp >> 1) & 3, hs = (grp & 1) * 16;
              sh = ((wi == 0 ? s8.x : wi == 1 ? s8.y : wi == 2 ? s8.z : s8.w) >> hs) & 0xFFFFu;
              bh = ((wi == 0 ? b8.x : wi == 1 ? b8.y : wi == 2 ? b8.z : b8.w) >> hs) & 0xFFFFu;
            } else {
              sh = lds16(s_addr + grp * 2);
              bh = lds16(b_addr + grp * 2);
            }
            if constexpr (BITS == 4) {         // operands in the scale dtype itself
              const uint32_t s2 = sh * 0x10001u, b2 = bh * 0x10001u;
#pragma unroll
              for (int c = 0; c < JT; ++c) dequant_chunk4<OT>(wb[ib][c], s2, b2, av + c * WPC);
            } else {
              const float sv = half_to_f32<SDT>(static_cast<uint16_t>(sh));
              const float bv = half_to_f32<SDT>(static_cast<uint16_t>(bh));
#pragma unroll
              for (int c = 0; c < JT; ++c) dequant_chunk8(wb[ib][c], sv, bv, av + c * WPC);
            }
          }
          GG_ADD(2, t2);
          GG_T(t1);
          const int why = mbar_wait_why(&s_empty[ar.slot], ar.phase ^ 1, abort_flag, rv.err, 3);
          if (__any_sync(0xffffffffu, why != 0)) {
            // ran out: the MMAs are stuck, one last arrival; aborted: catch up, throttled
            bail(it_step / KS, !__any_sync(0xffffffffu, why == 2));
            break;
          }
          tc_fence_after();
          GG_ADD(1, t1);
          GG_T(t3);
          if (have) {
            tmem_st<G::AW>(a_taddr + ar.slot * G::SLOT_COLS, av);
            tmem_wait_st();
          }
          tc_fence_before();                  // TMEM stores -> the MMA after the barrier
          // warp 0 also sees this iteration's token rows land, so a completed handoff
          // means both operands are in place
          bool bok = true;
          if (warp == 0) {
            const Ring& bw = G::SPLIT_B ? br : ar;
            bok = __all_sync(0xffffffffu, mbar_wait(&b_full[bw.slot], bw.phase, abort_flag, rv.err, 11));
          }
          if (G::SPLIT_B) br.next(SB);
          __syncwarp();
          nb_arrive(kReadyBar0 + ar.slot, kReadyCount);
          ar.next(S);
          GG_ADD(3, t3);
          GG_INC(6);
          if (!bok) {                         // arrived for this iteration: catch up after it
            if (it_step / KS + 1 < k_iters) bail(it_step / KS + 1, true);
            ok = false;
            break;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_empty[sb]);
    }
  } else if (warp < kMmaWarp) {
    // ---------------------------------------------------------------- epilogue (warps 8-15)
    // warp 8 + e drains TMEM lane quarter e % 4 (features m0 + 32 (e % 4) + lane) and the
    // 16-column groups of token columns g with g % 2 == e / 4
    const int eq = warp & 3, eh = (warp - kProducerWarps) >> 2;
    TileWalker tw;
    for (int j = 0; j < my_tiles; ++j) {
      const GemmTile t = tw.at(rv, tile_start, nseg, m_tiles, BN, blockIdx.x + j * gridDim.x);
      const int buf = NBUF == 2 ? (j & 1) : 0, use = NBUF == 2 ? (j >> 1) : j;
      GG_T(t8);
      if (!mbar_wait(&acc_full[buf], use & 1, abort_flag, rv.err, 4)) break;
      GG_ADD(8, t8);
      GG_T(t9);
      tc_fence_after();
      const int f = t.m0 + eq * 32 + lane;
      const bool fok = f < NF;
      // the 4-bit down pass reads h as its K-permuted token operand
      const int fcol = BITS == 4 && MODE != 1 ? (f & ~7) | k8_slot(f & 7) : f;
      // the projection biases of this lane's feature (BIGRIG_LAYOUT_BIAS), and the activation
      const uint8_t* ebase = slab + static_cast<int64_t>(t.slot >= 0 ? t.slot : 0) * L.slot_stride;
      const float bias0 = fok ? proj_bias(ebase, L, MODE == 1 ? 2 : 0, f) : 0.f;
      const float bias1 = MODE == 0 && fok ? proj_bias(ebase, L, 1, f) : 0.f;
      const int act = BIGRIG_LAYOUT_ACT(L.flags);
      const uint32_t lane_addr = tmem_acc + (static_cast<uint32_t>(eq * 32) << 16) + buf * G::ACC_COLS;
      const int prow = t.row0 + t.n0;            // sorted row of token column 0
      // MODE 1 scatters column c to output row order[prow + c]: lanes 0-15 hold the 16
      // rows of a column group, loaded one group ahead
      int ord_next = 0;
      if (MODE == 1 && eh * 16 + lane < t.rows && lane < 16) ord_next = rv.order[prow + eh * 16 + lane];
      if constexpr (MODE != 1) {
        // gate/up (fc1): h for all of this warp's column groups first, kept as packed 16-bit
        // pairs in registers, so that the accumulator goes back to the MMA before any
        // global store (with one accumulator buffer the next tile's MMAs wait for it)
        constexpr int NG = (BN / 16 + 1) / 2;   // 16-column groups per warp (every other)
        uint32_t hp[NG * 8];
        // the activation is chosen once per tile (a uniform branch), never per element: the
        // default expert's loop is the plain SiLU one
        auto drain = [&](auto actf) {
#pragma unroll
          for (int gi = 0; gi < NG; ++gi) {
            const int j0 = (eh + 2 * gi) * 16;
            if (j0 < t.rows) {
              uint32_t a[16], u[16];
              tmem_ld16_nowait(lane_addr + j0, a);
              if constexpr (MODE == 0) tmem_ld16_nowait(lane_addr + BN + j0, u);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; i += 2) {
                const float h0 = actf(a[i], MODE == 0 ? u[i] : 0u);
                const float h1 = actf(a[i + 1], MODE == 0 ? u[i + 1] : 0u);
                hp[gi * 8 + i / 2] = OT == BIGRIG_F16 ? pack_f16x2_sat(h0, h1) : pack_bf16x2(h0, h1);
              }
            }
          }
        };
        if constexpr (MODE == 2) {
          drain([&](uint32_t gq, uint32_t) { return act_plain(__uint_as_float(gq) + bias0, act); });
        } else {
          if (L.flags == 0)
            drain([](uint32_t gq, uint32_t uq) {
              return silu_fast(__uint_as_float(gq)) * __uint_as_float(uq);
            });
          else
            drain([&](uint32_t gq, uint32_t uq) {
              return act_gated(__uint_as_float(gq) + bias0, __uint_as_float(uq) + bias1, act);
            });
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          const int j0 = (eh + 2 * gi) * 16;
          if (j0 < t.rows && fok) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              if (j0 + i < t.rows)
                out[static_cast<int64_t>(prow + j0 + i) * NF + fcol] =
                    t.slot < 0 ? uint16_t(0) : static_cast<uint16_t>(hp[gi * 8 + i / 2] >> ((i & 1) * 16));
            }
          }
        }
      } else {
        for (int j0 = eh * 16; j0 < t.rows; j0 += 32) {
          uint32_t a[16];
          tmem_ld16_nowait(lane_addr + j0, a);
          const int ord = ord_next;
          if (j0 + 32 + lane < t.rows && lane < 16) ord_next = rv.order[prow + j0 + 32 + lane];
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int o = __shfl_sync(0xffffffffu, ord, i);
            if (j0 + i < t.rows && fok)
              out[static_cast<int64_t>(o) * NF + f] = t.slot >= 0 ? bf16_rn(__uint_as_float(a[i]) + bias0) : uint16_t(0);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      GG_ADD(9, t9);
      GG_INC(10);
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer (warp 16)
    // Touches shared memory only once per tile (the accumulator wait, the abort flag and
    // the next tile's width): each access holds up the next tcgen05.mma by hundreds of
    // cycles under tensor load.
    const volatile int* rows_ring = tile_rows;
    Ring ar, br;
    int rows = 0;                             // token columns of the current tile
    for (int j = 0; j < my_tiles; ++j) {
      const int buf = NBUF == 2 ? (j & 1) : 0, use = NBUF == 2 ? (j >> 1) : j;
      // the epilogue must have drained this accumulator buffer's previous tile
      GG_T(t11);
      if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, rv.err, 5)) break;
      GG_ADD(11, t11);
      if (*abort_flag) break;                 // once per tile: a producer that gave up
                                              // keeps arriving to the end of its tile
      tc_fence_after();
      const uint32_t acc = tmem_acc + buf * G::ACC_COLS;
      uint32_t idesc = 0;
      for (int kit = 0; kit < k_iters; ++kit) {
        GG_T(t12);
        nb_sync(kReadyBar0 + ar.slot, kReadyCount);   // A slot and token rows in place
        GG_ADD(12, t12);
        GG_T(t13);
        if (kit == 0) {
          if (j == 0) rows = rows_ring[0];    // posted before the first token rows
          idesc = instr_desc(kBlockM, (rows + 15) & ~15, OT);
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ast = tmem + ar.slot * G::SLOT_COLS;
          const uint32_t bst = smem_u32(b_ring + (G::SPLIT_B ? br.slot : ar.slot) * G::B_BYTES);
          const int steps = min(KS, k_steps - kit * KS);
#pragma unroll
          for (int st = 0; st < KS; ++st) {
            if (st < steps) {
#pragma unroll
              for (int kk = 0; kk < kBlockK / 16; ++kk) {
                const uint64_t db = smem_desc(bst + st * G::B_BOX + kk * 32);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
                  mma_tmem_a(acc + m * BN, ast + m * KS * 32 + st * 32 + kk * 8, db, idesc,
                             (kit > 0 || st > 0 || kk > 0) ? 1u : 0u);
              }
            }
          }
          mma_commit(&s_empty[ar.slot]);      // A (and unsplit, B) slot free once these are done
          if (G::SPLIT_B) mma_commit(&b_empty[br.slot]);
          if (kit == k_iters - 1) mma_commit(&acc_full[buf]);
        }
        __syncwarp();
        ar.next(S);
        if (G::SPLIT_B) br.next(SB);
        GG_ADD(13, t13);
        // the next tile's width, read with this tile's last MMAs already queued (the
        // loader posted it before this iteration's token rows)
        if (kit == k_iters - 1 && j + 1 < my_tiles) rows = rows_ring[(j + 1) & 7];
      }
    }
  } else if (lane == 0) {
    // ---------------------------------------------------------------- loader (warp 17, one lane)
    Ring cr, sr;
    TileWalker tw;
    int ns = 0, nc = 0, nb = 0;                       // scale tiles, code boxes, B boxes issued
    const int64_t s_off0 = MODE == 1 ? L.scales_off[2] : L.scales_off[0];
    const int64_t b_off0 = MODE == 1 ? L.biases_off[2] : L.biases_off[0];
    GemmTile t{};
    if (my_tiles > 0) {
      t = tw.at(rv, tile_start, nseg, m_tiles, BN, blockIdx.x);
      tile_rows[0] = t.rows;
    }
    for (int j = 0; j < my_tiles; ++j) {
      GemmTile tn{};
      if (j + 1 < my_tiles) tn = tw.at(rv, tile_start, nseg, m_tiles, BN, blockIdx.x + (j + 1) * gridDim.x);
      if (t.slot < 0 && t.local == 0) atomicAdd(rv.err, 1);
      const int slot = t.slot >= 0 ? t.slot : 0;     // a missing expert's tiles read slot 0;
                                                     // the epilogue writes zeros for them
      const uint8_t* base = slab + static_cast<int64_t>(slot) * L.slot_stride;
      // this tile's scale and bias blocks: rows [m0, m0 + rows) are contiguous
      const int sb = j % NSB;
      GG_T(t16);
      if (!mbar_wait(&sc_empty[sb], ((j / NSB) & 1) ^ 1, abort_flag, rv.err, 8)) break;
      GG_ADD(16, t16);
      const uint32_t rows = static_cast<uint32_t>(min(kBlockM, NF - t.m0));
      const uint32_t blk = rows * gpitch * 2;          // a multiple of 128: rows % 64 == 0
      bar_expect_tx(&sc_full[sb], NMAT * 2 * blk);
      ++ns;
      uint8_t* sdst = sc_ring + sb * rg.sc_bytes;
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const int64_t so = (MODE == 1 ? s_off0 : m ? L.scales_off[1] : s_off0) + int64_t(t.m0) * gpitch * 2;
        const int64_t bo = (MODE == 1 ? b_off0 : m ? L.biases_off[1] : b_off0) + int64_t(t.m0) * gpitch * 2;
        bulk_g2s(sdst + (m * 2) * sc_half, base + so, blk, &sc_full[sb]);
        bulk_g2s(sdst + (m * 2 + 1) * sc_half, base + bo, blk, &sc_full[sb]);
      }
      bool ok = true;
      for (int kit = 0; kit < k_iters && ok; ++kit) {
        if ((kit * KS) % F == 0) {
          GG_T(t17);
          if (!mbar_wait(&code_empty[cr.slot], cr.phase ^ 1, abort_flag, rv.err, 9)) { ok = false; break; }
          GG_ADD(17, t17);
          bar_expect_tx(&code_full[cr.slot], NMAT * G::CODE_BOX);
          const uint32_t dst = smem_u32(code_ring + cr.slot * G::CODE_SLOT);
          const int x = kit * KS * G::ROW_BYTES;
          tma_load_3d(dst, &tm_code0, x, t.m0, slot, smem_u32(&code_full[cr.slot]));
          if (NMAT == 2)
            tma_load_3d(dst + G::CODE_BOX, &tm_code1, x, t.m0, slot, smem_u32(&code_full[cr.slot]));
          cr.next(RS);
          ++nc;
        }
        // the next tile's width goes out before this tile's last token rows: the MMA lane
        // reads it after the handoff of that iteration
        if (kit == k_iters - 1 && j + 1 < my_tiles) tile_rows[(j + 1) & 7] = tn.rows;
        GG_T(t18);
        if (!mbar_wait(G::SPLIT_B ? &b_empty[sr.slot] : &s_empty[sr.slot], sr.phase ^ 1, abort_flag,
                       rv.err, 10)) { ok = false; break; }
        GG_ADD(18, t18);
        const int steps = min(KS, k_steps - kit * KS);
        bar_expect_tx(&b_full[sr.slot], steps * G::B_BOX);
        for (int st = 0; st < steps; ++st)
          tma_load_2d(smem_u32(b_ring + sr.slot * G::B_BYTES + st * G::B_BOX), &tm_act,
                      (kit * KS + st) * kBlockK, t.row0 + t.n0, smem_u32(&b_full[sr.slot]));
        sr.next(SB);
        ++nb;
        GG_INC(19);
      }
      if (!ok) break;
      t = tn;
    }
    // every copy issued must land before the CTA's shared memory goes away (after an
    // abort its consumers may never have waited for it): wait for the last use of each
    // slot, bounded
    auto drain = [&](uint64_t* bars, int n_issued, int n_slots) {
      for (int f = max(0, n_issued - n_slots); f < n_issued; ++f) {
        uint32_t n = 0;
        while (!mbar_try_wait(&bars[f % n_slots], (f / n_slots) & 1) && ++n < kSpinLimit) {
        }
      }
    };
    drain(sc_full, ns, NSB);
    drain(code_full, nc, RS);
    drain(b_full, nb, SB);
  }

#ifdef BIGRIG_GEMM_PROFILE
  GG_ADD(15, t_kernel);
  if (threadIdx.x == 0 || threadIdx.x == kProducerThreads || threadIdx.x == kMmaWarp * 32 ||
      threadIdx.x == kLoaderWarp * 32) {
    unsigned long long* g = g_gemm_prof + MODE * 32;
    for (int i = 0; i < 32; ++i)       // the four roles fill disjoint phase slots
      if (prof[i] && i != 15) atomicAdd(&g[i], static_cast<unsigned long long>(prof[i]));
    if (threadIdx.x == 0) atomicAdd(&g[15], static_cast<unsigned long long>(prof[15]));
    if (threadIdx.x == 0) atomicAdd(&g[31], 1ull);
  }
#endif
  // drain: every MMA this CTA issued must complete before TMEM is released.  On the
  // normal path the epilogue already waited for them; after an abort they may still
  // be in flight, so the issuing thread commits once more and waits (bounded).
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    if (*abort_flag) {
      if (lane == 0) mma_commit(drain_bar);
      __syncwarp();
      uint32_t n = 0;
      while (!mbar_try_wait(drain_bar, 0) && ++n < kSpinLimit) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem, G::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launchers
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// A tiled map of `rank` dimensions (innermost first), 128-byte swizzle, zero fill.
static bool encode_map(CUtensorMap* m, CUtensorMapDataType dt, cuuint32_t rank, const void* base,
                       const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, rank, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// launch_one's answer when the rings for this token tile and K do not fit in shared
// memory (not an error: a smaller tile may fit).
constexpr int kNoFit = 1 << 20;

// Slots a code map may address: the slab's extent is not passed in, and a TMA box only
// touches the slot it is given.
constexpr cuuint64_t kMapSlots = 1u << 16;

template <int MODE, int BN, int BITS, int SDT>
static int launch_one(const void* act, const RouteView& rv, const void* slab,
                      const bigrig_expert_layout& L, void* out, cudaStream_t s, int sms) {
  using G = GemmShape<MODE, BN, BITS>;
  const int K = MODE != 1 ? L.hidden : L.inter, NF = MODE != 1 ? L.inter : L.hidden;
  const int gpitch = K / L.group_size;
  GemmRings rg{0, 0, 0, (G::NMAT * 2 * kBlockM * gpitch * 2 + 127) & ~127};
  // (code slots, scale buffers) from the most buffered; a split token-row ring as deep as
  // fits beside them (at least 4), an unsplit one has the A slots' depth
  static const int prefs[][2] = {{3, 2}, {2, 2}, {3, 1}, {2, 1}};
  for (const auto& c : prefs) {
    for (int sb = G::SB; sb >= (G::SPLIT_B ? 4 : G::SB); --sb)
      if (G::smem(c[0], sb, c[1], rg.sc_bytes) <= static_cast<size_t>(G::kLimit)) {
        rg.rs = c[0]; rg.sb = sb; rg.nsb = c[1];
        break;
      }
    if (rg.rs) break;
  }
  if (!rg.rs) return kNoFit;                          // the caller tries a smaller token tile
  const size_t smem = G::smem(rg.rs, rg.sb, rg.nsb, rg.sc_bytes);

  CUtensorMap tm[3];
  // gate/up: gate and up; down: down; fc1 (MODE 2, plain experts): projection 0
  const int projs[2] = {MODE == 1 ? 2 : 0, MODE == 0 ? 1 : MODE == 1 ? 2 : 0};
  for (int i = 0; i < 2; ++i) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(K) * BITS / 8, static_cast<cuuint64_t>(NF), kMapSlots};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K) * BITS / 8, static_cast<cuuint64_t>(L.slot_stride)};
    const cuuint32_t box[3] = {128, kBlockM, 1};
    if (!encode_map(&tm[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3,
                    static_cast<const uint8_t*>(slab) + L.weight_off[projs[i]], dims, strides, box))
      return set_error(BIGRIG_ERR_CUDA, "grouped_gemm: cannot encode the code tensor map");
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rv.P)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {kBlockK, BN};         // one step's rows (G::B_BOX bytes)
    if (!encode_map(&tm[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, act, dims, strides, box))
      return set_error(BIGRIG_ERR_CUDA, "grouped_gemm: cannot encode the token tensor map");
  }
  auto kern = grouped_gemm_kernel<MODE, BN, BITS, SDT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "grouped_gemm: cannot reserve %zu bytes of smem", smem);
  TimedLaunch tl(MODE != 1 ? BIGRIG_K_GEMM_GATE_UP : BIGRIG_K_GEMM_DOWN, s);
  kern<<<sms, kThreads, smem, s>>>(tm[0], tm[1], tm[2], rv, static_cast<const uint8_t*>(slab), L, rg,
                                   static_cast<uint16_t*>(out));
  return check_launch(MODE == 0 ? "grouped_gemm_gate_up" : MODE == 1 ? "grouped_gemm_down"
                                                                     : "grouped_gemm_fc1");
}

template <int MODE, int BN>
static int dispatch_fmt(const void* act, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* out, cudaStream_t s, int sms) {
  if (L.bits == 4 && L.scale_dtype == BIGRIG_F16) return launch_one<MODE, BN, 4, BIGRIG_F16>(act, rv, slab, L, out, s, sms);
  if (L.bits == 4 && L.scale_dtype == BIGRIG_BF16) return launch_one<MODE, BN, 4, BIGRIG_BF16>(act, rv, slab, L, out, s, sms);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_F16) return launch_one<MODE, BN, 8, BIGRIG_F16>(act, rv, slab, L, out, s, sms);
  if (L.bits == 8 && L.scale_dtype == BIGRIG_BF16) return launch_one<MODE, BN, 8, BIGRIG_BF16>(act, rv, slab, L, out, s, sms);
  return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: bits=%d scale_dtype=%d", L.bits, L.scale_dtype);
}

}  // namespace sm100

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

// Mean rows per routed expert; each pass picks its token tile from it.
int gemm_mean_rows(int T, int k, int E) { return (T * k + E - 1) / E; }

// Token tile of a pass: the smallest offered that covers 1.25x the mean rows, so most
// experts take one slice (or the fewest equal slices) per feature tile.  Tiles stop at
// 160 columns: gate/up's one accumulator of 2 x 160 plus the A slots fill TMEM, and
// down keeps two accumulators (the epilogue of one tile overlaps the next one's MMAs).
// When the rings of that tile do not fit in shared memory for this K (large K means
// large per-tile scale blocks), the next smaller tile is used.
static int pick_tile(int mean, const int* opts, int n) {
  const int want = (mean * 5 + 3) / 4;
  for (int i = 0; i < n; ++i)
    if (opts[i] >= want) return i;
  return n - 1;
}

int launch_gemm_gate_up(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, void* xs, int T, int mean_rows,
                        cudaStream_t s) {
  if (L.group_size % sm100::kBlockK)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: group_size must be a multiple of 64");
  (void)T;
  // the token operand as expert-sorted rows (and for 4-bit formats in the operand type
  // and K order of the dequantised weights)
  const int cpr = L.hidden / 8;
  const int64_t n = static_cast<int64_t>(rv.P) * cpr;
  if (n > 0) {
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * sm_count()));
    const uint4* xv = static_cast<const uint4*>(x);
    uint4* xsv = static_cast<uint4*>(xs);
    if (L.bits == 4 && L.scale_dtype == BIGRIG_F16)
      sm100::gather_rows_kernel<BIGRIG_F16, true><<<blocks, 256, 0, s>>>(xv, rv.order, rv.k, rv.P, cpr, xsv);
    else if (L.bits == 4)
      sm100::gather_rows_kernel<BIGRIG_BF16, true><<<blocks, 256, 0, s>>>(xv, rv.order, rv.k, rv.P, cpr, xsv);
    else
      sm100::gather_rows_kernel<BIGRIG_BF16, false><<<blocks, 256, 0, s>>>(xv, rv.order, rv.k, rv.P, cpr, xsv);
    if (int rc = check_launch("gather_rows")) return rc;
  }
  static const int opts[] = {32, 64, 96, 128, 160};
  const bool plain = L.flags & BIGRIG_LAYOUT_PLAIN;
  for (int i = pick_tile(mean_rows, opts, 5); i >= 0 && plain; --i) {
    // a plain expert's fc1: one matrix, h = act(fc1(x) + bias)
    int rc = sm100::kNoFit;
    switch (opts[i]) {
      case 32: rc = sm100::dispatch_fmt<2, 32>(xs, rv, slab, L, h, s, sm_count()); break;
      case 64: rc = sm100::dispatch_fmt<2, 64>(xs, rv, slab, L, h, s, sm_count()); break;
      case 96: rc = sm100::dispatch_fmt<2, 96>(xs, rv, slab, L, h, s, sm_count()); break;
      case 128: rc = sm100::dispatch_fmt<2, 128>(xs, rv, slab, L, h, s, sm_count()); break;
      case 160: rc = sm100::dispatch_fmt<2, 160>(xs, rv, slab, L, h, s, sm_count()); break;
    }
    if (rc != sm100::kNoFit) return rc;
  }
  for (int i = pick_tile(mean_rows, opts, 5); i >= 0 && !plain; --i) {
    int rc = sm100::kNoFit;
    switch (opts[i]) {
      case 32: rc = sm100::dispatch_fmt<0, 32>(xs, rv, slab, L, h, s, sm_count()); break;
      case 64: rc = sm100::dispatch_fmt<0, 64>(xs, rv, slab, L, h, s, sm_count()); break;
      case 96: rc = sm100::dispatch_fmt<0, 96>(xs, rv, slab, L, h, s, sm_count()); break;
      case 128: rc = sm100::dispatch_fmt<0, 128>(xs, rv, slab, L, h, s, sm_count()); break;
      case 160: rc = sm100::dispatch_fmt<0, 160>(xs, rv, slab, L, h, s, sm_count()); break;
    }
    if (rc != sm100::kNoFit) return rc;
  }
  return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: hidden=%d needs more shared memory than a CTA has",
                   L.hidden);
}

int launch_gemm_down(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, int mean_rows, cudaStream_t s) {
  if (L.group_size % sm100::kBlockK)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: group_size must be a multiple of 64");
  static const int opts[] = {32, 64, 128, 160};
  for (int i = pick_tile(mean_rows, opts, 4); i >= 0; --i) {
    int rc = sm100::kNoFit;
    switch (opts[i]) {
      case 32: rc = sm100::dispatch_fmt<1, 32>(h, rv, slab, L, y, s, sm_count()); break;
      case 64: rc = sm100::dispatch_fmt<1, 64>(h, rv, slab, L, y, s, sm_count()); break;
      case 128: rc = sm100::dispatch_fmt<1, 128>(h, rv, slab, L, y, s, sm_count()); break;
      case 160: rc = sm100::dispatch_fmt<1, 160>(h, rv, slab, L, y, s, sm_count()); break;
    }
    if (rc != sm100::kNoFit) return rc;
  }
  return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: inter=%d needs more shared memory than a CTA has",
                   L.inter);
}

}  // namespace bigrig

#ifdef BIGRIG_GEMM_PROFILE
extern "C" BIGRIG_API int bigrig_gemm_prof_read(unsigned long long* out) {
  if (cudaMemcpyFromSymbol(out, bigrig::sm100::g_gemm_prof, sizeof(unsigned long long) * 64) !=
      cudaSuccess)
    return 1;
  static const unsigned long long zero[64] = {};
  return cudaMemcpyToSymbol(bigrig::sm100::g_gemm_prof, zero, sizeof(zero)) != cudaSuccess;
}
#endif
