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
// are the N dimension (a multiple of 16 up to 256).  Both operands are K-major
// bf16 tiles of 64 K-elements in 128-byte-swizzled shared memory, one swizzle
// atom per 8 rows, so each of the four K=16 MMAs of a stage starts 32 bytes
// further into the atom.
//
// Warp roles in a CTA of 288 threads, persistent over (expert, feature tile,
// token tile) work items:
//   warps 0-7  producers: load codes, scales, biases, dequantise
//              w = bf16(f32(scale) * q + f32(bias)) in registers and store the A
//              tile; gather the routed token rows (B tile); fence the generic
//              proxy against the async proxy; arrive on the stage's full barrier.
//              Warps 0-3 then run the epilogue from TMEM (lane quarter = warp).
//   warp 8     MMA issuer: one elected lane waits for a full stage, issues
//              tcgen05.mma, and commits the stage back to its empty barrier and
//              the finished tile to the accumulator barrier.
// Every mbarrier wait is bounded: past the limit the CTA records an error,
// raises a shared abort flag so every other wait returns at once, drains the
// MMAs it issued, frees its TMEM and returns.
#include "gemv_common.cuh"

namespace bigrig {
namespace sm100 {

constexpr int kProducerWarps = 8;
constexpr int kThreads = (kProducerWarps + 1) * 32;
constexpr int kBlockM = 128;
constexpr int kBlockK = 64;                 // one 128-byte swizzle atom of bf16 per row
constexpr int kATile = kBlockM * kBlockK * 2;
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

// Bounded wait on phase `parity`.  Returns false when the CTA is aborting.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* err, int where) {
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
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

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
  return (1u << 4)                                   // D format f32
         | (1u << 7)                                 // A format bf16
         | (1u << 10)                                // B format bf16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N
         | (static_cast<uint32_t>(M >> 4) << 24);    // M
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

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
template <int BITS>
__device__ __forceinline__ void dequant_chunk(uint8_t* tile, int row, int jbase, uint4 w, float s,
                                              float b) {
  constexpr float M = 8388608.f;
  constexpr uint32_t E23 = 0x4B000000u;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  if constexpr (BITS == 4) {
    const float s1 = s * 0.0625f, s2 = s * 0.00390625f, s3 = s * 0.000244140625f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {          // word i: codes 8i..8i+7 -> 16 bytes of bf16
      const uint32_t lo = ws[i], hi = ws[i] >> 16;
      const float q0 = __uint_as_float((lo & 0x000Fu) | E23) - M;
      const float q1 = __uint_as_float((lo & 0x00F0u) | E23) - M;
      const float q2 = __uint_as_float((lo & 0x0F00u) | E23) - M;
      const float q3 = __uint_as_float((lo & 0xF000u) | E23) - M;
      const float q4 = __uint_as_float((hi & 0x000Fu) | E23) - M;
      const float q5 = __uint_as_float((hi & 0x00F0u) | E23) - M;
      const float q6 = __uint_as_float((hi & 0x0F00u) | E23) - M;
      const float q7 = __uint_as_float((hi & 0xF000u) | E23) - M;
      uint4 o;
      o.x = pack_bf16x2(fmaf(s, q0, b), fmaf(s1, q1, b));
      o.y = pack_bf16x2(fmaf(s2, q2, b), fmaf(s3, q3, b));
      o.z = pack_bf16x2(fmaf(s, q4, b), fmaf(s1, q5, b));
      o.w = pack_bf16x2(fmaf(s2, q6, b), fmaf(s3, q7, b));
      *reinterpret_cast<uint4*>(tile + swz(row, jbase + i)) = o;
    }
  } else {
    const float s1 = s * 0.00390625f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {          // words 2i, 2i+1: 8 codes -> 16 bytes
      const uint32_t a = ws[2 * i], c = ws[2 * i + 1];
      uint4 o;
      o.x = pack_bf16x2(fmaf(s, __uint_as_float((a & 0x00FFu) | E23) - M, b),
                        fmaf(s1, __uint_as_float((a & 0xFF00u) | E23) - M, b));
      o.y = pack_bf16x2(fmaf(s, __uint_as_float(((a >> 16) & 0x00FFu) | E23) - M, b),
                        fmaf(s1, __uint_as_float(((a >> 16) & 0xFF00u) | E23) - M, b));
      o.z = pack_bf16x2(fmaf(s, __uint_as_float((c & 0x00FFu) | E23) - M, b),
                        fmaf(s1, __uint_as_float((c & 0xFF00u) | E23) - M, b));
      o.w = pack_bf16x2(fmaf(s, __uint_as_float(((c >> 16) & 0x00FFu) | E23) - M, b),
                        fmaf(s1, __uint_as_float(((c >> 16) & 0xFF00u) | E23) - M, b));
      *reinterpret_cast<uint4*>(tile + swz(row, jbase + i)) = o;
    }
  }
}

// ------------------------------------------------------------------ the kernel
// MODE 0: gate/up (two weight matrices, output h); MODE 1: down (one matrix, output y).
template <int MODE, int BN, int BITS, int SDT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(
    const uint16_t* __restrict__ act,   // MODE 0: x [T, H]; MODE 1: h [P, I] (sorted rows)
    RouteView rv, const uint8_t* __restrict__ slab, bigrig_expert_layout L,
    uint16_t* __restrict__ out) {       // MODE 0: h [P, I]; MODE 1: y [P, H] ((token, k) order)
  constexpr int NMAT = MODE == 0 ? 2 : 1;
  constexpr int BTILE = BN * kBlockK * 2;
  constexpr int STAGE_BYTES = NMAT * kATile + BTILE;
  constexpr int TMEM_COLS = (NMAT * BN) <= 32 ? 32 : (NMAT * BN) <= 64 ? 64 : (NMAT * BN) <= 128 ? 128 : (NMAT * BN) <= 256 ? 256 : 512;
  constexpr int CHUNKS_PER_ROW = kBlockK * BITS / 128;        // 16-byte code chunks per row per stage
  constexpr int CODES_PER_CHUNK = 128 / BITS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accum_full = empty_bar + STAGES;
  uint64_t* accum_empty = accum_full + 1;
  uint64_t* drain_bar = accum_empty + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);
  int* tile_start = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_base_s + 2));  // [S+1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = MODE == 0 ? L.hidden : L.inter;        // reduction length
  const int NF = MODE == 0 ? L.inter : L.hidden;       // output features
  const int m_tiles = (NF + kBlockM - 1) / kBlockM;
  const int k_iters = K / kBlockK;
  const int nseg = min(min(*rv.num_seg, rv.s_max), kMaxExperts);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], kProducerWarps * 32);
      mbar_init(&empty_bar[i], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(accum_empty, 4);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // tile prefix over segments: segment s owns m_tiles * ceil(R_s / BN) work items
  if (warp == 0) {
    if (lane == 0) {
      int acc = 0;
      for (int s = 0; s < nseg; ++s) {
        tile_start[s] = acc;
        int row0, R;
        segment_slot(rv, s, row0, R);      // R = 0 for inconsistent metadata: no tiles
        acc += m_tiles * ((R + BN - 1) / BN);
      }
      tile_start[nseg] = acc;
    }
  }
  if (warp == kProducerWarps) tmem_alloc(tmem_base_s, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  const int total = tile_start[nseg];

  if (warp < kProducerWarps) {
    // ---------------------------------------------------------------- producers (+ epilogue)
    const int ptid = threadIdx.x;             // 0..255
    uint32_t stage = 0, phase = 0, accum_phase = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      int s = 0;
      while (s + 1 < nseg && tile_start[s + 1] <= tile) ++s;
      const int local = tile - tile_start[s];
      int row0, R;
      const int slot = segment_slot(rv, s, row0, R);
      const int n_tiles = (R + BN - 1) / BN;
      const int mt = local / n_tiles, nt = local - mt * n_tiles;
      const int m0 = mt * kBlockM, n0 = nt * BN;
      const bool valid_slot = slot >= 0;
      if (!valid_slot && ptid == 0 && mt == 0 && nt == 0) atomicAdd(rv.err, 1);
      const uint8_t* base = slab + static_cast<int64_t>(valid_slot ? slot : 0) * L.slot_stride;
      const int64_t code_pitch = static_cast<int64_t>(K) * BITS / 8;
      const int gpitch = K / L.group_size;
      // token rows of this tile this thread gathers (B operand): chunk c = ptid + 256*i
      for (int kit = 0; kit < k_iters; ++kit) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, rv.err, 1)) break;
        uint8_t* st = tiles + stage * STAGE_BYTES;
        const int k0 = kit * kBlockK;
        const int grp = k0 / L.group_size;
        // A tiles: NMAT x 128 rows x CHUNKS_PER_ROW chunks
        for (int job = ptid; job < NMAT * kBlockM * CHUNKS_PER_ROW; job += kProducerWarps * 32) {
          const int mat = job / (kBlockM * CHUNKS_PER_ROW);
          const int rem = job - mat * kBlockM * CHUNKS_PER_ROW;
          const int r = rem / CHUNKS_PER_ROW, ch = rem - r * CHUNKS_PER_ROW;
          const int f = m0 + r;
          const int proj = MODE == 0 ? mat : 2;
          uint8_t* atile = st + mat * kATile;
          const int jbase = ch * (CODES_PER_CHUNK * 2 / 16);
          if (f < NF && valid_slot) {
            const uint8_t* codes = base + L.weight_off[proj] + f * code_pitch + (k0 * BITS / 8) + ch * 16;
            const uint4 w = ld_stream_v4(codes);
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + L.scales_off[proj]);
            const uint16_t* bi = reinterpret_cast<const uint16_t*>(base + L.biases_off[proj]);
            const float sv = half_to_f32<SDT>(ld_nc_u16(sc + static_cast<int64_t>(f) * gpitch + grp));
            const float bv = half_to_f32<SDT>(ld_nc_u16(bi + static_cast<int64_t>(f) * gpitch + grp));
            dequant_chunk<BITS>(atile, r, jbase, w, sv, bv);
          } else {
#pragma unroll
            for (int j = 0; j < CODES_PER_CHUNK * 2 / 16; ++j)
              *reinterpret_cast<uint4*>(atile + swz(r, jbase + j)) = make_uint4(0, 0, 0, 0);
          }
        }
        // B tile: BN token rows x 8 chunks of 16 bytes
        uint8_t* btile = st + NMAT * kATile;
        for (int c = ptid; c < BN * 8; c += kProducerWarps * 32) {
          const int r = c >> 3, j = c & 7;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (n0 + r < R) {
            const int p = row0 + n0 + r;
            const int64_t src_row = MODE == 0 ? (rv.order[p] / rv.k) : p;
            v = *reinterpret_cast<const uint4*>(act + src_row * K + k0 + j * 8);
          }
          *reinterpret_cast<uint4*>(btile + swz(r, j)) = v;
        }
        fence_proxy_async();               // generic-proxy stores -> visible to the tensor core
        mbar_arrive(&full_bar[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (*abort_flag) break;
      // ---------------------------------------------------------------- epilogue (warps 0-3)
      if (warp < 4) {
        if (!mbar_wait(accum_full, accum_phase, abort_flag, rv.err, 2)) break;
        tc_fence_after();
        const int f = m0 + warp * 32 + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        for (int j0 = 0; j0 < BN; j0 += 8) {
          if (n0 + j0 >= R) break;
          float a[8], u[8];
          tmem_ld8(lane_addr + j0, a);
          if (MODE == 0) tmem_ld8(lane_addr + BN + j0, u);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int row = n0 + j0 + i;
            if (row < R && f < NF && valid_slot) {
              const int p = row0 + row;
              if (MODE == 0) {
                out[static_cast<int64_t>(p) * NF + f] = f32_to_bf16_bits(silu_f32(a[i]) * u[i]);
              } else {
                out[static_cast<int64_t>(rv.order[p]) * NF + f] = f32_to_bf16_bits(a[i]);
              }
            } else if (row < R && f < NF) {
              const int p = row0 + row;
              const int64_t o = MODE == 0 ? static_cast<int64_t>(p) : rv.order[p];
              out[o * NF + f] = 0;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accum_empty);
        accum_phase ^= 1;
      }
    }
  } else {
    // ---------------------------------------------------------------- MMA issuer (warp 8)
    uint32_t stage = 0, phase = 0, accum_phase = 0;
    constexpr uint32_t idesc = instr_desc(kBlockM, BN);
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      // the previous tile's epilogue must have drained the accumulators
      if (!mbar_wait(accum_empty, accum_phase ^ 1, abort_flag, rv.err, 3)) break;
      tc_fence_after();
      for (int kit = 0; kit < k_iters; ++kit) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, rv.err, 4)) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = smem_u32(tiles + stage * STAGE_BYTES);
          const uint32_t bst = st + NMAT * kATile;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t db = smem_desc(bst + kk * 32);
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
              const uint64_t da = smem_desc(st + mat * kATile + kk * 32);
              mma_bf16(tmem + mat * BN, da, db, idesc, (kit > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty_bar[stage]);
          if (kit == k_iters - 1) mma_commit(accum_full);
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (*abort_flag) break;
      accum_phase ^= 1;
    }
  }

  // drain: every MMA this CTA issued must complete before TMEM is released.  On the
  // normal path the epilogue already waited for them; after an abort they may still
  // be in flight, so the issuing thread commits once more and waits (bounded).
  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarps) {
    if (*abort_flag) {
      if (lane == 0) mma_commit(drain_bar);
      __syncwarp();
      uint32_t n = 0;
      while (!mbar_try_wait(drain_bar, 0) && ++n < kSpinLimit) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launchers
template <int MODE, int BN, int BITS, int SDT>
static int launch_one(const void* act, const RouteView& rv, const void* slab,
                      const bigrig_expert_layout& L, void* out, cudaStream_t s, int sms) {
  constexpr int STAGES = MODE == 0 ? (BN <= 128 ? 4 : 3) : (BN <= 128 ? 6 : 4);
  constexpr int NMAT = MODE == 0 ? 2 : 1;
  constexpr int STAGE_BYTES = NMAT * kATile + BN * kBlockK * 2;
  const size_t smem = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 2 * STAGES * 8 + 24 + 16 +
                      (kMaxExperts + 1) * sizeof(int);
  auto kern = grouped_gemm_kernel<MODE, BN, BITS, SDT, STAGES>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "grouped_gemm: cannot reserve %zu bytes of smem", smem);
  TimedLaunch tl(MODE == 0 ? BIGRIG_K_GEMM_GATE_UP : BIGRIG_K_GEMM_DOWN, s);
  kern<<<sms, kThreads, smem, s>>>(static_cast<const uint16_t*>(act), rv,
                                   static_cast<const uint8_t*>(slab), L,
                                   static_cast<uint16_t*>(out));
  return check_launch(MODE == 0 ? "grouped_gemm_gate_up" : "grouped_gemm_down");
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

// Token tile: the smallest of 32/64/128/256 that covers the mean rows per expert.
int gemm_token_tile(int T, int k, int E) {
  const int mean = (T * k + E - 1) / E;
  return mean <= 32 ? 32 : mean <= 64 ? 64 : mean <= 128 ? 128 : 256;
}

int launch_gemm_gate_up(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, int bn, cudaStream_t s) {
  if (L.group_size % sm100::kBlockK)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: group_size must be a multiple of 64");
  switch (bn) {
    case 32: return sm100::dispatch_fmt<0, 32>(x, rv, slab, L, h, s, sm_count());
    case 64: return sm100::dispatch_fmt<0, 64>(x, rv, slab, L, h, s, sm_count());
    case 128: return sm100::dispatch_fmt<0, 128>(x, rv, slab, L, h, s, sm_count());
    case 256: return sm100::dispatch_fmt<0, 256>(x, rv, slab, L, h, s, sm_count());
  }
  return set_error(BIGRIG_ERR_INVALID, "grouped_gemm: token tile %d", bn);
}

int launch_gemm_down(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, int bn, cudaStream_t s) {
  if (L.group_size % sm100::kBlockK)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "grouped_gemm: group_size must be a multiple of 64");
  switch (bn) {
    case 32: return sm100::dispatch_fmt<1, 32>(h, rv, slab, L, y, s, sm_count());
    case 64: return sm100::dispatch_fmt<1, 64>(h, rv, slab, L, y, s, sm_count());
    case 128: return sm100::dispatch_fmt<1, 128>(h, rv, slab, L, y, s, sm_count());
    case 256: return sm100::dispatch_fmt<1, 256>(h, rv, slab, L, y, s, sm_count());
  }
  return set_error(BIGRIG_ERR_INVALID, "grouped_gemm: token tile %d", bn);
}

}  // namespace bigrig
