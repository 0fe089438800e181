// Expert parallelism over peer memory: the exchange steps of bigrig_peer_layer.
//
// The reference has no distributed code (it runs on one Mac); this is the B200 design's
// shard of its MoE layer across the GPUs of one NVSwitch node.  Every rank owns one
// buffer (PeerLayout) that all ranks map through CUDA IPC; these kernels move rows
// between those buffers with plain 16-byte stores over NVLink and order them with
// 64-bit flags: release stores at system scope after the data, acquire loads before
// reading it.  The steps between them (router, experts) are the library's own kernels.
//
//   peer_gather_kernel    one CTA: this rank's rows into every rank's gathered rows,
//                         a flag at each; then wait until every rank's flag has arrived
//                         here.  It also advances the layer counter whose value the
//                         flags carry (each call of every rank raises them to the same
//                         count, so a stale flag never satisfies a newer wait).
//   peer_localize_kernel  global expert ids -> this rank's expert numbering, -1 for the
//                         pairs another rank owns (padding for the expert kernels).
//   peer_scatter_kernel   CTA d: the output rows of the pairs of rank d's tokens that
//                         this rank computed, stored at their (token, k) places in rank
//                         d's buffer; then rank d's flag for this rank.
//   peer_combine_kernel   wait for every rank's scatter flag; out = residual +
//                         sum_j score * y in k order (combine_kernel's arithmetic).
//
// Why no write-after-read hazard needs a second buffer: rank r overwrites rank p's
// gathered rows (next layer) only after r's combine saw p's scatter flag of this layer,
// which p raises after its expert kernels (the readers of those rows) finished; and r
// overwrites p's pair outputs only after r's gather saw p's flag of the next layer,
// which p raises after its combine (their reader) finished.
//
// The three are launched with programmatic dependent launch: each may be scheduled while
// the kernel before it finishes, and waits for that kernel (griddepcontrol.wait) before it
// touches anything -- so a flag it polls is only ever raised by another GPU or by a kernel
// that has already completed.
//
// Waits are bounded by the GPU's global timer; a wait that runs out counts in the
// group's error word and every later wait returns at once until the host clears it,
// so a rank that stopped (or a peer that never came) costs each other rank one bounded
// wait, never a hang.
#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "routing.cuh"

namespace bigrig {

namespace {

constexpr int kPeerThreads = 512;
constexpr uint64_t kPeerWaitDefaultMs = 10000;    // per wait, when the group sets none

struct PeerArgs {
  int world, rank, tokens, hidden, k;
  uint64_t wait_ns;
  PeerLayout lay;
  uint8_t* base[BIGRIG_PEER_MAX_RANKS];
};

PeerArgs peer_args(const bigrig_peer_group& g) {
  PeerArgs a;
  a.world = g.world;
  a.rank = g.rank;
  a.tokens = g.tokens;
  a.hidden = g.hidden;
  a.k = g.top_k;
  a.wait_ns = (g.wait_ms > 0 ? static_cast<uint64_t>(g.wait_ms) : kPeerWaitDefaultMs) * 1000000ull;
  a.lay = peer_layout(g.world, g.tokens, g.hidden, g.top_k);
  for (int i = 0; i < BIGRIG_PEER_MAX_RANKS; ++i)
    a.base[i] = i < g.world ? static_cast<uint8_t*>(g.base[i]) : nullptr;
  return a;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t* flag_at(const PeerArgs& a, int owner, size_t off, int slot) {
  return reinterpret_cast<uint64_t*>(a.base[owner] + off) + slot;
}

__device__ __forceinline__ uint64_t* ctrl_of(const PeerArgs& a) {
  return reinterpret_cast<uint64_t*>(a.base[a.rank] + a.lay.ctrl);
}

__device__ __forceinline__ int32_t* err_of(const PeerArgs& a) {
  return reinterpret_cast<int32_t*>(a.base[a.rank] + a.lay.ctrl + 8);
}

// Wait until *flag >= want; false after the time limit (counted in err) or at once when
// the group has already failed.
__device__ bool peer_wait(const uint64_t* flag, uint64_t want, int32_t* err, uint64_t limit_ns) {
  if (*reinterpret_cast<volatile int32_t*>(err) != 0) return false;
  const uint64_t t0 = global_ns();
  while (ld_acquire_sys(flag) < want) {
    if (global_ns() - t0 > limit_ns) {
      atomicAdd(err, 1);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Raise `flag` (in any rank's buffer) to `v` after every thread of the CTA has issued its
// stores: the barrier before the call orders them before this thread's system-scope fence
// and release.
__device__ __forceinline__ void peer_signal(uint64_t* flag, uint64_t v) {
  __threadfence_system();
  st_release_sys(flag, v);
}

__global__ void __launch_bounds__(kPeerThreads) peer_gather_kernel(PeerArgs a,
                                                                   const uint4* __restrict__ x) {
  __shared__ uint64_t s_layer;
  pdl_wait();
  pdl_trigger();
  uint64_t* ctrl = ctrl_of(a);
  if (threadIdx.x == 0) s_layer = ctrl[0] + 1;
  __syncthreads();
  const uint64_t layer = s_layer;
  const int nvec = a.tokens * a.hidden / 8;                 // 16-byte vectors of our rows
  const size_t at = a.lay.xin + static_cast<size_t>(a.rank) * a.tokens * a.hidden * 2;
  for (int d = 0; d < a.world; ++d) {
    uint4* dst = reinterpret_cast<uint4*>(a.base[d] + at);
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) dst[i] = x[i];
  }
  __syncthreads();
  if (threadIdx.x < a.world) {
    peer_signal(flag_at(a, threadIdx.x, a.lay.gflag, a.rank), layer);
    peer_wait(flag_at(a, a.rank, a.lay.gflag, threadIdx.x), layer, err_of(a), a.wait_ns);
  }
  __syncthreads();
  if (threadIdx.x == 0) ctrl[0] = layer;
}

__global__ void peer_localize_kernel(const int32_t* __restrict__ idx, int P, int first, int n_local,
                                     int32_t* __restrict__ idx_local) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p < P) {
    const int e = idx[p];
    idx_local[p] = (e >= first && e < first + n_local) ? e - first : -1;
  }
}

__global__ void __launch_bounds__(kPeerThreads) peer_scatter_kernel(
    PeerArgs a, const uint4* __restrict__ y, const int32_t* __restrict__ idx_local) {
  const int d = blockIdx.x;                                  // destination rank
  pdl_wait();
  pdl_trigger();
  const uint64_t layer = ctrl_of(a)[0];
  const int per = a.tokens * a.k;                            // pairs of rank d's tokens
  const int vpr = a.hidden / 8;                              // 16-byte vectors per row
  uint4* dst = reinterpret_cast<uint4*>(a.base[d] + a.lay.ybuf);
  const size_t p0 = static_cast<size_t>(d) * per;
  for (int i = threadIdx.x; i < per * vpr; i += blockDim.x) {
    const int q = i / vpr, v = i - q * vpr;
    if (idx_local[p0 + q] >= 0) dst[static_cast<size_t>(q) * vpr + v] = y[(p0 + q) * vpr + v];
  }
  __syncthreads();
  if (threadIdx.x == 0) peer_signal(flag_at(a, d, a.lay.pflag, a.rank), layer);
}

// grid (ceil(H / 2 / threads), tokens); each thread two adjacent features of one row
__global__ void __launch_bounds__(256) peer_combine_kernel(PeerArgs a,
                                                           const float* __restrict__ scores,
                                                           const uint16_t* __restrict__ residual,
                                                           uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const uint64_t layer = ctrl_of(a)[0];
  if (threadIdx.x < a.world)
    peer_wait(flag_at(a, a.rank, a.lay.pflag, threadIdx.x), layer, err_of(a), a.wait_ns);
  __syncthreads();
  const int t = blockIdx.y, H = a.hidden, k = a.k;
  const int f = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (f >= H) return;
  const float* sc = scores + (static_cast<size_t>(a.rank) * a.tokens + t) * k;
  const uint16_t* yb = reinterpret_cast<const uint16_t*>(a.base[a.rank] + a.lay.ybuf) +
                       static_cast<size_t>(t) * k * H;
  float a0 = 0.f, a1 = 0.f;
  for (int j = 0; j < k; ++j) {
    const float s = sc[j];
    const uint32_t v = __ldcg(reinterpret_cast<const unsigned int*>(yb + static_cast<size_t>(j) * H + f));
    a0 = a0 + s * __uint_as_float(v << 16);
    a1 = a1 + s * __uint_as_float(v & 0xffff0000u);
  }
  if (residual) {
    const uint32_t r = *reinterpret_cast<const uint32_t*>(residual + static_cast<size_t>(t) * H + f);
    a0 = __uint_as_float(r << 16) + bf16_round(a0);
    a1 = __uint_as_float(r & 0xffff0000u) + bf16_round(a1);
  }
  *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(t) * H + f) =
      static_cast<uint32_t>(f32_to_bf16_bits(a0)) | (static_cast<uint32_t>(f32_to_bf16_bits(a1)) << 16);
}

}  // namespace

// A launch that may start while the previous kernel on the stream finishes (the kernel
// itself waits for it with griddepcontrol.wait before touching memory).
template <typename... KArgs, typename... Args>
static int launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                            const char* name, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  return check_launch(name);
}

int launch_peer_gather(const bigrig_peer_group& g, const void* x, cudaStream_t s) {
  TimedLaunch tl(BIGRIG_K_PEER_GATHER, s);
  return launch_dependent(peer_gather_kernel, dim3(1), dim3(kPeerThreads), s, "peer_gather_kernel",
                          peer_args(g), static_cast<const uint4*>(x));
}

int launch_peer_localize(const int32_t* idx, int P, int first, int n_local, int32_t* idx_local,
                         cudaStream_t s) {
  TimedLaunch tl(BIGRIG_K_PEER_LOCALIZE, s);
  peer_localize_kernel<<<(P + 255) / 256, 256, 0, s>>>(idx, P, first, n_local, idx_local);
  return check_launch("peer_localize_kernel");
}

int launch_peer_scatter(const bigrig_peer_group& g, const void* y, const int32_t* idx_local,
                        cudaStream_t s) {
  TimedLaunch tl(BIGRIG_K_PEER_SCATTER, s);
  return launch_dependent(peer_scatter_kernel, dim3(g.world), dim3(kPeerThreads), s,
                          "peer_scatter_kernel", peer_args(g), static_cast<const uint4*>(y),
                          idx_local);
}

int launch_peer_combine(const bigrig_peer_group& g, const float* scores, const void* residual,
                        void* out, cudaStream_t s) {
  TimedLaunch tl(BIGRIG_K_PEER_COMBINE, s);
  const dim3 grid((g.hidden / 2 + 255) / 256, g.tokens);
  return launch_dependent(peer_combine_kernel, grid, dim3(256), s, "peer_combine_kernel",
                          peer_args(g), scores, static_cast<const uint16_t*>(residual),
                          static_cast<uint16_t*>(out));
}

}  // namespace bigrig

using namespace bigrig;

extern "C" {

size_t bigrig_peer_buffer_bytes(int world, int tokens, int hidden, int top_k) {
  if (world < 1 || world > BIGRIG_PEER_MAX_RANKS || tokens < 1 || hidden < 8 || top_k < 1)
    return 0;
  return peer_layout(world, tokens, hidden, top_k).total;
}

int bigrig_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return set_error(BIGRIG_ERR_INVALID, "peer_alloc: bad argument");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    cudaGetLastError();
    return set_error(BIGRIG_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return BIGRIG_OK;
}

int bigrig_peer_free(void* ptr) {
  if (!ptr) return BIGRIG_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(BIGRIG_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
  return BIGRIG_OK;
}

int bigrig_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return set_error(BIGRIG_ERR_INVALID, "peer_open: NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(BIGRIG_ERR_CUDA, "peer_open: %s", cudaGetErrorString(e));
  }
  return BIGRIG_OK;
}

int bigrig_peer_close(void* ptr) {
  if (!ptr) return BIGRIG_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(BIGRIG_ERR_CUDA, "peer_close: %s", cudaGetErrorString(e));
  return BIGRIG_OK;
}

int bigrig_peer_errors(const bigrig_peer_group* g, int32_t* out, void* stream) {
  if (!g || !out || g->rank < 0 || g->rank >= g->world || !g->base[g->rank])
    return set_error(BIGRIG_ERR_INVALID, "peer_errors: bad group");
  const PeerLayout lay = peer_layout(g->world, g->tokens, g->hidden, g->top_k);
  int32_t* word = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(g->base[g->rank]) + lay.ctrl + 8);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, word, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(word, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return set_error(BIGRIG_ERR_CUDA, "peer_errors: %s", cudaGetErrorString(e));
  return BIGRIG_OK;
}

}  // extern "C"
