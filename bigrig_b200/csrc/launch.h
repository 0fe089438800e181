// Host-side launcher declarations shared by the translation units of the library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "bigrig_b200.h"

namespace bigrig {

// Record `msg` as the calling thread's last error and return `code`.
int set_error(int code, const char* fmt, ...);
// cudaGetLastError after a launch: 0, or BIGRIG_ERR_CUDA with the kernel name recorded.
int check_launch(const char* what);

// RAII bracket of one kernel launch with CUDA events when timing is enabled.
class TimedLaunch {
 public:
  TimedLaunch(int kernel_id, cudaStream_t s);
  ~TimedLaunch();
 private:
  int id_;
  cudaStream_t s_;
  void* start_;
};

int launch_router_logits(const void* x, const void* w, const float* bias, float* logits, int T,
                         int H, int E, cudaStream_t s);
int launch_router_topk(const void* logits, int dtype, int T, int E, int k, int mode, int norm,
                       int32_t* indices, float* scores, cudaStream_t s);
int launch_permute(const int32_t* indices, int P, int E, int32_t* order, int32_t* inv,
                   int32_t* offsets, int32_t* seg_expert, int32_t* seg_start, int32_t* num_seg,
                   int32_t* err, cudaStream_t s);

int launch_dequant(const void* slab, const bigrig_expert_layout& L, int slot, int proj, void* out,
                   cudaStream_t s);

// Grouped GEMV path (decode-sized calls): gate/up -> SiLU*mul into h (expert-sorted rows),
// then down written to y[t, j, :] at each pair's unpermuted position.
struct RouteView {
  const int32_t* order;      // [P] pair id at each sorted position
  const int32_t* inv;        // [P] sorted position of each pair
  const int32_t* seg_expert; // [S_max]
  const int32_t* seg_start;  // [S_max + 1]
  const int32_t* num_seg;    // [1]
  const int32_t* g2s;        // [E] expert -> slot, or nullptr for identity
  int32_t* err;              // [1] device error counter
  int P, k, s_max;
  int max_rows;              // largest number of rows one expert can receive (<= T)
  int n_experts;             // valid expert ids are [0, n_experts)
};

// Outputs of the routing step (see bigrig_moe_permute).
struct RouteOut {
  int32_t* order;
  int32_t* inv;
  int32_t* offsets;
  int32_t* seg_expert;
  int32_t* seg_start;
  int32_t* num_seg;
  int32_t* err;
};

int launch_route(const void* x, const void* gate_w, const float* gate_b, const void* logits_in,
                 int logits_dtype, int T, int H, int E, int k, int mode, int norm, float* logits_ws,
                 int32_t* ticket, int32_t* idx_out, float* sc_out, const RouteOut& ro,
                 cudaStream_t s, int local_first = 0, int local_n = 0,
                 int32_t* idx_local = nullptr);
size_t down_combine_smem(int P, const bigrig_expert_layout& L);
size_t down_combine_smem(int P, const bigrig_expert_layout& L, int nf);
int launch_down_combine(const void* h, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, const float* scores, const void* residual,
                        void* out, void* y_out, int T, cudaStream_t s);

int launch_gemv_gate_up(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, cudaStream_t s);
int launch_gemv_down(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, cudaStream_t s);
int gemm_mean_rows(int T, int k, int E);  // mean rows per routed expert (token tile input)
// x [T, H] bf16; xs [P, H] scratch for the token operand: x's rows in expert-sorted
// order (for 4-bit formats in the K order and operand type of the dequantised weights,
// fp16 for fp16-scaled formats).  4-bit h rows come out in that K order and type, and
// launch_gemm_down expects them so.
int launch_gemm_gate_up(const void* x, const RouteView& rv, const void* slab,
                        const bigrig_expert_layout& L, void* h, void* xs, int T, int mean_rows,
                        cudaStream_t s);
int launch_gemm_down(const void* h, const RouteView& rv, const void* slab,
                     const bigrig_expert_layout& L, void* y, int mean_rows, cudaStream_t s);
bool decode_layer_fits(const bigrig_expert_layout& L, int k, int E);
// Test hook of the persistent kernel's bounded waits (bigrig_test_grid_barrier).
void set_dl_wait_test(uint32_t phantom, uint32_t spin_limit);
int launch_decode_layer(const void* x, const void* gate_w, const float* gate_b, int E, int k,
                        int mode, int norm, const int32_t* g2s, const void* slab,
                        const bigrig_expert_layout& L, const void* residual, void* out,
                        int32_t* idx_out, float* sc_out, void* h, void* tagged, void* arrivals,
                        int32_t* err, cudaStream_t s, const int32_t* pre_idx = nullptr,
                        const float* pre_sc = nullptr);
// The split one-token layer (decode_split.cu): units of (routed expert, 64-feature group),
// integer tensor-core dot products, one grid barrier before the combine.  Scratch: ypart,
// decode_split_scratch(L, k) bytes (no zero-fill needed).
bool decode_split_fits(const bigrig_expert_layout& L, int k, int E);
bool decode_split_preferred(const bigrig_expert_layout& L, int k, int E);
size_t decode_split_scratch(const bigrig_expert_layout& L, int k);
int launch_decode_split(const void* x, const void* gate_w, const float* gate_b, int E, int k,
                        int mode, int norm, const int32_t* g2s, const void* slab,
                        const bigrig_expert_layout& L, const void* residual, void* out,
                        int32_t* idx_out, float* sc_out, float* ypart, void* tagged,
                        void* arrivals, int32_t* err, cudaStream_t s, const int32_t* pre_idx,
                        const float* pre_sc);
// A 3-bit expert's packed bytes (src, the 4-bit layout with 3-bit code streams) widened
// into a 4-bit slot laid out by L (L.bits == 4).
int launch_widen_expert(const void* src, void* dst, const bigrig_expert_layout& L, cudaStream_t s);
int launch_combine(const void* y, const float* scores, int T, int k, int H, void* out,
                   cudaStream_t s, const void* residual = nullptr);

// Peer buffer of one rank of an expert-parallel group (ep_peer.cu), the same offsets on
// every rank: gather flags [world] u64 (slot i raised by rank i), scatter flags [world],
// control (u64 layer counter, i32 timeout count), the gathered rows [world * tokens][H]
// bf16, the pair outputs of this rank's rows [tokens][k][H] bf16.
struct PeerLayout {
  size_t gflag, pflag, ctrl, xin, ybuf, total;
};
inline PeerLayout peer_layout(int world, int tokens, int hidden, int k) {
  auto up = [](size_t n) { return (n + 255) / 256 * 256; };
  PeerLayout l;
  l.gflag = 0;
  l.pflag = 64;
  l.ctrl = 128;
  l.xin = 256;
  l.ybuf = l.xin + up(static_cast<size_t>(world) * tokens * hidden * 2);
  l.total = l.ybuf + up(static_cast<size_t>(tokens) * k * hidden * 2);
  return l;
}
int launch_peer_gather(const bigrig_peer_group& g, const void* x, cudaStream_t s);
int launch_peer_localize(const int32_t* idx, int P, int first, int n_local, int32_t* idx_local,
                         cudaStream_t s);
int launch_peer_scatter(const bigrig_peer_group& g, const void* y, const int32_t* idx_local,
                        cudaStream_t s);
int launch_peer_combine(const bigrig_peer_group& g, const float* scores, const void* residual,
                        void* out, cudaStream_t s);

}  // namespace bigrig
