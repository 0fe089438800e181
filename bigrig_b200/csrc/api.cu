// extern "C" entry points of libbigrig_b200.so: argument checks, workspace carving
// and the launch sequence of each hot-path call.  See include/bigrig_b200.h.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "launch.h"

namespace bigrig {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(BIGRIG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return BIGRIG_OK;
}

// ------------------------------------------------------------------ launch timing
namespace {
struct TimingRecord {
  int id;
  cudaEvent_t start, end;
};
std::atomic<int> g_timing_on{0};
std::atomic<long long> g_launches[BIGRIG_K_COUNT];
std::mutex g_timing_mu;
std::vector<TimingRecord> g_records;
std::vector<cudaEvent_t> g_event_pool;
constexpr size_t kMaxRecords = 1 << 16;

cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}
const char* kKernelNames[BIGRIG_K_COUNT] = {
    "router_logits_kernel", "router_topk_kernel", "permute_kernel",
    "gemv_gate_up_kernel",  "gemv_down_kernel",   "combine_kernel",
    "dequant_kernel",       "grouped_gemm_kernel<gate_up>", "grouped_gemm_kernel<down>",
    "route_kernel",         "down_combine_kernel", "decode_layer_kernel",
    "decode_split_kernel",  "peer_gather_kernel",  "peer_localize_kernel",
    "peer_scatter_kernel",  "peer_combine_kernel"};
std::atomic<int> g_path{BIGRIG_PATH_AUTO};
std::atomic<int> g_gemm_min_rows{8};
constexpr int kDecodePairs = 32;     // routed pairs the fused decode chain / GEMV path takes
constexpr int kPeerGemvPairs = 16;   // a peer layer's expected pairs per rank on the GEMV pair
}  // namespace

TimedLaunch::TimedLaunch(int kernel_id, cudaStream_t s) : id_(kernel_id), s_(s), start_(nullptr) {
  g_launches[kernel_id].fetch_add(1, std::memory_order_relaxed);
  if (!((g_timing_on.load(std::memory_order_relaxed) >> kernel_id) & 1)) return;
  std::lock_guard<std::mutex> lock(g_timing_mu);
  if (g_records.size() >= kMaxRecords) return;
  cudaEvent_t e = take_event();
  if (e && cudaEventRecord(e, s) == cudaSuccess) start_ = e;
}

TimedLaunch::~TimedLaunch() {
  if (!start_) return;
  std::lock_guard<std::mutex> lock(g_timing_mu);
  cudaEvent_t e = take_event();
  if (e && cudaEventRecord(e, s_) == cudaSuccess) {
    g_records.push_back({id_, static_cast<cudaEvent_t>(start_), e});
  } else {
    g_event_pool.push_back(static_cast<cudaEvent_t>(start_));
    if (e) g_event_pool.push_back(e);
  }
}

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

// Scratch regions of one MoE call, carved in this order from the workspace.
struct Workspace {
  int32_t* err;
  int32_t* order;
  int32_t* inv;
  int32_t* offsets;
  int32_t* seg_expert;
  int32_t* seg_start;
  int32_t* num_seg;
  uint16_t* h;        // [P, I] bf16, expert-sorted rows
  uint16_t* xp;       // [P, H] the grouped GEMM's token operand: x rows in expert order
  uint16_t* y;        // [P, H] bf16, (token, k) order (moe_forward only)
  int32_t* indices;   // [P] (moe_forward when the caller passes none)
  float* scores;      // [P]
  float* logits;      // [T, E] (fused decode route)
  int32_t* ticket;    // last-CTA counter of the fused route, zero between calls (err[3])
  uint64_t* arrivals; // grid-barrier arrivals of the persistent decode kernel over all its
                      // launches on this workspace (err[4..5]); its launch index is this / G
  uint64_t* tagged;   // [E] the persistent decode kernel's logits, tagged with the epoch
  float* ypart;       // [k * I / 64, H] the split one-token kernel's unit partials (T == 1)
};

size_t carve(void* base, int T, int k, int E, const bigrig_expert_layout& L, Workspace* w) {
  const size_t P = static_cast<size_t>(T) * k;
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    void* p = base ? static_cast<char*>(base) + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  Workspace ws;
  ws.err = static_cast<int32_t*>(take(8 * sizeof(int32_t)));
  ws.order = static_cast<int32_t*>(take(P * sizeof(int32_t)));
  ws.inv = static_cast<int32_t*>(take(P * sizeof(int32_t)));
  ws.offsets = static_cast<int32_t*>(take((E + 1) * sizeof(int32_t)));
  ws.seg_expert = static_cast<int32_t*>(take(E * sizeof(int32_t)));
  ws.seg_start = static_cast<int32_t*>(take((E + 1) * sizeof(int32_t)));
  ws.num_seg = static_cast<int32_t*>(take(sizeof(int32_t)));
  ws.h = static_cast<uint16_t*>(take(P * L.inter * sizeof(uint16_t)));
  ws.xp = static_cast<uint16_t*>(take(P * L.hidden * sizeof(uint16_t)));
  ws.y = static_cast<uint16_t*>(take(P * L.hidden * sizeof(uint16_t)));
  ws.indices = static_cast<int32_t*>(take(P * sizeof(int32_t)));
  ws.scores = static_cast<float*>(take(P * sizeof(float)));
  ws.logits = static_cast<float*>(take(static_cast<size_t>(T) * E * sizeof(float)));
  ws.tagged = static_cast<uint64_t*>(take(static_cast<size_t>(E) * sizeof(uint64_t)));
  ws.ypart = static_cast<float*>(take(T == 1 ? decode_split_scratch(L, k) : 0));
  // the fused route's ticket lives at a fixed place -- word 3 of the error words -- so a
  // call of any shape finds it where the previous call left it, back at zero
  ws.ticket = ws.err ? ws.err + 3 : nullptr;
  ws.arrivals = ws.err ? reinterpret_cast<uint64_t*>(ws.err + 4) : nullptr;
  if (w) *w = ws;
  return off;
}

// Scratch of one expert-parallel layer call after its switch_glu workspace (which keeps the
// head of every workspace -- error words, route ticket, the persistent kernel's barrier
// arrivals -- where the other entry points sharing the workspace expect them): the route
// of all T gathered rows over the full router (logits, global ids, scores), the ids in
// this rank's numbering, and the pairs' output rows.
struct PeerScratch {
  float* logits;      // [T, E]
  int32_t* idx;       // [T * k]
  float* scores;      // [T * k]
  int32_t* idx_local; // [T * k]
  uint16_t* y;        // [T * k, H]
};

size_t peer_carve(void* base, int T, int k, int E, int H, PeerScratch* ps) {
  const size_t P = static_cast<size_t>(T) * k;
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    void* p = base ? static_cast<char*>(base) + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  PeerScratch s;
  s.logits = static_cast<float*>(take(static_cast<size_t>(T) * E * sizeof(float)));
  s.idx = static_cast<int32_t*>(take(P * sizeof(int32_t)));
  s.scores = static_cast<float*>(take(P * sizeof(float)));
  s.idx_local = static_cast<int32_t*>(take(P * sizeof(int32_t)));
  s.y = static_cast<uint16_t*>(take(P * H * sizeof(uint16_t)));
  if (ps) *ps = s;
  return off;
}

int check_peer_group(const bigrig_peer_group* g) {
  if (!g) return set_error(BIGRIG_ERR_INVALID, "peer group is NULL");
  if (g->world < 1 || g->world > BIGRIG_PEER_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
    return set_error(BIGRIG_ERR_INVALID, "peer group: world=%d rank=%d (world <= %d)", g->world,
                     g->rank, BIGRIG_PEER_MAX_RANKS);
  if (g->tokens < 1 || g->hidden < 8 || g->hidden % 8 || g->top_k < 1 || g->top_k > 32)
    return set_error(BIGRIG_ERR_INVALID, "peer group: tokens=%d hidden=%d top_k=%d", g->tokens,
                     g->hidden, g->top_k);
  for (int i = 0; i < g->world; ++i)
    if (!g->base[i] || reinterpret_cast<uintptr_t>(g->base[i]) % 256)
      return set_error(BIGRIG_ERR_INVALID, "peer group: buffer of rank %d missing or unaligned", i);
  return BIGRIG_OK;
}

int check_layout(const bigrig_expert_layout* Lp) {
  if (!Lp) return set_error(BIGRIG_ERR_INVALID, "layout is NULL");
  const bigrig_expert_layout& L = *Lp;
  if (L.bits != 4 && L.bits != 8)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "bits=%d: only 4 and 8 are built", L.bits);
  if (L.scale_dtype != BIGRIG_F16 && L.scale_dtype != BIGRIG_BF16)
    return set_error(BIGRIG_ERR_INVALID, "scale_dtype=%d: must be F16 or BF16", L.scale_dtype);
  if (L.group_size < 32 || L.group_size % 32)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "group_size=%d: must be a multiple of 32",
                     L.group_size);
  if (L.hidden <= 0 || L.inter <= 0 || L.hidden % L.group_size || L.inter % L.group_size)
    return set_error(BIGRIG_ERR_INVALID, "hidden=%d inter=%d must be positive multiples of %d",
                     L.hidden, L.inter, L.group_size);
  if (L.slot_stride < L.bytes_per_expert || L.slot_stride % 16)
    return set_error(BIGRIG_ERR_INVALID, "slot_stride=%lld must be >= bytes_per_expert=%lld "
                     "and a multiple of 16", (long long)L.slot_stride, (long long)L.bytes_per_expert);
  const int known = BIGRIG_LAYOUT_PLAIN | BIGRIG_LAYOUT_BIAS | (3 << 2) | (15 << 8);
  if (L.flags & ~known) return set_error(BIGRIG_ERR_INVALID, "flags=0x%x: unknown bits", L.flags);
  const bool plain = L.flags & BIGRIG_LAYOUT_PLAIN, bias = L.flags & BIGRIG_LAYOUT_BIAS;
  const int act = BIGRIG_LAYOUT_ACT(L.flags);
  if (plain ? (act != BIGRIG_ACT_SILU && act != BIGRIG_ACT_RELU2)
            : (act != BIGRIG_ACT_SILU && act != BIGRIG_ACT_GPT_OSS))
    return set_error(BIGRIG_ERR_UNSUPPORTED, "activation %d is not built for the %s expert", act,
                     plain ? "plain fc1/fc2" : "gated");
  const int bdt = BIGRIG_LAYOUT_BIAS_DTYPE(L.flags);
  if (!bias && bdt != 0)
    return set_error(BIGRIG_ERR_INVALID, "a bias dtype without BIGRIG_LAYOUT_BIAS");
  const int64_t bias_elem = bdt == BIGRIG_F32 ? 4 : 2;
  for (int p = 0; p < 3; ++p) {
    if (plain && p == 1) continue;             // fc1 at 0, fc2 at 2
    const int64_t rows = p == 2 ? L.hidden : L.inter;
    const int64_t cols = p == 2 ? L.inter : L.hidden;
    const int64_t wbytes = rows * cols * L.bits / 8;
    const int64_t sbytes = rows * (cols / L.group_size) * 2;
    if (L.weight_off[p] % 16 || L.scales_off[p] % 16 || L.biases_off[p] % 16 ||
        (bias && L.bias_off[p] % 16))
      return set_error(BIGRIG_ERR_INVALID, "projection %d: weight, scale and bias offsets must "
                       "be 16-byte aligned", p);
    if (L.weight_off[p] < 0 || L.weight_off[p] + wbytes > L.bytes_per_expert ||
        L.scales_off[p] < 0 || L.scales_off[p] + sbytes > L.bytes_per_expert ||
        L.biases_off[p] < 0 || L.biases_off[p] + sbytes > L.bytes_per_expert ||
        (bias && (L.bias_off[p] < 0 || L.bias_off[p] + rows * bias_elem > L.bytes_per_expert)))
      return set_error(BIGRIG_ERR_INVALID, "projection %d lies outside the %lld-byte expert", p,
                       (long long)L.bytes_per_expert);
  }
  return BIGRIG_OK;
}

int check_route(int T, int k, int E) {
  if (T < 0) return set_error(BIGRIG_ERR_INVALID, "T=%d must be >= 0", T);
  if (E < 1 || E > kMaxExperts)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "n_experts=%d: must be in [1, %d]", E, kMaxExperts);
  if (k < 1 || k > E || k > 32)
    return set_error(BIGRIG_ERR_INVALID, "top_k=%d: must be in [1, min(n_experts, 32)]", k);
  return BIGRIG_OK;
}

RouteView route_view(const Workspace& ws, const int32_t* g2s, int T, int k, int E) {
  RouteView rv;
  rv.order = ws.order;
  rv.inv = ws.inv;
  rv.seg_expert = ws.seg_expert;
  rv.seg_start = ws.seg_start;
  rv.num_seg = ws.num_seg;
  rv.g2s = g2s;
  rv.err = ws.err;
  rv.P = T * k;
  rv.k = k;
  rv.s_max = rv.P < E ? rv.P : E;
  rv.max_rows = T;
  rv.n_experts = E;
  return rv;
}

// Decode-sized calls take the fused three-kernel chain.
bool fused_decode(int T, int k, const bigrig_expert_layout& L) {
  const int path = g_path.load();
  return path != BIGRIG_PATH_GEMM && T * k <= kDecodePairs &&
         down_combine_smem(T * k, L) <= 200 * 1024;
}

int run_fused(const void* x, const void* gate_w, const float* gate_b, const void* logits,
              int logits_dtype, int T, int k, int E, int mode, int norm, const int32_t* g2s,
              const void* slab, const bigrig_expert_layout& L, const void* residual, void* out,
              int32_t* idx, float* sc, const Workspace& ws, cudaStream_t s) {
  RouteOut ro{ws.order, ws.inv, ws.offsets, ws.seg_expert, ws.seg_start, ws.num_seg, ws.err};
  if (int rc = launch_route(x, gate_w, gate_b, logits, logits_dtype, T, L.hidden, E, k, mode, norm,
                            ws.logits, ws.ticket, idx, sc, ro, s))
    return rc;
  const RouteView rv = route_view(ws, g2s, T, k, E);
  if (int rc = launch_gemv_gate_up(x, rv, slab, L, ws.h, s)) return rc;
  return launch_down_combine(ws.h, rv, slab, L, sc, residual, out, nullptr, T, s);
}

// The tensor-core GEMM once a call has more pairs than the decode chain takes (its
// dequant streams weights far faster than the GEMV's passes over an expert's rows, even
// at 16-column MMAs), or when the mean rows per routed expert reaches gemm_min_rows.
bool switch_glu_gemm(int P, int E) {
  const int path = g_path.load();
  return path == BIGRIG_PATH_GEMM ||
         ((path == BIGRIG_PATH_AUTO || path == BIGRIG_PATH_CHAIN || path == BIGRIG_PATH_TILED ||
           path == BIGRIG_PATH_SPLIT) &&
          (P > kDecodePairs || P >= g_gemm_min_rows.load() * (P < E ? P : E)));
}

int run_switch_glu(const void* x, const int32_t* indices, int T, int k, int E, const int32_t* g2s,
                   const void* slab, const bigrig_expert_layout& L, void* y, const Workspace& ws,
                   cudaStream_t s) {
  const int P = T * k;
  if (int rc = launch_permute(indices, P, E, ws.order, ws.inv, ws.offsets, ws.seg_expert,
                              ws.seg_start, ws.num_seg, ws.err, s))
    return rc;
  const RouteView rv = route_view(ws, g2s, T, k, E);
  const bool gemm = switch_glu_gemm(P, E);
  if (gemm) {
    const int mean = gemm_mean_rows(T, k, E);
    if (int rc = launch_gemm_gate_up(x, rv, slab, L, ws.h, ws.xp, T, mean, s)) return rc;
    return launch_gemm_down(ws.h, rv, slab, L, y, mean, s);
  }
  if (int rc = launch_gemv_gate_up(x, rv, slab, L, ws.h, s)) return rc;
  return launch_gemv_down(ws.h, rv, slab, L, y, s);
}

}  // namespace
}  // namespace bigrig

using namespace bigrig;

extern "C" {

const char* bigrig_version(void) { return "bigrig_b200 0.1 sm_100a"; }

const char* bigrig_last_error(void) { return g_last_error.c_str(); }

int bigrig_check_layout(const bigrig_expert_layout* layout) { return check_layout(layout); }

size_t bigrig_moe_workspace_bytes(int T, int k, int n_experts, const bigrig_expert_layout* layout) {
  if (!layout || T < 0 || k < 1 || n_experts < 1) return 0;
  return carve(nullptr, T, k, n_experts, *layout, nullptr);
}

int bigrig_dequant(const void* slab, const bigrig_expert_layout* layout, int slot, int proj,
                   void* out, void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (!slab || !out) return set_error(BIGRIG_ERR_INVALID, "dequant: NULL pointer");
  if (slot < 0) return set_error(BIGRIG_ERR_INVALID, "dequant: slot=%d < 0", slot);
  if (proj < 0 || proj > 2 || (proj == 1 && (layout->flags & BIGRIG_LAYOUT_PLAIN)))
    return set_error(BIGRIG_ERR_INVALID, "dequant: proj=%d (a plain expert has 0 and 2)", proj);
  return launch_dequant(slab, *layout, slot, proj, out, static_cast<cudaStream_t>(stream));
}

int bigrig_router_logits(const void* x, const void* w, const float* bias, float* logits, int T,
                         int H, int E, void* stream) {
  if (T < 0 || H <= 0 || E <= 0 || H % 8)
    return set_error(BIGRIG_ERR_INVALID, "router_logits: T=%d H=%d E=%d (H must be a multiple of 8)",
                     T, H, E);
  if (T == 0) return BIGRIG_OK;
  if (!x || !w || !logits) return set_error(BIGRIG_ERR_INVALID, "router_logits: NULL pointer");
  return launch_router_logits(x, w, bias, logits, T, H, E, static_cast<cudaStream_t>(stream));
}

int bigrig_router_topk(const void* logits, int logits_dtype, int T, int E, int k, int mode,
                       int norm_topk, int32_t* indices, float* scores, void* stream) {
  if (int rc = check_route(T, k, E)) return rc;
  if (logits_dtype != BIGRIG_F32 && logits_dtype != BIGRIG_BF16)
    return set_error(BIGRIG_ERR_INVALID, "router_topk: logits dtype must be F32 or BF16");
  if (mode != BIGRIG_SOFTMAX_TOPK && mode != BIGRIG_TOPK_SOFTMAX)
    return set_error(BIGRIG_ERR_INVALID, "router_topk: mode=%d", mode);
  if (T == 0) return BIGRIG_OK;
  if (!logits || !indices || !scores) return set_error(BIGRIG_ERR_INVALID, "router_topk: NULL pointer");
  return launch_router_topk(logits, logits_dtype, T, E, k, mode, norm_topk, indices, scores,
                            static_cast<cudaStream_t>(stream));
}

int bigrig_moe_permute(const int32_t* indices, int T, int k, int E, int32_t* order, int32_t* inv,
                       int32_t* offsets, int32_t* seg_expert, int32_t* seg_start, int32_t* num_seg,
                       int32_t* err_count, void* stream) {
  if (int rc = check_route(T, k, E)) return rc;
  if (!offsets || !seg_expert || !seg_start || !num_seg || (T > 0 && (!indices || !order || !inv)))
    return set_error(BIGRIG_ERR_INVALID, "moe_permute: NULL pointer");
  return launch_permute(indices, T * k, E, order, inv, offsets, seg_expert, seg_start, num_seg,
                        err_count, static_cast<cudaStream_t>(stream));
}

int bigrig_switch_glu(const void* x, const int32_t* indices, int T, int k, int n_experts,
                      const int32_t* g2s, const void* slab, const bigrig_expert_layout* layout,
                      void* y, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (int rc = check_route(T, k, n_experts)) return rc;
  if (T == 0) return BIGRIG_OK;
  if (!x || !indices || !slab || !y || !workspace)
    return set_error(BIGRIG_ERR_INVALID, "switch_glu: NULL pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(slab) % 16)
    return set_error(BIGRIG_ERR_INVALID, "switch_glu: x and slab must be 16-byte aligned");
  const size_t need = carve(nullptr, T, k, n_experts, *layout, nullptr);
  if (workspace_bytes < need)
    return set_error(BIGRIG_ERR_WORKSPACE, "switch_glu: workspace %zu bytes < %zu needed",
                     workspace_bytes, need);
  Workspace ws;
  carve(workspace, T, k, n_experts, *layout, &ws);
  return run_switch_glu(x, indices, T, k, n_experts, g2s, slab, *layout, y, ws,
                        static_cast<cudaStream_t>(stream));
}

int bigrig_combine(const void* y, const float* scores, int T, int k, int H, void* out,
                   void* stream) {
  if (T < 0 || k < 1 || H <= 0 || H % 2)
    return set_error(BIGRIG_ERR_INVALID, "combine: T=%d k=%d H=%d", T, k, H);
  if (T == 0) return BIGRIG_OK;
  if (!y || !scores || !out) return set_error(BIGRIG_ERR_INVALID, "combine: NULL pointer");
  return launch_combine(y, scores, T, k, H, out, static_cast<cudaStream_t>(stream));
}

int bigrig_moe_forward(const void* x, const void* logits, int logits_dtype, int T, int E, int k,
                       int mode, int norm_topk, const int32_t* g2s, const void* slab,
                       const bigrig_expert_layout* layout, void* out, int32_t* indices_out,
                       float* scores_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (int rc = check_route(T, k, E)) return rc;
  if (T == 0) return BIGRIG_OK;
  if (!x || !logits || !slab || !out || !workspace)
    return set_error(BIGRIG_ERR_INVALID, "moe_forward: NULL pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(slab) % 16)
    return set_error(BIGRIG_ERR_INVALID, "moe_forward: x and slab must be 16-byte aligned");
  const size_t need = carve(nullptr, T, k, E, *layout, nullptr);
  if (workspace_bytes < need)
    return set_error(BIGRIG_ERR_WORKSPACE, "moe_forward: workspace %zu bytes < %zu needed",
                     workspace_bytes, need);
  Workspace ws;
  carve(workspace, T, k, E, *layout, &ws);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* idx = indices_out ? indices_out : ws.indices;
  float* sc = scores_out ? scores_out : ws.scores;
  if (mode != BIGRIG_SOFTMAX_TOPK && mode != BIGRIG_TOPK_SOFTMAX)
    return set_error(BIGRIG_ERR_INVALID, "moe_forward: mode=%d", mode);
  if (logits_dtype != BIGRIG_F32 && logits_dtype != BIGRIG_BF16)
    return set_error(BIGRIG_ERR_INVALID, "moe_forward: logits dtype must be F32 or BF16");
  if (fused_decode(T, k, *layout))
    return run_fused(x, nullptr, nullptr, logits, logits_dtype, T, k, E, mode, norm_topk, g2s, slab,
                     *layout, nullptr, out, idx, sc, ws, s);
  if (int rc = bigrig_router_topk(logits, logits_dtype, T, E, k, mode, norm_topk, idx, sc, stream))
    return rc;
  if (int rc = run_switch_glu(x, idx, T, k, E, g2s, slab, *layout, ws.y, ws, s)) return rc;
  return launch_combine(ws.y, sc, T, k, layout->hidden, out, s);
}

int bigrig_moe_layer(const void* x, const void* gate_w, const float* gate_b, int T, int E, int k,
                     int mode, int norm_topk, const int32_t* g2s, const void* slab,
                     const bigrig_expert_layout* layout, const void* residual, void* out,
                     int32_t* indices_out, float* scores_out, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (int rc = check_route(T, k, E)) return rc;
  if (T == 0) return BIGRIG_OK;
  if (!x || !gate_w || !slab || !out || !workspace)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer: NULL pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(gate_w) % 16 ||
      reinterpret_cast<uintptr_t>(slab) % 16)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer: x, gate_w and slab must be 16-byte aligned");
  if (mode != BIGRIG_SOFTMAX_TOPK && mode != BIGRIG_TOPK_SOFTMAX)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer: mode=%d", mode);
  if (layout->hidden % 8)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer: hidden must be a multiple of 8");
  const size_t need = carve(nullptr, T, k, E, *layout, nullptr);
  if (workspace_bytes < need)
    return set_error(BIGRIG_ERR_WORKSPACE, "moe_layer: workspace %zu bytes < %zu needed",
                     workspace_bytes, need);
  Workspace ws;
  carve(workspace, T, k, E, *layout, &ws);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* idx = indices_out ? indices_out : ws.indices;
  float* sc = scores_out ? scores_out : ws.scores;
  const int path = g_path.load();
  const bool one = T == 1 && (path == BIGRIG_PATH_AUTO || path == BIGRIG_PATH_GEMV);
  if (T == 1 && ((one && decode_split_preferred(*layout, k, E)) ||
                 (path == BIGRIG_PATH_SPLIT && decode_split_fits(*layout, k, E))))
    return launch_decode_split(x, gate_w, gate_b, E, k, mode, norm_topk, g2s, slab, *layout,
                               residual, out, idx, sc, ws.ypart, ws.tagged, ws.arrivals, ws.err, s,
                               nullptr, nullptr);
  if ((one || (T == 1 && (path == BIGRIG_PATH_TILED || path == BIGRIG_PATH_SPLIT))) &&
      decode_layer_fits(*layout, k, E))
    return launch_decode_layer(x, gate_w, gate_b, E, k, mode, norm_topk, g2s, slab, *layout,
                               residual, out, idx, sc, ws.h, ws.tagged, ws.arrivals, ws.err, s);
  if (fused_decode(T, k, *layout))
    return run_fused(x, gate_w, gate_b, nullptr, BIGRIG_F32, T, k, E, mode, norm_topk, g2s, slab,
                     *layout, residual, out, idx, sc, ws, s);
  if (int rc = launch_router_logits(x, gate_w, gate_b, ws.logits, T, layout->hidden, E, s)) return rc;
  if (int rc = launch_router_topk(ws.logits, BIGRIG_F32, T, E, k, mode, norm_topk, idx, sc, s))
    return rc;
  if (int rc = run_switch_glu(x, idx, T, k, E, g2s, slab, *layout, ws.y, ws, s)) return rc;
  return launch_combine(ws.y, sc, T, k, layout->hidden, out, s, residual);
}

int bigrig_moe_layer_routed(const void* x, const int32_t* indices, const float* scores, int T,
                            int E, int k, const int32_t* g2s, const void* slab,
                            const bigrig_expert_layout* layout, const void* residual, void* out,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (int rc = check_route(T, k, E)) return rc;
  if (T == 0) return BIGRIG_OK;
  if (!x || !indices || !scores || !slab || !out || !workspace)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer_routed: NULL pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(slab) % 16)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer_routed: x and slab must be 16-byte aligned");
  if (layout->hidden % 8)
    return set_error(BIGRIG_ERR_INVALID, "moe_layer_routed: hidden must be a multiple of 8");
  const size_t need = carve(nullptr, T, k, E, *layout, nullptr);
  if (workspace_bytes < need)
    return set_error(BIGRIG_ERR_WORKSPACE, "moe_layer_routed: workspace %zu bytes < %zu needed",
                     workspace_bytes, need);
  Workspace ws;
  carve(workspace, T, k, E, *layout, &ws);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int path = g_path.load();
  const bool one = T == 1 && (path == BIGRIG_PATH_AUTO || path == BIGRIG_PATH_GEMV);
  if (T == 1 && ((one && decode_split_preferred(*layout, k, E)) ||
                 (path == BIGRIG_PATH_SPLIT && decode_split_fits(*layout, k, E))))
    return launch_decode_split(x, nullptr, nullptr, E, k, BIGRIG_SOFTMAX_TOPK, 0, g2s, slab,
                               *layout, residual, out, const_cast<int32_t*>(indices),
                               const_cast<float*>(scores), ws.ypart, ws.tagged, ws.arrivals,
                               ws.err, s, indices, scores);
  if ((one || (T == 1 && (path == BIGRIG_PATH_TILED || path == BIGRIG_PATH_SPLIT))) &&
      decode_layer_fits(*layout, k, E))
    return launch_decode_layer(x, nullptr, nullptr, E, k, BIGRIG_SOFTMAX_TOPK, 0, g2s, slab,
                               *layout, residual, out, const_cast<int32_t*>(indices),
                               const_cast<float*>(scores), ws.h, ws.tagged, ws.arrivals, ws.err, s,
                               indices, scores);
  if (int rc = run_switch_glu(x, indices, T, k, E, g2s, slab, *layout, ws.y, ws, s)) return rc;
  return launch_combine(ws.y, scores, T, k, layout->hidden, out, s, residual);
}

int bigrig_widen_expert(const void* src, void* dst, const bigrig_expert_layout* layout,
                        int src_bits, void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (!src || !dst) return set_error(BIGRIG_ERR_INVALID, "widen_expert: NULL pointer");
  if (layout->flags != 0)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "widen_expert: 3-bit codes of the gated SwiGLU "
                     "expert without projection biases only");
  if (src_bits != 3 || layout->bits != 4)
    return set_error(BIGRIG_ERR_UNSUPPORTED, "widen_expert: %d-bit codes into a %d-bit layout "
                     "(only 3 -> 4 is built)", src_bits, layout->bits);
  if ((layout->hidden % 32) || (layout->inter % 32) || (reinterpret_cast<uintptr_t>(src) % 4) ||
      (reinterpret_cast<uintptr_t>(dst) % 16))
    return set_error(BIGRIG_ERR_INVALID, "widen_expert: dims must be multiples of 32, src 4-byte "
                     "and dst 16-byte aligned");
  return launch_widen_expert(src, dst, *layout, static_cast<cudaStream_t>(stream));
}

int bigrig_test_grid_barrier(int phantom_ctas, unsigned int spin_limit) {
  if (phantom_ctas < 0)
    return set_error(BIGRIG_ERR_INVALID, "test_grid_barrier: phantom_ctas=%d", phantom_ctas);
  set_dl_wait_test(static_cast<uint32_t>(phantom_ctas), spin_limit);
  return BIGRIG_OK;
}

int bigrig_set_path(int mode, int gemm_min_rows) {
  if (mode < BIGRIG_PATH_AUTO || mode > BIGRIG_PATH_SPLIT || gemm_min_rows < 1)
    return set_error(BIGRIG_ERR_INVALID, "set_path: mode=%d gemm_min_rows=%d", mode, gemm_min_rows);
  const int prev = g_path.exchange(mode);
  g_gemm_min_rows.store(gemm_min_rows);
  return prev;
}

int bigrig_get_path(int* mode, int* gemm_min_rows) {
  if (mode) *mode = g_path.load();
  if (gemm_min_rows) *gemm_min_rows = g_gemm_min_rows.load();
  return BIGRIG_OK;
}

int bigrig_timing_enable(int mask) {
  g_timing_on.store(mask);
  return BIGRIG_OK;
}

int bigrig_launch_counts(int64_t* out) {
  if (!out) return set_error(BIGRIG_ERR_INVALID, "launch_counts: NULL pointer");
  for (int i = 0; i < BIGRIG_K_COUNT; ++i) out[i] = g_launches[i].load();
  return BIGRIG_OK;
}

int bigrig_timing_read(int kernel_id, double* total_ms, int64_t* launches) {
  if (kernel_id < 0 || kernel_id >= BIGRIG_K_COUNT || !total_ms || !launches)
    return set_error(BIGRIG_ERR_INVALID, "timing_read: kernel_id=%d", kernel_id);
  std::lock_guard<std::mutex> lock(g_timing_mu);
  double sum = 0.0;
  int64_t n = 0;
  std::vector<TimingRecord> keep;
  for (const TimingRecord& r : g_records) {
    if (r.id != kernel_id) {
      keep.push_back(r);
      continue;
    }
    float ms = 0.f;
    if (cudaEventSynchronize(r.end) == cudaSuccess &&
        cudaEventElapsedTime(&ms, r.start, r.end) == cudaSuccess) {
      sum += ms;
      ++n;
    }
    g_event_pool.push_back(r.start);
    g_event_pool.push_back(r.end);
  }
  g_records.swap(keep);
  *total_ms = sum;
  *launches = n;
  return BIGRIG_OK;
}

const char* bigrig_kernel_name(int kernel_id) {
  return (kernel_id >= 0 && kernel_id < BIGRIG_K_COUNT) ? kKernelNames[kernel_id] : "";
}

int bigrig_copy_regions(void* const* dst, const void* const* src, const size_t* bytes, int n,
                        void* stream) {
  if (n < 0 || (n > 0 && (!dst || !src || !bytes)))
    return set_error(BIGRIG_ERR_INVALID, "copy_regions: n=%d or NULL arrays", n);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    if (bytes[i] == 0) continue;
    if (!dst[i] || !src[i]) return set_error(BIGRIG_ERR_INVALID, "copy_regions: NULL pointer %d", i);
    const cudaError_t rc = cudaMemcpyAsync(dst[i], src[i], bytes[i], cudaMemcpyDefault, s);
    if (rc != cudaSuccess)
      return set_error(BIGRIG_ERR_CUDA, "copy_regions: copy %d: %s", i, cudaGetErrorString(rc));
  }
  return BIGRIG_OK;
}

int bigrig_workspace_errors(void* workspace, int32_t* out, void* stream) {
  if (!workspace || !out) return set_error(BIGRIG_ERR_INVALID, "workspace_errors: NULL pointer");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* err = static_cast<int32_t*>(workspace);
  if (cudaMemcpyAsync(out, err, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemsetAsync(err, 0, sizeof(int32_t), s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "workspace_errors: %s", cudaGetErrorString(cudaGetLastError()));
  return BIGRIG_OK;
}

size_t bigrig_peer_workspace_bytes(const bigrig_peer_group* g, int n_experts, int n_local,
                                   const bigrig_expert_layout* layout) {
  if (!g || !layout || g->world < 1 || g->tokens < 1 || g->top_k < 1 || n_experts < 1 ||
      n_local < 1)
    return 0;
  const int T = g->world * g->tokens;
  return peer_carve(nullptr, T, g->top_k, n_experts, layout->hidden, nullptr) +
         carve(nullptr, T, g->top_k, n_local, *layout, nullptr);
}

int bigrig_peer_layer(const bigrig_peer_group* g, const void* x, const void* gate_w,
                      const float* gate_b, int E, int mode, int norm_topk, int first_expert,
                      int n_local, const int32_t* g2s, const void* slab,
                      const bigrig_expert_layout* layout, const void* residual, void* out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_peer_group(g)) return rc;
  if (int rc = check_layout(layout)) return rc;
  const int k = g->top_k, H = layout->hidden;
  if (int rc = check_route(g->tokens, k, E)) return rc;
  if (H != g->hidden)
    return set_error(BIGRIG_ERR_INVALID, "peer_layer: layout hidden %d != group hidden %d", H,
                     g->hidden);
  if (n_local < 1 || first_expert < 0 || first_expert + n_local > E)
    return set_error(BIGRIG_ERR_INVALID, "peer_layer: experts [%d, %d) outside [0, %d)",
                     first_expert, first_expert + n_local, E);
  if (mode != BIGRIG_SOFTMAX_TOPK && mode != BIGRIG_TOPK_SOFTMAX)
    return set_error(BIGRIG_ERR_INVALID, "peer_layer: mode=%d", mode);
  if (!x || !gate_w || !slab || !out || !workspace)
    return set_error(BIGRIG_ERR_INVALID, "peer_layer: NULL pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(gate_w) % 16 ||
      reinterpret_cast<uintptr_t>(slab) % 16 || (residual && reinterpret_cast<uintptr_t>(residual) % 4) ||
      reinterpret_cast<uintptr_t>(out) % 4)
    return set_error(BIGRIG_ERR_INVALID, "peer_layer: x, gate_w, slab must be 16-byte aligned, "
                     "residual and out 4-byte aligned");
  const int T = g->world * g->tokens;
  const size_t sbytes = carve(nullptr, T, k, n_local, *layout, nullptr);
  const size_t need = sbytes + peer_carve(nullptr, T, k, E, H, nullptr);
  if (workspace_bytes < need)
    return set_error(BIGRIG_ERR_WORKSPACE, "peer_layer: workspace %zu bytes < %zu needed",
                     workspace_bytes, need);
  Workspace ws;
  carve(workspace, T, k, n_local, *layout, &ws);
  PeerScratch ps;
  peer_carve(static_cast<char*>(workspace) + sbytes, T, k, E, H, &ps);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const PeerLayout lay = peer_layout(g->world, g->tokens, H, k);
  const void* rows = static_cast<const uint8_t*>(g->base[g->rank]) + lay.xin;   // [T, H] gathered
  if (int rc = launch_peer_gather(*g, x, s)) return rc;
  const int P = T * k;
  // Most of the T * k pairs belong to other ranks: about P / world are this rank's.  Under
  // the automatic rule the GEMV pair takes the call while that share is decode-sized (the
  // grouped GEMM's per-iteration handoff dominates tiles of a few rows).
  const int share = (P + g->world - 1) / g->world;
  const bool gemv = !switch_glu_gemm(P, n_local) ||
                    (g_path.load() == BIGRIG_PATH_AUTO && share <= kPeerGemvPairs);
  if (gemv && P <= kDecodePairs) {
    // decode-sized: router, top-k, the local numbering and the permutation in one launch
    // (the chain's route kernel), then the GEMV pair
    const RouteOut ro{ws.order, ws.inv, ws.offsets, ws.seg_expert, ws.seg_start, ws.num_seg, ws.err};
    if (int rc = launch_route(rows, gate_w, gate_b, nullptr, BIGRIG_F32, T, H, E, k, mode,
                              norm_topk, ps.logits, ws.ticket, ps.idx, ps.scores, ro, s,
                              first_expert, n_local, ps.idx_local))
      return rc;
    const RouteView rv = route_view(ws, g2s, T, k, n_local);
    if (int rc = launch_gemv_gate_up(rows, rv, slab, *layout, ws.h, s)) return rc;
    if (int rc = launch_gemv_down(ws.h, rv, slab, *layout, ps.y, s)) return rc;
    if (int rc = launch_peer_scatter(*g, ps.y, ps.idx_local, s)) return rc;
    return launch_peer_combine(*g, ps.scores, residual, out, s);
  }
  if (int rc = launch_router_logits(rows, gate_w, gate_b, ps.logits, T, H, E, s)) return rc;
  if (int rc = launch_router_topk(ps.logits, BIGRIG_F32, T, E, k, mode, norm_topk, ps.idx,
                                  ps.scores, s))
    return rc;
  if (int rc = launch_peer_localize(ps.idx, T * k, first_expert, n_local, ps.idx_local, s)) return rc;
  if (gemv) {
    if (int rc = launch_permute(ps.idx_local, P, n_local, ws.order, ws.inv, ws.offsets,
                                ws.seg_expert, ws.seg_start, ws.num_seg, ws.err, s))
      return rc;
    const RouteView rv = route_view(ws, g2s, T, k, n_local);
    if (int rc = launch_gemv_gate_up(rows, rv, slab, *layout, ws.h, s)) return rc;
    if (int rc = launch_gemv_down(ws.h, rv, slab, *layout, ps.y, s)) return rc;
  } else if (int rc = run_switch_glu(rows, ps.idx_local, T, k, n_local, g2s, slab, *layout,
                                     ps.y, ws, s)) {
    return rc;
  }
  if (int rc = launch_peer_scatter(*g, ps.y, ps.idx_local, s)) return rc;
  return launch_peer_combine(*g, ps.scores, residual, out, s);
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation entry point
// For callers that cannot allocate device memory at call time (see the header): the
// scratch of bigrig_switch_glu_noalloc lives in a file-scope device array that every
// GPU loading this library holds until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[BIGRIG_NOALLOC_SCRATCH_BYTES];

namespace bigrig {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// The device address of the scratch array on the current device, resolved once per
// device (cudaGetSymbolAddress with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(BIGRIG_ERR_CUDA, "switch_glu_noalloc: no usable current device (%d)", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(BIGRIG_ERR_CUDA, "switch_glu_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return BIGRIG_OK;
}
}  // namespace
}  // namespace bigrig

extern "C" int bigrig_switch_glu_noalloc(const void* x, const int32_t* indices, int T, int k,
                                         int n_experts, const int32_t* g2s, const void* slab,
                                         const bigrig_expert_layout* layout, void* y,
                                         void* stream) {
  if (int rc = check_layout(layout)) return rc;
  if (int rc = check_route(T, k, n_experts)) return rc;
  if (T == 0) return BIGRIG_OK;
  if (!x || !indices || !slab || !y)
    return set_error(BIGRIG_ERR_INVALID, "switch_glu_noalloc: NULL pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(slab) % 16)
    return set_error(BIGRIG_ERR_INVALID, "switch_glu_noalloc: x and slab must be 16-byte aligned");
  const size_t need = carve(nullptr, T, k, n_experts, *layout, nullptr);
  if (need > BIGRIG_NOALLOC_SCRATCH_BYTES)
    return set_error(BIGRIG_ERR_WORKSPACE,
                     "switch_glu_noalloc: this call needs %zu bytes of scratch but the static "
                     "array holds %zu; use bigrig_switch_glu with a workspace for calls this large",
                     need, static_cast<size_t>(BIGRIG_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the error words at the head of the scratch must start at zero; everything else is
  // written before it is read
  if (cudaMemsetAsync(scratch, 0, 4 * sizeof(int32_t), s) != cudaSuccess)
    return set_error(BIGRIG_ERR_CUDA, "switch_glu_noalloc: %s", cudaGetErrorString(cudaGetLastError()));
  Workspace ws;
  carve(scratch, T, k, n_experts, *layout, &ws);
  return run_switch_glu(x, indices, T, k, n_experts, g2s, slab, *layout, y, ws, s);
}

