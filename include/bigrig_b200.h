/*
 * bigrig_b200.h -- C ABI of the B200 (sm_100a) MoE expert hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, a cudaStream_t; NULL is the legacy default stream), never
 * allocates on the hot path, and returns 0 or a negative BIGRIG_ERR_* code.
 * bigrig_last_error() gives the calling thread's message for the last failure.
 * Scratch memory is passed in by the caller (bigrig_moe_workspace_bytes says
 * how much); the library keeps no device state between calls.
 *
 * Reference interfaces replaced (paths relative to the BigRig tree):
 *   bigrig_switch_glu     StreamingSwitchGLU.__call__(x, indices) -> y[..., k, H]
 *                         bigrig_engine/stream.py:1377-1577 (decode: _forward_views_one
 *                         1278-1318; prefill: _forward_views 1237-1276, _forward/_proj
 *                         1128-1172, 1605-1631)
 *   bigrig_moe_forward    the MoE block around it: router top-k/softmax, the call above,
 *                         then sum_k score * y (stream.py:1523-1525; router rule
 *                         bigrig_engine/adapter.py:74-92)
 *   bigrig_router_logits  the router gate x . W^T (+ bias) (stream.py:1436, 895)
 *   bigrig_router_topk    mx.softmax + mx.argpartition top-k (stream.py:1436-1439)
 *   bigrig_moe_permute    host np.argsort(kind="stable") permutation, order // k,
 *                         inverse argsort (stream.py:1246-1250, 1275-1276, 1527-1531)
 *   bigrig_dequant        mx.dequantize of one expert projection (tune.py:64-70,
 *                         precision.py:186-189)
 *   bigrig_combine        sum_k score * y of the calling MoE block
 */
#ifndef BIGRIG_B200_H
#define BIGRIG_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BIGRIG_API __attribute__((visibility("default")))
#else
#define BIGRIG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The Python host maps them onto the reference's exception types. */
#define BIGRIG_OK 0
#define BIGRIG_ERR_INVALID (-1)     /* bad argument            -> ValueError          */
#define BIGRIG_ERR_CUDA (-2)        /* CUDA runtime failure    -> RuntimeError        */
#define BIGRIG_ERR_UNSUPPORTED (-3) /* format not built        -> NotImplementedError */
#define BIGRIG_ERR_WORKSPACE (-4)   /* workspace too small     -> ValueError          */

/* Element types. */
#define BIGRIG_F32 0
#define BIGRIG_F16 1
#define BIGRIG_BF16 2

/* Router orders (see bigrig_router_topk). */
#define BIGRIG_SOFTMAX_TOPK 0 /* softmax over E, keep top-k (OLMoE; Qwen3 with norm) */
#define BIGRIG_TOPK_SOFTMAX 1 /* keep top-k logits, softmax over k (Mixtral, gpt-oss)  */

/* Byte layout of one expert inside a slot, in the reference's packed order
 * (bigrig_engine/stream.py:106-186): gate_proj{weight,scales,biases},
 * up_proj{...}, down_proj{...}.  weight is uint32 codes [out, in*bits/32],
 * scales/biases are half [out, in/group_size].  Index 0 gate, 1 up, 2 down.
 *
 * The two expert shapes of the reference (stream.py:48-76): the gated SwiGLU expert
 * down(act(gate(x), up(x))) and, with BIGRIG_LAYOUT_PLAIN, the plain two-layer MLP
 * fc2(act(fc1(x))) -- fc1 at index 0 (I x H), fc2 at index 2 (H x I), index 1 unused.
 * With BIGRIG_LAYOUT_BIAS every projection also carries the affine `bias` component
 * (stream.py:79-81), [out] elements of BIGRIG_LAYOUT_BIAS_DTYPE(flags) at bias_off[p],
 * added to the projection's output before the activation (gate/up, fc1) or before the
 * output is stored (down, fc2).  The activation, BIGRIG_LAYOUT_ACT(flags):
 *   BIGRIG_ACT_SILU    gated: silu(gate) * up;  plain: silu(fc1)
 *   BIGRIG_ACT_GPT_OSS gated only: g = min(gate, 7), u = clamp(up, -7, 7),
 *                      g * sigmoid(1.702 g) * (u + 1)  (gpt-oss's SwiGLU)
 *   BIGRIG_ACT_RELU2   plain only: max(fc1, 0)^2
 * Each computed in fp32 from the fp32 projection outputs (plus bias); the result is
 * rounded once to the down projection's input type. */
#define BIGRIG_LAYOUT_PLAIN 1
#define BIGRIG_LAYOUT_BIAS 2
#define BIGRIG_LAYOUT_BIAS_DTYPE(flags) (((flags) >> 2) & 3) /* BIGRIG_F32/F16/BF16 */
#define BIGRIG_LAYOUT_ACT(flags) (((flags) >> 8) & 15)
#define BIGRIG_ACT_SILU 0
#define BIGRIG_ACT_GPT_OSS 1
#define BIGRIG_ACT_RELU2 2
typedef struct bigrig_expert_layout {
  int32_t hidden;      /* H: input of gate/up, output of down            */
  int32_t inter;       /* I: output of gate/up, input of down            */
  int32_t bits;        /* 4 or 8                                         */
  int32_t group_size;  /* 64                                             */
  int32_t scale_dtype; /* BIGRIG_F16 or BIGRIG_BF16                      */
  int32_t flags;       /* BIGRIG_LAYOUT_* bits, bias dtype << 2, act << 8; 0 = gated SwiGLU */
  int64_t bytes_per_expert;
  int64_t slot_stride; /* bytes between slots of a slab, >= bytes_per_expert, multiple of 16 */
  int64_t weight_off[3];
  int64_t scales_off[3];
  int64_t biases_off[3];
  int64_t bias_off[3]; /* the affine bias per projection (BIGRIG_LAYOUT_BIAS), else 0 */
} bigrig_expert_layout;

/* Library identity and the calling thread's last error message. */
BIGRIG_API const char* bigrig_version(void);
BIGRIG_API const char* bigrig_last_error(void);

/* Check a layout for the shapes this build supports. 0 or BIGRIG_ERR_*. */
BIGRIG_API int bigrig_check_layout(const bigrig_expert_layout* layout);

/* Bytes of scratch bigrig_switch_glu / bigrig_moe_forward need for T tokens. */
BIGRIG_API size_t bigrig_moe_workspace_bytes(int T, int k, int n_experts, const bigrig_expert_layout* layout);

/* Dequantise projection `proj` (0 gate, 1 up, 2 down) of the expert in slot
 * `slot` into out[rows, cols] of the scale dtype:
 * out = round_to_scale_dtype(f32(scale) * q + f32(bias)). */
BIGRIG_API int bigrig_dequant(const void* slab, const bigrig_expert_layout* layout, int slot, int proj,
                   void* out, void* stream);

/* logits[T, E] (fp32) = x[T, H] (bf16) . w[E, H]^T (bf16) + bias[E] (fp32, may be NULL). */
BIGRIG_API int bigrig_router_logits(const void* x, const void* w, const float* bias, float* logits,
                         int T, int H, int E, void* stream);

/* Top-k routing over logits[T, E] (BIGRIG_F32 or BIGRIG_BF16).  indices[T, k] in
 * rank order (largest logit first, ties to the lower expert id); scores[T, k]
 * fp32 per `mode`; norm_topk renormalises softmax_topk scores to sum to 1. */
BIGRIG_API int bigrig_router_topk(const void* logits, int logits_dtype, int T, int E, int k, int mode,
                       int norm_topk, int32_t* indices, float* scores, void* stream);

/* Stable expert-sorted permutation of the T*k (token, k) pairs in indices[T, k].
 * order[P]: pair ids sorted by expert (stable); inv[P]: inverse permutation;
 * offsets[E+1]: counting-sort offsets per expert id; seg_expert[E] / seg_start[E+1]
 * / num_seg[1]: the non-empty experts in ascending id and where their run starts.
 * A negative expert id marks a padding row (expert-parallel dispatch buffers): it is
 * left out of the segments silently.  An id >= E is left out and counted in
 * err_count[1] (may be NULL). */
BIGRIG_API int bigrig_moe_permute(const int32_t* indices, int T, int k, int E, int32_t* order, int32_t* inv,
                       int32_t* offsets, int32_t* seg_expert, int32_t* seg_start, int32_t* num_seg,
                       int32_t* err_count, void* stream);

/* Unreduced SwiGLU experts: y[T, k, H] (bf16) with
 * y[t, j] = down(silu(gate(x[t])) * up(x[t])) of expert indices[t, j], read from
 * slot g2s[indices[t, j]] of `slab` (g2s NULL: slot == expert id).  x is bf16
 * [T, H].  A slot id < 0 is counted in the workspace error word and its rows are
 * written as zeros (the host pool guarantees residency before the call).  Pairs
 * whose expert id is negative are padding: skipped, their y rows left untouched. */
BIGRIG_API int bigrig_switch_glu(const void* x, const int32_t* indices, int T, int k, int n_experts,
                      const int32_t* g2s, const void* slab, const bigrig_expert_layout* layout,
                      void* y, void* workspace, size_t workspace_bytes, void* stream);

/* out[T, H] (bf16) = sum_j scores[t, j] * y[t, j, :], fp32 accumulation in j order. */
BIGRIG_API int bigrig_combine(const void* y, const float* scores, int T, int k, int H, void* out,
                   void* stream);

/* The whole MoE layer from router logits: top-k + softmax (mode, norm_topk),
 * bigrig_switch_glu, combine.  Writes out[T, H] bf16 and, when not NULL,
 * indices_out[T, k] / scores_out[T, k]. */
BIGRIG_API int bigrig_moe_forward(const void* x, const void* logits, int logits_dtype, int T, int E, int k,
                       int mode, int norm_topk, const int32_t* g2s, const void* slab,
                       const bigrig_expert_layout* layout, void* out, int32_t* indices_out,
                       float* scores_out, void* workspace, size_t workspace_bytes, void* stream);

/* Kernel ids for the timing hooks below. */
#define BIGRIG_K_ROUTER_LOGITS 0
#define BIGRIG_K_ROUTER_TOPK 1
#define BIGRIG_K_PERMUTE 2
#define BIGRIG_K_GATE_UP 3
#define BIGRIG_K_DOWN 4
#define BIGRIG_K_COMBINE 5
#define BIGRIG_K_DEQUANT 6
#define BIGRIG_K_GEMM_GATE_UP 7
#define BIGRIG_K_GEMM_DOWN 8
#define BIGRIG_K_ROUTE 9
#define BIGRIG_K_DOWN_COMBINE 10
#define BIGRIG_K_DECODE_LAYER 11
#define BIGRIG_K_DECODE_SPLIT 12
#define BIGRIG_K_PEER_GATHER 13
#define BIGRIG_K_PEER_LOCALIZE 14
#define BIGRIG_K_PEER_SCATTER 15
#define BIGRIG_K_PEER_COMBINE 16
#define BIGRIG_K_COUNT 17

/* Which expert kernels bigrig_switch_glu / bigrig_moe_forward / bigrig_moe_layer use:
 * BIGRIG_PATH_AUTO picks the grouped GEMV for calls of at most 32 routed pairs (decode)
 * and the tcgen05 grouped GEMM above that or when the mean rows per routed expert
 * reaches `gemm_min_rows`, and runs a one-token bigrig_moe_layer as one persistent kernel:
 * the feature-tiled kernel, or, for layers whose (routed expert, 64-feature group) units
 * fill at least two waves of SMs, the split kernel (one such unit per work item, integer
 * tensor-core dot products, no exchange between gate/up and down);
 * BIGRIG_PATH_GEMV and BIGRIG_PATH_GEMM force one expert path; BIGRIG_PATH_CHAIN is
 * AUTO with one-token layers on the three-kernel chain instead of a persistent kernel;
 * BIGRIG_PATH_TILED and BIGRIG_PATH_SPLIT are AUTO with one-token layers on that
 * persistent kernel (where its plan fits the layer).  All give results within the parity
 * bar of each other.  Process-wide; returns the previous mode. */
#define BIGRIG_PATH_AUTO 0
#define BIGRIG_PATH_GEMV 1
#define BIGRIG_PATH_GEMM 2
#define BIGRIG_PATH_CHAIN 3
#define BIGRIG_PATH_TILED 4
#define BIGRIG_PATH_SPLIT 5
BIGRIG_API int bigrig_set_path(int mode, int gemm_min_rows);

/* The current path mode and gemm_min_rows (either pointer may be NULL); 0. */
BIGRIG_API int bigrig_get_path(int* mode, int* gemm_min_rows);

/* CUDA-event timing of this library's kernel launches, off by default.  `mask`
 * selects kernel ids (bit i = id i); each selected launch is bracketed by two
 * events on its own stream (do not enable it while a stream is being captured
 * into a graph).  bigrig_timing_read waits for the recorded events of
 * `kernel_id`, returns the sum of their durations and how many launches were
 * timed since the last read, and forgets them.  bigrig_launch_counts fills
 * out[BIGRIG_K_COUNT] with every launch issued since the library loaded, timed
 * or not. */
BIGRIG_API int bigrig_timing_enable(int mask);
BIGRIG_API int bigrig_timing_read(int kernel_id, double* total_ms, int64_t* launches);
BIGRIG_API int bigrig_launch_counts(int64_t* out);
BIGRIG_API const char* bigrig_kernel_name(int kernel_id);

/* The whole MoE block of one decoder layer from its hidden states:
 * logits = x . gate_w^T (+ gate_b), top-k + softmax (mode, norm_topk), the SwiGLU
 * experts and out[T, H] = residual + sum_j score * y (residual may be NULL).
 * x, gate_w, residual, out bf16; gate_b fp32 [E] or NULL.  A one-token call runs as
 * ONE cooperative kernel, a CTA per SM (router, top-k, gate/up, down and combine
 * separated by a flag and one grid barrier whose words live in the workspace); other
 * decode-sized calls (T * k <= 32), and one-token layers too wide for that kernel,
 * run as three kernels chained by programmatic dependent launch.  The workspace must
 * start zero-filled and calls sharing one workspace must not overlap on the GPU.
 * Replaces the mlx_lm MoE block around StreamingSwitchGLU (stream.py:1377,
 * 1523-1525; router rule adapter.py:74-92). */
BIGRIG_API int bigrig_moe_layer(const void* x, const void* gate_w, const float* gate_b, int T,
                                int E, int k, int mode, int norm_topk, const int32_t* g2s,
                                const void* slab, const bigrig_expert_layout* layout,
                                const void* residual, void* out, int32_t* indices_out,
                                float* scores_out, void* workspace, size_t workspace_bytes,
                                void* stream);

/* bigrig_moe_layer for a caller that already holds the routing: indices int32 [T, k] and
 * scores fp32 [T, k] on the device (typically bigrig_router_topk's output that the host
 * also read back to make the experts resident), out[T, H] = residual + sum_j score * y.
 * Nothing is routed again: a one-token call runs the persistent kernel without its router
 * phase, other calls the expert kernels and the combine.  Expert ids outside [0, E) or
 * without a slot contribute zeros and are counted in the workspace's error word.  Same
 * workspace rules as bigrig_moe_layer.  Replaces the block's combine around
 * StreamingSwitchGLU.__call__ after the routing readback (stream.py:1447-1450,
 * 1523-1525). */
BIGRIG_API int bigrig_moe_layer_routed(const void* x, const int32_t* indices, const float* scores,
                                       int T, int E, int k, const int32_t* g2s, const void* slab,
                                       const bigrig_expert_layout* layout, const void* residual,
                                       void* out, void* workspace, size_t workspace_bytes,
                                       void* stream);

/* Admission of a 3-bit expert: `src` (device) holds its packed bytes as the blob stores
 * them -- per projection (gate, up, down) the 3-bit code stream of each row, scales,
 * biases -- and `dst` receives the same expert in the 4-bit layout `layout` describes
 * (layout->bits == 4), each code widened (q in [0, 7] is a 4-bit code with the same
 * scale and bias, so dequantised weights are unchanged).  Runs on `stream`; src and dst
 * must not overlap.  Replaces the 3-bit slot write of ExpertPool.admit / build_arrays
 * (stream.py:692-780) for the quantisation the blob's manifest records
 * (stream.py:144-151). */
BIGRIG_API int bigrig_widen_expert(const void* src, void* dst, const bigrig_expert_layout* layout,
                                   int src_bits, void* stream);

/* Test hook for the failure path of the persistent one-token kernel: its grid barrier
 * also waits for `phantom_ctas` CTAs that do not exist, and every bounded wait polls at
 * most `spin_limit` times (0: the default, about half a second).  With phantom_ctas > 0
 * the barrier's wait runs out in every CTA, each adds 1 to the workspace's wait-timeout
 * word (error word 1) and the kernel finishes (its output is then not meaningful); the
 * next launch with the hook cleared (0, 0) is correct again.  No counterpart in the
 * reference (failure detection is tested by making a bounded wait run out, never by a
 * fault). */
BIGRIG_API int bigrig_test_grid_barrier(int phantom_ctas, unsigned int spin_limit);

/* Device error word of a workspace (slots < 0, ids out of range), copied to *out
 * with a synchronous read on `stream`; resets it to 0.  For tests and debugging. */
BIGRIG_API int bigrig_workspace_errors(void* workspace, int32_t* out, void* stream);

/* n asynchronous copies on `stream`, one cudaMemcpyAsync each: dst[i] <- src[i], bytes[i]
 * (host or device pointers; pinned host sources stay asynchronous).  The pool's admissions
 * of one step in a single call -- replaces the per-expert slot writes of ExpertPool.admit /
 * admit_arrays (stream.py:692-705, 757-780) so that a decode step pays one host call per
 * layer instead of one per expert. */
BIGRIG_API int bigrig_copy_regions(void* const* dst, const void* const* src, const size_t* bytes,
                                   int n, void* stream);

/* bigrig_switch_glu for callers that cannot allocate device memory when they call: a
 * process whose device memory is carved up once at start-up by another allocator, or a
 * caller in a latency-critical loop where cudaMalloc (which synchronises the device) is
 * not allowed.  No counterpart in the reference (MLX allocates inside every call).
 * Same arguments and result as bigrig_switch_glu minus the workspace: the scratch is a
 * file-scope device array of BIGRIG_NOALLOC_SCRATCH_BYTES (4 MiB) that every GPU that
 * loads the library holds until the process exits.  Calls needing more scratch than that
 * (bigrig_moe_workspace_bytes) return BIGRIG_ERR_WORKSPACE.  The first call on a device
 * resolves the array's address with cudaGetSymbolAddress and keeps it for that device;
 * under CUDA's lazy module loading that first call may also load the module and commit
 * the 4 MiB, so make it (or a warm-up call) at initialisation, before any stream capture
 * and before a fixed memory budget is carved.  The kept address does not survive a
 * cudaDeviceReset: after one, reload the library.  Every call shares the one array, so
 * calls that overlap on the GPU (different streams, or different host threads) race:
 * serialise them.  Device-side routing errors (an expert id >= n_experts, a routed
 * expert without a slot) are counted in the array's error word, which each call clears
 * and nothing reads back: this entry does not report them; use bigrig_switch_glu with a
 * workspace and bigrig_workspace_errors where they must be seen.  The call itself
 * allocates nothing (no cudaMalloc/cudaFree, no library allocator). */
#define BIGRIG_NOALLOC_SCRATCH_BYTES (4u << 20)
BIGRIG_API int bigrig_switch_glu_noalloc(const void* x, const int32_t* indices, int T, int k,
                                         int n_experts, const int32_t* g2s, const void* slab,
                                         const bigrig_expert_layout* layout, void* y,
                                         void* stream);

/* ---------------------------------------------------------------------------------
 * Expert parallelism over peer memory (NVLink / NVSwitch), one process per GPU.
 *
 * No counterpart in the reference, which runs on one Mac: this is the B200 way of
 * sharding its MoE layer.  Rank r of a group of `world` GPUs owns a contiguous block of
 * every layer's experts, [first_expert, first_expert + n_local).  Each rank keeps one
 * device buffer (bigrig_peer_alloc) that every other rank maps (bigrig_peer_open of its
 * IPC handle); bigrig_peer_group lists them, in rank order, as this process sees them.
 * One layer call (bigrig_peer_layer) on every rank, `tokens` rows each:
 *   1. gather   each rank stores its rows into every rank's buffer and raises a flag
 *               there; each waits for all ranks' flags (all world * tokens rows present);
 *   2. route    the replicated router over all rows: logits, top-k, scores;
 *   3. experts  this rank's experts over the pairs routed to them (the others are
 *               padding), the same kernels as bigrig_switch_glu;
 *   4. scatter  each pair's output row is stored into the buffer of the rank that owns
 *               the pair's token, at the pair's (token, k) place; a flag per source rank;
 *   5. combine  each rank waits for every rank's flag and forms
 *               out = residual + sum_j score * y for its own rows, in k order -- the
 *               combine of bigrig_moe_layer, so results match one GPU holding every
 *               expert to the expert kernels' own tolerance.
 * Flags are 64-bit counters written with release stores at system scope and polled with
 * acquire loads; every wait is bounded (wait_ms of GPU time): past it the layer counts
 * a timeout in the group's error word (bigrig_peer_errors), stops waiting for the rest
 * of the process's calls until that word is cleared, and finishes (its output is then
 * not meaningful).  Every rank must make the same sequence of calls with the same
 * `tokens`, and keep their hosts within wait_ms of each other (a rank whose host is busy
 * elsewhere -- loading, compiling, a long synchronous step -- must first meet the others
 * at a host barrier).  All of it is ordinary kernel launches on `stream` and can be
 * captured in a CUDA graph.  Peer memory is only read and written by plain loads and
 * stores. */
#define BIGRIG_PEER_MAX_RANKS 8
#define BIGRIG_PEER_HANDLE_BYTES 64

typedef struct {
  int32_t world;     /* ranks in the group, <= BIGRIG_PEER_MAX_RANKS */
  int32_t rank;      /* this process's rank */
  int32_t tokens;    /* rows every rank brings to each layer call */
  int32_t hidden;    /* H of the layers the group serves */
  int32_t top_k;     /* k of the layers the group serves */
  int32_t wait_ms;   /* bound on each wait for another rank, ms of GPU time; 0: 10000 */
  void* base[BIGRIG_PEER_MAX_RANKS]; /* rank i's buffer as mapped here (base[rank]: own) */
} bigrig_peer_group;

/* Bytes of one rank's peer buffer for a group of this shape. */
BIGRIG_API size_t bigrig_peer_buffer_bytes(int world, int tokens, int hidden, int top_k);

/* Allocate a zero-filled peer buffer on the current device and write its IPC handle
 * (BIGRIG_PEER_HANDLE_BYTES bytes) to `handle`; bigrig_peer_free releases it.  Set-up
 * only (cudaMalloc, a device synchronisation). */
BIGRIG_API int bigrig_peer_alloc(size_t bytes, void** ptr, void* handle);
BIGRIG_API int bigrig_peer_free(void* ptr);

/* Map another rank's buffer from its handle into this process (peer access enabled on
 * first use); bigrig_peer_close unmaps it.  A handle of this process's own buffer is
 * refused: use the pointer bigrig_peer_alloc returned. */
BIGRIG_API int bigrig_peer_open(const void* handle, void** ptr);
BIGRIG_API int bigrig_peer_close(void* ptr);

/* Scratch of one bigrig_peer_layer call (bigrig_moe_workspace_bytes for all
 * world * tokens rows over the n_local experts, laid out as for the other entry points so
 * one workspace serves them all, then the route and expert outputs of those rows);
 * zero-filled once, like the other workspaces. */
BIGRIG_API size_t bigrig_peer_workspace_bytes(const bigrig_peer_group* group, int n_experts,
                                              int n_local, const bigrig_expert_layout* layout);

/* One MoE layer of the group (steps 1-5 above) for this rank's `group->tokens` rows:
 * x, residual (may be NULL), out bf16 [tokens, H]; gate_w bf16 [E, H], gate_b fp32 [E] or
 * NULL (the full router, identical on every rank); g2s int32 [n_local] maps this rank's
 * experts (numbered from 0) to slots of `slab`.  Returns after issuing the launches. */
BIGRIG_API int bigrig_peer_layer(const bigrig_peer_group* group, const void* x,
                                 const void* gate_w, const float* gate_b, int E, int mode,
                                 int norm_topk, int first_expert, int n_local,
                                 const int32_t* g2s, const void* slab,
                                 const bigrig_expert_layout* layout, const void* residual,
                                 void* out, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* The group's wait-timeout count in this rank's buffer, read synchronously on `stream`
 * into *out and reset to 0 (which also re-arms the waits). */
BIGRIG_API int bigrig_peer_errors(const bigrig_peer_group* group, int32_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BIGRIG_B200_H */
