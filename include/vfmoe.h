/*
 * vfmoe.h -- C ABI of libvfmoe.so, the B200 (sm_100a) GLM-style MoE layer.
 *
 * Drop-in for the MoE path of rickenator/VybForge (paths relative to that
 * project).  The reference crosses its device boundary with PTX kernels that
 * take ONE pointer to a params block of 8-byte words
 * (native/kernels/moe.vyb:15-19), launched through cuda_launch4i /
 * tensor::launch1 (native/host/moe_driver.vyb:20-23,150; native/tensor/tensor.vyb:173-181),
 * and with host loops in native/glm53/glm_engine.vyb:2728-2991.  This header
 * replaces those entry points with plain extern "C" functions:
 *
 *   - every device address, stream and handle is an int64_t (a Vyb `Int`);
 *   - every status is an int: 0 = OK, negative = error (VFMOE_ERR_*), mirroring
 *     the CUresult checks of moe_driver.vyb:101-160; the library never exits
 *     or aborts, and vfmoe_last_error() returns the message;
 *   - descriptors are structs made only of 8-byte words (int64_t / double), so
 *     a host without struct FFI can build one as a params block of words;
 *   - all device work is enqueued on the caller's stream (0 = legacy default
 *     stream); no call synchronizes except where stated;
 *   - the caller owns activations, outputs and weights (weights are borrowed,
 *     never freed); the library owns handle state and, only when the caller
 *     passes workspace = 0, an internal workspace it grows on demand.
 *
 * Data formats
 *   x        [T, hidden], dtype VFMOE_DT_BF16 or VFMOE_DT_F32
 *   router   W_r fp32 [n_experts, hidden], selection bias fp32 [n_experts]
 *   Q8_0     per matrix: output rows, each K/32 GGUF blocks of 34 bytes
 *            (fp16 d, int8 q[32]); gate/up [inter][hidden], down [hidden][inter]
 *            (or the same blocks stage-tiled, VFMOE_WFMT_Q8_0_TILED / vfmoe_q8_0_tile)
 *   EXL3     per matrix (in, out) = (K, N): trellis uint16 [K/16][N/16][16*bits],
 *            suh fp16 [K], svh fp16 [N] (native/exl3/README.md:26-31)
 *   idx      int32 [T, topk] (the reference stores float32, moe.vyb:76)
 *   w        fp32 [T, topk]
 *   out      [T, hidden], dtype VFMOE_DT_BF16 or VFMOE_DT_F32
 */
#ifndef VFMOE_H
#define VFMOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VFMOE_ABI_VERSION 3

/* status codes */
#define VFMOE_OK 0
#define VFMOE_ERR_INVALID (-1)     /* bad argument or descriptor */
#define VFMOE_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define VFMOE_ERR_NOMEM (-3)       /* device allocation failed */
#define VFMOE_ERR_HANDLE (-4)      /* unknown or destroyed handle */
#define VFMOE_ERR_WORKSPACE (-5)   /* caller workspace smaller than vfmoe_workspace_bytes */
#define VFMOE_ERR_DEVICE (-6)      /* a kernel flagged an error (bounded wait expired, bad id) */
#define VFMOE_ERR_UNSUPPORTED (-7) /* shape or format not supported by this build */
#define VFMOE_ERR_NCCL (-8)        /* NCCL unavailable or an NCCL call failed */

/* dtype ids: identical to native/dtype/dtype.vyb:26-28 (dt_f32/dt_f16/dt_bf16) */
#define VFMOE_DT_F32 0
#define VFMOE_DT_F16 1
#define VFMOE_DT_BF16 2

/* expert weight formats */
#define VFMOE_WFMT_Q8_0 1
#define VFMOE_WFMT_EXL3 2
/* Q8_0 blocks of the same matrices in stage-tiled order (no counterpart in the reference,
 * which reads GGUF rows; made from GGUF rows by vfmoe_q8_0_tile at load time): a matrix
 * [rows][K] is tiles of 64 rows x 256 K, 64 x 272 B each (every tile row = that row's 8
 * GGUF blocks), tile (rt, kr) at byte ((rt * K/256) + kr) * 17408.  Same size, expert
 * strides and values as GGUF rows; the expert kernels stream one tile as one contiguous
 * copy.  Not accepted by the SIMT path (VFMOE_PATH_SIMT). */
#define VFMOE_WFMT_Q8_0_TILED 3
/* Dense bf16 matrices, rows = output channels ([out][in], the Hugging Face layout).  Accepted for
 * the shared expert (vfmoe_layer_desc.shared_format): GLM-5.3 stores its routed experts EXL3 and
 * its shared expert bf16.  Converted to fp16 at create (exact for |w| in [2^-14, 65504]; smaller
 * values keep an absolute error below 2^-25) and run by a dense variant of the decode GEMV. */
#define VFMOE_WFMT_BF16 4

/* Expert-product kernels (vfmoe_layer_desc.expert_path).  AUTO picks per call: the decode GEMV
 * (register-operand tensor-core MMAs) while the routed rows average at most 16 per expert, the
 * tcgen05 grouped GEMM above that; fp32 activations (x_dtype F32) always take the decode GEMV in its
 * split-precision form (fp16 hi + lo operand planes, about fp32 accuracy).  The other values force
 * one kernel family for every call: TC the tcgen05 GEMM (fp16 operands, also for fp32 x), GEMV the
 * decode GEMV, SIMT the plain-SIMT kernels that the tensor-core paths are checked against (GGUF
 * row order only).  EXL3 layers choose between their own GEMV and GEMM by the same row rule. */
#define VFMOE_PATH_AUTO 0
#define VFMOE_PATH_SIMT 1
#define VFMOE_PATH_TC 2
#define VFMOE_PATH_GEMV 3
/* TC1: the tcgen05 GEMM with single-CTA tiles only.  AUTO and TC run tiles of N >= 32 token rows
 * on CTA pairs (tcgen05 cta_group::2: 256 channels per tile, 128 per SM); TC1 is the form they are
 * checked against. */
#define VFMOE_PATH_TC1 4

/* One projection (gate, up or down) of a stack of experts.  Expert e's data
 * starts at data + e * expert_stride (bytes); for EXL3 its suh/svh start at
 * suh + e * suh_stride and svh + e * svh_stride.  For a single matrix (the
 * shared expert) the strides are ignored. */
typedef struct vfmoe_matrix {
    int64_t data;
    int64_t expert_stride;
    int64_t suh;
    int64_t suh_stride;
    int64_t svh;
    int64_t svh_stride;
} vfmoe_matrix;

/* One MoE layer (native/glm53/moe_ref.py:25-30 constants become fields;
 * moe.vyb's params block +8 gateW, +16 bias, +56..+96 expert/shared weights). */
typedef struct vfmoe_layer_desc {
    int64_t hidden;         /* H */
    int64_t inter;          /* moe_intermediate I */
    int64_t n_experts;      /* routed experts E */
    int64_t topk;           /* k */
    int64_t weight_format;  /* VFMOE_WFMT_* */
    int64_t exl3_bits;      /* 3 or 4 when weight_format == VFMOE_WFMT_EXL3 */
    int64_t x_dtype;        /* VFMOE_DT_BF16 or VFMOE_DT_F32 */
    int64_t out_dtype;      /* VFMOE_DT_BF16 or VFMOE_DT_F32 */
    double routed_scale;    /* routed_scaling_factor, 2.5 in GLM (moe_ref.py:29) */
    double swiglu_limit;    /* 10.0 in GLM (moe_ref.py:30) */
    int64_t router_w;       /* fp32 [E, H] */
    int64_t router_bias;    /* fp32 [E], e_score_correction_bias (selection only) */
    vfmoe_matrix gate, up, down;          /* routed experts, stacked over E */
    vfmoe_matrix sh_gate, sh_up, sh_down; /* shared expert; sh_gate.data == 0: none */
    int64_t n_local_experts; /* routed experts whose weights gate/up/down hold; 0 = n_experts.
                                Fewer on an expert-parallel rank (vfmoe_forward_rows only). */
    int64_t expert_path;     /* VFMOE_PATH_*; 0 = AUTO */
    int64_t shared_format;   /* format of sh_gate/sh_up/sh_down: 0 = weight_format, or VFMOE_WFMT_BF16 */
} vfmoe_layer_desc;

/* ABI version (VFMOE_ABI_VERSION). */
int vfmoe_version(void);

/* Select the CUDA device for the calling thread and check it is sm_100.
 * Replaces tensor_init (native/tensor/tensor.vyb:32-45). */
int vfmoe_init(int device);

/* Copy the calling thread's last error message into buf (NUL-terminated,
 * at most n bytes).  Returns the message length. */
int vfmoe_last_error(char *buf, int64_t n);

/* Validate a layer descriptor and build its launch state (tensor maps, tile
 * plans).  Returns a handle > 0, or a negative VFMOE_ERR_*. */
int64_t vfmoe_layer_create(const vfmoe_layer_desc *desc);

/* Release a handle and any internal workspace it owns. */
int vfmoe_layer_destroy(int64_t handle);

/* Bytes of workspace vfmoe_forward / vfmoe_route need for up to t_max tokens. */
int64_t vfmoe_workspace_bytes(int64_t handle, int64_t t_max);

/* Router only: idx int32 [T, topk], w fp32 [T, topk] from x [T, H].
 * logits = x . W_r^T, score = sigmoid(logit), top-k on score + bias (lowest
 * index wins ties), w = score / (sum + 1e-20) * scale.  The selection equals the
 * one made on exact (fp64) logits: fp32 logits with rigorous error bounds pick the
 * candidates, float-float and then fp64 arithmetic order those whose bounds overlap.
 * Replaces moe_route (native/kernels/moe.vyb:32-95) and the host router of
 * glm_engine.vyb:2728-2803.  workspace may be 0 (internal). */
int vfmoe_route(int64_t handle, int64_t x, int64_t T, int64_t idx_out, int64_t w_out,
                int64_t workspace, int64_t ws_bytes, int64_t stream);

/* The router's first level alone, for diagnostics: fp32 logits [T, n_experts] of x . W_r^T (the
 * kernel vfmoe_route would use for this T and dtype: SIMT fp32, or tcgen05 on bf16 parts of W_r
 * for bf16 x and T > 32) and *bound_out = c with |logit - exact| <= c * |x_t|_2 * |w_e|_2, the
 * bound vfmoe_route's refinement relies on.  No counterpart in the reference. */
int vfmoe_route_logits(int64_t handle, int64_t x, int64_t T, int64_t logits_out, double *bound_out,
                       int64_t workspace, int64_t ws_bytes, int64_t stream);

/* Router with no device allocation, for hosts that cannot call cudaMalloc at routing
 * time (it may synchronize the device, and it fails once the host has reserved all of
 * device memory in its own pool).  No counterpart in the reference.  Same result as
 * vfmoe_route.  Scratch is a fixed VFMOE_ROUTE_NOALLOC_SCRATCH_BYTES device array inside
 * the library, held on every GPU that loads it until exit; larger T is rejected with
 * VFMOE_ERR_UNSUPPORTED: the scratch holds the router's fp32 partial logits (T x E x K-slices)
 * plus the expert counts, which allows T <= 127 at E = 256, H = 6144 (decode batches).  The first call on a device looks
 * up the array's address; make it before any stream capture.  Calls share the array:
 * calls that overlap on the GPU race. */
#define VFMOE_ROUTE_NOALLOC_SCRATCH_BYTES (4 << 20)
int vfmoe_route_noalloc(int64_t handle, int64_t x, int64_t T, int64_t idx_out, int64_t w_out, int64_t stream);

/* Full MoE layer: out = sum_l w[t,l] * FFN_{idx[t,l]}(x[t]) + FFN_shared(x[t]),
 * FFN = clamped SwiGLU (moe_ref.py:81-112).  idx_out / w_out may be 0.
 * Replaces moe_route + moe_act + moe_down (moe.vyb:32-170) and tail_site's
 * router, expert loop and shared expert (glm_engine.vyb:2728-2991). */
int vfmoe_forward(int64_t handle, int64_t x, int64_t T, int64_t out,
                  int64_t idx_out, int64_t w_out,
                  int64_t workspace, int64_t ws_bytes, int64_t stream);

/* The dispatch step of vfmoe_forward on its own: the canonical permutation of the T*k routed
 * (token, lane) pairs, experts ascending and tokens ascending within an expert (the host gather
 * of native/glm53/glm_engine.vyb:2827-2845).  Same kernels as inside vfmoe_forward.
 *   idx      int32 [T, k] expert ids in [0, n_experts)
 *   counts   int32 [n_experts + 2]: per-expert row counts (scratch and output)
 *   offsets  int32 [n_experts + 2]: expert e's rows are [offsets[e], offsets[e+1]); offsets[E] = T*k
 *   perm_tok int32 [T*k]: token of each permuted row
 *   pos_of   int32 [T*k]: permuted row of lane (t, l) at t*k + l (-1 for an id out of range)
 * err_word: device int that records an id out of range (DEV_BAD_EXPERT_ID = 1), may be 0. */
int vfmoe_dispatch(int64_t idx, int64_t T, int64_t k, int64_t n_experts, int64_t counts, int64_t offsets,
                   int64_t perm_tok, int64_t pos_of, int64_t err_word, int64_t stream);

/* ---- expert parallelism (no counterpart in the reference, which has no multi-GPU code;
 * the exchange itself is NCCL all-to-all between these calls) ---- */

/* Bytes of workspace vfmoe_forward_rows needs for up to n_max rows. */
int64_t vfmoe_rows_workspace_bytes(int64_t handle, int64_t n_max);

/* Expert FFN on arbitrary rows: y_out[i] = FFN_{slots[i]}(rows[i]), fp32 [n, H].  slots
 * are local expert indices in [0, n_local_experts); slot == n_local_experts selects the
 * shared expert.  rows: [n, H] bf16 or fp32 (rows_dtype).  The per-expert products are the
 * ones vfmoe_forward runs (moe.vyb:98-170). */
int vfmoe_forward_rows(int64_t handle, int64_t rows, int64_t rows_dtype, int64_t slots, int64_t n, int64_t y_out,
                       int64_t workspace, int64_t ws_bytes, int64_t stream);

/* Weighted combine: out[t] = sum_l w[t,l] * y[pos_of[t*k+l]] + y_shared[t].  y rows and
 * y_shared are y_dtype VFMOE_DT_F32 or VFMOE_DT_F16; w may be 0 for weight 1; y_shared may
 * be 0; a negative pos_of entry skips that lane.  out_dtype F32, BF16 or F16.
 * glm_engine.vyb:2925-2938, :2991. */
int vfmoe_combine(int64_t y, int64_t y_dtype, int64_t pos_of, int64_t w, int64_t T, int64_t k, int64_t H,
                  int64_t y_shared, int64_t out, int64_t out_dtype, int64_t stream);

/* Bytes of workspace vfmoe_forward_routed needs for up to n_max rows of k lanes. */
int64_t vfmoe_routed_workspace_bytes(int64_t handle, int64_t n_max, int64_t k);

/* Expert products with caller routing: y_out[i] = sum_l w[i,l] * FFN_{slots[i,l]}(rows[i])
 * over the lanes with slots[i,l] >= 0 (local expert slots; n_local_experts = the shared
 * expert), lanes added in lane order.  rows [n, H] bf16 or fp32; slots int32 [n, k]; w fp32
 * [n, k] (0: weight 1); y_out [n, H] of y_dtype F32, F16 or BF16.  The expert side of the
 * token-level exchange: the received rows with their lanes, plus this rank's own rows
 * with the shared slot. */
int vfmoe_forward_routed(int64_t handle, int64_t rows, int64_t rows_dtype, int64_t n, int64_t k, int64_t slots,
                         int64_t w, int64_t y_out, int64_t y_dtype, int64_t workspace, int64_t ws_bytes,
                         int64_t stream);

/* Failure injection for tests of the device-error path (no counterpart in the reference, whose
 * drivers only check CUresult codes).  kind VFMOE_INJECT_STALL_LOADS makes the Q8_0 decode GEMV's
 * producer warp issue no weight or token loads, so every consumer's bounded wait for its first
 * stage expires after wait_ns (nothing is in flight when it does); the kernels raise
 * DEV_WAIT_TIMEOUT (2) in the device error word and return, vfmoe_check_device_error then
 * reports VFMOE_ERR_DEVICE, and the output of that call is undefined.  wait_ns = 0 keeps the
 * production bound (2 s).  VFMOE_INJECT_NONE restores normal operation. */
#define VFMOE_INJECT_NONE 0
#define VFMOE_INJECT_STALL_LOADS 1
int vfmoe_debug_inject(int64_t handle, int64_t kind, int64_t wait_ns);

/* ---- expert parallelism inside the library: NCCL between ranks, one process per GPU ----
 *
 * The reference has no multi-GPU code; these entry points serve the callers that would run the
 * MoE expert-parallel: tail_site's router, expert loop and shared expert
 * (native/glm53/glm_engine.vyb:2728-2991) and the prefill driver (native/host/glm_prefill.vyb:1458).
 *
 * Tokens are sharded over ranks; the router and the shared expert are replicated; routed experts
 * (plus optional copies of hot experts) are sharded by a placement.  Per layer forward:
 *   prepare  route this rank's T tokens, plan one send entry per (token, rank owning one of its k
 *            experts), pack the rows; entries for rank d sit at d * t_cap + i (i < count[d]).
 *   exchange every peer block is t_cap entries, whatever its count: rows (x dtype), lane slots
 *            (int32 [t_cap][k]) and lane weights (fp32 [t_cap][k]); padding entries carry slot -1.
 *   shared   the shared expert on this rank's tokens (overlaps the exchange).
 *   experts  this rank's experts on the n_ranks * t_cap received rows, each row's local lanes summed
 *            with their weights into one partial row (fp16; fp32 when out_dtype is F32).
 *   exchange partial rows back, block d to rank d.
 *   combine  out[t] = the partials returned for t, in rank order, + shared(x[t]).
 * t_cap (>= every rank's T, the same on all ranks) fixes every transfer size, so no count
 * crosses to the host and the whole forward is one stream of device work.
 * vfmoe_ep_forward runs all of it with NCCL send/recv; a host with its own transport calls the
 * phases and moves the blocks that vfmoe_ep_buffers locates. */

/* 128 bytes of NCCL unique id for vfmoe_ep_init; one rank makes it, the host shares it. */
int vfmoe_ep_unique_id(void *id_out, int64_t n);

/* Communicator over nranks processes (one GPU each, the calling thread's current device).
 * NCCL is opened at run time (libnccl.so.2; VFMOE_ERR_NCCL if absent).  Waits for every rank to
 * join for at most timeout_ms (0 = no limit); on expiry the partial communicator is aborted and
 * VFMOE_ERR_NCCL returned.  Returns a communicator handle > 0. */
int64_t vfmoe_ep_init(int64_t nranks, int64_t rank, const void *unique_id, int64_t timeout_ms);
int vfmoe_ep_destroy(int64_t comm);

/* Placement of a layer handle that holds rank `rank`'s experts (n_local_experts of them, in
 * ascending virtual id): owner int32 [n_virtual] (host) gives the rank of each virtual expert,
 * n_virtual = n_experts + n_replicas; virtual expert n_experts + j is a copy of expert
 * replica_of[j] (host int32 [n_replicas]) and takes the lanes (t, l) of that expert with t + l
 * odd.  Copies the placement to the device (call at set-up, not per forward). */
int vfmoe_ep_set_placement(int64_t handle, int64_t n_ranks, int64_t rank, const int32_t *owner, int64_t n_virtual,
                           const int32_t *replica_of, int64_t n_replicas);

/* Workspace bytes of the expert-parallel calls for capacity t_cap. */
int64_t vfmoe_ep_workspace_bytes(int64_t handle, int64_t t_cap);

/* Byte offsets in that workspace of the exchange buffers (and block sizes), indexed by: */
#define VFMOE_EP_SEND_ROWS 0
#define VFMOE_EP_RECV_ROWS 1
#define VFMOE_EP_ROWS_BLOCK 2       /* bytes of one peer block of rows */
#define VFMOE_EP_SEND_SLOTS 3
#define VFMOE_EP_RECV_SLOTS 4
#define VFMOE_EP_SEND_WEIGHTS 5
#define VFMOE_EP_RECV_WEIGHTS 6
#define VFMOE_EP_LANES_BLOCK 7      /* bytes of one peer block of slots (or of weights) */
#define VFMOE_EP_SEND_PARTIALS 8    /* partial rows computed here, block d belongs to rank d */
#define VFMOE_EP_RECV_PARTIALS 9    /* partial rows returned to this rank, block d from rank d */
#define VFMOE_EP_PARTIALS_BLOCK 10
#define VFMOE_EP_SEND_COUNTS 11     /* int32 [n_ranks]: valid entries per send block */
#define VFMOE_EP_BUF_COUNT 12
int vfmoe_ep_buffers(int64_t handle, int64_t t_cap, int64_t *offsets, int64_t n);

/* The phases (all on `stream`, no host synchronization).  Between prepare and experts the send
 * blocks of rows, slots and weights of rank d must reach rank d's receive blocks (this rank's own
 * block is already in place); between experts and combine the partial blocks likewise. */
int vfmoe_ep_prepare(int64_t handle, int64_t x, int64_t T, int64_t t_cap, int64_t idx_out, int64_t w_out,
                     int64_t workspace, int64_t ws_bytes, int64_t stream);
int vfmoe_ep_shared(int64_t handle, int64_t x, int64_t T, int64_t t_cap, int64_t workspace, int64_t ws_bytes,
                    int64_t stream);
int vfmoe_ep_experts(int64_t handle, int64_t t_cap, int64_t workspace, int64_t ws_bytes, int64_t stream);
int vfmoe_ep_combine(int64_t handle, int64_t T, int64_t t_cap, int64_t out, int64_t workspace, int64_t ws_bytes,
                     int64_t stream);

/* The whole expert-parallel layer forward over NCCL: out [T, H] for this rank's x [T, H].
 * The dispatch exchange runs on the communicator's own stream, forked from and joined back to
 * `stream` with events, while the shared expert runs on `stream`.  Every rank must make the
 * same calls with the same t_cap.  idx_out / w_out (optional) receive the routing. */
int vfmoe_ep_forward(int64_t comm, int64_t handle, int64_t x, int64_t T, int64_t t_cap, int64_t out, int64_t idx_out,
                     int64_t w_out, int64_t workspace, int64_t ws_bytes, int64_t stream);

/* Synchronize `stream` and report whether any kernel of this handle flagged a
 * device-side error since the last call (VFMOE_ERR_DEVICE), then clear it. */
int vfmoe_check_device_error(int64_t handle, int64_t stream);

/* Per-stage device timing (replaces the reference's T_MOE / MMT / DEQT wall-clock tag
 * lines, native/glm53/glm_engine.vyb:2951).  enable = 1 makes every later
 * vfmoe_forward on this handle record CUDA events on its stream between stages. */
int vfmoe_profile_enable(int64_t handle, int enable);

/* Synchronize on the recorded events and return, in stage_ms[0..n), the summed
 * device milliseconds per stage since the last read: 0 router, 1 dispatch+gather,
 * 2 gate/up+SwiGLU, 3 down, 4 combine (vfmoe_ep_forward: 0 route+plan+pack, 1 shared expert,
 * 2 wait for the dispatch exchange, 3 experts, 4 return exchange, 5 combine).  *launches (if non-null) gets the number of
 * kernels launched by those forwards.  Returns the number of forwards measured and
 * resets the accumulators. */
int vfmoe_profile_read(int64_t handle, double *stage_ms, int64_t n, int64_t *launches);

/* RMSNorm: y = x * w / sqrt(mean(x^2) + eps) over rows of D, x/y dtype
 * VFMOE_DT_BF16 or VFMOE_DT_F32, w fp32 [D].  Replaces tensor::rmsnorm
 * (native/tensor/tensor.vyb:217-231, kernel native/kernels/rmsnorm.vyb). */
int vfmoe_rmsnorm(int64_t x, int64_t w, int64_t y, int64_t S, int64_t D, double eps,
                  int64_t dtype, int64_t stream);

/* Residual step of a pre-norm layer stack, one pass over S rows of D:
 *   x_out = x + y           when y != 0 (rounded to dtype)
 *   h     = RMSNorm_w(x_out or x)   when w != 0 (statistics of the rounded values)
 * so layer l's residual add and layer l+1's input norm share a kernel.  The
 * reference stack (native/glm53/glm_engine.vyb) mixes layers through
 * hyper-connections; this entry implements the plain residual x + MoE(RMSNorm(x))
 * of the expert-parallel stack and has no single reference counterpart.
 * dtype VFMOE_DT_BF16 or VFMOE_DT_F32; w fp32 [D]; x_out may alias x. */
int vfmoe_residual_rmsnorm(int64_t x, int64_t y, int64_t w, int64_t x_out, int64_t h, int64_t S,
                           int64_t D, double eps, int64_t dtype, int64_t stream);

/* ---- hyper-connections around the MoE (GLM-5.3 multi-stream residual) ----
 * A layer keeps n_streams = 4 residual streams of width hidden per token, fp32 [R][4][hidden].
 * Per sublayer site the checkpoint holds fn [24][4 * hidden] (bf16 or fp32; 24 = 4 pre + 4 post
 * + 16 comb), base fp32 [24] and scale fp32 [3]. */
typedef struct vfmoe_hc_desc {
    int64_t n_streams;      /* 4 */
    int64_t hidden;         /* D: 2048, 4096, 6144 or 8192 */
    int64_t fn;             /* device [24][4 * hidden] */
    int64_t fn_dtype;       /* VFMOE_DT_BF16 or VFMOE_DT_F32 */
    int64_t base;           /* device fp32 [24] */
    int64_t scale;          /* device fp32 [3]: pre, post, comb */
    double rms_eps;         /* unweighted RMSNorm of the flattened streams */
    double hc_eps;          /* 1e-6 in GLM-5.3 */
    int64_t sinkhorn_iters; /* 20 in GLM-5.3 */
    int64_t norm_w;         /* device fp32 [hidden]: the layernorm before the sublayer; 0 = none */
    double norm_eps;
} vfmoe_hc_desc;

/* Mix (hc_glue, native/glm53/glm_engine.vyb:437-612; hc_ref.mix, native/glm53/hc_ref.py:27-57)
 * fused with the RMSNorm that feeds the sublayer:
 *   pre, post, comb from RMSNorm(streams[r]) . fn^T (Sinkhorn-normalised comb),
 *   h[r] = RMSNorm_norm_w(sum_h pre[h] * streams[r, h])   (h_dtype BF16 or F32)
 * post fp32 [R][4] and comb fp32 [R][4][4] are kept for vfmoe_hc_apply. */
int vfmoe_hc_mix(const vfmoe_hc_desc *desc, int64_t streams, int64_t R, int64_t h_out, int64_t h_dtype,
                 int64_t post_out, int64_t comb_out, int64_t stream);

/* Apply (hc_apply, glm_engine.vyb:783-809; hc_ref.apply_, hc_ref.py:60-63):
 *   out[r, h] = post[r, h] * y[r] + sum_j comb[r, j, h] * streams[r, j]
 * y [R][hidden] (y_dtype BF16 or F32), out fp32 [R][4][hidden]; out may be streams itself. */
int vfmoe_hc_apply(int64_t streams, int64_t y, int64_t y_dtype, int64_t post, int64_t comb, int64_t R,
                   int64_t n_streams, int64_t hidden, int64_t out, int64_t stream);

/* ---- packed layer files (replace the reference's dequant cache, native/glm53/deq_cache.vyb:1-93,
 * which stores dequantized f64 tensors): the router and the expert stacks on disk in the byte
 * layout the kernels stream (stage-tiled Q8_0 or EXL3 trellis + suh/svh), 4096-aligned sections
 * behind a 4096-byte header holding the descriptor with device pointers as offsets. ---- */

/* Write the layer that desc describes (device pointers) to path.  Synchronous. */
int vfmoe_pack_save(const char *path, const vfmoe_layer_desc *desc);
/* Device bytes a vfmoe_pack_load of path needs (or a negative status). */
int64_t vfmoe_pack_bytes(const char *path);
/* Read path into the caller's device buffer (256-byte aligned, at least vfmoe_pack_bytes) with
 * chunked reads through pinned staging buffers, and fill *desc_out with pointers into it, ready
 * for vfmoe_layer_create.  Synchronous; allocates only the pinned staging. */
int vfmoe_pack_load(const char *path, int64_t dev_base, int64_t dev_bytes, vfmoe_layer_desc *desc_out);

/* ---- checkpoint access: safetensors shards behind model.safetensors.index.json ----
 * Replaces the gx index (native/glm53/gx.vyb:41-99: gx_shard_for, gx_resolve) and the safetensors
 * reader (native/torchload/safetensors.vyb): a name resolves through the index to its shard, the
 * shard's header (parsed once, checked against the file's size) to its dtype, shape and byte range,
 * and the bytes are read straight into host or device memory.  A directory without an index is
 * read as the single file model.safetensors. */
#define VFMOE_ST_F32 0
#define VFMOE_ST_F16 1
#define VFMOE_ST_BF16 2
#define VFMOE_ST_F64 3
#define VFMOE_ST_I64 4
#define VFMOE_ST_I32 5
#define VFMOE_ST_I16 6
#define VFMOE_ST_I8 7
#define VFMOE_ST_U8 8
#define VFMOE_ST_BOOL 9
#define VFMOE_ST_U16 10
#define VFMOE_ST_U32 11
#define VFMOE_ST_U64 12
#define VFMOE_ST_F8_E4M3 13
#define VFMOE_ST_F8_E5M2 14

typedef struct vfmoe_tensor_info {
    int64_t dtype;        /* VFMOE_ST_* */
    int64_t ndim;
    int64_t shape[8];
    int64_t nbytes;
    int64_t file_offset;  /* absolute offset of the data in its shard */
    int64_t shard;        /* index of the shard file */
} vfmoe_tensor_info;

int64_t vfmoe_ckpt_open(const char *dir);
int vfmoe_ckpt_close(int64_t ckpt);
/* dtype, shape and byte range of a tensor (VFMOE_ERR_INVALID if the checkpoint lacks it). */
int vfmoe_ckpt_find(int64_t ckpt, const char *name, vfmoe_tensor_info *info);
/* The tensor's bytes into dst (device memory when device != 0, through pinned staging; else host
 * memory).  Synchronous. */
int vfmoe_ckpt_read(int64_t ckpt, const char *name, int64_t dst, int64_t dst_bytes, int64_t device);

/* Q8_0 rows -> dense [rows, k] (dst_dtype VFMOE_DT_F32 or VFMOE_DT_F16).
 * Replaces q8_0deq (native/kernels/q8_0.vyb:11-30, which widens to f64). */
int vfmoe_q8_0_dequant(int64_t src, int64_t dst, int64_t rows, int64_t k,
                       int64_t dst_dtype, int64_t stream);

/* fp32 [rows, k] -> Q8_0 rows (ggml quantize_row_q8_0_ref rule; the reference
 * has no quantizer, it reads GGUF bytes). */
int vfmoe_q8_0_quantize(int64_t src_f32, int64_t dst, int64_t rows, int64_t k, int64_t stream);

/* n_mats Q8_0 matrices [rows][k] in GGUF row order, back to back, -> the same matrices in
 * VFMOE_WFMT_Q8_0_TILED order at dst (same total size; dst must not overlap src).
 * rows % 64 == 0, k % 256 == 0, both pointers 16-byte aligned.  No counterpart in the
 * reference (a load-time layout step; its kernels read GGUF rows in place). */
int vfmoe_q8_0_tile(int64_t src, int64_t dst, int64_t rows, int64_t k, int64_t n_mats, int64_t stream);

/* EXL3 trellis -> rotated-basis values W^ as fp16 [K, N] (no Hadamard).
 * Replaces exl3deq / exl3deq32 (native/kernels/exl3.vyb:207-242,375-422).
 * bits = 3 (layout defined by this library) or 4 (the reference's format: its slot map,
 * native/exl3/map.bin and exl3_ref.py:66-107, applied in closed form); trellis 16-byte
 * aligned, 16*bits uint16 words per 16x16 tile. */
int vfmoe_exl3_decode(int64_t trellis, int64_t dst_f16, int64_t K, int64_t N, int64_t bits,
                      int64_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VFMOE_H */
