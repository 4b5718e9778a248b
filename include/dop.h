/*
 * dop.h — C ABI of the B200 tensor-lens library (libdop.so).
 *
 * The reference crate (dependent-optics, Rust) exposes its tensor lenses as
 * Rust functions: `mixtral::forward_backward` and the private block lens
 * `forward_layer`/`backward_layer` (src/mixtral.rs), and the small programs of
 * src/kernel.rs.  This header is the drop-in boundary a foreign caller (a Rust
 * `extern "C"` block, Python ctypes, C++) binds.  Conventions:
 *
 *   - every entry point returns an int status: 0 ok, < 0 a DOP_E_* code;
 *     dop_last_error() returns the message of the calling thread's last error;
 *   - device buffers are caller-owned and passed as plain pointers; residuals
 *     ("tapes") are owned by the lens handle that wrote them;
 *   - streams are passed as `void*` (a cudaStream_t; NULL = legacy stream);
 *   - parameter slices use the crate's flat layout: every matrix is row-major
 *     with the contraction index first, W[k * dout + n] (src/mixtral.rs:101-102);
 *   - parameter adjoints are ACCUMULATED (+=), as `add_assign` into `grad`
 *     in src/mixtral.rs:473-593; program adjoints (src/kernel.rs:342,351) are
 *     assigned.
 *
 * Precision: DOP_F32 computes every contraction in fp32 (the crate's own
 * arithmetic); DOP_BF16 keeps weights and GEMM operands in bf16 with fp32
 * accumulation, the residual stream and all adjoints in fp32.
 */
#ifndef DOP_H
#define DOP_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ errors */
#define DOP_OK 0
#define DOP_E_INVALID (-1)      /* bad argument (shape, null pointer, config) */
#define DOP_E_CUDA (-2)         /* a CUDA runtime/driver call failed */
#define DOP_E_NOMEM (-3)        /* device allocation failed */
#define DOP_E_UNSUPPORTED (-4)  /* shape outside what the kernels implement */
#define DOP_E_STATE (-5)        /* call order violated (backward before forward) */
#define DOP_E_NCCL (-6)         /* a collective failed */
#define DOP_E_TIMEOUT (-7)      /* a bounded device wait ran out */
/* cluster.rs StageError variants (src/cluster.rs:265-292) */
#define DOP_E_NO_DEVICE (-20)
#define DOP_E_PARAMS_EXCEED_CLUSTER (-21)
#define DOP_E_TAPE_EXCEEDS_CLUSTER (-22)
#define DOP_E_TILE_EXCEEDS_DEVICES (-23)
#define DOP_E_CODE_EXCEEDS_DEVICES (-24)
#define DOP_E_ROUTE_UNAVAILABLE (-25)

/* Message of the calling thread's last failed call ("" if none). */
const char* dop_last_error(void);
/* Library version string. */
const char* dop_version(void);

/* --------------------------------------------------------------- precision */
#define DOP_F32 0
#define DOP_BF16 1

/* ------------------------------------------------------------ Mixtral config
 * Field-for-field the crate's `MixtralConfig` (src/mixtral.rs:34-48).
 * `sliding_window` counts the keys a query may attend to, itself included. */
typedef struct dop_mixtral_cfg {
  int64_t vocab;
  int64_t dim;
  int64_t layers;
  int64_t heads;
  int64_t kv_heads;
  int64_t head_dim;
  int64_t intermediate;
  int64_t experts;
  int64_t top_k;
  float rms_eps;
  float rope_theta;
  int64_t sliding_window;
} dop_mixtral_cfg;

/* Offsets of one layer inside its own parameter slice (the slice starts at
 * `attn_norm`).  Mirrors `LayerLayout` (src/mixtral.rs:115-126); gate/up/down
 * of expert e are at gate0 + e * expert_stride etc. */
typedef struct dop_layer_layout {
  int64_t attn_norm, q, k, v, o, ffn_norm, router;
  int64_t gate0, up0, down0, expert_stride;
  int64_t total; /* floats in one layer slice */
} dop_layer_layout;

/* `layout` (src/mixtral.rs:128-181) for one layer, and the whole-model count
 * `parameter_count` (src/mixtral.rs:183-185). */
int dop_layer_layout_of(const dop_mixtral_cfg* cfg, dop_layer_layout* out);
int64_t dop_parameter_count(const dop_mixtral_cfg* cfg);

/* ---------------------------------------------------------- the block lens
 * One Mixtral block as a lens.  get: x[T,D] -> y[T,D] (+ residual kept in the
 * handle); put: (residual, dy) -> dx, dparams += grad.  Replaces the crate's
 * `forward_layer` (src/mixtral.rs:291-380) and `backward_layer`
 * (src/mixtral.rs:434-598).  T = batch * seq, t = b * seq + s.
 *
 * `params` is the layer's parameter slice (dop_layer_layout order) on the
 * device: fp32 for DOP_F32, bf16 (uint16 bit patterns) for DOP_BF16.
 * `x`, `y`, `dy`, `dx` are fp32 device arrays [T, D]; `dparams` is an fp32
 * device array of dop_layer_layout.total floats that is accumulated into.
 * `router_bias` (may be NULL) is an fp32 device array [E] added to the router
 * logits before the softmax (the skewed-routing workload; the crate has none). */
typedef struct dop_block dop_block;

int dop_block_create(const dop_mixtral_cfg* cfg, int64_t batch, int64_t seq,
                     int precision, dop_block** out);
int dop_block_destroy(dop_block* blk);
int dop_block_set_router_bias(dop_block* blk, const float* router_bias);
int dop_block_forward(dop_block* blk, const void* params, const float* x,
                      float* y, void* stream);
int dop_block_backward(dop_block* blk, const void* params, const float* dy,
                       float* dx, float* dparams, void* stream);
/* Bytes of device memory the handle holds (residual + workspace). */
int64_t dop_block_workspace_bytes(const dop_block* blk);

/* Routing decisions of the last forward, copied to device buffers:
 * top_i [T*k] int32, top_w [T*k] fp32 (renormalised gate), top_p [T*k] fp32,
 * router_probs [T*E] fp32 (any may be NULL). */
int dop_block_routing(const dop_block* blk, int32_t* top_i, float* top_w,
                      float* top_p, float* router_probs, void* stream);
/* The deterministic permutation of the last forward: for each (token, slot)
 * pair in token-major order, its row in the expert-sorted buffer
 * (slot_row [T*k] int32), the padded row offset of each expert's segment
 * (seg_off [E+1] int32) and the token of each permuted row (row_token
 * [rows] int32, -1 for padding; rows = dop_block_permuted_rows()). */
int dop_block_permutation(const dop_block* blk, int32_t* slot_row,
                          int32_t* seg_off, int32_t* row_token, void* stream);
int64_t dop_block_permuted_rows(const dop_block* blk);
/* The feed-forward input of the last forward, mid = x + attention [T, D]
 * fp32, copied to a device buffer: the router's input (src/mixtral.rs:308-312),
 * for checking the router stage on the lens's own input. */
int dop_block_ffn_input(const dop_block* blk, float* mid, void* stream);
/* Number of kernels the library launched on this handle since creation. */
int64_t dop_block_launches(const dop_block* blk);
/* Overlap of the adjoint reduction with the rest of the backward: after
 * this call, every dop_block_backward makes `stream` (a cudaStream_t; NULL
 * turns it off) wait until the experts' parameter adjoints — the layer slice
 * from gate0 to the end — are final, which happens before the attention half
 * of the backward runs.  A data-parallel caller reduces that slice on
 * `stream` while the backward continues on its own stream. */
int dop_block_set_adjoint_stream(dop_block* blk, void* stream);
/* ---------------------------------------------- expert-parallel block lens
 * One process per GPU, `world` ranks (2..8, experts % world == 0), bf16
 * only.  Rank r owns experts [r*E/world, (r+1)*E/world): it runs their
 * grouped GEMMs over the expert-sorted rows that EVERY rank routed to them
 * and accumulates only their slices of dparams (the other experts' slices
 * are left untouched; the shared slice [0, gate0) is this rank's own
 * adjoint and is summed over ranks by the caller, as in data parallelism).
 * The exchange has no counterpart in the crate (its experts run in one
 * process, src/mixtral.rs:330-357, 456-542): the owners read the sources'
 * rows and the sources read the owners' outputs through CUDA IPC mappings
 * of each other's workspaces, with four device-side barriers per step.
 * Every rank must call forward and backward the same number of times.
 * Set-up: create on every rank, exchange the DOP_IPC_HANDLE_BYTES handles
 * (e.g. an all-gather), then connect.  Destroy only after every rank's last
 * backward has completed on the device (e.g. after a host barrier). */
#define DOP_IPC_HANDLE_BYTES 64
int dop_block_create_ep(const dop_mixtral_cfg* cfg, int64_t batch, int64_t seq,
                        int precision, int rank, int world, dop_block** out);
/* Copy this rank's workspace IPC handle (DOP_IPC_HANDLE_BYTES bytes). */
int dop_block_ep_handle(const dop_block* blk, void* handle);
/* Map the peers' workspaces: `handles` holds world x DOP_IPC_HANDLE_BYTES
 * bytes in rank order (this rank's own entry is ignored). */
int dop_block_ep_connect(dop_block* blk, const void* handles);

/* Per-phase device timing (CUDA events on the caller's stream around each
 * phase of forward/backward: "expert_gate_up", "attn_fwd", ...).  Off by
 * default; dop_block_phase() synchronises the phase's events. */
int dop_block_set_timing(dop_block* blk, int on);
int dop_block_phase_count(const dop_block* blk);
int dop_block_phase(const dop_block* blk, int i, const char** name, float* ms);

/* ---------------------------------------------------------- the model lens
 * `mixtral::forward_backward` (src/mixtral.rs:245-261): embed, `layers`
 * block lenses, final RMSNorm, LM head, mean next-token cross-entropy
 * (:966-991), and the adjoint of every parameter.  `params` is the whole
 * flat parameter vector in `layout` order (fp32 or bf16 per precision);
 * tokens/targets are device int64 [batch*seq]; `loss` is a device float;
 * `dparams` (fp32, dop_model_parameter_count floats) is OVERWRITTEN with a
 * fresh adjoint, like the crate's returned `grad`; `logits` (fp32
 * [batch*seq, vocab], may be NULL) receives the logits.  Each layer keeps its
 * own residual, so memory grows with `layers` x the block workspace. */
typedef struct dop_model dop_model;
int dop_model_create(const dop_mixtral_cfg* cfg, int64_t batch, int64_t seq,
                     int precision, dop_model** out);
int dop_model_destroy(dop_model* m);
int dop_model_forward_backward(dop_model* m, const void* params,
                               const int64_t* tokens, const int64_t* targets,
                               float* loss, float* dparams, float* logits,
                               void* stream);
int64_t dop_model_parameter_count(const dop_model* m);

/* ------------------------------------------------------- lens composition
 * `compose(g, f)` means g after f (src/dlens.rs:74-113; README "compose(g, f)
 * always means g ∘ f").  Forward runs f then g; backward runs g's put then
 * f's; the composite residual is the pair of residuals.  A lens is a block or
 * a composite; composites own no memory beyond a scratch activation buffer. */
typedef struct dop_lens dop_lens;
int dop_lens_from_block(dop_block* blk, const void* params, float* dparams,
                        dop_lens** out);
int dop_compose(dop_lens* g, dop_lens* f, dop_lens** out);
int dop_lens_forward(dop_lens* l, const float* x, float* y, void* stream);
int dop_lens_backward(dop_lens* l, const float* dy, float* dx, void* stream);
int dop_lens_destroy(dop_lens* l);

/* ---------------------------------------------------- kernel.rs programs
 * Mirrors `Stage` / `Program` (src/kernel.rs:27-61).  Offsets index the flat
 * f32 tape, the u8 mask tape and the flat parameter vector exactly as the
 * crate's builders lay them out (src/kernel.rs:78-170). */
#define DOP_STAGE_GEMM 0
#define DOP_STAGE_ATTENTION 1
#define DOP_STAGE_ADD 2
typedef struct dop_stage {
  int32_t kind;
  int32_t relu;
  int64_t batch, din, dout;       /* Gemm */
  int64_t save_at, mask_at, param_at;
  int64_t tokens, dim, x_at, probs_at; /* Attention (uses batch too) */
  int64_t from, len;              /* Add */
} dop_stage;

typedef struct dop_program dop_program;
int dop_program_create(const dop_stage* stages, int64_t n_stages,
                       int64_t input_len, int64_t output_len,
                       int64_t param_len, int64_t tape_f32, int64_t tape_u8,
                       dop_program** out);
int dop_program_destroy(dop_program* prog);
/* Number of kernels the library launched on this handle since creation. */
int64_t dop_program_launches(const dop_program* prog);
/* get: y = program(x); the residual stays in the handle.  Forward and
 * backward only enqueue work on `stream` (no allocation, no host
 * synchronisation), so a training step can be captured in a CUDA graph. */
int dop_program_forward(dop_program* prog, const float* x, const float* params,
                        float* y, void* stream);
/* put: dy (NULL = the crate's sum loss, dy = 1, src/kernel.rs:237) ->
 * dx, dparams (assigned). */
int dop_program_backward(dop_program* prog, const float* params,
                         const float* dy, float* dx, float* dparams,
                         void* stream);
/* `kernel::forward_backward` (src/kernel.rs:181-240) in one call. */
int dop_program_forward_backward(dop_program* prog, const float* x,
                                 const float* params, const float* dy,
                                 float* y, float* dx, float* dparams,
                                 void* stream);
/* Mean-squared-error head: loss = mean((y - t)^2), dy = 2 (y - t) / n.
 * `loss` is a device float. */
int dop_mse_loss_grad(const float* y, const float* target, int64_t n,
                      float* loss, float* dy, void* stream);

/* --------------------------------------------------------------- linear
 * The crate's `linear` contraction (src/mixtral.rs:616-659) on the tensor
 * cores: C[m, n] (+)= sum_k A(m, k) B(k, n) with bf16 A, B and fp32
 * accumulation.  A(m, k) = A[m*lda + k] (a_t = 0) or A[k*lda + m] (a_t = 1);
 * B(k, n) = B[k*ldb + n] (b_t = 0, the crate's W[k*dout + n]) or
 * B[n*ldb + k] (b_t = 1).  C is fp32 (c_f32 = 1) or bf16; accumulate = 1 adds
 * into an fp32 C.  Leading dimensions must be multiples of 8 elements and the
 * pointers 16-byte aligned. */
int dop_gemm_bf16(int64_t M, int64_t N, int64_t K, const uint16_t* A, int64_t lda,
                  int a_t, const uint16_t* B, int64_t ldb, int b_t, void* C,
                  int64_t ldc, int c_f32, int accumulate, void* stream);
/* ------------------------------------------------------------ attention
 * The crate's sliding-window grouped-query attention as a lens, gqa_forward /
 * gqa_backward (src/mixtral.rs:799-922): q [B*S, H, hd], k/v [B*S, KV, hd]
 * (post-RoPE), key j visible from query i iff j <= i && i - j < window, scale
 * 1/sqrt(hd).  The residual is lse [B, H, S] (log-sum-exp of the scaled
 * scores) instead of the probabilities.  Precision DOP_BF16 takes bf16 q/k/v/o
 * and runs on the tensor cores when hd == 128; DOP_F32 takes fp32 tensors.
 * Backward writes fp32 dq/dk/dv and needs `delta_ws`, B*H*S floats of scratch. */
int dop_gqa_forward(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads,
                    int64_t head_dim, int64_t window, int precision, const void* q,
                    const void* k, const void* v, void* o, float* lse, void* stream);
int dop_gqa_backward(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads,
                     int64_t head_dim, int64_t window, int precision, const void* q,
                     const void* k, const void* v, const void* o, const void* dout,
                     const float* lse, float* delta_ws, float* dq, float* dk, float* dv,
                     void* stream);

/* The fp32 attention backward of dop_gqa_backward(..., DOP_F32, ...) for
 * callers that may not allocate device memory (their memory belongs to
 * another allocator, e.g. a framework's pool or a fixed arena): no delta_ws
 * argument and no allocation inside the call.  It has no counterpart in the
 * reference crate.  Its scratch is a 4 MiB array inside libdop's own device
 * memory, held on every GPU that loads the library until exit, so it accepts
 * batch * heads * seq <= 1,048,576 and rejects larger shapes with
 * DOP_E_INVALID.  A call made while its stream is not capturing looks the
 * array up with cudaGetSymbolAddress (with the call's device current) and
 * keeps the address per device; a call made during a capture reuses it.
 * Make the first call on a device before any stream capture, and again after
 * a cudaDeviceReset (the kept address belongs to the old context).  All
 * calls share the array: calls that overlap on the GPU race. */
int dop_gqa_backward_f32_noalloc(int64_t batch, int64_t seq, int64_t heads,
                                 int64_t kv_heads, int64_t head_dim, int64_t window,
                                 const float* q, const float* k, const float* v,
                                 const float* o, const float* dout, const float* lse,
                                 float* dq, float* dk, float* dv, void* stream);

/* ------------------------------------------------- failure detection
 * Every wait a libdop kernel makes on another agent is bounded: mbarrier
 * waits of the tensor-core kernels (TMA copies, MMAs, the other CTA of a
 * pair) and the expert exchange's flag barriers (other ranks).  A wait that
 * runs out records a code in the current device's error word, drains what
 * its CTA has in flight (bounded), frees its TMEM and returns; every later
 * libdop kernel on that device skips its work until the word is cleared.
 * The crate's counterpart is its control plane's timeout (DistError,
 * src/dist.rs:36-56).
 *
 * dop_device_status: the first code recorded on the current device (0 =
 * none): 1..59 a tensor-core kernel's mbarrier wait, 60 + k the exchange's
 * barrier k, DOP_SELFTEST_MBARRIER_CODE the self-test below. */
int dop_device_status(void);
/* Clear the current device's error word (after synchronising the device). */
int dop_clear_device_status(void);
/* Wait limits of the current device in ns of device time, 0 = the built-in
 * default (4 s per tensor-core wait, 20 s per exchange barrier). */
int dop_set_wait_limits(int64_t tensor_core_ns, int64_t exchange_ns);
/* Make one bounded wait run out on purpose, on the current device:
 * which = 0 launches one CTA that holds TMEM while it waits on an mbarrier
 * nothing arrives at (records DOP_SELFTEST_MBARRIER_CODE); which = 1 runs the
 * exchange's barrier 0 over a two-rank view of this device's own memory in
 * which rank 1's flag is never written (records 60) and waits for it.  Each
 * returns after its wait limit; nothing faults or hangs. */
#define DOP_SELFTEST_MBARRIER_CODE 90
int dop_selftest_wait_expiry(int which, void* stream);

/* ----------------------------------------------------------- utilities */
/* fp32 -> bf16 (round to nearest even), device arrays. */
int dop_f32_to_bf16(const float* src, uint16_t* dst, int64_t n, void* stream);
/* y = 2^x (device arrays, x < 128) by the polynomial the tensor-core
 * attention softmax evaluates on the FMA pipe for a quarter of its
 * exponentials; for checking its error bound.  No counterpart in the crate,
 * whose softmax calls exp (src/mixtral.rs:924-929). */
int dop_exp2_poly(const float* x, float* y, int64_t n, void* stream);
/* p <- p - lr * g, returns nothing; `sgd_step` (src/mixtral.rs:994-1001). */
int dop_sgd_step(float* params, const float* grad, int64_t n, float lr,
                 void* stream);

/* ------------------------------------------------------- staging plan
 * The cluster.rs vocabulary (src/cluster.rs:27-292) for a stack of Mixtral
 * blocks on B200s: devices and links, homes (where a block's parameters and
 * each in-flight micro-batch's residual live), windows (one block lens on
 * one micro-batch, forward or backward, on one device) with the hops that
 * deliver their inputs and carry their outputs, and the StageError codes
 * DOP_E_NO_DEVICE .. DOP_E_ROUTE_UNAVAILABLE.  A home is a whole block (a
 * B200 holds one, where the crate's planner tiles matrices for small
 * buffers): the blocks are cut into PP pipeline stages (the largest divisor
 * of both the layer count and the GPU count), the remaining GPUs hold
 * data-parallel replicas, each stage runs one-forward-one-backward over its
 * replica's micro-batches, and a final Sgd window per parameter home takes
 * the other replicas' adjoints of that block. */
#define DOP_DEVICE_CPU 0
#define DOP_DEVICE_GPU 1
typedef struct {
  char name[32];
  int32_t kind;               /* DOP_DEVICE_* */
  int32_t pad_;
  int64_t buffer_bytes;       /* device memory the plan may use */
  int64_t code_bytes;
} dop_device;                 /* Device, src/cluster.rs:33-39 */
typedef struct { int32_t a, b; } dop_link;  /* undirected, Link :42-46 */
#define DOP_HOME_PARAM 0
#define DOP_HOME_TAPE 1
typedef struct {
  int32_t kind, device, layer, replica, slot, pad_;
  int64_t row_begin, row_end, col_begin, col_end, stride;
  int64_t bytes;
} dop_home;                   /* Home, :134-143 */
#define DOP_HOP_PARAM 0
#define DOP_HOP_ADJOINT 1
#define DOP_HOP_ACTIVATION 2
typedef struct {
  int32_t from, to, kind, pad_;
  int64_t bytes, offset, elems, row_begin, row_end, col_begin, col_end, stride;
  int32_t layer, micro, replica, pad2_;  /* what the message carries */
} dop_hop;                    /* Hop, :178-190 */
#define DOP_PASS_FWD 0
#define DOP_PASS_BWD 1
#define DOP_EXEC_SGD 13       /* Exec, :204-219 */
#define DOP_EXEC_BLOCK 14     /* one block lens (this library's window unit) */
typedef struct {
  int32_t device, pass, exec, layer, micro, replica, slot, home;
  int64_t batch_begin, batch_end;  /* sequences of the global batch */
  int64_t resident_bytes, tape_bytes, param_bytes, param_offset, din, dout;
  int32_t n_inbound, n_outbound;
} dop_window;                 /* Window, :222-250 */
typedef struct dop_stage_plan dop_stage_plan;
int dop_derive_links(const dop_device* devices, int64_t n_devices, dop_link* out,
                     int64_t cap, int64_t* count);            /* :307-336 */
/* Shortest path whose intermediate devices have `bytes` free
 * (route_message, :350-398); DOP_E_ROUTE_UNAVAILABLE when none. */
int dop_route_message(const dop_link* links, int64_t n_links,
                      const int64_t* free_bytes, int64_t n_devices, int32_t from,
                      int32_t to, int64_t bytes, int32_t* path, int64_t cap,
                      int64_t* len);
/* stage_mixtral / compile_mixtral (:401-490) for cfg->layers blocks of
 * global_batch sequences of length seq in micro_batches micro-batches;
 * links NULL derives them from the devices. */
int dop_stage_mixtral(const dop_mixtral_cfg* cfg, int64_t global_batch, int64_t seq,
                      int64_t micro_batches, int precision, const dop_device* devices,
                      int64_t n_devices, const dop_link* links, int64_t n_links,
                      dop_stage_plan** out);
int dop_plan_destroy(dop_stage_plan* plan);
int64_t dop_plan_home_count(const dop_stage_plan* plan);
int64_t dop_plan_window_count(const dop_stage_plan* plan);
int64_t dop_plan_hop_count(const dop_stage_plan* plan);
int dop_plan_home(const dop_stage_plan* plan, int64_t i, dop_home* out);
int dop_plan_window(const dop_stage_plan* plan, int64_t i, dop_window* out);
/* Index (into the plan's hops) of window i's j-th inbound or outbound hop. */
int dop_plan_window_hop(const dop_stage_plan* plan, int64_t i, int outbound, int64_t j,
                        int64_t* hop_index);
int dop_plan_hop(const dop_stage_plan* plan, int64_t i, dop_hop* out);
/* StagePlan::check (:1881-1928): one copy of param_elems parameters is
 * covered, no device stores or peaks above its buffer. */
int dop_plan_check(const dop_stage_plan* plan, const dop_device* devices,
                   int64_t n_devices, int64_t param_elems);
/* The run's expected control-plane trace (src/mixtral.rs:1393-1435):
 * MEMBERS n, JOIN r per device, then per window its inbound HOP lines,
 * COMPUTE device exec pass, its outbound HOP lines; DONE. */
int dop_plan_trace(const dop_stage_plan* plan, char* buf, int64_t cap, int64_t* len);
/* Run one block window (Compute::on_window, src/dist.rs:86-97): forward
 * reads `in` (x) and writes `out` (y); backward reads `in` (dy), writes
 * `out` (dx) and accumulates into dparams. */
int dop_run_window(dop_block* blk, const dop_window* w, const void* params,
                   const float* in, float* out, float* dparams, void* stream);

/* ------------------------------------------------ scalar lenses (host)
 * Exact rational reverse-mode AD with an explicit residual, src/ad.rs.
 * Host code only (no device work: environments of a few variables).  An
 * expression is a flat array of nodes, children referenced by index:
 *   VAR    var                  env[var]
 *   CONST  q                    the rational q
 *   NEG    a                    -a
 *   ADD    a, b                 a + b
 *   MUL    a, b                 a * b
 *   LET    a, b                 let x = a in b (x is variable 0 inside b,
 *                               the outer variables shift up by one)
 *   IFEQ   a, b, c, d           if a == b then c else d
 * Rationals are n/d, reduced, d > 0; i64 overflow is an error. */
typedef struct { int64_t n, d; } dop_q;
#define DOP_EXPR_VAR 0
#define DOP_EXPR_CONST 1
#define DOP_EXPR_NEG 2
#define DOP_EXPR_ADD 3
#define DOP_EXPR_MUL 4
#define DOP_EXPR_LET 5
#define DOP_EXPR_IFEQ 6
typedef struct {
  int32_t kind;
  int32_t pad_;
  int64_t a, b, c, d; /* child node indices */
  int64_t var;
  dop_q q;
} dop_expr_node;
typedef struct dop_ad_tape dop_ad_tape;
/* `ad::forward` (src/ad.rs:76-129): value and residual.  The residual
 * stores both factors of each product and the branch each conditional took,
 * nothing else. */
int dop_ad_forward(const dop_expr_node* nodes, int64_t n_nodes, int64_t root,
                   const dop_q* env, int64_t env_len, dop_q* value,
                   dop_ad_tape** tape);
/* `ad::backward` (src/ad.rs:131-176): cot_env[i] = d value / d env[i] times
 * cot, from the residual. */
int dop_ad_backward(const dop_expr_node* nodes, int64_t n_nodes, int64_t root,
                    const dop_ad_tape* tape, dop_q cot, int64_t env_len,
                    dop_q* cot_env);
/* `ad::stored_scalars` (src/ad.rs:179-196): the rationals the residual
 * holds, in tape order; out == NULL only counts. */
int dop_ad_stored_scalars(const dop_ad_tape* tape, dop_q* out, int64_t cap,
                          int64_t* count);
int dop_ad_tape_destroy(dop_ad_tape* tape);

/* GF(2) linear maps, src/vect.rs (host code).  A map stores the image of
 * each basis vector as a bitset: columns[j] for j < dom, bits < cod; dom,
 * cod <= 32.  `transpose` is the adjoint of a linear map. */
typedef struct {
  uint32_t dom, cod;
  uint32_t columns[32];
} dop_lin;
uint32_t dop_lin_apply(const dop_lin* f, uint32_t v);              /* :14-22 */
int dop_lin_zero(uint32_t dom, uint32_t cod, dop_lin* out);        /* :25-31 */
int dop_lin_identity(uint32_t n, dop_lin* out);                    /* :33-38 */
int dop_lin_compose(const dop_lin* g, const dop_lin* f, dop_lin* out); /* g after f, :40-47 */
int dop_lin_add(const dop_lin* f, const dop_lin* g, dop_lin* out); /* :49-63 */
int dop_lin_transpose(const dop_lin* f, dop_lin* out);             /* :65-79 */
int dop_lin_kronecker(const dop_lin* f, const dop_lin* g, dop_lin* out); /* :81-106 */
/* Every map dom -> cod (dom*cod <= 24) in the crate's enumeration order
 * (:108-126); out == NULL only counts. */
int dop_lin_all(uint32_t dom, uint32_t cod, dop_lin* out, int64_t cap,
                int64_t* count);

#ifdef __cplusplus
}
#endif
#endif /* DOP_H */
