/* bread_b200.h -- C ABI of the B200 (sm_100a) quantised-expert MoE library.
 *
 * A drop-in for the GPU hot path of the BREAD decode engine
 * (arahe-dev/breadv2): the Q4_K / Q6_K dequantise-and-multiply GEMVs and the
 * MoE FFN block around them (router top-k, SiLU-gate, weighted expert
 * combine).  Every entry point below names the reference interface it
 * replaces.
 *
 * Conventions (same as the reference unless stated):
 *   - all data pointers are DEVICE pointers owned by the caller, except
 *     functions whose name ends in _host;
 *   - calls only enqueue work on `stream` and never synchronise it;
 *   - weights are raw GGUF super-blocks, row-major, `cols/256` blocks per row
 *     (Q4_K: 144 B, Q6_K: 210 B) or `cols/32` blocks (Q8_0: 34 B);
 *   - qtype uses the GGML ids: 8 = Q8_0, 12 = Q4_K, 14 = Q6_K
 *     (reference gguf.h:31-37, kernels.cu:40-41,249);
 *   - `int` results are status codes (BREAD_OK = 0).  The reference aborts
 *     with exit(1) instead (kernels.cu:303-307, bread_utils.h:14-21); the
 *     void drop-in bread_matvec keeps that behaviour.
 *   - no entry point allocates device memory unless its comment says so;
 *     scratch comes from a caller-provided workspace.
 */
#ifndef BREAD_B200_H
#define BREAD_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#define BREAD_QTYPE_Q8_0 8
#define BREAD_QTYPE_Q4_K 12
#define BREAD_QTYPE_Q6_K 14

#define BREAD_OK 0
#define BREAD_ERR_ARG 1        /* bad size, NULL pointer, cols not a block multiple ... */
#define BREAD_ERR_QTYPE 2      /* qtype not 8, 12 or 14 */
#define BREAD_ERR_ALIGN 3      /* pointer alignment the entry point requires is not met */
#define BREAD_ERR_CUDA 4       /* a CUDA runtime call failed (see bread_last_error) */
#define BREAD_ERR_WORKSPACE 5  /* workspace missing or smaller than *_workspace_bytes */
#define BREAD_ERR_TIMEOUT 6    /* a bounded device-side wait ran out (peer never arrived) */
#define BREAD_ERR_STATE 7      /* object used in the wrong state (e.g. peers not set) */

/* ---------------------------------------------------------------------- */
/* Drop-in entry points with the reference's C++ signatures.               */
/* The reference's callers are nvcc-compiled C++ and declare these without */
/* extern "C", so they are exported with C++ linkage (same mangled names). */
/* ---------------------------------------------------------------------- */
#ifdef __cplusplus
/* Replaces bread_matvec, kernels.cu:289-308.  y[rows] = W[rows x cols] * x[cols],
 * fp16 in/out, fp32 arithmetic.  Aborts (exit 1) on an unknown qtype or a
 * launch error, like the reference. */
void bread_matvec(void *w, half *x, half *y, int rows, int cols, int qtype, cudaStream_t stream);

/* The launchers layer_logic.cu:28-31 declares (and the reference never
 * defines), with the semantics of one_layer.cu's kernels:
 *   rmsnorm_inplace one_layer.cu:158-180, silu_mul_inplace :190-197,
 *   scale_accum :203-208, copy_half :214-218.  Abort on a launch error. */
void bread_rmsnorm_half(half *x, const float *w, int n, float eps, cudaStream_t s);
void bread_silu_mul(half *gate, const half *up, int n, cudaStream_t s);
void bread_scale_accum(half *dst, const half *src, float scale, int n, cudaStream_t s);
void bread_copy_half(half *dst, const half *src, int n, cudaStream_t s);
extern "C" {
#endif

/* ---------------------------------------------------------------------- */
/* Errors                                                                  */
/* ---------------------------------------------------------------------- */
const char *bread_status_string(int status);
/* Text of the last error raised on the calling host thread ("" if none). */
const char *bread_last_error(void);
/* Device-side error word of the current device (bit 0: a bounded wait timed
 * out).  Synchronous; clears the word when `clear` != 0. */
int bread_device_error(unsigned *word_out, int clear);

/* ---------------------------------------------------------------------- */
/* GEMV (kernels.cu:150-308)                                               */
/* ---------------------------------------------------------------------- */
/* Status-returning C form of bread_matvec (kernels.cu:289): fp16 x/y. */
int bread_matvec_f16(const void *w, const void *x, void *y, int rows, int cols, int qtype, cudaStream_t stream);
/* fp32 I/O form: y = W x.  fp32 output keeps the 1e-3 relative-L2 bar that an
 * fp16 y (kernels.cu:191) would use up on its own. */
int bread_matvec_f32(const void *w, const float *x, float *y, int rows, int cols, int qtype, cudaStream_t stream);
/* T right-hand sides: Y[T x rows] = X[T x cols] * W^T, each weight read once
 * (the batched speculative-verify case; the reference runs T sequential
 * bread_matvec calls, main_speculative.cu:478-497). 1 <= T <= 64. */
int bread_matvec_batch_f32(const void *w, const float *x, float *y, int rows, int cols, int qtype, int T,
                           cudaStream_t stream);

/* Output head + greedy sampling on the device: compute_logits (main.cu:297-319,
 * bread_matvec of the [rows x cols] lm head) followed by greedy_sample
 * (main.cu:324-337), which copies all `rows` fp16 logits to the host and
 * scans them.  Here each warp of the GEMV folds its rows into a running
 * argmax and the last warp to finish writes *token (largest logit; among
 * equal values the lowest row, like the reference's strict `>` scan; NaN
 * never wins; 0 when every logit is NaN) and *value (that logit, or NULL to
 * skip).  round_half = 1 compares the fp16-rounded logits greedy_sample sees;
 * 0 compares fp32.  logits: optional fp32 [rows] copy (NULL to skip).
 * x: fp32 [cols].  state: 16 bytes of device memory, 8-byte aligned, zeroed by
 * the caller once before the first call; every call leaves it zeroed again
 * (calls sharing one state must not overlap on the GPU).  Enqueue-only. */
int bread_lm_head_argmax(const void *w, const float *x, int rows, int cols, int qtype, int round_half, float *logits,
                         int *token, float *value, void *state, cudaStream_t stream);

/* Bit-exact dequantisation of n_blocks consecutive blocks to fp32
 * (Q4_K/Q6_K: 256 values per block, Q8_0: 32).  Arithmetic of
 * layer_ops.cu:44-105 (exact fp16 scale decode, each product rounded). */
int bread_dequant(const void *w, float *out, long long n_blocks, int qtype, cudaStream_t stream);

/* Status-returning C forms of the layer_logic.cu:28-31 launchers. */
int bread_rmsnorm_half_c(void *x, const float *w, int n, float eps, cudaStream_t s);
int bread_silu_mul_c(void *gate, const void *up, int n, cudaStream_t s);
int bread_scale_accum_c(void *dst, const void *src, float scale, int n, cudaStream_t s);
int bread_copy_half_c(void *dst, const void *src, int n, cudaStream_t s);

/* ---------------------------------------------------------------------- */
/* MoE FFN block (one_layer.cu:937-992 routing, :1820-1985 experts)        */
/* ---------------------------------------------------------------------- */
/* Device-side replacement of route_layer (one_layer.cu:937-992), which is
 * host-blocking in the reference.  For each of T tokens: logits = W_r x
 * (W_r fp32 [E x H] row-major), softmax over E, top_k by repeated argmax
 * (lowest index wins ties, layer_ops.cu:231-250), weights renormalised to sum
 * to one; sg_weight[t] = sigmoid(w_sg . x_t) with w_sg fp16 [H], or 0.5 when
 * w_sg is NULL (one_layer.cu:944,1889).  Outputs idx [T x top_k] int32,
 * w [T x top_k] fp32, sg_weight [T] fp32 (NULL to skip).
 * Limits: 1 <= T <= 64, top_k <= E <= 512, top_k <= 16, H % 256 == 0,
 * H <= 4096. */
int bread_moe_route(const float *x, const float *W_r, const void *w_sg, int T, int H, int E, int top_k, int *idx,
                    float *w, float *sg_weight, void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* Bytes of workspace bread_moe_route / bread_moe_ffn need for these shapes
 * (pass I = 0 for the router alone).  The workspace holds the router logits,
 * the int16 activations, the per-expert token lists and the SiLU*mul
 * intermediate; its contents need not be initialised. */
size_t bread_moe_workspace_bytes(int T, int H, int I, int E, int top_k);

/* The whole MoE FFN of one layer for T tokens (the expert loop of
 * one_layer.cu:1931-1983 plus the shared expert of :1840-1894, with the
 * router of :937-992 run on the device):
 *   out[t] += sum_k w[t,k] * down_e(silu(gate_e x_t) * (up_e x_t))  (e = idx[t,k])
 *           + sg_weight[t] * down_s(silu(gate_s x_t) * (up_s x_t))
 * gate_ptrs/up_ptrs/down_ptrs: DEVICE arrays of E device pointers, expert e's
 * Q4_K gate [I x H], Q4_K up [I x H], Q6_K down [H x I] (the per-expert
 * tables of weight_cache_t, loader.h:79-84).  Every pointer must be 16-byte
 * aligned.  sh_gate/sh_up/sh_down: the shared expert (all NULL for none).
 * x: fp32 [T x H]; out: fp32 [T x H], accumulated into (like scale_accum).
 * idx_out/w_out/sg_out: optional copies of the routing (NULL to skip).
 * Two grouped launches do all experts of all T tokens: each distinct expert's
 * weights are read once per call.  Limits as bread_moe_route; I % 256 == 0,
 * I <= 2048.  workspace: >= bread_moe_workspace_bytes(...) bytes, 256-byte
 * aligned. */
int bread_moe_ffn(const void *const *gate_ptrs, const void *const *up_ptrs, const void *const *down_ptrs,
                  const float *W_r, const void *w_sg, const void *sh_gate, const void *sh_up, const void *sh_down,
                  const float *x, float *out, int T, int H, int I, int E, int top_k, int *idx_out, float *w_out,
                  float *sg_out, void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* bread_moe_ffn for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Some engines give all free HBM to their
 * resident weights and caches up front, so cudaMalloc has nothing left, and
 * some host loops must not call cudaMalloc on the decode path because it can
 * synchronise the device.  Same arguments and results as bread_moe_ffn minus
 * the workspace: the scratch is a fixed 256 KiB device array inside the
 * library (present on every GPU that loads it, until exit), enough for e.g.
 * T <= 16 at H = 2048, I = 512, E = 256, top_k = 8; larger shapes return
 * BREAD_ERR_WORKSPACE.  Allocates nothing.  The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress, no allocation),
 * so make that first call before any stream capture; later calls outside
 * capture look it up again, so an address from before a cudaDeviceReset is
 * never used.  All calls on a device share the array: calls that overlap on
 * the GPU race and must be ordered by the caller. */
int bread_moe_ffn_noalloc(const void *const *gate_ptrs, const void *const *up_ptrs, const void *const *down_ptrs,
                          const float *W_r, const void *w_sg, const void *sh_gate, const void *sh_up,
                          const void *sh_down, const float *x, float *out, int T, int H, int I, int E, int top_k,
                          int *idx_out, float *w_out, float *sg_out, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* GGUF tensor index (gguf.c:306-411; host only)                           */
/* ---------------------------------------------------------------------- */
typedef struct bread_gguf bread_gguf_t;
/* One tensor info record (gguf.h:80-88). */
typedef struct bread_gguf_tensor {
    const char *name;  /* owned by the open file */
    uint32_t type;     /* ggml type id: 0 F32, 1 F16, 8 Q8_0, 12 Q4_K, 14 Q6_K ... */
    uint32_t n_dims;
    uint64_t dims[4];  /* dims[0] innermost (row length) */
    uint64_t offset;   /* bytes from the start of the data section */
    uint64_t size;     /* bytes of tensor data (0 for an unknown type) */
    uint64_t n_elems;
} bread_gguf_tensor_t;
/* Opens a GGUF v2/v3 file and parses its header, metadata (keeping only
 * general.alignment) and tensor index; no tensor data is read.  Replaces
 * gguf_open (gguf.c:306-374), which exits on a malformed file: here any
 * truncation or corruption returns BREAD_ERR_ARG. */
int bread_gguf_open(const char *path, bread_gguf_t **out);
int bread_gguf_close(bread_gguf_t *g);
/* Header facts: version, tensor count, alignment, absolute data offset. */
int bread_gguf_info(const bread_gguf_t *g, uint32_t *version, uint64_t *n_tensors, uint32_t *alignment,
                    uint64_t *data_offset);
/* Tensor info by index (gguf_tensor_by_idx, gguf.c:400-403) or by exact name
 * (gguf_find_tensor, gguf.c:405-411; BREAD_ERR_ARG when absent). */
int bread_gguf_tensor(const bread_gguf_t *g, uint64_t index, bread_gguf_tensor_t *out);
int bread_gguf_find(const bread_gguf_t *g, const char *name, bread_gguf_tensor_t *out);
/* Reads `bytes` from `offset` (relative to the data section) into host memory. */
int bread_gguf_read(const bread_gguf_t *g, uint64_t offset, void *dst, uint64_t bytes);

/* ---------------------------------------------------------------------- */
/* Expert stack executor (the decode loop's MoE part, main.cu:683-687)     */
/* ---------------------------------------------------------------------- */
typedef struct bread_stack bread_stack_t;

typedef struct bread_stack_config {
    int n_layers;   /* 40 in the reference model (bread.h:17) */
    int hidden;     /* H = 2048 (bread.h:16) */
    int inter;      /* I = 512 (bread.h:59) */
    int n_experts;  /* E = 256 (bread.h:61) */
    int top_k;      /* 8 (bread.h:62) */
    int max_tokens; /* largest T a step may use (<= 64) */
    int shared_expert; /* 1: one always-on shared expert per layer */
    float norm_eps; /* RMSNorm epsilon between layers (< 0: layers take their input un-normalised) */
    uint64_t seed;  /* synthetic weights: seeded generator (bread_synth_*) */
    int rank;       /* expert-parallel rank (0 for one GPU) */
    int world;      /* expert-parallel world size (1, 2, 4 or 8) */
    int norm_weight; /* 1: each layer's RMSNorm multiplies by a weight vector
                        (post_attention_norm.weight, one_layer.cu:1803-1818;
                        synthetic: 1 + 0.1 N(0,1)); 0: unit weight */
} bread_stack_config_t;

/* The same stack with the weights of a GGUF model file (loader.c:156-206 and
 * :628-693, which keep experts in a host LRU and stream them on demand; here
 * every expert this rank holds is resident): per layer l < n_layers it reads
 * blk.l.ffn_{gate,up,down}_exps.weight (Q4_K, Q4_K, Q6_K, experts outermost:
 * this rank's experts are one contiguous byte range of each),
 * blk.l.ffn_{gate,up,down}_shexp.weight (shared expert, if present),
 * blk.l.ffn_gate_inp.weight (router, F32 [E x H]), blk.l.ffn_gate_inp_shexp.weight
 * (shared gate, F16 [H], optional) and blk.l.post_attention_norm.weight (F32
 * [H], optional).  hidden / inter / n_experts / shared_expert / norm_weight are
 * taken from the file (cfg values must be 0 or match); seed is unused.  One
 * device allocation per tensor kind per layer. */
int bread_stack_create_gguf(bread_stack_t **out, const char *path, const bread_stack_config_t *cfg);
/* Allocates and fills every weight this rank holds (experts [rank*E/world,
 * (rank+1)*E/world) of each layer, the router and shared-gate vector of every
 * layer, and the shared expert of the layers it owns), plus its scratch.
 * The only entry point that allocates device memory. */
int bread_stack_create(bread_stack_t **out, const bread_stack_config_t *cfg);
int bread_stack_destroy(bread_stack_t *st);
/* Device bytes this rank holds (weights + scratch). */
size_t bread_stack_device_bytes(const bread_stack_t *st);
/* The configuration the stack was built with (for a GGUF stack: with the
 * shapes and options read from the file). */
int bread_stack_get_config(const bread_stack_t *st, bread_stack_config_t *out);
/* Weights of one layer as device pointers (for parity checks). */
int bread_stack_layer(const bread_stack_t *st, int layer, const void **gate_base, const void **up_base,
                      const void **down_base, const float **W_r, const void **w_sg, const void **sh_gate,
                      const void **sh_up, const void **sh_down, int *expert_lo, int *expert_hi);
/* Copies the pre-MoE RMSNorm weight of one layer to host_out (fp32
 * [hidden]); *has_weight = 0 (and nothing copied) when the stack normalises
 * with unit weight.  Synchronous. */
int bread_stack_norm_weight(const bread_stack_t *st, int layer, float *host_out, int *has_weight);
/* Expert-parallel set-up (world > 1).  mailbox_bytes: size of the receive
 * mailbox this rank allocates (query with ptr = NULL).  bread_stack_mailbox
 * returns its device pointer; the caller exchanges CUDA IPC handles of every
 * rank's mailbox and passes the opened peer pointers (index = rank, own entry
 * = own mailbox) to bread_stack_set_peers. */
int bread_stack_mailbox(bread_stack_t *st, void **ptr, size_t *bytes);
int bread_stack_set_peers(bread_stack_t *st, void *const *peer_mailboxes, int world);
/* Bound of every device-side wait on another rank's data (default 20 s,
 * because peers may start their launch late).  A wait that runs out sets the
 * device error word (bread_device_error: bit 0) and every later wait on the
 * device gives up at once, so the launch finishes with undefined h instead of
 * hanging.  No reference counterpart (the reference runs on one GPU). */
int bread_stack_set_peer_timeout(bread_stack_t *st, double seconds);
/* CUDA IPC of a mailbox between the ranks' processes: 64-byte handle of a
 * device allocation; open a peer's handle (peer access enabled lazily); close
 * an opened mapping after bread_stack_destroy. */
int bread_ipc_get_handle(const void *dev_ptr, void *handle_out);
int bread_ipc_open_handle(const void *handle, void **dev_ptr);
int bread_ipc_close_handle(void *dev_ptr);
/* One decode step of T tokens through all layers.  h: device fp32 [T x H],
 * updated in place (h <- h + moe_l(norm(h)) for each layer l).  The first
 * call for a given T captures a CUDA graph; later calls replay it. */
int bread_stack_step(bread_stack_t *st, float *h, int T, cudaStream_t stream);
/* Same, from and to HOST memory (pinned for best speed): copies h_in to the
 * device, runs the step and copies the result back, all on `stream`. */
int bread_stack_step_host(bread_stack_t *st, const float *h_in, float *h_out, int T, cudaStream_t stream);
/* Kernel launches of one step for T tokens (all layers): 1, the whole step
 * is one cooperative launch of the persistent step kernel. */
int bread_stack_launches_per_step(const bread_stack_t *st, int T);
/* One step like bread_stack_step with phase timestamps recorded by every
 * CTA; synchronises `stream` and writes CTA 0's durations in ms of the router
 * phase, the gate/up phase, the down phase and the wait for the next layer's
 * expert-parallel combine (0 with world = 1) of every layer to
 * kernel_ms[4*layer + k], k = 0..3. */
int bread_stack_profile_step(bread_stack_t *st, float *h, int T, cudaStream_t stream, float *kernel_ms);
/* Raw timestamps (ns, %globaltimer) of the last profiled step:
 * out[(layer * ctas + cta) * 24 + k].  Consumer points k = 0 layer start,
 * 1 logits written, 2 after the router barrier, 3 routing tables built,
 * 4 first activation slot landed, 5 gate/up done, 6 after the gate/up
 * barrier, 7 first down stage landed, 8 down done, 9 layer end; producer
 * points 10 routing tables seen, 11 gate/up copies issued, 12 down weight
 * copies issued, 13 next router rows issued, 14 gate/up barrier seen, 15 all
 * down copies issued; consumer again 16 quantisation share done, 17 router
 * rows landed, 18 router dots done, 19 routing inputs read, 20 top-k done,
 * 21 tables built, 22 down stages done, 23 down columns stored.  *ctas
 * receives the grid size.  Synchronous. */
int bread_stack_profile_stamps(const bread_stack_t *st, unsigned long long *out, size_t n_words, int *ctas);
/* Routing of every layer of the last step (the device-side route_layer,
 * one_layer.cu:937-992, as the step kernel ran it): idx/w [n_layers x T x
 * top_k], sg_weight [n_layers x T] host arrays sized for that step's T
 * (returned in *T_out).  Synchronous. */
int bread_stack_routing(const bread_stack_t *st, int *idx, float *w, float *sg_weight, int *T_out);
/* Per layer of the last step: expert groups computed here (distinct routed
 * experts + the shared expert) and (token, expert) pairs.  Synchronous. */
int bread_stack_routing_stats(const bread_stack_t *st, int *groups, int *pairs);

/* ---------------------------------------------------------------------- */
/* Seeded synthetic inputs (benchmark data; identical bytes on host and     */
/* device).  Distributions of the reference path's benchmark configs:       */
/* Q4_K d, dmin = fp16(|N(0,1)| * 1e-3), scale/quant bytes uniform; Q6_K     */
/* ql/qh uniform, scales uniform in [-32,31], d = fp16(+-|N(0,1)| * 1e-3).  */
/* N(0,1) is an Irwin-Hall(4) draw from a counter-based hash.               */
/* ---------------------------------------------------------------------- */
int bread_synth_blocks(void *dst, long long n_blocks, int qtype, uint64_t seed, uint64_t stream_id,
                       cudaStream_t stream);
int bread_synth_normal_f32(float *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id,
                           cudaStream_t stream);
int bread_synth_normal_f16(void *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id,
                           cudaStream_t stream);
int bread_synth_blocks_host(void *dst, long long n_blocks, int qtype, uint64_t seed, uint64_t stream_id);
int bread_synth_normal_f32_host(float *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id);
int bread_synth_normal_f16_host(void *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id);

#ifdef __cplusplus
}
#endif
#endif /* BREAD_B200_H */
