/* ref_shim.cu -- extern "C" entry points over the reference's OWN CPU code.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline).  This file holds
 * no arithmetic of its own beyond loops that restate the reference's call
 * structure; the dequantisation, GEMV, softmax, top-k and SwiGLU it runs are
 * the reference's functions, compiled from arahe-dev/breadv2's sources
 * (layer_ops.cu, dequant_q4k_cpu.c, gguf.c, bread.c, sriracha_stubs.c) by
 * oracle/Makefile into oracle/_ref/libbread_ref.so.
 *
 * The reference compiles layer_ops.cu with nvcc, so its symbols carry C++
 * linkage; the wrappers below give them stable C names for ctypes.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#include "layer_ops.h" /* reference: layer_ops.h:16-46 */

extern "C" {
/* dequant_q4k_cpu.c:90,141 (compiled by gcc, C linkage) */
void dequant_q4k_block_cpu(const uint8_t *block, float *out);
void dequant_q6k_block_cpu(const uint8_t *block, float *out);
/* dequant_q4k_cpu.c:177 main(), renamed at compile time */
int ref_dq_kat_main(void);

int ref_kat(void) { return ref_dq_kat_main(); }

/* layer_ops.cu:44 / :77 -- exact fp16 decode */
void ref_dequant_q4k_block(const uint8_t *b, float *o) { cpu_dequant_q4k_block(b, o); }
void ref_dequant_q6k_block(const uint8_t *b, float *o) { cpu_dequant_q6k_block(b, o); }
/* dequant_q4k_cpu.c:90 / :141 -- flush-to-zero fp16 decode */
void ref_dequant_q4k_block_ftz(const uint8_t *b, float *o) { dequant_q4k_block_cpu(b, o); }
void ref_dequant_q6k_block_ftz(const uint8_t *b, float *o) { dequant_q6k_block_cpu(b, o); }

/* layer_ops.cu:169 cpu_tensor_matvec (qtype: GGML id, 12 = Q4_K, 14 = Q6_K) */
void ref_tensor_matvec(const uint8_t *w, uint32_t qtype, const float *x, float *y, int rows, int cols)
{
    cpu_tensor_matvec(w, qtype, x, y, rows, cols);
}

/* layer_ops.cu:214 / :222 / :231 / :252 */
void ref_swiglu(const float *g, const float *u, float *o, int n) { cpu_swiglu(g, u, o, n); }
void ref_softmax(float *x, int n) { cpu_softmax(x, n); }
void ref_topk(const float *p, int n, int K, int *idx, float *w) { cpu_topk(p, n, K, idx, w); }
float ref_sigmoid(float x) { return cpu_sigmoid(x); }

/* route_layer, one_layer.cu:937-992, for T tokens: fp32 router GEMV in the
 * reference's loop order (one_layer.cu:969-971), optional fp16 shared-gate
 * dot (one_layer.cu:973-980), then the reference's softmax and top-k, and
 * sigmoid of the shared-gate score (one_layer.cu:1889). */
void ref_route(const float *x, const float *W_r, const uint16_t *w_sg, int T, int H, int E, int top_k, int *idx,
               float *wt, float *sg_weight)
{
    float *lg = (float *)malloc((size_t)E * sizeof(float));
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * H;
        memset(lg, 0, (size_t)E * sizeof(float));
        for (int i = 0; i < E; i++)
            for (int j = 0; j < H; j++) lg[i] += W_r[(size_t)i * H + j] * xt[j];
        float score = 0.0f;
        if (w_sg) {
            const half *hs = (const half *)w_sg;
            for (int j = 0; j < H; j++) score += __half2float(hs[j]) * xt[j];
        }
        sg_weight[t] = cpu_sigmoid(score);
        cpu_softmax(lg, E);
        cpu_topk(lg, E, top_k, idx + (size_t)t * top_k, wt + (size_t)t * top_k);
    }
    free(lg);
}

/* The reference's CPU expert block, expert_bench.cu:158-179: an OpenMP
 * parallel-for over the routed experts (schedule(static,1), n_threads), each
 * running cpu_tensor_matvec gate/up -> cpu_swiglu -> down -> * weight into its
 * own buffer, then a serial sum in k order.  The shared expert (one_layer.cu:
 * 1840-1891) is one more slot with weight sg_weight[t] when sh_* are given.
 * Runs T tokens one after the other.  out: fp32 [T x H], overwritten. */
int ref_moe_block(const uint8_t *const *gate_ptrs, const uint8_t *const *up_ptrs, const uint8_t *const *down_ptrs,
                  const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *sh_down, const float *x,
                  const int *idx, const float *wt, const float *sg_weight, int T, int H, int I, int top_k,
                  int n_threads, float *out)
{
    const int K = top_k + ((sh_gate && sh_up && sh_down) ? 1 : 0);
    float *tmp = (float *)malloc((size_t)K * H * sizeof(float));
    float *tg = (float *)malloc((size_t)K * I * sizeof(float));
    float *tu = (float *)malloc((size_t)K * I * sizeof(float));
    if (!tmp || !tg || !tu) return -2;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * H;
#pragma omp parallel for schedule(static, 1) num_threads(n_threads)
        for (int k = 0; k < K; k++) {
            float *o = tmp + (size_t)k * H, *g = tg + (size_t)k * I, *u = tu + (size_t)k * I;
            const uint8_t *wg, *wu, *wd;
            float w;
            if (k < top_k) {
                const int e = idx[(size_t)t * top_k + k];
                wg = gate_ptrs[e]; wu = up_ptrs[e]; wd = down_ptrs[e];
                w = wt[(size_t)t * top_k + k];
            } else {
                wg = sh_gate; wu = sh_up; wd = sh_down;
                w = sg_weight[t];
            }
            memset(o, 0, (size_t)H * sizeof(float));
            cpu_tensor_matvec(wg, 12u, xt, g, I, H);
            cpu_tensor_matvec(wu, 12u, xt, u, I, H);
            cpu_swiglu(g, u, g, I);
            cpu_tensor_matvec(wd, 14u, g, o, H, I);
            for (int i = 0; i < H; i++) o[i] *= w;
        }
        float *ot = out + (size_t)t * H;
        memset(ot, 0, (size_t)H * sizeof(float));
        for (int k = 0; k < K; k++)
            for (int i = 0; i < H; i++) ot[i] += tmp[(size_t)k * H + i];
    }
    free(tmp);
    free(tg);
    free(tu);
    return 0;
}

int ref_max_threads(void) { return omp_get_max_threads(); }
}
