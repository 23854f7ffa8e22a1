/*
 * TEST INFRASTRUCTURE ONLY.  CPU restatement of llambda's quantized FFN path,
 * used as the parity checker for the CUDA kernels and as the timed CPU
 * baseline.  Nothing in the shipped library links or calls this code.
 *
 * Citations are file:line in jrm-code-project/llambda ("L" = llambda.lisp).
 */
#ifndef LLAMBDA_ORACLE_H
#define LLAMBDA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type tags, L24-31. */
enum {
  OR_TYPE_F32 = 0,
  OR_TYPE_F16 = 1,
  OR_TYPE_Q5_0 = 6,
  OR_TYPE_Q8_0 = 8,
  OR_TYPE_Q4_K = 12,
  OR_TYPE_Q5_K = 13,
  OR_TYPE_Q6_K = 14
};

/* A tensor as llambda sees it: dimensions (ne0 = columns, ne1 = rows,
 * ne2 = experts) over row-contiguous raw GGUF data (L3389-3400, L3909-3916). */
typedef struct {
  int type;
  const void *data;
  size_t ne0, ne1, ne2;
} or_tensor;

/* One MoE feed-forward layer.  Unused tensors have data == NULL. */
typedef struct {
  int arch;                 /* 0 = qwen3next, 1 = nemotron_h_moe */
  size_t hidden;            /* length of the input and output vectors */
  int top_k;                /* expert_used_count */
  float weight_scale;       /* nemotron expert_weights_scale (default 1.0) */
  int weights_norm;         /* nemotron expert_weights_norm */
  or_tensor router;         /* ffn_gate_inp, F32 [hidden x experts] */
  const float *router_bias; /* nemotron exp_probs_b.bias, or NULL */
  const float *shared_gate_inp; /* qwen3next ffn_gate_inp_shexp [hidden] */
  or_tensor gate_exps, up_exps, down_exps;    /* gate unused for nemotron */
  or_tensor gate_shexp, up_shexp, down_shexp; /* gate unused for nemotron */
  const float *input_norm;  /* post_attention_norm weight, or NULL */
  float norm_epsilon;
  int add_residual;         /* out = x + moe(rms_norm(x)) */
  /* nemotron ffn_latent_down [hidden -> latent] and ffn_latent_up
   * [latent -> hidden], both or neither (data NULL: none) */
  or_tensor latent_down, latent_up;
} or_moe_layer;

const char *or_last_error(void);
void or_set_workers(int workers);
int or_get_workers(void);

float or_fp16_to_f32(uint16_t bits, int *error);
void or_get_scale_min_k4(const uint8_t *scales, int index, int *scale, int *min);
int or_dequantize_q4_k(const uint8_t *blocks, size_t count, float *out);
int or_dequantize_q6_k(const uint8_t *blocks, size_t count, float *out);
int or_dot_q4_k(const uint8_t *row, const float *x, size_t count, float *out);
int or_dot_q6_k(const uint8_t *row, const float *x, size_t count, float *out);
int or_dequantize_q5_k(const uint8_t *blocks, size_t count, float *out);
int or_dot_q5_k(const uint8_t *row, const float *x, size_t count, float *out);
int or_dequantize_q5_0(const uint8_t *blocks, size_t count, float *out);
int or_dequantize_q8_0(const uint8_t *blocks, size_t count, float *out);
int or_dot_q5_0(const uint8_t *row, const float *x, size_t count, float *out);
int or_dot_q8_0(const uint8_t *row, const float *x, size_t count, float *out);
float or_dot_f32(const float *row, const float *x, size_t count);
float or_dot_product(const float *a, const float *b, size_t count);
size_t or_row_bytes(int type, size_t columns);
int or_gemv(const or_tensor *t, size_t start_row, size_t row_count,
            const float *x, float *y);
void or_select_top_k(const float *logits, size_t count, int k,
                     int32_t *top_indices, float *top_logits);
float or_sigmoid(float v);
float or_silu(float v);
float or_relu_squared(float v);
void or_rms_norm(const float *x, const float *w, size_t n, float eps, float *out);
int or_moe_forward(const or_moe_layer *layer, const float *x, size_t tokens,
                   float *out, int32_t *selected, float *weights);

/* Test-data helpers over the shared generator (synth.h). */
void or_synth_q4k(uint64_t seed, uint64_t stream, uint64_t first_block,
                  size_t blocks, float dscale, uint8_t *out);
void or_synth_q6k(uint64_t seed, uint64_t stream, uint64_t first_block,
                  size_t blocks, float dscale, uint8_t *out);
void or_synth_f32(uint64_t seed, uint64_t stream, uint64_t first, size_t count,
                  float sigma, float *out);
uint16_t or_f32_to_f16(float f);

#ifdef __cplusplus
}
#endif

#endif
