/*
 * model.h - GPT-2 model of libcngpt_cuda (drop-in for the reference's
 * src/model.h; struct layouts are byte-identical so code compiled against
 * either header links against this library).
 *
 * Memory model: param_buf / grad_buf / m_buf / v_buf / decay_buf and the
 * activation arena act_buf are single device allocations with the
 * reference's offsets (src/model.c:54-83, 333-436); every pointer in GPT is a
 * device pointer, or a managed pointer when managed mode is on
 * (cngpt_cuda_set_managed(1) or CNGPT_CUDA_MANAGED=1 in the environment),
 * which makes them host-dereferenceable as the reference's tests expect.
 *
 * Arena notes: the acts.attn_scores[l] slot holds the per-row log-sum-exp
 * of the fused attention (B*H*T floats) instead of the T x T score matrix;
 * acts.attn_probs[l] is left unwritten (the fused kernel never forms P).
 */
#ifndef CNGPT_MODEL_H
#define CNGPT_MODEL_H

#include <stddef.h>
#include <stdint.h>

#define CNGPT_MAGIC    0x434E4750   /* "CNGP"   ref src/model.h:19 */
#define CNGPT_VERSION  1

/* weight file header, 7 x int32 (ref src/model.h:22-30) */
typedef struct {
    int magic;
    int version;
    int n_layer;
    int n_head;
    int n_embd;
    int vocab_size;
    int block_size;
} GPTHeader;

/* ref src/model.h:35-42 */
typedef struct {
    int n_layer;
    int n_head;
    int n_embd;
    int vocab_size;
    int block_size;
    float dropout;
} GPTConfig;

/* views into the flat parameter (or gradient) buffer, ref src/model.h:68-80 */
typedef struct {
    float *wte;
    float *wpe;
    float **ln1_w, **ln1_b;
    float **c_attn_w, **c_attn_b;
    float **c_proj_w, **c_proj_b;
    float **ln2_w, **ln2_b;
    float **mlp_fc_w, **mlp_fc_b;
    float **mlp_proj_w, **mlp_proj_b;
    float *ln_f_w, *ln_f_b;
} GPTWeights;

/* views into the activation arena, ref src/model.h:86-115 */
typedef struct {
    float *emb;
    float **ln1_out;
    float **ln1_mean;
    float **ln1_rstd;
    float **qkv;
    float **attn_scores;
    float **attn_probs;
    float **attn_out;
    float **attn_proj;
    float **res1;
    float **ln2_out;
    float **ln2_mean;
    float **ln2_rstd;
    float **mlp_fc_out;
    float **mlp_gelu;
    float **mlp_proj_out;
    float **res2;
    float *ln_f_out;
    float *ln_f_mean;
    float *ln_f_rstd;
    float *logits;
    float *probs;
    unsigned char *emb_mask;
    unsigned char **res1_mask;
    unsigned char **res2_mask;
} GPTActivations;

/* ref src/model.h:120-137 */
typedef struct {
    GPTConfig     cfg;
    GPTWeights    params;
    GPTWeights    grads;
    GPTActivations acts;

    float *param_buf;
    float *grad_buf;
    float *act_buf;
    unsigned char *mask_buf;

    float *m_buf;
    float *v_buf;
    uint8_t *decay_buf;
    int    n_params;
    int    step;
} GPT;

#ifdef __cplusplus
extern "C" {
#endif

/* allocate device arenas, zero params, fill the decay mask  ref src/model.h:144 */
int  gpt_init(GPT *m, GPTConfig cfg);
/* N(0,0.02) init from the host rand() stream, uploaded      ref src/model.h:150 */
void gpt_init_weights(GPT *m);
/* weight file I/O through a host staging buffer             ref src/model.h:153,156 */
int  gpt_load(GPT *m, const char *path);
int  gpt_save(GPT *m, const char *path);
/* release device memory; zeroes *m                          ref src/model.h:159 */
void gpt_free(GPT *m);
/* (re)lay out the activation arena for B x T                ref src/model.h:163 */
int  gpt_resize_acts(GPT *m, int B, int T);
/* tokens/targets: host or device int[B*T]; returns the loss ref src/model.h:168 */
float gpt_forward(GPT *m, const int *tokens, const int *targets, int B, int T);
/* accumulates into the gradient arena                        ref src/model.h:174 */
void gpt_backward(GPT *m, const int *tokens, const int *targets, int B, int T);
/* ref src/model.h:177 */
void gpt_zero_grad(GPT *m);
/* clip by global norm (on device), AdamW                     ref src/model.h:182 */
void gpt_adamw(GPT *m, float lr, float beta1, float beta2,
               float eps, float wd, float grad_clip);
/* temperature / top-k sampling with the host rand() stream   ref src/model.h:189 */
void gpt_sample(GPT *m, const int *prompt_tokens, int prompt_len,
                int *out_tokens, int max_new_tokens,
                float temp, int top_k);
/* ref src/model.h:194 */
int gpt_num_params(const GPTConfig *cfg);

#ifdef __cplusplus
}
#endif
#endif /* CNGPT_MODEL_H */
