/*
 * Test infrastructure: NOT part of the product.
 *
 * Plain-C restatement of the NeuralSuite GPT training step (the oracle).  It
 * is the checker for the CUDA path: only tests/, __graft_entry__.smoke() and
 * the cpu_baseline leg of bench.py may load it.  Each function follows the
 * reference function named in its comment operation for operation (same loop
 * order, same float/double promotions, no FMA contraction), so on the same
 * inputs it reproduces the reference's bits; tests/test_oracle.py pins that
 * against oracle/_ref (the reference compiled from its own sources) and against
 * the committed fixtures in tests/golden/.
 *
 * Layouts are the reference's: fp32, row-major; token ids travel as floats and
 * are truncated to int (include/layers/embedding.h:43, include/losses.h:43).
 */
#ifndef NS_ORACLE_H_
#define NS_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/tensor.cpp:198-271  C[M,N] = A[M,K] * B[K,N], k-ascending sums. */
void nso_matmul(const float* A, const float* B, float* C, int M, int K, int N);
/* src/tensor.cpp:275-288 */
void nso_transpose(const float* A, float* C, int M, int N);
/* src/tensor.cpp:290-322 */
void nso_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* out,
                       float* mean, float* rstd, int rows, int dim, float eps);
/* src/tensor.cpp:324-359 (dgamma / dbeta are overwritten) */
void nso_layernorm_bwd(const float* dout, const float* x, const float* gamma, const float* mean,
                       const float* rstd, float* dx, float* dgamma, float* dbeta, int rows,
                       int dim);
/* src/tensor.cpp:428-443 */
void nso_gelu_fwd(const float* x, float* y, int64_t n);
/* src/tensor.cpp:445-461 */
void nso_gelu_bwd(const float* dout, const float* x, float* dx, int64_t n);
/* src/tensor.cpp:394-426, input [batch, T, T] */
void nso_causal_softmax(const float* in, float* out, int batch, int T);
/* include/losses.h:34-86: returns the mean loss, writes dlogits. */
float nso_cross_entropy(const float* logits, const float* targets, int rows, int classes,
                        float* dlogits);
/* include/layers/embedding.h:34-80.  Returns -1 (and writes nothing) on an
 * out-of-range token, the std::out_of_range of embedding.h:45-49. */
int nso_embedding_fwd(const float* weight, int num, int dim, const float* idx, int n_tok,
                      float* out);
void nso_embedding_bwd(const float* idx, int n_tok, int cached, const float* dout, int dim,
                       int num, float* dweight);
/* include/layers/attention.h:350-467 (MultiHeadAttention::Forward/Backward).
 * grads in registration order: c_attn.weight, c_attn.bias, c_proj.weight,
 * c_proj.bias.  Any of dout..g_b_proj may be NULL to run the forward only. */
int nso_mha(int B, int T, int C, int H, const float* w_attn, const float* b_attn,
            const float* w_proj, const float* b_proj, const float* x, const float* dout,
            float* y, float* dx, float* g_w_attn, float* g_b_attn, float* g_w_proj,
            float* g_b_proj);

/* include/optimizers.h:206-234 over a flat buffer cut into n_seg tensors
 * [offsets[t], offsets[t+1]) with decay[t]; `step` is the step count after
 * the increment (the reference's step_count_). */
void nso_adamw_flat(float* params, const float* grads, float* m, float* v, const int64_t* offsets,
                    const float* decay, int n_seg, float lr, float b1, float b2, float eps,
                    int step);

/* ------------------------------------------------------------- GPT model
 * include/gpt.h:136-327.  Parameters live in one flat buffer in the
 * registration order of Module::Parameters() (include/module.h:44-52):
 *   wte, wpe, per block [ln_1 g b, c_attn W b, c_proj W b, ln_2 g b,
 *   mlp_fc W b, mlp_proj W b], ln_f g b.
 */
typedef struct nso_gpt nso_gpt;

nso_gpt* nso_gpt_create(int vocab, int block, int n_layer, int n_head, int n_embd);
void nso_gpt_destroy(nso_gpt* g);
int nso_gpt_num_tensors(const nso_gpt* g);
int64_t nso_gpt_tensor_numel(const nso_gpt* g, int i);
int nso_gpt_tensor_rank(const nso_gpt* g, int i);
int64_t nso_gpt_num_params(const nso_gpt* g);
float* nso_gpt_params(nso_gpt* g);
float* nso_gpt_grads(nso_gpt* g);
/* Forward -> CrossEntropy -> Backward (tools/parity/parity_gpt.cpp:86-97).
 * Returns 0, or -1 on an out-of-range token. */
int nso_gpt_fwd_bwd(nso_gpt* g, const float* idx, const float* targets, int B, int T,
                    float* loss, float* logits);
/* train_llm.cpp:112-129; returns the pre-clip norm. */
float nso_gpt_clip_gradients(nso_gpt* g, float max_norm);
/* include/optimizers.h:148-162 / 206-234 */
void nso_gpt_adamw_init(nso_gpt* g, float lr, float b1, float b2, float eps, float wd);
void nso_gpt_adamw_set_lr(nso_gpt* g, float lr);
void nso_gpt_adamw_step(nso_gpt* g);

#ifdef __cplusplus
}
#endif

#endif /* NS_ORACLE_H_ */
