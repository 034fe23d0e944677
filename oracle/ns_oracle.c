/*
 * Test infrastructure: NOT part of the product.
 *
 * Plain-C restatement of the NeuralSuite GPT training step.  See ns_oracle.h
 * for the contract.  Build: oracle/Makefile (gcc -O3 -ffp-contract=off, the
 * same no-FMA arithmetic as the reference's x86-64 Release build).
 *
 * Every loop below keeps the reference's summation order, because the tests
 * require this oracle to be bit-identical to the reference on the same inputs.
 */
#include "ns_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static float* falloc(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

/* src/tensor.cpp:198-271.  The reference computes four rows at a time, but
 * every C[i][j] still accumulates a[i][k]*b[k][j] for k = 0..K-1 in order,
 * starting from zero; that per-element order is all that fixes the bits. */
void nso_matmul(const float* A, const float* B, float* C, int M, int K, int N) {
  memset(C, 0, sizeof(float) * (size_t)M * N);
  for (int i = 0; i < M; ++i) {
    float* c = C + (size_t)i * N;
    for (int k = 0; k < K; ++k) {
      const float a = A[(size_t)i * K + k];
      const float* b = B + (size_t)k * N;
      for (int j = 0; j < N; ++j) c[j] += a * b[j];
    }
  }
}

/* src/tensor.cpp:275-288 */
void nso_transpose(const float* A, float* C, int M, int N) {
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) C[(size_t)j * M + i] = A[(size_t)i * N + j];
}

/* src/tensor.cpp:290-322 */
void nso_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* out,
                       float* mean, float* rstd, int rows, int dim, float eps) {
  for (int i = 0; i < rows; ++i) {
    const float* xr = x + (size_t)i * dim;
    float m = 0.0f;
    for (int j = 0; j < dim; ++j) m += xr[j];
    m /= (float)dim;
    mean[i] = m;
    float v = 0.0f;
    for (int j = 0; j < dim; ++j) {
      const float d = xr[j] - m;
      v += d * d;
    }
    v /= (float)dim;
    const float rs = 1.0f / sqrtf(v + eps);
    rstd[i] = rs;
    for (int j = 0; j < dim; ++j) out[(size_t)i * dim + j] = ((xr[j] - m) * rs) * gamma[j] + beta[j];
  }
}

/* src/tensor.cpp:324-359 */
void nso_layernorm_bwd(const float* dout, const float* x, const float* gamma, const float* mean,
                       const float* rstd, float* dx, float* dgamma, float* dbeta, int rows,
                       int dim) {
  memset(dgamma, 0, sizeof(float) * dim);
  memset(dbeta, 0, sizeof(float) * dim);
  for (int i = 0; i < rows; ++i) {
    const float m = mean[i], rs = rstd[i];
    const float* xr = x + (size_t)i * dim;
    const float* dr = dout + (size_t)i * dim;
    float s1 = 0.0f, s2 = 0.0f;
    for (int j = 0; j < dim; ++j) {
      const float xh = (xr[j] - m) * rs;
      const float d = dr[j];
      dgamma[j] += d * xh;
      dbeta[j] += d;
      const float dxh = d * gamma[j];
      s1 += dxh;
      s2 += dxh * xh;
    }
    const float scale = rs / (float)dim;
    for (int j = 0; j < dim; ++j) {
      const float xh = (xr[j] - m) * rs;
      const float dxh = dr[j] * gamma[j];
      dx[(size_t)i * dim + j] = scale * ((float)dim * dxh - s1 - xh * s2);
    }
  }
}

/* src/tensor.cpp:428-443 (tanh GELU, constants 0.7978845608 and 0.044715) */
void nso_gelu_fwd(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    const float cube = 0.044715f * v * v * v;
    const float inner = 0.7978845608f * (v + cube);
    y[i] = 0.5f * v * (1.0f + tanhf(inner));
  }
}

/* src/tensor.cpp:445-461 */
void nso_gelu_bwd(const float* dout, const float* x, float* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    const float cube = 0.044715f * v * v * v;
    const float inner = 0.7978845608f * (v + cube);
    const float th = tanhf(inner);
    const float d_inner = 0.7978845608f * (1.0f + 3.0f * 0.044715f * v * v);
    const float d_gelu = 0.5f * (1.0f + th) + 0.5f * v * (1.0f - th * th) * d_inner;
    dx[i] = dout[i] * d_gelu;
  }
}

/* src/tensor.cpp:394-426 */
void nso_causal_softmax(const float* in, float* out, int batch, int T) {
  for (int b = 0; b < batch; ++b) {
    for (int i = 0; i < T; ++i) {
      const size_t off = ((size_t)b * T + i) * T;
      float mx = in[off];
      for (int j = 1; j <= i; ++j)
        if (in[off + j] > mx) mx = in[off + j];
      float sum = 0.0f;
      for (int j = 0; j <= i; ++j) {
        const float e = expf(in[off + j] - mx);
        out[off + j] = e;
        sum += e;
      }
      for (int j = 0; j <= i; ++j) out[off + j] /= sum;
      for (int j = i + 1; j < T; ++j) out[off + j] = 0.0f;
    }
  }
}

/* include/losses.h:34-86 */
float nso_cross_entropy(const float* logits, const float* targets, int rows, int classes,
                        float* dlogits) {
  float total = 0.0f;
  for (int i = 0; i < rows; ++i) {
    const float* p = logits + (size_t)i * classes;
    const int t = (int)targets[i];
    float mx = p[0];
    for (int c = 1; c < classes; ++c)
      if (p[c] > mx) mx = p[c];
    float s = 0.0f;
    for (int c = 0; c < classes; ++c) s += expf(p[c] - mx);
    const float log_prob = (p[t] - mx) - logf(s);
    total -= log_prob;
    if (dlogits) {
      float* d = dlogits + (size_t)i * classes;
      for (int c = 0; c < classes; ++c) {
        const float prob = expf(p[c] - mx) / s;
        const float tv = (c == t) ? 1.0f : 0.0f;
        d[c] = (prob - tv) / (float)rows;
      }
    }
  }
  return total / (float)rows;
}

/* include/layers/embedding.h:34-59 */
int nso_embedding_fwd(const float* weight, int num, int dim, const float* idx, int n_tok,
                      float* out) {
  for (int i = 0; i < n_tok; ++i) {
    const int tok = (int)idx[i];
    if (tok < 0 || tok >= num) return -1;
  }
  for (int i = 0; i < n_tok; ++i) {
    const int tok = (int)idx[i];
    memcpy(out + (size_t)i * dim, weight + (size_t)tok * dim, sizeof(float) * dim);
  }
  return 0;
}

/* include/layers/embedding.h:61-80: zero, then scatter-add in (b, t) order;
 * the cached token of row r is idx[r % cached]. */
void nso_embedding_bwd(const float* idx, int n_tok, int cached, const float* dout, int dim,
                       int num, float* dweight) {
  memset(dweight, 0, sizeof(float) * (size_t)num * dim);
  if (cached == 0) return;
  for (int r = 0; r < n_tok; ++r) {
    const int tok = (int)idx[r % cached];
    float* w = dweight + (size_t)tok * dim;
    const float* d = dout + (size_t)r * dim;
    for (int j = 0; j < dim; ++j) w[j] += d[j];
  }
}

/* ---------------------------------------------------------------- Linear
 * include/layers/linear.h:59-116: Y = X*W + b (bias added after the GEMM);
 * dX = dY * W^T, dW = X^T * dY (overwritten), db = column sums (overwritten). */
static void linear_fwd(const float* X, const float* W, const float* b, float* Y, int N, int in,
                       int out) {
  nso_matmul(X, W, Y, N, in, out);
  for (int i = 0; i < N; ++i)
    for (int j = 0; j < out; ++j) Y[(size_t)i * out + j] += b[j];
}

static void linear_bwd(const float* X, const float* W, const float* dY, float* dX, float* dW,
                       float* db, int N, int in, int out) {
  float* Wt = falloc((size_t)in * out);
  nso_transpose(W, Wt, in, out);
  nso_matmul(dY, Wt, dX, N, out, in);
  free(Wt);
  float* Xt = falloc((size_t)N * in);
  nso_transpose(X, Xt, N, in);
  nso_matmul(Xt, dY, dW, in, N, out);
  free(Xt);
  memset(db, 0, sizeof(float) * out);
  for (int i = 0; i < N; ++i)
    for (int j = 0; j < out; ++j) db[j] += dY[(size_t)i * out + j];
}

/* ------------------------------------------------------------- attention */

/* Per-(b,h) core of MultiHeadAttention::Forward, attention.h:364-384.
 * qkv [B*T, 3C] interleaved; att [B*T, C] (head h in columns h*D..);
 * probs [B, H, T, T]. */
static void attn_core_fwd(const float* qkv, float* att, float* probs, int B, int T, int C, int H) {
  const int D = C / H;
  const float scale = 1.0f / sqrtf((float)D);
  float* Q = falloc((size_t)T * D);
  float* Kt = falloc((size_t)D * T);
  float* V = falloc((size_t)T * D);
  float* S = falloc((size_t)T * T);
  float* O = falloc((size_t)T * D);
  for (int b = 0; b < B; ++b) {
    for (int h = 0; h < H; ++h) {
      for (int i = 0; i < T; ++i) {
        const float* row = qkv + ((size_t)b * T + i) * 3 * C;
        for (int d = 0; d < D; ++d) {
          Q[(size_t)i * D + d] = row[h * D + d];
          Kt[(size_t)d * T + i] = row[C + h * D + d];
          V[(size_t)i * D + d] = row[2 * C + h * D + d];
        }
      }
      nso_matmul(Q, Kt, S, T, D, T);
      for (size_t i = 0; i < (size_t)T * T; ++i) S[i] *= scale;
      float* P = probs + ((size_t)b * H + h) * T * T;
      nso_causal_softmax(S, P, 1, T);
      nso_matmul(P, V, O, T, T, D);
      for (int i = 0; i < T; ++i)
        memcpy(att + ((size_t)b * T + i) * C + h * D, O + (size_t)i * D, sizeof(float) * D);
    }
  }
  free(Q); free(Kt); free(V); free(S); free(O);
}

/* Per-(b,h) core of MultiHeadAttention::Backward, attention.h:405-461,
 * including the double-precision row sum of dP*P (432-443). */
static void attn_core_bwd(const float* qkv, const float* probs, const float* datt, float* dqkv,
                          int B, int T, int C, int H) {
  const int D = C / H;
  const float scale = 1.0f / sqrtf((float)D);
  float* Q = falloc((size_t)T * D);
  float* K = falloc((size_t)T * D);
  float* V = falloc((size_t)T * D);
  float* dO = falloc((size_t)T * D);
  float* Vt = falloc((size_t)D * T);
  float* Pt = falloc((size_t)T * T);
  float* dP = falloc((size_t)T * T);
  float* dV = falloc((size_t)T * D);
  float* dS = falloc((size_t)T * T);
  float* dSt = falloc((size_t)T * T);
  float* dQ = falloc((size_t)T * D);
  float* dK = falloc((size_t)T * D);
  memset(dqkv, 0, sizeof(float) * (size_t)B * T * 3 * C);
  for (int b = 0; b < B; ++b) {
    for (int h = 0; h < H; ++h) {
      for (int i = 0; i < T; ++i) {
        const float* row = qkv + ((size_t)b * T + i) * 3 * C;
        for (int d = 0; d < D; ++d) {
          Q[(size_t)i * D + d] = row[h * D + d];
          K[(size_t)i * D + d] = row[C + h * D + d];
          V[(size_t)i * D + d] = row[2 * C + h * D + d];
          dO[(size_t)i * D + d] = datt[((size_t)b * T + i) * C + h * D + d];
        }
      }
      const float* P = probs + ((size_t)b * H + h) * T * T;
      nso_transpose(V, Vt, T, D);
      nso_transpose(P, Pt, T, T);
      nso_matmul(dO, Vt, dP, T, D, T);
      nso_matmul(Pt, dO, dV, T, T, D);
      for (int i = 0; i < T; ++i) {
        double acc = 0.0;
        for (int j = 0; j <= i; ++j) acc += (double)dP[(size_t)i * T + j] * P[(size_t)i * T + j];
        const float accf = (float)acc;
        for (int j = 0; j < T; ++j) {
          const float p = P[(size_t)i * T + j];
          dS[(size_t)i * T + j] = (j <= i) ? p * (dP[(size_t)i * T + j] - accf) * scale : 0.0f;
        }
      }
      nso_transpose(dS, dSt, T, T);
      nso_matmul(dS, K, dQ, T, T, D);
      nso_matmul(dSt, Q, dK, T, T, D);
      for (int i = 0; i < T; ++i) {
        float* row = dqkv + ((size_t)b * T + i) * 3 * C;
        memcpy(row + h * D, dQ + (size_t)i * D, sizeof(float) * D);
        memcpy(row + C + h * D, dK + (size_t)i * D, sizeof(float) * D);
        memcpy(row + 2 * C + h * D, dV + (size_t)i * D, sizeof(float) * D);
      }
    }
  }
  free(Q); free(K); free(V); free(dO); free(Vt); free(Pt); free(dP); free(dV);
  free(dS); free(dSt); free(dQ); free(dK);
}

int nso_mha(int B, int T, int C, int H, const float* w_attn, const float* b_attn,
            const float* w_proj, const float* b_proj, const float* x, const float* dout,
            float* y, float* dx, float* g_w_attn, float* g_b_attn, float* g_w_proj,
            float* g_b_proj) {
  if (H <= 0 || C <= 0 || C % H != 0) return -2;
  const int M = B * T;
  float* qkv = falloc((size_t)M * 3 * C);
  float* att = falloc((size_t)M * C);
  float* probs = falloc((size_t)B * H * T * T);
  linear_fwd(x, w_attn, b_attn, qkv, M, C, 3 * C);
  attn_core_fwd(qkv, att, probs, B, T, C, H);
  linear_fwd(att, w_proj, b_proj, y, M, C, C);
  if (dout) {
    float* datt = falloc((size_t)M * C);
    float* dqkv = falloc((size_t)M * 3 * C);
    linear_bwd(att, w_proj, dout, datt, g_w_proj, g_b_proj, M, C, C);
    attn_core_bwd(qkv, probs, datt, dqkv, B, T, C, H);
    linear_bwd(x, w_attn, dqkv, dx, g_w_attn, g_b_attn, M, C, 3 * C);
    free(datt);
    free(dqkv);
  }
  free(qkv); free(att); free(probs);
  return 0;
}

/* ------------------------------------------------------------- GPT model */

enum { P_LN1G, P_LN1B, P_WATT, P_BATT, P_WPRJ, P_BPRJ, P_LN2G, P_LN2B, P_WFC, P_BFC, P_WMP,
       P_BMP, P_PER_BLOCK };

typedef struct {
  /* forward caches of one GPTBlock (the Layers' last_input_ / caches) */
  float *x_in, *ln1_out, *ln1_mean, *ln1_rstd, *qkv, *att, *probs, *x1, *ln2_out, *ln2_mean,
      *ln2_rstd, *fc, *gelu;
} block_cache;

struct nso_gpt {
  int V, block, L, H, C;
  int n_tensors;
  int64_t* offset; /* per tensor, into params / grads */
  int64_t* numel;
  int* rank;
  int64_t total;
  float* params;
  float* grads;
  /* AdamW state (include/optimizers.h:240-252) */
  float *m, *v;
  float lr, b1, b2, eps, wd;
  int step;
  int have_opt;
  /* forward caches sized for the last (B, T) */
  int B, T;
  block_cache* cache;
  float *idx, *xf_in, *lnf_out, *lnf_mean, *lnf_rstd;
};

static void add_tensor(nso_gpt* g, int* k, int64_t n, int rank) {
  g->numel[*k] = n;
  g->rank[*k] = rank;
  g->offset[*k] = g->total;
  g->total += n;
  ++*k;
}

nso_gpt* nso_gpt_create(int vocab, int block, int n_layer, int n_head, int n_embd) {
  if (n_head <= 0 || n_embd <= 0 || n_embd % n_head != 0) return NULL;
  nso_gpt* g = (nso_gpt*)calloc(1, sizeof(nso_gpt));
  g->V = vocab; g->block = block; g->L = n_layer; g->H = n_head; g->C = n_embd;
  g->n_tensors = 2 + P_PER_BLOCK * n_layer + 2;
  g->offset = (int64_t*)calloc(g->n_tensors, sizeof(int64_t));
  g->numel = (int64_t*)calloc(g->n_tensors, sizeof(int64_t));
  g->rank = (int*)calloc(g->n_tensors, sizeof(int));
  const int64_t C = n_embd;
  int k = 0;
  add_tensor(g, &k, (int64_t)vocab * C, 2);
  add_tensor(g, &k, (int64_t)block * C, 2);
  for (int l = 0; l < n_layer; ++l) {
    add_tensor(g, &k, C, 1);
    add_tensor(g, &k, C, 1);
    add_tensor(g, &k, C * 3 * C, 2);
    add_tensor(g, &k, 3 * C, 1);
    add_tensor(g, &k, C * C, 2);
    add_tensor(g, &k, C, 1);
    add_tensor(g, &k, C, 1);
    add_tensor(g, &k, C, 1);
    add_tensor(g, &k, C * 4 * C, 2);
    add_tensor(g, &k, 4 * C, 1);
    add_tensor(g, &k, 4 * C * C, 2);
    add_tensor(g, &k, C, 1);
  }
  add_tensor(g, &k, C, 1);
  add_tensor(g, &k, C, 1);
  g->params = falloc((size_t)g->total);
  g->grads = falloc((size_t)g->total);
  g->cache = (block_cache*)calloc(n_layer, sizeof(block_cache));
  return g;
}

static void free_caches(nso_gpt* g) {
  for (int l = 0; l < g->L; ++l) {
    block_cache* c = &g->cache[l];
    free(c->x_in); free(c->ln1_out); free(c->ln1_mean); free(c->ln1_rstd); free(c->qkv);
    free(c->att); free(c->probs); free(c->x1); free(c->ln2_out); free(c->ln2_mean);
    free(c->ln2_rstd); free(c->fc); free(c->gelu);
    memset(c, 0, sizeof(*c));
  }
  free(g->idx); free(g->xf_in); free(g->lnf_out); free(g->lnf_mean); free(g->lnf_rstd);
  g->idx = g->xf_in = g->lnf_out = g->lnf_mean = g->lnf_rstd = NULL;
}

void nso_gpt_destroy(nso_gpt* g) {
  if (!g) return;
  free_caches(g);
  free(g->cache); free(g->offset); free(g->numel); free(g->rank);
  free(g->params); free(g->grads); free(g->m); free(g->v);
  free(g);
}

int nso_gpt_num_tensors(const nso_gpt* g) { return g->n_tensors; }
int64_t nso_gpt_tensor_numel(const nso_gpt* g, int i) { return g->numel[i]; }
int nso_gpt_tensor_rank(const nso_gpt* g, int i) { return g->rank[i]; }
int64_t nso_gpt_num_params(const nso_gpt* g) { return g->total; }
float* nso_gpt_params(nso_gpt* g) { return g->params; }
float* nso_gpt_grads(nso_gpt* g) { return g->grads; }

#define PAR(g, i) ((g)->params + (g)->offset[i])
#define GRD(g, i) ((g)->grads + (g)->offset[i])
#define BT(l, p) (2 + (l) * P_PER_BLOCK + (p))

static void ensure_caches(nso_gpt* g, int B, int T) {
  if (g->B == B && g->T == T && g->idx) return;
  free_caches(g);
  g->B = B; g->T = T;
  const size_t M = (size_t)B * T, C = g->C;
  for (int l = 0; l < g->L; ++l) {
    block_cache* c = &g->cache[l];
    c->x_in = falloc(M * C); c->ln1_out = falloc(M * C); c->ln1_mean = falloc(M);
    c->ln1_rstd = falloc(M); c->qkv = falloc(M * 3 * C); c->att = falloc(M * C);
    c->probs = falloc((size_t)B * g->H * T * T); c->x1 = falloc(M * C);
    c->ln2_out = falloc(M * C); c->ln2_mean = falloc(M); c->ln2_rstd = falloc(M);
    c->fc = falloc(M * 4 * C); c->gelu = falloc(M * 4 * C);
  }
  g->idx = falloc(M);
  g->xf_in = falloc(M * C); g->lnf_out = falloc(M * C);
  g->lnf_mean = falloc(M); g->lnf_rstd = falloc(M);
}

/* GPTModel::Forward, include/gpt.h:192-232, with GPTBlock::Forward 66-80. */
static int gpt_forward(nso_gpt* g, const float* idx, int B, int T, float* logits) {
  const int C = g->C, M = B * T;
  ensure_caches(g, B, T);
  memcpy(g->idx, idx, sizeof(float) * M);
  float* tok = falloc((size_t)M * C);
  if (nso_embedding_fwd(PAR(g, 0), g->V, C, idx, M, tok) != 0) {
    free(tok);
    return -1;
  }
  /* wpe.Forward over positions 0..T-1 (gpt.h:199-201); a position beyond the
   * table raises out_of_range just like a bad token. */
  if (T > g->block) {
    free(tok);
    return -1;
  }
  float* x = falloc((size_t)M * C);
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t)
      for (int d = 0; d < C; ++d)
        x[((size_t)b * T + t) * C + d] =
            tok[((size_t)b * T + t) * C + d] + PAR(g, 1)[(size_t)t * C + d];
  free(tok);
  float* tmp = falloc((size_t)M * C);
  for (int l = 0; l < g->L; ++l) {
    block_cache* c = &g->cache[l];
    memcpy(c->x_in, x, sizeof(float) * M * C);
    nso_layernorm_fwd(x, PAR(g, BT(l, P_LN1G)), PAR(g, BT(l, P_LN1B)), c->ln1_out, c->ln1_mean,
                      c->ln1_rstd, M, C, 1e-5f);
    linear_fwd(c->ln1_out, PAR(g, BT(l, P_WATT)), PAR(g, BT(l, P_BATT)), c->qkv, M, C, 3 * C);
    attn_core_fwd(c->qkv, c->att, c->probs, B, T, C, g->H);
    linear_fwd(c->att, PAR(g, BT(l, P_WPRJ)), PAR(g, BT(l, P_BPRJ)), tmp, M, C, C);
    for (size_t i = 0; i < (size_t)M * C; ++i) c->x1[i] = x[i] + tmp[i];
    nso_layernorm_fwd(c->x1, PAR(g, BT(l, P_LN2G)), PAR(g, BT(l, P_LN2B)), c->ln2_out,
                      c->ln2_mean, c->ln2_rstd, M, C, 1e-5f);
    linear_fwd(c->ln2_out, PAR(g, BT(l, P_WFC)), PAR(g, BT(l, P_BFC)), c->fc, M, C, 4 * C);
    nso_gelu_fwd(c->fc, c->gelu, (int64_t)M * 4 * C);
    linear_fwd(c->gelu, PAR(g, BT(l, P_WMP)), PAR(g, BT(l, P_BMP)), tmp, M, 4 * C, C);
    for (size_t i = 0; i < (size_t)M * C; ++i) x[i] = c->x1[i] + tmp[i];
  }
  free(tmp);
  const int lnf = 2 + P_PER_BLOCK * g->L;
  memcpy(g->xf_in, x, sizeof(float) * M * C);
  nso_layernorm_fwd(x, PAR(g, lnf), PAR(g, lnf + 1), g->lnf_out, g->lnf_mean, g->lnf_rstd, M, C,
                    1e-5f);
  free(x);
  /* logits = x_2d * Transpose(wte) (gpt.h:226-228) */
  float* wte_t = falloc((size_t)g->V * C);
  nso_transpose(PAR(g, 0), wte_t, g->V, C);
  nso_matmul(g->lnf_out, wte_t, logits, M, C, g->V);
  free(wte_t);
  return 0;
}

/* GPTModel::Backward, include/gpt.h:234-272, with GPTBlock::Backward 82-100. */
static void gpt_backward(nso_gpt* g, const float* dlogits) {
  const int B = g->B, T = g->T, C = g->C, M = B * T, V = g->V;
  float* dx = falloc((size_t)M * C);
  nso_matmul(dlogits, PAR(g, 0), dx, M, V, C);
  float* dl_t = falloc((size_t)M * V);
  nso_transpose(dlogits, dl_t, M, V);
  float* dwte_out = falloc((size_t)V * C);
  nso_matmul(dl_t, g->lnf_out, dwte_out, V, M, C);
  free(dl_t);
  const int lnf = 2 + P_PER_BLOCK * g->L;
  float* dcur = falloc((size_t)M * C);
  nso_layernorm_bwd(dx, g->xf_in, PAR(g, lnf), g->lnf_mean, g->lnf_rstd, dcur, GRD(g, lnf),
                    GRD(g, lnf + 1), M, C);
  float* t1 = falloc((size_t)M * 4 * C);
  float* t2 = falloc((size_t)M * 4 * C);
  float* dx1 = falloc((size_t)M * C);
  float* dqkv = falloc((size_t)M * 3 * C);
  for (int l = g->L - 1; l >= 0; --l) {
    block_cache* c = &g->cache[l];
    /* mlp_proj.Backward(dout) */
    linear_bwd(c->gelu, PAR(g, BT(l, P_WMP)), dcur, t1, GRD(g, BT(l, P_WMP)),
               GRD(g, BT(l, P_BMP)), M, 4 * C, C);
    /* mlp_gelu.Backward */
    nso_gelu_bwd(t1, c->fc, t2, (int64_t)M * 4 * C);
    /* mlp_fc.Backward -> [M, C] in t1 */
    linear_bwd(c->ln2_out, PAR(g, BT(l, P_WFC)), t2, t1, GRD(g, BT(l, P_WFC)),
               GRD(g, BT(l, P_BFC)), M, C, 4 * C);
    /* ln_2.Backward -> dx_norm2 in dx */
    nso_layernorm_bwd(t1, c->x1, PAR(g, BT(l, P_LN2G)), c->ln2_mean, c->ln2_rstd, dx,
                      GRD(g, BT(l, P_LN2G)), GRD(g, BT(l, P_LN2B)), M, C);
    for (size_t i = 0; i < (size_t)M * C; ++i) dx1[i] = dcur[i] + dx[i];
    /* attn.Backward(dx1): c_proj, core, c_attn */
    linear_bwd(c->att, PAR(g, BT(l, P_WPRJ)), dx1, t1, GRD(g, BT(l, P_WPRJ)),
               GRD(g, BT(l, P_BPRJ)), M, C, C);
    attn_core_bwd(c->qkv, c->probs, t1, dqkv, B, T, C, g->H);
    linear_bwd(c->ln1_out, PAR(g, BT(l, P_WATT)), dqkv, t2, GRD(g, BT(l, P_WATT)),
               GRD(g, BT(l, P_BATT)), M, C, 3 * C);
    /* ln_1.Backward */
    nso_layernorm_bwd(t2, c->x_in, PAR(g, BT(l, P_LN1G)), c->ln1_mean, c->ln1_rstd, dx,
                      GRD(g, BT(l, P_LN1G)), GRD(g, BT(l, P_LN1B)), M, C);
    for (size_t i = 0; i < (size_t)M * C; ++i) dcur[i] = dx1[i] + dx[i];
  }
  /* wte.Backward(dx), wpe.Backward(dx) (gpt.h:262-263), then the head term. */
  nso_embedding_bwd(g->idx, M, M, dcur, C, V, GRD(g, 0));
  float* pos = falloc((size_t)T);
  for (int t = 0; t < T; ++t) pos[t] = (float)t;
  nso_embedding_bwd(pos, M, T, dcur, C, g->block, GRD(g, 1));
  free(pos);
  float* gw = GRD(g, 0);
  for (size_t i = 0; i < (size_t)V * C; ++i) gw[i] += dwte_out[i];
  free(dx); free(dwte_out); free(dcur); free(t1); free(t2); free(dx1); free(dqkv);
}

int nso_gpt_fwd_bwd(nso_gpt* g, const float* idx, const float* targets, int B, int T,
                    float* loss, float* logits) {
  const int M = B * T;
  float* lg = logits ? logits : falloc((size_t)M * g->V);
  int rc = gpt_forward(g, idx, B, T, lg);
  if (rc == 0) {
    float* dl = falloc((size_t)M * g->V);
    *loss = nso_cross_entropy(lg, targets, M, g->V, dl);
    gpt_backward(g, dl);
    free(dl);
  }
  if (!logits) free(lg);
  return rc;
}

/* train_llm.cpp:112-129 */
float nso_gpt_clip_gradients(nso_gpt* g, float max_norm) {
  float total = 0.0f;
  for (int64_t i = 0; i < g->total; ++i) total += g->grads[i] * g->grads[i];
  const float norm = sqrtf(total);
  if (norm > max_norm && norm > 0.0f) {
    const float s = max_norm / norm;
    for (int64_t i = 0; i < g->total; ++i) g->grads[i] *= s;
  }
  return norm;
}

void nso_gpt_adamw_init(nso_gpt* g, float lr, float b1, float b2, float eps, float wd) {
  free(g->m); free(g->v);
  g->m = falloc((size_t)g->total);
  g->v = falloc((size_t)g->total);
  g->lr = lr; g->b1 = b1; g->b2 = b2; g->eps = eps; g->wd = wd;
  g->step = 0;
  g->have_opt = 1;
}

void nso_gpt_adamw_set_lr(nso_gpt* g, float lr) { g->lr = lr; }

/* include/optimizers.h:206-234.  std::pow(float, int) is evaluated in double
 * (C++11 promotion), and the float locals round the result. */
void nso_adamw_flat(float* params, const float* grads, float* m, float* v, const int64_t* offsets,
                    const float* decay, int n_seg, float lr, float b1, float b2, float eps,
                    int step) {
  const float bc1 = (float)(1.0f - pow((double)b1, (double)step));
  const float bc2 = (float)(1.0f - pow((double)b2, (double)step));
  for (int t = 0; t < n_seg; ++t) {
    const float d = decay[t];
    for (int64_t k = offsets[t]; k < offsets[t + 1]; ++k) {
      const float gk = grads[k];
      m[k] = b1 * m[k] + (1.0f - b1) * gk;
      v[k] = b2 * v[k] + (1.0f - b2) * gk * gk;
      const float mh = m[k] / bc1;
      const float vh = v[k] / bc2;
      if (d > 0.0f) params[k] -= lr * d * params[k];
      params[k] -= lr * mh / (sqrtf(vh) + eps);
    }
  }
}

void nso_gpt_adamw_step(nso_gpt* g) {
  g->step++;
  float* decay = falloc((size_t)g->n_tensors);
  int64_t* offs = (int64_t*)calloc((size_t)g->n_tensors + 1, sizeof(int64_t));
  for (int t = 0; t < g->n_tensors; ++t) {
    decay[t] = g->rank[t] >= 2 ? g->wd : 0.0f;
    offs[t] = g->offset[t];
  }
  offs[g->n_tensors] = g->total;
  nso_adamw_flat(g->params, g->grads, g->m, g->v, offs, decay, g->n_tensors, g->lr, g->b1, g->b2,
                 g->eps, g->step);
  free(decay);
  free(offs);
}
