/*
 * CPU restatement of AccelEP's SimDevice arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the B200
 * kernels. Only tests, the smoke check and the CPU-baseline leg of bench.py
 * load it. The product library never links or calls it.
 *
 * Every function restates one reference routine, in the same operation order
 * and with the same rounding points, so that its results are bit-identical to
 * the reference on the same host. Reference paths are relative to the AccelEP
 * project root. Build with -ffp-contract=off: the reference multiplies and
 * adds as two rounded steps (x86-64 baseline, no FMA), and a contracted
 * multiply-add would change the low bits.
 *
 * Pinned by tests/test_oracle.py against the reference's own known-answer
 * tests (tests/test_sim_kernels.cc, tests/test_runtime.cc) and against the
 * reference compiled from source (oracle/_ref, built by oracle/Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- kernels */

/* src/sim_embed.cc:9-20. Rows before a bad id are written; returns -1 at the
 * first id outside [0, vocab), like the reference's throw. */
ORC_API int orc_embed(const int32_t* ids, int64_t id_offset, const float* table, float* out, int64_t seq,
                      int64_t hidden, int64_t vocab) {
  for (int64_t s = 0; s < seq; ++s) {
    const int32_t id = ids[id_offset + s];
    if (id < 0 || id >= vocab) return -1;
    memcpy(out + s * hidden, table + (int64_t)id * hidden, (size_t)hidden * sizeof(float));
  }
  return 0;
}

/* src/sim_rmsnorm.cc:7-20. Sum of squares in double, one double reciprocal
 * square root, the product cast to float, then a float weight multiply. */
ORC_API void orc_rmsnorm(const float* x, const float* weight, float* y, int64_t rows, int64_t dim, float eps,
                         int64_t row_offset) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* in = x + (row_offset + r) * dim;
    float* out = y + r * dim;
    double square = 0.0;
    for (int64_t i = 0; i < dim; ++i) square += (double)in[i] * (double)in[i];
    const double inv = 1.0 / sqrt(square / (double)dim + (double)eps);
    for (int64_t i = 0; i < dim; ++i) out[i] = (float)((double)in[i] * inv) * weight[i];
  }
}

/* src/sim_rope.cc:5-21. Rotate-half pairs (i, i + half); tables hold full
 * head_dim rows at absolute positions. */
ORC_API void orc_rope(float* states, const float* cos_t, const float* sin_t, int64_t seq, int64_t n_heads,
                      int64_t head_dim, int64_t position) {
  const int64_t half = head_dim / 2;
  for (int64_t s = 0; s < seq; ++s) {
    const float* c = cos_t + (position + s) * head_dim;
    const float* sn = sin_t + (position + s) * head_dim;
    for (int64_t h = 0; h < n_heads; ++h) {
      float* row = states + (s * n_heads + h) * head_dim;
      for (int64_t i = 0; i < half; ++i) {
        const float a = row[i];
        const float b = row[half + i];
        row[i] = a * c[i] - b * sn[i];
        row[half + i] = b * c[half + i] + a * sn[half + i];
      }
    }
  }
}

/* src/sim_cache.cc:8-13. */
ORC_API void orc_append_cache(const float* src, float* cache, int64_t seq, int64_t position, int64_t n_heads,
                              int64_t head_dim) {
  const int64_t row = n_heads * head_dim;
  memcpy(cache + position * row, src, (size_t)(seq * row) * sizeof(float));
}

/* src/sim_attend.cc:9-46. Causal GQA; query head h reads kv head
 * h / (heads / kv_heads). Sequential float dot, max, expf, sum, and a
 * per-term division by the sum inside the value accumulation. */
ORC_API void orc_attend(const float* q, const float* k, const float* v, float* scores, float* out, int64_t seq,
                        int64_t position, int64_t heads, int64_t kv_heads, int64_t head_dim) {
  const float scale = 1.f / sqrtf((float)head_dim);
  const int64_t repeats = heads / kv_heads;
  for (int64_t s = 0; s < seq; ++s) {
    const int64_t limit = position + s;
    for (int64_t h = 0; h < heads; ++h) {
      const int64_t kv = h / repeats;
      const float* qv = q + (s * heads + h) * head_dim;
      float max_score = -INFINITY;
      for (int64_t t = 0; t <= limit; ++t) {
        const float* kr = k + (t * kv_heads + kv) * head_dim;
        float dot = 0.f;
        for (int64_t d = 0; d < head_dim; ++d) dot += qv[d] * kr[d];
        scores[t] = dot * scale;
        if (scores[t] > max_score) max_score = scores[t];
      }
      float sum = 0.f;
      for (int64_t t = 0; t <= limit; ++t) {
        scores[t] = expf(scores[t] - max_score);
        sum += scores[t];
      }
      float* dest = out + (s * heads + h) * head_dim;
      for (int64_t d = 0; d < head_dim; ++d) {
        float acc = 0.f;
        for (int64_t t = 0; t <= limit; ++t) acc += (scores[t] / sum) * v[(t * kv_heads + kv) * head_dim + d];
        dest[d] = acc;
      }
    }
  }
}

/* src/sim_silu.cc:8-13. */
ORC_API void orc_silu_mul(float* gate, const float* up, int64_t count) {
  for (int64_t i = 0; i < count; ++i) {
    const float x = gate[i];
    gate[i] = (x / (1.f + expf(-x))) * up[i];
  }
}

/* src/sim_add.cc:5-9. */
ORC_API void orc_add(float* dest, const float* extra, int64_t count) {
  for (int64_t i = 0; i < count; ++i) dest[i] += extra[i];
}

/* src/sim_sample.cc:9-16. xorshift32 with shifts 13, 17, 5. */
static uint32_t orc_next_rand(uint32_t* state) {
  uint32_t x = *state;
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  *state = x;
  return x;
}

typedef struct {
  int64_t id;
  float logit;
} OrcSlot;

/* src/sim_sample.cc:25-115. Greedy: first maximum wins. Otherwise a top-k
 * table of at most 64 slots (evicting the lowest logit, later id on ties),
 * re-sorted by id, or the whole vocabulary; a double exp walk against one
 * xorshift draw. */
ORC_API void orc_sample(const float* logits, int32_t* chosen, int64_t index, int64_t vocab, float temperature,
                        uint32_t* rng, int top_k) {
  if (!(temperature > 0.f)) {
    int64_t best = 0;
    float best_v = logits[0];
    for (int64_t i = 1; i < vocab; ++i) {
      if (logits[i] > best_v) {
        best_v = logits[i];
        best = i;
      }
    }
    chosen[index] = (int32_t)best;
    return;
  }
  const int full = top_k <= 0 || (int64_t)top_k >= vocab;
  int capped = top_k > 64 ? 64 : top_k;
  OrcSlot table[64];
  int filled = 0;
  if (!full) {
    for (int64_t i = 0; i < vocab; ++i) {
      const float value = logits[i];
      if (filled < capped) {
        table[filled].id = i;
        table[filled].logit = value;
        ++filled;
        continue;
      }
      int worst = 0;
      for (int s = 1; s < filled; ++s) {
        const int lower = table[s].logit < table[worst].logit;
        const int later_tie = table[s].logit == table[worst].logit && table[s].id > table[worst].id;
        if (lower || later_tie) worst = s;
      }
      if (value > table[worst].logit || (value == table[worst].logit && i < table[worst].id)) {
        table[worst].id = i;
        table[worst].logit = value;
      }
    }
    for (int i = 1; i < filled; ++i) {
      const OrcSlot key = table[i];
      int j = i;
      while (j > 0 && table[j - 1].id > key.id) {
        table[j] = table[j - 1];
        --j;
      }
      table[j] = key;
    }
  }
  float max_v = full ? logits[0] : table[0].logit;
  if (full) {
    for (int64_t i = 1; i < vocab; ++i)
      if (logits[i] > max_v) max_v = logits[i];
  } else {
    for (int s = 1; s < filled; ++s)
      if (table[s].logit > max_v) max_v = table[s].logit;
  }
  const double inv_t = 1.0 / (double)temperature;
  const int64_t span = full ? vocab : filled;
  double sum = 0.0;
  for (int64_t s = 0; s < span; ++s) {
    const int64_t id = full ? s : table[s].id;
    sum += exp(((double)logits[id] - (double)max_v) * inv_t);
  }
  if (!(sum > 0.0)) {
    chosen[index] = 0;
    return;
  }
  const double draw = ((double)orc_next_rand(rng) + 0.5) / 4294967296.0 * sum;
  double acc = 0.0;
  for (int64_t s = 0; s < span; ++s) {
    const int64_t id = full ? s : table[s].id;
    acc += exp(((double)logits[id] - (double)max_v) * inv_t);
    if (acc >= draw) {
      chosen[index] = (int32_t)id;
      return;
    }
  }
  chosen[index] = (int32_t)(full ? vocab - 1 : table[filled - 1].id);
}

/* ------------------------------------------------------------- matrices */

/* src/sim_device.cc:331-369 (PackedMatMul) and :387-402 (ReferenceMatMul).
 * The packed blocking never reorders one output's terms: each C[i, j] is a
 * k-ascending chain of rounded products added to a float accumulator. This
 * i-k-j loop keeps that chain. */
ORC_API void orc_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n) {
  for (int64_t i = 0; i < m; ++i) {
    float* row = c + i * n;
    for (int64_t j = 0; j < n; ++j) row[j] = 0.f;
    for (int64_t kk = 0; kk < k; ++kk) {
      const float aik = a[i * k + kk];
      const float* brow = b + kk * n;
      for (int64_t j = 0; j < n; ++j) {
        const float prod = aik * brow[j];
        row[j] = row[j] + prod;
      }
    }
  }
}

/* src/sim_device.cc:406-424 (DequantAt): (float(q) - zero) * scale, where
 * axis < 0 means one scale (and one zero) for the whole tensor. */
static float orc_dequant_at(const int8_t* q, const float* scale, const int8_t* zero, const int64_t* shape, int rank,
                            int64_t axis, int64_t index) {
  float sc = scale[0];
  float zp = 0.f;
  if (axis >= 0) {
    int64_t stride = 1;
    for (int d = rank - 1; d > axis; --d) stride *= shape[d];
    const int64_t coord = (index / stride) % shape[axis];
    sc = scale[coord];
    if (zero != NULL) zp = (float)zero[coord];
  } else if (zero != NULL) {
    zp = (float)zero[0];
  }
  return ((float)q[index] - zp) * sc;
}

/* src/sim_device.cc:541-602 (MatMulQuantized with a right-hand plane). The
 * panel holds dequantized weights; each output is the same k-ascending
 * chain as orc_matmul over those weights. `offset` is QuantPlane::offset. */
ORC_API int orc_matmul_q(const float* a, const int8_t* q, const float* scale, const int8_t* zero,
                         const int64_t* shape, int rank, int64_t axis, int64_t offset, float* c, int64_t m, int64_t k,
                         int64_t n) {
  if (m < 0 || k < 0 || n < 0) return -1;
  float* deq = (float*)malloc((size_t)(k * n > 0 ? k * n : 1) * sizeof(float));
  if (deq == NULL) return -2;
  for (int64_t kk = 0; kk < k; ++kk)
    for (int64_t j = 0; j < n; ++j)
      deq[kk * n + j] = orc_dequant_at(q, scale, zero, shape, rank, axis, offset + kk * n + j);
  orc_matmul(a, deq, c, m, k, n);
  free(deq);
  return 0;
}

/* src/sim_device.cc:104-124 (BiasOffset): bias shape right-aligned against
 * [m, n]; size-1 dimensions broadcast. */
static int64_t orc_bias_offset(const int64_t* shape, int rank, int64_t i, int64_t j) {
  if (rank == 0) return 0;
  int64_t strides[2] = {1, 1};
  for (int d = rank - 2; d >= 0; --d) strides[d] = strides[d + 1] * shape[d + 1];
  const int64_t coords[2] = {i, j};
  int64_t off = 0;
  for (int d = 0; d < rank; ++d) {
    int64_t coord = coords[2 - rank + d];
    if (shape[d] == 1) coord = 0;
    off += coord * strides[d];
  }
  return off;
}

/* src/sim_device.cc:211-245 (GemmEpilogue). act: 0 none, 1 relu, 2 gelu.
 * Relu keeps NaN and -0 (only value < 0 becomes +0); Gelu is the exact erf
 * form in float. */
ORC_API int orc_gemm_epilogue(float* c, int64_t m, int64_t n, float alpha, const float* bias,
                              const int64_t* bias_shape, int bias_rank, float beta, int act) {
  if (bias_rank > 2) return -1;
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      const float prod = alpha * c[i * n + j];
      float value = prod;
      if (bias != NULL) {
        const float bprod = beta * bias[orc_bias_offset(bias_shape, bias_rank, i, j)];
        value = value + bprod;
      }
      if (act == 1) {
        if (value < 0.f) value = 0.f;
      } else if (act == 2) {
        value = 0.5f * value * (1.f + erff(value * 0.7071067811865476f));
      }
      c[i * n + j] = value;
    }
  }
  return 0;
}

/* src/sim_device.cc:198-209. */
ORC_API void orc_transpose(const float* src, float* dst, int64_t rows, int64_t cols) {
  for (int64_t i = 0; i < rows; ++i)
    for (int64_t j = 0; j < cols; ++j) dst[j * rows + i] = src[i * cols + j];
}

/* src/runtime.cc:272-350, the int8 branch of ExecuteFusedImpl with a 2-D
 * activation and a right-hand plane: MatMulQuantized, then GemmEpilogue over
 * the flattened output for the activation (alpha 1 leaves values unchanged),
 * then a residual added through GemmEpilogue with beta 1. */
ORC_API int orc_execute_matmul_q(const float* x, int64_t m, int64_t k, const int8_t* q, const float* scale,
                                 const int8_t* zero, int64_t axis, int64_t n, int act, const float* residual,
                                 float* out) {
  const int64_t shape[2] = {k, n};
  int rc = orc_matmul_q(x, q, scale, zero, shape, 2, axis, 0, out, m, k, n);
  if (rc != 0) return rc;
  const int64_t count = m * n;
  if (count > 0 && act != 0) orc_gemm_epilogue(out, count, 1, 1.f, NULL, NULL, 0, 0.f, act);
  if (residual != NULL && count > 0) {
    const int64_t bshape[1] = {count};
    orc_gemm_epilogue(out, 1, count, 1.f, residual, bshape, 1, 1.f, 0);
  }
  return 0;
}

/* One block of the int8 MLP stack as the plugin runs it (src/ep.cc:1602-1626):
 * h = Gelu(x @ W1), s = h @ W2 + x, x' = RmsNorm(s). `hbuf` is scratch of
 * m * inter floats; `sbuf` receives the pre-norm sum (m * hidden). Per-column
 * scales (axis 1), no zero point. */
ORC_API int orc_mlp_block(const float* x, int64_t m, int64_t hidden, int64_t inter, const int8_t* w1,
                          const float* s1, const int8_t* w2, const float* s2, const float* gamma, float eps,
                          float* hbuf, float* sbuf, float* out) {
  int rc = orc_execute_matmul_q(x, m, hidden, w1, s1, NULL, 1, inter, 2, NULL, hbuf);
  if (rc != 0) return rc;
  rc = orc_execute_matmul_q(hbuf, m, inter, w2, s2, NULL, 1, hidden, 0, x, sbuf);
  if (rc != 0) return rc;
  orc_rmsnorm(sbuf, gamma, out, m, hidden, eps, 0);
  return 0;
}

/* ----------------------------------------------------------------- llama */

/* src/llama_model.cc. Weights are kept in the device layout the reference
 * uploads: matrices transposed to [in, out] (UploadTransposed, :75-84), norms
 * and the embedding table as given. */
typedef struct {
  float *attn_norm, *post_norm, *q, *k, *v, *o, *gate, *up, *down;
} OrcLayer;

typedef struct {
  int32_t vocab, hidden, layers, heads, kv_heads, inter, context, head_dim;
  float eps, theta;
  int32_t filled;
  float *embed, *final_norm, *lm_head, *cos_t, *sin_t;
  float *hid, *normed, *query, *key, *value, *mixed, *delta, *gate, *up, *logits, *scores;
  int32_t *chosen, *prompt_ids;
  OrcLayer* layer;
  float **kc, **vc;
} OrcLlama;

#define ORC_ALLOC(n) ((float*)calloc((size_t)(n) > 0 ? (size_t)(n) : 1, sizeof(float)))

/* src/llama_model.cc:318-395: buffers sized for the whole context, RoPE
 * tables built in double and rounded to float. cfg = {vocab, hidden, layers,
 * heads, kv_heads, intermediate, context}. */
ORC_API OrcLlama* orc_llama_create(const int32_t* cfg, float eps, float theta) {
  OrcLlama* m = (OrcLlama*)calloc(1, sizeof(OrcLlama));
  if (m == NULL) return NULL;
  m->vocab = cfg[0];
  m->hidden = cfg[1];
  m->layers = cfg[2];
  m->heads = cfg[3];
  m->kv_heads = cfg[4];
  m->inter = cfg[5];
  m->context = cfg[6];
  m->eps = eps;
  m->theta = theta;
  m->head_dim = m->hidden / m->heads;
  const int64_t ctx = m->context, dim = m->head_dim, half = dim / 2;
  m->cos_t = ORC_ALLOC(ctx * dim);
  m->sin_t = ORC_ALLOC(ctx * dim);
  for (int64_t pos = 0; pos < ctx; ++pos) {
    for (int64_t i = 0; i < half; ++i) {
      const double inv = 1.0 / pow((double)theta, (2.0 * (double)i) / (double)dim);
      const double angle = (double)pos * inv;
      const float c = (float)cos(angle);
      const float s = (float)sin(angle);
      m->cos_t[pos * dim + i] = c;
      m->cos_t[pos * dim + half + i] = c;
      m->sin_t[pos * dim + i] = s;
      m->sin_t[pos * dim + half + i] = s;
    }
  }
  const int64_t qn = ctx * m->heads * dim, kn = ctx * m->kv_heads * dim;
  m->hid = ORC_ALLOC(ctx * m->hidden);
  m->normed = ORC_ALLOC(ctx * m->hidden);
  m->query = ORC_ALLOC(qn);
  m->key = ORC_ALLOC(kn);
  m->value = ORC_ALLOC(kn);
  m->mixed = ORC_ALLOC(qn);
  m->delta = ORC_ALLOC(ctx * m->hidden);
  m->gate = ORC_ALLOC(ctx * m->inter);
  m->up = ORC_ALLOC(ctx * m->inter);
  m->logits = ORC_ALLOC(m->vocab);
  m->scores = ORC_ALLOC(ctx);
  m->chosen = (int32_t*)calloc((size_t)ctx, sizeof(int32_t));
  m->prompt_ids = (int32_t*)calloc((size_t)ctx, sizeof(int32_t));
  m->layer = (OrcLayer*)calloc((size_t)m->layers, sizeof(OrcLayer));
  m->kc = (float**)calloc((size_t)m->layers, sizeof(float*));
  m->vc = (float**)calloc((size_t)m->layers, sizeof(float*));
  for (int32_t l = 0; l < m->layers; ++l) {
    m->kc[l] = ORC_ALLOC(kn);
    m->vc[l] = ORC_ALLOC(kn);
  }
  return m;
}

ORC_API void orc_llama_destroy(OrcLlama* m) {
  if (m == NULL) return;
  float* bufs[] = {m->embed, m->final_norm, m->lm_head, m->cos_t, m->sin_t, m->hid,   m->normed,
                   m->query, m->key,        m->value,   m->mixed, m->delta, m->gate, m->up,
                   m->logits, m->scores};
  for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); ++i) free(bufs[i]);
  for (int32_t l = 0; l < m->layers; ++l) {
    OrcLayer* L = &m->layer[l];
    float* ws[] = {L->attn_norm, L->post_norm, L->q, L->k, L->v, L->o, L->gate, L->up, L->down};
    for (size_t i = 0; i < 9; ++i) free(ws[i]);
    free(m->kc[l]);
    free(m->vc[l]);
  }
  free(m->layer);
  free(m->kc);
  free(m->vc);
  free(m->chosen);
  free(m->prompt_ids);
  free(m);
}

/* Weight kinds follow include/accel/sim_api.h:56-69 (1 embed ... 12 down). */
ORC_API int orc_llama_weight(OrcLlama* m, int32_t kind, int32_t layer, const float* data, int64_t rows,
                             int64_t cols) {
  float** slot = NULL;
  if (kind == 1) slot = &m->embed;
  else if (kind == 2) slot = &m->final_norm;
  else if (kind == 3) slot = &m->lm_head;
  else {
    if (layer < 0 || layer >= m->layers) return -1;
    OrcLayer* L = &m->layer[layer];
    switch (kind) {
      case 4: slot = &L->attn_norm; break;
      case 5: slot = &L->post_norm; break;
      case 6: slot = &L->q; break;
      case 7: slot = &L->k; break;
      case 8: slot = &L->v; break;
      case 9: slot = &L->o; break;
      case 10: slot = &L->gate; break;
      case 11: slot = &L->up; break;
      case 12: slot = &L->down; break;
      default: return -1;
    }
  }
  free(*slot);
  float* buf = ORC_ALLOC(rows * cols);
  const int plain = kind == 1 || kind == 2 || kind == 4 || kind == 5;
  if (plain) {
    memcpy(buf, data, (size_t)(rows * cols) * sizeof(float));
  } else {
    orc_transpose(data, buf, rows, cols);
  }
  *slot = buf;
  return 0;
}

/* src/llama_model.cc:209-247 (Forward): the 17 calls per layer in the same
 * order, then the final norm of the last row and the M=1 vocabulary product. */
static int orc_llama_forward_at(OrcLlama* m, const int32_t* ids, int32_t seq, int64_t id_offset) {
  if (seq <= 0 || m->filled < 0 || seq > m->context || m->filled > m->context - seq) return -1;
  const int64_t H = m->hidden, D = m->head_dim, pos = m->filled;
  const int64_t qn = (int64_t)m->heads * D, kvn = (int64_t)m->kv_heads * D;
  if (orc_embed(ids, id_offset, m->embed, m->hid, seq, H, m->vocab) != 0) return -2;
  for (int32_t l = 0; l < m->layers; ++l) {
    OrcLayer* L = &m->layer[l];
    orc_rmsnorm(m->hid, L->attn_norm, m->normed, seq, H, m->eps, 0);
    orc_matmul(m->normed, L->q, m->query, seq, H, qn);
    orc_matmul(m->normed, L->k, m->key, seq, H, kvn);
    orc_matmul(m->normed, L->v, m->value, seq, H, kvn);
    orc_rope(m->query, m->cos_t, m->sin_t, seq, m->heads, D, pos);
    orc_rope(m->key, m->cos_t, m->sin_t, seq, m->kv_heads, D, pos);
    orc_append_cache(m->key, m->kc[l], seq, pos, m->kv_heads, D);
    orc_append_cache(m->value, m->vc[l], seq, pos, m->kv_heads, D);
    orc_attend(m->query, m->kc[l], m->vc[l], m->scores, m->mixed, seq, pos, m->heads, m->kv_heads, D);
    orc_matmul(m->mixed, L->o, m->delta, seq, qn, H);
    orc_add(m->hid, m->delta, seq * H);
    orc_rmsnorm(m->hid, L->post_norm, m->normed, seq, H, m->eps, 0);
    orc_matmul(m->normed, L->gate, m->gate, seq, H, m->inter);
    orc_matmul(m->normed, L->up, m->up, seq, H, m->inter);
    orc_silu_mul(m->gate, m->up, (int64_t)seq * m->inter);
    orc_matmul(m->gate, L->down, m->delta, seq, m->inter, H);
    orc_add(m->hid, m->delta, seq * H);
  }
  orc_rmsnorm(m->hid, m->final_norm, m->normed, 1, H, m->eps, (int64_t)seq - 1);
  orc_matmul(m->normed, m->lm_head, m->logits, 1, H, m->vocab);
  return 0;
}

/* src/llama_model.cc:150-166 (ForwardIds): reset clears the fill count. */
ORC_API int orc_llama_forward_ids(OrcLlama* m, const int32_t* ids, int32_t count, int32_t reset) {
  if (ids == NULL || count <= 0) return -1;
  if (reset) m->filled = 0;
  if (m->filled < 0 || count > m->context - m->filled) return -1;
  memcpy(m->prompt_ids, ids, (size_t)count * sizeof(int32_t));
  int rc = orc_llama_forward_at(m, m->prompt_ids, count, 0);
  if (rc != 0) return rc;
  m->filled += count;
  return 0;
}

/* Largest minus second-largest logit of the current row (ties give 0). */
static float orc_top2_gap(const float* row, int64_t n) {
  float a = -INFINITY, b = -INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    const float v = row[i];
    if (v > a) {
      b = a;
      a = v;
    } else if (v > b) {
      b = v;
    }
  }
  return a - b;
}

/* src/llama_model.cc:101-131 (Generate): prefill, then sample / forward until
 * max_new ids, the eos id, or a full context. `gaps`, when set, receives the
 * top-2 logit gap of the row each id was drawn from. */
ORC_API int orc_llama_generate(OrcLlama* m, const int32_t* prompt, int32_t prompt_count, int32_t max_new,
                               int32_t eos_id, float temperature, uint32_t seed, int32_t top_k, int32_t* out_ids,
                               int32_t* out_count, float* gaps) {
  m->filled = 0;
  if (prompt == NULL || prompt_count <= 0 || prompt_count > m->context) return -1;
  memcpy(m->prompt_ids, prompt, (size_t)prompt_count * sizeof(int32_t));
  int rc = orc_llama_forward_at(m, m->prompt_ids, prompt_count, 0);
  if (rc != 0) return rc;
  m->filled = prompt_count;
  uint32_t rng = seed == 0 ? 0x6d2b79f5u : seed;
  int32_t produced = 0;
  for (int32_t n = 0; n < max_new; ++n) {
    if (produced >= m->context) return -3;
    if (gaps != NULL) gaps[produced] = orc_top2_gap(m->logits, m->vocab);
    orc_sample(m->logits, m->chosen, produced, m->vocab, temperature, &rng, top_k);
    const int32_t id = m->chosen[produced];
    produced += 1;
    if (id == eos_id || m->filled >= m->context) break;
    rc = orc_llama_forward_at(m, m->chosen, 1, (int64_t)produced - 1);
    if (rc != 0) return rc;
    m->filled += 1;
  }
  memcpy(out_ids, m->chosen, (size_t)produced * sizeof(int32_t));
  *out_count = produced;
  return 0;
}

ORC_API const float* orc_llama_logits(const OrcLlama* m) { return m->logits; }
ORC_API int32_t orc_llama_filled(const OrcLlama* m) { return m->filled; }
/* which: 0 key cache, 1 value cache; layout [context, kv_heads, head_dim]. */
ORC_API const float* orc_llama_cache(const OrcLlama* m, int32_t layer, int32_t which) {
  if (layer < 0 || layer >= m->layers) return NULL;
  return which == 0 ? m->kc[layer] : m->vc[layer];
}
