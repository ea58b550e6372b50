/*
 * accel_b200_llama.h: the one-matmul and Llama C API of AccelEP, served by
 * the B200 backend.
 *
 * The functions named accel_sim_* and accel_llama_* keep the names,
 * argument meanings, return codes (0 ok, 1 failure with a thread-local
 * message) and struct layout of the reference API in
 * include/accel/sim_api.h:15-116, so the reference's ctypes bindings
 * (serve/sim.py:22-106, serve/llama.py:96-187) load this library unchanged.
 * Weights, activations, the KV cache and the chosen ids live in HBM of the
 * CUDA device that was current when the object was created.
 *
 * Additions (no reference counterpart; they extend the same API):
 *   accel_llama_weight_q8        int8 weights with per-output-row scales
 *   accel_llama_generate_batch   many independent sequences in one decode loop
 *   accel_llama_stream           the CUDA stream the model runs on
 *
 * The tokenizer entry points (accel_llama_tokenizer / encode / decode /
 * complete / complete_stream) are part of the reference's host-side text
 * path, which this backend does not re-implement: they fail with a message.
 */
#ifndef ACCEL_B200_LLAMA_H_
#define ACCEL_B200_LLAMA_H_

#include <stdint.h>

#include "accel_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ one matmul */

typedef struct AccelSim AccelSim;
typedef struct AccelBuf AccelBuf;

/* include/accel/sim_api.h:19-20. */
ACCEL_B200_API AccelSim* accel_sim_create(void);
ACCEL_B200_API void accel_sim_destroy(AccelSim* sim);
/* sim_api.h:22-24: copies `count` floats into HBM. */
ACCEL_B200_API AccelBuf* accel_sim_upload(AccelSim* sim, const float* data, int64_t count);
ACCEL_B200_API void accel_sim_release(AccelSim* sim, AccelBuf* buf);
/* sim_api.h:26-29: c[m, n] = a[m, k] @ b[k, n] with host a and c, b uploaded.
   Runs Device::MatMul, so the result has the reference's bits. */
ACCEL_B200_API int accel_sim_matmul(AccelSim* sim, const float* a, int64_t m, int64_t k, AccelBuf* b, int64_t n,
                                    float* c);
/* sim_api.h:31-37: process-wide counters of the backend. */
ACCEL_B200_API void accel_sim_reset_stats(void);
ACCEL_B200_API int64_t accel_sim_matmuls(void);
ACCEL_B200_API int64_t accel_sim_bytes_to_device(void);
ACCEL_B200_API int64_t accel_sim_bytes_to_host(void);
ACCEL_B200_API const char* accel_sim_last_error(void);

/* ------------------------------------------------------------------ llama */

typedef struct AccelLlama AccelLlama;

/* Layout of include/accel/sim_api.h:44-54. */
typedef struct AccelLlamaConfig {
  int32_t vocab;
  int32_t hidden;
  int32_t layers;
  int32_t heads;
  int32_t kv_heads;
  int32_t intermediate;
  int32_t context;
  float eps;
  float rope_theta;
} AccelLlamaConfig;

/* Weight kinds, values of include/accel/sim_api.h:56-69. */
enum {
  ACCEL_W_EMBED = 1,
  ACCEL_W_FINAL_NORM = 2,
  ACCEL_W_LM_HEAD = 3,
  ACCEL_W_ATTN_NORM = 4,
  ACCEL_W_POST_NORM = 5,
  ACCEL_W_Q = 6,
  ACCEL_W_K = 7,
  ACCEL_W_V = 8,
  ACCEL_W_O = 9,
  ACCEL_W_GATE = 10,
  ACCEL_W_UP = 11,
  ACCEL_W_DOWN = 12
};

ACCEL_B200_API AccelLlama* accel_llama_create(const AccelLlamaConfig* config);
ACCEL_B200_API void accel_llama_destroy(AccelLlama* model);
/* sim_api.h:73-75: Hugging Face layout, matrices [out, in], norms [dim] with cols 1. */
ACCEL_B200_API int accel_llama_weight(AccelLlama* model, int32_t kind, int32_t layer, const float* data, int64_t rows,
                                      int64_t cols);
/* Int8 form of a linear weight or the LM head: q is [rows = out, cols = in]
   (Hugging Face layout), dequantizing to float(q[o, i]) * scale[o]. The
   embedding table and the norms stay fp32 (accel_llama_weight). A model
   may mix fp32 and int8 linear weights. */
ACCEL_B200_API int accel_llama_weight_q8(AccelLlama* model, int32_t kind, int32_t layer, const int8_t* q,
                                         const float* scale, int64_t rows, int64_t cols);
ACCEL_B200_API int accel_llama_tokenizer(AccelLlama* model, const char* path);
/* sim_api.h:78-83. */
ACCEL_B200_API int accel_llama_generate(AccelLlama* model, const int32_t* prompt, int32_t prompt_count, int32_t max_new,
                                        int32_t eos_id, float temperature, uint32_t seed, int32_t top_k,
                                        int32_t* out_ids, int32_t* out_count);
/* `batch` independent sequences decoded together, each exactly as
   accel_llama_generate would decode it alone. prompts holds the prompts
   back to back, prompt_counts[b] ids each; seeds[b] seeds sequence b (NULL:
   `seed` for all). out_ids is [batch, max_new]; out_counts[b] is the number
   of ids sequence b produced. Each prompt must fit the context. The KV
   cache for `batch` sequences is allocated on first use and kept. */
ACCEL_B200_API int accel_llama_generate_batch(AccelLlama* model, const int32_t* prompts, const int32_t* prompt_counts,
                                              int32_t batch, int32_t max_new, int32_t eos_id, float temperature,
                                              uint32_t seed, const uint32_t* seeds, int32_t top_k, int32_t* out_ids,
                                              int32_t* out_counts);
ACCEL_B200_API int accel_llama_encode(AccelLlama* model, const char* text, int32_t text_len, int32_t* out_ids,
                                      int32_t out_cap, int32_t* out_count);
ACCEL_B200_API int accel_llama_decode(AccelLlama* model, const int32_t* ids, int32_t count, int32_t skip_special,
                                      char* out_text, int32_t out_cap, int32_t* out_len);
ACCEL_B200_API int accel_llama_complete(AccelLlama* model, const char* prompt, int32_t prompt_len, int32_t max_new,
                                        int32_t eos_id, float temperature, uint32_t seed, int32_t top_k,
                                        char* out_text, int32_t out_text_cap, int32_t* out_text_len, int32_t* out_ids,
                                        int32_t out_ids_cap, int32_t* out_count, int32_t* prompt_tokens);
typedef void (*AccelLlamaTokenFn)(int32_t token_id, void* user);
ACCEL_B200_API int accel_llama_complete_stream(AccelLlama* model, const char* prompt, int32_t prompt_len,
                                               int32_t max_new, int32_t eos_id, float temperature, uint32_t seed,
                                               int32_t top_k, char* out_text, int32_t out_text_cap,
                                               int32_t* out_text_len, int32_t* out_ids, int32_t out_ids_cap,
                                               int32_t* out_count, int32_t* prompt_tokens, AccelLlamaTokenFn on_token,
                                               void* user);
/* sim_api.h:109-114 test hooks: a forward that leaves logits in HBM, and the
   largest |logit - reference| computed on the device (the row itself is not
   copied back). */
ACCEL_B200_API int accel_llama_forward_ids(AccelLlama* model, const int32_t* ids, int32_t count, int32_t reset);
ACCEL_B200_API int accel_llama_logit_max_abs(AccelLlama* model, const float* reference, int32_t count,
                                             float* out_max_abs);
/* Copies the logit rows of the last forward to the host: count = r * vocab
   floats give rows 0..r-1 (one per sequence of the last forward or batched
   generate, in slot order). Test hook; not counted. */
ACCEL_B200_API int accel_llama_logits(AccelLlama* model, float* out, int32_t count);
/* Copies rows [0, rows) of one layer's key (which 0) or value (which 1) cache
   of sequence slot `slot` to the host in the reference layout [rows,
   kv_heads, head_dim]. Test hook; not counted. */
ACCEL_B200_API int accel_llama_cache_rows(AccelLlama* model, int32_t slot, int32_t layer, int32_t which, int32_t rows,
                                          float* out);
ACCEL_B200_API void accel_llama_reset(AccelLlama* model);
ACCEL_B200_API const char* accel_llama_last_error(void);
/* The cudaStream_t every launch of this model goes to. */
ACCEL_B200_API void* accel_llama_stream(AccelLlama* model);

#ifdef __cplusplus
}
#endif

#endif /* ACCEL_B200_LLAMA_H_ */
