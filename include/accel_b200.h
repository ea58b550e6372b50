/*
 * accel_b200.h: the C ABI of the B200 kernels behind AccelEP's device calls.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL is the legacy default stream) and
 * returns 0 or a nonzero ACCEL_B200_E* status. The message of the last
 * failure on the calling thread is in accel_b200_last_error(). Launches are
 * asynchronous: a status of 0 means the launch was accepted, and an error a
 * kernel detects on the device (for example a token id outside the
 * vocabulary) is raised through a device status word the caller passes.
 *
 * Each entry point replaces one routine of the reference SimDevice; the
 * citation names the reference file and line (paths relative to the AccelEP
 * project root). Floating-point results agree with the reference within
 * rtol = atol = 1e-4; index, copy and integer results are bit-identical.
 * Entry points marked "bit-exact" also round every floating-point step where
 * the reference does and so give the reference's bits.
 */
#ifndef ACCEL_B200_H_
#define ACCEL_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define ACCEL_B200_API __declspec(dllexport)
#else
#define ACCEL_B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ACCEL_B200_OK = 0,
  ACCEL_B200_EINVAL = 1,    /* argument out of range: std::invalid_argument in the reference */
  ACCEL_B200_EOVERFLOW = 2, /* size arithmetic overflows: std::overflow_error in the reference */
  ACCEL_B200_ECUDA = 3,     /* a CUDA runtime call failed */
  ACCEL_B200_EDEVICE = 4,   /* a kernel reported an error through its status word */
  ACCEL_B200_ENOMEM = 5     /* an allocation failed: std::bad_alloc in the reference */
};

/* Activation codes: include/accel/device.h:11 (Activation::None/Relu/Gelu). */
enum { ACCEL_B200_ACT_NONE = 0, ACCEL_B200_ACT_RELU = 1, ACCEL_B200_ACT_GELU = 2 };

/* Bits of a device status word written by kernels that validate data or
   that gave up a bounded wait. */
enum { ACCEL_B200_STATUS_BAD_TOKEN = 1, ACCEL_B200_STATUS_COPY_TIMEOUT = 2 };

ACCEL_B200_API const char* accel_b200_last_error(void);
/* Number of kernel launches this library has issued in this process
   (each replayed graph node counts once per replay). */
ACCEL_B200_API int64_t accel_b200_launch_count(void);

/* ---------------------------------------------------------- named kernels */

/* src/sim_embed.cc:9-20. out[s, :] = table[ids[id_offset + s], :]. An id
   outside [0, vocab) leaves its row untouched and ORs
   ACCEL_B200_STATUS_BAD_TOKEN into *status (device int; may be NULL).
   Bit-exact. */
ACCEL_B200_API int accel_b200_embed(const int32_t* ids, int64_t id_offset, const float* table, float* out, int64_t seq,
                                    int64_t hidden, int64_t vocab, int32_t* status, void* stream);

/* src/sim_rmsnorm.cc:7-20. y[r, :] = float(x[row_offset + r, :] * inv) * w with the
   sum of squares and inv in double. */
ACCEL_B200_API int accel_b200_rmsnorm(const float* x, const float* weight, float* y, int64_t rows, int64_t dim,
                                      float eps, int64_t row_offset, void* stream);

/* src/sim_rope.cc:5-21. In-place rotate-half RoPE on [seq, n_heads, head_dim]
   with table rows at absolute positions position + s. Bit-exact. */
ACCEL_B200_API int accel_b200_rope(float* states, const float* cos_table, const float* sin_table, int64_t seq,
                                   int64_t n_heads, int64_t head_dim, int64_t position, void* stream);

/* src/sim_cache.cc:8-13. Copies seq rows of n_heads * head_dim floats into
   cache rows [position, position + seq). Bit-exact. */
ACCEL_B200_API int accel_b200_append_cache(const float* src, float* cache, int64_t seq, int64_t position,
                                           int64_t n_heads, int64_t head_dim, void* stream);

/* src/sim_attend.cc:9-46. Causal grouped-query attention. q and out are
   [seq, heads, head_dim]; k and v hold rows [0, position + seq) of
   [rows, kv_heads, head_dim]. heads must be a multiple of kv_heads. The
   reference's `scores` scratch is not needed. */
ACCEL_B200_API int accel_b200_attention(const float* q, const float* k, const float* v, float* out, int64_t seq,
                                        int64_t position, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                        void* stream);

/* src/sim_silu.cc:8-13. gate[i] = gate[i] / (1 + exp(-gate[i])) * up[i]. */
ACCEL_B200_API int accel_b200_silu_mul(float* gate, const float* up, int64_t count, void* stream);

/* src/sim_add.cc:5-9. dest[i] += extra[i]. Bit-exact. */
ACCEL_B200_API int accel_b200_residual_add(float* dest, const float* extra, int64_t count, void* stream);

/* src/sim_sample.cc:25-115. Writes one int32 at chosen[chosen_index].
   temperature <= 0: argmax, the earlier id wins a tie (bit-exact). Otherwise
   top-k (at most 64 logits, walked in id order) or the whole vocabulary,
   with one xorshift32 draw from *rng_state (a device uint32, advanced in
   place like the reference's host state). */
ACCEL_B200_API int accel_b200_sample(const float* logits, int32_t* chosen, int64_t chosen_index, int64_t vocab,
                                     float temperature, uint32_t* rng_state, int32_t top_k, void* stream);

/* Greedy choice for `rows` logit rows of row stride ld: chosen[r * chosen_stride
   + chosen_offset] = argmax(logits[r, :]). Same tie and NaN rules as
   accel_b200_sample at temperature 0 (batched form of src/sim_sample.cc:27-38). */
ACCEL_B200_API int accel_b200_argmax_rows(const float* logits, int64_t rows, int64_t vocab, int64_t ld, int32_t* chosen,
                                          int64_t chosen_stride, int64_t chosen_offset, void* stream);

/* ---------------------------------------------------------------- matrices */

/* src/sim_device.cc:185-196 (MatMul -> PackedMatMul :331-369). Row-major
   C[m, n] = A[m, k] @ B[k, n], each output a k-ascending chain of rounded
   products and rounded adds, as the reference computes it. Bit-exact. */
ACCEL_B200_API int accel_b200_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n,
                                     void* stream);

/* src/sim_device.cc:198-209. dst[j, i] = src[i, j]; src is [rows, cols]. Bit-exact. */
ACCEL_B200_API int accel_b200_transpose(const float* src, float* dst, int64_t rows, int64_t cols, void* stream);

/* src/sim_device.cc:211-245 with BiasOffset :104-124.
   c = act(alpha * c + beta * broadcast(bias)); bias may be NULL; bias_shape
   (rank 0..2) is right-aligned against [m, n] with size-1 axes broadcast.
   Relu keeps NaN and -0; Gelu is 0.5 x (1 + erf(x / sqrt 2)). */
ACCEL_B200_API int accel_b200_gemm_epilogue(float* c, int64_t m, int64_t n, float alpha, const float* bias,
                                            const int64_t* bias_shape, int32_t bias_rank, float beta, int32_t act,
                                            void* stream);

/* An int8 weight plane (include/accel/runtime.h:71-78, QuantPlane) holding B
   of a [k, n] product. The element at (kk, j) is q[offset + kk * n + j] and
   dequantizes to (float(q) - zero) * scale, with scale and zero indexed by the
   plane's `axis` coordinate of a [k, n] tensor (axis 0: per row kk, axis 1:
   per column j, -1: one value). `zero` may be NULL. */
typedef struct accel_b200_q8_plane {
  const int8_t* q;
  const float* scale;
  const int8_t* zero;
  int64_t offset;
  int32_t axis;
} accel_b200_q8_plane;

/* Output stage fused into a product (src/runtime.cc:332-344 and
   sim_device.cc:211-245): out = act(alpha * acc + beta * bias) + residual.
   bias is NULL or broadcast by (bias_row_stride, bias_col_stride) in floats
   (0 for a broadcast axis); residual is NULL or [m, n] with row stride
   residual_ld. residual may alias the output. */
typedef struct accel_b200_epilogue {
  float alpha;
  float beta;
  const float* bias;
  int64_t bias_row_stride;
  int64_t bias_col_stride;
  int32_t act;
  const float* residual;
  int64_t residual_ld;
  /* Optional (NULL: none), int8 products on the GEMV and tensor-core paths:
     for each output row r and each 128-column block t of the output, the sum
     of squares of the final output values (in double; the four values a lane
     holds in order, then a butterfly over the block's 32 lanes) is written to
     row_sq[r * row_sq_ld + t], row_sq_ld >= ceil(n / 128). A following
     RmsNorm-fed product reads these sums instead of the rows
     (accel_b200_matmul_q8_rmsnorm_stats). */
  double* row_sq;
  int64_t row_sq_ld;
  /* Launch options (0: none). ACCEL_B200_EP_TRIGGER_AFTER_WAIT, on the GEMV
     and tensor-core paths: the product lets the next kernel of the stream
     launch early (programmatic dependent launch) only once it has itself
     waited for the kernel before it, instead of at entry. When the next
     kernel starts, every kernel before this product has then completed. No
     effect on results. */
  int32_t flags;
} accel_b200_epilogue;

#define ACCEL_B200_EP_TRIGGER_AFTER_WAIT 1

/* Scratch, in bytes, accel_b200_matmul_q8 needs for these sizes. */
ACCEL_B200_API size_t accel_b200_matmul_q8_workspace(int64_t m, int64_t k, int64_t n);

/* Which kernel the int8 products launched FROM THE CALLING THREAD use: 0 by
   shape (the default: for per-column or single scales without zero points
   and 16-byte aligned rows, the int8 GEMV for m <= 8 and the tcgen05
   tensor-core kernel above; CUDA cores otherwise), 1 CUDA cores only, 2 the
   tensor-core kernel where eligible, 3 the GEMV where eligible. The choice is
   thread-local: products launched by other threads (another model, another
   device) keep the by-shape choice. For comparisons and tests. */
ACCEL_B200_API int accel_b200_set_q8_path(int32_t path);

/* src/sim_device.cc:541-602 (MatMulQuantized with a right-hand plane) and
   the epilogue the runtime applies after it (src/runtime.cc:326-344):
   c[m, n] = epilogue(A[m, k] @ dequant(B)), with A fp32 row-major (row
   stride lda) and C row stride ldc. ep may be NULL (plain product).
   workspace must hold accel_b200_matmul_q8_workspace(m, k, n) bytes whose
   first 64 KiB were zero before the first call (arrival counters, left zero
   by every call); calls that share a workspace must not overlap on the GPU. */
ACCEL_B200_API int accel_b200_matmul_q8(const float* a, int64_t lda, const accel_b200_q8_plane* b, float* c,
                                        int64_t ldc, int64_t m, int64_t k, int64_t n,
                                        const accel_b200_epilogue* ep, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* accel_b200_matmul_q8 that also stores every output element to each of
   `n_peers` (<= 7) peer buffers at the same offset from the peer's base as
   from `c`: device memory of other GPUs mapped into this process (symmetric
   memory), written over NVLink from the product's epilogue. No reference
   counterpart: the reference runs one device. It fuses the all-gather of the
   N-sharded C5 product into the product: rank r passes c = Y + r * Nr (its
   column block of a row-major Y [m, N], ldc = N) and the same column block of
   every peer's Y. Only the GEMV and tensor-core paths take peers (per-column
   or single scale, no zero points, 16-byte aligned rows); the caller
   synchronizes the ranks (all stores of a launch are visible system-wide when
   it completes). */
ACCEL_B200_API int accel_b200_matmul_q8_peers(const float* a, int64_t lda, const accel_b200_q8_plane* b, float* c,
                                              int64_t ldc, int64_t m, int64_t k, int64_t n, float* const* peers,
                                              int32_t n_peers, const accel_b200_epilogue* ep, void* workspace,
                                              size_t workspace_bytes, void* stream);

/* Barrier of `world` (<= 8) ranks over peer memory, for the fused product +
   all-gather above. No reference counterpart. peer_flags[p] is rank p's array
   of `world` int32 flags (symmetric memory mapped into this process;
   peer_flags[rank] may be NULL) and my_flags this rank's own array, all zero
   before the first call; *epoch_counter is a device int32 of this rank,
   zero before the first call, that the kernel advances by one per call (so a
   captured launch replays correctly). Rank `rank` stores the new epoch into
   slot `rank` of every peer's array and waits until every peer's slot in its
   own array holds at least that epoch. The wait is bounded by limit_cycles SM
   clock cycles (<= 0: about one second); a peer that does not arrive in time
   ORs ACCEL_B200_STATUS_COPY_TIMEOUT into *status (device int, may be NULL)
   and the call returns. Run one rank per GPU, every rank calling equally
   often. */
ACCEL_B200_API int accel_b200_peer_barrier(int32_t* const* peer_flags, int32_t* my_flags, int32_t rank, int32_t world,
                                           int32_t* epoch_counter, int64_t limit_cycles, int32_t* status,
                                           void* stream);

/* c[m, n] = epilogue(SiluMul(gate_up) @ dequant(b)) for fused gate|up rows:
   row r of the product's A is silu(g) * u with g = gate_up[r * ld + i] and
   u = gate_up[r * ld + inter + i], i < inter (src/sim_silu.cc:8-13 followed by
   the down projection, src/llama_model.cc:239-240), so k = inter. The SiluMul
   value is rounded exactly as accel_b200_silu_mul_rows rounds it; the
   product and epilogue are those of accel_b200_matmul_q8. `workspace` holds
   accel_b200_matmul_q8_silu_workspace(m, inter, n) bytes whose first 64 KiB
   are zero (the same rule as accel_b200_matmul_q8). */
ACCEL_B200_API size_t accel_b200_matmul_q8_silu_workspace(int64_t m, int64_t inter, int64_t n);
ACCEL_B200_API int accel_b200_matmul_q8_silu(const float* gate_up, int64_t ld, int64_t inter,
                                             const accel_b200_q8_plane* b, float* c, int64_t ldc, int64_t m,
                                             int64_t n, const accel_b200_epilogue* ep, void* workspace,
                                             size_t workspace_bytes, void* stream);

/* c[m, n] = epilogue(RmsNorm(x) @ dequant(b)): row r of the product's A is
   RmsNorm of x row r (length k, row stride ldx) with weights gamma [k] and
   eps (src/sim_rmsnorm.cc:7-20 followed by the projection, as
   src/llama_model.cc:228-229 and :237-238 chain them). The normalized values
   are bit-identical to accel_b200_rmsnorm's; product and epilogue as
   accel_b200_matmul_q8. `workspace` holds
   accel_b200_matmul_q8_rmsnorm_workspace(m, k, n) bytes whose first 64 KiB
   are zero. */
ACCEL_B200_API size_t accel_b200_matmul_q8_rmsnorm_workspace(int64_t m, int64_t k, int64_t n);
/* The same with each row's sum of squares supplied by the kernel that wrote
   x (accel_b200_epilogue.row_sq): row_sq[r * row_sq_ld + t], t < row_sq_n,
   added in order, replaces reading the whole row. No reference counterpart
   (the norm itself is src/sim_rmsnorm.cc:7-20). The normalized values equal
   accel_b200_matmul_q8_rmsnorm's up to the last bit of the double sum of
   squares (another summation order). Where the planes pass runs (m > 64 or
   long K) the rows are read as in accel_b200_matmul_q8_rmsnorm. */
ACCEL_B200_API int accel_b200_matmul_q8_rmsnorm_stats(const float* x, int64_t ldx, const double* row_sq,
                                                      int64_t row_sq_ld, int32_t row_sq_n, const float* gamma,
                                                      float eps, const accel_b200_q8_plane* b, float* c, int64_t ldc,
                                                      int64_t m, int64_t k, int64_t n, const accel_b200_epilogue* ep,
                                                      void* workspace, size_t workspace_bytes, void* stream);

/* RmsNorm rows (as accel_b200_matmul_q8_rmsnorm; with row_sq non-NULL, from
   the row sums of squares as accel_b200_matmul_q8_rmsnorm_stats) through a
   fused gate|up product, then SiluMul (src/sim_silu.cc:8-13, the MLP of
   src/llama_model.cc:237-240) in the product's epilogue. The plane's n
   columns (n % 128 == 0) hold gate and up in 64-column pairs: columns
   128 t .. 128 t + 63 are gate columns 64 t .. 64 t + 63 and columns
   128 t + 64 .. 128 t + 127 the up columns of the same outputs. c[m, n / 2]
   (row stride ldc) receives SiluMul(gate, up) of output columns 0 .. n / 2,
   each value as the plain product followed by accel_b200_silu_mul_rows
   computes it. Tensor-core path only (per-column or single scales, no zero
   points, k % 8 == 0, 16-byte aligned rows and gamma); the workspace is
   accel_b200_matmul_q8_rmsnorm_workspace(m, k, n). */
ACCEL_B200_API int accel_b200_matmul_q8_rmsnorm_silu_pairs(const float* x, int64_t ldx, const double* row_sq,
                                                           int64_t row_sq_ld, int32_t row_sq_n, const float* gamma,
                                                           float eps, const accel_b200_q8_plane* b, float* c,
                                                           int64_t ldc, int64_t m, int64_t k, int64_t n,
                                                           void* workspace, size_t workspace_bytes, void* stream);
ACCEL_B200_API int accel_b200_matmul_q8_rmsnorm(const float* x, int64_t ldx, const float* gamma, float eps,
                                                const accel_b200_q8_plane* b, float* c, int64_t ldc, int64_t m,
                                                int64_t k, int64_t n, const accel_b200_epilogue* ep, void* workspace,
                                                size_t workspace_bytes, void* stream);

/* fp32 weights with the same fused epilogue and split-K scheme: the fast
   (fused multiply-add, reassociated) product the Llama engine uses. */
ACCEL_B200_API size_t accel_b200_matmul_f32_workspace(int64_t m, int64_t k, int64_t n);
ACCEL_B200_API int accel_b200_matmul_f32(const float* a, int64_t lda, const float* b, float* c, int64_t ldc, int64_t m,
                                         int64_t k, int64_t n, const accel_b200_epilogue* ep, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* ------------------------------------------------- batched decode kernels
   Fused forms of reference call sequences, used by the Llama engine
   (src/llama_model.cc:209-247 and :101-131). Rows of one launch may belong
   to different sequences: `row_seq[r]` is a row's sequence slot and
   `row_pos[r]` its absolute position (-1: a finished sequence, skipped). */

/* Rope on the query and key heads and AppendCache of key and value
   (src/llama_model.cc:229-232) over fused projection rows
   qkv[r] = [q (heads * head_dim) | k (kv_heads * head_dim) | v]. Queries are
   rotated in place; keys and values land in cache row row_pos[r] of slot
   row_seq[r] (row_seq may be NULL: slot 0). Element (slot s, kv head g,
   row t, dim d) of a cache is at s * seq_stride + g * head_stride + t *
   row_stride + d (floats): the reference layout [context, kv_heads,
   head_dim] is (head_stride, row_stride) = (head_dim, kv_heads * head_dim).
   Bit-exact. */
ACCEL_B200_API int accel_b200_rope_append(float* qkv, int64_t qkv_ld, const int32_t* row_seq, const int32_t* row_pos,
                                          int64_t rows, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                          const float* cos_table, const float* sin_table, float* k_cache,
                                          float* v_cache, int64_t cache_seq_stride, int64_t cache_head_stride,
                                          int64_t cache_row_stride, void* stream);

/* Causal attention of each row over its own sequence's cache rows
   [0, row_pos[r]] (src/sim_attend.cc:9-46 with per-row sequence and
   position). q row r: q + r * q_row_stride; cache strides as in
   accel_b200_rope_append. */
ACCEL_B200_API int accel_b200_attention_rows(const float* q, int64_t q_row_stride, const float* k, const float* v,
                                             int64_t kv_row_stride, int64_t kv_head_stride, int64_t kv_seq_stride,
                                             float* out, int64_t out_row_stride, const int32_t* row_seq,
                                             const int32_t* row_pos, int64_t rows, int32_t heads, int32_t kv_heads,
                                             int32_t head_dim, void* stream);

/* Causal attention of prefill rows, tiled (src/sim_attend.cc:9-46 over the
   prompt rows of `batch` sequences, src/llama_model.cc:233). The rows of
   sequence b are q rows first[b] .. first[b] + count[b] - 1 (device arrays)
   at positions pos0[b] + i, attending to cache rows [0, pos0[b] + i] of slot
   b; max_rows >= every count[b]. head_dim 64, at most 4 query heads per kv
   head; the cache is head-major as in accel_b200_decode_attention (rows of
   64 floats, element (s, g, t, d) at s * seq_stride + g * head_stride + t * 64
   + d) and already holds the roped keys of these rows. Agrees with
   accel_b200_attention_rows within 1e-4. */
ACCEL_B200_API int accel_b200_attention_prefill(const float* q, int64_t q_stride, const float* k_cache,
                                                const float* v_cache, int64_t seq_stride, int64_t head_stride,
                                                float* out, int64_t out_stride, const int32_t* first,
                                                const int32_t* count, const int32_t* pos0, int32_t batch,
                                                int32_t max_rows, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                                void* stream);

/* Split-KV decode attention, head_dim 64: one query row per sequence b over
   cache rows [0, lens[b]) of slot b (1 <= lens[b] <= max_len; cache strides
   as in accel_b200_rope_append, 16-byte aligned). Chunks of `chunk` (<= 128)
   rows are reduced in parallel into `workspace` and merged in chunk order by
   the last CTA of each (sequence, kv head). The workspace must hold
   accel_b200_attention_decode_workspace(...) bytes whose first 64 KiB
   (arrival counters) are zero before the first call; every call leaves them
   zero, so one zeroed buffer serves any mix of products and attention. Calls that share a workspace must not overlap
   on the GPU. A bulk copy that does not land within the wait bound ORs
   ACCEL_B200_STATUS_COPY_TIMEOUT into *status (device int; may be NULL). */
ACCEL_B200_API size_t accel_b200_attention_decode_workspace(int32_t batch, int32_t heads, int32_t kv_heads,
                                                            int32_t max_len, int32_t chunk);
ACCEL_B200_API int accel_b200_attention_decode(const float* q, int64_t q_row_stride, const float* k, const float* v,
                                               int64_t kv_row_stride, int64_t kv_head_stride, int64_t kv_seq_stride,
                                               const int32_t* lens, int32_t batch, int32_t heads, int32_t kv_heads,
                                               int32_t head_dim, int32_t max_len, int32_t chunk, float* out,
                                               int64_t out_row_stride, void* workspace, size_t workspace_bytes,
                                               int32_t* status, void* stream);

/* The same decode attention for callers that must not allocate device
   memory: a plugin running inside a host runtime that owns all device memory
   through its own arena (ONNX Runtime, for one), or a serving loop that forbids
   allocation after warm-up, since cudaMalloc and cudaFree synchronize the
   device and stall every stream. No reference counterpart: an addition of
   this backend. The scratch is a fixed 4 MiB array in the library's own
   device memory (accel_b200_attention_decode_noalloc_limit() bytes; each GPU
   that loads the library holds it until the process exits); sizes whose
   workspace would exceed it are rejected with ACCEL_B200_EINVAL. The entry
   point calls no cudaMalloc, cudaFree or allocating library routine. Every
   argument is checked before the array is touched; a rejected call queues
   nothing. The first call on a device (and the first after a device reset,
   which gives the device a new context) looks up the array's device address
   with cudaGetSymbolAddress, so make that first call before any stream
   capture. All calls share the array and each clears the arrival counters it
   needs on its own stream; calls that overlap on the GPU (different streams,
   several threads) race on the array. */
ACCEL_B200_API size_t accel_b200_attention_decode_noalloc_limit(void);
ACCEL_B200_API int accel_b200_attention_decode_noalloc(const float* q, int64_t q_row_stride, const float* k,
                                                       const float* v, int64_t kv_row_stride, int64_t kv_head_stride,
                                                       int64_t kv_seq_stride, const int32_t* lens, int32_t batch,
                                                       int32_t heads, int32_t kv_heads, int32_t head_dim,
                                                       int32_t max_len, int32_t chunk, float* out,
                                                       int64_t out_row_stride, int32_t* status, void* stream);

/* One decode step of a layer's attention, fused (src/llama_model.cc:229-233
   for one new token per sequence): Rope on the query and key heads of row r,
   AppendCache of its key and value at position row_pos[r] of slot row_seq[r]
   (row_seq may be NULL: slot r), and causal attention of the query heads over
   cache rows [0, row_pos[r]] (src/sim_attend.cc:9-46). qkv rows as in
   accel_b200_rope_append; qkv is only read (the rotated queries stay in
   shared memory). head_dim 64; the cache must be head-major (row stride
   64 floats): element (slot s, kv head g, row t, dim d) at s * seq_stride +
   g * head_stride + t * 64 + d, head_stride >= context * 64. Rows with
   row_pos[r] < 0 are skipped (their output is not written). Needs no
   workspace: the context splits merge inside a thread-block cluster. The
   cache rows written are bit-identical to accel_b200_rope_append's; the
   attention output agrees with accel_b200_attention_decode within 1e-4. A
   bulk copy that does not land within the wait bound ORs
   ACCEL_B200_STATUS_COPY_TIMEOUT into *status (device int; may be NULL). */
ACCEL_B200_API int accel_b200_decode_attention(const float* qkv, int64_t qkv_ld, const int32_t* row_seq,
                                               const int32_t* row_pos, int64_t rows, int32_t heads, int32_t kv_heads,
                                               int32_t head_dim, const float* cos_table, const float* sin_table,
                                               int32_t context, float* k_cache, float* v_cache, int64_t seq_stride,
                                               int64_t head_stride, float* out, int64_t out_ld, int32_t* status,
                                               void* stream);

/* Up to four device ranges to bring into L2 (a hint: no completion, no
   effect on results), and launch options of the kernel that takes them. */
typedef struct accel_b200_l2_prefetch {
  const void* ptr[4];
  int64_t bytes[4];
  int32_t count;
  int32_t flags;
} accel_b200_l2_prefetch;

/* accel_b200_decode_attention_prefetch: the cache rows and the row positions
   and slots are read before the kernel waits for the previous kernel of the
   stream (only the q|k|v rows after it). The caller guarantees that no kernel
   still running when this one starts writes them: the previous kernel is a
   product launched with ACCEL_B200_EP_TRIGGER_AFTER_WAIT, a kernel that does
   not launch its dependents early, or none. */
#define ACCEL_B200_ATTN_CACHE_BEFORE_WAIT 1

/* accel_b200_decode_attention that also brings `prefetch`'s ranges into L2
   while it waits for its inputs and streams the cache (the engine passes the
   weights of the layer's next products, which then read them from L2
   instead of HBM). The cache rows are read with an evict-first L2 policy so
   the stream of keys and values does not displace them. Results are those of
   accel_b200_decode_attention. prefetch may be NULL. */
ACCEL_B200_API int accel_b200_decode_attention_prefetch(
    const float* qkv, int64_t qkv_ld, const int32_t* row_seq, const int32_t* row_pos, int64_t rows, int32_t heads,
    int32_t kv_heads, int32_t head_dim, const float* cos_table, const float* sin_table, int32_t context,
    float* k_cache, float* v_cache, int64_t seq_stride, int64_t head_stride, float* out, int64_t out_ld,
    int32_t* status, const accel_b200_l2_prefetch* prefetch, void* stream);

/* SiluMul (src/sim_silu.cc:8-13) over fused rows [gate (inter) | up (inter)]
   of row stride ld into out[r, i] (row stride ldo). */
ACCEL_B200_API int accel_b200_silu_mul_rows(const float* gate_up, int64_t ld, float* out, int64_t ldo, int64_t rows,
                                            int64_t inter, void* stream);

/* Batched SampleToken (src/sim_sample.cc:25-115): row r draws with its own
   device state rng_states[r] and writes chosen[r * chosen_stride +
   chosen_offset]. */
ACCEL_B200_API int accel_b200_sample_rows(const float* logits, int64_t rows, int64_t vocab, int64_t ld, int32_t* chosen,
                                          int64_t chosen_stride, int64_t chosen_offset, float temperature,
                                          uint32_t* rng_states, int32_t top_k, void* stream);

/* One step of Generate's loop (src/llama_model.cc:113-128) for `batch`
   sequences at once. Sequence b (unless done[b]): id = argmax(logits[b])
   (or pre_ids[b] when pre_ids is not NULL); ids[b * ids_stride + step] = id;
   count[b] = step + 1; then id == eos or lens[b] >= context ends it (done[b]
   = 1, row_pos[b] = -1, *finished += 1), else tokens[b] = id, row_pos[b] =
   lens[b], lens[b] += 1. step points to two device ints {step, 0}; the
   launch advances step[0] by one, so it can be replayed from a graph. */
ACCEL_B200_API int accel_b200_greedy_step(const float* logits, const int32_t* pre_ids, int64_t vocab, int64_t ld,
                                          int32_t* ids, int64_t ids_stride, int32_t* count, int32_t* done,
                                          int32_t* tokens, int32_t* row_pos, int32_t* lens, int32_t eos,
                                          int32_t context, int32_t* step, int32_t* finished, int32_t batch,
                                          void* stream);

/* Runs one CTA whose bulk-copy wait can never be satisfied: after the one-
   second wait bound it ORs ACCEL_B200_STATUS_COPY_TIMEOUT into *status and
   returns, leaving the context usable. Exercises the bounded-wait error path
   without a fault. */
ACCEL_B200_API int accel_b200_wait_selftest(int32_t* status, void* stream);

/* dst[r, :] = src[idx[r], :] for r < rows (cols floats per row): the last
   prompt row of each sequence before the final norm (src/llama_model.cc:244). */
ACCEL_B200_API int accel_b200_gather_rows(const float* src, int64_t ld, const int32_t* idx, int64_t rows, int64_t cols,
                                          float* dst, int64_t ldd, void* stream);

/* *out = max over i of |a[i] - b[i]|, NaN differences ignored: the logit
   check of src/llama_model.cc:168-181 done on the device. */
ACCEL_B200_API int accel_b200_max_abs_diff(const float* a, const float* b, int64_t n, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ACCEL_B200_H_ */
