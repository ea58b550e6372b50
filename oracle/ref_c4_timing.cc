// The AccelEP reference Llama with one added entry point, for timing its
// decode at deep contexts.
//
// TEST INFRASTRUCTURE ONLY: bench.py's reference arm and its cpu_baseline
// leg time this library; the product never links or calls it.
// oracle/Makefile compiles the reference's own model (src/llama_model.cc of
// the AccelEP checkout, included by path below, unmodified) into
// oracle/_ref/libaccel_ref_c4.so together with the reference's other
// objects. Every accel_llama_* call is the reference's own code.
//
// The added entry point, ref_llama_fill_context, places a model at context
// length `rows` without running the forward passes that would normally fill
// it: it writes pseudo-random rows into every layer's key and value cache and
// sets the model's fill counter. A following accel_llama_forward_ids of one
// id then runs the reference's decode step at position `rows`, attention over
// rows + 1 cache rows included, exactly as it would deep into a generation.
// The cache values only feed that timing (scalar fp32 arithmetic does not
// depend on them, and they are never denormal); the logits are not used.

#include "src/llama_model.cc"

#include <cstdint>

extern "C" __attribute__((visibility("default"))) int ref_llama_fill_context(AccelLlama* handle, int32_t rows,
                                                                             uint32_t seed) {
  LlamaModel* model = reinterpret_cast<LlamaModel*>(handle);
  if (model == nullptr || rows < 0 || rows > model->config.context) {
    Fail("invalid fill");
    return 1;
  }
  std::lock_guard<std::mutex> lock(model->mu);
  const size_t row_floats = static_cast<size_t>(model->config.kv_heads) * static_cast<size_t>(model->head_dim);
  uint32_t state = seed == 0 ? 0x9e3779b9u : seed;
  for (size_t layer = 0; layer < model->k_cache.size(); ++layer) {
    for (accel::OwnedBuffer* cache : {&model->k_cache[layer], &model->v_cache[layer]}) {
      float* data = static_cast<float*>(cache->buffer.data);
      for (size_t i = 0; i < static_cast<size_t>(rows) * row_floats; ++i) {
        state ^= state << 13;
        state ^= state >> 17;
        state ^= state << 5;
        // Uniform in [-1, 1) with 2^-23 steps: normal floats only.
        data[i] = static_cast<float>(static_cast<int32_t>(state >> 8) - (1 << 23)) * (1.0f / (1 << 23));
      }
    }
  }
  model->filled = rows;
  Clear();
  return 0;
}
