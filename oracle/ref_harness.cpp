// ref_harness.cpp -- TEST INFRASTRUCTURE: drives the reference's own C-ABI
// sampler (tg_generate, wasm/src/model.cpp:473-522, declared at
// wasm/src/model.h:39-43) on logits chosen by the test.
//
// The reference sampler has no "sample these logits" entry point: it runs its
// model forward and samples the last row.  A model with n_layers = 0 and
// d_model = 1 whose final LayerNorm has gain 0 and bias 1 emits
// logits[v] = 1 * tok_emb[v] exactly for every position, so writing the wanted
// logits into tok_emb (through the reference's own tg_import_state,
// wasm/src/model.cpp:541-553; parameter order tok_emb, pos_emb, ln_f_g, ln_f_b
// from collect_params, wasm/src/model.cpp:126-135) makes tg_generate sample
// exactly those logits at every step.  Ids come back as bytes, so vocab <= 256.
//
// Built from the reference sources where they lie by oracle/Makefile into
// oracle/_ref/libtgref.so.  Nothing here is product code.
#include <cstring>
#include <random>
#include <vector>

#include "model.h"

extern "C" int tgref_generate_fixed_logits(const float* logits, int vocab, float temperature,
                                           int top_k, unsigned int seed, int n_steps,
                                           unsigned char* out) {
  if (vocab <= 0 || vocab > 256) return -1;
  TgModel m = tg_model_create(vocab, 4, 0, 1, 1, 1, seed);
  if (!m) return -2;
  const int nbytes = tg_state_bytes(m);
  std::vector<unsigned char> st(static_cast<size_t>(nbytes));
  tg_export_state(m, st.data());
  // layout: int32 step, then per param (w, m, v) each size*4 bytes.
  size_t off = 4;
  auto param = [&](size_t n) { float* w = reinterpret_cast<float*>(st.data() + off); off += 3 * n * 4; return w; };
  float* tok = param(static_cast<size_t>(vocab));  // [V, C=1]
  param(4);                                         // pos_emb [ctx=4, C=1]
  float* lng = param(1);
  float* lnb = param(1);
  std::memcpy(tok, logits, sizeof(float) * static_cast<size_t>(vocab));
  lng[0] = 0.0f;
  lnb[0] = 1.0f;
  tg_import_state(m, st.data());
  const unsigned char prompt = 0;
  const int n = tg_generate(m, &prompt, 1, out, n_steps, temperature, top_k, seed);
  tg_model_free(m);
  return n;
}

// The canonical uniforms in [0,1) the reference draw consumes, one per step:
// std::uniform_real_distribution<float>(0, sum) is a + (b - a) * canonical on
// a std::mt19937 seeded like tg_generate (wasm/src/model.cpp:477).
extern "C" void tgref_canonical_uniforms(unsigned int seed, int n, float* out) {
  std::mt19937 gen(seed);
  for (int i = 0; i < n; ++i) out[i] = std::generate_canonical<float, 24>(gen);
}
