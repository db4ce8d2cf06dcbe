// C ABI of axropus_deploy_b200 (libkorith_b200.so).
//
// Two surfaces, with the reference's names and signatures so that C callers of the
// reference link against this library unchanged:
//   * korith_init / korith_tokenize / korith_step / korith_shutdown -- one sequence,
//     greedy decoding (reference: korith_c_api/korith.h:9-24, a llama.cpp wrapper);
//   * korith_engine_* -- the engine ABI of the control plane (reference:
//     platform/engine/cpp/korith_engine.h:12-43, whose reference implementation returns
//     fake timings). Here every call runs this framework's model, paged KV cache and
//     sm_100a kernels.
// model_path names a model preset ("llama3-8b", "tiny128", "preset:layers") or a
// directory with a config.json {"preset": ..., "layers": ...}; weights are random-
// initialised (no checkpoints on these boxes). Text is tokenised byte-wise.
// The library embeds the Python runtime of the framework: loaded into a Python process
// it uses that interpreter; loaded by a C program it starts one. Calls are serialised.
#pragma once

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

bool korith_init(const char* model_path, int n_ctx);
// Prefill of the byte-tokenised prompt; number of prompt tokens, or -1.
int korith_tokenize(const char* prompt);
// One greedy token (evaluated into the context); -1 when the context is full or on error.
int korith_step(void);
void korith_shutdown(void);

struct korith_engine_params {
  int32_t n_ctx;
  int32_t n_batch;
  int32_t n_gpu;
  const char* model_path;
};

struct korith_engine_metrics {
  double prefill_ms;
  double decode_ms;
  double total_ms;
  double restore_ms;
  double verify_ms;
  double draft_ms;
  int32_t tokens_out;
  int32_t accepted_tokens;
  int32_t rejected_tokens;
};

bool korith_engine_init_model(const struct korith_engine_params* params);
bool korith_engine_prefill(const int32_t* tokens, int32_t n_tokens);
bool korith_engine_decode_step(int32_t* token_out);
bool korith_engine_get_logits(float* out_logits, int32_t n_vocab);
// AMFK blob (header + per-layer K/V pages) written into the cache as the first pages.
bool korith_engine_apply_kv_replay(const uint8_t* blob, size_t n_bytes);
// AMFK file of the sequence's full pages (+ "<path>.tok" with the token ids).
bool korith_engine_export_snapshot(const char* path);
bool korith_engine_import_snapshot(const char* path);
// Greedy verification of proposed tokens; the accepted prefix is appended.
bool korith_engine_verify_tokens(const int32_t* proposed_tokens, int32_t n_tokens, int32_t* accepted_prefix);
void korith_engine_get_metrics(struct korith_engine_metrics* out_metrics);
void korith_engine_shutdown(void);
bool korith_engine_cuda_probe(void);
// Last error message of this library ("" when none).
const char* korith_last_error(void);

#ifdef __cplusplus
}  // extern "C"
#endif
