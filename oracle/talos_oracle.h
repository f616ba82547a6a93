/*
 * talos_oracle.h -- CPU restatement of the Talos (Tsuskov/talos, Rust) decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * decode path in talos_b200/. It is linked or loaded only by tests/,
 * __graft_entry__.smoke() and the cpu_baseline / --impl reference legs of
 * bench.py. The product never calls it.
 *
 * Every function names the reference file:line it restates (paths inside the
 * Tsuskov/talos source tree). The reference is Rust; no Rust toolchain exists in
 * this image, so it cannot be built and run here. The restatement is pinned by
 * the reference's own known-answer tests (ops, matvec, dequant round trip, GGUF
 * parse, GQA == replicated MHA), restated in tests/test_oracle_kat.py.
 *
 * Known bit-level freedom (no reference test pins it): the 8-lane dot of
 * src/math/matmul.rs:15-30 uses the `wide` 0.7 crate. Here the lanes combine as
 * ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)) and `mul_add` is a separate multiply and
 * add (what `wide` does on an x86_64 target without the `fma` feature). Both
 * only move the last bits; the reference's own tolerance for it is 1e-5
 * (src/math/matmul.rs:66-76).
 */
#ifndef TALOS_ORACLE_H
#define TALOS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type tags (src/gguf/dtype.rs:31-41). */
enum { OR_F32 = 0, OR_Q4_0 = 2, OR_Q8_0 = 8, OR_Q6_K = 14 };

typedef struct oracle_config {
    uint32_t n_layer, n_head, n_head_kv, n_embd, n_ff, context_length, vocab_size, rope_dim;
    float rms_eps, rope_freq_base;
} oracle_config;

const char* oracle_last_error(void);
void oracle_set_threads(int n);
int oracle_get_threads(void);

/* f16 <-> f32 (the `half` crate's exact widening; round-to-nearest-even narrowing). */
float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);

int oracle_block_elems(int type);
int oracle_block_bytes(int type);
/* src/gguf/dtype.rs:64-121 */
int oracle_dequant(int type, const uint8_t* raw, size_t n_elems, float* out);

/* src/math/matmul.rs:15-47 */
float oracle_dot(const float* a, const float* b, size_t n);
void oracle_matvec_f32(const float* w, const float* x, float* out, size_t rows, size_t cols);
/* src/math/quant.rs:18-51 */
int oracle_matvec_quant(const uint8_t* bytes, int type, const float* x, float* out, size_t rows,
                        size_t cols);

/* src/math/ops.rs:5-61 */
void oracle_rmsnorm(const float* x, const float* w, float eps, float* out, size_t n);
void oracle_softmax(float* x, size_t n);
float oracle_silu(float x);
void oracle_swiglu(const float* gate, const float* up, float* out, size_t n);
void oracle_rope(float* v, size_t pos, size_t n_head, size_t head_dim, float freq_base);
/* src/sample.rs:7-14 */
uint32_t oracle_argmax(const float* logits, size_t n);

/* Quantizers: src/math/metal/mod.rs:551-574 (Q8_0, Q4_0); Q6_K from the k-quant layout. */
void oracle_quantize_q8_0(const float* x, size_t n, uint8_t* out);
void oracle_quantize_q4_0(const float* x, size_t n, uint8_t* out);
void oracle_quantize_q6_k(const float* x, size_t n, uint8_t* out);

/* GGUF v3 reader: src/gguf/reader.rs:173-351 */
typedef struct oracle_gguf oracle_gguf;
int oracle_gguf_open(const char* path, oracle_gguf** out);
int oracle_gguf_from_bytes(const uint8_t* bytes, size_t len, oracle_gguf** out); /* copies */
void oracle_gguf_free(oracle_gguf* g);
int oracle_gguf_get_u32(const oracle_gguf* g, const char* key, uint32_t* out);
int oracle_gguf_get_f32(const oracle_gguf* g, const char* key, float* out);
int oracle_gguf_get_bool(const oracle_gguf* g, const char* key, int* out);
int oracle_gguf_get_str(const oracle_gguf* g, const char* key, const char** out, size_t* len);
int oracle_gguf_arr_str_len(const oracle_gguf* g, const char* key, size_t* n);
int oracle_gguf_arr_str_item(const oracle_gguf* g, const char* key, size_t i, const char** out,
                             size_t* len);
int oracle_gguf_arr_i32(const oracle_gguf* g, const char* key, const int32_t** out, size_t* n);
size_t oracle_gguf_n_tensors(const oracle_gguf* g);
const char* oracle_gguf_tensor_name(const oracle_gguf* g, size_t i);
int oracle_gguf_tensor_meta(const oracle_gguf* g, size_t i, uint32_t* n_dims, uint64_t dims[4],
                            int* type, uint64_t* offset);
int oracle_gguf_tensor_f32(const oracle_gguf* g, const char* name, const float** out, size_t* n);
int oracle_gguf_tensor_raw(const oracle_gguf* g, const char* name, const uint8_t** out,
                           size_t* len, int* type);

/* Model: src/model/llama.rs:20-238, config.rs:40-67, weights.rs:91-114, kv_cache.rs */
typedef struct oracle_model oracle_model;
int oracle_model_open(const char* path, oracle_model** out);
int oracle_model_from_bytes(const uint8_t* bytes, size_t len, oracle_model** out);
void oracle_model_free(oracle_model* m);
int oracle_model_config(const oracle_model* m, oracle_config* out);
void oracle_model_cap_context(oracle_model* m, size_t max_ctx);
void oracle_model_reset(oracle_model* m);
/* The CUDA path's opt-in f16 KV cache (not in the reference): K/V rounded to f16 when appended. */
void oracle_model_set_kv_f16(oracle_model* m, int on);
int oracle_forward(oracle_model* m, uint32_t token, size_t pos, float* logits);
int oracle_forward_hidden(oracle_model* m, uint32_t token, size_t pos, float* hidden);

#ifdef __cplusplus
}
#endif
#endif
