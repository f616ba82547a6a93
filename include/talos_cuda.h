/*
 * talos_cuda.h -- C ABI of the B200 (sm_100a) decode path for Talos.
 *
 * This library replaces the Apple-Metal twin of Talos's CPU forward pass
 * (Tsuskov/talos, Rust). Each entry point names the reference interface it
 * stands in for. The Rust side binds these symbols from a `cuda` cargo feature
 * that mirrors the existing `metal` feature (Cargo.toml:28-31), with one
 * `extern "C"` declaration per entry point below.
 *
 * Conventions
 *  - Every call returns a talos_status; talos_last_error() gives the message of
 *    the last failure on the calling thread.
 *  - Host pointers everywhere unless a name ends in `_dev`; output buffers are
 *    owned by the caller.
 *  - One context drives one GPU. A context is not thread-safe: use it from one
 *    thread at a time (the reference's backend is a thread_local context,
 *    src/math/metal/mod.rs:25-29).
 *  - Calls are synchronous unless documented otherwise (the reference commits
 *    and waits once per token, src/math/metal/mod.rs:511-513).
 *  - Weights are copied to the GPU once, keyed by tensor name
 *    (src/math/metal/mod.rs:37-41,63-72), and repacked there into the
 *    GPU-friendly layouts the kernels read; the GGUF bytes are not kept.
 *  - ggml type tags: F32 = 0, Q4_0 = 2, Q8_0 = 8, Q6_K = 14
 *    (src/gguf/dtype.rs:31-41).
 */
#ifndef TALOS_CUDA_H
#define TALOS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum talos_status {
    TALOS_OK = 0,
    TALOS_ERR_INVALID_ARG = 1, /* bad pointer, size, name, type or shape */
    TALOS_ERR_OOM = 2,         /* device or pinned-host allocation failed */
    TALOS_ERR_CUDA = 3,        /* a CUDA runtime call failed */
    TALOS_ERR_NCCL = 4,        /* an NCCL call failed */
    TALOS_ERR_TIMEOUT = 5,     /* a bounded wait ran out */
    TALOS_ERR_OOB = 6,         /* a device-side bounds check fired */
    TALOS_ERR_STATE = 7,       /* call not valid in the current state (e.g. weights missing) */
    TALOS_ERR_UNSUPPORTED = 8  /* ggml type or shape this build does not handle */
} talos_status;

enum { TALOS_F32 = 0, TALOS_Q4_0 = 2, TALOS_Q8_0 = 8, TALOS_Q6_K = 14 };

/* Model hyper-parameters: the fields of `Config` (src/model/config.rs:14-25) as
 * fixed-width C types (usize -> uint32_t); a binding copies them by name. */
typedef struct talos_cfg {
    uint32_t n_layer;
    uint32_t n_head;
    uint32_t n_head_kv;
    uint32_t n_embd;
    uint32_t n_ff;
    uint32_t context_length;
    uint32_t vocab_size;
    uint32_t rope_dim;
    float rms_eps;
    float rope_freq_base;
} talos_cfg;

typedef struct talos_ctx talos_ctx;
/* A packed weight on the device, for the single-matvec entry points. */
typedef struct talos_weight talos_weight;

/* Message of the last failed call on this thread ("" if none). */
const char* talos_last_error(void);

/* Number of CUDA devices visible (0 when there is no GPU). */
talos_status talos_device_count(int* out);

/* ------------------------------------------------------------ context */

/*
 * Create a decode context on CUDA device `device`. Replaces the lazily built
 * Metal context (src/math/metal/mod.rs:43-61) and `GpuKv::new`
 * (src/math/metal/mod.rs:272-281). Checks n_head_kv > 0 and
 * n_head % n_head_kv == 0 like Model::from_gguf (src/model/llama.rs:43-51).
 * The KV cache holds cfg->context_length positions.
 */
talos_status talos_ctx_create(const talos_cfg* cfg, int device, talos_ctx** out);

/*
 * Tensor-parallel context: rank `tp_rank` of `tp_size` ranks, one process per
 * GPU, joined through the 128-byte NCCL unique id that rank 0 made with
 * talos_nccl_unique_id() and shared out of band. No reference counterpart (the
 * reference is single-device); it follows the same rules as talos_ctx_create.
 */
talos_status talos_ctx_create_tp(const talos_cfg* cfg, int device, int tp_size, int tp_rank,
                                 const uint8_t* nccl_unique_id, talos_ctx** out);
talos_status talos_nccl_unique_id(uint8_t out[128]);

/*
 * Tensor parallel: the ranks of a context wait for each other inside every
 * step, each wait bounded (2 s). When any rank's step returns
 * TALOS_ERR_TIMEOUT (a rank that never launched its step, or one that stopped),
 * the ranks' barrier counters no longer agree: every rank then calls
 * talos_ctx_tp_resync while no rank has a step in flight (between two host-side
 * barriers of the caller), which waits for this rank's stream and clears its
 * counters; the next step on all ranks starts afresh. Until then every batched
 * step of a rank that saw the failure reports it again. On one GPU it only
 * clears the per-token kernel's counters. No reference counterpart.
 */
talos_status talos_ctx_tp_resync(talos_ctx* ctx);

talos_status talos_ctx_destroy(talos_ctx* ctx);

/*
 * Copy one GGUF tensor to the GPU under its GGUF name and repack it for the
 * kernels. Replaces `resident_weight` (src/math/metal/mod.rs:63-72) fed from
 * `QTensor::gpu_parts` (src/model/weights.rs:66-69). `bytes` are the raw
 * GGUF data (`len` bytes) of a row-major [rows, cols] matrix of `ggml_type`;
 * 1-D norm weights pass rows = 1. Names and shapes must be those
 * `Weights::from_gguf` binds (src/model/weights.rs:91-114). Uploading a name
 * again replaces its data. Under tensor parallelism each rank passes the FULL
 * tensor and keeps its own shard.
 */
talos_status talos_weight_upload(talos_ctx* ctx, const char* name, const void* bytes, size_t len,
                                 int ggml_type, size_t rows, size_t cols);

/*
 * How a decode step is launched. TALOS_STEP_FUSED: one persistent kernel per
 * token runs every layer, with grid-wide barriers between the phases and the
 * weight stream running on across them. TALOS_STEP_LAYERED: a graph of about
 * five kernels per layer. TALOS_STEP_AUTO (the default): FUSED when the model
 * fits it (q/k/v of a layer share a ggml type, head_dim <= 128,
 * n_embd <= 8192), else LAYERED. Both give the same results within the parity
 * bars, each bit-identical run to run. No reference counterpart (the Metal path
 * encodes one command buffer per token, src/math/metal/mod.rs:414-513).
 * talos_ctx_step_kernel reports what the next step will run (FUSED or
 * LAYERED); with FUSED requested for a model it cannot run, the next step fails
 * with TALOS_ERR_UNSUPPORTED.
 */
enum { TALOS_STEP_AUTO = 0, TALOS_STEP_FUSED = 1, TALOS_STEP_LAYERED = 2 };
talos_status talos_ctx_set_step_kernel(talos_ctx* ctx, int kind);
talos_status talos_ctx_step_kernel(talos_ctx* ctx, int* kind_out);

/* Bytes of device memory the context holds (weights + KV cache + work areas). */
talos_status talos_ctx_device_bytes(talos_ctx* ctx, size_t* out);

/*
 * The CUDA stream (cudaStream_t, as void*) every call on `ctx` runs on, so a
 * caller can time steps with CUDA events recorded on it. No reference
 * counterpart (the Metal path exposes its command queue only internally,
 * src/math/metal/mod.rs:31-34).
 */
talos_status talos_ctx_stream(talos_ctx* ctx, void** stream_out);

/*
 * Shrink the KV cache to `max_ctx` positions (never above the model's own
 * context_length) and empty it. Model::cap_context (src/model/llama.rs:69-81).
 */
talos_status talos_cap_context(talos_ctx* ctx, size_t max_ctx);

/*
 * KV cache element type: TALOS_KV_F32 (the default; the reference's KvCache
 * holds f32, src/kv_cache.rs:9-10) or TALOS_KV_F16, opt-in: K (after RoPE) and
 * V are rounded to f16 (nearest, ties to even) when appended and widened to f32
 * when read, which halves the cache's memory and its traffic per token at the
 * price of parity with the reference. Setting it reallocates and empties the
 * cache. No reference counterpart (the reference has no KV type choice).
 */
enum { TALOS_KV_F32 = 0, TALOS_KV_F16 = 1 };
talos_status talos_ctx_set_kv_dtype(talos_ctx* ctx, int dtype);
talos_status talos_ctx_kv_dtype(talos_ctx* ctx, int* dtype_out);

/*
 * Start a fresh sequence. Model::reset (src/model/llama.rs:236-238). The
 * device KV cache is indexed by position, so this only forgets the cached
 * length; positions are overwritten as they are decoded.
 */
talos_status talos_kv_reset(talos_ctx* ctx);

/* ------------------------------------------------------------ decode */

/*
 * One decode step for `token` at position `pos`; writes vocab_size logits to
 * `logits_out` (host). Model::forward_gpu (src/model/llama.rs:188-195) ->
 * math::metal::forward (src/math/metal/mod.rs:351-359). Unlike the Metal path
 * the embedding row is looked up on the GPU, so the call takes the token id.
 * Requires 0 <= pos < context length and token < vocab_size. The whole step is
 * one CUDA graph replay.
 */
talos_status talos_forward(talos_ctx* ctx, uint32_t token, size_t pos, float* logits_out);

/*
 * Like talos_forward but returns the final-norm hidden state (n_embd floats).
 * Model::forward_hidden_gpu (src/model/llama.rs:199-206) ->
 * math::metal::forward_hidden (src/math/metal/mod.rs:363-366).
 */
talos_status talos_forward_hidden(talos_ctx* ctx, uint32_t token, size_t pos, float* hidden_out);

/*
 * Greedy decode entirely on the GPU: feeds `token` at `pos`, then the argmax of
 * each step's logits at pos+1, pos+2, ... for `n` steps, and writes the n chosen
 * tokens to `tokens_out` (host). The argmax follows sample::argmax
 * (src/sample.rs:7-14): total order, last maximal index on ties. This is the
 * decode loop of src/main.rs:97-113 / benches/tokps.rs:33-41 with the logits
 * never leaving the GPU.
 */
talos_status talos_generate_greedy(talos_ctx* ctx, uint32_t token, size_t pos, size_t n,
                                   uint32_t* tokens_out);

/*
 * Feed `n` prompt tokens at positions pos0 .. pos0+n-1 (the prefill loop of
 * src/main.rs:88-95) and write the logits after the last one to `last_logits`
 * (host, may be NULL). With an f32 cache and Q4_0 / Q8_0 / Q6_K matrices the
 * prompt goes through the batched step, up to 128 consecutive positions per
 * weight pass on the tensor cores (each position attends to the ones before it,
 * as token-by-token feeding does); otherwise one token per step. Under tensor
 * parallelism every rank makes the call with the same arguments.
 */
talos_status talos_prefill(talos_ctx* ctx, const uint32_t* tokens, size_t n, size_t pos0,
                           float* last_logits);

/*
 * Batched decode: up to TALOS_MAX_BATCH independent sequences per step, each
 * with its own KV cache slot and position; every weight is read once per step
 * for all of them (a tensor-core GEMM). talos_ctx_set_batch reserves
 * `max_seqs` cache slots of the context's current context length each (0 frees
 * them; reserving empties them) for the context's model, which must have
 * Q4_0 / Q8_0 / Q6_K matrices and head_dim <= 128 (TALOS_ERR_UNSUPPORTED
 * otherwise). Under tensor parallelism every rank makes each of these calls
 * with the same arguments (talos_ctx_set_batch maps the ranks' exchange areas;
 * each step's row-parallel products are summed across ranks inside the step)
 * and every rank gets all vocab_size logits. talos_forward_batch runs one step
 * for sequences 0 .. n-1 (n <= max_seqs): sequence i feeds tokens[i] at
 * position pos[i] into slot i and gets its vocab_size logits at
 * logits_out + i * vocab_size (host). Each sequence computes what
 * Model::forward (src/model/llama.rs:85-183) computes for it alone; this is the
 * batched decode of the multi-prompt workload, which the reference runs as
 * separate token-by-token loops (src/main.rs:88-113). talos_cap_context and
 * talos_ctx_set_kv_dtype release the slots (reserve them again afterwards). No
 * reference counterpart as an entry point.
 */
#define TALOS_MAX_BATCH 64
talos_status talos_ctx_set_batch(talos_ctx* ctx, int max_seqs);
talos_status talos_forward_batch(talos_ctx* ctx, const uint32_t* tokens, const size_t* pos, int n,
                                 float* logits_out);

/*
 * The prompt of one sequence of the batch: feeds tokens[0..n) at positions
 * pos0 .. pos0+n-1 into cache slot `slot` (< max_seqs of talos_ctx_set_batch),
 * up to 128 positions per weight pass on the tensor cores, each position
 * attending to the ones before it (the prefill loop of src/main.rs:88-95 for
 * one of the multi-prompt workload's sequences); the logits after the last one
 * go to `last_logits` (host, may be NULL). Other slots are untouched.
 */
talos_status talos_prefill_slot(talos_ctx* ctx, int slot, const uint32_t* tokens, size_t n, size_t pos0,
                                float* last_logits);

/*
 * Batched greedy decode on the GPU: sequence i (slot i, i < n) feeds tokens[i]
 * at pos[i], then the argmax of its logits at pos[i]+1, ... for `steps` steps;
 * the chosen tokens go to tokens_out[k * n + i] (host, step k). The argmax is
 * sample::argmax (src/sample.rs:7-14: total order, last maximal index), taken
 * per sequence on the device, so no logits leave the GPU: talos_generate_greedy
 * for a batch, i.e. the decode loops of src/main.rs:97-113 run together.
 */
talos_status talos_generate_batch_greedy(talos_ctx* ctx, const uint32_t* tokens, const size_t* pos, int n,
                                         size_t steps, uint32_t* tokens_out);

/*
 * Teacher-forced perplexity of tokens[0..n) (n >= 2): eval::perplexity
 * (src/eval.rs:35-52). The tokens are scored in chunks of the context length,
 * each from an empty KV cache; at each position the negative log-likelihood of
 * the next token (token_nll, src/eval.rs:18-23: log-sum-exp in f64) is added on
 * the GPU, so no logits leave the device (up to 128 positions per weight
 * pass where talos_prefill takes its batched steps). Writes exp(mean NLL) to *ppl_out and,
 * if not NULL, the NLL sum and the number of scored positions. Leaves the KV
 * cache holding the last chunk.
 */
talos_status talos_perplexity(talos_ctx* ctx, const uint32_t* tokens, size_t n, float* ppl_out,
                              double* nll_sum_out, size_t* scored_out);

/*
 * Run one decode step (as talos_forward, logits stay on the GPU) and add the
 * device time in milliseconds of each part of it into kernel_ms[kind] and the
 * number of such parts into launches[kind] (either may be NULL), kind =
 * talos_kernel_kind. LAYERED steps launch their kernels one by one with CUDA
 * events between them. FUSED steps run the per-token kernel once with phase
 * time stamps (the device's global timer, read by CTA 0 as it passes each
 * grid barrier); the last phase also carries the launch and drain time. For
 * benchmarks. No reference counterpart.
 */
enum talos_kernel_kind {
    TALOS_K_EMBED = 0,  /* token embedding row dequant */
    TALOS_K_QKV = 1,    /* RMSNorm + q/k/v matvec + RoPE + KV append */
    TALOS_K_ATTN = 2,   /* split-position GQA attention */
    TALOS_K_OPROJ = 3,  /* attn_output matvec + residual */
    TALOS_K_GATEUP = 4, /* RMSNorm + gate/up matvec + SwiGLU */
    TALOS_K_DOWN = 5,   /* ffn_down matvec + residual */
    TALOS_K_OUTPUT = 6, /* final RMSNorm + output matvec (+ argmax) */
    TALOS_K_COUNT = 7
};
talos_status talos_profile_step(talos_ctx* ctx, uint32_t token, size_t pos, double* kernel_ms,
                                uint32_t* launches);

/*
 * Run one decode step of the per-token kernel with profiling stamps and copy
 * them to `out` (host): for phase p (in step order: per layer q/k/v,
 * attention, o-proj, gate/up, down; then the output phase) and CTA c, four
 * device global-timer values in ns at out[(p * n_cta + c) * 4 + k]: k = 0 the
 * CTA entered the phase, 1 its inputs were staged, 2 its compute finished,
 * 3 it arrived at the phase's barrier (0 where a stamp does not apply). `cap`
 * is the length of `out` in elements; *n_phase and *n_cta receive the
 * dimensions. TALOS_ERR_UNSUPPORTED when steps run the layered graph. For
 * benchmarks; no reference counterpart.
 */
talos_status talos_profile_phases(talos_ctx* ctx, uint32_t token, size_t pos, uint64_t* out, size_t cap,
                                  int* n_phase, int* n_cta);

/* ------------------------------------------------------------ kernels */

/*
 * Dequantize n_elems values of `ggml_type` from raw GGUF `bytes` (host) into
 * `out` (host) on the GPU, bit-exact with GgmlType::dequantize
 * (src/gguf/dtype.rs:64-121). Test hook for the bit-exact contract.
 */
talos_status talos_dequant(int ggml_type, const void* bytes, size_t n_elems, float* out);

/*
 * Greedy choice over n logits (host) on the current CUDA device:
 * sample::argmax (src/sample.rs:7-14), the maximum under f32::total_cmp
 * (-NaN < -inf < ... < -0.0 < +0.0 < ... < +inf < +NaN) and the LAST maximal
 * index on ties. The decode step's own argmax (talos_generate_greedy, the
 * logits epilogue) uses the same key. n must be 1 .. 2^32-1 (the reference
 * panics on empty logits).
 */
talos_status talos_argmax(const float* logits, size_t n, uint32_t* index_out);

/*
 * One fused dequant-matvec y = W x on device `device`, with W uploaded for this
 * call only. math::metal::matvec_f32 / matvec_quant
 * (src/math/metal/mod.rs:195-225). x: cols floats, y: rows floats (host).
 */
talos_status talos_matvec(int device, int ggml_type, const void* bytes, size_t len, size_t rows,
                          size_t cols, const float* x, float* y);

/*
 * Matvec against a weight kept on the GPU under `name` in `ctx`: uploaded on
 * first use and reused while the byte length stays the same, even if the bytes
 * differ. math::metal::matvec_f32_resident / matvec_quant_resident
 * (src/math/metal/mod.rs:227-253), with the cache rule of
 * src/math/metal/mod.rs:63-72.
 */
talos_status talos_matvec_resident(talos_ctx* ctx, const char* name, int ggml_type,
                                   const void* bytes, size_t len, size_t rows, size_t cols,
                                   const float* x, float* y);

/*
 * Device-level matvec for benchmarks: pack a weight onto device `device` once,
 * then run y_dev = W x_dev on a CUDA stream (cudaStream_t passed as void*,
 * NULL = legacy default stream) without synchronizing. x_dev/y_dev are device
 * pointers of cols / rows floats. No reference counterpart; it exposes the
 * kernel that QTensor::matvec (src/model/weights.rs:47-55) becomes.
 */
talos_status talos_weight_create(int device, int ggml_type, const void* bytes, size_t len,
                                 size_t rows, size_t cols, talos_weight** out);
talos_status talos_weight_destroy(talos_weight* w);
talos_status talos_weight_packed_bytes(const talos_weight* w, size_t* out);
talos_status talos_matvec_dev(const talos_weight* w, const float* x_dev, float* y_dev,
                              void* stream);

/*
 * talos_matvec_dev without allocating: a split-K variant (each CTA takes one
 * 16-row tile and one slice of the columns; the slices' partial sums meet in a
 * fixed-size scratch array that the library holds as static device memory, and
 * the last slice of a tile adds them in slice order). For callers that must not
 * allocate device memory during decoding: a runtime that reserves the device's
 * memory up front, or a loop that cannot take the device-wide synchronisation
 * of cudaMalloc / cudaFree. Limits: at most 65,536 rows (the scratch is 2 MB of
 * partial sums + 16 KB of arrival counters) and columns whose staged input
 * fits shared memory (about 47,000); larger weights fail with
 * TALOS_ERR_UNSUPPORTED. The first call on a device resolves the scratch's
 * address (cudaGetSymbolAddress); make it before any stream capture. Calls
 * share the scratch: two calls in flight at once (other streams, other
 * threads) race, so serialise them. Results agree with talos_matvec_dev to
 * rounding (another summation order) and are identical call to call. Every
 * device wait is bounded (2 s): a 16-row tile any of whose K slices gave up
 * waiting for its weight copy comes out as 16 NaN rows (the call itself still
 * returns TALOS_OK, since it does not synchronise). No reference counterpart.
 */
talos_status talos_matvec_dev_noalloc(const talos_weight* w, const float* x_dev, float* y_dev, void* stream);

/*
 * Benchmark helper: capture `reps` back-to-back talos_matvec_dev launches that
 * cycle through the n weights ws[0..n-1] (same shape) into one CUDA graph, replay
 * it once to warm up and once timed with CUDA events, and write the average
 * device microseconds per launch to *us_per_launch. Host launch overhead is not
 * in the number. No reference counterpart.
 */
talos_status talos_matvec_bench(const talos_weight* const* ws, int n, const float* x_dev,
                                float* y_dev, int reps, float* us_per_launch);

#ifdef __cplusplus
}
#endif
#endif
