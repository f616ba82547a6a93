// kernels.cuh -- launch interface of the Talos sm_100a kernels (kernels.cu).
#pragma once

#include "common.cuh"

namespace talos {

// ---------------------------------------------------------------- packing

// Bytes of device memory a packed weight needs, split per array.
struct PackSizes {
    size_t b0, b1, b2, b3;
    int rows_pad, nk;
};
bool pack_sizes(int type, int rows, int cols, PackSizes* out);
// Repack raw GGUF bytes (device) of a [rows, cols] weight into `w` (arrays
// already allocated with pack_sizes).
cudaError_t launch_pack(const uint8_t* raw, const PackedW& w, cudaStream_t s);

// Bit-exact GgmlType::dequantize of n elements (device in, device out).
cudaError_t launch_dequant(int type, const uint8_t* raw, size_t n, float* out, cudaStream_t s);

// ---------------------------------------------------------------- matvec

// EPI_PEER (per-token kernel, tensor parallel): the tile's rows are this rank's
// partial sums of a row-parallel matvec; they go to every rank's receive slot.
enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_LOGITS = 4, EPI_PEER = 5 };

// A run of 16-row tiles inside one matvec launch.
//  pair == 0: tile t covers rows 16t .. 16t+15 of A (B is ignored).
//  pair == 1: tile t covers rows 8t .. 8t+7 of A and of B (SwiGLU gate/up).
struct Seg {
    PackedW A, B;
    int pair;
    int ntiles;
    int role;      // EPI_QKV: 0 = q, 1 = k, 2 = v
    float* out;    // destination vector
    int out_rows;  // logical rows written
};

struct MatvecArgs {
    Seg seg[3];
    int nseg;
    int ntiles;
    int K;             // logical input length
    const float* x;    // input vector (device)
    const float* norm_w;  // if set: x is RMS-normalised with this weight first
    float eps;
    int epi;
    StepParams* step;
    void* kcache;      // EPI_QKV: this layer's K/V cache, [ctx][kv_dim] f32 (or f16)
    void* vcache;
    int kv_f16;        // the cache holds f16 (round to nearest even) instead of f32
    int kv_dim;
    int hd;
    const float2* rope_cs;  // [ctx][hd/2] (cos, sin)
};

// Tiles in a segment for a weight of `rows` rows.
inline int seg_tiles(int rows, int pair) { return pair ? (rows + 7) / 8 : (rows + 15) / 16; }
// pdl: launch with programmatic stream serialization (the kernel streams its
// weights before waiting on the previous kernel of the stream).
cudaError_t launch_matvec(const MatvecArgs& a, int type, int max_ctas, cudaStream_t s, bool pdl);
size_t matvec_smem_bytes(int type, int K);
cudaError_t matvec_configure();  // opt-in shared memory limits, once per process
int matvec_ctas_per_sm(int type, int K);
int matvec_max_k(int type);      // largest input length the staged activation fits

// Split-K matvec whose partial sums live in a static device array (no allocation):
// the array's address and limits, and the launch (nslice K slices per 16-row tile).
cudaError_t noalloc_scratch(float** part, unsigned** cnt, int* max_tiles, int* max_slices);
size_t noalloc_smem_bytes(int type, int K);
cudaError_t launch_matvec_noalloc(const PackedW& w, const float* x, float* y, int nslice, float* part,
                                  unsigned* cnt, cudaStream_t s);

// ---------------------------------------------------------------- batched steps
//
// A batched step runs up to MB_SEQ token columns through every weight at once:
// the independent sequences of a batched decode step, or consecutive prompt
// positions of one sequence (prefill). Its matrix products are the tcgen05 GEMM
// of gemm.cu: k_xfmt_g formats each matrix input (RMSNorm, per-column power-of-
// two scale, f16 hi / lo planes), k_gemm multiplies the packed weights into it.

constexpr int MB_SEQ = 128;
constexpr int TALOS_MAX_TP = 8;  // tensor-parallel ranks (one per GPU)

struct BatchParams {
    int n;                     // active token columns (1 .. MB_SEQ)
    uint32_t token[MB_SEQ];
    uint32_t pos[MB_SEQ];
    uint32_t slot[MB_SEQ];     // cache slot of each column (steps on the sequences' slots)
    uint32_t ngen[MB_SEQ];     // batched greedy: tokens chosen so far per column
    uint32_t error;            // device-side error bits (1: token out of range, 2: a bounded wait expired)
    uint32_t tpstep;           // tensor parallel: earlier batched steps of the context (k_tp_join_b targets)
};

// Batched epilogues: store / add rows; RoPE of q rows (stored to y); RoPE of k
// rows and v rows, appended to the column's cache slot at its position;
// EPI_B_PEER (tensor parallel): the rows go to every rank r at
// GemmArgs::peer[r] + t * ldy + row (this rank's receive slot of a row-parallel
// product, or its vocabulary range of the gathered logits).
enum { EPI_B_STORE = 0, EPI_B_ADD = 1, EPI_B_SWIGLU = 2, EPI_B_ROPE = 3, EPI_B_KCACHE = 4, EPI_B_VCACHE = 5,
       EPI_B_PEER = 6 };

// One weight of a GEMM launch: tiles of 128 rows of A. map_lrec / map_sc are
// A's two tensor maps (CUtensorMap, gemm_weight_maps) when wmap is set.
struct GemmSeg {
    alignas(64) uint8_t map_lrec[128];
    alignas(64) uint8_t map_sc[128];
    PackedW A;
    int wmap;
    int ntiles;
    float* y;      // [MB_SEQ][ldy] outputs (EPI_B_KCACHE / VCACHE: unused)
    int ldy;
    int rows;      // logical output rows
    int epi;
};
struct GemmArgs {
    GemmSeg seg[3];  // same type and input; row tiles numbered across segments
    int nseg;
    int nrt;         // row tiles over all segments
    int S;           // K slices per output tile (split-K; 1 = none)
    int K, KP;       // input length; KP = K rounded up to 128
    const float* xs;       // per-column scale 2^e_t of the formatted input (k_xfmt_g)
    const float2* rope_cs; // RoPE (cos, sin) [ctx][hd/2]
    int hd, kv_dim;
    float* kc;             // this layer's caches: column t's rows at kc + t * seq_stride
    float* vc;
    size_t seq_stride;
    const BatchParams* bp;
    float* ws;             // split-K partial tiles [tiles][S][NT][128]
    unsigned* cnt;         // split-K arrival counters [tiles][4], zero between launches
    // tensor parallel (EPI_B_PEER): each rank's destination (CUDA IPC mappings;
    // this rank's own memory at [rank]), and the local counter every CTA adds 1
    // to at exit, after its peer stores (k_tp_join_b reads it)
    float* peer[TALOS_MAX_TP];
    int npeer;
    unsigned long long* lar;
};
// Format columns 0 .. ncols-1 of `x` ([n][ldx] f32; columns n .. ncols-1
// become zeros) for a GEMM whose weights have K inputs: f16 hi / lo planes
// [2][Tp][ldp] and xs[] (ncols <= Tp).
cudaError_t launch_xfmt_g(const float* x, int ldx, int K, int KP, int ldp, int Tp, int ncols, const float* norm_w,
                          float eps, const BatchParams* bp, void* planes, float* xs, cudaStream_t s);
// The tensor map (CUtensorMap, gemm_map_bytes() bytes) the GEMM's activation
// producer reads `planes` through with token tiles of nt columns.
cudaError_t gemm_tensor_map(void* planes, int ldp, int Tp, int nt, void* map_out);
size_t gemm_map_bytes();
// The two tensor maps (gemm_map_bytes() each) of a packed Q4_0 / Q8_0 / Q6_K
// weight through which the GEMM copies its lane records and scales.
cudaError_t gemm_weight_maps(const PackedW& w, void* lrec_map, void* sc_map);
// nt: token columns per tile (32, 64 or 128); grid: CTAs (one per SM at most).
// pdl: programmatic dependent launch (the GEMM starts its weight copies while the
// previous kernel of the stream finishes; it reads that kernel's output only after it).
cudaError_t launch_gemm(const void* map, const GemmArgs& a, int type, int nt, int grid, cudaStream_t s,
                        bool pdl = false);
cudaError_t gemm_configure();

// Tensor-parallel join after an EPI_B_PEER GEMM of `grid` CTAs (instance `inst`
// of the step): signal every rank, wait (bounded) for all ranks' rows, and when
// rx is set add the ranks' partial rows (rx: [tp][MB_SEQ][E], rank order) to
// the residual x ([MB_SEQ][E]). abort: this rank's abort word, which a rank that
// gave up a wait sets on every rank so that all of them report the failure.
struct TpJoin {
    unsigned long long* lar;                  // local: CTAs of the GEMM that have exited
    unsigned lar_target;                      // the GEMM's grid
    unsigned long long* rarr;                 // own arrival counters [instances]
    unsigned long long* prarr[TALOS_MAX_TP];  // every rank's arrival counters
    unsigned* abort;                          // own abort word
    unsigned* pabort[TALOS_MAX_TP];           // every rank's abort word
    int inst, tp;
    const float* rx;                          // receive slots of this instance, or null
    float* x;
    int E;
};
cudaError_t launch_tp_join_b(const TpJoin& j, BatchParams* bp, int grid, cudaStream_t s);

// x[s] = dequant(token_embd row of token[s]) (src/model/weights.rs:57-62)
cudaError_t launch_embed_b(const uint8_t* embd_raw, int type, int cols, int vocab, const BatchParams* bp, float* x,
                           int ldx, cudaStream_t s);
// h[s][i] = silu(g[s][i]) * u[s][i] for the live columns (src/math/ops.rs:28-37)
// Batched greedy: per live column s, the argmax of its logits row (total order,
// last maximal index: sample::argmax) becomes its next token at pos + 1 and is
// appended to gen[s * cap + ngen[s]]; then tpstep advances by one.
cudaError_t launch_greedy_advance_b(const float* logits, int V, BatchParams* bp, uint32_t* gen, int cap,
                                    cudaStream_t s);
cudaError_t launch_swiglu_b(const float* g, const float* u, float* h, int ld, int n_ff, const BatchParams* bp,
                            cudaStream_t s);
// GQA attention per (head, sequence) over positions 0 .. pos[s] (src/model/llama.rs:135-155)
cudaError_t launch_attention_b(const float* q, int ldq, const float* kc, const float* vc, size_t seq_stride,
                               int kv_dim, int n_head, int n_kv, int hd, float* out, int ldo, const BatchParams* bp,
                               cudaStream_t s);

// ---------------------------------------------------------------- attention

struct AttnArgs {
    const float* q;     // [n_head * hd], RoPE applied
    const void* kc;     // [ctx][kv_dim] this layer, f32 (or f16 when kv_f16)
    const void* vc;
    int kv_f16;
    float* out;         // [n_head * hd]
    StepParams* step;
    int n_head, n_kv, hd, kv_dim;
    float scale;
};
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);
cudaError_t attention_configure();
size_t attention_smem_bytes(int hd, int group);

// ---------------------------------------------------------------- small kernels

// x = dequant(token_embd row step->token); also clears step->argmax_key.
cudaError_t launch_embed(const uint8_t* embd_raw, int type, int cols, int vocab, StepParams* step,
                         float* x, cudaStream_t s, bool pdl);
// out = rmsnorm(x, w)
cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, float* out,
                           cudaStream_t s, bool pdl);
// acc[0] += the negative log-likelihood logits[0..n) give `target` (f64 log-sum-exp),
// acc[1] += 1 (src/eval.rs:18-23).
cudaError_t launch_token_nll(const float* logits, int n, uint32_t target, double* acc, cudaStream_t s);
// *key = the largest argmax_key of v[0..n) (sample::argmax, src/sample.rs:7-14);
// the index is its low 32 bits.
cudaError_t launch_argmax(const float* v, size_t n, unsigned long long* key, cudaStream_t s);
// Greedy feedback: token = argmax, append it to gen[], pos += 1.
cudaError_t launch_greedy_advance(StepParams* step, uint32_t* gen, int gen_cap, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------- per-token kernel
//
// k_token runs a whole decode step in one launch as a list of phases separated
// by grid barriers (matvec.cu).

enum PhaseKind : int { PH_MATVEC = 0, PH_ATTN = 1, PH_HIDDEN = 2 };

struct TokenPhase {
    int kind;
    int type;       // PH_MATVEC: ggml type of every segment
    int embed_in;   // PH_MATVEC: the input is the token's embedding row (first phase)
    int prof_kind;  // talos_kernel_kind the phase is reported under
    // tensor parallel (TokenArgs::tp > 1)
    int xsum;       // input = xbuf[xsrc] + sum over ranks of rx slot xslot; CTA 0 stores it to xbuf[xdst]
    int xsrc, xdst, xslot;
    int rx_slot;    // EPI_PEER: receive slot written
    int xrank;      // arrivals at this phase's barrier come from every rank
    int att_merge;  // the input is the attention output, merged from TokenArgs::att_part
    MatvecArgs mv;  // PH_MATVEC
    AttnArgs at;    // PH_ATTN
};

struct TokenArgs {
    const TokenPhase* ph;       // device array of nph phases
    int nph;
    unsigned long long* bars;   // [nph] arrival counters, never reset
    unsigned long long* epoch;  // number of completed launches
    StepParams* step;
    const uint8_t* embd;        // raw GGUF token_embd rows
    int embd_type, vocab;
    float* x;                   // residual stream [E]
    int E;
    float* hidden;              // PH_HIDDEN output [E]
    const float* out_norm;
    float eps;
    float* att_part;            // [n_head][nsplit][hd + 4] split-softmax partials {m, l, -, -, o}
    int nsplit;                 // most attention splits per kv head (<= 8)
    int nst;                    // ring stages
    int prefetch;               // chunks of a phase streamed before its input is staged
    int union_bytes;            // staged input / attention scratch bytes
    unsigned long long* stamps; // optional [nph][grid][4] global-timer stamps (ns): phase
                                // entered, inputs staged, compute done, barrier arrival
    // tensor parallel: tp ranks, one per GPU; peer pointers are CUDA IPC mappings
    int tp, rank;
    unsigned long long* rbars;                // [nph] rank arrivals at cross-rank phases
    unsigned long long* prbars[TALOS_MAX_TP]; // each rank's rbars (own: rbars)
    float* prx[TALOS_MAX_TP];                 // each rank's receive slots [2][tp][E]
    float* plogits[TALOS_MAX_TP];             // each rank's full logits [vocab]
    unsigned long long* pkey[TALOS_MAX_TP];   // each rank's StepParams::argmax_key
    int vocab_off;                            // first vocab row of this rank's output shard
    float* xbuf[2];                           // residual stream, double-buffered (tp > 1)
};

// Whether attention items are single query heads (else kv heads with their group).
bool token_attn_per_head();
// Staged-input elements the k_token scratch region must hold for input length K.
int token_stage_elems(int type, int K);
// Scratch bytes attention needs for `group` heads of `hd` dims.
int token_attn_bytes(int group, int hd);
size_t token_smem_bytes(int nst, int union_bytes);
// Ring stages that fit next to `union_bytes` of scratch (0 if none fit).
int token_max_stages(int union_bytes);
cudaError_t token_configure();
// One CTA per SM; `cooperative` asks the launch to guarantee co-residency.
cudaError_t launch_token(const TokenArgs& a, int grid, cudaStream_t s, bool cooperative);

}  // namespace talos
