// runtime.cu -- the decode context behind include/talos_cuda.h.
//
// Host side of the B200 twin of Model::forward_gpu (Tsuskov/talos
// src/model/llama.rs:188-206 -> src/math/metal/mod.rs:351-520):
//  * weights are copied once, keyed by GGUF tensor name, and repacked on the
//    GPU (src/math/metal/mod.rs:63-72 keeps them resident the same way);
//  * the KV cache is a position-indexed device array per layer
//    (src/math/metal/mod.rs:391-396,443-454);
//  * activations live in one arena allocated once, not per token
//    (src/math/metal/mod.rs:398-412 allocates 14 buffers every token);
//  * one token = one CUDA graph replay; the graph reads token and position from
//    device memory, so the same graph serves every step. The graph holds either
//    the per-token kernel k_token (one launch for the whole step, the default)
//    or the layered sequence of ~5 kernels per layer.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <dlfcn.h>
#include <nccl.h>

#include "../../include/talos_cuda.h"
#include "kernels.cuh"

using namespace talos;

// ------------------------------------------------------------------ NCCL, opened on first use
//
// NCCL only bootstraps tensor-parallel contexts, so it is opened with dlopen
// when the first one is made instead of being linked: a process that also loads
// PyTorch gets one NCCL (an already loaded libnccl.so.2 is reused), and the
// library still loads where NCCL is absent.

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    const char* (*GetErrorString)(ncclResult_t);
    bool ok;
};

static const NcclApi& nccl() {
    static NcclApi api = [] {
        NcclApi a{};
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        a.CommInitRank = (decltype(a.CommInitRank))dlsym(h, "ncclCommInitRank");
        a.AllGather = (decltype(a.AllGather))dlsym(h, "ncclAllGather");
        a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
        a.ok = a.GetUniqueId && a.CommInitRank && a.AllGather && a.CommDestroy && a.GetErrorString;
        return a;
    }();
    return api;
}

// ------------------------------------------------------------------ errors

static thread_local std::string g_last_error;

static talos_status set_err(talos_status st, const char* fmt, ...) {
    char buf[768];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

#define CK(call)                                                                                 \
    do {                                                                                         \
        cudaError_t e_ = (call);                                                                 \
        if (e_ != cudaSuccess)                                                                   \
            return set_err(e_ == cudaErrorMemoryAllocation ? TALOS_ERR_OOM : TALOS_ERR_CUDA,     \
                           "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__,     \
                           __LINE__);                                                            \
    } while (0)

#define TRY(call)                              \
    do {                                       \
        talos_status s_ = (call);              \
        if (s_ != TALOS_OK) return s_;         \
    } while (0)

extern "C" const char* talos_last_error(void) { return g_last_error.c_str(); }

extern "C" talos_status talos_device_count(int* out) {
    if (!out) return set_err(TALOS_ERR_INVALID_ARG, "out is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    *out = n;
    return TALOS_OK;
}

static int block_elems(int t) { return t == GT_F32 ? 1 : t == GT_Q6_K ? 256 : (t == GT_Q4_0 || t == GT_Q8_0) ? 32 : 0; }
static int block_bytes(int t) {
    return t == GT_F32 ? 4 : t == GT_Q6_K ? 210 : t == GT_Q4_0 ? 18 : t == GT_Q8_0 ? 34 : 0;
}

// Raw GGUF byte length of a [rows, cols] tensor, 0 if the shape is invalid for the type.
static size_t raw_len(int type, size_t rows, size_t cols) {
    int be = block_elems(type);
    if (!be || cols % be) return 0;
    return rows * (cols / be) * block_bytes(type);
}

// ------------------------------------------------------------------ device tensors

struct DevTensor {
    int type = -1;
    size_t rows = 0, cols = 0;
    void* mem = nullptr;  // one range holding every array
    size_t bytes = 0;
    size_t cap = 0;       // bytes of the range (>= bytes)
    bool in_arena = false;  // carved from a WeightArena block, not freed alone
    PackedW w{};          // packed matrix view (kind == PACKED)
    enum Kind { PACKED, FLOATS, RAW } kind = PACKED;
    // the tensor maps through which the batched GEMM copies a packed quant
    // matrix (gemm_weight_maps); gmap false: it copies row group by row group
    bool gmap = false;
    alignas(64) uint8_t gmaps[2][128];
    void release() {
        if (mem && !in_arena) cudaFree(mem);
        mem = nullptr;
        bytes = cap = 0;
        in_arena = false;
    }
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Device memory for a context's weights: a few large blocks handed out by a
// bump pointer. cudaMalloc costs milliseconds per call and cudaFree more (it
// waits for the device), so a separate allocation per tensor made a model
// upload allocation-bound. Blocks grow geometrically from 16 MB to 256 MB (a
// tensor larger than that gets a block of its own), so a tiny model holds
// little and a 7B model about 20 blocks. A re-uploaded tensor reuses its range
// when the new one fits; otherwise the old range stays unused until the
// context is destroyed.
struct WeightArena {
    static constexpr size_t kMinBlock = (size_t)16 << 20, kMaxBlock = (size_t)256 << 20;
    struct Block {
        uint8_t* base;
        size_t size, used;
    };
    std::vector<Block> blocks;
    size_t total = 0;
    talos_status alloc(size_t n, void** out) {
        n = align256(n);
        for (Block& b : blocks)
            if (b.size - b.used >= n) {
                *out = b.base + b.used;
                b.used += n;
                return TALOS_OK;
            }
        size_t want = std::max(n, std::min(kMaxBlock, std::max(kMinBlock, total)));
        void* p = nullptr;
        CK(cudaMalloc(&p, want));
        blocks.push_back({(uint8_t*)p, want, n});
        total += want;
        *out = p;
        return TALOS_OK;
    }
    // a range for `t` of `n` bytes: its own when large enough, else a new one
    talos_status place(DevTensor* t, size_t n, void** out) {
        if (t->in_arena && t->mem && t->cap >= n) {
            *out = t->mem;
            return TALOS_OK;
        }
        return alloc(n, out);
    }
    void release() {
        for (Block& b : blocks) cudaFree(b.base);
        blocks.clear();
        total = 0;
    }
};

// Fill a packed matrix from raw GGUF bytes already on the device, in a range
// of `arena` (or its own allocation when `arena` is null).
static talos_status pack_from_device(int type, size_t rows, size_t cols, const uint8_t* raw_dev,
                                     DevTensor* t, cudaStream_t s, WeightArena* arena) {
    PackSizes ps;
    if (rows == 0 || cols == 0 || rows > (1u << 30) || cols > (1u << 30) ||
        !pack_sizes(type, (int)rows, (int)cols, &ps))
        return set_err(TALOS_ERR_UNSUPPORTED, "cannot pack a [%zu, %zu] tensor of ggml type %d", rows,
                       cols, type);
    size_t o1 = align256(ps.b0), o2 = o1 + align256(ps.b1), o3 = o2 + align256(ps.b2);
    size_t total = o3 + align256(ps.b3);
    void* mem = nullptr;
    if (arena)
        TRY(arena->place(t, total, &mem));
    else
        CK(cudaMalloc(&mem, total));
    PackedW w{};
    w.type = type;
    w.rows = (int)rows;
    w.cols = (int)cols;
    w.rows_pad = ps.rows_pad;
    w.nk = ps.nk;
    w.p0 = mem;
    w.p1 = ps.b1 ? (uint8_t*)mem + o1 : nullptr;
    w.p2 = ps.b2 ? (uint8_t*)mem + o2 : nullptr;
    w.p3 = ps.b3 ? (uint8_t*)mem + o3 : nullptr;
    cudaError_t e = launch_pack(raw_dev, w, s);
    if (e != cudaSuccess) {
        if (!arena) cudaFree(mem);
        return set_err(TALOS_ERR_CUDA, "pack kernel: %s", cudaGetErrorString(e));
    }
    const size_t cap = arena ? (mem == t->mem ? t->cap : align256(total)) : total;
    if (mem != t->mem) t->release();
    t->type = type;
    t->rows = rows;
    t->cols = cols;
    t->mem = mem;
    t->bytes = total;
    t->cap = cap;
    t->in_arena = arena != nullptr;
    t->w = w;
    t->kind = DevTensor::PACKED;
    t->gmap = type != GT_F32 && gemm_map_bytes() <= sizeof t->gmaps[0] &&
              gemm_weight_maps(w, t->gmaps[0], t->gmaps[1]) == cudaSuccess;
    return TALOS_OK;
}

// Upload staging. Host bytes are copied into a ring of pinned chunks by a few
// host threads, and each chunk goes to the device with cudaMemcpyAsync while
// the next one is being filled, so the host copy, the PCIe transfer and the
// repack kernels of earlier tensors overlap. A call returns once the caller's
// bytes sit in pinned memory (the caller may free them); the device side
// finishes on the stream, and `finish` waits for it. Raw GGUF bytes of a
// packed matrix land in `dev` first, where the pack kernel reads them.
struct Staging {
    static constexpr int kChunks = 4;
    static constexpr size_t kChunk = (size_t)32 << 20;
    uint8_t* dev = nullptr;
    size_t cap = 0;
    uint8_t* host[kChunks] = {};
    cudaEvent_t freed[kChunks] = {};
    int next = 0;
    talos_status reserve(size_t n) {
        if (n <= cap) return TALOS_OK;
        if (dev) cudaFree(dev);  // waits for the kernels still reading it
        dev = nullptr;
        cap = 0;
        CK(cudaMalloc(&dev, n));
        cap = n;
        return TALOS_OK;
    }
    talos_status ring() {
        if (host[0]) return TALOS_OK;
        for (int i = 0; i < kChunks; ++i) {
            CK(cudaHostAlloc((void**)&host[i], kChunk, cudaHostAllocPortable));
            CK(cudaEventCreateWithFlags(&freed[i], cudaEventDisableTiming));
        }
        return TALOS_OK;
    }
    // memcpy split over up to 8 threads (page faults of a freshly mapped file
    // are taken in parallel too)
    static void host_copy(uint8_t* dst, const uint8_t* src, size_t n) {
        const size_t per = (size_t)4 << 20;
        unsigned hw = std::thread::hardware_concurrency();
        size_t nt = std::min<size_t>({(n + per - 1) / per, hw ? hw : 1, 8});
        if (nt <= 1) {
            memcpy(dst, src, n);
            return;
        }
        const size_t part = (n / nt + 4095) & ~(size_t)4095;
        std::vector<std::thread> th;
        for (size_t i = 1; i < nt; ++i) {
            const size_t o = i * part;
            if (o >= n) break;
            th.emplace_back([=] { memcpy(dst + o, src + o, std::min(part, n - o)); });
        }
        memcpy(dst, src, std::min(part, n));
        for (auto& t : th) t.join();
    }
    // host -> device through the pinned ring, asynchronous on `s`
    talos_status h2d(void* dst, const void* src, size_t n, cudaStream_t s) {
        TRY(ring());
        for (size_t o = 0; o < n; o += kChunk) {
            const size_t k = std::min(kChunk, n - o);
            const int i = next;
            next = (next + 1) % kChunks;
            CK(cudaEventSynchronize(freed[i]));  // the chunk's previous transfer is done
            host_copy(host[i], (const uint8_t*)src + o, k);
            CK(cudaMemcpyAsync((uint8_t*)dst + o, host[i], k, cudaMemcpyHostToDevice, s));
            CK(cudaEventRecord(freed[i], s));
        }
        return TALOS_OK;
    }
    talos_status finish(cudaStream_t s) {
        CK(cudaStreamSynchronize(s));
        return TALOS_OK;
    }
    void release() {
        for (int i = 0; i < kChunks; ++i) {
            if (freed[i]) {
                cudaEventSynchronize(freed[i]);
                cudaEventDestroy(freed[i]);
            }
            if (host[i]) cudaFreeHost(host[i]);
            host[i] = nullptr;
            freed[i] = nullptr;
        }
        next = 0;
        if (dev) cudaFree(dev);
        dev = nullptr;
        cap = 0;
    }
};

// Raw GGUF bytes -> packed device matrix. Asynchronous on `s`: the pack kernel
// and the transfer it reads may still run when this returns.
static talos_status upload_packed(int type, const void* bytes, size_t len, size_t rows, size_t cols,
                                  DevTensor* t, Staging* st, cudaStream_t s, WeightArena* arena = nullptr) {
    TRY(st->reserve(len));
    TRY(st->h2d(st->dev, bytes, len, s));
    TRY(pack_from_device(type, rows, cols, st->dev, t, s, arena));
    return TALOS_OK;
}

static int g_sms[64];
static std::once_flag g_cfg_once;
static cudaError_t g_cfg_err = cudaSuccess;

static talos_status device_setup(int device) {
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return set_err(TALOS_ERR_INVALID_ARG, "device %d of %d", device, n);
    CK(cudaSetDevice(device));
    std::call_once(g_cfg_once, [] {
        g_cfg_err = matvec_configure();
        if (g_cfg_err == cudaSuccess) g_cfg_err = attention_configure();
        if (g_cfg_err == cudaSuccess) g_cfg_err = token_configure();
        if (g_cfg_err == cudaSuccess) g_cfg_err = gemm_configure();
    });
    if (g_cfg_err != cudaSuccess) return set_err(TALOS_ERR_CUDA, "matvec_configure: %s", cudaGetErrorString(g_cfg_err));
    if (device < 64 && g_sms[device] == 0) {
        int sms = 0;
        CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        g_sms[device] = sms;
    }
    return TALOS_OK;
}

static int sm_count_dev(int device) {
    if (device >= 0 && device < 64 && g_sms[device]) return g_sms[device];
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) return 148;
    return sms;
}

static int max_ctas(int device, int type, int K) {
    int sms = (device >= 0 && device < 64 && g_sms[device]) ? g_sms[device] : 148;
    return sms * matvec_ctas_per_sm(type, K);
}

// ------------------------------------------------------------------ context

struct LayerW {
    DevTensor* attn_norm;
    DevTensor *q, *k, *v, *o, *ffn_norm, *gate, *up, *down;
};

enum GraphMode { GM_LOGITS = 0, GM_HIDDEN = 1, GM_GREEDY = 2, GM_COUNT = 3 };

struct talos_ctx {
    talos_cfg cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    int hd = 0, kv_dim = 0, group = 0;
    // tensor parallelism: this rank's share of heads, kv heads, ff rows and vocab
    // (all equal to the full sizes when tp == 1)
    int tp = 1, rank = 0;
    int nh_l = 0, nkv_l = 0, q_rows = 0, kv_l = 0, ff_l = 0, v_l = 0, v_off = 0;
    ncclComm_t comm = nullptr;
    void* shared = nullptr;  // tp > 1: IPC-exported {bars, StepParams, rx slots, logits}
    size_t shared_bytes = 0, shared_bars_bytes = 0;
    void* peer_base[TALOS_MAX_TP] = {};
    float* xbuf[2] = {nullptr, nullptr};
    size_t kv_ctx = 0;  // positions the KV cache holds

    WeightArena weights;                                  // device memory of `w`
    std::unordered_map<std::string, DevTensor> w;         // model weights by GGUF name
    std::unordered_map<std::string, DevTensor> resident;  // talos_matvec_resident cache
    Staging staging;

    // activation arena
    void* arena = nullptr;
    size_t arena_bytes = 0;
    float *x = nullptr, *q = nullptr, *att = nullptr, *ff = nullptr, *logits = nullptr, *hidden = nullptr;
    double* nll_acc = nullptr;  // talos_perplexity: [NLL sum, positions scored]
    StepParams* step = nullptr;
    uint32_t* gen = nullptr;
    // KV + RoPE table
    void* kcache = nullptr;  // [n_layer][kv_ctx][kv_l], f32 or (kv_f16) f16
    void* vcache = nullptr;
    int kv_f16 = 0;
    float2* rope_cs = nullptr;
    size_t kv_bytes = 0;

    // pinned host staging
    float* h_out = nullptr;
    StepParams* h_step = nullptr;
    uint32_t* h_gen = nullptr;

    cudaGraphExec_t graph[GM_COUNT] = {nullptr, nullptr, nullptr};
    bool weights_dirty = true;

    // per-token kernel (k_token)
    int step_pref = TALOS_STEP_AUTO;  // talos_ctx_set_step_kernel
    bool fused = false;               // the current graphs run k_token
    std::string fused_why;            // why k_token cannot run this model ("" = it can)
    bool coop = true;                 // capture k_token as a cooperative launch
    void* sync_mem = nullptr;         // barrier counters, epoch, attention partials
    size_t sync_bytes = 0;
    unsigned long long* bars = nullptr;
    unsigned long long* rbars = nullptr;  // tensor parallel: rank arrivals (shared area)
    unsigned long long* epoch = nullptr;
    unsigned long long* stamps = nullptr;
    float* att_part = nullptr;
    int nsplit = 0, nph_max = 0;
    TokenPhase* d_phases[GM_COUNT] = {nullptr, nullptr, nullptr};
    int nph[GM_COUNT] = {0, 0, 0};
    int tk_nst = 0, tk_union = 0;
    std::vector<unsigned long long>* last_stamps = nullptr;  // talos_profile_phases
    // talos_profile_step: events recorded after each launch, tagged by kernel kind
    std::vector<std::pair<cudaEvent_t, int>>* prof = nullptr;
    std::vector<LayerW> layers;

    // batched steps (talos_forward_batch, talos_prefill, talos_perplexity): one
    // allocation for the parameters, the [MB_SEQ][..] activations, the GEMM's
    // formatted input and split-K workspace, and the sequences' cache slots
    int bmax = 0;              // sequences with cache slots (talos_ctx_set_batch)
    void* bmem = nullptr;
    size_t bbytes = 0;
    BatchParams* bp = nullptr;
    BatchParams* h_bp = nullptr;  // pinned
    float *bx = nullptr, *bq = nullptr, *batt = nullptr;
    float *bg = nullptr, *bu = nullptr, *bh = nullptr, *blog = nullptr;
    void* bplanes = nullptr;   // [2][MB_SEQ][bldp] f16: the GEMM input's hi / lo planes
    float* bxs = nullptr;      // [MB_SEQ] per-column scales of the formatted input
    int bldp = 0;
    float* bws = nullptr;      // split-K partial tiles
    unsigned* bcnt = nullptr;  // split-K arrival counters (zero between launches)
    float *bkc = nullptr, *bvc = nullptr;  // [bmax][n_layer][kv_ctx][kv_dim]
    size_t bseq_stride = 0;                // floats per sequence in bkc / bvc
    float* h_blog = nullptr;               // pinned [TALOS_MAX_BATCH][V]
    alignas(64) uint8_t bmaps[3][128];     // tensor maps of bplanes for 32 / 64 / 128-column tiles
    cudaGraphExec_t bgraph[5][3] = {};     // [BatchMode][token-tile size]
    uint32_t* bgen = nullptr;              // batched greedy: [MB_SEQ][kv_ctx] chosen tokens
    int bgen_cap = 0;
    // tensor parallel: the batched steps' IPC-exported area {arrival counters
    // [2 n_layer + 1], abort word, receive slots [2][tp][MB_SEQ][E], gathered
    // logits [MB_SEQ][V]}, every rank's mapping of it, and the local count of
    // exited GEMM CTAs (k_tp_join_b)
    void* bsh = nullptr;
    void* bsh_peer[TALOS_MAX_TP] = {};
    size_t bsh_sync_bytes = 0, bsh_o_abort = 0, bsh_o_rx = 0, bsh_o_log = 0;
    unsigned long long* blar = nullptr;
    uint32_t btpstep = 0;                  // batched steps run (every rank runs the same ones)

    void drop_batch_graphs() {
        for (auto& row : bgraph)
            for (auto& g : row)
                if (g) {
                    cudaGraphExecDestroy(g);
                    g = nullptr;
                }
    }
    void drop_graphs() {
        for (auto& g : graph)
            if (g) {
                cudaGraphExecDestroy(g);
                g = nullptr;
            }
        drop_batch_graphs();
        for (auto& p : d_phases)
            if (p) {
                cudaFree(p);
                p = nullptr;
            }
    }
};

static std::string lname(uint32_t l, const char* s) { return "blk." + std::to_string(l) + "." + s; }

// Expected (rows, cols) of a model tensor by name; false if the name is not part
// of the model (src/model/weights.rs:91-114).
static bool expected_shape(const talos_ctx* c, const std::string& name, size_t* rows, size_t* cols,
                           bool* is_norm) {
    const size_t E = c->cfg.n_embd, F = c->cfg.n_ff, V = c->cfg.vocab_size, KV = (size_t)c->kv_dim;
    *is_norm = false;
    if (name == "token_embd.weight" || name == "output.weight") {
        *rows = V;
        *cols = E;
        return true;
    }
    if (name == "output_norm.weight") {
        *rows = 1;
        *cols = E;
        *is_norm = true;
        return true;
    }
    if (name.compare(0, 4, "blk.") != 0) return false;
    size_t dot = name.find('.', 4);
    if (dot == std::string::npos) return false;
    std::string idx = name.substr(4, dot - 4);
    if (idx.empty() || idx.size() > 9 || idx.find_first_not_of("0123456789") != std::string::npos) return false;
    unsigned long l = strtoul(idx.c_str(), nullptr, 10);
    if (l >= c->cfg.n_layer || std::to_string(l) != idx) return false;
    std::string rest = name.substr(dot + 1);
    if (rest == "attn_norm.weight" || rest == "ffn_norm.weight") {
        *rows = 1;
        *cols = E;
        *is_norm = true;
    } else if (rest == "attn_q.weight" || rest == "attn_output.weight") {
        *rows = E;
        *cols = E;
    } else if (rest == "attn_k.weight" || rest == "attn_v.weight") {
        *rows = KV;
        *cols = E;
    } else if (rest == "ffn_gate.weight" || rest == "ffn_up.weight") {
        *rows = F;
        *cols = E;
    } else if (rest == "ffn_down.weight") {
        *rows = E;
        *cols = F;
    } else {
        return false;
    }
    return true;
}

static size_t kv_elem(const talos_ctx* c) { return c->kv_f16 ? sizeof(__half) : sizeof(float); }

static talos_status batch_free(talos_ctx* c);

// (Re)allocates the cache for c->kv_ctx positions. The batched step's buffers
// are sized by the cache, so they are released too (talos_ctx_set_batch again).
static talos_status alloc_kv(talos_ctx* c) {
    if (c->bmem) TRY(batch_free(c));
    if (c->kcache) cudaFree(c->kcache);
    if (c->vcache) cudaFree(c->vcache);
    if (c->rope_cs) cudaFree(c->rope_cs);
    c->kcache = c->vcache = nullptr;
    c->rope_cs = nullptr;
    size_t per = (size_t)c->cfg.n_layer * c->kv_ctx * c->kv_l * kv_elem(c);
    CK(cudaMalloc(&c->kcache, per ? per : 4));
    CK(cudaMalloc(&c->vcache, per ? per : 4));
    CK(cudaMemsetAsync(c->kcache, 0, per ? per : 4, c->stream));
    CK(cudaMemsetAsync(c->vcache, 0, per ? per : 4, c->stream));
    // RoPE table: theta = pos * base^(-2i/hd) in f32 with the C library's powf /
    // sinf / cosf, the functions Rust's f32::powf / sin_cos call
    // (src/math/ops.rs:53-54).
    size_t half = (size_t)c->hd / 2;
    std::vector<float2> cs(c->kv_ctx * (half ? half : 1));
    for (size_t p = 0; p < c->kv_ctx; ++p)
        for (size_t i = 0; i < half; ++i) {
            float theta = (float)p * powf(c->cfg.rope_freq_base, -2.0f * (float)i / (float)c->hd);
            cs[p * half + i] = make_float2(cosf(theta), sinf(theta));
        }
    CK(cudaMalloc(&c->rope_cs, cs.size() * sizeof(float2)));
    CK(cudaMemcpyAsync(c->rope_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    c->kv_bytes = 2 * per + cs.size() * sizeof(float2);
    if (c->gen) {
        cudaFree(c->gen);
        c->gen = nullptr;
    }
    CK(cudaMalloc(&c->gen, (c->kv_ctx + 1) * sizeof(uint32_t)));
    if (c->h_gen) cudaFreeHost(c->h_gen);
    c->h_gen = nullptr;
    CK(cudaMallocHost(&c->h_gen, (c->kv_ctx + 1) * sizeof(uint32_t)));
    c->drop_graphs();
    return TALOS_OK;
}

static talos_status alloc_arena(talos_ctx* c) {
    const size_t E = c->cfg.n_embd, F = c->cfg.n_ff, V = c->cfg.vocab_size;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    size_t o_x = take(E * 4), o_q = take(E * 4 + 64), o_att = take(E * 4), o_ff = take(F * 4),
           o_log = take(V * 4), o_hid = take(E * 4), o_step = take(sizeof(StepParams)), o_xb0 = take(E * 4),
           o_xb1 = take(E * 4), o_nll = take(2 * sizeof(double));
    CK(cudaMalloc(&c->arena, off));
    CK(cudaMemsetAsync(c->arena, 0, off, c->stream));
    c->arena_bytes = off;
    uint8_t* b = (uint8_t*)c->arena;
    c->x = (float*)(b + o_x);
    c->q = (float*)(b + o_q);
    c->att = (float*)(b + o_att);
    c->ff = (float*)(b + o_ff);
    c->logits = (float*)(b + o_log);
    c->hidden = (float*)(b + o_hid);
    c->step = (StepParams*)(b + o_step);
    c->xbuf[0] = (float*)(b + o_xb0);
    c->xbuf[1] = (float*)(b + o_xb1);
    c->nll_acc = (double*)(b + o_nll);
    CK(cudaMallocHost(&c->h_out, (V > E ? V : E) * sizeof(float)));
    CK(cudaMallocHost(&c->h_step, sizeof(StepParams)));
    CK(cudaStreamSynchronize(c->stream));
    return TALOS_OK;
}

// Grid-barrier counters, launch epoch, phase stamps and attention partials of
// k_token, zeroed.
static talos_status alloc_sync(talos_ctx* c) {
    const int sms = (c->device < 64 && g_sms[c->device]) ? g_sms[c->device] : 148;
    // attention: (kv head, position split) items; 8 splits keep ~64 CTAs busy on
    // the 7B shape and the o-proj staging's merge short
    c->nsplit = std::max(1, std::min(8, sms / (token_attn_per_head() ? c->nh_l : c->nkv_l)));
    c->nph_max = (int)c->cfg.n_layer * 5 + 1;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    const size_t o_bars = take((size_t)c->nph_max * 8), o_epoch = take(8),
                 o_stamps = take((size_t)c->nph_max * sms * 4 * 8),
                 o_part = take((size_t)c->nh_l * c->nsplit * (c->hd + 4) * 4);
    CK(cudaMalloc(&c->sync_mem, off));
    c->sync_bytes = off;
    uint8_t* b = (uint8_t*)c->sync_mem;
    c->bars = (unsigned long long*)(b + o_bars);
    c->epoch = (unsigned long long*)(b + o_epoch);
    c->stamps = (unsigned long long*)(b + o_stamps);
    c->att_part = (float*)(b + o_part);
    CK(cudaMemsetAsync(c->sync_mem, 0, off, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return TALOS_OK;
}

// After a failed step the barrier counters may be part-way through a launch:
// start them again from zero (no kernel of this context is running).
static void reset_sync(talos_ctx* c) {
    if (c->sync_mem) {
        cudaMemsetAsync(c->sync_mem, 0, c->sync_bytes, c->stream);
        if (c->shared) cudaMemsetAsync(c->shared, 0, c->shared_bars_bytes, c->stream);
        cudaStreamSynchronize(c->stream);
    }
}

// Export `mem` (a cudaMalloc base) by CUDA IPC and map every rank's export
// into peers[] (peers[rank] = mem): one NCCL all-gather of the handles, so every
// rank makes this call at the same point. With check_gpus, ranks sharing a GPU
// are refused (their kernels wait on each other and must run concurrently).
static talos_status ipc_exchange(talos_ctx* c, void* mem, void** peers, bool check_gpus) {
    struct Xch {
        cudaIpcMemHandle_t h;
        int pci_domain, pci_bus, pci_dev, pad;
    };
    Xch me{};
    CK(cudaIpcGetMemHandle(&me.h, mem));
    CK(cudaDeviceGetAttribute(&me.pci_domain, cudaDevAttrPciDomainId, c->device));
    CK(cudaDeviceGetAttribute(&me.pci_bus, cudaDevAttrPciBusId, c->device));
    CK(cudaDeviceGetAttribute(&me.pci_dev, cudaDevAttrPciDeviceId, c->device));
    void* d = nullptr;
    CK(cudaMalloc(&d, sizeof(Xch) * (c->tp + 1)));
    CK(cudaMemcpy(d, &me, sizeof me, cudaMemcpyHostToDevice));
    ncclResult_t nr = nccl().AllGather(d, (uint8_t*)d + sizeof(Xch), sizeof(Xch), ncclUint8, c->comm, c->stream);
    cudaError_t e = cudaStreamSynchronize(c->stream);
    std::vector<Xch> all(c->tp);
    if (nr == ncclSuccess && e == cudaSuccess)
        e = cudaMemcpy(all.data(), (uint8_t*)d + sizeof(Xch), sizeof(Xch) * c->tp, cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (nr != ncclSuccess)
        return set_err(TALOS_ERR_NCCL, "all-gather of IPC handles: %s", nccl().GetErrorString(nr));
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "all-gather of IPC handles: %s", cudaGetErrorString(e));
    if (check_gpus)
        for (int r = 0; r < c->tp; ++r)
            for (int q = 0; q < r; ++q)
                if (all[r].pci_domain == all[q].pci_domain && all[r].pci_bus == all[q].pci_bus &&
                    all[r].pci_dev == all[q].pci_dev)
                    return set_err(TALOS_ERR_UNSUPPORTED, "ranks %d and %d share one GPU (one rank per GPU)", q, r);
    for (int r = 0; r < c->tp; ++r) {
        if (r == c->rank) {
            peers[r] = mem;
            continue;
        }
        CK(cudaIpcOpenMemHandle(&peers[r], all[r].h, cudaIpcMemLazyEnablePeerAccess));
    }
    return TALOS_OK;
}

// Tensor parallel: the area other ranks write into (barrier counters, step
// parameters with the argmax key, all-reduce receive slots [2][tp][E], full
// logits), exported by CUDA IPC and mapped by every rank. The handles and the
// GPUs' PCI ids travel over one NCCL all-gather.
static talos_status alloc_shared(talos_ctx* c) {
    const size_t E = c->cfg.n_embd, V = c->cfg.vocab_size;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    const size_t o_bars = take((size_t)c->nph_max * 8), o_rbars = take((size_t)c->nph_max * 8);
    c->shared_bars_bytes = off;
    const size_t o_step = take(sizeof(StepParams)), o_rx = take(2 * (size_t)c->tp * E * 4), o_log = take(V * 4);
    CK(cudaMalloc(&c->shared, off));
    c->shared_bytes = off;
    CK(cudaMemset(c->shared, 0, off));
    uint8_t* b = (uint8_t*)c->shared;
    c->bars = (unsigned long long*)(b + o_bars);
    c->rbars = (unsigned long long*)(b + o_rbars);
    c->step = (StepParams*)(b + o_step);
    c->logits = (float*)(b + o_log);
    (void)o_rx;

    return ipc_exchange(c, c->shared, c->peer_base, true);
}

static talos_status ctx_create(const talos_cfg* cfg, int device, int tp, int rank, const uint8_t* id,
                               talos_ctx** out) {
    if (!cfg || !out) return set_err(TALOS_ERR_INVALID_ARG, "cfg/out is NULL");
    *out = nullptr;
    if (cfg->n_head_kv == 0 || cfg->n_head == 0 || cfg->n_head % cfg->n_head_kv)
        return set_err(TALOS_ERR_INVALID_ARG, "head_count %u must be a positive multiple of head_count_kv %u",
                       cfg->n_head, cfg->n_head_kv);
    if (cfg->n_layer == 0 || cfg->n_embd == 0 || cfg->n_ff == 0 || cfg->vocab_size == 0 ||
        cfg->context_length == 0)
        return set_err(TALOS_ERR_INVALID_ARG, "zero-sized model dimension");
    if (cfg->n_embd % cfg->n_head)
        return set_err(TALOS_ERR_UNSUPPORTED, "n_embd %u not a multiple of n_head %u", cfg->n_embd, cfg->n_head);
    // Every matvec stages its whole input vector in shared memory (4 B/element).
    int kmax = matvec_max_k(GT_Q8_0);
    for (int t : {(int)GT_F32, (int)GT_Q4_0, (int)GT_Q6_K})
        if (matvec_max_k(t) < kmax) kmax = matvec_max_k(t);
    if ((int)cfg->n_embd > kmax || (int)cfg->n_ff > kmax)
        return set_err(TALOS_ERR_UNSUPPORTED, "n_embd %u / n_ff %u above the staged input limit (%d)",
                       cfg->n_embd, cfg->n_ff, kmax);
    uint32_t hd = cfg->n_embd / cfg->n_head;
    const uint32_t grp = cfg->n_head / cfg->n_head_kv;
    if (hd % 4 || hd > 256 || grp > 8 || grp * hd / 4 > 256)
        return set_err(TALOS_ERR_UNSUPPORTED,
                       "head_dim %u / group %u outside this build (head_dim a multiple of 4, <= 256; "
                       "group <= 8; group * head_dim <= 1024)", hd, grp);
    if (tp != 1) {
        if (tp != 2 && tp != 4 && tp != 8) return set_err(TALOS_ERR_INVALID_ARG, "tp_size %d (1, 2, 4 or 8)", tp);
        if (rank < 0 || rank >= tp) return set_err(TALOS_ERR_INVALID_ARG, "tp_rank %d of %d", rank, tp);
        if (!id) return set_err(TALOS_ERR_INVALID_ARG, "NCCL unique id is NULL");
        if (cfg->n_head_kv % tp || cfg->n_ff % tp)
            return set_err(TALOS_ERR_UNSUPPORTED, "n_head_kv %u and n_ff %u must split evenly over %d ranks",
                           cfg->n_head_kv, cfg->n_ff, tp);
    }
    TRY(device_setup(device));
    std::unique_ptr<talos_ctx> c(new talos_ctx());
    c->cfg = *cfg;
    c->device = device;
    c->hd = (int)hd;
    c->kv_dim = (int)(cfg->n_head_kv * hd);
    c->group = (int)(cfg->n_head / cfg->n_head_kv);
    c->kv_ctx = cfg->context_length;
    c->tp = tp;
    c->rank = rank;
    c->nh_l = (int)cfg->n_head / tp;
    c->nkv_l = (int)cfg->n_head_kv / tp;
    c->q_rows = c->nh_l * (int)hd;
    c->kv_l = c->nkv_l * (int)hd;
    c->ff_l = (int)cfg->n_ff / tp;
    const int vchunk = ((int)cfg->vocab_size + tp - 1) / tp;
    c->v_off = rank * vchunk;
    c->v_l = std::min(vchunk, (int)cfg->vocab_size - c->v_off);
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    TRY(alloc_arena(c.get()));
    TRY(alloc_kv(c.get()));
    TRY(alloc_sync(c.get()));
    if (tp > 1) {
        ncclUniqueId uid;
        static_assert(sizeof(uid.internal) == 128, "NCCL unique id size");
        memcpy(uid.internal, id, 128);
        if (!nccl().ok) return set_err(TALOS_ERR_NCCL, "libnccl.so.2 could not be opened");
        ncclResult_t nr = nccl().CommInitRank(&c->comm, tp, uid, rank);
        if (nr != ncclSuccess) return set_err(TALOS_ERR_NCCL, "ncclCommInitRank: %s", nccl().GetErrorString(nr));
        talos_status st = alloc_shared(c.get());
        if (st != TALOS_OK) {
            talos_ctx_destroy(c.release());
            return st;
        }
    }
    *out = c.release();
    return TALOS_OK;
}

extern "C" talos_status talos_ctx_create(const talos_cfg* cfg, int device, talos_ctx** out) {
    return ctx_create(cfg, device, 1, 0, nullptr, out);
}

extern "C" talos_status talos_ctx_destroy(talos_ctx* c) {
    if (!c) return TALOS_OK;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    c->drop_graphs();
    batch_free(c);
    if (c->h_bp) cudaFreeHost(c->h_bp);
    if (c->h_blog) cudaFreeHost(c->h_blog);
    for (auto& kv : c->w) kv.second.release();
    c->weights.release();
    for (auto& kv : c->resident) kv.second.release();
    c->staging.release();
    for (int r = 0; r < TALOS_MAX_TP; ++r)
        if (c->peer_base[r] && r != c->rank) cudaIpcCloseMemHandle(c->peer_base[r]);
    if (c->shared) cudaFree(c->shared);
    if (c->comm) nccl().CommDestroy(c->comm);
    if (c->arena) cudaFree(c->arena);
    if (c->sync_mem) cudaFree(c->sync_mem);
    if (c->kcache) cudaFree(c->kcache);
    if (c->vcache) cudaFree(c->vcache);
    if (c->rope_cs) cudaFree(c->rope_cs);
    if (c->gen) cudaFree(c->gen);
    if (c->h_out) cudaFreeHost(c->h_out);
    if (c->h_step) cudaFreeHost(c->h_step);
    if (c->h_gen) cudaFreeHost(c->h_gen);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return TALOS_OK;
}

extern "C" talos_status talos_weight_upload(talos_ctx* c, const char* name, const void* bytes, size_t len,
                                            int type, size_t rows, size_t cols) {
    if (!c || !name || (!bytes && len)) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    CK(cudaSetDevice(c->device));
    size_t er, ec;
    bool is_norm;
    std::string nm(name);
    if (!expected_shape(c, nm, &er, &ec, &is_norm))
        return set_err(TALOS_ERR_INVALID_ARG, "\"%s\" is not a tensor of this model", name);
    if (is_norm) {
        if (type != GT_F32) return set_err(TALOS_ERR_INVALID_ARG, "norm weight \"%s\" must be F32", name);
        if (rows * cols != ec || len != ec * 4)
            return set_err(TALOS_ERR_INVALID_ARG, "\"%s\": expected %zu floats, got rows*cols=%zu len=%zu", name,
                           ec, rows * cols, len);
    } else {
        if (rows != er || cols != ec)
            return set_err(TALOS_ERR_INVALID_ARG, "\"%s\": expected [%zu, %zu], got [%zu, %zu]", name, er, ec, rows,
                           cols);
        size_t want = raw_len(type, rows, cols);
        if (!want) return set_err(TALOS_ERR_UNSUPPORTED, "\"%s\": ggml type %d with %zu cols", name, type, cols);
        if (len != want)
            return set_err(TALOS_ERR_INVALID_ARG, "\"%s\": %zu bytes, expected %zu", name, len, want);
    }
    std::vector<uint8_t> shard;
    if (c->tp > 1 && !is_norm && nm != "token_embd.weight") {
        // this rank's shard: column-parallel q/k/v/gate/up/output keep a row
        // range, row-parallel o/down a column range (whole ggml blocks)
        const std::string rest = nm.compare(0, 4, "blk.") == 0 ? nm.substr(nm.find('.', 4) + 1) : nm;
        size_t r0 = 0, r1 = rows, c0 = 0, c1 = cols;
        if (rest == "attn_q.weight") {
            r0 = (size_t)c->rank * c->q_rows, r1 = r0 + c->q_rows;
        } else if (rest == "attn_k.weight" || rest == "attn_v.weight") {
            r0 = (size_t)c->rank * c->kv_l, r1 = r0 + c->kv_l;
        } else if (rest == "ffn_gate.weight" || rest == "ffn_up.weight") {
            r0 = (size_t)c->rank * c->ff_l, r1 = r0 + c->ff_l;
        } else if (rest == "output.weight") {
            r0 = (size_t)c->v_off, r1 = r0 + c->v_l;
        } else if (rest == "attn_output.weight") {
            c0 = (size_t)c->rank * c->q_rows, c1 = c0 + c->q_rows;
        } else if (rest == "ffn_down.weight") {
            c0 = (size_t)c->rank * c->ff_l, c1 = c0 + c->ff_l;
        }
        const size_t be = (size_t)gguf_block_elems(type), bb = (size_t)gguf_block_bytes(type);
        if (c0 % be || c1 % be)
            return set_err(TALOS_ERR_UNSUPPORTED, "\"%s\": rank %d's columns %zu..%zu are not whole %zu-element blocks",
                           name, c->rank, c0, c1, be);
        const size_t rb = cols / be * bb, sb0 = c0 / be * bb, sbn = (c1 - c0) / be * bb;
        shard.resize((r1 - r0) * sbn);
        for (size_t r = r0; r < r1; ++r)
            memcpy(shard.data() + (r - r0) * sbn, (const uint8_t*)bytes + r * rb + sb0, sbn);
        bytes = shard.data();
        len = shard.size();
        rows = r1 - r0;
        cols = c1 - c0;
    }
    DevTensor& t = c->w[nm];
    if (is_norm || nm == "token_embd.weight") {
        // Kept as-is: norm weights as f32, the embedding as raw GGUF blocks (one
        // row is dequantized per token on the GPU).
        void* mem = nullptr;
        TRY(c->weights.place(&t, len, &mem));
        if (mem != t.mem) {
            t.release();
            t.cap = align256(len);
        }
        TRY(c->staging.h2d(mem, bytes, len, c->stream));
        t.type = type;
        t.rows = is_norm ? 1 : rows;
        t.cols = is_norm ? ec : cols;
        t.mem = mem;
        t.bytes = len;
        t.in_arena = true;
        t.kind = is_norm ? DevTensor::FLOATS : DevTensor::RAW;
    } else {
        TRY(upload_packed(type, bytes, len, rows, cols, &t, &c->staging, c->stream, &c->weights));
    }
    c->weights_dirty = true;
    c->drop_graphs();
    return TALOS_OK;
}

extern "C" talos_status talos_ctx_device_bytes(talos_ctx* c, size_t* out) {
    if (!c || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    size_t n = c->arena_bytes + c->kv_bytes + c->staging.cap + c->sync_bytes + c->weights.total + c->bbytes;
    for (auto& kv : c->resident) n += kv.second.bytes;
    *out = n;
    return TALOS_OK;
}

extern "C" talos_status talos_ctx_stream(talos_ctx* c, void** out) {
    if (!c || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    *out = (void*)c->stream;
    return TALOS_OK;
}

extern "C" talos_status talos_cap_context(talos_ctx* c, size_t max_ctx) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    size_t cap = max_ctx > 1 ? max_ctx : 1;
    if (cap < c->cfg.context_length) c->cfg.context_length = (uint32_t)cap;
    c->kv_ctx = c->cfg.context_length;
    return alloc_kv(c);
}

extern "C" talos_status talos_ctx_set_kv_dtype(talos_ctx* c, int dtype) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    if (dtype != TALOS_KV_F32 && dtype != TALOS_KV_F16)
        return set_err(TALOS_ERR_INVALID_ARG, "KV dtype %d", dtype);
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    if ((dtype == TALOS_KV_F16) == (c->kv_f16 != 0)) return TALOS_OK;
    c->kv_f16 = dtype == TALOS_KV_F16;
    c->weights_dirty = true;  // the per-token kernel's checks run again at the next step
    return alloc_kv(c);
}

extern "C" talos_status talos_ctx_kv_dtype(talos_ctx* c, int* out) {
    if (!c || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    *out = c->kv_f16 ? TALOS_KV_F16 : TALOS_KV_F32;
    return TALOS_OK;
}

extern "C" talos_status talos_kv_reset(talos_ctx* c) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    return TALOS_OK;
}

// ------------------------------------------------------------------ the decode step

static talos_status bind_layers(talos_ctx* c) {
    auto get = [&](const std::string& n, DevTensor** out) -> talos_status {
        auto it = c->w.find(n);
        if (it == c->w.end() || !it->second.mem)
            return set_err(TALOS_ERR_STATE, "weight \"%s\" has not been uploaded", n.c_str());
        *out = &it->second;
        return TALOS_OK;
    };
    c->layers.assign(c->cfg.n_layer, LayerW{});
    for (uint32_t l = 0; l < c->cfg.n_layer; ++l) {
        LayerW& L = c->layers[l];
        TRY(get(lname(l, "attn_norm.weight"), &L.attn_norm));
        TRY(get(lname(l, "attn_q.weight"), &L.q));
        TRY(get(lname(l, "attn_k.weight"), &L.k));
        TRY(get(lname(l, "attn_v.weight"), &L.v));
        TRY(get(lname(l, "attn_output.weight"), &L.o));
        TRY(get(lname(l, "ffn_norm.weight"), &L.ffn_norm));
        TRY(get(lname(l, "ffn_gate.weight"), &L.gate));
        TRY(get(lname(l, "ffn_up.weight"), &L.up));
        TRY(get(lname(l, "ffn_down.weight"), &L.down));
        if (L.gate->type != L.up->type)
            return set_err(TALOS_ERR_UNSUPPORTED, "layer %u: ffn_gate and ffn_up must share a ggml type", l);
    }
    DevTensor* t;
    TRY(get("token_embd.weight", &t));
    TRY(get("output_norm.weight", &t));
    TRY(get("output.weight", &t));
    return TALOS_OK;
}

static Seg make_seg(const DevTensor* A, const DevTensor* B, int pair, float* out, int out_rows, int role) {
    Seg s{};
    s.A = A->w;
    s.B = B ? B->w : A->w;
    s.pair = pair;
    s.ntiles = seg_tiles(A->w.rows, pair);
    s.out = out;
    s.out_rows = out_rows;
    s.role = role;
    return s;
}

static talos_status run_mv(talos_ctx* c, MatvecArgs& a, int type) {
    a.ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) a.ntiles += a.seg[i].ntiles;
    cudaError_t e = launch_matvec(a, type, max_ctas(c->device, type, a.K), c->stream, true);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "matvec launch: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

// Record a profiling event after the launch of kernel `kind` (profiling only).
static talos_status mark(talos_ctx* c, int kind) {
    if (!c->prof) return TALOS_OK;
    cudaEvent_t e;
    CK(cudaEventCreate(&e));
    c->prof->push_back({e, kind});
    CK(cudaEventRecord(e, c->stream));
    return TALOS_OK;
}

// Enqueue one token step (llama.rs:96-183 + :89) on c->stream.
static talos_status enqueue_step(talos_ctx* c, GraphMode mode) {
    const talos_cfg& cfg = c->cfg;
    const int E = (int)cfg.n_embd, F = (int)cfg.n_ff;
    cudaStream_t s = c->stream;
    const DevTensor& embd = c->w["token_embd.weight"];
    TRY(mark(c, -1));
    cudaError_t e = launch_embed((const uint8_t*)embd.mem, embd.type, E, (int)cfg.vocab_size, c->step, c->x, s, true);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "embed: %s", cudaGetErrorString(e));
    TRY(mark(c, TALOS_K_EMBED));
    const size_t kv_layer = c->kv_ctx * (size_t)c->kv_dim;
    for (uint32_t l = 0; l < cfg.n_layer; ++l) {
        const LayerW& L = c->layers[l];
        void* kc = (uint8_t*)c->kcache + l * kv_layer * kv_elem(c);
        void* vc = (uint8_t*)c->vcache + l * kv_layer * kv_elem(c);
        // --- rmsnorm + q/k/v + RoPE + KV append (llama.rs:118-130)
        {
            const DevTensor* qkv[3] = {L.q, L.k, L.v};
            float* outs[3] = {c->q, nullptr, nullptr};
            int rows[3] = {E, c->kv_dim, c->kv_dim};
            bool same = L.q->type == L.k->type && L.k->type == L.v->type;
            for (int i = 0; i < 3;) {
                MatvecArgs a{};
                a.K = E;
                a.x = c->x;
                a.norm_w = (const float*)L.attn_norm->mem;
                a.eps = cfg.rms_eps;
                a.epi = EPI_QKV;
                a.step = c->step;
                a.kcache = kc;
                a.vcache = vc;
                a.kv_f16 = c->kv_f16;
                a.kv_dim = c->kv_dim;
                a.hd = c->hd;
                a.rope_cs = c->rope_cs;
                int type = qkv[i]->type;
                int n = same ? 3 : 1;
                for (int j = 0; j < n; ++j)
                    a.seg[a.nseg++] = make_seg(qkv[i + j], nullptr, 0, outs[i + j], rows[i + j], i + j);
                TRY(run_mv(c, a, type));
                TRY(mark(c, TALOS_K_QKV));
                i += n;
            }
        }
        // --- attention (llama.rs:135-155)
        {
            AttnArgs a{};
            a.q = c->q;
            a.kc = kc;
            a.vc = vc;
            a.kv_f16 = c->kv_f16;
            a.out = c->att;
            a.step = c->step;
            a.n_head = (int)cfg.n_head;
            a.n_kv = (int)cfg.n_head_kv;
            a.hd = c->hd;
            a.kv_dim = c->kv_dim;
            a.scale = 1.0f / sqrtf((float)c->hd);
            e = launch_attention(a, s, true);
            if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "attention: %s", cudaGetErrorString(e));
            TRY(mark(c, TALOS_K_ATTN));
        }
        // --- o-proj + residual (llama.rs:157-161)
        {
            MatvecArgs a{};
            a.K = E;
            a.x = c->att;
            a.epi = EPI_ADD;
            a.step = c->step;
            a.seg[a.nseg++] = make_seg(L.o, nullptr, 0, c->x, E, 0);
            TRY(run_mv(c, a, L.o->type));
            TRY(mark(c, TALOS_K_OPROJ));
        }
        // --- rmsnorm + gate/up + SwiGLU (llama.rs:164-171)
        {
            MatvecArgs a{};
            a.K = E;
            a.x = c->x;
            a.norm_w = (const float*)L.ffn_norm->mem;
            a.eps = cfg.rms_eps;
            a.epi = EPI_SWIGLU;
            a.step = c->step;
            a.seg[a.nseg++] = make_seg(L.gate, L.up, 1, c->ff, F, 0);
            TRY(run_mv(c, a, L.gate->type));
            TRY(mark(c, TALOS_K_GATEUP));
        }
        // --- down + residual (llama.rs:172-176)
        {
            MatvecArgs a{};
            a.K = F;
            a.x = c->ff;
            a.epi = EPI_ADD;
            a.step = c->step;
            a.seg[a.nseg++] = make_seg(L.down, nullptr, 0, c->x, E, 0);
            TRY(run_mv(c, a, L.down->type));
            TRY(mark(c, TALOS_K_DOWN));
        }
    }
    const DevTensor& onorm = c->w["output_norm.weight"];
    if (mode == GM_HIDDEN) {
        e = launch_rmsnorm(c->x, (const float*)onorm.mem, cfg.rms_eps, E, c->hidden, s, true);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "rmsnorm: %s", cudaGetErrorString(e));
        return TALOS_OK;
    }
    // --- final rmsnorm + output projection (llama.rs:181, :89)
    {
        const DevTensor& ow = c->w["output.weight"];
        MatvecArgs a{};
        a.K = E;
        a.x = c->x;
        a.norm_w = (const float*)onorm.mem;
        a.eps = cfg.rms_eps;
        a.epi = EPI_LOGITS;
        a.step = c->step;
        a.seg[a.nseg++] = make_seg(&ow, nullptr, 0, c->logits, (int)cfg.vocab_size, 0);
        TRY(run_mv(c, a, ow.type));
        TRY(mark(c, TALOS_K_OUTPUT));
    }
    if (mode == GM_GREEDY) {
        e = launch_greedy_advance(c->step, c->gen, (int)c->kv_ctx + 1, s, true);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "greedy advance: %s", cudaGetErrorString(e));
    }
    return TALOS_OK;
}

// ------------------------------------------------------------------ per-token kernel

// The phases of one step for k_token (llama.rs:96-183, then :89 or :181).
static void build_phases(talos_ctx* c, GraphMode mode, std::vector<TokenPhase>& ph) {
    const talos_cfg& cfg = c->cfg;
    const int E = (int)cfg.n_embd;
    const bool tp = c->tp > 1;
    const size_t kv_layer = c->kv_ctx * (size_t)c->kv_l;
    // tensor parallel: the residual stream alternates between xbuf[0] (written by
    // q/k/v staging) and xbuf[1] (written by gate/up staging); the o-proj partials
    // go to receive slot 0, the down partials to slot 1
    auto xsum = [&](TokenPhase& p, int src, int dst, int slot) {
        p.xsum = tp;
        p.xsrc = src;
        p.xdst = dst;
        p.xslot = slot;
    };
    ph.clear();
    for (uint32_t l = 0; l < cfg.n_layer; ++l) {
        const LayerW& L = c->layers[l];
        void* kc = (uint8_t*)c->kcache + l * kv_layer * kv_elem(c);
        void* vc = (uint8_t*)c->vcache + l * kv_layer * kv_elem(c);
        TokenPhase p{};
        // rmsnorm + q/k/v + RoPE + KV append (llama.rs:118-130); layer 0 reads the embedding row
        p.kind = PH_MATVEC;
        p.type = L.q->type;
        p.embed_in = l == 0;
        p.prof_kind = TALOS_K_QKV;
        xsum(p, 1, 0, 1);
        p.mv.K = E;
        p.mv.x = c->x;
        p.mv.norm_w = (const float*)L.attn_norm->mem;
        p.mv.eps = cfg.rms_eps;
        p.mv.epi = EPI_QKV;
        p.mv.step = c->step;
        p.mv.kcache = kc;
        p.mv.vcache = vc;
        p.mv.kv_f16 = c->kv_f16;
        p.mv.kv_dim = c->kv_l;
        p.mv.hd = c->hd;
        p.mv.rope_cs = c->rope_cs;
        p.mv.seg[p.mv.nseg++] = make_seg(L.q, nullptr, 0, c->q, c->q_rows, 0);
        p.mv.seg[p.mv.nseg++] = make_seg(L.k, nullptr, 0, nullptr, c->kv_l, 1);
        p.mv.seg[p.mv.nseg++] = make_seg(L.v, nullptr, 0, nullptr, c->kv_l, 2);
        ph.push_back(p);
        // attention (llama.rs:135-155)
        p = TokenPhase{};
        p.kind = PH_ATTN;
        p.prof_kind = TALOS_K_ATTN;
        p.at.q = c->q;
        p.at.kc = kc;
        p.at.vc = vc;
        p.at.kv_f16 = c->kv_f16;
        p.at.out = c->att;
        p.at.step = c->step;
        p.at.n_head = c->nh_l;
        p.at.n_kv = c->nkv_l;
        p.at.hd = c->hd;
        p.at.kv_dim = c->kv_l;
        p.at.scale = 1.0f / sqrtf((float)c->hd);
        ph.push_back(p);
        // o-proj + residual (llama.rs:157-161)
        p = TokenPhase{};
        p.kind = PH_MATVEC;
        p.type = L.o->type;
        p.prof_kind = TALOS_K_OPROJ;
        p.att_merge = 1;
        p.mv.hd = c->hd;
        p.mv.K = c->q_rows;
        p.mv.x = c->att;
        p.mv.epi = tp ? EPI_PEER : EPI_ADD;
        p.rx_slot = 0;
        p.xrank = tp;
        p.mv.step = c->step;
        p.mv.seg[p.mv.nseg++] = make_seg(L.o, nullptr, 0, c->x, E, 0);
        ph.push_back(p);
        // rmsnorm + gate/up + SwiGLU (llama.rs:164-171)
        p = TokenPhase{};
        p.kind = PH_MATVEC;
        p.type = L.gate->type;
        p.prof_kind = TALOS_K_GATEUP;
        xsum(p, 0, 1, 0);
        p.mv.K = E;
        p.mv.x = c->x;
        p.mv.norm_w = (const float*)L.ffn_norm->mem;
        p.mv.eps = cfg.rms_eps;
        p.mv.epi = EPI_SWIGLU;
        p.mv.step = c->step;
        p.mv.seg[p.mv.nseg++] = make_seg(L.gate, L.up, 1, c->ff, c->ff_l, 0);
        ph.push_back(p);
        // down + residual (llama.rs:172-176)
        p = TokenPhase{};
        p.kind = PH_MATVEC;
        p.type = L.down->type;
        p.prof_kind = TALOS_K_DOWN;
        p.mv.K = c->ff_l;
        p.mv.x = c->ff;
        p.mv.epi = tp ? EPI_PEER : EPI_ADD;
        p.rx_slot = 1;
        p.xrank = tp;
        p.mv.step = c->step;
        p.mv.seg[p.mv.nseg++] = make_seg(L.down, nullptr, 0, c->x, E, 0);
        ph.push_back(p);
    }
    TokenPhase p{};
    p.prof_kind = TALOS_K_OUTPUT;
    xsum(p, 1, 0, 1);
    p.xrank = tp;  // tensor parallel: a last barrier over every rank (logits, argmax key)
    if (mode == GM_HIDDEN) {
        p.kind = PH_HIDDEN;  // final rmsnorm (llama.rs:181)
    } else {                 // final rmsnorm + output projection (llama.rs:181, :89)
        const DevTensor& ow = c->w["output.weight"];
        const DevTensor& onorm = c->w["output_norm.weight"];
        p.kind = PH_MATVEC;
        p.type = ow.type;
        p.mv.K = E;
        p.mv.x = c->x;
        p.mv.norm_w = (const float*)onorm.mem;
        p.mv.eps = cfg.rms_eps;
        p.mv.epi = EPI_LOGITS;
        p.mv.step = c->step;
        p.mv.seg[p.mv.nseg++] = make_seg(&ow, nullptr, 0, c->logits, c->v_l, 0);
    }
    ph.push_back(p);
    for (auto& q : ph) {
        q.mv.ntiles = 0;
        for (int i = 0; i < q.mv.nseg; ++i) q.mv.ntiles += q.mv.seg[i].ntiles;
    }
}

// Whether k_token can run this model; sets c->fused_why, tk_union and tk_nst.
static void fused_check(talos_ctx* c) {
    c->fused_why.clear();
    char buf[256];
    if (c->hd > 128) {
        snprintf(buf, sizeof buf, "head_dim %d above 128", c->hd);
        c->fused_why = buf;
        return;
    }
    if (c->kv_f16 && c->hd != 32 && c->hd != 64 && c->hd != 128) {
        snprintf(buf, sizeof buf, "f16 KV cache with head_dim %d (32, 64 or 128)", c->hd);
        c->fused_why = buf;
        return;
    }
    if (!token_attn_per_head() && c->group != 1 && c->group != 2 && c->group != 3 && c->group != 4 &&
        c->group != 8) {
        snprintf(buf, sizeof buf, "%d query heads per kv head (1, 2, 3, 4 or 8)", c->group);
        c->fused_why = buf;
        return;
    }
    if (c->cfg.n_embd > 8192) {
        snprintf(buf, sizeof buf, "n_embd %u above 8192", c->cfg.n_embd);
        c->fused_why = buf;
        return;
    }
    const DevTensor& embd = c->w["token_embd.weight"];
    if (c->cfg.n_embd % gguf_block_elems(embd.type)) {
        c->fused_why = "n_embd is not a whole number of token_embd blocks";
        return;
    }
    std::vector<TokenPhase> ph;
    build_phases(c, GM_LOGITS, ph);
    int ub = token_attn_bytes(c->group, c->hd);
    for (uint32_t l = 0; l < c->cfg.n_layer; ++l) {
        const LayerW& L = c->layers[l];
        if (L.k->type != L.q->type || L.v->type != L.q->type) {
            snprintf(buf, sizeof buf, "layer %u: attn_q/k/v do not share a ggml type", l);
            c->fused_why = buf;
            return;
        }
    }
    for (const auto& p : ph)
        if (p.kind == PH_MATVEC) {
            const int kp = token_stage_elems(p.type, p.mv.K);
            // staged input + block sums (+ the attention merge weights of o-proj, or
            // the prefetched norm weights of a normed phase)
            const int b = kp * 4 + kp / 16 * 4 + (p.att_merge ? c->nh_l * c->nsplit * 4 : 0) +
                          (p.mv.norm_w ? kp * 4 : 0);
            if (b > ub) ub = b;
        }
    ub = (ub + 15) / 16 * 16;
    c->tk_union = ub;
    c->tk_nst = token_max_stages(ub);
    if (c->tk_nst < 2) {
        snprintf(buf, sizeof buf, "staged input (%d bytes) leaves no room for the weight ring", ub);
        c->fused_why = buf;
    }
}

static talos_status use_fused(talos_ctx* c, bool* out) {
    *out = false;
    if (c->tp > 1) {  // the all-reduce lives inside the per-token kernel
        if (c->step_pref == TALOS_STEP_LAYERED)
            return set_err(TALOS_ERR_UNSUPPORTED, "tensor parallel steps run the per-token kernel only");
        if (!c->fused_why.empty())
            return set_err(TALOS_ERR_UNSUPPORTED, "tensor parallel: the per-token kernel cannot run this model: %s",
                           c->fused_why.c_str());
        *out = true;
        return TALOS_OK;
    }
    if (c->step_pref == TALOS_STEP_LAYERED) return TALOS_OK;
    if (c->fused_why.empty()) {
        *out = true;
        return TALOS_OK;
    }
    if (c->step_pref == TALOS_STEP_FUSED)
        return set_err(TALOS_ERR_UNSUPPORTED, "the per-token kernel cannot run this model: %s", c->fused_why.c_str());
    return TALOS_OK;
}

// Chunks of a phase's weights the per-token kernel streams before the phase's
// input vector is staged: the whole ring, so the weight stream never pauses at a
// phase boundary (7B shape, decode tok/s by prefetch depth: 2 chunks 524, 4 535,
// 6 546, the 9-stage ring 555; the staging loads were not measurably delayed).
static int tk_prefetch_chunks(const talos_ctx* c) { return c->tk_nst; }

static TokenArgs token_args(talos_ctx* c, GraphMode mode, unsigned long long* stamps) {
    TokenArgs a{};
    const DevTensor& embd = c->w["token_embd.weight"];
    a.ph = c->d_phases[mode];
    a.nph = c->nph[mode];
    a.bars = c->bars;
    a.epoch = c->epoch;
    a.step = c->step;
    a.embd = (const uint8_t*)embd.mem;
    a.embd_type = embd.type;
    a.vocab = (int)c->cfg.vocab_size;
    a.x = c->x;
    a.E = (int)c->cfg.n_embd;
    a.hidden = c->hidden;
    a.out_norm = (const float*)c->w["output_norm.weight"].mem;
    a.eps = c->cfg.rms_eps;
    a.att_part = c->att_part;
    a.nsplit = c->nsplit;
    a.nst = c->tk_nst;
    a.prefetch = tk_prefetch_chunks(c);
    a.union_bytes = c->tk_union;
    a.stamps = stamps;
    a.tp = c->tp;
    a.rank = c->rank;
    a.vocab_off = c->v_off;
    a.xbuf[0] = c->xbuf[0];
    a.xbuf[1] = c->xbuf[1];
    a.rbars = c->rbars;
    if (c->tp > 1) {
        // peer addresses: the same offsets inside every rank's shared area
        const size_t o_rbars = (uint8_t*)c->rbars - (uint8_t*)c->shared;
        const size_t o_key = (uint8_t*)&c->step->argmax_key - (uint8_t*)c->shared;
        const size_t o_log = (uint8_t*)c->logits - (uint8_t*)c->shared;
        const size_t o_rx = 2 * align256((size_t)c->nph_max * 8) + align256(sizeof(StepParams));
        for (int r = 0; r < c->tp; ++r) {
            uint8_t* b = (uint8_t*)c->peer_base[r];
            a.prbars[r] = (unsigned long long*)(b + o_rbars);
            a.pkey[r] = (unsigned long long*)(b + o_key);
            a.plogits[r] = (float*)(b + o_log);
            a.prx[r] = (float*)(b + o_rx);
        }
    }
    return a;
}

static int sm_count(const talos_ctx* c) { return (c->device < 64 && g_sms[c->device]) ? g_sms[c->device] : 148; }

// Upload the phase list of `mode` (outside any capture).
static talos_status prepare_phases(talos_ctx* c, GraphMode mode) {
    if (c->d_phases[mode]) return TALOS_OK;
    std::vector<TokenPhase> ph;
    build_phases(c, mode, ph);
    if ((int)ph.size() > c->nph_max) return set_err(TALOS_ERR_STATE, "phase list longer than the barrier area");
    CK(cudaMalloc(&c->d_phases[mode], ph.size() * sizeof(TokenPhase)));
    CK(cudaMemcpy(c->d_phases[mode], ph.data(), ph.size() * sizeof(TokenPhase), cudaMemcpyHostToDevice));
    c->nph[mode] = (int)ph.size();
    return TALOS_OK;
}

static talos_status enqueue_fused(talos_ctx* c, GraphMode mode, unsigned long long* stamps) {
    TokenArgs a = token_args(c, mode, stamps);
    cudaError_t e = launch_token(a, sm_count(c), c->stream, c->coop);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "per-token kernel launch: %s", cudaGetErrorString(e));
    if (mode == GM_GREEDY) {
        e = launch_greedy_advance(c->step, c->gen, (int)c->kv_ctx + 1, c->stream, false);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "greedy advance: %s", cudaGetErrorString(e));
    }
    return TALOS_OK;
}

static talos_status bind_if_dirty(talos_ctx* c) {
    if (c->weights_dirty) {
        // the uploads ran asynchronously: wait for them, then drop the staging
        TRY(c->staging.finish(c->stream));
        c->staging.release();
        TRY(bind_layers(c));
        fused_check(c);
        c->drop_graphs();
        c->weights_dirty = false;
    }
    return TALOS_OK;
}

static talos_status capture(talos_ctx* c, GraphMode mode, bool fused, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    talos_status st = fused ? enqueue_fused(c, mode, nullptr) : enqueue_step(c, mode);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (st != TALOS_OK) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return st;
    }
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

static talos_status ensure_graph(talos_ctx* c, GraphMode mode) {
    TRY(bind_if_dirty(c));
    if (c->graph[mode]) return TALOS_OK;
    bool fused = false;
    TRY(use_fused(c, &fused));
    c->fused = fused;
    if (!fused) return capture(c, mode, false, &c->graph[mode]);
    TRY(prepare_phases(c, mode));
    talos_status st = capture(c, mode, true, &c->graph[mode]);
    if (st != TALOS_OK && c->coop) {
        // a graph that cannot hold a cooperative launch: every CTA is still
        // resident (one per SM, the kernel's shared memory allows no second)
        c->coop = false;
        st = capture(c, mode, true, &c->graph[mode]);
    }
    return st;
}

extern "C" talos_status talos_ctx_set_step_kernel(talos_ctx* c, int kind) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    if (kind != TALOS_STEP_AUTO && kind != TALOS_STEP_FUSED && kind != TALOS_STEP_LAYERED)
        return set_err(TALOS_ERR_INVALID_ARG, "step kernel kind %d", kind);
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    c->step_pref = kind;
    c->drop_graphs();
    return TALOS_OK;
}

extern "C" talos_status talos_ctx_step_kernel(talos_ctx* c, int* out) {
    if (!c || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    CK(cudaSetDevice(c->device));
    TRY(bind_if_dirty(c));
    bool fused = false;
    TRY(use_fused(c, &fused));
    *out = fused ? TALOS_STEP_FUSED : TALOS_STEP_LAYERED;
    return TALOS_OK;
}

static talos_status check_tok_pos(talos_ctx* c, uint32_t token, size_t pos) {
    if (token >= c->cfg.vocab_size)
        return set_err(TALOS_ERR_INVALID_ARG, "token %u out of range (vocab %u)", token, c->cfg.vocab_size);
    if (pos >= c->kv_ctx)
        return set_err(TALOS_ERR_INVALID_ARG, "pos %zu outside the KV cache (%zu positions)", pos, c->kv_ctx);
    return TALOS_OK;
}

static talos_status set_step(talos_ctx* c, uint32_t token, size_t pos) {
    StepParams* h = c->h_step;
    memset(h, 0, sizeof *h);
    h->token = token;
    h->pos = (uint32_t)pos;
    CK(cudaMemcpyAsync(c->step, h, sizeof *h, cudaMemcpyHostToDevice, c->stream));
    return TALOS_OK;
}

// Error bits of StepParams::error: 1 = token id out of range, 2 = the weight
// stream gave up waiting, 4 = a barrier or hand-off wait ran out, 8 = a matvec
// input of the per-token kernel stayed beyond the f16 hi / lo split's range
// after its one 2^-16 rescale (an element of magnitude 2^31 or more).
static talos_status finish_step(talos_ctx* c) {
    CK(cudaMemcpyAsync(c->h_step, c->step, sizeof(StepParams), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    const uint32_t err = c->h_step->error;
    if (!err) return TALOS_OK;
    reset_sync(c);
    if (err & 6u) return set_err(TALOS_ERR_TIMEOUT, "a bounded device wait ran out (code %u)", err);
    if (err & 8u)
        return set_err(TALOS_ERR_UNSUPPORTED, "an activation of magnitude 2^31 or more (code %u); the layered "
                       "step kernel (TALOS_STEP_LAYERED) rescales further", err);
    return set_err(TALOS_ERR_OOB, "device bounds check fired (code %u)", err);
}

static talos_status forward_common(talos_ctx* c, uint32_t token, size_t pos, float* out, GraphMode mode) {
    if (!c || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    CK(cudaSetDevice(c->device));
    TRY(check_tok_pos(c, token, pos));
    TRY(ensure_graph(c, mode));
    TRY(set_step(c, token, pos));
    CK(cudaGraphLaunch(c->graph[mode], c->stream));
    size_t n = mode == GM_HIDDEN ? c->cfg.n_embd : c->cfg.vocab_size;
    CK(cudaMemcpyAsync(c->h_out, mode == GM_HIDDEN ? c->hidden : c->logits, n * 4, cudaMemcpyDeviceToHost,
                       c->stream));
    TRY(finish_step(c));
    memcpy(out, c->h_out, n * 4);
    return TALOS_OK;
}

extern "C" talos_status talos_forward(talos_ctx* c, uint32_t token, size_t pos, float* logits_out) {
    return forward_common(c, token, pos, logits_out, GM_LOGITS);
}

extern "C" talos_status talos_forward_hidden(talos_ctx* c, uint32_t token, size_t pos, float* hidden_out) {
    return forward_common(c, token, pos, hidden_out, GM_HIDDEN);
}

extern "C" talos_status talos_generate_greedy(talos_ctx* c, uint32_t token, size_t pos, size_t n,
                                              uint32_t* tokens_out) {
    if (!c || (!tokens_out && n)) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (n == 0) return TALOS_OK;
    CK(cudaSetDevice(c->device));
    TRY(check_tok_pos(c, token, pos));
    if (pos + n > c->kv_ctx)
        return set_err(TALOS_ERR_INVALID_ARG, "pos %zu + %zu steps exceeds the KV cache (%zu)", pos, n, c->kv_ctx);
    TRY(ensure_graph(c, GM_GREEDY));
    TRY(set_step(c, token, pos));
    for (size_t i = 0; i < n; ++i) CK(cudaGraphLaunch(c->graph[GM_GREEDY], c->stream));
    CK(cudaMemcpyAsync(c->h_gen, c->gen, n * 4, cudaMemcpyDeviceToHost, c->stream));
    TRY(finish_step(c));
    memcpy(tokens_out, c->h_gen, n * 4);
    return TALOS_OK;
}

// Per-token step parameters for a prefill, set by a kernel so the host never
// rewrites a buffer a pending copy still reads.
__global__ void k_set_step(StepParams* s, uint32_t token, uint32_t pos) {
    s->token = token;
    s->pos = pos;
}

static talos_status prefill_chunked(talos_ctx* c, const uint32_t* tokens, size_t n, size_t pos0, float* last_logits,
                                    bool* taken);

extern "C" talos_status talos_prefill(talos_ctx* c, const uint32_t* tokens, size_t n, size_t pos0,
                                      float* last_logits) {
    if (!c || (!tokens && n)) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (n == 0) return TALOS_OK;
    CK(cudaSetDevice(c->device));
    for (size_t i = 0; i < n; ++i) TRY(check_tok_pos(c, tokens[i], pos0 + i));
    bool taken = false;
    TRY(prefill_chunked(c, tokens, n, pos0, last_logits, &taken));
    if (taken) return TALOS_OK;
    TRY(ensure_graph(c, GM_LOGITS));
    TRY(set_step(c, tokens[0], pos0));
    for (size_t i = 0; i < n; ++i) {
        if (i) {
            k_set_step<<<1, 1, 0, c->stream>>>(c->step, tokens[i], (uint32_t)(pos0 + i));
            CK(cudaGetLastError());
        }
        CK(cudaGraphLaunch(c->graph[GM_LOGITS], c->stream));
    }
    if (last_logits)
        CK(cudaMemcpyAsync(c->h_out, c->logits, c->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, c->stream));
    TRY(finish_step(c));
    if (last_logits) memcpy(last_logits, c->h_out, c->cfg.vocab_size * 4);
    return TALOS_OK;
}

static talos_status profile_fused(talos_ctx* c, double* kernel_ms, uint32_t* launches) {
    TRY(prepare_phases(c, GM_LOGITS));
    const int nph = c->nph[GM_LOGITS];
    std::vector<TokenPhase> ph;
    build_phases(c, GM_LOGITS, ph);
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0, c->stream));
    talos_status st = enqueue_fused(c, GM_LOGITS, c->stamps);
    CK(cudaEventRecord(e1, c->stream));
    const int G = sm_count(c);
    std::vector<unsigned long long> raw((size_t)nph * G * 4), stamps(nph);
    CK(cudaMemcpyAsync(raw.data(), c->stamps, raw.size() * 8, cudaMemcpyDeviceToHost, c->stream));
    if (st == TALOS_OK) st = finish_step(c);
    float total = 0.f;
    if (st == TALOS_OK) CK(cudaEventElapsedTime(&total, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    TRY(st);
    for (int p = 0; p < nph; ++p) stamps[p] = raw[(size_t)p * G * 4];  // CTA 0 entering phase p
    if (c->last_stamps) *c->last_stamps = raw;
    double inner = 0.0;
    for (int p = 0; p < nph; ++p) {
        double ms;
        if (p + 1 < nph) {
            ms = (double)(stamps[p + 1] - stamps[p]) * 1e-6;
            inner += ms;
        } else {
            ms = (double)total - inner;  // last phase + launch and drain
        }
        const int k = ph[p].prof_kind;
        if (kernel_ms) kernel_ms[k] += ms;
        if (launches) launches[k] += 1;
    }
    return TALOS_OK;
}

// ------------------------------------------------------------------ batched steps
//
// Up to MB_SEQ token columns per step, every weight read once per step for all
// of them through the tcgen05 GEMM (gemm.cu). Three uses, one captured CUDA
// graph per use and token-tile size (32, 64 or 128 columns), each reading the
// column count, tokens and positions from device memory:
//  * BM_DECODE (talos_forward_batch): independent sequences, each with its own
//    cache slot and position, and their logits;
//  * BM_PREFILL (talos_prefill): consecutive prompt positions of the one
//    sequence of the main cache (src/main.rs:88-95), no logits;
//  * BM_SCORE (talos_perplexity): the same with every column's logits;
//  * BM_FILL (talos_prefill_slot): consecutive prompt positions of one
//    sequence of the batch, into its cache slot, no logits;
//  * BM_GREEDY (talos_generate_batch_greedy): BM_DECODE, then each column's
//    argmax becomes its next token on the device (replayed step after step).
// The step is the layered sequence of src/model/llama.rs:96-183 per column:
// embedding row; per layer GEMM q/k/v (RoPE, cache append), attention, GEMM
// o-proj (+ residual), GEMM gate/up (SwiGLU), GEMM down (+ residual); then the
// final norm and the output GEMM. A column at position p attends to positions
// 0 .. p of its cache, so prompt positions of one step see each other's rows.

enum BatchMode { BM_DECODE = 0, BM_PREFILL = 1, BM_SCORE = 2, BM_FILL = 3, BM_GREEDY = 4 };
static bool mode_slots(int mode) { return mode == BM_DECODE || mode == BM_FILL || mode == BM_GREEDY; }
static bool mode_logits(int mode) { return mode != BM_PREFILL && mode != BM_FILL; }
static int nt_of(int ntc) { return 32 << ntc; }
static int ntc_for(int n) { return n <= 32 ? 0 : (n <= 64 ? 1 : 2); }
constexpr int GM_MAX_WAVES = 5;   // split-K never makes more than 5 units per SM
constexpr int GM_MAX_CNT = 4096;  // split-K counters (4 per output tile)

static talos_status batch_free(talos_ctx* c) {
    CK(cudaStreamSynchronize(c->stream));
    c->drop_batch_graphs();
    if (c->bmem) cudaFree(c->bmem);
    c->bmem = nullptr;
    c->bbytes = 0;
    c->bmax = 0;
    for (int r = 0; r < TALOS_MAX_TP; ++r) {
        if (c->bsh_peer[r] && r != c->rank) cudaIpcCloseMemHandle(c->bsh_peer[r]);
        c->bsh_peer[r] = nullptr;
    }
    if (c->bsh) cudaFree(c->bsh);
    c->bsh = nullptr;
    c->blar = nullptr;
    c->btpstep = 0;
    return TALOS_OK;
}

// Tensor parallel: the batched steps' shared area (see talos_ctx::bsh), mapped
// by every rank; every rank allocates it at the same point (talos_ctx_set_batch,
// or the first prefill / perplexity call that takes the batched steps).
static talos_status batch_alloc_shared(talos_ctx* c) {
    const size_t E = c->cfg.n_embd, V = c->cfg.vocab_size, ninst = 2 * (size_t)c->cfg.n_layer + 1;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    take(ninst * 8);
    c->bsh_o_abort = take(4);
    c->bsh_sync_bytes = off;
    c->bsh_o_rx = take(2 * (size_t)c->tp * MB_SEQ * E * 4);
    c->bsh_o_log = take((size_t)MB_SEQ * V * 4);
    CK(cudaMalloc(&c->bsh, off));
    CK(cudaMemset(c->bsh, 0, off));
    TRY(ipc_exchange(c, c->bsh, c->bsh_peer, false));
    c->blog = (float*)((uint8_t*)c->bsh + c->bsh_o_log);
    return TALOS_OK;
}

// The batched steps' buffers, with cache slots for max_seqs sequences (0: the
// activations only, for prefill and perplexity on the main cache).
static talos_status batch_alloc_body(talos_ctx* c, int max_seqs) {
    const size_t E = c->cfg.n_embd, F = c->cfg.n_ff, V = c->cfg.vocab_size, L = c->cfg.n_layer;
    const size_t KPmax = ((std::max(E, F) + 127) / 128) * 128;  // largest GEMM input, rounded to 128
    const int sms = sm_count_dev(c->device);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    // tensor parallel: this rank's q / attention rows, ff rows, kv rows; the
    // logits are gathered in the shared area
    const size_t Q = c->q_rows, Fl = c->ff_l;
    const size_t o_bp = take(sizeof(BatchParams)), o_lar = take(8);
    const size_t o_x = take(MB_SEQ * E * 4), o_q = take(MB_SEQ * Q * 4), o_att = take(MB_SEQ * Q * 4),
                 o_g = take(MB_SEQ * Fl * 4), o_u = take(MB_SEQ * Fl * 4), o_h = take(MB_SEQ * Fl * 4),
                 o_log = c->tp > 1 ? 0 : take(MB_SEQ * V * 4);
    const size_t o_pl = take(2 * MB_SEQ * KPmax * 2), o_xs = take(MB_SEQ * 4);
    const size_t o_ws = take((size_t)GM_MAX_WAVES * sms * 128 * 128 * 4), o_cnt = take(GM_MAX_CNT * 4);
    const size_t seq_stride = L * c->kv_ctx * (size_t)c->kv_l;
    const size_t o_kc = take((size_t)max_seqs * seq_stride * 4 + 4), o_vc = take((size_t)max_seqs * seq_stride * 4 + 4);
    const int gen_cap = max_seqs ? (int)c->kv_ctx : 0;
    const size_t o_gen = take((size_t)MB_SEQ * gen_cap * 4 + 4);
    void* mem = nullptr;
    CK(cudaMalloc(&mem, off));
    CK(cudaMemsetAsync(mem, 0, off, c->stream));
    uint8_t* b = (uint8_t*)mem;
    c->bmem = mem;
    c->bbytes = off;
    c->bp = (BatchParams*)(b + o_bp);
    c->blar = (unsigned long long*)(b + o_lar);
    c->bx = (float*)(b + o_x), c->bq = (float*)(b + o_q);
    c->batt = (float*)(b + o_att), c->bg = (float*)(b + o_g), c->bu = (float*)(b + o_u), c->bh = (float*)(b + o_h);
    c->blog = (float*)(b + o_log);
    if (c->tp > 1) TRY(batch_alloc_shared(c));
    c->bplanes = b + o_pl, c->bxs = (float*)(b + o_xs), c->bldp = (int)KPmax;
    c->bws = (float*)(b + o_ws), c->bcnt = (unsigned*)(b + o_cnt);
    c->bkc = (float*)(b + o_kc), c->bvc = (float*)(b + o_vc);
    c->bgen = (uint32_t*)(b + o_gen), c->bgen_cap = gen_cap;
    c->bseq_stride = seq_stride;
    if (gemm_map_bytes() > sizeof c->bmaps[0]) return set_err(TALOS_ERR_CUDA, "tensor map larger than its slot");
    for (int i = 0; i < 3; ++i) {
        cudaError_t e = gemm_tensor_map(c->bplanes, c->bldp, MB_SEQ, nt_of(i), c->bmaps[i]);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "tensor map: %s", cudaGetErrorString(e));
    }
    if (!c->h_bp) CK(cudaMallocHost(&c->h_bp, sizeof(BatchParams)));
    if (!c->h_blog) CK(cudaMallocHost(&c->h_blog, (size_t)TALOS_MAX_BATCH * V * 4));
    c->bmax = max_seqs;
    CK(cudaStreamSynchronize(c->stream));
    return TALOS_OK;
}

// batch_alloc_body, or on any failure no batch area at all (a half-made one
// would pass chunked_ready's check); the error message is the body's.
static talos_status batch_alloc(talos_ctx* c, int max_seqs) {
    TRY(batch_free(c));
    const talos_status st = batch_alloc_body(c, max_seqs);
    if (st != TALOS_OK) {
        const std::string msg = g_last_error;
        batch_free(c);
        g_last_error = msg;
    }
    return st;
}

extern "C" talos_status talos_ctx_set_batch(talos_ctx* c, int max_seqs) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    if (max_seqs < 0 || max_seqs > TALOS_MAX_BATCH)
        return set_err(TALOS_ERR_INVALID_ARG, "batch of %d sequences (at most %d)", max_seqs, TALOS_MAX_BATCH);
    CK(cudaSetDevice(c->device));
    if (max_seqs == 0) return batch_free(c);
    return batch_alloc(c, max_seqs);
}

// The input of the previous GEMM of the step, when formatted the same way (the
// next GEMM reads it again without a new k_xfmt_g).
struct GmInput {
    const float* in = nullptr;
    const float* norm = nullptr;
    int K = 0;
};

static GemmSeg gseg(const DevTensor* A, float* y, int ldy, int rows, int epi) {
    GemmSeg g{};
    g.A = A->w;
    g.wmap = A->gmap;
    if (A->gmap) {
        memcpy(g.map_lrec, A->gmaps[0], sizeof g.map_lrec);
        memcpy(g.map_sc, A->gmaps[1], sizeof g.map_sc);
    }
    g.ntiles = (A->w.rows + 127) / 128;
    g.y = y;
    g.ldy = ldy;
    g.rows = rows;
    g.epi = epi;
    return g;
}

// K slices per output tile: the split that fills the SMs' waves best (a slice
// costs a partial tile's round trip through L2, in proportion to the tile's nt
// columns, so more slices must earn it).
static int gm_split(int nrt, int R, int sms, int nt) {
    int best = 1;
    double bscore = -1.0;
    for (int S = 1; S <= std::min(R, 16); ++S) {
        const long units = (long)nrt * S;
        if (S > 1 && (units > (long)GM_MAX_WAVES * sms || nrt * 4 > GM_MAX_CNT)) break;
        const long waves = (units + sms - 1) / sms;
        const double score = (double)units / (double)(waves * sms) - 0.02 * (nt / 32) * (S - 1);
        if (score > bscore + 1e-9) {
            bscore = score;
            best = S;
        }
    }
    return best;
}

// One GEMM of the batched step: format its input unless the previous GEMM read
// the same one, then every segment's rows for every live column.
static talos_status gm(talos_ctx* c, GmInput& fi, GemmArgs a, const float* in, const float* norm, int ntc,
                       int* grid_out = nullptr) {
    const int type = a.seg[0].A.type, nt = nt_of(ntc);
    const int K = a.K, KP = (K + 127) / 128 * 128;
    cudaError_t e = cudaSuccess;
    if (fi.in != in || fi.norm != norm || fi.K != K) {
        e = launch_xfmt_g(in, K, K, KP, c->bldp, MB_SEQ, nt, norm, c->cfg.rms_eps, c->bp, c->bplanes, c->bxs,
                          c->stream);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "GEMM input format: %s", cudaGetErrorString(e));
        fi = GmInput{in, norm, K};
    }
    const int sms = sm_count(c);
    a.KP = KP;
    a.nrt = 0;
    for (int i = 0; i < a.nseg; ++i) a.nrt += a.seg[i].ntiles;
    a.S = gm_split(a.nrt, KP / 128, sms, nt);
    a.xs = c->bxs;
    a.bp = c->bp;
    a.ws = c->bws;
    a.cnt = c->bcnt;
    const int units = a.nrt * a.S;  // one token tile: a step holds at most nt columns
    const int grid = std::min(units, sms);
    e = launch_gemm(c->bmaps[ntc], a, type, nt, grid, c->stream, true);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "GEMM launch: %s", cudaGetErrorString(e));
    if (grid_out) *grid_out = grid;
    return TALOS_OK;
}

// Tensor parallel: a GEMM segment whose rows go to every rank (EPI_B_PEER) at
// offset `off` floats of each rank's shared area with row stride ldy; the
// GEMM's CTAs count their exits in blar.
static void peer_out(talos_ctx* c, GemmArgs& a, size_t off) {
    for (int r = 0; r < c->tp; ++r) a.peer[r] = (float*)((uint8_t*)c->bsh_peer[r]) + off;
    a.npeer = c->tp;
    a.lar = c->blar;
}

// Tensor parallel: the join after an EPI_B_PEER GEMM of `grid` CTAs (instance
// `inst` of the step); with sum, this rank's receive slots `buf` are added to bx.
static talos_status tp_join(talos_ctx* c, int inst, int grid, bool sum, int buf) {
    TpJoin j{};
    j.lar = c->blar;
    j.lar_target = (unsigned)grid;
    j.rarr = (unsigned long long*)c->bsh;
    j.abort = (unsigned*)((uint8_t*)c->bsh + c->bsh_o_abort);
    for (int r = 0; r < c->tp; ++r) {
        j.prarr[r] = (unsigned long long*)c->bsh_peer[r];
        j.pabort[r] = (unsigned*)((uint8_t*)c->bsh_peer[r] + c->bsh_o_abort);
    }
    j.inst = inst;
    j.tp = c->tp;
    j.rx = sum ? (const float*)((uint8_t*)c->bsh + c->bsh_o_rx) + (size_t)buf * c->tp * MB_SEQ * c->cfg.n_embd
               : nullptr;
    j.x = c->bx;
    j.E = (int)c->cfg.n_embd;
    cudaError_t e = launch_tp_join_b(j, c->bp, sm_count(c), c->stream);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "tensor-parallel join: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

static talos_status enqueue_batch(talos_ctx* c, int mode, int ntc) {
    const talos_cfg& cfg = c->cfg;
    const int E = (int)cfg.n_embd, Fl = c->ff_l, V = (int)cfg.vocab_size, Q = c->q_rows;
    const bool tp = c->tp > 1;
    // tensor parallel: receive slot buf of this rank, in floats from a shared area's base
    const size_t slot = (size_t)MB_SEQ * E;
    auto rx_off = [&](int buf) { return c->bsh_o_rx / 4 + ((size_t)buf * c->tp + c->rank) * slot; };
    const DevTensor& embd = c->w["token_embd.weight"];
    cudaError_t e = launch_embed_b((const uint8_t*)embd.mem, embd.type, E, V, c->bp, c->bx, E, c->stream);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "batched embed: %s", cudaGetErrorString(e));
    GmInput fi;
    const bool slots = mode_slots(mode);
    const size_t kv_layer = c->kv_ctx * (size_t)c->kv_l;
    const size_t seq_stride = slots ? c->bseq_stride : 0;
    for (uint32_t l = 0; l < cfg.n_layer; ++l) {
        const LayerW& L = c->layers[l];
        float* kc = (slots ? c->bkc : (float*)c->kcache) + l * kv_layer;
        float* vc = (slots ? c->bvc : (float*)c->vcache) + l * kv_layer;
        // rmsnorm + q/k/v + RoPE + KV append (llama.rs:118-130): one GEMM when
        // the three share a type; under tensor parallelism this rank's heads
        {
            const DevTensor* w3[3] = {L.q, L.k, L.v};
            const int epi3[3] = {EPI_B_ROPE, EPI_B_KCACHE, EPI_B_VCACHE};
            const int rows3[3] = {Q, c->kv_l, c->kv_l};
            for (int i = 0; i < 3;) {
                GemmArgs a{};
                a.K = E;
                a.rope_cs = c->rope_cs;
                a.hd = c->hd;
                a.kv_dim = c->kv_l;
                a.kc = kc;
                a.vc = vc;
                a.seq_stride = seq_stride;
                do {
                    a.seg[a.nseg++] = gseg(w3[i], c->bq, Q, rows3[i], epi3[i]);
                    ++i;
                } while (i < 3 && a.seg[0].A.type == w3[i]->type);
                TRY(gm(c, fi, a, c->bx, (const float*)L.attn_norm->mem, ntc));
            }
        }
        // attention (llama.rs:135-155), o-proj + residual (:157-161); under
        // tensor parallelism the o-proj is row-parallel: partial rows to every
        // rank, summed into the residual by the join
        e = launch_attention_b(c->bq, Q, kc, vc, seq_stride, c->kv_l, c->nh_l, c->nkv_l, c->hd, c->batt, Q, c->bp,
                               c->stream);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "batched attention: %s", cudaGetErrorString(e));
        {
            GemmArgs a{};
            a.K = Q;
            int grid = 0;
            a.seg[a.nseg++] = gseg(L.o, c->bx, E, E, tp ? EPI_B_PEER : EPI_B_ADD);
            if (tp) peer_out(c, a, rx_off(0));
            TRY(gm(c, fi, a, c->batt, nullptr, ntc, &grid));
            if (tp) TRY(tp_join(c, 2 * (int)l, grid, true, 0));
        }
        // rmsnorm + SwiGLU FFN (gate and up in one GEMM launch; they share a
        // type, bind_layers) + residual (:163-176)
        {
            GemmArgs a{};
            a.K = E;
            a.seg[a.nseg++] = gseg(L.gate, c->bg, Fl, Fl, EPI_B_STORE);
            a.seg[a.nseg++] = gseg(L.up, c->bu, Fl, Fl, EPI_B_STORE);
            TRY(gm(c, fi, a, c->bx, (const float*)L.ffn_norm->mem, ntc));
            e = launch_swiglu_b(c->bg, c->bu, c->bh, Fl, Fl, c->bp, c->stream);
            if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "batched SwiGLU: %s", cudaGetErrorString(e));
        }
        {
            GemmArgs a{};
            a.K = Fl;
            int grid = 0;
            a.seg[a.nseg++] = gseg(L.down, c->bx, E, E, tp ? EPI_B_PEER : EPI_B_ADD);
            if (tp) peer_out(c, a, rx_off(1));
            TRY(gm(c, fi, a, c->bh, nullptr, ntc, &grid));
            if (tp) TRY(tp_join(c, 2 * (int)l + 1, grid, true, 1));
        }
        fi = GmInput{};  // bx changed in place
    }
    if (!mode_logits(mode)) {
        // prefill: the last column's logits come separately. Every step passes
        // every join instance (their targets count steps), so under tensor
        // parallelism the logits join still runs, without data.
        if (tp) TRY(tp_join(c, 2 * (int)cfg.n_layer, 0, false, 0));
        return TALOS_OK;
    }
    // final norm + logits (:89, :181); under tensor parallelism each rank's
    // vocabulary range goes to every rank's gathered logits
    GemmArgs a{};
    a.K = E;
    int grid = 0;
    a.seg[a.nseg++] = gseg(&c->w["output.weight"], c->blog, V, c->v_l, tp ? EPI_B_PEER : EPI_B_STORE);
    if (tp) peer_out(c, a, c->bsh_o_log / 4 + (size_t)c->v_off);
    TRY(gm(c, fi, a, c->bx, (const float*)c->w["output_norm.weight"].mem, ntc, &grid));
    if (tp) TRY(tp_join(c, 2 * (int)cfg.n_layer, grid, false, 0));
    if (mode == BM_GREEDY) {
        e = launch_greedy_advance_b(c->blog, V, c->bp, c->bgen, c->bgen_cap, c->stream);
        if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "batched greedy: %s", cudaGetErrorString(e));
    }
    return TALOS_OK;
}

static talos_status batch_check(talos_ctx* c) {
    auto ok = [](const DevTensor* t) { return t->type == GT_Q4_0 || t->type == GT_Q8_0 || t->type == GT_Q6_K; };
    for (const LayerW& L : c->layers)
        if (!ok(L.q) || !ok(L.k) || !ok(L.v) || !ok(L.o) || !ok(L.gate) || !ok(L.up) || !ok(L.down))
            return set_err(TALOS_ERR_UNSUPPORTED, "batched steps need Q4_0 / Q8_0 / Q6_K matrices");
    if (!ok(&c->w["output.weight"]))
        return set_err(TALOS_ERR_UNSUPPORTED, "batched steps need a Q4_0 / Q8_0 / Q6_K output matrix");
    if (c->hd > 128 || c->hd % 4) return set_err(TALOS_ERR_UNSUPPORTED, "batched attention needs head_dim <= 128");
    return TALOS_OK;
}

// keep_err: the error bits of the call's earlier steps stay for batch_finish
__global__ void k_set_batch(BatchParams* d, BatchParams v, bool keep_err) {
    if (keep_err) v.error = d->error;
    *d = v;
}

static talos_status batch_graph(talos_ctx* c, int mode, int ntc) {
    cudaGraphExec_t* out = &c->bgraph[mode][ntc];
    if (*out) return TALOS_OK;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    talos_status st = enqueue_batch(c, mode, ntc);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (st != TALOS_OK) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return st;
    }
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "batched graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "batched graph instantiate: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

// The parameters of a batched step of n columns, set by a kernel
// (stream-ordered, so the host never rewrites a buffer a pending copy reads).
// slots: each column's cache slot (NULL: column i in slot i).
static talos_status set_batch_params(talos_ctx* c, const uint32_t* tokens, const size_t* pos, const int* slots,
                                     int n, bool first) {
    BatchParams v{};
    v.n = n;
    for (int i = 0; i < n; ++i) {
        v.token[i] = tokens[i];
        v.pos[i] = (uint32_t)pos[i];
        v.slot[i] = slots ? (uint32_t)slots[i] : (uint32_t)i;
    }
    v.tpstep = c->btpstep;
    k_set_batch<<<1, 1, 0, c->stream>>>(c->bp, v, !first);
    CK(cudaGetLastError());
    return TALOS_OK;
}

// One batched step of n columns: its parameters, then the graph of the
// smallest token tile that holds n.
static talos_status batch_step(talos_ctx* c, int mode, const uint32_t* tokens, const size_t* pos, const int* slots,
                               int n, bool first) {
    if (n < 1 || n > MB_SEQ) return set_err(TALOS_ERR_INVALID_ARG, "%d columns in a batched step", n);
    const int ntc = ntc_for(n);
    TRY(batch_graph(c, mode, ntc));
    TRY(set_batch_params(c, tokens, pos, slots, n, first));
    CK(cudaGraphLaunch(c->bgraph[mode][ntc], c->stream));
    if (c->tp > 1) ++c->btpstep;
    return TALOS_OK;
}

// Copy n x V logits of the last batched step (host may be NULL) and check its errors.
static talos_status batch_finish(talos_ctx* c, int n, float* logits_out) {
    const size_t V = c->cfg.vocab_size;
    if (logits_out) CK(cudaMemcpyAsync(c->h_blog, c->blog, (size_t)n * V * 4, cudaMemcpyDeviceToHost, c->stream));
    BatchParams& hp = *c->h_bp;
    CK(cudaMemcpyAsync(&hp, c->bp, sizeof hp, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (hp.error & 2u) return set_err(TALOS_ERR_TIMEOUT, "batched step: a bounded wait expired");
    if (hp.error) return set_err(TALOS_ERR_OOB, "batched step: device check failed (%u)", hp.error);
    if (logits_out) memcpy(logits_out, c->h_blog, (size_t)n * V * 4);
    return TALOS_OK;
}

extern "C" talos_status talos_forward_batch(talos_ctx* c, const uint32_t* tokens, const size_t* pos, int n,
                                            float* logits_out) {
    if (!c || !tokens || !pos || !logits_out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (n < 1 || n > c->bmax)
        return set_err(TALOS_ERR_INVALID_ARG, "%d sequences (the context holds %d; talos_ctx_set_batch)", n, c->bmax);
    CK(cudaSetDevice(c->device));
    for (int i = 0; i < n; ++i) TRY(check_tok_pos(c, tokens[i], pos[i]));
    TRY(bind_if_dirty(c));
    TRY(batch_check(c));
    TRY(batch_step(c, BM_DECODE, tokens, pos, nullptr, n, true));
    return batch_finish(c, n, logits_out);
}

extern "C" talos_status talos_prefill_slot(talos_ctx* c, int slot, const uint32_t* tokens, size_t n, size_t pos0,
                                           float* last_logits) {
    if (!c || (!tokens && n)) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (slot < 0 || slot >= c->bmax)
        return set_err(TALOS_ERR_INVALID_ARG, "slot %d (the context holds %d; talos_ctx_set_batch)", slot, c->bmax);
    if (n == 0) return TALOS_OK;
    CK(cudaSetDevice(c->device));
    for (size_t i = 0; i < n; ++i) TRY(check_tok_pos(c, tokens[i], pos0 + i));
    TRY(bind_if_dirty(c));
    TRY(batch_check(c));
    std::vector<size_t> pos(MB_SEQ);
    const std::vector<int> slots(MB_SEQ, slot);
    int last_n = 1;
    for (size_t i = 0; i < n; i += MB_SEQ) {
        const int k = (int)std::min<size_t>(MB_SEQ, n - i);
        for (int j = 0; j < k; ++j) pos[j] = pos0 + i + j;
        // the last step also computes its columns' logits when they are wanted
        const int mode = last_logits && i + k == n ? BM_DECODE : BM_FILL;
        TRY(batch_step(c, mode, tokens + i, pos.data(), slots.data(), k, i == 0));
        last_n = k;
    }
    const size_t V = c->cfg.vocab_size;
    if (last_logits)
        CK(cudaMemcpyAsync(c->h_out, c->blog + (size_t)(last_n - 1) * V, V * 4, cudaMemcpyDeviceToHost, c->stream));
    TRY(batch_finish(c, 0, nullptr));
    if (last_logits) memcpy(last_logits, c->h_out, V * 4);
    return TALOS_OK;
}

extern "C" talos_status talos_generate_batch_greedy(talos_ctx* c, const uint32_t* tokens, const size_t* pos, int n,
                                                    size_t steps, uint32_t* tokens_out) {
    if (!c || !tokens || !pos || (!tokens_out && steps)) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (n < 1 || n > c->bmax)
        return set_err(TALOS_ERR_INVALID_ARG, "%d sequences (the context holds %d; talos_ctx_set_batch)", n, c->bmax);
    if (steps == 0) return TALOS_OK;
    CK(cudaSetDevice(c->device));
    for (int i = 0; i < n; ++i) {
        TRY(check_tok_pos(c, tokens[i], pos[i]));
        if (pos[i] + steps > c->kv_ctx)
            return set_err(TALOS_ERR_INVALID_ARG, "sequence %d: positions %zu .. %zu beyond the context (%zu)", i,
                           pos[i], pos[i] + steps - 1, c->kv_ctx);
    }
    TRY(bind_if_dirty(c));
    TRY(batch_check(c));
    const int ntc = ntc_for(n);
    TRY(batch_graph(c, BM_GREEDY, ntc));
    TRY(set_batch_params(c, tokens, pos, nullptr, n, true));
    // the graph advances every column's token and position itself (and the
    // tensor-parallel step count), so the replays need no host work
    for (size_t k = 0; k < steps; ++k) CK(cudaGraphLaunch(c->bgraph[BM_GREEDY][ntc], c->stream));
    if (c->tp > 1) c->btpstep += (uint32_t)steps;
    TRY(batch_finish(c, 0, nullptr));
    std::vector<uint32_t> g((size_t)n * c->bgen_cap);
    CK(cudaMemcpy(g.data(), c->bgen, g.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t k = 0; k < steps; ++k)
        for (int i = 0; i < n; ++i) tokens_out[k * n + i] = g[(size_t)i * c->bgen_cap + k];
    return TALOS_OK;
}

// Whether the batched steps can run consecutive positions of the main cache
// (f32 cache, Q4_0 / Q8_0 / Q6_K matrices); if so their buffers exist. The
// decision depends only on the model and settings every rank shares, so under
// tensor parallelism all ranks take the same path.
static talos_status chunked_ready(talos_ctx* c, bool* ok) {
    *ok = false;
    if (c->kv_f16) return TALOS_OK;
    TRY(bind_if_dirty(c));
    if (batch_check(c) != TALOS_OK) return TALOS_OK;
    if (!c->bmem) TRY(batch_alloc(c, 0));
    *ok = true;
    return TALOS_OK;
}

// logits of one residual-stream row x (device): final norm + output matvec
// (llama.rs:181, :89) into c->logits.
static talos_status row_logits(talos_ctx* c, const float* x) {
    const DevTensor& ow = c->w["output.weight"];
    MatvecArgs a{};
    a.K = (int)c->cfg.n_embd;
    a.x = x;
    a.norm_w = (const float*)c->w["output_norm.weight"].mem;
    a.eps = c->cfg.rms_eps;
    a.epi = EPI_STORE;
    a.step = c->step;
    a.seg[a.nseg++] = make_seg(&ow, nullptr, 0, c->logits, (int)c->cfg.vocab_size, 0);
    return run_mv(c, a, ow.type);
}

// talos_prefill in steps of up to MB_SEQ consecutive prompt positions: one
// weight pass per step instead of one per token. Taken when the batched step
// runs the model and the main cache is f32; false in *taken otherwise. The last
// position's logits: final norm + output matvec of its row on one GPU; under
// tensor parallelism the last step computes its columns' gathered logits.
static talos_status prefill_chunked(talos_ctx* c, const uint32_t* tokens, size_t n, size_t pos0, float* last_logits,
                                    bool* taken) {
    *taken = false;
    if (n < 2) return TALOS_OK;
    TRY(chunked_ready(c, taken));
    if (!*taken) return TALOS_OK;
    int last_n = 1;
    std::vector<size_t> pos(MB_SEQ);
    const std::vector<int> slot0(MB_SEQ, 0);  // the main cache
    const size_t V = c->cfg.vocab_size;
    for (size_t i = 0; i < n; i += MB_SEQ) {
        const int k = (int)std::min<size_t>(MB_SEQ, n - i);
        for (int j = 0; j < k; ++j) pos[j] = pos0 + i + j;
        const bool score = c->tp > 1 && last_logits && i + k == n;
        TRY(batch_step(c, score ? BM_SCORE : BM_PREFILL, tokens + i, pos.data(), slot0.data(), k, i == 0));
        last_n = k;
    }
    if (last_logits && c->tp > 1) {
        CK(cudaMemcpyAsync(c->h_out, c->blog + (size_t)(last_n - 1) * V, V * 4, cudaMemcpyDeviceToHost, c->stream));
    } else if (last_logits) {
        TRY(row_logits(c, c->bx + (size_t)(last_n - 1) * c->cfg.n_embd));
        CK(cudaMemcpyAsync(c->h_out, c->logits, V * 4, cudaMemcpyDeviceToHost, c->stream));
    }
    TRY(batch_finish(c, 0, nullptr));
    if (last_logits) memcpy(last_logits, c->h_out, c->cfg.vocab_size * 4);
    return TALOS_OK;
}

extern "C" talos_status talos_perplexity(talos_ctx* c, const uint32_t* tokens, size_t n, float* ppl_out,
                                         double* nll_sum_out, size_t* scored_out) {
    if (!c || (!tokens && n) || !ppl_out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (n < 2) return set_err(TALOS_ERR_INVALID_ARG, "perplexity needs at least 2 tokens, got %zu", n);
    CK(cudaSetDevice(c->device));
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] >= c->cfg.vocab_size)
            return set_err(TALOS_ERR_INVALID_ARG, "token %u at %zu out of range (vocab %u)", tokens[i], i,
                           c->cfg.vocab_size);
    // positions in steps of up to MB_SEQ through the batched step where it runs the model
    bool chunked = false;
    TRY(chunked_ready(c, &chunked));
    if (!chunked) TRY(ensure_graph(c, GM_LOGITS));
    double* acc = c->nll_acc;  // [nll sum, scored] on the device, cleared on the stream
    talos_status st = TALOS_OK;
    cudaError_t e = cudaMemsetAsync(acc, 0, 2 * sizeof(double), c->stream);
    const int V = (int)c->cfg.vocab_size;
    bool first = true;
    std::vector<size_t> pos(MB_SEQ);
    const std::vector<int> slot0(MB_SEQ, 0);  // the main cache
    // chunks of the context length, each from an empty cache (src/eval.rs:35-52)
    const size_t chunk = c->kv_ctx;
    for (size_t c0 = 0; e == cudaSuccess && st == TALOS_OK && c0 + 1 < n; c0 += chunk) {
        const size_t len = std::min(chunk, n - c0);
        if (len < 2) break;  // a trailing single token predicts nothing
        if (chunked) {
            // scored positions 0 .. len-2, up to MB_SEQ per step, NLLs added in position order
            for (size_t p0 = 0; e == cudaSuccess && st == TALOS_OK && p0 + 1 < len; p0 += MB_SEQ) {
                const int k = (int)std::min<size_t>(MB_SEQ, len - 1 - p0);
                for (int j = 0; j < k; ++j) pos[j] = p0 + j;
                st = batch_step(c, BM_SCORE, tokens + c0 + p0, pos.data(), slot0.data(), k, first);
                first = false;
                for (int j = 0; j < k && st == TALOS_OK && e == cudaSuccess; ++j)
                    e = launch_token_nll(c->blog + (size_t)j * V, V, tokens[c0 + p0 + j + 1], acc, c->stream);
            }
            continue;
        }
        for (size_t pos1 = 0; e == cudaSuccess && pos1 + 1 < len; ++pos1) {
            k_set_step<<<1, 1, 0, c->stream>>>(c->step, tokens[c0 + pos1], (uint32_t)pos1);
            e = cudaGetLastError();
            if (e == cudaSuccess) e = cudaGraphLaunch(c->graph[GM_LOGITS], c->stream);
            if (e == cudaSuccess)
                e = launch_token_nll(c->logits, V, tokens[c0 + pos1 + 1], acc, c->stream);
        }
    }
    double h[2] = {0.0, 0.0};
    if (e == cudaSuccess && st == TALOS_OK) e = cudaMemcpyAsync(h, acc, sizeof h, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess && st == TALOS_OK) st = chunked ? batch_finish(c, 0, nullptr) : finish_step(c);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "perplexity: %s", cudaGetErrorString(e));
    TRY(st);
    *ppl_out = (float)exp(h[0] / h[1]);
    if (nll_sum_out) *nll_sum_out = h[0];
    if (scored_out) *scored_out = (size_t)h[1];
    return TALOS_OK;
}

extern "C" talos_status talos_profile_phases(talos_ctx* c, uint32_t token, size_t pos, uint64_t* out, size_t cap,
                                             int* n_phase, int* n_cta) {
    if (!c || !out || !n_phase || !n_cta) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    CK(cudaSetDevice(c->device));
    TRY(check_tok_pos(c, token, pos));
    TRY(bind_if_dirty(c));
    bool fused = false;
    TRY(use_fused(c, &fused));
    if (!fused) return set_err(TALOS_ERR_UNSUPPORTED, "steps run the layered graph: no phase stamps");
    TRY(prepare_phases(c, GM_LOGITS));
    const size_t n = (size_t)c->nph[GM_LOGITS] * sm_count(c) * 4;
    if (cap < n) return set_err(TALOS_ERR_INVALID_ARG, "out holds %zu values, %zu needed", cap, n);
    CK(cudaMemsetAsync(c->stamps, 0, n * 8, c->stream));
    TRY(set_step(c, token, pos));
    std::vector<unsigned long long> raw;
    c->last_stamps = &raw;
    talos_status st = profile_fused(c, nullptr, nullptr);
    c->last_stamps = nullptr;
    TRY(st);
    memcpy(out, raw.data(), n * 8);
    *n_phase = c->nph[GM_LOGITS];
    *n_cta = sm_count(c);
    return TALOS_OK;
}

extern "C" talos_status talos_profile_step(talos_ctx* c, uint32_t token, size_t pos, double* kernel_ms,
                                           uint32_t* launches) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    CK(cudaSetDevice(c->device));
    TRY(check_tok_pos(c, token, pos));
    TRY(bind_if_dirty(c));
    bool fused = false;
    TRY(use_fused(c, &fused));
    TRY(set_step(c, token, pos));
    if (fused) return profile_fused(c, kernel_ms, launches);
    std::vector<std::pair<cudaEvent_t, int>> ev;
    c->prof = &ev;
    talos_status st = enqueue_step(c, GM_LOGITS);
    c->prof = nullptr;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (st == TALOS_OK && e != cudaSuccess) st = set_err(TALOS_ERR_CUDA, "profile step: %s", cudaGetErrorString(e));
    for (size_t i = 1; st == TALOS_OK && i < ev.size(); ++i) {
        float ms = 0.f;
        e = cudaEventElapsedTime(&ms, ev[i - 1].first, ev[i].first);
        if (e != cudaSuccess) {
            st = set_err(TALOS_ERR_CUDA, "event timing: %s", cudaGetErrorString(e));
            break;
        }
        int k = ev[i].second;
        if (k >= 0 && k < TALOS_K_COUNT) {
            if (kernel_ms) kernel_ms[k] += ms;
            if (launches) launches[k] += 1;
        }
    }
    for (auto& p : ev) cudaEventDestroy(p.first);
    return st;
}

// ------------------------------------------------------------------ tensor parallel

extern "C" talos_status talos_nccl_unique_id(uint8_t out[128]) {
    if (!out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    ncclUniqueId uid;
    if (!nccl().ok) return set_err(TALOS_ERR_NCCL, "libnccl.so.2 could not be opened");
    ncclResult_t nr = nccl().GetUniqueId(&uid);
    if (nr != ncclSuccess) return set_err(TALOS_ERR_NCCL, "ncclGetUniqueId: %s", nccl().GetErrorString(nr));
    memcpy(out, uid.internal, 128);
    return TALOS_OK;
}

extern "C" talos_status talos_ctx_create_tp(const talos_cfg* cfg, int device, int tp_size, int tp_rank,
                                            const uint8_t* id, talos_ctx** out) {
    return ctx_create(cfg, device, tp_size, tp_rank, id, out);
}

extern "C" talos_status talos_ctx_tp_resync(talos_ctx* c) {
    if (!c) return set_err(TALOS_ERR_INVALID_ARG, "NULL ctx");
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    reset_sync(c);  // the per-token kernel's counters and launch epoch
    if (c->bsh) CK(cudaMemsetAsync(c->bsh, 0, c->bsh_sync_bytes, c->stream));  // arrivals, abort word
    if (c->blar) CK(cudaMemsetAsync(c->blar, 0, 8, c->stream));
    c->btpstep = 0;
    CK(cudaStreamSynchronize(c->stream));
    return TALOS_OK;
}

// ------------------------------------------------------------------ kernels as calls

extern "C" talos_status talos_dequant(int type, const void* bytes, size_t n, float* out) {
    if ((!bytes || !out) && n) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    int be = block_elems(type);
    if (!be) return set_err(TALOS_ERR_UNSUPPORTED, "ggml type %d", type);
    if (n % be) return set_err(TALOS_ERR_INVALID_ARG, "%zu elements is not a multiple of block %d", n, be);
    if (n == 0) return TALOS_OK;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    TRY(device_setup(dev));
    size_t len = n / be * block_bytes(type);
    uint8_t* d_raw = nullptr;
    float* d_out = nullptr;
    CK(cudaMalloc(&d_raw, len));
    cudaError_t e = cudaMalloc(&d_out, n * 4);
    if (e == cudaSuccess) e = cudaMemcpy(d_raw, bytes, len, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_dequant(type, d_raw, n, d_out, 0);
    if (e == cudaSuccess) e = cudaMemcpy(out, d_out, n * 4, cudaMemcpyDeviceToHost);
    cudaFree(d_raw);
    if (d_out) cudaFree(d_out);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "dequant: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

extern "C" talos_status talos_argmax(const float* logits, size_t n, uint32_t* index_out) {
    if (!logits || !index_out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (n == 0) return set_err(TALOS_ERR_INVALID_ARG, "argmax of no logits");
    if (n > 0xffffffffull) return set_err(TALOS_ERR_INVALID_ARG, "%zu logits: indices are 32-bit", n);
    int dev = 0;
    CK(cudaGetDevice(&dev));
    TRY(device_setup(dev));
    float* d_v = nullptr;
    unsigned long long* d_key = nullptr;
    CK(cudaMalloc(&d_v, n * 4));
    cudaError_t e = cudaMalloc(&d_key, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemcpy(d_v, logits, n * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_argmax(d_v, n, d_key, 0);
    unsigned long long key = 0ull;
    if (e == cudaSuccess) e = cudaMemcpy(&key, d_key, sizeof key, cudaMemcpyDeviceToHost);
    cudaFree(d_v);
    if (d_key) cudaFree(d_key);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "argmax: %s", cudaGetErrorString(e));
    *index_out = (uint32_t)(key & 0xffffffffull);
    return TALOS_OK;
}

struct talos_weight {
    int device;
    DevTensor t;
};

static talos_status matvec_on(const DevTensor& t, int device, const float* x_dev, float* y_dev, cudaStream_t s) {
    MatvecArgs a{};
    a.K = (int)t.cols;
    a.x = x_dev;
    a.epi = EPI_STORE;
    Seg sg{};
    sg.A = sg.B = t.w;
    sg.ntiles = seg_tiles(t.w.rows, 0);
    sg.out = y_dev;
    sg.out_rows = (int)t.rows;
    a.seg[0] = sg;
    a.nseg = 1;
    a.ntiles = sg.ntiles;
    cudaError_t e = launch_matvec(a, t.type, max_ctas(device, t.type, a.K), s, false);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "matvec launch: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

static talos_status check_matrix(int type, size_t len, size_t rows, size_t cols) {
    size_t want = raw_len(type, rows, cols);
    if (!want) return set_err(TALOS_ERR_UNSUPPORTED, "ggml type %d with %zu cols", type, cols);
    if (len != want) return set_err(TALOS_ERR_INVALID_ARG, "%zu bytes, expected %zu for [%zu, %zu]", len, want, rows, cols);
    if (cols > (size_t)matvec_max_k(type))
        return set_err(TALOS_ERR_UNSUPPORTED, "cols %zu exceed the staged input limit (%d)", cols,
                       matvec_max_k(type));
    return TALOS_OK;
}

extern "C" talos_status talos_weight_create(int device, int type, const void* bytes, size_t len, size_t rows,
                                            size_t cols, talos_weight** out) {
    if (!bytes || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    TRY(check_matrix(type, len, rows, cols));
    TRY(device_setup(device));
    std::unique_ptr<talos_weight> w(new talos_weight());
    w->device = device;
    Staging st;
    talos_status s = upload_packed(type, bytes, len, rows, cols, &w->t, &st, 0);
    if (s == TALOS_OK) s = st.finish(0);
    st.release();
    TRY(s);
    *out = w.release();
    return TALOS_OK;
}

extern "C" talos_status talos_weight_destroy(talos_weight* w) {
    if (!w) return TALOS_OK;
    cudaSetDevice(w->device);
    w->t.release();
    delete w;
    return TALOS_OK;
}

extern "C" talos_status talos_weight_packed_bytes(const talos_weight* w, size_t* out) {
    if (!w || !out) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    *out = w->t.bytes;
    return TALOS_OK;
}

extern "C" talos_status talos_matvec_dev(const talos_weight* w, const float* x_dev, float* y_dev, void* stream) {
    if (!w || !x_dev || !y_dev) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    CK(cudaSetDevice(w->device));
    return matvec_on(w->t, w->device, x_dev, y_dev, (cudaStream_t)stream);
}

// talos_matvec_dev_noalloc: the static scratch's address on each device,
// resolved on the first call there (cudaGetSymbolAddress allocates nothing).
static std::mutex g_noalloc_mu;
static float* g_noalloc_part_dev[64];
static unsigned* g_noalloc_cnt_dev[64];
static int g_noalloc_max_tiles = 0, g_noalloc_max_slices = 0;

extern "C" talos_status talos_matvec_dev_noalloc(const talos_weight* w, const float* x_dev, float* y_dev,
                                                 void* stream) {
    if (!w || !x_dev || !y_dev) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    if (w->device < 0 || w->device >= 64) return set_err(TALOS_ERR_INVALID_ARG, "device %d", w->device);
    CK(cudaSetDevice(w->device));
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_part_dev[w->device]) {
            cudaError_t e = noalloc_scratch(&g_noalloc_part_dev[w->device], &g_noalloc_cnt_dev[w->device],
                                            &g_noalloc_max_tiles, &g_noalloc_max_slices);
            if (e != cudaSuccess) {
                g_noalloc_part_dev[w->device] = nullptr;
                return set_err(TALOS_ERR_CUDA, "scratch address: %s", cudaGetErrorString(e));
            }
        }
    }
    const PackedW& pw = w->t.w;
    const int ntiles = pw.rows_pad / 16;
    if (ntiles > g_noalloc_max_tiles)
        return set_err(TALOS_ERR_UNSUPPORTED, "%d rows: the static scratch holds %d rows", pw.rows,
                       16 * g_noalloc_max_tiles);
    if (noalloc_smem_bytes(pw.type, pw.cols) > 220 * 1024)
        return set_err(TALOS_ERR_UNSUPPORTED, "%d columns: the staged input does not fit shared memory", pw.cols);
    // K slices per tile: enough units for two per SM, whole chunks, at most the scratch's slices
    const int sms = sm_count_dev(w->device);
    int nslice = (2 * sms + ntiles - 1) / ntiles;
    nslice = std::max(1, std::min(nslice, std::min(g_noalloc_max_slices, pw.nk)));
    cudaError_t e = launch_matvec_noalloc(pw, x_dev, y_dev, nslice, g_noalloc_part_dev[w->device],
                                          g_noalloc_cnt_dev[w->device], (cudaStream_t)stream);
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "split-K matvec: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

extern "C" talos_status talos_matvec_bench(const talos_weight* const* ws, int n, const float* x_dev, float* y_dev,
                                           int reps, float* us_per_launch) {
    if (!ws || n <= 0 || !x_dev || !y_dev || reps <= 0 || !us_per_launch)
        return set_err(TALOS_ERR_INVALID_ARG, "bad argument");
    for (int i = 0; i < n; ++i)
        if (!ws[i] || ws[i]->device != ws[0]->device || ws[i]->t.rows != ws[0]->t.rows ||
            ws[i]->t.cols != ws[0]->t.cols || ws[i]->t.type != ws[0]->t.type)
            return set_err(TALOS_ERR_INVALID_ARG, "weights differ in device, shape or type");
    CK(cudaSetDevice(ws[0]->device));
    cudaStream_t s = nullptr;
    CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    talos_status st = TALOS_OK;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    for (int i = 0; e == cudaSuccess && st == TALOS_OK && i < reps; ++i)
        st = matvec_on(ws[i % n]->t, ws[0]->device, x_dev, y_dev, s);
    cudaError_t e_end = cudaStreamEndCapture(s, &g);
    if (e == cudaSuccess) e = e_end;
    if (st == TALOS_OK && e == cudaSuccess) e = cudaGraphInstantiate(&ge, g, 0);
    if (st == TALOS_OK && e == cudaSuccess) e = cudaEventCreate(&e0);
    if (st == TALOS_OK && e == cudaSuccess) e = cudaEventCreate(&e1);
    if (st == TALOS_OK && e == cudaSuccess) e = cudaGraphLaunch(ge, s);  // warm-up replay
    if (st == TALOS_OK && e == cudaSuccess) e = cudaEventRecord(e0, s);
    if (st == TALOS_OK && e == cudaSuccess) e = cudaGraphLaunch(ge, s);
    if (st == TALOS_OK && e == cudaSuccess) e = cudaEventRecord(e1, s);
    if (st == TALOS_OK && e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (st == TALOS_OK && e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    cudaStreamDestroy(s);
    if (st != TALOS_OK) return st;
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "matvec bench: %s", cudaGetErrorString(e));
    *us_per_launch = ms * 1000.f / (float)reps;
    return TALOS_OK;
}

static talos_status matvec_host(const DevTensor& t, int device, const float* x, float* y, cudaStream_t s) {
    float *dx = nullptr, *dy = nullptr;
    CK(cudaMalloc(&dx, t.cols * 4));
    cudaError_t e = cudaMalloc(&dy, t.rows * 4);
    talos_status st = TALOS_OK;
    if (e == cudaSuccess) e = cudaMemcpyAsync(dx, x, t.cols * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) st = matvec_on(t, device, dx, dy, s);
    if (e == cudaSuccess && st == TALOS_OK) e = cudaMemcpyAsync(y, dy, t.rows * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && st == TALOS_OK) e = cudaStreamSynchronize(s);
    cudaFree(dx);
    if (dy) cudaFree(dy);
    if (st != TALOS_OK) return st;
    if (e != cudaSuccess) return set_err(TALOS_ERR_CUDA, "matvec: %s", cudaGetErrorString(e));
    return TALOS_OK;
}

extern "C" talos_status talos_matvec(int device, int type, const void* bytes, size_t len, size_t rows, size_t cols,
                                     const float* x, float* y) {
    if (!bytes || !x || !y) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    talos_weight* w = nullptr;
    TRY(talos_weight_create(device, type, bytes, len, rows, cols, &w));
    talos_status st = matvec_host(w->t, device, x, y, 0);
    talos_weight_destroy(w);
    return st;
}

extern "C" talos_status talos_matvec_resident(talos_ctx* c, const char* name, int type, const void* bytes,
                                              size_t len, size_t rows, size_t cols, const float* x, float* y) {
    if (!c || !name || !bytes || !x || !y) return set_err(TALOS_ERR_INVALID_ARG, "NULL argument");
    CK(cudaSetDevice(c->device));
    TRY(check_matrix(type, len, rows, cols));
    DevTensor& t = c->resident[name];
    // src/math/metal/mod.rs:63-72: reuse the cached buffer while the byte length matches.
    bool hit = t.mem && t.type == type && t.rows == rows && t.cols == cols &&
               raw_len(t.type, t.rows, t.cols) == len;
    if (!hit) {
        TRY(upload_packed(type, bytes, len, rows, cols, &t, &c->staging, c->stream));
        TRY(c->staging.finish(c->stream));
    }
    return matvec_host(t, c->device, x, y, c->stream);
}
