/*
 * talos_oracle.c -- CPU restatement of the Talos decode path (test infrastructure
 * only; see talos_oracle.h). Build: oracle/Makefile (gcc -O2 -ffp-contract=off
 * -pthread). Floating-point contraction is off so every `a * b + c` below rounds
 * twice, like the Rust code it restates.
 */
#define _GNU_SOURCE
#include "talos_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------ errors */

static __thread char g_err[512];

static int fail(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return -1;
}

const char* oracle_last_error(void) { return g_err; }

/*
 * Row-parallel pool standing in for rayon's `par_iter` over output rows
 * (src/math/matmul.rs:37-40, src/math/quant.rs:46-47). Rows are split into equal
 * contiguous ranges, one per thread; the per-row arithmetic does not depend on
 * the split.
 */
typedef void (*row_fn)(void* arg, size_t r0, size_t r1);

static struct {
    pthread_mutex_t mu;
    pthread_cond_t go, done;
    pthread_t th[256];
    int n_workers; /* threads besides the caller */
    int want;      /* requested total threads */
    unsigned gen;
    int pending;
    row_fn fn;
    void* arg;
    size_t rows;
    int parts;
} P = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER};

static void run_part(int part) {
    size_t per = (P.rows + P.parts - 1) / P.parts;
    size_t r0 = (size_t)part * per, r1 = r0 + per;
    if (r1 > P.rows) r1 = P.rows;
    if (r0 < r1) P.fn(P.arg, r0, r1);
}

static void* worker(void* idp) {
    int id = (int)(intptr_t)idp;
    unsigned seen = 0;
    pthread_mutex_lock(&P.mu);
    for (;;) {
        while (P.gen == seen) pthread_cond_wait(&P.go, &P.mu);
        seen = P.gen;
        int part = id + 1;
        int parts = P.parts;
        pthread_mutex_unlock(&P.mu);
        if (part < parts) run_part(part);
        pthread_mutex_lock(&P.mu);
        if (--P.pending == 0) pthread_cond_signal(&P.done);
    }
    return NULL;
}

static int default_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void ensure_pool(void) {
    if (P.want <= 0) P.want = default_threads();
    int need = P.want - 1;
    if (need > 255) need = 255;
    while (P.n_workers < need) {
        pthread_create(&P.th[P.n_workers], NULL, worker, (void*)(intptr_t)P.n_workers);
        P.n_workers++;
    }
}

static void parallel_rows(row_fn fn, void* arg, size_t rows) {
    pthread_mutex_lock(&P.mu);
    ensure_pool();
    int parts = P.want < P.n_workers + 1 ? P.want : P.n_workers + 1;
    if (parts <= 1 || rows < 2) {
        pthread_mutex_unlock(&P.mu);
        fn(arg, 0, rows);
        return;
    }
    P.fn = fn;
    P.arg = arg;
    P.rows = rows;
    P.parts = parts;
    P.pending = P.n_workers;
    P.gen++;
    pthread_cond_broadcast(&P.go);
    pthread_mutex_unlock(&P.mu);
    run_part(0);
    pthread_mutex_lock(&P.mu);
    while (P.pending) pthread_cond_wait(&P.done, &P.mu);
    pthread_mutex_unlock(&P.mu);
}

void oracle_set_threads(int n) {
    pthread_mutex_lock(&P.mu);
    P.want = n > 0 ? n : default_threads();
    pthread_mutex_unlock(&P.mu);
}
int oracle_get_threads(void) { return P.want > 0 ? P.want : default_threads(); }

/* ------------------------------------------------------------------ f16 */

/* half::f16::to_f32 (exact widening), as used at src/gguf/dtype.rs:73,83,102. */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while (!(man & 0x400u));
            bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13) | (man ? 0x00400000u : 0u);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* half::f16::from_f32: round to nearest, ties to even; overflow to infinity. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t half = 1u << (shift - 1);
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t res = man >> shift;
        if (rem > half || (rem == half && (res & 1u))) res++;
        return (uint16_t)(sign | res);
    }
    uint32_t res = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (res & 1u))) res++;
    return (uint16_t)(sign | res);
}

static inline float ld_f16(const uint8_t* p) { return oracle_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------------------ dtype */

/* src/gguf/dtype.rs:43-60 */
int oracle_block_elems(int type) {
    switch (type) {
        case OR_F32: return 1;
        case OR_Q8_0:
        case OR_Q4_0: return 32;
        case OR_Q6_K: return 256;
    }
    return 0;
}
int oracle_block_bytes(int type) {
    switch (type) {
        case OR_F32: return 4;
        case OR_Q8_0: return 34;
        case OR_Q4_0: return 18;
        case OR_Q6_K: return 210;
    }
    return 0;
}

/* One block of `type` -> block_elems floats; src/gguf/dtype.rs:64-121. */
static void dequant_block(int type, const uint8_t* b, float* y) {
    switch (type) {
        case OR_F32: memcpy(y, b, 4); break;
        case OR_Q8_0: { /* dtype.rs:69-78: x = d * (i8)q */
            float d = ld_f16(b);
            for (int i = 0; i < 32; ++i) y[i] = d * (float)(int8_t)b[2 + i];
            break;
        }
        case OR_Q4_0: { /* dtype.rs:79-91: low nibble -> j, high nibble -> j+16 */
            float d = ld_f16(b);
            const uint8_t* qs = b + 2;
            for (int j = 0; j < 16; ++j) {
                int lo = (qs[j] & 0x0F) - 8;
                int hi = (qs[j] >> 4) - 8;
                y[j] = d * (float)lo;
                y[j + 16] = d * (float)hi;
            }
            break;
        }
        case OR_Q6_K: { /* dtype.rs:93-119: y = (d * sc) * q, two halves of 128 */
            const uint8_t* ql0 = b;
            const uint8_t* qh0 = b + 128;
            const int8_t* sc0 = (const int8_t*)(b + 192);
            float d = ld_f16(b + 208);
            for (int n = 0; n < 2; ++n) {
                const uint8_t* ql = ql0 + n * 64;
                const uint8_t* qh = qh0 + n * 32;
                const int8_t* sc = sc0 + n * 8;
                float* yy = y + n * 128;
                for (int l = 0; l < 32; ++l) {
                    int is = l / 16;
                    int q1 = ((ql[l] & 0xF) | ((qh[l] & 0x03) << 4)) - 32;
                    int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 0x03) << 4)) - 32;
                    int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 0x03) << 4)) - 32;
                    int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 0x03) << 4)) - 32;
                    yy[l] = d * (float)sc[is] * (float)q1;
                    yy[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    yy[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    yy[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
            }
            break;
        }
    }
}

int oracle_dequant(int type, const uint8_t* raw, size_t n, float* out) {
    int be = oracle_block_elems(type), bb = oracle_block_bytes(type);
    if (!be) return fail("unsupported ggml type %d", type);
    if (n % (size_t)be) return fail("%zu elements is not a multiple of block %d", n, be);
    for (size_t blk = 0; blk < n / be; ++blk) dequant_block(type, raw + blk * bb, out + blk * be);
    return 0;
}

/* ------------------------------------------------------------------ matvec */

/* src/math/matmul.rs:15-30: f32x8 lanes (mul then add), lane reduce, scalar tail. */
float oracle_dot(const float* a, const float* b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t n8 = n / 8 * 8;
    for (size_t k = 0; k < n8; k += 8)
        for (int i = 0; i < 8; ++i) acc[i] = acc[i] + a[k + i] * b[k + i];
    float s = ((acc[0] + acc[4]) + (acc[2] + acc[6])) + ((acc[1] + acc[5]) + (acc[3] + acc[7]));
    for (size_t k = n8; k < n; ++k) s += a[k] * b[k];
    return s;
}

/* src/math/matmul.rs:34-47: rayon over rows -> OpenMP over rows. */
typedef struct {
    const float* w;
    const float* x;
    float* out;
    size_t cols;
} f32_job;
static void f32_rows(void* a, size_t r0, size_t r1) {
    f32_job* j = (f32_job*)a;
    for (size_t m = r0; m < r1; ++m) j->out[m] = oracle_dot(j->w + m * j->cols, j->x, j->cols);
}
void oracle_matvec_f32(const float* w, const float* x, float* out, size_t rows, size_t cols) {
    f32_job j = {w, x, out, cols};
    parallel_rows(f32_rows, &j, rows);
}

typedef struct {
    const uint8_t* bytes;
    int type;
    const float* x;
    float* out;
    size_t nb, be, bb;
} q_job;
static void q_rows(void* a, size_t r0, size_t r1) {
    q_job* j = (q_job*)a;
    size_t row_bytes = j->nb * j->bb;
    float buf[256];
    for (size_t m = r0; m < r1; ++m) {
        const uint8_t* row = j->bytes + m * row_bytes;
        float sum = 0.0f;
        for (size_t b = 0; b < j->nb; ++b) {
            dequant_block(j->type, row + b * j->bb, buf);
            sum += oracle_dot(buf, j->x + b * j->be, j->be);
        }
        j->out[m] = sum;
    }
}

/* src/math/quant.rs:18-51: per row, per block: dequant into a stack buffer, dot, sum +=. */
int oracle_matvec_quant(const uint8_t* bytes, int type, const float* x, float* out, size_t rows,
                        size_t cols) {
    int be = oracle_block_elems(type), bb = oracle_block_bytes(type);
    if (!be) return fail("unsupported ggml type %d", type);
    if (type == OR_F32) {
        oracle_matvec_f32((const float*)bytes, x, out, rows, cols);
        return 0;
    }
    if (cols % (size_t)be) return fail("cols %zu not a multiple of block %d", cols, be);
    q_job j = {bytes, type, x, out, cols / be, (size_t)be, (size_t)bb};
    parallel_rows(q_rows, &j, rows);
    return 0;
}

/* ------------------------------------------------------------------ ops */

/* src/math/ops.rs:5-12 */
void oracle_rmsnorm(const float* x, const float* w, float eps, float* out, size_t n) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float mean_sq = ss / (float)n;
    float scale = 1.0f / sqrtf(mean_sq + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* src/math/ops.rs:15-25 */
void oracle_softmax(float* x, size_t n) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (size_t i = 0; i < n; ++i) x[i] /= sum;
}

/* src/math/ops.rs:28-37 */
float oracle_silu(float x) { return x / (1.0f + expf(-x)); }
void oracle_swiglu(const float* gate, const float* up, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = oracle_silu(gate[i]) * up[i];
}

/* src/math/ops.rs:48-61: interleaved pairs, theta = pos * base^(-2i/hd) in f32. */
void oracle_rope(float* v, size_t pos, size_t n_head, size_t head_dim, float freq_base) {
    size_t half = head_dim / 2;
    for (size_t h = 0; h < n_head; ++h) {
        size_t base = h * head_dim;
        for (size_t i = 0; i < half; ++i) {
            float theta = (float)pos * powf(freq_base, -2.0f * (float)i / (float)head_dim);
            float s = sinf(theta), c = cosf(theta);
            float a = v[base + 2 * i], b = v[base + 2 * i + 1];
            v[base + 2 * i] = a * c - b * s;
            v[base + 2 * i + 1] = a * s + b * c;
        }
    }
}

/* src/sample.rs:7-14: max_by(total_cmp) -> the LAST maximal element wins ties. */
static inline int32_t total_key(float f) {
    int32_t b;
    memcpy(&b, &f, 4);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}
uint32_t oracle_argmax(const float* logits, size_t n) {
    size_t best = 0;
    int32_t bk = total_key(logits[0]);
    for (size_t i = 1; i < n; ++i) {
        int32_t k = total_key(logits[i]);
        if (k >= bk) {
            bk = k;
            best = i;
        }
    }
    return (uint32_t)best;
}

/* ------------------------------------------------------------------ quantizers */

/* src/math/metal/mod.rs:551-560 (the guarded form of src/gguf/dtype.rs:133-147). */
void oracle_quantize_q8_0(const float* x, size_t n, uint8_t* out) {
    for (size_t blk = 0; blk < n / 32; ++blk) {
        const float* v = x + blk * 32;
        uint8_t* o = out + blk * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        float d = amax / 127.0f;
        uint16_t dh = oracle_f32_to_f16(d);
        o[0] = (uint8_t)(dh & 0xFF);
        o[1] = (uint8_t)(dh >> 8);
        for (int i = 0; i < 32; ++i) {
            float q = 0.0f;
            if (d != 0.0f) {
                q = roundf(v[i] / d);
                if (q < -128.0f) q = -128.0f;
                if (q > 127.0f) q = 127.0f;
            }
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* Rust `f as i32`: truncation toward zero, saturating, NaN -> 0. */
static inline int32_t rust_f32_as_i32(float f) {
    if (f != f) return 0;
    if (f >= 2147483647.0f) return 2147483647;
    if (f <= -2147483648.0f) return (-2147483647 - 1);
    return (int32_t)f;
}

/* src/math/metal/mod.rs:563-574 (the clamped form of src/gguf/dtype.rs:149-167). */
void oracle_quantize_q4_0(const float* x, size_t n, uint8_t* out) {
    for (size_t blk = 0; blk < n / 32; ++blk) {
        const float* v = x + blk * 32;
        uint8_t* o = out + blk * 18;
        float mx = 0.0f;
        for (int i = 0; i < 32; ++i)
            if (fabsf(v[i]) > fabsf(mx)) mx = v[i];
        float d = mx / -8.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        uint16_t dh = oracle_f32_to_f16(d);
        o[0] = (uint8_t)(dh & 0xFF);
        o[1] = (uint8_t)(dh >> 8);
        for (int j = 0; j < 16; ++j) {
            int32_t a = rust_f32_as_i32(v[j] * id + 8.5f);
            int32_t b = rust_f32_as_i32(v[j + 16] * id + 8.5f);
            a = a < 0 ? 0 : (a > 15 ? 15 : a);
            b = b < 0 ? 0 : (b > 15 ? 15 : b);
            o[2 + j] = (uint8_t)(a | (b << 4));
        }
    }
}

/*
 * Q6_K quantizer. The reference has none (its Q6_K test uses random valid blocks,
 * src/math/metal/mod.rs:657-668), so this is written from the block layout that
 * src/gguf/dtype.rs:93-119 decodes: 16 sub-blocks of 16 with an int8 scale each,
 * one f16 super-scale, 6-bit quants biased by 32. Sub-block scale: signed value of
 * largest magnitude / -32; super-scale d = max |scale| / 127; sc = round(scale/d);
 * q = clamp(round(v / (d*sc)), -32, 31).
 */
void oracle_quantize_q6_k(const float* x, size_t n, uint8_t* out) {
    for (size_t sb = 0; sb < n / 256; ++sb) {
        const float* v = x + sb * 256;
        uint8_t* o = out + sb * 210;
        float sub[16];
        float smax = 0.0f;
        for (int s = 0; s < 16; ++s) {
            float mx = 0.0f;
            for (int i = 0; i < 16; ++i)
                if (fabsf(v[s * 16 + i]) > fabsf(mx)) mx = v[s * 16 + i];
            sub[s] = mx / -32.0f;
            if (fabsf(sub[s]) > smax) smax = fabsf(sub[s]);
        }
        float d = smax / 127.0f;
        uint16_t dh = oracle_f32_to_f16(d);
        float dq = oracle_f16_to_f32(dh);
        int8_t sc[16];
        for (int s = 0; s < 16; ++s) {
            float r = (dq != 0.0f) ? roundf(sub[s] / dq) : 0.0f;
            if (r > 127.0f) r = 127.0f;
            if (r < -128.0f) r = -128.0f;
            sc[s] = (int8_t)r;
        }
        uint8_t q[256];
        for (int i = 0; i < 256; ++i) {
            float step = dq * (float)sc[i / 16];
            float r = (step != 0.0f) ? roundf(v[i] / step) : 0.0f;
            if (r > 31.0f) r = 31.0f;
            if (r < -32.0f) r = -32.0f;
            q[i] = (uint8_t)((int)r + 32);
        }
        uint8_t* ql = o;
        uint8_t* qh = o + 128;
        memset(o, 0, 210);
        for (int nh = 0; nh < 2; ++nh) {
            const uint8_t* qq = q + nh * 128;
            for (int l = 0; l < 32; ++l) {
                ql[nh * 64 + l] = (uint8_t)((qq[l] & 0xF) | ((qq[l + 64] & 0xF) << 4));
                ql[nh * 64 + l + 32] = (uint8_t)((qq[l + 32] & 0xF) | ((qq[l + 96] & 0xF) << 4));
                qh[nh * 32 + l] = (uint8_t)((qq[l] >> 4) | ((qq[l + 32] >> 4) << 2) |
                                            ((qq[l + 64] >> 4) << 4) | ((qq[l + 96] >> 4) << 6));
            }
        }
        for (int s = 0; s < 16; ++s) o[192 + s] = (uint8_t)sc[s];
        o[208] = (uint8_t)(dh & 0xFF);
        o[209] = (uint8_t)(dh >> 8);
    }
}

/* ------------------------------------------------------------------ GGUF */

/* Metadata type tags: src/gguf/reader.rs:24-30. */
enum { T_UINT32 = 4, T_INT32 = 5, T_FLOAT32 = 6, T_BOOL = 7, T_STRING = 8, T_ARRAY = 9 };

typedef struct {
    const uint8_t* p;
    size_t len;
} span;

typedef struct {
    char* key;
    uint32_t tag, inner;
    union {
        uint32_t u32;
        float f32;
        int b;
    } v;
    span str;
    size_t count;
    span* strs;          /* ARRAY of STRING */
    const uint8_t* raw;  /* ARRAY of INT32 / FLOAT32 (little-endian, unaligned) */
    int32_t* i32s;
} meta_kv;

typedef struct {
    char* name;
    uint32_t n_dims;
    uint64_t dims[8];
    int type;
    uint64_t offset;
} tensor_info;

struct oracle_gguf {
    uint8_t* buf;
    size_t len;
    int mapped;
    meta_kv* kv;
    size_t n_kv;
    tensor_info* t;
    size_t n_t;
    size_t data_start;
};

typedef struct {
    const uint8_t* b;
    size_t len, pos;
} cursor;

/* reader.rs:90-101: every read is bounds checked. */
static int take(cursor* c, size_t n, const uint8_t** out) {
    if (n > c->len || c->pos > c->len - n)
        return fail("unexpected end of file (need %zu bytes at %zu)", n, c->pos);
    *out = c->b + c->pos;
    c->pos += n;
    return 0;
}
static int rd_u32(cursor* c, uint32_t* v) {
    const uint8_t* p = NULL;
    if (take(c, 4, &p)) return -1;
    memcpy(v, p, 4);
    return 0;
}
static int rd_u64(cursor* c, uint64_t* v) {
    const uint8_t* p = NULL;
    if (take(c, 8, &p)) return -1;
    memcpy(v, p, 8);
    return 0;
}
static int utf8_ok(const uint8_t* s, size_t n) {
    size_t i = 0;
    while (i < n) {
        uint8_t c = s[i];
        size_t k;
        uint32_t cp;
        if (c < 0x80) {
            i++;
            continue;
        } else if ((c & 0xE0) == 0xC0) {
            k = 1;
            cp = c & 0x1F;
        } else if ((c & 0xF0) == 0xE0) {
            k = 2;
            cp = c & 0x0F;
        } else if ((c & 0xF8) == 0xF0) {
            k = 3;
            cp = c & 0x07;
        } else {
            return 0;
        }
        if (i + k >= n) return 0;
        for (size_t j = 1; j <= k; ++j) {
            if ((s[i + j] & 0xC0) != 0x80) return 0;
            cp = (cp << 6) | (s[i + j] & 0x3F);
        }
        if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) ||
            cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
            return 0;
        i += k + 1;
    }
    return 1;
}
/* reader.rs:127-131: u64 length + UTF-8 bytes. */
static int rd_str(cursor* c, span* s) {
    uint64_t n;
    if (rd_u64(c, &n)) return -1;
    if (take(c, (size_t)n, &s->p)) return -1;
    s->len = (size_t)n;
    if (!utf8_ok(s->p, s->len)) return fail("metadata string is not valid UTF-8");
    return 0;
}

static void gguf_release(oracle_gguf* g) {
    if (!g) return;
    for (size_t i = 0; i < g->n_kv; ++i) {
        free(g->kv[i].key);
        free(g->kv[i].strs);
        free(g->kv[i].i32s);
    }
    free(g->kv);
    for (size_t i = 0; i < g->n_t; ++i) free(g->t[i].name);
    free(g->t);
    if (g->mapped)
        munmap(g->buf, g->len);
    else
        free(g->buf);
    free(g);
}
void oracle_gguf_free(oracle_gguf* g) { gguf_release(g); }

static char* dup_span(span s) {
    char* k = (char*)malloc(s.len + 1);
    memcpy(k, s.p, s.len);
    k[s.len] = 0;
    return k;
}

/* reader.rs:135-171 */
static int read_value(cursor* c, meta_kv* kv) {
    const uint8_t* p = NULL;
    switch (kv->tag) {
        case T_UINT32: return rd_u32(c, &kv->v.u32);
        case T_FLOAT32: return rd_u32(c, (uint32_t*)&kv->v.f32);
        case T_BOOL:
            if (take(c, 1, &p)) return -1;
            kv->v.b = p[0] != 0;
            return 0;
        case T_STRING: return rd_str(c, &kv->str);
        case T_ARRAY: {
            uint64_t cnt;
            if (rd_u32(c, &kv->inner) || rd_u64(c, &cnt)) return -1;
            kv->count = (size_t)cnt;
            if (kv->inner == T_STRING) {
                if (cnt > c->len) return fail("unexpected end of file (array of %llu)", (unsigned long long)cnt);
                kv->strs = (span*)malloc(sizeof(span) * (kv->count ? kv->count : 1));
                for (size_t i = 0; i < kv->count; ++i)
                    if (rd_str(c, &kv->strs[i])) return -1;
                return 0;
            }
            if (kv->inner == T_INT32 || kv->inner == T_FLOAT32) {
                if (cnt > (c->len / 4) + 1) return fail("unexpected end of file (array of %llu)", (unsigned long long)cnt);
                if (take(c, kv->count * 4, &kv->raw)) return -1;
                if (kv->inner == T_INT32) {
                    kv->i32s = (int32_t*)malloc(4 * (kv->count ? kv->count : 1));
                    memcpy(kv->i32s, kv->raw, kv->count * 4);
                }
                return 0;
            }
            return fail("unsupported array element type tag %u", kv->inner);
        }
    }
    return fail("unsupported metadata value type tag %u", kv->tag);
}

static int is_supported_type(uint32_t t) { return t == 0 || t == 2 || t == 8 || t == 14; }

/* reader.rs:193-246 */
static int gguf_parse(oracle_gguf* g) {
    cursor c = {g->buf, g->len, 0};
    const uint8_t* magic = NULL;
    if (take(&c, 4, &magic)) return -1;
    if (memcmp(magic, "GGUF", 4)) return fail("not a GGUF file (bad magic)");
    uint32_t version;
    uint64_t n_t, n_kv;
    if (rd_u32(&c, &version)) return -1;
    if (version != 3) return fail("unsupported GGUF version %u (expected 3)", version);
    if (rd_u64(&c, &n_t) || rd_u64(&c, &n_kv)) return -1;
    if (n_kv > g->len || n_t > g->len) return fail("unexpected end of file (counts)");
    g->kv = (meta_kv*)calloc(n_kv ? n_kv : 1, sizeof(meta_kv));
    for (uint64_t i = 0; i < n_kv; ++i) {
        meta_kv* kv = &g->kv[g->n_kv];
        span key;
        if (rd_str(&c, &key)) return -1;
        if (rd_u32(&c, &kv->tag)) return -1;
        kv->key = dup_span(key);
        g->n_kv++;
        if (read_value(&c, kv)) {
            char tmp[1200];
            snprintf(tmp, sizeof tmp, "reading metadata key \"%.200s\": %.900s", kv->key, g_err);
            return fail("%s", tmp);
        }
    }
    g->t = (tensor_info*)calloc(n_t ? n_t : 1, sizeof(tensor_info));
    for (uint64_t i = 0; i < n_t; ++i) {
        tensor_info* t = &g->t[g->n_t];
        span name;
        if (rd_str(&c, &name)) return -1;
        t->name = dup_span(name);
        g->n_t++;
        if (rd_u32(&c, &t->n_dims)) return -1;
        for (uint32_t d = 0; d < t->n_dims; ++d) {
            uint64_t v;
            if (rd_u64(&c, &v)) return -1;
            if (d < 8) t->dims[d] = v;
        }
        if (t->n_dims > 8) return fail("tensor \"%s\" has %u dims", t->name, t->n_dims);
        uint32_t tag;
        if (rd_u32(&c, &tag)) return -1;
        if (!is_supported_type(tag)) return fail("tensor \"%s\" has unsupported ggml type %u", t->name, tag);
        t->type = (int)tag;
        if (rd_u64(&c, &t->offset)) return -1;
    }
    size_t ds = (c.pos + 31) / 32 * 32;
    if (ds > g->len) return fail("data section start %zu past end of file %zu", ds, g->len);
    g->data_start = ds;
    return 0;
}

int oracle_gguf_open(const char* path, oracle_gguf** out) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return fail("opening %s", path);
    struct stat st;
    if (fstat(fd, &st)) {
        close(fd);
        return fail("stat %s", path);
    }
    oracle_gguf* g = (oracle_gguf*)calloc(1, sizeof *g);
    g->len = (size_t)st.st_size;
    if (g->len) {
        g->buf = (uint8_t*)mmap(NULL, g->len, PROT_READ, MAP_SHARED, fd, 0);
        if (g->buf == MAP_FAILED) {
            close(fd);
            free(g);
            return fail("mmapping %s", path);
        }
        g->mapped = 1;
    } else {
        g->buf = (uint8_t*)malloc(1);
    }
    close(fd);
    if (gguf_parse(g)) {
        gguf_release(g);
        return -1;
    }
    *out = g;
    return 0;
}

int oracle_gguf_from_bytes(const uint8_t* bytes, size_t len, oracle_gguf** out) {
    oracle_gguf* g = (oracle_gguf*)calloc(1, sizeof *g);
    g->buf = (uint8_t*)malloc(len ? len : 1);
    memcpy(g->buf, bytes, len);
    g->len = len;
    if (gguf_parse(g)) {
        gguf_release(g);
        return -1;
    }
    *out = g;
    return 0;
}

/* HashMap::insert semantics: a repeated key keeps the last value. */
static const meta_kv* find_kv(const oracle_gguf* g, const char* key) {
    for (size_t i = g->n_kv; i-- > 0;)
        if (!strcmp(g->kv[i].key, key)) return &g->kv[i];
    return NULL;
}
int oracle_gguf_get_u32(const oracle_gguf* g, const char* key, uint32_t* out) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_UINT32) return 0;
    *out = kv->v.u32;
    return 1;
}
int oracle_gguf_get_f32(const oracle_gguf* g, const char* key, float* out) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_FLOAT32) return 0;
    *out = kv->v.f32;
    return 1;
}
int oracle_gguf_get_bool(const oracle_gguf* g, const char* key, int* out) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_BOOL) return 0;
    *out = kv->v.b;
    return 1;
}
int oracle_gguf_get_str(const oracle_gguf* g, const char* key, const char** out, size_t* len) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_STRING) return 0;
    *out = (const char*)kv->str.p;
    *len = kv->str.len;
    return 1;
}
int oracle_gguf_arr_str_len(const oracle_gguf* g, const char* key, size_t* n) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_ARRAY || kv->inner != T_STRING) return 0;
    *n = kv->count;
    return 1;
}
int oracle_gguf_arr_str_item(const oracle_gguf* g, const char* key, size_t i, const char** out,
                             size_t* len) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_ARRAY || kv->inner != T_STRING || i >= kv->count) return 0;
    *out = (const char*)kv->strs[i].p;
    *len = kv->strs[i].len;
    return 1;
}
int oracle_gguf_arr_i32(const oracle_gguf* g, const char* key, const int32_t** out, size_t* n) {
    const meta_kv* kv = find_kv(g, key);
    if (!kv || kv->tag != T_ARRAY || kv->inner != T_INT32) return 0;
    *out = kv->i32s;
    *n = kv->count;
    return 1;
}
size_t oracle_gguf_n_tensors(const oracle_gguf* g) { return g->n_t; }
const char* oracle_gguf_tensor_name(const oracle_gguf* g, size_t i) {
    return i < g->n_t ? g->t[i].name : NULL;
}
int oracle_gguf_tensor_meta(const oracle_gguf* g, size_t i, uint32_t* n_dims, uint64_t dims[4],
                            int* type, uint64_t* offset) {
    if (i >= g->n_t) return 0;
    *n_dims = g->t[i].n_dims;
    for (int d = 0; d < 4; ++d) dims[d] = d < (int)g->t[i].n_dims ? g->t[i].dims[d] : 0;
    *type = g->t[i].type;
    *offset = g->t[i].offset;
    return 1;
}
static const tensor_info* find_tensor(const oracle_gguf* g, const char* name) {
    for (size_t i = g->n_t; i-- > 0;)
        if (!strcmp(g->t[i].name, name)) return &g->t[i];
    return NULL;
}
static int elem_count(const tensor_info* t, size_t* out) {
    unsigned __int128 e = 1;
    for (uint32_t d = 0; d < t->n_dims; ++d) e *= t->dims[d];
    if (e > (unsigned __int128)SIZE_MAX) return fail("tensor element count overflow");
    *out = (size_t)e;
    return 0;
}
/* reader.rs:302-325 */
int oracle_gguf_tensor_f32(const oracle_gguf* g, const char* name, const float** out, size_t* n) {
    const tensor_info* t = find_tensor(g, name);
    if (!t) return fail("no tensor named \"%s\"", name);
    if (t->type != OR_F32) return fail("tensor \"%s\" is type %d, not F32", name, t->type);
    size_t e = 0;
    if (elem_count(t, &e)) return -1;
    if (t->offset > g->len || g->data_start > g->len - t->offset) return fail("tensor offset overflow");
    size_t start = g->data_start + (size_t)t->offset;
    if (e > SIZE_MAX / 4 || start + e * 4 < start) return fail("tensor byte range overflow");
    if (start + e * 4 > g->len) return fail("tensor \"%s\" data range past end of file", name);
    *out = (const float*)(g->buf + start);
    *n = e;
    return 0;
}
/* reader.rs:328-351 */
int oracle_gguf_tensor_raw(const oracle_gguf* g, const char* name, const uint8_t** out,
                           size_t* len, int* type) {
    const tensor_info* t = find_tensor(g, name);
    if (!t) return fail("no tensor named \"%s\"", name);
    size_t e = 0;
    if (elem_count(t, &e)) return -1;
    size_t be = (size_t)oracle_block_elems(t->type);
    if (e % be) return fail("tensor \"%s\" has %zu elems, not a multiple of block %zu", name, e, be);
    size_t bl = (e / be) * (size_t)oracle_block_bytes(t->type);
    if (t->offset > g->len || g->data_start > g->len - t->offset) return fail("tensor offset overflow");
    size_t start = g->data_start + (size_t)t->offset;
    if (start + bl < start) return fail("tensor byte range overflow");
    if (start + bl > g->len) return fail("tensor \"%s\" data range past end of file", name);
    *out = g->buf + start;
    *len = bl;
    *type = t->type;
    return 0;
}

/* ------------------------------------------------------------------ model */

typedef struct {
    const uint8_t* bytes;
    int type;
    size_t rows, cols;
} qtensor;

typedef struct {
    const float* attn_norm;
    qtensor q, k, v, o;
    const float* ffn_norm;
    qtensor gate, up, down;
} layer_w;

struct oracle_model {
    oracle_gguf* g;
    oracle_config cfg;
    qtensor token_embd, output;
    const float* output_norm;
    layer_w* layers;
    /* kv_cache.rs: per-layer append-only rows of n_kv*hd */
    float** kc;
    float** vc;
    size_t* klen; /* rows appended per layer */
    size_t* kcap;
    int kv_f16;   /* opt-in f16 cache of the CUDA path: rows rounded to f16 when appended */
};

/* config.rs:40-67 */
static int config_from_gguf(const oracle_gguf* g, oracle_config* c) {
    const char* arch = "";
    size_t alen = 0;
    if (!oracle_gguf_get_str(g, "general.architecture", &arch, &alen)) {
        arch = "";
        alen = 0;
    }
    if (alen != 5 || memcmp(arch, "llama", 5)) return fail("unsupported architecture (expected \"llama\")");
    size_t vocab;
    if (!oracle_gguf_arr_str_len(g, "tokenizer.ggml.tokens", &vocab))
        return fail("missing tokenizer.ggml.tokens (needed for vocab size)");
    struct {
        const char* k;
        uint32_t* dst;
    } req[] = {{"llama.block_count", &c->n_layer},
               {"llama.attention.head_count", &c->n_head},
               {"llama.attention.head_count_kv", &c->n_head_kv},
               {"llama.embedding_length", &c->n_embd},
               {"llama.feed_forward_length", &c->n_ff},
               {"llama.context_length", &c->context_length},
               {"llama.rope.dimension_count", &c->rope_dim}};
    for (size_t i = 0; i < sizeof req / sizeof req[0]; ++i)
        if (!oracle_gguf_get_u32(g, req[i].k, req[i].dst)) return fail("missing metadata key %s", req[i].k);
    c->vocab_size = (uint32_t)vocab;
    if (!oracle_gguf_get_f32(g, "llama.attention.layer_norm_rms_epsilon", &c->rms_eps)) c->rms_eps = 1e-5f;
    if (!oracle_gguf_get_f32(g, "llama.rope.freq_base", &c->rope_freq_base)) c->rope_freq_base = 10000.0f;
    return 0;
}

static int bind(const oracle_gguf* g, const char* name, size_t rows, size_t cols, qtensor* t) {
    size_t len;
    if (oracle_gguf_tensor_raw(g, name, &t->bytes, &len, &t->type)) return -1;
    t->rows = rows;
    t->cols = cols;
    size_t be = (size_t)oracle_block_elems(t->type);
    if (cols % be || len != rows * (cols / be) * (size_t)oracle_block_bytes(t->type))
        return fail("tensor \"%s\" does not hold a [%zu, %zu] matrix", name, rows, cols);
    return 0;
}
static int bind_norm(const oracle_gguf* g, const char* name, size_t n, const float** out) {
    size_t got;
    if (oracle_gguf_tensor_f32(g, name, out, &got)) return -1;
    if (got != n) return fail("tensor \"%s\" has %zu elements, expected %zu", name, got, n);
    return 0;
}

static void kv_alloc(oracle_model* m) {
    size_t L = m->cfg.n_layer;
    size_t row = (size_t)m->cfg.n_head_kv * (m->cfg.n_embd / m->cfg.n_head);
    for (size_t l = 0; l < L; ++l) {
        free(m->kc[l]);
        free(m->vc[l]);
        m->kcap[l] = m->cfg.context_length ? m->cfg.context_length : 1;
        m->kc[l] = (float*)malloc(sizeof(float) * m->kcap[l] * (row ? row : 1));
        m->vc[l] = (float*)malloc(sizeof(float) * m->kcap[l] * (row ? row : 1));
        m->klen[l] = 0;
    }
}

/* weights.rs:91-114 + llama.rs:43-62 */
static int model_init(oracle_model* m) {
    oracle_config* c = &m->cfg;
    if (config_from_gguf(m->g, c)) return -1;
    if (c->n_head_kv == 0 || c->n_head == 0 || c->n_head % c->n_head_kv)
        return fail("head_count %u must be a positive multiple of head_count_kv %u", c->n_head, c->n_head_kv);
    size_t E = c->n_embd, F = c->n_ff, V = c->vocab_size;
    size_t KV = (size_t)c->n_head_kv * (E / c->n_head);
    char nm[128];
    m->layers = (layer_w*)calloc(c->n_layer ? c->n_layer : 1, sizeof(layer_w));
    for (uint32_t l = 0; l < c->n_layer; ++l) {
        layer_w* lw = &m->layers[l];
#define NM(s) (snprintf(nm, sizeof nm, "blk.%u." s, l), nm)
        if (bind_norm(m->g, NM("attn_norm.weight"), E, &lw->attn_norm)) return -1;
        if (bind(m->g, NM("attn_q.weight"), E, E, &lw->q)) return -1;
        if (bind(m->g, NM("attn_k.weight"), KV, E, &lw->k)) return -1;
        if (bind(m->g, NM("attn_v.weight"), KV, E, &lw->v)) return -1;
        if (bind(m->g, NM("attn_output.weight"), E, E, &lw->o)) return -1;
        if (bind_norm(m->g, NM("ffn_norm.weight"), E, &lw->ffn_norm)) return -1;
        if (bind(m->g, NM("ffn_gate.weight"), F, E, &lw->gate)) return -1;
        if (bind(m->g, NM("ffn_up.weight"), F, E, &lw->up)) return -1;
        if (bind(m->g, NM("ffn_down.weight"), E, F, &lw->down)) return -1;
#undef NM
    }
    if (bind(m->g, "token_embd.weight", V, E, &m->token_embd)) return -1;
    if (bind_norm(m->g, "output_norm.weight", E, &m->output_norm)) return -1;
    if (bind(m->g, "output.weight", V, E, &m->output)) return -1;
    m->kc = (float**)calloc(c->n_layer + 1, sizeof(float*));
    m->vc = (float**)calloc(c->n_layer + 1, sizeof(float*));
    m->klen = (size_t*)calloc(c->n_layer + 1, sizeof(size_t));
    m->kcap = (size_t*)calloc(c->n_layer + 1, sizeof(size_t));
    kv_alloc(m);
    return 0;
}

void oracle_model_free(oracle_model* m) {
    if (!m) return;
    if (m->kc)
        for (uint32_t l = 0; l < m->cfg.n_layer; ++l) {
            free(m->kc[l]);
            free(m->vc[l]);
        }
    free(m->kc);
    free(m->vc);
    free(m->klen);
    free(m->kcap);
    free(m->layers);
    gguf_release(m->g);
    free(m);
}

int oracle_model_open(const char* path, oracle_model** out) {
    oracle_model* m = (oracle_model*)calloc(1, sizeof *m);
    if (oracle_gguf_open(path, &m->g) || model_init(m)) {
        oracle_model_free(m);
        return -1;
    }
    *out = m;
    return 0;
}
int oracle_model_from_bytes(const uint8_t* bytes, size_t len, oracle_model** out) {
    oracle_model* m = (oracle_model*)calloc(1, sizeof *m);
    if (oracle_gguf_from_bytes(bytes, len, &m->g) || model_init(m)) {
        oracle_model_free(m);
        return -1;
    }
    *out = m;
    return 0;
}
int oracle_model_config(const oracle_model* m, oracle_config* out) {
    *out = m->cfg;
    return 0;
}
/* llama.rs:69-81 */
void oracle_model_cap_context(oracle_model* m, size_t max_ctx) {
    size_t cap = max_ctx > 1 ? max_ctx : 1;
    if (cap < m->cfg.context_length) m->cfg.context_length = (uint32_t)cap;
    kv_alloc(m);
}
/* llama.rs:236-238 -> kv_cache.rs:48-52 */
void oracle_model_reset(oracle_model* m) {
    for (uint32_t l = 0; l < m->cfg.n_layer; ++l) m->klen[l] = 0;
}

/* weights.rs:47-55 */
static int qt_matvec(const qtensor* t, const float* x, float* out) {
    return oracle_matvec_quant(t->bytes, t->type, x, out, t->rows, t->cols);
}

/* kv_cache.rs:21-26 (grows past the reserved capacity like Vec::extend_from_slice). */
static void kv_append(oracle_model* m, size_t l, const float* k, const float* v, size_t row) {
    if (m->klen[l] == m->kcap[l]) {
        m->kcap[l] *= 2;
        m->kc[l] = (float*)realloc(m->kc[l], sizeof(float) * m->kcap[l] * row);
        m->vc[l] = (float*)realloc(m->vc[l], sizeof(float) * m->kcap[l] * row);
    }
    float* kd = m->kc[l] + m->klen[l] * row;
    float* vd = m->vc[l] + m->klen[l] * row;
    if (m->kv_f16) {
        /* the values an f16 cache holds, widened back (round to nearest, ties to even) */
        for (size_t i = 0; i < row; ++i) {
            kd[i] = oracle_f16_to_f32(oracle_f32_to_f16(k[i]));
            vd[i] = oracle_f16_to_f32(oracle_f32_to_f16(v[i]));
        }
    } else {
        memcpy(kd, k, sizeof(float) * row);
        memcpy(vd, v, sizeof(float) * row);
    }
    m->klen[l]++;
}

/* Not in the reference: the CUDA path's opt-in f16 KV cache, for its parity tests.
 * Empties the cache. */
void oracle_model_set_kv_f16(oracle_model* m, int on) {
    m->kv_f16 = on != 0;
    oracle_model_reset(m);
}

/* llama.rs:96-183 */
int oracle_forward_hidden(oracle_model* m, uint32_t token, size_t pos, float* xf) {
    const oracle_config* cfg = &m->cfg;
    size_t c = cfg->n_embd, nh = cfg->n_head, nkv = cfg->n_head_kv;
    size_t hd = c / nh, kv_dim = nkv * hd, group = nh / nkv, f = cfg->n_ff;
    float eps = cfg->rms_eps;
    float scale = 1.0f / sqrtf((float)hd);
    if (token >= cfg->vocab_size) return fail("token %u out of range (vocab %u)", token, cfg->vocab_size);

    float* x = (float*)calloc(c, sizeof(float));
    float* normed = (float*)calloc(c, sizeof(float));
    float* q = (float*)calloc(c, sizeof(float));
    float* k = (float*)calloc(kv_dim ? kv_dim : 1, sizeof(float));
    float* v = (float*)calloc(kv_dim ? kv_dim : 1, sizeof(float));
    float* atty = (float*)calloc(c, sizeof(float));
    float* attproj = (float*)calloc(c, sizeof(float));
    float* gate = (float*)calloc(f ? f : 1, sizeof(float));
    float* up = (float*)calloc(f ? f : 1, sizeof(float));
    float* glu = (float*)calloc(f ? f : 1, sizeof(float));
    float* down = (float*)calloc(c, sizeof(float));
    float* scores = NULL;

    /* weights.rs:58-62: embedding row dequant */
    {
        const qtensor* te = &m->token_embd;
        size_t rb = (te->cols / oracle_block_elems(te->type)) * oracle_block_bytes(te->type);
        oracle_dequant(te->type, te->bytes + (size_t)token * rb, te->cols, x);
    }
    int rc = 0;
    for (size_t l = 0; l < cfg->n_layer && rc == 0; ++l) {
        const layer_w* lw = &m->layers[l];
        oracle_rmsnorm(x, lw->attn_norm, eps, normed, c);
        rc |= qt_matvec(&lw->q, normed, q);
        rc |= qt_matvec(&lw->k, normed, k);
        rc |= qt_matvec(&lw->v, normed, v);
        oracle_rope(q, pos, nh, hd, cfg->rope_freq_base);
        oracle_rope(k, pos, nkv, hd, cfg->rope_freq_base);
        kv_append(m, l, k, v, kv_dim);
        const float* keys = m->kc[l];
        const float* vals = m->vc[l];
        size_t seq = m->klen[0];
        scores = (float*)realloc(scores, sizeof(float) * (seq ? seq : 1));
        memset(atty, 0, sizeof(float) * c);
        for (size_t h = 0; h < nh; ++h) {
            size_t kvh = h / group;
            const float* qh = q + h * hd;
            for (size_t t = 0; t < seq; ++t) {
                const float* kh = keys + t * kv_dim + kvh * hd;
                float dot = 0.0f;
                for (size_t i = 0; i < hd; ++i) dot += qh[i] * kh[i];
                scores[t] = dot * scale;
            }
            oracle_softmax(scores, seq);
            float* oh = atty + h * hd;
            for (size_t t = 0; t < seq; ++t) {
                const float* vh = vals + t * kv_dim + kvh * hd;
                float a = scores[t];
                for (size_t i = 0; i < hd; ++i) oh[i] += a * vh[i];
            }
        }
        rc |= qt_matvec(&lw->o, atty, attproj);
        for (size_t i = 0; i < c; ++i) x[i] += attproj[i];
        oracle_rmsnorm(x, lw->ffn_norm, eps, normed, c);
        rc |= qt_matvec(&lw->gate, normed, gate);
        rc |= qt_matvec(&lw->up, normed, up);
        oracle_swiglu(gate, up, glu, f);
        rc |= qt_matvec(&lw->down, glu, down);
        for (size_t i = 0; i < c; ++i) x[i] += down[i];
    }
    if (rc == 0) oracle_rmsnorm(x, m->output_norm, eps, xf, c);
    free(x); free(normed); free(q); free(k); free(v); free(atty); free(attproj);
    free(gate); free(up); free(glu); free(down); free(scores);
    return rc ? -1 : 0;
}

/* llama.rs:85-91 */
int oracle_forward(oracle_model* m, uint32_t token, size_t pos, float* logits) {
    float* xf = (float*)malloc(sizeof(float) * m->cfg.n_embd);
    int rc = oracle_forward_hidden(m, token, pos, xf);
    if (rc == 0) rc = qt_matvec(&m->output, xf, logits);
    free(xf);
    return rc;
}
