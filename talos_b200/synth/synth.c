/*
 * synth.c -- seeded synthetic weights for the Talos benchmark and test models.
 *
 * Stands in for the external trainer/exporter (Hephaistos) that produces the
 * reference's models: it draws N(0, sigma) weights and quantizes them with the
 * quantizers the reference itself uses in its tests:
 *   Q8_0: src/math/metal/mod.rs:551-560 (d = amax/127, q = round(v/d))
 *   Q4_0: src/math/metal/mod.rs:563-574 (d = max/-8, q = clamp(trunc(v/d + 8.5)))
 *   Q6_K: no quantizer exists in the reference; this one follows the block layout
 *         src/gguf/dtype.rs:93-119 decodes (sub-block scale = max/-32, int8 scales
 *         against d = max|scale|/127, q = clamp(round(v/(d*sc)), -32, 31)).
 *
 * Random numbers: element i of a tensor is a function of (seed, stream, i) only,
 * so the bytes do not depend on the thread count or on generation order.
 *   key   = splitmix64(seed ^ splitmix64(stream))
 *   pair p = i / 2: a = splitmix64(key + 2p), b = splitmix64(key + 2p + 1)
 *   u1 = ((a >> 11) + 1) / 2^53 in (0, 1],  u2 = (b >> 11) / 2^53 in [0, 1)
 *   Box-Muller in double: r = sqrt(-2 ln u1); z = r cos(2 pi u2) (even i),
 *   r sin(2 pi u2) (odd i); value = (float)(sigma * z).
 * SplitMix64 is Steele, Lea & Flood (2014); Box-Muller is Box & Muller (1958).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint64_t synth_stream_of(const char* name) {
    uint64_t h = 0xcbf29ce484222325ull; /* FNV-1a 64 */
    for (const unsigned char* p = (const unsigned char*)name; *p; ++p) {
        h ^= *p;
        h *= 0x100000001b3ull;
    }
    return h;
}

void synth_fill_normal(uint64_t seed, uint64_t stream, uint64_t start, uint64_t n, float sigma, float* out) {
    uint64_t key = splitmix64(seed ^ splitmix64(stream));
    const double two_pi = 6.283185307179586476925286766559;
    uint64_t i = start, end = start + n;
    while (i < end) {
        uint64_t p = i >> 1;
        uint64_t a = splitmix64(key + 2 * p), b = splitmix64(key + 2 * p + 1);
        double u1 = (double)((a >> 11) + 1) * (1.0 / 9007199254740992.0);
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        double ang = two_pi * u2;
        if ((i & 1) == 0) {
            out[i - start] = (float)(sigma * (r * cos(ang)));
            if (i + 1 < end) out[i + 1 - start] = (float)(sigma * (r * sin(ang)));
            i += 2;
        } else {
            out[i - start] = (float)(sigma * (r * sin(ang)));
            i += 1;
        }
    }
}

/* ---------------------------------------------------------------- f16 */

static uint16_t f32_to_f16(float f) { /* round to nearest even, like half::f16::from_f32 */
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xFFu, man = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t half = 1u << (shift - 1), rem = man & ((1u << shift) - 1u), res = man >> shift;
        if (rem > half || (rem == half && (res & 1u))) res++;
        return (uint16_t)(sign | res);
    }
    uint32_t res = ((uint32_t)e << 10) | (man >> 13), rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (res & 1u))) res++;
    return (uint16_t)(sign | res);
}

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (!man) {
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
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ---------------------------------------------------------------- quantizers */

static void q8_0(const float* v, uint8_t* o) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    float d = amax / 127.0f;
    uint16_t dh = f32_to_f16(d);
    o[0] = (uint8_t)dh;
    o[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
        float q = 0.0f;
        if (d != 0.0f) {
            q = roundf(v[i] / d);
            q = q < -128.0f ? -128.0f : (q > 127.0f ? 127.0f : q);
        }
        o[2 + i] = (uint8_t)(int8_t)q;
    }
}

static int32_t as_i32(float f) { /* Rust `as i32`: truncating, saturating, NaN -> 0 */
    if (f != f) return 0;
    if (f >= 2147483647.0f) return 2147483647;
    if (f <= -2147483648.0f) return -2147483647 - 1;
    return (int32_t)f;
}

static void q4_0(const float* v, uint8_t* o) {
    float mx = 0.0f;
    for (int i = 0; i < 32; ++i)
        if (fabsf(v[i]) > fabsf(mx)) mx = v[i];
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = f32_to_f16(d);
    o[0] = (uint8_t)dh;
    o[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 16; ++j) {
        int32_t a = as_i32(v[j] * id + 8.5f), b = as_i32(v[j + 16] * id + 8.5f);
        a = a < 0 ? 0 : (a > 15 ? 15 : a);
        b = b < 0 ? 0 : (b > 15 ? 15 : b);
        o[2 + j] = (uint8_t)(a | (b << 4));
    }
}

static void q6_k(const float* v, uint8_t* o) {
    float sub[16], smax = 0.0f;
    for (int s = 0; s < 16; ++s) {
        float mx = 0.0f;
        for (int i = 0; i < 16; ++i)
            if (fabsf(v[s * 16 + i]) > fabsf(mx)) mx = v[s * 16 + i];
        sub[s] = mx / -32.0f;
        if (fabsf(sub[s]) > smax) smax = fabsf(sub[s]);
    }
    float d = smax / 127.0f;
    uint16_t dh = f32_to_f16(d);
    float dq = f16_to_f32(dh);
    int8_t sc[16];
    for (int s = 0; s < 16; ++s) {
        float r = dq != 0.0f ? roundf(sub[s] / dq) : 0.0f;
        r = r > 127.0f ? 127.0f : (r < -128.0f ? -128.0f : r);
        sc[s] = (int8_t)r;
    }
    uint8_t q[256];
    for (int i = 0; i < 256; ++i) {
        float step = dq * (float)sc[i / 16];
        float r = step != 0.0f ? roundf(v[i] / step) : 0.0f;
        r = r > 31.0f ? 31.0f : (r < -32.0f ? -32.0f : r);
        q[i] = (uint8_t)((int)r + 32);
    }
    memset(o, 0, 210);
    uint8_t *ql = o, *qh = o + 128;
    for (int nh = 0; nh < 2; ++nh) {
        const uint8_t* qq = q + nh * 128;
        for (int l = 0; l < 32; ++l) {
            ql[nh * 64 + l] = (uint8_t)((qq[l] & 0xF) | ((qq[l + 64] & 0xF) << 4));
            ql[nh * 64 + l + 32] = (uint8_t)((qq[l + 32] & 0xF) | ((qq[l + 96] & 0xF) << 4));
            qh[nh * 32 + l] = (uint8_t)((qq[l] >> 4) | ((qq[l + 32] >> 4) << 2) | ((qq[l + 64] >> 4) << 4) |
                                        ((qq[l + 96] >> 4) << 6));
        }
    }
    for (int s = 0; s < 16; ++s) o[192 + s] = (uint8_t)sc[s];
    o[208] = (uint8_t)dh;
    o[209] = (uint8_t)(dh >> 8);
}

static int bel(int t) { return t == 0 ? 1 : t == 14 ? 256 : (t == 2 || t == 8) ? 32 : 0; }
static int bby(int t) { return t == 0 ? 4 : t == 14 ? 210 : t == 2 ? 18 : t == 8 ? 34 : 0; }

/* Quantize n floats (multiple of the block size) of `type` into out. */
int synth_quantize(int type, const float* x, uint64_t n, uint8_t* out) {
    int be = bel(type), bb = bby(type);
    if (!be || n % be) return -1;
    for (uint64_t b = 0; b < n / be; ++b) {
        const float* v = x + b * be;
        uint8_t* o = out + b * bb;
        switch (type) {
            case 0: memcpy(o, v, 4); break;
            case 8: q8_0(v, o); break;
            case 2: q4_0(v, o); break;
            case 14: q6_k(v, o); break;
        }
    }
    return 0;
}

typedef struct {
    uint64_t seed, stream, rows, cols, r0, r1;
    int type;
    float sigma;
    uint8_t* out;
} job_t;

static void* run_job(void* p) {
    job_t* j = (job_t*)p;
    uint64_t rb = j->cols / bel(j->type) * bby(j->type);
    float* buf = (float*)malloc(sizeof(float) * j->cols);
    for (uint64_t r = j->r0; r < j->r1; ++r) {
        synth_fill_normal(j->seed, j->stream, r * j->cols, j->cols, j->sigma, buf);
        synth_quantize(j->type, buf, j->cols, j->out + r * rb);
    }
    free(buf);
    return NULL;
}

/* Generate a [rows, cols] N(0, sigma) tensor of `type` (raw GGUF bytes) into out. */
int synth_tensor(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, int type, float sigma,
                 uint8_t* out, int nthreads) {
    int be = bel(type);
    if (!be || cols % be) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((uint64_t)nthreads > rows) nthreads = rows ? (int)rows : 1;
    pthread_t th[256];
    job_t jobs[256];
    uint64_t per = (rows + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; ++t) {
        uint64_t r0 = t * per, r1 = r0 + per;
        if (r1 > rows) r1 = rows;
        if (r0 > rows) r0 = rows;
        jobs[t] = (job_t){seed, stream, rows, cols, r0, r1, type, sigma, out};
        pthread_create(&th[t], NULL, run_job, &jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* n token ids uniform in [0, vocab): splitmix64(key + i) mod vocab (the modulo
 * bias is below 2^-40 for vocab < 2^24). */
void synth_token_ids(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t* out) {
    uint64_t key = splitmix64(seed ^ splitmix64(stream));
    for (uint64_t i = 0; i < n; ++i) out[i] = (uint32_t)(splitmix64(key + i) % (vocab ? vocab : 1));
}
