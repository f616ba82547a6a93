// kernels.cu -- the Talos decode kernels for B200 (sm_100a).
//
// Reference algorithm (Tsuskov/talos, Rust): src/model/llama.rs:96-183 and the
// kernels it calls in src/math/{ops,matmul,quant}.rs and src/gguf/dtype.rs.
// Built without --use_fast_math: expf / division / sqrt are the accurate CUDA
// forms, and the few places that must round like the reference use explicit
// __fmul_rn / __fadd_rn.
#include <math.h>

#include "kernels.cuh"

namespace talos {

static inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// =====================================================================
// Dequantization (bit-exact with src/gguf/dtype.rs:64-121)
// =====================================================================

__device__ __forceinline__ float ld_half_bytes(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// Element `i` of a tensor stored as raw GGUF blocks.
__device__ __forceinline__ float dequant_elem(int type, const uint8_t* raw, size_t i) {
    switch (type) {
        case GT_F32: {
            const uint8_t* p = raw + 4 * i;
            uint32_t b = p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24);
            return __uint_as_float(b);
        }
        case GT_Q8_0: {  // dtype.rs:69-78
            const uint8_t* b = raw + (i / 32) * 34;
            return __fmul_rn(ld_half_bytes(b), (float)(int8_t)b[2 + i % 32]);
        }
        case GT_Q4_0: {  // dtype.rs:79-91
            const uint8_t* b = raw + (i / 32) * 18;
            int j = (int)(i % 32);
            int q = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
            return __fmul_rn(ld_half_bytes(b), (float)(q - 8));
        }
        case GT_Q6_K: {  // dtype.rs:93-119, y = (d * sc) * q
            const uint8_t* b = raw + (i / 256) * 210;
            int e = (int)(i % 256);
            int n = e / 128, r = e % 128;
            int l = r % 32, j = r / 32;  // element l + 32 j of half n
            const uint8_t* ql = b + n * 64;
            const uint8_t* qh = b + 128 + n * 32;
            const int8_t* sc = (const int8_t*)(b + 192 + n * 8);
            int lo = (j & 1) ? ql[l + 32] : ql[l];
            lo = (j & 2) ? (lo >> 4) : (lo & 0xF);
            int hi = (qh[l] >> (2 * j)) & 3;
            int q = (lo | (hi << 4)) - 32;
            float d = ld_half_bytes(b + 208);
            return __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * j]), (float)q);
        }
    }
    return 0.f;
}

__global__ void k_dequant(int type, const uint8_t* raw, size_t n, float* out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = dequant_elem(type, raw, i);
}

cudaError_t launch_dequant(int type, const uint8_t* raw, size_t n, float* out, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_dequant<<<(unsigned)blocks, 256, 0, s>>>(type, raw, n, out);
    return cudaGetLastError();
}

// =====================================================================
// Weight repacking (lossless; runs once per tensor at upload)
// =====================================================================

bool pack_sizes(int type, int rows, int cols, PackSizes* o) {
    *o = PackSizes{};
    o->rows_pad = ceil_div(rows, 16) * 16;
    size_t R = (size_t)o->rows_pad;
    switch (type) {
        case GT_F32:
            o->nk = cols;
            o->b0 = R * cols * 4;
            return true;
        case GT_Q8_0:
            if (cols % 32) return false;
            o->nk = cols / 32;
            o->b0 = R * o->nk * 32;
            o->b1 = R * o->nk * 2;
            return true;
        case GT_Q4_0:
            if (cols % 32) return false;
            o->nk = ceil_div(cols / 32, 4);  // block quads
            o->b0 = (R / 8) * o->nk * 32 * 16;
            o->b1 = (R / 8) * o->nk * 8 * 8;
            return true;
        case GT_Q6_K:
            if (cols % 256) return false;
            o->nk = cols / 256;
            o->b0 = R * o->nk * 32 * 4;
            o->b1 = R * o->nk * 32 * 2;
            o->b2 = R * o->nk * 16;
            o->b3 = R * o->nk * 2;
            return true;
    }
    return false;
}

__global__ void k_pack_f32(const uint8_t* raw, PackedW w) {
    size_t n = (size_t)w.rows_pad * w.cols;
    float* dst = (float*)w.p0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / w.cols;
        float v = 0.f;
        if (r < (size_t)w.rows) {
            const uint8_t* p = raw + 4 * i;
            v = __uint_as_float(p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24));
        }
        dst[i] = v;
    }
}

// One thread per (row, block).
__global__ void k_pack_q8_0(const uint8_t* raw, PackedW w) {
    size_t nb = (size_t)w.nk;
    size_t n = (size_t)w.rows_pad * nb;
    int8_t* qs = (int8_t*)w.p0;
    uint16_t* d = (uint16_t*)w.p1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / nb;
        if (r < (size_t)w.rows) {
            const uint8_t* b = raw + i * 34;
            d[i] = (uint16_t)(b[0] | (b[1] << 8));
            for (int k = 0; k < 32; ++k) qs[i * 32 + k] = (int8_t)b[2 + k];
        } else {
            d[i] = 0;
            for (int k = 0; k < 32; ++k) qs[i * 32 + k] = 0;
        }
    }
}

// Q4_0 -> MMA fragment order. For row r (group g = r/8), block b (quad q = b/4,
// slot j = b%4) and k-lane t (0..3, k0 = 2t), lane L = (r%8)*4 + t holds word j:
//   bits  0-3  q[k0]      bits 16-19 q[k0+1]     (A fragment, k 0-15, cols 2t..2t+1)
//   bits  4-7  q[k0+8]    bits 20-23 q[k0+9]     (A fragment, k 0-15, cols 2t+8..)
//   bits  8-11 q[16+k0]   bits 24-27 q[17+k0]    (same, k 16-31, after >> 8)
//   bits 12-15 q[24+k0]   bits 28-31 q[25+k0]
// where q[e] is the 4-bit quant of element e (dtype.rs:85-89: low nibble of
// byte j is element j, high nibble is element j+16). Pad blocks/rows: q = 8, d = 0.
__global__ void k_pack_q4_0(const uint8_t* raw, PackedW w) {
    size_t nb_src = (size_t)(w.cols / 32);
    size_t nb_pad = (size_t)w.nk * 4;
    size_t n = (size_t)w.rows_pad * nb_pad;
    uint32_t* qs = (uint32_t*)w.p0;
    uint16_t* sc = (uint16_t*)w.p1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / nb_pad, b = i % nb_pad;
        size_t g = r / 8, q = b / 4, j = b % 4;
        uint8_t bytes[16];
        uint16_t dbits = 0;
        if (r < (size_t)w.rows && b < nb_src) {
            const uint8_t* blk = raw + (r * nb_src + b) * 18;
            dbits = (uint16_t)(blk[0] | (blk[1] << 8));
            for (int k = 0; k < 16; ++k) bytes[k] = blk[2 + k];
        } else {
            for (int k = 0; k < 16; ++k) bytes[k] = 0x88;
        }
        sc[((g * w.nk + q) * 8 + (r % 8)) * 4 + j] = dbits;
        for (int t = 0; t < 4; ++t) {
            int k0 = 2 * t;
            uint32_t b0 = (bytes[k0] & 0xF) | ((bytes[k0 + 8] & 0xF) << 4);
            uint32_t b1 = (bytes[k0] >> 4) | ((bytes[k0 + 8] >> 4) << 4);
            uint32_t b2 = (bytes[k0 + 1] & 0xF) | ((bytes[k0 + 9] & 0xF) << 4);
            uint32_t b3 = (bytes[k0 + 1] >> 4) | ((bytes[k0 + 9] >> 4) << 4);
            size_t lane = (r % 8) * 4 + t;
            qs[((g * w.nk + q) * 32 + lane) * 4 + j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
    }
}

// Q6_K -> per-lane words. One thread per (row, super-block, lane).
__global__ void k_pack_q6_k(const uint8_t* raw, PackedW w) {
    size_t nsb = (size_t)w.nk;
    size_t n = (size_t)w.rows_pad * nsb * 32;
    uint32_t* qlp = (uint32_t*)w.p0;
    uint16_t* qhp = (uint16_t*)w.p1;
    int8_t* sc = (int8_t*)w.p2;
    uint16_t* d = (uint16_t*)w.p3;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t rs = i / 32;  // row * nsb + s
        int l = (int)(i % 32);
        size_t r = rs / nsb;
        if (r < (size_t)w.rows) {
            const uint8_t* b = raw + rs * 210;
            const uint8_t* ql = b;
            const uint8_t* qh = b + 128;
            qlp[i] = ql[l] | (ql[l + 32] << 8) | (ql[64 + l] << 16) | ((uint32_t)ql[96 + l] << 24);
            qhp[i] = (uint16_t)(qh[l] | (qh[32 + l] << 8));
            if (l < 16) sc[rs * 16 + l] = (int8_t)b[192 + l];
            if (l == 0) d[rs] = (uint16_t)(b[208] | (b[209] << 8));
        } else {
            qlp[i] = 0;
            qhp[i] = 0;
            if (l < 16) sc[rs * 16 + l] = 0;
            if (l == 0) d[rs] = 0;
        }
    }
}

cudaError_t launch_pack(const uint8_t* raw, const PackedW& w, cudaStream_t s) {
    const int T = 256;
    const unsigned G = 148 * 16;
    switch (w.type) {
        case GT_F32: k_pack_f32<<<G, T, 0, s>>>(raw, w); break;
        case GT_Q8_0: k_pack_q8_0<<<G, T, 0, s>>>(raw, w); break;
        case GT_Q4_0: k_pack_q4_0<<<G, T, 0, s>>>(raw, w); break;
        case GT_Q6_K: k_pack_q6_k<<<G, T, 0, s>>>(raw, w); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// =====================================================================
// Fused dequant-matvec (+ RMSNorm prologue, + epilogues)
// =====================================================================
//
// One CTA of 8 warps stages the (optionally RMS-normalised) input vector in
// shared memory once, then walks 16-row tiles (t = blockIdx.x, += gridDim.x).
// Each tile's 16 results land in shared memory and the epilogue of the launch
// consumes them: store, residual add (src/model/llama.rs:159-161,174-176),
// SwiGLU of interleaved gate/up rows (src/math/ops.rs:28-37), q/k RoPE with the
// KV-cache append (src/math/ops.rs:48-61, src/kv_cache.rs:21-26), or logits with
// a running argmax (src/sample.rs:7-14).
//
// Q4_0 computes on the tensor cores with mma.sync m16n8k16: the 4-bit quants are
// turned into exact f16 (q - 8) values in registers, the activation is split
// into f16 hi + lo parts (x = hi + lo to ~22 bits) that form B columns 0 and 1,
// and each 32-wide block's f32 sum is scaled by its f16 d on the CUDA cores:
//   y[r] = sum_b d[r,b] * sum_{k in b} (q[r,k] - 8) * (hi[k] + lo[k]).
// F32, Q8_0 and Q6_K use CUDA-core FMAs with one warp per two rows.

constexpr int MV_THREADS = 256;
constexpr int MV_WARPS = MV_THREADS / 32;

__device__ __forceinline__ float silu_ref(float g) {
    // src/math/ops.rs:28-30: x / (1 + exp(-x))
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}

// Stage layout for Q4_0: per 32-element block, 8 lanes x uint4 =
// {step0 reg0, step0 reg1, step1 reg0, step1 reg1}; lanes 0-3 carry the hi part,
// lanes 4-7 the lo part; reg0 = x[2t, 2t+1], reg1 = x[2t+8, 2t+9] (+16 for step 1).
__device__ __forceinline__ void split_pair(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
    half l0 = __float2half_rn(v0 - __half2float(h0));
    half l1 = __float2half_rn(v1 - __half2float(h1));
    hi = pack_half2(h0, h1);
    lo = pack_half2(l0, l1);
}

template <int TYPE>
struct MvStage {
    // Padded stage length (elements) for input length K.
    static __host__ __device__ int kpad(int K) {
        if (TYPE == GT_Q4_0) return ((K / 32 + 3) / 4) * 4 * 32;
        return K;
    }
};

// Row r (0..15) of tile lt in segment sg -> (weight, weight row).
__device__ __forceinline__ void tile_row(const Seg& sg, int lt, int r, const PackedW*& W, int& row) {
    if (sg.pair) {
        W = r < 8 ? &sg.A : &sg.B;
        row = 8 * lt + (r & 7);
    } else {
        W = &sg.A;
        row = 16 * lt + r;
    }
}

// ---- per-format tile compute: every warp adds its share into part[warp][16] ----

__device__ __forceinline__ void tile_q4_0(const Seg& sg, int lt, const uint4* xfrag, float* part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const PackedW& WA = sg.A;
    const PackedW& WB = sg.pair ? sg.B : sg.A;
    const int gA = sg.pair ? lt : 2 * lt;
    const int gB = sg.pair ? lt : 2 * lt + 1;
    const int nq = WA.nk;
    const uint4* qA = (const uint4*)WA.p0 + (size_t)gA * nq * 32 + lane;
    const uint4* qB = (const uint4*)WB.p0 + (size_t)gB * nq * 32 + lane;
    const uint2* sA = (const uint2*)WA.p1 + (size_t)gA * nq * 8 + (lane >> 2);
    const uint2* sB = (const uint2*)WB.p1 + (size_t)gB * nq * 8 + (lane >> 2);
    float accA = 0.f, accB = 0.f;
    constexpr int U = 4;
    for (int q0 = warp; q0 < nq; q0 += MV_WARPS * U) {
        uint4 wa[U], wb[U];
        uint2 ca[U], cb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int q = q0 + MV_WARPS * u;
            if (q < nq) {
                wa[u] = ldg_stream_u4(qA + (size_t)q * 32);
                wb[u] = ldg_stream_u4(qB + (size_t)q * 32);
                ca[u] = ldg_stream_u2(sA + (size_t)q * 8);
                cb[u] = ldg_stream_u2(sB + (size_t)q * 8);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int q = q0 + MV_WARPS * u;
            if (q < nq) {
                float2 a01 = __half22float2(*reinterpret_cast<const half2*>(&ca[u].x));
                float2 a23 = __half22float2(*reinterpret_cast<const half2*>(&ca[u].y));
                float2 b01 = __half22float2(*reinterpret_cast<const half2*>(&cb[u].x));
                float2 b23 = __half22float2(*reinterpret_cast<const half2*>(&cb[u].y));
                const float dA[4] = {a01.x, a01.y, a23.x, a23.y};
                const float dB[4] = {b01.x, b01.y, b23.x, b23.y};
                const uint32_t xa[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                const uint32_t xb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint4 bx = make_uint4(0, 0, 0, 0);
                    if (lane < 8) bx = xfrag[(q * 4 + j) * 8 + lane];
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
                    mma_16816(d, q4_lo_f16x2(xa[j]), q4_lo_f16x2(xb[j]), q4_hi_f16x2(xa[j]),
                              q4_hi_f16x2(xb[j]), bx.x, bx.y);
                    uint32_t ya = xa[j] >> 8, yb = xb[j] >> 8;
                    mma_16816(d, q4_lo_f16x2(ya), q4_lo_f16x2(yb), q4_hi_f16x2(ya), q4_hi_f16x2(yb),
                              bx.z, bx.w);
                    accA = fmaf(dA[j], d[0] + d[1], accA);
                    accB = fmaf(dB[j], d[2] + d[3], accB);
                }
            }
        }
    }
    if ((lane & 3) == 0) {
        part[warp * 16 + (lane >> 2)] = accA;
        part[warp * 16 + 8 + (lane >> 2)] = accB;
    }
}

// Row dot products on CUDA cores: warp w computes tile rows 2w and 2w+1.
__device__ __forceinline__ float row_f32(const PackedW& W, int row, const float* xs) {
    const int lane = threadIdx.x & 31;
    const int K = W.cols;
    const float* wr = (const float*)W.p0 + (size_t)row * K;
    float acc = 0.f;
    if ((K & 3) == 0) {
        const float4* w4 = (const float4*)wr;
        const float4* x4 = (const float4*)xs;
#pragma unroll 4
        for (int k = lane; k < K / 4; k += 32) {
            uint4 u = ldg_stream_u4(w4 + k);
            float4 xv = x4[k];
            acc = fmaf(__uint_as_float(u.x), xv.x, acc);
            acc = fmaf(__uint_as_float(u.y), xv.y, acc);
            acc = fmaf(__uint_as_float(u.z), xv.z, acc);
            acc = fmaf(__uint_as_float(u.w), xv.w, acc);
        }
    } else {
        for (int k = lane; k < K; k += 32) acc = fmaf(__ldg(wr + k), xs[k], acc);
    }
    return acc;
}

__device__ __forceinline__ float i8_to_f32(uint32_t w, int k) {
    // byte k of w (signed) -> float, exact: (2^23 + 128 + q) - (2^23 + 128)
    return __int_as_float(__byte_perm(w ^ 0x80808080u, 0x4B000000u, 0x7540 + k)) - 8388736.0f;
}

__device__ __forceinline__ float row_q8_0(const PackedW& W, int row, const float* xs) {
    const int lane = threadIdx.x & 31;
    const int nb = W.nk;
    const uint4* qs = (const uint4*)((const int8_t*)W.p0 + (size_t)row * nb * 32);
    const half* dd = (const half*)W.p1 + (size_t)row * nb;
    float acc = 0.f;
#pragma unroll 2
    for (int c = lane; c < 2 * nb; c += 32) {  // 16-byte chunk c: block c/2, half c%2
        uint4 u = ldg_stream_u4(qs + c);
        const float4* x4 = (const float4*)(xs + 16 * c);
        float s = 0.f;
        const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float4 xv = x4[i];
            s = fmaf(i8_to_f32(wv[i], 0), xv.x, s);
            s = fmaf(i8_to_f32(wv[i], 1), xv.y, s);
            s = fmaf(i8_to_f32(wv[i], 2), xv.z, s);
            s = fmaf(i8_to_f32(wv[i], 3), xv.w, s);
        }
        acc = fmaf(__half2float(dd[c >> 1]), s, acc);
    }
    return acc;
}

__device__ __forceinline__ float row_q6_k(const PackedW& W, int row, const float* xs) {
    const int lane = threadIdx.x & 31;
    const int nsb = W.nk;
    const uint32_t* qlp = (const uint32_t*)W.p0 + (size_t)row * nsb * 32;
    const uint16_t* qhp = (const uint16_t*)W.p1 + (size_t)row * nsb * 32;
    const int8_t* scp = (const int8_t*)W.p2 + (size_t)row * nsb * 16;
    const half* dp = (const half*)W.p3 + (size_t)row * nsb;
    const int is = lane >> 4;  // l / 16
    float acc = 0.f;
    for (int s = 0; s < nsb; ++s) {
        uint32_t w = ldg_stream_u1(qlp + s * 32 + lane);
        uint32_t h = __ldg(qhp + s * 32 + lane);
        uint4 sc4 = __ldg((const uint4*)(scp + s * 16));
        float d = __half2float(dp[s]);
        const int8_t* sc = (const int8_t*)&sc4;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            uint32_t qa = (w >> (16 * n)) & 0xFF, qb = (w >> (16 * n + 8)) & 0xFF;
            uint32_t hb = (h >> (8 * n)) & 0xFF;
            const float* xb = xs + s * 256 + n * 128 + lane;
            uint32_t q1 = (qa & 0xF) | ((hb & 3) << 4);
            uint32_t q2 = (qb & 0xF) | (((hb >> 2) & 3) << 4);
            uint32_t q3 = (qa >> 4) | (((hb >> 4) & 3) << 4);
            uint32_t q4 = (qb >> 4) | (((hb >> 6) & 3) << 4);
            const int so = 8 * n + is;
            // (q - 32) exactly: (2^23 + q) - (2^23 + 32)
            float f1 = __int_as_float(0x4B000000 | q1) - 8388640.0f;
            float f2 = __int_as_float(0x4B000000 | q2) - 8388640.0f;
            float f3 = __int_as_float(0x4B000000 | q3) - 8388640.0f;
            float f4 = __int_as_float(0x4B000000 | q4) - 8388640.0f;
            acc = fmaf(d * (float)sc[so], f1 * xb[0], acc);
            acc = fmaf(d * (float)sc[so + 2], f2 * xb[32], acc);
            acc = fmaf(d * (float)sc[so + 4], f3 * xb[64], acc);
            acc = fmaf(d * (float)sc[so + 6], f4 * xb[96], acc);
        }
    }
    return acc;
}

template <int TYPE>
__device__ __forceinline__ void tile_cuda_core(const Seg& sg, int lt, const float* xs, float* part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        int r = 2 * warp + k;
        const PackedW* W;
        int row;
        tile_row(sg, lt, r, W, row);
        float v;
        if (TYPE == GT_F32)
            v = row_f32(*W, row, xs);
        else if (TYPE == GT_Q8_0)
            v = row_q8_0(*W, row, xs);
        else
            v = row_q6_k(*W, row, xs);
        v = warp_sum(v);
        if (lane == 0) part[r] = v;
    }
}

template <int TYPE>
__global__ void __launch_bounds__(MV_THREADS) k_matvec(const __grid_constant__ MatvecArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int K = a.K;
    const int KP = MvStage<TYPE>::kpad(K);
    float* stage = (float*)smem;                 // KP floats (Q4_0: fragments, same bytes)
    float* part = stage + KP;                    // MV_WARPS * 16
    float* res = part + MV_WARPS * 16;           // 16
    float* red = res + 16;                       // 32

    // ---- prologue: RMSNorm scale (src/math/ops.rs:5-12) ----
    float scale = 1.f;
    if (a.norm_w) {
        float ss = 0.f;
        for (int k = tid; k < K; k += MV_THREADS) {
            float v = a.x[k];
            ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid < 32) {
            float v = tid < MV_WARPS ? red[tid] : 0.f;
            v = warp_sum(v);
            if (tid == 0) red[0] = v;
        }
        __syncthreads();
        scale = 1.0f / sqrtf(red[0] / (float)K + a.eps);
    }
    // ---- stage x (normed: (x * scale) * w, the reference's rounding order) ----
    if (TYPE == GT_Q4_0) {
        uint4* xf = (uint4*)stage;
        const int nblk = KP / 32;
        for (int idx = tid; idx < nblk * 8; idx += MV_THREADS) {
            int j = idx >> 3, l8 = idx & 7, t = l8 & 3;
            uint32_t r[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                int e = 32 * j + 16 * (m >> 1) + 2 * t + 8 * (m & 1);
                float v0 = 0.f, v1 = 0.f;
                if (e < K) {
                    v0 = a.x[e];
                    v1 = a.x[e + 1];
                    if (a.norm_w) {
                        v0 = __fmul_rn(__fmul_rn(v0, scale), a.norm_w[e]);
                        v1 = __fmul_rn(__fmul_rn(v1, scale), a.norm_w[e + 1]);
                    }
                }
                uint32_t hi, lo;
                split_pair(v0, v1, hi, lo);
                r[m] = l8 < 4 ? hi : lo;
            }
            xf[idx] = make_uint4(r[0], r[1], r[2], r[3]);
        }
    } else {
        for (int k = tid; k < KP; k += MV_THREADS) {
            float v = a.x[k];
            if (a.norm_w) v = __fmul_rn(__fmul_rn(v, scale), a.norm_w[k]);
            stage[k] = v;
        }
    }
    __syncthreads();

    const uint32_t pos = a.step ? a.step->pos : 0u;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x) {
        int si = 0, lt = t;
        while (si + 1 < a.nseg && lt >= a.seg[si].ntiles) {
            lt -= a.seg[si].ntiles;
            ++si;
        }
        const Seg& sg = a.seg[si];
        if (TYPE == GT_Q4_0) {
            tile_q4_0(sg, lt, (const uint4*)stage, part);
            __syncthreads();
            if (tid < 16) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < MV_WARPS; ++w) v += part[w * 16 + tid];
                res[tid] = v;
            }
        } else {
            tile_cuda_core<TYPE>(sg, lt, stage, res);
        }
        __syncthreads();

        // ---- epilogue ----
        if (a.epi == EPI_SWIGLU) {
            if (tid < 8) {
                int j = 8 * lt + tid;
                if (j < sg.out_rows) sg.out[j] = __fmul_rn(silu_ref(res[tid]), res[8 + tid]);
            }
        } else if (a.epi == EPI_QKV) {
            if (sg.role == 2) {
                if (tid < 16) {
                    int r = 16 * lt + tid;
                    if (r < sg.out_rows) a.vcache[(size_t)pos * a.kv_dim + r] = res[tid];
                }
            } else if (tid < 8) {
                int r0 = 16 * lt + 2 * tid;
                if (r0 < sg.out_rows) {
                    int i = (r0 % a.hd) >> 1;
                    float2 cs = a.rope_cs[(size_t)pos * (a.hd >> 1) + i];
                    float x0 = res[2 * tid], x1 = res[2 * tid + 1];
                    // src/math/ops.rs:57-58: a*cos - b*sin, a*sin + b*cos (no FMA)
                    float o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
                    float o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
                    float* dst = sg.role == 0 ? sg.out + r0 : a.kcache + (size_t)pos * a.kv_dim + r0;
                    dst[0] = o0;
                    dst[1] = o1;
                }
            }
        } else {
            if (tid < 16) {
                int r = 16 * lt + tid;
                if (r < sg.out_rows) {
                    float v = res[tid];
                    if (a.epi == EPI_ADD)
                        sg.out[r] = __fadd_rn(sg.out[r], v);
                    else
                        sg.out[r] = v;
                }
            }
            if (a.epi == EPI_LOGITS && tid < 32) {
                unsigned long long key = 0ull;
                if (tid < 16) {
                    int r = 16 * lt + tid;
                    if (r < sg.out_rows)
                        key = ((unsigned long long)total_order_key(res[tid]) << 32) | (unsigned)r;
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) {
                    unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                    key = other > key ? other : key;
                }
                if (tid == 0 && key) atomicMax(&a.step->argmax_key, key);
            }
        }
        __syncthreads();
    }
}

size_t matvec_smem_bytes(int type, int K) {
    int KP = type == GT_Q4_0 ? MvStage<GT_Q4_0>::kpad(K) : K;
    return (size_t)KP * 4 + (MV_WARPS * 16 + 16 + 32) * 4;
}

template <int TYPE>
static void* mv_kernel() {
    return (void*)k_matvec<TYPE>;
}

cudaError_t matvec_configure() {
    const int big = 200 * 1024;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, big))) return e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, big))) return e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, big))) return e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, big))) return e;
    return cudaSuccess;
}

int matvec_ctas_per_sm(int type, int K) {
    int n = 0;
    size_t sm = matvec_smem_bytes(type, K);
    void* f = type == GT_F32 ? mv_kernel<GT_F32>() : type == GT_Q8_0 ? mv_kernel<GT_Q8_0>()
            : type == GT_Q4_0 ? mv_kernel<GT_Q4_0>() : mv_kernel<GT_Q6_K>();
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, f, MV_THREADS, sm) != cudaSuccess) return 1;
    return n > 0 ? n : 1;
}

cudaError_t launch_matvec(const MatvecArgs& a, int type, int max_ctas, cudaStream_t s) {
    if (a.ntiles <= 0) return cudaSuccess;
    int grid = a.ntiles < max_ctas ? a.ntiles : max_ctas;
    size_t sm = matvec_smem_bytes(type, a.K);
    switch (type) {
        case GT_F32: k_matvec<GT_F32><<<grid, MV_THREADS, sm, s>>>(a); break;
        case GT_Q8_0: k_matvec<GT_Q8_0><<<grid, MV_THREADS, sm, s>>>(a); break;
        case GT_Q4_0: k_matvec<GT_Q4_0><<<grid, MV_THREADS, sm, s>>>(a); break;
        case GT_Q6_K: k_matvec<GT_Q6_K><<<grid, MV_THREADS, sm, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// =====================================================================
// Decode attention: split over positions, online softmax, fixed-order combine
// =====================================================================
//
// src/model/llama.rs:135-155: for query head h (kv head h/group), scores over
// the cached positions, softmax (src/math/ops.rs:15-25), weighted sum of V.
// CTA (kvh, s) takes positions [s*chunk, (s+1)*chunk) for all `group` query
// heads that share kv head kvh, so each K/V row is read once. The last CTA of a
// kv head (arrival counter) merges the splits in split order, which keeps the
// result independent of scheduling.

constexpr int AT_WARPS = 4;
constexpr int AT_MAXG = 8;   // query heads per kv head
constexpr int AT_MAXD = 8;   // head_dim / 32

__global__ void __launch_bounds__(AT_WARPS * 32) k_attention(const __grid_constant__ AttnArgs a) {
    __shared__ float sm_m[AT_WARPS][AT_MAXG], sm_l[AT_WARPS][AT_MAXG];
    __shared__ float sm_o[AT_WARPS][AT_MAXG][AT_MAXD * 32];
    __shared__ unsigned sm_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kvh = blockIdx.x, s = blockIdx.y;
    const int group = a.n_head / a.n_kv;
    const int hd = a.hd;
    const int seq = (int)a.step->pos + 1;
    const int chunk = (seq + a.nsplit - 1) / a.nsplit;
    const int t0 = s * chunk;
    const int t1 = min(seq, t0 + chunk);

    float qv[AT_MAXG][AT_MAXD];
    float o[AT_MAXG][AT_MAXD];
    float m[AT_MAXG], l[AT_MAXG];
#pragma unroll
    for (int g = 0; g < AT_MAXG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int i = 0; i < AT_MAXD; ++i) {
            int d = lane + 32 * i;
            o[g][i] = 0.f;
            qv[g][i] = (g < group && d < hd) ? a.q[(size_t)(kvh * group + g) * hd + d] : 0.f;
        }
    }
    for (int t = t0 + warp; t < t1; t += AT_WARPS) {
        const float* kr = a.kc + (size_t)t * a.kv_dim + (size_t)kvh * hd;
        const float* vr = a.vc + (size_t)t * a.kv_dim + (size_t)kvh * hd;
        float kd[AT_MAXD], vd[AT_MAXD];
#pragma unroll
        for (int i = 0; i < AT_MAXD; ++i) {
            int d = lane + 32 * i;
            kd[i] = d < hd ? __ldcg(kr + d) : 0.f;
            vd[i] = d < hd ? __ldcg(vr + d) : 0.f;
        }
#pragma unroll
        for (int g = 0; g < AT_MAXG; ++g) {
            if (g < group) {
                float dot = 0.f;
#pragma unroll
                for (int i = 0; i < AT_MAXD; ++i) dot = fmaf(qv[g][i], kd[i], dot);
                float sc = __fmul_rn(warp_sum(dot), a.scale);
                float mn = fmaxf(m[g], sc);
                float corr = expf(m[g] - mn);
                float p = expf(sc - mn);
                l[g] = fmaf(l[g], corr, p);
#pragma unroll
                for (int i = 0; i < AT_MAXD; ++i) o[g][i] = fmaf(o[g][i], corr, p * vd[i]);
                m[g] = mn;
            }
        }
    }
    // combine the warps of this CTA (warp order)
#pragma unroll
    for (int g = 0; g < AT_MAXG; ++g) {
        if (g < group) {
            if (lane == 0) {
                sm_m[warp][g] = m[g];
                sm_l[warp][g] = l[g];
            }
#pragma unroll
            for (int i = 0; i < AT_MAXD; ++i) sm_o[warp][g][lane + 32 * i] = o[g][i];
        }
    }
    __syncthreads();
    const int W = hd + 2;
    for (int idx = threadIdx.x; idx < group * hd; idx += AT_WARPS * 32) {
        int g = idx / hd, d = idx % hd;
        float M = -INFINITY;
        for (int w = 0; w < AT_WARPS; ++w) M = fmaxf(M, sm_m[w][g]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < AT_WARPS; ++w) {
                float c = expf(sm_m[w][g] - M);
                L = fmaf(sm_l[w][g], c, L);
                O = fmaf(sm_o[w][g][d], c, O);
            }
        }
        float* pp = a.part + ((size_t)(kvh * group + g) * a.nsplit + s) * W;
        pp[2 + d] = O;
        if (d == 0) {
            pp[0] = M;
            pp[1] = L;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sm_last = atomicAdd(&a.counters[kvh], 1u) == (unsigned)(a.nsplit - 1);
    __syncthreads();
    if (!sm_last) return;
    __threadfence();
    const int nused = (seq + chunk - 1) / chunk;
    for (int idx = threadIdx.x; idx < group * hd; idx += AT_WARPS * 32) {
        int g = idx / hd, d = idx % hd;
        const float* pg = a.part + (size_t)(kvh * group + g) * a.nsplit * W;
        float M = -INFINITY;
        for (int j = 0; j < nused; ++j) M = fmaxf(M, __ldcg(pg + j * W));
        float L = 0.f, O = 0.f;
        for (int j = 0; j < nused; ++j) {
            float c = expf(__ldcg(pg + j * W) - M);
            L = fmaf(__ldcg(pg + j * W + 1), c, L);
            O = fmaf(__ldcg(pg + j * W + 2 + d), c, O);
        }
        a.out[(size_t)(kvh * group + g) * hd + d] = O / L;
    }
    if (threadIdx.x == 0) a.counters[kvh] = 0u;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.n_head / a.n_kv > AT_MAXG || a.hd > AT_MAXD * 32) return cudaErrorInvalidValue;
    dim3 grid(a.n_kv, a.nsplit);
    k_attention<<<grid, AT_WARPS * 32, 0, s>>>(a);
    return cudaGetLastError();
}

// =====================================================================
// Small kernels
// =====================================================================

__global__ void k_embed(const uint8_t* raw, int type, int cols, int vocab, StepParams* step, float* x) {
    uint32_t tok = step->token;
    if (tok >= (uint32_t)vocab) {
        if (threadIdx.x == 0) step->error = 1;
        tok = 0;
    }
    int be = type == GT_F32 ? 1 : (type == GT_Q6_K ? 256 : 32);
    int bb = type == GT_F32 ? 4 : (type == GT_Q6_K ? 210 : (type == GT_Q8_0 ? 34 : 18));
    const uint8_t* row = raw + (size_t)tok * (cols / be) * bb;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) x[i] = dequant_elem(type, row, i);
    if (threadIdx.x == 0) step->argmax_key = 0ull;
}

cudaError_t launch_embed(const uint8_t* raw, int type, int cols, int vocab, StepParams* step,
                         float* x, cudaStream_t s) {
    k_embed<<<1, 256, 0, s>>>(raw, type, cols, vocab, step, x);
    return cudaGetLastError();
}

__global__ void k_rmsnorm(const float* x, const float* w, float eps, int n, float* out) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int k = threadIdx.x; k < n; k += blockDim.x) ss = fmaf(x[k], x[k], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    float scale = 1.0f / sqrtf(red[0] / (float)n + eps);
    for (int k = threadIdx.x; k < n; k += blockDim.x) out[k] = __fmul_rn(__fmul_rn(x[k], scale), w[k]);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, float* out, cudaStream_t s) {
    k_rmsnorm<<<1, 1024, 0, s>>>(x, w, eps, n, out);
    return cudaGetLastError();
}

__global__ void k_greedy_advance(StepParams* step, uint32_t* gen, int cap) {
    uint32_t tok = (uint32_t)(step->argmax_key & 0xffffffffull);
    uint32_t n = step->n_gen;
    if (n < (uint32_t)cap) gen[n] = tok;
    step->n_gen = n + 1;
    step->token = tok;
    step->pos = step->pos + 1;
}

cudaError_t launch_greedy_advance(StepParams* step, uint32_t* gen, int cap, cudaStream_t s) {
    k_greedy_advance<<<1, 1, 0, s>>>(step, gen, cap);
    return cudaGetLastError();
}

}  // namespace talos
