// matvec.cu -- weight repacking and the fused dequant-matvec of the Talos decode
// path on B200 (sm_100a).
//
// Reference: QTensor::matvec (Tsuskov/talos src/model/weights.rs:47-55) ->
// quant::matvec (src/math/quant.rs:18-51) / matmul::matvec
// (src/math/matmul.rs:34-47): y[r] = sum_k dequant(W)[r, k] * x[k], with the
// block formats of src/gguf/dtype.rs:64-121.
//
// Design (HBM-bound: every weight byte is read once per token):
//  * Weights are repacked at upload into "group-chunks": 8 rows x CK input
//    elements, contiguous, in the register order the math below consumes.
//  * One persistent CTA per SM. A producer warp streams the group-chunks of the
//    CTA's tiles (16 rows = two 8-row groups) into a ring of shared-memory stages
//    with cp.async.bulk (1-D TMA) completing on mbarriers; 16 consumer warps
//    compute from shared memory and release the stage.
//  * Programmatic dependent launch: weights do not depend on earlier kernels, so
//    the producer starts streaming before griddepcontrol.wait; only the
//    activation read waits for the previous kernel.
//  * Q4_0 / Q8_0 / Q6_K run on the tensor cores (mma.sync m16n8k16, f16 in,
//    f32 out). A quant u (0..15 / 0..255 / 0..63) enters the MMA as the f16
//    SUBNORMAL u * 2^-24, which a single AND / byte-permute of the packed bits
//    produces exactly; Q4_0's high nibbles come in as 16u * 2^-24 and meet
//    activations pre-divided by 16. The activation is split into f16 hi + lo
//    parts (two B columns, x = hi + lo to ~22 bits). Per block b and row r:
//        sum_k (u_k - z) x_k = 2^24 * D(r, b) - z * S_b,   S_b = sum_{k in b} x_k
//    (z = 8 / 128 / 32 is the format's zero point), then scaled by the block's
//    f16 scale on the CUDA cores. F32 weights use CUDA-core FMAs.
#include <math.h>

#include "kernels.cuh"
#include "ptx.cuh"

namespace talos {

static inline int ceil_div_h(int a, int b) { return (a + b - 1) / b; }

// ----------------------------------------------------------------------------
// Per-format constants
// ----------------------------------------------------------------------------
//   CK    input elements per chunk
//   GCB   bytes of one group-chunk (8 rows x CK)
//   NST   ring stages
template <int TYPE>
struct Fmt;
template <>
struct Fmt<GT_Q4_0> {  // 64 blocks = 16 quads per chunk
    static constexpr int CK = 2048, GCB = 16 * 512 + 16 * 64, NST = 4;
};
template <>
struct Fmt<GT_Q8_0> {  // 32 blocks = 8 quads per chunk
    static constexpr int CK = 1024, GCB = 8 * 1024 + 8 * 64, NST = 4;
};
template <>
struct Fmt<GT_Q6_K> {  // 4 super-blocks = 64 sub-blocks per chunk
    static constexpr int CK = 1024, GCB = 16 * 512 + 8 * 64 + 8 * 4 * 2, NST = 4;
};
template <>
struct Fmt<GT_F32> {
    static constexpr int CK = 256, GCB = 8 * 256 * 4, NST = 4;
};

static int fmt_ck(int type) {
    switch (type) {
        case GT_Q4_0: return Fmt<GT_Q4_0>::CK;
        case GT_Q8_0: return Fmt<GT_Q8_0>::CK;
        case GT_Q6_K: return Fmt<GT_Q6_K>::CK;
        case GT_F32: return Fmt<GT_F32>::CK;
    }
    return 0;
}
static int fmt_gcb(int type) {
    switch (type) {
        case GT_Q4_0: return Fmt<GT_Q4_0>::GCB;
        case GT_Q8_0: return Fmt<GT_Q8_0>::GCB;
        case GT_Q6_K: return Fmt<GT_Q6_K>::GCB;
        case GT_F32: return Fmt<GT_F32>::GCB;
    }
    return 0;
}
static int fmt_nst(int type) {
    switch (type) {
        case GT_Q4_0: return Fmt<GT_Q4_0>::NST;
        case GT_Q8_0: return Fmt<GT_Q8_0>::NST;
        case GT_Q6_K: return Fmt<GT_Q6_K>::NST;
        case GT_F32: return Fmt<GT_F32>::NST;
    }
    return 0;
}

bool pack_sizes(int type, int rows, int cols, PackSizes* o) {
    *o = PackSizes{};
    int ck = fmt_ck(type);
    if (!ck) return false;
    if (type == GT_Q4_0 || type == GT_Q8_0) {
        if (cols % 32) return false;
    } else if (type == GT_Q6_K) {
        if (cols % 256) return false;
    }
    o->rows_pad = ceil_div_h(rows, 16) * 16;
    o->nk = ceil_div_h(cols, ck);  // chunks per row group
    o->b0 = (size_t)(o->rows_pad / 8) * o->nk * fmt_gcb(type);
    o->b1 = type == GT_F32 ? 0 : 16;  // the value bound k_wbound records
    return true;
}

// ----------------------------------------------------------------------------
// Repacking (lossless), one thread per (row, block)
// ----------------------------------------------------------------------------

// Q4_0 group-chunk: [16 quads][32 lanes][4 words] then [16 quads][8 rows][4] f16.
// Lane L (row 8g + L/4, t = L%4, k0 = 2t) word j of quad q holds block
// b = 4q + j of the chunk as nibbles:
//   bits  0-3 u[k0]     16-19 u[k0+1]    (A fragment, k 0-15, cols 2t, 2t+1)
//   bits  4-7 u[k0+8]   20-23 u[k0+9]    (cols 2t+8, 2t+9)
//   bits  8-11 u[16+k0] 24-27 u[17+k0]   (k 16-31, after >> 8)
//   bits 12-15 u[24+k0] 28-31 u[25+k0]
// with u[e] the 4-bit quant of element e (dtype.rs:85-89: the low nibble of byte
// j is element j, the high nibble element j+16). Pad blocks and rows: u = 8, d = 0.
__global__ void k_pack_q4_0(const uint8_t* raw, PackedW w) {
    constexpr int QPC = Fmt<GT_Q4_0>::CK / 128;  // quads per chunk
    const int nb_src = w.cols / 32;
    const int nb_pad = w.nk * (Fmt<GT_Q4_0>::CK / 32);
    const size_t n = (size_t)w.rows_pad * nb_pad;
    uint8_t* base = (uint8_t*)w.p0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / nb_pad), b = (int)(i % nb_pad);
        const int g = r / 8, c = b / (4 * QPC), bq = (b % (4 * QPC)) / 4, j = b % 4;
        uint8_t bytes[16];
        uint16_t dbits = 0;
        if (r < w.rows && b < nb_src) {
            const uint8_t* blk = raw + ((size_t)r * nb_src + b) * 18;
            dbits = (uint16_t)(blk[0] | (blk[1] << 8));
            for (int k = 0; k < 16; ++k) bytes[k] = blk[2 + k];
        } else {
            for (int k = 0; k < 16; ++k) bytes[k] = 0x88;
        }
        uint8_t* gc = base + ((size_t)g * w.nk + c) * Fmt<GT_Q4_0>::GCB;
        uint32_t* qs = (uint32_t*)gc;
        uint16_t* sc = (uint16_t*)(gc + QPC * 512);
        sc[(bq * 8 + (r % 8)) * 4 + j] = dbits;
        for (int t = 0; t < 4; ++t) {
            const int k0 = 2 * t;
            const uint32_t b0 = (bytes[k0] & 0xF) | ((bytes[k0 + 8] & 0xF) << 4);
            const uint32_t b1 = (bytes[k0] >> 4) | ((bytes[k0 + 8] >> 4) << 4);
            const uint32_t b2 = (bytes[k0 + 1] & 0xF) | ((bytes[k0 + 9] & 0xF) << 4);
            const uint32_t b3 = (bytes[k0 + 1] >> 4) | ((bytes[k0 + 9] >> 4) << 4);
            const int lane = (r % 8) * 4 + t;
            qs[(bq * 32 + lane) * 4 + j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
    }
}

// Q8_0 group-chunk: [8 quads][32 lanes][4 blocks][8 bytes] then [8 quads][8 rows][4] f16.
// Lane L (row 8g + L/4, t = L%4) bytes of block j: int8 q at elements
// {2t, 2t+1, 2t+8, 2t+9, 16+2t, 17+2t, 24+2t, 25+2t}.
__global__ void k_pack_q8_0(const uint8_t* raw, PackedW w) {
    const int nb_src = w.cols / 32;
    const int nb_pad = w.nk * 32;
    const size_t n = (size_t)w.rows_pad * nb_pad;
    uint8_t* base = (uint8_t*)w.p0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / nb_pad), b = (int)(i % nb_pad);
        const int g = r / 8, c = b / 32, bq = (b % 32) / 4, j = b % 4;
        int8_t q[32];
        uint16_t dbits = 0;
        if (r < w.rows && b < nb_src) {
            const uint8_t* blk = raw + ((size_t)r * nb_src + b) * 34;
            dbits = (uint16_t)(blk[0] | (blk[1] << 8));
            for (int k = 0; k < 32; ++k) q[k] = (int8_t)blk[2 + k];
        } else {
            for (int k = 0; k < 32; ++k) q[k] = 0;
        }
        uint8_t* gc = base + ((size_t)g * w.nk + c) * Fmt<GT_Q8_0>::GCB;
        uint16_t* sc = (uint16_t*)(gc + 8 * 1024);
        sc[(bq * 8 + (r % 8)) * 4 + j] = dbits;
        for (int t = 0; t < 4; ++t) {
            const int lane = (r % 8) * 4 + t;
            int8_t* dst = (int8_t*)gc + ((bq * 32 + lane) * 4 + j) * 8;
            const int e[8] = {2 * t, 2 * t + 1, 2 * t + 8, 2 * t + 9, 16 + 2 * t, 17 + 2 * t, 24 + 2 * t, 25 + 2 * t};
            for (int k = 0; k < 8; ++k) dst[k] = q[e[k]];
        }
    }
}

// Q6_K group-chunk (4 super-blocks = 64 sub-blocks of 16):
//   [16 step-quads][32 lanes][4 steps][4 bytes]: lane L (row 8g + L/4, t = L%4) bytes of
//   sub-block s: the 6-bit quant u (0..63) at elements {2t, 2t+1, 2t+8, 2t+9};
//   then int8 sc [8 rows][64], then f16 d [8 rows][4].
// The quants are widened to bytes with the decoding of dtype.rs:106-111; the scales
// are the block's own sc and d, so (d * sc) is formed as in dtype.rs:112-115.
__global__ void k_pack_q6_k(const uint8_t* raw, PackedW w) {
    const int nsb_src = w.cols / 256;
    const int nsb_pad = w.nk * 4;
    const size_t n = (size_t)w.rows_pad * nsb_pad;
    uint8_t* base = (uint8_t*)w.p0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / nsb_pad), sb = (int)(i % nsb_pad);
        const int g = r / 8, c = sb / 4, sbc = sb % 4;
        uint8_t q[256];
        int8_t scv[16];
        uint16_t dbits = 0;
        if (r < w.rows && sb < nsb_src) {
            const uint8_t* b = raw + ((size_t)r * nsb_src + sb) * 210;
            for (int h = 0; h < 2; ++h) {
                const uint8_t* ql = b + h * 64;
                const uint8_t* qh = b + 128 + h * 32;
                for (int l = 0; l < 32; ++l) {
                    q[h * 128 + l] = (uint8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4));
                    q[h * 128 + l + 32] = (uint8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4));
                    q[h * 128 + l + 64] = (uint8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4));
                    q[h * 128 + l + 96] = (uint8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4));
                }
            }
            for (int s = 0; s < 16; ++s) scv[s] = (int8_t)b[192 + s];
            dbits = (uint16_t)(b[208] | (b[209] << 8));
        } else {
            for (int k = 0; k < 256; ++k) q[k] = 32;
            for (int s = 0; s < 16; ++s) scv[s] = 0;
        }
        uint8_t* gc = base + ((size_t)g * w.nk + c) * Fmt<GT_Q6_K>::GCB;
        int8_t* sc = (int8_t*)(gc + 16 * 512);
        uint16_t* dd = (uint16_t*)(gc + 16 * 512 + 8 * 64);
        dd[(r % 8) * 4 + sbc] = dbits;
        for (int s = 0; s < 16; ++s) {
            const int step = sbc * 16 + s;  // sub-block index in the chunk, 0..63
            sc[(r % 8) * 64 + step] = scv[s];
            const int sq = step / 4, sj = step % 4;
            for (int t = 0; t < 4; ++t) {
                const int lane = (r % 8) * 4 + t;
                uint8_t* dst = gc + ((sq * 32 + lane) * 4 + sj) * 4;
                dst[0] = q[16 * s + 2 * t];
                dst[1] = q[16 * s + 2 * t + 1];
                dst[2] = q[16 * s + 2 * t + 8];
                dst[3] = q[16 * s + 2 * t + 9];
            }
        }
    }
}

// F32 group-chunk: [8 rows][256] floats.
__global__ void k_pack_f32(const uint8_t* raw, PackedW w) {
    const int ck = Fmt<GT_F32>::CK;
    const int kp = w.nk * ck;
    const size_t n = (size_t)w.rows_pad * kp;
    uint8_t* base = (uint8_t*)w.p0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kp), k = (int)(i % kp);
        const int g = r / 8, c = k / ck;
        float v = 0.f;
        if (r < w.rows && k < w.cols) {
            const uint8_t* p = raw + 4 * ((size_t)r * w.cols + k);
            v = __uint_as_float(p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24));
        }
        float* gc = (float*)(base + ((size_t)g * w.nk + c) * Fmt<GT_F32>::GCB);
        gc[(r % 8) * ck + (k % ck)] = v;
    }
}

// The largest |value| a quant tensor's blocks can dequantize to, recorded at p1
// (f32) for the tensor-core GEMM's power-of-two prescale: max |d| x 8 (Q4_0:
// |nibble - 8| <= 8), x 128 (Q8_0), and max |d * sc| x 32 (Q6_K: |q - 32| <= 32).
// Non-negative f32 values order like their bit patterns, so atomicMax on the
// bits takes the maximum.
__global__ void k_wbound(const uint8_t* raw, int type, size_t nblocks, float* out) {
    float m = 0.f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nblocks; i += (size_t)gridDim.x * blockDim.x) {
        if (type == GT_Q4_0) {
            m = fmaxf(m, fabsf(ld_half_bytes(raw + i * 18)) * 8.f);
        } else if (type == GT_Q8_0) {
            m = fmaxf(m, fabsf(ld_half_bytes(raw + i * 34)) * 128.f);
        } else {
            const uint8_t* b = raw + i * 210;
            int sm = 0;
            for (int j = 0; j < 16; ++j) sm = max(sm, abs((int)(int8_t)b[192 + j]));
            m = fmaxf(m, fabsf(ld_half_bytes(b + 208)) * (float)sm * 32.f);
        }
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) atomicMax((unsigned*)out, __float_as_uint(m));
}

cudaError_t launch_pack(const uint8_t* raw, const PackedW& w, cudaStream_t s) {
    const int T = 256;
    const unsigned G = 148 * 16;
    switch (w.type) {
        case GT_F32: k_pack_f32<<<G, T, 0, s>>>(raw, w); break;
        case GT_Q8_0: k_pack_q8_0<<<G, T, 0, s>>>(raw, w); break;
        case GT_Q4_0: k_pack_q4_0<<<G, T, 0, s>>>(raw, w); break;
        case GT_Q6_K: k_pack_q6_k<<<G, 64, 0, s>>>(raw, w); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || w.type == GT_F32 || !w.p1) return e;
    if ((e = cudaMemsetAsync((void*)w.p1, 0, sizeof(float), s)) != cudaSuccess) return e;
    const size_t nb = (size_t)w.rows * (w.cols / gguf_block_elems(w.type));
    k_wbound<<<148 * 4, 256, 0, s>>>(raw, w.type, nb, (float*)w.p1);
    return cudaGetLastError();
}

// PTX helpers (mbarrier, 1-D bulk copy, programmatic dependent launch): ptx.cuh

constexpr int MV_CONSUMERS = 512;              // 16 consumer warps
constexpr int MV_CWARPS = MV_CONSUMERS / 32;
constexpr int MV_THREADS = MV_CONSUMERS + 64;  // + 1 producer warp + 1 epilogue warp
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }
// consumer_sync that also ORs a flag over the 512 consumer threads.
__device__ __forceinline__ bool consumer_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 512, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// f16 range of the staged activation. Its f16 hi part overflows from 65,520 on,
// so an input with an element of magnitude 2^15 or more is staged again scaled
// by 2^-16 (exact for f32), as often as needed (at most kStageRetries times),
// and the tile's row sums are multiplied back by the same power of two. Inputs
// in range take one pass; the check rides on the staging's last barrier.
constexpr float kStageBig = 32768.f;
constexpr float kStageDown = 1.52587890625e-05f;  // 2^-16
constexpr int kStageRetries = 6;
__device__ __forceinline__ bool big4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) >= kStageBig;
}
__device__ __forceinline__ float4 scale4(float4 v, float s) { return make_float4(v.x * s, v.y * s, v.z * s, v.w * s); }

// D = A(16x16 f16) * B(16x8 f16), f32 accumulate from zero / from d. Not
// volatile: the MMAs of independent blocks may be scheduled around each other.
__device__ __forceinline__ void mma_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
__device__ __forceinline__ void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two bytes (sel picks them) of w -> f16x2 subnormals u * 2^-24, exact.
__device__ __forceinline__ uint32_t bytes_sub(uint32_t w, uint32_t sel) { return __byte_perm(w, 0u, sel); }

constexpr float kTwo24 = 16777216.0f;

// ----------------------------------------------------------------------------
// Consumers: one stage (two group-chunks A, B) -> per-lane partial sums.
// p* accumulate sum_b d_b * 2^-24-scaled MMA sums, q* accumulate sum_b d_b * S_b;
// the row value is 2^24 p - z q.
// xf: staged activation, per 32-element block: 8 lanes x uint4 (lanes 0-3 hi,
// 4-7 lo; {k 2t,2t+1 | 2t+8,2t+9} of step 0 then step 1). xs16: per 16 elements S.
// ----------------------------------------------------------------------------

struct Acc {
    float pA, qA, pB, qB;
};

// Consumer warp w of 16 takes quad w (blocks 4w .. 4w+3) of the chunk's 64.
__device__ __forceinline__ void consume_q4_0(const uint8_t* sA, const uint8_t* sB, const uint4* xf,
                                             const float* xs16, int chunk, Acc& acc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int QPC = Fmt<GT_Q4_0>::CK / 128;
    const uint4 wa = *(const uint4*)(sA + (warp * 32 + lane) * 16);
    const uint4 wb = *(const uint4*)(sB + (warp * 32 + lane) * 16);
    const uint2 ca = *(const uint2*)(sA + QPC * 512 + (warp * 8 + (lane >> 2)) * 8);
    const uint2 cb = *(const uint2*)(sB + QPC * 512 + (warp * 8 + (lane >> 2)) * 8);
    const float2 a01 = __half22float2(*reinterpret_cast<const half2*>(&ca.x));
    const float2 a23 = __half22float2(*reinterpret_cast<const half2*>(&ca.y));
    const float2 b01 = __half22float2(*reinterpret_cast<const half2*>(&cb.x));
    const float2 b23 = __half22float2(*reinterpret_cast<const half2*>(&cb.y));
    const float dA[4] = {a01.x, a01.y, a23.x, a23.y};
    const float dB[4] = {b01.x, b01.y, b23.x, b23.y};
    const uint32_t xa[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t xb[4] = {wb.x, wb.y, wb.z, wb.w};
    const int blk0 = chunk * (Fmt<GT_Q4_0>::CK / 32) + warp * 4;
    // B fragments: lanes 8-31 read lanes 0-7's words, so B columns 2-7 hold finite
    // copies whose products land in D columns this code never reads.
    const uint4* xbp = xf + blk0 * 8 + (lane & 7);
    const float4 S4 = *(const float4*)(xs16 + blk0);  // per-32-block sums (xs32)
    const float S[4] = {S4.x, S4.y, S4.z, S4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 bx = xbp[j * 8];
        float d[4];
        mma_z(d, xa[j] & 0x000F000Fu, xb[j] & 0x000F000Fu, xa[j] & 0x00F000F0u, xb[j] & 0x00F000F0u, bx.x, bx.y);
        const uint32_t ya = xa[j] >> 8, yb = xb[j] >> 8;
        mma_acc(d, ya & 0x000F000Fu, yb & 0x000F000Fu, ya & 0x00F000F0u, yb & 0x00F000F0u, bx.z, bx.w);
        acc.pA = fmaf(dA[j], d[0], fmaf(dA[j], d[1], acc.pA));
        acc.pB = fmaf(dB[j], d[2], fmaf(dB[j], d[3], acc.pB));
        acc.qA = fmaf(dA[j], S[j], acc.qA);
        acc.qB = fmaf(dB[j], S[j], acc.qB);
    }
}

// Consumer warp w of 16 takes blocks 2w, 2w+1 of the chunk's 32 (half of quad w/2).
__device__ __forceinline__ void consume_q8_0(const uint8_t* sA, const uint8_t* sB, const uint4* xf,
                                             const float* xs16, int chunk, Acc& acc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int quad = warp >> 1, half_ = warp & 1;
    const uint4 wa = *(const uint4*)(sA + (quad * 32 + lane) * 32 + half_ * 16);
    const uint4 wb = *(const uint4*)(sB + (quad * 32 + lane) * 32 + half_ * 16);
    const uint32_t ca = *(const uint32_t*)(sA + 8 * 1024 + (quad * 8 + (lane >> 2)) * 8 + half_ * 4);
    const uint32_t cb = *(const uint32_t*)(sB + 8 * 1024 + (quad * 8 + (lane >> 2)) * 8 + half_ * 4);
    const float2 fa = __half22float2(*reinterpret_cast<const half2*>(&ca));
    const float2 fb = __half22float2(*reinterpret_cast<const half2*>(&cb));
    const float dA[2] = {fa.x, fa.y};
    const float dB[2] = {fb.x, fb.y};
    // int8 q -> u = q + 128 via the sign flip; per block two words
    const uint32_t A[4] = {wa.x ^ 0x80808080u, wa.y ^ 0x80808080u, wa.z ^ 0x80808080u, wa.w ^ 0x80808080u};
    const uint32_t B[4] = {wb.x ^ 0x80808080u, wb.y ^ 0x80808080u, wb.z ^ 0x80808080u, wb.w ^ 0x80808080u};
    const int blk0 = chunk * 32 + warp * 2;
    const uint4* xbp = xf + blk0 * 8 + (lane & 7);  // lanes 8-31: unused B columns
    const float2 S2 = *(const float2*)(xs16 + blk0);  // per-32-block sums
    const float Sb[2] = {S2.x, S2.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint4 bx = xbp[j * 8];
        float d[4];
        mma_z(d, bytes_sub(A[2 * j], 0x4140), bytes_sub(B[2 * j], 0x4140), bytes_sub(A[2 * j], 0x4342),
              bytes_sub(B[2 * j], 0x4342), bx.x, bx.y);
        mma_acc(d, bytes_sub(A[2 * j + 1], 0x4140), bytes_sub(B[2 * j + 1], 0x4140), bytes_sub(A[2 * j + 1], 0x4342),
                bytes_sub(B[2 * j + 1], 0x4342), bx.z, bx.w);
        acc.pA = fmaf(dA[j], d[0], fmaf(dA[j], d[1], acc.pA));
        acc.pB = fmaf(dB[j], d[2], fmaf(dB[j], d[3], acc.pB));
        acc.qA = fmaf(dA[j], Sb[j], acc.qA);
        acc.qB = fmaf(dB[j], Sb[j], acc.qB);
    }
}

// Q6_K: consumer warp w of 16 takes sub-blocks 4w .. 4w+3 of the chunk (step-quad w).
__device__ __forceinline__ void consume_q6_k(const uint8_t* sA, const uint8_t* sB, const uint4* xf,
                                             const float* xs16, int chunk, Acc& acc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = lane >> 2;
    const uint32_t scA = *(const uint32_t*)(sA + 16 * 512 + row * 64 + warp * 4);
    const uint32_t scB = *(const uint32_t*)(sB + 16 * 512 + row * 64 + warp * 4);
    const float dA = __half2float(*(const half*)(sA + 16 * 512 + 8 * 64 + (row * 4 + (warp >> 2)) * 2));
    const float dB = __half2float(*(const half*)(sB + 16 * 512 + 8 * 64 + (row * 4 + (warp >> 2)) * 2));
    const uint4 wa = *(const uint4*)(sA + (warp * 32 + lane) * 16);
    const uint4 wb = *(const uint4*)(sB + (warp * 32 + lane) * 16);
    const uint32_t A[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t B[4] = {wb.x, wb.y, wb.z, wb.w};
    const int step0 = chunk * 64 + warp * 4;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        // sub-blocks step0 + 2p, +1 = one 32-element x block
        const int blk = (step0 + 2 * p) / 2;
        const uint4 bx = xf[blk * 8 + (lane & 7)];  // lanes 8-31: unused B columns
        const float2 s = *(const float2*)(xs16 + step0 + 2 * p);
        float d0[4], d1[4];
        mma_z(d0, bytes_sub(A[2 * p], 0x4140), bytes_sub(B[2 * p], 0x4140), bytes_sub(A[2 * p], 0x4342),
              bytes_sub(B[2 * p], 0x4342), bx.x, bx.y);
        mma_z(d1, bytes_sub(A[2 * p + 1], 0x4140), bytes_sub(B[2 * p + 1], 0x4140), bytes_sub(A[2 * p + 1], 0x4342),
              bytes_sub(B[2 * p + 1], 0x4342), bx.z, bx.w);
        // (d * sc), the order of src/gguf/dtype.rs:112-115
        const float a0 = __fmul_rn(dA, (float)(int8_t)(scA >> (16 * p))),
                    a1 = __fmul_rn(dA, (float)(int8_t)(scA >> (16 * p + 8)));
        const float b0 = __fmul_rn(dB, (float)(int8_t)(scB >> (16 * p))),
                    b1 = __fmul_rn(dB, (float)(int8_t)(scB >> (16 * p + 8)));
        acc.pA = fmaf(a0, d0[0] + d0[1], acc.pA);
        acc.pA = fmaf(a1, d1[0] + d1[1], acc.pA);
        acc.qA = fmaf(a0, s.x, fmaf(a1, s.y, acc.qA));
        acc.pB = fmaf(b0, d0[2] + d0[3], acc.pB);
        acc.pB = fmaf(b1, d1[2] + d1[3], acc.pB);
        acc.qB = fmaf(b0, s.x, fmaf(b1, s.y, acc.qB));
    }
}

// F32: consumer warp w of 16 computes tile row w (group A rows 0-7, B rows 8-15)
// over the chunk's 256 inputs into acc.pA.
__device__ __forceinline__ void consume_f32(const uint8_t* sA, const uint8_t* sB, const float* xs, int chunk,
                                            Acc& acc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* g = (const float*)(warp < 8 ? sA : sB);
    const float4* w0 = (const float4*)(g + (warp & 7) * 256);
    const float4* x4 = (const float4*)(xs + chunk * 256);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float4 xv = x4[lane + 32 * i];
        const float4 u = w0[lane + 32 * i];
        acc.pA = fmaf(u.x, xv.x, fmaf(u.y, xv.y, fmaf(u.z, xv.z, fmaf(u.w, xv.w, acc.pA))));
    }
}

// ----------------------------------------------------------------------------
// The kernel
// ----------------------------------------------------------------------------

template <int TYPE>
struct Zero;  // the format's zero point z in sum (u - z) x
template <>
struct Zero<GT_Q4_0> {
    static constexpr float z = 8.f;
};
template <>
struct Zero<GT_Q8_0> {
    static constexpr float z = 128.f;
};
template <>
struct Zero<GT_Q6_K> {
    static constexpr float z = 32.f;
};
template <>
struct Zero<GT_F32> {
    static constexpr float z = 0.f;
};


__device__ __forceinline__ void split_pair(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
    const half l0 = __float2half_rn(v0 - __half2float(h0));
    const half l1 = __float2half_rn(v1 - __half2float(h1));
    hi = pack_half2(h0, h1);
    lo = pack_half2(l0, l1);
}

// Group-chunk sources of tile lt of segment sg at chunk c.
template <int TYPE>
__device__ __forceinline__ void tile_src(const Seg& sg, int lt, int c, const uint8_t*& a, const uint8_t*& b) {
    const PackedW& WA = sg.A;
    const PackedW& WB = sg.pair ? sg.B : sg.A;
    const int gA = sg.pair ? lt : 2 * lt;
    const int gB = sg.pair ? lt : 2 * lt + 1;
    a = (const uint8_t*)WA.p0 + ((size_t)gA * WA.nk + c) * Fmt<TYPE>::GCB;
    b = (const uint8_t*)WB.p0 + ((size_t)gB * WB.nk + c) * Fmt<TYPE>::GCB;
}

__device__ __forceinline__ void find_seg(const MatvecArgs& a, int t, int& si, int& lt) {
    si = 0;
    lt = t;
    while (si + 1 < a.nseg && lt >= a.seg[si].ntiles) {
        lt -= a.seg[si].ntiles;
        ++si;
    }
}

// Shared memory: ring | full[NST] empty[NST] tdone[2] tfree[2] | xf (KP*4 B) |
//                xs16 (KP/16 f32) | part[2][16][16] | res[16] | red[32]
template <int TYPE>
__host__ __device__ constexpr size_t mv_smem_fixed() {
    return (size_t)Fmt<TYPE>::NST * 2 * Fmt<TYPE>::GCB + (2 * Fmt<TYPE>::NST + 4) * 8 +
           (2 * MV_CWARPS * 16 + 16 + 32) * 4;
}
__host__ __device__ inline size_t mv_smem_per_k(int KP) { return (size_t)KP * 4 + (size_t)KP / 16 * 4; }

// The epilogue warp: per tile, sums the 16 consumer warps' partials in warp order,
// frees the partial buffer, then applies the launch's epilogue: store, residual
// add (src/model/llama.rs:159-161,174-176), SwiGLU of paired gate/up rows
// (src/math/ops.rs:28-37), q/k RoPE with the KV append (src/math/ops.rs:48-61,
// src/kv_cache.rs:21-26), or logits with a running argmax (src/sample.rs:7-14).
// Global inputs of a tile's epilogue, loaded before its partials are ready: the
// residual row (EPI_ADD, lanes 0-15) and the RoPE (cos, sin) of the lane's pair
// (EPI_QKV q and k, lanes 0-7).
struct EpiPre {
    float xres;
    float2 cs;
};
__device__ __forceinline__ EpiPre epi_prefetch(const MatvecArgs& a, const Seg& sg, int lt, uint32_t pos, int lane) {
    EpiPre e{0.f, make_float2(1.f, 0.f)};
    if (a.epi == EPI_ADD) {
        const int row = 16 * lt + lane;
        if (lane < 16 && row < sg.out_rows) e.xres = __ldcg(sg.out + row);  // another CTA may have written it
    } else if (a.epi == EPI_QKV && sg.role != 2 && lane < 8) {
        const int r0 = 16 * lt + 2 * lane;
        if (r0 < sg.out_rows) e.cs = a.rope_cs[(size_t)pos * (a.hd >> 1) + ((r0 % a.hd) >> 1)];
    }
    return e;
}

__device__ __forceinline__ void apply_epilogue(const MatvecArgs& a, const Seg& sg, int lt, const float* res,
                                               uint32_t pos, int lane, const EpiPre& pre);

template <int TYPE>
__device__ __forceinline__ void epilogue_warp(const MatvecArgs& a, const float* part, float* res, uint64_t* tdone,
                                              uint64_t* tfree, int* s_err) {
    const int lane = threadIdx.x & 31;
    pdl_wait();  // outputs (residual stream, caches) belong to the previous kernel until it completes
    const uint32_t pos = a.step ? a.step->pos : 0u;
    int n = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, ++n) {
        int si, lt;
        find_seg(a, t, si, lt);
        const Seg& sg = a.seg[si];
        const int b = n & 1;
        const EpiPre pre = epi_prefetch(a, sg, lt, pos, lane);
        if (!mbar_wait(&tdone[b], (uint32_t)(n >> 1) & 1)) {
            *s_err = 1;
            if (a.step) atomicOr(&a.step->error, 2u);
            return;
        }
        // lane l sums row (l & 15) over warps 8h .. 8h+7, h = l >> 4; halves then add
        const float* pb = part + b * MV_CWARPS * 16;
        const int r = lane & 15, h = lane >> 4;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < MV_CWARPS / 2; ++w) v += pb[(8 * h + w) * 16 + r];
        const float other = __shfl_xor_sync(0xffffffffu, v, 16);
        v = h == 0 ? v + other : other + v;  // (warps 0-7) + (warps 8-15) on every lane
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfree[b]);
        if (lane < 16) res[lane] = v;
        __syncwarp();
        apply_epilogue(a, sg, lt, res, pos, lane, pre);
        __syncwarp();
    }
}

// The epilogue of one tile: res[0..15] are its 16 row values (8 gate + 8 up rows
// for SwiGLU); called by all 32 lanes of one warp.
__device__ __forceinline__ void apply_epilogue(const MatvecArgs& a, const Seg& sg, int lt, const float* res,
                                               uint32_t pos, int lane, const EpiPre& pre) {
    {
        if (a.epi == EPI_SWIGLU) {  // src/math/ops.rs:33-37
            if (lane < 8) {
                const int j = 8 * lt + lane;
                if (j < sg.out_rows) sg.out[j] = __fmul_rn(silu_ref(res[lane]), res[8 + lane]);
            }
        } else if (a.epi == EPI_QKV) {
            if (sg.role == 2) {  // v -> cache row pos (src/kv_cache.rs:21-26)
                if (lane < 16) {
                    const int row = 16 * lt + lane;
                    if (row < sg.out_rows) {
                        const size_t i = (size_t)pos * a.kv_dim + row;
                        if (a.kv_f16)
                            ((__half*)a.vcache)[i] = __float2half_rn(res[lane]);
                        else
                            ((float*)a.vcache)[i] = res[lane];
                    }
                }
            } else if (lane < 8) {  // RoPE on pairs (2i, 2i+1) (src/math/ops.rs:48-61)
                const int r0 = 16 * lt + 2 * lane;
                if (r0 < sg.out_rows) {
                    const float2 cs = pre.cs;
                    const float x0 = res[2 * lane], x1 = res[2 * lane + 1];
                    const float o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
                    const float o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
                    if (sg.role == 1 && a.kv_f16) {
                        *(__half2*)((__half*)a.kcache + (size_t)pos * a.kv_dim + r0) = __floats2half2_rn(o0, o1);
                    } else {
                        float* dst = sg.role == 0 ? sg.out + r0 : (float*)a.kcache + (size_t)pos * a.kv_dim + r0;
                        dst[0] = o0;
                        dst[1] = o1;
                    }
                }
            }
        } else {
            unsigned long long key = 0ull;
            if (lane < 16) {
                const int row = 16 * lt + lane;
                if (row < sg.out_rows) {
                    sg.out[row] = a.epi == EPI_ADD ? __fadd_rn(pre.xres, res[lane]) : res[lane];
                    key = argmax_key(res[lane], (uint32_t)row);
                }
            }
            if (a.epi == EPI_LOGITS) {  // running argmax (src/sample.rs:7-14)
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) {
                    const unsigned long long oth = __shfl_xor_sync(0xffffffffu, key, o);
                    key = oth > key ? oth : key;
                }
                if (lane == 0 && key) atomicMax(&a.step->argmax_key, key);
            }
        }
    }
}

// __launch_bounds__(.., 2): registers for two resident CTAs per SM, so the next
// kernel's CTA can start streaming while this one finishes.
template <int TYPE>
__global__ void __launch_bounds__(MV_THREADS, 2) k_matvec(const __grid_constant__ MatvecArgs a) {
    constexpr int NST = Fmt<TYPE>::NST, GCB = Fmt<TYPE>::GCB, CK = Fmt<TYPE>::CK;
    constexpr int STAGE = 2 * GCB;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int K = a.K;
    const int nchunk = (K + CK - 1) / CK;
    const int KP = nchunk * CK;
    uint8_t* ring = smem;
    uint64_t* full = (uint64_t*)(smem + NST * STAGE);
    uint64_t* empty = full + NST;
    uint64_t* tdone = empty + NST;  // [2] partials of a tile written (16 consumer warps)
    uint64_t* tfree = tdone + 2;    // [2] partials of a tile read by the epilogue warp
    float* stage_x = (float*)(tfree + 2);  // KP floats (Q types: fragments, same bytes)
    float* xs16 = stage_x + KP;              // KP / 16
    float* part = xs16 + KP / 16;            // [2][MV_CWARPS][16]
    float* res = part + 2 * MV_CWARPS * 16;  // 16
    float* red = res + 16;                   // 32
    __shared__ int s_err;

    if (tid == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], MV_CWARPS);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tdone[i], MV_CWARPS);
            mbar_init(&tfree[i], 1);
        }
        s_err = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (tid >= MV_CONSUMERS + 32) {
        epilogue_warp<TYPE>(a, part, res, tdone, tfree, &s_err);
        return;
    }
    if (tid >= MV_CONSUMERS) {
        // ---------------- producer warp: stream weights (independent of earlier kernels)
        if (tid == MV_CONSUMERS) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.ntiles && ok; t += gridDim.x) {
                int si, lt;
                find_seg(a, t, si, lt);
                const Seg& sg = a.seg[si];
                for (int c = 0; c < nchunk; ++c, ++it) {
                    const int slot = it % NST;
                    if (!mbar_wait(&empty[slot], ((it / NST) & 1) ^ 1) || *(volatile int*)&s_err) {
                        ok = false;
                        break;
                    }
                    const uint8_t *ga, *gb;
                    tile_src<TYPE>(sg, lt, c, ga, gb);
                    uint8_t* dst = ring + slot * STAGE;
                    mbar_expect_tx(&full[slot], STAGE);
                    bulk_g2s(dst, ga, GCB, &full[slot]);
                    bulk_g2s(dst + GCB, gb, GCB, &full[slot]);
                }
            }
            // drain: every issued copy has landed before this thread exits
            const uint32_t first = it > (uint32_t)NST ? it - NST : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % NST], (j / NST) & 1);
            if (!ok) {
                s_err = 1;
                if (a.step) atomicOr(&a.step->error, 2u);
            }
        }
        return;
    }

    // ---------------- consumers: the activation depends on the previous kernel
    pdl_wait();
    float scale = 1.f;
    if (a.norm_w) {  // RMSNorm (src/math/ops.rs:5-12)
        float ss = 0.f;
#pragma unroll 8
        for (int k = tid; k < K; k += MV_CONSUMERS) {
            const float v = a.x[k];
            ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        consumer_sync();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < MV_CWARPS; ++w) tot += red[w];
        scale = 1.0f / sqrtf(tot / (float)K + a.eps);
    }
    // normalised input element e ((x * scale) * w, the reference's rounding order)
    auto xin = [&](int e) -> float {
        if (e >= K) return 0.f;
        float v = a.x[e];
        if (a.norm_w) v = __fmul_rn(__fmul_rn(v, scale), a.norm_w[e]);
        return v;
    };
    float sdown = 1.f, sup = 1.f;  // f16 range scale of the staged input (kStageBig)
    for (int tries = 0;; ++tries) {
        // One coalesced pass, one 32-element block per warp iteration: lane l holds
        // element 32j + l, writes its f16 hi / lo halves into the B-fragment slots
        // and the warp sums the block for the zero-point term (per 16 for Q6_K
        // sub-blocks, per 32 otherwise).
        const int lane = tid & 31, warp = tid >> 5;
        half* xh = (half*)stage_x;
        const int s16 = lane >> 4, r16 = lane & 15;
        const int m = 2 * s16 + (r16 >> 3), t = (r16 & 7) >> 1, hp = r16 & 1;
        bool big = false;
#pragma unroll 4
        for (int j = warp; j < KP / 32; j += MV_CONSUMERS / 32) {
            const float v = xin(32 * j + lane) * sdown;
            if (TYPE == GT_F32) {
                stage_x[32 * j + lane] = v;
                continue;
            }
            big |= fabsf(v) >= kStageBig;
            // Q4_0 high-nibble positions (k 2t+8, 2t+9) meet A = 16 u 2^-24: pre-divide by 16
            const float vv = (TYPE == GT_Q4_0 && (r16 >> 3)) ? v * 0.0625f : v;
            const half hi = __float2half_rn(vv);
            const half lo = __float2half_rn(vv - __half2float(hi));
            xh[((j * 8 + t) * 4 + m) * 2 + hp] = hi;
            xh[((j * 8 + 4 + t) * 4 + m) * 2 + hp] = lo;
            float s = v;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (TYPE == GT_Q6_K) {
                if (r16 == 0) xs16[2 * j + s16] = s;
            } else {
                s += __shfl_xor_sync(0xffffffffu, s, 16);
                if (lane == 0) xs16[j] = s;
            }
        }
        if (!consumer_sync_or(big) || TYPE == GT_F32 || tries == kStageRetries) break;
        sdown *= kStageDown;
        sup *= 1.f / kStageDown;
    }
    pdl_launch();

    const int lane = tid & 31, warp = tid >> 5;
    uint32_t it = 0;
    int buf = 0, ntile = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, buf ^= 1) {
        Acc acc = {0.f, 0.f, 0.f, 0.f};
        bool ok = true;
        for (int c = 0; c < nchunk; ++c, ++it) {
            const int slot = it % NST;
            if (!mbar_wait(&full[slot], (it / NST) & 1)) {
                ok = false;
                break;
            }
            const uint8_t* sA = ring + slot * STAGE;
            const uint8_t* sB = sA + GCB;
            if (TYPE == GT_Q4_0)
                consume_q4_0(sA, sB, (const uint4*)stage_x, xs16, c, acc);
            else if (TYPE == GT_Q8_0)
                consume_q8_0(sA, sB, (const uint4*)stage_x, xs16, c, acc);
            else if (TYPE == GT_Q6_K)
                consume_q6_k(sA, sB, (const uint4*)stage_x, xs16, c, acc);
            else
                consume_f32(sA, sB, stage_x, c, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (!ok) {
            s_err = 1;
            if (a.step) atomicOr(&a.step->error, 2u);
            break;
        }
        // ---- hand the tile's partials to the epilogue warp (double-buffered)
        const int b = buf;
        const uint32_t u = (uint32_t)(ntile >> 1);
        if (!mbar_wait(&tfree[b], (u & 1) ^ 1)) {
            s_err = 1;
            if (a.step) atomicOr(&a.step->error, 2u);
            break;
        }
        float* pb = part + b * MV_CWARPS * 16;
        if (TYPE == GT_F32) {
            const float v = warp_sum(acc.pA);
            if (lane < 16) pb[warp * 16 + lane] = (lane == warp) ? v : 0.f;
        } else if ((lane & 3) == 0) {
            pb[warp * 16 + (lane >> 2)] = fmaf(acc.pA, kTwo24, -Zero<TYPE>::z * acc.qA) * sup;
            pb[warp * 16 + 8 + (lane >> 2)] = fmaf(acc.pB, kTwo24, -Zero<TYPE>::z * acc.qB) * sup;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tdone[b]);
        ++ntile;
    }
}

static int fmt_fixed(int type) {
    switch (type) {
        case GT_Q4_0: return (int)mv_smem_fixed<GT_Q4_0>();
        case GT_Q8_0: return (int)mv_smem_fixed<GT_Q8_0>();
        case GT_Q6_K: return (int)mv_smem_fixed<GT_Q6_K>();
        case GT_F32: return (int)mv_smem_fixed<GT_F32>();
    }
    return 0;
}

size_t matvec_smem_bytes(int type, int K) {
    const int ck = fmt_ck(type);
    if (!ck) return 0;
    const int kp = ceil_div_h(K, ck) * ck;
    return (size_t)fmt_fixed(type) + mv_smem_per_k(kp);
}

static const int kMaxSmem = 220 * 1024;

cudaError_t matvec_configure() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem))) return e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem))) return e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem))) return e;
    if ((e = cudaFuncSetAttribute(k_matvec<GT_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem))) return e;
    return cudaSuccess;
}

int matvec_max_k(int type) {
    const int ck = fmt_ck(type);
    if (!ck) return 0;
    // (kMaxSmem - fixed) / (4 + 4/16) bytes per input element, in whole chunks
    const double per = 4.0 + 0.25;
    const int k = (int)((kMaxSmem - fmt_fixed(type)) / per);
    return k / ck * ck;
}

int matvec_ctas_per_sm(int, int) { return 1; }

cudaError_t launch_matvec(const MatvecArgs& a, int type, int max_ctas, cudaStream_t s, bool pdl) {
    if (a.ntiles <= 0) return cudaSuccess;
    const int grid = a.ntiles < max_ctas ? a.ntiles : max_ctas;
    const size_t sm = matvec_smem_bytes(type, a.K);
    if (!sm || sm > (size_t)kMaxSmem) return cudaErrorInvalidValue;
    (void)fmt_nst;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (type) {
        case GT_F32: return cudaLaunchKernelEx(&cfg, k_matvec<GT_F32>, a);
        case GT_Q8_0: return cudaLaunchKernelEx(&cfg, k_matvec<GT_Q8_0>, a);
        case GT_Q4_0: return cudaLaunchKernelEx(&cfg, k_matvec<GT_Q4_0>, a);
        case GT_Q6_K: return cudaLaunchKernelEx(&cfg, k_matvec<GT_Q6_K>, a);
    }
    return cudaErrorInvalidValue;
}

// ============================================================================
// The per-token kernel
// ============================================================================
//
// One launch runs a whole decode step (src/model/llama.rs:96-183, then the
// logits of :89 or the final norm of :181) as a list of phases: per layer
// q/k/v -> attention -> o-proj -> gate/up -> down, then the output projection.
// One CTA per SM with the roles of k_matvec: a producer warp streaming packed
// weights through a shared-memory ring, 16 consumer warps, an epilogue warp.
// The producer walks the weights of ALL of the CTA's matvec phases in order, so
// while the consumers wait for the previous phase to finish grid-wide, the ring
// is already filling with the next phase's weights; there is no launch, no
// pipeline fill and no tail between the ~5 L phases of a token.
//
// Phase boundaries are grid barriers on 64-bit arrival counters in global
// memory. When a CTA's outputs of phase p are written (by its epilogue warp, or
// by its consumers for attention) it fences and adds 1 to bars[p]; the consumers
// of phase p+1 wait until bars[p] reaches (epoch + 1) * gridDim.x, epoch being
// the number of earlier launches. Counters are never reset. Every CTA must be
// resident at once (one CTA per SM); every wait is bounded (2 s) and on expiry
// the kernel records an error in StepParams::error and leaves.
//
// Cross-CTA data (residual stream, q, K/V rows, partials) are read with
// ld.global.cg (L2), never from a possibly stale L1 line.

constexpr int TK_STAGE = 2 * Fmt<GT_Q4_0>::GCB;  // largest two-group stage of the four formats
static_assert(2 * Fmt<GT_Q8_0>::GCB <= TK_STAGE && 2 * Fmt<GT_Q6_K>::GCB <= TK_STAGE &&
                  2 * Fmt<GT_F32>::GCB <= TK_STAGE,
              "ring stage too small");
constexpr int TK_NORM_REGS = 16;               // normed-input registers per thread: K <= 16 * 512
constexpr int TK_MAX_SPLIT = 8;                // position splits per kv head in attention
#ifndef TK_SPLIT_POS
#define TK_SPLIT_POS 128  // positions per split the split count aims for (64: -0.7 % tok/s at the bench positions)
#endif
#ifndef TK_ATT_PER_HEAD
#define TK_ATT_PER_HEAD 1                      // attention items per query head (else per kv head)
#endif
#ifndef TK_PAIR_CHUNKS
#define TK_PAIR_CHUNKS 1                       // consume two ring stages per step
#endif

// Splits of a kv head's positions this step: about TK_SPLIT_POS positions each,
// at most `nsplit` (short sequences need no cross-CTA merge at all).
__device__ __forceinline__ int tk_splits(int nsplit, uint32_t pos) {
    const int want = ((int)pos + TK_SPLIT_POS) / TK_SPLIT_POS;  // ceil((pos + 1) / TK_SPLIT_POS)
    return want < nsplit ? want : nsplit;
}
constexpr int TK_BAR_BYTES = 64 * 8;           // room for the ring's mbarriers (nst <= 30)
constexpr int TK_TAIL_BYTES = (2 * MV_CWARPS * 16 + 16 + 32) * 4;
constexpr uint64_t TK_WAIT_NS = 2000000000ull;

__host__ __device__ constexpr int ck_of(int type) {
    return type == GT_Q4_0 ? Fmt<GT_Q4_0>::CK
                           : (type == GT_Q8_0 ? Fmt<GT_Q8_0>::CK
                                              : (type == GT_Q6_K ? Fmt<GT_Q6_K>::CK : Fmt<GT_F32>::CK));
}
__host__ __device__ constexpr int gcb_of(int type) {
    return type == GT_Q4_0 ? Fmt<GT_Q4_0>::GCB
                           : (type == GT_Q8_0 ? Fmt<GT_Q8_0>::GCB
                                              : (type == GT_Q6_K ? Fmt<GT_Q6_K>::GCB : Fmt<GT_F32>::GCB));
}

// Bounded spin of one thread until *bar >= target.
__device__ __noinline__ bool grid_wait_one(const unsigned long long* bar, unsigned long long target, bool sys) {
    auto ld = [&]() { return sys ? ld_acquire_sys_u64(bar) : ld_acquire_u64(bar); };
    if (ld() >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 16; ++i)
            if (ld() >= target) return true;
        if (globaltimer_ns() - t0 > TK_WAIT_NS) return false;
    }
}
// One CTA's arrival at phase p's barrier. A cross-rank phase (xrank) arrives at
// system scope so that its stores into the peers' memory travel with the
// release chain: local counter -> CTA 0 -> one add on every rank's rank counter
// (tk_rank_wait), instead of 148 remote adds per rank on one address.
__device__ __forceinline__ void tk_arrive(const TokenArgs& a, int p, bool xrank) {
    if (xrank)
        red_release_sys_add_u64(&a.bars[p], 1ull);
    else
        red_release_add_u64(&a.bars[p], 1ull);
}
// Cross-rank barrier of phase p (thread 0 of each CTA): CTA 0 waits for this
// rank's CTAs and signals every rank; then every CTA waits for all ranks.
__device__ __forceinline__ bool tk_rank_wait(const TokenArgs& a, int p, unsigned long long target) {
    if (blockIdx.x == 0) {
        if (!grid_wait_one(&a.bars[p], target, true)) return false;
        for (int r = 0; r < a.tp; ++r) red_release_sys_add_u64(a.prbars[r] + p, 1ull);
    }
    return grid_wait_one(&a.rbars[p], (target / gridDim.x) * (unsigned)a.tp, true);
}
// Bounded spin until the shared counter reaches v.
__device__ __forceinline__ bool smem_wait_geq(const volatile int* p, int v) {
    if (*p >= v) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (*p >= v) return true;
        if (globaltimer_ns() - t0 > TK_WAIT_NS) return false;
    }
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Bounded wait of one thread until the shared counter reaches v, sleeping between
// polls (the waiter shares its sub-partition's issue slots with consumer warps).
__device__ __forceinline__ bool smem_wait_geq_sleep(const volatile int* p, int v) {
    if (*p >= v) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(100);
        if (*p >= v) return true;
        if (globaltimer_ns() - t0 > TK_WAIT_NS) return false;
    }
}
__device__ __forceinline__ void bulk_g2s_evict_first(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

struct TkShared {
    int err;      // any role gave up on a wait (set at any time)
    int stop;     // consumer thread 0's snapshot of err at a phase start, read after the sync
    int started;  // last phase the consumers entered (epilogue warp follows it)
    int staged;   // last phase whose input the consumers have staged (producer follows it)
    float sup;    // the staged input's f16 range factor (kStageBig), applied to the row sums
};

// Profiling stamps (TokenArgs::stamps): [phase][cta][4] = phase entered,
// inputs staged, compute done, arrival at the phase's barrier.
__device__ __forceinline__ void tk_stamp(const TokenArgs& a, int p, int k) {
    if (a.stamps) a.stamps[((size_t)p * gridDim.x + blockIdx.x) * 4 + k] = globaltimer_ns();
}

__device__ __forceinline__ void tk_fail(const TokenArgs& a, TkShared* sh, uint32_t code) {
    *(volatile int*)&sh->err = 1;
    atomicOr(&a.step->error, code);
}

// Inputs of phase P that do not depend on the previous phase, copied into the
// staging area with cp.async while thread 0 waits at the barrier: the norm
// weights of a normed matvec (the same float4s each thread reads in tk_stage).
// (Prefetching attention's cached K/V rows the same way measured slower.)
// The per-token kernel's dynamic shared memory: the weight ring, its mbarriers
// (full, empty; tdone, tfree for the epilogue hand-off), the staging union U,
// the epilogue's partials, the tile's reduced rows and a reduction scratch.
struct TkSmem {
    uint8_t* ring;
    uint64_t *full, *empty, *tdone, *tfree;
    float *U, *part, *res, *red;
};
__device__ __forceinline__ TkSmem tk_smem(const TokenArgs& a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nst = (uint32_t)a.nst;
    TkSmem m;
    m.ring = smem;
    m.full = (uint64_t*)(smem + (size_t)nst * TK_STAGE);
    m.empty = m.full + nst;
    m.tdone = m.empty + nst;  // [2]
    m.tfree = m.tdone + 2;    // [2]
    m.U = (float*)(smem + (size_t)nst * TK_STAGE + TK_BAR_BYTES);
    m.part = m.U + a.union_bytes / 4;     // [2][16][16]
    m.res = m.part + 2 * MV_CWARPS * 16;  // 16
    m.red = m.res + 16;                   // 32
    return m;
}

// Phase entry, called by the consumers from inside the phase's code once its
// prologue is done (that code is then fetched while the CTA waits, not after
// the barrier): thread 0 waits for the previous phase's barrier and tells the
// epilogue warp the phase has started; every consumer warp then reads one stop
// snapshot. False: the kernel is stopping.
__device__ __forceinline__ bool tk_gate(const TokenArgs& a, int p, TkShared* sh, unsigned long long target) {
    if (p == 0) {
        if (threadIdx.x == 0) tk_stamp(a, 0, 0);
        return true;
    }
    if (threadIdx.x == 0) {
        const bool xr = a.ph[p - 1].xrank != 0;
        // the acquire load orders the phase's reads; consumer_sync passes it on
        if (!(xr ? tk_rank_wait(a, p - 1, target) : grid_wait_one(&a.bars[p - 1], target, false)))
            tk_fail(a, sh, 4u);
        *(volatile int*)&sh->started = p;
        sh->stop = *(volatile int*)&sh->err;
        tk_stamp(a, p, 0);
    }
    consumer_sync();
    return !sh->stop;
}

__device__ __noinline__ void tk_prefetch(const TokenArgs& a, const TokenPhase& P, float* U) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (P.kind == PH_MATVEC) {
        const MatvecArgs& m = P.mv;
        if (!m.norm_w || (m.K & 3) || (int)blockIdx.x >= m.ntiles) return;
        const int ck = ck_of(P.type), KP = (m.K + ck - 1) / ck * ck;
        float* wpre = U + KP + KP / 16;
        for (int r = warp; r < KP / 128; r += MV_CWARPS) {
            const int e0 = 128 * r + 4 * lane;
            if (e0 < m.K) cp_async16(wpre + e0, m.norm_w + e0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
}

// Four consecutive inputs e0 .. e0+3 (e0 % 4 == 0) into the staged layout
// consume_* reads: f16 hi / lo B fragments per 32-element block (Q4_0's
// high-nibble slots pre-divided by 16) or plain floats (F32).
template <int TYPE>
__device__ __forceinline__ void tk_put4(float* U, int e0, float4 v) {
    if (TYPE == GT_F32) {
        *(float4*)(U + e0) = v;
        return;
    }
    const int j = e0 >> 5, k0 = e0 & 31;
    const int r0 = k0 & 15, mq = 2 * (k0 >> 4) + (r0 >> 3), t0 = (r0 & 7) >> 1;
    float a0 = v.x, a1 = v.y, a2 = v.z, a3 = v.w;
    if (TYPE == GT_Q4_0 && (r0 >> 3)) {
        a0 *= 0.0625f;
        a1 *= 0.0625f;
        a2 *= 0.0625f;
        a3 *= 0.0625f;
    }
    uint32_t h01, l01, h23, l23;
    split_pair(a0, a1, h01, l01);
    split_pair(a2, a3, h23, l23);
    uint32_t* xw = (uint32_t*)U;  // one 32-bit word = the (hp 0, hp 1) half pair
    xw[(j * 8 + t0) * 4 + mq] = h01;
    xw[(j * 8 + t0 + 1) * 4 + mq] = h23;
    xw[(j * 8 + 4 + t0) * 4 + mq] = l01;
    xw[(j * 8 + 4 + t0 + 1) * 4 + mq] = l23;
}

// Block sums S of the zero-point term: lane l of a warp holds elements 4l..4l+3
// of a 128-element run, so 8 lanes make a 32-element block (4 a 16-element half).
template <int TYPE>
__device__ __forceinline__ void tk_sums(float* xs16, int e0, float4 v, int lane) {
    if (TYPE == GT_F32) return;
    float s = (v.x + v.y) + (v.z + v.w);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (TYPE == GT_Q6_K) {
        if ((lane & 3) == 0) xs16[e0 >> 4] = s;
        return;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if ((lane & 7) == 0) xs16[e0 >> 5] = s;
}

// Stage phase P's input for the format TYPE: RMSNorm with P.mv.norm_w when set
// (src/math/ops.rs:5-12, (x * s) * w), the token's embedding row for the first
// phase (src/model/weights.rs:57-62). All global loads of a round are issued
// before any is used (one L2 round trip per round, not one per element).
#ifndef TK_ROUND
#define TK_ROUND 4  // 128-element runs per warp and round
#endif
// Input sources, one instantiation each (only the code a phase uses is fetched:
// staging runs once per phase and is latency-bound, instruction fetch included).
enum : int { SRC_PLAIN = 0, SRC_EMBED = 1, SRC_XSUM = 2, SRC_ATT = 3 };
// The staging pass of tk_stage_src at f16 range scale `sdown` (1 in range,
// then 2^-16 steps, kStageBig); true when an element of the scaled input is
// still out of range. Ends at the consumers' barrier (which ORs the flag).
template <int TYPE, int SRC>
__device__ __forceinline__ bool tk_stage_body(const TokenArgs& a, const TokenPhase& P, uint32_t tok, uint32_t pos,
                                              float* U, float* red, float sdown) {
    const MatvecArgs& m = P.mv;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = m.K, KP = ((K + Fmt<TYPE>::CK - 1) / Fmt<TYPE>::CK) * Fmt<TYPE>::CK, nrun = KP / 128;
    float* xs16 = U + KP;
    const uint8_t* erow = nullptr;
    if (SRC == SRC_EMBED)
        erow = a.embd + (size_t)tok * (K / gguf_block_elems(a.embd_type)) * gguf_block_bytes(a.embd_type);
    // tensor parallel: x = xbuf[xsrc] + the ranks' partial sums, in rank order
    // (every rank computes the same bits); CTA 0 keeps it in xbuf[xdst]
    constexpr bool xs = SRC == SRC_XSUM;
    const float* xsrc = xs ? a.xbuf[P.xsrc] : nullptr;
    const float* rxs = xs ? a.prx[a.rank] + (size_t)P.xslot * a.tp * a.E : nullptr;
    auto load4 = [&](int e0) -> float4 {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (xs) {
            if (e0 < K) {  // K = E, a multiple of 4
                v = __ldcg((const float4*)(xsrc + e0));
                for (int r = 0; r < a.tp; ++r) {
                    const float4 d = __ldcg((const float4*)(rxs + (size_t)r * a.E + e0));
                    v = make_float4(v.x + d.x, v.y + d.y, v.z + d.z, v.w + d.w);
                }
                if (blockIdx.x == 0) *(float4*)(a.xbuf[P.xdst] + e0) = v;
            }
        } else if constexpr (SRC == SRC_EMBED) {
            float t[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) t[i] = e0 + i < K ? dequant_elem(a.embd_type, erow, e0 + i) : 0.f;
            v = make_float4(t[0], t[1], t[2], t[3]);
            if (blockIdx.x == 0 && e0 < K) {  // the residual stream starts as the embedding
                float* x0 = a.tp > 1 ? a.xbuf[P.xdst] : a.x;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (e0 + i < K) x0[e0 + i] = t[i];
            }
        } else if (e0 + 4 <= K && !(K & 3)) {
            v = __ldcg((const float4*)(m.x + e0));
        } else {
            float t[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) t[i] = e0 + i < K ? __ldcg(m.x + e0 + i) : 0.f;
            v = make_float4(t[0], t[1], t[2], t[3]);
        }
        return v;
    };
    auto loadw4 = [&](int e0) -> float4 {
        if (e0 + 4 <= K && !(K & 3)) return __ldg((const float4*)(m.norm_w + e0));
        float t[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) t[i] = e0 + i < K ? __ldg(m.norm_w + e0 + i) : 0.f;
        return make_float4(t[0], t[1], t[2], t[3]);
    };
    // normed phases: the norm weights were copied to wpre before the barrier
    // (tk_prefetch) when K is a multiple of 4
    const float* wpre = (m.norm_w && !(K & 3)) ? U + KP + KP / 16 : nullptr;
    bool big = false;
    if constexpr (SRC == SRC_ATT) {
        // the attention output, merged from the softmax partials of each head's
        // splits (src/math/ops.rs:15-25 normalisation, applied to the merged sums):
        // per head the weights exp(m_q - M) / L, then o = sum_q w_q o_q
        const int hd = m.hd, nh = K / hd, ns = tk_splits(a.nsplit, pos), hs = hd + 4;
        float* wsm = xs16 + KP / 16;  // [nh][ns]
        for (int h = tid; h < nh; h += MV_CONSUMERS) {
            const float* base = a.att_part + (size_t)h * a.nsplit * hs;
            float mv[TK_MAX_SPLIT], lv[TK_MAX_SPLIT];
            float M = -INFINITY;
#pragma unroll
            for (int q = 0; q < TK_MAX_SPLIT; ++q) {
                mv[q] = q < ns ? __ldcg(base + q * hs) : -INFINITY;
                lv[q] = q < ns ? __ldcg(base + q * hs + 1) : 0.f;
            }
#pragma unroll
            for (int q = 0; q < TK_MAX_SPLIT; ++q) M = fmaxf(M, mv[q]);
            float L = 0.f;
#pragma unroll
            for (int q = 0; q < TK_MAX_SPLIT; ++q) {
                mv[q] = mv[q] != -INFINITY ? expf(mv[q] - M) : 0.f;
                L = fmaf(lv[q], mv[q], L);
            }
#pragma unroll
            for (int q = 0; q < TK_MAX_SPLIT; ++q)
                if (q < ns) wsm[h * ns + q] = mv[q] / L;
        }
        consumer_sync();
#pragma unroll 2
        for (int r = warp; r < nrun; r += MV_CWARPS) {
            const int e0 = 128 * r + 4 * lane;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e0 < K) {
                const int h = e0 / hd;
                const float* ob = a.att_part + (size_t)h * a.nsplit * hs + 4 + e0 % hd;
#pragma unroll
                for (int q = 0; q < TK_MAX_SPLIT; ++q) {
                    if (q < ns) {
                        const float4 o = __ldcg((const float4*)(ob + q * hs));
                        const float w = wsm[h * ns + q];
                        v = make_float4(fmaf(o.x, w, v.x), fmaf(o.y, w, v.y), fmaf(o.z, w, v.z), fmaf(o.w, w, v.w));
                    }
                }
            }
            v = scale4(v, sdown);
            big |= big4(v);
            tk_put4<TYPE>(U, e0, v);
            tk_sums<TYPE>(xs16, e0, v, lane);
        }
    } else if (m.norm_w) {
        // the whole input in registers (K <= 16 * 128 * 4 = 8192), one reduction
        float4 xv[TK_NORM_REGS / 4], wv[TK_NORM_REGS / 4];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < TK_NORM_REGS / 4; ++i) {
            const int r = warp + MV_CWARPS * i, e0 = 128 * r + 4 * lane;
            xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            wv[i] = xv[i];
            if (r < nrun) {
                xv[i] = load4(e0);
                wv[i] = wpre ? (e0 < K ? *(const float4*)(wpre + e0) : make_float4(0.f, 0.f, 0.f, 0.f)) : loadw4(e0);
            }
        }
#pragma unroll
        for (int i = 0; i < TK_NORM_REGS / 4; ++i)
            ss = fmaf(xv[i].w, xv[i].w, fmaf(xv[i].z, xv[i].z, fmaf(xv[i].y, xv[i].y, fmaf(xv[i].x, xv[i].x, ss))));
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        consumer_sync();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < MV_CWARPS; ++w) tot += red[w];
        const float sc = 1.0f / sqrtf(tot / (float)K + m.eps);
#pragma unroll
        for (int i = 0; i < TK_NORM_REGS / 4; ++i) {
            const int r = warp + MV_CWARPS * i, e0 = 128 * r + 4 * lane;
            if (r < nrun) {
                const float4 v = scale4(make_float4(__fmul_rn(__fmul_rn(xv[i].x, sc), wv[i].x),
                                                    __fmul_rn(__fmul_rn(xv[i].y, sc), wv[i].y),
                                                    __fmul_rn(__fmul_rn(xv[i].z, sc), wv[i].z),
                                                    __fmul_rn(__fmul_rn(xv[i].w, sc), wv[i].w)),
                                        sdown);
                big |= big4(v);
                tk_put4<TYPE>(U, e0, v);
                tk_sums<TYPE>(xs16, e0, v, lane);
            }
        }
    } else {
        for (int r0 = 0; r0 < nrun; r0 += MV_CWARPS * TK_ROUND) {
            float4 xv[TK_ROUND];
#pragma unroll
            for (int i = 0; i < TK_ROUND; ++i) {
                const int r = r0 + warp + MV_CWARPS * i;
                xv[i] = r < nrun ? load4(128 * r + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < TK_ROUND; ++i) {
                const int r = r0 + warp + MV_CWARPS * i;
                if (r < nrun) {
                    const float4 v = scale4(xv[i], sdown);
                    big |= big4(v);
                    tk_put4<TYPE>(U, 128 * r + 4 * lane, v);
                    tk_sums<TYPE>(xs16, 128 * r + 4 * lane, v, lane);
                }
            }
        }
    }
    return consumer_sync_or(big);
}

template <int TYPE, int SRC>
__device__ __noinline__ bool tk_stage_src(const TokenArgs& a, const TokenPhase& P, uint32_t tok, uint32_t pos,
                                          float* U, float* red, int p, TkShared* sh, unsigned long long target) {
    const MatvecArgs& m = P.mv;
    const int K = m.K, KP = ((K + Fmt<TYPE>::CK - 1) / Fmt<TYPE>::CK) * Fmt<TYPE>::CK;
    // normed phases: the norm weights were copied to wpre before the barrier
    // (tk_prefetch) when K is a multiple of 4
    if (m.norm_w && !(K & 3)) cp_async_commit_wait();
    (void)KP;
    if (!tk_gate(a, p, sh, target)) return false;
    float sup = 1.f;
    if (tk_stage_body<TYPE, SRC>(a, P, tok, pos, U, red, 1.f) && TYPE != GT_F32) {
        sup = 1.f / kStageDown;
        if (tk_stage_body<TYPE, SRC>(a, P, tok, pos, U, red, kStageDown)) atomicOr(&a.step->error, 8u);
    }
    if (threadIdx.x == 0) sh->sup = sup;  // read after the consumers' next barrier
    return true;
}

template <int TYPE>
__device__ __forceinline__ bool tk_stage(const TokenArgs& a, const TokenPhase& P, uint32_t tok, uint32_t pos, float* U,
                                         float* red, int p, TkShared* sh, unsigned long long target) {
    if (P.embed_in) return tk_stage_src<TYPE, SRC_EMBED>(a, P, tok, pos, U, red, p, sh, target);
    if (P.att_merge) return tk_stage_src<TYPE, SRC_ATT>(a, P, tok, pos, U, red, p, sh, target);
    if (a.tp > 1 && P.xsum) return tk_stage_src<TYPE, SRC_XSUM>(a, P, tok, pos, U, red, p, sh, target);
    return tk_stage_src<TYPE, SRC_PLAIN>(a, P, tok, pos, U, red, p, sh, target);
}

// tk_matvec results
enum : int { TK_DONE = 0, TK_FAILED = 1, TK_STOPPED = 2 };

// Consumers of one matvec phase: stage the input, then every tile of this CTA.
template <int TYPE>
__device__ __noinline__ int tk_matvec(const TokenArgs& a, const TokenPhase& P, int p, uint32_t tok, uint32_t pos,
                                      unsigned long long target, TkShared* sh, uint32_t& slot_io, uint32_t& par_io,
                                      int& ntile_io) {
    const TkSmem S = tk_smem(a);
    uint8_t* ring = S.ring;
    uint64_t *full = S.full, *empty = S.empty, *tfree = S.tfree, *tdone = S.tdone;
    float *U = S.U, *part = S.part, *red = S.red;
    const MatvecArgs& m = P.mv;
    if ((int)blockIdx.x >= m.ntiles)  // no tiles here: read nothing
        return tk_gate(a, p, sh, target) ? TK_DONE : TK_STOPPED;
    // The ring position lives in registers for the phase: the caller's variables
    // sit in the stack frame (local memory), and every asm statement with a
    // memory clobber in the loop would reload them from there.
    uint32_t slot = slot_io, par = par_io;
    int ntile = ntile_io;
    if (!tk_stage<TYPE>(a, P, tok, pos, U, red, p, sh, target)) return TK_STOPPED;
    if (threadIdx.x == 0) {
        *(volatile int*)&sh->staged = p;  // the producer may stream the rest of this phase
        tk_stamp(a, p, 1);
    }
    constexpr int GCB = Fmt<TYPE>::GCB, CK = Fmt<TYPE>::CK;
    const int nchunk = (m.K + CK - 1) / CK, KP = nchunk * CK;
    const float* stage_x = U;
    const float* xs16 = U + KP;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nst = (uint32_t)a.nst;
    auto consume = [&](const uint8_t* sA, int c, Acc& acc) {
        const uint8_t* sB = sA + GCB;
        if (TYPE == GT_Q4_0)
            consume_q4_0(sA, sB, (const uint4*)stage_x, xs16, c, acc);
        else if (TYPE == GT_Q8_0)
            consume_q8_0(sA, sB, (const uint4*)stage_x, xs16, c, acc);
        else if (TYPE == GT_Q6_K)
            consume_q6_k(sA, sB, (const uint4*)stage_x, xs16, c, acc);
        else
            consume_f32(sA, sB, stage_x, c, acc);
    };
    auto next = [&](uint32_t& s_, uint32_t& p_) {
        if (++s_ == nst) {
            s_ = 0;
            p_ ^= 1u;
        }
    };
    for (int t = blockIdx.x; t < m.ntiles; t += gridDim.x) {
        Acc acc = {0.f, 0.f, 0.f, 0.f};
        int c = 0;
#if TK_PAIR_CHUNKS
        // two stages per step, two independent accumulators: twice the MMA and FMA
        // chains in flight per warp (the consumers are latency-bound, not issue-bound)
        for (; c + 1 < nchunk; c += 2) {
            uint32_t s2 = slot, p2 = par;
            next(s2, p2);
            if (!mbar_wait(&full[slot], par) || !mbar_wait(&full[s2], p2)) return TK_FAILED;
            Acc acc2 = {0.f, 0.f, 0.f, 0.f};
            consume(ring + slot * TK_STAGE, c, acc);
            consume(ring + s2 * TK_STAGE, c + 1, acc2);
            acc.pA += acc2.pA;
            acc.qA += acc2.qA;
            acc.pB += acc2.pB;
            acc.qB += acc2.qB;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[slot]);
                mbar_arrive(&empty[s2]);
            }
            slot = s2;
            par = p2;
            next(slot, par);
        }
#endif
        for (; c < nchunk; ++c) {
            if (!mbar_wait(&full[slot], par)) return TK_FAILED;
            consume(ring + slot * TK_STAGE, c, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            next(slot, par);
        }
        // hand the tile's partials to the epilogue warp (double-buffered)
        const int b = ntile & 1;
        if (!mbar_wait(&tfree[b], ((uint32_t)(ntile >> 1) & 1u) ^ 1u)) return TK_FAILED;
        float* pb = part + b * MV_CWARPS * 16;
        if (TYPE == GT_F32) {
            const float v = warp_sum(acc.pA);
            if (lane < 16) pb[warp * 16 + lane] = (lane == warp) ? v : 0.f;
        } else if ((lane & 3) == 0) {
            pb[warp * 16 + (lane >> 2)] = fmaf(acc.pA, kTwo24, -Zero<TYPE>::z * acc.qA);
            pb[warp * 16 + 8 + (lane >> 2)] = fmaf(acc.pB, kTwo24, -Zero<TYPE>::z * acc.qB);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tdone[b]);
        ++ntile;
    }
    slot_io = slot;
    par_io = par;
    ntile_io = ntile;
    if (threadIdx.x == 0) tk_stamp(a, p, 2);
    return TK_DONE;
}

// Attention for one (kv head, position split) item per CTA (src/model/llama.rs:
// 135-155): scores q.k * scale, softmax, sum of p V. Each warp keeps online
// softmax state (max m, sum l, unnormalised o) over its positions, with
// TK_ATT_UNROLL positions' K/V loads in flight; the warps merge in shared
// memory and the split writes its partial to att_part. The o-proj phase merges
// the splits while it stages its input (cheaper, measured, than an arrival
// counter and a merge by the last split's CTA).
// Instantiated per query-head group size G, so the unrolled loops hold exactly
// the heads a model has (the kernel's code must stay small enough for the
// instruction cache: every phase of every layer runs through it).
#ifndef TK_ATT_UNROLL
#define TK_ATT_UNROLL 4  // positions per warp and round
#endif
// The f16-cache round loop of tk_attention: LPR = hd/8 lanes hold one
// position's row (8 halves, one 16-byte load each), so one load instruction of
// the warp covers R = 32/LPR positions; a round is TK_ATT_UNROLL such loads for
// K and V. Each lane keeps the V sum of its own row group's positions; the
// running max and sum are warp-wide (maxima and sums cross the row groups by
// shuffles), and the groups' V sums are added at the end. Writes the warp's
// (m, l, o) record to ws like the f32 loop.
template <int G, int LPR>
__device__ __forceinline__ void tk_att_f16(const AttnArgs& A, const float* qs, float* ws, int p0, int p1, int kh,
                                           float (&m)[G], float (&l)[G]) {
    constexpr int R = 32 / LPR, RU = TK_ATT_UNROLL, hd = 8 * LPR;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gi = lane / LPR, d0 = 8 * (lane % LPR), hs = hd + 4;
    float oh[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) oh[g][e] = 0.f;
    const size_t hoff = (size_t)kh * hd + d0;
    for (int t0 = p0 + warp; t0 < p1; t0 += MV_CWARPS * R * RU) {
        uint4 kr[RU], vr[RU];
#pragma unroll
        for (int u = 0; u < RU; ++u) {
            const int t = t0 + (u * R + gi) * MV_CWARPS;
            kr[u] = make_uint4(0u, 0u, 0u, 0u);
            vr[u] = kr[u];
            if (t < p1) {
                const size_t i = (size_t)t * A.kv_dim + hoff;
                kr[u] = __ldcg((const uint4*)((const __half*)A.kc + i));
                vr[u] = __ldcg((const uint4*)((const __half*)A.vc + i));
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float4 qa = *(const float4*)(qs + g * hd + d0), qb = *(const float4*)(qs + g * hd + d0 + 4);
            const float q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            float sc[RU];
#pragma unroll
            for (int u = 0; u < RU; ++u) {
                const __half2* h = reinterpret_cast<const __half2*>(&kr[u]);
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(h[e]);
                    d = fmaf(q[2 * e], f.x, fmaf(q[2 * e + 1], f.y, d));
                }
                sc[u] = d;
            }
#pragma unroll
            for (int off = LPR / 2; off > 0; off >>= 1)
#pragma unroll
                for (int u = 0; u < RU; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
            float mx = -INFINITY;
#pragma unroll
            for (int u = 0; u < RU; ++u) {
                sc[u] = t0 + (u * R + gi) * MV_CWARPS < p1 ? sc[u] * A.scale : -INFINITY;
                mx = fmaxf(mx, sc[u]);
            }
#pragma unroll
            for (int off = LPR; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            mx = fmaxf(mx, m[g]);  // finite: position t0 is in range
            const float cr = expf(m[g] - mx);
            float ps = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) oh[g][e] *= cr;
#pragma unroll
            for (int u = 0; u < RU; ++u) {
                const float pe = expf(sc[u] - mx);
                ps += pe;
                const __half2* h = reinterpret_cast<const __half2*>(&vr[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(h[e]);
                    oh[g][2 * e] = fmaf(pe, f.x, oh[g][2 * e]);
                    oh[g][2 * e + 1] = fmaf(pe, f.y, oh[g][2 * e + 1]);
                }
            }
#pragma unroll
            for (int off = LPR; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l[g] = fmaf(l[g], cr, ps);
            m[g] = mx;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int off = LPR; off < 32; off <<= 1) oh[g][e] += __shfl_xor_sync(0xffffffffu, oh[g][e], off);
        float* w = ws + (warp * G + g) * hs;
        if (lane == 0) {
            w[0] = m[g];
            w[1] = l[g];
        }
        if (gi == 0) {
            *(float4*)(w + 4 + d0) = make_float4(oh[g][0], oh[g][1], oh[g][2], oh[g][3]);
            *(float4*)(w + 8 + d0) = make_float4(oh[g][4], oh[g][5], oh[g][6], oh[g][7]);
        }
    }
}

template <int G, bool KV16>
__device__ __noinline__ bool tk_attention(const TokenArgs& a, const AttnArgs& A, int p, uint32_t pos, float* U,
                                          TkShared* sh, unsigned long long target) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nsplit = a.nsplit, ns = tk_splits(nsplit, pos);
    // item = (G consecutive query heads of one kv head, position split)
    if ((int)blockIdx.x >= A.n_head / G * ns) return tk_gate(a, p, sh, target);
    const int group = A.n_head / A.n_kv, hd = A.hd, hs = hd + 4;
    const int h0 = (blockIdx.x / ns) * G, s = blockIdx.x % ns, kh = h0 / group;
    // partial records {m, l, pad, pad, o[hd]} (16-byte aligned o), in shared and global memory
    const int seq = (int)pos + 1;
    const int per = (seq + ns - 1) / ns;
    const int p0 = s * per, p1 = min(seq, p0 + per);
    float* qs = U;           // [G][hd]
    float* ws = U + G * hd;  // [16 warps][G][hd + 4]
    const float* qsrc = A.q + (size_t)h0 * hd;
    if (!tk_gate(a, p, sh, target)) return false;
    for (int i = tid; i < G * hd; i += MV_CONSUMERS) qs[i] = __ldcg(qsrc + i);
    consumer_sync();
    if (tid == 0) tk_stamp(a, p, 1);

    const bool act = 4 * lane < hd;
    float m[G], l[G], o[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    }
    if constexpr (KV16) {
        if (hd == 128)
            tk_att_f16<G, 16>(A, qs, ws, p0, p1, kh, m, l);
        else if (hd == 64)
            tk_att_f16<G, 8>(A, qs, ws, p0, p1, kh, m, l);
        else
            tk_att_f16<G, 4>(A, qs, ws, p0, p1, kh, m, l);  // hd == 32 (checked on the host)
    } else {
    const size_t hoff = (size_t)kh * hd + 4 * lane;
    for (int t0 = p0 + warp; t0 < p1; t0 += MV_CWARPS * TK_ATT_UNROLL) {
        float4 kv[TK_ATT_UNROLL], vv[TK_ATT_UNROLL];
#pragma unroll
        for (int u = 0; u < TK_ATT_UNROLL; ++u) {
            const int t = t0 + u * MV_CWARPS;
            kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            vv[u] = kv[u];
            if (act && t < p1) {
                const size_t i = (size_t)t * A.kv_dim + hoff;
                kv[u] = __ldcg((const float4*)((const float*)A.kc + i));
                vv[u] = __ldcg((const float4*)((const float*)A.vc + i));
            }
        }
        // the round's positions at once: independent dot products and one
        // rescale of the running state per round (t0 < p1, so the maximum is finite)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float sc[TK_ATT_UNROLL];
            float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (act) q4 = *(const float4*)(qs + g * hd + 4 * lane);
#pragma unroll
            for (int u = 0; u < TK_ATT_UNROLL; ++u)
                sc[u] = act ? fmaf(q4.x, kv[u].x, fmaf(q4.y, kv[u].y, fmaf(q4.z, kv[u].z, q4.w * kv[u].w))) : 0.f;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int u = 0; u < TK_ATT_UNROLL; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
            float mx = m[g];
#pragma unroll
            for (int u = 0; u < TK_ATT_UNROLL; ++u) {
                sc[u] = t0 + u * MV_CWARPS < p1 ? sc[u] * A.scale : -INFINITY;
                mx = fmaxf(mx, sc[u]);
            }
            const float cr = expf(m[g] - mx);
            float ls = l[g] * cr, o0 = o[g][0] * cr, o1 = o[g][1] * cr, o2 = o[g][2] * cr, o3 = o[g][3] * cr;
#pragma unroll
            for (int u = 0; u < TK_ATT_UNROLL; ++u) {
                const float pe = expf(sc[u] - mx);
                ls += pe;
                o0 = fmaf(pe, vv[u].x, o0);
                o1 = fmaf(pe, vv[u].y, o1);
                o2 = fmaf(pe, vv[u].z, o2);
                o3 = fmaf(pe, vv[u].w, o3);
            }
            m[g] = mx;
            l[g] = ls;
            o[g][0] = o0;
            o[g][1] = o1;
            o[g][2] = o2;
            o[g][3] = o3;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        {
            float* w = ws + (warp * G + g) * hs;
            if (lane == 0) {
                w[0] = m[g];
                w[1] = l[g];
            }
            if (act) *(float4*)(w + 4 + 4 * lane) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
        }
    }
    }
    consumer_sync();
    // merge the 16 warps: one thread per (head, dim)
    for (int idx = tid; idx < G * hd; idx += MV_CONSUMERS) {
        const int g = idx / hd, d = idx % hd;
        float M = -INFINITY;
        for (int w = 0; w < MV_CWARPS; ++w) M = fmaxf(M, ws[(w * G + g) * hs]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < MV_CWARPS; ++w) {
                const float* ww = ws + (w * G + g) * hs;
                const float e = expf(ww[0] - M);
                L = fmaf(ww[1], e, L);
                O = fmaf(ww[4 + d], e, O);
            }
        }

        float* dst = a.att_part + ((size_t)(h0 + g) * nsplit + s) * hs;
        if (d == 0) {
            dst[0] = M;
            dst[1] = L;
        }
        dst[4 + d] = O;
    }
    if (tid == 0) tk_stamp(a, p, 2);
    return true;
}

// the cache's element type picks the instantiation (the loads stay branch-free)
template <int G>
__device__ __forceinline__ bool tk_attention_kv(const TokenArgs& a, const AttnArgs& A, int p, uint32_t pos, float* U,
                                                TkShared* sh, unsigned long long target) {
    return A.kv_f16 ? tk_attention<G, true>(a, A, p, pos, U, sh, target)
                    : tk_attention<G, false>(a, A, p, pos, U, sh, target);
}

// Final norm to the hidden state (src/model/llama.rs:181), CTA 0 only.
__device__ __noinline__ bool tk_hidden(const TokenArgs& a, const TokenPhase& P, int p, float* red, TkShared* sh,
                                       unsigned long long target) {
    if (!tk_gate(a, p, sh, target)) return false;
    if (blockIdx.x != 0) return true;
    const int tid = threadIdx.x;
    float* x = a.x;
    if (a.tp > 1 && P.xsum) {  // the last down-proj's partial sums, as in tk_stage
        x = a.xbuf[P.xdst];
        const float* rxs = a.prx[a.rank] + (size_t)P.xslot * a.tp * a.E;
        for (int k = tid; k < a.E; k += MV_CONSUMERS) {
            float v = __ldcg(a.xbuf[P.xsrc] + k);
            for (int r = 0; r < a.tp; ++r) v += __ldcg(rxs + (size_t)r * a.E + k);
            x[k] = v;
        }
        consumer_sync();
    }
    float ss = 0.f;
    for (int k = tid; k < a.E; k += MV_CONSUMERS) {
        const float v = __ldcg(x + k);
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    consumer_sync();
    float tot = 0.f;
    for (int w = 0; w < MV_CWARPS; ++w) tot += red[w];
    const float scale = 1.0f / sqrtf(tot / (float)a.E + a.eps);
    for (int k = tid; k < a.E; k += MV_CONSUMERS)
        a.hidden[k] = __fmul_rn(__fmul_rn(__ldcg(x + k), scale), a.out_norm[k]);
    return true;
}

__device__ __forceinline__ void tk_tile_src(const Seg& sg, int lt, int c, int gcb, const uint8_t*& pa,
                                            const uint8_t*& pb) {
    const PackedW& WA = sg.A;
    const PackedW& WB = sg.pair ? sg.B : sg.A;
    const int gA = sg.pair ? lt : 2 * lt;
    const int gB = sg.pair ? lt : 2 * lt + 1;
    pa = (const uint8_t*)WA.p0 + ((size_t)gA * WA.nk + c) * gcb;
    pb = (const uint8_t*)WB.p0 + ((size_t)gB * WB.nk + c) * gcb;
}

__global__ void __launch_bounds__(MV_THREADS, 1) k_token(const __grid_constant__ TokenArgs a) {
    __shared__ TkShared sh;
    const int tid = threadIdx.x;
    const uint32_t nst = (uint32_t)a.nst;
    const TkSmem S = tk_smem(a);
    uint8_t* ring = S.ring;
    uint64_t *full = S.full, *empty = S.empty, *tdone = S.tdone, *tfree = S.tfree;
    float *U = S.U, *part = S.part, *res = S.res, *red = S.red;

    const unsigned long long epoch = *a.epoch;
    const uint32_t pos = a.step->pos;
    uint32_t tok = a.step->token;
    if (tok >= (uint32_t)a.vocab) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(&a.step->error, 1u);
        tok = 0;
    }
    if (tid == 0) {
        for (uint32_t i = 0; i < nst; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], MV_CWARPS);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tdone[i], MV_CWARPS);
            mbar_init(&tfree[i], 1);
        }
        sh.err = 0;
        sh.stop = 0;
        sh.started = 0;
        sh.staged = -1;
        if (blockIdx.x == 0) a.step->argmax_key = 0ull;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const unsigned long long target = (epoch + 1ull) * gridDim.x;

    if (tid >= MV_CONSUMERS + 32) {
        // ---------------- epilogue warp
        const int lane = tid & 31;
        int n = 0;
        for (int p = 0; p < a.nph; ++p) {
            const TokenPhase& P = a.ph[p];
            if (P.kind != PH_MATVEC) continue;
            if (!smem_wait_geq(&sh.started, p)) {
                if (lane == 0) tk_fail(a, &sh, 4u);
                return;
            }
            if (*(volatile int*)&sh.err) return;
            const MatvecArgs& m = P.mv;
            for (int t = blockIdx.x; t < m.ntiles; t += gridDim.x, ++n) {
                int si, lt;
                find_seg(m, t, si, lt);
                const Seg& sg = m.seg[si];
                const int b = n & 1;
                const EpiPre pre = epi_prefetch(m, sg, lt, pos, lane);
                if (!mbar_wait(&tdone[b], (uint32_t)(n >> 1) & 1u)) {
                    if (lane == 0) tk_fail(a, &sh, 4u);
                    return;
                }
                const float* pb = part + b * MV_CWARPS * 16;
                const int r = lane & 15, h = lane >> 4;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < MV_CWARPS / 2; ++w) v += pb[(8 * h + w) * 16 + r];
                const float other = __shfl_xor_sync(0xffffffffu, v, 16);
                v = h == 0 ? v + other : other + v;
                // the staged input's f16 range factor (1 unless it was rescaled);
                // the consumers set it before their first tile's partials
                v *= *(volatile float*)&sh.sup;
                __syncwarp();
                if (lane == 0) mbar_arrive(&tfree[b]);
                if (lane < 16) res[lane] = v;
                __syncwarp();
                if (m.epi == EPI_PEER) {
                    // this rank's partial rows to every rank's receive slot (all-reduce, one shot)
                    const int row = 16 * lt + lane;
                    if (lane < 16 && row < sg.out_rows)
                        for (int r = 0; r < a.tp; ++r)
                            a.prx[r][((size_t)P.rx_slot * a.tp + a.rank) * a.E + row] = res[lane];
                } else if (m.epi == EPI_LOGITS && a.tp > 1) {
                    // this rank's vocab shard to every rank's logits, argmax over global indices
                    unsigned long long key = 0ull;
                    const int row = 16 * lt + lane;
                    if (lane < 16 && row < sg.out_rows) {
                        const int g = a.vocab_off + row;
                        for (int r = 0; r < a.tp; ++r) a.plogits[r][g] = res[lane];
                        key = argmax_key(res[lane], (uint32_t)g);
                    }
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) {
                        const unsigned long long oth = __shfl_xor_sync(0xffffffffu, key, o);
                        key = oth > key ? oth : key;
                    }
                    if (lane == 0 && key)
                        for (int r = 0; r < a.tp; ++r) atomicMax(a.pkey[r], key);
                } else {
                    apply_epilogue(m, sg, lt, res, pos, lane, pre);
                }
                __syncwarp();
            }
            if (p + 1 < a.nph || a.tp > 1) {
                // The release add orders every lane's stores before the arrival (the
                // warp barrier makes them precede it; release is cumulative), so no
                // separate fence: a fence here also waits out this SM's in-flight
                // weight copies (about 1 us, measured).
                __syncwarp();
                if (lane == 0) {
                    tk_arrive(a, p, P.xrank != 0);
                    tk_stamp(a, p, 3);
                }
            }
        }
        return;
    }
    if (tid >= MV_CONSUMERS) {
        // ---------------- producer warp: the weights of every matvec phase, in order
        if (tid == MV_CONSUMERS) {
            uint64_t policy;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
            uint32_t slot = 0, par = 0, issued = 0;
            bool ok = true;
            for (int p = 0; p < a.nph && ok; ++p) {
                const TokenPhase& P = a.ph[p];
                if (P.kind != PH_MATVEC) continue;
                const MatvecArgs& m = P.mv;
                const int gcb = gcb_of(P.type), ck = ck_of(P.type);
                const int nchunk = (m.K + ck - 1) / ck;
                int pc = 0;  // chunks of this phase issued so far
                for (int t = blockIdx.x; t < m.ntiles && ok; t += gridDim.x) {
                    int si, lt;
                    find_seg(m, t, si, lt);
                    for (int c = 0; c < nchunk; ++c, ++pc) {
                        // Past the first a.prefetch chunks, wait until the consumers have
                        // staged this phase's input. The host passes the ring size, so
                        // the whole ring fills across the phase boundary (measured best);
                        // a smaller value keeps the staging loads ahead of weight copies.
                        if (pc == a.prefetch && !smem_wait_geq_sleep(&sh.staged, p)) {
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&empty[slot], par ^ 1u) || *(volatile int*)&sh.err) {
                            ok = false;
                            break;
                        }
                        const uint8_t *ga, *gb;
                        tk_tile_src(m.seg[si], lt, c, gcb, ga, gb);
                        uint8_t* dst = ring + slot * TK_STAGE;
                        mbar_expect_tx(&full[slot], 2 * gcb);
                        bulk_g2s_evict_first(dst, ga, gcb, &full[slot], policy);
                        bulk_g2s_evict_first(dst + gcb, gb, gcb, &full[slot], policy);
                        ++issued;
                        if (++slot == nst) {
                            slot = 0;
                            par ^= 1u;
                        }
                    }
                }
            }
            // drain: every issued copy has landed before this thread exits
            const uint32_t first = issued > nst ? issued - nst : 0;
            for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % nst], (j / nst) & 1u);
            if (!ok) tk_fail(a, &sh, 2u);
        }
        return;
    }

    // ---------------- consumers
    // The phase descriptor is copied to shared memory while thread 0 waits at the
    // barrier (double-buffered: a slow warp may still read the previous one), so
    // the phase's first instructions do not wait on global loads of its fields.
    __shared__ __align__(16) TokenPhase sph[2];
    uint32_t slot = 0, par = 0;
    int ntile = 0;
    for (int p = 0; p < a.nph; ++p) {
        {
            const int* src = (const int*)(a.ph + p);
            int* dst = (int*)&sph[p & 1];
            for (int i = tid; i < (int)(sizeof(TokenPhase) / 4); i += MV_CONSUMERS) dst[i] = __ldg(src + i);
        }
        const TokenPhase& P = sph[p & 1];
        consumer_sync();  // the descriptor is in place; every warp is done with phase p - 1
        tk_prefetch(a, P, U);
        // Each phase's code waits for the previous phase's barrier itself (tk_gate),
        // after its prologue. A stop is seen by every consumer warp at the same gate.
        if (P.kind == PH_MATVEC) {
            int r = TK_DONE;
            switch (P.type) {
                case GT_Q4_0:
                    r = tk_matvec<GT_Q4_0>(a, P, p, tok, pos, target, &sh, slot, par, ntile);
                    break;
                case GT_Q8_0:
                    r = tk_matvec<GT_Q8_0>(a, P, p, tok, pos, target, &sh, slot, par, ntile);
                    break;
                case GT_Q6_K:
                    r = tk_matvec<GT_Q6_K>(a, P, p, tok, pos, target, &sh, slot, par, ntile);
                    break;
                default:
                    r = tk_matvec<GT_F32>(a, P, p, tok, pos, target, &sh, slot, par, ntile);
                    break;
            }
            if (r == TK_STOPPED) break;
            if (r == TK_FAILED) {
                // no early exit: the other consumer warps meet this one at the next
                // phase's gate, see the error there and leave together
                if ((tid & 31) == 0) tk_fail(a, &sh, 4u);
                continue;
            }
        } else if (P.kind == PH_ATTN) {
            bool go = true;
#if TK_ATT_PER_HEAD
            go = tk_attention_kv<1>(a, P.at, p, pos, U, &sh, target);  // one query head per item
#else
            switch (P.at.n_head / P.at.n_kv) {
                case 1: go = tk_attention_kv<1>(a, P.at, p, pos, U, &sh, target); break;
                case 2: go = tk_attention_kv<2>(a, P.at, p, pos, U, &sh, target); break;
                case 3: go = tk_attention_kv<3>(a, P.at, p, pos, U, &sh, target); break;
                case 4: go = tk_attention_kv<4>(a, P.at, p, pos, U, &sh, target); break;
                case 8: go = tk_attention_kv<8>(a, P.at, p, pos, U, &sh, target); break;
                default: go = tk_gate(a, p, &sh, target); break;  // excluded on the host (fused_check)
            }
#endif
            if (!go) break;
            consumer_sync();  // every warp's partial stores precede thread 0's release
            if (tid == 0 && p + 1 < a.nph) {
                red_release_add_u64(&a.bars[p], 1ull);
                tk_stamp(a, p, 3);
            }
        } else {
            if (!tk_hidden(a, P, p, red, &sh, target)) break;
            consumer_sync();
            if (tid == 0 && a.tp > 1) tk_arrive(a, p, P.xrank != 0);
        }
    }
    // a phase left at its gate may still have norm-weight copies in flight
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (tid == 0 && blockIdx.x == 0 && !*(volatile int*)&sh.err) {
        // tensor parallel: the kernel ends only when every rank's last phase (its
        // stores into this rank's logits and argmax key) is done
        if (a.tp > 1 && !tk_rank_wait(a, a.nph - 1, target)) tk_fail(a, &sh, 4u);
        // every CTA has read the epoch once it arrived at the last barrier
        atomicAdd(a.epoch, 1ull);
    }
}

// ============================================================================
// Split-K matvec with static scratch (talos_matvec_dev_noalloc)
// ============================================================================
//
// y = W x like k_matvec, but each CTA takes one (16-row tile, K slice) unit, so
// a short matrix still spreads over every SM. A unit's 16 partial row sums go
// to a scratch array; the CTA that completes a tile's last slice (an arrival
// counter per tile) adds the slices in slice order and writes the rows, then
// sets the counter back to zero. The scratch is a file-scope __device__ array of
// fixed size, so the entry point allocates nothing: it serves callers that must
// not allocate, e.g. a decode loop driven by a runtime that reserves all device
// memory up front, or a caller that cannot afford the device-wide
// synchronisation cudaMalloc / cudaFree imply. Limits: at most
// NOALLOC_MAX_TILES tiles (65,536 rows) and NOALLOC_MAX_SLICES slices.
// Concurrent calls share the scratch and race; callers serialise them.

constexpr int NOALLOC_MAX_TILES = 4096;
constexpr int NOALLOC_MAX_SLICES = 8;
// partial row sums [tile][slice][16] (2 MB) and arrival counters [tile], zero at
// module load; every call leaves the counters at zero again
static __device__ __align__(256) float g_noalloc_part[NOALLOC_MAX_TILES * NOALLOC_MAX_SLICES * 16];
static __device__ __align__(256) unsigned g_noalloc_cnt[NOALLOC_MAX_TILES];

template <int TYPE>
__global__ void __launch_bounds__(MV_CONSUMERS, 1)
    k_matvec_splitk(const PackedW w, const float* __restrict__ x, float* __restrict__ y, int nslice, float* part,
                    unsigned* cnt) {
    constexpr int GCB = Fmt<TYPE>::GCB, CK = Fmt<TYPE>::CK;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float red[MV_CWARPS * 16];
    __shared__ int last, sok;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = w.cols, nchunk = w.nk, KP = nchunk * CK;
    const int tile = blockIdx.x / nslice, slice = blockIdx.x % nslice;
    const int per = (nchunk + nslice - 1) / nslice, c0 = slice * per, c1 = min(nchunk, c0 + per);
    uint8_t* stage = smem;                      // one chunk: two group-chunks
    float* U = (float*)(smem + 2 * GCB);        // staged x: KP floats, then KP / 16 block sums
    float* xs16 = U + KP;
    if (tid == 0) {
        mbar_init(&bar, 1);
        sok = 1;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // stage x (all of it: consume_* index the staged input by absolute chunk),
    // again scaled by 2^-16 while an element is out of f16 range (kStageBig)
    float sdown = 1.f, sup = 1.f;
    for (int tries = 0;; ++tries) {
        bool big = false;
        for (int r = warp; r < KP / 128; r += MV_CWARPS) {
            const int e0 = 128 * r + 4 * lane;
            float t4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) t4[i] = e0 + i < K ? x[e0 + i] : 0.f;
            const float4 v = scale4(make_float4(t4[0], t4[1], t4[2], t4[3]), sdown);
            big |= big4(v);
            tk_put4<TYPE>(U, e0, v);
            tk_sums<TYPE>(xs16, e0, v, lane);
        }
        if (!__syncthreads_or(big) || TYPE == GT_F32 || tries == kStageRetries) break;
        sdown *= kStageDown;
        sup *= 1.f / kStageDown;
    }
    Acc acc = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    int issued = 0;  // thread 0: chunks copied
    for (int c = c0; c < c1; ++c) {
        const uint32_t parity = (uint32_t)(c - c0) & 1u;
        if (tid == 0 && *(volatile int*)&sok) {
            ++issued;
            const uint8_t* ga = (const uint8_t*)w.p0 + ((size_t)(2 * tile) * w.nk + c) * GCB;
            const uint8_t* gb = (const uint8_t*)w.p0 + ((size_t)(2 * tile + 1) * w.nk + c) * GCB;
            mbar_expect_tx(&bar, 2 * GCB);
            bulk_g2s(stage, ga, GCB, &bar);
            bulk_g2s(stage + GCB, gb, GCB, &bar);
        }
        if (ok && !mbar_wait(&bar, parity)) {  // bounded (2 s): record it, stop copying
            ok = false;
            *(volatile int*)&sok = 0;
        }
        if (ok) {
            if (TYPE == GT_Q4_0)
                consume_q4_0(stage, stage + GCB, (const uint4*)U, xs16, c, acc);
            else if (TYPE == GT_Q8_0)
                consume_q8_0(stage, stage + GCB, (const uint4*)U, xs16, c, acc);
            else if (TYPE == GT_Q6_K)
                consume_q6_k(stage, stage + GCB, (const uint4*)U, xs16, c, acc);
            else
                consume_f32(stage, stage + GCB, U, c, acc);
        }
        __syncthreads();  // the stage is free for the next chunk
    }
    // the 16 warps' partials of the unit -> 16 row sums
    if (TYPE == GT_F32) {
        const float v = warp_sum(acc.pA);
        if (lane < 16) red[warp * 16 + lane] = (lane == warp) ? v : 0.f;
    } else if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = fmaf(acc.pA, kTwo24, -Zero<TYPE>::z * acc.qA) * sup;
        red[warp * 16 + 8 + (lane >> 2)] = fmaf(acc.pB, kTwo24, -Zero<TYPE>::z * acc.qB) * sup;
    }
    __syncthreads();
    if (tid < 16) {
        float v = 0.f;
        for (int q = 0; q < MV_CWARPS; ++q) v += red[q * 16 + tid];
        // a slice whose copy wait expired covers only part of its chunks: its
        // partials are NaN, so the tile's rows come out NaN whichever slice the
        // wait expired in (the CTA that adds the slices sees only its own flag)
        part[((size_t)tile * nslice + slice) * 16 + tid] = sok ? v : __int_as_float(0x7fc00000);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        // a copy still in flight after a timed-out wait lands before the CTA leaves
        if (!sok && issued) mbar_wait(&bar, (uint32_t)(issued - 1) & 1u);
        const unsigned old = atomicAdd(&cnt[tile], 1u);
        last = old == (unsigned)(nslice - 1);
        if (last) cnt[tile] = 0u;  // every slice has arrived: ready for the next call
    }
    __syncthreads();
    if (!last || tid >= 16) return;
    __threadfence();
    float v = 0.f;
    for (int q = 0; q < nslice; ++q) v += __ldcg(part + ((size_t)tile * nslice + q) * 16 + tid);
    const int row = 16 * tile + tid;
    if (row < w.rows) y[row] = sok ? v : __int_as_float(0x7fc00000);  // NaN rows: some slice's copy timed out
}

size_t noalloc_smem_bytes(int type, int K) {
    const int ck = fmt_ck(type);
    if (!ck) return 0;
    const int kp = ceil_div_h(K, ck) * ck;
    return (size_t)2 * fmt_gcb(type) + (size_t)kp * 4 + (size_t)kp / 16 * 4;
}

cudaError_t noalloc_scratch(float** part, unsigned** cnt, int* max_tiles, int* max_slices) {
    cudaError_t e = cudaGetSymbolAddress((void**)part, g_noalloc_part);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)cnt, g_noalloc_cnt);
    *max_tiles = NOALLOC_MAX_TILES;
    *max_slices = NOALLOC_MAX_SLICES;
    return e;
}

cudaError_t launch_matvec_noalloc(const PackedW& w, const float* x, float* y, int nslice, float* part, unsigned* cnt,
                                  cudaStream_t s) {
    const int ntiles = w.rows_pad / 16;
    const size_t sm = noalloc_smem_bytes(w.type, w.cols);
    if (!sm || sm > (size_t)kMaxSmem || ntiles > NOALLOC_MAX_TILES || nslice < 1 || nslice > NOALLOC_MAX_SLICES)
        return cudaErrorInvalidValue;
    cudaError_t e;
    const dim3 grid(ntiles * nslice), block(MV_CONSUMERS);
    switch (w.type) {
        case GT_F32:
            if ((e = cudaFuncSetAttribute(k_matvec_splitk<GT_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)))
                return e;
            k_matvec_splitk<GT_F32><<<grid, block, sm, s>>>(w, x, y, nslice, part, cnt);
            break;
        case GT_Q8_0:
            if ((e = cudaFuncSetAttribute(k_matvec_splitk<GT_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)))
                return e;
            k_matvec_splitk<GT_Q8_0><<<grid, block, sm, s>>>(w, x, y, nslice, part, cnt);
            break;
        case GT_Q4_0:
            if ((e = cudaFuncSetAttribute(k_matvec_splitk<GT_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)))
                return e;
            k_matvec_splitk<GT_Q4_0><<<grid, block, sm, s>>>(w, x, y, nslice, part, cnt);
            break;
        case GT_Q6_K:
            if ((e = cudaFuncSetAttribute(k_matvec_splitk<GT_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)))
                return e;
            k_matvec_splitk<GT_Q6_K><<<grid, block, sm, s>>>(w, x, y, nslice, part, cnt);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

int token_stage_elems(int type, int K) {
    const int ck = fmt_ck(type);
    if (!ck) return 0;
    return ceil_div_h(K, ck) * ck;
}

bool token_attn_per_head() { return TK_ATT_PER_HEAD; }
int token_attn_bytes(int group, int hd) { return (group * hd + MV_CWARPS * group * (hd + 4)) * 4; }

size_t token_smem_bytes(int nst, int union_bytes) {
    return (size_t)nst * TK_STAGE + TK_BAR_BYTES + (size_t)union_bytes + TK_TAIL_BYTES;
}

// Dynamic shared memory k_token may use: the opt-in maximum less its static part.
static int token_smem_limit() {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, k_token) != cudaSuccess) return 0;
    return v - (int)fa.sharedSizeBytes;
}

int token_max_stages(int union_bytes) {
    const long room = (long)token_smem_limit() - TK_BAR_BYTES - union_bytes - TK_TAIL_BYTES;
    long n = room / TK_STAGE;
    if (n > 24) n = 24;
    return n < 2 ? 0 : (int)n;
}

cudaError_t token_configure() {
    const int lim = token_smem_limit();
    if (lim <= 0) return cudaErrorInvalidValue;
    return cudaFuncSetAttribute(k_token, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
}

cudaError_t launch_token(const TokenArgs& a, int grid, cudaStream_t s, bool cooperative) {
    if (a.nst < 2 || a.nst > 24 || a.union_bytes % 16) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = token_smem_bytes(a.nst, a.union_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_token, a);
}


}  // namespace talos
