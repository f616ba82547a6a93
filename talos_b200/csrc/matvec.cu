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
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------
// PTX helpers: mbarrier, 1-D bulk copy, programmatic dependent launch
// ----------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: false once 2 s have passed without the phase completing (only on
// a broken pipeline); the caller records an error and leaves its loop.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

constexpr int MV_CONSUMERS = 512;              // 16 consumer warps
constexpr int MV_CWARPS = MV_CONSUMERS / 32;
constexpr int MV_THREADS = MV_CONSUMERS + 64;  // + 1 producer warp + 1 epilogue warp
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

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

__device__ __forceinline__ float silu_ref(float g) {
    // src/math/ops.rs:28-30: x / (1 + exp(-x))
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}

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

        if (a.epi == EPI_SWIGLU) {  // src/math/ops.rs:33-37
            if (lane < 8) {
                const int j = 8 * lt + lane;
                if (j < sg.out_rows) sg.out[j] = __fmul_rn(silu_ref(res[lane]), res[8 + lane]);
            }
        } else if (a.epi == EPI_QKV) {
            if (sg.role == 2) {  // v -> cache row pos (src/kv_cache.rs:21-26)
                if (lane < 16) {
                    const int row = 16 * lt + lane;
                    if (row < sg.out_rows) a.vcache[(size_t)pos * a.kv_dim + row] = res[lane];
                }
            } else if (lane < 8) {  // RoPE on pairs (2i, 2i+1) (src/math/ops.rs:48-61)
                const int r0 = 16 * lt + 2 * lane;
                if (r0 < sg.out_rows) {
                    const int i = (r0 % a.hd) >> 1;
                    const float2 cs = a.rope_cs[(size_t)pos * (a.hd >> 1) + i];
                    const float x0 = res[2 * lane], x1 = res[2 * lane + 1];
                    const float o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
                    const float o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
                    float* dst = sg.role == 0 ? sg.out + r0 : a.kcache + (size_t)pos * a.kv_dim + r0;
                    dst[0] = o0;
                    dst[1] = o1;
                }
            }
        } else {
            unsigned long long key = 0ull;
            if (lane < 16) {
                const int row = 16 * lt + lane;
                if (row < sg.out_rows) {
                    sg.out[row] = a.epi == EPI_ADD ? __fadd_rn(sg.out[row], res[lane]) : res[lane];
                    key = ((unsigned long long)total_order_key(res[lane]) << 32) | (unsigned)row;
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
        __syncwarp();
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
    {
        // One coalesced pass, one 32-element block per warp iteration: lane l holds
        // element 32j + l, writes its f16 hi / lo halves into the B-fragment slots
        // and the warp sums the block for the zero-point term (per 16 for Q6_K
        // sub-blocks, per 32 otherwise).
        const int lane = tid & 31, warp = tid >> 5;
        half* xh = (half*)stage_x;
        const int s16 = lane >> 4, r16 = lane & 15;
        const int m = 2 * s16 + (r16 >> 3), t = (r16 & 7) >> 1, hp = r16 & 1;
#pragma unroll 4
        for (int j = warp; j < KP / 32; j += MV_CWARPS) {
            const float v = xin(32 * j + lane);
            if (TYPE == GT_F32) {
                stage_x[32 * j + lane] = v;
                continue;
            }
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
    }
    consumer_sync();
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
            pb[warp * 16 + (lane >> 2)] = fmaf(acc.pA, kTwo24, -Zero<TYPE>::z * acc.qA);
            pb[warp * 16 + 8 + (lane >> 2)] = fmaf(acc.pB, kTwo24, -Zero<TYPE>::z * acc.qB);
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

}  // namespace talos
