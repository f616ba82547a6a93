// common.cuh -- device-side types and helpers shared by the Talos sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace talos {

enum GType : int { GT_F32 = 0, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_Q6_K = 14 };

// A weight matrix after repacking on the device (k_pack_* in matvec.cu): one
// array p0 of group-chunks, each 8 rows x CK input elements, contiguous and in
// the register order the consumers read, ordered [row group][chunk]; a 16-row
// tile is two group-chunks. CK and bytes per group-chunk: Q4_0 2048, 9216 B
// (nibbles + f16 block scales); Q8_0 1024, 8704 B; Q6_K 1024, 8768 B (6-bit
// quants widened to bytes, sub-block scales, f16 super-block scales); F32 256,
// 8192 B. Rows pad to a multiple of 16 and columns to CK with entries that add
// nothing (quant at the zero point, scale 0). p1 (quant types): one f32, the
// largest |value| the blocks dequantize to (k_wbound). p2, p3 are unused (null).
struct PackedW {
    int type;
    int rows, cols;   // logical shape [rows, cols]
    int rows_pad;     // multiple of 16
    int nk;           // chunks per row group (cols rounded up to CK)
    const void* p0;
    const void* p1;
    const void* p2;
    const void* p3;
};

// Device-resident step parameters, read by every kernel of a captured graph so
// one graph serves every token.
struct StepParams {
    uint32_t token;
    uint32_t pos;
    uint32_t n_gen;      // tokens written to gen_tokens so far (greedy loop)
    uint32_t error;      // first device-side error code (0 = none)
    unsigned long long argmax_key;  // packed (total-order key << 32) | index
};

__device__ __forceinline__ float silu_ref(float g) {
    // src/math/ops.rs:28-30: x / (1 + exp(-x))
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u1(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

template <int LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return d;
}

// Four 4-bit quants in bit positions {0-3, 16-19} -> f16x2 (q - 8), exact.
__device__ __forceinline__ uint32_t q4_lo_f16x2(uint32_t w) {
    uint32_t t = lop3<0xEA>(w, 0x000F000Fu, 0x64006400u);  // 1024 + q
    uint32_t r;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(0x64086408u));  // - 1032
    return r;
}
// Quants in bit positions {4-7, 20-23} -> f16x2 (q - 8), exact.
__device__ __forceinline__ uint32_t q4_hi_f16x2(uint32_t w) {
    uint32_t t = lop3<0xEA>(w, 0x00F000F0u, 0x64006400u);  // 1024 + 16 q
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(t), "r"(0x2C002C00u), "r"(0xD480D480u));  // /16 - 72
    return r;
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(half lo, half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Order-preserving map of f32 onto u32 following Rust's f32::total_cmp.
__device__ __forceinline__ uint32_t total_order_key(float f) {
    int32_t b = __float_as_int(f);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return (uint32_t)b ^ 0x80000000u;
}

// Argmax key of value v at index i: (total-order key << 32) | i. The largest key
// is the maximum under f32::total_cmp and, among equal values, the LAST index,
// which is what sample::argmax's max_by keeps (src/sample.rs:7-14). Keys combine
// with max / atomicMax in any order.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
    return ((unsigned long long)total_order_key(v) << 32) | i;
}

__device__ __forceinline__ float ld_half_bytes(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// Element `i` of a tensor stored as raw GGUF blocks, bit-exact with
// GgmlType::dequantize (src/gguf/dtype.rs:64-121).
__device__ __forceinline__ float dequant_elem(int type, const uint8_t* raw, size_t i) {
    switch (type) {
        case GT_F32: {
            const uint8_t* p = raw + 4 * i;
            uint32_t b = p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24);
            return __uint_as_float(b);
        }
        case GT_Q8_0: {  // dtype.rs:69-78: d * q
            const uint8_t* b = raw + (i / 32) * 34;
            return __fmul_rn(ld_half_bytes(b), (float)(int8_t)b[2 + i % 32]);
        }
        case GT_Q4_0: {  // dtype.rs:79-91: d * (nibble - 8)
            const uint8_t* b = raw + (i / 32) * 18;
            int j = (int)(i % 32);
            int q = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
            return __fmul_rn(ld_half_bytes(b), (float)(q - 8));
        }
        case GT_Q6_K: {  // dtype.rs:93-119: (d * sc) * q
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

// Bytes and elements of one GGUF block of `type`.
__host__ __device__ inline int gguf_block_bytes(int type) {
    return type == GT_F32 ? 4 : (type == GT_Q6_K ? 210 : (type == GT_Q8_0 ? 34 : 18));
}
__host__ __device__ inline int gguf_block_elems(int type) {
    return type == GT_F32 ? 1 : (type == GT_Q6_K ? 256 : 32);
}

}  // namespace talos
