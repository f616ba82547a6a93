// gemm.cu -- the tensor-core (tcgen05) GEMM of the prefill and batched-decode
// steps on B200 (sm_100a).
//
// Y[t][r] = sum_k dequant(W)[r][k] * X[t][k] for up to 128 token columns per
// tile: the prompt positions of a prefill chunk, or the independent sequences
// of a batched decode step. The arithmetic of every (r, t) element is what
// quant::matvec (Tsuskov/talos src/math/quant.rs:18-51) computes for that row
// and input, to f32 rounding.
//
// Exactness. The tensor cores multiply f16 (kind::f16) into f32 accumulators.
//  * Weights: a Q4_0 / Q8_0 value (q - z) * d has at most 4 + 11 / 8 + 11
//    significant bits, so it is EXACTLY A_hi + A_lo with A_hi = f16(v) and
//    A_lo = v - A_hi (computed with one f16 multiply and one f16 FMA, both exact
//    here). The tensor's values are first scaled by a power of two 2^eA that
//    keeps them inside f16's normal range (the bound comes from the tensor's
//    largest block scale, recorded when it was packed); the epilogue multiplies
//    by 2^-eA. Q6_K's (d * sc) * q (src/gguf/dtype.rs:112-115) has up to 25
//    bits: it is formed in f32 like the reference and split into hi + lo
//    (22 bits).
//  * Activations: each token's input row is scaled by a power of two 2^-e_t
//    into [2^14, 2^15) at its largest element and split into f16 x_hi + x_lo
//    (~22 bits); the epilogue multiplies by 2^e_t. No input overflows f16 and
//    small inputs keep their relative precision.
//  * Per K step of 16: D[:, 0:2N] += A_hi x [x_hi | x_lo] and
//    D[:, 0:N] += A_lo x x_hi (the A_lo x_lo term is below f32 rounding; up to
//    64 columns this term has columns 2N .. 3N of its own); the result is
//    D[:, t] + D[:, N + t] (+ D[:, 2N + t]).
//
// Structure: one CTA per SM (persistent over work units = 128-row tile x token
// tile x K slice), warp-specialised:
//  * warps 0-3: epilogue. Warp q reads TMEM lanes 32q .. 32q+31 (its tile rows)
//    with tcgen05.ld, combines, scales and applies the step's epilogue (store,
//    residual add, SwiGLU, RoPE + KV-cache append); with split-K the partial
//    tile goes to a workspace and the unit that completes the tile adds the
//    slices in slice order (deterministic). The four warps never wait for one
//    another.
//  * warp 4: weight producer. Two tiled TMA copies per raw slot (128 inputs)
//    of the packed group-chunks (k_pack_*: 8 rows x CK) of the tile's 16 row
//    groups: their lane records, then their scales, through two tensor maps of
//    the packed weight (encoded when it was packed; without them, 1-D bulk
//    copies per row group).
//  * warp 5: activation producer. One tiled TMA copy per stage
//    (cp.async.bulk.tensor.3d, no multicast) of the formatted [x_hi; x_lo]
//    planes into the B stage.
//  * warp 6: allocates TMEM (two accumulators: double buffering across units);
//    its lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M 128, K 16) of A_hi
//    against [x_hi | x_lo] (N 2NT) and tcgen05.commit to the stage's "empty" and
//    the accumulator's "full" barrier. Up to 64 token columns warp 7 issues the
//    A_lo x x_hi MMAs (N NT) into a third part of the accumulator (two issuers:
//    one thread's issue costs more than a narrow MMA takes); at 128 columns warp
//    6 issues both into the same 2N columns.
//  * warps 8-15: dequantizers. Raw slot -> A_hi / A_lo stage tiles (f16, one
//    stmatrix per four 8 x 8 blocks), fence.proxy.async, arrive; up to 64
//    columns both stages of a raw slot at once.
// A and B stage tiles are K-major with the 128-byte swizzle of tcgen05 (and of
// TMA): one 128-byte row per matrix row (64 inputs of f16), its 16-byte chunk c
// stored at chunk c ^ (row % 8), 8-row atoms 1024 bytes apart.
// Every mbarrier wait is bounded (2 s); on expiry the CTA records an error bit
// in BatchParams::error and every role leaves its loop; TMEM is freed at exit.
#include <cuda.h>
#include <math.h>

#include "kernels.cuh"
#include "ptx.cuh"

namespace talos {

constexpr int GM_BM = 128;   // weight rows per tile = TMEM lanes
constexpr int GM_BK = 64;    // K per A/B stage
constexpr int GM_RK = 128;   // K per raw weight slot (two stages)
#ifndef TALOS_GM_NDQ
#define TALOS_GM_NDQ 8
#endif
constexpr int GM_NDQ = TALOS_GM_NDQ;  // dequantizer warps (8 or 16: each takes 16 / GM_NDQ row groups per stage)
constexpr int GM_WP = 4, GM_XP = 5, GM_MMA = 6, GM_MMA2 = 7, GM_DQ0 = 8;
constexpr int GM_THREADS = (GM_DQ0 + GM_NDQ) * 32;
constexpr int GM_SMEM = 220 * 1024;
constexpr int GM_MAXRAW = 8;

// Bytes per row group of one raw slot (128 inputs): lane records, then scales.
//  Q4_0: quad q of the group-chunk (512 B) + its f16 scales [8 rows][4] (64 B)
//  Q8_0: quad q (1024 B) + scales [8 rows][4] (64 B)
//  Q6_K: step-quads 2m, 2m+1 (1024 B) + the chunk's sc [8][64] and d [8][4] (576 B)
// A raw slot holds the 16 groups' lane records [16][LREC], then their scales
// [16][SC]. GCB: bytes of one group-chunk; CK: its inputs.
template <int TYPE>
struct GmFmt;
template <>
struct GmFmt<GT_Q4_0> {
    static constexpr int LREC = 512, SC = 64, GCB = 16 * 512 + 16 * 64, CK = 2048;
};
template <>
struct GmFmt<GT_Q8_0> {
    static constexpr int LREC = 1024, SC = 64, GCB = 8 * 1024 + 8 * 64, CK = 1024;
};
template <>
struct GmFmt<GT_Q6_K> {
    static constexpr int LREC = 1024, SC = 576, GCB = 16 * 512 + 8 * 64 + 8 * 4 * 2, CK = 1024;
};
// Where raw slot rs's data sits inside a group-chunk (bytes): lane records at
// lrec_off, scales at sc_off, in chunk rs * 128 / CK.
template <int TYPE>
__host__ __device__ constexpr int gm_lrec_off(int rs) {
    return (rs * 128 % GmFmt<TYPE>::CK) / 128 * GmFmt<TYPE>::LREC;
}
template <int TYPE>
__host__ __device__ constexpr int gm_sc_off(int rs) {
    return TYPE == GT_Q6_K ? 16 * 512 : (TYPE == GT_Q4_0 ? 16 * 512 : 8 * 1024) + (rs * 128 % GmFmt<TYPE>::CK) / 128 * 64;
}

// Shared memory of one configuration: NS A/B stages (4, 3 or 2: as many as fit
// beside a ring of at least two raw slots; more stages hide more of the
// dequantize -> MMA -> release round trip), then as many raw slots as fit (<= 8).
template <int TYPE, int NT>
struct GmCfg {
    static constexpr int GRP = GmFmt<TYPE>::LREC + GmFmt<TYPE>::SC;
    static constexpr int RAW = 16 * GRP;
    static constexpr int A_BYTES = 2 * GM_BM * GM_BK * 2;  // A_hi + A_lo
    static constexpr int B_BYTES = 2 * NT * GM_BK * 2;     // [x_hi; x_lo]
    static constexpr int BAR_BYTES = 1024;
    static constexpr int EPI_BYTES = 4 * NT * 12;  // the epilogue warps' column scales, positions, slots
    static constexpr int fixed(int ns) { return ns * (A_BYTES + B_BYTES) + BAR_BYTES + EPI_BYTES; }
    static constexpr int NS = fixed(4) + 2 * RAW <= GM_SMEM ? 4 : (fixed(3) + 2 * RAW <= GM_SMEM ? 3 : 2);
    static constexpr int FIXED = fixed(NS);
    static constexpr int NRAW_FIT = (GM_SMEM - FIXED) / RAW;
    static constexpr int NRAW = NRAW_FIT > GM_MAXRAW ? GM_MAXRAW : NRAW_FIT;
    static constexpr int SMEM = FIXED + NRAW * RAW;
    // Up to 64 columns the A_lo MMAs have an issuer (warp GM_MMA2) and an
    // accumulator of their own: D = [A_hi x (x_hi | x_lo) : 2N][A_lo x x_hi : N].
    // At 128 columns (tensor-bound) one thread issues both into 2N columns.
    static constexpr int ISS = NT <= 64 ? 2 : 1;
    static constexpr int ACCW = ISS == 2 ? 3 * NT : 2 * NT;  // TMEM columns of one accumulator
    static constexpr int TCOLS = 2 * ACCW <= 128 ? 128 : (2 * ACCW <= 256 ? 256 : 512);  // two accumulators
    static_assert(2 * ACCW <= 512, "TMEM");
    static_assert(NRAW >= 2, "raw ring too small");
};

// ---------------------------------------------------------------- PTX

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major shared-memory matrix descriptor (tcgen05) with the 128-byte swizzle:
// start address (16-byte units; a K step of 16 inputs adds 32 bytes), LBO 16
// bytes (unused by this layout), SBO 1024 bytes between 8-row atoms, version 1
// (bits 46-47) for sm_100, layout type 2 (bits 61-63) = SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// Instruction descriptor, kind::f16: f32 accumulate, f16 A and B, both K-major, M 128.
__host__ __device__ constexpr uint32_t umma_idesc(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(GM_BM >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Bounded wait of a role that mostly waits (producers, MMA issuers, epilogue):
// it sleeps between polls so that its sub-partition's issue slots go to the
// dequantizer warps beside it (128-column tiles: 94 -> 85 us on 28672 x 4096).
__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(64);
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}

// ---------------------------------------------------------------- work units

struct GmUnit {
    int si, lt;  // segment, tile within it
    int tt, ks;  // token tile, K slice
    int r0, r1;  // raw slots [r0, r1) of the slice
    int tile;    // output tile index (row tile x token tile) for the split-K counters
};
__device__ __forceinline__ GmUnit gm_unit(const GemmArgs& a, int u, int ntt) {
    GmUnit w;
    w.ks = u % a.S;
    int rest = u / a.S;
    w.tt = rest % ntt;
    int rt = rest / ntt;
    w.tile = rt * ntt + w.tt;
    w.si = 0;
    while (w.si + 1 < a.nseg && rt >= a.seg[w.si].ntiles) rt -= a.seg[w.si++].ntiles;
    w.lt = rt;
    const int R = a.KP / GM_RK;
    w.r0 = (int)((long)w.ks * R / a.S);
    w.r1 = (int)((long)(w.ks + 1) * R / a.S);
    return w;
}

// Group g's raw slot rs data in the packed weight: lane records and scales.
template <int TYPE>
__device__ __forceinline__ void gm_src(const PackedW& w, int g, int rs, const uint8_t*& lrec, const uint8_t*& sc) {
    const uint8_t* gc =
        (const uint8_t*)w.p0 + ((size_t)g * w.nk + rs * 128 / GmFmt<TYPE>::CK) * GmFmt<TYPE>::GCB;
    lrec = gc + gm_lrec_off<TYPE>(rs);
    sc = gc + gm_sc_off<TYPE>(rs);
}

// The segment's scale exponent eA: its values * 2^eA stay below 2^14 (the bound
// is recorded at pack time: the largest |value| the format can give, k_wbound).
__device__ __forceinline__ int gm_wexp(const GemmSeg& sg) {
    const float b = sg.A.p1 ? *(const float*)sg.A.p1 : 0.f;
    if (!(b > 0.f) || !isfinite(b)) return 0;
    int ex;
    frexpf(b, &ex);  // b in [2^(ex-1), 2^ex)
    int e = 14 - ex;
    return e > 60 ? 60 : (e < -60 ? -60 : e);
}

// ---------------------------------------------------------------- dequantizers
//
// Thread (lr, t) = (lane / 4, lane % 4) of a group task holds, per 32-element
// block (16 for Q6_K), the k pairs {2t, 2t+1}, {2t+8, 2t+9}, {16+2t, 17+2t},
// {24+2t, 25+2t} (the packed lane records): for each 8-k group kg of the block,
// row lr's columns 2t, 2t+1 of an 8 x 8 f16 matrix, the fragment layout of
// stmatrix. One stmatrix.x4 per four groups writes the warp's 8 rows; lane L
// gives the address of row L % 8 of group kg0 + L / 8, in the swizzled layout
// (the row's 16-byte chunk kg at row * 128 + (kg ^ row % 8) * 16).
__device__ __forceinline__ void gm_stsm4(uint8_t* A, int gi, int kg0, int lane, uint32_t r0, uint32_t r1,
                                         uint32_t r2, uint32_t r3) {
    const int m = lane >> 3, r = lane & 7;
    const uint32_t addr = smem_u32(A + (gi * 8 + r) * 128 + (((kg0 + m) ^ r) << 4));
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}
// (q - z) d = hi + lo exactly (see the file comment), as f16x2 words.
__device__ __forceinline__ void gm_split(__half2 q, __half2 d, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __hmul2(q, d);
    const __half2 l = __hfma2(q, d, __hneg2(h));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
// Two f32 values -> f16x2 hi and the f16x2 of their remainders.
__device__ __forceinline__ void gm_split_f32(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
// Q8_0 bytes (two int8 in byte positions sel) -> f16x2 exactly: 1024 + (q + 128) - 1152.
__device__ __forceinline__ __half2 q8_pair(uint32_t w, uint32_t sel) {
    const uint32_t b = __byte_perm(w ^ 0x80808080u, 0x64646464u, sel);
    __half2 h = *reinterpret_cast<const __half2*>(&b);
    return __hsub2(h, __half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));  // 1152
}

// One group task of one stage (half h of the raw slot): raw group data -> A rows
// 8 gi .. 8 gi + 7 of this stage's A_hi / A_lo (Q4_0, Q8_0; Q6_K: gm_dequant_q6).
template <int TYPE>
__device__ __forceinline__ void gm_dequant(const uint8_t* lrec, const uint8_t* scs, uint8_t* Ahi, uint8_t* Alo, int gi,
                                           int h, int lane, float wsc) {
    const int lr = lane >> 2;
    if (TYPE == GT_Q4_0) {
        const uint4 rec = *(const uint4*)(lrec + lane * 16);
        const uint32_t sc2 = *(const uint32_t*)(scs + lr * 8 + h * 4);
        const uint32_t wv[2] = {h ? rec.z : rec.x, h ? rec.w : rec.y};
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const float d = __half2float(__ushort_as_half((unsigned short)(sc2 >> (16 * jj)))) * wsc;
            const __half2 dd = __float2half2_rn(d);
            const uint32_t w = wv[jj];
            uint32_t q[4] = {q4_lo_f16x2(w), q4_hi_f16x2(w), q4_lo_f16x2(w >> 8), q4_hi_f16x2(w >> 8)};
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) gm_split(*reinterpret_cast<__half2*>(&q[m]), dd, hi[m], lo[m]);
            gm_stsm4(Ahi, gi, 4 * jj, lane, hi[0], hi[1], hi[2], hi[3]);
            gm_stsm4(Alo, gi, 4 * jj, lane, lo[0], lo[1], lo[2], lo[3]);
        }
    } else if (TYPE == GT_Q8_0) {
        const uint4 rec = *(const uint4*)(lrec + lane * 32 + h * 16);
        const uint32_t sc2 = *(const uint32_t*)(scs + lr * 8 + h * 4);
        const uint32_t wv[4] = {rec.x, rec.y, rec.z, rec.w};
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const float d = __half2float(__ushort_as_half((unsigned short)(sc2 >> (16 * jj)))) * wsc;
            const __half2 dd = __float2half2_rn(d);
            // bytes of block jj: {2t, 2t+1, 2t+8, 2t+9} then {16+2t, 17+2t, 24+2t, 25+2t}
            uint32_t hi[4], lo[4];
            gm_split(q8_pair(wv[2 * jj], 0x4140), dd, hi[0], lo[0]);
            gm_split(q8_pair(wv[2 * jj], 0x4342), dd, hi[1], lo[1]);
            gm_split(q8_pair(wv[2 * jj + 1], 0x4140), dd, hi[2], lo[2]);
            gm_split(q8_pair(wv[2 * jj + 1], 0x4342), dd, hi[3], lo[3]);
            gm_stsm4(Ahi, gi, 4 * jj, lane, hi[0], hi[1], hi[2], hi[3]);
            gm_stsm4(Alo, gi, 4 * jj, lane, lo[0], lo[1], lo[2], lo[3]);
        }
    }
}

// Q6_K needs the sub-block position inside its 1024-input chunk for the scales.
__device__ __forceinline__ void gm_dequant_q6(const uint8_t* lrec, const uint8_t* scs, uint8_t* Ahi, uint8_t* Alo,
                                              int gi, int h, int lane, float wsc, int step0) {
    const int lr = lane >> 2;
    const uint4 rec = *(const uint4*)(lrec + h * 512 + lane * 16);
    const uint32_t wv[4] = {rec.x, rec.y, rec.z, rec.w};
    const int8_t* scp = (const int8_t*)scs + lr * 64;
    const uint16_t* dp = (const uint16_t*)(scs + 512) + lr * 4;
    uint32_t hi[8], lo[8];  // 8-k groups 2s (k 2t, 2t+1 of sub-block s) and 2s+1 (k 2t+8, 2t+9)
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int step = step0 + h * 4 + s;  // sub-block index in the chunk, 0..63
        const float d = __half2float(__ushort_as_half(dp[step >> 4]));
        const float dsc = __fmul_rn(d, (float)scp[step]);
        const uint32_t w = wv[s];
        const float v0 = __fmul_rn(dsc, (float)((int)(w & 0xFF) - 32)) * wsc;
        const float v1 = __fmul_rn(dsc, (float)((int)((w >> 8) & 0xFF) - 32)) * wsc;
        const float v2 = __fmul_rn(dsc, (float)((int)((w >> 16) & 0xFF) - 32)) * wsc;
        const float v3 = __fmul_rn(dsc, (float)((int)(w >> 24) - 32)) * wsc;
        gm_split_f32(v0, v1, hi[2 * s], lo[2 * s]);
        gm_split_f32(v2, v3, hi[2 * s + 1], lo[2 * s + 1]);
    }
    gm_stsm4(Ahi, gi, 0, lane, hi[0], hi[1], hi[2], hi[3]);
    gm_stsm4(Ahi, gi, 4, lane, hi[4], hi[5], hi[6], hi[7]);
    gm_stsm4(Alo, gi, 0, lane, lo[0], lo[1], lo[2], lo[3]);
    gm_stsm4(Alo, gi, 4, lane, lo[4], lo[5], lo[6], lo[7]);
}

// ---------------------------------------------------------------- epilogue

// The epilogue of W consecutive token columns t0 .. t0+W-1 of tile row r:
// v[j] are the raw sums, xs[j] the column scales (2^e_t * 2^-eA, 0 past the
// live columns), ps[j] the columns' positions, sl[j] their cache slots. Every global load of the W
// columns is issued before any is used (one memory round trip per W columns,
// not one per column). Called by all 32 lanes of an epilogue warp (shuffles).
template <int W>
__device__ __forceinline__ void gm_epi(const GemmArgs& a, const GemmSeg& sg, int lt, int r, int t0, int ntok,
                                       float* v, const float* xs, const uint32_t* ps, const uint32_t* sl) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] *= xs[j];
    const int row = lt * GM_BM + r;
    if (sg.epi >= EPI_B_ROPE && sg.epi <= EPI_B_VCACHE) {
        // pairs (2i, 2i+1) on lanes l, l ^ 1 (src/math/ops.rs:48-61); then the cache
        // append of src/kv_cache.rs:21-26 at the column's slot and position
        float pv[W];
#pragma unroll
        for (int j = 0; j < W; ++j) pv[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
        if (row >= sg.rows) return;
        float2 cs[W];
        if (sg.epi != EPI_B_VCACHE) {
            const size_t col = (size_t)((row % a.hd) >> 1);
#pragma unroll
            for (int j = 0; j < W; ++j) cs[j] = a.rope_cs[(size_t)ps[j] * (a.hd >> 1) + col];
        }
#pragma unroll
        for (int j = 0; j < W; ++j) {
            const int t = t0 + j;
            if (t >= ntok) continue;
            float o = v[j];
            if (sg.epi != EPI_B_VCACHE)
                o = (row & 1) ? __fadd_rn(__fmul_rn(pv[j], cs[j].y), __fmul_rn(v[j], cs[j].x))
                              : __fsub_rn(__fmul_rn(v[j], cs[j].x), __fmul_rn(pv[j], cs[j].y));
            float* dst = sg.epi == EPI_B_ROPE ? sg.y + (size_t)t * sg.ldy
                                              : (sg.epi == EPI_B_KCACHE ? a.kc : a.vc) + (size_t)sl[j] * a.seq_stride +
                                                    (size_t)ps[j] * a.kv_dim;
            dst[row] = o;
        }
        return;
    }
    if (row >= sg.rows) return;
    if (sg.epi == EPI_B_ADD) {  // residual (src/model/llama.rs:159-161, 174-176)
        float old[W];
#pragma unroll
        for (int j = 0; j < W; ++j) old[j] = t0 + j < ntok ? sg.y[(size_t)(t0 + j) * sg.ldy + row] : 0.f;
#pragma unroll
        for (int j = 0; j < W; ++j)
            if (t0 + j < ntok) sg.y[(size_t)(t0 + j) * sg.ldy + row] = __fadd_rn(old[j], v[j]);
        return;
    }
    if (sg.epi == EPI_B_PEER) {  // tensor parallel: this rank's rows to every rank
        for (int pr = 0; pr < a.npeer; ++pr) {
            float* dst = a.peer[pr] + row;
#pragma unroll
            for (int j = 0; j < W; ++j)
                if (t0 + j < ntok) dst[(size_t)(t0 + j) * sg.ldy] = v[j];
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < W; ++j)
        if (t0 + j < ntok) sg.y[(size_t)(t0 + j) * sg.ldy + row] = v[j];
}

// ---------------------------------------------------------------- the kernel

template <int TYPE, int NT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ GemmArgs a) {
    using C = GmCfg<TYPE, NT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sA = smem;                                   // [NS][hi 16 KB | lo 16 KB]
    uint8_t* sB = smem + C::NS * C::A_BYTES;              // [NS][kg 8][2 NT][16 B]
    uint8_t* sR = sB + C::NS * C::B_BYTES;                // [NRAW][16 groups][GRP]
    uint64_t* bars = (uint64_t*)(sR + C::NRAW * C::RAW);  // barriers
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + C::NRAW;
    uint64_t* a_full = raw_empty + C::NRAW;
    uint64_t* b_full = a_full + C::NS;
    uint64_t* st_empty = b_full + C::NS;
    uint64_t* acc_full = st_empty + C::NS;   // [2]
    uint64_t* acc_empty = acc_full + 2;      // [2]
    uint64_t* done = acc_empty + 2;          // the MMA thread's final commit
    uint32_t* tmem_slot = (uint32_t*)(done + 1);
    int* s_flag = (int*)(tmem_slot + 1);     // [0]: some role gave up on a wait
    float* ep_xs = (float*)(sR + C::NRAW * C::RAW + C::BAR_BYTES);  // [4 warps][NT] column scales
    uint32_t* ep_pos = (uint32_t*)(ep_xs + 4 * NT);                   // [4 warps][NT] column positions
    uint32_t* ep_slot = ep_pos + 4 * NT;                              // [4 warps][NT] column cache slots
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int ntok = a.bp->n;
    const int ntt = (ntok + NT - 1) / NT;
    const int nunits = a.nrt * ntt * a.S;

    if (tid == 0) {
        for (int i = 0; i < C::NRAW; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], GM_NDQ);
        }
        for (int i = 0; i < C::NS; ++i) {
            mbar_init(&a_full[i], GM_NDQ);
            mbar_init(&b_full[i], 1);
            mbar_init(&st_empty[i], C::ISS);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], C::ISS);
            mbar_init(&acc_empty[i], 4);
        }
        mbar_init(done, C::ISS);
        s_flag[0] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == GM_MMA) {  // TMEM: two accumulators of ACCW f32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        *(volatile int*)&s_flag[0] = 1;
        atomicOr((unsigned*)&a.bp->error, 2u);
    };
    auto stop = [&]() { return *(volatile int*)&s_flag[0] != 0; };

    if (warp == GM_WP) {
        // ---------------- weight producer: per raw slot, two TMA copies (the 16
        // groups' lane records, then their scales) through the segment's tensor
        // maps, or (no maps) lane gi's 1-D bulk copies of row group gi
        uint32_t ri = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok && !stop(); u += gridDim.x) {
            const GmUnit U = gm_unit(a, u, ntt);
            const GemmSeg& sg = a.seg[U.si];
            const int g = U.lt * 16 + lane;
            const bool valid = lane < 16 && g < sg.A.rows_pad / 8;
            const uint32_t bytes =
                sg.wmap ? (uint32_t)C::RAW : (uint32_t)__popc(__ballot_sync(0xffffffffu, valid)) * C::GRP;
            for (int rs = U.r0; rs < U.r1; ++rs, ++ri) {
                const int slot = ri % C::NRAW;
                uint8_t* dst = sR + slot * C::RAW;
                bool w_ok = true;
                if (lane == 0) {
                    w_ok = mbar_wait_idle(&raw_empty[slot], ((ri / C::NRAW) & 1) ^ 1);
                    if (w_ok) {
                        mbar_expect_tx(&raw_full[slot], bytes);
                        if (sg.wmap) {  // out-of-range groups of the last tile read as zeros
                            const int c = rs * GM_RK / GmFmt<TYPE>::CK;
                            tma_load_3d(dst, (const CUtensorMap*)sg.map_lrec, gm_lrec_off<TYPE>(rs) / 4, c, U.lt * 16,
                                        &raw_full[slot]);
                            tma_load_3d(dst + 16 * GmFmt<TYPE>::LREC, (const CUtensorMap*)sg.map_sc,
                                        gm_sc_off<TYPE>(rs) / 4, c, U.lt * 16, &raw_full[slot]);
                        }
                    }
                }
                if (!__shfl_sync(0xffffffffu, (int)w_ok, 0)) {
                    ok = false;
                    break;
                }
                if (!sg.wmap && valid) {
                    const uint8_t *lr, *sc;
                    gm_src<TYPE>(sg.A, g, rs, lr, sc);
                    bulk_g2s(dst + lane * GmFmt<TYPE>::LREC, lr, GmFmt<TYPE>::LREC, &raw_full[slot]);
                    bulk_g2s(dst + 16 * GmFmt<TYPE>::LREC + lane * GmFmt<TYPE>::SC, sc, GmFmt<TYPE>::SC,
                             &raw_full[slot]);
                }
            }
        }
        if (!ok && lane == 0) fail();
        // copies in flight land before the CTA exits
        if (lane == 0) {
            const uint32_t first = ri > (uint32_t)C::NRAW ? ri - C::NRAW : 0;
            for (uint32_t j = first; j < ri; ++j) mbar_wait(&raw_full[j % C::NRAW], (j / C::NRAW) & 1);
        }
    } else if (warp == GM_XP) {
        // ---------------- activation producer: one TMA box per stage, the stage's
        // 64 inputs of the tile's columns in both planes (128-byte swizzle). With
        // programmatic dependent launch the kernel may start while the kernel
        // before it (the input's formatter) still runs: the roles that read what
        // it writes (this one and the epilogue) wait for it here; weight copies,
        // dequantization and TMEM set-up go ahead.
        pdl_wait();
        uint32_t si = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok && !stop(); u += gridDim.x) {
            const GmUnit U = gm_unit(a, u, ntt);
            for (int rs = U.r0; rs < U.r1 && ok; ++rs)
                for (int h = 0; h < 2; ++h, ++si) {
                    const int s = si % C::NS;
                    bool w_ok = true;
                    if (lane == 0) {
                        w_ok = mbar_wait_idle(&st_empty[s], ((si / C::NS) & 1) ^ 1);
                        if (w_ok) mbar_expect_tx(&b_full[s], C::B_BYTES);
                    }
                    if (!__shfl_sync(0xffffffffu, (int)w_ok, 0)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) tma_load_3d(sB + s * C::B_BYTES, &tmx, rs * GM_RK + h * GM_BK, U.tt * NT, 0, &b_full[s]);
                }
        }
        if (!ok && lane == 0) fail();
        if (lane == 0) {
            const uint32_t first = si > (uint32_t)C::NS ? si - C::NS : 0;
            for (uint32_t j = first; j < si; ++j) mbar_wait(&b_full[j % C::NS], (j / C::NS) & 1);
        }
    } else if (warp == GM_MMA || warp == GM_MMA2) {
        // ---------------- MMA issuers. One thread's tcgen05.mma costs it ~55 cycles,
        // more than a 128 x 64 x 16 MMA takes the tensor core, so below 128 columns
        // the A_hi MMAs (warp GM_MMA) and the A_lo MMAs (warp GM_MMA2) have an
        // issuer each, into separate accumulators. Descriptors are formed once per
        // stage: a K step of 16 inputs is +32 bytes = +2 in the start-address field.
        const bool lo_iss = warp == GM_MMA2;
        if (lane == 0 && (C::ISS == 2 || !lo_iss)) {
            const uint32_t idesc = lo_iss ? umma_idesc(NT) : umma_idesc(2 * NT);
            const uint32_t col = lo_iss ? 2 * NT : 0;
            uint32_t si = 0, nu = 0;
            for (int u = blockIdx.x; u < nunits && !stop(); u += gridDim.x, ++nu) {
                const GmUnit U = gm_unit(a, u, ntt);
                const int ab = nu & 1;
                if (!mbar_wait_idle(&acc_empty[ab], ((nu >> 1) & 1) ^ 1)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + ab * C::ACCW + col;
                uint32_t acc = 0u;
                bool ok = true;
                for (int rs = U.r0; rs < U.r1 && ok; ++rs)
                    for (int h = 0; h < 2; ++h, ++si) {
                        const int s = si % C::NS;
                        const uint32_t par = (si / C::NS) & 1;
                        if (!mbar_wait_idle(&a_full[s], par) || !mbar_wait_idle(&b_full[s], par)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t ah = smem_u32(sA + s * C::A_BYTES);
                        const uint64_t bd = umma_desc_sw128(smem_u32(sB + s * C::B_BYTES));
                        if (C::ISS == 2) {
                            const uint64_t ad = umma_desc_sw128(lo_iss ? ah + GM_BM * GM_BK * 2 : ah);
#pragma unroll
                            for (int kk = 0; kk < GM_BK / 16; ++kk) {
                                umma_f16(d, ad + 2 * kk, bd + 2 * kk, idesc, acc);
                                acc = 1u;
                            }
                        } else {
                            const uint64_t hd = umma_desc_sw128(ah), ld = umma_desc_sw128(ah + GM_BM * GM_BK * 2);
#pragma unroll
                            for (int kk = 0; kk < GM_BK / 16; ++kk) {
                                umma_f16(d, hd + 2 * kk, bd + 2 * kk, idesc, acc);
                                umma_f16(d, ld + 2 * kk, bd + 2 * kk, umma_idesc(NT), 1u);
                                acc = 1u;
                            }
                        }
                        umma_commit(&st_empty[s]);  // the stage's A and B are free once these MMAs finish
                    }
                if (!ok) {
                    fail();
                    break;
                }
                umma_commit(&acc_full[ab]);
            }
            // every MMA issued has finished before TMEM is freed (by warp GM_MMA)
            umma_commit(done);
            if (!lo_iss) mbar_wait(done, 0);
        }
        __syncwarp();
    } else if (warp >= GM_DQ0) {
        // ---------------- dequantizers: warp dw takes row groups dw, dw + GM_NDQ, ...
        const int dw = warp - GM_DQ0;
        uint32_t ri = 0, si = 0;
        int cur_si = -1;
        float wsc = 1.f;
        for (int u = blockIdx.x; u < nunits && !stop(); u += gridDim.x) {
            const GmUnit U = gm_unit(a, u, ntt);
            const GemmSeg& sg = a.seg[U.si];
            if (U.si != cur_si) {
                cur_si = U.si;
                wsc = ldexpf(1.f, gm_wexp(sg));
            }
            bool ok = true;
            for (int rs = U.r0; rs < U.r1 && ok; ++rs, ++ri) {
                const int slot = ri % C::NRAW;
                // every wait's outcome is made warp-uniform (the lanes leave together)
                if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[slot], (ri / C::NRAW) & 1))) {
                    ok = false;
                    break;
                }
                const uint8_t* raw = sR + slot * C::RAW;
                if (C::ISS == 2) {
                    // up to 64 columns: both stages of the slot at once, for more
                    // independent work per warp (28672 x 4096 Q4_0 at 32 columns:
                    // 68 -> 63 us; at 128 columns it is slower, waiting for two stages)
                    const int s0 = si % C::NS, s1 = (si + 1) % C::NS;
                    if (!__all_sync(0xffffffffu, mbar_wait(&st_empty[s0], ((si / C::NS) & 1) ^ 1) &&
                                                     mbar_wait(&st_empty[s1], (((si + 1) / C::NS) & 1) ^ 1))) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint8_t* Ahi = sA + (h ? s1 : s0) * C::A_BYTES;
                        uint8_t* Alo = Ahi + GM_BM * GM_BK * 2;
#pragma unroll
                        for (int j = 0; j < 16 / GM_NDQ; ++j) {
                            const int gi = dw + GM_NDQ * j;
                            const uint8_t* lrec = raw + gi * GmFmt<TYPE>::LREC;
                            const uint8_t* scs = raw + 16 * GmFmt<TYPE>::LREC + gi * GmFmt<TYPE>::SC;
                            if (TYPE == GT_Q6_K)
                                gm_dequant_q6(lrec, scs, Ahi, Alo, gi, h, lane, wsc, ((rs * GM_RK) % 1024) / 16);
                            else
                                gm_dequant<TYPE>(lrec, scs, Ahi, Alo, gi, h, lane, wsc);
                        }
                    }
                    fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's reads
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&a_full[s0]);
                        mbar_arrive(&a_full[s1]);
                    }
                    si += 2;
                } else {
                    for (int h = 0; h < 2; ++h, ++si) {
                        const int s = si % C::NS;
                        if (!__all_sync(0xffffffffu, mbar_wait(&st_empty[s], ((si / C::NS) & 1) ^ 1))) {
                            ok = false;
                            break;
                        }
                        uint8_t* Ahi = sA + s * C::A_BYTES;
                        uint8_t* Alo = Ahi + GM_BM * GM_BK * 2;
#pragma unroll
                        for (int j = 0; j < 16 / GM_NDQ; ++j) {
                            const int gi = dw + GM_NDQ * j;
                            const uint8_t* lrec = raw + gi * GmFmt<TYPE>::LREC;
                            const uint8_t* scs = raw + 16 * GmFmt<TYPE>::LREC + gi * GmFmt<TYPE>::SC;
                            if (TYPE == GT_Q6_K)
                                gm_dequant_q6(lrec, scs, Ahi, Alo, gi, h, lane, wsc, ((rs * GM_RK) % 1024) / 16);
                            else
                                gm_dequant<TYPE>(lrec, scs, Ahi, Alo, gi, h, lane, wsc);
                        }
                        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's reads
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[s]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[slot]);
            }
            if (!ok) {
                if (lane == 0) fail();
                break;
            }
        }
    } else {
        // ---------------- epilogue: warp q owns TMEM lanes / tile rows 32q .. 32q+31.
        // The four warps never wait for each other: with split-K each warp has its
        // own arrival counter per output tile (cnt[tile * 4 + q]).
        pdl_wait();  // column scales, residual rows, caches: after the previous kernel
        const int q = warp, r = q * 32 + lane;
        float* exs = ep_xs + q * NT;
        uint32_t* eps = ep_pos + q * NT;
        uint32_t* esl = ep_slot + q * NT;
        uint32_t nu = 0;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++nu) {
            const GmUnit U = gm_unit(a, u, ntt);
            const GemmSeg& sg = a.seg[U.si];
            const int ab = nu & 1;
            const int t0 = U.tt * NT;
            // the unit's column scales (2^e_t of the input, 2^-eA of the weights) and positions
            {
                const float wsc = ldexpf(1.f, -gm_wexp(sg));
                for (int j = lane; j < NT; j += 32) {
                    const int t = t0 + j;
                    exs[j] = t < ntok ? a.xs[t] * wsc : 0.f;
                    eps[j] = t < ntok ? a.bp->pos[t] : 0u;
                    esl[j] = t < ntok ? a.bp->slot[t] : 0u;
                }
                __syncwarp();
            }
            if (!__all_sync(0xffffffffu, mbar_wait_idle(&acc_full[ab], (nu >> 1) & 1))) {
                if (lane == 0) fail();
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * C::ACCW;
            float* part = a.S > 1 ? a.ws + ((size_t)(U.tile * a.S + U.ks) * NT) * GM_BM : nullptr;
#pragma unroll 1
            for (int c = 0; c < NT; c += 16) {
                float vh[16], vl[16];
                tmem_ld16(tbase + c, vh);
                tmem_ld16(tbase + NT + c, vl);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) vh[j] += vl[j];
                if (C::ISS == 2) {  // + A_lo x x_hi
                    tmem_ld16(tbase + 2 * NT + c, vl);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) vh[j] += vl[j];
                }
                if (part) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) part[(size_t)(c + j) * GM_BM + r] = vh[j];
                } else {
                    gm_epi<8>(a, sg, U.lt, r, t0 + c, ntok, vh, exs + c, eps + c, esl + c);
                    gm_epi<8>(a, sg, U.lt, r, t0 + c + 8, ntok, vh + 8, exs + c + 8, eps + c + 8, esl + c + 8);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
            if (!part) continue;
            // split-K: the unit that completes the tile's rows adds the slices in
            // slice order (the same order every run)
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                unsigned* cp = &a.cnt[U.tile * 4 + q];
                last = atomicAdd(cp, 1u) == (unsigned)(a.S - 1);
                if (last) *cp = 0u;  // every slice has arrived: ready for the next launch
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            __threadfence();
            const float* base = a.ws + ((size_t)U.tile * a.S * NT) * GM_BM;
            // 8 columns of up to 4 slices per round trip to L2 (32 loads in flight),
            // added in slice order
#pragma unroll 1
            for (int c = 0; c < NT; c += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = 0.f;
                for (int s0 = 0; s0 < a.S; s0 += 4) {
                    float w[4][8];
#pragma unroll
                    for (int k = 0; k < 4; ++k)
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            w[k][j] = s0 + k < a.S ? __ldcg(base + ((size_t)(s0 + k) * NT + c + j) * GM_BM + r) : 0.f;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (s0 + k < a.S) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) v[j] += w[k][j];
                        }
                }
                gm_epi<8>(a, sg, U.lt, r, t0 + c, ntok, v, exs + c, eps + c, esl + c);
            }
        }
    }
    // ---------------- teardown: every role is out of its loop
    tc_fence_before();
    __syncthreads();
    // tensor parallel: the CTA's peer stores are done; the release at system
    // scope carries them (through the barrier above) to k_tp_join_b's acquire
    if (a.lar && threadIdx.x == 0) red_release_sys_add_u64(a.lar, 1ull);
    if (warp == GM_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TCOLS));
    }
}

// ---------------------------------------------------------------- activation format

// One CTA per token column t (prefill position or sequence) of the first
// `gridDim.x` columns of the [2][Tp][ldp] planes: the input row
// x[t] (RMSNorm with norm_w first when set: src/math/ops.rs:5-12, (x * s) * w),
// scaled by 2^-e_t so its largest |value| lies in [2^14, 2^15), split into
// f16 hi / lo planes [2][Tp][ldp] (zeros past K and for t >= n); xs[t] = 2^e_t.
// R: elements per thread (the row is read once into registers); KP <= 1024 R.
template <int R>
__global__ void __launch_bounds__(1024) k_xfmt_g(const float* x, int ldx, int K, int KP, int ldp, int Tp,
                                                 const float* norm_w, float eps, const BatchParams* bp, __half* planes,
                                                 float* xs) {
    __shared__ float red[32];
    pdl_launch();  // the GEMM that reads these planes may start its weight copies now
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __half* hi = planes + (size_t)t * ldp;
    __half* lo = planes + ((size_t)Tp + t) * ldp;
    if (t >= bp->n) {
        for (int k = tid; k < KP; k += blockDim.x) hi[k] = lo[k] = __float2half_rn(0.f);
        if (tid == 0) xs[t] = 0.f;
        return;
    }
    const float* xr = x + (size_t)t * ldx;
    auto block_reduce = [&](float v, bool is_max) -> float {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        __syncthreads();
        if (lane == 0) red[warp] = v;
        __syncthreads();
        float tot = 0.f;
        const int nw = blockDim.x >> 5;
        for (int i = 0; i < nw; ++i) tot = is_max ? fmaxf(tot, red[i]) : tot + red[i];
        return tot;
    };
    float v[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int k = tid + i * 1024;
        v[i] = k < K ? xr[k] : 0.f;
    }
    if (norm_w) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < R; ++i)
            if (tid + i * 1024 < K) ss = fmaf(v[i], v[i], ss);
        const float tot = block_reduce(ss, false);
        const float s = 1.0f / sqrtf(tot / (float)K + eps);
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int k = tid + i * 1024;
            if (k < K) v[i] = __fmul_rn(__fmul_rn(v[i], s), norm_w[k]);
        }
    }
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < R; ++i)
        if (tid + i * 1024 < K) m = fmaxf(m, fabsf(v[i]));
    m = block_reduce(m, true);
    int e = 0;
    if (m > 0.f && isfinite(m)) {
        int ex;
        frexpf(m, &ex);  // m in [2^(ex-1), 2^ex)
        e = ex - 15;
    }
    const float down = ldexpf(1.f, -e);
    if (tid == 0) xs[t] = ldexpf(1.f, e);
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int k = tid + i * 1024;
        if (k < KP) {
            const float y = k < K ? v[i] * down : 0.f;
            const __half h = __float2half_rn(y);
            hi[k] = h;
            lo[k] = __float2half_rn(y - __half2float(h));
        }
    }
}

// ---------------------------------------------------------------- host side

template <int TYPE, int NT>
static cudaError_t gemm_attr() {
    return cudaFuncSetAttribute(k_gemm<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, GmCfg<TYPE, NT>::SMEM);
}

cudaError_t gemm_configure() {
    cudaError_t e;
#define TALOS_GM_ATTR(T)                                   \
    if ((e = gemm_attr<T, 32>()) != cudaSuccess) return e; \
    if ((e = gemm_attr<T, 64>()) != cudaSuccess) return e; \
    if ((e = gemm_attr<T, 128>()) != cudaSuccess) return e;
    TALOS_GM_ATTR(GT_Q4_0)
    TALOS_GM_ATTR(GT_Q8_0)
    TALOS_GM_ATTR(GT_Q6_K)
#undef TALOS_GM_ATTR
    return cudaSuccess;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn g_enc = nullptr;
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link to libcuda).
static cudaError_t gemm_encoder() {
    if (g_enc) return cudaSuccess;
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    g_enc = (EncodeTiledFn)fn;
    return cudaSuccess;
}

cudaError_t gemm_tensor_map(void* planes, int ldp, int Tp, int nt, void* map_out) {
    cudaError_t e = gemm_encoder();
    if (e != cudaSuccess) return e;
    EncodeTiledFn enc = g_enc;
    // dims: k (ldp halves, contiguous), token t (Tp), plane (2: hi, lo); box
    // 64 x nt x 2: one stage's inputs, 128 bytes per (plane, column) row, swizzled
    const cuuint64_t dims[3] = {(cuuint64_t)ldp, (cuuint64_t)Tp, 2};
    const cuuint64_t strides[2] = {(cuuint64_t)ldp * 2, (cuuint64_t)Tp * ldp * 2};
    const cuuint32_t box[3] = {GM_BK, (cuuint32_t)nt, 2};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc((CUtensorMap*)map_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, planes, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The two tensor maps of a packed quant weight for the GEMM's weight producer:
// the packed array viewed as u32 [groups][chunks][GCB / 4], boxes of 16 groups x
// one chunk x (the lane records of one raw slot | its scales).
template <int TYPE>
static cudaError_t gemm_weight_maps_t(const PackedW& w, void* lrec_map, void* sc_map) {
    using F = GmFmt<TYPE>;
    const cuuint64_t dims[3] = {(cuuint64_t)F::GCB / 4, (cuuint64_t)w.nk, (cuuint64_t)w.rows_pad / 8};
    const cuuint64_t strides[2] = {(cuuint64_t)F::GCB, (cuuint64_t)F::GCB * w.nk};
    const cuuint32_t box_l[3] = {(cuuint32_t)F::LREC / 4, 1, 16};
    const cuuint32_t box_s[3] = {(cuuint32_t)F::SC / 4, 1, 16};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_enc((CUtensorMap*)lrec_map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, (void*)w.p0, dims, strides, box_l,
                       estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
        r = g_enc((CUtensorMap*)sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, (void*)w.p0, dims, strides, box_s, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t gemm_weight_maps(const PackedW& w, void* lrec_map, void* sc_map) {
    cudaError_t e = gemm_encoder();
    if (e != cudaSuccess) return e;
    switch (w.type) {
        case GT_Q4_0: return gemm_weight_maps_t<GT_Q4_0>(w, lrec_map, sc_map);
        case GT_Q8_0: return gemm_weight_maps_t<GT_Q8_0>(w, lrec_map, sc_map);
        case GT_Q6_K: return gemm_weight_maps_t<GT_Q6_K>(w, lrec_map, sc_map);
    }
    return cudaErrorInvalidValue;
}

size_t gemm_map_bytes() { return sizeof(CUtensorMap); }

template <int TYPE, int NT>
static cudaError_t gemm_go(const void* map, const GemmArgs& a, int grid, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GM_THREADS);
    cfg.dynamicSmemBytes = GmCfg<TYPE, NT>::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemm<TYPE, NT>, *(const CUtensorMap*)map, a);
}

cudaError_t launch_gemm(const void* map, const GemmArgs& a, int type, int nt, int grid, cudaStream_t s, bool pdl) {
    if (a.KP % GM_RK || a.nseg < 1 || a.nseg > 3 || a.S < 1 || grid < 1) return cudaErrorInvalidValue;
#define TALOS_GM_GO(T)                                      \
    if (type == T) {                                        \
        if (nt == 32) return gemm_go<T, 32>(map, a, grid, s, pdl);   \
        if (nt == 64) return gemm_go<T, 64>(map, a, grid, s, pdl);   \
        if (nt == 128) return gemm_go<T, 128>(map, a, grid, s, pdl); \
    }
    TALOS_GM_GO(GT_Q4_0)
    TALOS_GM_GO(GT_Q8_0)
    TALOS_GM_GO(GT_Q6_K)
#undef TALOS_GM_GO
    return cudaErrorInvalidValue;
}

cudaError_t launch_xfmt_g(const float* x, int ldx, int K, int KP, int ldp, int Tp, int ncols, const float* norm_w,
                          float eps, const BatchParams* bp, void* planes, float* xs, cudaStream_t s) {
    if (KP > ldp || KP < K || ncols < 1 || ncols > Tp || KP > 32 * 1024) return cudaErrorInvalidValue;
    __half* pl = (__half*)planes;
    if (KP <= 4 * 1024)
        k_xfmt_g<4><<<ncols, 1024, 0, s>>>(x, ldx, K, KP, ldp, Tp, norm_w, eps, bp, pl, xs);
    else if (KP <= 8 * 1024)
        k_xfmt_g<8><<<ncols, 1024, 0, s>>>(x, ldx, K, KP, ldp, Tp, norm_w, eps, bp, pl, xs);
    else if (KP <= 16 * 1024)
        k_xfmt_g<16><<<ncols, 1024, 0, s>>>(x, ldx, K, KP, ldp, Tp, norm_w, eps, bp, pl, xs);
    else
        k_xfmt_g<32><<<ncols, 1024, 0, s>>>(x, ldx, K, KP, ldp, Tp, norm_w, eps, bp, pl, xs);
    return cudaGetLastError();
}

}  // namespace talos
