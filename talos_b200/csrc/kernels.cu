// kernels.cu -- dequantization, attention and the small per-token kernels of the
// Talos decode path on B200 (sm_100a). The matvec lives in matvec.cu.
//
// Reference algorithm (Tsuskov/talos, Rust): src/model/llama.rs:96-183 and the
// kernels it calls in src/math/ops.rs and src/gguf/dtype.rs. Built without
// --use_fast_math; where the reference's rounding order matters the code uses
// explicit __fmul_rn / __fadd_rn.
#include <cooperative_groups.h>
#include <math.h>

#include "kernels.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace talos {

__device__ __forceinline__ void pdl_wait_k() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_k() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch `kernel` with programmatic stream serialization (PDL) when pdl is set.
template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             bool pdl, int cluster_x, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// =====================================================================
// Dequantization (bit-exact with src/gguf/dtype.rs:64-121)
// =====================================================================

__global__ void k_dequant(int type, const uint8_t* raw, size_t n, float* out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
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
// Decode attention (src/model/llama.rs:135-155)
// =====================================================================
//
// One cluster of AT_CL CTAs per kv head; CTA r of the cluster takes positions
// [r*ch, (r+1)*ch) of the seq = pos + 1 cached ones, for all `group` query heads
// that share the kv head (h / group == kvh), so every K/V row is read once.
//   1. K/V rows of the CTA's range are staged in shared memory; rows before pos
//      are fetched before griddepcontrol.wait (the KV prefix is written by
//      earlier tokens), the row at pos after it (written by this token's qkv).
//   2. scores s = (q . k) * (1/sqrt(hd)) for (position, head) pairs, one per
//      lane; softmax pieces m = max s, l = sum exp(s - m) per head;
//   3. o = sum_t exp(s_t - m) v_t per (head, 4 dims) per thread;
//   4. the CTAs of the cluster merge (m, l, o) through distributed shared memory
//      in rank order: out = sum_r o_r e^(m_r - M) / sum_r l_r e^(m_r - M).
// The merge is fixed-order, so the result does not depend on scheduling.

constexpr int AT_CL = 8;        // CTAs per kv head (portable cluster size)
constexpr int AT_THREADS = 128;
constexpr int AT_PB = 64;       // positions staged per pass
constexpr int AT_MAXG = 8;

struct AttnSmem {
    static __host__ __device__ int stride(int hd) { return hd + 4; }  // floats; 16-B aligned, bank-skewed rows
    static __host__ __device__ size_t bytes(int hd, int group) {
        int st = stride(hd);
        return (size_t)(2 * AT_PB * st + group * st + group * AT_PB + 2 * AT_MAXG + group * hd) * 4;
    }
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(AT_THREADS) k_attention(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = a.hd, st = AttnSmem::stride(hd), nrow4 = hd / 4;
    const int group = a.n_head / a.n_kv;
    const int kvh = blockIdx.x / AT_CL;
    const int rank = (int)cluster.block_rank();
    float* Ks = sm;                        // [AT_PB][st]
    float* Vs = Ks + AT_PB * st;           // [AT_PB][st]
    float* qs = Vs + AT_PB * st;           // [group][st]
    float* ps = qs + group * st;           // [group][AT_PB]
    float* ml = ps + group * AT_PB;        // (m, l) per head, 2 * AT_MAXG
    float* os = ml + 2 * AT_MAXG;          // [group][hd]

    // pos was written at least two kernels earlier in the stream; read it through L2.
    const int pos = (int)__ldcg(&a.step->pos);
    const int seq = pos + 1;
    const int ch = (seq + AT_CL - 1) / AT_CL;
    const int t0 = rank * ch;
    const int t1 = min(seq, t0 + ch);

    // cp.async rows [base, base + n) that satisfy lo <= t < hi
    auto stage_rows = [&](int base, int n, int lo, int hi) {
        for (int i = tid; i < n * nrow4; i += AT_THREADS) {
            const int r = i / nrow4, c4 = i % nrow4;
            const int t = base + r;
            if (t >= lo && t < hi) {
                const size_t off = (size_t)t * a.kv_dim + (size_t)kvh * hd + 4 * c4;
                if (a.kv_f16) {  // widen on the way into shared memory
                    const uint2 kr = __ldcg((const uint2*)((const __half*)a.kc + off));
                    const uint2 vr = __ldcg((const uint2*)((const __half*)a.vc + off));
                    const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kr.x));
                    const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kr.y));
                    const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
                    const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
                    *(float4*)(Ks + r * st + 4 * c4) = make_float4(k0.x, k0.y, k1.x, k1.y);
                    *(float4*)(Vs + r * st + 4 * c4) = make_float4(v0.x, v0.y, v1.x, v1.y);
                } else {
                    cp_async16(Ks + r * st + 4 * c4, (const float*)a.kc + off);
                    cp_async16(Vs + r * st + 4 * c4, (const float*)a.vc + off);
                }
            }
        }
    };

    const int n_items = group * nrow4;  // (head, 4 dims) output items, <= 2 per thread
    float4 oacc[2] = {make_float4(0, 0, 0, 0), make_float4(0, 0, 0, 0)};
    float m_it[2] = {-INFINITY, -INFINITY}, l_it[2] = {0.f, 0.f};

    // Rows before pos are cached by earlier tokens: fetch them before waiting on
    // this token's qkv kernel; the row at pos and q come after the wait.
    const int first_n = min(AT_PB, max(t1 - t0, 0));
    stage_rows(t0, first_n, 0, pos);
    pdl_wait_k();
    pdl_launch_k();
    stage_rows(t0, first_n, pos, pos + 1);
    for (int i = tid; i < group * nrow4; i += AT_THREADS) {
        const int g = i / nrow4, c4 = i % nrow4;
        *(float4*)(qs + g * st + 4 * c4) = *(const float4*)(a.q + (size_t)(kvh * group + g) * hd + 4 * c4);
    }

    const int per_warp = 32 / group;  // positions per warp per pass
    const int g_l = lane % group, t_l = lane / group;
    for (int base = t0; base < t1; base += AT_PB) {
        const int n = min(AT_PB, t1 - base);
        if (base != t0) {
            __syncthreads();  // previous pass done with Ks/Vs
            stage_rows(base, n, 0, seq);
        }
        cp_async_wait_all();
        __syncthreads();
        // ---- scores s = (q . k) * scale: lane -> (position, head)
        for (int p0 = warp * per_warp; p0 < n; p0 += (AT_THREADS / 32) * per_warp) {
            const int p = p0 + t_l;
            if (t_l < per_warp && p < n) {
                const float* kr = Ks + p * st;
                const float* qr = qs + g_l * st;
                float dot = 0.f;
                for (int c = 0; c < hd; c += 4) {
                    const float4 kv = *(const float4*)(kr + c);
                    const float4 qv = *(const float4*)(qr + c);
                    dot = fmaf(qv.x, kv.x, dot);
                    dot = fmaf(qv.y, kv.y, dot);
                    dot = fmaf(qv.z, kv.z, dot);
                    dot = fmaf(qv.w, kv.w, dot);
                }
                ps[g_l * AT_PB + p] = __fmul_rn(dot, a.scale);
            }
        }
        __syncthreads();
        // ---- per head: pass max, exp, pass sum (src/math/ops.rs:15-25 pieces)
        for (int gg = warp; gg < group; gg += AT_THREADS / 32) {
            float mx = -INFINITY;
            for (int p = lane; p < n; p += 32) mx = fmaxf(mx, ps[gg * AT_PB + p]);
            mx = warp_max(mx);
            float sum = 0.f;
            for (int p = lane; p < n; p += 32) {
                const float e = expf(ps[gg * AT_PB + p] - mx);
                ps[gg * AT_PB + p] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                ml[2 * gg] = mx;
                ml[2 * gg + 1] = sum;
            }
        }
        __syncthreads();
        // ---- o = sum_p e_p v_p, merged into the running (m, l, o) of each item
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int idx = tid + k * AT_THREADS;
            if (idx < n_items) {
                const int gi = idx / nrow4, c4 = idx % nrow4;
                const float mp = ml[2 * gi], lp = ml[2 * gi + 1];
                const float mn = fmaxf(m_it[k], mp);
                const float c_old = expf(m_it[k] - mn), c_new = expf(mp - mn);
                float4 acc = make_float4(0, 0, 0, 0);
                for (int p = 0; p < n; ++p) {
                    const float e = ps[gi * AT_PB + p];
                    const float4 v = *(const float4*)(Vs + p * st + 4 * c4);
                    acc.x = fmaf(e, v.x, acc.x);
                    acc.y = fmaf(e, v.y, acc.y);
                    acc.z = fmaf(e, v.z, acc.z);
                    acc.w = fmaf(e, v.w, acc.w);
                }
                oacc[k].x = fmaf(oacc[k].x, c_old, acc.x * c_new);
                oacc[k].y = fmaf(oacc[k].y, c_old, acc.y * c_new);
                oacc[k].z = fmaf(oacc[k].z, c_old, acc.z * c_new);
                oacc[k].w = fmaf(oacc[k].w, c_old, acc.w * c_new);
                l_it[k] = fmaf(l_it[k], c_old, lp * c_new);
                m_it[k] = mn;
            }
        }
    }
    __syncthreads();
    // ---- publish this CTA's (m, l, o); CTAs without positions publish m = -inf
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int idx = tid + k * AT_THREADS;
        if (idx < n_items) {
            const int gi = idx / nrow4, c4 = idx % nrow4;
            *(float4*)(os + gi * hd + 4 * c4) = oacc[k];
            if (c4 == 0) {
                ml[2 * gi] = m_it[k];
                ml[2 * gi + 1] = l_it[k];
            }
        }
    }
    cluster.sync();
    // ---- merge over the cluster in rank order; CTA `rank` writes every AT_CL-th output
    for (int idx = rank * AT_THREADS + tid; idx < group * hd; idx += AT_CL * AT_THREADS) {
        const int gi = idx / hd, d = idx % hd;
        float M = -INFINITY;
        for (int r = 0; r < AT_CL; ++r) M = fmaxf(M, cluster.map_shared_rank(ml, r)[2 * gi]);
        float L = 0.f, O = 0.f;
        for (int r = 0; r < AT_CL; ++r) {
            const float* rml = cluster.map_shared_rank(ml, r);
            const float mr = rml[2 * gi];
            if (mr != -INFINITY) {
                const float c = expf(mr - M);
                L = fmaf(rml[2 * gi + 1], c, L);
                O = fmaf(cluster.map_shared_rank(os, r)[gi * hd + d], c, O);
            }
        }
        a.out[(size_t)(kvh * group + gi) * hd + d] = O / L;
    }
    cluster.sync();
}

size_t attention_smem_bytes(int hd, int group) { return AttnSmem::bytes(hd, group); }

cudaError_t attention_configure() {
    return cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int group = a.n_head / a.n_kv;
    if (group > AT_MAXG || a.hd % 4 || a.hd > 256 || group * (a.hd / 4) > 2 * AT_THREADS)
        return cudaErrorInvalidValue;
    return launch_ex(k_attention, dim3(a.n_kv * AT_CL), dim3(AT_THREADS), AttnSmem::bytes(a.hd, group), s, pdl,
                     AT_CL, a);
}

// =====================================================================
// Small kernels
// =====================================================================

// x = dequant(token_embd row step->token) (weights.rs:58-62); clears the argmax key.
__global__ void k_embed(const uint8_t* raw, int type, int cols, int vocab, StepParams* step, float* x) {
    pdl_wait_k();
    pdl_launch_k();
    uint32_t tok = step->token;
    if (tok >= (uint32_t)vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) step->error |= 1u;
        tok = 0;
    }
    const int be = type == GT_F32 ? 1 : (type == GT_Q6_K ? 256 : 32);
    const int bb = type == GT_F32 ? 4 : (type == GT_Q6_K ? 210 : (type == GT_Q8_0 ? 34 : 18));
    const uint8_t* row = raw + (size_t)tok * (cols / be) * bb;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
        x[i] = dequant_elem(type, row, i);
    if (threadIdx.x == 0 && blockIdx.x == 0) step->argmax_key = 0ull;
}

cudaError_t launch_embed(const uint8_t* raw, int type, int cols, int vocab, StepParams* step, float* x,
                         cudaStream_t s, bool pdl) {
    int blocks = (cols + 255) / 256;
    if (blocks > 64) blocks = 64;
    return launch_ex(k_embed, dim3(blocks), dim3(256), 0, s, pdl, 1, raw, type, cols, vocab, step, x);
}

__global__ void k_rmsnorm(const float* x, const float* w, float eps, int n, float* out) {
    pdl_wait_k();
    pdl_launch_k();
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
    const float scale = 1.0f / sqrtf(red[0] / (float)n + eps);
    for (int k = threadIdx.x; k < n; k += blockDim.x) out[k] = __fmul_rn(__fmul_rn(x[k], scale), w[k]);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, float* out, cudaStream_t s, bool pdl) {
    return launch_ex(k_rmsnorm, dim3(1), dim3(1024), 0, s, pdl, 1, x, w, eps, n, out);
}

__global__ void k_greedy_advance(StepParams* step, uint32_t* gen, int cap) {
    pdl_wait_k();
    pdl_launch_k();
    const uint32_t tok = (uint32_t)(step->argmax_key & 0xffffffffull);
    const uint32_t n = step->n_gen;
    if (n < (uint32_t)cap) gen[n] = tok;
    step->n_gen = n + 1;
    step->token = tok;
    step->pos = step->pos + 1;
}

// Perplexity (src/eval.rs:18-23): acc[0] += -log softmax(logits)[target], the
// log-sum-exp in f64 like token_nll; acc[1] counts the scored positions.
// One block of 1024 threads, fixed reduction order (deterministic).
__global__ void k_token_nll(const float* logits, int n, uint32_t target, double* acc) {
    __shared__ float smax[32];
    __shared__ double ssum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float m = -INFINITY;
    for (int i = tid; i < n; i += blockDim.x) m = fmaxf(m, logits[i]);
    m = warp_max(m);
    if (lane == 0) smax[warp] = m;
    __syncthreads();
    m = smax[0];
    for (int w = 1; w < (int)(blockDim.x / 32); ++w) m = fmaxf(m, smax[w]);
    double se = 0.0;
    for (int i = tid; i < n; i += blockDim.x) se += exp((double)(logits[i] - m));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    if (lane == 0) ssum[warp] = se;
    __syncthreads();
    if (tid == 0) {
        double tot = 0.0;
        for (int w = 0; w < (int)(blockDim.x / 32); ++w) tot += ssum[w];
        const double log_prob = (double)(logits[target] - m) - log(tot);
        const float nll = (float)(-log_prob);
        acc[0] += (double)nll;
        acc[1] += 1.0;
    }
}

cudaError_t launch_token_nll(const float* logits, int n, uint32_t target, double* acc, cudaStream_t s) {
    k_token_nll<<<1, 1024, 0, s>>>(logits, n, target, acc);
    return cudaGetLastError();
}

// sample::argmax (src/sample.rs:7-14) over n values: the largest argmax_key, the
// same key the logits epilogues of the decode step reduce.
__global__ void k_argmax(const float* v, size_t n, unsigned long long* key) {
    unsigned long long best = 0ull;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const unsigned long long k = argmax_key(v[i], (uint32_t)i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long oth = __shfl_xor_sync(0xffffffffu, best, o);
        best = oth > best ? oth : best;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(key, best);
}

cudaError_t launch_argmax(const float* v, size_t n, unsigned long long* key, cudaStream_t s) {
    size_t blocks = (n + 255) / 256;
    if (blocks > 1184) blocks = 1184;
    if (blocks == 0) blocks = 1;
    cudaError_t e = cudaMemsetAsync(key, 0, sizeof(unsigned long long), s);
    if (e != cudaSuccess) return e;
    k_argmax<<<(unsigned)blocks, 256, 0, s>>>(v, n, key);
    return cudaGetLastError();
}

cudaError_t launch_greedy_advance(StepParams* step, uint32_t* gen, int cap, cudaStream_t s, bool pdl) {
    return launch_ex(k_greedy_advance, dim3(1), dim3(1), 0, s, pdl, 1, step, gen, cap);
}


// ----------------------------------------------------------------------------
// Batched decode: the small per-sequence steps around the batched matvec
// ----------------------------------------------------------------------------

__global__ void k_embed_b(const uint8_t* raw, int type, int cols, int vocab, const BatchParams* bp, float* x,
                          int ldx) {
    const int s = blockIdx.y;
    if (s >= bp->n) return;
    uint32_t tok = bp->token[s];
    if (tok >= (uint32_t)vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr((unsigned*)&bp->error, 1u);
        tok = 0;
    }
    const int be = type == GT_F32 ? 1 : (type == GT_Q6_K ? 256 : 32);
    const int bb = type == GT_F32 ? 4 : (type == GT_Q6_K ? 210 : (type == GT_Q8_0 ? 34 : 18));
    const uint8_t* row = raw + (size_t)tok * (cols / be) * bb;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < cols) x[(size_t)s * ldx + i] = dequant_elem(type, row, i);
}

cudaError_t launch_embed_b(const uint8_t* raw, int type, int cols, int vocab, const BatchParams* bp, float* x,
                           int ldx, cudaStream_t s) {
    k_embed_b<<<dim3((cols + 255) / 256, MB_SEQ), 256, 0, s>>>(raw, type, cols, vocab, bp, x, ldx);
    return cudaGetLastError();
}

// One CTA per (query head, sequence), 8 warps: warp w takes positions w, w+8, ...
// in rounds of 4 (all K/V loads of a round in flight), keeps an online softmax
// (max m, sum l, unnormalised o; lane = 4 dims), and the warps merge in shared
// memory: out = o / l (src/math/ops.rs:15-25 applied to the merged sums).
#ifndef TALOS_ATB_MINB
#define TALOS_ATB_MINB 4
#endif
#ifndef TALOS_ATB_ROUND
#define TALOS_ATB_ROUND 4
#endif
constexpr int ATB_WARPS = 8, ATB_ROUND = TALOS_ATB_ROUND;
__global__ void __launch_bounds__(ATB_WARPS * 32, TALOS_ATB_MINB) k_attention_b(const float* q, int ldq, const float* kc,
                                                                const float* vc, size_t seq_stride, int kv_dim,
                                                                int n_head, int n_kv, int hd, float* out, int ldo,
                                                                const BatchParams* bp) {
    const int h = blockIdx.x, s = blockIdx.y;
    if (s >= bp->n) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int seq = (int)bp->pos[s] + 1, kh = h / (n_head / n_kv), hs = hd + 4;
    const float scale = 1.0f / sqrtf((float)hd);
    extern __shared__ float wsm[];  // [8 warps][hd + 4]
    const bool act = 4 * lane < hd;
    float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (act) q4 = *(const float4*)(q + (size_t)s * ldq + (size_t)h * hd + 4 * lane);
    const size_t so = (size_t)bp->slot[s] * seq_stride;
    const float* K0 = kc + so + (size_t)kh * hd + 4 * lane;
    const float* V0 = vc + so + (size_t)kh * hd + 4 * lane;
    float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    for (int t0 = warp; t0 < seq; t0 += ATB_WARPS * ATB_ROUND) {
        float4 kv[ATB_ROUND], vv[ATB_ROUND];
#pragma unroll
        for (int u = 0; u < ATB_ROUND; ++u) {
            const int t = t0 + u * ATB_WARPS;
            kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            vv[u] = kv[u];
            if (act && t < seq) {
                kv[u] = *(const float4*)(K0 + (size_t)t * kv_dim);
                vv[u] = *(const float4*)(V0 + (size_t)t * kv_dim);
            }
        }
        float sc[ATB_ROUND];
#pragma unroll
        for (int u = 0; u < ATB_ROUND; ++u)
            sc[u] = fmaf(q4.x, kv[u].x, fmaf(q4.y, kv[u].y, fmaf(q4.z, kv[u].z, q4.w * kv[u].w)));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < ATB_ROUND; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
        float mx = m;
#pragma unroll
        for (int u = 0; u < ATB_ROUND; ++u) {
            sc[u] = t0 + u * ATB_WARPS < seq ? sc[u] * scale : -INFINITY;
            mx = fmaxf(mx, sc[u]);
        }
        const float cr = expf(m - mx);
        l *= cr;
        o0 *= cr, o1 *= cr, o2 *= cr, o3 *= cr;
#pragma unroll
        for (int u = 0; u < ATB_ROUND; ++u) {
            const float pe = expf(sc[u] - mx);
            l += pe;
            o0 = fmaf(pe, vv[u].x, o0);
            o1 = fmaf(pe, vv[u].y, o1);
            o2 = fmaf(pe, vv[u].z, o2);
            o3 = fmaf(pe, vv[u].w, o3);
        }
        m = mx;
    }
    float* w = wsm + warp * hs;
    if (lane == 0) {
        w[0] = m;
        w[1] = l;
    }
    if (act) *(float4*)(w + 4 + 4 * lane) = make_float4(o0, o1, o2, o3);
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float M = -INFINITY;
        for (int ww = 0; ww < ATB_WARPS; ++ww) M = fmaxf(M, wsm[ww * hs]);
        float L = 0.f, O = 0.f;
        for (int ww = 0; ww < ATB_WARPS; ++ww) {
            const float* r = wsm + ww * hs;
            const float e = r[0] == -INFINITY ? 0.f : expf(r[0] - M);
            L = fmaf(r[1], e, L);
            O = fmaf(r[4 + d], e, O);
        }
        out[(size_t)s * ldo + (size_t)h * hd + d] = O / L;
    }
}

__global__ void k_swiglu_b(const float* g, const float* u, float* h, int ld, int n_ff, const BatchParams* bp) {
    const int s = blockIdx.y;
    if (s >= bp->n) return;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_ff) {
        const size_t o = (size_t)s * ld + i;
        h[o] = __fmul_rn(silu_ref(g[o]), u[o]);
    }
}

// One CTA per column: its logits row's sample::argmax key (argmax_key: total
// order, the larger index on ties), reduced warp by warp then across warps.
__global__ void __launch_bounds__(1024) k_greedy_advance_b(const float* logits, int V, BatchParams* bp,
                                                           uint32_t* gen, int cap) {
    __shared__ unsigned long long wk[32];
    const int s = blockIdx.x;
    if (s >= bp->n) return;
    const float* row = logits + (size_t)s * V;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long k = argmax_key(row[i], (uint32_t)i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long oth = __shfl_xor_sync(0xffffffffu, best, o);
        best = oth > best ? oth : best;
    }
    if ((threadIdx.x & 31) == 0) wk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = wk[w] > best ? wk[w] : best;
        best = wk[0] > best ? wk[0] : best;
        const uint32_t tok = (uint32_t)(best & 0xffffffffull);
        const uint32_t n = bp->ngen[s];
        if (n < (uint32_t)cap) gen[(size_t)s * cap + n] = tok;
        bp->ngen[s] = n + 1;
        bp->token[s] = tok;
        bp->pos[s] += 1;
        if (s == 0) bp->tpstep += 1;  // read only by the next step's kernels
    }
}

cudaError_t launch_greedy_advance_b(const float* logits, int V, BatchParams* bp, uint32_t* gen, int cap,
                                    cudaStream_t s) {
    k_greedy_advance_b<<<MB_SEQ, 1024, 0, s>>>(logits, V, bp, gen, cap);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_b(const float* g, const float* u, float* h, int ld, int n_ff, const BatchParams* bp,
                            cudaStream_t s) {
    k_swiglu_b<<<dim3((n_ff + 255) / 256, MB_SEQ), 256, 0, s>>>(g, u, h, ld, n_ff, bp);
    return cudaGetLastError();
}

cudaError_t launch_attention_b(const float* q, int ldq, const float* kc, const float* vc, size_t seq_stride,
                               int kv_dim, int n_head, int n_kv, int hd, float* out, int ldo, const BatchParams* bp,
                               cudaStream_t s) {
    if (hd > 128 || hd % 4) return cudaErrorInvalidValue;
    const size_t sm = (size_t)ATB_WARPS * (hd + 4) * 4;
    k_attention_b<<<dim3(n_head, MB_SEQ), ATB_WARPS * 32, sm, s>>>(q, ldq, kc, vc, seq_stride, kv_dim, n_head, n_kv,
                                                                   hd, out, ldo, bp);
    return cudaGetLastError();
}


// ---------------------------------------------------------------- tensor-parallel join

// Bounded spin of one thread until *c >= target (system scope: peers add to c).
__device__ __noinline__ bool tp_wait(const unsigned long long* c, unsigned long long target) {
    if (ld_acquire_sys_u64(c) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 16; ++i)
            if (ld_acquire_sys_u64(c) >= target) return true;
        if (globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) { return *(const volatile unsigned*)p; }

// The join after each EPI_B_PEER GEMM of a tensor-parallel batched step. CTA 0
// takes the GEMM's exit arrivals (an acquire of what its CTAs released, so their
// peer stores are ordered before what this thread releases next), clears that
// counter for the next GEMM, and adds 1 at system scope to counter `inst` of
// every rank. Then every CTA waits until all tp ranks have arrived in this step:
// (tpstep + 1) * tp, the counters growing across steps until talos_ctx_tp_resync
// clears them. With rx set the ranks' partial rows are added to the residual in
// rank order, x += ((rx_0 + rx_1) + ...) (src/model/llama.rs:159-161, 174-176,
// the row-parallel product split over ranks); every rank sums the same slots in
// the same order, so the residual stays identical on all ranks.
// A wait that runs out (2 s) sets error bit 2 and every rank's abort word. A
// step that has already failed, or whose abort word a peer has set, skips its
// waits but still signals, so every rank leaves the step soon and reports it.
__global__ void __launch_bounds__(256) k_tp_join_b(TpJoin j, BatchParams* bp) {
    __shared__ int go;
    if (threadIdx.x == 0) {
        bool ok = true;
        if (blockIdx.x == 0) {
            // the GEMM ended before this launch (stream order): no real wait
            ok = tp_wait(j.lar, j.lar_target);
            *j.lar = 0ull;
            for (int r = 0; r < j.tp; ++r) red_release_sys_add_u64(j.prarr[r] + j.inst, 1ull);
        }
        const bool failed = ld_volatile_u32(&bp->error) != 0u || ld_volatile_u32(j.abort) != 0u;
        if (ok && !failed) ok = tp_wait(j.rarr + j.inst, ((unsigned long long)bp->tpstep + 1ull) * (unsigned)j.tp);
        if (!ok) {
            atomicOr(&bp->error, 2u);
            for (int r = 0; r < j.tp; ++r) atomicExch_system(j.pabort[r], 1u);
        }
        go = ok && !failed && ld_volatile_u32(j.abort) == 0u;
    }
    __syncthreads();
    if (!go || !j.rx) return;
    const size_t n = (size_t)bp->n * j.E, slot = (size_t)MB_SEQ * j.E;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float acc = __ldcg(j.rx + i);
        for (int r = 1; r < j.tp; ++r) acc = __fadd_rn(acc, __ldcg(j.rx + r * slot + i));
        j.x[i] = __fadd_rn(j.x[i], acc);
    }
}

cudaError_t launch_tp_join_b(const TpJoin& j, BatchParams* bp, int grid, cudaStream_t s) {
    k_tp_join_b<<<grid, 256, 0, s>>>(j, bp);
    return cudaGetLastError();
}

}  // namespace talos
