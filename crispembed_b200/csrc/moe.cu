// moe.cu -- router, softmax, top-k, expert histogram + stable permutation,
// and the gate-weighted combine of the NomicBERT-MoE feed-forward block.
//
// Reference: the MoE branch of build_encoder_graph, src/crispembed.cpp:1327-1381:
//   logits = W_r x                      (ggml_mul_mat, :1333)
//   probs  = softmax(logits)            (ggml_soft_max, :1336)
//   ids    = top_k(probs, K)            (ggml_top_k, :1339)
//   w      = probs[ids]                 (ggml_get_rows, :1343-1345; not renormalised)
//   up     = gelu_erf(W1[ids] x)        (ggml_mul_mat_id + ggml_gelu_erf, :1365-1368)
//   down   = W2[ids] up                 (ggml_mul_mat_id, :1371)
//   y      = sum_k w_k down_k (+ bias)  (permute + ggml_mul_mat + ggml_add, :1375-1381)
//
// Device pipeline: route_rows_kernel (router, optionally fused with the
// residual + LayerNorm that produces its input) -> scan_kernel (one CTA)
// -> scatter_kernel (stable counting sort by expert, gathers fp16 rows) ->
// grouped GEMM fc1 (+GELU) -> grouped GEMM fc2 -> combine_kernel.  The expert
// row order is (expert, token, slot), the order ggml_mul_mat_id groups rows
// in, so the permutation is deterministic and identical across runs.
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <type_traits>
#include <vector>

#include "ceb_internal.h"
#include "ceb_ep_internal.h"
#include "ceb_moe_internal.h"
#include "common.cuh"
#include "rowwise.cuh"

namespace {

using ceb_row::LN_MAXV;

constexpr int CHUNK = 64;                            // tokens per histogram block
constexpr int RT_WARPS = 8;                          // warps per router CTA
constexpr int RT_TOK_PER_WARP = CHUNK / RT_WARPS;    // 8
constexpr int RT_GROUP = 4;                          // tokens a warp routes side by side (lane = token x 8)
#ifndef CEB_RT_MIN_BLOCKS
#define CEB_RT_MIN_BLOCKS 4                          // resident router CTAs per SM the register budget aims at
#endif
constexpr int RT_MIN_BLOCKS = CEB_RT_MIN_BLOCKS;
constexpr int MAXE = 64;
constexpr int MAXD = 128 * LN_MAXV;  // rows live in registers, 4 values per lane per 128 columns

template <typename T>
CEB_DEV float4 ld_act4(const T* p, size_t i);
template <>
CEB_DEV float4 ld_act4<float>(const float* p, size_t i) { return *reinterpret_cast<const float4*>(p + i); }
template <>
CEB_DEV float4 ld_act4<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
    const uint2 u = *reinterpret_cast<const uint2*>(p + i);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
template <>
CEB_DEV float4 ld_act4<__half>(const __half* p, size_t i) {
    const uint2 u = *reinterpret_cast<const uint2*>(p + i);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// ---------------------------------------------------------------------------
// Router.  Q8_0 router weights reproduce ggml's CPU arithmetic bit for bit:
// the token row is re-quantized to Q8_0 (amax/127 scale stored as fp16,
// multiplier 127/amax, round half to even), each 32-block contributes eight
// 4-product integer partial sums (dp4a), partial l accumulates
// fma(d_w*d_x, (float)isum_l, acc_l) over the blocks in order, and the eight
// partials are summed as ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)).  F32 router
// weights use a plain fp32 dot.
//
// Work layout: a CTA of RT_WARPS warps loops over histogram blocks of CHUNK
// tokens (persistent grid; the router weights are staged in shared memory
// once per CTA).  A warp takes RT_GROUP tokens at a time: it brings each row
// into registers (lane holds 4 values per 128 columns), quantizes it into
// shared memory, then lane (token tt = lane/8, expert e = lane%8 + 8j) computes
// all eight partial sums of its (token, expert) pairs from 16-byte shared
// loads, so the softmax and top-K of the RT_GROUP tokens run side by side in
// 8-lane groups.  The next row is prefetched into L2 while a row is processed.
// ---------------------------------------------------------------------------
constexpr int RT_MAXJ = 4;  // experts per lane: E <= 8 * RT_MAXJ

struct RouteSmem {
    int* cnt;     // [MAXE] expert histogram of the current block
    float* wd;    // [nb][E] router block scales
    float* xd;    // [warps][RT_GROUP][nb] activation block scales
    int8_t* wq;   // [E][d + 16] router quants (row pitch spreads 8 experts over the 32 banks)
    int8_t* xq;   // [warps][RT_GROUP][d] activation quants
    int nb, wpitch;
};

__host__ __device__ inline size_t route_smem_bytes(int d, int E) {
    const int nb = d / 32;
    return MAXE * 4 + (size_t)nb * E * 4 + (size_t)RT_WARPS * RT_GROUP * nb * 4 + (size_t)E * (d + 16) +
           (size_t)RT_WARPS * RT_GROUP * d;
}

CEB_DEV RouteSmem route_carve(uint8_t* sm, int d, int E) {
    RouteSmem s;
    s.nb = d / 32;
    s.wpitch = d + 16;
    s.cnt = reinterpret_cast<int*>(sm);
    s.wd = reinterpret_cast<float*>(sm + MAXE * 4);
    s.xd = s.wd + (size_t)s.nb * E;
    s.wq = reinterpret_cast<int8_t*>(s.xd + (size_t)RT_WARPS * RT_GROUP * s.nb);
    s.xq = s.wq + (size_t)E * s.wpitch;
    return s;
}

// Q8_0 router weights to shared memory: block (e, b) -> scale wd[b][e], quants
// wq[e][b*32 .. +31]; one thread per 4 quants (the 34-byte ggml blocks leave
// them 2-byte aligned).  Ends with __syncthreads().
CEB_DEV void route_stage(const RouteSmem& s, int E, int rtype, const uint8_t* __restrict__ rw) {
    if (rtype == CEB_GGML_Q8_0) {
        for (int i = threadIdx.x; i < E * s.nb * 8; i += blockDim.x) {
            const int blk_i = i >> 3, j = i & 7;
            const int e = blk_i / s.nb, b = blk_i - e * s.nb;
            const uint16_t* blk = reinterpret_cast<const uint16_t*>(rw + (size_t)blk_i * 34);
            if (j == 0) s.wd[b * E + e] = __half2float(__ushort_as_half(__ldg(blk)));
            const uint32_t q = (uint32_t)__ldg(blk + 1 + 2 * j) | ((uint32_t)__ldg(blk + 2 + 2 * j) << 16);
            *reinterpret_cast<uint32_t*>(s.wq + (size_t)e * s.wpitch + b * 32 + 4 * j) = q;
        }
    }
    __syncthreads();
}

CEB_DEV void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Row sources: where a token's row comes from before it is routed.
template <typename T, int NV>
struct ActRows {  // the activations, already in memory
    const T* x;
    CEB_DEV void prefetch(int t, int lane) const {
        constexpr int LINES = NV * 128 * (int)sizeof(T) / 128;
        const char* r = reinterpret_cast<const char*>(x + (size_t)t * NV * 128);
        for (int i = lane; i < LINES; i += 32) prefetch_l2(r + (size_t)i * 128);
    }
    CEB_DEV void row(int t, float4 (&v)[NV], int lane) const {
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = ld_act4<T>(x + (size_t)t * NV * 128, (size_t)(i * 32 + lane) * 4);
    }
};

template <int NV, typename TY>
struct AddLnRows {  // out = LN(res + y), stored, and routed from the registers
    const float* res;
    const TY* y;
    const float* gamma;
    const float* beta;
    float eps;
    float* out32;
    __half* out16;
    CEB_DEV void prefetch(int t, int lane) const {
        constexpr int LINES = NV * 4;                   // 128-byte lines per fp32 row
        constexpr int YLINES = LINES * sizeof(TY) / 4;  // and per y row
        for (int i = lane; i < LINES + YLINES; i += 32) {
            if (i < LINES) prefetch_l2(res + (size_t)t * NV * 128 + (size_t)i * 32);
            else prefetch_l2(y + (size_t)t * NV * 128 + (size_t)(i - LINES) * (128 / sizeof(TY)));
        }
    }
    CEB_DEV void row(int t, float4 (&v)[NV], int lane) const {
        constexpr int d = NV * 128;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const size_t c = (size_t)t * d + (i * 32 + lane) * 4;
            v[i] = ceb_row::f4add(*reinterpret_cast<const float4*>(res + c), ceb_row::ldg4(y + c));
        }
        ceb_row::ln_row(v, NV, d, gamma, beta, eps, out32 + (size_t)t * d, out16 ? out16 + (size_t)t * d : nullptr, lane);
    }
};

// Q8_0 quants and block scales of one row held in registers.  8 lanes hold one
// 32-value block, whose amax three xor-shuffles combine.
template <int NV>
CEB_DEV void quantize_row(const float4 (&v)[NV], int8_t* q, float* qd, int lane) {
#pragma unroll
    for (int seg = 0; seg < NV; ++seg) {
        const float4 x = v[seg];
        float am = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
        const float id = am != 0.0f ? 127.0f / am : 0.0f;
        const uint32_t b0 = (uint32_t)(__float2int_rn(x.x * id) & 0xFF);
        const uint32_t b1 = (uint32_t)(__float2int_rn(x.y * id) & 0xFF);
        const uint32_t b2 = (uint32_t)(__float2int_rn(x.z * id) & 0xFF);
        const uint32_t b3 = (uint32_t)(__float2int_rn(x.w * id) & 0xFF);
        reinterpret_cast<uint32_t*>(q)[seg * 32 + lane] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        if ((lane & 7) == 0) qd[seg * 4 + (lane >> 3)] = __half2float(__float2half_rn(am / 127.0f));
    }
}

// F32 router for two tokens of the group at once (tt0, tt0 + 1): every weight float4
// loaded feeds both rows, halving the L1 traffic of the router weights, which are
// re-read for every token.  Experts in passes of P (8 or 16): lane l's partial dot
// products over its columns, then a transposing butterfly leaves expert e0 + (l % P)
// of the pass on lane l.  Logits differ from the one-token form only in the order of
// the cross-lane fp32 sums.
template <int NV, int P>
CEB_DEV void f32_logits_pair(const float4 (&v0)[NV], const float4 (&v1)[NV], const float* __restrict__ wf, int E,
                             int lane, int tt0, float (&lgv)[RT_MAXJ]) {
    constexpr int d = NV * 128;
    const int tt_l = lane >> 3, el = lane & 7;
    for (int e0 = 0; e0 < E; e0 += P) {
        float a0[P], a1[P];
#pragma unroll
        for (int e = 0; e < P; ++e) {
            float s0 = 0.0f, s1 = 0.0f;
            if (e0 + e < E) {
                const float* wr = wf + (size_t)(e0 + e) * d;
#pragma unroll
                for (int i = 0; i < NV; ++i) {
                    const float4 w = __ldg(reinterpret_cast<const float4*>(wr + (i * 32 + lane) * 4));
                    s0 = __fmaf_rn(v0[i].x, w.x, s0);
                    s0 = __fmaf_rn(v0[i].y, w.y, s0);
                    s0 = __fmaf_rn(v0[i].z, w.z, s0);
                    s0 = __fmaf_rn(v0[i].w, w.w, s0);
                    s1 = __fmaf_rn(v1[i].x, w.x, s1);
                    s1 = __fmaf_rn(v1[i].y, w.y, s1);
                    s1 = __fmaf_rn(v1[i].z, w.z, s1);
                    s1 = __fmaf_rn(v1[i].w, w.w, s1);
                }
            }
            a0[e] = s0;
            a1[e] = s1;
        }
#pragma unroll
        for (int o = P / 2; o >= 1; o >>= 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < o; ++i) {
                const float snd0 = up ? a0[i] : a0[i + o], kp0 = up ? a0[i + o] : a0[i];
                const float snd1 = up ? a1[i] : a1[i + o], kp1 = up ? a1[i + o] : a1[i];
                a0[i] = __fadd_rn(kp0, __shfl_xor_sync(0xffffffffu, snd0, o));
                a1[i] = __fadd_rn(kp1, __shfl_xor_sync(0xffffffffu, snd1, o));
            }
        }
#pragma unroll
        for (int o = P; o < 32; o <<= 1) {
            a0[0] = __fadd_rn(a0[0], __shfl_xor_sync(0xffffffffu, a0[0], o));
            a1[0] = __fadd_rn(a1[0], __shfl_xor_sync(0xffffffffu, a1[0], o));
        }
#pragma unroll
        for (int jj = 0; jj < P / 8; ++jj) {
            const float r0 = __shfl_sync(0xffffffffu, a0[0], el + 8 * jj);
            const float r1 = __shfl_sync(0xffffffffu, a1[0], el + 8 * jj);
            const int j = e0 / 8 + jj;
#pragma unroll
            for (int q = 0; q < RT_MAXJ; ++q)
                if (q == j) {
                    if (tt_l == tt0) lgv[q] = r0;
                    if (tt_l == tt0 + 1) lgv[q] = r1;
                }
        }
    }
}

// Q8_0 router: lane (tt, el) computes the logits of experts el + 8j for token
// tt of the group from the quantized row in shared memory.
template <int NV>
CEB_DEV void q8_logits(const RouteSmem& s, const int8_t* xrow, const float* xd, int E, int el,
                       float (&lgv)[RT_MAXJ]) {
    constexpr int nb = NV * 4;
#pragma unroll
    for (int j = 0; j < RT_MAXJ; ++j) {
        const int e = el + 8 * j;
        if (e >= E) break;
        const int8_t* wrow = s.wq + (size_t)e * s.wpitch;
        float a[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) a[l] = 0.0f;
#pragma unroll 2
        for (int b = 0; b < nb; ++b) {
            const int4 w0 = *reinterpret_cast<const int4*>(wrow + b * 32);
            const int4 w1 = *reinterpret_cast<const int4*>(wrow + b * 32 + 16);
            const int4 x0 = *reinterpret_cast<const int4*>(xrow + b * 32);
            const int4 x1 = *reinterpret_cast<const int4*>(xrow + b * 32 + 16);
            const float sc = __fmul_rn(s.wd[b * E + e], xd[b]);
            a[0] = __fmaf_rn(sc, (float)__dp4a(w0.x, x0.x, 0), a[0]);
            a[1] = __fmaf_rn(sc, (float)__dp4a(w0.y, x0.y, 0), a[1]);
            a[2] = __fmaf_rn(sc, (float)__dp4a(w0.z, x0.z, 0), a[2]);
            a[3] = __fmaf_rn(sc, (float)__dp4a(w0.w, x0.w, 0), a[3]);
            a[4] = __fmaf_rn(sc, (float)__dp4a(w1.x, x1.x, 0), a[4]);
            a[5] = __fmaf_rn(sc, (float)__dp4a(w1.y, x1.y, 0), a[5]);
            a[6] = __fmaf_rn(sc, (float)__dp4a(w1.z, x1.z, 0), a[6]);
            a[7] = __fmaf_rn(sc, (float)__dp4a(w1.w, x1.w, 0), a[7]);
        }
        lgv[j] = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[2], a[6])),
                           __fadd_rn(__fadd_rn(a[1], a[5]), __fadd_rn(a[3], a[7])));
    }
}

// Softmax over the E logits of each 8-lane group's token, then top-K by repeated
// argmax (ties to the lower expert index); weights are the probabilities, not
// renormalised.  All lanes take part (shuffles); `valid` gates the stores.
CEB_DEV void group_route(const float (&lgv)[RT_MAXJ], int E, int K, bool valid, size_t t, int el,
                         int32_t* __restrict__ ids, float* __restrict__ wts, float* __restrict__ logits_out,
                         int* cnt) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < RT_MAXJ; ++j)
        if (el + 8 * j < E) mx = fmaxf(mx, lgv[j]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    float ex[RT_MAXJ];
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < RT_MAXJ; ++j) {
        ex[j] = el + 8 * j < E ? expf(lgv[j] - mx) : 0.0f;
        sum += ex[j];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    const float inv = (float)(1.0 / sum);
    if (logits_out && valid) {
#pragma unroll
        for (int j = 0; j < RT_MAXJ; ++j)
            if (el + 8 * j < E) logits_out[t * E + el + 8 * j] = lgv[j];
    }
    unsigned taken = 0;
    for (int k = 0; k < K; ++k) {
        float bv = -2.0f;
        int bi = 1 << 20;
#pragma unroll
        for (int j = 0; j < RT_MAXJ; ++j) {
            const float p = ex[j] * inv;
            if (el + 8 * j < E && !((taken >> j) & 1u) && p > bv) {
                bv = p;
                bi = el + 8 * j;
            }
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 7) == el) taken |= 1u << (bi >> 3);
        if (el == 0 && valid) {
            ids[t * K + k] = bi;
            wts[t * K + k] = bv;
            atomicAdd(&cnt[bi], 1);
        }
    }
}

// The router over histogram blocks [blockIdx.x, nblk) step gridDim.x; rows come
// from `rows` (activations in memory, or the fused residual + LayerNorm).
// Q8 = true: Q8_0 router weights; false: F32, two tokens' rows and partial sums in
// registers at once (hence the register budget of two CTAs per SM).
template <int NV, bool Q8, class Rows>
__global__ void __launch_bounds__(RT_WARPS * 32, Q8 ? RT_MIN_BLOCKS : 2)
    route_rows_kernel(Rows rows, int T_tokens, int nblk, int E, int K, const uint8_t* __restrict__ rw,
                      int32_t* __restrict__ ids, float* __restrict__ wts, float* __restrict__ logits_out,
                      int32_t* __restrict__ block_counts) {
    extern __shared__ __align__(16) uint8_t sm[];
    constexpr int d = NV * 128;
    const RouteSmem s = route_carve(sm, d, E);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tt_l = lane >> 3, el = lane & 7;
    route_stage(s, E, Q8 ? CEB_GGML_Q8_0 : CEB_GGML_F32, rw);
    int8_t* xq = s.xq + (size_t)warp * RT_GROUP * d;
    float* xd = s.xd + (size_t)warp * RT_GROUP * s.nb;
    for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        for (int i = threadIdx.x; i < E; i += blockDim.x) s.cnt[i] = 0;
        __syncthreads();
        const int t_base = blk * CHUNK + warp * RT_TOK_PER_WARP;
        if (t_base < T_tokens) rows.prefetch(t_base, lane);
        for (int g = 0; g < RT_TOK_PER_WARP; g += RT_GROUP) {
            float lgv[RT_MAXJ];
#pragma unroll
            for (int j = 0; j < RT_MAXJ; ++j) lgv[j] = -INFINITY;
            if constexpr (Q8) {
                for (int tt = 0; tt < RT_GROUP; ++tt) {
                    const int t = t_base + g + tt;
                    if (t >= T_tokens) break;
                    if (g + tt + 1 < RT_TOK_PER_WARP && t + 1 < T_tokens) rows.prefetch(t + 1, lane);
                    float4 v[NV];
                    rows.row(t, v, lane);
                    quantize_row<NV>(v, xq + (size_t)tt * d, xd + tt * s.nb, lane);
                }
            } else {
                static_assert(RT_GROUP % 2 == 0, "tokens are routed in pairs");
                for (int tt = 0; tt < RT_GROUP; tt += 2) {
                    const int t = t_base + g + tt;
                    if (t >= T_tokens) break;
                    for (int n = 2; n < 4; ++n)
                        if (g + tt + n < RT_TOK_PER_WARP && t + n < T_tokens) rows.prefetch(t + n, lane);
                    float4 v0[NV], v1[NV];
                    rows.row(t, v0, lane);
                    if (t + 1 < T_tokens) {
                        rows.row(t + 1, v1, lane);
                    } else {
#pragma unroll
                        for (int i = 0; i < NV; ++i) v1[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    if (E > 8)
                        f32_logits_pair<NV, 16>(v0, v1, reinterpret_cast<const float*>(rw), E, lane, tt, lgv);
                    else
                        f32_logits_pair<NV, 8>(v0, v1, reinterpret_cast<const float*>(rw), E, lane, tt, lgv);
                }
            }
            __syncwarp();
            const int t_mine = t_base + g + tt_l;
            const bool valid = t_mine < T_tokens;
            if (Q8 && valid) q8_logits<NV>(s, xq + (size_t)tt_l * d, xd + tt_l * s.nb, E, el, lgv);
            __syncwarp();
            group_route(lgv, E, K, valid, (size_t)t_mine, el, ids, wts, logits_out, s.cnt);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < E; i += blockDim.x) block_counts[(size_t)blk * E + i] = s.cnt[i];
        __syncthreads();
    }
}

// F32 router over activations in memory, for 8 < E <= 32 (the wide-routing shape E = 32,
// d = 1024): the router product as a register-blocked SIMT GEMM.  A CTA of 8 warps keeps
// the router rows in shared memory ([E][d + 4] fp32); each warp takes 64-token histogram
// blocks in turn (one block = one warp's tile), staged in k-chunks as fp32 in its shared
// tile while the next chunk's loads are in flight.  Lane (tg, eg) = (lane / 4, lane % 4)
// computes tokens tg + 8i (i < 8) x experts eg + 4j (j < 8): per 4 k, 8 + 8 sixteen-byte
// shared reads (strided rows: no bank conflicts) feed 256 FMAs.  Each logit is summed in
// k order.  Softmax, top-K and counts as in route_rows_kernel (group_route, 4 tokens per
// pass from the logits transposed through shared memory).
constexpr int RF_WARPS = 8, RF_TOK = 64, RF_XLD_PAD = 4, RF_LLD = 33;
static_assert(RF_TOK == CHUNK, "one warp's token tile is one histogram block");
template <typename T>
__host__ __device__ constexpr int rf_kc() { return sizeof(T) == 4 ? 16 : 32; }  // k per chunk: 8 sixteen-byte pieces per lane
template <typename T>
__host__ __device__ constexpr int rf_xld() { return rf_kc<T>() + RF_XLD_PAD; }
template <typename T>
inline size_t route_f32_smem_bytes(int d, int E) {
    const size_t tile = (size_t)RF_TOK * (rf_xld<T>() > RF_LLD ? rf_xld<T>() : RF_LLD) * 4;
    return (size_t)E * (d + 4) * 4 + (size_t)RF_WARPS * tile + (size_t)RF_WARPS * MAXE * 4;
}

template <typename T>
CEB_DEV void rf_cvt8(uint4 raw, float (&f)[8]);
template <>
CEB_DEV void rf_cvt8<__nv_bfloat16>(uint4 raw, float (&f)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
template <>
CEB_DEV void rf_cvt8<__half>(uint4 raw, float (&f)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

// One warp's RF_TOK token rows x KC columns as raw 16-byte pieces: lane l holds pieces
// l, l + 32, ... of the (row, piece) grid (rows past T are zero).
template <typename T>
struct RfStage {
    static constexpr int KC = rf_kc<T>(), XLD = rf_xld<T>();
    static constexpr int PIECE = 16 / (int)sizeof(T);  // elements per 16-byte piece
    static constexpr int PER_ROW = KC / PIECE;         // pieces per row
    static constexpr int N = RF_TOK * PER_ROW / 32;    // pieces per lane
    uint4 raw[N];
    CEB_DEV void load(const T* __restrict__ x, int d, int t0, int T_tokens, int k0, int lane) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int p = lane + 32 * i, r = p / PER_ROW, c = (p % PER_ROW) * PIECE;
            raw[i] = t0 + r < T_tokens ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + r) * d + k0 + c))
                                       : make_uint4(0u, 0u, 0u, 0u);
        }
    }
    CEB_DEV void store(float* xs, int lane) const {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int p = lane + 32 * i, r = p / PER_ROW, c = (p % PER_ROW) * PIECE;
            float* dst = xs + r * XLD + c;
            if constexpr (sizeof(T) == 4) {
                *reinterpret_cast<uint4*>(dst) = raw[i];
            } else {
                float f[8];
                rf_cvt8<T>(raw[i], f);
                *reinterpret_cast<float4*>(dst) = make_float4(f[0], f[1], f[2], f[3]);
                *reinterpret_cast<float4*>(dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
            }
        }
    }
};

template <typename T>
__global__ void __launch_bounds__(RF_WARPS * 32, 1)
    route_f32_tile_kernel(const T* __restrict__ x, int T_tokens, int d, int nblk, int E, int K,
                          const float* __restrict__ rw, int32_t* __restrict__ ids, float* __restrict__ wts,
                          float* __restrict__ logits_out, int32_t* __restrict__ block_counts) {
    constexpr int KC = rf_kc<T>(), XLD = rf_xld<T>();
    constexpr int TILE = RF_TOK * (XLD > RF_LLD ? XLD : RF_LLD);
    extern __shared__ __align__(16) uint8_t sm[];
    float* wT = reinterpret_cast<float*>(sm);            // [E][d + 4]
    float* xs_all = wT + (size_t)E * (d + 4);            // [warps][TILE]
    int* cnt = reinterpret_cast<int*>(xs_all + RF_WARPS * TILE);  // [8][MAXE]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tg = lane >> 2, eg = lane & 3;
    for (int i = threadIdx.x; i < E * d / 4; i += blockDim.x) {
        const int e = (i * 4) / d, k = i * 4 - e * d;
        *reinterpret_cast<float4*>(wT + (size_t)e * (d + 4) + k) = __ldg(reinterpret_cast<const float4*>(rw) + i);
    }
    float* xs = xs_all + warp * TILE;
    int* wcnt = cnt + warp * MAXE;  // this warp's histogram block
    __syncthreads();                // the router rows are staged
    // Warp-major order: histogram block b goes to warp b / gridDim.x % RF_WARPS of CTA
    // b % gridDim.x, so a partial last round spreads over every SM (each gets its share
    // of blocks to within one) instead of leaving whole CTAs idle.
    for (int b = warp * gridDim.x + blockIdx.x; b < nblk; b += gridDim.x * RF_WARPS) {
        for (int i = lane; i < MAXE; i += 32) wcnt[i] = 0;
        __syncwarp();
        const int t0 = b * RF_TOK;
        float acc[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
        RfStage<T> st;
        st.load(x, d, t0, T_tokens, 0, lane);
        for (int k0 = 0; k0 < d; k0 += KC) {
            __syncwarp();
            st.store(xs, lane);
            __syncwarp();
            if (k0 + KC < d) st.load(x, d, t0, T_tokens, k0 + KC, lane);
#pragma unroll
            for (int kk = 0; kk < KC; kk += 4) {
                float4 xv[8], wv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) xv[i] = *reinterpret_cast<const float4*>(xs + (tg + 8 * i) * XLD + kk);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int e = eg + 4 * j < E ? eg + 4 * j : 0;
                    wv[j] = *reinterpret_cast<const float4*>(wT + (size_t)e * (d + 4) + k0 + kk);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        acc[i][j] = fmaf(xv[i].x, wv[j].x, acc[i][j]);
                        acc[i][j] = fmaf(xv[i].y, wv[j].y, acc[i][j]);
                        acc[i][j] = fmaf(xv[i].z, wv[j].z, acc[i][j]);
                        acc[i][j] = fmaf(xv[i].w, wv[j].w, acc[i][j]);
                    }
            }
        }
        // logits [token][expert] through the warp's tile, then 4 tokens per routing pass
        __syncwarp();
        float* lg = xs;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) lg[(tg + 8 * i) * RF_LLD + eg + 4 * j] = acc[i][j];
        __syncwarp();
        const int tt_l = lane >> 3, el = lane & 7;
        for (int g = 0; g < RF_TOK; g += RT_GROUP) {
            const int tl = g + tt_l;
            float lgv[RT_MAXJ];
#pragma unroll
            for (int j = 0; j < RT_MAXJ; ++j) lgv[j] = el + 8 * j < E ? lg[tl * RF_LLD + el + 8 * j] : -INFINITY;
            const int t = t0 + tl;
            group_route(lgv, E, K, t < T_tokens, (size_t)t, el, ids, wts, logits_out, wcnt);
        }
        __syncwarp();
        for (int e = lane; e < E; e += 32) block_counts[(size_t)b * E + e] = wcnt[e];
        __syncwarp();  // read before the next block clears it
    }
}

// Expert offsets (exclusive scan of the totals) and, per histogram block, the
// first output row of each expert.  Warp w owns a run of consecutive histogram
// blocks and lane l the experts l, l + 32, ...: every load and store of a block's
// counts is one coalesced row, the warps' per-expert sums are scanned across warps
// in shared memory, and a second pass over the same rows writes the bases.
// Expert-parallel runs also publish the totals: row `rank` of every peer's count
// matrix, then a release of the peer's counts flag.
constexpr int SCAN_WARPS = 32;
__global__ void __launch_bounds__(SCAN_WARPS * 32) scan_kernel(const int32_t* __restrict__ block_counts, int nblk,
                                                               int E, int32_t* __restrict__ block_base,
                                                               int32_t* __restrict__ offsets,
                                                               int32_t* __restrict__ expert_counts, ceb_ep_args ep) {
    __shared__ int wbase[SCAN_WARPS][MAXE];  // per warp and expert: sum, then the warp's first row
    __shared__ int tot[MAXE];
    __shared__ int ebase[MAXE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (nblk + SCAN_WARPS - 1) / SCAN_WARPS;
    const int b0 = min(nblk, warp * per), b1 = min(nblk, b0 + per);
    for (int e = lane; e < E; e += 32) {
        int sum = 0;
#pragma unroll 4
        for (int b = b0; b < b1; ++b) sum += block_counts[(size_t)b * E + e];
        wbase[warp][e] = sum;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < SCAN_WARPS; ++w) {
            const int v = wbase[w][e];
            wbase[w][e] = run;
            run += v;
        }
        tot[e] = run;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int base = 0;
        offsets[0] = 0;
        for (int e = 0; e < E; ++e) {
            ebase[e] = base;
            base += tot[e];
            offsets[e + 1] = base;
        }
    }
    __syncthreads();
    if (expert_counts)
        for (int e = threadIdx.x; e < E; e += blockDim.x) expert_counts[e] = tot[e];
    for (int e = lane; e < E; e += 32) {
        int run = ebase[e] + wbase[warp][e];
#pragma unroll 4
        for (int b = b0; b < b1; ++b) {
            block_base[(size_t)b * E + e] = run;
            run += block_counts[(size_t)b * E + e];
        }
    }
    if (ep.peers) {
        for (int i = threadIdx.x; i < ep.world * E; i += blockDim.x) {
            const int p = i / E, e = i - p * E;
            ep.peers[p].counts[((size_t)ep.par * ep.world + ep.rank) * E + e] = tot[e];
        }
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x < ep.world)
            st_release_sys(ep.peers[threadIdx.x].flags + CEB_EPF_COUNTS * ep.world + ep.rank, ep.epoch);
    }
}

// Stable placement of every (token, slot) into its expert's row range, then a
// gather of the token rows (converted to fp16) into the permuted activation
// matrix consumed by fc1: one warp per token reads the row once and writes it
// to each of the token's K rows.
//
// Expert-parallel runs (ep.peers set) write each row straight into the receive
// buffer of the rank owning its expert, at (the expert's rows from lower ranks
// and lower local experts of that owner) + (the row's rank within this rank's
// rows of the expert); the last CTA to finish releases every peer's dispatch
// flag.  CTA 0 also derives the row ranges of the local experts in the local
// receive buffer for the expert GEMMs.
template <typename T>
__global__ void __launch_bounds__(256)
    scatter_kernel(const T* __restrict__ x, const __half* __restrict__ x16, int T_tokens, int d, int E, int K,
                   const int32_t* __restrict__ ids, const int32_t* __restrict__ block_base,
                   int32_t* __restrict__ slot_pos, __half* __restrict__ x_perm, int* __restrict__ err,
                   ceb_ep_args ep) {
    __shared__ int running[MAXE];
    __shared__ int s_pos[CHUNK * 4];
    __shared__ int s_key[CHUNK * 4];
    __shared__ long long s_dst[MAXE];  // EP: destination row of local position 0 of each expert
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * CHUNK;
    const int n_tok = min(CHUNK, T_tokens - t0);
    const int n_slots = n_tok * K;
    if (ep.peers && threadIdx.x >= 32 && threadIdx.x < 32 + E) {
        const int e = threadIdx.x - 32, q = e / ep.E_loc;
        long long base = 0;
        for (int e2 = q * ep.E_loc; e2 < e; ++e2)
            for (int p = 0; p < ep.world; ++p) base += ep.C[p * E + e2];
        for (int p = 0; p < ep.rank; ++p) base += ep.C[p * E + e];
        s_dst[e] = base - ep.my_offsets[e];
    }
    if (ep.peers && blockIdx.x == 0) {  // first row of each local expert in the local receive buffer
        for (int el = threadIdx.x; el <= ep.E_loc; el += blockDim.x) {
            long long r = 0;
            for (int e2 = 0; e2 < el; ++e2)
                for (int p = 0; p < ep.world; ++p) r += ep.C[p * E + ep.rank * ep.E_loc + e2];
            ep.offsets_recv[el] = (int32_t)r;
        }
    }
    if (warp == 0) {
        for (int e = lane; e < E; e += 32) running[e] = block_base[(size_t)blockIdx.x * E + e];
        __syncwarp();
        for (int s0 = 0; s0 < n_slots; s0 += 32) {
            const int s = s0 + lane;
            const bool act = s < n_slots;
            const int key = act ? ids[(size_t)t0 * K + s] : -1 - lane;  // inactive lanes never match
            const unsigned peers = __match_any_sync(0xffffffffu, key);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            int pos = 0;
            if (act) {
                if (key < 0 || key >= E) {
                    pos = -1;
                } else {
                    pos = running[key] + rank;
                }
            }
            __syncwarp();
            if (act && key >= 0 && key < E && rank == 0) running[key] += __popc(peers);
            __syncwarp();
            if (act) {
                s_pos[s] = pos;
                s_key[s] = key;
                slot_pos[(size_t)t0 * K + s] = pos;
            }
        }
    }
    __syncthreads();
    const int nv = d / 128;
    if (x16) {  // fp16 rows: 16-byte chunks, chunk i*32 + lane of a row per lane
        const int nc = d / 8;
        for (int tl = warp; tl < n_tok; tl += blockDim.x / 32) {
            const uint4* src = reinterpret_cast<const uint4*>(x16 + (size_t)(t0 + tl) * d);
            uint4 r[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (i * 32 + lane < nc) r[i] = __ldg(src + i * 32 + lane);
            for (int j = 0; j < K; ++j) {
                const int pos = s_pos[tl * K + j];
                if (pos < 0) continue;
                __half* dst;
                if (ep.peers) {
                    const int e = s_key[tl * K + j];
                    const long long row = s_dst[e] + pos;
                    if (row < 0 || row >= ep.recv_rows) {
                        if (lane == 0) atomicCAS(err, 0, (int)CEB_DEVERR_EP_OVERFLOW);
                        continue;
                    }
                    dst = ep.peers[e / ep.E_loc].recv + (size_t)row * d;
                } else {
                    dst = x_perm + (size_t)pos * d;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (i * 32 + lane < nc) reinterpret_cast<uint4*>(dst)[i * 32 + lane] = r[i];
            }
        }
    }
    for (int tl = warp; tl < n_tok && !x16; tl += blockDim.x / 32) {
        const size_t t = (size_t)(t0 + tl);
        uint2 r[LN_MAXV];  // 4 fp16 values per lane per 128-column segment
#pragma unroll
        for (int i = 0; i < LN_MAXV; ++i)
            if (i < nv) {
                const size_t c = (size_t)(i * 32 + lane) * 4;
                const float4 f = ld_act4<T>(x + t * d, c);
                const __half2 lo = __floats2half2_rn(f.x, f.y), hi = __floats2half2_rn(f.z, f.w);
                r[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
            }
        for (int j = 0; j < K; ++j) {
            const int pos = s_pos[tl * K + j];
            if (pos < 0) continue;
            __half* dst;
            if (ep.peers) {
                const int e = s_key[tl * K + j];
                const long long row = s_dst[e] + pos;
                if (row < 0 || row >= ep.recv_rows) {
                    if (lane == 0) atomicCAS(err, 0, (int)CEB_DEVERR_EP_OVERFLOW);
                    continue;
                }
                dst = ep.peers[e / ep.E_loc].recv + (size_t)row * d;
            } else {
                dst = x_perm + (size_t)pos * d;
            }
#pragma unroll
            for (int i = 0; i < LN_MAXV; ++i)
                if (i < nv) *reinterpret_cast<uint2*>(dst + (i * 32 + lane) * 4) = r[i];
        }
    }
    if (ep.peers) {  // the last CTA to finish tells every peer that this rank's rows have landed
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) {
            if (atomicAdd(ep.done, 1) == (int)gridDim.x - 1) {
                atomicExch(ep.done, 0);
                __threadfence_system();
                for (int p = 0; p < ep.world; ++p)
                    st_release_sys(ep.peers[p].flags + CEB_EPF_DISPATCH * ep.world + ep.rank, ep.epoch);
            }
        }
    }
}

// y[t, c] = sum_j w[t,j] * down[pos(t,j), c] (fmaf in slot order) + bias[c]
__global__ void combine_kernel(const __half* __restrict__ down, const int32_t* __restrict__ slot_pos,
                               const float* __restrict__ wts, int T_tokens, int d, int K, const float* __restrict__ bias,
                               float* __restrict__ y) {
    const int t = blockIdx.x;
    if (t >= T_tokens) return;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        float s = 0.0f;
        for (int j = 0; j < K; ++j) {
            const int pos = slot_pos[(size_t)t * K + j];
            s = __fmaf_rn(wts[(size_t)t * K + j], __half2float(down[(size_t)pos * d + c]), s);
        }
        y[(size_t)t * d + c] = bias ? __fadd_rn(s, bias[c]) : s;
    }
}

#ifndef CEB_COMBINE_ROWS
#define CEB_COMBINE_ROWS 1
#endif
// Same sums as combine_kernel, one warp per token with NV float4 columns per lane:
// the rows of two slots are requested whole before their FMAs (accumulated in slot
// order), so two expert rows of every token are in flight.
template <int NV>
__global__ void __launch_bounds__(128) combine_rows_kernel(const __half* __restrict__ down,
                                                           const int32_t* __restrict__ slot_pos,
                                                           const float* __restrict__ wts, int T_tokens, int K,
                                                           const float* __restrict__ bias, float* __restrict__ y) {
    constexpr int d = NV * 128;
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= T_tokens) return;
    float4 acc[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    int j = 0;
    for (; j + 1 < K; j += 2) {
        const int p0 = slot_pos[(size_t)t * K + j], p1 = slot_pos[(size_t)t * K + j + 1];
        const float w0 = wts[(size_t)t * K + j], w1 = wts[(size_t)t * K + j + 1];
        float4 r0[NV], r1[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = (i * 32 + lane) * 4;
            r0[i] = ceb_row::ldg4(down + (size_t)p0 * d + c);
            r1[i] = ceb_row::ldg4(down + (size_t)p1 * d + c);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            acc[i].x = __fmaf_rn(w1, r1[i].x, __fmaf_rn(w0, r0[i].x, acc[i].x));
            acc[i].y = __fmaf_rn(w1, r1[i].y, __fmaf_rn(w0, r0[i].y, acc[i].y));
            acc[i].z = __fmaf_rn(w1, r1[i].z, __fmaf_rn(w0, r0[i].z, acc[i].z));
            acc[i].w = __fmaf_rn(w1, r1[i].w, __fmaf_rn(w0, r0[i].w, acc[i].w));
        }
    }
    for (; j < K; ++j) {
        const int p = slot_pos[(size_t)t * K + j];
        const float w = wts[(size_t)t * K + j];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float4 r = ceb_row::ldg4(down + (size_t)p * d + (i * 32 + lane) * 4);
            acc[i].x = __fmaf_rn(w, r.x, acc[i].x);
            acc[i].y = __fmaf_rn(w, r.y, acc[i].y);
            acc[i].z = __fmaf_rn(w, r.z, acc[i].z);
            acc[i].w = __fmaf_rn(w, r.w, acc[i].w);
        }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = (i * 32 + lane) * 4;
        float4 o = acc[i];
        if (bias) {
            const float4 b = *reinterpret_cast<const float4*>(bias + c);
            o = make_float4(__fadd_rn(o.x, b.x), __fadd_rn(o.y, b.y), __fadd_rn(o.z, b.z), __fadd_rn(o.w, b.w));
        }
        *reinterpret_cast<float4*>(y + (size_t)t * d + c) = o;
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

size_t ceb_moe_ws_layout(int T, int d, int E, int K, int F, ceb_moe_ws* ws, uint8_t* base) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += (bytes + 255) & ~size_t(255);
        return base ? base + o : nullptr;
    };
    const int nblk = (T + CHUNK - 1) / CHUNK;
    const size_t S = (size_t)T * K;
    ceb_moe_ws w;
    w.ids = (int32_t*)take(S * 4);
    w.wts = (float*)take(S * 4);
    w.block_counts = (int32_t*)take((size_t)nblk * E * 4);
    w.block_base = (int32_t*)take((size_t)nblk * E * 4);
    w.offsets = (int32_t*)take((size_t)(E + 1) * 4);
    w.slot_pos = (int32_t*)take(S * 4);
    w.x_perm = (__half*)take(S * d * 2);
    w.h_perm = (__half*)take(S * F * 2);
    w.down = (__half*)take(S * d * 2);
    if (ws) *ws = w;
    return off;
}

namespace {

int moe_shape_check(const ceb_moe_weights& mw) {
    const int d = mw.d, E = mw.n_experts, K = mw.top_k, F = mw.ffn;
    if (E > 32 || E < 1 || K < 1 || K > E || K > 4 || d > MAXD || F % 128 || d % 128)
        return ceb_set_error(2, "moe: unsupported shape d=%d E=%d K=%d F=%d", d, E, K, F);
    return 0;
}

// One launch of route_rows_kernel: a persistent grid of (resident CTAs per SM) x SMs.
template <int NV, bool Q8, class Rows>
int launch_route_rows_t(const Rows& rows, int T, int E, int K, const uint8_t* rw, const ceb_moe_ws& ws,
                        float* logits_out, cudaStream_t st) {
    auto kern = route_rows_kernel<NV, Q8, Rows>;
    const size_t smem = route_smem_bytes(NV * 128, E);
    static int occ_of[CEB_MAX_DEVICES] = {};  // resident CTAs per SM, per device
    static size_t smem_of[CEB_MAX_DEVICES] = {};
    const int dev = ceb_device_index();
    if (!occ_of[dev] || smem_of[dev] != smem) {
        if (int rc = ceb_func_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
        int n = 0;
        CEB_CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, RT_WARPS * 32, smem));
        occ_of[dev] = std::max(n, 1);
        smem_of[dev] = smem;
    }
    const int occ = occ_of[dev];
    const int nblk = (T + CHUNK - 1) / CHUNK;
    const int grid = std::min(nblk, occ * ceb_num_sms());
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0,
               kern<<<grid, RT_WARPS * 32, smem, st>>>(rows, T, nblk, E, K, rw, ws.ids, ws.wts, logits_out,
                                                       ws.block_counts));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

template <class Rows>
struct ActRowsType {
    using type = void;
};
template <typename T, int NV>
struct ActRowsType<ActRows<T, NV>> {
    using type = T;
};

// The tiled F32 router (route_f32_tile_kernel) for activations in memory; 1 when the shape
// is not its own (nothing launched).
template <typename T>
int launch_route_f32_tile(const T* x, int T_tokens, int d, int E, int K, const float* rw, const ceb_moe_ws& ws,
                          float* logits_out, cudaStream_t st) {
    const size_t smem = route_f32_smem_bytes<T>(d, E);
    if (E <= 8 || E > 8 * RT_MAXJ || d % rf_kc<T>() || smem > 220 * 1024) return 1;
    auto kern = route_f32_tile_kernel<T>;
    if (int rc = ceb_func_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
    const int nblk = (T_tokens + CHUNK - 1) / CHUNK;
    const int grid = std::min((nblk + RF_WARPS - 1) / RF_WARPS, ceb_num_sms());
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0,
               kern<<<grid, RF_WARPS * 32, smem, st>>>(x, T_tokens, d, nblk, E, K, rw, ws.ids, ws.wts, logits_out,
                                                       ws.block_counts));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

template <int NV, class Rows>
int launch_route_rows(const Rows& rows, int T, int E, int K, int rtype, const uint8_t* rw, const ceb_moe_ws& ws,
                      float* logits_out, cudaStream_t st) {
    if (rtype == CEB_GGML_Q8_0) return launch_route_rows_t<NV, true>(rows, T, E, K, rw, ws, logits_out, st);
    using AT = typename ActRowsType<Rows>::type;
    if constexpr (!std::is_void<AT>::value) {
        if (T > 0) {
            const int rc = launch_route_f32_tile<AT>(rows.x, T, NV * 128, E, K, reinterpret_cast<const float*>(rw), ws,
                                                     logits_out, st);
            if (rc != 1) return rc;
        }
    }
    return launch_route_rows_t<NV, false>(rows, T, E, K, rw, ws, logits_out, st);
}

// Calls f(std::integral_constant<int, d / 128>) for the supported widths.
template <class F>
int with_nv(int d, F&& f) {
    switch (d / 128) {
        case 1: return f(std::integral_constant<int, 1>{});
        case 2: return f(std::integral_constant<int, 2>{});
        case 3: return f(std::integral_constant<int, 3>{});
        case 4: return f(std::integral_constant<int, 4>{});
        case 5: return f(std::integral_constant<int, 5>{});
        case 6: return f(std::integral_constant<int, 6>{});
        case 7: return f(std::integral_constant<int, 7>{});
        case 8: return f(std::integral_constant<int, 8>{});
        default: return ceb_set_error(2, "moe: d=%d unsupported", d);
    }
}

// combine of T tokens' K expert rows (fp16) into y [T, d] (fp32)
int launch_combine(const __half* down, const int32_t* slot_pos, const float* wts, int T, int d, int K,
                   const float* bias, float* y, cudaStream_t st) {
    const bool vec = CEB_COMBINE_ROWS && d % 128 == 0 && d <= 1024 &&
                     ((reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(down) |
                       reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (!vec) {
        CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0, combine_kernel<<<T, 256, 0, st>>>(down, slot_pos, wts, T, d, K, bias, y));
        CEB_CUDA_OK(cudaGetLastError());
        return 0;
    }
    const int grid = (T + 3) / 4;
    return with_nv(d, [&](auto nvc) {
        constexpr int NV = decltype(nvc)::value;
        CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
                   combine_rows_kernel<NV><<<grid, 128, 0, st>>>(down, slot_pos, wts, T, K, bias, y));
        CEB_CUDA_OK(cudaGetLastError());
        return 0;
    });
}


}  // namespace

int ceb_add_ln_route(const float* res, const void* y, bool y_f16, int M, int d, const float* gamma, const float* beta,
                     float eps, float* out32, __half* out16, const ceb_moe_weights& mw, const ceb_moe_ws& ws,
                     float* logits_out, cudaStream_t st) {
    if (int rc = moe_shape_check(mw)) return rc;
    if (d != mw.d) return ceb_set_error(2, "add_ln_route: d=%d but the MoE block has d=%d", d, mw.d);
    if (M <= 0) return 0;
    return with_nv(d, [&](auto nvc) {
        constexpr int NV = decltype(nvc)::value;
        if (y_f16) {
            const AddLnRows<NV, __half> rows{res, static_cast<const __half*>(y), gamma, beta, eps, out32, out16};
            return launch_route_rows<NV>(rows, M, mw.n_experts, mw.top_k, mw.router_type, mw.router, ws, logits_out,
                                         st);
        }
        const AddLnRows<NV, float> rows{res, static_cast<const float*>(y), gamma, beta, eps, out32, out16};
        return launch_route_rows<NV>(rows, M, mw.n_experts, mw.top_k, mw.router_type, mw.router, ws, logits_out, st);
    });
}

int ceb_moe_permute(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T,
                    const ceb_moe_ws& ws, int32_t* expert_counts, const ceb_ep_args* ep, int* dev_err,
                    cudaStream_t st) {
    const int d = mw.d, E = mw.n_experts, K = mw.top_k;
    const int nblk = (T + CHUNK - 1) / CHUNK;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x16)) & 15)
        return ceb_set_error(1, "moe: activations must be 16-byte aligned");
    const ceb_ep_args none;
    const ceb_ep_args& ea = ep ? *ep : none;
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0,
               scan_kernel<<<1, SCAN_WARPS * 32, 0, st>>>(ws.block_counts, nblk, E, ws.block_base, ws.offsets, expert_counts,
                                                 ea));
    CEB_CUDA_OK(cudaGetLastError());
    if (ep)
        if (int rc = ceb_ep_wait(*ep, CEB_EPF_COUNTS, dev_err, st)) return rc;
    const int grid = std::max(nblk, 1);  // an expert-parallel rank without tokens still signals its peers
    int* err = dev_err;
    const int cat = ep ? CEB_PROF_EXCHANGE : CEB_PROF_ROUTE;
    if (x_dtype == CEB_ACT_F32)
        CEB_LAUNCH(cat, st, 0.0, 0.0,
                   scatter_kernel<float><<<grid, 256, 0, st>>>((const float*)x, x16, T, d, E, K, ws.ids, ws.block_base,
                                                               ws.slot_pos, ws.x_perm, err, ea));
    else if (x_dtype == CEB_ACT_BF16)
        CEB_LAUNCH(cat, st, 0.0, 0.0,
                   scatter_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, x16, T, d, E, K,
                                                                       ws.ids, ws.block_base, ws.slot_pos, ws.x_perm,
                                                                       err, ea));
    else
        CEB_LAUNCH(cat, st, 0.0, 0.0,
                   scatter_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, x16, T, d, E, K, ws.ids,
                                                                ws.block_base, ws.slot_pos, ws.x_perm, err, ea));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_moe_dispatch(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T, float* y,
                     const ceb_moe_ws& ws, int32_t* expert_counts, int* dev_err, cudaStream_t st) {
    if (int rc = moe_shape_check(mw)) return rc;
    const int d = mw.d, K = mw.top_k, F = mw.ffn;
    if (T <= 0) return 0;
    if (int rc = ceb_moe_permute(mw, x, x_dtype, x16, T, ws, expert_counts, nullptr, dev_err, st)) return rc;

    const int rows = T * K;
    ceb_gemm_args a1;
    a1.offsets = ws.offsets;
    a1.m_rows = rows;
    a1.out = ws.h_perm;
    a1.ldo = F;
    a1.epi = CEB_EPI_F16_OUT | CEB_EPI_GELU;
    a1.err = dev_err;
    a1.prof_cat = CEB_PROF_MOE_GEMM;
    int rc = ceb_gemm_launch(mw.fc1, ws.x_perm, rows, a1, st);
    if (rc) return rc;
    ceb_gemm_args a2;
    a2.offsets = ws.offsets;
    a2.m_rows = rows;
    a2.out = ws.down;
    a2.ldo = d;
    a2.epi = CEB_EPI_F16_OUT;
    a2.err = dev_err;
    a2.prof_cat = CEB_PROF_MOE_GEMM;
    rc = ceb_gemm_launch(mw.fc2, ws.h_perm, rows, a2, st);
    if (rc) return rc;
    if (y) {
        if (int rc = launch_combine(ws.down, ws.slot_pos, ws.wts, T, d, K, mw.bias, y, st)) return rc;
        CEB_CUDA_OK(cudaGetLastError());
    }
    return 0;
}

int ceb_moe_route(const ceb_moe_weights& mw, const void* x, int x_dtype, int T, const ceb_moe_ws& ws,
                  float* logits_out, cudaStream_t st) {
    if (int rc = moe_shape_check(mw)) return rc;
    const int d = mw.d, E = mw.n_experts, K = mw.top_k;
    if (T <= 0) return 0;
    // rows are read as 16-byte (f32) or 8-byte (bf16 / f16) vectors
    if (reinterpret_cast<uintptr_t>(x) & 15) return ceb_set_error(1, "moe: activations must be 16-byte aligned");
    return with_nv(d, [&](auto nvc) {
        constexpr int NV = decltype(nvc)::value;
        if (x_dtype == CEB_ACT_F32)
            return launch_route_rows<NV>(ActRows<float, NV>{(const float*)x}, T, E, K, mw.router_type, mw.router, ws,
                                         logits_out, st);
        if (x_dtype == CEB_ACT_BF16)
            return launch_route_rows<NV>(ActRows<__nv_bfloat16, NV>{(const __nv_bfloat16*)x}, T, E, K,
                                         mw.router_type, mw.router, ws, logits_out, st);
        return launch_route_rows<NV>(ActRows<__half, NV>{(const __half*)x}, T, E, K, mw.router_type, mw.router, ws,
                                     logits_out, st);
    });
}

int ceb_moe_run(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T, float* y,
                const ceb_moe_ws& ws, int32_t* expert_counts, float* logits_out, int* dev_err, cudaStream_t st) {
    if (int rc = ceb_moe_route(mw, x, x_dtype, T, ws, logits_out, st)) return rc;
    return ceb_moe_dispatch(mw, x, x_dtype, x16, T, y, ws, expert_counts, dev_err, st);
}

int ceb_moe_combine(const __half* down, const int32_t* slot_pos, const float* wts, int T, int d, int K,
                    const float* bias, float* y, cudaStream_t st) {
    if (T <= 0) return 0;
    if (int rc = launch_combine(down, slot_pos, wts, T, d, K, bias, y, st)) return rc;
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}
