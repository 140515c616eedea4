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
// Device pipeline: route_kernel (one warp per token) -> scan_kernel (one CTA)
// -> scatter_kernel (stable counting sort by expert, gathers fp16 rows) ->
// grouped GEMM fc1 (+GELU) -> grouped GEMM fc2 -> combine_kernel.  The expert
// row order is (expert, token, slot), the order ggml_mul_mat_id groups rows
// in, so the permutation is deterministic and identical across runs.
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <vector>

#include "ceb_internal.h"
#include "ceb_moe_internal.h"
#include "common.cuh"

namespace {

constexpr int ROUTE_WARPS = 16;         // tokens per route CTA = ROUTE_WARPS * TOK_PER_WARP
constexpr int TOK_PER_WARP = 4;
constexpr int CHUNK = ROUTE_WARPS * TOK_PER_WARP;  // tokens per histogram block (256)
constexpr int MAXE = 64;
constexpr int MAXD = 1024;  // the router gives each lane one 32-value block

template <typename T>
CEB_DEV float ld_act(const T* p, size_t i);
template <>
CEB_DEV float ld_act<float>(const float* p, size_t i) { return p[i]; }
template <>
CEB_DEV float ld_act<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) { return __bfloat162float(p[i]); }
template <>
CEB_DEV float ld_act<__half>(const __half* p, size_t i) { return __half2float(p[i]); }

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

CEB_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
CEB_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Router.  Q8_0 router weights reproduce ggml's CPU arithmetic bit for bit:
// the token row is re-quantized to Q8_0 (amax/127 scale stored as fp16,
// multiplier 127/amax, round half to even), each 32-block contributes eight
// 4-product integer partial sums (dp4a) scaled by d_w*d_x with one FMA per lane
// and block, and the eight lanes are summed as ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)).
// The Q8_0 weights are staged once per CTA in shared memory (quants padded by
// 32 B per expert row so the four experts of a pass hit distinct banks).
// F32 router weights use a plain fp32 dot read through the L1 cache.
// One warp per token, ROUTE_WARPS warps per CTA, CHUNK tokens per CTA.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(ROUTE_WARPS * 32)
    route_kernel(const T* __restrict__ x, int T_tokens, int d, int E, int K, int rtype, const uint8_t* __restrict__ rw,
                 int32_t* __restrict__ ids, float* __restrict__ wts, float* __restrict__ logits_out,
                 int32_t* __restrict__ block_counts) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int nb = d / 32;
    const int wpitch = d + 32;
    int* s_cnt = reinterpret_cast<int*>(sm);                                            // [MAXE]
    float* s_wd = reinterpret_cast<float*>(sm + MAXE * 4);                              // [E][nb]
    float* s_xd = s_wd + (size_t)E * nb;                                                // [warps][nb]
    int8_t* s_wq = reinterpret_cast<int8_t*>(s_xd + (size_t)ROUTE_WARPS * nb);         // [E][wpitch]
    int8_t* s_xq = s_wq + (size_t)E * wpitch;                                           // [warps][d]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < E; i += blockDim.x) s_cnt[i] = 0;
    if (rtype == CEB_GGML_Q8_0) {
        // stage weights: block (e, b) -> scale s_wd[e][b], quants s_wq[e][b*32 .. +31]
        for (int i = threadIdx.x; i < E * nb; i += blockDim.x) {
            const uint8_t* blk = rw + (size_t)i * 34;
            const int e = i / nb, b = i - e * nb;
            s_wd[i] = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
            int8_t* dst = s_wq + (size_t)e * wpitch + b * 32;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) dst[j] = (int8_t)blk[2 + j];
        }
    }
    __syncthreads();
    int8_t* q = s_xq + (size_t)warp * d;
    float* qd = s_xd + (size_t)warp * nb;

    for (int tt = 0; tt < TOK_PER_WARP; ++tt) {
        const int t = blockIdx.x * CHUNK + warp * TOK_PER_WARP + tt;
        if (t >= T_tokens) break;
        const T* xr = x + (size_t)t * d;
        float lg_mine = -INFINITY;  // lane e < E ends up holding logit e
        if (rtype == CEB_GGML_Q8_0) {
            // 128 values per pass, 4 per lane (coalesced); 8 lanes hold one 32-value
            // block, whose amax three xor-shuffles combine.  Packed quants land in
            // consecutive shared-memory words.
            for (int seg = 0; seg < d / 128; ++seg) {
                const float4 v = ld_act4<T>(xr, (size_t)seg * 128 + 4 * lane);
                float am = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
                const float id = am != 0.0f ? 127.0f / am : 0.0f;
                const uint32_t b0 = (uint32_t)(__float2int_rn(v.x * id) & 0xFF);
                const uint32_t b1 = (uint32_t)(__float2int_rn(v.y * id) & 0xFF);
                const uint32_t b2 = (uint32_t)(__float2int_rn(v.z * id) & 0xFF);
                const uint32_t b3 = (uint32_t)(__float2int_rn(v.w * id) & 0xFF);
                reinterpret_cast<uint32_t*>(q)[seg * 32 + lane] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
                if ((lane & 7) == 0) qd[seg * 4 + (lane >> 3)] = __half2float(__float2half_rn(am / 127.0f));
            }
            __syncwarp();
            // lane = (expert-in-pass, partial-lane): 4 experts x 8 lanes per pass
            for (int e0 = 0; e0 < E; e0 += 4) {
                const int e = e0 + (lane >> 3), l = lane & 7;
                float acc = 0.0f;
                if (e < E) {
                    const int8_t* wq = s_wq + (size_t)e * wpitch + 4 * l;
                    const float* wd = s_wd + (size_t)e * nb;
                    const int8_t* xq = q + 4 * l;
                    for (int b = 0; b < nb; ++b) {
                        const int s = __dp4a(*reinterpret_cast<const int*>(wq + b * 32),
                                             *reinterpret_cast<const int*>(xq + b * 32), 0);
                        acc = __fmaf_rn(__fmul_rn(wd[b], qd[b]), (float)s, acc);
                    }
                }
                // ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)) within each group of 8 lanes
                const float p4 = __shfl_xor_sync(0xffffffffu, acc, 4);
                const float s1 = __fadd_rn(acc, p4);                       // lane l<4: l + (l+4)
                const float p2 = __shfl_xor_sync(0xffffffffu, s1, 2);
                const float s2 = __fadd_rn(s1, p2);                        // l=0: (0+4)+(2+6), l=1: (1+5)+(3+7)
                const float p1 = __shfl_xor_sync(0xffffffffu, s2, 1);
                const float tot = __fadd_rn(s2, p1);
                // lane 8j holds expert e0+j; hand it to lane e0+j
                for (int j = 0; j < 4; ++j) {
                    const float r = __shfl_sync(0xffffffffu, tot, j * 8);
                    if (lane == e0 + j) lg_mine = r;
                }
            }
            __syncwarp();
        } else {
            for (int e = 0; e < E; ++e) {
                const float* wr = reinterpret_cast<const float*>(rw) + (size_t)e * d;
                float acc = 0.0f;
                for (int i = lane; i < d; i += 32) acc = __fmaf_rn(ld_act<T>(xr, i), __ldg(wr + i), acc);
                acc = warp_sum(acc);
                if (lane == e) lg_mine = acc;
            }
        }
        // softmax over lanes 0..E-1 (E <= 32 handled in registers)
        const float mx = warp_max(lane < E ? lg_mine : -INFINITY);
        const float ex = lane < E ? expf(lg_mine - mx) : 0.0f;
        double sum = ex;
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float p = lane < E ? ex * (float)(1.0 / sum) : -1.0f;
        if (logits_out && lane < E) logits_out[(size_t)t * E + lane] = lg_mine;
        // top-K: repeated argmax, ties to the lower expert index
        bool taken = false;
        for (int j = 0; j < K; ++j) {
            float v = (lane < E && !taken) ? p : -2.0f;
            int idx = lane;
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (ov > v || (ov == v && oi < idx)) {
                    v = ov;
                    idx = oi;
                }
            }
            if (lane == idx) taken = true;
            if (lane == 0) {
                ids[(size_t)t * K + j] = idx;
                wts[(size_t)t * K + j] = v;
                atomicAdd(&s_cnt[idx], 1);
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) block_counts[(size_t)blockIdx.x * E + i] = s_cnt[i];
}

// One CTA: expert offsets (exclusive scan of the totals) and, per histogram
// block, the first output row of each expert.  The per-block counts are staged
// in shared memory first (coalesced), then each expert's thread walks them.
constexpr int SCAN_MAX_SMEM_INTS = 48 * 1024 / 4;

__global__ void __launch_bounds__(256) scan_kernel(const int32_t* __restrict__ block_counts, int nblk, int E,
                                                   int32_t* __restrict__ block_base, int32_t* __restrict__ offsets,
                                                   int32_t* __restrict__ expert_counts) {
    extern __shared__ int sc[];  // [nblk*E] counts (when they fit), then [E] totals
    const int n = nblk * E;
    const bool staged = n <= SCAN_MAX_SMEM_INTS - MAXE;
    int* tot = staged ? sc + n : sc;
    if (staged)
        for (int i = threadIdx.x; i < n; i += blockDim.x) sc[i] = block_counts[i];
    __syncthreads();
    const int e = threadIdx.x;
    if (e < E) {
        int s = 0;
        if (staged)
            for (int b = 0; b < nblk; ++b) s += sc[b * E + e];
        else
            for (int b = 0; b < nblk; ++b) s += block_counts[(size_t)b * E + e];
        tot[e] = s;
        if (expert_counts) expert_counts[e] = s;
    }
    __syncthreads();
    if (e < E) {
        int base = 0;
        for (int i = 0; i < e; ++i) base += tot[i];
        if (e == 0) offsets[0] = 0;
        offsets[e + 1] = base + tot[e];
        for (int b = 0; b < nblk; ++b) {
            block_base[(size_t)b * E + e] = base;
            base += staged ? sc[b * E + e] : block_counts[(size_t)b * E + e];
        }
    }
}

// Stable placement of every (token, slot) into its expert's row range, then a
// gather of the token rows (converted to fp16) into the permuted activation
// matrix consumed by fc1.
template <typename T>
__global__ void __launch_bounds__(256)
    scatter_kernel(const T* __restrict__ x, const __half* __restrict__ x16, int T_tokens, int d, int E, int K,
                   const int32_t* __restrict__ ids, const int32_t* __restrict__ block_base,
                   int32_t* __restrict__ slot_pos, __half* __restrict__ x_perm) {
    __shared__ int running[MAXE];
    __shared__ int s_pos[CHUNK * 4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * CHUNK;
    const int n_tok = min(CHUNK, T_tokens - t0);
    const int n_slots = n_tok * K;
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
                slot_pos[(size_t)t0 * K + s] = pos;
            }
        }
    }
    __syncthreads();
    // gather rows: one warp per slot.  With an fp16 copy of x available the rows
    // move as 16-byte vectors; otherwise they are converted on the fly.
    for (int s = warp; s < n_slots; s += blockDim.x / 32) {
        const int pos = s_pos[s];
        if (pos < 0) continue;
        __half* dst = x_perm + (size_t)pos * d;
        if (x16) {
            const uint4* src = reinterpret_cast<const uint4*>(x16 + (size_t)(t0 + s / K) * d);
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            for (int c = lane; c < d / 8; c += 32) d4[c] = __ldg(src + c);
        } else {
            const T* src = x + (size_t)(t0 + s / K) * d;
            for (int c = lane * 2; c < d; c += 64) {
                const float a = ld_act<T>(src, c), b = ld_act<T>(src, c + 1);
                *reinterpret_cast<__half2*>(dst + c) = __floats2half2_rn(a, b);
            }
        }
    }
}

// y[t, c] = sum_j w[t,j] * down[pos(t,j), c] (fmaf in slot order) + bias[c]
__global__ void combine_kernel(const float* __restrict__ down, const int32_t* __restrict__ slot_pos,
                               const float* __restrict__ wts, int T_tokens, int d, int K, const float* __restrict__ bias,
                               float* __restrict__ y) {
    const int t = blockIdx.x;
    if (t >= T_tokens) return;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        float s = 0.0f;
        for (int j = 0; j < K; ++j) {
            const int pos = slot_pos[(size_t)t * K + j];
            s = __fmaf_rn(wts[(size_t)t * K + j], down[(size_t)pos * d + c], s);
        }
        y[(size_t)t * d + c] = bias ? __fadd_rn(s, bias[c]) : s;
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
    w.down = (float*)take(S * d * 4);
    if (ws) *ws = w;
    return off;
}

int ceb_moe_run(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T, float* y,
                const ceb_moe_ws& ws, int32_t* expert_counts, float* logits_out, int* dev_err, cudaStream_t st) {
    const int d = mw.d, E = mw.n_experts, K = mw.top_k, F = mw.ffn;
    if (T <= 0) return 0;
    if (E > 32 || E < 1 || K < 1 || K > E || K > 4 || d > MAXD || F % 128 || d % 128)
        return ceb_set_error(2, "moe: unsupported shape d=%d E=%d K=%d F=%d", d, E, K, F);
    const int nblk = (T + CHUNK - 1) / CHUNK;
    const size_t route_smem = MAXE * 4 + (size_t)(E + ROUTE_WARPS) * (d / 32) * 4 + (size_t)E * (d + 32) +
                              (size_t)ROUTE_WARPS * d;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(route_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        cudaFuncSetAttribute(route_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        cudaFuncSetAttribute(route_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        attr = true;
    }
    if (x_dtype == CEB_ACT_F32) {
        CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, route_kernel<float><<<nblk, ROUTE_WARPS * 32, route_smem, st>>>((const float*)x, T, d, E, K, mw.router_type,
                                                                        mw.router, ws.ids, ws.wts, logits_out,
                                                                        ws.block_counts));
    } else if (x_dtype == CEB_ACT_BF16) {
        CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, route_kernel<__nv_bfloat16><<<nblk, ROUTE_WARPS * 32, route_smem, st>>>(
            (const __nv_bfloat16*)x, T, d, E, K, mw.router_type, mw.router, ws.ids, ws.wts, logits_out,
            ws.block_counts));
    } else {
        CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, route_kernel<__half><<<nblk, ROUTE_WARPS * 32, route_smem, st>>>((const __half*)x, T, d, E, K, mw.router_type,
                                                                         mw.router, ws.ids, ws.wts, logits_out,
                                                                         ws.block_counts));
    }
    CEB_CUDA_OK(cudaGetLastError());
    const size_t scan_smem = (size_t)std::min(nblk * E + MAXE, SCAN_MAX_SMEM_INTS) * sizeof(int);
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, scan_kernel<<<1, 256, scan_smem, st>>>(ws.block_counts, nblk, E, ws.block_base, ws.offsets, expert_counts));
    CEB_CUDA_OK(cudaGetLastError());
    if (x_dtype == CEB_ACT_F32)
        CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, scatter_kernel<float><<<nblk, 256, 0, st>>>((const float*)x, x16, T, d, E, K, ws.ids, ws.block_base, ws.slot_pos,
                                                    ws.x_perm));
    else if (x_dtype == CEB_ACT_BF16)
        CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, scatter_kernel<__nv_bfloat16><<<nblk, 256, 0, st>>>((const __nv_bfloat16*)x, x16, T, d, E, K, ws.ids,
                                                            ws.block_base, ws.slot_pos, ws.x_perm));
    else
        CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0, scatter_kernel<__half><<<nblk, 256, 0, st>>>((const __half*)x, x16, T, d, E, K, ws.ids, ws.block_base, ws.slot_pos,
                                                     ws.x_perm));
    CEB_CUDA_OK(cudaGetLastError());

    const int rows = T * K;
    ceb_gemm_args a1;
    a1.offsets = ws.offsets;
    a1.m_rows = rows;
    a1.out = ws.h_perm;
    a1.ldo = F;
    a1.epi = CEB_EPI_F16_OUT | CEB_EPI_GELU;
    a1.err = dev_err;
    int rc = ceb_gemm_launch(mw.fc1, ws.x_perm, rows, a1, st);
    if (rc) return rc;
    ceb_gemm_args a2;
    a2.offsets = ws.offsets;
    a2.m_rows = rows;
    a2.out = ws.down;
    a2.ldo = d;
    a2.epi = 0;
    a2.err = dev_err;
    rc = ceb_gemm_launch(mw.fc2, ws.h_perm, rows, a2, st);
    if (rc) return rc;
    if (y) {
        CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0, combine_kernel<<<T, 256, 0, st>>>(ws.down, ws.slot_pos, ws.wts, T, d, K, mw.bias, y));
        CEB_CUDA_OK(cudaGetLastError());
    }
    return 0;
}
