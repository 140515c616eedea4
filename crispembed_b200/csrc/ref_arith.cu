// ref_arith.cu -- the encoder in the reference's CPU arithmetic, bit for bit.
//
// The default encoder runs its matrix products on the tensor cores with fp16
// operands.  The reference's ggml CPU backend instead re-quantizes every
// activation that meets a Q8_0 weight to Q8_0 (32 values, fp16 scale) and sums
// integer block dots into eight float lanes (ggml_vec_dot_q8_0_q8_0); its
// attention, LayerNorm, softmax and pooling accumulate in fixed sequential
// orders.  With activations re-quantized, a difference of one ulp anywhere
// upstream can move a value across a Q8_0 rounding step and change a token's
// expert choice downstream, so the expert ids of the reference can only be
// reproduced by reproducing its arithmetic exactly.  These kernels do that, op
// for op, in the order of the CPU restatement of the reference graph
// (src/crispembed.cpp:1068-1428 and :1794-1846 with ggml's x86 CPU kernels):
//
//   * Q8_0 activations: d = amax/127 stored as fp16, q = round-half-even(x*127/amax);
//   * Q8_0 x Q8_0 dots: lane l of a block = integer sum of products 4l..4l+3
//     (one dp4a), acc_l = fma(d_w*d_x, lane, acc_l) block by block, result
//     ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)) (an xor-4/2/1 shuffle butterfly);
//   * float weights: acc = fma(x_i, w_i, acc) for i = 0..k-1;
//   * LayerNorm: mean and variance summed in double, in index order;
//   * attention: per query, keys in order with an online softmax;
//   * exp / erf: the shared double-precision routines of ceb_portable_math.h.
//
// This file is compiled with -fmad=false: every multiply-add that is fused is an
// explicit fmaf, as in the restatement.  Throughput is not the goal here
// (CUDA-core integer dots, one thread per attention query); the mode exists so
// the expert choice can be checked against the reference arithmetic exactly.
#include <cuda_fp16.h>

#include <cstring>
#include <vector>

#include "ceb_encoder_internal.h"
#include "ceb_portable_math.h"
#include "common.cuh"

namespace {

constexpr int QK = 32;  // Q8_0 block

}  // namespace

int ceb_refmat_create(ceb_refmat* r, int ggml_type, const void* host, int groups, int n_out, int k) {
    ceb_refmat_free(r);
    if (groups <= 0 || n_out <= 0 || k <= 0) return ceb_set_error(1, "reference arithmetic: bad weight shape");
    const size_t rows = (size_t)groups * n_out;
    const uint8_t* src = static_cast<const uint8_t*>(host);
    if (ggml_type == CEB_GGML_Q8_0) {
        if (k % QK) return ceb_set_error(2, "reference arithmetic: Q8_0 rows of %d values", k);
        const int nb = k / QK;
        std::vector<int8_t> q(rows * k);
        std::vector<float> d(rows * nb);
        for (size_t row = 0; row < rows; ++row)
            for (int b = 0; b < nb; ++b) {
                const uint8_t* blk = src + (row * nb + b) * 34;
                __half_raw h;
                h.x = (uint16_t)(blk[0] | (blk[1] << 8));
                d[row * nb + b] = __half2float(__half(h));
                memcpy(&q[row * k + (size_t)b * QK], blk + 2, QK);
            }
        if (cudaMalloc(&r->q, q.size()) != cudaSuccess || cudaMalloc(&r->d, d.size() * 4) != cudaSuccess) {
            ceb_refmat_free(r);
            return ceb_set_error(4, "reference arithmetic: out of device memory");
        }
        if (cudaMemcpy(r->q, q.data(), q.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(r->d, d.data(), d.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return ceb_set_error(3, "reference arithmetic: weight upload failed");
        r->type = CEB_GGML_Q8_0;
    } else if (ggml_type == CEB_GGML_F32 || ggml_type == CEB_GGML_F16 || ggml_type == CEB_GGML_BF16) {
        std::vector<float> f(rows * k);
        if (ggml_type == CEB_GGML_F32) {
            memcpy(f.data(), src, f.size() * 4);
        } else {
            for (size_t i = 0; i < f.size(); ++i) {
                const uint16_t v = (uint16_t)(src[2 * i] | (src[2 * i + 1] << 8));
                if (ggml_type == CEB_GGML_F16) {
                    __half_raw h;
                    h.x = v;
                    f[i] = __half2float(__half(h));
                } else {
                    const uint32_t bits = (uint32_t)v << 16;
                    memcpy(&f[i], &bits, 4);
                }
            }
        }
        if (cudaMalloc(&r->f, f.size() * 4) != cudaSuccess) return ceb_set_error(4, "reference arithmetic: out of device memory");
        if (cudaMemcpy(r->f, f.data(), f.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return ceb_set_error(3, "reference arithmetic: weight upload failed");
        r->type = CEB_GGML_F32;
    } else {
        return ceb_set_error(2, "reference arithmetic covers F32/F16/BF16/Q8_0 weights (type %d given)", ggml_type);
    }
    r->n_groups = groups;
    r->n_out = n_out;
    r->k = k;
    return 0;
}

void ceb_refmat_free(ceb_refmat* r) {
    if (r->q) cudaFree(r->q);
    if (r->d) cudaFree(r->d);
    if (r->f) cudaFree(r->f);
    *r = ceb_refmat();
}

namespace {

// ------------------------------------------------------------ row-wise
// out[t] = (tok[id] + pos[t - cu[s] + pos_offset]) + type0, one block per sequence
__global__ void ref_embed_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int d, int n_vocab,
                                 const float* __restrict__ tok, const float* __restrict__ pos, int n_pos,
                                 int pos_offset, const float* __restrict__ type0, float* __restrict__ out,
                                 int* __restrict__ err) {
    const int s = blockIdx.x;
    const int t0 = cu[s], t1 = cu[s + 1];
    for (int64_t e = (int64_t)t0 * d + threadIdx.x; e < (int64_t)t1 * d; e += blockDim.x) {
        const int t = (int)(e / d), c = (int)(e % d);
        const int id = ids[t];
        const int p = t - t0 + pos_offset;
        if (id < 0 || id >= n_vocab || (pos && (p < 0 || p >= n_pos))) {
            if (err) atomicCAS(err, 0, 0x201);
            out[e] = 0.0f;
            continue;
        }
        float x = tok[(int64_t)id * d + c];
        if (pos) x = x + pos[(int64_t)p * d + c];
        if (type0) x = x + type0[c];
        out[e] = x;
    }
}

// out = LN(a + b) * gamma + beta as the restatement computes it: the row sum and
// the sum of squared centred values accumulated in double in index order (lane 0
// of the row's warp, from shared memory), centred values and the scaling in
// float.  Warp per row.
constexpr int LN_WARPS = 8;
__global__ void __launch_bounds__(LN_WARPS * 32) ref_ln_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                               int M, int d, const float* __restrict__ gamma,
                                                               const float* __restrict__ beta, float eps,
                                                               float* __restrict__ out) {
    extern __shared__ float ln_rows[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * LN_WARPS + warp;
    if (r >= M) return;
    float* row = ln_rows + (size_t)warp * d;
    __shared__ float scale_s[LN_WARPS];
    for (int i = lane; i < d; i += 32) {
        float v = a[(int64_t)r * d + i];
        if (b) v = v + b[(int64_t)r * d + i];
        row[i] = v;
    }
    __syncwarp();
    if (lane == 0) {
        double sum = 0.0;
        for (int i = 0; i < d; ++i) sum += (double)row[i];
        const float mean = (float)(sum / (double)d);
        double sum2 = 0.0;
        for (int i = 0; i < d; ++i) {
            const float v = row[i] - mean;
            row[i] = v;
            sum2 += (double)(v * v);
        }
        const float variance = (float)(sum2 / (double)d);
        scale_s[warp] = 1.0f / sqrtf(variance + eps);
    }
    __syncwarp();
    const float scale = scale_s[warp];
    for (int i = lane; i < d; i += 32) {
        float v = row[i] * scale;
        if (gamma) v = v * gamma[i];
        if (beta) v = v + beta[i];
        out[(int64_t)r * d + i] = v;
    }
}

// Q8_0 quantization of activation rows (ggml's x86 quantize_row_q8_0): one
// thread per 32-value block.  xq [rows x k] int8, xd [rows x k/32] scales as the
// float value of the stored fp16.
__global__ void ref_quant_kernel(const float* __restrict__ x, int64_t n_blocks, int nb_row, int k,
                                 int8_t* __restrict__ xq, float* __restrict__ xd) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n_blocks) return;
    const int64_t row = g / nb_row;
    const int b = (int)(g % nb_row);
    const float* xb = x + row * k + (int64_t)b * QK;
    float v[QK];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < QK; j += 4) {
        const float4 f = *reinterpret_cast<const float4*>(xb + j);
        v[j] = f.x;
        v[j + 1] = f.y;
        v[j + 2] = f.z;
        v[j + 3] = f.w;
    }
#pragma unroll
    for (int j = 0; j < QK; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float dv = amax / 127.0f;
    const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
    xd[g] = __half2float(__float2half_rn(dv));
    int8_t* q = xq + row * k + (int64_t)b * QK;
#pragma unroll
    for (int j = 0; j < QK; j += 4) {
        char4 c;
        c.x = (signed char)(int)rintf(v[j] * id);
        c.y = (signed char)(int)rintf(v[j + 1] * id);
        c.z = (signed char)(int)rintf(v[j + 2] * id);
        c.w = (signed char)(int)rintf(v[j + 3] * id);
        *reinterpret_cast<char4*>(q + j) = c;
    }
}

// ------------------------------------------------------------ matrix products
// out[m, n] = dot(W_g[n], x[m]) (+ bias_g[n]), 32 x 32 output tiles; grouped
// products give every 32-row tile one group (tile_group[tile], -1 = unused tile).
constexpr int MT = 32, KB = 8;                 // tile side, Q8_0 blocks per staged chunk
constexpr int Q8_STRIDE = KB * QK / 4 + 8;     // int words per staged row: rows 8 banks apart

__global__ void __launch_bounds__(256) ref_matmul_q8_kernel(const int8_t* __restrict__ xq,
                                                            const float* __restrict__ xd, int rows, int k,
                                                            const int8_t* __restrict__ wq,
                                                            const float* __restrict__ wd, int n_out,
                                                            const int32_t* __restrict__ tile_group,
                                                            const float* __restrict__ bias, int64_t bias_gstride,
                                                            float* __restrict__ out, int ldo) {
    __shared__ int xs[MT][Q8_STRIDE];
    __shared__ int ws[MT][Q8_STRIDE];
    __shared__ float xds[MT][KB];
    __shared__ float wds[MT][KB];
    const int tile = blockIdx.y;
    const int g = tile_group ? tile_group[tile] : 0;
    if (g < 0) return;
    const int m0 = tile * MT, n0 = blockIdx.x * MT;
    const int nb = k / QK;
    const int8_t* wg = wq + (size_t)g * n_out * k;
    const float* wdg = wd + (size_t)g * n_out * nb;
    const int tid = threadIdx.x, l = tid & 7, slot = tid >> 3;
    const int rsub = slot >> 2, csub = slot & 3;  // rows rsub*4+i, columns csub+4j
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += KB) {
        const int kb = min(KB, nb - b0);
        __syncthreads();
        // stage 32 rows x kb blocks of x and of W (int words), and their scales
        for (int e = tid; e < MT * KB * QK / 16; e += 256) {
            const int rr = e / (KB * 2), c16 = e % (KB * 2);  // 16-byte chunk c16 of row rr
            if (c16 < kb * 2) {
                const int mrow = m0 + rr, nrow = n0 + rr;
                int4 xv = make_int4(0, 0, 0, 0), wv = make_int4(0, 0, 0, 0);
                if (mrow < rows) xv = *reinterpret_cast<const int4*>(xq + (int64_t)mrow * k + b0 * QK + c16 * 16);
                if (nrow < n_out) wv = *reinterpret_cast<const int4*>(wg + (int64_t)nrow * k + b0 * QK + c16 * 16);
                xs[rr][c16 * 4] = xv.x;
                xs[rr][c16 * 4 + 1] = xv.y;
                xs[rr][c16 * 4 + 2] = xv.z;
                xs[rr][c16 * 4 + 3] = xv.w;
                ws[rr][c16 * 4] = wv.x;
                ws[rr][c16 * 4 + 1] = wv.y;
                ws[rr][c16 * 4 + 2] = wv.z;
                ws[rr][c16 * 4 + 3] = wv.w;
            }
        }
        for (int e = tid; e < MT * KB; e += 256) {
            const int rr = e / KB, bb = e % KB;
            if (bb < kb) {
                const int mrow = m0 + rr, nrow = n0 + rr;
                xds[rr][bb] = mrow < rows ? xd[(int64_t)mrow * nb + b0 + bb] : 0.0f;
                wds[rr][bb] = nrow < n_out ? wdg[(int64_t)nrow * nb + b0 + bb] : 0.0f;
            }
        }
        __syncthreads();
        for (int bb = 0; bb < kb; ++bb) {
            int xw[4], ww[8];
            float xdv[4], wdv[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xw[i] = xs[rsub * 4 + i][bb * 8 + l];
                xdv[i] = xds[rsub * 4 + i][bb];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                ww[j] = ws[csub + 4 * j][bb * 8 + l];
                wdv[j] = wds[csub + 4 * j][bb];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float dd = wdv[j] * xdv[i];
                    const int s = __dp4a(ww[j], xw[i], 0);
                    acc[i][j] = fmaf(dd, (float)s, acc[i][j]);
                }
        }
    }
    // ggml's horizontal sum of the eight lanes: ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7))
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float v = acc[i][j];
            v = v + __shfl_xor_sync(0xffffffffu, v, 4);
            v = v + __shfl_xor_sync(0xffffffffu, v, 2);
            v = v + __shfl_xor_sync(0xffffffffu, v, 1);
            const int m = m0 + rsub * 4 + i, n = n0 + csub + 4 * j;
            if (l == 0 && m < rows && n < n_out) {
                const float* bg = bias ? bias + (int64_t)g * bias_gstride : nullptr;
                out[(int64_t)m * ldo + n] = bg ? v + bg[n] : v;
            }
        }
}

// float weights: sequential fma over k per output (32 x 32 tile, 4 rows per thread)
__global__ void __launch_bounds__(256) ref_matmul_f32_kernel(const float* __restrict__ x, int rows, int k,
                                                             const float* __restrict__ w, int n_out,
                                                             const int32_t* __restrict__ tile_group,
                                                             const float* __restrict__ bias, int64_t bias_gstride,
                                                             float* __restrict__ out, int ldo) {
    __shared__ float xs[MT][MT + 1];
    __shared__ float wsm[MT][MT + 1];
    const int tile = blockIdx.y;
    const int g = tile_group ? tile_group[tile] : 0;
    if (g < 0) return;
    const int m0 = tile * MT, n0 = blockIdx.x * MT;
    const float* wg = w + (size_t)g * n_out * k;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int k0 = 0; k0 < k; k0 += MT) {
        __syncthreads();
        for (int e = threadIdx.x; e < MT * MT; e += 256) {
            const int rr = e / MT, kk = e % MT;
            const int mrow = m0 + rr, nrow = n0 + rr, kc = k0 + kk;
            xs[rr][kk] = (mrow < rows && kc < k) ? x[(int64_t)mrow * k + kc] : 0.0f;
            wsm[rr][kk] = (nrow < n_out && kc < k) ? wg[(int64_t)nrow * k + kc] : 0.0f;
        }
        __syncthreads();
        const int kn = min(MT, k - k0);
        for (int kk = 0; kk < kn; ++kk) {
            const float wv = wsm[tx][kk];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = fmaf(xs[ty * 4 + i][kk], wv, acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i, n = n0 + tx;
        if (m < rows && n < n_out) {
            const float* bg = bias ? bias + (int64_t)g * bias_gstride : nullptr;
            out[(int64_t)m * ldo + n] = bg ? acc[i] + bg[n] : acc[i];
        }
    }
}

// ------------------------------------------------------------ attention
// One thread per (query, head): keys in order, online softmax (running max M,
// sum S, accumulator rescaled by exp(M_old - M)), as the restatement of ggml's
// flash_attn_ext over f32 K/V.  head_dim 64.
constexpr int HD = 64;
__global__ void __launch_bounds__(64) ref_attention_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ cu,
                                                           int d, float scale, float* __restrict__ out) {
    const int s = blockIdx.z, h = blockIdx.y;
    const int t0 = cu[s], len = cu[s + 1] - t0;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= len) return;
    const int64_t ld = 3 * (int64_t)d;
    float q[HD], acc[HD];
    const float* qi = qkv + (int64_t)(t0 + i) * ld + h * HD;
#pragma unroll
    for (int c = 0; c < HD; ++c) {
        q[c] = qi[c];
        acc[c] = 0.0f;
    }
    float M = -INFINITY, S = 0.0f;
    for (int j = 0; j < len; ++j) {
        const float* kj = qkv + (int64_t)(t0 + j) * ld + d + h * HD;
        const float* vj = kj + d;
        float sdot = 0.0f;
#pragma unroll
        for (int c = 0; c < HD; ++c) sdot = fmaf(q[c], kj[c], sdot);
        const float sc = sdot * scale;
        float ms = 1.0f, vs = 1.0f;
        if (sc > M) {
            const float Mold = M;
            M = sc;
            ms = ceb_expf(Mold - M);
#pragma unroll
            for (int c = 0; c < HD; ++c) acc[c] *= ms;
        } else {
            vs = ceb_expf(sc - M);
        }
#pragma unroll
        for (int c = 0; c < HD; ++c) acc[c] = fmaf(vj[c], vs, acc[c]);
        S = S * ms + vs;
    }
    const float inv = S == 0.0f ? 0.0f : 1.0f / S;
    float* o = out + (int64_t)(t0 + i) * d + h * HD;
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] = acc[c] * inv;
}

// ------------------------------------------------------------ elementwise
__global__ void ref_gelu_kernel(float* __restrict__ x, int64_t n) {
    const float s2 = 0.70710678118654752440f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = 0.5f * x[i] * (1.0f + ceb_erff(x[i] * s2));
}

// ------------------------------------------------------------ MoE
// softmax (max-subtracted exp, double sum, scaled by 1/sum) and top-k by
// probability, ties to the lower index; weights not renormalised.  Thread per token.
__global__ void ref_route_kernel(const float* __restrict__ logits, int T, int E, int K, int32_t* __restrict__ ids,
                                 float* __restrict__ wts) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const float* lg = logits + (int64_t)t * E;
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = lg[e] > mx ? lg[e] : mx;
    float p[32];
    double sum = 0.0;
    for (int e = 0; e < E; ++e) {
        p[e] = ceb_expf(lg[e] - mx);
        sum += (double)p[e];
    }
    const float inv = (float)(1.0 / sum);
    for (int e = 0; e < E; ++e) p[e] *= inv;
    unsigned used = 0;
    for (int j = 0; j < K; ++j) {
        int best = -1;
        for (int e = 0; e < E; ++e)
            if (!(used >> e & 1u) && (best < 0 || p[e] > p[best])) best = e;
        used |= 1u << best;
        ids[(int64_t)t * K + j] = best;
        wts[(int64_t)t * K + j] = p[best];
    }
}

// Rows of each expert, each expert's range padded to whole 32-row tiles: pos[r]
// = permuted row of (token, slot) r, src[p] = token of permuted row p (-1 for
// padding), tile_group[tile] = expert (-1 past the last used tile).  The order
// inside an expert's range does not matter: every row is computed on its own.
// One block.
__global__ void ref_group_kernel(const int32_t* __restrict__ ids, int T, int K, int E, int n_tiles_max,
                                 int32_t* __restrict__ pos, int32_t* __restrict__ src,
                                 int32_t* __restrict__ tile_group) {
    __shared__ int cnt[32], off[33], cursor[32];
    const int R = T * K;
    if (threadIdx.x < 32) cnt[threadIdx.x] = 0;
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) atomicAdd(&cnt[ids[r]], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        off[0] = 0;
        for (int e = 0; e < E; ++e) off[e + 1] = off[e] + ((cnt[e] + MT - 1) / MT) * MT;
        for (int e = 0; e < E; ++e) cursor[e] = off[e];
    }
    __syncthreads();
    for (int tl = threadIdx.x; tl < n_tiles_max; tl += blockDim.x) {
        int g = -1;
        for (int e = 0; e < E; ++e)
            if (tl * MT >= off[e] && tl * MT < off[e + 1]) g = e;
        tile_group[tl] = g;
    }
    for (int p = threadIdx.x; p < n_tiles_max * MT; p += blockDim.x) src[p] = -1;
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int p = atomicAdd(&cursor[ids[r]], 1);
        pos[r] = p;
        src[p] = r / K;
    }
}

// x_perm[p] = x[src[p]] (zeros for padding rows)
__global__ void ref_gather_kernel(const float* __restrict__ x, const int32_t* __restrict__ src, int64_t n_rows, int d,
                                  float* __restrict__ xp) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_rows * d;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = e / d;
        const int t = src[p];
        xp[e] = t >= 0 ? x[(int64_t)t * d + e % d] : 0.0f;
    }
}

// y[t, c] = sum_j fma(w[t, j], down[pos[t, j], c], .) in slot order (+ bias[c])
__global__ void ref_combine_kernel(const float* __restrict__ down, const int32_t* __restrict__ pos,
                                   const float* __restrict__ wts, int T, int K, int d, const float* __restrict__ bias,
                                   float* __restrict__ y) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)T * d;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = e / d;
        const int c = (int)(e % d);
        float s = 0.0f;
        for (int j = 0; j < K; ++j) s = fmaf(wts[t * K + j], down[(int64_t)pos[t * K + j] * d + c], s);
        y[e] = bias ? s + bias[c] : s;
    }
}

// ------------------------------------------------------------ pooling
// p[h] = (sum over the sequence's rows, in order) / n, then p / sqrt(max(sum p^2,
// 1e-12)) with the squares summed in index order; with out_dim < d the first
// out_dim values are normalised again over themselves (Matryoshka).  Block per
// sequence.
__global__ void ref_pool_kernel(const float* __restrict__ x, const int32_t* __restrict__ cu, int d, int out_dim,
                                float* __restrict__ out) {
    extern __shared__ float pool_p[];
    __shared__ float norm_s;
    const int s = blockIdx.x;
    const int t0 = cu[s], t1 = cu[s + 1], n = t1 - t0;
    for (int h = threadIdx.x; h < d; h += blockDim.x) {
        float p = 0.0f;
        for (int t = t0; t < t1; ++t) p += x[(int64_t)t * d + h];
        if (n > 0) p /= (float)n;
        pool_p[h] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float norm = 0.0f;
        for (int h = 0; h < d; ++h) norm += pool_p[h] * pool_p[h];
        norm = sqrtf(norm > 1e-12f ? norm : 1e-12f);
        for (int h = 0; h < d; ++h) pool_p[h] /= norm;
        if (out_dim < d) {
            float n2 = 0.0f;
            for (int h = 0; h < out_dim; ++h) n2 += pool_p[h] * pool_p[h];
            norm_s = sqrtf(n2 > 1e-12f ? n2 : 1e-12f);
        } else {
            norm_s = 1.0f;
        }
    }
    __syncthreads();
    for (int h = threadIdx.x; h < out_dim; h += blockDim.x)
        out[(int64_t)s * out_dim + h] = out_dim < d ? pool_p[h] / norm_s : pool_p[h];
}

int grid_1d(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return (int)(b < 148 * 64 ? (b > 0 ? b : 1) : 148 * 64);
}

}  // namespace

// ================================================================ launchers
int ceb_ref_embed(const int32_t* ids, const int32_t* cu, int n_seqs, int d, int n_vocab, const float* tok,
                  const float* pos, int n_pos, int pos_offset, const float* type0, float* out, int* err,
                  cudaStream_t st) {
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               ref_embed_kernel<<<n_seqs, 256, 0, st>>>(ids, cu, d, n_vocab, tok, pos, n_pos, pos_offset, type0, out,
                                                        err));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_ln(const float* a, const float* b, int M, int d, const float* gamma, const float* beta, float eps,
               float* out, cudaStream_t st) {
    if (M <= 0) return 0;
    const size_t smem = (size_t)LN_WARPS * d * 4;
    if (smem > 48 * 1024) return ceb_set_error(2, "reference LayerNorm: rows of %d values too wide", d);
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               ref_ln_kernel<<<(M + LN_WARPS - 1) / LN_WARPS, LN_WARPS * 32, smem, st>>>(a, b, M, d, gamma, beta, eps,
                                                                                       out));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_quant(const float* x, int rows, int k, int8_t* xq, float* xd, cudaStream_t st) {
    if (rows <= 0) return 0;
    if (k % QK) return ceb_set_error(2, "reference quantization: rows of %d values", k);
    const int64_t nbk = (int64_t)rows * (k / QK);
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               ref_quant_kernel<<<(unsigned)((nbk + 255) / 256), 256, 0, st>>>(x, nbk, k / QK, k, xq, xd));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_matmul(const ceb_refmat& w, const float* x32, const int8_t* xq, const float* xd, int rows,
                   const int32_t* tile_group, const float* bias, int64_t bias_gstride, float* out, int ldo,
                   cudaStream_t st) {
    if (rows <= 0) return 0;
    const dim3 grid((unsigned)((w.n_out + MT - 1) / MT), (unsigned)((rows + MT - 1) / MT));
    if (grid.y > 65535u) return ceb_set_error(2, "reference matmul: %d rows exceed the grid", rows);
    const double flops = 2.0 * rows * w.n_out * w.k;
    if (w.type == CEB_GGML_Q8_0)
        CEB_LAUNCH(CEB_PROF_GEMM, st, flops, 0.0,
                   ref_matmul_q8_kernel<<<grid, 256, 0, st>>>(xq, xd, rows, w.k, w.q, w.d, w.n_out, tile_group, bias,
                                                              bias_gstride, out, ldo));
    else
        CEB_LAUNCH(CEB_PROF_GEMM, st, flops, 0.0,
                   ref_matmul_f32_kernel<<<grid, 256, 0, st>>>(x32, rows, w.k, w.f, w.n_out, tile_group, bias,
                                                               bias_gstride, out, ldo));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_attention(const float* qkv, const int32_t* cu, int n_seqs, int max_len, int d, int n_head, float* out,
                      cudaStream_t st) {
    if (d != n_head * HD) return ceb_set_error(2, "reference attention: head_dim must be %d", HD);
    if (n_seqs <= 0 || max_len <= 0) return 0;
    const dim3 grid((unsigned)((max_len + 63) / 64), (unsigned)n_head, (unsigned)n_seqs);
    CEB_LAUNCH(CEB_PROF_ATTN, st, 0.0, 0.0,
               ref_attention_kernel<<<grid, 64, 0, st>>>(qkv, cu, d, 1.0f / 8.0f, out));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_gelu(float* x, int64_t n, cudaStream_t st) {
    if (n <= 0) return 0;
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0, ref_gelu_kernel<<<grid_1d(n, 256), 256, 0, st>>>(x, n));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_route(const float* logits, int T, int E, int K, int32_t* ids, float* wts, cudaStream_t st) {
    if (T <= 0) return 0;
    if (E > 32) return ceb_set_error(2, "reference routing: %d experts (32 at most)", E);
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0,
               ref_route_kernel<<<(T + 127) / 128, 128, 0, st>>>(logits, T, E, K, ids, wts));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_group(const int32_t* ids, int T, int K, int E, int n_tiles_max, int32_t* pos, int32_t* src,
                  int32_t* tile_group, cudaStream_t st) {
    if (T <= 0) return 0;
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0,
               ref_group_kernel<<<1, 1024, 0, st>>>(ids, T, K, E, n_tiles_max, pos, src, tile_group));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_gather(const float* x, const int32_t* src, int64_t n_rows, int d, float* xp, cudaStream_t st) {
    if (n_rows <= 0) return 0;
    CEB_LAUNCH(CEB_PROF_ROUTE, st, 0.0, 0.0,
               ref_gather_kernel<<<grid_1d(n_rows * d, 256), 256, 0, st>>>(x, src, n_rows, d, xp));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_combine(const float* down, const int32_t* pos, const float* wts, int T, int K, int d, const float* bias,
                    float* y, cudaStream_t st) {
    if (T <= 0) return 0;
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               ref_combine_kernel<<<grid_1d((int64_t)T * d, 256), 256, 0, st>>>(down, pos, wts, T, K, d, bias, y));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ref_pool(const float* x, const int32_t* cu, int n_seqs, int d, int out_dim, float* out, cudaStream_t st) {
    if (n_seqs <= 0) return 0;
    if ((size_t)d * 4 > 48 * 1024) return ceb_set_error(2, "reference pooling: rows of %d values too wide", d);
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               ref_pool_kernel<<<n_seqs, 256, (size_t)d * 4, st>>>(x, cu, d, out_dim, out));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}
