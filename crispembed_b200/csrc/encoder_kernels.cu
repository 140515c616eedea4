// encoder_kernels.cu -- the row-wise and attention kernels around the MoE FFN:
// embedding gather + LayerNorm, residual add + LayerNorm (post-LN), the MoE
// combine fused with its residual + LayerNorm, varlen multi-head attention and
// the mean-pool + L2 epilogue.
//
// Reference: build_encoder_graph (src/crispembed.cpp:1068-1135 embeddings and
// embedding LN, :1278-1297 attention, :1316-1323 and :1423-1428 residual +
// post-LN) and encode_tokens' pooling (:1822-1846).
#include <cstdlib>

#include "ceb_encoder_internal.h"
#include "ceb_internal.h"
#include "common.cuh"
#include "rowwise.cuh"

namespace {

using ceb_row::LN_MAXV;
using ceb_row::f4add;
using ceb_row::wsum;

CEB_DEV int find_seq(const int32_t* cu, int n_seqs, int t) {
    int lo = 0, hi = n_seqs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// x = tok[id] + pos[t - start + pos_offset] (+ type[0]); LN(embd_ln)
__global__ void embed_ln_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int n_seqs, int M,
                                int d, int n_vocab, const float* __restrict__ tok, const float* __restrict__ pos,
                                int n_pos, int pos_offset, const float* __restrict__ type0,
                                const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                                float* __restrict__ out32, __half* __restrict__ out16, int* err) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const int t = warp;
    int id = ids[t];
    if (id < 0 || id >= n_vocab) {
        if (lane == 0) atomicCAS(err, 0, (int)CEB_DEVERR_BAD_INDEX);
        id = 0;
    }
    int p = 0;
    if (pos) {
        const int s = find_seq(cu, n_seqs, t);
        p = t - cu[s] + pos_offset;
        if (p < 0 || p >= n_pos) {
            if (lane == 0) atomicCAS(err, 0, (int)CEB_DEVERR_BAD_INDEX);
            p = 0;
        }
    }
    const int nv = d / 128;
    float4 v[LN_MAXV];
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i)
        if (i < nv) {
            const int c = (i * 32 + lane) * 4;
            float4 x = __ldg(reinterpret_cast<const float4*>(tok + (size_t)id * d + c));
            if (pos) x = f4add(x, __ldg(reinterpret_cast<const float4*>(pos + (size_t)p * d + c)));
            if (type0) x = f4add(x, __ldg(reinterpret_cast<const float4*>(type0 + c)));
            v[i] = x;
        }
    if (gamma) {
        ceb_row::ln_row(v, nv, d, gamma, beta, eps, out32 + (size_t)t * d, out16 + (size_t)t * d, lane);
    } else {
#pragma unroll
        for (int i = 0; i < LN_MAXV; ++i)
            if (i < nv) {
                const int c = (i * 32 + lane) * 4;
                *reinterpret_cast<float4*>(out32 + (size_t)t * d + c) = v[i];
                __half2* h = reinterpret_cast<__half2*>(out16 + (size_t)t * d + c);
                h[0] = __floats2half2_rn(v[i].x, v[i].y);
                h[1] = __floats2half2_rn(v[i].z, v[i].w);
            }
    }
}

// out = LN(res + y)   (out32 may alias res); y fp16 (the GEMM outputs) or float
template <typename TY>
__global__ void add_ln_kernel(const float* res, const TY* __restrict__ y, int M, int d,
                              const float* __restrict__ gamma, const float* __restrict__ beta, float eps, float* out32,
                              __half* __restrict__ out16) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= M) return;
    const int nv = d / 128;
    float4 v[LN_MAXV];
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i)
        if (i < nv) {
            const int c = (i * 32 + lane) * 4;
            v[i] = f4add(*reinterpret_cast<const float4*>(res + (size_t)t * d + c), ceb_row::ld4(y + (size_t)t * d + c));
        }
    __syncwarp();
    ceb_row::ln_row(v, nv, d, gamma, beta, eps, out32 + (size_t)t * d, out16 + (size_t)t * d, lane);
}

// ffn = sum_j w_j * down[pos_j] (fmaf in slot order) + moe_bias; out = LN(cur + ffn).
// down: the fp16 expert rows written by the fc2 GEMM.
// NV = d / 128 float4 registers per lane; the residual row and two slots' expert rows
// are requested together so a warp has three rows of loads in flight.
template <int NV>
__global__ void moe_combine_ln_kernel(const __half* __restrict__ down, const int32_t* __restrict__ slot_pos,
                                      const float* __restrict__ wts, int K, const float* __restrict__ moe_bias,
                                      const float* cur, int M, const float* __restrict__ gamma,
                                      const float* __restrict__ beta, float eps, float* out32,
                                      __half* __restrict__ out16) {
    constexpr int d = NV * 128;
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= M) return;
    float4 acc[NV], res[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        res[i] = *reinterpret_cast<const float4*>(cur + (size_t)t * d + (i * 32 + lane) * 4);
    }
    int jj = 0;
    for (; jj + 1 < K; jj += 2) {  // two slots' rows per pass, accumulated in slot order
        const int p0 = slot_pos[(size_t)t * K + jj], p1 = slot_pos[(size_t)t * K + jj + 1];
        const float w0 = wts[(size_t)t * K + jj], w1 = wts[(size_t)t * K + jj + 1];
        float4 d0[NV], d1[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = (i * 32 + lane) * 4;
            d0[i] = ceb_row::ldg4(down + (size_t)p0 * d + c);
            d1[i] = ceb_row::ldg4(down + (size_t)p1 * d + c);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            acc[i].x = __fmaf_rn(w1, d1[i].x, __fmaf_rn(w0, d0[i].x, acc[i].x));
            acc[i].y = __fmaf_rn(w1, d1[i].y, __fmaf_rn(w0, d0[i].y, acc[i].y));
            acc[i].z = __fmaf_rn(w1, d1[i].z, __fmaf_rn(w0, d0[i].z, acc[i].z));
            acc[i].w = __fmaf_rn(w1, d1[i].w, __fmaf_rn(w0, d0[i].w, acc[i].w));
        }
    }
    for (; jj < K; ++jj) {
        const int p = slot_pos[(size_t)t * K + jj];
        const float w = wts[(size_t)t * K + jj];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float4 dv = ceb_row::ldg4(down + (size_t)p * d + (i * 32 + lane) * 4);
            acc[i].x = __fmaf_rn(w, dv.x, acc[i].x);
            acc[i].y = __fmaf_rn(w, dv.y, acc[i].y);
            acc[i].z = __fmaf_rn(w, dv.z, acc[i].z);
            acc[i].w = __fmaf_rn(w, dv.w, acc[i].w);
        }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = (i * 32 + lane) * 4;
        if (moe_bias) acc[i] = f4add(acc[i], *reinterpret_cast<const float4*>(moe_bias + c));
        acc[i] = f4add(res[i], acc[i]);
    }
    __syncwarp();
    ceb_row::ln_row(acc, NV, d, gamma, beta, eps, out32 + (size_t)t * d, out16 + (size_t)t * d, lane);
}

// ------------------------------------------------------------------ RoPE
// One CTA per token, thread = (head, pair i < 32): dims i and i + 32 of the head's
// Q and K rotate by pos * theta^(-2i/64) (NEOX pairing, ggml_rope_ext with n_dims =
// head_dim, no frequency scaling), in fp32, stored back as fp16.
__global__ void rope_neox_kernel(__half* __restrict__ qkv, const int32_t* __restrict__ cu, int n_seqs, int d,
                                 int pos_offset, float log2_theta) {
    const int t = blockIdx.x;
    const int seq = find_seq(cu, n_seqs, t);
    const float pos = (float)(t - cu[seq] + pos_offset);
    const int h = threadIdx.x >> 5, i = threadIdx.x & 31;
    const float ang = pos * exp2f(-(float)(2 * i) / 64.0f * log2_theta);
    float sn, cs;
    sincosf(ang, &sn, &cs);
#pragma unroll
    for (int part = 0; part < 2; ++part) {  // Q, then K
        __half* base = qkv + (size_t)t * 3 * d + part * d + h * 64;
        const float x0 = __half2float(base[i]), x1 = __half2float(base[i + 32]);
        base[i] = __float2half_rn(x0 * cs - x1 * sn);
        base[i + 32] = __float2half_rn(x0 * sn + x1 * cs);
    }
}

// ------------------------------------------------------------------ attention
// S = Q K^T and O = P V on mma.sync m16n8k16 (fp16 in, fp32 accumulate) with a
// one-pass online softmax over the keys; keys beyond the sequence are masked.
constexpr int AT_NW = 4;                                    // warps per CTA, 32 query rows each
constexpr int AT_Q = 32 * AT_NW, AT_K = 64, AT_HD = 64, AT_LD = 72;  // padded smem row (halfs)

CEB_DEV float ex2_approx(float x) {  // MUFU 2^x (ex2(-inf) = 0)
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// 2^t for two exponents: the pair rounded to fp16 (one conversion), then one MUFU
// op for both; the result is the packed fp16 pair the P V product consumes.
CEB_DEV uint32_t ex2_h2(float t0, float t1) {
    uint32_t in = h2_as_u32(__floats2half2_rn(t0, t1)), r;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(in));
    return r;
}

CEB_DEV void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
CEB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CEB_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
CEB_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
CEB_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
CEB_DEV void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, "
        "%2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Rows of one tile (ROWS x 64 fp16, rows beyond n_valid zero-filled) by NT threads.
template <int NT, int ROWS>
CEB_DEV void load_rows(__half* s, const __half* g, size_t g_ld, int n_valid, int tid) {
    static_assert((ROWS * 8) % NT == 0, "16-byte chunks per thread");
#pragma unroll
    for (int i = 0; i < ROWS * 8 / NT; ++i) {
        const int chunk = tid + i * NT;
        const int row = chunk >> 3, col = (chunk & 7) * 8;
        const bool ok = row < n_valid;
        const __half* src = g + (size_t)(ok ? row : 0) * g_ld + col;
        cp_async16(smem_u32(s + row * AT_LD + col), src, ok ? 16 : 0);
    }
}

// One CTA = AT_Q queries of one (sequence, head); each warp owns 32 query rows as
// two m16 tiles, so every K / V fragment read from shared memory feeds two MMAs
// (two independent MMA chains per warp).  Keys in 64-key tiles (cp.async,
// double-buffered), processed in 32-key steps; a step wholly past the sequence's
// end is skipped.  Q is staged in the second buffer's space and moved to registers
// before the first prefetch lands there.  168 registers: 3 CTAs per SM.
__global__ void __launch_bounds__(AT_NW * 32, 3) attention_kernel(const __half* __restrict__ qkv,
                                                                  const int32_t* __restrict__ cu, int d,
                                                                  float scale_log2, __half* __restrict__ out,
                                                                  int total_rows, int max_len, int* __restrict__ err) {
    constexpr int NT = AT_NW * 32, QT = AT_Q, TILE = AT_K * AT_LD;
    static_assert(QT <= 2 * AT_K, "Q staging uses the second K and V buffers");
    __shared__ __align__(128) __half sm[4 * TILE];  // K0, V0, K1, V1
    const int seq = blockIdx.z, head = blockIdx.y;
    const int start = cu[seq], len = cu[seq + 1] - start;
    if (start < 0 || len < 0 || len > total_rows - start || len > max_len) {
        if (blockIdx.x == 0 && head == 0 && threadIdx.x == 0 && err) atomicCAS(err, 0, (int)CEB_DEVERR_BAD_INDEX);
        return;
    }
    const int q0 = blockIdx.x * QT;
    if (q0 >= len) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t ld = (size_t)3 * d;
    const __half* Qg = qkv + (size_t)(start + q0) * ld + head * AT_HD;
    const __half* Kg = qkv + (size_t)start * ld + d + head * AT_HD;
    const __half* Vg = qkv + (size_t)start * ld + 2 * d + head * AT_HD;
    const int nq = min(QT, len - q0);
    const int n_kt = (len + AT_K - 1) / AT_K;
    const bool active = warp * 32 < nq;  // warp-uniform: this warp holds a valid query row
    __half* const sQ = sm + 2 * TILE;

    load_rows<NT, QT>(sQ, Qg, ld, nq, tid);
    load_rows<NT, AT_K>(sm, Kg, ld, min(AT_K, len), tid);
    load_rows<NT, AT_K>(sm + TILE, Vg, ld, min(AT_K, len), tid);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    uint32_t qf[2][4][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const int row = warp * 32 + m * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
            const int col = ks * 16 + 8 * (lane >> 4);
            ldsm_x4(smem_u32(sQ + row * AT_LD + col), qf[m][ks][0], qf[m][ks][1], qf[m][ks][2], qf[m][ks][3]);
        }
    __syncthreads();  // the second buffer is free for the first prefetch

    float o[2][8][4];
    float o_sum[2][4];
    float m_r[2][2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[m][i][0] = o[m][i][1] = o[m][i][2] = o[m][i][3] = 0.0f;
        o_sum[m][0] = o_sum[m][1] = o_sum[m][2] = o_sum[m][3] = 0.0f;
        m_r[m][0] = m_r[m][1] = -INFINITY;
    }
    const int tq = lane & 3;

    for (int kt = 0; kt < n_kt; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < n_kt) {
            const int k0n = (kt + 1) * AT_K;
            load_rows<NT, AT_K>(sm + (2 * (buf ^ 1)) * TILE, Kg + (size_t)k0n * ld, ld, min(AT_K, len - k0n), tid);
            load_rows<NT, AT_K>(sm + (2 * (buf ^ 1) + 1) * TILE, Vg + (size_t)k0n * ld, ld, min(AT_K, len - k0n), tid);
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const __half* sK = sm + (2 * buf) * TILE;
        const __half* sV = sm + (2 * buf + 1) * TILE;
        if (active) {
            for (int h = 0; h < 2; ++h) {
                const int kbase = kt * AT_K + 32 * h;
                if (kbase >= len) break;
                // S = Q K^T for 32 keys: 4 n-tiles of 8 keys, both m-tiles per K fragment
                float s[2][4][4];
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int j = 0; j < 4; ++j) s[m][j][0] = s[m][j][1] = s[m][j][2] = s[m][j][3] = 0.0f;
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
                    for (int jp = 0; jp < 2; ++jp) {
                        const int key = 32 * h + jp * 16 + (lane & 7) + 8 * (lane >> 4);
                        const int col = ks * 16 + 8 * ((lane >> 3) & 1);
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(smem_u32(sK + key * AT_LD + col), b0, b1, b2, b3);
#pragma unroll
                        for (int m = 0; m < 2; ++m) {
                            mma16816(s[m][2 * jp], qf[m][ks], b0, b1);
                            mma16816(s[m][2 * jp + 1], qf[m][ks], b2, b3);
                        }
                    }
                }
                if (kbase + 32 > len) {
#pragma unroll
                    for (int m = 0; m < 2; ++m)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (kbase + j * 8 + 2 * tq + (e & 1) >= len) s[m][j][e] = -INFINITY;
                }
                uint32_t pf[2][2][4];
                float corr[2][2];
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    float mx[2] = {m_r[m][0], m_r[m][1]};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        mx[0] = fmaxf(mx[0], fmaxf(s[m][j][0], s[m][j][1]));
                        mx[1] = fmaxf(mx[1], fmaxf(s[m][j][2], s[m][j][3]));
                    }
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                    }
                    float nm[2];
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        nm[r] = -mx[r] * scale_log2;
                        corr[m][r] = ex2_approx(fmaf(m_r[m][r], scale_log2, nm[r]));
                        m_r[m][r] = mx[r];
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int kk = j >> 1, hi = j & 1;
                        pf[m][kk][hi * 2 + 0] =
                            ex2_h2(fmaf(s[m][j][0], scale_log2, nm[0]), fmaf(s[m][j][1], scale_log2, nm[0]));
                        pf[m][kk][hi * 2 + 1] =
                            ex2_h2(fmaf(s[m][j][2], scale_log2, nm[1]), fmaf(s[m][j][3], scale_log2, nm[1]));
                    }
                }
                if (__any_sync(0xffffffffu, corr[0][0] != 1.0f || corr[0][1] != 1.0f || corr[1][0] != 1.0f ||
                                                corr[1][1] != 1.0f)) {
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            o[m][i][0] *= corr[m][0];
                            o[m][i][1] *= corr[m][0];
                            o[m][i][2] *= corr[m][1];
                            o[m][i][3] *= corr[m][1];
                        }
                        o_sum[m][0] *= corr[m][0];
                        o_sum[m][1] *= corr[m][0];
                        o_sum[m][2] *= corr[m][1];
                        o_sum[m][3] *= corr[m][1];
                    }
                }
                // O += P V over the 32 keys, both m-tiles per V fragment; row sums from P x ones
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
                    for (int m = 0; m < 2; ++m) mma16816(o_sum[m], pf[m][kk], 0x3C003C00u, 0x3C003C00u);
#pragma unroll
                    for (int np = 0; np < 4; ++np) {
                        const int key = 32 * h + kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                        const int col = np * 16 + 8 * (lane >> 4);
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_t(smem_u32(sV + key * AT_LD + col), b0, b1, b2, b3);
#pragma unroll
                        for (int m = 0; m < 2; ++m) {
                            mma16816(o[m][2 * np], pf[m][kk], b0, b1);
                            mma16816(o[m][2 * np + 1], pf[m][kk], b2, b3);
                        }
                    }
                }
            }
        }
        __syncthreads();
    }
    if (!active) return;
    const int g = lane >> 2;
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int q = q0 + warp * 32 + m * 16 + g + 8 * r;
            if (q >= len) continue;
            const float l = o_sum[m][2 * r];
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            __half* dst = out + (size_t)(start + q) * d + head * AT_HD;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int col = i * 8 + 2 * tq;
                *reinterpret_cast<__half2*>(dst + col) =
                    __floats2half2_rn(o[m][i][2 * r] * inv, o[m][i][2 * r + 1] * inv);
            }
        }
}

// ------------------------------------------------------------------ pooling
// One CTA per sequence: mean over rows (row-parallel partial sums reduced in a
// fixed order, so results are identical run to run), then L2 over out_dim.
// mode 0 = mean over the sequence's rows, 1 = first row ([CLS]), 2 = last row.
__global__ void pool_l2_kernel(const float* __restrict__ hidden, const int32_t* __restrict__ cu, int d, int out_dim,
                               float* __restrict__ out, int mode) {
    extern __shared__ float sp[];  // [d] pooled + [32] scratch
    const int s = blockIdx.x;
    const int r0 = cu[s], n = cu[s + 1] - cu[s];
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        if (mode == 0) {
            float acc = 0.0f;
            for (int t = 0; t < n; ++t) acc += hidden[(size_t)(r0 + t) * d + c];
            sp[c] = n > 0 ? acc / (float)n : 0.0f;
        } else {
            sp[c] = n > 0 ? hidden[(size_t)(mode == 1 ? r0 : r0 + n - 1) * d + c] : 0.0f;
        }
    }
    __syncthreads();
    float part = 0.0f;
    for (int c = threadIdx.x; c < out_dim; c += blockDim.x) part += sp[c] * sp[c];
    part = wsum(part);
    float* red = sp + d;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        red[31] = sqrtf(fmaxf(tot, 1e-12f));
    }
    __syncthreads();
    const float norm = red[31];
    for (int c = threadIdx.x; c < out_dim; c += blockDim.x) out[(size_t)s * out_dim + c] = sp[c] / norm;
}

// Mean pool + L2 for mode 0, one cluster of POOL_SPLIT CTAs per sequence: CTA x sums
// the sequence's 8-row blocks x, x + POOL_SPLIT, ... (float4 columns, the block's rows
// loaded together, added in row order), the cluster's rank 0 then adds the partials of
// ranks 0..POOL_SPLIT-1 in rank order from their shared memory, divides by the row
// count and normalises.  Fixed orders: results identical run to run and independent
// of the rest of the batch.  d / 4 threads (one float4 column each).
constexpr int POOL_SPLIT = 8, POOL_ROWS = 8;
__global__ void __cluster_dims__(POOL_SPLIT, 1, 1) pool_mean_cluster_kernel(const float* __restrict__ hidden,
                                                                            const int32_t* __restrict__ cu, int d,
                                                                            int out_dim, float* __restrict__ out) {
    extern __shared__ float4 pp[];  // [d/4] partial + [32] scratch
    const int s = blockIdx.y;
    const uint32_t x = cluster_ctarank();
    const int r0 = cu[s], n = cu[s + 1] - cu[s];
    const int c4 = threadIdx.x, nc4 = d >> 2;
    const float4* h = reinterpret_cast<const float4*>(hidden) + (size_t)r0 * nc4 + c4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = (int)x * POOL_ROWS; b < n; b += POOL_SPLIT * POOL_ROWS) {
        float4 v[POOL_ROWS];
#pragma unroll
        for (int i = 0; i < POOL_ROWS; ++i)
            v[i] = b + i < n ? __ldcs(h + (size_t)(b + i) * nc4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < POOL_ROWS; ++i) {
            acc.x += v[i].x;
            acc.y += v[i].y;
            acc.z += v[i].z;
            acc.w += v[i].w;
        }
    }
    pp[c4] = acc;
    cluster_sync();  // every partial written
    if (x == 0) {
        float4 t = acc;
        for (uint32_t r = 1; r < POOL_SPLIT; ++r) {
            const uint32_t a = mapa_shared(smem_u32(&pp[c4]), r);
            float4 q;
            asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(q.x), "=f"(q.y), "=f"(q.z), "=f"(q.w)
                         : "r"(a));
            t.x += q.x;
            t.y += q.y;
            t.z += q.z;
            t.w += q.w;
        }
        const float inv_n = 1.0f / (float)(n > 0 ? n : 1);
        t = n > 0 ? make_float4(t.x * inv_n, t.y * inv_n, t.z * inv_n, t.w * inv_n) : make_float4(0.f, 0.f, 0.f, 0.f);
        float part = 0.0f;
        const int base = 4 * c4;
        if (base < out_dim) part += t.x * t.x;
        if (base + 1 < out_dim) part += t.y * t.y;
        if (base + 2 < out_dim) part += t.z * t.z;
        if (base + 3 < out_dim) part += t.w * t.w;
        part = wsum(part);
        float* red = reinterpret_cast<float*>(pp + nc4);
        __syncthreads();  // rank 0 only: all its threads take this branch
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x == 0) {
            float tot = 0.0f;
            for (int w = 0; w < (int)((blockDim.x + 31) >> 5); ++w) tot += red[w];
            red[31] = sqrtf(fmaxf(tot, 1e-12f));
        }
        __syncthreads();
        const float norm = red[31];
        float* o = out + (size_t)s * out_dim + base;
        if (base < out_dim) o[0] = t.x / norm;
        if (base + 1 < out_dim) o[1] = t.y / norm;
        if (base + 2 < out_dim) o[2] = t.z / norm;
        if (base + 3 < out_dim) o[3] = t.w / norm;
    }
    cluster_sync();  // rank 0 has read every partial before any CTA of the cluster exits
}

}  // namespace

int ceb_embed_ln(const int32_t* ids, const int32_t* cu, int n_seqs, int M, int d, int n_vocab, const float* tok,
                 const float* pos, int n_pos, int pos_offset, const float* type0, const float* gamma,
                 const float* beta, float eps, float* out32, __half* out16, int* err, cudaStream_t st) {
    if (d % 128 || d > 128 * LN_MAXV) return ceb_set_error(2, "embed: d=%d unsupported", d);
    const int threads = 256, per = threads / 32;
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0, embed_ln_kernel<<<(M + per - 1) / per, threads, 0, st>>>(ids, cu, n_seqs, M, d, n_vocab, tok, pos, n_pos,
                                                             pos_offset, type0, gamma, beta, eps, out32, out16, err));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_rope_neox(__half* qkv, int M, const int32_t* cu, int n_seqs, int d, int n_head, int pos_offset, float theta,
                  cudaStream_t st) {
    if (d != n_head * 64 || n_head > 32) return ceb_set_error(2, "rope: head_dim 64 and <= 32 heads supported");
    if (M <= 0) return 0;
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               rope_neox_kernel<<<M, 32 * n_head, 0, st>>>(qkv, cu, n_seqs, d, pos_offset, log2f(theta)));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_add_ln(const float* res, const __half* y, int M, int d, const float* gamma, const float* beta, float eps,
               float* out32, __half* out16, cudaStream_t st) {
    if (d % 128 || d > 128 * LN_MAXV) return ceb_set_error(2, "add_ln: d=%d unsupported", d);
    const int threads = 256, per = threads / 32;
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
               add_ln_kernel<__half><<<(M + per - 1) / per, threads, 0, st>>>(res, y, M, d, gamma, beta, eps, out32,
                                                                             out16));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_moe_combine_ln(const __half* down, const int32_t* slot_pos, const float* wts, int K, const float* moe_bias,
                       const float* cur, int M, int d, const float* gamma, const float* beta, float eps, float* out32,
                       __half* out16, cudaStream_t st) {
    if (d % 128 || d > 128 * LN_MAXV) return ceb_set_error(2, "combine: d=%d unsupported", d);
    const int threads = 128, per = threads / 32, grid = (M + per - 1) / per;  // small CTAs: ~88 registers a thread
#define CEB_COMBINE_CASE(NVC)                                                                                    \
    case NVC:                                                                                                   \
        CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,                                                              \
                   moe_combine_ln_kernel<NVC><<<grid, threads, 0, st>>>(down, slot_pos, wts, K, moe_bias, cur, M, \
                                                                       gamma, beta, eps, out32, out16));        \
        break;
    switch (d / 128) {
        CEB_COMBINE_CASE(1)
        CEB_COMBINE_CASE(2)
        CEB_COMBINE_CASE(3)
        CEB_COMBINE_CASE(4)
        CEB_COMBINE_CASE(5)
        CEB_COMBINE_CASE(6)
        CEB_COMBINE_CASE(7)
        CEB_COMBINE_CASE(8)
    }
#undef CEB_COMBINE_CASE
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_attention(const __half* qkv, int total_rows, const int32_t* cu, int n_seqs, int max_len, int d, int n_head,
                  __half* out, int* d_err, cudaStream_t st, int* sched) {
    if (n_head <= 0 || d % n_head || d / n_head != AT_HD)
        return ceb_set_error(2, "attention: head_dim %d unsupported (64 only)", n_head > 0 ? d / n_head : -1);
    if (n_seqs <= 0 || max_len <= 0) return 0;
    // Default: the single-CTA tcgen05 kernel (attn_fa.cu); on the benchmark batch (256
    // sequences, 32..512 tokens, 12 heads) 0.253 ms per layer against 0.358 ms for the
    // mma.sync kernel below, which remains for operands the tensor maps cannot take and
    // for callers without a work-item counter.  CEB_ATTN_MMA=1 forces the mma.sync kernel;
    // CEB_ATTN_TC=1 selects the CTA-pair tcgen05 kernel (attn_tc.cu, sequences of up to 512
    // tokens; 0.391-0.395 ms on the same batch).
    const char* tc = getenv("CEB_ATTN_TC");
    if (tc && tc[0] == '1') {
        const int rc = ceb_attention_tc(qkv, total_rows, cu, n_seqs, max_len, d, n_head, out, d_err, st);
        if (rc != 1) return rc;  // launched (0) or failed
    }
    const char* mma = getenv("CEB_ATTN_MMA");
    if (!(mma && mma[0] == '1') && sched) {
        const int rc = ceb_attention_fa(qkv, total_rows, cu, n_seqs, max_len, d, n_head, out, d_err, st, sched);
        if (rc != 1) return rc;
    }
    const float scale_log2 = (1.0f / sqrtf((float)AT_HD)) * 1.4426950408889634f;
    dim3 grid((max_len + AT_Q - 1) / AT_Q, n_head, n_seqs);
    CEB_LAUNCH(CEB_PROF_ATTN, st, 0.0, 0.0, attention_kernel<<<grid, AT_NW * 32, 0, st>>>(qkv, cu, d, scale_log2, out, total_rows, max_len,
                                                                             d_err));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_pool_l2_launch(const float* hidden, const int32_t* cu, int n_seqs, int d, int out_dim, float* out,
                       cudaStream_t st, int mode) {
    if (n_seqs <= 0) return 0;
    if (out_dim <= 0 || out_dim > d) return ceb_set_error(1, "pool: out_dim %d outside (0, %d]", out_dim, d);
    if (mode == 0 && d % 128 == 0 && d <= 4096 && (reinterpret_cast<uintptr_t>(hidden) & 15) == 0) {
        const size_t smem = (size_t)d * sizeof(float) + 32 * sizeof(float4);
        CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0,
                   pool_mean_cluster_kernel<<<dim3(POOL_SPLIT, n_seqs), d / 4, smem, st>>>(hidden, cu, d, out_dim,
                                                                                            out));
        CEB_CUDA_OK(cudaGetLastError());
        return 0;
    }
    const size_t smem = (size_t)(d + 32) * sizeof(float);
    CEB_LAUNCH(CEB_PROF_ROWWISE, st, 0.0, 0.0, pool_l2_kernel<<<n_seqs, 256, smem, st>>>(hidden, cu, d, out_dim, out, mode));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}
