// rowwise.cuh -- warp-per-row LayerNorm helpers shared by the encoder's row-wise
// kernels and the fused residual + LayerNorm + router kernel of the MoE block.
//
// A row of d <= 1024 floats is held by one warp as LN_MAXV float4 registers per
// lane: register i of lane l holds columns (i*32 + l)*4 .. +3.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace ceb_row {

constexpr int LN_MAXV = 8;  // float4 per lane: d <= 1024

CEB_DEV float wsum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

CEB_DEV float4 f4add(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// four consecutive values of a float or fp16 row as float4 (16- / 8-byte loads);
// ldg4 reads through the read-only path
CEB_DEV float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
CEB_DEV float4 ld4(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(u32_as_h2(u.x)), b = __half22float2(u32_as_h2(u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
CEB_DEV float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
CEB_DEV float4 ldg4(const __half* p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 a = __half22float2(u32_as_h2(u.x)), b = __half22float2(u32_as_h2(u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// LayerNorm of one row in place (v becomes the normalised row; the first nv of
// its N registers are used) and, where the pointers are set, its fp32 and fp16
// stores.  ggml_norm order
// (src/crispembed.cpp:1316-1323 via ggml_norm + ggml_mul + ggml_add): mean,
// centred values, variance of the centred values, scale = 1/sqrtf(var+eps),
// then *gamma and +beta as separate roundings.
template <int N>
CEB_DEV void ln_row(float4 (&v)[N], int nv, int d, const float* gamma, const float* beta, float eps,
                    float* out32, __half* out16, int lane) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (i < nv) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = wsum(s) / (float)d;
    float s2 = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (i < nv) {
            v[i].x = __fsub_rn(v[i].x, mean);
            v[i].y = __fsub_rn(v[i].y, mean);
            v[i].z = __fsub_rn(v[i].z, mean);
            v[i].w = __fsub_rn(v[i].w, mean);
            s2 += (__fmul_rn(v[i].x, v[i].x) + __fmul_rn(v[i].y, v[i].y)) +
                  (__fmul_rn(v[i].z, v[i].z) + __fmul_rn(v[i].w, v[i].w));
        }
    const float var = wsum(s2) / (float)d;
    const float scale = 1.0f / sqrtf(var + eps);
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (i < nv) {
            const int c = (i * 32 + lane) * 4;
            const float4 g = gamma ? *reinterpret_cast<const float4*>(gamma + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 b = beta ? *reinterpret_cast<const float4*>(beta + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 o;
            o.x = __fadd_rn(__fmul_rn(__fmul_rn(v[i].x, scale), g.x), b.x);
            o.y = __fadd_rn(__fmul_rn(__fmul_rn(v[i].y, scale), g.y), b.y);
            o.z = __fadd_rn(__fmul_rn(__fmul_rn(v[i].z, scale), g.z), b.z);
            o.w = __fadd_rn(__fmul_rn(__fmul_rn(v[i].w, scale), g.w), b.w);
            v[i] = o;
            if (out32) *reinterpret_cast<float4*>(out32 + c) = o;
            if (out16) {
                __half2* h = reinterpret_cast<__half2*>(out16 + c);
                h[0] = __floats2half2_rn(o.x, o.y);
                h[1] = __floats2half2_rn(o.z, o.w);
            }
        }
}

}  // namespace ceb_row
