// gguf_quants.cpp -- host decoding of GGUF/ggml block formats for weights that the
// device GEMM does not read in their stored form.
//
// The reference loads whatever ggml can read; GGUFs met in practice beside its own
// converter's F32/F16/Q8_0 output (models/convert-bert-to-gguf.py:68-77) are the
// llama.cpp community exports (Q4_K_M = Q4_K + Q6_K, Q5_K_M = Q5_K + Q6_K, legacy
// Q4_0/Q4_1/Q5_0/Q5_1, BF16) and the registry's IQ4_XS files
// (examples/cli/model_mgr.cpp:728-743).  The block layouts below are ggml's
// published formats (they have to be bit-compatible to read the files); each
// decoder is checked against gguf-py's dequantizer in tests/test_formats.py.
//
// How the library uses them:
//   * Q8_0, Q4_K            stay in their own form; the GEMM dequantizes them in
//                           shared memory (runtime.cpp, gemm_tc.cu).
//   * IQ4_NL, IQ4_XS        become Q8_0-form blocks: the 4-bit index's codebook
//                           value is an int8 and the 32-value block scale an fp16
//                           (IQ4_XS: d * (ls - 32) rounded to fp16), so the Q8_0
//                           GEMM path runs them.
//   * the other formats     are decoded to fp32 here and stored as fp16 planes.
//   * float tables (token / position embeddings) of any listed type are decoded
//     to fp32.
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>

#include "ceb_internal.h"

namespace {

inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
inline float h2f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}
inline float bf2f(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// 6-bit scale / min of sub-block j of a Q4_K / Q5_K super-block
inline void k4_scale_min(int j, const uint8_t* s, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// IQ4_NL / IQ4_XS non-linear codebook (ggml's kvalues_iq4nl)
constexpr int8_t kIq4[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

struct Fmt {
    int block;  // values per block
    int bytes;  // bytes per block
};

bool fmt_of(int type, Fmt* f) {
    switch (type) {
        case CEB_GGML_F32: *f = {1, 4}; return true;
        case CEB_GGML_F16: *f = {1, 2}; return true;
        case CEB_GGML_BF16: *f = {1, 2}; return true;
        case CEB_GGML_Q4_0: *f = {32, 18}; return true;
        case CEB_GGML_Q4_1: *f = {32, 20}; return true;
        case CEB_GGML_Q5_0: *f = {32, 22}; return true;
        case CEB_GGML_Q5_1: *f = {32, 24}; return true;
        case CEB_GGML_Q8_0: *f = {32, 34}; return true;
        case CEB_GGML_Q4_K: *f = {256, 144}; return true;
        case CEB_GGML_Q5_K: *f = {256, 176}; return true;
        case CEB_GGML_Q6_K: *f = {256, 210}; return true;
        case CEB_GGML_IQ4_NL: *f = {32, 18}; return true;
        case CEB_GGML_IQ4_XS: *f = {256, 136}; return true;
    }
    return false;
}

// the 32 values of a Q4_0/Q4_1/Q5_0/Q5_1/IQ4_NL block: element j < 16 from the low
// nibble of byte j, element j + 16 from its high nibble
void dequant_32(int type, const uint8_t* b, float* y) {
    const float d = h2f(rd16(b));
    switch (type) {
        case CEB_GGML_Q4_0:
            for (int j = 0; j < 16; ++j) {
                y[j] = d * (float)((b[2 + j] & 0xF) - 8);
                y[j + 16] = d * (float)((b[2 + j] >> 4) - 8);
            }
            break;
        case CEB_GGML_Q4_1: {
            const float m = h2f(rd16(b + 2));
            for (int j = 0; j < 16; ++j) {
                y[j] = d * (float)(b[4 + j] & 0xF) + m;
                y[j + 16] = d * (float)(b[4 + j] >> 4) + m;
            }
            break;
        }
        case CEB_GGML_Q5_0: {
            uint32_t qh;
            memcpy(&qh, b + 2, 4);
            for (int j = 0; j < 16; ++j) {
                const int h0 = ((qh >> j) & 1) << 4, h1 = ((qh >> (j + 16)) & 1) << 4;
                y[j] = d * (float)(((b[6 + j] & 0xF) | h0) - 16);
                y[j + 16] = d * (float)(((b[6 + j] >> 4) | h1) - 16);
            }
            break;
        }
        case CEB_GGML_Q5_1: {
            const float m = h2f(rd16(b + 2));
            uint32_t qh;
            memcpy(&qh, b + 4, 4);
            for (int j = 0; j < 16; ++j) {
                const int h0 = ((qh >> j) & 1) << 4, h1 = ((qh >> (j + 16)) & 1) << 4;
                y[j] = d * (float)((b[8 + j] & 0xF) | h0) + m;
                y[j + 16] = d * (float)((b[8 + j] >> 4) | h1) + m;
            }
            break;
        }
        case CEB_GGML_IQ4_NL:
            for (int j = 0; j < 16; ++j) {
                y[j] = d * (float)kIq4[b[2 + j] & 0xF];
                y[j + 16] = d * (float)kIq4[b[2 + j] >> 4];
            }
            break;
    }
}

void dequant_q4k(const uint8_t* b, float* y) {
    const float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    const uint8_t* qs = b + 16;
    for (int c = 0; c < 4; ++c) {  // 64 values per chunk: low nibbles, then high nibbles
        int s0, m0, s1, m1;
        k4_scale_min(2 * c, b + 4, &s0, &m0);
        k4_scale_min(2 * c + 1, b + 4, &s1, &m1);
        const float d1 = d * (float)s0, mm1 = dmin * (float)m0, d2 = d * (float)s1, mm2 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) y[64 * c + l] = d1 * (float)(qs[32 * c + l] & 0xF) - mm1;
        for (int l = 0; l < 32; ++l) y[64 * c + 32 + l] = d2 * (float)(qs[32 * c + l] >> 4) - mm2;
    }
}

// Q5_K: d, dmin, 12 bytes of 6-bit scales/mins, qh[32] (bit 2c / 2c+1 of byte l =
// fifth bit of value l of chunk c's low / high half), qs[128]
void dequant_q5k(const uint8_t* b, float* y) {
    const float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    const uint8_t *qh = b + 16, *qs = b + 48;
    for (int c = 0; c < 4; ++c) {
        int s0, m0, s1, m1;
        k4_scale_min(2 * c, b + 4, &s0, &m0);
        k4_scale_min(2 * c + 1, b + 4, &s1, &m1);
        const float d1 = d * (float)s0, mm1 = dmin * (float)m0, d2 = d * (float)s1, mm2 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) {
            const int lo = (qs[32 * c + l] & 0xF) | (((qh[l] >> (2 * c)) & 1) << 4);
            const int hi = (qs[32 * c + l] >> 4) | (((qh[l] >> (2 * c + 1)) & 1) << 4);
            y[64 * c + l] = d1 * (float)lo - mm1;
            y[64 * c + 32 + l] = d2 * (float)hi - mm2;
        }
    }
}

// Q6_K: ql[128] low 4 bits, qh[64] high 2 bits, int8 scales[16] (one per 16 values),
// fp16 d at the end; two halves of 128 values, each four runs of 32
void dequant_q6k(const uint8_t* b, float* y) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
    const float d = h2f(rd16(b + 208));
    for (int n = 0; n < 2; ++n) {
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[l] = d * (float)sc[is] * (float)q1;
            y[l + 32] = d * (float)sc[is + 2] * (float)q2;
            y[l + 64] = d * (float)sc[is + 4] * (float)q3;
            y[l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
        y += 128;
        ql += 64;
        qh += 32;
        sc += 8;
    }
}

// IQ4_XS: fp16 d, scales_h (2 high bits per sub-block), scales_l[4] (4 low bits per
// sub-block), qs[128]; sub-block scale d * (ls - 32), codebook values
inline int iq4xs_ls(const uint8_t* b, int ib) {
    const uint16_t sh = rd16(b + 2);
    return ((b[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
}
void dequant_iq4xs(const uint8_t* b, float* y) {
    const float d = h2f(rd16(b));
    const uint8_t* qs = b + 8;
    for (int ib = 0; ib < 8; ++ib) {
        const float dl = d * (float)(iq4xs_ls(b, ib) - 32);
        for (int j = 0; j < 16; ++j) {
            y[32 * ib + j] = dl * (float)kIq4[qs[16 * ib + j] & 0xF];
            y[32 * ib + j + 16] = dl * (float)kIq4[qs[16 * ib + j] >> 4];
        }
    }
}

}  // namespace

int64_t ceb_ggml_row_bytes(int type, int64_t k) {
    Fmt f;
    if (!fmt_of(type, &f) || k % f.block) return -1;
    return k / f.block * f.bytes;
}

bool ceb_ggml_dequant_row(int type, const uint8_t* src, int64_t k, float* dst) {
    Fmt f;
    if (!fmt_of(type, &f) || k % f.block) return false;
    const int64_t nb = k / f.block;
    for (int64_t i = 0; i < nb; ++i) {
        const uint8_t* b = src + i * f.bytes;
        float* y = dst + i * f.block;
        switch (type) {
            case CEB_GGML_F32: memcpy(y, b, 4); break;
            case CEB_GGML_F16: *y = h2f(rd16(b)); break;
            case CEB_GGML_BF16: *y = bf2f(rd16(b)); break;
            case CEB_GGML_Q8_0: {
                const float d = h2f(rd16(b));
                for (int j = 0; j < 32; ++j) y[j] = d * (float)(int8_t)b[2 + j];
                break;
            }
            case CEB_GGML_Q4_K: dequant_q4k(b, y); break;
            case CEB_GGML_Q5_K: dequant_q5k(b, y); break;
            case CEB_GGML_Q6_K: dequant_q6k(b, y); break;
            case CEB_GGML_IQ4_XS: dequant_iq4xs(b, y); break;
            default: dequant_32(type, b, y); break;
        }
    }
    return true;
}

bool ceb_ggml_as_q8_0_blocks(int type, const uint8_t* src, int64_t k, uint8_t* dst) {
    if (k % 32) return false;
    if (type == CEB_GGML_Q8_0) {
        memcpy(dst, src, (size_t)(k / 32) * 34);
        return true;
    }
    if (type == CEB_GGML_IQ4_NL) {
        for (int64_t i = 0; i < k / 32; ++i) {
            const uint8_t* b = src + i * 18;
            uint8_t* o = dst + i * 34;
            memcpy(o, b, 2);  // the block scale d as it is
            for (int j = 0; j < 16; ++j) {
                o[2 + j] = (uint8_t)kIq4[b[2 + j] & 0xF];
                o[2 + j + 16] = (uint8_t)kIq4[b[2 + j] >> 4];
            }
        }
        return true;
    }
    if (type == CEB_GGML_IQ4_XS) {
        if (k % 256) return false;
        for (int64_t s = 0; s < k / 256; ++s) {
            const uint8_t* b = src + s * 136;
            const float d = h2f(rd16(b));
            for (int ib = 0; ib < 8; ++ib) {
                uint8_t* o = dst + (s * 8 + ib) * 34;
                const __half dl = __float2half_rn(d * (float)(iq4xs_ls(b, ib) - 32));
                const uint16_t dh = __half_raw(dl).x;
                o[0] = (uint8_t)(dh & 0xFF);
                o[1] = (uint8_t)(dh >> 8);
                const uint8_t* qs = b + 8 + 16 * ib;
                for (int j = 0; j < 16; ++j) {
                    o[2 + j] = (uint8_t)kIq4[qs[j] & 0xF];
                    o[2 + j + 16] = (uint8_t)kIq4[qs[j] >> 4];
                }
            }
        }
        return true;
    }
    return false;
}
