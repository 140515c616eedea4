// runtime.cpp -- error reporting, TMA descriptor creation and the load-time
// repack of GGUF weight blocks into the planes the grouped GEMM streams.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ceb_internal.h"
#include "../../include/ceb_ops.h"

namespace {
thread_local std::string g_last_error;
}

int ceb_set_error(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    fprintf(stderr, "crispembed-b200: %s\n", buf);
    return code;
}

int ceb_set_cuda_error(cudaError_t e, const char* what, const char* file, int line) {
    return ceb_set_error(3, "CUDA error %s (%s) at %s:%d: %s", cudaGetErrorName(e), cudaGetErrorString(e), file, line,
                         what);
}

const char* ceb_last_error_message() { return g_last_error.c_str(); }

int ceb_device_index() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= CEB_MAX_DEVICES) dev = 0;
    return dev;
}

int ceb_num_sms() {
    static int n_of[CEB_MAX_DEVICES] = {};
    const int dev = ceb_device_index();
    if (!n_of[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        n_of[dev] = n > 0 ? n : 148;
    }
    return n_of[dev];
}

namespace {
// (device, kernel, dynamic shared memory) triples whose limit has been raised:
// cudaFuncSetAttribute acts on the current device only.
struct FuncSmem {
    int dev;
    const void* func;
    size_t smem;
};
std::mutex g_func_mu;
std::vector<FuncSmem> g_func_smem;
}  // namespace

int ceb_func_smem(const void* func, size_t smem) {
    const int dev = ceb_device_index();
    std::lock_guard<std::mutex> lk(g_func_mu);
    for (const FuncSmem& f : g_func_smem)
        if (f.dev == dev && f.func == func && f.smem >= smem) return 0;
    cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "cudaFuncSetAttribute", __FILE__, __LINE__);
    g_func_smem.push_back({dev, func, smem});
    return 0;
}

// ------------------------------------------------------------------ TMA maps
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
}  // namespace

int ceb_make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
    return ceb_make_tmap_2d_sw(map, base, elem_bytes, inner, rows, row_stride_bytes, box_inner, box_rows,
                               swizzle128 ? 128 : 0);
}

int ceb_make_tmap_2d_sw(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return ceb_set_error(3, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15))
        return ceb_set_error(2, "tensor map: base/stride not 16-byte aligned");
    if ((box_inner * (uint32_t)elem_bytes) & 15) return ceb_set_error(2, "tensor map: box inner extent not 16-byte multiple");
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                    : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                    : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                          : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return ceb_set_error(3, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

int ceb_make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                         uint32_t box_inner, uint32_t box_rows) {
    return ceb_make_tmap_2d(map, base, 2, inner, rows, row_stride_bytes, box_inner, box_rows, true);
}

// ------------------------------------------------------------------ repack
namespace {
inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
inline float h2f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}
inline uint16_t f2h(float f) {
    __half h = __float2half_rn(f);
    return __half_raw(h).x;
}
// Q4_K 6-bit sub-block scale/min of sub-block j (published Q4_K block layout)
inline void q4k_scale_min(int j, const uint8_t* s, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}
}  // namespace

// GGUF rows -> tile-major device blocks (layout in ceb_internal.h).  Values are
// not changed: Q8_0 keeps its int8 quants and fp16 scales, Q4_K its nibbles with
// (d*sc, dmin*m) computed per sub-block exactly as ggml's dequantizer does, F32
// weights are rounded to fp16 (nearest even).  IQ4_NL / IQ4_XS rows are first
// re-encoded as Q8_0 blocks (codebook value as int8, block scale as fp16), every
// other block format is decoded to fp32 and rounded to fp16 (gguf_quants.cpp).
int ceb_repack_weights(ceb_wplane* dst, int ggml_type, const void* host_raw, int n_groups, int n_out, int k,
                       cudaStream_t stream) {
    int64_t rb = ceb_ggml_row_bytes(ggml_type, k);
    if (rb < 0) return ceb_set_error(2, "repack: unsupported type %d for k=%d", ggml_type, k);
    if (n_out % 128 || k % 64)
        return ceb_set_error(2, "repack: n_out=%d must be a multiple of 128 and k=%d of 64", n_out, k);
    const uint8_t* src = static_cast<const uint8_t*>(host_raw);
    const int64_t rows = (int64_t)n_groups * n_out;
    std::vector<uint8_t> conv;  // re-encoded (Q8_0 blocks) or decoded (fp32) rows
    if (ggml_type == CEB_GGML_IQ4_NL || ggml_type == CEB_GGML_IQ4_XS) {
        const int64_t qrb = ceb_ggml_row_bytes(CEB_GGML_Q8_0, k);
        conv.resize((size_t)(rows * qrb));
        for (int64_t r = 0; r < rows; ++r)
            if (!ceb_ggml_as_q8_0_blocks(ggml_type, src + r * rb, k, conv.data() + r * qrb))
                return ceb_set_error(2, "repack: type %d rows of %d values cannot be re-encoded", ggml_type, k);
        src = conv.data();
        rb = qrb;
        ggml_type = CEB_GGML_Q8_0;
    } else if (ggml_type != CEB_GGML_Q8_0 && ggml_type != CEB_GGML_Q4_K && ggml_type != CEB_GGML_F16 &&
               ggml_type != CEB_GGML_F32) {
        conv.resize((size_t)(rows * k * 4));
        for (int64_t r = 0; r < rows; ++r)
            ceb_ggml_dequant_row(ggml_type, src + r * rb, k, reinterpret_cast<float*>(conv.data()) + r * k);
        src = conv.data();
        rb = (int64_t)k * 4;
        ggml_type = CEB_GGML_F32;
    }
    ceb_wplane w;
    w.n_groups = n_groups;
    w.n_out = n_out;
    w.k = k;
    w.format = ggml_type == CEB_GGML_Q8_0 ? CEB_W_Q8_0 : ggml_type == CEB_GGML_Q4_K ? CEB_W_Q4_K : CEB_W_F16;
    w.blk_bytes = ceb_wblock_bytes(w.format);
    const int nft = n_out / 128, nkb = k / 64;
    std::vector<uint8_t> q((size_t)n_groups * nft * nkb * w.blk_bytes);
    for (int g = 0; g < n_groups; ++g)
        for (int ft = 0; ft < nft; ++ft)
            for (int kb = 0; kb < nkb; ++kb) {
                uint8_t* blk = &q[(((size_t)g * nft + ft) * nkb + kb) * w.blk_bytes];
                for (int r = 0; r < 128; ++r) {
                    const uint8_t* row = src + ((int64_t)g * n_out + (int64_t)ft * 128 + r) * rb;
                    if (w.format == CEB_W_Q8_0) {
                        for (int b = 0; b < 2; ++b) {  // the two 32-value blocks of this k-block
                            const uint8_t* qb = row + (int64_t)(2 * kb + b) * 34;
                            memcpy(blk + 8192 + 4 * r + 2 * b, qb, 2);
                            for (int c2 = 0; c2 < 2; ++c2) {
                                const int c = 2 * b + c2;
                                memcpy(blk + r * 64 + ((c ^ ((r >> 1) & 3)) << 4), qb + 2 + 16 * c2, 16);
                            }
                        }
                    } else if (w.format == CEB_W_Q4_K) {
                        const uint8_t* sb = row + (int64_t)(kb / 4) * 144;  // 256-super-block
                        const uint8_t* qs = sb + 16 + (kb % 4) * 32;        // this 64-chunk's nibble bytes
                        for (int c = 0; c < 2; ++c) memcpy(blk + r * 32 + ((c ^ ((r >> 2) & 1)) << 4), qs + 16 * c, 16);
                        const float d = h2f(rd16(sb)), dmin = h2f(rd16(sb + 2));
                        float sm[4];
                        for (int j = 0; j < 2; ++j) {
                            int sc, mn;
                            q4k_scale_min(2 * (kb % 4) + j, sb + 4, &sc, &mn);
                            sm[2 * j] = d * (float)sc;
                            sm[2 * j + 1] = dmin * (float)mn;
                        }
                        memcpy(blk + 4096 + 16 * r, sm, 16);
                    } else {
                        uint16_t h[64];
                        if (ggml_type == CEB_GGML_F16) {
                            memcpy(h, row + (int64_t)kb * 128, 128);
                        } else {
                            const float* f = reinterpret_cast<const float*>(row) + (int64_t)kb * 64;
                            for (int i = 0; i < 64; ++i) h[i] = f2h(f[i]);
                        }
                        for (int c = 0; c < 8; ++c) memcpy(blk + r * 128 + ((c ^ (r & 7)) << 4), h + 8 * c, 16);
                    }
                }
            }
    w.q_bytes = q.size();
    w.s_bytes = 0;
    if (cudaMalloc(&w.q, w.q_bytes) != cudaSuccess) return ceb_set_error(4, "repack: out of device memory");
    cudaError_t e = cudaMemcpyAsync(w.q, q.data(), w.q_bytes, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);  // the host vector dies at return
    if (e != cudaSuccess) {
        cudaFree(w.q);
        return ceb_set_cuda_error(e, "repack upload", __FILE__, __LINE__);
    }
    // Planes the CTA-pair GEMM takes (widths a multiple of 256) are expanded once to
    // fp16 on the device, so the GEMM loads the MMA's operand image directly instead of
    // dequantizing every tile again; CEB_WEIGHT_EXPAND=0 keeps the quantized blocks
    // (half to a quarter of the bytes, dequantized in the GEMM).
    const char* ex = getenv("CEB_WEIGHT_EXPAND");
    if (!(ex && ex[0] == '0') && n_out % 256 == 0 && w.format != CEB_W_F16) {
        if (int rc = ceb_wplane_expand_f16(&w, stream)) {
            ceb_wplane_free(&w);
            return rc;
        }
    }
    *dst = w;
    return 0;
}

void ceb_wplane_free(ceb_wplane* w) {
    if (!w) return;
    if (w->q) cudaFree(w->q);
    *w = ceb_wplane();
}

// ------------------------------------------------------------------ profiling
namespace {
struct ProfRec {
    cudaEvent_t a = nullptr, b = nullptr;
    int cat = 0;
    double flops = 0, bytes = 0;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
long long g_launches = 0;
std::vector<ProfRec> g_prof_recs;
size_t g_prof_used = 0;
}  // namespace

int ceb_prof_begin(cudaStream_t st, int cat) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    ++g_launches;
    if (!g_prof_on) return -1;
    if (g_prof_used == g_prof_recs.size()) {
        ProfRec r;
        if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return -1;
        g_prof_recs.push_back(r);
    }
    ProfRec& r = g_prof_recs[g_prof_used];
    r.cat = cat;
    r.flops = r.bytes = 0;
    cudaEventRecord(r.a, st);
    return (int)g_prof_used++;
}

void ceb_prof_end(int token, cudaStream_t st, double flops, double bytes) {
    if (token < 0) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    ProfRec& r = g_prof_recs[(size_t)token];
    r.flops = flops;
    r.bytes = bytes;
    cudaEventRecord(r.b, st);
}

void ceb_count_launches(long long n) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_launches += n;
}

bool ceb_profiling_on() {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    return g_prof_on;
}

extern "C" long long ceb_launch_count(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    return g_launches;
}

extern "C" void ceb_profile_enable(int on) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_on = on != 0;
    g_prof_used = 0;
}

// Per category: launches, summed kernel milliseconds, algorithmic flops and bytes.
// Synchronises on the recorded events and clears the record list.
extern "C" int ceb_profile_read(long long* launches, double* ms, double* flops, double* bytes, int n_cat) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (int c = 0; c < n_cat; ++c) launches[c] = 0, ms[c] = flops[c] = bytes[c] = 0;
    for (size_t i = 0; i < g_prof_used; ++i) {
        ProfRec& r = g_prof_recs[i];
        if (r.cat >= n_cat) continue;
        float t = 0;
        if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&t, r.a, r.b) != cudaSuccess)
            return ceb_set_error(3, "profile event read failed");
        launches[r.cat] += 1;
        ms[r.cat] += t;
        flops[r.cat] += r.flops;
        bytes[r.cat] += r.bytes;
    }
    g_prof_used = 0;
    return 0;
}
