// runtime.cpp -- error reporting, TMA descriptor creation and the load-time
// repack of GGUF weight blocks into the planes the grouped GEMM streams.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
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

int ceb_num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
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
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
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

int64_t ceb_ggml_row_bytes(int type, int64_t k) {
    switch (type) {
        case CEB_GGML_F32: return k * 4;
        case CEB_GGML_F16: return k * 2;
        case CEB_GGML_Q8_0: return k % 32 ? -1 : k / 32 * 34;
        case CEB_GGML_Q4_K: return k % 256 ? -1 : k / 256 * 144;
    }
    return -1;
}

// GGUF rows -> device planes.
//   Q8_0: int8 quants [rows][k], fp16 scales [rows][k/32] (block headers split off).
//   Q4_K: the 128 quant bytes of every super-block back to back (ggml's in-chunk
//         nibble order kept), plus per 32-value sub-block the pair
//         (d*sc, dmin*m) as floats, computed exactly as ggml's dequantizer does.
//   F32/F16: fp16 plane (F32 rounded to nearest even).
int ceb_repack_weights(ceb_wplane* dst, int ggml_type, const void* host_raw, int n_groups, int n_out, int k,
                       cudaStream_t stream) {
    const int64_t rows = (int64_t)n_groups * n_out;
    const int64_t rb = ceb_ggml_row_bytes(ggml_type, k);
    if (rb < 0) return ceb_set_error(2, "repack: unsupported type %d for k=%d", ggml_type, k);
    const uint8_t* src = static_cast<const uint8_t*>(host_raw);
    ceb_wplane w;
    w.n_groups = n_groups;
    w.n_out = n_out;
    w.k = k;
    std::vector<uint8_t> q, s;
    if (ggml_type == CEB_GGML_Q8_0) {
        w.format = CEB_W_Q8_0;
        w.q_row_bytes = k;
        w.s_row_bytes = (int64_t)(k / 32) * 2;
        q.resize((size_t)(rows * w.q_row_bytes));
        s.resize((size_t)(rows * w.s_row_bytes));
        for (int64_t r = 0; r < rows; ++r) {
            const uint8_t* row = src + r * rb;
            for (int b = 0; b < k / 32; ++b) {
                memcpy(&s[(size_t)(r * w.s_row_bytes + b * 2)], row + b * 34, 2);
                memcpy(&q[(size_t)(r * w.q_row_bytes + b * 32)], row + b * 34 + 2, 32);
            }
        }
    } else if (ggml_type == CEB_GGML_Q4_K) {
        w.format = CEB_W_Q4_K;
        w.q_row_bytes = k / 2;
        w.s_row_bytes = (int64_t)(k / 32) * 8;
        q.resize((size_t)(rows * w.q_row_bytes));
        s.resize((size_t)(rows * w.s_row_bytes));
        for (int64_t r = 0; r < rows; ++r) {
            const uint8_t* row = src + r * rb;
            float* sr = reinterpret_cast<float*>(&s[(size_t)(r * w.s_row_bytes)]);
            for (int b = 0; b < k / 256; ++b) {
                const uint8_t* blk = row + b * 144;
                const float d = h2f(rd16(blk)), dmin = h2f(rd16(blk + 2));
                for (int j = 0; j < 8; ++j) {
                    int sc, mn;
                    q4k_scale_min(j, blk + 4, &sc, &mn);
                    sr[2 * (b * 8 + j)] = d * (float)sc;
                    sr[2 * (b * 8 + j) + 1] = dmin * (float)mn;
                }
                memcpy(&q[(size_t)(r * w.q_row_bytes + b * 128)], blk + 16, 128);
            }
        }
    } else {
        w.format = CEB_W_F16;
        w.q_row_bytes = (int64_t)k * 2;
        q.resize((size_t)(rows * w.q_row_bytes));
        uint16_t* qh = reinterpret_cast<uint16_t*>(q.data());
        if (ggml_type == CEB_GGML_F16) {
            memcpy(q.data(), src, q.size());
        } else {
            const float* f = reinterpret_cast<const float*>(src);
            for (int64_t i = 0; i < rows * k; ++i) qh[i] = f2h(f[i]);
        }
    }
    w.q_bytes = q.size();
    w.s_bytes = s.size();
    if (cudaMalloc(&w.q, w.q_bytes) != cudaSuccess) return ceb_set_error(4, "repack: out of device memory");
    if (w.s_bytes && cudaMalloc(&w.s, w.s_bytes) != cudaSuccess) {
        cudaFree(w.q);
        return ceb_set_error(4, "repack: out of device memory");
    }
    cudaError_t e = cudaMemcpyAsync(w.q, q.data(), w.q_bytes, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess && w.s_bytes) e = cudaMemcpyAsync(w.s, s.data(), w.s_bytes, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);  // host vectors die at return
    if (e != cudaSuccess) {
        cudaFree(w.q);
        if (w.s) cudaFree(w.s);
        return ceb_set_cuda_error(e, "repack upload", __FILE__, __LINE__);
    }
    *dst = w;
    return 0;
}

void ceb_wplane_free(ceb_wplane* w) {
    if (!w) return;
    if (w->q) cudaFree(w->q);
    if (w->s) cudaFree(w->s);
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
