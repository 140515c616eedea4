// ceb_internal.h -- host-side declarations shared by the .cu/.cpp files of the
// library.  Nothing here is part of the public C ABI (see include/*.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

// ggml tensor types used on the path (values are ggml's enum)
enum {
    CEB_GGML_F32 = 0, CEB_GGML_F16 = 1, CEB_GGML_Q4_0 = 2, CEB_GGML_Q4_1 = 3, CEB_GGML_Q5_0 = 6, CEB_GGML_Q5_1 = 7,
    CEB_GGML_Q8_0 = 8, CEB_GGML_Q4_K = 12, CEB_GGML_Q5_K = 13, CEB_GGML_Q6_K = 14, CEB_GGML_IQ4_NL = 20,
    CEB_GGML_IQ4_XS = 23, CEB_GGML_BF16 = 30,
};

// GGUF block formats (gguf_quants.cpp): bytes of a k-value row (-1: unsupported type
// or k not a whole number of blocks), host decoding of one row to fp32, and the
// types the Q8_0 GEMM path runs after a re-encoding into Q8_0 blocks (Q8_0 itself,
// IQ4_NL, IQ4_XS).
int64_t ceb_ggml_row_bytes(int type, int64_t k);
bool ceb_ggml_dequant_row(int type, const uint8_t* src, int64_t k, float* dst);
bool ceb_ggml_as_q8_0_blocks(int type, const uint8_t* src, int64_t k, uint8_t* dst);

// Device weight formats consumed by the grouped GEMM.  Weights are stored
// tile-major: one contiguous block per (group, 128-row feature tile, 64-wide
// k-block), blocks ordered [group][feature tile][k-block], so the GEMM streams
// each block into shared memory with one bulk copy.  Inside a block (row r of
// the tile, 16-byte chunks XOR-swizzled so a warp reading one chunk of 32
// consecutive rows hits distinct shared-memory banks):
enum ceb_wformat : int {
    CEB_W_F16 = 0,   // 16384 B: row r at r*128, chunk c (k 8c..8c+7) at chunk c^(r&7) -- the
                     //          128-byte-swizzled K-major image the MMA reads directly
    CEB_W_Q8_0 = 1,  //  8704 B: int8 quants row r at r*64, chunk c (k 16c..16c+15) at chunk c^((r>>1)&3);
                     //          then the two fp16 block scales of each row at 8192 + 4r
    CEB_W_Q4_K = 2,  //  6144 B: ggml nibble bytes of the 64-chunk, row r at r*32, chunk c at c^((r>>2)&1);
                     //          then (d*sc, dmin*m) floats of the two sub-blocks of each row at 4096 + 16r
};

constexpr int ceb_wblock_bytes(int format) {
    return format == CEB_W_F16 ? 16384 : format == CEB_W_Q8_0 ? 8704 : 6144;
}

// A repacked weight matrix set: n_groups matrices of [n_out x k] (experts, or 1 for dense).
struct ceb_wplane {
    int format = CEB_W_F16;
    int n_groups = 0, n_out = 0, k = 0;
    uint8_t* q = nullptr;    // tile-major blocks (device)
    int64_t blk_bytes = 0;   // bytes per (group, feature tile, k-block) block
    size_t q_bytes = 0, s_bytes = 0;
};

// Epilogue flags of the grouped GEMM
enum : int {
    CEB_EPI_F16_OUT = 1,  // store fp16 (else fp32)
    CEB_EPI_BIAS = 2,     // add bias[n] (bias pointer per group: bias + g*bias_group_stride)
    CEB_EPI_GELU = 4,     // erf-GELU after bias
};

// ---- launch accounting and optional per-category CUDA-event timing ---------
enum ceb_prof_cat : int {
    CEB_PROF_GEMM = 0,
    CEB_PROF_ATTN = 1,
    CEB_PROF_ROUTE = 2,   // router + histogram/scan + permutation
    CEB_PROF_ROWWISE = 3, // embedding, residual+LN, combine+LN, pooling
    CEB_PROF_EXCHANGE = 4, // expert-parallel peer copies (dispatching permutation, return)
    CEB_PROF_EP_WAIT = 5,  // expert-parallel waits for peers' flags
    CEB_PROF_MOE_GEMM = 6, // the grouped expert GEMMs of MoE blocks (fc1 + GELU, fc2)
    CEB_PROF_NCAT = 7,
};

struct ceb_gemm_args {
    const int* offsets = nullptr;  // device [n_groups+1] activation-row ranges per group; null = dense
    int m_rows = 0;                // dense: activation rows; grouped: capacity of the activation buffer
    void* out = nullptr;
    int ldo = 0;                   // output row stride (elements)
    int epi = 0;
    const float* bias = nullptr;
    int64_t bias_group_stride = 0;
    int* err = nullptr;            // device error word
    int prof_cat = CEB_PROF_GEMM;  // profiling category of the launch
};

// status / errors
int ceb_set_error(int code, const char* fmt, ...);
int ceb_set_cuda_error(cudaError_t e, const char* what, const char* file, int line);
const char* ceb_last_error_message();

// tensor maps
int ceb_make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, bool swizzle128);
// Same with the shared-memory swizzle span in bytes (0, 32, 64 or 128).
int ceb_make_tmap_2d_sw(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes);
int ceb_make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                         uint32_t box_inner, uint32_t box_rows);

// kernels (launchers return 0 or an error code)
int ceb_gemm_launch(const ceb_wplane& w, const void* act_f16, int act_rows_capacity, const ceb_gemm_args& a,
                    cudaStream_t stream, int max_ctas = 0);
int ceb_repack_weights(ceb_wplane* dst, int ggml_type, const void* host_raw, int n_groups, int n_out, int k,
                       cudaStream_t stream);
void ceb_wplane_free(ceb_wplane* w);
// Replace a Q8_0 / Q4_K plane by the fp16 plane of the same values (the GEMM's own
// dequantizer run once over every block); fp16 planes are left as they are.
int ceb_wplane_expand_f16(ceb_wplane* w, cudaStream_t st);

// Launch setup is per device: a process may drive several GPUs.
constexpr int CEB_MAX_DEVICES = 64;
int ceb_device_index();  // the current device (0 when it cannot be read)
int ceb_num_sms();       // SMs of the current device
// Raises the dynamic shared-memory limit of kernel `func` to `smem` bytes on the
// current device, once per (device, kernel).
int ceb_func_smem(const void* func, size_t smem);
// device error word shared by the operator-level entry points (api.cpp)
int* ceb_op_error_word();


// Counts one kernel launch; when profiling is on, records a start event on `st`.
int ceb_prof_begin(cudaStream_t st, int cat);
// Records the stop event of the token returned by ceb_prof_begin (no-op for -1)
// with the launch's algorithmic flops / bytes.
void ceb_prof_end(int token, cudaStream_t st, double flops, double bytes);

// Adds n launches to the count (a CUDA-graph replay of n recorded kernels), and
// whether per-launch profiling events are being recorded.
void ceb_count_launches(long long n);
bool ceb_profiling_on();
// Current value of the launch counter (ceb_launch_count).
extern "C" long long ceb_launch_count(void);

// Wraps one kernel launch statement with ceb_prof_begin / ceb_prof_end.
#define CEB_LAUNCH(cat, st, flops, bytes, ...)          \
    do {                                                \
        const int tk__ = ceb_prof_begin((st), (cat));   \
        __VA_ARGS__;                                    \
        ceb_prof_end(tk__, (st), (flops), (bytes));     \
    } while (0)
