// ceb_moe_internal.h -- MoE layer state shared between moe.cu, the encoder and the C ABI.
#pragma once

#include <cuda_fp16.h>

#include <vector>

#include "ceb_internal.h"

// activation element types (same values as include/ceb_ops.h)
#ifndef CEB_ACT_F32
#define CEB_ACT_F32 0
#define CEB_ACT_BF16 1
#define CEB_ACT_F16 2
#endif

// Device-resident weights of one MoE feed-forward block.
struct ceb_moe_weights {
    int d = 0, n_experts = 0, top_k = 0, ffn = 0;
    int router_type = CEB_GGML_F32;   // CEB_GGML_F32 ([E][d] floats) or CEB_GGML_Q8_0 (raw ggml blocks)
    uint8_t* router = nullptr;        // device
    ceb_wplane fc1;                   // E x [ffn x d]
    ceb_wplane fc2;                   // E x [d x ffn]
    float* bias = nullptr;            // [d] or null
};

// Per-call scratch, carved from one caller-provided buffer.
struct ceb_moe_ws {
    int32_t* ids = nullptr;           // [T*K] expert of each (token, slot)
    float* wts = nullptr;             // [T*K] gate weight
    int32_t* block_counts = nullptr;  // [nblk*E]
    int32_t* block_base = nullptr;    // [nblk*E]
    int32_t* offsets = nullptr;       // [E+1] expert row ranges in the permuted matrices
    int32_t* slot_pos = nullptr;      // [T*K] permuted row of each (token, slot)
    __half* x_perm = nullptr;         // [T*K x d]
    __half* h_perm = nullptr;         // [T*K x ffn]
    __half* down = nullptr;           // [T*K x d] fc2 outputs (fp16)
};

size_t ceb_moe_ws_layout(int T, int d, int E, int K, int F, ceb_moe_ws* ws, uint8_t* base);
// x: router input ([T x d], x_dtype); x16: optional fp16 copy of x used for the
// expert row gather (else x is converted on the fly).  y may be null when the
// caller fuses the combine (the permuted expert outputs stay in ws.down).
int ceb_moe_run(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T, float* y,
                const ceb_moe_ws& ws, int32_t* expert_counts, float* logits_out, int* dev_err, cudaStream_t st);
// The two halves of ceb_moe_run: ceb_add_ln_route computes out = LN(res + y)
// and routes the normalised rows in the same pass (ids, wts, block_counts of
// ws), then ceb_moe_dispatch (scan, scatter, expert GEMMs, optional combine)
// runs on those routes with x = out32 (x_dtype F32) and x16 = out16.
// y is fp16 when y_f16 (the encoder's GEMM output), else float (the operator entry point).
int ceb_add_ln_route(const float* res, const void* y, bool y_f16, int M, int d, const float* gamma, const float* beta,
                     float eps, float* out32, __half* out16, const ceb_moe_weights& mw, const ceb_moe_ws& ws,
                     float* logits_out, cudaStream_t st);
int ceb_moe_dispatch(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T, float* y,
                     const ceb_moe_ws& ws, int32_t* expert_counts, int* dev_err, cudaStream_t st);

// Handle behind the ceb_moe_layer* of include/ceb_ops.h.
struct ceb_moe_layer {
    ceb_moe_weights w;
    std::vector<void*> allocs;  // router / bias buffers owned by the handle
};
