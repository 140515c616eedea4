// ceb_encoder_internal.h -- NomicBERT-MoE encoder model state and forward pass.
#pragma once

#include <cuda_fp16.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "ceb_internal.h"
#include "ceb_moe_internal.h"

// row-wise / attention kernel launchers (encoder_kernels.cu)
int ceb_embed_ln(const int32_t* ids, const int32_t* cu, int n_seqs, int M, int d, int n_vocab, const float* tok,
                 const float* pos, int n_pos, int pos_offset, const float* type0, const float* gamma,
                 const float* beta, float eps, float* out32, __half* out16, int* err, cudaStream_t st);
// y: the fp16 output of the GEMM in front of the residual
int ceb_add_ln(const float* res, const __half* y, int M, int d, const float* gamma, const float* beta, float eps,
               float* out32, __half* out16, cudaStream_t st);
// down: the fp16 expert rows of the MoE block (fc2 output, permuted order)
int ceb_moe_combine_ln(const __half* down, const int32_t* slot_pos, const float* wts, int K, const float* moe_bias,
                       const float* cur, int M, int d, const float* gamma, const float* beta, float eps, float* out32,
                       __half* out16, cudaStream_t st);
// sched: two device ints, zero before the first call, that the tcgen05 kernel uses to
// hand out its work items (and returns to zero); calls sharing them must be ordered
// on one stream.  nullptr: the mma.sync kernel.
int ceb_attention(const __half* qkv, int total_rows, const int32_t* cu, int n_seqs, int max_len, int d, int n_head,
                  __half* out, int* d_err, cudaStream_t st, int* sched);
// tcgen05 CTA-pair attention (attn_tc.cu); returns 1 without launching when the
// shape is not handled there (head_dim != 64 or a sequence longer than 512)
int ceb_attention_tc(const __half* qkv, int total_rows, const int32_t* cu, int n_seqs, int max_len, int d, int n_head,
                     __half* out, int* d_err, cudaStream_t st);
// single-CTA tcgen05 attention (attn_fa.cu); returns 1 without launching when the shape
// is not handled there (head_dim != 64, operands not 16-byte aligned)
int ceb_attention_fa(const __half* qkv, int total_rows, const int32_t* cu, int n_seqs, int max_len, int d, int n_head,
                     __half* out, int* d_err, cudaStream_t st, int* sched);
// RoPE, NEOX pairing (dims i and i + 32 of each 64-dim head), on the Q and K thirds of
// fused fp16 qkv rows in place; position = row - cu[seq] + pos_offset.
int ceb_rope_neox(__half* qkv, int M, const int32_t* cu, int n_seqs, int d, int n_head, int pos_offset, float theta,
                  cudaStream_t st);
int ceb_pool_l2_launch(const float* hidden, const int32_t* cu, int n_seqs, int d, int out_dim, float* out,
                       cudaStream_t st, int mode = 0);

// Weights in the form the reference-arithmetic kernels read (ref_arith.cu):
// Q8_0 as int8 quants [groups][n_out][k] + block scales [groups][n_out][k/32]
// (the fp16 values as float); F32 / F16 / BF16 widened to float [groups][n_out][k].
struct ceb_refmat {
    int type = 0;  // CEB_GGML_Q8_0 or CEB_GGML_F32
    int n_groups = 0, n_out = 0, k = 0;
    int8_t* q = nullptr;
    float* d = nullptr;
    float* f = nullptr;
};
int ceb_refmat_create(ceb_refmat* r, int ggml_type, const void* host, int groups, int n_out, int k);
void ceb_refmat_free(ceb_refmat* r);

// Reference-arithmetic kernels (ref_arith.cu): the encoder's operations in the
// reference's CPU arithmetic, bit for bit (Q8_0 activation re-quantization,
// ggml's dot-product lane order, sequential-order attention, LayerNorm, softmax
// and pooling).
int ceb_ref_embed(const int32_t* ids, const int32_t* cu, int n_seqs, int d, int n_vocab, const float* tok,
                  const float* pos, int n_pos, int pos_offset, const float* type0, float* out, int* err,
                  cudaStream_t st);
int ceb_ref_ln(const float* a, const float* b, int M, int d, const float* gamma, const float* beta, float eps,
               float* out, cudaStream_t st);
int ceb_ref_quant(const float* x, int rows, int k, int8_t* xq, float* xd, cudaStream_t st);
// out[m, n] = W_g[n] . x[m] (+ bias + g*bias_gstride); Q8_0 weights read xq/xd, float weights x32;
// tile_group: expert of every 32-row tile (-1 = unused), null for one group.
int ceb_ref_matmul(const ceb_refmat& w, const float* x32, const int8_t* xq, const float* xd, int rows,
                   const int32_t* tile_group, const float* bias, int64_t bias_gstride, float* out, int ldo,
                   cudaStream_t st);
int ceb_ref_attention(const float* qkv, const int32_t* cu, int n_seqs, int max_len, int d, int n_head, float* out,
                      cudaStream_t st);
int ceb_ref_gelu(float* x, int64_t n, cudaStream_t st);
int ceb_ref_route(const float* logits, int T, int E, int K, int32_t* ids, float* wts, cudaStream_t st);
int ceb_ref_group(const int32_t* ids, int T, int K, int E, int n_tiles_max, int32_t* pos, int32_t* src,
                  int32_t* tile_group, cudaStream_t st);
int ceb_ref_gather(const float* x, const int32_t* src, int64_t n_rows, int d, float* xp, cudaStream_t st);
int ceb_ref_combine(const float* down, const int32_t* pos, const float* wts, int T, int K, int d, const float* bias,
                    float* y, cudaStream_t st);
int ceb_ref_pool(const float* x, const int32_t* cu, int n_seqs, int d, int out_dim, float* out, cudaStream_t st);

struct ceb_layer {
    ceb_wplane qkv, o, fc1, fc2;
    ceb_refmat r_qkv, r_o, r_fc1, r_fc2, r_router, r_e1, r_e2;  // reference arithmetic only
    float *qkv_b = nullptr, *o_b = nullptr, *fc1_b = nullptr, *fc2_b = nullptr;
    float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
    bool moe = false;
    ceb_moe_weights moew;
};

struct ceb_hparams_c {  // mirrors crispembed_hparams (include/crispembed.h)
    int32_t n_vocab, n_max_tokens, n_embd, n_head, n_layer, n_intermediate, n_output;
    float layer_norm_eps;
    int32_t n_experts, n_experts_per_tok;
};

struct ceb_model {
    ceb_hparams_c hp{};
    int pool_method = 0;   // 0 mean, 1 cls, 2 last
    int pos_offset = 0;
    int n_pos = 0;
    float* tok = nullptr;  // [n_vocab x d] f32
    float* pos = nullptr;  // [n_pos x d] f32 or null (RoPE models)
    bool use_rope = false;  // no position table: RoPE (NEOX pairing) on Q and K
    float rope_theta = 10000.0f;
    float* type0 = nullptr;  // row 0 of the token-type table or null
    float *embd_ln_w = nullptr, *embd_ln_b = nullptr;
    std::vector<ceb_layer> layers;
    std::vector<void*> allocs;  // every device buffer owned by the model
    size_t weight_bytes = 0;
    struct ceb_ep* ep = nullptr;  // expert-parallel exchange (not owned); the MoE planes then hold its experts only
    bool ref_arith = false;       // forward in the reference's CPU arithmetic (ref_arith.cu), set before loading
};

// Buffers of the reference-arithmetic forward (one allocation, ceb_workspace_reserve)
struct ceb_ref_ws {
    float *qkv = nullptr, *attn = nullptr, *h = nullptr, *xp = nullptr, *down = nullptr, *logits = nullptr,
          *wts = nullptr, *xd = nullptr;
    int8_t* xq = nullptr;
    int32_t *ids = nullptr, *pos = nullptr, *src = nullptr, *tile_group = nullptr;
    int n_tiles_max = 0;  // 32-row tiles of the padded expert rows
};

struct ceb_workspace {
    int cap_tokens = 0;
    int cap_seqs = 0;
    void* base = nullptr;
    size_t bytes = 0;
    float *x32 = nullptr, *c32 = nullptr, *t32 = nullptr;
    __half *x16 = nullptr, *c16 = nullptr, *qkv16 = nullptr, *a16 = nullptr, *h16 = nullptr;
    __half* t16 = nullptr;     // fp16 output of the GEMMs in front of a residual (attn-out, dense fc2)
    ceb_moe_ws moe;
    ceb_ref_ws ref;            // reference-arithmetic models only
    int32_t* ids = nullptr;    // [cap_tokens]
    int32_t* cu = nullptr;     // [cap_seqs + 1]
    float* out = nullptr;      // [cap_seqs x d]
    int* attn_sched = nullptr;  // [2] attention work-item counter (zeroed at allocation)
};

int ceb_model_load(ceb_model* m, const std::string& path, std::string* err_out);
// Keeps only the exchange's local experts of every MoE block (the other experts'
// weights are freed) and routes the MoE blocks through it from then on.
int ceb_model_ep_attach(ceb_model* m, struct ceb_ep* ep);
void ceb_model_free(ceb_model* m);
int ceb_workspace_reserve(ceb_workspace* ws, const ceb_model& m, int tokens, int seqs);
void ceb_workspace_free(ceb_workspace* ws);
// Optional record of every MoE block's routing during a forward pass (diagnostics and
// parity tests): block b's expert ids go to ids + b*M*K ([M x K], slot j = j-th largest
// probability) and its router logits to logits + b*M*E ([M x E]); device buffers.
struct ceb_route_capture {
    int32_t* ids = nullptr;
    float* logits = nullptr;
};

// Full forward pass on device-resident ids; writes [n_seqs x out_dim] pooled, L2-normalised rows.
int ceb_encoder_forward(const ceb_model& m, ceb_workspace& ws, const int32_t* d_ids, const int32_t* d_cu, int n_seqs,
                        int n_tokens, int max_len, float* d_out, int out_dim, int* d_err, cudaStream_t st,
                        const ceb_route_capture* cap = nullptr);
