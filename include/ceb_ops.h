/*
 * ceb_ops.h -- operator-level C ABI of crispembed-b200 (sm_100a).
 *
 * These entry points expose, one by one, the device implementations of the
 * operations CrispEmbed's NomicBERT-MoE encoder builds as ggml graph nodes, so a
 * host that drives its own graph (or a test) can call them directly.  All
 * pointers named d_* are device pointers, h_* host pointers; `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Calls are
 * asynchronous on `stream` unless stated otherwise.  Every function returns 0 on
 * success and a nonzero status otherwise; ceb_last_error() then holds a message
 * (also printed to stderr, the reference's error channel).
 *
 * Status codes: 1 bad argument / not supported, 2 unsupported shape,
 * 3 CUDA error, 4 out of device memory, 5 device-side check failed.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#if defined(CRISPEMBED_BUILD)
#define CEB_API __attribute__((visibility("default")))
#else
#define CEB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ggml tensor types accepted for weights (values of ggml's enum) */
#define CEB_TYPE_F32 0
#define CEB_TYPE_F16 1
#define CEB_TYPE_Q8_0 8
#define CEB_TYPE_Q4_K 12

/* activation element types */
#define CEB_ACT_F32 0
#define CEB_ACT_BF16 1
#define CEB_ACT_F16 2

typedef struct ceb_moe_layer ceb_moe_layer;
typedef struct crispembed_context crispembed_context;

/*
 * Upload one MoE feed-forward block.  Host buffers hold ggml tensor bytes as a
 * GGUF file stores them (the reference binds the same tensors in load_model,
 * src/crispembed.cpp:838-844):
 *   router  [n_experts rows x d]        (ffn.moe_gate.weight; F32 or Q8_0)
 *   fc1     [n_experts][ffn rows x d]   (ffn.expert_fc1.weight; F32/F16/Q8_0/Q4_K)
 *   fc2     [n_experts][d rows x ffn]   (ffn.expert_fc2.weight; same type as fc1)
 *   bias    [d] floats or NULL          (ffn.moe_bias)
 * Returns NULL on failure.  Limits: n_experts <= 32, top_k <= 4, d and ffn
 * multiples of 128 (of 256 for Q4_K).
 */
CEB_API ceb_moe_layer* ceb_moe_layer_create(int d, int n_experts, int top_k, int ffn, int router_type,
                                            const void* h_router, int expert_type, const void* h_fc1,
                                            const void* h_fc2, const float* h_bias);
CEB_API void ceb_moe_layer_free(ceb_moe_layer* layer);

/* Bytes of device scratch ceb_moe_ffn needs for up to max_tokens tokens. */
CEB_API size_t ceb_moe_workspace_size(const ceb_moe_layer* layer, int max_tokens);

/*
 * The MoE feed-forward block, replacing the graph branch of
 * build_encoder_graph at src/crispembed.cpp:1327-1381:
 *   y[t] = sum_j w[t,j] * fc2_{e_j}( gelu_erf( fc1_{e_j}( x[t] ) ) ) + bias,
 *   (e_j, w[t,j]) = top_k(softmax(router x[t])), weights not renormalised.
 * d_x: [n_tokens x d] activations of type x_dtype, 16-byte aligned (status 1
 * otherwise, nothing launched).  d_y: [n_tokens x d] floats.
 * Optional outputs (may be NULL): d_ids / d_weights [n_tokens x top_k] (slot j =
 * j-th largest probability), d_expert_counts [n_experts], d_logits
 * [n_tokens x n_experts] router logits.  d_workspace: at least
 * ceb_moe_workspace_size(layer, n_tokens) bytes, 256-byte aligned.
 */
CEB_API int ceb_moe_ffn(const ceb_moe_layer* layer, const void* d_x, int x_dtype, int n_tokens, float* d_y,
                        int32_t* d_ids, float* d_weights, int32_t* d_expert_counts, float* d_logits, void* d_workspace,
                        size_t workspace_bytes, void* stream);

/*
 * Where the routing of the last ceb_moe_ffn / ceb_moe_route_ln call on a workspace
 * lives inside it (device pointers into d_workspace, valid until the next call on
 * it; no counterpart in the reference, where the grouping stays inside
 * ggml_mul_mat_id, src/crispembed.cpp:1365,1371): ids / weights [n_tokens x
 * top_k], slot_pos [n_tokens x top_k] = row of (token, slot) in the permuted
 * expert matrices, offsets [n_experts + 1] = first row of each expert.  Rows are
 * ordered by expert, then token, then slot -- ggml_mul_mat_id's grouping.
 * offsets and slot_pos are written by the expert dispatch (ceb_moe_ffn), not by
 * ceb_moe_route_ln alone.  Any output pointer may be NULL.
 */
CEB_API int ceb_moe_workspace_routing(const ceb_moe_layer* layer, int n_tokens, void* d_workspace, int32_t** d_ids,
                                      float** d_weights, int32_t** d_slot_pos, int32_t** d_offsets);

/*
 * The residual + LayerNorm that feeds the MoE block and the block's router in
 * one pass (src/crispembed.cpp:1316-1323 post-attention LN, then :1333-1345
 * router, softmax, top_k, gate weights): d_out = LN(d_res + d_y) * gamma + beta
 * (ggml_norm, then separate *gamma and +beta roundings; gamma/beta may be NULL),
 * and the expert choice of every normalised row computed from the registers
 * that hold it, so the router never re-reads the activations.
 * d_res, d_y, d_out: [n_tokens x d] floats (d_out may alias d_res).  d_out16:
 * optional fp16 copy of d_out.  d_ids / d_weights / d_logits as in ceb_moe_ffn
 * (optional).  d_workspace as for ceb_moe_ffn; its routing part keeps the
 * routes.  The encoder uses this form in front of every MoE block.
 */
CEB_API int ceb_moe_route_ln(const ceb_moe_layer* layer, const float* d_res, const float* d_y, int n_tokens,
                             const float* d_gamma, const float* d_beta, float eps, float* d_out, void* d_out16,
                             int32_t* d_ids, float* d_weights, float* d_logits, void* d_workspace,
                             size_t workspace_bytes, void* stream);

/*
 * ceb_moe_ffn without any device allocation (no counterpart in the reference).
 *
 * For callers that must not allocate device memory once running -- a host whose
 * GPU memory belongs to another allocator, a plugin handed only a stream, or a
 * latency-critical path that cannot take the device-wide synchronisation of
 * cudaMalloc/cudaFree.  The scratch is a fixed CEB_MOE_STATIC_SCRATCH_BYTES
 * array inside this library, reserved on a device when the library's device code
 * is loaded there -- with lazy module loading (CUDA_MODULE_LOADING=LAZY, the
 * default since CUDA 12.2) at the first use of that code on the device, with
 * EAGER on every device the process initialises, callers of this entry or not --
 * and held until the process exits; the call itself allocates nothing (with
 * instrumentation off, the default).  Computes what ceb_moe_ffn computes (y only).
 *
 * Limits and rules:
 *  - n_tokens is limited by the scratch: ceb_moe_workspace_size(layer, n_tokens)
 *    must not exceed CEB_MOE_STATIC_SCRATCH_BYTES (about 3600 tokens for d=768,
 *    ffn=3072, top-2); larger batches are rejected with status 1 -- split them.
 *  - The first call on a device looks the scratch up on that device; make that
 *    first call before any stream capture.
 *  - All calls on a device share the one scratch, which keeps the previous
 *    call's contents: calls that overlap on the GPU (other streams, other host
 *    threads) race and corrupt each other.  Serialise them.
 */
#define CEB_MOE_STATIC_SCRATCH_BYTES (64u << 20)
CEB_API int ceb_moe_ffn_static(const ceb_moe_layer* layer, const void* d_x, int x_dtype, int n_tokens, float* d_y,
                               void* stream);

/*
 * crispembed_init with options (no counterpart in the reference).  flags:
 *
 * CEB_INIT_REFERENCE_ARITHMETIC -- run the encoder in the arithmetic of the
 *   reference's ggml CPU path, bit for bit: every activation that meets a Q8_0
 *   weight is re-quantized to Q8_0 and dotted in integers with ggml's x86 lane
 *   order, float weights accumulate with one fma per element in index order,
 *   attention, LayerNorm, softmax and pooling sum in the reference's sequential
 *   orders, and exp / erf are shared double-precision routines that round
 *   correctly.  The expert choice of every MoE block then equals the reference
 *   arithmetic's, which the default fp16 tensor-core path cannot promise: there a
 *   token whose 2nd and 3rd router logits lie closer than the Q8_0 rounding noise
 *   (~1e-2 after a few layers) may take the other expert.  CUDA cores only, far
 *   slower than the default; F32/F16/BF16/Q8_0 weights, learned positions and
 *   mean pooling; no expert parallelism.  crispembed_init selects it when the
 *   environment variable CEB_REFERENCE_ARITHMETIC is 1.
 * Returns NULL on failure (message in ceb_last_error()).
 */
#define CEB_INIT_REFERENCE_ARITHMETIC 1
CEB_API crispembed_context* ceb_init_ex(const char* model_path, int n_threads, int flags);

/*
 * Diagnostic encode that also returns every MoE block's routing (no counterpart in
 * the reference, whose expert choice stays inside its graph at
 * src/crispembed.cpp:1333-1345).  Encodes the packed ids (h_lens[i] tokens per
 * sequence, M tokens in all) like crispembed_encode_ids_batch, synchronously and
 * without graph capture, and copies to host memory: h_out [n_seqs x dim]
 * embeddings (may be NULL), h_route_ids [n_moe x M x top_k] expert ids (slot j =
 * j-th largest probability) and h_route_logits [n_moe x M x n_experts] router
 * logits, n_moe = the number of MoE blocks in layer order (either may be NULL).
 * Allocates its capture buffers for the call.  Returns 0 or a status.
 */
CEB_API int ceb_encode_ids_routes(crispembed_context* ctx, const int32_t* h_ids, const int32_t* h_lens, int n_seqs,
                                  float* h_out, int32_t* h_route_ids, float* h_route_logits);
/* Number of MoE blocks of the context's model (the n_moe above). */
CEB_API int ceb_moe_block_count(const crispembed_context* ctx);

/*
 * Mean pool + L2 normalise, replacing the host loops of encode_tokens
 * (src/crispembed.cpp:1822-1846) and pool_and_norm (:2024-2045):
 *   p = mean over the rows of each sequence; out = p / sqrt(max(sum p^2, 1e-12)).
 * d_hidden [n_rows x d] floats; d_cu_seqlens [n_seqs+1] row offsets (int32);
 * d_out [n_seqs x out_dim] with out_dim <= d: the first out_dim pooled values,
 * normalised over those out_dim values (Matryoshka truncation,
 * src/crispembed.cpp:2786-2793, when out_dim < d).
 */
CEB_API int ceb_pool_l2(const float* d_hidden, const int32_t* d_cu_seqlens, int n_seqs, int d, int out_dim,
                        float* d_out, void* stream);

/*
 * Expert parallelism across the GPUs of one node (no counterpart in the
 * reference, which runs every expert of a block on one device inside
 * ggml_mul_mat_id, src/crispembed.cpp:1365-1371).  One process per GPU, rank r
 * of `world` owns experts [r*E/world, (r+1)*E/world) of every MoE block and
 * routes its own tokens.  Each rank exports one device region through CUDA IPC;
 * the permutation kernel stores every routed row straight into the owner's
 * receive buffer over NVLink and the owner stores the expert outputs back, with
 * release/acquire flags and bounded on-device waits (status 5, code 0x107, when
 * a peer does not answer within the timeout).  No host synchronisation.
 *
 * Setup (every rank, same arguments except rank):
 *   ep = ceb_ep_create(rank, world, E, K, d, F, max_local_tokens);
 *   ceb_ep_ipc_handle(ep, mine);              // CEB_EP_HANDLE_BYTES bytes
 *   ...all-gather the handles in rank order (host collective of the caller)...
 *   ceb_ep_connect(ep, all_handles);          // world * CEB_EP_HANDLE_BYTES
 * Every rank must then issue the same sequence of expert-parallel calls (each
 * MoE block is one exchange), also when it has no tokens of its own.
 * ceb_ep_free waits for the device and unmaps the peers' regions.
 */
#define CEB_EP_HANDLE_BYTES 64
typedef struct ceb_ep ceb_ep;
CEB_API ceb_ep* ceb_ep_create(int rank, int world, int n_experts, int top_k, int d, int ffn, int max_local_tokens);
CEB_API int ceb_ep_ipc_handle(const ceb_ep* ep, void* handle_out);
CEB_API int ceb_ep_connect(ceb_ep* ep, const void* handles);
CEB_API void ceb_ep_set_timeout_ms(ceb_ep* ep, int ms);
CEB_API void ceb_ep_free(ceb_ep* ep);

/*
 * Runs every MoE block of an encoder context through the exchange from now on
 * (crispembed_encode* and crispembed_encode_ids_batch on this rank's own
 * sequences; every rank must encode in lockstep, one call per call).  The
 * context keeps only this rank's experts; the other experts' weights are freed.
 * The exchange must outlive the context's use of it.
 */
CEB_API int ceb_ep_attach(crispembed_context* ctx, ceb_ep* ep);

/*
 * ceb_moe_ffn over the exchange: this rank's n_tokens rows (0 allowed) are
 * routed here, their rows go to the experts' owners and the outputs come back
 * for the combine.  y is bit-identical to ceb_moe_ffn on one GPU.  The layer
 * holds all experts; only this rank's slice is used.
 */
CEB_API int ceb_moe_ffn_ep(const ceb_moe_layer* layer, ceb_ep* ep, const void* d_x, int x_dtype, int n_tokens,
                           float* d_y, void* d_workspace, size_t workspace_bytes, void* stream);

/*
 * Host decoding of GGUF weight rows to fp32 (no device needed): F32, F16, BF16,
 * Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K, IQ4_NL, IQ4_XS -- ggml's block
 * formats, as the model loader decodes tensors the GEMM does not read in their
 * stored form.  h_src holds n_rows rows of k values; returns 0, or 1 for an
 * unsupported type or a k that is not a whole number of blocks.
 */
CEB_API int ceb_gguf_dequantize(int ggml_type, const void* h_src, int64_t n_rows, int64_t k, float* h_dst);

/*
 * The text tokenizer of a GGUF on its own (no device needed): the family the
 * reference would pick (src/tokenizer.h:37-52), WordPiece or SentencePiece
 * Unigram, wrapping and truncation to max_tokens as the text ABI applies them.
 * ceb_tokenizer_encode writes up to `cap` ids and returns the full count (-1 on
 * error).  No counterpart in the reference's exported API: the reference keeps
 * its tokenizers internal; these serve tests and tools.
 */
typedef struct ceb_text_tokenizer ceb_text_tokenizer;
CEB_API ceb_text_tokenizer* ceb_tokenizer_load(const char* gguf_path, int max_tokens);
CEB_API int ceb_tokenizer_encode(const ceb_text_tokenizer* tok, const char* text, int32_t* ids, int cap);
CEB_API int ceb_tokenizer_kind_of(const ceb_text_tokenizer* tok);
CEB_API void ceb_tokenizer_free(ceb_text_tokenizer* tok);

/*
 * Multi-head self-attention over packed sequences, the attention block of the
 * encoder graph (src/crispembed.cpp:1278-1297): for every sequence s (rows
 * cu[s] .. cu[s+1]-1) and head h, softmax(Q K^T / sqrt(head_dim)) V, no mask
 * beyond the sequence bounds.  d_qkv [n_rows x 3d] fp16 holds Q | K | V per row
 * (head h at columns h*64 .. h*64+63 of each third); d_out [n_rows x d] fp16.
 * head_dim must be 64; d_qkv and d_out 16-byte aligned (status 1 otherwise).
 * The default kernel runs single-CTA tcgen05 MMAs with an online softmax and
 * takes its work items from a counter the library keeps per (device, stream), so
 * calls on different streams may overlap; the first call on a stream allocates
 * that counter (8 bytes).  CEB_ATTN_MMA=1 in the environment selects the mma.sync
 * kernel, CEB_ATTN_TC=1 the tcgen05 CTA-pair kernel (sequences of up to 512
 * tokens).  Asynchronous on `stream`; device-side failures surface through
 * ceb_sync_check.
 */
CEB_API int ceb_attention_forward(const void* d_qkv, int n_rows, const int32_t* d_cu_seqlens, int n_seqs, int max_len,
                                  int d, int n_head, void* d_out, void* stream);

/*
 * A device-resident linear layer (one ggml_mul_mat weight of the encoder,
 * src/crispembed.cpp:1160-1416): W [n_out rows x k] given as GGUF bytes on the
 * host, repacked once into the planes the tensor-core GEMM streams.
 * ceb_linear_forward: d_out[m, n] = sum_k W[n, k] * d_x[m, k] (+ d_bias[n]),
 * optional erf-GELU; d_x [m x k] fp16; d_out fp16 if out_f16 else float.
 * Asynchronous on `stream`.  n_out a multiple of 128, k of 64 (256 for Q4_K).
 */
typedef struct ceb_linear ceb_linear;
CEB_API ceb_linear* ceb_linear_create(int w_type, const void* h_w, int n_out, int k);
CEB_API int ceb_linear_forward(const ceb_linear* lin, const void* d_x, int m, const float* d_bias, int gelu,
                               int out_f16, void* d_out, void* stream);
CEB_API void ceb_linear_free(ceb_linear* lin);

/*
 * One block-quantized matrix product on the tensor cores (the ggml_mul_mat of
 * the encoder's dense layers): d_out[m, n] = sum_k W[n, k] * d_x[m, k] (+ bias[n]),
 * optional erf-GELU.  h_w: GGUF bytes of W [n_out rows x k] (host); d_x: [m x k]
 * fp16; d_out: [m x n_out], fp16 if out_f16 else float.  Synchronous (uploads W
 * for the call).  n_out a multiple of 128, k a multiple of 64 (256 for Q4_K).
 */
CEB_API int ceb_matmul(int w_type, const void* h_w, int n_out, int k, const void* d_x, int m, const float* d_bias,
                       int gelu, int out_f16, void* d_out, void* stream);

/*
 * Instrumentation (no counterpart in the reference beyond its
 * CRISPEMBED_CRISPEMBED_BENCH wall-clock prints, src/crispembed.cpp:1707-1712).
 * ceb_launch_count: kernels this library has launched since it was loaded.
 * ceb_profile_enable(1): from now on record CUDA events around every launch,
 * on the launch's own stream.  ceb_profile_read: per category (0 dense GEMMs of
 * the encoder and the linear entry points, 1 attention, 2 routing + permutation,
 * 3 row-wise: embedding / LayerNorm / combine / pooling, 4 expert-parallel peer
 * copies, 5 expert-parallel waits for peers, 6 grouped expert GEMMs of MoE
 * blocks) the number of launches, summed kernel milliseconds and
 * algorithmic flops / bytes; synchronises on the recorded events and clears
 * them.  Returns 0 on success.
 */
CEB_API long long ceb_launch_count(void);
CEB_API void ceb_profile_enable(int on);
CEB_API int ceb_profile_read(long long* launches, double* ms, double* flops, double* bytes, int n_categories);

/* Message of the last failing call on this thread ("" if none). */
CEB_API const char* ceb_last_error(void);

/*
 * Synchronise `stream` and report any CUDA error or device-side check (a
 * bounded wait that gave up, a bad group range) raised by this library's kernels
 * since the last call.  Returns 0 when clean.
 */
CEB_API int ceb_sync_check(void* stream);

#ifdef __cplusplus
}
#endif
