/*
 * crispembed.h -- C ABI of crispembed-b200, a drop-in for the embedding entry
 * points of CrispEmbed's src/crispembed.h on NVIDIA B200 (sm_100a).
 *
 * Every declaration below keeps the reference's name, signature, ownership and
 * error behaviour (NULL return + message on stderr) so the reference's Python
 * ctypes binding (python/crispembed/_binding.py:165-330) and Rust FFI
 * (crispembed-sys/src/lib.rs:238-252) load this library unchanged.  Returned
 * vectors are owned by the context and stay valid until the next call on that
 * context or crispembed_free (src/crispembed.h:128-137).  A context is not
 * thread-safe.  Model scope: post-LN BERT-family encoders with learned
 * positions, GELU or MoE (NomicBERT-MoE) feed-forward blocks, head_dim 64,
 * F32/F16/Q8_0/Q4_K linear weights; other architectures fail at init with a
 * message.
 */
#pragma once

#include <stdint.h>

#if defined(CRISPEMBED_BUILD)
#define CRISPEMBED_API __attribute__((visibility("default")))
#else
#define CRISPEMBED_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct crispembed_context crispembed_context;

/* Same layout as the reference (src/crispembed.h:45-56). */
typedef struct crispembed_hparams {
    int32_t n_vocab;
    int32_t n_max_tokens;
    int32_t n_embd;
    int32_t n_head;
    int32_t n_layer;
    int32_t n_intermediate;
    int32_t n_output;
    float layer_norm_eps;
    int32_t n_experts;
    int32_t n_experts_per_tok;
} crispembed_hparams;

/* src/crispembed.h:57-66 / src/crispembed.cpp:2390.  Loads the GGUF onto the
 * current CUDA device.  n_threads <= 0 selects min(4, cores) (host tokenizer
 * work only).  NULL on failure. */
CRISPEMBED_API crispembed_context* crispembed_init(const char* model_path, int n_threads);

/* src/crispembed.h:68-74.  Accepted for ABI compatibility: this build has one
 * backend (CUDA); any other name is reported on stderr and ignored. */
CRISPEMBED_API void crispembed_set_gpu_backend(const char* name);

/* src/crispembed.h:76-79 / src/crispembed.cpp:2806.  Matryoshka output size,
 * 0 = model default. */
CRISPEMBED_API void crispembed_set_dim(crispembed_context* ctx, int dim);

/* src/crispembed.h:81-89 / src/crispembed.cpp:2810-2816 */
CRISPEMBED_API void crispembed_set_prefix(crispembed_context* ctx, const char* prefix);
CRISPEMBED_API const char* crispembed_get_prefix(const crispembed_context* ctx);

/* src/crispembed.h:103 / src/crispembed.cpp:2604 */
CRISPEMBED_API const crispembed_hparams* crispembed_get_hparams(const crispembed_context* ctx);

/* src/crispembed.h:128-131 / src/crispembed.cpp:2672.  WordPiece and
 * SentencePiece Unigram GGUFs (tokenizer.ggml.type 0 / 2, or the
 * tokenizer.ggml.model string); a BPE tokenizer returns NULL with a message. */
CRISPEMBED_API const float* crispembed_encode(crispembed_context* ctx, const char* text, int* out_n_dim);

/* src/crispembed.h:133-137 / src/crispembed.cpp:2856.  Flat [n_texts x dim]. */
CRISPEMBED_API const float* crispembed_encode_batch(crispembed_context* ctx, const char** texts, int n_texts,
                                                    int* out_n_dim);

/* src/crispembed.cpp:4938-4976 */
CRISPEMBED_API void crispembed_free(crispembed_context* ctx);

/* Per-token outputs, src/crispembed.h:189-211 / src/crispembed.cpp:3272-3393.
 * encode_tokens: the final hidden state of every token of `text` (prefix
 * applied, wrap tokens included), each row L2-normalised; _raw: unnormalised.
 * Flat [*out_n_tokens x *out_dim], ctx-owned until the next encode_tokens call.
 * last_token_ids: the [n_tokens] ids of that call.  token_str: the piece of an
 * id ("" out of range).  tokenizer_kind: 1 WordPiece, 2 SentencePiece, 3 BPE. */
CRISPEMBED_API const float* crispembed_encode_tokens(crispembed_context* ctx, const char* text, int* out_n_tokens,
                                                     int* out_dim);
CRISPEMBED_API const float* crispembed_encode_tokens_raw(crispembed_context* ctx, const char* text,
                                                         int* out_n_tokens, int* out_dim);
CRISPEMBED_API const int32_t* crispembed_last_token_ids(const crispembed_context* ctx);
CRISPEMBED_API const char* crispembed_token_str(const crispembed_context* ctx, int32_t id);
CRISPEMBED_API int crispembed_tokenizer_kind(const crispembed_context* ctx);

/* Capability queries the reference bindings call at setup
 * (src/crispembed.cpp:3009-3024): this build has no sparse/ColBERT/reranker
 * heads, so they return 0, and the head entry points fail cleanly. */
CRISPEMBED_API int crispembed_has_sparse(const crispembed_context* ctx);
CRISPEMBED_API int crispembed_has_colbert(const crispembed_context* ctx);
CRISPEMBED_API int crispembed_is_reranker(const crispembed_context* ctx);
CRISPEMBED_API int crispembed_encode_sparse(crispembed_context* ctx, const char* text, const int32_t** out_indices,
                                            const float** out_values);
CRISPEMBED_API const float* crispembed_encode_multivec(crispembed_context* ctx, const char* text, int* out_n_tokens,
                                                       int* out_dim);
CRISPEMBED_API float crispembed_rerank(crispembed_context* ctx, const char* query, const char* document);
/* src/crispembed.cpp:4279: ColBERT MaxSim over host vectors (pure function). */
CRISPEMBED_API float crispembed_colbert_score(const float* query_vecs, int n_query, const float* doc_vecs, int n_doc,
                                              int dim);

/* Model-registry helpers of src/crispembed.h:105-126.  No registry ships with
 * this build: resolve_model returns its argument, the table is empty. */
CRISPEMBED_API const char* crispembed_cache_dir(void);
CRISPEMBED_API const char* crispembed_resolve_model(const char* arg, int auto_download);
CRISPEMBED_API const char* crispembed_query_prefix(const char* model_name);
CRISPEMBED_API const char* crispembed_passage_prefix(const char* model_name);
CRISPEMBED_API const char* crispembed_ctx_query_prefix(const crispembed_context* ctx);
CRISPEMBED_API const char* crispembed_ctx_passage_prefix(const crispembed_context* ctx);
CRISPEMBED_API int crispembed_n_models(void);
CRISPEMBED_API const char* crispembed_model_name(int index);
CRISPEMBED_API const char* crispembed_model_desc(int index);
CRISPEMBED_API const char* crispembed_model_filename(int index);
CRISPEMBED_API const char* crispembed_model_size(int index);
CRISPEMBED_API const char* crispembed_model_license(int index);
CRISPEMBED_API const char* crispembed_model_card_url(int index);

/* ---- extensions (no counterpart in the reference ABI) ------------------- */

/* Token-id entry: n_seqs sequences, concatenated in h_ids, lengths in h_lens
 * (each 1..n_max_tokens).  Ids are used as given (no [CLS]/[SEP] added).
 * Returns ctx-owned [n_seqs x dim] L2-normalised embeddings, like
 * crispembed_encode_batch.  Host buffers in, host buffer out. */
CRISPEMBED_API const float* crispembed_encode_ids_batch(crispembed_context* ctx, const int32_t* h_ids,
                                                        const int32_t* h_lens, int n_seqs, int* out_n_dim);

/* Same computation on device-resident ids: d_ids [sum(h_lens)] on the context's
 * device, d_out [n_seqs x dim] floats (dim as reported by *out_n_dim).  Runs
 * asynchronously on `stream` (cudaStream_t as void*).  Returns 0 on success. */
CRISPEMBED_API int crispembed_encode_ids_device(crispembed_context* ctx, const int32_t* d_ids, const int32_t* h_lens,
                                                int n_seqs, float* d_out, int* out_n_dim, void* stream);

/* Stream used by the host-buffer entry points (cudaStream_t as void*). */
CRISPEMBED_API void* crispembed_stream(crispembed_context* ctx);

#ifdef __cplusplus
}
#endif
