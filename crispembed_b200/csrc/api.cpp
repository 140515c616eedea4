// api.cpp -- the extern "C" entry points of include/crispembed.h and
// include/ceb_ops.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#define CRISPEMBED_BUILD 1
#include "../../include/ceb_ops.h"
#include "../../include/crispembed.h"
#include "ceb_encoder_internal.h"
#include "gguf.h"
#include "tokenizer.h"

static_assert(sizeof(crispembed_hparams) == sizeof(ceb_hparams_c), "hparams layout");

int ceb_moe_static_take_error(int* code);  // moe_static.cu

struct crispembed_context {
    ceb_model model;
    ceb_workspace ws;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;  // fences around work moved off the legacy stream
    int device = 0;
    int* d_err = nullptr;
    int* h_err = nullptr;  // pinned copy of the device error word
    int n_threads = 1;
    std::string prefix;
    int matryoshka_dim = 0;
    ceb_tokenizer tok;
    // per-token results (crispembed_encode_tokens*)
    std::vector<float> last_tokens;
    std::vector<int32_t> last_token_ids;
    // CUDA graphs of the forward pass, one per batch shape seen twice (see run_device)
    struct Graph {
        int M = 0, n_seqs = 0, max_len = 0, out_dim = 0, variant = 0;
        const int32_t* d_ids = nullptr;
        float* d_out = nullptr;
        cudaStream_t st = nullptr;
        cudaGraphExec_t exec = nullptr;
        long long launches = 0, last_use = 0;
    };
    std::vector<Graph> graphs;
    std::vector<Graph> graph_seen;  // shapes met once (captured on the second call)
    void* graph_ws_base = nullptr;
    long long graph_clock = 0;
    // pinned staging for host-buffer calls
    int32_t* h_ids = nullptr;
    float* h_out = nullptr;
    size_t h_ids_cap = 0, h_out_cap = 0;
    // pinned staging of cu_seqlens, one slot per call in flight: a slot is written again
    // only after the event recorded behind its copy has completed
    struct CuSlot {
        int32_t* h = nullptr;
        size_t cap = 0;
        cudaEvent_t ev = nullptr;
    };
    static constexpr int N_CU_SLOTS = 4;
    CuSlot cu_slots[N_CU_SLOTS];
    unsigned cu_next = 0;
    cudaEvent_t ev_last = nullptr;  // end of the previous call's work: the workspace is shared
};

namespace {

int resolve_threads(int n) {
    if (n > 0) return n;
    unsigned hc = std::thread::hardware_concurrency();
    return (int)std::min(4u, hc ? hc : 1u);
}

int out_dim_of(const crispembed_context* ctx) {
    const int dim = ctx->model.hp.n_output > 0 ? ctx->model.hp.n_output : ctx->model.hp.n_embd;
    return (ctx->matryoshka_dim > 0 && ctx->matryoshka_dim < dim) ? ctx->matryoshka_dim : dim;
}

template <typename T>
int grow_pinned(T** p, size_t* cap, size_t n) {
    if (n <= *cap) return 0;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMallocHost((void**)p, n * sizeof(T)) != cudaSuccess) return ceb_set_error(4, "pinned host allocation failed");
    *cap = n;
    return 0;
}

// Checks the device error word written by bounded waits / index checks.
int check_device(crispembed_context* ctx, cudaStream_t st) {
    // the error word rides the stream behind the work (one synchronisation per call)
    cudaError_t e = cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "error word read", __FILE__, __LINE__);
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "stream synchronize", __FILE__, __LINE__);
    const int h = *ctx->h_err;
    if (h) {
        cudaMemset(ctx->d_err, 0, sizeof(int));
        return ceb_set_error(5, "device-side check failed (code 0x%x)", h);
    }
    return 0;
}

void drop_graphs(crispembed_context* ctx) {
    for (auto& g : ctx->graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    ctx->graphs.clear();
    ctx->graph_seen.clear();
}

bool graphs_enabled() {
    static const bool off = [] {
        const char* e = getenv("CEB_GRAPHS");
        return e && e[0] == '0';
    }();
    return !off;
}

// The forward pass of one batch.  Small batches are launch-bound (about a hundred
// kernels for a few microseconds of work each), so a batch shape met a second time
// -- same token and sequence counts, longest sequence, output width, id / output
// buffers and workspace -- is captured into a CUDA graph on that call and replayed
// from then on (every pointer and grid the kernels take is fixed by that key; ids
// and row offsets are uploaded into the fixed workspace buffers before the
// replay).  Not used while per-launch profiling runs, for expert-parallel contexts
// (each exchange carries a new epoch), or with CEB_GRAPHS=0.
int forward_maybe_graph(crispembed_context* ctx, const int32_t* d_ids, int n_seqs, int M, int max_len, float* d_out,
                        cudaStream_t st) {
    const int out_dim = out_dim_of(ctx);
    auto eager = [&] {
        return ceb_encoder_forward(ctx->model, ctx->ws, d_ids, ctx->ws.cu, n_seqs, M, max_len, d_out, out_dim,
                                   ctx->d_err, st);
    };
    if (!graphs_enabled() || ctx->model.ep || ceb_profiling_on()) return eager();
    if (ctx->graph_ws_base != ctx->ws.base) {  // a new workspace: every recorded pointer is stale
        drop_graphs(ctx);
        ctx->graph_ws_base = ctx->ws.base;
    }
    // the attention kernel is chosen per call: a graph records the one of its capture
    const char* tc = getenv("CEB_ATTN_TC");
    const char* mma = getenv("CEB_ATTN_MMA");
    const int variant = ((tc && tc[0] == '1') ? 1 : 0) | ((mma && mma[0] == '1') ? 2 : 0);
    auto same = [&](const crispembed_context::Graph& g) {
        return g.M == M && g.n_seqs == n_seqs && g.max_len == max_len && g.out_dim == out_dim && g.d_ids == d_ids &&
               g.d_out == d_out && g.st == st && g.variant == variant;
    };
    ++ctx->graph_clock;
    for (auto& g : ctx->graphs)
        if (same(g)) {
            g.last_use = ctx->graph_clock;
            const cudaError_t le = cudaGraphLaunch(g.exec, st);
            if (le != cudaSuccess) return ceb_set_cuda_error(le, "graph launch", __FILE__, __LINE__);
            ceb_count_launches(g.launches);
            return 0;
        }
    bool seen = false;
    for (auto& g : ctx->graph_seen) seen = seen || same(g);
    crispembed_context::Graph key;
    key.M = M;
    key.n_seqs = n_seqs;
    key.max_len = max_len;
    key.out_dim = out_dim;
    key.d_ids = d_ids;
    key.d_out = d_out;
    key.st = st;
    key.variant = variant;
    if (!seen) {
        if (ctx->graph_seen.size() >= 64) ctx->graph_seen.erase(ctx->graph_seen.begin());
        ctx->graph_seen.push_back(key);
        return eager();
    }
    const long long n0 = ceb_launch_count();
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return eager();
    }
    const int rc = eager();
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(st, &graph);
    if (rc || ce != cudaSuccess || !graph) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        return rc ? rc : eager();  // capture refused: the same work, launched directly
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
        cudaGetLastError();
        return eager();
    }
    key.exec = exec;
    key.launches = ceb_launch_count() - n0;
    key.last_use = ctx->graph_clock;
    if (ctx->graphs.size() >= 8) {  // keep the 8 most recently used shapes
        auto lru = std::min_element(ctx->graphs.begin(), ctx->graphs.end(),
                                    [](const auto& a, const auto& b) { return a.last_use < b.last_use; });
        cudaGraphExecDestroy(lru->exec);
        ctx->graphs.erase(lru);
    }
    ctx->graphs.push_back(key);
    const cudaError_t le = cudaGraphLaunch(exec, st);
    if (le != cudaSuccess) return ceb_set_cuda_error(le, "graph launch", __FILE__, __LINE__);
    return 0;
}

// Runs the encoder on device ids; cu_host [n_seqs+1] row offsets.
int run_device(crispembed_context* ctx, const int32_t* d_ids, const int32_t* h_lens, int n_seqs, float* d_out,
               cudaStream_t st) {
    if (n_seqs <= 0) return ceb_set_error(1, "no sequences");
    auto& slot = ctx->cu_slots[ctx->cu_next++ % crispembed_context::N_CU_SLOTS];
    if (!slot.ev && cudaEventCreateWithFlags(&slot.ev, cudaEventDisableTiming) != cudaSuccess)
        return ceb_set_error(3, "event creation failed");
    if (cudaEventSynchronize(slot.ev) != cudaSuccess) return ceb_set_error(3, "cu_seqlens staging wait failed");
    int rc = grow_pinned(&slot.h, &slot.cap, (size_t)n_seqs + 1);
    if (rc) return rc;
    int64_t M = 0;
    int max_len = 0;
    slot.h[0] = 0;
    for (int i = 0; i < n_seqs; ++i) {
        const int n = h_lens[i];
        if (n <= 0 || n > ctx->model.hp.n_max_tokens)
            return ceb_set_error(1, "sequence %d has %d tokens (allowed 1..%d)", i, n, ctx->model.hp.n_max_tokens);
        M += n;
        max_len = std::max(max_len, n);
        slot.h[i + 1] = (int32_t)M;
    }
    if (M > (1 << 30)) return ceb_set_error(1, "too many tokens");
    if ((rc = ceb_workspace_reserve(&ctx->ws, ctx->model, (int)M, n_seqs))) return rc;
    // The legacy default stream cannot be captured into a graph: its work runs on the
    // context's stream between two event fences, in the caller's stream order.
    const bool legacy = st == nullptr || st == cudaStreamLegacy;
    cudaStream_t run = legacy ? ctx->stream : st;
    if (legacy && (cudaEventRecord(ctx->ev_in, st) != cudaSuccess || cudaStreamWaitEvent(run, ctx->ev_in, 0) != cudaSuccess))
        return ceb_set_error(3, "stream fence failed");
    // calls on other streams share the workspace: this one starts after the previous one
    if (cudaStreamWaitEvent(run, ctx->ev_last, 0) != cudaSuccess) return ceb_set_error(3, "stream fence failed");
    cudaError_t e = cudaMemcpyAsync(ctx->ws.cu, slot.h, (size_t)(n_seqs + 1) * 4, cudaMemcpyHostToDevice, run);
    if (e == cudaSuccess) e = cudaEventRecord(slot.ev, run);
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "cu_seqlens upload", __FILE__, __LINE__);
    rc = forward_maybe_graph(ctx, d_ids, n_seqs, (int)M, max_len, d_out, run);
    if (cudaEventRecord(ctx->ev_last, run) != cudaSuccess) return rc ? rc : ceb_set_error(3, "stream fence failed");
    if (legacy && (cudaEventRecord(ctx->ev_out, run) != cudaSuccess || cudaStreamWaitEvent(st, ctx->ev_out, 0) != cudaSuccess))
        return rc ? rc : ceb_set_error(3, "stream fence failed");
    return rc;
}

// Batches above CEB_MAX_BATCH_TOKENS tokens (default 262144, at least the model's
// longest sequence) run as consecutive groups of whole sequences, so the
// activation workspace stays bounded; a sequence's embedding does not depend on
// the rest of its batch, so the result is that of one call.  Expert-parallel
// contexts run every call whole: all ranks take the same exchange steps.
int64_t max_batch_tokens(const crispembed_context* ctx) {
    int64_t cap = 262144;
    if (const char* e = getenv("CEB_MAX_BATCH_TOKENS")) {
        const long long v = atoll(e);
        if (v > 0) cap = v;
    }
    return std::max<int64_t>(cap, ctx->model.hp.n_max_tokens);
}

const float* encode_ids_host(crispembed_context* ctx, const int32_t* ids, const int32_t* lens, int n_seqs,
                             int* out_n_dim) {
    if (!ctx || !ids || !lens || n_seqs <= 0) return nullptr;
    int64_t M = 0;
    for (int i = 0; i < n_seqs; ++i) M += std::max(lens[i], 0);
    const int dim = out_dim_of(ctx);
    if (grow_pinned(&ctx->h_ids, &ctx->h_ids_cap, (size_t)std::max<int64_t>(M, 1)) ||
        grow_pinned(&ctx->h_out, &ctx->h_out_cap, (size_t)n_seqs * dim))
        return nullptr;
    int max_len = 0;
    for (int i = 0; i < n_seqs; ++i) max_len = std::max(max_len, lens[i]);
    if (max_len <= 0 || max_len > ctx->model.hp.n_max_tokens) {
        ceb_set_error(1, "sequence lengths must lie in 1..%d", ctx->model.hp.n_max_tokens);
        return nullptr;
    }
    // groups [first sequence, end) of at most `cap` tokens (one group unless the batch is larger)
    const int64_t cap = ctx->model.ep ? INT64_MAX : max_batch_tokens(ctx);
    std::vector<int> cut{0};
    int64_t g_tokens = 0, max_g_tokens = 0;
    int max_g_seqs = 0;
    for (int i = 0; i < n_seqs; ++i) {
        const int64_t n = std::max(lens[i], 0);
        if (i > cut.back() && g_tokens + n > cap) {
            cut.push_back(i);
            g_tokens = 0;
        }
        g_tokens += n;
        max_g_tokens = std::max(max_g_tokens, g_tokens);
        max_g_seqs = std::max(max_g_seqs, i + 1 - cut.back());
    }
    cut.push_back(n_seqs);
    if (max_g_tokens > (1 << 30)) {
        ceb_set_error(1, "too many tokens");
        return nullptr;
    }
    // the workspace must exist before the id uploads target it, sized for the largest group
    if (ceb_workspace_reserve(&ctx->ws, ctx->model, (int)max_g_tokens, max_g_seqs)) return nullptr;
    memcpy(ctx->h_ids, ids, (size_t)M * 4);
    cudaStream_t st = ctx->stream;
    int64_t t0 = 0;
    for (size_t g = 0; g + 1 < cut.size(); ++g) {
        const int s0 = cut[g], ns = cut[g + 1] - cut[g];
        int64_t m = 0;
        for (int i = s0; i < s0 + ns; ++i) m += std::max(lens[i], 0);
        // each group's ids come from their own part of the pinned buffer, its embeddings
        // land in their own rows: stream order alone separates the groups
        if (cudaMemcpyAsync(ctx->ws.ids, ctx->h_ids + t0, (size_t)m * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
            ceb_set_error(3, "id upload failed");
            return nullptr;
        }
        if (run_device(ctx, ctx->ws.ids, lens + s0, ns, ctx->ws.out, st)) return nullptr;
        if (cudaMemcpyAsync(ctx->h_out + (size_t)s0 * dim, ctx->ws.out, (size_t)ns * dim * 4, cudaMemcpyDeviceToHost,
                            st) != cudaSuccess) {
            ceb_set_error(3, "embedding download failed");
            return nullptr;
        }
        t0 += m;
    }
    if (check_device(ctx, st)) return nullptr;
    if (out_n_dim) *out_n_dim = dim;
    return ctx->h_out;  // pinned, owned by the context, valid until the next call
}

const float* encode_texts(crispembed_context* ctx, const char** texts, int n, int* out_n_dim) {
    std::vector<int32_t> ids, lens, t;
    for (int i = 0; i < n; ++i) {
        if (ctx->tok.encode(ctx->prefix + (texts[i] ? texts[i] : ""), &t)) return nullptr;
        lens.push_back((int32_t)t.size());
        ids.insert(ids.end(), t.begin(), t.end());
    }
    return encode_ids_host(ctx, ids.data(), lens.data(), n, out_n_dim);
}

// Final hidden states [T x d] of one tokenized text (the reference's encode_tokens
// path, src/crispembed.cpp:3272-3373): the encoder runs as for a batch of one and
// the last layer's output rows are copied back; `normalize` L2-normalises each row
// as the reference does (sum of squares in float, sqrt(max(., 1e-12))).
const float* encode_tokens(crispembed_context* ctx, const char* text, int* out_n_tokens, int* out_dim,
                           bool normalize) {
    if (out_n_tokens) *out_n_tokens = 0;
    if (out_dim) *out_dim = 0;
    if (!ctx || !text) return nullptr;
    std::vector<int32_t> ids;
    if (ctx->tok.encode(ctx->prefix + text, &ids)) return nullptr;
    if (ids.empty()) return nullptr;
    const int T = (int)ids.size();
    if (!encode_ids_host(ctx, ids.data(), &T, 1, nullptr)) return nullptr;
    const int d = ctx->model.hp.n_embd;
    ctx->last_tokens.resize((size_t)T * d);
    cudaStream_t st = ctx->stream;
    if (cudaMemcpyAsync(ctx->last_tokens.data(), ctx->ws.x32, (size_t)T * d * 4, cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        ceb_set_error(3, "hidden-state download failed");
        return nullptr;
    }
    if (normalize)
        for (int t = 0; t < T; ++t) {
            float* v = ctx->last_tokens.data() + (size_t)t * d;
            float ss = 0.0f;
            for (int j = 0; j < d; ++j) ss += v[j] * v[j];
            const float nrm = std::sqrt(std::max(ss, 1e-12f));
            for (int j = 0; j < d; ++j) v[j] /= nrm;
        }
    ctx->last_token_ids = ids;
    if (out_n_tokens) *out_n_tokens = T;
    if (out_dim) *out_dim = d;
    return ctx->last_tokens.data();
}

std::string g_str;  // backing store for the registry helpers

}  // namespace

// =========================================================== crispembed.h ===
extern "C" crispembed_context* crispembed_init(const char* model_path, int n_threads) {
    const char* ra = getenv("CEB_REFERENCE_ARITHMETIC");
    return ceb_init_ex(model_path, n_threads, (ra && ra[0] == '1') ? CEB_INIT_REFERENCE_ARITHMETIC : 0);
}

extern "C" crispembed_context* ceb_init_ex(const char* model_path, int n_threads, int flags) {
    if (!model_path) return nullptr;
    if (flags & ~CEB_INIT_REFERENCE_ARITHMETIC) {
        ceb_set_error(1, "init: unknown flags 0x%x", flags);
        return nullptr;
    }
    auto* ctx = new crispembed_context;
    ctx->model.ref_arith = (flags & CEB_INIT_REFERENCE_ARITHMETIC) != 0;
    ctx->n_threads = resolve_threads(n_threads);
    if (cudaGetDevice(&ctx->device) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
        ceb_set_error(3, "no CUDA device available");
        delete ctx;
        return nullptr;
    }
    std::string err;
    if (ceb_model_load(&ctx->model, model_path, &err)) {
        delete ctx;
        return nullptr;
    }
    {
        ceb_gguf g;
        if (!g.open(model_path, &err) || ctx->tok.load(g, ctx->model.hp.n_max_tokens)) {
            if (!err.empty()) ceb_set_error(1, "%s", err.c_str());
            ceb_model_free(&ctx->model);
            delete ctx;
            return nullptr;
        }
    }
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess || cudaMemset(ctx->d_err, 0, sizeof(int)) != cudaSuccess ||
        cudaMallocHost((void**)&ctx->h_err, sizeof(int)) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_out, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_last, cudaEventDisableTiming) != cudaSuccess) {
        ceb_set_error(3, "context setup failed");
        crispembed_free(ctx);
        return nullptr;
    }
    int moe = 0;
    for (const auto& Ly : ctx->model.layers) moe += Ly.moe;
    fprintf(stderr, "crispembed-b200: loaded %d layers (%d MoE, %d experts top-%d), %d dims, %d vocab, %.1f MB weights%s\n",
            ctx->model.hp.n_layer, moe, ctx->model.hp.n_experts, ctx->model.hp.n_experts_per_tok,
            ctx->model.hp.n_embd, ctx->model.hp.n_vocab, ctx->model.weight_bytes / 1e6,
            ctx->model.ref_arith ? ", reference arithmetic" : "");
    return ctx;
}

extern "C" void crispembed_set_gpu_backend(const char* name) {
    if (name && name[0] && strcasecmp(name, "cuda") != 0)
        fprintf(stderr, "crispembed-b200: backend '%s' not available, using CUDA\n", name);
}

extern "C" void crispembed_set_dim(crispembed_context* ctx, int dim) {
    if (ctx) ctx->matryoshka_dim = dim;
}

extern "C" void crispembed_set_prefix(crispembed_context* ctx, const char* prefix) {
    if (ctx) ctx->prefix = prefix ? prefix : "";
}

extern "C" const char* crispembed_get_prefix(const crispembed_context* ctx) { return ctx ? ctx->prefix.c_str() : ""; }

extern "C" const crispembed_hparams* crispembed_get_hparams(const crispembed_context* ctx) {
    return ctx ? reinterpret_cast<const crispembed_hparams*>(&ctx->model.hp) : nullptr;
}

extern "C" const float* crispembed_encode(crispembed_context* ctx, const char* text, int* out_n_dim) {
    if (!ctx || !text) return nullptr;
    const char* t[1] = {text};
    return encode_texts(ctx, t, 1, out_n_dim);
}

extern "C" const float* crispembed_encode_batch(crispembed_context* ctx, const char** texts, int n_texts,
                                                int* out_n_dim) {
    if (!ctx || !texts || n_texts <= 0) return nullptr;
    return encode_texts(ctx, texts, n_texts, out_n_dim);
}

extern "C" const float* crispembed_encode_ids_batch(crispembed_context* ctx, const int32_t* h_ids,
                                                    const int32_t* h_lens, int n_seqs, int* out_n_dim) {
    return encode_ids_host(ctx, h_ids, h_lens, n_seqs, out_n_dim);
}

extern "C" int crispembed_encode_ids_device(crispembed_context* ctx, const int32_t* d_ids, const int32_t* h_lens,
                                            int n_seqs, float* d_out, int* out_n_dim, void* stream) {
    if (!ctx || !d_ids || !h_lens || !d_out) return ceb_set_error(1, "null argument");
    if (out_n_dim) *out_n_dim = out_dim_of(ctx);
    return run_device(ctx, d_ids, h_lens, n_seqs, d_out, static_cast<cudaStream_t>(stream));
}

extern "C" int ceb_moe_block_count(const crispembed_context* ctx) {
    int n = 0;
    if (ctx)
        for (const auto& Ly : ctx->model.layers) n += Ly.moe;
    return n;
}

extern "C" int ceb_encode_ids_routes(crispembed_context* ctx, const int32_t* h_ids, const int32_t* h_lens, int n_seqs,
                                     float* h_out, int32_t* h_route_ids, float* h_route_logits) {
    if (!ctx || !h_ids || !h_lens || n_seqs <= 0) return ceb_set_error(1, "encode_ids_routes: bad arguments");
    if (ctx->model.ep) return ceb_set_error(1, "encode_ids_routes: not available on an expert-parallel context");
    int n_moe = 0, E = 0, K = 0;
    for (const auto& Ly : ctx->model.layers)
        if (Ly.moe) {
            ++n_moe;
            E = Ly.moew.n_experts;
            K = Ly.moew.top_k;
        }
    std::vector<int32_t> cu((size_t)n_seqs + 1, 0);
    int max_len = 0;
    for (int i = 0; i < n_seqs; ++i) {
        if (h_lens[i] <= 0 || h_lens[i] > ctx->model.hp.n_max_tokens)
            return ceb_set_error(1, "sequence %d has %d tokens (allowed 1..%d)", i, h_lens[i], ctx->model.hp.n_max_tokens);
        cu[(size_t)i + 1] = cu[(size_t)i] + h_lens[i];
        max_len = std::max(max_len, (int)h_lens[i]);
    }
    const int M = cu[(size_t)n_seqs];
    int rc = ceb_workspace_reserve(&ctx->ws, ctx->model, M, n_seqs);
    if (rc) return rc;
    cudaStream_t st = ctx->stream;
    if (cudaStreamSynchronize(st) != cudaSuccess) return ceb_set_error(3, "stream synchronize");
    ceb_route_capture cap;
    const size_t ids_bytes = (size_t)n_moe * M * K * 4, lg_bytes = (size_t)n_moe * M * E * 4;
    if (n_moe && (cudaMalloc(&cap.ids, ids_bytes) != cudaSuccess || cudaMalloc(&cap.logits, lg_bytes) != cudaSuccess)) {
        cudaFree(cap.ids);
        return ceb_set_error(4, "encode_ids_routes: out of device memory");
    }
    const int dim = out_dim_of(ctx);
    cudaError_t e = cudaMemcpyAsync(ctx->ws.ids, h_ids, (size_t)M * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->ws.cu, cu.data(), cu.size() * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) rc = ceb_set_cuda_error(e, "encode_ids_routes upload", __FILE__, __LINE__);
    if (!rc)
        rc = ceb_encoder_forward(ctx->model, ctx->ws, ctx->ws.ids, ctx->ws.cu, n_seqs, M, max_len, ctx->ws.out, dim,
                                 ctx->d_err, st, &cap);
    if (!rc && h_out) e = cudaMemcpyAsync(h_out, ctx->ws.out, (size_t)n_seqs * dim * 4, cudaMemcpyDeviceToHost, st);
    if (!rc && n_moe && h_route_ids && e == cudaSuccess)
        e = cudaMemcpyAsync(h_route_ids, cap.ids, ids_bytes, cudaMemcpyDeviceToHost, st);
    if (!rc && n_moe && h_route_logits && e == cudaSuccess)
        e = cudaMemcpyAsync(h_route_logits, cap.logits, lg_bytes, cudaMemcpyDeviceToHost, st);
    if (!rc && e != cudaSuccess) rc = ceb_set_cuda_error(e, "encode_ids_routes download", __FILE__, __LINE__);
    if (!rc) rc = check_device(ctx, st);
    cudaStreamSynchronize(st);
    cudaFree(cap.ids);
    cudaFree(cap.logits);
    return rc;
}

extern "C" void* crispembed_stream(crispembed_context* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

extern "C" void crispembed_free(crispembed_context* ctx) {
    if (!ctx) return;
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    drop_graphs(ctx);
    ceb_workspace_free(&ctx->ws);
    ceb_model_free(&ctx->model);
    if (ctx->d_err) cudaFree(ctx->d_err);
    if (ctx->h_ids) cudaFreeHost(ctx->h_ids);
    for (auto& slot : ctx->cu_slots) {
        if (slot.h) cudaFreeHost(slot.h);
        if (slot.ev) cudaEventDestroy(slot.ev);
    }
    if (ctx->ev_last) cudaEventDestroy(ctx->ev_last);
    if (ctx->h_out) cudaFreeHost(ctx->h_out);
    if (ctx->h_err) cudaFreeHost(ctx->h_err);
    if (ctx->ev_in) cudaEventDestroy(ctx->ev_in);
    if (ctx->ev_out) cudaEventDestroy(ctx->ev_out);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

extern "C" const float* crispembed_encode_tokens(crispembed_context* ctx, const char* text, int* out_n_tokens,
                                                 int* out_dim) {
    return encode_tokens(ctx, text, out_n_tokens, out_dim, true);
}

extern "C" const float* crispembed_encode_tokens_raw(crispembed_context* ctx, const char* text, int* out_n_tokens,
                                                     int* out_dim) {
    return encode_tokens(ctx, text, out_n_tokens, out_dim, false);
}

extern "C" const int32_t* crispembed_last_token_ids(const crispembed_context* ctx) {
    return (ctx && !ctx->last_token_ids.empty()) ? ctx->last_token_ids.data() : nullptr;
}

extern "C" const char* crispembed_token_str(const crispembed_context* ctx, int32_t id) {
    return ctx ? ctx->tok.token_str(id).c_str() : nullptr;
}

extern "C" int crispembed_tokenizer_kind(const crispembed_context* ctx) { return ctx ? ctx->tok.kind() : 0; }

extern "C" int crispembed_has_sparse(const crispembed_context*) { return 0; }
extern "C" int crispembed_has_colbert(const crispembed_context*) { return 0; }
extern "C" int crispembed_is_reranker(const crispembed_context*) { return 0; }
extern "C" int crispembed_encode_sparse(crispembed_context*, const char*, const int32_t**, const float**) { return 0; }
extern "C" const float* crispembed_encode_multivec(crispembed_context*, const char*, int* out_n_tokens, int* out_dim) {
    if (out_n_tokens) *out_n_tokens = 0;
    if (out_dim) *out_dim = 0;
    return nullptr;
}
extern "C" float crispembed_rerank(crispembed_context*, const char*, const char*) {
    ceb_set_error(1, "this model has no reranker head");
    return NAN;
}
extern "C" float crispembed_colbert_score(const float* q, int n_query, const float* dv, int n_doc, int dim) {
    float score = 0.0f;
    for (int qi = 0; qi < n_query; qi++) {
        float best = -1e30f;
        for (int di = 0; di < n_doc; di++) {
            float dot = 0.0f;
            for (int k = 0; k < dim; k++) dot += q[(size_t)qi * dim + k] * dv[(size_t)di * dim + k];
            best = std::max(best, dot);
        }
        score += best;
    }
    return score;
}

extern "C" const char* crispembed_cache_dir(void) {
    const char* h = getenv("CRISPEMBED_CACHE_DIR");
    g_str = h ? h : "";
    return g_str.c_str();
}
extern "C" const char* crispembed_resolve_model(const char* arg, int) {
    g_str = arg ? arg : "";
    return g_str.c_str();
}
extern "C" const char* crispembed_query_prefix(const char*) { return nullptr; }
extern "C" const char* crispembed_passage_prefix(const char*) { return nullptr; }
extern "C" const char* crispembed_ctx_query_prefix(const crispembed_context*) { return nullptr; }
extern "C" const char* crispembed_ctx_passage_prefix(const crispembed_context*) { return nullptr; }
extern "C" int crispembed_n_models(void) { return 0; }
extern "C" const char* crispembed_model_name(int) { return ""; }
extern "C" const char* crispembed_model_desc(int) { return ""; }
extern "C" const char* crispembed_model_filename(int) { return ""; }
extern "C" const char* crispembed_model_size(int) { return ""; }
extern "C" const char* crispembed_model_license(int) { return ""; }
extern "C" const char* crispembed_model_card_url(int) { return ""; }

// ============================================================= ceb_ops.h ===
extern "C" ceb_moe_layer* ceb_moe_layer_create(int d, int n_experts, int top_k, int ffn, int router_type,
                                               const void* h_router, int expert_type, const void* h_fc1,
                                               const void* h_fc2, const float* h_bias) {
    if (d <= 0 || n_experts <= 0 || n_experts > 32 || top_k <= 0 || top_k > 4 || top_k > n_experts || ffn <= 0 ||
        !h_router || !h_fc1 || !h_fc2) {
        ceb_set_error(1, "moe_layer_create: bad arguments");
        return nullptr;
    }
    if (router_type != CEB_TYPE_F32 && router_type != CEB_TYPE_Q8_0) {
        ceb_set_error(1, "moe_layer_create: router type %d unsupported (F32 or Q8_0)", router_type);
        return nullptr;
    }
    if (d % 128 || ffn % 128 || (expert_type == CEB_TYPE_Q4_K && (d % 256 || ffn % 256))) {
        ceb_set_error(2, "moe_layer_create: d=%d ffn=%d must be multiples of 128 (256 for Q4_K)", d, ffn);
        return nullptr;
    }
    auto* L = new ceb_moe_layer;
    L->w.d = d;
    L->w.n_experts = n_experts;
    L->w.top_k = top_k;
    L->w.ffn = ffn;
    L->w.router_type = router_type;
    const int64_t rrb = router_type == CEB_TYPE_F32 ? (int64_t)d * 4 : (int64_t)d / 32 * 34;
    const size_t rbytes = (size_t)(rrb * n_experts);
    void* p = nullptr;
    int rc = 0;
    if (cudaMalloc(&p, rbytes) != cudaSuccess) rc = ceb_set_error(4, "out of device memory");
    else {
        L->allocs.push_back(p);
        L->w.router = static_cast<uint8_t*>(p);
        if (cudaMemcpy(p, h_router, rbytes, cudaMemcpyHostToDevice) != cudaSuccess) rc = ceb_set_error(3, "upload");
    }
    if (!rc) rc = ceb_repack_weights(&L->w.fc1, expert_type, h_fc1, n_experts, ffn, d, nullptr);
    if (!rc) rc = ceb_repack_weights(&L->w.fc2, expert_type, h_fc2, n_experts, d, ffn, nullptr);
    if (!rc && h_bias) {
        if (cudaMalloc(&p, (size_t)d * 4) != cudaSuccess) rc = ceb_set_error(4, "out of device memory");
        else {
            L->allocs.push_back(p);
            L->w.bias = static_cast<float*>(p);
            if (cudaMemcpy(p, h_bias, (size_t)d * 4, cudaMemcpyHostToDevice) != cudaSuccess)
                rc = ceb_set_error(3, "upload");
        }
    }
    if (rc) {
        ceb_moe_layer_free(L);
        return nullptr;
    }
    return L;
}

extern "C" void ceb_moe_layer_free(ceb_moe_layer* L) {
    if (!L) return;
    ceb_wplane_free(&L->w.fc1);
    ceb_wplane_free(&L->w.fc2);
    for (void* p : L->allocs) cudaFree(p);
    delete L;
}

extern "C" size_t ceb_moe_workspace_size(const ceb_moe_layer* L, int max_tokens) {
    if (!L || max_tokens <= 0) return 0;
    return ceb_moe_ws_layout(max_tokens, L->w.d, L->w.n_experts, L->w.top_k, L->w.ffn, nullptr, nullptr);
}

extern "C" int ceb_moe_workspace_routing(const ceb_moe_layer* L, int n_tokens, void* d_workspace, int32_t** d_ids,
                                         float** d_weights, int32_t** d_slot_pos, int32_t** d_offsets) {
    if (!L || n_tokens <= 0 || !d_workspace) return ceb_set_error(1, "moe_workspace_routing: bad arguments");
    ceb_moe_ws ws;
    ceb_moe_ws_layout(n_tokens, L->w.d, L->w.n_experts, L->w.top_k, L->w.ffn, &ws, static_cast<uint8_t*>(d_workspace));
    if (d_ids) *d_ids = ws.ids;
    if (d_weights) *d_weights = ws.wts;
    if (d_slot_pos) *d_slot_pos = ws.slot_pos;
    if (d_offsets) *d_offsets = ws.offsets;
    return 0;
}

namespace {
// Device error words of the operator-level calls, one per device: kernels write
// the word of the device they run on, and ceb_sync_check reads the current
// device's (a process may drive several GPUs).
constexpr int OP_MAX_DEVICES = 64;
int* g_op_err[OP_MAX_DEVICES] = {};
std::mutex g_op_mu;
int* op_err_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= OP_MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lk(g_op_mu);
    if (!g_op_err[dev]) {
        int* p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
            cudaFree(p);
            return nullptr;
        }
        g_op_err[dev] = p;
    }
    return g_op_err[dev];
}
}  // namespace

int* ceb_op_error_word() { return op_err_word(); }

namespace {
// Work-item counters of the operator-level attention entry, one pair per (device, stream):
// launches on one stream run in order and share theirs, launches on different streams do
// not (the kernel returns its counter to zero when it ends).
struct SchedKey {
    int dev;
    cudaStream_t st;
    bool operator<(const SchedKey& o) const { return dev != o.dev ? dev < o.dev : st < o.st; }
};
std::map<SchedKey, int*> g_attn_sched;
int* attn_sched_words(cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_op_mu);
    int*& p = g_attn_sched[SchedKey{dev, st}];
    if (!p) {
        if (cudaMalloc(&p, 2 * sizeof(int)) != cudaSuccess) {
            p = nullptr;
            return nullptr;
        }
        if (cudaMemset(p, 0, 2 * sizeof(int)) != cudaSuccess) {
            cudaFree(p);
            p = nullptr;
            return nullptr;
        }
    }
    return p;
}
}  // namespace

extern "C" int ceb_moe_ffn(const ceb_moe_layer* L, const void* d_x, int x_dtype, int n_tokens, float* d_y,
                           int32_t* d_ids, float* d_weights, int32_t* d_expert_counts, float* d_logits,
                           void* d_workspace, size_t workspace_bytes, void* stream) {
    if (!L || !d_x || !d_y || n_tokens < 0 || (n_tokens > 0 && !d_workspace))
        return ceb_set_error(1, "moe_ffn: bad arguments");
    if (x_dtype != CEB_ACT_F32 && x_dtype != CEB_ACT_BF16 && x_dtype != CEB_ACT_F16)
        return ceb_set_error(1, "moe_ffn: x_dtype %d unsupported", x_dtype);
    if (n_tokens == 0) return 0;
    const size_t need = ceb_moe_workspace_size(L, n_tokens);
    if (workspace_bytes < need)
        return ceb_set_error(1, "moe_ffn: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(d_workspace) & 255) return ceb_set_error(1, "moe_ffn: workspace not 256-B aligned");
    int* err = op_err_word();
    if (!err) return ceb_set_error(4, "out of device memory");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ceb_moe_ws ws;
    ceb_moe_ws_layout(n_tokens, L->w.d, L->w.n_experts, L->w.top_k, L->w.ffn, &ws, static_cast<uint8_t*>(d_workspace));
    int rc = ceb_moe_run(L->w, d_x, x_dtype, nullptr, n_tokens, d_y, ws, d_expert_counts, d_logits, err, st);
    if (rc) return rc;
    const size_t S = (size_t)n_tokens * L->w.top_k;
    if (d_ids && cudaMemcpyAsync(d_ids, ws.ids, S * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ceb_set_error(3, "ids copy");
    if (d_weights && cudaMemcpyAsync(d_weights, ws.wts, S * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ceb_set_error(3, "weights copy");
    return 0;
}

extern "C" int ceb_moe_route_ln(const ceb_moe_layer* L, const float* d_res, const float* d_y, int n_tokens,
                                const float* d_gamma, const float* d_beta, float eps, float* d_out, void* d_out16,
                                int32_t* d_ids, float* d_weights, float* d_logits, void* d_workspace,
                                size_t workspace_bytes, void* stream) {
    if (!L || !d_res || !d_y || !d_out || n_tokens < 0 || (n_tokens > 0 && !d_workspace))
        return ceb_set_error(1, "moe_route_ln: bad arguments");
    if (n_tokens == 0) return 0;
    const size_t need = ceb_moe_workspace_size(L, n_tokens);
    if (workspace_bytes < need)
        return ceb_set_error(1, "moe_route_ln: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(d_workspace) & 255)
        return ceb_set_error(1, "moe_route_ln: workspace not 256-B aligned");
    if ((reinterpret_cast<uintptr_t>(d_res) | reinterpret_cast<uintptr_t>(d_y) | reinterpret_cast<uintptr_t>(d_out) |
         reinterpret_cast<uintptr_t>(d_out16) | reinterpret_cast<uintptr_t>(d_gamma) |
         reinterpret_cast<uintptr_t>(d_beta)) & 15)
        return ceb_set_error(1, "moe_route_ln: rows must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ceb_moe_ws ws;
    ceb_moe_ws_layout(n_tokens, L->w.d, L->w.n_experts, L->w.top_k, L->w.ffn, &ws, static_cast<uint8_t*>(d_workspace));
    int rc = ceb_add_ln_route(d_res, d_y, false, n_tokens, L->w.d, d_gamma, d_beta, eps, d_out, static_cast<__half*>(d_out16),
                              L->w, ws, d_logits, st);
    if (rc) return rc;
    const size_t S = (size_t)n_tokens * L->w.top_k;
    if (d_ids && cudaMemcpyAsync(d_ids, ws.ids, S * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ceb_set_error(3, "ids copy");
    if (d_weights && cudaMemcpyAsync(d_weights, ws.wts, S * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ceb_set_error(3, "weights copy");
    return 0;
}

extern "C" int ceb_ep_attach(crispembed_context* ctx, ceb_ep* ep) {
    if (!ctx || !ep) return ceb_set_error(1, "ep_attach: bad arguments");
    if (ctx->model.ref_arith) return ceb_set_error(1, "ep_attach: not available with reference arithmetic");
    cudaSetDevice(ctx->device);
    return ceb_model_ep_attach(&ctx->model, ep);
}

extern "C" int ceb_gguf_dequantize(int ggml_type, const void* h_src, int64_t n_rows, int64_t k, float* h_dst) {
    const int64_t rb = ceb_ggml_row_bytes(ggml_type, k);
    if (!h_src || !h_dst || n_rows < 0 || rb < 0)
        return ceb_set_error(1, "gguf_dequantize: type %d with rows of %lld values unsupported", ggml_type,
                             (long long)k);
    const uint8_t* src = static_cast<const uint8_t*>(h_src);
    for (int64_t r = 0; r < n_rows; ++r) ceb_ggml_dequant_row(ggml_type, src + r * rb, k, h_dst + r * k);
    return 0;
}

extern "C" int ceb_pool_l2(const float* d_hidden, const int32_t* d_cu_seqlens, int n_seqs, int d, int out_dim,
                           float* d_out, void* stream) {
    if (!d_hidden || !d_cu_seqlens || !d_out || n_seqs < 0 || d <= 0) return ceb_set_error(1, "pool_l2: bad arguments");
    return ceb_pool_l2_launch(d_hidden, d_cu_seqlens, n_seqs, d, out_dim, d_out, static_cast<cudaStream_t>(stream), 0);
}

extern "C" int ceb_attention_forward(const void* d_qkv, int n_rows, const int32_t* d_cu_seqlens, int n_seqs,
                                     int max_len, int d, int n_head, void* d_out, void* stream) {
    if (!d_qkv || !d_cu_seqlens || !d_out || n_rows < 0 || n_seqs < 0 || max_len < 0)
        return ceb_set_error(1, "attention: bad arguments");
    if (n_rows == 0 || n_seqs == 0) return 0;
    if ((reinterpret_cast<uintptr_t>(d_qkv) | reinterpret_cast<uintptr_t>(d_out)) & 15)
        return ceb_set_error(1, "attention: qkv and out must be 16-byte aligned");
    int* err = op_err_word();
    if (!err) return ceb_set_error(3, "attention: device error word");
    int* sched = attn_sched_words(static_cast<cudaStream_t>(stream));
    if (!sched) return ceb_set_error(3, "attention: work-item counter");
    return ceb_attention(static_cast<const __half*>(d_qkv), n_rows, d_cu_seqlens, n_seqs, max_len, d, n_head,
                         static_cast<__half*>(d_out), err, static_cast<cudaStream_t>(stream), sched);
}

struct ceb_linear {
    ceb_wplane w;
};

extern "C" ceb_linear* ceb_linear_create(int w_type, const void* h_w, int n_out, int k) {
    if (!h_w || n_out <= 0 || k <= 0) {
        ceb_set_error(1, "linear_create: bad arguments");
        return nullptr;
    }
    auto* L = new ceb_linear;
    if (ceb_repack_weights(&L->w, w_type, h_w, 1, n_out, k, nullptr)) {
        delete L;
        return nullptr;
    }
    return L;
}

extern "C" int ceb_linear_forward(const ceb_linear* L, const void* d_x, int m, const float* d_bias, int gelu,
                                  int out_f16, void* d_out, void* stream) {
    if (m == 0) return 0;
    if (!L || !d_x || !d_out || m < 0) return ceb_set_error(1, "linear_forward: bad arguments");
    int* err = op_err_word();
    if (!err) return ceb_set_error(4, "out of device memory");
    ceb_gemm_args a;
    a.m_rows = m;
    a.out = d_out;
    a.ldo = L->w.n_out;
    a.epi = (out_f16 ? CEB_EPI_F16_OUT : 0) | (gelu ? CEB_EPI_GELU : 0) | (d_bias ? CEB_EPI_BIAS : 0);
    a.bias = d_bias;
    a.err = err;
    return ceb_gemm_launch(L->w, d_x, m, a, static_cast<cudaStream_t>(stream));
}

extern "C" void ceb_linear_free(ceb_linear* L) {
    if (!L) return;
    ceb_wplane_free(&L->w);
    delete L;
}

extern "C" int ceb_matmul(int w_type, const void* h_w, int n_out, int k, const void* d_x, int m, const float* d_bias,
                          int gelu, int out_f16, void* d_out, void* stream) {
    if (m == 0) return 0;
    if (!h_w || !d_x || !d_out || m < 0) return ceb_set_error(1, "matmul: bad arguments");
    int* err = op_err_word();
    if (!err) return ceb_set_error(4, "out of device memory");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ceb_wplane w;
    int rc = ceb_repack_weights(&w, w_type, h_w, 1, n_out, k, st);
    if (rc) return rc;
    ceb_gemm_args a;
    a.m_rows = m;
    a.out = d_out;
    a.ldo = n_out;
    a.epi = (out_f16 ? CEB_EPI_F16_OUT : 0) | (gelu ? CEB_EPI_GELU : 0) | (d_bias ? CEB_EPI_BIAS : 0);
    a.bias = d_bias;
    a.err = err;
    rc = ceb_gemm_launch(w, d_x, m, a, st);
    cudaError_t e = cudaStreamSynchronize(st);
    ceb_wplane_free(&w);
    if (rc) return rc;
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "matmul", __FILE__, __LINE__);
    return 0;
}

extern "C" const char* ceb_last_error(void) { return ceb_last_error_message(); }

extern "C" int ceb_sync_check(void* stream) {
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "stream synchronize", __FILE__, __LINE__);
    e = cudaGetLastError();
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "pending error", __FILE__, __LINE__);
    // both device error words of the current device are read and cleared, so a pending
    // error is reported once, by this call
    int hs = 0, h = 0;
    const int rs = ceb_moe_static_take_error(&hs);
    int ro = 0;
    if (int* err = op_err_word()) {
        if (cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) ro = 3;
        else if (h && cudaMemset(err, 0, sizeof(int)) != cudaSuccess) ro = 3;
    } else {
        ro = 3;
    }
    if (hs && h)
        return ceb_set_error(5, "device-side checks failed: operator code 0x%x, ceb_moe_ffn_static code 0x%x", h, hs);
    if (h) return ceb_set_error(5, "device-side check failed (code 0x%x)", h);
    if (hs) return ceb_set_error(5, "device-side check failed in ceb_moe_ffn_static (code 0x%x)", hs);
    if (rs || ro) return ceb_set_error(3, "device error word could not be read");
    return 0;
}

// ---------------------------------------------------- tokenizer (no device needed)
struct ceb_text_tokenizer {
    ceb_tokenizer tok;
};

extern "C" ceb_text_tokenizer* ceb_tokenizer_load(const char* gguf_path, int max_tokens) {
    if (!gguf_path) return nullptr;
    ceb_gguf g;
    std::string err;
    if (!g.open(gguf_path, &err)) {
        ceb_set_error(1, "%s", err.c_str());
        return nullptr;
    }
    auto* t = new ceb_text_tokenizer;
    if (t->tok.load(g, max_tokens)) {
        delete t;
        return nullptr;
    }
    return t;
}

extern "C" int ceb_tokenizer_encode(const ceb_text_tokenizer* t, const char* text, int32_t* ids, int cap) {
    if (!t || !text) return ceb_set_error(1, "null argument"), -1;
    std::vector<int32_t> v;
    if (t->tok.encode(text, &v)) return -1;
    const int n = (int)v.size();
    for (int i = 0; i < n && i < cap; ++i) ids[i] = v[i];
    return n;
}

extern "C" int ceb_tokenizer_kind_of(const ceb_text_tokenizer* t) { return t ? t->tok.kind() : 0; }

extern "C" void ceb_tokenizer_free(ceb_text_tokenizer* t) { delete t; }
