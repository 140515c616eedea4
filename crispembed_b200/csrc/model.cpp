// model.cpp -- GGUF model binding, device upload and the encoder forward pass.
//
// Metadata and tensor-name resolution follow the reference's load_model
// (src/crispembed.cpp:437-526 hparams incl. arch-derived "<arch>.*" keys,
// :456-471 pooling, :748-845 tensor names in CrispEmbed-native "enc.N.*" and
// llama.cpp "blk.N.*" spellings, :208-245 validation).  The forward pass follows
// build_encoder_graph for post-LN NomicBERT(-MoE) with learned positions
// (src/crispembed.cpp:1068-1428) and encode_tokens' pooling (:1794-1846).
#include <cuda_runtime.h>

#include <cstdio>
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "ceb_encoder_internal.h"
#include "ceb_ep_internal.h"
#include "gguf.h"

namespace {

struct Loader {
    const ceb_gguf& g;
    ceb_model* m;
    std::string arch;
    cudaStream_t st = nullptr;

    const ceb_gguf_tensor* any(std::initializer_list<std::string> names) const {
        for (const auto& n : names)
            if (const ceb_gguf_tensor* t = g.tensor(n)) return t;
        return nullptr;
    }
    int u32(std::initializer_list<std::string> keys, int def) const {
        for (const auto& k : keys) {
            int v;
            if (!k.empty() && g.get_u32(k, &v)) return v;
        }
        return def;
    }
    float f32(std::initializer_list<std::string> keys, float def) const {
        for (const auto& k : keys) {
            float v;
            if (!k.empty() && g.get_f32(k, &v)) return v;
        }
        return def;
    }
    std::string ak(const char* field) const { return arch.empty() ? std::string() : arch + "." + field; }

    // float vector upload (F32 tensor, or F16 widened); nullptr if absent
    int upload_f32(const ceb_gguf_tensor* t, float** out, int64_t expect) {
        *out = nullptr;
        if (!t) return 0;
        int64_t n = 1;
        for (int64_t x : t->ne) n *= x;
        if (expect >= 0 && n != expect)
            return ceb_set_error(1, "tensor '%s' has %lld values, expected %lld", t->name.c_str(), (long long)n,
                                 (long long)expect);
        std::vector<float> h((size_t)n);
        if (t->type == CEB_GGML_F32) {
            memcpy(h.data(), g.data(*t), (size_t)n * 4);
        } else if (t->type == CEB_GGML_F16) {
            const uint16_t* s = reinterpret_cast<const uint16_t*>(g.data(*t));
            for (int64_t i = 0; i < n; ++i) {
                __half_raw r;
                r.x = s[i];
                h[(size_t)i] = __half2float(__half(r));
            }
        } else {
            // quantized tables (llama.cpp exports quantize the token embeddings): decoded row by row
            const int64_t k = t->ne.empty() ? n : t->ne[0];
            const int64_t rb = ceb_ggml_row_bytes(t->type, k);
            if (rb < 0)
                return ceb_set_error(1, "tensor '%s': type %d not supported for a float table", t->name.c_str(),
                                     t->type);
            const uint8_t* src = static_cast<const uint8_t*>(g.data(*t));
            for (int64_t r = 0; r < n / k; ++r) ceb_ggml_dequant_row(t->type, src + r * rb, k, h.data() + r * k);
        }
        void* d = nullptr;
        if (cudaMalloc(&d, (size_t)n * 4) != cudaSuccess) return ceb_set_error(4, "out of device memory (%s)", t->name.c_str());
        m->allocs.push_back(d);
        m->weight_bytes += (size_t)n * 4;
        if (cudaMemcpy(d, h.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return ceb_set_error(3, "upload of '%s' failed", t->name.c_str());
        *out = static_cast<float*>(d);
        return 0;
    }

    int upload_raw(const void* src, size_t bytes, uint8_t** out) {
        void* d = nullptr;
        if (cudaMalloc(&d, bytes) != cudaSuccess) return ceb_set_error(4, "out of device memory");
        m->allocs.push_back(d);
        m->weight_bytes += bytes;
        if (cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return ceb_set_error(3, "upload failed");
        *out = static_cast<uint8_t*>(d);
        return 0;
    }

    // one linear weight [n_out x k] (2-D tensor ne = {k, n_out}); with reference
    // arithmetic also the form its kernels read
    int plane(const ceb_gguf_tensor* t, int n_out, int k, ceb_wplane* w, ceb_refmat* r) {
        if (!t || t->ne.size() < 2 || t->ne[0] != k || t->ne[1] != n_out)
            return ceb_set_error(1, "weight '%s' has an unexpected shape", t ? t->name.c_str() : "?");
        int rc = ceb_repack_weights(w, t->type, g.data(*t), 1, n_out, k, st);
        if (!rc) m->weight_bytes += w->q_bytes + w->s_bytes;
        if (!rc) rc = ref(r, t->type, g.data(*t), 1, n_out, k);
        return rc;
    }

    int ref(ceb_refmat* r, int type, const void* data, int groups, int n_out, int k) {
        if (!m->ref_arith) return 0;
        const int rc = ceb_refmat_create(r, type, data, groups, n_out, k);
        if (!rc) m->weight_bytes += (size_t)groups * n_out * k * (r->type == CEB_GGML_Q8_0 ? 1 : 4) +
                                    (r->type == CEB_GGML_Q8_0 ? (size_t)groups * n_out * (k / 32) * 4 : 0);
        return rc;
    }
};

}  // namespace

int ceb_model_load(ceb_model* m, const std::string& path, std::string* err_out) {
    ceb_gguf g;
    std::string err;
    if (!g.open(path, &err)) return ceb_set_error(1, "failed to open '%s': %s", path.c_str(), err.c_str());
    Loader L{g, m, g.get_str("general.architecture")};
    if (g.find("decoder.hidden_size"))
        return ceb_set_error(1, "'%s' is a decoder-embedding model; this library implements the encoder path",
                             path.c_str());
    auto& hp = m->hp;
    hp.n_vocab = L.u32({"bert.vocab_size", L.ak("vocab_size")}, 30522);
    hp.n_max_tokens = L.u32({"bert.max_position_embeddings", "bert.context_length", "xlmr.context_length",
                             L.ak("context_length")},
                            512);
    hp.n_embd = L.u32({"bert.hidden_size", "bert.embedding_length", "xlmr.embedding_length", L.ak("embedding_length"),
                       L.ak("hidden_size")},
                      384);
    hp.n_head = L.u32({"bert.num_attention_heads", "bert.attention.head_count", "xlmr.attention.head_count",
                       L.ak("attention.head_count")},
                      12);
    hp.n_layer = L.u32({"bert.num_hidden_layers", "bert.block_count", "xlmr.block_count", L.ak("block_count")}, 6);
    hp.n_intermediate = L.u32({"bert.intermediate_size", "bert.feed_forward_length", "xlmr.feed_forward_length",
                               L.ak("feed_forward_length")},
                              1536);
    hp.n_output = L.u32({"bert.output_dim"}, hp.n_embd);
    hp.layer_norm_eps = L.f32({"bert.layer_norm_eps", "bert.attention.layer_norm_epsilon",
                               "xlmr.attention.layer_norm_epsilon", L.ak("attention.layer_norm_epsilon")},
                              1e-12f);
    hp.n_experts = L.u32({"bert.num_experts", L.ak("expert_count")}, 0);
    hp.n_experts_per_tok = L.u32({"bert.num_experts_per_tok", L.ak("expert_used_count")}, 0);
    {
        int pm = L.u32({"bert.pooling_method"}, -1);
        if (pm < 0) {
            const int pt = L.u32({"bert.pooling_type", "xlmr.pooling_type", L.ak("pooling_type")}, -1);
            pm = pt > 0 ? pt - 1 : 0;
        }
        m->pool_method = pm;
    }
    m->pos_offset = L.u32({"bert.position_offset", "xlmr.position_offset"}, 0);
    if (L.u32({"bert.pre_ln"}, 0) != 0)
        return ceb_set_error(1, "pre-LN encoders are outside this build's NomicBERT-MoE path");

    (void)err_out;

    cudaStream_t st;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return ceb_set_error(3, "stream create");
    L.st = st;
    int rc = 0;
    const ceb_gguf_tensor* tok = g.tensor("token_embd.weight");
    if (!tok) rc = ceb_set_error(1, "missing token_embd.weight");
    if (!rc) {
        // hparams inferred from tensor shapes when metadata disagrees (src/crispembed.cpp:779-800)
        hp.n_vocab = (int)tok->ne[1];
        if (tok->ne[0] != hp.n_embd) {
            hp.n_embd = (int)tok->ne[0];
            hp.n_output = hp.n_embd;
        }
        int counted = 0;
        for (const auto& kv : g.tensors()) {
            int il = -1;
            if (sscanf(kv.first.c_str(), "enc.%d.", &il) == 1 || sscanf(kv.first.c_str(), "blk.%d.", &il) == 1)
                if (il + 1 > counted) counted = il + 1;
        }
        if (counted > 0) hp.n_layer = counted;
    }
    const int d = hp.n_embd;
    if (!rc) rc = L.upload_f32(tok, &m->tok, (int64_t)hp.n_vocab * d);
    if (!rc) {
        const ceb_gguf_tensor* pe = g.tensor("position_embd.weight");
        if (!pe) {
            // no position table: RoPE with NEOX pairing (src/crispembed.cpp:788-795, :1182-1195); base from
            // bert.rope_theta or <arch>.rope.freq_base (src/crispembed.cpp:482-483)
            m->use_rope = true;
            m->rope_theta = L.f32({"bert.rope_theta", L.ak("rope.freq_base")}, 10000.0f);
            m->n_pos = hp.n_max_tokens + m->pos_offset;
        } else {
            m->n_pos = (int)pe->ne[1];
            rc = L.upload_f32(pe, &m->pos, (int64_t)m->n_pos * d);
        }
    }
    if (!rc) {
        const ceb_gguf_tensor* te = L.any({"token_type_embd.weight", "token_types.weight"});
        if (te) {
            float* full = nullptr;
            rc = L.upload_f32(te, &full, -1);
            m->type0 = full;  // row 0 (type ids are 0 for single-segment embedding input)
        }
    }
    if (!rc) rc = L.upload_f32(L.any({"embd_ln.weight", "token_embd_norm.weight"}), &m->embd_ln_w, d);
    if (!rc) rc = L.upload_f32(L.any({"embd_ln.bias", "token_embd_norm.bias"}), &m->embd_ln_b, d);
    if (hp.n_head <= 0 || d % hp.n_head || d / hp.n_head != 64)
        rc = rc ? rc : ceb_set_error(1, "head_dim %d unsupported (64 only)", hp.n_head > 0 ? d / hp.n_head : -1);

    m->layers.resize(hp.n_layer);
    for (int il = 0; il < hp.n_layer && !rc; ++il) {
        const std::string p = "enc." + std::to_string(il) + ".", b = "blk." + std::to_string(il) + ".";
        ceb_layer& Ly = m->layers[il];
        // attention: separate q/k/v (or fused qkv) rows stacked q|k|v into one plane
        const ceb_gguf_tensor* qkv = L.any({p + "attn.qkv.weight", b + "attn_qkv.weight"});
        const ceb_gguf_tensor* q = L.any({p + "attn.q.weight", b + "attn_q.weight"});
        const ceb_gguf_tensor* k = L.any({p + "attn.k.weight", b + "attn_k.weight"});
        const ceb_gguf_tensor* v = L.any({p + "attn.v.weight", b + "attn_v.weight"});
        if (qkv) {
            rc = L.plane(qkv, 3 * d, d, &Ly.qkv, &Ly.r_qkv);
        } else if (q && k && v && q->type == k->type && k->type == v->type) {
            const int64_t rbytes = (int64_t)q->nbytes;
            std::vector<uint8_t> cat((size_t)(3 * rbytes));
            memcpy(cat.data(), g.data(*q), (size_t)rbytes);
            memcpy(cat.data() + rbytes, g.data(*k), (size_t)rbytes);
            memcpy(cat.data() + 2 * rbytes, g.data(*v), (size_t)rbytes);
            rc = ceb_repack_weights(&Ly.qkv, q->type, cat.data(), 1, 3 * d, d, st);
            if (!rc) rc = L.ref(&Ly.r_qkv, q->type, cat.data(), 1, 3 * d, d);
        } else if (q && k && v) {
            // mixed formats (llama.cpp's K-quant mixes give attn_v its own type): rows
            // re-encoded as Q8_0 blocks when every part allows it, else decoded to fp32
            const ceb_gguf_tensor* parts[3] = {q, k, v};
            auto q8able = [](int t) { return t == CEB_GGML_Q8_0 || t == CEB_GGML_IQ4_NL || t == CEB_GGML_IQ4_XS; };
            const bool as_q8 = q8able(q->type) && q8able(k->type) && q8able(v->type);
            const int64_t orb = as_q8 ? ceb_ggml_row_bytes(CEB_GGML_Q8_0, d) : (int64_t)d * 4;
            std::vector<uint8_t> cat((size_t)(3 * d * orb));
            for (int j = 0; j < 3 && !rc; ++j) {
                const int64_t rb = ceb_ggml_row_bytes(parts[j]->type, d);
                if (rb < 0 || parts[j]->ne.size() < 2 || parts[j]->ne[0] != d || parts[j]->ne[1] != d) {
                    rc = ceb_set_error(1, "layer %d: attention weight of type %d / shape unsupported", il,
                                       parts[j]->type);
                    break;
                }
                const uint8_t* src = static_cast<const uint8_t*>(g.data(*parts[j]));
                for (int r = 0; r < d; ++r) {
                    uint8_t* dst = cat.data() + ((size_t)j * d + r) * orb;
                    if (as_q8)
                        ceb_ggml_as_q8_0_blocks(parts[j]->type, src + r * rb, d, dst);
                    else
                        ceb_ggml_dequant_row(parts[j]->type, src + r * rb, d, reinterpret_cast<float*>(dst));
                }
            }
            if (!rc)
                rc = ceb_repack_weights(&Ly.qkv, as_q8 ? CEB_GGML_Q8_0 : CEB_GGML_F32, cat.data(), 1, 3 * d, d, st);
            // the reference multiplies each part in its own format: the common form is exact only for floats
            auto flt = [](int t) { return t == CEB_GGML_F32 || t == CEB_GGML_F16 || t == CEB_GGML_BF16; };
            if (!rc && m->ref_arith && !(flt(q->type) && flt(k->type) && flt(v->type)))
                rc = ceb_set_error(2, "reference arithmetic: layer %d mixes attention weight formats", il);
            if (!rc) rc = L.ref(&Ly.r_qkv, CEB_GGML_F32, cat.data(), 1, 3 * d, d);
        } else {
            rc = ceb_set_error(1, "layer %d: missing attention q/k/v weights", il);
        }
        if (rc) break;
        {
            const ceb_gguf_tensor* qb = L.any({p + "attn.q.bias", b + "attn_q.bias"});
            const ceb_gguf_tensor* kb = L.any({p + "attn.k.bias", b + "attn_k.bias"});
            const ceb_gguf_tensor* vb = L.any({p + "attn.v.bias", b + "attn_v.bias"});
            const ceb_gguf_tensor* qkvb = L.any({p + "attn.qkv.bias", b + "attn_qkv.bias"});
            if (qkvb) {
                rc = L.upload_f32(qkvb, &Ly.qkv_b, 3 * d);
            } else if (qb || kb || vb) {
                std::vector<float> cat((size_t)3 * d, 0.0f);
                const ceb_gguf_tensor* parts[3] = {qb, kb, vb};
                for (int j = 0; j < 3; ++j)
                    if (parts[j]) {
                        if (parts[j]->type != CEB_GGML_F32 || parts[j]->ne[0] != d) {
                            rc = ceb_set_error(1, "layer %d: attention bias must be F32[%d]", il, d);
                            break;
                        }
                        memcpy(&cat[(size_t)j * d], g.data(*parts[j]), (size_t)d * 4);
                    }
                if (!rc) rc = L.upload_raw(cat.data(), cat.size() * 4, reinterpret_cast<uint8_t**>(&Ly.qkv_b));
            }
        }
        if (!rc) rc = L.plane(L.any({p + "attn.o.weight", b + "attn_output.weight"}), d, d, &Ly.o, &Ly.r_o);
        if (!rc) rc = L.upload_f32(L.any({p + "attn.o.bias", b + "attn_output.bias"}), &Ly.o_b, d);
        if (!rc) rc = L.upload_f32(L.any({p + "ln1.weight", b + "attn_output_norm.weight", b + "attn_norm.weight"}),
                                   &Ly.ln1_w, d);
        if (!rc) rc = L.upload_f32(L.any({p + "ln1.bias", b + "attn_output_norm.bias", b + "attn_norm.bias"}),
                                   &Ly.ln1_b, d);
        if (!rc) rc = L.upload_f32(L.any({p + "ln2.weight", b + "layer_output_norm.weight", b + "ffn_norm.weight"}),
                                   &Ly.ln2_w, d);
        if (!rc) rc = L.upload_f32(L.any({p + "ln2.bias", b + "layer_output_norm.bias", b + "ffn_norm.bias"}),
                                   &Ly.ln2_b, d);
        if (!rc && (!Ly.ln1_w || !Ly.ln2_w)) rc = ceb_set_error(1, "layer %d: missing ln1/ln2 (post-LN encoder)", il);
        if (rc) break;
        const ceb_gguf_tensor* gate = L.any({p + "ffn.moe_gate.weight", b + "ffn_gate_inp.weight"});
        if (gate) {
            const ceb_gguf_tensor* e1 = L.any({p + "ffn.expert_fc1.weight", b + "ffn_up_exps.weight"});
            const ceb_gguf_tensor* e2 = L.any({p + "ffn.expert_fc2.weight", b + "ffn_down_exps.weight"});
            if (!e1 || !e2 || e1->ne.size() != 3 || e2->ne.size() != 3) {
                rc = ceb_set_error(1, "layer %d: MoE layer without stacked expert weights", il);
                break;
            }
            const int E = (int)e1->ne[2], F = (int)e1->ne[1];
            if (hp.n_experts <= 0) hp.n_experts = E;
            if (E != hp.n_experts || e1->ne[0] != d || e2->ne[0] != F || e2->ne[1] != d || e2->ne[2] != E ||
                gate->ne[0] != d || gate->ne[1] != E || hp.n_experts_per_tok <= 0) {
                rc = ceb_set_error(1, "layer %d: inconsistent MoE shapes / expert counts", il);
                break;
            }
            if (gate->type != CEB_GGML_F32 && gate->type != CEB_GGML_Q8_0) {
                rc = ceb_set_error(1, "layer %d: router type %d unsupported (F32 or Q8_0)", il, gate->type);
                break;
            }
            Ly.moe = true;
            ceb_moe_weights& mw = Ly.moew;
            mw.d = d;
            mw.n_experts = E;
            mw.top_k = hp.n_experts_per_tok;
            mw.ffn = F;
            mw.router_type = gate->type;
            rc = L.upload_raw(g.data(*gate), gate->nbytes, &mw.router);
            if (!rc) rc = ceb_repack_weights(&mw.fc1, e1->type, g.data(*e1), E, F, d, st);
            if (!rc) rc = ceb_repack_weights(&mw.fc2, e2->type, g.data(*e2), E, d, F, st);
            if (!rc) rc = L.ref(&Ly.r_router, gate->type, g.data(*gate), 1, E, d);
            if (!rc) rc = L.ref(&Ly.r_e1, e1->type, g.data(*e1), E, F, d);
            if (!rc) rc = L.ref(&Ly.r_e2, e2->type, g.data(*e2), E, d, F);
            if (!rc) m->weight_bytes += mw.fc1.q_bytes + mw.fc1.s_bytes + mw.fc2.q_bytes + mw.fc2.s_bytes;
            if (!rc) rc = L.upload_f32(g.tensor(p + "ffn.moe_bias"), &mw.bias, d);
        } else {
            const ceb_gguf_tensor* f1 = L.any({p + "ffn.fc1.weight", b + "ffn_up.weight"});
            const ceb_gguf_tensor* f2 = L.any({p + "ffn.fc2.weight", b + "ffn_down.weight"});
            if (!f1 || !f2) {
                rc = ceb_set_error(1, "layer %d: missing ffn.fc1/ffn.fc2 (GELU FFN)", il);
                break;
            }
            if (L.any({p + "ffn_gate.weight", b + "ffn_gate.weight", p + "ffn_up_gate.weight"})) {
                rc = ceb_set_error(1, "layer %d: gated FFN variants are outside this build", il);
                break;
            }
            const int F = (int)f1->ne[1];
            rc = L.plane(f1, F, d, &Ly.fc1, &Ly.r_fc1);
            if (!rc) rc = L.upload_f32(L.any({p + "ffn.fc1.bias", b + "ffn_up.bias"}), &Ly.fc1_b, F);
            if (!rc) rc = L.plane(f2, d, F, &Ly.fc2, &Ly.r_fc2);
            if (!rc) rc = L.upload_f32(L.any({p + "ffn.fc2.bias", b + "ffn_down.bias"}), &Ly.fc2_b, d);
        }
    }
    if (!rc && m->ref_arith) {
        if (m->use_rope) rc = ceb_set_error(2, "reference arithmetic covers encoders with learned positions");
        else if (m->pool_method != 0) rc = ceb_set_error(2, "reference arithmetic covers mean pooling");
        else if ((size_t)d * 4 * 8 > 48 * 1024) rc = ceb_set_error(2, "reference arithmetic: width %d too large", d);
    }
    cudaStreamDestroy(st);
    if (rc) ceb_model_free(m);
    return rc;
}

int ceb_model_ep_attach(ceb_model* m, ceb_ep* ep) {
    if (!ep || !ep->connected) return ceb_set_error(1, "ep_attach: the exchange is not connected");
    if (m->ep) return ceb_set_error(1, "ep_attach: the model already runs expert-parallel");
    for (auto& Ly : m->layers) {
        if (!Ly.moe) continue;
        const ceb_moe_weights& mw = Ly.moew;
        if (mw.n_experts != ep->E || mw.top_k != ep->K || mw.d != ep->d || mw.ffn != ep->F)
            return ceb_set_error(1, "ep_attach: MoE block (E=%d K=%d d=%d F=%d) does not match the exchange "
                                    "(E=%d K=%d d=%d F=%d)",
                                 mw.n_experts, mw.top_k, mw.d, mw.ffn, ep->E, ep->K, ep->d, ep->F);
    }
    for (auto& Ly : m->layers) {
        if (!Ly.moe) continue;
        for (ceb_wplane* w : {&Ly.moew.fc1, &Ly.moew.fc2}) {
            const ceb_wplane view = ceb_wplane_slice(*w, ep->rank * ep->E_loc, ep->E_loc);
            ceb_wplane local = view;
            local.q = nullptr;
            if (cudaMalloc(&local.q, view.q_bytes) != cudaSuccess)
                return ceb_set_error(4, "ep_attach: out of device memory for the local experts");
            const cudaError_t e = cudaMemcpy(local.q, view.q, view.q_bytes, cudaMemcpyDeviceToDevice);
            if (e != cudaSuccess) {
                cudaFree(local.q);
                return ceb_set_cuda_error(e, "ep_attach: local expert copy", __FILE__, __LINE__);
            }
            m->weight_bytes -= w->q_bytes + w->s_bytes - local.q_bytes - local.s_bytes;
            ceb_wplane_free(w);
            *w = local;
        }
    }
    m->ep = ep;
    return 0;
}

void ceb_model_free(ceb_model* m) {
    for (auto& Ly : m->layers) {
        for (ceb_refmat* r : {&Ly.r_qkv, &Ly.r_o, &Ly.r_fc1, &Ly.r_fc2, &Ly.r_router, &Ly.r_e1, &Ly.r_e2})
            ceb_refmat_free(r);
        ceb_wplane_free(&Ly.qkv);
        ceb_wplane_free(&Ly.o);
        ceb_wplane_free(&Ly.fc1);
        ceb_wplane_free(&Ly.fc2);
        ceb_wplane_free(&Ly.moew.fc1);
        ceb_wplane_free(&Ly.moew.fc2);
    }
    for (void* p : m->allocs) cudaFree(p);
    m->allocs.clear();
    m->layers.clear();
}

// ------------------------------------------------------------------ workspace
int ceb_workspace_reserve(ceb_workspace* ws, const ceb_model& m, int tokens, int seqs) {
    if (tokens <= ws->cap_tokens && seqs <= ws->cap_seqs && ws->base) return 0;
    const int T = tokens > ws->cap_tokens ? tokens : ws->cap_tokens;
    const int S = seqs > ws->cap_seqs ? seqs : ws->cap_seqs;
    const int d = m.hp.n_embd;
    int F = 0, E = 1, K = 1, Fm = 128;
    for (const auto& Ly : m.layers) {
        if (Ly.moe) {
            E = Ly.moew.n_experts;
            K = Ly.moew.top_k;
            Fm = Fm > Ly.moew.ffn ? Fm : Ly.moew.ffn;
        } else if (Ly.fc1.n_out > F) {
            F = Ly.fc1.n_out;
        }
    }
    size_t off = 0;
    auto take = [&](size_t b) {
        size_t o = off;
        off += (b + 255) & ~size_t(255);
        return o;
    };
    const size_t o_x32 = take((size_t)T * d * 4), o_c32 = take((size_t)T * d * 4), o_t32 = take((size_t)T * d * 4);
    const size_t o_x16 = take((size_t)T * d * 2), o_c16 = take((size_t)T * d * 2), o_t16 = take((size_t)T * d * 2);
    const size_t o_qkv = take((size_t)T * 3 * d * 2), o_a16 = take((size_t)T * d * 2);
    const size_t o_h16 = take((size_t)T * (F > 0 ? F : 128) * 2);
    const size_t moe_bytes = ceb_moe_ws_layout(T, d, E, K, Fm, nullptr, nullptr);
    const size_t o_moe = take(moe_bytes);
    const size_t o_ids = take((size_t)T * 4), o_cu = take((size_t)(S + 1) * 4), o_out = take((size_t)S * d * 4);
    const size_t o_sched = take(2 * sizeof(int));
    // reference arithmetic: fp32 activations, Q8_0 copies of every matrix input, expert rows
    // padded to whole 32-row tiles per expert
    size_t r_qkv = 0, r_attn = 0, r_h = 0, r_xp = 0, r_down = 0, r_lg = 0, r_wts = 0, r_xq = 0, r_xd = 0, r_ids = 0,
           r_pos = 0, r_src = 0, r_tg = 0;
    int n_tiles = 0;
    if (m.ref_arith) {
        n_tiles = (int)(((int64_t)T * K + (int64_t)E * 31 + 31) / 32);
        const size_t rows_pad = (size_t)n_tiles * 32;
        const size_t wmax = (size_t)std::max(std::max(d, F), Fm);
        const size_t qrows = std::max((size_t)T, rows_pad);
        r_qkv = take((size_t)T * 3 * d * 4);
        r_attn = take((size_t)T * d * 4);
        r_h = take(std::max((size_t)T * (F > 0 ? F : 128), rows_pad * Fm) * 4);
        r_xp = take(rows_pad * d * 4);
        r_down = take(rows_pad * d * 4);
        r_lg = take((size_t)T * E * 4);
        r_wts = take((size_t)T * K * 4);
        r_xq = take(qrows * wmax);
        r_xd = take(qrows * (wmax / 32) * 4);
        r_ids = take((size_t)T * K * 4);
        r_pos = take((size_t)T * K * 4);
        r_src = take(rows_pad * 4);
        r_tg = take((size_t)n_tiles * 4);
    }
    void* base = nullptr;
    if (cudaMalloc(&base, off) != cudaSuccess)
        return ceb_set_error(4, "out of device memory for a %d-token workspace (%.2f GB)", T, off / 1e9);
    ceb_workspace_free(ws);
    uint8_t* b = static_cast<uint8_t*>(base);
    ws->base = base;
    ws->bytes = off;
    ws->cap_tokens = T;
    ws->cap_seqs = S;
    ws->x32 = reinterpret_cast<float*>(b + o_x32);
    ws->c32 = reinterpret_cast<float*>(b + o_c32);
    ws->t32 = reinterpret_cast<float*>(b + o_t32);
    ws->x16 = reinterpret_cast<__half*>(b + o_x16);
    ws->c16 = reinterpret_cast<__half*>(b + o_c16);
    ws->t16 = reinterpret_cast<__half*>(b + o_t16);
    ws->qkv16 = reinterpret_cast<__half*>(b + o_qkv);
    ws->a16 = reinterpret_cast<__half*>(b + o_a16);
    ws->h16 = reinterpret_cast<__half*>(b + o_h16);
    ceb_moe_ws_layout(T, d, E, K, Fm, &ws->moe, b + o_moe);
    ws->ids = reinterpret_cast<int32_t*>(b + o_ids);
    ws->cu = reinterpret_cast<int32_t*>(b + o_cu);
    ws->out = reinterpret_cast<float*>(b + o_out);
    ws->attn_sched = reinterpret_cast<int*>(b + o_sched);
    if (cudaMemset(ws->attn_sched, 0, 2 * sizeof(int)) != cudaSuccess) return ceb_set_error(3, "workspace: clearing");
    if (m.ref_arith) {
        ceb_ref_ws& r = ws->ref;
        r.qkv = reinterpret_cast<float*>(b + r_qkv);
        r.attn = reinterpret_cast<float*>(b + r_attn);
        r.h = reinterpret_cast<float*>(b + r_h);
        r.xp = reinterpret_cast<float*>(b + r_xp);
        r.down = reinterpret_cast<float*>(b + r_down);
        r.logits = reinterpret_cast<float*>(b + r_lg);
        r.wts = reinterpret_cast<float*>(b + r_wts);
        r.xq = reinterpret_cast<int8_t*>(b + r_xq);
        r.xd = reinterpret_cast<float*>(b + r_xd);
        r.ids = reinterpret_cast<int32_t*>(b + r_ids);
        r.pos = reinterpret_cast<int32_t*>(b + r_pos);
        r.src = reinterpret_cast<int32_t*>(b + r_src);
        r.tile_group = reinterpret_cast<int32_t*>(b + r_tg);
        r.n_tiles_max = n_tiles;
    }
    return 0;
}

void ceb_workspace_free(ceb_workspace* ws) {
    if (ws->base) cudaFree(ws->base);
    *ws = ceb_workspace();
}

// ------------------------------------------------------------------ forward, reference arithmetic
namespace {

// The encoder in the reference's CPU arithmetic (ref_arith.cu), in the order of
// build_encoder_graph (src/crispembed.cpp:1068-1428): every matrix input that
// meets a Q8_0 weight is re-quantized to Q8_0 first, as ggml's mul_mat does for
// vec_dot_type Q8_0; everything stays fp32 between the products.
int encoder_forward_ref(const ceb_model& m, ceb_workspace& ws, const int32_t* d_ids, const int32_t* d_cu, int n_seqs,
                        int M, int max_len, float* d_out, int out_dim, int* d_err, cudaStream_t st,
                        const ceb_route_capture* cap) {
    const auto& hp = m.hp;
    const int d = hp.n_embd;
    const float eps = hp.layer_norm_eps;
    const ceb_ref_ws& r = ws.ref;
    int rc = ceb_ref_embed(d_ids, d_cu, n_seqs, d, hp.n_vocab, m.tok, m.pos, m.n_pos, m.pos_offset, m.type0, ws.t32,
                           d_err, st);
    if (rc) return rc;
    if (m.embd_ln_w) {  // the graph normalises the embeddings when the model has embd_ln
        if ((rc = ceb_ref_ln(ws.t32, nullptr, M, d, m.embd_ln_w, m.embd_ln_b, eps, ws.x32, st))) return rc;
    } else if (cudaMemcpyAsync(ws.x32, ws.t32, (size_t)M * d * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
        return ceb_set_error(3, "embedding copy");
    }
    // y = W x (+ bias) for `rows` rows of x (k values each), x re-quantized first for Q8_0 weights
    auto linear = [&](const ceb_refmat& w, const float* x, int rows, const int32_t* tile_group, const float* bias,
                      float* y) {
        if (w.type == CEB_GGML_Q8_0)
            if (int e = ceb_ref_quant(x, rows, w.k, r.xq, r.xd, st)) return e;
        return ceb_ref_matmul(w, x, r.xq, r.xd, rows, tile_group, bias, 0, y, w.n_out, st);
    };
    int moe_block = 0;
    for (const ceb_layer& Ly : m.layers) {
        if ((rc = linear(Ly.r_qkv, ws.x32, M, nullptr, Ly.qkv_b, r.qkv))) return rc;
        if ((rc = ceb_ref_attention(r.qkv, d_cu, n_seqs, max_len, d, hp.n_head, r.attn, st))) return rc;
        if ((rc = linear(Ly.r_o, r.attn, M, nullptr, Ly.o_b, ws.t32))) return rc;
        if ((rc = ceb_ref_ln(ws.x32, ws.t32, M, d, Ly.ln1_w, Ly.ln1_b, eps, ws.c32, st))) return rc;
        if (Ly.moe) {
            const ceb_moe_weights& mw = Ly.moew;
            const int E = mw.n_experts, K = mw.top_k, F = mw.ffn;
            // router logits (no bias), softmax, top-k (src/crispembed.cpp:1333-1345)
            if ((rc = linear(Ly.r_router, ws.c32, M, nullptr, nullptr, r.logits))) return rc;
            if ((rc = ceb_ref_route(r.logits, M, E, K, r.ids, r.wts, st))) return rc;
            if (cap && cap->logits &&
                cudaMemcpyAsync(cap->logits + (size_t)moe_block * M * E, r.logits, (size_t)M * E * 4,
                                cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                return ceb_set_error(3, "route capture");
            if (cap && cap->ids &&
                cudaMemcpyAsync(cap->ids + (size_t)moe_block * M * K, r.ids, (size_t)M * K * 4,
                                cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                return ceb_set_error(3, "route capture");
            ++moe_block;
            // expert rows grouped per expert (ggml_mul_mat_id), fc1 -> erf-GELU -> fc2 (:1365-1371)
            const int rows_pad = r.n_tiles_max * 32;
            if ((rc = ceb_ref_group(r.ids, M, K, E, r.n_tiles_max, r.pos, r.src, r.tile_group, st))) return rc;
            if ((rc = ceb_ref_gather(ws.c32, r.src, rows_pad, d, r.xp, st))) return rc;
            if ((rc = linear(Ly.r_e1, r.xp, rows_pad, r.tile_group, nullptr, r.h))) return rc;
            if ((rc = ceb_ref_gelu(r.h, (int64_t)rows_pad * F, st))) return rc;
            if ((rc = linear(Ly.r_e2, r.h, rows_pad, r.tile_group, nullptr, r.down))) return rc;
            // gate-weighted combine + MoE bias (:1375-1381)
            if ((rc = ceb_ref_combine(r.down, r.pos, r.wts, M, K, d, mw.bias, ws.t32, st))) return rc;
        } else {
            const int F = Ly.r_fc1.n_out;
            if ((rc = linear(Ly.r_fc1, ws.c32, M, nullptr, Ly.fc1_b, r.h))) return rc;
            if ((rc = ceb_ref_gelu(r.h, (int64_t)M * F, st))) return rc;
            if ((rc = linear(Ly.r_fc2, r.h, M, nullptr, Ly.fc2_b, ws.t32))) return rc;
        }
        if ((rc = ceb_ref_ln(ws.c32, ws.t32, M, d, Ly.ln2_w, Ly.ln2_b, eps, ws.x32, st))) return rc;
    }
    return ceb_ref_pool(ws.x32, d_cu, n_seqs, d, out_dim, d_out, st);
}

}  // namespace

// ------------------------------------------------------------------ forward
int ceb_encoder_forward(const ceb_model& m, ceb_workspace& ws, const int32_t* d_ids, const int32_t* d_cu, int n_seqs,
                        int M, int max_len, float* d_out, int out_dim, int* d_err, cudaStream_t st,
                        const ceb_route_capture* cap) {
    const auto& hp = m.hp;
    const int d = hp.n_embd;
    const float eps = hp.layer_norm_eps;
    if (M > ws.cap_tokens) return ceb_set_error(1, "forward: %d tokens exceed the workspace (%d)", M, ws.cap_tokens);
    if (max_len > m.n_pos - m.pos_offset)
        return ceb_set_error(1, "sequence of %d tokens exceeds the model's %d positions", max_len, m.n_pos);
    if (m.ref_arith) return encoder_forward_ref(m, ws, d_ids, d_cu, n_seqs, M, max_len, d_out, out_dim, d_err, st, cap);
    int rc = ceb_embed_ln(d_ids, d_cu, n_seqs, M, d, hp.n_vocab, m.tok, m.pos, m.n_pos, m.pos_offset, m.type0,
                          m.embd_ln_w, m.embd_ln_b, eps, ws.x32, ws.x16, d_err, st);
    if (rc) return rc;
    int moe_block = 0;
    for (const ceb_layer& Ly : m.layers) {
        ceb_gemm_args a;
        a.m_rows = M;
        a.err = d_err;
        // QKV projection (+bias) -> fp16 [M, 3d]
        a.out = ws.qkv16;
        a.ldo = 3 * d;
        a.epi = CEB_EPI_F16_OUT | (Ly.qkv_b ? CEB_EPI_BIAS : 0);
        a.bias = Ly.qkv_b;
        if ((rc = ceb_gemm_launch(Ly.qkv, ws.x16, M, a, st))) return rc;
        if (m.use_rope &&
            (rc = ceb_rope_neox(ws.qkv16, M, d_cu, n_seqs, d, hp.n_head, m.pos_offset, m.rope_theta, st)))
            return rc;
        if ((rc = ceb_attention(ws.qkv16, M, d_cu, n_seqs, max_len, d, hp.n_head, ws.a16, d_err, st, ws.attn_sched))) return rc;
        // output projection (+bias) -> fp16, residual + LN1
        a.out = ws.t16;
        a.ldo = d;
        a.epi = CEB_EPI_F16_OUT | (Ly.o_b ? CEB_EPI_BIAS : 0);
        a.bias = Ly.o_b;
        if ((rc = ceb_gemm_launch(Ly.o, ws.a16, M, a, st))) return rc;
        if (Ly.moe) {
            const ceb_moe_weights& mw = Ly.moew;
            float* cap_logits = cap && cap->logits ? cap->logits + (size_t)moe_block * M * mw.n_experts : nullptr;
            if ((rc = ceb_add_ln_route(ws.x32, ws.t16, true, M, d, Ly.ln1_w, Ly.ln1_b, eps, ws.c32, ws.c16, mw, ws.moe,
                                       cap_logits, st)))
                return rc;
            if (cap && cap->ids) {
                const cudaError_t e = cudaMemcpyAsync(cap->ids + (size_t)moe_block * M * mw.top_k, ws.moe.ids,
                                                      (size_t)M * mw.top_k * 4, cudaMemcpyDeviceToDevice, st);
                if (e != cudaSuccess) return ceb_set_cuda_error(e, "route capture", __FILE__, __LINE__);
            }
            ++moe_block;
            const __half* down = ws.moe.down;
            if (m.ep) {
                if ((rc = ceb_ep_moe(m.ep, mw, ws.c32, CEB_ACT_F32, ws.c16, M, ws.moe, d_err, st))) return rc;
                down = m.ep->self.ret;
            } else if ((rc = ceb_moe_dispatch(mw, ws.c32, CEB_ACT_F32, ws.c16, M, nullptr, ws.moe, nullptr, d_err,
                                              st))) {
                return rc;
            }
            if ((rc = ceb_moe_combine_ln(down, ws.moe.slot_pos, ws.moe.wts, mw.top_k, mw.bias, ws.c32, M, d,
                                         Ly.ln2_w, Ly.ln2_b, eps, ws.x32, ws.x16, st)))
                return rc;
        } else {
            if ((rc = ceb_add_ln(ws.x32, ws.t16, M, d, Ly.ln1_w, Ly.ln1_b, eps, ws.c32, ws.c16, st))) return rc;
            a.out = ws.h16;
            a.ldo = Ly.fc1.n_out;
            a.epi = CEB_EPI_F16_OUT | CEB_EPI_GELU | (Ly.fc1_b ? CEB_EPI_BIAS : 0);
            a.bias = Ly.fc1_b;
            if ((rc = ceb_gemm_launch(Ly.fc1, ws.c16, M, a, st))) return rc;
            a.out = ws.t16;
            a.ldo = d;
            a.epi = CEB_EPI_F16_OUT | (Ly.fc2_b ? CEB_EPI_BIAS : 0);
            a.bias = Ly.fc2_b;
            if ((rc = ceb_gemm_launch(Ly.fc2, ws.h16, M, a, st))) return rc;
            if ((rc = ceb_add_ln(ws.c32, ws.t16, M, d, Ly.ln2_w, Ly.ln2_b, eps, ws.x32, ws.x16, st))) return rc;
        }
    }
    return ceb_pool_l2_launch(ws.x32, d_cu, n_seqs, d, out_dim, d_out, st, m.pool_method);
}
