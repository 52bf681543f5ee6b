// ref_shim.cpp -- extern "C" entry points over the reference engine's own CPU
// path (src/cpu/ops.cpp, src/model/forward_cpu.cpp), compiled together with
// those unmodified reference sources by oracle/Makefile (target `ref`) into
// oracle/_ref/libref_cpu.so.
//
// TEST INFRASTRUCTURE ONLY: used to pin the oracle restatement (b2oracle.c)
// and as the timed CPU baseline.  Nothing in the product links it.
#include "src/cpu/ops.h"
#include "src/model/config.h"
#include "src/model/forward_cpu.h"

#include <cstdint>
#include <cstring>
#include <vector>

using namespace engine;

extern "C" {

void ref_embedding_lookup(const int64_t* ids, const float* table, float* out, int64_t s, int64_t h) {
    cpu::embedding_lookup(ids, table, out, s, h);
}
void ref_rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t dim, float eps) {
    cpu::rmsnorm(x, w, out, rows, dim, eps);
}
void ref_matmul_transB_naive(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    cpu::matmul_transB_naive(A, B, C, M, K, N);
}
void ref_matmul_transB_blocked(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    cpu::matmul_transB_blocked(A, B, C, M, K, N);
}
void ref_bias_add(const float* x, const float* b, float* out, int64_t M, int64_t N) {
    cpu::bias_add(x, b, out, M, N);
}
void ref_residual_add(const float* a, const float* b, float* out, int64_t n) {
    cpu::residual_add(a, b, out, n);
}
void ref_apply_rope(float* q, float* k, int64_t S, int64_t nq, int64_t nkv, int64_t D, int64_t p0, float theta) {
    cpu::apply_rope(q, k, S, nq, nkv, D, p0, theta);
}
void ref_causal_gqa(const float* q, const float* k, const float* v, float* out, int64_t S, int64_t nq,
                    int64_t nkv, int64_t D) {
    cpu::causal_gqa(q, k, v, out, S, nq, nkv, D);
}
void ref_swiglu(const float* g, const float* u, float* out, int64_t n) { cpu::swiglu(g, u, out, n); }

// Layer tensors in ModelWeightsFP32::LayerFP32 order (src/model/forward_cpu.h:18-38):
// ln1, ln2, wq, bq, wk, bk, wv, bv, wo, wg, wu, wd.
struct ref_layer {
    const float *ln1, *ln2, *wq, *bq, *wk, *bk, *wv, *bv, *wo, *wg, *wu, *wd;
};

static void put(std::vector<float>& dst, const float* src, size_t n) { dst.assign(src, src + n); }

// engine::forward_cpu over S tokens with a tied lm_head (the reference always
// uses embed_tokens as the lm_head, forward_cpu.cpp:165-167).  Biases are
// required by the reference; Llama-shaped callers pass zero vectors.
// logits_out: [S, V].  Returns 0 on success.
int ref_forward_cpu(int64_t vocab, int64_t hidden, int64_t inter, int64_t layers, int64_t nq, int64_t nkv,
                    int64_t head_dim, float eps, float theta, const float* embed, const float* final_norm,
                    const ref_layer* lw, const int64_t* ids, int64_t S, float* logits_out) {
    ModelConfig cfg;
    cfg.model_type = "llama";
    cfg.vocab_size = (int)vocab;
    cfg.hidden_size = (int)hidden;
    cfg.intermediate_size = (int)inter;
    cfg.num_hidden_layers = (int)layers;
    cfg.num_attention_heads = (int)nq;
    cfg.num_key_value_heads = (int)nkv;
    cfg.head_dim = (int)head_dim;
    cfg.rms_norm_eps = eps;
    cfg.rope_theta = theta;
    cfg.tie_word_embeddings = true;

    const size_t H = hidden, kvd = nkv * head_dim, I = inter;
    ModelWeightsFP32 w;
    put(w.embed_tokens, embed, (size_t)vocab * H);
    put(w.final_norm, final_norm, H);
    w.layers.resize(layers);
    for (int64_t l = 0; l < layers; ++l) {
        auto& d = w.layers[l];
        const ref_layer& s = lw[l];
        put(d.input_layernorm, s.ln1, H);
        put(d.post_attention_layernorm, s.ln2, H);
        put(d.q_proj_weight, s.wq, H * H);
        put(d.q_proj_bias, s.bq, H);
        put(d.k_proj_weight, s.wk, kvd * H);
        put(d.k_proj_bias, s.bk, kvd);
        put(d.v_proj_weight, s.wv, kvd * H);
        put(d.v_proj_bias, s.bv, kvd);
        put(d.o_proj_weight, s.wo, H * H);
        put(d.gate_proj_weight, s.wg, I * H);
        put(d.up_proj_weight, s.wu, I * H);
        put(d.down_proj_weight, s.wd, H * I);
    }
    std::vector<int64_t> tok(ids, ids + S);
    std::vector<float> out = forward_cpu(tok, cfg, w, "");
    if ((int64_t)out.size() != S * vocab) return -1;
    std::memcpy(logits_out, out.data(), out.size() * sizeof(float));
    return 0;
}

// Persistent form for timing: the weights are converted once, then
// engine::forward_cpu runs on them (const, so several host threads may run
// forwards on one model concurrently).
struct ref_model {
    ModelConfig cfg;
    ModelWeightsFP32 w;
};

void* ref_model_create(int64_t vocab, int64_t hidden, int64_t inter, int64_t layers, int64_t nq, int64_t nkv,
                       int64_t head_dim, float eps, float theta, const float* embed, const float* final_norm,
                       const ref_layer* lw) {
    ref_model* m = new ref_model();
    ModelConfig& cfg = m->cfg;
    cfg.model_type = "llama";
    cfg.vocab_size = (int)vocab;
    cfg.hidden_size = (int)hidden;
    cfg.intermediate_size = (int)inter;
    cfg.num_hidden_layers = (int)layers;
    cfg.num_attention_heads = (int)nq;
    cfg.num_key_value_heads = (int)nkv;
    cfg.head_dim = (int)head_dim;
    cfg.rms_norm_eps = eps;
    cfg.rope_theta = theta;
    cfg.tie_word_embeddings = true;
    const size_t H = hidden, kvd = nkv * head_dim, I = inter;
    put(m->w.embed_tokens, embed, (size_t)vocab * H);
    put(m->w.final_norm, final_norm, H);
    m->w.layers.resize(layers);
    for (int64_t l = 0; l < layers; ++l) {
        auto& d = m->w.layers[l];
        const ref_layer& s = lw[l];
        put(d.input_layernorm, s.ln1, H);
        put(d.post_attention_layernorm, s.ln2, H);
        put(d.q_proj_weight, s.wq, H * H);
        put(d.q_proj_bias, s.bq, H);
        put(d.k_proj_weight, s.wk, kvd * H);
        put(d.k_proj_bias, s.bk, kvd);
        put(d.v_proj_weight, s.wv, kvd * H);
        put(d.v_proj_bias, s.bv, kvd);
        put(d.o_proj_weight, s.wo, H * H);
        put(d.gate_proj_weight, s.wg, I * H);
        put(d.up_proj_weight, s.wu, I * H);
        put(d.down_proj_weight, s.wd, H * I);
    }
    return m;
}

int ref_model_forward(void* h, const int64_t* ids, int64_t S, float* logits_out) {
    ref_model* m = static_cast<ref_model*>(h);
    std::vector<int64_t> tok(ids, ids + S);
    std::vector<float> out = forward_cpu(tok, m->cfg, m->w, "");
    if (logits_out) std::memcpy(logits_out, out.data(), out.size() * sizeof(float));
    return 0;
}

void ref_model_destroy(void* h) { delete static_cast<ref_model*>(h); }

}  // extern "C"
