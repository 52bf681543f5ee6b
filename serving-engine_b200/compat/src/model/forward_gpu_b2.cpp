// compat/src/model/forward_gpu_b2.cpp -- the reference's ModelWeightsGPU /
// ActivationBuffersGPU / forward_gpu / prefill_gpu / decode_step_gpu
// (src/model/forward_gpu.h:15-113) implemented over the b2engine C-ABI.
// Built together with the reference's own callers against the compatibility
// headers; see forward_gpu.h for what maps onto what.
#include "src/model/forward_gpu.h"

#include <algorithm>
#include <chrono>
#include <filesystem>
#include <iostream>
#include <stdexcept>

#include "src/cpu/npy.h"

namespace engine {

namespace {

b2_model* model_of(const ModelWeightsGPU& w) {
    if (!w.model) throw std::runtime_error("b2engine: ModelWeightsGPU used before init_from_weights");
    return w.model.get();
}

cudaStream_t stream_of(b2_model* m) { return static_cast<cudaStream_t>(b2_model_stream(m)); }

// The reference enqueues everything on the legacy default stream; the model
// runs on its own stream, so each call is ordered against the legacy stream
// on both sides with events.
void model_after_legacy(b2_model* m) {
    cudaEvent_t e;
    cuda::b2_check((int)cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
    cudaEventRecord(e, 0);
    cudaStreamWaitEvent(stream_of(m), e, 0);
    cudaEventDestroy(e);
}

void legacy_after_model(b2_model* m) {
    cudaEvent_t e;
    cuda::b2_check((int)cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
    cudaEventRecord(e, stream_of(m));
    cudaStreamWaitEvent(0, e, 0);
    cudaEventDestroy(e);
}

void check_len(const ModelWeightsGPU& w, int64_t positions, const char* what) {
    if (positions > w.max_seq)
        throw std::runtime_error(std::string("b2engine ") + what + ": " + std::to_string(positions) +
                                 " positions exceed the model's KV capacity of " + std::to_string(w.max_seq));
}

double ms_since(std::chrono::high_resolution_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0).count();
}

}  // namespace

bool ModelWeightsGPU::init_from_weights(const ModelConfig& config, const ModelWeights& weights) {
    try {
        const int L = config.num_hidden_layers, H = config.hidden_size, I = config.intermediate_size;
        const int D = config.head_dim, kvd = config.num_key_value_heads * D, qd = config.num_attention_heads * D;
        bool bias = !weights.layers.empty();
        for (const auto& lw : weights.layers)
            bias = bias && lw.q_proj_bias && lw.k_proj_bias && lw.v_proj_bias;
        b2_model_config mc{};
        mc.vocab_size = config.vocab_size;
        mc.hidden_size = H;
        mc.intermediate_size = I;
        mc.num_layers = L;
        mc.num_q_heads = config.num_attention_heads;
        mc.num_kv_heads = config.num_key_value_heads;
        mc.head_dim = D;
        mc.rms_norm_eps = config.rms_norm_eps;
        mc.rope_theta = config.rope_theta;
        mc.tie_word_embeddings = config.tie_word_embeddings ? 1 : 0;
        mc.has_qkv_bias = bias ? 1 : 0;
        mc.max_batch = 1;
        mc.max_seq = std::min(config.max_position_embeddings, 4096);
        b2_model* m = nullptr;
        cuda::b2_check(b2_model_create(&mc, 0, 1, nullptr, &m), "ModelWeightsGPU::init_from_weights");
        model.reset(m, [](b2_model* p) { b2_model_destroy(p); });
        max_seq = mc.max_seq;
        auto put = [&](const std::string& name, const void* src, int64_t rows, int64_t cols) {
            cuda::b2_check(b2_model_set_tensor_bf16(m, name.c_str(), static_cast<const uint16_t*>(src), rows, cols),
                           ("upload " + name).c_str());
        };
        put("embed", weights.embed_tokens, config.vocab_size, H);
        if (!config.tie_word_embeddings) put("lm_head", weights.lm_head, config.vocab_size, H);
        put("final_norm", weights.final_norm, 1, H);
        for (int l = 0; l < L; ++l) {
            const LayerWeights& lw = weights.layers[l];
            const std::string p = std::to_string(l) + ".";
            put(p + "ln1", lw.input_layernorm, 1, H);
            put(p + "ln2", lw.post_attention_layernorm, 1, H);
            put(p + "wq", lw.q_proj_weight, qd, H);
            put(p + "wk", lw.k_proj_weight, kvd, H);
            put(p + "wv", lw.v_proj_weight, kvd, H);
            if (bias) {
                put(p + "bq", lw.q_proj_bias, 1, qd);
                put(p + "bk", lw.k_proj_bias, 1, kvd);
                put(p + "bv", lw.v_proj_bias, 1, kvd);
            }
            put(p + "wo", lw.o_proj_weight, H, qd);
            put(p + "wg", lw.gate_proj_weight, I, H);
            put(p + "wu", lw.up_proj_weight, I, H);
            put(p + "wd", lw.down_proj_weight, H, I);
        }
        layers.resize(L);
        return true;
    } catch (const std::exception& e) {
        std::cerr << "init_from_weights failed: " << e.what() << std::endl;
        model.reset();
        return false;
    }
}

void ActivationBuffersGPU::allocate(const ModelConfig& config, int64_t max_seq_len) {
    logits.allocate((size_t)config.vocab_size);
    max_seq = max_seq_len;
}

std::vector<float> forward_gpu(const std::vector<int64_t>& token_ids, const ModelConfig& config,
                               const ModelWeightsGPU& weights, ActivationBuffersGPU& buffers,
                               cublasHandle_t cublas_handle, const std::string& dump_dir,
                               std::vector<KernelRecord>* profile_records) {
    (void)buffers;
    (void)cublas_handle;
    b2_model* m = model_of(weights);
    const int64_t S = (int64_t)token_ids.size();
    check_len(weights, S, "forward_gpu");
    std::vector<float> logits((size_t)S * config.vocab_size);
    model_after_legacy(m);
    const auto t0 = std::chrono::high_resolution_clock::now();
    cuda::b2_check(b2_model_forward_logits(m, token_ids.data(), (int)S, logits.data()), "forward_gpu");
    if (profile_records) profile_records->push_back({"forward (b2engine prefill + lm_head)", (float)ms_since(t0)});
    if (!dump_dir.empty()) {
        std::filesystem::create_directories(dump_dir);
        NpyWriter::write_f32(dump_dir + "/logits.npy", logits.data(), {1, S, (int64_t)config.vocab_size});
    }
    return logits;
}

std::vector<float> prefill_gpu(const std::vector<int64_t>& token_ids, const ModelConfig& config,
                               const ModelWeightsGPU& weights, ActivationBuffersGPU& buffers, KVCache& kv_cache,
                               cublasHandle_t cublas_handle, float* d_last_logits,
                               std::vector<KernelRecord>* profile_records) {
    (void)buffers;
    (void)cublas_handle;
    b2_model* m = model_of(weights);
    const int64_t S = (int64_t)token_ids.size();
    check_len(weights, S, "prefill_gpu");
    std::vector<float> out;
    if (!d_last_logits) out.resize((size_t)config.vocab_size);
    model_after_legacy(m);
    const auto t0 = std::chrono::high_resolution_clock::now();
    cuda::b2_check(b2_model_reset(m), "prefill_gpu");
    cuda::b2_check(b2_model_prefill(m, token_ids.data(), 1, (int)S, d_last_logits ? nullptr : out.data()),
                   "prefill_gpu");
    if (d_last_logits) {
        cuda::b2_check((int)cudaMemcpyAsync(d_last_logits, b2_model_buffer(m, "logits"),
                                            (size_t)config.vocab_size * sizeof(float), cudaMemcpyDeviceToDevice,
                                            stream_of(m)),
                       "prefill_gpu");
        legacy_after_model(m);
    }
    if (profile_records) profile_records->push_back({"prefill (b2engine)", (float)ms_since(t0)});
    kv_cache.set_current_seq_len((int)S);
    return out;
}

std::vector<float> decode_step_gpu(int64_t token_id, int current_pos, const ModelConfig& config,
                                   const ModelWeightsGPU& weights, ActivationBuffersGPU& buffers, KVCache& kv_cache,
                                   cublasHandle_t cublas_handle, float* d_last_logits,
                                   std::vector<KernelRecord>* profile_records) {
    (void)buffers;
    (void)cublas_handle;
    b2_model* m = model_of(weights);
    check_len(weights, (int64_t)current_pos + 1, "decode_step_gpu");
    std::vector<float> out;
    model_after_legacy(m);
    const auto t0 = std::chrono::high_resolution_clock::now();
    if (d_last_logits) {
        cuda::b2_check(b2_model_decode_enqueue(m, &token_id, &current_pos, 1, d_last_logits), "decode_step_gpu");
        legacy_after_model(m);
    } else {
        out.resize((size_t)config.vocab_size);
        cuda::b2_check(b2_model_decode_step(m, &token_id, &current_pos, 1, out.data(), nullptr), "decode_step_gpu");
    }
    if (profile_records) {
        if (d_last_logits) cudaStreamSynchronize(stream_of(m));
        profile_records->push_back({"decode_step (b2engine graph)", (float)ms_since(t0)});
    }
    kv_cache.set_current_seq_len(current_pos + 1);
    return out;
}

}  // namespace engine
