// compat/src/model/forward_gpu.h -- the reference's model-level GPU API
// (src/model/forward_gpu.h:15-113) over the b2engine model runtime, so that
// its callers (apps/generate.cpp, tests/test_kv_cache.cpp) build unchanged.
//
// The weights, the KV cache and the captured decode-step graph live in one
// b2engine model (b2_model, include/b2engine.h) held by ModelWeightsGPU:
//   * init_from_weights uploads every bf16 checkpoint tensor with
//     b2_model_set_tensor_bf16, which converts it to fp16 on the device (the
//     reference converts on the host, src/model/forward_gpu.cu:18-28);
//   * prefill_gpu / decode_step_gpu run b2_model_prefill / b2_model_decode_step
//     (or b2_model_decode_enqueue when d_last_logits is given, without a host
//     round trip), and keep KVCache's length in step as the reference does;
//     the cache contents themselves are the model's (same [layer][K,V][head]
//     [pos][dim] layout for its single sequence), so KVCache carries only the
//     length here;
//   * forward_gpu is b2_model_forward_logits (full recompute on the tensor
//     cores, logits of every position).
// The public data members of the reference's structs are kept so that code
// naming them compiles; the DeviceBuffer members of ModelWeightsGPU stay
// empty, and of ActivationBuffersGPU only `logits` ([vocab] fp32, the usual
// d_last_logits target) is allocated.  Work is ordered against the legacy
// default stream, like the reference's launches.  The cuBLAS handle argument
// is accepted and not used (no cuBLAS call remains on this path).
#pragma once

#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "src/b2_compat.h"
#include "src/common/cuda_utils.h"
#include "src/model/config.h"
#include "src/runtime/kv_cache.h"

namespace engine {

struct ModelWeightsGPU {
    DeviceBuffer<half> embed_tokens;  // left empty: the weights live in `model`
    DeviceBuffer<half> final_norm;

    struct LayerGPU {
        DeviceBuffer<half> input_layernorm;
        DeviceBuffer<half> post_attention_layernorm;
        DeviceBuffer<half> q_proj_weight;
        DeviceBuffer<half> q_proj_bias;
        DeviceBuffer<half> k_proj_weight;
        DeviceBuffer<half> k_proj_bias;
        DeviceBuffer<half> v_proj_weight;
        DeviceBuffer<half> v_proj_bias;
        DeviceBuffer<half> o_proj_weight;
        DeviceBuffer<half> gate_proj_weight;
        DeviceBuffer<half> up_proj_weight;
        DeviceBuffer<half> down_proj_weight;
    };

    std::vector<LayerGPU> layers;

    // Creates the b2engine model (one sequence, KV capacity
    // min(max_position_embeddings, 4096) positions) and uploads the bf16
    // checkpoint tensors, converted to fp16 on the device.  false on failure
    // (the reason goes to stderr), as in the reference.
    bool init_from_weights(const ModelConfig& config, const ModelWeights& weights);

    std::shared_ptr<b2_model> model;  // weights, KV cache, decode-step graph
    int max_seq = 0;                  // positions the model's KV cache holds
};

struct ActivationBuffersGPU {
    DeviceBuffer<half> hidden_states;
    DeviceBuffer<half> norm_out;
    DeviceBuffer<half> q;
    DeviceBuffer<half> k;
    DeviceBuffer<half> v;
    DeviceBuffer<half> attn_out;
    DeviceBuffer<half> proj_out;
    DeviceBuffer<half> gate;
    DeviceBuffer<half> up;
    DeviceBuffer<half> act;
    DeviceBuffer<half> mlp_out;
    DeviceBuffer<float> logits;  // [vocab_size] fp32
    DeviceBuffer<int64_t> token_ids_d;
    DeviceBuffer<int> decode_seq_len;
    DeviceBuffer<float> split_kv_buf;

    int64_t max_seq = 0;

    void allocate(const ModelConfig& config, int64_t max_seq_len);
};

struct KernelRecord {
    std::string name;
    float ms;
};

// Logits of every position, host fp32 [seq_len * vocab_size].  dump_dir:
// only the logits are written (logits.npy); profile_records receives one
// record for the whole forward.
std::vector<float> forward_gpu(const std::vector<int64_t>& token_ids, const ModelConfig& config,
                               const ModelWeightsGPU& weights, ActivationBuffersGPU& buffers,
                               cublasHandle_t cublas_handle, const std::string& dump_dir = "",
                               std::vector<KernelRecord>* profile_records = nullptr);

// Prefill from position 0; last-position logits as host fp32 [vocab_size],
// or (d_last_logits != nullptr) on the device only, returning an empty vector.
std::vector<float> prefill_gpu(const std::vector<int64_t>& token_ids, const ModelConfig& config,
                               const ModelWeightsGPU& weights, ActivationBuffersGPU& buffers, KVCache& kv_cache,
                               cublasHandle_t cublas_handle, float* d_last_logits = nullptr,
                               std::vector<KernelRecord>* profile_records = nullptr);

// One token at current_pos; logits as for prefill_gpu.  With d_last_logits
// the step is only enqueued (ordered before later work on the legacy stream).
std::vector<float> decode_step_gpu(int64_t token_id, int current_pos, const ModelConfig& config,
                                   const ModelWeightsGPU& weights, ActivationBuffersGPU& buffers, KVCache& kv_cache,
                                   cublasHandle_t cublas_handle, float* d_last_logits = nullptr,
                                   std::vector<KernelRecord>* profile_records = nullptr);

}  // namespace engine
