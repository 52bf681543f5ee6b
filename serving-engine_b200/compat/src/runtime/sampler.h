// compat/src/runtime/sampler.h -- the reference's SamplerGPU / SamplerConfig
// (src/runtime/sampler.h:10-65) over the b2engine sampler: repetition
// penalty, argmax or top-k / temperature / top-p selection and the seeded LCG
// draw all run on the device (b2_sampler_sample); only the chosen id comes
// back.  Public interface and defaults as in the reference.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "src/b2_compat.h"

namespace engine {

struct SamplerConfig {
    float temperature = 0.0f;         // 0.0 = greedy argmax
    int top_k = 0;                    // <= 0: default top-k (64)
    float top_p = 1.0f;               // >= 1.0: disabled
    float repetition_penalty = 1.0f;  // 1.0 = no penalty
    uint64_t seed = 42;
};

class SamplerGPU {
public:
    SamplerGPU() = default;
    explicit SamplerGPU(int vocab_size, int max_top_k = 1024) { init(vocab_size, max_top_k); }
    ~SamplerGPU() { release(); }
    SamplerGPU(const SamplerGPU&) = delete;
    SamplerGPU& operator=(const SamplerGPU&) = delete;

    void init(int vocab_size, int max_top_k = 1024) {
        release();
        vocab_size_ = vocab_size;
        cuda::b2_check(b2_sampler_create(vocab_size, max_top_k, &s_), "SamplerGPU::init");
        cuda::b2_check((int)cudaMalloc(&d_logits_, (size_t)vocab_size * sizeof(float)), "SamplerGPU::init");
    }

    // d_logits: device fp32 [vocab_size], left unmodified; history: host ids.
    int sample(const float* d_logits, const std::vector<int64_t>& history, const SamplerConfig& config,
               cudaStream_t stream = 0) {
        const b2_sampler_config c{config.temperature, config.top_k, config.top_p, config.repetition_penalty,
                                  config.seed};
        int token = 0;
        cuda::b2_check(b2_sampler_sample(s_, d_logits, history.data(), (int)history.size(), &c, stream, &token),
                       "SamplerGPU::sample");
        return token;
    }

    // fp16 logits: widened on the host, then sampled as fp32 (the reference's
    // sample_half does the same, src/runtime/sampler.cu:342-355).
    int sample_half(const half* d_logits, const std::vector<int64_t>& history, const SamplerConfig& config,
                    cudaStream_t stream = 0) {
        std::vector<half> h(vocab_size_);
        cuda::b2_check((int)cudaMemcpyAsync(h.data(), d_logits, (size_t)vocab_size_ * sizeof(half),
                                            cudaMemcpyDeviceToHost, stream),
                       "SamplerGPU::sample_half");
        cuda::b2_check((int)cudaStreamSynchronize(stream), "SamplerGPU::sample_half");
        std::vector<float> f(vocab_size_);
        for (int i = 0; i < vocab_size_; ++i) f[i] = __half2float(h[i]);
        return sample_from_float_host(f.data(), history, config);
    }

    // Host fp32 logits [vocab_size]: uploaded, then sampled on the device.
    int sample_from_float_host(const float* h_logits, const std::vector<int64_t>& history,
                               const SamplerConfig& config) {
        cuda::b2_check((int)cudaMemcpy(d_logits_, h_logits, (size_t)vocab_size_ * sizeof(float),
                                       cudaMemcpyHostToDevice),
                       "SamplerGPU::sample_from_float_host");
        return sample(d_logits_, history, config);
    }

private:
    void release() {
        if (s_) b2_sampler_destroy(s_);
        if (d_logits_) cudaFree(d_logits_);
        s_ = nullptr;
        d_logits_ = nullptr;
    }

    int vocab_size_ = 0;
    b2_sampler* s_ = nullptr;
    float* d_logits_ = nullptr;
};

}  // namespace engine
