// sampler.cu -- on-device token selection.
//
//   * repetition penalty once per distinct history id;
//   * greedy: multi-CTA argmax, one packed (value, id) 64-bit atomicMax per
//     CTA (ties to the lowest id);
//   * top-k / temperature / top-p: one 1024-thread CTA finds the k-th largest
//     key by 4 passes of 8-bit radix selection (warp-aggregated shared-memory
//     histograms), gathers exactly k candidates (ties at the threshold taken in
//     id order), bitonic-sorts them by (value desc, id asc) and runs the
//     reference's sequential float tail (softmax, top-p cut, renormalise, CDF
//     walk against the LCG uniform) in one thread.
// The LCG itself is the reference's host generator (state kept in the sampler
// object), so draws match the reference given identical logits and seed.
// Reference replaced: src/runtime/sampler.cu:13-73, 145-184, 202-339 (1-CTA
// argmax; top-k, softmax and draw on the host after a device->host copy).
#include <cmath>
#include <cstdlib>
#include <new>

#include "common.cuh"

namespace b2 {

constexpr int kRealVocab = 151665;  // padded-vocabulary rule, sampler.cu:231-248
constexpr int kTopkThreads = 1024;

__global__ void copy_logits_kernel(const float* __restrict__ src, float* __restrict__ dst, int V,
                                   unsigned long long* key) {
    griddep_wait();
    if (blockIdx.x == 0 && threadIdx.x == 0) *key = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

__global__ void penalty_kernel(float* __restrict__ logits, const int64_t* __restrict__ hist, int n, int V,
                               float penalty) {
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int64_t t = hist[i];
        if (t < 0 || t >= V) continue;
        bool dup = false;
        for (int j = 0; j < i && !dup; ++j) dup = hist[j] == t;
        if (dup) continue;
        const float l = logits[t];
        logits[t] = l > 0.f ? l / penalty : l * penalty;
    }
}

__global__ void argmax_kernel(const float* __restrict__ logits, int active, unsigned long long* key) {
    __shared__ unsigned long long s_best[32];
    griddep_wait();
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < active; i += gridDim.x * blockDim.x) {
        const unsigned long long k = argmax_key(logits[i], (uint32_t)i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = s_best[w] > best ? s_best[w] : best;
        if (best) atomicMax(key, best);
    }
}

// Token id of the packed argmax key (0 when no candidate) into *token.
__global__ void key_to_token_kernel(const unsigned long long* __restrict__ key, int* __restrict__ token) {
    griddep_wait();
    const unsigned long long k = *key;
    *token = k ? (int)(~static_cast<uint32_t>(k & 0xffffffffull)) : 0;
}

__device__ __forceinline__ float masked_logit(const float* logits, int i, int V) {
    return (V > kRealVocab && i >= kRealVocab) ? -1e9f : logits[i];
}

// Exclusive prefix sum over the block (1024 threads); returns the prefix and
// writes the total to *total.
__device__ int block_exclusive_scan(int v, int* s_warp, int* total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    if (lane == 31) s_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int w = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        s_warp[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    const int before = wid > 0 ? s_warp[wid - 1] : 0;
    *total = s_warp[(blockDim.x >> 5) - 1];
    return before + x - v;
}

// One CTA of 1024 threads: top-k selection, sort, sequential tail; the id
// goes to *token_out (thread 0).  K <= 1024.
__device__ __forceinline__ int topk_select(const float* __restrict__ logits, int V, int K, float temperature,
                                           float top_p, float u) {
    __shared__ unsigned int s_hist[256];
    __shared__ unsigned int s_prefix, s_remaining;
    __shared__ int s_warp[32];
    __shared__ int s_count;
    __shared__ float s_val[kTopkThreads];
    __shared__ int s_id[kTopkThreads];
    __shared__ float s_prob[kTopkThreads];
    __shared__ int s_token;

    const int tid = threadIdx.x;
    unsigned int prefix = 0, pmask = 0;
    if (tid == 0) {
        s_prefix = 0;
        s_remaining = (unsigned)K;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kTopkThreads) s_hist[i] = 0;
        __syncthreads();
        prefix = s_prefix;
        for (int base = 0; base < V; base += kTopkThreads) {
            const int i = base + tid;
            bool ok = false;
            unsigned bin = 0;
            if (i < V) {
                const unsigned key = float_key(masked_logit(logits, i, V));
                ok = (key & pmask) == prefix;
                bin = (key >> shift) & 255u;
            }
            const unsigned act = __ballot_sync(0xffffffffu, ok);
            if (ok) {
                const unsigned peers = __match_any_sync(act, bin);
                if ((threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&s_hist[bin], (unsigned)__popc(peers));
            }
        }
        __syncthreads();
        if (tid == 0) {
            unsigned rem = s_remaining, cum = 0;
            int d = 255;
            for (; d > 0; --d) {
                if (cum + s_hist[d] >= rem) break;
                cum += s_hist[d];
            }
            s_prefix = prefix | ((unsigned)d << shift);
            s_remaining = rem - cum;
        }
        pmask |= 255u << shift;
        __syncthreads();
    }
    const unsigned thr = s_prefix;
    const int need_ties = (int)s_remaining;

    // gather: strictly greater anywhere, ties in id order
    if (tid == 0) s_count = 0;
    __syncthreads();
    const int chunk = (V + kTopkThreads - 1) / kTopkThreads;
    const int i0 = tid * chunk, i1 = min(V, i0 + chunk);
    int ties = 0;
    for (int i = i0; i < i1; ++i) {
        const float v = masked_logit(logits, i, V);
        const unsigned key = float_key(v);
        if (key > thr) {
            const int slot = atomicAdd(&s_count, 1);
            s_val[slot] = v;
            s_id[slot] = i;
        } else if (key == thr) {
            ++ties;
        }
    }
    int total_ties = 0;
    const int before = block_exclusive_scan(ties, s_warp, &total_ties);
    __syncthreads();
    if (before < need_ties) {
        int take = need_ties - before;
        for (int i = i0; i < i1 && take > 0; ++i) {
            const float v = masked_logit(logits, i, V);
            if (float_key(v) == thr) {
                const int slot = atomicAdd(&s_count, 1);
                s_val[slot] = v;
                s_id[slot] = i;
                --take;
            }
        }
    }
    __syncthreads();

    // bitonic sort of P = next pow2 >= K entries: value desc, id asc
    int P = 1;
    while (P < K) P <<= 1;
    if (tid >= K && tid < P) {
        s_val[tid] = -INFINITY;
        s_id[tid] = 0x7fffffff;
    }
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int ixj = tid ^ j;
            if (tid < P && ixj > tid) {
                const float a = s_val[tid], b = s_val[ixj];
                const int ia = s_id[tid], ib = s_id[ixj];
                const bool a_first = a > b || (a == b && ia < ib);
                const bool up = (tid & k) == 0;
                if (up ? !a_first : a_first) {
                    s_val[tid] = b; s_val[ixj] = a;
                    s_id[tid] = ib; s_id[ixj] = ia;
                }
            }
            __syncthreads();
        }
    }

    // probabilities in parallel, exp evaluated in double and rounded to float
    const float maxv = s_val[0] / temperature;
    if (tid < K) {
        const float val = s_val[tid] / temperature;
        s_prob[tid] = (float)exp((double)(val - maxv));
    }
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int i = 0; i < K; ++i) sum += s_prob[i];
        for (int i = 0; i < K; ++i) s_prob[i] /= sum;
        int cut = K;
        float cum = 0.f;
        for (int i = 0; i < K; ++i) {
            cum += s_prob[i];
            if (cum >= top_p) { cut = i + 1; break; }
        }
        float sub = 0.f;
        for (int i = 0; i < cut; ++i) sub += s_prob[i];
        for (int i = 0; i < cut; ++i) s_prob[i] /= sub;
        float cdf = 0.f;
        int sel = cut - 1;
        for (int i = 0; i < cut; ++i) {
            cdf += s_prob[i];
            if (u <= cdf) { sel = i; break; }
        }
        s_token = s_id[sel];
    }
    __syncthreads();
    return s_token;
}

__global__ void __launch_bounds__(kTopkThreads) topk_sample_kernel(const float* __restrict__ logits, int V, int K,
                                                                   float temperature, float top_p, float u,
                                                                   int* __restrict__ token_out) {
    griddep_wait();
    const int t = topk_select(logits, V, K, temperature, top_p, u);
    if (threadIdx.x == 0) *token_out = t;
}

// The reference's LCG draw (src/runtime/sampler.cu:321-328): reseed iff
// seed != 0 and seed != state, advance, u = (state >> 40) * 2^-24.
__device__ __forceinline__ float lcg_draw(uint64_t* state, uint64_t seed) {
    uint64_t st = *state;
    if (seed != 0 && seed != st) st = seed;
    st = st * 6364136223846793005ull + 1442695040888963407ull;
    *state = st;
    return static_cast<float>(static_cast<double>(st >> 40) * (1.0 / 16777216.0));
}

// Decode-step sampling: CTA b draws sequence b's token from its logits row
// with its own LCG state (cfg in device memory, so a captured step picks up
// a new configuration without recapture) and stores it as a packed argmax
// key, which the step's end kernel turns into the next token.
__global__ void __launch_bounds__(kTopkThreads) step_sample_kernel(const float* __restrict__ logits, int64_t ld,
                                                                   int V, const b2_sampler_config* __restrict__ cfg,
                                                                   int max_top_k, uint64_t* __restrict__ rng,
                                                                   unsigned long long* __restrict__ argmax) {
    griddep_wait();
    const int b = blockIdx.x;
    __shared__ float s_u;
    const b2_sampler_config c = *cfg;
    if (threadIdx.x == 0) s_u = lcg_draw(rng + b, c.seed);
    __syncthreads();
    int K = c.top_k;
    if (K <= 0 || K > max_top_k) K = max_top_k < 64 ? max_top_k : 64;
    if (K > V) K = V;
    const int t = topk_select(logits + (int64_t)b * ld, V, K, c.temperature, c.top_p, s_u);
    if (threadIdx.x == 0) argmax[b] = argmax_key(0.f, (uint32_t)t);
}

int step_sample_launch(const float* logits, int64_t ld, int V, int B, const b2_sampler_config* d_cfg,
                       uint64_t* d_rng, unsigned long long* d_argmax, cudaStream_t s) {
    B2_TRY(launch(step_sample_kernel, dim3((unsigned)B), dim3(kTopkThreads), 0, s, true, logits, ld, V, d_cfg,
                  kTopkThreads, d_rng, d_argmax));
    return B2_OK;
}

}  // namespace b2

using namespace b2;

#define M_TRY_S(expr)                 \
    do {                              \
        const int rc_ = (expr);       \
        if (rc_ != B2_OK) return rc_; \
    } while (0)

struct b2_sampler {
    int device = 0;
    int vocab = 0;
    int max_top_k = 1024;
    uint64_t rng = 13374269ull;  // initial state of the reference sampler (sampler.cu:195)
    float* d_work = nullptr;
    int64_t* d_hist = nullptr;
    int hist_cap = 0;
    unsigned long long* d_key = nullptr;
    int* d_token = nullptr;
    unsigned long long* h_key = nullptr;  // pinned
    int* h_token = nullptr;               // pinned
};

extern "C" int b2_sampler_create(int vocab, int max_top_k, b2_sampler** out) {
    B2_REQUIRE(out && vocab > 0 && max_top_k > 0);
    *out = nullptr;
    b2_sampler* s = new (std::nothrow) b2_sampler();
    if (!s) return B2_ERR_INVALID;
    cudaGetDevice(&s->device);
    s->vocab = vocab;
    s->max_top_k = max_top_k > kTopkThreads ? kTopkThreads : max_top_k;
    s->hist_cap = 4096;
    cudaError_t e = cudaMalloc(&s->d_work, sizeof(float) * (size_t)vocab);
    if (e == cudaSuccess) e = cudaMalloc(&s->d_hist, sizeof(int64_t) * (size_t)s->hist_cap);
    if (e == cudaSuccess) e = cudaMalloc(&s->d_key, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_token, sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&s->h_key, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMallocHost(&s->h_token, sizeof(int));
    if (e != cudaSuccess) {
        b2_sampler_destroy(s);
        return (int)e;
    }
    *out = s;
    return B2_OK;
}

extern "C" int b2_sampler_destroy(b2_sampler* s) {
    if (!s) return B2_OK;
    cudaFree(s->d_work);
    cudaFree(s->d_hist);
    cudaFree(s->d_key);
    cudaFree(s->d_token);
    cudaFreeHost(s->h_key);
    cudaFreeHost(s->h_token);
    delete s;
    return B2_OK;
}

extern "C" uint64_t b2_sampler_rng_state(const b2_sampler* s) { return s ? s->rng : 0; }

extern "C" int b2_sampler_set_rng_state(b2_sampler* s, uint64_t state) {
    B2_REQUIRE(s);
    s->rng = state;
    return B2_OK;
}

// Enqueue the selection for logits `d_logits` with a device-side history;
// the chosen id goes to d_token (device).  Host-side state: the LCG.
static int sample_enqueue(b2_sampler* s, const float* d_logits, const int64_t* d_hist, int history_len,
                          const b2_sampler_config* cfg, cudaStream_t st, int* d_token) {
    const int V = s->vocab;
    const float* lg = d_logits;
    const int blocks = sm_count() * 2;
    if (cfg->repetition_penalty != 1.0f && history_len > 0) {
        B2_TRY(launch(copy_logits_kernel, dim3(blocks), dim3(256), 0, st, false, d_logits, s->d_work, V, s->d_key));
        B2_TRY(launch(penalty_kernel, dim3((history_len + 127) / 128), dim3(128), 0, st, false, s->d_work, d_hist,
                      history_len, V, cfg->repetition_penalty));
        lg = s->d_work;
    }
    if (cfg->temperature <= 1e-6f) {
        const int active = V > kRealVocab ? kRealVocab : V;
        B2_TRY(cudaMemsetAsync(s->d_key, 0, sizeof(unsigned long long), st));
        B2_TRY(launch(argmax_kernel, dim3(blocks), dim3(256), 0, st, false, lg, active, s->d_key));
        B2_TRY(launch(key_to_token_kernel, dim3(1), dim3(1), 0, st, false, (const unsigned long long*)s->d_key, d_token));
        return B2_OK;
    }
    int K = cfg->top_k;
    if (K <= 0 || K > s->max_top_k) K = s->max_top_k < 64 ? s->max_top_k : 64;
    if (K > V) K = V;
    // host LCG exactly as the reference (sampler.cu:321-328)
    if (cfg->seed != 0 && cfg->seed != s->rng) s->rng = cfg->seed;
    s->rng = s->rng * 6364136223846793005ull + 1442695040888963407ull;
    const float u = static_cast<float>(static_cast<double>(s->rng >> 40) * (1.0 / 16777216.0));
    B2_TRY(launch(topk_sample_kernel, dim3(1), dim3(kTopkThreads), 0, st, false, lg, V, K, cfg->temperature,
                  cfg->top_p, u, d_token));
    return B2_OK;
}

extern "C" int b2_sampler_sample_async(b2_sampler* s, const float* d_logits, const int64_t* d_history,
                                       int history_len, const b2_sampler_config* cfg, void* stream, int* d_token) {
    B2_REQUIRE(s && d_logits && cfg && d_token && history_len >= 0 && (history_len == 0 || d_history));
    return sample_enqueue(s, d_logits, d_history, history_len, cfg, as_stream(stream), d_token);
}

extern "C" int b2_sampler_sample(b2_sampler* s, const float* d_logits, const int64_t* history, int history_len,
                                 const b2_sampler_config* cfg, void* stream, int* token_out) {
    B2_REQUIRE(s && d_logits && cfg && token_out && history_len >= 0 && (history_len == 0 || history));
    cudaStream_t st = as_stream(stream);
    const bool pen = cfg->repetition_penalty != 1.0f && history_len > 0;
    if (pen) {
        if (history_len > s->hist_cap) {  // grown here; b2_sampler_sample_async never allocates
            cudaFree(s->d_hist);
            s->d_hist = nullptr;
            s->hist_cap = 0;
            B2_TRY(cudaMalloc(&s->d_hist, sizeof(int64_t) * (size_t)history_len * 2));
            s->hist_cap = history_len * 2;
        }
        B2_TRY(cudaMemcpyAsync(s->d_hist, history, sizeof(int64_t) * (size_t)history_len, cudaMemcpyHostToDevice, st));
    }
    M_TRY_S(sample_enqueue(s, d_logits, s->d_hist, pen ? history_len : 0, cfg, st, s->d_token));
    B2_TRY(cudaMemcpyAsync(s->h_token, s->d_token, sizeof(int), cudaMemcpyDeviceToHost, st));
    B2_TRY(cudaStreamSynchronize(st));
    *token_out = *s->h_token;
    return B2_OK;
}
