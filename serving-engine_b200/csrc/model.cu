// model.cu -- decode-step runtime: sharded weights, KV cache, seeded
// initialisation, the per-token step as one captured CUDA graph, greedy
// generation on the device, and Megatron tensor parallelism over NCCL.
//
// One decode step for B sequences (per rank, tp = tensor-parallel degree):
//   step_begin   hidden[b] = embed[token[b]] (fp32 residual stream),
//                seq_len[b] = pos[b] + 1, argmax[b] = 0
//   per layer    qkv     RMSNorm(ln1) prologue, fused q|k|v GEMV, RoPE
//                        epilogue, K/V written straight into the cache
//                attn    split-KV GQA attention, splits merged in-kernel
//                o       GEMV, residual added into hidden (rank 0 only) ...
//                [tp>1]  ncclAllReduce(hidden, sum)  ... the sum is the new hidden
//                gateup  RMSNorm(ln2) prologue, gate and up GEMV, SwiGLU epilogue
//                down    GEMV, residual into hidden; [tp>1] ncclAllReduce
//   lm_head      RMSNorm(final) prologue, vocabulary-shard GEMV to fp32 logits
//                with a packed per-sequence argmax; [tp>1] ncclAllReduce(max)
//   step_end     token[b] = argmax id, pos[b] += 1, history append
// Everything reads tokens / positions from device memory, so the captured
// graph is replayed unchanged step after step.
//
// Reference replaced: src/model/forward_gpu.cu:30-101 (weights, buffers),
// :329-520 (prefill), :523-707 (decode_step_gpu: 13 launches per layer on the
// legacy stream, synchronous H2D/D2H each token, no graph), and the KV layout
// of src/runtime/kv_cache.h:12-73.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "prefill.cuh"
#include "skinny.cuh"

#include <cooperative_groups.h>
namespace cg = cooperative_groups;

namespace b2 {

// Batches up to kGemvMaxBatch decode with the fused GEMVs; larger batches
// run the projections on the tensor cores (skinny weight stream, weights
// read once per step for the whole batch).  Past 4 sequences a GEMV is
// bound by its multiply-adds and shared-memory reads rather than HBM
// (Llama-3-8B shape, batch 8: 1200 tok/s against 1993 on the tensor cores;
// batch 4: 1039 against 998).
constexpr int kGemvMaxBatch = 4;
// FP8 weights (b2_model_quantize_weights) are read by the GEMV step up to
// this batch; above it the E4M3 decode adds to a compute-bound kernel
// (batch 4: 927 tok/s against 1039 with fp16 weights) and the fp16 copies
// are streamed instead.  The batched tensor-core step (batch > 4) reads the
// FP8 copies up to 128 sequences (skinny.cu: weight tiles decoded into TMEM).
constexpr int kFp8MaxBatch = 2;
// 4-bit weights: the GEMV step at batch 1-2 only (the batched tensor-core
// step streams the fp16 weights).
constexpr int kI4MaxBatch = 2;
constexpr int kMaxBatch = 256;

struct AttnParams;
int attn_pick_splits(int batch, int nq, int nkv, int D, int max_len, size_t cap_floats);
size_t attn_scratch_floats(int batch, int nq, int nkv, int D, int splits);
bool attn_head_dim_supported(int D);
int attn_decode_launch_step(const __half* q, const __half* kbase, const __half* vbase, int64_t sb, int64_t sh,
                            int64_t ss, const int* seq_lens, __half* out, float* part, int splits, int B, int nq,
                            int nkv, int D, cudaStream_t s, TraceSlot trace);

enum TcEpi : int { TC_HALF = 0, TC_F32 = 1, TC_F32_ADD = 2 };
int gemm_tc(const __half* A, const __half* B, void* C, int M, int N, int K, int epi, cudaStream_t s);
int attn_decode_launch_step_q(const __half* q, int64_t q_sb, const __half* kbase, const __half* vbase, int64_t sb,
                              int64_t sh, int64_t ss, const int* seq_lens, __half* out, float* part, int splits,
                              int B, int nq, int nkv, int D, cudaStream_t s);
int* wait_error_word();
int step_sample_launch(const float* logits, int64_t ld, int V, int B, const b2_sampler_config* d_cfg,
                       uint64_t* d_rng, unsigned long long* d_argmax, cudaStream_t s);

// ---------------------------------------------------------------------------
// seeded initialisation (bit-identical to oracle/b2oracle.c ora_init_value)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// dst[r * cols + c] = value(tensor_id, (row0 + r) * ld_global + col0 + c)
__global__ void init_tensor_kernel(__half* __restrict__ dst, int64_t rows, int64_t cols, uint64_t seed,
                                   uint64_t tensor_id, int64_t row0, int64_t col0, int64_t ld_global, float scale) {
    const uint64_t key = mix64(seed + 0x9E3779B97F4A7C15ull * (tensor_id + 1));
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i - (i / cols) * cols;
        const uint64_t idx = (uint64_t)(row0 + r) * (uint64_t)ld_global + (uint64_t)(col0 + c);
        const uint64_t h = mix64(key ^ idx);
        const int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
                          (int32_t)((h >> 48) & 0xFFFF);
        dst[i] = __float2half_rn(__fmul_rn((float)(s - 131070), scale));
    }
}

__global__ void fill_half_kernel(__half* dst, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(v);
}

// ---------------------------------------------------------------------------
// step boundary kernels
// ---------------------------------------------------------------------------
// bf16 -> fp16 in place, by the checkpoint loader's bit rule
// (src/loader/safetensors.cpp:307-328): the 8-bit exponent is rebased to 5
// bits, values below the fp16 normal range become signed zero, values above
// it (and inf / NaN) signed infinity, and the 7 mantissa bits move up
// unchanged (bf16's mantissa fits fp16's, so normal values convert exactly).
__global__ void bf16_to_f16_kernel(uint16_t* __restrict__ p, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t u = p[i];
        const uint32_t sign = u & 0x8000u;
        const int e = (int)((u >> 7) & 0xFFu) - 127 + 15;
        const uint32_t mant = (u & 0x7Fu) << 3;
        uint32_t o;
        if (e <= 0) o = sign;
        else if (e >= 31) o = sign | 0x7C00u;
        else o = sign | ((uint32_t)e << 10) | mant;
        p[i] = (uint16_t)o;
    }
}

// Step inputs passed by value (kernel parameters are captured at launch, so
// the caller's host memory is free as soon as the launch returns).
struct StepInputs {
    int64_t tokens[kMaxBatch];
    int positions[kMaxBatch];
};

__global__ void set_step_inputs_kernel(const StepInputs in, int B, int64_t* __restrict__ tokens,
                                       int* __restrict__ positions) {
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        tokens[b] = in.tokens[b];
        positions[b] = in.positions[b];
    }
}

__global__ void step_begin_kernel(const int64_t* __restrict__ tokens, const int* __restrict__ positions,
                                  const __half* __restrict__ embed, float* __restrict__ hidden, int H,
                                  int* __restrict__ seq_lens, unsigned long long* __restrict__ argmax,
                                  int64_t* __restrict__ hist, const int* __restrict__ hist_count, int hist_cap,
                                  TraceSlot trace) {
    griddep_wait();
    griddep_launch_dependents();
    trace_begin(trace);
    const int b = blockIdx.x;
    const int64_t id = tokens[b];
    const uint4* src = reinterpret_cast<const uint4*>(embed + id * H);
    float4* dst = reinterpret_cast<float4*>(hidden + (int64_t)b * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
        float f[8];
        unpack8(ldg16(src + i), f);
        dst[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
        dst[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
    }
    if (threadIdx.x == 0) {
        seq_lens[b] = positions[b] + 1;
        argmax[b] = 0ull;
        // the history records the token each step consumes
        const int c = *hist_count;
        if (c < hist_cap) hist[(int64_t)c * gridDim.x + b] = id;
    }
    __syncthreads();
    trace_end(trace);
}

// token[b] = argmax id, pos[b] += 1, history counter += 1.  With the peer
// exchange on, the argmax is the max over every rank's vocabulary shard
// (bounded wait for their flags) and the step counter advances.
__global__ void step_end_kernel(const unsigned long long* __restrict__ argmax, int64_t* __restrict__ tokens,
                                int* __restrict__ positions, int B, int* __restrict__ hist_count, int hist_cap,
                                int tp_on, const unsigned long long* am_recv, const unsigned* am_flags, int tp,
                                int Bmax, int* step, int* err, TraceSlot trace) {
    griddep_wait();
    trace_begin(trace);
    const int b = threadIdx.x;
    if (tp_on) {
        const unsigned tag = (unsigned)(*step) + 1u;
        if (b < tp) wait_flag_geq(am_flags + b, tag, err, 99);
        __syncthreads();
        if (b < B) {
            unsigned long long best = 0ull;
            for (int r = 0; r < tp; ++r) {
                const unsigned long long v = __ldcg(am_recv + (size_t)r * Bmax + b);
                best = v > best ? v : best;
            }
            tokens[b] = (int64_t)argmax_key_id(best);
            positions[b] += 1;
        }
        __syncthreads();
        if (b == 0) *step += 1;
    } else if (b < B) {
        tokens[b] = (int64_t)argmax_key_id(argmax[b]);
        positions[b] += 1;
    }
    if (b == 0) {
        const int c = *hist_count;
        if (c < hist_cap) *hist_count = c + 1;
    }
    __syncthreads();
    trace_end(trace);
}

// ---------------------------------------------------------------------------
// prefill kernels (all prompt tokens of all sequences at once, token-major
// rows t = b * S + s)
// ---------------------------------------------------------------------------
// hidden[t] = embed[ids[t]] as fp32
__global__ void embed_rows_kernel(const int64_t* __restrict__ ids, const __half* __restrict__ embed,
                                  float* __restrict__ hidden, int H) {
    const int64_t t = blockIdx.x;
    const uint4* src = reinterpret_cast<const uint4*>(embed + ids[t] * H);
    float4* dst = reinterpret_cast<float4*>(hidden + t * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
        float f[8];
        unpack8(ldg16(src + i), f);
        dst[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
        dst[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
    }
}

// out[t] = half(h * rsqrt(mean(h^2) + eps) * w) for the fp32 row h = hidden[t]
// (the arithmetic of the decode GEMV's RMSNorm prologue)
__global__ void rmsnorm_rows_kernel(const float* __restrict__ hidden, const __half* __restrict__ w,
                                    __half* __restrict__ out, int H, float eps) {
    __shared__ float red[32];
    const int64_t t = blockIdx.x;
    const float4* h = reinterpret_cast<const float4*>(hidden + t * H);
    float ss = 0.f;
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        const float4 v = h[i];
        ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
    }
    const float r = rsqrtf(block_sum(ss, red) / (float)H + eps);
    uint4* o = reinterpret_cast<uint4*>(out + t * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
        const float4 a0 = h[2 * c], a1 = h[2 * c + 1];
        float wv[8];
        unpack8(ldg16(reinterpret_cast<const uint4*>(w) + c), wv);
        float f[8] = {a0.x * r * wv[0], a0.y * r * wv[1], a0.z * r * wv[2], a0.w * r * wv[3],
                      a1.x * r * wv[4], a1.y * r * wv[5], a1.z * r * wv[6], a1.w * r * wv[7]};
        o[c] = pack8(f);
    }
}

// Rotate-half RoPE (model table) on the q and k heads of the fused q|k|v rows
// in place, and K / V of every token written into this layer's cache.
// grid (T, nq + 2 nkv), D/2 threads.
__global__ void rope_append_kernel(__half* __restrict__ qkv, int64_t ld, const float2* __restrict__ rope, int S,
                                   int nq, int nkv, int D, const KvLayout kv, int skip_pos,
                                   const int* __restrict__ positions) {
    griddep_wait();
    const int64_t t = blockIdx.x;
    // prefill: row t is position t % S of sequence t / S; decode (positions
    // given): row t is sequence t at positions[t]
    const int b = positions ? (int)t : (int)(t / S);
    const int pos = positions ? positions[t] : (int)(t - (int64_t)b * S);
    const int head = blockIdx.y, half = D >> 1, i = threadIdx.x;
    __half* row = qkv + t * ld + (int64_t)head * D;
    float x1 = __half2float(row[i]), x2 = __half2float(row[i + half]);
    if (head < nq + nkv) {
        const float2 cs = rope[(int64_t)pos * half + i];
        const float o1 = x1 * cs.x - x2 * cs.y;
        const float o2 = x2 * cs.x + x1 * cs.y;
        row[i] = __float2half_rn(o1);
        row[i + half] = __float2half_rn(o2);
        if (head >= nq && pos >= skip_pos) {
            __half* k = kv.k + kv_row(kv, b, head - nq, pos, D);
            k[i] = __float2half_rn(o1);
            k[i + half] = __float2half_rn(o2);
        }
    } else if (pos >= skip_pos) {
        __half* v = kv.v + kv_row(kv, b, head - nq - nkv, pos, D);
        v[i] = row[i];
        v[i + half] = row[i + half];
    }
}

// out[b] = hidden[b * S + S - 1] (the last prompt position of each sequence)
__global__ void gather_last_kernel(const float* __restrict__ hidden, float* __restrict__ out, int S, int H) {
    const int b = blockIdx.x;
    const float* src = hidden + ((int64_t)b * S + S - 1) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(int64_t)b * H + i] = src[i];
}

// decode state after a prefill of S tokens: next token = argmax, position S
__global__ void prefill_end_kernel(const unsigned long long* __restrict__ argmax, int64_t* __restrict__ tokens,
                                   int* __restrict__ positions, int B, int S) {
    griddep_wait();
    const int b = threadIdx.x;
    if (b < B) {
        tokens[b] = (int64_t)argmax_key_id(argmax[b]);
        positions[b] = S;
    }
}

// ---------------------------------------------------------------------------
// consumers of the skinny (decode-batch) projections: each sums the fp32
// partial slabs of its columns in slab order (skinny.cu) and fuses the
// operation that follows the projection.
// ---------------------------------------------------------------------------
struct SkSlabs {
    const float* ws;  // [slab][B][N]
    int N, nk, per;
    int col0;  // column of element 0 of this operand inside N
};

// columns n .. n+3 (n % 4 == 0, so one tile and one partial count)
__device__ __forceinline__ float4 sk_sum4(const SkSlabs& a, int B, int b, int n) {
    n += a.col0;
    const int ns = sk_nseg(n, a.nk, a.per);
    const size_t step = (size_t)B * a.N;
    const float* p = a.ws + (size_t)b * a.N + n;
    float4 x = *reinterpret_cast<const float4*>(p);
#pragma unroll 4
    for (int z = 1; z < ns; ++z) {
        const float4 v = *reinterpret_cast<const float4*>(p + z * step);
        x.x += v.x; x.y += v.y; x.z += v.z; x.w += v.w;
    }
    return x;
}

__device__ __forceinline__ float sk_sum(const SkSlabs& a, int B, int b, int n) {
    n += a.col0;
    const int ns = sk_nseg(n, a.nk, a.per);
    const size_t step = (size_t)B * a.N;
    const float* p = a.ws + (size_t)b * a.N + n;
    float x = p[0];
    for (int z = 1; z < ns; ++z) x += p[z * step];
    return x;
}

// q|k|v of sequence b: sum + bias, rounded to half (the projection's output
// type), RoPE (model table) on q and k, q into qkv row b, k and v appended
// to the cache at positions[b].  Thread = (head, 4 rotation pairs i..i+3 and
// i+D/2..); grid (B, ceil((nq + 2 nkv) D/8 / 256)), 256 threads.
__global__ void sk_qkv_rope_kernel(SkSlabs a, int B, const __half* __restrict__ bias, __half* __restrict__ qkv,
                                   int64_t ld, const float2* __restrict__ rope, int nq, int nkv, int D,
                                   const KvLayout kv, const int* __restrict__ positions, TraceSlot tr) {
    const int b = blockIdx.x, half = D >> 1, per_head = D >> 3;
    const int t = blockIdx.y * blockDim.x + threadIdx.x;
    const int head = t / per_head, i = (t - head * per_head) * 4;
    const bool live = head < nq + 2 * nkv;
    const int n1 = head * D + i, n2 = n1 + half;
    // the bias is never written by a kernel: fetch it before the wait
    __half bv1[4] = {}, bv2[4] = {};
    if (bias && live) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            bv1[e] = bias[n1 + e];
            bv2[e] = bias[n2 + e];
        }
    }
    griddep_wait();
    griddep_launch_dependents();
    trace_begin(tr);
    if (!live) {
        trace_end(tr);
        return;
    }
    const float4 s1 = sk_sum4(a, B, b, n1), s2 = sk_sum4(a, B, b, n2);
    float x1[4] = {s1.x, s1.y, s1.z, s1.w}, x2[4] = {s2.x, s2.y, s2.z, s2.w};
    __half o1[4], o2[4];
    const int pos = positions[b];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        if (bias) {
            x1[e] += __half2float(bv1[e]);
            x2[e] += __half2float(bv2[e]);
        }
        x1[e] = __half2float(__float2half_rn(x1[e]));
        x2[e] = __half2float(__float2half_rn(x2[e]));
        if (head < nq + nkv) {
            const float2 cs = rope[(int64_t)pos * half + i + e];
            o1[e] = __float2half_rn(x1[e] * cs.x - x2[e] * cs.y);
            o2[e] = __float2half_rn(x2[e] * cs.x + x1[e] * cs.y);
        } else {
            o1[e] = __float2half_rn(x1[e]);
            o2[e] = __float2half_rn(x2[e]);
        }
    }
    __half* dst;
    if (head < nq) dst = qkv + (int64_t)b * ld + (int64_t)head * D;
    else if (head < nq + nkv) dst = kv.k + kv_row(kv, b, head - nq, pos, D);
    else dst = kv.v + kv_row(kv, b, head - nq - nkv, pos, D);
    __half2 p0 = __halves2half2(o1[0], o1[1]), p1 = __halves2half2(o1[2], o1[3]);
    __half2 q0 = __halves2half2(o2[0], o2[1]), q1 = __halves2half2(o2[2], o2[3]);
    uint2 w1, w2;
    w1.x = *reinterpret_cast<uint32_t*>(&p0);
    w1.y = *reinterpret_cast<uint32_t*>(&p1);
    w2.x = *reinterpret_cast<uint32_t*>(&q0);
    w2.y = *reinterpret_cast<uint32_t*>(&q1);
    *reinterpret_cast<uint2*>(dst + i) = w1;
    *reinterpret_cast<uint2*>(dst + i + half) = w2;
    trace_end(tr);
}

// hidden[b] = (add ? hidden[b] : 0) + projection; then, when norm_w is set,
// xn[b] = half(hidden[b] * rsqrt(mean(hidden[b]^2) + eps) * norm_w).  One
// 1024-thread CTA per row (grid B), 4 columns per thread and pass; the row's
// sum of squares is reduced inside the CTA (warp trees, then a tree over the
// 32 warp sums: a fixed order, so deterministic).  (An 8-CTA cluster per row, partials shared
// through distributed shared memory, took 7.4 us against 5.5 at batch 8.)
constexpr int kAddNormRowThreads = 1024;

__global__ void __launch_bounds__(kAddNormRowThreads) sk_add_norm_kernel(SkSlabs a, int B,
                                                                            float* __restrict__ hidden, int add,
                                                                            int H, const __half* __restrict__ norm_w,
                                                                            __half* __restrict__ xn, float eps,
                                                                            TraceSlot tr) {
    __shared__ float red[kAddNormRowThreads / 32];
    __shared__ float s_rs;
    constexpr int kMaxV = 4;  // float4 groups per thread (H <= 16384)
    // the norm weights are never written by a kernel: fetch them before the wait
    uint2 wv[kMaxV];
#pragma unroll
    for (int k = 0; k < kMaxV; ++k) {
        const int n = 4 * ((int)threadIdx.x + k * kAddNormRowThreads);
        wv[k] = norm_w && n < H ? *reinterpret_cast<const uint2*>(norm_w + n) : make_uint2(0u, 0u);
    }
    // The dependent is the next skinny projection, which reads only weights
    // before its own wait: let it launch (and start its weight stream) now.
    griddep_launch_dependents();
    griddep_wait();
    trace_begin(tr);
    const int b = blockIdx.x;
    float4 hv[kMaxV];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxV; ++k) {
        const int n = 4 * ((int)threadIdx.x + k * kAddNormRowThreads);
        if (n < H) {
            float4 v = sk_sum4(a, B, b, n);
            float4* h = reinterpret_cast<float4*>(hidden + (int64_t)b * H + n);
            if (add) {
                const float4 o = *h;
                v.x = o.x + v.x; v.y = o.y + v.y; v.z = o.z + v.z; v.w = o.w + v.w;
            }
            *h = v;
            hv[k] = v;
            ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
        }
    }
    if (norm_w) {  // uniform over the grid
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {  // the 32 warp sums, as a fixed shuffle tree
            const float tot = warp_sum(red[threadIdx.x]);
            if (threadIdx.x == 0) s_rs = rsqrtf(tot / (float)H + eps);
        }
        __syncthreads();
        const float rs = s_rs;
#pragma unroll
        for (int k = 0; k < kMaxV; ++k) {
            const int n = 4 * ((int)threadIdx.x + k * kAddNormRowThreads);
            if (n < H) {
                const float4 v = hv[k];
                const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv[k].x));
                const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv[k].y));
                __half2 o0 = __floats2half2_rn(v.x * rs * w01.x, v.y * rs * w01.y);
                __half2 o1 = __floats2half2_rn(v.z * rs * w23.x, v.w * rs * w23.y);
                uint2 ov;
                ov.x = *reinterpret_cast<uint32_t*>(&o0);
                ov.y = *reinterpret_cast<uint32_t*>(&o1);
                *reinterpret_cast<uint2*>(xn + (int64_t)b * H + n) = ov;
            }
        }
    }
    trace_end(tr);
}

// act[b][i] = half(silu(gate) * up), silu(x) = x / (1 + exp(-x)) in fp32
__global__ void sk_swiglu_kernel(SkSlabs g, SkSlabs u, int B, int I, __half* __restrict__ act, TraceSlot tr) {
    griddep_launch_dependents();  // as sk_add_norm_kernel: the down projection follows
    griddep_wait();
    trace_begin(tr);
    const int64_t n = (int64_t)B * I / 4;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(4 * e / I), i = (int)(4 * e - (int64_t)b * I);
        const float4 x = sk_sum4(g, B, b, i), y = sk_sum4(u, B, b, i);
        __half2 o0 = __floats2half2_rn(x.x / (1.0f + expf(-x.x)) * y.x, x.y / (1.0f + expf(-x.y)) * y.y);
        __half2 o1 = __floats2half2_rn(x.z / (1.0f + expf(-x.z)) * y.z, x.w / (1.0f + expf(-x.w)) * y.w);
        uint2 ov;
        ov.x = *reinterpret_cast<uint32_t*>(&o0);
        ov.y = *reinterpret_cast<uint32_t*>(&o1);
        *reinterpret_cast<uint2*>(act + 4 * e) = ov;
    }
    trace_end(tr);
}

// logits[b][v] = lm_head projection (fp32) and the packed argmax of each row
// (ties to the lower id, ids >= limit excluded); argmax zeroed before.
// grid (chunks, B), 256 threads.
__global__ void sk_logits_argmax_kernel(SkSlabs a, int B, float* __restrict__ logits, int V, int row_offset,
                                        int limit, unsigned long long* __restrict__ argmax, TraceSlot tr) {
    __shared__ unsigned long long red[32];
    griddep_wait();
    griddep_launch_dependents();
    trace_begin(tr);
    const int b = blockIdx.y;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        const float x = sk_sum(a, B, b, i);
        logits[(int64_t)b * V + i] = x;
        const int gid = row_offset + i;
        if (gid < limit) {
            const unsigned long long k = argmax_key(x, (uint32_t)gid);
            best = k > best ? k : best;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, best, o);
        best = x > best ? x : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        if (best) atomicMax(argmax + b, best);
    }
    trace_end(tr);
}

// ---------------------------------------------------------------------------
// NCCL, resolved at run time.  Linking libnccl would pin whichever
// libnccl.so.2 the loader meets first for the whole process (and a host
// framework loaded later may need a newer one), so the library binds the few
// entry points it uses only when a tensor-parallel model is created: an NCCL
// already loaded in the process is preferred, then $B2_NCCL_LIB, then the
// default search path.
// ---------------------------------------------------------------------------
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    const char* (*GetLastError)(ncclComm_t) = nullptr;
    bool ok = false;
};

static NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, []() {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        const char* env = getenv("B2_NCCL_LIB");
        if (!h && env && env[0]) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.GetLastError = reinterpret_cast<decltype(api.GetLastError)>(dlsym(h, "ncclGetLastError"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.AllGather;
    });
    return api;
}

}  // namespace b2

using namespace b2;

// ---------------------------------------------------------------------------
// model object
// ---------------------------------------------------------------------------
// One quantised copy of a projection: E4M3 codes [rows][K] and a scale per
// row, or 4-bit codes [rows][K/2] and a scale per 128 weights (kI4Group).
struct Fp8W {
    uint8_t* q = nullptr;
    float* sc = nullptr;
};

struct LayerW {
    __half *wqkv = nullptr, *bqkv = nullptr, *wo = nullptr, *wg = nullptr, *wu = nullptr, *wd = nullptr;
    __half *ln1 = nullptr, *ln2 = nullptr;
    Fp8W f8qkv, f8o, f8g, f8u, f8d;  // b2_model_quantize_weights
    Fp8W i4qkv, i4o, i4g, i4u, i4d;  // its 4-bit form
};

struct b2_model {
    b2_model_config cfg{};
    int rank = 0, tp = 1, device = 0;
    int nq = 0, nkv = 0, inter = 0, vocab_l = 0, vocab_off = 0;  // per-rank sizes
    int qkv_rows = 0;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;

    std::vector<void*> allocs;
    __half* embed = nullptr;
    __half* lm_head = nullptr;  // local vocabulary shard
    Fp8W f8lm;                  // its quantised copy
    Fp8W i4lm;                  // its 4-bit copy
    bool wfp8 = false;          // decode GEMVs read the FP8 copies
    bool wint4 = false;         // decode GEMVs (batch 1-2) read the 4-bit copies
    __half* final_norm = nullptr;
    std::vector<LayerW> layers;

    __half* kv = nullptr;
    int64_t kv_s_layer = 0, kv_s_batch = 0, kv_s_kv = 0, kv_s_head = 0;
    // paged KV (b2_model_create_paged): pool [layer][K|V][block][slot][kv head][D]
    // and device block tables [max_batch][kv_maxb]
    int paged = 0, kv_blocks = 0, kv_bs = 0, kv_maxb = 0;
    int* block_tables = nullptr;
    int* h_bt = nullptr;  // pinned staging of the block tables
    // sampling inside the step (b2_model_set_sampling): configuration in
    // device memory, one LCG state per sequence
    int sampling = 0;
    b2_sampler_config* d_samp_cfg = nullptr;
    uint64_t* d_rng = nullptr;
    float2* rope = nullptr;

    float* hidden = nullptr;
    __half* q = nullptr;
    __half* attn = nullptr;
    __half* act = nullptr;
    float* logits = nullptr;
    float* logits_gather = nullptr;  // [tp][B][vocab_l] (tp > 1)
    float* part = nullptr;
    size_t part_floats = 0;
    unsigned long long* argmax = nullptr;
    int64_t* tokens = nullptr;
    int* positions = nullptr;
    int* seq_lens = nullptr;
    int64_t* hist = nullptr;
    int* hist_count = nullptr;
    int hist_cap = 0;

    // pinned staging
    int64_t* h_tokens = nullptr;
    int* h_pos = nullptr;
    unsigned long long* h_argmax = nullptr;
    float* h_logits = nullptr;

    // prefill workspace, grown on demand: rows of all prompt tokens
    int64_t pf_tokens = 0;
    float* pf_hidden = nullptr;  // [T, H] fp32 residual stream
    __half* pf_xn = nullptr;     // [T, H] normed activations
    __half* pf_qkv = nullptr;    // [T, qkv_rows]
    __half* pf_attn = nullptr;   // [T, nq * D]
    __half* pf_gate = nullptr;   // [T, inter] (SwiGLU output in place)
    __half* pf_up = nullptr;     // [T, inter]
    int64_t* pf_ids = nullptr;   // [T]
    float* pf_logits = nullptr;  // [rows, vocab] logits of every position (b2_model_forward_logits)
    int64_t pf_logits_rows = 0;

    // tensor-parallel exchange over peer memory (see TpExchange)
    void* p2p_base = nullptr;           // this rank's exchange region (IPC-exported)
    size_t p2p_bytes = 0;
    size_t off_recv = 0, off_am_recv = 0, off_am_flags = 0;
    std::vector<void*> peer_bases;      // opened IPC mappings (index = rank; own = p2p_base)
    float* hidden2 = nullptr;           // second residual-stream buffer
    int* step_ctr = nullptr;            // decode steps completed
    int* push_ctr = nullptr;            // arrival counter of pushing kernels
    bool p2p_on = false;
    TpExchange tpx{};
    // batched decode step (B > kGemvMaxBatch): split-K GEMM partial slabs and
    // the fused q|k|v rows / normed activations of the step
    float* bws_a = nullptr;
    float* bws_b = nullptr;
    size_t bws_floats = 0;
    __half* bqkv = nullptr;  // [max_batch, qkv_rows]
    __half* bxn = nullptr;   // [max_batch, H]

    unsigned long long* trace_buf = nullptr;  // step trace [slots][start, end]
    unsigned long long* trace_cur = nullptr;  // non-null while a traced step is enqueued
    int trace_next = 0;

    std::vector<cudaGraphExec_t> graphs;  // per batch size
    int splits = 1;
    int last_B = 0;  // batch of the most recent prefill / decode step
};

// Whether a decode step of B sequences runs the fused GEMVs: B within
// kGemvMaxBatch and within the batch tile every projection's width allows
// (the activation rows are staged in shared memory).  Otherwise the batched
// tensor-core step runs.
static bool gemv_step(const b2_model* m, int B) {
    if (B > kGemvMaxBatch) return false;
    const int Ks[3] = {m->cfg.hidden_size, m->nq * m->cfg.head_dim, m->inter};
    for (int K : Ks)
        if (B > gemv_batch_tile(K)) return false;
    return true;
}

static int model_alloc(b2_model* m, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes > 0 ? bytes : 16);
    if (e != cudaSuccess) return (int)e;
    m->allocs.push_back(*p);
    return B2_OK;
}

#define M_ALLOC(ptr, bytes)                                              \
    do {                                                                 \
        int rc_ = model_alloc(m, reinterpret_cast<void**>(&(ptr)), (bytes)); \
        if (rc_ != B2_OK) { b2_model_destroy(m); return rc_; }           \
    } while (0)

// Text of the last error a C-ABI call of this thread recorded (NCCL
// messages, for instance); empty when none.
static thread_local std::string g_last_error;
static void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

extern "C" const char* b2_last_error(void) { return g_last_error.c_str(); }

// the same record for the host-only parts of the library (tokenizer.cpp)
void b2_record_error(const char* msg) { set_last_error(msg); }

extern "C" int b2_nccl_unique_id(void* out128) {
    B2_REQUIRE(out128);
    ncclUniqueId id;
    if (!nccl().ok || nccl().GetUniqueId(&id) != ncclSuccess) return B2_ERR_NCCL;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    memcpy(out128, &id, sizeof(id));
    return B2_OK;
}

extern "C" int b2_model_destroy(b2_model* m) {
    if (!m) return B2_OK;
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto g : m->graphs)
        if (g) cudaGraphExecDestroy(g);
    m->graphs.clear();
    if (m->comm) nccl().CommDestroy(m->comm);
    for (size_t r = 0; r < m->peer_bases.size(); ++r)
        if (m->peer_bases[r] && m->peer_bases[r] != m->p2p_base) cudaIpcCloseMemHandle(m->peer_bases[r]);
    for (void* p : m->allocs) cudaFree(p);
    cudaFree(m->trace_buf);
    for (void* p : {(void*)m->pf_hidden, (void*)m->pf_xn, (void*)m->pf_qkv, (void*)m->pf_attn, (void*)m->pf_gate,
                    (void*)m->pf_up, (void*)m->pf_ids, (void*)m->pf_logits})
        cudaFree(p);
    cudaFreeHost(m->h_tokens);
    cudaFreeHost(m->h_pos);
    cudaFreeHost(m->h_argmax);
    cudaFreeHost(m->h_logits);
    cudaFreeHost(m->h_bt);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return B2_OK;
}

static int model_create(const b2_model_config* cfg, int tp_rank, int tp_size, const void* nccl_id, int num_blocks,
                        int block_size, b2_model** out);

extern "C" int b2_model_create(const b2_model_config* cfg, int tp_rank, int tp_size, const void* nccl_id,
                               b2_model** out) {
    return model_create(cfg, tp_rank, tp_size, nccl_id, 0, 0, out);
}

extern "C" int b2_model_create_paged(const b2_model_config* cfg, int num_blocks, int block_size, int tp_rank,
                                     int tp_size, const void* nccl_id, b2_model** out) {
    B2_REQUIRE(num_blocks >= 1 && block_size >= 1);
    return model_create(cfg, tp_rank, tp_size, nccl_id, num_blocks, block_size, out);
}

static int model_create(const b2_model_config* cfg, int tp_rank, int tp_size, const void* nccl_id, int num_blocks,
                        int block_size, b2_model** out) {
    B2_REQUIRE(cfg && out && tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size);
    *out = nullptr;
    const b2_model_config& c = *cfg;
    B2_REQUIRE(c.vocab_size > 0 && c.hidden_size > 0 && c.intermediate_size > 0 && c.num_layers > 0);
    B2_REQUIRE(c.num_q_heads > 0 && c.num_kv_heads > 0 && c.num_q_heads % c.num_kv_heads == 0);
    B2_REQUIRE(c.max_batch >= 1 && c.max_batch <= kMaxBatch && c.max_seq >= 1);
    if (c.num_kv_heads % tp_size || c.intermediate_size % tp_size || c.vocab_size % tp_size) return B2_ERR_UNSUPPORTED;
    if (!attn_head_dim_supported(c.head_dim) || c.hidden_size % 8 || (c.intermediate_size / tp_size) % 8 ||
        (c.num_q_heads / tp_size * c.head_dim) % 8)
        return B2_ERR_UNSUPPORTED;
    if (tp_size > 1 && !nccl_id) return B2_ERR_INVALID;
    // the paged cache is read by the tensor-core attention (head_dim 128), one
    // 128-position tile as whole blocks of whole 8-row swizzle atoms
    if (num_blocks > 0 && (c.head_dim != 128 || block_size < 8 || (block_size & 7) || 128 % block_size))
        return B2_ERR_UNSUPPORTED;

    b2_model* m = new (std::nothrow) b2_model();
    if (!m) return B2_ERR_INVALID;
    m->cfg = c;
    m->rank = tp_rank;
    m->tp = tp_size;
    cudaGetDevice(&m->device);
    const int H = c.hidden_size, D = c.head_dim, L = c.num_layers, B = c.max_batch;
    m->nq = c.num_q_heads / tp_size;
    m->nkv = c.num_kv_heads / tp_size;
    m->inter = c.intermediate_size / tp_size;
    m->vocab_l = c.vocab_size / tp_size;
    m->vocab_off = tp_rank * m->vocab_l;
    m->qkv_rows = (m->nq + 2 * m->nkv) * D;
    {
        cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    if (tp_size > 1) {
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        if (!nccl().ok) {
            set_last_error("NCCL could not be loaded (libnccl.so.2 / B2_NCCL_LIB)");
            b2_model_destroy(m);
            return B2_ERR_NCCL;
        }
        const ncclResult_t r = nccl().CommInitRank(&m->comm, tp_size, id, tp_rank);
        if (r != ncclSuccess) {
            std::string msg = "ncclCommInitRank: ";
            msg += nccl().GetErrorString ? nccl().GetErrorString(r) : "error";
            if (nccl().GetLastError) {
                msg += ": ";
                msg += nccl().GetLastError(nullptr);
            }
            set_last_error(msg.c_str());
            m->comm = nullptr;
            b2_model_destroy(m);
            return B2_ERR_NCCL;
        }
    }

    const size_t hs = sizeof(__half);
    M_ALLOC(m->embed, (size_t)c.vocab_size * H * hs);
    if (c.tie_word_embeddings) {
        m->lm_head = m->embed + (size_t)m->vocab_off * H;
    } else {
        M_ALLOC(m->lm_head, (size_t)m->vocab_l * H * hs);
    }
    M_ALLOC(m->final_norm, (size_t)H * hs);
    m->layers.resize(L);
    for (int l = 0; l < L; ++l) {
        LayerW& w = m->layers[l];
        M_ALLOC(w.wqkv, (size_t)m->qkv_rows * H * hs);
        if (c.has_qkv_bias) M_ALLOC(w.bqkv, (size_t)m->qkv_rows * hs);
        M_ALLOC(w.wo, (size_t)H * m->nq * D * hs);
        M_ALLOC(w.wg, (size_t)m->inter * H * hs);
        M_ALLOC(w.wu, (size_t)m->inter * H * hs);
        M_ALLOC(w.wd, (size_t)H * m->inter * hs);
        M_ALLOC(w.ln1, (size_t)H * hs);
        M_ALLOC(w.ln2, (size_t)H * hs);
    }
    if (num_blocks > 0) {
        // paged: pool [layer][K/V][block][slot][kv head][D], block tables
        // [max_batch][blocks per sequence at max_seq]
        m->paged = 1;
        m->kv_blocks = num_blocks;
        m->kv_bs = block_size;
        m->kv_maxb = (c.max_seq + block_size - 1) / block_size;
        m->kv_s_kv = (int64_t)num_blocks * block_size * m->nkv * D;
        m->kv_s_layer = 2 * m->kv_s_kv;
        M_ALLOC(m->block_tables, (size_t)B * m->kv_maxb * sizeof(int));
        cudaError_t e = cudaMemset(m->block_tables, 0, (size_t)B * m->kv_maxb * sizeof(int));
        if (e == cudaSuccess) e = cudaMallocHost(&m->h_bt, (size_t)B * m->kv_maxb * sizeof(int));
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    } else {
        // KV cache [layer][batch][K/V][kv head][max_seq][D]
        m->kv_s_head = (int64_t)c.max_seq * D;
        m->kv_s_kv = m->kv_s_head * m->nkv;
        m->kv_s_batch = m->kv_s_kv * 2;
        m->kv_s_layer = m->kv_s_batch * B;
    }
    M_ALLOC(m->kv, (size_t)m->kv_s_layer * L * hs);
    {
        cudaError_t e = cudaMemset(m->kv, 0, (size_t)m->kv_s_layer * L * hs);
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    // RoPE table with the reference CPU arithmetic (src/cpu/ops.cpp:174-189)
    {
        const int half = D / 2;
        std::vector<float> inv(half);
        for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(c.rope_theta, (float)(2 * i) / (float)D);
        std::vector<float2> tab((size_t)c.max_seq * half);
        for (int p = 0; p < c.max_seq; ++p)
            for (int i = 0; i < half; ++i) {
                const float a = (float)p * inv[i];
                tab[(size_t)p * half + i] = make_float2(cosf(a), sinf(a));
            }
        M_ALLOC(m->rope, tab.size() * sizeof(float2));
        cudaError_t e = cudaMemcpy(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    M_ALLOC(m->hidden, (size_t)B * H * sizeof(float));
    M_ALLOC(m->q, (size_t)B * m->nq * D * hs);
    M_ALLOC(m->attn, (size_t)B * m->nq * D * hs);
    M_ALLOC(m->act, (size_t)B * m->inter * hs);
    M_ALLOC(m->logits, (size_t)B * m->vocab_l * sizeof(float));
    if (tp_size > 1) M_ALLOC(m->logits_gather, (size_t)B * c.vocab_size * sizeof(float));
    m->splits = attn_pick_splits(B, m->nq, m->nkv, D, c.max_seq, (size_t)1 << 40);
    m->part_floats = attn_scratch_floats(B, m->nq, m->nkv, D, m->splits);
    M_ALLOC(m->part, m->part_floats * sizeof(float));
    {   // arrival counters start at zero; the attention kernel resets them after each use
        cudaError_t e = cudaMemset(m->part, 0, m->part_floats * sizeof(float));
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    M_ALLOC(m->argmax, (size_t)B * sizeof(unsigned long long));
    M_ALLOC(m->tokens, (size_t)B * sizeof(int64_t));
    M_ALLOC(m->positions, (size_t)B * sizeof(int));
    M_ALLOC(m->seq_lens, (size_t)B * sizeof(int));
    M_ALLOC(m->hidden2, (size_t)B * H * sizeof(float));
    if (!gemv_step(m, B)) {  // batched decode step: skinny partial slabs, q|k|v rows, normed rows
        if (H % 4 || H > 4 * 4 * kAddNormRowThreads || m->inter % 4 || D % 8) {
            b2_model_destroy(m);
            return B2_ERR_UNSUPPORTED;
        }
        const int qd = m->nq * D, I = m->inter;
        auto need = [&](int N, int K) {  // half (64-deep k blocks) or FP8 (128-deep) weights
            const SkinnyPlan p = skinny_plan(N, K, 64), q = skinny_plan(N, K, 128);
            return (size_t)std::max(p.max_slabs, q.max_slabs) * B * N;
        };
        size_t f = need(m->qkv_rows, H);
        f = std::max(f, need(H, qd));
        f = std::max(f, (I % 128) == 0 ? need(2 * I, H) : need(I, H));
        f = std::max(f, need(H, I));
        f = std::max(f, need(m->vocab_l, H));
        m->bws_floats = f;
        M_ALLOC(m->bws_a, m->bws_floats * sizeof(float));
        M_ALLOC(m->bws_b, m->bws_floats * sizeof(float));
        M_ALLOC(m->bqkv, (size_t)B * m->qkv_rows * hs);
        M_ALLOC(m->bxn, (size_t)B * H * hs);
    }
    M_ALLOC(m->step_ctr, 256);
    M_ALLOC(m->push_ctr, 256);
    if (tp_size > 1) {
        auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
        m->off_recv = 0;
        m->off_am_recv = up((size_t)2 * tp_size * B * H * sizeof(unsigned long long));
        m->off_am_flags = m->off_am_recv + up((size_t)tp_size * B * sizeof(unsigned long long));
        m->p2p_bytes = m->off_am_flags + up((size_t)tp_size * sizeof(unsigned));
        M_ALLOC(m->p2p_base, m->p2p_bytes);
        cudaError_t e = cudaMemset(m->p2p_base, 0, m->p2p_bytes);
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    {
        cudaError_t e = cudaMemset(m->step_ctr, 0, 256);
        if (e == cudaSuccess) e = cudaMemset(m->push_ctr, 0, 256);
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    M_ALLOC(m->d_samp_cfg, sizeof(b2_sampler_config));
    M_ALLOC(m->d_rng, (size_t)B * sizeof(uint64_t));
    m->hist_cap = 4096;
    M_ALLOC(m->hist, (size_t)m->hist_cap * B * sizeof(int64_t));
    M_ALLOC(m->hist_count, sizeof(int));
    {
        cudaError_t e = cudaMemset(m->tokens, 0, (size_t)B * sizeof(int64_t));
        if (e == cudaSuccess) e = cudaMemset(m->positions, 0, (size_t)B * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(m->hist_count, 0, sizeof(int));
        if (e == cudaSuccess) e = cudaMallocHost(&m->h_tokens, (size_t)B * sizeof(int64_t));
        if (e == cudaSuccess) e = cudaMallocHost(&m->h_pos, (size_t)B * sizeof(int));
        if (e == cudaSuccess) e = cudaMallocHost(&m->h_argmax, (size_t)B * sizeof(unsigned long long));
        if (e == cudaSuccess) e = cudaMallocHost(&m->h_logits, (size_t)B * c.vocab_size * sizeof(float));
        if (e != cudaSuccess) { b2_model_destroy(m); return (int)e; }
    }
    m->graphs.assign(B + 1, nullptr);
    *out = m;
    return B2_OK;
}

// ---------------------------------------------------------------------------
// tensor-parallel exchange over peer memory
// ---------------------------------------------------------------------------
static void invalidate_graphs(b2_model* m) {
    for (auto& g : m->graphs)
        if (g) {
            cudaGraphExecDestroy(g);
            g = nullptr;
        }
}

extern "C" int b2_model_p2p_handle(b2_model* m, void* out64) {
    B2_REQUIRE(m && out64);
    if (m->tp < 2 || !m->p2p_base) return B2_ERR_STATE;
    cudaIpcMemHandle_t h;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    B2_TRY(cudaIpcGetMemHandle(&h, m->p2p_base));
    memcpy(out64, &h, sizeof(h));
    return B2_OK;
}

extern "C" int b2_model_p2p_open(b2_model* m, const void* handles) {
    B2_REQUIRE(m && handles);
    if (m->tp < 2 || !m->p2p_base || m->tp > kMaxTp) return B2_ERR_STATE;
    if (m->p2p_on) return B2_OK;
    B2_TRY(cudaStreamSynchronize(m->stream));
    std::vector<void*> bases(m->tp, nullptr);
    for (int r = 0; r < m->tp; ++r) {
        if (r == m->rank) {
            bases[r] = m->p2p_base;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + 64 * (size_t)r, sizeof(h));
        const cudaError_t e = cudaIpcOpenMemHandle(&bases[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (bases[q] && q != m->rank) cudaIpcCloseMemHandle(bases[q]);
            set_last_error("cudaIpcOpenMemHandle failed for a peer's exchange buffer");
            return (int)e;
        }
    }
    m->peer_bases = bases;
    TpExchange& x = m->tpx;
    x = TpExchange{};
    x.tp = m->tp;
    x.rank = m->rank;
    x.Bmax = m->cfg.max_batch;
    x.H = m->cfg.hidden_size;
    char* own = static_cast<char*>(m->p2p_base);
    x.recv = reinterpret_cast<unsigned long long*>(own + m->off_recv);
    x.am_recv = reinterpret_cast<unsigned long long*>(own + m->off_am_recv);
    x.am_flags = reinterpret_cast<unsigned*>(own + m->off_am_flags);
    for (int r = 0; r < m->tp; ++r) {
        char* pb = static_cast<char*>(bases[r]);
        x.peer_recv[r] = reinterpret_cast<unsigned long long*>(pb + m->off_recv);
        x.peer_am_recv[r] = reinterpret_cast<unsigned long long*>(pb + m->off_am_recv);
        x.peer_am_flags[r] = reinterpret_cast<unsigned*>(pb + m->off_am_flags);
    }
    x.step = m->step_ctr;
    x.ctr = m->push_ctr;
    x.err = wait_error_word();
    if (!x.err) return B2_ERR_STATE;
    m->p2p_on = true;
    invalidate_graphs(m);  // recapture the step with the exchange in place of NCCL
    return B2_OK;
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------
static int init_block(b2_model* m, __half* dst, int64_t rows, int64_t cols, uint64_t seed, uint64_t tid, int64_t row0,
                      int64_t col0, int64_t ld, float scale) {
    if (rows <= 0 || cols <= 0) return B2_OK;
    const int64_t n = rows * cols;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)sm_count() * 32) blocks = (int64_t)sm_count() * 32;
    init_tensor_kernel<<<(unsigned)blocks, 256, 0, m->stream>>>(dst, rows, cols, seed, tid, row0, col0, ld, scale);
    B2_CHECK_LAUNCH();
    return B2_OK;
}

static int fill_block(b2_model* m, __half* dst, int64_t n, float v) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    fill_half_kernel<<<(unsigned)blocks, 256, 0, m->stream>>>(dst, n, v);
    B2_CHECK_LAUNCH();
    return B2_OK;
}

enum : uint64_t { T_EMBED = 1, T_LM_HEAD = 2, T_FINAL_NORM = 3 };
static uint64_t layer_tid(int l, int k) { return 16 + 16 * (uint64_t)l + (uint64_t)k; }
enum { K_WQ = 0, K_WK = 1, K_WV = 2, K_WO = 3, K_WG = 4, K_WU = 5, K_WD = 6, K_LN1 = 7, K_LN2 = 8, K_BQ = 9,
       K_BK = 10, K_BV = 11 };

#define M_TRY(expr)                       \
    do {                                  \
        int rc_ = (expr);                 \
        if (rc_ != B2_OK) return rc_;     \
    } while (0)

extern "C" int b2_model_init_random(b2_model* m, uint64_t seed, float stddev) {
    B2_REQUIRE(m);
    const b2_model_config& c = m->cfg;
    const int64_t H = c.hidden_size, D = c.head_dim;
    const double var1 = (65536.0 * 65536.0 - 1.0) / 12.0;
    const float scale = (float)((double)stddev / sqrt(4.0 * var1));
    M_TRY(init_block(m, m->embed, c.vocab_size, H, seed, T_EMBED, 0, 0, H, scale));
    if (!c.tie_word_embeddings) M_TRY(init_block(m, m->lm_head, m->vocab_l, H, seed, T_LM_HEAD, m->vocab_off, 0, H, scale));
    M_TRY(fill_block(m, m->final_norm, H, 1.0f));
    const int64_t qd = (int64_t)m->nq * D, kvd = (int64_t)m->nkv * D;
    const int64_t qd_g = (int64_t)c.num_q_heads * D, kvd_g = (int64_t)c.num_kv_heads * D;
    for (int l = 0; l < c.num_layers; ++l) {
        LayerW& w = m->layers[l];
        M_TRY(init_block(m, w.wqkv, qd, H, seed, layer_tid(l, K_WQ), m->rank * qd, 0, H, scale));
        M_TRY(init_block(m, w.wqkv + qd * H, kvd, H, seed, layer_tid(l, K_WK), m->rank * kvd, 0, H, scale));
        M_TRY(init_block(m, w.wqkv + (qd + kvd) * H, kvd, H, seed, layer_tid(l, K_WV), m->rank * kvd, 0, H, scale));
        if (w.bqkv) {
            M_TRY(init_block(m, w.bqkv, 1, qd, seed, layer_tid(l, K_BQ), 0, m->rank * qd, qd_g, scale));
            M_TRY(init_block(m, w.bqkv + qd, 1, kvd, seed, layer_tid(l, K_BK), 0, m->rank * kvd, kvd_g, scale));
            M_TRY(init_block(m, w.bqkv + qd + kvd, 1, kvd, seed, layer_tid(l, K_BV), 0, m->rank * kvd, kvd_g, scale));
        }
        M_TRY(init_block(m, w.wo, H, qd, seed, layer_tid(l, K_WO), 0, m->rank * qd, qd_g, scale));
        M_TRY(init_block(m, w.wg, m->inter, H, seed, layer_tid(l, K_WG), (int64_t)m->rank * m->inter, 0, H, scale));
        M_TRY(init_block(m, w.wu, m->inter, H, seed, layer_tid(l, K_WU), (int64_t)m->rank * m->inter, 0, H, scale));
        M_TRY(init_block(m, w.wd, H, m->inter, seed, layer_tid(l, K_WD), 0, (int64_t)m->rank * m->inter,
                         c.intermediate_size, scale));
        M_TRY(fill_block(m, w.ln1, H, 1.0f));
        M_TRY(fill_block(m, w.ln2, H, 1.0f));
    }
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

static int convert_block(b2_model* m, __half* dst, int64_t rows, int64_t cols);

// Copy the [rows, cols] sub-block at (row0, col0) of a host [*, ld] fp16 tensor
// (bf16: converted to fp16 on the device after the copy).
static int upload_block(b2_model* m, __half* dst, const uint16_t* src, int64_t rows, int64_t cols, int64_t row0,
                        int64_t col0, int64_t ld, bool bf16 = false) {
    B2_TRY(cudaMemcpy2DAsync(dst, cols * 2, src + row0 * ld + col0, ld * 2, cols * 2, rows, cudaMemcpyHostToDevice,
                             m->stream));
    if (bf16) return convert_block(m, dst, rows, cols);
    return B2_OK;
}

// Convert the [rows, cols] block just uploaded at dst from bf16 to fp16.
static int convert_block(b2_model* m, __half* dst, int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    if (n <= 0) return B2_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
    bf16_to_f16_kernel<<<(unsigned)blocks, 256, 0, m->stream>>>(reinterpret_cast<uint16_t*>(dst), n);
    B2_CHECK_LAUNCH();
    return B2_OK;
}

static int set_tensor(b2_model* m, const char* name, const uint16_t* src, int64_t rows, int64_t cols, bool bf16);

extern "C" int b2_model_set_tensor(b2_model* m, const char* name, const uint16_t* src, int64_t rows, int64_t cols) {
    return set_tensor(m, name, src, rows, cols, false);
}

extern "C" int b2_model_set_tensor_bf16(b2_model* m, const char* name, const uint16_t* src, int64_t rows,
                                        int64_t cols) {
    return set_tensor(m, name, src, rows, cols, true);
}

// Upload (and for bf16 sources convert on the device) this rank's block of a
// global tensor.
static int set_tensor(b2_model* m, const char* name, const uint16_t* src, int64_t rows, int64_t cols, bool bf16) {
    B2_REQUIRE(m && name && src);
    const b2_model_config& c = m->cfg;
    const int64_t H = c.hidden_size, D = c.head_dim;
    const int64_t qd = (int64_t)m->nq * D, kvd = (int64_t)m->nkv * D;
    std::string n(name);
    int rc = B2_ERR_INVALID;
    auto shape = [&](int64_t r, int64_t cc) { return rows == r && cols == cc; };
    if (n == "embed" && shape(c.vocab_size, H)) {
        rc = upload_block(m, m->embed, src, c.vocab_size, H, 0, 0, H, bf16);
    } else if (n == "lm_head" && shape(c.vocab_size, H) && !c.tie_word_embeddings) {
        rc = upload_block(m, m->lm_head, src, m->vocab_l, H, m->vocab_off, 0, H, bf16);
    } else if (n == "final_norm" && rows * cols == H) {
        rc = upload_block(m, m->final_norm, src, 1, H, 0, 0, H, bf16);
    } else {
        const size_t dot = n.find('.');
        if (dot == std::string::npos) return B2_ERR_INVALID;
        const int l = atoi(n.substr(0, dot).c_str());
        const std::string t = n.substr(dot + 1);
        if (l < 0 || l >= c.num_layers) return B2_ERR_INVALID;
        LayerW& w = m->layers[l];
        const int64_t I = c.intermediate_size;
        if (t == "ln1" && rows * cols == H) rc = upload_block(m, w.ln1, src, 1, H, 0, 0, H, bf16);
        else if (t == "ln2" && rows * cols == H) rc = upload_block(m, w.ln2, src, 1, H, 0, 0, H, bf16);
        else if (t == "wq" && shape((int64_t)c.num_q_heads * D, H)) rc = upload_block(m, w.wqkv, src, qd, H, m->rank * qd, 0, H, bf16);
        else if (t == "wk" && shape((int64_t)c.num_kv_heads * D, H))
            rc = upload_block(m, w.wqkv + qd * H, src, kvd, H, m->rank * kvd, 0, H, bf16);
        else if (t == "wv" && shape((int64_t)c.num_kv_heads * D, H))
            rc = upload_block(m, w.wqkv + (qd + kvd) * H, src, kvd, H, m->rank * kvd, 0, H, bf16);
        else if (t == "bq" && w.bqkv && rows * cols == (int64_t)c.num_q_heads * D)
            rc = upload_block(m, w.bqkv, src, 1, qd, 0, m->rank * qd, rows * cols, bf16);
        else if (t == "bk" && w.bqkv && rows * cols == (int64_t)c.num_kv_heads * D)
            rc = upload_block(m, w.bqkv + qd, src, 1, kvd, 0, m->rank * kvd, rows * cols, bf16);
        else if (t == "bv" && w.bqkv && rows * cols == (int64_t)c.num_kv_heads * D)
            rc = upload_block(m, w.bqkv + qd + kvd, src, 1, kvd, 0, m->rank * kvd, rows * cols, bf16);
        else if (t == "wo" && shape(H, (int64_t)c.num_q_heads * D))
            rc = upload_block(m, w.wo, src, H, qd, 0, m->rank * qd, (int64_t)c.num_q_heads * D, bf16);
        else if (t == "wg" && shape(I, H)) rc = upload_block(m, w.wg, src, m->inter, H, (int64_t)m->rank * m->inter, 0, H, bf16);
        else if (t == "wu" && shape(I, H)) rc = upload_block(m, w.wu, src, m->inter, H, (int64_t)m->rank * m->inter, 0, H, bf16);
        else if (t == "wd" && shape(H, I)) rc = upload_block(m, w.wd, src, H, m->inter, 0, (int64_t)m->rank * m->inter, I, bf16);
    }
    if (rc != B2_OK) return rc;
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

// ---------------------------------------------------------------------------
// the decode step
// ---------------------------------------------------------------------------
static int nccl_sum_hidden(b2_model* m, int B) {
    if (m->tp == 1) return B2_OK;
    if (nccl().AllReduce(m->hidden, m->hidden, (size_t)B * m->cfg.hidden_size, ncclFloat, ncclSum, m->comm, m->stream) !=
        ncclSuccess)
        return B2_ERR_NCCL;
    return B2_OK;
}

// With the peer exchange on (xch), the step keeps its residual stream in two
// buffers: exchange 2l (after o of layer l) is consumed by that layer's
// gate/up GEMV, hidden -> hidden2; exchange 2l+1 (after down) by the next
// layer's q|k|v GEMV or the lm_head, hidden2 -> hidden.
// Launch slot of the next kernel of a traced step (tracing off: buf null).
static TraceSlot next_trace(b2_model* m) {
    TraceSlot t = {m->trace_cur, 0};
    if (m->trace_cur) t.slot = m->trace_next++;
    return t;
}

static void set_exchange(b2_model* m, GemvParams& p, int slot, const float* hin, float* hout) {
    p.tp_on = 1;
    p.tpx = m->tpx;
    p.slot = slot;
    p.nslots = 2 * m->cfg.num_layers;
    p.hid_in = hin;
    p.hid_out = hout;
}

// Layer l's K / V rows: the contiguous cache or the paged pool.
static KvLayout layer_kv(const b2_model* m, int l) {
    KvLayout k = {};
    k.k = m->kv + (int64_t)l * m->kv_s_layer;
    k.v = k.k + m->kv_s_kv;
    if (m->paged) {
        k.bt = m->block_tables;
        k.maxb = m->kv_maxb;
        k.bs = m->kv_bs;
        k.nkv = m->nkv;
    } else {
        k.sb = m->kv_s_batch;
        k.sh = m->kv_s_head;
    }
    return k;
}

static int launch_qkv(b2_model* m, int l, int B, bool pdl, bool xch = false) {
    const b2_model_config& c = m->cfg;
    LayerW& w = m->layers[l];
    GemvParams p = {};
    p.trace = next_trace(m);
    p.W = w.wqkv;
    p.K = c.hidden_size;
    p.tasks = m->qkv_rows / 2;
    p.B = B;
    p.x = m->hidden;
    p.ldx = c.hidden_size;
    p.norm_w = w.ln1;
    p.eps = c.rms_norm_eps;
    p.bias = w.bqkv;
    p.y = m->q;
    p.ldy = (int64_t)m->nq * c.head_dim;
    p.nq = m->nq;
    p.nkv = m->nkv;
    p.D = c.head_dim;
    p.rope = m->rope;
    p.pos = m->positions;
    p.kv = layer_kv(m, l);
    if (m->wfp8 && B <= kFp8MaxBatch) {
        p.W8 = w.f8qkv.q;
        p.wsc = w.f8qkv.sc;
    } else if (m->wint4 && B <= kI4MaxBatch) {
        p.W8 = w.i4qkv.q;
        p.wsc = w.i4qkv.sc;
        p.w4 = 1;
    }
    if (xch && l > 0) {
        set_exchange(m, p, 2 * (l - 1) + 1, m->hidden2, m->hidden);
        p.x = m->hidden2;
        return gemv_launch(p, X_SUM, OUT_QKV, m->stream, pdl);
    }
    return gemv_launch(p, X_NORM, OUT_QKV, m->stream, pdl);
}

// Decode attention of layer l over the paged pool (q rows q_sb apart).
static int launch_attn_paged(b2_model* m, int l, const __half* q, int64_t q_sb, int B, int lean, TraceSlot tr) {
    const KvLayout kv = layer_kv(m, l);
    const int D = m->cfg.head_dim, qd = m->nq * D;
    return attn_tc_launch_paged(q, q_sb, m->attn, qd, kv.k, kv.v, m->kv_blocks, m->kv_bs, m->block_tables, m->kv_maxb,
                                m->cfg.max_seq, m->seq_lens, B, m->nq, m->nkv, D, 1, lean, tr, m->stream, true);
}

static int launch_attn(b2_model* m, int l, int B, bool pdl) {
    (void)pdl;  // the step form always uses programmatic launch
    const int D = m->cfg.head_dim;
    __half* kbase = m->kv + (int64_t)l * m->kv_s_layer;
    const TraceSlot tr = next_trace(m);
    const int qd = m->nq * D;
    if (m->paged) return launch_attn_paged(m, l, m->q, qd, B, 1, tr);
    const int rc = attn_cl_launch(m->q, qd, m->attn, qd, kbase, kbase + m->kv_s_kv, m->kv_s_batch, m->kv_s_head, D,
                                  m->cfg.max_seq, m->seq_lens, 0, B, m->nq, m->nkv, D, 1, 1, tr, m->stream, true);
    if (rc != B2_ERR_UNSUPPORTED) return rc;
    return attn_decode_launch_step(m->q, kbase, kbase + m->kv_s_kv, m->kv_s_batch, m->kv_s_head, D, m->seq_lens,
                                   m->attn, m->part, m->splits, B, m->nq, m->nkv, D, m->stream, tr);
}

static int launch_o(b2_model* m, int l, int B, bool pdl, bool xch = false) {
    const b2_model_config& c = m->cfg;
    GemvParams p = {};
    p.trace = next_trace(m);
    p.W = m->layers[l].wo;
    if (m->wfp8 && B <= kFp8MaxBatch) {
        p.W8 = m->layers[l].f8o.q;
        p.wsc = m->layers[l].f8o.sc;
    } else if (m->wint4 && B <= kI4MaxBatch) {
        p.W8 = m->layers[l].i4o.q;
        p.wsc = m->layers[l].i4o.sc;
        p.w4 = 1;
    }
    p.K = m->nq * c.head_dim;
    p.tasks = c.hidden_size;
    p.B = B;
    p.x = m->attn;
    p.ldx = (int64_t)m->nq * c.head_dim;
    p.resid_add = m->rank == 0 ? 1 : 0;
    p.y = m->hidden;
    p.ldy = c.hidden_size;
    if (xch) {
        set_exchange(m, p, 2 * l, nullptr, nullptr);
        return gemv_launch(p, X_HALF, OUT_PUSH, m->stream, pdl);
    }
    return gemv_launch(p, X_HALF, OUT_RESID, m->stream, pdl);
}

static int launch_gateup(b2_model* m, int l, int B, bool pdl, bool xch = false) {
    const b2_model_config& c = m->cfg;
    LayerW& w = m->layers[l];
    GemvParams p = {};
    p.trace = next_trace(m);
    p.W = w.wg;
    p.W2 = w.wu;
    if (m->wfp8 && B <= kFp8MaxBatch) {
        p.W8 = w.f8g.q;
        p.W8b = w.f8u.q;
        p.wsc = w.f8g.sc;
        p.wsc2 = w.f8u.sc;
    } else if (m->wint4 && B <= kI4MaxBatch) {
        p.W8 = w.i4g.q;
        p.W8b = w.i4u.q;
        p.wsc = w.i4g.sc;
        p.wsc2 = w.i4u.sc;
        p.w4 = 1;
    }
    p.K = c.hidden_size;
    p.tasks = m->inter;
    p.B = B;
    p.x = m->hidden;
    p.ldx = c.hidden_size;
    p.norm_w = w.ln2;
    p.eps = c.rms_norm_eps;
    p.y = m->act;
    p.ldy = m->inter;
    if (xch) {
        set_exchange(m, p, 2 * l, m->hidden, m->hidden2);
        return gemv_launch(p, X_SUM, OUT_SWIGLU, m->stream, pdl);
    }
    return gemv_launch(p, X_NORM, OUT_SWIGLU, m->stream, pdl);
}

static int launch_down(b2_model* m, int l, int B, bool pdl, bool xch = false) {
    const b2_model_config& c = m->cfg;
    GemvParams p = {};
    p.trace = next_trace(m);
    p.W = m->layers[l].wd;
    if (m->wfp8 && B <= kFp8MaxBatch) {
        p.W8 = m->layers[l].f8d.q;
        p.wsc = m->layers[l].f8d.sc;
    } else if (m->wint4 && B <= kI4MaxBatch) {
        p.W8 = m->layers[l].i4d.q;
        p.wsc = m->layers[l].i4d.sc;
        p.w4 = 1;
    }
    p.K = m->inter;
    p.tasks = c.hidden_size;
    p.B = B;
    p.x = m->act;
    p.ldx = m->inter;
    p.resid_add = m->rank == 0 ? 1 : 0;
    p.y = m->hidden;
    p.ldy = c.hidden_size;
    if (xch) {
        set_exchange(m, p, 2 * l + 1, nullptr, nullptr);
        return gemv_launch(p, X_HALF, OUT_PUSH, m->stream, pdl);
    }
    return gemv_launch(p, X_HALF, OUT_RESID, m->stream, pdl);
}

static int launch_lm_head(b2_model* m, int B, bool pdl, bool xch = false) {
    const b2_model_config& c = m->cfg;
    GemvParams p = {};
    p.trace = next_trace(m);
    p.W = m->lm_head;
    if (m->wfp8 && B <= kFp8MaxBatch) {
        p.W8 = m->f8lm.q;
        p.wsc = m->f8lm.sc;
    } else if (m->wint4 && B <= kI4MaxBatch) {
        p.W8 = m->i4lm.q;
        p.wsc = m->i4lm.sc;
        p.w4 = 1;
    }
    p.K = c.hidden_size;
    p.tasks = m->vocab_l;
    p.B = B;
    p.x = m->hidden;
    p.ldx = c.hidden_size;
    p.norm_w = m->final_norm;
    p.eps = c.rms_norm_eps;
    p.y = m->logits;
    p.ldy = m->vocab_l;
    p.argmax = m->argmax;
    p.row_offset = m->vocab_off;
    p.argmax_limit = c.vocab_size > 151665 ? 151665 : c.vocab_size;
    if (xch) {
        set_exchange(m, p, 2 * c.num_layers - 1, m->hidden2, m->hidden);
        p.x = m->hidden2;
        return gemv_launch(p, X_SUM, OUT_LOGITS, m->stream, pdl);
    }
    return gemv_launch(p, X_NORM, OUT_LOGITS, m->stream, pdl);
}


// Decode step for B > kGemvMaxBatch sequences: every projection is a
// tensor-core GEMM with M = B (weights streamed once for the whole batch),
// split along K so the grid covers the SMs; the partial slabs are reduced in
// order by kernels fused with bias, RoPE + KV append, SwiGLU or the residual
// add.  Attention, step begin / end are those of the GEMV step.
// Skinny projection X W^T of B rows into `ws`, and the slab descriptor its
// consumer kernel reads.
// f0 / f1: the FP8 copies of W0 / W1 (b2_model_quantize_weights), streamed
// instead of the half weights when set.
static int sk_proj(b2_model* m, const __half* X, int B, const __half* W0, int N0, const __half* W1, int N1, int K,
                   float* ws, SkSlabs* out, const Fp8W* f0 = nullptr, const Fp8W* f1 = nullptr) {
    SkinnyPlan pl;
    if (m->wfp8 && f0 && f0->q && B <= 128)
        M_TRY(gemm_skinny_f8(X, B, f0->q, f0->sc, N0, f1 ? f1->q : nullptr, f1 ? f1->sc : nullptr, N1, K, ws,
                             m->bws_floats, &pl, m->stream, next_trace(m)));
    else
        M_TRY(gemm_skinny(X, B, W0, N0, W1, N1, K, ws, m->bws_floats, &pl, m->stream, next_trace(m)));
    out->ws = ws;
    out->N = N0 + N1;
    out->nk = pl.nk;
    out->per = pl.per;
    out->col0 = 0;
    return B2_OK;
}

// lm_head of the normalised rows m->bxn (skinny projection), logits and the
// packed argmax of each row; argmax must be zero before.
static int lm_head_rows(b2_model* m, int B) {
    const b2_model_config& c = m->cfg;
    SkSlabs lg;
    M_TRY(sk_proj(m, m->bxn, B, m->lm_head, m->vocab_l, nullptr, 0, c.hidden_size, m->bws_a, &lg, &m->f8lm));
    const int limit = c.vocab_size > 151665 ? 151665 : c.vocab_size;
    const unsigned chunks = (unsigned)((m->vocab_l + 4095) / 4096);
    B2_TRY(launch(sk_logits_argmax_kernel, dim3(chunks, (unsigned)B), dim3(256), 0, m->stream, true, lg, B,
                  m->logits, m->vocab_l, m->vocab_off, limit, m->argmax, next_trace(m)));
    return B2_OK;
}

// one thread per sequence for the step / prefill end kernels
static unsigned end_threads(int B) { return (unsigned)(((B + 31) / 32) * 32); }

// hidden += projection (rank 0 adds the residual), then the next RMSNorm
// into m->bxn: fused when there is no all-reduce in between.
static int add_and_norm(b2_model* m, const SkSlabs& a, int B, const __half* norm_w) {
    const b2_model_config& c = m->cfg;
    const int H = c.hidden_size;
    const int add = m->rank == 0 ? 1 : 0;
    if (m->tp == 1) {
        B2_TRY(launch(sk_add_norm_kernel, dim3((unsigned)B), dim3(kAddNormRowThreads), 0, m->stream, true, a, B,
                      m->hidden, add, H, norm_w, m->bxn, c.rms_norm_eps, next_trace(m)));
        return B2_OK;
    }
    B2_TRY(launch(sk_add_norm_kernel, dim3((unsigned)B), dim3(kAddNormRowThreads), 0, m->stream, true, a, B,
                  m->hidden, add, H, (const __half*)nullptr, (__half*)nullptr, c.rms_norm_eps, next_trace(m)));
    M_TRY(nccl_sum_hidden(m, B));
    rmsnorm_rows_kernel<<<B, 256, 0, m->stream>>>(m->hidden, norm_w, m->bxn, H, c.rms_norm_eps);
    B2_CHECK_LAUNCH();
    return B2_OK;
}

// Decode step for batches the GEMV step does not take (B > kGemvMaxBatch, or
// a weight width that caps the GEMV batch tile below B): every projection is
// a skinny tensor-core weight stream (skinny.cu) whose partial slabs are
// summed by the kernel of the operation that follows it -- q|k|v + RoPE + KV
// append, residual add + next RMSNorm, SwiGLU, logits + argmax.  Attention,
// step begin / end are those of the GEMV step.
static int enqueue_step_batched(b2_model* m, int B) {
    const b2_model_config& c = m->cfg;
    cudaStream_t s = m->stream;
    const int H = c.hidden_size, D = c.head_dim, I = m->inter, qd = m->nq * D, R = m->qkv_rows;
    const bool fuse_gu = (I % 128) == 0;
    B2_TRY(launch(step_begin_kernel, dim3(B), dim3(256), 0, s, true, (const int64_t*)m->tokens,
                  (const int*)m->positions, (const __half*)m->embed, m->hidden, H, m->seq_lens, m->argmax, m->hist,
                  (const int*)m->hist_count, m->hist_cap, next_trace(m)));
    rmsnorm_rows_kernel<<<B, 256, 0, s>>>(m->hidden, m->layers[0].ln1, m->bxn, H, c.rms_norm_eps);
    B2_CHECK_LAUNCH();
    for (int l = 0; l < c.num_layers; ++l) {
        LayerW& w = m->layers[l];
        __half* kbase = m->kv + (int64_t)l * m->kv_s_layer;
        SkSlabs qkv, o, g, u, d;
        M_TRY(sk_proj(m, m->bxn, B, w.wqkv, R, nullptr, 0, H, m->bws_a, &qkv, &w.f8qkv));
        const unsigned qkv_threads = (unsigned)((m->nq + 2 * m->nkv) * (D / 8));
        B2_TRY(launch(sk_qkv_rope_kernel, dim3((unsigned)B, (qkv_threads + 255) / 256), dim3(256), 0, s, true,
                      qkv, B, (const __half*)w.bqkv, m->bqkv, (int64_t)R, (const float2*)m->rope, m->nq, m->nkv, D,
                      layer_kv(m, l), (const int*)m->positions, next_trace(m)));
        const TraceSlot tr_attn = next_trace(m);
        if (m->paged) {
            M_TRY(launch_attn_paged(m, l, m->bqkv, R, B, 0, tr_attn));
        } else {
            const int rc = attn_cl_launch(m->bqkv, R, m->attn, qd, kbase, kbase + m->kv_s_kv, m->kv_s_batch,
                                          m->kv_s_head, D, c.max_seq, m->seq_lens, 0, B, m->nq, m->nkv, D, 1, 0,
                                          tr_attn, s, true);
            if (rc == B2_ERR_UNSUPPORTED)
                M_TRY(attn_decode_launch_step_q(m->bqkv, R, kbase, kbase + m->kv_s_kv, m->kv_s_batch, m->kv_s_head, D,
                                                m->seq_lens, m->attn, m->part, m->splits, B, m->nq, m->nkv, D, s));
            else
                M_TRY(rc);
        }
        const __half* next_ln = l + 1 < c.num_layers ? m->layers[l + 1].ln1 : m->final_norm;
        M_TRY(sk_proj(m, m->attn, B, w.wo, H, nullptr, 0, qd, m->bws_a, &o, &w.f8o));
        M_TRY(add_and_norm(m, o, B, w.ln2));
        if (fuse_gu) {
            M_TRY(sk_proj(m, m->bxn, B, w.wg, I, w.wu, I, H, m->bws_a, &g, &w.f8g, &w.f8u));
            u = g;
            u.col0 = I;
        } else {
            M_TRY(sk_proj(m, m->bxn, B, w.wg, I, nullptr, 0, H, m->bws_a, &g, &w.f8g));
            M_TRY(sk_proj(m, m->bxn, B, w.wu, I, nullptr, 0, H, m->bws_b, &u, &w.f8u));
        }
        {
            int64_t blocks = ((int64_t)B * I / 4 + 255) / 256;
            if (blocks > (int64_t)sm_count() * 8) blocks = (int64_t)sm_count() * 8;
            B2_TRY(launch(sk_swiglu_kernel, dim3((unsigned)blocks), dim3(256), 0, s, true, g, u, B, I, m->act,
                          next_trace(m)));
        }
        M_TRY(sk_proj(m, m->act, B, w.wd, H, nullptr, 0, I, m->bws_a, &d, &w.f8d));
        M_TRY(add_and_norm(m, d, B, next_ln));
    }
    M_TRY(lm_head_rows(m, B));
    if (m->sampling)
        M_TRY(step_sample_launch(m->logits, m->vocab_l, m->vocab_l, B, m->d_samp_cfg, m->d_rng, m->argmax, s));
    if (m->tp > 1) {
        if (nccl().AllReduce(m->argmax, m->argmax, (size_t)B, ncclUint64, ncclMax, m->comm, s) != ncclSuccess)
            return B2_ERR_NCCL;
    }
    B2_TRY(launch(step_end_kernel, dim3(1), dim3(end_threads(B)), 0, s, true, (const unsigned long long*)m->argmax,
                  m->tokens, m->positions, B, m->hist_count, m->hist_cap, 0, (const unsigned long long*)nullptr,
                  (const unsigned*)nullptr, m->tp, c.max_batch, m->step_ctr, (int*)nullptr, next_trace(m)));
    return B2_OK;
}

// Issue every launch of one decode step for B sequences on m->stream.
static int enqueue_step(b2_model* m, int B) {
    if (!gemv_step(m, B)) return enqueue_step_batched(m, B);
    const b2_model_config& c = m->cfg;
    cudaStream_t s = m->stream;
    const bool pdl = true;
    const bool xch = m->p2p_on;
    B2_TRY(launch(step_begin_kernel, dim3(B), dim3(256), 0, s, pdl, (const int64_t*)m->tokens,
                  (const int*)m->positions, (const __half*)m->embed, m->hidden, c.hidden_size, m->seq_lens, m->argmax,
                  m->hist, (const int*)m->hist_count, m->hist_cap, next_trace(m)));
    for (int l = 0; l < c.num_layers; ++l) {
        M_TRY(launch_qkv(m, l, B, pdl, xch));
        M_TRY(launch_attn(m, l, B, pdl));
        M_TRY(launch_o(m, l, B, pdl, xch));
        if (!xch) M_TRY(nccl_sum_hidden(m, B));
        M_TRY(launch_gateup(m, l, B, pdl, xch));
        M_TRY(launch_down(m, l, B, pdl, xch));
        if (!xch) M_TRY(nccl_sum_hidden(m, B));
    }
    M_TRY(launch_lm_head(m, B, pdl, xch));
    if (m->sampling)
        M_TRY(step_sample_launch(m->logits, m->vocab_l, m->vocab_l, B, m->d_samp_cfg, m->d_rng, m->argmax, s));
    if (m->tp > 1 && !xch) {
        if (nccl().AllReduce(m->argmax, m->argmax, (size_t)B, ncclUint64, ncclMax, m->comm, s) != ncclSuccess)
            return B2_ERR_NCCL;
    }
    const unsigned long long* am_recv =
        xch ? reinterpret_cast<const unsigned long long*>(static_cast<char*>(m->p2p_base) + m->off_am_recv) : nullptr;
    const unsigned* am_flags =
        xch ? reinterpret_cast<const unsigned*>(static_cast<char*>(m->p2p_base) + m->off_am_flags) : nullptr;
    B2_TRY(launch(step_end_kernel, dim3(1), dim3(end_threads(B)), 0, s, pdl, (const unsigned long long*)m->argmax, m->tokens,
                  m->positions, B, m->hist_count, m->hist_cap, xch ? 1 : 0, am_recv, am_flags, m->tp,
                  c.max_batch, m->step_ctr, m->tpx.err, next_trace(m)));
    return B2_OK;
}

static int ensure_graph(b2_model* m, int B) {
    if (m->graphs[B]) return B2_OK;
    cudaGraph_t g = nullptr;
    B2_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(m, B);
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc != B2_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return (int)e;
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return (int)e;
    m->graphs[B] = ex;
    return B2_OK;
}

static int run_step(b2_model* m, int B) {
    static int use_graph = -1;
    if (use_graph < 0) {
        const char* e = getenv("B2_GRAPH");
        use_graph = (e && e[0] == '0') ? 0 : 1;
    }
    if (!use_graph) return enqueue_step(m, B);
    M_TRY(ensure_graph(m, B));
    B2_TRY(cudaGraphLaunch(m->graphs[B], m->stream));
    return B2_OK;
}

extern "C" int b2_model_set_sampling(b2_model* m, const b2_sampler_config* cfg) {
    B2_REQUIRE(m && cfg);
    const int on = cfg->temperature > 1e-6f ? 1 : 0;
    if (on && (m->tp != 1 || cfg->repetition_penalty != 1.0f || !(cfg->top_p > 0.f))) return B2_ERR_UNSUPPORTED;
    B2_TRY(cudaMemcpyAsync(m->d_samp_cfg, cfg, sizeof(*cfg), cudaMemcpyHostToDevice, m->stream));
    std::vector<uint64_t> st((size_t)m->cfg.max_batch, 13374269ull);  // a fresh sampler's state
    B2_TRY(cudaMemcpyAsync(m->d_rng, st.data(), st.size() * sizeof(uint64_t), cudaMemcpyHostToDevice, m->stream));
    B2_TRY(cudaStreamSynchronize(m->stream));
    if (on != m->sampling) {
        m->sampling = on;
        invalidate_graphs(m);  // the step gains or loses its sampling kernel
    }
    return B2_OK;
}

// Quantised copy of one projection (allocated on first use, kept).
static int quantize_proj(b2_model* m, const __half* w, int64_t rows, int K, Fp8W& f) {
    if (!f.q) {
        M_TRY(model_alloc(m, reinterpret_cast<void**>(&f.q), (size_t)rows * K));
        M_TRY(model_alloc(m, reinterpret_cast<void**>(&f.sc), (size_t)rows * sizeof(float)));
    }
    return quantize_e4m3_rows(w, rows, K, f.q, f.sc, m->stream);
}

static int quantize_proj_i4(b2_model* m, const __half* w, int64_t rows, int K, Fp8W& f) {
    if (!f.q) {
        M_TRY(model_alloc(m, reinterpret_cast<void**>(&f.q), (size_t)rows * (K / 2)));
        M_TRY(model_alloc(m, reinterpret_cast<void**>(&f.sc), (size_t)rows * (K / kI4Group) * sizeof(float)));
    }
    return quantize_i4_rows(w, rows, K, f.q, f.sc, m->stream);
}

extern "C" int b2_model_quantize_weights(b2_model* m, int format) {
    B2_REQUIRE(m && (format == B2_WEIGHTS_FP16 || format == B2_WEIGHTS_FP8_E4M3 || format == B2_WEIGHTS_INT4));
    const b2_model_config& c = m->cfg;
    const int H = c.hidden_size, qd = m->nq * c.head_dim;
    const bool f8 = format == B2_WEIGHTS_FP8_E4M3, i4 = format == B2_WEIGHTS_INT4;
    if (f8) {
        if ((H % 16) || (qd % 16) || (m->inter % 16)) return B2_ERR_UNSUPPORTED;
        for (int l = 0; l < c.num_layers; ++l) {
            LayerW& w = m->layers[l];
            M_TRY(quantize_proj(m, w.wqkv, m->qkv_rows, H, w.f8qkv));
            M_TRY(quantize_proj(m, w.wo, H, qd, w.f8o));
            M_TRY(quantize_proj(m, w.wg, m->inter, H, w.f8g));
            M_TRY(quantize_proj(m, w.wu, m->inter, H, w.f8u));
            M_TRY(quantize_proj(m, w.wd, H, m->inter, w.f8d));
        }
        M_TRY(quantize_proj(m, m->lm_head, m->vocab_l, H, m->f8lm));
        B2_TRY(cudaStreamSynchronize(m->stream));
    }
    if (i4) {
        if ((H % kI4Group) || (qd % kI4Group) || (m->inter % kI4Group)) return B2_ERR_UNSUPPORTED;
        for (int l = 0; l < c.num_layers; ++l) {
            LayerW& w = m->layers[l];
            M_TRY(quantize_proj_i4(m, w.wqkv, m->qkv_rows, H, w.i4qkv));
            M_TRY(quantize_proj_i4(m, w.wo, H, qd, w.i4o));
            M_TRY(quantize_proj_i4(m, w.wg, m->inter, H, w.i4g));
            M_TRY(quantize_proj_i4(m, w.wu, m->inter, H, w.i4u));
            M_TRY(quantize_proj_i4(m, w.wd, H, m->inter, w.i4d));
        }
        M_TRY(quantize_proj_i4(m, m->lm_head, m->vocab_l, H, m->i4lm));
        B2_TRY(cudaStreamSynchronize(m->stream));
    }
    if (f8 != m->wfp8 || i4 != m->wint4) {
        m->wfp8 = f8;
        m->wint4 = i4;
        invalidate_graphs(m);  // the step's GEMVs change form
    }
    return B2_OK;
}

extern "C" int b2_model_reset(b2_model* m) {
    B2_REQUIRE(m);
    B2_TRY(cudaMemsetAsync(m->positions, 0, (size_t)m->cfg.max_batch * sizeof(int), m->stream));
    B2_TRY(cudaMemsetAsync(m->hist_count, 0, sizeof(int), m->stream));
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

// true when the `bytes` at `p` are page-locked host memory (cudaMallocHost /
// cudaHostRegister), which the copy engine can write directly: both the first
// and the last byte must be, so a buffer registered only at its start goes
// through the staging copy instead.
static bool host_pinned(const void* p, size_t bytes) {
    const char* ends[2] = {static_cast<const char*>(p), static_cast<const char*>(p) + (bytes ? bytes - 1 : 0)};
    for (const char* q : ends) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (a.type != cudaMemoryTypeHost) return false;
    }
    return true;
}

static int copy_logits_out(b2_model* m, int B, float* host_logits) {
    const int V = m->cfg.vocab_size;
    if (m->tp == 1) {
        if (host_pinned(host_logits, (size_t)B * V * sizeof(float))) {  // the caller's buffer is page-locked: no staging copy
            B2_TRY(cudaMemcpyAsync(host_logits, m->logits, (size_t)B * V * sizeof(float), cudaMemcpyDeviceToHost,
                                   m->stream));
            B2_TRY(cudaStreamSynchronize(m->stream));
            return B2_OK;
        }
        B2_TRY(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)B * V * sizeof(float), cudaMemcpyDeviceToHost, m->stream));
        B2_TRY(cudaStreamSynchronize(m->stream));
        memcpy(host_logits, m->h_logits, (size_t)B * V * sizeof(float));
        return B2_OK;
    }
    const size_t nl = (size_t)B * m->vocab_l;
    if (nccl().AllGather(m->logits, m->logits_gather, nl, ncclFloat, m->comm, m->stream) != ncclSuccess) return B2_ERR_NCCL;
    B2_TRY(cudaMemcpyAsync(m->h_logits, m->logits_gather, nl * m->tp * sizeof(float), cudaMemcpyDeviceToHost, m->stream));
    B2_TRY(cudaStreamSynchronize(m->stream));
    for (int r = 0; r < m->tp; ++r)
        for (int b = 0; b < B; ++b)
            memcpy(host_logits + (size_t)b * V + (size_t)r * m->vocab_l, m->h_logits + r * nl + (size_t)b * m->vocab_l,
                   (size_t)m->vocab_l * sizeof(float));
    return B2_OK;
}

static int read_next(b2_model* m, int B, int64_t* host_next) {
    B2_TRY(cudaMemcpyAsync(m->h_tokens, m->tokens, (size_t)B * sizeof(int64_t), cudaMemcpyDeviceToHost, m->stream));
    B2_TRY(cudaStreamSynchronize(m->stream));
    memcpy(host_next, m->h_tokens, (size_t)B * sizeof(int64_t));
    return B2_OK;
}

extern "C" int b2_model_decode_step(b2_model* m, const int64_t* host_tokens, const int* host_positions, int B,
                                    float* host_logits, int64_t* host_next) {
    B2_REQUIRE(m && host_tokens && host_positions && B >= 1 && B <= m->cfg.max_batch);
    if (m->paged) return B2_ERR_STATE;
    for (int b = 0; b < B; ++b) {
        if (host_positions[b] < 0 || host_positions[b] >= m->cfg.max_seq) return B2_ERR_INVALID;
        if (host_tokens[b] < 0 || host_tokens[b] >= m->cfg.vocab_size) return B2_ERR_INVALID;
    }
    memcpy(m->h_tokens, host_tokens, (size_t)B * sizeof(int64_t));
    memcpy(m->h_pos, host_positions, (size_t)B * sizeof(int));
    B2_TRY(cudaMemcpyAsync(m->tokens, m->h_tokens, (size_t)B * sizeof(int64_t), cudaMemcpyHostToDevice, m->stream));
    B2_TRY(cudaMemcpyAsync(m->positions, m->h_pos, (size_t)B * sizeof(int), cudaMemcpyHostToDevice, m->stream));
    M_TRY(run_step(m, B));
    m->last_B = B;
    if (host_logits) M_TRY(copy_logits_out(m, B, host_logits));
    if (host_next) M_TRY(read_next(m, B, host_next));
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

extern "C" int b2_model_decode_enqueue(b2_model* m, const int64_t* host_tokens, const int* host_positions, int B,
                                       float* d_logits) {
    B2_REQUIRE(m && host_tokens && host_positions && B >= 1 && B <= m->cfg.max_batch);
    if (m->paged) return B2_ERR_STATE;
    if (d_logits && m->tp != 1) return B2_ERR_UNSUPPORTED;
    StepInputs in;
    for (int b = 0; b < B; ++b) {
        if (host_positions[b] < 0 || host_positions[b] >= m->cfg.max_seq) return B2_ERR_INVALID;
        if (host_tokens[b] < 0 || host_tokens[b] >= m->cfg.vocab_size) return B2_ERR_INVALID;
        in.tokens[b] = host_tokens[b];
        in.positions[b] = host_positions[b];
    }
    set_step_inputs_kernel<<<1, 32, 0, m->stream>>>(in, B, m->tokens, m->positions);
    B2_CHECK_LAUNCH();
    M_TRY(run_step(m, B));
    m->last_B = B;
    if (d_logits)
        B2_TRY(cudaMemcpyAsync(d_logits, m->logits, (size_t)B * m->cfg.vocab_size * sizeof(float),
                               cudaMemcpyDeviceToDevice, m->stream));
    return B2_OK;
}

static int ensure_prefill_ws(b2_model* m, int64_t T) {
    if (T <= m->pf_tokens) return B2_OK;
    for (void* p : {(void*)m->pf_hidden, (void*)m->pf_xn, (void*)m->pf_qkv, (void*)m->pf_attn, (void*)m->pf_gate,
                    (void*)m->pf_up, (void*)m->pf_ids})
        cudaFree(p);
    m->pf_hidden = nullptr; m->pf_xn = m->pf_qkv = m->pf_attn = m->pf_gate = m->pf_up = nullptr; m->pf_ids = nullptr;
    m->pf_tokens = 0;
    const b2_model_config& c = m->cfg;
    const size_t H = c.hidden_size, hs = sizeof(__half);
    B2_TRY(cudaMalloc(&m->pf_hidden, T * H * sizeof(float)));
    B2_TRY(cudaMalloc(&m->pf_xn, T * H * hs));
    B2_TRY(cudaMalloc(&m->pf_qkv, T * (size_t)m->qkv_rows * hs));
    B2_TRY(cudaMalloc(&m->pf_attn, T * (size_t)m->nq * c.head_dim * hs));
    B2_TRY(cudaMalloc(&m->pf_gate, T * (size_t)m->inter * hs));
    B2_TRY(cudaMalloc(&m->pf_up, T * (size_t)m->inter * hs));
    B2_TRY(cudaMalloc(&m->pf_ids, T * sizeof(int64_t)));
    m->pf_tokens = T;
    return B2_OK;
}

static int nccl_sum_rows(b2_model* m, float* buf, int64_t rows) {
    if (m->tp == 1) return B2_OK;
    if (nccl().AllReduce(buf, buf, (size_t)rows * m->cfg.hidden_size, ncclFloat, ncclSum, m->comm, m->stream) !=
        ncclSuccess)
        return B2_ERR_NCCL;
    return B2_OK;
}

// All prompt tokens of all sequences through the layers at once: tensor-core
// GEMMs for every projection, the tensor-core flash prefill for attention,
// K/V written into the cache, then the lm_head (with argmax) of each
// sequence's last position through the decode GEMV.
static int prefill_batched(b2_model* m, int B, int S, int skip_pos = 0) {
    const b2_model_config& c = m->cfg;
    cudaStream_t st = m->stream;
    const int64_t T = (int64_t)B * S;
    const int H = c.hidden_size, D = c.head_dim, I = m->inter, qd = m->nq * D;
    const int rows = (int)T;
    embed_rows_kernel<<<(unsigned)T, 128, 0, st>>>(m->pf_ids, m->embed, m->pf_hidden, H);
    B2_CHECK_LAUNCH();
    const int norm_threads = H >= 1024 ? 256 : 128;
    for (int l = 0; l < c.num_layers; ++l) {
        LayerW& w = m->layers[l];
        rmsnorm_rows_kernel<<<(unsigned)T, norm_threads, 0, st>>>(m->pf_hidden, w.ln1, m->pf_xn, H, c.rms_norm_eps);
        B2_CHECK_LAUNCH();
        M_TRY(gemm_tc(m->pf_xn, w.wqkv, m->pf_qkv, rows, m->qkv_rows, H, TC_HALF, st));
        if (w.bqkv) M_TRY(b2_bias_add(m->pf_qkv, w.bqkv, m->pf_qkv, T, m->qkv_rows, st));
        rope_append_kernel<<<dim3((unsigned)T, (unsigned)(m->nq + 2 * m->nkv)), D / 2, 0, st>>>(
            m->pf_qkv, m->qkv_rows, m->rope, S, m->nq, m->nkv, D, layer_kv(m, l), skip_pos, nullptr);
        B2_CHECK_LAUNCH();
        FlashArgs fa = {};
        fa.q = m->pf_qkv;
        fa.k = m->pf_qkv + qd;
        fa.v = m->pf_qkv + qd + m->nkv * D;
        fa.out = m->pf_attn;
        fa.S = S;
        fa.nq = m->nq;
        fa.nkv = m->nkv;
        fa.D = D;
        fa.batch = B;
        fa.ldq = fa.ldkv = m->qkv_rows;
        fa.ldo = qd;
        int rc = flash_prefill_tc(fa, st);
        if (rc == B2_ERR_UNSUPPORTED)
            rc = causal_attention_rows_ld(m->pf_qkv, m->qkv_rows, m->pf_qkv + qd, m->pf_qkv + qd + m->nkv * D,
                                          m->qkv_rows, m->pf_attn, qd, S, m->nq, m->nkv, D, B, st);
        M_TRY(rc);
        M_TRY(gemm_tc(m->pf_attn, w.wo, m->pf_hidden, rows, H, qd, m->rank == 0 ? TC_F32_ADD : TC_F32, st));
        M_TRY(nccl_sum_rows(m, m->pf_hidden, T));
        rmsnorm_rows_kernel<<<(unsigned)T, norm_threads, 0, st>>>(m->pf_hidden, w.ln2, m->pf_xn, H, c.rms_norm_eps);
        B2_CHECK_LAUNCH();
        M_TRY(gemm_tc(m->pf_xn, w.wg, m->pf_gate, rows, I, H, TC_HALF, st));
        M_TRY(gemm_tc(m->pf_xn, w.wu, m->pf_up, rows, I, H, TC_HALF, st));
        M_TRY(b2_swiglu(m->pf_gate, m->pf_up, m->pf_gate, T * I, st));
        M_TRY(gemm_tc(m->pf_gate, w.wd, m->pf_hidden, rows, H, I, m->rank == 0 ? TC_F32_ADD : TC_F32, st));
        M_TRY(nccl_sum_rows(m, m->pf_hidden, T));
    }
    gather_last_kernel<<<B, 256, 0, st>>>(m->pf_hidden, m->hidden, S, H);
    B2_CHECK_LAUNCH();
    B2_TRY(cudaMemsetAsync(m->argmax, 0, (size_t)B * sizeof(unsigned long long), st));
    if (gemv_step(m, B)) {
        M_TRY(launch_lm_head(m, B, false));
    } else {
        rmsnorm_rows_kernel<<<B, 256, 0, st>>>(m->hidden, m->final_norm, m->bxn, H, c.rms_norm_eps);
        B2_CHECK_LAUNCH();
        M_TRY(lm_head_rows(m, B));
    }
    if (m->sampling)
        M_TRY(step_sample_launch(m->logits, m->vocab_l, m->vocab_l, B, m->d_samp_cfg, m->d_rng, m->argmax, st));
    if (m->tp > 1) {
        if (nccl().AllReduce(m->argmax, m->argmax, (size_t)B, ncclUint64, ncclMax, m->comm, st) != ncclSuccess)
            return B2_ERR_NCCL;
    }
    prefill_end_kernel<<<1, end_threads(B), 0, st>>>(m->argmax, m->tokens, m->positions, B, S);
    B2_CHECK_LAUNCH();
    return B2_OK;
}

extern "C" int b2_model_prefill(b2_model* m, const int64_t* host_ids, int B, int S, float* host_logits) {
    B2_REQUIRE(m && host_ids && B >= 1 && B <= m->cfg.max_batch && S >= 1 && S <= m->cfg.max_seq);
    if (m->paged) return B2_ERR_STATE;
    for (int64_t i = 0; i < (int64_t)B * S; ++i)
        if (host_ids[i] < 0 || host_ids[i] >= m->cfg.vocab_size) return B2_ERR_INVALID;
    M_TRY(ensure_prefill_ws(m, (int64_t)B * S));
    B2_TRY(cudaMemcpyAsync(m->pf_ids, host_ids, (size_t)B * S * sizeof(int64_t), cudaMemcpyHostToDevice, m->stream));
    B2_TRY(cudaMemsetAsync(m->hist_count, 0, sizeof(int), m->stream));
    M_TRY(prefill_batched(m, B, S));
    m->last_B = B;
    if (host_logits) M_TRY(copy_logits_out(m, B, host_logits));
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

// Copy B block-table rows (host, max_blocks wide) into the device tables
// (kv_maxb wide, zero-padded), checking the entries every sequence of
// lens[b] positions uses.
static int upload_block_tables(b2_model* m, const int* host_bt, int max_blocks, int B, const int* lens) {
    for (int b = 0; b < B; ++b) {
        const int used = (lens[b] + m->kv_bs - 1) / m->kv_bs;
        if (used > max_blocks || used > m->kv_maxb) return B2_ERR_INVALID;
        for (int j = 0; j < used; ++j) {
            const int blk = host_bt[(int64_t)b * max_blocks + j];
            if (blk < 0 || blk >= m->kv_blocks) return B2_ERR_INVALID;
        }
        int* row = m->h_bt + (int64_t)b * m->kv_maxb;
        const int w = max_blocks < m->kv_maxb ? max_blocks : m->kv_maxb;
        for (int j = 0; j < m->kv_maxb; ++j) {
            int v = j < w ? host_bt[(int64_t)b * max_blocks + j] : 0;
            row[j] = (v >= 0 && v < m->kv_blocks) ? v : 0;  // padding slots read a valid block, masked
        }
    }
    B2_TRY(cudaMemcpyAsync(m->block_tables, m->h_bt, (size_t)B * m->kv_maxb * sizeof(int), cudaMemcpyHostToDevice,
                           m->stream));
    return B2_OK;
}

extern "C" int b2_model_prefill_paged(b2_model* m, const int64_t* host_ids, int S, const int* host_block_table,
                                      int n_blocks, int skip_blocks, float* host_logits, int64_t* first_token) {
    B2_REQUIRE(m && host_ids && host_block_table && S >= 1 && S <= m->cfg.max_seq && n_blocks >= 1 &&
               skip_blocks >= 0);
    if (!m->paged) return B2_ERR_STATE;
    for (int64_t i = 0; i < S; ++i)
        if (host_ids[i] < 0 || host_ids[i] >= m->cfg.vocab_size) return B2_ERR_INVALID;
    M_TRY(upload_block_tables(m, host_block_table, n_blocks, 1, &S));
    M_TRY(ensure_prefill_ws(m, S));
    B2_TRY(cudaMemcpyAsync(m->pf_ids, host_ids, (size_t)S * sizeof(int64_t), cudaMemcpyHostToDevice, m->stream));
    B2_TRY(cudaMemsetAsync(m->hist_count, 0, sizeof(int), m->stream));
    M_TRY(prefill_batched(m, 1, S, skip_blocks * m->kv_bs));
    m->last_B = 1;
    if (host_logits) M_TRY(copy_logits_out(m, 1, host_logits));
    if (first_token) M_TRY(read_next(m, 1, first_token));
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

extern "C" int b2_model_decode_step_paged(b2_model* m, const int64_t* host_tokens, const int* host_seq_lens,
                                          const int* host_block_tables, int max_blocks, int B, float* host_logits,
                                          int64_t* host_next) {
    B2_REQUIRE(m && host_tokens && host_seq_lens && host_block_tables && max_blocks >= 1 && B >= 1 &&
               B <= m->cfg.max_batch);
    if (!m->paged) return B2_ERR_STATE;
    for (int b = 0; b < B; ++b) {
        if (host_seq_lens[b] < 1 || host_seq_lens[b] > m->cfg.max_seq) return B2_ERR_INVALID;
        if (host_tokens[b] < 0 || host_tokens[b] >= m->cfg.vocab_size) return B2_ERR_INVALID;
    }
    M_TRY(upload_block_tables(m, host_block_tables, max_blocks, B, host_seq_lens));
    memcpy(m->h_tokens, host_tokens, (size_t)B * sizeof(int64_t));
    for (int b = 0; b < B; ++b) m->h_pos[b] = host_seq_lens[b] - 1;  // the new token's position
    B2_TRY(cudaMemcpyAsync(m->tokens, m->h_tokens, (size_t)B * sizeof(int64_t), cudaMemcpyHostToDevice, m->stream));
    B2_TRY(cudaMemcpyAsync(m->positions, m->h_pos, (size_t)B * sizeof(int), cudaMemcpyHostToDevice, m->stream));
    M_TRY(run_step(m, B));
    m->last_B = B;
    if (host_logits) M_TRY(copy_logits_out(m, B, host_logits));
    if (host_next) M_TRY(read_next(m, B, host_next));
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

extern "C" int b2_model_forward_logits(b2_model* m, const int64_t* host_ids, int S, float* host_logits) {
    B2_REQUIRE(m && host_ids && host_logits && S >= 1 && S <= m->cfg.max_seq);
    if (m->paged) return B2_ERR_STATE;
    if (m->tp != 1) return B2_ERR_UNSUPPORTED;
    const b2_model_config& c = m->cfg;
    for (int64_t i = 0; i < S; ++i)
        if (host_ids[i] < 0 || host_ids[i] >= c.vocab_size) return B2_ERR_INVALID;
    M_TRY(ensure_prefill_ws(m, S));
    if (S > m->pf_logits_rows) {
        cudaFree(m->pf_logits);
        m->pf_logits = nullptr;
        m->pf_logits_rows = 0;
        B2_TRY(cudaMalloc(&m->pf_logits, (size_t)S * c.vocab_size * sizeof(float)));
        m->pf_logits_rows = S;
    }
    cudaStream_t st = m->stream;
    B2_TRY(cudaMemcpyAsync(m->pf_ids, host_ids, (size_t)S * sizeof(int64_t), cudaMemcpyHostToDevice, st));
    B2_TRY(cudaMemsetAsync(m->hist_count, 0, sizeof(int), st));
    M_TRY(prefill_batched(m, 1, S));
    m->last_B = 1;
    // every position through the final norm and the lm_head (tensor cores)
    const int H = c.hidden_size;
    rmsnorm_rows_kernel<<<(unsigned)S, H >= 1024 ? 256 : 128, 0, st>>>(m->pf_hidden, m->final_norm, m->pf_xn, H,
                                                                      c.rms_norm_eps);
    B2_CHECK_LAUNCH();
    M_TRY(gemm_tc(m->pf_xn, m->lm_head, m->pf_logits, S, c.vocab_size, H, TC_F32, st));
    B2_TRY(cudaMemcpyAsync(host_logits, m->pf_logits, (size_t)S * c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost,
                           st));
    B2_TRY(cudaStreamSynchronize(st));
    return B2_OK;
}

extern "C" int b2_model_generate_greedy(b2_model* m, int steps, int64_t* host_tokens_out) {
    B2_REQUIRE(m && steps >= 0);
    if (m->last_B <= 0) return B2_ERR_STATE;
    const int B = m->last_B;
    if (host_tokens_out && steps > m->hist_cap) return B2_ERR_INVALID;
    B2_TRY(cudaMemsetAsync(m->hist_count, 0, sizeof(int), m->stream));
    for (int i = 0; i < steps; ++i) M_TRY(run_step(m, B));
    if (host_tokens_out && steps > 0) {
        B2_TRY(cudaMemcpyAsync(host_tokens_out, m->hist, (size_t)steps * B * sizeof(int64_t), cudaMemcpyDeviceToHost,
                               m->stream));
        B2_TRY(cudaStreamSynchronize(m->stream));
    }
    return B2_OK;
}

extern "C" int b2_model_sync(b2_model* m) {
    B2_REQUIRE(m);
    B2_TRY(cudaStreamSynchronize(m->stream));
    return B2_OK;
}

extern "C" void* b2_model_stream(b2_model* m) { return m ? (void*)m->stream : nullptr; }

extern "C" void* b2_model_buffer(b2_model* m, const char* name) {
    if (!m || !name) return nullptr;
    std::string n(name);
    if (n == "logits") return m->logits;
    if (n == "hidden") return m->hidden;
    if (n == "kv") return m->kv;
    if (n == "tokens") return m->tokens;
    if (n == "positions") return m->positions;
    if (n == "history") return m->hist;
    if (n == "history_count") return m->hist_count;
    return nullptr;
}

extern "C" int b2_model_read(b2_model* m, const char* name, void* dst, size_t offset, size_t bytes) {
    B2_REQUIRE(m && name && dst);
    char* src = static_cast<char*>(b2_model_buffer(m, name));
    B2_REQUIRE(src);
    B2_TRY(cudaStreamSynchronize(m->stream));
    B2_TRY(cudaMemcpy(dst, src + offset, bytes, cudaMemcpyDeviceToHost));
    return B2_OK;
}

extern "C" int b2_model_kv_layout(const b2_model* m, int64_t* sl, int64_t* sb, int64_t* skv, int64_t* sh, int64_t* sp) {
    B2_REQUIRE(m && sl && sb && skv && sh && sp);
    if (m->paged) return B2_ERR_STATE;
    *sl = m->kv_s_layer;
    *sb = m->kv_s_batch;
    *skv = m->kv_s_kv;
    *sh = m->kv_s_head;
    *sp = m->cfg.head_dim;
    return B2_OK;
}

extern "C" double b2_model_step_bytes(const b2_model* m, int B, int ctx) {
    if (!m) return 0.0;
    const b2_model_config& c = m->cfg;
    const double H = c.hidden_size, D = c.head_dim, L = c.num_layers;
    const double rows = L * ((double)m->qkv_rows + H + 2.0 * m->inter + H) + m->vocab_l;
    const double lin = L * ((double)m->qkv_rows * H + H * m->nq * D + 2.0 * m->inter * H + H * m->inter) +
                       (double)m->vocab_l * H;
    // decode GEMVs on FP8 copies: 1 byte per weight and an fp32 scale per row;
    // on 4-bit copies: half a byte per weight and an fp32 scale per 128
    const bool f8 = m->wfp8 && (gemv_step(m, B) ? B <= kFp8MaxBatch : B <= 128);
    const bool i4 = m->wint4 && gemv_step(m, B) && B <= kI4MaxBatch;
    double bytes = f8 ? lin + 4.0 * rows : i4 ? 0.5 * lin + 4.0 * lin / kI4Group : 2.0 * lin;
    if (c.has_qkv_bias) bytes += 2.0 * L * m->qkv_rows;
    bytes += 2.0 * B * H;                               // embedding rows
    bytes += 2.0 * (2.0 * L + 1.0) * H;                 // norm weights
    bytes += (double)B * L * 2.0 * m->nkv * D * 2.0 * ctx;  // KV read
    bytes += (double)B * L * 2.0 * m->nkv * D * 2.0;        // KV write
    bytes += 4.0 * B * m->vocab_l;                      // logits
    return bytes;
}

extern "C" int b2_model_time_kernel(b2_model* m, int kind, int B, int reps, float* avg_ms) {
    B2_REQUIRE(m && avg_ms && B >= 1 && B <= m->cfg.max_batch && reps >= 1 && kind >= 0 && kind <= 5);
    if (!gemv_step(m, B)) return B2_ERR_UNSUPPORTED;  // the batched step has no single fused kernel per kind
    const int L = m->cfg.num_layers;
    auto one = [&](int l) -> int {
        switch (kind) {
            case 0: return launch_qkv(m, l, B, true);
            case 1: return launch_attn(m, l, B, true);
            case 2: return launch_o(m, l, B, true);
            case 3: return launch_gateup(m, l, B, true);
            case 4: return launch_down(m, l, B, true);
            default: return launch_lm_head(m, B, true);
        }
    };
    // warm-up pass
    for (int l = 0; l < L; ++l) M_TRY(one(l));
    cudaEvent_t e0, e1;
    B2_TRY(cudaEventCreate(&e0));
    B2_TRY(cudaEventCreate(&e1));
    B2_TRY(cudaEventRecord(e0, m->stream));
    int n = 0;
    for (int r = 0; r < reps; ++r)
        for (int l = 0; l < L; ++l, ++n) M_TRY(one(l));
    B2_TRY(cudaEventRecord(e1, m->stream));
    B2_TRY(cudaEventSynchronize(e1));
    float ms = 0.f;
    B2_TRY(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *avg_ms = ms / (float)n;
    return B2_OK;
}

extern "C" double b2_model_kernel_bytes(const b2_model* m, int kind, int B, int ctx) {
    if (!m) return 0.0;
    const b2_model_config& c = m->cfg;
    const double H = c.hidden_size, D = c.head_dim;
    // weight bytes of `rows` rows of width K: fp16, or FP8 codes + fp32 scales
    const bool f8 = m->wfp8 && (gemv_step(m, B) ? B <= kFp8MaxBatch : B <= 128);
    const bool i4 = m->wint4 && gemv_step(m, B) && B <= kI4MaxBatch;
    auto wb = [&](double rows, double K) {
        return f8 ? rows * K + 4.0 * rows : i4 ? 0.5 * rows * K + 4.0 * rows * K / kI4Group : 2.0 * rows * K;
    };
    switch (kind) {
        case 0: return wb(m->qkv_rows, H) + 4.0 * B * H + 2.0 * H + 2.0 * B * m->qkv_rows;
        case 1: return 2.0 * B * m->nkv * D * 2.0 * ctx + 2.0 * 2.0 * B * m->nq * D;
        case 2: return wb(H, m->nq * D) + 2.0 * B * m->nq * D + 8.0 * B * H;
        case 3: return 2.0 * wb(m->inter, H) + 4.0 * B * H + 2.0 * H + 2.0 * B * m->inter;
        case 4: return wb(H, m->inter) + 2.0 * B * m->inter + 8.0 * B * H;
        default: return wb(m->vocab_l, H) + 4.0 * B * H + 2.0 * H + 4.0 * B * m->vocab_l;
    }
}

extern "C" int b2_model_trace_step(b2_model* m, int B, unsigned long long* host_ns, int max_slots, int* n_slots) {
    B2_REQUIRE(m && host_ns && n_slots && B >= 1 && B <= m->cfg.max_batch && max_slots > 0);
    const int need = b2_model_step_launches(m, B);
    if (!m->trace_buf) B2_TRY(cudaMalloc(&m->trace_buf, (size_t)2 * need * sizeof(unsigned long long)));
    std::vector<unsigned long long> init(2 * (size_t)need);
    for (int i = 0; i < need; ++i) {
        init[2 * i] = ~0ull;
        init[2 * i + 1] = 0ull;
    }
    B2_TRY(cudaMemcpyAsync(m->trace_buf, init.data(), init.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice,
                           m->stream));
    m->trace_cur = m->trace_buf;
    m->trace_next = 0;
    const int rc = enqueue_step(m, B);
    m->trace_cur = nullptr;
    if (rc != B2_OK) return rc;
    m->last_B = B;
    B2_TRY(cudaMemcpyAsync(init.data(), m->trace_buf, init.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                           m->stream));
    B2_TRY(cudaStreamSynchronize(m->stream));
    const int n = m->trace_next < max_slots ? m->trace_next : max_slots;
    for (int i = 0; i < 2 * n; ++i) host_ns[i] = init[i];
    *n_slots = m->trace_next;
    return B2_OK;
}

extern "C" int b2_model_step_launches(const b2_model* m, int B) {
    if (!m) return 0;
    if (!gemv_step(m, B))  // batched step: 13 launches per layer, final norm + lm_head GEMM + argmax
        return 5 + m->cfg.num_layers * 13;
    // step_begin, per layer {qkv, attention (merges its own splits), o, gateup, down}, lm_head, step_end
    return 3 + m->cfg.num_layers * 5;
}
