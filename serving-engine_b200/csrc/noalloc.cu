// noalloc.cu -- split-KV decode attention for callers that cannot allocate.
//
// Some callers may not call cudaMalloc at all: code that runs inside a
// host-side allocator or memory-pool callback (where allocating again would
// re-enter the allocator), plugin hosts that own every device byte and hand
// out no scratch, and hot paths that have to stay free of allocator locks and
// implicit synchronisation.  b2_decode_gqa_split needs a scratch buffer for
// its per-split partial results when its global-merge kernel cuts a long
// context into several splits; this file gives those callers the same
// kernels with that scratch taken from a fixed array that lives in the
// library's device image.
//
// Shapes the cluster-merged kernels take (head_dim 32/64/128/256 with
// 8-element-aligned strides; head_dim 128 on the tensor cores) need no
// scratch at all and run exactly as b2_decode_gqa_split runs them.  The rest
// go to the global-merge kernel with as many splits as the shape prefers,
// capped so that the partial results fit the array: the array bounds the
// split count (and so the speed of very large problems), never which shapes
// run.  One split per (sequence, kv head) needs no scratch.
//
// The array is a file-scope __device__ object, so every GPU that loads this
// library holds kNoAllocScratchBytes for it until the process exits, and all
// calls on one device share it: two of these calls that overlap on the GPU
// (different streams, or concurrent host threads) race on the same scratch.
// The arrival counters inside it are cleared at the start of every call; the
// partial results are overwritten before they are read.
#include <mutex>

#include "attention.cuh"
#include "common.cuh"

namespace b2 {

struct AttnParams;
int attn_pick_splits(int batch, int nq, int nkv, int D, int max_len, size_t cap_floats);
size_t attn_scratch_floats(int batch, int nq, int nkv, int D, int splits);
bool attn_head_dim_supported(int D);
int attn_decode_launch_model(const __half* q, const __half* kbase, const __half* vbase, int64_t sb, int64_t sh,
                             int64_t ss, const int* seq_lens, __half* out, float* part, int splits, int B, int nq,
                             int nkv, int D, cudaStream_t s, bool pdl);

// 4 MiB of partial results (1,048,576 floats).
constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocScratchFloats = kNoAllocScratchBytes / sizeof(float);

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch per device, looked up (with that device
// current) by the first call on that device that needs it and cached for the
// life of the process.
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64];

static int noalloc_scratch(float** out) {
    int dev = 0;
    B2_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return B2_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        B2_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return B2_OK;
}

}  // namespace b2

using namespace b2;

extern "C" int b2_decode_gqa_split_noalloc(const void* q, b2_kv_view kv, b2_kv_view vv, const int* seq_lens,
                                           void* out, int B, int nq, int nkv, int D, int max_seq_len,
                                           void* stream) {
    if (B <= 0) return B2_OK;
    B2_REQUIRE(q && out && seq_lens && nq > 0 && nkv > 0 && nq % nkv == 0 && max_seq_len >= 0);
    if (!attn_head_dim_supported(D)) return B2_ERR_UNSUPPORTED;
    if (!kv.data || !vv.data || kv.stride_d != 1 || vv.stride_d != 1 || !aligned16(kv.data) || !aligned16(vv.data) ||
        kv.stride_b != vv.stride_b || kv.stride_h != vv.stride_h || kv.stride_s != vv.stride_s ||
        (kv.stride_b % 8) || (kv.stride_h % 8) || (kv.stride_s % 8) || !aligned16(q) || !aligned16(out))
        return B2_ERR_UNSUPPORTED;
    cudaStream_t s = as_stream(stream);
    {   // cluster-merged kernels: the splits meet in distributed shared memory
        const int rc = attn_cl_launch((const __half*)q, (int64_t)nq * D, (__half*)out, (int64_t)nq * D,
                                      (const __half*)kv.data, (const __half*)vv.data, kv.stride_b, kv.stride_h,
                                      kv.stride_s, max_seq_len, seq_lens, 0, B, nq, nkv, D, 0, 0, TraceSlot{nullptr, 0},
                                      s, true);
        if (rc != B2_ERR_UNSUPPORTED) return rc;
    }
    // Global-merge kernel: the split count the shape prefers, lowered until
    // its partial results fit the fixed array (fewer splits give the same
    // result with fewer CTAs streaming each (sequence, kv head)).
    const int splits = attn_pick_splits(B, nq, nkv, D, max_seq_len, kNoAllocScratchFloats);
    float* scratch = nullptr;
    if (splits > 1) {
        const int rc = noalloc_scratch(&scratch);
        if (rc != B2_OK) return rc;
        const size_t need = attn_scratch_floats(B, nq, nkv, D, splits);
        const size_t off = (size_t)B * nq * splits * (D + 2);
        B2_TRY(cudaMemsetAsync(scratch + off, 0, (need - off) * sizeof(int), s));
    }
    return attn_decode_launch_model((const __half*)q, (const __half*)kv.data, (const __half*)vv.data, kv.stride_b,
                                    kv.stride_h, kv.stride_s, seq_lens, (__half*)out, scratch, splits, B, nq, nkv, D,
                                    s, true);
}
