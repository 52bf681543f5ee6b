// noalloc.cu -- split-KV decode attention for callers that cannot allocate.
//
// Some callers may not call cudaMalloc at all: code that runs inside a
// host-side allocator or memory-pool callback (where allocating again would
// re-enter the allocator), plugin hosts that own every device byte and hand
// out no scratch, and hot paths that have to stay free of allocator locks and
// implicit synchronisation.  b2_decode_gqa_split needs a scratch buffer for
// its per-split partial results when it cuts a long context into several
// splits; this file gives those callers the same kernel with its scratch
// taken from a fixed array that lives in the library's device image.
//
// The array is a file-scope __device__ object, so every GPU that loads this
// library holds kNoAllocScratchBytes for it until the process exits, and all
// calls on one device share it: two of these calls that overlap on the GPU
// (different streams, or concurrent host threads) race on the same scratch.
// The arrival counters inside it are cleared at the start of every call; the
// partial results are overwritten before they are read.
#include <mutex>

#include "common.cuh"

namespace b2 {

struct AttnParams;
int attn_pick_splits(int batch, int nq, int nkv, int D, int max_len, size_t cap_floats);
size_t attn_scratch_floats(int batch, int nq, int nkv, int D, int splits);
bool attn_head_dim_supported(int D);
int attn_decode_launch_model(const __half* q, const __half* kbase, const __half* vbase, int64_t sb, int64_t sh,
                             int64_t ss, const int* seq_lens, __half* out, float* part, int splits, int B, int nq,
                             int nkv, int D, cudaStream_t s, bool pdl);

// 4 MiB: enough for the preferred split count of every configuration with
// head_dim <= 128 at any batch size and context length.
constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocScratchFloats = kNoAllocScratchBytes / sizeof(float);

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch per device, looked up once per device
// (with that device current) on the first call made on it.
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
    // The split count this shape prefers when scratch is not a constraint;
    // problems whose partial results for that count do not fit the fixed
    // array are refused rather than silently run with fewer splits.
    const int splits = attn_pick_splits(B, nq, nkv, D, max_seq_len, (size_t)-1);
    const size_t need = attn_scratch_floats(B, nq, nkv, D, splits);
    if (need > kNoAllocScratchFloats) return B2_ERR_WORKSPACE;
    float* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != B2_OK) return rc;
    cudaStream_t s = as_stream(stream);
    if (splits > 1) {
        const size_t off = (size_t)B * nq * splits * (D + 2);
        B2_TRY(cudaMemsetAsync(scratch + off, 0, (need - off) * sizeof(int), s));
    }
    return attn_decode_launch_model((const __half*)q, (const __half*)kv.data, (const __half*)vv.data, kv.stride_b,
                                    kv.stride_h, kv.stride_s, seq_lens, (__half*)out, scratch, splits, B, nq, nkv, D,
                                    s, true);
}
