// common.cuh -- device helpers shared by the sm_100a kernels of b2engine.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b2engine.h"

namespace b2 {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// status helpers (host)
// ---------------------------------------------------------------------------

#define B2_TRY(expr)                                   \
    do {                                               \
        cudaError_t e_ = (expr);                       \
        if (e_ != cudaSuccess) return (int)e_;         \
    } while (0)

#define B2_CHECK_LAUNCH()                              \
    do {                                               \
        cudaError_t e_ = cudaGetLastError();           \
        if (e_ != cudaSuccess) return (int)e_;         \
    } while (0)

#define B2_REQUIRE(cond)                               \
    do {                                               \
        if (!(cond)) return B2_ERR_INVALID;            \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Whether kernels are launched with programmatic dependent launch (PDL).
// On by default; B2_PDL=0 in the environment turns it off.
bool pdl_enabled();

// Launch `kernel` with cudaLaunchKernelEx, adding the programmatic
// stream-serialisation attribute when PDL is on.  The kernel must call
// griddep_wait() before touching anything the previous kernel writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool allow_pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (allow_pdl && pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// As launch(), with thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, bool allow_pdl, unsigned cluster_x, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (allow_pdl && pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------

// Programmatic dependent launch: wait until the preceding kernel in the
// stream has completed and its writes are visible.  No-op when the kernel was
// not launched with the PDL attribute.
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Allow the next kernel in the stream to begin launching its CTAs.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

// Step trace: one (start, end) pair of %globaltimer nanoseconds per launch
// slot; start = the first CTA past its programmatic-launch wait, end = the
// last CTA to finish.  buf == nullptr: tracing off.
struct TraceSlot {
    unsigned long long* buf;
    int slot;
};

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void trace_begin(const TraceSlot& tr) {
    if (tr.buf && threadIdx.x == 0) atomicMin(tr.buf + 2 * tr.slot, globaltimer_ns());
}

__device__ __forceinline__ void trace_end(const TraceSlot& tr) {
    if (tr.buf && threadIdx.x == 0) atomicMax(tr.buf + 2 * tr.slot + 1, globaltimer_ns());
}

// Where one layer's K and V rows live.  Contiguous: element d of (sequence
// b, kv head h, position pos) at base + b*sb + h*sh + pos*D + d (the model's
// [batch][K|V][head][max_seq][D] cache).  Paged (bt != null): block tables
// [B][maxb] of physical blocks of `bs` positions, a block's rows stored
// [slot][head][D], so the row is at base + ((bt[b][pos/bs]*bs + pos%bs)*nkv
// + h)*D -- the pool layout [num_blocks][block_size][kv_heads][head_dim] of
// the reference's paged runner contract.
struct KvLayout {
    __half* k;
    __half* v;
    int64_t sb, sh;
    const int* bt;
    int maxb, bs, nkv;
};

__device__ __forceinline__ int64_t kv_row(const KvLayout& L, int b, int h, int pos, int D) {
    if (L.bt) {
        const int blk = L.bt[(int64_t)b * L.maxb + pos / L.bs];
        return (((int64_t)blk * L.bs + pos % L.bs) * L.nkv + h) * D;
    }
    return (int64_t)b * L.sb + (int64_t)h * L.sh + (int64_t)pos * D;
}

// 16-byte streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// 16-byte load through the normal path (data other kernels of this step wrote).
__device__ __forceinline__ uint4 ldg16(const void* p) {
    return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// acc + a * b for the low (H = 0) or high (H = 1) halves of two half2
// words: sm_100's mixed-precision FMA (f16 operands, f32 addend and result,
// one rounding) -- the value of fmaf(float(a), float(b), acc), since every
// half converts to float exactly, in one instruction instead of three.
template <int H>
__device__ __forceinline__ float fma_f16_f32(uint32_t a, uint32_t b, float acc) {
    const unsigned short x = (unsigned short)(H ? (a >> 16) : (a & 0xffffu));
    const unsigned short y = (unsigned short)(H ? (b >> 16) : (b & 0xffffu));
    asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(x), "h"(y));
    return acc;
}

// dot8 with the mixed-precision FMA: the same products in the same order,
// so the same bits.
__device__ __forceinline__ float dot8_mixed(const uint4& w, const uint4& x, float acc) {
    acc = fma_f16_f32<0>(w.x, x.x, acc); acc = fma_f16_f32<1>(w.x, x.x, acc);
    acc = fma_f16_f32<0>(w.y, x.y, acc); acc = fma_f16_f32<1>(w.y, x.y, acc);
    acc = fma_f16_f32<0>(w.z, x.z, acc); acc = fma_f16_f32<1>(w.z, x.z, acc);
    acc = fma_f16_f32<0>(w.w, x.w, acc); acc = fma_f16_f32<1>(w.w, x.w, acc);
    return acc;
}

// 8-element dot product of two packed half vectors, fp32 accumulation.
__device__ __forceinline__ float dot8(const uint4& w, const uint4& x, float acc) {
    float2 a, b;
    a = h2_to_f2(w.x); b = h2_to_f2(x.x); acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
    a = h2_to_f2(w.y); b = h2_to_f2(x.y); acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
    a = h2_to_f2(w.z); b = h2_to_f2(x.z); acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
    a = h2_to_f2(w.w); b = h2_to_f2(x.w); acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
    return acc;
}

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
    float2 t;
    t = h2_to_f2(v.x); f[0] = t.x; f[1] = t.y;
    t = h2_to_f2(v.y); f[2] = t.x; f[3] = t.y;
    t = h2_to_f2(v.z); f[4] = t.x; f[5] = t.y;
    t = h2_to_f2(v.w); f[6] = t.x; f[7] = t.y;
}

__device__ __forceinline__ uint4 pack8(const float* f) {
    uint4 v;
    v.x = f2_to_h2(f[0], f[1]);
    v.y = f2_to_h2(f[2], f[3]);
    v.z = f2_to_h2(f[4], f[5]);
    v.w = f2_to_h2(f[6], f[7]);
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; `red` must hold blockDim.x/32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
    return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : -3.0e38f;
    return warp_max(t);
}

// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// Packed (value, id) key for a 64-bit atomicMax argmax: larger value wins,
// ties go to the lower id.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t id) {
    return (static_cast<unsigned long long>(float_key(v)) << 32) | static_cast<uint32_t>(~id);
}
__device__ __forceinline__ uint32_t argmax_key_id(unsigned long long k) {
    return ~static_cast<uint32_t>(k & 0xffffffffull);
}

}  // namespace b2
