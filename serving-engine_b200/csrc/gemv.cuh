// gemv.cuh -- parameters of the decode GEMV family (shared by gemv.cu and the
// model runtime).
#pragma once

#include "common.cuh"

namespace b2 {

// How the activation vector x is produced in the CTA prologue.
enum XMode : int {
    X_HALF = 0,  // x is half [B, ldx] written by the previous kernel
    X_NORM = 1,  // x = half(h * rsqrt(mean(h^2) + eps) * norm_w), h float [B, ldx]
    X_SUM = 2,   // as X_NORM with h = hid_in + the partial rows every tensor-parallel
                 // rank pushed (waits for their flags); CTA 0 stores h to hid_out
};

// What the epilogue does with the fp32 dot products of a warp task.
enum OutMode : int {
    OUT_HALF = 0,    // y half [B, ldy] (+bias / +residual)
    OUT_F32 = 1,     // y float [B, ldy] (+bias / +residual)
    OUT_RESID = 2,   // hidden float [B, ldy]: y = dot + (resid_add ? y : 0)
    OUT_QKV = 3,     // fused q|k|v rows, rotate-half RoPE, K/V into the cache
    OUT_SWIGLU = 4,  // act half [B, ldy] = silu(dot(Wg)) * dot(Wu)
    OUT_LOGITS = 5,  // logits float [B, ldy] and a packed argmax per sequence
    OUT_PUSH = 6,    // fp32 partial rows pushed into every tensor-parallel rank's
                     // receive slots, then one flag per rank (row-parallel o / down)
};

constexpr int kMaxTp = 8;

// One-shot all-reduce of the row-parallel projections over peer memory.
// Rank r's fp32 partial [B, H] goes into slot [parity][r] of every rank's
// receive buffer as 8-byte words, value in the low half and the exchange's
// epoch in the high half, written with single 8-byte stores over NVLink: a
// word is valid once its tag equals the epoch, so the producer needs no
// fence or flag and the consumer polls each word it needs (bounded).  The
// consumer sums the tp slots in rank order (identical arithmetic on every
// rank).  The epoch of exchange `slot` of decode step s is
// s * nslots + slot + 1 and its parity picks one of two buffers: no rank can
// push exchange e + 2 before every rank has consumed exchange e.
// The lm_head's argmax (64-bit keys) is exchanged with one flag per rank.
struct TpExchange {
    int tp, rank, Bmax, H;
    unsigned long long* recv;              // this rank's words [2][tp][Bmax][H]
    unsigned long long* peer_recv[kMaxTp]; // every rank's word buffer (own included)
    unsigned long long* am_recv;           // this rank's argmax slots [tp][Bmax]
    unsigned* am_flags;                    // [tp], set to step + 1
    unsigned long long* peer_am_recv[kMaxTp];
    unsigned* peer_am_flags[kMaxTp];
    int* step;                             // decode steps completed (device)
    int* ctr;                              // arrival counter of the lm_head
    int* err;                              // bounded-wait error word
};

// (value, tag) word of the exchange
__device__ __forceinline__ unsigned long long ll_word(float v, unsigned tag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
}

__device__ __forceinline__ void ll_store2(unsigned long long* dst, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a), "l"(b) : "memory");
}

// Two consecutive words once both carry `tag` (bounded poll); values in v.
__device__ __forceinline__ bool ll_load2(const unsigned long long* src, unsigned tag, float2& v, int* err, int where) {
    unsigned long long a, b;
    const long long t0 = clock64();
    for (unsigned i = 0;; ++i) {
        asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
        if ((unsigned)(a >> 32) == tag && (unsigned)(b >> 32) == tag) break;
        if (i >= 4) __nanosleep(32);
        if ((i & 63u) == 63u) {
            if (*reinterpret_cast<volatile int*>(err) != 0 || clock64() - t0 > 2000000000ll) {
                atomicCAS(err, 0, where);
                v = make_float2(0.f, 0.f);
                return false;
            }
        }
    }
    v = make_float2(__uint_as_float((unsigned)a), __uint_as_float((unsigned)b));
    return true;
}

struct GemvParams {
    const __half* W;   // [rows, K] row-major
    const __half* W2;  // OUT_SWIGLU: up-projection rows
    int K;
    int tasks;  // warp tasks: rows (R=1) or row pairs (R=2)
    int B;      // sequences in this launch (<= the batch tile)

    const void* x;  // half or float [B, ldx]
    int64_t ldx;
    const __half* norm_w;
    float eps;

    const __half* bias;   // [rows] or null
    const __half* resid;  // half residual [B, ld_resid] or null (OUT_HALF/OUT_F32)
    int64_t ld_resid;
    int resid_add;        // OUT_RESID: 1 adds the existing y (residual stream)
    void* y;
    int64_t ldy;

    // OUT_QKV
    int nq, nkv, D;
    const float2* rope;  // [max_pos, D/2] (cos, sin)
    const int* pos;      // [B] positions of the new token
    KvLayout kv;         // this layer's K / V rows

    // OUT_LOGITS
    unsigned long long* argmax;  // [B] packed (value, id), 0 before the launch
    int row_offset;              // global id of local row 0 (vocabulary shard)
    int argmax_limit;            // global ids >= limit are not candidates

    // X_SUM / OUT_PUSH / argmax push (tensor parallelism over peer memory)
    int tp_on;                   // 1: the exchange below is live
    TpExchange tpx;
    int slot, nslots;            // this exchange's index in the step
    const float* hid_in;         // X_SUM: residual stream before the exchange
    float* hid_out;              // X_SUM: residual stream after it
    int rows_per_cta;            // OUT_PUSH: contiguous block of rows per CTA (set at launch)
    TraceSlot trace;             // step trace (buf null: off)

    // FP8 weights (a quantised model's decode GEMVs): W8 / W8b are [rows][K]
    // e4m3 codes with one fp32 scale per row (wsc / wsc2).  When W8 is set
    // they stand in for W / W2, and each row's dot product is multiplied by
    // its scale before the epilogue.  K % 16 == 0.
    const uint8_t* W8;
    const uint8_t* W8b;
    const float* wsc;
    const float* wsc2;
    // w4 = 1: W8 / W8b hold 4-bit weights instead ([rows][K/2] bytes, the
    // layout of kI4Group below) and wsc / wsc2 one fp32 scale per 128
    // weights ([rows][K/128]), applied to each group's partial dot product.
    // K % 128 == 0; batch tiles of 1 and 2.
    int w4;
};

// 4-bit weights (b2_quantize_int4_rows): per group of 128 consecutive
// weights of a row, scale = max|w| / 7 (fp32 division; 0 for an all-zero
// group) and q = rint(w / scale) in [-7, 7], stored as q + 8.  A row is K/2
// bytes; each 32-bit word holds 8 consecutive weights, weight j of the word
// at bit 16*(j & 1) + 4*(j >> 1), so (word >> 4p) & 0x000F000F is the pair
// (2p, 2p + 1) as the low bits of two halves.
constexpr int kI4Group = 128;

constexpr int kPushRows = 128;   // OUT_PUSH rows per CTA at most

// Bounded poll until *flag >= v (wrap-safe); false (and *err set) when it gives up.
__device__ __forceinline__ bool wait_flag_geq(const unsigned* flag, unsigned v, int* err, int where) {
    const long long t0 = clock64();
    for (unsigned i = 0;; ++i) {
        unsigned x;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(x) : "l"(flag) : "memory");
        if ((int)(x - v) >= 0) return true;
        if (i >= 8) __nanosleep(32);
        if ((i & 63u) == 63u) {
            if (*reinterpret_cast<volatile int*>(err) != 0) return false;
            if (clock64() - t0 > 2000000000ll) {
                atomicCAS(err, 0, where);
                return false;
            }
        }
    }
}

// Release fence at system scope: the calling thread's prior writes, and those
// of the CTA that a preceding __syncthreads ordered before it, become visible
// to other GPUs before its later writes.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void store_release_sys(unsigned* flag, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

// Launch the vectorised GEMV.  Requires K % 8 == 0 and 16-byte aligned W,
// W2, x rows; returns B2_ERR_UNSUPPORTED otherwise.  B <= 8 per launch.
int gemv_launch(const GemvParams& p, XMode xm, OutMode om, cudaStream_t s, bool pdl);

// Maximum batch tile handled by one gemv_launch for row length K.
int gemv_batch_tile(int K);

// Per-row FP8 (E4M3) quantisation of a half matrix [rows][K] (quant.cu).
int quantize_e4m3_rows(const __half* w, int64_t rows, int K, uint8_t* q, float* scales, cudaStream_t s);
// 4-bit codes [rows][K/2] and group scales [rows][K/128] (layout: kI4Group)
int quantize_i4_rows(const __half* w, int64_t rows, int K, uint8_t* q, float* scales, cudaStream_t s);

}  // namespace b2
