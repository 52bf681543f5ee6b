// attention.cuh -- launchers of the cluster-merged decode attention kernels
// (attention_cl.cu: CUDA-core form; attention_tc.cu: tcgen05 form, dense
// and paged caches).
#pragma once

#include "common.cuh"

namespace b2 {

// q [B] rows q_sb apart, out [B] rows o_sb apart, K/V views (sb, sh, ss)
// covering max_len positions; lengths from seq_lens (or len_const when it is
// null).  early_kv: K/V tiles are fetched before the programmatic-launch
// wait (the decode step, where only the newest row is still being written).
// lean: fewer ring stages, for callers that run register-streaming GEMVs
// around the attention.
// B2_ERR_UNSUPPORTED when the shape fits neither kernel.
int attn_cl_launch(const __half* q, int64_t q_sb, __half* out, int64_t o_sb, const __half* k, const __half* v,
                   int64_t sb, int64_t sh, int64_t ss, int max_len, const int* seq_lens, int len_const, int B,
                   int nq, int nkv, int D, int early_kv, int lean, TraceSlot trace, cudaStream_t s, bool pdl);

// The tensor-core form alone (head_dim 128, group <= 8 per head group).
int attn_tc_launch(const __half* q, int64_t q_sb, __half* out, int64_t o_sb, const __half* k, const __half* v,
                   int64_t sb, int64_t sh, int64_t ss, int max_len, const int* seq_lens, int len_const, int B,
                   int nq, int nkv, int D, int early_kv, int lean, TraceSlot trace, cudaStream_t s, bool pdl);

// Paged form: K / V pools [num_blocks][bs][nkv][128], block tables [B][maxb]
// (bs a multiple of 8 dividing 128), sequence lengths seq_lens[B] <= max_len.
int attn_tc_launch_paged(const __half* q, int64_t q_sb, __half* out, int64_t o_sb, const __half* kpool,
                         const __half* vpool, int num_blocks, int bs, const int* bt, int maxb, int max_len,
                         const int* seq_lens, int B, int nq, int nkv, int D, int early_kv, int lean, TraceSlot trace,
                         cudaStream_t s, bool pdl);

}  // namespace b2
