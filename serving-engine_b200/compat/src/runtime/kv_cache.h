// compat/src/runtime/kv_cache.h -- the reference's KVCache container and
// cuda::append_kv_cache (src/runtime/kv_cache.h:12-91) for callers that keep
// their own single-sequence cache: layout [layer][K=0,V=1][kv_head][max_seq]
// [head_dim] half, storage in the reference's DeviceBuffer; the append runs
// b2_append_kv_cache.  (The b2engine model runtime keeps its own batched
// cache, [layer][batch][K,V][kv_head][max_seq][head_dim].)
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "src/b2_compat.h"
#include "src/common/cuda_utils.h"

namespace engine {

class KVCache {
public:
    KVCache() = default;
    KVCache(int num_layers, int num_kv_heads, int head_dim, int max_seq) {
        allocate(num_layers, num_kv_heads, head_dim, max_seq);
    }

    void allocate(int num_layers, int num_kv_heads, int head_dim, int max_seq) {
        layers_ = num_layers;
        heads_ = num_kv_heads;
        dim_ = head_dim;
        max_seq_ = max_seq;
        data_.allocate((size_t)layers_ * 2 * heads_ * max_seq_ * dim_);
        data_.zero();
        len_ = 0;
    }

    half* get_layer_ptr(int layer, int is_v) { return data_.data() + slab(layer, is_v, 0); }
    const half* get_layer_ptr(int layer, int is_v) const { return data_.data() + slab(layer, is_v, 0); }
    half* get_head_ptr(int layer, int is_v, int kv_head) { return data_.data() + slab(layer, is_v, kv_head); }
    const half* get_head_ptr(int layer, int is_v, int kv_head) const {
        return data_.data() + slab(layer, is_v, kv_head);
    }

    int num_layers() const { return layers_; }
    int num_kv_heads() const { return heads_; }
    int head_dim() const { return dim_; }
    int max_seq() const { return max_seq_; }
    int current_seq_len() const { return len_; }
    void set_current_seq_len(int len) { len_ = len; }

    half* raw_data() { return data_.data(); }
    const half* raw_data() const { return data_.data(); }

private:
    size_t slab(int layer, int is_v, int kv_head) const {
        return (((size_t)layer * 2 + is_v) * heads_ + kv_head) * max_seq_ * dim_;
    }

    int layers_ = 0, heads_ = 0, dim_ = 0, max_seq_ = 0, len_ = 0;
    DeviceBuffer<half> data_;
};

namespace cuda {

inline void append_kv_cache(const half* src_k, const half* src_v, half* dst_k_head_base, half* dst_v_head_base,
                            int num_tokens, int start_pos, int num_kv_heads, int max_seq, int head_dim,
                            cudaStream_t stream = 0) {
    b2_check(b2_append_kv_cache(src_k, src_v, dst_k_head_base, dst_v_head_base, num_tokens, start_pos, num_kv_heads,
                                max_seq, head_dim, stream),
             "append_kv_cache");
}

}  // namespace cuda
}  // namespace engine
