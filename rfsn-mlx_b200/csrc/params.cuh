// Kernel parameter blocks and host launchers shared between the kernel
// translation units and the C ABI layer (capi.cu).
#pragma once

#include "common.cuh"

// One layer's K/V arena and its TMA descriptors (opaque to C ABI users).
struct rfsn_arena {
    void* k;
    void* v;
    int dtype;
    int groups;
    int rows;
    int head_dim;
    int device;
    bool has_tma;
    CUtensorMap maps[4];  // K 64-row box, V 64-row box, K 8-row box, V 8-row box
};

namespace rfsn {
namespace fast {
struct Params {
    const float* q;
    float* out;
    float* lse;
    const int4* records;
    int n_blocks, archived_tiles;
    int ring_row0, capacity, head, hlen, hstart;
    int rows;                 // arena rows per head
    int q_heads, kv_heads, q_len, q_pos0, groups_per_kv, nslots;
    int total_tiles, tiles_per_split, splits, groups;
    float qscale;             // 1/sqrt(D) * log2(e)
    float pscale;             // power-of-two scale applied to p before the 16-bit split
    WsView ws;
    PeerParams peer;          // world == 0: local result only
    const int* dyn;           // device step state (RFSN_STEP_*) or nullptr
};
}  // namespace fast

// Chunked-prefill tensor-core kernel (prefill_attn.cu).
struct PrefillParams {
    const float* q;
    float* out;
    float* lse;
    const int4* records;
    int n_blocks;
    int ring_row0, capacity, head, hlen, hstart;
    int rows;                 // arena rows per head
    int batch, q_heads, kv_heads, q_len, q_pos0, groups_per_kv;
    float qscale;             // 1/sqrt(D) * log2(e)
    int nqb;                  // query blocks per KV head
    int full_units;           // units (query block, KV head) run whole, in launch order
    int tail_splits;          // key ranges each later unit is split into (1: none)
    int head_group;           // KV heads whose units are interleaved per band of the launch order
    WsView ws;                // error word; with split units also counters and partial (O, LSE)
};

namespace generic {
struct Params {
    const float* q;
    float* out;
    float* lse;
    int head_dim, q_heads, kv_heads, q_len, q_pos0, groups_per_kv, nslots_total, slots_ws;
    int total_tiles, tiles_per_split, splits, qblocks;
    float qscale;
    WsView ws;
    // paged mode
    const void* arena_k;
    const void* arena_v;
    int rows;
    const int4* records;
    int n_blocks, archived_tiles;
    int ring_row0, capacity, head, hlen, hstart;
    // segment-list mode
    const rfsn_segment_desc* segs;
    int n_segs;
};
}  // namespace generic

// decode_attn.cu
int fast_max_splits();
rfsn_status fast_launch(int dtype, const CUtensorMap* maps, const fast::Params& p, int stages, cudaStream_t stream);
// generic_attn.cu
rfsn_status generic_launch(int dtype, bool paged, const generic::Params& p, int groups, cudaStream_t stream);
// capi.cu: shared body of the paged-attention entry points (peer may be NULL)
rfsn_status paged_attention_impl(const rfsn_arena* arena, const float* q, int batch, int q_heads, int kv_heads,
                                 int q_len, int q_pos0, const rfsn_page_table* table, const rfsn_hot_window* hot,
                                 float* out, float* lse, void* workspace, size_t workspace_bytes, int max_splits,
                                 const PeerParams* peer, cudaStream_t stream, bool dry_run = false);
// dry_run: every argument check, the kernel choice and the workspace sizing of
// a real call, then return without launching (status as the call would give).
// prefill_attn.cu
rfsn_status prefill_launch(int dtype, const CUtensorMap* maps, const PrefillParams& p, cudaStream_t stream);
// merge.cu
rfsn_status lse_merge_launch(const float* parts_out, const float* parts_lse, int n_parts, int rows, int head_dim,
                             float* out, float* lse_out, cudaStream_t stream);
// ring.cu
rfsn_status rope_append_launch(int dtype, const void* q, const void* k, const void* v, const float* inv_freq, int pos0,
                               int batch, int q_heads, int kv_heads, int len, int head_dim, float* q_out, void* ak,
                               void* av, int rows, int ring_row0, int capacity, int write_index, cudaStream_t stream,
                               const int* step_state = nullptr, int* step_state_copy = nullptr);
rfsn_status rope_tables_append_launch(int dtype, int tab_dtype, const void* q, const void* k, const void* v,
                                      const void* cos_t, const void* sin_t, const float* inv_freq, int pos0,
                                      int batch, int q_heads, int kv_heads, int len, int head_dim, float* q_out,
                                      void* ak, void* av, int rows, int ring_row0, int capacity, int write_index,
                                      cudaStream_t stream);
rfsn_status copy_rows_launch(void* ak, void* av, int groups, int rows, int row_bytes, int src_row0, int src_offset,
                             int src_wrap, int dst_row0, int count, cudaStream_t stream);

// Load every kernel of the library on the current device now (under lazy
// module loading a kernel is otherwise loaded at its first launch, which can
// stall a decode step by milliseconds, e.g. at the first seal copy).
void preload_fast_kernels();
void preload_generic_kernels();
void preload_ring_kernels();
void preload_merge_kernels();
void preload_prefill_kernels();
void preload_model_kernels();

rfsn_status rms_norm_dispatch(int dtype, const void* x, const void* res, const void* w, void* s_out, void* y, int rows,
                              int n, float eps, cudaStream_t s);
rfsn_status silu_mul_dispatch(int dtype, const void* gu, void* y, int rows, int n, cudaStream_t s);
rfsn_status gemv_dispatch(int dtype, const void* w, const void* x, void* y, int N, int K, int xrows, cudaStream_t s);
int gemv_max_rows();

}  // namespace rfsn
