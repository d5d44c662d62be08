/*
 * rfsn_b200.h - C ABI of the B200 (sm_100a) exact segmented-attention path.
 *
 * The reference implementation (rfsn-MLX, package rfsn_v10_5) is pure Python
 * on MLX and exposes no foreign-function interface. These entry points are the
 * native operations behind its Python cache/attention API; each declaration
 * names the reference function (file:line) whose work it takes over. The
 * Python host package (rfsn-mlx_b200/rfsn_b200) binds them with ctypes.
 *
 * Conventions
 *   - Plain pointers and sizes only. Device pointers are marked "device";
 *     host pointers "host". `stream` is a cudaStream_t (NULL = legacy stream).
 *   - Every call returns an rfsn_status; 0 is success. On failure
 *     rfsn_last_error() returns a thread-local, human-readable message.
 *   - All launches are stream-ordered and asynchronous; nothing blocks the
 *     host except rfsn_event_wait and rfsn_workspace_check (both bounded).
 *   - Tensor layouts are row-major. A K or V "arena" is one layer's storage:
 *     [batch * kv_heads][rows][head_dim] in the cache dtype. Rows
 *     [ring_row0, ring_row0 + capacity) hold the hot ring buffer; the other
 *     rows hold archived blocks, each a contiguous run of rows per head.
 *   - Attention outputs are float32, [batch][q_heads][q_len][head_dim], the
 *     dtype the reference returns (q is float32 after RoPE promotion,
 *     layer.py:131-132, and run_segmented_attention casts to q.dtype,
 *     attention_exact.py:164).
 */
#ifndef RFSN_B200_H
#define RFSN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RFSN_ABI_VERSION 1

#if defined(__GNUC__)
#define RFSN_API __attribute__((visibility("default")))
#else
#define RFSN_API
#endif

typedef int rfsn_status;
#define RFSN_OK 0
#define RFSN_ERR_INVALID_ARG 1   /* bad shape / pointer / size (maps to ValueError) */
#define RFSN_ERR_UNSUPPORTED 2   /* shape or dtype this build does not handle */
#define RFSN_ERR_OVERFLOW 3      /* hot ring or workspace overflow (RuntimeError) */
#define RFSN_ERR_TIMEOUT 4       /* a bounded wait expired */
#define RFSN_ERR_CUDA 5          /* CUDA runtime error */
#define RFSN_ERR_DEVICE 6        /* a kernel reported an error in the workspace flag */

/* element types of K/V storage and of q/k/v inputs */
#define RFSN_F32 0
#define RFSN_F16 1
#define RFSN_BF16 2

/* Keys per attention tile. Page-table tile prefix sums are in these units. */
#define RFSN_TILE_KEYS 64

/* Every call returns an rfsn_status; on failure rfsn_last_error() describes it
 * (kept per calling thread). The Python layer raises the reference's
 * exception types for them: ValueError for bad arguments (config.py:88-129,
 * model.py:77-99), RuntimeError for ring or scratch overflow
 * (cache.py:345-375), TimeoutError for bounded waits. */
RFSN_API const char* rfsn_last_error(void);
RFSN_API int rfsn_abi_version(void);
/* Number of SMs of the current device (used to size split-KV grids). */
RFSN_API rfsn_status rfsn_device_sm_count(int* out);

/* ------------------------------------------------------------------------
 * Archived-block page table (device-resident).
 *
 * Replaces the reference's per-layer PageTable list walk
 * (block_manager.py:203-256, iterated by cache.py:413-423 on every attention
 * call) with a device int32 array: one record per attended archived block,
 * in logical order,
 *     {row, pos, len, tile_begin}
 * row        arena row of the block's first token
 * pos        absolute position of the block's first token (logical_start)
 * len        tokens in the block
 * tile_begin sum over previous blocks of ceil(len / RFSN_TILE_KEYS)
 * followed by one sentinel record whose tile_begin is the total tile count.
 * ---------------------------------------------------------------------- */
typedef struct rfsn_page_table {
    const int32_t* records;   /* device, (n_blocks + 1) * 4 int32 */
    int32_t n_blocks;
    int32_t archived_tokens;  /* sum of len */
    int32_t archived_tiles;   /* records[4 * n_blocks + 3] */
    int32_t reserved;
} rfsn_page_table;

/* Live hot window: cache.py:108-110 (hot_head_index, hot_seq_len, hot_start)
 * and its 1-2 physical pieces, cache.py:184-218. */
typedef struct rfsn_hot_window {
    int32_t ring_row0;    /* arena row of ring slot 0 */
    int32_t capacity;     /* hot_capacity */
    int32_t head_index;   /* hot_head_index */
    int32_t length;       /* hot_seq_len */
    int32_t start_pos;    /* hot_start */
    int32_t reserved;
    /* Optional device int32[RFSN_STEP_STATE_LEN] read by the kernel when it
     * runs (so one captured CUDA graph serves every decode step): the query
     * position replaces q_pos0 and the hot window replaces head_index / length
     * / start_pos (a context that turns out empty gives zero output and -inf
     * LSE instead of the argument error). NULL: the fields above are used.
     * See RFSN_STEP_*. */
    const int32_t* step_state;
} rfsn_hot_window;

/* Layout of a device step state (int32). */
#define RFSN_STEP_POS 0          /* absolute position of the first new token */
#define RFSN_STEP_WRITE_INDEX 1  /* ring slot the new tokens are written to */
#define RFSN_STEP_HEAD 2         /* hot_head_index after the append */
#define RFSN_STEP_LENGTH 3       /* hot_seq_len after the append */
#define RFSN_STEP_START 4        /* hot_start after the append */
#define RFSN_STEP_STATE_LEN 8

/* One K/V arena pair of a layer: the storage of the hot ring (hot_k / hot_v,
 * cache.py:100-107) and of the archived block arrays that _seal_hot_prefix
 * creates (cache.py:324-339), as rows of one buffer per K and V; holds the
 * TMA descriptors the decode kernel streams tiles with. Created once per cache layer. The first arena created
 * on a device also loads every kernel of the library there (none is then
 * loaded lazily at its first launch, in the middle of a decode step). */
typedef struct rfsn_arena rfsn_arena;

RFSN_API rfsn_status rfsn_arena_create(void* k_arena,      /* device */
                              void* v_arena,      /* device */
                              int dtype,          /* RFSN_F32 / F16 / BF16 */
                              int batch_kv_heads, /* batch * kv_heads */
                              int rows,           /* rows per head */
                              int head_dim,
                              rfsn_arena** out);
RFSN_API rfsn_status rfsn_arena_destroy(rfsn_arena* arena);

/* ------------------------------------------------------------------------
 * Fused RoPE + hot-ring append.
 *
 * Replaces layer.py:131-135: _apply_rope on q and k (layer.py:38-51) with the
 * float32 tables of build_rope_tables (layer.py:20-35), then
 * LayerKVCache.append_exact (cache.py:341-361): cast k, v to the cache dtype
 * and write them at ring slots (write_index + i) % capacity, splitting at the
 * end of the ring. q is written out rotated, in float32.
 *
 * q: [batch][q_heads][len][head_dim], k, v: [batch][kv_heads][len][head_dim],
 * contiguous, element type in_dtype (the model dtype). inv_freq: device
 * float32 [head_dim / 2], 1 / base ** (i / half) computed on the host exactly
 * as layer.py:29. If inv_freq is NULL no rotation is applied (plain
 * append_exact of already-rotated keys) and q / q_out may be NULL. If k and
 * v are NULL only q is rotated and nothing is written to the ring (ranks of a
 * sharded decode that do not own the hot window still need the rotated q).
 * The ring must have room: the caller runs the seal rule first
 * (evict_for_append, cache.py:363-383).
 * ---------------------------------------------------------------------- */
RFSN_API rfsn_status rfsn_rope_append(const void* q, const void* k, const void* v, int in_dtype,
                             const float* inv_freq, int pos0,
                             int batch, int q_heads, int kv_heads, int len, int head_dim,
                             float* q_out,
                             const rfsn_arena* arena, int ring_row0, int capacity, int write_index,
                             void* stream);

/* rfsn_rope_append with the position and ring write index read on the device
 * from step_state[RFSN_STEP_POS] and step_state[RFSN_STEP_WRITE_INDEX] when the
 * kernel runs (capturable once in a CUDA graph and replayed for every decode
 * step). k and v may be NULL to rotate q alone. q, k, v and step_state may be
 * page-locked host memory (read over the bus by the kernel; see
 * rfsn_host_device_pointer). step_state_copy (device int32[RFSN_STEP_STATE_LEN],
 * may be NULL) receives the step state, for a decode kernel that reads it from
 * device memory. No counterpart in the reference: it only moves two arguments
 * of layer.py:131-135 into device memory. */
RFSN_API rfsn_status rfsn_rope_append_step(const void* q, const void* k, const void* v, int in_dtype,
                                           const float* inv_freq, const int32_t* step_state,
                                           int32_t* step_state_copy, int batch, int q_heads, int kv_heads, int len,
                                           int head_dim, float* q_out, const rfsn_arena* arena, int ring_row0,
                                           int capacity, void* stream);

/* RoPE from explicit cos/sin tables, fused with the append
 * (layer.py:118-135 for a layer called with rope_tables, or without them,
 * when the layer builds its tables in the model dtype, layer.py:118-126).
 * cos_t / sin_t: device [len][head_dim] in tab_dtype, row l for position
 * pos0 + l; both NULL to build them from inv_freq (float32 products and
 * cos/sin, rounded to tab_dtype: build_rope_tables with dtype = tab_dtype).
 * Every product and sum is rounded to the promoted dtype of in_dtype and
 * tab_dtype (the 16-bit type when both are it, else float32), as the
 * reference's elementwise ops round each result. q_out (float32) holds the
 * rotated q; the rotated k and v go to ring slots write_index.. like
 * rfsn_rope_append. */
RFSN_API rfsn_status rfsn_rope_append_tables(const void* q, const void* k, const void* v, int in_dtype,
                                             const void* cos_t, const void* sin_t, int tab_dtype,
                                             const float* inv_freq, int pos0, int batch, int q_heads,
                                             int kv_heads, int len, int head_dim, float* q_out,
                                             const rfsn_arena* arena, int ring_row0, int capacity,
                                             int write_index, void* stream);

/* ------------------------------------------------------------------------
 * Dense-layer helpers of the model driver (not on the attention path).
 *
 * RMSNorm (layer.py:54-64): out = weight * x / sqrt(mean(x^2) + eps) per row
 * of n elements, in float32, rounded to dtype once; x, weight and out share
 * the dtype (RFSN_F32 / F16 / BF16), rows are contiguous. With residual
 * (and sum_out) non-NULL the row is first s = x + residual rounded to dtype,
 * written to sum_out, and s is normalised (16-byte aligned rows of at most
 * 1024 16-byte vectors). */
RFSN_API rfsn_status rfsn_rms_norm(const void* x, const void* residual, const void* weight, void* sum_out, void* out,
                                   int rows, int n, int dtype, float eps, void* stream);

/* SwiGLU on a fused gate|up projection (layer.py:94-95): gate_up rows hold
 * [gate (n), up (n)]; out[r, c] = silu(gate[r, c]) * up[r, c], silu rounded to
 * dtype first, the product in float32 rounded once. */
RFSN_API rfsn_status rfsn_silu_mul(const void* gate_up, void* out, int rows, int n, int dtype, void* stream);

/* y[r, n] = sum_k weight[n, k] * x[r, k] for rows = 1..4 rows of x (a decode
 * token's q|k|v, o, gate|up or down projection, layer.py:82-89; weight
 * [n_out, k] row-major, 16-byte aligned rows),
 * float32 accumulation, y [rows, n_out] rounded to dtype once. */
RFSN_API rfsn_status rfsn_gemv(const void* weight, const void* x, void* y, int n_out, int k, int rows, int dtype,
                               void* stream);

/* Launch plan of a tensor-core prefill call of this shape (rfsn_paged_attention
 * with q_len >= 64, bf16/f16 K/V, head_dim 128): the units (query block of
 * 128 / (q_heads / kv_heads) positions x KV head) are launched in bands of KV
 * heads whose K/V fits 40 MB of L2 (all heads in one band for short contexts),
 * longest causal range first inside a band; the first *cta_units_whole run
 * whole, each later one is split
 * into *tail_splits key ranges whose last CTA merges them; *ctas CTAs in all.
 * Host-only (uses the current device's SM count, 148 without a device). */
RFSN_API rfsn_status rfsn_prefill_plan(int batch, int q_heads, int kv_heads, int q_len, int q_pos0,
                                       int archived_tokens, int hot_start, int hot_length, int* cta_units_whole,
                                       int* tail_splits, int* ctas);

/* Device address of page-locked host memory (the same value under unified
 * addressing), for kernels that read their inputs or write their outputs
 * across the bus instead of through copy operations. RFSN_ERR_INVALID_ARG when
 * host_ptr is not page-locked memory mapped for the current device. */
RFSN_API rfsn_status rfsn_host_device_pointer(const void* host_ptr, void** device_ptr);

/* ------------------------------------------------------------------------
 * Copy rows inside an arena (both K and V, every batch*kv head).
 *
 * Seal: _seal_hot_prefix / _materialize_hot_span (cache.py:324-339,
 * :220-234) copy the ring's oldest `count` tokens (logical offset 0 = slot
 * head_index, wrapping at capacity) into a fresh block. Here the block is a
 * run of arena rows: src rows are read modulo src_wrap (pass 0 for no wrap),
 * starting at src_row0 + src_offset; dst rows are dst_row0 .. + count.
 * ---------------------------------------------------------------------- */
RFSN_API rfsn_status rfsn_arena_copy_rows(const rfsn_arena* arena,
                                 int src_row0, int src_offset, int src_wrap,
                                 int dst_row0, int count, void* stream);

/* ------------------------------------------------------------------------
 * Block transfer between an arena and a host (pinned) or device buffer laid
 * out [batch*kv_heads][count][head_dim] (the reference's per-block payload
 * shape, cache.py:240). Used by the warm tier: demotion (to host) and the
 * prefetch/sync load back (residency.py:85-145, cache.py:385-408). Issued with
 * cudaMemcpy2DAsync on `stream`; if `done_event` is non-NULL it is recorded
 * after the copies.
 * ---------------------------------------------------------------------- */
RFSN_API rfsn_status rfsn_block_upload(const rfsn_arena* arena, int dst_row0, int count,
                              const void* k_src, const void* v_src,
                              void* stream, void* done_event);
RFSN_API rfsn_status rfsn_block_download(const rfsn_arena* arena, int src_row0, int count,
                                void* k_dst, void* v_dst,
                                void* stream, void* done_event);

/* Bounded wait on a CUDA event: polls cudaEventQuery until it completes or
 * timeout_us elapses (RFSN_ERR_TIMEOUT). Mirrors the reference's
 * wait_for_prefetches(timeout=1.0) (residency.py:147-150). */
RFSN_API rfsn_status rfsn_event_wait(void* event, int64_t timeout_us);

/* ------------------------------------------------------------------------
 * Exact attention of q against the archived blocks of a page table plus the
 * live hot window, all in one arena.
 *
 * Replaces the per-step segment walk + GQA expansion + segmented attention of
 * layer.py:139-162 -> cache.get_attention_segments (cache.py:425-428),
 * mx.repeat (layer.py:140-150), run_segmented_attention / exact_attention
 * (attention_exact.py:111-164). Semantics: scaled dot products
 * (scale 1/sqrt(head_dim)), causal by absolute position (key pos <= query
 * pos, attention_exact.py:27-61), one softmax over every segment, float32
 * accumulation. Query head h reads KV head h / (q_heads / kv_heads). A query
 * row that sees no key at all (every key after it) gets zeros and LSE -inf;
 * the reference's additive -1e9 mask gives such a row the softmax of the
 * masked scores instead. Decode and prefill never produce such a row: a
 * query always sees its own key.
 *
 * q: device float32 [batch][q_heads][q_len][head_dim]; query row r sits at
 * absolute position q_pos0 + r. out: device float32, same shape. lse
 * (optional, may be NULL): device float32 [batch][q_heads][q_len], the
 * natural-log log-sum-exp of the scaled logits (what the cross-GPU merge
 * needs).
 *
 * Work is split over the keys (split-KV): bf16/f16 arenas with head_dim 128
 * and q_len * (q_heads / kv_heads) <= 4 stream tiles with TMA and reduce on
 * tensor cores with float32-accurate split operands; other shapes run a
 * CUDA-core kernel. Both merge their splits in-kernel.
 *
 * workspace: device scratch of rfsn_attention_workspace_size() bytes, zeroed
 * once before its first use (the kernels leave it zeroed). Calls that share a
 * workspace must be ordered on one stream.
 * ---------------------------------------------------------------------- */
RFSN_API rfsn_status rfsn_attention_workspace_size(int batch, int q_heads, int kv_heads, int q_len,
                                          int head_dim, int max_splits, size_t* bytes);

RFSN_API rfsn_status rfsn_paged_attention(const rfsn_arena* arena,
                                 const float* q, int batch, int q_heads, int kv_heads,
                                 int q_len, int q_pos0,
                                 const rfsn_page_table* table,
                                 const rfsn_hot_window* hot,
                                 float* out, float* lse,
                                 void* workspace, size_t workspace_bytes,
                                 int max_splits, /* 0 = choose from the SM count */
                                 void* stream);

/* ------------------------------------------------------------------------
 * Exact segmented attention over an arbitrary list of K/V segments
 * (run_segmented_attention, attention_exact.py:122-164, and the single
 * segment exact path, :64-108, for tensors that do not live in an arena).
 *
 * segments: device array of n_segments descriptors (below), in the order the
 * caller lists them; each segment is [batch][kv_heads][len][head_dim] with
 * the given element strides (innermost stride must be 1).
 * ---------------------------------------------------------------------- */
typedef struct rfsn_segment_desc {
    uint64_t k_ptr;         /* device address of element [0][0][0][0] */
    uint64_t v_ptr;
    int64_t k_stride_b, k_stride_h, k_stride_t;
    int64_t v_stride_b, v_stride_h, v_stride_t;
    int32_t pos;            /* absolute position of the segment's first key */
    int32_t len;            /* keys in the segment (> 0) */
    int32_t tile_begin;     /* sum over previous segments of ceil(len / RFSN_TILE_KEYS) */
    int32_t reserved;
} rfsn_segment_desc;

RFSN_API rfsn_status rfsn_segmented_attention(const float* q, int batch, int q_heads, int kv_heads,
                                     int q_len, int q_pos0, int head_dim, int kv_dtype,
                                     const rfsn_segment_desc* segments, /* device */
                                     int n_segments, int total_tiles,
                                     float* out, float* lse,
                                     void* workspace, size_t workspace_bytes,
                                     int max_splits, void* stream);

/* ------------------------------------------------------------------------
 * Log-sum-exp merge of attention results over disjoint key sets (the
 * associative form of the global-max merge, attention_exact.py:141-164).
 * Used after the cross-GPU gather of sharded decode: parts_out
 * [n_parts][rows][head_dim], parts_lse [n_parts][rows] (natural log),
 * out [rows][head_dim], lse_out [rows] (may be NULL). A part whose lse is
 * -inf (it saw no visible key) contributes nothing.
 * ---------------------------------------------------------------------- */
RFSN_API rfsn_status rfsn_lse_merge(const float* parts_out, const float* parts_lse,
                           int n_parts, int rows, int head_dim,
                           float* out, float* lse_out, void* stream);

/* ------------------------------------------------------------------------
 * Paged attention without any device allocation. No counterpart in the
 * reference (which has no native interface); this is a variant of
 * rfsn_paged_attention for callers that cannot allocate device memory when
 * they run attention (engines that own all device memory through their own
 * pool, frozen memory budgets, plugin hosts that only pass inputs and
 * outputs). Same arguments and results as rfsn_paged_attention, minus the
 * workspace: the split scratch lives in one built-in device array of
 * RFSN_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
 * the process exits. Calls sharing a device share the array; calls that
 * overlap on the GPU race and must be ordered by the caller. Shapes whose
 * split scratch does not fit are rejected with RFSN_ERR_OVERFLOW (lower
 * max_splits, or use rfsn_paged_attention); a rejected call issues no CUDA
 * work. The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) and should be made before any stream capture.
 * Kernel-side failures (an expired bounded wait, a page-table record outside
 * the arena) set the array's error word, which stays set until
 * rfsn_noalloc_check reads it.
 * ---------------------------------------------------------------------- */
#define RFSN_NOALLOC_SCRATCH_BYTES (8u << 20)

RFSN_API rfsn_status rfsn_paged_attention_noalloc(const rfsn_arena* arena,
                                         const float* q, int batch, int q_heads, int kv_heads,
                                         int q_len, int q_pos0,
                                         const rfsn_page_table* table,
                                         const rfsn_hot_window* hot,
                                         float* out, float* lse,
                                         int max_splits, void* stream);

/* Error check of rfsn_paged_attention_noalloc on the current device (no
 * counterpart in the reference): waits for `stream` (bounded by timeout_us),
 * then reads and clears the built-in array's error word, with the statuses of
 * rfsn_workspace_check (RFSN_ERR_TIMEOUT for an expired wait, RFSN_ERR_DEVICE
 * for a record outside the arena). Allocates no device memory. */
RFSN_API rfsn_status rfsn_noalloc_check(void* stream, int64_t timeout_us);

/* Number of kernels this library has launched in the process so far
 * (instrumentation: lets callers count native launches in a timed region). */
RFSN_API uint64_t rfsn_launch_count(void);

/* ------------------------------------------------------------------------
 * Sharded decode with the cross-GPU merge fused into the attention kernel.
 *
 * The reference has no multi-GPU path. For a context whose archived blocks
 * are partitioned over the GPUs of one node (one process per GPU), each rank
 * attends over its own blocks; the last CTA of every KV head then stores its
 * (output, LSE) into every rank's mailbox over NVLink and merges the parts of
 * all ranks in rank order (the merge of attention_exact.py:141-164), so every
 * rank ends with the full result after one kernel, without a collective
 * library call. Waits for peers are bounded (rfsn_peer_group_set_timeout,
 * default 2 s) and report RFSN_ERR_TIMEOUT through rfsn_workspace_check.
 * After a peer wait has expired the group is unusable: its later calls skip
 * the exchange, write this rank's local result and report RFSN_ERR_TIMEOUT
 * again (the ranks' call stamps no longer agree), until every rank destroys
 * the group and creates a new one.
 *
 * Set-up per rank: rfsn_peer_group_create (allocates the mailbox on the
 * current device and writes its CUDA IPC handle, rfsn_peer_ipc_handle_bytes()
 * bytes), exchange the handles (e.g. an all-gather), then
 * rfsn_peer_group_connect with all handles in rank order. Every rank must make
 * the same sequence of rfsn_paged_attention_peer calls.
 * ---------------------------------------------------------------------- */
typedef struct rfsn_peer_group rfsn_peer_group;

RFSN_API int rfsn_peer_ipc_handle_bytes(void);
RFSN_API rfsn_status rfsn_peer_group_create(int world, int rank, int groups, int head_dim,
                                            rfsn_peer_group** out, void* ipc_handle_out);
RFSN_API rfsn_status rfsn_peer_group_connect(rfsn_peer_group* group, const void* all_handles);
RFSN_API rfsn_status rfsn_peer_group_set_timeout(rfsn_peer_group* group, int64_t timeout_us);
RFSN_API rfsn_status rfsn_peer_group_destroy(rfsn_peer_group* group);
RFSN_API rfsn_status rfsn_paged_attention_peer(const rfsn_arena* arena,
                                               const float* q, int batch, int q_heads, int kv_heads,
                                               int q_len, int q_pos0,
                                               const rfsn_page_table* table,
                                               const rfsn_hot_window* hot,
                                               rfsn_peer_group* peers,
                                               float* out, float* lse,
                                               void* workspace, size_t workspace_bytes,
                                               int max_splits, void* stream);

/* Reads the device error word of a workspace (after synchronising `stream`,
 * bounded by timeout_us) and clears it. RFSN_ERR_DEVICE if a kernel set it. */
RFSN_API rfsn_status rfsn_workspace_check(void* workspace, void* stream, int64_t timeout_us);

#ifdef __cplusplus
}
#endif

#endif /* RFSN_B200_H */
