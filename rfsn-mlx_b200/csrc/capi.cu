// C ABI entry points (include/rfsn_b200.h): argument checking, kernel
// selection, split-KV sizing, TMA descriptor management and the small
// utility kernels (row copies are in ring.cu, attention in *_attn.cu).
#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <functional>
#include <map>
#include <mutex>
#include <vector>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>

#include "attn_common.cuh"
#include "params.cuh"

namespace rfsn {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

rfsn_status cuda_status(cudaError_t e, const char* what) {
    set_error("%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return RFSN_ERR_CUDA;
}

}  // namespace rfsn



using namespace rfsn;


namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        }
    }
    return fn;
}

rfsn_status encode_map(CUtensorMap* map, void* base, int dtype, int groups, int rows, int head_dim, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) {
        set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
        return RFSN_ERR_CUDA;
    }
    const int es = dtype_size(dtype);
    cuuint64_t gdim[2] = {(cuuint64_t)head_dim, (cuuint64_t)groups * (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)head_dim * es};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = fn(map, dtype == RFSN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base,
                    gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed with CUresult %d", (int)r);
        return RFSN_ERR_CUDA;
    }
    return RFSN_OK;
}

int sm_count_cached() {
    int dev = 0;
    cudaGetDevice(&dev);
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

bool valid_dtype(int dt) { return dt == RFSN_F32 || dt == RFSN_F16 || dt == RFSN_BF16; }

// Split-KV sizing: `target` CTAs in total, at most max_splits per group, at
// least one tile per split; returns splits and tiles per split.
void choose_splits(int total_tiles, int groups_x_qblocks, int target, int max_splits, int* splits, int* tps) {
    int s = target / (groups_x_qblocks > 0 ? groups_x_qblocks : 1);
    if (s < 1) s = 1;
    if (s > max_splits) s = max_splits;
    if (s > total_tiles) s = total_tiles;
    if (s < 1) s = 1;
    int per = (total_tiles + s - 1) / s;
    if (per < 1) per = 1;
    *tps = per;
    *splits = (total_tiles + per - 1) / per;
    if (*splits < 1) *splits = 1;
}

constexpr int kFastStages = 3;
constexpr int kPrefillMinRows = 64;  // query rows from which the tcgen05 prefill kernel is used
constexpr int kFastCtasPerSm = 2;
constexpr int kGenericMaxSplits = 256;

int generic_max_splits(int head_dim) {
    // finish_splits scratch in the generic kernel lives in the staged-key buffer.
    const int avail = 32 * (head_dim + 1) + 32 * head_dim;
    int m = avail / 16 - 1;
    return m < kGenericMaxSplits ? m : kGenericMaxSplits;
}

// Every kernel of the library is loaded on a device when its first arena is
// created, so no decode step pays a module load at a kernel's first launch.
void preload_kernels_once(int dev) {
    static std::atomic<bool> done[64];
    if (dev < 0 || dev >= 64 || done[dev].exchange(true)) return;
    preload_fast_kernels();
    preload_generic_kernels();
    preload_ring_kernels();
    preload_merge_kernels();
    preload_prefill_kernels();
    preload_model_kernels();
    cudaGetLastError();  // a kernel that cannot be loaded here reports the error at its launch
}

// ---- launch plan of the tensor-core prefill ----
// The kernel runs one CTA per SM; its units (query block, KV head) are
// launched in bands of KV heads, latest query blocks first inside a band
// (prefill_unit_level below). Costs are in 128-key tiles: a CTA costs
// its tiles plus a fixed set-up / epilogue share, a split part also the
// partial write and merge.
constexpr double kPrefillCtaCost = 4.0;
constexpr double kPrefillMergeCost = 3.0;
constexpr int kPrefillMaxParts = 4;       // split parts per SM at most (bounds the workspace)

struct PrefillPlan {
    int full_units;   // units run whole (the first ones in launch order)
    int tail_splits;  // key ranges of each later unit
    int head_group;   // KV heads interleaved per band of the launch order
};

// Launch order: bands of `head_group` KV heads (the last band may be smaller);
// inside a band, latest query blocks first with the band's heads interleaved.
// A band's K/V then stays in L2 while its waves stream it. Returns the launch
// level (0 = latest query block) of unit u.
inline int prefill_unit_level(int u, int nqb, int groups, int head_group) {
    const int band = u / (nqb * head_group);
    const int hs = std::min(head_group, groups - band * head_group);
    return (u - band * nqb * head_group) / hs;
}

// K/V bytes of the heads whose units share L2 at once: bands are sized so that
// about this much of a long context is streamed per band.
constexpr double kPrefillBandBytes = 40.0 * 1024 * 1024;

// Makespan of greedy list scheduling (each CTA, in launch order, takes the SM
// that frees first) when the units after the first `full` are split S ways.
double prefill_makespan(const std::vector<double>& level_tiles, int groups, int head_group, int full, int S, int sms,
                        std::vector<double>& heap) {
    heap.assign(sms, 0.0);  // all-zero: already a min-heap
    double end = 0.0;
    auto place = [&](double cost) {
        std::pop_heap(heap.begin(), heap.end(), std::greater<double>());
        heap.back() += cost;
        end = std::max(end, heap.back());
        std::push_heap(heap.begin(), heap.end(), std::greater<double>());
    };
    const int nqb = (int)level_tiles.size(), units = nqb * groups;
    for (int u = 0; u < units; ++u) {
        const double t = level_tiles[prefill_unit_level(u, nqb, groups, head_group)];
        if (u < full) {
            place(t + kPrefillCtaCost);
        } else {
            for (int s = 0; s < S; ++s) place(t / S + kPrefillCtaCost + kPrefillMergeCost);
        }
    }
    return end;
}

// A launch's final wave is often partly empty (e.g. 512 units on 148 SMs:
// 3.46 waves) while its units cost about the same, so the last SMs idle for
// most of a unit. Candidates split the last `tail` units (the partial last
// wave, that plus one more wave, or all units) into S = 2..4 key ranges; the
// plan with the shortest estimated makespan is used when it beats the unsplit
// launch by 3 %. Plans are cached per shape (every layer of a model repeats
// them).
PrefillPlan plan_prefill(int nqb, int groups, int ppc, int q_len, int q_pos0, int archived_tokens, int hstart,
                         int hlen, int sms) {
    static std::mutex mu;
    static std::map<std::array<int, 9>, PrefillPlan> cache;
    const std::array<int, 9> key = {nqb, groups, ppc, q_len, q_pos0 - hstart, archived_tokens, hlen, sms, 0};
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    std::vector<double> level(nqb);  // key tiles of launch level l (query block nqb - 1 - l)
    for (int l = 0; l < nqb; ++l) {
        const int qb = nqb - 1 - l;
        const int qlast = q_pos0 + std::min((qb + 1) * ppc, q_len) - 1;
        const int hot_keys = std::max(0, std::min(hlen, qlast - hstart + 1));
        level[l] = (archived_tokens + hot_keys) / 128.0;
    }
    const int units = nqb * groups;
    // bands of KV heads whose K/V (16-bit K and V of head_dim 128: 512 bytes per
    // key) fit the band budget; short contexts interleave every head
    const double head_bytes = 512.0 * (archived_tokens + hlen);
    const int head_group = std::max(1, std::min(groups, (int)(kPrefillBandBytes / std::max(head_bytes, 1.0))));
    std::vector<double> heap;
    PrefillPlan best{units, 1, head_group};
    double best_t = 0.97 * prefill_makespan(level, groups, head_group, units, 1, sms, heap);
    const int rem = units % sms;
    for (int S = 2; S <= 4; ++S) {
        for (int tail : {rem, rem + sms, units}) {
            if (tail <= 0 || tail > units || tail > kMaxCounters || (long long)tail * S > (long long)kPrefillMaxParts * sms)
                continue;
            if (level[nqb - 1] / S < 8.0) continue;  // parts of the shortest units would be mostly overhead
            const double t = prefill_makespan(level, groups, head_group, units - tail, S, sms, heap);
            if (t < best_t) {
                best_t = t;
                best = {units - tail, S, head_group};
            }
        }
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cache.size() > 1024) cache.clear();
    cache[key] = best;
    return best;
}

}  // namespace

extern "C" {

const char* rfsn_last_error(void) { return g_last_error.c_str(); }

int rfsn_abi_version(void) { return RFSN_ABI_VERSION; }

uint64_t rfsn_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

rfsn_status rfsn_device_sm_count(int* out) {
    RFSN_CHECK_ARG(out != nullptr, "rfsn_device_sm_count: out is NULL");
    int dev = 0;
    RFSN_CUDA(cudaGetDevice(&dev));
    RFSN_CUDA(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev));
    return RFSN_OK;
}

rfsn_status rfsn_arena_create(void* k_arena, void* v_arena, int dtype, int batch_kv_heads, int rows, int head_dim,
                              rfsn_arena** out) {
    RFSN_CHECK_ARG(out != nullptr, "rfsn_arena_create: out is NULL");
    RFSN_CHECK_ARG(k_arena != nullptr && v_arena != nullptr, "rfsn_arena_create: NULL arena pointer");
    RFSN_CHECK_ARG(valid_dtype(dtype), "rfsn_arena_create: unknown dtype %d", dtype);
    RFSN_CHECK_ARG(batch_kv_heads > 0 && rows > 0 && head_dim > 0, "rfsn_arena_create: non-positive shape");
    RFSN_CHECK_ARG(head_dim % 2 == 0, "rfsn_arena_create: head_dim must be even (RoPE pairs), got %d", head_dim);
    RFSN_CHECK_ARG((uintptr_t)k_arena % 16 == 0 && (uintptr_t)v_arena % 16 == 0,
                   "rfsn_arena_create: arena pointers must be 16-byte aligned");
    rfsn_arena* a = new rfsn_arena();
    a->k = k_arena;
    a->v = v_arena;
    a->dtype = dtype;
    a->groups = batch_kv_heads;
    a->rows = rows;
    a->head_dim = head_dim;
    cudaGetDevice(&a->device);
    preload_kernels_once(a->device);
    a->has_tma = false;
    if ((dtype == RFSN_BF16 || dtype == RFSN_F16) && head_dim == 128) {
        rfsn_status st = encode_map(&a->maps[0], k_arena, dtype, batch_kv_heads, rows, head_dim, 64);
        if (st == RFSN_OK) st = encode_map(&a->maps[1], v_arena, dtype, batch_kv_heads, rows, head_dim, 64);
        if (st == RFSN_OK) st = encode_map(&a->maps[2], k_arena, dtype, batch_kv_heads, rows, head_dim, 8);
        if (st == RFSN_OK) st = encode_map(&a->maps[3], v_arena, dtype, batch_kv_heads, rows, head_dim, 8);
        if (st != RFSN_OK) {
            delete a;
            return st;
        }
        a->has_tma = true;
    }
    *out = a;
    return RFSN_OK;
}

rfsn_status rfsn_arena_destroy(rfsn_arena* arena) {
    delete arena;
    return RFSN_OK;
}

rfsn_status rfsn_rope_append(const void* q, const void* k, const void* v, int in_dtype, const float* inv_freq, int pos0,
                             int batch, int q_heads, int kv_heads, int len, int head_dim, float* q_out,
                             const rfsn_arena* arena, int ring_row0, int capacity, int write_index, void* stream) {
    RFSN_CHECK_ARG(arena != nullptr, "rfsn_rope_append: NULL arena");
    RFSN_CHECK_ARG((k != nullptr) == (v != nullptr), "rfsn_rope_append: k and v must both be given or both NULL");
    if (k == nullptr) {
        RFSN_CHECK_ARG(q != nullptr && q_out != nullptr && inv_freq != nullptr,
                       "rfsn_rope_append: rotating q alone needs q, q_out and inv_freq");
        kv_heads = 0;
    }
    RFSN_CHECK_ARG(valid_dtype(in_dtype), "rfsn_rope_append: unknown dtype %d", in_dtype);
    RFSN_CHECK_ARG(in_dtype == arena->dtype, "rfsn_rope_append: input dtype %d differs from cache dtype %d", in_dtype,
                   arena->dtype);
    RFSN_CHECK_ARG(batch > 0 && kv_heads >= 0 && len > 0 && q_heads >= 0, "rfsn_rope_append: non-positive shape");
    RFSN_CHECK_ARG(head_dim == arena->head_dim, "rfsn_rope_append: head_dim %d != arena head_dim %d", head_dim,
                   arena->head_dim);
    RFSN_CHECK_ARG(k == nullptr || batch * kv_heads == arena->groups,
                   "rfsn_rope_append: batch*kv_heads %d != arena groups %d", batch * kv_heads, arena->groups);
    RFSN_CHECK_ARG(capacity > 0 && ring_row0 >= 0 && ring_row0 + capacity <= arena->rows,
                   "rfsn_rope_append: ring rows [%d, %d) outside the arena (%d rows)", ring_row0, ring_row0 + capacity,
                   arena->rows);
    RFSN_CHECK_ARG(write_index >= 0 && write_index < capacity, "rfsn_rope_append: write_index %d outside [0, %d)",
                   write_index, capacity);
    if (len > capacity) {
        set_error("append_exact: chunk of %d tokens exceeds the ring capacity %d", len, capacity);
        return RFSN_ERR_OVERFLOW;
    }
    const int qh = (inv_freq != nullptr && q != nullptr) ? q_heads : 0;
    return rope_append_launch(in_dtype, q, k, v, inv_freq, pos0, batch, qh, kv_heads, len, head_dim, q_out, arena->k,
                              arena->v, arena->rows, ring_row0, capacity, write_index, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_rope_append_step(const void* q, const void* k, const void* v, int in_dtype, const float* inv_freq,
                                  const int32_t* step_state, int32_t* step_state_copy, int batch, int q_heads,
                                  int kv_heads, int len, int head_dim, float* q_out, const rfsn_arena* arena,
                                  int ring_row0, int capacity, void* stream) {
    RFSN_CHECK_ARG(step_state != nullptr, "rfsn_rope_append_step: NULL step state");
    RFSN_CHECK_ARG(arena != nullptr, "rfsn_rope_append_step: NULL arena");
    RFSN_CHECK_ARG((k != nullptr) == (v != nullptr), "rfsn_rope_append_step: k and v must both be given or both NULL");
    if (k == nullptr) {  // rotate q alone (a shard that does not own the hot window)
        RFSN_CHECK_ARG(q != nullptr && q_out != nullptr && inv_freq != nullptr,
                       "rfsn_rope_append_step: rotating q alone needs q, q_out and inv_freq");
        kv_heads = 0;
    }
    RFSN_CHECK_ARG(valid_dtype(in_dtype) && in_dtype == arena->dtype,
                   "rfsn_rope_append_step: input dtype %d differs from cache dtype %d", in_dtype, arena->dtype);
    RFSN_CHECK_ARG(batch > 0 && kv_heads >= 0 && len > 0 && q_heads >= 0, "rfsn_rope_append_step: non-positive shape");
    RFSN_CHECK_ARG(head_dim == arena->head_dim && (k == nullptr || batch * kv_heads == arena->groups),
                   "rfsn_rope_append_step: shape does not match the arena");
    RFSN_CHECK_ARG(capacity > 0 && ring_row0 >= 0 && ring_row0 + capacity <= arena->rows,
                   "rfsn_rope_append_step: ring rows outside the arena");
    if (len > capacity) {
        set_error("append_exact: chunk of %d tokens exceeds the ring capacity %d", len, capacity);
        return RFSN_ERR_OVERFLOW;
    }
    const int qh = (inv_freq != nullptr && q != nullptr) ? q_heads : 0;
    return rope_append_launch(in_dtype, q, k, v, inv_freq, 0, batch, qh, kv_heads, len, head_dim, q_out, arena->k,
                              arena->v, arena->rows, ring_row0, capacity, 0, static_cast<cudaStream_t>(stream),
                              step_state, step_state_copy);
}

rfsn_status rfsn_rope_append_tables(const void* q, const void* k, const void* v, int in_dtype, const void* cos_t,
                                    const void* sin_t, int tab_dtype, const float* inv_freq, int pos0, int batch,
                                    int q_heads, int kv_heads, int len, int head_dim, float* q_out,
                                    const rfsn_arena* arena, int ring_row0, int capacity, int write_index,
                                    void* stream) {
    RFSN_CHECK_ARG(arena != nullptr, "rfsn_rope_append_tables: NULL arena");
    RFSN_CHECK_ARG(q != nullptr && k != nullptr && v != nullptr && q_out != nullptr,
                   "rfsn_rope_append_tables: NULL q/k/v/q_out");
    RFSN_CHECK_ARG((cos_t == nullptr) == (sin_t == nullptr), "rfsn_rope_append_tables: cos and sin go together");
    RFSN_CHECK_ARG(cos_t != nullptr || inv_freq != nullptr, "rfsn_rope_append_tables: no tables and no inv_freq");
    RFSN_CHECK_ARG(valid_dtype(in_dtype) && valid_dtype(tab_dtype), "rfsn_rope_append_tables: unknown dtype");
    RFSN_CHECK_ARG(in_dtype == arena->dtype, "rfsn_rope_append_tables: input dtype %d differs from cache dtype %d",
                   in_dtype, arena->dtype);
    RFSN_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && len > 0, "rfsn_rope_append_tables: non-positive shape");
    RFSN_CHECK_ARG(head_dim == arena->head_dim && batch * kv_heads == arena->groups,
                   "rfsn_rope_append_tables: shape does not match the arena");
    RFSN_CHECK_ARG(capacity > 0 && ring_row0 >= 0 && ring_row0 + capacity <= arena->rows,
                   "rfsn_rope_append_tables: ring rows outside the arena");
    RFSN_CHECK_ARG(write_index >= 0 && write_index < capacity, "rfsn_rope_append_tables: write_index %d outside [0, %d)",
                   write_index, capacity);
    if (len > capacity) {
        set_error("append_exact: chunk of %d tokens exceeds the ring capacity %d", len, capacity);
        return RFSN_ERR_OVERFLOW;
    }
    return rope_tables_append_launch(in_dtype, tab_dtype, q, k, v, cos_t, sin_t, inv_freq, pos0, batch, q_heads,
                                     kv_heads, len, head_dim, q_out, arena->k, arena->v, arena->rows, ring_row0,
                                     capacity, write_index, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_rms_norm(const void* x, const void* residual, const void* weight, void* sum_out, void* out, int rows,
                          int n, int dtype, float eps, void* stream) {
    RFSN_CHECK_ARG(x != nullptr && weight != nullptr && out != nullptr, "rfsn_rms_norm: NULL pointer");
    RFSN_CHECK_ARG((residual == nullptr) == (sum_out == nullptr), "rfsn_rms_norm: residual and sum_out go together");
    RFSN_CHECK_ARG(rows >= 0 && n > 0 && valid_dtype(dtype), "rfsn_rms_norm: bad shape or dtype");
    if (rows == 0) return RFSN_OK;
    return rms_norm_dispatch(dtype, x, residual, weight, sum_out, out, rows, n, eps, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_silu_mul(const void* gate_up, void* out, int rows, int n, int dtype, void* stream) {
    RFSN_CHECK_ARG(gate_up != nullptr && out != nullptr, "rfsn_silu_mul: NULL pointer");
    RFSN_CHECK_ARG(rows >= 0 && n > 0 && valid_dtype(dtype), "rfsn_silu_mul: bad shape or dtype");
    if (rows == 0) return RFSN_OK;
    return silu_mul_dispatch(dtype, gate_up, out, rows, n, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_gemv(const void* weight, const void* x, void* y, int n_out, int k, int rows, int dtype, void* stream) {
    RFSN_CHECK_ARG(weight != nullptr && x != nullptr && y != nullptr, "rfsn_gemv: NULL pointer");
    RFSN_CHECK_ARG(valid_dtype(dtype) && n_out > 0 && k > 0 && rows >= 1 && rows <= gemv_max_rows(),
                   "rfsn_gemv: bad shape or dtype (rows of x: 1..%d)", gemv_max_rows());
    const int vec = 16 / dtype_size(dtype);
    RFSN_CHECK_ARG(k % vec == 0 && reinterpret_cast<uintptr_t>(weight) % 16 == 0,
                   "rfsn_gemv: weight rows must be 16-byte aligned (k a multiple of %d)", vec);
    RFSN_CHECK_ARG((size_t)rows * k * sizeof(float) <= 200 * 1024, "rfsn_gemv: x too large for shared memory");
    return gemv_dispatch(dtype, weight, x, y, n_out, k, rows, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_prefill_plan(int batch, int q_heads, int kv_heads, int q_len, int q_pos0, int archived_tokens,
                              int hot_start, int hot_length, int* cta_units_whole, int* tail_splits, int* ctas) {
    RFSN_CHECK_ARG(cta_units_whole != nullptr && tail_splits != nullptr && ctas != nullptr, "rfsn_prefill_plan: NULL output");
    RFSN_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && q_len > 0 && q_heads % kv_heads == 0,
                   "rfsn_prefill_plan: bad shape");
    const int G = q_heads / kv_heads;
    RFSN_CHECK_ARG(G <= 128, "rfsn_prefill_plan: %d query heads per KV head (max 128)", G);
    const int ppc = 128 / G, nqb = (q_len + ppc - 1) / ppc, units = nqb * batch * kv_heads;
    const PrefillPlan plan = plan_prefill(nqb, batch * kv_heads, ppc, q_len, q_pos0, archived_tokens, hot_start,
                                          hot_length, sm_count_cached());
    *cta_units_whole = plan.full_units;
    *tail_splits = plan.tail_splits;
    *ctas = plan.full_units + (units - plan.full_units) * plan.tail_splits;
    return RFSN_OK;
}

rfsn_status rfsn_host_device_pointer(const void* host_ptr, void** device_ptr) {
    RFSN_CHECK_ARG(host_ptr != nullptr && device_ptr != nullptr, "rfsn_host_device_pointer: NULL pointer");
    *device_ptr = nullptr;
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, host_ptr) != cudaSuccess) {
        cudaGetLastError();
        set_error("rfsn_host_device_pointer: not memory known to CUDA");
        return RFSN_ERR_INVALID_ARG;
    }
    RFSN_CHECK_ARG(attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr,
                   "rfsn_host_device_pointer: not page-locked host memory mapped for the device");
    *device_ptr = attr.devicePointer;
    return RFSN_OK;
}

rfsn_status rfsn_arena_copy_rows(const rfsn_arena* arena, int src_row0, int src_offset, int src_wrap, int dst_row0,
                                 int count, void* stream) {
    RFSN_CHECK_ARG(arena != nullptr, "rfsn_arena_copy_rows: NULL arena");
    RFSN_CHECK_ARG(count >= 0, "rfsn_arena_copy_rows: negative count");
    if (count == 0) return RFSN_OK;
    RFSN_CHECK_ARG(src_wrap >= 0 && src_offset >= 0, "rfsn_arena_copy_rows: negative offset/wrap");
    const int src_span = src_wrap > 0 ? src_wrap : src_offset + count;
    RFSN_CHECK_ARG(src_row0 >= 0 && src_row0 + src_span <= arena->rows, "rfsn_arena_copy_rows: source rows outside the arena");
    RFSN_CHECK_ARG(src_wrap == 0 || (src_offset < src_wrap && count <= src_wrap),
                   "rfsn_arena_copy_rows: wrapped source range larger than the ring");
    RFSN_CHECK_ARG(dst_row0 >= 0 && dst_row0 + count <= arena->rows, "rfsn_arena_copy_rows: destination rows outside the arena");
    const int row_bytes = arena->head_dim * dtype_size(arena->dtype);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (row_bytes % 16 == 0) {
        return copy_rows_launch(arena->k, arena->v, arena->groups, arena->rows, row_bytes, src_row0, src_offset,
                                src_wrap, dst_row0, count, s);
    }
    // Rows not a multiple of 16 bytes: per-piece 2-D copies (at most two pieces when wrapping).
    const size_t pitch = (size_t)arena->rows * row_bytes;
    int done = 0;
    while (done < count) {
        int srow = src_offset + done;
        if (src_wrap > 0) srow %= src_wrap;
        int n = count - done;
        if (src_wrap > 0 && srow + n > src_wrap) n = src_wrap - srow;
        for (int t = 0; t < 2; ++t) {
            uint8_t* base = static_cast<uint8_t*>(t == 0 ? arena->k : arena->v);
            RFSN_CUDA(cudaMemcpy2DAsync(base + (size_t)(dst_row0 + done) * row_bytes, pitch,
                                        base + (size_t)(src_row0 + srow) * row_bytes, pitch, (size_t)n * row_bytes,
                                        arena->groups, cudaMemcpyDeviceToDevice, s));
        }
        done += n;
    }
    return RFSN_OK;
}

static rfsn_status block_xfer(const rfsn_arena* arena, int row0, int count, const void* k_host, const void* v_host,
                              void* k_out, void* v_out, void* stream, void* done_event, bool upload) {
    RFSN_CHECK_ARG(arena != nullptr, "block transfer: NULL arena");
    RFSN_CHECK_ARG(count > 0 && row0 >= 0 && row0 + count <= arena->rows, "block transfer: rows [%d, %d) outside the arena",
                   row0, row0 + count);
    const size_t row_bytes = (size_t)arena->head_dim * dtype_size(arena->dtype);
    const size_t pitch = (size_t)arena->rows * row_bytes;
    const size_t blk_pitch = (size_t)count * row_bytes;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int t = 0; t < 2; ++t) {
        uint8_t* base = static_cast<uint8_t*>(t == 0 ? arena->k : arena->v) + (size_t)row0 * row_bytes;
        if (upload) {
            const void* src = t == 0 ? k_host : v_host;
            RFSN_CHECK_ARG(src != nullptr, "rfsn_block_upload: NULL source");
            RFSN_CUDA(cudaMemcpy2DAsync(base, pitch, src, blk_pitch, blk_pitch, arena->groups, cudaMemcpyDefault, s));
        } else {
            void* dst = t == 0 ? k_out : v_out;
            RFSN_CHECK_ARG(dst != nullptr, "rfsn_block_download: NULL destination");
            RFSN_CUDA(cudaMemcpy2DAsync(dst, blk_pitch, base, pitch, blk_pitch, arena->groups, cudaMemcpyDefault, s));
        }
    }
    if (done_event != nullptr) RFSN_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(done_event), s));
    return RFSN_OK;
}

rfsn_status rfsn_block_upload(const rfsn_arena* arena, int dst_row0, int count, const void* k_src, const void* v_src,
                              void* stream, void* done_event) {
    return block_xfer(arena, dst_row0, count, k_src, v_src, nullptr, nullptr, stream, done_event, true);
}

rfsn_status rfsn_block_download(const rfsn_arena* arena, int src_row0, int count, void* k_dst, void* v_dst, void* stream,
                                void* done_event) {
    return block_xfer(arena, src_row0, count, nullptr, nullptr, k_dst, v_dst, stream, done_event, false);
}

rfsn_status rfsn_event_wait(void* event, int64_t timeout_us) {
    RFSN_CHECK_ARG(event != nullptr, "rfsn_event_wait: NULL event");
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
        if (e == cudaSuccess) return RFSN_OK;
        if (e != cudaErrorNotReady) return cuda_status(e, "cudaEventQuery");
        const auto us = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (us >= timeout_us) {
            set_error("event not complete after %lld us", (long long)timeout_us);
            return RFSN_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

rfsn_status rfsn_attention_workspace_size(int batch, int q_heads, int kv_heads, int q_len, int head_dim, int max_splits,
                                          size_t* bytes) {
    RFSN_CHECK_ARG(bytes != nullptr, "rfsn_attention_workspace_size: bytes is NULL");
    RFSN_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && q_len > 0 && head_dim > 0,
                   "rfsn_attention_workspace_size: non-positive shape");
    RFSN_CHECK_ARG(q_heads % kv_heads == 0, "num_heads (%d) must be divisible by num_kv_heads (%d)", q_heads, kv_heads);
    // The largest layout any kernel can choose for this shape: split counts
    // follow from the SM count (at least 148 assumed, so a size computed
    // without a device still serves a B200).
    const int G = q_heads / kv_heads;
    const int nslots = q_len * G;
    const int slots_ws = nslots < 4 ? 4 : nslots;
    const int qblocks = (nslots + 7) / 8;
    const int groups = batch * kv_heads;
    const int sms = std::max(sm_count_cached(), 148);
    auto bound = [&](int cap, int target, int units) {
        int s = std::max(1, target / std::max(units, 1));
        if (max_splits > 0) s = std::min(s, max_splits);
        return std::max(1, std::min(s, cap));
    };
    size_t need = ws_layout(groups, qblocks, bound(generic_max_splits(head_dim), sms * 4, groups * qblocks), slots_ws,
                            head_dim).total;  // CUDA-core kernel
    if (head_dim == 128 && nslots <= 4) {  // tensor-core decode kernel
        need = std::max(need, ws_layout(groups, 1, bound(fast_max_splits(), sms * kFastCtasPerSm, groups), slots_ws,
                                        128).total);
    }
    if (head_dim == 128 && q_len >= kPrefillMinRows) {  // tensor-core prefill: split parts
        need = std::max(need, ws_layout(1, 1, kPrefillMaxParts * sms, 128, 128).total);
    }
    *bytes = need;
    return RFSN_OK;
}

}  // extern "C"

namespace {

struct CommonArgs {
    int batch, q_heads, kv_heads, q_len, head_dim, G, nslots, slots_ws, qblocks, groups;
};

rfsn_status check_common(const float* q, int batch, int q_heads, int kv_heads, int q_len, int head_dim, float* out,
                         void* workspace, CommonArgs* a) {
    RFSN_CHECK_ARG(q != nullptr && out != nullptr, "attention: NULL q/out");
    RFSN_CHECK_ARG(workspace != nullptr, "attention: NULL workspace");
    RFSN_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && q_len > 0, "attention: non-positive shape");
    RFSN_CHECK_ARG(q_heads % kv_heads == 0, "num_heads (%d) must be divisible by num_kv_heads (%d)", q_heads, kv_heads);
    RFSN_CHECK_ARG(head_dim > 0 && head_dim <= 256, "attention: head_dim %d outside [1, 256]", head_dim);
    // the kernels store output rows as float4 when head_dim allows it
    RFSN_CHECK_ARG(head_dim % 4 != 0 || reinterpret_cast<uintptr_t>(out) % 16 == 0,
                   "attention: out must be 16-byte aligned");
    RFSN_CHECK_ARG(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "attention: workspace must be 16-byte aligned");
    a->batch = batch;
    a->q_heads = q_heads;
    a->kv_heads = kv_heads;
    a->q_len = q_len;
    a->head_dim = head_dim;
    a->G = q_heads / kv_heads;
    a->nslots = q_len * a->G;
    a->slots_ws = a->nslots < 4 ? 4 : a->nslots;
    a->qblocks = (a->nslots + 7) / 8;
    a->groups = batch * kv_heads;
    RFSN_CHECK_ARG((long)a->groups * a->qblocks <= kMaxCounters, "attention: batch*kv_heads*q_blocks above %d",
                   kMaxCounters);
    return RFSN_OK;
}

float qscale_for(int head_dim) {
    // scale = 1 / sqrt(D) (attention_exact.py:139), times log2(e) for exp2.
    const float scale = (float)(1.0 / std::sqrt((double)head_dim));
    return scale * 1.4426950408889634f;
}

}  // namespace

extern "C" {

rfsn_status rfsn_paged_attention(const rfsn_arena* arena, const float* q, int batch, int q_heads, int kv_heads, int q_len,
                                 int q_pos0, const rfsn_page_table* table, const rfsn_hot_window* hot, float* out,
                                 float* lse, void* workspace, size_t workspace_bytes, int max_splits, void* stream) {
    return rfsn::paged_attention_impl(arena, q, batch, q_heads, kv_heads, q_len, q_pos0, table, hot, out, lse, workspace,
                                      workspace_bytes, max_splits, nullptr, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

rfsn_status rfsn::paged_attention_impl(const rfsn_arena* arena, const float* q, int batch, int q_heads, int kv_heads,
                                       int q_len, int q_pos0, const rfsn_page_table* table, const rfsn_hot_window* hot,
                                       float* out, float* lse, void* workspace, size_t workspace_bytes, int max_splits,
                                       const PeerParams* peer, cudaStream_t s, bool dry_run) {
    RFSN_CHECK_ARG(arena != nullptr && table != nullptr && hot != nullptr, "rfsn_paged_attention: NULL arena/table/hot");
    CommonArgs a;
    rfsn_status st = check_common(q, batch, q_heads, kv_heads, q_len, arena->head_dim, out, workspace, &a);
    if (st != RFSN_OK) return st;
    RFSN_CHECK_ARG(a.groups == arena->groups, "rfsn_paged_attention: batch*kv_heads %d != arena groups %d", a.groups,
                   arena->groups);
    RFSN_CHECK_ARG(table->n_blocks >= 0 && (table->n_blocks == 0 || table->records != nullptr),
                   "rfsn_paged_attention: bad page table");
    RFSN_CHECK_ARG(hot->length >= 0 && hot->length <= hot->capacity && hot->head_index >= 0 &&
                       hot->head_index < (hot->capacity > 0 ? hot->capacity : 1) &&
                       hot->ring_row0 >= 0 && hot->ring_row0 + hot->capacity <= arena->rows,
                   "rfsn_paged_attention: bad hot window");
    const int first = hot->length < hot->capacity - hot->head_index ? hot->length : hot->capacity - hot->head_index;
    const int hot_tiles = (first + kTile - 1) / kTile + (hot->length - first + kTile - 1) / kTile;
    const int total_tiles = table->archived_tiles + hot_tiles;
    // With a device step state the window is only known when the kernel runs
    // (an empty context then gives zero output and -inf LSE).
    if (total_tiles <= 0 && peer == nullptr && hot->step_state == nullptr) {
        set_error("run_segmented_attention requires at least one KV segment");
        return RFSN_ERR_INVALID_ARG;
    }
    const int sms = sm_count_cached();
    const bool use_fast = arena->has_tma && arena->head_dim == 128 && a.nslots <= 4;
    // chunked prefill on the tensor cores: float4 q/out rows need 16-byte alignment
    const bool stepped = hot->step_state != nullptr;  // position / hot window read on the device
    const bool use_prefill = !stepped && peer == nullptr && arena->has_tma && arena->head_dim == 128 &&
                             q_len >= kPrefillMinRows && a.G <= 128 && (uintptr_t)q % 16 == 0 &&
                             (uintptr_t)out % 16 == 0;
    if (stepped && !use_fast) {
        set_error("a device step state needs the tensor-core decode shape (bf16/f16, head_dim 128, <= 4 query "
                  "slots per KV head)");
        return RFSN_ERR_UNSUPPORTED;
    }
    if (use_prefill) {
        // One CTA per (query block, KV head) streams the whole causal key range; the
        // units of a partly filled last wave (or of a launch too small for the SMs)
        // may be split into key ranges merged by their last CTA (plan_prefill).
        const int ppc = 128 / a.G;
        const int nqb = (q_len + ppc - 1) / ppc;
        const int units = nqb * a.groups;
        PrefillPlan plan = plan_prefill(nqb, a.groups, ppc, q_len, q_pos0, table->archived_tokens, hot->start_pos,
                                        hot->length, sms);
        const int parts = (units - plan.full_units) * plan.tail_splits;
        WsLayout w = ws_layout(1, 1, plan.tail_splits > 1 ? parts : 1, 128, 128);
        if (w.total > workspace_bytes && plan.tail_splits > 1) {  // a small workspace: run every unit whole
            plan = {units, 1, plan.head_group};
            w = ws_layout(1, 1, 1, 128, 128);
        }
        if (w.total > workspace_bytes) {
            set_error("attention workspace too small: need %zu bytes, have %zu", w.total, workspace_bytes);
            return RFSN_ERR_OVERFLOW;
        }
        PrefillParams pp;
        memset(&pp, 0, sizeof(pp));
        pp.nqb = nqb;
        pp.full_units = plan.full_units;
        pp.tail_splits = plan.tail_splits;
        pp.head_group = plan.head_group;
        pp.q = q;
        pp.out = out;
        pp.lse = lse;
        pp.records = reinterpret_cast<const int4*>(table->records);
        pp.n_blocks = table->n_blocks;
        pp.ring_row0 = hot->ring_row0;
        pp.capacity = hot->capacity;
        pp.head = hot->head_index;
        pp.hlen = hot->length;
        pp.hstart = hot->start_pos;
        pp.rows = arena->rows;
        pp.batch = batch;
        pp.q_heads = q_heads;
        pp.kv_heads = kv_heads;
        pp.q_len = q_len;
        pp.q_pos0 = q_pos0;
        pp.groups_per_kv = a.G;
        pp.qscale = qscale_for(128);
        pp.ws = ws_view(workspace, w);
        if (dry_run) return RFSN_OK;
        return prefill_launch(arena->dtype, arena->maps, pp, s);
    }
    if (peer != nullptr && !use_fast) {
        set_error("fused cross-GPU merge needs the tensor-core decode shape (bf16/f16, head_dim 128, <= 4 query "
                  "slots per KV head)");
        return RFSN_ERR_UNSUPPORTED;
    }
    if (use_fast) {
        fast::Params p;
        int splits, tps;
        const int cap = max_splits > 0 ? (max_splits < fast_max_splits() ? max_splits : fast_max_splits()) : fast_max_splits();
        // With a device step state the hot window is only known when the kernel
        // runs: the split count is chosen for the largest window the ring holds
        // (two pieces), and the kernel derives its tile ranges itself.
        const int plan_tiles = stepped ? table->archived_tiles + (hot->capacity + kTile - 1) / kTile + 1 : total_tiles;
        choose_splits(plan_tiles, a.groups, sms * kFastCtasPerSm, cap, &splits, &tps);
        const WsLayout w = ws_layout(a.groups, 1, splits, a.slots_ws, 128);
        if (w.total > workspace_bytes) {
            set_error("attention workspace too small: need %zu bytes, have %zu", w.total, workspace_bytes);
            return RFSN_ERR_OVERFLOW;
        }
        p.q = q;
        p.out = out;
        p.lse = lse;
        p.records = reinterpret_cast<const int4*>(table->records);
        p.n_blocks = table->n_blocks;
        p.archived_tiles = table->archived_tiles;
        p.ring_row0 = hot->ring_row0;
        p.capacity = hot->capacity;
        p.head = hot->head_index;
        p.hlen = hot->length;
        p.hstart = hot->start_pos;
        p.rows = arena->rows;
        p.q_heads = q_heads;
        p.kv_heads = kv_heads;
        p.q_len = q_len;
        p.q_pos0 = q_pos0;
        p.groups_per_kv = a.G;
        p.nslots = a.nslots;
        p.total_tiles = total_tiles;
        p.tiles_per_split = tps;
        p.splits = splits;
        p.groups = a.groups;
        p.qscale = qscale_for(128);
        p.pscale = arena->dtype == RFSN_F16 ? 4096.f : 1.f;
        p.ws = ws_view(workspace, w);
        memset(&p.peer, 0, sizeof(p.peer));
        if (peer != nullptr) p.peer = *peer;
        p.dyn = hot->step_state;
        if (dry_run) return RFSN_OK;
        return fast_launch(arena->dtype, arena->maps, p, kFastStages, s);
    }
    generic::Params p;
    memset(&p, 0, sizeof(p));
    int splits, tps;
    int cap = generic_max_splits(arena->head_dim);
    if (max_splits > 0 && max_splits < cap) cap = max_splits;
    choose_splits(total_tiles, a.groups * a.qblocks, sms * 4, cap, &splits, &tps);
    const WsLayout w = ws_layout(a.groups, a.qblocks, splits, a.slots_ws, arena->head_dim);
    if (w.total > workspace_bytes) {
        set_error("attention workspace too small: need %zu bytes, have %zu", w.total, workspace_bytes);
        return RFSN_ERR_OVERFLOW;
    }
    p.q = q;
    p.out = out;
    p.lse = lse;
    p.head_dim = arena->head_dim;
    p.q_heads = q_heads;
    p.kv_heads = kv_heads;
    p.q_len = q_len;
    p.q_pos0 = q_pos0;
    p.groups_per_kv = a.G;
    p.nslots_total = a.nslots;
    p.slots_ws = a.slots_ws;
    p.total_tiles = total_tiles;
    p.tiles_per_split = tps;
    p.splits = splits;
    p.qblocks = a.qblocks;
    p.qscale = qscale_for(arena->head_dim);
    p.ws = ws_view(workspace, w);
    p.arena_k = arena->k;
    p.arena_v = arena->v;
    p.rows = arena->rows;
    p.records = reinterpret_cast<const int4*>(table->records);
    p.n_blocks = table->n_blocks;
    p.archived_tiles = table->archived_tiles;
    p.ring_row0 = hot->ring_row0;
    p.capacity = hot->capacity;
    p.head = hot->head_index;
    p.hlen = hot->length;
    p.hstart = hot->start_pos;
    if (dry_run) return RFSN_OK;
    return generic_launch(arena->dtype, true, p, a.groups, s);
}

extern "C" {

rfsn_status rfsn_segmented_attention(const float* q, int batch, int q_heads, int kv_heads, int q_len, int q_pos0,
                                     int head_dim, int kv_dtype, const rfsn_segment_desc* segments, int n_segments,
                                     int total_tiles, float* out, float* lse, void* workspace, size_t workspace_bytes,
                                     int max_splits, void* stream) {
    CommonArgs a;
    rfsn_status st = check_common(q, batch, q_heads, kv_heads, q_len, head_dim, out, workspace, &a);
    if (st != RFSN_OK) return st;
    RFSN_CHECK_ARG(valid_dtype(kv_dtype), "rfsn_segmented_attention: unknown dtype %d", kv_dtype);
    if (n_segments <= 0 || total_tiles <= 0) {
        set_error("run_segmented_attention requires at least one KV segment");
        return RFSN_ERR_INVALID_ARG;
    }
    RFSN_CHECK_ARG(segments != nullptr, "rfsn_segmented_attention: NULL segment table");
    generic::Params p;
    memset(&p, 0, sizeof(p));
    int splits, tps;
    int cap = generic_max_splits(head_dim);
    if (max_splits > 0 && max_splits < cap) cap = max_splits;
    choose_splits(total_tiles, a.groups * a.qblocks, sm_count_cached() * 4, cap, &splits, &tps);
    const WsLayout w = ws_layout(a.groups, a.qblocks, splits, a.slots_ws, head_dim);
    if (w.total > workspace_bytes) {
        set_error("attention workspace too small: need %zu bytes, have %zu", w.total, workspace_bytes);
        return RFSN_ERR_OVERFLOW;
    }
    p.q = q;
    p.out = out;
    p.lse = lse;
    p.head_dim = head_dim;
    p.q_heads = q_heads;
    p.kv_heads = kv_heads;
    p.q_len = q_len;
    p.q_pos0 = q_pos0;
    p.groups_per_kv = a.G;
    p.nslots_total = a.nslots;
    p.slots_ws = a.slots_ws;
    p.total_tiles = total_tiles;
    p.tiles_per_split = tps;
    p.splits = splits;
    p.qblocks = a.qblocks;
    p.qscale = qscale_for(head_dim);
    p.ws = ws_view(workspace, w);
    p.segs = segments;
    p.n_segs = n_segments;
    return generic_launch(kv_dtype, false, p, a.groups, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_lse_merge(const float* parts_out, const float* parts_lse, int n_parts, int rows, int head_dim,
                           float* out, float* lse_out, void* stream) {
    RFSN_CHECK_ARG(parts_out != nullptr && parts_lse != nullptr && out != nullptr, "rfsn_lse_merge: NULL pointer");
    RFSN_CHECK_ARG(n_parts > 0 && rows > 0 && head_dim > 0, "rfsn_lse_merge: non-positive shape");
    return lse_merge_launch(parts_out, parts_lse, n_parts, rows, head_dim, out, lse_out, static_cast<cudaStream_t>(stream));
}

rfsn_status rfsn_workspace_check(void* workspace, void* stream, int64_t timeout_us) {
    RFSN_CHECK_ARG(workspace != nullptr, "rfsn_workspace_check: NULL workspace");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaEvent_t ev;
    RFSN_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaError_t e = cudaEventRecord(ev, s);
    if (e != cudaSuccess) {
        cudaEventDestroy(ev);
        return cuda_status(e, "cudaEventRecord");
    }
    rfsn_status st = rfsn_event_wait(ev, timeout_us);
    cudaEventDestroy(ev);
    if (st != RFSN_OK) return st;
    int word = 0;
    RFSN_CUDA(cudaMemcpy(&word, workspace, sizeof(int), cudaMemcpyDeviceToHost));
    if (word != 0) {
        const int zero = 0;
        RFSN_CUDA(cudaMemcpy(workspace, &zero, sizeof(int), cudaMemcpyHostToDevice));
        if (word == kDevErrPeerTimeout) {
            set_error("attention kernel: the cross-GPU merge timed out waiting for a peer's partial results (in this "
                      "call or an earlier one of the same peer group; the group must be destroyed and created again)");
            return RFSN_ERR_TIMEOUT;
        }
        if (word == kDevErrTimeout) {
            set_error("attention kernel: a bounded pipeline wait expired");
            return RFSN_ERR_TIMEOUT;
        }
        if (word == kDevErrBadTable) {
            set_error("attention kernel: a page-table record or step state points outside the arena");
            return RFSN_ERR_DEVICE;
        }
        set_error("attention kernel reported device error %d", word);
        return RFSN_ERR_DEVICE;
    }
    return RFSN_OK;
}

}  // extern "C"
