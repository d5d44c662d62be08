// rfsn_paged_attention_noalloc: paged attention that allocates nothing.
//
// Some callers cannot call cudaMalloc at the point where they run attention:
// an inference engine that owns every byte of device memory through its own
// pool (and forbids allocations behind its back), code running while a
// memory budget is frozen, or a plugin host that only hands out the input and
// output buffers. For them this entry point keeps the split-KV scratch (arrival
// counters, per-split partial results) in one fixed array compiled into the
// library, so the call needs no workspace argument and performs no device
// allocation of any kind.
//
// The array is kNoallocScratchBytes long and every GPU that loads this library
// holds its own copy until the process exits. All calls on a device share it
// and it keeps whatever the previous call left there; the arrival counters
// that must start at zero are cleared (cudaMemsetAsync, no allocation) at the
// start of every accepted call. Calls whose execution overlaps on the GPU
// (different streams, or different host threads) race on the array and must be
// ordered by the caller.
//
// Kernel-side failures (a bounded wait that expired, a page-table record
// outside the arena) are recorded in the array's error word, which no call
// clears: rfsn_noalloc_check reads it (after the stream's work is done) and
// resets it, like rfsn_workspace_check does for a caller's workspace. An
// error therefore stays visible until it is checked.
//
// The device address of the array is looked up with cudaGetSymbolAddress the
// first time the entry point runs on each device, with that device current.
// That first call on a device therefore performs set-up work and should be
// made before any CUDA stream capture begins.
#include <mutex>
#include <string>

#include "params.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = RFSN_NOALLOC_SCRATCH_BYTES;

// File-scope device scratch (zero at module load). In host code this name is
// only a stand-in for the symbol; its device address comes from
// cudaGetSymbolAddress below and is the only pointer passed to kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {nullptr};

rfsn_status scratch_address(void** out) {
    int dev = 0;
    RFSN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        rfsn::set_error("rfsn_paged_attention_noalloc: device index %d above %d", dev, kMaxDevices - 1);
        return RFSN_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return rfsn::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(g_noalloc_scratch)");
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return RFSN_OK;
}

}  // namespace

extern "C" rfsn_status rfsn_paged_attention_noalloc(const rfsn_arena* arena, const float* q, int batch, int q_heads,
                                                    int kv_heads, int q_len, int q_pos0, const rfsn_page_table* table,
                                                    const rfsn_hot_window* hot, float* out, float* lse, int max_splits,
                                                    void* stream) {
    RFSN_CHECK_ARG(arena != nullptr && table != nullptr && hot != nullptr,
                   "rfsn_paged_attention_noalloc: NULL arena/table/hot");
    RFSN_CHECK_ARG(q != nullptr && out != nullptr, "rfsn_paged_attention_noalloc: NULL q/out");
    void* scratch = nullptr;
    rfsn_status st = scratch_address(&scratch);
    if (st != RFSN_OK) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Every check of the real call first (shape, page table, hot window, the
    // scratch size the chosen kernel needs), without launching: a rejected call
    // issues no CUDA work and leaves the shared array as it was.
    st = rfsn::paged_attention_impl(arena, q, batch, q_heads, kv_heads, q_len, q_pos0, table, hot, out, lse, scratch,
                                    kNoallocScratchBytes, max_splits, nullptr, s, /*dry_run=*/true);
    if (st == RFSN_ERR_OVERFLOW) {
        // The shape needs more split scratch than the built-in array holds.
        const std::string inner = rfsn_last_error();
        rfsn::set_error(
            "rfsn_paged_attention_noalloc: the built-in scratch holds %zu bytes and this call needs more (%s); pass "
            "a smaller max_splits or use rfsn_paged_attention with a caller-provided workspace",
            kNoallocScratchBytes, inner.c_str());
    }
    if (st != RFSN_OK) return st;
    // The arrival counters must start at zero; the error word (offset 0) is left
    // for rfsn_noalloc_check.
    RFSN_CUDA(cudaMemsetAsync(static_cast<char*>(scratch) + 256, 0, sizeof(int) * (size_t)rfsn::kMaxCounters, s));
    return rfsn::paged_attention_impl(arena, q, batch, q_heads, kv_heads, q_len, q_pos0, table, hot, out, lse, scratch,
                                      kNoallocScratchBytes, max_splits, nullptr, s);
}

extern "C" rfsn_status rfsn_noalloc_check(void* stream, int64_t timeout_us) {
    void* scratch = nullptr;
    rfsn_status st = scratch_address(&scratch);
    if (st != RFSN_OK) return st;
    return rfsn_workspace_check(scratch, stream, timeout_us);
}
