// Peer groups for the fused cross-GPU merge of sharded decode.
//
// One process per GPU. Each rank allocates a mailbox in its own HBM (layout in
// common.cuh, PeerParams), exports it as a CUDA IPC handle, and maps every
// peer's mailbox (cudaIpcOpenMemHandle; NVLink peer access is enabled lazily).
// rfsn_paged_attention_peer then runs the split-KV decode kernel whose last
// CTA per KV head stamps its (output, LSE) into every rank's mailbox and
// merges the parts of all ranks itself (attn_common.cuh,
// peer_store_and_merge): no collective library call and no extra kernel per
// decode step.
#include <cstring>
#include <vector>

#include "attn_common.cuh"
#include "params.cuh"

struct rfsn_peer_group {
    int world = 0, rank = 0, groups = 0, head_dim = 0, device = 0;
    void* local = nullptr;          // own mailbox (cudaMalloc)
    size_t bytes = 0;
    size_t calls_off = 0, words_off = 0;
    std::vector<void*> mapped;      // mailbox base of every rank (own included)
    bool connected = false;
    long long timeout_ns = 2000000000LL;
};

namespace {

void layout(rfsn_peer_group* g) {
    const size_t calls = sizeof(int) * (size_t)g->groups;
    const size_t words = sizeof(uint2) * 2 * (size_t)rfsn::kMaxPeers * g->groups * rfsn::kPeerSlots * (g->head_dim + 2);
    g->calls_off = 256;
    g->words_off = rfsn::align_up(g->calls_off + calls, 256);
    g->bytes = rfsn::align_up(g->words_off + words, 256);
}

}  // namespace

extern "C" {

rfsn_status rfsn_peer_group_create(int world, int rank, int groups, int head_dim, rfsn_peer_group** out,
                                   void* ipc_handle_out) {
    RFSN_CHECK_ARG(out != nullptr && ipc_handle_out != nullptr, "rfsn_peer_group_create: NULL output");
    RFSN_CHECK_ARG(world >= 1 && world <= rfsn::kMaxPeers, "rfsn_peer_group_create: world %d outside [1, %d]", world,
                   rfsn::kMaxPeers);
    RFSN_CHECK_ARG(rank >= 0 && rank < world, "rfsn_peer_group_create: rank %d outside [0, %d)", rank, world);
    RFSN_CHECK_ARG(groups > 0 && head_dim > 0 && head_dim % 4 == 0, "rfsn_peer_group_create: bad shape");
    rfsn_peer_group* g = new rfsn_peer_group();
    g->world = world;
    g->rank = rank;
    g->groups = groups;
    g->head_dim = head_dim;
    cudaGetDevice(&g->device);
    layout(g);
    cudaError_t e = cudaMalloc(&g->local, g->bytes);
    if (e == cudaSuccess) e = cudaMemset(g->local, 0, g->bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
    if (e != cudaSuccess) {
        if (g->local) cudaFree(g->local);
        delete g;
        return rfsn::cuda_status(e, "rfsn_peer_group_create");
    }
    memcpy(ipc_handle_out, &h, sizeof(h));
    g->mapped.assign(world, nullptr);
    g->mapped[rank] = g->local;
    *out = g;
    return RFSN_OK;
}

int rfsn_peer_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

rfsn_status rfsn_peer_group_connect(rfsn_peer_group* g, const void* all_handles) {
    RFSN_CHECK_ARG(g != nullptr && all_handles != nullptr, "rfsn_peer_group_connect: NULL argument");
    const unsigned char* hs = static_cast<const unsigned char*>(all_handles);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)r * sizeof(h), sizeof(h));
        void* p = nullptr;
        RFSN_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        g->mapped[r] = p;
    }
    g->connected = true;
    return RFSN_OK;
}

rfsn_status rfsn_peer_group_set_timeout(rfsn_peer_group* g, int64_t timeout_us) {
    RFSN_CHECK_ARG(g != nullptr && timeout_us > 0, "rfsn_peer_group_set_timeout: bad argument");
    g->timeout_ns = timeout_us * 1000;
    return RFSN_OK;
}

rfsn_status rfsn_peer_group_destroy(rfsn_peer_group* g) {
    if (g == nullptr) return RFSN_OK;
    for (int r = 0; r < g->world; ++r) {
        if (r != g->rank && g->mapped[r] != nullptr) cudaIpcCloseMemHandle(g->mapped[r]);
    }
    if (g->local) cudaFree(g->local);
    delete g;
    return RFSN_OK;
}

rfsn_status rfsn_paged_attention_peer(const rfsn_arena* arena, const float* q, int batch, int q_heads, int kv_heads,
                                      int q_len, int q_pos0, const rfsn_page_table* table, const rfsn_hot_window* hot,
                                      rfsn_peer_group* peers, float* out, float* lse, void* workspace,
                                      size_t workspace_bytes, int max_splits, void* stream) {
    RFSN_CHECK_ARG(peers != nullptr && peers->connected, "rfsn_paged_attention_peer: peer group not connected");
    RFSN_CHECK_ARG(peers->groups == batch * kv_heads, "rfsn_paged_attention_peer: peer group made for %d groups, "
                   "call has %d", peers->groups, batch * kv_heads);
    RFSN_CHECK_ARG(arena != nullptr && arena->head_dim == peers->head_dim,
                   "rfsn_paged_attention_peer: head_dim differs from the peer group's");
    int dev = 0;
    RFSN_CUDA(cudaGetDevice(&dev));
    RFSN_CHECK_ARG(dev == peers->device, "rfsn_paged_attention_peer: current device %d, peer group on %d", dev,
                   peers->device);
    rfsn::PeerParams pp;
    memset(&pp, 0, sizeof(pp));
    pp.world = peers->world;
    pp.rank = peers->rank;
    for (int r = 0; r < peers->world; ++r) {
        char* base = static_cast<char*>(peers->mapped[r]);
        pp.words[r] = reinterpret_cast<uint2*>(base + peers->words_off);
    }
    pp.calls = reinterpret_cast<int*>(static_cast<char*>(peers->local) + peers->calls_off);
    pp.poison = static_cast<int*>(peers->local);  // header word 0 of the own mailbox
    pp.timeout_ns = peers->timeout_ns;
    return rfsn::paged_attention_impl(arena, q, batch, q_heads, kv_heads, q_len, q_pos0, table, hot, out, lse, workspace,
                                      workspace_bytes, max_splits, &pp, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
