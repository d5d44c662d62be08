// Shared device/host helpers for the rfsn_b200 kernels (sm_100a).
//
// PTX wrappers are written from the public PTX ISA: mbarrier (init, arrive,
// expect_tx, try_wait.parity), cp.async.bulk.tensor (TMA tiled loads),
// ldmatrix / movmatrix, and mma.sync m16n8k16 with float32 accumulation.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rfsn_b200.h"

namespace rfsn {

// ------------------------------------------------------------------------------------------
// host-side error plumbing
// ------------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void note_launch();
rfsn_status cuda_status(cudaError_t e, const char* what);

#define RFSN_CHECK_ARG(cond, ...)          \
    do {                                   \
        if (!(cond)) {                     \
            ::rfsn::set_error(__VA_ARGS__); \
            return RFSN_ERR_INVALID_ARG;   \
        }                                  \
    } while (0)

#define RFSN_CUDA(call)                                                  \
    do {                                                                 \
        cudaError_t _e = (call);                                         \
        if (_e != cudaSuccess) return ::rfsn::cuda_status(_e, #call);    \
    } while (0)

inline int dtype_size(int dt) { return dt == RFSN_F32 ? 4 : 2; }

// ------------------------------------------------------------------------------------------
// element conversion
// ------------------------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// ------------------------------------------------------------------------------------------
// shared-memory / barrier PTX
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ long long global_ns() {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase. try_wait suspends the thread for a
// hardware-defined interval per attempt (long enough that a count of attempts
// is no bound on the time), so the limit is taken on the global timer: the
// wait gives up (returns false) after kWaitNs, or early once *abort_flag (if
// given) becomes non-zero.
constexpr long long kWaitNs = 2000000000LL;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, const int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 0) {
            if (abort_flag != nullptr && *(volatile const int*)abort_flag) return false;
            if (global_ns() - t0 > kWaitNs) return false;
        }
    }
}

// TMA: 2-D tiled bulk tensor load global -> shared, completion on an mbarrier.
// No multicast: every CTA fetches its own tiles.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch (sm_90+). In a kernel launched with the
// programmatic-stream-serialization attribute, griddep_wait() blocks until the
// preceding kernel in the stream has completed and its memory is visible;
// griddep_launch_dependents() lets the next such kernel start launching. Both
// are no-ops in kernels launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel on the stream runs (once that one triggers its
// dependents) and must call griddep_wait() before reading what it produced.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------------------------------
// warp-level matrix PTX
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

template <typename T> struct MmaOp;

template <> struct MmaOp<__nv_bfloat16> {
    __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

template <> struct MmaOp<__half> {
    __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// Pack two float32 values into a 16-bit pair (lo in bits 0..15), RNE.
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Split x into a 16-bit "head" h = round(x) and the 16-bit rounding of the
// remainder x - h, so that h + r carries about 16 significand bits of x: the
// two-term split used to recover single-precision products from 16-bit tensor
// core operands (Markidis et al., "NVIDIA Tensor Core Programmability,
// Performance & Precision", IPDPSW 2018; Ootomo & Yokota, IJHPCA 2022).
template <typename T> __device__ __forceinline__ float round16(float x) { return to_f32<T>(from_f32<T>(x)); }

// ------------------------------------------------------------------------------------------
// workspace layout shared by the attention kernels
// ------------------------------------------------------------------------------------------
// [0, 256)          header: int32 error word at offset 0
// [256, 256 + C)    int32 arrival counters, one per (bh, q-block), zero between
//                   calls; a fixed-size region so that calls of different shapes
//                   sharing one workspace never see each other's partials there
// then              float partial max   [groups][splits][slots]
//                   float partial sum   [groups][splits][slots]
//                   float partial out   [groups][splits][slots][head_dim]
// where groups = batch * kv_heads and slots = q_len * (q_heads / kv_heads).
struct WsLayout {
    size_t counters_off, m_off, l_off, o_off, total;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr int kMaxCounters = 16384;  // groups * q-blocks per call

inline WsLayout ws_layout(int groups, int qblocks, int splits, int slots, int head_dim) {
    WsLayout w;
    w.counters_off = 256;
    (void)qblocks;
    size_t off = w.counters_off + sizeof(int) * (size_t)kMaxCounters;
    w.m_off = off;
    off = align_up(off + sizeof(float) * (size_t)groups * splits * slots, 256);
    w.l_off = off;
    off = align_up(off + sizeof(float) * (size_t)groups * splits * slots, 256);
    w.o_off = off;
    off = align_up(off + sizeof(float) * (size_t)groups * splits * slots * head_dim, 256);
    w.total = off;
    return w;
}

// Device-side view of the workspace.
struct WsView {
    int* error;
    int* counters;
    float* m;
    float* l;
    float* o;
};

inline WsView ws_view(void* base, const WsLayout& w) {
    char* b = static_cast<char*>(base);
    return WsView{reinterpret_cast<int*>(b), reinterpret_cast<int*>(b + w.counters_off),
                  reinterpret_cast<float*>(b + w.m_off), reinterpret_cast<float*>(b + w.l_off),
                  reinterpret_cast<float*>(b + w.o_off)};
}

// Error words written by kernels into the workspace header.
constexpr int kDevErrTimeout = 1;
constexpr int kDevErrBadTable = 2;  // a page-table record points outside the arena

// Cross-GPU exchange of the fused sharded merge (see peer.cu). Each rank owns
// a mailbox in its HBM that every peer maps with CUDA IPC:
//   poison int32            set once a wait for a peer has expired (local only):
//                           the ranks' call stamps may then disagree, so later
//                           calls skip the exchange and report the timeout again
//   calls  int32 [groups]   this rank's call counter per group (local only)
//   words  uint2 [2][kMaxPeers][groups][kPeerSlots][head_dim + 2]
//          (call parity, source rank, group, query slot; head_dim output
//          words, the LSE word, one pad word). Each 8-byte word is
//          {float bits, call stamp}: a receiver knows a word has arrived
//          when its stamp equals the current call, so data needs no separate
//          flag and no fence (low-latency "data + flag" words written with
//          16-byte stores, the scheme NCCL's LL protocol uses).
constexpr int kMaxPeers = 8;
constexpr int kPeerSlots = 4;
constexpr int kDevErrPeerTimeout = 3;

struct PeerParams {
    int world;                     // 0: no cross-GPU merge
    int rank;
    uint2* words[kMaxPeers];       // every rank's word region (own one included)
    int* calls;                    // own call counters
    int* poison;                   // own group-state word: non-zero once a peer wait has expired
    long long timeout_ns;          // bounded wait for peers
};

__device__ __forceinline__ void st_volatile_v4(uint2* p, uint32_t a, uint32_t fa, uint32_t b, uint32_t fb) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(fa), "r"(b), "r"(fb)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_volatile_v4(const uint2* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// 16-byte global -> shared copies that bypass registers (L2 only), and the
// wait for this thread's outstanding ones.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32: about 2 ulp,
// results below 2^-126 flush to +0, 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// Arrival counter of a split merge: release orders the CTA's partial-result
// stores (made visible to this thread by the preceding CTA barrier) before the
// increment; acquire makes the other CTAs' released stores visible to the CTA
// that sees the last arrival (shared with its threads by the next barrier).
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Output addressing: slot j of kv group (b, hk) is query row r = j / G of q
// head hk * G + j % G (GQA head mapping of layer.py:140-150).
struct OutMap {
    int q_heads, kv_heads, q_len, head_dim, groups_per_kv;
    __device__ __forceinline__ size_t row(int bh, int slot) const {
        int b = bh / kv_heads, hk = bh % kv_heads;
        int r = slot / groups_per_kv, g = slot % groups_per_kv;
        return ((size_t)(b * q_heads + hk * groups_per_kv + g) * q_len + r);
    }
};

}  // namespace rfsn
