// Split-KV exact segmented attention on CUDA cores, float32 throughout.
//
// Covers every shape the tensor-core decode kernel does not: float32 caches
// (the reference's float32 model dtype), head_dim other than 128 (up to 256),
// more than four (query row, head) slots per KV head (prefill chunks, larger
// GQA groups), and arbitrary segment lists passed by address
// (run_segmented_attention over tensors that are not in an arena,
// attention_exact.py:122-164). One CTA handles up to 8 query slots of one
// (batch, kv head) group over a contiguous range of 64-key tiles; keys are
// staged 32 at a time in shared memory as float32, scores and the online
// softmax are float32, and the splits are merged in-kernel (finish_splits).
#include <math_constants.h>

#include "attn_common.cuh"
#include "params.cuh"

namespace rfsn {
namespace generic {

constexpr int NT = 128;   // threads per CTA
constexpr int QB = 8;     // query slots per CTA
constexpr int KC = 32;    // keys staged per step
constexpr int MAX_D = 256;


// Segment-list cursor: same walk as PagedCursor over caller descriptors.
struct SegCursor {
    const rfsn_segment_desc* segs;
    int n;
    int span, tile_in_span, span_tiles, s_len, s_pos;

    __device__ void load_span(int s) {
        span = s;
        if (s < n) {
            s_len = segs[s].len;
            s_pos = segs[s].pos;
        } else {
            s_len = 0;
            s_pos = 0;
        }
        span_tiles = (s_len + kTile - 1) / kTile;
    }
    __device__ void seek(int gt) {
        int lo = 0, hi = n - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (segs[mid].tile_begin <= gt) lo = mid; else hi = mid - 1;
        }
        load_span(lo);
        tile_in_span = gt - segs[lo].tile_begin;
        while (span_tiles == 0 && span < n) { load_span(span + 1); tile_in_span = 0; }
    }
    __device__ void advance() {
        if (++tile_in_span >= span_tiles) {
            load_span(span + 1);
            tile_in_span = 0;
            while (span_tiles == 0 && span < n) { load_span(span + 1); tile_in_span = 0; }
        }
    }
};

template <typename T, bool PAGED>
__global__ void __launch_bounds__(NT) generic_attn_kernel(const Params p) {
    extern __shared__ float smem[];
    __shared__ int s_flag;
    __shared__ float s_alpha[QB], s_m[QB], s_l[QB];
    __shared__ int s_qpos[QB];

    const int D = p.head_dim;
    float* qs = smem;                    // [QB][D]
    float* ks = qs + QB * D;             // [KC][D + 1]
    float* vs = ks + KC * (D + 1);       // [KC][D]
    float* ps = vs + KC * D;             // [QB][KC]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, bh = blockIdx.y, qblk = blockIdx.z;
    const int slot0 = qblk * QB;
    const int ns = min(QB, p.nslots_total - slot0);
    const OutMap om{p.q_heads, p.kv_heads, p.q_len, D, p.groups_per_kv};

    for (int i = tid; i < QB * D; i += NT) {
        const int sl = i / D, d = i - sl * D;
        qs[i] = sl < ns ? p.q[om.row(bh, slot0 + sl) * D + d] * p.qscale : 0.f;
    }
    if (tid < QB) {
        s_m[tid] = -CUDART_INF_F;
        s_l[tid] = 0.f;
        s_qpos[tid] = p.q_pos0 + (slot0 + tid) / p.groups_per_kv;
    }
    float acc[QB][2];
#pragma unroll
    for (int s = 0; s < QB; ++s) acc[s][0] = acc[s][1] = 0.f;

    const int tile0 = split * p.tiles_per_split;
    const int ntiles = max(0, min(p.tiles_per_split, p.total_tiles - tile0));
    const int b = bh / p.kv_heads, hk = bh % p.kv_heads;

    PagedCursor pc;
    SegCursor sc;
    if (ntiles > 0) {
        if (PAGED) {
            pc.records = p.records;
            pc.n_blocks = p.n_blocks;
            pc.archived_tiles = p.archived_tiles;
            pc.init_hot(p.ring_row0, p.capacity, p.head, p.hlen, p.hstart);
            pc.seek_warp(tile0);
        } else {
            sc.segs = p.segs;
            sc.n = p.n_segs;
            sc.seek(tile0);
        }
    }

    for (int it = 0; it < ntiles; ++it) {
        const T* kbase;
        const T* vbase;
        long kstride, vstride;
        int kpos0, nvalid;
        if (PAGED) {
            const TileRef t = pc.current();
            if (t.row < 0 || t.row + t.nvalid > p.rows) {  // corrupt record: flag it, read nothing
                if (tid == 0) atomicExch(p.ws.error, kDevErrBadTable);
                pc.advance();
                continue;
            }
            kbase = static_cast<const T*>(p.arena_k) + ((long)bh * p.rows + t.row) * D;
            vbase = static_cast<const T*>(p.arena_v) + ((long)bh * p.rows + t.row) * D;
            kstride = vstride = D;
            kpos0 = t.kpos0;
            nvalid = t.nvalid;
            pc.advance();
        } else {
            const rfsn_segment_desc& sd = p.segs[sc.span];
            const int off = sc.tile_in_span * kTile;
            kbase = reinterpret_cast<const T*>(sd.k_ptr) + b * sd.k_stride_b + hk * sd.k_stride_h + off * sd.k_stride_t;
            vbase = reinterpret_cast<const T*>(sd.v_ptr) + b * sd.v_stride_b + hk * sd.v_stride_h + off * sd.v_stride_t;
            kstride = sd.k_stride_t;
            vstride = sd.v_stride_t;
            kpos0 = sc.s_pos + off;
            nvalid = min(kTile, sc.s_len - off);
            sc.advance();
        }
        for (int c0 = 0; c0 < nvalid; c0 += KC) {
            const int nk = min(KC, nvalid - c0);
            __syncthreads();
            for (int i = tid; i < KC * D; i += NT) {
                const int key = i / D, d = i - key * D;
                float kx = 0.f, vx = 0.f;
                if (key < nk) {
                    kx = to_f32<T>(kbase[(long)(c0 + key) * kstride + d]);
                    vx = to_f32<T>(vbase[(long)(c0 + key) * vstride + d]);
                }
                ks[key * (D + 1) + d] = kx;
                vs[key * D + d] = vx;
            }
            __syncthreads();
            for (int i = tid; i < QB * KC; i += NT) {
                const int sl = i / KC, key = i - sl * KC;
                float s = -CUDART_INF_F;
                if (sl < ns && key < nk && kpos0 + c0 + key <= s_qpos[sl]) {
                    const float* qr = qs + sl * D;
                    const float* kr = ks + key * (D + 1);
                    float a = 0.f;
                    for (int d = 0; d < D; ++d) a = fmaf(qr[d], kr[d], a);
                    s = a;
                }
                ps[i] = s;
            }
            __syncthreads();
            for (int sl = warp * 2; sl < warp * 2 + 2; ++sl) {
                const float x = ps[sl * KC + lane];
                float tm = x;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
                const float mold = s_m[sl];
                const float mn = fmaxf(mold, tm);
                const float al = (mn == -CUDART_INF_F) ? 1.f : exp2f(mold - mn);
                const float pv = exp2f(x - ((mn == -CUDART_INF_F) ? 0.f : mn));
                float sum = pv;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                ps[sl * KC + lane] = pv;
                __syncwarp();
                if (lane == 0) {
                    s_l[sl] = s_l[sl] * al + sum;
                    s_m[sl] = mn;
                    s_alpha[sl] = al;
                }
            }
            __syncthreads();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int d = tid + h * NT;
                if (d < D) {
#pragma unroll
                    for (int sl = 0; sl < QB; ++sl) {
                        float a = acc[sl][h] * s_alpha[sl];
                        for (int key = 0; key < nk; ++key) a = fmaf(ps[sl * KC + key], vs[key * D + d], a);
                        acc[sl][h] = a;
                    }
                }
            }
        }
    }
    __syncthreads();

    // write this CTA's partial
    const int part_base = bh * p.splits * p.slots_ws;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int d = tid + h * NT;
        if (d < D) {
            for (int sl = 0; sl < ns; ++sl) {
                const size_t pidx = (size_t)part_base + split * p.slots_ws + slot0 + sl;
                p.ws.o[pidx * D + d] = acc[sl][h];
            }
        }
    }
    if (tid < ns) {
        const int pidx = part_base + split * p.slots_ws + slot0 + tid;
        p.ws.m[pidx] = s_m[tid];
        p.ws.l[pidx] = s_l[tid];
    }
    // finish_splits scratch: reuse the staged-key buffer (>= QB * (MAX_SPLITS + 2) floats for D >= 32)
    finish_splits(p.ws, bh * p.qblocks + qblk, part_base, p.slots_ws, p.splits, slot0, ns, D, om, bh, p.out, p.lse,
                  &s_flag, ks, 1, NT);
}

inline size_t smem_bytes(int D) { return sizeof(float) * ((size_t)QB * D + (size_t)KC * (D + 1) + (size_t)KC * D + QB * KC); }

template <typename T, bool PAGED>
rfsn_status launch(const Params& p, int groups, cudaStream_t stream) {
    const size_t smem = smem_bytes(p.head_dim);
    auto kern = generic_attn_kernel<T, PAGED>;
    RFSN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(p.splits, groups, p.qblocks);
    kern<<<grid, NT, smem, stream>>>(p);
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

}  // namespace generic

void preload_generic_kernels() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, generic::generic_attn_kernel<float, true>);
    cudaFuncGetAttributes(&a, generic::generic_attn_kernel<float, false>);
    cudaFuncGetAttributes(&a, generic::generic_attn_kernel<__half, true>);
    cudaFuncGetAttributes(&a, generic::generic_attn_kernel<__half, false>);
    cudaFuncGetAttributes(&a, generic::generic_attn_kernel<__nv_bfloat16, true>);
    cudaFuncGetAttributes(&a, generic::generic_attn_kernel<__nv_bfloat16, false>);
}

rfsn_status generic_launch(int dtype, bool paged, const generic::Params& p, int groups, cudaStream_t stream) {
    if (p.head_dim > generic::MAX_D) {
        set_error("attention: head_dim %d above %d", p.head_dim, generic::MAX_D);
        return RFSN_ERR_UNSUPPORTED;
    }
    if (dtype == RFSN_F32) return paged ? generic::launch<float, true>(p, groups, stream) : generic::launch<float, false>(p, groups, stream);
    if (dtype == RFSN_F16) return paged ? generic::launch<__half, true>(p, groups, stream) : generic::launch<__half, false>(p, groups, stream);
    if (dtype == RFSN_BF16)
        return paged ? generic::launch<__nv_bfloat16, true>(p, groups, stream) : generic::launch<__nv_bfloat16, false>(p, groups, stream);
    set_error("attention: unsupported dtype %d", dtype);
    return RFSN_ERR_UNSUPPORTED;
}

}  // namespace rfsn
