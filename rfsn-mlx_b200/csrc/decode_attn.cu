// Split-KV exact decode attention over an arena page table + hot ring (sm_100a).
//
// Replaces the per-step work of layer.py:139-162 (segment walk, GQA
// mx.repeat, run_segmented_attention / exact_attention) for bf16/f16 K/V with
// head_dim 128 and up to 4 (query row, q head) slots per KV head, i.e.
// batch-1 decode with GQA groups of <= 4.
//
// Work decomposition: the keys of one (batch, kv head) group are the tiles of
// the archived blocks (page-table order) followed by the hot-window pieces;
// each CTA takes a contiguous range of tiles (grid = splits x groups). Within
// a CTA one producer warp streams 64-key K/V tiles into a STAGES-deep
// shared-memory ring with TMA (128B-swizzled boxes; 8-row boxes for the
// ragged last tile of a span so no bytes beyond the span are fetched), and
// four consumer warps each own a 16-key strip of every tile:
//   S^T[16 keys x 8] = K[16 x 128] . Q^T[128 x 8]      (mma.sync m16n8k16)
//   O^T[128 x 8]    += V^T[128 x 16] . P^T[16 x 8]
// The 8 columns are the 4 query slots twice: a 16-bit head and a 16-bit
// remainder of the float32 operand (q after scaling; p after exp), so the
// contraction keeps ~16 significand bits of q and p while K/V enter exactly,
// with float32 accumulation. The P^T operand is produced from the S^T
// accumulator fragment with one movmatrix transpose per 8x8 block. Online
// softmax runs in float32 (exp2 on log2-scaled scores) with warp shuffles;
// partials are merged across warps in shared memory and across splits by the
// last CTA of each group (finish_splits).
#include <math_constants.h>

#include "attn_common.cuh"
#include "params.cuh"

namespace rfsn {
namespace fast {

constexpr int D = 128;
constexpr int NCW = 4;                       // consumer warps (one 16-key strip each)
constexpr int NTHREADS = (NCW + 1) * 32;     // + one producer warp
constexpr int SLOTS = 4;                     // query slots per KV head handled
constexpr int HALF_BYTES = kTile * 128;      // 64 rows x 64 elements x 2 B
// The split merge keeps 2 * nslots * (splits + 1) floats in red_o (NCW * SLOTS * D floats).
constexpr int MAX_SPLITS = 240;


template <int STAGES>
struct Smem {
    uint8_t k[STAGES][2][HALF_BYTES];
    uint8_t v[STAGES][2][HALF_BYTES];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    int2 tinfo[STAGES];
    float red_m[NCW][SLOTS];
    float red_l[NCW][SLOTS];
    alignas(16) float red_o[NCW][SLOTS][D];
    int flag;
    int abort;
    int call;  // cross-GPU merge: this call's stamp for the group
};

// K and V stage buffers are contiguous (k then v): the merge staging area in float4.
template <int STAGES>
constexpr int stage_vec4() { return STAGES * 2 * 2 * HALF_BYTES / 16; }

template <typename T, int STAGES>
__global__ void __launch_bounds__(NTHREADS, 2)
paged_decode_kernel(const __grid_constant__ CUtensorMap mapK64, const __grid_constant__ CUtensorMap mapV64,
                    const __grid_constant__ CUtensorMap mapK8, const __grid_constant__ CUtensorMap mapV8,
                    const Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem<STAGES>& sm = *reinterpret_cast<Smem<STAGES>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, bh = blockIdx.y;
    // Query position and hot window: launch arguments, or a device step state
    // (RFSN_STEP_*) read when the kernel runs. The state may be written by the
    // work this launch overlaps, so it is read after the dependency wait, and
    // the number of hot tiles follows from it; the split ranges were planned on
    // the host for the largest window the ring holds, so a split's archived
    // tiles are known before the wait and the producer streams them first.
    int q_pos0 = p.q_pos0, head = p.head, hlen = p.hlen, hstart = p.hstart;
    int total_tiles = p.total_tiles;
    const int tiles_per_split = p.tiles_per_split;
    const int tile0 = split * tiles_per_split;
    auto read_state = [&](bool report) {
        q_pos0 = p.dyn[0];
        head = p.dyn[2];
        hlen = p.dyn[3];
        hstart = p.dyn[4];
        if (head < 0 || head >= p.capacity || hlen < 0 || hlen > p.capacity) {  // malformed: attend to no hot key
            if (report) atomicExch(p.ws.error, kDevErrBadTable);
            head = 0;
            hlen = 0;
        }
        const int first = min(hlen, p.capacity - head);
        total_tiles = p.archived_tiles + (first + kTile - 1) / kTile + (hlen - first + kTile - 1) / kTile;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], NCW);
        }
        sm.abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer: one elected lane issues all TMA loads ----------------
        const bool dyn = p.dyn != nullptr;
        bool have_state = !dyn;
        if (dyn && tile0 >= p.archived_tiles) {  // the split starts in the hot window
            griddep_wait();
            read_state(false);
            have_state = true;
        }
        // without the state, the split's archived tiles are the ones certainly there
        int ntiles = min(tiles_per_split, (have_state ? total_tiles : p.archived_tiles) - tile0);
        PagedCursor cur;
        if (ntiles > 0) {
            if (lane == 0) {
                prefetch_tmap(&mapK64);
                prefetch_tmap(&mapV64);
                prefetch_tmap(&mapK8);
                prefetch_tmap(&mapV8);
            }
            cur.records = p.records;
            cur.n_blocks = p.n_blocks;
            cur.archived_tiles = p.archived_tiles;
            if (have_state) cur.init_hot(p.ring_row0, p.capacity, head, hlen, hstart);
            cur.seek_warp(tile0);  // an archived tile when the hot window is not known yet
        }
        if (lane == 0 && ntiles > 0) {
            const int row_base = bh * p.rows;
            bool waited = dyn && have_state;
            for (int it = 0; it < ntiles; ++it) {
                const int s = it % STAGES;
                if (it >= STAGES) {
                    if (!mbar_wait_bounded(&sm.empty[s], ((it / STAGES) + 1) & 1, &sm.abort)) {
                        atomicExch(&sm.abort, 1);
                        atomicExch(p.ws.error, kDevErrTimeout);
                        break;
                    }
                }
                TileRef t = cur.current();
                if (!waited && t.span >= p.n_blocks) {
                    // hot-window rows may be written by the kernel this one overlaps (ring append)
                    griddep_wait();
                    waited = true;
                }
                if (t.row < 0 || t.row + t.nvalid > p.rows) {
                    // corrupt record: flag it and stream nothing useful (keys masked out)
                    atomicExch(p.ws.error, kDevErrBadTable);
                    t.row = 0;
                    t.nvalid = 0;
                }
                sm.tinfo[s] = make_int2(t.kpos0, t.nvalid);
                const int grow = row_base + t.row;
                if (t.nvalid == kTile) {
                    mbar_arrive_expect_tx(&sm.full[s], 4 * HALF_BYTES);
                    tma_load_2d(sm.k[s][0], &mapK64, 0, grow, &sm.full[s]);
                    tma_load_2d(sm.k[s][1], &mapK64, 64, grow, &sm.full[s]);
                    tma_load_2d(sm.v[s][0], &mapV64, 0, grow, &sm.full[s]);
                    tma_load_2d(sm.v[s][1], &mapV64, 64, grow, &sm.full[s]);
                } else if (t.nvalid == 0) {
                    mbar_arrive(&sm.full[s]);  // nothing to load
                } else {
                    const int nb = (t.nvalid + 7) >> 3;  // 8-row boxes, 1 KB each
                    mbar_arrive_expect_tx(&sm.full[s], nb * 4 * 1024);
                    for (int b = 0; b < nb; ++b) {
                        tma_load_2d(sm.k[s][0] + b * 1024, &mapK8, 0, grow + 8 * b, &sm.full[s]);
                        tma_load_2d(sm.k[s][1] + b * 1024, &mapK8, 64, grow + 8 * b, &sm.full[s]);
                        tma_load_2d(sm.v[s][0] + b * 1024, &mapV8, 0, grow + 8 * b, &sm.full[s]);
                        tma_load_2d(sm.v[s][1] + b * 1024, &mapV8, 64, grow + 8 * b, &sm.full[s]);
                    }
                }
                if (!have_state && tile0 + it + 1 >= p.archived_tiles) {
                    // the next tile is a hot one: the window's rows and the split's
                    // tile count come from the step state (before the cursor moves on)
                    griddep_wait();
                    waited = true;
                    read_state(false);
                    have_state = true;
                    ntiles = min(tiles_per_split, total_tiles - tile0);
                    cur.init_hot(p.ring_row0, p.capacity, head, hlen, hstart);
                }
                cur.advance();
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int g = lane >> 2, t4 = lane & 3;
    const bool hi_lane = (t4 & 2) == 0;
    const int sl0 = 2 * (t4 & 1);
    const OutMap om{p.q_heads, p.kv_heads, p.q_len, D, p.groups_per_kv};

    // Q^T operand fragments: column n = g holds slot n & 3; n < 4 the 16-bit
    // head of q*qscale, n >= 4 the 16-bit remainder.
    // q (and the workspace written later) may come from the kernel this one
    // overlaps under programmatic dependent launch: wait for it first.
    griddep_wait();
    if (p.dyn != nullptr) read_state(threadIdx.x == 0 && split == 0 && bh == 0);
    const int ntiles = min(tiles_per_split, total_tiles - tile0);
    if (threadIdx.x == 0) sm.call = p.peer.world > 0 ? p.peer.calls[bh] + 1 : 0;
    uint32_t qf[8][2];
    {
        const int slot = g & 3;
        const bool head_part = g < 4;
        const bool live = slot < p.nslots;
        const float* qrow = p.q + om.row(bh, live ? slot : 0) * D;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int d = 16 * kk + 2 * t4 + 8 * hh;
                float x0 = live ? qrow[d] * p.qscale : 0.f;
                float x1 = live ? qrow[d + 1] * p.qscale : 0.f;
                const float h0 = round16<T>(x0), h1 = round16<T>(x1);
                qf[kk][hh] = head_part ? pack2<T>(h0, h1) : pack2<T>(x0 - h0, x1 - h1);
            }
        }
    }
    const int qp0 = q_pos0 + sl0 / p.groups_per_kv;
    const int qp1 = q_pos0 + (sl0 + 1) / p.groups_per_kv;

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;

    const int mi = lane >> 3, ri = lane & 7;
    // ldmatrix row owned by this lane for the K (non-transposed) and V (transposed) loads
    const int kkey = 16 * warp + ri + 8 * (mi & 1);
    const int kchunk_add = mi >> 1;
    const int vkey = 16 * warp + ri + 8 * (mi >> 1);
    const int vchunk_add = mi & 1;

    int consumed = 0;
    for (int it = 0; it < ntiles; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait_bounded(&sm.full[s], (it / STAGES) & 1, &sm.abort)) {
            atomicExch(&sm.abort, 1);
            atomicExch(p.ws.error, kDevErrTimeout);
            break;
        }
        consumed = it + 1;
        const int2 ti = sm.tinfo[s];
        const int sv = ti.y - 16 * warp;  // valid keys in this warp's strip
        if (sv > 0) {
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t kb = smem_u32(sm.k[s][0]);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int chunk = (kk & 3) * 2 + kchunk_add;
                const uint32_t addr = kb + (kk >> 2) * HALF_BYTES + kkey * 128 + ((chunk ^ (kkey & 7)) << 4);
                uint32_t a[4];
                ldmatrix_x4(a, addr);
                MmaOp<T>::run(c, a, qf[kk][0], qf[kk][1]);
            }
            float sc[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[j] = c[j] + __shfl_xor_sync(0xffffffffu, c[j], 2);
            const int k0 = 16 * warp + g, k1 = k0 + 8;
            const int kp0 = ti.x + k0, kp1 = ti.x + k1;
            if (!(k0 < ti.y && kp0 <= qp0)) sc[0] = -CUDART_INF_F;
            if (!(k0 < ti.y && kp0 <= qp1)) sc[1] = -CUDART_INF_F;
            if (!(k1 < ti.y && kp1 <= qp0)) sc[2] = -CUDART_INF_F;
            if (!(k1 < ti.y && kp1 <= qp1)) sc[3] = -CUDART_INF_F;
            float tm0 = fmaxf(sc[0], sc[2]), tm1 = fmaxf(sc[1], sc[3]);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
                tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
            }
            const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);
            const float al0 = (mn0 == -CUDART_INF_F) ? 1.f : exp2f(m0 - mn0);
            const float al1 = (mn1 == -CUDART_INF_F) ? 1.f : exp2f(m1 - mn1);
            const float ms0 = (mn0 == -CUDART_INF_F) ? 0.f : mn0;
            const float ms1 = (mn1 == -CUDART_INF_F) ? 0.f : mn1;
            float pv[4];
            pv[0] = exp2f(sc[0] - ms0);
            pv[1] = exp2f(sc[1] - ms1);
            pv[2] = exp2f(sc[2] - ms0);
            pv[3] = exp2f(sc[3] - ms1);
            m0 = mn0;
            m1 = mn1;
            l0 = l0 * al0 + pv[0] + pv[2];
            l1 = l1 * al1 + pv[1] + pv[3];
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
                acc[dt][0] *= al0;
                acc[dt][1] *= al1;
                acc[dt][2] *= al0;
                acc[dt][3] *= al1;
            }
            float e[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float x = pv[j] * p.pscale;
                const float h = round16<T>(x);
                e[j] = hi_lane ? h : (x - h);
            }
            const uint32_t b0 = movmatrix_trans(pack2<T>(e[0], e[1]));
            const uint32_t b1 = movmatrix_trans(pack2<T>(e[2], e[3]));
            uint32_t m01 = 0xffffffffu, m23 = 0xffffffffu;
            if (sv < 16) {
                const int ka = 2 * t4;
                m01 = (ka < sv ? 0x0000ffffu : 0u) | (ka + 1 < sv ? 0xffff0000u : 0u);
                m23 = (ka + 8 < sv ? 0x0000ffffu : 0u) | (ka + 9 < sv ? 0xffff0000u : 0u);
            }
            const uint32_t vb = smem_u32(sm.v[s][0]);
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
                const int chunk = (dt & 3) * 2 + vchunk_add;
                const uint32_t addr = vb + (dt >> 2) * HALF_BYTES + vkey * 128 + ((chunk ^ (vkey & 7)) << 4);
                uint32_t a[4];
                ldmatrix_x4_trans(a, addr);
                a[0] &= m01;
                a[1] &= m01;
                a[2] &= m23;
                a[3] &= m23;
                MmaOp<T>::run(acc[dt], a, b0, b1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
    }

    griddep_launch_dependents();
    if (sm.abort) {
        // Drain: wait (bounded) for loads already issued into stages we did not consume.
        for (int it = consumed; it < min(ntiles, consumed + STAGES); ++it) {
            mbar_wait_bounded(&sm.full[it % STAGES], (it / STAGES) & 1, nullptr);
        }
    }

    // ---------------- warp -> CTA merge ----------------
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
#pragma unroll
    for (int dt = 0; dt < 8; ++dt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[dt][j] += __shfl_xor_sync(0xffffffffu, acc[dt][j], 2);
    if (hi_lane) {
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
            sm.red_o[warp][sl0][16 * dt + g] = acc[dt][0];
            sm.red_o[warp][sl0 + 1][16 * dt + g] = acc[dt][1];
            sm.red_o[warp][sl0][16 * dt + g + 8] = acc[dt][2];
            sm.red_o[warp][sl0 + 1][16 * dt + g + 8] = acc[dt][3];
        }
        if (g == 0) {
            sm.red_m[warp][sl0] = m0;
            sm.red_m[warp][sl0 + 1] = m1;
            sm.red_l[warp][sl0] = l0;
            sm.red_l[warp][sl0 + 1] = l1;
        }
    }
    named_barrier_sync(1, NCW * 32);

    const int part_base = bh * p.splits * SLOTS;
    if (warp < p.nslots) {
        // one warp per query slot, lane = output float4: the CTA partial of the slot
        const int slot = warp;
        float mw[NCW];
        float M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < NCW; ++w) {
            mw[w] = sm.red_m[w][slot];
            M = fmaxf(M, mw[w]);
        }
        float L = 0.f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        if (M != -CUDART_INF_F) {
#pragma unroll
            for (int w = 0; w < NCW; ++w) {
                const float wt = exp2f(mw[w] - M);
                const float4 o = reinterpret_cast<const float4*>(sm.red_o[w][slot])[lane];
                L += wt * sm.red_l[w][slot];
                O.x += wt * o.x;
                O.y += wt * o.y;
                O.z += wt * o.z;
                O.w += wt * o.w;
            }
        }
        const float inv_ps = 1.f / p.pscale;
        const int pidx = part_base + split * SLOTS + slot;
        reinterpret_cast<float4*>(p.ws.o + (size_t)pidx * D)[lane] =
            make_float4(O.x * inv_ps, O.y * inv_ps, O.z * inv_ps, O.w * inv_ps);
        if (lane == 0) {
            p.ws.m[pidx] = M;
            p.ws.l[pidx] = L;
        }
    }
    // The split merge reuses red_o as scratch once every consumer thread is past
    // the reads above (finish_splits starts with a barrier).
    // The K/V stages are idle now (every load issued was consumed or drained):
    // the last CTA stages all splits' partial outputs there in one round trip.
    finish_splits(p.ws, bh, part_base, SLOTS, p.splits, 0, p.nslots, D, om, bh, p.out, p.lse, &sm.flag,
                  &sm.red_o[0][0][0], 1, NCW * 32, p.peer.world > 0 ? &p.peer : nullptr, sm.call,
                  reinterpret_cast<float4*>(&sm.k[0][0][0]), stage_vec4<STAGES>());
}

template <typename T, int STAGES>
rfsn_status launch(const CUtensorMap* maps, const Params& p, cudaStream_t stream) {
    const size_t smem = sizeof(Smem<STAGES>) + 1024;
    auto kern = paged_decode_kernel<T, STAGES>;
    RFSN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, p.groups);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    RFSN_CUDA(cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], p));
    note_launch();
    return RFSN_OK;
}

}  // namespace fast

int fast_max_splits() { return fast::MAX_SPLITS; }

void preload_fast_kernels() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, fast::paged_decode_kernel<__nv_bfloat16, 3>);
    cudaFuncGetAttributes(&a, fast::paged_decode_kernel<__half, 3>);
}

rfsn_status fast_launch(int dtype, const CUtensorMap* maps, const fast::Params& p, int stages, cudaStream_t stream) {
    if (stages != 3) {
        set_error("fast decode kernel: unsupported stage count %d", stages);
        return RFSN_ERR_UNSUPPORTED;
    }
    if (dtype == RFSN_BF16) return fast::launch<__nv_bfloat16, 3>(maps, p, stream);
    if (dtype == RFSN_F16) return fast::launch<__half, 3>(maps, p, stream);
    set_error("fast decode kernel: unsupported dtype %d", dtype);
    return RFSN_ERR_UNSUPPORTED;
}

}  // namespace rfsn
