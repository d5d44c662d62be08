// Chunked-prefill exact attention on tcgen05 tensor cores (sm_100a).
//
// The prefill chunk of layer.py:152-162 (q_len = chunk tokens) attends to
// every archived block plus the hot window, causally by absolute position
// (attention_exact.py:27-61, 122-164). This is the dense contraction of the
// path, so it runs on the 5th-generation tensor cores with TMEM accumulators.
//
// CTA = one KV head and 128 query rows packed GQA-style: row r is query head
// (kv_head * G + r % G) at chunk position (base + r / G), so every K/V tile
// staged in shared memory serves all G query heads of its KV head.
//
// float32 accuracy: q and the probabilities P are each split into a 16-bit
// high part and a 16-bit residual (x = hi + lo to ~16 significand bits);
// S = Qhi K^T + Qlo K^T and O += Phi V + Plo V, all accumulated in float32 in
// TMEM, and the softmax scales S by log2(e)/sqrt(d) in float32. K and V are
// stored in 16 bits already, so they enter the products exactly. When every q
// element of the CTA is a 16-bit value (the q of a bf16/fp16 model: projection
// and RoPE round to the model dtype) all residuals are zero and the Qlo K^T
// product, which would add exact zeros, is not issued: 3 products per tile
// instead of 4.
//
// Warps:
//   0-7  softmax: warp w owns TMEM lane quarter w % 4 (32 rows, thread = row)
//        and key half w / 4 (64 of the 128 keys of a tile). They split q into
//        TMEM (the A operand of S: shared memory bandwidth is left to the K/V
//        operands and the TMA fills); per key tile they read their S
//        half from TMEM, apply the causal/validity mask, exchange row maxima
//        with the partner warp (mbarrier per quarter), run the float32 online
//        softmax on exp2, write Phi/Plo back over the S columns (the A operand
//        of the PV product, read from TMEM) and rescale their half of the O row
//        when the reference maximum moves; finally O / l -> out and the
//        log-sum-exp.
//   8    K producer: walks the page table (archived blocks in order, then the
//        hot pieces) in 128-key tiles up to the CTA's causal limit, posts each
//        tile's {position, length} and streams K with TMA into a 3-stage ring
//        (8-row boxes for ragged span ends).
//   9    MMA issuer (one thread): S(t) = Q K(t)^T into S buffer t % 2, then
//        O += P(t-1) V(t-1), both with A from TMEM; tcgen05.commit signals the
//        softmax warps and releases K stages (after S) and V stages (after PV).
//   10   V producer: the same walk, streaming V into a 3-stage ring.
// TMEM: two S/P buffers at columns [0,256), O at [256,384), q hi/lo at [384,512).
// Every mbarrier wait is bounded (error flag + early exit) and TMEM is
// released on every path.
#include <math_constants.h>

#include <type_traits>

#include "attn_common.cuh"
#include "params.cuh"
#include "tcgen05.cuh"

namespace rfsn {
namespace prefill {

constexpr int D = 128;
constexpr int BM = 128;   // rows per CTA (positions x query heads of one KV head)
constexpr int BN = 128;   // keys per tile
constexpr int KST = 3;    // K ring stages (released after S)
constexpr int VST = 3;    // V ring stages (released after PV)
constexpr int NSB = 2;    // S/P buffers in TMEM
// Tile-info ring: slot t % NINFO is rewritten for tile t + NINFO after K stage
// reuse (S(t + NINFO - KST) done), which needs PV(t + NINFO - KST - NSB) done,
// i.e. the softmax of tile t finished when NINFO >= KST + NSB.
constexpr int NINFO = 8;
static_assert(NINFO >= KST + NSB, "tile-info ring too short");
constexpr int SOFTMAX_WARPS = 8;  // two warps per 32-row TMEM quarter, one per 64-key half
constexpr int KPROD_WARP = SOFTMAX_WARPS, MMA_WARP = SOFTMAX_WARPS + 1, VPROD_WARP = SOFTMAX_WARPS + 2;
constexpr int NTHREADS = (SOFTMAX_WARPS + 3) * 32;
constexpr int SOFTMAX_THREADS = SOFTMAX_WARPS * 32;
constexpr int TILE_HALF = BN * 128;  // bytes of one 64-column half of a 128-row tile
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_O = 256;                  // float32 O accumulator, 128 columns
constexpr uint32_t COL_QHI = 384, COL_QLO = 448;  // q as the A operand of S: 16-bit pairs, 64 columns each

struct Smem {
    uint8_t k[KST][2][TILE_HALF];
    uint8_t v[VST][2][TILE_HALF];
    uint64_t k_full[KST], k_empty[KST];  // K stage loaded / free again (after S)
    uint64_t v_full[VST], v_empty[VST];  // V stage loaded / free again (after PV)
    uint64_t info_full[NINFO];           // tile info posted (count 1)
    uint64_t s_full[NSB];                // S(t) in TMEM buffer t % NSB
    uint64_t p_full[NSB];                // P(t) written over it (count: softmax threads)
    uint64_t pv_done[NSB];               // PV(t) complete, per S/P buffer t % NSB
    uint64_t mma_done;
    uint64_t pair[4][2];  // per 32-row quarter and tile parity: both key halves posted their maxima
    uint64_t pair_l[4];   // per quarter: both halves posted their partial sums (end of the stream)
    float red[2][2][BM];  // [tile parity][key half][row] partial maxima; [0][*] reused for sums
    int2 tinfo[NINFO];    // {kpos0, nvalid} per tile (ring); nvalid < 0 marks the end of the key stream
    uint32_t tmem;
    int abort;
    int flag;  // this CTA merges the key-range splits of its query block
    int q_lo;  // some q element of the CTA has a nonzero 16-bit residual
};

// Paired float32 arithmetic (PTX .f32x2, sm_100): two lanes of work per
// instruction issue, each rounded as the scalar operation.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// (a, b) -> packed 16-bit high parts and packed 16-bit residuals (a = hi + lo to
// ~16 significand bits): both packs by the round-to-nearest pair conversion
// (cvt.rn.{bf16x2,f16x2}.f32, one instruction per pair). For bf16 the high parts
// widen back to float32 by a shift or a mask of the packed word, so the exact
// residuals cost two subtractions.
template <typename T>
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    hi = pack2<T>(a, b);
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const float2 r = fsub2(make_float2(a, b), make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u)));
        lo = pack2<T>(r.x, r.y);
    } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hi));
        lo = pack2<T>(a - f.x, b - f.y);
    }
}

// Bounded wait whose result is the same on every lane of the warp, so the
// warp stays converged for the .sync.aligned tcgen05 instructions after it.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* abort_flag) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag));
}

__device__ __forceinline__ void fail(int* abort_flag, const PrefillParams& p) {
    atomicExch(abort_flag, 1);
    atomicExch(p.ws.error, kDevErrTimeout);
}

// The CTA's key stream: archived blocks in table order, then the hot window's
// two ring pieces, cut into tiles of at most BN keys, up to the causal limit.
struct TileWalk {
    int span = 0, off = 0;
    int s_row = 0, s_pos = 0, s_len = 0;

    __device__ __forceinline__ bool load_span(const PrefillParams& p) {
        while (span < p.n_blocks + 2) {
            if (span < p.n_blocks) {
                const int4 r = p.records[span];
                s_row = r.x;
                s_pos = r.y;
                s_len = r.z;
            } else {
                const int first = min(p.hlen, p.capacity - p.head);
                if (span == p.n_blocks) {
                    s_row = p.ring_row0 + p.head;
                    s_pos = p.hstart;
                    s_len = first;
                } else {
                    s_row = p.ring_row0;
                    s_pos = p.hstart + first;
                    s_len = p.hlen - first;
                }
            }
            if (s_len > 0) return true;
            ++span;
        }
        return false;
    }
    // Next tile: key positions [kpos0, kpos0 + nvalid) at arena row `row`.
    __device__ __forceinline__ bool next(const PrefillParams& p, int qlast, int& kpos0, int& row, int& nvalid) {
        if (off == 0 && !load_span(p)) return false;
        kpos0 = s_pos + off;
        if (kpos0 > qlast) return false;  // spans are in increasing position order
        row = s_row + off;
        nvalid = min(BN, s_len - off);
        off += BN;
        if (off >= s_len) {
            off = 0;
            ++span;
        }
        return true;
    }
};

// Tiles in the CTA's key stream (the walk above, counted).
__device__ __forceinline__ int count_tiles(const PrefillParams& p, int qlast) {
    TileWalk w;
    int kpos0, row, nvalid, n = 0;
    while (w.next(p, qlast, kpos0, row, nvalid)) ++n;
    return n;
}

// One K or V tile -> a stage (two 64-column halves): 64-row boxes for a full
// tile, 8-row boxes for a ragged span end.
__device__ __forceinline__ void load_tile(uint8_t (*dst)[TILE_HALF], const CUtensorMap* m64, const CUtensorMap* m8,
                                          int grow, int nvalid, uint64_t* bar) {
    if (nvalid == BN) {
        mbar_arrive_expect_tx(bar, 2 * TILE_HALF);
        for (int hh = 0; hh < 2; ++hh)
            for (int r64 = 0; r64 < 2; ++r64) tma_load_2d(dst[hh] + r64 * 64 * 128, m64, 64 * hh, grow + 64 * r64, bar);
    } else {
        const int nb = (nvalid + 7) >> 3;
        mbar_arrive_expect_tx(bar, nb * 2 * 1024);
        for (int hh = 0; hh < 2; ++hh)
            for (int bb = 0; bb < nb; ++bb) tma_load_2d(dst[hh] + bb * 1024, m8, 64 * hh, grow + 8 * bb, bar);
    }
}

template <typename T>
__global__ void __launch_bounds__(NTHREADS, 1)
prefill_attn_kernel(const __grid_constant__ CUtensorMap mapK64, const __grid_constant__ CUtensorMap mapV64,
                    const __grid_constant__ CUtensorMap mapK8, const __grid_constant__ CUtensorMap mapV8,
                    const PrefillParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // The swizzled operand tiles need 1024-byte alignment; the dynamic window
    // starts aligned when the kernel has no static shared memory (checked).
    if ((smem_u32(smem_raw) & 1023u) != 0) {
        if (threadIdx.x == 0) atomicExch(p.ws.error, kDevErrBadTable);
        return;
    }
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.groups_per_kv;
    const int ppc = BM / G;                                   // chunk positions per CTA
    // Work units (query block, KV head) in launch order: bands of head_group KV
    // heads (so a band's K/V stays in L2 while its waves stream it), inside a
    // band latest query blocks first (the longest causal key ranges) with the
    // band's heads interleaved. The first full_units run whole; each later unit
    // is split into tail_splits key ranges run by consecutive CTAs, and the last
    // of them to finish merges the partial results (so the launch's final wave
    // is evenly filled).
    const int groups = p.batch * p.kv_heads;
    int unit, split, nsplit;
    if ((int)blockIdx.x < p.full_units) {
        unit = blockIdx.x;
        split = 0;
        nsplit = 1;
    } else {
        const int j = blockIdx.x - p.full_units;
        unit = p.full_units + j / p.tail_splits;
        split = j % p.tail_splits;
        nsplit = p.tail_splits;
    }
    const int tail_index = unit - p.full_units;               // counters and partials of split units
    const int band = unit / (p.nqb * p.head_group);
    const int band_heads = min(p.head_group, groups - band * p.head_group);
    const int in_band = unit - band * p.nqb * p.head_group;
    const int qb = p.nqb - 1 - in_band / band_heads;
    const int bh = band * p.head_group + in_band % band_heads;  // b * kv_heads + kv head
    const int b = bh / p.kv_heads, hk = bh % p.kv_heads;
    const int pos_base = qb * ppc;                            // first chunk position of the CTA
    const int qlast = p.q_pos0 + min(pos_base + ppc, p.q_len) - 1;  // causal limit of the CTA

    // ---- set-up: zero the K/V stages (rows past a ragged span end stay finite),
    //      barriers, TMEM ----
    for (int i = tid; i < (KST + VST) * 2 * TILE_HALF / 16; i += NTHREADS) {
        reinterpret_cast<uint4*>(sm.k)[i] = make_uint4(0, 0, 0, 0);
    }
    if (tid == 0) {
        for (int s = 0; s < KST; ++s) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.k_empty[s], 1);
        }
        for (int s = 0; s < VST; ++s) {
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.v_empty[s], 1);
        }
        for (int i = 0; i < NINFO; ++i) mbar_init(&sm.info_full[i], 1);
        for (int i = 0; i < NSB; ++i) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.p_full[i], SOFTMAX_THREADS);
            mbar_init(&sm.pv_done[i], 1);
        }
        mbar_init(&sm.mma_done, 1);
        for (int qd = 0; qd < 4; ++qd) {
            mbar_init(&sm.pair[qd][0], 64);
            mbar_init(&sm.pair[qd][1], 64);
            mbar_init(&sm.pair_l[qd], 64);
        }
        sm.abort = 0;
        sm.q_lo = 0;
        fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        tc::tmem_alloc(&sm.tmem, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sm.tmem;

    if (warp == KPROD_WARP) {
        // ---------------- K producer (+ tile info) ----------------
        if (lane == 0) {
            prefetch_tmap(&mapK64);
            prefetch_tmap(&mapK8);
            int t0 = 0, t1 = 1 << 30;
            if (nsplit > 1) {  // this CTA streams tiles [t0, t1) of the unit's key stream (even shares)
                const int ntile = count_tiles(p, qlast);
                t0 = (int)((long long)split * ntile / nsplit);
                t1 = (int)((long long)(split + 1) * ntile / nsplit);
            }
            TileWalk walk;
            int it = 0, gi = -1, kpos0, row, nvalid;
            while (walk.next(p, qlast, kpos0, row, nvalid)) {
                if (++gi < t0) continue;
                if (gi >= t1) break;
                const int s = it % KST;
                // stage free once S(it - KST) is done
                if (it >= KST && !mbar_wait_bounded(&sm.k_empty[s], ((it / KST) + 1) & 1, &sm.abort)) {
                    fail(&sm.abort, p);
                    break;
                }
                const bool bad = row < 0 || row + nvalid > p.rows;
                if (bad) atomicExch(p.ws.error, kDevErrBadTable);
                sm.tinfo[it % NINFO] = make_int2(kpos0, bad ? 0 : nvalid);
                mbar_arrive(&sm.info_full[it % NINFO]);
                if (bad) {
                    mbar_arrive(&sm.k_full[s]);
                } else {
                    load_tile(sm.k[s], &mapK64, &mapK8, bh * p.rows + row, nvalid, &sm.k_full[s]);
                }
                ++it;
            }
            // K fills in flight land first (bounded): the marker below reuses a K barrier
            for (int j = max(0, it - KST); j < it; ++j) mbar_wait_bounded(&sm.k_full[j % KST], (j / KST) & 1, nullptr);
            // end-of-stream marker: tile info for the softmax warps, a K "fill" for the MMA issuer
            const int s = it % KST;
            if (!sm.abort && (it < KST || mbar_wait_bounded(&sm.k_empty[s], ((it / KST) + 1) & 1, &sm.abort))) {
                sm.tinfo[it % NINFO] = make_int2(0, -1);
                mbar_arrive(&sm.info_full[it % NINFO]);
                mbar_arrive(&sm.k_full[s]);
            } else {
                fail(&sm.abort, p);
            }
        }
    } else if (warp == VPROD_WARP) {
        // ---------------- V producer ----------------
        if (lane == 0) {
            prefetch_tmap(&mapV64);
            prefetch_tmap(&mapV8);
            int t0 = 0, t1 = 1 << 30;
            if (nsplit > 1) {  // this CTA streams tiles [t0, t1) of the unit's key stream (even shares)
                const int ntile = count_tiles(p, qlast);
                t0 = (int)((long long)split * ntile / nsplit);
                t1 = (int)((long long)(split + 1) * ntile / nsplit);
            }
            TileWalk walk;
            int it = 0, gi = -1, kpos0, row, nvalid;
            while (walk.next(p, qlast, kpos0, row, nvalid)) {
                if (++gi < t0) continue;
                if (gi >= t1) break;
                const int s = it % VST;
                // stage free once PV(it - VST) is done
                if (it >= VST && !mbar_wait_bounded(&sm.v_empty[s], ((it / VST) + 1) & 1, &sm.abort)) {
                    fail(&sm.abort, p);
                    break;
                }
                if (row < 0 || row + nvalid > p.rows) {
                    mbar_arrive(&sm.v_full[s]);
                } else {
                    load_tile(sm.v[s], &mapV64, &mapV8, bh * p.rows + row, nvalid, &sm.v_full[s]);
                }
                ++it;
            }
            // V fills in flight land before the CTA can exit
            for (int j = max(0, it - VST); j < it; ++j) mbar_wait_bounded(&sm.v_full[j % VST], (j / VST) & 1, nullptr);
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issuer ----------------
        named_barrier_sync(1, SOFTMAX_THREADS + 32);  // q written into TMEM by the softmax warps
        tc::fence_after_sync();
        if (lane == 0) {
            constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
            const uint32_t id_qk = tc::idesc_f16(kBf16, false, false, BM, BN);
            const uint32_t id_pv = tc::idesc_f16(kBf16, false, true, BM, D);
            const uint32_t tO = tmem + COL_O;
            const int q_parts = sm.q_lo ? 2 : 1;  // written before barrier 1
            bool pending = false;  // tensor-core work issued whose completion is not yet observed
            // t: tile whose S is issued this round; it = t - 1: tile whose PV follows
            for (int t = 0;; ++t) {
                const int it = t - 1;
                const int ks = t % KST;
                if (!mbar_wait_bounded(&sm.k_full[ks], (t / KST) & 1, &sm.abort)) {
                    fail(&sm.abort, p);
                    break;
                }
                const bool issue = sm.tinfo[t % NINFO].y >= 0;
                if (issue) {
                    // S buffer t % NSB last held P(t - NSB): PV(t - NSB) must be done.
                    // Every wait for a PV completion uses the barrier of that PV's
                    // buffer, whose previous phase (PV(t - 2 NSB)) the issuer has already
                    // observed: the parity then names the phase, whatever the order in
                    // which the arrivals of different commits land.
                    if (t >= NSB && !mbar_wait_bounded(&sm.pv_done[t % NSB], ((t / NSB) + 1) & 1, &sm.abort)) {
                        fail(&sm.abort, p);
                        break;
                    }
                    tc::fence_after_sync();
                    // S(t) = Qhi K^T (+ Qlo K^T when q has residuals)
                    const uint32_t tS = tmem + 128 * (t % NSB);
#pragma unroll 1
                    for (int part = 0; part < q_parts; ++part) {
                        const uint32_t tQ = tmem + (part ? COL_QLO : COL_QHI);
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint32_t ka = smem_u32(sm.k[ks][kk >> 2]) + (kk & 3) * 32;
                            tc::mma_f16_ts(tS, tQ + 8 * kk, tc::smem_desc_sw128(ka, 16, 1024), id_qk, part > 0 || kk > 0);
                        }
                    }
                    tc::commit(&sm.s_full[t % NSB]);
                    tc::commit(&sm.k_empty[ks]);
                    pending = true;
                }
                if (it >= 0) {
                    // P(it) in TMEM (and O rescaled): O += Phi V + Plo V
                    const int vs = it % VST;
                    if (!mbar_wait_bounded(&sm.p_full[it % NSB], (it / NSB) & 1, &sm.abort) ||
                        !mbar_wait_bounded(&sm.v_full[vs], (it / VST) & 1, &sm.abort)) {
                        fail(&sm.abort, p);
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t tP = tmem + 128 * (it % NSB);
#pragma unroll 1
                    for (int part = 0; part < 2; ++part) {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint32_t va = smem_u32(sm.v[vs][0]) + kk * 16 * 128;
                            tc::mma_f16_ts(tO, tP + 64 * part + 8 * kk, tc::smem_desc_sw128(va, TILE_HALF, 1024),
                                           id_pv, it > 0 || part > 0 || kk > 0);
                        }
                    }
                    tc::commit(&sm.pv_done[it % NSB]);
                    tc::commit(&sm.v_empty[vs]);
                }
                if (!issue) break;  // end of the key stream
            }
            // drain: no tensor-core work may be in flight when TMEM is released
            // (tcgen05.commit tracks all earlier tensor-core work of this thread)
            if (pending) {
                tc::commit(&sm.mma_done);  // single-use barrier: phase 0 = everything issued
                mbar_wait_bounded(&sm.mma_done, 0, nullptr);
            }
        }
    } else {
        // ---------------- softmax warps ----------------
        // warp w: TMEM lane quarter qd = w % 4 (rows 32 qd + lane), key half ch = w / 4
        const int qd = warp & 3, ch = warp >> 2;
        {
            // q row -> TMEM (A operand layout: row = lane, dims packed in pairs along the
            // columns). Warp w stages dims [64 (w / 4), +64) of the rows of its quarter.
            const int r = 32 * qd + lane;
            const int g = r % G, j = r / G;
            const int qrow = pos_base + j;
            const bool ok_row = j < ppc && qrow < p.q_len;
            const float* src = p.q + (((size_t)b * p.q_heads + hk * G + g) * p.q_len + (ok_row ? qrow : 0)) * D + 64 * ch;
            uint32_t hi[32], lo[32], any_lo = 0;
#pragma unroll
            for (int c = 0; c < 16; ++c) {  // 16 chunks of 4 elements
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                if (ok_row) a = *reinterpret_cast<const float4*>(src + 4 * c);
                split2<T>(a.x, a.y, hi[2 * c], lo[2 * c]);
                split2<T>(a.z, a.w, hi[2 * c + 1], lo[2 * c + 1]);
                any_lo |= lo[2 * c] | lo[2 * c + 1];
            }
            // a residual of 16 zero bits contributes nothing to S: the Qlo product is
            // needed only if some residual of the CTA is nonzero (same value from every
            // writer; barrier 1 orders it before the MMA issuer reads it)
            if (__any_sync(0xffffffffu, any_lo != 0) && lane == 0) sm.q_lo = 1;
            const uint32_t lane_q = (uint32_t)(32 * qd) << 16;
            tc::st_32x32b_x32(tmem + lane_q + COL_QHI + 32 * ch, hi);
            tc::st_32x32b_x32(tmem + lane_q + COL_QLO + 32 * ch, lo);
            tc::wait_st();
        }
        tc::fence_before_sync();
        named_barrier_sync(1, SOFTMAX_THREADS + 32);

        const int r = 32 * qd + lane;  // this thread's row = TMEM lane
        const int g = r % G, j = r / G;
        const int h = hk * G + g;
        const int qrow = pos_base + j;
        const bool row_ok = j < ppc && qrow < p.q_len;
        const int qpos = p.q_pos0 + qrow;
        const uint32_t lane_base = (uint32_t)(32 * qd) << 16;
        const uint32_t tO = tmem + COL_O + lane_base + 64 * ch;
        float m = -CUDART_INF_F, l = 0.f;
        bool failed = false;
        int it = 0;
        for (;; ++it) {
            if (!warp_wait(&sm.info_full[it % NINFO], (it / NINFO) & 1, &sm.abort)) { failed = true; break; }
            const int2 ti = sm.tinfo[it % NINFO];
            if (ti.y < 0) break;
            if (!warp_wait(&sm.s_full[it % NSB], (it / NSB) & 1, &sm.abort)) { failed = true; break; }
            tc::fence_after_sync();
            const uint32_t tS = tmem + 128 * (it % NSB) + lane_base;
            uint32_t sr[64];
            tc::ld_32x32b_x64_sync(tS + 64 * ch, sr);
            // keys [kpos0, kpos0 + nvalid) are valid; causal: key position <= query position
            const int lim = min(ti.y, qpos - ti.x + 1) - 64 * ch;
            float mx[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
            if (__all_sync(0xffffffffu, lim >= 64)) {
#pragma unroll
                for (int c = 0; c < 64; ++c) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(sr[c]));
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    const float x = c < lim ? __uint_as_float(sr[c]) : -CUDART_INF_F;
                    sr[c] = __float_as_uint(x);
                    mx[c & 3] = fmaxf(mx[c & 3], x);
                }
            }
            // S holds q.k unscaled; maxima and probabilities are in units of
            // log2(e)/sqrt(d) (qscale > 0, so the maximum commutes with the scale)
            float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.qscale;
            // row maximum over both key halves
            sm.red[it & 1][ch][r] = tmax;
            mbar_arrive(&sm.pair[qd][it & 1]);
            if (!warp_wait(&sm.pair[qd][it & 1], (it >> 1) & 1, &sm.abort)) { failed = true; break; }
            tmax = fmaxf(tmax, sm.red[it & 1][ch ^ 1][r]);
            // Lazy rescaling: probabilities are taken relative to a reference maximum m
            // that moves only when the row maximum exceeds it by more than 2^8 (or on the
            // first tile). O and l share the reference, so O / l and the log-sum-exp are
            // unchanged; p <= 256 keeps every term far from float32/bf16 overflow. Both
            // warps of a row see the same values and take the same decision.
            const float mn = fmaxf(m, tmax);
            bool rescale = false;
            if (it == 0) {
                m = mn;
            } else {
                rescale = __any_sync(0xffffffffu, mn > m + 8.f);
            }
            float alpha = 1.f;
            if (rescale && mn != m) {
                alpha = (m == -CUDART_INF_F) ? 0.f : tc::ex2(m - mn);
                m = mn;
            }
            const float ms = (m == -CUDART_INF_F) ? 0.f : m;
            const float2 qs2 = make_float2(p.qscale, p.qscale), nms2 = make_float2(-ms, -ms);
            float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const float2 x = ffma2(make_float2(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1])), qs2, nms2);
                const float2 pp = make_float2(tc::ex2(x.x), tc::ex2(x.y));
                rs2[e & 1] = fadd2(rs2[e & 1], pp);
                split2<T>(pp.x, pp.y, hi[e], lo[e]);
            }
            const float rs[4] = {rs2[0].x, rs2[0].y, rs2[1].x, rs2[1].y};
            // P columns: key k of the tile -> 16-bit element k (column k / 2); lo after hi
            tc::st_32x32b_x32(tS + 32 * ch, hi);
            tc::st_32x32b_x32(tS + 64 + 32 * ch, lo);
            l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
            if (rescale) {
                // PV of the previous tile must be done before O is rescaled
                if (!warp_wait(&sm.pv_done[(it - 1) % NSB], ((it - 1) / NSB) & 1, &sm.abort)) { failed = true; break; }
                tc::fence_after_sync();
#pragma unroll 1
                for (int cc = 0; cc < 2; ++cc) {
                    uint32_t rr[32];
                    tc::ld_32x32b_x32_sync(tO + 32 * cc, rr);
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) rr[jj] = __float_as_uint(__uint_as_float(rr[jj]) * alpha);
                    tc::st_32x32b_x32(tO + 32 * cc, rr);
                }
            }
            tc::wait_st();
            tc::fence_before_sync();
            mbar_arrive(&sm.p_full[it % NSB]);
        }
        if (failed) fail(&sm.abort, p);
        // row sum over both key halves. Once the last PV is done the partner has
        // read every maximum posted here (it read them before publishing its P), so
        // red[0] is free for the partial sums.
        bool ok = !failed && it > 0 && warp_wait(&sm.pv_done[(it - 1) % NSB], ((it - 1) / NSB) & 1, &sm.abort);
        if (ok) {
            sm.red[0][ch][r] = l;
            mbar_arrive(&sm.pair_l[qd]);
            ok = warp_wait(&sm.pair_l[qd], 0, &sm.abort);
        }
        ok = ok && __all_sync(0xffffffffu, sm.abort == 0);
        tc::fence_after_sync();
        const float lt = ok ? l + sm.red[0][ch ^ 1][r] : 0.f;
        float* dst = p.out + (((size_t)b * p.q_heads + h) * p.q_len + (row_ok ? qrow : 0)) * D + 64 * ch;
        const float inv = (ok && lt > 0.f) ? 1.f / lt : 0.f;
        if (nsplit > 1) {
            // this split's normalised output and natural-log LSE -> workspace; the last
            // split CTA of the unit combines them (an empty range: LSE -inf)
            const size_t prow = ((size_t)tail_index * nsplit + split) * BM + r;
            float* po = p.ws.o + prow * D + 64 * ch;
#pragma unroll 1
            for (int cc = 0; cc < 2; ++cc) {
                uint32_t rr[32];
                tc::ld_32x32b_x32_sync(tO + 32 * cc, rr);
#pragma unroll
                for (int jj = 0; jj < 32; jj += 4) {
                    *reinterpret_cast<float4*>(po + 32 * cc + jj) =
                        make_float4(__uint_as_float(rr[jj]) * inv, __uint_as_float(rr[jj + 1]) * inv,
                                    __uint_as_float(rr[jj + 2]) * inv, __uint_as_float(rr[jj + 3]) * inv);
                }
            }
            if (ch == 0) p.ws.m[prow] = (ok && lt > 0.f) ? (m + log2f(lt)) * 0.69314718055994531f : -CUDART_INF_F;
            if (!ok && tid == 0 && it > 0) atomicExch(p.ws.error, kDevErrTimeout);
            // release-acquire arrival by one thread between CTA barriers (as finish_splits)
            named_barrier_sync(3, SOFTMAX_THREADS);
            if (tid == 0) sm.flag = atom_add_acq_rel_gpu(&p.ws.counters[tail_index], 1) == nsplit - 1;
            named_barrier_sync(3, SOFTMAX_THREADS);
            if (sm.flag) {
                const size_t base = (size_t)tail_index * nsplit * BM + r;
                float M = -CUDART_INF_F;
                for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(p.ws.m + base + (size_t)s * BM));
                float acc[64];
#pragma unroll
                for (int d = 0; d < 64; ++d) acc[d] = 0.f;
                float L = 0.f;
                for (int s = 0; s < nsplit; ++s) {
                    const float ls = __ldcg(p.ws.m + base + (size_t)s * BM);
                    const float wgt = (M == -CUDART_INF_F) ? 0.f : exp2f((ls - M) * 1.4426950408889634f);
                    L += wgt;
                    const float4* src = reinterpret_cast<const float4*>(p.ws.o + (base + (size_t)s * BM) * D + 64 * ch);
#pragma unroll
                    for (int d4 = 0; d4 < 16; ++d4) {
                        const float4 o4 = __ldcg(src + d4);
                        acc[4 * d4] += wgt * o4.x;
                        acc[4 * d4 + 1] += wgt * o4.y;
                        acc[4 * d4 + 2] += wgt * o4.z;
                        acc[4 * d4 + 3] += wgt * o4.w;
                    }
                }
                const float invL = L > 0.f ? 1.f / L : 0.f;
                if (row_ok) {
#pragma unroll
                    for (int d4 = 0; d4 < 16; ++d4) {
                        *reinterpret_cast<float4*>(dst + 4 * d4) = make_float4(
                            acc[4 * d4] * invL, acc[4 * d4 + 1] * invL, acc[4 * d4 + 2] * invL, acc[4 * d4 + 3] * invL);
                    }
                    if (ch == 0 && p.lse != nullptr) {
                        p.lse[((size_t)b * p.q_heads + h) * p.q_len + qrow] =
                            L > 0.f ? M + logf(L) : -CUDART_INF_F;
                    }
                }
                if (tid == 0) p.ws.counters[tail_index] = 0;  // ready for the next call
            }
        } else {
#pragma unroll 1
            for (int cc = 0; cc < 2; ++cc) {
                uint32_t rr[32];
                tc::ld_32x32b_x32_sync(tO + 32 * cc, rr);
                if (row_ok) {
#pragma unroll
                    for (int jj = 0; jj < 32; jj += 4) {
                        *reinterpret_cast<float4*>(dst + 32 * cc + jj) =
                            ok ? make_float4(__uint_as_float(rr[jj]) * inv, __uint_as_float(rr[jj + 1]) * inv,
                                             __uint_as_float(rr[jj + 2]) * inv, __uint_as_float(rr[jj + 3]) * inv)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
            }
            if (row_ok && ch == 0 && p.lse != nullptr) {
                p.lse[((size_t)b * p.q_heads + h) * p.q_len + qrow] =
                    (ok && lt > 0.f) ? (m + log2f(lt)) * 0.69314718055994531f : -CUDART_INF_F;
            }
            if (!ok && tid == 0 && it > 0) atomicExch(p.ws.error, kDevErrTimeout);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == MMA_WARP) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <typename T>
rfsn_status launch(const CUtensorMap* maps, const PrefillParams& p, cudaStream_t stream) {
    const size_t smem = sizeof(Smem);
    auto kern = prefill_attn_kernel<T>;
    RFSN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int units = p.nqb * p.batch * p.kv_heads;
    dim3 grid(p.full_units + (units - p.full_units) * p.tail_splits);
    kern<<<grid, NTHREADS, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], p);
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

}  // namespace prefill

void preload_prefill_kernels() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, prefill::prefill_attn_kernel<__nv_bfloat16>);
    cudaFuncGetAttributes(&a, prefill::prefill_attn_kernel<__half>);
}

rfsn_status prefill_launch(int dtype, const CUtensorMap* maps, const PrefillParams& p, cudaStream_t stream) {
    if (p.groups_per_kv < 1 || p.groups_per_kv > prefill::BM) {
        set_error("tensor-core prefill: %d query heads per KV head (max %d)", p.groups_per_kv, prefill::BM);
        return RFSN_ERR_UNSUPPORTED;
    }
    if (dtype == RFSN_BF16) return prefill::launch<__nv_bfloat16>(maps, p, stream);
    if (dtype == RFSN_F16) return prefill::launch<__half>(maps, p, stream);
    set_error("tensor-core prefill: unsupported dtype %d", dtype);
    return RFSN_ERR_UNSUPPORTED;
}

}  // namespace rfsn
