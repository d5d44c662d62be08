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
// float32 accuracy: q (pre-scaled by log2(e)/sqrt(d)) and the probabilities
// P are each split into a 16-bit high part and a 16-bit residual
// (x = hi + lo to ~16 significand bits); S = Qhi K^T + Qlo K^T and
// O += Phi V + Plo V, all accumulated in float32 in TMEM. K and V are stored
// in 16 bits already, so they enter the products exactly.
//
// Warps:
//   0-3  softmax (thread = row = TMEM lane): split q into shared memory
//        (128B-swizzled K-major), then per key tile read the S row from TMEM,
//        causal/validity mask, float32 online softmax on exp2, write Phi/Plo
//        back over the S columns (A operand of the PV product, read from
//        TMEM), rescale the O row in TMEM when its maximum grew; finally
//        O / l -> out and the log-sum-exp.
//   4    producer: walks the page table (archived blocks in order, then the
//        hot pieces) in 128-key tiles up to the CTA's causal limit, streaming
//        K/V with TMA into a 2-stage ring (8-row boxes for ragged span ends).
//   5    MMA issuer (one thread): S(it+1) into the other S buffer while the
//        softmax works on tile it, then O += P(it) V(it); tcgen05.commit
//        signals the softmax warps and releases the K/V stage.
// TMEM: S buffers at columns [0,128) and [128,256), O at [256,384).
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
constexpr int NST = 2;    // K/V pipeline stages
constexpr int NTHREADS = 6 * 32;
constexpr int TILE_HALF = BN * 128;  // bytes of one 64-column half of a 128-row tile
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S0 = 0, COL_S1 = 128, COL_O = 256;

struct Smem {
    uint8_t q[2][2][BM * 128];  // [hi/lo][column half]
    uint8_t k[NST][2][TILE_HALF];
    uint8_t v[NST][2][TILE_HALF];
    uint64_t kv_full[NST];
    uint64_t kv_empty[NST];
    uint64_t s_full[2];
    uint64_t p_full;
    uint64_t o_done;
    uint64_t mma_done;
    int2 tinfo[NST];  // {kpos0, nvalid}; nvalid < 0 marks the end of the key stream
    uint32_t tmem;
    int abort;
};

// (a, b) -> packed 16-bit high parts and packed 16-bit residuals.
template <typename T>
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    hi = pack2<T>(a, b);
    float ha, hb;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        ha = __uint_as_float(hi << 16);
        hb = __uint_as_float(hi & 0xffff0000u);
    } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hi));
        ha = f.x;
        hb = f.y;
    }
    lo = pack2<T>(a - ha, b - hb);
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

template <typename T>
__global__ void __launch_bounds__(NTHREADS, 1)
prefill_attn_kernel(const __grid_constant__ CUtensorMap mapK64, const __grid_constant__ CUtensorMap mapV64,
                    const __grid_constant__ CUtensorMap mapK8, const __grid_constant__ CUtensorMap mapV8,
                    const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.groups_per_kv;
    const int ppc = BM / G;                                   // chunk positions per CTA
    const int qb = gridDim.x - 1 - blockIdx.x;                // longest (latest) rows first
    const int bh = blockIdx.y;                                // b * kv_heads + kv head
    const int b = bh / p.kv_heads, hk = bh % p.kv_heads;
    const int pos_base = qb * ppc;                            // first chunk position of the CTA
    const int qlast = p.q_pos0 + min(pos_base + ppc, p.q_len) - 1;  // causal limit of the CTA

    // ---- set-up: zero the K/V stages (rows past a ragged span end stay finite),
    //      barriers, TMEM ----
    for (int i = tid; i < NST * 2 * 2 * TILE_HALF / 16; i += NTHREADS) {
        reinterpret_cast<uint4*>(sm.k)[i] = make_uint4(0, 0, 0, 0);
    }
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&sm.kv_full[s], 1);
            mbar_init(&sm.kv_empty[s], 1);
        }
        mbar_init(&sm.s_full[0], 1);
        mbar_init(&sm.s_full[1], 1);
        mbar_init(&sm.p_full, 4 * 32);
        mbar_init(&sm.o_done, 1);
        mbar_init(&sm.mma_done, 1);
        sm.abort = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tc::tmem_alloc(&sm.tmem, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sm.tmem;

    if (warp == 4) {
        // ---------------- producer ----------------
        if (lane == 0) {
            prefetch_tmap(&mapK64);
            prefetch_tmap(&mapV64);
            int it = 0;
            bool stop = false;
            for (int span = 0; span < p.n_blocks + 2 && !stop; ++span) {
                int s_row, s_pos, s_len;
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
                for (int off = 0; off < s_len; off += BN) {
                    const int kpos0 = s_pos + off;
                    if (kpos0 > qlast) {  // spans are in increasing position order
                        stop = true;
                        break;
                    }
                    const int nvalid = min(BN, s_len - off);
                    const int row = s_row + off;
                    const int s = it % NST;
                    if (it >= NST && !mbar_wait_bounded(&sm.kv_empty[s], ((it / NST) + 1) & 1, &sm.abort)) {
                        fail(&sm.abort, p);
                        stop = true;
                        break;
                    }
                    const bool bad = row < 0 || row + nvalid > p.rows;
                    if (bad) atomicExch(p.ws.error, kDevErrBadTable);
                    sm.tinfo[s] = make_int2(kpos0, bad ? 0 : nvalid);
                    const int grow = bh * p.rows + row;
                    if (bad) {
                        mbar_arrive(&sm.kv_full[s]);
                    } else if (nvalid == BN) {
                        mbar_arrive_expect_tx(&sm.kv_full[s], 4 * TILE_HALF);
                        for (int hh = 0; hh < 2; ++hh) {
                            for (int r64 = 0; r64 < 2; ++r64) {
                                tma_load_2d(sm.k[s][hh] + r64 * 64 * 128, &mapK64, 64 * hh, grow + 64 * r64, &sm.kv_full[s]);
                                tma_load_2d(sm.v[s][hh] + r64 * 64 * 128, &mapV64, 64 * hh, grow + 64 * r64, &sm.kv_full[s]);
                            }
                        }
                    } else {
                        const int nb = (nvalid + 7) >> 3;
                        mbar_arrive_expect_tx(&sm.kv_full[s], nb * 4 * 1024);
                        for (int hh = 0; hh < 2; ++hh) {
                            for (int bb = 0; bb < nb; ++bb) {
                                tma_load_2d(sm.k[s][hh] + bb * 1024, &mapK8, 64 * hh, grow + 8 * bb, &sm.kv_full[s]);
                                tma_load_2d(sm.v[s][hh] + bb * 1024, &mapV8, 64 * hh, grow + 8 * bb, &sm.kv_full[s]);
                            }
                        }
                    }
                    ++it;
                }
            }
            // let the fills in flight land (bounded) before the marker reuses a stage
            for (int j = max(0, it - NST); j < it; ++j) mbar_wait_bounded(&sm.kv_full[j % NST], (j / NST) & 1, nullptr);
            // end-of-stream marker
            const int s = it % NST;
            if (it < NST || mbar_wait_bounded(&sm.kv_empty[s], ((it / NST) + 1) & 1, &sm.abort)) {
                sm.tinfo[s] = make_int2(0, -1);
                mbar_arrive(&sm.kv_full[s]);
            } else {
                fail(&sm.abort, p);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        named_barrier_sync(2, 5 * 32);  // q tiles written by the softmax warps
        tc::fence_after_sync();
        if (lane == 0) {
            constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
            const uint32_t id_qk = tc::idesc_f16(kBf16, false, false, BM, BN);
            const uint32_t id_pv = tc::idesc_f16(kBf16, false, true, BM, D);
            const uint32_t tO = tmem + COL_O;
            int it = 0;
            bool pending = false;  // tensor-core work issued whose completion is not yet observed
            bool have_first = mbar_wait_bounded(&sm.kv_full[0], 0, &sm.abort);
            if (!have_first) fail(&sm.abort, p);
            have_first = have_first && sm.tinfo[0].y >= 0;
            for (int t = 0; have_first; ++t) {
                // S(t) = Qhi K^T + Qlo K^T into S buffer t % 2; t = 0 first, then S(it+1)
                // one tile ahead while the softmax works on tile it
                if (t > 0) {
                    it = t - 1;
                    const int s1 = t % NST;
                    if (!mbar_wait_bounded(&sm.kv_full[s1], (t / NST) & 1, &sm.abort)) {
                        fail(&sm.abort, p);
                        break;
                    }
                }
                const bool issue = (t == 0) || sm.tinfo[t % NST].y >= 0;
                if (issue) {
                    // S buffer t % 2 last held P(t-2): PV(t-2) must be done
                    if (t >= 2 && !mbar_wait_bounded(&sm.o_done, (t - 2) & 1, &sm.abort)) {
                        fail(&sm.abort, p);
                        break;
                    }
                    tc::fence_after_sync();
                    const int s = t % NST;
                    const uint32_t tS = tmem + ((t & 1) ? COL_S1 : COL_S0);
#pragma unroll 1
                    for (int part = 0; part < 2; ++part) {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint32_t qa = smem_u32(sm.q[part][kk >> 2]) + (kk & 3) * 32;
                            const uint32_t ka = smem_u32(sm.k[s][kk >> 2]) + (kk & 3) * 32;
                            tc::mma_f16_ss(tS, tc::smem_desc_sw128(qa, 16, 1024), tc::smem_desc_sw128(ka, 16, 1024),
                                           id_qk, part > 0 || kk > 0);
                        }
                    }
                    tc::commit(&sm.s_full[t & 1]);
                    pending = true;
                }
                if (t == 0) continue;
                // P(it) in TMEM (and O rescaled): O += Phi V + Plo V
                if (!mbar_wait_bounded(&sm.p_full, it & 1, &sm.abort)) {
                    fail(&sm.abort, p);
                    break;
                }
                tc::fence_after_sync();
                const int s = it % NST;
                const uint32_t tP = tmem + ((it & 1) ? COL_S1 : COL_S0);
#pragma unroll 1
                for (int part = 0; part < 2; ++part) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t va = smem_u32(sm.v[s][0]) + kk * 16 * 128;
                        tc::mma_f16_ts(tO, tP + 64 * part + 8 * kk, tc::smem_desc_sw128(va, TILE_HALF, 1024), id_pv,
                                       it > 0 || part > 0 || kk > 0);
                    }
                }
                tc::commit(&sm.o_done);
                tc::commit(&sm.kv_empty[s]);
                if (!issue) break;  // tile it was the last one
            }
            // drain: no tensor-core work may be in flight when TMEM is released
            // (tcgen05.commit tracks all earlier tensor-core work of this thread)
            if (pending) {
                tc::commit(&sm.mma_done);  // single-use barrier: phase 0 = everything issued
                mbar_wait_bounded(&sm.mma_done, 0, nullptr);
            }
        }
    } else {
        // ---------------- softmax warps (thread = row = TMEM lane) ----------------
        const int r = tid;
        const int g = r % G, j = r / G;
        const int h = hk * G + g;
        const int qrow = pos_base + j;
        const bool row_ok = j < ppc && qrow < p.q_len;
        const int qpos = p.q_pos0 + qrow;
        {
            const float* src = p.q + (((size_t)b * p.q_heads + h) * p.q_len + (row_ok ? qrow : 0)) * D;
#pragma unroll
            for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 elements
                float x[8];
                if (row_ok) {
                    const float4 a = *reinterpret_cast<const float4*>(src + 8 * c);
                    const float4 bq = *reinterpret_cast<const float4*>(src + 8 * c + 4);
                    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                    x[4] = bq.x; x[5] = bq.y; x[6] = bq.z; x[7] = bq.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[e] = 0.f;
                }
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split2<T>(x[2 * e] * p.qscale, x[2 * e + 1] * p.qscale, hi[e], lo[e]);
                const uint32_t off = tc::sw128_offset(r, c & 7);
                *reinterpret_cast<uint4*>(sm.q[0][c >> 3] + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(sm.q[1][c >> 3] + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        named_barrier_sync(2, 5 * 32);
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        const uint32_t tO = tmem + COL_O + lane_base;
        float m = -CUDART_INF_F, l = 0.f;
        int it = 0;
        for (;; ++it) {
            const int s = it % NST;
            if (!warp_wait(&sm.kv_full[s], (it / NST) & 1, &sm.abort)) break;
            const int2 ti = sm.tinfo[s];
            if (ti.y < 0) break;
            if (!warp_wait(&sm.s_full[it & 1], (it >> 1) & 1, &sm.abort)) break;
            tc::fence_after_sync();
            const uint32_t tS = tmem + ((it & 1) ? COL_S1 : COL_S0) + lane_base;
            float sv[BN];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t rr[32];
                tc::ld_32x32b_x32(tS + 32 * cc, rr);
                tc::wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) sv[32 * cc + jj] = __uint_as_float(rr[jj]);
            }
            // keys [kpos0, kpos0 + nvalid) are valid; causal: key position <= query position
            const int lim = min(ti.y, qpos - ti.x + 1);
            float tmax = -CUDART_INF_F;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                sv[c] = c < lim ? sv[c] : -CUDART_INF_F;
                tmax = fmaxf(tmax, sv[c]);
            }
            const float mn = fmaxf(m, tmax);
            const float alpha = (mn == -CUDART_INF_F) ? 1.f : exp2f(m - mn);
            const float ms = (mn == -CUDART_INF_F) ? 0.f : mn;
            float rs = 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float p0 = exp2f(sv[32 * cc + 2 * e] - ms);
                    const float p1 = exp2f(sv[32 * cc + 2 * e + 1] - ms);
                    rs += p0 + p1;
                    split2<T>(p0, p1, hi[e], lo[e]);
                }
                tc::st_32x32b_x16(tS + 16 * cc, hi);
                tc::st_32x32b_x16(tS + 64 + 16 * cc, lo);
            }
            l = l * alpha + rs;
            m = mn;
            if (it > 0) {
                // PV of the previous tile must be done before O is rescaled (and before
                // this tile's P is published: one p_full phase per tile)
                if (!warp_wait(&sm.o_done, (it - 1) & 1, &sm.abort)) break;
                tc::fence_after_sync();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t rr[32];
                        tc::ld_32x32b_x32(tO + 32 * cc, rr);
                        tc::wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) rr[jj] = __float_as_uint(__uint_as_float(rr[jj]) * alpha);
                        tc::st_32x32b_x32(tO + 32 * cc, rr);
                    }
                }
            }
            tc::wait_st();
            tc::fence_before_sync();
            mbar_arrive(&sm.p_full);
        }
        const bool ok = it > 0 && warp_wait(&sm.o_done, (it - 1) & 1, &sm.abort) &&
                        __all_sync(0xffffffffu, sm.abort == 0);
        tc::fence_after_sync();
        float* dst = p.out + (((size_t)b * p.q_heads + h) * p.q_len + (row_ok ? qrow : 0)) * D;
        const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            uint32_t rr[32];
            tc::ld_32x32b_x32(tO + 32 * cc, rr);
            tc::wait_ld();
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
        if (row_ok && p.lse != nullptr) {
            p.lse[((size_t)b * p.q_heads + h) * p.q_len + qrow] =
                (ok && l > 0.f) ? (m + log2f(l)) * 0.69314718055994531f : -CUDART_INF_F;
        }
        if (!ok && tid == 0 && it > 0) atomicExch(p.ws.error, kDevErrTimeout);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <typename T>
rfsn_status launch(const CUtensorMap* maps, const PrefillParams& p, cudaStream_t stream) {
    const size_t smem = sizeof(Smem) + 1024;
    auto kern = prefill_attn_kernel<T>;
    RFSN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int ppc = BM / p.groups_per_kv;
    dim3 grid((p.q_len + ppc - 1) / ppc, p.batch * p.kv_heads);
    kern<<<grid, NTHREADS, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], p);
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

}  // namespace prefill

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
