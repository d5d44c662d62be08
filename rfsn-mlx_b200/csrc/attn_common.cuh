// Split-KV bookkeeping shared by the attention kernels: page-table / hot-window
// tile cursor and the in-kernel cross-split merge.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace rfsn {

constexpr int kTile = RFSN_TILE_KEYS;  // keys per tile

// One tile of keys: its absolute position, number of valid keys, the span it
// belongs to and its first row inside that span.
struct TileRef {
    int span;     // index into the span list (archived blocks, then hot pieces)
    int kpos0;    // absolute position of the tile's first key
    int nvalid;   // valid keys in the tile (1..kTile)
    int row;      // arena row of the tile's first key (paged mode)
    int offset;   // key offset of the tile inside its span
};

// Walks the tiles of: archived blocks in page-table order (cache.py:413-423)
// followed by the 1-2 physical pieces of the hot window (cache.py:184-218).
struct PagedCursor {
    const int4* records;  // {row, pos, len, tile_begin}, n_blocks + 1 entries
    int n_blocks, archived_tiles;
    // the two hot pieces
    int h0_row, h0_pos, h0_len, h1_row, h1_pos, h1_len;
    // current position
    int span, tile_in_span, span_tiles, s_row, s_pos, s_len;
    int4 next_rec;  // record span + 1, prefetched

    __device__ void init_hot(int ring_row0, int capacity, int head, int length, int start_pos) {
        const int first = min(length, capacity - head);
        h0_row = ring_row0 + head;
        h0_pos = start_pos;
        h0_len = first;
        h1_row = ring_row0;
        h1_pos = start_pos + first;
        h1_len = length - first;
    }

    __device__ void set_span(int s, int4 rec) {
        span = s;
        if (s < n_blocks) {
            s_row = rec.x;
            s_pos = rec.y;
            s_len = rec.z;
            next_rec = (s + 1 < n_blocks) ? records[s + 1] : make_int4(0, 0, 0, 0);
        } else if (s == n_blocks) {
            s_row = h0_row;
            s_pos = h0_pos;
            s_len = h0_len;
        } else if (s == n_blocks + 1) {
            s_row = h1_row;
            s_pos = h1_pos;
            s_len = h1_len;
        } else {
            s_row = s_pos = s_len = 0;
        }
        span_tiles = (s_len + kTile - 1) / kTile;
    }

    // Largest i in [0, n_blocks) with records[i].tile_begin <= gt, found by the
    // 32 lanes of the calling warp together (two rounds of loads for up to
    // ~1000 blocks instead of a dependent binary search). All lanes return it.
    __device__ int warp_find(int gt) const {
        const int lane = threadIdx.x & 31;
        int lo = 0, hi = n_blocks;  // answer in [lo, hi)
        while (hi - lo > 1) {
            const int step = (hi - lo + 31) / 32;
            const int idx = lo + lane * step;
            const bool ok = idx < hi && records[idx].w <= gt;
            const unsigned m = __ballot_sync(0xffffffffu, ok);
            const int last = 31 - __clz(m);  // lane 0 always qualifies (records[lo].w <= gt)
            lo = lo + last * step;
            hi = min(hi, lo + step);
        }
        return lo;
    }

    // Position on global tile index gt. Called by a whole warp.
    __device__ void seek_warp(int gt) {
        if (gt < archived_tiles) {
            const int i = warp_find(gt);
            const int4 rec = records[i];
            set_span(i, rec);
            tile_in_span = gt - rec.w;
        } else {
            const int rem = gt - archived_tiles;
            const int t0 = (h0_len + kTile - 1) / kTile;
            if (rem < t0) {
                set_span(n_blocks, make_int4(0, 0, 0, 0));
                tile_in_span = rem;
            } else {
                set_span(n_blocks + 1, make_int4(0, 0, 0, 0));
                tile_in_span = rem - t0;
            }
        }
        skip_empty();
    }

    __device__ void skip_empty() {
        while (span_tiles == 0 && span < n_blocks + 2) {
            set_span(span + 1, next_rec);
            tile_in_span = 0;
        }
    }

    __device__ TileRef current() const {
        TileRef t;
        t.span = span;
        t.offset = tile_in_span * kTile;
        t.kpos0 = s_pos + t.offset;
        t.nvalid = min(kTile, s_len - t.offset);
        t.row = s_row + t.offset;
        return t;
    }

    __device__ void advance() {
        if (++tile_in_span >= span_tiles) {
            set_span(span + 1, next_rec);
            tile_in_span = 0;
            skip_empty();
        }
    }
};

// Cross-split merge. Every CTA of a (group, q-block) writes its partial
// (max m, sum l, unnormalised out o) for its split into the workspace; the
// last CTA to arrive combines them:
//   M = max_s m_s,  L = sum_s 2^(m_s - M) l_s,  O = sum_s 2^(m_s - M) o_s,
//   out = O / max(L, 1e-9)           (attention_exact.py:155-164),
//   lse = (M + log2 L) * ln 2        (natural log, for cross-GPU merges).
// Scores are kept in log2 units (q pre-multiplied by log2 e).
//
// The merge is latency-critical (it runs after every other CTA of the group
// has finished), so all loads are issued in parallel: the per-split (m, l)
// pairs in one sweep, the per-slot max / weight / sum by one warp per slot
// with shuffles, and the outputs as float4 loads eight splits deep per thread.
// Must be called by all `nthreads` (a multiple of 32) participating threads
// (thread 0 included) after the CTA partial has been written. `flag` is a
// shared int; `sbuf` is shared scratch of merge_scratch_floats() floats.
__host__ __device__ constexpr int merge_scratch_floats(int nslots, int splits) { return 2 * nslots * splits + 2 * nslots; }
// (totals holds L then the LSE per slot: 2 * nslots floats)

// Fused cross-GPU merge of one float4 of one query slot (called by the last
// CTA of a group in every rank, one thread per (slot, 4 output columns)):
// the rank's final local value r (and its LSE) is stamped with the call
// number and stored into the same place of every rank's mailbox (NVLink
// stores for peers), then the thread polls the P sources' words for the same
// place until all carry this call's stamp (bounded by peer.timeout_ns) and
// merges them in rank order:  out = sum_r e^(lse_r - M) O_r / sum_r e^(lse_r - M).
// Mailbox halves alternate with the call parity: a rank cannot publish call
// c + 2 before every peer has published (so finished reading) call c + 1.
__device__ __forceinline__ void peer_store_and_merge(const PeerParams& peer, const WsView& ws, int call, int group,
                                                     int sl, int d4, int head_dim, float4 r, float my_lse,
                                                     const OutMap& om, float* out, float* lse) {
    if (*reinterpret_cast<volatile const int*>(peer.poison) != 0) {
        // An earlier call of this group gave up waiting for a peer: the ranks'
        // call stamps may no longer agree, so words carrying this call's stamp
        // could belong to another decode step. Keep the local result and fail.
        *reinterpret_cast<float4*>(out + om.row(group, sl) * head_dim + 4 * d4) = r;
        if (lse != nullptr && d4 == 0) lse[om.row(group, sl)] = my_lse;
        if (d4 == 0) atomicExch(ws.error, kDevErrPeerTimeout);
        return;
    }
    const int P = peer.world;
    const int groups = (int)gridDim.y;  // grid = splits x groups
    const size_t slot_words = (size_t)head_dim + 2;
    const size_t half = (size_t)kMaxPeers * groups * kPeerSlots * slot_words;
    const uint32_t stamp = (uint32_t)call;
    const size_t src_off = (size_t)(call & 1) * half + (((size_t)peer.rank * groups + group) * kPeerSlots + sl) * slot_words;
    for (int d = 0; d < P; ++d) {
        uint2* w = peer.words[d] + src_off;
        st_volatile_v4(w + 4 * d4, __float_as_uint(r.x), stamp, __float_as_uint(r.y), stamp);
        st_volatile_v4(w + 4 * d4 + 2, __float_as_uint(r.z), stamp, __float_as_uint(r.w), stamp);
        if (d4 == 0) st_volatile_v4(w + head_dim, __float_as_uint(my_lse), stamp, 0u, stamp);
    }
    const uint2* local = peer.words[peer.rank] + (size_t)(call & 1) * half + ((size_t)group * kPeerSlots + sl) * slot_words;
    const size_t src_stride = (size_t)groups * kPeerSlots * slot_words;
    // Sources are polled two at a time: the words of a group are requested
    // together (one round trip per poll instead of one per rank), and the
    // sources that have not arrived are polled again. Merged in rank order.
    constexpr int kGroup = 2;  // the load results of a group stay in registers (no spill at 2 CTAs per SM)
    const long long t0 = global_ns();
    bool timed_out = false;
    // online merge in rank order: running max M, weight sum W, weighted sum acc
    float M = -CUDART_INF_F, W = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int g0 = 0; g0 < P && !timed_out; g0 += kGroup) {
        const int n = min(kGroup, P - g0);
        const unsigned want = (1u << n) - 1u;
        unsigned ready = 0;
        uint4 a[kGroup], b[kGroup], l[kGroup];
#pragma unroll
        for (int s = 0; s < kGroup; ++s) a[s] = b[s] = l[s] = make_uint4(0, 0, 0, 0);
        for (;;) {
#pragma unroll
            for (int s = 0; s < kGroup; ++s) {
                if (s < n && !((ready >> s) & 1u)) {
                    const uint2* w = local + (g0 + s) * src_stride;
                    a[s] = ld_volatile_v4(w + 4 * d4);
                    b[s] = ld_volatile_v4(w + 4 * d4 + 2);
                    l[s] = ld_volatile_v4(w + head_dim);
                }
            }
#pragma unroll
            for (int s = 0; s < kGroup; ++s) {
                if (s < n && a[s].y == stamp && a[s].w == stamp && b[s].y == stamp && b[s].w == stamp &&
                    l[s].y == stamp)
                    ready |= 1u << s;
            }
            if (ready == want) break;
            if (global_ns() - t0 > peer.timeout_ns) {
                timed_out = true;
                break;
            }
            __nanosleep(20);
        }
#pragma unroll
        for (int s = 0; s < kGroup; ++s) {
            if (s >= n || !((ready >> s) & 1u)) continue;  // after a timeout only the parts that arrived
            const float ls = __uint_as_float(l[s].x);
            if (ls == -CUDART_INF_F) continue;  // a part that saw no visible key
            const float4 v = make_float4(__uint_as_float(a[s].x), __uint_as_float(a[s].z), __uint_as_float(b[s].x),
                                         __uint_as_float(b[s].z));
            if (ls > M) {
                const float sc = (M == -CUDART_INF_F) ? 0.f : expf(M - ls);
                W = W * sc + 1.f;
                acc = make_float4(acc.x * sc + v.x, acc.y * sc + v.y, acc.z * sc + v.z, acc.w * sc + v.w);
                M = ls;
            } else {
                const float wgt = expf(ls - M);
                W += wgt;
                acc = make_float4(acc.x + wgt * v.x, acc.y + wgt * v.y, acc.z + wgt * v.z, acc.w + wgt * v.w);
            }
        }
    }
    if (timed_out) {
        atomicExch(peer.poison, 1);
        atomicExch(ws.error, kDevErrPeerTimeout);
    }
    const float inv = W > 0.f ? 1.f / W : 0.f;
    *reinterpret_cast<float4*>(out + om.row(group, sl) * head_dim + 4 * d4) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    if (lse != nullptr && d4 == 0) lse[om.row(group, sl)] = W > 0.f ? M + logf(W) : -CUDART_INF_F;
}

constexpr int kMergeDepth = 24;  // independent loads in flight per thread in the split merge (default)

template <int kDepth = kMergeDepth>
__device__ __forceinline__ void finish_splits(const WsView& ws, int counter_idx, int part_base, int split_stride,
                                              int splits, int slot0, int nslots, int head_dim, const OutMap& om,
                                              int bh, float* out, float* lse, int* flag, float* sbuf, int bar_id,
                                              int nthreads, const PeerParams* peer = nullptr, int call = 0,
                                              float4* stage = nullptr, int stage_vec4 = 0) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = nthreads >> 5;
    // One release-acquire arrival per CTA after a CTA barrier (no per-thread
    // fences): the barrier orders every thread's partial stores before thread
    // 0's release, and the last CTA's acquire followed by the barrier orders
    // the other CTAs' partials before its threads' loads.
    named_barrier_sync(bar_id, nthreads);
    if (splits > 1) {
        if (tid == 0) {
            int prev = atom_add_acq_rel_gpu(&ws.counters[counter_idx], 1);
            *flag = (prev == splits - 1);
        }
        named_barrier_sync(bar_id, nthreads);
        if (!*flag) return;
    }
    // The merge is a chain of L2 round trips (arrival atomic, m/l, O). Without
    // a staging area each thread's first kDepth partial-output vectors are
    // requested first, so they travel while the weights are computed; the rest
    // follow in chunks of kDepth independent loads.
    const int d4n = head_dim >> 2;
    const bool vec4 = (head_dim & 3) == 0;
    const int items = vec4 ? nslots * d4n : 0;
    const size_t o_stride = (size_t)split_stride * d4n;
    // With a shared staging area large enough for every split's partial outputs
    // (splits x items float4), they are all requested at once by cp.async: one
    // round trip whatever the split count, no registers held.
    // The group's m and l runs (splits x split_stride floats each, from
    // part_base) travel in the same round trip as 16-byte chunks.
    const int ml_vec4 = splits * split_stride / 4;
    const bool aligned16 = ((reinterpret_cast<uintptr_t>(ws.m) | reinterpret_cast<uintptr_t>(ws.l) |
                             reinterpret_cast<uintptr_t>(ws.o)) & 15) == 0;
    const bool staged = stage != nullptr && vec4 && d4n == 32 && aligned16 && (split_stride & 3) == 0 && (part_base & 3) == 0 &&
                        (size_t)splits * items + 2 * (size_t)ml_vec4 <= (size_t)stage_vec4;
    float4* st_m = stage + (size_t)splits * items;
    float4* st_l = st_m + ml_vec4;
    float4 ov[kDepth];
    if (staged) {
        const float4* gm = reinterpret_cast<const float4*>(ws.m + part_base);
        const float4* gl = reinterpret_cast<const float4*>(ws.l + part_base);
        for (int i = tid; i < ml_vec4; i += nthreads) {
            cp_async_16(st_m + i, gm + i);
            cp_async_16(st_l + i, gl + i);
        }
        for (int idx = tid; idx < items; idx += nthreads) {
            const int sl = idx / d4n, d4 = idx - sl * d4n;
            const float4* src = reinterpret_cast<const float4*>(ws.o) + (size_t)(part_base + slot0 + sl) * d4n + d4;
            float4* dst = stage + idx;
#pragma unroll 4
            for (int s = 0; s < splits; ++s, src += o_stride, dst += items) cp_async_16(dst, src);
        }
        cp_async_commit();
        cp_async_wait_all();
        named_barrier_sync(bar_id, nthreads);  // every thread's m/l chunks have landed
        // One warp per query slot, lane j = output float4 j of the slot (head_dim
        // 128): the slot's max and weight sum over the splits with the lanes
        // across splits and shuffle reductions, the weights written back over
        // m, then each lane's weighted sum of its column vector over the splits.
        const uint32_t a_m = smem_u32(st_m), a_l = smem_u32(st_l), a_o = smem_u32(stage);
        const uint32_t ml_step = 4u * split_stride, o_step = 16u * items;
        constexpr int kB = 8;  // splits per batch: independent loads issued together
        for (int sl = warp; sl < nslots; sl += nwarps) {
            const int d4 = lane, idx = sl * d4n + d4;
            const uint32_t am = a_m + 4u * (slot0 + sl), al = a_l + 4u * (slot0 + sl), ao = a_o + 16u * idx;
            float M = -CUDART_INF_F;
            for (int s = lane; s < splits; s += 32) M = fmaxf(M, lds_f32(am + s * ml_step));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            float L = 0.f;
            for (int s = lane; s < splits; s += 32) {
                const float w = (M == -CUDART_INF_F) ? 0.f : ex2_approx(lds_f32(am + s * ml_step) - M);
                L += w * lds_f32(al + s * ml_step);
                sts_f32(am + s * ml_step, w);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
            __syncwarp();
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s0 = 0; s0 < splits; s0 += kB) {
                float c[kB];
                float4 ob[kB];
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    const bool in = s0 + u < splits;
                    c[u] = in ? lds_f32(am + (s0 + u) * ml_step) : 0.f;
                    ob[u] = in ? lds_f4(ao + (s0 + u) * o_step) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    acc.x += c[u] * ob[u].x;
                    acc.y += c[u] * ob[u].y;
                    acc.z += c[u] * ob[u].z;
                    acc.w += c[u] * ob[u].w;
                }
            }
            const float inv = 1.f / fmaxf(L, 1e-9f);
            const float4 r = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
            const float my_lse = (L > 0.f) ? (M + log2f(L)) * 0.69314718055994531f : -CUDART_INF_F;
            if (peer == nullptr) {
                *reinterpret_cast<float4*>(out + om.row(bh, slot0 + sl) * head_dim + 4 * d4) = r;
                if (lse != nullptr && d4 == 0) lse[om.row(bh, slot0 + sl)] = my_lse;
            } else {
                peer_store_and_merge(*peer, ws, call, bh, sl, d4, head_dim, r, my_lse, om, out, lse);
            }
        }
        if (splits > 1 && tid == 0) ws.counters[counter_idx] = 0;
        if (peer != nullptr && tid == 0) peer->calls[bh] = call;
        return;
    }
    if (tid < items) {
        const int sl = tid / d4n, d4 = tid - sl * d4n;
        const float4* base = reinterpret_cast<const float4*>(ws.o) + (size_t)(part_base + slot0 + sl) * d4n + d4;
#pragma unroll
        for (int u = 0; u < kDepth; ++u) ov[u] = u < splits ? __ldcg(base + (size_t)u * o_stride)
                                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float* wts = sbuf;                          // [nslots][splits] m_s, then weights
    float* ls = sbuf + nslots * splits;         // [nslots][splits] l_s
    float* totals = ls + nslots * splits;       // [nslots] L, then [nslots] natural-log LSE
    for (int i = tid; i < nslots * splits; i += nthreads) {
        const int sl = i / splits, s = i - sl * splits;
        const int p = part_base + s * split_stride + slot0 + sl;
        wts[i] = __ldcg(ws.m + p);
        ls[i] = __ldcg(ws.l + p);
    }
    named_barrier_sync(bar_id, nthreads);
    for (int sl = warp; sl < nslots; sl += nwarps) {
        float* w = wts + sl * splits;
        const float* l = ls + sl * splits;
        float M = -CUDART_INF_F;
        for (int s = lane; s < splits; s += 32) M = fmaxf(M, w[s]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int s = lane; s < splits; s += 32) {
            const float ws_ = (M == -CUDART_INF_F) ? 0.f : exp2f(w[s] - M);
            w[s] = ws_;
            L += ws_ * l[s];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        if (lane == 0) {
            totals[sl] = L;
            const float my_lse = (L > 0.f) ? (M + log2f(L)) * 0.69314718055994531f : -CUDART_INF_F;
            totals[nslots + sl] = my_lse;
            if (lse != nullptr && peer == nullptr) lse[om.row(bh, slot0 + sl)] = my_lse;
        }
    }
    named_barrier_sync(bar_id, nthreads);
    if (vec4) {
        for (int idx = tid; idx < items; idx += nthreads) {
            const int sl = idx / d4n, d4 = idx - sl * d4n;
            const float* w = wts + sl * splits;
            const float4* base = reinterpret_cast<const float4*>(ws.o) +
                                 (size_t)(part_base + slot0 + sl) * d4n + d4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s0 = 0; s0 < splits; s0 += kDepth) {
                if (idx != tid || s0 != 0) {  // the first chunk of the first item is already in flight
#pragma unroll
                    for (int u = 0; u < kDepth; ++u) {
                        ov[u] = s0 + u < splits ? __ldcg(base + (size_t)(s0 + u) * o_stride)
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
#pragma unroll
                for (int u = 0; u < kDepth; ++u) {
                    const float c = s0 + u < splits ? w[s0 + u] : 0.f;
                    acc.x += c * ov[u].x;
                    acc.y += c * ov[u].y;
                    acc.z += c * ov[u].z;
                    acc.w += c * ov[u].w;
                }
            }
            const float inv = 1.f / fmaxf(totals[sl], 1e-9f);
            float4 r = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
            if (peer == nullptr) {
                *reinterpret_cast<float4*>(out + om.row(bh, slot0 + sl) * head_dim + 4 * d4) = r;
            } else {
                peer_store_and_merge(*peer, ws, call, bh, sl, d4, head_dim, r, totals[nslots + sl], om, out, lse);
            }
        }
    } else {
        for (int idx = tid; idx < nslots * head_dim; idx += nthreads) {
            const int sl = idx / head_dim, d = idx - sl * head_dim;
            const float* w = wts + sl * splits;
            float O = 0.f;
            for (int s = 0; s < splits; ++s) {
                const size_t p = (size_t)(part_base + s * split_stride + slot0 + sl);
                O += w[s] * __ldcg(ws.o + p * head_dim + d);
            }
            out[om.row(bh, slot0 + sl) * head_dim + d] = O / fmaxf(totals[sl], 1e-9f);
        }
    }
    if (splits > 1 && tid == 0) ws.counters[counter_idx] = 0;
    if (peer != nullptr && tid == 0) peer->calls[bh] = call;
}

}  // namespace rfsn
