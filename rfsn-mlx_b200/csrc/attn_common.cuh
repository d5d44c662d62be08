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
    // hot pieces
    int h_row[2], h_pos[2], h_len[2];
    // current position
    int span, tile_in_span, span_tiles, s_row, s_pos, s_len;

    __device__ void init_hot(int ring_row0, int capacity, int head, int length, int start_pos) {
        int first = min(length, capacity - head);
        h_row[0] = ring_row0 + head;
        h_pos[0] = start_pos;
        h_len[0] = first;
        h_row[1] = ring_row0;
        h_pos[1] = start_pos + first;
        h_len[1] = length - first;
    }

    __device__ void load_span(int s) {
        span = s;
        if (s < n_blocks) {
            int4 r = records[s];
            s_row = r.x;
            s_pos = r.y;
            s_len = r.z;
        } else {
            int h = s - n_blocks;
            if (h < 2) {
                s_row = h_row[h];
                s_pos = h_pos[h];
                s_len = h_len[h];
            } else {
                s_row = s_pos = s_len = 0;
            }
        }
        span_tiles = (s_len + kTile - 1) / kTile;
    }

    // Position the cursor on global tile index gt.
    __device__ void seek(int gt) {
        if (gt < archived_tiles) {
            int lo = 0, hi = n_blocks - 1;  // largest i with tile_begin[i] <= gt
            while (lo < hi) {
                int mid = (lo + hi + 1) >> 1;
                if (records[mid].w <= gt) lo = mid; else hi = mid - 1;
            }
            load_span(lo);
            tile_in_span = gt - records[lo].w;
        } else {
            int rem = gt - archived_tiles;
            int t0 = (h_len[0] + kTile - 1) / kTile;
            if (rem < t0) {
                load_span(n_blocks);
                tile_in_span = rem;
            } else {
                load_span(n_blocks + 1);
                tile_in_span = rem - t0;
            }
        }
        skip_empty();
    }

    __device__ void skip_empty() {
        while (span_tiles == 0 && span < n_blocks + 2) {
            load_span(span + 1);
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
            load_span(span + 1);
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
// Must be called by all `nthreads` participating threads (thread 0 included)
// after the CTA partial has been written. `flag` is a shared int and `sbuf`
// shared scratch of at least nslots * (splits + 2) floats.
__device__ __forceinline__ void finish_splits(const WsView& ws, int counter_idx, int part_base, int split_stride,
                                              int splits, int slot0, int nslots, int head_dim, const OutMap& om,
                                              int bh, float* out, float* lse, int* flag, float* sbuf, int bar_id,
                                              int nthreads) {
    const int tid = threadIdx.x;
    __threadfence();
    named_barrier_sync(bar_id, nthreads);
    if (splits > 1) {
        if (tid == 0) {
            int prev = atomicAdd(&ws.counters[counter_idx], 1);
            *flag = (prev == splits - 1);
        }
        named_barrier_sync(bar_id, nthreads);
        if (!*flag) return;
        __threadfence();
    }
    float* wts = sbuf;                      // [nslots][splits] weights 2^(m_s - M)
    float* totals = sbuf + nslots * splits; // [nslots] L
    for (int i = tid; i < nslots * splits; i += nthreads) {
        const int sl = i / splits, s = i - sl * splits;
        wts[i] = __ldcg(ws.m + part_base + s * split_stride + slot0 + sl);
    }
    named_barrier_sync(bar_id, nthreads);
    if (tid < nslots) {
        float* w = wts + tid * splits;
        float M = -CUDART_INF_F;
        for (int s = 0; s < splits; ++s) M = fmaxf(M, w[s]);
        float L = 0.f;
        for (int s = 0; s < splits; ++s) {
            const float ws_ = (M == -CUDART_INF_F) ? 0.f : exp2f(w[s] - M);
            w[s] = ws_;
            L += ws_ * __ldcg(ws.l + part_base + s * split_stride + slot0 + tid);
        }
        totals[tid] = L;
        if (lse != nullptr) {
            lse[om.row(bh, slot0 + tid)] = (L > 0.f) ? (M + log2f(L)) * 0.69314718055994531f : -CUDART_INF_F;
        }
    }
    named_barrier_sync(bar_id, nthreads);
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
    if (splits > 1 && tid == 0) ws.counters[counter_idx] = 0;
}

}  // namespace rfsn
