// Hot-ring kernels: fused RoPE + append, and arena row copies (seal).
#include <type_traits>

#include "params.cuh"

namespace rfsn {
namespace ring {

// One thread per (tensor row, rotation pair j): rotates x[j], x[j + half]
// exactly as layer.py:38-51 with the float32 tables of layer.py:20-35:
//   f = pos * inv_freq[j]                (one float32 product)
//   out[j]        = x1 * cos f - x2 * sin f
//   out[j + half] = x1 * sin f + x2 * cos f
// Products and sums are rounded separately (no FMA contraction) like the
// reference's elementwise ops; cosf/sinf are the accurate CUDA versions.
template <typename TIn, typename TCache>
__global__ void rope_append_kernel(const TIn* __restrict__ q, const TIn* __restrict__ k, const TIn* __restrict__ v,
                                   const float* __restrict__ inv_freq, int pos0, int batch, int q_heads, int kv_heads,
                                   int len, int head_dim, float* __restrict__ q_out, TCache* __restrict__ ak,
                                   TCache* __restrict__ av, int rows, int ring_row0, int capacity, int write_index,
                                   const int* __restrict__ step_state, int* __restrict__ step_state_copy) {
    // A decode kernel launched after this one under programmatic dependent
    // launch may start now: before its dependency wait it only reads archived
    // arena rows, which this kernel never writes (it writes ring rows, q_out
    // and the state copy, all read after that wait). This kernel is itself
    // launched that way and reads its inputs after its own wait.
    griddep_launch_dependents();
    griddep_wait();  // its inputs may come from the kernel this launch overlaps
    const int half = head_dim >> 1;
    const long q_rows = (long)batch * q_heads * len;
    const long kv_rows = (long)batch * kv_heads * len;
    const long total = (q_rows + kv_rows) * half;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const long r = idx / half;
        const int j = (int)(idx - r * half);
        const bool is_q = r < q_rows;
        const long rr = is_q ? r : r - q_rows;
        const int l = (int)(rr % len);
        // element loads first: with inputs in page-locked host memory they and
        // the step-state loads below cross the bus together
        float x1, x2, v1 = 0.f, v2 = 0.f;
        if (is_q) {
            x1 = to_f32<TIn>(q[rr * head_dim + j]);
            x2 = to_f32<TIn>(q[rr * head_dim + j + half]);
        } else {
            x1 = to_f32<TIn>(k[rr * head_dim + j]);
            x2 = to_f32<TIn>(k[rr * head_dim + j + half]);
            v1 = to_f32<TIn>(v[rr * head_dim + j]);
            v2 = to_f32<TIn>(v[rr * head_dim + j + half]);
        }
        int pos_s = pos0, wi = write_index;
        if (step_state != nullptr) {  // position and write slot chosen when the kernel runs
            pos_s = step_state[0];
            wi = step_state[1];
            if (kv_heads > 0 && (unsigned)wi >= (unsigned)capacity) continue;  // never write outside the ring
        }
        float o1 = x1, o2 = x2;
        if (inv_freq != nullptr) {
            const float f = __fmul_rn((float)(pos_s + l), inv_freq[j]);
            const float c = cosf(f), s = sinf(f);
            o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
            o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
        }
        if (is_q) {
            if (q_out != nullptr) {
                q_out[rr * head_dim + j] = o1;
                q_out[rr * head_dim + j + half] = o2;
            }
        } else {
            // rr = (b * kv_heads + h) * len + l  ->  arena row of the ring slot
            const long bh = rr / len;
            const int slot = (wi + l) % capacity;
            const long dst = (bh * rows + ring_row0 + slot) * head_dim;
            ak[dst + j] = from_f32<TCache>(o1);
            ak[dst + j + half] = from_f32<TCache>(o2);
            av[dst + j] = from_f32<TCache>(v1);
            av[dst + j + half] = from_f32<TCache>(v2);
        }
    }
    if (step_state_copy != nullptr && blockIdx.x == 0 && threadIdx.x < RFSN_STEP_STATE_LEN) {
        step_state_copy[threadIdx.x] = step_state[threadIdx.x];  // for the decode kernel that follows
    }
}

// RoPE from explicit tables, then the append (layer.py:118-135 when the caller
// passes rope_tables, or when the layer builds them in the model dtype). One
// thread per (tensor row, pair j); the tables are [len][head_dim] rows of
// positions pos0 + l and each half uses its own columns, as _apply_rope reads
// them (layer.py:38-51):
//   out[j]        = x1 * cos[l][j]        - x2 * sin[l][j]
//   out[j + half] = x1 * sin[l][j + half] + x2 * cos[l][j + half]
// Every product and sum is rounded to the promoted dtype of x and the tables
// (the 16-bit type when both are that type, else float32), the way the
// reference's elementwise ops round each result. Without tables (cos_t NULL)
// they are built from inv_freq in float32 and rounded to TTab
// (build_rope_tables with dtype = the table dtype).
template <typename TIn, typename TTab>
__global__ void rope_tables_append_kernel(const TIn* __restrict__ q, const TIn* __restrict__ k,
                                          const TIn* __restrict__ v, const TTab* __restrict__ cos_t,
                                          const TTab* __restrict__ sin_t, const float* __restrict__ inv_freq, int pos0,
                                          int batch, int q_heads, int kv_heads, int len, int head_dim,
                                          float* __restrict__ q_out, TIn* __restrict__ ak, TIn* __restrict__ av,
                                          int rows, int ring_row0, int capacity, int write_index) {
    constexpr bool kRound16 = std::is_same<TIn, TTab>::value && !std::is_same<TIn, float>::value;
    auto rnd = [](float x) { return kRound16 ? to_f32<TIn>(from_f32<TIn>(x)) : x; };
    griddep_wait();
    const int half = head_dim >> 1;
    const long q_rows = (long)batch * q_heads * len;
    const long kv_rows = (long)batch * kv_heads * len;
    const long total = (q_rows + kv_rows) * half;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const long r = idx / half;
        const int j = (int)(idx - r * half);
        const bool is_q = r < q_rows;
        const long rr = is_q ? r : r - q_rows;
        const int l = (int)(rr % len);
        const TIn* src = is_q ? q : k;
        const float x1 = to_f32<TIn>(src[rr * head_dim + j]);
        const float x2 = to_f32<TIn>(src[rr * head_dim + j + half]);
        float c_lo, s_lo, c_hi, s_hi;
        if (cos_t != nullptr) {
            c_lo = to_f32<TTab>(cos_t[(long)l * head_dim + j]);
            s_lo = to_f32<TTab>(sin_t[(long)l * head_dim + j]);
            c_hi = to_f32<TTab>(cos_t[(long)l * head_dim + j + half]);
            s_hi = to_f32<TTab>(sin_t[(long)l * head_dim + j + half]);
        } else {
            const float f = __fmul_rn((float)(pos0 + l), inv_freq[j]);
            c_lo = c_hi = to_f32<TTab>(from_f32<TTab>(cosf(f)));
            s_lo = s_hi = to_f32<TTab>(from_f32<TTab>(sinf(f)));
        }
        const float o1 = rnd(__fsub_rn(rnd(__fmul_rn(x1, c_lo)), rnd(__fmul_rn(x2, s_lo))));
        const float o2 = rnd(__fadd_rn(rnd(__fmul_rn(x1, s_hi)), rnd(__fmul_rn(x2, c_hi))));
        if (is_q) {
            q_out[rr * head_dim + j] = o1;
            q_out[rr * head_dim + j + half] = o2;
        } else {
            const long bh = rr / len;
            const int slot = (write_index + l) % capacity;
            const long dst = (bh * rows + ring_row0 + slot) * head_dim;
            ak[dst + j] = from_f32<TIn>(o1);
            ak[dst + j + half] = from_f32<TIn>(o2);
            av[dst + j] = v[rr * head_dim + j];
            av[dst + j + half] = v[rr * head_dim + j + half];
        }
    }
    griddep_launch_dependents();
}

// Copy `count` rows of every head from src (read modulo src_wrap when > 0)
// to dst, 16 bytes per thread step, for K and V. Source and destination
// row ranges must not overlap (seal copies ring rows into block rows).
__global__ void copy_rows_kernel(uint8_t* __restrict__ ak, uint8_t* __restrict__ av, int groups, int rows,
                                 int row_bytes, int src_row0, int src_offset, int src_wrap, int dst_row0, int count) {
    const int vec_per_row = row_bytes / 16;
    const long total = (long)groups * count * vec_per_row;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const int vi = (int)(idx % vec_per_row);
        const long rr = idx / vec_per_row;
        const int i = (int)(rr % count);
        const long gidx = rr / count;
        int s = src_offset + i;
        if (src_wrap > 0) s %= src_wrap;
        const long src = ((gidx * rows + src_row0 + s) * row_bytes) + vi * 16;
        const long dst = ((gidx * rows + dst_row0 + i) * row_bytes) + vi * 16;
        *reinterpret_cast<uint4*>(ak + dst) = *reinterpret_cast<const uint4*>(ak + src);
        *reinterpret_cast<uint4*>(av + dst) = *reinterpret_cast<const uint4*>(av + src);
    }
}

}  // namespace ring

rfsn_status rope_append_launch(int dtype, const void* q, const void* k, const void* v, const float* inv_freq, int pos0,
                               int batch, int q_heads, int kv_heads, int len, int head_dim, float* q_out, void* ak,
                               void* av, int rows, int ring_row0, int capacity, int write_index, cudaStream_t stream,
                               const int* step_state, int* step_state_copy) {
    const long total = ((long)batch * (q_heads + kv_heads) * len) * (head_dim / 2);
    const int threads = 256;
    long blocks = (total + threads - 1) / threads;
    if (blocks > 65535L * 8) blocks = 65535L * 8;
    if (blocks < 1) blocks = 1;
#define RFSN_ROPE_LAUNCH(T)                                                                                     \
    RFSN_CUDA(launch_pdl(ring::rope_append_kernel<T, T>, dim3((unsigned)blocks), dim3(threads), 0, stream,        \
                         static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), inv_freq,  \
                         pos0, batch, q_heads, kv_heads, len, head_dim, q_out, static_cast<T*>(ak),              \
                         static_cast<T*>(av), rows, ring_row0, capacity, write_index, step_state,                 \
                         step_state_copy))
    if (dtype == RFSN_F32) {
        RFSN_ROPE_LAUNCH(float);
    } else if (dtype == RFSN_F16) {
        RFSN_ROPE_LAUNCH(__half);
    } else {
        RFSN_ROPE_LAUNCH(__nv_bfloat16);
    }
#undef RFSN_ROPE_LAUNCH
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

template <typename TIn>
static rfsn_status rope_tables_launch_in(int tab_dtype, const void* q, const void* k, const void* v, const void* cos_t,
                                         const void* sin_t, const float* inv_freq, int pos0, int batch, int q_heads,
                                         int kv_heads, int len, int head_dim, float* q_out, void* ak, void* av,
                                         int rows, int ring_row0, int capacity, int write_index, dim3 grid,
                                         cudaStream_t stream) {
#define RFSN_ROPE_TAB_LAUNCH(TT)                                                                                  \
    RFSN_CUDA(launch_pdl(ring::rope_tables_append_kernel<TIn, TT>, grid, dim3(256), 0, stream,                    \
                         static_cast<const TIn*>(q), static_cast<const TIn*>(k), static_cast<const TIn*>(v),       \
                         static_cast<const TT*>(cos_t), static_cast<const TT*>(sin_t), inv_freq, pos0, batch,     \
                         q_heads, kv_heads, len, head_dim, q_out, static_cast<TIn*>(ak), static_cast<TIn*>(av),  \
                         rows, ring_row0, capacity, write_index))
    if (tab_dtype == RFSN_F32) {
        RFSN_ROPE_TAB_LAUNCH(float);
    } else if (tab_dtype == RFSN_F16) {
        RFSN_ROPE_TAB_LAUNCH(__half);
    } else {
        RFSN_ROPE_TAB_LAUNCH(__nv_bfloat16);
    }
#undef RFSN_ROPE_TAB_LAUNCH
    return RFSN_OK;
}

rfsn_status rope_tables_append_launch(int dtype, int tab_dtype, const void* q, const void* k, const void* v,
                                      const void* cos_t, const void* sin_t, const float* inv_freq, int pos0,
                                      int batch, int q_heads, int kv_heads, int len, int head_dim, float* q_out,
                                      void* ak, void* av, int rows, int ring_row0, int capacity, int write_index,
                                      cudaStream_t stream) {
    const long total = ((long)batch * (q_heads + kv_heads) * len) * (head_dim / 2);
    long blocks = (total + 255) / 256;
    if (blocks > 65535L * 8) blocks = 65535L * 8;
    if (blocks < 1) blocks = 1;
    const dim3 grid((unsigned)blocks);
    rfsn_status st;
    if (dtype == RFSN_F32) {
        st = rope_tables_launch_in<float>(tab_dtype, q, k, v, cos_t, sin_t, inv_freq, pos0, batch, q_heads, kv_heads,
                                          len, head_dim, q_out, ak, av, rows, ring_row0, capacity, write_index, grid,
                                          stream);
    } else if (dtype == RFSN_F16) {
        st = rope_tables_launch_in<__half>(tab_dtype, q, k, v, cos_t, sin_t, inv_freq, pos0, batch, q_heads, kv_heads,
                                           len, head_dim, q_out, ak, av, rows, ring_row0, capacity, write_index, grid,
                                           stream);
    } else {
        st = rope_tables_launch_in<__nv_bfloat16>(tab_dtype, q, k, v, cos_t, sin_t, inv_freq, pos0, batch, q_heads,
                                                  kv_heads, len, head_dim, q_out, ak, av, rows, ring_row0, capacity,
                                                  write_index, grid, stream);
    }
    if (st != RFSN_OK) return st;
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

void preload_ring_kernels() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, ring::rope_append_kernel<float, float>);
    cudaFuncGetAttributes(&a, ring::rope_append_kernel<__half, __half>);
    cudaFuncGetAttributes(&a, ring::rope_append_kernel<__nv_bfloat16, __nv_bfloat16>);
    cudaFuncGetAttributes(&a, ring::copy_rows_kernel);
    cudaFuncGetAttributes(&a, ring::rope_tables_append_kernel<__nv_bfloat16, __nv_bfloat16>);
    cudaFuncGetAttributes(&a, ring::rope_tables_append_kernel<__nv_bfloat16, float>);
    cudaFuncGetAttributes(&a, ring::rope_tables_append_kernel<__half, __half>);
    cudaFuncGetAttributes(&a, ring::rope_tables_append_kernel<__half, float>);
    cudaFuncGetAttributes(&a, ring::rope_tables_append_kernel<float, float>);
}

rfsn_status copy_rows_launch(void* ak, void* av, int groups, int rows, int row_bytes, int src_row0, int src_offset,
                             int src_wrap, int dst_row0, int count, cudaStream_t stream) {
    const long total = (long)groups * count * (row_bytes / 16);
    long blocks = (total + 255) / 256;
    if (blocks > 65535L * 4) blocks = 65535L * 4;
    if (blocks < 1) blocks = 1;
    ring::copy_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<uint8_t*>(ak), static_cast<uint8_t*>(av),
                                                                  groups, rows, row_bytes, src_row0, src_offset,
                                                                  src_wrap, dst_row0, count);
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

}  // namespace rfsn
