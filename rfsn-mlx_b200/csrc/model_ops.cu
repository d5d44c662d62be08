// Fused dense-layer helpers of the model driver (the reference's layer.py
// RMSNorm and SwiGLU): one kernel each instead of a chain of elementwise ops.
#include "params.cuh"

namespace rfsn {
namespace model_ops {

constexpr int kThreads = 256;

// layer.py:54-64: y = weight * x / sqrt(mean(x^2) + eps) in float32, rounded
// to the storage type once. One CTA per row.
template <typename T>
__global__ void __launch_bounds__(kThreads) rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                            T* __restrict__ y, int n, float eps) {
    griddep_wait();               // x may come from the kernel this launch overlaps
    griddep_launch_dependents();  // the next kernel waits for this one's completion before reading
    const T* xr = x + (size_t)blockIdx.x * n;
    T* yr = y + (size_t)blockIdx.x * n;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const float v = to_f32<T>(xr[i]);
        s += v * v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    __shared__ float part[kThreads / 32];
    __shared__ float rms;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < kThreads / 32; ++i) t += part[i];
        rms = sqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float r = rms;
    for (int i = threadIdx.x; i < n; i += kThreads) {
        yr[i] = from_f32<T>(to_f32<T>(w[i]) * (to_f32<T>(xr[i]) / r));
    }
}

// The same with the row held in registers as 16-byte vectors (all of a
// thread's loads in flight at once; rows of up to kThreads * PER vectors) and
// an optional residual added first: s = x + r rounded to T (stored to s_out,
// the layer's new residual stream), y = weight * s / rms(s).
template <typename T, int PER>
__global__ void __launch_bounds__(kThreads) rms_norm_vec_kernel(const T* __restrict__ x, const T* __restrict__ res,
                                                                const T* __restrict__ w, T* __restrict__ s_out,
                                                                T* __restrict__ y, int n, float eps) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int VEC = 16 / sizeof(T);
    const int nvec = n / VEC;
    const size_t row = (size_t)blockIdx.x * n;
    uint4 xv[PER];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int vi = threadIdx.x + k * kThreads;
        if (vi < nvec) {
            xv[k] = *reinterpret_cast<const uint4*>(x + row + (size_t)vi * VEC);
            if (res != nullptr) {
                const uint4 rv = *reinterpret_cast<const uint4*>(res + row + (size_t)vi * VEC);
                T* a = reinterpret_cast<T*>(&xv[k]);
                const T* b = reinterpret_cast<const T*>(&rv);
#pragma unroll
                for (int e = 0; e < VEC; ++e) a[e] = from_f32<T>(to_f32<T>(a[e]) + to_f32<T>(b[e]));
                *reinterpret_cast<uint4*>(s_out + row + (size_t)vi * VEC) = xv[k];
            }
            const T* a = reinterpret_cast<const T*>(&xv[k]);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                const float v = to_f32<T>(a[e]);
                s += v * v;
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    __shared__ float part[kThreads / 32];
    __shared__ float rms;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < kThreads / 32; ++i) t += part[i];
        rms = sqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float r = rms;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int vi = threadIdx.x + k * kThreads;
        if (vi < nvec) {
            const uint4 wv = *reinterpret_cast<const uint4*>(w + (size_t)vi * VEC);
            const T* a = reinterpret_cast<const T*>(&xv[k]);
            const T* b = reinterpret_cast<const T*>(&wv);
            uint4 ov;
            T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
            for (int e = 0; e < VEC; ++e) o[e] = from_f32<T>(to_f32<T>(b[e]) * (to_f32<T>(a[e]) / r));
            *reinterpret_cast<uint4*>(y + row + (size_t)vi * VEC) = ov;
        }
    }
}

// layer.py:94-95 SwiGLU on a fused gate|up projection row [2n]: y = silu(g) * u,
// silu rounded to the storage type first (as an elementwise op would), the
// product in float32 rounded once.
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ y, long long rows, int n) {
    griddep_wait();
    griddep_launch_dependents();
    const long long total = rows * n;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long r = idx / n;
        const int c = (int)(idx - r * n);
        const float g = to_f32<T>(gu[r * 2 * n + c]);
        const float u = to_f32<T>(gu[r * 2 * n + n + c]);
        const float s = to_f32<T>(from_f32<T>(g / (1.f + expf(-g))));
        y[idx] = from_f32<T>(s * u);
    }
}

// y[r, n] = sum_k W[n, k] * x[r, k] for a few rows r of x (decode: one token):
// W [N, K] row-major in the storage type, read once with 16-byte loads, x
// staged in shared memory (float32), float32 accumulation, y rounded once.
// Each warp owns ROWS consecutive output columns n at a time (their loads in
// flight together); lanes stride K in 16-byte vectors.
constexpr int GV_THREADS = 256;
constexpr int GV_MAX_X = 4;  // rows of x handled per launch

template <typename T, int XR, int ROWS>
__global__ void __launch_bounds__(GV_THREADS, XR == 1 ? 2 : 1) gemv_kernel(const T* __restrict__ w,
                                                                           const T* __restrict__ x,
                                                                           T* __restrict__ y, int N, int K, int xrows) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ float4 xs4[];  // [xrows][K / 4]
    float* xs = reinterpret_cast<float*>(xs4);
    for (int i = threadIdx.x; i < xrows * K; i += GV_THREADS) xs[i] = to_f32<T>(x[i]);
    __syncthreads();
    constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte load
    constexpr int U = (16 + ROWS - 1) / ROWS;  // K steps whose loads are issued together (~16 per lane)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nvec = K / VEC;
    const int warps_total = gridDim.x * (GV_THREADS / 32);
    for (int n0 = (blockIdx.x * (GV_THREADS / 32) + warp) * ROWS; n0 < N; n0 += warps_total * ROWS) {
        float acc[ROWS][XR];
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
            for (int j = 0; j < XR; ++j) acc[r][j] = 0.f;
        for (int v0 = lane; v0 < nvec; v0 += 32 * U) {
            uint4 wv[U][ROWS];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int v = v0 + 32 * u;
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    wv[u][r] = (v < nvec && n0 + r < N)
                                   ? __ldcs(reinterpret_cast<const uint4*>(w + (size_t)(n0 + r) * K) + v)
                                   : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int v = v0 + 32 * u;
                if (v >= nvec) break;
#pragma unroll
                for (int j = 0; j < XR; ++j) {
                    if (j >= xrows) break;
                    float xv[VEC];
#pragma unroll
                    for (int q4 = 0; q4 < VEC / 4; ++q4) {
                        const float4 t = xs4[(j * K + v * VEC) / 4 + q4];
                        xv[4 * q4] = t.x;
                        xv[4 * q4 + 1] = t.y;
                        xv[4 * q4 + 2] = t.z;
                        xv[4 * q4 + 3] = t.w;
                    }
#pragma unroll
                    for (int r = 0; r < ROWS; ++r) {
                        const T* e = reinterpret_cast<const T*>(&wv[u][r]);
#pragma unroll
                        for (int q = 0; q < VEC; ++q) acc[r][j] += to_f32<T>(e[q]) * xv[q];
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
            for (int j = 0; j < XR; ++j) {
                float a = acc[r][j];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
                if (lane == 0 && j < xrows && n0 + r < N) y[(size_t)j * N + n0 + r] = from_f32<T>(a);
            }
    }
}

// The same, 16-byte vectors per thread (n a multiple of the vector width,
// 16-byte aligned rows, fewer than 2^31 vectors).
template <typename T>
__global__ void silu_mul_vec_kernel(const T* __restrict__ gu, T* __restrict__ y, int total_vec, int nvec) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int VEC = 16 / sizeof(T);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total_vec; i += gridDim.x * blockDim.x) {
        const int r = i / nvec, c = i - r * nvec;
        const uint4 gv = reinterpret_cast<const uint4*>(gu)[(size_t)r * 2 * nvec + c];
        const uint4 uv = reinterpret_cast<const uint4*>(gu)[(size_t)r * 2 * nvec + nvec + c];
        const T* g = reinterpret_cast<const T*>(&gv);
        const T* u = reinterpret_cast<const T*>(&uv);
        uint4 ov;
        T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
            const float gf = to_f32<T>(g[e]);
            const float s = to_f32<T>(from_f32<T>(gf / (1.f + expf(-gf))));
            o[e] = from_f32<T>(s * to_f32<T>(u[e]));
        }
        reinterpret_cast<uint4*>(y)[i] = ov;
    }
}

constexpr int kVecPer = 4;  // vectors per thread held in registers: rows up to 8192 bf16 / 4096 fp32 elements

template <typename T>
rfsn_status rms_norm_launch(const void* x, const void* res, const void* w, void* s_out, void* y, int rows, int n,
                            float eps, cudaStream_t s) {
    constexpr int VEC = 16 / sizeof(T);
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(res) |
                           reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(s_out) |
                           reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (aligned && n % VEC == 0 && n / VEC <= kThreads * kVecPer) {
        RFSN_CUDA(launch_pdl(rms_norm_vec_kernel<T, kVecPer>, dim3(rows), dim3(kThreads), 0, s,
                             static_cast<const T*>(x), static_cast<const T*>(res), static_cast<const T*>(w),
                             static_cast<T*>(s_out), static_cast<T*>(y), n, eps));
    } else {
        if (res != nullptr) {
            set_error("rfsn_rms_norm: a residual needs 16-byte aligned rows of at most %d vectors", kThreads * kVecPer);
            return RFSN_ERR_UNSUPPORTED;
        }
        RFSN_CUDA(launch_pdl(rms_norm_kernel<T>, dim3(rows), dim3(kThreads), 0, s, static_cast<const T*>(x),
                             static_cast<const T*>(w), static_cast<T*>(y), n, eps));
    }
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

template <typename T, int XR, int ROWS>
rfsn_status gemv_launch_rows(const void* w, const void* x, void* y, int N, int K, int xrows, int blocks,
                             cudaStream_t s) {
    const size_t smem = sizeof(float) * (size_t)xrows * K;
    auto kern = gemv_kernel<T, XR, ROWS>;
    RFSN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    RFSN_CUDA(launch_pdl(kern, dim3(blocks), dim3(GV_THREADS), smem, s, static_cast<const T*>(w),
                         static_cast<const T*>(x), static_cast<T*>(y), N, K, xrows));
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

// Rows per warp: the count (2, 3 or 4) that fills the most of two CTAs per SM
// in one pass (4 with a loop when N is larger).
template <typename T, int XR>
rfsn_status gemv_launch_xr(const void* w, const void* x, void* y, int N, int K, int xrows, cudaStream_t s) {
    const int slots = 148 * (XR == 1 ? 2 : 1), warps_per_cta = GV_THREADS / 32;  // resident CTAs
    int best_rows = 4, best_ctas = 0;
    for (int rows = 4; rows >= 2; --rows) {
        const int ctas = (N + rows * warps_per_cta - 1) / (rows * warps_per_cta);
        if (ctas <= slots && ctas > best_ctas) {
            best_ctas = ctas;
            best_rows = rows;
        }
    }
    if (best_ctas == 0) best_ctas = slots;  // more rows than one pass: warps loop
    if (best_rows == 2) return gemv_launch_rows<T, XR, 2>(w, x, y, N, K, xrows, best_ctas, s);
    if (best_rows == 3) return gemv_launch_rows<T, XR, 3>(w, x, y, N, K, xrows, best_ctas, s);
    return gemv_launch_rows<T, XR, 4>(w, x, y, N, K, xrows, best_ctas, s);
}

template <typename T>
rfsn_status gemv_launch(const void* w, const void* x, void* y, int N, int K, int xrows, cudaStream_t s) {
    return xrows == 1 ? gemv_launch_xr<T, 1>(w, x, y, N, K, xrows, s)
                      : gemv_launch_xr<T, GV_MAX_X>(w, x, y, N, K, xrows, s);
}

template <typename T>
rfsn_status silu_mul_launch(const void* gu, void* y, int rows, int n, cudaStream_t s) {
    constexpr int VEC = 16 / sizeof(T);
    const long long total_vec = (long long)rows * (n / VEC);
    if (n % VEC == 0 && ((reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(y)) & 15) == 0 &&
        total_vec < (1LL << 31)) {
        long long blocks = (total_vec + kThreads - 1) / kThreads;
        if (blocks > 148LL * 8) blocks = 148LL * 8;
        RFSN_CUDA(launch_pdl(silu_mul_vec_kernel<T>, dim3((unsigned)blocks), dim3(kThreads), 0, s,
                             static_cast<const T*>(gu), static_cast<T*>(y), (int)total_vec, n / VEC));
        note_launch();
        return RFSN_OK;
    }
    const long long total = (long long)rows * n;
    long long blocks = (total + kThreads - 1) / kThreads;
    if (blocks > 148LL * 16) blocks = 148LL * 16;
    RFSN_CUDA(launch_pdl(silu_mul_kernel<T>, dim3((unsigned)blocks), dim3(kThreads), 0, s,
                         static_cast<const T*>(gu), static_cast<T*>(y), (long long)rows, n));
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

}  // namespace model_ops

template <typename T>
void preload_gemv() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, model_ops::gemv_kernel<T, 1, 2>);
    cudaFuncGetAttributes(&a, model_ops::gemv_kernel<T, 1, 3>);
    cudaFuncGetAttributes(&a, model_ops::gemv_kernel<T, 1, 4>);
    cudaFuncGetAttributes(&a, model_ops::gemv_kernel<T, model_ops::GV_MAX_X, 2>);
    cudaFuncGetAttributes(&a, model_ops::gemv_kernel<T, model_ops::GV_MAX_X, 3>);
    cudaFuncGetAttributes(&a, model_ops::gemv_kernel<T, model_ops::GV_MAX_X, 4>);
}

void preload_model_kernels() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, model_ops::rms_norm_kernel<float>);
    cudaFuncGetAttributes(&a, model_ops::rms_norm_kernel<__half>);
    cudaFuncGetAttributes(&a, model_ops::rms_norm_kernel<__nv_bfloat16>);
    cudaFuncGetAttributes(&a, model_ops::rms_norm_vec_kernel<float, model_ops::kVecPer>);
    cudaFuncGetAttributes(&a, model_ops::rms_norm_vec_kernel<__half, model_ops::kVecPer>);
    cudaFuncGetAttributes(&a, model_ops::rms_norm_vec_kernel<__nv_bfloat16, model_ops::kVecPer>);
    preload_gemv<float>();
    preload_gemv<__half>();
    preload_gemv<__nv_bfloat16>();
    cudaFuncGetAttributes(&a, model_ops::silu_mul_vec_kernel<float>);
    cudaFuncGetAttributes(&a, model_ops::silu_mul_vec_kernel<__half>);
    cudaFuncGetAttributes(&a, model_ops::silu_mul_vec_kernel<__nv_bfloat16>);
    cudaFuncGetAttributes(&a, model_ops::silu_mul_kernel<float>);
    cudaFuncGetAttributes(&a, model_ops::silu_mul_kernel<__half>);
    cudaFuncGetAttributes(&a, model_ops::silu_mul_kernel<__nv_bfloat16>);
}

rfsn_status rms_norm_dispatch(int dtype, const void* x, const void* res, const void* w, void* s_out, void* y, int rows,
                              int n, float eps, cudaStream_t s) {
    if (dtype == RFSN_F32) return model_ops::rms_norm_launch<float>(x, res, w, s_out, y, rows, n, eps, s);
    if (dtype == RFSN_F16) return model_ops::rms_norm_launch<__half>(x, res, w, s_out, y, rows, n, eps, s);
    return model_ops::rms_norm_launch<__nv_bfloat16>(x, res, w, s_out, y, rows, n, eps, s);
}

rfsn_status silu_mul_dispatch(int dtype, const void* gu, void* y, int rows, int n, cudaStream_t s) {
    if (dtype == RFSN_F32) return model_ops::silu_mul_launch<float>(gu, y, rows, n, s);
    if (dtype == RFSN_F16) return model_ops::silu_mul_launch<__half>(gu, y, rows, n, s);
    return model_ops::silu_mul_launch<__nv_bfloat16>(gu, y, rows, n, s);
}

rfsn_status gemv_dispatch(int dtype, const void* w, const void* x, void* y, int N, int K, int xrows, cudaStream_t s) {
    if (dtype == RFSN_F32) return model_ops::gemv_launch<float>(w, x, y, N, K, xrows, s);
    if (dtype == RFSN_F16) return model_ops::gemv_launch<__half>(w, x, y, N, K, xrows, s);
    return model_ops::gemv_launch<__nv_bfloat16>(w, x, y, N, K, xrows, s);
}

int gemv_max_rows() { return model_ops::GV_MAX_X; }

}  // namespace rfsn
