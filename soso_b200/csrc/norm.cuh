// norm.cuh -- RMSNorm rows, optionally fused with the residual add.
//
// Follows gemm::rmsnorm (crates/soso-llm-core/src/gemm.rs:93-100):
//   scale = 1 / sqrtf(sum(x^2) / n + eps);  x[i] = x[i] * scale * w[i]
// and the residual adds add_f32 / add_assign_f32 (gemm.rs:265-290).  The sum
// of squares is a tree reduction instead of the reference's left fold, so
// results agree to rounding (tolerance in the tests).
#pragma once
#include "common.cuh"

namespace sb {

constexpr int NORM_THREADS = 256;

__device__ __forceinline__ float block_sum(float v, float *red)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    return t;
}

// One CTA per row.  If res != nullptr: h = x + res is written to h_out (the new
// residual stream) and normalised into y; else y = rmsnorm(x).  h_out may alias
// res (each element is read, then written, by the same thread).
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_rows_kernel(const float *x,
                                                                    const float *res,
                                                                    float *h_out,
                                                                    const float *__restrict__ w,
                                                                    float *y, int n, float eps)
{
    __shared__ float red[32];
    griddep_wait();
    const long long base = (long long)blockIdx.x * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[base + i];
        if (res) {
            v += res[base + i];
            h_out[base + i] = v;
        }
        ss += v * v;
    }
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = res ? h_out[base + i] : x[base + i];
        y[base + i] = v * scale * w[i];
    }
    griddep_launch();
}

}  // namespace sb

extern "C" int sbk_rmsnorm(const float *x, const float *res, float *h_out, const float *w, float *y, size_t rows,
                           size_t n, float eps, void *stream)
{
    if (!x || !w || !y || !rows || !n || n > (1u << 24) || rows > (1u << 30)) return -1;
    if (res && !h_out) return -1;
    sb::rmsnorm_rows_kernel<<<(unsigned)rows, sb::NORM_THREADS, 0, (cudaStream_t)stream>>>(x, res, h_out, w, y,
                                                                                          (int)n, eps);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
