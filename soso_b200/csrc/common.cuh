// common.cuh -- shared device helpers for the sm_100a decode kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sb {

// ---- error word ---------------------------------------------------------
// Kernels never trap.  A bounded wait that gives up, or a guard that finds an
// impossible index, records a code here and skips the access; the host reads
// and clears it with sbk_take_device_error().
// (The library is one translation unit, sosob200.cu, so this is its only definition.)
__device__ unsigned int g_dev_error = 0;

__device__ __forceinline__ void set_dev_error(unsigned int code) { atomicCAS(&g_dev_error, 0u, code); }

// ---- work split ---------------------------------------------------------
// Balanced [start, end) of worker i of n -- the reference's row_strip
// (crates/soso-llm-core/src/parallel.rs:22-31), used for rows over CTAs and for
// blocks over 8-lane workers.
// 32-bit: every count the kernels split (rows, blocks) is below 2^31, and
// 64-bit division is a long emulated sequence on the GPU.
__host__ __device__ __forceinline__ void row_strip(int rows, int i, int n, int &s, int &e)
{
    const int base = rows / n, rem = rows - base * n;
    s = i * base + (i < rem ? i : rem);
    e = s + base + (i < rem ? 1 : 0);
}

// ---- programmatic dependent launch ------------------------------------
// wait: block until the previous grid on the stream has completed and its
// writes are visible.  launch: allow the next grid to begin its prologue.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- memory ---------------------------------------------------------------
// Bulk L2 prefetch of [p, p+bytes): p 16-B aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch the byte range [lo, hi) of a tensor of `total` bytes into L2,
// rounded inward to 16-B boundaries; pieces of <= 64 KiB spread over the
// first warp's lanes.
__device__ __forceinline__ void prefetch_range_l2(const uint8_t *base, long long lo, long long hi)
{
    long long a = (lo + 15) & ~15LL, b = hi & ~15LL;
    if (b <= a) return;
    const long long piece = 65536;
    long long n = (b - a + piece - 1) / piece;
    for (long long k = threadIdx.x; k < n; k += 32) {
        long long s = a + k * piece, e = s + piece < b ? s + piece : b;
        prefetch_l2_bulk(base + s, (uint32_t)(e - s));
    }
}

__device__ __forceinline__ uint4 ldg_stream_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ldg_u32(const void *p)
{
    uint32_t r;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ unsigned short ldg_u16(const void *p)
{
    unsigned short r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

// 32-bit little-endian word at a 2-byte aligned address, from the two aligned
// words that cover it.
__device__ __forceinline__ uint32_t ldg_u32_a2(const uint8_t *p)
{
    uintptr_t a = (uintptr_t)p;
    const uint32_t *q = (const uint32_t *)(a & ~(uintptr_t)3);
    const uint32_t lo = ldg_u32(q), hi = (a & 3) ? ldg_u32(q + 1) : 0u;  // never reads past p+3
    return __funnelshift_r(lo, hi, (uint32_t)(a & 3) * 8u);
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// A code isolated in place inside a 32-bit register (no shift), read as an
// IEEE-754 bit pattern: a subnormal of value code * 2^(pos) * 2^-149.  Kernels
// multiply it by x pre-scaled by 2^(89 - pos), so every product equals
// code * x * 2^-60 exactly and no int->float conversion is issued.
__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }

constexpr float TWO_P60 = 1152921504606846976.0f;  // 2^60

// Sum over the warp (a butterfly: every lane ends with the same sum).
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over the 8-lane group that contains this lane.  The mask names only the
// group, so groups of one warp may call it at different times.
__device__ __forceinline__ float warp8_sum(float v)
{
    const unsigned m = 0xffu << (threadIdx.x & 24);
    v += __shfl_xor_sync(m, v, 1);
    v += __shfl_xor_sync(m, v, 2);
    v += __shfl_xor_sync(m, v, 4);
    return v;
}

}  // namespace sb
