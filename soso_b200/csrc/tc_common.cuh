// tc_common.cuh -- building blocks of the tensor-core matvec kernels (tc_mmv.cuh):
// mbarrier ring primitives, the 2-D TMA tensor load (into this CTA only) and
// the warp-level MMA forms the quantized formats use.
#pragma once
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace sb {
namespace tcmv {

constexpr unsigned SPIN_LIMIT = 1u << 26;

// workspace (global): per CTA two boundary partials (16 floats each), then one counter per group
struct Ws {
    float *part;    // [grid][2][16]
    unsigned *cnt;  // [groups]
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx_arrive(uint64_t *b, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// Bounded wait for the phase with the given parity; false if the limit ran out.
// (The suspend-time hint lets a waiting warp yield its issue slots.)
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity, unsigned limit = SPIN_LIMIT)
{
    const uint32_t a = smem_u32(b);
    for (unsigned i = 0; i < limit; i++) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(1000u)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// L2 policy for streamed weights: each byte is read once per token, so let it be
// the first to go and keep activations, KV rows and code resident in L2.
__device__ __forceinline__ uint64_t l2_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 2-D tiled TMA load into this CTA: box at element coords (x = u64 column, y = row).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
        "[%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// u8 x s8 -> s32 tensor-core MMA, m16n8k32 (integer: exact).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// s8 x s8 -> s32 tensor-core MMA, m16n8k32 (integer: exact).
__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 pieces of each of four values (|v| < 128): v = p0 + p1/2^7 + p2/2^14 + p3/2^21
// to 28 bits.  v * 2^21 is rounded to an integer i (|i| < 2^28, exact scaling); p0 = i >> 21
// (-128..127) and p1, p2, p3 are the next 7-bit fields of i (0..127), so
// i = p0*2^21 + p1*2^14 + p2*2^7 + p3 exactly.  Byte k of pk[p] gets piece p of value k.
__device__ __forceinline__ void int8_pieces4(float4 v, uint32_t (&pk)[4])
{
    const int i[4] = {__float2int_rn(v.x * 2097152.0f), __float2int_rn(v.y * 2097152.0f),
                      __float2int_rn(v.z * 2097152.0f), __float2int_rn(v.w * 2097152.0f)};
    uint32_t p0 = 0u, p1 = 0u, p2 = 0u, p3 = 0u;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        p0 |= (uint32_t)((i[k] >> 21) & 255) << (8 * k);
        p1 |= (uint32_t)((i[k] >> 14) & 127) << (8 * k);
        p2 |= (uint32_t)((i[k] >> 7) & 127) << (8 * k);
        p3 |= (uint32_t)(i[k] & 127) << (8 * k);
    }
    pk[0] = p0, pk[1] = p1, pk[2] = p2, pk[3] = p3;
}

// 2^e with 2^e > max |v| over the warp (from the max's biased exponent), clamped for
// zero and non-finite input.
__device__ __forceinline__ int warp_exp_above(float mx)
{
    // mx >= 0 (an absolute value): its bits order like the values, so one integer
    // reduction over the warp gives the maximum
    const uint32_t mxb = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
    const int ex = (int)(mxb >> 23) - 126;
    return (mxb == 0u || mxb >= 0x7f800000u) ? 0 : ex < -100 ? -100 : ex > 100 ? 100 : ex;
}

// PTX prmt in its generic mode: a selector nibble with bit 3 set replicates the
// sign bit of the selected byte (used to sign-extend one int8 into 32 bits).
__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// How the input vector of the matvecs of one launch is formed while it is prepared,
// so that the step producing it needs no launch of its own.  With a = the matrix's x:
//   XS_PLAIN   x = a
//   XS_NORM    h = a (+ b when b is set: the residual add, gemm.rs:265-290),
//              x = h * (1 / sqrtf(sum(h^2) / n + eps)) * w   (gemm::rmsnorm, gemm.rs:93-100);
//              CTA 0 also stores h to h_out when set (the new residual stream; h_out
//              must not alias a or b, which other CTAs are still reading)
//   XS_SWIGLU  x = silu(a) * b, silu(v) = v / (1 + expf(-v))  (gemm.rs:210-226; a = gate, b = up)
enum { XS_PLAIN = 0, XS_NORM = 1, XS_SWIGLU = 2 };

struct XSrc {
    const float *b;
    const float *w;
    float *h_out;
    float eps;
    int mode;
    // XS_NORM with a weighted set of residual vectors (a MoE layer's expert outputs):
    // h = (sum_k yw[k] * ys[k * ystride + e], k = 0..ny-1 in order) + a   (layer.rs:1922-1933,
    // then add_assign_f32 :1389); used instead of b when ny > 0
    const float *ys;
    const float *yw;
    int ny, ystride;
};

constexpr int XS_MAXY = 16;

// Element loader of the preparation: float4 i of the (transformed) input vector.
struct XLoad {
    const float4 *a, *b, *w;
    const float4 *ys;
    float scale;
    int mode, ny, ys4;
    float yw[XS_MAXY];

    __device__ __forceinline__ float4 h(int i) const
    {
        float4 v = a[i];
        if (ny) {
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int k = 0; k < ny; k++) {
                const float4 y = __ldcg(ys + k * ys4 + i);  // may be written by peers: read at L2
                acc.x += y.x * yw[k], acc.y += y.y * yw[k], acc.z += y.z * yw[k], acc.w += y.w * yw[k];
            }
            v.x = acc.x + v.x, v.y = acc.y + v.y, v.z = acc.z + v.z, v.w = acc.w + v.w;
        } else if (b) {
            const float4 r = b[i];
            v.x += r.x, v.y += r.y, v.z += r.z, v.w += r.w;
        }
        return v;
    }
    __device__ __forceinline__ float4 operator()(int i) const
    {
        if (mode == XS_NORM) {
            float4 v = h(i);
            const float4 g = w[i];
            v.x = v.x * scale * g.x, v.y = v.y * scale * g.y, v.z = v.z * scale * g.z, v.w = v.w * scale * g.w;
            return v;
        }
        float4 v = a[i];
        if (mode == XS_SWIGLU) {
            const float4 u = b[i];
            v.x = v.x / (1.0f + expf(-v.x)) * u.x;
            v.y = v.y / (1.0f + expf(-v.y)) * u.y;
            v.z = v.z / (1.0f + expf(-v.z)) * u.z;
            v.w = v.w / (1.0f + expf(-v.w)) * u.w;
        }
        return v;
    }
};

}  // namespace tcmv
}  // namespace sb
